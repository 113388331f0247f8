"""CUDA path vs the reference, through the C ABI of libsmol_b200.so (needs a B200).

Oracles: tests/golden/reference_cases.npz (outputs of the compiled reference) and
the restatement in oracle/ on fresh seeded inputs.  Attention inputs are rounded to
bf16 first and the oracle is fed their fp32 upcast; the bar is rel-L2 <= 1e-3 and
max-abs <= 1e-2 (conftest.REL_L2_TOL / MAX_ABS_TOL).  Cache slot addressing and
RoPE position indexing are checked bit for bit.
"""
import numpy as np
import pytest
import torch

import pyoracle
import smol_b200
from conftest import assert_close

pytestmark = pytest.mark.gpu


def qkv(g, name):
    return [pyoracle.bf16_to_f32(g[f"{name}/{t}_bf16"]) for t in ("q", "k", "v")]


def case_names(g, prefixes):
    return sorted({k.split("/")[0] for k in g.files if k.split("/")[0].startswith(prefixes)})


def no_error():
    assert smol_b200.last_error() == 0, smol_b200.lib().smol_cuda_error_string(smol_b200.last_error())
    assert smol_b200.device_error() == 0


def rnd_bf16(rng, *shape):
    return pyoracle.round_bf16(rng.standard_normal(shape).astype(np.float32))


def dev_bf16(a, cuda):
    return torch.from_numpy(np.ascontiguousarray(a, np.float32)).to(cuda).to(torch.bfloat16)


def dev_f16(a, cuda):
    return torch.from_numpy(np.ascontiguousarray(a, np.float32)).to(cuda).to(torch.float16)


@pytest.fixture(autouse=True)
def _clean():
    smol_b200.clear_error()
    yield


# ---------------------------------------------------------------------------
# Drop-in entry points on the reference's golden cases
# ---------------------------------------------------------------------------
@pytest.mark.parametrize("device_buffers", [False, True])
def test_dropin_causal_family_golden(golden, cuda, device_buffers):
    names = case_names(golden, ("causal", "sliding"))
    for name in names:
        sq, sk, hq, hkv, hd, qo, win = (int(x) for x in golden[f"{name}/meta"])
        scale, cap = (float(x) for x in golden[f"{name}/fmeta"])
        q, k, v = qkv(golden, name)
        if device_buffers:
            tq, tk, tv = (torch.from_numpy(a).to(cuda) for a in (q, k, v))
            tout = torch.full((sq, hq * hd), 7.0, device=cuda)
            smol_b200.causal_attention(tout, tq, tk, tv, sq, sk, hq, hkv, hd, scale, qo, window=win, cap=cap)
            out = tout.cpu().numpy()
        else:
            out = np.full((sq, hq * hd), 7.0, np.float32)
            smol_b200.causal_attention(out, q, k, v, sq, sk, hq, hkv, hd, scale, qo, window=win, cap=cap)
        no_error()
        assert_close(out, golden[f"{name}/out"], name)


def test_dropin_empty_rows_are_zero(golden, cuda):
    q, k, v = qkv(golden, "causal_empty_rows")
    out = np.full((6, 2 * 64), 7.0, np.float32)
    smol_b200.causal_attention(out, q, k, v, 6, 4, 2, 1, 64, 0.125, -3)
    no_error()
    assert np.all(out[:3] == 0.0)


def test_dropin_bidirectional_golden(golden, cuda):
    for name in case_names(golden, ("bidir",)):
        seq, h, hd = (int(x) for x in golden[f"{name}/meta"])
        q, k, v = qkv(golden, name)
        out = np.zeros((seq, h * hd), np.float32)
        smol_b200.bidirectional_attention(out, q, k, v, seq, h, hd, float(golden[f"{name}/fmeta"][0]),
                                          golden[f"{name}/ws"])
        no_error()
        assert_close(out, golden[f"{name}/out"], name)


def test_dropin_bidirectional_leaves_uncovered_rows(cuda):
    # attention.c:38-43 only writes rows inside a window
    rng = np.random.default_rng(5)
    seq, h, hd = 70, 2, 64
    q, k, v = (rnd_bf16(rng, seq, h * hd) for _ in range(3))
    ws = [5, 30, 60]
    out = np.full((seq, h * hd), 3.0, np.float32)
    smol_b200.bidirectional_attention(out, q, k, v, seq, h, hd, 0.125, ws)
    no_error()
    want = pyoracle.oracle().bidirectional_attention(q, k, v, seq, h, hd, 0.125, ws,
                                                     out=np.full((seq, h * hd), 3.0, np.float32))
    assert np.all(out[:5] == 3.0) and np.all(out[60:] == 3.0)
    assert_close(out[5:60], want[5:60], "windows")


@pytest.mark.new_on_gpu
def test_dropin_bidirectional_audio_encoder_windows(cuda):
    # Qwen3-ASR audio encoder shape (encoder.c:426-465): 104-token windows, 16 heads,
    # hd 64, a ragged last window; every 128-row query tile spans two or three windows
    rng = np.random.default_rng(6)
    h, hd = 16, 64
    ws = list(range(0, 9 * 104 + 1, 104)) + [9 * 104 + 50]
    seq = ws[-1]
    q, k, v = (rnd_bf16(rng, seq, h * hd) for _ in range(3))
    out = np.zeros((seq, h * hd), np.float32)
    smol_b200.bidirectional_attention(out, q, k, v, seq, h, hd, 0.125, ws)
    no_error()
    want = pyoracle.oracle().bidirectional_attention(q, k, v, seq, h, hd, 0.125, ws)
    assert_close(out, want, "audio encoder windows")


@pytest.mark.new_on_gpu
def test_dropin_bidirectional_nomic_batch(cuda):
    # nomic's embedder (exports/nomic/nomic.c:176-182, :438-447): a batch of sequences of
    # different lengths packed end to end, each sequence one window, 12 heads of hd 64,
    # RoPE positions restarting at 0 in every sequence -- windows from 1 token to several
    # 128-row query tiles, starting anywhere inside a tile
    rng = np.random.default_rng(7)
    h, hd = 12, 64
    lens = [1, 37, 128, 300, 5, 129, 64]
    ws = [0] + np.cumsum(lens).tolist()
    seq = ws[-1]
    pos = np.concatenate([np.arange(n) for n in lens]).astype(np.int32)
    cos, sin = (np.zeros((seq, hd), np.float32) for _ in range(2))
    smol_b200.compute_rope(cos, sin, pos, seq, hd, 1000.0)
    q, k, v = (rnd_bf16(rng, seq, h * hd) for _ in range(3))
    for x in (q, k):
        smol_b200.apply_rope(x, cos, sin, seq, h, hd)
    q, k = pyoracle.round_bf16(q), pyoracle.round_bf16(k)   # the parity protocol's bf16-exact inputs
    out = np.zeros((seq, h * hd), np.float32)
    smol_b200.bidirectional_attention(out, q, k, v, seq, h, hd, 0.125, ws)
    no_error()
    want = pyoracle.oracle().bidirectional_attention(q, k, v, seq, h, hd, 0.125, ws)
    assert_close(out, want, "nomic batch windows")


def test_dropin_rope_and_norm_golden(golden, cuda):
    for name in ("rope_neox", "rope_interleaved", "rope_neox_odd"):
        hd, inter = (int(x) for x in golden[f"{name}/meta"])
        x = golden[f"{name}/x"].copy()
        smol_b200.apply_rope(x, golden[f"{name}/cos"], golden[f"{name}/sin"], len(x), 3, hd, interleaved=bool(inter))
        no_error()
        assert np.allclose(x, golden[f"{name}/out"], rtol=1e-6, atol=2e-6), name
    x = golden["rms_per_head/x"].copy()
    smol_b200.rms_norm_per_head(x, golden["rms_per_head/w"], 4, 3, 128, 1e-6)
    assert np.allclose(x, golden["rms_per_head/out"], rtol=1e-5, atol=1e-6)
    out = np.zeros_like(golden["rms_row/x"])
    smol_b200.rms_norm(out, golden["rms_row/x"], golden["rms_row/w"], 3, 1024, 1e-6)
    assert np.allclose(out, golden["rms_row/out"], rtol=1e-5, atol=1e-6)
    no_error()


def test_dropin_rope_tables_match_oracle_bitwise(cuda):
    o = pyoracle.oracle()
    pos = np.array([0, 1, 2, 513, 8191, 32767], np.int32)
    for inter in (False, True):
        c = np.zeros((len(pos), 128), np.float32)
        s = np.zeros_like(c)
        smol_b200.compute_rope(c, s, pos, len(pos), 128, 1e6, interleaved=inter)
        c2, s2 = o.compute_rope(pos, 128, 1e6, interleaved=inter)
        assert np.array_equal(c, c2) and np.array_equal(s, s2)
    pe = np.zeros((9, 32), np.float32)
    smol_b200.sinusoidal_pe(pe, 9, 32)
    assert np.array_equal(pe, o.sinusoidal_pe(9, 32))


# ---------------------------------------------------------------------------
# Fused prologue: exact position indexing and slot addressing
# ---------------------------------------------------------------------------
def test_rope_position_indexing_exact(cuda):
    # Table row p holds values that identify p; with x = 1 and sin = 0 the rotated
    # value must equal row positions[t] of the table exactly.
    n_pos, hd, nt = 300, 128, 7
    tab_c = (np.arange(n_pos, dtype=np.float32)[:, None] + np.arange(hd, dtype=np.float32)[None, :] / 256.0)
    tab_s = np.zeros_like(tab_c)
    positions = np.array([0, 1, 255, 256, 299, 17, 17], np.int32)
    slots = np.arange(nt, dtype=np.int64)
    q = torch.ones((nt, 2 * hd), device=cuda)
    k = torch.ones((nt, hd), device=cuda)
    qo = torch.zeros_like(q)
    kc = torch.zeros((nt, hd), dtype=torch.bfloat16, device=cuda)
    vc = torch.zeros((nt, hd), dtype=torch.float16, device=cuda)
    smol_b200.qknorm_rope_append(q, k, k, nt, 2, 1, hd, None, None, 1e-6, torch.from_numpy(tab_c).to(cuda),
                                 torch.from_numpy(tab_s).to(cuda), False,
                                 torch.from_numpy(positions).to(cuda), torch.from_numpy(slots).to(cuda), qo, None,
                                 kc, vc, nt)
    torch.cuda.synchronize()
    no_error()
    got = qo.cpu().numpy().reshape(nt, 2, hd)
    # NeoX: x1' = x1*c - x2*s = c,  x2' = x2*c + x1*s = c
    for t in range(nt):
        assert np.array_equal(got[t, 0], tab_c[positions[t]]), t
        assert np.array_equal(got[t, 1], tab_c[positions[t]]), t


def test_kv_slot_addressing_exact(cuda):
    # qkn_decoder.c:212-220: row ((layer*max)+pos); every other row keeps its sentinel.
    layers, cap, hkv, hd = 3, 40, 2, 64
    kv_dim = hkv * hd
    rows = layers * cap
    rng = np.random.default_rng(9)
    layer, start, n = 1, 13, 9
    slots = np.array([layer * cap + start + i for i in range(n)], np.int64)
    k_in = rng.standard_normal((n, kv_dim)).astype(np.float32)
    v_in = rng.standard_normal((n, kv_dim)).astype(np.float32)
    q_in = rng.standard_normal((n, 2 * kv_dim)).astype(np.float32)
    kc = torch.full((rows, kv_dim), -7.0, dtype=torch.bfloat16, device=cuda)
    vc = torch.full((rows, kv_dim), -7.0, dtype=torch.float16, device=cuda)
    smol_b200.qknorm_rope_append(torch.from_numpy(q_in).to(cuda), torch.from_numpy(k_in).to(cuda),
                                 torch.from_numpy(v_in).to(cuda), n, 4, hkv, hd, None, None, 1e-6, None, None, False,
                                 None, torch.from_numpy(slots).to(cuda), None, None, kc, vc, rows)
    torch.cuda.synchronize()
    no_error()
    kb = kc.view(torch.int16).cpu().numpy().view(np.uint16)
    vb = vc.view(torch.int16).cpu().numpy().view(np.uint16)
    written = np.zeros(rows, bool)
    written[slots] = True
    sentinel_k = pyoracle.bf16_bits(np.float32([-7.0]))[0]
    assert np.all(kb[~written] == sentinel_k)
    assert np.all(vb[~written] == np.float16(-7.0).view(np.uint16))
    assert np.array_equal(kb[slots], pyoracle.bf16_bits(k_in))            # bf16 round-to-nearest-even
    assert np.array_equal(vb[slots], v_in.astype(np.float16).view(np.uint16))


def test_qknorm_rope_append_matches_oracle(cuda):
    # cfg 1 prologue: 512 tokens, 16 Q / 8 KV heads, hd 128, per-head RMSNorm eps 1e-6
    # with weights ~N(1,0.02), NeoX RoPE theta 1e6, positions 0..511; plus an
    # interleaved hd-256 MQA variant (PaliGemma shape).
    for n, hq, hkv, hd, theta, inter, with_norm in [(512, 16, 8, 128, 1e6, False, True),
                                                   (64, 8, 1, 256, 1e4, True, False)]:
        rng = np.random.default_rng(0)
        q = rnd_bf16(rng, n, hq * hd)
        k = rnd_bf16(rng, n, hkv * hd)
        v = rnd_bf16(rng, n, hkv * hd)
        qw = (1 + 0.02 * rng.standard_normal(hd)).astype(np.float32) if with_norm else None
        kw = (1 + 0.02 * rng.standard_normal(hd)).astype(np.float32) if with_norm else None
        cos_t, sin_t = pyoracle.fill_rope_table(1024, hd, theta, interleaved=inter)
        pos = np.arange(n, dtype=np.int32)
        slots = (pos + 5).astype(np.int64)
        rows = n + 10
        kc_o = np.zeros((rows, hkv * hd), np.uint16)
        vc_o = np.zeros((rows, hkv * hd), np.uint16)
        q_o = pyoracle.qknorm_rope_append(q, k, v, hq, hkv, hd, qw, kw, 1e-6, cos_t, sin_t, inter, pos, slots,
                                          kc_o, vc_o)
        t = lambda a: None if a is None else torch.from_numpy(np.ascontiguousarray(a)).to(cuda)  # noqa: E731
        qo = torch.zeros((n, hq * hd), device=cuda)
        qb = torch.zeros((n, hq * hd), dtype=torch.bfloat16, device=cuda)
        kc = torch.zeros((rows, hkv * hd), dtype=torch.bfloat16, device=cuda)
        vc = torch.zeros((rows, hkv * hd), dtype=torch.float16, device=cuda)
        smol_b200.qknorm_rope_append(t(q), t(k), t(v), n, hq, hkv, hd, t(qw), t(kw), 1e-6, t(cos_t), t(sin_t), inter,
                                     t(pos), t(slots), qo, qb, kc, vc, rows)
        torch.cuda.synchronize()
        no_error()
        assert pyoracle.rel_l2(qo.cpu().numpy(), q_o) < 1e-6
        assert torch.equal(qb.float(), qo.to(torch.bfloat16).float())
        kd = kc.view(torch.int16).cpu().numpy().view(np.uint16).astype(np.int32)
        # fp32 results may differ in the last bit, so bf16 bits may differ by one step
        assert np.abs(kd - kc_o.astype(np.int32)).max() <= 1
        assert np.array_equal(vc.view(torch.int16).cpu().numpy().view(np.uint16), vc_o)


def test_fp16_v_overflow_is_reported(cuda):
    # The V cache is fp16 (largest finite 65504): a V value it cannot hold sets bit 6 of
    # the device error word instead of being stored silently as infinity; the drop-in
    # attention (which stages V as fp16) fails with SMOL_B200_ERR_RANGE and zeroes out.
    n, hq, hkv, hd = 4, 2, 1, 64
    q, k = torch.randn((n, hq * hd), device=cuda), torch.randn((n, hkv * hd), device=cuda)
    v = torch.randn((n, hkv * hd), device=cuda)
    kc = torch.zeros((n, hkv * hd), dtype=torch.bfloat16, device=cuda)
    vc = torch.zeros((n, hkv * hd), dtype=torch.float16, device=cuda)
    pos = torch.arange(n, dtype=torch.int32, device=cuda)
    args = (n, hq, hkv, hd, None, None, 1e-6, None, None, False, pos, pos.to(torch.int64), None, None, kc, vc, n)
    smol_b200.qknorm_rope_append(q, k, v, *args)
    torch.cuda.synchronize()
    assert smol_b200.device_error() == 0
    v[2, 7] = 65519.0                                   # rounds to 65504: still fits
    smol_b200.qknorm_rope_append(q, k, v, *args)
    torch.cuda.synchronize()
    assert smol_b200.device_error() == 0
    v[1, 3] = -7.0e4
    smol_b200.qknorm_rope_append(q, k, v, *args)
    torch.cuda.synchronize()
    assert smol_b200.device_error() == smol_b200.DEVERR_VALUE_RANGE
    smol_b200.clear_error()
    assert smol_b200.device_error() == 0
    Q = np.ones((3, hq * hd), np.float32)
    K = np.ones((3, hkv * hd), np.float32)
    V = np.ones((3, hkv * hd), np.float32)
    V[1, 0] = 1.0e5
    out = np.full((3, hq * hd), 9.0, np.float32)
    smol_b200.causal_attention(out, Q, K, V, 3, 3, hq, hkv, hd, 0.125, 0)
    assert smol_b200.last_error() == 7 and not out.any()
    smol_b200.clear_error()


# ---------------------------------------------------------------------------
# Batched split-KV decode
# ---------------------------------------------------------------------------
def make_pool(rng, lens, hkv, hd, cuda, extra_rows=37):
    lens = np.asarray(lens, np.int32)
    row0 = np.concatenate([[0], np.cumsum(lens + 3)[:-1]]).astype(np.int64)   # gaps between sequences
    rows = int(row0[-1] + lens[-1] + extra_rows)
    K = rnd_bf16(rng, rows, hkv * hd)
    V = rnd_bf16(rng, rows, hkv * hd)
    return row0, rows, K, V


def run_decode(cuda, Q, K, V, row0, lens, hq, hkv, hd, scale, q_bf16=False, window=0, softcap=0.0):
    n = len(lens)
    kp, vp = dev_bf16(K, cuda), dev_f16(V, cuda)
    q = torch.from_numpy(Q).to(cuda)
    if q_bf16:
        q = q.to(torch.bfloat16)
    out = torch.full((n, hq * hd), 5.0, device=cuda)
    max_len = int(max(lens)) if n else 0
    ws = torch.empty(smol_b200.decode_workspace_bytes(n, max_len, hq, hkv, hd), dtype=torch.uint8, device=cuda)
    smol_b200.decode_attention(out, q, kp, vp, K.shape[0], torch.from_numpy(row0).to(cuda),
                               torch.from_numpy(np.asarray(lens, np.int32)).to(cuda), n, max_len, hq, hkv, hd, scale,
                               ws, window=window, softcap=softcap)
    torch.cuda.synchronize()
    no_error()
    return out.cpu().numpy()


@pytest.mark.parametrize("hq,hkv,hd", [(16, 8, 128), (8, 1, 256), (12, 12, 64), (16, 1, 128), (32, 32, 64)])
def test_decode_batched_vs_oracle(cuda, hq, hkv, hd):
    rng = np.random.default_rng(hq * 1000 + hd)
    lens = [1, 2, 15, 16, 17, 63, 64, 65, 127, 513, 1000, 2049]
    row0, rows, K, V = make_pool(rng, lens, hkv, hd, cuda)
    Q = rng.standard_normal((len(lens), hq * hd)).astype(np.float32)    # fp32 Q (hi/lo split path)
    scale = 1.0 / np.sqrt(hd)
    got = run_decode(cuda, Q, K, V, row0, lens, hq, hkv, hd, scale)
    Vh = V.astype(np.float16).view(np.uint16)
    want = pyoracle.decode_batched(Q, pyoracle.bf16_bits(K), Vh, row0, lens, hq, hkv, hd, scale)
    assert_close(got, want, f"decode {hq}/{hkv}/{hd}")
    # bf16 Q
    Qb = pyoracle.round_bf16(Q)
    got = run_decode(cuda, Qb, K, V, row0, lens, hq, hkv, hd, scale, q_bf16=True)
    want = pyoracle.decode_batched(Qb, pyoracle.bf16_bits(K), Vh, row0, lens, hq, hkv, hd, scale)
    assert_close(got, want, f"decode bf16 q {hq}/{hkv}/{hd}")


def test_decode_zero_length_and_window_softcap(cuda):
    rng = np.random.default_rng(2)
    hq, hkv, hd = 4, 2, 128
    lens = [0, 5, 300, 129]
    row0, rows, K, V = make_pool(rng, lens, hkv, hd, cuda)
    Q = rng.standard_normal((len(lens), hq * hd)).astype(np.float32)
    o = pyoracle.oracle()
    for window, cap in [(0, 0.0), (64, 0.0), (0, 20.0), (100, 30.0)]:
        got = run_decode(cuda, Q, K, V, row0, lens, hq, hkv, hd, 0.09, window=window, softcap=cap)
        assert np.all(got[0] == 0.0)
        for b in range(1, len(lens)):
            r = slice(int(row0[b]), int(row0[b]) + lens[b])
            want = o.causal_attention(Q[b:b + 1], K[r], V[r].astype(np.float16).astype(np.float32), 1, lens[b], hq,
                                      hkv, hd, 0.09, lens[b] - 1, window=window, cap=cap)
            assert_close(got[b:b + 1], want, f"decode window={window} cap={cap} b={b}")


def test_decode_full_size_sampled(cuda):
    # cfg 2 at full size for one layer: 256 sequences, lengths ~U[1024, 8192] (seed 0),
    # 16 Q / 8 KV heads, hd 128; 24 sequences are checked against the oracle and the
    # rest through a size-independent property (uniform V rows -> output == that row).
    rng = np.random.default_rng(0)
    lens = rng.integers(1024, 8193, size=256).astype(np.int32)
    hq, hkv, hd = 16, 8, 128
    row0 = np.concatenate([[0], np.cumsum(lens)[:-1]]).astype(np.int64)
    rows = int(lens.sum())
    g = torch.Generator(device=cuda).manual_seed(0)
    kp = torch.randn((rows, hkv * hd), device=cuda, generator=g).to(torch.bfloat16)
    vp = torch.randn((rows, hkv * hd), device=cuda, generator=g).to(torch.float16)
    q = torch.randn((256, hq * hd), device=cuda, generator=g)
    out = torch.zeros((256, hq * hd), device=cuda)
    ws = torch.empty(smol_b200.decode_workspace_bytes(256, 8192, hq, hkv, hd), dtype=torch.uint8, device=cuda)
    r0 = torch.from_numpy(row0).to(cuda)
    kl = torch.from_numpy(lens).to(cuda)
    smol_b200.decode_attention(out, q, kp, vp, rows, r0, kl, 256, 8192, hq, hkv, hd, 1 / np.sqrt(hd), ws)
    torch.cuda.synchronize()
    no_error()
    pick = rng.choice(256, size=24, replace=False)
    Kb = kp.view(torch.int16)
    Vb = vp.view(torch.int16)
    for b in pick:
        r = slice(int(row0[b]), int(row0[b] + lens[b]))
        Kh = Kb[r].cpu().numpy().view(np.uint16)
        Vh = Vb[r].cpu().numpy().view(np.uint16)
        want = pyoracle.decode_batched(q[b:b + 1].cpu().numpy(), Kh, Vh, np.array([0], np.int64), lens[b:b + 1], hq,
                                       hkv, hd, 1 / np.sqrt(hd))
        assert_close(out[b:b + 1].cpu().numpy(), want, f"cfg2 seq {b}")
    # property: V rows constant per sequence -> every head's output equals that row
    vconst = torch.randn((256, hkv * hd), device=cuda, generator=g).to(torch.float16)
    seq_of_row = torch.repeat_interleave(torch.arange(256, device=cuda), kl.long())
    vp2 = vconst[seq_of_row]
    smol_b200.decode_attention(out, q, kp, vp2, rows, r0, kl, 256, 8192, hq, hkv, hd, 1 / np.sqrt(hd), ws)
    torch.cuda.synchronize()
    no_error()
    want = vconst.float().view(256, hkv, 1, hd).expand(256, hkv, hq // hkv, hd).reshape(256, hq * hd)
    assert_close(out.cpu().numpy(), want.cpu().numpy(), "uniform V")


# ---------------------------------------------------------------------------
# tcgen05 prefill through the device API
# ---------------------------------------------------------------------------
def run_prefill(cuda, q, k, v, batch, sq, sk, hq, hkv, hd, scale, mask=smol_b200.MASK_CAUSAL, **kw):
    out = torch.full((batch, sq, hq * hd), 9.0, device=cuda)
    smol_b200.prefill_attention(out, dev_bf16(q, cuda), dev_bf16(k, cuda), dev_f16(v, cuda), batch, sq, sk, hq, hkv,
                                hd, scale, mask_kind=mask, **kw)
    torch.cuda.synchronize()
    no_error()
    return out.cpu().numpy()


def test_prefill_cfg1_causal(cuda):
    # cfg 1: 512 tokens, 16 Q / 8 KV heads, hd 128, N(0,1) bf16, seed 0
    rng = np.random.default_rng(0)
    q, k, v = rnd_bf16(rng, 512, 16 * 128), rnd_bf16(rng, 512, 8 * 128), rnd_bf16(rng, 512, 8 * 128)
    got = run_prefill(cuda, q, k, v, 1, 512, 512, 16, 8, 128, 1 / np.sqrt(128))
    want = pyoracle.oracle().causal_attention(q, k, v, 512, 512, 16, 8, 128, 1 / np.sqrt(128), 0)
    assert_close(got[0], want, "cfg1 prefill")


def test_prefill_cfg3_siglip_image(cuda):
    # cfg 3: 1024 patches, 12 heads, hd 64, non-causal, window {0, N} (siglip.c:108)
    rng = np.random.default_rng(1)
    q, k, v = (rnd_bf16(rng, 1024, 12 * 64) for _ in range(3))
    ws = torch.tensor([0, 1024], dtype=torch.int32, device=cuda)
    got = run_prefill(cuda, q, k, v, 1, 1024, 1024, 12, 12, 64, 0.125, mask=smol_b200.MASK_WINDOWS,
                      window_starts=ws)
    want = pyoracle.oracle().bidirectional_attention(q, k, v, 1024, 12, 64, 0.125, [0, 1024])
    assert_close(got[0], want, "cfg3 siglip")
    got2 = run_prefill(cuda, q, k, v, 1, 1024, 1024, 12, 12, 64, 0.125, mask=smol_b200.MASK_FULL)
    assert_close(got2[0], want, "cfg3 full mask")


@pytest.mark.parametrize("hd", [256, 136])
def test_prefill_windows_wide_heads_vs_oracle(cuda, hd):
    # Window masks on the 256-wide kernel: its epilogue warps store row by row where a
    # warp holds rows no window covers, and those rows stay untouched (attention.c:39-43).
    rng = np.random.default_rng(hd)
    S, h = 300, 2
    q, k, v = (rnd_bf16(rng, S, h * hd) for _ in range(3))
    starts = [7, 100, 230, 290]
    ws = torch.tensor(starts, dtype=torch.int32, device=cuda)
    got = run_prefill(cuda, q, k, v, 1, S, S, h, h, hd, 0.1, mask=smol_b200.MASK_WINDOWS, window_starts=ws)
    want = pyoracle.oracle().bidirectional_attention(q, k, v, S, h, hd, 0.1, starts,
                                                     out=np.full((S, h * hd), 9.0, np.float32))
    assert_close(got[0], want, f"windows hd {hd}")
    assert (got[0][:7] == 9.0).all() and (got[0][290:] == 9.0).all()


def test_prefill_cfg4_prefix_lm(cuda):
    # cfg 4: prefix 320 (256 image + 64 text) bidirectional, then a causal suffix,
    # MQA 8/1, hd 256.  Oracle: the reference's two-call composition.
    rng = np.random.default_rng(4)
    seq, P = 448, 320
    q, k, v = rnd_bf16(rng, seq, 8 * 256), rnd_bf16(rng, seq, 256), rnd_bf16(rng, seq, 256)
    got = run_prefill(cuda, q, k, v, 1, seq, seq, 8, 1, 256, 1 / 16, mask=smol_b200.MASK_PREFIX_LM, prefix_len=P)
    want = pyoracle.oracle().prefix_lm_attention(q, k, v, seq, P, 8, 1, 256, 1 / 16)
    assert_close(got[0], want, "cfg4 prefix-LM")


def test_prefill_golden_prefix_lm(golden, cuda):
    seq, P, hq, hkv, hd = (int(x) for x in golden["prefix_lm/meta"])
    q, k, v = qkv(golden, "prefix_lm")
    got = run_prefill(cuda, q, k, v, 1, seq, seq, hq, hkv, hd, float(golden["prefix_lm/fmeta"][0]),
                      mask=smol_b200.MASK_PREFIX_LM, prefix_len=P)
    assert_close(got[0], golden["prefix_lm/out"], "golden prefix-LM")


@pytest.mark.parametrize("sq,sk,qo,hq,hkv,hd,win,cap", [
    (1, 1, 0, 2, 1, 64, 0, 0.0),
    (5, 5, 0, 2, 2, 128, 0, 0.0),
    (129, 129, 0, 4, 2, 128, 0, 0.0),
    (257, 300, 43, 2, 1, 256, 0, 0.0),
    (200, 200, 0, 16, 8, 128, 64, 0.0),
    (150, 150, 0, 4, 4, 64, 0, 40.0),
    (300, 700, 400, 8, 2, 64, 128, 25.0),
    (64, 0, 0, 2, 1, 128, 0, 0.0),
    (40, 30, -20, 2, 1, 128, 0, 0.0),
    (64, 0, 0, 8, 1, 256, 0, 0.0),        # head dim 256, packed MQA rows: no keys at all
    (40, 30, -20, 8, 1, 256, 0, 0.0),     # rows before the first key are zero
    (300, 300, 0, 4, 2, 256, 40, 30.0),   # packed GQA pairs, window + softcap
    (129, 200, 71, 4, 2, 72, 0, 0.0),     # head dim 72 (SigLIP-So400m) on the 128-wide kernel
    (150, 150, 0, 2, 2, 40, 0, 20.0),     # head dim 40 on the 64-wide kernel
    (100, 140, 40, 8, 1, 136, 50, 0.0),   # head dim 136 on the 256-wide kernel, packed MQA rows
])
def test_prefill_edges_vs_oracle(cuda, sq, sk, qo, hq, hkv, hd, win, cap):
    rng = np.random.default_rng(sq * 7 + sk)
    q, k, v = rnd_bf16(rng, sq, hq * hd), rnd_bf16(rng, max(sk, 1), hkv * hd), rnd_bf16(rng, max(sk, 1), hkv * hd)
    got = run_prefill(cuda, q, k, v, 1, sq, sk, hq, hkv, hd, 0.1, q_offset=qo, window=win, softcap=cap)
    want = pyoracle.oracle().causal_attention(q, k, v, sq, sk, hq, hkv, hd, 0.1, qo, window=win, cap=cap)
    assert_close(got[0], want, f"prefill {sq}x{sk} qo={qo} win={win} cap={cap}")


@pytest.mark.parametrize("sq,cut,qo,hq,hkv,hd,win,cap", [
    (299, 150, 0, 8, 1, 256, 64, 50.0),    # Gemma-2 shape: MQA hd 256 (v1 kernel), window + softcap
    (400, 173, 37, 16, 8, 128, 64, 0.0),   # hd 128 (v2 kernel, paired heads), q_offset > 0
    (333, 100, 5, 3, 1, 64, 100, 0.0),     # hd 64, odd GQA group (v2, consecutive row blocks)
])
def test_prefill_window_chunk_invariant(cuda, sq, cut, qo, hq, hkv, hd, win, cap):
    # A chunked prefill under a sliding window (the second chunk continues at
    # q_offset + cut) must write exactly what one call writes: streaming prefix reuse
    # truncates the cache and prefills only the delta (qwen_asr.c:1599-1614).
    rng = np.random.default_rng(sq + cut)
    sk = qo + sq
    q, k, v = rnd_bf16(rng, sq, hq * hd), rnd_bf16(rng, sk, hkv * hd), rnd_bf16(rng, sk, hkv * hd)
    one = run_prefill(cuda, q, k, v, 1, sq, sk, hq, hkv, hd, 0.1, q_offset=qo, window=win, softcap=cap)[0]
    a = run_prefill(cuda, q[:cut], k, v, 1, cut, qo + cut, hq, hkv, hd, 0.1, q_offset=qo, window=win,
                    softcap=cap)[0]
    b = run_prefill(cuda, q[cut:], k, v, 1, sq - cut, sk, hq, hkv, hd, 0.1, q_offset=qo + cut, window=win,
                    softcap=cap)[0]
    two = np.concatenate([a, b])
    diff = np.abs(two - one)
    assert np.array_equal(two, one), f"chunked != one call: max |d| {diff.max():.3e} at row {diff.max(1).argmax()}"
    want = pyoracle.oracle().causal_attention(q, k, v, sq, sk, hq, hkv, hd, 0.1, qo, window=win, cap=cap)
    assert_close(one, want, f"prefill window {win} qo={qo}")


@pytest.mark.parametrize("hd,hq,hkv,mask", [(64, 4, 4, "windows"), (128, 8, 4, "causal"), (128, 3, 1, "full"),
                                             (256, 8, 1, "prefix")])
def test_prefill_bf16_output_is_rounded_fp32_output(cuda, hd, hq, hkv, mask):
    # smol_b200_prefill_attention_bf16: the same result rounded to bf16 (nearest even),
    # bit for bit, in a strided output; rows no window covers stay untouched.
    rng = np.random.default_rng(hd + hq)
    B, S = 2, 333
    q, k, v = rnd_bf16(rng, B, S, hq * hd), rnd_bf16(rng, B, S, hkv * hd), rnd_bf16(rng, B, S, hkv * hd)
    kw = {}
    kind = {"windows": smol_b200.MASK_WINDOWS, "causal": smol_b200.MASK_CAUSAL, "full": smol_b200.MASK_FULL,
            "prefix": smol_b200.MASK_PREFIX_LM}[mask]
    if mask == "windows":
        kw["window_starts"] = torch.tensor([5, 104, 208, 300], dtype=torch.int32, device=cuda)
    if mask == "prefix":
        kw["prefix_len"] = 200
    ow = hq * hd + 8
    strides = ((ow, S * ow), (hq * hd, S * hq * hd), (hkv * hd, S * hkv * hd), (hkv * hd, S * hkv * hd))
    args = (dev_bf16(q, cuda), dev_bf16(k, cuda), dev_f16(v, cuda), B, S, S, hq, hkv, hd, 0.09)
    out32 = torch.full((B, S, ow), 5.0, device=cuda)
    smol_b200.prefill_attention(out32, *args, mask_kind=kind, strides=strides, **kw)
    out16 = torch.full((B, S, ow), 5.0, device=cuda, dtype=torch.bfloat16)
    smol_b200.prefill_attention(out16, *args, mask_kind=kind, strides=strides, **kw)
    torch.cuda.synchronize()
    no_error()
    want = out32.to(torch.bfloat16)
    assert torch.equal(out16.view(torch.int16), want.view(torch.int16)), \
        float((out16.float() - want.float()).abs().max())
    if mask == "windows":
        assert bool((out16[:, :5].float() == 5.0).all()) and bool((out16[:, 300:].float() == 5.0).all())


@pytest.mark.parametrize("hd,hq,hkv,mask", [(64, 4, 4, "full"), (64, 2, 1, "causal"), (128, 4, 2, "causal"),
                                             (72, 2, 2, "full"), (256, 8, 1, "causal")])
def test_prefill_scores_growing_across_key_tiles(cuda, hd, hq, hkv, mask):
    # Even rows' scores grow by ~20 (natural units) from one 128-key tile to the next and
    # odd rows' fall: an even row's exponentials against its first tile's maximum would
    # pass fp16 on every later tile, so its reference maximum must move (the rescale
    # path), while the odd rows of the same warp keep theirs.
    rng = np.random.default_rng(hd * 3 + hq)
    S = 600
    scale = 1 / np.sqrt(hd)
    B = 8.0
    u = np.ones(hd, np.float32) / np.sqrt(hd)
    a = np.arange(S, dtype=np.float32) * (20.0 / (128 * B * scale))
    sign = np.where(np.arange(S) % 2 == 0, 1.0, -1.0).astype(np.float32)
    q = (sign[:, None, None] * B * u[None, None, :] + 0.05 * rng.standard_normal((S, hq, hd))).reshape(S, hq * hd)
    k = (a[:, None, None] * u[None, None, :] + 0.05 * rng.standard_normal((S, hkv, hd))).reshape(S, hkv * hd)
    q, k = pyoracle.round_bf16(q.astype(np.float32)), pyoracle.round_bf16(k.astype(np.float32))
    v = rnd_bf16(rng, S, hkv * hd)
    o = pyoracle.oracle()
    if mask == "full":
        got = run_prefill(cuda, q, k, v, 1, S, S, hq, hkv, hd, scale, mask=smol_b200.MASK_FULL)
        want = o.bidirectional_attention(q, k, v, S, hq, hd, scale, [0, S])
    else:
        got = run_prefill(cuda, q, k, v, 1, S, S, hq, hkv, hd, scale)
        want = o.causal_attention(q, k, v, S, S, hq, hkv, hd, scale, 0)
    assert np.isfinite(got).all()
    assert_close(got[0], want, f"growing scores hd {hd} {mask}")


def test_prefill_siglip_so400m_head_dim_72(cuda):
    # SmolVLM's vision tower (SigLIP-So400m: 729 patches, 16 heads of 72) -- bidirectional
    # attention per image on the 128-wide kernel with the caller's 72-column rows: the
    # columns past 72 are read as zero and never written, so the output rows (and the
    # 8 columns of padding the strided output keeps between them) stay exact.
    rng = np.random.default_rng(729)
    B, N, h, hd = 2, 729, 16, 72
    q, k, v = rnd_bf16(rng, B, N, h * hd), rnd_bf16(rng, B, N, h * hd), rnd_bf16(rng, B, N, h * hd)
    ow = h * hd + 8
    strides = ((ow, N * ow), (h * hd, N * h * hd), (h * hd, N * h * hd), (h * hd, N * h * hd))
    args = (dev_bf16(q, cuda), dev_bf16(k, cuda), dev_f16(v, cuda), B, N, N, h, h, hd, 1 / np.sqrt(hd))
    out32 = torch.full((B, N, ow), 5.0, device=cuda)
    smol_b200.prefill_attention(out32, *args, mask_kind=smol_b200.MASK_FULL, strides=strides)
    out16 = torch.full((B, N, ow), 5.0, device=cuda, dtype=torch.bfloat16)
    smol_b200.prefill_attention(out16, *args, mask_kind=smol_b200.MASK_FULL, strides=strides)
    torch.cuda.synchronize()
    no_error()
    got = out32.cpu().numpy()
    assert bool((got[:, :, h * hd:] == 5.0).all())
    for b in range(B):
        want = pyoracle.oracle().bidirectional_attention(q[b], k[b], v[b], N, h, hd, 1 / np.sqrt(hd), [0, N])
        assert_close(got[b, :, :h * hd], want, f"so400m image {b}")
    assert torch.equal(out16.view(torch.int16), out32.to(torch.bfloat16).view(torch.int16))


def test_bf16_decoder_reference_second_oracle(cuda):
    # The reference's own bf16-cache attention (qkn_bf16_decoder.c:120-233: fp32 scores,
    # two-pass softmax, output truncated to bf16; fixtures from
    # tests/golden/make_bf16_golden.py) on the device path: seq_q > 1 through the tcgen05
    # prefill, seq_q == 1 through the split-KV decode over a pool, with the PaliGemma
    # decoder's settings (MQA 8/1, head dim 256, softcap 50, sliding window).  V goes in
    # as fp16 (every bf16 value of these inputs is exact in fp16).  The device's fp32
    # result must lie within 2e-3 relative or 4e-4 absolute of the interval each truncated
    # reference value stands for: P in fp16 (2^-11 relative per weight) moves an output of
    # ~0.1, an average of ~70 values ~N(0,1), by up to ~2e-4.
    import os

    from conftest import assert_within_bf16_truncation
    g = np.load(os.path.join(os.path.dirname(__file__), "golden", "bf16_decoder_cases.npz"))
    for name in sorted({k.split("/")[0] for k in g.files}):
        sq, sk, hq, hkv, hd, qo, win = (int(x) for x in g[f"{name}/meta"])
        scale, cap = (float(x) for x in g[f"{name}/fmeta"])
        q, k, v = (pyoracle.bf16_to_f32(g[f"{name}/{t}_bf16"]) for t in ("q", "k", "v"))
        if sq > 1:
            got = run_prefill(cuda, q, k, v, 1, sq, sk, hq, hkv, hd, scale, q_offset=qo, window=win, softcap=cap)[0]
        else:
            assert qo == sk - 1
            out = torch.zeros((1, hq * hd), device=cuda)
            ws = torch.empty(smol_b200.decode_workspace_bytes(1, sk, hq, hkv, hd), dtype=torch.uint8, device=cuda)
            smol_b200.decode_attention(out, dev_bf16(q, cuda), dev_bf16(k, cuda), dev_f16(v, cuda), sk,
                                       torch.zeros(1, dtype=torch.int64, device=cuda),
                                       torch.full((1,), sk, dtype=torch.int32, device=cuda), 1, sk, hq, hkv, hd,
                                       scale, ws, window=win, softcap=cap)
            torch.cuda.synchronize()
            no_error()
            got = out.cpu().numpy()
        assert_within_bf16_truncation(got, g[f"{name}/out_bf16"], rel_tol=2e-3, abs_tol=4e-4, what=name)


def test_prefill_batched_strided(cuda):
    # batch of 3 sequences inside wider buffers (row strides > heads*hd)
    rng = np.random.default_rng(8)
    B, S, hq, hkv, hd = 3, 200, 4, 2, 128
    qw, kw = hq * hd + 64, hkv * hd + 128
    Q = rnd_bf16(rng, B, S, qw)
    K = rnd_bf16(rng, B, S, kw)
    V = rnd_bf16(rng, B, S, kw)
    out = torch.zeros((B, S, hq * hd + 32), device=cuda)
    smol_b200.prefill_attention(out, dev_bf16(Q, cuda), dev_bf16(K, cuda), dev_f16(V, cuda), B, S, S, hq, hkv, hd, 0.1,
                                strides=((hq * hd + 32, S * (hq * hd + 32)), (qw, S * qw), (kw, S * kw),
                                         (kw, S * kw)))
    torch.cuda.synchronize()
    no_error()
    o = pyoracle.oracle()
    got = out.cpu().numpy()
    for b in range(B):
        want = o.causal_attention(np.ascontiguousarray(Q[b, :, :hq * hd]), np.ascontiguousarray(K[b, :, :hkv * hd]),
                                  np.ascontiguousarray(V[b, :, :hkv * hd]), S, S, hq, hkv, hd, 0.1, 0)
        assert_close(got[b, :, :hq * hd], want, f"batch {b}")


def test_prefill_cfg5_full_length_sampled(cuda):
    # cfg 5 shape at full length for one KV head: L = 32768 causal, 2 Q heads, hd 128.
    # Sampled rows against the oracle (per row the oracle costs O(L*hd)), and the
    # uniform-V property on all rows.
    L, hq, hkv, hd = 32768, 2, 1, 128
    g = torch.Generator(device=cuda).manual_seed(5)
    q = torch.randn((1, L, hq * hd), device=cuda, generator=g).to(torch.bfloat16)
    k = torch.randn((1, L, hkv * hd), device=cuda, generator=g).to(torch.bfloat16)
    v = torch.randn((1, L, hkv * hd), device=cuda, generator=g).to(torch.float16)
    out = torch.zeros((1, L, hq * hd), device=cuda)
    smol_b200.prefill_attention(out, q, k, v, 1, L, L, hq, hkv, hd, 1 / np.sqrt(hd))
    torch.cuda.synchronize()
    no_error()
    o = pyoracle.oracle()
    qn, kn, vn = q[0].float().cpu().numpy(), k[0].float().cpu().numpy(), v[0].float().cpu().numpy()
    for row in [0, 1, 127, 128, 129, 4095, 20000, L - 1]:
        want = o.causal_attention(qn[row:row + 1], kn[:row + 1], vn[:row + 1], 1, row + 1, hq, hkv, hd,
                                  1 / np.sqrt(hd), row)
        assert_close(out[0, row:row + 1].cpu().numpy(), want, f"cfg5 row {row}")
    vconst = torch.randn((1, 1, hkv * hd), device=cuda, generator=g).to(torch.float16).expand(1, L, hkv * hd)
    smol_b200.prefill_attention(out, q, k, vconst.contiguous(), 1, L, L, hq, hkv, hd, 1 / np.sqrt(hd))
    torch.cuda.synchronize()
    no_error()
    want = vconst[:, :, None, :].float().expand(1, L, hq, hd).reshape(1, L, hq * hd)
    assert_close(out.cpu().numpy(), want.cpu().numpy(), "cfg5 uniform V")


# ---------------------------------------------------------------------------
# The host-buffer decode step (the call bench.py's end-to-end number goes through)
# ---------------------------------------------------------------------------
@pytest.mark.parametrize("n", [6, 70, 130])   # one chunk, and two pipelined chunks (a quarter, then the rest)
def test_decode_step_host_vs_oracle(cuda, n):
    rng = np.random.default_rng(12 + n)
    hq, hkv, hd = 16, 8, 128
    lens = (np.array([1, 100, 512, 513, 700, 64], np.int32) if n == 6
            else rng.integers(1, 700, size=n).astype(np.int32))
    cap_rows = lens + 1
    row0 = np.concatenate([[0], np.cumsum(cap_rows)[:-1]]).astype(np.int64)
    rows = int(cap_rows.sum())
    K = rnd_bf16(rng, rows, hkv * hd)
    V = rnd_bf16(rng, rows, hkv * hd)
    kp, vp = dev_bf16(K, cuda), dev_f16(V, cuda)
    cos_t, sin_t = pyoracle.fill_rope_table(1024, hd, 1e6)
    qw = (1 + 0.02 * rng.standard_normal(hd)).astype(np.float32)
    kw = (1 + 0.02 * rng.standard_normal(hd)).astype(np.float32)
    qh = rnd_bf16(rng, n, hq * hd)
    kh = rnd_bf16(rng, n, hkv * hd)
    vh = rnd_bf16(rng, n, hkv * hd)
    out = np.zeros((n, hq * hd), np.float32)
    if n > 6:   # pinned host memory, so the chunks' copies overlap their compute
        pin = lambda a: torch.from_numpy(np.ascontiguousarray(a)).pin_memory().numpy()  # noqa: E731
        out, qh, kh, vh = pin(out), pin(qh), pin(kh), pin(vh)
    scratch = torch.empty(smol_b200.decode_step_scratch_bytes(n, int(lens.max()), hq, hkv, hd), dtype=torch.uint8,
                          device=cuda)
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(cuda)  # noqa: E731
    smol_b200.decode_step_host(out, qh, kh, vh, n, hq, hkv, hd, t(qw), t(kw), 1e-6, t(cos_t), t(sin_t), False, kp, vp,
                               rows, t(row0), t(lens), int(lens.max()), 1 / np.sqrt(hd), scratch)
    no_error()
    # oracle: prologue into a numpy copy of the cache, then per-sequence decode
    kb = pyoracle.bf16_bits(K)
    vb = V.astype(np.float16).view(np.uint16)
    qr = pyoracle.qknorm_rope_append(qh, kh, vh, hq, hkv, hd, qw, kw, 1e-6, cos_t, sin_t, False, lens, row0 + lens,
                                     kb, vb)
    want = pyoracle.decode_batched(qr, kb, vb, row0, lens + 1, hq, hkv, hd, 1 / np.sqrt(hd))
    assert_close(out, want, "decode step (host buffers)")
    # the appended rows landed exactly in rows row0+len
    got_k = kp.view(torch.int16).cpu().numpy().view(np.uint16)
    assert np.abs(got_k[row0 + lens].astype(np.int32) - kb[row0 + lens].astype(np.int32)).max() <= 1
