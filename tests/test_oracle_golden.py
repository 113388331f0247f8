"""The oracle restatement, pinned against the reference's own outputs.

tests/golden/reference_cases.npz holds outputs of the compiled reference
(common/kernels/attention.c, rope.c, rmsnorm.c of tmzt/smol-genius; generator:
tests/golden/make_golden.py).  The restatement in oracle/smol_oracle.c must agree
with them to fp32 rounding; where the compiled reference itself is present
(oracle/_ref) the two are also compared on fresh seeded cases.
"""
import numpy as np
import pytest

import pyoracle

TIGHT = 2e-6   # restatement vs reference: only summation order differs


def qkv(g, name):
    return [pyoracle.bf16_to_f32(g[f"{name}/{t}_bf16"]) for t in ("q", "k", "v")]


def case_names(g, prefixes):
    return sorted({k.split("/")[0] for k in g.files if k.split("/")[0].startswith(prefixes)})


def test_causal_family_matches_reference(golden):
    o = pyoracle.oracle()
    names = case_names(golden, ("causal", "sliding"))
    assert len(names) >= 8
    for name in names:
        sq, sk, hq, hkv, hd, qo, win = golden[f"{name}/meta"]
        scale, cap = golden[f"{name}/fmeta"]
        q, k, v = qkv(golden, name)
        out = o.causal_attention(q, k, v, sq, sk, hq, hkv, hd, scale, qo, window=win, cap=cap)
        assert pyoracle.rel_l2(out, golden[f"{name}/out"]) < TIGHT, name


def test_empty_rows_are_zero(golden):
    # rows whose key range is empty keep the zeroed output (attention.c:100, :120)
    out = golden["causal_empty_rows/out"]
    assert np.all(out[:3] == 0.0) and np.any(out[3:] != 0.0)


def test_bidirectional_matches_reference(golden):
    o = pyoracle.oracle()
    for name in case_names(golden, ("bidir",)):
        seq, h, hd = golden[f"{name}/meta"]
        q, k, v = qkv(golden, name)
        out = o.bidirectional_attention(q, k, v, seq, h, hd, golden[f"{name}/fmeta"][0], golden[f"{name}/ws"])
        assert pyoracle.rel_l2(out, golden[f"{name}/out"]) < TIGHT, name


def test_prefix_lm_matches_reference(golden):
    o = pyoracle.oracle()
    seq, P, hq, hkv, hd = golden["prefix_lm/meta"]
    q, k, v = qkv(golden, "prefix_lm")
    scale = golden["prefix_lm/fmeta"][0]
    # the restatement's single prefix-LM pass against the reference's two-call composition
    from ctypes import c_float, c_int, c_void_p
    lib = pyoracle._load(pyoracle.ORACLE_SO)
    out = np.zeros((seq, hq * hd), np.float32)
    q, k, v = (np.ascontiguousarray(a) for a in (q, k, v))
    lib.oracle_prefix_lm_attention(c_void_p(out.ctypes.data), c_void_p(q.ctypes.data), c_void_p(k.ctypes.data),
                                   c_void_p(v.ctypes.data), c_int(seq), c_int(seq), c_int(hq), c_int(hkv),
                                   c_int(hd), c_float(scale), c_int(0), c_int(P))
    assert pyoracle.rel_l2(out, golden["prefix_lm/out"]) < TIGHT


def test_rope_tables_match_reference(golden):
    # The reference is built with -ffast-math (its Makefile:6), so gcc evaluates
    # powf/cosf/sinf through vectorised approximations: one ulp of inv_freq moves the
    # angle pos*inv_freq by up to pos*6e-8 rad (2.3e-4 at pos 4095).  The tables agree
    # to that bound; positions index rows bit-exactly (checked on the GPU).
    o = pyoracle.oracle()
    for name in ("rope_neox", "rope_interleaved", "rope_neox_odd"):
        hd, inter = golden[f"{name}/meta"]
        theta = golden[f"{name}/fmeta"][0]
        pos = golden[f"{name}/pos"].astype(np.float64)
        c, s = o.compute_rope(golden[f"{name}/pos"], hd, theta, interleaved=bool(inter))
        bound = (2e-6 + 1.2e-7 * pos)[:, None]
        assert np.all(np.abs(c - golden[f"{name}/cos"]) <= bound), name
        assert np.all(np.abs(s - golden[f"{name}/sin"]) <= bound), name
        c, s = golden[f"{name}/cos"], golden[f"{name}/sin"]
        y = o.apply_rope(golden[f"{name}/x"], c, s, len(c), 3, hd, interleaved=bool(inter))
        assert np.allclose(y, golden[f"{name}/out"], rtol=1e-6, atol=1e-6), name


def test_decoder_rope_table_matches_compute_rope():
    # qkn_decoder.c:261-311 builds rows pos*hd with the same formula as rope.c:27-45
    c, s = pyoracle.fill_rope_table(300, 128, 1e6, interleaved=False)
    c2, s2 = pyoracle.oracle().compute_rope(np.arange(300), 128, 1e6)
    assert np.array_equal(c, c2) and np.array_equal(s, s2)


def test_rms_norms(golden):
    o = pyoracle.oracle()
    out = o.rms_norm_per_head(golden["rms_per_head/x"], golden["rms_per_head/w"], 4, 3, 128, 1e-6)
    assert np.allclose(out, golden["rms_per_head/out"], rtol=1e-5, atol=1e-6)
    out = o.rms_norm(golden["rms_row/x"], golden["rms_row/w"], 3, 1024, 1e-6)
    assert np.allclose(out, golden["rms_row/out"], rtol=1e-5, atol=1e-6)
    assert np.allclose(o.sinusoidal_pe(9, 32), golden["sinusoidal/out"], rtol=1e-6, atol=1e-6)


def test_decode_batched_is_per_sequence_causal():
    rng = np.random.default_rng(3)
    hq, hkv, hd = 4, 2, 64
    lens = np.array([5, 1, 17], np.int32)
    row0 = np.array([0, 20, 40], np.int64)
    K = pyoracle.bf16_bits(rng.standard_normal((60, hkv * hd)).astype(np.float32))
    Vf = pyoracle.round_bf16(rng.standard_normal((60, hkv * hd)).astype(np.float32))
    V = Vf.astype(np.float16).view(np.uint16)
    Q = rng.standard_normal((3, hq * hd)).astype(np.float32)
    out = pyoracle.decode_batched(Q, K, V, row0, lens, hq, hkv, hd, 0.125)
    o = pyoracle.oracle()
    Kf = pyoracle.bf16_to_f32(K)
    for b in range(3):
        r = slice(row0[b], row0[b] + lens[b])
        want = o.causal_attention(Q[b:b + 1], Kf[r], Vf[r], 1, lens[b], hq, hkv, hd, 0.125, lens[b] - 1)
        assert np.allclose(out[b], want[0], rtol=1e-6, atol=1e-6)


@pytest.mark.skipif(pyoracle.reference() is None, reason="compiled reference not present")
def test_restatement_vs_live_reference_random():
    rng = np.random.default_rng(11)
    o, r = pyoracle.oracle(), pyoracle.reference()
    pyoracle.set_reference_threads(1)
    for sq, sk, hq, hkv, hd, qo, win, cap in [(9, 64, 6, 3, 32, 55, 0, 0.0), (3, 3, 1, 1, 16, 0, 2, 5.0),
                                              (1, 200, 16, 8, 128, 199, 0, 0.0)]:
        q = rng.standard_normal((sq, hq * hd)).astype(np.float32)
        k = rng.standard_normal((sk, hkv * hd)).astype(np.float32)
        v = rng.standard_normal((sk, hkv * hd)).astype(np.float32)
        a = o.causal_attention(q, k, v, sq, sk, hq, hkv, hd, 0.3, qo, window=win, cap=cap)
        b = r.causal_attention(q, k, v, sq, sk, hq, hkv, hd, 0.3, qo, window=win, cap=cap)
        assert pyoracle.rel_l2(a, b) < TIGHT


def test_oracle_matches_reference_bf16_decoder_attention():
    """Second oracle for the bf16-cache path: the reference's own bf16 decoder attention
    (qkn_bf16_decoder.c:120-233, fp32 two-pass softmax, output truncated to bf16;
    fixtures from tests/golden/make_bf16_golden.py).  The restatement's fp32 result must
    lie within fp32 rounding of the interval the truncated value stands for: relative
    2e-5, and absolute 1e-5 for outputs that nearly cancel (the reference sums up to 200
    weighted |v| <= ~5 in fp32 in its own order, ~1e-6 apart from ours)."""
    import os

    from conftest import assert_within_bf16_truncation
    g = np.load(os.path.join(os.path.dirname(__file__), "golden", "bf16_decoder_cases.npz"))
    o = pyoracle.oracle()
    names = sorted({k.split("/")[0] for k in g.files})
    assert len(names) == 7
    for name in names:
        sq, sk, hq, hkv, hd, qo, win = (int(x) for x in g[f"{name}/meta"])
        scale, cap = (float(x) for x in g[f"{name}/fmeta"])
        q, k, v = (pyoracle.bf16_to_f32(g[f"{name}/{t}_bf16"]) for t in ("q", "k", "v"))
        got = o.causal_attention(q, k, v, sq, sk, hq, hkv, hd, scale, qo, window=win, cap=cap)
        assert_within_bf16_truncation(got, g[f"{name}/out_bf16"], rel_tol=2e-5, abs_tol=1e-5, what=name)
