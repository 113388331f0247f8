"""Device prefill of the decoder (smol_b200_qkn_prefill) against the CPU restatement.

The device prefill runs qkn_decoder_prefill (qkn_decoder.c:369-564) with tcgen05 GEMMs
over bf16 activations; the oracle (oracle/qkn_decoder_oracle.py) restates it with the
same bf16 operand roundings (`device_formats=True`).  Checked, for a 2-layer Qwen3 model
and the Gemma 2 settings (MQA 8/1, head dim 256, GeGLU, sublayer norms, softcap, a
sliding layer with its own RoPE table):
  * the K / V cache rows the prefill writes, within rel-L2 1e-2 of the oracle's per layer
    (a K element whose value lies within the accumulation-order difference of a bf16
    rounding boundary is stored one bf16 unit away; layer 1's rows inherit layer 0's);
  * a prefill in two chunks (start > 0) writes the same rows as one call (rel-L2 1e-5);
  * 16 teacher-forced device decode steps that continue from the device cache: the final
    normalised state within rel-L2 5e-3 of the oracle's, the token equal wherever the
    oracle's top-2 margin exceeds 0.05.
Unit QK-norm and value gains keep the attention soft, so that bf16 operand rounding is
not amplified past the tolerances by a few near-tie scores.
"""
import numpy as np
import pytest
import torch

import pyoracle
import smol_b200
from qkn_decoder_oracle import GEMMA2_SMALL, GEMMA_SHAPE, QknOracle

pytestmark = [pytest.mark.gpu, pytest.mark.new_on_gpu(stage=2)]

CASES = {"qwen3": (None, {}), "gemma2": ({**GEMMA2_SMALL, "sliding_window": 64}, GEMMA_SHAPE)}


def _dev(cuda):
    return lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(cuda)   # noqa: E731


def _model(m, t, keep):
    emb, fnorm, layers = m.device_weights(t)
    local = (t(m.cos_local), t(m.sin_local)) if m.has_local else (None, None)
    keep += [emb, fnorm, layers, local]
    return smol_b200.qkn_model(m.H, m.HQ, m.HKV, m.HD, m.I, m.V, m.eps, emb, fnorm, layers,
                               rope_interleaved=m.interleaved,
                               activation=smol_b200.ACT_GEGLU if m.gemma else smol_b200.ACT_SWIGLU,
                               embed_normalizer=float(m.embed_normalizer), attn_softcap=m.attn_softcap,
                               sliding_window=m.sliding_window, rope_cos_local=local[0], rope_sin_local=local[1],
                               sliding=m.sliding)


@pytest.mark.parametrize("case", list(CASES))
def test_device_prefill_then_decode(cuda, case):
    gemma, shape = CASES[case]
    cap, n_prompt, steps = 512, 300, 16
    m = QknOracle(layers=2, seed=31, qk_gain=1.0, vo_gain=1.0, cap=cap, gemma=gemma, **shape)
    rng = np.random.default_rng(31)
    prompt = rng.integers(0, m.V, n_prompt).astype(np.int32)
    feed = [int(prompt[-1])] + rng.integers(0, m.V, steps - 1).tolist()
    t = _dev(cuda)
    keep = []
    model = _model(m, t, keep)
    kvd = m.HKV * m.HD
    rows = m.L * cap
    row0 = np.array([l * cap for l in range(m.L)], np.int64)
    cos, sin = t(m.cos), t(m.sin)
    n = n_prompt - 1
    ws = torch.zeros(smol_b200.qkn_prefill_workspace_bytes(model, n), dtype=torch.uint8, device=cuda)

    def pools():
        return (torch.zeros((rows, kvd), dtype=torch.int16, device=cuda),
                torch.zeros((rows, kvd), dtype=torch.int16, device=cuda))

    # one call, and the same prompt in two chunks
    k_pool, v_pool = pools()
    smol_b200.qkn_prefill(model, t(prompt[:n]), n, 0, k_pool, v_pool, rows, row0, cos, sin, ws)
    k2, v2 = pools()
    smol_b200.qkn_prefill(model, t(prompt[:150]), 150, 0, k2, v2, rows, row0, cos, sin, ws)
    smol_b200.qkn_prefill(model, t(prompt[150:n]), n - 150, 150, k2, v2, rows, row0, cos, sin, ws)
    torch.cuda.synchronize()
    assert smol_b200.last_error() == 0 and smol_b200.device_error() == 0

    m.prefill(prompt[:n].tolist(), device_formats=True)
    kb = k_pool.cpu().numpy().view(np.uint16)
    vb = v_pool.cpu().numpy().view(np.uint16)
    for l in range(m.L):
        sl = slice(l * cap, l * cap + n)
        ek = pyoracle.rel_l2(pyoracle.bf16_to_f32(kb[sl]), pyoracle.bf16_to_f32(m.kc[l][:n]))
        ev = pyoracle.rel_l2(vb[sl].view(np.float16).astype(np.float32), m.vc[l][:n].view(np.float16).astype(np.float32))
        assert ek < 1e-2 and ev < 1e-2, (l, ek, ev)
    k2b, v2b = k2.cpu().numpy().view(np.uint16), v2.cpu().numpy().view(np.uint16)
    for l in range(m.L):
        sl = slice(l * cap, l * cap + n)
        assert pyoracle.rel_l2(pyoracle.bf16_to_f32(k2b[sl]), pyoracle.bf16_to_f32(kb[sl])) < 1e-5
        assert pyoracle.rel_l2(v2b[sl].view(np.float16).astype(np.float32),
                               vb[sl].view(np.float16).astype(np.float32)) < 1e-5

    # decode from the device cache
    row0_d = t(row0)
    kv_len = torch.tensor([n], dtype=torch.int32, device=cuda)
    sws = torch.zeros(smol_b200.qkn_step_workspace_bytes(model, 1, cap - 1), dtype=torch.uint8, device=cuda)
    tok_in = torch.zeros(1, dtype=torch.int32, device=cuda)
    tok_out = torch.zeros(1, dtype=torch.int32, device=cuda)
    xn_off = (m.H * 4 + 255) // 256 * 256
    checked, worst = 0, 0.0
    for s in range(steps):
        tok_in.fill_(feed[s])
        smol_b200.qkn_decode_step(model, 1, tok_in, tok_out, k_pool, v_pool, rows, row0_d, kv_len, cap - 1, cos, sin,
                                  sws, advance=True)
        want, margin, xf = m.forward(feed[s])
        torch.cuda.synchronize()
        assert smol_b200.last_error() == 0 and smol_b200.device_error() == 0
        err = pyoracle.rel_l2(sws[xn_off:xn_off + m.H * 4].view(torch.float32).cpu().numpy(), xf)
        worst = max(worst, err)
        assert err < 5e-3, (s, err)
        if margin > 0.05:
            checked += 1
            assert int(tok_out.item()) == want, (s, int(tok_out.item()), want, margin)
    assert checked >= steps // 2
    print(f"{case}: prefill {n} tokens, {steps} decode steps, worst hidden-state rel-L2 {worst:.2e}")
