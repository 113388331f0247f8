"""Device-resident decoder step (smol_b200.h Part 4) in the Gemma configuration.

The configuration the exports set for Gemma decoders (paligemma.c:206-230): embedding
scale, interleaved RoPE, GeGLU, a norm on each sublayer's output before its residual
add (qkn_decoder.c:681-704), attention softcap, sliding-window layers with their own
RoPE tables, QK-norm optional.  The oracle (oracle/qkn_decoder_oracle.py, pinned to
the reference decoder on the same settings by tests/test_decoder_oracle_e2e.py)
prefills the prompt and the device pool gets its cache rows; then both sides run the
same teacher-forced steps.  Checked:
  * the GELU-tanh-gated matrix-vector product (mode 3) against fp32 numpy, and the
    product with a 16384-wide input (fewer sequences per launch);
  * 2-layer Gemma 2 / Gemma 3 style decoders (MQA 8/1, head dim 256, one sliding layer
    with a 64-token window over a 300-token prompt), and SmolVLM's decoder (MHA with head
    dim 64, no QK-norm, an untied lm_head): every step's final normalised state within
    rel-L2 1e-3 of the oracle's and the same token wherever the oracle's top-2 margin
    exceeds 0.05.
"""
import numpy as np
import pytest
import torch

import pyoracle
import smol_b200
from qkn_decoder_oracle import GEMMA2_SMALL, GEMMA3_SMALL, GEMMA_SHAPE, SMOLVLM_SHAPE, QknOracle, geglu

pytestmark = [pytest.mark.gpu, pytest.mark.new_on_gpu]

# the pinned Gemma settings with a window that binds over a 300-token prompt
GEMMA2 = {**GEMMA2_SMALL, "sliding_window": 64}
GEMMA3 = {**GEMMA3_SMALL, "sliding_window": 64}


def _dev(cuda):
    return lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(cuda)   # noqa: E731


@pytest.mark.parametrize("n_out,k_dim,nb", [(1024, 1024, 1), (2048, 1024, 3), (512, 3072, 11)])
def test_gemv_bf16_geglu(cuda, n_out, k_dim, nb):
    rng = np.random.default_rng(n_out + k_dim + nb)
    t = _dev(cuda)
    X = rng.standard_normal((nb, k_dim)).astype(np.float32)
    W = pyoracle.round_bf16((rng.standard_normal((2 * n_out, k_dim)) / np.sqrt(k_dim)).astype(np.float32))
    y = torch.zeros((nb, n_out), device=cuda)
    smol_b200.gemv_bf16(y, n_out, t(X), k_dim, t(pyoracle.bf16_bits(W)), n_out, k_dim, nb, 3)
    torch.cuda.synchronize()
    assert smol_b200.last_error() == 0
    want = geglu((X.astype(np.float64) @ W.T.astype(np.float64)).astype(np.float32))
    assert pyoracle.rel_l2(y.cpu().numpy(), want) < 1e-5


@pytest.mark.parametrize("nb", [1, 3, 5])
def test_gemv_bf16_wide_k(cuda, nb):
    """A 16384-wide input (Gemma 2B's down projection): fewer sequences per launch, so
    the staged activations still fit shared memory."""
    rng = np.random.default_rng(40 + nb)
    t = _dev(cuda)
    n_out, k_dim = 512, 16384
    X = rng.standard_normal((nb, k_dim)).astype(np.float32)
    W = pyoracle.round_bf16((rng.standard_normal((n_out, k_dim)) / np.sqrt(k_dim)).astype(np.float32))
    y0 = rng.standard_normal((nb, n_out)).astype(np.float32)
    y = t(y0)
    smol_b200.gemv_bf16(y, n_out, t(X), k_dim, t(pyoracle.bf16_bits(W)), n_out, k_dim, nb, 1)
    torch.cuda.synchronize()
    assert smol_b200.last_error() == 0
    want = y0 + (X.astype(np.float64) @ W.T.astype(np.float64)).astype(np.float32)
    assert pyoracle.rel_l2(y.cpu().numpy(), want) < 1e-5


@pytest.mark.parametrize("gemma,seed", [(GEMMA2, 21), (GEMMA3, 22)], ids=["gemma2", "gemma3"])
def test_gemma_decoder_step_teacher_forced(cuda, gemma, seed):
    cap, steps = 512, 32
    m = QknOracle(layers=2, seed=seed, qk_gain=3.0, vo_gain=4.0, cap=cap, gemma=gemma, **GEMMA_SHAPE)
    rng = np.random.default_rng(seed)
    prompt = rng.integers(0, m.V, 300)
    feed = [int(prompt[-1])] + rng.integers(0, m.V, steps - 1).tolist()
    t = _dev(cuda)
    m.prefill(prompt[:-1])
    emb, fnorm, layers = m.device_weights(t)
    local = (t(m.cos_local), t(m.sin_local)) if m.has_local else (None, None)
    model = smol_b200.qkn_model(m.H, m.HQ, m.HKV, m.HD, m.I, m.V, m.eps, emb, fnorm, layers,
                                rope_interleaved=m.interleaved, activation=smol_b200.ACT_GEGLU,
                                embed_normalizer=float(m.embed_normalizer), attn_softcap=m.attn_softcap,
                                sliding_window=m.sliding_window, rope_cos_local=local[0], rope_sin_local=local[1],
                                sliding=m.sliding)
    kvd = m.HKV * m.HD
    k_pool = torch.zeros((m.L * cap, kvd), dtype=torch.int16, device=cuda)
    v_pool = torch.zeros((m.L * cap, kvd), dtype=torch.int16, device=cuda)
    for l in range(m.L):
        k_pool[l * cap:(l + 1) * cap] = torch.from_numpy(m.kc[l].view(np.int16)).to(cuda)
        v_pool[l * cap:(l + 1) * cap] = torch.from_numpy(m.vc[l].view(np.int16)).to(cuda)
    row0 = torch.tensor([l * cap for l in range(m.L)], dtype=torch.int64, device=cuda)   # [layer][seq]
    kv_len = torch.tensor([m.len], dtype=torch.int32, device=cuda)
    ws = torch.zeros(smol_b200.qkn_step_workspace_bytes(model, 1, cap - 1), dtype=torch.uint8, device=cuda)
    cos, sin = t(m.cos), t(m.sin)
    tok_in = torch.zeros(1, dtype=torch.int32, device=cuda)
    tok_out = torch.zeros(1, dtype=torch.int32, device=cuda)
    xn_off = (m.H * 4 + 255) // 256 * 256              # second workspace piece: the normalised state
    checked, worst = 0, 0.0
    for s in range(steps):
        tok_in.fill_(feed[s])
        smol_b200.qkn_decode_step(model, 1, tok_in, tok_out, k_pool, v_pool, m.L * cap, row0, kv_len, cap - 1, cos,
                                  sin, ws, advance=True)
        want, margin, xf = m.forward(feed[s])
        torch.cuda.synchronize()
        assert smol_b200.last_error() == 0 and smol_b200.device_error() == 0
        x_dev = ws[xn_off:xn_off + m.H * 4].view(torch.float32).cpu().numpy()
        err = pyoracle.rel_l2(x_dev, xf)
        worst = max(worst, err)
        assert err < 1e-3, (s, err)
        if margin > 0.05:
            checked += 1
            assert int(tok_out.item()) == want, (s, int(tok_out.item()), want, margin)
    assert int(kv_len.item()) == 299 + steps
    assert checked >= steps // 2
    print(f"{steps} teacher-forced Gemma steps: worst hidden-state rel-L2 {worst:.2e}; {checked} clear tokens equal")


def test_smolvlm_decoder_step_teacher_forced(cuda):
    """SmolVLM's decoder (exports/smolvlm/decoder.c:391-476): the Qwen3 step without
    QK-norm, greedy over an untied lm_head."""
    cap, steps = 512, 32
    m = QknOracle(layers=2, seed=23, qk_gain=3.0, vo_gain=4.0, cap=cap, **SMOLVLM_SHAPE)
    rng = np.random.default_rng(23)
    prompt = rng.integers(0, m.V, 300)
    feed = [int(prompt[-1])] + rng.integers(0, m.V, steps - 1).tolist()
    t = _dev(cuda)
    m.prefill(prompt[:-1])
    emb, fnorm, layers = m.device_weights(t)
    head = t(pyoracle.bf16_bits(m.lm_head))
    model = smol_b200.qkn_model(m.H, m.HQ, m.HKV, m.HD, m.I, m.V, m.eps, emb, fnorm, layers, lm_head=head)
    kvd = m.HKV * m.HD
    k_pool = torch.zeros((m.L * cap, kvd), dtype=torch.int16, device=cuda)
    v_pool = torch.zeros((m.L * cap, kvd), dtype=torch.int16, device=cuda)
    for l in range(m.L):
        k_pool[l * cap:(l + 1) * cap] = torch.from_numpy(m.kc[l].view(np.int16)).to(cuda)
        v_pool[l * cap:(l + 1) * cap] = torch.from_numpy(m.vc[l].view(np.int16)).to(cuda)
    row0 = torch.tensor([l * cap for l in range(m.L)], dtype=torch.int64, device=cuda)
    kv_len = torch.tensor([m.len], dtype=torch.int32, device=cuda)
    ws = torch.zeros(smol_b200.qkn_step_workspace_bytes(model, 1, cap - 1), dtype=torch.uint8, device=cuda)
    cos, sin = t(m.cos), t(m.sin)
    tok_in = torch.zeros(1, dtype=torch.int32, device=cuda)
    tok_out = torch.zeros(1, dtype=torch.int32, device=cuda)
    xn_off = (m.H * 4 + 255) // 256 * 256
    checked = 0
    for s in range(steps):
        tok_in.fill_(feed[s])
        smol_b200.qkn_decode_step(model, 1, tok_in, tok_out, k_pool, v_pool, m.L * cap, row0, kv_len, cap - 1, cos,
                                  sin, ws, advance=True)
        want, margin, xf = m.forward(feed[s])
        torch.cuda.synchronize()
        assert smol_b200.last_error() == 0 and smol_b200.device_error() == 0
        err = pyoracle.rel_l2(ws[xn_off:xn_off + m.H * 4].view(torch.float32).cpu().numpy(), xf)
        assert err < 1e-3, (s, err)
        if margin > 0.05:
            checked += 1
            assert int(tok_out.item()) == want, (s, int(tok_out.item()), want, margin)
    assert checked >= steps // 2
