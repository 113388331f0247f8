"""Greedy decode parity over 128 steps (BASELINE cfg 1 shape).

A one-layer Qwen3-0.6B-shaped attention decoder with seeded synthetic weights
(hidden 1024, 16 Q / 8 KV heads, head_dim 128, per-head RMSNorm eps 1e-6, NeoX
RoPE theta 1e6, tied embeddings): a 512-token prefill, then 129 greedy tokens.
The QK-norm weights are ~N(3,0.02) and Wv / Wo carry a gain of 4 so that attention
is sharp and its read-out, not the token's own embedding, decides the next token:
with unit gains the stream is one token repeated, which would prove nothing.  With
these weights the 129 tokens take ~88 distinct values and the test asserts at
least 32.  The projections, residual, final norm and argmax run in
numpy for both sides from the same fp32 values, so the only difference between the
two runs is the hot path: on one side libsmol_b200 (fused QK-norm + RoPE + cache
append, tcgen05 prefill, split-KV decode through smol_b200_decode_step_host), on the
other the oracle restatement of qkn_decoder.c:488-528 / :642-677 over a cache holding
the same bf16 K / fp16 V values.  The generated tokens must be identical; the
smallest top-1/top-2 logit margin is reported.
"""
import numpy as np
import pytest
import torch

import pyoracle
import smol_b200

pytestmark = pytest.mark.gpu

H, HQ, HKV, HD, VOCAB = 1024, 16, 8, 128, 4096
PREFILL, STEPS = 512, 129
QK_GAIN, VO_GAIN = 3.0, 4.0


def rms_norm(x, w, eps=1e-6):
    return x / np.sqrt(np.mean(x.astype(np.float64) ** 2, axis=-1, keepdims=True) + eps).astype(np.float32) * w


class Model:
    def __init__(self, seed=0):
        rng = np.random.default_rng(seed)
        bf = lambda *s, sc=1.0: pyoracle.round_bf16((rng.standard_normal(s) * sc).astype(np.float32))  # noqa: E731
        self.E = bf(VOCAB, H)
        self.Wq = bf(HQ * HD, H, sc=1 / np.sqrt(H))
        self.Wk = bf(HKV * HD, H, sc=1 / np.sqrt(H))
        self.Wv = bf(HKV * HD, H, sc=VO_GAIN / np.sqrt(H))
        self.Wo = bf(H, HQ * HD, sc=VO_GAIN / np.sqrt(HQ * HD))
        self.qn = (QK_GAIN + 0.02 * rng.standard_normal(HD)).astype(np.float32)
        self.kn = (QK_GAIN + 0.02 * rng.standard_normal(HD)).astype(np.float32)
        self.norm = (1 + 0.02 * rng.standard_normal(H)).astype(np.float32)
        self.prompt = rng.integers(0, VOCAB, size=PREFILL)

    def qkv(self, x):
        return x @ self.Wq.T, x @ self.Wk.T, x @ self.Wv.T

    def next_token(self, x_last, attn_last):
        h = x_last + attn_last @ self.Wo.T
        logits = self.E @ rms_norm(h, self.norm)
        top = np.argsort(logits)[-2:]
        return int(top[-1]), float(logits[top[-1]] - logits[top[-2]])


def test_greedy_tokens_identical_over_128_steps(cuda):
    m = Model(0)
    scale = 1 / np.sqrt(HD)
    cap = PREFILL + STEPS + 8
    cos_t, sin_t = pyoracle.fill_rope_table(cap, HD, 1e6)
    kv_dim = HKV * HD

    # ---------------- oracle ----------------
    ok_cache = np.zeros((cap, kv_dim), np.uint16)
    ov_cache = np.zeros((cap, kv_dim), np.uint16)
    o = pyoracle.oracle()

    def oracle_attend(q_rot, L, q_offset, n):
        K = pyoracle.bf16_to_f32(ok_cache[:L])
        V = ov_cache[:L].view(np.float16).astype(np.float32)
        return o.causal_attention(q_rot, K, V, n, L, HQ, HKV, HD, scale, q_offset)

    # ---------------- device ----------------
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(cuda)  # noqa: E731
    kp = torch.zeros((cap, kv_dim), dtype=torch.bfloat16, device=cuda)
    vp = torch.zeros((cap, kv_dim), dtype=torch.float16, device=cuda)
    dcos, dsin, dqn, dkn = t(cos_t), t(sin_t), t(m.qn), t(m.kn)
    row0 = torch.zeros(1, dtype=torch.int64, device=cuda)
    scratch = torch.empty(smol_b200.decode_step_scratch_bytes(1, cap, HQ, HKV, HD), dtype=torch.uint8, device=cuda)

    # prefill (identical fp32 projections on both sides)
    x = m.E[m.prompt]
    q, k, v = m.qkv(x)
    pos = np.arange(PREFILL, dtype=np.int32)
    q_rot = pyoracle.qknorm_rope_append(q, k, v, HQ, HKV, HD, m.qn, m.kn, 1e-6, cos_t, sin_t, False, pos,
                                        pos.astype(np.int64), ok_cache, ov_cache)
    attn_o = oracle_attend(q_rot, PREFILL, 0, PREFILL)

    qb = torch.zeros((PREFILL, HQ * HD), dtype=torch.bfloat16, device=cuda)
    smol_b200.qknorm_rope_append(t(q), t(k), t(v), PREFILL, HQ, HKV, HD, dqn, dkn, 1e-6, dcos, dsin, False, t(pos),
                                 t(pos.astype(np.int64)), None, qb, kp, vp, cap)
    out = torch.zeros((1, PREFILL, HQ * HD), device=cuda)
    smol_b200.prefill_attention(out, qb, kp, vp, 1, PREFILL, PREFILL, HQ, HKV, HD, scale,
                                strides=((HQ * HD, 0), (HQ * HD, 0), (kv_dim, 0), (kv_dim, 0)))
    torch.cuda.synchronize()
    attn_d = out[0].cpu().numpy()
    # The tensor-core prefill takes Q in bf16.  Against the oracle fed the same bf16 Q
    # the kernel meets the parity bar; against the unrounded fp32 Q of the reference the
    # layer output moves ~5e-3 (rel-L2) with these sharp QK-norm gains, which the token
    # stream below absorbs (the first token's top-2 margin is 1.3, the shift 0.17).
    attn_ob = oracle_attend(pyoracle.round_bf16(q_rot), PREFILL, 0, PREFILL)
    assert pyoracle.rel_l2(attn_d, attn_ob) < 1e-3
    assert pyoracle.rel_l2(attn_d, attn_o) < 1e-2

    tok_o, marg = m.next_token(x[-1], attn_o[-1])
    tok_d, _ = m.next_token(x[-1], attn_d[-1])
    toks_o, toks_d, margins = [tok_o], [tok_d], [marg]
    out_h = np.zeros((1, HQ * HD), np.float32)
    for step in range(STEPS - 1):
        L = PREFILL + step          # tokens already cached
        # oracle step
        xo = m.E[toks_o[-1]][None]
        qo, ko, vo = m.qkv(xo)
        qr = pyoracle.qknorm_rope_append(qo, ko, vo, HQ, HKV, HD, m.qn, m.kn, 1e-6, cos_t, sin_t, False,
                                         np.array([L], np.int32), np.array([L], np.int64), ok_cache, ov_cache)
        ao = oracle_attend(qr, L + 1, L, 1)
        # device step: host buffers in and out through the C ABI
        xd = m.E[toks_d[-1]][None]
        qd, kd, vd = (np.ascontiguousarray(a, np.float32) for a in m.qkv(xd))
        smol_b200.decode_step_host(out_h, qd, kd, vd, 1, HQ, HKV, HD, dqn, dkn, 1e-6, dcos, dsin, False, kp, vp, cap,
                                   row0, torch.tensor([L], dtype=torch.int32, device=cuda), cap, scale, scratch)
        tok, marg = m.next_token(xo[0], ao[0])
        toks_o.append(tok)
        margins.append(marg)
        toks_d.append(m.next_token(xd[0], out_h[0])[0])
        if toks_d[-1] != toks_o[-1]:
            break
    assert smol_b200.last_error() == 0
    assert len(toks_o) == STEPS
    assert toks_d == toks_o, (f"diverged at step {len(toks_o) - 1}: device {toks_d[-1]} vs oracle {toks_o[-1]}, "
                              f"oracle top-2 margin {margins[-1]:.4f}")
    assert len(set(toks_o)) >= 32, f"degenerate token stream: {len(set(toks_o))} distinct tokens"
    print(f"129 greedy tokens identical ({len(set(toks_o))} distinct); smallest top-1/top-2 margin {min(margins):.4f}")
