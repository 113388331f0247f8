"""Device-resident decoder step (smol_b200.h Part 4) against the CPU restatement.

The oracle (oracle/qkn_decoder_oracle.py) restates qkn_decoder_prefill / _forward
(qkn_decoder.c:369-714) in fp32 numpy over a cache in the device formats, so both
sides attend over identical K/V values.  Checked:
  * the bf16 matrix-vector product in its three forms (store, residual add, SiLU-gated
    pairs) against fp32 numpy, for batches that need one and several launches;
  * the greedy argmax, including equal maxima (the lowest row wins, as the
    reference's strict '>' scan);
  * a 2-layer Qwen3-shaped decoder (hidden 1024, 16/8 heads, head_dim 128, SwiGLU
    3072, vocab 4096) teacher-forced for 48 steps: every step's final normed hidden
    state within rel-L2 1e-3 of the oracle's, and the same token wherever the oracle's
    top-2 margin exceeds 0.05;
  * the same decoder free-running for 128 greedy steps, the step captured once as a
    CUDA graph and replayed: the 128 tokens equal the oracle's.
"""
import numpy as np
import pytest
import torch

import pyoracle
import smol_b200
from qkn_decoder_oracle import QknOracle, swiglu

pytestmark = pytest.mark.gpu


def _dev(cuda):
    return lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(cuda)   # noqa: E731


@pytest.mark.parametrize("n_out,k_dim,nb", [(1024, 1024, 1), (3072, 1024, 3), (1000, 136, 8), (512, 3072, 11)])
def test_gemv_bf16_modes(cuda, n_out, k_dim, nb):
    rng = np.random.default_rng(n_out + k_dim + nb)
    t = _dev(cuda)
    X = rng.standard_normal((nb, k_dim)).astype(np.float32)
    for mode in (0, 1, 2):
        rows = 2 * n_out if mode == 2 else n_out
        W = pyoracle.round_bf16((rng.standard_normal((rows, k_dim)) / np.sqrt(k_dim)).astype(np.float32))
        y0 = rng.standard_normal((nb, n_out)).astype(np.float32)
        y = t(y0)
        smol_b200.gemv_bf16(y, n_out, t(X), k_dim, t(pyoracle.bf16_bits(W)), n_out, k_dim, nb, mode)
        torch.cuda.synchronize()
        s = (X.astype(np.float64) @ W.T.astype(np.float64)).astype(np.float32)
        want = s if mode == 0 else (y0 + s if mode == 1 else swiglu(s))
        got = y.cpu().numpy()
        assert smol_b200.last_error() == 0
        assert pyoracle.rel_l2(got, want) < 1e-5, (mode, pyoracle.rel_l2(got, want))


def test_argmax_bf16_lowest_index_on_ties(cuda):
    rng = np.random.default_rng(7)
    t = _dev(cuda)
    V, H, nb = 5000, 1024, 3
    E = pyoracle.round_bf16(rng.standard_normal((V, H)).astype(np.float32))
    targets = [4321, 17, 2999]
    E[4322] = E[4321]          # equal maxima: rows 4321 and 4322, and 17 / 4000
    E[4000] = E[17]
    X = np.stack([E[t_] * 3 + 0.01 * rng.standard_normal(H).astype(np.float32) for t_ in targets]).astype(np.float32)
    out = torch.full((nb,), -1, dtype=torch.int32, device=cuda)
    ws = torch.empty(smol_b200.argmax_workspace_bytes(nb, V), dtype=torch.uint8, device=cuda)
    smol_b200.argmax_bf16(out, t(X), H, t(pyoracle.bf16_bits(E)), V, H, nb, ws)
    torch.cuda.synchronize()
    assert out.cpu().tolist() == targets
    want = [int(np.argmax(E @ x)) for x in X]
    assert want == targets


def _setup(m: QknOracle, cuda, prompt):
    """Oracle prefill of prompt[:-1]; the device pool gets the same cache rows."""
    t = _dev(cuda)
    m.prefill(prompt[:-1])
    emb, fnorm, layers = m.device_weights(t)
    model = smol_b200.qkn_model(m.H, m.HQ, m.HKV, m.HD, m.I, m.V, m.eps, emb, fnorm, layers)
    kvd = m.HKV * m.HD
    k_pool = torch.zeros((m.L * m.cap, kvd), dtype=torch.int16, device=cuda)
    v_pool = torch.zeros((m.L * m.cap, kvd), dtype=torch.int16, device=cuda)
    for l in range(m.L):
        k_pool[l * m.cap:(l + 1) * m.cap] = torch.from_numpy(m.kc[l].view(np.int16)).to(cuda)
        v_pool[l * m.cap:(l + 1) * m.cap] = torch.from_numpy(m.vc[l].view(np.int16)).to(cuda)
    row0 = torch.tensor([l * m.cap for l in range(m.L)], dtype=torch.int64, device=cuda)   # [layer][seq]
    kv_len = torch.tensor([m.len], dtype=torch.int32, device=cuda)
    ws = torch.zeros(smol_b200.qkn_step_workspace_bytes(model, 1, m.cap - 1), dtype=torch.uint8, device=cuda)
    keep = (emb, fnorm, layers)
    return dict(model=model, k_pool=k_pool, v_pool=v_pool, row0=row0, kv_len=kv_len, ws=ws, cos=t(m.cos),
                sin=t(m.sin), keep=keep)


def _step(m, d, tok_in, tok_out):
    smol_b200.qkn_decode_step(d["model"], 1, tok_in, tok_out, d["k_pool"], d["v_pool"], m.L * m.cap, d["row0"],
                              d["kv_len"], m.cap - 1, d["cos"], d["sin"], d["ws"], advance=True)


def test_decoder_step_teacher_forced(cuda):
    m = QknOracle(layers=2, seed=0, qk_gain=3.0, vo_gain=4.0, cap=1024)
    prompt = np.random.default_rng(100).integers(0, m.V, 512)
    d = _setup(m, cuda, prompt)
    tok_in = torch.zeros(1, dtype=torch.int32, device=cuda)
    tok_out = torch.zeros(1, dtype=torch.int32, device=cuda)
    feed = int(prompt[-1])
    checked, worst = 0, 0.0
    for step in range(48):
        tok_in.fill_(feed)
        _step(m, d, tok_in, tok_out)
        want, margin, xf = m.forward(feed)
        torch.cuda.synchronize()
        assert smol_b200.last_error() == 0 and smol_b200.device_error() == 0
        # final normed hidden state: the workspace's second piece (after x, 256-byte aligned)
        x_dev = d["ws"][m.H * 4:2 * m.H * 4].view(torch.float32).cpu().numpy()
        err = pyoracle.rel_l2(x_dev, xf)
        worst = max(worst, err)
        assert err < 1e-3, (step, err)
        if margin > 0.05:
            checked += 1
            assert int(tok_out.item()) == want, (step, int(tok_out.item()), want, margin)
        feed = want                                # teacher forcing: both continue from the oracle's token
    assert int(d["kv_len"].item()) == 511 + 48
    assert checked >= 40
    print(f"48 teacher-forced steps: worst hidden-state rel-L2 {worst:.2e}; tokens equal on {checked} clear steps")


def test_decoder_greedy_128_in_cuda_graph(cuda):
    m = QknOracle(layers=2, seed=3, qk_gain=3.0, vo_gain=4.0, cap=1024)
    prompt = np.random.default_rng(103).integers(0, m.V, 512)
    d = _setup(m, cuda, prompt)
    # oracle: free-running greedy
    want, margins, tok = [], [], int(prompt[-1])
    for _ in range(128):
        tok, mg, _ = m.forward(tok)
        want.append(tok)
        margins.append(mg)
    # device: the first step eagerly (one-time set-up), the rest as graph replays
    tokens = torch.tensor([int(prompt[-1])], dtype=torch.int32, device=cuda)
    got = []
    _step(m, d, tokens, tokens)
    torch.cuda.synchronize()
    got.append(int(tokens.item()))
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=side):
        _step(m, d, tokens, tokens)
    for _ in range(127):
        graph.replay()
        got.append(int(tokens.item()))
    assert smol_b200.last_error() == 0 and smol_b200.device_error() == 0
    assert int(d["kv_len"].item()) == 511 + 128
    assert len(set(want)) >= 32
    first = next((i for i, (a, b) in enumerate(zip(want, got)) if a != b), None)
    assert got == want, f"diverged at step {first} (oracle margin {margins[first]:.4f})"
    print(f"128 greedy tokens identical in a CUDA graph ({len(set(want))} distinct, min margin {min(margins):.3f})")


def test_decoder_step_batched_ragged(cuda):
    """10 sequences (two launches of the 8-sequence projections) with prompts of 40-130
    tokens, one layer, teacher-forced for 6 steps: per sequence the final normalised
    state matches the oracle's and the token matches wherever the margin is clear."""
    n, cap = 10, 256
    lens = [40 + 10 * i for i in range(n)]
    oracles = [QknOracle(layers=1, seed=5, qk_gain=3.0, vo_gain=4.0, cap=cap) for _ in range(n)]
    prompts = [np.random.default_rng(200 + i).integers(0, oracles[0].V, lens[i]) for i in range(n)]
    t = _dev(cuda)
    for o, pr in zip(oracles, prompts):
        o.prefill(pr[:-1])
    m = oracles[0]
    emb, fnorm, layers = m.device_weights(t)
    model = smol_b200.qkn_model(m.H, m.HQ, m.HKV, m.HD, m.I, m.V, m.eps, emb, fnorm, layers)
    kvd = m.HKV * m.HD
    k_pool = torch.zeros((n * cap, kvd), dtype=torch.int16, device=cuda)
    v_pool = torch.zeros((n * cap, kvd), dtype=torch.int16, device=cuda)
    for b, o in enumerate(oracles):
        k_pool[b * cap:(b + 1) * cap] = torch.from_numpy(o.kc[0].view(np.int16)).to(cuda)
        v_pool[b * cap:(b + 1) * cap] = torch.from_numpy(o.vc[0].view(np.int16)).to(cuda)
    row0 = torch.arange(n, dtype=torch.int64, device=cuda) * cap          # [layer 0][seq]
    kv_len = torch.tensor([o.len for o in oracles], dtype=torch.int32, device=cuda)
    ws = torch.zeros(smol_b200.qkn_step_workspace_bytes(model, n, cap - 1), dtype=torch.uint8, device=cuda)
    feed = [int(pr[-1]) for pr in prompts]
    tok_in = torch.zeros(n, dtype=torch.int32, device=cuda)
    tok_out = torch.zeros(n, dtype=torch.int32, device=cuda)
    checked, worst = 0, 0.0
    xn_off = (n * m.H * 4 + 255) // 256 * 256          # second workspace piece: the normalised state
    for step in range(6):
        tok_in.copy_(torch.tensor(feed, dtype=torch.int32))
        smol_b200.qkn_decode_step(model, n, tok_in, tok_out, k_pool, v_pool, n * cap, row0, kv_len, cap - 1,
                                  t(m.cos), t(m.sin), ws, advance=True)
        outs = [o.forward(f) for o, f in zip(oracles, feed)]
        torch.cuda.synchronize()
        assert smol_b200.last_error() == 0 and smol_b200.device_error() == 0
        x_dev = ws[xn_off:xn_off + n * m.H * 4].view(torch.float32).cpu().numpy().reshape(n, m.H)
        got = tok_out.cpu().tolist()
        for b, (want, margin, xf) in enumerate(outs):
            err = pyoracle.rel_l2(x_dev[b], xf)
            worst = max(worst, err)
            assert err < 1e-3, (step, b, err)
            if margin > 0.05:
                checked += 1
                assert got[b] == want, (step, b, got[b], want, margin)
        feed = [w for w, _, _ in outs]
    assert kv_len.cpu().tolist() == [L - 1 + 6 for L in lens]
    assert checked >= 40
    print(f"10 ragged sequences x 6 steps: worst hidden-state rel-L2 {worst:.2e}; {checked} clear tokens equal")
