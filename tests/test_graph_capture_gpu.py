"""The device API under CUDA-graph capture.

Every Part-3 entry point is asynchronous on the caller's stream (no host
synchronisation, no allocation after the first call), so a decode loop can be
captured once and replayed.  The replay must produce bit-identical results to the
eager calls: same kernels, same launch shapes, deterministic reductions.
"""
import numpy as np
import pytest
import torch

import smol_b200

pytestmark = pytest.mark.gpu


def test_decode_loop_graph_replay_matches_eager(cuda):
    hq, hkv, hd, P, T = 16, 8, 128, 300, 12
    cap = P + T + 8
    kv = hkv * hd
    g = torch.Generator(device=cuda).manual_seed(5)
    cos_h = np.zeros((cap, hd), np.float32)
    sin_h = np.zeros((cap, hd), np.float32)
    smol_b200.compute_rope(cos_h, sin_h, np.arange(cap, dtype=np.int32), cap, hd, 1e6)
    dc, ds = torch.from_numpy(cos_h).to(cuda), torch.from_numpy(sin_h).to(cuda)
    qn = 1 + 0.02 * torch.randn(hd, device=cuda, generator=g)
    kn = 1 + 0.02 * torch.randn(hd, device=cuda, generator=g)
    init_k = torch.randn((cap, kv), device=cuda, generator=g).to(torch.bfloat16)
    init_v = torch.randn((cap, kv), device=cuda, generator=g).to(torch.float16)
    qs = torch.randn((T, 1, hq * hd), device=cuda, generator=g)
    ks = torch.randn((T, 1, kv), device=cuda, generator=g)
    vs = torch.randn((T, 1, kv), device=cuda, generator=g)
    lens = [torch.tensor([P + t], dtype=torch.int32, device=cuda) for t in range(T)]
    lens1 = [torch.tensor([P + t + 1], dtype=torch.int32, device=cuda) for t in range(T)]
    slots = [x.to(torch.int64) for x in lens]
    r0 = torch.zeros(1, dtype=torch.int64, device=cuda)
    ws = torch.empty(smol_b200.decode_workspace_bytes(1, cap, hq, hkv, hd), dtype=torch.uint8, device=cuda)

    def make_state():
        return init_k.clone(), init_v.clone(), torch.empty((1, hq * hd), device=cuda), \
            torch.zeros((T, 1, hq * hd), device=cuda)

    def loop(kp, vp, qr, outs):
        for t in range(T):
            smol_b200.qknorm_rope_append(qs[t], ks[t], vs[t], 1, hq, hkv, hd, qn, kn, 1e-6, dc, ds, False, lens[t],
                                         slots[t], qr, None, kp, vp, cap)
            smol_b200.decode_attention(outs[t], qr, kp, vp, cap, r0, lens1[t], 1, cap, hq, hkv, hd, hd ** -0.5, ws)

    eager = make_state()
    loop(*eager)
    torch.cuda.synchronize()

    graphed = make_state()
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        loop(*make_state())                  # warm-up outside the capture
    torch.cuda.current_stream().wait_stream(side)
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        loop(*graphed)
    graph.replay()
    torch.cuda.synchronize()
    assert smol_b200.last_error() == 0 and smol_b200.device_error() == 0
    assert torch.equal(graphed[3], eager[3])
    assert torch.equal(graphed[0], eager[0]) and torch.equal(graphed[1], eager[1])
    assert graphed[3].abs().sum() > 0
