"""Bounded waits on the GPU: a wait that can never succeed must end with an error
status the host can read, and leave the CUDA context usable.

smol_b200_watchdog_selftest launches one kernel that waits on an mbarrier nothing
arrives on (the same bounded wait every pipeline of the library uses).  No fault,
trap or hang is involved: the wait gives up after ~2 s and the kernel returns.
"""
import time

import numpy as np
import pytest
import torch

import smol_b200

pytestmark = pytest.mark.gpu


def test_wait_that_never_completes_reports_and_recovers(cuda):
    smol_b200.clear_error()
    t0 = time.time()
    assert smol_b200.watchdog_selftest() == 0
    word = smol_b200.device_error()          # synchronises the device
    elapsed = time.time() - t0
    assert word & 1, f"device error word {word:#x}"
    assert 1.0 < elapsed < 30.0
    smol_b200.clear_error()
    assert smol_b200.device_error() == 0
    # the context is still usable: a decode call runs and is correct
    hq, hkv, hd = 4, 2, 128
    L = 100
    g = torch.Generator(device=cuda).manual_seed(0)
    kp = torch.randn((L, hkv * hd), device=cuda, generator=g).to(torch.bfloat16)
    vp = torch.ones((L, hkv * hd), device=cuda, dtype=torch.float16)
    q = torch.randn((1, hq * hd), device=cuda, generator=g)
    out = torch.zeros((1, hq * hd), device=cuda)
    ws = torch.empty(smol_b200.decode_workspace_bytes(1, L, hq, hkv, hd), dtype=torch.uint8, device=cuda)
    smol_b200.decode_attention(out, q, kp, vp, L, torch.zeros(1, dtype=torch.int64, device=cuda),
                               torch.full((1,), L, dtype=torch.int32, device=cuda), 1, L, hq, hkv, hd, 0.1, ws)
    torch.cuda.synchronize()
    assert np.allclose(out.cpu().numpy(), 1.0, atol=1e-3)   # V rows of ones -> output of ones
    assert smol_b200.device_error() == 0 and smol_b200.last_error() == 0
