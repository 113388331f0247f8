"""The allocation-free decode entry point (smol_b200_decode_attention_noalloc).

Some callers cannot call cudaMalloc -- a plugin inside another framework's memory
manager that owns all device memory, or a serving loop that must not allocate
after start-up -- so this entry point keeps its split-KV partial results in a fixed
16 MiB device array inside the library instead of a caller workspace.  These
tests call it through the C ABI first (before anything else in this file touches
the library, so a fresh process exercises its one-time set-up), check two calls in
a row against smol_b200_decode_attention on the same inputs, and check that a
batch too large for the array is refused with a clear error.

The file is named to be collected last: if it fails, a run that stops at the first
failure has already run every other test.
"""
import numpy as np
import pytest
import torch

import smol_b200
from conftest import assert_close

pytestmark = pytest.mark.gpu


def make_batch(cuda, seed, n, lo, hi, hq, hkv, hd):
    rng = np.random.default_rng(seed)
    lens = rng.integers(lo, hi + 1, size=n).astype(np.int32)
    row0 = np.concatenate([[0], np.cumsum(lens + 2)[:-1]]).astype(np.int64)
    rows = int(row0[-1] + lens[-1] + 2)
    g = torch.Generator(device=cuda).manual_seed(seed)
    kp = torch.randn((rows, hkv * hd), device=cuda, generator=g).to(torch.bfloat16)
    vp = torch.randn((rows, hkv * hd), device=cuda, generator=g).to(torch.float16)
    q = torch.randn((n, hq * hd), device=cuda, generator=g)
    return dict(q=q, kp=kp, vp=vp, rows=rows, r0=torch.from_numpy(row0).to(cuda), kl=torch.from_numpy(lens).to(cuda),
                n=n, max_len=int(lens.max()))


def test_noalloc_matches_workspace_entry_point_on_two_calls(cuda):
    hq, hkv, hd = 16, 8, 128
    first = make_batch(cuda, 1, 96, 1, 8192, hq, hkv, hd)
    second = make_batch(cuda, 2, 40, 1, 3000, hq, hkv, hd)   # smaller: stale partials of call 1 stay behind
    outs = []
    for b in (first, second):   # the allocation-free calls come first, back to back
        out = torch.full((b["n"], hq * hd), 7.0, device=cuda)
        rc = smol_b200.decode_attention_noalloc(out, b["q"], b["kp"], b["vp"], b["rows"], b["r0"], b["kl"], b["n"],
                                                b["max_len"], hq, hkv, hd, 1 / np.sqrt(hd))
        assert rc == 0, smol_b200.lib().smol_cuda_error_string(rc)
        outs.append(out)
    torch.cuda.synchronize()
    for b, out in zip((first, second), outs):
        ref = torch.zeros_like(out)
        ws = torch.empty(smol_b200.decode_workspace_bytes(b["n"], b["max_len"], hq, hkv, hd), dtype=torch.uint8,
                         device=cuda)
        smol_b200.decode_attention(ref, b["q"], b["kp"], b["vp"], b["rows"], b["r0"], b["kl"], b["n"], b["max_len"],
                                   hq, hkv, hd, 1 / np.sqrt(hd), ws)
        torch.cuda.synchronize()
        assert_close(out.cpu().numpy(), ref.cpu().numpy(), "no-alloc vs workspace entry point")
    assert smol_b200.device_error() == 0


def test_noalloc_rejects_batches_beyond_the_static_array(cuda):
    # one chunk per sequence needs n_seqs * n_heads * (hd + 2) * 4 bytes: 2048 x 32
    # heads x 258 x 4 = 67.6 MB > 16 MiB
    hq, hkv, hd = 32, 8, 256
    n = 2048
    out = torch.zeros((n, hq * hd), device=cuda)
    q = torch.zeros((n, hq * hd), device=cuda)
    kp = torch.zeros((64, hkv * hd), dtype=torch.bfloat16, device=cuda)
    vp = torch.zeros((64, hkv * hd), dtype=torch.float16, device=cuda)
    r0 = torch.zeros(n, dtype=torch.int64, device=cuda)
    kl = torch.ones(n, dtype=torch.int32, device=cuda)
    rc = smol_b200.decode_attention_noalloc(out, q, kp, vp, 64, r0, kl, n, 64, hq, hkv, hd, 0.0625)
    assert rc == 1                                  # SMOL_B200_ERR_ARGS
    assert smol_b200.last_error() == 1
    smol_b200.clear_error()
