"""The allocation-free decode entry point (smol_b200_decode_attention_noalloc).

Some callers cannot call cudaMalloc -- a plugin inside another framework's memory
manager that owns all device memory, or a serving loop that must not allocate
after start-up -- so this entry point keeps its split-KV partial results in a fixed
16 MiB device array inside the library instead of a caller workspace.  These tests
call it through the C ABI and check:

* two calls in a row against smol_b200_decode_attention on the same inputs (in this
  process, which has usually run the other GPU tests first, so the library's other
  state already exists);
* a batch whose partials fit the array only after the call widens its key chunks;
* the same two calls in a freshly spawned process that has not used the library
  before, so the entry point's one-time set-up (looking up the array's device
  address) runs there, and smol_cuda_device_error() is read while no other entry
  point has run (its watchdog word is then a word of the array);
* that a batch too large for the array is refused with a clear error.

The file is named to be collected last: if it fails, a run that stops at the first
failure has already run every other test.
"""
import json
import os
import subprocess
import sys

import numpy as np
import pytest
import torch

import smol_b200
from conftest import assert_close

pytestmark = pytest.mark.gpu

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
ARRAY_BYTES = (16 << 20) - 256      # the static array, less its 256-byte header


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


def run_noalloc(b, hq, hkv, hd):
    out = torch.full((b["n"], hq * hd), 7.0, device=b["q"].device)
    rc = smol_b200.decode_attention_noalloc(out, b["q"], b["kp"], b["vp"], b["rows"], b["r0"], b["kl"], b["n"],
                                            b["max_len"], hq, hkv, hd, 1 / np.sqrt(hd))
    assert rc == 0, smol_b200.lib().smol_cuda_error_string(rc)
    return out


def run_workspace(b, hq, hkv, hd):
    out = torch.zeros((b["n"], hq * hd), device=b["q"].device)
    ws = torch.empty(smol_b200.decode_workspace_bytes(b["n"], b["max_len"], hq, hkv, hd), dtype=torch.uint8,
                     device=b["q"].device)
    smol_b200.decode_attention(out, b["q"], b["kp"], b["vp"], b["rows"], b["r0"], b["kl"], b["n"], b["max_len"],
                               hq, hkv, hd, 1 / np.sqrt(hd), ws)
    torch.cuda.synchronize()
    return out


def two_calls(cuda):
    """Two allocation-free calls back to back, the second smaller (stale partials of
    the first stay behind in the array), then the workspace entry point on each."""
    hq, hkv, hd = 16, 8, 128
    first = make_batch(cuda, 1, 96, 1, 8192, hq, hkv, hd)
    second = make_batch(cuda, 2, 40, 1, 3000, hq, hkv, hd)
    outs = [run_noalloc(b, hq, hkv, hd) for b in (first, second)]
    torch.cuda.synchronize()
    device_error_noalloc_only = smol_b200.device_error()
    pairs = [(out.cpu().numpy(), run_workspace(b, hq, hkv, hd).cpu().numpy()) for b, out in zip((first, second), outs)]
    return pairs, device_error_noalloc_only


def test_noalloc_matches_workspace_entry_point_on_two_calls(cuda):
    pairs, err = two_calls(cuda)
    assert err == 0
    for i, (got, want) in enumerate(pairs):
        assert_close(got, want, f"call {i + 1}: no-alloc vs workspace entry point")
    assert smol_b200.device_error() == 0


def _default_partial_bytes(n, L, hq, hkv, hd):
    """Partials at the regular entry point's chunk (the library's rule restated)."""
    w = n * hkv * ((hq // hkv + 7) // 8)
    c = -(-w * L // 1184)                  # keys per CTA for ~8 CTAs per SM of 148
    c = min(max(-(-c // 64) * 64, 64), 2048)
    return n * hq * -(-L // c) * (hd + 2) * 4


def test_noalloc_widens_chunks_until_partials_fit(cuda):
    # 256 sequences x 32 heads, 7000-8192 keys: at the regular chunk (2048 keys, 4
    # chunks) the partials take 17.0 MB, more than the array holds; 4096-key chunks
    # (2 per sequence) need 8.5 MB.
    hq, hkv, hd = 32, 8, 128
    b = make_batch(cuda, 3, 256, 7000, 8192, hq, hkv, hd)
    assert _default_partial_bytes(b["n"], b["max_len"], hq, hkv, hd) > ARRAY_BYTES
    got = run_noalloc(b, hq, hkv, hd)
    torch.cuda.synchronize()
    assert smol_b200.last_error() == 0 and smol_b200.device_error() == 0
    assert_close(got.cpu().numpy(), run_workspace(b, hq, hkv, hd).cpu().numpy(), "widened chunks")


def _child_main():
    """Run in a fresh process: the allocation-free calls are this process's first use
    of the library."""
    cuda = torch.device("cuda:0")
    pairs, err = two_calls(cuda)
    import pyoracle
    print(json.dumps({"device_error_noalloc_only": int(err),
                      "rel_l2": [float(pyoracle.rel_l2(g, w)) for g, w in pairs],
                      "max_abs": [float(np.abs(g - w).max()) for g, w in pairs],
                      "finite": [bool(np.isfinite(g).all()) for g, _ in pairs],
                      "last_error": int(smol_b200.last_error()), "device_error": int(smol_b200.device_error())}))


def test_noalloc_first_use_in_a_fresh_process(cuda):
    paths = [HERE, os.path.join(ROOT, "smol-genius_b200"), os.path.join(ROOT, "oracle")]
    code = ("import sys; sys.path[:0] = %r; import test_zz_no_alloc as t; t._child_main()" % paths)
    r = subprocess.run([sys.executable, "-c", code], capture_output=True, text=True, timeout=600, cwd=ROOT)
    assert r.returncode == 0, r.stderr[-3000:]
    res = json.loads(r.stdout.strip().splitlines()[-1])
    assert res["device_error_noalloc_only"] == 0 and res["device_error"] == 0 and res["last_error"] == 0, res
    from conftest import REL_L2_TOL, MAX_ABS_TOL
    assert all(res["finite"]), res
    assert all(e <= REL_L2_TOL for e in res["rel_l2"]) and all(m <= MAX_ABS_TOL for m in res["max_abs"]), res


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
