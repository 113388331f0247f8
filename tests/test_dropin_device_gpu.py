"""The decoder-level drop-in, end to end: the reference's driver with qkn_decoder_prefill /
qkn_decoder_forward from smol-genius_b200/dropin/qkn_decoder_device.c.

oracle/Makefile (target `dropin`) builds oracle/_ref/qkn_dropin_device from
tests/dropin/qkn_dropin_main.c and the reference's common/decoder/qkn_decoder.c compiled
with those two functions renamed, so the reference loader fills the qkn_ctx_t and every
prefill and decode step then runs on the device: weights uploaded once, the KV cache,
RoPE tables and the greedy argmax on the GPU (Part 4 of smol_b200.h).  On the decisive
model (smallest top-2 logit margin 9.0) the 128 greedy tokens equal those of the
unmodified fp32 reference (oracle/_ref/qkn_dropin_ref).
"""
import os
import subprocess

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
BIN = {k: os.path.join(ROOT, "oracle", "_ref", f"qkn_dropin_{k}") for k in ("ref", "device")}
DECISIVE = (512, 128, 2, 4, 2, 1, 1)   # prefill, steps, seed, qk_gain, vo_gain, layers, copy

pytestmark = [pytest.mark.gpu, pytest.mark.new_on_gpu(stage=2),
              pytest.mark.skipif(not all(os.path.exists(b) for b in BIN.values()),
                                 reason="drop-in binaries not built (reference checkout absent at build time)")]


def test_device_decoder_tokens_equal_unmodified_reference(cuda):
    out = {}
    for kind in ("ref", "device"):
        p = subprocess.run([BIN[kind], *map(str, DECISIVE)], capture_output=True, text=True, timeout=600, check=True)
        assert "(device)" not in p.stderr and "smol_b200:" not in p.stderr, p.stderr
        out[kind] = [int(t) for t in p.stdout.split()]
    assert len(out["ref"]) == DECISIVE[1] and len(set(out["ref"])) >= 32
    d = next((i for i, (a, b) in enumerate(zip(out["ref"], out["device"])) if a != b), None)
    assert d is None, f"diverged at step {d}: {out['ref'][d:d + 4]} vs {out['device'][d:d + 4]}"
