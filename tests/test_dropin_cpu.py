"""CPU half of the drop-in evidence: what bf16 / fp16 cache storage does to the reference.

Runs only the reference builds (qkn_dropin_ref: fp32 host cache; qkn_dropin_emul: the
same kernels on bf16 K / fp16 V / bf16 prefill Q values) of tests/dropin/qkn_dropin_main.c.
On the decisive model the storage precision leaves all 128 greedy tokens unchanged; on
the random-read-out model, whose top-2 logit margins fall to ~0.02, it flips step 116.
The GPU test checks that libsmol_b200 reproduces the emulated stream in both cases.
"""
import os
import subprocess

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
BIN = {k: os.path.join(ROOT, "oracle", "_ref", f"qkn_dropin_{k}") for k in ("ref", "emul")}

pytestmark = pytest.mark.skipif(not all(os.path.exists(b) for b in BIN.values()),
                                reason="reference drop-in binaries not built (reference checkout absent)")


def tokens(kind, args, env=None):
    p = subprocess.run([BIN[kind], *map(str, args)], capture_output=True, text=True, timeout=300, check=True,
                       env=None if env is None else {**os.environ, **env})
    return p.stdout.split()


def first_divergence(a, b):
    return next((i for i, (x, y) in enumerate(zip(a, b)) if x != y), None)


def test_storage_precision_keeps_decisive_stream():
    args = (512, 128, 2, 4, 2, 1, 1)
    ref, emul = tokens("ref", args), tokens("emul", args)
    assert len(ref) == 128 and len(set(ref)) >= 32
    assert ref == emul


def test_warm_run_prints_the_same_stream():
    """SMOL_DROPIN_WARM=1 (the bench's steady-state timing) runs the generation once
    unreported, resets the cache with qkn_kv_cache_reset and prints the second run: the
    same tokens as a first run, and only one line of them."""
    args = (64, 16, 2, 4, 2, 1, 1)
    cold = tokens("ref", args)
    warm = tokens("ref", args, {"SMOL_DROPIN_WARM": "1"})
    assert len(cold) == 16 and warm == cold


def test_storage_precision_flips_near_tie_of_random_readout():
    args = (512, 128, 1, 3, 4, 1, 0)
    assert first_divergence(tokens("ref", args), tokens("emul", args)) == 116


def test_device_decoder_dropin_fails_loudly_without_a_device():
    """The decoder-level drop-in has no CPU path: without a GPU the prefill and the forward
    say why on stderr and the forward returns the reference's allocation-failure
    sentinel (151645), which the driver reports and stops on."""
    import torch
    device_bin = os.path.join(ROOT, "oracle", "_ref", "qkn_dropin_device")
    if not os.path.exists(device_bin):
        pytest.skip("qkn_dropin_device not built")
    if torch.cuda.is_available():
        pytest.skip("a CUDA device is present")
    p = subprocess.run([device_bin, "32", "3"], capture_output=True, text=True, timeout=120)
    assert p.returncode == 3 and p.stdout.split() == ["151645"], (p.returncode, p.stdout)
    assert "qkn_decoder_prefill (device)" in p.stderr and "qkn_decoder_forward (device)" in p.stderr
