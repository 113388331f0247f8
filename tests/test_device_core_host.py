"""Host logic of the decoder-level drop-ins (smol-genius_b200/dropin/device_decoder.c) on the CPU.

tests/dropin/device_core_fake_main.c links the core against fakes of the libsmol_b200 calls
it makes (device memory as registered host memory; prefill / decode calls that check and
tag the KV pool rows) and checks: the weights handed to the library are device copies of
the host weights (Qwen3 and Gemma / untied-head settings); pool growth keeps every row
written earlier at the row the library reads it from; positions past the ones held are
refused and truncation is honoured; the side table recognises a context address reused
for other weights, runs out after its 8 slots and releases everything; and every single
failed allocation -- during the upload, or during a pool growth -- fails cleanly, frees
what it must and is retried by the next call.  No GPU and no reference checkout needed.

The two shims themselves (qkn_decoder_device.c, smolvlm_decoder_device.c) are checked the
same way by oracle/_ref/{qkn,smolvlm}_shim_fake (tests/dropin/shim_fake_main.c, built
against the reference's headers by `make -C oracle dropin`): the reference context's
configuration and every weight reach the library unchanged (Gemma 2 settings for
qkn_decoder, the untied head for SmolVLM); kv_cache_len and dec_x follow the reference's
contract; a position past the held ones returns the export's sentinel; release and a
reloaded context set up afresh.
"""
import os
import shutil
import subprocess

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


@pytest.mark.skipif(shutil.which("gcc") is None, reason="gcc not available")
def test_device_core_host_logic(tmp_path):
    exe = tmp_path / "device_core_fake"
    dropin = os.path.join(ROOT, "tests", "dropin")
    subprocess.run(["gcc", "-O2", "-Wall", "-Wextra", "-Werror", "-std=c11",
                    "-I", os.path.join(ROOT, "include"), "-I", os.path.join(ROOT, "smol-genius_b200", "dropin"),
                    "-I", dropin, "-o", str(exe), os.path.join(dropin, "device_core_fake_main.c"),
                    os.path.join(dropin, "fake_smol_b200.c"),
                    os.path.join(ROOT, "smol-genius_b200", "dropin", "device_decoder.c")],
                   check=True, capture_output=True, text=True)
    p = subprocess.run([str(exe)], capture_output=True, text=True, timeout=120)
    assert p.returncode == 0, p.stderr
    assert "failures 0" in p.stdout
    assert "past the" in p.stderr   # the refusals say why


@pytest.mark.parametrize("shim", ["qkn", "smolvlm"])
def test_dropin_shim_hands_over_the_context(shim):
    exe = os.path.join(ROOT, "oracle", "_ref", f"{shim}_shim_fake")
    if not os.path.exists(exe):
        pytest.skip(f"{exe} not built (reference checkout absent at build time)")
    p = subprocess.run([exe], capture_output=True, text=True, timeout=120)
    assert p.returncode == 0, p.stderr
    assert "failures 0" in p.stdout
