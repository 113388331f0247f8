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
"""
import os
import shutil
import subprocess

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


@pytest.mark.skipif(shutil.which("gcc") is None, reason="gcc not available")
def test_device_core_host_logic(tmp_path):
    exe = tmp_path / "device_core_fake"
    subprocess.run(["gcc", "-O2", "-Wall", "-Wextra", "-Werror", "-std=c11",
                    "-I", os.path.join(ROOT, "include"), "-I", os.path.join(ROOT, "smol-genius_b200", "dropin"),
                    "-o", str(exe), os.path.join(ROOT, "tests", "dropin", "device_core_fake_main.c"),
                    os.path.join(ROOT, "smol-genius_b200", "dropin", "device_decoder.c")],
                   check=True, capture_output=True, text=True)
    p = subprocess.run([str(exe)], capture_output=True, text=True, timeout=120)
    assert p.returncode == 0, p.stderr
    assert "failures 0" in p.stdout
    assert "past the" in p.stderr   # the refusals say why
