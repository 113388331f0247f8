"""The decoder-level drop-ins, end to end: the reference's drivers with qkn_decoder_prefill /
qkn_decoder_forward from smol-genius_b200/dropin/qkn_decoder_device.c, and SmolVLM's
decoder from smol-genius_b200/dropin/smolvlm_decoder_device.c.

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
SMOLVLM_BIN = os.path.join(ROOT, "oracle", "_ref", "smolvlm_weights_device")
DECISIVE = (512, 128, 2, 4, 2, 1, 1)   # prefill, steps, seed, qk_gain, vo_gain, layers, copy

pytestmark = [pytest.mark.gpu, pytest.mark.new_on_gpu(stage=2)]


@pytest.mark.skipif(not all(os.path.exists(b) for b in BIN.values()),
                    reason="drop-in binaries not built (reference checkout absent at build time)")

def test_device_decoder_tokens_equal_unmodified_reference(cuda):
    out = {}
    for kind in ("ref", "device"):
        p = subprocess.run([BIN[kind], *map(str, DECISIVE)], capture_output=True, text=True, timeout=600, check=True)
        assert "(device)" not in p.stderr and "smol_b200:" not in p.stderr, p.stderr
        out[kind] = [int(t) for t in p.stdout.split()]
    assert len(out["ref"]) == DECISIVE[1] and len(set(out["ref"])) >= 32
    d = next((i for i, (a, b) in enumerate(zip(out["ref"], out["device"])) if a != b), None)
    assert d is None, f"diverged at step {d}: {out['ref'][d:d + 4]} vs {out['device'][d:d + 4]}"


@pytest.mark.skipif(not all(os.path.exists(b) for b in BIN.values()),
                    reason="drop-in binaries not built (reference checkout absent at build time)")
def test_device_decoder_release_and_position_guard(cuda):
    """qkn_decoder_device_release frees the context's device state and zeroes
    kv_cache_len; the same context then runs the same prompt again from scratch (weights
    uploaded again) with the same tokens.  A kv_cache_len past the positions the device
    holds returns the failure sentinel 151645 instead of attending unwritten rows."""
    args = list(map(str, (DECISIVE[0], 32) + DECISIVE[2:]))   # the decisive stream's first 32 steps
    ref = subprocess.run([BIN["ref"], *args], capture_output=True, text=True, timeout=600, check=True)
    p = subprocess.run([BIN["device"], *args], capture_output=True, text=True, timeout=600,
                       env={**os.environ, "SMOL_DROPIN_RERUN": "1"})
    assert p.returncode == 0, p.stderr
    lines = [[int(t) for t in ln.split()] for ln in p.stdout.splitlines() if ln.strip()]
    assert len(lines) == 2 and len(lines[0]) == 32, p.stdout
    assert lines[0] == lines[1] == [int(t) for t in ref.stdout.split()]
    assert "past_held_token 151645" in p.stderr, p.stderr
    assert "past the" in p.stderr


@pytest.mark.skipif(not os.path.exists(SMOLVLM_BIN), reason="smolvlm_weights_device not built")
def test_smolvlm_device_decoder_matches_oracle(cuda, tmp_path):
    """SmolVLM's decoder-level drop-in (smol-genius_b200/dropin/smolvlm_decoder_device.c)
    driven by tests/dropin/smolvlm_weights_main.c on the oracle's SmolVLM pin case: every
    teacher-forced step's final normalised state within rel-L2 5e-3 of the oracle with the
    device prefill's bf16 operands, the token equal wherever the margin exceeds 0.05."""
    import numpy as np

    import pyoracle
    from qkn_decoder_oracle import pin_case, read_reference_steps, write_weights_file
    m, prompt, feed = pin_case("smolvlm-2")
    write_weights_file(tmp_path / "model.bin", m, prompt, feed)
    p = subprocess.run([SMOLVLM_BIN, str(tmp_path / "model.bin"), str(tmp_path / "steps.bin")], capture_output=True,
                       text=True, timeout=600)
    assert p.returncode == 0 and "(device)" not in p.stderr, p.stderr
    tokens, xs = read_reference_steps(tmp_path / "steps.bin", len(feed), m.H)
    m.prefill(prompt[:-1], device_formats=True)
    for s, f in enumerate(feed):
        want, margin, xf = m.forward(f)
        assert pyoracle.rel_l2(xs[s], xf) < 5e-3, (s, pyoracle.rel_l2(xs[s], xf))
        if margin > 0.05:
            assert int(tokens[s]) == want, (s, int(tokens[s]), want, margin)
    assert len(set(np.asarray(tokens).tolist())) > 1
