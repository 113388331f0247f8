"""Pins the SigLIP encoder restatement (oracle/siglip_oracle.py) to the reference's siglip_forward.

The oracle's seeded encoder and images go through a file to oracle/_ref/siglip_weights_ref
(tests/dropin/siglip_weights_main.c: the reference's common/vision/siglip.c with its
kernels: conv2d patch embedding, LayerNorm, linear with bias, bidirectional attention,
GELU, post-LayerNorm).  In the reference's all-fp32 arithmetic the oracle agrees to
rel-L2 1e-5.  With the device's 16-bit operands (LayerNorm, attention and GELU outputs
and Q/K bf16, V fp16, pixels bf16) the gap to the fp32 reference is that of bf16
rounding -- about 3e-3 rel-L2 -- and is bounded here at 1e-2, the tolerance the device
encoder is held to against the reference (against the device-format oracle it is held
to 1e-3).  Where the binary is built the comparison runs live; everywhere it also runs
against the reference's outputs in tests/golden/siglip_cases.npz
(tests/golden/make_siglip_golden.py).  CPU only.
"""
import os
import subprocess

import numpy as np
import pytest

import pyoracle
from siglip_oracle import SIGLIP_PIN_CASES, siglip_pin_case

BIN = os.path.join(os.path.dirname(pyoracle.__file__), "_ref", "siglip_weights_ref")
GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "siglip_cases.npz")


def _check(m, images, ref):
    assert pyoracle.rel_l2(m.forward(images, device_formats=False), ref) < 1e-5
    assert pyoracle.rel_l2(m.forward(images, device_formats=True), ref) < 1e-2


@pytest.mark.skipif(not os.path.exists(BIN), reason="oracle/_ref/siglip_weights_ref not built")
@pytest.mark.parametrize("case", list(SIGLIP_PIN_CASES))
def test_siglip_oracle_matches_reference_encoder(tmp_path, case):
    m, images = siglip_pin_case(case)
    m.write_weights_file(tmp_path / "model.bin", images)
    subprocess.run([BIN, str(tmp_path / "model.bin"), str(tmp_path / "out.bin")], check=True, timeout=300)
    ref = np.fromfile(tmp_path / "out.bin", np.float32).reshape(len(images), m.n_pos, m.H)
    _check(m, images, ref)


@pytest.mark.skipif(not os.path.exists(GOLDEN), reason="tests/golden/siglip_cases.npz not generated")
@pytest.mark.parametrize("case", list(SIGLIP_PIN_CASES))
def test_siglip_oracle_matches_reference_golden(case):
    m, images = siglip_pin_case(case)
    _check(m, images, np.load(GOLDEN)[f"{case}/out"])
