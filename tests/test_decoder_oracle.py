"""Pins the decoder-step restatement (oracle/qkn_decoder_oracle.py) to the compiled reference.

The pieces the device decoder step adds around attention -- RMSNorm, the bf16
matrix-vector product, the SwiGLU gate and the greedy argmax -- are computed by the
restatement and by the reference's own functions (smol_rms_norm, smol_linear_nobias_bf16
with seq_len 1, smol_swiglu_multiply, smol_argmax_matvec_bf16 from oracle/_ref) on the
same seeded inputs.  CPU only; skipped where the reference was not built.
"""
import ctypes

import numpy as np
import pytest

import pyoracle
from qkn_decoder_oracle import argmax_first, rms_norm, swiglu

REF = pyoracle.reference()
pytestmark = pytest.mark.skipif(REF is None, reason="compiled reference (oracle/_ref) not built")
_p = lambda a: ctypes.c_void_p(a.ctypes.data)   # noqa: E731


def test_rms_norm_matches_reference():
    rng = np.random.default_rng(1)
    x = rng.standard_normal((3, 1024)).astype(np.float32)
    w = (1 + 0.02 * rng.standard_normal(1024)).astype(np.float32)
    got = rms_norm(x, w, 1e-6)
    want = REF.rms_norm(x, w, 3, 1024, 1e-6)
    assert pyoracle.rel_l2(got, want) < 1e-6


def test_bf16_matvec_matches_reference():
    rng = np.random.default_rng(2)
    W = pyoracle.round_bf16((rng.standard_normal((2048, 1024)) / 32).astype(np.float32))
    x = rng.standard_normal(1024).astype(np.float32)
    y = np.zeros(2048, np.float32)
    bits = np.ascontiguousarray(pyoracle.bf16_bits(W))
    REF.lib.smol_linear_nobias_bf16(_p(y), _p(x), _p(bits), ctypes.c_int(1), ctypes.c_int(1024), ctypes.c_int(2048))
    assert pyoracle.rel_l2(x @ W.T, y) < 1e-6


def test_swiglu_matches_reference():
    rng = np.random.default_rng(3)
    gu = (3 * rng.standard_normal(2 * 3072)).astype(np.float32)
    out = np.zeros(3072, np.float32)
    REF.lib.smol_swiglu_multiply(_p(out), _p(gu), ctypes.c_int(1), ctypes.c_int(3072))
    assert pyoracle.rel_l2(swiglu(gu), out) < 1e-6


def test_argmax_matches_reference_including_ties():
    rng = np.random.default_rng(4)
    E = pyoracle.round_bf16(rng.standard_normal((4096, 1024)).astype(np.float32))
    E[3001] = E[1234]                      # equal maxima at rows 1234 and 3001
    x = (E[1234] * 2).astype(np.float32)
    bits = np.ascontiguousarray(pyoracle.bf16_bits(E))
    REF.lib.smol_argmax_matvec_bf16.restype = ctypes.c_int
    for threads in (1, 8):
        pyoracle.set_reference_threads(threads)
        want = REF.lib.smol_argmax_matvec_bf16(_p(x), _p(bits), ctypes.c_int(1024), ctypes.c_int(4096))
        assert want == 1234 == argmax_first(E @ x)
