"""The pre-LayerNorm encoder-layer restatement (oracle/siglip_oracle.py, SiglipOracle.layer)
with attention windows, against the reference's own kernels composed in the order of the
Qwen3-ASR audio encoder's layer loop (exports/qwen_asr/encoder.c:449-484):
smol_layer_norm -> smol_linear (Q, K, V, with bias) -> smol_bidirectional_attention over
the windows -> smol_linear (O) + smol_add_inplace -> smol_layer_norm -> smol_linear (fc1)
-> smol_gelu -> smol_linear (fc2) + smol_add_inplace, eps 1e-5.  All-fp32 agreement is
held to rel-L2 1e-5.  CPU only; skipped where the reference was not built.
"""
import ctypes

import numpy as np
import pytest

import pyoracle
from siglip_oracle import SiglipOracle

REF = pyoracle.reference()
pytestmark = pytest.mark.skipif(REF is None, reason="compiled reference (oracle/_ref) not built")
_p = lambda a: ctypes.c_void_p(a.ctypes.data)   # noqa: E731


def _ref_layers(m: SiglipOracle, x: np.ndarray, ws) -> np.ndarray:
    lib, T, H, F = REF.lib, x.shape[0], m.H, m.F
    x = np.ascontiguousarray(x, np.float32).copy()
    xn, q, k, v = (np.zeros((T, H), np.float32) for _ in range(4))
    attn, proj, fo = (np.zeros((T, H), np.float32) for _ in range(3))
    mid = np.zeros((T, F), np.float32)
    wsa = np.ascontiguousarray(ws, np.int32)
    c = ctypes.c_int
    f = ctypes.c_float
    for lw in m.layers:
        W = {n: np.ascontiguousarray(lw[n], np.float32) for n in lw}
        lib.smol_layer_norm(_p(xn), _p(x), _p(W["ln1_w"]), _p(W["ln1_b"]), c(T), c(H), f(m.eps))
        for out, wn, bn in ((q, "wq", "bq"), (k, "wk", "bk"), (v, "wv", "bv")):
            lib.smol_linear(_p(out), _p(xn), _p(W[wn]), _p(W[bn]), c(T), c(H), c(H))
        lib.smol_bidirectional_attention(_p(attn), _p(q), _p(k), _p(v), c(T), c(m.NH), c(m.HD),
                                         f(1.0 / np.sqrt(np.float32(m.HD))), _p(wsa), c(len(ws) - 1))
        lib.smol_linear(_p(proj), _p(attn), _p(W["wo"]), _p(W["bo"]), c(T), c(H), c(H))
        lib.smol_add_inplace(_p(x), _p(proj), c(T * H))
        lib.smol_layer_norm(_p(xn), _p(x), _p(W["ln2_w"]), _p(W["ln2_b"]), c(T), c(H), f(m.eps))
        lib.smol_linear(_p(mid), _p(xn), _p(W["fc1"]), _p(W["b1"]), c(T), c(H), c(F))
        lib.smol_gelu(_p(mid), c(T * F))
        lib.smol_linear(_p(fo), _p(mid), _p(W["fc2"]), _p(W["b2"]), c(T), c(F), c(H))
        lib.smol_add_inplace(_p(x), _p(fo), c(T * H))
    return x


def test_windowed_encoder_layers_match_reference_composition():
    m = SiglipOracle(hidden=256, heads=4, ffn=512, layers=2, eps=1e-5, seed=8)
    ws = list(range(0, 5 * 26 + 1, 26)) + [5 * 26 + 11]          # six windows, the last ragged
    T = ws[-1]
    x = np.random.default_rng(9).standard_normal((T, m.H)).astype(np.float32)
    want = _ref_layers(m, x, ws)
    got = m.encoder_layers(x[None], device_formats=False, window_starts=ws)[0]
    assert pyoracle.rel_l2(got, want) < 1e-5
    # the device formats move it by the bf16 operand rounding only
    assert pyoracle.rel_l2(m.encoder_layers(x[None], device_formats=True, window_starts=ws)[0], want) < 1e-2
