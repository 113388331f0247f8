"""Generate tests/golden/bf16_decoder_cases.npz from the reference's bf16 decoder attention.

Run after ``make -C oracle ref REF=<reference checkout>`` (which builds
oracle/_ref/libsmol_bf16_ref.so from oracle/bf16_attention_ref.c):

    python tests/golden/make_bf16_golden.py

The reference's bf16 Gemma decoder (common/decoder/qkn_bf16_decoder.c of
tmzt/smol-genius) attends over a bf16 KV cache with its own attention:
bf16_causal_attention_softcap (:120-172) and bf16_swa_attention_softcap (:175-233) --
fp32 scores, a two-pass softmax with expf, the output truncated to bf16.  That is the
reference's own form of the bf16-cache path the device implements, so its outputs are
a second oracle for it.  Cases use the PaliGemma decoder's attention settings
(paligemma.c:206-222: 8 Q heads / 1 KV head, head dim 256, softcap 50, sliding layers)
plus a GQA case without a cap; inputs are seeded bf16 values, Q scaled so that the
softcap bends the scores.
"""
from __future__ import annotations

import ctypes
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, os.path.join(ROOT, "oracle"))
import pyoracle  # noqa: E402

LIB = os.path.join(ROOT, "oracle", "_ref", "libsmol_bf16_ref.so")

# (name, seq_q, seq_k, hq, hkv, hd, q_offset, window, cap, q_scale)
CASES = [
    ("mqa_prefill_softcap", 64, 64, 8, 1, 256, 0, 0, 50.0, 4.0),
    ("mqa_chunk_softcap", 24, 100, 8, 1, 256, 76, 0, 50.0, 4.0),
    ("mqa_decode_softcap", 1, 200, 8, 1, 256, 199, 0, 50.0, 4.0),
    ("mqa_sliding_prefill", 80, 80, 8, 1, 256, 0, 32, 50.0, 4.0),
    ("mqa_sliding_decode", 1, 200, 8, 1, 256, 199, 64, 50.0, 4.0),
    ("gqa_prefill_nocap", 70, 70, 4, 2, 128, 0, 0, 0.0, 1.0),
    ("gqa_decode_nocap", 1, 129, 4, 2, 128, 128, 0, 0.0, 1.0),
]


def main() -> None:
    if not os.path.exists(LIB):
        raise SystemExit("oracle/_ref/libsmol_bf16_ref.so missing: make -C oracle ref REF=<reference checkout>")
    lib = ctypes.CDLL(LIB)
    f = lib.ref_bf16_attention
    f.restype = None
    f.argtypes = [ctypes.c_void_p] * 4 + [ctypes.c_int] * 5 + [ctypes.c_float, ctypes.c_int, ctypes.c_int,
                                                                 ctypes.c_float]
    rng = np.random.default_rng(20261202)
    out: dict[str, np.ndarray] = {}
    for name, sq, sk, hq, hkv, hd, qo, win, cap, qs in CASES:
        q = pyoracle.bf16_bits(pyoracle.round_bf16((qs * rng.standard_normal((sq, hq * hd))).astype(np.float32)))
        k = pyoracle.bf16_bits(pyoracle.round_bf16(rng.standard_normal((sk, hkv * hd)).astype(np.float32)))
        v = pyoracle.bf16_bits(pyoracle.round_bf16(rng.standard_normal((sk, hkv * hd)).astype(np.float32)))
        o = np.zeros((sq, hq * hd), np.uint16)
        scale = float(1.0 / np.sqrt(hd))
        f(o.ctypes.data, q.ctypes.data, k.ctypes.data, v.ctypes.data, sq, sk, hq, hkv, hd, scale, qo, win, cap)
        out[f"{name}/q_bf16"], out[f"{name}/k_bf16"], out[f"{name}/v_bf16"] = q, k, v
        out[f"{name}/out_bf16"] = o
        out[f"{name}/meta"] = np.array([sq, sk, hq, hkv, hd, qo, win], np.int64)
        out[f"{name}/fmeta"] = np.array([scale, cap], np.float32)
    path = os.path.join(HERE, "bf16_decoder_cases.npz")
    np.savez_compressed(path, **out)
    print(f"wrote {path}: {len(CASES)} cases")


if __name__ == "__main__":
    main()
