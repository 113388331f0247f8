"""Generate tests/golden/*.npz from the compiled reference (oracle/_ref).

Run after ``make -C oracle ref REF=<reference checkout>``:

    python tests/golden/make_golden.py

Every case draws seeded inputs with numpy's default_rng, rounds attention inputs to
bf16 (the device format), runs the reference's own C entry points
(common/kernels/attention.c, rope.c, rmsnorm.c of tmzt/smol-genius, compiled by
oracle/Makefile) and stores inputs and outputs.  The tests pin the oracle
restatement and the CUDA path to these outputs on machines where the reference is
not present.
"""
from __future__ import annotations

import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, os.path.join(ROOT, "oracle"))
import pyoracle  # noqa: E402


def attn_inputs(rng, seq_q, seq_k, hq, hkv, hd):
    q = pyoracle.round_bf16(rng.standard_normal((seq_q, hq * hd)).astype(np.float32))
    k = pyoracle.round_bf16(rng.standard_normal((seq_k, hkv * hd)).astype(np.float32))
    v = pyoracle.round_bf16(rng.standard_normal((seq_k, hkv * hd)).astype(np.float32))
    return q, k, v


def put_qkv(cases, name, q, k, v):
    """Attention inputs are exactly bf16: store their bit patterns (uint16)."""
    for t, a in (("q", q), ("k", k), ("v", v)):
        cases[f"{name}/{t}_bf16"] = pyoracle.bf16_bits(a)


def main() -> None:
    ref = pyoracle.reference()
    if ref is None:
        raise SystemExit("compiled reference missing: make -C oracle ref REF=<reference checkout>")
    pyoracle.set_reference_threads(1)
    rng = np.random.default_rng(20261201)
    cases: dict[str, np.ndarray] = {}

    # ---- causal family: (name, seq_q, seq_k, hq, hkv, hd, q_offset, window, cap) ----
    causal = [
        ("causal_gqa", 37, 37, 4, 2, 64, 0, 0, 0.0),
        ("causal_chunk", 20, 57, 4, 2, 128, 37, 0, 0.0),
        ("causal_decode", 1, 150, 4, 2, 128, 149, 0, 0.0),
        ("causal_decode_short_offset", 1, 150, 4, 2, 128, 90, 0, 0.0),
        ("causal_mqa_hd256", 19, 19, 4, 1, 256, 0, 0, 0.0),
        ("sliding_window", 50, 50, 2, 1, 64, 0, 16, 0.0),
        ("causal_softcap", 33, 33, 2, 2, 64, 0, 0, 50.0),
        ("sliding_softcap", 40, 40, 4, 2, 64, 0, 12, 30.0),
        ("causal_hd80_padded", 21, 21, 2, 1, 80, 0, 0, 0.0),
        ("causal_empty_rows", 6, 4, 2, 1, 64, -3, 0, 0.0),
    ]
    for name, sq, sk, hq, hkv, hd, qo, win, cap in causal:
        q, k, v = attn_inputs(rng, sq, sk, hq, hkv, hd)
        scale = 1.0 / np.sqrt(hd)
        out = ref.causal_attention(q, k, v, sq, sk, hq, hkv, hd, scale, qo, window=win, cap=cap)
        put_qkv(cases, name, q, k, v)
        cases[f"{name}/meta"] = np.array([sq, sk, hq, hkv, hd, qo, win], np.int64)
        cases[f"{name}/fmeta"] = np.array([scale, cap], np.float32)
        cases[f"{name}/out"] = out

    # ---- bidirectional windows (siglip.c:108 uses {0, N}; qwen encoder uses many) ----
    for name, seq, h, hd, ws in [("bidir_windows", 70, 3, 64, [0, 26, 52, 70]),
                                 ("bidir_global", 64, 2, 64, [0, 64])]:
        q, k, v = attn_inputs(rng, seq, seq, h, h, hd)
        scale = 1.0 / np.sqrt(hd)
        out = ref.bidirectional_attention(q, k, v, seq, h, hd, scale, ws)
        put_qkv(cases, name, q, k, v)
        cases[f"{name}/ws"] = np.array(ws, np.int32)
        cases[f"{name}/meta"] = np.array([seq, h, hd], np.int64)
        cases[f"{name}/fmeta"] = np.array([scale], np.float32)
        cases[f"{name}/out"] = out

    # ---- prefix-LM (two causal calls, PaliGemma shape scaled down) ----
    seq, P, hq, hkv, hd = 40, 24, 4, 1, 256
    q, k, v = attn_inputs(rng, seq, seq, hq, hkv, hd)
    scale = 1.0 / np.sqrt(hd)
    put_qkv(cases, "prefix_lm", q, k, v)
    cases["prefix_lm/meta"] = np.array([seq, P, hq, hkv, hd], np.int64)
    cases["prefix_lm/fmeta"] = np.array([scale], np.float32)
    cases["prefix_lm/out"] = ref.prefix_lm_attention(q, k, v, seq, P, hq, hkv, hd, scale)

    # ---- RoPE tables and application ----
    for name, hd, theta, inter in [("rope_neox", 128, 1e6, False), ("rope_interleaved", 256, 1e4, True),
                                   ("rope_neox_odd", 10, 1e4, False)]:
        pos = np.array([0, 1, 7, 100, 4095], np.int32)
        c, s = ref.compute_rope(pos, hd, theta, interleaved=inter)
        x = rng.standard_normal((len(pos), 3 * hd)).astype(np.float32)
        y = ref.apply_rope(x, c, s, len(pos), 3, hd, interleaved=inter)
        cases[f"{name}/pos"] = pos
        cases[f"{name}/meta"] = np.array([hd, int(inter)], np.int64)
        cases[f"{name}/fmeta"] = np.array([theta], np.float32)
        cases[f"{name}/cos"], cases[f"{name}/sin"] = c, s
        cases[f"{name}/x"], cases[f"{name}/out"] = x, y

    # ---- RMSNorm ----
    x = rng.standard_normal((4, 3 * 128)).astype(np.float32)
    w = (1.0 + 0.02 * rng.standard_normal(128)).astype(np.float32)
    cases["rms_per_head/x"], cases["rms_per_head/w"] = x, w
    cases["rms_per_head/out"] = ref.rms_norm_per_head(x, w, 4, 3, 128, 1e-6)
    x = rng.standard_normal((3, 1024)).astype(np.float32)
    w = (1.0 + 0.02 * rng.standard_normal(1024)).astype(np.float32)
    cases["rms_row/x"], cases["rms_row/w"] = x, w
    cases["rms_row/out"] = ref.rms_norm(x, w, 3, 1024, 1e-6)

    cases["sinusoidal/out"] = ref.sinusoidal_pe(9, 32)

    path = os.path.join(HERE, "reference_cases.npz")
    np.savez_compressed(path, **cases)
    print(f"wrote {path}: {len(cases)} arrays, {os.path.getsize(path)} bytes")


if __name__ == "__main__":
    main()
