"""pyoracle -- ctypes access to the CPU oracle.  TEST INFRASTRUCTURE ONLY.

Two libraries, both plain C on the host cores:
  * ``libsmol_oracle.so``: this repository's restatement (smol_oracle.c), always built;
  * ``_ref/libsmol_ref_{avx2,avx512}.so``: the reference's own sources compiled by
    oracle/Makefile, present wherever the reference checkout was available at build
    time (the built files travel with the repository snapshot).

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg import this
module.  It is the checker, never the thing measured or shipped.
"""
from __future__ import annotations

import ctypes
import os

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ORACLE_SO = os.path.join(HERE, "libsmol_oracle.so")
REF_DIR = os.path.join(HERE, "_ref")

_c_int, _c_float, _c_void = ctypes.c_int, ctypes.c_float, ctypes.c_void_p


def _cpu_has_avx512() -> bool:
    try:
        with open("/proc/cpuinfo") as f:
            return " avx512f " in f.read().replace("\n", " ")
    except OSError:
        return False


def ref_path() -> str | None:
    """Path of the compiled reference suited to this CPU, or None when not built."""
    for name in (["libsmol_ref_avx512.so"] if _cpu_has_avx512() else []) + ["libsmol_ref_avx2.so"]:
        p = os.path.join(REF_DIR, name)
        if os.path.exists(p):
            return p
    return None


_libs: dict[str, ctypes.CDLL] = {}


def _load(path: str) -> ctypes.CDLL:
    if path not in _libs:
        _libs[path] = ctypes.CDLL(path)
    return _libs[path]


def _p(a):
    return None if a is None else ctypes.c_void_p(a.ctypes.data)


def f32(a) -> np.ndarray:
    return np.ascontiguousarray(a, dtype=np.float32)


# ---------------------------------------------------------------------------
# number formats (numpy, for building inputs)
# ---------------------------------------------------------------------------
def bf16_bits(x: np.ndarray) -> np.ndarray:
    """fp32 -> bf16 bit patterns, round to nearest even."""
    u = f32(x).view(np.uint32).astype(np.uint64)
    u = (u + 0x7FFF + ((u >> 16) & 1)) >> 16
    return u.astype(np.uint16)


def bf16_to_f32(bits: np.ndarray) -> np.ndarray:
    return (np.ascontiguousarray(bits, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


def round_bf16(x: np.ndarray) -> np.ndarray:
    return bf16_to_f32(bf16_bits(x))


class Kernels:
    """The attention / RoPE / RMSNorm entry points of one CPU library.

    ``prefix`` is "oracle_" for the restatement and "smol_" for the compiled
    reference; the argument lists are identical.
    """

    def __init__(self, lib: ctypes.CDLL, prefix: str):
        self.lib, self.pre = lib, prefix

    def fn(self, name):
        return getattr(self.lib, self.pre + name)

    def causal_attention(self, Q, K, V, seq_q, seq_k, n_heads, n_kv_heads, head_dim, scale, q_offset,
                         window=0, cap=0.0):
        out = np.zeros((seq_q, n_heads * head_dim), np.float32)
        Q, K, V = f32(Q), f32(K), f32(V)
        a = [_p(out), _p(Q), _p(K), _p(V), _c_int(seq_q), _c_int(seq_k), _c_int(n_heads), _c_int(n_kv_heads),
             _c_int(head_dim), _c_float(scale), _c_int(q_offset)]
        if window > 0 and cap > 0:
            self.fn("sliding_window_attention_softcap")(*a, _c_int(window), _c_float(cap))
        elif window > 0:
            self.fn("sliding_window_attention")(*a, _c_int(window))
        elif cap > 0:
            self.fn("causal_attention_softcap")(*a, _c_float(cap))
        else:
            self.fn("causal_attention")(*a)
        return out

    def bidirectional_attention(self, Q, K, V, seq, n_heads, head_dim, scale, window_starts, out=None):
        out = np.zeros((seq, n_heads * head_dim), np.float32) if out is None else out
        ws = np.ascontiguousarray(window_starts, dtype=np.int32)
        Q, K, V = f32(Q), f32(K), f32(V)
        self.fn("bidirectional_attention")(_p(out), _p(Q), _p(K), _p(V), _c_int(seq), _c_int(n_heads),
                                           _c_int(head_dim), _c_float(scale), _p(ws), _c_int(len(ws) - 1))
        return out

    def prefix_lm_attention(self, Q, K, V, seq, prefix_len, n_heads, n_kv_heads, head_dim, scale):
        """Prefix-LM via two causal calls (q_offset=P-1 for the prefix rows, P for the suffix)."""
        Q = f32(Q)
        qw = n_heads * head_dim
        P = prefix_len
        top = self.causal_attention(Q[:P], K, V, P, P, n_heads, n_kv_heads, head_dim, scale, P - 1)
        if seq == P:
            return top
        bot = self.causal_attention(np.ascontiguousarray(Q[P:]), K, V, seq - P, seq, n_heads, n_kv_heads, head_dim,
                                    scale, P)
        return np.concatenate([top.reshape(P, qw), bot.reshape(seq - P, qw)], axis=0)

    def apply_rope(self, x, cos, sin, seq, n_heads, head_dim, interleaved=False):
        x = f32(x).copy()
        cos, sin = f32(cos), f32(sin)
        self.fn("apply_rope_interleaved" if interleaved else "apply_rope_neox")(
            _p(x), _p(cos), _p(sin), _c_int(seq), _c_int(n_heads), _c_int(head_dim))
        return x

    def compute_rope(self, positions, head_dim, theta, interleaved=False):
        pos = np.ascontiguousarray(positions, dtype=np.int32)
        c = np.zeros((len(pos), head_dim), np.float32)
        s = np.zeros((len(pos), head_dim), np.float32)
        self.fn("compute_rope_interleaved" if interleaved else "compute_rope_neox")(
            _p(c), _p(s), _p(pos), _c_int(len(pos)), _c_int(head_dim), _c_float(theta))
        return c, s

    def rms_norm_per_head(self, x, w, seq, n_heads, head_dim, eps):
        x = f32(x).copy()
        w = f32(w)
        self.fn("rms_norm_per_head")(_p(x), _p(w), _c_int(seq), _c_int(n_heads), _c_int(head_dim),
                                     _c_float(eps))
        return x

    def rms_norm(self, x, w, seq, hidden, eps):
        x, w = f32(x), f32(w)
        out = np.zeros_like(x)
        self.fn("rms_norm")(_p(out), _p(x), _p(w), _c_int(seq), _c_int(hidden), _c_float(eps))
        return out

    def sinusoidal_pe(self, n_pos, d_model):
        pe = np.zeros((n_pos, d_model), np.float32)
        self.fn("sinusoidal_pe")(_p(pe), _c_int(n_pos), _c_int(d_model))
        return pe


def oracle() -> Kernels:
    if not os.path.exists(ORACLE_SO):
        raise FileNotFoundError(f"{ORACLE_SO} missing: run `make -C oracle`")
    return Kernels(_load(ORACLE_SO), "oracle_")


def reference() -> Kernels | None:
    p = ref_path()
    return None if p is None else Kernels(_load(p), "smol_")


def set_reference_threads(n: int) -> None:
    """smol_set_threads of the compiled reference (threading.c:76-102, capped at 16)."""
    p = ref_path()
    if p is not None:
        _load(p).smol_set_threads(_c_int(n))


# ---------------------------------------------------------------------------
# oracle-only helpers (no reference counterpart)
# ---------------------------------------------------------------------------
def decode_batched(Q, K_bf16_bits, V_f16_bits, row0, kv_len, n_heads, n_kv_heads, head_dim, scale):
    """smol_decode per sequence over a pooled bf16-K / fp16-V cache (oracle_decode_batched)."""
    lib = _load(ORACLE_SO)
    Q = f32(Q)
    n = len(kv_len)
    out = np.zeros((n, n_heads * head_dim), np.float32)
    K = np.ascontiguousarray(K_bf16_bits, dtype=np.uint16)
    V = np.ascontiguousarray(V_f16_bits, dtype=np.uint16)
    r0 = np.ascontiguousarray(row0, dtype=np.int64)
    kl = np.ascontiguousarray(kv_len, dtype=np.int32)
    lib.oracle_decode_batched(_p(out), _p(Q), _p(K), _p(V), _p(r0), _p(kl), _c_int(n), _c_int(n_heads),
                              _c_int(n_kv_heads), _c_int(head_dim), _c_float(scale))
    return out


def qknorm_rope_append(q, k, v, n_heads, n_kv_heads, head_dim, q_w, k_w, eps, cos_tab, sin_tab, interleaved,
                       positions, slots, k_cache_bits, v_cache_bits):
    """Fused prologue restated (oracle_qknorm_rope_append); returns rotated q, updates caches in place."""
    lib = _load(ORACLE_SO)
    q, k, v = f32(q).copy(), f32(k).copy(), f32(v)
    n = len(positions)
    pos = np.ascontiguousarray(positions, dtype=np.int32)
    sl = np.ascontiguousarray(slots, dtype=np.int64)
    qw = None if q_w is None else f32(q_w)
    kw = None if k_w is None else f32(k_w)
    ct, st = f32(cos_tab), f32(sin_tab)
    assert k_cache_bits.dtype == np.uint16 and k_cache_bits.flags["C_CONTIGUOUS"]
    assert v_cache_bits.dtype == np.uint16 and v_cache_bits.flags["C_CONTIGUOUS"]
    lib.oracle_qknorm_rope_append(_p(q), _p(k), _p(v), _c_int(n), _c_int(n_heads), _c_int(n_kv_heads),
                                  _c_int(head_dim), _p(qw), _p(kw), _c_float(eps), _p(ct), _p(st),
                                  _c_int(int(interleaved)), _p(pos), _p(sl), _p(k_cache_bits), _p(v_cache_bits))
    return q


def fill_rope_table(n_pos, head_dim, theta, interleaved=False):
    lib = _load(ORACLE_SO)
    c = np.zeros((n_pos, head_dim), np.float32)
    s = np.zeros((n_pos, head_dim), np.float32)
    lib.oracle_fill_rope_table(_p(c), _p(s), _c_int(n_pos), _c_int(head_dim), _c_float(theta),
                               _c_int(int(interleaved)))
    return c, s


def rel_l2(a, b) -> float:
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    d = np.linalg.norm(a - b)
    n = np.linalg.norm(b)
    return float(d / n) if n > 0 else float(d)
