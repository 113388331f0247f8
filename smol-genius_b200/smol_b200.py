"""smol_b200 -- Python binding of libsmol_b200.so (the C ABI in include/smol_b200.h).

This is the ctypes stub a Python caller of the reference would bind
(``ctypes.CDLL("libsmol_b200.so")``), with typed wrappers for tests and bench.py.
Device buffers are passed as torch CUDA tensors (torch is used for allocation and
streams only); host buffers of the drop-in entry points are numpy float32 arrays.

The product path is the CUDA library: if ``libsmol_b200.so`` is missing this module
raises instead of computing anything on the CPU.
"""
from __future__ import annotations

import ctypes
import os
import re
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
# SMOL_B200_LIB points the binding at another build of the library (e.g. a tuning variant).
LIB_PATH = os.environ.get("SMOL_B200_LIB") or os.path.join(HERE, "libsmol_b200.so")
HEADER_PATH = os.path.join(os.path.dirname(HERE), "include", "smol_b200.h")

MASK_CAUSAL, MASK_PREFIX_LM, MASK_WINDOWS, MASK_FULL = 0, 1, 2, 3

ERR_NAMES = {0: "ok", 1: "args", 2: "cuda", 3: "no_device", 4: "oom", 5: "watchdog", 6: "workspace", 7: "range"}
DEVERR_VALUE_RANGE = 1 << 6   # device error word: a value stored as fp16 had |x| >= 65520


class SmolB200Error(RuntimeError):
    """A call into libsmol_b200 returned a non-zero status."""


_lib = None

_c_int, _c_float, _c_void = ctypes.c_int, ctypes.c_float, ctypes.c_void_p
_c_i64, _c_size = ctypes.c_int64, ctypes.c_size_t
_fp = ctypes.POINTER(ctypes.c_float)
_ip = ctypes.POINTER(ctypes.c_int)

# name -> (restype, argtypes)
_SIGNATURES = {
    # Part 1 (smol_kernels.h)
    "smol_bidirectional_attention": (None, [_c_void] * 4 + [_c_int, _c_int, _c_int, _c_float, _c_void, _c_int]),
    "smol_causal_attention": (None, [_c_void] * 4 + [_c_int] * 5 + [_c_float, _c_int]),
    "smol_sliding_window_attention": (None, [_c_void] * 4 + [_c_int] * 5 + [_c_float, _c_int, _c_int]),
    "smol_causal_attention_softcap": (None, [_c_void] * 4 + [_c_int] * 5 + [_c_float, _c_int, _c_float]),
    "smol_sliding_window_attention_softcap": (
        None, [_c_void] * 4 + [_c_int] * 5 + [_c_float, _c_int, _c_int, _c_float]),
    "smol_sinusoidal_pe": (None, [_c_void, _c_int, _c_int]),
    "smol_compute_rope_neox": (None, [_c_void, _c_void, _c_void, _c_int, _c_int, _c_float]),
    "smol_compute_rope_interleaved": (None, [_c_void, _c_void, _c_void, _c_int, _c_int, _c_float]),
    "smol_apply_rope_neox": (None, [_c_void, _c_void, _c_void, _c_int, _c_int, _c_int]),
    "smol_apply_rope_interleaved": (None, [_c_void, _c_void, _c_void, _c_int, _c_int, _c_int]),
    "smol_rms_norm": (None, [_c_void, _c_void, _c_void, _c_int, _c_int, _c_float]),
    "smol_rms_norm_per_head": (None, [_c_void, _c_void, _c_int, _c_int, _c_int, _c_float]),
    # Part 2
    "smol_cuda_last_error": (_c_int, []),
    "smol_cuda_error_string": (ctypes.c_char_p, [_c_int]),
    "smol_cuda_clear_error": (None, []),
    "smol_cuda_device_error": (ctypes.c_uint, []),
    "smol_b200_watchdog_selftest": (_c_int, [_c_void]),
    # Part 3
    "smol_b200_qknorm_rope_append": (
        _c_int, [_c_void, _c_void, _c_void, _c_void, _c_int, _c_int, _c_int, _c_int, _c_void, _c_void, _c_float,
                 _c_void, _c_void, _c_int, _c_void, _c_void, _c_void, _c_void, _c_void, _c_void, _c_i64]),
    "smol_b200_decode_workspace_bytes": (_c_size, [_c_int] * 5),
    "smol_b200_decode_attention": (
        _c_int, [_c_void, _c_void, _c_void, _c_int, _c_void, _c_void, _c_i64, _c_void, _c_void, _c_int, _c_int,
                 _c_int, _c_int, _c_int, _c_float, _c_int, _c_float, _c_void, _c_size]),
    "smol_b200_decode_attention_noalloc": (
        _c_int, [_c_void, _c_void, _c_void, _c_int, _c_void, _c_void, _c_i64, _c_void, _c_void, _c_int, _c_int,
                 _c_int, _c_int, _c_int, _c_float, _c_int, _c_float]),
    "smol_b200_prefill_attention": (
        _c_int, [_c_void, _c_void, _c_i64, _c_i64, _c_void, _c_i64, _c_i64, _c_void, _c_i64, _c_i64, _c_void, _c_i64,
                 _c_i64, _c_int, _c_int, _c_int, _c_int, _c_int, _c_int, _c_float, _c_int, _c_int, _c_int, _c_int,
                 _c_float, _c_void, _c_int]),
    "smol_b200_prefill_attention_bf16": (
        _c_int, [_c_void, _c_void, _c_i64, _c_i64, _c_void, _c_i64, _c_i64, _c_void, _c_i64, _c_i64, _c_void, _c_i64,
                 _c_i64, _c_int, _c_int, _c_int, _c_int, _c_int, _c_int, _c_float, _c_int, _c_int, _c_int, _c_int,
                 _c_float, _c_void, _c_int]),
    "smol_b200_decode_step_scratch_bytes": (_c_size, [_c_int] * 5),
    "smol_b200_decode_step_host": (
        _c_int, [_c_void, _c_void, _c_void, _c_void, _c_void, _c_int, _c_int, _c_int, _c_int, _c_void, _c_void,
                 _c_float, _c_void, _c_void, _c_int, _c_void, _c_void, _c_i64, _c_void, _c_void, _c_int, _c_float,
                 _c_void, _c_size]),
    # Part 4 (device-resident decoder step)
    "smol_b200_qkn_step_workspace_bytes": (_c_size, [_c_void, _c_int, _c_int]),
    "smol_b200_qkn_prefill_workspace_bytes": (_c_size, [_c_void, _c_int]),
    "smol_b200_qkn_prefill_embeds": (_c_int, [_c_void, _c_void, _c_void, _c_int, _c_int, _c_void, _c_void, _c_i64,
                                              _c_void, _c_void, _c_void, _c_void, _c_size]),
    "smol_b200_qkn_decode_step_embeds": (
        _c_int, [_c_void, _c_void, _c_int, _c_void, _c_void, _c_void, _c_void, _c_i64, _c_void, _c_void, _c_int,
                 _c_void, _c_void, _c_int, _c_void, _c_size, _c_void]),
    "smol_b200_device_alloc": (_c_void, [_c_size]),
    "smol_b200_device_free": (None, [_c_void]),
    "smol_b200_copy": (_c_int, [_c_void, _c_void, _c_size]),
    "smol_b200_qkn_prefill": (_c_int, [_c_void, _c_void, _c_void, _c_int, _c_int, _c_void, _c_void, _c_i64, _c_void,
                                       _c_void, _c_void, _c_void, _c_size]),
    "smol_b200_qkn_decode_step": (
        _c_int, [_c_void, _c_void, _c_int, _c_void, _c_void, _c_void, _c_void, _c_i64, _c_void, _c_void, _c_int,
                 _c_void, _c_void, _c_int, _c_void, _c_size]),
    "smol_b200_gemv_bf16": (_c_int, [_c_void, _c_void, _c_i64, _c_void, _c_i64, _c_void, _c_int, _c_int, _c_int,
                                     _c_int]),
    "smol_b200_argmax_bf16": (_c_int, [_c_void, _c_void, _c_void, _c_i64, _c_void, _c_int, _c_int, _c_int, _c_void,
                                       _c_size]),
    "smol_b200_argmax_workspace_bytes": (_c_size, [_c_int, _c_int]),
    "smol_b200_prefill_attention_multi": (
        _c_int, [_c_void, _c_void, _c_int, _c_i64, _c_i64, _c_void, _c_i64, _c_i64, _c_void, _c_i64, _c_i64, _c_void,
                 _c_i64, _c_i64, _c_int, _c_int, _c_int, _c_int, _c_int, _c_int, _c_float, _c_int, _c_int, _c_int,
                 _c_int, _c_float, _c_void, _c_int]),
    "smol_b200_prefill_attention_multi_bf16": (
        _c_int, [_c_void, _c_void, _c_int, _c_i64, _c_i64, _c_void, _c_i64, _c_i64, _c_void, _c_i64, _c_i64, _c_void,
                 _c_i64, _c_i64, _c_int, _c_int, _c_int, _c_int, _c_int, _c_int, _c_float, _c_int, _c_int, _c_int,
                 _c_int, _c_float, _c_void, _c_int]),
    "smol_b200_ipc_get_handle": (_c_int, [_c_void, _c_void, ctypes.POINTER(ctypes.c_size_t)]),
    "smol_b200_ipc_open_handle": (_c_int, [_c_void, ctypes.POINTER(ctypes.c_void_p)]),
    "smol_b200_ipc_close": (_c_int, [_c_void]),
    # Part 5 (SigLIP encoder)
    "smol_b200_siglip_workspace_bytes": (_c_size, [_c_void, _c_int]),
    "smol_b200_siglip_forward": (_c_int, [_c_void, _c_void, _c_void, _c_int, _c_void, _c_void, _c_size]),
    "smol_b200_encoder_workspace_bytes": (_c_size, [_c_int, _c_int, _c_int]),
    "smol_b200_encoder_layers": (_c_int, [_c_void, _c_void, _c_int, _c_int, _c_void, _c_int, _c_int, _c_int, _c_int,
                                          _c_float, _c_void, _c_int, _c_void, _c_size]),
    "smol_b200_gemm_bf16": (_c_int, [_c_void, _c_void, _c_i64, _c_int, _c_void, _c_i64, _c_void, _c_i64, _c_void,
                                     _c_void, _c_i64, _c_int, _c_int, _c_int, _c_int, _c_int]),
    "smol_b200_layer_norm": (_c_int, [_c_void, _c_void, _c_int, _c_void, _c_void, _c_void, _c_int, _c_int,
                                      _c_float]),
}


def header_symbols(path: str = HEADER_PATH) -> list[str]:
    """Names of every function include/smol_b200.h declares with SMOL_B200_API."""
    text = open(path).read()
    return re.findall(r"SMOL_B200_API\s+[\w\s\*]+?\b(\w+)\s*\(", text)


def lib() -> ctypes.CDLL:
    """The loaded library (raises SmolB200Error when it has not been built)."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise SmolB200Error(f"{LIB_PATH} is missing: build it with `make -C smol-genius_b200` "
                                "(there is no CPU fallback)")
        l = ctypes.CDLL(LIB_PATH)
        for name, (res, args) in _SIGNATURES.items():
            f = getattr(l, name)
            f.restype = res
            f.argtypes = args
        _lib = l
    return _lib


def _ptr(x) -> int | None:
    """Address of a torch tensor / numpy array (None -> NULL)."""
    if x is None:
        return None
    if isinstance(x, int):
        return x
    if isinstance(x, np.ndarray):
        if not x.flags["C_CONTIGUOUS"]:
            raise ValueError("numpy arrays passed to libsmol_b200 must be C-contiguous")
        return x.ctypes.data
    return x.data_ptr()


def _stream(stream) -> int | None:
    """The CUDA stream handle to launch on.  None means torch's current stream when
    torch has initialised CUDA in this process (so calls inside `torch.cuda.stream(s)`
    or `torch.cuda.graph(g)` land on that stream and can be captured), else the
    legacy default stream (NULL)."""
    if stream is None:
        torch = sys.modules.get("torch")
        if torch is not None and torch.cuda.is_initialized():
            return torch.cuda.current_stream().cuda_stream or None
        return None
    if isinstance(stream, int):
        return stream
    return stream.cuda_stream


def check(rc: int, what: str) -> None:
    if rc != 0:
        raise SmolB200Error(f"{what} failed: {ERR_NAMES.get(rc, rc)} "
                            f"({lib().smol_cuda_error_string(rc).decode()})")


def last_error() -> int:
    return lib().smol_cuda_last_error()


def clear_error() -> None:
    lib().smol_cuda_clear_error()


def device_error() -> int:
    return lib().smol_cuda_device_error()


def watchdog_selftest(stream=None) -> int:
    return lib().smol_b200_watchdog_selftest(_stream(stream))


# ---------------------------------------------------------------------------
# Part 1: drop-in entry points (host numpy or device torch buffers)
# ---------------------------------------------------------------------------
def causal_attention(out, Q, K, V, seq_q, seq_k, n_heads, n_kv_heads, head_dim, scale, q_offset,
                     window=0, cap=0.0):
    L = lib()
    a = (_ptr(out), _ptr(Q), _ptr(K), _ptr(V), seq_q, seq_k, n_heads, n_kv_heads, head_dim, scale, q_offset)
    if window > 0 and cap > 0:
        L.smol_sliding_window_attention_softcap(*a, window, cap)
    elif window > 0:
        L.smol_sliding_window_attention(*a, window)
    elif cap > 0:
        L.smol_causal_attention_softcap(*a, cap)
    else:
        L.smol_causal_attention(*a)


def bidirectional_attention(out, Q, K, V, seq, n_heads, head_dim, scale, window_starts):
    ws = np.ascontiguousarray(window_starts, dtype=np.int32)
    lib().smol_bidirectional_attention(_ptr(out), _ptr(Q), _ptr(K), _ptr(V), seq, n_heads, head_dim, scale,
                                       _ptr(ws), len(ws) - 1)


def apply_rope(x, cos, sin, seq, n_heads, head_dim, interleaved=False):
    f = lib().smol_apply_rope_interleaved if interleaved else lib().smol_apply_rope_neox
    f(_ptr(x), _ptr(cos), _ptr(sin), seq, n_heads, head_dim)


def compute_rope(cos_out, sin_out, positions, seq, head_dim, theta, interleaved=False):
    f = lib().smol_compute_rope_interleaved if interleaved else lib().smol_compute_rope_neox
    f(_ptr(cos_out), _ptr(sin_out), _ptr(positions), seq, head_dim, theta)


def rms_norm_per_head(x, w, seq, n_heads, head_dim, eps):
    lib().smol_rms_norm_per_head(_ptr(x), _ptr(w), seq, n_heads, head_dim, eps)


def rms_norm(out, x, w, seq, hidden, eps):
    lib().smol_rms_norm(_ptr(out), _ptr(x), _ptr(w), seq, hidden, eps)


def sinusoidal_pe(pe, n_pos, d_model):
    lib().smol_sinusoidal_pe(_ptr(pe), n_pos, d_model)


# ---------------------------------------------------------------------------
# Part 3: device API (torch CUDA tensors)
# ---------------------------------------------------------------------------
def qknorm_rope_append(q_in, k_in, v_in, n_tokens, n_heads, n_kv_heads, head_dim, q_norm_w, k_norm_w, eps,
                       rope_cos, rope_sin, interleaved, positions, slots, q_out_f32, q_out_bf16, k_cache, v_cache,
                       cache_rows, stream=None):
    rc = lib().smol_b200_qknorm_rope_append(
        _stream(stream), _ptr(q_in), _ptr(k_in), _ptr(v_in), n_tokens, n_heads, n_kv_heads, head_dim,
        _ptr(q_norm_w), _ptr(k_norm_w), eps, _ptr(rope_cos), _ptr(rope_sin), int(interleaved), _ptr(positions),
        _ptr(slots), _ptr(q_out_f32), _ptr(q_out_bf16), _ptr(k_cache), _ptr(v_cache), cache_rows)
    check(rc, "smol_b200_qknorm_rope_append")


def decode_workspace_bytes(n_seqs, max_kv_len, n_heads, n_kv_heads, head_dim) -> int:
    return lib().smol_b200_decode_workspace_bytes(n_seqs, max_kv_len, n_heads, n_kv_heads, head_dim)


def decode_attention(out, q, k_pool, v_pool, pool_rows, seq_row0, kv_len, n_seqs, max_kv_len, n_heads, n_kv_heads,
                     head_dim, scale, workspace, window=0, softcap=0.0, stream=None):
    import torch
    q_is_bf16 = 1 if q.dtype == torch.bfloat16 else 0
    rc = lib().smol_b200_decode_attention(
        _stream(stream), _ptr(out), _ptr(q), q_is_bf16, _ptr(k_pool), _ptr(v_pool), pool_rows, _ptr(seq_row0),
        _ptr(kv_len), n_seqs, max_kv_len, n_heads, n_kv_heads, head_dim, scale, window, softcap, _ptr(workspace),
        workspace.numel() * workspace.element_size())
    check(rc, "smol_b200_decode_attention")


def decode_attention_noalloc(out, q, k_pool, v_pool, pool_rows, seq_row0, kv_len, n_seqs, max_kv_len, n_heads,
                             n_kv_heads, head_dim, scale, window=0, softcap=0.0, stream=None) -> int:
    """Allocation-free form of decode_attention (partials in the library's static array).
    Returns the status code instead of raising, so callers can test the size limit."""
    import torch
    q_is_bf16 = 1 if q.dtype == torch.bfloat16 else 0
    return lib().smol_b200_decode_attention_noalloc(
        _stream(stream), _ptr(out), _ptr(q), q_is_bf16, _ptr(k_pool), _ptr(v_pool), pool_rows, _ptr(seq_row0),
        _ptr(kv_len), n_seqs, max_kv_len, n_heads, n_kv_heads, head_dim, scale, window, softcap)


def prefill_attention(out, q, k, v, batch, seq_q, seq_k, n_heads, n_kv_heads, head_dim, scale, mask_kind=MASK_CAUSAL,
                      q_offset=0, prefix_len=0, window=0, softcap=0.0, window_starts=None, stream=None,
                      strides=None):
    """q/k: bf16 [batch, seq, heads*hd]; v: fp16; out: fp32 [batch, seq_q, n_heads*hd] (contiguous unless
    `strides` = ((out_row, out_batch), (q_row, q_batch), (k_row, k_batch), (v_row, v_batch)) in elements).
    A bf16 `out` selects smol_b200_prefill_attention_bf16."""
    import torch
    if strides is None:
        qw, kw = n_heads * head_dim, n_kv_heads * head_dim
        strides = ((qw, seq_q * qw), (qw, seq_q * qw), (kw, seq_k * kw), (kw, seq_k * kw))
    (ors, obs), (qrs, qbs), (krs, kbs), (vrs, vbs) = strides
    nw = 0 if window_starts is None else window_starts.numel() - 1
    name = "smol_b200_prefill_attention_bf16" if out.dtype == torch.bfloat16 else "smol_b200_prefill_attention"
    rc = getattr(lib(), name)(
        _stream(stream), _ptr(out), ors, obs, _ptr(q), qrs, qbs, _ptr(k), krs, kbs, _ptr(v), vrs, vbs, batch, seq_q,
        seq_k, n_heads, n_kv_heads, head_dim, scale, mask_kind, q_offset, prefix_len, window, softcap,
        _ptr(window_starts), nw)
    check(rc, name)


def decode_step_scratch_bytes(n_seqs, max_kv_len, n_heads, n_kv_heads, head_dim) -> int:
    return lib().smol_b200_decode_step_scratch_bytes(n_seqs, max_kv_len, n_heads, n_kv_heads, head_dim)


def decode_step_host(out_host, q_host, k_host, v_host, n_seqs, n_heads, n_kv_heads, head_dim, q_norm_w, k_norm_w, eps,
                     rope_cos, rope_sin, interleaved, k_pool, v_pool, pool_rows, seq_row0, kv_len, max_kv_len, scale,
                     scratch, stream=None):
    rc = lib().smol_b200_decode_step_host(
        _stream(stream), _ptr(out_host), _ptr(q_host), _ptr(k_host), _ptr(v_host), n_seqs, n_heads, n_kv_heads,
        head_dim, _ptr(q_norm_w), _ptr(k_norm_w), eps, _ptr(rope_cos), _ptr(rope_sin), int(interleaved),
        _ptr(k_pool), _ptr(v_pool), pool_rows, _ptr(seq_row0), _ptr(kv_len), max_kv_len, scale, _ptr(scratch),
        scratch.numel() * scratch.element_size())
    check(rc, "smol_b200_decode_step_host")


# ---------------------------------------------------------------------------
# Part 4: device-resident decoder step
# ---------------------------------------------------------------------------
class QknLayer(ctypes.Structure):
    """smol_b200_qkn_layer: device pointers of one layer's weights (Gemma fields NULL / 0 for Qwen3)."""
    _fields_ = [("wq", ctypes.c_void_p), ("wk", ctypes.c_void_p), ("wv", ctypes.c_void_p), ("wo", ctypes.c_void_p),
                ("gate_up", ctypes.c_void_p), ("down", ctypes.c_void_p), ("input_norm", ctypes.c_void_p),
                ("post_attn_norm", ctypes.c_void_p), ("q_norm", ctypes.c_void_p), ("k_norm", ctypes.c_void_p),
                ("pre_ffn_norm", ctypes.c_void_p), ("post_ffn_norm", ctypes.c_void_p), ("is_sliding", ctypes.c_int)]


class QknModel(ctypes.Structure):
    """smol_b200_qkn_model (the layers array stays referenced by the Python object)."""
    _fields_ = [("hidden", ctypes.c_int), ("n_layers", ctypes.c_int), ("n_heads", ctypes.c_int),
                ("n_kv_heads", ctypes.c_int), ("head_dim", ctypes.c_int), ("intermediate", ctypes.c_int),
                ("vocab", ctypes.c_int), ("eps", ctypes.c_float), ("rope_interleaved", ctypes.c_int),
                ("tok_embeddings", ctypes.c_void_p), ("final_norm", ctypes.c_void_p),
                ("layers", ctypes.POINTER(QknLayer)), ("activation", ctypes.c_int),
                ("embed_normalizer", ctypes.c_float), ("attn_softcap", ctypes.c_float),
                ("sliding_window", ctypes.c_int), ("rope_cos_local", ctypes.c_void_p),
                ("rope_sin_local", ctypes.c_void_p), ("lm_head", ctypes.c_void_p)]


ACT_SWIGLU, ACT_GEGLU = 0, 1


def qkn_model(hidden, n_heads, n_kv_heads, head_dim, intermediate, vocab, eps, tok_embeddings, final_norm, layers,
              rope_interleaved=False, activation=ACT_SWIGLU, embed_normalizer=0.0, attn_softcap=0.0,
              sliding_window=0, rope_cos_local=None, rope_sin_local=None, sliding=None, lm_head=None) -> QknModel:
    """layers: list of dicts mapping QknLayer pointer field names to device tensors (absent
    names -> NULL); sliding: per-layer is_sliding flags (default all 0)."""
    arr = (QknLayer * len(layers))()
    for i, lw in enumerate(layers):
        for name, ctype in QknLayer._fields_:
            if ctype is ctypes.c_void_p:
                setattr(arr[i], name, _ptr(lw.get(name)))
        arr[i].is_sliding = int(bool(sliding[i])) if sliding is not None else 0
    m = QknModel(hidden, len(layers), n_heads, n_kv_heads, head_dim, intermediate, vocab, eps, int(rope_interleaved),
                 _ptr(tok_embeddings), _ptr(final_norm), ctypes.cast(arr, ctypes.POINTER(QknLayer)), int(activation),
                 float(embed_normalizer), float(attn_softcap), int(sliding_window), _ptr(rope_cos_local),
                 _ptr(rope_sin_local), _ptr(lm_head))
    m._layers = arr   # keep the array alive with the struct
    return m


def qkn_prefill_workspace_bytes(model: QknModel, n_tokens: int) -> int:
    return lib().smol_b200_qkn_prefill_workspace_bytes(ctypes.byref(model), n_tokens)


def qkn_prefill(model: QknModel, tokens, n_tokens, start, k_pool, v_pool, pool_rows, layer_row0_host, rope_cos,
                rope_sin, workspace, stream=None):
    """layer_row0_host: numpy int64 [n_layers] (host); tokens, pools, tables, workspace on the device."""
    row0 = np.ascontiguousarray(layer_row0_host, dtype=np.int64)
    rc = lib().smol_b200_qkn_prefill(_stream(stream), ctypes.byref(model), _ptr(tokens), n_tokens, start, _ptr(k_pool),
                                     _ptr(v_pool), pool_rows, _ptr(row0), _ptr(rope_cos), _ptr(rope_sin),
                                     _ptr(workspace), workspace.numel() * workspace.element_size())
    check(rc, "smol_b200_qkn_prefill")


def qkn_step_workspace_bytes(model: QknModel, n_seqs: int, max_kv_len: int) -> int:
    return lib().smol_b200_qkn_step_workspace_bytes(ctypes.byref(model), n_seqs, max_kv_len)


def qkn_decode_step(model: QknModel, n_seqs, tokens_in, tokens_out, k_pool, v_pool, pool_rows, layer_row0, kv_len,
                    max_kv_len, rope_cos, rope_sin, workspace, advance=False, stream=None):
    rc = lib().smol_b200_qkn_decode_step(
        _stream(stream), ctypes.byref(model), n_seqs, _ptr(tokens_in), _ptr(tokens_out), _ptr(k_pool), _ptr(v_pool),
        pool_rows, _ptr(layer_row0), _ptr(kv_len), max_kv_len, _ptr(rope_cos), _ptr(rope_sin), int(advance),
        _ptr(workspace), workspace.numel() * workspace.element_size())
    check(rc, "smol_b200_qkn_decode_step")


def gemv_bf16(y, ldy, x, ldx, w, n_out, k_dim, n_seqs, mode=0, stream=None):
    check(lib().smol_b200_gemv_bf16(_stream(stream), _ptr(y), ldy, _ptr(x), ldx, _ptr(w), n_out, k_dim, n_seqs, mode),
          "smol_b200_gemv_bf16")


def argmax_workspace_bytes(n_seqs: int, vocab: int) -> int:
    return lib().smol_b200_argmax_workspace_bytes(n_seqs, vocab)


def argmax_bf16(tokens_out, x, ldx, emb, vocab, k_dim, n_seqs, workspace, stream=None):
    check(lib().smol_b200_argmax_bf16(_stream(stream), _ptr(tokens_out), _ptr(x), ldx, _ptr(emb), vocab, k_dim, n_seqs,
                                      _ptr(workspace), workspace.numel() * workspace.element_size()),
          "smol_b200_argmax_bf16")


# ---------------------------------------------------------------------------
# Prefill with several output destinations (fused all-gather) and CUDA IPC
# ---------------------------------------------------------------------------
def prefill_attention_multi(out_ptrs, row_stride, batch_stride, q, k, v, batch, seq_q, seq_k, n_heads, n_kv_heads,
                            head_dim, scale, mask_kind=MASK_CAUSAL, q_offset=0, prefix_len=0, window=0, softcap=0.0,
                            strides=None, stream=None, bf16=False):
    """out_ptrs: device addresses (ints) of every destination, same strides (elements); fp32 elements, or bf16
    with bf16=True (smol_b200_prefill_attention_multi_bf16)."""
    if strides is None:
        strides = ((n_heads * head_dim, seq_q * n_heads * head_dim), (n_kv_heads * head_dim, seq_k * n_kv_heads * head_dim),
                   (n_kv_heads * head_dim, seq_k * n_kv_heads * head_dim))
    (qs, qb), (ks, kb), (vs, vb) = strides
    arr = (ctypes.c_void_p * len(out_ptrs))(*out_ptrs)
    name = "smol_b200_prefill_attention_multi_bf16" if bf16 else "smol_b200_prefill_attention_multi"
    rc = getattr(lib(), name)(
        _stream(stream), ctypes.cast(arr, ctypes.c_void_p), len(out_ptrs), row_stride, batch_stride, _ptr(q), qs, qb,
        _ptr(k), ks, kb, _ptr(v), vs, vb, batch, seq_q, seq_k, n_heads, n_kv_heads, head_dim, scale, mask_kind,
        q_offset, prefix_len, window, softcap, None, 0)
    check(rc, name)


def ipc_handle(t) -> tuple[bytes, int]:
    """(64-byte handle of the allocation holding t, t's byte offset inside it)."""
    buf = ctypes.create_string_buffer(64)
    off = ctypes.c_size_t()
    check(lib().smol_b200_ipc_get_handle(_ptr(t), buf, ctypes.byref(off)), "smol_b200_ipc_get_handle")
    return buf.raw, off.value


def ipc_open(handle: bytes) -> int:
    ptr = ctypes.c_void_p()
    buf = ctypes.create_string_buffer(handle, 64)
    check(lib().smol_b200_ipc_open_handle(buf, ctypes.byref(ptr)), "smol_b200_ipc_open_handle")
    return ptr.value


def ipc_close(ptr: int) -> None:
    check(lib().smol_b200_ipc_close(ptr), "smol_b200_ipc_close")


# ---------------------------------------------------------------------------
# Part 5: SigLIP encoder
# ---------------------------------------------------------------------------
GEMM_OUT_F32, GEMM_OUT_BF16, GEMM_OUT_F16, GEMM_OUT_F32_ADD = 0, 1, 2, 3
ACT_NONE, ACT_GELU, ACT_SWIGLU_PAIRS, ACT_GEGLU_PAIRS = 0, 1, 2, 3


class SiglipLayer(ctypes.Structure):
    """smol_b200_siglip_layer: device pointers of one encoder layer."""
    _fields_ = [(n, ctypes.c_void_p) for n in ("ln1_w", "ln1_b", "wq", "wk", "wv", "wo", "bq", "bk", "bv", "bo",
                                               "ln2_w", "ln2_b", "fc1", "b1", "fc2", "b2")]


class SiglipModel(ctypes.Structure):
    """smol_b200_siglip_model (the layers array stays referenced by the Python object)."""
    _fields_ = [("hidden", ctypes.c_int), ("heads", ctypes.c_int), ("ffn", ctypes.c_int), ("n_layers", ctypes.c_int),
                ("patch", ctypes.c_int), ("image_size", ctypes.c_int), ("num_positions", ctypes.c_int),
                ("eps", ctypes.c_float), ("patch_w", ctypes.c_void_p), ("patch_ld", ctypes.c_int),
                ("patch_b", ctypes.c_void_p), ("pos", ctypes.c_void_p), ("post_w", ctypes.c_void_p),
                ("post_b", ctypes.c_void_p), ("layers", ctypes.POINTER(SiglipLayer))]


def siglip_model(hidden, heads, ffn, patch, image_size, num_positions, eps, patch_w, patch_ld, patch_b, pos, post_w,
                 post_b, layers) -> SiglipModel:
    """layers: list of dicts mapping the SiglipLayer field names to device tensors."""
    arr = (SiglipLayer * len(layers))()
    for i, lw in enumerate(layers):
        for name, _ in SiglipLayer._fields_:
            setattr(arr[i], name, _ptr(lw[name]))
    m = SiglipModel(hidden, heads, ffn, len(layers), patch, image_size, num_positions, eps, _ptr(patch_w), patch_ld,
                    _ptr(patch_b), _ptr(pos), _ptr(post_w), _ptr(post_b), ctypes.cast(arr, ctypes.POINTER(SiglipLayer)))
    m._layers = arr
    return m


def siglip_layers(layers) -> ctypes.Array:
    """A SiglipLayer array from a list of dicts of device tensors (keep it referenced)."""
    arr = (SiglipLayer * len(layers))()
    for i, lw in enumerate(layers):
        for name, _ in SiglipLayer._fields_:
            setattr(arr[i], name, _ptr(lw[name]))
    return arr


def encoder_workspace_bytes(n_tokens: int, hidden: int, ffn: int) -> int:
    return lib().smol_b200_encoder_workspace_bytes(n_tokens, hidden, ffn)


def encoder_layers(x, batch, seq, layer_array, hidden, heads, ffn, eps, workspace, window_starts=None, stream=None):
    """window_starts: device int32 tensor of n_windows + 1 entries, or None (whole sequence)."""
    nw = 0 if window_starts is None else window_starts.numel() - 1
    check(lib().smol_b200_encoder_layers(_stream(stream), _ptr(x), batch, seq,
                                         ctypes.addressof(layer_array), len(layer_array), hidden,
                                         heads, ffn, eps, _ptr(window_starts), nw, _ptr(workspace),
                                         workspace.numel() * workspace.element_size()),
          "smol_b200_encoder_layers")


def siglip_workspace_bytes(model: SiglipModel, n_images: int) -> int:
    return lib().smol_b200_siglip_workspace_bytes(ctypes.byref(model), n_images)


def siglip_forward(out, images, n_images, model: SiglipModel, workspace, stream=None):
    check(lib().smol_b200_siglip_forward(_stream(stream), _ptr(out), _ptr(images), n_images, ctypes.byref(model),
                                         _ptr(workspace), workspace.numel() * workspace.element_size()),
          "smol_b200_siglip_forward")


def gemm_bf16(out, ldo, out_kind, a, lda, w, ldw, m, n, k, bias=None, add=None, ld_add=0, add_rows=0, gelu=False,
              act=None, stream=None):
    """act: ACT_* (gelu=True is ACT_GELU)."""
    a_code = act if act is not None else (ACT_GELU if gelu else ACT_NONE)
    check(lib().smol_b200_gemm_bf16(_stream(stream), _ptr(out), ldo, out_kind, _ptr(a), lda, _ptr(w), ldw, _ptr(bias),
                                    _ptr(add), ld_add, add_rows, m, n, k, a_code),
          "smol_b200_gemm_bf16")


def layer_norm(out, x, w, b, rows, hidden, eps, out_bf16=False, stream=None):
    check(lib().smol_b200_layer_norm(_stream(stream), _ptr(out), int(out_bf16), _ptr(x), _ptr(w), _ptr(b), rows,
                                     hidden, eps),
          "smol_b200_layer_norm")
