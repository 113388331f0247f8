"""The ctypes binding (smol-genius_b200/smol_b200.py) hands each argument to the C parameter
of the same meaning.

The binding's wrappers are called with a fake library that records the arguments of
every call; each recorded argument is matched to the parameter name of
include/smol_b200.h's prototype (Part 1 repeats the reference's drop-in prototypes) and
compared with what the caller passed: a buffer's address, a size, a stride, a flag.
test_abi.py checks the argument counts and types; this checks their order -- two ints
swapped (lda and ldw, M and N) would otherwise only show up as wrong numbers on a GPU.
CPU tensors stand in for device buffers (only their addresses are used).
"""
import ctypes
import os
import re
import sys

import numpy as np
import pytest
import torch

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, os.path.join(ROOT, "smol-genius_b200"))
import smol_b200  # noqa: E402


def header_params() -> dict[str, list[str]]:
    text = re.sub(r"/\*.*?\*/", "", open(smol_b200.HEADER_PATH).read(), flags=re.S)
    out = {}
    for name, args in re.findall(r"SMOL_B200_API\s+[\w\s\*]+?\b(\w+)\s*\(([^;]*?)\)\s*;", text, flags=re.S):
        args = args.strip()
        out[name] = [] if args in ("", "void") else [re.findall(r"\w+", a)[-1] for a in args.split(",")]
    return out


PARAMS = header_params()


class FakeLib:
    """Records (name, args) of every call; returns 0, or a size for *_bytes queries."""

    def __init__(self):
        self.calls = []

    def __getattr__(self, name):
        def call(*args):
            self.calls.append((name, args))
            return 4096 if name.endswith("_bytes") else 0
        return call


@pytest.fixture
def fake(monkeypatch):
    f = FakeLib()
    monkeypatch.setattr(smol_b200, "_lib", f)
    return f


_next = iter(range(10**6))


def buf(n=8, dtype=torch.float32):
    """A distinct small tensor (its address identifies it)."""
    next(_next)
    return torch.zeros(n, dtype=dtype)


def addr(t):
    return t.data_ptr() if isinstance(t, torch.Tensor) else t.ctypes.data


def recorded(fake, fname, expect):
    """The last call must be fname and every named parameter must hold its expected value."""
    name, args = fake.calls[-1]
    assert name == fname, (name, fname)
    names = PARAMS[fname]
    assert len(args) == len(names), (fname, len(args), len(names))
    got = dict(zip(names, args))
    for k, v in expect.items():
        assert k in got, (fname, k, names)
        g = got[k]
        if hasattr(g, "_obj"):   # ctypes.byref(struct): compare the struct's address
            g = ctypes.addressof(g._obj)
        if isinstance(v, float):
            assert g == pytest.approx(v), (fname, k, g, v)
        else:
            assert g == v, (fname, k, g, v)


def test_prefill_attention_arguments(fake):
    out, q, k, v, ws = buf(), buf(dtype=torch.bfloat16), buf(dtype=torch.bfloat16), buf(dtype=torch.float16), \
        buf(3, torch.int32)
    smol_b200.prefill_attention(out, q, k, v, 3, 5, 7, 4, 2, 64, 0.125, mask_kind=smol_b200.MASK_WINDOWS,
                                q_offset=11, prefix_len=13, window=17, softcap=19.0, window_starts=ws,
                                strides=((101, 102), (103, 104), (105, 106), (107, 108)))
    recorded(fake, "smol_b200_prefill_attention", dict(
        out=addr(out), out_row_stride=101, out_batch_stride=102, q=addr(q), q_row_stride=103, q_batch_stride=104,
        k=addr(k), k_row_stride=105, k_batch_stride=106, v=addr(v), v_row_stride=107, v_batch_stride=108, batch=3,
        seq_q=5, seq_k=7, n_heads=4, n_kv_heads=2, head_dim=64, scale=0.125, mask_kind=smol_b200.MASK_WINDOWS,
        q_offset=11, prefix_len=13, window=17, softcap=19.0, window_starts=addr(ws), n_windows=2))


def test_decode_attention_arguments(fake):
    out, q, kp, vp, row0, kvl = buf(), buf(), buf(dtype=torch.bfloat16), buf(dtype=torch.float16), \
        buf(dtype=torch.int64), buf(dtype=torch.int32)
    ws = buf(64, torch.uint8)
    smol_b200.decode_attention(out, q, kp, vp, 1000, row0, kvl, 3, 77, 16, 8, 128, 0.25, ws, window=9, softcap=30.0)
    recorded(fake, "smol_b200_decode_attention", dict(
        out=addr(out), q=addr(q), q_is_bf16=0, k_pool=addr(kp), v_pool=addr(vp), pool_rows=1000,
        seq_row0=addr(row0), kv_len=addr(kvl), n_seqs=3, max_kv_len=77, n_heads=16, n_kv_heads=8, head_dim=128,
        scale=0.25, window=9, softcap=30.0, workspace=addr(ws), workspace_bytes=64))
    smol_b200.decode_attention_noalloc(out, q.bfloat16(), kp, vp, 1000, row0, kvl, 3, 77, 16, 8, 128, 0.25)
    recorded(fake, "smol_b200_decode_attention_noalloc", dict(q_is_bf16=1, pool_rows=1000, n_seqs=3, max_kv_len=77))


def test_qknorm_rope_append_arguments(fake):
    t = [buf() for _ in range(13)]
    smol_b200.qknorm_rope_append(t[0], t[1], t[2], 5, 4, 2, 64, t[3], t[4], 1e-6, t[5], t[6], True, t[7], t[8],
                                 t[9], t[10], t[11], t[12], 999)
    recorded(fake, "smol_b200_qknorm_rope_append", dict(
        q_in=addr(t[0]), k_in=addr(t[1]), v_in=addr(t[2]), n_tokens=5, n_heads=4, n_kv_heads=2, head_dim=64,
        q_norm_w=addr(t[3]), k_norm_w=addr(t[4]), eps=1e-6, rope_cos=addr(t[5]), rope_sin=addr(t[6]),
        rope_interleaved=1, positions=addr(t[7]), slots=addr(t[8]), q_out_f32=addr(t[9]), q_out_bf16=addr(t[10]),
        k_cache_bf16=addr(t[11]), v_cache_f16=addr(t[12]), cache_rows=999))


def test_decoder_step_and_prefill_arguments(fake):
    tok, fin = buf(dtype=torch.uint16 if hasattr(torch, "uint16") else torch.int16), buf()
    layer = {"wq": buf(), "down": buf(), "q_norm": buf()}
    m = smol_b200.qkn_model(1024, 16, 8, 128, 3072, 151936, 1e-6, tok, fin, [layer, layer], activation=1,
                            embed_normalizer=32.0, sliding=[1, 0])
    assert m.n_layers == 2 and m.layers[0].is_sliding == 1 and m.layers[1].is_sliding == 0
    assert m.layers[1].wq == addr(layer["wq"]) and m.layers[1].wk is None and m.activation == 1
    t_in, t_out, kp, vp, row0, kvl, cs, sn, ws = (buf() for _ in range(9))
    smol_b200.qkn_decode_step(m, 3, t_in, t_out, kp, vp, 5000, row0, kvl, 444, cs, sn, ws, advance=True)
    recorded(fake, "smol_b200_qkn_decode_step", dict(
        model=ctypes.addressof(m), n_seqs=3, tokens_in=addr(t_in), tokens_out=addr(t_out), k_pool=addr(kp),
        v_pool=addr(vp), pool_rows=5000, layer_row0=addr(row0), kv_len=addr(kvl), max_kv_len=444,
        rope_cos=addr(cs), rope_sin=addr(sn), advance=1, workspace=addr(ws), workspace_bytes=32))
    row0_host = np.arange(2, dtype=np.int64) * 100
    smol_b200.qkn_prefill(m, t_in, 7, 3, kp, vp, 5000, row0_host, cs, sn, ws)
    name, args = fake.calls[-1]
    got = dict(zip(PARAMS[name], args))
    assert name == "smol_b200_qkn_prefill"
    assert (got["n_tokens"], got["start"], got["pool_rows"], got["workspace_bytes"]) == (7, 3, 5000, 32)
    assert got["tokens"] == addr(t_in) and got["k_pool"] == addr(kp) and got["rope_sin"] == addr(sn)
    assert got["layer_row0_host"] is not None


def test_gemv_and_argmax_arguments(fake):
    y, x, w, ws = buf(), buf(), buf(), buf(16)
    smol_b200.gemv_bf16(y, 11, x, 13, w, 17, 19, 3, mode=2)
    recorded(fake, "smol_b200_gemv_bf16", dict(y=addr(y), ldy=11, x=addr(x), ldx=13, w=addr(w), n_out=17, k_dim=19,
                                               n_seqs=3, mode=2))
    smol_b200.argmax_bf16(y, x, 13, w, 1000, 19, 3, ws)
    recorded(fake, "smol_b200_argmax_bf16", dict(tokens_out=addr(y), x=addr(x), ldx=13, emb=addr(w), vocab=1000,
                                                 k_dim=19, n_seqs=3, workspace=addr(ws), workspace_bytes=64))


def test_gemm_and_layer_norm_arguments(fake):
    out, a, w, bias, add = buf(), buf(), buf(), buf(), buf()
    smol_b200.gemm_bf16(out, 11, smol_b200.GEMM_OUT_F32_ADD, a, 13, w, 17, 3, 5, 7, bias=bias, add=add, ld_add=19,
                        add_rows=23, gelu=True)
    recorded(fake, "smol_b200_gemm_bf16", dict(
        out=addr(out), ldo=11, out_kind=smol_b200.GEMM_OUT_F32_ADD, a=addr(a), lda=13, w=addr(w), ldw=17,
        bias=addr(bias), add=addr(add), ld_add=19, add_rows=23, m=3, n=5, k=7, act=smol_b200.ACT_GELU))
    smol_b200.gemm_bf16(out, 11, smol_b200.GEMM_OUT_BF16, a, 13, w, 17, 3, 6, 7, act=smol_b200.ACT_GEGLU_PAIRS)
    recorded(fake, "smol_b200_gemm_bf16", dict(bias=None, add=None, n=6, act=smol_b200.ACT_GEGLU_PAIRS))
    x, g, b = buf(), buf(), buf()
    smol_b200.layer_norm(out, x, g, b, 9, 768, 1e-6, out_bf16=True)
    recorded(fake, "smol_b200_layer_norm", dict(out=addr(out), out_bf16=1, x=addr(x), w=addr(g), b=addr(b), rows=9,
                                                hidden=768, eps=1e-6))


def test_siglip_and_encoder_arguments(fake):
    names = [n for n, _ in smol_b200.SiglipLayer._fields_]
    layer = {n: buf() for n in names}
    pw, pb, pos, post_w, post_b = (buf() for _ in range(5))
    m = smol_b200.siglip_model(768, 12, 3072, 16, 512, 1024, 1e-6, pw, 768, pb, pos, post_w, post_b, [layer])
    assert (m.hidden, m.heads, m.ffn, m.n_layers, m.patch, m.image_size, m.num_positions, m.patch_ld) == \
        (768, 12, 3072, 1, 16, 512, 1024, 768)
    assert m.patch_w == addr(pw) and m.pos == addr(pos) and m.layers[0].fc2 == addr(layer["fc2"])
    out, images, ws = buf(), buf(), buf(32)
    smol_b200.siglip_forward(out, images, 3, m, ws)
    recorded(fake, "smol_b200_siglip_forward", dict(out=addr(out), images=addr(images), n_images=3,
                                                    model=ctypes.addressof(m), workspace=addr(ws),
                                                    workspace_bytes=128))
    arr = smol_b200.siglip_layers([layer, layer])
    x, wst = buf(), buf(3, torch.int32)
    smol_b200.encoder_layers(x, 2, 100, arr, 768, 12, 3072, 1e-5, ws, window_starts=wst)
    recorded(fake, "smol_b200_encoder_layers", dict(x=addr(x), batch=2, seq=100, layers=ctypes.addressof(arr),
                                                    n_layers=2, hidden=768, heads=12, ffn=3072, eps=1e-5,
                                                    window_starts=addr(wst), n_windows=2, workspace=addr(ws),
                                                    workspace_bytes=128))


def test_decode_step_host_arguments(fake):
    t = [buf() for _ in range(12)]
    smol_b200.decode_step_host(t[0], t[1], t[2], t[3], 3, 16, 8, 128, t[4], t[5], 1e-6, t[6], t[7], False, t[8],
                               t[9], 4000, t[10], t[11], 555, 0.0625, buf(16))
    recorded(fake, "smol_b200_decode_step_host", dict(
        out_host=addr(t[0]), q_host=addr(t[1]), k_host=addr(t[2]), v_host=addr(t[3]), n_seqs=3, n_heads=16,
        n_kv_heads=8, head_dim=128, q_norm_w=addr(t[4]), k_norm_w=addr(t[5]), eps=1e-6, rope_cos=addr(t[6]),
        rope_sin=addr(t[7]), rope_interleaved=0, k_pool=addr(t[8]), v_pool=addr(t[9]), pool_rows=4000,
        seq_row0=addr(t[10]), kv_len=addr(t[11]), max_kv_len=555, scale=0.0625, scratch_bytes=64))


def test_dropin_entry_point_arguments(fake):
    out, q, k, v = buf(), buf(), buf(), buf()
    smol_b200.causal_attention(out, q, k, v, 3, 5, 4, 2, 64, 0.125, 7, window=11, cap=13.0)
    recorded(fake, "smol_sliding_window_attention_softcap", dict(
        out=addr(out), Q=addr(q), K=addr(k), V=addr(v), seq_q=3, seq_k=5, n_heads=4, n_kv_heads=2, head_dim=64,
        scale=0.125, q_offset=7, window_size=11, cap=13.0))
    smol_b200.causal_attention(out, q, k, v, 3, 5, 4, 2, 64, 0.125, 7, cap=13.0)
    recorded(fake, "smol_causal_attention_softcap", dict(q_offset=7, cap=13.0))
    smol_b200.causal_attention(out, q, k, v, 3, 5, 4, 2, 64, 0.125, 7, window=11)
    recorded(fake, "smol_sliding_window_attention", dict(q_offset=7, window_size=11))
    smol_b200.causal_attention(out, q, k, v, 3, 5, 4, 2, 64, 0.125, 7)
    recorded(fake, "smol_causal_attention", dict(seq_q=3, seq_k=5, q_offset=7))
    smol_b200.bidirectional_attention(out, q, k, v, 9, 4, 64, 0.5, [0, 4, 9])
    recorded(fake, "smol_bidirectional_attention", dict(out=addr(out), Q=addr(q), seq=9, n_heads=4, head_dim=64,
                                                        scale=0.5, n_windows=2))
    cs, sn, pos = buf(), buf(), buf(4, torch.int32)
    smol_b200.compute_rope(cs, sn, pos, 4, 64, 1e4, interleaved=True)
    recorded(fake, "smol_compute_rope_interleaved", dict(cos_out=addr(cs), sin_out=addr(sn), positions=addr(pos),
                                                         seq=4, head_dim=64, theta=1e4))
    w = buf()
    smol_b200.rms_norm(out, q, w, 3, 64, 1e-6)
    recorded(fake, "smol_rms_norm", dict(out=addr(out), x=addr(q), weight=addr(w), seq_len=3, hidden=64, eps=1e-6))


def test_every_header_function_has_named_parameters():
    assert PARAMS and all(all(re.fullmatch(r"\w+", p) for p in ps) for ps in PARAMS.values())
