"""The C ABI of libsmol_b200.so, checked without a GPU.

* the library loads and exports every function include/smol_b200.h declares;
* the drop-in prototypes are exactly those of the reference's
  common/kernels/smol_kernels.h:86-161 (types and order of parameters);
* without a usable device a drop-in call records SMOL_B200_ERR_NO_DEVICE and
  zero-fills its output -- it never computes on the CPU.
"""
import ctypes
import os
import re
import subprocess

import numpy as np
import pytest

import smol_b200

# smol_kernels.h:86-161 -- the prototypes attention.o, rope.o and rmsnorm.o export.
REFERENCE_PROTOTYPES = """
void smol_rms_norm(float *out, const float *x, const float *weight, int seq_len, int hidden, float eps);
void smol_rms_norm_per_head(float *x, const float *weight, int seq_len, int n_heads, int head_dim, float eps);
void smol_bidirectional_attention(float *out, const float *Q, const float *K, const float *V, int seq, int n_heads, int head_dim, float scale, const int *window_starts, int n_windows);
void smol_causal_attention(float *out, const float *Q, const float *K, const float *V, int seq_q, int seq_k, int n_heads, int n_kv_heads, int head_dim, float scale, int q_offset);
void smol_sliding_window_attention(float *out, const float *Q, const float *K, const float *V, int seq_q, int seq_k, int n_heads, int n_kv_heads, int head_dim, float scale, int q_offset, int window_size);
void smol_causal_attention_softcap(float *out, const float *Q, const float *K, const float *V, int seq_q, int seq_k, int n_heads, int n_kv_heads, int head_dim, float scale, int q_offset, float cap);
void smol_sliding_window_attention_softcap(float *out, const float *Q, const float *K, const float *V, int seq_q, int seq_k, int n_heads, int n_kv_heads, int head_dim, float scale, int q_offset, int window_size, float cap);
void smol_sinusoidal_pe(float *pe, int n_pos, int d_model);
void smol_compute_rope_neox(float *cos_out, float *sin_out, const int *positions, int seq, int head_dim, float theta);
void smol_apply_rope_neox(float *x, const float *cos_vals, const float *sin_vals, int seq, int n_heads, int head_dim);
void smol_compute_rope_interleaved(float *cos_out, float *sin_out, const int *positions, int seq, int head_dim, float theta);
void smol_apply_rope_interleaved(float *x, const float *cos_vals, const float *sin_vals, int seq, int n_heads, int head_dim);
"""


def prototypes(text: str) -> dict[str, tuple[str, tuple[str, ...]]]:
    """name -> (return type, parameter types) for every smol_* prototype in C text."""
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    text = text.replace('__attribute__((visibility("default")))', "").replace("SMOL_B200_API", "")
    out = {}
    for ret, name, params in re.findall(r"(\w[\w\s\*]*?)\s*\b(smol_\w+)\s*\(([^)]*)\)\s*;", text):
        types = []
        for prm in params.split(","):
            prm = " ".join(prm.split())
            if not prm or prm == "void":
                continue
            t = re.sub(r"\b\w+$", "", prm).replace(" ", "")
            types.append(t)
        out[name] = (ret.split()[-1], tuple(types))
    return out


def test_library_exports_every_header_symbol():
    names = smol_b200.header_symbols()
    assert len(names) >= 22, names
    lib = smol_b200.lib()
    for n in names:
        assert hasattr(lib, n), n
    dyn = subprocess.run(["nm", "-D", "--defined-only", smol_b200.LIB_PATH], capture_output=True, text=True,
                         check=True).stdout
    exported = {line.split()[-1] for line in dyn.splitlines() if " T " in line}
    assert set(names) <= exported, set(names) - exported
    # nothing but the header's functions leaks out of the library
    assert {s for s in exported if s.startswith("smol")} == set(names)


def test_dropin_prototypes_match_reference():
    ours = prototypes(open(smol_b200.HEADER_PATH).read())
    want = prototypes(REFERENCE_PROTOTYPES)
    assert len(want) == 12
    for name, sig in want.items():
        assert ours.get(name) == sig, (name, ours.get(name), sig)


REF_HEADER = os.path.join(os.environ.get("SMOL_REFERENCE_DIR") or
                          os.path.join(os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__)))),
                                       "reference"), "common", "kernels", "smol_kernels.h")


@pytest.mark.skipif(not os.path.exists(REF_HEADER), reason="reference checkout not present ($SMOL_REFERENCE_DIR)")
def test_dropin_prototypes_match_reference_header_file():
    ref = prototypes(open(REF_HEADER).read())
    ours = prototypes(open(smol_b200.HEADER_PATH).read())
    for name in prototypes(REFERENCE_PROTOTYPES):
        assert ours[name] == ref[name], name


def test_error_strings():
    lib = smol_b200.lib()
    for code in range(8):
        assert lib.smol_cuda_error_string(code)
    assert lib.smol_cuda_error_string(0) == b"ok"


def test_workspace_sizes():
    a = smol_b200.decode_workspace_bytes(256, 8192, 16, 8, 128)
    b = smol_b200.decode_workspace_bytes(512, 8192, 16, 8, 128)
    assert 0 < a < b
    assert smol_b200.decode_workspace_bytes(1, 0, 16, 8, 128) > 0
    assert smol_b200.decode_step_scratch_bytes(256, 8192, 16, 8, 128) > a


def _decode_call_bytes(n_seqs, L, n_heads, n_kv_heads, hd):
    """Partials one decode call of max_kv_len L writes: the library's chunk rule (about
    8 CTAs per SM of 148, multiples of 64 keys, at most 2048) restated."""
    w = n_seqs * n_kv_heads * ((n_heads // n_kv_heads + 7) // 8)
    c = -(-w * max(L, 1) // (148 * 8))
    c = min(max(-(-c // 64) * 64, 64), 2048)
    return n_seqs * n_heads * max(-(-L // c), 1) * (hd + 2) * 4


@pytest.mark.parametrize("n_seqs,n_heads,n_kv_heads,hd", [(1, 16, 8, 128), (1, 8, 1, 256), (3, 12, 12, 64),
                                                          (256, 16, 8, 128)])
def test_decode_workspace_never_shrinks(n_seqs, n_heads, n_kv_heads, hd):
    """A workspace sized once for a cache capacity must serve every shorter call: the
    chunk grows in steps of 64 keys, so a call's own partial count is not monotonic in
    its length (Qwen3 shapes, one sequence: 9409 keys need more than 9600 would)."""
    prev = 0
    lens = list(range(1, 20001, 7)) + [9409, 9472, 9600, 20000, 65536, 300000]
    for L in sorted(set(lens)):
        got = smol_b200.decode_workspace_bytes(n_seqs, L, n_heads, n_kv_heads, hd)
        assert got >= prev, (L, got, prev)
        assert got >= _decode_call_bytes(n_seqs, L, n_heads, n_kv_heads, hd), L
        prev = got


def _siglip_model(**over):
    """A model struct with dummy (never dereferenced) device addresses: the workspace
    query only validates the shape and pointer presence."""
    fake = 1 << 20
    layer = {name: fake for name, _ in smol_b200.SiglipLayer._fields_}
    kw = dict(hidden=768, heads=12, ffn=3072, patch=16, image_size=512, num_positions=1024, eps=1e-6, patch_w=fake,
              patch_ld=768, patch_b=fake, pos=fake, post_w=fake, post_b=fake, layers=[layer, layer])
    kw.update(over)
    return smol_b200.siglip_model(**kw)


def test_qkn_model_configuration_checks():
    """Host-side rules of the Part-4 model struct: the Qwen3 and Gemma configurations are
    accepted (non-zero workspace), malformed ones are not (0: the step would return
    SMOL_B200_ERR_ARGS)."""
    fake = 1 << 20
    layer = {name: fake for name, t in smol_b200.QknLayer._fields_ if t is ctypes.c_void_p}

    def ws(**over):
        kw = dict(hidden=1024, n_heads=16, n_kv_heads=8, head_dim=128, intermediate=3072, vocab=4096, eps=1e-6,
                  tok_embeddings=fake, final_norm=fake, layers=[layer, layer])
        kw.update(over)
        return smol_b200.qkn_step_workspace_bytes(smol_b200.qkn_model(**kw), 2, 511)

    qwen = ws()
    assert qwen > 0
    assert ws(activation=smol_b200.ACT_GEGLU, embed_normalizer=32.0, attn_softcap=50.0, sliding_window=4096,
              rope_cos_local=fake, rope_sin_local=fake, sliding=[True, False], rope_interleaved=True) == qwen
    assert ws(activation=2) == 0
    assert ws(sliding_window=-1) == 0
    assert ws(rope_cos_local=fake) == 0              # one local table without the other
    assert ws(n_kv_heads=5) == 0                     # 16 heads do not split into 5 groups
    assert ws(intermediate=3070) == 0


def test_siglip_workspace_sizes_and_shape_checks():
    """Host-side shape rules of Part 5: the workspace grows with the batch and is 0 (the
    call would return SMOL_B200_ERR_ARGS) for shapes the device path does not take."""
    one = smol_b200.siglip_workspace_bytes(_siglip_model(), 1)
    assert one > 0 and smol_b200.siglip_workspace_bytes(_siglip_model(), 4) > 3 * one
    # per image: unfolded patches, 4 bf16 activations and the bf16 attention output (the
    # prefill kernel writes it in bf16 for the output projection), the bf16 fc1 output
    # (1024 patches)
    T = 1024
    assert one >= T * (768 * 2 + 5 * 768 * 2 + 3072 * 2)
    # head dims: any multiple of 8 up to 256 (the prefill kernel zero-fills the columns
    # up to its own 64/128/256), so 48 and SigLIP-So400m's 72 run; 12 and 153.6 do not
    assert smol_b200.siglip_workspace_bytes(_siglip_model(heads=16), 1) > 0            # head dim 48
    assert smol_b200.siglip_workspace_bytes(_siglip_model(heads=64), 1) == 0           # head dim 12
    assert smol_b200.siglip_workspace_bytes(_siglip_model(heads=5), 1) == 0            # 768 / 5
    so400m = dict(hidden=1152, heads=16, ffn=4304, patch=14, image_size=378, num_positions=729, patch_ld=592)
    assert smol_b200.siglip_workspace_bytes(_siglip_model(**so400m), 1) > 0             # head dim 72
    assert smol_b200.siglip_workspace_bytes(_siglip_model(num_positions=1000), 1) == 0  # fewer positions than patches
    assert smol_b200.siglip_workspace_bytes(_siglip_model(patch_ld=770), 1) == 0       # stride not a multiple of 8
    assert smol_b200.siglip_workspace_bytes(_siglip_model(ffn=3070), 1) == 0
    assert smol_b200.siglip_workspace_bytes(_siglip_model(patch_w=None), 1) == 0


def test_host_tables_match_oracle_and_reference():
    """The RoPE tables and sinusoidal embeddings of Part 1 are built on the host (every
    device path only indexes them): bit for bit the oracle's, and the reference's golden
    tables within the one-ulp frequency difference of its -ffast-math build
    (2e-6 + 1.2e-7 * position)."""
    import pyoracle
    golden = np.load(os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "reference_cases.npz"))
    o = pyoracle.oracle()
    pos = np.arange(4096, dtype=np.int32)
    for inter in (False, True):
        for hd, theta in ((128, 1e6), (256, 1e4), (80, 1e4)):
            c = np.zeros((len(pos), hd), np.float32)
            s = np.zeros_like(c)
            smol_b200.compute_rope(c, s, pos, len(pos), hd, theta, interleaved=inter)
            c2, s2 = o.compute_rope(pos, hd, theta, interleaved=inter)
            assert np.array_equal(c, c2) and np.array_equal(s, s2), (inter, hd)
    for name in ("rope_neox", "rope_interleaved", "rope_neox_odd"):
        hd, inter = (int(x) for x in golden[f"{name}/meta"])
        p = golden[f"{name}/pos"].astype(np.int32)
        c = np.zeros((len(p), hd), np.float32)
        s = np.zeros_like(c)
        smol_b200.compute_rope(c, s, p, len(p), hd, float(golden[f"{name}/fmeta"][0]), interleaved=bool(inter))
        bound = (2e-6 + 1.2e-7 * p.astype(np.float64))[:, None]
        assert np.all(np.abs(c - golden[f"{name}/cos"]) <= bound) and np.all(np.abs(s - golden[f"{name}/sin"]) <= bound)
    pe = np.zeros((9, 32), np.float32)
    smol_b200.sinusoidal_pe(pe, 9, 32)
    assert np.allclose(pe, golden["sinusoidal/out"], rtol=1e-6, atol=1e-6)
    assert smol_b200.last_error() == 0


def test_gemm_argument_rules():
    """smol_b200_gemm_bf16 refuses what its kernel cannot take before touching a device
    (1 = SMOL_B200_ERR_ARGS): activations out of range, gated pairs with an odd N or a
    residual add, unaligned operands or strides, K <= 0, short leading dimensions.  A
    well-formed call gets as far as the device (3 = SMOL_B200_ERR_NO_DEVICE here)."""
    import torch
    if torch.cuda.is_available():
        pytest.skip("the addresses below are placeholders: never hand them to a device")
    L = smol_b200.lib()
    base = 1 << 20   # 16-byte aligned placeholder addresses, never dereferenced without a device

    def gemm(**over):
        kw = dict(out=base, ldo=256, out_kind=smol_b200.GEMM_OUT_F32, a=base, lda=128, w=base, ldw=128, bias=None,
                  add=None, ld_add=0, add_rows=0, m=64, n=256, k=128, act=smol_b200.ACT_NONE)
        kw.update(over)
        return L.smol_b200_gemm_bf16(None, *kw.values())

    assert gemm() == 3
    assert gemm(act=smol_b200.ACT_GEGLU_PAIRS, out_kind=smol_b200.GEMM_OUT_BF16, ldo=128) == 3
    assert gemm(act=4) == 1 and gemm(act=-1) == 1
    assert gemm(act=smol_b200.ACT_SWIGLU_PAIRS, n=255) == 1                         # odd N
    assert gemm(act=smol_b200.ACT_SWIGLU_PAIRS, out_kind=smol_b200.GEMM_OUT_F32_ADD) == 1
    assert gemm(act=smol_b200.ACT_SWIGLU_PAIRS, add=base, ld_add=256, add_rows=1) == 1
    assert gemm(a=base + 8) == 1 and gemm(w=base + 4) == 1                          # TMA base alignment
    assert gemm(lda=132) == 1 and gemm(ldw=120) == 1                                # strides
    assert gemm(k=0) == 1 and gemm(ldo=255) == 1
    assert gemm(add=base, ld_add=256, add_rows=0) == 1
    assert gemm(m=0) == 0                                                           # nothing to do
    smol_b200.clear_error()


def test_no_device_fails_loudly():
    import torch
    if torch.cuda.is_available():
        pytest.skip("a device is present: the no-device contract is exercised on CPU-only hosts")
    smol_b200.clear_error()
    q = np.ones((4, 2 * 64), np.float32)
    k = np.ones((4, 64), np.float32)
    out = np.full((4, 2 * 64), 7.0, np.float32)
    smol_b200.causal_attention(out, q, k, k, 4, 4, 2, 1, 64, 0.125, 0)
    assert smol_b200.last_error() == 3          # SMOL_B200_ERR_NO_DEVICE
    assert np.all(out == 0.0)                   # zero-filled, never computed on the CPU
    smol_b200.clear_error()
    assert smol_b200.last_error() == 0


def test_binding_signatures_match_header():
    """Every prototype of include/smol_b200.h has a ctypes signature in the binding with
    the same number of arguments and a matching return kind, so a changed C prototype
    cannot silently mis-marshal calls (which only a GPU run would otherwise reveal)."""
    import ctypes
    import re
    text = re.sub(r"/\*.*?\*/", "", open(smol_b200.HEADER_PATH).read(), flags=re.S)
    protos = re.findall(r"SMOL_B200_API\s+([\w\s\*]+?)\b(\w+)\s*\(([^;]*?)\)\s*;", text, flags=re.S)
    assert len(protos) == len(smol_b200.header_symbols())
    kinds = {"void": None, "int": ctypes.c_int, "size_t": ctypes.c_size_t, "unsigned": ctypes.c_uint,
             "const char *": ctypes.c_char_p, "void *": ctypes.c_void_p}
    for ret, name, args in protos:
        args = args.strip()
        n_args = 0 if args in ("", "void") else len(args.split(","))
        assert name in smol_b200._SIGNATURES, name
        res, argtypes = smol_b200._SIGNATURES[name]
        assert len(argtypes) == n_args, (name, n_args, len(argtypes))
        ret = " ".join(ret.split())
        assert ret in kinds, (name, ret)
        assert res == kinds[ret], (name, ret, res)


def test_binding_structs_match_header(tmp_path):
    """The ctypes mirrors of the Part-4 / Part-5 structs have the C layout: field names in
    header order, and every offset and the size as gcc lays them out for include/smol_b200.h."""
    import ctypes
    import re
    text = re.sub(r"/\*.*?\*/", "", open(smol_b200.HEADER_PATH).read(), flags=re.S)
    for cname, pystruct in (("smol_b200_qkn_layer", smol_b200.QknLayer), ("smol_b200_qkn_model", smol_b200.QknModel),
                            ("smol_b200_siglip_layer", smol_b200.SiglipLayer),
                            ("smol_b200_siglip_model", smol_b200.SiglipModel)):
        body = re.search(r"typedef struct " + cname + r"\s*\{(.*?)\}\s*" + cname + r"\s*;", text, flags=re.S).group(1)
        names = []
        for decl in body.split(";"):
            decl = " ".join(decl.split())
            if not decl:
                continue
            # "const float *a, *b" / "int x, y": the names are the last word of each declarator
            names += [re.findall(r"\w+", d)[-1] for d in decl.split(",")]
        assert names == [f[0] for f in pystruct._fields_], (cname, names)
        src = tmp_path / f"{cname}.c"
        src.write_text("#include <stdio.h>\n#include <stddef.h>\n#include \"smol_b200.h\"\nint main(void){\n" +
                       "".join(f'printf("%zu\\n", offsetof({cname}, {n}));\n' for n in names) +
                       f'printf("%zu\\n", sizeof({cname}));\nreturn 0;\n}}\n')
        exe = tmp_path / cname
        subprocess.run(["gcc", "-std=c11", "-I", os.path.dirname(smol_b200.HEADER_PATH), "-o", str(exe), str(src)],
                       check=True)
        got = [int(v) for v in subprocess.run([str(exe)], capture_output=True, text=True, check=True).stdout.split()]
        want = [getattr(pystruct, n).offset for n in names] + [ctypes.sizeof(pystruct)]
        assert got == want, (cname, got, want)
