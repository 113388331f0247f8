"""SigLIP encoder on the device (smol_b200.h Part 5) against numpy and the CPU restatement.

Checked:
  * the tcgen05 GEMM in every output kind (fp32, bf16, fp16, added into fp32) with bias,
    a broadcast addend and GELU, on shapes with ragged M, N and K tails, against float64
    numpy (fp32 outputs within rel-L2 1e-5; 16-bit outputs within their rounding);
  * LayerNorm (layernorm.c:17-124) in fp32 and bf16, in place;
  * the whole encoder (siglip_forward, siglip.c:71-156) on the oracle's pin cases:
    within rel-L2 5e-3 of oracle/siglip_oracle.py with the device's 16-bit operands
    (bf16 rounding of LayerNorm / attention / GELU outputs turns the attention kernel's
    ~3e-4 difference into a few 1e-3), and within 1e-2 of the reference's own outputs
    (tests/golden/siglip_cases.npz);
  * the layer stack alone with attention windows (the audio encoder's form), against the
    same oracle.
"""
import os

import numpy as np
import pytest
import torch

import pyoracle
import smol_b200
from siglip_oracle import SIGLIP_PIN_CASES, SiglipOracle, gelu_tanh, layer_norm, siglip_pin_case

pytestmark = [pytest.mark.gpu, pytest.mark.new_on_gpu(stage=2)]
GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "siglip_cases.npz")


def _dev(cuda):
    return lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(cuda)   # noqa: E731


def _no_error():
    assert smol_b200.last_error() == 0, smol_b200.lib().smol_cuda_error_string(smol_b200.last_error())
    assert smol_b200.device_error() == 0


@pytest.mark.new_on_gpu(stage=1)
@pytest.mark.parametrize("M,N,K", [(256, 256, 128), (200, 136, 200), (1000, 768, 768), (130, 520, 588)])
def test_gemm_bf16_output_kinds(cuda, M, N, K):
    rng = np.random.default_rng(M + N + K)
    t = _dev(cuda)
    lda = ldw = (K + 7) // 8 * 8
    A = pyoracle.round_bf16(rng.standard_normal((M, K)).astype(np.float32))
    W = pyoracle.round_bf16((rng.standard_normal((N, K)) / np.sqrt(K)).astype(np.float32))
    Ap = np.zeros((M, lda), np.float32)
    Ap[:, :K] = A
    Wp = np.zeros((N, ldw), np.float32)
    Wp[:, :K] = W
    bias = rng.standard_normal(N).astype(np.float32)
    add = rng.standard_normal((7, N)).astype(np.float32)
    a_d, w_d = t(pyoracle.bf16_bits(Ap)), t(pyoracle.bf16_bits(Wp))
    base = (A.astype(np.float64) @ W.T.astype(np.float64)).astype(np.float32)
    full = (base + bias + add[np.arange(M) % 7]).astype(np.float32)

    y = torch.zeros((M, N), device=cuda)
    smol_b200.gemm_bf16(y, N, smol_b200.GEMM_OUT_F32, a_d, lda, w_d, ldw, M, N, K)
    torch.cuda.synchronize()
    _no_error()
    assert pyoracle.rel_l2(y.cpu().numpy(), base) < 1e-5

    y = torch.zeros((M, N), device=cuda)
    smol_b200.gemm_bf16(y, N, smol_b200.GEMM_OUT_F32, a_d, lda, w_d, ldw, M, N, K, bias=t(bias), add=t(add), ld_add=N,
                        add_rows=7, gelu=True)
    torch.cuda.synchronize()
    assert pyoracle.rel_l2(y.cpu().numpy(), gelu_tanh(full)) < 1e-5

    y0 = rng.standard_normal((M, N)).astype(np.float32)
    y = t(y0)
    smol_b200.gemm_bf16(y, N, smol_b200.GEMM_OUT_F32_ADD, a_d, lda, w_d, ldw, M, N, K, bias=t(bias))
    torch.cuda.synchronize()
    assert pyoracle.rel_l2(y.cpu().numpy(), y0 + base + bias) < 1e-5

    for kind, dt in ((smol_b200.GEMM_OUT_BF16, torch.bfloat16), (smol_b200.GEMM_OUT_F16, torch.float16)):
        y = torch.zeros((M, N), dtype=dt, device=cuda)
        smol_b200.gemm_bf16(y, N, kind, a_d, lda, w_d, ldw, M, N, K, bias=t(bias))
        torch.cuda.synchronize()
        got = y.float().cpu().numpy()
        assert pyoracle.rel_l2(got, base + bias) < (4e-3 if kind == smol_b200.GEMM_OUT_BF16 else 6e-4)
    _no_error()


@pytest.mark.new_on_gpu(stage=1)
@pytest.mark.parametrize("M,I,K", [(300, 1536, 1024), (77, 200, 256)])
def test_gemm_bf16_gated_pairs(cuda, M, I, K):
    """Interleaved gate/up weight rows: out[m][j] = act(c[2j]) * c[2j+1] (the decoder
    prefill's MLP, activation.c:55-126), SiLU and GELU-tanh, fp32 and bf16 out."""
    from qkn_decoder_oracle import geglu, swiglu
    rng = np.random.default_rng(M + I)
    t = _dev(cuda)
    A = pyoracle.round_bf16(rng.standard_normal((M, K)).astype(np.float32))
    W = pyoracle.round_bf16((rng.standard_normal((2 * I, K)) / np.sqrt(K)).astype(np.float32))
    c = (A.astype(np.float64) @ W.T.astype(np.float64)).astype(np.float32)
    for act, fn in ((smol_b200.ACT_SWIGLU_PAIRS, swiglu), (smol_b200.ACT_GEGLU_PAIRS, geglu)):
        y = torch.zeros((M, I), device=cuda)
        smol_b200.gemm_bf16(y, I, smol_b200.GEMM_OUT_F32, t(pyoracle.bf16_bits(A)), K, t(pyoracle.bf16_bits(W)), K, M,
                            2 * I, K, act=act)
        yb = torch.zeros((M, I), dtype=torch.bfloat16, device=cuda)
        smol_b200.gemm_bf16(yb, I, smol_b200.GEMM_OUT_BF16, t(pyoracle.bf16_bits(A)), K, t(pyoracle.bf16_bits(W)), K,
                            M, 2 * I, K, act=act)
        torch.cuda.synchronize()
        _no_error()
        assert pyoracle.rel_l2(y.cpu().numpy(), fn(c)) < 1e-5
        assert pyoracle.rel_l2(yb.float().cpu().numpy(), fn(c)) < 4e-3


@pytest.mark.new_on_gpu(stage=1)
@pytest.mark.parametrize("M,N,K", [(4096, 1280, 768), (8192, 1024, 256), (20000, 768, 200), (37000, 520, 588)])
def test_gemm_bf16_wide_form(cuda, M, N, K):
    """Shapes whose 128 x 256 tiles fill a wave of SMs run the wide persistent GEMM: more
    tiles than SMs (both TMEM accumulators reused), ragged M, N and K tails; fp32 with
    bias + GELU, fp32 added into C, bf16 out; against float64 numpy on sampled rows."""
    rng = np.random.default_rng(M + N)
    t = _dev(cuda)
    lda = (K + 7) // 8 * 8
    A = pyoracle.round_bf16(rng.standard_normal((M, K)).astype(np.float32))
    W = pyoracle.round_bf16((rng.standard_normal((N, K)) / np.sqrt(K)).astype(np.float32))
    Ap = np.zeros((M, lda), np.float32)
    Ap[:, :K] = A
    Wp = np.zeros((N, lda), np.float32)
    Wp[:, :K] = W
    bias = rng.standard_normal(N).astype(np.float32)
    a_d, w_d, b_d = t(pyoracle.bf16_bits(Ap)), t(pyoracle.bf16_bits(Wp)), t(bias)
    rows = np.unique(np.concatenate([np.arange(0, 300), rng.integers(0, M, 700), np.arange(M - 300, M)]))
    base = (A[rows].astype(np.float64) @ W.T.astype(np.float64)).astype(np.float32)

    y = torch.zeros((M, N), device=cuda)
    smol_b200.gemm_bf16(y, N, smol_b200.GEMM_OUT_F32, a_d, lda, w_d, ldw=lda, m=M, n=N, k=K, bias=b_d, gelu=True)
    torch.cuda.synchronize()
    _no_error()
    assert pyoracle.rel_l2(y.cpu().numpy()[rows], gelu_tanh(base + bias)) < 1e-5

    y0 = torch.randn((M, N), device=cuda)
    y = y0.clone()
    smol_b200.gemm_bf16(y, N, smol_b200.GEMM_OUT_F32_ADD, a_d, lda, w_d, ldw=lda, m=M, n=N, k=K, bias=b_d)
    torch.cuda.synchronize()
    assert pyoracle.rel_l2(y.cpu().numpy()[rows], y0.cpu().numpy()[rows] + base + bias) < 1e-5

    yb = torch.zeros((M, N), dtype=torch.bfloat16, device=cuda)
    smol_b200.gemm_bf16(yb, N, smol_b200.GEMM_OUT_BF16, a_d, lda, w_d, ldw=lda, m=M, n=N, k=K, bias=b_d)
    torch.cuda.synchronize()
    _no_error()
    assert pyoracle.rel_l2(yb.float().cpu().numpy()[rows], base + bias) < 4e-3


@pytest.mark.new_on_gpu(stage=1)
def test_gemm_bf16_wide_gated_pairs(cuda):
    """The gated gate/up epilogue on the wide form: 4096 rows x 2*1536 interleaved columns."""
    from qkn_decoder_oracle import swiglu
    M, I, K = 4096, 1536, 1024
    rng = np.random.default_rng(9)
    t = _dev(cuda)
    A = pyoracle.round_bf16(rng.standard_normal((M, K)).astype(np.float32))
    W = pyoracle.round_bf16((rng.standard_normal((2 * I, K)) / np.sqrt(K)).astype(np.float32))
    rows = rng.integers(0, M, 400)
    c = (A[rows].astype(np.float64) @ W.T.astype(np.float64)).astype(np.float32)
    yb = torch.zeros((M, I), dtype=torch.bfloat16, device=cuda)
    smol_b200.gemm_bf16(yb, I, smol_b200.GEMM_OUT_BF16, t(pyoracle.bf16_bits(A)), K, t(pyoracle.bf16_bits(W)), K, M,
                        2 * I, K, act=smol_b200.ACT_SWIGLU_PAIRS)
    torch.cuda.synchronize()
    _no_error()
    assert pyoracle.rel_l2(yb.float().cpu().numpy()[rows], swiglu(c)) < 4e-3


@pytest.mark.new_on_gpu(stage=1)
def test_layer_norm_fp32_bf16_in_place(cuda):
    rng = np.random.default_rng(3)
    t = _dev(cuda)
    rows, hidden = 300, 768
    x = (3 * rng.standard_normal((rows, hidden)) + 1).astype(np.float32)
    w = (1 + 0.1 * rng.standard_normal(hidden)).astype(np.float32)
    b = (0.1 * rng.standard_normal(hidden)).astype(np.float32)
    want = layer_norm(x, w, b, 1e-6)
    out = torch.zeros((rows, hidden), device=cuda)
    smol_b200.layer_norm(out, t(x), t(w), t(b), rows, hidden, 1e-6)
    o16 = torch.zeros((rows, hidden), dtype=torch.bfloat16, device=cuda)
    smol_b200.layer_norm(o16, t(x), t(w), t(b), rows, hidden, 1e-6, out_bf16=True)
    xin = t(x)
    smol_b200.layer_norm(xin, xin, t(w), t(b), rows, hidden, 1e-6)
    torch.cuda.synchronize()
    _no_error()
    assert pyoracle.rel_l2(out.cpu().numpy(), want) < 1e-6
    assert pyoracle.rel_l2(xin.cpu().numpy(), want) < 1e-6
    assert pyoracle.rel_l2(o16.float().cpu().numpy(), want) < 4e-3


def _upload(m, cuda):
    t = _dev(cuda)
    bits = lambda a: t(pyoracle.bf16_bits(a))   # noqa: E731
    layers = []
    for lw in m.layers:
        layers.append({"ln1_w": t(lw["ln1_w"]), "ln1_b": t(lw["ln1_b"]), "wq": bits(lw["wq"]), "wk": bits(lw["wk"]),
                       "wv": bits(lw["wv"]), "wo": bits(lw["wo"]), "bq": t(lw["bq"]), "bk": t(lw["bk"]),
                       "bv": t(lw["bv"]), "bo": t(lw["bo"]), "ln2_w": t(lw["ln2_w"]), "ln2_b": t(lw["ln2_b"]),
                       "fc1": bits(lw["fc1"]), "b1": t(lw["b1"]), "fc2": bits(lw["fc2"]), "b2": t(lw["b2"])})
    keep = dict(patch_w=bits(m.patch_w), patch_b=t(m.patch_b), pos=t(m.pos), post_w=t(m.post_w), post_b=t(m.post_b),
                layers=layers)
    model = smol_b200.siglip_model(m.H, m.NH, m.F, m.P, m.image, m.n_pos, m.eps, keep["patch_w"],
                                   3 * m.P * m.P, keep["patch_b"], keep["pos"], keep["post_w"], keep["post_b"], layers)
    return model, keep


@pytest.mark.parametrize("case", list(SIGLIP_PIN_CASES))
def test_siglip_forward_matches_oracle_and_reference(cuda, case):
    m, images = siglip_pin_case(case)
    model, keep = _upload(m, cuda)
    n = len(images)
    ws = torch.zeros(smol_b200.siglip_workspace_bytes(model, n), dtype=torch.uint8, device=cuda)
    out = torch.zeros((n, m.n_pos, m.H), device=cuda)
    smol_b200.siglip_forward(out, _dev(cuda)(images), n, model, ws)
    torch.cuda.synchronize()
    _no_error()
    got = out.cpu().numpy()
    want = m.forward(images, device_formats=True)
    e = pyoracle.rel_l2(got, want)
    assert e < 5e-3, e
    ref = np.load(GOLDEN)[f"{case}/out"]
    assert pyoracle.rel_l2(got, ref) < 1e-2
    print(f"{case}: rel-L2 {e:.2e} vs the device-format oracle, {pyoracle.rel_l2(got, ref):.2e} vs the reference")


def test_siglip_forward_head_dim_72(cuda):
    """SmolVLM's SigLIP-So400m layer shape (hidden 1152, 16 heads of 72) through the whole
    device forward: the attention runs the 128-wide prefill kernel on 72-column heads.
    Two layers, a 224-pixel image of 16-pixel patches (196 patches) and a shorter MLP
    keep the oracle quick; the head dim is what this checks."""
    m = SiglipOracle(hidden=1152, heads=16, ffn=1536, layers=2, patch=16, image=224, seed=11)
    images = m.images(2, 13)
    model, keep = _upload(m, cuda)
    ws = torch.zeros(smol_b200.siglip_workspace_bytes(model, 2), dtype=torch.uint8, device=cuda)
    out = torch.zeros((2, m.n_pos, m.H), device=cuda)
    smol_b200.siglip_forward(out, _dev(cuda)(images), 2, model, ws)
    torch.cuda.synchronize()
    _no_error()
    e = pyoracle.rel_l2(out.cpu().numpy(), m.forward(images, device_formats=True))
    assert e < 5e-3, e


def test_encoder_layers_with_windows(cuda):
    """The layer stack alone with attention windows -- the Qwen3-ASR audio encoder's form
    (encoder.c:449-484, eps 1e-5): ten 104-token windows, the last ragged, 4 heads of 64
    (tests/test_encoder_layers_oracle.py pins the windowed oracle to the reference)."""
    m = SiglipOracle(hidden=256, heads=4, ffn=512, layers=2, eps=1e-5, seed=8)
    ws = list(range(0, 9 * 104 + 1, 104)) + [9 * 104 + 50]
    T = ws[-1]
    x = np.random.default_rng(9).standard_normal((T, m.H)).astype(np.float32)
    t = _dev(cuda)
    bits = lambda a: t(pyoracle.bf16_bits(a))   # noqa: E731
    keep = [{"ln1_w": t(lw["ln1_w"]), "ln1_b": t(lw["ln1_b"]), "wq": bits(lw["wq"]), "wk": bits(lw["wk"]),
             "wv": bits(lw["wv"]), "wo": bits(lw["wo"]), "bq": t(lw["bq"]), "bk": t(lw["bk"]), "bv": t(lw["bv"]),
             "bo": t(lw["bo"]), "ln2_w": t(lw["ln2_w"]), "ln2_b": t(lw["ln2_b"]), "fc1": bits(lw["fc1"]),
             "b1": t(lw["b1"]), "fc2": bits(lw["fc2"]), "b2": t(lw["b2"])} for lw in m.layers]
    arr = smol_b200.siglip_layers(keep)
    xd = t(x)
    ws_d = t(np.asarray(ws, np.int32))
    work = torch.zeros(smol_b200.encoder_workspace_bytes(T, m.H, m.F), dtype=torch.uint8, device=cuda)
    smol_b200.encoder_layers(xd, 1, T, arr, m.H, m.NH, m.F, m.eps, work, window_starts=ws_d)
    torch.cuda.synchronize()
    _no_error()
    got = xd.cpu().numpy()
    e = pyoracle.rel_l2(got, m.encoder_layers(x[None], device_formats=True, window_starts=ws)[0])
    assert e < 5e-3, e
    assert pyoracle.rel_l2(got, m.encoder_layers(x[None], device_formats=False, window_starts=ws)[0]) < 1e-2
