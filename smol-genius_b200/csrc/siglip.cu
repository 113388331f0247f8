// siglip.cu -- the SigLIP vision encoder (siglip_forward, siglip.c:71-156) and the
// pre-LayerNorm encoder layers it shares with the Qwen3-ASR audio encoder
// (encoder.c:449-484, attention within the windows of :426-435) on the device.
//
// Per batch of images: the patches are unfolded into bf16 rows (the im2col of the
// kernel = stride = patch convolution, conv2d.c:13-50, one row per patch) and the patch
// embedding is one GEMM whose epilogue adds the conv bias and the position embedding
// (siglip.c:85-89); then per layer
//     LayerNorm (bf16 out) -> Q, K (bf16), V (fp16) GEMMs with bias
//     -> bidirectional attention over all patches (the tcgen05 prefill kernel, full mask)
//     -> attention output to bf16 -> output-projection GEMM added into the fp32 stream
//     -> LayerNorm -> fc1 GEMM with bias and GELU (bf16 out) -> fc2 GEMM added into the stream
// and the post-LayerNorm writes the fp32 output.  Every GEMM is gemm.cu's tcgen05 kernel;
// LayerNorm, the unfold and the conversion are memory-bound kernels here.
#include <math.h>
#include <string.h>

#include "b200_common.cuh"
#include "runtime.h"

namespace smolb200 {
namespace {

constexpr int kLnWarps = 8;   // rows per CTA of the LayerNorm kernel (one warp per row)

__device__ __forceinline__ float warp_sum(float v)
{
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

// smol_layer_norm (layernorm.c:17-124): mean, then the mean of squared deviations, then
// (x - mean) * 1/sqrtf(var + eps) * w + b.  One warp per row; out may alias x (each
// element is read by the thread that writes it, after both reductions).
__global__ void __launch_bounds__(kLnWarps * 32) layer_norm_kernel(void *out, int out_bf16, const float *x,
                                                                   const float *w, const float *b, int rows,
                                                                   int hidden, float eps)
{
    const int row = blockIdx.x * kLnWarps + threadIdx.x / 32, lane = threadIdx.x % 32;
    if (row >= rows) return;
    const float *xr = x + static_cast<long long>(row) * hidden;
    float s = 0.f;
    for (int i = lane; i < hidden; i += 32) s += xr[i];
    const float mean = warp_sum(s) / static_cast<float>(hidden);
    float ss = 0.f;
    for (int i = lane; i < hidden; i += 32) {
        const float d = xr[i] - mean;
        ss += d * d;
    }
    const float var = warp_sum(ss) / static_cast<float>(hidden);
    const float inv = 1.0f / sqrtf(var + eps);
    if (out_bf16) {
        uint16_t *o = static_cast<uint16_t *>(out) + static_cast<long long>(row) * hidden;
        for (int i = lane; i < hidden; i += 32) {
            const float y = (xr[i] - mean) * inv * w[i] + b[i];
            o[i] = static_cast<uint16_t>(pack_bf16x2(y, 0.f) & 0xffffu);
        }
    } else {
        float *o = static_cast<float *>(out) + static_cast<long long>(row) * hidden;
        for (int i = lane; i < hidden; i += 32) o[i] = (xr[i] - mean) * inv * w[i] + b[i];
    }
}

// The same for rows of a multiple of 128 floats up to 2048 (SigLIP-base 768, So400m
// 1152): the warp reads its row once as float4 pieces kept in registers (lane l holds
// elements 4l..4l+3 of every 128-float block), both reductions run on those registers,
// and the output leaves as 8-byte (bf16) or 16-byte (fp32) pieces.
constexpr int kLnMaxVec = 16;   // float4 pieces per lane: hidden <= 16 * 128
__global__ void __launch_bounds__(kLnWarps * 32) layer_norm_vec_kernel(void *out, int out_bf16, const float *x,
                                                                       const float *w, const float *b, int rows,
                                                                       int hidden, float eps)
{
    const int row = blockIdx.x * kLnWarps + threadIdx.x / 32, lane = threadIdx.x % 32;
    if (row >= rows) return;
    const int nv = hidden / 128;
    const float4 *xr = reinterpret_cast<const float4 *>(x + static_cast<long long>(row) * hidden);
    float4 v[kLnMaxVec];
    float s = 0.f;
#pragma unroll
    for (int i = 0; i < kLnMaxVec; ++i)
        if (i < nv) {
            v[i] = xr[i * 32 + lane];
            s += (v[i].x + v[i].y) + (v[i].z + v[i].w);
        }
    const float mean = warp_sum(s) / static_cast<float>(hidden);
    float ss = 0.f;
#pragma unroll
    for (int i = 0; i < kLnMaxVec; ++i)
        if (i < nv) {
            const float a = v[i].x - mean, c = v[i].y - mean, d = v[i].z - mean, e = v[i].w - mean;
            ss += (a * a + c * c) + (d * d + e * e);
        }
    const float inv = 1.0f / sqrtf(warp_sum(ss) / static_cast<float>(hidden) + eps);
    const float4 *w4 = reinterpret_cast<const float4 *>(w), *b4 = reinterpret_cast<const float4 *>(b);
#pragma unroll
    for (int i = 0; i < kLnMaxVec; ++i) {
        if (i >= nv) break;
        const float4 wv = __ldg(w4 + i * 32 + lane), bv = __ldg(b4 + i * 32 + lane);
        const float y0 = (v[i].x - mean) * inv * wv.x + bv.x, y1 = (v[i].y - mean) * inv * wv.y + bv.y;
        const float y2 = (v[i].z - mean) * inv * wv.z + bv.z, y3 = (v[i].w - mean) * inv * wv.w + bv.w;
        const long long e = static_cast<long long>(row) * hidden + i * 128 + 4 * lane;
        if (out_bf16)
            *reinterpret_cast<uint2 *>(static_cast<uint16_t *>(out) + e) = make_uint2(pack_bf16x2(y0, y1),
                                                                                       pack_bf16x2(y2, y3));
        else
            *reinterpret_cast<float4 *>(static_cast<float *>(out) + e) = make_float4(y0, y1, y2, y3);
    }
}

// a[img * n_patches + py * pw + px][(c * patch + ky) * patch + kx] =
//     bf16(image[img][c][py * patch + ky][px * patch + kx]); columns [kin, lda) zero.
__global__ void unfold_patches_kernel(uint16_t *a, long long lda, const float *images, int n_images, int size,
                                      int patch)
{
    const int pw = size / patch, n_patches = pw * pw, kin = 3 * patch * patch;
    const long long total = static_cast<long long>(n_images) * n_patches * lda;
    for (long long e = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x; e < total;
         e += static_cast<long long>(gridDim.x) * blockDim.x) {
        const long long r = e / lda;
        const int col = static_cast<int>(e % lda);
        float v = 0.f;
        if (col < kin) {
            const int img = static_cast<int>(r / n_patches), pi = static_cast<int>(r % n_patches);
            const int py = pi / pw, px = pi % pw;
            const int c = col / (patch * patch), ky = (col / patch) % patch, kx = col % patch;
            v = images[((static_cast<long long>(img) * 3 + c) * size + py * patch + ky) * size + px * patch + kx];
        }
        a[e] = static_cast<uint16_t>(pack_bf16x2(v, 0.f) & 0xffffu);
    }
}

unsigned grid_for(long long work, int block)
{
    const long long g = (work + block - 1) / block;
    return static_cast<unsigned>(g < 148LL * 32 ? (g > 0 ? g : 1) : 148LL * 32);
}

// Workspace of the encoder layers for T tokens (256-byte aligned pieces).
struct EncoderWs {
    uint16_t *xn, *q, *k, *v, *attn16, *h;
    size_t total;
};

EncoderWs carve_encoder(size_t T, size_t H, size_t F, uint8_t *base)
{
    EncoderWs w;
    memset(&w, 0, sizeof(w));
    size_t off = 0;
    auto take = [&](size_t bytes) {
        uint8_t *p = base ? base + off : nullptr;
        off += (bytes + 255) / 256 * 256;
        return p;
    };
    w.xn = reinterpret_cast<uint16_t *>(take(T * H * 2));
    w.q = reinterpret_cast<uint16_t *>(take(T * H * 2));
    w.k = reinterpret_cast<uint16_t *>(take(T * H * 2));
    w.v = reinterpret_cast<uint16_t *>(take(T * H * 2));
    w.attn16 = reinterpret_cast<uint16_t *>(take(T * H * 2));
    w.h = reinterpret_cast<uint16_t *>(take(T * F * 2));
    w.total = off;
    return w;
}

// SigLIP: the unfolded patches, then the encoder pieces.
struct SiglipWs {
    uint16_t *patches;
    uint8_t *enc;
    size_t enc_bytes;
    int lda, n_patches;
    size_t total;
};

SiglipWs carve(const smol_b200_siglip_model &m, int n_images, uint8_t *base)
{
    SiglipWs w;
    memset(&w, 0, sizeof(w));
    const int pw = m.image_size / m.patch;
    w.n_patches = pw * pw;
    w.lda = (3 * m.patch * m.patch + 7) / 8 * 8;
    const size_t T = static_cast<size_t>(n_images) * w.n_patches;
    const size_t patch_bytes = (T * w.lda * 2 + 255) / 256 * 256;
    w.patches = base ? reinterpret_cast<uint16_t *>(base) : nullptr;
    w.enc = base ? base + patch_bytes : nullptr;
    w.enc_bytes = carve_encoder(T, m.hidden, m.ffn, nullptr).total;
    w.total = patch_bytes + w.enc_bytes;
    return w;
}

bool layers_ok(const smol_b200_siglip_layer *layers, int n_layers)
{
    if (!layers || n_layers <= 0) return false;
    for (int l = 0; l < n_layers; ++l) {
        const smol_b200_siglip_layer &L = layers[l];
        if (!L.ln1_w || !L.ln1_b || !L.wq || !L.wk || !L.wv || !L.wo || !L.bq || !L.bk || !L.bv || !L.bo ||
            !L.ln2_w || !L.ln2_b || !L.fc1 || !L.b1 || !L.fc2 || !L.b2)
            return false;
    }
    return true;
}

bool encoder_shape_ok(int hidden, int heads, int ffn)
{
    if (hidden <= 0 || heads <= 0 || hidden % heads || ffn <= 0 || hidden % 8 || ffn % 8) return false;
    // any head dim the prefill kernel takes: a multiple of 8 up to 256 (SigLIP-base 64,
    // SigLIP-So400m 72)
    const int hd = hidden / heads;
    return hd % 8 == 0 && hd <= 256;
}

bool model_ok(const smol_b200_siglip_model *m)
{
    if (!m || !encoder_shape_ok(m->hidden, m->heads, m->ffn) || m->patch <= 0 || m->image_size < m->patch ||
        !m->patch_w || !m->patch_b || !m->pos || !m->post_w || !m->post_b ||
        m->patch_ld < 3 * m->patch * m->patch || m->patch_ld % 8)
        return false;
    const int pw = m->image_size / m->patch;
    if (pw * pw > m->num_positions) return false;
    return layers_ok(m->layers, m->n_layers);
}

}  // namespace

int layer_norm(cudaStream_t st, void *out, int out_bf16, const float *x, const float *w, const float *b, int rows,
               int hidden, float eps)
{
    if (rows <= 0) return SMOL_B200_OK;
    if (!out || !x || !w || !b || hidden <= 0) return SMOL_B200_ERR_ARGS;
    const unsigned grid = static_cast<unsigned>((rows + kLnWarps - 1) / kLnWarps);
    const uintptr_t al = reinterpret_cast<uintptr_t>(out) | reinterpret_cast<uintptr_t>(x) |
                         reinterpret_cast<uintptr_t>(w) | reinterpret_cast<uintptr_t>(b);
    const bool vec = hidden % 128 == 0 && hidden <= kLnMaxVec * 128 && (al & 15) == 0;
    return launch_kernel(vec ? layer_norm_vec_kernel : layer_norm_kernel, dim3(grid), dim3(kLnWarps * 32), 0, st,
                         out, out_bf16, x, w, b, rows, hidden, eps) == cudaSuccess
               ? SMOL_B200_OK
               : SMOL_B200_ERR_CUDA;
}

size_t encoder_workspace_bytes(int n_tokens, int hidden, int ffn)
{
    if (n_tokens <= 0 || hidden <= 0 || ffn <= 0) return 0;
    return carve_encoder(static_cast<size_t>(n_tokens), hidden, ffn, nullptr).total;
}

int encoder_layers(cudaStream_t st, float *x, int batch, int seq, const smol_b200_siglip_layer *layers, int n_layers,
                   int hidden, int heads, int ffn, float eps, const int *window_starts, int n_windows,
                   void *workspace, size_t workspace_bytes)
{
    if (batch <= 0 || seq <= 0) return SMOL_B200_OK;
    if (!x || !encoder_shape_ok(hidden, heads, ffn) || !layers_ok(layers, n_layers) ||
        (window_starts && n_windows <= 0))
        return SMOL_B200_ERR_ARGS;
    const int H = hidden, F = ffn, T = batch * seq, hd = H / heads;
    const EncoderWs w = carve_encoder(static_cast<size_t>(T), H, F, static_cast<uint8_t *>(workspace));
    if (!workspace || workspace_bytes < w.total) return SMOL_B200_ERR_WORKSPACE;
    const float scale = 1.0f / sqrtf(static_cast<float>(hd));   // siglip.c:108, encoder.c:447
    const int64_t bs = static_cast<int64_t>(seq) * H;           // elements between batch elements
    const int mask = window_starts ? SMOL_MASK_WINDOWS : SMOL_MASK_FULL;
    int rc = SMOL_B200_OK;
    for (int l = 0; l < n_layers && rc == SMOL_B200_OK; ++l) {
        const smol_b200_siglip_layer &L = layers[l];
        rc = layer_norm(st, w.xn, 1, x, L.ln1_w, L.ln1_b, T, H, eps);
        if (rc == SMOL_B200_OK)
            rc = gemm_bf16(st, w.q, H, SMOL_B200_GEMM_OUT_BF16, w.xn, H, L.wq, H, L.bq, nullptr, 0, 0, T, H, H, 0);
        if (rc == SMOL_B200_OK)
            rc = gemm_bf16(st, w.k, H, SMOL_B200_GEMM_OUT_BF16, w.xn, H, L.wk, H, L.bk, nullptr, 0, 0, T, H, H, 0);
        if (rc == SMOL_B200_OK)
            rc = gemm_bf16(st, w.v, H, SMOL_B200_GEMM_OUT_F16, w.xn, H, L.wv, H, L.bv, nullptr, 0, 0, T, H, H, 0);
        // bidirectional attention: all tokens of a batch element (siglip.c:104-127) or the
        // tokens of each window (encoder.c:426-435, :462-464)
        if (rc == SMOL_B200_OK)
            rc = prefill_attention(st, w.attn16, H, bs, w.q, H, bs, w.k, H, bs, w.v, H, bs, batch, seq, seq, heads,
                                   heads, hd, scale, mask, 0, 0, 0, 0.f, window_starts, n_windows, nullptr, 0,
                                   1 /* bf16 output: the o_proj GEMM's operand */);
        if (rc == SMOL_B200_OK)
            rc = gemm_bf16(st, x, H, SMOL_B200_GEMM_OUT_F32_ADD, w.attn16, H, L.wo, H, L.bo, nullptr, 0, 0, T, H, H, 0);
        if (rc == SMOL_B200_OK) rc = layer_norm(st, w.xn, 1, x, L.ln2_w, L.ln2_b, T, H, eps);
        if (rc == SMOL_B200_OK)
            rc = gemm_bf16(st, w.h, F, SMOL_B200_GEMM_OUT_BF16, w.xn, H, L.fc1, H, L.b1, nullptr, 0, 0, T, F, H, 1);
        if (rc == SMOL_B200_OK)
            rc = gemm_bf16(st, x, H, SMOL_B200_GEMM_OUT_F32_ADD, w.h, F, L.fc2, F, L.b2, nullptr, 0, 0, T, H, F, 0);
    }
    return rc;
}

size_t siglip_workspace_bytes(const smol_b200_siglip_model *m, int n_images)
{
    if (!model_ok(m) || n_images <= 0) return 0;
    return carve(*m, n_images, nullptr).total;
}

int siglip_forward(cudaStream_t st, float *out, const float *images, int n_images, const smol_b200_siglip_model *mp,
                   void *workspace, size_t workspace_bytes)
{
    if (n_images <= 0) return SMOL_B200_OK;
    if (!model_ok(mp) || !out || !images) return SMOL_B200_ERR_ARGS;
    const smol_b200_siglip_model &m = *mp;
    const SiglipWs w = carve(m, n_images, static_cast<uint8_t *>(workspace));
    if (!workspace || workspace_bytes < w.total) return SMOL_B200_ERR_WORKSPACE;
    const int H = m.hidden, NP = w.n_patches, T = n_images * NP;
    const int kin = 3 * m.patch * m.patch;
    float *x = out;   // the fp32 residual stream

    // patch embedding: conv bias and position embedding in the GEMM epilogue (siglip.c:80-89)
    {
        const long long n = static_cast<long long>(T) * w.lda;
        if (launch_kernel(unfold_patches_kernel, dim3(grid_for(n, 256)), dim3(256), 0, st, w.patches,
                          static_cast<long long>(w.lda), images, n_images, m.image_size, m.patch) != cudaSuccess)
            return SMOL_B200_ERR_CUDA;
    }
    int rc = gemm_bf16(st, x, H, SMOL_B200_GEMM_OUT_F32, w.patches, w.lda, m.patch_w, m.patch_ld, m.patch_b, m.pos,
                       H, NP, T, H, kin, 0);
    // the encoder layers, every patch attending to every patch of its image (siglip.c:112-147)
    if (rc == SMOL_B200_OK)
        rc = encoder_layers(st, x, n_images, NP, m.layers, m.n_layers, H, m.heads, m.ffn, m.eps, nullptr, 0, w.enc,
                            w.enc_bytes);
    // post-LayerNorm in place (siglip.c:150-151)
    if (rc == SMOL_B200_OK) rc = layer_norm(st, x, 0, x, m.post_w, m.post_b, T, H, m.eps);
    return rc;
}

}  // namespace smolb200
