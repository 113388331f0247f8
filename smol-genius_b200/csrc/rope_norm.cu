// rope_norm.cu -- per-head QK-RMSNorm, RoPE and the KV-cache append, plus the
// staging kernels of the drop-in attention path.
//
// These are elementwise, HBM-bound kernels: one warp owns one [head_dim] slice, so
// the per-head sum of squares is one warp reduction and the RoPE partner of every
// element (d+half for NeoX, d^1 for interleaved) sits in the same warp.
//
// Formulas follow the reference exactly in structure:
//   RMSNorm  x*(1/sqrtf(sum(x^2)/hd + eps))*w     rmsnorm.c:113 (per head), :50 (row)
//   NeoX     x1' = x1*c - x2*s, x2' = x2*c + x1*s  rope.c:154-160
//   interl.  x0' = x0*c - x1*s, x1' = x1*c + x0*s  rope.c:85-90
// with cos/sin read from tables the host built with the reference's libm formula
// (qkn_decoder.c:261-311), so positions index bit-identical table rows.
#include "b200_common.cuh"
#include "runtime.h"

namespace smolb200 {
namespace {

constexpr int kWarpsPerBlock = 8;

__device__ __forceinline__ float warp_sum(float v)
{
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) v += __shfl_xor_sync(0xffffffffu, v, off);
    return v;
}

// One warp normalises (optional) and rotates (optional) one [hd] slice held in
// global memory, in place.  NeoX pairs (d, d+half); interleaved pairs (2d, 2d+1).
__device__ __forceinline__ void norm_rope_slice(float *v, int hd, const float *w, float eps, const float *c,
                                                const float *s, int interleaved, int lane)
{
    float r = 1.f;
    if (w) {
        float ss = 0.f;
        for (int d = lane; d < hd; d += 32) ss += v[d] * v[d];
        ss = warp_sum(ss);
        r = 1.0f / sqrtf(ss / hd + eps);
    }
    const int half = hd / 2;
    if (c) {
        for (int i = lane; i < half; i += 32) {
            const int d0 = interleaved ? 2 * i : i;
            const int d1 = interleaved ? 2 * i + 1 : i + half;
            float x0 = v[d0], x1 = v[d1];
            if (w) {
                x0 = x0 * r * w[d0];
                x1 = x1 * r * w[d1];
            }
            v[d0] = x0 * c[d0] - x1 * s[d0];
            v[d1] = x1 * c[d1] + x0 * s[d1];
        }
        if (hd & 1) {   // odd head_dim: the last element has no partner (reference leaves it rotated by nothing)
            if (lane == 0 && w) v[hd - 1] = v[hd - 1] * r * w[hd - 1];
        }
    } else if (w) {
        for (int d = lane; d < hd; d += 32) v[d] = v[d] * r * w[d];
    }
}

__global__ void rms_norm_per_head_kernel(float *x, const float *w, long long rows, int hd, float eps)
{
    const long long row = static_cast<long long>(blockIdx.x) * kWarpsPerBlock + threadIdx.x / 32;
    if (row >= rows) return;
    norm_rope_slice(x + row * hd, hd, w, eps, nullptr, nullptr, 0, threadIdx.x % 32);
}

__global__ void rms_norm_kernel(float *out, const float *x, const float *w, int hidden, float eps)
{
    const long long row = blockIdx.x;
    const float *xr = x + row * hidden;
    float *orow = out + row * hidden;
    __shared__ float part[32];
    float ss = 0.f;
    for (int i = threadIdx.x; i < hidden; i += blockDim.x) ss += xr[i] * xr[i];
    ss = warp_sum(ss);
    if (threadIdx.x % 32 == 0) part[threadIdx.x / 32] = ss;
    __syncthreads();
    if (threadIdx.x < 32) {
        float t = threadIdx.x < blockDim.x / 32 ? part[threadIdx.x] : 0.f;
        t = warp_sum(t);
        if (threadIdx.x == 0) part[0] = t;
    }
    __syncthreads();
    const float r = 1.0f / sqrtf(part[0] / hidden + eps);
    for (int i = threadIdx.x; i < hidden; i += blockDim.x) orow[i] = xr[i] * r * w[i];
}

// x [seq, n_heads, hd]; cos/sin [seq, hd] (row s for token s).
__global__ void rope_kernel(float *x, const float *cs, const float *sn, long long rows, int n_heads, int hd,
                            int interleaved)
{
    const long long row = static_cast<long long>(blockIdx.x) * kWarpsPerBlock + threadIdx.x / 32;
    if (row >= rows) return;
    const long long tok = row / n_heads;
    norm_rope_slice(x + row * hd, hd, nullptr, 0.f, cs + tok * hd, sn + tok * hd, interleaved, threadIdx.x % 32);
}

// Fused prologue.  Warps [0, n_tokens*n_heads) handle q slices, the next
// n_tokens*n_kv_heads warps handle k slices (k is normed, rotated and stored as bf16;
// the matching v slice is stored as fp16 by the same warp).
__global__ void qknorm_rope_append_kernel(const float *__restrict__ q_in, const float *__restrict__ k_in,
                                          const float *__restrict__ v_in, int n_tokens, int n_heads,
                                          int n_kv_heads, int hd, const float *q_w, const float *k_w, float eps,
                                          const float *cs, const float *sn, int interleaved,
                                          const int *__restrict__ positions, const int64_t *__restrict__ slots,
                                          float *q_out_f32, uint16_t *q_out_bf16, uint16_t *k_cache,
                                          uint16_t *v_cache, long long cache_rows, unsigned *err)
{
    griddep_wait();
    griddep_trigger();
    const long long wid = static_cast<long long>(blockIdx.x) * kWarpsPerBlock + threadIdx.x / 32;
    const int lane = threadIdx.x % 32;
    const long long nq = static_cast<long long>(n_tokens) * n_heads;
    const long long nk = static_cast<long long>(n_tokens) * n_kv_heads;
    if (wid >= nq + nk) return;
    const bool is_q = wid < nq;
    const long long idx = is_q ? wid : wid - nq;
    const int heads = is_q ? n_heads : n_kv_heads;
    const long long tok = idx / heads;
    const int h = static_cast<int>(idx % heads);
    const float *src = (is_q ? q_in : k_in) + (tok * heads + h) * hd;
    const float *w = is_q ? q_w : k_w;
    const float *c = cs ? cs + static_cast<long long>(positions[tok]) * hd : nullptr;
    const float *s = sn ? sn + static_cast<long long>(positions[tok]) * hd : nullptr;

    // Load the slice into registers (hd <= 256 -> <= 8 values per lane).
    float r = 1.f;
    if (w) {
        float ss = 0.f;
        for (int d = lane; d < hd; d += 32) ss += src[d] * src[d];
        ss = warp_sum(ss);
        r = 1.0f / sqrtf(ss / hd + eps);
    }
    long long slot = 0;
    if (!is_q) {
        slot = slots[tok];
        if (slot < 0 || slot >= cache_rows) {
            if (lane == 0) atomicOr(err, kErrBadArgs);
            return;
        }
    }
    auto emit = [&](int d, float val) {
        if (is_q) {
            const long long o = (tok * heads + h) * hd + d;
            if (q_out_f32) q_out_f32[o] = val;
            if (q_out_bf16) {
                __nv_bfloat16 b = __float2bfloat16_rn(val);
                q_out_bf16[o] = *reinterpret_cast<uint16_t *>(&b);
            }
        } else {
            __nv_bfloat16 b = __float2bfloat16_rn(val);
            k_cache[(slot * heads + h) * hd + d] = *reinterpret_cast<uint16_t *>(&b);
        }
    };
    const int half = hd / 2;
    if (c) {
        for (int i = lane; i < half; i += 32) {
            const int d0 = interleaved ? 2 * i : i;
            const int d1 = interleaved ? 2 * i + 1 : i + half;
            float x0 = src[d0], x1 = src[d1];
            if (w) {
                x0 = x0 * r * w[d0];
                x1 = x1 * r * w[d1];
            }
            emit(d0, x0 * c[d0] - x1 * s[d0]);
            emit(d1, x1 * c[d1] + x0 * s[d1]);
        }
        if ((hd & 1) && lane == 0) emit(hd - 1, w ? src[hd - 1] * r * w[hd - 1] : src[hd - 1]);
    } else {
        for (int d = lane; d < hd; d += 32) emit(d, w ? src[d] * r * w[d] : src[d]);
    }
    if (!is_q) {
        const float *vs = v_in + (tok * heads + h) * hd;
        uint16_t *vd = v_cache + (slot * heads + h) * hd;
        bool over = false;
        for (int d = lane; d < hd; d += 32) {
            __half hv = __float2half_rn(vs[d]);
            vd[d] = *reinterpret_cast<uint16_t *>(&hv);
            over |= f16_overflows(vs[d]);
        }
        // the V cache is fp16: a value it cannot hold is reported, not stored silently as inf
        if (__any_sync(0xffffffffu, over) && lane == 0 && err) atomicOr(err, kErrValueRange);
    }
}

// dst[r, hh*padded_hd + d] = convert(src[r, hh*head_dim + d]) for d < head_dim, 0 for the padding.
__global__ void pack_rows_kernel(uint16_t *dst, long long dst_stride, int dst_width, const float *src,
                                 long long src_stride, int src_heads, int head_dim, int padded_hd, long long rows,
                                 int to_f16, unsigned *err)
{
    const long long total = rows * dst_width;
    for (long long i = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x; i < total;
         i += static_cast<long long>(gridDim.x) * blockDim.x) {
        const long long r = i / dst_width;
        const int col = static_cast<int>(i % dst_width);
        const int hh = col / padded_hd, d = col % padded_hd;
        float v = 0.f;
        if (hh < src_heads && d < head_dim) v = src[r * src_stride + static_cast<long long>(hh) * head_dim + d];
        uint16_t bits;
        if (to_f16) {
            __half x = __float2half_rn(v);
            bits = *reinterpret_cast<uint16_t *>(&x);
            if (f16_overflows(v) && err) atomicOr(err, kErrValueRange);
        } else {
            __nv_bfloat16 x = __float2bfloat16_rn(v);
            bits = *reinterpret_cast<uint16_t *>(&x);
        }
        dst[r * dst_stride + col] = bits;
    }
}

__global__ void unpack_rows_kernel(float *dst, long long dst_stride, const float *src, long long src_stride,
                                   int heads, int head_dim, int padded_hd, long long rows)
{
    const int width = heads * head_dim;
    const long long total = rows * width;
    for (long long i = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x; i < total;
         i += static_cast<long long>(gridDim.x) * blockDim.x) {
        const long long r = i / width;
        const int col = static_cast<int>(i % width);
        const int hh = col / head_dim, d = col % head_dim;
        dst[r * dst_stride + col] = src[r * src_stride + static_cast<long long>(hh) * padded_hd + d];
    }
}

__global__ void decode_step_index_kernel(int *positions, int64_t *slots, int *kv_len_next, const int64_t *seq_row0,
                                         const int *kv_len, int n)
{
    const int b = blockIdx.x * blockDim.x + threadIdx.x;
    if (b >= n) return;
    const int L = kv_len[b];
    positions[b] = L;
    slots[b] = seq_row0[b] + L;
    kv_len_next[b] = L + 1;
}

// One thread waits on phase 0 of an mbarrier that nothing ever arrives on: the
// bounded wait runs out after kWaitLimitNs, or-s kErrWaitTmaFull into the device error
// word and the kernel returns normally (no fault, no trap, no hang).
__global__ void watchdog_selftest_kernel(unsigned *err)
{
    __shared__ __align__(8) uint64_t bar;
    if (threadIdx.x == 0) {
        mbar_init(smem_u32(&bar), 1);
        fence_mbar_init();
        mbar_wait(smem_u32(&bar), 0, err, kErrWaitTmaFull);
    }
}

int grid_for(long long total, int per_block)
{
    long long g = (total + per_block - 1) / per_block;
    if (g > 148LL * 64) g = 148LL * 64;
    return static_cast<int>(g < 1 ? 1 : g);
}

}  // namespace

int launch_rms_norm_per_head(cudaStream_t st, float *x, const float *w, int seq_len, int n_heads, int head_dim,
                             float eps)
{
    const long long rows = static_cast<long long>(seq_len) * n_heads;
    if (rows <= 0 || head_dim <= 0) return SMOL_B200_OK;
    const long long blocks = (rows + kWarpsPerBlock - 1) / kWarpsPerBlock;
    if (blocks > 0x7fffffffLL) return SMOL_B200_ERR_ARGS;
    rms_norm_per_head_kernel<<<static_cast<unsigned>(blocks), kWarpsPerBlock * 32, 0, st>>>(x, w, rows, head_dim,
                                                                                             eps);
    return cudaGetLastError() == cudaSuccess ? SMOL_B200_OK : SMOL_B200_ERR_CUDA;
}

int launch_rms_norm(cudaStream_t st, float *out, const float *x, const float *w, int seq_len, int hidden, float eps)
{
    if (seq_len <= 0 || hidden <= 0) return SMOL_B200_OK;
    rms_norm_kernel<<<seq_len, 256, 0, st>>>(out, x, w, hidden, eps);
    return cudaGetLastError() == cudaSuccess ? SMOL_B200_OK : SMOL_B200_ERR_CUDA;
}

int launch_rope(cudaStream_t st, float *x, const float *cos_vals, const float *sin_vals, int seq, int n_heads,
                int head_dim, int interleaved)
{
    const long long rows = static_cast<long long>(seq) * n_heads;
    if (rows <= 0 || head_dim <= 1) return SMOL_B200_OK;
    const long long blocks = (rows + kWarpsPerBlock - 1) / kWarpsPerBlock;
    if (blocks > 0x7fffffffLL) return SMOL_B200_ERR_ARGS;
    rope_kernel<<<static_cast<unsigned>(blocks), kWarpsPerBlock * 32, 0, st>>>(x, cos_vals, sin_vals, rows, n_heads,
                                                                                head_dim, interleaved);
    return cudaGetLastError() == cudaSuccess ? SMOL_B200_OK : SMOL_B200_ERR_CUDA;
}

int qknorm_rope_append(cudaStream_t st, const float *q_in, const float *k_in, const float *v_in, int n_tokens,
                       int n_heads, int n_kv_heads, int head_dim, const float *q_norm_w, const float *k_norm_w,
                       float eps, const float *rope_cos, const float *rope_sin, int rope_interleaved,
                       const int *positions, const int64_t *slots, float *q_out_f32, uint16_t *q_out_bf16,
                       uint16_t *k_cache_bf16, uint16_t *v_cache_f16, int64_t cache_rows)
{
    if (n_tokens <= 0) return SMOL_B200_OK;
    if (!q_in || !k_in || !v_in || !slots || !k_cache_bf16 || !v_cache_f16 || n_heads <= 0 || n_kv_heads <= 0 ||
        head_dim <= 0 || head_dim > 1024 || ((rope_cos || rope_sin) && (!rope_cos || !rope_sin || !positions)))
        return SMOL_B200_ERR_ARGS;
    unsigned *err = device_error_word();
    if (!err) return SMOL_B200_ERR_NO_DEVICE;
    const long long warps = static_cast<long long>(n_tokens) * (n_heads + n_kv_heads);
    const long long blocks = (warps + kWarpsPerBlock - 1) / kWarpsPerBlock;
    if (blocks > 0x7fffffffLL) return SMOL_B200_ERR_ARGS;
    PdlScope pdl(g_api_pdl);   // the kernel waits (griddepcontrol.wait) before reading its inputs
    const cudaError_t e = launch_kernel(
        qknorm_rope_append_kernel, dim3(static_cast<unsigned>(blocks)), dim3(kWarpsPerBlock * 32), 0, st, q_in, k_in,
        v_in, n_tokens, n_heads, n_kv_heads, head_dim, q_norm_w, k_norm_w, eps, rope_cos, rope_sin, rope_interleaved,
        positions, slots, q_out_f32, q_out_bf16, k_cache_bf16, v_cache_f16, static_cast<long long>(cache_rows), err);
    return e == cudaSuccess ? SMOL_B200_OK : SMOL_B200_ERR_CUDA;
}

int launch_pack_rows(cudaStream_t st, uint16_t *dst, int64_t dst_stride, int dst_width, const float *src,
                     int64_t src_stride, int src_heads, int head_dim, int padded_hd, int64_t rows, int to_f16)
{
    if (rows <= 0 || dst_width <= 0) return SMOL_B200_OK;
    pack_rows_kernel<<<grid_for(rows * dst_width, 256), 256, 0, st>>>(dst, dst_stride, dst_width, src, src_stride,
                                                                       src_heads, head_dim, padded_hd, rows, to_f16,
                                                                       to_f16 ? device_error_word() : nullptr);
    return cudaGetLastError() == cudaSuccess ? SMOL_B200_OK : SMOL_B200_ERR_CUDA;
}

int launch_unpack_rows(cudaStream_t st, float *dst, int64_t dst_stride, const float *src, int64_t src_stride,
                       int heads, int head_dim, int padded_hd, int64_t rows)
{
    if (rows <= 0 || heads <= 0 || head_dim <= 0) return SMOL_B200_OK;
    unpack_rows_kernel<<<grid_for(rows * heads * head_dim, 256), 256, 0, st>>>(dst, dst_stride, src, src_stride,
                                                                                heads, head_dim, padded_hd, rows);
    return cudaGetLastError() == cudaSuccess ? SMOL_B200_OK : SMOL_B200_ERR_CUDA;
}

int launch_watchdog_selftest(cudaStream_t st)
{
    unsigned *err = device_error_word();
    if (!err) return SMOL_B200_ERR_NO_DEVICE;
    watchdog_selftest_kernel<<<1, 32, 0, st>>>(err);
    return cudaGetLastError() == cudaSuccess ? SMOL_B200_OK : SMOL_B200_ERR_CUDA;
}

int launch_decode_step_index(cudaStream_t st, int *positions, int64_t *slots, int *kv_len_next,
                             const int64_t *seq_row0, const int *kv_len, int n_seqs)
{
    if (n_seqs <= 0) return SMOL_B200_OK;
    decode_step_index_kernel<<<(n_seqs + 255) / 256, 256, 0, st>>>(positions, slots, kv_len_next, seq_row0, kv_len,
                                                                    n_seqs);
    return cudaGetLastError() == cudaSuccess ? SMOL_B200_OK : SMOL_B200_ERR_CUDA;
}

}  // namespace smolb200
