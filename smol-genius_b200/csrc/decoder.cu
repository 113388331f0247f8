// decoder.cu -- the rest of a decode step around attention, on the device.
//
// Replaces what qkn_decoder_forward (qkn_decoder.c:570-714) runs on the host between
// the attention calls: bf16 matrix-vector products (bf16_matvec_fused,
// bf16_matvec_avx.c:24-150: fp32 activations times bf16 weights widened to fp32,
// fp32 accumulation), the SwiGLU gate (activation.c:55-86), residual adds
// (matmul.c:33-35), RMSNorm (rmsnorm.c:17-70) and the greedy argmax over the tied
// embedding matrix (matmul.c:371-398, bf16_matvec_avx.c:156-250).
//
// The products are HBM-bound for a batch of a few sequences: every weight is read
// once per step and reused for all (<= 8) sequences of a launch.  One warp owns one
// output row (two for the gated form); its lanes stream the row in 16-byte pieces
// (8 bf16 weights), several pieces in flight per lane, while the activations of the
// launch's sequences sit in shared memory.  Algorithmic bytes per launch: rows *
// k_dim * 2 (weights) + n_seqs * (k_dim + rows) * 4 (activations).
#include <stdio.h>
#include <string.h>

#include <vector>

#include "b200_common.cuh"
#include "runtime.h"

namespace smolb200 {
namespace {

constexpr int kGemvWarps = 8;
constexpr int kGemvThreads = kGemvWarps * 32;
constexpr int kMaxBatch = 8;   // sequences per launch (larger batches loop)
constexpr int kMaxXsBytes = 200 * 1024;   // staged activations: kMaxBatch x k_dim fp32 (k_dim <= 6400)

struct GemvSeg {
    const uint16_t *w;
    float *y;
    long long ldy;   // row stride of y (per sequence)
    int rows;        // rows of W in this segment
};

struct GemvParams {
    GemvSeg seg[3];
    int nseg;
    int total_rows;
    const float *x;
    long long ldx;
    const float *norm_w;   // non-null: x is RMS-normalised with these weights first
    float eps;
    int k_dim;
    int nb;     // sequences in this launch (<= NB)
    int mode;   // 0 store, 1 add, 2 gated pairs
};

__device__ __forceinline__ uint4 ldg_stream(const void *p)
{
    uint4 v;
    asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0, %1, %2, %3}, [%4];"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                 : "l"(p));
    return v;
}

__device__ __forceinline__ float warp_sum(float v)
{
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

// acc[b] += dot(8 weights in w, x[b][k..k+8))
template <int NB>
__device__ __forceinline__ void fma8(float (&acc)[NB], const uint4 &w, const float *xs, int k_dim, int k, int nb)
{
    float wf[8];
    const uint32_t u[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        wf[2 * j] = bf16lo_f32(u[j]);
        wf[2 * j + 1] = bf16hi_f32(u[j]);
    }
#pragma unroll
    for (int b = 0; b < NB; ++b) {
        if (b < nb) {
            const float4 xa = *reinterpret_cast<const float4 *>(xs + b * k_dim + k);
            const float4 xb = *reinterpret_cast<const float4 *>(xs + b * k_dim + k + 4);
            float a = acc[b];
            a = fmaf(wf[0], xa.x, a);
            a = fmaf(wf[1], xa.y, a);
            a = fmaf(wf[2], xa.z, a);
            a = fmaf(wf[3], xa.w, a);
            a = fmaf(wf[4], xb.x, a);
            a = fmaf(wf[5], xb.y, a);
            a = fmaf(wf[6], xb.z, a);
            a = fmaf(wf[7], xb.w, a);
            acc[b] = a;
        }
    }
}

// Stage x[b][0..k_dim) of the launch's sequences in shared memory (float4 pieces).
// With norm_w, each row becomes smol_rms_norm's (x * w) * 1/sqrtf(mean(x^2) + eps)
// (rmsnorm.c:17-70), so the normalised activations never go through global memory.
template <int NB>
__device__ __forceinline__ void stage_x(float *xs, const float *x, long long ldx, int k_dim, int nb,
                                        const float *norm_w, float eps)
{
    const int n4 = nb * k_dim / 4;
    float ss[NB];
#pragma unroll
    for (int b = 0; b < NB; ++b) ss[b] = 0.f;
    for (int i = threadIdx.x; i < n4; i += blockDim.x) {
        const int e = i * 4, b = e / k_dim, k = e % k_dim;
        const float4 v = *reinterpret_cast<const float4 *>(x + b * ldx + k);
        *reinterpret_cast<float4 *>(xs + e) = v;
        if (norm_w) {
#pragma unroll
            for (int bb = 0; bb < NB; ++bb)
                if (bb == b) ss[bb] += v.x * v.x + v.y * v.y + v.z * v.z + v.w * v.w;
        }
    }
    if (norm_w) {
        __shared__ float part[kGemvWarps][NB];
        __shared__ float rinv[NB];
        const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
#pragma unroll
        for (int b = 0; b < NB; ++b) {
            const float t = warp_sum(ss[b]);
            if (lane == 0) part[warp][b] = t;
        }
        __syncthreads();
        if (threadIdx.x < nb) {
            float t = 0.f;
            for (int w = 0; w < kGemvWarps; ++w) t += part[w][threadIdx.x];
            rinv[threadIdx.x] = 1.0f / sqrtf(t / static_cast<float>(k_dim) + eps);
        }
        __syncthreads();
        for (int i = threadIdx.x; i < n4; i += blockDim.x) {
            const int e = i * 4, b = e / k_dim, k = e % k_dim;
            float4 v = *reinterpret_cast<float4 *>(xs + e);
            const float4 w = *reinterpret_cast<const float4 *>(norm_w + k);
            const float r = rinv[b];
            v.x = v.x * w.x * r;
            v.y = v.y * w.y * r;
            v.z = v.z * w.z * r;
            v.w = v.w * w.w * r;
            *reinterpret_cast<float4 *>(xs + e) = v;
        }
    }
    __syncthreads();
}

// Pull a weight row into L2 ahead of the dependency wait (weights never change).
__device__ __forceinline__ void prefetch_row_l2(const uint16_t *row, int k_dim, int lane)
{
    const char *p = reinterpret_cast<const char *>(row);
    for (int off = lane * 128; off < k_dim * 2; off += 32 * 128)
        asm volatile("prefetch.global.L2 [%0];" ::"l"(p + off));
}

template <int NB>
__global__ void __launch_bounds__(kGemvThreads) gemv_bf16_kernel(const __grid_constant__ GemvParams p)
{
    extern __shared__ float xs[];   // [nb][k_dim]
    griddep_trigger();
    const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
    const int rpw = p.mode == 2 ? 2 : 1;   // weight rows per warp
    const int k_dim = p.k_dim;
    {   // this warp's first rows stream from HBM while the previous kernel finishes
        const int r0 = (blockIdx.x * kGemvWarps + warp) * rpw;
        if (r0 < p.total_rows) {
            int s = 0, r = r0;
            while (s + 1 < p.nseg && r >= p.seg[s].rows) {
                r -= p.seg[s].rows;
                ++s;
            }
            for (int i = 0; i < rpw; ++i) prefetch_row_l2(p.seg[s].w + static_cast<size_t>(r + i) * k_dim, k_dim, lane);
        }
    }
    griddep_wait();
    stage_x<NB>(xs, p.x, p.ldx, p.k_dim, p.nb, p.norm_w, p.eps);
    for (int r0 = (blockIdx.x * kGemvWarps + warp) * rpw; r0 < p.total_rows; r0 += gridDim.x * kGemvWarps * rpw) {
        int s = 0, r = r0;
        while (s + 1 < p.nseg && r >= p.seg[s].rows) {
            r -= p.seg[s].rows;
            ++s;
        }
        const uint16_t *w0 = p.seg[s].w + static_cast<size_t>(r) * k_dim;
        float acc0[NB], acc1[NB];
#pragma unroll
        for (int b = 0; b < NB; ++b) acc0[b] = acc1[b] = 0.f;
        if (rpw == 1) {
            int k = lane * 8;
            // four 16-byte pieces in flight per lane
            for (; k + 3 * 256 < k_dim; k += 4 * 256) {
                const uint4 a = ldg_stream(w0 + k), b1 = ldg_stream(w0 + k + 256), c = ldg_stream(w0 + k + 512),
                            d = ldg_stream(w0 + k + 768);
                fma8<NB>(acc0, a, xs, k_dim, k, p.nb);
                fma8<NB>(acc0, b1, xs, k_dim, k + 256, p.nb);
                fma8<NB>(acc0, c, xs, k_dim, k + 512, p.nb);
                fma8<NB>(acc0, d, xs, k_dim, k + 768, p.nb);
            }
            for (; k < k_dim; k += 256) fma8<NB>(acc0, ldg_stream(w0 + k), xs, k_dim, k, p.nb);
        } else {
            const uint16_t *w1 = w0 + k_dim;
            int k = lane * 8;
            for (; k + 256 < k_dim; k += 2 * 256) {
                const uint4 a = ldg_stream(w0 + k), b1 = ldg_stream(w1 + k), c = ldg_stream(w0 + k + 256),
                            d = ldg_stream(w1 + k + 256);
                fma8<NB>(acc0, a, xs, k_dim, k, p.nb);
                fma8<NB>(acc1, b1, xs, k_dim, k, p.nb);
                fma8<NB>(acc0, c, xs, k_dim, k + 256, p.nb);
                fma8<NB>(acc1, d, xs, k_dim, k + 256, p.nb);
            }
            for (; k < k_dim; k += 256) {
                fma8<NB>(acc0, ldg_stream(w0 + k), xs, k_dim, k, p.nb);
                fma8<NB>(acc1, ldg_stream(w1 + k), xs, k_dim, k, p.nb);
            }
        }
#pragma unroll
        for (int b = 0; b < NB; ++b) {
            if (b < p.nb) {
                const float s0 = warp_sum(acc0[b]);
                const float s1 = rpw == 2 ? warp_sum(acc1[b]) : 0.f;
                if (lane == 0) {
                    float *y = p.seg[s].y + b * p.seg[s].ldy;
                    if (p.mode == 0) {
                        y[r] = s0;
                    } else if (p.mode == 1) {
                        y[r] = y[r] + s0;
                    } else {
                        const float g = s0 / (1.0f + expf(-s0));   // SiLU, activation.c:81
                        y[r / 2] = g * s1;
                    }
                }
            }
        }
    }
}

// Greedy argmax over the rows of E: per CTA the best (value, row) of each sequence.
// A row wins over another when its value is larger, or equal with a lower index
// (the reference's strict '>' scan from row 0 keeps the first maximum).
template <int NB>
__global__ void __launch_bounds__(kGemvThreads) argmax_rows_kernel(float *part_val, int *part_idx, const float *x,
                                                                    long long ldx, const uint16_t *emb, int vocab,
                                                                    int k_dim, int nb, const float *norm_w, float eps,
                                                                    float *x_normed)
{
    extern __shared__ float xs[];
    griddep_trigger();
    {
        const int r = blockIdx.x * kGemvWarps + threadIdx.x / 32;
        if (r < vocab) prefetch_row_l2(emb + static_cast<size_t>(r) * k_dim, k_dim, threadIdx.x % 32);
    }
    griddep_wait();
    stage_x<NB>(xs, x, ldx, k_dim, nb, norm_w, eps);
    if (x_normed && blockIdx.x == 0) {   // the normalised final state, for callers that read it
        for (int i = threadIdx.x; i < nb * k_dim; i += blockDim.x)
            x_normed[(i / k_dim) * ldx + i % k_dim] = xs[i];
    }
    __shared__ float wbest[kGemvWarps][NB];
    __shared__ int wbidx[kGemvWarps][NB];
    const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
    float best[NB];
    int bidx[NB];
#pragma unroll
    for (int b = 0; b < NB; ++b) {
        best[b] = -1e30f;   // the reference's initial best value (bf16_matvec_avx.c:160)
        bidx[b] = 0;
    }
    for (int r = blockIdx.x * kGemvWarps + warp; r < vocab; r += gridDim.x * kGemvWarps) {
        const uint16_t *w0 = emb + static_cast<size_t>(r) * k_dim;
        float acc[NB];
#pragma unroll
        for (int b = 0; b < NB; ++b) acc[b] = 0.f;
        int k = lane * 8;
        for (; k + 256 < k_dim; k += 2 * 256) {
            const uint4 a = ldg_stream(w0 + k), c = ldg_stream(w0 + k + 256);
            fma8<NB>(acc, a, xs, k_dim, k, nb);
            fma8<NB>(acc, c, xs, k_dim, k + 256, nb);
        }
        for (; k < k_dim; k += 256) fma8<NB>(acc, ldg_stream(w0 + k), xs, k_dim, k, nb);
#pragma unroll
        for (int b = 0; b < NB; ++b) {
            const float v = warp_sum(acc[b]);   // identical in every lane
            if (v > best[b] || (v == best[b] && r < bidx[b])) {
                best[b] = v;
                bidx[b] = r;
            }
        }
    }
    if (lane == 0) {
#pragma unroll
        for (int b = 0; b < NB; ++b) {
            wbest[warp][b] = best[b];
            wbidx[warp][b] = bidx[b];
        }
    }
    __syncthreads();
    if (threadIdx.x < nb) {
        const int b = threadIdx.x;
        float bv = wbest[0][b];
        int bi = wbidx[0][b];
        for (int w = 1; w < kGemvWarps; ++w) {
            const float v = wbest[w][b];
            const int i = wbidx[w][b];
            if (v > bv || (v == bv && i < bi)) {
                bv = v;
                bi = i;
            }
        }
        part_val[blockIdx.x * kMaxBatch + b] = bv;
        part_idx[blockIdx.x * kMaxBatch + b] = bi;
    }
}

__global__ void argmax_final_kernel(int *tokens_out, const float *part_val, const int *part_idx, int nparts)
{
    griddep_trigger();
    griddep_wait();
    // one warp per sequence (blockIdx.x)
    const int b = blockIdx.x, lane = threadIdx.x;
    float bv = -1e30f;
    int bi = 0;
    for (int i = lane; i < nparts; i += 32) {
        const float v = part_val[i * kMaxBatch + b];
        const int ix = part_idx[i * kMaxBatch + b];
        if (v > bv || (v == bv && ix < bi)) {
            bv = v;
            bi = ix;
        }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const float v = __shfl_xor_sync(0xffffffffu, bv, o);
        const int ix = __shfl_xor_sync(0xffffffffu, bi, o);
        if (v > bv || (v == bv && ix < bi)) {
            bv = v;
            bi = ix;
        }
    }
    if (lane == 0) tokens_out[b] = bi;
}

// x[b][:] = E[tokens[b]][:] (bf16 -> fp32)
__global__ void embed_kernel(float *x, const int *tokens, const uint16_t *emb, int hidden, int vocab, unsigned *err)
{
    griddep_trigger();
    griddep_wait();
    const int b = blockIdx.x;
    int t = tokens[b];
    if (t < 0 || t >= vocab) {
        if (threadIdx.x == 0) atomicOr(err, kErrBadArgs);
        t = 0;
    }
    const uint16_t *e = emb + static_cast<size_t>(t) * hidden;
    for (int i = threadIdx.x; i < hidden; i += blockDim.x)
        x[static_cast<size_t>(b) * hidden + i] = __uint_as_float(static_cast<uint32_t>(e[i]) << 16);
}

// positions[b] = kv_len[b]; kv_next[b] = kv_len[b] + 1; slots[l][b] = row0[l][b] + kv_len[b]
__global__ void step_index_kernel(int *positions, int *kv_next, int64_t *slots, const int64_t *layer_row0,
                                  const int *kv_len, int n_seqs, int n_layers)
{
    griddep_trigger();
    griddep_wait();
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n_seqs * n_layers) return;
    const int b = i % n_seqs;
    const int len = kv_len[b];
    slots[i] = layer_row0[i] + len;
    if (i < n_seqs) {
        positions[b] = len;
        kv_next[b] = len + 1;
    }
}

__global__ void advance_kernel(int *kv_len, int n_seqs)
{
    griddep_trigger();
    griddep_wait();
    const int b = blockIdx.x * blockDim.x + threadIdx.x;
    if (b < n_seqs) kv_len[b] += 1;
}

int gemv_smem_bytes(int nb, int k_dim)
{
    return nb * k_dim * static_cast<int>(sizeof(float));
}

template <int NB>
int launch_gemv_nb(cudaStream_t st, GemvParams &p)
{
    const int smem = gemv_smem_bytes(p.nb, p.k_dim);
    if (smem > 48 * 1024) {
        static bool raised[64] = {};
        const int dev = current_device();
        if (dev < 0 || dev >= 64) return SMOL_B200_ERR_CUDA;
        if (!raised[dev]) {
            // dynamic + static (the norm partials) must stay within the 227 KB per block
            if (cudaFuncSetAttribute(gemv_bf16_kernel<NB>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     kMaxXsBytes) != cudaSuccess)
                return SMOL_B200_ERR_CUDA;
            raised[dev] = true;
        }
    }
    const int rpw = p.mode == 2 ? 2 : 1;
    const long long warps = (p.total_rows + rpw - 1) / rpw;
    long long grid = (warps + kGemvWarps - 1) / kGemvWarps;
    if (grid > 148LL * 16) grid = 148LL * 16;
    return launch_kernel(gemv_bf16_kernel<NB>, dim3(static_cast<unsigned>(grid)), dim3(kGemvThreads), smem, st, p) ==
                   cudaSuccess
               ? SMOL_B200_OK
               : SMOL_B200_ERR_CUDA;
}

// Runs the segmented product for every sequence, kMaxBatch sequences per launch.
int run_gemv(cudaStream_t st, GemvParams p, int n_seqs)
{
    if (p.k_dim <= 0 || p.k_dim % 8 || (p.ldx & 3) || p.total_rows <= 0) return SMOL_B200_ERR_ARGS;
    if (gemv_smem_bytes(kMaxBatch, p.k_dim) > kMaxXsBytes) return SMOL_B200_ERR_ARGS;
    for (int s = 0; s < p.nseg; ++s)
        if (!p.seg[s].w || !p.seg[s].y || (reinterpret_cast<uintptr_t>(p.seg[s].w) & 15)) return SMOL_B200_ERR_ARGS;
    if (!p.x || (reinterpret_cast<uintptr_t>(p.x) & 15)) return SMOL_B200_ERR_ARGS;
    for (int b0 = 0; b0 < n_seqs; b0 += kMaxBatch) {
        GemvParams q = p;
        q.nb = n_seqs - b0 < kMaxBatch ? n_seqs - b0 : kMaxBatch;
        q.x = p.x + static_cast<long long>(b0) * p.ldx;
        for (int s = 0; s < p.nseg; ++s) q.seg[s].y = p.seg[s].y + static_cast<long long>(b0) * p.seg[s].ldy;
        int rc;
        if (q.nb == 1) rc = launch_gemv_nb<1>(st, q);
        else if (q.nb == 2) rc = launch_gemv_nb<2>(st, q);
        else if (q.nb <= 4) rc = launch_gemv_nb<4>(st, q);
        else rc = launch_gemv_nb<8>(st, q);
        if (rc != SMOL_B200_OK) return rc;
    }
    return SMOL_B200_OK;
}

constexpr int kArgmaxBlocks = 148 * 4;

size_t argmax_ws_bytes(int n_seqs)
{
    const int launches = (n_seqs + kMaxBatch - 1) / kMaxBatch;
    (void)launches;
    return static_cast<size_t>(kArgmaxBlocks) * kMaxBatch * (sizeof(float) + sizeof(int));
}

template <int NB>
int launch_argmax_nb(cudaStream_t st, float *pv, int *pi, const float *x, long long ldx, const uint16_t *emb,
                     int vocab, int k_dim, int nb, const float *norm_w, float eps, float *x_normed)
{
    const int smem = gemv_smem_bytes(nb, k_dim);
    if (smem > 48 * 1024) {
        static bool raised[64] = {};
        const int dev = current_device();
        if (dev < 0 || dev >= 64) return SMOL_B200_ERR_CUDA;
        if (!raised[dev]) {
            if (cudaFuncSetAttribute(argmax_rows_kernel<NB>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     kMaxXsBytes) != cudaSuccess)
                return SMOL_B200_ERR_CUDA;
            raised[dev] = true;
        }
    }
    return launch_kernel(argmax_rows_kernel<NB>, dim3(kArgmaxBlocks), dim3(kGemvThreads), smem, st, pv, pi, x, ldx,
                         emb, vocab, k_dim, nb, norm_w, eps, x_normed) == cudaSuccess
               ? SMOL_B200_OK
               : SMOL_B200_ERR_CUDA;
}

int run_argmax(cudaStream_t st, int *tokens_out, const float *x, long long ldx, const uint16_t *emb, int vocab,
               int k_dim, int n_seqs, void *ws, size_t ws_bytes, const float *norm_w = nullptr, float eps = 0.f,
               float *x_normed = nullptr)
{
    if (n_seqs <= 0) return SMOL_B200_OK;
    if (!tokens_out || !x || !emb || vocab <= 0 || k_dim <= 0 || k_dim % 8 || (ldx & 3) ||
        (reinterpret_cast<uintptr_t>(emb) & 15) || (reinterpret_cast<uintptr_t>(x) & 15))
        return SMOL_B200_ERR_ARGS;
    if (!ws || ws_bytes < argmax_ws_bytes(n_seqs)) return SMOL_B200_ERR_WORKSPACE;
    if (gemv_smem_bytes(kMaxBatch, k_dim) > kMaxXsBytes) return SMOL_B200_ERR_ARGS;
    float *pv = static_cast<float *>(ws);
    int *pi = reinterpret_cast<int *>(pv + kArgmaxBlocks * kMaxBatch);
    for (int b0 = 0; b0 < n_seqs; b0 += kMaxBatch) {
        const int nb = n_seqs - b0 < kMaxBatch ? n_seqs - b0 : kMaxBatch;
        const float *xb = x + static_cast<long long>(b0) * ldx;
        float *xo = x_normed ? x_normed + static_cast<long long>(b0) * ldx : nullptr;
        int rc;
        if (nb == 1) rc = launch_argmax_nb<1>(st, pv, pi, xb, ldx, emb, vocab, k_dim, nb, norm_w, eps, xo);
        else if (nb == 2) rc = launch_argmax_nb<2>(st, pv, pi, xb, ldx, emb, vocab, k_dim, nb, norm_w, eps, xo);
        else if (nb <= 4) rc = launch_argmax_nb<4>(st, pv, pi, xb, ldx, emb, vocab, k_dim, nb, norm_w, eps, xo);
        else rc = launch_argmax_nb<8>(st, pv, pi, xb, ldx, emb, vocab, k_dim, nb, norm_w, eps, xo);
        if (rc != SMOL_B200_OK) return rc;
        if (launch_kernel(argmax_final_kernel, dim3(nb), dim3(32), 0, st, tokens_out + b0, pv, pi, kArgmaxBlocks) !=
            cudaSuccess)
            return SMOL_B200_ERR_CUDA;
    }
    return SMOL_B200_OK;
}

// Workspace of one decoder step, carved in 256-byte aligned pieces.
struct StepWs {
    float *x, *xn, *q, *k, *v, *qr, *attn, *act;
    int *positions, *kv_next;
    int64_t *slots;
    void *attn_ws;
    size_t attn_ws_bytes;
    void *argmax_ws;
    size_t argmax_ws_bytes;
    size_t total;
};

StepWs carve(const smol_b200_qkn_model &m, int n_seqs, int max_kv_len, uint8_t *base)
{
    StepWs w;
    memset(&w, 0, sizeof(w));
    size_t off = 0;
    auto take = [&](size_t bytes) {
        uint8_t *p = base ? base + off : nullptr;
        off += (bytes + 255) / 256 * 256;
        return p;
    };
    const size_t B = static_cast<size_t>(n_seqs);
    const size_t qd = static_cast<size_t>(m.n_heads) * m.head_dim, kvd = static_cast<size_t>(m.n_kv_heads) * m.head_dim;
    w.x = reinterpret_cast<float *>(take(B * m.hidden * 4));
    w.xn = reinterpret_cast<float *>(take(B * m.hidden * 4));
    w.q = reinterpret_cast<float *>(take(B * qd * 4));
    w.k = reinterpret_cast<float *>(take(B * kvd * 4));
    w.v = reinterpret_cast<float *>(take(B * kvd * 4));
    w.qr = reinterpret_cast<float *>(take(B * qd * 4));
    w.attn = reinterpret_cast<float *>(take(B * qd * 4));
    w.act = reinterpret_cast<float *>(take(B * m.intermediate * 4));
    w.positions = reinterpret_cast<int *>(take(B * 4));
    w.kv_next = reinterpret_cast<int *>(take(B * 4));
    w.slots = reinterpret_cast<int64_t *>(take(B * m.n_layers * 8));
    w.attn_ws_bytes = decode_workspace_bytes(n_seqs, max_kv_len + 1, m.n_heads, m.n_kv_heads, m.head_dim);
    w.attn_ws = take(w.attn_ws_bytes);
    w.argmax_ws_bytes = argmax_ws_bytes(n_seqs);
    w.argmax_ws = take(w.argmax_ws_bytes);
    w.total = off;
    return w;
}

bool model_ok(const smol_b200_qkn_model *m)
{
    return m && m->hidden > 0 && m->n_layers > 0 && m->n_heads > 0 && m->n_kv_heads > 0 && m->head_dim > 0 &&
           m->n_heads % m->n_kv_heads == 0 && m->intermediate > 0 && m->vocab > 0 && m->tok_embeddings &&
           m->final_norm && m->layers && m->hidden % 8 == 0 && m->intermediate % 8 == 0 &&
           (m->n_heads * m->head_dim) % 8 == 0;
}

}  // namespace

int gemv_norm_bf16(cudaStream_t st, float *y, int64_t ldy, const float *x, int64_t ldx, const uint16_t *w,
                   int n_out, int k_dim, int n_seqs, int mode, const float *norm_w, float eps)
{
    if (n_seqs <= 0 || n_out <= 0) return SMOL_B200_OK;
    if (mode < 0 || mode > 2 || (ldy < n_out)) return SMOL_B200_ERR_ARGS;
    GemvParams p;
    memset(&p, 0, sizeof(p));
    p.seg[0] = {w, y, ldy, mode == 2 ? 2 * n_out : n_out};
    p.nseg = 1;
    p.total_rows = p.seg[0].rows;
    p.x = x;
    p.ldx = ldx;
    p.norm_w = norm_w;
    p.eps = eps;
    p.k_dim = k_dim;
    p.mode = mode;
    return run_gemv(st, p, n_seqs);
}

int gemv_bf16(cudaStream_t st, float *y, int64_t ldy, const float *x, int64_t ldx, const uint16_t *w, int n_out,
              int k_dim, int n_seqs, int mode)
{
    return gemv_norm_bf16(st, y, ldy, x, ldx, w, n_out, k_dim, n_seqs, mode, nullptr, 0.f);
}

int argmax_bf16(cudaStream_t st, int *tokens_out, const float *x, int64_t ldx, const uint16_t *emb, int vocab,
                int k_dim, int n_seqs, void *ws, size_t ws_bytes)
{
    return run_argmax(st, tokens_out, x, ldx, emb, vocab, k_dim, n_seqs, ws, ws_bytes);
}

size_t argmax_workspace_bytes(int n_seqs)
{
    return argmax_ws_bytes(n_seqs);
}

size_t qkn_step_workspace_bytes(const smol_b200_qkn_model *m, int n_seqs, int max_kv_len)
{
    if (!model_ok(m) || n_seqs <= 0 || max_kv_len < 0) return 0;
    return carve(*m, n_seqs, max_kv_len, nullptr).total;
}

int qkn_decode_step(cudaStream_t st, const smol_b200_qkn_model *mp, int n_seqs, const int *tokens_in,
                    int *tokens_out, uint16_t *k_pool, uint16_t *v_pool, int64_t pool_rows,
                    const int64_t *layer_row0, int *kv_len, int max_kv_len, const float *rope_cos,
                    const float *rope_sin, int advance, void *workspace, size_t workspace_bytes)
{
    if (n_seqs <= 0) return SMOL_B200_OK;
    if (!model_ok(mp) || !tokens_in || !tokens_out || !k_pool || !v_pool || !layer_row0 || !kv_len || !rope_cos ||
        !rope_sin || max_kv_len < 0)
        return SMOL_B200_ERR_ARGS;
    const smol_b200_qkn_model &m = *mp;
    const StepWs w = carve(m, n_seqs, max_kv_len, static_cast<uint8_t *>(workspace));
    if (!workspace || workspace_bytes < w.total) return SMOL_B200_ERR_WORKSPACE;
    unsigned *err = device_error_word();
    if (!err) return SMOL_B200_ERR_CUDA;
    const int H = m.hidden, qd = m.n_heads * m.head_dim, kvd = m.n_kv_heads * m.head_dim;
    const float scale = 1.0f / sqrtf(static_cast<float>(m.head_dim));   // qkn_decoder.c:620

    // Every kernel of the step launches with programmatic dependent launch: it starts
    // while its predecessor runs and streams its (constant) weights before waiting.
    PdlScope pdl;
    const int n_idx = n_seqs * m.n_layers;
    if (launch_kernel(step_index_kernel, dim3((n_idx + 255) / 256), dim3(256), 0, st, w.positions, w.kv_next, w.slots,
                      layer_row0, static_cast<const int *>(kv_len), n_seqs, m.n_layers) != cudaSuccess ||
        launch_kernel(embed_kernel, dim3(n_seqs), dim3(256), 0, st, w.x, tokens_in, m.tok_embeddings, H, m.vocab,
                      err) != cudaSuccess)
        return SMOL_B200_ERR_CUDA;

    int rc = SMOL_B200_OK;
    for (int l = 0; l < m.n_layers && rc == SMOL_B200_OK; ++l) {
        const smol_b200_qkn_layer &L = m.layers[l];
        {   // input RMSNorm + Q, K, V in one launch (smol_linear_nobias_bf16_qkv, matmul.c:308-334)
            GemvParams p;
            memset(&p, 0, sizeof(p));
            p.seg[0] = {L.wq, w.q, qd, qd};
            p.seg[1] = {L.wk, w.k, kvd, kvd};
            p.seg[2] = {L.wv, w.v, kvd, kvd};
            p.nseg = 3;
            p.total_rows = qd + 2 * kvd;
            p.x = w.x;
            p.ldx = H;
            p.norm_w = L.input_norm;
            p.eps = m.eps;
            p.k_dim = H;
            p.mode = 0;
            rc = run_gemv(st, p, n_seqs);
        }
        if (rc != SMOL_B200_OK) break;
        rc = qknorm_rope_append(st, w.q, w.k, w.v, n_seqs, m.n_heads, m.n_kv_heads, m.head_dim, L.q_norm, L.k_norm,
                                m.eps, rope_cos, rope_sin, m.rope_interleaved, w.positions,
                                w.slots + static_cast<size_t>(l) * n_seqs, w.qr, nullptr, k_pool, v_pool, pool_rows);
        if (rc != SMOL_B200_OK) break;
        rc = decode_attention(st, w.attn, w.qr, 0, k_pool, v_pool, pool_rows,
                              layer_row0 + static_cast<size_t>(l) * n_seqs, w.kv_next, n_seqs, max_kv_len + 1,
                              m.n_heads, m.n_kv_heads, m.head_dim, scale, 0, 0.f, w.attn_ws, w.attn_ws_bytes);
        if (rc != SMOL_B200_OK) break;
        rc = gemv_norm_bf16(st, w.x, H, w.attn, qd, L.wo, H, qd, n_seqs, 1, nullptr, 0.f);   // x += o_proj(attn)
        if (rc != SMOL_B200_OK) break;
        // post-attention RMSNorm + gate/up + SiLU gate
        rc = gemv_norm_bf16(st, w.act, m.intermediate, w.x, H, L.gate_up, m.intermediate, H, n_seqs, 2,
                            L.post_attn_norm, m.eps);
        if (rc != SMOL_B200_OK) break;
        rc = gemv_norm_bf16(st, w.x, H, w.act, m.intermediate, L.down, H, m.intermediate, n_seqs, 1, nullptr,
                            0.f);   // x += down(act)
    }
    if (rc != SMOL_B200_OK) return rc;
    // final RMSNorm (qkn_decoder.c:710) folded into the argmax; the normalised state lands in xn
    rc = run_argmax(st, tokens_out, w.x, H, m.tok_embeddings, m.vocab, H, n_seqs, w.argmax_ws, w.argmax_ws_bytes,
                    m.final_norm, m.eps, w.xn);
    if (rc != SMOL_B200_OK) return rc;
    if (advance && launch_kernel(advance_kernel, dim3((n_seqs + 255) / 256), dim3(256), 0, st, kv_len, n_seqs) !=
                       cudaSuccess)
        return SMOL_B200_ERR_CUDA;
    return SMOL_B200_OK;
}

}  // namespace smolb200
