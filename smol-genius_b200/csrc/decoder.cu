// decoder.cu -- the rest of a decode step around attention, on the device.
//
// Replaces what qkn_decoder_forward (qkn_decoder.c:570-714) runs on the host between
// the attention calls: bf16 matrix-vector products (bf16_matvec_fused,
// bf16_matvec_avx.c:24-150: fp32 activations times bf16 weights widened to fp32,
// fp32 accumulation), the SwiGLU / GeGLU gates (activation.c:55-126), residual adds
// (matmul.c:33-35), RMSNorm (rmsnorm.c:17-70), Gemma's embedding scale and
// sublayer-output norms (qkn_decoder.c:596-599, :681-702) and the greedy argmax over
// the tied embedding matrix (matmul.c:392-417, bf16_matvec_avx.c:156-250).
//
// The products are HBM-bound for a batch of a few sequences: every weight is read
// once per step and reused for all (<= 8) sequences of a launch.  One warp owns one
// output row (two for the gated form); its lanes stream the row in 16-byte pieces
// (8 bf16 weights), several pieces in flight per lane, while the activations of the
// launch's sequences sit in shared memory.  Algorithmic bytes per launch: rows *
// k_dim * 2 (weights) + n_seqs * (k_dim + rows) * 4 (activations).
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include "b200_common.cuh"
#include "runtime.h"

namespace smolb200 {
namespace {

constexpr int kGemvWarps = 8;
constexpr int kGemvThreads = kGemvWarps * 32;
constexpr int kMaxBatch = 8;   // sequences per launch (larger batches loop)
// Shared memory for the staged activations of one launch: launches carry up to
// kMaxBatch sequences, fewer when k_dim is large (8 x 6400 fp32 fill it; a 16384-wide
// down projection takes 3 sequences per launch).
constexpr int kMaxXsBytes = 200 * 1024;
// Warps per SM the K split aims for (SMOL_GEMV_WARPS_PER_SM, measurement knob).
const int g_gemv_warps_per_sm = [] {
    const char *e = getenv("SMOL_GEMV_WARPS_PER_SM");
    const int v = e ? atoi(e) : 0;
    return v > 0 ? v : 8;
}();
// Cap on the CTAs of one projection per SM (SMOL_GEMV_CTAS_PER_SM, measurement knob):
// fewer resident CTAs leave room for the next kernel of the step to start early.
const int g_gemv_ctas_per_sm = [] {
    const char *e = getenv("SMOL_GEMV_CTAS_PER_SM");
    const int v = e ? atoi(e) : 0;
    return v > 0 ? v : 16;
}();

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
    float *x_normed;       // non-null: CTA 0 also writes the staged (normalised) x here
    int k_dim;
    int nb;       // sequences in this launch (<= NB)
    int mode;     // 0 store, 1 add, 2 SiLU-gated pairs, 3 GELU-tanh-gated pairs
    int ksplit;   // warps of a CTA that share one row group, each a slice of K (1, 2, 4, 8)
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

// The gate of a gated pair: SiLU g/(1+exp(-g)) (mode 2, activation.c:81) or GELU with
// the tanh approximation 0.5*g*(1+tanh(sqrt(2/pi)*(g+0.044715*g^3))) (mode 3,
// activation.c:119-123).
__device__ __forceinline__ float gate_act(float g, int mode)
{
    if (mode == 3) {
        const float x3 = g * g * g;
        const float inner = 0.7978845608028654f * (g + 0.044715f * x3);
        return 0.5f * g * (1.0f + tanhf(inner));
    }
    return g / (1.0f + expf(-g));
}

// Row `r` of the concatenated segments: its weights and its output column.
struct RowRef {
    const uint16_t *w;
    float *y;
    long long ldy;
    int col;
};

__device__ __forceinline__ RowRef row_ref(const GemvParams &p, int r, int k_dim)
{
    int s = 0;
    while (s + 1 < p.nseg && r >= p.seg[s].rows) {
        r -= p.seg[s].rows;
        ++s;
    }
    return {p.seg[s].w + static_cast<size_t>(r) * k_dim, p.seg[s].y, p.seg[s].ldy, r};
}

// A warp owns R consecutive weight rows (R even for the gated form: gate, up pairs),
// so each 16-byte piece of the staged activations read from shared memory serves R
// rows: with 8 sequences and R = 4 the shared-memory traffic is 4x the weight
// traffic instead of 16x.  With ksplit = S the CTA's 8 warps form 8/S row groups of S
// warps, each warp streaming every S-th 256-element piece of K, and the S partial
// sums meet in shared memory -- so a projection with few rows still spreads over
// enough warps to keep HBM busy.
// XReg (one sequence, at most kXPieces 256-element pieces of K per lane, and the norm
// only where one warp covers all of K): the activations never go through shared memory
// -- each lane loads the pieces it multiplies straight into registers after the wait,
// the warp's lanes together hold all of x for the RMSNorm, and no CTA barrier is needed.
constexpr int kXPieces = 4;

template <int NB, int R, bool Pre, bool XReg = false>
__global__ void __launch_bounds__(kGemvThreads) gemv_bf16_kernel(const __grid_constant__ GemvParams p)
{
    static_assert(!XReg || NB == 1, "register activations: one sequence");
    extern __shared__ float xs[];   // [nb][k_dim]
    __shared__ float part[kGemvWarps][R][NB];
    const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
    const int k_dim = p.k_dim;
    const int S = p.ksplit, G = kGemvWarps / S;
    const int slice = warp % S, grp = warp / S;
    const int n_groups = (p.total_rows + R - 1) / R;
    const int k_first = (slice * 32 + lane) * 8, k_step = S * 256;
    // Small products at small batches (Pre, R <= 2): the first kPre weight pieces of this
    // warp's first rows are loaded into registers before the wait -- most warps own one
    // row group, so its weights are in flight while the previous kernel finishes, and the
    // product after the wait waits only for the staged activations.  (Large products keep
    // the registers for occupancy: they are bound by HBM, not by the wait.)
    constexpr int kPre = !Pre ? 0 : XReg ? kXPieces : R == 1 ? 8 : R == 2 ? 6 : 0;
    uint4 pre[R][kPre > 0 ? kPre : 1];
    {   // this warp's first rows stream from HBM while the previous kernel finishes
        const int rg = blockIdx.x * G + grp;
        if (rg < n_groups) {
#pragma unroll
            for (int i = 0; i < R; ++i) {
                if (rg * R + i >= p.total_rows) break;
                const uint16_t *wrow = row_ref(p, rg * R + i, k_dim).w;
#pragma unroll
                for (int n = 0; n < kPre; ++n)
                    if (k_first + n * k_step < k_dim) pre[i][n] = ldg_stream(wrow + k_first + n * k_step);
                // the rest of the row (past the preloaded pieces) on its way to L2: this warp
                // reads the 512-byte pieces slice, slice+S, ... of the row: lane l takes
                // 128-byte line l%4 of piece slice + (l/4)*S, 8 pieces per pass
                const char *row = reinterpret_cast<const char *>(wrow);
                for (int off = (slice + (lane / 4) * S) * 512 + (lane % 4) * 128 + kPre * S * 512; off < k_dim * 2;
                     off += 8 * S * 512)
                    asm volatile("prefetch.global.L2 [%0];" ::"l"(row + off));
            }
        }
    }
    griddep_wait();
    griddep_trigger();   // one successor may start (and prefetch) while this one works
    float xr[XReg ? kXPieces : 1][8];   // XReg: this lane's pieces of x (k = k_first + n * k_step)
    if constexpr (XReg) {
        float ss = 0.f;
#pragma unroll
        for (int n = 0; n < kXPieces; ++n) {
            const int k = k_first + n * k_step;
            if (k < k_dim) {
                const float4 a = *reinterpret_cast<const float4 *>(p.x + k);
                const float4 c = *reinterpret_cast<const float4 *>(p.x + k + 4);
                xr[n][0] = a.x, xr[n][1] = a.y, xr[n][2] = a.z, xr[n][3] = a.w;
                xr[n][4] = c.x, xr[n][5] = c.y, xr[n][6] = c.z, xr[n][7] = c.w;
#pragma unroll
                for (int j = 0; j < 8; ++j) ss += xr[n][j] * xr[n][j];
            } else {
#pragma unroll
                for (int j = 0; j < 8; ++j) xr[n][j] = 0.f;
            }
        }
        if (p.norm_w) {   // smol_rms_norm's (x * w) * 1/sqrtf(mean(x^2) + eps); one warp holds all of x
            const float r = 1.0f / sqrtf(warp_sum(ss) / static_cast<float>(k_dim) + p.eps);
#pragma unroll
            for (int n = 0; n < kXPieces; ++n) {
                const int k = k_first + n * k_step;
                if (k < k_dim) {
                    const float4 a = __ldg(reinterpret_cast<const float4 *>(p.norm_w + k));
                    const float4 c = __ldg(reinterpret_cast<const float4 *>(p.norm_w + k + 4));
                    const float wn[8] = {a.x, a.y, a.z, a.w, c.x, c.y, c.z, c.w};
#pragma unroll
                    for (int j = 0; j < 8; ++j) xr[n][j] = xr[n][j] * wn[j] * r;
                }
            }
        }
        if (p.x_normed && blockIdx.x == 0 && warp == 0) {
#pragma unroll
            for (int n = 0; n < kXPieces; ++n) {
                const int k = k_first + n * k_step;
                if (k < k_dim)
#pragma unroll
                    for (int j = 0; j < 8; ++j) p.x_normed[k + j] = xr[n][j];
            }
        }
    } else {
        stage_x<NB>(xs, p.x, p.ldx, k_dim, p.nb, p.norm_w, p.eps);
        if (p.x_normed && blockIdx.x == 0)
            for (int i = threadIdx.x; i < p.nb * k_dim; i += blockDim.x)
                p.x_normed[(i / k_dim) * p.ldx + i % k_dim] = xs[i];
    }
    // every warp runs the same number of rounds (the CTA meets at the partial-sum barriers)
    for (int base = blockIdx.x * G; base < n_groups; base += gridDim.x * G) {
        const int rg = base + grp;
        const int r0 = rg * R;
        RowRef rr[R];
        bool valid[R];
#pragma unroll
        for (int i = 0; i < R; ++i) {
            valid[i] = rg < n_groups && r0 + i < p.total_rows;
            rr[i] = row_ref(p, valid[i] ? r0 + i : 0, k_dim);
        }
        float acc[R][NB];
#pragma unroll
        for (int i = 0; i < R; ++i)
#pragma unroll
            for (int b = 0; b < NB; ++b) acc[i][b] = 0.f;
        // acc[i][b] += dot(8 weights of row i at k, x[b][k..k+8))
        auto consume = [&](int k, const uint4 (&wv)[R]) {
            float wf[R][8];
#pragma unroll
            for (int i = 0; i < R; ++i) {
                const uint4 w = wv[i];
                const uint32_t u[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    wf[i][2 * j] = bf16lo_f32(u[j]);
                    wf[i][2 * j + 1] = bf16hi_f32(u[j]);
                }
            }
#pragma unroll
            for (int b = 0; b < NB; ++b) {
                if (b < p.nb) {
                    const float4 xa = *reinterpret_cast<const float4 *>(xs + b * k_dim + k);
                    const float4 xb = *reinterpret_cast<const float4 *>(xs + b * k_dim + k + 4);
                    const float xv[8] = {xa.x, xa.y, xa.z, xa.w, xb.x, xb.y, xb.z, xb.w};
#pragma unroll
                    for (int i = 0; i < R; ++i) {
                        float a = acc[i][b];
#pragma unroll
                        for (int j = 0; j < 8; ++j) a = fmaf(wf[i][j], xv[j], a);
                        acc[i][b] = a;
                    }
                }
            }
        };
        if constexpr (XReg) {   // x in registers: piece n of every row against xr[n]
            const bool first = base == blockIdx.x * G;
#pragma unroll
            for (int n = 0; n < kXPieces; ++n) {
                const int k = k_first + n * k_step;
                if (k >= k_dim) break;
#pragma unroll
                for (int i = 0; i < R; ++i) {
                    const uint4 w = !valid[i]               ? make_uint4(0, 0, 0, 0)
                                    : (first && n < kPre) ? pre[i][n < kPre ? n : 0]
                                                          : ldg_stream(rr[i].w + k);
                    const uint32_t u[4] = {w.x, w.y, w.z, w.w};
                    float a = acc[i][0];
#pragma unroll
                    for (int j = 0; j < 4; ++j) {
                        a = fmaf(bf16lo_f32(u[j]), xr[n][2 * j], a);
                        a = fmaf(bf16hi_f32(u[j]), xr[n][2 * j + 1], a);
                    }
                    acc[i][0] = a;
                }
            }
        }
        int k = XReg ? k_dim : k_first;
        if (!XReg && kPre > 0 && base == blockIdx.x * G) {   // the first row group: its preloaded pieces
#pragma unroll
            for (int n = 0; n < kPre; ++n, k += k_step) {
                if (k >= k_dim) break;
                uint4 wv[R];
#pragma unroll
                for (int i = 0; i < R; ++i) wv[i] = valid[i] ? pre[i][n] : make_uint4(0, 0, 0, 0);
                consume(k, wv);
            }
        }
#pragma unroll 2
        for (; k < k_dim; k += k_step) {
            uint4 wv[R];
#pragma unroll
            for (int i = 0; i < R; ++i) wv[i] = valid[i] ? ldg_stream(rr[i].w + k) : make_uint4(0, 0, 0, 0);
            consume(k, wv);
        }
        if (S == 1) {   // the warp holds whole rows: write from lane 0, no CTA barrier
#pragma unroll
            for (int b = 0; b < NB; ++b) {
                if (b >= p.nb) continue;
                float sums[R];
#pragma unroll
                for (int i = 0; i < R; ++i) sums[i] = warp_sum(acc[i][b]);
                if (lane == 0) {
#pragma unroll
                    for (int i = 0; i < R; ++i) {
                        if (!valid[i]) continue;
                        float *y = rr[i].y + b * rr[i].ldy;
                        if (p.mode == 0) {
                            y[rr[i].col] = sums[i];
                        } else if (p.mode == 1) {
                            y[rr[i].col] = y[rr[i].col] + sums[i];
                        } else if ((i & 1) == 0) {
                            y[rr[i].col / 2] = gate_act(sums[i], p.mode) * sums[i + 1];
                        }
                    }
                }
            }
            continue;
        }
#pragma unroll
        for (int i = 0; i < R; ++i)
#pragma unroll
            for (int b = 0; b < NB; ++b) {
                const float v = warp_sum(acc[i][b]);
                if (lane == 0) part[warp][i][b] = v;
            }
        __syncthreads();
        if (slice == 0 && lane < R * NB) {
            const int i = lane / NB, b = lane % NB;
            if (valid[i] && b < p.nb) {
                float v = 0.f;
                for (int sl = 0; sl < S; ++sl) v += part[grp * S + sl][i][b];
                const RowRef r = row_ref(p, r0 + i, k_dim);
                float *y = r.y + b * r.ldy;
                if (p.mode == 0) {
                    y[r.col] = v;
                } else if (p.mode == 1) {
                    y[r.col] = y[r.col] + v;
                } else if ((i & 1) == 0) {   // gate row i, up row i+1 (pairs never straddle a warp)
                    float u = 0.f;
                    for (int sl = 0; sl < S; ++sl) u += part[grp * S + sl][i + 1][b];
                    y[r.col / 2] = gate_act(v, p.mode) * u;
                }
            }
        }
        __syncthreads();
    }
}

// Greedy argmax over the logits of each sequence: the largest value, the lowest index
// among equal ones -- the reference's strict '>' scan from row 0 with best = -1e30
// (bf16_matvec_avx.c:156-250, matmul.c:392-417).  Stage 1: kArgmaxParts CTAs per
// sequence each reduce a contiguous part; stage 2: one warp per sequence.
constexpr int kArgmaxParts = 64;

__device__ __forceinline__ void better(float &bv, int &bi, float v, int i)
{
    if (v > bv || (v == bv && i < bi)) {
        bv = v;
        bi = i;
    }
}

__device__ __forceinline__ void warp_best(float &bv, int &bi)
{
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const float v = __shfl_xor_sync(0xffffffffu, bv, o);
        const int i = __shfl_xor_sync(0xffffffffu, bi, o);
        better(bv, bi, v, i);
    }
}

__global__ void __launch_bounds__(256) argmax_part_kernel(float *part_val, int *part_idx, const float *logits,
                                                          long long ld, int vocab)
{
    griddep_wait();
    griddep_trigger();
    const int b = blockIdx.y, part = blockIdx.x;
    const int per = (vocab + kArgmaxParts - 1) / kArgmaxParts;
    const int lo = part * per, hi = min(vocab, lo + per);
    const float *lg = logits + b * ld;
    float bv = -1e30f;
    int bi = lo < vocab ? lo : 0;
    for (int i = lo + threadIdx.x; i < hi; i += blockDim.x) better(bv, bi, lg[i], i);
    warp_best(bv, bi);
    __shared__ float sv[8];
    __shared__ int si[8];
    if (threadIdx.x % 32 == 0) {
        sv[threadIdx.x / 32] = bv;
        si[threadIdx.x / 32] = bi;
    }
    __syncthreads();
    if (threadIdx.x < 32) {
        bv = threadIdx.x < 8 ? sv[threadIdx.x] : -1e30f;
        bi = threadIdx.x < 8 ? si[threadIdx.x] : si[0];
        warp_best(bv, bi);
        if (threadIdx.x == 0) {
            part_val[b * kArgmaxParts + part] = bv;
            part_idx[b * kArgmaxParts + part] = bi;
        }
    }
}

__global__ void argmax_final_kernel(int *tokens_out, const float *part_val, const int *part_idx)
{
    griddep_wait();
    griddep_trigger();
    const int b = blockIdx.x;
    float bv = -1e30f;
    int bi = 0;
    for (int i = threadIdx.x; i < kArgmaxParts; i += 32)
        better(bv, bi, part_val[b * kArgmaxParts + i], part_idx[b * kArgmaxParts + i]);
    warp_best(bv, bi);
    if (threadIdx.x == 0) tokens_out[b] = bi;
}

// x[b][:] = E[tokens[b]][:] (bf16 -> fp32) -- or x_in[b][:] when the caller passes its
// own embeddings -- times `scale` when it is positive (Gemma's embed_normalizer,
// qkn_decoder.c:596-599)
__global__ void embed_kernel(float *x, const int *tokens, const uint16_t *emb, int hidden, int vocab, float scale,
                             unsigned *err, const float *x_in)
{
    griddep_wait();
    griddep_trigger();
    const int b = blockIdx.x;
    if (x_in) {   // the caller's embeddings (qkn_decoder_forward's input_embed), scaled the same way
        for (int i = threadIdx.x; i < hidden; i += blockDim.x) {
            float v = x_in[static_cast<size_t>(b) * hidden + i];
            if (scale > 0.f) v *= scale;
            x[static_cast<size_t>(b) * hidden + i] = v;
        }
        return;
    }
    int t = tokens[b];
    if (t < 0 || t >= vocab) {
        if (threadIdx.x == 0) atomicOr(err, kErrBadArgs);
        t = 0;
    }
    const uint16_t *e = emb + static_cast<size_t>(t) * hidden;
    for (int i = threadIdx.x; i < hidden; i += blockDim.x) {
        float v = __uint_as_float(static_cast<uint32_t>(e[i]) << 16);
        if (scale > 0.f) v *= scale;
        x[static_cast<size_t>(b) * hidden + i] = v;
    }
}

// x[b][:] += rmsnorm(y[b][:]) with weights w: smol_rms_norm of a sublayer's output
// followed by smol_add_inplace (qkn_decoder.c:683-684, :701-704; rmsnorm.c:17-70:
// (y * w) * 1/sqrtf(mean(y^2) + eps)).  One CTA of kNormAddThreads per sequence.
constexpr int kNormAddThreads = 256;

__global__ void __launch_bounds__(kNormAddThreads) norm_add_kernel(float *x, const float *y, const float *w,
                                                                  int hidden, float eps)
{
    griddep_wait();
    griddep_trigger();
    const size_t row = static_cast<size_t>(blockIdx.x) * hidden;
    float ss = 0.f;
    for (int i = threadIdx.x; i < hidden; i += kNormAddThreads) ss += y[row + i] * y[row + i];
    ss = warp_sum(ss);
    __shared__ float part[kNormAddThreads / 32];
    __shared__ float rinv;
    if (threadIdx.x % 32 == 0) part[threadIdx.x / 32] = ss;
    __syncthreads();
    if (threadIdx.x == 0) {
        float t = 0.f;
        for (int i = 0; i < kNormAddThreads / 32; ++i) t += part[i];
        rinv = 1.0f / sqrtf(t / static_cast<float>(hidden) + eps);
    }
    __syncthreads();
    const float r = rinv;
    for (int i = threadIdx.x; i < hidden; i += kNormAddThreads) x[row + i] = x[row + i] + y[row + i] * w[i] * r;
}

// positions[b] = kv_len[b]; kv_next[b] = kv_len[b] + 1; slots[l][b] = row0[l][b] + kv_len[b]
__global__ void step_index_kernel(int *positions, int *kv_next, int64_t *slots, const int64_t *layer_row0,
                                  const int *kv_len, int n_seqs, int n_layers)
{
    griddep_wait();
    griddep_trigger();
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

// Prefill: out[t][:] = bf16(smol_rms_norm(x[t][:])) -- (x * w) * 1/sqrtf(mean(x^2) + eps)
// (rmsnorm.c:17-70), one warp per row, as the operand of the next GEMM.
constexpr int kRowNormWarps = 8;

// out = bf16(rmsnorm(x) * w); with out_lo also the residual bf16(y - out), so that a
// GEMM over out and then out_lo (added) sees y to ~2^-17 relative instead of 2^-9.
__global__ void __launch_bounds__(kRowNormWarps * 32) rms_norm_rows_bf16_kernel(uint16_t *out, uint16_t *out_lo,
                                                                                const float *x, const float *w,
                                                                                int rows, int hidden, float eps)
{
    const int row = blockIdx.x * kRowNormWarps + threadIdx.x / 32, lane = threadIdx.x % 32;
    if (row >= rows) return;
    const float *xr = x + static_cast<long long>(row) * hidden;
    float ss = 0.f;
    for (int i = lane; i < hidden; i += 32) ss += xr[i] * xr[i];
    const float r = 1.0f / sqrtf(warp_sum(ss) / static_cast<float>(hidden) + eps);
    uint16_t *o = out + static_cast<long long>(row) * hidden;
    uint16_t *ol = out_lo ? out_lo + static_cast<long long>(row) * hidden : nullptr;
    for (int i = lane; i < hidden; i += 32) {
        const float y = xr[i] * w[i] * r;
        __nv_bfloat16 b = __float2bfloat16_rn(y);
        o[i] = *reinterpret_cast<uint16_t *>(&b);
        if (ol) {
            __nv_bfloat16 bl = __float2bfloat16_rn(y - __bfloat162float(b));
            ol[i] = *reinterpret_cast<uint16_t *>(&bl);
        }
    }
}

// Prefill positions and pool rows of one layer: positions[t] = start + t,
// slots[t] = row0 + start + t.
__global__ void prefill_index_kernel(int *positions, int64_t *slots, int64_t row0, int start, int n)
{
    const int t = blockIdx.x * blockDim.x + threadIdx.x;
    if (t >= n) return;
    if (positions) positions[t] = start + t;
    slots[t] = row0 + start + t;
}

__global__ void advance_kernel(int *kv_len, int n_seqs)
{
    griddep_wait();
    griddep_trigger();
    const int b = blockIdx.x * blockDim.x + threadIdx.x;
    if (b < n_seqs) kv_len[b] += 1;
}

int gemv_smem_bytes(int nb, int k_dim)
{
    return nb * k_dim * static_cast<int>(sizeof(float));
}

// SMOL_GEMV_XREG=0 in the environment stages the activations in shared memory for every
// product (measurement knob).
const bool g_gemv_xreg = [] {
    const char *e = getenv("SMOL_GEMV_XREG");
    return !(e && e[0] == '0');
}();

// Products of at most this many weight bytes take the register preload (latency-bound
// at small batches); larger ones keep the registers for occupancy.
constexpr long long kGemvPreMaxBytes = 32ll << 20;

template <int NB, int R, bool Pre>
int launch_gemv_pre(cudaStream_t st, const GemvParams &p, long long grid, int smem)
{
    if constexpr (NB == 1 && Pre) {
        // one sequence, a small product whose K fits kXPieces pieces per lane, with the
        // norm only where a warp covers all of K: activations in registers
        const int pieces = (p.k_dim + p.ksplit * 256 - 1) / (p.ksplit * 256);
        if (g_gemv_xreg && pieces <= kXPieces && (p.ksplit == 1 || !p.norm_w))
            return launch_kernel(gemv_bf16_kernel<NB, R, Pre, true>, dim3(static_cast<unsigned>(grid)),
                                 dim3(kGemvThreads), 0, st, p) == cudaSuccess
                       ? SMOL_B200_OK
                       : SMOL_B200_ERR_CUDA;
    }
    if (smem > 48 * 1024) {
        static bool raised[64] = {};
        const int dev = current_device();
        if (dev < 0 || dev >= 64) return SMOL_B200_ERR_CUDA;
        if (!raised[dev]) {
            // dynamic + static (the norm partials) must stay within the 227 KB per block
            if (cudaFuncSetAttribute(gemv_bf16_kernel<NB, R, Pre>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     kMaxXsBytes) != cudaSuccess)
                return SMOL_B200_ERR_CUDA;
            raised[dev] = true;
        }
    }
    return launch_kernel(gemv_bf16_kernel<NB, R, Pre>, dim3(static_cast<unsigned>(grid)), dim3(kGemvThreads), smem,
                         st, p) == cudaSuccess
               ? SMOL_B200_OK
               : SMOL_B200_ERR_CUDA;
}

template <int NB, int R>
int launch_gemv_nb(cudaStream_t st, GemvParams &p)
{
    const int smem = gemv_smem_bytes(p.nb, p.k_dim);
    // K slices per row group: enough warps in flight for HBM (~16 per SM), while each
    // slice keeps at least one 256-element piece per lane.
    const long long groups = (p.total_rows + R - 1) / R;
    const long long want_warps = 148LL * g_gemv_warps_per_sm;
    int S = 1;
    while (S < kGemvWarps && groups * S < want_warps && p.k_dim >= 256 * 2 * S) S *= 2;
    p.ksplit = S;
    const int G = kGemvWarps / S;
    long long grid = (groups + G - 1) / G;
    if (grid > 148LL * g_gemv_ctas_per_sm) grid = 148LL * g_gemv_ctas_per_sm;
    if (static_cast<long long>(p.total_rows) * p.k_dim * 2 <= kGemvPreMaxBytes)
        return launch_gemv_pre<NB, R, true>(st, p, grid, smem);
    return launch_gemv_pre<NB, R, false>(st, p, grid, smem);
}

// Rows per warp: 1 for a single sequence (most warps in flight), 2 for two, 4 from four
// sequences on; the gated forms need an even count (gate, up).
template <int NB>
int launch_gemv_rows(cudaStream_t st, GemvParams &p)
{
    if (NB >= 4) return launch_gemv_nb<NB, 4>(st, p);
    if (NB == 2 || p.mode >= 2) return launch_gemv_nb<NB, 2>(st, p);
    return launch_gemv_nb<NB, 1>(st, p);
}

// Runs the segmented product for every sequence, kMaxBatch sequences per launch.
int run_gemv(cudaStream_t st, GemvParams p, int n_seqs)
{
    if (p.k_dim <= 0 || p.k_dim % 8 || (p.ldx & 3) || p.total_rows <= 0) return SMOL_B200_ERR_ARGS;
    const int per_launch = kMaxXsBytes / gemv_smem_bytes(1, p.k_dim) < kMaxBatch
                               ? kMaxXsBytes / gemv_smem_bytes(1, p.k_dim)
                               : kMaxBatch;
    if (per_launch < 1) return SMOL_B200_ERR_ARGS;   // k_dim > 51200
    for (int s = 0; s < p.nseg; ++s)
        if (!p.seg[s].w || !p.seg[s].y || (reinterpret_cast<uintptr_t>(p.seg[s].w) & 15) ||
            (p.mode >= 2 && (p.seg[s].rows & 1)))
            return SMOL_B200_ERR_ARGS;
    if (!p.x || (reinterpret_cast<uintptr_t>(p.x) & 15)) return SMOL_B200_ERR_ARGS;
    for (int b0 = 0; b0 < n_seqs; b0 += per_launch) {
        GemvParams q = p;
        q.nb = n_seqs - b0 < per_launch ? n_seqs - b0 : per_launch;
        q.x = p.x + static_cast<long long>(b0) * p.ldx;
        if (p.x_normed) q.x_normed = p.x_normed + static_cast<long long>(b0) * p.ldx;
        for (int s = 0; s < p.nseg; ++s) q.seg[s].y = p.seg[s].y + static_cast<long long>(b0) * p.seg[s].ldy;
        int rc;
        if (q.nb == 1) rc = launch_gemv_rows<1>(st, q);
        else if (q.nb == 2) rc = launch_gemv_rows<2>(st, q);
        else if (q.nb <= 4) rc = launch_gemv_rows<4>(st, q);
        else rc = launch_gemv_rows<8>(st, q);
        if (rc != SMOL_B200_OK) return rc;
    }
    return SMOL_B200_OK;
}

// Logits of every sequence (fp32, [n_seqs][vocab]) between the lm_head product and the
// reduction.
size_t argmax_ws_bytes(int n_seqs, int vocab)
{
    const size_t logits = (static_cast<size_t>(n_seqs) * static_cast<size_t>(vocab) * sizeof(float) + 255) / 256 * 256;
    return logits + static_cast<size_t>(n_seqs) * kArgmaxParts * (sizeof(float) + sizeof(int));
}

// tokens_out[b] = argmax_v sum_k norm(x)[b][k] * E[v][k]: the tied lm_head as a GEMV into
// the logits, then the lowest-index maximum.  norm_w (optional) applies the final RMSNorm
// while x is staged; x_normed (optional) receives the normalised rows.
int run_argmax(cudaStream_t st, int *tokens_out, const float *x, long long ldx, const uint16_t *emb, int vocab,
               int k_dim, int n_seqs, void *ws, size_t ws_bytes, const float *norm_w = nullptr, float eps = 0.f,
               float *x_normed = nullptr)
{
    if (n_seqs <= 0) return SMOL_B200_OK;
    if (!tokens_out || !x || !emb || vocab <= 0) return SMOL_B200_ERR_ARGS;
    if (!ws || ws_bytes < argmax_ws_bytes(n_seqs, vocab)) return SMOL_B200_ERR_WORKSPACE;
    float *logits = static_cast<float *>(ws);
    GemvParams p;
    memset(&p, 0, sizeof(p));
    p.seg[0] = {emb, logits, vocab, vocab};
    p.nseg = 1;
    p.total_rows = vocab;
    p.x = x;
    p.ldx = ldx;
    p.norm_w = norm_w;
    p.eps = eps;
    p.x_normed = x_normed;
    p.k_dim = k_dim;
    p.mode = 0;
    int rc = run_gemv(st, p, n_seqs);
    if (rc != SMOL_B200_OK) return rc;
    uint8_t *rest = static_cast<uint8_t *>(ws) +
                    (static_cast<size_t>(n_seqs) * static_cast<size_t>(vocab) * sizeof(float) + 255) / 256 * 256;
    float *pv = reinterpret_cast<float *>(rest);
    int *pi = reinterpret_cast<int *>(pv + static_cast<size_t>(n_seqs) * kArgmaxParts);
    if (launch_kernel(argmax_part_kernel, dim3(kArgmaxParts, n_seqs), dim3(256), 0, st, pv, pi,
                      static_cast<const float *>(logits), static_cast<long long>(vocab), vocab) != cudaSuccess ||
        launch_kernel(argmax_final_kernel, dim3(n_seqs), dim3(32), 0, st, tokens_out,
                      static_cast<const float *>(pv), static_cast<const int *>(pi)) != cudaSuccess)
        return SMOL_B200_ERR_CUDA;
    return SMOL_B200_OK;
}

// Workspace of one decoder step, carved in 256-byte aligned pieces.
struct StepWs {
    float *x, *xn, *q, *k, *v, *qr, *attn, *act, *sub;   // sub: a sublayer's output before its norm
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
    w.argmax_ws_bytes = argmax_ws_bytes(n_seqs, m.vocab);
    w.argmax_ws = take(w.argmax_ws_bytes);
    w.sub = reinterpret_cast<float *>(take(B * m.hidden * 4));
    w.total = off;
    return w;
}

bool model_ok(const smol_b200_qkn_model *m)
{
    return m && m->hidden > 0 && m->n_layers > 0 && m->n_heads > 0 && m->n_kv_heads > 0 && m->head_dim > 0 &&
           m->n_heads % m->n_kv_heads == 0 && m->intermediate > 0 && m->vocab > 0 && m->tok_embeddings &&
           m->final_norm && m->layers && m->hidden % 8 == 0 && m->intermediate % 8 == 0 &&
           (m->n_heads * m->head_dim) % 8 == 0 && (m->activation == 0 || m->activation == 1) &&
           m->sliding_window >= 0 && !m->rope_cos_local == !m->rope_sin_local;
}

}  // namespace

int gemv_norm_bf16(cudaStream_t st, float *y, int64_t ldy, const float *x, int64_t ldx, const uint16_t *w,
                   int n_out, int k_dim, int n_seqs, int mode, const float *norm_w, float eps)
{
    if (n_seqs <= 0 || n_out <= 0) return SMOL_B200_OK;
    if (mode < 0 || mode > 3 || (ldy < n_out)) return SMOL_B200_ERR_ARGS;
    GemvParams p;
    memset(&p, 0, sizeof(p));
    p.seg[0] = {w, y, ldy, mode >= 2 ? 2 * n_out : n_out};
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

size_t argmax_workspace_bytes(int n_seqs, int vocab)
{
    return argmax_ws_bytes(n_seqs, vocab);
}

// Workspace of one prefill of n tokens, carved in 256-byte aligned pieces.
struct PrefillWs {
    float *x, *q, *k, *v, *sub;
    uint16_t *xn, *xn_lo, *qb, *attn16, *act;
    int *positions;
    int64_t *slots;
    size_t total;
};

static PrefillWs carve_prefill(const smol_b200_qkn_model &m, int n, uint8_t *base)
{
    PrefillWs w;
    memset(&w, 0, sizeof(w));
    size_t off = 0;
    auto take = [&](size_t bytes) {
        uint8_t *p = base ? base + off : nullptr;
        off += (bytes + 255) / 256 * 256;
        return p;
    };
    const size_t T = static_cast<size_t>(n), H = m.hidden, I = m.intermediate;
    const size_t qd = static_cast<size_t>(m.n_heads) * m.head_dim, kvd = static_cast<size_t>(m.n_kv_heads) * m.head_dim;
    w.x = reinterpret_cast<float *>(take(T * H * 4));
    w.q = reinterpret_cast<float *>(take(T * qd * 4));
    w.k = reinterpret_cast<float *>(take(T * kvd * 4));
    w.v = reinterpret_cast<float *>(take(T * kvd * 4));
    w.sub = reinterpret_cast<float *>(take(T * H * 4));
    w.xn = reinterpret_cast<uint16_t *>(take(T * H * 2));
    w.xn_lo = reinterpret_cast<uint16_t *>(take(T * H * 2));
    w.qb = reinterpret_cast<uint16_t *>(take(T * qd * 2));
    w.attn16 = reinterpret_cast<uint16_t *>(take(T * qd * 2));
    w.act = reinterpret_cast<uint16_t *>(take(T * I * 2));
    w.positions = reinterpret_cast<int *>(take(T * 4));
    w.slots = reinterpret_cast<int64_t *>(take(T * 8));
    w.total = off;
    return w;
}

size_t qkn_prefill_workspace_bytes(const smol_b200_qkn_model *m, int n_tokens)
{
    if (!model_ok(m) || n_tokens <= 0) return 0;
    return carve_prefill(*m, n_tokens, nullptr).total;
}

int qkn_prefill(cudaStream_t st, const smol_b200_qkn_model *mp, const int *tokens, const float *x_in, int n,
                int start, uint16_t *k_pool, uint16_t *v_pool, int64_t pool_rows, const int64_t *layer_row0,
                const float *rope_cos, const float *rope_sin, void *workspace, size_t workspace_bytes)
{
    if (n <= 0) return SMOL_B200_OK;
    if (!model_ok(mp) || (!tokens == !x_in) || !k_pool || !v_pool || !layer_row0 || !rope_cos || !rope_sin || start < 0)
        return SMOL_B200_ERR_ARGS;
    const smol_b200_qkn_model &m = *mp;
    const int hd = m.head_dim;
    if (hd != 64 && hd != 128 && hd != 256) return SMOL_B200_ERR_ARGS;   // the prefill kernel's head dims
    for (int l = 0; l < m.n_layers; ++l)
        if (layer_row0[l] < 0 || layer_row0[l] + start + n > pool_rows) return SMOL_B200_ERR_ARGS;
    const PrefillWs w = carve_prefill(m, n, static_cast<uint8_t *>(workspace));
    if (!workspace || workspace_bytes < w.total) return SMOL_B200_ERR_WORKSPACE;
    unsigned *err = device_error_word();
    if (!err) return SMOL_B200_ERR_NO_DEVICE;
    const int H = m.hidden, I = m.intermediate, qd = m.n_heads * hd, kvd = m.n_kv_heads * hd;
    const int L_k = start + n;                                          // keys attended by the last token
    const float scale = 1.0f / sqrtf(static_cast<float>(hd));            // qkn_decoder.c:430
    const int gate = m.activation == 1 ? 3 : 2;                         // GeGLU / SwiGLU (:548-551)
    const unsigned rows_grid = static_cast<unsigned>((n + kRowNormWarps - 1) / kRowNormWarps);
    auto rms_bf16 = [&](const float *norm_w, bool with_lo = false) {
        if (!norm_w) return SMOL_B200_ERR_ARGS;
        return launch_kernel(rms_norm_rows_bf16_kernel, dim3(rows_grid), dim3(kRowNormWarps * 32), 0, st, w.xn,
                             with_lo ? w.xn_lo : nullptr, static_cast<const float *>(w.x), norm_w, n, H,
                             m.eps) == cudaSuccess
                   ? SMOL_B200_OK
                   : SMOL_B200_ERR_CUDA;
    };
    auto norm_add = [&](const float *norm_w) {   // x += rmsnorm(sub) (Gemma, :535-537, :555-558)
        if (!norm_w) return SMOL_B200_ERR_ARGS;
        return launch_kernel(norm_add_kernel, dim3(n), dim3(kNormAddThreads), 0, st, w.x,
                             static_cast<const float *>(w.sub), norm_w, H, m.eps) == cudaSuccess
                   ? SMOL_B200_OK
                   : SMOL_B200_ERR_CUDA;
    };
    // embedding rows, scaled by the Gemma normaliser when set (qkn_decoder.c:408-419)
    if (launch_kernel(embed_kernel, dim3(n), dim3(256), 0, st, w.x, tokens, m.tok_embeddings, H, m.vocab,
                      m.embed_normalizer, err, x_in) != cudaSuccess)
        return SMOL_B200_ERR_CUDA;
    int rc = SMOL_B200_OK;
    for (int l = 0; l < m.n_layers && rc == SMOL_B200_OK; ++l) {
        const smol_b200_qkn_layer &L = m.layers[l];
        const bool local_rope = L.is_sliding && m.rope_cos_local;
        const int window = L.is_sliding && m.sliding_window > 0 ? m.sliding_window : 0;
        const float softcap = m.attn_softcap > 0.f ? m.attn_softcap : 0.f;
        const int64_t row0 = layer_row0[l];
        // input RMSNorm, Q / K / V projections (qkn_decoder.c:470-476).  These feed the KV
        // cache, so their input keeps fp32 accuracy as two bf16 operands: W x = W hi + W lo
        // (the second product added into the first's fp32 result).  With sharp attention a
        // bf16-rounded input (2^-9 relative) moves cached keys enough to change a later
        // greedy token that the reference's fp32 projection keeps.
        rc = rms_bf16(L.input_norm, true);
        struct Proj {
            float *out;
            const uint16_t *wt;
            int n_out;
        } const proj[3] = {{w.q, L.wq, qd}, {w.k, L.wk, kvd}, {w.v, L.wv, kvd}};
        for (int j = 0; j < 3 && rc == SMOL_B200_OK; ++j) {
            rc = gemm_bf16(st, proj[j].out, proj[j].n_out, SMOL_B200_GEMM_OUT_F32, w.xn, H, proj[j].wt, H, nullptr,
                           nullptr, 0, 0, n, proj[j].n_out, H, 0);
            if (rc == SMOL_B200_OK)
                rc = gemm_bf16(st, proj[j].out, proj[j].n_out, SMOL_B200_GEMM_OUT_F32_ADD, w.xn_lo, H, proj[j].wt, H,
                               nullptr, nullptr, 0, 0, n, proj[j].n_out, H, 0);
        }
        // QK-norm, RoPE at positions start.., K / V into the pool (qkn_decoder.c:486-503)
        if (rc == SMOL_B200_OK &&
            launch_kernel(prefill_index_kernel, dim3((n + 255) / 256), dim3(256), 0, st, l == 0 ? w.positions : nullptr,
                          w.slots, row0, start, n) != cudaSuccess)
            rc = SMOL_B200_ERR_CUDA;
        if (rc == SMOL_B200_OK)
            rc = qknorm_rope_append(st, w.q, w.k, w.v, n, m.n_heads, m.n_kv_heads, hd, L.q_norm, L.k_norm, m.eps,
                                    local_rope ? m.rope_cos_local : rope_cos, local_rope ? m.rope_sin_local : rope_sin,
                                    m.rope_interleaved, w.positions, w.slots, nullptr, w.qb, k_pool, v_pool,
                                    pool_rows);
        // causal attention over the layer's cached rows [0, start + n) (qkn_decoder.c:505-531)
        if (rc == SMOL_B200_OK) {
            const uint16_t *kl = k_pool + row0 * kvd, *vl = v_pool + row0 * kvd;
            rc = prefill_attention(st, w.attn16, qd, static_cast<int64_t>(n) * qd, w.qb, qd, static_cast<int64_t>(n) * qd,
                                   kl, kvd, static_cast<int64_t>(L_k) * kvd, vl, kvd, static_cast<int64_t>(L_k) * kvd,
                                   1, n, L_k, m.n_heads, m.n_kv_heads, hd, scale, SMOL_MASK_CAUSAL, start, 0, window,
                                   softcap, nullptr, 0, nullptr, 0, 1 /* bf16 output: the o_proj GEMM's operand */);
        }
        // output projection and residual, then the MLP input norm (qkn_decoder.c:530-543)
        if (rc == SMOL_B200_OK) {
            if (L.pre_ffn_norm) {
                rc = gemm_bf16(st, w.sub, H, SMOL_B200_GEMM_OUT_F32, w.attn16, qd, L.wo, qd, nullptr, nullptr, 0, 0, n,
                               H, qd, 0);
                if (rc == SMOL_B200_OK) rc = norm_add(L.post_attn_norm);
                if (rc == SMOL_B200_OK) rc = rms_bf16(L.pre_ffn_norm);
            } else {
                rc = gemm_bf16(st, w.x, H, SMOL_B200_GEMM_OUT_F32_ADD, w.attn16, qd, L.wo, qd, nullptr, nullptr, 0, 0,
                               n, H, qd, 0);
                if (rc == SMOL_B200_OK) rc = rms_bf16(L.post_attn_norm);
            }
        }
        // gate/up with the gated activation, down projection and residual (qkn_decoder.c:546-560)
        if (rc == SMOL_B200_OK)
            rc = gemm_bf16(st, w.act, I, SMOL_B200_GEMM_OUT_BF16, w.xn, H, L.gate_up, H, nullptr, nullptr, 0, 0, n,
                           2 * I, H, 0, gate);
        if (rc == SMOL_B200_OK) {
            if (L.post_ffn_norm) {
                rc = gemm_bf16(st, w.sub, H, SMOL_B200_GEMM_OUT_F32, w.act, I, L.down, I, nullptr, nullptr, 0, 0, n, H,
                               I, 0);
                if (rc == SMOL_B200_OK) rc = norm_add(L.post_ffn_norm);
            } else {
                rc = gemm_bf16(st, w.x, H, SMOL_B200_GEMM_OUT_F32_ADD, w.act, I, L.down, I, nullptr, nullptr, 0, 0, n,
                               H, I, 0);
            }
        }
    }
    return rc;
}

size_t qkn_step_workspace_bytes(const smol_b200_qkn_model *m, int n_seqs, int max_kv_len)
{
    if (!model_ok(m) || n_seqs <= 0 || max_kv_len < 0) return 0;
    return carve(*m, n_seqs, max_kv_len, nullptr).total;
}

int qkn_decode_step(cudaStream_t st, const smol_b200_qkn_model *mp, int n_seqs, const int *tokens_in,
                    const float *x_in, int *tokens_out, uint16_t *k_pool, uint16_t *v_pool, int64_t pool_rows,
                    const int64_t *layer_row0, int *kv_len, int max_kv_len, const float *rope_cos,
                    const float *rope_sin, int advance, void *workspace, size_t workspace_bytes,
                    float *x_normed_out)
{
    if (n_seqs <= 0) return SMOL_B200_OK;
    if (!model_ok(mp) || (!tokens_in == !x_in) || !tokens_out || !k_pool || !v_pool || !layer_row0 || !kv_len || !rope_cos ||
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
                      m.embed_normalizer, err, x_in) != cudaSuccess)
        return SMOL_B200_ERR_CUDA;

    const int gate_mode = m.activation == 1 ? 3 : 2;   // GeGLU / SwiGLU (qkn_decoder.c:695-698)
    // x[b] += rmsnorm(sub[b]) (Gemma's sublayer-output norm before the residual add)
    auto norm_add = [&](const float *w_norm) {
        if (!w_norm) return SMOL_B200_ERR_ARGS;
        return launch_kernel(norm_add_kernel, dim3(n_seqs), dim3(kNormAddThreads), 0, st, w.x,
                             static_cast<const float *>(w.sub), w_norm, H, m.eps) == cudaSuccess
                   ? SMOL_B200_OK
                   : SMOL_B200_ERR_CUDA;
    };
    int rc = SMOL_B200_OK;
    for (int l = 0; l < m.n_layers && rc == SMOL_B200_OK; ++l) {
        const smol_b200_qkn_layer &L = m.layers[l];
        // sliding layers: their own RoPE tables when given, the window when set
        // (qkn_decoder.c:626-632, :659-667)
        const bool local_rope = L.is_sliding && m.rope_cos_local;
        const int window = L.is_sliding && m.sliding_window > 0 ? m.sliding_window : 0;
        const float softcap = m.attn_softcap > 0.f ? m.attn_softcap : 0.f;
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
                                m.eps, local_rope ? m.rope_cos_local : rope_cos,
                                local_rope ? m.rope_sin_local : rope_sin, m.rope_interleaved, w.positions,
                                w.slots + static_cast<size_t>(l) * n_seqs, w.qr, nullptr, k_pool, v_pool, pool_rows);
        if (rc != SMOL_B200_OK) break;
        rc = decode_attention(st, w.attn, w.qr, 0, k_pool, v_pool, pool_rows,
                              layer_row0 + static_cast<size_t>(l) * n_seqs, w.kv_next, n_seqs, max_kv_len + 1,
                              m.n_heads, m.n_kv_heads, m.head_dim, scale, window, softcap, w.attn_ws,
                              w.attn_ws_bytes);
        if (rc != SMOL_B200_OK) break;
        if (L.pre_ffn_norm) {
            // Gemma (qkn_decoder.c:681-685): x += rmsnorm(o_proj(attn)); the MLP input is
            // rmsnorm(x) with pre_ffn_norm
            rc = gemv_norm_bf16(st, w.sub, H, w.attn, qd, L.wo, H, qd, n_seqs, 0, nullptr, 0.f);
            if (rc == SMOL_B200_OK) rc = norm_add(L.post_attn_norm);
            if (rc == SMOL_B200_OK)
                rc = gemv_norm_bf16(st, w.act, m.intermediate, w.x, H, L.gate_up, m.intermediate, H, n_seqs,
                                    gate_mode, L.pre_ffn_norm, m.eps);
        } else {
            rc = gemv_norm_bf16(st, w.x, H, w.attn, qd, L.wo, H, qd, n_seqs, 1, nullptr, 0.f);   // x += o_proj(attn)
            // post-attention RMSNorm + gate/up + gate
            if (rc == SMOL_B200_OK)
                rc = gemv_norm_bf16(st, w.act, m.intermediate, w.x, H, L.gate_up, m.intermediate, H, n_seqs,
                                    gate_mode, L.post_attn_norm, m.eps);
        }
        if (rc != SMOL_B200_OK) break;
        if (L.post_ffn_norm) {   // Gemma (qkn_decoder.c:701-704): x += rmsnorm(down(act))
            rc = gemv_norm_bf16(st, w.sub, H, w.act, m.intermediate, L.down, H, m.intermediate, n_seqs, 0, nullptr,
                                0.f);
            if (rc == SMOL_B200_OK) rc = norm_add(L.post_ffn_norm);
        } else {
            rc = gemv_norm_bf16(st, w.x, H, w.act, m.intermediate, L.down, H, m.intermediate, n_seqs, 1, nullptr,
                                0.f);   // x += down(act)
        }
    }
    if (rc != SMOL_B200_OK) return rc;
    // final RMSNorm (qkn_decoder.c:710) folded into the argmax; the normalised state lands in xn
    // the greedy token over the output head: tied embeddings, or SmolVLM's lm_head (decoder.c:473-475)
    rc = run_argmax(st, tokens_out, w.x, H, m.lm_head ? m.lm_head : m.tok_embeddings, m.vocab, H, n_seqs, w.argmax_ws,
                    w.argmax_ws_bytes, m.final_norm, m.eps, w.xn);
    if (rc != SMOL_B200_OK) return rc;
    if (x_normed_out && !cuda_check(cudaMemcpyAsync(x_normed_out, w.xn, static_cast<size_t>(n_seqs) * H * sizeof(float),
                                                    cudaMemcpyDeviceToDevice, st),
                                    "cudaMemcpyAsync(x_normed)"))
        return SMOL_B200_ERR_CUDA;
    if (advance && launch_kernel(advance_kernel, dim3((n_seqs + 255) / 256), dim3(256), 0, st, kv_len, n_seqs) !=
                       cudaSuccess)
        return SMOL_B200_ERR_CUDA;
    return SMOL_B200_OK;
}

}  // namespace smolb200
