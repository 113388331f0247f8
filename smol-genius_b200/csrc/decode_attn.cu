// decode_attn.cu -- split-KV flash-decoding over the pooled bf16-K / fp16-V cache.
//
// Replaces smol_causal_attention(seq_q=1) as qkn_decoder_forward calls it
// (qkn_decoder.c:658-677; algorithm attention.c:79-126) for a whole batch of
// sequences at once.
//
// Work split.  One CTA owns (sequence b, KV head, group of <=8 Q heads, chunk of
// `chunk` keys).  A producer warp streams the chunk's K and V rows of that KV head
// into shared memory with 2-D TMA tensor copies (64 keys x 64 dims per box,
// 128-byte swizzle) through a STAGES-deep mbarrier ring.  Four consumer warps each
// take 16 keys of every 64-key tile and keep their own online-softmax state.
//
// Math.  The KV head's keys are the M dimension of warp-level MMAs and the (padded
// to 8) Q heads the N dimension, so one K/V tile in shared memory serves every Q
// head of the GQA group (the reference re-reads each KV row once per Q head):
//   S^T(16 keys x 8 heads)   = K(16 x hd, bf16) . Q^T(hd x 8, bf16; fp32 Q is split
//                              into bf16 hi + lo terms so scores keep fp32 accuracy)
//   O^T(hd x 8 heads)       += V^T(hd x 16, fp16) . P^T(16 x 8, fp16)
// P^T reaches the B-operand layout with one movmatrix transpose per 8 keys.  P and V
// are fp16 because bf16 probabilities alone put the output ~1.3e-3 (rel-L2) away from
// an fp32 reference; fp16 keeps it near 1.5e-4.
//
// Q.  The consumer warps copy the CTA's (<= 8) Q rows into shared memory with
// coalesced 16-byte loads, all issued before the first use, while the producer's
// first TMA is in flight; the MMA fragments are then built from shared memory.  (A
// CTA of a small batch often owns a single tile, so this prologue is on the critical
// path: per-thread fragment loads straight from global memory serialise on it.)
//
// Stages.  The ring depth is a launch parameter (at most kMaxStages): a chunk of one
// or two tiles gets one or two stages, so a head-dim-256 CTA of a short chunk needs
// 73 KB of shared memory instead of 137 KB and two fit on an SM.
//
// Each CTA merges its 4 warps and writes one partial (O unnormalised, running max,
// running sum) per Q head; a second kernel merges the chunks of a sequence.
// Algorithmic traffic: every attended key costs n_kv_heads*hd*2 (K,V) * 2 bytes.
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include <mutex>

#include "b200_common.cuh"
#include "runtime.h"

namespace smolb200 {
namespace {

constexpr int kKeysPerTile = 64;
constexpr int kConsumerWarps = 4;
constexpr int kThreads = (kConsumerWarps + 1) * 32;
constexpr int kSubtileBytes = kKeysPerTile * 128;   // 64 rows x 64 halves (128 B)

template <int HD>
struct DecodeShape {
    static constexpr int kSubtiles = HD / 64;
    static constexpr int kTileBytes = kSubtiles * kSubtileBytes;   // K or V of one tile
    static constexpr int kStageBytes = 2 * kTileBytes;
    static constexpr int kMaxStages = HD == 256 ? 2 : (HD == 128 ? 3 : 4);
    static constexpr int kQRowFloats = HD + 8;                     // padded fp32 Q row
    static constexpr int kQBytes = 8 * kQRowFloats * 4;
    static constexpr int kQVecPerThread = 8 * HD * 4 / 16 / (kConsumerWarps * 32);   // 16-byte loads
    // After the K/V tiles: the 4-warp merge area, then the CTA's partial [8][m, l, O[HD]].
    static constexpr int kRedBytes = kConsumerWarps * 8 * (HD + 2) * 4;
    static constexpr int kCpartOff = kRedBytes;
    static_assert(kRedBytes + 8 * (HD + 2) * 4 <= kStageBytes, "merge areas must fit one stage");
    // Layout: [stages x stage][Q rows][barriers], base aligned to 1024 (SW128 tiles).
    static constexpr size_t smem_bytes(int stages)
    {
        return static_cast<size_t>(stages) * kStageBytes + kQBytes + 256 + 1024;
    }
};

struct DecodeParams {
    CUtensorMap tmap_k;             // bf16 [pool_rows, kv_dim], box 64x64, SW128
    CUtensorMap tmap_v;             // fp16 [pool_rows, kv_dim], box 64x64, SW128
    const void *q;                  // [n_seqs, n_heads*hd] fp32 or bf16
    const int64_t *seq_row0;
    const int *kv_len;
    float *part_o;                  // [n_seqs*n_heads*max_chunks, hd]
    float *part_ml;                 // [n_seqs*n_heads*max_chunks, 2]
    unsigned *err;
    int q_is_bf16;
    int n_heads, n_kv_heads, group, n_qgroups;
    int chunk, max_chunks, window;
    float *out;                     // [n_seqs, n_heads*hd] fp32 (cluster form writes it directly)
    int stages;                     // K/V ring depth, 1..kMaxStages
    int q_vec16;                    // q base 16-byte aligned: Q rows copied with 16-byte loads
    float scale, softcap;
};

__device__ __forceinline__ float fast_exp2(float x)
{
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

// Splits two fp32 values into packed bf16 hi and lo (x ~= hi + lo).
__device__ __forceinline__ void split_bf16x2(float x0, float x1, uint32_t &hi, uint32_t &lo)
{
    hi = pack_bf16x2(x0, x1);
    lo = pack_bf16x2(x0 - bf16lo_f32(hi), x1 - bf16hi_f32(hi));
}

// Cluster form (InCluster): the max_chunks CTAs of one (sequence, KV head, Q-head
// group) form a thread-block cluster along x.  Each leaves its partial in its own
// shared memory; after a cluster barrier every CTA merges a slice of the outputs by
// reading the partials of the others through distributed shared memory and writes
// `out` directly, and a second cluster barrier keeps every CTA resident until the
// others finished reading it.  Every thread of every CTA, idle chunks included,
// passes both barriers.  Used for small batches, whose grid fits one wave and whose
// separate merge launch would otherwise cost as much as the split itself.
template <int HD, bool InCluster>
__global__ void __launch_bounds__(kThreads, 2) decode_split_kernel(const __grid_constant__ DecodeParams p)
{
    using S = DecodeShape<HD>;
    constexpr int KSTEPS = HD / 16;

    griddep_wait();   // q, kv_len and the appended cache rows come from earlier kernels
    griddep_trigger();
    const int b = blockIdx.z;
    const int kvh = blockIdx.y / p.n_qgroups;
    const int qg = blockIdx.y % p.n_qgroups;
    const int c = blockIdx.x;

    const int L = p.kv_len[b];
    const int ks = (p.window > 0 && L > p.window) ? L - p.window : 0;
    int n = L - ks;
    if (n > p.max_chunks * p.chunk) n = p.max_chunks * p.chunk;   // flagged by the merge
    const int key0 = c * p.chunk;                                  // relative to ks
    const bool active = n > 0 && key0 < n;                         // uniform for the CTA
    if (!InCluster && !active) return;
    const int nkeys = active ? min(p.chunk, n - key0) : 0;
    const int ntiles = (nkeys + kKeysPerTile - 1) / kKeysPerTile;
    const int h_first = kvh * p.group + qg * 8;
    const int nh = min(8, p.group - qg * 8);
    const long long row_base = p.seq_row0[b] + ks + key0;

    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    const int stages = p.stages;
    float *qs = reinterpret_cast<float *>(smem + stages * S::kStageBytes);
    uint64_t *full_bar = reinterpret_cast<uint64_t *>(smem + stages * S::kStageBytes + S::kQBytes);
    uint64_t *empty_bar = full_bar + S::kMaxStages;

    const int warp = threadIdx.x / 32;
    const int lane = threadIdx.x % 32;

    if (threadIdx.x == 0) {
        for (int s = 0; s < stages; ++s) {
            mbar_init(smem_u32(&full_bar[s]), 1);
            mbar_init(smem_u32(&empty_bar[s]), kConsumerWarps);
        }
        fence_mbar_init();
    }
    __syncthreads();

    if (warp == kConsumerWarps) {
        // ---------------- producer warp ----------------
        if (lane == 0 && ntiles > 0) {
            tma_prefetch_desc(&p.tmap_k);
            tma_prefetch_desc(&p.tmap_v);
            int issued = 0;
            int s = 0, phase = 0;
            for (int t = 0; t < ntiles; ++t) {
                if (t >= stages && !mbar_wait(smem_u32(&empty_bar[s]), phase ^ 1, p.err, kErrWaitTmaEmpty))
                    break;
                const uint32_t fb = smem_u32(&full_bar[s]);
                mbar_arrive_expect_tx(fb, S::kStageBytes);
                const uint32_t kdst = smem_u32(smem + s * S::kStageBytes);
                const uint32_t vdst = kdst + S::kTileBytes;
                const int y = static_cast<int>(row_base + t * kKeysPerTile);
#pragma unroll
                for (int sub = 0; sub < S::kSubtiles; ++sub) {
                    const int x = kvh * HD + sub * 64;
                    tma_load_2d(kdst + sub * kSubtileBytes, &p.tmap_k, fb, x, y);
                    tma_load_2d(vdst + sub * kSubtileBytes, &p.tmap_v, fb, x, y);
                }
                ++issued;
                if (++s == stages) {
                    s = 0;
                    phase ^= 1;
                }
            }
            // Drain: every issued tile must have landed before the CTA may exit.
            for (int t = max(0, issued - stages); t < issued; ++t) {
                if (!mbar_wait(smem_u32(&full_bar[t % stages]), (t / stages) & 1, p.err, kErrDrain))
                    break;
            }
        }
        if (!InCluster) return;
    } else if (active) {
        // ---------------- consumer warps ----------------
        const int g = lane >> 2;   // key row (S^T) / head column (B operand)
        const int tq = lane & 3;

        // Q rows h_first .. h_first+nh-1 of sequence b (contiguous in global memory) to
        // shared memory as fp32, one padded row per head.
        {
            const int tid = threadIdx.x;   // 0..127
            const size_t esize = p.q_is_bf16 ? 2 : 4;
            const uint8_t *qsrc = static_cast<const uint8_t *>(p.q) +
                                  (static_cast<long long>(b) * p.n_heads + h_first) * HD * esize;
            const int nelem = nh * HD;
            if (p.q_vec16) {
                const int nvec = static_cast<int>(nelem * esize / 16);
                uint4 buf[S::kQVecPerThread];
    #pragma unroll
                for (int i = 0; i < S::kQVecPerThread; ++i) {
                    const int v = tid + i * kConsumerWarps * 32;
                    if (v < nvec) buf[i] = __ldg(reinterpret_cast<const uint4 *>(qsrc) + v);
                }
    #pragma unroll
                for (int i = 0; i < S::kQVecPerThread; ++i) {
                    const int v = tid + i * kConsumerWarps * 32;
                    if (v < nvec) {
                        if (p.q_is_bf16) {
                            const int e = v * 8, row = e / HD, col = e % HD;
                            float *dst = qs + row * S::kQRowFloats + col;
                            const uint32_t w[4] = {buf[i].x, buf[i].y, buf[i].z, buf[i].w};
    #pragma unroll
                            for (int j = 0; j < 4; ++j) {
                                dst[2 * j] = bf16lo_f32(w[j]);
                                dst[2 * j + 1] = bf16hi_f32(w[j]);
                            }
                        } else {
                            const int e = v * 4, row = e / HD, col = e % HD;
                            *reinterpret_cast<uint4 *>(qs + row * S::kQRowFloats + col) = buf[i];
                        }
                    }
                }
            } else {
                for (int e = tid; e < nelem; e += kConsumerWarps * 32) {
                    const float x = p.q_is_bf16 ? __bfloat162float(reinterpret_cast<const __nv_bfloat16 *>(qsrc)[e])
                                                : reinterpret_cast<const float *>(qsrc)[e];
                    qs[(e / HD) * S::kQRowFloats + e % HD] = x;
                }
            }
            asm volatile("bar.sync 1, %0;" ::"n"(kConsumerWarps * 32) : "memory");
        }

        // Q^T as B fragments (k = head dim, n = head g), bf16 hi (+ lo for fp32 Q).
        uint32_t qhi[KSTEPS][2], qlo[KSTEPS][2];
        {
            const bool valid = g < nh;
            const float *qrow = qs + (valid ? g : 0) * S::kQRowFloats;
    #pragma unroll
            for (int kk = 0; kk < KSTEPS; ++kk) {
    #pragma unroll
                for (int half = 0; half < 2; ++half) {
                    const int d = kk * 16 + half * 8 + tq * 2;
                    const float2 v = *reinterpret_cast<const float2 *>(qrow + d);
                    split_bf16x2(valid ? v.x : 0.f, valid ? v.y : 0.f, qhi[kk][half], qlo[kk][half]);
                }
            }
        }
        const bool use_lo = !p.q_is_bf16;

        const float kLog2e = 1.4426950408889634f;
        const float cap = p.softcap;
        const float inv_cap = cap > 0.f ? 1.f / cap : 0.f;

        float m_run[2] = {-INFINITY, -INFINITY};   // heads 2tq, 2tq+1 (warp-uniform per column)
        float l_run[2] = {0.f, 0.f};                // this thread's keys only
        float o[KSTEPS][4];
    #pragma unroll
        for (int i = 0; i < KSTEPS; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;

        bool ok = true;
        int s = 0, phase = 0;
        for (int t = 0; t < ntiles; ++t) {
            if (!mbar_wait(smem_u32(&full_bar[s]), phase, p.err, kErrWaitTmaFull)) {
                ok = false;
                break;
            }
            const int kb = t * kKeysPerTile + warp * 16;   // first key of this warp's block
            const int nv = nkeys - kb;                     // valid keys in the block (may be <=0 or >16)
            if (nv > 0) {
                const uint32_t kbase = smem_u32(smem + s * S::kStageBytes);
                const uint32_t vbase = kbase + S::kTileBytes;

                // ---- S^T = K . Q^T ----
                float acc[4] = {0.f, 0.f, 0.f, 0.f};
                {
                    const int row = warp * 16 + (lane & 7) + ((lane >> 3) & 1) * 8;
    #pragma unroll
                    for (int kk = 0; kk < KSTEPS; ++kk) {
                        const int chunk = (kk & 3) * 2 + (lane >> 4);
                        uint32_t a0, a1, a2, a3;
                        ldsm_x4(kbase + (kk >> 2) * kSubtileBytes + sw128_offset(row, chunk), a0, a1, a2, a3);
                        mma_bf16_16816(acc, a0, a1, a2, a3, qhi[kk][0], qhi[kk][1]);
                        if (use_lo) mma_bf16_16816(acc, a0, a1, a2, a3, qlo[kk][0], qlo[kk][1]);
                    }
                }
                // acc[0]=(key g, head 2tq) acc[1]=(key g, head 2tq+1) acc[2]=(key g+8, 2tq) acc[3]=(key g+8, 2tq+1)
                float sc[4];
    #pragma unroll
                for (int i = 0; i < 4; ++i) {
                    float x = acc[i] * p.scale;
                    if (cap > 0.f) x = cap * tanhf(x * inv_cap);
                    const int key = g + (i >> 1) * 8;
                    sc[i] = key < nv ? x : -INFINITY;
                }
                float mb0 = fmaxf(sc[0], sc[2]);
                float mb1 = fmaxf(sc[1], sc[3]);
    #pragma unroll
                for (int off = 4; off < 32; off <<= 1) {
                    mb0 = fmaxf(mb0, __shfl_xor_sync(0xffffffffu, mb0, off));
                    mb1 = fmaxf(mb1, __shfl_xor_sync(0xffffffffu, mb1, off));
                }
                const float mn0 = fmaxf(m_run[0], mb0);
                const float mn1 = fmaxf(m_run[1], mb1);
                const float corr0 = fast_exp2((m_run[0] - mn0) * kLog2e);
                const float corr1 = fast_exp2((m_run[1] - mn1) * kLog2e);
                m_run[0] = mn0;
                m_run[1] = mn1;
                const float p0 = fast_exp2((sc[0] - mn0) * kLog2e);
                const float p1 = fast_exp2((sc[1] - mn1) * kLog2e);
                const float p2 = fast_exp2((sc[2] - mn0) * kLog2e);
                const float p3 = fast_exp2((sc[3] - mn1) * kLog2e);
                l_run[0] = l_run[0] * corr0 + p0 + p2;
                l_run[1] = l_run[1] * corr1 + p1 + p3;
    #pragma unroll
                for (int i = 0; i < KSTEPS; ++i) {
                    o[i][0] *= corr0;
                    o[i][1] *= corr1;
                    o[i][2] *= corr0;
                    o[i][3] *= corr1;
                }
                const uint32_t pb0 = movmatrix_t(pack_f16x2(p0, p1));   // keys 0-7
                const uint32_t pb1 = movmatrix_t(pack_f16x2(p2, p3));   // keys 8-15

                // ---- O^T += V^T . P^T ----
                {
                    const int m = lane >> 3;
                    const int row = warp * 16 + (lane & 7) + (m >> 1) * 8;
                    const bool tail = nv < 16;
                    const int k0 = 2 * tq, k1 = 2 * tq + 8;   // keys held in a0/a1 and a2/a3
    #pragma unroll
                    for (int db = 0; db < KSTEPS; ++db) {
                        const int chunk = (db & 3) * 2 + (m & 1);
                        uint32_t a0, a1, a2, a3;
                        ldsm_x4_t(vbase + (db >> 2) * kSubtileBytes + sw128_offset(row, chunk), a0, a1, a2, a3);
                        if (tail) {
                            const uint32_t mlo = (k0 < nv ? 0x0000ffffu : 0u) | (k0 + 1 < nv ? 0xffff0000u : 0u);
                            const uint32_t mhi = (k1 < nv ? 0x0000ffffu : 0u) | (k1 + 1 < nv ? 0xffff0000u : 0u);
                            a0 &= mlo;
                            a1 &= mlo;
                            a2 &= mhi;
                            a3 &= mhi;
                        }
                        mma_f16_16816(o[db], a0, a1, a2, a3, pb0, pb1);
                    }
                }
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(smem_u32(&empty_bar[s]));
            if (++s == stages) {
                s = 0;
                phase ^= 1;
            }
        }

        // ---- merge the 4 consumer warps (stage buffers are free: every tile was consumed) ----
        // Layout: per warp, per head column: [m, l] then O[hd].
        float *red = reinterpret_cast<float *>(smem);
        constexpr int kRowF = HD + 2;
        asm volatile("bar.sync 1, %0;" ::"n"(kConsumerWarps * 32) : "memory");
        {
            // total l over the 8 key rows (lanes sharing tq)
            float l0 = l_run[0], l1 = l_run[1];
    #pragma unroll
            for (int off = 4; off < 32; off <<= 1) {
                l0 += __shfl_xor_sync(0xffffffffu, l0, off);
                l1 += __shfl_xor_sync(0xffffffffu, l1, off);
            }
            float *wbase = red + warp * 8 * kRowF;
            if (g == 0) {
                wbase[(2 * tq) * kRowF + 0] = m_run[0];
                wbase[(2 * tq) * kRowF + 1] = l0;
                wbase[(2 * tq + 1) * kRowF + 0] = m_run[1];
                wbase[(2 * tq + 1) * kRowF + 1] = l1;
            }
    #pragma unroll
            for (int db = 0; db < KSTEPS; ++db) {
                const int d0 = db * 16 + g;
                wbase[(2 * tq) * kRowF + 2 + d0] = o[db][0];
                wbase[(2 * tq + 1) * kRowF + 2 + d0] = o[db][1];
                wbase[(2 * tq) * kRowF + 2 + d0 + 8] = o[db][2];
                wbase[(2 * tq + 1) * kRowF + 2 + d0 + 8] = o[db][3];
            }
        }
        asm volatile("bar.sync 1, %0;" ::"n"(kConsumerWarps * 32) : "memory");
        if (!InCluster && !ok) return;
        for (int idx = threadIdx.x; idx < nh * HD; idx += kConsumerWarps * 32) {
            const int h = idx / HD, d = idx % HD;
            float M = -INFINITY;
    #pragma unroll
            for (int w = 0; w < kConsumerWarps; ++w) M = fmaxf(M, red[(w * 8 + h) * kRowF]);
            float acc = 0.f, lsum = 0.f;
    #pragma unroll
            for (int w = 0; w < kConsumerWarps; ++w) {
                const float mw = red[(w * 8 + h) * kRowF];
                const float f = mw == -INFINITY ? 0.f : fast_exp2((mw - M) * kLog2e);
                acc += f * red[(w * 8 + h) * kRowF + 2 + d];
                lsum += f * red[(w * 8 + h) * kRowF + 1];
            }
            if constexpr (InCluster) {
                float *cp = reinterpret_cast<float *>(smem + S::kCpartOff) + h * (HD + 2);
                cp[2 + d] = acc;
                if (d == 0) {
                    cp[0] = M;
                    cp[1] = lsum;
                }
            } else {
                const long long item = (static_cast<long long>(b) * p.n_heads + h_first + h) * p.max_chunks + c;
                p.part_o[item * HD + d] = acc;
                if (d == 0) {
                    p.part_ml[item * 2 + 0] = M;
                    p.part_ml[item * 2 + 1] = lsum;
                }
            }
        }
    } else {
        // idle chunk of a cluster (InCluster only): an empty partial
        float *cp = reinterpret_cast<float *>(smem + S::kCpartOff);
        for (int idx = threadIdx.x; idx < 8 * (HD + 2); idx += kConsumerWarps * 32)
            cp[idx] = (idx % (HD + 2)) == 0 ? -INFINITY : 0.f;
    }

    if constexpr (InCluster) {
        // ---- merge the chunks of this cluster; CTA rank r takes elements r, r+C, ... ----
        cluster_sync_all();
        const int C = static_cast<int>(gridDim.x);   // cluster size = chunks
        int nact = n > 0 ? (n + p.chunk - 1) / p.chunk : 0;
        if ((L - ks) > p.max_chunks * p.chunk) {
            if (c == 0 && threadIdx.x == 0) atomicOr(p.err, kErrBadArgs);
            nact = p.max_chunks;
        }
        const uint32_t cp0 = smem_u32(smem + S::kCpartOff);
        const float kLog2e = 1.4426950408889634f;
        for (int e = c * kThreads + threadIdx.x; e < nh * HD; e += C * kThreads) {
            const int h = e / HD, d = e % HD;
            const uint32_t hoff = static_cast<uint32_t>(h * (HD + 2)) * 4u;
            float M = -INFINITY;
            for (int r = 0; r < nact; ++r)
                M = fmaxf(M, ld_shared_cluster_f32(map_shared_rank(cp0 + hoff, r)));
            float acc = 0.f, lsum = 0.f;
            for (int r = 0; r < nact; ++r) {
                const uint32_t base = map_shared_rank(cp0 + hoff, r);
                const float mr = ld_shared_cluster_f32(base);
                const float f = mr == -INFINITY ? 0.f : fast_exp2((mr - M) * kLog2e);
                lsum += f * ld_shared_cluster_f32(base + 4);
                acc += f * ld_shared_cluster_f32(base + 8 + 4 * d);
            }
            p.out[(static_cast<long long>(b) * p.n_heads + h_first + h) * HD + d] = lsum > 0.f ? acc / lsum : 0.f;
        }
        cluster_sync_all();
    }
}

// out[b, h, :] = merge over the chunks of sequence b.
template <int HD>
__global__ void decode_combine_kernel(float *__restrict__ out, const float *__restrict__ part_o,
                                      const float *__restrict__ part_ml, const int *__restrict__ kv_len,
                                      int n_heads, int chunk, int max_chunks, int window, unsigned *err)
{
    griddep_wait();
    griddep_trigger();
    const int b = blockIdx.y, h = blockIdx.x, d = threadIdx.x;
    const int L = kv_len[b];
    const int ks = (window > 0 && L > window) ? L - window : 0;
    const int n = L - ks;
    int nch = n > 0 ? (n + chunk - 1) / chunk : 0;
    if (nch > max_chunks) {
        if (d == 0) atomicOr(err, kErrBadArgs);
        nch = max_chunks;
    }
    const long long item0 = (static_cast<long long>(b) * n_heads + h) * max_chunks;
    const float kLog2e = 1.4426950408889634f;
    float M = -INFINITY;
    for (int c = 0; c < nch; ++c) M = fmaxf(M, part_ml[(item0 + c) * 2]);
    float acc = 0.f, lsum = 0.f;
    for (int c = 0; c < nch; ++c) {
        const float f = fast_exp2((part_ml[(item0 + c) * 2] - M) * kLog2e);
        acc += f * part_o[(item0 + c) * HD + d];
        lsum += f * part_ml[(item0 + c) * 2 + 1];
    }
    out[(static_cast<long long>(b) * n_heads + h) * HD + d] = lsum > 0.f ? acc / lsum : 0.f;
}

// Keys per CTA: enough CTAs for ~8 per SM, at most SMOL_DECODE_MAX_CHUNK keys (larger
// chunks mean fewer partial results to merge, smaller ones a shorter tail).
#ifndef SMOL_DECODE_MAX_CHUNK
#define SMOL_DECODE_MAX_CHUNK 2048
#endif
// SMOL_DECODE_CLUSTER=0 in the environment forces the two-kernel form (measurement knob).
const bool g_decode_cluster = [] {
    const char *e = getenv("SMOL_DECODE_CLUSTER");
    return !(e && e[0] == '0');
}();
int decode_chunk_size(int n_seqs, int max_kv_len, int n_kv_heads, int n_qgroups)
{
    const long long work = static_cast<long long>(n_seqs) * n_kv_heads * n_qgroups * (max_kv_len > 0 ? max_kv_len : 1);
    long long c = (work + 148 * 8 - 1) / (148 * 8);
    c = (c + kKeysPerTile - 1) / kKeysPerTile * kKeysPerTile;
    if (c < kKeysPerTile) c = kKeysPerTile;
    if (c > SMOL_DECODE_MAX_CHUNK) c = SMOL_DECODE_MAX_CHUNK;
    return static_cast<int>(c);
}

// Raise the dynamic shared-memory limit of decode_split_kernel<HD, InCluster> on the
// current device, once per device (the attribute is per function and device).
template <int HD, bool InCluster>
bool ensure_split_smem_attr()
{
    static std::mutex mu;
    static bool done[64] = {};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) {
        cudaGetLastError();
        return false;
    }
    std::lock_guard<std::mutex> lock(mu);
    if (!done[dev]) {
        if (cudaFuncSetAttribute(decode_split_kernel<HD, InCluster>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 static_cast<int>(DecodeShape<HD>::smem_bytes(DecodeShape<HD>::kMaxStages))) !=
            cudaSuccess) {
            cudaGetLastError();
            return false;
        }
        done[dev] = true;
    }
    return true;
}

int device_sm_count()
{
    static int cached[64] = {};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) {
        cudaGetLastError();
        return 0;
    }
    if (!cached[dev]) {
        int n = 0;
        if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) {
            cudaGetLastError();
            return 0;
        }
        cached[dev] = n;
    }
    return cached[dev];
}

// Cluster form when the whole grid fits one wave with at most 8 chunks per
// (sequence, KV head, Q-head group): the smallest chunk (multiple of 64 keys) that
// satisfies both, i.e. the most CTAs that still run at once.  Returns the chunk, or 0
// for the two-kernel form.
template <int HD>
int cluster_chunk(int units, int max_kv_len)
{
    using S = DecodeShape<HD>;
    const int sms = device_sm_count();
    if (sms <= 0 || max_kv_len <= 0 || units <= 0) return 0;
    constexpr size_t kSmPerSm = 228 * 1024;   // shared memory per SM on sm_100
    for (int chunk = kKeysPerTile; chunk <= SMOL_DECODE_MAX_CHUNK; chunk += kKeysPerTile) {
        const int nch = (max_kv_len + chunk - 1) / chunk;
        if (nch > 8) continue;
        const int tiles = chunk / kKeysPerTile;
        const int stages = tiles < S::kMaxStages ? tiles : S::kMaxStages;
        size_t per_sm = kSmPerSm / (S::smem_bytes(stages) + 1024);
        if (per_sm > 2) per_sm = 2;   // __launch_bounds__(kThreads, 2)
        if (static_cast<long long>(units) * nch <= static_cast<long long>(sms) * static_cast<long long>(per_sm))
            return chunk;
    }
    return 0;
}

// Completes p (ring depth, Q load width) and launches the split and merge: one
// cluster kernel for single-wave problems, else the split kernel and the combine
// kernel over the partials in the workspace.
template <int HD>
int launch_split_combine(cudaStream_t st, DecodeParams &p, float *out, int n_seqs, int max_kv_len)
{
    using S = DecodeShape<HD>;
    p.out = out;
    p.q_vec16 = (reinterpret_cast<uintptr_t>(p.q) & 15) == 0;
    const int units = n_seqs * p.n_kv_heads * p.n_qgroups;
    const int cchunk = g_decode_cluster ? cluster_chunk<HD>(units, max_kv_len) : 0;
    if (cchunk > 0) {
        p.chunk = cchunk;
        p.max_chunks = (max_kv_len + cchunk - 1) / cchunk;
        const int tiles = cchunk / kKeysPerTile;
        p.stages = tiles < S::kMaxStages ? tiles : S::kMaxStages;
        if (!ensure_split_smem_attr<HD, true>()) return SMOL_B200_ERR_CUDA;
        cudaLaunchConfig_t cfg = {};
        cfg.gridDim = dim3(p.max_chunks, p.n_kv_heads * p.n_qgroups, n_seqs);
        cfg.blockDim = dim3(kThreads, 1, 1);
        cfg.dynamicSmemBytes = S::smem_bytes(p.stages);
        cfg.stream = st;
        cudaLaunchAttribute attr[2];
        attr[0].id = cudaLaunchAttributeClusterDimension;
        attr[0].val.clusterDim.x = p.max_chunks;
        attr[0].val.clusterDim.y = 1;
        attr[0].val.clusterDim.z = 1;
        attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        attr[1].val.programmaticStreamSerializationAllowed = 1;
        cfg.attrs = attr;
        cfg.numAttrs = g_pdl_scope ? 2 : 1;
        if (cudaLaunchKernelEx(&cfg, decode_split_kernel<HD, true>, p) != cudaSuccess) {
            cudaGetLastError();
            return SMOL_B200_ERR_CUDA;
        }
        return SMOL_B200_OK;
    }
    const int tiles = (p.chunk + kKeysPerTile - 1) / kKeysPerTile;   // most tiles one CTA streams
    p.stages = tiles < S::kMaxStages ? tiles : S::kMaxStages;
    if (!ensure_split_smem_attr<HD, false>()) return SMOL_B200_ERR_CUDA;
    dim3 grid(p.max_chunks, p.n_kv_heads * p.n_qgroups, n_seqs);
    if (launch_kernel(decode_split_kernel<HD, false>, grid, dim3(kThreads), S::smem_bytes(p.stages), st, p) !=
        cudaSuccess)
        return SMOL_B200_ERR_CUDA;
    dim3 cgrid(p.n_heads, n_seqs);
    return launch_kernel(decode_combine_kernel<HD>, cgrid, dim3(HD), 0, st, out,
                         static_cast<const float *>(p.part_o), static_cast<const float *>(p.part_ml), p.kv_len,
                         p.n_heads, p.chunk, p.max_chunks, p.window, p.err) == cudaSuccess
               ? SMOL_B200_OK
               : SMOL_B200_ERR_CUDA;
}

template <int HD>
int launch_decode(cudaStream_t st, float *out, const void *q, int q_is_bf16, const uint16_t *k_pool,
                  const uint16_t *v_pool, int64_t pool_rows, const int64_t *seq_row0, const int *kv_len,
                  int n_seqs, int max_kv_len, int n_heads, int n_kv_heads, float scale, int window,
                  float softcap, void *workspace)
{
    using S = DecodeShape<HD>;
    DecodeParams p;
    memset(&p, 0, sizeof(p));
    const int kv_dim = n_kv_heads * HD;
    if (!make_tmap_2d(&p.tmap_k, k_pool, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, kv_dim, pool_rows, 64, kKeysPerTile))
        return SMOL_B200_ERR_CUDA;
    if (!make_tmap_2d(&p.tmap_v, v_pool, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, kv_dim, pool_rows, 64, kKeysPerTile))
        return SMOL_B200_ERR_CUDA;
    p.group = n_heads / n_kv_heads;
    p.n_qgroups = (p.group + 7) / 8;
    p.chunk = decode_chunk_size(n_seqs, max_kv_len, n_kv_heads, p.n_qgroups);
    p.max_chunks = (max_kv_len + p.chunk - 1) / p.chunk;
    if (p.max_chunks < 1) p.max_chunks = 1;
    const size_t n_items = static_cast<size_t>(n_seqs) * n_heads * p.max_chunks;
    p.part_o = static_cast<float *>(workspace);
    p.part_ml = p.part_o + n_items * HD;
    p.q = q;
    p.q_is_bf16 = q_is_bf16;
    p.seq_row0 = seq_row0;
    p.kv_len = kv_len;
    p.err = device_error_word();
    p.n_heads = n_heads;
    p.n_kv_heads = n_kv_heads;
    p.window = window;
    p.scale = scale;
    p.softcap = softcap;

    return launch_split_combine<HD>(st, p, out, n_seqs, max_kv_len);
}

}  // namespace

// Partials for any call whose max_kv_len is at most `max_kv_len`.  The chunk count of a
// call, ceil(L / decode_chunk_size(L)), is not monotonic in L (the chunk grows in steps
// of 64 keys), so the size is that of the largest count over [1, max_kv_len]:
//   chunk == 64 (lower clamp)      count = ceil(L/64)       <= ceil(max/64)
//   64 <= chunk < 2048             chunk >= W*L/1184, so count <= ceil(1184/W)
//   chunk == SMOL_DECODE_MAX_CHUNK count = ceil(L/2048)     <= ceil(max/2048)
// with W = n_seqs * n_kv_heads * Q-head groups (the work per key); the first two cases
// together give min(ceil(max/64), ceil(1184/W)).  A workspace sized for max_kv_len
// therefore serves every shorter call, as a decoder that sizes it once for its cache
// capacity relies on.
size_t decode_workspace_bytes(int n_seqs, int max_kv_len, int n_heads, int n_kv_heads, int head_dim)
{
    if (n_seqs <= 0 || n_heads <= 0 || n_kv_heads <= 0 || head_dim <= 0) return 0;
    const int group = n_heads / n_kv_heads;
    const long long w = static_cast<long long>(n_seqs) * n_kv_heads * ((group + 7) / 8);
    const long long len = max_kv_len > 0 ? max_kv_len : 1;
    long long small = (len + kKeysPerTile - 1) / kKeysPerTile;
    const long long by_work = (148 * 8 + w - 1) / w;
    if (small > by_work) small = by_work;
    const long long big = (len + SMOL_DECODE_MAX_CHUNK - 1) / SMOL_DECODE_MAX_CHUNK;
    long long max_chunks = small > big ? small : big;
    if (max_chunks < 1) max_chunks = 1;
    const size_t n_items = static_cast<size_t>(n_seqs) * n_heads * static_cast<size_t>(max_chunks);
    return n_items * (static_cast<size_t>(head_dim) + 2) * sizeof(float);
}

int decode_attention(cudaStream_t st, float *out, const void *q, int q_is_bf16, const uint16_t *k_pool,
                     const uint16_t *v_pool, int64_t pool_rows, const int64_t *seq_row0, const int *kv_len,
                     int n_seqs, int max_kv_len, int n_heads, int n_kv_heads, int head_dim, float scale,
                     int window, float softcap, void *workspace, size_t workspace_bytes)
{
    if (n_seqs <= 0) return SMOL_B200_OK;
    if (!out || !q || !k_pool || !v_pool || !seq_row0 || !kv_len || n_heads <= 0 || n_kv_heads <= 0 ||
        n_heads % n_kv_heads != 0 || max_kv_len < 0 || pool_rows <= 0 || pool_rows >= (1ll << 31) ||
        n_seqs > 65535 || n_kv_heads * ((n_heads / n_kv_heads + 7) / 8) > 65535)
        return SMOL_B200_ERR_ARGS;
    if (head_dim != 64 && head_dim != 128 && head_dim != 256) return SMOL_B200_ERR_ARGS;
    if ((reinterpret_cast<uintptr_t>(k_pool) | reinterpret_cast<uintptr_t>(v_pool)) & 15) return SMOL_B200_ERR_ARGS;
    if (q_is_bf16 ? (reinterpret_cast<uintptr_t>(q) & 3) : (reinterpret_cast<uintptr_t>(q) & 7))
        return SMOL_B200_ERR_ARGS;
    const size_t need = decode_workspace_bytes(n_seqs, max_kv_len, n_heads, n_kv_heads, head_dim);
    if (!workspace || workspace_bytes < need) return SMOL_B200_ERR_WORKSPACE;
    // The split (and merge) kernels wait (griddepcontrol.wait) before reading anything, so
    // they may launch while the stream's previous kernel finishes.
    PdlScope pdl(g_api_pdl);
    switch (head_dim) {
    case 64:
        return launch_decode<64>(st, out, q, q_is_bf16, k_pool, v_pool, pool_rows, seq_row0, kv_len, n_seqs,
                                 max_kv_len, n_heads, n_kv_heads, scale, window, softcap, workspace);
    case 128:
        return launch_decode<128>(st, out, q, q_is_bf16, k_pool, v_pool, pool_rows, seq_row0, kv_len, n_seqs,
                                  max_kv_len, n_heads, n_kv_heads, scale, window, softcap, workspace);
    default:
        return launch_decode<256>(st, out, q, q_is_bf16, k_pool, v_pool, pool_rows, seq_row0, kv_len, n_seqs,
                                  max_kv_len, n_heads, n_kv_heads, scale, window, softcap, workspace);
    }
}


// ===========================================================================
// Allocation-free variant: smol_b200_decode_attention_noalloc
// ===========================================================================
// For callers that cannot call cudaMalloc: code that runs inside another
// framework's memory manager (which owns all device memory and forbids side
// allocations), allocation-free real-time paths, and hosts that must not allocate
// between set-up and teardown.  The split-KV partial results, which the regular
// entry point keeps in a caller-provided workspace, live here in one file-scope
// device array of fixed size.  Every GPU that loads this library holds the array
// until the process exits.
namespace {

constexpr size_t kNoAllocBytes = size_t(16) << 20;        // 16 MiB of partial results
constexpr size_t kNoAllocHeader = 256;                    // word 0: watchdog bits of this variant
static __device__ __align__(256) uint8_t g_noalloc_scratch[kNoAllocBytes];

std::mutex g_noalloc_mutex;
void *g_noalloc_ptr[16] = {};

// Set-up, once per device and with that device current: the host-side name of a
// __device__ array is only a stand-in, so its device address is looked up.
void *noalloc_scratch_for_current(int dev)
{
    std::lock_guard<std::mutex> lock(g_noalloc_mutex);
    if (!g_noalloc_ptr[dev]) {
        void *ptr = nullptr;
        const cudaError_t e = cudaGetSymbolAddress(&ptr, g_noalloc_scratch);
        if (e != cudaSuccess || !ptr) {
            cudaGetLastError();
            set_error(SMOL_B200_ERR_CUDA, "cudaGetSymbolAddress(no-alloc scratch) failed");
            return nullptr;
        }
        g_noalloc_ptr[dev] = ptr;
    }
    return g_noalloc_ptr[dev];
}

template <int HD>
int launch_decode_noalloc(cudaStream_t st, int dev, uint8_t *scratch, float *out, const void *q, int q_is_bf16,
                          const uint16_t *k_pool, const uint16_t *v_pool, int64_t pool_rows,
                          const int64_t *seq_row0, const int *kv_len, int n_seqs, int max_kv_len, int n_heads,
                          int n_kv_heads, float scale, int window, float softcap)
{
    using S = DecodeShape<HD>;
    DecodeParams p;
    memset(&p, 0, sizeof(p));
    const int kv_dim = n_kv_heads * HD;
    p.group = n_heads / n_kv_heads;
    p.n_qgroups = (p.group + 7) / 8;
    // Same chunking as the regular entry point, widened until the partials fit.
    const size_t cap = kNoAllocBytes - kNoAllocHeader;
    const int max_len = max_kv_len > 0 ? max_kv_len : 1;
    int chunk = decode_chunk_size(n_seqs, max_kv_len, n_kv_heads, p.n_qgroups);
    auto need = [&](int c) {
        const size_t chunks = static_cast<size_t>((max_len + c - 1) / c);
        return static_cast<size_t>(n_seqs) * n_heads * chunks * (HD + 2) * sizeof(float);
    };
    while (need(chunk) > cap && chunk < max_len) chunk *= 2;
    if (need(chunk) > cap) {
        char buf[192];
        snprintf(buf, sizeof(buf),
                 "smol_b200_decode_attention_noalloc: %d sequences x %d heads need %zu bytes of partials, "
                 "the static maximum is %zu",
                 n_seqs, n_heads, need(chunk), cap);
        set_error(SMOL_B200_ERR_ARGS, buf);
        return SMOL_B200_ERR_ARGS;
    }
    if (!make_tmap_2d(&p.tmap_k, k_pool, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, kv_dim, pool_rows, 64, kKeysPerTile))
        return SMOL_B200_ERR_CUDA;
    if (!make_tmap_2d(&p.tmap_v, v_pool, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, kv_dim, pool_rows, 64, kKeysPerTile))
        return SMOL_B200_ERR_CUDA;
    p.chunk = chunk;
    p.max_chunks = (max_len + chunk - 1) / chunk;
    const size_t n_items = static_cast<size_t>(n_seqs) * n_heads * p.max_chunks;
    p.part_o = reinterpret_cast<float *>(scratch + kNoAllocHeader);
    p.part_ml = p.part_o + n_items * HD;
    p.q = q;
    p.q_is_bf16 = q_is_bf16;
    p.seq_row0 = seq_row0;
    p.kv_len = kv_len;
    // Watchdog bits go to the library's device error word when this device already
    // has one (read by smol_cuda_device_error), else to word 0 of the static array.
    unsigned *err = device_error_word_if_created();
    p.err = err ? err : reinterpret_cast<unsigned *>(scratch);
    p.n_heads = n_heads;
    p.n_kv_heads = n_kv_heads;
    p.window = window;
    p.scale = scale;
    p.softcap = softcap;
    (void)dev;
    return launch_split_combine<HD>(st, p, out, n_seqs, max_kv_len);
}

}  // namespace

// Whether the allocation-free entry point has set up its array on the current device.
bool noalloc_in_use()
{
    int dev = -1;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 16) {
        cudaGetLastError();
        return false;
    }
    std::lock_guard<std::mutex> lock(g_noalloc_mutex);
    return g_noalloc_ptr[dev] != nullptr;
}

// Watchdog bits the allocation-free kernels left in word 0 of the array on the current
// device (they go there when no device error word had been created); `clear` resets
// the word.  0 when the entry point has not run on this device.  Copies, never
// allocates.
unsigned noalloc_watchdog_bits(bool clear)
{
    int dev = -1;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 16) {
        cudaGetLastError();
        return 0;
    }
    void *ptr = nullptr;
    {
        std::lock_guard<std::mutex> lock(g_noalloc_mutex);
        ptr = g_noalloc_ptr[dev];
    }
    if (!ptr) return 0;
    unsigned v = 0;
    if (cudaMemcpy(&v, ptr, sizeof(v), cudaMemcpyDeviceToHost) != cudaSuccess) {
        cudaGetLastError();
        return 0xffffffffu;
    }
    if (clear && v && cudaMemset(ptr, 0, sizeof(unsigned)) != cudaSuccess) cudaGetLastError();
    return v;
}

}  // namespace smolb200

// Part 3 of smol_b200.h: the allocation-free entry point (declared there).
extern "C" int smol_b200_decode_attention_noalloc(void *stream, float *out, const void *q, int q_is_bf16,
                                                  const uint16_t *k_pool, const uint16_t *v_pool, int64_t pool_rows,
                                                  const int64_t *seq_row0, const int *kv_len, int n_seqs,
                                                  int max_kv_len, int n_heads, int n_kv_heads, int head_dim,
                                                  float scale, int window, float softcap)
{
    using namespace smolb200;
    if (n_seqs <= 0) return SMOL_B200_OK;
    int rc = SMOL_B200_OK;
    if (!out || !q || !k_pool || !v_pool || !seq_row0 || !kv_len || n_heads <= 0 || n_kv_heads <= 0 ||
        n_heads % n_kv_heads != 0 || max_kv_len < 0 || pool_rows <= 0 || pool_rows >= (1ll << 31) ||
        n_seqs > 65535 || n_kv_heads * ((n_heads / n_kv_heads + 7) / 8) > 65535 ||
        (head_dim != 64 && head_dim != 128 && head_dim != 256) ||
        ((reinterpret_cast<uintptr_t>(k_pool) | reinterpret_cast<uintptr_t>(v_pool)) & 15) ||
        (q_is_bf16 ? (reinterpret_cast<uintptr_t>(q) & 3) : (reinterpret_cast<uintptr_t>(q) & 7)))
        rc = SMOL_B200_ERR_ARGS;
    int dev = -1;
    if (rc == SMOL_B200_OK && (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 16)) {
        cudaGetLastError();
        rc = SMOL_B200_ERR_NO_DEVICE;
    }
    uint8_t *scratch = nullptr;
    if (rc == SMOL_B200_OK) {
        scratch = static_cast<uint8_t *>(noalloc_scratch_for_current(dev));
        if (!scratch) rc = SMOL_B200_ERR_CUDA;
    }
    if (rc == SMOL_B200_OK) {
        cudaStream_t st = static_cast<cudaStream_t>(stream);
        switch (head_dim) {
        case 64:
            rc = launch_decode_noalloc<64>(st, dev, scratch, out, q, q_is_bf16, k_pool, v_pool, pool_rows, seq_row0,
                                           kv_len, n_seqs, max_kv_len, n_heads, n_kv_heads, scale, window, softcap);
            break;
        case 128:
            rc = launch_decode_noalloc<128>(st, dev, scratch, out, q, q_is_bf16, k_pool, v_pool, pool_rows, seq_row0,
                                            kv_len, n_seqs, max_kv_len, n_heads, n_kv_heads, scale, window, softcap);
            break;
        default:
            rc = launch_decode_noalloc<256>(st, dev, scratch, out, q, q_is_bf16, k_pool, v_pool, pool_rows, seq_row0,
                                            kv_len, n_seqs, max_kv_len, n_heads, n_kv_heads, scale, window, softcap);
            break;
        }
    }
    if (rc != SMOL_B200_OK && smol_cuda_last_error() == SMOL_B200_OK)
        set_error(rc, "smol_b200_decode_attention_noalloc");
    return rc;
}
