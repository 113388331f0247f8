// gemm.cu -- bf16 GEMM on the 5th-generation tensor cores, with the epilogues the
// SigLIP encoder's linear layers need.
//
//   C[m][n] = sum_k A[m][k] * W[n][k]  (+ bias[n]) (+ add[m % add_rows][n]) (GELU-tanh)
//   stored as fp32, bf16 or fp16, or added into an fp32 C (the residual stream); or,
//   for an interleaved gate/up weight, C[m][j] = act(c[2j]) * c[2j+1] (SwiGLU / GeGLU)
//
// This is smol_linear (matmul.c:70-100: y = x W^T + b) and the bias + GELU / residual
// steps around it in siglip_forward (siglip.c:116-146), with A and W in bf16 and fp32
// accumulation.  Both operands are K-major, as the reference stores them (x rows, W
// rows), so TMA copies 128-row x 64-column boxes straight into 128-byte-swizzled
// shared memory and tcgen05.mma reads them through matrix descriptors.  Rows past M or
// N and columns past K are outside the tensor maps and arrive as zeros; the epilogue
// writes only rows < M and columns < N.
//
// One CTA computes one 128 x 128 tile of C: warp 0 issues the TMA loads of a 3-stage
// ring of A / W boxes, warp 1 allocates 128 TMEM columns and issues the MMAs (4 per
// 64-wide k block, K = 16 each), warps 2-5 read the fp32 accumulator back from TMEM
// (each warp the 32 lanes its index allows) and apply the epilogue.  96 KB of shared
// memory, so two CTAs share an SM and one's epilogue overlaps the other's MMAs.
// Every wait is bounded (2 s), reports through the device error word and lets the CTA
// drain its copies and MMAs before it exits.
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include "b200_common.cuh"
#include "runtime.h"

namespace smolb200 {
namespace {

constexpr int kBM = 128, kBN = 128, kBK = 64;
constexpr int kStages = 3;
constexpr int kGemmThreads = 192;
constexpr int kProducerWarp = 0, kMmaWarp = 1;
constexpr int kABytes = kBM * kBK * 2;   // 16 KB
constexpr int kWBytes = kBN * kBK * 2;   // 16 KB
constexpr int kStageBytes = kABytes + kWBytes;
constexpr int kTmemCols = kBN;
constexpr uint32_t kIdesc = umma_idesc_f16(kBM, kBN, true, false);   // bf16 x bf16 -> f32, both K-major

struct GemmBarriers {
    uint64_t full[kStages], empty[kStages];
    uint64_t acc_full, mma_done;
    uint32_t tmem_base;
    int abort;
};

constexpr int kSmemBytes = 1024 + kStages * kStageBytes + 256;   // alignment slack, ring, barriers

struct GemmParams {
    CUtensorMap ta, tw;
    CUtensorMap to;           // the output as a 32-row box map (staged epilogue)
    int tma_out;              // 1: the epilogue stores through `to` (TMA store, or reduce-add for F32_ADD)
    void *out;
    long long ldo;
    const float *bias;        // [N] or null
    const float *add;         // [add_rows][ld_add] or null
    long long ld_add;
    int add_rows;
    int M, N, K;
    int out_kind;             // SMOL_B200_GEMM_OUT_*
    int gelu;
    int gate;                 // 0, or 2 / 3: columns (2j, 2j+1) -> out[j] = act(c[2j]) * c[2j+1], act SiLU / GELU-tanh
    int vec_ok;               // rows of `out` (and `add`) are 16-byte aligned
    int bias_vec, add_vec;    // bias / rows of `add` are 16-byte aligned: 16-byte loads
    unsigned *err;
};

__device__ __forceinline__ float gelu_tanh(float x)
{
    // smol_gelu (activation.c:29-36)
    const float x3 = x * x * x;
    const float inner = 0.7978845608028654f * (x + 0.044715f * x3);
    return 0.5f * x * (1.0f + tanhf(inner));
}

// The gated forms of smol_swiglu_multiply / smol_geglu_multiply (activation.c:55-126):
// gate g = column 2j, up u = column 2j+1 of the interleaved gate/up product.
__device__ __forceinline__ float gated(float g, float u, int gate)
{
    return (gate == 3 ? gelu_tanh(g) : g / (1.0f + expf(-g))) * u;
}

// Epilogue math of one 32-column chunk of one row: bias, addend, activation (in place).
__device__ __forceinline__ void chunk_math(const GemmParams &p, int row, int nb, float (&v)[32])
{
    const bool whole = nb + 32 <= p.N;
    if (p.bias) {
        if (whole && p.bias_vec) {   // the same 32 values for every row: 8 broadcast 16-byte loads
#pragma unroll
            for (int q = 0; q < 8; ++q) {
                const float4 b4 = __ldg(reinterpret_cast<const float4 *>(p.bias + nb) + q);
                v[4 * q] += b4.x;
                v[4 * q + 1] += b4.y;
                v[4 * q + 2] += b4.z;
                v[4 * q + 3] += b4.w;
            }
        } else {
#pragma unroll
            for (int i = 0; i < 32; ++i)
                if (nb + i < p.N) v[i] += p.bias[nb + i];
        }
    }
    if (p.add) {
        const float *ar = p.add + static_cast<long long>(row % p.add_rows) * p.ld_add + nb;
        if (whole && p.add_vec) {
#pragma unroll
            for (int q = 0; q < 8; ++q) {
                const float4 a4 = __ldg(reinterpret_cast<const float4 *>(ar) + q);
                v[4 * q] += a4.x;
                v[4 * q + 1] += a4.y;
                v[4 * q + 2] += a4.z;
                v[4 * q + 3] += a4.w;
            }
        } else {
#pragma unroll
            for (int i = 0; i < 32; ++i)
                if (nb + i < p.N) v[i] += ar[i];
        }
    }
    if (p.gelu) {
#pragma unroll
        for (int i = 0; i < 32; ++i) v[i] = gelu_tanh(v[i]);
    }
}

// Epilogue of one 32-column chunk of one row: bias, addend, activation, store.
__device__ __forceinline__ void store_chunk(const GemmParams &p, int row, int nb, const uint32_t (&r)[32])
{
    if (row >= p.M || nb >= p.N) return;
    float v[32];
#pragma unroll
    for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
    chunk_math(p, row, nb, v);
    const bool full = p.vec_ok && nb + 32 <= p.N;
    if (p.gate) {   // 16 outputs from the 32 columns: out[nb/2 + j]
        float gv[16];
#pragma unroll
        for (int j = 0; j < 16; ++j) gv[j] = gated(v[2 * j], v[2 * j + 1], p.gate);
        const long long ob = static_cast<long long>(row) * p.ldo + nb / 2;
        if (p.out_kind == SMOL_B200_GEMM_OUT_BF16) {
            uint16_t *o = static_cast<uint16_t *>(p.out) + ob;
            if (full) {
#pragma unroll
                for (int q = 0; q < 2; ++q) {
                    uint4 w;
                    uint32_t *wp = reinterpret_cast<uint32_t *>(&w);
#pragma unroll
                    for (int j = 0; j < 4; ++j) wp[j] = pack_bf16x2(gv[q * 8 + 2 * j], gv[q * 8 + 2 * j + 1]);
                    *reinterpret_cast<uint4 *>(o + q * 8) = w;
                }
            } else {
#pragma unroll
                for (int j = 0; j < 16; ++j)
                    if (nb + 2 * j + 1 < p.N) o[j] = static_cast<uint16_t>(pack_bf16x2(gv[j], 0.f) & 0xffffu);
            }
        } else {
            float *o = static_cast<float *>(p.out) + ob;
#pragma unroll
            for (int j = 0; j < 16; ++j)
                if (nb + 2 * j + 1 < p.N) o[j] = gv[j];
        }
        return;
    }
    if (p.out_kind == SMOL_B200_GEMM_OUT_BF16 || p.out_kind == SMOL_B200_GEMM_OUT_F16) {
        uint16_t *o = static_cast<uint16_t *>(p.out) + static_cast<long long>(row) * p.ldo + nb;
        const bool h = p.out_kind == SMOL_B200_GEMM_OUT_F16;
        if (h) {   // an fp16 output (SigLIP's V) reports values it cannot hold instead of storing inf
            bool over = false;
#pragma unroll
            for (int i = 0; i < 32; ++i) over |= nb + i < p.N && f16_overflows(v[i]);
            if (over) atomicOr(p.err, kErrValueRange);
        }
        if (full) {
#pragma unroll
            for (int q = 0; q < 4; ++q) {
                uint4 w;
                uint32_t *wp = reinterpret_cast<uint32_t *>(&w);
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    const float a = v[q * 8 + 2 * j], b = v[q * 8 + 2 * j + 1];
                    wp[j] = h ? pack_f16x2(a, b) : pack_bf16x2(a, b);
                }
                *reinterpret_cast<uint4 *>(o + q * 8) = w;
            }
        } else {
#pragma unroll
            for (int i = 0; i < 32; ++i) {   // unrolled: v stays in registers
                if (nb + i >= p.N) continue;
                const uint32_t w = h ? pack_f16x2(v[i], 0.f) : pack_bf16x2(v[i], 0.f);
                o[i] = static_cast<uint16_t>(w & 0xffffu);
            }
        }
    } else {
        float *o = static_cast<float *>(p.out) + static_cast<long long>(row) * p.ldo + nb;
        const bool acc = p.out_kind == SMOL_B200_GEMM_OUT_F32_ADD;
        if (full) {
#pragma unroll
            for (int q = 0; q < 8; ++q) {
                float4 w = make_float4(v[4 * q], v[4 * q + 1], v[4 * q + 2], v[4 * q + 3]);
                if (acc) {
                    const float4 o4 = *reinterpret_cast<const float4 *>(o + 4 * q);
                    w.x += o4.x;
                    w.y += o4.y;
                    w.z += o4.z;
                    w.w += o4.w;
                }
                *reinterpret_cast<float4 *>(o + 4 * q) = w;
            }
        } else {
#pragma unroll
            for (int i = 0; i < 32; ++i)
                if (nb + i < p.N) o[i] = acc ? o[i] + v[i] : v[i];
        }
    }
}

// Staged epilogue of one 32-column chunk (columns n0 + 32c) of a warp's 32 rows (from
// y0): the values go into one of the warp's two alternating 4 KB boxes (32 rows x 128
// bytes, 128B-swizzled) in `stage`, and a full box leaves as a TMA tensor store -- or,
// for an fp32 output that is added to, as a TMA reduce-add, so the residual is added in
// L2 and never read into the SM -- with one box in flight while the next is written.
// fp32: one box per chunk; 16-bit: chunks 2j and 2j+1 share a box of 64 columns.
__device__ __forceinline__ void staged_chunk(const GemmParams &p, uint8_t *stage, int &boxes, int row, int y0, int n0,
                                             int c, int n_chunks, int lane, const uint32_t (&r)[32])
{
    const bool f32 = p.out_kind == SMOL_B200_GEMM_OUT_F32 || p.out_kind == SMOL_B200_GEMM_OUT_F32_ADD;
    float v[32];
#pragma unroll
    for (int k = 0; k < 32; ++k) v[k] = __uint_as_float(r[k]);
    chunk_math(p, row, n0 + c * 32, v);
    // fp32: one box per chunk; 16-bit: chunks 2j, 2j+1 share a box (64 columns)
    const bool first_half = f32 || (c & 1) == 0;
    uint8_t *box = stage + (boxes & 1) * 4096;
    if (first_half) {
        if (lane == 0 && boxes >= 1) bulk_wait_read1();   // this slot's previous store read it
        __syncwarp();
    }
    if (f32) {
#pragma unroll
        for (int q = 0; q < 8; ++q)
            *reinterpret_cast<float4 *>(box + sw128_offset(lane, q)) =
                make_float4(v[4 * q], v[4 * q + 1], v[4 * q + 2], v[4 * q + 3]);
    } else {
        const bool h = p.out_kind == SMOL_B200_GEMM_OUT_F16;
        if (h) {   // an fp16 output reports values it cannot hold instead of storing inf
            bool over = false;
#pragma unroll
            for (int k = 0; k < 32; ++k) over |= row < p.M && n0 + c * 32 + k < p.N && f16_overflows(v[k]);
            if (over) atomicOr(p.err, kErrValueRange);
        }
#pragma unroll
        for (int u = 0; u < 4; ++u) {
            uint4 w4;
            uint32_t *wp = reinterpret_cast<uint32_t *>(&w4);
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                const float x0 = v[u * 8 + 2 * j], x1 = v[u * 8 + 2 * j + 1];
                wp[j] = h ? pack_f16x2(x0, x1) : pack_bf16x2(x0, x1);
            }
            *reinterpret_cast<uint4 *>(box + sw128_offset(lane, (c & 1) * 4 + u)) = w4;
        }
    }
    // a box leaves when full: every fp32 chunk, every second 16-bit chunk, or the
    // last chunk holding columns < N (columns past N are clipped by the store)
    if (f32 || (c & 1) == 1 || c == n_chunks - 1) {
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) {
            const int x = n0 + (f32 ? c : (c & ~1)) * 32, y = y0;
            if (p.out_kind == SMOL_B200_GEMM_OUT_F32_ADD)
                tma_reduce_add_4d(&p.to, smem_u32(box), x, y, 0, 0);
            else
                tma_store_4d(&p.to, smem_u32(box), x, y, 0, 0);
            bulk_commit();
        }
        __syncwarp();
        ++boxes;
    }
}

__global__ void __launch_bounds__(kGemmThreads, 2) gemm_bf16_kernel(const __grid_constant__ GemmParams p)
{
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    GemmBarriers *bars = reinterpret_cast<GemmBarriers *>(smem + kStages * kStageBytes);
    const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
    const int n0 = blockIdx.x * kBN, m0 = blockIdx.y * kBM;
    const int n_kb = (p.K + kBK - 1) / kBK;

    if (threadIdx.x == 0) {
        for (int s = 0; s < kStages; ++s) {
            mbar_init(smem_u32(&bars->full[s]), 1);
            mbar_init(smem_u32(&bars->empty[s]), 1);
        }
        mbar_init(smem_u32(&bars->acc_full), 1);
        mbar_init(smem_u32(&bars->mma_done), 1);
        bars->abort = 0;
        fence_mbar_init();
    }
    if (warp == kMmaWarp) {
        tmem_alloc(smem_u32(&bars->tmem_base), kTmemCols);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = bars->tmem_base;

    if (warp == kProducerWarp) {
        if (lane == 0) {
            tma_prefetch_desc(&p.ta);
            tma_prefetch_desc(&p.tw);
            int issued = 0;
            for (int kb = 0; kb < n_kb; ++kb) {
                const int st = kb % kStages;
                if (kb >= kStages &&
                    !mbar_wait(smem_u32(&bars->empty[st]), ((kb / kStages) - 1) & 1, p.err, kErrWaitTmaEmpty)) {
                    atomicExch(&bars->abort, 1);
                    break;
                }
                if (atomicAdd(&bars->abort, 0)) break;
                const uint32_t full = smem_u32(&bars->full[st]);
                const uint32_t sa = smem_u32(smem + st * kStageBytes);
                mbar_arrive_expect_tx(full, kStageBytes);
                tma_load_2d(sa, &p.ta, full, kb * kBK, m0);
                tma_load_2d(sa + kABytes, &p.tw, full, kb * kBK, n0);
                ++issued;
            }
            // every issued copy lands before the CTA may exit
            for (int kb = issued > kStages ? issued - kStages : 0; kb < issued; ++kb)
                mbar_wait(smem_u32(&bars->full[kb % kStages]), (kb / kStages) & 1, p.err, kErrDrain);
        }
    } else if (warp == kMmaWarp) {
        if (lane == 0) {
            for (int kb = 0; kb < n_kb; ++kb) {
                const int st = kb % kStages;
                if (!mbar_wait(smem_u32(&bars->full[st]), (kb / kStages) & 1, p.err, kErrWaitTmaFull) ||
                    atomicAdd(&bars->abort, 0)) {
                    atomicExch(&bars->abort, 1);
                    break;
                }
                tc_fence_after();
                const uint32_t sa = smem_u32(smem + st * kStageBytes);
#pragma unroll
                for (int kk = 0; kk < kBK / 16; ++kk) {   // 16 bf16 = 32 bytes along K inside the swizzled row
                    const uint64_t adesc = umma_sdesc_sw128(sa + kk * 32, 16, 1024);
                    const uint64_t bdesc = umma_sdesc_sw128(sa + kABytes + kk * 32, 16, 1024);
                    umma_ss(tmem, adesc, bdesc, kIdesc, (kb > 0 || kk > 0) ? 1u : 0u);
                }
                umma_commit(smem_u32(&bars->empty[st]));
            }
            // the epilogue waits for this (it checks `abort` before it reads TMEM)
            umma_commit(smem_u32(&bars->acc_full));
            // every MMA completes before TMEM is released
            umma_commit(smem_u32(&bars->mma_done));
            mbar_wait(smem_u32(&bars->mma_done), 0, p.err, kErrDrain);
        }
    } else {
        // ================= epilogue: thread = one row of the tile =================
        const int quarter = warp & 3;                       // TMEM lanes this warp may read
        const int row = m0 + quarter * 32 + lane;
        const bool waited = mbar_wait(smem_u32(&bars->acc_full), 0, p.err, kErrWaitMma);
        tc_fence_after();
        // warp-uniform: tcgen05.ld is a warp-collective instruction
        if (__all_sync(0xffffffffu, waited && atomicAdd(&bars->abort, 0) == 0)) {
            const uint32_t taddr = tmem + (static_cast<uint32_t>(quarter * 32) << 16);
            // staged epilogue (p.tma_out) in the first ring stage, free once the last MMA
            // completed: two alternating 4 KB boxes per warp, as in the wide form
            static_assert(kStageBytes >= 4 * 2 * 4096, "epilogue staging in ring stage 0");
            uint8_t *my_stage = smem + quarter * 2 * 4096;
            int boxes = 0;
            const int n_chunks = min(kBN, p.N - n0 + 31) / 32;
            for (int c = 0; c < kBN / 32; ++c) {
                if (c >= n_chunks) break;
                uint32_t r[32];
                tmem_ld32(taddr + c * 32, r);
                tmem_ld_wait();
                if (p.tma_out) staged_chunk(p, my_stage, boxes, row, m0 + quarter * 32, n0, c, n_chunks, lane, r);
                else store_chunk(p, row, n0 + c * 32, r);
            }
            if (lane == 0 && boxes > 0) bulk_wait_all0();   // the stores have completed before the CTA exits
            __syncwarp();
        }
    }

    tc_fence_before();
    __syncthreads();
    if (warp == kMmaWarp) {
        tc_fence_after();
        tmem_dealloc(tmem, kTmemCols);
    }
}

// ---------------------------------------------------------------------------
// Wide persistent form: one CTA per SM walks output tiles of 128 x 256 (N fastest, so
// the CTAs running together share A rows in L2).  A 128 x 128 tile streams 32 KB from
// L2 per 2.1 MFLOP (64 FLOP/B), which at the full tensor rate asks ~26 TB/s of L2;
// 128 x 256 streams 48 KB per 4.2 MFLOP (87 FLOP/B).  A 4-stage ring of 48 KB stages
// runs on across tiles, and two 256-column TMEM accumulators let the MMAs of tile i+1
// run while the epilogue warps drain tile i (tcgen05.mma kind::f16, M = 128, N = 256).
// ---------------------------------------------------------------------------
constexpr int kWBN = 256;
constexpr int kWStages = 4;
constexpr int kWBBytes = kWBN * kBK * 2;                  // 32 KB
constexpr int kWStageBytes = kABytes + kWBBytes;          // 48 KB
constexpr int kWTmemCols = 2 * kWBN;                      // two accumulators
constexpr uint32_t kWIdesc = umma_idesc_f16(kBM, kWBN, true, false);

struct WideBarriers {
    uint64_t full[kWStages], empty[kWStages];
    uint64_t acc_full[2], acc_empty[2];
    uint64_t mma_done;
    uint32_t tmem_base;
    int abort;
};

// Epilogue staging: per epilogue warp two 4 KB boxes (32 rows x 128 bytes), alternating.
constexpr int kWStageOut = 4 * 2 * 4096;
constexpr int kWSmemBytes = 1024 + kWStages * kWStageBytes + 256 + kWStageOut;
static_assert(kWSmemBytes <= 227 * 1024, "shared memory");

__global__ void __launch_bounds__(kGemmThreads, 1) gemm_bf16_wide_kernel(const __grid_constant__ GemmParams p)
{
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t *stage_out = smem + kWStages * kWStageBytes;   // 1024-aligned: the epilogue's swizzled boxes
    WideBarriers *bars = reinterpret_cast<WideBarriers *>(stage_out + kWStageOut);
    const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
    const int n_kb = (p.K + kBK - 1) / kBK;
    const int tiles_n = (p.N + kWBN - 1) / kWBN;
    const int n_tiles = tiles_n * ((p.M + kBM - 1) / kBM);

    if (threadIdx.x == 0) {
        for (int s = 0; s < kWStages; ++s) {
            mbar_init(smem_u32(&bars->full[s]), 1);
            mbar_init(smem_u32(&bars->empty[s]), 1);
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(smem_u32(&bars->acc_full[b]), 1);
            mbar_init(smem_u32(&bars->acc_empty[b]), 128);   // every epilogue thread
        }
        mbar_init(smem_u32(&bars->mma_done), 1);
        bars->abort = 0;
        fence_mbar_init();
    }
    if (warp == kMmaWarp) {
        tmem_alloc(smem_u32(&bars->tmem_base), kWTmemCols);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = bars->tmem_base;

    if (warp == kProducerWarp) {
        if (lane == 0) {
            tma_prefetch_desc(&p.ta);
            tma_prefetch_desc(&p.tw);
            int g = 0;   // k blocks issued so far (the ring's running index)
            bool ok = true;
            for (int t = blockIdx.x; t < n_tiles && ok; t += gridDim.x) {
                const int m0 = (t / tiles_n) * kBM, n0 = (t % tiles_n) * kWBN;
                for (int kb = 0; kb < n_kb; ++kb, ++g) {
                    const int st = g % kWStages;
                    if ((g >= kWStages &&
                         !mbar_wait(smem_u32(&bars->empty[st]), ((g / kWStages) - 1) & 1, p.err, kErrWaitTmaEmpty)) ||
                        atomicAdd(&bars->abort, 0)) {
                        atomicExch(&bars->abort, 1);
                        ok = false;
                        break;
                    }
                    const uint32_t full = smem_u32(&bars->full[st]);
                    const uint32_t sa = smem_u32(smem + st * kWStageBytes);
                    mbar_arrive_expect_tx(full, kWStageBytes);
                    tma_load_2d(sa, &p.ta, full, kb * kBK, m0);
                    tma_load_2d(sa + kABytes, &p.tw, full, kb * kBK, n0);
                }
            }
            // every issued copy lands before the CTA may exit
            for (int q = g > kWStages ? g - kWStages : 0; q < g; ++q)
                mbar_wait(smem_u32(&bars->full[q % kWStages]), (q / kWStages) & 1, p.err, kErrDrain);
        }
    } else if (warp == kMmaWarp) {
        if (lane == 0) {
            int g = 0, i = 0;
            bool ok = true;
            for (int t = blockIdx.x; t < n_tiles && ok; t += gridDim.x, ++i) {
                const int b = i & 1;
                const uint32_t acc = tmem + b * kWBN;
                // the epilogue has drained this accumulator (tile i - 2)
                if (i >= 2 && !mbar_wait(smem_u32(&bars->acc_empty[b]), ((i >> 1) - 1) & 1, p.err, kErrWaitSoftmax)) {
                    atomicExch(&bars->abort, 1);
                    break;
                }
                tc_fence_after();
                for (int kb = 0; kb < n_kb; ++kb, ++g) {
                    const int st = g % kWStages;
                    if (!mbar_wait(smem_u32(&bars->full[st]), (g / kWStages) & 1, p.err, kErrWaitTmaFull) ||
                        atomicAdd(&bars->abort, 0)) {
                        atomicExch(&bars->abort, 1);
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t sa = smem_u32(smem + st * kWStageBytes);
#pragma unroll
                    for (int kk = 0; kk < kBK / 16; ++kk) {   // 16 bf16 = 32 bytes along K inside the swizzled row
                        const uint64_t adesc = umma_sdesc_sw128(sa + kk * 32, 16, 1024);
                        const uint64_t bdesc = umma_sdesc_sw128(sa + kABytes + kk * 32, 16, 1024);
                        umma_ss(acc, adesc, bdesc, kWIdesc, (kb > 0 || kk > 0) ? 1u : 0u);
                    }
                    umma_commit(smem_u32(&bars->empty[st]));
                }
                umma_commit(smem_u32(&bars->acc_full[b]));   // also after an abort: wakes the epilogue
            }
            umma_commit(smem_u32(&bars->mma_done));
            mbar_wait(smem_u32(&bars->mma_done), 0, p.err, kErrDrain);
        }
    } else {
        const int quarter = warp & 3;
        // staged epilogue (p.tma_out): this warp's 32 rows leave through two alternating
        // 4 KB boxes (32 rows x 128 bytes, 128B-swizzled) as TMA tensor stores -- or, for an
        // fp32 output that is added to, as TMA reduce-adds, so the residual is never read
        // into the SM -- with one box in flight while the next is written
        uint8_t *my_stage = stage_out + quarter * 2 * 4096;
        int boxes = 0;   // boxes this warp has issued (lane 0 commits one bulk group per box)
        int i = 0;
        for (int t = blockIdx.x; t < n_tiles; t += gridDim.x, ++i) {
            const int b = i & 1;
            const int m0 = (t / tiles_n) * kBM, n0 = (t % tiles_n) * kWBN;
            const int row = m0 + quarter * 32 + lane;
            // An fp32 output that is added to (the residual stream): start this thread's row
            // of it (1 KB) on the way to L2 while the tile's MMAs run, where the epilogue's
            // TMA reduce-adds (or, without them, its read-add-writes) will find it.
            if (p.out_kind == SMOL_B200_GEMM_OUT_F32_ADD && row < p.M) {
                const char *orow = reinterpret_cast<const char *>(static_cast<const float *>(p.out) +
                                                                  static_cast<long long>(row) * p.ldo + n0);
                const int bytes = min(kWBN, p.N - n0) * 4;
                for (int off = 0; off < bytes; off += 128) asm volatile("prefetch.global.L2 [%0];" ::"l"(orow + off));
            }
            const bool waited = mbar_wait(smem_u32(&bars->acc_full[b]), (i >> 1) & 1, p.err, kErrWaitMma);
            tc_fence_after();
            if (!__all_sync(0xffffffffu, waited && atomicAdd(&bars->abort, 0) == 0)) break;
            const uint32_t taddr = tmem + b * kWBN + (static_cast<uint32_t>(quarter * 32) << 16);
            const int n_chunks = min(kWBN, p.N - n0 + 31) / 32;   // chunks holding columns < N
            for (int c = 0; c < kWBN / 32; ++c) {
                uint32_t r[32];
                if (c < n_chunks) {
                    tmem_ld32(taddr + c * 32, r);
                    tmem_ld_wait();
                }
                if (c == kWBN / 32 - 1) {   // the accumulator is free for tile i + 2
                    tc_fence_before();
                    mbar_arrive(smem_u32(&bars->acc_empty[b]));
                }
                if (c >= n_chunks) continue;
                if (!p.tma_out) {
                    store_chunk(p, row, n0 + c * 32, r);
                    continue;
                }
                staged_chunk(p, my_stage, boxes, row, m0 + quarter * 32, n0, c, n_chunks, lane, r);
            }
        }
        if (lane == 0 && boxes > 0) bulk_wait_all0();   // the stores have completed before the CTA exits
        __syncwarp();
    }

    tc_fence_before();
    __syncthreads();
    if (warp == kMmaWarp) {
        tc_fence_after();
        tmem_dealloc(tmem, kWTmemCols);
    }
}

// SMOL_GEMM_TMA_OUT=0 in the environment keeps the wide form's per-row stores
// (measurement knob).
const bool g_gemm_tma_out = [] {
    const char *e = getenv("SMOL_GEMM_TMA_OUT");
    return !(e && e[0] == '0');
}();

// SMOL_GEMM_WIDE=0 in the environment keeps every GEMM on the one-tile-per-CTA
// 128 x 128 form (measurement knob).
const bool g_gemm_wide = [] {
    const char *e = getenv("SMOL_GEMM_WIDE");
    return !(e && e[0] == '0');
}();

int sm_count()
{
    static int cached[64] = {};
    const int dev = current_device();
    if (dev < 0 || dev >= 64) return 148;
    if (!cached[dev]) {
        int n = 0;
        if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) n = 148;
        cached[dev] = n;
    }
    return cached[dev];
}

}  // namespace

int gemm_bf16(cudaStream_t st, void *out, int64_t ldo, int out_kind, const uint16_t *a, int64_t lda,
              const uint16_t *w, int64_t ldw, const float *bias, const float *add, int64_t ld_add, int add_rows,
              int M, int N, int K, int gelu, int gate)
{
    if (M <= 0 || N <= 0) return SMOL_B200_OK;
    if (gate && (gate < 2 || gate > 3 || (N & 1) || gelu || add ||
                 (out_kind != SMOL_B200_GEMM_OUT_BF16 && out_kind != SMOL_B200_GEMM_OUT_F32) || ldo < N / 2))
        return SMOL_B200_ERR_ARGS;
    if (!out || !a || !w || K <= 0 || lda < K || ldw < K || lda % 8 || ldw % 8 || (!gate && ldo < N) ||
        (reinterpret_cast<uintptr_t>(a) & 15) || (reinterpret_cast<uintptr_t>(w) & 15) ||
        out_kind < SMOL_B200_GEMM_OUT_F32 || out_kind > SMOL_B200_GEMM_OUT_F32_ADD || (add && (add_rows <= 0 || ld_add < N)))
        return SMOL_B200_ERR_ARGS;
    if ((M + kBM - 1) / kBM > 65535 || (N + kBN - 1) / kBN > 65535) return SMOL_B200_ERR_ARGS;   // grid limits
    unsigned *err = device_error_word();
    if (!err) return SMOL_B200_ERR_NO_DEVICE;
    const int dev = current_device();
    if (dev < 0 || dev >= 64) return SMOL_B200_ERR_CUDA;
    static bool raised[64] = {};
    if (!raised[dev]) {
        if (cudaFuncSetAttribute(gemm_bf16_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemBytes) !=
            cudaSuccess)
            return SMOL_B200_ERR_CUDA;
        raised[dev] = true;
    }
    // The wide persistent form when its 128 x 256 tiles fill at least one wave of SMs;
    // narrow outputs and small batches keep one 128 x 128 tile per CTA (more CTAs).
    const int sms = sm_count();
    const long long wide_tiles = static_cast<long long>((N + kWBN - 1) / kWBN) * ((M + kBM - 1) / kBM);
    const bool wide = g_gemm_wide && N >= kWBN && wide_tiles >= sms;
    GemmParams p;
    memset(&p, 0, sizeof(p));
    if (!make_tmap_2d(&p.ta, a, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, K, M, kBK, kBM, lda) ||
        !make_tmap_2d(&p.tw, w, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, K, N, kBK, wide ? kWBN : kBN, ldw))
        return SMOL_B200_ERR_CUDA;
    const int esz = out_kind == SMOL_B200_GEMM_OUT_BF16 || out_kind == SMOL_B200_GEMM_OUT_F16 ? 2 : 4;
    p.out = out;
    p.ldo = ldo;
    p.bias = bias;
    p.add = add;
    p.ld_add = ld_add;
    p.add_rows = add_rows > 0 ? add_rows : 1;
    p.M = M;
    p.N = N;
    p.K = K;
    p.out_kind = out_kind;
    p.gelu = gelu ? 1 : 0;
    p.gate = gate;
    p.vec_ok = (reinterpret_cast<uintptr_t>(out) % 16 == 0) && (ldo * esz) % 16 == 0;
    p.bias_vec = bias && reinterpret_cast<uintptr_t>(bias) % 16 == 0;
    p.add_vec = add && reinterpret_cast<uintptr_t>(add) % 16 == 0 && ld_add % 4 == 0;
    p.err = err;
    // The epilogue stages through TMA stores when the output rows are 16-byte aligned and
    // there is no gated pairing (whose 16 outputs per 32 columns keep the row stores):
    // 32-row boxes of 128 bytes (32 fp32 / 64 bf16 or fp16 columns).
    if (p.vec_ok && !gate && g_gemm_tma_out) {
        const CUtensorMapDataType dt = out_kind == SMOL_B200_GEMM_OUT_BF16   ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16
                                       : out_kind == SMOL_B200_GEMM_OUT_F16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16
                                                                             : CU_TENSOR_MAP_DATA_TYPE_FLOAT32;
        const long long plane = static_cast<long long>(ldo) * M;
        if (!make_tmap_4d(&p.to, out, dt, esz, N, M, 1, 1, ldo, plane, plane, esz == 4 ? 32 : 64, 32, 1))
            return SMOL_B200_ERR_CUDA;
        p.tma_out = 1;
    }
    if (wide) {
        static bool raised_w[64] = {};
        if (!raised_w[dev]) {
            if (cudaFuncSetAttribute(gemm_bf16_wide_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     kWSmemBytes) != cudaSuccess)
                return SMOL_B200_ERR_CUDA;
            raised_w[dev] = true;
        }
        const unsigned grid = static_cast<unsigned>(wide_tiles < sms ? wide_tiles : sms);
        return launch_kernel(gemm_bf16_wide_kernel, dim3(grid), dim3(kGemmThreads), kWSmemBytes, st, p) ==
                       cudaSuccess
                   ? SMOL_B200_OK
                   : SMOL_B200_ERR_CUDA;
    }
    const dim3 grid((N + kBN - 1) / kBN, (M + kBM - 1) / kBM);
    return launch_kernel(gemm_bf16_kernel, grid, dim3(kGemmThreads), kSmemBytes, st, p) == cudaSuccess
               ? SMOL_B200_OK
               : SMOL_B200_ERR_CUDA;
}

}  // namespace smolb200
