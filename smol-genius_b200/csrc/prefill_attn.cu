// prefill_attn.cu -- flash attention for prefill and encoders on tcgen05 tensor cores.
//
// Replaces smol_causal_attention with seq_q > 1 (attention.c:79-170), its sliding-
// window and softcap variants (:176-462), smol_bidirectional_attention (:32-77) and
// the prefix-LM composition PaliGemma needs, as one kernel with a mask kind.
//
// Two kernels.  v2 (head dims 64 and 128, below) computes two 128-row query tiles per
// work item and ping-pongs the tensor pipe between them.  v1 (head dim 256, whose O
// needs 256 TMEM columns) computes one: a work item is a 128-row query tile of one
// head of one batch element, and the CTA walks the key range its rows can see in
// tiles of BN keys.  Both run persistent CTAs over their work items (v2 for head dim
// 64; head dim 128 launches one CTA per item).  v1 warp roles (192 threads):
//   warps 0-3  softmax: thread t of warp w owns query row 32w+t, which is exactly
//              TMEM lane 32w+t, so row max / row sum need no shuffles;
//   warp 4     TMA producer: each item's Q, then K and V tiles through 2-slot rings;
//   warp 5     TMEM allocator and single-thread tcgen05.mma issuer.
// Per key tile j:
//   S_j = Q K_j^T    kind::f16, bf16 A/B from 128B-swizzled shared memory, fp32 in TMEM
//                    (two S buffers, so S_{j+1} runs while softmax works on S_j);
//   P_j = exp2(S_j*scale*log2e - m)  written back over S_j's TMEM columns as fp16;
//   O  += P_j V_j    A = P from TMEM, B = V (fp16, MN-major) from shared memory.
// P and V are fp16: with bf16 probabilities alone the result sits ~1.3e-3 (rel-L2)
// from an fp32 reference, fp16 keeps it near 1.5e-4.  The running maximum used for
// the exponent only moves when the row maximum grows by more than 2^8, so O is
// rescaled (TMEM load / scale / store by its owning thread) rarely; values stay
// below 256 and the final division uses the same maximum for O and the row sum.
#include <stdio.h>
#include <stdlib.h>

#include "b200_common.cuh"
#include "runtime.h"

namespace smolb200 {
namespace {

constexpr int kBM = 128;
// v1 warps: 0-3 softmax (one query row per thread), 4 TMA producer, 5 MMA issuer, 6-9
// epilogue (each reads the TMEM lanes of warp index % 4, i.e. the rows of softmax warp
// index % 4), so an item's output leaves while the next item's scores are computed.
constexpr int kThreads = 320;
constexpr int kSoftmaxThreads = 128;
constexpr int kProducerWarp = 4;
constexpr int kMmaWarp = 5;
constexpr int kEpiWarp0 = 6;
constexpr int kEpiWarps = 4;
// A tile's row sum of exponentials against the row's reference point may reach 2^15
// before the row moves its reference (each P value then fits fp16)
constexpr float kSpecSumLimit = 32768.0f;

template <int HD>
struct PrefillShape {
    static constexpr int BN = HD == 256 ? 64 : 128;
    static constexpr int kSub = HD / 64;                     // 64-column sub-tiles
    static constexpr int kQSubBytes = kBM * 128;
    static constexpr int kQBytes = kSub * kQSubBytes;
    static constexpr int kKvSubBytes = BN * 128;
    static constexpr int kKvBytes = kSub * kKvSubBytes;
    static constexpr int kStages = 2;
    static constexpr int kOffQ = 0;
    static constexpr int kOffK = kOffQ + kQBytes;
    static constexpr int kOffV = kOffK + kStages * kKvBytes;
    // Epilogue staging: 8 KB per epilogue warp (two 32-row x 128-byte TMA store boxes).
    static constexpr int kStageWarpBytes = 2 * 32 * 128;
    static constexpr int kOffStage = kOffV + kStages * kKvBytes;
    static constexpr int kOffBar = kOffStage + kEpiWarps * kStageWarpBytes;
    static constexpr int kUsed = kOffBar + 256 + 1024;
    static_assert(kUsed <= 227 * 1024, "shared memory");
    // At least ~116 KB so that a single CTA is resident per SM: every CTA
    // allocates all 512 TMEM columns.
    static constexpr int kSmemBytes = kUsed > 118 * 1024 ? kUsed : 118 * 1024;
    static constexpr int kTmS0 = 0, kTmS1 = BN, kTmO = 2 * BN;
    // Two columns after O hold each row's sum of exponentials for the epilogue warps,
    // by item parity (an item's sum is written while the epilogue may still read the
    // previous item's).
    static constexpr int kTmL = 2 * BN + HD;
    static constexpr int kTmCols = 512;
    static_assert(kTmL + 2 <= 512, "TMEM budget");
};

constexpr int kMaxExtraOuts = 7;   // further copies of the output (peers of an all-gather)

struct PrefillParams {
    CUtensorMap tq, tk, tv;
    // Output for the v2 epilogue's TMA stores, 128B swizzle: fp32 boxes of 32 columns x
    // 32 rows, or bf16 boxes of 64 columns x 32 rows when out_bf16.
    CUtensorMap to;
    // Further destinations of every output row (v2), same strides and type as `out`:
    // plain 16-byte stores, so a peer GPU's buffer mapped through CUDA IPC receives its
    // copy over NVLink while later tiles compute.
    void *out_more[kMaxExtraOuts];
    int n_more;
    int out_bf16;                   // output elements: 0 fp32, 1 bf16 (round to nearest even)
    void *out;
    long long out_row_stride, out_batch_stride;
    const int *window_starts;
    unsigned *err;
    int n_windows;
    int seq_q, seq_k, n_heads, group, mask_kind, q_offset, prefix_len, window;
    int hd;   // the caller's head dim (<= the kernel's HD: columns past it are zero on load, not stored)
    // v1: query rows per position in a tile -- the `pack` heads of a KV group that share
    // its keys (row r of a tile is position r / pack of head h + r % pack); 1 = one head
    int pack;
    float scale, scale_log2, softcap;
    // v2 work items: n_qblocks x n_ygroups (head pairs or heads) x batch
    int n_qblocks, n_ygroups, batch, pair_heads, heavy_first;
};

struct Barriers {
    uint64_t q_full, q_empty;
    uint64_t k_full[2], k_empty[2], v_full[2], v_empty[2];
    uint64_t s_full[2], p_full[2];
    uint64_t o_done, mma_done;
    uint64_t o_final;   // an item's last PV is complete (O and its row sums are final)
    uint64_t o_free;    // the epilogue warps have read O (the next item's first PV may start)
    uint32_t tmem_base;
};

__device__ __forceinline__ float fast_exp2(float x)
{
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

__device__ __forceinline__ uint64_t f2_pack(float lo, float hi)
{
    return static_cast<uint64_t>(__float_as_uint(lo)) | (static_cast<uint64_t>(__float_as_uint(hi)) << 32);
}
__device__ __forceinline__ uint64_t f2_fma(uint64_t a, uint64_t b, uint64_t c)
{
    uint64_t d;
    asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
    return d;
}
__device__ __forceinline__ uint64_t f2_add(uint64_t a, uint64_t b)
{
    uint64_t d;
    asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
    return d;
}
// The same two operations on float pairs: the pairs are formed and split with mov.b64
// inside the asm, which the register allocator maps onto register pairs, instead of
// 64-bit shifts and ors in C++ that can cost integer instructions per element.
__device__ __forceinline__ void fma2(float &d0, float &d1, float a0, float a1, float b0, float b1, float c0, float c1)
{
    asm("{\n\t.reg .b64 a, b, c, d;\n\t"
        "mov.b64 a, {%2, %3};\n\tmov.b64 b, {%4, %5};\n\tmov.b64 c, {%6, %7};\n\t"
        "fma.rn.f32x2 d, a, b, c;\n\tmov.b64 {%0, %1}, d;\n\t}"
        : "=f"(d0), "=f"(d1)
        : "f"(a0), "f"(a1), "f"(b0), "f"(b1), "f"(c0), "f"(c1));
}
__device__ __forceinline__ void add2(float &d0, float &d1, float a0, float a1, float b0, float b1)
{
    asm("{\n\t.reg .b64 a, b, d;\n\t"
        "mov.b64 a, {%2, %3};\n\tmov.b64 b, {%4, %5};\n\t"
        "add.rn.f32x2 d, a, b;\n\tmov.b64 {%0, %1}, d;\n\t}"
        : "=f"(d0), "=f"(d1)
        : "f"(a0), "f"(a1), "f"(b0), "f"(b1));
}
// 2^x for a pair of floats on the FMA pipe instead of MUFU (Cody-Waite range reduction
// + polynomial, the published method FlashAttention-4 applies to this bottleneck):
// n = round(x) via the 1.5*2^23 constant, f = x - n in [-1/2, 1/2], 2^f from a degree-3
// polynomial fitted here for relative error (max 7.5e-5 on the interval, below the fp16
// rounding of P), and n added to the exponent field.  x is clamped to >= -126 so the
// result stays a normal float (2^-126 rounds to 0 in fp16).  Pairs go through f32x2
// adds and FMAs on register pairs.
__device__ __forceinline__ void exp2_poly2(float x0, float x1, float &e0, float &e1)
{
    constexpr float kMagic = 12582912.0f;   // 1.5 * 2^23: x + kMagic holds round(x) in its low bits
    x0 = fmaxf(x0, -126.f);
    x1 = fmaxf(x1, -126.f);
    float j0, j1, r0, r1, f0, f1, p0, p1;
    add2(j0, j1, x0, x1, kMagic, kMagic);
    add2(r0, r1, j0, j1, -kMagic, -kMagic);          // r = round(x)
    fma2(f0, f1, r0, r1, -1.f, -1.f, x0, x1);        // f = x - r in [-1/2, 1/2]
    fma2(p0, p1, 0.05517166f, 0.05517166f, f0, f1, 0.24261113f, 0.24261113f);
    fma2(p0, p1, p0, p1, f0, f1, 0.69326097f, 0.69326097f);
    fma2(p0, p1, p0, p1, f0, f1, 0.99992806f, 0.99992806f);
    e0 = __uint_as_float(__float_as_uint(p0) + (__float_as_uint(j0) << 23));
    e1 = __uint_as_float(__float_as_uint(p1) + (__float_as_uint(j1) << 23));
}

__device__ __forceinline__ float max3f(float a, float b, float c)
{
    float d;
    asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
    return d;
}

// The first `ncols` (a multiple of 8, <= 32) of 32 consecutive output values of one row
// (rr scaled by inv), as fp32 or bf16, to `dst` (element offset `off` of an output
// buffer) with 16-byte stores.
__device__ __forceinline__ void store_row32(void *dst, long long off, const uint32_t (&rr)[32], float inv,
                                            bool bf16, int ncols = 32)
{
    if (bf16) {
        uint16_t *o = static_cast<uint16_t *>(dst) + off;
#pragma unroll
        for (int i = 0; i < 32; i += 8) {
            if (i >= ncols) break;
            uint4 v;
            v.x = pack_bf16x2(__uint_as_float(rr[i]) * inv, __uint_as_float(rr[i + 1]) * inv);
            v.y = pack_bf16x2(__uint_as_float(rr[i + 2]) * inv, __uint_as_float(rr[i + 3]) * inv);
            v.z = pack_bf16x2(__uint_as_float(rr[i + 4]) * inv, __uint_as_float(rr[i + 5]) * inv);
            v.w = pack_bf16x2(__uint_as_float(rr[i + 6]) * inv, __uint_as_float(rr[i + 7]) * inv);
            *reinterpret_cast<uint4 *>(o + i) = v;
        }
    } else {
        float *o = static_cast<float *>(dst) + off;
#pragma unroll
        for (int i = 0; i < 32; i += 4)
            if (i < ncols)
                *reinterpret_cast<float4 *>(o + i) =
                make_float4(__uint_as_float(rr[i]) * inv, __uint_as_float(rr[i + 1]) * inv,
                            __uint_as_float(rr[i + 2]) * inv, __uint_as_float(rr[i + 3]) * inv);
    }
}

// Keys [lo, hi) visible to query row i; written=false for rows no window covers
// (smol_bidirectional_attention leaves those rows untouched, attention.c:39-43).
__device__ __forceinline__ void row_range(const PrefillParams &p, int i, int &lo, int &hi, bool &written)
{
    const int pos = p.q_offset + i;
    written = true;
    lo = 0;
    switch (p.mask_kind) {
    case SMOL_MASK_CAUSAL: hi = pos + 1; break;
    case SMOL_MASK_PREFIX_LM: hi = max(pos + 1, p.prefix_len); break;
    case SMOL_MASK_WINDOWS: {
        int a = 0, b = p.n_windows;   // find w with ws[w] <= i < ws[w+1]
        if (p.n_windows <= 0 || i < p.window_starts[0] || i >= p.window_starts[p.n_windows]) {
            written = false;
            hi = 0;
            break;
        }
        while (b - a > 1) {
            const int mid = (a + b) >> 1;
            if (p.window_starts[mid] <= i) a = mid; else b = mid;
        }
        lo = p.window_starts[a];
        hi = p.window_starts[a + 1];
        break;
    }
    default: hi = p.seq_k; break;
    }
    if (hi > p.seq_k) hi = p.seq_k;
    if (p.window > 0 && pos >= p.window) lo = max(lo, pos - p.window + 1);   // attention.c:194-196
    if (lo < 0) lo = 0;
    if (hi < lo) hi = lo;
}

// First key of a work item's key tiles, given the lowest key `lo` any of its rows sees.
// Under a sliding window `lo` moves with the item's first row, so it is rounded down to
// a multiple of BN in absolute key index: a query row then meets the same key-tile
// boundaries -- hence the same online-softmax rescale points and the same fp16
// rounding of P -- whichever chunk of a chunked prefill (q_offset) it falls in.  The
// extra keys in front are masked for every row, and a fully masked tile changes
// neither the running maximum nor O (its P is exactly 0).  Causal and prefix-LM rows
// start at key 0 already; window masks are never chunked and keep their exact start.
template <int BN>
__device__ __forceinline__ int first_key_tile(const PrefillParams &p, int lo)
{
    return p.window > 0 ? (lo / BN) * BN : lo;
}

// Work item k of a v1 launch: (query tile qt, head h, batch b), query tiles fastest --
// in decreasing order of work for causal-like masks -- so that CTAs running at the same
// time share one (batch, KV head)'s K and V in L2.  A persistent CTA takes the items
// of rounds r = 0, 1, ... at positions blockIdx.x (even rounds) and gridDim.x-1-blockIdx.x
// (odd rounds).
struct Item1 {
    int qt, h, b, q0;      // h: first head of the tile; q0: first packed row (position q0 / pack)
    int lo_min, n_tiles;   // key tiles [lo_min, lo_min + n_tiles*BN) cover every row's keys
};

template <int BN>
__device__ __forceinline__ Item1 item1_geometry(const PrefillParams &p, int k)
{
    Item1 it;
    const int nq = p.n_qblocks;
    it.qt = p.heavy_first ? nq - 1 - k % nq : k % nq;
    const int r = k / nq;
    it.h = (r % p.n_ygroups) * p.pack;
    it.b = r / p.n_ygroups;
    it.q0 = it.qt * kBM;
    // every mask's [lo, hi) is non-decreasing in the position: first position -> lowest
    // key, last position -> highest
    int a = it.q0 / p.pack, z = (min(it.q0 + kBM, p.seq_q * p.pack) - 1) / p.pack;
    if (p.mask_kind == SMOL_MASK_WINDOWS) {
        a = max(a, p.window_starts[0]);
        z = min(z, p.window_starts[p.n_windows] - 1);
    }
    it.lo_min = 0;
    it.n_tiles = 0;
    if (z >= a) {
        int lo_a, hi_a, lo_z, hi_z;
        bool w;
        row_range(p, a, lo_a, hi_a, w);
        row_range(p, z, lo_z, hi_z, w);
        if (hi_z > lo_a) {
            it.lo_min = first_key_tile<BN>(p, lo_a);
            it.n_tiles = (hi_z - it.lo_min + BN - 1) / BN;
        }
    }
    return it;
}

__device__ __forceinline__ int item1_index(int r)
{
    const int c = (r & 1) ? static_cast<int>(gridDim.x) - 1 - static_cast<int>(blockIdx.x)
                          : static_cast<int>(blockIdx.x);
    return r * static_cast<int>(gridDim.x) + c;
}

// v1 (head dim 256): one 128-row query tile per work item; CTAs are persistent -- TMEM
// is allocated once and every barrier's phase runs on across items (q_full / q_empty,
// o_final / o_free once per item with key tiles, the K/V ring, S buffers and o_done once
// per key tile).
template <int HD>
__global__ void __launch_bounds__(kThreads, 1) prefill_kernel(const __grid_constant__ PrefillParams p)
{
    griddep_wait();   // programmatic launch: nothing of earlier kernels is read before this
    griddep_trigger();
    using S = PrefillShape<HD>;
    constexpr int BN = S::BN;
    const int n_items = p.n_qblocks * p.n_ygroups * p.batch;
    const int n_rounds = (n_items + static_cast<int>(gridDim.x) - 1) / static_cast<int>(gridDim.x);

    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    Barriers *bars = reinterpret_cast<Barriers *>(smem + S::kOffBar);

    const int warp = threadIdx.x / 32;
    const int lane = threadIdx.x % 32;

    if (threadIdx.x == 0) {
        mbar_init(smem_u32(&bars->q_full), 1);
        mbar_init(smem_u32(&bars->q_empty), 1);
        for (int s = 0; s < 2; ++s) {
            mbar_init(smem_u32(&bars->k_full[s]), 1);
            mbar_init(smem_u32(&bars->k_empty[s]), 1);
            mbar_init(smem_u32(&bars->v_full[s]), 1);
            mbar_init(smem_u32(&bars->v_empty[s]), 1);
            mbar_init(smem_u32(&bars->s_full[s]), 1);
            mbar_init(smem_u32(&bars->p_full[s]), kSoftmaxThreads);
        }
        mbar_init(smem_u32(&bars->o_done), 1);
        mbar_init(smem_u32(&bars->mma_done), 1);
        mbar_init(smem_u32(&bars->o_final), 1);
        mbar_init(smem_u32(&bars->o_free), kEpiWarps);
        fence_mbar_init();
    }
    if (warp == kMmaWarp) {
        tmem_alloc(smem_u32(&bars->tmem_base), S::kTmCols);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = bars->tmem_base;

    uint8_t *sQ = smem + S::kOffQ;
    uint8_t *sK = smem + S::kOffK;
    uint8_t *sV = smem + S::kOffV;

    if (warp == kProducerWarp) {
        // ================= TMA producer =================
        if (lane == 0) {
            tma_prefetch_desc(&p.tq);
            tma_prefetch_desc(&p.tk);
            tma_prefetch_desc(&p.tv);
            int qit = 0, g = 0, gv = 0;            // Q, K and V tiles issued
            int v_kvh = 0, v_key0 = 0, v_b = 0;   // V tile gv, owed until K tile gv + 1 is issued
            bool ok = true;
            // Within an item V(t) follows K(t+1): K(t+1) then waits only for S(t-1), not
            // behind V(t)'s wait for PV(t-2).  An item's last V goes before the next Q's wait.
            auto load_v = [&]() -> bool {
                const int st = gv & 1;
                if (gv >= 2 &&
                    !mbar_wait(smem_u32(&bars->v_empty[st]), ((gv >> 1) - 1) & 1, p.err, kErrWaitTmaEmpty))
                    return false;
                const uint32_t vb = smem_u32(&bars->v_full[st]);
                mbar_arrive_expect_tx(vb, S::kKvBytes);
#pragma unroll
                for (int sub = 0; sub < S::kSub; ++sub)
                    tma_load_4d(smem_u32(sV + st * S::kKvBytes + sub * S::kKvSubBytes), &p.tv, vb, sub * 64, v_kvh,
                                v_key0, v_b);
                ++gv;
                return true;
            };
            for (int r = 0; r < n_rounds && ok; ++r) {
                const int k = item1_index(r);
                if (k >= n_items) break;
                const Item1 it = item1_geometry<BN>(p, k);
                if (it.n_tiles == 0) continue;
                if (gv < g && !(ok = load_v())) break;
                // this item's Q overwrites the last one's: wait for its final S MMA
                if (qit > 0 && !(ok = mbar_wait(smem_u32(&bars->q_empty), (qit - 1) & 1, p.err, kErrWaitTmaEmpty)))
                    break;
                const uint32_t qb = smem_u32(&bars->q_full);
                mbar_arrive_expect_tx(qb, S::kQBytes);
#pragma unroll
                for (int sub = 0; sub < S::kSub; ++sub)   // box: 64 columns x pack heads x 128/pack positions
                    tma_load_4d(smem_u32(sQ + sub * S::kQSubBytes), &p.tq, qb, sub * 64, it.h, it.q0 / p.pack, it.b);
                ++qit;
                const int kvh = it.h / p.group;
                for (int j = 0; j < it.n_tiles; ++j, ++g) {
                    const int st = g & 1;
                    const int key0 = it.lo_min + j * BN;
                    if (g >= 2 &&
                        !(ok = mbar_wait(smem_u32(&bars->k_empty[st]), ((g >> 1) - 1) & 1, p.err, kErrWaitTmaEmpty)))
                        break;
                    const uint32_t kb = smem_u32(&bars->k_full[st]);
                    mbar_arrive_expect_tx(kb, S::kKvBytes);
#pragma unroll
                    for (int sub = 0; sub < S::kSub; ++sub)
                        tma_load_4d(smem_u32(sK + st * S::kKvBytes + sub * S::kKvSubBytes), &p.tk, kb, sub * 64,
                                    kvh, key0, it.b);
                    if (gv < g && !(ok = load_v())) break;
                    v_kvh = kvh;
                    v_key0 = key0;
                    v_b = it.b;
                }
            }
            if (ok && gv < g) load_v();
            // Drain: whatever was issued must land before the CTA can exit.
            if (qit > 0) mbar_wait(smem_u32(&bars->q_full), (qit - 1) & 1, p.err, kErrDrain);
            for (int j = max(0, g - 2); j < g; ++j)
                if (!mbar_wait(smem_u32(&bars->k_full[j & 1]), (j >> 1) & 1, p.err, kErrDrain)) break;
            for (int j = max(0, gv - 2); j < gv; ++j)
                if (!mbar_wait(smem_u32(&bars->v_full[j & 1]), (j >> 1) & 1, p.err, kErrDrain)) break;
        }
    } else if (warp == kMmaWarp) {
        // ================= tcgen05 issuer: the whole warp, converged; one elected
        // lane issues each MMA and commit =================
        {
            constexpr uint32_t idesc_s = umma_idesc_f16(kBM, BN, true, false);
            constexpr uint32_t idesc_pv = umma_idesc_f16(kBM, HD, false, true);
            const uint32_t q_addr = smem_u32(sQ);
            int oit = 0;   // items with key tiles issued so far
            // O += P(g) V(g); `first` starts the accumulation of an item, which overwrites O:
            // the epilogue warps must have read the previous item's O first
            auto issue_pv = [&](int g, bool first) -> bool {
                const int st = g & 1;
                if (first && oit > 0 &&
                    !mbar_wait_warp(smem_u32(&bars->o_free), (oit - 1) & 1, p.err, kErrWaitSoftmax))
                    return false;
                if (!mbar_wait_warp(smem_u32(&bars->p_full[st]), (g >> 1) & 1, p.err, kErrWaitSoftmax)) return false;
                if (!mbar_wait_warp(smem_u32(&bars->v_full[st]), (g >> 1) & 1, p.err, kErrWaitTmaFull)) return false;
                tc_fence_after();
                const uint32_t v_addr = smem_u32(sV + st * S::kKvBytes);
                const uint32_t p_col = tmem + (st ? S::kTmS1 : S::kTmS0);
#pragma unroll
                for (int kk = 0; kk < BN / 16; ++kk) {
                    const uint64_t bdesc = umma_sdesc_sw128(v_addr + kk * 16 * 128, S::kKvSubBytes, 1024);
                    umma_ts_elect(tmem + S::kTmO, p_col + kk * 8, bdesc, idesc_pv, (!first || kk > 0) ? 1u : 0u);
                }
                umma_commit_elect(smem_u32(&bars->o_done));
                umma_commit_elect(smem_u32(&bars->v_empty[st]));
                return true;
            };
            int qit = 0, g0 = 0;
            bool ok = true;
            for (int r = 0; r < n_rounds && ok; ++r) {
                const int k = item1_index(r);
                if (k >= n_items) break;
                const Item1 it = item1_geometry<BN>(p, k);
                const int n = it.n_tiles;
                if (n == 0) continue;
                ok = mbar_wait_warp(smem_u32(&bars->q_full), qit & 1, p.err, kErrWaitTmaFull);
                for (int j = 0; j < n && ok; ++j) {
                    const int g = g0 + j;
                    const int st = g & 1;
                    if (!(ok = mbar_wait_warp(smem_u32(&bars->k_full[st]), (g >> 1) & 1, p.err, kErrWaitTmaFull))) break;
                    tc_fence_after();
                    const uint32_t k_addr = smem_u32(sK + st * S::kKvBytes);
                    const uint32_t s_col = tmem + (st ? S::kTmS1 : S::kTmS0);
#pragma unroll
                    for (int kk = 0; kk < HD / 16; ++kk) {
                        const uint32_t off = (kk & 3) * 32;   // 16 halves = 32 B along K
                        const uint64_t adesc = umma_sdesc_sw128(q_addr + (kk >> 2) * S::kQSubBytes + off, 16, 1024);
                        const uint64_t bdesc = umma_sdesc_sw128(k_addr + (kk >> 2) * S::kKvSubBytes + off, 16, 1024);
                        umma_ss_elect(s_col, adesc, bdesc, idesc_s, kk > 0 ? 1u : 0u);
                    }
                    umma_commit_elect(smem_u32(&bars->s_full[st]));
                    umma_commit_elect(smem_u32(&bars->k_empty[st]));
                    if (j + 1 == n) umma_commit_elect(smem_u32(&bars->q_empty));   // the item's last S read Q
                    if (j >= 1 && !(ok = issue_pv(g - 1, j == 1))) break;
                }
                if (ok) ok = issue_pv(g0 + n - 1, n == 1);
                if (ok) umma_commit_elect(smem_u32(&bars->o_final));
                g0 += n;
                ++qit;
                ++oit;
            }
            // Every MMA must be complete before TMEM is released.
            umma_commit_elect(smem_u32(&bars->mma_done));
            mbar_wait_warp(smem_u32(&bars->mma_done), 0, p.err, kErrDrain);
        }
    } else if (warp < kProducerWarp) {
        // ================= softmax: thread owns query row `row` =================
        // tcgen05.ld / tcgen05.st are warp-collective, so every branch around them is
        // made warp-uniform (votes) and per-row decisions only select values.
        const uint32_t lane_base = tmem + (static_cast<uint32_t>(warp * 32) << 16);
        const float cap = p.softcap;
        const float inv_cap = cap > 0.f ? 1.f / cap : 0.f;
        const float kLog2e = 1.4426950408889634f;
        int g0 = 0, oit = 0;
        bool ok = true;
        for (int r = 0; r < n_rounds && ok; ++r) {
            const int k = item1_index(r);
            if (k >= n_items) break;
            const Item1 it = item1_geometry<BN>(p, k);
            const int n_tiles = it.n_tiles;
            const int vrow = it.q0 + static_cast<int>(threadIdx.x);   // packed row of this thread
            const int row = vrow / p.pack;                            // its position
            const int head = it.h + vrow % p.pack;
            const bool row_valid = row < p.seq_q;
            int my_lo = 0, my_hi = 0;
            bool my_written = false;
            if (row_valid) row_range(p, row, my_lo, my_hi, my_written);
            float m = -INFINITY;   // running maximum in log2 units
            float l = 0.f;
            for (int j = 0; j < n_tiles; ++j) {
                const int g = g0 + j;
                const int st = g & 1;
                ok = __all_sync(0xffffffffu,
                                mbar_wait(smem_u32(&bars->s_full[st]), (g >> 1) & 1, p.err, kErrWaitMma));
                if (!ok) break;
                tc_fence_after();
                const uint32_t s_col = lane_base + (st ? S::kTmS1 : S::kTmS0);
                float t[BN];
                {
                    // all column groups in flight before one wait
                    uint32_t rr[BN / 32][32];
#pragma unroll
                    for (int c = 0; c < BN / 32; ++c) tmem_ld32(s_col + c * 32, rr[c]);
                    tmem_ld_wait();
#pragma unroll
                    for (int c = 0; c < BN / 32; ++c)
#pragma unroll
                        for (int i = 0; i < 32; ++i) t[c * 32 + i] = __uint_as_float(rr[c][i]);
                }
                const int key0 = it.lo_min + j * BN;
                const bool full_tile = row_valid && key0 >= my_lo && key0 + BN <= my_hi;
                if (cap > 0.f) {   // softcapped scores in log2 units; raw scores are scaled below
#pragma unroll
                    for (int c = 0; c < BN; ++c) t[c] = cap * tanhf(t[c] * p.scale * inv_cap) * kLog2e;
                }
                if (!full_tile) {
#pragma unroll
                    for (int c = 0; c < BN; ++c) {
                        const int key = key0 + c;
                        if (!row_valid || key < my_lo || key >= my_hi) t[c] = -INFINITY;
                    }
                }
                // Row max (log2 units) as 8 independent chains of 3-input maxima and a short tree.
                auto row_max_log2 = [&]() -> float {
                    float pm[8];
#pragma unroll
                    for (int q = 0; q < 8; ++q) pm[q] = fmaxf(t[2 * q], t[2 * q + 1]);
#pragma unroll
                    for (int c = 16; c < BN; c += 16)
#pragma unroll
                        for (int q = 0; q < 8; ++q) pm[q] = max3f(pm[q], t[c + 2 * q], t[c + 2 * q + 1]);
                    const float mx =
                        max3f(max3f(pm[0], pm[1], pm[2]), max3f(pm[3], pm[4], pm[5]), fmaxf(pm[6], pm[7]));
                    return cap > 0.f ? mx : mx * p.scale_log2;
                };
                // The reference point m of the exponentials: a row that has none yet (no
                // visible key so far) takes this tile's exact maximum; every other row keeps
                // its m until this tile's sum of exponentials passes 2^15 (then P would no
                // longer fit fp16), and only then takes the tile's maximum, rescales O and l
                // and recomputes.  Each decision depends on the row's own scores alone.
                const bool fresh = m == -INFINITY && row_valid && key0 < my_hi && key0 + BN > my_lo;
                if (__any_sync(0xffffffffu, fresh)) {
                    const float mxs = row_max_log2();
                    if (fresh) m = mxs;
                }
                // P = exp2(t*mul - m) as fp16 pairs over the first BN/2 columns of this S buffer,
                // one packed FMA per two scores.  A row with no visible key yet (m = -inf) has
                // every t at -inf, so with -m replaced by 0 its exponentials are exactly 0.
                const float mul = cap > 0.f ? 1.f : p.scale_log2;
                float lt = 0.f;   // this tile's row sum
#pragma unroll
                for (int pass = 0; pass < 2; ++pass) {
                    const float negm = m != -INFINITY ? -m : 0.f;
                    float acc0[4] = {0.f, 0.f, 0.f, 0.f}, acc1[4] = {0.f, 0.f, 0.f, 0.f};   // independent pair sums
                    {
                        uint32_t rr[32];
#pragma unroll
                        for (int c = 0; c < BN / 64; ++c) {
#pragma unroll
                            for (int i = 0; i < 32; ++i) {
                                float x0, x1;
                                fma2(x0, x1, t[c * 64 + 2 * i], t[c * 64 + 2 * i + 1], mul, mul, negm, negm);
                                const float e0 = fast_exp2(x0), e1 = fast_exp2(x1);
                                add2(acc0[i & 3], acc1[i & 3], acc0[i & 3], acc1[i & 3], e0, e1);
                                rr[i] = pack_f16x2(e0, e1);
                            }
                            tmem_st32(s_col + c * 32, rr);
                        }
                    }
                    lt = ((acc0[0] + acc0[1]) + (acc0[2] + acc0[3])) + ((acc1[0] + acc1[1]) + (acc1[2] + acc1[3]));
                    const bool over = !(lt <= kSpecSumLimit);   // also NaN / inf
                    if (pass == 1 || !__any_sync(0xffffffffu, over)) break;
                    // O holds P_0..P_{j-1} V: wait for the item's previous PV, then rescale the
                    // rows that move their reference; the other rows recompute the same P.
                    const float mxs = row_max_log2();
                    const float f = over ? fast_exp2(m - mxs) : 1.f;
                    if (over) m = mxs;
                    if (j > 0) {
                        ok = __all_sync(0xffffffffu,
                                        mbar_wait(smem_u32(&bars->o_done), (g - 1) & 1, p.err, kErrWaitMma));
                        if (!ok) break;
                        tc_fence_after();
                        uint32_t ro[32];
#pragma unroll
                        for (int c = 0; c < HD / 32; ++c) {
                            tmem_ld32(lane_base + S::kTmO + c * 32, ro);
                            tmem_ld_wait();
#pragma unroll
                            for (int i = 0; i < 32; ++i) ro[i] = __float_as_uint(__uint_as_float(ro[i]) * f);
                            tmem_st32(lane_base + S::kTmO + c * 32, ro);
                        }
                    }
                    l *= f;
                    tmem_st_wait();
                }
                if (!ok) break;
                l += lt;
                // the item's row sums for the epilogue warps (read after the last PV, which
                // waits for this arrival)
                if (j + 1 == n_tiles) tmem_st1(lane_base + S::kTmL + (oit & 1), __float_as_uint(l));
                tmem_st_wait();
                tc_fence_before();
                mbar_arrive(smem_u32(&bars->p_full[st]));
            }
            if (!ok) break;
            if (n_tiles > 0) ++oit;
            g0 += n_tiles;
        }
    } else {
        // ================= epilogue: O / l -> out, rows of TMEM lane quarter warp % 4 =================
        const int quarter = warp % 4;
        const uint32_t lane_base = tmem + (static_cast<uint32_t>(quarter * 32) << 16);
        bool stores_pending = false;   // lane 0: a TMA store from this warp's staging area
        int slot = 0;                  // staging slot of the warp's next box (alternates across items)
        int oit = 0;
        bool ok = true;
        for (int r = 0; r < n_rounds && ok; ++r) {
            const int k = item1_index(r);
            if (k >= n_items) break;
            const Item1 it = item1_geometry<BN>(p, k);
            const int n_tiles = it.n_tiles;
            const int vrow = it.q0 + quarter * 32 + lane;   // packed row of this thread
            const int row = vrow / p.pack;                 // its position
            const int head = it.h + vrow % p.pack;
            const bool row_valid = row < p.seq_q;
            int my_lo = 0, my_hi = 0;
            bool my_written = false;
            if (row_valid) row_range(p, row, my_lo, my_hi, my_written);
            bool have_o = n_tiles > 0;
            float inv = 0.f;
            if (have_o) {
                have_o = ok =
                    __all_sync(0xffffffffu, mbar_wait(smem_u32(&bars->o_final), oit & 1, p.err, kErrWaitMma));
                if (ok) {
                    tc_fence_after();
                    uint32_t lv;
                    tmem_ld1(lane_base + S::kTmL + (oit & 1), lv);
                    tmem_ld_wait();
                    const float l = __uint_as_float(lv);
                    inv = l > 0.f ? 1.f / l : 0.f;
                }
            }
            // Staged epilogue: the warp's 32 rows (32/pack positions x pack heads) go through
            // shared memory in 128B-swizzled boxes and leave with TMA tensor stores, so the
            // output is written as whole sectors instead of 16-byte pieces of 32 rows.  The
            // warp's two box slots alternate: box k is written while the store of box k-1
            // still reads the other slot (one bulk group in flight).  Rows no window covers
            // must stay untouched: such warps store rows.
            const bool staged = ok && __all_sync(0xffffffffu, my_written || !row_valid);
            if (staged) {
                const bool bf = p.out_bf16 != 0;
                const int box_cols = bf ? 64 : 32;
                uint8_t *stage = smem + S::kOffStage + (warp - kEpiWarp0) * S::kStageWarpBytes;
                const int pos0 = (it.q0 + quarter * 32) / p.pack;
                for (int c0 = 0; c0 < HD; c0 += box_cols, slot ^= 1) {   // one box per round
                    if (c0 >= p.hd) break;                                 // boxes wholly past the head dim
                    if (lane == 0 && stores_pending) bulk_wait_read1();    // this slot's last store read it
                    __syncwarp();
                    for (int c = c0; c < c0 + box_cols; c += 32) {         // 32 TMEM columns at a time
                        uint32_t rr[32];
                        if (have_o) {
                            tmem_ld32(lane_base + S::kTmO + c, rr);
                            tmem_ld_wait();
                        } else {
#pragma unroll
                            for (int i = 0; i < 32; ++i) rr[i] = 0u;
                        }
                        uint8_t *box = stage + slot * (32 * 128);
                        if (bf) {
                            const int u0 = ((c - c0) % 64) / 8;   // first 16-byte unit of these columns
#pragma unroll
                            for (int u = 0; u < 4; ++u) {
                                uint4 v;
                                v.x = pack_bf16x2(__uint_as_float(rr[8 * u]) * inv, __uint_as_float(rr[8 * u + 1]) * inv);
                                v.y = pack_bf16x2(__uint_as_float(rr[8 * u + 2]) * inv,
                                                  __uint_as_float(rr[8 * u + 3]) * inv);
                                v.z = pack_bf16x2(__uint_as_float(rr[8 * u + 4]) * inv,
                                                  __uint_as_float(rr[8 * u + 5]) * inv);
                                v.w = pack_bf16x2(__uint_as_float(rr[8 * u + 6]) * inv,
                                                  __uint_as_float(rr[8 * u + 7]) * inv);
                                *reinterpret_cast<uint4 *>(box + sw128_offset(lane, u0 + u)) = v;
                            }
                        } else {
#pragma unroll
                            for (int q = 0; q < 8; ++q) {
                                float4 v = make_float4(__uint_as_float(rr[4 * q]) * inv,
                                                       __uint_as_float(rr[4 * q + 1]) * inv,
                                                       __uint_as_float(rr[4 * q + 2]) * inv,
                                                       __uint_as_float(rr[4 * q + 3]) * inv);
                                *reinterpret_cast<float4 *>(box + sw128_offset(lane, q)) = v;
                            }
                        }
                    }
                    fence_proxy_async_smem();
                    __syncwarp();
                    if (lane == 0) {
                        tma_store_4d(&p.to, smem_u32(stage + slot * (32 * 128)), c0, it.h, pos0, it.b);
                        bulk_commit();
                        stores_pending = true;
                    }
                    __syncwarp();
                }
            } else if (ok) {
                const bool store = row_valid && my_written;
                const long long orow = static_cast<long long>(it.b) * p.out_batch_stride +
                                       static_cast<long long>(store ? row : 0) * p.out_row_stride +
                                       static_cast<long long>(head) * p.hd;
                uint32_t rr[32];
#pragma unroll
                for (int c = 0; c < HD / 32; ++c) {
                    if (have_o) {
                        tmem_ld32(lane_base + S::kTmO + c * 32, rr);
                        tmem_ld_wait();
                    } else {
#pragma unroll
                        for (int i = 0; i < 32; ++i) rr[i] = 0u;
                    }
                    if (store && c * 32 < p.hd)
                        store_row32(p.out, orow + c * 32, rr, inv, p.out_bf16 != 0, min(32, p.hd - c * 32));
                }
            }
            if (have_o) {   // every read of O has completed (tcgen05.wait::ld after each)
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(smem_u32(&bars->o_free));
                ++oit;
            }
        }
        if (lane == 0 && stores_pending) bulk_wait_read0();   // staging read before the CTA exits
        __syncwarp();
    }

    tc_fence_before();
    __syncthreads();
    if (warp == kMmaWarp) {
        tc_fence_after();
        tmem_dealloc(tmem, S::kTmCols);
    }
}

// ===========================================================================
// v2: two 128-row query tiles per CTA (head dims 64 and 128)
// ===========================================================================
// Tile pairing: for GQA groups of even size the two tiles are the same rows of two
// Q heads that share a KV head (identical key ranges); otherwise two consecutive
// row blocks of one head.  Warps 0-3 run the softmax of tile 0, warps 4-7 that of
// tile 1, warp 8 is the TMA producer, warp 9 allocates TMEM and issues MMAs.
// TMEM: tile t owns columns [256t, 256t+128) for S/P and [256t+128, 256t+128+HD) for O.
// Registers: the block launches with 384 x 168; warps 8-11 give theirs back down to 88
// (setmaxnreg.dec) and the two softmax warpgroups take 208 each (setmaxnreg.inc):
// 128*88 + 256*208 = 64512 = 384*168, so the increase never waits on registers the
// block does not own.  The host checks the compiled count before every launch.
// The MMA order per key tile j ping-pongs the tiles so that the tensor pipe works on
// one tile while the other tile's softmax runs:
//   ... PV0(j)  S0(j+1)  PV1(j)  S1(j+1)  PV0(j+1) ...
constexpr int kThreads2 = 384;
constexpr int kProducerWarp2 = 8;
constexpr int kMmaWarp2 = 9;
constexpr int kRegsLaunch2 = 168;
constexpr int kRegsSoftmax2 = 208;
constexpr int kRegsOther2 = 88;
static_assert(128 * kRegsOther2 + 256 * kRegsSoftmax2 <= kThreads2 * kRegsLaunch2, "register split");

// Key tile (BN = 128) and K/V ring depth (2) are the same for head dims 64 and 128:
// TMEM holds S/P (128 columns) and O (head-dim columns) for each of the two Q tiles.
// Measured alternatives for head dim 64 (cfg 3): 64-key tiles with a 4-deep ring ran
// 14 % slower; a look-ahead variant with two S buffers per Q tile failed parity on
// B200 and was left out.
template <int HD>
struct Prefill2Shape {
    static constexpr int BN = 128;
    static constexpr int kNSB = 1;                         // S/P buffers per Q tile
    // K and V ring depth: 4 for head dim 64 (the rings, two Q tiles and the epilogue's
    // own staging fill 224 KB), 2 for head dim 128 (the 32 KB tiles leave no room)
    static constexpr int kStages = HD == 64 ? 4 : 2;
    static constexpr int kSub = HD / 64;
    static constexpr int kQSubBytes = kBM * 128;
    static constexpr int kQBytes = kSub * kQSubBytes;      // one tile
    static constexpr int kKvSubBytes = BN * 128;
    static constexpr int kKvBytes = kSub * kKvSubBytes;
    static constexpr int kOffQ = 0;
    static constexpr int kOffK = 2 * kQBytes;
    static constexpr int kOffV = kOffK + kStages * kKvBytes;
    // Epilogue staging of its own (8 softmax warps x 32 rows x HD fp32) where it fits
    // beside the rings (head dim 64); head dim 128 stages in the rings after the last item.
    static constexpr int kEpiBytes = 8 * 32 * HD * 4;
    static constexpr int kOffEpi = kOffV + kStages * kKvBytes;
    static constexpr bool kEpiOwn = kOffEpi + kEpiBytes + 512 + 1024 <= 227 * 1024;
    static constexpr int kOffBar = kOffEpi + (kEpiOwn ? kEpiBytes : 0);
    static constexpr int kUsed = kOffBar + 512 + 1024;
    static constexpr int kSmemBytes = kUsed > 118 * 1024 ? kUsed : 118 * 1024;
    static constexpr int kTileCols = 256;
    static constexpr int kTmO = BN;
    // Look-ahead (head dim 64): P gets its own 64 columns after O instead of overwriting
    // S, so S of the next key tile can be computed while the softmax still works on
    // this one (S 128 + O 64 + P 64 = 256 columns per Q tile).  Head dim 128 has no room
    // (S 128 + O 128) and writes P over the first half of S.
    static constexpr bool kLookAhead = HD == 64;
    static constexpr int kTmP = kLookAhead ? BN + HD : 0;
    static_assert(kTmO + HD <= kTileCols, "TMEM budget");
    static_assert(!kLookAhead || kTmP + BN / 2 <= kTileCols, "TMEM budget (P region)");
    static_assert(kStages * kKvBytes >= kBM * HD * 4, "epilogue staging must fit a K or V ring");
};

constexpr int kMaxStages2 = 4;
struct Barriers2 {
    uint64_t q_full, q_empty;
    uint64_t k_full[kMaxStages2], k_empty[kMaxStages2], v_full[kMaxStages2], v_empty[kMaxStages2];
    uint64_t s_full[2], p_full[2], o_done[2];
    uint64_t s_free[2];   // look-ahead: the softmax warps of a tile have read its S
    uint64_t mma_done;
    uint32_t tmem_base;
};


// Exponentials per row and key tile: PolyPairs8 of every 8 pairs go to the FMA-pipe
// polynomial, the rest to MUFU ex2.  Measured on cfg 3 (hd 64, 128 images x 12 layers,
// two runs each) with the row-maximum-free softmax: 1/8 8.07 ms, 2/8 8.21, 3/8 8.60 --
// the default for head dim 64 is 1/8.  Head dim 128 keeps all on MUFU (2/8 on the
// So400m attention: 23.6 ms against 22.7).  The share is a build-time knob.
#ifndef SMOL_POLY8_HD64
#define SMOL_POLY8_HD64 1
#endif
#ifndef SMOL_POLY8_HD128
#define SMOL_POLY8_HD128 0
#endif
template <int HD>
struct PolyShare {
    static constexpr int kPairs8 = HD == 64 ? SMOL_POLY8_HD64 : SMOL_POLY8_HD128;
};

// Work item k of a launch: (query block, head pair or head, batch element), query
// blocks fastest -- in decreasing order of work for causal-like masks -- so that the
// CTAs that run at the same time read the K and V of one (batch, KV head), which
// stays in L2 (at 32k keys it is 16 MB; spreading concurrent CTAs over many heads
// measured 8 % slower on cfg 5).  A persistent CTA takes the items of rounds
// r = 0, 1, ... at positions blockIdx.x (even rounds) and gridDim.x-1-blockIdx.x (odd
// rounds).
struct Item2 {
    int b, head[2], row0[2];
    int lo_min, n_tiles;   // key tiles [lo_min, lo_min + n_tiles*BN) cover every row's keys
};

__device__ __forceinline__ int item_index(const PrefillParams &p, int r)
{
    const int c = (r & 1) ? static_cast<int>(gridDim.x) - 1 - static_cast<int>(blockIdx.x)
                          : static_cast<int>(blockIdx.x);
    return r * static_cast<int>(gridDim.x) + c;
}

template <int BN>
__device__ __forceinline__ Item2 item_geometry(const PrefillParams &p, int k)
{
    Item2 it;
    const int qb = p.heavy_first ? p.n_qblocks - 1 - k % p.n_qblocks : k % p.n_qblocks;
    const int r = k / p.n_qblocks;
    const int y = r % p.n_ygroups;
    it.b = r / p.n_ygroups;
    if (p.pair_heads) {
        it.head[0] = 2 * y;
        it.head[1] = 2 * y + 1;
        it.row0[0] = it.row0[1] = qb * kBM;
    } else {
        it.head[0] = it.head[1] = y;
        it.row0[0] = qb * 2 * kBM;
        it.row0[1] = it.row0[0] + kBM;
    }
    // Rows of the block, clipped to the query range (and, for window masks, to the
    // rows some window covers).  Every mask's [lo, hi) is non-decreasing in the row,
    // so the first row gives the lowest key and the last row the highest.
    int a = it.row0[0];
    int z = min(it.row0[1] + kBM, p.seq_q) - 1;
    if (p.mask_kind == SMOL_MASK_WINDOWS) {
        a = max(a, p.window_starts[0]);
        z = min(z, p.window_starts[p.n_windows] - 1);
    }
    it.lo_min = 0;
    it.n_tiles = 0;
    if (z >= a) {
        int lo_a, hi_a, lo_z, hi_z;
        bool w;
        row_range(p, a, lo_a, hi_a, w);
        row_range(p, z, lo_z, hi_z, w);
        if (hi_z > lo_a) {
            it.lo_min = first_key_tile<BN>(p, lo_a);
            it.n_tiles = (hi_z - it.lo_min + BN - 1) / BN;
        }
    }
    return it;
}

// The TMA producer of the two-tile kernels (one thread): an item's two Q tiles, then
// its K and V tiles through the ST-deep rings.  Barrier phases run on across items:
// q_full / q_empty once per item with key tiles (count qit), the rings once per key
// tile (global count g over all items of this CTA).
template <typename S, typename Bars>
__device__ __forceinline__ void produce_two_tiles(const PrefillParams &p, Bars *bars, uint8_t *sQ, uint8_t *sK,
                                                  uint8_t *sV, int n_items, int n_rounds)
{
    constexpr int BN = S::BN;
    constexpr int ST = S::kStages;
    tma_prefetch_desc(&p.tq);
    tma_prefetch_desc(&p.tk);
    tma_prefetch_desc(&p.tv);
    int qit = 0, g = 0;
    bool ok = true;
    for (int r = 0; r < n_rounds && ok; ++r) {
        const int k = item_index(p, r);
        if (k >= n_items) break;
        const Item2 it = item_geometry<BN>(p, k);
        if (it.n_tiles == 0) continue;
        // Q of this item overwrites the last one's: wait for its final S MMAs.
        if (qit > 0 && !(ok = mbar_wait(smem_u32(&bars->q_empty), (qit - 1) & 1, p.err, kErrWaitTmaEmpty)))
            break;
        const uint32_t qbar = smem_u32(&bars->q_full);
        mbar_arrive_expect_tx(qbar, 2 * S::kQBytes);
#pragma unroll
        for (int t = 0; t < 2; ++t)
#pragma unroll
            for (int sub = 0; sub < S::kSub; ++sub)
                tma_load_4d(smem_u32(sQ + t * S::kQBytes + sub * S::kQSubBytes), &p.tq, qbar, sub * 64,
                            it.head[t], it.row0[t], it.b);
        ++qit;
        const int kvh = it.head[0] / p.group;
        for (int j = 0; j < it.n_tiles; ++j, ++g) {
            const int st = g % ST;
            const int key0 = it.lo_min + j * BN;
            if (g >= ST &&
                !(ok = mbar_wait(smem_u32(&bars->k_empty[st]), ((g / ST) - 1) & 1, p.err, kErrWaitTmaEmpty)))
                break;
            const uint32_t kb = smem_u32(&bars->k_full[st]);
            mbar_arrive_expect_tx(kb, S::kKvBytes);
#pragma unroll
            for (int sub = 0; sub < S::kSub; ++sub)
                tma_load_4d(smem_u32(sK + st * S::kKvBytes + sub * S::kKvSubBytes), &p.tk, kb, sub * 64,
                            kvh, key0, it.b);
            if (g >= ST &&
                !(ok = mbar_wait(smem_u32(&bars->v_empty[st]), ((g / ST) - 1) & 1, p.err, kErrWaitTmaEmpty)))
                break;
            const uint32_t vb = smem_u32(&bars->v_full[st]);
            mbar_arrive_expect_tx(vb, S::kKvBytes);
#pragma unroll
            for (int sub = 0; sub < S::kSub; ++sub)
                tma_load_4d(smem_u32(sV + st * S::kKvBytes + sub * S::kKvSubBytes), &p.tv, vb, sub * 64,
                            kvh, key0, it.b);
        }
    }
    // Drain: the last Q and the last ST key tiles must have landed before exit.
    if (qit > 0) mbar_wait(smem_u32(&bars->q_full), (qit - 1) & 1, p.err, kErrDrain);
    for (int j = max(0, g - ST); j < g; ++j) {
        if (!mbar_wait(smem_u32(&bars->k_full[j % ST]), (j / ST) & 1, p.err, kErrDrain)) break;
        if (!mbar_wait(smem_u32(&bars->v_full[j % ST]), (j / ST) & 1, p.err, kErrDrain)) break;
    }
}

template <int HD, bool Persistent, int PolyPairs8 = PolyShare<HD>::kPairs8>
__global__ void __launch_bounds__(kThreads2, 1) prefill2_kernel(const __grid_constant__ PrefillParams p)
{
    griddep_wait();   // programmatic launch: nothing of earlier kernels is read before this
    griddep_trigger();
    using S = Prefill2Shape<HD>;
    constexpr int BN = S::BN;
    constexpr int ST = S::kStages;
    static_assert(ST <= kMaxStages2 && S::kUsed <= 227 * 1024, "ring depth / shared memory");
    // One item per CTA (grid = items) unless Persistent: then rounds until items run out.
    const int n_items = p.n_qblocks * p.n_ygroups * p.batch;
    const int n_rounds = Persistent ? (n_items + static_cast<int>(gridDim.x) - 1) / static_cast<int>(gridDim.x) : 1;

    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    Barriers2 *bars = reinterpret_cast<Barriers2 *>(smem + S::kOffBar);
    const int warp = threadIdx.x / 32;
    const int lane = threadIdx.x % 32;

    if (threadIdx.x == 0) {
        mbar_init(smem_u32(&bars->q_full), 1);
        mbar_init(smem_u32(&bars->q_empty), 1);
        for (int s = 0; s < ST; ++s) {
            mbar_init(smem_u32(&bars->k_full[s]), 1);
            mbar_init(smem_u32(&bars->k_empty[s]), 1);
            mbar_init(smem_u32(&bars->v_full[s]), 1);
            mbar_init(smem_u32(&bars->v_empty[s]), 1);
        }
        for (int t = 0; t < 2; ++t) {
            mbar_init(smem_u32(&bars->s_full[t]), 1);
            mbar_init(smem_u32(&bars->p_full[t]), kSoftmaxThreads);
            mbar_init(smem_u32(&bars->o_done[t]), 1);
            mbar_init(smem_u32(&bars->s_free[t]), 4);   // one arrival per softmax warp
        }
        mbar_init(smem_u32(&bars->mma_done), 1);
        fence_mbar_init();
    }
    if (warp == kMmaWarp2) {
        tmem_alloc(smem_u32(&bars->tmem_base), 512);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = bars->tmem_base;

    uint8_t *sQ = smem + S::kOffQ;
    uint8_t *sK = smem + S::kOffK;
    uint8_t *sV = smem + S::kOffV;

    // Barrier phases run on across items: q_full / q_empty once per item with key
    // tiles (count qit), the K/V ring and s_full / p_full / o_done once per key tile
    // (global count g over all items of this CTA).
    if (warp >= 8) {
    // warpgroup 2 (producer, MMA issuer, two idle warps) hands registers to the softmax
    asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(kRegsOther2));
    if (warp == kProducerWarp2) {
        if (lane == 0) produce_two_tiles<S>(p, bars, sQ, sK, sV, n_items, n_rounds);
    } else if (warp == kMmaWarp2) {
        {   // the whole warp, converged: one elected lane issues each MMA and commit
            constexpr uint32_t idesc_s = umma_idesc_f16(kBM, BN, true, false);
            constexpr uint32_t idesc_pv = umma_idesc_f16(kBM, HD, false, true);
            // A shared-memory descriptor is linear in its address (bits [0,14) hold
            // address / 16, and every address here is below 256 KB), so each MMA's operand
            // descriptors are a per-tile base plus a compile-time constant.
            const uint64_t q_desc0 = umma_sdesc_sw128(smem_u32(sQ), 16, 1024);
            const uint64_t k_desc0 = umma_sdesc_sw128(smem_u32(sK), 16, 1024);
            const uint64_t v_desc0 = umma_sdesc_sw128(smem_u32(sV), S::kKvSubBytes, 1024);
            // S of Q tile t for global key tile g; K/V of key tile g sit in ring slot g % ST.
            auto issue_s = [&](int t, int g) {
                const uint64_t qd = q_desc0 + static_cast<uint32_t>(t * (S::kQBytes >> 4));
                const uint64_t kd = k_desc0 + static_cast<uint32_t>((g % ST) * (S::kKvBytes >> 4));
                const uint32_t s_col = tmem + t * S::kTileCols;
#pragma unroll
                for (int kk = 0; kk < HD / 16; ++kk) {
                    const uint32_t aoff = ((kk >> 2) * S::kQSubBytes + (kk & 3) * 32) >> 4;
                    const uint32_t boff = ((kk >> 2) * S::kKvSubBytes + (kk & 3) * 32) >> 4;
                    umma_ss_elect(s_col, qd + aoff, kd + boff, idesc_s, kk > 0 ? 1u : 0u);
                }
                umma_commit_elect(smem_u32(&bars->s_full[t]));
            };
            // O_t (+)= P_t V for key tile g; `first` starts the accumulation of an item.
            auto issue_pv = [&](int t, int g, bool first) {
                const uint64_t vd = v_desc0 + static_cast<uint32_t>((g % ST) * (S::kKvBytes >> 4));
                const uint32_t p_col = tmem + t * S::kTileCols + S::kTmP;
                const uint32_t o_col = tmem + t * S::kTileCols + S::kTmO;
#pragma unroll
                for (int kk = 0; kk < BN / 16; ++kk)
                    umma_ts_elect(o_col, p_col + kk * 8, vd + ((kk * 16 * 128) >> 4), idesc_pv,
                                  (!first || kk > 0) ? 1u : 0u);
                umma_commit_elect(smem_u32(&bars->o_done[t]));
            };
            auto wait_k = [&](int g) {
                return mbar_wait_warp(smem_u32(&bars->k_full[g % ST]), (g / ST) & 1, p.err, kErrWaitTmaFull);
            };
            int qit = 0, g0 = 0;
            bool ok = true;
            // Look-ahead order per key tile g: S0(g+1), S1(g+1) as soon as each tile's
            // softmax has read S(g) (s_free), then PV0(g), PV1(g) once P(g) is written.
            auto wait_s_free = [&](int t, int g) {   // softmax of tile t has read S(g)
                return g < 0 || mbar_wait_warp(smem_u32(&bars->s_free[t]), g & 1, p.err, kErrWaitSoftmax);
            };
            if constexpr (S::kLookAhead) {
                for (int r = 0; r < n_rounds && ok; ++r) {
                    const int k = item_index(p, r);
                    if (k >= n_items) break;
                    const Item2 it = item_geometry<BN>(p, k);
                    const int n = it.n_tiles;
                    if (n == 0) continue;
                    ok = mbar_wait_warp(smem_u32(&bars->q_full), qit & 1, p.err, kErrWaitTmaFull) && wait_k(g0);
                    for (int t = 0; t < 2 && ok; ++t) {
                        if (!(ok = wait_s_free(t, g0 - 1))) break;
                        tc_fence_after();
                        issue_s(t, g0);
                    }
                    if (!ok) break;
                    umma_commit_elect(smem_u32(&bars->k_empty[g0 % ST]));
                    if (n == 1) umma_commit_elect(smem_u32(&bars->q_empty));
                    for (int j = 0; j < n && ok; ++j) {
                        const int g = g0 + j;
                        if (j + 1 < n) {
                            if (!(ok = wait_k(g + 1))) break;
                            for (int t = 0; t < 2 && ok; ++t) {
                                if (!(ok = wait_s_free(t, g))) break;
                                tc_fence_after();
                                issue_s(t, g + 1);
                            }
                            if (!ok) break;
                            umma_commit_elect(smem_u32(&bars->k_empty[(g + 1) % ST]));
                            if (j + 2 == n) umma_commit_elect(smem_u32(&bars->q_empty));   // last S of the item
                        }
                        if (!(ok = mbar_wait_warp(smem_u32(&bars->v_full[g % ST]), (g / ST) & 1, p.err, kErrWaitTmaFull)))
                            break;
                        // O_t is overwritten by the item's first PV: its readers (the previous
                        // item's epilogue) are the threads whose p_full arrival that PV waits for.
                        for (int t = 0; t < 2 && ok; ++t) {
                            if (!(ok = mbar_wait_warp(smem_u32(&bars->p_full[t]), g & 1, p.err, kErrWaitSoftmax))) break;
                            tc_fence_after();
                            issue_pv(t, g, j == 0);
                        }
                        if (ok) umma_commit_elect(smem_u32(&bars->v_empty[g % ST]));
                    }
                    g0 += n;
                    ++qit;
                }
            }
            for (int r = 0; r < n_rounds && ok && !S::kLookAhead; ++r) {
                const int k = item_index(p, r);
                if (k >= n_items) break;
                const Item2 it = item_geometry<BN>(p, k);
                const int n = it.n_tiles;
                if (n == 0) continue;
                // Prologue: S of the item's first key tile for both Q tiles.  (The
                // previous item's last PV read P from the same TMEM columns; MMAs of
                // this thread run in issue order.)
                ok = mbar_wait_warp(smem_u32(&bars->q_full), qit & 1, p.err, kErrWaitTmaFull) && wait_k(g0);
                if (!ok) break;
                tc_fence_after();
                issue_s(0, g0);
                issue_s(1, g0);
                umma_commit_elect(smem_u32(&bars->k_empty[g0 % ST]));
                if (n == 1) umma_commit_elect(smem_u32(&bars->q_empty));
                // O_t is overwritten by the item's first PV: its readers (the previous
                // item's epilogue) are the threads whose p_full arrival that PV waits for.
                for (int j = 0; j < n && ok; ++j) {
                    const int g = g0 + j;
                    const int st = g % ST;
                    ok = mbar_wait_warp(smem_u32(&bars->p_full[0]), g & 1, p.err, kErrWaitSoftmax) &&
                         mbar_wait_warp(smem_u32(&bars->v_full[st]), (g / ST) & 1, p.err, kErrWaitTmaFull);
                    if (!ok) break;
                    tc_fence_after();
                    issue_pv(0, g, j == 0);
                    const bool more = j + 1 < n;   // S buffer of tile 0 is free again after PV0
                    if (more) {
                        ok = wait_k(g + 1);
                        if (!ok) break;
                        tc_fence_after();
                        issue_s(0, g + 1);
                    }
                    ok = mbar_wait_warp(smem_u32(&bars->p_full[1]), g & 1, p.err, kErrWaitSoftmax);
                    if (!ok) break;
                    tc_fence_after();
                    issue_pv(1, g, j == 0);
                    umma_commit_elect(smem_u32(&bars->v_empty[st]));
                    if (more) {
                        issue_s(1, g + 1);
                        umma_commit_elect(smem_u32(&bars->k_empty[(g + 1) % ST]));
                        if (j + 2 == n) umma_commit_elect(smem_u32(&bars->q_empty));   // last S of the item
                    }
                }
                g0 += n;
                ++qit;
            }
            umma_commit_elect(smem_u32(&bars->mma_done));
            mbar_wait_warp(smem_u32(&bars->mma_done), 0, p.err, kErrDrain);
        }
    }
    } else {
        asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(kRegsSoftmax2));
        // ================= softmax of tile `tile`, thread owns query row `row` =================
        const int tile = warp >> 2;
        const uint32_t lane_base = tmem + (static_cast<uint32_t>((warp & 3) * 32) << 16) + tile * S::kTileCols;
        const float cap = p.softcap;
        const float inv_cap = cap > 0.f ? 1.f / cap : 0.f;
        const float kLog2e = 1.4426950408889634f;
        const float sl2 = p.scale_log2;
        const uint32_t s_full = smem_u32(&bars->s_full[tile]);
        const uint32_t p_full = smem_u32(&bars->p_full[tile]);
        const uint32_t o_done = smem_u32(&bars->o_done[tile]);
        const uint32_t s_free = smem_u32(&bars->s_free[tile]);
        bool stores_pending = false;   // lane 0: a TMA store from this warp's staging area
        int g0 = 0;
        bool ok = true;
        int k = item_index(p, 0);
        Item2 it_cur = k < n_items ? item_geometry<BN>(p, k) : Item2{};
        for (int r = 0; r < n_rounds && ok; ++r) {
            if (k >= n_items) break;
            const Item2 it = it_cur;
            const int n_tiles = it.n_tiles;
            const int row = it.row0[tile] + (threadIdx.x & 127);
            const bool row_valid = row < p.seq_q;
            int my_lo = 0, my_hi = 0;
            bool my_written = false;
            if (row_valid) row_range(p, row, my_lo, my_hi, my_written);
            float m = -INFINITY;   // running maximum of score*scale*log2(e)
            float l = 0.f;
            for (int j = 0; j < n_tiles; ++j) {
                const int g = g0 + j;
                const uint32_t s_base = lane_base;                // S of this key tile
                const uint32_t p_base = lane_base + S::kTmP;      // P: its own columns, or over S
                ok = __all_sync(0xffffffffu, mbar_wait(s_full, g & 1, p.err, kErrWaitMma));
                if (!ok) break;
                tc_fence_after();
                float t[BN];
                {
                    // all column groups in flight before one wait
                    uint32_t rr[BN / 32][32];
#pragma unroll
                    for (int c = 0; c < BN / 32; ++c) tmem_ld32(s_base + c * 32, rr[c]);
                    tmem_ld_wait();
#pragma unroll
                    for (int c = 0; c < BN / 32; ++c)
#pragma unroll
                        for (int i = 0; i < 32; ++i) t[c * 32 + i] = __uint_as_float(rr[c][i]);
                }
                if constexpr (S::kLookAhead) {   // S is in registers: the next S may overwrite it
                    tc_fence_before();
                    __syncwarp();
                    if (lane == 0) mbar_arrive(s_free);
                }
                const int key0 = it.lo_min + j * BN;
                const bool full_tile = row_valid && key0 >= my_lo && key0 + BN <= my_hi;
                if (cap > 0.f) {
#pragma unroll
                    for (int c = 0; c < BN; ++c) t[c] = cap * tanhf(t[c] * p.scale * inv_cap) * kLog2e;
                }
                if (!full_tile) {
#pragma unroll
                    for (int c = 0; c < BN; ++c) {
                        const int key = key0 + c;
                        if (!row_valid || key < my_lo || key >= my_hi) t[c] = -INFINITY;
                    }
                }
                // Row max as 8 independent chains of 3-input maxima and a short tree (a single
                // chain over BN scores would serialise BN/2 dependent instructions), in log2
                // units (scores are raw, scale applied here, unless softcapped).
                auto row_max_log2 = [&]() -> float {
                    float pm[8];
#pragma unroll
                    for (int q = 0; q < 8; ++q) pm[q] = fmaxf(t[2 * q], t[2 * q + 1]);
#pragma unroll
                    for (int c = 16; c < BN; c += 16)
#pragma unroll
                        for (int q = 0; q < 8; ++q) pm[q] = max3f(pm[q], t[c + 2 * q], t[c + 2 * q + 1]);
                    const float mx =
                        max3f(max3f(pm[0], pm[1], pm[2]), max3f(pm[3], pm[4], pm[5]), fmaxf(pm[6], pm[7]));
                    return cap > 0.f ? mx : mx * sl2;
                };
                // The reference point m of the exponentials.  A row that has none yet (no
                // visible key so far) takes this tile's exact maximum.  Every other row keeps
                // its m and computes the exponentials straight away; the tile's sum then
                // tells whether any of them passed 2^15 (its scores grew by more than 15 in
                // log2 units), and only such a row takes the tile's maximum, rescales O and
                // l and recomputes.  A P value thus stays below 2^15 (fp16 holds it) and no
                // row pays for a row maximum on a tile whose scores did not jump.  Each
                // decision depends on the row's own scores alone, so a row's result does not
                // depend on which rows share its warp (a chunked prefill stays bit-exact).
                const bool fresh = m == -INFINITY && row_valid && key0 < my_hi && key0 + BN > my_lo;
                if (__any_sync(0xffffffffu, fresh)) {
                    const float mxs = row_max_log2();
                    if (fresh) m = mxs;
                }
                const float mul = cap > 0.f ? 1.f : sl2;
                float lt = 0.f;        // this tile's row sum
                bool p_free = true;    // look-ahead: PV(g-1) has read the P columns
#pragma unroll
                for (int pass = 0; pass < 2; ++pass) {   // unrolled: each pass scheduled on its own
                    // P = exp2(s*scale_log2 - m): one packed FMA per two scores, then ex2.
                    // A row with no visible key yet (m = -inf) has every score at -inf, so with
                    // -m replaced by 0 its exponentials are exactly 0: no per-element select.
                    const float negm = m != -INFINITY ? -m : 0.f;
                    float acc0[4] = {0.f, 0.f, 0.f, 0.f}, acc1[4] = {0.f, 0.f, 0.f, 0.f};   // 4 pair sums
                    uint32_t rr[32];
#pragma unroll
                    for (int c = 0; c < BN / 64; ++c) {
#pragma unroll
                        for (int i = 0; i < 32; ++i) {
                            float x0, x1, e0, e1;
                            fma2(x0, x1, t[c * 64 + 2 * i], t[c * 64 + 2 * i + 1], mul, mul, negm, negm);
                            if ((i & 7) < PolyPairs8) {   // this pair on the FMA pipe
                                exp2_poly2(x0, x1, e0, e1);
                            } else {                      // this pair on MUFU
                                e0 = fast_exp2(x0);
                                e1 = fast_exp2(x1);
                            }
                            add2(acc0[i & 3], acc1[i & 3], acc0[i & 3], acc1[i & 3], e0, e1);
                            rr[i] = pack_f16x2(e0, e1);
                        }
                        if constexpr (S::kLookAhead) {
                            // P(g-1) in the same columns is read by PV(g-1): wait for it only now,
                            // after half of this tile's exponentials (the first P of an item follows
                            // the previous item's epilogue, which waited for that item's last PV)
                            if (pass == 0 && c == 0 && j > 0) {
                                p_free = __all_sync(0xffffffffu, mbar_wait(o_done, (g - 1) & 1, p.err, kErrWaitMma));
                                tc_fence_after();
                            }
                        }
                        if (p_free) tmem_st32(p_base + c * 32, rr);
                    }
                    if (!p_free) break;
                    lt = ((acc0[0] + acc0[1]) + (acc0[2] + acc0[3])) + ((acc1[0] + acc1[1]) + (acc1[2] + acc1[3]));
                    const bool over = !(lt <= kSpecSumLimit);   // also NaN / inf
                    if (pass == 1 || !__any_sync(0xffffffffu, over)) break;
                    // Rows whose sum passed the limit: this tile's maximum becomes m; O (the
                    // earlier tiles' PV, complete: waited for above or, without look-ahead,
                    // before this S) and l are scaled by 2^(m_old - m_new).  The other rows
                    // recompute the same values.
                    const float mxs = row_max_log2();
                    const float f = over ? fast_exp2(m - mxs) : 1.f;
                    if (over) m = mxs;
                    if (j > 0) {
                        if (!(p_free = __all_sync(0xffffffffu, mbar_wait(o_done, (g - 1) & 1, p.err, kErrWaitMma))))
                            break;
                        tc_fence_after();
                        uint32_t ro[32];
#pragma unroll
                        for (int c = 0; c < HD / 32; ++c) {
                            tmem_ld32(lane_base + S::kTmO + c * 32, ro);
                            tmem_ld_wait();
#pragma unroll
                            for (int i = 0; i < 32; ++i) ro[i] = __float_as_uint(__uint_as_float(ro[i]) * f);
                            tmem_st32(lane_base + S::kTmO + c * 32, ro);
                        }
                    }
                    l *= f;
                    tmem_st_wait();
                }
                if (!p_free) {
                    ok = false;
                    break;
                }
                l += lt;
                tmem_st_wait();
                tc_fence_before();
                mbar_arrive(p_full);
            }
            if (!ok) break;
            // the next item's geometry while this item's last PV products run (its row
            // ranges stay at the top of the loop: computing them here measured slower)
            k = item_index(p, r + 1);
            if (k < n_items) it_cur = item_geometry<BN>(p, k);

            // ---- epilogue: O / l -> out (fp32) ----
            bool have_o = n_tiles > 0;
            if (have_o) {
                have_o = __all_sync(0xffffffffu, mbar_wait(o_done, (g0 + n_tiles - 1) & 1, p.err, kErrWaitMma));
                ok = have_o;
            }
            tc_fence_after();
            const float inv = l > 0.f ? 1.f / l : 0.f;
            const int head = it.head[tile];
            // Staged epilogue: this warp's 32 rows go through shared memory (128B-swizzled
            // 32 x 32 fp32 boxes) and leave with TMA tensor stores, so every output row is
            // written as whole sectors.  The staging area is the CTA's own when it fits
            // beside the rings (head dim 64); otherwise the K ring (tile 0) or V ring
            // (tile 1), which are free only after the CTA's last item (no load left, and
            // this tile's last PV completed after every S of the item).  Rows no window
            // covers must stay untouched, so warps holding one fall back to row stores.
            const bool last_item = !Persistent || item_index(p, r + 1) >= n_items;
            const bool staged = ok && (S::kEpiOwn || last_item) && __all_sync(0xffffffffu, my_written || !row_valid);
            if (staged) {
                uint8_t *stage = S::kEpiOwn ? smem + S::kOffEpi + warp * (32 * HD * 4)
                                            : (tile == 0 ? sK : sV) + (warp & 3) * (32 * HD * 4);
                if (lane == 0 && stores_pending) bulk_wait_read0();   // previous store read its staging
                __syncwarp();
                const bool bf = p.out_bf16 != 0;
                uint32_t rr[32];
#pragma unroll
                for (int c = 0; c < HD / 32; ++c) {
                    if (have_o) {
                        tmem_ld32(lane_base + S::kTmO + c * 32, rr);
                        tmem_ld_wait();
                    } else {
#pragma unroll
                        for (int i = 0; i < 32; ++i) rr[i] = 0u;
                    }
                    if (bf) {
                        // bf16 boxes are 64 columns (128 B) wide: columns [32c, 32c+32) are the
                        // 16-byte units 4(c%2) .. 4(c%2)+3 of box c/2
                        uint8_t *box = stage + (c / 2) * (32 * 128);
#pragma unroll
                        for (int u = 0; u < 4; ++u) {
                            uint4 v;
                            v.x = pack_bf16x2(__uint_as_float(rr[8 * u]) * inv, __uint_as_float(rr[8 * u + 1]) * inv);
                            v.y = pack_bf16x2(__uint_as_float(rr[8 * u + 2]) * inv,
                                              __uint_as_float(rr[8 * u + 3]) * inv);
                            v.z = pack_bf16x2(__uint_as_float(rr[8 * u + 4]) * inv,
                                              __uint_as_float(rr[8 * u + 5]) * inv);
                            v.w = pack_bf16x2(__uint_as_float(rr[8 * u + 6]) * inv,
                                              __uint_as_float(rr[8 * u + 7]) * inv);
                            *reinterpret_cast<uint4 *>(box + sw128_offset(lane, (c % 2) * 4 + u)) = v;
                        }
                    } else {
                        uint8_t *box = stage + c * (32 * 128);
#pragma unroll
                        for (int q = 0; q < 8; ++q) {
                            float4 v = make_float4(__uint_as_float(rr[4 * q]) * inv,
                                                   __uint_as_float(rr[4 * q + 1]) * inv,
                                                   __uint_as_float(rr[4 * q + 2]) * inv,
                                                   __uint_as_float(rr[4 * q + 3]) * inv);
                            *reinterpret_cast<float4 *>(box + sw128_offset(lane, q)) = v;
                        }
                    }
                }
                __syncwarp();
                if (p.n_more > 0) {
                    // Further destinations (a peer GPU's buffer over NVLink): the warp copies its
                    // 32 staged rows one row per instruction -- lane l takes 16-byte unit l of the
                    // row (unit u%8 of box u/8) -- so each store is a contiguous run of the row,
                    // not 32 scattered 16-byte pieces.
                    const int y0 = it.row0[tile] + (warp & 3) * 32;
                    const int lanes_per_row = bf ? HD / 8 : HD / 4;   // 16-byte units per row
                    const int rows_per_step = 32 / lanes_per_row;
                    const int sub = lane / lanes_per_row, u = lane % lanes_per_row;
                    const int elems = bf ? 8 : 4;                     // per 16-byte unit
                    for (int r0 = 0; r0 < 32; r0 += rows_per_step) {
                        const int rr_ = r0 + sub, grow = y0 + rr_;
                        if (grow >= p.seq_q) break;   // rows past the end exist only in the staging
                        const uint4 v = *reinterpret_cast<const uint4 *>(stage + (u / 8) * (32 * 128) +
                                                                         sw128_offset(rr_, u % 8));
                        const long long off = static_cast<long long>(it.b) * p.out_batch_stride +
                                              static_cast<long long>(grow) * p.out_row_stride +
                                              static_cast<long long>(head) * p.hd + u * elems;
                        const long long boff = off * (bf ? 2 : 4);
                        for (int o = 0; o < p.n_more; ++o)
                            *reinterpret_cast<uint4 *>(static_cast<uint8_t *>(p.out_more[o]) + boff) = v;
                    }
                }
                fence_proxy_async_smem();
                __syncwarp();
                if (lane == 0) {
                    const int y = it.row0[tile] + (warp & 3) * 32;
                    const int box_cols = bf ? 64 : 32;
                    for (int c = 0; c < HD / box_cols; ++c)
                        if (c * box_cols < p.hd)   // boxes wholly past the caller's head dim: none
                            tma_store_4d(&p.to, smem_u32(stage + c * (32 * 128)), c * box_cols, head, y, it.b);
                    bulk_commit();
                    stores_pending = true;
                }
                __syncwarp();
            } else if (ok) {
                const bool store = row_valid && my_written;
                uint32_t rr[32];
#pragma unroll
                for (int c = 0; c < HD / 32; ++c) {
                    if (have_o) {
                        tmem_ld32(lane_base + S::kTmO + c * 32, rr);
                        tmem_ld_wait();
                    } else {
#pragma unroll
                        for (int i = 0; i < 32; ++i) rr[i] = 0u;
                    }
                    if (store && c * 32 < p.hd) {
                        const long long off = static_cast<long long>(it.b) * p.out_batch_stride +
                                              static_cast<long long>(row) * p.out_row_stride +
                                              static_cast<long long>(head) * p.hd + c * 32;
                        const int nc = min(32, p.hd - c * 32);
                        store_row32(p.out, off, rr, inv, p.out_bf16 != 0, nc);
                        for (int o = 0; o < p.n_more; ++o)
                            store_row32(p.out_more[o], off, rr, inv, p.out_bf16 != 0, nc);
                    }
                }
            }
            g0 += n_tiles;
        }
        if (lane == 0 && stores_pending) bulk_wait_read0();
        __syncwarp();
    }

    tc_fence_before();
    __syncthreads();
    if (warp == kMmaWarp2) {
        tc_fence_after();
        tmem_dealloc(tmem, 512);
    }
}

// Key-tile height of the kernel that runs for a head dim (v1 for 256, v2 otherwise).
template <int HD>
struct KvTileRows {
    static constexpr int value = Prefill2Shape<HD>::BN;
};
template <>
struct KvTileRows<256> {
    static constexpr int value = PrefillShape<256>::BN;
};

// SMOL_PREFILL_PERSISTENT=1 in the environment makes head dim 128 persistent for every
// mask (measurement knob; head dim 64, and full / window masks, always are).
const bool g_prefill_persistent_all = [] {
    const char *e = getenv("SMOL_PREFILL_PERSISTENT");
    return e && e[0] == '1';
}();

int sm_count()
{
    int dev = 0, n = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) {
        cudaGetLastError();
        return 0;
    }
    return n;
}

// Once per device and instantiation: check the register count the in-kernel split is
// sized for (the block launches with kRegsLaunch2 per thread; any other build is
// refused) and raise the dynamic shared-memory limit.
template <int HD, bool Persistent>
int prepare_v2(int dev)
{
    static bool done[16] = {};
    if (dev < 0 || dev >= 16) return SMOL_B200_ERR_CUDA;
    if (done[dev]) return SMOL_B200_OK;
    cudaFuncAttributes fa;
    if (cudaFuncGetAttributes(&fa, prefill2_kernel<HD, Persistent>) != cudaSuccess) return SMOL_B200_ERR_CUDA;
    if (fa.numRegs != kRegsLaunch2) {
        char buf[128];
        snprintf(buf, sizeof(buf), "prefill2_kernel compiled with %d registers, expected %d", fa.numRegs,
                 kRegsLaunch2);
        set_error(SMOL_B200_ERR_CUDA, buf);
        return SMOL_B200_ERR_CUDA;
    }
    if (cudaFuncSetAttribute(prefill2_kernel<HD, Persistent>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             Prefill2Shape<HD>::kSmemBytes) != cudaSuccess)
        return SMOL_B200_ERR_CUDA;
    done[dev] = true;
    return SMOL_B200_OK;
}

template <int HD>
int launch_prefill(cudaStream_t st, void *out, int64_t out_row_stride, int64_t out_batch_stride,
                   const uint16_t *q, int64_t q_row_stride, int64_t q_batch_stride, const uint16_t *k,
                   int64_t k_row_stride, int64_t k_batch_stride, const uint16_t *v, int64_t v_row_stride,
                   int64_t v_batch_stride, int batch, int seq_q, int seq_k, int n_heads, int n_kv_heads,
                   float scale, int mask_kind, int q_offset, int prefix_len, int window, float softcap,
                   const int *window_starts, int n_windows, void *const *more_outs, int n_more, int out_bf16,
                   int hd)
{
    using S = PrefillShape<HD>;
    PrefillParams p;
    memset(&p, 0, sizeof(p));
    // A tensor map needs at least one row; with seq_k == 0 no key tile is ever loaded.
    const int kv_rows = seq_k > 0 ? seq_k : 1;
    const int64_t qb = batch > 1 ? q_batch_stride : static_cast<int64_t>(seq_q) * q_row_stride;
    const int64_t kb = batch > 1 ? k_batch_stride : static_cast<int64_t>(kv_rows) * k_row_stride;
    const int64_t vb = batch > 1 ? v_batch_stride : static_cast<int64_t>(kv_rows) * v_row_stride;
    // Every operand is described as (column, head, row, batch) with the caller's head dim
    // `hd` <= HD: the kernel's 64-column boxes past `hd` read zeros (outside the tensor),
    // which change no score and no output column, and its stores there are clipped or
    // skipped -- so a head dim such as SigLIP-So400m's 72 runs the 128-wide kernel without
    // a padded copy.  v1 (head dim 256) packs the heads of a KV group into the rows of a
    // query tile when the group is a power of two up to 32: each K/V tile then serves all
    // of them, and a short prefix fills whole tiles (MQA 8/1: 16 positions x 8 heads).
    const int group = n_heads / n_kv_heads;
    const int pack = (HD == 256 && group <= 32 && (group & (group - 1)) == 0) ? group : 1;
    // Q: box 64 columns x pack heads x 128/pack positions
    if (!make_tmap_4d(&p.tq, q, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, hd, n_heads, seq_q, batch, hd, q_row_stride, qb,
                      64, pack, kBM / pack))
        return SMOL_B200_ERR_CUDA;
    p.pack = pack;
    p.hd = hd;
    // K/V boxes are one key tile high: the tile height of the kernel that will run
    // (v1 for head dim 256, v2 otherwise) -- the producer's expect_tx counts on it.
    constexpr int kv_box_rows = KvTileRows<HD>::value;
    if (!make_tmap_4d(&p.tk, k, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, hd, n_kv_heads, kv_rows, batch, hd, k_row_stride,
                      kb, 64, 1, kv_box_rows) ||
        !make_tmap_4d(&p.tv, v, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, hd, n_kv_heads, kv_rows, batch, hd, v_row_stride,
                      vb, 64, 1, kv_box_rows))
        return SMOL_B200_ERR_CUDA;
    {
        // output boxes: 32 rows (32/pack positions x pack heads) x 128 bytes
        const int64_t ob = batch > 1 ? out_batch_stride : static_cast<int64_t>(seq_q) * out_row_stride;
        const bool ok = out_bf16 ? make_tmap_4d(&p.to, out, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, hd, n_heads, seq_q,
                                                batch, hd, out_row_stride, ob, 64, pack, 32 / pack)
                                 : make_tmap_4d(&p.to, out, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, hd, n_heads, seq_q,
                                                batch, hd, out_row_stride, ob, 32, pack, 32 / pack);
        if (!ok) return SMOL_B200_ERR_CUDA;
        p.out_bf16 = out_bf16 ? 1 : 0;
        p.n_more = n_more;
        for (int i = 0; i < n_more; ++i) p.out_more[i] = more_outs[i];
    }
    p.out = out;
    p.out_row_stride = out_row_stride;
    p.out_batch_stride = out_batch_stride;
    p.window_starts = window_starts;
    p.n_windows = n_windows;
    p.err = device_error_word();
    p.seq_q = seq_q;
    p.seq_k = seq_k;
    p.n_heads = n_heads;
    p.group = n_heads / n_kv_heads;
    p.mask_kind = mask_kind;
    p.q_offset = q_offset;
    p.prefix_len = prefix_len;
    p.window = window;
    p.scale = scale;
    p.scale_log2 = scale * 1.4426950408889634f;
    p.softcap = softcap;

    static bool attr_set[16] = {};
    int dev = 0;
    cudaGetDevice(&dev);
    if constexpr (HD == 256) {
        if (dev >= 0 && dev < 16 && !attr_set[dev]) {
            if (cudaFuncSetAttribute(prefill_kernel<HD>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     S::kSmemBytes) != cudaSuccess)
                return SMOL_B200_ERR_CUDA;
            attr_set[dev] = true;
        }
        // work items (query tile of packed rows, head group, batch), query tiles fastest;
        // persistent CTAs
        const long long rows = static_cast<long long>(seq_q) * pack;
        if (rows > 0x7fffffffLL - kBM) return SMOL_B200_ERR_ARGS;
        p.n_qblocks = static_cast<int>((rows + kBM - 1) / kBM);
        p.n_ygroups = n_heads / pack;
        p.batch = batch;
        p.heavy_first = (mask_kind == SMOL_MASK_CAUSAL || mask_kind == SMOL_MASK_PREFIX_LM) ? 1 : 0;
        const long long n_items = static_cast<long long>(p.n_qblocks) * p.n_ygroups * batch;
        if (n_items > 0x7fffffffLL) return SMOL_B200_ERR_ARGS;
        int grid = static_cast<int>(n_items);
        const int sms = sm_count();
        if (sms > 0 && grid > sms) grid = sms;
        if (launch_kernel(prefill_kernel<HD>, dim3(grid), dim3(kThreads), S::kSmemBytes, st, p) != cudaSuccess)
            return SMOL_B200_ERR_CUDA;
    } else {
        using S2 = Prefill2Shape<HD>;
        p.pair_heads = (p.group % 2 == 0) ? 1 : 0;
        p.n_qblocks = p.pair_heads ? (seq_q + kBM - 1) / kBM : (seq_q + 2 * kBM - 1) / (2 * kBM);
        p.n_ygroups = p.pair_heads ? n_heads / 2 : n_heads;
        p.batch = batch;
        // Query blocks of causal-like masks carry more keys the later they start.
        p.heavy_first = (mask_kind == SMOL_MASK_CAUSAL || mask_kind == SMOL_MASK_PREFIX_LM) ? 1 : 0;
        const long long n_items = static_cast<long long>(p.n_qblocks) * p.n_ygroups * batch;
        if (n_items > 0x7fffffffLL) return SMOL_B200_ERR_ARGS;
        // Persistent CTAs (one per SM) for head dim 64, where items are short and a
        // CTA's fill and drain would otherwise be exposed, and for head dim 128 when every
        // item has the same work (full and window masks: So400m attention 22.9 -> 22.2 ms);
        // causal-like masks at head dim 128 keep one CTA per item, whose heavy-first order
        // the hardware balances better than a static schedule (cfg 5: 14.2 against 15.4 ms).
        int grid = static_cast<int>(n_items);
        const bool uniform = mask_kind == SMOL_MASK_FULL || mask_kind == SMOL_MASK_WINDOWS;
        if (HD == 64 || uniform || g_prefill_persistent_all) {
            const int sms = sm_count();
            if (sms > 0 && grid > sms) grid = sms;
            const int rc = prepare_v2<HD, true>(dev);
            if (rc != SMOL_B200_OK) return rc;
            if (launch_kernel(prefill2_kernel<HD, true>, dim3(grid), dim3(kThreads2), S2::kSmemBytes, st, p) !=
                cudaSuccess)
                return SMOL_B200_ERR_CUDA;
        } else {
            const int rc = prepare_v2<HD, false>(dev);
            if (rc != SMOL_B200_OK) return rc;
            if (launch_kernel(prefill2_kernel<HD, false>, dim3(grid), dim3(kThreads2), S2::kSmemBytes, st, p) !=
                cudaSuccess)
                return SMOL_B200_ERR_CUDA;
        }
    }
    return cudaGetLastError() == cudaSuccess ? SMOL_B200_OK : SMOL_B200_ERR_CUDA;
}

}  // namespace

int prefill_attention(cudaStream_t st, void *out, int64_t out_row_stride, int64_t out_batch_stride,
                      const uint16_t *q, int64_t q_row_stride, int64_t q_batch_stride, const uint16_t *k,
                      int64_t k_row_stride, int64_t k_batch_stride, const uint16_t *v, int64_t v_row_stride,
                      int64_t v_batch_stride, int batch, int seq_q, int seq_k, int n_heads, int n_kv_heads,
                      int head_dim, float scale, int mask_kind, int q_offset, int prefix_len, int window,
                      float softcap, const int *window_starts, int n_windows, void *const *more_outs, int n_more,
                      int out_bf16)
{
    if (batch <= 0 || seq_q <= 0) return SMOL_B200_OK;
    // the kernel's head dim: 64, 128 or 256, the smallest that holds head_dim
    const int kernel_hd = head_dim <= 64 ? 64 : head_dim <= 128 ? 128 : 256;
    if (n_more < 0 || n_more > kMaxExtraOuts ||
        (n_more > 0 && (!more_outs || head_dim == 256 || head_dim != kernel_hd)))
        return SMOL_B200_ERR_ARGS;
    for (int i = 0; i < n_more; ++i)
        if (!more_outs[i] || (reinterpret_cast<uintptr_t>(more_outs[i]) & 15)) return SMOL_B200_ERR_ARGS;
    if (!out || !q || !k || !v || n_heads <= 0 || n_kv_heads <= 0 || n_heads % n_kv_heads != 0 || seq_k < 0 ||
        batch > 65535 || n_heads > 65535 || mask_kind < 0 || mask_kind > SMOL_MASK_FULL)
        return SMOL_B200_ERR_ARGS;
    if (mask_kind == SMOL_MASK_WINDOWS && (!window_starts || n_windows <= 0)) return SMOL_B200_ERR_ARGS;
    if (head_dim <= 0 || head_dim > 256 || head_dim % 8) return SMOL_B200_ERR_ARGS;   // 16-byte head rows
    const uintptr_t align = reinterpret_cast<uintptr_t>(q) | reinterpret_cast<uintptr_t>(k) |
                            reinterpret_cast<uintptr_t>(v) | reinterpret_cast<uintptr_t>(out);
    if (align & 15) return SMOL_B200_ERR_ARGS;
    if ((q_row_stride | k_row_stride | v_row_stride) & 7) return SMOL_B200_ERR_ARGS;
    if (batch > 1 && ((q_batch_stride | k_batch_stride | v_batch_stride) & 7)) return SMOL_B200_ERR_ARGS;
    // output rows and batches start on 16 bytes: 4 fp32 or 8 bf16 elements
    const int64_t out_align = out_bf16 ? 7 : 3;
    if ((out_row_stride & out_align) || (batch > 1 && (out_batch_stride & out_align))) return SMOL_B200_ERR_ARGS;
    if (q_row_stride < static_cast<int64_t>(n_heads) * head_dim ||
        k_row_stride < static_cast<int64_t>(n_kv_heads) * head_dim ||
        v_row_stride < static_cast<int64_t>(n_kv_heads) * head_dim)
        return SMOL_B200_ERR_ARGS;
#define SMOL_PREFILL_ARGS                                                                                      \
    st, out, out_row_stride, out_batch_stride, q, q_row_stride, q_batch_stride, k, k_row_stride, k_batch_stride, \
        v, v_row_stride, v_batch_stride, batch, seq_q, seq_k, n_heads, n_kv_heads, scale,      \
        mask_kind, q_offset, prefix_len, window, softcap, window_starts, n_windows, more_outs, n_more, out_bf16, \
        head_dim
    // the kernels wait (griddepcontrol.wait) before reading anything, so they may launch
    // while the stream's previous kernel finishes
    PdlScope pdl(g_api_pdl);
    switch (kernel_hd) {
    case 64: return launch_prefill<64>(SMOL_PREFILL_ARGS);
    case 128: return launch_prefill<128>(SMOL_PREFILL_ARGS);
    default: return launch_prefill<256>(SMOL_PREFILL_ARGS);
    }
#undef SMOL_PREFILL_ARGS
}

}  // namespace smolb200
