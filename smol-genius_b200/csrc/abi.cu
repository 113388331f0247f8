// abi.cu -- the extern "C" entry points of libsmol_b200.so (include/smol_b200.h).
//
// Part 1 keeps the reference signatures of common/kernels/smol_kernels.h.  Their
// callers pass fp32 buffers and read the result right after the call returns
// (qkn_decoder.c:506-531, siglip.c:126-128), so each call is synchronous.  Host
// buffers are staged through the device: activations are packed into head-padded
// bf16 (Q, K) and fp16 (V) rows, the tcgen05 / split-KV kernels run, and the fp32
// result is unpacked and copied back.  Device buffers are used in place.  There is
// no CPU compute path: without a usable device the call records
// SMOL_B200_ERR_NO_DEVICE, zero-fills `out` and returns.
#include <math.h>
#include <stdio.h>
#include <string.h>

#include <mutex>
#include <vector>

#include "b200_common.cuh"
#include "runtime.h"

using namespace smolb200;

namespace {

std::mutex g_legacy_mutex;   // the reference's pool is global and non-reentrant too

enum Slot { kSlotQ = 0, kSlotK, kSlotV, kSlotQp, kSlotKp, kSlotVp, kSlotOut, kSlotAux };

int pad_head_dim(int hd) { return hd <= 64 ? 64 : (hd <= 128 ? 128 : (hd <= 256 ? 256 : -1)); }

// Returns a device view of `n` floats at `p` (staged into `slot` when p is host memory).
const float *device_view(const float *p, size_t n, int slot, cudaStream_t st)
{
    if (n == 0) return static_cast<const float *>(legacy_scratch(slot, 16));
    if (is_device_pointer(p)) return p;
    float *d = static_cast<float *>(legacy_scratch(slot, n * sizeof(float)));
    if (!d) return nullptr;
    if (!cuda_check(cudaMemcpyAsync(d, p, n * sizeof(float), cudaMemcpyHostToDevice, st), "copy to device"))
        return nullptr;
    return d;
}

bool finish(cudaStream_t st)
{
    if (!cuda_check(cudaStreamSynchronize(st), "synchronize")) return false;
    unsigned *w = device_error_word();
    unsigned v = 0;
    if (w && cudaMemcpy(&v, w, sizeof(v), cudaMemcpyDeviceToHost) == cudaSuccess && v != 0) {
        if (v == kErrValueRange)
            set_error(SMOL_B200_ERR_RANGE, "a value does not fit the fp16 V format (|v| >= 65520)");
        else
            set_error(SMOL_B200_ERR_WATCHDOG, "device error word set by a kernel");
        return false;
    }
    return true;
}

void zero_host_or_device(float *out, size_t n)
{
    if (!out || n == 0) return;
    if (is_device_pointer(out)) {
        cudaMemset(out, 0, n * sizeof(float));
        cudaDeviceSynchronize();
    } else {
        memset(out, 0, n * sizeof(float));
    }
}

// Common body of every Part-1 attention entry point.
//   kv_heads_in_rows: heads per K/V row (n_kv_heads; n_heads for the MHA bidirectional form).
void legacy_attention(float *out, const float *Q, const float *K, const float *V, int seq_q, int seq_k,
                      int n_heads, int n_kv_heads, int head_dim, float scale, int mask_kind, int q_offset,
                      int window, float cap, const int *window_starts, int n_windows)
{
    if (seq_q <= 0 || n_heads <= 0 || head_dim <= 0) return;
    const size_t out_n = static_cast<size_t>(seq_q) * n_heads * head_dim;
    const int hdp = pad_head_dim(head_dim);
    if (n_kv_heads <= 0 || n_heads % n_kv_heads != 0 || hdp < 0 || seq_k < 0) {
        set_error(SMOL_B200_ERR_ARGS, "attention: unsupported shape");
        zero_host_or_device(out, out_n);
        return;
    }
    int row_lo = 0, row_hi = seq_q;   // rows written back
    if (mask_kind == SMOL_MASK_WINDOWS) {
        if (!window_starts || n_windows <= 0 || window_starts[0] < 0 || window_starts[n_windows] > seq_q) {
            set_error(SMOL_B200_ERR_ARGS, "bidirectional attention: bad window table");
            return;
        }
        for (int w = 0; w < n_windows; ++w)
            if (window_starts[w + 1] < window_starts[w]) {
                set_error(SMOL_B200_ERR_ARGS, "bidirectional attention: window table not sorted");
                return;
            }
        row_lo = window_starts[0];
        row_hi = window_starts[n_windows];
        if (row_hi <= row_lo) return;
    }
    std::lock_guard<std::mutex> lock(g_legacy_mutex);
    cudaStream_t st = legacy_stream();
    if (!st) {
        zero_host_or_device(out, out_n);
        return;
    }
    const int q_w = n_heads * head_dim, kv_w = n_kv_heads * head_dim;
    const int qp_w = n_heads * hdp, kvp_w = n_kv_heads * hdp;
    const float *dQ = device_view(Q, static_cast<size_t>(seq_q) * q_w, kSlotQ, st);
    const float *dK = device_view(K, static_cast<size_t>(seq_k) * kv_w, kSlotK, st);
    const float *dV = device_view(V, static_cast<size_t>(seq_k) * kv_w, kSlotV, st);
    uint16_t *Kp = static_cast<uint16_t *>(legacy_scratch(kSlotKp, static_cast<size_t>(seq_k > 0 ? seq_k : 1) * kvp_w * 2));
    uint16_t *Vp = static_cast<uint16_t *>(legacy_scratch(kSlotVp, static_cast<size_t>(seq_k > 0 ? seq_k : 1) * kvp_w * 2));
    float *Op = static_cast<float *>(legacy_scratch(kSlotOut, static_cast<size_t>(seq_q) * qp_w * sizeof(float)));
    if (!dQ || !dK || !dV || !Kp || !Vp || !Op) {
        zero_host_or_device(out, out_n);
        return;
    }
    int rc = launch_pack_rows(st, Kp, kvp_w, kvp_w, dK, kv_w, n_kv_heads, head_dim, hdp, seq_k, 0);
    if (rc == SMOL_B200_OK) rc = launch_pack_rows(st, Vp, kvp_w, kvp_w, dV, kv_w, n_kv_heads, head_dim, hdp, seq_k, 1);

    const bool decode = seq_q == 1 && mask_kind == SMOL_MASK_CAUSAL;
    if (rc == SMOL_B200_OK && decode) {
        // seq_q == 1: split-KV decode over keys [0, min(q_offset+1, seq_k)) (attention.c:94-96).
        int L = q_offset + 1;
        if (L > seq_k) L = seq_k;
        if (L < 0) L = 0;
        // fp32 Q keeps full precision (bf16 hi + lo split inside the kernel); pad it if needed.
        const float *qf = dQ;
        if (hdp != head_dim) {
            float *qpad = static_cast<float *>(legacy_scratch(kSlotQp, static_cast<size_t>(qp_w) * sizeof(float)));
            if (!qpad) rc = SMOL_B200_ERR_OOM;
            else {
                cudaMemsetAsync(qpad, 0, static_cast<size_t>(qp_w) * sizeof(float), st);
                cudaMemcpy2DAsync(qpad, hdp * sizeof(float), dQ, head_dim * sizeof(float), head_dim * sizeof(float),
                                  n_heads, cudaMemcpyDeviceToDevice, st);
                qf = qpad;
            }
        }
        const size_t ws = decode_workspace_bytes(1, L, n_heads, n_kv_heads, hdp);
        uint8_t *aux = static_cast<uint8_t *>(legacy_scratch(kSlotAux, 256 + ws));
        if (!aux) rc = SMOL_B200_ERR_OOM;
        if (rc == SMOL_B200_OK) {
            struct {
                int64_t row0;
                int len;
                int pad;
            } hdr = {0, L, 0};
            static_assert(sizeof(hdr) == 16, "index header");
            cudaMemcpyAsync(aux, &hdr, sizeof(hdr), cudaMemcpyHostToDevice, st);
            rc = decode_attention(st, Op, qf, 0, Kp, Vp, seq_k > 0 ? seq_k : 1, reinterpret_cast<int64_t *>(aux),
                                  reinterpret_cast<int *>(aux + 8), 1, L, n_heads, n_kv_heads, hdp, scale, window,
                                  cap, aux + 256, ws);
            // The host header must stay alive until the copy ran: synchronise here.
            cudaStreamSynchronize(st);
        }
    } else if (rc == SMOL_B200_OK) {
        uint16_t *Qp = static_cast<uint16_t *>(legacy_scratch(kSlotQp, static_cast<size_t>(seq_q) * qp_w * 2));
        int *dws = nullptr;
        if (!Qp) rc = SMOL_B200_ERR_OOM;
        if (rc == SMOL_B200_OK)
            rc = launch_pack_rows(st, Qp, qp_w, qp_w, dQ, q_w, n_heads, head_dim, hdp, seq_q, 0);
        if (rc == SMOL_B200_OK && mask_kind == SMOL_MASK_WINDOWS) {
            dws = static_cast<int *>(legacy_scratch(kSlotAux, sizeof(int) * (n_windows + 1)));
            if (!dws) rc = SMOL_B200_ERR_OOM;
            else
                cudaMemcpyAsync(dws, window_starts, sizeof(int) * (n_windows + 1), cudaMemcpyHostToDevice, st);
        }
        if (rc == SMOL_B200_OK)
            rc = prefill_attention(st, Op, qp_w, 0, Qp, qp_w, 0, Kp, kvp_w, 0, Vp, kvp_w, 0, 1, seq_q, seq_k, n_heads,
                                   n_kv_heads, hdp, scale, mask_kind, q_offset, 0, window, cap, dws, n_windows);
        if (mask_kind == SMOL_MASK_WINDOWS) cudaStreamSynchronize(st);   // window table copy source
    }
    if (rc != SMOL_B200_OK) {
        set_error(rc, "attention launch failed");
        cudaStreamSynchronize(st);
        zero_host_or_device(out, out_n);
        return;
    }
    // Unpack rows [row_lo, row_hi) back to the caller's [rows, n_heads*head_dim] layout.
    const int64_t nrows = row_hi - row_lo;
    const bool out_dev = is_device_pointer(out);
    float *dst = out_dev ? out + static_cast<int64_t>(row_lo) * q_w
                         : static_cast<float *>(legacy_scratch(kSlotQ, static_cast<size_t>(nrows) * q_w * sizeof(float)));
    if (!dst) {
        zero_host_or_device(out, out_n);
        return;
    }
    rc = launch_unpack_rows(st, dst, q_w, Op + static_cast<int64_t>(row_lo) * qp_w, qp_w, n_heads, head_dim, hdp,
                            nrows);
    if (rc == SMOL_B200_OK && !out_dev)
        cuda_check(cudaMemcpyAsync(out + static_cast<int64_t>(row_lo) * q_w, dst, static_cast<size_t>(nrows) * q_w * 4,
                                   cudaMemcpyDeviceToHost, st),
                   "copy result to host");
    // a kernel that reported through the device word (a wait that ran out, a V value fp16
    // cannot hold) leaves no trustworthy rows: the caller gets zeros, as for other failures
    if (!finish(st)) zero_host_or_device(out, out_n);
}

// In-place fp32 op on x (host or device): stage, run `fn` on the device copy, copy back.
template <typename Fn>
void inplace_rows(float *x, size_t n, Fn fn)
{
    if (!x || n == 0) return;
    std::lock_guard<std::mutex> lock(g_legacy_mutex);
    cudaStream_t st = legacy_stream();
    if (!st) return;
    const bool dev = is_device_pointer(x);
    float *dx = x;
    if (!dev) {
        dx = static_cast<float *>(legacy_scratch(kSlotQ, n * sizeof(float)));
        if (!dx || !cuda_check(cudaMemcpyAsync(dx, x, n * sizeof(float), cudaMemcpyHostToDevice, st), "copy to device"))
            return;
    }
    const int rc = fn(st, dx);
    if (rc != SMOL_B200_OK) {
        set_error(rc, "kernel launch failed");
        cudaStreamSynchronize(st);
        return;
    }
    if (!dev) cuda_check(cudaMemcpyAsync(x, dx, n * sizeof(float), cudaMemcpyDeviceToHost, st), "copy to host");
    finish(st);
}

// Host table builders (qkn_decoder.c:261-311, rope.c:12-66): the values come from
// the same libm calls as the reference, so they are bit-identical; the device
// kernels only ever index them.
void rope_table_host(float *cos_out, float *sin_out, const int *positions, int seq, int head_dim, float theta,
                     bool interleaved)
{
    const int half = head_dim / 2;
    for (int s = 0; s < seq; ++s) {
        const float pos = static_cast<float>(positions[s]);
        for (int d = 0; d < half; ++d) {
            const float freq = 1.0f / powf(theta, static_cast<float>(2 * d) / static_cast<float>(head_dim));
            const float a = pos * freq;
            const float c = cosf(a), sn = sinf(a);
            if (interleaved) {
                cos_out[s * head_dim + 2 * d] = c;
                cos_out[s * head_dim + 2 * d + 1] = c;
                sin_out[s * head_dim + 2 * d] = sn;
                sin_out[s * head_dim + 2 * d + 1] = sn;
            } else {
                cos_out[s * head_dim + d] = c;
                cos_out[s * head_dim + half + d] = c;
                sin_out[s * head_dim + d] = sn;
                sin_out[s * head_dim + half + d] = sn;
            }
        }
    }
}

// Writes a host-computed table to `dst`, which may be host or device memory.
void deliver(float *dst, const std::vector<float> &src)
{
    if (src.empty()) return;
    if (is_device_pointer(dst)) {
        if (cuda_check(cudaMemcpy(dst, src.data(), src.size() * sizeof(float), cudaMemcpyHostToDevice),
                       "copy table to device"))
            return;
    } else {
        memcpy(dst, src.data(), src.size() * sizeof(float));
    }
}

void compute_rope(float *cos_out, float *sin_out, const int *positions, int seq, int head_dim, float theta,
                  bool interleaved)
{
    if (seq <= 0 || head_dim <= 0 || !cos_out || !sin_out || !positions) return;
    std::vector<int> pos(seq);
    if (is_device_pointer(positions)) {
        if (!cuda_check(cudaMemcpy(pos.data(), positions, seq * sizeof(int), cudaMemcpyDeviceToHost), "copy positions"))
            return;
    } else {
        memcpy(pos.data(), positions, seq * sizeof(int));
    }
    const size_t n = static_cast<size_t>(seq) * head_dim;
    std::vector<float> c(n, 0.f), s(n, 0.f);
    if (is_device_pointer(cos_out)) {   // keep untouched odd tail elements as they were
        cudaMemcpy(c.data(), cos_out, n * sizeof(float), cudaMemcpyDeviceToHost);
        cudaMemcpy(s.data(), sin_out, n * sizeof(float), cudaMemcpyDeviceToHost);
    } else {
        memcpy(c.data(), cos_out, n * sizeof(float));
        memcpy(s.data(), sin_out, n * sizeof(float));
    }
    rope_table_host(c.data(), s.data(), pos.data(), seq, head_dim, theta, interleaved);
    deliver(cos_out, c);
    deliver(sin_out, s);
}

void apply_rope(float *x, const float *cos_vals, const float *sin_vals, int seq, int n_heads, int head_dim,
                int interleaved)
{
    if (seq <= 0 || n_heads <= 0 || head_dim <= 1) return;
    const size_t n = static_cast<size_t>(seq) * n_heads * head_dim;
    const size_t tn = static_cast<size_t>(seq) * head_dim;
    inplace_rows(x, n, [&](cudaStream_t st, float *dx) {
        const float *dc = device_view(cos_vals, tn, kSlotK, st);
        const float *ds = device_view(sin_vals, tn, kSlotV, st);
        if (!dc || !ds) return static_cast<int>(SMOL_B200_ERR_OOM);
        return launch_rope(st, dx, dc, ds, seq, n_heads, head_dim, interleaved);
    });
}

}  // namespace

extern "C" {

// ---------------------------------------------------------------------------
// Part 1
// ---------------------------------------------------------------------------
void smol_bidirectional_attention(float *out, const float *Q, const float *K, const float *V, int seq, int n_heads,
                                  int head_dim, float scale, const int *window_starts, int n_windows)
{
    legacy_attention(out, Q, K, V, seq, seq, n_heads, n_heads, head_dim, scale, SMOL_MASK_WINDOWS, 0, 0, 0.f,
                     window_starts, n_windows);
}

void smol_causal_attention(float *out, const float *Q, const float *K, const float *V, int seq_q, int seq_k,
                           int n_heads, int n_kv_heads, int head_dim, float scale, int q_offset)
{
    legacy_attention(out, Q, K, V, seq_q, seq_k, n_heads, n_kv_heads, head_dim, scale, SMOL_MASK_CAUSAL, q_offset, 0,
                     0.f, nullptr, 0);
}

void smol_sliding_window_attention(float *out, const float *Q, const float *K, const float *V, int seq_q, int seq_k,
                                   int n_heads, int n_kv_heads, int head_dim, float scale, int q_offset,
                                   int window_size)
{
    legacy_attention(out, Q, K, V, seq_q, seq_k, n_heads, n_kv_heads, head_dim, scale, SMOL_MASK_CAUSAL, q_offset,
                     window_size > 0 ? window_size : 0, 0.f, nullptr, 0);
}

void smol_causal_attention_softcap(float *out, const float *Q, const float *K, const float *V, int seq_q, int seq_k,
                                   int n_heads, int n_kv_heads, int head_dim, float scale, int q_offset, float cap)
{
    legacy_attention(out, Q, K, V, seq_q, seq_k, n_heads, n_kv_heads, head_dim, scale, SMOL_MASK_CAUSAL, q_offset, 0,
                     cap, nullptr, 0);
}

void smol_sliding_window_attention_softcap(float *out, const float *Q, const float *K, const float *V, int seq_q,
                                           int seq_k, int n_heads, int n_kv_heads, int head_dim, float scale,
                                           int q_offset, int window_size, float cap)
{
    legacy_attention(out, Q, K, V, seq_q, seq_k, n_heads, n_kv_heads, head_dim, scale, SMOL_MASK_CAUSAL, q_offset,
                     window_size > 0 ? window_size : 0, cap, nullptr, 0);
}

void smol_sinusoidal_pe(float *pe, int n_pos, int d_model)
{
    if (!pe || n_pos <= 0 || d_model <= 1) return;
    const int half = d_model / 2;
    const size_t n = static_cast<size_t>(n_pos) * d_model;
    std::vector<float> t(n, 0.f);
    if (is_device_pointer(pe)) cudaMemcpy(t.data(), pe, n * sizeof(float), cudaMemcpyDeviceToHost);
    else memcpy(t.data(), pe, n * sizeof(float));
    const float log_ts = logf(10000.0f) / static_cast<float>(half - 1);   // rope.c:14
    for (int p = 0; p < n_pos; ++p) {
        for (int d = 0; d < half; ++d) {
            const float inv_ts = expf(-static_cast<float>(d) * log_ts);
            const float a = static_cast<float>(p) * inv_ts;
            t[static_cast<size_t>(p) * d_model + d] = sinf(a);
            t[static_cast<size_t>(p) * d_model + half + d] = cosf(a);
        }
    }
    deliver(pe, t);
}

void smol_compute_rope_neox(float *cos_out, float *sin_out, const int *positions, int seq, int head_dim, float theta)
{
    compute_rope(cos_out, sin_out, positions, seq, head_dim, theta, false);
}

void smol_compute_rope_interleaved(float *cos_out, float *sin_out, const int *positions, int seq, int head_dim,
                                   float theta)
{
    compute_rope(cos_out, sin_out, positions, seq, head_dim, theta, true);
}

void smol_apply_rope_neox(float *x, const float *cos_vals, const float *sin_vals, int seq, int n_heads, int head_dim)
{
    apply_rope(x, cos_vals, sin_vals, seq, n_heads, head_dim, 0);
}

void smol_apply_rope_interleaved(float *x, const float *cos_vals, const float *sin_vals, int seq, int n_heads,
                                 int head_dim)
{
    apply_rope(x, cos_vals, sin_vals, seq, n_heads, head_dim, 1);
}

void smol_rms_norm_per_head(float *x, const float *weight, int seq_len, int n_heads, int head_dim, float eps)
{
    if (seq_len <= 0 || n_heads <= 0 || head_dim <= 0) return;
    const size_t n = static_cast<size_t>(seq_len) * n_heads * head_dim;
    inplace_rows(x, n, [&](cudaStream_t st, float *dx) {
        const float *dw = device_view(weight, head_dim, kSlotK, st);
        if (!dw) return static_cast<int>(SMOL_B200_ERR_OOM);
        return launch_rms_norm_per_head(st, dx, dw, seq_len, n_heads, head_dim, eps);
    });
}

void smol_rms_norm(float *out, const float *x, const float *weight, int seq_len, int hidden, float eps)
{
    if (seq_len <= 0 || hidden <= 0 || !out || !x) return;
    const size_t n = static_cast<size_t>(seq_len) * hidden;
    std::lock_guard<std::mutex> lock(g_legacy_mutex);
    cudaStream_t st = legacy_stream();
    if (!st) return;
    const float *dx = device_view(x, n, kSlotQ, st);
    const float *dw = device_view(weight, hidden, kSlotK, st);
    const bool out_dev = is_device_pointer(out);
    float *dout = out_dev ? out : static_cast<float *>(legacy_scratch(kSlotOut, n * sizeof(float)));
    if (!dx || !dw || !dout) return;
    int rc = launch_rms_norm(st, dout, dx, dw, seq_len, hidden, eps);
    if (rc != SMOL_B200_OK) {
        set_error(rc, "rms_norm launch failed");
        cudaStreamSynchronize(st);
        return;
    }
    if (!out_dev) cuda_check(cudaMemcpyAsync(out, dout, n * sizeof(float), cudaMemcpyDeviceToHost, st), "copy to host");
    finish(st);
}

// ---------------------------------------------------------------------------
// Part 3
// ---------------------------------------------------------------------------
static int record(int rc, const char *what)
{
    if (rc != SMOL_B200_OK) set_error(rc, what);
    return rc;
}

int smol_b200_qknorm_rope_append(void *stream, const float *q_in, const float *k_in, const float *v_in, int n_tokens,
                                 int n_heads, int n_kv_heads, int head_dim, const float *q_norm_w,
                                 const float *k_norm_w, float eps, const float *rope_cos, const float *rope_sin,
                                 int rope_interleaved, const int *positions, const int64_t *slots, float *q_out_f32,
                                 uint16_t *q_out_bf16, uint16_t *k_cache_bf16, uint16_t *v_cache_f16,
                                 int64_t cache_rows)
{
    return record(qknorm_rope_append(static_cast<cudaStream_t>(stream), q_in, k_in, v_in, n_tokens, n_heads,
                                     n_kv_heads, head_dim, q_norm_w, k_norm_w, eps, rope_cos, rope_sin,
                                     rope_interleaved, positions, slots, q_out_f32, q_out_bf16, k_cache_bf16,
                                     v_cache_f16, cache_rows),
                  "smol_b200_qknorm_rope_append");
}

int smol_b200_watchdog_selftest(void *stream)
{
    return record(launch_watchdog_selftest(static_cast<cudaStream_t>(stream)), "smol_b200_watchdog_selftest");
}

size_t smol_b200_decode_workspace_bytes(int n_seqs, int max_kv_len, int n_heads, int n_kv_heads, int head_dim)
{
    return decode_workspace_bytes(n_seqs, max_kv_len, n_heads, n_kv_heads, head_dim);
}

int smol_b200_decode_attention(void *stream, float *out, const void *q, int q_is_bf16, const uint16_t *k_pool,
                               const uint16_t *v_pool, int64_t pool_rows, const int64_t *seq_row0, const int *kv_len,
                               int n_seqs, int max_kv_len, int n_heads, int n_kv_heads, int head_dim, float scale,
                               int window, float softcap, void *workspace, size_t workspace_bytes)
{
    return record(decode_attention(static_cast<cudaStream_t>(stream), out, q, q_is_bf16, k_pool, v_pool, pool_rows,
                                   seq_row0, kv_len, n_seqs, max_kv_len, n_heads, n_kv_heads, head_dim, scale, window,
                                   softcap, workspace, workspace_bytes),
                  "smol_b200_decode_attention");
}

int smol_b200_prefill_attention(void *stream, float *out, int64_t out_row_stride, int64_t out_batch_stride,
                                const uint16_t *q, int64_t q_row_stride, int64_t q_batch_stride, const uint16_t *k,
                                int64_t k_row_stride, int64_t k_batch_stride, const uint16_t *v, int64_t v_row_stride,
                                int64_t v_batch_stride, int batch, int seq_q, int seq_k, int n_heads, int n_kv_heads,
                                int head_dim, float scale, int mask_kind, int q_offset, int prefix_len, int window,
                                float softcap, const int *window_starts, int n_windows)
{
    return record(prefill_attention(static_cast<cudaStream_t>(stream), out, out_row_stride, out_batch_stride, q,
                                    q_row_stride, q_batch_stride, k, k_row_stride, k_batch_stride, v, v_row_stride,
                                    v_batch_stride, batch, seq_q, seq_k, n_heads, n_kv_heads, head_dim, scale,
                                    mask_kind, q_offset, prefix_len, window, softcap, window_starts, n_windows),
                  "smol_b200_prefill_attention");
}

// Scratch layout of smol_b200_decode_step_host (256-byte aligned pieces).
struct StepLayout {
    size_t q, k, v, qr, out, pos, slot, next, ws, total;
};

static StepLayout step_layout(int n_seqs, int max_kv_len, int n_heads, int n_kv_heads, int head_dim)
{
    auto al = [](size_t x) { return (x + 255) & ~size_t(255); };
    StepLayout L;
    const size_t qn = static_cast<size_t>(n_seqs) * n_heads * head_dim * 4;
    const size_t kn = static_cast<size_t>(n_seqs) * n_kv_heads * head_dim * 4;
    size_t o = 0;
    L.q = o; o += al(qn);
    L.k = o; o += al(kn);
    L.v = o; o += al(kn);
    L.qr = o; o += al(qn);
    L.out = o; o += al(qn);
    L.pos = o; o += al(static_cast<size_t>(n_seqs) * 4);
    L.slot = o; o += al(static_cast<size_t>(n_seqs) * 8);
    L.next = o; o += al(static_cast<size_t>(n_seqs) * 4);
    L.ws = o; o += al(decode_workspace_bytes(n_seqs, max_kv_len + 1, n_heads, n_kv_heads, head_dim));
    L.total = o;
    return L;
}

size_t smol_b200_decode_step_scratch_bytes(int n_seqs, int max_kv_len, int n_heads, int n_kv_heads, int head_dim)
{
    if (n_seqs <= 0 || n_heads <= 0 || n_kv_heads <= 0 || head_dim <= 0) return 0;
    return step_layout(n_seqs, max_kv_len, n_heads, n_kv_heads, head_dim).total;
}

// SMOL_STEP_CHUNKS=n in the environment sets the number of sequence chunks of
// smol_b200_decode_step_host (measurement knob; 0 or unset: by batch size, at most 4,
// at most kMaxChunks).
static const int g_step_chunks = [] {
    const char *e = getenv("SMOL_STEP_CHUNKS");
    const int v = e ? atoi(e) : 0;
    return v > 0 ? (v < smolb200::StepPipe::kMaxChunks ? v : smolb200::StepPipe::kMaxChunks) : 0;
}();
// SMOL_STEP_WEIGHTS="w0,w1,..." (measurement knob): relative chunk sizes, one per chunk.
static const std::vector<int> g_step_weights = [] {
    std::vector<int> w;
    const char *e = getenv("SMOL_STEP_WEIGHTS");
    for (const char *c = e; c && *c;) {
        const int v = atoi(c);
        if (v <= 0 || static_cast<int>(w.size()) >= smolb200::StepPipe::kMaxChunks) return std::vector<int>();
        w.push_back(v);
        while (*c && *c != ',') ++c;
        if (*c == ',') ++c;
    }
    return w;
}();

int smol_b200_decode_step_host(void *stream, float *out_host, const float *q_host, const float *k_host,
                               const float *v_host, int n_seqs, int n_heads, int n_kv_heads, int head_dim,
                               const float *q_norm_w, const float *k_norm_w, float eps, const float *rope_cos,
                               const float *rope_sin, int rope_interleaved, uint16_t *k_pool, uint16_t *v_pool,
                               int64_t pool_rows, const int64_t *seq_row0, const int *kv_len, int max_kv_len,
                               float scale, void *scratch, size_t scratch_bytes)
{
    if (n_seqs <= 0) return SMOL_B200_OK;
    if (!out_host || !q_host || !k_host || !v_host || !scratch || n_heads <= 0 || n_kv_heads <= 0)
        return record(SMOL_B200_ERR_ARGS, "smol_b200_decode_step_host");
    const StepLayout L = step_layout(n_seqs, max_kv_len, n_heads, n_kv_heads, head_dim);
    if (scratch_bytes < L.total) return record(SMOL_B200_ERR_WORKSPACE, "smol_b200_decode_step_host");
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    uint8_t *base = static_cast<uint8_t *>(scratch);
    float *q = reinterpret_cast<float *>(base + L.q);
    float *k = reinterpret_cast<float *>(base + L.k);
    float *v = reinterpret_cast<float *>(base + L.v);
    float *qr = reinterpret_cast<float *>(base + L.qr);
    float *out = reinterpret_cast<float *>(base + L.out);
    int *pos = reinterpret_cast<int *>(base + L.pos);
    int64_t *slot = reinterpret_cast<int64_t *>(base + L.slot);
    int *next = reinterpret_cast<int *>(base + L.next);
    StepPipe *P = step_pipe();
    if (!P) return record(SMOL_B200_ERR_CUDA, "smol_b200_decode_step_host");
    std::lock_guard<std::mutex> lock(*P->mu);
    // The batch goes in two chunks of sequences from 64 on: the inputs of the second copy
    // in and the result of the first copies out while the other computes (three streams).
    // More, smaller chunks measured slower end to end (cfg 2 with equal chunks: 4 chunks
    // 5686 GB/s, 8 chunks 5142, 2 chunks 5843-5916): each chunk's attention launch fills
    // the GPU less.  The first chunk is a quarter of the batch: only its copy in and the
    // last chunk's copy out are not overlapped with compute, and the copy in is twice the
    // copy out (q, k, v against the output): cfg 2 end to end ~6.0 TB/s against ~5.8 with
    // equal halves (weights 1,2 / 1,4 / 1,6 / 1,4,3 measured within 1 % of 1,3).
    static const int kDefaultWeights[2] = {1, 3};
    int chunks = n_seqs >= 64 ? 2 : 1;
    const int *weights = chunks == 2 ? kDefaultWeights : nullptr;
    if (g_step_chunks > 0) {
        chunks = g_step_chunks < n_seqs ? g_step_chunks : n_seqs;
        weights = nullptr;
    }
    if (!g_step_weights.empty() && static_cast<int>(g_step_weights.size()) <= n_seqs) {
        chunks = static_cast<int>(g_step_weights.size());
        weights = g_step_weights.data();
    }
    long long wsum = 0;
    for (int c = 0; weights && c < chunks; ++c) wsum += weights[c];
    auto bound = [&](int c) {   // first sequence of chunk c
        if (!weights) return static_cast<int>(static_cast<long long>(n_seqs) * c / chunks);
        long long acc = 0;
        for (int i = 0; i < c; ++i) acc += weights[i];
        return static_cast<int>(static_cast<long long>(n_seqs) * acc / wsum);
    };
    const size_t qw = static_cast<size_t>(n_heads) * head_dim, kw = static_cast<size_t>(n_kv_heads) * head_dim;
    bool ok = cuda_check(cudaEventRecord(P->start, st), "record") &&          // after the caller's prior work
              cuda_check(cudaStreamWaitEvent(P->h2d, P->start, 0), "wait") &&
              cuda_check(cudaStreamWaitEvent(P->compute, P->start, 0), "wait");
    int rc = SMOL_B200_OK;
    for (int c = 0; c < chunks && ok && rc == SMOL_B200_OK; ++c) {
        const int s0 = bound(c), s1 = bound(c + 1);
        const int nc = s1 - s0;
        if (nc <= 0) continue;
        ok = cuda_check(cudaMemcpyAsync(q + s0 * qw, q_host + s0 * qw, nc * qw * 4, cudaMemcpyHostToDevice, P->h2d),
                        "copy q") &&
             cuda_check(cudaMemcpyAsync(k + s0 * kw, k_host + s0 * kw, nc * kw * 4, cudaMemcpyHostToDevice, P->h2d),
                        "copy k") &&
             cuda_check(cudaMemcpyAsync(v + s0 * kw, v_host + s0 * kw, nc * kw * 4, cudaMemcpyHostToDevice, P->h2d),
                        "copy v") &&
             cuda_check(cudaEventRecord(P->in[c], P->h2d), "record") &&
             cuda_check(cudaStreamWaitEvent(P->compute, P->in[c], 0), "wait");
        if (!ok) break;
        rc = launch_decode_step_index(P->compute, pos + s0, slot + s0, next + s0, seq_row0 + s0, kv_len + s0, nc);
        if (rc == SMOL_B200_OK)
            rc = qknorm_rope_append(P->compute, q + s0 * qw, k + s0 * kw, v + s0 * kw, nc, n_heads, n_kv_heads,
                                    head_dim, q_norm_w, k_norm_w, eps, rope_cos, rope_sin, rope_interleaved, pos + s0,
                                    slot + s0, qr + s0 * qw, nullptr, k_pool, v_pool, pool_rows);
        if (rc == SMOL_B200_OK)
            rc = decode_attention(P->compute, out + s0 * qw, qr + s0 * qw, 0, k_pool, v_pool, pool_rows,
                                  seq_row0 + s0, next + s0, nc, max_kv_len + 1, n_heads, n_kv_heads, head_dim, scale,
                                  0, 0.f, base + L.ws, L.total - L.ws);
        if (rc != SMOL_B200_OK) break;
        ok = cuda_check(cudaEventRecord(P->done[c], P->compute), "record") &&
             cuda_check(cudaStreamWaitEvent(P->d2h, P->done[c], 0), "wait") &&
             cuda_check(cudaMemcpyAsync(out_host + s0 * qw, out + s0 * qw, nc * qw * 4, cudaMemcpyDeviceToHost,
                                        P->d2h),
                        "copy out");
    }
    // Nothing of this call may still be in flight when the caller reuses its buffers.
    // On success the last copy-out waited (through events) for every chunk's compute,
    // which waited for its copy-in, so draining the copy-out stream drains all three;
    // after a failure part of that chain may be missing, so each stream is drained.
    bool drained;
    if (ok && rc == SMOL_B200_OK)
        drained = cuda_check(cudaStreamSynchronize(P->d2h), "synchronize");
    else
        drained = cuda_check(cudaStreamSynchronize(P->h2d), "synchronize") &
                  cuda_check(cudaStreamSynchronize(P->compute), "synchronize") &
                  cuda_check(cudaStreamSynchronize(P->d2h), "synchronize");
    if (rc != SMOL_B200_OK) return record(rc, "smol_b200_decode_step_host");
    if (!ok || !drained) return SMOL_B200_ERR_CUDA;
    return SMOL_B200_OK;
}

int smol_b200_prefill_attention_multi(void *stream, float *const *out_list, int n_out, int64_t out_row_stride,
                                      int64_t out_batch_stride, const uint16_t *q, int64_t q_row_stride,
                                      int64_t q_batch_stride, const uint16_t *k, int64_t k_row_stride,
                                      int64_t k_batch_stride, const uint16_t *v, int64_t v_row_stride,
                                      int64_t v_batch_stride, int batch, int seq_q, int seq_k, int n_heads,
                                      int n_kv_heads, int head_dim, float scale, int mask_kind, int q_offset,
                                      int prefix_len, int window, float softcap, const int *window_starts,
                                      int n_windows)
{
    if (!out_list || n_out < 1 || n_out > 8) return record(SMOL_B200_ERR_ARGS, "smol_b200_prefill_attention_multi");
    return record(prefill_attention(static_cast<cudaStream_t>(stream), out_list[0], out_row_stride, out_batch_stride,
                                    q, q_row_stride, q_batch_stride, k, k_row_stride, k_batch_stride, v, v_row_stride,
                                    v_batch_stride, batch, seq_q, seq_k, n_heads, n_kv_heads, head_dim, scale,
                                    mask_kind, q_offset, prefix_len, window, softcap, window_starts, n_windows,
                                    reinterpret_cast<void *const *>(out_list + 1), n_out - 1),
                  "smol_b200_prefill_attention_multi");
}

int smol_b200_prefill_attention_bf16(void *stream, uint16_t *out, int64_t out_row_stride, int64_t out_batch_stride,
                                     const uint16_t *q, int64_t q_row_stride, int64_t q_batch_stride,
                                     const uint16_t *k, int64_t k_row_stride, int64_t k_batch_stride,
                                     const uint16_t *v, int64_t v_row_stride, int64_t v_batch_stride, int batch,
                                     int seq_q, int seq_k, int n_heads, int n_kv_heads, int head_dim, float scale,
                                     int mask_kind, int q_offset, int prefix_len, int window, float softcap,
                                     const int *window_starts, int n_windows)
{
    return record(prefill_attention(static_cast<cudaStream_t>(stream), out, out_row_stride, out_batch_stride, q,
                                    q_row_stride, q_batch_stride, k, k_row_stride, k_batch_stride, v, v_row_stride,
                                    v_batch_stride, batch, seq_q, seq_k, n_heads, n_kv_heads, head_dim, scale,
                                    mask_kind, q_offset, prefix_len, window, softcap, window_starts, n_windows,
                                    nullptr, 0, 1),
                  "smol_b200_prefill_attention_bf16");
}

int smol_b200_prefill_attention_multi_bf16(void *stream, uint16_t *const *out_list, int n_out,
                                           int64_t out_row_stride, int64_t out_batch_stride, const uint16_t *q,
                                           int64_t q_row_stride, int64_t q_batch_stride, const uint16_t *k,
                                           int64_t k_row_stride, int64_t k_batch_stride, const uint16_t *v,
                                           int64_t v_row_stride, int64_t v_batch_stride, int batch, int seq_q,
                                           int seq_k, int n_heads, int n_kv_heads, int head_dim, float scale,
                                           int mask_kind, int q_offset, int prefix_len, int window, float softcap,
                                           const int *window_starts, int n_windows)
{
    if (!out_list || n_out < 1 || n_out > 8)
        return record(SMOL_B200_ERR_ARGS, "smol_b200_prefill_attention_multi_bf16");
    return record(prefill_attention(static_cast<cudaStream_t>(stream), out_list[0], out_row_stride, out_batch_stride,
                                    q, q_row_stride, q_batch_stride, k, k_row_stride, k_batch_stride, v, v_row_stride,
                                    v_batch_stride, batch, seq_q, seq_k, n_heads, n_kv_heads, head_dim, scale,
                                    mask_kind, q_offset, prefix_len, window, softcap, window_starts, n_windows,
                                    reinterpret_cast<void *const *>(out_list + 1), n_out - 1, 1),
                  "smol_b200_prefill_attention_multi_bf16");
}

int smol_b200_ipc_get_handle(const void *dev_ptr, void *handle64, size_t *offset)
{
    static_assert(sizeof(cudaIpcMemHandle_t) == 64, "IPC handle size");
    if (!dev_ptr || !handle64 || !offset) return record(SMOL_B200_ERR_ARGS, "smol_b200_ipc_get_handle");
    cudaIpcMemHandle_t h;
    if (!cuda_check(cudaIpcGetMemHandle(&h, const_cast<void *>(dev_ptr)), "cudaIpcGetMemHandle"))
        return SMOL_B200_ERR_CUDA;
    uintptr_t base = 0;
    if (!allocation_base(dev_ptr, &base)) return record(SMOL_B200_ERR_CUDA, "smol_b200_ipc_get_handle");
    memcpy(handle64, &h, sizeof(h));
    *offset = reinterpret_cast<uintptr_t>(dev_ptr) - base;
    return SMOL_B200_OK;
}

int smol_b200_ipc_open_handle(const void *handle64, void **dev_ptr)
{
    if (!handle64 || !dev_ptr) return record(SMOL_B200_ERR_ARGS, "smol_b200_ipc_open_handle");
    cudaIpcMemHandle_t h;
    memcpy(&h, handle64, sizeof(h));
    if (!cuda_check(cudaIpcOpenMemHandle(dev_ptr, h, cudaIpcMemLazyEnablePeerAccess), "cudaIpcOpenMemHandle"))
        return SMOL_B200_ERR_CUDA;
    return SMOL_B200_OK;
}

int smol_b200_ipc_close(void *dev_ptr)
{
    if (!dev_ptr) return SMOL_B200_OK;
    return cuda_check(cudaIpcCloseMemHandle(dev_ptr), "cudaIpcCloseMemHandle") ? SMOL_B200_OK : SMOL_B200_ERR_CUDA;
}

// ---------------------------------------------------------------------------
// Part 5
// ---------------------------------------------------------------------------
size_t smol_b200_siglip_workspace_bytes(const smol_b200_siglip_model *model, int n_images)
{
    return siglip_workspace_bytes(model, n_images);
}

int smol_b200_siglip_forward(void *stream, float *out, const float *images, int n_images,
                             const smol_b200_siglip_model *model, void *workspace, size_t workspace_bytes)
{
    return record(siglip_forward(static_cast<cudaStream_t>(stream), out, images, n_images, model, workspace,
                                 workspace_bytes),
                  "smol_b200_siglip_forward");
}

size_t smol_b200_encoder_workspace_bytes(int n_tokens, int hidden, int ffn)
{
    return encoder_workspace_bytes(n_tokens, hidden, ffn);
}

int smol_b200_encoder_layers(void *stream, float *x, int batch, int seq, const smol_b200_siglip_layer *layers,
                             int n_layers, int hidden, int heads, int ffn, float eps, const int *window_starts,
                             int n_windows, void *workspace, size_t workspace_bytes)
{
    return record(encoder_layers(static_cast<cudaStream_t>(stream), x, batch, seq, layers, n_layers, hidden, heads,
                                 ffn, eps, window_starts, n_windows, workspace, workspace_bytes),
                  "smol_b200_encoder_layers");
}

int smol_b200_gemm_bf16(void *stream, void *out, int64_t ldo, int out_kind, const uint16_t *a, int64_t lda,
                        const uint16_t *w, int64_t ldw, const float *bias, const float *add, int64_t ld_add,
                        int add_rows, int m, int n, int k, int act)
{
    if (act < SMOL_B200_ACT_NONE || act > SMOL_B200_ACT_GEGLU) return record(SMOL_B200_ERR_ARGS, "smol_b200_gemm_bf16");
    return record(gemm_bf16(static_cast<cudaStream_t>(stream), out, ldo, out_kind, a, lda, w, ldw, bias, add, ld_add,
                            add_rows, m, n, k, act == SMOL_B200_ACT_GELU, act >= SMOL_B200_ACT_SWIGLU ? act : 0),
                  "smol_b200_gemm_bf16");
}

int smol_b200_layer_norm(void *stream, void *out, int out_bf16, const float *x, const float *w, const float *b,
                         int rows, int hidden, float eps)
{
    return record(layer_norm(static_cast<cudaStream_t>(stream), out, out_bf16, x, w, b, rows, hidden, eps),
                  "smol_b200_layer_norm");
}

// ---------------------------------------------------------------------------
// Part 4
// ---------------------------------------------------------------------------
size_t smol_b200_qkn_prefill_workspace_bytes(const smol_b200_qkn_model *model, int n_tokens)
{
    return qkn_prefill_workspace_bytes(model, n_tokens);
}

int smol_b200_qkn_prefill(void *stream, const smol_b200_qkn_model *model, const int *tokens, int n_tokens, int start,
                          uint16_t *k_pool, uint16_t *v_pool, int64_t pool_rows, const int64_t *layer_row0_host,
                          const float *rope_cos, const float *rope_sin, void *workspace, size_t workspace_bytes)
{
    return record(qkn_prefill(static_cast<cudaStream_t>(stream), model, tokens, nullptr, n_tokens, start, k_pool, v_pool,
                              pool_rows, layer_row0_host, rope_cos, rope_sin, workspace, workspace_bytes),
                  "smol_b200_qkn_prefill");
}

size_t smol_b200_qkn_step_workspace_bytes(const smol_b200_qkn_model *model, int n_seqs, int max_kv_len)
{
    return qkn_step_workspace_bytes(model, n_seqs, max_kv_len);
}

int smol_b200_qkn_prefill_embeds(void *stream, const smol_b200_qkn_model *model, const float *embeds, int n_tokens,
                                 int start, uint16_t *k_pool, uint16_t *v_pool, int64_t pool_rows,
                                 const int64_t *layer_row0_host, const float *rope_cos, const float *rope_sin,
                                 void *workspace, size_t workspace_bytes)
{
    if (!embeds) return record(SMOL_B200_ERR_ARGS, "smol_b200_qkn_prefill_embeds");
    return record(qkn_prefill(static_cast<cudaStream_t>(stream), model, nullptr, embeds, n_tokens, start, k_pool,
                              v_pool, pool_rows, layer_row0_host, rope_cos, rope_sin, workspace, workspace_bytes),
                  "smol_b200_qkn_prefill_embeds");
}

int smol_b200_qkn_decode_step_embeds(void *stream, const smol_b200_qkn_model *model, int n_seqs, const float *embeds,
                                     int *tokens_out, uint16_t *k_pool, uint16_t *v_pool, int64_t pool_rows,
                                     const int64_t *layer_row0, int *kv_len, int max_kv_len, const float *rope_cos,
                                     const float *rope_sin, int advance, void *workspace, size_t workspace_bytes,
                                     float *x_normed_out)
{
    if (!embeds) return record(SMOL_B200_ERR_ARGS, "smol_b200_qkn_decode_step_embeds");
    return record(qkn_decode_step(static_cast<cudaStream_t>(stream), model, n_seqs, nullptr, embeds, tokens_out, k_pool,
                                  v_pool, pool_rows, layer_row0, kv_len, max_kv_len, rope_cos, rope_sin, advance,
                                  workspace, workspace_bytes, x_normed_out),
                  "smol_b200_qkn_decode_step_embeds");
}

void *smol_b200_device_alloc(size_t bytes)
{
    if (bytes == 0) return nullptr;
    void *p = nullptr;
    if (!cuda_check(cudaMalloc(&p, bytes), "cudaMalloc")) return nullptr;
    return p;
}

void smol_b200_device_free(void *p)
{
    if (p) cuda_check(cudaFree(p), "cudaFree");
}

int smol_b200_copy(void *dst, const void *src, size_t bytes)
{
    if (bytes == 0) return SMOL_B200_OK;
    if (!dst || !src) return record(SMOL_B200_ERR_ARGS, "smol_b200_copy");
    return cuda_check(cudaMemcpy(dst, src, bytes, cudaMemcpyDefault), "cudaMemcpy") ? SMOL_B200_OK
                                                                                     : SMOL_B200_ERR_CUDA;
}

int smol_b200_qkn_decode_step(void *stream, const smol_b200_qkn_model *model, int n_seqs, const int *tokens_in,
                              int *tokens_out, uint16_t *k_pool, uint16_t *v_pool, int64_t pool_rows,
                              const int64_t *layer_row0, int *kv_len, int max_kv_len, const float *rope_cos,
                              const float *rope_sin, int advance, void *workspace, size_t workspace_bytes)
{
    return record(qkn_decode_step(static_cast<cudaStream_t>(stream), model, n_seqs, tokens_in, nullptr, tokens_out, k_pool,
                                  v_pool, pool_rows, layer_row0, kv_len, max_kv_len, rope_cos, rope_sin, advance,
                                  workspace, workspace_bytes),
                  "smol_b200_qkn_decode_step");
}

int smol_b200_gemv_bf16(void *stream, float *y, int64_t ldy, const float *x, int64_t ldx, const uint16_t *w,
                        int n_out, int k_dim, int n_seqs, int mode)
{
    return record(gemv_bf16(static_cast<cudaStream_t>(stream), y, ldy, x, ldx, w, n_out, k_dim, n_seqs, mode),
                  "smol_b200_gemv_bf16");
}

int smol_b200_argmax_bf16(void *stream, int *tokens_out, const float *x, int64_t ldx, const uint16_t *emb,
                          int vocab, int k_dim, int n_seqs, void *workspace, size_t workspace_bytes)
{
    return record(argmax_bf16(static_cast<cudaStream_t>(stream), tokens_out, x, ldx, emb, vocab, k_dim, n_seqs,
                              workspace, workspace_bytes),
                  "smol_b200_argmax_bf16");
}

size_t smol_b200_argmax_workspace_bytes(int n_seqs, int vocab)
{
    return argmax_workspace_bytes(n_seqs, vocab);
}

}  // extern "C"
