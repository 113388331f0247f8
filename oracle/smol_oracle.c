/*
 * smol_oracle.c -- CPU oracle for the attention hot path (TEST INFRASTRUCTURE).
 *
 * Plain single-threaded C that restates, in this repository's own code, the
 * reference algorithms the CUDA kernels replace.  It exists to check the GPU
 * path; only tests/, the smoke check and bench.py's CPU-baseline leg load it.
 * Reference citations are file:line within tmzt/smol-genius.
 *
 * The arithmetic order follows the reference (online softmax with the running
 * maximum initialised to -1e30 and a rescale whenever a larger score appears),
 * but the dot products are plain left-to-right sums, so results agree with the
 * reference's SIMD builds to fp32 rounding, not bit for bit.
 */
#include "smol_oracle.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>

/* ------------------------------------------------------------------------ */
/* One query row against keys [j0, j1) of one KV head.                       */
/* attention.c:98-123 (causal), :47-73 (bidirectional), :303-325 (softcap).  */
/* ------------------------------------------------------------------------ */
static void attend_row(float *o, const float *q, const float *K, const float *V,
                       long kv_stride, int j0, int j1, int head_dim, float scale,
                       float cap)
{
    float run_max = -1e30f;          /* attention.c:98 */
    float run_sum = 0.0f;
    float inv_cap = cap > 0.0f ? 1.0f / cap : 0.0f;   /* attention.c:288 */
    for (int d = 0; d < head_dim; d++) o[d] = 0.0f;   /* attention.c:100 */

    for (int j = j0; j < j1; j++) {
        const float *k = K + (long)j * kv_stride;
        const float *v = V + (long)j * kv_stride;
        float s = 0.0f;
        for (int d = 0; d < head_dim; d++) s += q[d] * k[d];
        s *= scale;
        if (cap > 0.0f) s = cap * tanhf(s * inv_cap);  /* attention.c:308 */
        if (s > run_max) {                              /* attention.c:108-112 */
            float c = expf(run_max - s);
            run_sum = run_sum * c + 1.0f;
            for (int d = 0; d < head_dim; d++) o[d] = o[d] * c + v[d];
            run_max = s;
        } else {                                        /* attention.c:113-117 */
            float w = expf(s - run_max);
            run_sum += w;
            for (int d = 0; d < head_dim; d++) o[d] += w * v[d];
        }
    }
    if (run_sum > 0.0f) {                               /* attention.c:120-123 */
        float inv = 1.0f / run_sum;
        for (int d = 0; d < head_dim; d++) o[d] *= inv;
    }
}

/* GQA causal family.  attention.c:79-126 (causal), :176-226 (sliding window),
 * :281-328 (softcap), :370-421 (sliding window + softcap).  window<=0 disables the
 * window, cap<=0 disables the softcap; prefix_len>0 widens the key range of rows
 * that sit inside the prefix to [0, prefix_len) (prefix-LM). */
static void causal_family(float *out, const float *Q, const float *K, const float *V,
                          int seq_q, int seq_k, int n_heads, int n_kv_heads,
                          int head_dim, float scale, int q_offset, int window,
                          float cap, int prefix_len)
{
    int per_kv = n_heads / n_kv_heads;                  /* attention.c:84 */
    long q_stride = (long)n_heads * head_dim;
    long kv_stride = (long)n_kv_heads * head_dim;
    for (int h = 0; h < n_heads; h++) {
        int kvh = h / per_kv;                           /* attention.c:89 */
        for (int i = 0; i < seq_q; i++) {
            int pos = q_offset + i;                     /* attention.c:94 */
            int k_end = pos + 1;
            if (prefix_len > 0 && k_end < prefix_len) k_end = prefix_len;
            if (k_end > seq_k) k_end = seq_k;           /* attention.c:95-96 */
            int k_start = 0;
            if (window > 0 && pos >= window) k_start = pos - window + 1;  /* :194-196 */
            attend_row(out + i * q_stride + (long)h * head_dim,
                       Q + i * q_stride + (long)h * head_dim,
                       K + (long)kvh * head_dim, V + (long)kvh * head_dim,
                       kv_stride, k_start, k_end, head_dim, scale, cap);
        }
    }
}

void oracle_causal_attention(float *out, const float *Q, const float *K, const float *V,
                             int seq_q, int seq_k, int n_heads, int n_kv_heads,
                             int head_dim, float scale, int q_offset)
{
    causal_family(out, Q, K, V, seq_q, seq_k, n_heads, n_kv_heads, head_dim, scale,
                  q_offset, 0, 0.0f, 0);
}

void oracle_sliding_window_attention(float *out, const float *Q, const float *K,
                                     const float *V, int seq_q, int seq_k, int n_heads,
                                     int n_kv_heads, int head_dim, float scale,
                                     int q_offset, int window_size)
{
    causal_family(out, Q, K, V, seq_q, seq_k, n_heads, n_kv_heads, head_dim, scale,
                  q_offset, window_size, 0.0f, 0);
}

void oracle_causal_attention_softcap(float *out, const float *Q, const float *K,
                                     const float *V, int seq_q, int seq_k, int n_heads,
                                     int n_kv_heads, int head_dim, float scale,
                                     int q_offset, float cap)
{
    causal_family(out, Q, K, V, seq_q, seq_k, n_heads, n_kv_heads, head_dim, scale,
                  q_offset, 0, cap, 0);
}

void oracle_sliding_window_attention_softcap(float *out, const float *Q, const float *K,
                                             const float *V, int seq_q, int seq_k,
                                             int n_heads, int n_kv_heads, int head_dim,
                                             float scale, int q_offset, int window_size,
                                             float cap)
{
    causal_family(out, Q, K, V, seq_q, seq_k, n_heads, n_kv_heads, head_dim, scale,
                  q_offset, window_size, cap, 0);
}

void oracle_prefix_lm_attention(float *out, const float *Q, const float *K, const float *V,
                                int seq_q, int seq_k, int n_heads, int n_kv_heads,
                                int head_dim, float scale, int q_offset, int prefix_len)
{
    causal_family(out, Q, K, V, seq_q, seq_k, n_heads, n_kv_heads, head_dim, scale,
                  q_offset, 0, 0.0f, prefix_len);
}

/* attention.c:32-77: MHA (K/V share the Q stride, :36), each window [ws,we) attends
 * only to itself. */
void oracle_bidirectional_attention(float *out, const float *Q, const float *K,
                                    const float *V, int seq, int n_heads, int head_dim,
                                    float scale, const int *window_starts, int n_windows)
{
    (void)seq;
    long stride = (long)n_heads * head_dim;
    for (int h = 0; h < n_heads; h++) {
        for (int w = 0; w < n_windows; w++) {
            int ws = window_starts[w], we = window_starts[w + 1];
            for (int i = ws; i < we; i++) {
                attend_row(out + i * stride + (long)h * head_dim,
                           Q + i * stride + (long)h * head_dim,
                           K + (long)h * head_dim, V + (long)h * head_dim,
                           stride, ws, we, head_dim, scale, 0.0f);
            }
        }
    }
}

/* ------------------------------------------------------------------------ */
/* Number formats                                                            */
/* ------------------------------------------------------------------------ */
static inline uint32_t f32_bits(float f) { uint32_t u; memcpy(&u, &f, 4); return u; }
static inline float bits_f32(uint32_t u) { float f; memcpy(&f, &u, 4); return f; }

static inline uint16_t bf16_rne(float f)
{
    uint32_t u = f32_bits(f);
    if ((u & 0x7fffffffu) > 0x7f800000u) return (uint16_t)((u >> 16) | 0x40u); /* NaN */
    u += 0x7fffu + ((u >> 16) & 1u);
    return (uint16_t)(u >> 16);
}

void oracle_f32_to_bf16_rne(uint16_t *dst, const float *src, int64_t n)
{
    for (int64_t i = 0; i < n; i++) dst[i] = bf16_rne(src[i]);
}

/* qkn_decoder.c:44-48 / qkn_bf16_decoder.c:30-35: the reference's bf16 cast truncates. */
void oracle_f32_to_bf16_trunc(uint16_t *dst, const float *src, int64_t n)
{
    for (int64_t i = 0; i < n; i++) dst[i] = (uint16_t)(f32_bits(src[i]) >> 16);
}

void oracle_bf16_to_f32(float *dst, const uint16_t *src, int64_t n)
{
    for (int64_t i = 0; i < n; i++) dst[i] = bits_f32((uint32_t)src[i] << 16);
}

void oracle_f32_to_f16(uint16_t *dst, const float *src, int64_t n)
{
    for (int64_t i = 0; i < n; i++) {
        _Float16 h = (_Float16)src[i];
        memcpy(&dst[i], &h, 2);
    }
}

void oracle_f16_to_f32(float *dst, const uint16_t *src, int64_t n)
{
    for (int64_t i = 0; i < n; i++) {
        _Float16 h;
        memcpy(&h, &src[i], 2);
        dst[i] = (float)h;
    }
}

/* ------------------------------------------------------------------------ */
/* Batched decode over a pooled bf16-K / fp16-V cache                        */
/* ------------------------------------------------------------------------ */
void oracle_decode_batched(float *out, const float *Q, const uint16_t *K_bf16,
                           const uint16_t *V_f16, const int64_t *row0, const int *kv_len,
                           int n_seqs, int n_heads, int n_kv_heads, int head_dim,
                           float scale)
{
    long kv_dim = (long)n_kv_heads * head_dim;
    long q_dim = (long)n_heads * head_dim;
    for (int b = 0; b < n_seqs; b++) {
        int L = kv_len[b];
        float *k = (float *)malloc(sizeof(float) * (size_t)(L > 0 ? L : 1) * kv_dim);
        float *v = (float *)malloc(sizeof(float) * (size_t)(L > 0 ? L : 1) * kv_dim);
        if (!k || !v) {   /* out of host memory: NaN rows fail every comparison */
            for (long i = 0; i < q_dim; i++) out[b * q_dim + i] = NAN;
            free(k);
            free(v);
            continue;
        }
        oracle_bf16_to_f32(k, K_bf16 + row0[b] * kv_dim, (int64_t)L * kv_dim);
        oracle_f16_to_f32(v, V_f16 + row0[b] * kv_dim, (int64_t)L * kv_dim);
        /* qkn_decoder.c:658-677: seq_q=1, seq_k=pos+1, q_offset=pos */
        causal_family(out + b * q_dim, Q + b * q_dim, k, v, 1, L, n_heads, n_kv_heads,
                      head_dim, scale, L - 1, 0, 0.0f, 0);
        free(k);
        free(v);
    }
}

/* ------------------------------------------------------------------------ */
/* RoPE                                                                      */
/* ------------------------------------------------------------------------ */
/* rope.c:27-45: cos/sin duplicated over the two halves. */
void oracle_compute_rope_neox(float *cos_out, float *sin_out, const int *positions,
                              int seq, int head_dim, float theta)
{
    int half = head_dim / 2;
    for (int s = 0; s < seq; s++) {
        float p = (float)positions[s];
        for (int d = 0; d < half; d++) {
            float f = 1.0f / powf(theta, (float)(2 * d) / (float)head_dim);
            float a = p * f;
            float c = cosf(a), sn = sinf(a);
            cos_out[s * head_dim + d] = c;
            cos_out[s * head_dim + half + d] = c;
            sin_out[s * head_dim + d] = sn;
            sin_out[s * head_dim + half + d] = sn;
        }
    }
}

/* rope.c:51-66: cos/sin duplicated over each (2d, 2d+1) pair. */
void oracle_compute_rope_interleaved(float *cos_out, float *sin_out, const int *positions,
                                     int seq, int head_dim, float theta)
{
    int half = head_dim / 2;
    for (int s = 0; s < seq; s++) {
        float p = (float)positions[s];
        for (int d = 0; d < half; d++) {
            float f = 1.0f / powf(theta, (float)(2 * d) / (float)head_dim);
            float a = p * f;
            cos_out[s * head_dim + 2 * d] = cosf(a);
            cos_out[s * head_dim + 2 * d + 1] = cosf(a);
            sin_out[s * head_dim + 2 * d] = sinf(a);
            sin_out[s * head_dim + 2 * d + 1] = sinf(a);
        }
    }
}

/* qkn_decoder.c:261-274 (inv_freq) and :276-311 (table rows). */
void oracle_fill_rope_table(float *cos_tab, float *sin_tab, int n_pos, int head_dim,
                            float theta, int interleaved)
{
    int half = head_dim / 2;
    float *inv = (float *)malloc(sizeof(float) * (size_t)(half > 0 ? half : 1));
    if (!inv) {   /* out of host memory: NaN tables fail every comparison */
        for (long i = 0; i < (long)n_pos * head_dim; i++) cos_tab[i] = sin_tab[i] = NAN;
        return;
    }
    for (int d = 0; d < half; d++)
        inv[d] = 1.0f / powf(theta, (float)(2 * d) / (float)head_dim);
    for (int pos = 0; pos < n_pos; pos++) {
        float p = (float)pos;
        float *cr = cos_tab + (long)pos * head_dim;
        float *sr = sin_tab + (long)pos * head_dim;
        for (int d = 0; d < half; d++) {
            float a = p * inv[d];
            float c = cosf(a), s = sinf(a);
            if (interleaved) {
                cr[2 * d] = c; cr[2 * d + 1] = c;
                sr[2 * d] = s; sr[2 * d + 1] = s;
            } else {
                cr[d] = c; cr[half + d] = c;
                sr[d] = s; sr[half + d] = s;
            }
        }
    }
    free(inv);
}

/* rope.c:99-164 (scalar branch :154-160). */
void oracle_apply_rope_neox(float *x, const float *cos_vals, const float *sin_vals,
                            int seq, int n_heads, int head_dim)
{
    int half = head_dim / 2;
    long stride = (long)n_heads * head_dim;
    for (int s = 0; s < seq; s++) {
        const float *c = cos_vals + (long)s * head_dim;
        const float *sn = sin_vals + (long)s * head_dim;
        for (int h = 0; h < n_heads; h++) {
            float *v = x + s * stride + (long)h * head_dim;
            for (int d = 0; d < half; d++) {
                float a = v[d], b = v[half + d];
                v[d] = a * c[d] + (-b) * sn[d];
                v[half + d] = b * c[half + d] + a * sn[half + d];
            }
        }
    }
}

/* rope.c:68-93. */
void oracle_apply_rope_interleaved(float *x, const float *cos_vals, const float *sin_vals,
                                   int seq, int n_heads, int head_dim)
{
    int half = head_dim / 2;
    long stride = (long)n_heads * head_dim;
    for (int s = 0; s < seq; s++) {
        const float *c = cos_vals + (long)s * head_dim;
        const float *sn = sin_vals + (long)s * head_dim;
        for (int h = 0; h < n_heads; h++) {
            float *v = x + s * stride + (long)h * head_dim;
            for (int d = 0; d < half; d++) {
                float a = v[2 * d], b = v[2 * d + 1];
                v[2 * d] = a * c[2 * d] - b * sn[2 * d];
                v[2 * d + 1] = b * c[2 * d + 1] + a * sn[2 * d + 1];
            }
        }
    }
}

/* rope.c:12-25. */
void oracle_sinusoidal_pe(float *pe, int n_pos, int d_model)
{
    int half = d_model / 2;
    float lts = logf(10000.0f) / (float)(half - 1);
    for (int p = 0; p < n_pos; p++) {
        float *row = pe + (long)p * d_model;
        for (int d = 0; d < half; d++) {
            float it = expf(-(float)d * lts);
            float a = (float)p * it;
            row[d] = sinf(a);
            row[half + d] = cosf(a);
        }
    }
}

/* ------------------------------------------------------------------------ */
/* RMSNorm                                                                   */
/* ------------------------------------------------------------------------ */
/* rmsnorm.c:17-76 (formula :50). */
void oracle_rms_norm(float *out, const float *x, const float *weight, int seq_len,
                     int hidden, float eps)
{
    for (int s = 0; s < seq_len; s++) {
        const float *xr = x + (long)s * hidden;
        float *orow = out + (long)s * hidden;
        float ss = 0.0f;
        for (int i = 0; i < hidden; i++) ss += xr[i] * xr[i];
        float r = 1.0f / sqrtf(ss / hidden + eps);
        for (int i = 0; i < hidden; i++) orow[i] = xr[i] * r * weight[i];
    }
}

/* rmsnorm.c:78-140 (formula :113). */
void oracle_rms_norm_per_head(float *x, const float *weight, int seq_len, int n_heads,
                              int head_dim, float eps)
{
    long stride = (long)n_heads * head_dim;
    for (int s = 0; s < seq_len; s++) {
        for (int h = 0; h < n_heads; h++) {
            float *v = x + s * stride + (long)h * head_dim;
            float ss = 0.0f;
            for (int d = 0; d < head_dim; d++) ss += v[d] * v[d];
            float r = 1.0f / sqrtf(ss / head_dim + eps);
            for (int d = 0; d < head_dim; d++) v[d] = v[d] * r * weight[d];
        }
    }
}

/* ------------------------------------------------------------------------ */
/* Fused prologue: per-head norm + RoPE + cache store                        */
/* ------------------------------------------------------------------------ */
void oracle_qknorm_rope_append(float *q, float *k, const float *v, int n_tokens,
                               int n_heads, int n_kv_heads, int head_dim,
                               const float *q_norm_w, const float *k_norm_w, float eps,
                               const float *cos_tab, const float *sin_tab, int interleaved,
                               const int *positions, const int64_t *slots,
                               uint16_t *k_cache_bf16, uint16_t *v_cache_f16)
{
    long q_dim = (long)n_heads * head_dim;
    long kv_dim = (long)n_kv_heads * head_dim;
    for (int t = 0; t < n_tokens; t++) {
        float *qt = q + t * q_dim;
        float *kt = k + t * kv_dim;
        const float *c = cos_tab + (long)positions[t] * head_dim;   /* qkn_decoder.c:461-468 */
        const float *sn = sin_tab + (long)positions[t] * head_dim;
        if (q_norm_w) oracle_rms_norm_per_head(qt, q_norm_w, 1, n_heads, head_dim, eps);
        if (k_norm_w) oracle_rms_norm_per_head(kt, k_norm_w, 1, n_kv_heads, head_dim, eps);
        if (interleaved) {
            oracle_apply_rope_interleaved(qt, c, sn, 1, n_heads, head_dim);
            oracle_apply_rope_interleaved(kt, c, sn, 1, n_kv_heads, head_dim);
        } else {
            oracle_apply_rope_neox(qt, c, sn, 1, n_heads, head_dim);
            oracle_apply_rope_neox(kt, c, sn, 1, n_kv_heads, head_dim);
        }
        /* qkn_decoder.c:212-220 slot address ((layer*max)+pos)*kv_dim, here slots[t]. */
        oracle_f32_to_bf16_rne(k_cache_bf16 + slots[t] * kv_dim, kt, kv_dim);
        oracle_f32_to_f16(v_cache_f16 + slots[t] * kv_dim, v + t * kv_dim, kv_dim);
    }
}
