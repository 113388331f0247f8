/*
 * smol_oracle.h -- CPU oracle for the attention hot path (TEST INFRASTRUCTURE).
 *
 * A plain, single-threaded C restatement of the reference algorithms that the
 * CUDA kernels of this repository replace.  Only tests/, the smoke check and the
 * CPU-baseline leg of bench.py load it; no product code links or calls it.
 *
 * Every function names the reference file:line it follows (paths are relative
 * to the reference project root, tmzt/smol-genius).
 *
 * Layouts follow the reference: activations are row-major [tokens, heads*head_dim]
 * fp32; a KV cache is [layer][kv_cache_max][kv_heads*head_dim].
 */
#ifndef SMOL_ORACLE_H
#define SMOL_ORACLE_H

#include <stdint.h>

/* ---- attention (common/kernels/attention.c) ---- */
void oracle_causal_attention(float *out, const float *Q, const float *K, const float *V,
                             int seq_q, int seq_k, int n_heads, int n_kv_heads,
                             int head_dim, float scale, int q_offset);
void oracle_sliding_window_attention(float *out, const float *Q, const float *K,
                                     const float *V, int seq_q, int seq_k, int n_heads,
                                     int n_kv_heads, int head_dim, float scale,
                                     int q_offset, int window_size);
void oracle_causal_attention_softcap(float *out, const float *Q, const float *K,
                                     const float *V, int seq_q, int seq_k, int n_heads,
                                     int n_kv_heads, int head_dim, float scale,
                                     int q_offset, float cap);
void oracle_sliding_window_attention_softcap(float *out, const float *Q, const float *K,
                                             const float *V, int seq_q, int seq_k,
                                             int n_heads, int n_kv_heads, int head_dim,
                                             float scale, int q_offset, int window_size,
                                             float cap);
void oracle_bidirectional_attention(float *out, const float *Q, const float *K,
                                    const float *V, int seq, int n_heads, int head_dim,
                                    float scale, const int *window_starts, int n_windows);
/* Prefix-LM: row i (global position q_offset+i) attends keys
 * [0, min(seq_k, max(prefix_len, q_offset+i+1))).  No reference function; it is the
 * composition of two smol_causal_attention calls (q_offset=P-1 for the prefix rows,
 * q_offset=P for the suffix rows). */
void oracle_prefix_lm_attention(float *out, const float *Q, const float *K, const float *V,
                                int seq_q, int seq_k, int n_heads, int n_kv_heads,
                                int head_dim, float scale, int q_offset, int prefix_len);

/* Batched single-query decode over a pooled cache: sequence b reads rows
 * [row0[b], row0[b]+kv_len[b]) of K (bf16 bits) and V (fp16 bits), each row
 * kv_heads*head_dim wide; Q and out are [n_seqs, n_heads*head_dim] fp32.
 * Per sequence this is smol_causal_attention(seq_q=1, seq_k=kv_len, q_offset=kv_len-1)
 * (qkn_decoder.c:658-677) on the upcast cache rows. */
void oracle_decode_batched(float *out, const float *Q, const uint16_t *K_bf16,
                           const uint16_t *V_f16, const int64_t *row0, const int *kv_len,
                           int n_seqs, int n_heads, int n_kv_heads, int head_dim,
                           float scale);

/* ---- RoPE (common/kernels/rope.c, common/decoder/qkn_decoder.c) ---- */
void oracle_compute_rope_neox(float *cos_out, float *sin_out, const int *positions,
                              int seq, int head_dim, float theta);
void oracle_compute_rope_interleaved(float *cos_out, float *sin_out, const int *positions,
                                     int seq, int head_dim, float theta);
void oracle_apply_rope_neox(float *x, const float *cos_vals, const float *sin_vals,
                            int seq, int n_heads, int head_dim);
void oracle_apply_rope_interleaved(float *x, const float *cos_vals, const float *sin_vals,
                                   int seq, int n_heads, int head_dim);
void oracle_sinusoidal_pe(float *pe, int n_pos, int d_model);
/* qkn_decoder.c:261-311: table rows 0..n_pos-1 built from inv_freq = 1/powf(theta,2d/hd). */
void oracle_fill_rope_table(float *cos_tab, float *sin_tab, int n_pos, int head_dim,
                            float theta, int interleaved);

/* ---- RMSNorm (common/kernels/rmsnorm.c) ---- */
void oracle_rms_norm(float *out, const float *x, const float *weight, int seq_len,
                     int hidden, float eps);
void oracle_rms_norm_per_head(float *x, const float *weight, int seq_len, int n_heads,
                              int head_dim, float eps);

/* ---- fused per-token prologue of qkn_decoder_prefill/forward ----
 * qkn_decoder.c:488-503 (prefill) and :642-652 (decode): per-head RMSNorm of q and k
 * (skipped when the weight is NULL), RoPE of q and k from table row positions[t],
 * then K/V stored into cache row slots[t].  q is rotated in place (fp32); the cache
 * here stores K as bf16 (round-to-nearest-even) and V as fp16, the device format. */
void oracle_qknorm_rope_append(float *q, float *k, const float *v, int n_tokens,
                               int n_heads, int n_kv_heads, int head_dim,
                               const float *q_norm_w, const float *k_norm_w, float eps,
                               const float *cos_tab, const float *sin_tab, int interleaved,
                               const int *positions, const int64_t *slots,
                               uint16_t *k_cache_bf16, uint16_t *v_cache_f16);

/* ---- number formats ---- */
void oracle_f32_to_bf16_rne(uint16_t *dst, const float *src, int64_t n);
void oracle_f32_to_bf16_trunc(uint16_t *dst, const float *src, int64_t n);
void oracle_bf16_to_f32(float *dst, const uint16_t *src, int64_t n);
void oracle_f32_to_f16(uint16_t *dst, const float *src, int64_t n);
void oracle_f16_to_f32(float *dst, const uint16_t *src, int64_t n);

#endif /* SMOL_ORACLE_H */
