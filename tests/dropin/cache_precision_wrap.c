/*
 * cache_precision_wrap.c -- CPU emulation of libsmol_b200's storage precision inside
 * the reference decoder, for choosing the drop-in test's model.
 *
 * Linked with -Wl,--wrap for smol_causal_attention and its softcap and sliding-window
 * forms, so qkn_decoder.c's attention calls (qkn_decoder.c:510-528, :659-677) land
 * here.  K is rounded to bf16 and V to fp16 (the device KV cache formats), and Q to
 * bf16 when seq_q > 1 (the tensor-core prefill's operand format; decode keeps fp32 Q).  The reference kernel then runs on the
 * rounded values.  The binary built from this (qkn_dropin_emul) shows how far the
 * cache precision alone moves each step's logits, which bounds the top-2 margin a
 * drop-in token-identity test needs.
 *
 * Built with -DSMOL_WRAP_FP32_Q, prefill Q stays fp32 as well: that is the precision
 * of the decoder-step oracle's prefill (oracle/qkn_decoder_oracle.py), which the
 * qkn_weights_emul binary pins to the reference.
 */
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

void __real_smol_causal_attention(float *out, const float *Q, const float *K, const float *V, int seq_q,
                                  int seq_k, int n_heads, int n_kv_heads, int head_dim, float scale,
                                  int q_offset);
void __real_smol_causal_attention_softcap(float *out, const float *Q, const float *K, const float *V, int seq_q,
                                          int seq_k, int n_heads, int n_kv_heads, int head_dim, float scale,
                                          int q_offset, float cap);
void __real_smol_sliding_window_attention(float *out, const float *Q, const float *K, const float *V, int seq_q,
                                          int seq_k, int n_heads, int n_kv_heads, int head_dim, float scale,
                                          int q_offset, int window_size);
void __real_smol_sliding_window_attention_softcap(float *out, const float *Q, const float *K, const float *V,
                                                  int seq_q, int seq_k, int n_heads, int n_kv_heads, int head_dim,
                                                  float scale, int q_offset, int window_size, float cap);

static float round_bf16(float f)
{
    uint32_t u;
    memcpy(&u, &f, 4);
    u += 0x7fffu + ((u >> 16) & 1u);
    u &= 0xffff0000u;
    memcpy(&f, &u, 4);
    return f;
}

static float *rounded(const float *x, size_t n, int fp16)
{
    float *y = (float *)malloc(sizeof(float) * (n ? n : 1));
    for (size_t i = 0; i < n; i++) y[i] = fp16 ? (float)(_Float16)x[i] : round_bf16(x[i]);
    return y;
}

/* The rounded copies of one call's Q (prefill only), K and V. */
typedef struct {
    float *q, *k, *v;
} rounded_qkv;

static rounded_qkv round_inputs(const float *Q, const float *K, const float *V, int seq_q, int seq_k, int n_heads,
                                int n_kv_heads, int head_dim)
{
    size_t kv_n = (size_t)seq_k * n_kv_heads * head_dim;
    size_t q_n = (size_t)seq_q * n_heads * head_dim;
    rounded_qkv r;
    r.k = rounded(K, kv_n, 0);
    r.v = rounded(V, kv_n, 1);
#ifdef SMOL_WRAP_FP32_Q
    r.q = NULL;
    (void)q_n;
    (void)Q;
#else
    r.q = seq_q > 1 ? rounded(Q, q_n, 0) : NULL;
#endif
    return r;
}

static void release(rounded_qkv r)
{
    free(r.q);
    free(r.k);
    free(r.v);
}

void __wrap_smol_causal_attention(float *out, const float *Q, const float *K, const float *V, int seq_q,
                                  int seq_k, int n_heads, int n_kv_heads, int head_dim, float scale,
                                  int q_offset)
{
    rounded_qkv r = round_inputs(Q, K, V, seq_q, seq_k, n_heads, n_kv_heads, head_dim);
    __real_smol_causal_attention(out, r.q ? r.q : Q, r.k, r.v, seq_q, seq_k, n_heads, n_kv_heads, head_dim, scale,
                                 q_offset);
    release(r);
}

void __wrap_smol_causal_attention_softcap(float *out, const float *Q, const float *K, const float *V, int seq_q,
                                          int seq_k, int n_heads, int n_kv_heads, int head_dim, float scale,
                                          int q_offset, float cap)
{
    rounded_qkv r = round_inputs(Q, K, V, seq_q, seq_k, n_heads, n_kv_heads, head_dim);
    __real_smol_causal_attention_softcap(out, r.q ? r.q : Q, r.k, r.v, seq_q, seq_k, n_heads, n_kv_heads, head_dim,
                                         scale, q_offset, cap);
    release(r);
}

void __wrap_smol_sliding_window_attention(float *out, const float *Q, const float *K, const float *V, int seq_q,
                                          int seq_k, int n_heads, int n_kv_heads, int head_dim, float scale,
                                          int q_offset, int window_size)
{
    rounded_qkv r = round_inputs(Q, K, V, seq_q, seq_k, n_heads, n_kv_heads, head_dim);
    __real_smol_sliding_window_attention(out, r.q ? r.q : Q, r.k, r.v, seq_q, seq_k, n_heads, n_kv_heads, head_dim,
                                         scale, q_offset, window_size);
    release(r);
}

void __wrap_smol_sliding_window_attention_softcap(float *out, const float *Q, const float *K, const float *V,
                                                  int seq_q, int seq_k, int n_heads, int n_kv_heads, int head_dim,
                                                  float scale, int q_offset, int window_size, float cap)
{
    rounded_qkv r = round_inputs(Q, K, V, seq_q, seq_k, n_heads, n_kv_heads, head_dim);
    __real_smol_sliding_window_attention_softcap(out, r.q ? r.q : Q, r.k, r.v, seq_q, seq_k, n_heads, n_kv_heads,
                                                 head_dim, scale, q_offset, window_size, cap);
    release(r);
}
