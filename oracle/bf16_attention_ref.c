/*
 * bf16_attention_ref.c -- TEST INFRASTRUCTURE ONLY (a checker, never shipped or timed).
 *
 * The reference's bf16 decoder (common/decoder/qkn_bf16_decoder.c of tmzt/smol-genius)
 * keeps its attention `static`: bf16_causal_attention_softcap (:120-172) and
 * bf16_swa_attention_softcap (:175-233) -- bf16 Q / K / V in, scores and a two-pass
 * softmax in fp32 with expf, the output truncated to bf16 (:30-35).  This file
 * compiles that source unchanged, where it lies (oracle/Makefile puts its directory
 * on the include path), and exports one entry point over the two functions, so that
 * tests/golden/make_bf16_golden.py can record the reference's own bf16-path outputs as
 * a second oracle for the device's bf16 K / fp16 V cache path.
 */
#include "qkn_bf16_decoder.c"

/* window > 0 selects the sliding-window form (keys [pos - window + 1, pos]). */
__attribute__((visibility("default"))) void ref_bf16_attention(uint16_t *out, const uint16_t *q, const uint16_t *k,
                                                                const uint16_t *v, int seq_q, int seq_k, int n_heads,
                                                                int n_kv_heads, int head_dim, float scale,
                                                                int q_offset, int window, float cap)
{
    if (window > 0)
        bf16_swa_attention_softcap(out, q, k, v, seq_q, seq_k, n_heads, n_kv_heads, head_dim, scale, q_offset, window,
                                   cap);
    else
        bf16_causal_attention_softcap(out, q, k, v, seq_q, seq_k, n_heads, n_kv_heads, head_dim, scale, q_offset,
                                      cap);
}
