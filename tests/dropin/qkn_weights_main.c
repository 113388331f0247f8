/*
 * qkn_weights_main.c -- runs the reference's own decoder (common/decoder/qkn_decoder.c
 * of tmzt/smol-genius) on weights and tokens read from a file, teacher-forced, and
 * writes every step's greedy token and final normalised hidden state.
 *
 * The CPU test of the decoder-step oracle (tests/test_decoder_oracle_e2e.py) writes
 * the file from the oracle's own seeded weights, runs this program and compares.
 * oracle/Makefile links it with the reference kernels and smol_causal_attention
 * wrapped by cache_precision_wrap.c (K bf16, V fp16, prefill Q bf16: the values the
 * device cache and the tensor-core prefill hold, which the oracle also uses).
 *
 * Input (little-endian): "QKNW", int32 hidden, layers, heads, kv_heads, head_dim,
 * intermediate, vocab, n_prompt, n_steps, activation (qkn_activation_t), rope_interleaved,
 * sliding_window, has_qk_norm, has_ffn_norms; float32 eps, rope_theta, rope_local_theta,
 * embed_normalizer, attn_logit_softcap; uint16 bf16 E[vocab][hidden]; float32
 * final_norm[hidden]; per layer: int32 is_sliding, bf16 wq, wk, wv, wo, gate_up (rows
 * interleaved), down; float32 input_norm, post_attn_norm, then q_norm, k_norm when
 * has_qk_norm, then pre_ffn_norm, post_ffn_norm when has_ffn_norms; int32
 * prompt[n_prompt]; int32 feed[n_steps] (the token fed at each step).
 * Output: per step int32 token, float32 x[hidden].
 *
 * Usage: qkn_weights_xxx <in> <out>
 */
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include "qkn_decoder.h"
#include "smol_kernels.h"

static FILE *g_in;

static void *take(size_t bytes)
{
    void *p = malloc(bytes ? bytes : 1);
    if (!p || fread(p, 1, bytes, g_in) != bytes) {
        fprintf(stderr, "short read\n");
        exit(2);
    }
    return p;
}

static float from_bf16(uint16_t h)
{
    uint32_t u = (uint32_t)h << 16;
    float f;
    memcpy(&f, &u, 4);
    return f;
}

int main(int argc, char **argv)
{
    if (argc != 3) return 2;
    g_in = fopen(argv[1], "rb");
    FILE *out = fopen(argv[2], "wb");
    if (!g_in || !out) return 2;
    char magic[4];
    if (fread(magic, 1, 4, g_in) != 4 || memcmp(magic, "QKNW", 4)) return 2;
    int32_t *h = (int32_t *)take(14 * sizeof(int32_t));
    const int H = h[0], L = h[1], HQ = h[2], HKV = h[3], HD = h[4], I = h[5], V = h[6], NP = h[7], NS = h[8];
    const int has_qk_norm = h[12], has_ffn_norms = h[13];
    float *fh = (float *)take(5 * sizeof(float));
    if (L < 1 || L > QKN_MAX_DEC_LAYERS || NP < 2) return 2;
    const size_t qd = (size_t)HQ * HD, kvd = (size_t)HKV * HD;

    qkn_ctx_t *ctx = (qkn_ctx_t *)calloc(1, sizeof(qkn_ctx_t));
    qkn_config_t *c = &ctx->config;
    c->dec_hidden = H;
    c->dec_layers = L;
    c->dec_heads = HQ;
    c->dec_kv_heads = HKV;
    c->dec_head_dim = HD;
    c->dec_intermediate = I;
    c->vocab_size = V;
    c->activation = h[9] ? QKN_ACT_GEGLU : QKN_ACT_SWIGLU;
    c->rope_type = h[10] ? QKN_ROPE_INTERLEAVED : QKN_ROPE_NEOX;
    c->sliding_window = h[11];
    c->dec_rms_norm_eps = fh[0];
    c->dec_rope_theta = fh[1];
    c->dec_rope_local_theta = fh[2];
    c->embed_normalizer = fh[3];
    c->attn_logit_softcap = fh[4];
    qkn_decoder_t *d = &ctx->decoder;
    d->tok_embeddings_bf16 = (uint16_t *)take((size_t)V * H * 2);
    d->norm = (float *)take((size_t)H * 4);
    for (int l = 0; l < L; l++) {
        qkn_dec_layer_t *ly = &d->layers[l];
        ly->is_sliding = *(int32_t *)take(4);
        ly->wq_weight_bf16 = (uint16_t *)take(qd * H * 2);
        ly->wk_weight_bf16 = (uint16_t *)take(kvd * H * 2);
        ly->wv_weight_bf16 = (uint16_t *)take(kvd * H * 2);
        ly->wo_weight_bf16 = (uint16_t *)take((size_t)H * qd * 2);
        ly->gate_up_fused_bf16 = (uint16_t *)take((size_t)2 * I * H * 2);
        ly->down_weight_bf16 = (uint16_t *)take((size_t)H * I * 2);
        ly->input_norm = (float *)take((size_t)H * 4);
        ly->post_attn_norm = (float *)take((size_t)H * 4);
        if (has_qk_norm) {
            ly->q_norm_weight = (float *)take((size_t)HD * 4);
            ly->k_norm_weight = (float *)take((size_t)HD * 4);
        }
        if (has_ffn_norms) {
            ly->pre_ffn_norm = (float *)take((size_t)H * 4);
            ly->post_ffn_norm = (float *)take((size_t)H * 4);
        }
    }
    int32_t *prompt = (int32_t *)take((size_t)NP * 4);
    int32_t *feed = (int32_t *)take((size_t)NS * 4);
    fclose(g_in);

    int threads = smol_get_num_cpus();
    smol_set_threads(threads > 16 ? 16 : threads);

    /* prefill all but the last prompt token (qkn_decoder.c:369-564) */
    float *embeds = (float *)malloc(sizeof(float) * (size_t)(NP - 1) * H);
    for (int i = 0; i < NP - 1; i++)
        for (int k = 0; k < H; k++)
            embeds[(size_t)i * H + k] = from_bf16(d->tok_embeddings_bf16[(size_t)prompt[i] * H + k]);
    qkn_decoder_prefill(ctx, embeds, NP - 1);

    /* teacher-forced steps; qkn_decoder_forward leaves the final-normed state in
       ctx->dec_x (qkn_decoder.c:584, :709-713) */
    float *x = (float *)malloc(sizeof(float) * (size_t)H);
    for (int s = 0; s < NS; s++) {
        for (int k = 0; k < H; k++) x[k] = from_bf16(d->tok_embeddings_bf16[(size_t)feed[s] * H + k]);
        const int32_t tok = qkn_decoder_forward(ctx, x);
        fwrite(&tok, 4, 1, out);
        fwrite(ctx->dec_x, 4, (size_t)H, out);
    }
    fclose(out);
    return 0;
}
