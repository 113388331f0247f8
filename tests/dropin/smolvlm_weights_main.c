/*
 * smolvlm_weights_main.c -- runs the reference's SmolVLM text decoder
 * (smolvlm_decoder_prefill / smolvlm_decoder_forward, exports/smolvlm/decoder.c of
 * tmzt/smol-genius) on weights and tokens read from a file, teacher-forced, and writes
 * every step's greedy token and final normalised hidden state.
 *
 * Input: the file tests/dropin/qkn_weights_main.c reads (its header comment gives the
 * format; has_qk_norm 0, activation 0, no FFN norms), followed by the bf16 lm_head
 * [vocab][hidden].  Output: per step int32 token, float32 x[hidden].  oracle/Makefile
 * links it with the reference's kernels and smol_causal_attention wrapped by
 * cache_precision_wrap.c (the decoder-step oracle's cache formats).
 *
 * Usage: smolvlm_weights_xxx <in> <out>
 */
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include "smolvlm.h"
#include "smol_kernels.h"

void smolvlm_decoder_prefill(smolvlm_ctx_t *ctx, const float *input_embeds, int seq_len);
int smolvlm_decoder_forward(smolvlm_ctx_t *ctx, const float *input_embed);

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
    if (h[9] != 0 || h[12] != 0 || h[13] != 0 || L < 1 || L > SMOLVLM_DEC_LAYERS || NP < 2) return 2;
    float *fh = (float *)take(5 * sizeof(float));
    const size_t qd = (size_t)HQ * HD, kvd = (size_t)HKV * HD;

    smolvlm_ctx_t *ctx = (smolvlm_ctx_t *)calloc(1, sizeof(smolvlm_ctx_t));
    smolvlm_config_t *c = &ctx->config;
    c->dec_hidden = H;
    c->dec_layers = L;
    c->dec_heads = HQ;
    c->dec_kv_heads = HKV;
    c->dec_head_dim = HD;
    c->dec_intermediate = I;
    c->vocab_size = V;
    c->dec_rms_norm_eps = fh[0];
    c->dec_rope_theta = fh[1];
    smolvlm_decoder_t *d = &ctx->decoder;
    d->tok_embeddings_bf16 = (uint16_t *)take((size_t)V * H * 2);
    d->norm = (float *)take((size_t)H * 4);
    for (int l = 0; l < L; l++) {
        smolvlm_dec_layer_t *ly = &d->layers[l];
        (void)take(4);   /* is_sliding: not used by this decoder */
        ly->wq_weight_bf16 = (uint16_t *)take(qd * H * 2);
        ly->wk_weight_bf16 = (uint16_t *)take(kvd * H * 2);
        ly->wv_weight_bf16 = (uint16_t *)take(kvd * H * 2);
        ly->wo_weight_bf16 = (uint16_t *)take((size_t)H * qd * 2);
        ly->gate_up_fused_bf16 = (uint16_t *)take((size_t)2 * I * H * 2);
        ly->down_weight_bf16 = (uint16_t *)take((size_t)H * I * 2);
        ly->input_norm = (float *)take((size_t)H * 4);
        ly->post_attn_norm = (float *)take((size_t)H * 4);
    }
    int32_t *prompt = (int32_t *)take((size_t)NP * 4);
    int32_t *feed = (int32_t *)take((size_t)NS * 4);
    d->lm_head_bf16 = (uint16_t *)take((size_t)V * H * 2);
    fclose(g_in);

    int threads = smol_get_num_cpus();
    smol_set_threads(threads > 16 ? 16 : threads);

    /* prefill all but the last prompt token (decoder.c:269-363) */
    float *embeds = (float *)malloc(sizeof(float) * (size_t)(NP - 1) * H);
    for (int i = 0; i < NP - 1; i++)
        for (int k = 0; k < H; k++)
            embeds[(size_t)i * H + k] = from_bf16(d->tok_embeddings_bf16[(size_t)prompt[i] * H + k]);
    smolvlm_decoder_prefill(ctx, embeds, NP - 1);

    /* teacher-forced steps; the forward leaves the final-normed state in ctx->dec_x
       (decoder.c:472-475) */
    float *x = (float *)malloc(sizeof(float) * (size_t)H);
    for (int s = 0; s < NS; s++) {
        for (int k = 0; k < H; k++) x[k] = from_bf16(d->tok_embeddings_bf16[(size_t)feed[s] * H + k]);
        const int32_t tok = smolvlm_decoder_forward(ctx, x);
        fwrite(&tok, 4, 1, out);
        fwrite(ctx->dec_x, 4, (size_t)H, out);
    }
    fclose(out);
    return 0;
}
