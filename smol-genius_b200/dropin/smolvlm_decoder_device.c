/*
 * smolvlm_decoder_device.c -- smolvlm_decoder_prefill / smolvlm_decoder_forward of
 * tmzt/smol-genius (exports/smolvlm/smolvlm.h:248-251, decoder.c:269-476) on the device.
 *
 * The decoder-level drop-in for the SmolVLM export, as qkn_decoder_device.c is for
 * qkn_decoder: smolvlm's loader fills smolvlm_ctx_t, the first call here uploads the
 * decoder weights (no QK-norm, its own lm_head), and the KV cache, RoPE tables and every
 * step then live on the GPU (device_decoder.c over libsmol_b200's Part 4).  The greedy
 * token is returned and the final normalised state left in ctx->dec_x
 * (decoder.c:472-475); ctx->kv_cache_len keeps its meaning; kv_cache_k / kv_cache_v stay
 * NULL; on failure the forward returns SMOLVLM_TOKEN_EOS (49154), the reference's
 * sentinel for a failed cache growth (decoder.c:420-425).  No CPU fallback.
 *
 * Build: compile exports/smolvlm/decoder.c with
 * -Dsmolvlm_decoder_prefill=smolvlm_decoder_prefill_host
 * -Dsmolvlm_decoder_forward=smolvlm_decoder_forward_host, add this file and
 * device_decoder.c, and -lsmol_b200.
 */
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include "device_decoder.h"
#include "smolvlm.h"

#define DEVICE_TOKEN_ON_ERROR 49154   /* SMOLVLM_TOKEN_EOS, smolvlm.h:54 */

static dd_state *state_for(smolvlm_ctx_t *ctx)
{
    if (ctx->config.dec_layers < 1 || ctx->config.dec_layers > DD_MAX_LAYERS) return NULL;
    const uint64_t fp = dd_fingerprint(ctx->config.dec_hidden, ctx->config.dec_layers, ctx->config.vocab_size,
                                       ctx->decoder.tok_embeddings_bf16, ctx->decoder.layers[0].wq_weight_bf16);
    int ready;
    dd_state *st = dd_slot_find(ctx, fp, &ready);
    if (!st || ready) return st;
    const smolvlm_config_t *c = &ctx->config;
    const smolvlm_decoder_t *d = &ctx->decoder;
    dd_config cfg;
    memset(&cfg, 0, sizeof(cfg));
    cfg.hidden = c->dec_hidden;
    cfg.layers = c->dec_layers;
    cfg.heads = c->dec_heads;
    cfg.kv_heads = c->dec_kv_heads;
    cfg.head_dim = c->dec_head_dim;
    cfg.intermediate = c->dec_intermediate;
    cfg.vocab = c->vocab_size;
    cfg.eps = c->dec_rms_norm_eps;
    cfg.theta = c->dec_rope_theta;   /* NeoX RoPE, SwiGLU, no sliding layers (decoder.c:391-476) */
    dd_layer layers[DD_MAX_LAYERS];
    for (int l = 0; l < c->dec_layers; l++) {
        const smolvlm_dec_layer_t *ly = &d->layers[l];
        layers[l] = (dd_layer){ly->wq_weight_bf16, ly->wk_weight_bf16, ly->wv_weight_bf16, ly->wo_weight_bf16,
                               ly->gate_up_fused_bf16, ly->down_weight_bf16, ly->input_norm, ly->post_attn_norm,
                               NULL, NULL, NULL, NULL, 0};
    }
    if (dd_setup(st, &cfg, layers, d->tok_embeddings_bf16, d->norm, d->lm_head_bf16) != 0)
        return NULL;
    dd_slot_claim(st, ctx, fp);
    return st;
}

void smolvlm_decoder_prefill(smolvlm_ctx_t *ctx, const float *input_embeds, int seq_len)
{
    if (seq_len <= 0) return;
    dd_state *st = state_for(ctx);
    if (!st || dd_prefill(st, input_embeds, seq_len, ctx->kv_cache_len) != 0) {
        fprintf(stderr, "smolvlm_decoder_prefill (device): %s\n", smol_cuda_error_string(smol_cuda_last_error()));
        return;
    }
    ctx->kv_cache_len += seq_len;
}

int smolvlm_decoder_forward(smolvlm_ctx_t *ctx, const float *input_embed)
{
    if (!ctx->dec_x) ctx->dec_x = (float *)malloc(sizeof(float) * (size_t)ctx->config.dec_hidden);
    dd_state *st = state_for(ctx);
    const int token = st && ctx->dec_x ? dd_forward(st, input_embed, ctx->kv_cache_len, ctx->dec_x) : -1;
    if (token < 0) {
        fprintf(stderr, "smolvlm_decoder_forward (device): %s\n", smol_cuda_error_string(smol_cuda_last_error()));
        return DEVICE_TOKEN_ON_ERROR;
    }
    ctx->kv_cache_len += 1;
    return token;
}

/* Frees the device weights, cache and workspaces held for ctx (a no-op for a context
 * never passed here) and sets ctx->kv_cache_len to 0: the cached positions are gone.
 * The reference has no call that frees a context (exports free its fields directly),
 * so device memory otherwise stays until the process exits; a context freed and
 * allocated again at the same address with other weights is recognised by the
 * fingerprint and set up afresh. */
void smolvlm_decoder_device_release(smolvlm_ctx_t *ctx)
{
    if (ctx && dd_slot_release(ctx)) ctx->kv_cache_len = 0;
}
