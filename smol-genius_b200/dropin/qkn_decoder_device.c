/*
 * qkn_decoder_device.c -- qkn_decoder_prefill / qkn_decoder_forward of tmzt/smol-genius
 * (common/decoder/qkn_decoder.h:155-167, qkn_decoder.c:369-714) on the device.
 *
 * The decoder-level drop-in: an export keeps calling qkn_decoder_load (host weights) and
 * these two functions with the reference's own qkn_ctx_t; the first call uploads the
 * context's weights once, and the KV cache, RoPE tables and every step then live on the
 * GPU (device_decoder.c over libsmol_b200's Part 4).
 *
 * Contract kept from the reference:
 *   - inputs are host fp32 embeddings ([seq_len][hidden] / [hidden]); the greedy token
 *     is returned, and the final normalised hidden state is left in ctx->dec_x
 *     (qkn_decoder.c:584, :709-713; allocated with malloc when NULL, as
 *     ensure_dec_buffers does);
 *   - ctx->kv_cache_len is the number of cached positions: it advances by seq_len /
 *     by one, and qkn_kv_cache_reset (or any truncation) is honoured on the next call;
 *   - ctx->kv_cache_k / kv_cache_v stay NULL (exports free() them), the device cache
 *     is held in a side table keyed by the context;
 *   - on failure forward returns SMOL_TOKEN_IM_END (151645), the reference's sentinel
 *     for an allocation failure (qkn_decoder.c:605-611); the reason is printed and
 *     readable through smol_cuda_last_error().  There is no CPU fallback.
 *
 * Build (a maintainer's recipe; the reference sources stay unmodified): compile
 * qkn_decoder.c with -Dqkn_decoder_prefill=qkn_decoder_prefill_host
 * -Dqkn_decoder_forward=qkn_decoder_forward_host, add this file and device_decoder.c,
 * and -lsmol_b200.
 */
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include "device_decoder.h"
#include "qkn_decoder.h"

#define DEVICE_TOKEN_ON_ERROR 151645   /* SMOL_TOKEN_IM_END, qkn_decoder.c:20 */

static dd_state *state_for(qkn_ctx_t *ctx)
{
    if (ctx->config.dec_layers < 1 || ctx->config.dec_layers > DD_MAX_LAYERS) return NULL;
    const uint64_t fp = dd_fingerprint(ctx->config.dec_hidden, ctx->config.dec_layers, ctx->config.vocab_size,
                                       ctx->decoder.tok_embeddings_bf16, ctx->decoder.layers[0].wq_weight_bf16);
    int ready;
    dd_state *st = dd_slot_find(ctx, fp, &ready);
    if (!st || ready) return st;
    const qkn_config_t *c = &ctx->config;
    const qkn_decoder_t *d = &ctx->decoder;
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
    cfg.theta = c->dec_rope_theta;
    cfg.local_theta = c->dec_rope_local_theta;
    cfg.embed_normalizer = c->embed_normalizer;
    cfg.attn_softcap = c->attn_logit_softcap;
    cfg.sliding_window = c->sliding_window;
    cfg.geglu = c->activation == QKN_ACT_GEGLU;
    cfg.interleaved = c->rope_type == QKN_ROPE_INTERLEAVED;
    dd_layer layers[DD_MAX_LAYERS];
    for (int l = 0; l < c->dec_layers; l++) {
        const qkn_dec_layer_t *ly = &d->layers[l];
        layers[l] = (dd_layer){ly->wq_weight_bf16, ly->wk_weight_bf16, ly->wv_weight_bf16, ly->wo_weight_bf16,
                               ly->gate_up_fused_bf16, ly->down_weight_bf16, ly->input_norm, ly->post_attn_norm,
                               ly->q_norm_weight, ly->k_norm_weight, ly->pre_ffn_norm, ly->post_ffn_norm,
                               ly->is_sliding};
    }
    if (dd_setup(st, &cfg, layers, d->tok_embeddings_bf16, d->norm, NULL) != 0) return NULL;
    dd_slot_claim(st, ctx, fp);
    return st;
}

void qkn_decoder_prefill(qkn_ctx_t *ctx, const float *input_embeds, int seq_len)
{
    if (seq_len <= 0) return;
    dd_state *st = state_for(ctx);
    if (!st || dd_prefill(st, input_embeds, seq_len, ctx->kv_cache_len) != 0) {
        fprintf(stderr, "qkn_decoder_prefill (device): %s\n", smol_cuda_error_string(smol_cuda_last_error()));
        return;
    }
    ctx->kv_cache_len += seq_len;
}

int qkn_decoder_forward(qkn_ctx_t *ctx, const float *input_embed)
{
    if (!ctx->dec_x) ctx->dec_x = (float *)malloc(sizeof(float) * (size_t)ctx->config.dec_hidden);
    dd_state *st = state_for(ctx);
    const int token = st && ctx->dec_x ? dd_forward(st, input_embed, ctx->kv_cache_len, ctx->dec_x) : -1;
    if (token < 0) {
        fprintf(stderr, "qkn_decoder_forward (device): %s\n", smol_cuda_error_string(smol_cuda_last_error()));
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
void qkn_decoder_device_release(qkn_ctx_t *ctx)
{
    if (ctx && dd_slot_release(ctx)) ctx->kv_cache_len = 0;
}
