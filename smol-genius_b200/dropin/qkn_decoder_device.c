/*
 * qkn_decoder_device.c -- qkn_decoder_prefill / qkn_decoder_forward of tmzt/smol-genius
 * (common/decoder/qkn_decoder.h:155-167, qkn_decoder.c:369-714) on the device.
 *
 * The decoder-level drop-in: an export keeps calling qkn_decoder_load (host weights) and
 * these two functions with the reference's own qkn_ctx_t; the first call uploads the
 * context's weights once, and the KV cache, RoPE tables and every step then live on the
 * GPU (libsmol_b200's Part 4: smol_b200_qkn_prefill_embeds, smol_b200_qkn_decode_step_embeds).
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
 *     for an allocation failure (qkn_decoder.c:605-611); the error is readable through
 *     smol_cuda_last_error().  There is no CPU fallback.
 *
 * Build (a maintainer's recipe; the reference sources stay unmodified): compile
 * qkn_decoder.c with -Dqkn_decoder_prefill=qkn_decoder_prefill_host
 * -Dqkn_decoder_forward=qkn_decoder_forward_host, add this file and -lsmol_b200.
 */
#include <math.h>
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include "qkn_decoder.h"
#include "smol_b200.h"
#include "smol_kernels.h"

#define DEVICE_TOKEN_ON_ERROR 151645   /* SMOL_TOKEN_IM_END, qkn_decoder.c:20 */
#define MAX_CONTEXTS 8

typedef struct {
    const qkn_ctx_t *ctx;
    smol_b200_qkn_layer layers[QKN_MAX_DEC_LAYERS];
    smol_b200_qkn_model model;
    int64_t cap;                      /* positions per layer in the pools */
    uint16_t *k_pool, *v_pool;        /* [layers * cap][kv_dim] bf16 / fp16 */
    int64_t row0_host[QKN_MAX_DEC_LAYERS];
    int64_t *row0_dev;                /* [layers] for the one-sequence step */
    int rope_cap;                     /* rows of the tables */
    float *cos, *sin, *cos_local, *sin_local;
    int *kv_len_dev, *token_dev;
    float *x_dev, *xn_dev;            /* embeddings in / the final normalised state out */
    int x_cap;                        /* rows of x_dev */
    void *step_ws, *prefill_ws;
    size_t step_ws_bytes, prefill_ws_bytes;
    int prefill_cap;
} device_state;

static device_state g_states[MAX_CONTEXTS];

static void *upload(const void *host, size_t bytes)
{
    if (!host) return NULL;
    void *d = smol_b200_device_alloc(bytes);
    if (d && smol_b200_copy(d, host, bytes) != SMOL_B200_OK) {
        smol_b200_device_free(d);
        return NULL;
    }
    return d;
}

/* RoPE tables for positions [0, rows) with the decoder's own formula
 * (qkn_decoder.c:261-311 -- the same inv_freq / cos / sin as smol_compute_rope_*). */
static int rope_tables(float **cos_d, float **sin_d, int rows, int head_dim, float theta, int interleaved)
{
    int *pos = (int *)malloc(sizeof(int) * (size_t)rows);
    float *c = (float *)malloc(sizeof(float) * (size_t)rows * head_dim);
    float *s = (float *)malloc(sizeof(float) * (size_t)rows * head_dim);
    int ok = pos && c && s;
    if (ok) {
        for (int i = 0; i < rows; i++) pos[i] = i;
        if (interleaved)
            smol_compute_rope_interleaved(c, s, pos, rows, head_dim, theta);
        else
            smol_compute_rope_neox(c, s, pos, rows, head_dim, theta);
        smol_b200_device_free(*cos_d);
        smol_b200_device_free(*sin_d);
        *cos_d = (float *)upload(c, sizeof(float) * (size_t)rows * head_dim);
        *sin_d = (float *)upload(s, sizeof(float) * (size_t)rows * head_dim);
        ok = *cos_d && *sin_d;
    }
    free(pos);
    free(c);
    free(s);
    return ok;
}

static device_state *state_for(qkn_ctx_t *ctx)
{
    device_state *free_slot = NULL;
    for (int i = 0; i < MAX_CONTEXTS; i++) {
        if (g_states[i].ctx == ctx) return &g_states[i];
        if (!g_states[i].ctx && !free_slot) free_slot = &g_states[i];
    }
    if (!free_slot) return NULL;
    const qkn_config_t *c = &ctx->config;
    const qkn_decoder_t *d = &ctx->decoder;
    const size_t H = (size_t)c->dec_hidden, I = (size_t)c->dec_intermediate, HD = (size_t)c->dec_head_dim;
    const size_t qd = (size_t)c->dec_heads * HD, kvd = (size_t)c->dec_kv_heads * HD;
    device_state *st = free_slot;
    memset(st, 0, sizeof(*st));
    for (int l = 0; l < c->dec_layers; l++) {
        const qkn_dec_layer_t *ly = &d->layers[l];
        smol_b200_qkn_layer *o = &st->layers[l];
        o->wq = (const uint16_t *)upload(ly->wq_weight_bf16, qd * H * 2);
        o->wk = (const uint16_t *)upload(ly->wk_weight_bf16, kvd * H * 2);
        o->wv = (const uint16_t *)upload(ly->wv_weight_bf16, kvd * H * 2);
        o->wo = (const uint16_t *)upload(ly->wo_weight_bf16, H * qd * 2);
        o->gate_up = (const uint16_t *)upload(ly->gate_up_fused_bf16, 2 * I * H * 2);
        o->down = (const uint16_t *)upload(ly->down_weight_bf16, H * I * 2);
        o->input_norm = (const float *)upload(ly->input_norm, H * 4);
        o->post_attn_norm = (const float *)upload(ly->post_attn_norm, H * 4);
        o->q_norm = (const float *)upload(ly->q_norm_weight, HD * 4);
        o->k_norm = (const float *)upload(ly->k_norm_weight, HD * 4);
        o->pre_ffn_norm = (const float *)upload(ly->pre_ffn_norm, H * 4);
        o->post_ffn_norm = (const float *)upload(ly->post_ffn_norm, H * 4);
        o->is_sliding = ly->is_sliding;
        if (!o->wq || !o->wk || !o->wv || !o->wo || !o->gate_up || !o->down || !o->input_norm || !o->post_attn_norm)
            return NULL;
    }
    smol_b200_qkn_model *m = &st->model;
    m->hidden = c->dec_hidden;
    m->n_layers = c->dec_layers;
    m->n_heads = c->dec_heads;
    m->n_kv_heads = c->dec_kv_heads;
    m->head_dim = c->dec_head_dim;
    m->intermediate = c->dec_intermediate;
    m->vocab = c->vocab_size;
    m->eps = c->dec_rms_norm_eps;
    m->rope_interleaved = c->rope_type == QKN_ROPE_INTERLEAVED;
    m->tok_embeddings = (const uint16_t *)upload(d->tok_embeddings_bf16, (size_t)c->vocab_size * H * 2);
    m->final_norm = (const float *)upload(d->norm, H * 4);
    m->layers = st->layers;
    m->activation = c->activation == QKN_ACT_GEGLU;
    m->embed_normalizer = c->embed_normalizer;
    m->attn_softcap = c->attn_logit_softcap;
    m->sliding_window = c->sliding_window;
    st->kv_len_dev = (int *)smol_b200_device_alloc(sizeof(int));
    st->token_dev = (int *)smol_b200_device_alloc(sizeof(int));
    st->xn_dev = (float *)smol_b200_device_alloc(H * 4);
    if (!m->tok_embeddings || !m->final_norm || !st->kv_len_dev || !st->token_dev || !st->xn_dev) return NULL;
    st->ctx = ctx;
    return st;
}

/* Pools, tables and buffers large enough for positions [0, need). */
static int ensure_capacity(device_state *st, const qkn_ctx_t *ctx, int need, int n_in)
{
    const qkn_config_t *c = &ctx->config;
    const size_t H = (size_t)c->dec_hidden, kvd = (size_t)c->dec_kv_heads * c->dec_head_dim;
    const int L = c->dec_layers;
    if (need > st->cap) {
        const int64_t cap = need + 1024 > 2 * st->cap ? need + 1024 : 2 * st->cap;
        uint16_t *k = (uint16_t *)smol_b200_device_alloc((size_t)L * cap * kvd * 2);
        uint16_t *v = (uint16_t *)smol_b200_device_alloc((size_t)L * cap * kvd * 2);
        if (!k || !v) return 0;
        const int keep = ctx->kv_cache_len < st->cap ? ctx->kv_cache_len : (int)st->cap;
        for (int l = 0; l < L && st->k_pool && keep > 0; l++) {
            if (smol_b200_copy(k + (size_t)l * cap * kvd, st->k_pool + (size_t)l * st->cap * kvd,
                               (size_t)keep * kvd * 2) != SMOL_B200_OK ||
                smol_b200_copy(v + (size_t)l * cap * kvd, st->v_pool + (size_t)l * st->cap * kvd,
                               (size_t)keep * kvd * 2) != SMOL_B200_OK)
                return 0;
        }
        smol_b200_device_free(st->k_pool);
        smol_b200_device_free(st->v_pool);
        st->k_pool = k;
        st->v_pool = v;
        st->cap = cap;
        for (int l = 0; l < L; l++) st->row0_host[l] = (int64_t)l * cap;
        smol_b200_device_free(st->row0_dev);
        st->row0_dev = (int64_t *)upload(st->row0_host, sizeof(int64_t) * (size_t)L);
        smol_b200_device_free(st->step_ws);
        st->step_ws_bytes = smol_b200_qkn_step_workspace_bytes(&st->model, 1, (int)cap - 1);
        st->step_ws = smol_b200_device_alloc(st->step_ws_bytes);
        if (!st->row0_dev || !st->step_ws) return 0;
    }
    if (need > st->rope_cap) {
        const int rows = (int)st->cap;
        const int inter = c->rope_type == QKN_ROPE_INTERLEAVED;
        if (!rope_tables(&st->cos, &st->sin, rows, c->dec_head_dim, c->dec_rope_theta, inter)) return 0;
        /* sliding layers' own theta (qkn_decoder.c:313-340) */
        if (c->dec_rope_local_theta > 0.0f && c->dec_rope_local_theta != c->dec_rope_theta) {
            if (!rope_tables(&st->cos_local, &st->sin_local, rows, c->dec_head_dim, c->dec_rope_local_theta, inter))
                return 0;
            st->model.rope_cos_local = st->cos_local;
            st->model.rope_sin_local = st->sin_local;
        }
        st->rope_cap = rows;
    }
    if (n_in > st->x_cap) {
        smol_b200_device_free(st->x_dev);
        st->x_dev = (float *)smol_b200_device_alloc((size_t)n_in * H * 4);
        if (!st->x_dev) return 0;
        st->x_cap = n_in;
    }
    return 1;
}

void qkn_decoder_prefill(qkn_ctx_t *ctx, const float *input_embeds, int seq_len)
{
    if (seq_len <= 0) return;
    device_state *st = state_for(ctx);
    const int start = ctx->kv_cache_len;
    if (!st || !ensure_capacity(st, ctx, start + seq_len + 1, seq_len)) {
        fprintf(stderr, "qkn_decoder_prefill (device): %s\n", smol_cuda_error_string(smol_cuda_last_error()));
        return;
    }
    if (seq_len > st->prefill_cap) {
        smol_b200_device_free(st->prefill_ws);
        st->prefill_ws_bytes = smol_b200_qkn_prefill_workspace_bytes(&st->model, seq_len);
        st->prefill_ws = smol_b200_device_alloc(st->prefill_ws_bytes);
        st->prefill_cap = st->prefill_ws ? seq_len : 0;
    }
    const size_t H = (size_t)ctx->config.dec_hidden;
    if (!st->prefill_ws || smol_b200_copy(st->x_dev, input_embeds, (size_t)seq_len * H * 4) != SMOL_B200_OK ||
        smol_b200_qkn_prefill_embeds(NULL, &st->model, st->x_dev, seq_len, start, st->k_pool, st->v_pool,
                                     (int64_t)ctx->config.dec_layers * st->cap, st->row0_host, st->cos, st->sin,
                                     st->prefill_ws, st->prefill_ws_bytes) != SMOL_B200_OK) {
        fprintf(stderr, "qkn_decoder_prefill (device): %s\n", smol_cuda_error_string(smol_cuda_last_error()));
        return;
    }
    ctx->kv_cache_len = start + seq_len;
}

int qkn_decoder_forward(qkn_ctx_t *ctx, const float *input_embed)
{
    device_state *st = state_for(ctx);
    const int pos = ctx->kv_cache_len;
    const size_t H = (size_t)ctx->config.dec_hidden;
    if (!ctx->dec_x) ctx->dec_x = (float *)malloc(H * sizeof(float));
    int token = DEVICE_TOKEN_ON_ERROR;
    if (!st || !ctx->dec_x || !ensure_capacity(st, ctx, pos + 2, 1) ||
        smol_b200_copy(st->x_dev, input_embed, H * 4) != SMOL_B200_OK ||
        smol_b200_copy(st->kv_len_dev, &pos, sizeof(int)) != SMOL_B200_OK ||
        smol_b200_qkn_decode_step_embeds(NULL, &st->model, 1, st->x_dev, st->token_dev, st->k_pool, st->v_pool,
                                         (int64_t)ctx->config.dec_layers * st->cap, st->row0_dev, st->kv_len_dev,
                                         (int)st->cap - 1, st->cos, st->sin, 0, st->step_ws, st->step_ws_bytes,
                                         st->xn_dev) != SMOL_B200_OK ||
        smol_b200_copy(&token, st->token_dev, sizeof(int)) != SMOL_B200_OK ||
        smol_b200_copy(ctx->dec_x, st->xn_dev, H * 4) != SMOL_B200_OK) {
        fprintf(stderr, "qkn_decoder_forward (device): %s\n", smol_cuda_error_string(smol_cuda_last_error()));
        return DEVICE_TOKEN_ON_ERROR;
    }
    ctx->kv_cache_len = pos + 1;
    return token;
}
