/*
 * device_decoder.c -- see device_decoder.h.
 */
#include "device_decoder.h"

#include <stdio.h>
#include <stdlib.h>
#include <string.h>

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

/* RoPE tables for positions [0, rows): the formula of qkn_decoder.c:261-311 and
 * smol_compute_rope_* (rope.c:27-66) -- 1/powf(theta, 2d/hd), cosf / sinf of pos * f. */
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

void dd_release(dd_state *st)
{
    for (int l = 0; l < DD_MAX_LAYERS; l++) {
        smol_b200_qkn_layer *o = &st->layers[l];
        const void *bufs[] = {o->wq, o->wk, o->wv, o->wo, o->gate_up, o->down, o->input_norm, o->post_attn_norm,
                              o->q_norm, o->k_norm, o->pre_ffn_norm, o->post_ffn_norm};
        for (size_t i = 0; i < sizeof(bufs) / sizeof(bufs[0]); i++) smol_b200_device_free((void *)bufs[i]);
    }
    const void *bufs[] = {st->model.tok_embeddings, st->model.final_norm, st->model.lm_head, st->k_pool, st->v_pool,
                          st->row0_dev, st->cos, st->sin, st->cos_local, st->sin_local, st->step_in_dev,
                          st->step_out_dev, st->x_dev, st->step_ws, st->prefill_ws};
    for (size_t i = 0; i < sizeof(bufs) / sizeof(bufs[0]); i++) smol_b200_device_free((void *)bufs[i]);
    free(st->step_in_host);
    free(st->step_out_host);
    memset(st, 0, sizeof(*st));
}

uint64_t dd_fingerprint(int hidden, int layers, int vocab, const uint16_t *tok_embeddings, const uint16_t *wq0)
{
    uint64_t h = 1469598103934665603ull;   /* FNV-1a over the addresses, the shape and a few values */
    const uint64_t words[] = {(uint64_t)(uintptr_t)tok_embeddings, (uint64_t)(uintptr_t)wq0, (uint64_t)hidden,
                              (uint64_t)layers, (uint64_t)vocab};
    for (size_t i = 0; i < sizeof(words) / sizeof(words[0]); i++) h = (h ^ words[i]) * 1099511628211ull;
    for (int i = 0; i < 32 && tok_embeddings && wq0; i++) {
        h = (h ^ tok_embeddings[i]) * 1099511628211ull;
        h = (h ^ wq0[i]) * 1099511628211ull;
    }
    return h;
}

static struct {
    const void *ctx;
    uint64_t fingerprint;
    dd_state st;
} g_slots[DD_MAX_CONTEXTS];

dd_state *dd_slot_find(const void *ctx, uint64_t fingerprint, int *ready)
{
    int free_slot = -1;
    *ready = 0;
    for (int i = 0; i < DD_MAX_CONTEXTS; i++) {
        if (g_slots[i].ctx == ctx) {
            if (g_slots[i].fingerprint == fingerprint) {
                *ready = 1;
                return &g_slots[i].st;
            }
            /* the same address now holds another model: start over */
            dd_release(&g_slots[i].st);
            g_slots[i].ctx = NULL;
        }
        if (!g_slots[i].ctx && free_slot < 0) free_slot = i;
    }
    return free_slot < 0 ? NULL : &g_slots[free_slot].st;
}

void dd_slot_claim(dd_state *st, const void *ctx, uint64_t fingerprint)
{
    for (int i = 0; i < DD_MAX_CONTEXTS; i++) {
        if (&g_slots[i].st != st) continue;
        g_slots[i].ctx = ctx;
        g_slots[i].fingerprint = fingerprint;
    }
}

int dd_slot_release(const void *ctx)
{
    int found = 0;
    for (int i = 0; i < DD_MAX_CONTEXTS; i++) {
        if (!ctx || g_slots[i].ctx != ctx) continue;
        dd_release(&g_slots[i].st);
        g_slots[i].ctx = NULL;
        g_slots[i].fingerprint = 0;
        found = 1;
    }
    return found;
}

int dd_setup(dd_state *st, const dd_config *c, const dd_layer *layers, const uint16_t *tok_embeddings,
             const float *final_norm, const uint16_t *lm_head)
{
    if (c->layers < 1 || c->layers > DD_MAX_LAYERS) return -1;
    memset(st, 0, sizeof(*st));
    st->cfg = *c;
    const size_t H = (size_t)c->hidden, I = (size_t)c->intermediate, HD = (size_t)c->head_dim;
    const size_t qd = (size_t)c->heads * HD, kvd = (size_t)c->kv_heads * HD;
    for (int l = 0; l < c->layers; l++) {
        const dd_layer *ly = &layers[l];
        smol_b200_qkn_layer *o = &st->layers[l];
        o->wq = (const uint16_t *)upload(ly->wq, qd * H * 2);
        o->wk = (const uint16_t *)upload(ly->wk, kvd * H * 2);
        o->wv = (const uint16_t *)upload(ly->wv, kvd * H * 2);
        o->wo = (const uint16_t *)upload(ly->wo, H * qd * 2);
        o->gate_up = (const uint16_t *)upload(ly->gate_up, 2 * I * H * 2);
        o->down = (const uint16_t *)upload(ly->down, H * I * 2);
        o->input_norm = (const float *)upload(ly->input_norm, H * 4);
        o->post_attn_norm = (const float *)upload(ly->post_attn_norm, H * 4);
        o->q_norm = (const float *)upload(ly->q_norm, HD * 4);
        o->k_norm = (const float *)upload(ly->k_norm, HD * 4);
        o->pre_ffn_norm = (const float *)upload(ly->pre_ffn_norm, H * 4);
        o->post_ffn_norm = (const float *)upload(ly->post_ffn_norm, H * 4);
        o->is_sliding = ly->is_sliding;
        /* the optional norms are absent only when the host has none (a failed upload is a failure) */
        if (!o->wq || !o->wk || !o->wv || !o->wo || !o->gate_up || !o->down || !o->input_norm || !o->post_attn_norm ||
            (ly->q_norm && !o->q_norm) || (ly->k_norm && !o->k_norm) || (ly->pre_ffn_norm && !o->pre_ffn_norm) ||
            (ly->post_ffn_norm && !o->post_ffn_norm)) {
            dd_release(st);
            return -1;
        }
    }
    smol_b200_qkn_model *m = &st->model;
    m->hidden = c->hidden;
    m->n_layers = c->layers;
    m->n_heads = c->heads;
    m->n_kv_heads = c->kv_heads;
    m->head_dim = c->head_dim;
    m->intermediate = c->intermediate;
    m->vocab = c->vocab;
    m->eps = c->eps;
    m->rope_interleaved = c->interleaved;
    m->tok_embeddings = (const uint16_t *)upload(tok_embeddings, (size_t)c->vocab * H * 2);
    m->final_norm = (const float *)upload(final_norm, H * 4);
    m->lm_head = (const uint16_t *)upload(lm_head, (size_t)c->vocab * H * 2);
    m->layers = st->layers;
    m->activation = c->geglu ? 1 : 0;
    m->embed_normalizer = c->embed_normalizer;
    m->attn_softcap = c->attn_softcap;
    m->sliding_window = c->sliding_window;
    st->step_in_dev = (float *)smol_b200_device_alloc((H + 1) * 4);
    st->step_out_dev = (float *)smol_b200_device_alloc((H + 1) * 4);
    st->step_in_host = (float *)malloc((H + 1) * 4);
    st->step_out_host = (float *)malloc((H + 1) * 4);
    if (!m->tok_embeddings || !m->final_norm || (lm_head && !m->lm_head) || !st->step_in_dev || !st->step_out_dev ||
        !st->step_in_host || !st->step_out_host) {
        dd_release(st);
        return -1;
    }
    st->ready = 1;
    return 0;
}

/* Pools, tables and buffers for positions [0, need) and n_in input rows; the first
 * `cached` positions (all the held ones) are kept when the pool grows (rows copied on
 * the device), so a call that fails after a growth loses none of them. */
static int ensure_capacity(dd_state *st, int need, int cached, int n_in)
{
    const dd_config *c = &st->cfg;
    const size_t H = (size_t)c->hidden, kvd = (size_t)c->kv_heads * c->head_dim;
    const int L = c->layers;
    if (need > st->cap) {
        const int64_t cap = need + 1024 > 2 * st->cap ? need + 1024 : 2 * st->cap;
        uint16_t *k = (uint16_t *)smol_b200_device_alloc((size_t)L * cap * kvd * 2);
        uint16_t *v = (uint16_t *)smol_b200_device_alloc((size_t)L * cap * kvd * 2);
        const int keep = cached < st->cap ? cached : (int)st->cap;
        int ok = k && v;
        for (int l = 0; l < L && ok && st->k_pool && keep > 0; l++) {
            if (smol_b200_copy(k + (size_t)l * cap * kvd, st->k_pool + (size_t)l * st->cap * kvd,
                               (size_t)keep * kvd * 2) != SMOL_B200_OK ||
                smol_b200_copy(v + (size_t)l * cap * kvd, st->v_pool + (size_t)l * st->cap * kvd,
                               (size_t)keep * kvd * 2) != SMOL_B200_OK)
                ok = 0;
        }
        if (!ok) {   /* the old pools stay as they were */
            smol_b200_device_free(k);
            smol_b200_device_free(v);
            return 0;
        }
        smol_b200_device_free(st->k_pool);
        smol_b200_device_free(st->v_pool);
        st->k_pool = k;
        st->v_pool = v;
        st->cap = cap;
        for (int l = 0; l < L; l++) st->row0_host[l] = (int64_t)l * cap;
        /* both depend on the capacity: made again below */
        smol_b200_device_free(st->row0_dev);
        st->row0_dev = NULL;
        smol_b200_device_free(st->step_ws);
        st->step_ws = NULL;
    }
    /* (also retried here after a failed allocation of an earlier call) */
    if (!st->row0_dev) {
        st->row0_dev = (int64_t *)upload(st->row0_host, sizeof(int64_t) * (size_t)L);
        if (!st->row0_dev) return 0;
    }
    if (!st->step_ws) {
        st->step_ws_bytes = smol_b200_qkn_step_workspace_bytes(&st->model, 1, (int)st->cap - 1);
        st->step_ws = smol_b200_device_alloc(st->step_ws_bytes);
        if (!st->step_ws) return 0;
    }
    /* sliding layers' own theta (qkn_decoder.c:313-340) */
    const int want_local = c->local_theta > 0.0f && c->local_theta != c->theta;
    if (need > st->rope_cap || !st->cos || !st->sin || (want_local && (!st->cos_local || !st->sin_local))) {
        /* until both sets are made again, nothing refers to the old ones */
        st->rope_cap = 0;
        st->model.rope_cos_local = NULL;
        st->model.rope_sin_local = NULL;
        const int rows = (int)st->cap;
        if (!rope_tables(&st->cos, &st->sin, rows, c->head_dim, c->theta, c->interleaved)) return 0;
        if (want_local) {
            if (!rope_tables(&st->cos_local, &st->sin_local, rows, c->head_dim, c->local_theta, c->interleaved))
                return 0;
            st->model.rope_cos_local = st->cos_local;
            st->model.rope_sin_local = st->sin_local;
        }
        st->rope_cap = rows;
    }
    if (n_in > st->x_cap || !st->x_dev) {
        const int rows = n_in > st->x_cap ? n_in : st->x_cap;
        smol_b200_device_free(st->x_dev);
        st->x_dev = (float *)smol_b200_device_alloc((size_t)rows * H * 4);
        st->x_cap = st->x_dev ? rows : 0;
        if (!st->x_dev) return 0;
    }
    return 1;
}

/* Positions past the ones written would be attended as uninitialised rows. */
static int position_held(const dd_state *st, int pos)
{
    if (pos >= 0 && pos <= st->held) return 1;
    fprintf(stderr, "device decoder: position %d is past the %d positions held on the device\n", pos, st->held);
    return 0;
}

/* After a call that failed inside the library the rows from `pos` on may hold a partial
 * write: only the positions before it stay trusted.  (A failed allocation before the
 * call leaves every held row in place: pool growth copies all of them.) */
static void distrust_from(dd_state *st, int pos)
{
    if (st->held > pos) st->held = pos;
}

int dd_prefill(dd_state *st, const float *embeds, int n, int start)
{
    if (n <= 0) return 0;
    if (!st->ready || !position_held(st, start) || !ensure_capacity(st, start + n + 1, st->held, n)) return -1;
    if (n > st->prefill_cap) {
        smol_b200_device_free(st->prefill_ws);
        st->prefill_ws_bytes = smol_b200_qkn_prefill_workspace_bytes(&st->model, n);
        st->prefill_ws = smol_b200_device_alloc(st->prefill_ws_bytes);
        st->prefill_cap = st->prefill_ws ? n : 0;
    }
    if (!st->prefill_ws || smol_b200_copy(st->x_dev, embeds, (size_t)n * st->cfg.hidden * 4) != SMOL_B200_OK)
        return -1;
    if (smol_b200_qkn_prefill_embeds(NULL, &st->model, st->x_dev, n, start, st->k_pool, st->v_pool,
                                     (int64_t)st->cfg.layers * st->cap, st->row0_host, st->cos, st->sin,
                                     st->prefill_ws, st->prefill_ws_bytes) != SMOL_B200_OK) {
        distrust_from(st, start);
        return -1;
    }
    st->held = start + n;
    return 0;
}

int dd_forward(dd_state *st, const float *embed, int pos, float *x_normed)
{
    int token = -1;
    const size_t H = (size_t)st->cfg.hidden;
    if (!st->ready || !position_held(st, pos) || !ensure_capacity(st, pos + 2, st->held, 1)) return -1;
    memcpy(st->step_in_host, embed, H * 4);
    memcpy(st->step_in_host + H, &pos, sizeof(int));
    if (smol_b200_copy(st->step_in_dev, st->step_in_host, (H + 1) * 4) != SMOL_B200_OK) return -1;
    if (smol_b200_qkn_decode_step_embeds(NULL, &st->model, 1, st->step_in_dev, (int *)(st->step_out_dev + H),
                                         st->k_pool, st->v_pool, (int64_t)st->cfg.layers * st->cap, st->row0_dev,
                                         (int *)(st->step_in_dev + H),
                                         pos /* the split-KV plan follows the actual length */, st->cos, st->sin, 0,
                                         st->step_ws, st->step_ws_bytes, st->step_out_dev) != SMOL_B200_OK ||
        smol_b200_copy(st->step_out_host, st->step_out_dev, (H + 1) * 4) != SMOL_B200_OK) {
        distrust_from(st, pos);
        return -1;
    }
    memcpy(&token, st->step_out_host + H, sizeof(int));
    if (x_normed) memcpy(x_normed, st->step_out_host, H * 4);
    st->held = pos + 1;
    return token;
}
