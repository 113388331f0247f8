/*
 * device_core_fake_main.c -- checks the host logic of smol-genius_b200/dropin/device_decoder.c
 * on the CPU: the side table of contexts, the upload of a decoder's weights, the growth of
 * the KV pools, the positions-held guard, release, and failed allocations.
 *
 * The calls into libsmol_b200 are replaced by fakes defined here.  "Device" memory is
 * host memory kept in a registry (so every pointer the core hands to the library can be
 * checked to be one of its own live allocations, of sufficient size), with a count of
 * live allocations and an optional failure of one chosen allocation.  The fake prefill and
 * decode calls check that every pool row written earlier still holds its tag at the row
 * the library would read it from (layer_row0[l] + position), then tag the rows they
 * write -- so a pool growth that lost or misplaced rows is caught.
 *
 * Exit status 0 when every check passes; otherwise 1, with the failing check on stderr.
 */
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include "device_decoder.h"

static int g_failures = 0;
#define CHECK(cond)                                                              \
    do {                                                                         \
        if (!(cond)) {                                                           \
            fprintf(stderr, "%s:%d: check failed: %s\n", __FILE__, __LINE__, #cond); \
            g_failures++;                                                        \
        }                                                                        \
    } while (0)

/* ---------------------------------------------------------------- fake device memory */
#define MAX_ALLOCS 4096
static struct {
    void *p;
    size_t bytes;
} g_reg[MAX_ALLOCS];
static int g_live = 0, g_allocs = 0, g_fail_at = -1;   /* the allocation with index g_fail_at fails */

void *smol_b200_device_alloc(size_t bytes)
{
    if (g_allocs++ == g_fail_at) return NULL;
    void *p = malloc(bytes ? bytes : 1);
    if (!p) return NULL;
    for (int i = 0; i < MAX_ALLOCS; i++)
        if (!g_reg[i].p) {
            g_reg[i].p = p;
            g_reg[i].bytes = bytes;
            g_live++;
            return p;
        }
    free(p);
    return NULL;
}

void smol_b200_device_free(void *p)
{
    if (!p) return;
    for (int i = 0; i < MAX_ALLOCS; i++)
        if (g_reg[i].p == p) {
            g_reg[i].p = NULL;
            g_live--;
            free(p);
            return;
        }
    fprintf(stderr, "free of a pointer that is not a live device allocation\n");
    g_failures++;
}

/* bytes of the live allocation holding p (0 when p is not inside one) */
static size_t dev_bytes_from(const void *p)
{
    for (int i = 0; i < MAX_ALLOCS; i++) {
        const char *b = (const char *)g_reg[i].p;
        if (b && (const char *)p >= b && (const char *)p < b + g_reg[i].bytes)
            return g_reg[i].bytes - (size_t)((const char *)p - b);
    }
    return 0;
}

int smol_b200_copy(void *dst, const void *src, size_t bytes)
{
    if (bytes == 0) return SMOL_B200_OK;
    if (!dst || !src) return SMOL_B200_ERR_ARGS;
    memcpy(dst, src, bytes);
    return SMOL_B200_OK;
}

size_t smol_b200_qkn_step_workspace_bytes(const smol_b200_qkn_model *m, int n_seqs, int max_kv_len)
{
    (void)m;
    return 256 + (size_t)n_seqs * (size_t)(max_kv_len + 1) * 4;
}

size_t smol_b200_qkn_prefill_workspace_bytes(const smol_b200_qkn_model *m, int n_tokens)
{
    (void)m;
    return 256 + (size_t)n_tokens * 8;
}

static void fake_rope(float *c, float *s, const int *pos, int seq, int head_dim)
{
    for (int i = 0; i < seq; i++)
        for (int d = 0; d < head_dim; d++) {
            c[(size_t)i * head_dim + d] = (float)pos[i];   /* row i holds its position */
            s[(size_t)i * head_dim + d] = 0.0f;
        }
}

void smol_compute_rope_neox(float *c, float *s, const int *pos, int seq, int head_dim, float theta)
{
    (void)theta;
    fake_rope(c, s, pos, seq, head_dim);
}

void smol_compute_rope_interleaved(float *c, float *s, const int *pos, int seq, int head_dim, float theta)
{
    (void)theta;
    fake_rope(c, s, pos, seq, head_dim);
}

/* ---------------------------------------------------------------- fake prefill / decode */
static uint16_t tag_k(int l, int p) { return (uint16_t)(1 + l * 2003 + p); }
static uint16_t tag_v(int l, int p) { return (uint16_t)(tag_k(l, p) ^ 0x8000u); }

static int g_prefills = 0, g_steps = 0;

/* rows [0, n_pos) of every layer hold their tags; row `write` (and up) gets tagged */
static int check_and_tag(const smol_b200_qkn_model *m, uint16_t *k_pool, uint16_t *v_pool, int64_t pool_rows,
                         const int64_t *row0, int n_pos, int write, int n_write)
{
    const int kvd = m->n_kv_heads * m->head_dim;
    if (dev_bytes_from(k_pool) < (size_t)pool_rows * kvd * 2 || dev_bytes_from(v_pool) < (size_t)pool_rows * kvd * 2)
        return 0;
    for (int l = 0; l < m->n_layers; l++) {
        if (row0[l] < 0 || row0[l] + write + n_write > pool_rows) return 0;
        for (int p = 0; p < n_pos; p++)
            for (int e = 0; e < kvd; e += kvd - 1)   /* the first and last element of each row */
                if (k_pool[(row0[l] + p) * kvd + e] != tag_k(l, p) || v_pool[(row0[l] + p) * kvd + e] != tag_v(l, p))
                    return 0;
        for (int p = write; p < write + n_write; p++)
            for (int e = 0; e < kvd; e++) {
                k_pool[(row0[l] + p) * kvd + e] = tag_k(l, p);
                v_pool[(row0[l] + p) * kvd + e] = tag_v(l, p);
            }
    }
    return 1;
}

/* the model struct handed to the library holds device copies, never the host pointers */
static int model_on_device(const smol_b200_qkn_model *m)
{
    const size_t H = (size_t)m->hidden, qd = (size_t)m->n_heads * m->head_dim;
    const size_t kvd = (size_t)m->n_kv_heads * m->head_dim;
    if (dev_bytes_from(m->tok_embeddings) < (size_t)m->vocab * H * 2 || dev_bytes_from(m->final_norm) < H * 4)
        return 0;
    if (m->lm_head && dev_bytes_from(m->lm_head) < (size_t)m->vocab * H * 2) return 0;
    for (int l = 0; l < m->n_layers; l++) {
        const smol_b200_qkn_layer *L = &m->layers[l];
        if (dev_bytes_from(L->wq) < qd * H * 2 || dev_bytes_from(L->wk) < kvd * H * 2 ||
            dev_bytes_from(L->wv) < kvd * H * 2 || dev_bytes_from(L->wo) < H * qd * 2 ||
            dev_bytes_from(L->gate_up) < 2 * (size_t)m->intermediate * H * 2 ||
            dev_bytes_from(L->down) < H * (size_t)m->intermediate * 2 || dev_bytes_from(L->input_norm) < H * 4 ||
            dev_bytes_from(L->post_attn_norm) < H * 4)
            return 0;
        if ((L->q_norm && dev_bytes_from(L->q_norm) < (size_t)m->head_dim * 4) ||
            (L->pre_ffn_norm && dev_bytes_from(L->pre_ffn_norm) < H * 4))
            return 0;
    }
    return 1;
}

int smol_b200_qkn_prefill_embeds(void *stream, const smol_b200_qkn_model *m, const float *embeds, int n, int start,
                                 uint16_t *k_pool, uint16_t *v_pool, int64_t pool_rows, const int64_t *row0_host,
                                 const float *cos, const float *sin, void *ws, size_t ws_bytes)
{
    (void)stream;
    g_prefills++;
    const size_t H = (size_t)m->hidden, hd = (size_t)m->head_dim;
    if (!model_on_device(m) || dev_bytes_from(embeds) < (size_t)n * H * 4 ||
        dev_bytes_from(ws) < ws_bytes || ws_bytes < smol_b200_qkn_prefill_workspace_bytes(m, n) ||
        dev_bytes_from(cos) < (size_t)(start + n) * hd * 4 || dev_bytes_from(sin) < (size_t)(start + n) * hd * 4 ||
        dev_bytes_from(row0_host) != 0)   /* the prefill takes the pool rows on the host */
        return SMOL_B200_ERR_ARGS;
    for (int t = 0; t < n; t++)
        if (embeds[(size_t)t * H] != (float)(start + t)) return SMOL_B200_ERR_ARGS;
    return check_and_tag(m, k_pool, v_pool, pool_rows, row0_host, start, start, n) ? SMOL_B200_OK : SMOL_B200_ERR_ARGS;
}

int smol_b200_qkn_decode_step_embeds(void *stream, const smol_b200_qkn_model *m, int n_seqs, const float *embeds,
                                     int *tokens_out, uint16_t *k_pool, uint16_t *v_pool, int64_t pool_rows,
                                     const int64_t *layer_row0, int *kv_len, int max_kv_len, const float *cos,
                                     const float *sin, int advance, void *ws, size_t ws_bytes, float *x_normed_out)
{
    (void)stream;
    g_steps++;
    const size_t H = (size_t)m->hidden, hd = (size_t)m->head_dim;
    if (n_seqs != 1 || advance != 0 || !model_on_device(m) || dev_bytes_from(embeds) < H * 4 ||
        dev_bytes_from(tokens_out) < 4 || dev_bytes_from(kv_len) < 4 || dev_bytes_from(layer_row0) < 8 * (size_t)m->n_layers ||
        dev_bytes_from(ws) < ws_bytes || ws_bytes < smol_b200_qkn_step_workspace_bytes(m, 1, max_kv_len) ||
        (x_normed_out && dev_bytes_from(x_normed_out) < H * 4))
        return SMOL_B200_ERR_ARGS;
    const int pos = kv_len[0];
    if (pos < 0 || pos > max_kv_len || dev_bytes_from(cos) < (size_t)(pos + 1) * hd * 4 ||
        dev_bytes_from(sin) < (size_t)(pos + 1) * hd * 4 || cos[(size_t)pos * hd] != (float)pos)
        return SMOL_B200_ERR_ARGS;
    if (m->rope_cos_local && dev_bytes_from(m->rope_cos_local) < (size_t)(pos + 1) * hd * 4) return SMOL_B200_ERR_ARGS;
    if (!check_and_tag(m, k_pool, v_pool, pool_rows, layer_row0, pos, pos, 1)) return SMOL_B200_ERR_ARGS;
    tokens_out[0] = pos % m->vocab;
    if (x_normed_out)
        for (size_t i = 0; i < H; i++) x_normed_out[i] = embeds[i] + 0.5f;
    return SMOL_B200_OK;
}

/* ---------------------------------------------------------------- the checks */
enum { HID = 64, LAYERS = 3, HEADS = 2, KV = 1, HD = 64, INTER = 96, VOCAB = 50 };

typedef struct {
    dd_config cfg;
    dd_layer layers[LAYERS];
    uint16_t *emb, *lm_head;
    float *final_norm;
} host_model;

static uint16_t *host_u16(size_t n, uint16_t seed)
{
    uint16_t *p = (uint16_t *)malloc(n * 2);
    for (size_t i = 0; i < n; i++) p[i] = (uint16_t)(seed + i * 7);
    return p;
}

static float *host_f32(size_t n)
{
    float *p = (float *)malloc(n * 4);
    for (size_t i = 0; i < n; i++) p[i] = 1.0f + 0.001f * (float)i;
    return p;
}

static void make_model(host_model *h, int gemma, uint16_t seed)
{
    memset(h, 0, sizeof(*h));
    dd_config *c = &h->cfg;
    c->hidden = HID;
    c->layers = LAYERS;
    c->heads = HEADS;
    c->kv_heads = KV;
    c->head_dim = HD;
    c->intermediate = INTER;
    c->vocab = VOCAB;
    c->eps = 1e-6f;
    c->theta = 1e4f;
    if (gemma) {
        c->local_theta = 1e3f;
        c->embed_normalizer = 8.0f;
        c->sliding_window = 4;
        c->geglu = 1;
        c->interleaved = 1;
    }
    for (int l = 0; l < LAYERS; l++) {
        dd_layer *L = &h->layers[l];
        L->wq = host_u16((size_t)HEADS * HD * HID, seed + 1);
        L->wk = host_u16((size_t)KV * HD * HID, seed + 2);
        L->wv = host_u16((size_t)KV * HD * HID, seed + 3);
        L->wo = host_u16((size_t)HID * HEADS * HD, seed + 4);
        L->gate_up = host_u16((size_t)2 * INTER * HID, seed + 5);
        L->down = host_u16((size_t)HID * INTER, seed + 6);
        L->input_norm = host_f32(HID);
        L->post_attn_norm = host_f32(HID);
        L->q_norm = host_f32(HD);
        L->k_norm = host_f32(HD);
        if (gemma) {
            L->pre_ffn_norm = host_f32(HID);
            L->post_ffn_norm = host_f32(HID);
            L->is_sliding = l % 2 == 0;
        }
    }
    h->emb = host_u16((size_t)VOCAB * HID, seed);
    h->final_norm = host_f32(HID);
    if (gemma) h->lm_head = host_u16((size_t)VOCAB * HID, seed + 9);
}

static uint64_t fingerprint(const host_model *h)
{
    return dd_fingerprint(HID, LAYERS, VOCAB, h->emb, h->layers[0].wq);
}

static dd_state *set_up(const void *ctx, const host_model *h)
{
    int ready = -1;
    const uint64_t fp = fingerprint(h);
    dd_state *st = dd_slot_find(ctx, fp, &ready);
    if (!st || ready) return st;
    if (dd_setup(st, &h->cfg, h->layers, h->emb, h->final_norm, h->lm_head) != 0) return NULL;
    dd_slot_claim(st, ctx, fp);
    return st;
}

static int step(dd_state *st, int pos, float *xn)
{
    float e[HID];
    for (int i = 0; i < HID; i++) e[i] = (float)pos;
    return dd_forward(st, e, pos, xn);
}

static int prefill(dd_state *st, int start, int n)
{
    float *e = (float *)malloc(sizeof(float) * (size_t)n * HID);
    for (int t = 0; t < n; t++)
        for (int i = 0; i < HID; i++) e[(size_t)t * HID + i] = (float)(start + t);
    const int rc = dd_prefill(st, e, n, start);
    free(e);
    return rc;
}

static void check_decoder(int gemma)
{
    host_model h;
    make_model(&h, gemma, gemma ? 300 : 100);
    int ctx_a;   /* any address serves as a context */
    int ready = -1;
    dd_state *st = set_up(&ctx_a, &h);
    CHECK(st != NULL);
    if (!st) return;
    CHECK(dd_slot_find(&ctx_a, fingerprint(&h), &ready) == st && ready == 1);
    CHECK(model_on_device(&st->model));
    CHECK(memcmp(st->model.layers[2].wq, h.layers[2].wq, (size_t)HEADS * HD * HID * 2) == 0);
    CHECK(memcmp(st->model.tok_embeddings, h.emb, (size_t)VOCAB * HID * 2) == 0);
    CHECK(st->model.embed_normalizer == h.cfg.embed_normalizer);
    CHECK(st->model.rope_interleaved == h.cfg.interleaved);
    CHECK(!gemma || (st->model.lm_head && memcmp(st->model.lm_head, h.lm_head, (size_t)VOCAB * HID * 2) == 0));
    CHECK(gemma || !st->model.lm_head);
    CHECK(!gemma || (st->model.layers[0].is_sliding == 1 && st->model.layers[1].is_sliding == 0));

    /* prefill, then decode past the first pool growth (capacity need + 1024 = 1035) */
    CHECK(prefill(st, 0, 10) == 0);
    float xn[HID];
    const int64_t cap0 = st->cap;
    int ok = 1;
    for (int pos = 10; pos < 1100 && ok; pos++) {
        const int tok = step(st, pos, xn);
        ok = tok == pos % VOCAB && xn[0] == (float)pos + 0.5f;
    }
    CHECK(ok);
    CHECK(st->cap > cap0 && st->held == 1100);
    CHECK(!gemma || (st->model.rope_cos_local && dev_bytes_from(st->model.rope_cos_local) >= (size_t)1100 * HD * 4));

    /* positions past the ones held are refused; truncation is honoured */
    CHECK(step(st, 1102, xn) == -1);
    CHECK(prefill(st, 1105, 2) == -1);
    CHECK(step(st, 5, xn) == 5 % VOCAB && st->held == 6);
    CHECK(prefill(st, 6, 3) == 0 && st->held == 9);
    CHECK(step(st, 9, xn) == 9);

    /* a failed pool growth keeps the old pools and rows; each allocation of the growth
     * (K pool, V pool, pool rows, step workspace, RoPE tables) failing in turn, on a
     * fresh context filled to one position short of the capacity */
    for (int k = 0; k < 8; k++) {
        int ctx_b;
        dd_state *sb = set_up(&ctx_b, &h);
        CHECK(sb != NULL);
        if (!sb) break;
        const int64_t cap = sb->cap > 0 ? sb->cap : 0;
        CHECK(prefill(sb, 0, 10) == 0);
        const int last = (int)sb->cap - 2;   /* the last position without growth */
        CHECK(cap == 0 && prefill(sb, 10, last - 10 + 1) == 0 && sb->held == last + 1);
        const int live = g_live;
        g_fail_at = g_allocs + k;
        const int tok = step(sb, last + 1, xn);
        g_fail_at = -1;
        CHECK(tok == -1 || tok == (last + 1) % VOCAB);
        if (tok == -1) {
            CHECK(k > 1 || g_live == live);                     /* a failed pool: nothing new kept */
            CHECK(step(sb, last + 1, xn) == (last + 1) % VOCAB);   /* retried, rows intact */
        }
        CHECK(sb->cap > last + 2 && step(sb, last + 2, xn) == (last + 2) % VOCAB);
        CHECK(dd_slot_release(&ctx_b) == 1);
    }

    /* the same address with other weights: the old state is released and set up afresh */
    host_model h2;
    make_model(&h2, gemma, 700);
    const int live_before = g_live;
    dd_state *st2 = dd_slot_find(&ctx_a, fingerprint(&h2), &ready);
    CHECK(st2 != NULL && ready == 0 && g_live < live_before);
    CHECK(st2 && dd_setup(st2, &h2.cfg, h2.layers, h2.emb, h2.final_norm, h2.lm_head) == 0);
    if (st2) dd_slot_claim(st2, &ctx_a, fingerprint(&h2));
    CHECK(st2 && memcmp(st2->model.tok_embeddings, h2.emb, (size_t)VOCAB * HID * 2) == 0);
    CHECK(st2 && prefill(st2, 0, 4) == 0 && step(st2, 4, xn) == 4);

    /* release frees everything, once */
    CHECK(dd_slot_release(&ctx_a) == 1);
    CHECK(g_live == 0);
    CHECK(dd_slot_release(&ctx_a) == 0);
}

static void check_slots(void)
{
    host_model h;
    make_model(&h, 0, 100);
    int ctxs[DD_MAX_CONTEXTS + 1];
    for (int i = 0; i < DD_MAX_CONTEXTS; i++) CHECK(set_up(&ctxs[i], &h) != NULL);
    int ready = -1;
    CHECK(dd_slot_find(&ctxs[DD_MAX_CONTEXTS], fingerprint(&h), &ready) == NULL);
    for (int i = 0; i < DD_MAX_CONTEXTS; i++) CHECK(dd_slot_release(&ctxs[i]) == 1);
    CHECK(g_live == 0);
}

/* every allocation of the upload is needed: each one failing in turn fails the set-up
 * and leaves nothing allocated (a missing optional norm would silently change the model) */
static void check_failed_uploads(int gemma)
{
    host_model h;
    make_model(&h, gemma, 500);
    int ctxs[1], ready = -1;
    const int a0 = g_allocs;
    CHECK(set_up(&ctxs[0], &h) != NULL && g_live > 0);
    const int n_setup = g_allocs - a0;
    CHECK(dd_slot_release(&ctxs[0]) == 1 && g_live == 0);
    for (int k = 0; k < n_setup; k++) {
        g_fail_at = g_allocs + k;
        dd_state *st = dd_slot_find(&ctxs[0], fingerprint(&h), &ready);
        CHECK(st != NULL && ready == 0);
        if (!st) break;
        CHECK(dd_setup(st, &h.cfg, h.layers, h.emb, h.final_norm, h.lm_head) == -1);
        CHECK(g_live == 0);
    }
    g_fail_at = -1;
    CHECK(set_up(&ctxs[0], &h) != NULL);
    CHECK(dd_slot_release(&ctxs[0]) == 1 && g_live == 0);
}

int main(void)
{
    check_decoder(0);
    check_decoder(1);
    check_slots();
    check_failed_uploads(0);
    check_failed_uploads(1);
    printf("prefills %d steps %d failures %d\n", g_prefills, g_steps, g_failures);
    return g_failures ? 1 : 0;
}
