/*
 * device_core_fake_main.c -- checks the host logic of smol-genius_b200/dropin/device_decoder.c
 * on the CPU: the side table of contexts, the upload of a decoder's weights, the growth of
 * the KV pools, the positions-held guard, release, and failed allocations.
 *
 * The calls into libsmol_b200 are the fakes of fake_smol_b200.c: registered host memory
 * as device memory, and prefill / decode calls that check the pool rows written earlier
 * are still where the library would read them -- so a pool growth that lost or
 * misplaced rows is caught.
 *
 * Exit status 0 when every check passes; otherwise 1, with the failing check on stderr.
 */
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include "fake_smol_b200.h"

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

/* A seeded random sequence of prefills, decode steps, truncations, cache resets,
 * releases, single failed allocations and failures inside the library calls, against a
 * model of what each must do: a call succeeds exactly when its position is within the
 * ones held and nothing was made to fail; after a failure inside the library the rows
 * from the call's position on are no longer held; and every call checks, through the
 * fakes, that all rows written before are still where the library reads them. */
static void check_random_operations(void)
{
    host_model h;
    make_model(&h, 1, 900);
    int ctx_r;
    uint64_t rng = 12345;
    int held = 0, failures_seen = 0, ok_ops = 0, max_held = 0;
    float xn[HID];
    dd_state *st = set_up(&ctx_r, &h);
    CHECK(st != NULL);
    for (int op = 0; op < 3000 && st; op++) {
        rng = rng * 6364136223846793005ull + 1442695040888963407ull;
        const unsigned r = (unsigned)(rng >> 33);
        const int inject = r % 7 == 0;                   /* one allocation of this call fails */
        const int fail_call = !inject && r % 23 == 0;    /* the library call itself fails */
        if (inject) g_fail_at = g_allocs + (int)((r >> 8) % 5);
        g_fail_call = fail_call;
        int want_ok, rc;
        const unsigned kind = (r >> 4) % 100;   /* 25 % prefill, 60 % decode, 10 % truncate, 3 % reset, 2 % release */
        if (kind < 25) {   /* prefill at a position near the end of what is held */
            const int start = held - (int)((r >> 12) % 4) + (int)((r >> 16) % 3) - 1;
            const int n = 1 + (int)((r >> 20) % 300);
            want_ok = start >= 0 && start <= held;
            rc = start >= 0 ? prefill(st, start, n) : -1;
            if (rc == 0) held = start + n;
            if (fail_call && want_ok) {
                CHECK(rc == -1);
                held = start < held ? start : held;
                want_ok = 0;
            }
        } else if (kind < 95) {   /* a decode step at the end (or just past it), or after a truncation */
            int pos = held + ((r >> 12) % 16 == 0 ? 1 : 0);
            if (kind >= 85) pos = held > 0 ? (int)((r >> 16) % (unsigned)held) : 0;
            want_ok = pos <= held;
            const int tok = step(st, pos, xn);
            rc = tok < 0 ? -1 : 0;
            if (rc == 0) {
                CHECK(tok == pos % VOCAB);
                held = pos + 1;
            }
            if (fail_call && want_ok) {
                CHECK(rc == -1);
                held = pos < held ? pos : held;
                want_ok = 0;
            }
        } else if (kind < 98) {   /* a cache reset: prefill from 0 */
            const int n = 1 + (int)((r >> 12) % 50);
            want_ok = !fail_call;
            rc = prefill(st, 0, n);
            if (rc == 0) held = n;
            if (fail_call) held = 0;
        } else {   /* release and set up again */
            g_fail_at = -1;
            g_fail_call = 0;
            CHECK(dd_slot_release(&ctx_r) == 1);
            st = set_up(&ctx_r, &h);
            CHECK(st != NULL);
            held = 0;
            continue;
        }
        g_fail_at = -1;
        g_fail_call = 0;
        if (inject && want_ok && rc != 0) {
            failures_seen++;   /* the failed allocation hit this call: the next calls must still work */
            continue;
        }
        CHECK((rc == 0) == want_ok);
        CHECK(st->held == held);
        ok_ops += rc == 0;
        max_held = held > max_held ? held : max_held;
    }
    CHECK(failures_seen > 10 && ok_ops > 1500 && max_held > 2100);   /* at least two pool growths */
    CHECK(dd_slot_release(&ctx_r) == 1 && g_live == 0);
    printf("random operations: %d succeeded, %d failed allocations, up to %d positions\n", ok_ops, failures_seen,
           max_held);
}

int main(void)
{
    check_decoder(0);
    check_decoder(1);
    check_slots();
    check_failed_uploads(0);
    check_failed_uploads(1);
    check_random_operations();
    printf("prefills %d steps %d failures %d\n", g_prefills, g_steps, g_failures);
    return g_failures ? 1 : 0;
}
