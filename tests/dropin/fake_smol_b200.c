/*
 * fake_smol_b200.c -- fakes of the libsmol_b200 calls the decoder-level drop-ins make
 * (smol-genius_b200/dropin/), for checking their host logic on the CPU.
 *
 * "Device" memory is host memory kept in a registry, so every pointer handed to the
 * library can be checked to be one of its own live allocations, of sufficient size; a
 * count of live allocations, and an optional failure of one chosen allocation
 * (g_fail_at).  The fake prefill and decode calls check that every pool row written
 * earlier still holds its tag at the row the library would read it from
 * (layer_row0[l] + position), then tag the rows they write; the decode returns token
 * position % vocab and writes embed + 0.5 as the normalised state.  Both keep a copy of
 * the model struct they were given (g_last_model).  With g_fail_call set, the next of
 * them corrupts the first row it wrote and fails (a failure inside the library).
 */
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include "fake_smol_b200.h"

int g_failures = 0;

/* ---------------------------------------------------------------- fake device memory */
#define MAX_ALLOCS 4096
static struct {
    void *p;
    size_t bytes;
} g_reg[MAX_ALLOCS];
int g_live = 0, g_allocs = 0, g_fail_at = -1;   /* the allocation with index g_fail_at fails */

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
size_t dev_bytes_from(const void *p)
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
uint16_t tag_k(int l, int p) { return (uint16_t)(1 + l * 2003 + p); }
uint16_t tag_v(int l, int p) { return (uint16_t)(tag_k(l, p) ^ 0x8000u); }

int g_prefills = 0, g_steps = 0, g_check_embeds = 1, g_fail_call = 0;
smol_b200_qkn_model g_last_model;
static smol_b200_qkn_layer g_last_layers[DD_MAX_LAYERS];

/* the model struct of the last call, with its layers */
static void keep_model(const smol_b200_qkn_model *m)
{
    g_last_model = *m;
    for (int l = 0; l < m->n_layers && l < DD_MAX_LAYERS; l++) g_last_layers[l] = m->layers[l];
    g_last_model.layers = g_last_layers;
}

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
int model_on_device(const smol_b200_qkn_model *m)
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
    keep_model(m);
    const size_t H = (size_t)m->hidden, hd = (size_t)m->head_dim;
    if (!model_on_device(m) || dev_bytes_from(embeds) < (size_t)n * H * 4 ||
        dev_bytes_from(ws) < ws_bytes || ws_bytes < smol_b200_qkn_prefill_workspace_bytes(m, n) ||
        dev_bytes_from(cos) < (size_t)(start + n) * hd * 4 || dev_bytes_from(sin) < (size_t)(start + n) * hd * 4 ||
        dev_bytes_from(row0_host) != 0)   /* the prefill takes the pool rows on the host */
        return SMOL_B200_ERR_ARGS;
    for (int t = 0; t < n && g_check_embeds; t++)
        if (embeds[(size_t)t * H] != (float)(start + t)) return SMOL_B200_ERR_ARGS;
    if (!check_and_tag(m, k_pool, v_pool, pool_rows, row0_host, start, start, n)) return SMOL_B200_ERR_ARGS;
    if (g_fail_call) {   /* a failure inside the library after a partial write */
        g_fail_call = 0;
        k_pool[(size_t)(row0_host[0] + start) * m->n_kv_heads * m->head_dim] = 0xdead;
        return SMOL_B200_ERR_CUDA;
    }
    return SMOL_B200_OK;
}

int smol_b200_qkn_decode_step_embeds(void *stream, const smol_b200_qkn_model *m, int n_seqs, const float *embeds,
                                     int *tokens_out, uint16_t *k_pool, uint16_t *v_pool, int64_t pool_rows,
                                     const int64_t *layer_row0, int *kv_len, int max_kv_len, const float *cos,
                                     const float *sin, int advance, void *ws, size_t ws_bytes, float *x_normed_out)
{
    (void)stream;
    g_steps++;
    keep_model(m);
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
    if (g_fail_call) {   /* a failure inside the library after a partial write */
        g_fail_call = 0;
        k_pool[(size_t)(layer_row0[0] + pos) * m->n_kv_heads * m->head_dim] = 0xdead;
        return SMOL_B200_ERR_CUDA;
    }
    tokens_out[0] = pos % m->vocab;
    if (x_normed_out)
        for (size_t i = 0; i < H; i++) x_normed_out[i] = embeds[i] + 0.5f;
    return SMOL_B200_OK;
}

int smol_cuda_last_error(void)
{
    return SMOL_B200_ERR_ARGS;
}

const char *smol_cuda_error_string(int code)
{
    (void)code;
    return "fake library";
}
