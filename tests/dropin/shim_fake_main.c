/*
 * shim_fake_main.c -- checks, on the CPU, that a decoder-level drop-in hands the
 * reference context's configuration and weights to the library unchanged.
 *
 * Built twice by oracle/Makefile (target `dropin`) against the reference's own headers:
 *   -DSHIM_QKN     with smol-genius_b200/dropin/qkn_decoder_device.c and qkn_ctx_t in its
 *                  Gemma 2 settings (GeGLU, interleaved RoPE, a local RoPE theta, sliding
 *                  layers, softcap, embedding normaliser, QK-norm and the sublayer norms);
 *   -DSHIM_SMOLVLM with smol-genius_b200/dropin/smolvlm_decoder_device.c and smolvlm_ctx_t
 *                  (no QK-norm, untied output head).
 * The library calls are the fakes of fake_smol_b200.c; the model struct the fakes last
 * received is compared field by field and weight by weight with the context.  Also:
 * kv_cache_len and dec_x after prefill / forward, a chunked prefill and a cache reset
 * (the fake prefill checks each chunk's inputs arrive at their positions), the failure
 * sentinel for a position past the ones the device holds, release, and a context whose
 * weights changed.
 *
 * Exit status 0 when every check passes; otherwise 1, with the failing check on stderr.
 */
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include "fake_smol_b200.h"

#if defined(SHIM_QKN)
#include "qkn_decoder.h"
typedef qkn_ctx_t ctx_t;
typedef qkn_dec_layer_t layer_t;
#define PREFILL qkn_decoder_prefill
#define FORWARD qkn_decoder_forward
#define RELEASE qkn_decoder_device_release
#define SENTINEL 151645
#define GEMMA 1
#elif defined(SHIM_SMOLVLM)
#include "smolvlm.h"
typedef smolvlm_ctx_t ctx_t;
typedef smolvlm_dec_layer_t layer_t;
#define PREFILL smolvlm_decoder_prefill
#define FORWARD smolvlm_decoder_forward
#define RELEASE smolvlm_decoder_device_release
#define SENTINEL 49154
#define GEMMA 0
#else
#error "build with -DSHIM_QKN or -DSHIM_SMOLVLM"
#endif

void RELEASE(ctx_t *ctx);

enum { HID = 64, LAYERS = 3, HEADS = 2, KV = 1, HD = 64, INTER = 96, VOCAB = 50 };

static uint16_t *host_u16(size_t n, unsigned seed)
{
    uint16_t *p = (uint16_t *)malloc(n * 2);
    for (size_t i = 0; i < n; i++) p[i] = (uint16_t)(seed * 131u + i * 7u);
    return p;
}

static float *host_f32(size_t n, float base)
{
    float *p = (float *)malloc(n * 4);
    for (size_t i = 0; i < n; i++) p[i] = base + 0.001f * (float)i;
    return p;
}

static int same(const void *dev, const void *host, size_t bytes)
{
    return dev && host && dev != host && dev_bytes_from(dev) >= bytes && memcmp(dev, host, bytes) == 0;
}

int main(void)
{
    ctx_t *ctx = (ctx_t *)calloc(1, sizeof(ctx_t));
    ctx->config.dec_hidden = HID;
    ctx->config.dec_layers = LAYERS;
    ctx->config.dec_heads = HEADS;
    ctx->config.dec_kv_heads = KV;
    ctx->config.dec_head_dim = HD;
    ctx->config.dec_intermediate = INTER;
    ctx->config.vocab_size = VOCAB;
    ctx->config.dec_rms_norm_eps = 1e-5f;
    ctx->config.dec_rope_theta = 1e4f;
#if GEMMA
    ctx->config.activation = QKN_ACT_GEGLU;
    ctx->config.rope_type = QKN_ROPE_INTERLEAVED;
    ctx->config.dec_rope_local_theta = 1e3f;
    ctx->config.sliding_window = 16;
    ctx->config.attn_logit_softcap = 50.0f;
    ctx->config.embed_normalizer = 8.0f;
#endif
    const size_t qd = (size_t)HEADS * HD, kvd = (size_t)KV * HD;
    for (int l = 0; l < LAYERS; l++) {
        layer_t *ly = &ctx->decoder.layers[l];
        ly->wq_weight_bf16 = host_u16(qd * HID, 10 + l);
        ly->wk_weight_bf16 = host_u16(kvd * HID, 20 + l);
        ly->wv_weight_bf16 = host_u16(kvd * HID, 30 + l);
        ly->wo_weight_bf16 = host_u16(HID * qd, 40 + l);
        ly->gate_up_fused_bf16 = host_u16(2 * (size_t)INTER * HID, 50 + l);
        ly->down_weight_bf16 = host_u16((size_t)HID * INTER, 60 + l);
        ly->input_norm = host_f32(HID, 1.0f + l);
        ly->post_attn_norm = host_f32(HID, 2.0f + l);
#if GEMMA
        ly->q_norm_weight = host_f32(HD, 3.0f + l);
        ly->k_norm_weight = host_f32(HD, 4.0f + l);
        ly->pre_ffn_norm = host_f32(HID, 5.0f + l);
        ly->post_ffn_norm = host_f32(HID, 6.0f + l);
        ly->is_sliding = l % 2 == 0;
#endif
    }
    ctx->decoder.tok_embeddings_bf16 = host_u16((size_t)VOCAB * HID, 1);
    ctx->decoder.norm = host_f32(HID, 0.5f);
#if !GEMMA
    ctx->decoder.lm_head_bf16 = host_u16((size_t)VOCAB * HID, 2);
#endif

    /* prefill 5 positions, then one decode step */
    float embeds[6 * HID];
    for (int t = 0; t < 6; t++)
        for (int i = 0; i < HID; i++) embeds[t * HID + i] = (float)t;
    PREFILL(ctx, embeds, 5);
    CHECK(ctx->kv_cache_len == 5 && g_prefills == 1);
    const int tok = FORWARD(ctx, embeds + 5 * HID);
    CHECK(tok == 5 % VOCAB && ctx->kv_cache_len == 6 && g_steps == 1);
    CHECK(ctx->dec_x && ctx->dec_x[0] == 5.5f && ctx->dec_x[HID - 1] == 5.5f);

    /* the configuration and weights the library received */
    const smol_b200_qkn_model *m = &g_last_model;
    CHECK(m->hidden == HID && m->n_layers == LAYERS && m->n_heads == HEADS && m->n_kv_heads == KV &&
          m->head_dim == HD && m->intermediate == INTER && m->vocab == VOCAB && m->eps == 1e-5f);
    CHECK(model_on_device(m));
    CHECK(same(m->tok_embeddings, ctx->decoder.tok_embeddings_bf16, (size_t)VOCAB * HID * 2));
    CHECK(same(m->final_norm, ctx->decoder.norm, HID * 4));
    for (int l = 0; l < LAYERS; l++) {
        const layer_t *ly = &ctx->decoder.layers[l];
        const smol_b200_qkn_layer *L = &m->layers[l];
        CHECK(same(L->wq, ly->wq_weight_bf16, qd * HID * 2) && same(L->wk, ly->wk_weight_bf16, kvd * HID * 2) &&
              same(L->wv, ly->wv_weight_bf16, kvd * HID * 2) && same(L->wo, ly->wo_weight_bf16, HID * qd * 2));
        CHECK(same(L->gate_up, ly->gate_up_fused_bf16, 2 * (size_t)INTER * HID * 2) &&
              same(L->down, ly->down_weight_bf16, (size_t)HID * INTER * 2));
        CHECK(same(L->input_norm, ly->input_norm, HID * 4) && same(L->post_attn_norm, ly->post_attn_norm, HID * 4));
#if GEMMA
        CHECK(same(L->q_norm, ly->q_norm_weight, HD * 4) && same(L->k_norm, ly->k_norm_weight, HD * 4));
        CHECK(same(L->pre_ffn_norm, ly->pre_ffn_norm, HID * 4) && same(L->post_ffn_norm, ly->post_ffn_norm, HID * 4));
        CHECK(L->is_sliding == (l % 2 == 0));
#else
        CHECK(!L->q_norm && !L->k_norm && !L->pre_ffn_norm && !L->post_ffn_norm && !L->is_sliding);
#endif
    }
#if GEMMA
    CHECK(m->activation == 1 && m->rope_interleaved == 1 && m->embed_normalizer == 8.0f &&
          m->attn_softcap == 50.0f && m->sliding_window == 16);
    CHECK(m->rope_cos_local && m->rope_sin_local && !m->lm_head);
#else
    CHECK(m->activation == 0 && m->rope_interleaved == 0 && m->embed_normalizer == 0.0f &&
          m->attn_softcap == 0.0f && m->sliding_window == 0);
    CHECK(!m->rope_cos_local && !m->rope_sin_local);
    CHECK(same(m->lm_head, ctx->decoder.lm_head_bf16, (size_t)VOCAB * HID * 2));
#endif

    /* chunked prefill continues at kv_cache_len; a cache reset (qkn_kv_cache_reset sets
     * kv_cache_len = 0, qkn_decoder.h:165-167) starts again at position 0 */
    float more[3 * HID];
    for (int t = 0; t < 3; t++)
        for (int i = 0; i < HID; i++) more[t * HID + i] = (float)(6 + t);
    PREFILL(ctx, more, 3);
    CHECK(ctx->kv_cache_len == 9 && g_prefills == 2);
    ctx->kv_cache_len = 0;
    PREFILL(ctx, embeds, 5);
    CHECK(ctx->kv_cache_len == 5 && g_prefills == 3);
    CHECK(FORWARD(ctx, embeds + 5 * HID) == 5 % VOCAB && ctx->kv_cache_len == 6);

    /* a position past the ones the device holds: the export's failure sentinel */
    ctx->kv_cache_len = 9;
    CHECK(FORWARD(ctx, embeds) == SENTINEL && ctx->kv_cache_len == 9);
    ctx->kv_cache_len = 6;
    CHECK(FORWARD(ctx, embeds) == 6 % VOCAB && ctx->kv_cache_len == 7);

    /* release: everything freed, the cache length reset; the next call sets up afresh */
    RELEASE(ctx);
    CHECK(g_live == 0 && ctx->kv_cache_len == 0);
    CHECK(FORWARD(ctx, embeds) == 0 && ctx->kv_cache_len == 1 && g_live > 0);

    /* the same context with other weights (an export that reloaded it) */
    ctx->decoder.tok_embeddings_bf16 = host_u16((size_t)VOCAB * HID, 99);
    ctx->kv_cache_len = 0;
    CHECK(FORWARD(ctx, embeds) == 0);
    CHECK(same(g_last_model.tok_embeddings, ctx->decoder.tok_embeddings_bf16, (size_t)VOCAB * HID * 2));
    RELEASE(ctx);
    CHECK(g_live == 0);

    printf("prefills %d steps %d failures %d\n", g_prefills, g_steps, g_failures);
    return g_failures ? 1 : 0;
}
