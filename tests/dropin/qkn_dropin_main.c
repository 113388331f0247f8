/*
 * qkn_dropin_main.c -- drives the reference's own decoder (common/decoder/qkn_decoder.c
 * of tmzt/smol-genius) through qkn_decoder_prefill / qkn_decoder_forward with a seeded,
 * synthetic Qwen3-shaped model, and prints the greedy tokens.
 *
 * oracle/Makefile links this file four times:
 *   qkn_dropin_ref    -- with every reference kernel object (the baseline);
 *   qkn_dropin_b200   -- with the reference objects minus attention.o, rope.o and
 *                        rmsnorm.o, and with libsmol_b200.so in their place, exactly as
 *                        a maintainer links the exports (those three sources
 *                        filtered out of libsmol.a's list, -lsmol_b200 added);
 *   qkn_dropin_device -- with qkn_decoder_prefill / qkn_decoder_forward taken from
 *                        smol-genius_b200/dropin/qkn_decoder_device.c (the whole decoder
 *                        on the device; qkn_decoder.c compiled with the two renamed;
 *                        SMOL_DROPIN_DEVICE defined: SMOL_DROPIN_RERUN=1 in the
 *                        environment also checks qkn_decoder_device_release);
 *   qkn_dropin_emul   -- with every reference object and smol_causal_attention wrapped
 *                        (cache_precision_wrap.c) to attend over bf16 K / fp16 V values.
 * The tests compare the token streams; stderr also carries the wall-clock time of the
 * prefill call and the mean of the forward calls.  SMOL_DROPIN_WARM=1 in the environment
 * runs the whole generation once unreported first (then qkn_kv_cache_reset), so the
 * reported times leave out the one-time costs of a process's first calls (the device
 * context, module loading and weight upload; the CPU thread pool).  Nothing in the
 * reference changes.
 *
 * Usage: qkn_dropin_xxx [prefill_len=512] [steps=128] [seed=2] [qk_gain=4] [vo_gain=2] [layers=1] [copy=1]
 *
 * The model has to make token identity a meaningful test.  With unit gains attention
 * is nearly uniform and the stream is one token repeated.  With plain random weights
 * (copy=0) and sharp attention the tokens vary, but the top-1 / top-2 logit gaps of a
 * random read-out are small enough (~0.02 over 128 steps) that storing K in bf16 and V
 * in fp16 -- the device cache formats, ~1e-3 relative on the attention output --
 * flips some step, on the CPU too (cache_precision_wrap.c).  A trained decoder's
 * greedy choice is usually far from a tie; copy=1 builds that in:
 *   - every KV group g has a sign vector S_g over the 64 rotary pairs (applied to
 *     coordinates i and i+64, so it commutes with NeoX RoPE); Wq rows of query head h
 *     are S_g(h) * Wq0 and Wk rows of KV head g are S_g * Wk0.  The heads hold
 *     different Q/K data, but every head's scores are the same, so all heads attend
 *     the same tokens (a wrong head-to-KV-head mapping changes the scores);
 *   - Wv is a signed permutation times vo_gain and each query head's Wo block is the
 *     transpose of its KV head's Wv rows, halved per head pair, so Wo.attn reproduces
 *     the attended tokens' normalised embeddings times vo_gain^2.
 * The next token is then the token that the sharp QK-norm attention (mean weight
 * qk_gain) selected, ahead of the runner-up by ~1024 * vo_gain^2 * (w1 - w2) / |h|.
 */
#include <math.h>
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>
#include <time.h>

#include "qkn_decoder.h"
#include "smol_kernels.h"

#define HIDDEN 1024
#define HEADS 16
#define KV_HEADS 8
#define HEAD_DIM 128
#define INTER 1024
#define VOCAB 4096

static uint64_t rng_state;

static uint64_t splitmix64(void)
{
    uint64_t z = (rng_state += 0x9E3779B97F4A7C15ull);
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}

/* Standard normal by Box-Muller from two 53-bit uniforms. */
static double normal(void)
{
    double u1 = ((splitmix64() >> 11) + 1.0) * (1.0 / 9007199254740993.0);
    double u2 = (splitmix64() >> 11) * (1.0 / 9007199254740992.0);
    return sqrt(-2.0 * log(u1)) * cos(6.283185307179586 * u2);
}

static uint16_t to_bf16(float f)
{
    uint32_t u;
    memcpy(&u, &f, 4);
    u += 0x7fffu + ((u >> 16) & 1u);
    return (uint16_t)(u >> 16);
}

static float from_bf16(uint16_t h)
{
    uint32_t u = (uint32_t)h << 16;
    float f;
    memcpy(&f, &u, 4);
    return f;
}

static uint16_t *bf16_matrix(int rows, int cols, double scale)
{
    uint16_t *w = (uint16_t *)malloc(sizeof(uint16_t) * (size_t)rows * cols);
    for (size_t i = 0; i < (size_t)rows * cols; i++) w[i] = to_bf16((float)(normal() * scale));
    return w;
}

static float *f32_vector(int n, double mean, double sd)
{
    float *v = (float *)malloc(sizeof(float) * (size_t)n);
    for (int i = 0; i < n; i++) v[i] = (float)(mean + sd * normal());
    return v;
}

/* Wq / Wk whose heads differ by rotary-pair sign flips: same scores, different data. */
static void shared_scores(qkn_dec_layer_t *l)
{
    const int group = HEADS / KV_HEADS;
    uint16_t *q0 = bf16_matrix(HEAD_DIM, HIDDEN, 1.0 / sqrt(HIDDEN));
    uint16_t *k0 = bf16_matrix(HEAD_DIM, HIDDEN, 1.0 / sqrt(HIDDEN));
    l->wq_weight_bf16 = (uint16_t *)malloc(sizeof(uint16_t) * (size_t)HEADS * HEAD_DIM * HIDDEN);
    l->wk_weight_bf16 = (uint16_t *)malloc(sizeof(uint16_t) * (size_t)KV_HEADS * HEAD_DIM * HIDDEN);
    for (int g = 0; g < KV_HEADS; g++) {
        uint16_t flip[HEAD_DIM / 2];
        for (int i = 0; i < HEAD_DIM / 2; i++) flip[i] = (splitmix64() & 1) ? 0x8000u : 0u;   /* bf16 sign bit */
        for (int d = 0; d < HEAD_DIM; d++) {
            uint16_t sg = flip[d % (HEAD_DIM / 2)];
            for (int c = 0; c < HIDDEN; c++) {
                l->wk_weight_bf16[((size_t)g * HEAD_DIM + d) * HIDDEN + c] = k0[(size_t)d * HIDDEN + c] ^ sg;
                for (int j = 0; j < group; j++)
                    l->wq_weight_bf16[((size_t)(g * group + j) * HEAD_DIM + d) * HIDDEN + c] = q0[(size_t)d * HIDDEN + c] ^ sg;
            }
        }
    }
    free(q0);
    free(k0);
}

/* Wv = gain * (signed permutation), row r of Wv reading coordinate perm[r] with sign
 * sgn[r]; query head h reads KV head g = h / (HEADS / KV_HEADS), and its Wo block maps
 * v row r of that KV head back to coordinate perm[r] with the same sign and gain / 2
 * (two query heads per KV head), so Wo * Wv = gain^2 * I when every head attends the
 * same token.  Both are exact in bf16 for power-of-two gains. */
static void copy_readout(qkn_dec_layer_t *l, double gain)
{
    const int kv_dim = KV_HEADS * HEAD_DIM, group = HEADS / KV_HEADS;
    int perm[KV_HEADS * HEAD_DIM];
    float sgn[KV_HEADS * HEAD_DIM];
    for (int i = 0; i < kv_dim; i++) perm[i] = i;
    for (int i = kv_dim - 1; i > 0; i--) {   /* Fisher-Yates */
        int j = (int)(splitmix64() % (uint64_t)(i + 1)), t = perm[i];
        perm[i] = perm[j];
        perm[j] = t;
    }
    for (int i = 0; i < kv_dim; i++) sgn[i] = (splitmix64() & 1) ? 1.0f : -1.0f;
    l->wv_weight_bf16 = (uint16_t *)calloc((size_t)kv_dim * HIDDEN, sizeof(uint16_t));
    l->wo_weight_bf16 = (uint16_t *)calloc((size_t)HIDDEN * HEADS * HEAD_DIM, sizeof(uint16_t));
    for (int r = 0; r < kv_dim; r++) l->wv_weight_bf16[(size_t)r * HIDDEN + perm[r]] = to_bf16((float)gain * sgn[r]);
    for (int h = 0; h < HEADS; h++) {
        int g = h / group;
        for (int d = 0; d < HEAD_DIM; d++) {
            int r = g * HEAD_DIM + d;
            l->wo_weight_bf16[(size_t)perm[r] * HEADS * HEAD_DIM + h * HEAD_DIM + d] =
                to_bf16((float)(gain / group) * sgn[r]);
        }
    }
}

#ifdef SMOL_DROPIN_DEVICE
/* smol-genius_b200/dropin/qkn_decoder_device.c */
void qkn_decoder_device_release(qkn_ctx_t *ctx);
#endif

/* Prefill all but the last prompt token (as the exports do, e.g. qwen_asr.c:695-703),
 * then decode `steps` tokens from the last one, printing them on one stdout line unless
 * `quiet`.  With `report`, stderr gets the call times and the top-1 / top-2 logit margins.
 * Returns 3 when a forward call returns a failure sentinel instead of a token. */
static int generate(qkn_ctx_t *ctx, const int *prompt, const float *embeds, int prefill, int steps, int report,
                    int quiet)
{
    const qkn_decoder_t *d = &ctx->decoder;
    struct timespec t0, t1;
    clock_gettime(CLOCK_MONOTONIC, &t0);
    qkn_decoder_prefill(ctx, embeds, prefill - 1);
    clock_gettime(CLOCK_MONOTONIC, &t1);
    const double prefill_ms = (t1.tv_sec - t0.tv_sec) * 1e3 + (t1.tv_nsec - t0.tv_nsec) * 1e-6;
    double forward_ms = 0.0;

    /* qkn_decoder_forward leaves the final-normed hidden state in ctx->dec_x
     * (qkn_decoder.c:584, :709-713), so the top-1 / top-2 logit margin of each step is
     * recomputed from it here and the smallest one printed on stderr. */
    float *x = (float *)malloc(sizeof(float) * HIDDEN);
    int tok = prompt[prefill - 1];
    double min_margin = INFINITY;
    double *margins = (double *)malloc(sizeof(double) * (size_t)(steps > 0 ? steps : 1));
    int min_step = -1;
    for (int s = 0; s < steps; s++) {
        for (int k = 0; k < HIDDEN; k++) x[k] = from_bf16(d->tok_embeddings_bf16[(size_t)tok * HIDDEN + k]);
        clock_gettime(CLOCK_MONOTONIC, &t0);
        tok = qkn_decoder_forward(ctx, x);
        clock_gettime(CLOCK_MONOTONIC, &t1);
        forward_ms += (t1.tv_sec - t0.tv_sec) * 1e3 + (t1.tv_nsec - t0.tv_nsec) * 1e-6;
        if (!quiet) printf("%d%c", tok, s + 1 < steps ? ' ' : '\n');
        if (tok < 0 || tok >= VOCAB) {   /* a failure sentinel (qkn_decoder.c:605-611), not a token */
            if (!quiet) printf("\n");
            fprintf(stderr, "forward returned %d at step %d\n", tok, s);
            return 3;
        }
        double top1 = -INFINITY, top2 = -INFINITY;
        for (int v = 0; v < VOCAB; v++) {
            double dot = 0.0;
            for (int k = 0; k < HIDDEN; k++)
                dot += (double)from_bf16(d->tok_embeddings_bf16[(size_t)v * HIDDEN + k]) * ctx->dec_x[k];
            if (dot > top1) { top2 = top1; top1 = dot; } else if (dot > top2) top2 = dot;
        }
        margins[s] = top1 - top2;
        if (top1 - top2 < min_margin) { min_margin = top1 - top2; min_step = s; }
    }
    fflush(stdout);
    if (report) {
        /* wall-clock time of the decoder calls themselves (host buffers in and out) */
        fprintf(stderr, "prefill_ms %.3f forward_ms_per_step %.4f\n", prefill_ms,
                steps > 0 ? forward_ms / steps : 0.0);
        fprintf(stderr, "min top-2 margin %.4f at step %d\nmargins:", min_margin, min_step);
        for (int s = 0; s < steps; s++) fprintf(stderr, " %.5f", margins[s]);
        fprintf(stderr, "\n");
    }
    free(x);
    free(margins);
    return 0;
}

int main(int argc, char **argv)
{
    int prefill = argc > 1 ? atoi(argv[1]) : 512;
    int steps = argc > 2 ? atoi(argv[2]) : 128;
    rng_state = argc > 3 ? strtoull(argv[3], NULL, 10) : 2;
    const double qk_gain = argc > 4 ? atof(argv[4]) : 4.0;   /* mean of the QK-norm weights */
    const double vo_gain = argc > 5 ? atof(argv[5]) : 2.0;   /* gain of Wv and Wo */
    const int layers = argc > 6 ? atoi(argv[6]) : 1;
    const int copy = argc > 7 ? atoi(argv[7]) : 1;
    if (layers < 1 || layers > QKN_MAX_DEC_LAYERS) return 2;

    qkn_ctx_t *ctx = (qkn_ctx_t *)calloc(1, sizeof(qkn_ctx_t));
    qkn_config_t *c = &ctx->config;
    c->dec_hidden = HIDDEN;
    c->dec_layers = layers;
    c->dec_heads = HEADS;
    c->dec_kv_heads = KV_HEADS;
    c->dec_head_dim = HEAD_DIM;
    c->dec_intermediate = INTER;
    c->vocab_size = VOCAB;
    c->dec_rms_norm_eps = 1e-6f;
    c->dec_rope_theta = 1e6f;
    c->activation = QKN_ACT_SWIGLU;
    c->rope_type = QKN_ROPE_NEOX;

    /* Weight gains are chosen so that the attention read-out, not the token's own
     * embedding, decides the next token. */
    qkn_decoder_t *d = &ctx->decoder;
    d->tok_embeddings_bf16 = bf16_matrix(VOCAB, HIDDEN, 1.0);
    d->norm = f32_vector(HIDDEN, 1.0, 0.02);
    for (int li = 0; li < layers; li++) {
        qkn_dec_layer_t *l = &d->layers[li];
        if (copy) {
            shared_scores(l);
        } else {
            l->wq_weight_bf16 = bf16_matrix(HEADS * HEAD_DIM, HIDDEN, 1.0 / sqrt(HIDDEN));
            l->wk_weight_bf16 = bf16_matrix(KV_HEADS * HEAD_DIM, HIDDEN, 1.0 / sqrt(HIDDEN));
        }
        if (copy) {
            copy_readout(l, vo_gain);
        } else {
            l->wv_weight_bf16 = bf16_matrix(KV_HEADS * HEAD_DIM, HIDDEN, vo_gain / sqrt(HIDDEN));
            l->wo_weight_bf16 = bf16_matrix(HIDDEN, HEADS * HEAD_DIM, vo_gain / sqrt(HEADS * HEAD_DIM));
        }
        l->q_norm_weight = f32_vector(HEAD_DIM, qk_gain, 0.02);
        l->k_norm_weight = f32_vector(HEAD_DIM, qk_gain, 0.02);
        l->input_norm = f32_vector(HIDDEN, 1.0, 0.02);
        l->post_attn_norm = f32_vector(HIDDEN, 1.0, 0.02);
        l->gate_weight_bf16 = bf16_matrix(INTER, HIDDEN, 1.0 / sqrt(HIDDEN));
        l->up_weight_bf16 = bf16_matrix(INTER, HIDDEN, 1.0 / sqrt(HIDDEN));
        l->down_weight_bf16 = bf16_matrix(HIDDEN, INTER, 1.0 / sqrt(INTER));
        /* interleaved gate/up rows, as qkn_decoder_load builds them (qkn_decoder.c:140-154) */
        l->gate_up_fused_bf16 = (uint16_t *)malloc(sizeof(uint16_t) * 2 * (size_t)INTER * HIDDEN);
        for (int r = 0; r < INTER; r++) {
            memcpy(l->gate_up_fused_bf16 + (size_t)(2 * r) * HIDDEN, l->gate_weight_bf16 + (size_t)r * HIDDEN,
                   sizeof(uint16_t) * HIDDEN);
            memcpy(l->gate_up_fused_bf16 + (size_t)(2 * r + 1) * HIDDEN, l->up_weight_bf16 + (size_t)r * HIDDEN,
                   sizeof(uint16_t) * HIDDEN);
        }
    }

    int threads = smol_get_num_cpus();
    smol_set_threads(threads > 16 ? 16 : threads);

    /* prompt: random tokens; prefill all but the last (as the exports do, e.g.
     * qwen_asr.c:695-703), then decode from the last prompt token */
    int *prompt = (int *)malloc(sizeof(int) * (size_t)prefill);
    for (int i = 0; i < prefill; i++) prompt[i] = (int)(splitmix64() % VOCAB);
    float *embeds = (float *)malloc(sizeof(float) * (size_t)prefill * HIDDEN);
    for (int i = 0; i < prefill; i++)
        for (int k = 0; k < HIDDEN; k++)
            embeds[(size_t)i * HIDDEN + k] = from_bf16(d->tok_embeddings_bf16[(size_t)prompt[i] * HIDDEN + k]);
    const char *warm = getenv("SMOL_DROPIN_WARM");
    if (warm && atoi(warm)) {
        if (generate(ctx, prompt, embeds, prefill, steps, 0, 1) != 0) return 3;
        qkn_kv_cache_reset(ctx);
    }
    int rc = generate(ctx, prompt, embeds, prefill, steps, 1, 0);
#ifdef SMOL_DROPIN_DEVICE
    /* SMOL_DROPIN_RERUN=1: release the device state, run the same prompt again on the
     * same context (a second line of tokens), then ask for a position past the ones the
     * device holds, which must come back as the failure sentinel. */
    const char *rerun = getenv("SMOL_DROPIN_RERUN");
    if (rc == 0 && rerun && atoi(rerun)) {
        qkn_decoder_device_release(ctx);
        if (ctx->kv_cache_len != 0) return 4;
        rc = generate(ctx, prompt, embeds, prefill, steps, 0, 0);
        if (rc == 0) {
            for (int k = 0; k < HIDDEN; k++) embeds[k] = from_bf16(d->tok_embeddings_bf16[k]);
            ctx->kv_cache_len += 5;
            fprintf(stderr, "past_held_token %d\n", qkn_decoder_forward(ctx, embeds));
        }
    }
#endif
    return rc;
}
