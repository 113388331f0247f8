/*
 * device_decoder.h -- the device side shared by the decoder-level drop-ins
 * (qkn_decoder_device.c for common/decoder/qkn_decoder.c, smolvlm_decoder_device.c for
 * exports/smolvlm/decoder.c): one decoder's weights uploaded once, a KV cache pool grown
 * on the device, RoPE tables, workspaces, and prefill / forward calls over host
 * embeddings through libsmol_b200's Part 4 (smol_b200_qkn_prefill_embeds,
 * smol_b200_qkn_decode_step_embeds).  Plain C over the C ABI of include/smol_b200.h.
 */
#ifndef SMOL_B200_DEVICE_DECODER_H
#define SMOL_B200_DEVICE_DECODER_H

#include <stdint.h>

#include "smol_b200.h"

#define DD_MAX_LAYERS 64

/* A decoder's shape and settings, in the reference's terms. */
typedef struct {
    int hidden, layers, heads, kv_heads, head_dim, intermediate, vocab;
    float eps, theta, local_theta;        /* local_theta: sliding layers' own (0: none) */
    float embed_normalizer, attn_softcap; /* 0: off */
    int sliding_window;                   /* 0: off */
    int geglu, interleaved;               /* activation and RoPE layout */
} dd_config;

/* One layer's host weights (bf16 matrices [out][in], gate/up rows interleaved; fp32
 * norms; NULL for the optional ones). */
typedef struct {
    const uint16_t *wq, *wk, *wv, *wo, *gate_up, *down;
    const float *input_norm, *post_attn_norm, *q_norm, *k_norm, *pre_ffn_norm, *post_ffn_norm;
    int is_sliding;
} dd_layer;

typedef struct {
    int ready;
    dd_config cfg;
    smol_b200_qkn_layer layers[DD_MAX_LAYERS];
    smol_b200_qkn_model model;
    int64_t cap;                        /* positions per layer in the pools */
    int held;                           /* positions [0, held) hold written K / V rows */
    uint16_t *k_pool, *v_pool;
    int64_t row0_host[DD_MAX_LAYERS];
    int64_t *row0_dev;
    int rope_cap;
    float *cos, *sin, *cos_local, *sin_local;
    /* A decode step's input and output, each one block so that a step makes one copy
     * each way: [hidden] embedding + the position (an int in the last slot), and
     * [hidden] final normalised state + the greedy token (likewise); the host staging
     * buffers have the same layout. */
    float *step_in_dev, *step_out_dev;
    float *step_in_host, *step_out_host;
    float *x_dev;   /* prefill input rows */
    int x_cap;
    void *step_ws, *prefill_ws;
    size_t step_ws_bytes, prefill_ws_bytes;
    int prefill_cap;
} dd_state;

/* Uploads the weights (lm_head NULL: tied to tok_embeddings).  0 on success. */
int dd_setup(dd_state *st, const dd_config *cfg, const dd_layer *layers, const uint16_t *tok_embeddings,
             const float *final_norm, const uint16_t *lm_head);

/* Frees every device buffer of a state (set up or partly set up). */
void dd_release(dd_state *st);

/* The side table of device states the drop-ins keep for the reference's contexts (up
 * to DD_MAX_CONTEXTS), keyed by the context's address and a fingerprint of its weights
 * (their host addresses, the shape and a few values), so that a context freed and
 * allocated again at the same address with another model is set up afresh. */
#define DD_MAX_CONTEXTS 8

/* The fingerprint of a decoder's host weights. */
uint64_t dd_fingerprint(int hidden, int layers, int vocab, const uint16_t *tok_embeddings, const uint16_t *wq0);

/* The state of ctx when it was set up from weights with this fingerprint (*ready = 1);
 * otherwise a free slot for dd_setup (*ready = 0; a state ctx held for other weights is
 * released first), or NULL when every slot is taken. */
dd_state *dd_slot_find(const void *ctx, uint64_t fingerprint, int *ready);

/* Records that st (from dd_slot_find) now holds ctx's weights. */
void dd_slot_claim(dd_state *st, const void *ctx, uint64_t fingerprint);

/* Releases the state held for ctx, if any; returns 1 when there was one. */
int dd_slot_release(const void *ctx);

/* Prefill n host embeddings at positions start.. (the positions before `start` are
 * kept when the pool grows).  0 on success; -1 also when start is past the positions
 * the device holds (their rows were never written). */
int dd_prefill(dd_state *st, const float *embeds, int n, int start);

/* One decode step at position pos (= cached positions, at most the positions held):
 * returns the greedy token and writes the final normalised state to x_normed (host,
 * may be NULL), or -1. */
int dd_forward(dd_state *st, const float *embed, int pos, float *x_normed);

#endif /* SMOL_B200_DEVICE_DECODER_H */
