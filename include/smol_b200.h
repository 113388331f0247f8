/*
 * smol_b200.h -- C ABI of libsmol_b200.so, the B200 (sm_100a) attention hot path
 * for tmzt/smol-genius.
 *
 * Part 1 re-declares, with identical prototypes, the entry points of the three
 * reference objects this library replaces (attention.o, rope.o, rmsnorm.o of
 * common/kernels/smol_kernels.h).  A consumer that already includes the
 * reference's smol_kernels.h links libsmol_b200.so ahead of libsmol.a and the
 * linker resolves these names here.  Pointers may be host memory (the call
 * stages through the device and is synchronous on return, as the reference's
 * callers expect) or device memory (the call runs in place, still synchronous).
 *
 * Part 2 is the error interface the reference lacks: the Part-1 functions
 * return void like their originals and record failures here instead of aborting.
 *
 * Part 3 is the device API the fast path uses: a bf16-K / fp16-V KV cache that
 * stays in HBM, a fused QK-norm + RoPE + cache-append kernel, split-KV batched
 * decode, and tcgen05 prefill with a mask kind.  All pointers are device pointers
 * unless a name ends in _host; `stream` is a cudaStream_t (NULL = default stream).
 * Part-3 calls are asynchronous on `stream` unless stated.
 *
 * Reference citations are file:line within tmzt/smol-genius.
 */
#ifndef SMOL_B200_H
#define SMOL_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define SMOL_B200_API __attribute__((visibility("default")))

/* ======================================================================
 * Part 1 -- drop-in replacements (common/kernels/smol_kernels.h:86-161)
 * ====================================================================== */

/* smol_kernels.h:109-113, attention.c:32-77.  MHA; window w covers rows
 * [window_starts[w], window_starts[w+1]) and attends only to itself. */
SMOL_B200_API void smol_bidirectional_attention(float *out, const float *Q, const float *K,
                                                const float *V, int seq, int n_heads,
                                                int head_dim, float scale,
                                                const int *window_starts, int n_windows);

/* smol_kernels.h:115-118, attention.c:153-170.  Row i attends keys
 * [0, min(q_offset+i+1, seq_k)); GQA maps head h to KV head h/(n_heads/n_kv_heads). */
SMOL_B200_API void smol_causal_attention(float *out, const float *Q, const float *K,
                                         const float *V, int seq_q, int seq_k, int n_heads,
                                         int n_kv_heads, int head_dim, float scale,
                                         int q_offset);

/* smol_kernels.h:120-124, attention.c:254-273.  Keys start at pos-window+1. */
SMOL_B200_API void smol_sliding_window_attention(float *out, const float *Q, const float *K,
                                                 const float *V, int seq_q, int seq_k,
                                                 int n_heads, int n_kv_heads, int head_dim,
                                                 float scale, int q_offset, int window_size);

/* smol_kernels.h:127-131, attention.c:350-368.  score = cap*tanh(score/cap). */
SMOL_B200_API void smol_causal_attention_softcap(float *out, const float *Q, const float *K,
                                                 const float *V, int seq_q, int seq_k,
                                                 int n_heads, int n_kv_heads, int head_dim,
                                                 float scale, int q_offset, float cap);

/* smol_kernels.h:133-138, attention.c:443-462. */
SMOL_B200_API void smol_sliding_window_attention_softcap(float *out, const float *Q,
                                                         const float *K, const float *V,
                                                         int seq_q, int seq_k, int n_heads,
                                                         int n_kv_heads, int head_dim,
                                                         float scale, int q_offset,
                                                         int window_size, float cap);

/* smol_kernels.h:144-145, rope.c:12-25.  Table construction, computed on the host
 * with the reference's libm formula so the values are bit-identical. */
SMOL_B200_API void smol_sinusoidal_pe(float *pe, int n_pos, int d_model);

/* smol_kernels.h:147-149, rope.c:27-45.  Host-built table (bit-identical values). */
SMOL_B200_API void smol_compute_rope_neox(float *cos_out, float *sin_out, const int *positions,
                                          int seq, int head_dim, float theta);

/* smol_kernels.h:151-153, rope.c:99-164.  In place on [seq, n_heads*head_dim]. */
SMOL_B200_API void smol_apply_rope_neox(float *x, const float *cos_vals, const float *sin_vals,
                                        int seq, int n_heads, int head_dim);

/* smol_kernels.h:156-158, rope.c:51-66.  Host-built table (bit-identical values). */
SMOL_B200_API void smol_compute_rope_interleaved(float *cos_out, float *sin_out,
                                                 const int *positions, int seq, int head_dim,
                                                 float theta);

/* smol_kernels.h:159-161, rope.c:68-93.  In place. */
SMOL_B200_API void smol_apply_rope_interleaved(float *x, const float *cos_vals,
                                               const float *sin_vals, int seq, int n_heads,
                                               int head_dim);

/* smol_kernels.h:82-84, rmsnorm.c:17-76 (shares rmsnorm.o with the per-head form). */
SMOL_B200_API void smol_rms_norm(float *out, const float *x, const float *weight, int seq_len,
                                 int hidden, float eps);

/* smol_kernels.h:86-88, rmsnorm.c:78-140.  In place on each [head_dim] slice. */
SMOL_B200_API void smol_rms_norm_per_head(float *x, const float *weight, int seq_len,
                                          int n_heads, int head_dim, float eps);

/* ======================================================================
 * Part 2 -- status (no reference counterpart: the reference cannot fail,
 * smol_kernels.h returns void everywhere)
 * ====================================================================== */

enum {
    SMOL_B200_OK = 0,
    SMOL_B200_ERR_ARGS = 1,          /* arguments out of the supported range           */
    SMOL_B200_ERR_CUDA = 2,          /* a CUDA runtime call failed                     */
    SMOL_B200_ERR_NO_DEVICE = 3,     /* no sm_100 device visible                       */
    SMOL_B200_ERR_OOM = 4,           /* device allocation failed                       */
    SMOL_B200_ERR_WATCHDOG = 5,      /* a kernel's bounded wait ran out (see device word) */
    SMOL_B200_ERR_WORKSPACE = 6,     /* caller's workspace smaller than required        */
    SMOL_B200_ERR_RANGE = 7          /* a value too large for fp16 V storage (see device word) */
};

/* Last error recorded by any call on this thread's process (sticky until cleared). */
SMOL_B200_API int smol_cuda_last_error(void);
SMOL_B200_API const char *smol_cuda_error_string(int code);
SMOL_B200_API void smol_cuda_clear_error(void);
/* Device error word of the current device (0 = none), bits set by kernels:
 *   bits 0-4  a bounded wait ran out (TMA tile, free stage, tcgen05 commit, P / O,
 *             drain);
 *   bit 5     a kernel saw arguments its host wrapper should have rejected;
 *   bit 6     a value stored as fp16 (the V cache, fp16 GEMM outputs) had
 *             |x| >= 65520 and became infinity.
 * Synchronises the device.  Cleared by smol_cuda_clear_error.  The drop-in entry
 * points of Part 1 read it after every call (SMOL_B200_ERR_RANGE for bit 6 alone,
 * SMOL_B200_ERR_WATCHDOG otherwise). */
SMOL_B200_API unsigned smol_cuda_device_error(void);
/* Self test of the bounded waits: launches one kernel that waits on an mbarrier
 * nothing arrives on.  After about 2 s the wait gives up, sets bit 0 of the device
 * error word and the kernel returns; the context stays usable.  Asynchronous. */
SMOL_B200_API int smol_b200_watchdog_selftest(void *stream);

/* ======================================================================
 * Part 3 -- device API (new; replaces the host KV cache of
 * common/decoder/qkn_decoder.c:172-220 and the per-layer attention prologue of
 * qkn_decoder.c:488-528 / :642-677)
 * ====================================================================== */

enum {
    SMOL_MASK_CAUSAL = 0,     /* key j visible to row i iff j <= q_offset+i              */
    SMOL_MASK_PREFIX_LM = 1,  /* j < max(prefix_len, q_offset+i+1)                        */
    SMOL_MASK_WINDOWS = 2,    /* bidirectional inside [ws_w, ws_{w+1}) (siglip.c:108)     */
    SMOL_MASK_FULL = 3        /* every key                                               */
};

/* Fused prologue of one attention layer (qkn_decoder.c:488-503 prefill, :642-652
 * decode): for every token t, per-head RMSNorm of q and k (skipped when the weight
 * is NULL), RoPE from table row positions[t] (skipped when rope_cos is NULL), then
 * K is stored as bf16 and V as fp16 into cache row slots[t].  The rotated q goes
 * to q_out_f32 and/or q_out_bf16 (either may be NULL).
 * Inputs: q_in [n_tokens, n_heads*head_dim], k_in/v_in [n_tokens, n_kv_heads*head_dim]
 * fp32; cache rows are n_kv_heads*head_dim wide, cache_rows rows long.  A slot
 * outside [0, cache_rows) is skipped and flagged in the device error word. */
SMOL_B200_API int smol_b200_qknorm_rope_append(
    void *stream, const float *q_in, const float *k_in, const float *v_in, int n_tokens,
    int n_heads, int n_kv_heads, int head_dim, const float *q_norm_w, const float *k_norm_w,
    float eps, const float *rope_cos, const float *rope_sin, int rope_interleaved,
    const int *positions, const int64_t *slots, float *q_out_f32, uint16_t *q_out_bf16,
    uint16_t *k_cache_bf16, uint16_t *v_cache_f16, int64_t cache_rows);

/* Workspace (bytes) that smol_b200_decode_attention needs for these sizes. */
SMOL_B200_API size_t smol_b200_decode_workspace_bytes(int n_seqs, int max_kv_len, int n_heads,
                                                      int n_kv_heads, int head_dim);

/* Batched single-query decode, split-KV (qkn_decoder.c:658-677 per sequence):
 * sequence b attends pool rows [seq_row0[b] + ks, seq_row0[b] + kv_len[b]) where
 * ks = max(0, kv_len[b]-window) when window > 0, else 0.  q is
 * [n_seqs, n_heads*head_dim] fp32 (q_is_bf16=0) or bf16 (1); out is fp32 of the same
 * shape.  k_pool is bf16, v_pool fp16, both [pool_rows, n_kv_heads*head_dim].
 * max_kv_len bounds kv_len[] (it sizes the grid).  softcap<=0 disables the cap.
 * head_dim: 64, 128 or 256.  workspace: smol_b200_decode_workspace_bytes() bytes. */
SMOL_B200_API int smol_b200_decode_attention(
    void *stream, float *out, const void *q, int q_is_bf16, const uint16_t *k_pool,
    const uint16_t *v_pool, int64_t pool_rows, const int64_t *seq_row0, const int *kv_len,
    int n_seqs, int max_kv_len, int n_heads, int n_kv_heads, int head_dim, float scale,
    int window, float softcap, void *workspace, size_t workspace_bytes);

/* smol_b200_decode_attention without a workspace argument.  No counterpart in the
 * reference (it has no device memory at all).
 *
 * For callers that cannot call cudaMalloc: a plugin living inside another
 * framework's memory manager that owns all device memory, an allocation-free
 * real-time serving loop, a host that may not allocate between set-up and
 * teardown.  The per-chunk partial results that smol_b200_decode_attention keeps
 * in the caller's workspace live instead in one fixed 16 MiB device array inside
 * the library; every GPU that loads libsmol_b200.so holds that array until the
 * process exits.  The call itself allocates nothing.
 *
 * Limit: the partial results must fit in 16 MiB - 256 bytes.  The call widens its
 * key chunks until they fit; when even one chunk per sequence needs more
 * (n_seqs * n_heads * (head_dim + 2) * 4 bytes) it returns SMOL_B200_ERR_ARGS and
 * says so in the recorded error.
 * The first call on each device looks up the array's device address (that device
 * must be current); make that first call before any stream capture.
 * Every call shares the one array and leaves its contents behind: two calls whose
 * kernels overlap on the GPU (different streams, or different host threads) race
 * on it, so serialise them.  Arguments and results are those of
 * smol_b200_decode_attention.  A wait that timed out inside its kernels is reported
 * by smol_cuda_device_error(), which in a process that uses no other entry point reads
 * a word of the same array and allocates nothing; smol_cuda_clear_error() resets it. */
SMOL_B200_API int smol_b200_decode_attention_noalloc(
    void *stream, float *out, const void *q, int q_is_bf16, const uint16_t *k_pool,
    const uint16_t *v_pool, int64_t pool_rows, const int64_t *seq_row0, const int *kv_len,
    int n_seqs, int max_kv_len, int n_heads, int n_kv_heads, int head_dim, float scale,
    int window, float softcap);

/* Prefill / encoder attention on tcgen05 tensor cores.  For batch element b, row i
 * of head h attends the keys the mask allows (see SMOL_MASK_*), further limited to
 * [pos-window+1, ...] when window > 0 and capped by softcap when softcap > 0.
 * q, k: bf16; v: fp16; out: fp32.  Strides are in elements; row strides must be
 * multiples of 8 and pointers 16-byte aligned.  head_dim: any multiple of 8 up to 256
 * (the kernel for 64, 128 or 256 columns runs, reading the columns past head_dim as
 * zero: SigLIP-So400m's 72 takes the 128-wide kernel without a padded copy).
 * window_starts (device, n_windows+1 entries) is read for SMOL_MASK_WINDOWS only.
 * GQA: head h reads KV head h / (n_heads/n_kv_heads). */
SMOL_B200_API int smol_b200_prefill_attention(
    void *stream, float *out, int64_t out_row_stride, int64_t out_batch_stride,
    const uint16_t *q, int64_t q_row_stride, int64_t q_batch_stride, const uint16_t *k,
    int64_t k_row_stride, int64_t k_batch_stride, const uint16_t *v, int64_t v_row_stride,
    int64_t v_batch_stride, int batch, int seq_q, int seq_k, int n_heads, int n_kv_heads,
    int head_dim, float scale, int mask_kind, int q_offset, int prefix_len, int window,
    float softcap, const int *window_starts, int n_windows);

/* The same prefill with its output written to several places at once: out_list[i]
 * (device pointers, n_out <= 8, all with the same row / batch strides) each receive
 * the full result.  With CUDA IPC mappings of other GPUs' buffers in the list (the
 * slot of this rank in each peer's gather buffer), the KV-head-split prefill and the
 * all-gather of its output become one kernel: every output row leaves the CTA for this
 * GPU (TMA store) and, as plain stores over NVLink, for every peer, while later tiles
 * compute.
 * out_list is a host array.  Head dims exactly 64 or 128 (the tcgen05 two-tile kernel). */
SMOL_B200_API int smol_b200_prefill_attention_multi(
    void *stream, float *const *out_list, int n_out, int64_t out_row_stride,
    int64_t out_batch_stride, const uint16_t *q, int64_t q_row_stride, int64_t q_batch_stride,
    const uint16_t *k, int64_t k_row_stride, int64_t k_batch_stride, const uint16_t *v,
    int64_t v_row_stride, int64_t v_batch_stride, int batch, int seq_q, int seq_k, int n_heads,
    int n_kv_heads, int head_dim, float scale, int mask_kind, int q_offset, int prefix_len,
    int window, float softcap, const int *window_starts, int n_windows);

/* The two calls above with a bf16 output (rounded to nearest even from the fp32
 * result) instead of fp32: out / out_list[i] hold bf16 elements, and their row and
 * batch strides must be multiples of 8 elements.  For a consumer that takes the
 * attention output as a bf16 GEMM operand (an output projection), and for the
 * KV-head-split prefill, whose all-gather then moves 2 bytes per element instead of
 * 4.  No counterpart in the reference (its attention writes fp32,
 * common/kernels/attention.c:79-170). */
SMOL_B200_API int smol_b200_prefill_attention_bf16(
    void *stream, uint16_t *out, int64_t out_row_stride, int64_t out_batch_stride,
    const uint16_t *q, int64_t q_row_stride, int64_t q_batch_stride, const uint16_t *k,
    int64_t k_row_stride, int64_t k_batch_stride, const uint16_t *v, int64_t v_row_stride,
    int64_t v_batch_stride, int batch, int seq_q, int seq_k, int n_heads, int n_kv_heads,
    int head_dim, float scale, int mask_kind, int q_offset, int prefix_len, int window,
    float softcap, const int *window_starts, int n_windows);
SMOL_B200_API int smol_b200_prefill_attention_multi_bf16(
    void *stream, uint16_t *const *out_list, int n_out, int64_t out_row_stride,
    int64_t out_batch_stride, const uint16_t *q, int64_t q_row_stride, int64_t q_batch_stride,
    const uint16_t *k, int64_t k_row_stride, int64_t k_batch_stride, const uint16_t *v,
    int64_t v_row_stride, int64_t v_batch_stride, int batch, int seq_q, int seq_k, int n_heads,
    int n_kv_heads, int head_dim, float scale, int mask_kind, int q_offset, int prefix_len,
    int window, float softcap, const int *window_starts, int n_windows);

/* CUDA IPC for the above: a 64-byte handle of the device allocation that contains
 * dev_ptr (cudaIpcGetMemHandle) and dev_ptr's byte offset inside it, so the peer adds
 * the offset to the base its open returns (allocators sub-allocate); the mapping in
 * another process (cudaIpcOpenMemHandle, peer access enabled on first use); close
 * unmaps. */
SMOL_B200_API int smol_b200_ipc_get_handle(const void *dev_ptr, void *handle64, size_t *offset);
SMOL_B200_API int smol_b200_ipc_open_handle(const void *handle64, void **dev_ptr);
SMOL_B200_API int smol_b200_ipc_close(void *dev_ptr);

/* One batched decode step of one layer with host buffers, as a host-driven decoder
 * issues it: copies q/k/v of the new token of every sequence (fp32, host) to the
 * device, runs smol_b200_qknorm_rope_append (token of sequence b goes to pool row
 * seq_row0[b]+kv_len[b] at RoPE position kv_len[b]), attends [0, kv_len[b]+1), and
 * copies the fp32 result back to out_host.  kv_len is not advanced (the caller
 * owns it, as qkn_decoder.c:707 owns kv_cache_len).  Synchronous.  `scratch` is a
 * device buffer of smol_b200_decode_step_scratch_bytes() bytes. */
SMOL_B200_API size_t smol_b200_decode_step_scratch_bytes(int n_seqs, int max_kv_len, int n_heads,
                                                         int n_kv_heads, int head_dim);
SMOL_B200_API int smol_b200_decode_step_host(
    void *stream, float *out_host, const float *q_host, const float *k_host,
    const float *v_host, int n_seqs, int n_heads, int n_kv_heads, int head_dim,
    const float *q_norm_w, const float *k_norm_w, float eps, const float *rope_cos,
    const float *rope_sin, int rope_interleaved, uint16_t *k_pool, uint16_t *v_pool,
    int64_t pool_rows, const int64_t *seq_row0, const int *kv_len, int max_kv_len,
    float scale, void *scratch, size_t scratch_bytes);

/* ===========================================================================
 * Part 4 -- device-resident decoder step (qkn_decoder).
 *
 * One greedy token for each of n_seqs sequences, entirely on the device: the whole of
 * qkn_decoder_forward (qkn_decoder.c:570-714) -- embedding lookup, per layer input
 * RMSNorm, Q/K/V projections, QK-norm + RoPE + cache append, attention over the
 * pooled cache, output projection + residual, post-attention RMSNorm, fused gate/up
 * projection with the gated activation, down projection + residual; final RMSNorm and
 * the greedy argmax over the tied embedding matrix (smol_argmax_matvec_bf16,
 * matmul.c:392-417: the lowest index among equal maxima).  Weights use the
 * reference's layouts: bf16 [out][in] matrices, gate/up rows interleaved
 * (qkn_decoder.c:140-154), fp32 norm weights.  Projections compute in fp32 from the
 * bf16 weights (bf16_matvec_fused); the cache holds K bf16 / V fp16 as in Part 3.
 *
 * Two configurations, as qkn_decoder.c selects them: Qwen3 (the Gemma fields zero /
 * NULL) and Gemma as the exports set it (paligemma.c:206-230): embedding scale,
 * GeGLU, a norm on each sublayer's output before its residual add, attention softcap,
 * sliding-window layers with their own RoPE tables; QK-norm is optional in both.
 * SmolVLM's decoder (smolvlm_decoder_forward, exports/smolvlm/decoder.c:391-476) is
 * the Qwen3 configuration without QK-norm and with an untied `lm_head`.
 *
 * Every pointer below is device memory except `layers` (a host array).  The step is
 * asynchronous on `stream` and allocation-free, so a decode loop can be captured
 * once in a CUDA graph and replayed.
 * =========================================================================== */
typedef struct smol_b200_qkn_layer {
    const uint16_t *wq;              /* [n_heads*head_dim][hidden]           */
    const uint16_t *wk, *wv;         /* [n_kv_heads*head_dim][hidden]        */
    const uint16_t *wo;              /* [hidden][n_heads*head_dim]           */
    const uint16_t *gate_up;         /* [2*intermediate][hidden], interleaved */
    const uint16_t *down;            /* [hidden][intermediate]              */
    const float *input_norm, *post_attn_norm;   /* [hidden]   */
    const float *q_norm, *k_norm;               /* [head_dim]; NULL: no QK-norm */
    /* Gemma (NULL / 0 in the Qwen3 configuration): */
    const float *pre_ffn_norm;       /* [hidden]; set: post_attn_norm normalises the
                                        attention output before its residual add and
                                        this normalises x for the MLP (:681-685)   */
    const float *post_ffn_norm;      /* [hidden]; set: normalises the MLP output before
                                        its residual add (:701-702)                */
    int is_sliding;                  /* attends the last sliding_window positions, with
                                        the local RoPE tables (:626-632, :659-667)  */
} smol_b200_qkn_layer;

typedef struct smol_b200_qkn_model {
    int hidden, n_layers, n_heads, n_kv_heads, head_dim, intermediate, vocab;
    float eps;                        /* RMSNorm epsilon (all norms)            */
    int rope_interleaved;             /* 0: NeoX halves, 1: interleaved pairs  */
    const uint16_t *tok_embeddings;   /* [vocab][hidden] bf16, also the lm_head */
    const float *final_norm;          /* [hidden]                               */
    const smol_b200_qkn_layer *layers;   /* host array of n_layers              */
    /* Gemma (0 / NULL in the Qwen3 configuration): */
    int activation;                   /* 0: SwiGLU, 1: GeGLU (GELU-tanh gate)    */
    float embed_normalizer;           /* > 0: embedding rows are scaled by it    */
    float attn_softcap;               /* > 0: scores become cap*tanh(score/cap)  */
    int sliding_window;               /* > 0: window of the is_sliding layers    */
    const float *rope_cos_local;      /* tables of the is_sliding layers, as the */
    const float *rope_sin_local;      /* step's; NULL: the step's tables         */
    /* Untied output head (SmolVLM's decoder, exports/smolvlm/decoder.c:473-475): */
    const uint16_t *lm_head;          /* [vocab][hidden] bf16; NULL: tok_embeddings */
} smol_b200_qkn_model;

/* Device workspace one step needs for n_seqs sequences of at most max_kv_len cached
 * tokens (before the step); 0 when the model is malformed. */
SMOL_B200_API size_t smol_b200_qkn_step_workspace_bytes(const smol_b200_qkn_model *model, int n_seqs,
                                                        int max_kv_len);

/* tokens_in[b]: the token each sequence feeds (may alias tokens_out).
 * layer_row0[l*n_seqs + b]: pool row of position 0 of sequence b in layer l.
 * kv_len[b]: tokens already cached; the new token goes to position / row offset
 * kv_len[b] and attention covers [0, kv_len[b]+1).  advance != 0 increments kv_len
 * on the device at the end of the step (so a captured step replays as a loop).
 * rope_cos / rope_sin: [>= max_kv_len+1][head_dim] tables (row = position); the
 * model's local tables, when given, have the same shape.
 * tokens_out[b]: the greedy next token. */
SMOL_B200_API int smol_b200_qkn_decode_step(
    void *stream, const smol_b200_qkn_model *model, int n_seqs, const int *tokens_in,
    int *tokens_out, uint16_t *k_pool, uint16_t *v_pool, int64_t pool_rows,
    const int64_t *layer_row0, int *kv_len, int max_kv_len, const float *rope_cos,
    const float *rope_sin, int advance, void *workspace, size_t workspace_bytes);

/* Prefill of one sequence (qkn_decoder_prefill, qkn_decoder.c:369-564) on the device:
 * tokens[0..n_tokens) (device) at positions start.. .  Per layer the projections run as
 * tcgen05 GEMMs over bf16 activations (the RMSNorm outputs, the attention output and
 * the gated activation are rounded to bf16 as GEMM operands; the residual stream stays
 * fp32), K / V go to the pool rows layer_row0_host[l] + position (a HOST array of
 * n_layers rows), and the causal prefill attention covers positions [0, start +
 * n_tokens) (sliding layers their window).  No logits, as the reference; a decode step
 * with kv_len = start + n_tokens continues from it.  rope tables: >= start + n_tokens
 * rows.  head_dim 64, 128 or 256. */
/* 0 when the model is malformed (the call would return SMOL_B200_ERR_ARGS). */
SMOL_B200_API size_t smol_b200_qkn_prefill_workspace_bytes(const smol_b200_qkn_model *model, int n_tokens);
SMOL_B200_API int smol_b200_qkn_prefill(void *stream, const smol_b200_qkn_model *model, const int *tokens,
                                        int n_tokens, int start, uint16_t *k_pool, uint16_t *v_pool,
                                        int64_t pool_rows, const int64_t *layer_row0_host, const float *rope_cos,
                                        const float *rope_sin, void *workspace, size_t workspace_bytes);

/* The same two calls with the caller's input embeddings instead of token ids, as
 * qkn_decoder_prefill / qkn_decoder_forward take them (an export passes image or audio
 * features as embeddings): embeds fp32 [n][hidden] on the device, scaled by
 * embed_normalizer when it is set, as the reference does (qkn_decoder.c:415-419,
 * :596-599). */
SMOL_B200_API int smol_b200_qkn_prefill_embeds(void *stream, const smol_b200_qkn_model *model,
                                               const float *embeds, int n_tokens, int start, uint16_t *k_pool,
                                               uint16_t *v_pool, int64_t pool_rows,
                                               const int64_t *layer_row0_host, const float *rope_cos,
                                               const float *rope_sin, void *workspace, size_t workspace_bytes);
SMOL_B200_API int smol_b200_qkn_decode_step_embeds(
    void *stream, const smol_b200_qkn_model *model, int n_seqs, const float *embeds, int *tokens_out,
    uint16_t *k_pool, uint16_t *v_pool, int64_t pool_rows, const int64_t *layer_row0, int *kv_len,
    int max_kv_len, const float *rope_cos, const float *rope_sin, int advance, void *workspace,
    size_t workspace_bytes, float *x_normed_out /* optional [n_seqs][hidden]: the final normalised
                                                   state (the reference's ctx->dec_x) */);

/* Device memory for C callers that do not link the CUDA runtime themselves (the
 * decoder-level drop-in): allocation (NULL on failure, recorded), release, and a
 * synchronous copy in any direction between host and device pointers. */
SMOL_B200_API void *smol_b200_device_alloc(size_t bytes);
SMOL_B200_API void smol_b200_device_free(void *ptr);
SMOL_B200_API int smol_b200_copy(void *dst, const void *src, size_t bytes);

/* The building blocks of the step, for callers that orchestrate their own decoder:
 *   y[b][n] (+)= sum_k x[b][k] * W[n][k]    mode 0: store, 1: add into y (residual),
 *   2: SiLU-gated pairs, y[b][r] = silu(s[2r]) * s[2r+1] over W's 2*n_out rows
 *   (smol_swiglu_multiply, activation.c:55-86), 3: GELU-tanh-gated pairs
 *   (smol_geglu_multiply, activation.c:104-126); n_out = rows of y.
 * W bf16 [rows][k_dim] with k_dim a multiple of 8 and 16-byte aligned rows.
 * x fp32 with row stride ldx (multiple of 4), y fp32 with row stride ldy. */
SMOL_B200_API int smol_b200_gemv_bf16(void *stream, float *y, int64_t ldy, const float *x, int64_t ldx,
                                      const uint16_t *w, int n_out, int k_dim, int n_seqs, int mode);
/* tokens_out[b] = argmax_v sum_k x[b][k] * E[v][k] (lowest v among equal maxima); the
 * workspace holds the n_seqs x vocab fp32 logits. */
SMOL_B200_API int smol_b200_argmax_bf16(void *stream, int *tokens_out, const float *x, int64_t ldx,
                                        const uint16_t *emb, int vocab, int k_dim, int n_seqs,
                                        void *workspace, size_t workspace_bytes);
SMOL_B200_API size_t smol_b200_argmax_workspace_bytes(int n_seqs, int vocab);

/* ===========================================================================
 * Part 5 -- SigLIP vision encoder on the device (siglip_forward, siglip.c:71-156).
 *
 * Patch embedding (the kernel = stride = patch convolution of siglip.c:24-65 as a
 * GEMM over unfolded patches, conv2d.c:13-95), position embeddings, the encoder
 * layers (LayerNorm -> Q/K/V with bias -> bidirectional attention over all patches
 * -> output projection + residual; LayerNorm -> fc1 + bias -> GELU (tanh form) -> fc2
 * + bias + residual) and the post-LayerNorm, for a batch of images.  The linear layers
 * run as tcgen05 GEMMs with bf16 operands and fp32 accumulation; the residual stream
 * stays fp32; LayerNorm, attention and GELU outputs are rounded to bf16 (V to fp16)
 * where they become GEMM / attention operands.  head_dim must be 64, 128 or 256.
 * Every pointer is device memory except `layers` (a host array).
 * =========================================================================== */
#define SMOL_B200_GEMM_OUT_F32 0      /* C = result (fp32)                       */
#define SMOL_B200_GEMM_OUT_BF16 1     /* C = bf16(result)                        */
#define SMOL_B200_GEMM_OUT_F16 2      /* C = fp16(result)                        */
#define SMOL_B200_GEMM_OUT_F32_ADD 3  /* C += result (fp32, the residual stream) */

typedef struct smol_b200_siglip_layer {
    const float *ln1_w, *ln1_b;                   /* [hidden]                     */
    const uint16_t *wq, *wk, *wv, *wo;            /* [hidden][hidden] bf16        */
    const float *bq, *bk, *bv, *bo;               /* [hidden]                     */
    const float *ln2_w, *ln2_b;                   /* [hidden]                     */
    const uint16_t *fc1;                          /* [ffn][hidden] bf16           */
    const float *b1;                              /* [ffn]                        */
    const uint16_t *fc2;                          /* [hidden][ffn] bf16           */
    const float *b2;                              /* [hidden]                     */
} smol_b200_siglip_layer;

typedef struct smol_b200_siglip_model {
    int hidden, heads, ffn, n_layers, patch, image_size, num_positions;
    float eps;                                    /* LayerNorm epsilon            */
    const uint16_t *patch_w;                      /* [hidden][patch_ld] bf16, columns
                                                     (channel, ky, kx) of 3*patch^2 */
    int patch_ld;                                 /* >= 3*patch^2, multiple of 8  */
    const float *patch_b;                         /* [hidden]                     */
    const float *pos;                             /* [num_positions][hidden]      */
    const float *post_w, *post_b;                 /* [hidden]                     */
    const smol_b200_siglip_layer *layers;         /* host array of n_layers       */
} smol_b200_siglip_model;

/* Device workspace of smol_b200_siglip_forward for n_images images (0: a shape the
 * device path does not take -- the call would return SMOL_B200_ERR_ARGS). */
SMOL_B200_API size_t smol_b200_siglip_workspace_bytes(const smol_b200_siglip_model *model, int n_images);

/* images: [n_images][3][image_size][image_size] fp32; out: [n_images][n_patches][hidden]
 * fp32 with n_patches = (image_size/patch)^2 <= num_positions. */
SMOL_B200_API int smol_b200_siglip_forward(void *stream, float *out, const float *images, int n_images,
                                           const smol_b200_siglip_model *model, void *workspace,
                                           size_t workspace_bytes);

/* The pre-LayerNorm encoder layers on their own (siglip.c:112-147; the Qwen3-ASR audio
 * encoder's layers, exports/qwen_asr/encoder.c:449-484, have the same form): x
 * [batch][seq][hidden] fp32 in place; window_starts (device, n_windows + 1 entries, as
 * smol_bidirectional_attention takes them) limits attention to windows within every
 * batch element, NULL lets every token attend to its whole batch element.  eps: the
 * LayerNorm epsilon (SigLIP 1e-6, the audio encoder 1e-5). */
SMOL_B200_API size_t smol_b200_encoder_workspace_bytes(int n_tokens, int hidden, int ffn);
SMOL_B200_API int smol_b200_encoder_layers(void *stream, float *x, int batch, int seq,
                                           const smol_b200_siglip_layer *layers, int n_layers, int hidden,
                                           int heads, int ffn, float eps, const int *window_starts, int n_windows,
                                           void *workspace, size_t workspace_bytes);

/* The building blocks:
 *   C[m][n] (+)= sum_k A[m][k] * W[n][k] + bias[n] + add[m % add_rows][n], stored as
 *   out_kind says.  A bf16 [M][lda], W bf16 [N][ldw] (K-major, 16-byte aligned, lda / ldw
 *   multiples of 8); bias, add optional.  act: SMOL_B200_ACT_NONE, _GELU (GELU-tanh of
 *   every element), or _SWIGLU / _GEGLU: W's rows are interleaved gate/up pairs and
 *   C[m][j] = act(c[2j]) * c[2j+1] for j < n/2 (bf16 or fp32 out, no `add`). */
#define SMOL_B200_ACT_NONE 0
#define SMOL_B200_ACT_GELU 1
#define SMOL_B200_ACT_SWIGLU 2
#define SMOL_B200_ACT_GEGLU 3
SMOL_B200_API int smol_b200_gemm_bf16(void *stream, void *out, int64_t ldo, int out_kind, const uint16_t *a,
                                      int64_t lda, const uint16_t *w, int64_t ldw, const float *bias,
                                      const float *add, int64_t ld_add, int add_rows, int m, int n, int k,
                                      int act);
/* out[r] = (x[r] - mean) / sqrtf(var + eps) * w + b per row (smol_layer_norm,
 * layernorm.c:17-124); out bf16 when out_bf16 != 0, else fp32 (may alias x). */
SMOL_B200_API int smol_b200_layer_norm(void *stream, void *out, int out_bf16, const float *x, const float *w,
                                       const float *b, int rows, int hidden, float eps);

#ifdef __cplusplus
}
#endif

#endif /* SMOL_B200_H */
