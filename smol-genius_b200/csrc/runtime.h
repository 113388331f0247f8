// runtime.h -- host-side internals shared by the translation units of libsmol_b200.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

#include <mutex>

#include "smol_b200.h"

namespace smolb200 {

// ---- error state (process-wide, sticky until smol_cuda_clear_error) ----
void set_error(int code, const char *what);
bool cuda_check(cudaError_t e, const char *what);   // records SMOL_B200_ERR_CUDA on failure

// ---- per-device context ----
// Device error word of the current device (zeroed at creation).
unsigned *device_error_word();
// The same word if this device's context already exists, else NULL; never allocates.
unsigned *device_error_word_if_created();
// decode_attn.cu: the allocation-free entry point's array on the current device
bool noalloc_in_use();
unsigned noalloc_watchdog_bits(bool clear);
// Stream used by the drop-in (Part 1) entry points of the current device.
cudaStream_t legacy_stream();
// Grow-only device scratch of the current device for the drop-in entry points.
// Slot i is an independent buffer.  Returns NULL (error recorded) on failure.
void *legacy_scratch(int slot, size_t bytes);
// True when `p` is device or managed memory the current device can address.
bool is_device_pointer(const void *p);
// Base address of the device allocation that contains ptr (cuMemGetAddressRange).
bool allocation_base(const void *ptr, uintptr_t *base);
// Number of the current device, or -1 (error recorded) when none is usable.
int current_device();

// ---- TMA descriptors ----
// 2-D tensor [rows, inner] of 2-byte elements, row stride `row_stride` elements,
// box = box_rows x box_inner, 128-byte swizzle (box_inner*2 must be 128).
bool make_tmap_2d(CUtensorMap *map, const void *base, CUtensorMapDataType dtype, int64_t inner,
                  int64_t rows, int box_inner, int box_rows, int64_t row_stride = -1);
// 3-D tensor [outer, rows, inner] with strides in elements of `elem_bytes` bytes.
bool make_tmap_3d(CUtensorMap *map, const void *base, CUtensorMapDataType dtype, int64_t inner,
                  int64_t rows, int64_t outer, int64_t row_stride, int64_t outer_stride, int box_inner,
                  int box_rows, int elem_bytes = 2);
// 4-D tiled map over (inner, d1, d2, d3) with element strides s1, s2, s3 of d1..d3 and
// box (b0, b1, b2, 1), 128-byte swizzle.
bool make_tmap_4d(CUtensorMap *map, const void *base, CUtensorMapDataType dtype, int elem_bytes, int64_t inner,
                  int64_t d1, int64_t d2, int64_t d3, int64_t s1, int64_t s2, int64_t s3, int b0, int b1, int b2);

// ---- kernels (implemented in the .cu files) ----
size_t decode_workspace_bytes(int n_seqs, int max_kv_len, int n_heads, int n_kv_heads, int head_dim);
int decode_attention(cudaStream_t st, float *out, const void *q, int q_is_bf16, const uint16_t *k_pool,
                     const uint16_t *v_pool, int64_t pool_rows, const int64_t *seq_row0, const int *kv_len,
                     int n_seqs, int max_kv_len, int n_heads, int n_kv_heads, int head_dim, float scale,
                     int window, float softcap, void *workspace, size_t workspace_bytes);

// out (and each of more_outs) holds fp32 elements, or bf16 when out_bf16.
int prefill_attention(cudaStream_t st, void *out, int64_t out_row_stride, int64_t out_batch_stride,
                      const uint16_t *q, int64_t q_row_stride, int64_t q_batch_stride, const uint16_t *k,
                      int64_t k_row_stride, int64_t k_batch_stride, const uint16_t *v, int64_t v_row_stride,
                      int64_t v_batch_stride, int batch, int seq_q, int seq_k, int n_heads, int n_kv_heads,
                      int head_dim, float scale, int mask_kind, int q_offset, int prefix_len, int window,
                      float softcap, const int *window_starts, int n_windows, void *const *more_outs = nullptr,
                      int n_more = 0, int out_bf16 = 0);

int qknorm_rope_append(cudaStream_t st, const float *q_in, const float *k_in, const float *v_in, int n_tokens,
                       int n_heads, int n_kv_heads, int head_dim, const float *q_norm_w, const float *k_norm_w,
                       float eps, const float *rope_cos, const float *rope_sin, int rope_interleaved,
                       const int *positions, const int64_t *slots, float *q_out_f32, uint16_t *q_out_bf16,
                       uint16_t *k_cache_bf16, uint16_t *v_cache_f16, int64_t cache_rows);

// In-place fp32 kernels behind the drop-in RoPE / RMSNorm entry points.
int launch_rms_norm_per_head(cudaStream_t st, float *x, const float *w, int seq_len, int n_heads, int head_dim,
                             float eps);
int launch_rms_norm(cudaStream_t st, float *out, const float *x, const float *w, int seq_len, int hidden,
                    float eps);
int launch_rope(cudaStream_t st, float *x, const float *cos_vals, const float *sin_vals, int seq, int n_heads,
                int head_dim, int interleaved);

// Staging kernels of the drop-in attention path: fp32 rows -> padded bf16 / fp16 rows.
int launch_pack_rows(cudaStream_t st, uint16_t *dst, int64_t dst_stride, int dst_width, const float *src,
                     int64_t src_stride, int src_heads, int head_dim, int padded_hd, int64_t rows, int to_f16);
int launch_unpack_rows(cudaStream_t st, float *dst, int64_t dst_stride, const float *src, int64_t src_stride,
                       int heads, int head_dim, int padded_hd, int64_t rows);

// Per-token (position, slot) of a decode step: positions[b] = kv_len[b],
// slots[b] = seq_row0[b] + kv_len[b], kv_len_next[b] = kv_len[b] + 1.
// Bounded-wait self test: one kernel whose wait can never succeed (see rope_norm.cu).
int launch_watchdog_selftest(cudaStream_t st);

// Three streams and their events for calls that pipeline host copies with compute
// (smol_b200_decode_step_host): inputs in on h2d, kernels on compute, results out on
// d2h.  One per device, created on first use; `mu` serialises its users.
struct StepPipe {
    static constexpr int kMaxChunks = 8;
    cudaStream_t h2d = nullptr, compute = nullptr, d2h = nullptr;
    cudaEvent_t start = nullptr, in[kMaxChunks] = {}, done[kMaxChunks] = {};
    std::mutex *mu = nullptr;
};
StepPipe *step_pipe();

// Launches with programmatic dependent launch when the calling thread is inside a
// PdlScope (the device decoder step); otherwise a plain launch.  The kernels that
// go through it call griddep_wait() before touching data of earlier kernels.
extern thread_local bool g_pdl_scope;
extern const bool g_pdl_enabled;
extern const bool g_api_pdl;   // the attention entry points' own launches (SMOL_API_PDL=0: off)
struct PdlScope {
    bool prev;
    // on: launches inside the scope use programmatic dependent launch (an enclosing scope's
    // setting is kept when off)
    explicit PdlScope(bool on = true) : prev(g_pdl_scope) { g_pdl_scope = prev || (on && g_pdl_enabled); }
    ~PdlScope() { g_pdl_scope = prev; }
};
template <typename... KArgs, typename... Args>
cudaError_t launch_kernel(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st,
                          Args &&...args)
{
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    if (g_pdl_scope) {
        attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        attr[0].val.programmaticStreamSerializationAllowed = 1;
        cfg.attrs = attr;
        cfg.numAttrs = 1;
    }
    return cudaLaunchKernelEx(&cfg, kernel, static_cast<KArgs>(args)...);
}

// decoder.cu: the device-resident decode step (Part 4 of smol_b200.h)
int gemv_bf16(cudaStream_t st, float *y, int64_t ldy, const float *x, int64_t ldx, const uint16_t *w, int n_out,
              int k_dim, int n_seqs, int mode);
int argmax_bf16(cudaStream_t st, int *tokens_out, const float *x, int64_t ldx, const uint16_t *emb, int vocab,
                int k_dim, int n_seqs, void *ws, size_t ws_bytes);
size_t argmax_workspace_bytes(int n_seqs, int vocab);
size_t qkn_step_workspace_bytes(const smol_b200_qkn_model *m, int n_seqs, int max_kv_len);
int qkn_decode_step(cudaStream_t st, const smol_b200_qkn_model *m, int n_seqs, const int *tokens_in,
                    const float *x_in, int *tokens_out, uint16_t *k_pool, uint16_t *v_pool, int64_t pool_rows,
                    const int64_t *layer_row0, int *kv_len, int max_kv_len, const float *rope_cos,
                    const float *rope_sin, int advance, void *workspace, size_t workspace_bytes,
                    float *x_normed_out = nullptr);

size_t qkn_prefill_workspace_bytes(const smol_b200_qkn_model *m, int n_tokens);
int qkn_prefill(cudaStream_t st, const smol_b200_qkn_model *m, const int *tokens, const float *x_in, int n_tokens,
                int start,
                uint16_t *k_pool, uint16_t *v_pool, int64_t pool_rows, const int64_t *layer_row0,
                const float *rope_cos, const float *rope_sin, void *workspace, size_t workspace_bytes);

int launch_decode_step_index(cudaStream_t st, int *positions, int64_t *slots, int *kv_len_next,
                             const int64_t *seq_row0, const int *kv_len, int n_seqs);

// gemm.cu / siglip.cu: the SigLIP encoder (Part 5 of smol_b200.h)
int gemm_bf16(cudaStream_t st, void *out, int64_t ldo, int out_kind, const uint16_t *a, int64_t lda,
              const uint16_t *w, int64_t ldw, const float *bias, const float *add, int64_t ld_add, int add_rows,
              int M, int N, int K, int gelu, int gate = 0);
int layer_norm(cudaStream_t st, void *out, int out_bf16, const float *x, const float *w, const float *b, int rows,
               int hidden, float eps);
size_t encoder_workspace_bytes(int n_tokens, int hidden, int ffn);
int encoder_layers(cudaStream_t st, float *x, int batch, int seq, const smol_b200_siglip_layer *layers, int n_layers,
                   int hidden, int heads, int ffn, float eps, const int *window_starts, int n_windows,
                   void *workspace, size_t workspace_bytes);
size_t siglip_workspace_bytes(const smol_b200_siglip_model *m, int n_images);
int siglip_forward(cudaStream_t st, float *out, const float *images, int n_images, const smol_b200_siglip_model *m,
                   void *workspace, size_t workspace_bytes);

}  // namespace smolb200
