// runtime.cu -- per-device context, error state and TMA descriptor encoding.
//
// The reference's kernels run on a global, non-reentrant thread pool
// (common/kernels/threading.c:26-47).  The equivalent here is one context per
// CUDA device holding the stream and the grow-only scratch the drop-in entry
// points stage through, plus the device error word that bounded waits write.
#include <atomic>
#include <mutex>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include "runtime.h"

namespace smolb200 {

thread_local bool g_pdl_scope = false;
// SMOL_PDL=0 in the environment turns programmatic dependent launch off (measurement knob).
const bool g_pdl_enabled = [] {
    const char *e = getenv("SMOL_PDL");
    return !(e && e[0] == '0');
}();
const bool g_api_pdl = [] {
    const char *e = getenv("SMOL_API_PDL");
    return !(e && e[0] == '0');
}();

namespace {

constexpr int kMaxDevices = 16;
constexpr int kScratchSlots = 8;

struct DeviceCtx {
    // Set (release) after err_word and stream; read (acquire) without the lock, so a
    // reader that sees it set also sees both.
    std::atomic<bool> init{false};
    unsigned *err_word = nullptr;
    cudaStream_t stream = nullptr;
    void *scratch[kScratchSlots] = {};
    size_t scratch_bytes[kScratchSlots] = {};
    bool pipe_init = false;
    StepPipe pipe;
    std::mutex pipe_mu;
};

std::mutex g_mutex;
DeviceCtx g_ctx[kMaxDevices];
int g_last_error = SMOL_B200_OK;
bool g_reported = false;

// Signature of cuTensorMapEncodeTiled (cuda.h), resolved through the runtime so the
// library does not link libcuda directly.
typedef CUresult (*EncodeTiledFn)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *, const cuuint64_t *,
                                  const cuuint64_t *, const cuuint32_t *, const cuuint32_t *, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);
EncodeTiledFn g_encode = nullptr;

DeviceCtx *ctx_for_current()
{
    const int dev = current_device();
    if (dev < 0) return nullptr;
    DeviceCtx &c = g_ctx[dev];
    if (!c.init.load(std::memory_order_acquire)) {
        std::lock_guard<std::mutex> lock(g_mutex);
        if (!c.init.load(std::memory_order_relaxed)) {
            if (!cuda_check(cudaMalloc(&c.err_word, sizeof(unsigned)), "cudaMalloc(error word)")) return nullptr;
            if (!cuda_check(cudaMemset(c.err_word, 0, sizeof(unsigned)), "cudaMemset(error word)")) return nullptr;
            if (!cuda_check(cudaStreamCreateWithFlags(&c.stream, cudaStreamNonBlocking), "cudaStreamCreate"))
                return nullptr;
            c.init.store(true, std::memory_order_release);
        }
    }
    return &c;
}

// cuMemGetAddressRange (cuda.h), also resolved through the runtime.
typedef CUresult (*AddressRangeFn)(CUdeviceptr *, size_t *, CUdeviceptr);
AddressRangeFn g_address_range = nullptr;

bool encode_fn()
{
    if (g_encode) return true;
    void *fn = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess || !fn) {
        set_error(SMOL_B200_ERR_CUDA, "cuTensorMapEncodeTiled entry point not found");
        return false;
    }
    g_encode = reinterpret_cast<EncodeTiledFn>(fn);
    return true;
}

}  // namespace

StepPipe *step_pipe()
{
    DeviceCtx *c = ctx_for_current();
    if (!c) return nullptr;
    std::lock_guard<std::mutex> lock(g_mutex);
    if (!c->pipe_init) {
        StepPipe &P = c->pipe;
        cudaStream_t *streams[3] = {&P.h2d, &P.compute, &P.d2h};
        for (cudaStream_t *sp : streams)
            if (!cuda_check(cudaStreamCreateWithFlags(sp, cudaStreamNonBlocking), "cudaStreamCreate(pipe)"))
                return nullptr;
        if (!cuda_check(cudaEventCreateWithFlags(&P.start, cudaEventDisableTiming), "cudaEventCreate(pipe)"))
            return nullptr;
        for (int i = 0; i < StepPipe::kMaxChunks; ++i)
            if (!cuda_check(cudaEventCreateWithFlags(&P.in[i], cudaEventDisableTiming), "cudaEventCreate(pipe)") ||
                !cuda_check(cudaEventCreateWithFlags(&P.done[i], cudaEventDisableTiming), "cudaEventCreate(pipe)"))
                return nullptr;
        P.mu = &c->pipe_mu;
        c->pipe_init = true;
    }
    return &c->pipe;
}

bool allocation_base(const void *ptr, uintptr_t *base)
{
    if (!g_address_range) {
        void *fn = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuMemGetAddressRange", &fn, cudaEnableDefault, &q) != cudaSuccess ||
            q != cudaDriverEntryPointSuccess || !fn) {
            cudaGetLastError();
            set_error(SMOL_B200_ERR_CUDA, "cuMemGetAddressRange entry point not found");
            return false;
        }
        g_address_range = reinterpret_cast<AddressRangeFn>(fn);
    }
    CUdeviceptr b = 0;
    size_t sz = 0;
    if (g_address_range(&b, &sz, reinterpret_cast<CUdeviceptr>(ptr)) != CUDA_SUCCESS) {
        set_error(SMOL_B200_ERR_CUDA, "cuMemGetAddressRange failed");
        return false;
    }
    *base = static_cast<uintptr_t>(b);
    return true;
}

void set_error(int code, const char *what)
{
    g_last_error = code;
    if (!g_reported) {
        g_reported = true;
        fprintf(stderr, "smol_b200: %s (%s)\n", what, smol_cuda_error_string(code));
    }
}

bool cuda_check(cudaError_t e, const char *what)
{
    if (e == cudaSuccess) return true;
    char buf[256];
    snprintf(buf, sizeof(buf), "%s: %s", what, cudaGetErrorString(e));
    set_error(e == cudaErrorMemoryAllocation ? SMOL_B200_ERR_OOM : SMOL_B200_ERR_CUDA, buf);
    return false;
}

int current_device()
{
    int dev = -1;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) {
        cudaGetLastError();
        set_error(SMOL_B200_ERR_NO_DEVICE, "no usable CUDA device");
        return -1;
    }
    int n = 0;
    if (cudaGetDeviceCount(&n) != cudaSuccess || n <= 0) {
        cudaGetLastError();
        set_error(SMOL_B200_ERR_NO_DEVICE, "no usable CUDA device");
        return -1;
    }
    return dev;
}

unsigned *device_error_word()
{
    DeviceCtx *c = ctx_for_current();
    return c ? c->err_word : nullptr;
}

unsigned *device_error_word_if_created()
{
    int dev = -1;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) {
        cudaGetLastError();
        return nullptr;
    }
    return g_ctx[dev].init.load(std::memory_order_acquire) ? g_ctx[dev].err_word : nullptr;
}

cudaStream_t legacy_stream()
{
    DeviceCtx *c = ctx_for_current();
    return c ? c->stream : nullptr;
}

void *legacy_scratch(int slot, size_t bytes)
{
    DeviceCtx *c = ctx_for_current();
    if (!c || slot < 0 || slot >= kScratchSlots) return nullptr;
    if (bytes == 0) bytes = 16;
    if (c->scratch_bytes[slot] >= bytes) return c->scratch[slot];
    if (c->scratch[slot]) {
        cudaStreamSynchronize(c->stream);
        cudaFree(c->scratch[slot]);
        c->scratch[slot] = nullptr;
        c->scratch_bytes[slot] = 0;
    }
    size_t grown = bytes + bytes / 4;
    grown = (grown + 255) & ~size_t(255);
    if (!cuda_check(cudaMalloc(&c->scratch[slot], grown), "cudaMalloc(staging)")) return nullptr;
    c->scratch_bytes[slot] = grown;
    return c->scratch[slot];
}

bool is_device_pointer(const void *p)
{
    if (!p) return false;
    cudaPointerAttributes a;
    if (cudaPointerGetAttributes(&a, p) != cudaSuccess) {
        cudaGetLastError();
        return false;
    }
    return a.type == cudaMemoryTypeDevice || a.type == cudaMemoryTypeManaged;
}

bool make_tmap_2d(CUtensorMap *map, const void *base, CUtensorMapDataType dtype, int64_t inner, int64_t rows,
                  int box_inner, int box_rows, int64_t row_stride)
{
    if (!encode_fn()) return false;
    if (row_stride < 0) row_stride = inner;
    cuuint64_t dims[2] = {static_cast<cuuint64_t>(inner), static_cast<cuuint64_t>(rows)};
    cuuint64_t strides[1] = {static_cast<cuuint64_t>(row_stride) * 2};
    cuuint32_t box[2] = {static_cast<cuuint32_t>(box_inner), static_cast<cuuint32_t>(box_rows)};
    cuuint32_t estr[2] = {1, 1};
    CUresult r = g_encode(map, dtype, 2, const_cast<void *>(base), dims, strides, box, estr,
                          CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                          CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) {
        char buf[128];
        snprintf(buf, sizeof(buf), "cuTensorMapEncodeTiled(2d) failed with %d", static_cast<int>(r));
        set_error(SMOL_B200_ERR_CUDA, buf);
        return false;
    }
    return true;
}

bool make_tmap_3d(CUtensorMap *map, const void *base, CUtensorMapDataType dtype, int64_t inner, int64_t rows,
                  int64_t outer, int64_t row_stride, int64_t outer_stride, int box_inner, int box_rows,
                  int elem_bytes)
{
    if (!encode_fn()) return false;
    cuuint64_t dims[3] = {static_cast<cuuint64_t>(inner), static_cast<cuuint64_t>(rows),
                          static_cast<cuuint64_t>(outer)};
    cuuint64_t strides[2] = {static_cast<cuuint64_t>(row_stride) * elem_bytes,
                             static_cast<cuuint64_t>(outer_stride) * elem_bytes};
    cuuint32_t box[3] = {static_cast<cuuint32_t>(box_inner), static_cast<cuuint32_t>(box_rows), 1};
    cuuint32_t estr[3] = {1, 1, 1};
    CUresult r = g_encode(map, dtype, 3, const_cast<void *>(base), dims, strides, box, estr,
                          CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                          CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) {
        char buf[128];
        snprintf(buf, sizeof(buf), "cuTensorMapEncodeTiled(3d) failed with %d", static_cast<int>(r));
        set_error(SMOL_B200_ERR_CUDA, buf);
        return false;
    }
    return true;
}

bool make_tmap_4d(CUtensorMap *map, const void *base, CUtensorMapDataType dtype, int elem_bytes, int64_t inner,
                  int64_t d1, int64_t d2, int64_t d3, int64_t s1, int64_t s2, int64_t s3, int b0, int b1, int b2)
{
    if (!encode_fn()) return false;
    cuuint64_t dims[4] = {static_cast<cuuint64_t>(inner), static_cast<cuuint64_t>(d1), static_cast<cuuint64_t>(d2),
                          static_cast<cuuint64_t>(d3)};
    cuuint64_t strides[3] = {static_cast<cuuint64_t>(s1) * elem_bytes, static_cast<cuuint64_t>(s2) * elem_bytes,
                             static_cast<cuuint64_t>(s3) * elem_bytes};
    cuuint32_t box[4] = {static_cast<cuuint32_t>(b0), static_cast<cuuint32_t>(b1), static_cast<cuuint32_t>(b2), 1};
    cuuint32_t estr[4] = {1, 1, 1, 1};
    CUresult r = g_encode(map, dtype, 4, const_cast<void *>(base), dims, strides, box, estr,
                          CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                          CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) {
        char buf[128];
        snprintf(buf, sizeof(buf), "cuTensorMapEncodeTiled(4d) failed with %d", static_cast<int>(r));
        set_error(SMOL_B200_ERR_CUDA, buf);
        return false;
    }
    return true;
}

}  // namespace smolb200

// ---------------------------------------------------------------------------
// Part 2 of smol_b200.h
// ---------------------------------------------------------------------------
extern "C" {

int smol_cuda_last_error(void) { return smolb200::g_last_error; }

const char *smol_cuda_error_string(int code)
{
    switch (code) {
    case SMOL_B200_OK: return "ok";
    case SMOL_B200_ERR_ARGS: return "arguments outside the supported range";
    case SMOL_B200_ERR_CUDA: return "CUDA runtime error";
    case SMOL_B200_ERR_NO_DEVICE: return "no usable CUDA device";
    case SMOL_B200_ERR_OOM: return "device out of memory";
    case SMOL_B200_ERR_WATCHDOG: return "a kernel wait ran out of time";
    case SMOL_B200_ERR_WORKSPACE: return "workspace too small";
    case SMOL_B200_ERR_RANGE: return "a value outside the range of its storage format";
    default: return "unknown error";
    }
}

void smol_cuda_clear_error(void)
{
    smolb200::g_last_error = SMOL_B200_OK;
    smolb200::g_reported = false;
    int dev = -1;
    if (cudaGetDevice(&dev) == cudaSuccess && dev >= 0 && dev < smolb200::kMaxDevices &&
        smolb200::g_ctx[dev].init.load(std::memory_order_acquire)) {
        cudaMemset(smolb200::g_ctx[dev].err_word, 0, sizeof(unsigned));
        cudaDeviceSynchronize();
    }
    smolb200::noalloc_watchdog_bits(true);   // the allocation-free entry point's word, if it ran here
    cudaGetLastError();
}

unsigned smol_cuda_device_error(void)
{
    // A process that only uses the allocation-free entry point has no error word and
    // gets none here (making it allocates); that entry point's kernels leave their bits
    // in word 0 of its own array, read below.
    const bool noalloc = smolb200::noalloc_in_use();
    unsigned *w = noalloc ? smolb200::device_error_word_if_created() : smolb200::device_error_word();
    if (!w && !noalloc) return 0;
    unsigned v = 0;
    if (cudaDeviceSynchronize() != cudaSuccess) {
        cudaGetLastError();
        return 0xffffffffu;
    }
    if (w && cudaMemcpy(&v, w, sizeof(v), cudaMemcpyDeviceToHost) != cudaSuccess) {
        cudaGetLastError();
        return 0xffffffffu;
    }
    return v | smolb200::noalloc_watchdog_bits(false);
}

}  // extern "C"
