// noalloc.cu -- pfng_b200_compute_q4_0_noalloc: the q4_0 x q8_0 tensor-core
// matmul on fp32 activations for callers that must not allocate device memory.
//
// Some callers cannot call cudaMalloc (or have a caller-side allocator hand
// out a workspace) on this call path: an inference server that reserves all
// of a GPU's memory in its own pool when it starts and forbids any other
// allocation afterwards, or a latency-critical loop that cannot afford the
// device-wide synchronisation cudaMalloc / cudaFree can cause.  For them this
// entry point keeps its scratch -- the quantized activation rows of the
// tensor-core path and, for the small-m shapes that split k, the split
// products' fp32 tiles -- in a fixed array compiled into the library, so a
// call allocates nothing.  It makes the same kernel choices as
// pfng_b200_compute_q4_0 on the tensor-core path (the same split-k factor
// included), so its C is bit-identical to that call's.
//
// The array is kNoAllocScratchBytes (16 MiB), and every GPU that loads the
// library holds it until the process exits.  All calls on a device share it
// and it keeps the previous call's contents.  Every call writes the whole
// region it later reads (the quantizer fills every padded row, every split
// writes its whole tile) before anything reads it, so nothing has to be
// cleared first; but two calls whose kernels run at the same time on one
// device (different streams, or different host threads) would overwrite
// each other's scratch, so callers must keep them ordered.
//
// The device address of the array is looked up once per device and cached
// for the life of the process; like the rest of the library's per-device
// state it does not survive cudaDeviceReset (or a reset of the primary
// context), after which the library must not be used in this process.
#include <mutex>

#include "pfng_b200.h"
#include "pfng_common.cuh"
#include "pfng_internal.h"

namespace pfng {
namespace {

constexpr size_t kNoAllocScratchBytes = PFNG_B200_NOALLOC_SCRATCH_BYTES;

// The scratch itself.  In host code this name is only a stand-in for the
// device array: its device address comes from cudaGetSymbolAddress below.
static __device__ __align__(256) uint8_t g_noalloc_scratch[kNoAllocScratchBytes];

constexpr int kMaxDevices = 64;
void *g_scratch_ptr[kMaxDevices] = {};
std::mutex g_scratch_mutex;

int status_of(cudaError_t e) { return e == cudaSuccess ? PFNG_B200_OK : PFNG_B200_ERR_CUDA_BASE - static_cast<int>(e); }

// Device address of this device's scratch, looked up on the first call made
// with that device current.
int scratch_for_current_device(void **out) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return status_of(e);
    if (dev < 0 || dev >= kMaxDevices) return PFNG_B200_ERR_DEVICE;
    std::lock_guard<std::mutex> lock(g_scratch_mutex);
    if (!g_scratch_ptr[dev]) {
        int major = 0;
        if ((e = cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev)) != cudaSuccess)
            return status_of(e);
        if (major != 10) return PFNG_B200_ERR_DEVICE;
        void *p = nullptr;
        if ((e = cudaGetSymbolAddress(&p, g_noalloc_scratch)) != cudaSuccess) return status_of(e);
        g_scratch_ptr[dev] = p;
    }
    *out = g_scratch_ptr[dev];
    return PFNG_B200_OK;
}

bool aligned(const void *p, uintptr_t a) { return (reinterpret_cast<uintptr_t>(p) & (a - 1)) == 0; }

}  // namespace
}  // namespace pfng

using namespace pfng;

extern "C" int pfng_b200_compute_q4_0_noalloc(const void *w, const float *x, int64_t ldx, float *c, int64_t m,
                                              int64_t n, int64_t k, int64_t ldc, void *stream) {
    // argument checks, on the host, before any CUDA call
    if (m < 0 || n < 0 || k < 0) return PFNG_B200_ERR_INVALID_ARGUMENT;
    if (k % 32 != 0) return PFNG_B200_ERR_SHAPE;
    if (m > 0 && (ldc < n || ldx < k)) return PFNG_B200_ERR_SHAPE;
    if (m == 0 || n == 0) return PFNG_B200_OK;
    if (!w || !x || !c) return PFNG_B200_ERR_INVALID_ARGUMENT;
    if (!aligned(w, 2) || !aligned(x, 4) || !aligned(c, 4)) return PFNG_B200_ERR_ALIGNMENT;
    if (k == 0 || k % 256 != 0 || !aligned(w, 16)) return PFNG_B200_ERR_UNSUPPORTED;  // tensor-core path only
    // the split activation operand, then (shapes that split k) the split tiles
    const size_t a_bytes = split_a_bytes(m, k, 32);
    if (a_bytes > kNoAllocScratchBytes) return PFNG_B200_ERR_WORKSPACE;  // beyond the fixed scratch

    void *scratch = nullptr;
    int st = scratch_for_current_device(&scratch);
    if (st != PFNG_B200_OK) return st;
    if (!gemm_supported(PFNG_B200_Q4_0, m, n, k, w)) return PFNG_B200_ERR_UNSUPPORTED;

    // split-k tiles as pfng_b200_compute_q4_0 carves them from its workspace
    // (256-byte aligned, behind the activation operand)
    const size_t part = gemm_partial_bytes(m, n, k);
    if (part > 0 && a_bytes + part + 256 > kNoAllocScratchBytes) return PFNG_B200_ERR_WORKSPACE;

    const cudaStream_t s = static_cast<cudaStream_t>(stream);
    const SplitA sa = split_a_carve(scratch, m, k, 32);
    cudaError_t e = launch_quantize_q8_0_split(x, ldx, sa, m, k, s);
    if (e != cudaSuccess) return status_of(e);
    GemmArgs g{PFNG_B200_Q4_0, w, sa, c, ldc, nullptr, m, n, k, device_error_word()};
    if (part > 0) {
        const uintptr_t end = reinterpret_cast<uintptr_t>(scratch) + a_bytes;
        g.partial = reinterpret_cast<float *>((end + 255u) & ~uintptr_t(255));
        g.partial_bytes = part;
    }
    return status_of(launch_gemm(g, s));
}
