// api.cu -- the extern "C" entry points of libpfng_b200 (include/pfng_b200.h):
// host-side argument checks, kernel-path selection and workspace carving.
//
// Argument checks run before any CUDA call, so a rejected call has no device
// side effects and can be exercised on a machine without a GPU.
#include <cuda_runtime.h>

#include <cstring>
#include <mutex>

#include "pfng_b200.h"
#include "pfng_common.cuh"
#include "pfng_internal.h"

namespace pfng {

// Library error word for bounded waits (one per device, in the module).
__device__ int g_kernel_error_word;

namespace {

constexpr int kMaxDevices = 64;
struct DeviceInfo {
    int sm_count = 0;
    size_t smem_optin = 0;
    int major = 0;
    int *error_word = nullptr;
    bool ready = false;
};
DeviceInfo g_devices[kMaxDevices];
std::mutex g_devices_mutex;

int status_of(cudaError_t e) { return e == cudaSuccess ? PFNG_B200_OK : PFNG_B200_ERR_CUDA_BASE - static_cast<int>(e); }

// Queries (once per device) what the launchers need; returns a status.
int device_info(DeviceInfo **out) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return status_of(e);
    if (dev < 0 || dev >= kMaxDevices) return PFNG_B200_ERR_DEVICE;
    std::lock_guard<std::mutex> lock(g_devices_mutex);
    DeviceInfo &info = g_devices[dev];
    if (!info.ready) {
        int sms = 0, optin = 0, major = 0;
        if ((e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev)) != cudaSuccess) return status_of(e);
        if ((e = cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev)) != cudaSuccess)
            return status_of(e);
        if ((e = cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev)) != cudaSuccess)
            return status_of(e);
        void *word = nullptr;
        if ((e = cudaGetSymbolAddress(&word, g_kernel_error_word)) != cudaSuccess) return status_of(e);
        info.sm_count = sms;
        info.smem_optin = static_cast<size_t>(optin);
        info.major = major;
        info.error_word = static_cast<int *>(word);
        info.ready = true;
    }
    if (info.major != 10) return PFNG_B200_ERR_DEVICE;
    *out = &info;
    return PFNG_B200_OK;
}

DeviceInfo *current_info() {
    DeviceInfo *info = nullptr;
    return device_info(&info) == PFNG_B200_OK ? info : nullptr;
}

bool aligned(const void *p, uintptr_t a) { return (reinterpret_cast<uintptr_t>(p) & (a - 1)) == 0; }

static_assert(PFNG_B200_Q4_0 == kWQ4_0 && PFNG_B200_Q4_K == kWQ4_K && PFNG_B200_IQ2_XXS == kWIQ2 &&
                  PFNG_B200_Q4_0_PLANAR == kWQ4_0P,
              "weight type codes");
bool valid_wtype(int wtype) { return wtype >= PFNG_B200_Q4_0 && wtype <= PFNG_B200_Q4_0_PLANAR; }
// q4_0 (either layout) pairs with q8_0 activations, the others with q8_K
bool q8_0_act(int wtype) { return wtype == PFNG_B200_Q4_0 || wtype == PFNG_B200_Q4_0_PLANAR; }
int block_k(int wtype) { return q8_0_act(wtype) ? 32 : 256; }
size_t a_block_bytes(int wtype) { return q8_0_act(wtype) ? kQ8_0Bytes : kQ8_KBytes; }
uintptr_t w_align(int wtype) {
    return wtype == PFNG_B200_Q4_0_PLANAR ? 16 : wtype == PFNG_B200_Q4_K ? 4 : 2;
}
uintptr_t a_align(int wtype) { return q8_0_act(wtype) ? 2 : 4; }

// Common shape/pointer checks for the matmul-family entry points.
int check_mm(int wtype, const void *w, const void *a_or_x, const void *out, int64_t m, int64_t n, int64_t k,
             int64_t ldc, int64_t ldx, bool f32_input, bool partials, int path) {
    if (!valid_wtype(wtype)) return PFNG_B200_ERR_INVALID_ARGUMENT;
    if (m < 0 || n < 0 || k < 0) return PFNG_B200_ERR_INVALID_ARGUMENT;
    if (path < PFNG_B200_PATH_AUTO || path > PFNG_B200_PATH_SIMPLE) return PFNG_B200_ERR_INVALID_ARGUMENT;
    if (k % block_k(wtype) != 0) return PFNG_B200_ERR_SHAPE;
    if (wtype == PFNG_B200_Q4_0_PLANAR && k % 256 != 0) return PFNG_B200_ERR_SHAPE;
    if (!partials && m > 0 && ldc < n) return PFNG_B200_ERR_SHAPE;
    if (f32_input && m > 0 && ldx < k) return PFNG_B200_ERR_SHAPE;
    if (m == 0 || n == 0) return PFNG_B200_OK;
    if (!out) return PFNG_B200_ERR_INVALID_ARGUMENT;
    if (!aligned(out, 4)) return PFNG_B200_ERR_ALIGNMENT;
    if (k == 0) return PFNG_B200_OK;
    if (!w || !a_or_x) return PFNG_B200_ERR_INVALID_ARGUMENT;
    if (!aligned(w, w_align(wtype))) return PFNG_B200_ERR_ALIGNMENT;
    if (!aligned(a_or_x, f32_input ? 4 : a_align(wtype))) return PFNG_B200_ERR_ALIGNMENT;
    return PFNG_B200_OK;
}

int check_quant(const float *x, int64_t ldx, const void *y, int64_t rows, int64_t k, int qk, uintptr_t yalign) {
    if (rows < 0 || k < 0) return PFNG_B200_ERR_INVALID_ARGUMENT;
    if (k % qk != 0) return PFNG_B200_ERR_SHAPE;
    if (rows > 0 && ldx < k) return PFNG_B200_ERR_SHAPE;
    if (rows == 0 || k == 0) return PFNG_B200_OK;
    if (!x || !y) return PFNG_B200_ERR_INVALID_ARGUMENT;
    if (!aligned(x, 4) || !aligned(y, yalign)) return PFNG_B200_ERR_ALIGNMENT;
    return PFNG_B200_OK;
}

// Resolved kernel path for a matmul call.
int resolve_path(int wtype, int64_t m, int64_t n, int64_t k, const void *w, int path) {
    if (path == PFNG_B200_PATH_AUTO) {
        if (m <= 8 && gemv_supported(wtype, m, 1, &n, k, &w)) return PFNG_B200_PATH_GEMV;
        if (m > 8 && gemm_supported(wtype, m, n, k, w)) return PFNG_B200_PATH_MMA;
        return PFNG_B200_PATH_SIMPLE;
    }
    if (path == PFNG_B200_PATH_GEMV && !gemv_supported(wtype, m, 1, &n, k, &w)) return -1;
    if (path == PFNG_B200_PATH_MMA && !gemm_supported(wtype, m, n, k, w)) return -1;
    return path;
}

size_t raw_a_bytes(int wtype, int64_t m, int64_t k) {
    return static_cast<size_t>(m) * static_cast<size_t>(k / block_k(wtype)) * a_block_bytes(wtype);
}

// Workspace needed by a resolved path (f32: activations arrive as fp32).
size_t workspace_for(int wtype, int64_t m, int64_t n, int64_t k, int resolved, bool f32) {
    if (m == 0 || k == 0) return 0;
    if (resolved == PFNG_B200_PATH_MMA) {
        // the split activation operand, then the split-K partial tiles if the
        // shape is split (gemm_partial_bytes)
        const size_t part = gemm_partial_bytes(m, n, k);
        return split_a_bytes(m, k, block_k(wtype) == 32 ? 32 : 256) + (part > 0 ? part + 256 : 0);
    }
    if (resolved == PFNG_B200_PATH_SIMPLE && f32) return raw_a_bytes(wtype, m, k) + 256;
    return 0;
}

cudaError_t zero_c(float *c, int64_t m, int64_t n, int64_t ldc, cudaStream_t s) {
    return cudaMemset2DAsync(c, static_cast<size_t>(ldc) * sizeof(float), 0, static_cast<size_t>(n) * sizeof(float),
                             static_cast<size_t>(m), s);
}

void *align_ptr(void *p, uintptr_t a) {
    return reinterpret_cast<void *>((reinterpret_cast<uintptr_t>(p) + a - 1) & ~(a - 1));
}

// Split-K partial tiles behind the split activation operand in the workspace.
void carve_partial(GemmArgs &g, void *workspace, size_t workspace_need, int wtype, int64_t m, int64_t k) {
    const size_t a_bytes = split_a_bytes(m, k, block_k(wtype));
    if (workspace_need <= a_bytes) return;
    g.partial = static_cast<float *>(align_ptr(static_cast<uint8_t *>(workspace) + a_bytes, 256));
    g.partial_bytes = workspace_need - a_bytes - 256;
}

// The shared body of mm / compute / partials.
// `copies` (fp32 C only): ncopies more destinations that receive C with
// C's layout -- the MMA GEMM stores each tile to all of them in its
// epilogue, the other paths copy C after computing it.
int run_matmul(int wtype, const void *w, const void *a, const float *x, int64_t ldx, float *c, int64_t ldc,
               int32_t *partials, int64_t m, int64_t n, int64_t k, void *workspace, size_t workspace_bytes,
               int path, cudaStream_t s, float *const *copies = nullptr, int ncopies = 0) {
    const bool f32 = x != nullptr;
    int st = check_mm(wtype, w, f32 ? static_cast<const void *>(x) : a, partials ? static_cast<void *>(partials) : c,
                      m, n, k, ldc, ldx, f32, partials != nullptr, path);
    if (st != PFNG_B200_OK || m == 0 || n == 0) return st;
    DeviceInfo *info = nullptr;
    if ((st = device_info(&info)) != PFNG_B200_OK) return st;
    if (k == 0) {
        if (partials) return PFNG_B200_OK;
        cudaError_t e = zero_c(c, m, n, ldc, s);
        for (int d = 0; d < ncopies && e == cudaSuccess; ++d) e = zero_c(copies[d], m, n, ldc, s);
        return status_of(e);
    }
    const int resolved = resolve_path(wtype, m, n, k, w, path);
    if (resolved < 0) return PFNG_B200_ERR_UNSUPPORTED;
    const size_t need = workspace_for(wtype, m, n, k, resolved, f32);
    if (need > 0 && (!workspace || workspace_bytes < need)) return PFNG_B200_ERR_WORKSPACE;

    cudaError_t e = cudaSuccess;
    if (resolved == PFNG_B200_PATH_GEMV) {
        GemvArgs g{};
        g.wtype = wtype;
        g.count = 1;
        g.w[0] = w;
        g.c[0] = c;
        g.ldc[0] = ldc;
        g.n[0] = n;
        g.a = f32 ? nullptr : a;
        g.x = x;
        g.ldx = ldx;
        g.partials = partials;
        g.err = info->error_word;
        g.m = m;
        g.k = k;
        e = launch_gemv(g, s);
    } else if (resolved == PFNG_B200_PATH_MMA) {
        const int qk = block_k(wtype);
        const SplitA sa = split_a_carve(workspace, m, k, qk);
        if (q8_0_act(wtype))
            e = f32 ? launch_quantize_q8_0_split(x, ldx, sa, m, k, s) : launch_convert_q8_0_split(a, sa, m, k, s);
        else
            e = f32 ? launch_quantize_q8_K_split(x, ldx, sa, m, k, s) : launch_convert_q8_K_split(a, sa, m, k, s);
        if (e == cudaSuccess) {
            GemmArgs g{wtype, w, sa, c, ldc, partials, m, n, k, info->error_word};
            carve_partial(g, workspace, need, wtype, m, k);
            g.copies = copies;
            g.ncopies = ncopies;
            e = launch_gemm(g, s);
        }
        return status_of(e);
    } else {
        const void *araw = a;
        if (f32) {
            void *buf = align_ptr(workspace, 256);
            e = q8_0_act(wtype) ? launch_quantize_q8_0(x, ldx, buf, m, k, s)
                                : launch_quantize_q8_K(x, ldx, buf, m, k, s);
            araw = buf;
        }
        if (e == cudaSuccess) {
            SimpleArgs g{wtype, w, araw, c, ldc, partials, m, n, k};
            e = launch_simple(g, s);
        }
    }
    // GEMV and SIMPLE: C to the other destinations by device copies
    const size_t pitch = static_cast<size_t>(ldc) * sizeof(float);
    for (int d = 0; d < ncopies && e == cudaSuccess; ++d)
        e = cudaMemcpy2DAsync(copies[d], pitch, c, pitch, static_cast<size_t>(n) * sizeof(float),
                              static_cast<size_t>(m), cudaMemcpyDefault, s);
    return status_of(e);
}

static_assert(PFNG_B200_OUT_F32 == kOutF32 && PFNG_B200_OUT_F16 == kOutF16 && PFNG_B200_OUT_BF16 == kOutBF16 &&
                  PFNG_B200_OUT_Q8_0 == kOutQ8_0,
              "output format codes");

// fp32 C scratch the non-fused paths need for an output format.
size_t c_scratch_bytes(int64_t m, int64_t n) { return static_cast<size_t>(m) * static_cast<size_t>(n) * 4 + 256; }

// Workspace of a resolved path writing output format `fmt`: the MMA GEMM
// converts in its epilogue; GEMV and SIMPLE write fp32 C to scratch first.
size_t out_workspace_for(int wtype, int fmt, int64_t m, int64_t n, int64_t k, int resolved, bool f32) {
    const size_t base = workspace_for(wtype, m, n, k, resolved, f32);
    if (fmt == kOutF32 || resolved == PFNG_B200_PATH_MMA || m == 0 || n == 0) return base;
    return round_up(static_cast<int64_t>(base), 256) + c_scratch_bytes(m, n);
}

// The shared body of mm_out / compute_out.
int run_matmul_out(int wtype, const void *w, const void *a, const float *x, int64_t ldx, void *out, int fmt,
                   int64_t ldo, int64_t m, int64_t n, int64_t k, void *workspace, size_t workspace_bytes, int path,
                   cudaStream_t s) {
    if (fmt < kOutF32 || fmt > kOutQ8_0) return PFNG_B200_ERR_INVALID_ARGUMENT;
    if (fmt == kOutF32)
        return run_matmul(wtype, w, a, x, ldx, static_cast<float *>(out), ldo, nullptr, m, n, k, workspace,
                          workspace_bytes, path, s);
    const bool f32 = x != nullptr;
    // the common checks, with a stand-in for C: ldo and the (2-byte)
    // alignment of out are checked per format below
    const void *c_probe = out ? reinterpret_cast<const void *>(uintptr_t{256}) : nullptr;
    int st = check_mm(wtype, w, f32 ? static_cast<const void *>(x) : a, c_probe, m, n, k, n, ldx, f32, false, path);
    if (st != PFNG_B200_OK) return st;
    if (fmt == kOutQ8_0 && n % 32 != 0) return PFNG_B200_ERR_SHAPE;
    if (m > 0 && ldo < (fmt == kOutQ8_0 ? n / 32 : n)) return PFNG_B200_ERR_SHAPE;
    if (m == 0 || n == 0) return PFNG_B200_OK;
    if (!aligned(out, 2)) return PFNG_B200_ERR_ALIGNMENT;
    if (!w || !(f32 ? static_cast<const void *>(x) : a)) {
        if (k != 0) return PFNG_B200_ERR_INVALID_ARGUMENT;
    }
    DeviceInfo *info = nullptr;
    if ((st = device_info(&info)) != PFNG_B200_OK) return st;
    const int resolved = k == 0 ? PFNG_B200_PATH_SIMPLE : resolve_path(wtype, m, n, k, w, path);
    if (resolved < 0) return PFNG_B200_ERR_UNSUPPORTED;
    const size_t need = out_workspace_for(wtype, fmt, m, n, k, resolved, f32);
    if (need > 0 && (!workspace || workspace_bytes < need)) return PFNG_B200_ERR_WORKSPACE;
    cudaError_t e = cudaSuccess;
    if (resolved == PFNG_B200_PATH_MMA) {
        const int qk = block_k(wtype);
        const SplitA sa = split_a_carve(workspace, m, k, qk);
        if (q8_0_act(wtype))
            e = f32 ? launch_quantize_q8_0_split(x, ldx, sa, m, k, s) : launch_convert_q8_0_split(a, sa, m, k, s);
        else
            e = f32 ? launch_quantize_q8_K_split(x, ldx, sa, m, k, s) : launch_convert_q8_K_split(a, sa, m, k, s);
        if (e == cudaSuccess) {
            GemmArgs g{wtype, w, sa, nullptr, 0, nullptr, m, n, k, info->error_word};
            g.out_format = fmt;
            g.out = out;
            g.ldo = ldo;
            carve_partial(g, workspace, need, wtype, m, k);
            e = launch_gemm(g, s);
        }
        return status_of(e);
    }
    // fp32 C into scratch behind the path's own workspace, then convert
    const size_t base = workspace_for(wtype, m, n, k, resolved, f32);
    uint8_t *ws = static_cast<uint8_t *>(workspace);
    float *cs = static_cast<float *>(align_ptr(ws + round_up(static_cast<int64_t>(base), 256), 256));
    st = run_matmul(wtype, w, a, x, ldx, cs, n, nullptr, m, n, k, workspace, base, resolved, s);
    if (st != PFNG_B200_OK) return st;
    e = fmt == kOutQ8_0 ? launch_quantize_q8_0_strided(cs, n, out, ldo, m, n, s)
                        : launch_convert_out(cs, n, out, ldo, fmt, m, n, s);
    return status_of(e);
}

size_t query_out_workspace(int wtype, int fmt, int64_t m, int64_t n, int64_t k, int path, bool f32) {
    if (!valid_wtype(wtype) || fmt < kOutF32 || fmt > kOutQ8_0 || m <= 0 || n <= 0 || k <= 0) return 0;
    if (path == PFNG_B200_PATH_AUTO) {
        size_t best = 0;
        for (int cand : {PFNG_B200_PATH_GEMV, PFNG_B200_PATH_MMA, PFNG_B200_PATH_SIMPLE}) {
            if (cand == PFNG_B200_PATH_GEMV && m > 8) continue;
            if (cand == PFNG_B200_PATH_MMA && m <= 8) continue;
            const size_t need = out_workspace_for(wtype, fmt, m, n, k, cand, f32);
            best = need > best ? need : best;
        }
        return best;
    }
    return out_workspace_for(wtype, fmt, m, n, k, path, f32);
}

size_t query_workspace(int wtype, int64_t m, int64_t n, int64_t k, int path, bool f32) {
    if (!valid_wtype(wtype) || m <= 0 || n <= 0 || k <= 0) return 0;
    if (path == PFNG_B200_PATH_AUTO) {
        // AUTO may take the tensor-core or the simple path depending on the
        // pointers' alignment, so ask for what either needs.
        const size_t mma = m > 8 ? workspace_for(wtype, m, n, k, PFNG_B200_PATH_MMA, f32) : 0;
        const size_t simple = workspace_for(wtype, m, n, k, PFNG_B200_PATH_SIMPLE, f32);
        return mma > simple ? mma : simple;
    }
    return workspace_for(wtype, m, n, k, path, f32);
}

}  // namespace

int device_sm_count() {
    DeviceInfo *info = current_info();
    return info ? info->sm_count : 148;
}

int *device_error_word() {
    DeviceInfo *info = current_info();
    return info ? info->error_word : nullptr;
}

size_t device_smem_optin() {
    DeviceInfo *info = current_info();
    return info ? info->smem_optin : 0;
}

size_t split_a_bytes(int64_t m, int64_t k, int block) {
    const int64_t rows = round_up(m, kGemmTileM);
    const size_t qs = static_cast<size_t>(rows * k);
    const size_t d = static_cast<size_t>(rows * (k / block)) * sizeof(float);
    const size_t aux = static_cast<size_t>(rows * (k / 32)) * sizeof(int32_t);
    return 256 + round_up(static_cast<int64_t>(qs), 256) + round_up(static_cast<int64_t>(d), 256) +
           round_up(static_cast<int64_t>(aux), 256);
}

SplitA split_a_carve(void *workspace, int64_t m, int64_t k, int block) {
    SplitA s{};
    s.rows_pad = round_up(m, kGemmTileM);
    s.k = k;
    s.d_ld = s.rows_pad;
    uint8_t *p = static_cast<uint8_t *>(align_ptr(workspace, 256));
    s.qs = reinterpret_cast<int8_t *>(p);
    p += round_up(s.rows_pad * k, 256);
    s.d = reinterpret_cast<float *>(p);
    p += round_up(static_cast<int64_t>(s.rows_pad * (k / block) * sizeof(float)), 256);
    s.aux = reinterpret_cast<int32_t *>(p);
    return s;
}

}  // namespace pfng

using namespace pfng;

extern "C" {

int pfng_b200_version(void) { return 1; }

const char *pfng_b200_status_string(int status) {
    switch (status) {
    case PFNG_B200_OK: return "ok";
    case PFNG_B200_ERR_INVALID_ARGUMENT: return "invalid argument";
    case PFNG_B200_ERR_SHAPE: return "unsupported shape";
    case PFNG_B200_ERR_ALIGNMENT: return "misaligned pointer";
    case PFNG_B200_ERR_WORKSPACE: return "workspace missing or too small";
    case PFNG_B200_ERR_DEVICE: return "device is not compute capability 10.x";
    case PFNG_B200_ERR_KERNEL_TIMEOUT: return "a bounded wait inside a kernel gave up";
    case PFNG_B200_ERR_UNSUPPORTED: return "forced kernel path cannot run this shape";
    default:
        if (status <= PFNG_B200_ERR_CUDA_BASE)
            return cudaGetErrorString(static_cast<cudaError_t>(PFNG_B200_ERR_CUDA_BASE - status));
        return "unknown status";
    }
}

int pfng_b200_check_kernel_error(void *stream) {
    DeviceInfo *info = nullptr;
    int st = device_info(&info);
    if (st != PFNG_B200_OK) return st;
    cudaError_t e = cudaStreamSynchronize(static_cast<cudaStream_t>(stream));
    if (e != cudaSuccess) return status_of(e);
    int value = 0;
    if ((e = cudaMemcpy(&value, info->error_word, sizeof(int), cudaMemcpyDeviceToHost)) != cudaSuccess)
        return status_of(e);
    if (value == 0) return PFNG_B200_OK;
    const int zero = 0;
    if ((e = cudaMemcpy(info->error_word, &zero, sizeof(int), cudaMemcpyHostToDevice)) != cudaSuccess)
        return status_of(e);
    return PFNG_B200_ERR_KERNEL_TIMEOUT;
}

int pfng_b200_quantize_q8_0(const float *x, int64_t ldx, void *y, int64_t m, int64_t k, void *stream) {
    int st = check_quant(x, ldx, y, m, k, 32, 2);
    if (st != PFNG_B200_OK || m == 0 || k == 0) return st;
    DeviceInfo *info = nullptr;
    if ((st = device_info(&info)) != PFNG_B200_OK) return st;
    return status_of(launch_quantize_q8_0(x, ldx, y, m, k, static_cast<cudaStream_t>(stream)));
}

int pfng_b200_quantize_q8_K(const float *x, int64_t ldx, void *y, int64_t m, int64_t k, void *stream) {
    int st = check_quant(x, ldx, y, m, k, 256, 4);
    if (st != PFNG_B200_OK || m == 0 || k == 0) return st;
    DeviceInfo *info = nullptr;
    if ((st = device_info(&info)) != PFNG_B200_OK) return st;
    return status_of(launch_quantize_q8_K(x, ldx, y, m, k, static_cast<cudaStream_t>(stream)));
}

int pfng_b200_quantize_q4_0(const float *x, int64_t ldx, void *y, int64_t n, int64_t k, void *stream) {
    int st = check_quant(x, ldx, y, n, k, 32, 2);
    if (st != PFNG_B200_OK || n == 0 || k == 0) return st;
    DeviceInfo *info = nullptr;
    if ((st = device_info(&info)) != PFNG_B200_OK) return st;
    return status_of(launch_quantize_q4_0(x, ldx, y, n, k, static_cast<cudaStream_t>(stream)));
}

int pfng_b200_quantize_q4_K(const float *x, int64_t ldx, void *y, int64_t n, int64_t k, void *stream) {
    int st = check_quant(x, ldx, y, n, k, 256, 4);
    if (st != PFNG_B200_OK || n == 0 || k == 0) return st;
    DeviceInfo *info = nullptr;
    if ((st = device_info(&info)) != PFNG_B200_OK) return st;
    return status_of(launch_quantize_q4_K(x, ldx, y, n, k, static_cast<cudaStream_t>(stream)));
}

size_t pfng_b200_mm_workspace_size(int wtype, int64_t m, int64_t n, int64_t k, int path) {
    return query_workspace(wtype, m, n, k, path, false);
}

size_t pfng_b200_compute_workspace_size(int wtype, int64_t m, int64_t n, int64_t k, int path) {
    return query_workspace(wtype, m, n, k, path, true);
}

int pfng_b200_mm_q4_0_q8_0(const void *w, const void *a, float *c, int64_t m, int64_t n, int64_t k, int64_t ldc,
                           void *workspace, size_t workspace_bytes, int path, void *stream) {
    return run_matmul(PFNG_B200_Q4_0, w, a, nullptr, 0, c, ldc, nullptr, m, n, k, workspace, workspace_bytes, path,
                      static_cast<cudaStream_t>(stream));
}

int pfng_b200_mm_q4_K_q8_K(const void *w, const void *a, float *c, int64_t m, int64_t n, int64_t k, int64_t ldc,
                           void *workspace, size_t workspace_bytes, int path, void *stream) {
    return run_matmul(PFNG_B200_Q4_K, w, a, nullptr, 0, c, ldc, nullptr, m, n, k, workspace, workspace_bytes, path,
                      static_cast<cudaStream_t>(stream));
}

int pfng_b200_mm_iq2_xxs_q8_K(const void *w, const void *a, float *c, int64_t m, int64_t n, int64_t k, int64_t ldc,
                              void *workspace, size_t workspace_bytes, int path, void *stream) {
    return run_matmul(PFNG_B200_IQ2_XXS, w, a, nullptr, 0, c, ldc, nullptr, m, n, k, workspace, workspace_bytes, path,
                      static_cast<cudaStream_t>(stream));
}

int pfng_b200_compute_q4_0(const void *w, const float *x, int64_t ldx, float *c, int64_t m, int64_t n, int64_t k,
                           int64_t ldc, void *workspace, size_t workspace_bytes, int path, void *stream) {
    return run_matmul(PFNG_B200_Q4_0, w, nullptr, x, ldx, c, ldc, nullptr, m, n, k, workspace, workspace_bytes, path,
                      static_cast<cudaStream_t>(stream));
}

int pfng_b200_compute_q4_K(const void *w, const float *x, int64_t ldx, float *c, int64_t m, int64_t n, int64_t k,
                           int64_t ldc, void *workspace, size_t workspace_bytes, int path, void *stream) {
    return run_matmul(PFNG_B200_Q4_K, w, nullptr, x, ldx, c, ldc, nullptr, m, n, k, workspace, workspace_bytes, path,
                      static_cast<cudaStream_t>(stream));
}

int pfng_b200_compute_iq2_xxs(const void *w, const float *x, int64_t ldx, float *c, int64_t m, int64_t n, int64_t k,
                              int64_t ldc, void *workspace, size_t workspace_bytes, int path, void *stream) {
    return run_matmul(PFNG_B200_IQ2_XXS, w, nullptr, x, ldx, c, ldc, nullptr, m, n, k, workspace, workspace_bytes,
                      path, static_cast<cudaStream_t>(stream));
}

// ---- prepared activations: quantize once, multiply by several matrices ----
size_t pfng_b200_prepared_bytes(int wtype, int64_t m, int64_t k) {
    if (!valid_wtype(wtype) || m <= 0 || k <= 0 || k % 256 != 0) return 0;
    return split_a_bytes(m, k, block_k(wtype));
}

int pfng_b200_prepare_activations(int wtype, const float *x, int64_t ldx, void *prepared, size_t prepared_bytes,
                                  int64_t m, int64_t k, void *stream) {
    if (!valid_wtype(wtype) || m < 0 || k < 0) return PFNG_B200_ERR_INVALID_ARGUMENT;
    if (k % 256 != 0) return PFNG_B200_ERR_SHAPE;
    if (m > 0 && ldx < k) return PFNG_B200_ERR_SHAPE;
    if (m == 0 || k == 0) return PFNG_B200_OK;
    if (!x || !prepared) return PFNG_B200_ERR_INVALID_ARGUMENT;
    if (!aligned(x, 4) || !aligned(prepared, 256)) return PFNG_B200_ERR_ALIGNMENT;
    const int qk = block_k(wtype);
    if (prepared_bytes < split_a_bytes(m, k, qk)) return PFNG_B200_ERR_WORKSPACE;
    DeviceInfo *info = nullptr;
    int st = device_info(&info);
    if (st != PFNG_B200_OK) return st;
    const SplitA sa = split_a_carve(prepared, m, k, qk);
    const cudaStream_t s = static_cast<cudaStream_t>(stream);
    return status_of(q8_0_act(wtype) ? launch_quantize_q8_0_split(x, ldx, sa, m, k, s)
                                     : launch_quantize_q8_K_split(x, ldx, sa, m, k, s));
}

size_t pfng_b200_mm_prepared_workspace_size(int wtype, int64_t m, int64_t n, int64_t k) {
    if (!valid_wtype(wtype) || m <= 0 || n <= 0 || k <= 0 || k % 256 != 0) return 0;
    const size_t part = gemm_partial_bytes(m, n, k);
    return part > 0 ? part + 256 : 0;
}

int pfng_b200_mm_prepared(int wtype, const void *w, const void *prepared, float *c, int64_t m, int64_t n, int64_t k,
                          int64_t ldc, void *workspace, size_t workspace_bytes, void *stream) {
    int st = check_mm(wtype, w, prepared, c, m, n, k, ldc, 0, false, false, PFNG_B200_PATH_MMA);
    if (st != PFNG_B200_OK) return st;
    if (k % 256 != 0) return PFNG_B200_ERR_SHAPE;
    if (m == 0 || n == 0) return PFNG_B200_OK;
    DeviceInfo *info = nullptr;
    if (k == 0) {
        if ((st = device_info(&info)) != PFNG_B200_OK) return st;
        return status_of(zero_c(c, m, n, ldc, static_cast<cudaStream_t>(stream)));
    }
    if (!aligned(prepared, 256)) return PFNG_B200_ERR_ALIGNMENT;
    if ((st = device_info(&info)) != PFNG_B200_OK) return st;
    if (!gemm_supported(wtype, m, n, k, w)) return PFNG_B200_ERR_UNSUPPORTED;
    const SplitA sa = split_a_carve(const_cast<void *>(prepared), m, k, block_k(wtype));
    GemmArgs g{wtype, w, sa, c, ldc, nullptr, m, n, k, info->error_word};
    const size_t part = gemm_partial_bytes(m, n, k);
    if (part > 0 && workspace && workspace_bytes >= part + 256) {
        g.partial = static_cast<float *>(align_ptr(workspace, 256));
        g.partial_bytes = part;
    }
    return status_of(launch_gemm(g, static_cast<cudaStream_t>(stream)));
}

int pfng_b200_compute_grouped(int wtype, int count, const void *const *w, const int64_t *n, float *const *c,
                              const int64_t *ldc, const float *x, int64_t ldx, int64_t m, int64_t k, unsigned flags,
                              void *stream) {
    if (!valid_wtype(wtype) || count < 1 || !w || !n || !c || !ldc) return PFNG_B200_ERR_INVALID_ARGUMENT;
    if (flags & ~static_cast<unsigned>(PFNG_B200_OVERLAP_WEIGHTS)) return PFNG_B200_ERR_INVALID_ARGUMENT;
    if (count > kGemvMaxGroup) return PFNG_B200_ERR_UNSUPPORTED;
    for (int g = 0; g < count; ++g) {
        const int st = check_mm(wtype, w[g], x, c[g], m, n[g], k, ldc[g], ldx, true, false, PFNG_B200_PATH_GEMV);
        if (st != PFNG_B200_OK) return st;
    }
    if (m == 0) return PFNG_B200_OK;
    DeviceInfo *info = nullptr;
    int st = device_info(&info);
    if (st != PFNG_B200_OK) return st;
    GemvArgs ga{};
    ga.wtype = wtype;
    for (int g = 0; g < count; ++g) {
        if (n[g] == 0) continue;  // empty matrices take no part
        if (k == 0) {
            if ((st = status_of(zero_c(c[g], m, n[g], ldc[g], static_cast<cudaStream_t>(stream)))) != PFNG_B200_OK)
                return st;
            continue;
        }
        ga.w[ga.count] = w[g];
        ga.c[ga.count] = c[g];
        ga.ldc[ga.count] = ldc[g];
        ga.n[ga.count] = n[g];
        ++ga.count;
    }
    if (ga.count == 0) return PFNG_B200_OK;
    if (!gemv_supported(wtype, m, ga.count, ga.n, k, ga.w)) return PFNG_B200_ERR_UNSUPPORTED;
    ga.x = x;
    ga.ldx = ldx;
    ga.err = info->error_word;
    ga.m = m;
    ga.k = k;
    ga.overlap = (flags & PFNG_B200_OVERLAP_WEIGHTS) != 0;
    return status_of(launch_gemv(ga, static_cast<cudaStream_t>(stream)));
}

int pfng_b200_partials_q4_0_q8_0(const void *w, const void *a, int32_t *out, int64_t m, int64_t n, int64_t k,
                                 void *workspace, size_t workspace_bytes, int path, void *stream) {
    return run_matmul(PFNG_B200_Q4_0, w, a, nullptr, 0, nullptr, n, out, m, n, k, workspace, workspace_bytes, path,
                      static_cast<cudaStream_t>(stream));
}

int pfng_b200_partials_q4_K_q8_K(const void *w, const void *a, int32_t *out, int64_t m, int64_t n, int64_t k,
                                 void *workspace, size_t workspace_bytes, int path, void *stream) {
    return run_matmul(PFNG_B200_Q4_K, w, a, nullptr, 0, nullptr, n, out, m, n, k, workspace, workspace_bytes, path,
                      static_cast<cudaStream_t>(stream));
}

int pfng_b200_partials_iq2_xxs_q8_K(const void *w, const void *a, int32_t *out, int64_t m, int64_t n, int64_t k,
                                    void *workspace, size_t workspace_bytes, int path, void *stream) {
    return run_matmul(PFNG_B200_IQ2_XXS, w, a, nullptr, 0, nullptr, n, out, m, n, k, workspace, workspace_bytes,
                      path, static_cast<cudaStream_t>(stream));
}

size_t pfng_b200_mm_out_workspace_size(int wtype, int out_format, int64_t m, int64_t n, int64_t k, int path) {
    return query_out_workspace(wtype, out_format, m, n, k, path, false);
}

size_t pfng_b200_compute_out_workspace_size(int wtype, int out_format, int64_t m, int64_t n, int64_t k, int path) {
    return query_out_workspace(wtype, out_format, m, n, k, path, true);
}

int pfng_b200_mm_out(int wtype, const void *w, const void *a, void *out, int out_format, int64_t ldo, int64_t m,
                     int64_t n, int64_t k, void *workspace, size_t workspace_bytes, int path, void *stream) {
    return run_matmul_out(wtype, w, a, nullptr, 0, out, out_format, ldo, m, n, k, workspace, workspace_bytes, path,
                          static_cast<cudaStream_t>(stream));
}

int pfng_b200_compute_out(int wtype, const void *w, const float *x, int64_t ldx, void *out, int out_format,
                          int64_t ldo, int64_t m, int64_t n, int64_t k, void *workspace, size_t workspace_bytes,
                          int path, void *stream) {
    if (!x && m > 0 && n > 0 && k > 0) return PFNG_B200_ERR_INVALID_ARGUMENT;
    return run_matmul_out(wtype, w, nullptr, x, ldx, out, out_format, ldo, m, n, k, workspace, workspace_bytes, path,
                          static_cast<cudaStream_t>(stream));
}

int pfng_b200_mm_q4_0p_q8_0(const void *w_planar, const void *a, float *c, int64_t m, int64_t n, int64_t k,
                            int64_t ldc, void *workspace, size_t workspace_bytes, int path, void *stream) {
    return run_matmul(PFNG_B200_Q4_0_PLANAR, w_planar, a, nullptr, 0, c, ldc, nullptr, m, n, k, workspace,
                      workspace_bytes, path, static_cast<cudaStream_t>(stream));
}

int pfng_b200_compute_q4_0p(const void *w_planar, const float *x, int64_t ldx, float *c, int64_t m, int64_t n,
                            int64_t k, int64_t ldc, void *workspace, size_t workspace_bytes, int path, void *stream) {
    return run_matmul(PFNG_B200_Q4_0_PLANAR, w_planar, nullptr, x, ldx, c, ldc, nullptr, m, n, k, workspace,
                      workspace_bytes, path, static_cast<cudaStream_t>(stream));
}

int pfng_b200_partials_q4_0p_q8_0(const void *w_planar, const void *a, int32_t *out, int64_t m, int64_t n, int64_t k,
                                  void *workspace, size_t workspace_bytes, int path, void *stream) {
    return run_matmul(PFNG_B200_Q4_0_PLANAR, w_planar, a, nullptr, 0, nullptr, n, out, m, n, k, workspace,
                      workspace_bytes, path, static_cast<cudaStream_t>(stream));
}

// Shared checks of pack / unpack: raw side 2-byte aligned, planar side 16.
static int planar_copy(bool to_planar, const void *src, void *dst, int64_t n, int64_t k, void *stream) {
    if (n < 0 || k < 0) return PFNG_B200_ERR_INVALID_ARGUMENT;
    if (k % 256 != 0) return PFNG_B200_ERR_SHAPE;
    if (n == 0 || k == 0) return PFNG_B200_OK;
    if (!src || !dst) return PFNG_B200_ERR_INVALID_ARGUMENT;
    const void *raw = to_planar ? src : dst;
    const void *planar = to_planar ? dst : src;
    if (!aligned(raw, 2) || !aligned(planar, 16)) return PFNG_B200_ERR_ALIGNMENT;
    const uintptr_t bytes = static_cast<uintptr_t>(n) * static_cast<uintptr_t>(k / 32) * kQ4_0Bytes;
    const uintptr_t a0 = reinterpret_cast<uintptr_t>(src), b0 = reinterpret_cast<uintptr_t>(dst);
    if (a0 < b0 + bytes && b0 < a0 + bytes) return PFNG_B200_ERR_INVALID_ARGUMENT;  // overlapping buffers
    DeviceInfo *info = nullptr;
    int st = device_info(&info);
    if (st != PFNG_B200_OK) return st;
    const cudaStream_t s = static_cast<cudaStream_t>(stream);
    return status_of(to_planar ? launch_pack_q4_0_planar(src, dst, n, k, s)
                               : launch_unpack_q4_0_planar(src, dst, n, k, s));
}

int pfng_b200_pack_q4_0_planar(const void *w, void *w_planar, int64_t n, int64_t k, void *stream) {
    return planar_copy(true, w, w_planar, n, k, stream);
}

int pfng_b200_unpack_q4_0_planar(const void *w_planar, void *w, int64_t n, int64_t k, void *stream) {
    return planar_copy(false, w_planar, w, n, k, stream);
}

int pfng_b200_shard_rows(int64_t n, int world, int rank, int64_t granule, int64_t *begin, int64_t *end) {
    if (n < 0 || world < 1 || rank < 0 || rank >= world || granule < 1 || !begin || !end)
        return PFNG_B200_ERR_INVALID_ARGUMENT;
    // Split ceil(n / granule) granules as evenly as possible; the first
    // (granules % world) ranks take one extra; the last granule may be ragged.
    const int64_t granules = (n + granule - 1) / granule;
    const int64_t base = granules / world, extra = granules % world;
    const int64_t g0 = rank * base + (rank < extra ? rank : extra);
    const int64_t g1 = g0 + base + (rank < extra ? 1 : 0);
    *begin = g0 * granule < n ? g0 * granule : n;
    *end = g1 * granule < n ? g1 * granule : n;
    return PFNG_B200_OK;
}

int pfng_b200_unshard_columns(const float *slices, float *c, int64_t m, int64_t n, int64_t ldc, int world,
                              int64_t granule, int64_t slice_width, void *stream) {
    if (m < 0 || n < 0 || world < 1 || granule < 1 || slice_width < 0) return PFNG_B200_ERR_INVALID_ARGUMENT;
    if (m > 0 && ldc < n) return PFNG_B200_ERR_SHAPE;
    if (m == 0 || n == 0) return PFNG_B200_OK;
    if (!slices || !c) return PFNG_B200_ERR_INVALID_ARGUMENT;
    if (!aligned(slices, 4) || !aligned(c, 4)) return PFNG_B200_ERR_ALIGNMENT;
    for (int r = 0; r < world; ++r) {
        int64_t b = 0, e = 0;
        pfng_b200_shard_rows(n, world, r, granule, &b, &e);
        if (e - b > slice_width) return PFNG_B200_ERR_SHAPE;
    }
    DeviceInfo *info = nullptr;
    int st = device_info(&info);
    if (st != PFNG_B200_OK) return st;
    return status_of(launch_unshard_columns(slices, c, m, n, ldc, world, granule, slice_width,
                                            static_cast<cudaStream_t>(stream)));
}

}  // extern "C"

namespace {
// The destination checks of the gather entry points.
int check_destinations(float *const *dst, int ndst, int64_t m, int64_t n) {
    static_assert(PFNG_B200_MAX_DESTINATIONS == kMaxCopies + 1, "destination count");
    if (ndst < 1 || ndst > PFNG_B200_MAX_DESTINATIONS || !dst) return PFNG_B200_ERR_INVALID_ARGUMENT;
    if (m == 0 || n == 0) return PFNG_B200_OK;
    for (int d = 0; d < ndst; ++d) {
        if (!dst[d]) return PFNG_B200_ERR_INVALID_ARGUMENT;
        if (!aligned(dst[d], 4)) return PFNG_B200_ERR_ALIGNMENT;
    }
    return PFNG_B200_OK;
}
}  // namespace

extern "C" {

int pfng_b200_compute_gather(int wtype, const void *w, const float *x, int64_t ldx, float *const *dst, int ndst,
                             int64_t ldd, int64_t m, int64_t n, int64_t k, void *workspace, size_t workspace_bytes,
                             int path, void *stream) {
    const int st = check_destinations(dst, ndst, m, n);
    if (st != PFNG_B200_OK) return st;
    if (!x && m > 0 && n > 0 && k > 0) return PFNG_B200_ERR_INVALID_ARGUMENT;
    return run_matmul(wtype, w, nullptr, x, ldx, dst[0], ldd, nullptr, m, n, k, workspace, workspace_bytes, path,
                      static_cast<cudaStream_t>(stream), dst + 1, ndst - 1);
}

int pfng_b200_mm_gather(int wtype, const void *w, const void *a, float *const *dst, int ndst, int64_t ldd, int64_t m,
                        int64_t n, int64_t k, void *workspace, size_t workspace_bytes, int path, void *stream) {
    const int st = check_destinations(dst, ndst, m, n);
    if (st != PFNG_B200_OK) return st;
    if (!a && m > 0 && n > 0 && k > 0) return PFNG_B200_ERR_INVALID_ARGUMENT;
    return run_matmul(wtype, w, a, nullptr, 0, dst[0], ldd, nullptr, m, n, k, workspace, workspace_bytes, path,
                      static_cast<cudaStream_t>(stream), dst + 1, ndst - 1);
}

// Device buffers other processes can map: cudaMalloc'd (the unit CUDA IPC
// exports), so the handle maps the buffer from its first byte.
int pfng_b200_ipc_alloc(size_t bytes, void **ptr, void *handle) {
    if (!ptr || !handle || bytes == 0) return PFNG_B200_ERR_INVALID_ARGUMENT;
    static_assert(sizeof(cudaIpcMemHandle_t) == PFNG_B200_IPC_HANDLE_BYTES, "IPC handle size");
    *ptr = nullptr;
    void *p = nullptr;
    cudaError_t e = cudaMalloc(&p, bytes);
    if (e != cudaSuccess) return status_of(e);
    cudaIpcMemHandle_t h;
    e = cudaIpcGetMemHandle(&h, p);
    if (e != cudaSuccess) {
        cudaFree(p);
        return status_of(e);
    }
    std::memcpy(handle, &h, sizeof h);
    *ptr = p;
    return PFNG_B200_OK;
}

int pfng_b200_ipc_free(void *ptr) { return ptr ? status_of(cudaFree(ptr)) : PFNG_B200_OK; }

int pfng_b200_ipc_open(const void *handle, void **ptr) {
    if (!ptr || !handle) return PFNG_B200_ERR_INVALID_ARGUMENT;
    *ptr = nullptr;
    cudaIpcMemHandle_t h;
    std::memcpy(&h, handle, sizeof h);
    return status_of(cudaIpcOpenMemHandle(ptr, h, cudaIpcMemLazyEnablePeerAccess));
}

int pfng_b200_ipc_close(void *ptr) { return ptr ? status_of(cudaIpcCloseMemHandle(ptr)) : PFNG_B200_OK; }

}  // extern "C"
