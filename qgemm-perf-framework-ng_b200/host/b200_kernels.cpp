// b200_kernels.cpp -- the reference's kernel adapter interface implemented
// for the B200 library.
//
// Each adapter is what bench/framework expects of a kernel
// (KernelCallbacks, bench/framework/kernel_registry.h:92-101; registry
// contract bench/framework/kernel_registry.cpp:20-33), following the
// reference adapters' conventions (e.g. kernels/q4_0-q8_0-RVV-upstream/
// implementations/rvv/adapter.cpp):
//   * validate  -- shape rules of the block format and a B200 (sm_100) device;
//                  an unsupported request is a SKIP with a reason;
//   * prepare   -- uploads W (raw ggml blocks) and the fp32 activations once,
//                  quantizes the activations on the device (untimed, as the
//                  reference adapters quantize in prepare), allocates C and
//                  the workspace; a failure is a FAIL with the status text;
//   * run       -- `iterations` matmuls through pfng_b200_mm_* on the
//                  adapter's stream, then a stream synchronisation (the
//                  reference times run() with host counters);
//   * reset     -- zeroes C;
//   * export_output / checksum -- copy C to the host; run() has no error
//                  channel, so its first failing status is latched and
//                  reported by export_output; checksum sums every 257th
//                  element like the reference's checksum_common
//                  (kernels/common/adapter_common.cpp:18-23);
//   * destroy   -- frees everything.
// run_benchmark divides MACs by the HOST cycles of the timed run() (perf
// "cycles", user space) and reports the quotient against the peak returned
// here, so the peak is expressed per host cycle: the GPU's dense int8 MAC
// rate (nominal 4.5 Pop/s for B200, or PFNG_B200_PEAK_INT8_TOPS) divided by
// the host's clock (cpu MHz of /proc/cpuinfo).  The utilisation it prints is
// then the fraction of the GPU's int8 rate the timed run achieved,
// host-side launch and synchronisation included.
#include "b200_kernels.h"

#include <cuda_runtime.h>

#include <cstdint>
#include <cstring>
#include <string>
#include <variant>
#include <vector>

#include "kernel_registry.h"
#include "pfng_b200.h"

#include <cstdio>
#include <cstdlib>

#ifndef PFNG_B200_PLATFORM
// PlatformId::NvidiaB200 is the value the platform overlay adds to the
// reference's bench/framework/platform.h:11-16 (integration/build_pfng_bench.py).
#define PFNG_B200_PLATFORM pfng::bench::PlatformId::NvidiaB200
#endif

namespace pfng::bench::adapters {
namespace {

constexpr double kNominalInt8Tops = 4500.0;  // B200 dense int8 (4.5 Pop/s, the 2:4-sparse figure halved)

struct State {
    int wtype = 0;
    size_t m = 0, n = 0, k = 0;
    void *w = nullptr;        // device W blocks
    void *a = nullptr;        // device activation q8 blocks
    float *c = nullptr;       // device C [m][n]
    void *ws = nullptr;       // device workspace
    size_t ws_bytes = 0;
    cudaStream_t stream = nullptr;
    int status = PFNG_B200_OK;  // first failure of run()
    std::vector<float> host_c;
};

std::string describe(int status) { return std::string("pfng_b200: ") + pfng_b200_status_string(status); }
std::string describe(cudaError_t e) { return std::string("cuda: ") + cudaGetErrorString(e); }

size_t block_k(int wtype) { return wtype == PFNG_B200_Q4_0 ? 32 : 256; }
size_t weight_block_bytes(int wtype) {
    return wtype == PFNG_B200_Q4_0 ? 18 : wtype == PFNG_B200_Q4_K ? 144 : 66;
}
size_t act_block_bytes(int wtype) { return wtype == PFNG_B200_Q4_0 ? 34 : 292; }

bool b200_present(std::string &reason) {
    int count = 0;
    if (cudaGetDeviceCount(&count) != cudaSuccess || count == 0) {
        cudaGetLastError();
        reason = "no CUDA device";
        return false;
    }
    int dev = 0, major = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev);
    if (major != 10) {
        reason = "device is not a B200 (sm_100)";
        return false;
    }
    return true;
}

// Device bytes prepare() allocates for a request (W, activations, C, fp32
// staging of the activations, workspace).
template <int WT>
size_t device_bytes(const BenchmarkRequest &r) {
    const size_t w = r.n * (r.k / block_k(WT)) * weight_block_bytes(WT);
    const size_t a = r.m * (r.k / block_k(WT)) * act_block_bytes(WT);
    return w + a + r.m * r.n * sizeof(float) + r.m * r.k * sizeof(float) +
           pfng_b200_mm_workspace_size(WT, static_cast<int64_t>(r.m), static_cast<int64_t>(r.n),
                                       static_cast<int64_t>(r.k), PFNG_B200_PATH_AUTO);
}

template <int WT>
ValidationResult validate(const BenchmarkRequest &r) {
    if (r.m == 0 || r.n == 0 || r.k == 0) return {false, "m, n and k must be positive"};
    if (r.k % block_k(WT) != 0) return {false, "k must be a multiple of " + std::to_string(block_k(WT))};
    std::string reason;
    if (!b200_present(reason)) return {false, reason};
    size_t free_bytes = 0, total = 0;
    if (cudaMemGetInfo(&free_bytes, &total) != cudaSuccess) {
        cudaGetLastError();
        return {false, "cudaMemGetInfo failed"};
    }
    if (device_bytes<WT>(r) > free_bytes)
        return {false, "needs " + std::to_string(device_bytes<WT>(r) >> 20) + " MiB of device memory, " +
                           std::to_string(free_bytes >> 20) + " MiB free"};
    return {true, {}};
}

// Host clock in Hz from /proc/cpuinfo ("cpu MHz"), 0 if unknown.
double host_hz() {
    FILE *f = std::fopen("/proc/cpuinfo", "r");
    if (!f) return 0.0;
    char line[256];
    double mhz = 0.0;
    while (std::fgets(line, sizeof line, f)) {
        if (std::strncmp(line, "cpu MHz", 7) == 0) {
            const char *colon = std::strchr(line, ':');
            if (colon) mhz = std::atof(colon + 1);
            break;
        }
    }
    std::fclose(f);
    return mhz * 1e6;
}

PeakPerformance peak(const BenchmarkRequest &r) {
    const char *env = std::getenv("PFNG_B200_PEAK_INT8_TOPS");
    const double tops = env && std::atof(env) > 0 ? std::atof(env) : kNominalInt8Tops;
    const double hz = host_hz() > 0 ? host_hz() : 2.0e9;
    const double macs_per_host_cycle = tops * 1e12 / 2.0 / hz;
    return {static_cast<double>(r.m) * r.n * r.k, macs_per_host_cycle, "i8-i32 MAC"};
}

void free_state(State *s) {
    if (!s) return;
    cudaFree(s->w);
    cudaFree(s->a);
    cudaFree(s->c);
    cudaFree(s->ws);
    if (s->stream) cudaStreamDestroy(s->stream);
    delete s;
}

// The weight blocks and fp32 activations of one input variant.
template <int WT>
auto &input_of(const BenchmarkInput &input) {
    if constexpr (WT == PFNG_B200_Q4_0)
        return std::get<Q4_0Q8_0Input>(input);
    else if constexpr (WT == PFNG_B200_Q4_K)
        return std::get<Q4_KQ8_KInput>(input);
    else
        return std::get<IQ2_XXSQ8_KInput>(input);
}

template <int WT>
PrepareResult prepare(const BenchmarkRequest &r, const BenchmarkInput &generic) {
    const auto &in = input_of<WT>(generic);
    auto *s = new State;
    s->wtype = WT;
    s->m = r.m;
    s->n = r.n;
    s->k = r.k;
    s->host_c.assign(r.m * r.n, 0.0f);
    const size_t w_bytes = r.n * (r.k / block_k(WT)) * weight_block_bytes(WT);
    const size_t a_bytes = r.m * (r.k / block_k(WT)) * act_block_bytes(WT);
    float *x = nullptr;
    cudaError_t e = cudaStreamCreateWithFlags(&s->stream, cudaStreamNonBlocking);
    if (e == cudaSuccess) e = cudaMalloc(&s->w, w_bytes);
    if (e == cudaSuccess) e = cudaMalloc(&s->a, a_bytes);
    if (e == cudaSuccess) e = cudaMalloc(reinterpret_cast<void **>(&s->c), r.m * r.n * sizeof(float));
    if (e == cudaSuccess) e = cudaMalloc(reinterpret_cast<void **>(&x), r.m * r.k * sizeof(float));
    if (e == cudaSuccess) e = cudaMemcpy(s->w, in.weight.data(), w_bytes, cudaMemcpyHostToDevice);
    if (e == cudaSuccess) e = cudaMemcpy(x, in.activation.data(), r.m * r.k * sizeof(float), cudaMemcpyHostToDevice);
    if (e != cudaSuccess) {
        cudaFree(x);
        free_state(s);
        return {nullptr, describe(e)};
    }
    // activation quantization on the device (the reference adapters do it in prepare)
    int st = WT == PFNG_B200_Q4_0
                 ? pfng_b200_quantize_q8_0(x, static_cast<int64_t>(r.k), s->a, r.m, r.k, s->stream)
                 : pfng_b200_quantize_q8_K(x, static_cast<int64_t>(r.k), s->a, r.m, r.k, s->stream);
    if (st == PFNG_B200_OK) {
        s->ws_bytes = pfng_b200_mm_workspace_size(WT, r.m, r.n, r.k, PFNG_B200_PATH_AUTO);
        if (s->ws_bytes && (e = cudaMalloc(&s->ws, s->ws_bytes)) != cudaSuccess) st = PFNG_B200_ERR_CUDA_BASE - e;
    }
    if (st == PFNG_B200_OK) st = pfng_b200_check_kernel_error(s->stream);
    cudaFree(x);
    if (st != PFNG_B200_OK) {
        free_state(s);
        return {nullptr, describe(st)};
    }
    return {s, {}};
}

int mm_once(State &s) {
    const auto m = static_cast<int64_t>(s.m), n = static_cast<int64_t>(s.n), k = static_cast<int64_t>(s.k);
    switch (s.wtype) {
    case PFNG_B200_Q4_0:
        return pfng_b200_mm_q4_0_q8_0(s.w, s.a, s.c, m, n, k, n, s.ws, s.ws_bytes, PFNG_B200_PATH_AUTO, s.stream);
    case PFNG_B200_Q4_K:
        return pfng_b200_mm_q4_K_q8_K(s.w, s.a, s.c, m, n, k, n, s.ws, s.ws_bytes, PFNG_B200_PATH_AUTO, s.stream);
    default:
        return pfng_b200_mm_iq2_xxs_q8_K(s.w, s.a, s.c, m, n, k, n, s.ws, s.ws_bytes, PFNG_B200_PATH_AUTO,
                                         s.stream);
    }
}

void run(KernelState opaque, size_t iterations) noexcept {
    auto &s = *static_cast<State *>(opaque);
    for (size_t i = 0; i < iterations && s.status == PFNG_B200_OK; ++i) s.status = mm_once(s);
    const cudaError_t e = cudaStreamSynchronize(s.stream);
    if (s.status == PFNG_B200_OK && e != cudaSuccess) s.status = PFNG_B200_ERR_CUDA_BASE - e;
    if (s.status == PFNG_B200_OK) s.status = pfng_b200_check_kernel_error(s.stream);
}

void reset(KernelState opaque) {
    auto &s = *static_cast<State *>(opaque);
    const cudaError_t e = cudaMemsetAsync(s.c, 0, s.m * s.n * sizeof(float), s.stream);
    if (s.status == PFNG_B200_OK && e != cudaSuccess) s.status = PFNG_B200_ERR_CUDA_BASE - e;
    std::memset(s.host_c.data(), 0, s.host_c.size() * sizeof(float));
}

int copy_out(State &s) {
    if (s.status != PFNG_B200_OK) return s.status;
    const cudaError_t e = cudaMemcpyAsync(s.host_c.data(), s.c, s.host_c.size() * sizeof(float),
                                          cudaMemcpyDeviceToHost, s.stream);
    if (e != cudaSuccess) return PFNG_B200_ERR_CUDA_BASE - e;
    const cudaError_t e2 = cudaStreamSynchronize(s.stream);
    return e2 == cudaSuccess ? PFNG_B200_OK : PFNG_B200_ERR_CUDA_BASE - e2;
}

ExportResult export_output(KernelState opaque, std::span<float> out) {
    auto &s = *static_cast<State *>(opaque);
    if (out.size() != s.host_c.size()) return {false, "output span has the wrong size"};
    const int st = copy_out(s);
    if (st != PFNG_B200_OK) return {false, describe(st)};
    std::memcpy(out.data(), s.host_c.data(), out.size_bytes());
    return {true, {}};
}

double checksum(KernelState opaque) {
    auto &s = *static_cast<State *>(opaque);
    if (copy_out(s) != PFNG_B200_OK) return 0.0;
    double sum = 0.0;
    for (size_t i = 0; i < s.host_c.size(); i += 257) sum += s.host_c[i];
    return sum;
}

void destroy(KernelState opaque) noexcept { free_state(static_cast<State *>(opaque)); }

template <int WT>
KernelCallbacks callbacks() {
    return {peak, validate<WT>, prepare<WT>, reset, run, export_output, checksum, destroy};
}

const KernelRegistration kRegistrations[] = {
    {"q4_0-q8_0-B200", "q4_0 x q8_0 on B200 (GEMV m<=8, int8 tensor cores above)",
     QuantizationType::WeightQ4_0ActivationQ8_0, callbacks<PFNG_B200_Q4_0>(), PFNG_B200_PLATFORM},
    {"q4_K-q8_K-B200", "q4_K x q8_K on B200 (GEMV m<=8, int8 tensor cores above)",
     QuantizationType::WeightQ4_KActivationQ8_K, callbacks<PFNG_B200_Q4_K>(), PFNG_B200_PLATFORM},
    {"iq2_xxs-q8_K-B200", "iq2_xxs x q8_K on B200 (GEMV m<=8, int8 tensor cores above)",
     QuantizationType::WeightIQ2_XXSActivationQ8_K, callbacks<PFNG_B200_IQ2_XXS>(), PFNG_B200_PLATFORM},
};

}  // namespace

std::span<const KernelRegistration> b200_kernel_registrations() { return kRegistrations; }

void register_q4_0_q8_0_b200() { register_kernel(kRegistrations[0]); }
void register_q4_K_q8_K_b200() { register_kernel(kRegistrations[1]); }
void register_iq2_xxs_q8_K_b200() { register_kernel(kRegistrations[2]); }

void register_b200_kernels() {
    register_q4_0_q8_0_b200();
    register_q4_K_q8_K_b200();
    register_iq2_xxs_q8_K_b200();
}

}  // namespace pfng::bench::adapters
