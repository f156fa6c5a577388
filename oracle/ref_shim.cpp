// ref_shim.cpp -- extern "C" entry points over the reference's OWN sources.
//
// TEST INFRASTRUCTURE ONLY.  oracle/Makefile compiles this file together with
// the reference's bench/llama_reference/llama_reference.cpp and
// bench/framework/{benchmark,platform,kernel_registry}.cpp, read in place from
// the reference checkout, into oracle/_ref/libpfng_ref.so.  The library is
// the pin for the C restatement in pfng_oracle.c, the generator of the golden
// fixtures in tests/golden/, and the "reference" CPU arm of bench.py.
#include <cstdint>
#include <cstring>
#include <span>
#include <variant>
#include <vector>

#include "benchmark.h"
#include "iq2_xxs.h"
#include "llama_reference.h"

using namespace pfng::bench;

extern "C" {

float ref_fp16_to_fp32(uint16_t h) { return GGML_FP16_TO_FP32(h); }
uint16_t ref_fp32_to_fp16(float f) { return GGML_FP32_TO_FP16(f); }

void ref_fp32_to_fp16_array(const float *in, uint16_t *out, size_t count) {
    for (size_t i = 0; i < count; ++i) out[i] = GGML_FP32_TO_FP16(in[i]);
}

void ref_fp16_to_fp32_array(const uint16_t *in, float *out, size_t count) {
    for (size_t i = 0; i < count; ++i) out[i] = GGML_FP16_TO_FP32(in[i]);
}

void ref_quantize_q4_0(const float *x, void *y, size_t m, size_t k) {
    for (size_t r = 0; r < m; ++r)
        llama_reference::quantize_row_q4_0(x + r * k, static_cast<block_q4_0 *>(y) + r * (k / QK4_0), k);
}
void ref_quantize_q8_0(const float *x, void *y, size_t m, size_t k) {
    for (size_t r = 0; r < m; ++r)
        llama_reference::quantize_row_q8_0(x + r * k, static_cast<block_q8_0 *>(y) + r * (k / QK8_0), k);
}
void ref_quantize_q8_K(const float *x, void *y, size_t m, size_t k) {
    for (size_t r = 0; r < m; ++r)
        llama_reference::quantize_row_q8_K(x + r * k, static_cast<block_q8_K *>(y) + r * (k / QK_K), k);
}
void ref_quantize_q4_K(const float *x, void *y, size_t m, size_t k) {
    for (size_t r = 0; r < m; ++r)
        llama_reference::quantize_row_q4_K(x + r * k, static_cast<block_q4_K *>(y) + r * (k / QK_K), k);
}

float ref_dot_q4_0_q8_0(const void *w, const void *a, size_t nblocks) {
    return llama_reference::dot_q4_0_q8_0(std::span(static_cast<const block_q4_0 *>(w), nblocks),
                                          std::span(static_cast<const block_q8_0 *>(a), nblocks));
}
float ref_dot_q4_K_q8_K(const void *w, const void *a) {
    return llama_reference::dot_q4_K_q8_K(*static_cast<const block_q4_K *>(w), *static_cast<const block_q8_K *>(a));
}
float ref_dot_iq2_xxs_q8_K(const void *w, const void *a) {
    return llama_reference::dot_iq2_xxs_q8_K(*static_cast<const block_iq2_xxs *>(w),
                                             *static_cast<const block_q8_K *>(a));
}

void ref_iq2_decode_subblock(const uint8_t *packed, int8_t *values, int *scale) {
    int s = 0;
    iq2_xxs::decode_subblock(packed, values, s);
    *scale = s;
}

// The reference's full compute() (quantize activations, then dot products),
// bench/llama_reference/llama_reference.cpp:213.  type: 0 q4_0, 1 q4_K, 2 iq2_xxs.
int ref_compute(int type, const void *w, const float *x, float *c, size_t m, size_t n, size_t k) {
    std::span<const float> act(x, m * k);
    BenchmarkInput input;
    switch (type) {
    case 0: input = Q4_0Q8_0Input{m, n, k, act, std::span(static_cast<const block_q4_0 *>(w), n * (k / QK4_0))}; break;
    case 1: input = Q4_KQ8_KInput{m, n, k, act, std::span(static_cast<const block_q4_K *>(w), n * (k / QK_K))}; break;
    case 2: input = IQ2_XXSQ8_KInput{m, n, k, act, std::span(static_cast<const block_iq2_xxs *>(w), n * (k / QK_K))}; break;
    default: return -1;
    }
    const auto out = llama_reference::compute(static_cast<QuantizationType>(type), input);
    std::memcpy(c, out.data(), out.size() * sizeof(float));
    return 0;
}

// Element-parallel form of the same compute: every C element is the
// reference's own dot over the same blocks, in the same order as
// llama_reference.cpp:172-175 / :186-189 / :200-203, so the result is
// bit-identical to ref_compute; only the outer loop is spread over threads.
// `a` holds pre-quantized activations (ref_quantize_*).
int ref_mm_threads(int type, const void *w, const void *a, float *c, size_t m, size_t n, size_t k, size_t ldc,
                   int threads) {
    if (type < 0 || type > 2) return -1;
    const long long rows = static_cast<long long>(m) * static_cast<long long>(n);
#pragma omp parallel for schedule(static) num_threads(threads)
    for (long long e = 0; e < rows; ++e) {
        const size_t i = static_cast<size_t>(e) / n, j = static_cast<size_t>(e) % n;
        float value = 0.0f;
        if (type == 0) {
            const size_t nb = k / QK4_0;
            value = ref_dot_q4_0_q8_0(static_cast<const block_q4_0 *>(w) + j * nb,
                                      static_cast<const block_q8_0 *>(a) + i * nb, nb);
        } else {
            const size_t nb = k / QK_K;
            for (size_t b = 0; b < nb; ++b) {
                const auto *ab = static_cast<const block_q8_K *>(a) + i * nb + b;
                value += type == 1 ? ref_dot_q4_K_q8_K(static_cast<const block_q4_K *>(w) + j * nb + b, ab)
                                   : ref_dot_iq2_xxs_q8_K(static_cast<const block_iq2_xxs *>(w) + j * nb + b, ab);
            }
        }
        c[i * ldc + j] = value;
    }
    return 0;
}

// The reference's own seeded input generator, bench/framework/benchmark.cpp:34-94.
int ref_create_input(int type, size_t m, size_t n, size_t k, uint64_t seed, float *activation, void *weight) {
    BenchmarkRequest request;
    request.m = m;
    request.n = n;
    request.k = k;
    request.seed = seed;
    const auto owned = create_input(static_cast<QuantizationType>(type), request);
    std::visit(
        [&](const auto &o) {
            std::memcpy(activation, o.activation.data(), o.activation.size() * sizeof(float));
            std::memcpy(weight, o.weight.data(), o.weight.size() * sizeof(o.weight[0]));
        },
        owned);
    return 0;
}

size_t ref_sizeof_block(int type) {
    switch (type) {
    case 0: return sizeof(block_q4_0);
    case 1: return sizeof(block_q4_K);
    case 2: return sizeof(block_iq2_xxs);
    case 3: return sizeof(block_q8_0);
    case 4: return sizeof(block_q8_K);
    default: return 0;
    }
}

} // extern "C"
