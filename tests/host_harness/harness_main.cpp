// harness_main.cpp -- drives the B200 kernel adapters through the reference's
// own plugin interface, input generator and verification.  TEST HARNESS.
//
// The reference's CLI (bench/main.cpp) refuses to run on a host whose Device
// Tree is not one of its RISC-V boards (bench/framework/platform.cpp:85-99),
// register_kernel() aborts unless the build names one of those boards
// (bench/framework/kernel_registry.cpp:20-33) and run_benchmark() accepts only
// kernels of the build's board (bench/framework/benchmark.cpp:108-113); none of
// them knows a GPU platform.  This driver therefore takes the adapters'
// registrations directly and restates the verification stage of run_benchmark
// (benchmark.cpp:130-168): validate, prepare, reset, run(1), export_output,
// then compare element by element with llama_reference::compute on the same
// input, failing an element when both its absolute and relative error exceed
// 1e-3.  Inputs come from the reference's create_input (benchmark.cpp:102-104,
// generators :34-94) with the request's seed.  After a PASS it times `run`
// with a host clock like the reference does (run() synchronises its stream).
//
// Usage: pfng-bench-b200 --list
//        pfng-bench-b200 --kernel ID --m M --n N --k K [--iterations I] [--seed S]
// Exit status: 0 PASS, 1 FAIL, 2 usage, 4 SKIP (validate said unsupported).
#include <algorithm>
#include <chrono>
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <string>
#include <string_view>
#include <vector>

#include "b200_kernels.h"
#include "benchmark.h"
#include "kernel_registry.h"
#include "llama_reference.h"

using namespace pfng::bench;

namespace {

bool parse(const char *s, size_t &out) {
    char *end = nullptr;
    const unsigned long long v = std::strtoull(s, &end, 10);
    if (!end || *end || v == 0) return false;
    out = static_cast<size_t>(v);
    return true;
}

int usage(const char *argv0) {
    std::fprintf(stderr, "usage: %s --list | --kernel ID --m M --n N --k K [--iterations I] [--seed S]\n", argv0);
    return 2;
}

}  // namespace

const KernelRegistration *find_b200(std::string_view id) {
    for (const auto &k : adapters::b200_kernel_registrations())
        if (k.id == id) return &k;
    return nullptr;
}

int main(int argc, char **argv) {
    BenchmarkRequest request;
    request.seed = 1;
    size_t iterations = 10;
    std::string_view selected;
    bool list = false;
    for (int i = 1; i < argc; ++i) {
        const std::string_view a = argv[i];
        if (a == "--list") {
            list = true;
        } else if (a == "--kernel" && i + 1 < argc) {
            selected = argv[++i];
        } else if (a == "--m" && i + 1 < argc && parse(argv[++i], request.m)) {
        } else if (a == "--n" && i + 1 < argc && parse(argv[++i], request.n)) {
        } else if (a == "--k" && i + 1 < argc && parse(argv[++i], request.k)) {
        } else if (a == "--iterations" && i + 1 < argc && parse(argv[++i], iterations)) {
        } else if (a == "--seed" && i + 1 < argc) {
            size_t seed = 0;
            if (!parse(argv[++i], seed)) return usage(argv[0]);
            request.seed = seed;
        } else {
            return usage(argv[0]);
        }
    }
    if (list) {
        for (const auto &k : adapters::b200_kernel_registrations())
            std::printf("%.*s  %.*s\n", static_cast<int>(k.id.size()), k.id.data(), static_cast<int>(k.name.size()),
                        k.name.data());
        return 0;
    }
    const KernelRegistration *kernel = find_b200(selected);
    if (!kernel || !request.m || !request.n || !request.k) return usage(argv[0]);

    const auto validation = kernel->callbacks.validate(request);
    if (!validation.supported) {
        std::printf("status: SKIP (%s)\n", validation.reason.c_str());
        return 4;
    }
    const auto owner = create_input(kernel->quantization, request);
    const auto input = std::visit([](const auto &o) { return o.view(); }, owner);
    const auto prepared = kernel->callbacks.prepare(request, input);
    if (!prepared.state) {
        std::printf("status: FAIL (%s)\n", prepared.error.c_str());
        return 1;
    }
    struct Cleanup {
        const KernelRegistration *k;
        KernelState s;
        ~Cleanup() { k->callbacks.destroy(s); }
    } cleanup{kernel, prepared.state};

    kernel->callbacks.reset(prepared.state);
    kernel->callbacks.run(prepared.state, 1);
    std::vector<float> actual(request.m * request.n);
    const auto exported = kernel->callbacks.export_output(prepared.state, actual);
    if (!exported.success) {
        std::printf("status: FAIL (%s)\n", exported.error.c_str());
        return 1;
    }
    const auto expected = llama_reference::compute(kernel->quantization, input);
    float max_abs = 0.0f, max_rel = 0.0f;
    size_t errors = 0, first_bad = actual.size();
    for (size_t i = 0; i < actual.size(); ++i) {
        const float absolute = std::fabs(actual[i] - expected[i]);
        const float relative = absolute / std::max(std::fabs(expected[i]), 1.0e-6f);
        max_abs = std::max(max_abs, absolute);
        max_rel = std::max(max_rel, relative);
        if (absolute > 1.0e-3f && relative > 1.0e-3f) {
            if (first_bad == actual.size()) first_bad = i;
            ++errors;
        }
    }
    std::printf("[%.*s] m=%zu n=%zu k=%zu seed=%llu\n", static_cast<int>(kernel->id.size()), kernel->id.data(),
                request.m, request.n, request.k, static_cast<unsigned long long>(request.seed));
    std::printf("error elements: %zu/%zu\n", errors, actual.size());
    if (errors) {
        std::printf("status: FAIL (output differs from llama.cpp reference at index %zu: actual=%.9g expected=%.9g)\n",
                    first_bad, actual[first_bad], expected[first_bad]);
        return 1;
    }
    std::printf("verify: PASS, max_abs=%.6g, max_rel=%.6g\n", max_abs, max_rel);

    kernel->callbacks.reset(prepared.state);
    kernel->callbacks.run(prepared.state, 3);  // warm-up
    const auto t0 = std::chrono::steady_clock::now();
    kernel->callbacks.run(prepared.state, iterations);
    const auto t1 = std::chrono::steady_clock::now();
    const double us = std::chrono::duration<double, std::micro>(t1 - t0).count() / static_cast<double>(iterations);
    // run() latches failures; export_output reports them
    const auto after = kernel->callbacks.export_output(prepared.state, actual);
    if (!after.success) {
        std::printf("status: FAIL (%s)\n", after.error.c_str());
        return 1;
    }
    const double ops = 2.0 * request.m * request.n * request.k;
    std::printf("time: %.2f us per run (host clock, %zu iterations), %.1f Gop/s, checksum %.9g\n", us, iterations,
                ops / us / 1e3, kernel->callbacks.checksum(prepared.state));
    return 0;
}
