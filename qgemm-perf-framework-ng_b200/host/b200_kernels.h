// b200_kernels.h -- registration functions of the B200 kernel adapters.
//
// The adapters implement the reference's plugin interface
// (pfng::bench::KernelCallbacks, bench/framework/kernel_registry.h:92-101) on
// top of the C ABI of include/pfng_b200.h, one kernel ID per quantization
// type.  A maintainer declares them next to the other adapters
// (kernels/common/adapter_common.h:76-96) and lists them in the kernel
// registration that cmake/Kernel.cmake generates.
#pragma once

#include <span>

#include "kernel_registry.h"

namespace pfng::bench::adapters {

// The three registrations, for a host that keeps its own table (register_kernel
// of the reference accepts only kernels of a known build platform).
std::span<const KernelRegistration> b200_kernel_registrations();

void register_q4_0_q8_0_b200();     // kernel ID "q4_0-q8_0-B200"
void register_q4_K_q8_K_b200();     // kernel ID "q4_K-q8_K-B200"
void register_iq2_xxs_q8_K_b200();  // kernel ID "iq2_xxs-q8_K-B200"
void register_b200_kernels();       // all three

}  // namespace pfng::bench::adapters
