// ref_shim_ksigns.cpp -- exposes ggml's ksigns_iq2xs table as held by the
// reference (kernels/iq2_xxs-q8_K-RVV-common/ggml_min.h:58).
// TEST INFRASTRUCTURE ONLY (oracle/_ref).
#include <cstdint>

#include "ggml_min.h"

extern "C" {
uint8_t ref_ksigns_iq2xs(unsigned index) { return ksigns_iq2xs[index & 127u]; }
}
