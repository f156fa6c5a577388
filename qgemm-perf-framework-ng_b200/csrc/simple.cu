// simple.cu -- one thread per output element, any k that is a multiple of
// the block size, any pointer alignment the block types allow.
//
// This path restates the reference's per-element loops operation for
// operation (llama_reference.cpp:113-161, summed as in :165-205), so its fp32
// results are bit-identical to the reference's scalar path.  It is the
// correctness path for shapes the tuned kernels do not take; it is still
// device code (there is no CPU fallback anywhere in the library).
#include "iq2xxs_grid_codes.h"
#include "pfng_common.cuh"
#include "pfng_internal.h"

namespace pfng {
namespace {

PFNG_DEV uint32_t ld_u8(const uint8_t *p) { return __ldg(p); }
PFNG_DEV uint32_t ld_u16(const uint8_t *p) { return __ldg(reinterpret_cast<const uint16_t *>(p)); }

// kPlanar: W in the planar row layout (block b's nibbles at 16 b of the row,
// its scale at 16 nb + 2 b); otherwise raw 18-byte blocks.
template <bool kPartials, bool kPlanar>
__global__ void simple_q4_0(SimpleArgs a) {
    const int64_t e = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (e >= a.m * a.n) return;
    const int64_t i = e / a.n, j = e % a.n, nb = a.k / 32;
    const uint8_t *W = static_cast<const uint8_t *>(a.w) + j * nb * kQ4_0Bytes;
    const uint8_t *A = static_cast<const uint8_t *>(a.a) + i * nb * kQ8_0Bytes;
    float sum = 0.0f;
    for (int64_t b = 0; b < nb; ++b) {
        const uint8_t *wq = kPlanar ? W + 16 * b : W + b * kQ4_0Bytes + 2;
        const uint8_t *wd = kPlanar ? W + 16 * nb + 2 * b : W + b * kQ4_0Bytes;
        const uint8_t *ab = A + b * kQ8_0Bytes;
        int32_t isum = 0;
        for (int t = 0; t < 16; ++t) {
            const int q = static_cast<int>(ld_u8(wq + t));
            isum += ((q & 15) - 8) * static_cast<int8_t>(ld_u8(ab + 2 + t));
            isum += ((q >> 4) - 8) * static_cast<int8_t>(ld_u8(ab + 18 + t));
        }
        if constexpr (kPartials) {
            a.partials[e * nb + b] = isum;
        } else {
            const float dw = f16_bits_to_f32(ld_u16(wd)), da = f16_bits_to_f32(ld_u16(ab));
            sum = __fadd_rn(sum, __fmul_rn(__fmul_rn(static_cast<float>(isum), dw), da));
        }
    }
    if constexpr (!kPartials) a.c[i * a.ldc + j] = sum;
}

template <bool kPartials>
__global__ void simple_q4_K(SimpleArgs a) {
    const int64_t e = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (e >= a.m * a.n) return;
    const int64_t i = e / a.n, j = e % a.n, nb = a.k / 256;
    const uint8_t *W = static_cast<const uint8_t *>(a.w) + j * nb * kQ4_KBytes;
    const uint8_t *A = static_cast<const uint8_t *>(a.a) + i * nb * kQ8_KBytes;
    float total = 0.0f;
    for (int64_t b = 0; b < nb; ++b) {
        const uint8_t *wb = W + b * kQ4_KBytes, *ab = A + b * kQ8_KBytes;
        uint32_t sc[12];
        for (int t = 0; t < 12; ++t) sc[t] = ld_u8(wb + 4 + t);
        int scales[8], mins[8];
        for (int t = 0; t < 4; ++t) {
            scales[t] = sc[t] & 63;
            scales[t + 4] = (sc[t + 8] & 15) | ((sc[t] >> 6) << 4);
            mins[t] = sc[t + 4] & 63;
            mins[t + 4] = (sc[t + 8] >> 4) | ((sc[t + 4] >> 6) << 4);
        }
        const float d = f16_bits_to_f32(ld_u16(wb)), dmin = f16_bits_to_f32(ld_u16(wb + 2));
        float sum = 0.0f;
        for (int sb = 0; sb < 8; ++sb) {
            int32_t isum = 0;
            for (int t = 0; t < 32; ++t) {
                const uint32_t packed = ld_u8(wb + 16 + (sb / 2) * 32 + t);
                const int q = (sb % 2 == 0) ? static_cast<int>(packed & 15) : static_cast<int>(packed >> 4);
                const int av = static_cast<int8_t>(ld_u8(ab + kQ8_KQsOffset + sb * 32 + t));
                if constexpr (kPartials) {
                    isum += av * q;
                } else {
                    // llama_reference.cpp:129: a * (d * scale * q - dmin * min)
                    const float wv = __fsub_rn(__fmul_rn(__fmul_rn(d, static_cast<float>(scales[sb])), static_cast<float>(q)),
                                               __fmul_rn(dmin, static_cast<float>(mins[sb])));
                    sum = __fadd_rn(sum, __fmul_rn(static_cast<float>(av), wv));
                }
            }
            if constexpr (kPartials) a.partials[(e * nb + b) * 8 + sb] = isum;
        }
        if constexpr (!kPartials) {
            const float ad = __ldg(reinterpret_cast<const float *>(ab));
            total = __fadd_rn(total, __fmul_rn(ad, sum));
        }
    }
    if constexpr (!kPartials) a.c[i * a.ldc + j] = total;
}

template <bool kPartials>
__global__ void simple_iq2_xxs(SimpleArgs a) {
    const int64_t e = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (e >= a.m * a.n) return;
    const int64_t i = e / a.n, j = e % a.n, nb = a.k / 256;
    const uint8_t *W = static_cast<const uint8_t *>(a.w) + j * nb * kIQ2Bytes;
    const uint8_t *A = static_cast<const uint8_t *>(a.a) + i * nb * kQ8_KBytes;
    float total = 0.0f;
    for (int64_t b = 0; b < nb; ++b) {
        const uint8_t *wb = W + b * kIQ2Bytes, *ab = A + b * kQ8_KBytes;
        int32_t sum = 0;
        for (int sb = 0; sb < 8; ++sb) {
            const uint8_t *g8 = wb + 2 + 8 * sb;
            const uint32_t ss = ld_u16(g8 + 4) | (ld_u16(g8 + 6) << 16);
            int32_t sub = 0;
            for (int g = 0; g < 4; ++g) {
                const uint32_t code = pfng_iq2xxs_grid_codes[ld_u8(g8 + g)];
                const uint32_t sgn = iq2_sign_mask((ss >> (7 * g)) & 0x7fu);
                for (int l = 0; l < 8; ++l) {
                    const uint32_t c = (code >> (2 * l)) & 3u;
                    const int mag = static_cast<int>(8u + 17u * c + (c >> 1));
                    const int v = (sgn >> l) & 1u ? -mag : mag;
                    sub += v * static_cast<int8_t>(ld_u8(ab + kQ8_KQsOffset + sb * 32 + g * 8 + l));
                }
            }
            if constexpr (kPartials) a.partials[(e * nb + b) * 8 + sb] = sub;
            sum += (2 * static_cast<int>(ss >> 28) + 1) * sub;
        }
        if constexpr (!kPartials) {
            const float d = f16_bits_to_f32(ld_u16(wb)), ad = __ldg(reinterpret_cast<const float *>(ab));
            // llama_reference.cpp:160: 0.125f * d * a.d * sum
            total = __fadd_rn(total, __fmul_rn(__fmul_rn(__fmul_rn(0.125f, d), ad), static_cast<float>(sum)));
        }
    }
    if constexpr (!kPartials) a.c[i * a.ldc + j] = total;
}

}  // namespace

cudaError_t launch_simple(const SimpleArgs &args, cudaStream_t s) {
    const int64_t total = args.m * args.n;
    const int threads = 128;
    const int64_t blocks = (total + threads - 1) / threads;
    if (blocks > 0x7fffffff) return cudaErrorInvalidValue;
    const bool part = args.partials != nullptr;
    switch (args.wtype) {
    case kWQ4_0:
        if (part) simple_q4_0<true, false><<<blocks, threads, 0, s>>>(args);
        else simple_q4_0<false, false><<<blocks, threads, 0, s>>>(args);
        break;
    case kWQ4_0P:
        if (part) simple_q4_0<true, true><<<blocks, threads, 0, s>>>(args);
        else simple_q4_0<false, true><<<blocks, threads, 0, s>>>(args);
        break;
    case kWQ4_K:
        if (part) simple_q4_K<true><<<blocks, threads, 0, s>>>(args);
        else simple_q4_K<false><<<blocks, threads, 0, s>>>(args);
        break;
    default:
        if (part) simple_iq2_xxs<true><<<blocks, threads, 0, s>>>(args);
        else simple_iq2_xxs<false><<<blocks, threads, 0, s>>>(args);
        break;
    }
    return cudaGetLastError();
}

}  // namespace pfng
