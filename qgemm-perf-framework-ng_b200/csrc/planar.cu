// planar.cu -- q4_0 weights between the ggml layout and the planar row layout.
//
// Planar row layout (weight type PFNG_B200_Q4_0_PLANAR): a row of nb = k / 32
// blocks holds the 16-byte nibble fields of blocks 0..nb-1 (block j at byte
// 16 j), then their fp16 scales (block j at byte 16 nb + 2 j).  It has the
// same 18 nb bytes and the same row stride as the ggml layout, only
// reordered: with k % 256 == 0 every row, and so every nibble field, starts
// 16-byte aligned and loads with one 16-byte read, and a tile of consecutive
// rows is still one contiguous byte range.  The reference's adapters repack W
// once in `prepare` the same way (kernels/common/types.h:9-63,
// kernels/q4_0-q8_0-IME-m8b/implementations/smt-ime2/adapter.cpp:95-112);
// this is the B200 form of that step, run on the device.
//
// Both directions are byte permutations: unpack(pack(W)) == W for every W.
#include "pfng_common.cuh"
#include "pfng_internal.h"

namespace pfng {
namespace {

constexpr int kThreads = 256;

// One thread per block.  A raw block is 18 bytes at 18 b of its row
// (2-byte aligned): the fp16 scale, then the 16 nibble bytes.
template <bool kToPlanar>
__global__ void __launch_bounds__(kThreads)
    q4_0_planar_kernel(const uint8_t *__restrict__ src, uint8_t *__restrict__ dst, int64_t n, int64_t nb) {
    const int64_t e = static_cast<int64_t>(blockIdx.x) * kThreads + threadIdx.x;
    if (e >= n * nb) return;
    const int64_t row = e / nb, b = e % nb;
    const int64_t rb = nb * kQ4_0Bytes;
    if constexpr (kToPlanar) {
        const uint16_t *blk = reinterpret_cast<const uint16_t *>(src + row * rb + b * kQ4_0Bytes);
        uint32_t w[4];
#pragma unroll
        for (int i = 0; i < 4; ++i)
            w[i] = static_cast<uint32_t>(__ldg(blk + 1 + 2 * i)) | (static_cast<uint32_t>(__ldg(blk + 2 + 2 * i)) << 16);
        uint8_t *out = dst + row * rb;
        *reinterpret_cast<uint4 *>(out + 16 * b) = make_uint4(w[0], w[1], w[2], w[3]);
        *reinterpret_cast<uint16_t *>(out + 16 * nb + 2 * b) = __ldg(blk);
    } else {
        const uint8_t *in = src + row * rb;
        const uint4 v = __ldg(reinterpret_cast<const uint4 *>(in + 16 * b));
        const uint16_t d = __ldg(reinterpret_cast<const uint16_t *>(in + 16 * nb + 2 * b));
        uint16_t *blk = reinterpret_cast<uint16_t *>(dst + row * rb + b * kQ4_0Bytes);
        const uint32_t w[4] = {v.x, v.y, v.z, v.w};
        blk[0] = d;
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            blk[1 + 2 * i] = static_cast<uint16_t>(w[i] & 0xffffu);
            blk[2 + 2 * i] = static_cast<uint16_t>(w[i] >> 16);
        }
    }
}

cudaError_t launch(bool to_planar, const void *src, void *dst, int64_t n, int64_t k, cudaStream_t s) {
    const int64_t nb = k / 32;
    const int64_t blocks = (n * nb + kThreads - 1) / kThreads;
    if (blocks > 0x7fffffff) return cudaErrorInvalidValue;
    const uint8_t *in = static_cast<const uint8_t *>(src);
    uint8_t *out = static_cast<uint8_t *>(dst);
    if (to_planar)
        q4_0_planar_kernel<true><<<static_cast<unsigned>(blocks), kThreads, 0, s>>>(in, out, n, nb);
    else
        q4_0_planar_kernel<false><<<static_cast<unsigned>(blocks), kThreads, 0, s>>>(in, out, n, nb);
    return cudaGetLastError();
}

}  // namespace

cudaError_t launch_pack_q4_0_planar(const void *w, void *w_planar, int64_t n, int64_t k, cudaStream_t s) {
    return launch(true, w, w_planar, n, k, s);
}

cudaError_t launch_unpack_q4_0_planar(const void *w_planar, void *w, int64_t n, int64_t k, cudaStream_t s) {
    return launch(false, w_planar, w, n, k, s);
}

}  // namespace pfng
