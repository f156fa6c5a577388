// quantize.cu -- fp32 -> ggml block quantizers on sm_100a.
//
// Bit-exactness with the reference's scalar quantizers
// (bench/llama_reference/llama_reference.cpp:13-111) rests on doing the same
// IEEE fp32 operations in the same order: every multiply, add and divide is
// an explicit round-to-nearest intrinsic (no contraction into FMA, no
// approximate division), rounding to integers uses roundf (half away from
// zero, like std::round) or truncation where the reference casts, and the
// fp16 scale uses round-to-nearest-even.  Reductions (max, min, sums) are
// order-independent except for ties, which are broken toward the lowest
// index exactly as the reference's sequential loops do.
#include <cuda_bf16.h>

#include "pfng_common.cuh"
#include "pfng_internal.h"
#include "pfng_quant.cuh"

namespace pfng {
namespace {

constexpr int kThreads = 256;

template <bool kVec>
PFNG_DEV void load4(const float *p, float v[4]) {
    if constexpr (kVec) {
        const float4 t = __ldg(reinterpret_cast<const float4 *>(p));
        v[0] = t.x, v[1] = t.y, v[2] = t.z, v[3] = t.w;
    } else {
#pragma unroll
        for (int i = 0; i < 4; ++i) v[i] = __ldg(p + i);
    }
}

template <bool kVec, bool kSplit>
__global__ void __launch_bounds__(kThreads) quantize_q8_0_kernel(const float *__restrict__ x, int64_t ldx,
                                                                  uint8_t *__restrict__ y, int64_t ldy, SplitA split,
                                                                  int64_t m, int64_t k, int64_t rows) {
    // the GEMM that reads this operand may start now and fetch its weights;
    // it waits for this grid's completion before reading the operand
    if (threadIdx.x == 0) pdl_trigger();
    const int64_t nb = k / 32;
    const int64_t total = rows * nb;
    const int g = threadIdx.x & 7;
    const int64_t warp0 = (static_cast<int64_t>(blockIdx.x) * kThreads + threadIdx.x) >> 5;
    const int64_t wstride = (static_cast<int64_t>(gridDim.x) * kThreads) >> 5;
    // A warp covers 4 consecutive blocks (8 lanes each) and all its lanes run
    // the same trip count, so the group shuffles are warp-uniform; a group
    // past the end works on zeros and stores nothing.
    for (int64_t wb = warp0 * 4; wb < total; wb += wstride * 4) {
        const int64_t bi = wb + ((threadIdx.x >> 3) & 3);
        const bool live = bi < total;
        const int64_t row = live ? bi / nb : 0, col = live ? bi % nb : 0;
        float v[4] = {0.0f, 0.0f, 0.0f, 0.0f};
        if (live && row < m) load4<kVec>(x + row * ldx + col * 32 + 4 * g, v);
        const Q8_0Lane r = q8_0_quantize_lane(v);
        if (!live) continue;
        if constexpr (kSplit) {
            *reinterpret_cast<uint32_t *>(split.qs + row * k + col * 32 + 4 * g) = r.q;
            if (g == 0) {
                split.d[split_d_index(row, col, split.d_ld)] = f16_bits_to_f32(r.dbits);
                split.aux[row * nb + col] = 0x4B400000 - 8 * r.qsum;
            }
        } else {
            uint8_t *blk = y + (row * ldy + col) * kQ8_0Bytes;
            uint16_t *h = reinterpret_cast<uint16_t *>(blk + 2 + 4 * g);
            h[0] = static_cast<uint16_t>(r.q & 0xffffu);
            h[1] = static_cast<uint16_t>(r.q >> 16);
            if (g == 0) *reinterpret_cast<uint16_t *>(blk) = r.dbits;
        }
    }
}

// ---------------------------------------------------------------------------
// q8_K: one warp per 256-value block, lane l holds values 8l..8l+7.
// llama_reference.cpp:54-70.
// ---------------------------------------------------------------------------
template <bool kVec, bool kSplit>
__global__ void __launch_bounds__(kThreads) quantize_q8_K_kernel(const float *__restrict__ x, int64_t ldx,
                                                                  uint8_t *__restrict__ y, SplitA split,
                                                                  int64_t m, int64_t k, int64_t rows) {
    // the GEMM that reads this operand may start now and fetch its weights;
    // it waits for this grid's completion before reading the operand
    if (threadIdx.x == 0) pdl_trigger();
    const int64_t nb = k / 256;
    const int64_t total = rows * nb;
    const int lane = threadIdx.x & 31;
    const int64_t warp0 = (static_cast<int64_t>(blockIdx.x) * kThreads + threadIdx.x) >> 5;
    const int64_t stride = (static_cast<int64_t>(gridDim.x) * kThreads) >> 5;
    for (int64_t bi = warp0; bi < total; bi += stride) {
        const int64_t row = bi / nb, col = bi % nb;
        float v[8] = {0, 0, 0, 0, 0, 0, 0, 0};
        if (row < m) {
            const float *p = x + row * ldx + col * 256 + 8 * lane;
            load4<kVec>(p, v);
            load4<kVec>(p + 4, v + 4);
        }
        const Q8_KLane r = q8_K_quantize_lane(v);
        const uint32_t q0 = r.q0, q1 = r.q1;
        const int s16 = r.sum16, s32 = r.sum32;
        const float d = r.d;
        if constexpr (kSplit) {
            uint32_t *q = reinterpret_cast<uint32_t *>(split.qs + row * k + col * 256 + 8 * lane);
            q[0] = q0;
            q[1] = q1;
            if ((lane & 3) == 0) split.aux[row * (k / 32) + col * 8 + (lane >> 2)] = s32;
            if (lane == 0) split.d[row * nb + col] = d;
        } else {
            uint8_t *blk = y + bi * kQ8_KBytes;
            uint32_t *q = reinterpret_cast<uint32_t *>(blk + kQ8_KQsOffset + 8 * lane);
            q[0] = q0;
            q[1] = q1;
            if ((lane & 1) == 0)
                reinterpret_cast<int16_t *>(blk + kQ8_KBsumsOffset)[lane >> 1] = static_cast<int16_t>(s16);
            if (lane == 0) *reinterpret_cast<float *>(blk) = d;
        }
    }
}

// ---------------------------------------------------------------------------
// raw q8 blocks -> split operand
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(kThreads) convert_q8_0_split_kernel(const uint8_t *__restrict__ a, SplitA split,
                                                                       int64_t m, int64_t k, int64_t rows) {
    // the GEMM that reads this operand may start now and fetch its weights;
    // it waits for this grid's completion before reading the operand
    if (threadIdx.x == 0) pdl_trigger();
    const int64_t nb = k / 32;
    const int64_t total = rows * nb;
    const int g = threadIdx.x & 7;
    const int64_t warp0 = (static_cast<int64_t>(blockIdx.x) * kThreads + threadIdx.x) >> 5;
    const int64_t wstride = (static_cast<int64_t>(gridDim.x) * kThreads) >> 5;
    for (int64_t wb = warp0 * 4; wb < total; wb += wstride * 4) {
        const int64_t bi = wb + ((threadIdx.x >> 3) & 3);
        const bool live = bi < total;
        const int64_t row = live ? bi / nb : 0, col = live ? bi % nb : 0;
        uint32_t q = 0;
        uint32_t dbits = 0;
        if (live && row < m) {
            const uint8_t *blk = a + (row * nb + col) * kQ8_0Bytes;
            const uint16_t *h = reinterpret_cast<const uint16_t *>(blk + 2 + 4 * g);
            q = static_cast<uint32_t>(__ldg(h)) | (static_cast<uint32_t>(__ldg(h + 1)) << 16);
            dbits = __ldg(reinterpret_cast<const uint16_t *>(blk));
        }
        int s = __dp4a(static_cast<int>(q), 0x01010101, 0);
#pragma unroll
        for (int o = 1; o < 8; o <<= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
        if (!live) continue;
        *reinterpret_cast<uint32_t *>(split.qs + row * k + col * 32 + 4 * g) = q;
        if (g == 0) {
            split.d[split_d_index(row, col, split.d_ld)] = f16_bits_to_f32(dbits);
            split.aux[row * nb + col] = 0x4B400000 - 8 * s;
        }
    }
}

__global__ void __launch_bounds__(kThreads) convert_q8_K_split_kernel(const uint8_t *__restrict__ a, SplitA split,
                                                                       int64_t m, int64_t k, int64_t rows) {
    // the GEMM that reads this operand may start now and fetch its weights;
    // it waits for this grid's completion before reading the operand
    if (threadIdx.x == 0) pdl_trigger();
    const int64_t nb = k / 256;
    const int64_t total = rows * nb;
    const int lane = threadIdx.x & 31;
    const int64_t warp0 = (static_cast<int64_t>(blockIdx.x) * kThreads + threadIdx.x) >> 5;
    const int64_t stride = (static_cast<int64_t>(gridDim.x) * kThreads) >> 5;
    for (int64_t bi = warp0; bi < total; bi += stride) {
        const int64_t row = bi / nb, col = bi % nb;
        uint32_t q0 = 0, q1 = 0;
        float d = 0.0f;
        if (row < m) {
            const uint8_t *blk = a + (row * nb + col) * kQ8_KBytes;
            const uint32_t *q = reinterpret_cast<const uint32_t *>(blk + kQ8_KQsOffset + 8 * lane);
            q0 = __ldg(q);
            q1 = __ldg(q + 1);
            d = __ldg(reinterpret_cast<const float *>(blk));
        }
        int s = __dp4a(static_cast<int>(q0), 0x01010101, __dp4a(static_cast<int>(q1), 0x01010101, 0));
        s += __shfl_xor_sync(0xffffffffu, s, 1);
        s += __shfl_xor_sync(0xffffffffu, s, 2);
        uint32_t *dst = reinterpret_cast<uint32_t *>(split.qs + row * k + col * 256 + 8 * lane);
        dst[0] = q0;
        dst[1] = q1;
        if ((lane & 3) == 0) split.aux[row * (k / 32) + col * 8 + (lane >> 2)] = s;
        if (lane == 0) split.d[row * nb + col] = d;
    }
}

// ---------------------------------------------------------------------------
// q4_0 weights: 8 lanes per block.  llama_reference.cpp:13-36.
// The signed maximum is the first value (lowest index) of largest magnitude.
// ---------------------------------------------------------------------------
template <bool kVec>
__global__ void __launch_bounds__(kThreads) quantize_q4_0_kernel(const float *__restrict__ x, int64_t ldx,
                                                                  uint8_t *__restrict__ y, int64_t n, int64_t k) {
    const int64_t nb = k / 32;
    const int64_t total = n * nb;
    const int g = threadIdx.x & 7;
    const int64_t warp0 = (static_cast<int64_t>(blockIdx.x) * kThreads + threadIdx.x) >> 5;
    const int64_t wstride = (static_cast<int64_t>(gridDim.x) * kThreads) >> 5;
    for (int64_t wb = warp0 * 4; wb < total; wb += wstride * 4) {
        const int64_t bi = wb + ((threadIdx.x >> 3) & 3);
        const bool live = bi < total;
        const int64_t row = live ? bi / nb : 0, col = live ? bi % nb : 0;
        float v[4] = {0.0f, 0.0f, 0.0f, 0.0f};
        if (live) load4<kVec>(x + row * ldx + col * 32 + 4 * g, v);
        // lane-local first maximum
        float amax = 0.0f, smax = 0.0f;
        int idx = 1 << 30;
#pragma unroll
        for (int i = 0; i < 4; ++i)
            if (amax < fabsf(v[i])) amax = fabsf(v[i]), smax = v[i], idx = 4 * g + i;
#pragma unroll
        for (int o = 1; o < 8; o <<= 1) {
            const float oa = __shfl_xor_sync(0xffffffffu, amax, o);
            const float os = __shfl_xor_sync(0xffffffffu, smax, o);
            const int oi = __shfl_xor_sync(0xffffffffu, idx, o);
            if (oa > amax || (oa == amax && oi < idx)) amax = oa, smax = os, idx = oi;
        }
        const float scale = __fdiv_rn(smax, -8.0f);
        const float inv = scale != 0.0f ? __fdiv_rn(1.0f, scale) : 0.0f;
        uint32_t q = 0;
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            int qi = __float2int_rz(__fadd_rn(__fmul_rn(v[i], inv), 8.5f));
            qi = static_cast<int>(static_cast<int8_t>(qi));
            qi = qi < 15 ? qi : 15;
            q |= (static_cast<uint32_t>(qi) & 0xffu) << (8 * i);
        }
        // lanes 0-3 hold the low nibbles of qs[0..15], lanes 4-7 the high ones
        const uint32_t hi = __shfl_down_sync(0xffffffffu, q, 4);
        if (live && g < 4) {
            const uint32_t packed = (q & 0x0f0f0f0fu) | ((hi & 0x0f0f0f0fu) << 4);
            uint8_t *blk = y + bi * kQ4_0Bytes;
            uint16_t *h = reinterpret_cast<uint16_t *>(blk + 2 + 4 * g);
            h[0] = static_cast<uint16_t>(packed & 0xffffu);
            h[1] = static_cast<uint16_t>(packed >> 16);
            if (g == 0) *reinterpret_cast<uint16_t *>(blk) = f32_to_f16_bits(scale);
        }
    }
}

// ---------------------------------------------------------------------------
// q4_K weights: one warp per 256-value block, lane l holds values 8l..8l+7 of
// sub-block l / 4.  llama_reference.cpp:72-111.
// ---------------------------------------------------------------------------
template <bool kVec>
__global__ void __launch_bounds__(kThreads) quantize_q4_K_kernel(const float *__restrict__ x, int64_t ldx,
                                                                  uint8_t *__restrict__ y, int64_t n, int64_t k) {
    const int64_t nb = k / 256;
    const int64_t total = n * nb;
    const int lane = threadIdx.x & 31;
    const int64_t warp0 = (static_cast<int64_t>(blockIdx.x) * kThreads + threadIdx.x) >> 5;
    const int64_t stride = (static_cast<int64_t>(gridDim.x) * kThreads) >> 5;
    for (int64_t bi = warp0; bi < total; bi += stride) {
        const int64_t row = bi / nb, col = bi % nb;
        float v[8];
        const float *p = x + row * ldx + col * 256 + 8 * lane;
        load4<kVec>(p, v);
        load4<kVec>(p + 4, v + 4);
        // sub-block min / max with the reference's sequential semantics:
        // the first occurrence wins among equal values.
        float lo = v[0], hi = v[0];
        int ilo = 8 * lane, ihi = 8 * lane;
#pragma unroll
        for (int i = 1; i < 8; ++i) {
            if (v[i] < lo) lo = v[i], ilo = 8 * lane + i;
            if (hi < v[i]) hi = v[i], ihi = 8 * lane + i;
        }
#pragma unroll
        for (int o = 1; o < 4; o <<= 1) {
            const float olo = __shfl_xor_sync(0xffffffffu, lo, o), ohi = __shfl_xor_sync(0xffffffffu, hi, o);
            const int oilo = __shfl_xor_sync(0xffffffffu, ilo, o), oihi = __shfl_xor_sync(0xffffffffu, ihi, o);
            if (olo < lo || (olo == lo && oilo < ilo)) lo = olo, ilo = oilo;
            if (hi < ohi || (ohi == hi && oihi < ihi)) hi = ohi, ihi = oihi;
        }
        const float my_ls = __fdiv_rn(__fsub_rn(hi, lo), 15.0f);
        const float my_lm = __fdiv_rn(-lo, my_ls != 0.0f ? my_ls : 1.0f);
        // every lane replays the reference's sequential max over the 8 sub-blocks
        float ls[8], lm[8], maxs = 0.0f, maxm = 0.0f;
#pragma unroll
        for (int sb = 0; sb < 8; ++sb) {
            ls[sb] = __shfl_sync(0xffffffffu, my_ls, 4 * sb);
            lm[sb] = __shfl_sync(0xffffffffu, my_lm, 4 * sb);
            maxs = maxs < ls[sb] ? ls[sb] : maxs;
            maxm = maxm < lm[sb] ? lm[sb] : maxm;
        }
        const float ds = __fdiv_rn(maxs, 63.0f), dm = __fdiv_rn(maxm, 63.0f);
        uint8_t *blk = y + bi * kQ4_KBytes;
        if (lane < 12) {
            uint32_t s[8], mm[8];
#pragma unroll
            for (int i = 0; i < 8; ++i) {
                const int si = static_cast<int>(roundf(__fdiv_rn(ls[i], ds != 0.0f ? ds : 1.0f)));
                const int mi = static_cast<int>(roundf(__fdiv_rn(lm[i], dm != 0.0f ? dm : 1.0f)));
                s[i] = static_cast<uint32_t>(si < 63 ? si : 63) & 0xffu;
                mm[i] = static_cast<uint32_t>(mi < 63 ? mi : 63) & 0xffu;
            }
            const int i = lane & 3;
            uint32_t byte;
            if (lane < 4)
                byte = s[i] | ((s[i + 4] & 3u) << 6);
            else if (lane < 8)
                byte = mm[i] | ((mm[i + 4] & 3u) << 6);
            else
                byte = (s[i + 4] >> 2) | ((mm[i + 4] >> 2) << 4);
            blk[4 + lane] = static_cast<uint8_t>(byte);
        }
        if (lane == 0) {
            reinterpret_cast<uint16_t *>(blk)[0] = f32_to_f16_bits(ds);
            reinterpret_cast<uint16_t *>(blk)[1] = f32_to_f16_bits(dm);
        }
        const int sb = lane >> 2;
        const float l = ls[sb] != 0.0f ? ls[sb] : 1.0f;
        uint32_t q0 = 0, q1 = 0;
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            int qi = static_cast<int>(roundf(__fadd_rn(__fdiv_rn(v[i], l), lm[sb])));
            qi = qi < 0 ? 0 : (qi > 15 ? 15 : qi);
            if (i < 4)
                q0 |= static_cast<uint32_t>(qi) << (8 * i);
            else
                q1 |= static_cast<uint32_t>(qi) << (8 * (i - 4));
        }
        // sub-block 2p (low nibbles) pairs with sub-block 2p+1 (high nibbles),
        // which sits 4 lanes further on.
        const uint32_t h0 = __shfl_down_sync(0xffffffffu, q0, 4), h1 = __shfl_down_sync(0xffffffffu, q1, 4);
        if ((sb & 1) == 0) {
            const int pair = sb >> 1;
            uint8_t *dst = blk + 16 + pair * 32 + 8 * (lane & 3);
            const uint32_t w0 = q0 | (h0 << 4), w1 = q1 | (h1 << 4);
            reinterpret_cast<uint16_t *>(dst)[0] = static_cast<uint16_t>(w0 & 0xffffu);
            reinterpret_cast<uint16_t *>(dst)[1] = static_cast<uint16_t>(w0 >> 16);
            reinterpret_cast<uint16_t *>(dst)[2] = static_cast<uint16_t>(w1 & 0xffffu);
            reinterpret_cast<uint16_t *>(dst)[3] = static_cast<uint16_t>(w1 >> 16);
        }
    }
}

// fp32 C -> fp16 / bf16, round to nearest even (cuda_fp16 / cuda_bf16
// conversions); one thread per element.
template <bool kBf16>
__global__ void __launch_bounds__(kThreads) convert_out_kernel(const float *__restrict__ c, int64_t ldc, void *out,
                                                                int64_t ldo, int64_t m, int64_t n) {
    const int64_t total = m * n;
    for (int64_t e = static_cast<int64_t>(blockIdx.x) * kThreads + threadIdx.x; e < total;
         e += static_cast<int64_t>(gridDim.x) * kThreads) {
        const int64_t r = e / n, col = e % n;
        const float v = c[r * ldc + col];
        if constexpr (kBf16)
            static_cast<__nv_bfloat16 *>(out)[r * ldo + col] = __float2bfloat16_rn(v);
        else
            static_cast<__half *>(out)[r * ldo + col] = __float2half_rn(v);
    }
}

int grid_for(int64_t work_items, int items_per_block) {
    const int64_t blocks = (work_items + items_per_block - 1) / items_per_block;
    const int64_t cap = static_cast<int64_t>(device_sm_count()) * 8;
    return static_cast<int>(blocks < 1 ? 1 : (blocks > cap ? cap : blocks));
}

bool vec_ok(const float *x, int64_t ldx) { return (reinterpret_cast<uintptr_t>(x) & 15u) == 0 && (ldx & 3) == 0; }

}  // namespace

cudaError_t launch_quantize_q8_0_strided(const float *x, int64_t ldx, void *y, int64_t ldy, int64_t m, int64_t k,
                                         cudaStream_t s) {
    const int64_t blocks = m * (k / 32);
    const int grid = grid_for(blocks, kThreads / 8);
    SplitA none{};
    uint8_t *out = static_cast<uint8_t *>(y);
    if (vec_ok(x, ldx))
        quantize_q8_0_kernel<true, false><<<grid, kThreads, 0, s>>>(x, ldx, out, ldy, none, m, k, m);
    else
        quantize_q8_0_kernel<false, false><<<grid, kThreads, 0, s>>>(x, ldx, out, ldy, none, m, k, m);
    return cudaGetLastError();
}

cudaError_t launch_quantize_q8_0(const float *x, int64_t ldx, void *y, int64_t m, int64_t k, cudaStream_t s) {
    return launch_quantize_q8_0_strided(x, ldx, y, k / 32, m, k, s);
}

cudaError_t launch_convert_out(const float *c, int64_t ldc, void *out, int64_t ldo, int format, int64_t m, int64_t n,
                               cudaStream_t s) {
    const int grid = grid_for(m * n, kThreads);
    if (format == kOutBF16)
        convert_out_kernel<true><<<grid, kThreads, 0, s>>>(c, ldc, out, ldo, m, n);
    else
        convert_out_kernel<false><<<grid, kThreads, 0, s>>>(c, ldc, out, ldo, m, n);
    return cudaGetLastError();
}

cudaError_t launch_quantize_q8_0_split(const float *x, int64_t ldx, const SplitA &out, int64_t m, int64_t k,
                                       cudaStream_t s) {
    const int64_t blocks = out.rows_pad * (k / 32);
    const int grid = grid_for(blocks, kThreads / 8);
    if (vec_ok(x, ldx))
        quantize_q8_0_kernel<true, true><<<grid, kThreads, 0, s>>>(x, ldx, nullptr, 0, out, m, k, out.rows_pad);
    else
        quantize_q8_0_kernel<false, true><<<grid, kThreads, 0, s>>>(x, ldx, nullptr, 0, out, m, k, out.rows_pad);
    return cudaGetLastError();
}

cudaError_t launch_quantize_q8_K(const float *x, int64_t ldx, void *y, int64_t m, int64_t k, cudaStream_t s) {
    const int grid = grid_for(m * (k / 256), kThreads / 32);
    SplitA none{};
    if (vec_ok(x, ldx))
        quantize_q8_K_kernel<true, false><<<grid, kThreads, 0, s>>>(x, ldx, static_cast<uint8_t *>(y), none, m, k, m);
    else
        quantize_q8_K_kernel<false, false><<<grid, kThreads, 0, s>>>(x, ldx, static_cast<uint8_t *>(y), none, m, k, m);
    return cudaGetLastError();
}

cudaError_t launch_quantize_q8_K_split(const float *x, int64_t ldx, const SplitA &out, int64_t m, int64_t k,
                                       cudaStream_t s) {
    const int grid = grid_for(out.rows_pad * (k / 256), kThreads / 32);
    if (vec_ok(x, ldx))
        quantize_q8_K_kernel<true, true><<<grid, kThreads, 0, s>>>(x, ldx, nullptr, out, m, k, out.rows_pad);
    else
        quantize_q8_K_kernel<false, true><<<grid, kThreads, 0, s>>>(x, ldx, nullptr, out, m, k, out.rows_pad);
    return cudaGetLastError();
}

cudaError_t launch_convert_q8_0_split(const void *a, const SplitA &out, int64_t m, int64_t k, cudaStream_t s) {
    const int grid = grid_for(out.rows_pad * (k / 32), kThreads / 8);
    convert_q8_0_split_kernel<<<grid, kThreads, 0, s>>>(static_cast<const uint8_t *>(a), out, m, k, out.rows_pad);
    return cudaGetLastError();
}

cudaError_t launch_convert_q8_K_split(const void *a, const SplitA &out, int64_t m, int64_t k, cudaStream_t s) {
    const int grid = grid_for(out.rows_pad * (k / 256), kThreads / 32);
    convert_q8_K_split_kernel<<<grid, kThreads, 0, s>>>(static_cast<const uint8_t *>(a), out, m, k, out.rows_pad);
    return cudaGetLastError();
}

cudaError_t launch_quantize_q4_0(const float *x, int64_t ldx, void *y, int64_t n, int64_t k, cudaStream_t s) {
    const int grid = grid_for(n * (k / 32), kThreads / 8);
    if (vec_ok(x, ldx))
        quantize_q4_0_kernel<true><<<grid, kThreads, 0, s>>>(x, ldx, static_cast<uint8_t *>(y), n, k);
    else
        quantize_q4_0_kernel<false><<<grid, kThreads, 0, s>>>(x, ldx, static_cast<uint8_t *>(y), n, k);
    return cudaGetLastError();
}

cudaError_t launch_quantize_q4_K(const float *x, int64_t ldx, void *y, int64_t n, int64_t k, cudaStream_t s) {
    const int grid = grid_for(n * (k / 256), kThreads / 32);
    if (vec_ok(x, ldx))
        quantize_q4_K_kernel<true><<<grid, kThreads, 0, s>>>(x, ldx, static_cast<uint8_t *>(y), n, k);
    else
        quantize_q4_K_kernel<false><<<grid, kThreads, 0, s>>>(x, ldx, static_cast<uint8_t *>(y), n, k);
    return cudaGetLastError();
}

}  // namespace pfng
