// pfng_quant.cuh -- the activation-quantizer cores shared by the standalone
// quantizer kernels and the fused quantize+matmul kernels, so both produce
// the same bytes.  Operation order follows the reference's
// quantize_row_q8_0 / quantize_row_q8_K
// (bench/llama_reference/llama_reference.cpp:38-70): IEEE divide for the
// scale and its reciprocal, an IEEE multiply, then round half away from zero.
#pragma once

#include "pfng_common.cuh"

namespace pfng {

// roundf(y) (round half away from zero) as an int, for |y| < 2^22: the
// integer part of |y| + 0.5, sign restored.  |y| + 0.5 is rounded to float
// before the truncation, which changes the result for exactly one magnitude:
// 0.49999997 (the largest float below 0.5), whose sum with 0.5 is a tie that
// rounds up to 1.0.  Every other |y| < 2^22 either adds exactly or rounds to
// a value with the same integer part.  Same result as (int)roundf(y).
PFNG_DEV int round_half_away(float y) {
    const float a = fabsf(y);
    int r = __float2int_rz(__fadd_rn(a, 0.5f));
    if (a == 0.49999997f) r = 0;
    return y < 0.0f ? -r : r;
}

// ---------------------------------------------------------------------------
// q8_0 with 4 lanes per 32-value block, lane c of the group holding values
// 8c..8c+7 (llama_reference.cpp:38-52).  Two shuffle levels per reduction;
// the rounding is round_half_away above.
// ---------------------------------------------------------------------------
struct Q8_0Quad {
    uint32_t q0, q1;  // 8 packed int8
    uint16_t dbits;   // fp16 scale
    int qsum;         // sum of the whole block's int8 values (all 4 lanes)
};

template <int N>
PFNG_DEV void q8_0_quantize_quads(const float (&v)[N][8], Q8_0Quad (&r)[N]) {
    float amax[N], scale[N], inv[N];
    int s[N];
#pragma unroll
    for (int b = 0; b < N; ++b) {
        amax[b] = 0.0f;
#pragma unroll
        for (int i = 0; i < 8; ++i) amax[b] = fmaxf(amax[b], fabsf(v[b][i]));
    }
#pragma unroll
    for (int o = 1; o < 4; o <<= 1)
#pragma unroll
        for (int b = 0; b < N; ++b) amax[b] = fmaxf(amax[b], __shfl_xor_sync(0xffffffffu, amax[b], o));
#pragma unroll
    for (int b = 0; b < N; ++b) scale[b] = __fdiv_rn(amax[b], 127.0f);
#pragma unroll
    for (int b = 0; b < N; ++b) inv[b] = scale[b] != 0.0f ? __frcp_rn(scale[b]) : 0.0f;
#pragma unroll
    for (int b = 0; b < N; ++b) {
        r[b].q0 = r[b].q1 = 0;
        s[b] = 0;
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const int qi = round_half_away(__fmul_rn(v[b][i], inv[b]));
            s[b] += qi;
            if (i < 4)
                r[b].q0 |= (static_cast<uint32_t>(qi) & 0xffu) << (8 * i);
            else
                r[b].q1 |= (static_cast<uint32_t>(qi) & 0xffu) << (8 * (i - 4));
        }
    }
#pragma unroll
    for (int o = 1; o < 4; o <<= 1)
#pragma unroll
        for (int b = 0; b < N; ++b) s[b] += __shfl_xor_sync(0xffffffffu, s[b], o);
#pragma unroll
    for (int b = 0; b < N; ++b) {
        r[b].qsum = s[b];
        r[b].dbits = f32_to_f16_bits(scale[b]);
    }
}

// ---------------------------------------------------------------------------
// q8_0: 8 lanes per 32-value block, lane g of the group holds values 4g..4g+3.
// llama_reference.cpp:38-52.
// ---------------------------------------------------------------------------
struct Q8_0Lane {
    uint32_t q;      // 4 packed int8
    uint16_t dbits;  // fp16 scale
    int qsum;        // sum of the whole block's int8 values (all lanes)
};

// N independent blocks per lane group, each step applied to all N before the
// next so their dependency chains (shuffles, divisions) overlap.  Every block
// sees exactly the arithmetic of the single-block form.
template <int N>
PFNG_DEV void q8_0_quantize_lanes(const float (&v)[N][4], Q8_0Lane (&r)[N]) {
    float amax[N], scale[N], inv[N];
    int s[N];
#pragma unroll
    for (int b = 0; b < N; ++b) {
        amax[b] = 0.0f;
#pragma unroll
        for (int i = 0; i < 4; ++i) amax[b] = fmaxf(amax[b], fabsf(v[b][i]));
    }
#pragma unroll
    for (int o = 1; o < 8; o <<= 1)
#pragma unroll
        for (int b = 0; b < N; ++b) amax[b] = fmaxf(amax[b], __shfl_xor_sync(0xffffffffu, amax[b], o));
#pragma unroll
    for (int b = 0; b < N; ++b) scale[b] = __fdiv_rn(amax[b], 127.0f);
#pragma unroll
    for (int b = 0; b < N; ++b) inv[b] = scale[b] != 0.0f ? __fdiv_rn(1.0f, scale[b]) : 0.0f;
#pragma unroll
    for (int b = 0; b < N; ++b) {
        r[b].q = 0;
        s[b] = 0;
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const int qi = static_cast<int>(roundf(__fmul_rn(v[b][i], inv[b])));
            s[b] += qi;
            r[b].q |= (static_cast<uint32_t>(qi) & 0xffu) << (8 * i);
        }
    }
#pragma unroll
    for (int o = 1; o < 8; o <<= 1)
#pragma unroll
        for (int b = 0; b < N; ++b) s[b] += __shfl_xor_sync(0xffffffffu, s[b], o);
#pragma unroll
    for (int b = 0; b < N; ++b) {
        r[b].qsum = s[b];
        r[b].dbits = f32_to_f16_bits(scale[b]);
    }
}

PFNG_DEV Q8_0Lane q8_0_quantize_lane(const float v[4]) {
    float vv[1][4] = {{v[0], v[1], v[2], v[3]}};
    Q8_0Lane r[1];
    q8_0_quantize_lanes<1>(vv, r);
    return r[0];
}

// q8_K: one warp per 256-value block, lane l holds values 8l..8l+7.
struct Q8_KLane {
    uint32_t q0, q1;  // 8 packed int8 (values 8l..8l+3, 8l+4..8l+7)
    int sum16;        // sum over the 16 values of lanes (l & ~1, l | 1): the bsums entry
    int sum32;        // sum over the 32 values of lanes 4(l/4)..4(l/4)+3
    float d;          // fp32 scale
};

PFNG_DEV Q8_KLane q8_K_quantize_lane(const float v[8]) {
    float amax = 0.0f;
#pragma unroll
    for (int i = 0; i < 8; ++i) amax = fmaxf(amax, fabsf(v[i]));
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
    Q8_KLane r;
    r.d = __fdiv_rn(amax, 127.0f);
    const float inv = r.d != 0.0f ? __fdiv_rn(1.0f, r.d) : 0.0f;
    r.q0 = 0;
    r.q1 = 0;
    int s = 0;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        const int qi = static_cast<int>(roundf(__fmul_rn(v[i], inv)));
        s += qi;
        if (i < 4)
            r.q0 |= (static_cast<uint32_t>(qi) & 0xffu) << (8 * i);
        else
            r.q1 |= (static_cast<uint32_t>(qi) & 0xffu) << (8 * (i - 4));
    }
    r.sum16 = s + __shfl_xor_sync(0xffffffffu, s, 1);
    r.sum32 = r.sum16 + __shfl_xor_sync(0xffffffffu, r.sum16, 2);
    return r;
}

}  // namespace pfng
