// gemv.cu -- small-m (decode) block-quantized matmul, HBM-streaming.
//
// C[m][n] = A[m][k] . W[n][k]^T for m <= 8, W in the raw ggml layout.
// Semantics: compute_q4_0 / compute_q4_K / compute_iq2_xxs of
// bench/llama_reference/llama_reference.cpp:165-205 (dot products :113-161).
//
// Structure (one persistent CTA per SM, warp-specialised):
//   * a producer warp streams tiles of R consecutive weight rows -- a
//     contiguous byte range of W -- into a ring of S shared-memory stages with
//     bulk TMA copies (cp.async.bulk, mbarrier transaction counts, L2
//     evict-first since every weight byte is read once);
//   * 8 consumer warps first stage the activation rows in shared memory
//     (either the caller's q8 blocks, or fp32 rows quantized in place with
//     the same code as the standalone quantizer), then each takes one row of
//     a tile: lanes walk the row's blocks, unpack 4-bit / grid weights to
//     int8, dot them against the activations with dp4a, fold the integer
//     partials with the block scales in fp32 and reduce across the warp.
// The kernel is bound by HBM bandwidth; per weight byte it issues a handful
// of shared-memory reads and integer ops, well under what an SM sustains.
//
// Every mbarrier wait is bounded (pfng_common.cuh): a wait that gives up
// records an error code, stops the CTA's work and returns.
#include "iq2xxs_grid_codes.h"
#include "pfng_common.cuh"
#include "pfng_internal.h"
#include "pfng_quant.cuh"

namespace pfng {
namespace {

constexpr int kConsumerWarps = 8;
constexpr int kConsumerThreads = kConsumerWarps * 32;
constexpr int kGemvThreads = kConsumerThreads + 32;
constexpr int kMaxStages = 16;
constexpr uint32_t kBarrierBytes = 2 * kMaxStages * 8;
constexpr uint32_t kGridTableBytes = 256 * 8;
constexpr uint32_t kStageSlack = 32;  // bytes read past a window by aligned loads; never used

struct GemvParams {
    const uint8_t *w;
    const uint8_t *a;  // raw q8 blocks or nullptr
    const float *x;    // fp32 activations or nullptr
    int64_t ldx;
    float *c;
    int64_t ldc;
    int32_t *partials;
    int *err;  // library error word for bounded waits
    int m;
    int64_t n, k;
    int64_t row_bytes;
    int rows_per_tile;
    int64_t num_tiles;
    int stages;
    uint32_t stage_bytes;
    uint32_t grid_offset, act_offset, stage_offset;
};

// Activation rows staged in shared memory.
struct Act {
    const int8_t *qs;     // [MT][k]
    const float *d;       // [MT][k/32] (q8_0) or [MT][k/256] (q8_K)
    const int32_t *s8;    // q8_0: 8 * sum of the block's values, [MT][k/32]
    const int16_t *bs;    // q8_K: bsums [MT][k/16]
};

PFNG_DEV void consumer_sync() { asm volatile("bar.sync 1, %0;" ::"n"(kConsumerThreads) : "memory"); }

// --------------------------------------------------------------------------
// activation staging
// --------------------------------------------------------------------------
template <int MT, bool kF32>
PFNG_DEV void stage_act_q8_0(const GemvParams &p, uint8_t *smem, int tid) {
    const int64_t nb = p.k / 32;
    int8_t *qs = reinterpret_cast<int8_t *>(smem + p.act_offset);
    float *d = reinterpret_cast<float *>(qs + MT * p.k);
    int32_t *s8 = reinterpret_cast<int32_t *>(d + MT * nb);
    const int64_t total = MT * nb;
    const int lane = tid & 31, warp = tid >> 5, g = lane & 7;
    for (int64_t wb = warp * 4; wb < total; wb += kConsumerWarps * 4) {
        const int64_t bi = wb + (lane >> 3);
        const bool live = bi < total;
        const int64_t row = live ? bi / nb : 0, col = live ? bi % nb : 0;
        const bool valid = live && row < p.m;
        uint32_t q = 0;
        uint32_t dbits = 0;
        int qsum = 0;
        if constexpr (kF32) {
            float v[4] = {0.0f, 0.0f, 0.0f, 0.0f};
            if (valid) {
                const float *src = p.x + row * p.ldx + col * 32 + 4 * g;
#pragma unroll
                for (int i = 0; i < 4; ++i) v[i] = __ldg(src + i);
            }
            const Q8_0Lane r = q8_0_quantize_lane(v);
            q = r.q;
            dbits = r.dbits;
            qsum = r.qsum;
        } else {
            if (valid) {
                const uint8_t *blk = p.a + (row * nb + col) * kQ8_0Bytes;
                const uint16_t *h = reinterpret_cast<const uint16_t *>(blk + 2 + 4 * g);
                q = static_cast<uint32_t>(__ldg(h)) | (static_cast<uint32_t>(__ldg(h + 1)) << 16);
                dbits = __ldg(reinterpret_cast<const uint16_t *>(blk));
            }
            int s = __dp4a(static_cast<int>(q), 0x01010101, 0);
#pragma unroll
            for (int o = 1; o < 8; o <<= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
            qsum = s;
        }
        if (!live) continue;
        *reinterpret_cast<uint32_t *>(qs + row * p.k + col * 32 + 4 * g) = valid ? q : 0u;
        if (g == 0) {
            d[row * nb + col] = valid ? f16_bits_to_f32(dbits) : 0.0f;
            s8[row * nb + col] = valid ? 8 * qsum : 0;
        }
    }
}

template <int MT, bool kF32>
PFNG_DEV void stage_act_q8_K(const GemvParams &p, uint8_t *smem, int tid) {
    const int64_t nb = p.k / 256;
    int8_t *qs = reinterpret_cast<int8_t *>(smem + p.act_offset);
    float *d = reinterpret_cast<float *>(qs + MT * p.k);
    int16_t *bs = reinterpret_cast<int16_t *>(d + MT * nb);
    const int64_t total = MT * nb;
    const int lane = tid & 31, warp = tid >> 5;
    for (int64_t bi = warp; bi < total; bi += kConsumerWarps) {
        const int64_t row = bi / nb, col = bi % nb;
        const bool valid = row < p.m;
        uint32_t q0 = 0, q1 = 0;
        float dv = 0.0f;
        int bsum = 0;  // lanes < 16: bsums[lane]
        if constexpr (kF32) {
            float v[8] = {0, 0, 0, 0, 0, 0, 0, 0};
            if (valid) {
                const float *src = p.x + row * p.ldx + col * 256 + 8 * lane;
#pragma unroll
                for (int i = 0; i < 8; ++i) v[i] = __ldg(src + i);
            }
            const Q8_KLane r = q8_K_quantize_lane(v);
            q0 = r.q0;
            q1 = r.q1;
            dv = r.d;
            // bsums entry j lives in lanes 2j and 2j+1
            bsum = __shfl_sync(0xffffffffu, r.sum16, (2 * lane) & 31);
        } else if (valid) {
            const uint8_t *blk = p.a + (row * nb + col) * kQ8_KBytes;
            const uint32_t *q = reinterpret_cast<const uint32_t *>(blk + kQ8_KQsOffset + 8 * lane);
            q0 = __ldg(q);
            q1 = __ldg(q + 1);
            dv = __ldg(reinterpret_cast<const float *>(blk));
            if (lane < 16) bsum = __ldg(reinterpret_cast<const int16_t *>(blk + kQ8_KBsumsOffset) + lane);
        }
        uint32_t *dst = reinterpret_cast<uint32_t *>(qs + row * p.k + col * 256 + 8 * lane);
        dst[0] = q0;
        dst[1] = q1;
        if (lane < 16) bs[row * (p.k / 16) + col * 16 + lane] = static_cast<int16_t>(valid ? bsum : 0);
        if (lane == 0) d[row * nb + col] = dv;
    }
}

// --------------------------------------------------------------------------
// per-row dot products.  `tile` is the stage buffer, `row_off` the byte
// offset of the row inside it.  Loops are warp-uniform (shuffles inside).
// --------------------------------------------------------------------------
template <int MT>
PFNG_DEV void warp_reduce_store(const GemvParams &p, float (&acc)[MT], int64_t row, int lane) {
#pragma unroll
    for (int mi = 0; mi < MT; ++mi) {
        float v = acc[mi];
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
        if (lane == 0 && mi < p.m) p.c[mi * p.ldc + row] = v;
    }
}

template <int MT, bool kPartials>
PFNG_DEV void row_q4_0(const GemvParams &p, const Act &act, const uint8_t *tile, uint32_t row_off, int64_t row,
                       int lane) {
    const int nb = static_cast<int>(p.k / 32);
    float acc[MT];
#pragma unroll
    for (int mi = 0; mi < MT; ++mi) acc[mi] = 0.0f;
    for (int base = 0; base < nb; base += 32) {
        const int j = base + lane;
        if (j < nb) {
            uint32_t q[4], dbits;
            load_q4_0_block_smem(tile, row_off + 18u * j, q, dbits);
            const float dw = f16_bits_to_f32(dbits);
            uint32_t lo[4], hi[4];
#pragma unroll
            for (int i = 0; i < 4; ++i) lo[i] = q[i] & 0x0f0f0f0fu, hi[i] = (q[i] >> 4) & 0x0f0f0f0fu;
#pragma unroll
            for (int mi = 0; mi < MT; ++mi) {
                const int4 *a4 = reinterpret_cast<const int4 *>(act.qs + mi * p.k + 32 * j);
                const int4 a0 = a4[0], a1 = a4[1];
                int dot = dp4a(lo[0], a0.x, 0);
                dot = dp4a(lo[1], a0.y, dot);
                dot = dp4a(lo[2], a0.z, dot);
                dot = dp4a(lo[3], a0.w, dot);
                dot = dp4a(hi[0], a1.x, dot);
                dot = dp4a(hi[1], a1.y, dot);
                dot = dp4a(hi[2], a1.z, dot);
                dot = dp4a(hi[3], a1.w, dot);
                const int isum = dot - act.s8[mi * nb + j];
                if constexpr (kPartials) {
                    if (mi < p.m) p.partials[(mi * p.n + row) * nb + j] = isum;
                } else {
                    acc[mi] = __fmaf_rn(__fmul_rn(static_cast<float>(isum), dw), act.d[mi * nb + j], acc[mi]);
                }
            }
        }
    }
    if constexpr (!kPartials) warp_reduce_store<MT>(p, acc, row, lane);
}

PFNG_DEV uint32_t scale_byte(uint32_t s0, uint32_t s1, uint32_t s2, int i) {
    return (i < 8 ? __byte_perm(s0, s1, static_cast<uint32_t>(i)) : __byte_perm(s2, 0u, static_cast<uint32_t>(i - 8))) &
           0xffu;
}

// 6-bit scale and min of sub-block j (llama_reference.cpp:116-121).
PFNG_DEV void q4_K_scale_min(uint32_t s0, uint32_t s1, uint32_t s2, int j, int &sc, int &mn) {
    if (j < 4) {
        sc = scale_byte(s0, s1, s2, j) & 63;
        mn = scale_byte(s0, s1, s2, j + 4) & 63;
    } else {
        sc = (scale_byte(s0, s1, s2, j + 4) & 15) | ((scale_byte(s0, s1, s2, j - 4) >> 6) << 4);
        mn = (scale_byte(s0, s1, s2, j + 4) >> 4) | ((scale_byte(s0, s1, s2, j) >> 6) << 4);
    }
}

template <int MT, bool kPartials>
PFNG_DEV void row_q4_K(const GemvParams &p, const Act &act, const uint8_t *tile, uint32_t row_off, int64_t row,
                       int lane) {
    const int nbk = static_cast<int>(p.k / 256);
    const int units = nbk * 8;  // (block, nibble pair, half of the 32 bytes)
    float acc[MT];
#pragma unroll
    for (int mi = 0; mi < MT; ++mi) acc[mi] = 0.0f;
    for (int base = 0; base < units; base += 32) {
        const int u = base + lane;
        const bool live = u < units;
        const int b = live ? u >> 3 : 0, pr = (u >> 1) & 3, h = u & 1;
        const uint8_t *blk = tile + row_off + 144u * b;
        const uint32_t dd = *reinterpret_cast<const uint32_t *>(blk);
        const uint32_t s0 = *reinterpret_cast<const uint32_t *>(blk + 4);
        const uint32_t s1 = *reinterpret_cast<const uint32_t *>(blk + 8);
        const uint32_t s2 = *reinterpret_cast<const uint32_t *>(blk + 12);
        const uint4 qv = *reinterpret_cast<const uint4 *>(blk + 16 + 32 * pr + 16 * h);
        const int sbl = 2 * pr, sbh = 2 * pr + 1;
        int scl, mnl, sch, mnh;
        q4_K_scale_min(s0, s1, s2, sbl, scl, mnl);
        q4_K_scale_min(s0, s1, s2, sbh, sch, mnh);
        const float d = f16_bits_to_f32(dd & 0xffffu), dmin = f16_bits_to_f32(dd >> 16);
        const uint32_t lo0 = qv.x & 0x0f0f0f0fu, lo1 = qv.y & 0x0f0f0f0fu, lo2 = qv.z & 0x0f0f0f0fu,
                       lo3 = qv.w & 0x0f0f0f0fu;
        const uint32_t hi0 = (qv.x >> 4) & 0x0f0f0f0fu, hi1 = (qv.y >> 4) & 0x0f0f0f0fu,
                       hi2 = (qv.z >> 4) & 0x0f0f0f0fu, hi3 = (qv.w >> 4) & 0x0f0f0f0fu;
#pragma unroll
        for (int mi = 0; mi < MT; ++mi) {
            const int8_t *aq = act.qs + mi * p.k + b * 256 + 16 * h;
            const int4 al = *reinterpret_cast<const int4 *>(aq + sbl * 32);
            const int4 ah = *reinterpret_cast<const int4 *>(aq + sbh * 32);
            int ql = dp4a(lo0, al.x, 0);
            ql = dp4a(lo1, al.y, ql);
            ql = dp4a(lo2, al.z, ql);
            ql = dp4a(lo3, al.w, ql);
            int qh = dp4a(hi0, ah.x, 0);
            qh = dp4a(hi1, ah.y, qh);
            qh = dp4a(hi2, ah.z, qh);
            qh = dp4a(hi3, ah.w, qh);
            if constexpr (kPartials) {
                const int fl = ql + __shfl_xor_sync(0xffffffffu, ql, 1);
                const int fh = qh + __shfl_xor_sync(0xffffffffu, qh, 1);
                if (live && h == 0 && mi < p.m) {
                    int32_t *out = p.partials + (mi * p.n + row) * (p.k / 32) + b * 8;
                    out[sbl] = fl;
                    out[sbh] = fh;
                }
            } else if (live) {
                const int16_t *bs = act.bs + mi * (p.k / 16) + b * 16;
                const int i1 = scl * ql + sch * qh;
                const int i2 = mnl * bs[sbl * 2 + h] + mnh * bs[sbh * 2 + h];
                const float part = __fsub_rn(__fmul_rn(d, static_cast<float>(i1)), __fmul_rn(dmin, static_cast<float>(i2)));
                acc[mi] = __fmaf_rn(act.d[mi * nbk + b], part, acc[mi]);
            }
        }
    }
    if constexpr (!kPartials) warp_reduce_store<MT>(p, acc, row, lane);
}

template <int MT, bool kPartials>
PFNG_DEV void row_iq2_xxs(const GemvParams &p, const Act &act, const uint8_t *tile, uint32_t row_off, int64_t row,
                          int lane, const uint2 *grid) {
    const int nbk = static_cast<int>(p.k / 256);
    const int units = nbk * 8;  // (block, 32-value group)
    float acc[MT];
#pragma unroll
    for (int mi = 0; mi < MT; ++mi) acc[mi] = 0.0f;
    for (int base = 0; base < units; base += 32) {
        const int u = base + lane;
        if (u < units) {
            const int b = u >> 3, sb = u & 7;
            const uint32_t boff = row_off + 66u * b;
            const float d = f16_bits_to_f32(*reinterpret_cast<const uint16_t *>(tile + boff));
            const uint32_t off = boff + 2 + 8 * sb;
            const uint32_t *w = reinterpret_cast<const uint32_t *>(tile + (off & ~3u));
            const uint32_t sh = (off & 2u) ? 16u : 0u;
            const uint32_t w0 = w[0], w1 = w[1], w2 = w[2];
            const uint32_t idx = __funnelshift_r(w0, w1, sh);
            const uint32_t ss = __funnelshift_r(w1, w2, sh);
            uint32_t v[8];
#pragma unroll
            for (int g = 0; g < 4; ++g) {
                const uint2 gv = grid[(idx >> (8 * g)) & 0xffu];
                const uint32_t sgn = iq2_sign_mask((ss >> (7 * g)) & 0x7fu);
                v[2 * g] = apply_sign_bytes(gv.x, expand_bits4(sgn));
                v[2 * g + 1] = apply_sign_bytes(gv.y, expand_bits4(sgn >> 4));
            }
            const int scale = 2 * static_cast<int>(ss >> 28) + 1;
#pragma unroll
            for (int mi = 0; mi < MT; ++mi) {
                const int4 *a4 = reinterpret_cast<const int4 *>(act.qs + mi * p.k + b * 256 + sb * 32);
                const int4 a0 = a4[0], a1 = a4[1];
                int dot = dp4a(static_cast<int>(v[0]), a0.x, 0);
                dot = dp4a(static_cast<int>(v[1]), a0.y, dot);
                dot = dp4a(static_cast<int>(v[2]), a0.z, dot);
                dot = dp4a(static_cast<int>(v[3]), a0.w, dot);
                dot = dp4a(static_cast<int>(v[4]), a1.x, dot);
                dot = dp4a(static_cast<int>(v[5]), a1.y, dot);
                dot = dp4a(static_cast<int>(v[6]), a1.z, dot);
                dot = dp4a(static_cast<int>(v[7]), a1.w, dot);
                if constexpr (kPartials) {
                    if (mi < p.m) p.partials[(mi * p.n + row) * (p.k / 32) + b * 8 + sb] = dot;
                } else {
                    const float s = __fmul_rn(__fmul_rn(0.125f, d), act.d[mi * nbk + b]);
                    acc[mi] = __fmaf_rn(s, static_cast<float>(scale * dot), acc[mi]);
                }
            }
        }
    }
    if constexpr (!kPartials) warp_reduce_store<MT>(p, acc, row, lane);
}

// --------------------------------------------------------------------------
// the kernel
// --------------------------------------------------------------------------
template <int WT, int MT, bool kPartials, bool kF32>
__global__ void __launch_bounds__(kGemvThreads, 1) gemv_kernel(const GemvParams p) {
    extern __shared__ __align__(128) uint8_t smem[];
    uint64_t *full = reinterpret_cast<uint64_t *>(smem);
    uint64_t *empty = full + kMaxStages;
    __shared__ int abort_flag;
    const int tid = threadIdx.x;
    const int warp = tid >> 5, lane = tid & 31;
    const int R = p.rows_per_tile;
    const int S = p.stages;

    if (tid == 0) {
        for (int s = 0; s < S; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], R);
        }
        abort_flag = 0;
        fence_mbar_init();
    }
    __syncthreads();

    if (warp == kConsumerWarps) {
        // ---------------- producer ----------------
        if (lane == 0) {
            const uint64_t policy = l2_policy_evict_first();
            int64_t issued = 0;
            for (int64_t i = 0;; ++i) {
                const int64_t tile = blockIdx.x + i * gridDim.x;
                if (tile >= p.num_tiles) break;
                const int stage = static_cast<int>(i % S);
                if (i >= S && !mbar_wait(&empty[stage], static_cast<uint32_t>(((i / S) & 1) ^ 1), p.err, kErrWaitEmpty)) {
                    abort_flag = 1;
                    break;
                }
                if (*reinterpret_cast<volatile int *>(&abort_flag)) break;
                const int64_t start = tile * R * p.row_bytes;
                const int64_t last = (tile + 1) * R < p.n ? (tile + 1) * R : p.n;
                const int64_t end = last * p.row_bytes;
                const int64_t ws = start & ~int64_t(15), we = (end + 15) & ~int64_t(15);
                const uint32_t bytes = static_cast<uint32_t>(we - ws);
                uint8_t *dst = smem + p.stage_offset + static_cast<uint32_t>(stage) * p.stage_bytes;
                mbar_arrive_expect_tx(&full[stage], bytes);
                bulk_copy_g2s(dst, p.w + ws, bytes, &full[stage], policy);
                issued = i + 1;
            }
            // Do not leave while copies into this CTA's shared memory are in
            // flight (matters only when a consumer gave up early).
            for (int64_t i = issued - S > 0 ? issued - S : 0; i < issued; ++i)
                mbar_wait(&full[i % S], static_cast<uint32_t>((i / S) & 1), p.err, kErrWaitFull);
        }
        return;
    }

    // ---------------- consumers ----------------
    uint2 *grid = reinterpret_cast<uint2 *>(smem + p.grid_offset);
    if constexpr (WT == 2) {
        for (int i = tid; i < 256; i += kConsumerThreads) {
            const uint32_t code = pfng_iq2xxs_grid_codes[i];
            uint32_t lo = 0, hi = 0;
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                const uint32_t c = (code >> (2 * j)) & 3u;
                const uint32_t byte = 8u + 17u * c + (c >> 1);
                if (j < 4)
                    lo |= byte << (8 * j);
                else
                    hi |= byte << (8 * (j - 4));
            }
            grid[i] = make_uint2(lo, hi);
        }
    }
    Act act;
    if constexpr (WT == 0) {
        stage_act_q8_0<MT, kF32>(p, smem, tid);
        const int64_t nb = p.k / 32;
        act.qs = reinterpret_cast<const int8_t *>(smem + p.act_offset);
        act.d = reinterpret_cast<const float *>(act.qs + MT * p.k);
        act.s8 = reinterpret_cast<const int32_t *>(act.d + MT * nb);
        act.bs = nullptr;
    } else {
        stage_act_q8_K<MT, kF32>(p, smem, tid);
        const int64_t nb = p.k / 256;
        act.qs = reinterpret_cast<const int8_t *>(smem + p.act_offset);
        act.d = reinterpret_cast<const float *>(act.qs + MT * p.k);
        act.bs = reinterpret_cast<const int16_t *>(act.d + MT * nb);
        act.s8 = nullptr;
    }
    consumer_sync();

    const int G = kConsumerWarps / R;
    const int grp = warp / R, r = warp % R;
    for (int64_t i = grp;; i += G) {
        const int64_t tile = blockIdx.x + i * gridDim.x;
        if (tile >= p.num_tiles) break;
        if (*reinterpret_cast<volatile int *>(&abort_flag)) break;
        const int stage = static_cast<int>(i % S);
        if (!mbar_wait(&full[stage], static_cast<uint32_t>((i / S) & 1), p.err, kErrWaitFull)) {
            abort_flag = 1;
            break;
        }
        const int64_t row = tile * R + r;
        if (row < p.n) {
            const int64_t ws = (tile * R * p.row_bytes) & ~int64_t(15);
            const uint32_t row_off = static_cast<uint32_t>(row * p.row_bytes - ws);
            const uint8_t *buf = smem + p.stage_offset + static_cast<uint32_t>(stage) * p.stage_bytes;
            if constexpr (WT == 0)
                row_q4_0<MT, kPartials>(p, act, buf, row_off, row, lane);
            else if constexpr (WT == 1)
                row_q4_K<MT, kPartials>(p, act, buf, row_off, row, lane);
            else
                row_iq2_xxs<MT, kPartials>(p, act, buf, row_off, row, lane, grid);
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[stage]);
    }
}

int64_t row_bytes_of(int wtype, int64_t k) {
    switch (wtype) {
    case 0: return k / 32 * kQ4_0Bytes;
    case 1: return k / 256 * kQ4_KBytes;
    default: return k / 256 * kIQ2Bytes;
    }
}

int mt_of(int64_t m) { return m <= 1 ? 1 : m <= 2 ? 2 : m <= 4 ? 4 : 8; }

uint32_t act_bytes_of(int wtype, int mt, int64_t k) {
    if (wtype == 0) return static_cast<uint32_t>(mt * (k + (k / 32) * 8));
    return static_cast<uint32_t>(mt * (k + (k / 256) * 4 + (k / 16) * 2));
}

uint32_t align_up_u32(uint32_t v, uint32_t a) { return (v + a - 1) / a * a; }

// Fills the tiling / shared-memory plan; false if the shape does not fit.
bool plan(int wtype, int64_t m, int64_t n, int64_t k, GemvParams &p, uint32_t &smem_bytes) {
    const int mt = mt_of(m);
    p.row_bytes = row_bytes_of(wtype, k);
    p.rows_per_tile = p.row_bytes >= 1024 ? 4 : 8;
    p.num_tiles = (n + p.rows_per_tile - 1) / p.rows_per_tile;
    p.stage_bytes = align_up_u32(static_cast<uint32_t>(p.rows_per_tile * p.row_bytes) + 16 + kStageSlack, 128);
    p.grid_offset = kBarrierBytes;
    p.act_offset = p.grid_offset + (wtype == 2 ? kGridTableBytes : 0);
    p.stage_offset = align_up_u32(p.act_offset + act_bytes_of(wtype, mt, k), 128);
    const size_t budget = device_smem_optin() - 1024;  // static shared + reserve
    if (p.stage_offset + 2 * static_cast<size_t>(p.stage_bytes) > budget) return false;
    const size_t fit = (budget - p.stage_offset) / p.stage_bytes;
    p.stages = static_cast<int>(fit < kMaxStages ? fit : kMaxStages);
    smem_bytes = p.stage_offset + static_cast<uint32_t>(p.stages) * p.stage_bytes;
    return true;
}

template <int WT, int MT, bool kPartials, bool kF32>
cudaError_t launch_one(const GemvParams &p, uint32_t smem, cudaStream_t s) {
    auto kernel = gemv_kernel<WT, MT, kPartials, kF32>;
    cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
    if (e != cudaSuccess) return e;
    const int64_t sms = device_sm_count();
    const int grid = static_cast<int>(p.num_tiles < sms ? p.num_tiles : sms);
    kernel<<<grid, kGemvThreads, smem, s>>>(p);
    return cudaGetLastError();
}

template <int WT, int MT>
cudaError_t dispatch_flags(const GemvParams &p, uint32_t smem, bool partials, bool f32, cudaStream_t s) {
    if (partials) return f32 ? launch_one<WT, MT, true, true>(p, smem, s) : launch_one<WT, MT, true, false>(p, smem, s);
    return f32 ? launch_one<WT, MT, false, true>(p, smem, s) : launch_one<WT, MT, false, false>(p, smem, s);
}

template <int WT>
cudaError_t dispatch_mt(const GemvParams &p, uint32_t smem, bool partials, bool f32, cudaStream_t s) {
    switch (mt_of(p.m)) {
    case 1: return dispatch_flags<WT, 1>(p, smem, partials, f32, s);
    case 2: return dispatch_flags<WT, 2>(p, smem, partials, f32, s);
    case 4: return dispatch_flags<WT, 4>(p, smem, partials, f32, s);
    default: return dispatch_flags<WT, 8>(p, smem, partials, f32, s);
    }
}

}  // namespace

bool gemv_supported(int wtype, int64_t m, int64_t n, int64_t k, const void *w) {
    if (m < 1 || m > 8 || n < 1) return false;
    const int64_t rb = row_bytes_of(wtype, k);
    if ((reinterpret_cast<uintptr_t>(w) & 15u) != 0 || (n * rb) % 16 != 0) return false;
    GemvParams p{};
    uint32_t smem = 0;
    return plan(wtype, m, n, k, p, smem);
}

cudaError_t launch_gemv(const GemvArgs &args, cudaStream_t s) {
    GemvParams p{};
    uint32_t smem = 0;
    if (!plan(args.wtype, args.m, args.n, args.k, p, smem)) return cudaErrorInvalidValue;
    p.w = static_cast<const uint8_t *>(args.w);
    p.a = static_cast<const uint8_t *>(args.a);
    p.x = args.x;
    p.ldx = args.ldx;
    p.c = args.c;
    p.ldc = args.ldc;
    p.partials = args.partials;
    p.err = args.err;
    p.m = static_cast<int>(args.m);
    p.n = args.n;
    p.k = args.k;
    const bool partials = args.partials != nullptr;
    const bool f32 = args.x != nullptr;
    switch (args.wtype) {
    case 0: return dispatch_mt<0>(p, smem, partials, f32, s);
    case 1: return dispatch_mt<1>(p, smem, partials, f32, s);
    default: return dispatch_mt<2>(p, smem, partials, f32, s);
    }
}

}  // namespace pfng
