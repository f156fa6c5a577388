// gemv.cu -- small-m (decode) block-quantized matmul, HBM-streaming.
//
// C[m][n] = A[m][k] . W[n][k]^T for m <= 8, W in the raw ggml layout.
// Semantics: compute_q4_0 / compute_q4_K / compute_iq2_xxs of
// bench/llama_reference/llama_reference.cpp:165-205 (dot products :113-161).
//
// Structure (one persistent CTA per SM, warp-specialised):
//   * a producer warp streams the CTA's share of the weights -- one
//     contiguous range of rows, the same number of rows for every CTA -- in
//     tiles of up to R rows (one contiguous byte range of W each) into a ring
//     of S shared-memory stages with bulk TMA copies (cp.async.bulk, mbarrier
//     transaction counts, L2 evict-first since every weight byte is read
//     once);
//   * the consumer warps first stage the activation rows in shared memory
//     (either the caller's q8 blocks, or fp32 rows quantized in place with
//     the same rounding as the standalone quantizer), then each repeatedly
//     claims the next four rows of the CTA's tile sequence (a shared
//     counter, so warps that finish early take more work) and processes
//     them: lanes walk the rows' blocks, unpack 4-bit / grid weights to
//     int8, dot them against the activations with dp4a, fold the integer
//     partials with the block scales in fp32 and reduce across the warp.
//     For q4_0 at m = 1 a warp copies its claim's four rows of weights to
//     registers and releases the stage before computing, so stages return to
//     the producer early, and reduces the four rows in one butterfly.
//   Measured on B200 (decode step of two matrices, 35 MB): 11 consumer warps
//   with 8-row (18 KB) tiles and one CTA per SM stream fastest (7.3 us per
//   step).  The CTA's 12 warps put at most 3 on each SM sub-partition, which
//   leaves 168 registers per thread for a claim's four rows in registers;
//   with 13 or more warps the cap is 128 and the four-row path spills
//   (9.1 us).  Two-row claims with 12 warps: 7.8 us; 4-row tiles: 10.5 us.
//
// q4_0 lane mapping: lane l of a warp takes the block PAIR (2l, 2l+1) of each
// group of 64 blocks.  A pair is 36 contiguous bytes = 9 aligned words at word
// offset 9l + i, so the 32 lanes hit 32 distinct banks (9 is odd): the reads
// are conflict-free and need one funnel shift per word for the even block
// only.  The activations use the same pairing, stored chunk-major so each
// 16-byte read of a warp is one contiguous 512-byte line; for m = 1 they are
// held in registers for the whole kernel.
//
// Every mbarrier wait is bounded (pfng_common.cuh): a wait that gives up
// records an error code, stops the CTA's work and returns.
#include "iq2xxs_grid_codes.h"
#include "pfng_common.cuh"
#include "pfng_internal.h"
#include "pfng_quant.cuh"

namespace pfng {
namespace {

#ifndef PFNG_GEMV_CONSUMER_WARPS
#define PFNG_GEMV_CONSUMER_WARPS 11
#endif
#ifndef PFNG_GEMV_CTAS_PER_SM
#define PFNG_GEMV_CTAS_PER_SM 1
#endif
constexpr int kConsumerWarps = PFNG_GEMV_CONSUMER_WARPS;
constexpr int kCtasPerSm = PFNG_GEMV_CTAS_PER_SM;  // 2: half the shared memory, so two launches can overlap
constexpr int kConsumerThreads = kConsumerWarps * 32;
constexpr int kGemvThreads = kConsumerThreads + 32;
#ifndef PFNG_GEMV_MAX_STAGES
#define PFNG_GEMV_MAX_STAGES 32
#endif
constexpr int kMaxStages = PFNG_GEMV_MAX_STAGES;
constexpr int kPairRows = 2;         // rows a warp processes together
#ifndef PFNG_GEMV_CLAIM_ROWS
#define PFNG_GEMV_CLAIM_ROWS 4
#endif
constexpr int kClaimRows = PFNG_GEMV_CLAIM_ROWS;  // rows a warp claims at a time (pairs of rows)
#ifndef PFNG_GEMV_CLAIM4
#define PFNG_GEMV_CLAIM4 1  // m = 1: a claim's four rows computed together
#endif
#ifndef PFNG_GEMV_FOLD2
#define PFNG_GEMV_FOLD2 1  // m = 1 four-row path: bias-started dp4a chains and packed fmas
#endif
#ifndef PFNG_GEMV_EARLY_TRIGGER
#define PFNG_GEMV_EARLY_TRIGGER 0
#endif
// Copies a CTA may keep in flight (issued, not yet landed); at least the
// ring depth means no limit beyond the ring.  Measured on B200 (decode step,
// 35 MB): 2 / 4 / 8 in flight 9.8 / 8.9 / 8.5 us per step, unlimited 7.8 --
// under a full-chip stream the loaded HBM latency is long enough that every
// tile of the ring has to be requested at once to keep HBM busy.
#ifndef PFNG_GEMV_INFLIGHT
#define PFNG_GEMV_INFLIGHT 32
#endif
constexpr int kInflight = PFNG_GEMV_INFLIGHT;
// First wave: the producer issues this many tiles, then waits for the first
// to land before issuing the rest of the ring (0: no first wave).
#ifndef PFNG_GEMV_FIRST_WAVE
#define PFNG_GEMV_FIRST_WAVE 0
#endif
constexpr int kFirstWave = PFNG_GEMV_FIRST_WAVE;
#ifndef PFNG_GEMV_TILE_ROWS
#define PFNG_GEMV_TILE_ROWS 8
#endif
constexpr int kTileRowsLong = PFNG_GEMV_TILE_ROWS;  // rows per tile when a row is >= 2 KB
static_assert(kTileRowsLong >= kClaimRows && (kTileRowsLong & (kTileRowsLong - 1)) == 0, "tile rows");
constexpr int kMaxGroup = kGemvMaxGroup;
constexpr uint32_t kBarrierBytes = 2 * kMaxStages * 8;
// iq2_xxs tables: the 256 grid points, then the byte sign masks of the 128
// sign indices, 8 bytes each, in kGridCopies bank-striped copies: entry e,
// copy c at uint2 index kGridCopies e + c, i.e. in banks 2c, 2c + 1 whatever
// e is.  Lane l reads copy l % kGridCopies, so a warp's 32 random lookups use
// every bank at most twice (the minimum for 32 x 8 bytes) instead of piling
// onto the banks of popular entries.
#ifndef PFNG_GEMV_GRID_COPIES
#define PFNG_GEMV_GRID_COPIES 16
#endif
constexpr int kGridCopies = PFNG_GEMV_GRID_COPIES;
constexpr int kSignTable = 256 * kGridCopies;  // uint2 index of the sign masks
constexpr uint32_t kGridTableBytes = (256 + 128) * kGridCopies * 8;

PFNG_DEV int grid_slot(uint32_t entry, int lane) {
    return static_cast<int>(entry) * kGridCopies + (lane & (kGridCopies - 1));
}
constexpr uint32_t kStageSlack = 32;  // bytes read past a window by aligned loads; never used
constexpr int kRegGroupsMax = 2;      // m = 1 keeps up to 2 x 64 blocks (k <= 4096) in registers

struct GemvParams {
    const uint8_t *a;  // raw q8 blocks or nullptr
    const float *x;    // fp32 activations or nullptr
    int64_t ldx;
    int32_t *partials; // count == 1: [m][n][k / 32]
    int *err;  // library error word for bounded waits
    int m, n, k;       // n: rows of matrix 0 (partials indexing)
    int x_vec;         // fp32 rows are 16-byte aligned with ldx % 4 == 0
    int row_bytes;
    int rows_per_tile;  // kClaimRows times a power of two
    int claim_shift;    // log2(rows_per_tile / kClaimRows)
    int num_tiles;      // ceil(total_rows / rows_per_tile): CTAs beyond it would be idle
    int stages;        // ring depth (any count up to kMaxStages)
    uint32_t stage_bytes;
    uint32_t grid_offset, act_offset, stage_offset;
    int groups;        // q4_0: ceil(nb / 64)
    int overlap;       // launched as a programmatic dependent (see kernel)
    // weight matrices sharing the activations (count >= 1); tiles of matrix
    // g are rows [row_base[g], row_base[g + 1]) of the launch's row sequence
    int count;
    const uint8_t *wg[kMaxGroup];
    float *cg[kMaxGroup];
    int64_t ldcg[kMaxGroup];
    int ng[kMaxGroup];
    int row_base[kMaxGroup + 1];
    int total_rows;
};

// Output of one weight matrix.
struct Out {
    float *c;
    int64_t ldc;
};

PFNG_DEV void consumer_sync() { asm volatile("bar.sync 1, %0;" ::"n"(kConsumerThreads) : "memory"); }

// dp4a with an unsigned first operand: sum of (u8 a_i) * (s8 b_i) + c.
PFNG_DEV int dp4a_us(uint32_t a, int b, int c) {
    int d;
    asm("dp4a.u32.s32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
    return d;
}

// sum over 16 weights (4 words of nibbles: low nibbles are k 0..15, high
// nibbles k 16..31 of a q4_0 block) times the activations, without the -8.
PFNG_DEV int nibble_dot(const uint32_t (&q)[4], const uint4 &alo, const uint4 &ahi, int bias = 0) {
    int lo = dp4a_us(q[0] & 0x0f0f0f0fu, static_cast<int>(alo.x), bias);
    int hi = dp4a_us(q[0] & 0xf0f0f0f0u, static_cast<int>(ahi.x), 0);
    lo = dp4a_us(q[1] & 0x0f0f0f0fu, static_cast<int>(alo.y), lo);
    hi = dp4a_us(q[1] & 0xf0f0f0f0u, static_cast<int>(ahi.y), hi);
    lo = dp4a_us(q[2] & 0x0f0f0f0fu, static_cast<int>(alo.z), lo);
    hi = dp4a_us(q[2] & 0xf0f0f0f0u, static_cast<int>(ahi.z), hi);
    lo = dp4a_us(q[3] & 0x0f0f0f0fu, static_cast<int>(alo.w), lo);
    hi = dp4a_us(q[3] & 0xf0f0f0f0u, static_cast<int>(ahi.w), hi);
    return lo + (hi >> 4);  // hi holds 16 x the high-nibble dot product exactly
}

// ---------------------------------------------------------------------------
// q4_0 activation staging: "pair-chunk" layout.
//   qs:  per row m, per group t of 64 blocks, 4 chunks x 32 lanes x 16 B;
//        block j = 64 t + 2 l + h, bytes [16 c', 16 c' + 16) of the block
//        live in chunk c = 2 h + c' at lane slot l.
//   d:   float [m][64 * groups], s8: int [m][64 * groups] (8 * sum of q).
// Blocks past nb are zero.
// ---------------------------------------------------------------------------
PFNG_DEV uint32_t q4_0_act_qs_offset(int m, int groups, int j, int byte_in_block) {
    const int t = j >> 6, l = (j >> 1) & 31, h = j & 1;
    const int c = 2 * h + (byte_in_block >> 4);
    return static_cast<uint32_t>((((m * groups + t) * 4 + c) * 32 + l) * 16 + (byte_in_block & 15));
}

// Planar-layout weights (see rows_q4_0p_reg): per row m and group t of 32
// blocks, chunk c (bytes 16 c .. 16 c + 15 of block 32 t + l) at lane slot l.
PFNG_DEV uint32_t q4_0p_act_qs_offset(int m, int groups, int j, int byte_in_block) {
    const int t = j >> 5, l = j & 31, c = byte_in_block >> 4;
    return static_cast<uint32_t>((((m * groups + t) * 2 + c) * 32 + l) * 16 + (byte_in_block & 15));
}

constexpr int kMagicBits = 0x4B400000;  // float 12582912 = 2^23 + 2^22
constexpr float kMagic = 12582912.0f;

// kPlanar: the planar layout's staging; its per-block integer is the fold
// bias 0x4B400000 - 8 * sum(q) instead of 8 * sum(q).
template <int MT, bool kF32, bool kPlanar>
PFNG_DEV void stage_act_q8_0(const GemvParams &p, uint8_t *smem, int tid) {
    const int nb = p.k / 32;
    const int nbp = p.groups * (kPlanar ? 32 : 64);
    uint8_t *qs = smem + p.act_offset;
    float *d = reinterpret_cast<float *>(qs + MT * nbp * 32);
    int32_t *s8 = reinterpret_cast<int32_t *>(d + MT * nbp);
    const int total = MT * nbp;  // a multiple of 32
    auto qs_offset = [&](int row, int j, int byte) {
        return kPlanar ? q4_0p_act_qs_offset(row, p.groups, j, byte) : q4_0_act_qs_offset(row, p.groups, j, byte);
    };
    auto aux_of = [](bool valid, int qsum) {
        return kPlanar ? (valid ? kMagicBits - 8 * qsum : kMagicBits) : (valid ? 8 * qsum : 0);
    };
    const int lane = tid & 31, warp = tid >> 5;
    if constexpr (kF32) {
        // 4 lanes per block (8 values each), 8 blocks per warp and item
        const int c = lane & 3;
        constexpr int kBatch = 2;  // items whose loads are issued together
        for (int wb0 = warp * 8; wb0 < total; wb0 += kBatch * kConsumerWarps * 8) {
            float v[kBatch][8];
#pragma unroll
            for (int it = 0; it < kBatch; ++it) {
                const int bi = wb0 + it * kConsumerWarps * 8 + (lane >> 2);
                const int row = bi / nbp, j = bi % nbp;
#pragma unroll
                for (int i = 0; i < 8; ++i) v[it][i] = 0.0f;
                if (bi < total && row < p.m && j < nb) {
                    const float *src = p.x + row * p.ldx + j * 32 + 8 * c;
                    if (p.x_vec) {
                        const float4 t0 = __ldg(reinterpret_cast<const float4 *>(src));
                        const float4 t1 = __ldg(reinterpret_cast<const float4 *>(src + 4));
                        v[it][0] = t0.x, v[it][1] = t0.y, v[it][2] = t0.z, v[it][3] = t0.w;
                        v[it][4] = t1.x, v[it][5] = t1.y, v[it][6] = t1.z, v[it][7] = t1.w;
                    } else {
#pragma unroll
                        for (int i = 0; i < 8; ++i) v[it][i] = __ldg(src + i);
                    }
                }
            }
            Q8_0Quad qr[kBatch];
            q8_0_quantize_quads<kBatch>(v, qr);
#pragma unroll
            for (int it = 0; it < kBatch; ++it) {
                const int wb = wb0 + it * kConsumerWarps * 8;
                if (wb >= total) break;
                const int bi = wb + (lane >> 2);
                const int row = bi / nbp, j = bi % nbp;
                const bool valid = row < p.m && j < nb;
                *reinterpret_cast<uint2 *>(qs + qs_offset(row, j, 8 * c)) =
                    valid ? make_uint2(qr[it].q0, qr[it].q1) : make_uint2(0u, 0u);
                if (c == 0) {
                    d[row * nbp + j] = valid ? f16_bits_to_f32(qr[it].dbits) : 0.0f;
                    s8[row * nbp + j] = aux_of(valid, qr[it].qsum);
                }
            }
        }
    } else {
        // caller's q8_0 blocks: 8 lanes per block (4 bytes each)
        const int g = lane & 7;
        constexpr int kBatch = 4;
        for (int wb0 = warp * 4; wb0 < total; wb0 += kBatch * kConsumerWarps * 4) {
            uint32_t raw_q[kBatch], raw_d[kBatch];
#pragma unroll
            for (int it = 0; it < kBatch; ++it) {
                const int wb = wb0 + it * kConsumerWarps * 4;
                const int bi = wb + (lane >> 3);
                const int row = bi / nbp, j = bi % nbp;
                raw_q[it] = raw_d[it] = 0;
                if (wb < total && row < p.m && j < nb) {
                    const uint8_t *blk = p.a + (static_cast<int64_t>(row) * nb + j) * kQ8_0Bytes;
                    const uint16_t *h = reinterpret_cast<const uint16_t *>(blk + 2 + 4 * g);
                    raw_q[it] = static_cast<uint32_t>(__ldg(h)) | (static_cast<uint32_t>(__ldg(h + 1)) << 16);
                    raw_d[it] = __ldg(reinterpret_cast<const uint16_t *>(blk));
                }
            }
#pragma unroll
            for (int it = 0; it < kBatch; ++it) {
                const int wb = wb0 + it * kConsumerWarps * 4;
                if (wb >= total) break;
                const int bi = wb + (lane >> 3);
                const int row = bi / nbp, j = bi % nbp;
                const bool valid = row < p.m && j < nb;
                const uint32_t q = raw_q[it];
                int sm = __dp4a(static_cast<int>(q), 0x01010101, 0);
#pragma unroll
                for (int o = 1; o < 8; o <<= 1) sm += __shfl_xor_sync(0xffffffffu, sm, o);
                *reinterpret_cast<uint32_t *>(qs + qs_offset(row, j, 4 * g)) = valid ? q : 0u;
                if (g == 0) {
                    d[row * nbp + j] = valid ? f16_bits_to_f32(raw_d[it]) : 0.0f;
                    s8[row * nbp + j] = aux_of(valid, sm);
                }
            }
        }
    }
}

// q8_K activations (q4_K, iq2_xxs): qs [MT][k], d [MT][k/256], bsums [MT][k/16].
template <int MT, bool kF32>
PFNG_DEV void stage_act_q8_K(const GemvParams &p, uint8_t *smem, int tid) {
    const int nb = p.k / 256;
    int8_t *qs = reinterpret_cast<int8_t *>(smem + p.act_offset);
    float *d = reinterpret_cast<float *>(qs + MT * p.k);
    int16_t *bs = reinterpret_cast<int16_t *>(d + MT * nb);
    const int total = MT * nb;
    const int lane = tid & 31, warp = tid >> 5;
    constexpr int kBatch = 2;  // blocks whose loads are issued together
    for (int bi0 = warp; bi0 < total; bi0 += kBatch * kConsumerWarps) {
        float v[kBatch][8];
        uint32_t q0[kBatch], q1[kBatch];
        float dv[kBatch];
        int bsum[kBatch];
#pragma unroll
        for (int it = 0; it < kBatch; ++it) {
            const int bi = bi0 + it * kConsumerWarps;
            const int row = bi / nb, col = bi % nb;
            const bool valid = bi < total && row < p.m;
#pragma unroll
            for (int i = 0; i < 8; ++i) v[it][i] = 0.0f;
            q0[it] = q1[it] = 0;
            dv[it] = 0.0f;
            bsum[it] = 0;
            if (!valid) continue;
            if constexpr (kF32) {
                const float *src = p.x + row * p.ldx + col * 256 + 8 * lane;
                if (p.x_vec) {
                    const float4 t0 = __ldg(reinterpret_cast<const float4 *>(src));
                    const float4 t1 = __ldg(reinterpret_cast<const float4 *>(src + 4));
                    v[it][0] = t0.x, v[it][1] = t0.y, v[it][2] = t0.z, v[it][3] = t0.w;
                    v[it][4] = t1.x, v[it][5] = t1.y, v[it][6] = t1.z, v[it][7] = t1.w;
                } else {
#pragma unroll
                    for (int i = 0; i < 8; ++i) v[it][i] = __ldg(src + i);
                }
            } else {
                const uint8_t *blk = p.a + (static_cast<int64_t>(row) * nb + col) * kQ8_KBytes;
                const uint32_t *q = reinterpret_cast<const uint32_t *>(blk + kQ8_KQsOffset + 8 * lane);
                q0[it] = __ldg(q);
                q1[it] = __ldg(q + 1);
                dv[it] = __ldg(reinterpret_cast<const float *>(blk));
                if (lane < 16) bsum[it] = __ldg(reinterpret_cast<const int16_t *>(blk + kQ8_KBsumsOffset) + lane);
            }
        }
#pragma unroll
        for (int it = 0; it < kBatch; ++it) {
            const int bi = bi0 + it * kConsumerWarps;
            if (bi >= total) break;
            const int row = bi / nb, col = bi % nb;
            const bool valid = row < p.m;
            if constexpr (kF32) {
                const Q8_KLane r = q8_K_quantize_lane(v[it]);
                q0[it] = r.q0;
                q1[it] = r.q1;
                dv[it] = r.d;
                // bsums entry j lives in lanes 2j and 2j+1
                bsum[it] = __shfl_sync(0xffffffffu, r.sum16, (2 * lane) & 31);
            }
            uint32_t *dst = reinterpret_cast<uint32_t *>(qs + row * p.k + col * 256 + 8 * lane);
            dst[0] = q0[it];
            dst[1] = q1[it];
            if (lane < 16) bs[row * (p.k / 16) + col * 16 + lane] = static_cast<int16_t>(valid ? bsum[it] : 0);
            if (lane == 0) d[row * nb + col] = valid ? dv[it] : 0.0f;
        }
    }
}

// --------------------------------------------------------------------------
// per-row dot products.  `tile` is the stage buffer, `row_off` the byte
// offset of the row inside it.  Loops are warp-uniform (shuffles inside).
// --------------------------------------------------------------------------
template <int MT>
PFNG_DEV void warp_reduce_store(const GemvParams &p, const Out &o, float (&acc)[MT], int row, int lane) {
#pragma unroll
    for (int mi = 0; mi < MT; ++mi) {
        float v = acc[mi];
#pragma unroll
        for (int sh = 16; sh > 0; sh >>= 1) v += __shfl_xor_sync(0xffffffffu, v, sh);
        if (lane == 0 && mi < p.m) o.c[mi * o.ldc + row] = v;
    }
}

// Activations of one lane for the m = 1 register path.
template <int GM>
struct ActRegs {
    uint4 q[GM][4];   // chunks 0..3 of the lane's block pair in each group
    float2 d[GM];
    int2 s8[GM];
};

// Weights of one lane's block pair: 36 bytes at a 4-aligned offset.
struct PairW {
    uint32_t qa[4], qb[4];
    float da, db;
};

PFNG_DEV PairW load_pair(const uint8_t *tile, uint32_t off) {
    const uint32_t *w = reinterpret_cast<const uint32_t *>(tile + off);
    uint32_t v[9];
#pragma unroll
    for (int i = 0; i < 9; ++i) v[i] = w[i];
    PairW r;
#pragma unroll
    for (int i = 0; i < 4; ++i) r.qa[i] = __funnelshift_r(v[i], v[i + 1], 16);
#pragma unroll
    for (int i = 0; i < 4; ++i) r.qb[i] = v[5 + i];
    r.da = f16_bits_to_f32(v[0] & 0xffffu);
    r.db = f16_bits_to_f32(v[4] >> 16);
    return r;
}

// m = 1, activations in registers (groups <= GM).  Rows row0 and row0 + 1
// (the second only if nrows == 2) start at row_off and row_off + row_bytes.
// The weights are first copied to registers (load_rows_q4_0) so that the
// stage can be handed back to the producer before the arithmetic.
template <int GM>
struct RowsW {
    PairW w[GM][2];
};

template <int GM>
PFNG_DEV void load_rows_q4_0(const GemvParams &p, const uint8_t *tile, uint32_t row_off, int nrows, int lane,
                             RowsW<GM> &rw) {
    const int nb = p.k / 32;
    const uint32_t off1 = row_off + static_cast<uint32_t>(nrows > 1 ? p.row_bytes : 0);
#pragma unroll
    for (int t = 0; t < GM; ++t) {
        if (t < p.groups && 64 * t + 2 * lane < nb) {
            const uint32_t o = 1152u * t + 36u * lane;
            rw.w[t][0] = load_pair(tile, row_off + o);
            rw.w[t][1] = load_pair(tile, off1 + o);
        }
    }
}

template <int GM, bool kPartials>
PFNG_DEV void rows_q4_0_reg(const GemvParams &p, const Out &o, const ActRegs<GM> &ar, const RowsW<GM> &rw, int row0,
                            int nrows, int lane) {
    const int nb = p.k / 32;
    float acc0 = 0.0f, acc1 = 0.0f;
#pragma unroll
    for (int t = 0; t < GM; ++t) {
        if (t < p.groups && 64 * t + 2 * lane < nb) {
            const PairW &w0 = rw.w[t][0], &w1 = rw.w[t][1];
            const int ia0 = nibble_dot(w0.qa, ar.q[t][0], ar.q[t][1]) - ar.s8[t].x;
            const int ia1 = nibble_dot(w1.qa, ar.q[t][0], ar.q[t][1]) - ar.s8[t].x;
            const int ib0 = nibble_dot(w0.qb, ar.q[t][2], ar.q[t][3]) - ar.s8[t].y;
            const int ib1 = nibble_dot(w1.qb, ar.q[t][2], ar.q[t][3]) - ar.s8[t].y;
            if constexpr (kPartials) {
                const int j = 64 * t + 2 * lane;
                int32_t *out = p.partials + static_cast<int64_t>(row0) * nb + j;
                out[0] = ia0;
                out[1] = ib0;
                if (nrows > 1) {
                    out[nb] = ia1;
                    out[nb + 1] = ib1;
                }
            } else {
                acc0 = __fmaf_rn(__fmul_rn(static_cast<float>(ia0), w0.da), ar.d[t].x, acc0);
                acc1 = __fmaf_rn(__fmul_rn(static_cast<float>(ia1), w1.da), ar.d[t].x, acc1);
                acc0 = __fmaf_rn(__fmul_rn(static_cast<float>(ib0), w0.db), ar.d[t].y, acc0);
                acc1 = __fmaf_rn(__fmul_rn(static_cast<float>(ib1), w1.db), ar.d[t].y, acc1);
            }
        }
    }
    if constexpr (!kPartials) {
        // two rows in one butterfly: the first exchange leaves row 0's sums
        // in lanes 0..15 and row 1's in lanes 16..31
        const bool upper = (lane & 16) != 0;
        float v = (upper ? acc1 : acc0) + __shfl_xor_sync(0xffffffffu, upper ? acc0 : acc1, 16);
#pragma unroll
        for (int sh = 8; sh > 0; sh >>= 1) v += __shfl_xor_sync(0xffffffffu, v, sh);
        if (lane == 0) o.c[row0] = v;
        if (lane == 16 && nrows > 1) o.c[row0 + 1] = v;
    }
}

// Sum four rows' lane partials across the warp and store them (rows beyond
// nrows are not stored).  The first exchange splits rows {0, 1} / {2, 3}
// between the half-warps, the second rows 0 / 1 (2 / 3) between lane
// octets; each row's partials meet in the same tree as in a pair's or a
// single row's butterfly.
PFNG_DEV void reduce_store4(const Out &o, float a0, float a1, float a2, float a3, int row0, int nrows, int lane) {
    const bool up = (lane & 16) != 0, b8 = (lane & 8) != 0;
    const float v0 = (up ? a2 : a0) + __shfl_xor_sync(0xffffffffu, up ? a0 : a2, 16);
    const float v1 = (up ? a3 : a1) + __shfl_xor_sync(0xffffffffu, up ? a1 : a3, 16);
    float v = (b8 ? v1 : v0) + __shfl_xor_sync(0xffffffffu, b8 ? v0 : v1, 8);
#pragma unroll
    for (int sh = 4; sh > 0; sh >>= 1) v += __shfl_xor_sync(0xffffffffu, v, sh);
    // lane 0: row 0, lane 8: row 1, lane 16: row 2, lane 24: row 3
    const int r = (up ? 2 : 0) + (b8 ? 1 : 0);
    if ((lane & 7) == 0 && r < nrows) o.c[row0 + r] = v;
}

// m = 1, four rows (a whole claim): rows 0, 1 in r01 and 2, 3 in r23.  More
// independent dot-product chains than a pair, and one transposed butterfly
// for the four sums: the first exchange splits rows {0, 1} / {2, 3} between
// the half-warps, the second rows 0 / 1 (2 / 3) between lane octets.  Every
// row's lane sums meet in the same tree as in rows_q4_0_reg, so the results
// are bit-identical to processing the claim as two pairs.
template <int GM>
PFNG_DEV void rows4_q4_0_reg(const GemvParams &p, const Out &o, const ActRegs<GM> &ar, const RowsW<GM> &r01,
                             const RowsW<GM> &r23, int row0, int nrows, int lane) {
    const int nb = p.k / 32;
    float acc[4] = {0.0f, 0.0f, 0.0f, 0.0f};
#pragma unroll
    for (int t = 0; t < GM; ++t) {
        if (t < p.groups && 64 * t + 2 * lane < nb) {
#pragma unroll
            for (int r = 0; r < 4; ++r) {
                const PairW &w = r < 2 ? r01.w[t][r] : r23.w[t][r - 2];
                const int ia = nibble_dot(w.qa, ar.q[t][0], ar.q[t][1]) - ar.s8[t].x;
                const int ib = nibble_dot(w.qb, ar.q[t][2], ar.q[t][3]) - ar.s8[t].y;
                acc[r] = __fmaf_rn(__fmul_rn(static_cast<float>(ia), w.da), ar.d[t].x, acc[r]);
                acc[r] = __fmaf_rn(__fmul_rn(static_cast<float>(ib), w.db), ar.d[t].y, acc[r]);
            }
        }
    }
    reduce_store4(o, acc[0], acc[1], acc[2], acc[3], row0, nrows, lane);
}

// any m <= 8, activations in shared memory; two rows as above.
template <int MT, bool kPartials>
PFNG_DEV void rows_q4_0_smem(const GemvParams &p, const Out &o, const uint8_t *act, const uint8_t *tile,
                             uint32_t row_off, int row0, int nrows, int lane) {
    const int nb = p.k / 32;
    const int nbp = p.groups * 64;
    const float *ad = reinterpret_cast<const float *>(act + MT * p.groups * 2048);
    const int32_t *as8 = reinterpret_cast<const int32_t *>(ad + MT * nbp);
    const uint32_t off1 = row_off + static_cast<uint32_t>(nrows > 1 ? p.row_bytes : 0);
    float acc0[MT], acc1[MT];
#pragma unroll
    for (int mi = 0; mi < MT; ++mi) acc0[mi] = 0.0f, acc1[mi] = 0.0f;
    for (int t = 0; t < p.groups; ++t) {
        if (64 * t + 2 * lane >= nb) continue;
        const uint32_t o = 1152u * t + 36u * lane;
        const PairW w0 = load_pair(tile, row_off + o);
        const PairW w1 = load_pair(tile, off1 + o);
        const int j = 64 * t + 2 * lane;
#pragma unroll
        for (int mi = 0; mi < MT; ++mi) {
            const uint4 *aq = reinterpret_cast<const uint4 *>(act + ((mi * p.groups + t) * 4) * 512) + lane;
            const uint4 c0 = aq[0], c1 = aq[32], c2 = aq[64], c3 = aq[96];
            const float2 da = *reinterpret_cast<const float2 *>(ad + mi * nbp + j);
            const int2 s8 = *reinterpret_cast<const int2 *>(as8 + mi * nbp + j);
            const int ia0 = nibble_dot(w0.qa, c0, c1) - s8.x;
            const int ia1 = nibble_dot(w1.qa, c0, c1) - s8.x;
            const int ib0 = nibble_dot(w0.qb, c2, c3) - s8.y;
            const int ib1 = nibble_dot(w1.qb, c2, c3) - s8.y;
            if constexpr (kPartials) {
                if (mi < p.m) {
                    int32_t *out = p.partials + (static_cast<int64_t>(mi) * p.n + row0) * nb + j;
                    out[0] = ia0;
                    out[1] = ib0;
                    if (nrows > 1) {
                        out[nb] = ia1;
                        out[nb + 1] = ib1;
                    }
                }
            } else {
                acc0[mi] = __fmaf_rn(__fmul_rn(static_cast<float>(ia0), w0.da), da.x, acc0[mi]);
                acc1[mi] = __fmaf_rn(__fmul_rn(static_cast<float>(ia1), w1.da), da.x, acc1[mi]);
                acc0[mi] = __fmaf_rn(__fmul_rn(static_cast<float>(ib0), w0.db), da.y, acc0[mi]);
                acc1[mi] = __fmaf_rn(__fmul_rn(static_cast<float>(ib1), w1.db), da.y, acc1[mi]);
            }
        }
    }
    if constexpr (!kPartials) {
        warp_reduce_store<MT>(p, o, acc0, row0, lane);
        if (nrows > 1) warp_reduce_store<MT>(p, o, acc1, row0 + 1, lane);
    }
}

// ---------------------------------------------------------------------------
// q4_0 in the planar row layout (pfng_b200_pack_q4_0_planar): a row of nb
// blocks holds the 16-byte nibble fields of blocks 0..nb-1 (block j at byte
// 16 j), then their fp16 scales (block j at byte 16 nb + 2 j) -- 18 nb bytes
// as in the ggml layout, with rows 16-byte aligned (nb % 8 == 0).  Lane l
// takes blocks j = 32 t + l: one 16-byte read per block, and a warp's reads
// of one t are 512 contiguous bytes (conflict-free, no funnel shifts).
// Fold without an int -> float conversion: the low-nibble dp4a chain starts
// at the bias 0x4B400000 - 8 sum(q), so the chain's end y, read as a float,
// is 2^23 + 2^22 + P exactly (|P| < 2^22), and
//   t = fma(y, d_w, -(2^23 + 2^22) d_w) = round(P d_w)
// (the product (2^23 + 2^22) d_w is exact: d_w has 11 significant bits) --
// the same value as float(P) * d_w; then acc = fma(t, d_a, acc).  Two rows
// share each packed fma.rn.f32x2.
// ---------------------------------------------------------------------------
// Activations of one lane for the m = 1 register path, GT groups of 32 blocks.
template <int GT>
struct ActRegsP {
    uint4 lo[GT], hi[GT];  // bytes 0..15 and 16..31 of the lane's block 32 t + l
    float d[GT];
    int bias[GT];          // 0x4B400000 - 8 * sum(q)
};

// Weights of one row pair for the lane's blocks.
template <int GT>
struct RowsWP {
    uint4 q[GT][2];  // nibbles, rows 0 and 1
    uint32_t d[GT];  // fp16 scales: row 0 in the low half, row 1 in the high half
};

// sum over the block of nibble * a, plus the bias
PFNG_DEV int nibble_dot_biased(const uint4 &q, const uint4 &alo, const uint4 &ahi, int bias) {
    int lo = dp4a_us(q.x & 0x0f0f0f0fu, static_cast<int>(alo.x), bias);
    int hi = dp4a_us(q.x & 0xf0f0f0f0u, static_cast<int>(ahi.x), 0);
    lo = dp4a_us(q.y & 0x0f0f0f0fu, static_cast<int>(alo.y), lo);
    hi = dp4a_us(q.y & 0xf0f0f0f0u, static_cast<int>(ahi.y), hi);
    lo = dp4a_us(q.z & 0x0f0f0f0fu, static_cast<int>(alo.z), lo);
    hi = dp4a_us(q.z & 0xf0f0f0f0u, static_cast<int>(ahi.z), hi);
    lo = dp4a_us(q.w & 0x0f0f0f0fu, static_cast<int>(alo.w), lo);
    hi = dp4a_us(q.w & 0xf0f0f0f0u, static_cast<int>(ahi.w), hi);
    return lo + (hi >> 4);  // hi holds 16 x the high-nibble dot product exactly
}

PFNG_DEV float2 f16x2_bits_to_f32x2(uint32_t h) {
    return __half22float2(__halves2half2(__ushort_as_half(static_cast<unsigned short>(h & 0xffffu)),
                                         __ushort_as_half(static_cast<unsigned short>(h >> 16))));
}

// Fold of one block for two rows: y01 are the biased dot products.
PFNG_DEV float2 fold_pair(int y0, int y1, float2 dw, float da, float2 acc) {
    const float2 nm = __fmul2_rn(dw, make_float2(-kMagic, -kMagic));
    const float2 t = __ffma2_rn(make_float2(__int_as_float(y0), __int_as_float(y1)), dw, nm);
    return __ffma2_rn(t, make_float2(da, da), acc);
}

// rows4_q4_0_reg with the fold above: the low-nibble chain starts at the
// bias 0x4B400000 - 8 sum(q) and rows (0, 1) / (2, 3) share packed fmas.
// Same values as rows4_q4_0_reg (round(P d_w) either way).
template <int GM>
PFNG_DEV void rows4_q4_0_reg_f2(const GemvParams &p, const Out &o, const ActRegs<GM> &ar, const RowsW<GM> &r01,
                                const RowsW<GM> &r23, int row0, int nrows, int lane) {
    const int nb = p.k / 32;
    float2 acc01 = make_float2(0.0f, 0.0f), acc23 = make_float2(0.0f, 0.0f);
#pragma unroll
    for (int t = 0; t < GM; ++t) {
        if (t < p.groups && 64 * t + 2 * lane < nb) {
            const int ba = kMagicBits - ar.s8[t].x, bb = kMagicBits - ar.s8[t].y;
            const PairW &w0 = r01.w[t][0], &w1 = r01.w[t][1], &w2 = r23.w[t][0], &w3 = r23.w[t][1];
            const int y0a = nibble_dot(w0.qa, ar.q[t][0], ar.q[t][1], ba);
            const int y1a = nibble_dot(w1.qa, ar.q[t][0], ar.q[t][1], ba);
            const int y2a = nibble_dot(w2.qa, ar.q[t][0], ar.q[t][1], ba);
            const int y3a = nibble_dot(w3.qa, ar.q[t][0], ar.q[t][1], ba);
            const int y0b = nibble_dot(w0.qb, ar.q[t][2], ar.q[t][3], bb);
            const int y1b = nibble_dot(w1.qb, ar.q[t][2], ar.q[t][3], bb);
            const int y2b = nibble_dot(w2.qb, ar.q[t][2], ar.q[t][3], bb);
            const int y3b = nibble_dot(w3.qb, ar.q[t][2], ar.q[t][3], bb);
            acc01 = fold_pair(y0a, y1a, make_float2(w0.da, w1.da), ar.d[t].x, acc01);
            acc23 = fold_pair(y2a, y3a, make_float2(w2.da, w3.da), ar.d[t].x, acc23);
            acc01 = fold_pair(y0b, y1b, make_float2(w0.db, w1.db), ar.d[t].y, acc01);
            acc23 = fold_pair(y2b, y3b, make_float2(w2.db, w3.db), ar.d[t].y, acc23);
        }
    }
    reduce_store4(o, acc01.x, acc01.y, acc23.x, acc23.y, row0, nrows, lane);
}

template <int GT>
PFNG_DEV void load_rows_q4_0p(const GemvParams &p, const uint8_t *tile, uint32_t row_off, int nrows, int lane,
                              RowsWP<GT> &rw) {
    const int nb = p.k / 32;
    const uint32_t off1 = row_off + static_cast<uint32_t>(nrows > 1 ? p.row_bytes : 0);
    const uint32_t dplane = 16u * static_cast<uint32_t>(nb);
#pragma unroll
    for (int t = 0; t < GT; ++t) {
        const int j = 32 * t + lane;
        if (t < p.groups && j < nb) {
            rw.q[t][0] = *reinterpret_cast<const uint4 *>(tile + row_off + 16u * j);
            rw.q[t][1] = *reinterpret_cast<const uint4 *>(tile + off1 + 16u * j);
            const uint32_t d0 = *reinterpret_cast<const uint16_t *>(tile + row_off + dplane + 2u * j);
            const uint32_t d1 = *reinterpret_cast<const uint16_t *>(tile + off1 + dplane + 2u * j);
            rw.d[t] = d0 | (d1 << 16);
        }
    }
}

// Reduce the two rows' lane sums in one butterfly and store them.
PFNG_DEV void reduce_store_pair(const Out &o, float2 acc, int row0, int nrows, int lane) {
    // the first exchange leaves row 0's sums in lanes 0..15 and row 1's in 16..31
    const bool upper = (lane & 16) != 0;
    float v = (upper ? acc.y : acc.x) + __shfl_xor_sync(0xffffffffu, upper ? acc.x : acc.y, 16);
#pragma unroll
    for (int sh = 8; sh > 0; sh >>= 1) v += __shfl_xor_sync(0xffffffffu, v, sh);
    if (lane == 0) o.c[row0] = v;
    if (lane == 16 && nrows > 1) o.c[row0 + 1] = v;
}

template <int GT, bool kPartials>
PFNG_DEV void rows_q4_0p_reg(const GemvParams &p, const Out &o, const ActRegsP<GT> &ar, const RowsWP<GT> &rw,
                             int row0, int nrows, int lane) {
    const int nb = p.k / 32;
    float2 acc = make_float2(0.0f, 0.0f);
#pragma unroll
    for (int t = 0; t < GT; ++t) {
        const int j = 32 * t + lane;
        if (t < p.groups && j < nb) {
            const int y0 = nibble_dot_biased(rw.q[t][0], ar.lo[t], ar.hi[t], ar.bias[t]);
            const int y1 = nibble_dot_biased(rw.q[t][1], ar.lo[t], ar.hi[t], ar.bias[t]);
            if constexpr (kPartials) {
                int32_t *out = p.partials + static_cast<int64_t>(row0) * nb + j;
                out[0] = y0 - kMagicBits;
                if (nrows > 1) out[nb] = y1 - kMagicBits;
            } else {
                acc = fold_pair(y0, y1, f16x2_bits_to_f32x2(rw.d[t]), ar.d[t], acc);
            }
        }
    }
    if constexpr (!kPartials) reduce_store_pair(o, acc, row0, nrows, lane);
}

// m = 1, four rows (a whole claim), planar layout: rows 0, 1 in r01 and
// 2, 3 in r23.
template <int GT>
PFNG_DEV void rows4_q4_0p_reg(const GemvParams &p, const Out &o, const ActRegsP<GT> &ar, const RowsWP<GT> &r01,
                              const RowsWP<GT> &r23, int row0, int nrows, int lane) {
    const int nb = p.k / 32;
    float2 acc01 = make_float2(0.0f, 0.0f), acc23 = make_float2(0.0f, 0.0f);
#pragma unroll
    for (int t = 0; t < GT; ++t) {
        const int j = 32 * t + lane;
        if (t < p.groups && j < nb) {
            const int y0 = nibble_dot_biased(r01.q[t][0], ar.lo[t], ar.hi[t], ar.bias[t]);
            const int y1 = nibble_dot_biased(r01.q[t][1], ar.lo[t], ar.hi[t], ar.bias[t]);
            const int y2 = nibble_dot_biased(r23.q[t][0], ar.lo[t], ar.hi[t], ar.bias[t]);
            const int y3 = nibble_dot_biased(r23.q[t][1], ar.lo[t], ar.hi[t], ar.bias[t]);
            acc01 = fold_pair(y0, y1, f16x2_bits_to_f32x2(r01.d[t]), ar.d[t], acc01);
            acc23 = fold_pair(y2, y3, f16x2_bits_to_f32x2(r23.d[t]), ar.d[t], acc23);
        }
    }
    reduce_store4(o, acc01.x, acc01.y, acc23.x, acc23.y, row0, nrows, lane);
}

// any m <= 8, activations in shared memory; two rows as above.
template <int MT, bool kPartials>
PFNG_DEV void rows_q4_0p_smem(const GemvParams &p, const Out &o, const uint8_t *act, const uint8_t *tile,
                              uint32_t row_off, int row0, int nrows, int lane) {
    const int nb = p.k / 32;
    const int nbp = p.groups * 32;
    const float *ad = reinterpret_cast<const float *>(act + MT * nbp * 32);
    const int32_t *abias = reinterpret_cast<const int32_t *>(ad + MT * nbp);
    const uint32_t off1 = row_off + static_cast<uint32_t>(nrows > 1 ? p.row_bytes : 0);
    const uint32_t dplane = 16u * static_cast<uint32_t>(nb);
    float2 acc[MT];
#pragma unroll
    for (int mi = 0; mi < MT; ++mi) acc[mi] = make_float2(0.0f, 0.0f);
    for (int t = 0; t < p.groups; ++t) {
        const int j = 32 * t + lane;
        if (j >= nb) break;
        const uint4 q0 = *reinterpret_cast<const uint4 *>(tile + row_off + 16u * j);
        const uint4 q1 = *reinterpret_cast<const uint4 *>(tile + off1 + 16u * j);
        const uint32_t d0 = *reinterpret_cast<const uint16_t *>(tile + row_off + dplane + 2u * j);
        const uint32_t d1 = *reinterpret_cast<const uint16_t *>(tile + off1 + dplane + 2u * j);
        const float2 dw = f16x2_bits_to_f32x2(d0 | (d1 << 16));
#pragma unroll
        for (int mi = 0; mi < MT; ++mi) {
            const uint4 *aq = reinterpret_cast<const uint4 *>(act + (mi * p.groups + t) * 1024) + lane;
            const uint4 alo = aq[0], ahi = aq[32];
            const int bias = abias[mi * nbp + j];
            const int y0 = nibble_dot_biased(q0, alo, ahi, bias);
            const int y1 = nibble_dot_biased(q1, alo, ahi, bias);
            if constexpr (kPartials) {
                if (mi < p.m) {
                    int32_t *out = p.partials + (static_cast<int64_t>(mi) * p.n + row0) * nb + j;
                    out[0] = y0 - kMagicBits;
                    if (nrows > 1) out[nb] = y1 - kMagicBits;
                }
            } else {
                acc[mi] = fold_pair(y0, y1, dw, ad[mi * nbp + j], acc[mi]);
            }
        }
    }
    if constexpr (!kPartials) {
        float acc0[MT], acc1[MT];
#pragma unroll
        for (int mi = 0; mi < MT; ++mi) acc0[mi] = acc[mi].x, acc1[mi] = acc[mi].y;
        warp_reduce_store<MT>(p, o, acc0, row0, lane);
        if (nrows > 1) warp_reduce_store<MT>(p, o, acc1, row0 + 1, lane);
    }
}

// ---------------------------------------------------------------------------
// q4_K, m = 1, k <= 4096: activations in registers.  Lane l of iteration i
// takes the unit (block b = 8 i + l / 4, nibble pair pr = l & 3): the 32
// nibble bytes at 16 + 32 pr of the block, whose low nibbles are sub-block
// 2 pr and high nibbles sub-block 2 pr + 1.  A warp's units of one iteration
// cover eight whole blocks (16-byte reads, 4 lanes per 16-byte bank slot).
// Same integer sums as row_q4_K; the min term sum_j m_j * bsum_j of the two
// sub-blocks is one dp2a over the packed mins and sub-block sums.
// ---------------------------------------------------------------------------
template <int NI>
struct ActRegsK {
    uint4 a0[NI][2];  // 32 activations of sub-block 2 pr
    uint4 a1[NI][2];  // 32 activations of sub-block 2 pr + 1
    float d[NI];      // the block's activation scale
    int bs[NI];       // sums of the two sub-blocks' activations, two int16
};

// Weights of one row's units: the block header (d, dmin, 12 scale bytes) and
// the unit's 32 nibble bytes.
template <int NI, int R = 2>
struct RowsWK {
    uint4 hd[NI][R];    // [.][row]
    uint4 q[NI][R][2];  // [.][row][half]
};

template <int NI>
PFNG_DEV void load_act_q4_K(const GemvParams &p, const uint8_t *act, int lane, ActRegsK<NI> &ar) {
    const int nbk = p.k / 256;
    const int8_t *aqs = reinterpret_cast<const int8_t *>(act);
    const float *ad = reinterpret_cast<const float *>(aqs + p.k);
    const int16_t *abs16 = reinterpret_cast<const int16_t *>(ad + nbk);
    const int pr = lane & 3;
#pragma unroll
    for (int i = 0; i < NI; ++i) {
        const int b = 8 * i + (lane >> 2);
        if (b < nbk) {
            const uint4 *a = reinterpret_cast<const uint4 *>(aqs + b * 256 + 64 * pr);
            ar.a0[i][0] = a[0], ar.a0[i][1] = a[1], ar.a1[i][0] = a[2], ar.a1[i][1] = a[3];
            ar.d[i] = ad[b];
            const int16_t *bs = abs16 + b * 16 + 4 * pr;
            const int s0 = bs[0] + bs[1], s1 = bs[2] + bs[3];
            ar.bs[i] = static_cast<int>((static_cast<uint32_t>(s0) & 0xffffu) | (static_cast<uint32_t>(s1) << 16));
        } else {
            ar.a0[i][0] = ar.a0[i][1] = ar.a1[i][0] = ar.a1[i][1] = make_uint4(0, 0, 0, 0);
            ar.d[i] = 0.0f;
            ar.bs[i] = 0;
        }
    }
}

// R rows from row_off on; rows at or past nrows repeat the last valid row
// (loaded, never stored).
template <int NI, int R>
PFNG_DEV void load_rows_q4_K(const GemvParams &p, const uint8_t *tile, uint32_t row_off, int nrows, int lane,
                             RowsWK<NI, R> &rw) {
    const int nbk = p.k / 256;
    const int pr = lane & 3;
#pragma unroll
    for (int i = 0; i < NI; ++i) {
        const int b = 8 * i + (lane >> 2);
        if (b < nbk) {
#pragma unroll
            for (int r = 0; r < R; ++r) {
                const int rr = r < nrows ? r : nrows - 1;
                const uint8_t *blk = tile + row_off + static_cast<uint32_t>(rr * p.row_bytes) + 144u * b;
                rw.hd[i][r] = *reinterpret_cast<const uint4 *>(blk);
                rw.q[i][r][0] = *reinterpret_cast<const uint4 *>(blk + 16 + 32 * pr);
                rw.q[i][r][1] = *reinterpret_cast<const uint4 *>(blk + 32 + 32 * pr);
            }
        }
    }
}

// 6-bit scales and mins of sub-blocks 2 pr and 2 pr + 1 (llama_reference.cpp
// :116-121), two bytes each: hd.y, hd.z, hd.w are scale bytes 0-3, 4-7, 8-11.
// For pr < 2: sc = q[j] & 63, m = q[j + 4] & 63; otherwise
// sc = (q[j + 4] & 15) | (q[j - 4] >> 6) << 4, m = q[j + 4] >> 4 | (q[j] >> 6) << 4.
PFNG_DEV void q4_K_scales_pair(const uint4 &hd, int pr, uint32_t &scpk, uint32_t &mpk) {
    const bool lo = pr < 2;
    const uint32_t sh = (pr & 1) * 16;
    const uint32_t xa_sc = ((lo ? hd.y : hd.w) >> sh) & 0xffffu;
    const uint32_t xa_m = ((lo ? hd.z : hd.w) >> sh) & 0xffffu;
    const uint32_t xb_sc = (hd.y >> sh) & 0xffffu, xb_m = (hd.z >> sh) & 0xffffu;
    scpk = lo ? (xa_sc & 0x3f3fu) : ((xa_sc & 0x0f0fu) | ((xb_sc >> 2) & 0x3030u));
    mpk = lo ? (xa_m & 0x3f3fu) : (((xa_m >> 4) & 0x0f0fu) | ((xb_m >> 2) & 0x3030u));
}

template <int NI, int R, bool kPartials>
PFNG_DEV void rows_q4_K_reg(const GemvParams &p, const Out &o, const ActRegsK<NI> &ar, const RowsWK<NI, R> &rw,
                            int row0, int nrows, int lane) {
    const int nbk = p.k / 256;
    const int pr = lane & 3;
    float acc[R];
#pragma unroll
    for (int r = 0; r < R; ++r) acc[r] = 0.0f;
#pragma unroll
    for (int i = 0; i < NI; ++i) {
        const int b = 8 * i + (lane >> 2);
        if (b < nbk) {
#pragma unroll
            for (int r = 0; r < R; ++r) {
                const uint4 q0 = rw.q[i][r][0], q1 = rw.q[i][r][1];
                const uint4 l0 = ar.a0[i][0], l1 = ar.a0[i][1], h0 = ar.a1[i][0], h1 = ar.a1[i][1];
                int ql = dp4a_us(q0.x & 0x0f0f0f0fu, static_cast<int>(l0.x), 0);
                int qh = dp4a_us(q0.x & 0xf0f0f0f0u, static_cast<int>(h0.x), 0);
                ql = dp4a_us(q0.y & 0x0f0f0f0fu, static_cast<int>(l0.y), ql);
                qh = dp4a_us(q0.y & 0xf0f0f0f0u, static_cast<int>(h0.y), qh);
                ql = dp4a_us(q0.z & 0x0f0f0f0fu, static_cast<int>(l0.z), ql);
                qh = dp4a_us(q0.z & 0xf0f0f0f0u, static_cast<int>(h0.z), qh);
                ql = dp4a_us(q0.w & 0x0f0f0f0fu, static_cast<int>(l0.w), ql);
                qh = dp4a_us(q0.w & 0xf0f0f0f0u, static_cast<int>(h0.w), qh);
                ql = dp4a_us(q1.x & 0x0f0f0f0fu, static_cast<int>(l1.x), ql);
                qh = dp4a_us(q1.x & 0xf0f0f0f0u, static_cast<int>(h1.x), qh);
                ql = dp4a_us(q1.y & 0x0f0f0f0fu, static_cast<int>(l1.y), ql);
                qh = dp4a_us(q1.y & 0xf0f0f0f0u, static_cast<int>(h1.y), qh);
                ql = dp4a_us(q1.z & 0x0f0f0f0fu, static_cast<int>(l1.z), ql);
                qh = dp4a_us(q1.z & 0xf0f0f0f0u, static_cast<int>(h1.z), qh);
                ql = dp4a_us(q1.w & 0x0f0f0f0fu, static_cast<int>(l1.w), ql);
                qh = dp4a_us(q1.w & 0xf0f0f0f0u, static_cast<int>(h1.w), qh);
                qh >>= 4;  // 16 x the high-nibble sum, exactly
                if constexpr (kPartials) {
                    if (r < nrows) {
                        int32_t *out = p.partials + static_cast<int64_t>(row0 + r) * (p.k / 32) + b * 8 + 2 * pr;
                        out[0] = ql;
                        out[1] = qh;
                    }
                } else {
                    uint32_t scpk, mpk;
                    q4_K_scales_pair(rw.hd[i][r], pr, scpk, mpk);
                    const int i1 = static_cast<int>(scpk & 0xffu) * ql + static_cast<int>(scpk >> 8) * qh;
                    const int i2 = __dp2a_lo(ar.bs[i], static_cast<int>(mpk), 0);
                    const float d = f16_bits_to_f32(rw.hd[i][r].x & 0xffffu);
                    const float dmin = f16_bits_to_f32(rw.hd[i][r].x >> 16);
                    const float part =
                        __fsub_rn(__fmul_rn(d, static_cast<float>(i1)), __fmul_rn(dmin, static_cast<float>(i2)));
                    acc[r] = __fmaf_rn(ar.d[i], part, acc[r]);
                }
            }
        }
    }
    if constexpr (!kPartials) {
        if constexpr (R == 4) {
            reduce_store4(o, acc[0], acc[1], acc[2], acc[3], row0, nrows, lane);
        } else {
            const bool upper = (lane & 16) != 0;
            float v = (upper ? acc[1] : acc[0]) + __shfl_xor_sync(0xffffffffu, upper ? acc[0] : acc[1], 16);
#pragma unroll
            for (int sh = 8; sh > 0; sh >>= 1) v += __shfl_xor_sync(0xffffffffu, v, sh);
            if (lane == 0) o.c[row0] = v;
            if (lane == 16 && nrows > 1) o.c[row0 + 1] = v;
        }
    }
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
PFNG_DEV void row_q4_K(const GemvParams &p, const Out &o, const uint8_t *act, const uint8_t *tile, uint32_t row_off,
                       int row, int lane) {
    const int nbk = p.k / 256;
    const int8_t *aqs = reinterpret_cast<const int8_t *>(act);
    const float *ad = reinterpret_cast<const float *>(aqs + MT * p.k);
    const int16_t *abs16 = reinterpret_cast<const int16_t *>(ad + MT * nbk);
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
        const uint32_t q[4] = {qv.x, qv.y, qv.z, qv.w};
#pragma unroll
        for (int mi = 0; mi < MT; ++mi) {
            const int8_t *aq = aqs + mi * p.k + b * 256 + 16 * h;
            const int4 al = *reinterpret_cast<const int4 *>(aq + sbl * 32);
            const int4 ah = *reinterpret_cast<const int4 *>(aq + sbh * 32);
            int ql = dp4a_us(q[0] & 0x0f0f0f0fu, al.x, 0);
            int qh = dp4a_us(q[0] & 0xf0f0f0f0u, ah.x, 0);
            ql = dp4a_us(q[1] & 0x0f0f0f0fu, al.y, ql);
            qh = dp4a_us(q[1] & 0xf0f0f0f0u, ah.y, qh);
            ql = dp4a_us(q[2] & 0x0f0f0f0fu, al.z, ql);
            qh = dp4a_us(q[2] & 0xf0f0f0f0u, ah.z, qh);
            ql = dp4a_us(q[3] & 0x0f0f0f0fu, al.w, ql);
            qh = dp4a_us(q[3] & 0xf0f0f0f0u, ah.w, qh);
            qh >>= 4;
            if constexpr (kPartials) {
                const int fl = ql + __shfl_xor_sync(0xffffffffu, ql, 1);
                const int fh = qh + __shfl_xor_sync(0xffffffffu, qh, 1);
                if (live && h == 0 && mi < p.m) {
                    int32_t *out = p.partials + (static_cast<int64_t>(mi) * p.n + row) * (p.k / 32) + b * 8;
                    out[sbl] = fl;
                    out[sbh] = fh;
                }
            } else if (live) {
                const int16_t *bs = abs16 + mi * (p.k / 16) + b * 16;
                const int i1 = scl * ql + sch * qh;
                const int i2 = mnl * bs[sbl * 2 + h] + mnh * bs[sbh * 2 + h];
                const float part =
                    __fsub_rn(__fmul_rn(d, static_cast<float>(i1)), __fmul_rn(dmin, static_cast<float>(i2)));
                acc[mi] = __fmaf_rn(ad[mi * nbk + b], part, acc[mi]);
            }
        }
    }
    if constexpr (!kPartials) warp_reduce_store<MT>(p, o, acc, row, lane);
}

template <int MT, bool kPartials>
PFNG_DEV void row_iq2_xxs(const GemvParams &p, const Out &o, const uint8_t *act, const uint8_t *tile,
                          uint32_t row_off, int row, int lane, const uint2 *grid) {
    const int nbk = p.k / 256;
    const int8_t *aqs = reinterpret_cast<const int8_t *>(act);
    const float *ad = reinterpret_cast<const float *>(aqs + MT * p.k);
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
                const uint2 gv = grid[grid_slot((idx >> (8 * g)) & 0xffu, lane)];
                const uint32_t sgn = iq2_sign_mask((ss >> (7 * g)) & 0x7fu);
                v[2 * g] = apply_sign_bytes(gv.x, expand_bits4(sgn));
                v[2 * g + 1] = apply_sign_bytes(gv.y, expand_bits4(sgn >> 4));
            }
            const int scale = 2 * static_cast<int>(ss >> 28) + 1;
#pragma unroll
            for (int mi = 0; mi < MT; ++mi) {
                const int4 *a4 = reinterpret_cast<const int4 *>(aqs + mi * p.k + b * 256 + sb * 32);
                const int4 a0 = a4[0], a1 = a4[1];
                int dot0 = dp4a(static_cast<int>(v[0]), a0.x, 0);
                int dot1 = dp4a(static_cast<int>(v[4]), a1.x, 0);
                dot0 = dp4a(static_cast<int>(v[1]), a0.y, dot0);
                dot1 = dp4a(static_cast<int>(v[5]), a1.y, dot1);
                dot0 = dp4a(static_cast<int>(v[2]), a0.z, dot0);
                dot1 = dp4a(static_cast<int>(v[6]), a1.z, dot1);
                dot0 = dp4a(static_cast<int>(v[3]), a0.w, dot0);
                dot1 = dp4a(static_cast<int>(v[7]), a1.w, dot1);
                const int dot = dot0 + dot1;
                if constexpr (kPartials) {
                    if (mi < p.m) p.partials[(static_cast<int64_t>(mi) * p.n + row) * (p.k / 32) + b * 8 + sb] = dot;
                } else {
                    const float s = __fmul_rn(__fmul_rn(0.125f, d), ad[mi * nbk + b]);
                    acc[mi] = __fmaf_rn(s, static_cast<float>(scale * dot), acc[mi]);
                }
            }
        }
    }
    if constexpr (!kPartials) warp_reduce_store<MT>(p, o, acc, row, lane);
}

// ---------------------------------------------------------------------------
// iq2_xxs, m = 1, k <= 4096: activations in registers.  Lane l of iteration i
// takes the 32-value group sb = l & 7 of block b = 4 i + l / 8 (8 qs bytes at
// 2 + 8 sb).  Signs come from the table of byte masks m (0xff = negative)
// after the grid (both bank-striped, grid_slot): with signed dp4a, (g ^ m) is
// g or -g - 1, so
//   sum s g a = dp4a(g ^ m, a) + dp4a(m & 0x01010101, a)
// per 4 values -- the same integer as applying the signs first.
// ---------------------------------------------------------------------------
template <int NI>
struct ActRegsI {
    uint4 a[NI][2];  // the lane's 32 activations of iteration i
    float d[NI];     // their block's scale
};

template <int NI, int R>
struct RowsWI {
    uint32_t idx[NI][R];  // four grid indices
    uint32_t ss[NI][R];   // four 7-bit sign indices and the 4-bit scale
    uint32_t d[NI][R];    // fp16 block scale (bits)
};

template <int NI>
PFNG_DEV void load_act_iq2(const GemvParams &p, const uint8_t *act, int lane, ActRegsI<NI> &ar) {
    const int nbk = p.k / 256;
    const int8_t *aqs = reinterpret_cast<const int8_t *>(act);
    const float *ad = reinterpret_cast<const float *>(aqs + p.k);
#pragma unroll
    for (int i = 0; i < NI; ++i) {
        const int b = 4 * i + (lane >> 3), sb = lane & 7;
        if (b < nbk) {
            const uint4 *a = reinterpret_cast<const uint4 *>(aqs + b * 256 + 32 * sb);
            ar.a[i][0] = a[0], ar.a[i][1] = a[1];
            ar.d[i] = ad[b];
        } else {
            ar.a[i][0] = ar.a[i][1] = make_uint4(0, 0, 0, 0);
            ar.d[i] = 0.0f;
        }
    }
}

template <int NI, int R>
PFNG_DEV void load_rows_iq2(const GemvParams &p, const uint8_t *tile, uint32_t row_off, int nrows, int lane,
                            RowsWI<NI, R> &rw) {
    const int nbk = p.k / 256;
    const int sb = lane & 7;
#pragma unroll
    for (int i = 0; i < NI; ++i) {
        const int b = 4 * i + (lane >> 3);
        if (b < nbk) {
#pragma unroll
            for (int r = 0; r < R; ++r) {
                const int rr = r < nrows ? r : nrows - 1;
                const uint32_t boff = row_off + static_cast<uint32_t>(rr * p.row_bytes) + 66u * b;
                const uint32_t off = boff + 2 + 8 * sb;
                const uint32_t *w = reinterpret_cast<const uint32_t *>(tile + (off & ~3u));
                const uint32_t sh = (off & 2u) ? 16u : 0u;
                const uint32_t w0 = w[0], w1 = w[1], w2 = w[2];
                rw.idx[i][r] = __funnelshift_r(w0, w1, sh);
                rw.ss[i][r] = __funnelshift_r(w1, w2, sh);
                rw.d[i][r] = *reinterpret_cast<const uint16_t *>(tile + boff);
            }
        }
    }
}

template <int NI, int R, bool kPartials>
PFNG_DEV void rows_iq2_reg(const GemvParams &p, const Out &o, const ActRegsI<NI> &ar, const RowsWI<NI, R> &rw,
                           int row0, int nrows, int lane, const uint2 *grid) {
    const int nbk = p.k / 256;
    const int sb = lane & 7;
    float acc[R];
#pragma unroll
    for (int r = 0; r < R; ++r) acc[r] = 0.0f;
#pragma unroll
    for (int i = 0; i < NI; ++i) {
        const int b = 4 * i + (lane >> 3);
        if (b < nbk) {
            const uint32_t av[8] = {ar.a[i][0].x, ar.a[i][0].y, ar.a[i][0].z, ar.a[i][0].w,
                                    ar.a[i][1].x, ar.a[i][1].y, ar.a[i][1].z, ar.a[i][1].w};
#pragma unroll
            for (int r = 0; r < R; ++r) {
                const uint32_t idx = rw.idx[i][r], ss = rw.ss[i][r];
                int dot = 0, corr = 0;
#pragma unroll
                for (int g = 0; g < 4; ++g) {
                    const uint2 gv = grid[grid_slot((idx >> (8 * g)) & 0xffu, lane)];
                    const uint2 mk = grid[kSignTable + grid_slot((ss >> (7 * g)) & 0x7fu, lane)];
                    dot = dp4a(static_cast<int>(gv.x ^ mk.x), static_cast<int>(av[2 * g]), dot);
                    corr = dp4a(static_cast<int>(mk.x & 0x01010101u), static_cast<int>(av[2 * g]), corr);
                    dot = dp4a(static_cast<int>(gv.y ^ mk.y), static_cast<int>(av[2 * g + 1]), dot);
                    corr = dp4a(static_cast<int>(mk.y & 0x01010101u), static_cast<int>(av[2 * g + 1]), corr);
                }
                dot += corr;
                if constexpr (kPartials) {
                    if (r < nrows) p.partials[static_cast<int64_t>(row0 + r) * (p.k / 32) + b * 8 + sb] = dot;
                } else {
                    // llama_reference.cpp:160: 0.125 * d * a.d, times the scaled integer sum
                    const int scale = 2 * static_cast<int>(ss >> 28) + 1;
                    const float s = __fmul_rn(__fmul_rn(0.125f, f16_bits_to_f32(rw.d[i][r])), ar.d[i]);
                    acc[r] = __fmaf_rn(s, static_cast<float>(scale * dot), acc[r]);
                }
            }
        }
    }
    if constexpr (!kPartials) {
        if constexpr (R == 4) {
            reduce_store4(o, acc[0], acc[1], acc[2], acc[3], row0, nrows, lane);
        } else {
            const bool upper = (lane & 16) != 0;
            float v = (upper ? acc[1] : acc[0]) + __shfl_xor_sync(0xffffffffu, upper ? acc[0] : acc[1], 16);
#pragma unroll
            for (int sh = 8; sh > 0; sh >>= 1) v += __shfl_xor_sync(0xffffffffu, v, sh);
            if (lane == 0) o.c[row0] = v;
            if (lane == 16 && nrows > 1) o.c[row0 + 1] = v;
        }
    }
}

// Waits until the producer has issued local tile i: 1 once it has, 0 if the
// producer finished with fewer tiles, -1 (error recorded) if it never does.
PFNG_DEV int wait_issued(const int *issued_count, const int *final_count, int i, int *err) {
    const volatile int *ic = issued_count;
    const volatile int *fc = final_count;
    for (uint32_t n = 0; n < kWaitAttempts; ++n) {
        if (*ic > i) return 1;
        if (*fc >= 0) {
            __threadfence_block();  // final_count before issued_count
            return *ic > i ? 1 : 0;
        }
        __nanosleep(64);
    }
    report_error(err, kErrWaitIssue);
    return -1;
}

// --------------------------------------------------------------------------
// the kernel
// --------------------------------------------------------------------------
// RG > 0: q4_0 with m = 1 and the activations held in registers (RG groups).
template <int WT, int MT, int RG, bool kPartials, bool kF32>
__global__ void __launch_bounds__(kGemvThreads, kCtasPerSm) gemv_kernel(const GemvParams p) {
    extern __shared__ __align__(128) uint8_t smem[];
    uint64_t *full = reinterpret_cast<uint64_t *>(smem);
    uint64_t *empty = full + kMaxStages;
    __shared__ int abort_flag;
    __shared__ int next_tile;
    // per stage: {matrix, first row of the tile in that matrix, rows, 0}
    __shared__ int4 stage_info[kMaxStages];
    // Local tiles issued so far and, once the launch's tiles are all claimed,
    // their final number.  A consumer waits on a stage's mbarrier only after
    // its tile has been issued: the producer issues local tile i only after
    // tile i - S left the stage, so the barrier is then in tile i's phase (a
    // parity wait can only name the current or the previous phase).
    __shared__ int issued_count;
    __shared__ int final_count;
    const int tid = threadIdx.x;
    const int warp = tid >> 5, lane = tid & 31;
    const int S = p.stages;

    if (PFNG_GEMV_EARLY_TRIGGER && p.overlap && tid == 0) asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    if (tid < S) {
        mbar_init(&full[tid], 1);
        mbar_init(&empty[tid], p.rows_per_tile / kClaimRows);  // one arrival per claim
        fence_mbar_init();
    }
    if (tid == 0) {
        abort_flag = 0;
        next_tile = 0;
        issued_count = 0;
        final_count = -1;
    }
    __syncthreads();

    if (warp == kConsumerWarps) {
        // ---------------- producer ----------------
        // The CTA streams one contiguous range of the launch's rows (all CTAs
        // get the same number of rows, +-1), in tiles of up to rows_per_tile
        // rows that do not cross a matrix boundary.  issued_count publishes
        // how many tiles have been issued, final_count how many there are
        // once the last one is.
        if (lane == 0) {
            const uint64_t policy = l2_policy_evict_first();
            int issued = 0, stage = 0;
            uint32_t phase = 0;
            int g = 0;  // matrix of the current tile (rows only increase)
            bool ok = true;
            const int r_begin = static_cast<int>(static_cast<int64_t>(p.total_rows) * blockIdx.x / gridDim.x);
            const int r_end = static_cast<int>(static_cast<int64_t>(p.total_rows) * (blockIdx.x + 1) / gridDim.x);
            for (int r = r_begin; r < r_end;) {
                // tile issued - kInflight must have landed: its stage still
                // holds it (it is refilled only by tile issued - kInflight + S);
                // with kInflight >= S the empty-stage wait below bounds it
                const int old = kInflight < S ? issued - kInflight : (kFirstWave > 0 && issued == kFirstWave ? 0 : -1);
                if ((old >= 0 && !mbar_wait(&full[old % S], static_cast<uint32_t>((old / S) & 1), p.err, kErrWaitFull)) ||
                    (issued >= S && !mbar_wait(&empty[stage], phase ^ 1u, p.err, kErrWaitEmpty)) ||
                    *reinterpret_cast<volatile int *>(&abort_flag)) {
                    ok = false;
                    break;
                }
                while (r >= p.row_base[g + 1]) ++g;
                int rows = p.rows_per_tile;
                if (rows > r_end - r) rows = r_end - r;
                if (rows > p.row_base[g + 1] - r) rows = p.row_base[g + 1] - r;
                const int lr = r - p.row_base[g];
                const int64_t start = static_cast<int64_t>(lr) * p.row_bytes;
                const int64_t end = static_cast<int64_t>(lr + rows) * p.row_bytes;
                const int64_t ws = start & ~int64_t(15), we = (end + 15) & ~int64_t(15);
                const uint32_t bytes = static_cast<uint32_t>(we - ws);
                const uint8_t *src = p.wg[g] + ws;
                uint8_t *dst = smem + p.stage_offset + static_cast<uint32_t>(stage) * p.stage_bytes;
                stage_info[stage] = make_int4(g, lr, rows, 0);
                r += rows;
                mbar_arrive_expect_tx(&full[stage], bytes);
                bulk_copy_g2s(dst, src, bytes, &full[stage], policy);
                *reinterpret_cast<volatile int *>(&issued_count) = ++issued;
                if (++stage == S) stage = 0, phase ^= 1u;
            }
            __threadfence_block();  // issued_count before final_count
            *reinterpret_cast<volatile int *>(&final_count) = issued;
            if (!ok) {
                abort_flag = 1;
                // do not leave while copies into this CTA's shared memory are in flight
                for (int i = issued - S > 0 ? issued - S : 0; i < issued; ++i)
                    mbar_wait(&full[i % S], static_cast<uint32_t>((i / S) & 1), p.err, kErrWaitFull);
            }
        }
        return;
    }

    // ---------------- consumers ----------------
    uint2 *grid = reinterpret_cast<uint2 *>(smem + p.grid_offset);
    if constexpr (WT == kWIQ2) {
        for (int i = tid; i < 256 * kGridCopies; i += kConsumerThreads) {
            const uint32_t code = pfng_iq2xxs_grid_codes[i / kGridCopies];
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
        // byte masks (0xff = negative) of the 128 sign indices
        for (int i = tid; i < 128 * kGridCopies; i += kConsumerThreads) {
            const uint32_t sgn = iq2_sign_mask(static_cast<uint32_t>(i / kGridCopies));
            grid[kSignTable + i] = make_uint2(expand_bits4(sgn), expand_bits4(sgn >> 4));
        }
    }
    const uint8_t *act = smem + p.act_offset;
    if (p.overlap) asm volatile("griddepcontrol.wait;" ::: "memory");
    if constexpr (WT == kWQ4_0 || WT == kWQ4_0P)
        stage_act_q8_0<MT, kF32, WT == kWQ4_0P>(p, smem, tid);
    else
        stage_act_q8_K<MT, kF32>(p, smem, tid);
    consumer_sync();
    // Programmatic dependent launch: the next launch on the stream may start
    // once every CTA of this one has its activations staged; its CTAs take
    // SMs as this launch's CTAs exit and prefetch their weights.  Only that
    // prefetch runs before its griddepcontrol.wait; activations and outputs
    // stay ordered after this grid as usual.
    if (!PFNG_GEMV_EARLY_TRIGGER && p.overlap && tid == 0) asm volatile("griddepcontrol.launch_dependents;" ::: "memory");

    ActRegs<(RG > 0 ? RG : 1)> ar;
    ActRegsP<(RG > 0 ? RG : 1)> arp;
    ActRegsK<(RG > 0 ? RG : 1)> ark;
    if constexpr (WT == kWQ4_K && RG > 0) load_act_q4_K<RG>(p, act, lane, ark);
    ActRegsI<(RG > 0 ? RG : 1)> ari;
    if constexpr (WT == kWIQ2 && RG > 0) load_act_iq2<RG>(p, act, lane, ari);
    if constexpr (WT == kWQ4_0P && RG > 0) {
        const int nbp = p.groups * 32;
        const float *ad = reinterpret_cast<const float *>(act + nbp * 32);
        const int32_t *abias = reinterpret_cast<const int32_t *>(ad + nbp);
#pragma unroll
        for (int t = 0; t < RG; ++t) {
            if (t < p.groups) {
                const uint4 *aq = reinterpret_cast<const uint4 *>(act + t * 1024) + lane;
                arp.lo[t] = aq[0];
                arp.hi[t] = aq[32];
                arp.d[t] = ad[32 * t + lane];
                arp.bias[t] = abias[32 * t + lane];
            } else {
                arp.lo[t] = arp.hi[t] = make_uint4(0, 0, 0, 0);
                arp.d[t] = 0.0f;
                arp.bias[t] = kMagicBits;
            }
        }
    } else if constexpr (RG > 0) {
        const int nbp = p.groups * 64;
        const float *ad = reinterpret_cast<const float *>(act + p.groups * 2048);
        const int32_t *as8 = reinterpret_cast<const int32_t *>(ad + nbp);
#pragma unroll
        for (int t = 0; t < RG; ++t) {
            if (t < p.groups) {
                const uint4 *aq = reinterpret_cast<const uint4 *>(act + t * 2048) + lane;
#pragma unroll
                for (int c = 0; c < 4; ++c) ar.q[t][c] = aq[32 * c];
                ar.d[t] = *reinterpret_cast<const float2 *>(ad + 64 * t + 2 * lane);
                ar.s8[t] = *reinterpret_cast<const int2 *>(as8 + 64 * t + 2 * lane);
            } else {
#pragma unroll
                for (int c = 0; c < 4; ++c) ar.q[t][c] = make_uint4(0, 0, 0, 0);
                ar.d[t] = make_float2(0.0f, 0.0f);
                ar.s8[t] = make_int2(0, 0);
            }
        }
    }

    // Each warp holds two claims: the rows it works on and the next ones,
    // taken while the current ones are processed so that the atomic's
    // latency is off the critical path.  A claim is kClaimRows rows of one
    // tile, processed as two pairs.
    int q_next = 0;
    if (lane == 0) q_next = atomicAdd(&next_tile, 1);
    int cur_i = 0, stage = 0, lap = 0;  // ring position of the last claim (claims only increase)
    for (;;) {
        const int q = __shfl_sync(0xffffffffu, q_next, 0);
        const int i = q >> p.claim_shift;                   // local tile index
        const int qr = q & ((1 << p.claim_shift) - 1);      // claim within the tile
        stage += i - cur_i;
        cur_i = i;
        while (stage >= S) stage -= S, ++lap;
        const int avail = wait_issued(&issued_count, &final_count, i, p.err);
        if (avail <= 0) {
            if (avail < 0) abort_flag = 1;
            break;  // 0: the CTA's tiles are all taken
        }
        if (*reinterpret_cast<volatile int *>(&abort_flag)) break;
        if (!mbar_wait(&full[stage], static_cast<uint32_t>(lap & 1), p.err, kErrWaitFull)) {
            abort_flag = 1;
            break;
        }
        const int4 info = stage_info[stage];  // ordered after the mbarrier wait (memory clobber)
        if (lane == 0) q_next = atomicAdd(&next_tile, 1);
        const int g = info.x, tile_row = info.y, tile_rows = info.z;
        const Out o{p.cg[g], p.ldcg[g]};
        // the stage's window starts at the tile's first byte rounded down to 16
        const uint32_t mis = (static_cast<uint32_t>(tile_row) * static_cast<uint32_t>(p.row_bytes)) & 15u;
        const uint8_t *buf = smem + p.stage_offset + static_cast<uint32_t>(stage) * p.stage_bytes;
        if constexpr (WT == kWIQ2 && RG > 0 && !kPartials && kClaimRows == 4 && PFNG_GEMV_CLAIM4) {
            const int first = kClaimRows * qr;
            const int nrows = tile_rows - first < kClaimRows ? tile_rows - first : kClaimRows;
            const uint32_t row_off = static_cast<uint32_t>(first) * static_cast<uint32_t>(p.row_bytes) + mis;
            RowsWI<RG, 4> rw;
            if (nrows > 0) load_rows_iq2<RG, 4>(p, buf, row_off, nrows, lane, rw);
            __syncwarp();
            if (lane == 0) mbar_arrive(&empty[stage]);
            if (nrows > 0) rows_iq2_reg<RG, 4, kPartials>(p, o, ari, rw, tile_row + first, nrows, lane, grid);
        } else if constexpr (WT == kWQ4_K && RG > 0 && !kPartials && kClaimRows == 4 && PFNG_GEMV_CLAIM4) {
            const int first = kClaimRows * qr;
            const int nrows = tile_rows - first < kClaimRows ? tile_rows - first : kClaimRows;
            const uint32_t row_off = static_cast<uint32_t>(first) * static_cast<uint32_t>(p.row_bytes) + mis;
            RowsWK<RG, 4> rw;
            if (nrows > 0) load_rows_q4_K<RG, 4>(p, buf, row_off, nrows, lane, rw);
            __syncwarp();
            if (lane == 0) mbar_arrive(&empty[stage]);
            if (nrows > 0) rows_q4_K_reg<RG, 4, kPartials>(p, o, ark, rw, tile_row + first, nrows, lane);
        } else if constexpr (WT == kWQ4_0P && RG > 0 && !kPartials && kClaimRows == 4 && PFNG_GEMV_CLAIM4) {
            const int first = kClaimRows * qr;
            const int nrows = tile_rows - first < kClaimRows ? tile_rows - first : kClaimRows;
            const uint32_t row_off = static_cast<uint32_t>(first) * static_cast<uint32_t>(p.row_bytes) + mis;
            RowsWP<RG> r01, r23;
            if (nrows > 0) load_rows_q4_0p<RG>(p, buf, row_off, nrows < 2 ? nrows : 2, lane, r01);
            if (nrows > 2)
                load_rows_q4_0p<RG>(p, buf, row_off + 2u * static_cast<uint32_t>(p.row_bytes), nrows - 2, lane, r23);
            __syncwarp();
            if (lane == 0) mbar_arrive(&empty[stage]);
            if (nrows > 2)
                rows4_q4_0p_reg<RG>(p, o, arp, r01, r23, tile_row + first, nrows, lane);
            else if (nrows > 0)
                rows_q4_0p_reg<RG, kPartials>(p, o, arp, r01, tile_row + first, nrows, lane);
        } else if constexpr (WT == kWQ4_0 && RG > 0 && !kPartials && kClaimRows == 4 && PFNG_GEMV_CLAIM4) {
            // the claim's four rows at once: all weights to registers, release
            // the stage, then compute
            const int first = kClaimRows * qr;
            const int nrows = tile_rows - first < kClaimRows ? tile_rows - first : kClaimRows;
            const uint32_t row_off = static_cast<uint32_t>(first) * static_cast<uint32_t>(p.row_bytes) + mis;
            RowsW<RG> r01, r23;
            if (nrows > 0) load_rows_q4_0<RG>(p, buf, row_off, nrows < 2 ? nrows : 2, lane, r01);
            if (nrows > 2)
                load_rows_q4_0<RG>(p, buf, row_off + 2u * static_cast<uint32_t>(p.row_bytes), nrows - 2, lane, r23);
            __syncwarp();
            if (lane == 0) mbar_arrive(&empty[stage]);
            if (nrows > 2) {
                if constexpr (PFNG_GEMV_FOLD2)
                    rows4_q4_0_reg_f2<RG>(p, o, ar, r01, r23, tile_row + first, nrows, lane);
                else
                    rows4_q4_0_reg<RG>(p, o, ar, r01, r23, tile_row + first, nrows, lane);
            }
            else if (nrows > 0)
                rows_q4_0_reg<RG, kPartials>(p, o, ar, r01, tile_row + first, nrows, lane);
        } else {
#pragma unroll 1
        for (int h = 0; h < kClaimRows / kPairRows; ++h) {
            const int first = kClaimRows * qr + kPairRows * h;  // first row of the pair in the tile
            const int row0 = tile_row + first;
            const int nrows = tile_rows - first < kPairRows ? tile_rows - first : kPairRows;
            const uint32_t row_off = static_cast<uint32_t>(first) * static_cast<uint32_t>(p.row_bytes) + mis;
            const bool last = h == kClaimRows / kPairRows - 1;
            if constexpr (WT == kWQ4_0P && RG > 0) {
                RowsWP<RG> rw;
                if (nrows > 0) load_rows_q4_0p<RG>(p, buf, row_off, nrows, lane, rw);
                if (last) {
                    __syncwarp();
                    if (lane == 0) mbar_arrive(&empty[stage]);
                }
                if (nrows > 0) rows_q4_0p_reg<RG, kPartials>(p, o, arp, rw, row0, nrows, lane);
            } else if constexpr (WT == kWIQ2 && RG > 0) {
                RowsWI<RG, 2> rw;
                if (nrows > 0) load_rows_iq2<RG, 2>(p, buf, row_off, nrows, lane, rw);
                if (last) {
                    __syncwarp();
                    if (lane == 0) mbar_arrive(&empty[stage]);
                }
                if (nrows > 0) rows_iq2_reg<RG, 2, kPartials>(p, o, ari, rw, row0, nrows, lane, grid);
            } else if constexpr (WT == kWQ4_K && RG > 0) {
                RowsWK<RG, 2> rw;
                if (nrows > 0) load_rows_q4_K<RG, 2>(p, buf, row_off, nrows, lane, rw);
                if (last) {
                    __syncwarp();
                    if (lane == 0) mbar_arrive(&empty[stage]);
                }
                if (nrows > 0) rows_q4_K_reg<RG, 2, kPartials>(p, o, ark, rw, row0, nrows, lane);
            } else if constexpr (WT == kWQ4_0 && RG > 0) {
                // copy the pair's weights to registers; after the claim's last
                // pair is copied, release the stage, then compute
                RowsW<RG> rw;
                if (nrows > 0) load_rows_q4_0<RG>(p, buf, row_off, nrows, lane, rw);
                if (last) {
                    __syncwarp();
                    if (lane == 0) mbar_arrive(&empty[stage]);
                }
                if (nrows > 0) rows_q4_0_reg<RG, kPartials>(p, o, ar, rw, row0, nrows, lane);
            } else {
                if (nrows > 0) {
                    if constexpr (WT == kWQ4_0) {
                        rows_q4_0_smem<MT, kPartials>(p, o, act, buf, row_off, row0, nrows, lane);
                    } else if constexpr (WT == kWQ4_0P) {
                        rows_q4_0p_smem<MT, kPartials>(p, o, act, buf, row_off, row0, nrows, lane);
                    } else {
                        for (int r = 0; r < nrows; ++r) {
                            const uint32_t off = row_off + static_cast<uint32_t>(r * p.row_bytes);
                            if constexpr (WT == kWQ4_K)
                                row_q4_K<MT, kPartials>(p, o, act, buf, off, row0 + r, lane);
                            else
                                row_iq2_xxs<MT, kPartials>(p, o, act, buf, off, row0 + r, lane, grid);
                        }
                    }
                }
                if (last) {
                    __syncwarp();
                    if (lane == 0) mbar_arrive(&empty[stage]);
                }
            }
        }
        }
    }
}

int64_t row_bytes_of(int wtype, int64_t k) {
    switch (wtype) {
    case kWQ4_0:
    case kWQ4_0P: return k / 32 * kQ4_0Bytes;
    case kWQ4_K: return k / 256 * kQ4_KBytes;
    default: return k / 256 * kIQ2Bytes;
    }
}

int mt_of(int64_t m) { return m <= 1 ? 1 : m <= 2 ? 2 : m <= 4 ? 4 : 8; }

uint32_t act_bytes_of(int wtype, int mt, int64_t k) {
    if (wtype == kWQ4_0) {
        const int64_t groups = (k / 32 + 63) / 64;
        return static_cast<uint32_t>(mt * groups * (2048 + 64 * 8));
    }
    if (wtype == kWQ4_0P) {
        const int64_t groups = (k / 32 + 31) / 32;
        return static_cast<uint32_t>(mt * groups * (1024 + 32 * 8));
    }
    return static_cast<uint32_t>(mt * (k + (k / 256) * 4 + (k / 16) * 2));
}

uint32_t align_up_u32(uint32_t v, uint32_t a) { return (v + a - 1) / a * a; }

// Fills the tiling / shared-memory plan; false if the shape does not fit.
bool plan(int wtype, int64_t m, int count, const int64_t *ns, int64_t k, GemvParams &p, uint32_t &smem_bytes) {
    if (count < 1 || count > kMaxGroup || k > 0x7fffffff / 8) return false;
    for (int g = 0; g < count; ++g)
        if (ns[g] < 1 || ns[g] > 0x7fffffff / 8) return false;
    const int mt = mt_of(m);
    const int64_t rb = row_bytes_of(wtype, k);
    p.row_bytes = static_cast<int>(rb);
    p.rows_per_tile = rb >= 2048 ? kTileRowsLong : 8;
    p.claim_shift = 0;
    while ((kClaimRows << p.claim_shift) < p.rows_per_tile) ++p.claim_shift;
    p.count = count;
    int64_t rows = 0;
    for (int g = 0; g < count; ++g) {
        p.ng[g] = static_cast<int>(ns[g]);
        p.row_base[g] = static_cast<int>(rows);
        rows += ns[g];
    }
    if (rows > 0x3fffffff) return false;
    for (int g = count; g <= kMaxGroup; ++g) p.row_base[g] = static_cast<int>(rows);
    p.total_rows = static_cast<int>(rows);
    p.num_tiles = static_cast<int>((rows + p.rows_per_tile - 1) / p.rows_per_tile);
    p.groups = static_cast<int>(wtype == kWQ4_0P ? (k / 32 + 31) / 32 : (k / 32 + 63) / 64);
    p.stage_bytes = align_up_u32(static_cast<uint32_t>(p.rows_per_tile * rb) + 16 + kStageSlack, 128);
    p.grid_offset = kBarrierBytes;
    p.act_offset = align_up_u32(p.grid_offset + (wtype == kWIQ2 ? kGridTableBytes : 0), 128);
    p.stage_offset = align_up_u32(p.act_offset + act_bytes_of(wtype, mt, k), 128);
    // at most half the SM's shared memory, so that the next launch's CTA can
    // be resident beside this one (overlapped decode launches)
    const size_t optin = device_smem_optin();
    const size_t budget = (optin + 1024) / kCtasPerSm - 2048;
    if (p.stage_offset + 4 * static_cast<size_t>(p.stage_bytes) > budget) return false;
    const size_t fit = (budget - p.stage_offset) / p.stage_bytes;
    p.stages = static_cast<int>(fit < static_cast<size_t>(kMaxStages) ? fit : kMaxStages);
    smem_bytes = p.stage_offset + static_cast<uint32_t>(p.stages) * p.stage_bytes;
    return true;
}

template <int WT, int MT, int RG, bool kPartials, bool kF32>
cudaError_t launch_one(const GemvParams &p, uint32_t smem, cudaStream_t s) {
    auto kernel = gemv_kernel<WT, MT, RG, kPartials, kF32>;
    static thread_local int configured_smem[64] = {0};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 0 || dev >= 64 || configured_smem[dev] < static_cast<int>(smem)) {
        cudaError_t e =
            cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
        if (e != cudaSuccess) return e;
        if (dev >= 0 && dev < 64) configured_smem[dev] = static_cast<int>(smem);
    }
    const int sms = device_sm_count();
    const int grid = p.num_tiles < sms ? p.num_tiles : sms;
    if (!p.overlap) {
        kernel<<<grid, kGemvThreads, smem, s>>>(p);
        return cudaGetLastError();
    }
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3(static_cast<unsigned>(grid));
    cfg.blockDim = dim3(kGemvThreads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kernel, p);
}

template <int WT, int MT, int RG>
cudaError_t dispatch_flags(const GemvParams &p, uint32_t smem, bool partials, bool f32, cudaStream_t s) {
    if (partials)
        return f32 ? launch_one<WT, MT, RG, true, true>(p, smem, s) : launch_one<WT, MT, RG, true, false>(p, smem, s);
    return f32 ? launch_one<WT, MT, RG, false, true>(p, smem, s) : launch_one<WT, MT, RG, false, false>(p, smem, s);
}

template <int WT>
cudaError_t dispatch_mt(const GemvParams &p, uint32_t smem, bool partials, bool f32, cudaStream_t s) {
    if constexpr (WT == kWIQ2) {
        // units of 32 values, 32 per iteration: k <= 4096 in four iterations
        if (p.m == 1 && p.k <= 1024) return dispatch_flags<WT, 1, 1>(p, smem, partials, f32, s);
        if (p.m == 1 && p.k <= 2048) return dispatch_flags<WT, 1, 2>(p, smem, partials, f32, s);
        if (p.m == 1 && p.k <= 4096) return dispatch_flags<WT, 1, 4>(p, smem, partials, f32, s);
    }
    if constexpr (WT == kWQ4_K) {
        // units of 64 values, 32 per iteration: k <= 4096 in two iterations
        if (p.m == 1 && p.k <= 2048) return dispatch_flags<WT, 1, 1>(p, smem, partials, f32, s);
        if (p.m == 1 && p.k <= 4096) return dispatch_flags<WT, 1, 2>(p, smem, partials, f32, s);
    }
    if constexpr (WT == kWQ4_0P) {
        if (p.m == 1) {
            if (p.groups <= 1) return dispatch_flags<WT, 1, 1>(p, smem, partials, f32, s);
            if (p.groups <= 2) return dispatch_flags<WT, 1, 2>(p, smem, partials, f32, s);
            if (p.groups <= 4) return dispatch_flags<WT, 1, 4>(p, smem, partials, f32, s);
        }
    }
    if constexpr (WT == kWQ4_0) {
        if (p.m == 1) {
            if (p.groups <= 1) return dispatch_flags<WT, 1, 1>(p, smem, partials, f32, s);
            if (p.groups <= 2) return dispatch_flags<WT, 1, 2>(p, smem, partials, f32, s);
            if (p.groups <= kRegGroupsMax) return dispatch_flags<WT, 1, kRegGroupsMax>(p, smem, partials, f32, s);
        }
    }
    switch (mt_of(p.m)) {
    case 1: return dispatch_flags<WT, 1, 0>(p, smem, partials, f32, s);
    case 2: return dispatch_flags<WT, 2, 0>(p, smem, partials, f32, s);
    case 4: return dispatch_flags<WT, 4, 0>(p, smem, partials, f32, s);
    default: return dispatch_flags<WT, 8, 0>(p, smem, partials, f32, s);
    }
}

}  // namespace

bool gemv_supported(int wtype, int64_t m, int count, const int64_t *n, int64_t k, const void *const *w) {
    if (m < 1 || m > 8 || count < 1 || count > kMaxGroup) return false;
    if (wtype == kWQ4_0 && (k / 32) % 2 != 0) return false;  // block pairs
    if (wtype == kWQ4_0P && k % 256 != 0) return false;     // 16-byte aligned planar rows
    const int64_t rb = row_bytes_of(wtype, k);
    for (int g = 0; g < count; ++g)
        if (n[g] < 1 || (reinterpret_cast<uintptr_t>(w[g]) & 15u) != 0 || (n[g] * rb) % 16 != 0) return false;
    GemvParams p{};
    uint32_t smem = 0;
    return plan(wtype, m, count, n, k, p, smem);
}

cudaError_t launch_gemv(const GemvArgs &args, cudaStream_t s) {
    GemvParams p{};
    uint32_t smem = 0;
    if (!plan(args.wtype, args.m, args.count, args.n, args.k, p, smem)) return cudaErrorInvalidValue;
    for (int g = 0; g < args.count; ++g) {
        p.wg[g] = static_cast<const uint8_t *>(args.w[g]);
        p.cg[g] = args.c[g];
        p.ldcg[g] = args.ldc[g];
    }
    p.a = static_cast<const uint8_t *>(args.a);
    p.x = args.x;
    p.ldx = args.ldx;
    p.x_vec = args.x && (reinterpret_cast<uintptr_t>(args.x) & 15u) == 0 && (args.ldx & 3) == 0;
    p.partials = args.partials;
    p.err = args.err;
    p.overlap = args.overlap ? 1 : 0;
    p.m = static_cast<int>(args.m);
    p.n = static_cast<int>(args.n[0]);
    p.k = static_cast<int>(args.k);
    const bool partials = args.partials != nullptr;
    const bool f32 = args.x != nullptr;
    switch (args.wtype) {
    case kWQ4_0: return dispatch_mt<kWQ4_0>(p, smem, partials, f32, s);
    case kWQ4_K: return dispatch_mt<kWQ4_K>(p, smem, partials, f32, s);
    case kWQ4_0P: return dispatch_mt<kWQ4_0P>(p, smem, partials, f32, s);
    default: return dispatch_mt<kWIQ2>(p, smem, partials, f32, s);
    }
}

}  // namespace pfng
