// gemm.cu -- batched-m block-quantized matmul on the int8 tensor cores.
//
// C[m][n] = A[m][k] . W[n][k]^T with W in the raw ggml layout (or q4_0 in
// the planar row layout) and A in the split layout (int8 rows + per-block
// scales) produced by quantize.cu.
// Semantics: compute_q4_0 / compute_q4_K / compute_iq2_xxs,
// bench/llama_reference/llama_reference.cpp:113-205.
//
// CTA tile BM x BN (32..128 each, chosen per shape to fill the SMs), k-step
// 256, 8 warps (2 along m and 4 along n; 1 x 8 on 128 x 128 q4_0 tiles),
// every 32-deep sub-block one m16n8k32 s8 MMA per 16 x 8 fragment.  The
// stage ring holds the A rows, A scales and raw W bytes of a k-step: for
// q4_0 on 128 x 128, 64 x 64 and 32 x 128 tiles it is filled by tensor-map
// bulk copies issued by one thread (full / empty mbarriers per stage),
// otherwise by per-thread cp.async.  q4_0 and q4_K take their B fragments
// straight from the raw W rows ("direct operands"); iq2_xxs (and the
// comparison switches) unpack the raw W tile once per k-step into an int8
// [n][k] tile and a per-(sub-block, column) scale s.
//
// The fold (the per-sub-block scaling that makes this more than an int8
// GEMM) is the same for all three types and costs one packed instruction
// (fma.rn.f32x2) per element and sub-block:
//   * the MMA accumulator input is the constant 0x4B400000, so the int32 dot
//     product P (|P| < 2^22) comes back as the float 2^23 + 2^22 + P exactly;
//   * t = fma(y, s, -(2^23 + 2^22) * s) = round(P * s): the product M * s is
//     exact because s has at most 17 significant bits (fp16 scale times a
//     6-bit integer scale), so the only rounding is that of P * s;
//   * acc = fma(t, a_d, acc), a_d the activation block scale.
// s is d_w (q4_0), d * scale_sb (q4_K) or 0.125 * d * (2 k + 1) (iq2_xxs).
// q4_K's min term -a_d * dmin * sum_sb min_sb * bsum_sb is added once per 256
// block with dp4a over packed 6-bit mins and split bsums.  Integer partials
// are exact (int32 tensor-core accumulation); the fp32 fold follows the
// reference's block order (k ascending), so results differ from the
// reference only by where fp32 rounding happens.
#include <cstdlib>
#include <cstring>
#include <mutex>

#include <cuda_bf16.h>

#include "iq2xxs_grid_codes.h"
#include "pfng_common.cuh"
#include "pfng_internal.h"
#include "pfng_quant.cuh"
#include "pfng_tma.h"

namespace pfng {
namespace {

constexpr int BK = 256;
constexpr int kThreads = 256;
constexpr bool kTcDefault = false;
#ifndef PFNG_GEMM_STAGES
#define PFNG_GEMM_STAGES 3
#endif
constexpr int kStages = PFNG_GEMM_STAGES;  // cp.async ring depth
constexpr uint32_t kMagicBits = 0x4B400000u;  // float 12582912 = 2^23 + 2^22
constexpr float kMagic = 12582912.0f;
// true when the activations are q8_0 (one fp32 scale per 32 values)
template <int WT>
constexpr bool kQ8_0Act = WT == kWQ4_0 || WT == kWQ4_0P;
constexpr uint32_t kMaxSmemPerCta = 227 * 1024;  // opt-in dynamic shared memory per CTA on sm_100
constexpr uint32_t kWRowSlot = 160;          // >= 144 raw bytes + 8 window slack, multiple of 16
constexpr int kAScaleStride = 12;

template <int BM_, int BN_, int ST_ = kStages, uint32_t SLOT_ = kWRowSlot, int WGM_ = 2, bool TMA_ = false>
struct Cfg {
    static constexpr int BM = BM_, BN = BN_;
    static constexpr int ST = ST_;  // cp.async ring depth of the two-phase kernel
    static constexpr uint32_t kSlot = SLOT_;  // bytes per raw W row in shared memory
    // Stages loaded by tensor-map bulk copies from one thread (direct q4_0
    // operands on 128 x 128 tiles): the activation rows as two 128-byte-wide
    // boxes with the 128-byte swizzle ([half][row][128 B]), raw W rows of
    // step_bytes (kSlot = 144), the q8_0 scales as one [8][128] box; stages
    // 1024-byte aligned for the swizzle.
    static constexpr bool kTma = TMA_;
    // the 8 warps as WGM along m x WGN along n
    static constexpr int WGM = WGM_, WGN = 8 / WGM_;
    static constexpr int WM = BM / WGM, WN = BN / WGN;  // warp tile
    static constexpr int MT = WM / 16, NT = WN / 8;  // m16n8 fragments per warp
    static_assert(MT >= 1 && NT >= 2 && NT % 2 == 0, "tile shape");
    // shared memory (per stage, then single buffers)
    static constexpr uint32_t kAQs = BM * BK;
    // q8_0: d per (sub-block, row) as [kb][g][BM / 8] (load_a); q8_K: bsum32
    // per (row, sub-block), rows kAScaleStride words apart so that 8
    // consecutive rows hit 8 distinct banks.
    // (tensor-map stages: the q8_0 scales' [8][BM] box, no q8_K block scales)
    static constexpr uint32_t kAScale = kTma ? BM * 8 * 4 : BM * kAScaleStride * 4;
    static constexpr uint32_t kAD8K = kTma ? 0 : BM * 4;  // q8_K: d per row
    static constexpr uint32_t kWRaw = BN * kSlot;
    static constexpr uint32_t kStageRaw = kAQs + kAScale + kAD8K + kWRaw;
    static constexpr uint32_t kStage = kTma ? (kStageRaw + 1023) / 1024 * 1024 : kStageRaw;
    static_assert(!kTma || (BM % 32 == 0 && kSlot == 144), "tensor-map stages: 32-row multiples, 144-byte rows");
    static constexpr uint32_t kBTile = BN * BK;
    static constexpr uint32_t kFold = 8 * BN * 8;    // float2 (s, -M s) per (sub-block, column)
    static constexpr uint32_t kMin = BN * 16;        // q4_K: (dmin, -M dmin) and packed mins per column
    static constexpr uint32_t kAPack = BM * 16;      // q4_K: packed bsum bytes per row
    static constexpr uint32_t kGrid = 2048;          // iq2_xxs lattice table
    static constexpr uint32_t kSmem = ST * kStage + kBTile + kFold + kMin + kAPack + kGrid;
};

struct GemmParams {
    const uint8_t *w;
    SplitA a;
    float *c;
    int64_t ldc;
    int32_t *partials;
    int64_t m, n, k;
    int64_t row_bytes;    // bytes per weight row
    uint32_t step_bytes;  // raw weight bytes per row per k-step
    int w_vec16;          // 1: every row chunk is 16-byte aligned
    int64_t w_total;      // bytes of W
    int out_format;       // kOutF32 (C in c) or another output format (in out)
    void *out;
    int64_t ldo;          // elements (fp16 / bf16) or blocks (q8_0)
    // split-K: blockIdx.z takes k-steps [z ks_per_split, (z + 1) ks_per_split);
    // with splits > 1 every split writes its fp32 tile to partial [splits][m][n]
    // and a reduction sums them in split order
    int splits;
    int ks_per_split;
    float *partial;
    // fp32 C stored also to copies[0 .. ncopies) (same row stride ldc); c_vec4:
    // c, every copy and ldc allow 16-byte accesses of column quads
    float *copies[kMaxCopies];
    int ncopies;
    int c_vec4;
    // tile raster: 1 = blockIdx.x walks the m tiles (consecutive CTAs share
    // a W tile, which is then fetched from DRAM once), 0 = the n tiles
    int m_fast;
    int *err;  // library error word (bounded waits of the tensor-map stages)
};

// Origin (m0, n0) of this CTA's tile in the raster order of p.m_fast.
template <class C>
PFNG_DEV void tile_origin(const GemmParams &p, int64_t &m0, int64_t &n0) {
    const int64_t bx = blockIdx.x, by = blockIdx.y;
    m0 = (p.m_fast ? bx : by) * C::BM;
    n0 = (p.m_fast ? by : bx) * C::BN;
}

PFNG_DEV void cp_async16(void *dst, const void *src, uint32_t src_bytes) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(smem_u32(dst)), "l"(src), "r"(src_bytes)
                 : "memory");
}
PFNG_DEV void cp_async4(void *dst, const void *src, uint32_t src_bytes) {
    asm volatile("cp.async.ca.shared.global [%0], [%1], 4, %2;" ::"r"(smem_u32(dst)), "l"(src), "r"(src_bytes)
                 : "memory");
}
PFNG_DEV void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
PFNG_DEV void cp_async_wait() {
    asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

PFNG_DEV void ldmatrix_x4(uint32_t &r0, uint32_t &r1, uint32_t &r2, uint32_t &r3, const void *p) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
                 : "r"(smem_u32(p)));
}

PFNG_DEV void mma_s8(int (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1, int cin) {
    asm(
        "mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%10,%10,%10,%10};"
        : "=r"(d[0]), "=r"(d[1]), "=r"(d[2]), "=r"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1), "r"(cin));
}

// packed fp32 fma on two lanes of data: d = a * b + c, each rounded once
PFNG_DEV float2 ffma2(float2 a, float2 b, float2 c) { return __ffma2_rn(a, b, c); }

// byte offset of 16-byte chunk `chunk` of row `row` in a [rows][256 B] tile,
// XOR-swizzled so that ldmatrix over 8 rows touches 8 distinct bank groups.
PFNG_DEV uint32_t swz(int row, int chunk) { return static_cast<uint32_t>(row * 256 + ((chunk ^ (row & 7)) << 4)); }

template <class C>
struct Smem {
    uint8_t *base;
    PFNG_DEV uint8_t *stage(int s) const { return base + s * C::kStage; }
    PFNG_DEV int8_t *a_qs(int s) const { return reinterpret_cast<int8_t *>(stage(s)); }
    PFNG_DEV float *a_scale(int s) const { return reinterpret_cast<float *>(stage(s) + C::kAQs); }
    PFNG_DEV float *a_d8k(int s) const { return reinterpret_cast<float *>(stage(s) + C::kAQs + C::kAScale); }
    PFNG_DEV uint8_t *w_raw(int s) const { return stage(s) + C::kAQs + C::kAScale + C::kAD8K; }
    PFNG_DEV int8_t *b_tile() const { return reinterpret_cast<int8_t *>(base + C::ST * C::kStage); }
    PFNG_DEV float2 *fold() const { return reinterpret_cast<float2 *>(base + C::ST * C::kStage + C::kBTile); }
    PFNG_DEV float2 *mins_d() const {
        return reinterpret_cast<float2 *>(base + C::ST * C::kStage + C::kBTile + C::kFold);
    }
    PFNG_DEV uint2 *mins_pk() const { return reinterpret_cast<uint2 *>(mins_d() + C::BN); }
    PFNG_DEV uint4 *a_pack() const {
        return reinterpret_cast<uint4 *>(base + C::ST * C::kStage + C::kBTile + C::kFold + C::kMin);
    }
    PFNG_DEV uint2 *grid() const {
        return reinterpret_cast<uint2 *>(base + C::ST * C::kStage + C::kBTile + C::kFold + C::kMin + C::kAPack);
    }
};

// cp.async copies of k-step `ks` of the activation tile: int8 rows, the
// per-sub-block scales (q8_0) or sums (q8_K), and the q8_K block scales.
template <int WT, class C>
PFNG_DEV void load_a(const GemmParams &p, int8_t *a_qs, float *a_scale, float *a_d8k, int64_t ks, int64_t m0,
                     int tid) {
    const int64_t K = p.k;
    // A int8 rows: BM x 256 B
#pragma unroll
    for (int i = 0; i < C::BM * 16 / kThreads; ++i) {
        const int q = tid + i * kThreads;
        const int row = q >> 4, ch = q & 15;
        cp_async16(a_qs + swz(row, ch), p.a.qs + (m0 + row) * K + ks * BK + ch * 16, 16);
    }
    if (tid < C::BM * 2) {
        if constexpr (kQ8_0Act<WT>) {
            // q8_0 scales of the 8 blocks of k-step ks: stage layout
            // [kb][g][BM / 8], row 8 j + g of the tile at j (split_d_index's
            // order restricted to the tile's rows), BM / 32 chunks per (kb, g)
            constexpr int kChunks = C::BM / 32;
            const int kbg = tid / kChunks, c = tid % kChunks;
            const int kb = kbg >> 3, g = kbg & 7;
            const float *src = p.a.d + (ks * 8 + kb) * p.a.d_ld + (m0 & ~int64_t(127)) + g * 16 + ((m0 & 127) >> 3) + 4 * c;
            cp_async16(a_scale + kbg * (C::BM / 8) + 4 * c, src, 16);
        } else {
            const int row = tid >> 1, half = tid & 1;
            cp_async16(a_scale + row * kAScaleStride + half * 4, p.a.aux + (m0 + row) * (K / 32) + ks * 8 + half * 4, 16);
        }
    }
    if constexpr (!kQ8_0Act<WT>) {
        if (tid < C::BM) cp_async4(a_d8k + tid, p.a.d + (m0 + tid) * (K / 256) + ks, 4);
    }
}

// cp.async copies of k-step `ks` of the raw W tile: BN rows x step_bytes,
// each row into a C::kSlot-byte slot of `wr`.
template <int WT, class C>
PFNG_DEV void load_w(const GemmParams &p, uint8_t *wr, int64_t ks, int64_t n0, int tid) {
    const int64_t K = p.k;
    if constexpr (WT == kWQ4_0P) {
        // planar rows: the k-step's 8 nibble fields (128 B) into slot bytes
        // 0..127, their 8 fp16 scales (16 B) into bytes 128..143
        for (int q = tid; q < C::BN * 9; q += kThreads) {
            const int row = q / 9, ch = q % 9;
            const int64_t n = n0 + row;
            const bool ok = n < p.n;
            const int64_t off = ch < 8 ? ks * 128 + ch * 16 : K / 2 + ks * 16;
            const uint8_t *src = p.w + (ok ? n * p.row_bytes + off : 0);
            cp_async16(wr + row * C::kSlot + ch * 16, src, ok ? 16u : 0u);
        }
    } else if (p.w_vec16) {
        // 16-byte chunks per row and k-step: the raw bytes of 256 values
        constexpr int chunks = (WT == kWIQ2 ? 256 / 256 * kIQ2Bytes : 256 / 32 * kQ4_0Bytes) / 16;
        for (int q = tid; q < C::BN * chunks; q += kThreads) {
            const int row = q / chunks, ch = q % chunks;
            const int64_t n = n0 + row;
            const bool ok = n < p.n;
            const uint8_t *src = p.w + (ok ? n * p.row_bytes + ks * p.step_bytes + ch * 16 : 0);
            cp_async16(wr + row * C::kSlot + ch * 16, src, ok ? 16u : 0u);
        }
    } else {
        // word-granular window [start & ~3, start + step_bytes + 3) per row
        constexpr int kStep = WT == kWIQ2 ? kIQ2Bytes : (WT == kWQ4_K ? kQ4_KBytes : 256 / 32 * kQ4_0Bytes);
        constexpr int words = (kStep + 3) / 4 + 1;
        for (int q = tid; q < C::BN * words; q += kThreads) {
            const int row = q / words, wd = q % words;
            const int64_t n = n0 + row;
            const int64_t start = n * p.row_bytes + ks * p.step_bytes;
            const int64_t addr = (start & ~int64_t(3)) + 4 * wd;
            uint32_t bytes = 0;
            if (n < p.n && addr < p.w_total) bytes = p.w_total - addr >= 4 ? 4u : static_cast<uint32_t>(p.w_total - addr);
            cp_async4(wr + row * C::kSlot + 4 * wd, p.w + (bytes ? addr : 0), bytes);
        }
    }
}

// Issue the cp.async copies of k-step `ks` into stage `s`.
template <int WT, class C>
PFNG_DEV void load_stage(const GemmParams &p, const Smem<C> &sm, int s, int64_t ks, int64_t m0, int64_t n0, int tid) {
    load_a<WT, C>(p, sm.a_qs(s), sm.a_scale(s), sm.a_d8k(s), ks, m0, tid);
    load_w<WT, C>(p, sm.w_raw(s), ks, n0, tid);
}

PFNG_DEV uint32_t scale_byte(uint32_t s0, uint32_t s1, uint32_t s2, int i) {
    const uint32_t w = i < 4 ? s0 : (i < 8 ? s1 : s2);
    return (w >> (8 * (i & 3))) & 0xffu;
}

// Store two 16-byte chunks of one B-tile row.  The 8 threads that decode a
// row store together; `swap` picks which chunk goes first so that each of the
// two stores covers all 8 bank groups once (no 2-way conflict).
PFNG_DEV void store_pair(int8_t *bt, int row, int ca, uint4 va, int cb, uint4 vb, bool swap) {
    const int c0 = swap ? cb : ca, c1 = swap ? ca : cb;
    const uint4 v0 = swap ? vb : va, v1 = swap ? va : vb;
    *reinterpret_cast<uint4 *>(bt + swz(row, c0)) = v0;
    *reinterpret_cast<uint4 *>(bt + swz(row, c1)) = v1;
}

// Fold constants of sub-block u, column `col`: s and -(2^23 + 2^22) s, stored
// per column pair as {s_c, s_c+1, cm_c, cm_c+1} so that a thread's two
// adjacent columns read both packed-fma operands with one 16-byte load.
PFNG_DEV void store_fold(float *fold, int bn, int u, int col, float sv) {
    float *q = fold + (u * bn + (col & ~1)) * 2 + (col & 1);
    q[0] = sv;
    q[2] = -kMagic * sv;
}

// One decode task (row = task / 8, 32-value unit u = task % 8) of the raw W
// tile `wr` into the int8 B tile and the fold constants.  q4_K tasks with
// u == 0 also write the row's (dmin, -M dmin) pair and packed 6-bit mins to
// mins_d / mins_pk; no type's decode reads the activations.
// kTile = false (q4_K with direct operands): only the fold constants and
// the mins, no B tile.  kSlot: bytes per raw W row.
template <int WT, int BN, bool kTile = true, uint32_t kSlot = kWRowSlot>
PFNG_DEV void decode_task(const GemmParams &p, const uint8_t *wr, int8_t *bt, float *fold, const uint2 *grid,
                          int64_t ks, int64_t n0, int task, float *mins_d = nullptr, uint2 *mins_pk = nullptr) {
    static_assert(kTile || WT == kWQ4_K, "scales-only decode: q4_K");
    const int row = task >> 3, u = task & 7;
    const uint32_t mis = p.w_vec16 ? 0u : static_cast<uint32_t>((n0 + row) * p.row_bytes + ks * p.step_bytes) & 3u;
    const uint32_t base = row * kSlot + mis;
    if constexpr (WT == kWQ4_0 || WT == kWQ4_0P) {
        uint32_t q[4], dbits;
        if constexpr (WT == kWQ4_0) {
            load_q4_0_block_smem(wr, base + 18u * u, q, dbits);
        } else {
            const uint4 v = *reinterpret_cast<const uint4 *>(wr + base + 16u * u);
            q[0] = v.x, q[1] = v.y, q[2] = v.z, q[3] = v.w;
            dbits = *reinterpret_cast<const uint16_t *>(wr + base + 128u + 2u * u);
        }
        // nibble - 8 per byte: for b in 0..15, b + 0x78 stays below 0x100
        // (no carry into the next byte) and flipping bit 7 gives b - 8
        uint4 lo, hi;
        lo.x = ((q[0] & 0x0f0f0f0fu) + 0x78787878u) ^ 0x80808080u;
        lo.y = ((q[1] & 0x0f0f0f0fu) + 0x78787878u) ^ 0x80808080u;
        lo.z = ((q[2] & 0x0f0f0f0fu) + 0x78787878u) ^ 0x80808080u;
        lo.w = ((q[3] & 0x0f0f0f0fu) + 0x78787878u) ^ 0x80808080u;
        hi.x = (((q[0] >> 4) & 0x0f0f0f0fu) + 0x78787878u) ^ 0x80808080u;
        hi.y = (((q[1] >> 4) & 0x0f0f0f0fu) + 0x78787878u) ^ 0x80808080u;
        hi.z = (((q[2] >> 4) & 0x0f0f0f0fu) + 0x78787878u) ^ 0x80808080u;
        hi.w = (((q[3] >> 4) & 0x0f0f0f0fu) + 0x78787878u) ^ 0x80808080u;
        store_pair(bt, row, 2 * u, lo, 2 * u + 1, hi, u >= 4);
        store_fold(fold, BN, u, row, f16_bits_to_f32(dbits));
    } else if constexpr (WT == kWQ4_K) {
        // u = (nibble pair pr, half h): 16 payload bytes -> 16 values of sub-blocks 2pr and 2pr+1
        const uint8_t *blk = wr + base;
        if constexpr (kTile) {
            const int pr = u >> 1, h = u & 1;
            const uint4 v = *reinterpret_cast<const uint4 *>(blk + 16 + 32 * pr + 16 * h);
            uint4 lo, hi;
            lo.x = v.x & 0x0f0f0f0fu, lo.y = v.y & 0x0f0f0f0fu, lo.z = v.z & 0x0f0f0f0fu, lo.w = v.w & 0x0f0f0f0fu;
            hi.x = (v.x >> 4) & 0x0f0f0f0fu, hi.y = (v.y >> 4) & 0x0f0f0f0fu;
            hi.z = (v.z >> 4) & 0x0f0f0f0fu, hi.w = (v.w >> 4) & 0x0f0f0f0fu;
            // sub-block 2pr holds k = 64 pr + j, sub-block 2pr + 1 holds k = 64 pr + 32 + j
            store_pair(bt, row, 4 * pr + h, lo, 4 * pr + 2 + h, hi, pr >= 2);
        }
        // scale / min of sub-block u (llama_reference.cpp:116-121)
        const uint32_t dd = *reinterpret_cast<const uint32_t *>(blk);
        const uint32_t s0 = *reinterpret_cast<const uint32_t *>(blk + 4);
        const uint32_t s1 = *reinterpret_cast<const uint32_t *>(blk + 8);
        const uint32_t s2 = *reinterpret_cast<const uint32_t *>(blk + 12);
        uint32_t scv;
        if (u < 4)
            scv = scale_byte(s0, s1, s2, u) & 63u;
        else
            scv = (scale_byte(s0, s1, s2, u + 4) & 15u) | ((scale_byte(s0, s1, s2, u - 4) >> 6) << 4);
        const float sv = __fmul_rn(f16_bits_to_f32(dd & 0xffffu), static_cast<float>(scv));
        store_fold(fold, BN, u, row, sv);
        if (u == 0) {
            uint32_t mpk0 = 0, mpk1 = 0;
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                const uint32_t mnv = j < 4 ? scale_byte(s0, s1, s2, j + 4) & 63u
                                           : (scale_byte(s0, s1, s2, j + 4) >> 4) | ((scale_byte(s0, s1, s2, j) >> 6) << 4);
                if (j < 4)
                    mpk0 |= mnv << (8 * j);
                else
                    mpk1 |= mnv << (8 * (j - 4));
            }
            const float dmin = f16_bits_to_f32(dd >> 16);
            store_fold(mins_d, 0, 0, row, dmin);
            mins_pk[row] = make_uint2(mpk0, mpk1);
        }
    } else {
        // iq2_xxs: 32-value group u of the 66-byte block
        const uint32_t off = base + 2 + 8 * u;
        const uint32_t *w = reinterpret_cast<const uint32_t *>(wr + (off & ~3u));
        const uint32_t sh = (off & 2u) ? 16u : 0u;
        const uint32_t idx = __funnelshift_r(w[0], w[1], sh);
        const uint32_t ss = __funnelshift_r(w[1], w[2], sh);
        uint32_t v[8];
#pragma unroll
        for (int g = 0; g < 4; ++g) {
            const uint2 gv = grid[(idx >> (8 * g)) & 0xffu];
            const uint32_t sgn = iq2_sign_mask((ss >> (7 * g)) & 0x7fu);
            v[2 * g] = apply_sign_bytes(gv.x, expand_bits4(sgn));
            v[2 * g + 1] = apply_sign_bytes(gv.y, expand_bits4(sgn >> 4));
        }
        store_pair(bt, row, 2 * u, make_uint4(v[0], v[1], v[2], v[3]), 2 * u + 1, make_uint4(v[4], v[5], v[6], v[7]),
                   u >= 4);
        const float d = f16_bits_to_f32(*reinterpret_cast<const uint16_t *>(wr + base));
        const float sv = __fmul_rn(__fmul_rn(0.125f, d), static_cast<float>(2 * (ss >> 28) + 1));
        store_fold(fold, BN, u, row, sv);
    }
}

// q4_K min term, A side: the 8 sub-block sums of a row's q8_K activations
// split into 6-bit low bytes and high bytes (sum = lo + 64 hi), packed for
// dp4a against the packed 6-bit mins.
PFNG_DEV uint4 pack_bsum(const int32_t *bsum) {
    uint32_t l0 = 0, l1 = 0, h0 = 0, h1 = 0;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
        const int v = bsum[j];
        const uint32_t lo = static_cast<uint32_t>(v & 63), hi = static_cast<uint32_t>(v >> 6) & 0xffu;
        if (j < 4)
            l0 |= lo << (8 * j), h0 |= hi << (8 * j);
        else
            l1 |= lo << (8 * (j - 4)), h1 |= hi << (8 * (j - 4));
    }
    return make_uint4(l0, l1, h0, h1);
}

// Unpack the raw W tile of stage `s` into the int8 B tile and the
// per-(sub-block, column) fold data.  Runs once per CTA per k-step.
template <int WT, class C, bool kTile = true>
PFNG_DEV void decode_w(const GemmParams &p, const Smem<C> &sm, int s, int64_t ks, int64_t n0, int tid) {
    const uint8_t *wr = sm.w_raw(s);
    int8_t *bt = sm.b_tile();
    float *fold = reinterpret_cast<float *>(sm.fold());
    for (int task = tid; task < C::BN * 8; task += kThreads)
        decode_task<WT, C::BN, kTile, C::kSlot>(p, wr, bt, fold, sm.grid(), ks, n0, task,
                                                reinterpret_cast<float *>(sm.mins_d()), sm.mins_pk());
    if constexpr (WT == kWQ4_K) {
        for (int r = tid; r < C::BM; r += kThreads)
            sm.a_pack()[r] = pack_bsum(reinterpret_cast<const int32_t *>(sm.a_scale(s)) + r * kAScaleStride);
    }
}

// A and B fragments of sub-block kb for this warp's MT x NT m16n8k32 tiles.
PFNG_DEV void ldmatrix_x4_s(uint32_t &r0, uint32_t &r1, uint32_t &r2, uint32_t &r3, uint32_t addr) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
                 : "r"(addr));
}

// This thread's ldmatrix row offsets in a swizzled [rows][256 B] tile.
// swz(row, 2 kb + h) = row * 256 + ((2 kb + h) ^ (row & 7)) * 16 and the
// fragment rows have row & 7 = lane & 7, so the offset of sub-block kb is
// off ^ (32 kb) with off = row * 256 + ((h ^ (lane & 7)) << 4): one xor per
// load instead of the swizzle arithmetic.
template <class C>
struct FragOff {
    uint32_t a[C::MT];
    uint32_t b[C::NT / 2];
    PFNG_DEV FragOff(int wm, int wn, int lane) {
#pragma unroll
        for (int mt = 0; mt < C::MT; ++mt) {
            const int row = wm * C::WM + mt * 16 + (lane & 7) + ((lane >> 3) & 1) * 8;
            // tensor-map stages: 128-byte rows per half (a_off)
            a[mt] = static_cast<uint32_t>(row * (C::kTma ? 128 : 256) + ((((lane >> 4) & 1) ^ (lane & 7)) << 4));
        }
#pragma unroll
        for (int np = 0; np < C::NT / 2; ++np) {
            const int row = wn * C::WN + np * 16 + (lane & 7) + ((lane >> 4) & 1) * 8;
            b[np] = static_cast<uint32_t>(row * 256 + ((((lane >> 3) & 1) ^ (lane & 7)) << 4));
        }
    }
};

// load_frags from shared-space base addresses and precomputed offsets.
template <class C>
PFNG_DEV void load_frags_o(uint32_t at_s, uint32_t bt_s, int kb, const FragOff<C> &fo, uint32_t (&af)[C::MT][4],
                           uint32_t (&bf)[C::NT][2]) {
    const uint32_t x = static_cast<uint32_t>(kb) * 32u;
#pragma unroll
    for (int mt = 0; mt < C::MT; ++mt) ldmatrix_x4_s(af[mt][0], af[mt][1], af[mt][2], af[mt][3], at_s + (fo.a[mt] ^ x));
#pragma unroll
    for (int np = 0; np < C::NT / 2; ++np)
        ldmatrix_x4_s(bf[2 * np][0], bf[2 * np][1], bf[2 * np + 1][0], bf[2 * np + 1][1], bt_s + (fo.b[np] ^ x));
}

// Direct operands for q4_0 in either layout (kDirect): the
// m16n8k32 B fragment of thread (g, t4) holds column g's values
// k = 4 t4 .. 4 t4 + 3 and 16 + 4 t4 .. 16 + 4 t4 + 3 of the sub-block,
// which in a q4_0 block are the low and high nibbles of qs[4 t4 .. 4 t4 + 3]:
// one 32-bit word of the raw W tile gives both registers, with no B tile,
// no decode pass and no barrier between them.  Rows of the raw tile start
// 16-byte aligned (w_vec16 or planar), a ggml block's qs at 18 kb + 2.
template <int WT>
PFNG_DEV uint32_t raw_q4_word(const uint8_t *row, int kb, int t4) {
    if constexpr (WT == kWQ4_0P) {
        return *reinterpret_cast<const uint32_t *>(row + 16 * kb + 4 * t4);
    } else {
        const uint16_t *h = reinterpret_cast<const uint16_t *>(row + 18 * kb + 2 + 4 * t4);
        return static_cast<uint32_t>(h[0]) | (static_cast<uint32_t>(h[1]) << 16);
    }
}
template <int WT>
PFNG_DEV uint32_t raw_q4_scale(const uint8_t *row, int kb) {
    return *reinterpret_cast<const uint16_t *>(row + (WT == kWQ4_0P ? 128 + 2 * kb : 18 * kb));
}
template <int WT, class C>
PFNG_DEV void load_frags_direct(uint32_t at_s, const uint8_t *wr, int kb, const FragOff<C> &fo, int wn, int g, int t4,
                                uint32_t (&af)[C::MT][4], uint32_t (&bf)[C::NT][2]) {
    if constexpr (C::kTma) {
        // [half][row][128 B] with the 128-byte swizzle: sub-block kb is
        // 16-byte chunks 2 (kb & 3) + {0, 1} of half kb / 4
        const uint32_t half = at_s + static_cast<uint32_t>(kb >> 2) * (C::BM * 128u);
        const uint32_t x = static_cast<uint32_t>(kb & 3) * 32u;
#pragma unroll
        for (int mt = 0; mt < C::MT; ++mt)
            ldmatrix_x4_s(af[mt][0], af[mt][1], af[mt][2], af[mt][3], half + (fo.a[mt] ^ x));
    } else {
        const uint32_t x = static_cast<uint32_t>(kb) * 32u;
#pragma unroll
        for (int mt = 0; mt < C::MT; ++mt)
            ldmatrix_x4_s(af[mt][0], af[mt][1], af[mt][2], af[mt][3], at_s + (fo.a[mt] ^ x));
    }
#pragma unroll
    for (int nt = 0; nt < C::NT; ++nt) {
        const uint8_t *row = wr + (wn * C::WN + nt * 8 + g) * C::kSlot;
        if constexpr (WT == kWQ4_K) {
            // sub-block 2 pr + h is nibble h of qs[32 pr + j], j = 0..31 (values 0..15, no offset)
            const uint8_t *q = row + 16 + 32 * (kb >> 1) + 4 * t4;
            const int sh = (kb & 1) * 4;
            bf[nt][0] = (*reinterpret_cast<const uint32_t *>(q) >> sh) & 0x0f0f0f0fu;
            bf[nt][1] = (*reinterpret_cast<const uint32_t *>(q + 16) >> sh) & 0x0f0f0f0fu;
        } else {
            const uint32_t q = raw_q4_word<WT>(row, kb, t4);
            bf[nt][0] = ((q & 0x0f0f0f0fu) + 0x78787878u) ^ 0x80808080u;
            bf[nt][1] = (((q >> 4) & 0x0f0f0f0fu) + 0x78787878u) ^ 0x80808080u;
        }
    }
}

template <class C>
PFNG_DEV void load_frags(const int8_t *at, const int8_t *bt, int kb, int wm, int wn, int lane,
                         uint32_t (&af)[C::MT][4], uint32_t (&bf)[C::NT][2]) {
#pragma unroll
    for (int mt = 0; mt < C::MT; ++mt) {
        const int row = wm * C::WM + mt * 16 + (lane & 7) + ((lane >> 3) & 1) * 8;
        ldmatrix_x4(af[mt][0], af[mt][1], af[mt][2], af[mt][3], at + swz(row, 2 * kb + (lane >> 4)));
    }
#pragma unroll
    for (int np = 0; np < C::NT / 2; ++np) {
        const int row = wn * C::WN + np * 16 + (lane & 7) + ((lane >> 4) & 1) * 8;
        ldmatrix_x4(bf[2 * np][0], bf[2 * np][1], bf[2 * np + 1][0], bf[2 * np + 1][1],
                    bt + swz(row, 2 * kb + ((lane >> 3) & 1)));
    }
}

template <class C>
PFNG_DEV void epilogue_q8_0(const GemmParams &p, uint8_t *smem, const float2 (&acc)[C::MT][C::NT][2], int64_t m0,
                            int64_t n0, int tid);
PFNG_DEV void store_out2(const GemmParams &p, int64_t r, int64_t c, float2 v);
// fp32 C to the copies as well (kernels instantiated with kCopies): after
// the epilogue the CTA reads its finished tile back from C (in L2) and
// stores it to every copy in 16-byte pieces along rows, all of a thread's
// loads issued before its stores; a system-scope fence then makes the stores
// performed before the kernel ends, so that a collective the caller orders
// after this kernel publishes them.  Only the kCopies kernels carry this
// code: inlined into the kernels without copies, a copies loop cost the
// 2048 x 11008 x 4096 GEMM 35 % (626 -> 845 us).
template <class C>
PFNG_DEV void copy_tile_to_copies(const GemmParams &p) {
    if (p.ncopies == 0) return;
    // the tile origin from the special registers: nothing of it stays live
    // across the main loop
    int64_t m0, n0;
    tile_origin<C>(p, m0, n0);
    const int tid = threadIdx.x;
    const int rows = static_cast<int>(p.m - m0 < C::BM ? p.m - m0 : C::BM);
    const int cols = static_cast<int>(p.n - n0 < C::BN ? p.n - n0 : C::BN);
    constexpr int kQuads = C::BN / 4;
    constexpr int kPer = C::BM * kQuads / kThreads;
    static_assert(C::BM * kQuads % kThreads == 0, "whole tile rounds");
    __syncthreads();  // the whole tile is in C
    if (p.c_vec4 && cols == C::BN) {
        float4 v[kPer];
#pragma unroll
        for (int j = 0; j < kPer; ++j) {
            const int i = tid + j * kThreads, r = i / kQuads;
            if (r < rows) v[j] = *reinterpret_cast<const float4 *>(p.c + (m0 + r) * p.ldc + n0 + (i % kQuads) * 4);
        }
        for (int d = 0; d < p.ncopies; ++d) {
#pragma unroll
            for (int j = 0; j < kPer; ++j) {
                const int i = tid + j * kThreads, r = i / kQuads;
                if (r < rows) *reinterpret_cast<float4 *>(p.copies[d] + (m0 + r) * p.ldc + n0 + (i % kQuads) * 4) = v[j];
            }
        }
    } else {
        for (int i = tid; i < rows * C::BN; i += kThreads) {
            const int r = i / C::BN, col = i % C::BN;
            if (col >= cols) continue;
            const float v = p.c[(m0 + r) * p.ldc + n0 + col];
            for (int d = 0; d < p.ncopies; ++d) p.copies[d][(m0 + r) * p.ldc + n0 + col] = v;
        }
    }
    __threadfence_system();
}

// Tensor maps of a Cfg::kTma launch (unused otherwise): the split
// operand's int8 rows, the raw W rows, the split operand's q8_0 scales.
struct TmaMaps {
    CUtensorMap a, w, ad;
};

// Bounded wait on a stage barrier of a Cfg::kTma kernel: false once the
// CTA's abort flag is up, or after about a second, when it records `code`
// and raises the flag so that every other wait of the CTA ends too.
PFNG_DEV bool stage_wait(uint64_t *bar, uint32_t parity, int *abort_flag, int *err, int code) {
    volatile int *ab = abort_flag;
    for (uint32_t i = 0; i < kWaitAttempts; ++i) {
        if (mbar_try_wait(bar, parity)) return true;
        if (*ab) return false;
    }
    report_error(err, code);
    *ab = 1;
    return false;
}

template <int WT, class C, bool kPartials, bool kCopies = false, bool kDirect = false>
__global__ void __launch_bounds__(kThreads, kDirect && (C::BM == 64 || (C::BM == 32 && WT == kWQ4_K)) ? 2 : 1)
    gemm_kernel(const __grid_constant__ TmaMaps maps, const GemmParams p) {
    static_assert(!kDirect || WT == kWQ4_0 || WT == kWQ4_0P || WT == kWQ4_K, "direct operands: q4_0 and q4_K");
    static_assert(!C::kTma || (kDirect && WT == kWQ4_0), "tensor-map stages: direct q4_0 operands");
    extern __shared__ __align__(128) uint8_t smem_raw[];
    // tensor-map stages start on a 1024-byte boundary (the 128-byte swizzle;
    // the launch adds the slack)
    const Smem<C> sm{C::kTma ? smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u) : smem_raw};
    // Cfg::kTma: stage s holds its k-step once tma_full[s] completes, and is
    // free for the next copies once every warp has arrived on tma_empty[s]
    __shared__ uint64_t tma_full[C::ST], tma_empty[C::ST];
    __shared__ int tma_abort;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int wm = warp / C::WGN, wn = warp % C::WGN;
    const int g = lane >> 2, t4 = lane & 3;
    int64_t m0, n0;
    tile_origin<C>(p, m0, n0);
    const int64_t KT = p.k / BK;
    constexpr int MT = C::MT, NT = C::NT;
    const FragOff<C> fo(wm, wn, lane);

    if constexpr (WT == kWIQ2) {
        uint2 *grid = sm.grid();
        for (int i = tid; i < 256; i += kThreads) {
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

    float2 acc[MT][NT][2];  // [.][.][0]: row g, cols (2 t4, 2 t4 + 1); [1]: row g + 8
#pragma unroll
    for (int a = 0; a < MT; ++a)
#pragma unroll
        for (int b = 0; b < NT; ++b) acc[a][b][0] = acc[a][b][1] = make_float2(0.0f, 0.0f);
    const int cin = kPartials ? 0 : static_cast<int>(kMagicBits);

    // this CTA's k-steps [k0, k1) (the whole range without split-K)
    const int64_t k0 = static_cast<int64_t>(blockIdx.z) * p.ks_per_split;
    const int64_t k1 = k0 + p.ks_per_split < KT ? k0 + p.ks_per_split : KT;
    constexpr int ST = C::ST;

    // The kernel is a programmatic dependent of the activation quantizer: the
    // weights of the first stages are fetched before waiting for it, the
    // activations after.  Group s holds A[s] (group 0 also every W prologue
    // stage), so the wait_group accounting of the loop is unchanged.
    // Cfg::kTma: thread 0 issues every stage's copies; bytes one stage lands
    constexpr uint32_t kTmaTx = C::BM * BK + C::BN * 144u + C::BM * 8u * 4u;
    int tma_issued = 0, tma_used = 0;  // (thread 0) k-steps issued / consumed
    auto tma_w = [&](int st, int64_t ks) {
        mbar_arrive_expect_tx(&tma_full[st], kTmaTx);
        tma_load_2d(smem_u32(sm.w_raw(st)), &maps.w, static_cast<int>(ks * p.step_bytes), static_cast<int>(n0),
                    &tma_full[st]);
    };
    auto tma_a = [&](int st, int64_t ks) {
        const uint32_t a = smem_u32(sm.a_qs(st));
        tma_load_2d(a, &maps.a, static_cast<int>(ks * BK), static_cast<int>(m0), &tma_full[st]);
        tma_load_2d(a + C::BM * 128u, &maps.a, static_cast<int>(ks * BK + 128), static_cast<int>(m0), &tma_full[st]);
        if constexpr (C::BM == 128)  // the tile's 128-row group of the scales: a 2-D box
            tma_load_2d(smem_u32(sm.a_scale(st)), &maps.ad, static_cast<int>(m0), static_cast<int>(ks * 8),
                        &tma_full[st]);
        else  // j (BM / 8 of the group's 16), g, group, block
            tma_load_4d(smem_u32(sm.a_scale(st)), &maps.ad, static_cast<int>((m0 & 127) >> 3), 0,
                        static_cast<int>(m0 >> 7), static_cast<int>(ks * 8), &tma_full[st]);
    };
    if constexpr (C::kTma) {
        if (tid == 0) {
            for (int i = 0; i < ST; ++i) {
                mbar_init(&tma_full[i], 1);
                mbar_init(&tma_empty[i], kThreads / 32);
            }
            fence_mbar_init();
            tma_abort = 0;
            prefetch_map(&maps.a);
            prefetch_map(&maps.w);
            prefetch_map(&maps.ad);
        }
        __syncthreads();
        if (tid == 0)
            for (int s = 0; s < ST - 1; ++s)
                if (k0 + s < k1) tma_w(s, k0 + s);
        pdl_wait();
        if (tid == 0)
            for (int s = 0; s < ST - 1; ++s)
                if (k0 + s < k1) {
                    tma_a(s, k0 + s);
                    ++tma_issued;
                }
    } else {
#pragma unroll
        for (int s = 0; s < ST - 1; ++s)
            if (k0 + s < k1) load_w<WT, C>(p, sm.w_raw(s), k0 + s, n0, tid);
        pdl_wait();
#pragma unroll
        for (int s = 0; s < ST - 1; ++s) {
            if (k0 + s < k1) load_a<WT, C>(p, sm.a_qs(s), sm.a_scale(s), sm.a_d8k(s), k0 + s, m0, tid);
            cp_async_commit();
        }
    }

    for (int64_t ks = k0; ks < k1; ++ks) {
        const int s = static_cast<int>((ks - k0) % ST);
        if constexpr (C::kTma) {
            // refill the stage of k-step ks - 1 (free once every warp has
            // arrived on it) with k-step ks + ST - 1, then wait for k-step ks
            const int i = static_cast<int>(ks - k0);
            if (tid == 0 && ks + ST - 1 < k1) {
                const int j = i + ST - 1, t = j % ST;
                if (j < ST || stage_wait(&tma_empty[t], ((j / ST) - 1) & 1, &tma_abort, p.err, kErrWaitEmpty)) {
                    tma_w(t, ks + ST - 1);
                    tma_a(t, ks + ST - 1);
                    ++tma_issued;
                }
            }
            if (!stage_wait(&tma_full[s], (i / ST) & 1, &tma_abort, p.err, kErrWaitFull)) break;
            if (tid == 0) ++tma_used;
        } else {
            cp_async_wait<ST - 2>();
            __syncthreads();
            // q4_K with direct operands still decodes its 6-bit scales and mins
            // (fold constants, min term) -- everything but the B tile
            if constexpr (!kDirect)
                decode_w<WT, C>(p, sm, s, ks, n0, tid);
            else if constexpr (WT == kWQ4_K)
                decode_w<WT, C, false>(p, sm, s, ks, n0, tid);
            if (ks + ST - 1 < k1)
                load_stage<WT, C>(p, sm, static_cast<int>((ks - k0 + ST - 1) % ST), ks + ST - 1, m0, n0, tid);
            cp_async_commit();
            if constexpr (!kDirect || WT == kWQ4_K) __syncthreads();
        }

        const int8_t *at = sm.a_qs(s);
        const int8_t *bt = sm.b_tile();
        // activation block scales of this thread's rows (q8_K: one per 256 block)
        float da8k[MT][2];
        if constexpr (!kQ8_0Act<WT>) {
#pragma unroll
            for (int mt = 0; mt < MT; ++mt)
#pragma unroll
                for (int h = 0; h < 2; ++h) da8k[mt][h] = sm.a_d8k(s)[wm * C::WM + mt * 16 + g + 8 * h];
        }
        if constexpr (kPartials) {
#pragma unroll 1
            for (int kb = 0; kb < 8; ++kb) {
                uint32_t af[MT][4], bf[NT][2];
                if constexpr (kDirect)
                    load_frags_direct<WT, C>(smem_u32(at), sm.w_raw(s), kb, fo, wn, g, t4, af, bf);
                else
                    load_frags<C>(at, bt, kb, wm, wn, lane, af, bf);
                const int64_t nb32 = p.k / 32;
#pragma unroll
                for (int mt = 0; mt < MT; ++mt)
#pragma unroll
                    for (int nt = 0; nt < NT; ++nt) {
                        int res[4];
                        mma_s8(res, af[mt], bf[nt][0], bf[nt][1], 0);
#pragma unroll
                        for (int i = 0; i < 4; ++i) {
                            const int64_t r = m0 + wm * C::WM + mt * 16 + g + 8 * (i >> 1);
                            const int64_t c = n0 + wn * C::WN + nt * 8 + 2 * t4 + (i & 1);
                            if (r < p.m && c < p.n) p.partials[(r * p.n + c) * nb32 + ks * 8 + kb] = res[i];
                        }
                    }
            }
        } else {
            // Software pipeline over the 8 sub-blocks: the MMAs of sub-block
            // kb + 1 are issued fragment by fragment right after the fold of
            // sub-block kb has consumed that fragment's registers, and the
            // operands of kb + 2 are fetched while kb is folded, so tensor,
            // FMA and shared-memory pipes overlap inside one warp.
            uint32_t af[2][MT][4], bf[2][NT][2];
            int res[MT][NT][4];
            const uint32_t at_s = smem_u32(at), bt_s = smem_u32(bt);
            const uint8_t *wr = sm.w_raw(s);
            auto frags = [&](int kb, uint32_t(&a)[MT][4], uint32_t(&b)[NT][2]) {
                if constexpr (kDirect)
                    load_frags_direct<WT, C>(at_s, wr, kb, fo, wn, g, t4, a, b);
                else
                    load_frags_o<C>(at_s, bt_s, kb, fo, a, b);
            };
            // The per-sub-block scales of the fold are fetched one sub-block
            // ahead as well: the activation scales of this thread's rows
            // (dan) and, with direct operands, the two fp16 weight scales of
            // each column pair packed in one word (shs); measured on B200,
            // 2048x32000x4096 1641 -> 1618 us, 2048x11008x4096 598 -> 589 us,
            // same bits.
            uint32_t shs[2][NT];
            float dan[2][MT][2];
            // the q8_0 scales of this thread's rows for sub-block kb: rows
            // wm WM + 16 mt + 8 h + g sit at j = wm WM / 8 + 2 mt + h of
            // the stage's [kb][g][BM / 8] layout, four per 16-byte load
            auto load_da = [&](int kb, float(&d)[MT][2]) {
                if constexpr (kQ8_0Act<WT>) {
                    const float *base = sm.a_scale(s) + (kb * 8 + g) * (C::BM / 8) + wm * (C::WM / 8);
                    if constexpr (MT % 2 == 0) {
#pragma unroll
                        for (int q = 0; q < MT / 2; ++q) {
                            const float4 v = *reinterpret_cast<const float4 *>(base + 4 * q);
                            d[2 * q][0] = v.x, d[2 * q][1] = v.y, d[2 * q + 1][0] = v.z, d[2 * q + 1][1] = v.w;
                        }
                    } else {
                        static_assert(MT == 1, "one m16 fragment per warp, or an even count");
                        const float2 v = *reinterpret_cast<const float2 *>(base);
                        d[0][0] = v.x, d[0][1] = v.y;
                    }
                } else {
#pragma unroll
                    for (int mt = 0; mt < MT; ++mt)
#pragma unroll
                        for (int h = 0; h < 2; ++h) d[mt][h] = da8k[mt][h];
                }
            };
            load_da(0, dan[0]);
            if constexpr (kDirect && WT != kWQ4_K) {
#pragma unroll
                for (int nt = 0; nt < NT; ++nt) {
                    const uint8_t *row = wr + (wn * C::WN + nt * 8 + 2 * t4) * C::kSlot;
                    shs[0][nt] = raw_q4_scale<WT>(row, 0) | (raw_q4_scale<WT>(row + C::kSlot, 0) << 16);
                }
            }
            frags(0, af[0], bf[0]);
#pragma unroll
            for (int mt = 0; mt < MT; ++mt)
#pragma unroll
                for (int nt = 0; nt < NT; ++nt) mma_s8(res[mt][nt], af[0][mt], bf[0][nt][0], bf[0][nt][1], cin);
            frags(1, af[1], bf[1]);
#pragma unroll
            for (int kb = 0; kb < 8; ++kb) {
                const int nx = (kb + 1) & 1;
                float da[MT][2];
#pragma unroll
                for (int mt = 0; mt < MT; ++mt)
#pragma unroll
                    for (int h = 0; h < 2; ++h) da[mt][h] = dan[kb & 1][mt][h];
                if (kb + 1 < 8) load_da(kb + 1, dan[nx]);
                const float2 *fold = sm.fold() + kb * C::BN;
                if constexpr (kDirect && WT != kWQ4_K) {
                    if (kb + 1 < 8) {
#pragma unroll
                        for (int nt = 0; nt < NT; ++nt) {
                            const uint8_t *row = wr + (wn * C::WN + nt * 8 + 2 * t4) * C::kSlot;
                            shs[nx][nt] = raw_q4_scale<WT>(row, kb + 1) | (raw_q4_scale<WT>(row + C::kSlot, kb + 1) << 16);
                        }
                    }
                }
#pragma unroll
                for (int nt = 0; nt < NT; ++nt) {
                    float2 sv, cm;
                    if constexpr (kDirect && WT != kWQ4_K) {
                        const uint32_t sh = shs[kb & 1][nt];
                        sv = make_float2(f16_bits_to_f32(sh & 0xffffu), f16_bits_to_f32(sh >> 16));
                        cm = make_float2(-kMagic * sv.x, -kMagic * sv.y);
                    } else {
                        const float4 f = *reinterpret_cast<const float4 *>(fold + wn * C::WN + nt * 8 + 2 * t4);
                        sv = make_float2(f.x, f.y);
                        cm = make_float2(f.z, f.w);
                    }
#pragma unroll
                    for (int mt = 0; mt < MT; ++mt) {
#pragma unroll
                        for (int h = 0; h < 2; ++h) {
                            const float2 y = make_float2(__int_as_float(res[mt][nt][2 * h]),
                                                         __int_as_float(res[mt][nt][2 * h + 1]));
                            const float2 t = ffma2(y, sv, cm);
                            acc[mt][nt][h] = ffma2(t, make_float2(da[mt][h], da[mt][h]), acc[mt][nt][h]);
                        }
                        if (kb + 1 < 8) mma_s8(res[mt][nt], af[nx][mt], bf[nx][nt][0], bf[nx][nt][1], cin);
                    }
                }
                if (kb + 2 < 8) frags(kb + 2, af[kb & 1], bf[kb & 1]);
            }
        }

        if constexpr (!kPartials && WT == kWQ4_K) {
            // once per 256 block: acc -= a_d * dmin * sum_sb min_sb * bsum_sb
#pragma unroll
            for (int mt = 0; mt < MT; ++mt)
#pragma unroll
                for (int h = 0; h < 2; ++h) {
                    const int row = wm * C::WM + mt * 16 + g + 8 * h;
                    const uint4 ap = sm.a_pack()[row];
                    const float nad = -da8k[mt][h];
#pragma unroll
                    for (int nt = 0; nt < NT; ++nt) {
                        const int col = wn * C::WN + nt * 8 + 2 * t4;
                        int i2[2];
#pragma unroll
                        for (int e = 0; e < 2; ++e) {
                            const uint2 mv = sm.mins_pk()[col + e];
                            const int lo = __dp4a(static_cast<int>(mv.x), static_cast<int>(ap.x),
                                                  __dp4a(static_cast<int>(mv.y), static_cast<int>(ap.y), 0));
                            const int hi = __dp4a(static_cast<int>(mv.x), static_cast<int>(ap.z),
                                                  __dp4a(static_cast<int>(mv.y), static_cast<int>(ap.w), 0));
                            i2[e] = lo + 64 * hi;  // |i2| < 2^21
                        }
                        const float4 md = *reinterpret_cast<const float4 *>(sm.mins_d() + col);
                        const float2 y = make_float2(__int_as_float(static_cast<int>(kMagicBits) + i2[0]),
                                                     __int_as_float(static_cast<int>(kMagicBits) + i2[1]));
                        const float2 t = ffma2(y, make_float2(md.x, md.y), make_float2(md.z, md.w));
                        acc[mt][nt][h] = ffma2(t, make_float2(nad, nad), acc[mt][nt][h]);
                    }
                }
        }
        if constexpr (C::kTma) {
            // this warp is done with stage s
            __syncwarp();
            if (lane == 0) mbar_arrive(&tma_empty[s]);
        }
    }
    if constexpr (C::kTma) {
        // after an abort, copies issued for k-steps nobody consumed must
        // land before the CTA exits
        if (tid == 0)
            for (int j = tma_used; j < tma_issued; ++j)
                mbar_wait(&tma_full[j % ST], static_cast<uint32_t>((j / ST) & 1), p.err, kErrWaitFull);
        __syncthreads();
        if (tma_abort) return;
    } else {
        cp_async_wait<0>();
    }

    if constexpr (!kPartials) {
        if (p.splits > 1) {
            // this split's fp32 tile; reduce_splits_kernel adds the splits
            float *part = p.partial + static_cast<int64_t>(blockIdx.z) * p.m * p.n;
#pragma unroll
            for (int mt = 0; mt < MT; ++mt)
#pragma unroll
                for (int nt = 0; nt < NT; ++nt)
#pragma unroll
                    for (int h = 0; h < 2; ++h) {
                        const int64_t r = m0 + wm * C::WM + mt * 16 + g + 8 * h;
                        const int64_t c = n0 + wn * C::WN + nt * 8 + 2 * t4;
                        if (r >= p.m) continue;
                        if (c < p.n) part[r * p.n + c] = acc[mt][nt][h].x;
                        if (c + 1 < p.n) part[r * p.n + c + 1] = acc[mt][nt][h].y;
                    }
            return;
        }
        if (p.out_format == kOutQ8_0) {
            epilogue_q8_0<C>(p, smem_raw, acc, m0, n0, tid);
            return;
        }
#pragma unroll
        for (int mt = 0; mt < MT; ++mt)
#pragma unroll
            for (int nt = 0; nt < NT; ++nt)
#pragma unroll
                for (int h = 0; h < 2; ++h) {
                    const int64_t r = m0 + wm * C::WM + mt * 16 + g + 8 * h;
                    const int64_t c = n0 + wn * C::WN + nt * 8 + 2 * t4;
                    if (r < p.m) store_out2(p, r, c, acc[mt][nt][h]);
                }
        if constexpr (kCopies) copy_tile_to_copies<C>(p);
    }
}

// ---------------------------------------------------------------------------
// Overlapped variant for the types whose W decode reads nothing but W (q4_0
// in either layout, iq2_xxs): the W tile of k-step ks + 1 is decoded while
// k-step ks is multiplied.  Activation tiles and raw W tiles have separate
// two-deep cp.async rings -- during iteration ks they hold A[ks] (in use),
// A[ks + 1] (landing), raw W[ks + 1] (being decoded) and W[ks + 2]
// (landing) -- and the decoded B tile and its fold constants are
// double-buffered.  Each thread decodes its share of W[ks + 1] in pieces
// between the sub-blocks of ks, so the decode's integer work interleaves with
// every warp's MMAs and packed fmas, and one barrier per k-step publishes the
// decoded tile and retires the buffers.  Results are bit-identical to
// gemm_kernel (same integer partials, same fold order).
// ---------------------------------------------------------------------------
template <class C>
struct SmemOv {
    // one activation buffer: int8 rows, per-sub-block scales (q8_0) or sums
    // (q8_K), q8_K block scales
    static constexpr uint32_t kA = C::kAQs + C::kAScale + C::kAD8K;
    static constexpr uint32_t kTotal = 2 * kA + 2 * C::kWRaw + 2 * C::kBTile + 2 * C::kFold + C::kGrid;
    uint8_t *base;
    PFNG_DEV int8_t *a_qs(int b) const { return reinterpret_cast<int8_t *>(base + b * kA); }
    PFNG_DEV float *a_scale(int b) const { return reinterpret_cast<float *>(base + b * kA + C::kAQs); }
    PFNG_DEV float *a_d8k(int b) const { return reinterpret_cast<float *>(base + b * kA + C::kAQs + C::kAScale); }
    PFNG_DEV uint8_t *w_raw(int b) const { return base + 2 * kA + b * C::kWRaw; }
    PFNG_DEV int8_t *b_tile(int b) const {
        return reinterpret_cast<int8_t *>(base + 2 * kA + 2 * C::kWRaw + b * C::kBTile);
    }
    PFNG_DEV float2 *fold(int b) const {
        return reinterpret_cast<float2 *>(base + 2 * kA + 2 * C::kWRaw + 2 * C::kBTile + b * C::kFold);
    }
    PFNG_DEV uint2 *grid() const {
        return reinterpret_cast<uint2 *>(base + 2 * kA + 2 * C::kWRaw + 2 * C::kBTile + 2 * C::kFold);
    }
};

template <int WT, class C, bool kCopies = false, bool kPartials = false>
__global__ void __launch_bounds__(kThreads) gemm_kernel_ov(const GemmParams p) {
    static_assert(WT != kWQ4_K, "q4_K products run on the two-phase kernel");
    static_assert(C::kSlot == kWRowSlot, "decode_task reads kWRowSlot-byte rows");
    extern __shared__ __align__(128) uint8_t smem_raw[];
    const SmemOv<C> sm{smem_raw};
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int wm = warp / C::WGN, wn = warp % C::WGN;
    const int g = lane >> 2, t4 = lane & 3;
    int64_t m0, n0;
    tile_origin<C>(p, m0, n0);
    const int64_t KT = p.k / BK;
    constexpr int MT = C::MT, NT = C::NT;
    constexpr int kTasks = C::BN * 8 / kThreads;  // decode tasks per thread and k-step
    const FragOff<C> fo(wm, wn, lane);
    static_assert(kTasks >= 1 && 8 % kTasks == 0, "decode pieces");

    if constexpr (WT == kWIQ2) {
        uint2 *grid = sm.grid();
        for (int i = tid; i < 256; i += kThreads) {
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

    float2 acc[MT][NT][2];
#pragma unroll
    for (int a = 0; a < MT; ++a)
#pragma unroll
        for (int b = 0; b < NT; ++b) acc[a][b][0] = acc[a][b][1] = make_float2(0.0f, 0.0f);
    // partials mode: the plain integer products (no magic offset, no fold)
    const int cin = kPartials ? 0 : static_cast<int>(kMagicBits);

    // prologue: W[0], W[1], then (the kernel is a programmatic dependent of
    // the activation quantizer) wait for the activations and fetch A[0]
    // while W[0] is decoded
    load_w<WT, C>(p, sm.w_raw(0), 0, n0, tid);
    if (KT > 1) load_w<WT, C>(p, sm.w_raw(1), 1, n0, tid);
    cp_async_commit();
    pdl_wait();
    load_a<WT, C>(p, sm.a_qs(0), sm.a_scale(0), sm.a_d8k(0), 0, m0, tid);
    cp_async_commit();
    cp_async_wait<1>();
    __syncthreads();
#pragma unroll
    for (int t = 0; t < kTasks; ++t)
        decode_task<WT, C::BN>(p, sm.w_raw(0), sm.b_tile(0), reinterpret_cast<float *>(sm.fold(0)), sm.grid(), 0, n0,
                               tid + t * kThreads);
    cp_async_wait<0>();
    __syncthreads();

    for (int64_t ks = 0; ks < KT; ++ks) {
        const int cur = static_cast<int>(ks & 1), nxt = cur ^ 1;
        if (ks + 1 < KT) load_a<WT, C>(p, sm.a_qs(nxt), sm.a_scale(nxt), sm.a_d8k(nxt), ks + 1, m0, tid);
        if (ks + 2 < KT) load_w<WT, C>(p, sm.w_raw(cur), ks + 2, n0, tid);  // W[ks] was decoded last iteration
        cp_async_commit();
        const bool dec = ks + 1 < KT;
        const uint8_t *wr_next = sm.w_raw(nxt);
        int8_t *bt_next = sm.b_tile(nxt);
        float *fold_next = reinterpret_cast<float *>(sm.fold(nxt));

        const int8_t *at = sm.a_qs(cur);
        const int8_t *bt = sm.b_tile(cur);
        const float *ascale = sm.a_scale(cur);
        // activation block scales of this thread's rows (q8_K: one per 256 block)
        float da8k[MT][2];
        if constexpr (!kQ8_0Act<WT>) {
#pragma unroll
            for (int mt = 0; mt < MT; ++mt)
#pragma unroll
                for (int h = 0; h < 2; ++h) da8k[mt][h] = sm.a_d8k(cur)[wm * C::WM + mt * 16 + g + 8 * h];
        }
        uint32_t af[2][MT][4], bf[2][NT][2];
        int res[MT][NT][4];
        const uint32_t at_s = smem_u32(at), bt_s = smem_u32(bt);
        load_frags_o<C>(at_s, bt_s, 0, fo, af[0], bf[0]);
#pragma unroll
        for (int mt = 0; mt < MT; ++mt)
#pragma unroll
            for (int nt = 0; nt < NT; ++nt) mma_s8(res[mt][nt], af[0][mt], bf[0][nt][0], bf[0][nt][1], cin);
        load_frags_o<C>(at_s, bt_s, 1, fo, af[1], bf[1]);
#pragma unroll
        for (int kb = 0; kb < 8; ++kb) {
            const int nx = (kb + 1) & 1;
            float da[MT][2];
#pragma unroll
            for (int mt = 0; mt < MT; ++mt)
#pragma unroll
                for (int h = 0; h < 2; ++h)
                    da[mt][h] = kQ8_0Act<WT> ? ascale[(kb * 8 + g) * (C::BM / 8) + wm * (C::WM / 8) + 2 * mt + h]
                                             : da8k[mt][h];
            const float2 *fold = sm.fold(cur) + kb * C::BN;
#pragma unroll
            for (int nt = 0; nt < NT; ++nt) {
                const float4 f = *reinterpret_cast<const float4 *>(fold + wn * C::WN + nt * 8 + 2 * t4);
                const float2 sv = make_float2(f.x, f.y), cm = make_float2(f.z, f.w);
#pragma unroll
                for (int mt = 0; mt < MT; ++mt) {
                    if constexpr (kPartials) {
                        const int64_t nb32 = p.k / 32;
#pragma unroll
                        for (int i = 0; i < 4; ++i) {
                            const int64_t r = m0 + wm * C::WM + mt * 16 + g + 8 * (i >> 1);
                            const int64_t c = n0 + wn * C::WN + nt * 8 + 2 * t4 + (i & 1);
                            if (r < p.m && c < p.n) p.partials[(r * p.n + c) * nb32 + ks * 8 + kb] = res[mt][nt][i];
                        }
                    } else {
#pragma unroll
                        for (int h = 0; h < 2; ++h) {
                            const float2 y = make_float2(__int_as_float(res[mt][nt][2 * h]),
                                                         __int_as_float(res[mt][nt][2 * h + 1]));
                            const float2 t = ffma2(y, sv, cm);
                            acc[mt][nt][h] = ffma2(t, make_float2(da[mt][h], da[mt][h]), acc[mt][nt][h]);
                        }
                    }
                    if (kb + 1 < 8) mma_s8(res[mt][nt], af[nx][mt], bf[nx][nt][0], bf[nx][nt][1], cin);
                }
            }
            if (kb + 2 < 8) load_frags_o<C>(at_s, bt_s, kb + 2, fo, af[kb & 1], bf[kb & 1]);
            // a piece of the next k-step's decode after every (8 / kTasks)-th sub-block
            if ((kb + 1) % (8 / kTasks) == 0 && dec)
                decode_task<WT, C::BN>(p, wr_next, bt_next, fold_next, sm.grid(), ks + 1, n0,
                                       tid + ((kb + 1) / (8 / kTasks) - 1) * kThreads);
        }
        cp_async_wait<0>();
        __syncthreads();
    }

    if constexpr (kPartials) return;
    if (p.out_format == kOutQ8_0) {
        epilogue_q8_0<C>(p, smem_raw, acc, m0, n0, tid);
        return;
    }
#pragma unroll
    for (int mt = 0; mt < MT; ++mt)
#pragma unroll
        for (int nt = 0; nt < NT; ++nt)
#pragma unroll
            for (int h = 0; h < 2; ++h) {
                const int64_t r = m0 + wm * C::WM + mt * 16 + g + 8 * h;
                const int64_t c = n0 + wn * C::WN + nt * 8 + 2 * t4;
                if (r < p.m) store_out2(p, r, c, acc[mt][nt][h]);
            }
    if constexpr (kCopies) copy_tile_to_copies<C>(p);
}

// C tile of the CTA quantized to q8_0 along n: the tile is staged in shared
// memory (the main loop's buffers are free by then), then each warp
// quantizes four 32-column blocks at a time with the standalone quantizer's
// core, so the bytes are those of pfng_b200_quantize_q8_0 on the fp32 C.
template <class C>
PFNG_DEV void epilogue_q8_0(const GemmParams &p, uint8_t *smem, const float2 (&acc)[C::MT][C::NT][2], int64_t m0,
                            int64_t n0, int tid) {
    constexpr int CS = C::BN + 4;  // row stride of the staged tile (floats)
    static_assert(C::BM * CS * 4 <= C::kSmem, "staged C tile");
    const int warp = tid >> 5, lane = tid & 31, wm = warp / C::WGN, wn = warp % C::WGN, g = lane >> 2, t4 = lane & 3;
    float *ct = reinterpret_cast<float *>(smem);
    __syncthreads();  // every warp is past its last read of the stage buffers
#pragma unroll
    for (int mt = 0; mt < C::MT; ++mt)
#pragma unroll
        for (int nt = 0; nt < C::NT; ++nt)
#pragma unroll
            for (int h = 0; h < 2; ++h) {
                const int row = wm * C::WM + mt * 16 + g + 8 * h, col = wn * C::WN + nt * 8 + 2 * t4;
                *reinterpret_cast<float2 *>(ct + row * CS + col) = acc[mt][nt][h];
            }
    __syncthreads();
    constexpr int kBlocks = C::BM * C::BN / 32;  // a multiple of 32: every warp runs the same trip count
    const int gl = lane & 7;
    for (int b0 = warp * 4; b0 < kBlocks; b0 += (kThreads / 32) * 4) {
        const int bi = b0 + (lane >> 3);
        const int row = bi / (C::BN / 32), blk = bi % (C::BN / 32);
        const float4 t = *reinterpret_cast<const float4 *>(ct + row * CS + blk * 32 + 4 * gl);
        const float v[4] = {t.x, t.y, t.z, t.w};
        const Q8_0Lane r = q8_0_quantize_lane(v);
        const int64_t grow = m0 + row, gcol = n0 + blk * 32;
        if (grow < p.m && gcol < p.n) {
            uint8_t *b = static_cast<uint8_t *>(p.out) + (grow * p.ldo + gcol / 32) * kQ8_0Bytes;
            uint16_t *hq = reinterpret_cast<uint16_t *>(b + 2 + 4 * gl);
            hq[0] = static_cast<uint16_t>(r.q & 0xffffu);
            hq[1] = static_cast<uint16_t>(r.q >> 16);
            if (gl == 0) *reinterpret_cast<uint16_t *>(b) = r.dbits;
        }
    }
}

// Two adjacent outputs (r, c), (r, c + 1) in the requested format; c + 1 may
// be past n.
PFNG_DEV void store_out2(const GemmParams &p, int64_t r, int64_t c, float2 v) {
    if (p.out_format == kOutF32) {
        if (c < p.n) p.c[r * p.ldc + c] = v.x;
        if (c + 1 < p.n) p.c[r * p.ldc + c + 1] = v.y;
    } else if (p.out_format == kOutF16) {
        __half *o = static_cast<__half *>(p.out) + r * p.ldo + c;
        if (c < p.n) o[0] = __float2half_rn(v.x);
        if (c + 1 < p.n) o[1] = __float2half_rn(v.y);
    } else {
        __nv_bfloat16 *o = static_cast<__nv_bfloat16 *>(p.out) + r * p.ldo + c;
        if (c < p.n) o[0] = __float2bfloat16_rn(v.x);
        if (c + 1 < p.n) o[1] = __float2bfloat16_rn(v.y);
    }
}

int64_t row_bytes_of(int wtype, int64_t k) {
    switch (wtype) {
    case kWQ4_0:
    case kWQ4_0P: return k / 32 * kQ4_0Bytes;
    case 1: return k / 256 * kQ4_KBytes;
    default: return k / 256 * kIQ2Bytes;
    }
}

// Split-K reduction: C = sum of the splits' fp32 tiles in split order,
// written in the output format.  One warp per 128 columns of a row, four
// columns per lane; for q8_0 (n % 32 == 0) each 8-lane group holds one
// 32-column block and quantizes it with the standalone quantizer's core, so
// the bytes are those of pfng_b200_quantize_q8_0 on the reduced C.
__global__ void __launch_bounds__(kThreads) reduce_splits_kernel(const GemmParams p) {
    const int lane = threadIdx.x & 31;
    const int64_t wid = (static_cast<int64_t>(blockIdx.x) * kThreads + threadIdx.x) >> 5;
    const int64_t per_row = (p.n + 127) / 128;
    if (wid >= p.m * per_row) return;  // whole warps
    const int64_t r = wid / per_row;
    const int64_t c0 = (wid % per_row) * 128 + 4 * lane;
    float v[4] = {0.0f, 0.0f, 0.0f, 0.0f};
    for (int z = 0; z < p.splits; ++z) {
        const float *src = p.partial + (static_cast<int64_t>(z) * p.m + r) * p.n;
#pragma unroll
        for (int i = 0; i < 4; ++i)
            if (c0 + i < p.n) v[i] = __fadd_rn(v[i], src[c0 + i]);
    }
    if (p.out_format == kOutQ8_0) {
        const Q8_0Lane q = q8_0_quantize_lane(v);
        if (c0 < p.n) {
            uint8_t *b = static_cast<uint8_t *>(p.out) + (r * p.ldo + c0 / 32) * kQ8_0Bytes;
            const int gl = lane & 7;
            uint16_t *hq = reinterpret_cast<uint16_t *>(b + 2 + 4 * gl);
            hq[0] = static_cast<uint16_t>(q.q & 0xffffu);
            hq[1] = static_cast<uint16_t>(q.q >> 16);
            if (gl == 0) *reinterpret_cast<uint16_t *>(b) = q.dbits;
        }
        return;
    }
#pragma unroll
    for (int i = 0; i < 4; i += 2) store_out2(p, r, c0 + i, make_float2(v[i], v[i + 1]));
    if (p.ncopies > 0) {
        for (int d = 0; d < p.ncopies; ++d)
            for (int i = 0; i < 4; ++i)
                if (c0 + i < p.n) p.copies[d][r * p.ldc + c0 + i] = v[i];
        __threadfence_system();
    }
}

// Launch as a programmatic dependent of the preceding kernel on the stream
// (the activation quantizer): the kernels fetch weights before pdl_wait()
// and read activations after it.
template <class C, class K, class... Args>
cudaError_t launch_pdl(K kernel, const GemmParams &p, uint32_t smem, cudaStream_t s, const Args &...args) {
    cudaLaunchConfig_t cfg{};
    const unsigned nt = static_cast<unsigned>((p.n + C::BN - 1) / C::BN);
    const unsigned mt = static_cast<unsigned>((p.m + C::BM - 1) / C::BM);
    cfg.gridDim = p.m_fast ? dim3(mt, nt, static_cast<unsigned>(p.splits)) : dim3(nt, mt, static_cast<unsigned>(p.splits));
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kernel, args...);
}

// The tensor maps of a Cfg::kTma launch over p's operands (this GPU's
// memory): activation rows [rows_pad][k] int8 in BM x 128-byte boxes with
// the 128-byte swizzle, raw W rows [n][row_bytes] in BN x 144-byte boxes
// (rows past n read as zeros), and the q8_0 scales: with 128-row tiles
// [k / 32][d_ld] in 8 x 128 boxes, else as [block][group][g][j]
// (split_d_index) in boxes of {BM / 8 j, 8 g, 1 group, 8 blocks}
// (measured on 128-row tiles: the 2-D box 1% faster than the 4-D one).
template <class C>
bool encode_tma_maps(const GemmParams &p, TmaMaps *maps) {
    bool ok = encode_2d(&maps->a, CU_TENSOR_MAP_DATA_TYPE_UINT8, p.a.qs, static_cast<uint64_t>(p.k),
                        static_cast<uint64_t>(p.a.rows_pad), static_cast<uint64_t>(p.k), 128, C::BM,
                        CU_TENSOR_MAP_SWIZZLE_128B) &&
              encode_2d(&maps->w, CU_TENSOR_MAP_DATA_TYPE_UINT8, p.w, static_cast<uint64_t>(p.row_bytes),
                        static_cast<uint64_t>(p.n), static_cast<uint64_t>(p.row_bytes), p.step_bytes, C::BN,
                        CU_TENSOR_MAP_SWIZZLE_NONE);
    if (!ok) return false;
    if constexpr (C::BM == 128) {
        return encode_2d(&maps->ad, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, p.a.d, static_cast<uint64_t>(p.a.rows_pad),
                         static_cast<uint64_t>(p.k / 32), static_cast<uint64_t>(p.a.d_ld * 4), 128, 8,
                         CU_TENSOR_MAP_SWIZZLE_NONE);
    } else {
        const uint64_t dims[4] = {16, 8, static_cast<uint64_t>(p.a.rows_pad / 128), static_cast<uint64_t>(p.k / 32)};
        const uint64_t strides[3] = {64, 512, static_cast<uint64_t>(p.a.d_ld * 4)};
        const uint32_t box[4] = {C::BM / 8, 8, 1, 8};
        return encode_nd(&maps->ad, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, p.a.d, dims, strides, box);
    }
}

template <int WT, class C, bool kPartials, bool kCopies = false, bool kDirect = false>
cudaError_t launch_t(const GemmParams &p, cudaStream_t s) {
    auto kernel = gemm_kernel<WT, C, kPartials, kCopies, kDirect>;
    // direct q4_0 operands use the stage ring only (no B tile, fold data or
    // tables); q4_K keeps the layout for its fold data and mins
    // tensor-map stages: + the slack that aligns them to 1024 bytes
    constexpr uint32_t smem = kDirect && WT != kWQ4_K ? C::ST * C::kStage + (C::kTma ? 1024u : 0u) : C::kSmem;
    static_assert(smem <= kMaxSmemPerCta, "dynamic shared memory above the per-CTA limit");
    TmaMaps maps;
    if constexpr (C::kTma) {
        if (!encode_tma_maps<C>(p, &maps)) return cudaErrorNotSupported;  // the caller takes the cp.async kernel
    } else {
        std::memset(&maps, 0, sizeof maps);
    }
    // the q8_0 epilogue stages the CTA's C tile in the launched shared memory
    static_assert(C::BM * (C::BN + 4) * 4 <= smem, "staged C tile of the q8_0 epilogue");
    static thread_local bool configured[64] = {false};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 0 || dev >= 64 || !configured[dev]) {
        cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
        if (e != cudaSuccess) return e;
        if (dev >= 0 && dev < 64) configured[dev] = true;
    }
    return launch_pdl<C>(kernel, p, smem, s, maps, p);
}

template <int WT, class C, bool kCopies = false, bool kPartials = false>
cudaError_t launch_t_ov(const GemmParams &p, cudaStream_t s) {
    auto kernel = gemm_kernel_ov<WT, C, kCopies, kPartials>;
    constexpr uint32_t smem = SmemOv<C>::kTotal;
    static_assert(smem <= kMaxSmemPerCta, "dynamic shared memory above the per-CTA limit");
    static_assert(C::BM * (C::BN + 4) * 4 <= smem, "staged C tile of the q8_0 epilogue");
    static thread_local bool configured[64] = {false};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 0 || dev >= 64 || !configured[dev]) {
        cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
        if (e != cudaSuccess) return e;
        if (dev >= 0 && dev < 64) configured[dev] = true;
    }
    return launch_pdl<C>(kernel, p, smem, s, p);
}

// The overlapped kernel serves q4_0 (both layouts) and iq2_xxs products
// without split-K;
// PFNG_B200_GEMM_OV=0 selects the two-phase kernel instead (comparisons).
// Measured on B200 (us per quantize + GEMM step, overlapped vs two-phase):
// 2048x11008x4096 627 vs 698, 512x4096x4096 66 vs 73, 480x1536x1536 on 64 x 64
// tiles 20.2 vs 21.3 (q4_0) and 24.6 vs 25.3 (iq2_xxs).  q4_K, whose min term
// the overlapped kernel adds once per 256-block from the resident A tile, was
// slower there: 2048x4096x4096 353 vs 338, 512x4096x4096 90.0 vs 85.9.
template <int WT>
constexpr bool kOvType = WT != kWQ4_K;
// Direct operands for every q4_0 tile (both layouts, 16-byte aligned rows);
// PFNG_B200_GEMM_DIRECT=0 selects the decode pass instead (comparisons).
// Measured on B200 (us per quantize + GEMM step, direct vs decode pass):
// 32x4096x4096 14.4 vs 15.7, 32x11008x4096 26.0 vs 29.2, 32x4096x11008 28.4
// vs 31.5, 32x32000x4096 54.4 vs 63.1; on 64-row tiles (vs the overlapped or
// split two-phase kernel) 480x1536x1536 18.5 vs 20.1, 256x4096x4096 41.8 vs
// 45.5, 128x4096x4096 25.1 vs 28.8, 64x11008x4096 40.9 vs 44.7.  A deeper
// ring, which the smaller shared-memory footprint would allow, was slower
// (32x32000x4096: 3 stages 56.6, 4 stages 66.3 us), and so were three
// 32-row CTAs per SM at 80 registers (78.7 us).  64-row direct kernels, and
// 32-row q4_K ones (151 registers unbounded), are bounded to two CTAs per SM
// (<= 128 registers, no spills; q4_K 32x11008x4096 35.8 -> 31.3 us).  On 128 x 128
// tiles the direct two-phase kernel also beats the overlapped decode:
// 2048x11008x4096 589.6 vs 622.7, 2048x4096x4096 242.4 vs 255.4,
// 512x4096x4096 62.4 vs 65.5, 2048x4096x11008 629.8 vs 661.5.  Two variants
// of the 128 x 128 direct kernel gave the same bits and were slower
// (2048x32000x4096 / 2048x11008x4096 / 512x4096x4096, us): 16 warps of
// 64 x 16 (128 registers) 1705 / 621 / 64.8, and float4 fold constants that
// each warp converts once per k-step into shared memory 1651 / 601 / 63.3,
// against 1639 / 597 / 62.8 for 8 warps of 64 x 32 converting the fp16
// scales in the sub-block loop.
inline bool direct_enabled() {
    const char *e = std::getenv("PFNG_B200_GEMM_DIRECT");
    return !(e && std::strcmp(e, "0") == 0);
}
inline bool ov_enabled() {
    const char *e = std::getenv("PFNG_B200_GEMM_OV");
    return !(e && std::strcmp(e, "0") == 0);
}
inline bool tma_enabled() {
    const char *e = std::getenv("PFNG_B200_GEMM_TMA");
    return !(e && std::strcmp(e, "0") == 0);
}

// The partials mode (integer sub-block products instead of C) takes the
// same kernel as the product of the same shape, so the integers it exports
// are those the product folds.
template <int WT, class C, bool kPartials>
cudaError_t launch_pick(const GemmParams &p, cudaStream_t s) {
    // 32-row tiles keep the two-phase kernel: its two-deep ring fits two CTAs
    // per SM, the overlapped kernel's buffers one (32x32000x4096: 63 vs 74 us)
    // copies (fp32 C to more destinations): the kernels built with the copy
    // pass; with split-K the reduction stores the copies
    const bool copies = !kPartials && p.ncopies > 0 && p.splits == 1;
    if constexpr (WT == kWQ4_0 || WT == kWQ4_0P || WT == kWQ4_K) {
        // 176-byte row slots (44 words): the eight rows of a fragment read
        // start on banks 12 r mod 32, so with the four t4 words they hit
        // all 32 banks (160-byte slots: rows r and r + 4 collide).  q4_K
        // keeps 160-byte slots: its full layout (fold data, mins) with
        // 176-byte rows would pass the per-CTA limit on 128 x 128 tiles.
        //
        // 128 x 128 q4_0 tiles give each warp all 128 rows and 16 columns
        // (128 x 16 warp tiles, 8 m16 fragments per column group): every
        // column's unpack and scale conversion serves twice the MMAs of a
        // 64 x 32 warp tile (254 registers, no spills; 2048x32000x4096
        // 1621 -> 1585 us, 2048x11008x4096 591 -> 579 us, same bits).
        using D = Cfg<C::BM, C::BN, C::ST, WT == kWQ4_K ? kWRowSlot : 176u,
                      (C::BM == 128 && C::BN == 128 && WT == kWQ4_0) ? 1 : 2>;
        if constexpr (WT == kWQ4_0 && !(C::BM == 64 && C::BN == 128)) {
            // the same kernel with its stages loaded by tensor maps from one
            // thread (PFNG_B200_GEMM_TMA=0: the per-thread cp.async loads).
            // The 54 KB stages of 128 x 128 tiles fit a 4-deep ring
            // (2048x32000x4096: 1332 -> 1305 us against 3 stages); the
            // smaller tiles keep 3 stages and two CTAs per SM (480x1536x1536
            // 18.7 -> 17.5 us, 32x32000x4096 52.9 -> 47.3 us against
            // cp.async).  64 x 128 tiles (32 < m <= 128 with large n, no
            // BASELINE shape) keep the cp.async loads.
            if (p.w_vec16 && direct_enabled() && tma_enabled()) {
                using DT = Cfg<C::BM, C::BN, (C::BM == 128 && C::BN == 128) ? 4 : 3, 144u, D::WGM, true>;
                cudaError_t e;
                if constexpr (kPartials)
                    e = launch_t<WT, DT, true, false, true>(p, s);
                else
                    e = copies ? launch_t<WT, DT, false, true, true>(p, s) : launch_t<WT, DT, false, false, true>(p, s);
                if (e != cudaErrorNotSupported) return e;
            }
        }
        if ((WT == kWQ4_0P || p.w_vec16) && direct_enabled()) {
            if constexpr (kPartials) return launch_t<WT, D, true, false, true>(p, s);
            return copies ? launch_t<WT, D, false, true, true>(p, s) : launch_t<WT, D, false, false, true>(p, s);
        }
    }
    if constexpr (kOvType<WT> && C::BM > 32) {
        if (p.splits == 1 && ov_enabled()) {
            if constexpr (kPartials) return launch_t_ov<WT, C, false, true>(p, s);
            return copies ? launch_t_ov<WT, C, true>(p, s) : launch_t_ov<WT, C>(p, s);
        }
    }
    if constexpr (!kPartials) {
        if (copies) return launch_t<WT, C, false, true>(p, s);
    }
    return launch_t<WT, C, kPartials>(p, s);
}

// Tile shapes: 128 x 128 and 64 x 128 (one CTA per SM), 64 x 64 and, for
// m <= 32, 32 x 128 with a two-deep ring (two CTAs per SM).
enum TileKind { kT128x128, kT64x128, kT64x64, kT32x128 };
constexpr uint32_t kSmemPerSm2 = 113 * 1024;  // a CTA at most this size fits twice per SM

uint32_t tile_smem(TileKind t) {
    switch (t) {
    case kT128x128: return Cfg<128, 128>::kSmem;
    case kT64x128: return Cfg<64, 128>::kSmem;
    case kT64x64: return Cfg<64, 64>::kSmem;
    default: return Cfg<32, 128, 2>::kSmem;
    }
}
int tile_bm(TileKind t) { return t == kT128x128 ? 128 : t == kT32x128 ? 32 : 64; }
int tile_bn(TileKind t) { return t == kT64x64 ? 64 : 128; }

// measured on B200: 128x128 wins once it fills ~80% of the SMs (512x4096x4096:
// 66 us vs 95 us with 64x64); below that 64x64, whose CTAs fit two per SM,
// as long as they fit in one wave (480x1536x1536: 192 CTAs, 20.2 us vs 20.8
// with 64x128 and 30 with 128x128); m <= 32 takes 32-row tiles.
// PFNG_B200_GEMM_TILE = "128x128" / "64x128" / "64x64" / "32x128" forces one.
TileKind tile_choice(int64_t m, int64_t n, int64_t sms) {
    if (const char *t = std::getenv("PFNG_B200_GEMM_TILE")) {
        if (std::strcmp(t, "128x128") == 0) return kT128x128;
        if (std::strcmp(t, "64x128") == 0) return kT64x128;
        if (std::strcmp(t, "64x64") == 0) return kT64x64;
        if (std::strcmp(t, "32x128") == 0) return kT32x128;
    }
    auto ctas = [&](int bm, int bn) { return ((n + bn - 1) / bn) * ((m + bm - 1) / bm); };
    if (m <= 32) return kT32x128;
    if (ctas(128, 128) * 5 >= 4 * sms) return kT128x128;
    if (ctas(64, 64) <= 2 * sms) return kT64x64;
    return kT64x128;
}

// Split-K factor: when the tiles fill at most half of the resident CTA slots
// and k has at least 4 k-steps, each tile's k range is split so the splits
// fill the slots (at most 8, at least two k-steps each; PFNG_B200_GEMM_SPLITS
// lowers the cap, 1 disables splitting).  A split product adds the splits'
// fp32 tiles in split order: deterministic, but a different summation order
// than the unsplit kernel.
int splits_for(TileKind t, int64_t m, int64_t n, int64_t k, int64_t sms) {
    int64_t cap = 8;
    if (const char *e = std::getenv("PFNG_B200_GEMM_SPLITS")) cap = std::atoi(e) > 0 ? std::atoi(e) : 1;
    const int64_t tiles = ((n + tile_bn(t) - 1) / tile_bn(t)) * ((m + tile_bm(t) - 1) / tile_bm(t));
    const int64_t slots = sms * (tile_smem(t) <= kSmemPerSm2 ? 2 : 1);
    const int64_t kt = k / BK;
    if (tiles * 2 > slots || kt < 4 || cap < 2) return 1;
    int64_t sp = slots / tiles;
    if (sp > kt / 2) sp = kt / 2;
    if (sp > cap) sp = cap;
    // splits that are all non-empty
    const int64_t per = (kt + sp - 1) / sp;
    return static_cast<int>((kt + per - 1) / per);
}

// C [m][n] (row stride ldc) to every copy after the GEMM: one grid over all
// SMs, 16-byte pieces along rows where c_vec4 allows, then a system-scope
// fence (the stores are performed before the kernel ends).
__global__ void __launch_bounds__(kThreads) push_copies_kernel(const GemmParams p) {
    const int64_t stride = static_cast<int64_t>(gridDim.x) * kThreads;
    const int64_t tid = static_cast<int64_t>(blockIdx.x) * kThreads + threadIdx.x;
    if (p.c_vec4) {
        const int64_t quads = p.n / 4, total = p.m * quads;
        for (int64_t i = tid; i < total; i += stride) {
            const int64_t o = (i / quads) * p.ldc + (i % quads) * 4;
            const float4 v = *reinterpret_cast<const float4 *>(p.c + o);
            for (int d = 0; d < p.ncopies; ++d) *reinterpret_cast<float4 *>(p.copies[d] + o) = v;
        }
        for (int64_t i = tid; i < p.m * (p.n % 4); i += stride) {  // ragged columns
            const int64_t o = (i / (p.n % 4)) * p.ldc + quads * 4 + i % (p.n % 4);
            for (int d = 0; d < p.ncopies; ++d) p.copies[d][o] = p.c[o];
        }
    } else {
        for (int64_t i = tid; i < p.m * p.n; i += stride) {
            const int64_t o = (i / p.n) * p.ldc + i % p.n;
            for (int d = 0; d < p.ncopies; ++d) p.copies[d][o] = p.c[o];
        }
    }
    __threadfence_system();
}

// How the copies are written: by push_copies_kernel after the GEMM (default)
// or in the GEMM's epilogue (PFNG_B200_COPIES=epilogue).  Measured on two
// B200s (us per step of the row-sharded configs[4] shapes at m = 2048,
// push vs epilogue): 271 vs 278, 496 vs 515, 587 vs 598, 1172 vs 1224.  The
// 128 x 128 GEMM runs one CTA per SM, so nothing hides the epilogue's copy
// of its tile, while the push kernel streams C at copy bandwidth.
inline bool push_copies() {
    const char *e = std::getenv("PFNG_B200_COPIES");
    return !(e && std::strcmp(e, "epilogue") == 0);
}

// Raster order of the tiles.  With the n tiles fastest, each W tile is
// revisited by the next m tile only after all n tiles, by when the C stream
// has evicted it from L2: measured on 2048 x 32000 x 4096 (q4_0), 419 MB of
// DRAM reads per launch for 84 MB of W and activations.  With the m tiles
// fastest the CTAs running together share their W tiles, and the
// activations (the smaller operand) stay in L2, so the m tiles go fastest
// whenever there are several and the activation operand is at most 48 MB.
// PFNG_B200_GEMM_RASTER = "m" / "n" forces either (comparisons).
bool m_fast_raster(const GemmParams &p, int bm, int bn) {
    if (p.m > 65535LL * bm || p.n > 65535LL * bn) return p.n > 65535LL * bn;  // grid.y limit
    if (const char *e = std::getenv("PFNG_B200_GEMM_RASTER")) return std::strcmp(e, "m") == 0;
    const int64_t a_bytes = p.m * p.k + p.m * (p.k / 32) * 8;
    return p.m > bm && a_bytes <= (48LL << 20);
}

// Row bands of a product whose C also goes to other destinations (the
// all-gather of row-sharded weights): each band's rows are copied to the
// destinations while the next band is computed, so that most of the
// transfer over NVLink overlaps the GEMM instead of following it.  Every tile
// is computed exactly as without bands (bit-identical C).  Two bands, the
// last one the smallest under which the first band's copies still finish:
// with r = copy time / GEMM time per row ~ 1400 x destinations / k
// (measured on B200: ~416 Top/s for the GEMM, ~600 GB/s out over NVLink)
// it takes r / (1 + r) of the 128-row tiles.  Measured at 2048 x 32000 x
// 4096 (us per sharded step): two B200s, no bands 1101, two equal bands
// 1005, four 1077, eight 1061 (copy engines), four with the push kernel
// 1084; four B200s (where the copies take as long as the GEMM), two bands
// 666, four or eight equal bands 685.
// Products of fewer than four 128-row tiles run unbanded;
// PFNG_B200_GATHER_BANDS=1 turns the bands off, =2..8 forces that many
// equal bands (comparisons).  Returns the band count (0: unbanded) and the
// first row of each band in `start` (start[bands] = m).
constexpr int kMaxBands = 8;
int gather_bands(const GemmParams &p, int64_t tiles, int64_t (&start)[kMaxBands + 1]) {
    int forced = 0;
    if (const char *e = std::getenv("PFNG_B200_GATHER_BANDS")) {
        forced = std::atoi(e);
        if (forced == 1) return 0;
        if (forced < 2 || forced > kMaxBands) forced = 0;
    }
    if (tiles < 4) return 0;
    const double r = 1400.0 * p.ncopies / static_cast<double>(p.k);
    int bands = forced ? forced : 2;
    if (bands > tiles) bands = static_cast<int>(tiles);
    if (!forced && bands == 2) {
        int64_t last = static_cast<int64_t>(tiles * r / (1.0 + r) + 0.999);
        if (last < 1) last = 1;
        if (last > tiles - 1) last = tiles - 1;
        start[0] = 0;
        start[1] = (tiles - last) * kGemmTileM;
    } else {
        for (int b = 0; b < bands; ++b) start[b] = (tiles * b / bands) * kGemmTileM;
    }
    start[bands] = p.m;
    return bands;
}

// Side streams (one per destination, high priority) and their events, one
// set per device, created on first use.
struct SideStreams {
    cudaStream_t stream[kMaxCopies] = {};
    cudaEvent_t band = nullptr;
    cudaEvent_t join[kMaxCopies] = {};
    bool ready = false;
};
SideStreams g_side[64];
std::mutex g_side_mutex;  // also serialises the banded launch sequences of concurrent host threads

cudaError_t side_streams(SideStreams **out) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
    SideStreams &ss = g_side[dev];
    if (!ss.ready) {
        int least = 0, greatest = 0;
        if ((e = cudaDeviceGetStreamPriorityRange(&least, &greatest)) != cudaSuccess) return e;
        for (int i = 0; i < kMaxCopies; ++i) {
            if ((e = cudaStreamCreateWithPriority(&ss.stream[i], cudaStreamNonBlocking, greatest)) != cudaSuccess)
                return e;
            if ((e = cudaEventCreateWithFlags(&ss.join[i], cudaEventDisableTiming)) != cudaSuccess) return e;
        }
        if ((e = cudaEventCreateWithFlags(&ss.band, cudaEventDisableTiming)) != cudaSuccess) return e;
        ss.ready = true;
    }
    *out = &ss;
    return cudaSuccess;
}

template <int WT, bool kPartials>
cudaError_t launch_tile(GemmParams &p, cudaStream_t s);

// Rows [r0, r1) of the product (the activation operand and every output
// offset to them).
GemmParams row_band(const GemmParams &p, int64_t r0, int64_t r1, int64_t blk) {
    GemmParams q = p;
    q.m = r1 - r0;
    q.c = p.c + r0 * p.ldc;
    q.a.qs = p.a.qs + r0 * p.k;
    // q8_0 scales: r0 is a multiple of 128, so the rows keep their places
    // inside their 128-row groups and the block slabs keep their stride
    q.a.d = blk == 32 ? p.a.d + r0 : p.a.d + r0 * (p.k / blk);
    q.a.aux = p.a.aux + r0 * (p.k / 32);
    q.a.rows_pad = p.a.rows_pad - r0;
    for (int d = 0; d < p.ncopies; ++d) q.copies[d] = p.copies[d] + r0 * p.ldc;
    return q;
}

// Copies of rows [0, q.m) of q.c to q's destinations, each destination on
// its own side stream (the copy engines work on them in parallel).
cudaError_t copy_band(const GemmParams &q, SideStreams *side) {
    const size_t pitch = static_cast<size_t>(q.ldc) * sizeof(float);
    for (int d = 0; d < q.ncopies; ++d) {
        cudaError_t e = cudaStreamWaitEvent(side->stream[d], side->band, 0);
        if (e == cudaSuccess)
            e = cudaMemcpy2DAsync(q.copies[d], pitch, q.c, pitch, static_cast<size_t>(q.n) * sizeof(float),
                                  static_cast<size_t>(q.m), cudaMemcpyDeviceToDevice, side->stream[d]);
        if (e != cudaSuccess) return e;
    }
    return cudaSuccess;
}

template <int WT>
cudaError_t launch_banded_gather(const GemmParams &p, cudaStream_t s, const int64_t *bounds, int bands) {
    std::lock_guard<std::mutex> lock(g_side_mutex);
    SideStreams *side = nullptr;
    cudaError_t e = side_streams(&side);
    if (e != cudaSuccess) return e;
    const int64_t blk = kQ8_0Act<WT> ? 32 : 256;
    for (int b = 0; b < bands; ++b) {
        const GemmParams q = row_band(p, bounds[b], bounds[b + 1], blk);
        GemmParams g = q;
        g.ncopies = 0;
        if ((e = launch_tile<WT, false>(g, s)) != cudaSuccess) return e;
        if ((e = cudaEventRecord(side->band, s)) != cudaSuccess) return e;
        if ((e = copy_band(q, side)) != cudaSuccess) return e;
    }
    // the caller's stream continues once every copy has landed
    for (int d = 0; d < p.ncopies; ++d) {
        if ((e = cudaEventRecord(side->join[d], side->stream[d])) != cudaSuccess) return e;
        if ((e = cudaStreamWaitEvent(s, side->join[d], 0)) != cudaSuccess) return e;
    }
    return cudaSuccess;
}

template <int WT, bool kPartials>
cudaError_t launch_tile(GemmParams &p, cudaStream_t s) {
    if (p.ncopies > 0 && p.out_format == kOutF32 && push_copies()) {
        if constexpr (!kPartials) {
            const int64_t tiles = (p.m + kGemmTileM - 1) / kGemmTileM;
            int64_t start[kMaxBands + 1];
            const int bands = gather_bands(p, tiles, start);
            if (bands > 0) return launch_banded_gather<WT>(p, s, start, bands);
        }
        GemmParams q = p;
        q.ncopies = 0;
        cudaError_t e = launch_tile<WT, kPartials>(q, s);
        if (e != cudaSuccess) return e;
        const int64_t sms = device_sm_count();
        push_copies_kernel<<<static_cast<unsigned>(sms * 4), kThreads, 0, s>>>(p);
        return cudaGetLastError();
    }
    const int64_t sms = device_sm_count();
    const TileKind t = tile_choice(p.m, p.n, sms);
    const int64_t kt = p.k / BK;
    // the partials mode splits like the product (each CTA exports the
    // partials of its k range; nothing to reduce)
    p.splits = 1;
    const int sp = splits_for(t, p.m, p.n, p.k, sms);
    if (sp > 1 && p.partial) p.splits = sp;
    p.ks_per_split = static_cast<int>((kt + p.splits - 1) / p.splits);
    p.m_fast = m_fast_raster(p, tile_bm(t), tile_bn(t)) ? 1 : 0;
    cudaError_t e;
    switch (t) {
    case kT128x128: e = launch_pick<WT, Cfg<128, 128>, kPartials>(p, s); break;
    case kT64x128: e = launch_pick<WT, Cfg<64, 128>, kPartials>(p, s); break;
    case kT64x64: e = launch_pick<WT, Cfg<64, 64>, kPartials>(p, s); break;
    default: e = launch_pick<WT, Cfg<32, 128, 2>, kPartials>(p, s); break;
    }
    if (e != cudaSuccess || p.splits == 1 || kPartials) return e;
    const int64_t warps = p.m * ((p.n + 127) / 128);
    const int64_t blocks = (warps * 32 + kThreads - 1) / kThreads;
    if (blocks > 0x7fffffff) return cudaErrorInvalidValue;
    reduce_splits_kernel<<<static_cast<unsigned>(blocks), kThreads, 0, s>>>(p);
    return cudaGetLastError();
}

}  // namespace

size_t gemm_partial_bytes(int64_t m, int64_t n, int64_t k) {
    const int64_t sms = device_sm_count();
    const int sp = splits_for(tile_choice(m, n, sms), m, n, k, sms);
    return sp > 1 ? static_cast<size_t>(sp) * static_cast<size_t>(m) * static_cast<size_t>(n) * sizeof(float) : 0;
}

bool gemm_supported(int wtype, int64_t m, int64_t n, int64_t k, const void *w) {
    (void)wtype;
    (void)m;
    (void)n;
    if (k % BK != 0) return false;
    if ((reinterpret_cast<uintptr_t>(w) & 15u) != 0) return false;
    return Cfg<128, 128>::kSmem <= device_smem_optin();
}

// The q4_0 product runs on the tcgen05 kernel (gemm_tc.cu) unless the
// environment variable PFNG_B200_GEMM is "mma" (or the shape is unsupported);
// "tc" / "mma" select either kernel explicitly, for comparisons.
static bool use_tc(const GemmArgs &args) {
    if (args.wtype != kWQ4_0 || args.partials || args.out_format != kOutF32 || args.ncopies > 0) return false;
    const char *e = std::getenv("PFNG_B200_GEMM");
    const bool want = e ? std::strcmp(e, "tc") == 0 : kTcDefault;
    return want && gemm_tc_supported(args.wtype, args.m, args.n, args.k, args.w);
}

cudaError_t launch_gemm(const GemmArgs &args, cudaStream_t s) {
    if (use_tc(args)) return launch_gemm_tc(args, args.err, s);
    GemmParams p{};
    p.w = static_cast<const uint8_t *>(args.w);
    p.a = args.a;
    p.c = args.c;
    p.ldc = args.ldc;
    p.partials = args.partials;
    p.err = args.err;
    p.m = args.m;
    p.n = args.n;
    p.k = args.k;
    p.row_bytes = row_bytes_of(args.wtype, args.k);
    p.step_bytes = static_cast<uint32_t>(row_bytes_of(args.wtype, BK));
    p.w_total = p.row_bytes * args.n;
    p.w_vec16 = (p.row_bytes % 16 == 0 && p.step_bytes % 16 == 0) ? 1 : 0;
    p.out_format = args.out_format;
    p.out = args.out;
    p.ldo = args.ldo;
    p.ncopies = args.copies ? args.ncopies : 0;
    bool vec4 = reinterpret_cast<uintptr_t>(args.c) % 16 == 0 && args.ldc % 4 == 0;
    for (int d = 0; d < p.ncopies; ++d) {
        p.copies[d] = args.copies[d];
        vec4 = vec4 && reinterpret_cast<uintptr_t>(args.copies[d]) % 16 == 0;
    }
    p.c_vec4 = vec4 ? 1 : 0;
    // split-K partials, when the caller's workspace holds them
    const size_t need = gemm_partial_bytes(args.m, args.n, args.k);
    p.partial = (need > 0 && args.partial && args.partial_bytes >= need) ? args.partial : nullptr;
    const bool part = args.partials != nullptr;
    switch (args.wtype) {
    case kWQ4_0: return part ? launch_tile<kWQ4_0, true>(p, s) : launch_tile<kWQ4_0, false>(p, s);
    case kWQ4_K: return part ? launch_tile<kWQ4_K, true>(p, s) : launch_tile<kWQ4_K, false>(p, s);
    case kWQ4_0P: return part ? launch_tile<kWQ4_0P, true>(p, s) : launch_tile<kWQ4_0P, false>(p, s);
    default: return part ? launch_tile<kWIQ2, true>(p, s) : launch_tile<kWIQ2, false>(p, s);
    }
}

}  // namespace pfng
