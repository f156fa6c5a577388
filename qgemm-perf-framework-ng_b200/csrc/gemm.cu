// gemm.cu -- batched-m block-quantized matmul on the int8 tensor cores.
//
// C[m][n] = A[m][k] . W[n][k]^T with W in the raw ggml layout and A in the
// split layout (int8 rows + per-block scales) produced by quantize.cu.
// Semantics: compute_q4_0 / compute_q4_K / compute_iq2_xxs,
// bench/llama_reference/llama_reference.cpp:113-205.
//
// CTA tile 128 (m) x 128 (n), k-step 256, 8 warps of 64 x 32, a 3-stage
// cp.async ring for the A rows, A scales and raw W bytes.  Each k-step the
// CTA unpacks its raw W tile once into an int8 [n][k] tile (q4_0: nibble - 8;
// q4_K: nibble; iq2_xxs: signed grid value) plus per-column scale data, then
// every 32-deep sub-block is one m16n8k32 s8 MMA per 16 x 8 fragment:
//   q4_0:    the accumulator input is the constant 0x4B400000, so the int32
//            result P is returned as the float 2^23 + 2^22 + P exactly; then
//            t = fma(y, dw, -(2^23 + 2^22) * dw) = round(P * dw) (the second
//            product is exact: dw has 11 significant bits) and
//            acc = fma(t, da, acc): two FMAs per element and sub-block.
//   q4_K:    I1 += scale * P per sub-block (integer), and once per 256 block
//            acc += a.d * (d * I1 - dmin * I2), with I2 = sum_sb min * bsum
//            computed by dp4a from packed bytes.
//   iq2_xxs: I += scale * P per sub-block, acc += 0.125 * d * a.d * I per block.
// Integer partials are exact (int32 tensor-core accumulation), the fp32 fold
// follows the reference's block order (k ascending), so results differ from
// the reference only by the fused roundings of the fold.
#include "iq2xxs_grid_codes.h"
#include "pfng_common.cuh"
#include "pfng_internal.h"

namespace pfng {
namespace {

constexpr int BM = 128, BN = 128, BK = 256;
constexpr int kThreads = 256;
constexpr int kStages = 3;
constexpr uint32_t kMagicBits = 0x4B400000u;  // float 12582912 = 2^23 + 2^22
constexpr float kMagic = 12582912.0f;

// per-stage shared memory
constexpr uint32_t kAQsBytes = BM * BK;                 // 32768
constexpr uint32_t kAScaleBytes = BM * 8 * 4;           // q4_0: d per (row, sub-block); q8_K: bsum32 per (row, sb)
constexpr uint32_t kAD8KBytes = BM * 4;                 // q8_K: d per row (one block per k-step)
constexpr uint32_t kWRowSlot = 160;                     // >= 144 + 8 window slack, multiple of 16
constexpr uint32_t kWRawBytes = BN * kWRowSlot;         // 20480
constexpr uint32_t kStageBytes = kAQsBytes + kAScaleBytes + kAD8KBytes + kWRawBytes;
// single (non-staged) buffers
constexpr uint32_t kBTileBytes = BN * BK;               // 32768
constexpr uint32_t kWFoldBytes = 8 * BN * 8;            // 8192
constexpr uint32_t kAPackBytes = BM * 16;               // q4_K: packed bsum bytes per row
constexpr uint32_t kSmemBytes = kStages * kStageBytes + kBTileBytes + kWFoldBytes + kAPackBytes;

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
};

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

PFNG_DEV void mma_s8(int (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1, const int (&c)[4]) {
    asm volatile(
        "mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%10,%11,%12,%13};"
        : "=r"(d[0]), "=r"(d[1]), "=r"(d[2]), "=r"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1), "r"(c[0]), "r"(c[1]), "r"(c[2]),
          "r"(c[3]));
}

// byte offset of 16-byte chunk `chunk` of row `row` in a [rows][256 B] tile,
// XOR-swizzled so that ldmatrix over 8 rows touches 8 distinct bank groups.
PFNG_DEV uint32_t swz(int row, int chunk) { return static_cast<uint32_t>(row * 256 + ((chunk ^ (row & 7)) << 4)); }

struct Smem {
    uint8_t *base;
    PFNG_DEV uint8_t *stage(int s) const { return base + s * kStageBytes; }
    PFNG_DEV int8_t *a_qs(int s) const { return reinterpret_cast<int8_t *>(stage(s)); }
    PFNG_DEV int32_t *a_scale(int s) const { return reinterpret_cast<int32_t *>(stage(s) + kAQsBytes); }
    PFNG_DEV float *a_d8k(int s) const { return reinterpret_cast<float *>(stage(s) + kAQsBytes + kAScaleBytes); }
    PFNG_DEV uint8_t *w_raw(int s) const { return stage(s) + kAQsBytes + kAScaleBytes + kAD8KBytes; }
    PFNG_DEV int8_t *b_tile() const { return reinterpret_cast<int8_t *>(base + kStages * kStageBytes); }
    PFNG_DEV uint8_t *w_fold() const { return base + kStages * kStageBytes + kBTileBytes; }
    PFNG_DEV uint4 *a_pack() const { return reinterpret_cast<uint4 *>(w_fold() + kWFoldBytes); }
};

// Issue the cp.async copies of k-step `ks` into stage `s`.
template <int WT>
PFNG_DEV void load_stage(const GemmParams &p, const Smem &sm, int s, int64_t ks, int64_t m0, int64_t n0, int tid) {
    const int64_t K = p.k;
    // A int8 rows: 128 x 256 B = 2048 chunks
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        const int q = tid + i * kThreads;
        const int row = q >> 4, ch = q & 15;
        const int8_t *src = p.a.qs + (m0 + row) * K + ks * BK + ch * 16;
        cp_async16(sm.a_qs(s) + swz(row, ch), src, 16);
    }
    if constexpr (WT == 0) {
        // d per (row, sub-block): 8 floats per row = 2 chunks per row
        const int row = tid >> 1, half = tid & 1;
        const float *src = p.a.d + (m0 + row) * (K / 32) + ks * 8 + half * 4;
        cp_async16(reinterpret_cast<uint8_t *>(sm.a_scale(s)) + row * 32 + half * 16, src, 16);
    } else {
        // bsum32 per (row, sub-block) and d per row
        const int row = tid >> 1, half = tid & 1;
        const int32_t *src = p.a.aux + (m0 + row) * (K / 32) + ks * 8 + half * 4;
        cp_async16(reinterpret_cast<uint8_t *>(sm.a_scale(s)) + row * 32 + half * 16, src, 16);
        if (tid < BM) cp_async4(sm.a_d8k(s) + tid, p.a.d + (m0 + tid) * (K / 256) + ks, 4);
    }
    // raw W: 128 rows x step_bytes, each row into a kWRowSlot-byte slot
    uint8_t *wr = sm.w_raw(s);
    if (p.w_vec16) {
        const int chunks = static_cast<int>(p.step_bytes / 16);
        for (int q = tid; q < BN * chunks; q += kThreads) {
            const int row = q / chunks, ch = q % chunks;
            const int64_t n = n0 + row;
            const bool ok = n < p.n;
            const uint8_t *src = p.w + (ok ? n * p.row_bytes + ks * p.step_bytes + ch * 16 : 0);
            cp_async16(wr + row * kWRowSlot + ch * 16, src, ok ? 16u : 0u);
        }
    } else {
        // word-granular window [start & ~3, start + step_bytes + 3) per row
        const int words = static_cast<int>((p.step_bytes + 3) / 4) + 1;
        for (int q = tid; q < BN * words; q += kThreads) {
            const int row = q / words, wd = q % words;
            const int64_t n = n0 + row;
            const int64_t start = n * p.row_bytes + ks * p.step_bytes;
            const int64_t addr = (start & ~int64_t(3)) + 4 * wd;
            uint32_t bytes = 0;
            if (n < p.n && addr < p.w_total) bytes = p.w_total - addr >= 4 ? 4u : static_cast<uint32_t>(p.w_total - addr);
            cp_async4(wr + row * kWRowSlot + 4 * wd, p.w + (bytes ? addr : 0), bytes);
        }
    }
}

// Unpack the raw W tile of stage `s` into the int8 B tile and the
// per-column fold data.  Runs once per CTA per k-step.
template <int WT>
PFNG_DEV void decode_w(const GemmParams &p, const Smem &sm, int s, int64_t ks, int64_t n0, int tid) {
    const uint8_t *wr = sm.w_raw(s);
    int8_t *bt = sm.b_tile();
    uint8_t *wf = sm.w_fold();
    if constexpr (WT == 0) {
        // 128 rows x 8 blocks; thread -> (row, 4 blocks)
        const int row = tid >> 1, b0 = (tid & 1) * 4;
        const uint32_t base = row * kWRowSlot + (p.w_vec16 ? 0u : static_cast<uint32_t>((n0 + row) * p.row_bytes + ks * p.step_bytes) & 3u);
#pragma unroll
        for (int bb = 0; bb < 4; ++bb) {
            const int b = b0 + bb;
            uint32_t q[4], dbits;
            load_q4_0_block_smem(wr, base + 18u * b, q, dbits);
            uint4 lo, hi;
            lo.x = __vsub4(q[0] & 0x0f0f0f0fu, 0x08080808u);
            lo.y = __vsub4(q[1] & 0x0f0f0f0fu, 0x08080808u);
            lo.z = __vsub4(q[2] & 0x0f0f0f0fu, 0x08080808u);
            lo.w = __vsub4(q[3] & 0x0f0f0f0fu, 0x08080808u);
            hi.x = __vsub4((q[0] >> 4) & 0x0f0f0f0fu, 0x08080808u);
            hi.y = __vsub4((q[1] >> 4) & 0x0f0f0f0fu, 0x08080808u);
            hi.z = __vsub4((q[2] >> 4) & 0x0f0f0f0fu, 0x08080808u);
            hi.w = __vsub4((q[3] >> 4) & 0x0f0f0f0fu, 0x08080808u);
            *reinterpret_cast<uint4 *>(bt + swz(row, 2 * b)) = lo;
            *reinterpret_cast<uint4 *>(bt + swz(row, 2 * b + 1)) = hi;
            const float dw = f16_bits_to_f32(dbits);
            reinterpret_cast<float2 *>(wf)[b * BN + row] = make_float2(dw, -kMagic * dw);
        }
    } else if constexpr (WT == 1) {
        // one 144-byte block per row; thread -> (row, 2 nibble pairs)
        const int row = tid >> 1, h = tid & 1;
        const uint8_t *blk = wr + row * kWRowSlot;
#pragma unroll
        for (int pp = 0; pp < 2; ++pp) {
            const int pr = 2 * h + pp;
#pragma unroll
            for (int half = 0; half < 2; ++half) {
                const uint4 v = *reinterpret_cast<const uint4 *>(blk + 16 + 32 * pr + 16 * half);
                uint4 lo, hi;
                lo.x = v.x & 0x0f0f0f0fu, lo.y = v.y & 0x0f0f0f0fu, lo.z = v.z & 0x0f0f0f0fu, lo.w = v.w & 0x0f0f0f0fu;
                hi.x = (v.x >> 4) & 0x0f0f0f0fu, hi.y = (v.y >> 4) & 0x0f0f0f0fu;
                hi.z = (v.z >> 4) & 0x0f0f0f0fu, hi.w = (v.w >> 4) & 0x0f0f0f0fu;
                // sub-block 2pr holds k = 64 pr + j, sub-block 2pr + 1 holds k = 64 pr + 32 + j
                *reinterpret_cast<uint4 *>(bt + swz(row, 4 * pr + half)) = lo;
                *reinterpret_cast<uint4 *>(bt + swz(row, 4 * pr + 2 + half)) = hi;
            }
        }
        if (h == 0) {
            const uint32_t dd = *reinterpret_cast<const uint32_t *>(blk);
            const uint32_t s0 = *reinterpret_cast<const uint32_t *>(blk + 4);
            const uint32_t s1 = *reinterpret_cast<const uint32_t *>(blk + 8);
            const uint32_t s2 = *reinterpret_cast<const uint32_t *>(blk + 12);
            auto byte = [&](int i) -> uint32_t {
                const uint32_t w = i < 4 ? s0 : (i < 8 ? s1 : s2);
                return (w >> (8 * (i & 3))) & 0xffu;
            };
            int32_t *sc = reinterpret_cast<int32_t *>(wf);      // [8][BN]
            uint32_t mpk0 = 0, mpk1 = 0;
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                uint32_t scv, mnv;
                if (j < 4) {
                    scv = byte(j) & 63u;
                    mnv = byte(j + 4) & 63u;
                } else {
                    scv = (byte(j + 4) & 15u) | ((byte(j - 4) >> 6) << 4);
                    mnv = (byte(j + 4) >> 4) | ((byte(j) >> 6) << 4);
                }
                sc[j * BN + row] = static_cast<int32_t>(scv);
                if (j < 4)
                    mpk0 |= mnv << (8 * j);
                else
                    mpk1 |= mnv << (8 * (j - 4));
            }
            float2 *dm = reinterpret_cast<float2 *>(wf + 8 * BN * 4);       // [BN] (d, dmin)
            uint2 *mp = reinterpret_cast<uint2 *>(wf + 8 * BN * 4 + BN * 8);  // [BN] packed mins
            dm[row] = make_float2(f16_bits_to_f32(dd & 0xffffu), f16_bits_to_f32(dd >> 16));
            mp[row] = make_uint2(mpk0, mpk1);
        }
        // A side: bsum32 of each row split into 6-bit low bytes and high bytes
        if (tid < BM) {
            const int32_t *bsum = sm.a_scale(s) + tid * 8;
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
            sm.a_pack()[tid] = make_uint4(l0, l1, h0, h1);
        }
    } else {
        // iq2_xxs: one 66-byte block per row; thread -> (row, 4 groups of 32)
        const int row = tid >> 1, h = tid & 1;
        const uint32_t base = row * kWRowSlot + (p.w_vec16 ? 0u : static_cast<uint32_t>((n0 + row) * p.row_bytes + ks * p.step_bytes) & 3u);
        const uint2 *grid = reinterpret_cast<const uint2 *>(sm.a_pack());  // grid table lives past the fold data
        int32_t *scl = reinterpret_cast<int32_t *>(wf);                     // [8][BN]
#pragma unroll
        for (int gg = 0; gg < 4; ++gg) {
            const int sb = 4 * h + gg;
            const uint32_t off = base + 2 + 8 * sb;
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
            *reinterpret_cast<uint4 *>(bt + swz(row, 2 * sb)) = make_uint4(v[0], v[1], v[2], v[3]);
            *reinterpret_cast<uint4 *>(bt + swz(row, 2 * sb + 1)) = make_uint4(v[4], v[5], v[6], v[7]);
            scl[sb * BN + row] = 2 * static_cast<int32_t>(ss >> 28) + 1;
        }
        if (h == 0) {
            const uint16_t db = *reinterpret_cast<const uint16_t *>(wr + base);
            reinterpret_cast<float *>(wf + 8 * BN * 4)[row] = __fmul_rn(0.125f, f16_bits_to_f32(db));
        }
    }
}

template <int WT, bool kPartials>
__global__ void __launch_bounds__(kThreads, 1) gemm_kernel(const GemmParams p) {
    extern __shared__ __align__(128) uint8_t smem_raw[];
    Smem sm{smem_raw};
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int wm = warp >> 2, wn = warp & 3;  // 2 x 4 warps of 64 x 32
    const int g = lane >> 2, t4 = lane & 3;
    const int64_t n0 = static_cast<int64_t>(blockIdx.x) * BN;
    const int64_t m0 = static_cast<int64_t>(blockIdx.y) * BM;
    const int64_t KT = p.k / BK;

    if constexpr (WT == 2) {
        // iq2_xxs lattice table (2 KB) after the packed-bsum area
        uint2 *grid = reinterpret_cast<uint2 *>(sm.a_pack());
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

    float acc[4][4][4];
    int iacc[4][4][4];
#pragma unroll
    for (int a = 0; a < 4; ++a)
#pragma unroll
        for (int b = 0; b < 4; ++b)
#pragma unroll
            for (int c = 0; c < 4; ++c) acc[a][b][c] = 0.0f, iacc[a][b][c] = 0;

    int cin[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) cin[i] = (WT == 0 && !kPartials) ? static_cast<int>(kMagicBits) : 0;

#pragma unroll
    for (int s = 0; s < kStages - 1; ++s) {
        if (s < KT) load_stage<WT>(p, sm, s, s, m0, n0, tid);
        cp_async_commit();
    }

    for (int64_t ks = 0; ks < KT; ++ks) {
        const int s = static_cast<int>(ks % kStages);
        cp_async_wait<kStages - 2>();
        __syncthreads();
        decode_w<WT>(p, sm, s, ks, n0, tid);
        if (ks + kStages - 1 < KT) load_stage<WT>(p, sm, static_cast<int>((ks + kStages - 1) % kStages), ks + kStages - 1, m0, n0, tid);
        cp_async_commit();
        __syncthreads();

        const int8_t *at = sm.a_qs(s);
        const int8_t *bt = sm.b_tile();
#pragma unroll 1
        for (int kb = 0; kb < 8; ++kb) {
            uint32_t af[4][4];
#pragma unroll
            for (int mt = 0; mt < 4; ++mt) {
                const int row = wm * 64 + mt * 16 + (lane & 7) + ((lane >> 3) & 1) * 8;
                const int ch = 2 * kb + (lane >> 4);
                ldmatrix_x4(af[mt][0], af[mt][1], af[mt][2], af[mt][3], at + swz(row, ch));
            }
            uint32_t bf[4][2];
#pragma unroll
            for (int np = 0; np < 2; ++np) {
                const int row = wn * 32 + np * 16 + (lane & 7) + ((lane >> 4) & 1) * 8;
                const int ch = 2 * kb + ((lane >> 3) & 1);
                ldmatrix_x4(bf[2 * np][0], bf[2 * np][1], bf[2 * np + 1][0], bf[2 * np + 1][1], bt + swz(row, ch));
            }
            int res[4][4][4];
#pragma unroll
            for (int mt = 0; mt < 4; ++mt)
#pragma unroll
                for (int nt = 0; nt < 4; ++nt) mma_s8(res[mt][nt], af[mt], bf[nt][0], bf[nt][1], cin);

            if constexpr (kPartials) {
                const int64_t nb32 = p.k / 32;
#pragma unroll
                for (int mt = 0; mt < 4; ++mt)
#pragma unroll
                    for (int nt = 0; nt < 4; ++nt)
#pragma unroll
                        for (int i = 0; i < 4; ++i) {
                            const int64_t r = m0 + wm * 64 + mt * 16 + g + 8 * (i >> 1);
                            const int64_t c = n0 + wn * 32 + nt * 8 + 2 * t4 + (i & 1);
                            if (r < p.m && c < p.n) p.partials[(r * p.n + c) * nb32 + ks * 8 + kb] = res[mt][nt][i];
                        }
            } else if constexpr (WT == 0) {
                const float2 *wf = reinterpret_cast<const float2 *>(sm.w_fold()) + kb * BN;
                const float *ad = reinterpret_cast<const float *>(sm.a_scale(s));
                float da[4][2];
#pragma unroll
                for (int mt = 0; mt < 4; ++mt)
#pragma unroll
                    for (int h = 0; h < 2; ++h) da[mt][h] = ad[(wm * 64 + mt * 16 + g + 8 * h) * 8 + kb];
#pragma unroll
                for (int nt = 0; nt < 4; ++nt) {
                    const int col = wn * 32 + nt * 8 + 2 * t4;
                    const float4 f = *reinterpret_cast<const float4 *>(wf + col);  // (dw0, cm0, dw1, cm1)
#pragma unroll
                    for (int mt = 0; mt < 4; ++mt)
#pragma unroll
                        for (int i = 0; i < 4; ++i) {
                            const float y = __int_as_float(res[mt][nt][i]);
                            const float t = (i & 1) ? __fmaf_rn(y, f.z, f.w) : __fmaf_rn(y, f.x, f.y);
                            acc[mt][nt][i] = __fmaf_rn(t, da[mt][i >> 1], acc[mt][nt][i]);
                        }
                }
            } else {
                const int32_t *sc = reinterpret_cast<const int32_t *>(sm.w_fold()) + kb * BN;
#pragma unroll
                for (int nt = 0; nt < 4; ++nt) {
                    const int col = wn * 32 + nt * 8 + 2 * t4;
                    const int2 s2 = *reinterpret_cast<const int2 *>(sc + col);
#pragma unroll
                    for (int mt = 0; mt < 4; ++mt)
#pragma unroll
                        for (int i = 0; i < 4; ++i)
                            iacc[mt][nt][i] += ((i & 1) ? s2.y : s2.x) * res[mt][nt][i];
                }
            }
        }

        if constexpr (!kPartials && WT != 0) {
            // once per 256-block: fold the integer sums into fp32
            const float *ad = sm.a_d8k(s);
            if constexpr (WT == 1) {
                const float2 *dm = reinterpret_cast<const float2 *>(sm.w_fold() + 8 * BN * 4);
                const uint2 *mp = reinterpret_cast<const uint2 *>(sm.w_fold() + 8 * BN * 4 + BN * 8);
#pragma unroll
                for (int mt = 0; mt < 4; ++mt)
#pragma unroll
                    for (int h = 0; h < 2; ++h) {
                        const int row = wm * 64 + mt * 16 + g + 8 * h;
                        const float a_d = ad[row];
                        const uint4 ap = sm.a_pack()[row];
#pragma unroll
                        for (int nt = 0; nt < 4; ++nt)
#pragma unroll
                            for (int e = 0; e < 2; ++e) {
                                const int col = wn * 32 + nt * 8 + 2 * t4 + e;
                                const uint2 mv = mp[col];
                                const float2 dd = dm[col];
                                const int lo = __dp4a(static_cast<int>(mv.x), static_cast<int>(ap.x),
                                                      __dp4a(static_cast<int>(mv.y), static_cast<int>(ap.y), 0));
                                const int hi = __dp4a(static_cast<int>(mv.x), static_cast<int>(ap.z),
                                                      __dp4a(static_cast<int>(mv.y), static_cast<int>(ap.w), 0));
                                const int i2 = lo + 64 * hi;
                                int &i1 = iacc[mt][nt][2 * h + e];
                                const float part = __fsub_rn(__fmul_rn(dd.x, static_cast<float>(i1)),
                                                             __fmul_rn(dd.y, static_cast<float>(i2)));
                                acc[mt][nt][2 * h + e] = __fmaf_rn(a_d, part, acc[mt][nt][2 * h + e]);
                                i1 = 0;
                            }
                    }
            } else {
                const float *wd = reinterpret_cast<const float *>(sm.w_fold() + 8 * BN * 4);
#pragma unroll
                for (int mt = 0; mt < 4; ++mt)
#pragma unroll
                    for (int h = 0; h < 2; ++h) {
                        const float a_d = ad[wm * 64 + mt * 16 + g + 8 * h];
#pragma unroll
                        for (int nt = 0; nt < 4; ++nt)
#pragma unroll
                            for (int e = 0; e < 2; ++e) {
                                const int col = wn * 32 + nt * 8 + 2 * t4 + e;
                                int &ii = iacc[mt][nt][2 * h + e];
                                acc[mt][nt][2 * h + e] =
                                    __fmaf_rn(__fmul_rn(wd[col], a_d), static_cast<float>(ii), acc[mt][nt][2 * h + e]);
                                ii = 0;
                            }
                    }
            }
        }
    }
    cp_async_wait<0>();

    if constexpr (!kPartials) {
#pragma unroll
        for (int mt = 0; mt < 4; ++mt)
#pragma unroll
            for (int nt = 0; nt < 4; ++nt)
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    const int64_t r = m0 + wm * 64 + mt * 16 + g + 8 * (i >> 1);
                    const int64_t c = n0 + wn * 32 + nt * 8 + 2 * t4 + (i & 1);
                    if (r < p.m && c < p.n) p.c[r * p.ldc + c] = acc[mt][nt][i];
                }
    }
}

int64_t row_bytes_of(int wtype, int64_t k) {
    switch (wtype) {
    case 0: return k / 32 * kQ4_0Bytes;
    case 1: return k / 256 * kQ4_KBytes;
    default: return k / 256 * kIQ2Bytes;
    }
}

template <int WT, bool kPartials>
cudaError_t launch_t(const GemmParams &p, cudaStream_t s) {
    auto kernel = gemm_kernel<WT, kPartials>;
    cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(kSmemBytes));
    if (e != cudaSuccess) return e;
    const dim3 grid(static_cast<unsigned>((p.n + BN - 1) / BN), static_cast<unsigned>(p.a.rows_pad / BM));
    kernel<<<grid, kThreads, kSmemBytes, s>>>(p);
    return cudaGetLastError();
}

}  // namespace

bool gemm_supported(int wtype, int64_t m, int64_t n, int64_t k, const void *w) {
    (void)m;
    (void)n;
    if (k % BK != 0) return false;
    if ((reinterpret_cast<uintptr_t>(w) & 15u) != 0) return false;
    return kSmemBytes <= device_smem_optin();
}

cudaError_t launch_gemm(const GemmArgs &args, cudaStream_t s) {
    GemmParams p{};
    p.w = static_cast<const uint8_t *>(args.w);
    p.a = args.a;
    p.c = args.c;
    p.ldc = args.ldc;
    p.partials = args.partials;
    p.m = args.m;
    p.n = args.n;
    p.k = args.k;
    p.row_bytes = row_bytes_of(args.wtype, args.k);
    p.step_bytes = static_cast<uint32_t>(row_bytes_of(args.wtype, BK));
    p.w_total = p.row_bytes * args.n;
    p.w_vec16 = (p.row_bytes % 16 == 0 && p.step_bytes % 16 == 0) ? 1 : 0;
    const bool part = args.partials != nullptr;
    switch (args.wtype) {
    case 0: return part ? launch_t<0, true>(p, s) : launch_t<0, false>(p, s);
    case 1: return part ? launch_t<1, true>(p, s) : launch_t<1, false>(p, s);
    default: return part ? launch_t<2, true>(p, s) : launch_t<2, false>(p, s);
    }
}

}  // namespace pfng
