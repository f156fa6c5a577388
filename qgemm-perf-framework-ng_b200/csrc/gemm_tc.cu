// gemm_tc.cu -- q4_0 x q8_0 batched matmul on the 5th-generation tensor
// cores: tcgen05.mma kind::i8 with the integer sub-block products in tensor
// memory (TMEM), operands brought in by TMA.
//
// C[m][n] = A[m][k] . W[n][k]^T, W raw q4_0 blocks, A in the split layout
// (int8 rows + one fp32 scale per 32) from quantize.cu.  Semantics:
// compute_q4_0, bench/llama_reference/llama_reference.cpp:133-148 and :165-205.
//
// Tile: 128 weight rows (the MMA's M, one TMEM lane each) x 128 activation
// rows (the MMA's N, one TMEM column each), k-steps of 256.  The kernel is
// persistent: CTA c takes tiles c, c + grid, ... with the m tiles fastest, so
// the CTAs running together share their W tiles.  Warp roles (576 threads,
// one CTA per SM):
//   warp 0      TMA producer: per k-step one 2-D tensor copy of the raw W
//               rows (128 x 144 bytes; rows past n read as zeros), two of the
//               int8 activation rows (128 x 128 bytes each, 128-byte swizzle:
//               they land directly in the MMA's K-major operand layout) and
//               one of their scales (128 x 8 floats), all completing one
//               mbarrier's transaction count; two stages;
//   warp 1      TMEM owner and MMA issuer: one tcgen05.mma (M 128, N 128,
//               K 32) per 32-deep sub-block into one of four TMEM buffers
//               (512 columns), completion signalled with tcgen05.commit; the
//               MMA overwrites its buffer (no accumulate), the fold reads it;
//   warps 2-17  decode and fold.  Decode: before folding k-step g each warp
//               decodes its 1/16 of k-step g + 1 (8 weight rows: raw q4_0
//               blocks -> int8 (q - 8) operand rows in the swizzled layout,
//               their scales, and activation scales transposed to
//               [sub-block][row]) -- spread over all 16 warps so that every
//               scheduler carries the same load (with separate decode warps,
//               the fold warps sharing a scheduler with them set the pace
//               and the others waited for the MMA 20 % of the time).
//               Fold: warp w reads TMEM lane quarter w % 4 and column block
//               (w - 2) / 4 (32 activation rows) with two 16x256b loads per
//               sub-block -- thread t holds weight rows t/4 + {0, 8, 16, 24}
//               of the quarter and activation rows 8 j + 2 (t % 4) + {0, 1},
//               j = 0..3, so one activation scale serves four rows and one
//               weight scale eight columns -- hands the buffer back, and folds
//               the 32 products into 32 fp32 accumulators in registers; at
//               the end of a tile they store C and start the next one while
//               the MMA already fills the buffers again.
// The fold is the exact two-FMA scheme of gemm.cu: the int32 product P plus
// the integer 0x4B400000 is the float 2^23 + 2^22 + P exactly (one integer
// add, no conversion); t = fma(y, s, -(2^23+2^22) s) = round(P s) with
// s = d_w (fp16, exact products), acc = fma(t, d_a, acc), sub-blocks in k
// order -- the same operations in the same order as the mma.sync kernel, so
// the results are bit-identical to it (unsplit).
//
// Loads read this GPU's memory only (W, the activation operand), each CTA
// its own copy.  Every wait is bounded; a wait that gives up records an error,
// raises the CTA's abort flag (which ends every other role's waits at once)
// and the CTA frees its TMEM before returning.
#include <mutex>

#include "pfng_common.cuh"
#include "pfng_internal.h"
#include "pfng_tma.h"

namespace pfng {
namespace {

constexpr int TM = 128;        // weight rows per tile (TMEM lanes)
constexpr int TN = 128;        // activation rows per tile (TMEM columns)
constexpr int BK = 256;        // k per k-step
constexpr int kStages = 2;     // TMA load stages
constexpr int kDecBufs = 2;    // decoded weight operand buffers
constexpr int kTmemBufs = 4;   // sub-block products in TMEM
constexpr uint32_t kTmemCols = kTmemBufs * TN;  // 512: all of TMEM
constexpr int kThreads = 576;
constexpr int kFoldWarps = 16;
constexpr int kFoldWarp0 = 2;
constexpr uint32_t kRawRow = 144;  // raw q4_0 bytes of one weight row per k-step
constexpr uint32_t kMagicBits = 0x4B400000u;
constexpr float kMagic = 12582912.0f;

// shared memory plan (dynamic, base aligned to 1024 for the swizzle atoms)
constexpr uint32_t kRawBytes = TM * kRawRow;               // 18 KB: W rows as in memory
constexpr uint32_t kActBytes = TN * BK;                    // 32 KB: [2 col blocks][128 rows][128 B], swizzled
constexpr uint32_t kActScaleBytes = TN * 8 * 4;            // 4 KB: [8 blocks][128 rows] floats (split_d_index order)
constexpr uint32_t kStageBytes = kRawBytes + kActBytes + kActScaleBytes;  // 54 KB
constexpr uint32_t kWOpBytes = TM * BK;                    // 32 KB: decoded W, [2 col blocks][128 rows][128 B]
constexpr uint32_t kSwBytes = TM * 8 * 4;                  // 4 KB: weight scales [128 rows][8]
constexpr uint32_t kDaTBytes = 8 * TN * 4;                 // 4 KB: activation scales [8][128 rows]
constexpr uint32_t kDecBytes = kWOpBytes + kSwBytes + kDaTBytes;
constexpr uint32_t kOffStage = 0;
constexpr uint32_t kOffDec = kOffStage + kStages * kStageBytes;
constexpr uint32_t kOffBar = kOffDec + kDecBufs * kDecBytes;
constexpr uint32_t kNumBars = 2 * kStages + 2 * kDecBufs + 2 * kTmemBufs + 1;
constexpr uint32_t kSmemBytes = kOffBar + kNumBars * 8 + 16 + 1024;  // + TMEM address, alignment slack
static_assert(kRawBytes % 1024 == 0 && kStageBytes % 1024 == 0 && kDecBytes % 1024 == 0, "1024-byte atoms");
constexpr uint32_t kStageTx = kRawBytes + kActBytes + kActScaleBytes;  // bytes the TMA lands per stage

struct TcParams {
    float *c;
    int64_t ldc;
    int64_t m, n, k;
    int mtiles, ntiles;
    int *err;
};

// ---- TMA / tcgen05 / proxy primitives ----------------------------------------
PFNG_DEV void fence_proxy_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }
PFNG_DEV void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
PFNG_DEV void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

PFNG_DEV void tmem_alloc(uint32_t *holder, uint32_t ncols) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(holder)),
                 "r"(ncols)
                 : "memory");
}
PFNG_DEV void tmem_relinquish() { asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory"); }
PFNG_DEV void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}

// D[tmem] (+)= A[smem] . B[smem]^T, int8 x int8 -> int32; accumulate != 0 adds onto D.
PFNG_DEV void umma_i8(uint32_t tmem_d, uint64_t desc_a, uint64_t desc_b, uint32_t idesc, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, {%5, %5, %5, %5}, p;\n\t}"
        ::"r"(tmem_d), "l"(desc_a), "l"(desc_b), "r"(idesc), "r"(accumulate), "r"(0u)
        : "memory");
}
// Arrives on `bar` once every tcgen05.mma this thread issued before has completed.
PFNG_DEV void umma_commit(uint64_t *bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
                 : "memory");
}

#define PFNG_R32(x) \
    "=r"(x[0]), "=r"(x[1]), "=r"(x[2]), "=r"(x[3]), "=r"(x[4]), "=r"(x[5]), "=r"(x[6]), "=r"(x[7]), "=r"(x[8]), \
        "=r"(x[9]), "=r"(x[10]), "=r"(x[11]), "=r"(x[12]), "=r"(x[13]), "=r"(x[14]), "=r"(x[15]), "=r"(x[16]), \
        "=r"(x[17]), "=r"(x[18]), "=r"(x[19]), "=r"(x[20]), "=r"(x[21]), "=r"(x[22]), "=r"(x[23]), "=r"(x[24]), \
        "=r"(x[25]), "=r"(x[26]), "=r"(x[27]), "=r"(x[28]), "=r"(x[29]), "=r"(x[30]), "=r"(x[31])

// Two 16x256b.x4 loads (lanes base .. base + 15 at ta, base + 16 .. base + 31
// at tb; 32 consecutive columns each) and their wait, as one statement.
// Each load gives thread t, for column chunk j = 0..3, the values
// 4 j + {0, 1} = lane t/4, columns 8 j + 2 (t % 4) + {0, 1} and
// 4 j + {2, 3} = lane t/4 + 8, the same columns; value v of the second load
// is number 16 + v.  They come back packed in pairs (d[p] = values 2 p and
// 2 p + 1), the operand pairs of the packed fmas.
PFNG_DEV void tmem_ld_16x256b_2x4(uint32_t ta, uint32_t tb, uint64_t (&d)[16]) {
    asm volatile(
        "{\n\t.reg .b32 a<32>;\n\t"
        "tcgen05.ld.sync.aligned.16x256b.x4.b32 {a0, a1, a2, a3, a4, a5, a6, a7, a8, a9, a10, a11, a12, a13, a14, a15}, [%16];\n\t"
        "tcgen05.ld.sync.aligned.16x256b.x4.b32 {a16, a17, a18, a19, a20, a21, a22, a23, a24, a25, a26, a27, a28, a29, a30, a31}, [%17];\n\t"
        "tcgen05.wait::ld.sync.aligned;\n\t"
        "mov.b64 %0, {a0, a1};\n\t"
        "mov.b64 %1, {a2, a3};\n\t"
        "mov.b64 %2, {a4, a5};\n\t"
        "mov.b64 %3, {a6, a7};\n\t"
        "mov.b64 %4, {a8, a9};\n\t"
        "mov.b64 %5, {a10, a11};\n\t"
        "mov.b64 %6, {a12, a13};\n\t"
        "mov.b64 %7, {a14, a15};\n\t"
        "mov.b64 %8, {a16, a17};\n\t"
        "mov.b64 %9, {a18, a19};\n\t"
        "mov.b64 %10, {a20, a21};\n\t"
        "mov.b64 %11, {a22, a23};\n\t"
        "mov.b64 %12, {a24, a25};\n\t"
        "mov.b64 %13, {a26, a27};\n\t"
        "mov.b64 %14, {a28, a29};\n\t"
        "mov.b64 %15, {a30, a31};\n\t"
        "}"
        : "=l"(d[0]), "=l"(d[1]), "=l"(d[2]), "=l"(d[3]), "=l"(d[4]), "=l"(d[5]), "=l"(d[6]), "=l"(d[7]), "=l"(d[8]), "=l"(d[9]), "=l"(d[10]), "=l"(d[11]), "=l"(d[12]), "=l"(d[13]), "=l"(d[14]), "=l"(d[15])
        : "r"(ta), "r"(tb)
        : "memory");
}
#undef PFNG_R32


// Shared-memory matrix descriptor, K-major operand with the 128-byte swizzle:
// rows of 128 bytes, 8-row atoms of 1024 bytes stored back to back (stride
// byte offset 1024), the 16-byte chunk j of row r stored at chunk j ^ (r % 8)
// -- the layout a TMA copy with CU_TENSOR_MAP_SWIZZLE_128B and a 128-byte
// inner box writes.  `saddr` is the operand's first byte for this MMA (atom
// base + k offset).
PFNG_DEV uint64_t sw128_desc(uint32_t saddr) {
    uint64_t d = static_cast<uint64_t>((saddr >> 4) & 0x3FFFu);  // start address, 16-byte units
    d |= static_cast<uint64_t>(1u) << 16;                         // leading byte offset (unused with this swizzle)
    d |= static_cast<uint64_t>(1024u >> 4) << 32;                 // stride byte offset between 8-row atoms
    d |= static_cast<uint64_t>(1u) << 46;                         // descriptor version of sm_100
    d |= static_cast<uint64_t>(2u) << 61;                         // layout: 128-byte swizzle
    return d;
}
// Instruction descriptor: int32 accumulator, signed int8 A and B, both
// K-major, N = TN, M = TM.
constexpr uint32_t kIdesc = (2u << 4) | (1u << 7) | (1u << 10) | (static_cast<uint32_t>(TN >> 3) << 17) |
                            (static_cast<uint32_t>(TM >> 4) << 24);

// Byte offset of (row, 16-byte chunk c in 0..15 of the 256-byte k-step) in a
// 128-row operand tile: column block c / 8, swizzled chunk within it.
PFNG_DEV uint32_t op_off(uint32_t row, uint32_t c) {
    return (c >> 3) * TM * 128u + (row >> 3) * 1024u + (row & 7u) * 128u + (((c & 7u) ^ (row & 7u)) << 4);
}

// Bounded wait that also gives up (false) once the CTA's abort flag is up.
// Each attempt is a hardware-suspended try_wait, so a waiting warp issues
// almost nothing; the abort flag is looked at every 16 attempts.
PFNG_DEV bool wait_bar(uint64_t *bar, uint32_t parity, const int *abort_flag, int *err, int code) {
    for (uint32_t i = 0; i < kWaitAttempts; ++i) {
        if (mbar_try_wait(bar, parity)) return true;
        if ((i & 15u) == 15u && *reinterpret_cast<const volatile int *>(abort_flag)) return false;
    }
    report_error(err, code);
    return false;
}
PFNG_DEV bool aborted(const int *abort_flag) { return *reinterpret_cast<const volatile int *>(abort_flag) != 0; }
// The wait of the roles off the critical path (producer, MMA issuer): each
// attempt may suspend the thread for up to 20 us (or until the phase
// completes), so that its polling does not take issue slots from the fold
// warps on its scheduler; the wait is bounded by ~1 s of wall time
// (%globaltimer), whatever the suspensions actually last.
PFNG_DEV uint64_t global_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}
PFNG_DEV bool mbar_try_wait_long(uint64_t *bar, uint32_t parity) {
    uint32_t done;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, 20000;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(done)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return done != 0;
}
PFNG_DEV bool wait_bar_sleep(uint64_t *bar, uint32_t parity, const int *abort_flag, int *err, int code) {
    if (mbar_try_wait_long(bar, parity)) return true;
    const uint64_t t0 = global_ns();
    for (;;) {
        if (mbar_try_wait_long(bar, parity)) return true;
        if (*reinterpret_cast<const volatile int *>(abort_flag)) return false;
        if (global_ns() - t0 > 1000000000ull) break;
    }
    report_error(err, code);
    return false;
}

__global__ void __launch_bounds__(kThreads, 1)
    gemm_tc_q4_0_kernel(const __grid_constant__ CUtensorMap map_w, const __grid_constant__ CUtensorMap map_a,
                        const __grid_constant__ CUtensorMap map_ad, const TcParams p) {
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    // the 1024-byte aligned base as an offset into the shared array, so that
    // the compiler keeps shared-memory (not generic) accesses
    uint8_t *smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
    uint64_t *bars = reinterpret_cast<uint64_t *>(smem + kOffBar);
    uint64_t *ld_full = bars;                          // [kStages]  TMA transaction count
    uint64_t *ld_empty = ld_full + kStages;            // [kStages]  MMA commit (1) + fold warps (decode)
    uint64_t *dec_full = ld_empty + kStages;           // [kDecBufs] fold warps (decode)
    uint64_t *dec_empty = dec_full + kDecBufs;         // [kDecBufs] MMA commit (1) + fold warps
    uint64_t *tm_full = dec_empty + kDecBufs;          // [kTmemBufs] MMA commit (1)
    uint64_t *tm_empty = tm_full + kTmemBufs;          // [kTmemBufs] fold warps
    uint64_t *mma_done = tm_empty + kTmemBufs;         // every issued MMA has completed (commit)
    uint32_t *tmem_holder = reinterpret_cast<uint32_t *>(bars + kNumBars);
    __shared__ int abort_flag;

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int ksteps = static_cast<int>(p.k / BK);
    const int ntiles_total = p.mtiles * p.ntiles;

    if (tid == 0) {
        abort_flag = 0;
        for (int s = 0; s < kStages; ++s) {
            mbar_init(&ld_full[s], 1);
            mbar_init(&ld_empty[s], 1 + kFoldWarps);
        }
        for (int d = 0; d < kDecBufs; ++d) {
            mbar_init(&dec_full[d], kFoldWarps);
            mbar_init(&dec_empty[d], 1 + kFoldWarps);
        }
        for (int b = 0; b < kTmemBufs; ++b) {
            mbar_init(&tm_full[b], 1);
            mbar_init(&tm_empty[b], kFoldWarps);
        }
        mbar_init(mma_done, 1);
        fence_mbar_init();
        prefetch_map(&map_w);
        prefetch_map(&map_a);
        prefetch_map(&map_ad);
    }
    if (warp == 1) {
        tmem_alloc(tmem_holder, kTmemCols);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = *reinterpret_cast<volatile uint32_t *>(tmem_holder);
    const uint32_t s_base = smem_u32(smem);
    // a programmatic dependent of the activation quantizer: everything
    // above overlaps its tail, everything below reads its output
    pdl_wait();

    if (warp == 0) {
        // ---------------- TMA producer (one thread) ----------------
        if (lane == 0) {
            int g = 0;
            for (int t = blockIdx.x; t < ntiles_total && !aborted(&abort_flag); t += gridDim.x) {
                const int mb = t % p.mtiles, nb = t / p.mtiles;
                for (int ks = 0; ks < ksteps; ++ks, ++g) {
                    const int s = g % kStages;
                    if (g >= kStages &&
                        !wait_bar_sleep(&ld_empty[s], ((g / kStages) - 1) & 1, &abort_flag, p.err, kErrWaitEmpty)) {
                        abort_flag = 1;
                        break;
                    }
                    if (aborted(&abort_flag)) break;
                    const uint32_t st = s_base + kOffStage + s * kStageBytes;
                    mbar_arrive_expect_tx(&ld_full[s], kStageTx);
                    tma_load_2d(st, &map_w, ks * static_cast<int>(kRawRow), nb * TM, &ld_full[s]);
                    tma_load_2d(st + kRawBytes, &map_a, ks * BK, mb * TN, &ld_full[s]);
                    tma_load_2d(st + kRawBytes + kActBytes / 2, &map_a, ks * BK + 128, mb * TN, &ld_full[s]);
                    tma_load_2d(st + kRawBytes + kActBytes, &map_ad, mb * TN, ks * 8, &ld_full[s]);
                }
            }
            // on an abort the consumers stop waiting: do not let the CTA end
            // while copies into its shared memory are in flight
            if (aborted(&abort_flag))
                for (int i = g - kStages > 0 ? g - kStages : 0; i < g; ++i)
                    mbar_wait(&ld_full[i % kStages], static_cast<uint32_t>((i / kStages) & 1), p.err, kErrWaitFull);
        }
        __syncwarp();
    } else if (warp == 1) {
        // ---------------- MMA issue (one thread) ----------------
        if (lane == 0) {
            int g = 0, gsb = 0;
            bool ok = true;
            for (int t = blockIdx.x; t < ntiles_total && ok; t += gridDim.x) {
                for (int ks = 0; ks < ksteps && ok; ++ks, ++g) {
                    const int s = g % kStages, d = g % kDecBufs;
                    if (!wait_bar_sleep(&ld_full[s], (g / kStages) & 1, &abort_flag, p.err, kErrWaitFull) ||
                        !wait_bar_sleep(&dec_full[d], (g / kDecBufs) & 1, &abort_flag, p.err, kErrWaitFull)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t wop = s_base + kOffDec + d * kDecBytes;
                    const uint32_t aop = s_base + kOffStage + s * kStageBytes + kRawBytes;
                    for (int sb = 0; sb < 8; ++sb, ++gsb) {
                        const int buf = gsb % kTmemBufs;
                        if (!wait_bar_sleep(&tm_empty[buf], (gsb / kTmemBufs) & 1, &abort_flag, p.err, kErrWaitEmpty)) {
                            ok = false;
                            break;
                        }
                        tc_fence_after();
                        const uint32_t koff = (sb & 3) * 32u;  // k offset inside the 128-byte swizzled row
                        const uint64_t da = sw128_desc(wop + (sb >> 2) * (TM * 128u) + koff);
                        const uint64_t db = sw128_desc(aop + (sb >> 2) * (TN * 128u) + koff);
                        umma_i8(tmem_base + static_cast<uint32_t>(buf * TN), da, db, kIdesc, 0u);
                        umma_commit(&tm_full[buf]);
                    }
                    if (!ok) break;
                    umma_commit(&dec_empty[d]);
                    umma_commit(&ld_empty[s]);
                }
            }
            if (!ok) abort_flag = 1;
            // TMEM is freed at the end: wait until no MMA is in flight
            umma_commit(mma_done);
            if (!mbar_wait(mma_done, 0, p.err, kErrWaitFull)) abort_flag = 1;
        }
        __syncwarp();
    } else {
        // ---------------- decode + fold (warps 2..17) ----------------
        const int fw = warp - kFoldWarp0;
        const int qtr = warp & 3;                // TMEM lane quarter this warp may access
        const int cb = fw >> 2;                  // activation rows 32 cb .. 32 cb + 31 of the tile
        const int r0 = qtr * 32 + (lane >> 2);   // weight rows r0 + {0, 8, 16, 24} of the tile
        const int c0 = cb * 32 + 2 * (lane & 3); // activation rows c0 + 8 j + {0, 1}
        const uint32_t ta = tmem_base + (static_cast<uint32_t>(qtr * 32) << 16) + static_cast<uint32_t>(cb * 32);
        const uint32_t tb = ta + (16u << 16);
        // k-steps of this CTA: global index g = tile i * ksteps + ks
        const int my_tiles = (ntiles_total - static_cast<int>(blockIdx.x) + static_cast<int>(gridDim.x) - 1) /
                             static_cast<int>(gridDim.x);
        const int total = my_tiles * ksteps;
        // every TMEM buffer starts free
        if (lane == 0)
            for (int b = 0; b < kTmemBufs; ++b) mbar_arrive(&tm_empty[b]);

        // this warp's share of k-step gg: weight rows 8 fw .. 8 fw + 7 (two
        // blocks per thread) and 64 transposed activation scales
        auto decode = [&](int gg) -> bool {
            const int s = gg % kStages, d = gg % kDecBufs;
            if (!wait_bar(&ld_full[s], (gg / kStages) & 1, &abort_flag, p.err, kErrWaitFull) ||
                (gg >= kDecBufs &&
                 !wait_bar(&dec_empty[d], ((gg / kDecBufs) - 1) & 1, &abort_flag, p.err, kErrWaitEmpty)))
                return false;
            const uint8_t *raw = smem + kOffStage + s * kStageBytes;
            uint8_t *dec = smem + kOffDec + d * kDecBytes;
            float *sw = reinterpret_cast<float *>(dec + kWOpBytes);
#pragma unroll
            for (int i = 0; i < 2; ++i) {
                const int task = fw * 64 + i * 32 + lane;  // (row, block)
                const int row = task >> 3, u = task & 7;
                uint32_t q[4], dbits;
                load_q4_0_block_smem(raw, row * kRawRow + 18u * u, q, dbits);
                // q - 8 per byte: set bit 7, subtract 8 (no borrow crosses a byte), clear bit 7 again
                uint4 lo, hi;
                lo.x = (((q[0] & 0x0f0f0f0fu) | 0x80808080u) - 0x08080808u) ^ 0x80808080u;
                lo.y = (((q[1] & 0x0f0f0f0fu) | 0x80808080u) - 0x08080808u) ^ 0x80808080u;
                lo.z = (((q[2] & 0x0f0f0f0fu) | 0x80808080u) - 0x08080808u) ^ 0x80808080u;
                lo.w = (((q[3] & 0x0f0f0f0fu) | 0x80808080u) - 0x08080808u) ^ 0x80808080u;
                hi.x = ((((q[0] >> 4) & 0x0f0f0f0fu) | 0x80808080u) - 0x08080808u) ^ 0x80808080u;
                hi.y = ((((q[1] >> 4) & 0x0f0f0f0fu) | 0x80808080u) - 0x08080808u) ^ 0x80808080u;
                hi.z = ((((q[2] >> 4) & 0x0f0f0f0fu) | 0x80808080u) - 0x08080808u) ^ 0x80808080u;
                hi.w = ((((q[3] >> 4) & 0x0f0f0f0fu) | 0x80808080u) - 0x08080808u) ^ 0x80808080u;
                // the 8 threads of a row store together: order the two chunks so
                // that each store instruction covers 8 distinct bank groups
                const bool swap = u >= 4;
                *reinterpret_cast<uint4 *>(dec + op_off(row, swap ? 2 * u + 1 : 2 * u)) = swap ? hi : lo;
                *reinterpret_cast<uint4 *>(dec + op_off(row, swap ? 2 * u : 2 * u + 1)) = swap ? lo : hi;
                sw[row * 8 + u] = f16_bits_to_f32(dbits);
            }
            // activation scales: the stage holds [sub-block][g 16 + j] for
            // tile row 8 j + g (split_d_index); put them in row order
            const float *dar = reinterpret_cast<const float *>(raw + kRawBytes + kActBytes);
            float *dat = reinterpret_cast<float *>(dec + kWOpBytes + kSwBytes);
            static_assert(TN == 128, "one 128-row group of the split operand per tile");
#pragma unroll
            for (int i = 0; i < 2; ++i) {
                const int e = fw * 64 + i * 32 + lane;  // e = sb * TN + activation row
                const int row = e % TN;
                dat[e] = dar[(e / TN) * TN + (row & 7) * 16 + (row >> 3)];
            }
            fence_proxy_async_smem();  // the decoded operand is read by the tensor cores
            __syncwarp();
            if (lane == 0) {
                mbar_arrive(&dec_full[d]);
                mbar_arrive(&ld_empty[s]);
            }
            return true;
        };

        bool ok = total == 0 || decode(0);
        // acc[h][j][s]: weight row r0 + 16 h + 8 s, activation rows c0 + 8 j + {0, 1}
        float2 acc[2][4][2];
        for (int g = 0; g < total && ok; ++g) {
            const int ks = g % ksteps;
            if (ks == 0) {
#pragma unroll
                for (int h = 0; h < 2; ++h)
#pragma unroll
                    for (int j = 0; j < 4; ++j) acc[h][j][0] = acc[h][j][1] = make_float2(0.0f, 0.0f);
            }
            // the next k-step's decode first, then this one's fold
            if (g + 1 < total && !decode(g + 1)) {
                ok = false;
                break;
            }
            const int d = g % kDecBufs;
            if (!wait_bar(&dec_full[d], (g / kDecBufs) & 1, &abort_flag, p.err, kErrWaitFull)) {
                ok = false;
                break;
            }
            const uint8_t *dec = smem + kOffDec + d * kDecBytes;
            const float *swr = reinterpret_cast<const float *>(dec + kWOpBytes) + r0 * 8;
            const float *dat = reinterpret_cast<const float *>(dec + kWOpBytes + kSwBytes) + c0;
            // the sub-block counter advances by 8 (twice the buffer count) per
            // k-step, so each sub-block's buffer and phase parity are constants
            static_assert(kTmemBufs == 4, "buffer = sb % 4, parity = sb / 4");
#pragma unroll
            for (int sb = 0; sb < 8; ++sb) {
                const int buf = sb & 3;
                if (!wait_bar(&tm_full[buf], (sb >> 2) & 1, &abort_flag, p.err, kErrWaitFull)) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                uint64_t r[16];
                tmem_ld_16x256b_2x4(ta + buf * TN, tb + buf * TN, r);
                // the products are in registers: hand the buffer back to
                // the MMA issuer before the arithmetic
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(&tm_empty[buf]);
                // weight scales of rows r0 + 8 i (i = 2 h + s), activation scales of the columns
                float sv[4];
#pragma unroll
                for (int i = 0; i < 4; ++i) sv[i] = swr[i * 64 + sb];
                float2 da[4];
#pragma unroll
                for (int j = 0; j < 4; ++j) da[j] = *reinterpret_cast<const float2 *>(dat + sb * TN + 8 * j);
#pragma unroll
                for (int h = 0; h < 2; ++h)
#pragma unroll
                    for (int ss = 0; ss < 2; ++ss) {
                        const float s1 = sv[2 * h + ss];
                        const float2 sc = make_float2(s1, s1);
                        const float2 cm = make_float2(-kMagic * s1, -kMagic * s1);
#pragma unroll
                        for (int j = 0; j < 4; ++j) {
                            // P + 0x4B400000 as an integer is the float 2^23 + 2^22 + P
                            const uint64_t q = r[8 * h + 2 * j + ss];
                            const float2 y = make_float2(__uint_as_float(static_cast<uint32_t>(q) + kMagicBits),
                                                         __uint_as_float(static_cast<uint32_t>(q >> 32) + kMagicBits));
                            const float2 tt = __ffma2_rn(y, sc, cm);
                            acc[h][j][ss] = __ffma2_rn(tt, da[j], acc[h][j][ss]);
                        }
                    }
            }
            if (!ok) break;
            __syncwarp();
            if (lane == 0) mbar_arrive(&dec_empty[d]);
            if (ks == ksteps - 1) {
                // epilogue: C[m][n] for this thread's 4 weight rows x 8 activation rows
                const int t = static_cast<int>(blockIdx.x) + (g / ksteps) * static_cast<int>(gridDim.x);
                const int mb = t % p.mtiles, nb = t / p.mtiles;
                const int64_t m0 = static_cast<int64_t>(mb) * TN + c0;
#pragma unroll
                for (int h = 0; h < 2; ++h)
#pragma unroll
                    for (int ss = 0; ss < 2; ++ss) {
                        const int64_t n = static_cast<int64_t>(nb) * TM + r0 + 16 * h + 8 * ss;
                        if (n >= p.n) continue;
#pragma unroll
                        for (int j = 0; j < 4; ++j) {
                            const int64_t m = m0 + 8 * j;
                            if (m < p.m) p.c[m * p.ldc + n] = acc[h][j][ss].x;
                            if (m + 1 < p.m) p.c[(m + 1) * p.ldc + n] = acc[h][j][ss].y;
                        }
                    }
            }
        }
        if (!ok) abort_flag = 1;
    }

    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem_base, kTmemCols);
    }
}

}  // namespace

// ---- host: tensor maps ------------------------------------------------------
PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void *p = nullptr;
        cudaDriverEntryPointQueryResult q{};
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
    });
    return fn;
}

bool encode_nd(CUtensorMap *map, CUtensorMapDataType type, int rank, const void *base, const uint64_t *dims,
               const uint64_t *strides, const uint32_t *box) {
    auto fn = encode_fn();
    if (!fn || rank < 1 || rank > 5) return false;
    cuuint64_t d[5], st[4];
    cuuint32_t b[5], e[5];
    for (int i = 0; i < rank; ++i) {
        d[i] = dims[i];
        b[i] = box[i];
        e[i] = 1;
        if (i + 1 < rank) st[i] = strides[i];
    }
    return fn(map, type, static_cast<cuuint32_t>(rank), const_cast<void *>(base), d, st, b, e,
              CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

bool encode_2d(CUtensorMap *map, CUtensorMapDataType type, const void *base, uint64_t cols, uint64_t rows,
               uint64_t stride, uint32_t box_cols, uint32_t box_rows, CUtensorMapSwizzle swizzle) {
    auto fn = encode_fn();
    if (!fn) return false;
    const cuuint64_t dims[2] = {cols, rows};
    const cuuint64_t strides[1] = {stride};
    const cuuint32_t box[2] = {box_cols, box_rows};
    const cuuint32_t estr[2] = {1, 1};
    return fn(map, type, 2, const_cast<void *>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle,
              CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

bool gemm_tc_supported(int wtype, int64_t m, int64_t n, int64_t k, const void *w) {
    (void)m;
    (void)n;
    return wtype == 0 && k > 0 && k % BK == 0 && (reinterpret_cast<uintptr_t>(w) & 15u) == 0 &&
           kSmemBytes <= device_smem_optin() && encode_fn() != nullptr;
}

cudaError_t launch_gemm_tc(const GemmArgs &args, int *err, cudaStream_t s) {
    const int64_t row_bytes = args.k / 32 * kQ4_0Bytes;  // a multiple of 144 (k % 256 == 0)
    CUtensorMap map_w, map_a, map_ad;
    if (!encode_2d(&map_w, CU_TENSOR_MAP_DATA_TYPE_UINT8, args.w, static_cast<uint64_t>(row_bytes),
                   static_cast<uint64_t>(args.n), static_cast<uint64_t>(row_bytes), kRawRow, TM,
                   CU_TENSOR_MAP_SWIZZLE_NONE) ||
        !encode_2d(&map_a, CU_TENSOR_MAP_DATA_TYPE_UINT8, args.a.qs, static_cast<uint64_t>(args.k),
                   static_cast<uint64_t>(args.a.rows_pad), static_cast<uint64_t>(args.k), 128, TN,
                   CU_TENSOR_MAP_SWIZZLE_128B) ||
        // q8_0 scales: [k / 32] slabs of d_ld floats (split_d_index), a box
        // of one tile's 128 rows x the k-step's 8 blocks
        !encode_2d(&map_ad, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, args.a.d, static_cast<uint64_t>(args.a.rows_pad),
                   static_cast<uint64_t>(args.k / 32), static_cast<uint64_t>(args.a.d_ld * 4), TN, 8,
                   CU_TENSOR_MAP_SWIZZLE_NONE))
        return cudaErrorInvalidValue;
    TcParams p{};
    p.c = args.c;
    p.ldc = args.ldc;
    p.m = args.m;
    p.n = args.n;
    p.k = args.k;
    p.mtiles = static_cast<int>((args.m + TN - 1) / TN);
    p.ntiles = static_cast<int>((args.n + TM - 1) / TM);
    p.err = err;
    static thread_local bool configured[64] = {false};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 0 || dev >= 64 || !configured[dev]) {
        const cudaError_t e = cudaFuncSetAttribute(gemm_tc_q4_0_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                   static_cast<int>(kSmemBytes));
        if (e != cudaSuccess) return e;
        if (dev >= 0 && dev < 64) configured[dev] = true;
    }
    const int64_t tiles = static_cast<int64_t>(p.mtiles) * p.ntiles;
    const int64_t sms = device_sm_count();
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3(static_cast<unsigned>(tiles < sms ? tiles : sms));
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = kSmemBytes;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, gemm_tc_q4_0_kernel, map_w, map_a, map_ad, p);
}

}  // namespace pfng
