// gemm_tc.cu -- q4_0 x q8_0 batched matmul on the 5th-generation tensor
// cores: tcgen05.mma kind::i8 with the accumulators in tensor memory (TMEM).
//
// C[m][n] = A[m][k] . W[n][k]^T, W raw q4_0 blocks, A in the split layout
// (int8 rows + one fp32 scale per 32) from quantize.cu.  Semantics:
// compute_q4_0, bench/llama_reference/llama_reference.cpp:133-148 and :165-205.
//
// Tile: 128 weight rows (the MMA's M, one TMEM lane each) x 64 activation
// rows (the MMA's N), k-steps of 256.  Warp roles (384 threads, one CTA/SM):
//   warp 0      loads: raw W rows, activation int8 rows (written straight
//               into the 128-byte-swizzled K-major operand layout) and the
//               activation scales, with cp.async into a 3-stage ring whose
//               stages complete an mbarrier (cp.async.mbarrier.arrive);
//   warp 1      TMEM owner and MMA issuer: one tcgen05.mma (M 128, N 64,
//               K 32) per 32-deep sub-block, each into its own TMEM buffer
//               (8 buffers, a whole k-step), completion signalled with
//               tcgen05.commit; each MMA overwrites its buffer (no
//               accumulate), the fold reads it;
//   warps 2,3   decode: raw q4_0 blocks -> int8 (q - 8) operand rows in
//               the swizzled layout, the per-(row, sub-block) weight scales,
//               and the activation scales transposed to [sub-block][row];
//   warps 4-11  fold, thread = weight row, warps 4-7 activation rows 0-31 and
//               warps 8-11 rows 32-63 (two warps per scheduler hide the TMEM
//               load latency).  For each sub-block, tcgen05.ld the 32 int32
//               partials, release the buffer at once, and fold them into 32
//               fp32 accumulators in registers.
// The fold is the exact two-FMA scheme of gemm.cu: the int32 partial P read
// back plus the integer 0x4B400000 is the float 2^23 + 2^22 + P exactly (one
// integer add, no conversion); t = fma(y, s, -(2^23+2^22) s)
// = round(P s) with s = d_w (fp16, exact products), acc = fma(t, d_a, acc).
// Each output element costs an integer add and one packed FMA pair per
// sub-block; the MMAs, operand fetch and accumulation run beside them.
//
// Every wait is bounded; a wait that gives up records an error, raises the
// CTA's abort flag (which ends every other role's waits at once) and the CTA
// frees its TMEM before returning.
#include "pfng_common.cuh"
#include "pfng_internal.h"

namespace pfng {
namespace {

constexpr int TM = 128;        // weight rows per tile
constexpr int TN = 64;         // activation rows per tile
constexpr int BK = 256;        // k per stage
constexpr int kLoadStages = 3;
constexpr int kABufs = 2;      // decoded weight operand buffers
constexpr int kTmemBufs = 8;   // sub-block accumulators in TMEM
constexpr uint32_t kTmemCols = kTmemBufs * TN;  // 512: all of TMEM
constexpr int kThreads = 384;
constexpr int kFoldWarps = 8;
constexpr int kDecodeWarps = 2;
constexpr uint32_t kRawSlot = 160;  // bytes per raw weight row per stage (144 used)
constexpr uint32_t kMagicBits = 0x4B400000u;
constexpr float kMagic = 12582912.0f;

// shared memory plan (dynamic, base aligned to 1024 for the swizzle atoms)
constexpr uint32_t kAOpBytes = TM * BK;                    // 32 KB, [2 col blocks][128 rows][128 B]
constexpr uint32_t kBOpBytes = TN * BK;                    // 16 KB, [2 col blocks][64 rows][128 B]
constexpr uint32_t kRawBytes = TM * kRawSlot;              // 20 KB
constexpr uint32_t kDaRawBytes = TN * 8 * 4;               // 2 KB, [64 rows][8]
constexpr uint32_t kSwBytes = TM * 8 * 4;                  // 4 KB, weight scales [128 rows][8]
constexpr uint32_t kDaTBytes = 8 * TN * 4;                 // 2 KB, activation scales [8][64 rows]
constexpr uint32_t kOffA = 0;
constexpr uint32_t kOffB = kOffA + kABufs * kAOpBytes;                  // 64 KB
constexpr uint32_t kOffRaw = kOffB + kLoadStages * kBOpBytes;           // 112 KB
constexpr uint32_t kOffDaRaw = kOffRaw + kLoadStages * kRawBytes;       // 172 KB
constexpr uint32_t kOffSw = kOffDaRaw + kLoadStages * kDaRawBytes;
constexpr uint32_t kOffDaT = kOffSw + kABufs * kSwBytes;
constexpr uint32_t kOffBar = kOffDaT + kABufs * kDaTBytes;
constexpr uint32_t kNumBars = 2 * kLoadStages + 2 * kABufs + 2 * kTmemBufs + 1;
constexpr uint32_t kSmemBytes = kOffBar + kNumBars * 8 + 16 + 1024;     // + TMEM address, alignment slack

struct TcParams {
    const uint8_t *w;
    SplitA a;
    float *c;
    int64_t ldc;
    int64_t m, n, k;
    int64_t row_bytes;
    int *err;
};

// ---- tcgen05 / proxy primitives -------------------------------------------
PFNG_DEV void cp_async16(uint32_t dst, const void *src, uint32_t src_bytes) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(src_bytes) : "memory");
}
PFNG_DEV void cp_async_arrive_noinc(uint64_t *bar) {
    asm volatile("cp.async.mbarrier.arrive.noinc.shared::cta.b64 [%0];" ::"r"(smem_u32(bar)) : "memory");
}
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

// 32 consecutive TMEM columns of this warp's 32 lanes: thread t gets lane t.
// The load and its wait are one statement, so no use of the outputs can be
// scheduled before the data has arrived.
PFNG_DEV void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
        "%15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];\n\t"
        "tcgen05.wait::ld.sync.aligned;"
        : PFNG_R32(r)
        : "r"(taddr)
        : "memory");
}
#undef PFNG_R32

// Shared-memory matrix descriptor, K-major operand with the 128-byte swizzle:
// rows of 128 bytes, 8-row atoms of 1024 bytes stored back to back (stride
// byte offset 1024), the 16-byte chunk j of row r stored at chunk j ^ (r % 8).
// `saddr` is the operand's first byte for this MMA (atom base + k offset).
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

// Byte offset of (row, 16-byte chunk c in 0..15 of the 256-byte k-step) in an
// operand tile of `rows` rows: column block c / 8, swizzled chunk within it.
PFNG_DEV uint32_t op_off(uint32_t rows, uint32_t row, uint32_t c) {
    return (c >> 3) * rows * 128u + (row >> 3) * 1024u + (row & 7u) * 128u + (((c & 7u) ^ (row & 7u)) << 4);
}

PFNG_DEV bool aborted(const int *abort_flag) { return *reinterpret_cast<const volatile int *>(abort_flag) != 0; }

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

__global__ void __launch_bounds__(kThreads, 1) gemm_tc_q4_0_kernel(const TcParams p) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023u) & ~uintptr_t(1023));
    uint64_t *bars = reinterpret_cast<uint64_t *>(smem + kOffBar);
    uint64_t *ld_full = bars;                              // [kLoadStages] cp.async landed (32 lane arrivals)
    uint64_t *ld_empty = ld_full + kLoadStages;            // [kLoadStages] decode warps + MMA commit (1)
    uint64_t *dec_full = ld_empty + kLoadStages;           // [kABufs] decode warps done
    uint64_t *dec_empty = dec_full + kABufs;               // [kABufs] MMA commit (1) + fold warps
    uint64_t *tm_full = dec_empty + kABufs;                // [kTmemBufs] MMA commit (1)
    uint64_t *tm_empty = tm_full + kTmemBufs;              // [kTmemBufs] fold warps
    uint64_t *mma_done = tm_empty + kTmemBufs;             // every issued MMA has completed (commit)
    uint32_t *tmem_holder = reinterpret_cast<uint32_t *>(bars + kNumBars);
    __shared__ int abort_flag;

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int64_t n0 = static_cast<int64_t>(blockIdx.x) * TM;
    const int64_t m0 = static_cast<int64_t>(blockIdx.y) * TN;
    const int ksteps = static_cast<int>(p.k / BK);

    if (tid == 0) {
        abort_flag = 0;
        for (int s = 0; s < kLoadStages; ++s) {
            mbar_init(&ld_full[s], 32);
            mbar_init(&ld_empty[s], kDecodeWarps + 1);
        }
        for (int a = 0; a < kABufs; ++a) {
            mbar_init(&dec_full[a], kDecodeWarps);
            mbar_init(&dec_empty[a], 1 + kFoldWarps);
        }
        for (int b = 0; b < kTmemBufs; ++b) {
            mbar_init(&tm_full[b], 1);
            mbar_init(&tm_empty[b], kFoldWarps);
        }
        mbar_init(mma_done, 1);
        fence_mbar_init();
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

    if (warp == 0) {
        // ---------------- loads ----------------
        for (int ks = 0; ks < ksteps; ++ks) {
            const int s = ks % kLoadStages;
            if (ks >= kLoadStages &&
                !wait_bar(&ld_empty[s], ((ks / kLoadStages) - 1) & 1, &abort_flag, p.err, kErrWaitEmpty)) {
                abort_flag = 1;
                break;
            }
            // raw weights: 128 rows x 144 bytes (9 chunks)
            const uint32_t raw = s_base + kOffRaw + s * kRawBytes;
            for (int q = lane; q < TM * 9; q += 32) {
                const int row = q / 9, ch = q % 9;
                const int64_t n = n0 + row;
                const bool ok = n < p.n;
                const uint8_t *src = p.w + (ok ? n * p.row_bytes + static_cast<int64_t>(ks) * 144 + ch * 16 : 0);
                cp_async16(raw + row * kRawSlot + ch * 16, src, ok ? 16u : 0u);
            }
            // activation int8 rows, swizzled operand layout
            const uint32_t bop = s_base + kOffB + s * kBOpBytes;
            for (int q = lane; q < TN * 16; q += 32) {
                const int row = q >> 4, ch = q & 15;
                const int8_t *src = p.a.qs + (m0 + row) * p.k + static_cast<int64_t>(ks) * BK + ch * 16;
                cp_async16(bop + op_off(TN, row, ch), src, 16u);
            }
            // activation scales: 64 rows x 8 floats
            const uint32_t dar = s_base + kOffDaRaw + s * kDaRawBytes;
            for (int q = lane; q < TN * 2; q += 32) {
                const int row = q >> 1, h = q & 1;
                const float *src = p.a.d + (m0 + row) * (p.k / 32) + ks * 8 + h * 4;
                cp_async16(dar + row * 32 + h * 16, src, 16u);
            }
            cp_async_arrive_noinc(&ld_full[s]);
        }
        asm volatile("cp.async.wait_all;" ::: "memory");
    } else if (warp == 1) {
        // ---------------- MMA issue (one thread) ----------------
        if (lane == 0) {
            int gsb = 0;
            for (int ks = 0; ks < ksteps && !aborted(&abort_flag); ++ks) {
                const int s = ks % kLoadStages, a = ks % kABufs;
                if (!wait_bar(&ld_full[s], (ks / kLoadStages) & 1, &abort_flag, p.err, kErrWaitFull) ||
                    !wait_bar(&dec_full[a], (ks / kABufs) & 1, &abort_flag, p.err, kErrWaitFull)) {
                    abort_flag = 1;
                    break;
                }
                fence_proxy_async_smem();
                tc_fence_after();
                const uint32_t aop = s_base + kOffA + a * kAOpBytes;
                const uint32_t bop = s_base + kOffB + s * kBOpBytes;
                bool ok = true;
                for (int sb = 0; sb < 8; ++sb, ++gsb) {
                    const int buf = gsb % kTmemBufs;
                    if (!wait_bar(&tm_empty[buf], (gsb / kTmemBufs) & 1, &abort_flag, p.err, kErrWaitEmpty)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t koff = (sb & 3) * 32u;  // k offset inside the 128-byte swizzled row
                    const uint64_t da = sw128_desc(aop + (sb >> 2) * (TM * 128u) + koff);
                    const uint64_t db = sw128_desc(bop + (sb >> 2) * (TN * 128u) + koff);
                    umma_i8(tmem_base + static_cast<uint32_t>(buf * TN), da, db, kIdesc, 0u);
                    umma_commit(&tm_full[buf]);
                }
                if (!ok) {
                    abort_flag = 1;
                    break;
                }
                umma_commit(&dec_empty[a]);
                umma_commit(&ld_empty[s]);
            }
            // TMEM is freed at the end: wait until no MMA is in flight
            umma_commit(mma_done);
            if (!mbar_wait(mma_done, 0, p.err, kErrWaitFull)) abort_flag = 1;
        }
        __syncwarp();
    } else if (warp == 2 || warp == 3) {
        // ---------------- decode: 8 threads per weight row, one block each ----------------
        const int dt = (warp - 2) * 32 + lane;  // 0..63
        for (int ks = 0; ks < ksteps; ++ks) {
            const int s = ks % kLoadStages, a = ks % kABufs;
            if (!wait_bar(&ld_full[s], (ks / kLoadStages) & 1, &abort_flag, p.err, kErrWaitFull) ||
                (ks >= kABufs &&
                 !wait_bar(&dec_empty[a], ((ks / kABufs) - 1) & 1, &abort_flag, p.err, kErrWaitEmpty))) {
                abort_flag = 1;
                break;
            }
            const uint8_t *raw = smem + kOffRaw + s * kRawBytes;
            uint8_t *aop = smem + kOffA + a * kAOpBytes;
            float *sw = reinterpret_cast<float *>(smem + kOffSw + a * kSwBytes);
#pragma unroll 2
            for (int i = 0; i < (TM * 8) / (kDecodeWarps * 32); ++i) {
                const int task = dt + i * kDecodeWarps * 32;  // (row, block)
                const int row = task >> 3, u = task & 7;
                uint32_t q[4], dbits;
                load_q4_0_block_smem(raw, row * kRawSlot + 18u * u, q, dbits);
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
                *reinterpret_cast<uint4 *>(aop + op_off(TM, row, swap ? 2 * u + 1 : 2 * u)) = swap ? hi : lo;
                *reinterpret_cast<uint4 *>(aop + op_off(TM, row, swap ? 2 * u : 2 * u + 1)) = swap ? lo : hi;
                sw[row * 8 + u] = f16_bits_to_f32(dbits);
            }
            // activation scales, transposed to [sub-block][row]
            const float *dar = reinterpret_cast<const float *>(smem + kOffDaRaw + s * kDaRawBytes);
            float *dat = reinterpret_cast<float *>(smem + kOffDaT + a * kDaTBytes);
#pragma unroll
            for (int i = 0; i < (TN * 8) / (kDecodeWarps * 32); ++i) {
                const int e = dt + i * kDecodeWarps * 32;  // e = sb * TN + activation row
                dat[e] = dar[(e % TN) * 8 + e / TN];
            }
            fence_proxy_async_smem();
            __syncwarp();
            if (lane == 0) {
                mbar_arrive(&dec_full[a]);
                mbar_arrive(&ld_empty[s]);
            }
        }
    } else {
        // ---------------- fold (warps 4..11) ----------------
        const int qtr = warp & 3;                // TMEM lane quarter of this warp
        const int half = (warp - 4) >> 2;        // activation rows 32 * half .. + 31
        const int row = qtr * 32 + lane;         // weight row of this thread in the tile
        const uint32_t my_cols = tmem_base + (static_cast<uint32_t>(qtr * 32) << 16) + half * 32;
        // every TMEM buffer starts free
        if (lane == 0)
            for (int b = 0; b < kTmemBufs; ++b) mbar_arrive(&tm_empty[b]);

        float2 acc[16];
#pragma unroll
        for (int j = 0; j < 16; ++j) acc[j] = make_float2(0.0f, 0.0f);
        int gsb = 0;
        bool ok = true;
        for (int ks = 0; ks < ksteps && ok; ++ks) {
            const int a = ks % kABufs;
            if (!wait_bar(&dec_full[a], (ks / kABufs) & 1, &abort_flag, p.err, kErrWaitFull)) {
                ok = false;
                break;
            }
            const float4 *swr = reinterpret_cast<const float4 *>(smem + kOffSw + a * kSwBytes) + row * 2;
            const float4 s0 = swr[0], s1 = swr[1];
            const float sv[8] = {s0.x, s0.y, s0.z, s0.w, s1.x, s1.y, s1.z, s1.w};
            const float *dat = reinterpret_cast<const float *>(smem + kOffDaT + a * kDaTBytes) + half * 32;
#pragma unroll
            for (int sb = 0; sb < 8; ++sb) {
                const int buf = (gsb + sb) % kTmemBufs;
                if (!ok || !wait_bar(&tm_full[buf], ((gsb + sb) / kTmemBufs) & 1, &abort_flag, p.err, kErrWaitFull)) {
                    ok = false;
                    continue;
                }
                tc_fence_after();
                uint32_t r[32];
                tmem_ld32(my_cols + buf * TN, r);
                // the partials are in registers: hand the buffer back to the MMA
                // issuer before the arithmetic
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(&tm_empty[buf]);
                const float2 ss = make_float2(sv[sb], sv[sb]);
                const float2 cm = make_float2(-kMagic * sv[sb], -kMagic * sv[sb]);
                const float4 *dap = reinterpret_cast<const float4 *>(dat + sb * TN);
#pragma unroll
                for (int j = 0; j < 8; ++j) {
                    const float4 d4 = dap[j];  // activation scales of columns 4j .. 4j + 3
                    // P + 0x4B400000 as an integer is the float 2^23 + 2^22 + P
                    const float2 y0 = make_float2(__uint_as_float(r[4 * j] + kMagicBits),
                                                  __uint_as_float(r[4 * j + 1] + kMagicBits));
                    const float2 y1 = make_float2(__uint_as_float(r[4 * j + 2] + kMagicBits),
                                                  __uint_as_float(r[4 * j + 3] + kMagicBits));
                    const float2 t0 = __ffma2_rn(y0, ss, cm), t1 = __ffma2_rn(y1, ss, cm);
                    acc[2 * j] = __ffma2_rn(t0, make_float2(d4.x, d4.y), acc[2 * j]);
                    acc[2 * j + 1] = __ffma2_rn(t1, make_float2(d4.z, d4.w), acc[2 * j + 1]);
                }
            }
            gsb += 8;
            if (!ok) break;
            __syncwarp();
            if (lane == 0) mbar_arrive(&dec_empty[a]);
        }
        if (!ok) abort_flag = 1;
        // epilogue: this thread's weight row n, activation rows m0 + 32 half + 0..31
        const int64_t n = n0 + row;
        if (ok && n < p.n) {
#pragma unroll
            for (int j = 0; j < 16; ++j) {
                const int64_t m = m0 + half * 32 + 2 * j;
                if (m < p.m) p.c[m * p.ldc + n] = acc[j].x;
                if (m + 1 < p.m) p.c[(m + 1) * p.ldc + n] = acc[j].y;
            }
        }
    }

    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem_base, kTmemCols);
    }
}

}  // namespace

bool gemm_tc_supported(int wtype, int64_t m, int64_t n, int64_t k, const void *w) {
    (void)m;
    (void)n;
    return wtype == 0 && k > 0 && k % BK == 0 && (reinterpret_cast<uintptr_t>(w) & 15u) == 0 &&
           kSmemBytes <= device_smem_optin();
}

cudaError_t launch_gemm_tc(const GemmArgs &args, int *err, cudaStream_t s) {
    TcParams p{};
    p.w = static_cast<const uint8_t *>(args.w);
    p.a = args.a;
    p.c = args.c;
    p.ldc = args.ldc;
    p.m = args.m;
    p.n = args.n;
    p.k = args.k;
    p.row_bytes = args.k / 32 * kQ4_0Bytes;
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
    const dim3 grid(static_cast<unsigned>((args.n + TM - 1) / TM), static_cast<unsigned>((args.m + TN - 1) / TN));
    gemm_tc_q4_0_kernel<<<grid, kThreads, kSmemBytes, s>>>(p);
    return cudaGetLastError();
}

}  // namespace pfng
