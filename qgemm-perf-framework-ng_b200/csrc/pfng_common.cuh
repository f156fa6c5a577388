// pfng_common.cuh -- shared device helpers for the sm_100a kernels.
//
// Block layouts are the ggml wire format (reference include/ggml.h:125-159);
// the byte offsets used by the kernels are spelled out here once.
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#define PFNG_DEV __device__ __forceinline__

namespace pfng {

// ---- wire format -----------------------------------------------------------
constexpr int kQ4_0Bytes = 18;   // fp16 d, 16 B nibbles (low nibble = i, high = i + 16)
constexpr int kQ8_0Bytes = 34;   // fp16 d, 32 x int8
constexpr int kQ8_KBytes = 292;  // fp32 d, 256 x int8, 16 x int16 bsums
constexpr int kQ4_KBytes = 144;  // fp16 d, fp16 dmin, 12 B 6-bit scales/mins, 128 B nibbles
constexpr int kIQ2Bytes = 66;    // fp16 d, 32 x uint16 (8 B per 32-value group)
// Weight type codes (the PFNG_B200_* weight types of the C ABI).  kWQ4_0P
// is q4_0 in the planar row layout: per weight row of nb blocks, the 16-byte
// nibble fields of blocks 0..nb-1 (block j at byte 16 j), then their fp16
// scales (block j at byte 16 nb + 2 j); 18 nb bytes per row, like ggml's.
constexpr int kWQ4_0 = 0, kWQ4_K = 1, kWIQ2 = 2, kWQ4_0P = 3;
constexpr int kQ8_KQsOffset = 4;
constexpr int kQ8_KBsumsOffset = 260;

// fp32 -> fp16 with round-to-nearest-even, and fp16 -> fp32.  Both equal the
// reference's bit-trick codec (ggml.h:83-117) for every non-NaN value; the
// only difference is the NaN payload, and no quantizer here can produce a
// NaN scale (amax is a maximum of magnitudes that skips NaN).
PFNG_DEV uint16_t f32_to_f16_bits(float f) { return __half_as_ushort(__float2half_rn(f)); }
PFNG_DEV float f16_bits_to_f32(uint32_t h) { return __half2float(__ushort_as_half((unsigned short)(h & 0xffffu))); }

// ---- error reporting -------------------------------------------------------
// A kernel that gives up a bounded wait records a code in the library's
// device error word (a pointer every waiting kernel receives); the host reads
// and clears it with pfng_b200_check_kernel_error().
constexpr int kErrWaitFull = 1;
constexpr int kErrWaitEmpty = 2;
constexpr int kErrWaitIssue = 3;

PFNG_DEV void report_error(int *flag, int code) {
    if (flag) atomicCAS(flag, 0, code);
}

// ---- shared-memory addressing and mbarriers ---------------------------------
PFNG_DEV uint32_t smem_u32(const void *p) { return static_cast<uint32_t>(__cvta_generic_to_shared(p)); }

PFNG_DEV void mbar_init(uint64_t *bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
PFNG_DEV void fence_mbar_init() { asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory"); }
PFNG_DEV void mbar_arrive(uint64_t *bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
PFNG_DEV void mbar_arrive_expect_tx(uint64_t *bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
                 : "memory");
}
// One bounded attempt: the hardware may suspend the thread for a while
// (at most PFNG_WAIT_HINT_NS when that is non-zero, else a system-dependent
// limit) or until the phase completes.
#ifndef PFNG_WAIT_HINT_NS
#define PFNG_WAIT_HINT_NS 1000
#endif
PFNG_DEV bool mbar_try_wait(uint64_t *bar, uint32_t parity) {
    uint32_t done;
#if PFNG_WAIT_HINT_NS > 0
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(done)
        : "r"(smem_u32(bar)), "r"(parity), "n"(PFNG_WAIT_HINT_NS)
        : "memory");
#else
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(done)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
#endif
    return done != 0;
}
// Non-blocking probe of the phase with the given parity.
PFNG_DEV bool mbar_test_wait(uint64_t *bar, uint32_t parity) {
    uint32_t done;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(done)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return done != 0;
}
// Every wait in this library is bounded: about 2^20 attempts of <= ~1 us, so
// a wait that can never complete ends in about a second with `code` recorded.
constexpr uint32_t kWaitAttempts = 1u << 20;
// The wait with an explicit attempt limit (the self-test kernel passes a
// small one); every kernel's waits use kWaitAttempts.
PFNG_DEV bool mbar_wait_n(uint64_t *bar, uint32_t parity, int *flag, int code, uint32_t attempts) {
    for (uint32_t i = 0; i < attempts; ++i)
        if (mbar_try_wait(bar, parity)) return true;
    report_error(flag, code);
    return false;
}
PFNG_DEV bool mbar_wait(uint64_t *bar, uint32_t parity, int *flag, int code) {
    return mbar_wait_n(bar, parity, flag, code, kWaitAttempts);
}

// Bulk (non-tensor) TMA copy global -> this CTA's shared memory, completing
// `bytes` of transaction count on `bar`.  dst, src and bytes must be
// multiples of 16.  The destination is this CTA's own shared memory.
PFNG_DEV void bulk_copy_g2s(void *dst, const void *src, uint32_t bytes, uint64_t *bar, uint64_t policy) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], "
        "%4;" ::"r"(smem_u32(dst)),
        "l"(src), "r"(bytes), "r"(smem_u32(bar)), "l"(policy)
        : "memory");
}
PFNG_DEV uint64_t l2_policy_evict_first() {
    uint64_t policy;
    asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(policy));
    return policy;
}

// ---- programmatic dependent launch --------------------------------------------
// pdl_trigger: kernels launched after this one with programmatic stream
// serialization may start once every CTA of this grid has executed it (or
// exited).  pdl_wait: block until the preceding grid has completed and its
// memory is visible; a no-op in a kernel launched without the attribute.
PFNG_DEV void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }
PFNG_DEV void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

// ---- small integer helpers ---------------------------------------------------
// Read the 16 payload bytes and the fp16 scale of an 18-byte q4_0 block that
// starts at byte offset `off` (even) of shared memory `base`, using aligned
// 32-bit loads only.
PFNG_DEV void load_q4_0_block_smem(const uint8_t *base, uint32_t off, uint32_t q[4], uint32_t &d) {
    const uint32_t *w = reinterpret_cast<const uint32_t *>(base + (off & ~3u));
    const uint32_t w0 = w[0], w1 = w[1], w2 = w[2], w3 = w[3], w4 = w[4];
    const uint32_t sh = (off & 2u) ? 32u : 16u;  // clamped funnel shift: 32 selects the high word
    q[0] = __funnelshift_rc(w0, w1, sh);
    q[1] = __funnelshift_rc(w1, w2, sh);
    q[2] = __funnelshift_rc(w2, w3, sh);
    q[3] = __funnelshift_rc(w3, w4, sh);
    d = ((off & 2u) ? (w0 >> 16) : w0) & 0xffffu;
}

PFNG_DEV int dp4a(int a, int b, int c) { return __dp4a(a, b, c); }

// 8-bit sign mask of a 7-bit iq2_xxs sign index: bit 7 makes the number of
// negative lanes even (kernels/common/iq2_xxs.h:25-27).
PFNG_DEV uint32_t iq2_sign_mask(uint32_t idx7) { return idx7 | ((__popc(idx7) & 1u) << 7); }
// Expand 4 mask bits to 4 byte masks (0x00 or 0xff per byte).
PFNG_DEV uint32_t expand_bits4(uint32_t bits) {
    const uint32_t spread = ((bits & 0xfu) * 0x00204081u) & 0x01010101u;
    return spread * 0xffu;
}
// Apply byte masks: negate the bytes whose mask is 0xff.  For a byte b != 0,
// (b ^ 0xff) + 1 = 256 - b stays within the byte, so one 32-bit add negates
// every masked byte without a carry into its neighbour; the iq2_xxs grid
// magnitudes (8, 25, 43) are never 0.
PFNG_DEV uint32_t apply_sign_bytes(uint32_t v, uint32_t mask) { return (v ^ mask) + (mask & 0x01010101u); }

}  // namespace pfng
