// pfng_tma.h -- 2-D tensor maps (host) and tensor-map bulk copies (device)
// shared by the GEMM kernels.  Every map describes this GPU's own memory and
// every copy lands in the issuing CTA's own shared memory.
#pragma once

#include <cuda.h>
#include <cudaTypedefs.h>

#include "pfng_common.cuh"

namespace pfng {

// cuTensorMapEncodeTiled through the runtime's driver entry point (null when
// the driver does not provide it).
PFN_cuTensorMapEncodeTiled_v12000 encode_fn();

// 2-D tiled map over a row-major array [rows][cols] of elements of `type`
// (row stride `stride` bytes), boxes of box_cols x box_rows elements; the
// box rows past `rows` read as zeros.  False if the driver rejects it.
bool encode_2d(CUtensorMap *map, CUtensorMapDataType type, const void *base, uint64_t cols, uint64_t rows,
               uint64_t stride, uint32_t box_cols, uint32_t box_rows, CUtensorMapSwizzle swizzle);

// Tiled map of `rank` dimensions (dims[0] innermost; strides[i] = bytes
// between consecutive indices of dimension i + 1), boxes of box[] elements.
bool encode_nd(CUtensorMap *map, CUtensorMapDataType type, int rank, const void *base, const uint64_t *dims,
               const uint64_t *strides, const uint32_t *box);

// Box at element (x, y) of `map` into shared memory `dst`, completing its
// bytes of transaction count on `bar`.  x times the element size must be a
// multiple of 16 bytes.
PFNG_DEV void tma_load_2d(uint32_t dst, const CUtensorMap *map, int x, int y, uint64_t *bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::
            "r"(dst),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_u32(bar))
        : "memory");
}
PFNG_DEV void tma_load_4d(uint32_t dst, const CUtensorMap *map, int c0, int c1, int c2, int c3, uint64_t *bar) {
    asm volatile(
        "cp.async.bulk.tensor.4d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4, %5}], "
        "[%6];" ::"r"(dst),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(c2), "r"(c3), "r"(smem_u32(bar))
        : "memory");
}
PFNG_DEV void prefetch_map(const CUtensorMap *map) {
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

}  // namespace pfng
