// shard.cu -- reassembly of N-sharded output columns after an all-gather.
//
// With weight rows split across ranks by pfng_b200_shard_rows (granules of
// `granule` rows, the first (granules % world) ranks one granule more), rank
// r computes C[:, begin_r:end_r] into a [m][slice_width] slice; an
// all-gather stacks the slices as [world][m][slice_width].  This kernel writes
// them back into the row-major C[m][ldc].
#include "pfng_common.cuh"
#include "pfng_internal.h"

namespace pfng {
namespace {

__global__ void unshard_kernel(const float *__restrict__ slices, float *__restrict__ c, int64_t m, int64_t n,
                               int64_t ldc, int world, int64_t granule, int64_t slice_width) {
    const int64_t granules = (n + granule - 1) / granule;
    const int64_t base = granules / world, extra = granules % world;
    const int64_t total = m * n;
    for (int64_t e = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; e < total;
         e += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const int64_t i = e / n, j = e % n;
        const int64_t gi = j / granule;
        const int64_t big = extra * (base + 1);
        const int64_t r = gi < big ? gi / (base + 1) : extra + (gi - big) / base;
        const int64_t g0 = r * base + (r < extra ? r : extra);
        const int64_t local = j - g0 * granule;
        c[i * ldc + j] = slices[(r * m + i) * slice_width + local];
    }
}

}  // namespace

cudaError_t launch_unshard_columns(const float *slices, float *c, int64_t m, int64_t n, int64_t ldc, int world,
                                   int64_t granule, int64_t slice_width, cudaStream_t s) {
    const int64_t total = m * n;
    int64_t blocks = (total + 255) / 256;
    const int64_t cap = static_cast<int64_t>(device_sm_count()) * 16;
    if (blocks > cap) blocks = cap;
    unshard_kernel<<<static_cast<unsigned>(blocks), 256, 0, s>>>(slices, c, m, n, ldc, world, granule, slice_width);
    return cudaGetLastError();
}

}  // namespace pfng
