// pfng_internal.h -- host-side declarations shared by the .cu files of
// libpfng_b200 (not part of the public C ABI).
#pragma once

#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

namespace pfng {

// "Split" activation operand used by the tensor-core GEMMs: int8 values
// row-major [rows][k] (rows 16-byte aligned), one fp32 scale per block and an
// int32 per 32-value sub-block (see each producer for its meaning).  The
// layout lives in the caller's workspace and is rebuilt every call.
//
// q8_0 scales (one per 32-value block) are stored block-major: the scales
// of block b of every row form one slab of d_ld floats, and inside each
// 128-row group row 8 j + g sits at g * 16 + j (split_d_index).  A GEMM
// thread folds rows g, g + 8, g + 16, ... of a tile, so that order puts a
// thread's scales side by side (one 16-byte load for four rows), and a
// tile's rows of one block are 8 contiguous runs (16-byte copies).
// q8_K scales (one per 256 values) are row-major [rows_pad][k / 256].
struct SplitA {
    int8_t *qs;      // [rows_pad][k]
    float *d;        // q8_0: [k / 32][d_ld] as above; q8_K: [rows_pad][k / 256]
    int32_t *aux;    // [rows_pad][k / 32]
    int64_t rows_pad;
    int64_t k;
    int64_t d_ld;    // q8_0: floats between the block slabs of d (the carved rows_pad)
};

// Position of (row, 32-value block b) in a q8_0 split operand's d.
__host__ __device__ inline int64_t split_d_index(int64_t row, int64_t b, int64_t d_ld) {
    return b * d_ld + (row & ~int64_t(127)) + ((row & 7) << 4) + ((row >> 3) & 15);
}

constexpr int64_t kGemmTileM = 128;
inline int64_t round_up(int64_t v, int64_t m) { return (v + m - 1) / m * m; }
size_t split_a_bytes(int64_t m, int64_t k, int block);
SplitA split_a_carve(void *workspace, int64_t m, int64_t k, int block);

// quantize.cu
cudaError_t launch_quantize_q8_0(const float *x, int64_t ldx, void *y, int64_t m, int64_t k, cudaStream_t s);
cudaError_t launch_quantize_q8_K(const float *x, int64_t ldx, void *y, int64_t m, int64_t k, cudaStream_t s);
cudaError_t launch_quantize_q4_0(const float *x, int64_t ldx, void *y, int64_t n, int64_t k, cudaStream_t s);
cudaError_t launch_quantize_q4_K(const float *x, int64_t ldx, void *y, int64_t n, int64_t k, cudaStream_t s);
// fp32 -> split operand (q8_0: aux = 0x4B400000 - 8 * sum(q) per 32; q8_K: aux = sum(q) per 32)
cudaError_t launch_quantize_q8_0_split(const float *x, int64_t ldx, const SplitA &out, int64_t m, int64_t k,
                                       cudaStream_t s);
cudaError_t launch_quantize_q8_K_split(const float *x, int64_t ldx, const SplitA &out, int64_t m, int64_t k,
                                       cudaStream_t s);
// fp32 -> q8_0 blocks with an output row stride of ldy blocks
cudaError_t launch_quantize_q8_0_strided(const float *x, int64_t ldx, void *y, int64_t ldy, int64_t m, int64_t k,
                                         cudaStream_t s);
// fp32 C [m][ldc] -> fp16 / bf16 out [m][ldo] (round to nearest even)
cudaError_t launch_convert_out(const float *c, int64_t ldc, void *out, int64_t ldo, int format, int64_t m, int64_t n,
                               cudaStream_t s);
// raw blocks -> split operand
cudaError_t launch_convert_q8_0_split(const void *a, const SplitA &out, int64_t m, int64_t k, cudaStream_t s);
cudaError_t launch_convert_q8_K_split(const void *a, const SplitA &out, int64_t m, int64_t k, cudaStream_t s);

// gemv.cu -- small-m kernels.  `x` (fp32) or `a` (raw q8 blocks) is given.
// Up to kGemvMaxGroup weight matrices (same k) share the activations and run
// in one launch.  partials != nullptr (count == 1 only) selects the
// integer-partials output instead of C.
constexpr int kGemvMaxGroup = 8;
struct GemvArgs {
    int wtype;
    int count;
    const void *w[kGemvMaxGroup];
    float *c[kGemvMaxGroup];
    int64_t ldc[kGemvMaxGroup];
    int64_t n[kGemvMaxGroup];
    const void *a;      // raw q8_0 / q8_K blocks, or nullptr
    const float *x;     // fp32 activations, or nullptr
    int64_t ldx;
    int32_t *partials;
    int *err;
    int64_t m, k;
    bool overlap;       // programmatic dependent launch (weights not written by the previous kernel)
};
bool gemv_supported(int wtype, int64_t m, int count, const int64_t *n, int64_t k, const void *const *w);
cudaError_t launch_gemv(const GemvArgs &args, cudaStream_t s);

// Output formats of the matmul result (the PFNG_B200_OUT_* codes).
constexpr int kOutF32 = 0, kOutF16 = 1, kOutBF16 = 2, kOutQ8_0 = 3;

// gemm.cu -- tensor-core GEMM on a split activation operand.
struct GemmArgs {
    int wtype;
    const void *w;
    SplitA a;
    float *c;
    int64_t ldc;
    int32_t *partials;
    int64_t m, n, k;
    int *err = nullptr;  // library error word for bounded waits (tensor-memory kernel)
    // fused epilogue: kOutF32 writes c; other formats write out with row
    // stride ldo (elements, or q8_0 blocks along n)
    int out_format = kOutF32;
    void *out = nullptr;
    int64_t ldo = 0;
    // split-K partial tiles ([splits][m][n] fp32, gemm_partial_bytes); without
    // them the product runs unsplit
    float *partial = nullptr;
    size_t partial_bytes = 0;
    // fp32 C also stored to `ncopies` more destinations with C's layout (row
    // stride ldc), e.g. other GPUs' C mapped through CUDA IPC
    float *const *copies = nullptr;
    int ncopies = 0;
};
constexpr int kMaxCopies = 7;
bool gemm_supported(int wtype, int64_t m, int64_t n, int64_t k, const void *w);
// workspace bytes of the split-K partial tiles for this shape (0: no split)
size_t gemm_partial_bytes(int64_t m, int64_t n, int64_t k);
cudaError_t launch_gemm(const GemmArgs &args, cudaStream_t s);

// gemm_tc.cu -- q4_0 on tcgen05 / TMEM (k % 256 == 0, 16-byte aligned W)
bool gemm_tc_supported(int wtype, int64_t m, int64_t n, int64_t k, const void *w);
cudaError_t launch_gemm_tc(const GemmArgs &args, int *err, cudaStream_t s);

// simple.cu -- one thread per output element, any k multiple of the block.
struct SimpleArgs {
    int wtype;
    const void *w;
    const void *a;  // raw q8 blocks
    float *c;
    int64_t ldc;
    int32_t *partials;
    int64_t m, n, k;
};
cudaError_t launch_simple(const SimpleArgs &args, cudaStream_t s);

// planar.cu -- q4_0 between the ggml and the planar row layout (k % 256 == 0)
cudaError_t launch_pack_q4_0_planar(const void *w, void *w_planar, int64_t n, int64_t k, cudaStream_t s);
cudaError_t launch_unpack_q4_0_planar(const void *w_planar, void *w, int64_t n, int64_t k, cudaStream_t s);

// shard.cu
cudaError_t launch_unshard_columns(const float *slices, float *c, int64_t m, int64_t n, int64_t ldc, int world,
                                   int64_t granule, int64_t slice_width, cudaStream_t s);

int device_sm_count();
size_t device_smem_optin();
int *device_error_word();  // the current device's error word, nullptr if unavailable

}  // namespace pfng
