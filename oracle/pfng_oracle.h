/*
 * pfng_oracle.h -- CPU restatement of the reference's scalar ggml path.
 *
 * TEST INFRASTRUCTURE ONLY.  This library is the checker for the B200
 * kernels: only tests/, __graft_entry__.smoke() and bench.py's cpu_baseline /
 * reference legs may load it.  The product library never links it and has no
 * CPU fallback.
 *
 * Every function restates one function of perf-framework-ng's
 * bench/llama_reference/llama_reference.cpp (itself an extract of llama.cpp
 * 314e72934), in plain C, with the same floating-point operation order so
 * that results are bit-identical to the reference when compiled with
 * -ffp-contract=off.  Parity of this restatement is pinned against the
 * reference compiled from its own sources (oracle/Makefile -> oracle/_ref)
 * and against the committed fixtures in tests/golden/.
 *
 * Block layouts follow include/ggml.h:125-159 of the reference; they are the
 * wire format and are restated here so the oracle has no dependency on the
 * product headers.
 */
#ifndef PFNG_ORACLE_H
#define PFNG_ORACLE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define ORACLE_QK4_0 32
#define ORACLE_QK8_0 32
#define ORACLE_QK_K 256

typedef struct { uint16_t d; uint8_t qs[16]; } oracle_block_q4_0;              /* 18 B  */
typedef struct { uint16_t d; int8_t qs[32]; } oracle_block_q8_0;               /* 34 B  */
typedef struct { float d; int8_t qs[256]; int16_t bsums[16]; } oracle_block_q8_K; /* 292 B */
typedef struct { uint16_t d; uint16_t qs[32]; } oracle_block_iq2_xxs;          /* 66 B  */
typedef struct {
    uint16_t d;
    uint16_t dmin;
    uint8_t scales[12];
    uint8_t qs[128];
} oracle_block_q4_K;                                                            /* 144 B */

/* fp16 codec: include/ggml.h:83-117 (bit-exact; NaN -> 0x7E00 | sign). */
float oracle_fp16_to_fp32(uint16_t h);
uint16_t oracle_fp32_to_fp16(float f);

/* Quantizers: llama_reference.cpp:13-36, :38-52, :54-70, :72-111.
 * `k` is the number of fp32 values in the row (multiple of the block size). */
void oracle_quantize_row_q4_0(const float *x, oracle_block_q4_0 *y, size_t k);
void oracle_quantize_row_q8_0(const float *x, oracle_block_q8_0 *y, size_t k);
void oracle_quantize_row_q8_K(const float *x, oracle_block_q8_K *y, size_t k);
void oracle_quantize_row_q4_K(const float *x, oracle_block_q4_K *y, size_t k);

/* Row-batched quantizers (m rows of k values, row stride k). */
void oracle_quantize_q4_0(const float *x, void *y, size_t m, size_t k);
void oracle_quantize_q8_0(const float *x, void *y, size_t m, size_t k);
void oracle_quantize_q8_K(const float *x, void *y, size_t m, size_t k);
void oracle_quantize_q4_K(const float *x, void *y, size_t m, size_t k);

/* Dot products: llama_reference.cpp:134-146, :113-132, :148-161. */
float oracle_dot_q4_0_q8_0(const oracle_block_q4_0 *w, const oracle_block_q8_0 *a, size_t nblocks);
float oracle_dot_q4_K_q8_K(const oracle_block_q4_K *w, const oracle_block_q8_K *a);
float oracle_dot_iq2_xxs_q8_K(const oracle_block_iq2_xxs *w, const oracle_block_q8_K *a);

/* C[m][n] (row stride ldc) from pre-quantized activations.
 * Loop structure of compute_q4_0 / compute_q4_K / compute_iq2_xxs,
 * llama_reference.cpp:165-205, minus the activation quantization. */
void oracle_mm_q4_0_q8_0(const void *w, const void *a, float *c, size_t m, size_t n, size_t k, size_t ldc);
void oracle_mm_q4_K_q8_K(const void *w, const void *a, float *c, size_t m, size_t n, size_t k, size_t ldc);
void oracle_mm_iq2_xxs_q8_K(const void *w, const void *a, float *c, size_t m, size_t n, size_t k, size_t ldc);

/* Same with fp32 activations quantized first: the full reference compute(). */
void oracle_compute_q4_0(const void *w, const float *x, float *c, size_t m, size_t n, size_t k);
void oracle_compute_q4_K(const void *w, const float *x, float *c, size_t m, size_t n, size_t k);
void oracle_compute_iq2_xxs(const void *w, const float *x, float *c, size_t m, size_t n, size_t k);

/* Integer per-32 partial dot products, out[m][n][k/32]:
 *   q4_0:    sum_i (nibble_i - 8) * a_i                 (llama_reference.cpp:138-142)
 *   q4_K:    sum_i nibble_i * a_i for sub-block sb      (the q term of :125-130)
 *   iq2_xxs: sum_i grid_signed_i * a_i, before scale    (:155-157) */
void oracle_partials_q4_0_q8_0(const void *w, const void *a, int32_t *out, size_t m, size_t n, size_t k);
void oracle_partials_q4_K_q8_K(const void *w, const void *a, int32_t *out, size_t m, size_t n, size_t k);
void oracle_partials_iq2_xxs_q8_K(const void *w, const void *a, int32_t *out, size_t m, size_t n, size_t k);

/* Per-element error scale sum_k |w_k * a_k| (dequantized weight times
 * dequantized activation), in double, out[m][n].  The parity bar for fp32
 * outputs is |C - C_ref| <= 1e-5 * bound. */
void oracle_bound_q4_0_q8_0(const void *w, const void *a, double *out, size_t m, size_t n, size_t k);
void oracle_bound_q4_K_q8_K(const void *w, const void *a, double *out, size_t m, size_t n, size_t k);
void oracle_bound_iq2_xxs_q8_K(const void *w, const void *a, double *out, size_t m, size_t n, size_t k);

/* q4_0 planar row layout of the B200 library (no reference counterpart: a
 * byte permutation of block_q4_0 rows, the device form of the W repack the
 * reference's adapters do in prepare, kernels/common/types.h:9-63).  Row of
 * nb = k / 32 blocks: nibble fields of blocks 0..nb-1 at 16 j, then their
 * fp16 scales at 16 nb + 2 j.  Matmul parity on planar W is checked against
 * oracle_mm_q4_0_q8_0 on the ggml-layout W. */
void oracle_pack_q4_0_planar(const void *w, void *w_planar, size_t n, size_t k);
void oracle_unpack_q4_0_planar(const void *w_planar, void *w, size_t n, size_t k);

/* iq2_xxs decode of one 32-value group (kernels/common/iq2_xxs.h:29-41, with
 * the full 256-entry grid of the upstream kernel's tables.h:8-73). */
void oracle_iq2_xxs_decode_group(const uint8_t *packed8, int8_t *values32, int *scale);
uint64_t oracle_iq2_xxs_grid(unsigned index);
uint8_t oracle_iq2_xxs_sign_mask(unsigned index7);

#ifdef __cplusplus
}
#endif

#endif
