/*
 * pfng_b200.h -- C ABI of the B200 (sm_100a) block-quantized matmul library.
 *
 * The library computes perf-framework-ng's hot path on the GPU:
 *     C[m][n] = A_act[m][k] . W[n][k]^T
 * for the weight/activation pairs q4_0 x q8_0, q4_K x q8_K and
 * iq2_xxs x q8_K, plus the fp32 -> q8_0 / q8_K activation quantizers that
 * feed it and the fp32 -> q4_0 / q4_K weight quantizers that produce W.
 *
 * All buffers are DEVICE pointers in the unmodified ggml block layouts of the
 * reference (include/ggml.h:125-159):
 *     block_q4_0    18 B per 32 values    block_q8_0  34 B per 32 values
 *     block_q4_K   144 B per 256 values   block_q8_K 292 B per 256 values
 *     block_iq2_xxs 66 B per 256 values
 * W is [n][k / block_k] blocks, A is [m][k / block_k] blocks, C is fp32
 * row-major with row stride ldc (floats).  Every call is asynchronous on
 * `stream` (a cudaStream_t, 0 for the legacy default stream).
 *
 * Results: quantizer bytes and integer per-block partial dot products are
 * bit-identical to the reference's scalar path; fp32 outputs agree with it to
 * |C - C_ref| <= 1e-5 * sum_k |w_k * a_k| per element (summation order
 * differs).
 *
 * Return value: PFNG_B200_OK (0) or a negative status.  Argument checks run
 * on the host before any CUDA call, so a rejected call touches no device
 * state.  m == 0 or n == 0 is a valid no-op.
 */
#ifndef PFNG_B200_H
#define PFNG_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- status codes ------------------------------------------------------ */
#define PFNG_B200_OK 0
#define PFNG_B200_ERR_INVALID_ARGUMENT (-1) /* null pointer with non-zero size, negative size */
#define PFNG_B200_ERR_SHAPE (-2)            /* k not a multiple of the block size, ldc < n / ldx < k */
#define PFNG_B200_ERR_ALIGNMENT (-3)        /* pointer not aligned to its element or block type */
#define PFNG_B200_ERR_WORKSPACE (-4)        /* workspace missing or smaller than *_workspace_size() */
#define PFNG_B200_ERR_DEVICE (-5)           /* current device is not compute capability 10.0 */
#define PFNG_B200_ERR_KERNEL_TIMEOUT (-6)   /* a bounded wait inside a kernel gave up */
#define PFNG_B200_ERR_UNSUPPORTED (-7)      /* forced kernel path cannot run this shape */
#define PFNG_B200_ERR_CUDA_BASE (-1000)     /* -1000 - cudaError_t of a failed CUDA call */

/* ---- kernel path selection (the `path` argument) ------------------------ */
#define PFNG_B200_PATH_AUTO 0 /* choose by shape: GEMV for small m, tensor-core GEMM otherwise */
#define PFNG_B200_PATH_GEMV 1 /* small-m HBM-streaming kernel (dp4a); m <= 8 */
#define PFNG_B200_PATH_MMA 2  /* int8 tensor-core GEMM */
#define PFNG_B200_PATH_SIMPLE 3 /* one-thread-per-output kernel for any k; correctness fallback */

/* Weight types, in the order of the reference's QuantizationType
 * (bench/framework/kernel_registry.h:37-42). */
#define PFNG_B200_Q4_0 0
#define PFNG_B200_Q4_K 1
#define PFNG_B200_IQ2_XXS 2
/* q4_0 weights in the planar row layout (see pfng_b200_pack_q4_0_planar);
 * activations q8_0 as for PFNG_B200_Q4_0.  Accepted wherever a weight type
 * code is taken (workspace queries, pfng_b200_compute_grouped). */
#define PFNG_B200_Q4_0_PLANAR 3

/* Library version, and a readable name for a status code. */
int pfng_b200_version(void);
const char *pfng_b200_status_string(int status);

/* Reads and clears the kernel error flag after synchronizing `stream`.
 * Returns PFNG_B200_ERR_KERNEL_TIMEOUT if any kernel of this library gave up
 * a bounded wait since the last call, else PFNG_B200_OK (or a CUDA error). */
int pfng_b200_check_kernel_error(void *stream);

/* Self-test of the failure path above, for tests and health checks: one
 * small kernel in which a producer warp arrives on an mbarrier (or, with
 * skip_arrive != 0, does not) and a consumer warp waits for it through the
 * same bounded wait every pipelined kernel of the library uses, limited to
 * `attempts` tries of at most ~1 us each.  A wait that runs out records the
 * error that pfng_b200_check_kernel_error then returns
 * (PFNG_B200_ERR_KERNEL_TIMEOUT) and the kernel returns normally, so the
 * context stays usable.  completed: optional device int, set to 1 if the wait
 * succeeded and 0 if it gave up.  Asynchronous on `stream`.  The reference
 * has no device code and no counterpart; its failure convention is the
 * fail-closed registration of bench/framework/kernel_registry.cpp:13-17. */
int pfng_b200_selftest_wait(unsigned attempts, int skip_arrive, int *completed, void *stream);

/* ---- activation quantizers ---------------------------------------------
 * x: fp32 [m][ldx] (ldx >= k); y: blocks [m][k / 32] or [m][k / 256].
 * Replace llama_reference::quantize_row_q8_0 (llama_reference.cpp:38-52) and
 * quantize_row_q8_K (llama_reference.cpp:54-70), applied row by row. */
int pfng_b200_quantize_q8_0(const float *x, int64_t ldx, void *y, int64_t m, int64_t k, void *stream);
int pfng_b200_quantize_q8_K(const float *x, int64_t ldx, void *y, int64_t m, int64_t k, void *stream);

/* ---- weight quantizers (producers of W) ---------------------------------
 * Replace llama_reference::quantize_row_q4_0 (llama_reference.cpp:13-36) and
 * quantize_row_q4_K (llama_reference.cpp:72-111), which the reference runs on
 * the host in create_q4_0_input / create_q4_K_input
 * (bench/framework/benchmark.cpp:34-66). */
int pfng_b200_quantize_q4_0(const float *x, int64_t ldx, void *y, int64_t n, int64_t k, void *stream);
int pfng_b200_quantize_q4_K(const float *x, int64_t ldx, void *y, int64_t n, int64_t k, void *stream);

/* ---- matmul on quantized activations ------------------------------------
 * C = A . W^T with A already quantized (q8_0 for q4_0, q8_K otherwise).
 * Replace the per-element dot loops of compute_q4_0 / compute_q4_K /
 * compute_iq2_xxs (llama_reference.cpp:172-175, :186-189, :200-203) and the
 * KernelCallbacks::run of a reference adapter
 * (bench/framework/kernel_registry.h:97).
 * workspace: device scratch of at least pfng_b200_mm_workspace_size() bytes,
 * 256-byte aligned (may be NULL when that size is 0).  On the tensor-core
 * path it holds the activations in the GEMM's operand layout and, for shapes
 * whose tiles would leave SMs idle (small m), the fp32 tiles of a split-k
 * product, added in a fixed order (deterministic).  Results are identical
 * for identical arguments; a split product sums in a different order than
 * the unsplit one, within the same error bound. */
size_t pfng_b200_mm_workspace_size(int wtype, int64_t m, int64_t n, int64_t k, int path);
int pfng_b200_mm_q4_0_q8_0(const void *w, const void *a, float *c, int64_t m, int64_t n, int64_t k, int64_t ldc,
                           void *workspace, size_t workspace_bytes, int path, void *stream);
int pfng_b200_mm_q4_K_q8_K(const void *w, const void *a, float *c, int64_t m, int64_t n, int64_t k, int64_t ldc,
                           void *workspace, size_t workspace_bytes, int path, void *stream);
int pfng_b200_mm_iq2_xxs_q8_K(const void *w, const void *a, float *c, int64_t m, int64_t n, int64_t k,
                              int64_t ldc, void *workspace, size_t workspace_bytes, int path, void *stream);

/* ---- matmul on fp32 activations (quantize + matmul) ----------------------
 * The reference's full compute(type, input) (llama_reference.cpp:213): the
 * activations x [m][ldx] are quantized exactly as the quantizers above do,
 * then multiplied.  For small m the quantization is fused into the matmul
 * kernel (one launch); otherwise it goes through the workspace. */
size_t pfng_b200_compute_workspace_size(int wtype, int64_t m, int64_t n, int64_t k, int path);
int pfng_b200_compute_q4_0(const void *w, const float *x, int64_t ldx, float *c, int64_t m, int64_t n, int64_t k,
                           int64_t ldc, void *workspace, size_t workspace_bytes, int path, void *stream);
int pfng_b200_compute_q4_K(const void *w, const float *x, int64_t ldx, float *c, int64_t m, int64_t n, int64_t k,
                           int64_t ldc, void *workspace, size_t workspace_bytes, int path, void *stream);
int pfng_b200_compute_iq2_xxs(const void *w, const float *x, int64_t ldx, float *c, int64_t m, int64_t n,
                              int64_t k, int64_t ldc, void *workspace, size_t workspace_bytes, int path,
                              void *stream);

/* ---- prefill: activations quantized once, multiplied by several matrices ---
 * The projections that read the same layer input (Q/K/V, gate/up) quantize
 * it once: pfng_b200_prepare_activations quantizes x [m][ldx] (q8_0 for
 * q4_0 weights, q8_K otherwise, with the quantizers above -- the same bytes)
 * into the tensor-core GEMM's operand layout in `prepared` (256-byte
 * aligned, at least pfng_b200_prepared_bytes(wtype, m, k) bytes, 0 for
 * unsupported arguments); pfng_b200_mm_prepared then runs only the GEMM on
 * it, as often as needed, for any weight matrix of that type with the same
 * k.  Needs k % 256 == 0 and 16-byte aligned W (PFNG_B200_ERR_SHAPE /
 * PFNG_B200_ERR_UNSUPPORTED otherwise).  workspace (optional, at least
 * pfng_b200_mm_prepared_workspace_size bytes; 0 = none needed) holds the
 * split-k tiles of small-m shapes; with it C is bit-identical to
 * pfng_b200_compute_* with PFNG_B200_PATH_MMA, without it those shapes run
 * unsplit (same error bound, other summation order).
 * The reference quantizes the activations inside every compute() call
 * (llama_reference.cpp:213); this hoists that step out of a group of calls. */
size_t pfng_b200_prepared_bytes(int wtype, int64_t m, int64_t k);
int pfng_b200_prepare_activations(int wtype, const float *x, int64_t ldx, void *prepared, size_t prepared_bytes,
                                  int64_t m, int64_t k, void *stream);
size_t pfng_b200_mm_prepared_workspace_size(int wtype, int64_t m, int64_t n, int64_t k);
int pfng_b200_mm_prepared(int wtype, const void *w, const void *prepared, float *c, int64_t m, int64_t n, int64_t k,
                          int64_t ldc, void *workspace, size_t workspace_bytes, void *stream);

/* ---- decode: several weight matrices sharing one activation --------------
 * The projections that read the same layer input (Q/K/V, or gate/up) in ONE
 * launch: the fp32 activations x [m][ldx] are quantized once per CTA (q8_0
 * for q4_0, q8_K otherwise) and the weight rows of all `count` matrices are
 * streamed as one sequence, so the per-launch start-up is paid once.  Matrix
 * g has n[g] rows (all share k) and writes C_g [m][ldc[g]].  w, n, c and ldc
 * are HOST arrays of `count` entries holding device pointers / sizes.
 * Needs m <= 8, count <= 8 and 16-byte aligned weights (the GEMV path),
 * otherwise returns PFNG_B200_ERR_UNSUPPORTED.  Every C_g is bit-identical
 * to pfng_b200_compute_*(w[g], ..., PFNG_B200_PATH_GEMV).
 * flags: 0, or PFNG_B200_OVERLAP_WEIGHTS -- a promise that no kernel still
 * running before this call on `stream` writes the weights.  The launch may
 * then start (programmatic dependent launch) and stream the weights while
 * the preceding kernel finishes; reading x and writing C stay ordered after
 * it.  Back-to-back decode launches then form one continuous weight stream.
 * The reference has no counterpart: it multiplies one matrix per call
 * (llama_reference.cpp:213); this batches those calls. */
#define PFNG_B200_OVERLAP_WEIGHTS 1u
int pfng_b200_compute_grouped(int wtype, int count, const void *const *w, const int64_t *n, float *const *c,
                              const int64_t *ldc, const float *x, int64_t ldx, int64_t m, int64_t k, unsigned flags,
                              void *stream);

/* ---- output formats: the result written by the matmul's epilogue ----------
 * pfng_b200_mm_out / pfng_b200_compute_out are pfng_b200_mm_* /
 * pfng_b200_compute_* (any weight type code, same paths and checks) whose
 * result is written in `out_format`:
 *   PFNG_B200_OUT_F32   fp32, row stride ldo floats (the plain entry points)
 *   PFNG_B200_OUT_F16   fp16, round to nearest even, row stride ldo halves
 *   PFNG_B200_OUT_BF16  bf16, round to nearest even, row stride ldo
 *   PFNG_B200_OUT_Q8_0  C quantized along n into block_q8_0 -- the
 *                       activation operand of a next layer with q4_0 weights
 *                       -- row stride ldo blocks; requires n % 32 == 0
 * Every format is the conversion of the fp32 C the same path computes: the
 * q8_0 bytes equal pfng_b200_quantize_q8_0 applied to that C (the reference's
 * quantize_row_q8_0, llama_reference.cpp:38-52).  On the tensor-core path the
 * conversion is fused into the GEMM's epilogue (no fp32 C is written); the
 * GEMV and SIMPLE paths write fp32 C to the workspace and convert it in a
 * second launch (for decode, keep fp32 C and let the next layer's fused
 * quantizer read it).  out is 2-byte aligned.  Workspace sizes:
 * pfng_b200_mm_out_workspace_size / pfng_b200_compute_out_workspace_size.
 * No reference counterpart (the reference's consumer is its fp32 export,
 * bench/framework/kernel_registry.h:99). */
#define PFNG_B200_OUT_F32 0
#define PFNG_B200_OUT_F16 1
#define PFNG_B200_OUT_BF16 2
#define PFNG_B200_OUT_Q8_0 3
size_t pfng_b200_mm_out_workspace_size(int wtype, int out_format, int64_t m, int64_t n, int64_t k, int path);
size_t pfng_b200_compute_out_workspace_size(int wtype, int out_format, int64_t m, int64_t n, int64_t k, int path);
int pfng_b200_mm_out(int wtype, const void *w, const void *a, void *out, int out_format, int64_t ldo, int64_t m,
                     int64_t n, int64_t k, void *workspace, size_t workspace_bytes, int path, void *stream);
int pfng_b200_compute_out(int wtype, const void *w, const float *x, int64_t ldx, void *out, int out_format,
                          int64_t ldo, int64_t m, int64_t n, int64_t k, void *workspace, size_t workspace_bytes,
                          int path, void *stream);

/* ---- q4_0 in the planar row layout ---------------------------------------
 * A weight row of nb = k / 32 blocks holds the 16-byte nibble fields of
 * blocks 0..nb-1 (block j at byte 16 j), then their fp16 scales (block j at
 * byte 16 nb + 2 j): the same 18 nb bytes and row stride as block_q4_0,
 * reordered so that the kernels read every nibble field with one aligned
 * 16-byte load.  Requires k % 256 == 0 and a 16-byte aligned planar buffer
 * (PFNG_B200_ERR_SHAPE / PFNG_B200_ERR_ALIGNMENT otherwise); source and
 * destination must not overlap.  unpack(pack(W)) == W byte for byte.
 * The reference's adapters repack W once in KernelCallbacks::prepare
 * (kernels/common/types.h:9-63;
 * kernels/q4_0-q8_0-IME-m8b/implementations/smt-ime2/adapter.cpp:95-112);
 * this is that step for these kernels, run on the device.
 * The *_q4_0p entry points take planar W and behave as their q4_0
 * counterparts (same arguments, paths, workspace sizes and checks): integer
 * partials bit-identical, fp32 outputs within the same bound. */
int pfng_b200_pack_q4_0_planar(const void *w, void *w_planar, int64_t n, int64_t k, void *stream);
int pfng_b200_unpack_q4_0_planar(const void *w_planar, void *w, int64_t n, int64_t k, void *stream);
int pfng_b200_mm_q4_0p_q8_0(const void *w_planar, const void *a, float *c, int64_t m, int64_t n, int64_t k,
                            int64_t ldc, void *workspace, size_t workspace_bytes, int path, void *stream);
int pfng_b200_compute_q4_0p(const void *w_planar, const float *x, int64_t ldx, float *c, int64_t m, int64_t n,
                            int64_t k, int64_t ldc, void *workspace, size_t workspace_bytes, int path, void *stream);
int pfng_b200_partials_q4_0p_q8_0(const void *w_planar, const void *a, int32_t *out, int64_t m, int64_t n, int64_t k,
                                  void *workspace, size_t workspace_bytes, int path, void *stream);

/* ---- integer partials (verification) ------------------------------------
 * out: int32 [m][n][k / 32], the integer dot product of every 32-value
 * sub-block, produced by the same kernel path as the matmul (`path`) before
 * any scale is applied:
 *   q4_0:    sum (nibble - 8) * a          (llama_reference.cpp:138-142)
 *   q4_K:    sum nibble * a per sub-block  (the q term of :125-130)
 *   iq2_xxs: sum grid_value * a, unscaled  (:155-157)
 * Uses the same workspace size as the matmul. */
int pfng_b200_partials_q4_0_q8_0(const void *w, const void *a, int32_t *out, int64_t m, int64_t n, int64_t k,
                                 void *workspace, size_t workspace_bytes, int path, void *stream);
int pfng_b200_partials_q4_K_q8_K(const void *w, const void *a, int32_t *out, int64_t m, int64_t n, int64_t k,
                                 void *workspace, size_t workspace_bytes, int path, void *stream);
int pfng_b200_partials_iq2_xxs_q8_K(const void *w, const void *a, int32_t *out, int64_t m, int64_t n, int64_t k,
                                    void *workspace, size_t workspace_bytes, int path, void *stream);

/* ---- multi-GPU helpers (N-sharded weights) -------------------------------
 * Rank r of `world` owns weight rows [*begin, *end): the rows are split in
 * multiples of `granule` (a kernel tile), the last rank taking the ragged
 * remainder.  Pure host arithmetic. */
int pfng_b200_shard_rows(int64_t n, int world, int rank, int64_t granule, int64_t *begin, int64_t *end);
/* Reassemble C [m][ldc] from the all-gathered per-rank slices
 * `slices` = [world][m][slice_width] (rank r's slice holds its rows'
 * columns, width end_r - begin_r, zero-padded to slice_width). */
int pfng_b200_unshard_columns(const float *slices, float *c, int64_t m, int64_t n, int64_t ldc, int world,
                              int64_t granule, int64_t slice_width, void *stream);

/* ---- fused output all-gather over peer memory -----------------------------
 * pfng_b200_compute_* (fp32 activations, fp32 C) writing the same C [m][n]
 * to `ndst` destinations at once, each with row stride `ldd` floats.  With
 * weight rows sharded over the GPUs of a node, rank r passes the column
 * offset begin_r (pfng_b200_shard_rows) into every rank's full C -- its own
 * and the others', mapped with pfng_b200_ipc_open -- so that the matmul
 * itself stores C into every rank's C over NVLink: the all-gather of C done
 * by the call, with no collective and no reassembly pass.
 *   - On the MMA path the GEMM writes dst[0] and a copy kernel after it
 *     pushes C to the other destinations in 16-byte pieces over NVLink
 *     (PFNG_B200_COPIES=epilogue: the GEMM's epilogue writes every
 *     destination itself; measured slower), each followed by a system-scope
 *     fence; the GEMV and SIMPLE paths compute into dst[0] and copy it to
 *     the others on the stream.
 *   - The call does not wait for the other ranks.  Before a rank reads its C
 *     (or a next call writes into the others'), every rank's call must have
 *     completed: order the ranks with a barrier or collective on the stream
 *     (e.g. a one-element NCCL all-reduce) after the call.
 *   - workspace: pfng_b200_compute_workspace_size for (wtype, m, n, k, path).
 * No counterpart in the reference (a single-device library); C equals
 * pfng_b200_compute_* of the same arguments bit for bit. */
#define PFNG_B200_MAX_DESTINATIONS 8
int pfng_b200_compute_gather(int wtype, const void *w, const float *x, int64_t ldx, float *const *dst, int ndst,
                             int64_t ldd, int64_t m, int64_t n, int64_t k, void *workspace, size_t workspace_bytes,
                             int path, void *stream);
/* The same with activations already quantized (q8_0 / q8_K bytes, as
 * pfng_b200_mm_*; workspace: pfng_b200_mm_workspace_size) -- e.g. broadcast
 * to the ranks as q8_0, 1.06 bytes per value instead of fp32's 4. */
int pfng_b200_mm_gather(int wtype, const void *w, const void *a, float *const *dst, int ndst, int64_t ldd, int64_t m,
                        int64_t n, int64_t k, void *workspace, size_t workspace_bytes, int path, void *stream);

/* Device buffers shared between the processes of a node (CUDA IPC): alloc
 * returns a cudaMalloc'd buffer of the current device and its 64-byte
 * handle; another process opens the handle to a device pointer to the same
 * memory (peer access over NVLink), closes it when done, and the owner frees
 * the buffer after every opener has closed it. */
#define PFNG_B200_IPC_HANDLE_BYTES 64
int pfng_b200_ipc_alloc(size_t bytes, void **ptr, void *handle);
int pfng_b200_ipc_free(void *ptr);
int pfng_b200_ipc_open(const void *handle, void **ptr);
int pfng_b200_ipc_close(void *ptr);

/* ---- matmul without any allocation ----------------------------------------
 * pfng_b200_compute_q4_0 on the tensor-core path (fp32 activations x [m][ldx]
 * quantized to q8_0, then C = A . W^T), for callers that must not allocate
 * device memory on this call path -- e.g. a server whose memory pool owns the
 * whole GPU from start-up, or a loop that cannot take the device-wide
 * synchronisation of cudaMalloc / cudaFree.  It takes no workspace: its
 * scratch (the quantized activations and, for the small-m shapes whose k is
 * split across CTAs, the split products' fp32 tiles) is a fixed array of
 * PFNG_B200_NOALLOC_SCRATCH_BYTES inside the library, held by every GPU that
 * loads the library until the process exits.
 *   - Problems whose scratch would exceed that size (about m * k * 1.25
 *     bytes, m rounded up to 128, plus splits * m * n * 4 bytes when k is
 *     split; e.g. m <= 2048 at k = 4096) return PFNG_B200_ERR_WORKSPACE; k
 *     must be a multiple of 256 and w 16-byte aligned (else
 *     PFNG_B200_ERR_UNSUPPORTED).
 *   - The first call on each device looks up the array's device address
 *     (cudaGetSymbolAddress); make that first call before any stream capture.
 *     The address is cached for the process: do not use the library after a
 *     cudaDeviceReset.
 *   - All calls on a device share the array, which keeps the last call's
 *     contents; each call rewrites everything it reads, but calls whose
 *     kernels overlap on the GPU (other streams, other host threads) race on
 *     it and must be ordered by the caller.
 * No counterpart in the reference.  It makes the kernel choices of
 * pfng_b200_compute_q4_0 with PFNG_B200_PATH_MMA (split-k factor included),
 * so C is bit-identical to that call's. */
#define PFNG_B200_NOALLOC_SCRATCH_BYTES ((size_t)16 << 20)
int pfng_b200_compute_q4_0_noalloc(const void *w, const float *x, int64_t ldx, float *c, int64_t m, int64_t n,
                                   int64_t k, int64_t ldc, void *stream);

#ifdef __cplusplus
}
#endif

#endif
