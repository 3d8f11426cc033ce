/*
 * Library baselines reported beside tcaspmm (never on its hot path), in
 * libtcaspmm_baselines.so.  Both time `iters` launches with CUDA events on
 * `stream` after `warmup` untimed launches and return the average ms.
 */
#ifndef TCASPMM_BASELINES_H
#define TCASPMM_BASELINES_H

#include "tcaspmm.h"

#ifdef __cplusplus
extern "C" {
#endif

/* Flush L2 between timed calls: before each timed call the baselines write
 * `bytes` of the device buffer `buf` (larger than L2) and time that call alone;
 * buf NULL or bytes 0 restores back-to-back timing. */
void tcaspmm_baselines_set_flush(void *buf, size_t bytes);

/* cusparseSpMM on a device CSR (int32 offsets/indices, values in dt), row-major
 * B (K x N, ld ldb) in dt, fp32 C (M x N, ld ldc), fp32 compute,
 * CUSPARSE_SPMM_ALG_DEFAULT.  Replaces perform_cuSPARSE_SpMM
 * (src/spmm_cusparse.cu:446-580) minus its host conversion and copies. */
tcaspmm_status tcaspmm_cusparse_spmm(const int32_t *d_row_ptr, const int32_t *d_col, const void *d_val, int64_t M,
                                     int64_t K, int64_t nnz, const void *dB, int64_t ldb, float *dC, int64_t ldc,
                                     int64_t N, tcaspmm_dtype dt, int warmup, int iters, void *stream,
                                     double *ms_per_iter);

/* Dense cublasGemmEx: C (M x N, fp32) = A (M x K, row-major, dt) * B (K x N,
 * row-major, dt), computed as C^T = B^T A^T in column-major with
 * CUBLAS_COMPUTE_32F, as perform_GemmEx does (src/gemm_cublas.cu:60-67). */
tcaspmm_status tcaspmm_cublas_gemm(const void *dA, const void *dB, float *dC, int64_t M, int64_t N, int64_t K,
                                   tcaspmm_dtype dt, int warmup, int iters, void *stream, double *ms_per_iter);

/* cusparseSpMM with A in Blocked-ELL: the host CSR A is converted to blocks of
 * block x block (every block-row padded to the widest one with column -1),
 * values rounded to dt (16-bit only), then uploaded; B (K x N, ld ldb) and C (M
 * x N fp32, ld ldc) as above, fp32 compute.  Replaces perform_cuSPARSE_BlockSpMM
 * (src/spmm_cusparse.cu:181-444), which builds the same format from a dense A.
 * M and K need not be multiples of block: A is padded with zero rows/columns and
 * C gets only its M rows.  *ell_bytes = bytes of the Blocked-ELL arrays. */
tcaspmm_status tcaspmm_cusparse_blocked_ell(const tcaspmm_csr *A, int block, const void *dB, int64_t ldb, float *dC,
                                           int64_t ldc, int64_t N, tcaspmm_dtype dt, int warmup, int iters,
                                           void *stream, double *ms_per_iter, int64_t *ell_bytes);

/* Gather floor of a CSR SpMM (no counterpart in the reference; a measurement
 * aid): loads every nonzero's B row slice (ncols elements of dt, ld ldb, 16-byte
 * aligned rows) the way tcaspmm's CUDA-core kernel does -- 16 bytes per lane,
 * several rows per warp instruction when ncols is narrow, 8 loads in flight --
 * for the column indices d_col[0..nnz), with no arithmetic and no C write.  Its
 * time is the floor any per-nonzero-gather SpMM of this matrix has on this GPU
 * (the L2-to-SM gather rate), beside which the kernel's own time is reported. */
tcaspmm_status tcaspmm_gather_floor(const int32_t *d_col, int64_t nnz, const void *dB, int64_t ldb, int64_t ncols,
                                    tcaspmm_dtype dt, int warmup, int iters, void *stream, double *ms_per_iter);

/* Device CSR arrays that a plan uploaded for `shard` (int32 offsets, int32
 * columns, values in the plan's dtype); lets a baseline run on the same bytes. */
tcaspmm_status tcaspmm_plan_device_csr(const tcaspmm_plan *plan, int shard, const int32_t **row_ptr,
                                       const int32_t **col, const void **val);

#ifdef __cplusplus
}
#endif

#endif /* TCASPMM_BASELINES_H */
