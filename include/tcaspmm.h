/*
 * tcaspmm — B200-native SpMM, C = A * B, CSR A (M x K), dense row-major B (K x N),
 * fp32 C (M x N, row-major, overwritten; optionally through a fused epilogue).
 * C-ABI boundary of libtcaspmm.so.
 *
 * Every entry point returns a tcaspmm_status (never exits), except
 * our_spmm_balanced, which keeps the reference's void signature and its
 * exit-on-CUDA-error behaviour.  Reference citations are paths inside the
 * YaoLingF/SPMM tree.
 *
 * Threading: a plan may be executed from one host thread on one stream at a
 * time (its scratch buffers are shared by all launches of that plan).
 * Different plans may run concurrently.  A plan whose tensor-core windows
 * leave SMs idle and that also has CUDA-core rows runs its tensor-core kernel
 * on a side stream it owns, forked from the caller's stream and joined back to
 * it by events inside each execute call (CUDA-graph capture sees two parallel
 * kernel nodes); work ordered on the caller's stream before and after the
 * call is ordered against both kernels.
 */
#ifndef TCASPMM_H
#define TCASPMM_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef enum tcaspmm_status {
    TCASPMM_OK = 0,
    TCASPMM_ERR_INVALID_ARG = 1, /* bad pointer, shape, stride or dtype */
    TCASPMM_ERR_IO = 2,          /* file cannot be opened / written */
    TCASPMM_ERR_FORMAT = 3,      /* malformed .smtx contents */
    TCASPMM_ERR_ALLOC = 4,       /* host or device allocation failed */
    TCASPMM_ERR_CUDA = 5,        /* a CUDA runtime call failed */
    TCASPMM_ERR_UNSUPPORTED = 6, /* valid input outside the supported range */
    TCASPMM_ERR_TIMEOUT = 7,     /* a bounded device-side wait ran out */
    TCASPMM_ERR_NO_DEVICE = 8    /* no CUDA device (or fewer than requested) */
} tcaspmm_status;

/* Element type of B (and of the device copy of A's values). C is fp32 (or, with
 * an epilogue, fp16 / bf16).  fp32 runs the CUDA-core path in fp32; f16 / bf16 /
 * tf32 use the tensor-core tiles for dense windows with fp32 accumulation. */
typedef enum tcaspmm_dtype {
    TCASPMM_F32 = 0,
    TCASPMM_F16 = 1,
    TCASPMM_BF16 = 2,
    /* fp32 storage (B and A's values as fp32); tensor-core windows multiply in
     * TF32 (tcgen05 kind::tf32, 10-bit mantissa, fp32 accumulate), the CUDA-core
     * residue stays fp32.  Opt-in: TCASPMM_F32 never uses the tensor cores. */
    TCASPMM_TF32 = 3
} tcaspmm_dtype;

/* Replaces mat_format {dense, csr, coo} (src/mat_format.cuh:10-15). */
typedef enum tcaspmm_mat_format {
    TCASPMM_FORMAT_DENSE = 0,
    TCASPMM_FORMAT_CSR = 1,
    TCASPMM_FORMAT_COO = 2
} tcaspmm_mat_format;

/* Host CSR matrix.  0-based, rows in order, columns strictly ascending within a
 * row (the convention of convert_dense_to_csr, src/miscalleneous.cu:29-65).
 * val == NULL means a pattern matrix: every stored value is 1.0, as the .smtx
 * loader writes them (src/file_input.cu:189).  Replaces struct CSR
 * (src/general.cuh:125-134) with 64-bit row offsets and fp32 host values. */
typedef struct tcaspmm_csr {
    int64_t nrow;
    int64_t ncol;
    int64_t nnz;
    int64_t *row_ptr; /* nrow + 1 */
    int32_t *col_idx; /* nnz */
    float *val;       /* nnz, or NULL (pattern) */
} tcaspmm_csr;

/* Layout twin of the reference's struct CSR (src/general.cuh:125-134):
 * {int nRow, nCol, nnz; int *row_offset; int *col_idx; half *value}.
 * `value` points at IEEE binary16 bit patterns. */
typedef struct tcaspmm_ref_csr {
    int nRow;
    int nCol;
    int nnz;
    int *row_offset;
    int *col_idx;
    uint16_t *value;
} tcaspmm_ref_csr;

typedef struct tcaspmm_plan tcaspmm_plan;

/* Summary of a plan (host side), for reports and tests. */
typedef struct tcaspmm_plan_stats {
    int64_t nrow, ncol, nnz, ncols_total;
    int32_t num_shards;
    int32_t window_rows;      /* rows per tensor-core window */
    int64_t tc_windows;       /* windows run on the tensor-core tiles */
    int64_t tc_tiles;         /* condensed column tiles over all tc windows */
    int64_t tc_nnz;           /* nonzeros covered by tiles */
    int64_t residue_nnz;      /* nonzeros covered by the CUDA-core kernel */
    int64_t residue_row_warps;/* warps that each own a contiguous row range */
    int64_t residue_segments; /* long-row segments (partial sums + fix-up) */
    int64_t long_rows;        /* rows split into segments */
    double preprocess_ms;     /* host preprocessing (schedule) time */
    double upload_ms;         /* plan upload (alloc + H2D) time */
    int64_t device_bytes;     /* device memory held by shard 0 */
    int64_t algorithmic_bytes;/* A + B + C bytes (A: (M+1)*4 + nnz*(4+sizeof(val))) */
    int64_t tc_gathered_windows; /* tc windows of long rows grouped by length (row lists) */
    int64_t tc_tasks;         /* tensor-core work items per column block (windows split by tiles) */
    int64_t tc_ctas_per_sm;   /* resident tensor-core CTAs per SM (the persistent grid is this x SMs) */
    int64_t tc_side_stream;   /* 1: the tensor-core kernel runs beside the residue kernel on a side stream */
} tcaspmm_plan_stats;

/* ---------------------------------------------------------------- errors */
const char *tcaspmm_status_string(tcaspmm_status s);
/* Message describing the last failure on the calling thread ("" if none). */
const char *tcaspmm_last_error(void);

/* --------------------------------------------------------------- host CSR */
/* Allocate a host CSR (row_ptr zeroed; val allocated when with_values != 0). */
tcaspmm_status tcaspmm_csr_alloc(int64_t nrow, int64_t ncol, int64_t nnz, int with_values,
                                 tcaspmm_csr *out);
/* Free the arrays of a CSR made by this library and zero the struct. */
tcaspmm_status tcaspmm_csr_free(tcaspmm_csr *A);
/* Check the CSR invariants (monotone row_ptr, in-range ascending columns). */
tcaspmm_status tcaspmm_csr_validate(const tcaspmm_csr *A);

/* Read a .smtx file straight into CSR.  Format of smtx_input_to_Dense
 * (src/file_input.cu:135-193): line 1 "M, K, nnz", line 2 the M+1 row offsets,
 * later lines the column indices.  Values: if "<path>.val" exists (nnz
 * little-endian float32) it is read, else A is a pattern matrix (val = NULL).
 * Replaces smtx_input_to_Dense (src/file_input.cu:135) and the empty stub
 * smtx_input_to_CSR (src/file_input.cu:194-196). */
tcaspmm_status tcaspmm_smtx_read(const char *path, tcaspmm_csr *out);
/* Write A as .smtx (and "<path>.val" when A->val != NULL). */
tcaspmm_status tcaspmm_smtx_write(const char *path, const tcaspmm_csr *A);

/* Read a Matrix Market coordinate file (real / integer / pattern; general,
 * symmetric or skew-symmetric) into CSR: columns sorted per row, repeated
 * entries summed, symmetric files expanded.  Indices are 1-based as the format
 * says unless zero_based != 0 (the reference reader's default).  Replaces
 * mtx_input_to_CSR (src/file_input.cu:64-134). */
tcaspmm_status tcaspmm_mtx_read(const char *path, int zero_based, tcaspmm_csr *out);
/* Binary CSR companion ("TCACSR01" header, int64 offsets, int32 columns,
 * optional float32 values) for graphs too large for text. */
tcaspmm_status tcaspmm_csrbin_write(const char *path, const tcaspmm_csr *A);
tcaspmm_status tcaspmm_csrbin_read(const char *path, tcaspmm_csr *out);

/* Dense row-major M x K binary16 matrix -> CSR, dropping zeros.
 * Replaces convert_dense_to_csr (src/miscalleneous.cu:29-65). */
tcaspmm_status tcaspmm_dense_to_csr(const uint16_t *dense, int64_t M, int64_t K, tcaspmm_csr *out);

/* ----------------------------------------------------- seeded generators
 * Counter-based SplitMix64 streams: every value depends only on (seed, index),
 * so results are identical for any thread count.  Replaces the unseeded
 * prepare_cpu_matrix (src/general.cuh:140-174). */
/* rows x cols N(0,1) values rounded to dt, written to out (row-major, ld = cols). */
tcaspmm_status tcaspmm_gen_dense(int64_t rows, int64_t cols, uint64_t seed, tcaspmm_dtype dt,
                                 void *out);
/* Each entry kept with probability density, values N(0,1). */
tcaspmm_status tcaspmm_gen_uniform(int64_t M, int64_t K, double density, uint64_t seed,
                                   tcaspmm_csr *out);
/* Magnitude pruning: W = s_i * Z_ij, s_i ~ LogNormal(0, 0.5), Z ~ N(0,1); keep
 * the globally largest (1 - sparsity) fraction of |W|; values are W. */
tcaspmm_status tcaspmm_gen_magnitude(int64_t M, int64_t K, double sparsity, uint64_t seed,
                                     tcaspmm_csr *out);
/* R-MAT(a, b, c) graph on 2^scale nodes with `edges` directed draws.
 * kind 0 (GCN): symmetrise, add self-loops, dedupe, values 1/sqrt(d_i d_j).
 * kind 1 (SAGE mean): dedupe directed edges, values 1/deg(i). */
tcaspmm_status tcaspmm_gen_rmat(int scale, int64_t edges, double a, double b, double c, int kind,
                                uint64_t seed, tcaspmm_csr *out);
/* Extreme skew: n x n, `hubs` rows (evenly spaced) with hub_nnz distinct uniform
 * columns, every other row Poisson(lambda) uniform columns; values U(-1, 1). */
tcaspmm_status tcaspmm_gen_skew(int64_t n, int64_t hubs, int64_t hub_nnz, double lambda,
                                uint64_t seed, tcaspmm_csr *out);

/* --------------------------------------------------------- multi-GPU split
 * Column partition of B and C over `world` GPUs: contiguous blocks of
 * ceil(N / world) columns rounded up to a 16-byte multiple of dt. */
tcaspmm_status tcaspmm_partition_columns(int64_t N, tcaspmm_dtype dt, int world, int rank,
                                         int64_t *col_begin, int64_t *col_count);
/* Row partition of A and C over `parts` GPUs (the 2-D / A-splitting variant for
 * when A's bytes dominate): row_begin[0..parts] (parts + 1 entries, row_begin[0]
 * = 0, row_begin[parts] = M), contiguous blocks of about equal cost (nnz + 2 per
 * row); B is replicated.  Deterministic. */
tcaspmm_status tcaspmm_partition_rows(const tcaspmm_csr *A, int parts, int64_t *row_begin);

/* ------------------------------------------------------------------ plans
 * A plan holds the preprocessed schedule of A and every device buffer the
 * kernels read (A's CSR arrays, the schedule, tensor-core tiles, scratch).
 * Replaces workload_manager (src/our_spmm.cu:353-477) and the per-call device
 * setup of our_spmm_balanced (src/our_spmm.cu:486-550).
 *
 * Schedule tuning, read from the environment when a plan is created (integers;
 * unset = the measured defaults):
 *   TCASPMM_DISABLE_TC=1       every row on the CUDA-core residue kernel
 *   TCASPMM_BUDGET_MAX=1024    cap on a residue warp's nonzeros (per lane group
 *                              for one or two groups per warp, divided among
 *                              the groups otherwise, halved from eight groups)
 *   TCASPMM_BUDGET_MIN=128     floor on a lane group's nonzeros
 *   TCASPMM_WARPS_PER_SM=32    residue warps per SM the work is spread over
 *   TCASPMM_HUB_WINDOWS=0      1: long rows grouped by length into gathered
 *                              tensor-core windows
 *   TCASPMM_SPLIT_TILES=128    tiles per work item of a gathered window
 *   TCASPMM_WINDOW_PARTS=0     parts per consecutive tensor-core window (0: cut
 *                              into parts of at least 4 stages only while the
 *                              work items leave SMs without one)
 *   TCASPMM_GATHER_TMA=1       0: gathered 16-bit tiles fetched by cp.async from
 *                              all producer threads instead of TMA gather4
 *   TCASPMM_DENSE_RUNS=1       0: windows whose columns are one consecutive run
 *                              fetched through tile indices like gathered ones
 *   TCASPMM_TC_DENSITY=32      a consecutive window needs at least 1/this of its
 *                              tile entries nonzero
 *   TCASPMM_OVERLAP=1          0: the tensor-core kernel never runs beside the
 *                              residue kernel on a side stream
 * Values are clamped (BUDGET_MAX to [16, 2^20], BUDGET_MIN to [1, 2^20],
 * WARPS_PER_SM to [1, 1024], TC_DENSITY to [1, 1024], DISABLE_TC, HUB_WINDOWS,
 * GATHER_TMA, DENSE_RUNS and OVERLAP to [0, 1], SPLIT_TILES to [1, 4096],
 * WINDOW_PARTS to [0, 64]); a value that is not a whole number falls back to
 * the default.  The results stay within the same
 * tolerances whatever these are; long rows may be summed in a different order. */

/* One plan over num_gpus devices (devices[i], or 0..num_gpus-1 when NULL); the
 * N columns are split by tcaspmm_partition_columns. */
tcaspmm_status tcaspmm_plan_create(const tcaspmm_csr *A, int64_t N, tcaspmm_dtype dt, int num_gpus,
                                   const int *devices, tcaspmm_plan **out);
/* One process per GPU: a plan for rank's column block only, on `device`. */
tcaspmm_status tcaspmm_plan_create_shard(const tcaspmm_csr *A, int64_t N, tcaspmm_dtype dt, int rank,
                                         int world, int device, tcaspmm_plan **out);
/* Row-split plans (tcaspmm_partition_rows): shard s holds rows [row_begin[s],
 * row_begin[s+1]) of A and all N columns; at execute, dB[s] is the whole K x N
 * B on its device and dC[s] the shard's (row_count x N) block of C. */
tcaspmm_status tcaspmm_plan_create_rows(const tcaspmm_csr *A, int64_t N, tcaspmm_dtype dt, int num_gpus,
                                        const int *devices, tcaspmm_plan **out);
/* One process per GPU: the plan of rank's row block only, on `device`. */
tcaspmm_status tcaspmm_plan_create_rows_shard(const tcaspmm_csr *A, int64_t N, tcaspmm_dtype dt, int rank,
                                              int world, int device, tcaspmm_plan **out);
/* 2-D plans: grid_rows x grid_cols shards; shard s = (s / grid_cols, s % grid_cols)
 * holds row block s / grid_cols of tcaspmm_partition_rows(A, grid_rows) and column
 * block s % grid_cols of tcaspmm_partition_columns(N, dt, grid_cols, .): each GPU
 * streams part of A and copies part of B.  dB[s] is the K x col_count block of B,
 * dC[s] the row_count x col_count block of C. */
tcaspmm_status tcaspmm_plan_create_2d(const tcaspmm_csr *A, int64_t N, tcaspmm_dtype dt, int grid_rows,
                                      int grid_cols, const int *devices, tcaspmm_plan **out);
/* One process per GPU: the plan of shard `rank` of the grid, on `device`. */
tcaspmm_status tcaspmm_plan_create_2d_shard(const tcaspmm_csr *A, int64_t N, tcaspmm_dtype dt, int rank,
                                            int grid_rows, int grid_cols, int device, tcaspmm_plan **out);
/* Shard s's row block [row_begin, row_begin + row_count) (0 and M for column-split plans). */
tcaspmm_status tcaspmm_plan_shard_rows(const tcaspmm_plan *plan, int shard, int64_t *row_begin,
                                       int64_t *row_count);
tcaspmm_status tcaspmm_plan_destroy(tcaspmm_plan *plan);
tcaspmm_status tcaspmm_plan_get_stats(const tcaspmm_plan *plan, tcaspmm_plan_stats *out);
/* Shard s of the plan: its device and its column block [col_begin, col_begin + col_count). */
tcaspmm_status tcaspmm_plan_shard(const tcaspmm_plan *plan, int shard, int *device,
                                  int64_t *col_begin, int64_t *col_count);

/* Run C = A * B on every shard.  Per shard s: dB[s] is the device K x col_count
 * block of B with leading dimension ldb[s] (elements), dC[s] the device M x
 * col_count block of C with leading dimension ldc[s], streams[s] a cudaStream_t
 * (NULL = legacy default stream).  Asynchronous: returns after the launches. */
tcaspmm_status tcaspmm_execute(tcaspmm_plan *plan, const void *const *dB, const int64_t *ldb,
                               float *const *dC, const int64_t *ldc, void *const *streams);
/* Single-shard convenience form of tcaspmm_execute. */
tcaspmm_status tcaspmm_execute1(tcaspmm_plan *plan, const void *dB, int64_t ldb, float *dC,
                                int64_t ldc, void *stream);
/* Fused output epilogue (no counterpart in the reference, whose kernel ignores
 * alpha/beta, src/our_spmm.cu:296-352): per shard,
 *     C[r][c] = relu?( row_scale[r] * (A B)[r][c] + bias[c] )
 * with row_scale (one float per row of the shard: M, or row_count for a
 * row-split plan) and bias (col_count floats, the shard's column block) device
 * arrays on the shard's device, NULL meaning 1 and 0, and C
 * stored as out_dtype: TCASPMM_F32, TCASPMM_F16 or TCASPMM_BF16 (16-bit C halves
 * the C bytes).  GraphSAGE mean aggregation is a pattern A with
 * row_scale = 1/deg; a GCN layer's bias and ReLU fold in the same way. */
typedef struct tcaspmm_epilogue {
    const float *row_scale;
    const float *bias;
    int relu;
    tcaspmm_dtype out_dtype;
} tcaspmm_epilogue;

/* tcaspmm_execute with an epilogue per shard (epilogues NULL = plain fp32 C);
 * dC[s] has out_dtype elements and ldc[s] counts them. */
tcaspmm_status tcaspmm_execute_ex(tcaspmm_plan *plan, const void *const *dB, const int64_t *ldb,
                                  void *const *dC, const int64_t *ldc, void *const *streams,
                                  const tcaspmm_epilogue *epilogues);
/* Single-shard form of tcaspmm_execute_ex (ep NULL = plain fp32 C). */
tcaspmm_status tcaspmm_execute1_ex(tcaspmm_plan *plan, const void *dB, int64_t ldb, void *dC,
                                   int64_t ldc, void *stream, const tcaspmm_epilogue *ep);
/* Wait for the plan's shards and report a device-side error (a bounded wait
 * that ran out in a tensor-core kernel) as TCASPMM_ERR_TIMEOUT. */
tcaspmm_status tcaspmm_plan_sync_check(tcaspmm_plan *plan);

/* ------------------------------------------------- schedule inspection
 * Build the host schedule without touching a GPU and report, for every
 * nonzero j of A, how many work units cover it (cover[j], must be 1) and which
 * kind covers it (kind[j]: 1 residue row, 2 residue segment, 3 tensor-core tile
 * cell).  Tile cells are also checked against A's column and value. */
tcaspmm_status tcaspmm_schedule_coverage(const tcaspmm_csr *A, int64_t N, tcaspmm_dtype dt,
                                         int32_t *cover, int8_t *kind, tcaspmm_plan_stats *stats);

/* ------------------------------------------------------------ self-test
 * Failure detection of the tensor-core kernel without a GPU fault: launches one
 * tensor-core window on `device` whose producer never issues its copies, so the
 * MMA thread's bounded wait runs out after `wait_cycles` SM clocks; the kernel
 * records the time-out, stops, frees its tensor memory and returns, and the
 * context stays usable.  Returns TCASPMM_ERR_TIMEOUT (the designed outcome) with
 * the device error word in *err_code; TCASPMM_OK would mean no time-out was seen. */
tcaspmm_status tcaspmm_selftest_tc_timeout(int device, unsigned long long wait_cycles, int *err_code);

/* ------------------------------------------------- reference entry point
 * Same signature, argument meaning and behaviour as our_spmm_balanced
 * (src/our_spmm.cuh:4, src/our_spmm.cu:478-594): host CSR with binary16 values,
 * host binary16 B (K x N), host fp32 C (M x N) overwritten; allocates device
 * memory, copies in, preprocesses, runs 5 warm-up and n_iter timed launches,
 * copies C back, frees, and stores the average kernel milliseconds in
 * *elapsed (if not NULL).  On a CUDA error it prints the error and exits, as
 * CHECK_CUDA does (src/general.cuh:8-16). */
void our_spmm_balanced(tcaspmm_ref_csr *A_csr, uint16_t *B, float *C, int M, int N, int K,
                       int n_iter, double *elapsed);
/* Status-returning form of our_spmm_balanced (no exit). */
tcaspmm_status tcaspmm_our_spmm_balanced(const tcaspmm_ref_csr *A_csr, const uint16_t *B, float *C,
                                         int M, int N, int K, int n_iter, double *elapsed);

/* ------------------------------------------------ no-allocation entry point
 * No counterpart in the reference: an addition for callers that must not
 * allocate device memory at the moment they multiply (a plugin inside a host
 * framework that owns every device allocation, a latency-critical loop where an
 * allocation could block or fragment a memory pool, a caller with a fixed
 * memory budget).  C = A * B with A in CSR already in the caller's device memory
 * (int32 offsets [M+1], int32 columns [nnz], values [nnz] in dt), B (K x N, ld
 * ldb, dt) and fp32 C (M x N, ld ldc) in device memory, launched on `stream`.
 * It calls no cudaMalloc / cudaFree and no allocating library routine: its only
 * scratch is a fixed 16 MiB array inside the library image, which every GPU
 * that loads the library holds until the process exits.  Limit: two partial
 * rows of N floats (N rounded up to 4) must fit in that array, so N <= 2097152;
 * larger N, and nnz above 2^31 - 65, return TCASPMM_ERR_UNSUPPORTED.  All calls
 * on one device share that device's array: calls whose kernels overlap on the
 * GPU race and must be serialised by the caller.  The first call on each device
 * looks up the array's device address with that device current; with lazy
 * module loading (the CUDA default since 12.2) that is also when the driver
 * loads the library's device code and commits the 16 MiB on that device, so the
 * first call can fail with an out-of-memory error.  Make one warm-up call per
 * device at initialisation: before any stream capture and before the caller's
 * memory budget is fixed. */
tcaspmm_status tcaspmm_spmm_csr_noalloc(const int32_t *d_row_ptr, const int32_t *d_col, const void *d_val,
                                        int64_t M, int64_t K, int64_t nnz, const void *dB, int64_t ldb, float *dC,
                                        int64_t ldc, int64_t N, tcaspmm_dtype dt, void *stream);

#ifdef __cplusplus
}
#endif

#endif /* TCASPMM_H */
