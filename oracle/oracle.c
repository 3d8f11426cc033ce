/*
 * CPU oracle for C = A * B with CSR A (M x K) and dense row-major B (K x N).
 *
 * TEST INFRASTRUCTURE ONLY.  Only tests/, __graft_entry__.smoke() and the
 * cpu_baseline / --impl reference legs of bench.py may load this library, and
 * only as the checker or the timed CPU baseline; the product (spmm_b200/) never
 * links or calls it.
 *
 * What it restates (paths are inside the YaoLingF/SPMM source tree):
 *   - The arithmetic of the hot path, our_spmm_balanced / kernel_our_spmm_balanced
 *     (src/our_spmm.cu:41-61 gathers val[j] * B[col[j]][n] for j in the row's
 *     range; src/our_spmm.cu:555 launches with alpha=1, beta=0 and the kernel
 *     overwrites C).  So C[i][n] = sum_{j=row_ptr[i]}^{row_ptr[i+1]-1} val[j]*B[col[j]][n].
 *     The reference ships no CPU CSR loop; its only CPU product is the dense
 *     naive_gemm (src/miscalleneous.cu:114-134), which the golden fixtures use
 *     to pin this restatement (tests/golden/make_golden.py).
 *   - The input conventions of convert_dense_to_csr (src/miscalleneous.cu:29-65:
 *     0-based, rows in order, columns ascending within a row, explicit zeros
 *     dropped) and of smtx_input_to_Dense (src/file_input.cu:135-193: header
 *     "M, K, nnz" split on ',', one line of M+1 row offsets split on ' ',
 *     every later line holds column indices split on ' ', every entry has the
 *     value 1.0).
 *
 * Parity is pinned: tests/test_oracle.py checks this file against fixtures
 * produced by the reference's own loader, dense->CSR conversion and naive_gemm
 * compiled from its sources (oracle/Makefile target `ref`).
 */
#include <math.h>
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

/* fp64 reference: inputs already rounded to the path's dtype and widened to
 * float; accumulation in double, fixed order j = row_ptr[i] .. row_ptr[i+1]-1.
 * Rows are independent, so the OpenMP split does not change any result. */
void oracle_spmm_f64(int64_t M, int64_t N, const int64_t *row_ptr, const int32_t *col,
                     const float *val, const float *B, int64_t ldb, double *C, int64_t ldc)
{
    int64_t i;
#pragma omp parallel for schedule(dynamic, 64)
    for (i = 0; i < M; i++) {
        double *c = C + i * ldc;
        for (int64_t n = 0; n < N; n++) c[n] = 0.0;
        for (int64_t j = row_ptr[i]; j < row_ptr[i + 1]; j++) {
            const double v = (double)val[j];
            const float *b = B + (int64_t)col[j] * ldb;
            for (int64_t n = 0; n < N; n++) c[n] += v * (double)b[n];
        }
    }
}

/* fp32 CPU CSR loop: the "reference CPU CSR loop" baseline that the benchmark
 * times on the host's cores.  OpenMP dynamic schedule over rows, the inner loop
 * over N is contiguous in both B and C so the compiler vectorises it. */
void oracle_spmm_f32(int64_t M, int64_t N, const int64_t *row_ptr, const int32_t *col,
                     const float *val, const float *B, int64_t ldb, float *C, int64_t ldc,
                     int nthreads)
{
#ifdef _OPENMP
    if (nthreads > 0) omp_set_num_threads(nthreads);
#endif
    int64_t i;
#pragma omp parallel for schedule(dynamic, 256)
    for (i = 0; i < M; i++) {
        float *restrict c = C + i * ldc;
        for (int64_t n = 0; n < N; n++) c[n] = 0.0f;
        for (int64_t j = row_ptr[i]; j < row_ptr[i + 1]; j++) {
            const float v = val[j];
            const float *restrict b = B + (int64_t)col[j] * ldb;
            for (int64_t n = 0; n < N; n++) c[n] += v * b[n];
        }
    }
}

/* Same loop restricted to a list of rows (a bounded sample of a large
 * workload); output row r of C_sample belongs to rows[r]. */
void oracle_spmm_f32_rows(int64_t nrows, const int64_t *rows, int64_t N, const int64_t *row_ptr,
                          const int32_t *col, const float *val, const float *B, int64_t ldb,
                          float *C_sample, int nthreads)
{
#ifdef _OPENMP
    if (nthreads > 0) omp_set_num_threads(nthreads);
#endif
    int64_t r;
#pragma omp parallel for schedule(dynamic, 256)
    for (r = 0; r < nrows; r++) {
        const int64_t i = rows[r];
        float *restrict c = C_sample + r * N;
        for (int64_t n = 0; n < N; n++) c[n] = 0.0f;
        for (int64_t j = row_ptr[i]; j < row_ptr[i + 1]; j++) {
            const float v = val[j];
            const float *restrict b = B + (int64_t)col[j] * ldb;
            for (int64_t n = 0; n < N; n++) c[n] += v * b[n];
        }
    }
}

int oracle_max_threads(void)
{
#ifdef _OPENMP
    return omp_get_max_threads();
#else
    return 1;
#endif
}

/* ---------------------------------------------------------------------------
 * .smtx pattern reader, restating smtx_input_to_Dense (src/file_input.cu:135-193)
 * but producing CSR instead of a dense matrix.  Two passes: oracle_smtx_header
 * returns M, K, nnz; oracle_smtx_read fills caller-owned arrays.
 * Returns 0 on success, a negative code on malformed input.
 * ------------------------------------------------------------------------- */
static int read_line(FILE *f, char **buf, size_t *cap)
{
    size_t len = 0;
    int ch;
    while ((ch = fgetc(f)) != EOF) {
        if (len + 2 > *cap) {
            *cap = *cap ? 2 * *cap : 4096;
            *buf = (char *)realloc(*buf, *cap);
        }
        if (ch == '\n') break;
        (*buf)[len++] = (char)ch;
    }
    if (ch == EOF && len == 0) return -1;
    if (!*buf) { *cap = 16; *buf = (char *)malloc(*cap); }
    (*buf)[len] = 0;
    return 0;
}

int oracle_smtx_header(const char *path, int64_t *M, int64_t *K, int64_t *nnz)
{
    FILE *f = fopen(path, "r");
    if (!f) return -1;
    char *line = NULL;
    size_t cap = 0;
    int rc = read_line(f, &line, &cap);
    if (rc == 0) {
        long long m, k, z;
        /* header fields are separated by ',' (src/file_input.cu:141-148) */
        if (sscanf(line, " %lld , %lld , %lld", &m, &k, &z) == 3) {
            *M = m; *K = k; *nnz = z;
        } else {
            rc = -2;
        }
    }
    free(line);
    fclose(f);
    return rc;
}

int oracle_smtx_read(const char *path, int64_t M, int64_t nnz, int64_t *row_ptr, int32_t *col)
{
    FILE *f = fopen(path, "r");
    if (!f) return -1;
    char *line = NULL;
    size_t cap = 0;
    int rc = 0;
    if (read_line(f, &line, &cap) != 0) { rc = -2; goto out; }       /* header */
    if (read_line(f, &line, &cap) != 0) { rc = -3; goto out; }       /* row_ptr */
    {
        int64_t idx = 0;
        char *p = line, *end;
        for (;;) {
            long long v = strtoll(p, &end, 10);
            if (end == p) break;
            if (idx > M) { rc = -4; goto out; }
            row_ptr[idx++] = v;
            p = end;
        }
        if (idx != M + 1) { rc = -4; goto out; }
    }
    {
        int64_t idx = 0;
        while (read_line(f, &line, &cap) == 0) {
            char *p = line, *end;
            for (;;) {
                long v = strtol(p, &end, 10);
                if (end == p) break;
                if (idx >= nnz) { rc = -5; goto out; }
                col[idx++] = (int32_t)v;
                p = end;
            }
        }
        if (idx != nnz) rc = -5;
    }
out:
    free(line);
    fclose(f);
    return rc;
}
