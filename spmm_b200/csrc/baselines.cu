// cuSPARSE and cuBLAS baselines (libtcaspmm_baselines.so).  Reported next to
// tcaspmm, never called by it.
#include <algorithm>
#include <cstdio>
#include <cstring>
#include <vector>

#include <cublas_v2.h>
#include <cuda_runtime.h>
#include <cusparse.h>

#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include "tcaspmm_baselines.h"

namespace {

thread_local char g_msg[512];

tcaspmm_status bfail(tcaspmm_status s, const char *what, int code)
{
    std::snprintf(g_msg, sizeof(g_msg), "%s failed (%d)", what, code);
    std::fprintf(stderr, "tcaspmm baselines: %s\n", g_msg);
    return s;
}

cudaDataType_t cuda_type(tcaspmm_dtype dt)
{
    return (dt == TCASPMM_F32 || dt == TCASPMM_TF32) ? CUDA_R_32F : dt == TCASPMM_F16 ? CUDA_R_16F : CUDA_R_16BF;
}

// L2 flush between timed calls (set by tcaspmm_baselines_set_flush): the same
// protocol bench.py uses for tcaspmm on inputs smaller than L2.
void *g_flush = nullptr;
size_t g_flush_bytes = 0;

template <typename F>
tcaspmm_status time_loop(F &&f, int warmup, int iters, cudaStream_t st, double *ms)
{
    for (int i = 0; i < warmup; i++)
        if (!f()) return bfail(TCASPMM_ERR_CUDA, "baseline warm-up", 0);
    cudaEvent_t a, b;
    cudaEventCreate(&a);
    cudaEventCreate(&b);
    bool ok = true;
    float t = 0.0f;
    if (g_flush) {
        // Per call: flush, then events around the call alone.
        for (int i = 0; i < iters && ok; i++) {
            cudaMemsetAsync(g_flush, i & 0xff, g_flush_bytes, st);
            cudaEventRecord(a, st);
            ok = f();
            cudaEventRecord(b, st);
            cudaEventSynchronize(b);
            float ti = 0.0f;
            cudaEventElapsedTime(&ti, a, b);
            t += ti;
        }
    } else {
        cudaEventRecord(a, st);
        for (int i = 0; i < iters && ok; i++) ok = f();
        cudaEventRecord(b, st);
        cudaEventSynchronize(b);
        cudaEventElapsedTime(&t, a, b);
    }
    cudaEventDestroy(a);
    cudaEventDestroy(b);
    cudaError_t e = cudaGetLastError();
    if (!ok || e != cudaSuccess) return bfail(TCASPMM_ERR_CUDA, "baseline timed loop", (int)e);
    *ms = iters > 0 ? t / iters : 0.0;
    return TCASPMM_OK;
}

}  // namespace

extern "C" void tcaspmm_baselines_set_flush(void *buf, size_t bytes)
{
    g_flush = bytes ? buf : nullptr;
    g_flush_bytes = bytes;
}

extern "C" tcaspmm_status tcaspmm_cusparse_spmm(const int32_t *d_row_ptr, const int32_t *d_col, const void *d_val,
                                                int64_t M, int64_t K, int64_t nnz, const void *dB, int64_t ldb,
                                                float *dC, int64_t ldc, int64_t N, tcaspmm_dtype dt, int warmup,
                                                int iters, void *stream, double *ms_per_iter)
{
    if (!ms_per_iter) return TCASPMM_ERR_INVALID_ARG;
    cudaStream_t st = (cudaStream_t)stream;
    cusparseHandle_t h = nullptr;
    cusparseSpMatDescr_t A = nullptr;
    cusparseDnMatDescr_t Bd = nullptr, Cd = nullptr;
    void *buf = nullptr;
    size_t bsz = 0;
    const float alpha = 1.0f, beta = 0.0f;
    tcaspmm_status s = TCASPMM_OK;
    int rc;
    if ((rc = cusparseCreate(&h)) != CUSPARSE_STATUS_SUCCESS) return bfail(TCASPMM_ERR_CUDA, "cusparseCreate", rc);
    cusparseSetStream(h, st);
    rc = cusparseCreateCsr(&A, M, K, nnz, (void *)d_row_ptr, (void *)d_col, (void *)d_val, CUSPARSE_INDEX_32I,
                           CUSPARSE_INDEX_32I, CUSPARSE_INDEX_BASE_ZERO, cuda_type(dt));
    if (rc == CUSPARSE_STATUS_SUCCESS)
        rc = cusparseCreateDnMat(&Bd, K, N, ldb, (void *)dB, cuda_type(dt), CUSPARSE_ORDER_ROW);
    if (rc == CUSPARSE_STATUS_SUCCESS) rc = cusparseCreateDnMat(&Cd, M, N, ldc, dC, CUDA_R_32F, CUSPARSE_ORDER_ROW);
    if (rc == CUSPARSE_STATUS_SUCCESS)
        rc = cusparseSpMM_bufferSize(h, CUSPARSE_OPERATION_NON_TRANSPOSE, CUSPARSE_OPERATION_NON_TRANSPOSE, &alpha, A,
                                     Bd, &beta, Cd, CUDA_R_32F, CUSPARSE_SPMM_ALG_DEFAULT, &bsz);
    if (rc != CUSPARSE_STATUS_SUCCESS) {
        s = bfail(TCASPMM_ERR_CUDA, "cusparse setup", rc);
    } else if (bsz && cudaMalloc(&buf, bsz) != cudaSuccess) {
        s = bfail(TCASPMM_ERR_ALLOC, "cusparse workspace", 0);
    } else {
        auto run = [&]() {
            return cusparseSpMM(h, CUSPARSE_OPERATION_NON_TRANSPOSE, CUSPARSE_OPERATION_NON_TRANSPOSE, &alpha, A, Bd,
                                &beta, Cd, CUDA_R_32F, CUSPARSE_SPMM_ALG_DEFAULT, buf) == CUSPARSE_STATUS_SUCCESS;
        };
        s = time_loop(run, warmup, iters, st, ms_per_iter);
    }
    if (buf) cudaFree(buf);
    if (Cd) cusparseDestroyDnMat(Cd);
    if (Bd) cusparseDestroyDnMat(Bd);
    if (A) cusparseDestroySpMat(A);
    cusparseDestroy(h);
    return s;
}

namespace {

// Gather floor: every nonzero's B row slice loaded the way the residue kernel
// loads it -- G lanes x 16 bytes per row (P = 32 / G rows per warp instruction),
// 8 loads in flight per lane, each warp streaming 1024 consecutive nonzeros --
// with no multiply, no value load and no C write.  A checksum of the loaded bits
// keeps the loads alive.
template <int G>
__global__ void __launch_bounds__(128) gather_floor_kernel(const int32_t *__restrict__ col, long long nnz,
                                                           const uint4 *__restrict__ B, long long pitch16, int nvec,
                                                           unsigned int *sink)
{
    constexpr int P = 32 / G, U = 8;
    const int lane = threadIdx.x & 31, sub = lane / G, gl = lane % G;
    const long long warp = ((long long)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const long long j0 = warp * 1024, j1 = j0 + 1024 < nnz ? j0 + 1024 : nnz;
    if (j0 >= j1) return;
    const long long jb = j0 + (j1 - j0) * sub / P, je = j0 + (j1 - j0) * (sub + 1) / P;
    unsigned int x = 0;
    for (int v = gl; v < nvec; v += G) {
        long long j = jb;
        for (; j + U <= je; j += U) {
            int c[U];
#pragma unroll
            for (int u = 0; u < U; ++u) c[u] = __ldg(col + j + u);
            uint4 r[U];
#pragma unroll
            for (int u = 0; u < U; ++u) r[u] = __ldg(B + (long long)c[u] * pitch16 + v);
#pragma unroll
            for (int u = 0; u < U; ++u) x ^= r[u].x ^ r[u].y ^ r[u].z ^ r[u].w;
        }
        for (; j < je; ++j) {
            const uint4 r = __ldg(B + (long long)__ldg(col + j) * pitch16 + v);
            x ^= r.x ^ r.y ^ r.z ^ r.w;
        }
    }
    if (x == 0x9e3779b9u) *sink = x;
}

}  // namespace

extern "C" tcaspmm_status tcaspmm_gather_floor(const int32_t *d_col, int64_t nnz, const void *dB, int64_t ldb,
                                               int64_t ncols, tcaspmm_dtype dt, int warmup, int iters, void *stream,
                                               double *ms_per_iter)
{
    if (!ms_per_iter || nnz < 0 || ncols <= 0) return TCASPMM_ERR_INVALID_ARG;
    const int64_t es = (dt == TCASPMM_F32 || dt == TCASPMM_TF32) ? 4 : 2;
    if ((ncols * es) % 16 != 0 || (ldb * es) % 16 != 0 || (uintptr_t)dB % 16 != 0)
        return bfail(TCASPMM_ERR_UNSUPPORTED, "gather floor: B rows must be 16-byte aligned", 0);
    const int nvec = (int)(ncols * es / 16);
    int G = 1;
    while (G < nvec && G < 32) G *= 2;
    cudaStream_t st = (cudaStream_t)stream;
    unsigned int *sink = nullptr;
    if (cudaMalloc((void **)&sink, sizeof(unsigned int)) != cudaSuccess)
        return bfail(TCASPMM_ERR_ALLOC, "gather floor sink", 0);
    const long long warps = (nnz + 1023) / 1024;
    const unsigned blocks = (unsigned)((warps + 3) / 4);
    const long long pitch16 = ldb * es / 16;
    const uint4 *B = static_cast<const uint4 *>(dB);
    auto run = [&]() {
        if (blocks == 0) return true;
        switch (G) {
        case 1: gather_floor_kernel<1><<<blocks, 128, 0, st>>>(d_col, nnz, B, pitch16, nvec, sink); break;
        case 2: gather_floor_kernel<2><<<blocks, 128, 0, st>>>(d_col, nnz, B, pitch16, nvec, sink); break;
        case 4: gather_floor_kernel<4><<<blocks, 128, 0, st>>>(d_col, nnz, B, pitch16, nvec, sink); break;
        case 8: gather_floor_kernel<8><<<blocks, 128, 0, st>>>(d_col, nnz, B, pitch16, nvec, sink); break;
        case 16: gather_floor_kernel<16><<<blocks, 128, 0, st>>>(d_col, nnz, B, pitch16, nvec, sink); break;
        default: gather_floor_kernel<32><<<blocks, 128, 0, st>>>(d_col, nnz, B, pitch16, nvec, sink); break;
        }
        return cudaGetLastError() == cudaSuccess;
    };
    tcaspmm_status s = time_loop(run, warmup, iters, st, ms_per_iter);
    cudaFree(sink);
    return s;
}

extern "C" tcaspmm_status tcaspmm_cublas_gemm(const void *dA, const void *dB, float *dC, int64_t M, int64_t N,
                                              int64_t K, tcaspmm_dtype dt, int warmup, int iters, void *stream,
                                              double *ms_per_iter)
{
    if (!ms_per_iter) return TCASPMM_ERR_INVALID_ARG;
    cudaStream_t st = (cudaStream_t)stream;
    cublasHandle_t h = nullptr;
    int rc = cublasCreate(&h);
    if (rc != CUBLAS_STATUS_SUCCESS) return bfail(TCASPMM_ERR_CUDA, "cublasCreate", rc);
    cublasSetStream(h, st);
    const float alpha = 1.0f, beta = 0.0f;
    auto run = [&]() {
        return cublasGemmEx(h, CUBLAS_OP_N, CUBLAS_OP_N, (int)N, (int)M, (int)K, &alpha, dB, cuda_type(dt), (int)N,
                            dA, cuda_type(dt), (int)K, &beta, dC, CUDA_R_32F, (int)N, CUBLAS_COMPUTE_32F,
                            CUBLAS_GEMM_DEFAULT) == CUBLAS_STATUS_SUCCESS;
    };
    tcaspmm_status s = time_loop(run, warmup, iters, st, ms_per_iter);
    cublasDestroy(h);
    return s;
}

extern "C" tcaspmm_status tcaspmm_cusparse_blocked_ell(const tcaspmm_csr *A, int block, const void *dB, int64_t ldb,
                                                      float *dC, int64_t ldc, int64_t N, tcaspmm_dtype dt, int warmup,
                                                      int iters, void *stream, double *ms_per_iter, int64_t *ell_bytes)
{
    if (!A || !ms_per_iter || block < 1 || dt == TCASPMM_F32 || dt == TCASPMM_TF32) return TCASPMM_ERR_INVALID_ARG;
    tcaspmm_status s = tcaspmm_csr_validate(A);
    if (s != TCASPMM_OK) return s;
    const int64_t M = A->nrow, K = A->ncol;
    const int64_t brows = (M + block - 1) / block, Mp = brows * block, Kp = (K + block - 1) / block * block;
    // Nonzero block-columns of every block-row, ascending.
    std::vector<std::vector<int32_t>> bcols((size_t)brows);
    int64_t width = 0;
    for (int64_t br = 0; br < brows; br++) {
        std::vector<int32_t> &v = bcols[br];
        for (int64_t r = br * block; r < std::min(M, (br + 1) * block); r++)
            for (int64_t j = A->row_ptr[r]; j < A->row_ptr[r + 1]; j++) v.push_back(A->col_idx[j] / block);
        std::sort(v.begin(), v.end());
        v.erase(std::unique(v.begin(), v.end()), v.end());
        width = std::max<int64_t>(width, (int64_t)v.size());
    }
    width = std::max<int64_t>(width, 1);
    const int64_t ell_cols = width * block;
    std::vector<int32_t> colidx((size_t)(brows * width), -1);
    std::vector<uint16_t> vals((size_t)(Mp * ell_cols), 0);
    for (int64_t br = 0; br < brows; br++) {
        const std::vector<int32_t> &v = bcols[br];
        std::copy(v.begin(), v.end(), colidx.begin() + br * width);
        for (int64_t r = br * block; r < std::min(M, (br + 1) * block); r++)
            for (int64_t j = A->row_ptr[r]; j < A->row_ptr[r + 1]; j++) {
                const int32_t c = A->col_idx[j];
                const int64_t slot = std::lower_bound(v.begin(), v.end(), c / block) - v.begin();
                const float x = A->val ? A->val[j] : 1.0f;
                uint16_t h;
                if (dt == TCASPMM_F16) {
                    const __half hv = __float2half_rn(x);
                    std::memcpy(&h, &hv, 2);
                } else {
                    const __nv_bfloat16 bv = __float2bfloat16_rn(x);
                    std::memcpy(&h, &bv, 2);
                }
                vals[(size_t)(r * ell_cols + slot * block + c % block)] = h;
            }
    }
    if (ell_bytes) *ell_bytes = (int64_t)(colidx.size() * 4 + vals.size() * 2);
    cudaStream_t st = (cudaStream_t)stream;
    int32_t *d_cols = nullptr;
    void *d_vals = nullptr, *d_Bp = nullptr, *buf = nullptr;
    float *d_Cp = nullptr;
    cusparseHandle_t h = nullptr;
    cusparseSpMatDescr_t Ad = nullptr;
    cusparseDnMatDescr_t Bd = nullptr, Cd = nullptr;
    const float alpha = 1.0f, beta = 0.0f;
    size_t bsz = 0;
    int rc = CUSPARSE_STATUS_SUCCESS;
    // Padded B / C when K or M is not a multiple of the block (B rows past K are zero).
    const bool padB = Kp != K, padC = Mp != M;
    if (cudaMalloc((void **)&d_cols, colidx.size() * 4) != cudaSuccess ||
        cudaMalloc(&d_vals, vals.size() * 2) != cudaSuccess ||
        (padB && cudaMalloc(&d_Bp, (size_t)(Kp * N * 2)) != cudaSuccess) ||
        (padC && cudaMalloc((void **)&d_Cp, (size_t)(Mp * N * 4)) != cudaSuccess)) {
        s = bfail(TCASPMM_ERR_ALLOC, "blocked-ELL buffers", 0);
    } else {
        cudaMemcpy(d_cols, colidx.data(), colidx.size() * 4, cudaMemcpyHostToDevice);
        cudaMemcpy(d_vals, vals.data(), vals.size() * 2, cudaMemcpyHostToDevice);
        if (padB) {
            cudaMemset(d_Bp, 0, (size_t)(Kp * N * 2));
            cudaMemcpy2D(d_Bp, N * 2, dB, ldb * 2, N * 2, K, cudaMemcpyDeviceToDevice);
        }
        if ((rc = cusparseCreate(&h)) != CUSPARSE_STATUS_SUCCESS) {
            s = bfail(TCASPMM_ERR_CUDA, "cusparseCreate", rc);
        } else {
            cusparseSetStream(h, st);
            rc = cusparseCreateBlockedEll(&Ad, Mp, Kp, block, ell_cols, d_cols, d_vals, CUSPARSE_INDEX_32I,
                                          CUSPARSE_INDEX_BASE_ZERO, cuda_type(dt));
            if (rc == CUSPARSE_STATUS_SUCCESS)
                rc = cusparseCreateDnMat(&Bd, Kp, N, padB ? N : ldb, padB ? d_Bp : (void *)dB, cuda_type(dt),
                                         CUSPARSE_ORDER_ROW);
            if (rc == CUSPARSE_STATUS_SUCCESS)
                rc = cusparseCreateDnMat(&Cd, Mp, N, padC ? N : ldc, padC ? d_Cp : dC, CUDA_R_32F, CUSPARSE_ORDER_ROW);
            if (rc == CUSPARSE_STATUS_SUCCESS)
                rc = cusparseSpMM_bufferSize(h, CUSPARSE_OPERATION_NON_TRANSPOSE, CUSPARSE_OPERATION_NON_TRANSPOSE,
                                             &alpha, Ad, Bd, &beta, Cd, CUDA_R_32F, CUSPARSE_SPMM_ALG_DEFAULT, &bsz);
            if (rc != CUSPARSE_STATUS_SUCCESS) {
                s = bfail(TCASPMM_ERR_CUDA, "cusparse blocked-ELL setup", rc);
            } else if (bsz && cudaMalloc(&buf, bsz) != cudaSuccess) {
                s = bfail(TCASPMM_ERR_ALLOC, "cusparse workspace", 0);
            } else {
                auto run = [&]() {
                    return cusparseSpMM(h, CUSPARSE_OPERATION_NON_TRANSPOSE, CUSPARSE_OPERATION_NON_TRANSPOSE, &alpha,
                                        Ad, Bd, &beta, Cd, CUDA_R_32F, CUSPARSE_SPMM_ALG_DEFAULT,
                                        buf) == CUSPARSE_STATUS_SUCCESS;
                };
                s = time_loop(run, warmup, iters, st, ms_per_iter);
                if (s == TCASPMM_OK && padC)
                    cudaMemcpy2DAsync(dC, ldc * 4, d_Cp, N * 4, N * 4, M, cudaMemcpyDeviceToDevice, st);
                cudaStreamSynchronize(st);
            }
        }
    }
    if (Cd) cusparseDestroyDnMat(Cd);
    if (Bd) cusparseDestroyDnMat(Bd);
    if (Ad) cusparseDestroySpMat(Ad);
    if (h) cusparseDestroy(h);
    for (void *q : {(void *)d_cols, d_vals, d_Bp, (void *)d_Cp, buf})
        if (q) cudaFree(q);
    return s;
}
