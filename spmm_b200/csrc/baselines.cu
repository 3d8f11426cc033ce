// cuSPARSE and cuBLAS baselines (libtcaspmm_baselines.so).  Reported next to
// tcaspmm, never called by it.
#include <cstdio>

#include <cublas_v2.h>
#include <cuda_runtime.h>
#include <cusparse.h>

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
    return dt == TCASPMM_F32 ? CUDA_R_32F : dt == TCASPMM_F16 ? CUDA_R_16F : CUDA_R_16BF;
}

template <typename F>
tcaspmm_status time_loop(F &&f, int warmup, int iters, cudaStream_t st, double *ms)
{
    for (int i = 0; i < warmup; i++)
        if (!f()) return bfail(TCASPMM_ERR_CUDA, "baseline warm-up", 0);
    cudaEvent_t a, b;
    cudaEventCreate(&a);
    cudaEventCreate(&b);
    cudaEventRecord(a, st);
    bool ok = true;
    for (int i = 0; i < iters && ok; i++) ok = f();
    cudaEventRecord(b, st);
    cudaEventSynchronize(b);
    float t = 0.0f;
    cudaEventElapsedTime(&t, a, b);
    cudaEventDestroy(a);
    cudaEventDestroy(b);
    cudaError_t e = cudaGetLastError();
    if (!ok || e != cudaSuccess) return bfail(TCASPMM_ERR_CUDA, "baseline timed loop", (int)e);
    *ms = iters > 0 ? t / iters : 0.0;
    return TCASPMM_OK;
}

}  // namespace

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
