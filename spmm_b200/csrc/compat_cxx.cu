// C++-linkage twin of our_spmm_balanced, so an unmodified C++ caller compiled
// against the reference header (src/our_spmm.cuh:4, which declares
// `void our_spmm_balanced(CSR *, half *, float *, int, int, int, int, double *)`
// without extern "C") links against this library as-is.
#include <cuda_fp16.h>

#include "tcaspmm.h"

// Layout of the reference's struct CSR (src/general.cuh:125-134).
typedef struct CSR {
    int nRow;
    int nCol;
    int nnz;
    int *row_offset;
    int *col_idx;
    half *value;
} CSR;

static_assert(sizeof(CSR) == sizeof(tcaspmm_ref_csr), "CSR layout twin");

void our_spmm_balanced(CSR *A_csr, half *B, float *C, const int M, const int N, const int K, int n_iter,
                       double *elapsed)
{
    ::our_spmm_balanced(reinterpret_cast<tcaspmm_ref_csr *>(A_csr), reinterpret_cast<uint16_t *>(B), C, M, N, K,
                        n_iter, elapsed);
}
