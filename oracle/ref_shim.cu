// C-ABI shim over the reference's own host code, compiled from the reference
// sources where they lie (oracle/Makefile target `ref`, output in oracle/_ref/).
//
// TEST INFRASTRUCTURE ONLY: used by tests/golden/make_golden.py to produce the
// golden fixtures that pin oracle/oracle.c and the product's .smtx reader.
// Nothing here runs device code; the wrapped functions are host-only:
//   smtx_input_to_Dense   src/file_input.cu:135-193
//   convert_dense_to_csr  src/miscalleneous.cu:29-65
//   naive_gemm            src/miscalleneous.cu:114-134
//   mtx_input_to_CSR      src/file_input.cu:64-134
#include <cstdint>
#include <cstdlib>
#include <cstring>
#include <fstream>

#include "file_input.cuh"

extern "C" {

// Load a .smtx file with the reference loader (dense half, 1.0 per nonzero),
// then convert it with the reference's dense->CSR routine.  Arrays are
// malloc'd; release them with ref_free.
int ref_smtx_to_csr(const char *path, int *M, int *K, int *nnz_header, int *nnz_csr,
                    int **row_ptr, int **col, uint16_t **val)
{
    std::ifstream fin;
    fin.open(path, std::ifstream::in);
    if (!fin.is_open()) return -1;
    half *dense = nullptr;
    smtx_input_to_Dense(fin, &dense, const_cast<char *>(path), M, K, nnz_header);
    CSR *csr = nullptr;
    convert_dense_to_csr(dense, &csr, *M, *K);
    free(dense);
    *nnz_csr = csr->nnz;
    *row_ptr = csr->row_offset;
    *col = csr->col_idx;
    *val = reinterpret_cast<uint16_t *>(csr->value);
    free(csr);
    return 0;
}

// Dense M x K half matrix -> CSR with the reference routine.
int ref_dense_to_csr(const uint16_t *dense, int M, int K, int *nnz, int **row_ptr, int **col,
                     uint16_t **val)
{
    CSR *csr = nullptr;
    convert_dense_to_csr(reinterpret_cast<half *>(const_cast<uint16_t *>(dense)), &csr, M, K);
    *nnz = csr->nnz;
    *row_ptr = csr->row_offset;
    *col = csr->col_idx;
    *val = reinterpret_cast<uint16_t *>(csr->value);
    free(csr);
    return 0;
}

// The reference's only CPU product of A and B: dense fp16 x fp16 -> fp32.
void ref_naive_gemm(const uint16_t *A, const uint16_t *B, float *C, int M, int N, int K)
{
    naive_gemm(reinterpret_cast<half *>(const_cast<uint16_t *>(A)),
               reinterpret_cast<half *>(const_cast<uint16_t *>(B)), C, M, N, K);
}

void ref_free(void *p) { free(p); }

}  // extern "C"
