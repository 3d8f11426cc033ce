// Errors, dtype conversion, random streams and host CSR helpers.
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <cstring>

#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include "internal.h"

namespace tca {

static thread_local std::string g_last_error;

tcaspmm_status fail(tcaspmm_status s, const char *fmt, ...)
{
    char buf[1024];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof(buf), fmt, ap);
    va_end(ap);
    g_last_error = buf;
    return s;
}

void clear_error() { g_last_error.clear(); }

uint16_t float_to_half_bits(float f)
{
    const __half_raw r = __float2half_rn(f);
    return r.x;
}

uint16_t float_to_bf16_bits(float f)
{
    const __nv_bfloat16_raw r = __float2bfloat16_rn(f);
    return r.x;
}

float half_bits_to_float(uint16_t b)
{
    __half_raw r;
    r.x = b;
    return __half2float(__half(r));
}

// Box-Muller on two independent counter draws.  Normal streams live above
// 0x100 so they never alias the uniform streams callers use directly.
double rng_normal(uint64_t seed, uint64_t stream, uint64_t i)
{
    double u1 = rng_unit(seed, 0x100 + stream * 2 + 0, i);
    double u2 = rng_unit(seed, 0x100 + stream * 2 + 1, i);
    if (u1 < 1e-300) u1 = 1e-300;
    return std::sqrt(-2.0 * std::log(u1)) * std::cos(6.283185307179586 * u2);
}

tcaspmm_status csr_from_rows(int64_t nrow, int64_t ncol, const std::vector<int64_t> &row_ptr,
                             const std::vector<int32_t> &col, const std::vector<float> *val,
                             tcaspmm_csr *out)
{
    const int64_t nnz = (int64_t)col.size();
    tcaspmm_status s = tcaspmm_csr_alloc(nrow, ncol, nnz, val != nullptr, out);
    if (s != TCASPMM_OK) return s;
    std::memcpy(out->row_ptr, row_ptr.data(), sizeof(int64_t) * (nrow + 1));
    if (nnz) std::memcpy(out->col_idx, col.data(), sizeof(int32_t) * nnz);
    if (val && nnz) std::memcpy(out->val, val->data(), sizeof(float) * nnz);
    return TCASPMM_OK;
}

int64_t algorithmic_bytes(int64_t M, int64_t K, int64_t nnz, int64_t N, tcaspmm_dtype dt)
{
    const int64_t e = dtype_size(dt);
    return (M + 1) * 4 + nnz * (4 + e) + K * N * e + M * N * 4;
}

}  // namespace tca

using namespace tca;

extern "C" {

const char *tcaspmm_status_string(tcaspmm_status s)
{
    switch (s) {
    case TCASPMM_OK: return "ok";
    case TCASPMM_ERR_INVALID_ARG: return "invalid argument";
    case TCASPMM_ERR_IO: return "i/o error";
    case TCASPMM_ERR_FORMAT: return "malformed input";
    case TCASPMM_ERR_ALLOC: return "allocation failed";
    case TCASPMM_ERR_CUDA: return "cuda error";
    case TCASPMM_ERR_UNSUPPORTED: return "unsupported";
    case TCASPMM_ERR_TIMEOUT: return "device wait timed out";
    case TCASPMM_ERR_NO_DEVICE: return "no cuda device";
    }
    return "unknown status";
}

const char *tcaspmm_last_error(void) { return g_last_error.c_str(); }

tcaspmm_status tcaspmm_csr_alloc(int64_t nrow, int64_t ncol, int64_t nnz, int with_values,
                                 tcaspmm_csr *out)
{
    if (!out) return fail(TCASPMM_ERR_INVALID_ARG, "csr_alloc: out is NULL");
    std::memset(out, 0, sizeof(*out));
    if (nrow < 0 || ncol < 0 || nnz < 0)
        return fail(TCASPMM_ERR_INVALID_ARG, "csr_alloc: negative size (%lld, %lld, %lld)",
                    (long long)nrow, (long long)ncol, (long long)nnz);
    out->row_ptr = (int64_t *)std::calloc((size_t)nrow + 1, sizeof(int64_t));
    out->col_idx = (int32_t *)std::malloc(sizeof(int32_t) * (size_t)(nnz ? nnz : 1));
    out->val = with_values ? (float *)std::malloc(sizeof(float) * (size_t)(nnz ? nnz : 1)) : nullptr;
    if (!out->row_ptr || !out->col_idx || (with_values && !out->val)) {
        tcaspmm_csr_free(out);
        return fail(TCASPMM_ERR_ALLOC, "csr_alloc: host allocation of %lld nonzeros failed",
                    (long long)nnz);
    }
    out->nrow = nrow;
    out->ncol = ncol;
    out->nnz = nnz;
    return TCASPMM_OK;
}

tcaspmm_status tcaspmm_csr_free(tcaspmm_csr *A)
{
    if (!A) return TCASPMM_OK;
    std::free(A->row_ptr);
    std::free(A->col_idx);
    std::free(A->val);
    std::memset(A, 0, sizeof(*A));
    return TCASPMM_OK;
}

tcaspmm_status tcaspmm_csr_validate(const tcaspmm_csr *A)
{
    if (!A) return fail(TCASPMM_ERR_INVALID_ARG, "csr is NULL");
    if (A->nrow < 0 || A->ncol < 0 || A->nnz < 0)
        return fail(TCASPMM_ERR_INVALID_ARG, "csr has a negative dimension");
    if (A->nrow > INT32_MAX - 1 || A->ncol > INT32_MAX || A->nnz > INT32_MAX)
        return fail(TCASPMM_ERR_UNSUPPORTED,
                    "csr dimensions above 2^31-1 are not supported (M=%lld K=%lld nnz=%lld)",
                    (long long)A->nrow, (long long)A->ncol, (long long)A->nnz);
    if (!A->row_ptr || (A->nnz > 0 && !A->col_idx))
        return fail(TCASPMM_ERR_INVALID_ARG, "csr arrays are NULL");
    if (A->row_ptr[0] != 0 || A->row_ptr[A->nrow] != A->nnz)
        return fail(TCASPMM_ERR_FORMAT, "row_ptr[0]=%lld, row_ptr[M]=%lld, nnz=%lld",
                    (long long)A->row_ptr[0], (long long)A->row_ptr[A->nrow], (long long)A->nnz);
    for (int64_t i = 0; i < A->nrow; i++) {
        const int64_t b = A->row_ptr[i], e = A->row_ptr[i + 1];
        if (e < b) return fail(TCASPMM_ERR_FORMAT, "row_ptr decreases at row %lld", (long long)i);
        for (int64_t j = b; j < e; j++) {
            const int32_t c = A->col_idx[j];
            if (c < 0 || c >= A->ncol)
                return fail(TCASPMM_ERR_FORMAT, "column %d out of range [0, %lld) in row %lld", c,
                            (long long)A->ncol, (long long)i);
            if (j > b && c <= A->col_idx[j - 1])
                return fail(TCASPMM_ERR_FORMAT, "columns not strictly ascending in row %lld",
                            (long long)i);
        }
    }
    return TCASPMM_OK;
}

tcaspmm_status tcaspmm_dense_to_csr(const uint16_t *dense, int64_t M, int64_t K, tcaspmm_csr *out)
{
    if (!out || (!dense && M * K > 0) || M < 0 || K < 0)
        return fail(TCASPMM_ERR_INVALID_ARG, "dense_to_csr: bad arguments");
    std::vector<int64_t> rp(M + 1, 0);
    std::vector<int32_t> col;
    std::vector<float> val;
    for (int64_t r = 0; r < M; r++) {
        for (int64_t c = 0; c < K; c++) {
            const uint16_t h = dense[r * K + c];
            // binary16 +0 and -0 both compare equal to 0.0f and are dropped,
            // as in src/miscalleneous.cu:41,51.
            if ((h & 0x7fff) != 0) {
                col.push_back((int32_t)c);
                val.push_back(half_bits_to_float(h));
            }
        }
        rp[r + 1] = (int64_t)col.size();
    }
    return csr_from_rows(M, K, rp, col, &val, out);
}

tcaspmm_status tcaspmm_partition_columns(int64_t N, tcaspmm_dtype dt, int world, int rank,
                                         int64_t *col_begin, int64_t *col_count)
{
    if (!dtype_valid(dt) || world < 1 || rank < 0 || rank >= world || N < 0 || !col_begin ||
        !col_count)
        return fail(TCASPMM_ERR_INVALID_ARG, "partition_columns: bad arguments");
    const int64_t vec = 16 / dtype_size(dt);  // elements per 16-byte vector
    int64_t block = (N + world - 1) / world;
    block = (block + vec - 1) / vec * vec;
    int64_t b = block * rank;
    if (b > N) b = N;
    int64_t e = b + block;
    if (e > N) e = N;
    *col_begin = b;
    *col_count = e - b;
    return TCASPMM_OK;
}

tcaspmm_status tcaspmm_partition_rows(const tcaspmm_csr *A, int parts, int64_t *row_begin)
{
    if (!A || parts < 1 || !row_begin) return fail(TCASPMM_ERR_INVALID_ARG, "partition_rows: bad arguments");
    tcaspmm_status s = tcaspmm_csr_validate(A);
    if (s != TCASPMM_OK) return s;
    // Cost of rows [0, r) = row_ptr[r] + 2 r; block i starts at the first row
    // whose prefix cost reaches i / parts of the total.
    const int64_t M = A->nrow;
    const int64_t total = A->row_ptr[M] + 2 * M;
    row_begin[0] = 0;
    int64_t r = 0;
    for (int i = 1; i < parts; i++) {
        const int64_t target = (int64_t)((__int128)total * i / parts);
        while (r < M && A->row_ptr[r] + 2 * r < target) r++;
        row_begin[i] = r;
    }
    row_begin[parts] = M;
    return TCASPMM_OK;
}

}  // extern "C"
