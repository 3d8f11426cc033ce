// tcaspmm_spmm_csr_noalloc: C = A * B from caller-owned device buffers, with no
// device allocation at all.
//
// Who needs this: code that may not call cudaMalloc / cudaFree (or any routine
// that allocates) at the moment it multiplies -- for example a plugin that runs
// inside a host framework which owns every device allocation, a latency-critical
// loop where an allocation could block or fragment a memory pool, or a caller
// that already holds its inputs and outputs and must not grow its footprint.
// The plan API (tcaspmm_plan_create) allocates device buffers for A's schedule
// and its scratch; this entry point takes A in CSR straight from the caller's
// device memory and keeps its only scratch in a fixed array that is part of the
// library image.
//
// How it works: the nonzeros are cut into equal chunks, one warp per chunk
// (a merge-path split, so no host preprocessing is needed).  A warp writes every
// C row that ends inside its chunk; a row that crosses chunk boundaries leaves
// one partial row per chunk it touches in the scratch array, and a second
// kernel adds those partials in chunk order and writes the row, so the result
// does not depend on timing.
//
// The scratch array g_noalloc_carry below (NOALLOC_SCRATCH_BYTES) is held by
// every GPU that loads this library, until the process exits; each device has
// its own copy.  All calls on one device share that copy: calls whose kernels
// overlap on the GPU (different streams or host threads) race on it and must be
// serialised by the caller.  Every scratch slot a call reads is written earlier
// in the same call, so no part of it has to start at zero, and leftovers of an
// earlier call are never read.  The first call on each device looks up the
// array's device address (cudaGetSymbolAddress) with that device current.
// Under lazy module loading (the CUDA default since 12.2) that first call is
// also when the driver loads this library's device code and commits the array
// on the device, so it can fail with out-of-memory; callers make one warm-up
// call per device at initialisation, before any stream capture and before
// their memory budget is fixed.
#include <algorithm>
#include <climits>
#include <cstdint>
#include <mutex>

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include "internal.h"
#include "residue.cuh"

namespace tca {
namespace {

constexpr int64_t NOALLOC_SCRATCH_BYTES = 16ll << 20;  // 16 MiB per device
constexpr int64_t NOALLOC_SCRATCH_FLOATS = NOALLOC_SCRATCH_BYTES / 4;
constexpr int64_t NOALLOC_MIN_CHUNK = 256;              // nonzeros per warp, at least
constexpr int NOALLOC_MAX_DEVICES = 64;
// Nonzero indices are 32-bit in the kernels; the chunk loop reads up to 8 past
// a chunk start, so nnz stays this far below 2^31.
constexpr int64_t NOALLOC_MAX_NNZ = (int64_t)INT32_MAX - 64;

// Two partial rows per chunk: [chunk][0] = the chunk's piece of a row that began
// in an earlier chunk, [chunk][1] = the piece of a row that continues past it.
static __device__ __align__(256) float g_noalloc_carry[NOALLOC_SCRATCH_FLOATS];

struct NoallocParams {
    const int32_t *row_ptr;
    const int32_t *col;
    const void *val;
    const void *B;
    long long ldb;
    float *C;
    long long ldc;
    int M;
    int nnz;
    int ncols;
    int chunk;     // nonzeros per warp
    int nchunks;
    int cstride;   // floats per carry row (ncols rounded up to 4)
    float *carry;  // device address of g_noalloc_carry
};

// Last row r in [0, M) with row_ptr[r] <= j (rows are empty-tolerant).
__device__ __forceinline__ int row_of(const int32_t *row_ptr, int M, int j)
{
    int lo = 0, hi = M - 1;
    while (lo < hi) {
        const int mid = (lo + hi + 1) >> 1;
        if (__ldg(row_ptr + mid) <= j)
            lo = mid;
        else
            hi = mid - 1;
    }
    return lo;
}

template <int VEC>
__device__ __forceinline__ void zero_acc(float (&a)[VEC])
{
#pragma unroll
    for (int k = 0; k < VEC; ++k) a[k] = 0.0f;
}

// Kernel 1: warp w streams nonzeros [w*chunk, min((w+1)*chunk, nnz)).
// It writes every row whose end lies in (j0, j1] -- and, for chunk 0, the
// leading empty rows -- unless the row began before j0, in which case its
// piece goes to carry[w][0].  The row still open at j1 goes to carry[w][0]
// when it began before j0 (the chunk is inside it) and to carry[w][1] otherwise.
template <typename T, int VEC>
__global__ void __launch_bounds__(256) noalloc_chunks(const NoallocParams p)
{
    const int w = (int)((blockIdx.x * blockDim.x + threadIdx.x) >> 5);
    const int lane = threadIdx.x & 31;
    if (w >= p.nchunks) return;
    const int j0 = w * p.chunk;  // < nnz
    const int j1 = (int)min((long long)j0 + p.chunk, (long long)p.nnz);
    const int r0 = w == 0 ? 0 : row_of(p.row_ptr, p.M, j0);
    const bool head_split = __ldg(p.row_ptr + r0) < j0;
    const T *__restrict__ val = static_cast<const T *>(p.val);
    constexpr int CPP = 32 * VEC;
    for (int c0 = lane * VEC; c0 < p.ncols; c0 += CPP) {
        const T *__restrict__ B = static_cast<const T *>(p.B) + c0;
        int r = r0;
        int e = __ldg(p.row_ptr + r + 1);
        float acc[VEC];
        zero_acc(acc);
        auto finish_row = [&](bool complete) {
            float *dst;
            if (r == r0 && head_split)
                dst = p.carry + ((long long)w * 2 + 0) * p.cstride + c0;
            else if (complete)
                dst = p.C + (long long)r * p.ldc + c0;
            else
                dst = p.carry + ((long long)w * 2 + 1) * p.cstride + c0;
            if (complete && !(r == r0 && head_split))
                store_c<VEC>(dst, acc);
            else
                store_l2<VEC>(dst, acc);
        };
        for (int j = j0; j < j1; j += 8) {
            int cc[8];
            float vv[8];
#pragma unroll
            for (int u = 0; u < 8; ++u) {
                const bool ok = j + u < j1;
                cc[u] = ok ? __ldg(p.col + j + u) : 0;
                vv[u] = ok ? to_f<T>(__ldg(val + j + u)) : 0.0f;
            }
            Raw<T, VEC> rb[8];
#pragma unroll
            for (int u = 0; u < 8; ++u) {
                if (j + u < j1)
                    load_raw<T, VEC>(B + (long long)cc[u] * p.ldb, rb[u]);
                else
                    zero_raw<T, VEC>(rb[u]);
            }
#pragma unroll
            for (int u = 0; u < 8; ++u) {
                if (j + u < j1) {
                    while (j + u >= e) {  // row r ends before this nonzero
                        finish_row(true);
                        zero_acc(acc);
                        ++r;
                        e = __ldg(p.row_ptr + r + 1);
                    }
                    fma_raw<T, VEC>(vv[u], rb[u], acc);
                }
            }
        }
        // Close row r and every following row that ends at or before j1 (this
        // writes trailing empty rows); the row still open past j1 is a carry.
        for (;;) {
            if (r >= p.M) break;
            if (e > j1) {
                finish_row(false);
                break;
            }
            finish_row(true);
            zero_acc(acc);
            ++r;
            if (r >= p.M) break;
            e = __ldg(p.row_ptr + r + 1);
        }
    }
}

// Kernel 2: one warp per chunk w whose first row began in an earlier chunk and
// ends inside chunk w.  Row total = carry[a][1] + sum_{c=a+1..w} carry[c][0],
// a = the chunk holding the row's first nonzero, added in chunk order.
template <int VEC>
__global__ void __launch_bounds__(256) noalloc_fixup(const NoallocParams p)
{
    const int w = (int)((blockIdx.x * blockDim.x + threadIdx.x) >> 5);
    const int lane = threadIdx.x & 31;
    if (w == 0 || w >= p.nchunks) return;
    const int j0 = w * p.chunk;  // < nnz
    const int j1 = (int)min((long long)j0 + p.chunk, (long long)p.nnz);
    const int r0 = row_of(p.row_ptr, p.M, j0);
    const int b = __ldg(p.row_ptr + r0), e = __ldg(p.row_ptr + r0 + 1);
    if (!(b < j0 && e <= j1)) return;
    const int a = b / p.chunk;
    constexpr int CPP = 32 * VEC;
    for (int c0 = lane * VEC; c0 < p.ncols; c0 += CPP) {
        float acc[VEC];
        zero_acc(acc);
        add_l2<VEC>(p.carry + ((long long)a * 2 + 1) * p.cstride + c0, acc);
        for (int c = a + 1; c <= w; ++c) add_l2<VEC>(p.carry + ((long long)c * 2 + 0) * p.cstride + c0, acc);
        store_c<VEC>(p.C + (long long)r0 * p.ldc + c0, acc);
    }
}

template <typename T, int VEC>
void launch(const NoallocParams &p, cudaStream_t st)
{
    const int blocks = (p.nchunks + 7) / 8;
    noalloc_chunks<T, VEC><<<blocks, 256, 0, st>>>(p);
    noalloc_fixup<VEC><<<blocks, 256, 0, st>>>(p);
}

template <typename T>
void launch_t(bool vec, const NoallocParams &p, cudaStream_t st)
{
    if (vec)
        launch<T, 16 / sizeof(T)>(p, st);
    else
        launch<T, 1>(p, st);
}

// Zero C when A has no nonzeros (every row is empty).
__global__ void noalloc_zero(float *C, long long ldc, int M, int ncols)
{
    const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (i < (long long)M * ncols) C[(i / ncols) * ldc + i % ncols] = 0.0f;
}

std::mutex g_mu;
float *g_carry_ptr[NOALLOC_MAX_DEVICES] = {};

// Device address of the scratch array on `dev` (looked up once per device, with
// that device current).
tcaspmm_status scratch_address(int dev, float **out)
{
    if (dev < 0 || dev >= NOALLOC_MAX_DEVICES) return fail(TCASPMM_ERR_UNSUPPORTED, "device %d out of range", dev);
    std::lock_guard<std::mutex> lk(g_mu);
    if (!g_carry_ptr[dev]) {
        void *ptr = nullptr;
        cudaError_t e = cudaGetSymbolAddress(&ptr, g_noalloc_carry);
        if (e != cudaSuccess)
            return fail(TCASPMM_ERR_CUDA, "cudaGetSymbolAddress(scratch) on device %d: %s", dev, cudaGetErrorString(e));
        g_carry_ptr[dev] = (float *)ptr;
    }
    *out = g_carry_ptr[dev];
    return TCASPMM_OK;
}

}  // namespace
}  // namespace tca

using namespace tca;

extern "C" tcaspmm_status tcaspmm_spmm_csr_noalloc(const int32_t *d_row_ptr, const int32_t *d_col, const void *d_val,
                                                   int64_t M, int64_t K, int64_t nnz, const void *dB, int64_t ldb,
                                                   float *dC, int64_t ldc, int64_t N, tcaspmm_dtype dt, void *stream)
{
    clear_error();
    if (!dtype_valid(dt)) return fail(TCASPMM_ERR_INVALID_ARG, "spmm_csr_noalloc: unknown dtype %d", (int)dt);
    if (M < 0 || K < 0 || nnz < 0 || N < 0 || ldb < N || ldc < N)
        return fail(TCASPMM_ERR_INVALID_ARG, "spmm_csr_noalloc: bad sizes M=%lld K=%lld nnz=%lld N=%lld ldb=%lld ldc=%lld",
                    (long long)M, (long long)K, (long long)nnz, (long long)N, (long long)ldb, (long long)ldc);
    if (M > INT32_MAX - 1 || nnz > NOALLOC_MAX_NNZ || N > INT32_MAX)
        return fail(TCASPMM_ERR_UNSUPPORTED, "spmm_csr_noalloc: M and N must be below 2^31 and nnz at most %lld",
                    (long long)NOALLOC_MAX_NNZ);
    const int64_t cstride = (N + 3) / 4 * 4;
    // Two carry rows per chunk must fit in the fixed scratch.
    const int64_t max_chunks = NOALLOC_SCRATCH_FLOATS / std::max<int64_t>(1, 2 * cstride);
    if (max_chunks < 1)
        return fail(TCASPMM_ERR_UNSUPPORTED,
                    "spmm_csr_noalloc: N=%lld needs %lld bytes of scratch per chunk; the fixed scratch holds %lld bytes "
                    "(N <= %lld)",
                    (long long)N, (long long)(2 * cstride * 4), (long long)NOALLOC_SCRATCH_BYTES,
                    (long long)(NOALLOC_SCRATCH_FLOATS / 2));
    if (M == 0 || N == 0) return TCASPMM_OK;
    if (!d_row_ptr || !dC || (nnz > 0 && (!d_col || !d_val || !dB)))
        return fail(TCASPMM_ERR_INVALID_ARG, "spmm_csr_noalloc: NULL device pointer");
    cudaStream_t st = (cudaStream_t)stream;
    int dev = 0;
    cudaError_t ce = cudaGetDevice(&dev);
    if (ce != cudaSuccess) return fail(TCASPMM_ERR_CUDA, "cudaGetDevice: %s", cudaGetErrorString(ce));
    if (nnz == 0) {
        const long long n = M * N;
        noalloc_zero<<<(unsigned)((n + 255) / 256), 256, 0, st>>>(dC, ldc, (int)M, (int)N);
        ce = cudaGetLastError();
        return ce == cudaSuccess ? TCASPMM_OK : fail(TCASPMM_ERR_CUDA, "zero kernel: %s", cudaGetErrorString(ce));
    }
    float *carry = nullptr;
    tcaspmm_status s = scratch_address(dev, &carry);
    if (s != TCASPMM_OK) return s;
    int64_t chunk = std::max<int64_t>(NOALLOC_MIN_CHUNK, (nnz + max_chunks - 1) / max_chunks);
    NoallocParams p;
    p.row_ptr = d_row_ptr;
    p.col = d_col;
    p.val = d_val;
    p.B = dB;
    p.ldb = ldb;
    p.C = dC;
    p.ldc = ldc;
    p.M = (int)M;
    p.nnz = (int)nnz;
    p.ncols = (int)N;
    p.chunk = (int)chunk;
    p.nchunks = (int)((nnz + chunk - 1) / chunk);
    p.cstride = (int)cstride;
    p.carry = carry;
    const int elem = dtype_size(dt);
    const bool vec = ((uintptr_t)dB % 16 == 0) && ((ldb * elem) % 16 == 0) && ((uintptr_t)dC % 16 == 0) &&
                     (ldc % 4 == 0) && (N % (16 / elem) == 0);
    if (dtype_fp32(dt))  // TF32 plans have fp32 storage; this path computes in fp32
        launch_t<float>(vec, p, st);
    else if (dt == TCASPMM_F16)
        launch_t<__half>(vec, p, st);
    else
        launch_t<__nv_bfloat16>(vec, p, st);
    ce = cudaGetLastError();
    return ce == cudaSuccess ? TCASPMM_OK : fail(TCASPMM_ERR_CUDA, "spmm_csr_noalloc launch: %s", cudaGetErrorString(ce));
}
