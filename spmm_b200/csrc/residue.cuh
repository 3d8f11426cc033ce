// CUDA-core residue kernel: C rows that are not covered by tensor-core windows.
//
// Replaces the short-row / long-row paths of kernel_our_spmm_balanced
// (multirow_per_tb src/our_spmm.cu:24-160, multitb_per_row :161-295), which
// push each nonzero through a 1/8-useful mma.sync.m16n8k8 after a shared-memory
// transpose.  Here a nonzero is one 16-byte B load per lane and VEC fp32 FMAs:
//   * a lane group of G lanes (power of two) covers G*VEC columns of one B row
//     with 16-byte loads (VEC = 4 fp32 or 8 fp16/bf16); a warp holds P = 32/G
//     groups, and columns beyond G*VEC are covered by extra passes;
//   * row warps: each group streams the nonzeros of its contiguous share of a
//     row range in chunks of U (U independent B loads in flight per lane,
//     however short the rows) and writes each finished C row with streaming
//     16-byte stores as the stream passes the row's end;
//   * segment warps: the P groups split one segment of a long row, reduce with
//     __shfl_xor_sync, and store a partial row; the warp that completes a long
//     row's last segment (atomic counter) sums all its partials in segment
//     order and writes C, so the result does not depend on timing.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cstdint>
#include <type_traits>

namespace tca {

// Fused output epilogue, applied where a C element is written:
//   C[r][c] = relu?( row_scale[r] * (A B)[r][c] + bias[c] )  stored as fp32, fp16 or bf16.
// row_scale / bias are device arrays (NULL = 1 / 0); c is the column within the
// launch's column block.
struct EpiParams {
    const float *__restrict__ row_scale;
    const float *__restrict__ bias;
    int relu;
    int out;  // 0 fp32, 1 fp16, 2 bf16
};

struct ResidueParams {
    const int32_t *__restrict__ row_ptr;
    const int32_t *__restrict__ col;
    const void *__restrict__ val;
    const void *__restrict__ B;
    long long ldb;
    float *__restrict__ C;
    long long ldc;
    int ncols;
    const int2 *__restrict__ ranges;
    int n_ranges;
    const int4 *__restrict__ segs;   // {row, begin, end, long id}
    int n_segs;
    const int4 *__restrict__ longs;  // {row, first seg, number of segs, 0}
    float *partials;                 // n_segs x pstride
    int pstride;
    unsigned int *counters;          // one per long row, zero between launches
    EpiParams ep;                    // used by the EPI instantiations only
};

template <typename T> __device__ __forceinline__ float to_f(T x);
template <> __device__ __forceinline__ float to_f<float>(float x) { return x; }
template <> __device__ __forceinline__ float to_f<__half>(__half x) { return __half2float(x); }
template <> __device__ __forceinline__ float to_f<__nv_bfloat16>(__nv_bfloat16 x) { return __bfloat162float(x); }

// Raw 16-byte (or one-element) load of a B row slice, converted at FMA time.
template <typename T, int VEC> struct Raw { uint4 u; };
template <typename T> struct Raw<T, 1> { T s; };

template <typename T, int VEC>
__device__ __forceinline__ void load_raw(const T *p, Raw<T, VEC> &r)
{
    if constexpr (VEC == 1)
        r.s = __ldg(p);
    else
        r.u = __ldg(reinterpret_cast<const uint4 *>(p));
}

// Start of B row `c` at this lane's columns: Bb points at the lane's first
// column of row 0 and `pitch` is the row pitch in bytes (< 2^32, checked on the
// host), so the address is one 32 x 32 -> 64-bit multiply-add.
template <typename T>
__device__ __forceinline__ const T *brow(const char *Bb, int c, unsigned pitch)
{
    return reinterpret_cast<const T *>(Bb + (unsigned long long)(unsigned)c * pitch);
}

template <typename T, int VEC>
__device__ __forceinline__ void zero_raw(Raw<T, VEC> &r)
{
    if constexpr (VEC == 1)
        r.s = T(0.0f);
    else
        r.u = make_uint4(0u, 0u, 0u, 0u);
}

template <typename T, int VEC>
__device__ __forceinline__ void fma_raw(float v, const Raw<T, VEC> &r, float (&acc)[VEC])
{
    if constexpr (VEC == 1) {
        acc[0] = fmaf(v, to_f<T>(r.s), acc[0]);
    } else if constexpr (sizeof(T) == 4) {
        const float *f = reinterpret_cast<const float *>(&r.u);
#pragma unroll
        for (int k = 0; k < VEC; ++k) acc[k] = fmaf(v, f[k], acc[k]);
    } else if constexpr (std::is_same<T, __half>::value) {
        const __half2 *h = reinterpret_cast<const __half2 *>(&r.u);
#pragma unroll
        for (int k = 0; k < VEC / 2; ++k) {
            const float2 f = __half22float2(h[k]);
            acc[2 * k] = fmaf(v, f.x, acc[2 * k]);
            acc[2 * k + 1] = fmaf(v, f.y, acc[2 * k + 1]);
        }
    } else {
        const __nv_bfloat162 *h = reinterpret_cast<const __nv_bfloat162 *>(&r.u);
#pragma unroll
        for (int k = 0; k < VEC / 2; ++k) {
            const float2 f = __bfloat1622float2(h[k]);
            acc[2 * k] = fmaf(v, f.x, acc[2 * k]);
            acc[2 * k + 1] = fmaf(v, f.y, acc[2 * k + 1]);
        }
    }
}

// Streaming (evict-first) store of VEC fp32 results: C is written once and
// should not push B rows out of L2.
template <int VEC>
__device__ __forceinline__ void store_c(float *c, const float (&a)[VEC])
{
    if constexpr (VEC == 1) {
        __stcs(c, a[0]);
    } else {
#pragma unroll
        for (int k = 0; k < VEC; k += 4)
            __stcs(reinterpret_cast<float4 *>(c + k), make_float4(a[k], a[k + 1], a[k + 2], a[k + 3]));
    }
}

template <int VEC>
__device__ __forceinline__ void store_l2(float *c, const float (&a)[VEC])
{
    if constexpr (VEC == 1) {
        __stcg(c, a[0]);
    } else {
#pragma unroll
        for (int k = 0; k < VEC; k += 4)
            __stcg(reinterpret_cast<float4 *>(c + k), make_float4(a[k], a[k + 1], a[k + 2], a[k + 3]));
    }
}

template <int VEC>
__device__ __forceinline__ void add_l2(const float *c, float (&a)[VEC])
{
    if constexpr (VEC == 1) {
        a[0] += __ldcg(c);
    } else {
#pragma unroll
        for (int k = 0; k < VEC; k += 4) {
            const float4 x = __ldcg(reinterpret_cast<const float4 *>(c + k));
            a[k] += x.x;
            a[k + 1] += x.y;
            a[k + 2] += x.z;
            a[k + 3] += x.w;
        }
    }
}

// Epilogue operands held in registers by a lane while it streams rows: the
// bias of its VEC columns (loaded once per pass) and the scale of the current
// row (loaded when the row starts, so the store at the row's end does not wait
// on a load).  Empty without the epilogue.
template <int VEC, bool EPI> struct EpiRegs {
    __device__ __forceinline__ void load_bias(const ResidueParams &, int) {}
    __device__ __forceinline__ void load_scale(const ResidueParams &, long long) {}
};
template <int VEC> struct EpiRegs<VEC, true> {
    float bias[VEC];
    float scale;
    __device__ __forceinline__ void load_bias(const ResidueParams &p, int c0)
    {
#pragma unroll
        for (int k = 0; k < VEC; ++k) bias[k] = p.ep.bias ? __ldg(p.ep.bias + c0 + k) : 0.0f;
    }
    __device__ __forceinline__ void load_scale(const ResidueParams &p, long long r)
    {
        scale = p.ep.row_scale ? __ldg(p.ep.row_scale + r) : 1.0f;
    }
};

// Epilogue then store of VEC outputs of row r at column c0 of the block.
template <int VEC>
__device__ __forceinline__ void store_epi(const ResidueParams &p, long long r, int c0, float (&a)[VEC],
                                          const EpiRegs<VEC, true> &er)
{
    const EpiParams &ep = p.ep;
#pragma unroll
    for (int k = 0; k < VEC; ++k) {
        const float x = fmaf(a[k], er.scale, er.bias[k]);
        a[k] = ep.relu ? fmaxf(x, 0.0f) : x;
    }
    if (ep.out == 0) {
        store_c<VEC>(p.C + r * p.ldc + c0, a);
        return;
    }
    // 16-bit outputs: VEC = 1 one element, 4 -> 8 bytes, 8 -> 16 bytes.
    uint16_t *c = reinterpret_cast<uint16_t *>(p.C) + r * p.ldc + c0;
    if constexpr (VEC == 1) {
        *c = ep.out == 1 ? __half_as_ushort(__float2half_rn(a[0])) : __bfloat16_as_ushort(__float2bfloat16_rn(a[0]));
    } else {
        uint32_t h[VEC / 2];
#pragma unroll
        for (int k = 0; k < VEC / 2; ++k) {
            if (ep.out == 1) {
                const __half2 v = __floats2half2_rn(a[2 * k], a[2 * k + 1]);
                h[k] = *reinterpret_cast<const uint32_t *>(&v);
            } else {
                const __nv_bfloat162 v = __floats2bfloat162_rn(a[2 * k], a[2 * k + 1]);
                h[k] = *reinterpret_cast<const uint32_t *>(&v);
            }
        }
        if constexpr (VEC == 4)
            __stcs(reinterpret_cast<uint2 *>(c), make_uint2(h[0], h[1]));
        else
            __stcs(reinterpret_cast<uint4 *>(c), make_uint4(h[0], h[1], h[2], h[3]));
    }
}

// The store of a finished output slice: plain fp32, or through the epilogue.
template <int VEC, bool EPI>
__device__ __forceinline__ void emit(const ResidueParams &p, long long r, int c0, float (&a)[VEC],
                                     const EpiRegs<VEC, EPI> &er)
{
    if constexpr (EPI)
        store_epi<VEC>(p, r, c0, a, er);
    else
        store_c<VEC>(p.C + r * p.ldc + c0, a);
}

// acc += sum_{j in [b, e)} val[j] * B[col[j]][c0 .. c0+VEC): full chunks of U
// without predicates (U indices, U independent B loads, U FMAs), then the
// remainder one nonzero at a time.
template <typename T, int VEC, int U, bool PF = false>
__device__ __forceinline__ void accumulate_lean(const ResidueParams &p, int b, const int e, int c0, float (&acc)[VEC])
{
    const char *Bb = reinterpret_cast<const char *>(static_cast<const T *>(p.B) + c0);
    const unsigned pitch = (unsigned)(p.ldb * (long long)sizeof(T));
    const T *__restrict__ val = static_cast<const T *>(p.val);
    int cn[U];  // PF: columns of the next full chunk, loaded one chunk ahead
    if constexpr (PF) {
        if (b + U <= e)
#pragma unroll
            for (int u = 0; u < U; ++u) cn[u] = __ldg(p.col + b + u);
    }
    for (; b + U <= e; b += U) {
        int cc[U];
        float vv[U];
#pragma unroll
        for (int u = 0; u < U; ++u) {
            cc[u] = PF ? cn[u] : __ldg(p.col + b + u);
            vv[u] = to_f<T>(__ldg(val + b + u));
        }
        Raw<T, VEC> rb[U];
#pragma unroll
        for (int u = 0; u < U; ++u) load_raw<T, VEC>(brow<T>(Bb, cc[u], pitch), rb[u]);
        if constexpr (PF) {
            if (b + 2 * U <= e)
#pragma unroll
                for (int u = 0; u < U; ++u) cn[u] = __ldg(p.col + b + U + u);
        }
#pragma unroll
        for (int u = 0; u < U; ++u) fma_raw<T, VEC>(vv[u], rb[u], acc);
    }
    for (; b < e; ++b) {
        Raw<T, VEC> rb;
        const float v = to_f<T>(__ldg(val + b));
        load_raw<T, VEC>(brow<T>(Bb, __ldg(p.col + b), pitch), rb);
        fma_raw<T, VEC>(v, rb, acc);
    }
}

// Lean nonzero stream over C rows [r_lo, r_hi) for one lane: full chunks of U
// run without predicates (U indices, U B loads, U FMAs with a row-end check),
// the remainder one nonzero at a time; each row is written when the stream
// passes its end, trailing empty rows too.
template <typename T, int VEC, int U, bool EPI, bool PF = false>
__device__ __forceinline__ void stream_lean(const ResidueParams &p, int r_lo, int r_hi, int c0)
{
    if (r_lo >= r_hi) return;
    const char *Bb = reinterpret_cast<const char *>(static_cast<const T *>(p.B) + c0);
    const unsigned pitch = (unsigned)(p.ldb * (long long)sizeof(T));
    const T *__restrict__ val = static_cast<const T *>(p.val);
    int r = r_lo;
    int e = __ldg(p.row_ptr + r + 1);
    // PF: end of the next row, loaded one row ahead, so passing a row end does
    // not wait on a row-offset load.
    int e_next = 0;
    if constexpr (PF) e_next = r + 1 < r_hi ? __ldg(p.row_ptr + r + 2) : 0;
    int j = __ldg(p.row_ptr + r_lo);
    const int jend = __ldg(p.row_ptr + r_hi);
    EpiRegs<VEC, EPI> er;
    er.load_bias(p, c0);
    er.load_scale(p, r);
    float acc[VEC];
#pragma unroll
    for (int k = 0; k < VEC; ++k) acc[k] = 0.0f;
    auto pass_row_ends = [&](int jj) {
        while (jj >= e) {
            emit<VEC, EPI>(p, r, c0, acc, er);
#pragma unroll
            for (int k = 0; k < VEC; ++k) acc[k] = 0.0f;
            ++r;  // < r_hi: nonzero jj < jend lies in a later row
            if constexpr (PF) {
                e = e_next;
                if (r + 1 < r_hi) e_next = __ldg(p.row_ptr + r + 2);
            } else {
                e = __ldg(p.row_ptr + r + 1);
            }
            er.load_scale(p, r);
        }
    };
    int cn[U];  // PF: columns of the next full chunk, loaded one chunk ahead
    if constexpr (PF) {
        if (j + U <= jend)
#pragma unroll
            for (int u = 0; u < U; ++u) cn[u] = __ldg(p.col + j + u);
    }
    for (; j + U <= jend; j += U) {
        int cc[U];
        float vv[U];
#pragma unroll
        for (int u = 0; u < U; ++u) {
            cc[u] = PF ? cn[u] : __ldg(p.col + j + u);
            vv[u] = to_f<T>(__ldg(val + j + u));
        }
        Raw<T, VEC> rb[U];
#pragma unroll
        for (int u = 0; u < U; ++u) load_raw<T, VEC>(brow<T>(Bb, cc[u], pitch), rb[u]);
        if constexpr (PF) {
            if (j + 2 * U <= jend)
#pragma unroll
                for (int u = 0; u < U; ++u) cn[u] = __ldg(p.col + j + U + u);
        }
        if (j + U <= e) {  // the whole chunk lies in the current row: no row-end checks
#pragma unroll
            for (int u = 0; u < U; ++u) fma_raw<T, VEC>(vv[u], rb[u], acc);
        } else {
#pragma unroll
            for (int u = 0; u < U; ++u) {
                pass_row_ends(j + u);
                fma_raw<T, VEC>(vv[u], rb[u], acc);
            }
        }
    }
    for (; j < jend; ++j) {
        Raw<T, VEC> rb;
        const float v = to_f<T>(__ldg(val + j));
        load_raw<T, VEC>(brow<T>(Bb, __ldg(p.col + j), pitch), rb);
        pass_row_ends(j);
        fma_raw<T, VEC>(v, rb, acc);
    }
    while (r < r_hi) {
        emit<VEC, EPI>(p, r, c0, acc, er);
#pragma unroll
        for (int k = 0; k < VEC; ++k) acc[k] = 0.0f;
        if (++r < r_hi) er.load_scale(p, r);
    }
}

// First row r in [lo, hi] with row_ptr[r] >= target.
__device__ __forceinline__ int first_row_at(const int32_t *row_ptr, int lo, int hi, int target)
{
    while (lo < hi) {
        const int mid = (lo + hi) >> 1;
        if (__ldg(row_ptr + mid) < target)
            lo = mid + 1;
        else
            hi = mid;
    }
    return lo;
}

// BLOCK threads (256 or 128), register budget of 64 (32 resident warps per SM):
// measured faster than 40 registers / 48 warps and than 80 / 24 on GCN, SAGE
// and the skew config, the epilogue instantiations included (at 80 registers
// they ran 25% slower on GCN for the lost occupancy).
template <typename T, int VEC, int G, int U, bool EPI, bool PF = false, int BLOCK = 256>
__global__ void __launch_bounds__(BLOCK, 1024 / BLOCK) residue_kernel(const ResidueParams p)
{
    constexpr int P = 32 / G;
    constexpr int CPP = G * VEC;  // columns per pass
    const int lane = threadIdx.x & 31;
    const int warp = (int)((blockIdx.x * blockDim.x + threadIdx.x) >> 5);
    const int sub = lane / G, gl = lane % G;
    const int npass = (p.ncols + CPP - 1) / CPP;

    if (warp < p.n_segs) {
        const int4 s = p.segs[warp];
        // Group `sub` takes a contiguous 1/P of the segment; the groups are then
        // reduced with shuffles in a fixed order.
        const int len = s.z - s.y;
        const int jb = s.y + (int)((long long)len * sub / P);
        const int je = s.y + (int)((long long)len * (sub + 1) / P);
        for (int pass = 0; pass < npass; ++pass) {
            const int c0 = pass * CPP + gl * VEC;
            float acc[VEC];
#pragma unroll
            for (int k = 0; k < VEC; ++k) acc[k] = 0.0f;
            if (c0 < p.ncols) accumulate_lean<T, VEC, U, PF>(p, jb, je, c0, acc);
#pragma unroll
            for (int off = G; off < 32; off <<= 1)
#pragma unroll
                for (int k = 0; k < VEC; ++k) acc[k] += __shfl_xor_sync(0xffffffffu, acc[k], off);
            if (sub == 0 && c0 < p.ncols) store_l2<VEC>(p.partials + (long long)warp * p.pstride + c0, acc);
        }
        // Publish the partial row, then count this segment in.
        __threadfence();
        __syncwarp();
        unsigned int prev = 0;
        if (lane == 0) prev = atomicAdd(p.counters + s.w, 1u);
        prev = __shfl_sync(0xffffffffu, prev, 0);
        const int4 L = p.longs[s.w];
        if (prev + 1 == (unsigned int)L.z) {
            // Last segment of this row: fixed-order reduction of all partials.
            __threadfence();
            for (int pass = 0; pass < npass; ++pass) {
                const int c0 = pass * CPP + gl * VEC;
                float acc[VEC];
#pragma unroll
                for (int k = 0; k < VEC; ++k) acc[k] = 0.0f;
                if (c0 < p.ncols)
                    for (int q = L.y + sub; q < L.y + L.z; q += P)
                        add_l2<VEC>(p.partials + (long long)q * p.pstride + c0, acc);
#pragma unroll
                for (int off = G; off < 32; off <<= 1)
#pragma unroll
                    for (int k = 0; k < VEC; ++k) acc[k] += __shfl_xor_sync(0xffffffffu, acc[k], off);
                if (sub == 0 && c0 < p.ncols) {
                    EpiRegs<VEC, EPI> er;
                    er.load_bias(p, c0);
                    er.load_scale(p, L.x);
                    emit<VEC, EPI>(p, L.x, c0, acc, er);
                }
            }
            if (lane == 0) p.counters[s.w] = 0u;  // ready for the next launch
        }
        return;
    }

    const int w = warp - p.n_segs;
    if (w >= p.n_ranges) return;
    // Row range: contiguous rows, none of them long.  Group `sub` streams the
    // nonzeros of its contiguous share of the rows, U loads in flight whatever
    // the row lengths, and flushes each C row when the stream passes its end
    // (empty rows are written as zeros).
    const int2 rg = p.ranges[w];
    int r_lo = rg.x, r_hi = rg.y;
    if constexpr (P > 1) {
        // Split the range between the P groups by nonzeros (binary search on
        // the row offsets); each group gets a contiguous run of rows.
        const int jb = __ldg(p.row_ptr + rg.x), je = __ldg(p.row_ptr + rg.y);
        r_lo = sub == 0 ? rg.x : first_row_at(p.row_ptr, rg.x, rg.y, jb + (int)((long long)(je - jb) * sub / P));
        r_hi = sub == P - 1 ? rg.y
                            : first_row_at(p.row_ptr, rg.x, rg.y, jb + (int)((long long)(je - jb) * (sub + 1) / P));
    }
    for (int pass = 0; pass < npass; ++pass) {
        const int c0 = pass * CPP + gl * VEC;
        if (c0 >= p.ncols) break;
        stream_lean<T, VEC, U, EPI, PF>(p, r_lo, r_hi, c0);
    }
}

}  // namespace tca
