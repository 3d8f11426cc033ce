// Tensor-core path for dense windows: tcgen05.mma with TMEM accumulators.
//
// Replaces the reference's use of mma.sync.m16n8k8 (src/our_spmm.cu:118-125,
// :255-262), where only the 8 "diagonal" products of each MMA are kept.  Here a
// window of R = 32 rows is condensed on the host into tiles of 16 columns (the
// union of its rows' columns); every MMA product is a real product of the
// condensed tile (zeros only where a row lacks a column of the union).
//
// One unit = (window, block of 128 output columns).  Per unit the kernel
// computes the transposed tile  C^T[128 x R] = Bpanel^T[128 x 16k] * V^T[16k x R]
// with tcgen05.mma.kind::f16, M = 128 (output columns -> TMEM lanes),
// N = R (window rows -> TMEM columns), K = 16 per tile, fp32 accumulation in
// TMEM across the window's tiles.
//
// Shared-memory operands, canonical no-swizzle layouts (16-byte core-matrix rows):
//   A = B panel, MN-major: 16 gathered B rows x 128 columns, core matrix =
//       8 k-rows x 8 columns (128 B); columns step SBO = 256 B, k step LBO = 128 B.
//   B = value tile, K-major: R rows x 16 k, core matrix = 8 rows x 8 k;
//       k step LBO = 128 B, rows step SBO = 256 B.  The host stores each tile's
//       values already in this image, so one 16-byte copy per 8 values lands it.
//
// Warp roles (288 threads): warps 0-3 epilogue (tcgen05.ld of TMEM lanes
// 32w..32w+31 -> coalesced fp32 C rows), warp 4 TMEM allocation + MMA issue
// (one thread), warps 5-8 producers (cp.async 16-byte gathers of B rows and
// value tiles into a 16-stage mbarrier ring; B-row indices staged in smem).  Two TMEM accumulators let the
// epilogue of one unit overlap the MMAs of the next.
//
// Every mbarrier wait is bounded: on time-out the kernel records a code in the
// plan's error word, stops issuing work, drains its MMAs (bounded), frees TMEM
// and returns; tcaspmm_plan_sync_check reports TCASPMM_ERR_TIMEOUT.
#include <algorithm>
#include <climits>
#include <cstring>
#include <vector>

#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include "plan.h"
#include "residue.cuh"

namespace tca {

namespace {

constexpr int R = 32;            // window rows = MMA N
constexpr int KT = 16;           // condensed columns per tile = MMA K (16-bit inputs)
constexpr int MB = 128;          // output columns per unit = MMA M
constexpr int STAGES = 16;
constexpr int IDX_TILES = 32;           // tile column indices staged per producer warp per refill
constexpr int PANEL_BYTES = MB * KT * 2;  // 4096
constexpr int VAL_BYTES = R * KT * 2;     // 1024
constexpr int STAGE_BYTES = PANEL_BYTES + VAL_BYTES;
constexpr int TMEM_COLS = 2 * R;          // two accumulators
constexpr int NUM_THREADS = 288;
constexpr int PRODUCER_THREADS = 128;
constexpr int EPI_THREADS = 128;
constexpr unsigned long long WAIT_CYCLES = 4ull << 30;  // ~2 s at 2 GHz

struct TcParams {
    const int4 *windows;     // {first row, first tile, tiles, rows}
    const int32_t *order;    // windows by decreasing tile count
    const int32_t *tile_cols;
    const uint16_t *tile_vals;
    const void *B;
    long long ldb;
    float *C;
    long long ldc;
    int ncols;
    int n_units;
    int nfb;                 // column blocks of 128
    int *err;
};

__device__ __forceinline__ uint32_t smem_u32(const void *p) { return (uint32_t)__cvta_generic_to_shared(p); }

__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count)
{
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t parity)
{
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(bar), "r"(parity)
        : "memory");
    return ok != 0;
}

__device__ __forceinline__ void mbar_arrive(uint32_t bar)
{
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}

// Bounded wait: false (and the abort flag raised, error recorded) on time-out.
__device__ __forceinline__ bool wait_bounded(uint32_t bar, uint32_t parity, volatile int *abort_flag, int *err,
                                             int code)
{
    if (mbar_try_wait(bar, parity)) return true;
    const unsigned long long t0 = clock64();
    for (;;) {
        if (mbar_try_wait(bar, parity)) return true;
        if (*abort_flag) return false;
        if (clock64() - t0 > WAIT_CYCLES) {
            atomicOr(err, code);
            *abort_flag = 1;
            return false;
        }
    }
}

__device__ __forceinline__ void cp_async_16(uint32_t dst, const void *src, uint32_t src_size)
{
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(src_size) : "memory");
}

__device__ __forceinline__ void cp_async_arrive_noinc(uint32_t bar)
{
    asm volatile("cp.async.mbarrier.arrive.noinc.shared::cta.b64 [%0];" ::"r"(bar) : "memory");
}

__device__ __forceinline__ uint64_t smem_desc(uint32_t addr, uint32_t lbo, uint32_t sbo)
{
    // tcgen05 shared-memory descriptor: start address, leading / stride byte
    // offsets (all >> 4), version 1 (bits 46-47), no swizzle (bits 61-63 = 0).
    return (uint64_t)((addr >> 4) & 0x3FFF) | ((uint64_t)((lbo >> 4) & 0x3FFF) << 16) |
           ((uint64_t)((sbo >> 4) & 0x3FFF) << 32) | (1ull << 46);
}

template <bool BF16>
__device__ __forceinline__ constexpr uint32_t instr_desc()
{
    // kind::f16 instruction descriptor: D fp32 (bits 4-5 = 1), A/B format
    // (bits 7-9, 10-12: 0 f16, 1 bf16), A MN-major (bit 15), B K-major (bit 16 = 0),
    // N >> 3 (bits 17-22), M >> 4 (bits 24-28).
    return (1u << 4) | ((BF16 ? 1u : 0u) << 7) | ((BF16 ? 1u : 0u) << 10) | (1u << 15) | ((uint32_t)(R >> 3) << 17) |
           ((uint32_t)(MB >> 4) << 24);
}

__device__ __forceinline__ void mma_f16(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                        uint32_t accumulate)
{
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
        : "memory");
}

__device__ __forceinline__ void mma_commit(uint32_t bar)
{
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar)
                 : "memory");
}

__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

__device__ __forceinline__ void tmem_ld32(uint32_t taddr, float (&v)[32])
{
    uint32_t r[32];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
        "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "
        "%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
          "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
          "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
        : "r"(taddr));
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
    for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}

template <bool BF16>
__global__ void __launch_bounds__(NUM_THREADS, 1) tc_kernel(const TcParams p)
{
    extern __shared__ uint8_t smem_raw[];
    // 1024-byte aligned stage ring, then barriers.
    uint8_t *smem = (uint8_t *)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
    int32_t *idxbuf = (int32_t *)(smem + STAGES * STAGE_BYTES);  // [4 warps][IDX_TILES][KT]
    uint64_t *bars = (uint64_t *)(smem + STAGES * STAGE_BYTES + 4 * IDX_TILES * KT * 4);
    uint64_t *full = bars;                 // [STAGES] producers -> MMA
    uint64_t *empty = bars + STAGES;       // [STAGES] MMA -> producers
    uint64_t *accf = bars + 2 * STAGES;    // [2] MMA -> epilogue
    uint64_t *acce = bars + 2 * STAGES + 2;// [2] epilogue -> MMA
    uint64_t *drain = bars + 2 * STAGES + 4;
    uint32_t *tmem_holder = (uint32_t *)(bars + 2 * STAGES + 5);
    volatile int *abort_flag = (volatile int *)(tmem_holder + 1);

    const int tid = threadIdx.x;
    const int warp = tid >> 5;
    const int lane = tid & 31;

    if (tid == 0) {
        for (int s = 0; s < STAGES; ++s) {
            mbar_init(smem_u32(&full[s]), PRODUCER_THREADS);
            mbar_init(smem_u32(&empty[s]), 1);
        }
        for (int a = 0; a < 2; ++a) {
            mbar_init(smem_u32(&accf[a]), 1);
            mbar_init(smem_u32(&acce[a]), EPI_THREADS);
        }
        mbar_init(smem_u32(drain), 1);
        *abort_flag = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == 4) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_holder)),
                     "r"(TMEM_COLS)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_holder;

    if (warp >= 5) {
        // ------------------------------ producers ------------------------------
        // Each producer warp stages the B-row indices of up to IDX_TILES tiles in
        // its own shared-memory slice with one cooperative load, so no cp.async
        // waits on a dependent load.  Only warp-level syncs are used, and every
        // abort decision is warp-uniform, so a time-out cannot strand a barrier.
        const int pt = tid - 160;       // 0..127
        const int pw = pt >> 5;         // producer warp 0..3: column chunks 4pw..4pw+3
        const int kr = lane & 7;        // row within a core matrix
        const int cc = pw * 4 + (lane >> 3);
        int32_t *widx = idxbuf + pw * IDX_TILES * KT;
        const char *Bb = (const char *)p.B;
        uint32_t g = 0;
        bool ok = true;
        for (int u = blockIdx.x; ok && u < p.n_units; u += gridDim.x) {
            const int4 w = p.windows[p.order[u / p.nfb]];
            const int f = (u % p.nfb) * MB + cc * 8;  // first of this thread's 8 columns
            const bool fvalid = f < p.ncols;
            for (int t0 = 0; ok && t0 < w.z; t0 += IDX_TILES) {
                const int nt = min(IDX_TILES, w.z - t0);
                __syncwarp();  // previous indices consumed
                for (int q = lane; q < nt * KT; q += 32) widx[q] = __ldg(p.tile_cols + ((long long)w.y + t0) * KT + q);
                __syncwarp();  // indices visible to the warp
                for (int t = 0; t < nt; ++t, ++g) {
                    const int s = g % STAGES;
                    ok = __all_sync(0xffffffffu,
                                    wait_bounded(smem_u32(&empty[s]), ((g / STAGES) & 1) ^ 1, abort_flag, p.err, 1));
                    if (!ok) break;
                    const long long tile = (long long)w.y + t0 + t;
                    const uint32_t panel = smem_u32(smem + s * STAGE_BYTES);
#pragma unroll
                    for (int i = 0; i < 2; ++i) {
                        const int brow = widx[t * KT + i * 8 + kr];
                        const char *src = fvalid ? Bb + ((long long)brow * p.ldb + f) * 2 : Bb;
                        cp_async_16(panel + cc * 256 + i * 128 + kr * 16, src, fvalid ? 16u : 0u);
                    }
                    if (pt < VAL_BYTES / 16)
                        cp_async_16(panel + PANEL_BYTES + pt * 16, p.tile_vals + tile * (R * KT) + pt * 8, 16u);
                    cp_async_arrive_noinc(smem_u32(&full[s]));
                }
            }
        }
        asm volatile("cp.async.wait_all;" ::: "memory");
    } else if (warp == 4) {
        // ------------------------------ MMA issuer -----------------------------
        if (lane == 0) {
            constexpr uint32_t idesc = instr_desc<BF16>();
            uint32_t g = 0, i = 0;
            bool ok = true;
            for (int u = blockIdx.x; ok && u < p.n_units; u += gridDim.x, ++i) {
                const int4 w = p.windows[p.order[u / p.nfb]];
                const uint32_t a = i & 1;
                if (!wait_bounded(smem_u32(&acce[a]), ((i >> 1) & 1) ^ 1, abort_flag, p.err, 2)) break;
                tc_fence_after();
                const uint32_t dcol = tmem + a * R;
                for (int t = 0; t < w.z; ++t, ++g) {
                    const int s = g % STAGES;
                    if (!wait_bounded(smem_u32(&full[s]), (g / STAGES) & 1, abort_flag, p.err, 2)) {
                        ok = false;
                        break;
                    }
                    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
                    tc_fence_after();
                    const uint32_t panel = smem_u32(smem + s * STAGE_BYTES);
                    const uint64_t adesc = smem_desc(panel, 128, 256);
                    const uint64_t bdesc = smem_desc(panel + PANEL_BYTES, 128, 256);
                    mma_f16(dcol, adesc, bdesc, idesc, t > 0 ? 1u : 0u);
                    mma_commit(smem_u32(&empty[s]));
                }
                if (!ok) break;
                mma_commit(smem_u32(&accf[a]));
            }
            // Drain: every MMA issued above has completed once `drain` flips.
            mma_commit(smem_u32(drain));
            int dummy = 0;
            wait_bounded(smem_u32(drain), 0, (volatile int *)&dummy, p.err, 8);
        }
        __syncwarp();
    } else {
        // ------------------------------ epilogue -------------------------------
        uint32_t i = 0;
        for (int u = blockIdx.x; u < p.n_units; u += gridDim.x, ++i) {
            const int4 w = p.windows[p.order[u / p.nfb]];
            const uint32_t a = i & 1;
            if (!__all_sync(0xffffffffu, wait_bounded(smem_u32(&accf[a]), (i >> 1) & 1, abort_flag, p.err, 4))) break;
            tc_fence_after();
            float v[32];
            tmem_ld32(tmem + ((uint32_t)(warp * 32) << 16) + a * R, v);
            tc_fence_before();
            mbar_arrive(smem_u32(&acce[a]));
            const int f = (u % p.nfb) * MB + warp * 32 + lane;
            if (f < p.ncols) {
                float *c = p.C + (long long)w.x * p.ldc + f;
#pragma unroll
                for (int r = 0; r < R; ++r)
                    if (r < w.w) __stcs(c + (long long)r * p.ldc, v[r]);
            }
        }
    }

    tc_fence_before();
    __syncthreads();
    if (warp == 4) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(TMEM_COLS) : "memory");
    }
}

// Tail: 2 * STAGES + 5 mbarriers, the TMEM address and the abort flag.
constexpr size_t kBarBytes = (2 * STAGES + 5) * 8 + 8;
constexpr size_t kSmemBytes = 1024 + STAGES * STAGE_BYTES + 4 * IDX_TILES * KT * 4 + (kBarBytes + 127) / 128 * 128;  // ~89 KB

template <typename X>
tcaspmm_status upload_vec(Shard *sh, X **dst, const std::vector<X> &v, const char *what)
{
    *dst = nullptr;
    if (v.empty()) return TCASPMM_OK;
    cudaError_t e = cudaMalloc((void **)dst, sizeof(X) * v.size());
    if (e != cudaSuccess) {
        *dst = nullptr;
        return fail(TCASPMM_ERR_ALLOC, "cudaMalloc for %s failed: %s", what, cudaGetErrorString(e));
    }
    sh->allocs.push_back(*dst);
    sh->bytes += (int64_t)(sizeof(X) * v.size());
    e = cudaMemcpy(*dst, v.data(), sizeof(X) * v.size(), cudaMemcpyHostToDevice);
    return e == cudaSuccess ? TCASPMM_OK : cuda_fail(e, what);
}

}  // namespace

bool tc_supported()
{
    int dev = 0, major = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return false;
    if (cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev) != cudaSuccess) return false;
    return major == 10;
}

tcaspmm_status tc_upload(const tcaspmm_csr &, tcaspmm_dtype dt, Shard *sh)
{
    const TileSchedule &T = sh->sched.tc;
    sh->n_windows = (int)T.windows.size();
    if (sh->n_windows == 0) return TCASPMM_OK;
    if (T.R != R || T.KT != KT) return fail(TCASPMM_ERR_UNSUPPORTED, "tile shape %dx%d not built", T.R, T.KT);
    // Windows by decreasing tile count, so the persistent grid balances.
    std::vector<int32_t> order(sh->n_windows);
    for (int i = 0; i < sh->n_windows; i++) order[i] = i;
    std::stable_sort(order.begin(), order.end(),
                     [&](int32_t a, int32_t b) { return T.windows[a].z > T.windows[b].z; });
    // Value tiles -> shared-memory image (K-major, no swizzle, LBO 128 B, SBO 256 B).
    const size_t ntiles = T.tile_cols.size() / KT;
    std::vector<uint16_t> img(ntiles * R * KT);
    for (size_t t = 0; t < ntiles; t++)
        for (int n = 0; n < R; n++)
            for (int k = 0; k < KT; k++) {
                const float v = T.tile_vals[(t * R + n) * KT + k];
                img[t * R * KT + (n / 8) * 128 + (k / 8) * 64 + (n % 8) * 8 + (k % 8)] =
                    dt == TCASPMM_BF16 ? float_to_bf16_bits(v) : float_to_half_bits(v);
            }
    // Fallback row ranges over tc rows (run on the CUDA cores when B or C is
    // not 16-byte aligned at execute time).
    std::vector<Int2> fb;
    for (const Int4 &w : T.windows) fb.push_back(Int2{w.x, w.x + w.w});
    tcaspmm_status s;
    if ((s = upload_vec(sh, &sh->tc_windows, T.windows, "tc windows")) != TCASPMM_OK) return s;
    if ((s = upload_vec(sh, &sh->tc_order, order, "tc order")) != TCASPMM_OK) return s;
    if ((s = upload_vec(sh, &sh->tc_cols, T.tile_cols, "tc columns")) != TCASPMM_OK) return s;
    if ((s = upload_vec(sh, (uint16_t **)&sh->tc_vals, img, "tc values")) != TCASPMM_OK) return s;
    if ((s = upload_vec(sh, &sh->tc_fallback, fb, "tc fallback ranges")) != TCASPMM_OK) return s;
    int nsm = 148;
    cudaDeviceGetAttribute(&nsm, cudaDevAttrMultiProcessorCount, sh->device);
    sh->num_sms = nsm;
    // More than 48 KB of dynamic shared memory needs the opt-in, per device.
    cudaError_t e = cudaFuncSetAttribute(tc_kernel<false>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kSmemBytes);
    if (e == cudaSuccess)
        e = cudaFuncSetAttribute(tc_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kSmemBytes);
    return e == cudaSuccess ? TCASPMM_OK : cuda_fail(e, "tc kernel shared-memory opt-in");
}

tcaspmm_status launch_tc(const Shard &sh, tcaspmm_dtype dt, const void *dB, int64_t ldb, float *dC, int64_t ldc,
                         cudaStream_t st)
{
    if (sh.n_windows == 0 || sh.ncols == 0) return TCASPMM_OK;
    const bool aligned = ((uintptr_t)dB % 16 == 0) && ((ldb * 2) % 16 == 0) && (sh.ncols % 8 == 0);
    if (!aligned)  // CUDA-core fallback over the tc rows: whole rows, no segments
        return launch_residue(sh, dt, dB, ldb, dC, ldc, st, sh.tc_fallback, sh.n_windows);
    TcParams p;
    p.windows = (const int4 *)sh.tc_windows;
    p.order = sh.tc_order;
    p.tile_cols = sh.tc_cols;
    p.tile_vals = (const uint16_t *)sh.tc_vals;
    p.B = dB;
    p.ldb = ldb;
    p.C = dC;
    p.ldc = ldc;
    p.ncols = (int)sh.ncols;
    p.nfb = (int)((sh.ncols + MB - 1) / MB);
    p.n_units = sh.n_windows * p.nfb;
    p.err = sh.err;
    const int grid = std::min(p.n_units, 4 * sh.num_sms);
    if (dt == TCASPMM_BF16)
        tc_kernel<true><<<grid, NUM_THREADS, kSmemBytes, st>>>(p);
    else
        tc_kernel<false><<<grid, NUM_THREADS, kSmemBytes, st>>>(p);
    cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? TCASPMM_OK : cuda_fail(e, "tc kernel launch");
}

}  // namespace tca
