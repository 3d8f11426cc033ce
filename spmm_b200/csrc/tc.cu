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
// with tcgen05.mma.kind::f16 (fp16 / bf16) or kind::tf32, M = 128 (output
// columns -> TMEM lanes), N = R (window rows -> TMEM columns), fp32 accumulation
// in TMEM across the window's tiles.
//
// Shared-memory operands.  B = value tile, K-major, no swizzle: R rows x 16 k,
// core matrices of 8 rows x 16 bytes, 16-byte k chunks LBO = 128 B apart, 8-row
// groups SBO apart (256 B for 16-bit types, 512 B for tf32); the host stores each
// tile's values in exactly this image.  A = B panel (gathered B rows x 128
// columns), MN-major, swizzled 128-byte atom rows written by TMA, in pieces of 64
// (16-bit) or 32 (fp32) columns.  One pipeline stage is 16 KB of panel (4 tiles
// of 16-bit, 2 of tf32) + 4 KB of values.  One lane fills a stage with, per
// piece, a single TMA box of all the stage's rows when they are consecutive
// (dense windows), else per tile a box of 16 rows (16 consecutive rows) or four
// tile::gather4 loads of 4 rows, plus one cp.async.bulk of the stage's value
// tiles; the 2-D tensor maps over B write the swizzle and zero-fill columns past
// N.  The MMA thread issues the stage's MMAs (4 of K = 16, or 4 of K = 8) and one
// commit, so the barrier round trips are paid per stage.
//
// Warp roles: warps 0-3 epilogue (tcgen05.ld of TMEM lanes 32w..32w+31 ->
// coalesced fp32 C rows), warp 4 TMEM allocation + MMA issue (one thread),
// warps 5-7 producers on a 4-stage mbarrier ring (TMA stages round-robin from one
// lane each, cp.async stages by all three warps together).  Two TMEM
// accumulators let the epilogue of one work item overlap the MMAs of the next.
//
// Work items ("tasks") are windows or, for the gathered windows of long rows
// (rows grouped by length, any row indices), consecutive parts of a window's
// tile chain, so one hub window's thousands of tiles spread over many CTAs.  A
// part's epilogue warps store their 32 x 32 partial tile to scratch and count it
// in; the warp that completes the window's last part adds the parts in part
// order (deterministic) and writes the C rows through the window's row list.
//
// Every mbarrier wait is bounded: on time-out the kernel records a code in the
// plan's error word, stops issuing work, drains its copies and MMAs (bounded),
// frees TMEM and returns; tcaspmm_plan_sync_check reports TCASPMM_ERR_TIMEOUT and
// tcaspmm_selftest_tc_timeout exercises that path.
#include <algorithm>
#include <climits>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <vector>

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include "plan.h"
#include "residue.cuh"

namespace tca {

namespace {

constexpr int R = 32;            // window rows = MMA N
constexpr int KT = 16;           // condensed columns per tile
constexpr int MB = 128;          // output columns per unit = MMA M
constexpr int STAGES = 4;        // pipeline stages of 20 KB
constexpr int IDX_TILES = 16;    // tile column indices staged per refill (a multiple of every TPS), two
                                 // buffers a producer warp; 16 keeps a CTA's shared memory low enough for
                                 // two CTAs per SM
constexpr int IDX_INTS = IDX_TILES * KT;  // ints of one index buffer
constexpr int PANEL_BYTES = 16384;                     // B panel per stage (any element type)
constexpr int STAGE_BYTES = PANEL_BYTES + 4096;        // + the stage's value tiles

// Element-type geometry.  FMT 0 = fp16, 1 = bf16 (kind::f16, 2-byte elements),
// 2 = tf32 (kind::tf32, fp32 storage).  A 128-byte swizzle atom row holds CPB
// columns, so the 128-column panel is NPC column pieces; a stage holds TPS tiles
// (SROWS B rows), so every stage is 16 KB of panel + 4 KB of values.  Within a
// piece, B row k of the stage sits in atom k / 8 (1 KB apart), so tile j starts
// 2 KB into every piece whatever the type.
template <int FMT> struct Geo {
    static constexpr int ES = FMT == 2 ? 4 : 2;      // element bytes
    static constexpr int TPS = 8 / ES;               // tiles per stage: 4 or 2
    static constexpr int SROWS = TPS * KT;           // B rows per stage: 64 or 32
    static constexpr int CPB = 128 / ES;             // columns per piece: 64 or 32
    static constexpr int NPC = MB / CPB;             // pieces per panel: 2 or 4
    static constexpr int PIECE = SROWS / 8 * 1024;   // bytes of one piece in a stage: 8 or 4 KB
    static constexpr int TILE_PANEL = MB * KT * ES;  // panel bytes per tile: 4 or 8 KB
    static constexpr int TILE_VAL = R * KT * ES;     // value bytes per tile: 1 or 2 KB
    static constexpr int KSTEP = 32 / ES;            // K of one MMA: 16 or 8
    static constexpr int KCH = KT * ES / 16;         // 16-byte k chunks per value-tile row: 2 or 4
    // Panel swizzle, as the smem-descriptor layout type: 128-byte swizzle of
    // 16-byte chunks (2) for 16-bit types; MN-major tf32 operands take the
    // 128-byte swizzle of 32-byte chunks (1), which TMA writes with
    // CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B.
    static constexpr uint32_t LAYOUT = FMT == 2 ? 1u : 2u;
    // Stride between the k-row groups the MMA walks through (SBO): 8-row atoms
    // of 1 KB for 16-bit types; 4-row groups (512 B) for tf32 (measured: with
    // 1 KB, k rows 4-7 of each group were read from rows 8-11).
    static constexpr uint32_t KGROUP = FMT == 2 ? 512u : 1024u;
    static_assert(TPS * TILE_PANEL == PANEL_BYTES && TPS * TILE_VAL == STAGE_BYTES - PANEL_BYTES, "stage size");
    static_assert(IDX_TILES % TPS == 0, "stages must not straddle index refills");
};
constexpr int TMEM_COLS = 2 * R;  // two accumulators
// Producer warps: TMA stages round-robin, cp.async stages together.  Three, so a
// CTA has eight warps: warps are spread over the SM's four schedulers, whose
// register files hold 16K registers each, and with eight warps two CTAs fit at up
// to 128 registers a thread (nine warps put six on one scheduler: 85 at most).
constexpr int NPROD = 3;
constexpr int PTHREADS = NPROD * 32;
constexpr int ROW_STEP = PTHREADS / 16;                     // B rows a cp.async pass covers (16 threads a row)
constexpr int ROW_PASSES = (64 + ROW_STEP - 1) / ROW_STEP;  // passes over a stage's 64 rows
static_assert(PTHREADS % 16 == 0, "a B row slice is copied by 16 threads");
static_assert(2 * ROW_PASSES <= 32, "a producer warp's lanes hold the indices of its rows of a stage");
// Stages ahead at which a cp.async producer loads B-row indices (a stage lasts
// ~0.4 us, an index load from HBM up to ~1 us).
constexpr int IDX_AHEAD = 3;
constexpr int NUM_THREADS = 160 + 32 * NPROD;
constexpr int CBUF_BYTES = 4 * 32 * 32 * 4;  // C staging: a 32 x 32 fp32 tile per epilogue warp
constexpr int EPI_THREADS = 128;
constexpr unsigned long long WAIT_CYCLES = 4ull << 30;  // ~2 s at 2 GHz: no legitimate wait comes close

struct TcParams {
    const int4 *tasks;       // {x, first tile, tiles, rows} (x as in TileSchedule::windows), by decreasing tiles
    const int4 *splits;      // per task {split window id or -1, part, parts, first partial slot of the window}
    const int32_t *rows;     // row lists of the gathered windows
    float *partials;         // [slot][column block][epilogue warp][32 x 32] partial tiles of split windows
    unsigned int *counters;  // [split window][column block][epilogue warp], zero between launches
    const int32_t *dense_c0; // per task: first column when its columns are one consecutive run; else
                             // -2 (tiles fetched by TMA gather4) or -1 (16-bit tiles fetched by cp.async)
    const int32_t *tile_cols;
    const uint8_t *tile_vals;  // per tile: the value tile's shared-memory image
    const void *B;
    long long ldb;
    void *C;                 // fp32, or 16-bit with the epilogue
    long long ldc;           // elements of C's type
    int ncols;
    int K;                   // rows of B
    int n_units;
    int nfb;                 // column blocks of 128
    int *err;
    unsigned long long wait_cycles;  // bound of every mbarrier wait
    int stall_test;          // self-test: the producer issues no copies, so waits must time out
    int has_ep;              // apply `ep` (row scale, bias, ReLU, 16-bit C)
    EpiParams ep;
    int tma_store;           // C written by bulk tensor stores through `cmap` (aligned C)
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
// err[0] collects the codes of every wait that ran out; the first one also
// records where it gave up: err[1] its code, err[2] the barrier's shared-memory
// address, err[3] the phase parity waited for, err[4] the CTA, err[5] the thread.
__device__ __forceinline__ bool wait_bounded(uint32_t bar, uint32_t parity, volatile int *abort_flag, int *err,
                                             int code, unsigned long long limit)
{
    if (mbar_try_wait(bar, parity)) return true;
    const unsigned long long t0 = clock64();
    for (;;) {
        if (mbar_try_wait(bar, parity)) return true;
        if (*abort_flag) return false;
        if (clock64() - t0 > limit) {
            atomicOr(err, code);
            if (atomicCAS(err + 1, 0, code) == 0) {
                err[2] = (int)bar;
                err[3] = (int)parity;
                err[4] = (int)blockIdx.x;
                err[5] = (int)threadIdx.x;
            }
            *abort_flag = 1;
            return false;
        }
    }
}

__device__ __forceinline__ void mbar_arrive_n(uint32_t bar, uint32_t count)
{
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}

// 16-byte asynchronous copy global -> shared (L2 only); src_bytes 0 writes zeros.
__device__ __forceinline__ void cp_async16(uint32_t dst, const void *src, uint32_t src_bytes)
{
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(src_bytes) : "memory");
}
// Arrive on the barrier once every cp.async this thread issued so far has landed;
// the arrival counts against the barrier's expected count (.noinc), so a thread
// never blocks on its own copies.
__device__ __forceinline__ void cp_async_arrive_noinc(uint32_t bar)
{
    asm volatile("cp.async.mbarrier.arrive.noinc.shared::cta.b64 [%0];" ::"r"(bar) : "memory");
}

__device__ __forceinline__ void mbar_expect_tx(uint32_t bar, uint32_t bytes)
{
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes) : "memory");
}

// Box of the tensor map (64 columns x 16 or 64 rows) at (x, y) -> dst.
__device__ __forceinline__ void tma_box(uint32_t dst, const void *tmap, int x, int y, uint32_t bar)
{
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
            dst),
        "l"(tmap), "r"(x), "r"(y), "r"(bar)
        : "memory");
}

// 4 rows (y0..y3) x 64 columns from x of the gather tensor map -> dst.
__device__ __forceinline__ void tma_gather4(uint32_t dst, const void *tmap, int x, int y0, int y1, int y2, int y3,
                                            uint32_t bar)
{
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile::gather4.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%2, %3, %4, %5, %6}], [%7];" ::"r"(dst),
        "l"(tmap), "r"(x), "r"(y0), "r"(y1), "r"(y2), "r"(y3), "r"(bar)
        : "memory");
}

__device__ __forceinline__ void bulk_copy(uint32_t dst, const void *src, uint32_t bytes, uint32_t bar)
{
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(dst),
                 "l"(src), "r"(bytes), "r"(bar)
                 : "memory");
}

// 2-D bulk tensor store of the box at (x, y) of tmap from shared memory, and
// its bulk-group bookkeeping (per issuing thread).
__device__ __forceinline__ void tma_store_2d(const void *tmap, int x, int y, uint32_t src)
{
    asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%1, %2}], [%3];" ::"l"(tmap), "r"(x),
                 "r"(y), "r"(src)
                 : "memory");
}
__device__ __forceinline__ void bulk_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
__device__ __forceinline__ void bulk_wait_read() { asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory"); }
__device__ __forceinline__ void bulk_wait_all() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }
__device__ __forceinline__ void fence_proxy_async() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

__device__ __forceinline__ uint64_t smem_desc(uint32_t addr, uint32_t lbo, uint32_t sbo, uint32_t layout)
{
    // tcgen05 shared-memory descriptor: start address, leading / stride byte
    // offsets (all >> 4), version 1 (bits 46-47), layout type (bits 61-63:
    // 0 no swizzle, 1 128-byte swizzle of 32-byte chunks, 2 128-byte swizzle).
    return (uint64_t)((addr >> 4) & 0x3FFF) | ((uint64_t)((lbo >> 4) & 0x3FFF) << 16) |
           ((uint64_t)((sbo >> 4) & 0x3FFF) << 32) | (1ull << 46) | ((uint64_t)layout << 61);
}

// Stage k of a unit in load order, for a unit of nst stages that starts at
// stage rot.  Each window starts at its own offset (window index mod nst), so
// CTAs that run different windows at the same time read different B rows; when
// every window starts at stage 0, all CTAs request the same lines together and
// queue on the L2 slices holding them.  The order is fixed per plan, so results
// are deterministic.
__device__ __forceinline__ int stage_at(int k, int rot, int nst) { return k + rot < nst ? k + rot : k + rot - nst; }

// Per-thread stores of one output column f of a task's rows: lane i holds
// `rid`, the C row of the window's row i (row scales already applied).  Bias and
// ReLU when the epilogue is on, then fp32 / fp16 / bf16 stores; a warp writes 32
// consecutive columns of each row.  Every lane of the warp calls this (the row
// ids are broadcast by shuffles); lanes past the last column store nothing.
__device__ __forceinline__ void epilogue_rows(const TcParams &p, int rid, int rows, int f, const float (&v)[32])
{
    const EpiParams &ep = p.ep;
    const bool colok = f < p.ncols;
    const float b = (p.has_ep && ep.bias && colok) ? __ldg(ep.bias + f) : 0.0f;
#pragma unroll
    for (int r = 0; r < R; ++r) {
        const long long row = __shfl_sync(0xffffffffu, rid, r);
        if (r < rows && colok) {
            float x = v[r];
            if (p.has_ep) {
                x += b;
                if (ep.relu) x = fmaxf(x, 0.0f);
            }
            const long long o = row * p.ldc + f;
            if (!p.has_ep || ep.out == 0)
                __stcs(static_cast<float *>(p.C) + o, x);
            else if (ep.out == 1)
                static_cast<__half *>(p.C)[o] = __float2half_rn(x);
            else
                static_cast<__nv_bfloat16 *>(p.C)[o] = __float2bfloat16_rn(x);
        }
    }
}

// The tensor maps over the B block of a launch, all 128-byte swizzled: box
// 64 x 1 (gather4), 64 x 16 and 64 x 64 (consecutive rows).
struct BMaps {
    CUtensorMap gather;
    CUtensorMap box16;
    CUtensorMap box64;
};

template <int FMT>
__device__ __forceinline__ constexpr uint32_t instr_desc()
{
    // kind::f16 / kind::tf32 instruction descriptor: D fp32 (bits 4-5 = 1), A/B
    // format (bits 7-9, 10-12: 0 f16, 1 bf16, 2 tf32), A MN-major (bit 15), B
    // K-major (bit 16 = 0), N >> 3 (bits 17-22), M >> 4 (bits 24-28).
    return (1u << 4) | ((uint32_t)FMT << 7) | ((uint32_t)FMT << 10) | (1u << 15) | ((uint32_t)(R >> 3) << 17) |
           ((uint32_t)(MB >> 4) << 24);
}

template <int FMT>
__device__ __forceinline__ void mma_issue(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                          uint32_t accumulate)
{
    if constexpr (FMT == 2)
        asm volatile(
            "{\n\t.reg .pred p;\n\t"
            "setp.ne.b32 p, %4, 0;\n\t"
            "tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
            "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
            : "memory");
    else
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

template <int FMT>
__global__ void __launch_bounds__(NUM_THREADS, 2)
    tc_kernel(const TcParams p, const __grid_constant__ BMaps maps, const __grid_constant__ CUtensorMap cmap)
{
    extern __shared__ uint8_t smem_raw[];
    // 1024-byte aligned stage ring, then the index buffer and the barriers.
    uint8_t *smem = (uint8_t *)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
    uint8_t *cbuf = smem + STAGES * STAGE_BYTES;                             // [4 warps][32 rows][32 columns]
    int32_t *idxbuf = (int32_t *)(smem + STAGES * STAGE_BYTES + CBUF_BYTES);  // [NPROD][2][IDX_TILES][KT]
    uint64_t *bars = (uint64_t *)(smem + STAGES * STAGE_BYTES + CBUF_BYTES + NPROD * 2 * IDX_INTS * 4);
    uint64_t *full = bars;                  // [STAGES] producer -> MMA
    uint64_t *empty = bars + STAGES;        // [STAGES] MMA -> producer
    uint64_t *accf = bars + 2 * STAGES;     // [2] MMA -> epilogue
    uint64_t *acce = bars + 2 * STAGES + 2; // [2] epilogue -> MMA
    uint64_t *drain = bars + 2 * STAGES + 4;
    uint32_t *tmem_holder = (uint32_t *)(bars + 2 * STAGES + 5);
    volatile int *abort_flag = (volatile int *)(tmem_holder + 1);

    using G = Geo<FMT>;
    const int tid = threadIdx.x;
    const int warp = tid >> 5;
    const int lane = tid & 31;
    // The producer's first window descriptor, loaded before the set-up barrier so
    // its latency overlaps the barrier initialisation and the TMEM allocation.
    int4 w_first = make_int4(0, 0, 0, 0);
    int c_first = -1;
    if (warp >= 5 && (int)blockIdx.x < p.n_units) {
        w_first = p.tasks[blockIdx.x / p.nfb];
        c_first = p.dense_c0[blockIdx.x / p.nfb];
    }

    if (tid == 0) {
        for (int s = 0; s < STAGES; ++s) {
            // One arrival per producer thread: a TMA stage's issuer arrives with
            // expect_tx plus PTHREADS - 1 more (TMA completes the bytes); in a
            // cp.async stage every producer thread arrives once its copies landed.
            mbar_init(smem_u32(&full[s]), PTHREADS);
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
        // Warps 5 .. 5 + NPROD - 1 walk the same stage sequence.
        //  * TMA stages (windows whose columns are one consecutive run, and
        //    gathered tiles): warp 5 + i fills the stages g with g % NPROD == i from
        //    one lane -- one 64 x 64 box per column piece when the stage's B rows
        //    are consecutive, else per tile a 64 x 16 box or four gather4 loads,
        //    plus one bulk copy of the stage's value tiles -- and arrives for all
        //    producer threads.
        //  * cp.async stages (gathered 16-bit tiles under TCASPMM_GATHER_TMA=0):
        //    all PTHREADS threads copy
        //    the stage's B row slices (16 bytes each, coalesced per row) straight
        //    into the 128-byte-swizzled panel layout, and the value tiles; each
        //    thread's arrival on the stage's full barrier is triggered by the
        //    landing of its copies, so every free slot of the ring is in flight
        //    (the MMA issuer fences the proxies before its tensor cores read them).
        const int pw = warp - 5;
        const int ptid = tid - 160;  // 0 .. PTHREADS - 1
        int32_t *const mybufs = idxbuf + pw * 2 * IDX_INTS;  // this warp's two index buffers
        uint32_t g = 0;  // stages of this CTA (issued by this warp or the other producers)
        bool ok = true;
        uint32_t tma_mine = 0;  // bit s: this lane issued the TMA copies of the stage now in slot s
        const void *tm_g = &maps.gather, *tm_16 = &maps.box16, *tm_64 = &maps.box64;
        if (lane == 0) {
            asm volatile("prefetch.tensormap [%0];" ::"l"(tm_g) : "memory");
            asm volatile("prefetch.tensormap [%0];" ::"l"(tm_16) : "memory");
            asm volatile("prefetch.tensormap [%0];" ::"l"(tm_64) : "memory");
        }
        const char *Bbytes = static_cast<const char *>(p.B);
        const long long pitch = p.ldb * G::ES;
        for (int u = blockIdx.x; ok && u < p.n_units; u += gridDim.x) {
            const int win = u / p.nfb;  // task
            const bool first = u == (int)blockIdx.x;
            const int4 w = first ? w_first : p.tasks[win];
            const int c0 = first ? c_first : p.dense_c0[win];
            const int n0 = (u % p.nfb) * MB;
            const int nst = (w.z + G::TPS - 1) / G::TPS;  // stages of this unit (w.z >= 1)
            const int rot = win % nst;
            if (c0 == -1 && FMT != 2) {
                // Gathered 16-bit tiles through cp.async: thread ptid copies the
                // 16-byte chunk cc = ptid % 16 of B rows k = ptid / 16 + ROW_STEP i.
                // The B-row indices are loaded IDX_AHEAD stages ahead, one per lane:
                // lane j < 2 ROW_PASSES of producer warp pw holds the index of the
                // stage's row 2 pw + j % 2 + ROW_STEP (j / 2), which lanes
                // 16 (j % 2) .. + 15 of the warp copy in pass j / 2, and hands it to
                // them by a shuffle.  So issuing a stage never waits on an index load.
                const int cc = ptid & 15, pc = cc >> 3, c = cc & 7;
                const int col = n0 + cc * 8;  // first of the chunk's 8 columns
                const bool colok = col < p.ncols;
                const int jr = 2 * pw + (lane & 1) + ROW_STEP * (lane >> 1);
                auto load_row = [&](int k) -> int {
                    if (k >= nst || lane >= 2 * ROW_PASSES) return 0;
                    const int t = stage_at(k, rot, nst) * G::TPS;
                    const int rows = min(G::TPS, w.z - t) * KT;
                    return jr < rows ? __ldg(p.tile_cols + ((long long)w.y + t) * KT + jr) : 0;
                };
                static_assert(IDX_AHEAD == 3, "the index ring below holds three stages");
                int ia = load_row(0), ib = load_row(1), ic = load_row(2);
                for (int k = 0; k < nst; ++k, ++g) {
                    const int t = stage_at(k, rot, nst) * G::TPS;
                    const int s = g % STAGES;
                    const int n = min(G::TPS, w.z - t);
                    const int cur = ia;
                    ia = ib;
                    ib = ic;
                    ic = load_row(k + IDX_AHEAD);
                    // Abort decisions stay warp-uniform (the lanes of a producer warp
                    // walk the same stages).
                    ok = __all_sync(0xffffffffu, wait_bounded(smem_u32(&empty[s]), ((g / STAGES) & 1) ^ 1,
                                                              abort_flag, p.err, 1, p.wait_cycles));
                    if (!ok) break;
                    tma_mine &= ~(1u << s);
                    if (p.stall_test) continue;  // self-test: nothing copied, nothing arrives
                    const uint32_t panel = smem_u32(smem + s * STAGE_BYTES);
                    const int rows = n * KT;
#pragma unroll
                    for (int i = 0; i < ROW_PASSES; ++i) {
                        const int kr = (ptid >> 4) + ROW_STEP * i;
                        const int brow = __shfl_sync(0xffffffffu, cur, 2 * i + (lane >> 4));
                        if (kr < rows) {
                            const uint32_t dst = panel + pc * G::PIECE + (kr >> 3) * 1024 + (kr & 7) * 128 +
                                                 ((c ^ (kr & 7)) << 4);
                            const char *src = colok ? Bbytes + (long long)brow * pitch + (long long)col * G::ES
                                                    : Bbytes;
                            cp_async16(dst, src, colok ? 16u : 0u);
                        }
                    }
                    const uint8_t *vsrc = p.tile_vals + ((long long)w.y + t) * G::TILE_VAL;
                    for (int q = ptid; q < n * (G::TILE_VAL / 16); q += PTHREADS)
                        cp_async16(panel + PANEL_BYTES + q * 16, vsrc + q * 16, 16u);
                    cp_async_arrive_noinc(smem_u32(&full[s]));
                }
                continue;
            }
            if (c0 >= 0) {
                // One consecutive run of columns c0, c0 + 1, ...: tile t covers B
                // rows c0 + 16 t .. + 15 (rows past the run have zero values, rows
                // past K are zero-filled by TMA), so no indices are loaded.
                for (int k = 0; ok && k < nst; ++k, ++g) {
                    tma_mine &= ~(1u << (g % STAGES));
                    if ((int)(g % NPROD) != pw) continue;
                    const int t = stage_at(k, rot, nst) * G::TPS;
                    const int s = g % STAGES;
                    const int n = min(G::TPS, w.z - t);
                    ok = __all_sync(0xffffffffu, wait_bounded(smem_u32(&empty[s]), ((g / STAGES) & 1) ^ 1,
                                                              abort_flag, p.err, 1, p.wait_cycles));
                    if (!ok) break;
                    if (lane == 0 && !p.stall_test) {
                        const uint32_t fb = smem_u32(&full[s]);
                        const uint32_t panel = smem_u32(smem + s * STAGE_BYTES);
                        const int y = c0 + t * KT;
                        mbar_expect_tx(fb, (uint32_t)n * (G::TILE_PANEL + G::TILE_VAL));
                        // One box of a whole stage only when all its rows lie inside B;
                        // a stage that runs past the last row takes a box per tile.
                        if (n == G::TPS && y + G::SROWS <= p.K) {
#pragma unroll
                            for (int c = 0; c < G::NPC; ++c) tma_box(panel + c * G::PIECE, tm_64, n0 + c * G::CPB, y, fb);
                        } else {
                            for (int j = 0; j < n; ++j)
#pragma unroll
                                for (int c = 0; c < G::NPC; ++c)
                                    tma_box(panel + c * G::PIECE + j * 2048, tm_16, n0 + c * G::CPB, y + j * KT, fb);
                        }
                        bulk_copy(panel + PANEL_BYTES, p.tile_vals + ((long long)w.y + t) * G::TILE_VAL,
                                  (uint32_t)n * G::TILE_VAL, fb);
                        mbar_arrive_n(fb, PTHREADS - 1);
                        tma_mine |= 1u << s;
                    }
                }
                continue;
            }
            // Tile indices in IDX_TILES-tile chunks, two buffers a warp: when the
            // stages reach a new chunk, the chunk after it in this task's stage
            // order is fetched by cp.async into the other buffer, so its load
            // overlaps a chunk's worth of stages (a task's first chunk is waited for).
            constexpr int SPC = IDX_TILES / G::TPS;  // stages a chunk
            int chunk = -1, pre = -1, cur = 0;       // staged chunk, chunk in flight, buffer of `chunk`
            const int32_t *myidx = mybufs;
            auto fetch = [&](int ch, int32_t *dst) {
                const int t0 = ch * IDX_TILES, n16 = min(IDX_TILES, w.z - t0) * (KT / 4);
                const int32_t *src = p.tile_cols + ((long long)w.y + t0) * KT;
                for (int q = lane; q < n16; q += 32) cp_async16(smem_u32(dst + 4 * q), src + 4 * q, 16u);
            };
            for (int k = 0; ok && k < nst; ++k, ++g) {
                const int sk = stage_at(k, rot, nst);
                const int t = sk * G::TPS;  // first tile of the stage
                if (t / IDX_TILES != chunk) {
                    chunk = t / IDX_TILES;
                    __syncwarp();  // previous indices consumed
                    if (chunk == pre) {
                        cur ^= 1;
                    } else {
                        // Not prefetched: any copy still landing in a buffer ends first.
                        asm volatile("cp.async.wait_all;" ::: "memory");
                        fetch(chunk, mybufs + cur * IDX_INTS);
                    }
                    asm volatile("cp.async.wait_all;" ::: "memory");
                    __syncwarp();  // indices visible to the warp
                    myidx = mybufs + cur * IDX_INTS;
                    // This chunk's run of stages ends at its last stage or the task's;
                    // the stage after the run starts the next chunk.
                    const int k2 = k + min((chunk + 1) * SPC, nst) - sk;
                    pre = -1;
                    if (k2 < nst) {
                        pre = stage_at(k2, rot, nst) / SPC;
                        fetch(pre, mybufs + (cur ^ 1) * IDX_INTS);
                    }
                }
                tma_mine &= ~(1u << (g % STAGES));
                if ((int)(g % NPROD) != pw) continue;
                const int s = g % STAGES;
                const int n = min(G::TPS, w.z - t);  // tiles in this stage
                ok = __all_sync(0xffffffffu, wait_bounded(smem_u32(&empty[s]), ((g / STAGES) & 1) ^ 1, abort_flag,
                                                          p.err, 1, p.wait_cycles));
                if (!ok) break;
                if (lane == 0 && !p.stall_test) {
                    const uint32_t fb = smem_u32(&full[s]);
                    const uint32_t panel = smem_u32(smem + s * STAGE_BYTES);
                    const int32_t *ix = myidx + (t - chunk * IDX_TILES) * KT;
                    mbar_expect_tx(fb, (uint32_t)n * (G::TILE_PANEL + G::TILE_VAL));
                    // A window's columns ascend, distinct except the padding of
                    // its last tile, which repeats the last column.  So m
                    // indices whose span is m - 1 and whose last two differ
                    // are m consecutive B rows.
                    if (n == G::TPS && ix[G::SROWS - 1] - ix[0] == G::SROWS - 1 && ix[G::SROWS - 2] != ix[G::SROWS - 1]) {
#pragma unroll
                        for (int c = 0; c < G::NPC; ++c) tma_box(panel + c * G::PIECE, tm_64, n0 + c * G::CPB, ix[0], fb);
                    } else {
                        for (int j = 0; j < n; ++j) {
                            const int32_t *jx = ix + j * KT;
                            const uint32_t tp = panel + j * 2048;
                            if (jx[KT - 1] - jx[0] == KT - 1 && jx[KT - 2] != jx[KT - 1]) {
#pragma unroll
                                for (int c = 0; c < G::NPC; ++c)
                                    tma_box(tp + c * G::PIECE, tm_16, n0 + c * G::CPB, jx[0], fb);
                            } else {
#pragma unroll
                                for (int c = 0; c < G::NPC; ++c)
#pragma unroll
                                    for (int q = 0; q < 4; ++q)
                                        tma_gather4(tp + c * G::PIECE + (q >> 1) * 1024 + (q & 1) * 512, tm_g,
                                                    n0 + c * G::CPB, jx[4 * q], jx[4 * q + 1], jx[4 * q + 2],
                                                    jx[4 * q + 3], fb);
                            }
                        }
                    }
                    bulk_copy(panel + PANEL_BYTES, p.tile_vals + ((long long)w.y + t) * G::TILE_VAL,
                              (uint32_t)n * G::TILE_VAL, fb);
                    mbar_arrive_n(fb, PTHREADS - 1);
                    tma_mine |= 1u << s;
                }
            }
        }
        // Drain: this thread's cp.async copies have landed, and the TMA copies
        // this lane issued for the last STAGES stages, before the CTA may exit
        // (already true unless the kernel is aborting).
        asm volatile("cp.async.wait_all;" ::: "memory");
        if (!p.stall_test) {
            int no_abort = 0;
            for (uint32_t k = g > (uint32_t)STAGES ? g - STAGES : 0; k < g; ++k)
                if ((tma_mine >> (k % STAGES)) & 1u)
                    wait_bounded(smem_u32(&full[k % STAGES]), (k / STAGES) & 1, (volatile int *)&no_abort, p.err, 16,
                                 p.wait_cycles);
        }
        __syncwarp();
    } else if (warp == 4) {
        // ------------------------------ MMA issuer -----------------------------
        if (lane == 0) {
            constexpr uint32_t idesc = instr_desc<FMT>();
            uint32_t g = 0, i = 0;
            bool ok = true;
            // Task descriptors (and whether the producers fill the task's stages
            // through cp.async) are loaded one task ahead.
            const bool first_ok = (int)blockIdx.x < p.n_units;
            int4 wn = first_ok ? p.tasks[blockIdx.x / p.nfb] : make_int4(0, 0, 1, 0);
            bool cpn = FMT != 2 && first_ok && p.dense_c0[blockIdx.x / p.nfb] == -1;
            for (int u = blockIdx.x; ok && u < p.n_units; u += gridDim.x, ++i) {
                const int4 w = wn;
                const bool cp = cpn;
                if (u + (int)gridDim.x < p.n_units) {
                    wn = p.tasks[(u + gridDim.x) / p.nfb];
                    cpn = FMT != 2 && p.dense_c0[(u + gridDim.x) / p.nfb] == -1;
                }
                const uint32_t a = i & 1;
                if (!wait_bounded(smem_u32(&acce[a]), ((i >> 1) & 1) ^ 1, abort_flag, p.err, 2, p.wait_cycles)) break;
                tc_fence_after();
                const uint32_t dcol = tmem + a * R;
                // Stages in the producer's order: TPS tiles each, starting at
                // the window's stage offset.
                const int nst = (w.z + G::TPS - 1) / G::TPS;
                const int rot = (u / p.nfb) % nst;
                for (int k = 0; k < nst; ++k, ++g) {
                    const int s = g % STAGES;
                    const int t = stage_at(k, rot, nst) * G::TPS;
                    const int n = min(G::TPS, w.z - t);
                    if (!wait_bounded(smem_u32(&full[s]), (g / STAGES) & 1, abort_flag, p.err, 2, p.wait_cycles)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    if (cp) fence_proxy_async();  // cp.async (generic proxy) writes -> tensor-core reads
                    const uint32_t panel = smem_u32(smem + s * STAGE_BYTES);
                    for (int j = 0; j < n; ++j) {
#pragma unroll
                        for (int h = 0; h < KT / G::KSTEP; ++h) {
                            // A: MN-major, 128-byte swizzle, pieces LBO apart, 8-row
                            // atoms SBO apart; B: K-major, no swizzle, 16-byte k chunks
                            // LBO apart, 8-row groups SBO apart.
                            const uint64_t adesc =
                                smem_desc(panel + j * 2048 + h * (G::KSTEP / 8) * 1024, G::PIECE, G::KGROUP, G::LAYOUT);
                            const uint64_t bdesc = smem_desc(
                                panel + PANEL_BYTES + j * G::TILE_VAL + h * (G::KSTEP * G::ES / 16) * 128, 128,
                                G::KCH * 128, 0);
                            mma_issue<FMT>(dcol, adesc, bdesc, idesc, (k | j | h) != 0 ? 1u : 0u);
                        }
                    }
                    mma_commit(smem_u32(&empty[s]));
                }
                if (!ok) break;
                mma_commit(smem_u32(&accf[a]));
            }
            // Drain: every MMA issued above has completed once `drain` flips.
            mma_commit(smem_u32(drain));
            int dummy = 0;
            wait_bounded(smem_u32(drain), 0, (volatile int *)&dummy, p.err, 8, p.wait_cycles);
        }
        __syncwarp();
    } else if (warp < 4) {
        // ------------------------------ epilogue -------------------------------
        uint32_t i = 0;
        for (int u = blockIdx.x; u < p.n_units; u += gridDim.x, ++i) {
            const int t = u / p.nfb, fb = u % p.nfb;
            // The task's descriptor, split and row ids load while the MMAs run.
            const int4 w = p.tasks[t];
            const int4 sp = p.splits[t];
            // C row of the window's row `lane` (gathered windows read their row list).
            const int rid = w.x >= 0 ? w.x + lane : (lane < w.w ? __ldg(p.rows + (-(w.x + 1)) + lane) : 0);
            const uint32_t a = i & 1;
            if (!__all_sync(0xffffffffu,
                            wait_bounded(smem_u32(&accf[a]), (i >> 1) & 1, abort_flag, p.err, 4, p.wait_cycles)))
                break;
            tc_fence_after();
            float v[32];
            tmem_ld32(tmem + ((uint32_t)(warp * 32) << 16) + a * R, v);
            tc_fence_before();
            mbar_arrive(smem_u32(&acce[a]));
            if (sp.x >= 0) {
                // One part of a split window: publish this warp's 32 x 32 partial
                // tile and count it in; the warp that completes the window's last
                // part sums all parts in part order and writes C.
                float *mine = p.partials + ((((long long)(sp.w + sp.y) * p.nfb + fb) * 4 + warp) << 10);
#pragma unroll
                for (int r = 0; r < R; ++r) __stcg(mine + r * 32 + lane, v[r]);
                __threadfence();
                __syncwarp();
                unsigned int *cnt = p.counters + ((long long)sp.x * p.nfb + fb) * 4 + warp;
                unsigned int prev = 0;
                if (lane == 0) prev = atomicAdd(cnt, 1u);
                prev = __shfl_sync(0xffffffffu, prev, 0);
                if (prev + 1 != (unsigned int)sp.z) continue;
                __threadfence();
#pragma unroll
                for (int r = 0; r < R; ++r) v[r] = 0.0f;
                for (int q = 0; q < sp.z; ++q) {
                    const float *part = p.partials + ((((long long)(sp.w + q) * p.nfb + fb) * 4 + warp) << 10);
#pragma unroll
                    for (int r = 0; r < R; ++r) v[r] += __ldcg(part + r * 32 + lane);
                }
                if (lane == 0) *cnt = 0u;  // ready for the next launch
            }
            if (p.has_ep && p.ep.row_scale) {
                // One load of the window's row scales, then a broadcast per row
                // (all lanes converged here).
                const float sc = lane < w.w ? __ldg(p.ep.row_scale + rid) : 1.0f;
#pragma unroll
                for (int r = 0; r < R; ++r) v[r] *= __shfl_sync(0xffffffffu, sc, r);
            }
            const int x = fb * MB + warp * 32;  // this warp's first output column
            const int f = x + lane;
            if (p.tma_store && w.x >= 0) {
                // Stage the warp's 32 x 32 tile in shared memory (row r at
                // 32 r elements, conflict-free), then one bulk tensor store; the
                // tensor map clips rows past the block's end and columns past N.
                if (x < p.ncols) {  // warp-uniform
                    if (lane == 0) bulk_wait_read();  // the previous store has read the buffer
                    __syncwarp();
                    uint8_t *cw = cbuf + warp * 4096;
                    if (!p.has_ep) {
#pragma unroll
                        for (int r = 0; r < R; ++r) reinterpret_cast<float *>(cw)[r * 32 + lane] = v[r];
                    } else {
                        const float b = (p.ep.bias && f < p.ncols) ? __ldg(p.ep.bias + f) : 0.0f;
#pragma unroll
                        for (int r = 0; r < R; ++r) {
                            float y = v[r] + b;
                            if (p.ep.relu) y = fmaxf(y, 0.0f);
                            if (p.ep.out == 0)
                                reinterpret_cast<float *>(cw)[r * 32 + lane] = y;
                            else if (p.ep.out == 1)
                                reinterpret_cast<__half *>(cw)[r * 32 + lane] = __float2half_rn(y);
                            else
                                reinterpret_cast<__nv_bfloat16 *>(cw)[r * 32 + lane] = __float2bfloat16_rn(y);
                        }
                    }
                    fence_proxy_async();  // generic-proxy writes -> visible to the bulk copy
                    __syncwarp();
                    if (lane == 0) {
                        tma_store_2d(&cmap, x, w.x, smem_u32(cw));
                        bulk_commit();
                    }
                }
            } else if (x < p.ncols) {  // warp-uniform
                epilogue_rows(p, rid, w.w, f, v);
            }
        }
        if (p.tma_store && lane == 0) bulk_wait_all();  // C is written before the CTA exits
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
constexpr size_t kSmemBytes =
    1024 + STAGES * STAGE_BYTES + CBUF_BYTES + NPROD * 2 * IDX_INTS * 4 + (kBarBytes + 127) / 128 * 128;  // ~104 KB: two CTAs per SM

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

// cuTensorMapEncodeTiled from the driver, looked up once through the runtime
// (no link-time dependency on libcuda).
typedef CUresult (*EncodeTiledFn)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *, const cuuint64_t *,
                                  const cuuint64_t *, const cuuint32_t *, const cuuint32_t *, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn()
{
    static EncodeTiledFn fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void *f = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &f, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = (EncodeTiledFn)f;
    });
    return fn;
}

// The kernel's element format for a plan dtype: 0 fp16, 1 bf16, 2 tf32.
int fmt_of(tcaspmm_dtype dt) { return dt == TCASPMM_BF16 ? 1 : dt == TCASPMM_TF32 ? 2 : 0; }

// Tensor maps over a B block of ncols columns x K rows (x = column, zero fill
// beyond ncols; y = B row), 128-byte swizzle, boxes of one 128-byte piece (64
// 16-bit or 32 fp32 columns) x 1, 16 and one stage of rows (64 or 32).
tcaspmm_status encode_b_maps(tcaspmm_dtype dt, const void *dB, int64_t ncols, int64_t K, int64_t ldb, BMaps *m)
{
    EncodeTiledFn fn = encode_fn();
    if (!fn) return fail(TCASPMM_ERR_CUDA, "cuTensorMapEncodeTiled is not available from the driver");
    const int fmt = fmt_of(dt);
    const int es = fmt == 2 ? 4 : 2;
    const cuuint32_t cpb = 128 / es, srows = fmt == 2 ? Geo<2>::SROWS : Geo<0>::SROWS;
    const cuuint64_t dims[2] = {(cuuint64_t)ncols, (cuuint64_t)K};
    const cuuint64_t strides[1] = {(cuuint64_t)(ldb * es)};
    const cuuint32_t estr[2] = {1, 1};
    const CUtensorMapDataType ty = fmt == 1   ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16
                                   : fmt == 2 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32
                                              : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
    // Boxes of 16 / one stage of rows are used only where that many consecutive
    // B rows exist, so on a B of fewer rows they are clipped to K (never issued).
    const cuuint32_t k16 = (cuuint32_t)std::min<int64_t>(KT, K), ks = (cuuint32_t)std::min<int64_t>(srows, K);
    const cuuint32_t boxes[3][2] = {{cpb, 1}, {cpb, k16}, {cpb, ks}};
    CUtensorMap *maps[3] = {&m->gather, &m->box16, &m->box64};
    CUresult r = CUDA_SUCCESS;
    const CUtensorMapSwizzle sw = fmt == 2 ? CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B : CU_TENSOR_MAP_SWIZZLE_128B;
    for (int i = 0; i < 3 && r == CUDA_SUCCESS; ++i)
        r = fn(maps[i], ty, 2, const_cast<void *>(dB), dims, strides, boxes[i], estr, CU_TENSOR_MAP_INTERLEAVE_NONE, sw,
               CU_TENSOR_MAP_L2_PROMOTION_L2_128B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS ? TCASPMM_OK : fail(TCASPMM_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d)", (int)r);
}

static_assert(sizeof(BMaps) <= sizeof(Shard::maps) && sizeof(CUtensorMap) <= sizeof(Shard::cmap), "tensor-map storage in Shard");

template <int FMT>
cudaError_t smem_optin()
{
    cudaError_t e = cudaFuncSetAttribute(tc_kernel<FMT>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kSmemBytes);
    // The largest shared-memory carveout, so two CTAs of ~104 KB can be resident
    // on an SM (left to itself the driver configures 135 KB: one CTA).
    if (e == cudaSuccess)
        e = cudaFuncSetAttribute(tc_kernel<FMT>, cudaFuncAttributePreferredSharedMemoryCarveout,
                                 (int)cudaSharedmemCarveoutMaxShared);
    return e;
}

void launch_kernel(int fmt, int grid, const TcParams &p, const BMaps &maps, const CUtensorMap &cmap, cudaStream_t st)
{
    if (fmt == 1)
        tc_kernel<1><<<grid, NUM_THREADS, kSmemBytes, st>>>(p, maps, cmap);
    else if (fmt == 2)
        tc_kernel<2><<<grid, NUM_THREADS, kSmemBytes, st>>>(p, maps, cmap);
    else
        tc_kernel<0><<<grid, NUM_THREADS, kSmemBytes, st>>>(p, maps, cmap);
}

// Tensor map over a C block of ncols x rows elements of the output type (ldc
// elements per row), box 32 x 32, no swizzle: the epilogue's bulk stores.
tcaspmm_status encode_c_map(int out, void *dC, int64_t ncols, int64_t rows, int64_t ldc, CUtensorMap *m)
{
    EncodeTiledFn fn = encode_fn();
    if (!fn) return fail(TCASPMM_ERR_CUDA, "cuTensorMapEncodeTiled is not available from the driver");
    const int esize = out == 0 ? 4 : 2;
    const cuuint64_t dims[2] = {(cuuint64_t)ncols, (cuuint64_t)rows};
    const cuuint64_t strides[1] = {(cuuint64_t)(ldc * esize)};
    const cuuint32_t box[2] = {32, 32}, estr[2] = {1, 1};
    const CUtensorMapDataType ty = out == 0   ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32
                                   : out == 1 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16
                                              : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
    const CUresult r = fn(m, ty, 2, dC, dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                          CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_NONE, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS ? TCASPMM_OK : fail(TCASPMM_ERR_CUDA, "cuTensorMapEncodeTiled (C) failed (%d)", (int)r);
}

}  // namespace

bool tc_supported()
{
    int dev = 0, major = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return false;
    if (cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev) != cudaSuccess) return false;
    return major == 10;
}

// Tiles per task of a gathered window: its tile chain is cut into parts of at
// most this many tiles (about 32 pipeline stages), so a hub window's work spreads
// over many CTAs while each part still amortises its epilogue.  The tuning
// variable TCASPMM_SPLIT_TILES (clamped to [1, 4096]) overrides it.
constexpr int SPLIT_TILES = 128;
// Fewest pipeline stages in a part of a consecutive window cut for idle SMs: a
// part's epilogue and reduction cost about a stage.
constexpr int MIN_PART_STAGES = 4;

tcaspmm_status tc_upload(const tcaspmm_csr &A, tcaspmm_dtype dt, Shard *sh)
{
    const TileSchedule &T = sh->sched.tc;
    sh->n_windows = (int)T.windows.size();
    if (sh->n_windows == 0) return TCASPMM_OK;
    if (T.R != R || T.KT != KT) return fail(TCASPMM_ERR_UNSUPPORTED, "tile shape %dx%d not built", T.R, T.KT);
    // Windows whose columns are one consecutive run (padding repeats the last
    // column) need no index loads: their tiles are boxes of consecutive B rows.
    // Only when K >= 64, so that the 64- and 16-row boxes are never clipped.
    auto dense_run = [&](const Int4 &w) -> int32_t {
        if (sh->K < 64) return -1;
        const int32_t *c = T.tile_cols.data() + (size_t)w.y * KT;
        const int64_t n = (int64_t)w.z * KT;
        int64_t q = 1;
        for (; q < n && c[q] == c[0] + q; q++) {
        }
        for (; q < n; q++)
            if (c[q] != c[q - 1]) return -1;  // not padding
        return c[0];
    };
    // Tasks: consecutive windows whole; gathered windows in parts of at most
    // SPLIT_TILES tiles (a window of one part needs no reduction).
    struct Task {
        Int4 d, sp;
        int32_t dense;
    };
    int nsm = 148;
    cudaDeviceGetAttribute(&nsm, cudaDevAttrMultiProcessorCount, sh->device);
    sh->num_sms = nsm;
    std::vector<Task> tasks;
    int32_t groups = 0, slots = 0;
    const int split = (int)env_int("TCASPMM_SPLIT_TILES", SPLIT_TILES, 1, 4096);
    // Consecutive windows: when their work items (with the gathered windows'
    // parts, per column block) leave SMs without one, each tile chain is cut into
    // up to SMs / items parts of at least MIN_PART_STAGES stages, so a few long
    // chains spread over idle SMs; otherwise they stay whole (one CTA per SM
    // streams a chain as fast as two half chains).  TCASPMM_WINDOW_PARTS (clamped
    // to [0, 64], 0 = this rule) sets the parts instead, at most one per stage.  A
    // part of a consecutive column run starts 16 t0 columns in.
    const int64_t nfb = (sh->ncols + MB - 1) / MB;
    int64_t items = 0;
    for (const Int4 &w : T.windows) items += w.x >= 0 ? 1 : (w.z + split - 1) / split;
    items *= nfb;
    const int auto_parts = items > 0 ? (int)std::min<int64_t>(64, std::max<int64_t>(1, nsm / items)) : 1;
    const int env_parts = (int)env_int("TCASPMM_WINDOW_PARTS", 0, 0, 64);
    // TCASPMM_DENSE_RUNS=0 sends consecutive column runs through the gathered
    // path (tile indices and the gathered-tile producer) instead of TMA boxes.
    const bool dense_runs = env_flag("TCASPMM_DENSE_RUNS", true);
    // Gathered 16-bit tiles are fetched by TMA gather4 (as TF32 tiles are);
    // TCASPMM_GATHER_TMA=0 fetches them by cp.async from all producer threads
    // (measured slower: C2 at 80% sparsity 45 against 25 us, C3 gathered
    // windows 1.64 against 1.53 ms).
    const int32_t gathered = env_flag("TCASPMM_GATHER_TMA", true) ? -2 : -1;
    for (const Int4 &w : T.windows) {
        const int stages = (w.z + Geo<0>::TPS - 1) / Geo<0>::TPS;
        const int parts = w.x < 0       ? (w.z + split - 1) / split
                          : env_parts > 0 ? std::max(1, std::min(env_parts, stages))
                                          : std::max(1, std::min(auto_parts, stages / MIN_PART_STAGES));
        const int32_t run = w.x >= 0 && dense_runs ? dense_run(w) : -1;
        const int32_t dense = run >= 0 ? run : gathered;
        if (parts == 1) {
            tasks.push_back(Task{w, Int4{-1, 0, 1, 0}, dense});
            continue;
        }
        for (int q = 0; q < parts; q++) {
            const int32_t t0 = (int32_t)((int64_t)w.z * q / parts), t1 = (int32_t)((int64_t)w.z * (q + 1) / parts);
            tasks.push_back(Task{Int4{w.x, w.y + t0, t1 - t0, w.w}, Int4{groups, q, parts, slots},
                                 dense >= 0 ? dense + t0 * KT : dense});
        }
        groups++;
        slots += parts;
    }
    // Tasks by decreasing tile count, so the persistent grid balances (sorted on
    // the host, so the kernel reads a unit's task with one load).
    std::stable_sort(tasks.begin(), tasks.end(), [](const Task &a, const Task &b) { return a.d.z > b.d.z; });
    std::vector<Int4> td(tasks.size()), ts(tasks.size());
    std::vector<int32_t> dense(tasks.size());
    for (size_t i = 0; i < tasks.size(); i++) {
        td[i] = tasks[i].d;
        ts[i] = tasks[i].sp;
        dense[i] = tasks[i].dense;
    }
    sh->n_tasks = (int)tasks.size();
    sh->n_split_groups = groups;
    // Value tiles -> shared-memory image (K-major, no swizzle): core matrices of
    // 8 rows x 16 bytes, 16-byte k chunks 128 B apart (LBO), 8-row groups
    // kch * 128 B apart (SBO); fp16 / bf16 bits, or fp32 bits for tf32.
    // Each nonzero of a window's row i lands at (tile, k) = the position of its
    // column among the window's condensed columns; every other cell is zero.
    const int es = dtype_size(dt), kch = KT * es / 16, tile_bytes = R * KT * es;
    const size_t ntiles = T.tile_cols.size() / KT;
    std::vector<uint8_t> img(ntiles * tile_bytes, 0);
#pragma omp parallel for schedule(dynamic, 1)
    for (int64_t wi = 0; wi < (int64_t)T.windows.size(); wi++) {
        const Int4 &w = T.windows[wi];
        const int32_t *cols = T.tile_cols.data() + (size_t)w.y * KT;
        const int64_t ncond = (int64_t)w.z * KT;
        for (int n = 0; n < w.w; n++) {
            const int64_t r = T.row(w, n);
            for (int64_t j = A.row_ptr[r]; j < A.row_ptr[r + 1]; j++) {
                const int64_t q = std::lower_bound(cols, cols + ncond, A.col_idx[j]) - cols;
                const int64_t t = w.y + q / KT, k = q % KT;
                const float v = A.val ? A.val[j] : 1.0f;
                uint8_t *dst = img.data() + t * tile_bytes + (n / 8) * (kch * 128) + (k * es / 16) * 128 +
                               (n % 8) * 16 + (k * es) % 16;
                if (es == 4) {
                    std::memcpy(dst, &v, 4);
                } else {
                    const uint16_t h = dt == TCASPMM_BF16 ? float_to_bf16_bits(v) : float_to_half_bits(v);
                    std::memcpy(dst, &h, 2);
                }
            }
        }
    }
    // Fallback row ranges over the tc rows (run on the CUDA cores when B is not
    // 16-byte aligned at execute time): a consecutive window is one range, a
    // gathered window one range per row.
    std::vector<Int2> fb;
    for (const Int4 &w : T.windows) {
        if (w.x >= 0) {
            fb.push_back(Int2{w.x, w.x + w.w});
        } else {
            for (int i = 0; i < w.w; i++) fb.push_back(Int2{T.row(w, i), T.row(w, i) + 1});
        }
    }
    sh->n_fallback = (int)fb.size();
    tcaspmm_status s;
    if ((s = upload_vec(sh, &sh->tc_tasks, td, "tc tasks")) != TCASPMM_OK) return s;
    if ((s = upload_vec(sh, &sh->tc_splits, ts, "tc splits")) != TCASPMM_OK) return s;
    if ((s = upload_vec(sh, &sh->tc_dense, dense, "tc dense runs")) != TCASPMM_OK) return s;
    if ((s = upload_vec(sh, &sh->tc_rows, T.rows, "tc row lists")) != TCASPMM_OK) return s;
    if ((s = upload_vec(sh, &sh->tc_cols, T.tile_cols, "tc columns")) != TCASPMM_OK) return s;
    if ((s = upload_vec(sh, (uint8_t **)&sh->tc_vals, img, "tc values")) != TCASPMM_OK) return s;
    if ((s = upload_vec(sh, &sh->tc_fallback, fb, "tc fallback ranges")) != TCASPMM_OK) return s;
    if (slots > 0) {
        // Partial tiles: [slot][column block][4 epilogue warps][32 x 32] fp32, and
        // one counter per (split window, column block, epilogue warp).
        if ((s = upload_vec(sh, &sh->tc_counters, std::vector<unsigned int>((size_t)groups * nfb * 4, 0u),
                            "tc split counters")) != TCASPMM_OK)
            return s;
        const size_t pbytes = (size_t)slots * nfb * 4 * 1024 * sizeof(float);
        cudaError_t e = cudaMalloc((void **)&sh->tc_partials, pbytes);
        if (e != cudaSuccess) {
            sh->tc_partials = nullptr;
            return fail(TCASPMM_ERR_ALLOC, "cudaMalloc of %zu bytes for tc partial tiles failed: %s", pbytes,
                        cudaGetErrorString(e));
        }
        sh->allocs.push_back(sh->tc_partials);
        sh->bytes += (int64_t)pbytes;
    }
    // More than 48 KB of dynamic shared memory needs the opt-in, per device.
    cudaError_t e = smem_optin<0>();
    if (e == cudaSuccess) e = smem_optin<1>();
    if (e == cudaSuccess) e = smem_optin<2>();
    int per_sm = 0;
    if (e == cudaSuccess)
        e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, tc_kernel<0>, NUM_THREADS, kSmemBytes);
    // The occupancy query does not see the carveout preference set above (it
    // answers 1 where ncu reports two resident CTAs), so the residency the SM's
    // shared memory and register file allow is computed here as well, and the
    // larger figure (at most 2) sizes the persistent grid.
    if (e == cudaSuccess) {
        int smem_sm = 0, reserved = 0, regs_sm = 0;
        cudaFuncAttributes fa{};
        if (cudaDeviceGetAttribute(&smem_sm, cudaDevAttrMaxSharedMemoryPerMultiprocessor, sh->device) ==
                cudaSuccess &&
            cudaDeviceGetAttribute(&reserved, cudaDevAttrReservedSharedMemoryPerBlock, sh->device) == cudaSuccess &&
            cudaDeviceGetAttribute(&regs_sm, cudaDevAttrMaxRegistersPerMultiprocessor, sh->device) == cudaSuccess &&
            cudaFuncGetAttributes(&fa, tc_kernel<0>) == cudaSuccess && fa.numRegs > 0) {
            const int by_smem = smem_sm / ((int)kSmemBytes + reserved);
            const int by_regs = regs_sm / (NUM_THREADS * ((fa.numRegs + 7) / 8 * 8));
            per_sm = std::max(per_sm, std::min(2, std::min(by_smem, by_regs)));
        }
        cudaGetLastError();
    }
    sh->tc_ctas_per_sm = std::max(1, per_sm);
    return e == cudaSuccess ? TCASPMM_OK : cuda_fail(e, "tc kernel shared-memory opt-in");
}

tcaspmm_status launch_tc(const Shard &sh, tcaspmm_dtype dt, const void *dB, int64_t ldb, void *dC, int64_t ldc,
                         const Epilogue *ep, cudaStream_t st)
{
    if (sh.n_tasks == 0 || sh.ncols == 0) return TCASPMM_OK;
    const bool aligned = ((uintptr_t)dB % 16 == 0) && ((ldb * dtype_size(dt)) % 16 == 0) && (sh.ncols % 8 == 0);
    if (!aligned)  // CUDA-core fallback over the tc rows: whole rows, no segments
        return launch_residue(sh, dt, dB, ldb, dC, ldc, ep, st, sh.tc_fallback, sh.n_fallback);
    TcParams p;
    p.tasks = (const int4 *)sh.tc_tasks;
    p.splits = (const int4 *)sh.tc_splits;
    p.rows = sh.tc_rows;
    p.partials = sh.tc_partials;
    p.counters = sh.tc_counters;
    p.dense_c0 = sh.tc_dense;
    p.tile_cols = sh.tc_cols;
    p.tile_vals = (const uint8_t *)sh.tc_vals;
    p.B = dB;
    p.ldb = ldb;
    p.C = dC;
    p.ldc = ldc;
    p.ncols = (int)sh.ncols;
    p.K = (int)sh.K;
    p.nfb = (int)((sh.ncols + MB - 1) / MB);
    p.n_units = sh.n_tasks * p.nfb;
    p.err = sh.err;
    p.wait_cycles = WAIT_CYCLES;
    p.stall_test = 0;
    p.has_ep = ep != nullptr;
    p.ep = ep ? EpiParams{ep->row_scale, ep->bias, ep->relu, ep->out} : EpiParams{nullptr, nullptr, 0, 0};
    // Bulk tensor stores of C need a 16-byte aligned C with 16-byte row pitch;
    // the C tensor map is rebuilt only when C, its pitch or its type change.
    const int out = ep ? ep->out : 0;
    const int esize = out == 0 ? 4 : 2;
    p.tma_store = ((uintptr_t)dC % 16 == 0) && ((ldc * esize) % 16 == 0);
    if (p.tma_store && !(sh.cmap_valid && sh.cmap_ptr == dC && sh.cmap_ldc == ldc && sh.cmap_out == out)) {
        sh.cmap_valid = false;
        tcaspmm_status ms = encode_c_map(out, dC, sh.ncols, sh.nrows, ldc, (CUtensorMap *)sh.cmap);
        if (ms != TCASPMM_OK) return ms;
        sh.cmap_valid = true;
        sh.cmap_ptr = dC;
        sh.cmap_ldc = ldc;
        sh.cmap_out = out;
    }
    const int grid = std::min(p.n_units, sh.tc_ctas_per_sm * sh.num_sms);  // persistent
    // Tensor maps depend on the B block: rebuilt only when it changes.
    if (!(sh.maps_valid && sh.maps_ptr == dB && sh.maps_ldb == ldb)) {
        sh.maps_valid = false;
        tcaspmm_status ms = encode_b_maps(dt, dB, sh.ncols, sh.K, ldb, (BMaps *)sh.maps);
        if (ms != TCASPMM_OK) return ms;
        sh.maps_valid = true;
        sh.maps_ptr = dB;
        sh.maps_ldb = ldb;
    }
    launch_kernel(fmt_of(dt), grid, p, *(const BMaps *)sh.maps, *(const CUtensorMap *)sh.cmap, st);
    cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? TCASPMM_OK : cuda_fail(e, "tc kernel launch");
}

}  // namespace tca

using namespace tca;

// Failure-detection self-test: one tensor-core window whose producer issues no
// copies (a flag nothing sets), so the MMA thread's bounded wait must run out
// after `wait_cycles`; the kernel records the time-out, frees its TMEM and
// returns, and the context stays usable.  Returns TCASPMM_ERR_TIMEOUT with the
// device error word in *err_code when that happened as designed.
extern "C" tcaspmm_status tcaspmm_selftest_tc_timeout(int device, unsigned long long wait_cycles, int *err_code)
{
    clear_error();
    cudaError_t e = cudaSetDevice(device);
    if (e != cudaSuccess) return cuda_fail(e, "cudaSetDevice");
    if (!tc_supported()) return fail(TCASPMM_ERR_UNSUPPORTED, "device %d is not sm_100", device);
    const int4 win = make_int4(0, 0, 1, R);
    const int4 nosplit = make_int4(-1, 0, 1, 0);
    const std::vector<int32_t> cols(KT, 0);
    const std::vector<uint16_t> vals(R * KT, 0);
    const int32_t no_run = -1;
    void *d_win = nullptr, *d_split = nullptr, *d_dense = nullptr, *d_cols = nullptr, *d_vals = nullptr,
         *d_b = nullptr, *d_c = nullptr;
    int *d_err = nullptr;
    tcaspmm_status st = TCASPMM_OK;
    auto alloc = [&](void **ptr, size_t n) {
        if (st == TCASPMM_OK && (e = cudaMalloc(ptr, n)) != cudaSuccess) st = cuda_fail(e, "self-test allocation");
    };
    alloc(&d_win, sizeof(win));
    alloc(&d_split, sizeof(nosplit));
    alloc(&d_dense, sizeof(no_run));
    alloc(&d_cols, cols.size() * 4);
    alloc(&d_vals, vals.size() * 2);
    alloc(&d_b, Geo<0>::SROWS * MB * 2);
    alloc(&d_c, R * MB * 4);
    alloc((void **)&d_err, 6 * sizeof(int));
    BMaps maps;
    if (st == TCASPMM_OK) {
        cudaMemcpy(d_win, &win, sizeof(win), cudaMemcpyHostToDevice);
        cudaMemcpy(d_split, &nosplit, sizeof(nosplit), cudaMemcpyHostToDevice);
        cudaMemcpy(d_dense, &no_run, sizeof(no_run), cudaMemcpyHostToDevice);
        cudaMemcpy(d_cols, cols.data(), cols.size() * 4, cudaMemcpyHostToDevice);
        cudaMemcpy(d_vals, vals.data(), vals.size() * 2, cudaMemcpyHostToDevice);
        cudaMemset(d_b, 0, Geo<0>::SROWS * MB * 2);
        cudaMemset(d_err, 0, 6 * sizeof(int));
        st = encode_b_maps(TCASPMM_F16, d_b, MB, Geo<0>::SROWS, MB, &maps);
    }
    if (st == TCASPMM_OK) {
        TcParams p;
        p.tasks = (const int4 *)d_win;
        p.splits = (const int4 *)d_split;
        p.rows = nullptr;
        p.partials = nullptr;
        p.counters = nullptr;
        p.dense_c0 = (const int32_t *)d_dense;
        p.tile_cols = (const int32_t *)d_cols;
        p.tile_vals = (const uint8_t *)d_vals;
        p.B = d_b;
        p.ldb = MB;
        p.C = (float *)d_c;
        p.ldc = MB;
        p.ncols = MB;
        p.nfb = 1;
        p.n_units = 1;
        p.err = d_err;
        p.wait_cycles = wait_cycles;
        p.stall_test = 1;
        p.has_ep = 0;
        p.ep = EpiParams{nullptr, nullptr, 0, 0};
        p.tma_store = 0;
        e = smem_optin<0>();
        if (e == cudaSuccess) {
            launch_kernel(0, 1, p, maps, CUtensorMap{}, 0);
            e = cudaGetLastError();
        }
        if (e == cudaSuccess) e = cudaDeviceSynchronize();
        int err = 0;
        if (e == cudaSuccess) e = cudaMemcpy(&err, d_err, sizeof(int), cudaMemcpyDeviceToHost);
        if (e != cudaSuccess) {
            st = cuda_fail(e, "self-test kernel");
        } else {
            if (err_code) *err_code = err;
            st = err ? fail(TCASPMM_ERR_TIMEOUT, "tensor-core wait timed out as designed (code 0x%x)", err)
                     : fail(TCASPMM_OK, "no time-out recorded");
        }
    }
    for (void *ptr : {d_win, d_split, d_dense, d_cols, d_vals, d_b, d_c, (void *)d_err})
        if (ptr) cudaFree(ptr);
    return st;
}
