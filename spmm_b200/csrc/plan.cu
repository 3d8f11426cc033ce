// Plans: host schedule -> device buffers per shard, and kernel launches.
//
// Replaces the device half of our_spmm_balanced (src/our_spmm.cu:486-565):
// the reference allocates and uploads A, B, C and three schedule arrays per
// call and launches kernel_our_spmm_balanced<64> on the default stream.  A plan
// uploads A and its schedule once; execute only launches (on caller streams).
#include <algorithm>
#include <chrono>
#include <climits>
#include <cstdlib>
#include <cstring>
#include <memory>
#include <vector>

#include <cuda_runtime.h>
#include <omp.h>

#include "internal.h"
#include "plan.h"
#include "residue_dispatch.cuh"

using namespace tca;

namespace tca {

tcaspmm_status cuda_fail(cudaError_t e, const char *what)
{
    return fail(TCASPMM_ERR_CUDA, "%s: %s (%d)", what, cudaGetErrorString(e), (int)e);
}

namespace {

struct DeviceGuard {
    int prev = -1;
    explicit DeviceGuard(int dev)
    {
        if (cudaGetDevice(&prev) != cudaSuccess) prev = -1;
        if (prev != dev) cudaSetDevice(dev);
    }
    ~DeviceGuard()
    {
        int cur = -1;
        if (prev >= 0 && cudaGetDevice(&cur) == cudaSuccess && cur != prev) cudaSetDevice(prev);
    }
};

template <typename X>
tcaspmm_status upload(Shard &sh, X **dst, const X *src, size_t n, const char *what)
{
    *dst = nullptr;
    if (n == 0) return TCASPMM_OK;
    cudaError_t e = cudaMalloc((void **)dst, sizeof(X) * n);
    if (e != cudaSuccess) {
        *dst = nullptr;
        return fail(TCASPMM_ERR_ALLOC, "cudaMalloc of %zu bytes for %s failed: %s", sizeof(X) * n, what,
                    cudaGetErrorString(e));
    }
    sh.allocs.push_back(*dst);
    sh.bytes += (int64_t)(sizeof(X) * n);
    if (src) {
        e = cudaMemcpy(*dst, src, sizeof(X) * n, cudaMemcpyHostToDevice);
        if (e != cudaSuccess) return cuda_fail(e, what);
    }
    return TCASPMM_OK;
}

// Round fp32 host values to the device dtype.
std::vector<uint16_t> to_16bit(const float *v, int64_t n, tcaspmm_dtype dt)
{
    std::vector<uint16_t> out((size_t)n);
#pragma omp parallel for schedule(static)
    for (int64_t i = 0; i < n; i++)
        out[i] = dt == TCASPMM_F16 ? float_to_half_bits(v[i]) : float_to_bf16_bits(v[i]);
    return out;
}

tcaspmm_status build_shard(const tcaspmm_csr &Afull, tcaspmm_dtype dt, int device, int64_t col_begin,
                           int64_t ncols, int64_t row_begin, int64_t nrows, Shard *sh, double *prep_ms)
{
    sh->device = device;
    sh->col_begin = col_begin;
    sh->ncols = ncols;
    sh->row_begin = row_begin;
    sh->nrows = nrows;
    sh->K = Afull.ncol;
    // A row block is the CSR view of rows [row_begin, row_begin + nrows) with
    // rebased offsets.
    std::vector<int64_t> sub_rp;
    tcaspmm_csr A = Afull;
    if (row_begin != 0 || nrows != Afull.nrow) {
        const int64_t base = Afull.row_ptr[row_begin];
        sub_rp.resize((size_t)nrows + 1);
        for (int64_t i = 0; i <= nrows; i++) sub_rp[i] = Afull.row_ptr[row_begin + i] - base;
        A.nrow = nrows;
        A.nnz = sub_rp[nrows];
        A.row_ptr = sub_rp.data();
        A.col_idx = Afull.col_idx + base;
        A.val = Afull.val ? Afull.val + base : nullptr;
    }
    DeviceGuard g(device);
    int nsm = 148;
    cudaError_t e = cudaDeviceGetAttribute(&nsm, cudaDevAttrMultiProcessorCount, device);
    if (e != cudaSuccess) return cuda_fail(e, "query SM count");

    ScheduleOptions opt;
    opt.num_sms = nsm;
    opt.allow_tc = tc_supported();
    tcaspmm_status s = build_schedule(A, ncols, dt, opt, &sh->sched);
    if (s != TCASPMM_OK) return s;
    *prep_ms += sh->sched.build_ms;
    const Schedule &S = sh->sched;

    // A in CSR: int32 row offsets, int32 columns, values in dt.
    std::vector<int32_t> rp32((size_t)A.nrow + 1);
    for (int64_t i = 0; i <= A.nrow; i++) rp32[i] = (int32_t)A.row_ptr[i];
    if ((s = upload(*sh, &sh->row_ptr, rp32.data(), rp32.size(), "row offsets")) != TCASPMM_OK) return s;
    if ((s = upload(*sh, &sh->col, A.col_idx, (size_t)A.nnz, "column indices")) != TCASPMM_OK) return s;
    {
        std::vector<float> ones;
        const float *v = A.val;
        if (!v) {
            ones.assign((size_t)A.nnz, 1.0f);
            v = ones.data();
        }
        if (dtype_fp32(dt)) {
            float *d = nullptr;
            if ((s = upload(*sh, &d, v, (size_t)A.nnz, "values")) != TCASPMM_OK) return s;
            sh->val = d;
        } else {
            std::vector<uint16_t> h = to_16bit(v, A.nnz, dt);
            uint16_t *d = nullptr;
            if ((s = upload(*sh, &d, h.data(), h.size(), "values")) != TCASPMM_OK) return s;
            sh->val = d;
        }
    }
    // Residue schedule and its scratch (partials + counters).
    const ResidueSchedule &RS = S.res;
    static_assert(sizeof(Int2) == sizeof(int2) && sizeof(Int4) == sizeof(int4), "layout");
    if ((s = upload(*sh, (Int2 **)&sh->ranges, RS.ranges.data(), RS.ranges.size(), "row ranges")) != TCASPMM_OK) return s;
    if ((s = upload(*sh, (Int4 **)&sh->segs, RS.segs.data(), RS.segs.size(), "segments")) != TCASPMM_OK) return s;
    if ((s = upload(*sh, (Int4 **)&sh->longs, RS.longs.data(), RS.longs.size(), "long rows")) != TCASPMM_OK) return s;
    sh->n_ranges = (int)RS.ranges.size();
    sh->n_segs = (int)RS.segs.size();
    sh->n_longs = (int)RS.longs.size();
    sh->long_thr = RS.long_thr;
    sh->pstride = (int)((ncols + 3) / 4 * 4);
    if ((s = upload<float>(*sh, &sh->partials, nullptr, (size_t)sh->n_segs * sh->pstride, "partials")) != TCASPMM_OK) return s;
    if ((s = upload<unsigned int>(*sh, &sh->counters, nullptr, (size_t)sh->n_longs, "counters")) != TCASPMM_OK) return s;
    if (sh->n_longs) {
        e = cudaMemset(sh->counters, 0, sizeof(unsigned int) * sh->n_longs);
        if (e != cudaSuccess) return cuda_fail(e, "zero counters");
    }
    if ((s = upload<int>(*sh, &sh->err, nullptr, 6, "error words")) != TCASPMM_OK) return s;
    e = cudaMemset(sh->err, 0, 6 * sizeof(int));
    if (e != cudaSuccess) return cuda_fail(e, "zero error word");
    if ((s = tc_upload(A, dt, sh)) != TCASPMM_OK) return s;
    // Both kernels in one launch: when the tensor-core work items leave CTA slots
    // free, the tensor-core kernel runs on a side stream beside the residue rows
    // instead of before them (a few long tile chains no longer add their latency
    // to the residue kernel's); when they fill every slot, the two kernels would
    // only contend (one tile CTA per SM beside the residue warps measured 1.71 ms on
    // C3 with gathered windows, against 1.51 ms one after the other), and run one
    // after the other.  TCASPMM_OVERLAP=0 never forks.
    const int64_t tc_units = (int64_t)sh->n_tasks * ((ncols + 127) / 128);
    if (sh->n_tasks > 0 && sh->n_ranges + sh->n_segs > 0 && tc_units < (int64_t)sh->tc_ctas_per_sm * sh->num_sms &&
        env_flag("TCASPMM_OVERLAP", true)) {
        int least = 0, greatest = 0;
        e = cudaDeviceGetStreamPriorityRange(&least, &greatest);
        if (e == cudaSuccess) e = cudaStreamCreateWithPriority(&sh->side, cudaStreamNonBlocking, greatest);
        if (e == cudaSuccess) e = cudaEventCreateWithFlags(&sh->ev_fork, cudaEventDisableTiming);
        if (e == cudaSuccess) e = cudaEventCreateWithFlags(&sh->ev_join, cudaEventDisableTiming);
        if (e != cudaSuccess) return cuda_fail(e, "side stream");
    }
    e = cudaDeviceSynchronize();
    if (e != cudaSuccess) return cuda_fail(e, "plan upload");
    return TCASPMM_OK;
}

}  // namespace

tcaspmm_status launch_residue(const Shard &sh, tcaspmm_dtype dt, const void *dB, int64_t ldb, void *dC, int64_t ldc,
                              const Epilogue *ep, cudaStream_t st, const Int2 *ranges, int n_ranges)
{
    const bool whole_rows = ranges != nullptr;
    const int n_segs = whole_rows ? 0 : sh.n_segs;
    if (!whole_rows) {
        ranges = sh.ranges;
        n_ranges = sh.n_ranges;
    }
    const int total = n_segs + n_ranges;
    if (total == 0 || sh.ncols == 0) return TCASPMM_OK;
    const int elem = dtype_size(dt);
    // The residue kernel forms B row addresses from a 32-bit row pitch in bytes.
    if ((uint64_t)ldb * (uint64_t)elem > 0xffffffffull)
        return fail(TCASPMM_ERR_UNSUPPORTED, "B row pitch of %lld elements exceeds 4 GiB", (long long)ldb);
    // 16-byte vector path needs 16-byte aligned B rows and aligned C rows
    // (16 bytes for fp32 C; 8 or 16 bytes for 16-bit C, VEC = 4 or 8).
    const int out_elem = ep ? ep->out_size() : 4;
    const bool vec = ((uintptr_t)dB % 16 == 0) && ((ldb * elem) % 16 == 0) && ((uintptr_t)dC % 16 == 0) &&
                     ((ldc * out_elem) % 16 == 0) && (sh.ncols % (16 / elem) == 0);
    int G, VEC;
    residue_shape(sh.ncols, dt, vec, &G, &VEC);
    // The row ranges were cut for the vector shape; the scalar path uses the
    // same ranges with its own G (more passes), which stays correct.
    ResidueParams p;
    p.row_ptr = sh.row_ptr;
    p.col = sh.col;
    p.val = sh.val;
    p.B = dB;
    p.ldb = ldb;
    p.C = static_cast<float *>(dC);
    p.ldc = ldc;
    p.ncols = (int)sh.ncols;
    p.ranges = (const int2 *)ranges;
    p.n_ranges = n_ranges;
    p.segs = (const int4 *)sh.segs;
    p.n_segs = n_segs;
    p.longs = (const int4 *)sh.longs;
    p.partials = sh.partials;
    p.pstride = sh.pstride;
    p.counters = sh.counters;
    p.ep = EpiParams{nullptr, nullptr, 0, 0};
    if (ep) {
        p.ep = EpiParams{ep->row_scale, ep->bias, ep->relu, ep->out};
        launch_residue_epi(dt, vec, G, p, total, st);
    } else {
        launch_res_dt<false>(dt, vec, G, p, total, st);
    }
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return cuda_fail(e, "residue kernel launch");
    return TCASPMM_OK;
}

void free_shard(Shard &sh)
{
    if (sh.allocs.empty() && !sh.side && !sh.ev_fork && !sh.ev_join) return;
    DeviceGuard g(sh.device);
    if (sh.ev_join) cudaEventDestroy(sh.ev_join);
    if (sh.ev_fork) cudaEventDestroy(sh.ev_fork);
    if (sh.side) cudaStreamDestroy(sh.side);
    sh.ev_join = sh.ev_fork = nullptr;
    sh.side = nullptr;
    for (void *p : sh.allocs) cudaFree(p);
    sh.allocs.clear();
}

}  // namespace tca

struct tcaspmm_plan {
    int64_t M = 0, K = 0, nnz = 0, N = 0;
    tcaspmm_dtype dt = TCASPMM_F32;
    std::vector<std::unique_ptr<Shard>> shards;
    tcaspmm_plan_stats stats{};
    ~tcaspmm_plan()
    {
        for (auto &s : shards) free_shard(*s);
    }
};

// Shards: column blocks (begins/counts) of all rows, or, with row blocks given
// (row_begins/row_counts), row blocks of all N columns.
static tcaspmm_status create_common(const tcaspmm_csr *A, int64_t N, tcaspmm_dtype dt,
                                    const std::vector<int> &devices, const std::vector<int64_t> &begins,
                                    const std::vector<int64_t> &counts, tcaspmm_plan **out,
                                    const std::vector<int64_t> &row_begins = {},
                                    const std::vector<int64_t> &row_counts = {})
{
    const bool split_rows = !row_begins.empty();
    auto t0 = std::chrono::steady_clock::now();
    std::unique_ptr<tcaspmm_plan> P(new tcaspmm_plan());
    P->M = A->nrow;
    P->K = A->ncol;
    P->nnz = A->nnz;
    P->N = N;
    P->dt = dt;
    double prep = 0.0;
    for (size_t i = 0; i < devices.size(); i++) {
        P->shards.emplace_back(new Shard());
        tcaspmm_status s = build_shard(*A, dt, devices[i], begins[i], counts[i], split_rows ? row_begins[i] : 0,
                                       split_rows ? row_counts[i] : A->nrow, P->shards.back().get(), &prep);
        if (s != TCASPMM_OK) return s;
    }
    const double total = std::chrono::duration<double, std::milli>(std::chrono::steady_clock::now() - t0).count();
    tcaspmm_plan_stats &st = P->stats;
    const Schedule &S = P->shards[0]->sched;
    st.nrow = A->nrow;
    st.ncol = A->ncol;
    st.nnz = A->nnz;
    st.ncols_total = N;
    st.num_shards = (int32_t)P->shards.size();
    st.window_rows = S.tc.R;
    // Column shards of one row block share a schedule (the first column block
    // speaks for the others); row blocks add up.
    for (size_t i = 0; i < P->shards.size(); i++) {
        st.device_bytes = std::max<int64_t>(st.device_bytes, P->shards[i]->bytes);
        if (split_rows ? P->shards[i]->col_begin != 0 : i != 0) continue;
        const Schedule &Si = P->shards[i]->sched;
        st.tc_windows += (int64_t)Si.tc.windows.size();
        st.tc_gathered_windows += Si.tc.gathered;
        st.tc_tasks += P->shards[i]->n_tasks;
        if (P->shards[i]->n_tasks) st.tc_ctas_per_sm = P->shards[i]->tc_ctas_per_sm;
        if (P->shards[i]->side) st.tc_side_stream = 1;
        st.tc_tiles += Si.tc.KT ? (int64_t)Si.tc.tile_cols.size() / Si.tc.KT : 0;
        st.tc_nnz += Si.tc.nnz;
        st.residue_nnz += Si.res.nnz;
        st.residue_row_warps += (int64_t)Si.res.ranges.size();
        st.residue_segments += (int64_t)Si.res.segs.size();
        st.long_rows += (int64_t)Si.res.longs.size();
    }
    st.preprocess_ms = prep;
    st.upload_ms = total - prep;
    st.algorithmic_bytes = algorithmic_bytes(A->nrow, A->ncol, A->nnz, N, dt);
    for (auto &sh : P->shards) sh->sched = Schedule();  // host copies are on the device now
    *out = P.release();
    return TCASPMM_OK;
}

static tcaspmm_status check_inputs(const tcaspmm_csr *A, int64_t N, tcaspmm_dtype dt, tcaspmm_plan **out)
{
    if (!out) return fail(TCASPMM_ERR_INVALID_ARG, "plan_create: out is NULL");
    *out = nullptr;
    if (!A) return fail(TCASPMM_ERR_INVALID_ARG, "plan_create: A is NULL");
    if (!dtype_valid(dt)) return fail(TCASPMM_ERR_INVALID_ARG, "plan_create: unknown dtype %d", (int)dt);
    if (N < 0 || N > INT32_MAX) return fail(TCASPMM_ERR_INVALID_ARG, "plan_create: N=%lld out of range", (long long)N);
    return tcaspmm_csr_validate(A);
}

extern "C" {

tcaspmm_status tcaspmm_plan_create(const tcaspmm_csr *A, int64_t N, tcaspmm_dtype dt, int num_gpus,
                                   const int *devices, tcaspmm_plan **out)
{
    clear_error();
    tcaspmm_status s = check_inputs(A, N, dt, out);
    if (s != TCASPMM_OK) return s;
    int ndev = 0;
    if (cudaGetDeviceCount(&ndev) != cudaSuccess || ndev == 0) {
        cudaGetLastError();
        return fail(TCASPMM_ERR_NO_DEVICE, "no CUDA device");
    }
    if (num_gpus < 1) return fail(TCASPMM_ERR_INVALID_ARG, "num_gpus=%d", num_gpus);
    std::vector<int> devs(num_gpus);
    std::vector<int64_t> b(num_gpus), c(num_gpus);
    for (int i = 0; i < num_gpus; i++) {
        devs[i] = devices ? devices[i] : i;
        if (devs[i] < 0 || devs[i] >= ndev)
            return fail(TCASPMM_ERR_NO_DEVICE, "device %d requested, %d present", devs[i], ndev);
        tcaspmm_partition_columns(N, dt, num_gpus, i, &b[i], &c[i]);
    }
    return create_common(A, N, dt, devs, b, c, out);
}

tcaspmm_status tcaspmm_plan_create_shard(const tcaspmm_csr *A, int64_t N, tcaspmm_dtype dt, int rank, int world,
                                         int device, tcaspmm_plan **out)
{
    clear_error();
    tcaspmm_status s = check_inputs(A, N, dt, out);
    if (s != TCASPMM_OK) return s;
    int ndev = 0;
    if (cudaGetDeviceCount(&ndev) != cudaSuccess || ndev == 0) {
        cudaGetLastError();
        return fail(TCASPMM_ERR_NO_DEVICE, "no CUDA device");
    }
    if (device < 0 || device >= ndev) return fail(TCASPMM_ERR_NO_DEVICE, "device %d requested, %d present", device, ndev);
    int64_t b, c;
    s = tcaspmm_partition_columns(N, dt, world, rank, &b, &c);
    if (s != TCASPMM_OK) return s;
    return create_common(A, N, dt, {device}, {b}, {c}, out);
}

static tcaspmm_status device_count_check(int n, const int *devices, std::vector<int> *devs)
{
    int ndev = 0;
    if (cudaGetDeviceCount(&ndev) != cudaSuccess || ndev == 0) {
        cudaGetLastError();
        return fail(TCASPMM_ERR_NO_DEVICE, "no CUDA device");
    }
    devs->resize(n);
    for (int i = 0; i < n; i++) {
        (*devs)[i] = devices ? devices[i] : i;
        if ((*devs)[i] < 0 || (*devs)[i] >= ndev)
            return fail(TCASPMM_ERR_NO_DEVICE, "device %d requested, %d present", (*devs)[i], ndev);
    }
    return TCASPMM_OK;
}

tcaspmm_status tcaspmm_plan_create_rows(const tcaspmm_csr *A, int64_t N, tcaspmm_dtype dt, int num_gpus,
                                        const int *devices, tcaspmm_plan **out)
{
    clear_error();
    tcaspmm_status s = check_inputs(A, N, dt, out);
    if (s != TCASPMM_OK) return s;
    if (num_gpus < 1) return fail(TCASPMM_ERR_INVALID_ARG, "num_gpus=%d", num_gpus);
    std::vector<int> devs;
    if ((s = device_count_check(num_gpus, devices, &devs)) != TCASPMM_OK) return s;
    std::vector<int64_t> rb(num_gpus + 1);
    if ((s = tcaspmm_partition_rows(A, num_gpus, rb.data())) != TCASPMM_OK) return s;
    std::vector<int64_t> b(num_gpus, 0), c(num_gpus, N), r0(num_gpus), rc(num_gpus);
    for (int i = 0; i < num_gpus; i++) {
        r0[i] = rb[i];
        rc[i] = rb[i + 1] - rb[i];
    }
    return create_common(A, N, dt, devs, b, c, out, r0, rc);
}

tcaspmm_status tcaspmm_plan_create_rows_shard(const tcaspmm_csr *A, int64_t N, tcaspmm_dtype dt, int rank,
                                              int world, int device, tcaspmm_plan **out)
{
    clear_error();
    tcaspmm_status s = check_inputs(A, N, dt, out);
    if (s != TCASPMM_OK) return s;
    if (world < 1 || rank < 0 || rank >= world)
        return fail(TCASPMM_ERR_INVALID_ARG, "plan_create_rows_shard: rank %d of %d", rank, world);
    std::vector<int> devs;
    if ((s = device_count_check(1, &device, &devs)) != TCASPMM_OK) return s;
    std::vector<int64_t> rb(world + 1);
    if ((s = tcaspmm_partition_rows(A, world, rb.data())) != TCASPMM_OK) return s;
    return create_common(A, N, dt, devs, {0}, {N}, out, {rb[rank]}, {rb[rank + 1] - rb[rank]});
}

tcaspmm_status tcaspmm_plan_create_2d(const tcaspmm_csr *A, int64_t N, tcaspmm_dtype dt, int grid_rows,
                                      int grid_cols, const int *devices, tcaspmm_plan **out)
{
    clear_error();
    tcaspmm_status s = check_inputs(A, N, dt, out);
    if (s != TCASPMM_OK) return s;
    if (grid_rows < 1 || grid_cols < 1)
        return fail(TCASPMM_ERR_INVALID_ARG, "plan_create_2d: grid %d x %d", grid_rows, grid_cols);
    const int g = grid_rows * grid_cols;
    std::vector<int> devs;
    if ((s = device_count_check(g, devices, &devs)) != TCASPMM_OK) return s;
    std::vector<int64_t> rb(grid_rows + 1);
    if ((s = tcaspmm_partition_rows(A, grid_rows, rb.data())) != TCASPMM_OK) return s;
    std::vector<int64_t> b(g), c(g), r0(g), rc(g);
    for (int i = 0; i < g; i++) {
        const int r = i / grid_cols, q = i % grid_cols;
        tcaspmm_partition_columns(N, dt, grid_cols, q, &b[i], &c[i]);
        r0[i] = rb[r];
        rc[i] = rb[r + 1] - rb[r];
    }
    return create_common(A, N, dt, devs, b, c, out, r0, rc);
}

tcaspmm_status tcaspmm_plan_create_2d_shard(const tcaspmm_csr *A, int64_t N, tcaspmm_dtype dt, int rank,
                                            int grid_rows, int grid_cols, int device, tcaspmm_plan **out)
{
    clear_error();
    tcaspmm_status s = check_inputs(A, N, dt, out);
    if (s != TCASPMM_OK) return s;
    if (grid_rows < 1 || grid_cols < 1 || rank < 0 || rank >= grid_rows * grid_cols)
        return fail(TCASPMM_ERR_INVALID_ARG, "plan_create_2d_shard: rank %d of %d x %d", rank, grid_rows, grid_cols);
    std::vector<int> devs;
    if ((s = device_count_check(1, &device, &devs)) != TCASPMM_OK) return s;
    std::vector<int64_t> rb(grid_rows + 1);
    if ((s = tcaspmm_partition_rows(A, grid_rows, rb.data())) != TCASPMM_OK) return s;
    const int r = rank / grid_cols, q = rank % grid_cols;
    int64_t b = 0, c = 0;
    tcaspmm_partition_columns(N, dt, grid_cols, q, &b, &c);
    return create_common(A, N, dt, devs, {b}, {c}, out, {rb[r]}, {rb[r + 1] - rb[r]});
}

tcaspmm_status tcaspmm_plan_shard_rows(const tcaspmm_plan *plan, int shard, int64_t *row_begin, int64_t *row_count)
{
    if (!plan || shard < 0 || shard >= (int)plan->shards.size())
        return fail(TCASPMM_ERR_INVALID_ARG, "plan_shard_rows: bad shard %d", shard);
    const Shard &s = *plan->shards[shard];
    if (row_begin) *row_begin = s.row_begin;
    if (row_count) *row_count = s.nrows;
    return TCASPMM_OK;
}

tcaspmm_status tcaspmm_plan_destroy(tcaspmm_plan *plan)
{
    delete plan;
    return TCASPMM_OK;
}

tcaspmm_status tcaspmm_plan_get_stats(const tcaspmm_plan *plan, tcaspmm_plan_stats *out)
{
    if (!plan || !out) return fail(TCASPMM_ERR_INVALID_ARG, "plan_get_stats: NULL argument");
    *out = plan->stats;
    return TCASPMM_OK;
}

tcaspmm_status tcaspmm_plan_shard(const tcaspmm_plan *plan, int shard, int *device, int64_t *col_begin,
                                  int64_t *col_count)
{
    if (!plan || shard < 0 || shard >= (int)plan->shards.size())
        return fail(TCASPMM_ERR_INVALID_ARG, "plan_shard: bad shard %d", shard);
    const Shard &s = *plan->shards[shard];
    if (device) *device = s.device;
    if (col_begin) *col_begin = s.col_begin;
    if (col_count) *col_count = s.ncols;
    return TCASPMM_OK;
}

tcaspmm_status tcaspmm_execute_ex(tcaspmm_plan *plan, const void *const *dB, const int64_t *ldb, void *const *dC,
                                  const int64_t *ldc, void *const *streams, const tcaspmm_epilogue *epilogues)
{
    if (!plan || !dB || !ldb || !dC || !ldc) return fail(TCASPMM_ERR_INVALID_ARG, "execute: NULL argument");
    for (size_t i = 0; i < plan->shards.size(); i++) {
        const Shard &sh = *plan->shards[i];
        if (sh.ncols == 0 || sh.nrows == 0) continue;
        if (ldb[i] < sh.ncols || ldc[i] < sh.ncols)
            return fail(TCASPMM_ERR_INVALID_ARG, "execute: shard %zu ldb=%lld ldc=%lld below %lld columns", i,
                        (long long)ldb[i], (long long)ldc[i], (long long)sh.ncols);
        if (!dC[i] || (!dB[i] && plan->K > 0))
            return fail(TCASPMM_ERR_INVALID_ARG, "execute: shard %zu has a NULL B or C", i);
        Epilogue ep;
        if (epilogues) {
            const tcaspmm_epilogue &e = epilogues[i];
            ep.row_scale = e.row_scale;
            ep.bias = e.bias;
            ep.relu = e.relu != 0;
            switch (e.out_dtype) {
            case TCASPMM_F32: ep.out = 0; break;
            case TCASPMM_F16: ep.out = 1; break;
            case TCASPMM_BF16: ep.out = 2; break;
            default: return fail(TCASPMM_ERR_INVALID_ARG, "execute: shard %zu has an unknown output dtype", i);
            }
        }
        cudaStream_t st = streams ? (cudaStream_t)streams[i] : (cudaStream_t)0;
        DeviceGuard g(sh.device);
        const Epilogue *epp = epilogues ? &ep : nullptr;
        if (sh.side) {
            // Fork: the tensor-core kernel on the side stream, the residue kernel on
            // the caller's; joined before anything later on the caller's stream.
            // The join is recorded even when a launch failed, so a stream capture
            // never holds an unjoined fork.
            cudaError_t e = cudaEventRecord(sh.ev_fork, st);
            if (e == cudaSuccess) e = cudaStreamWaitEvent(sh.side, sh.ev_fork, 0);
            if (e != cudaSuccess) return cuda_fail(e, "fork to the side stream");
            const tcaspmm_status s_tc = launch_tc(sh, plan->dt, dB[i], ldb[i], dC[i], ldc[i], epp, sh.side);
            const tcaspmm_status s_res = launch_residue(sh, plan->dt, dB[i], ldb[i], dC[i], ldc[i], epp, st);
            e = cudaEventRecord(sh.ev_join, sh.side);
            if (e == cudaSuccess) e = cudaStreamWaitEvent(st, sh.ev_join, 0);
            if (s_tc != TCASPMM_OK) return s_tc;
            if (s_res != TCASPMM_OK) return s_res;
            if (e != cudaSuccess) return cuda_fail(e, "join from the side stream");
            continue;
        }
        tcaspmm_status s = launch_tc(sh, plan->dt, dB[i], ldb[i], dC[i], ldc[i], epp, st);
        if (s != TCASPMM_OK) return s;
        s = launch_residue(sh, plan->dt, dB[i], ldb[i], dC[i], ldc[i], epp, st);
        if (s != TCASPMM_OK) return s;
    }
    return TCASPMM_OK;
}

tcaspmm_status tcaspmm_execute(tcaspmm_plan *plan, const void *const *dB, const int64_t *ldb, float *const *dC,
                               const int64_t *ldc, void *const *streams)
{
    return tcaspmm_execute_ex(plan, dB, ldb, reinterpret_cast<void *const *>(dC), ldc, streams, nullptr);
}

tcaspmm_status tcaspmm_execute1_ex(tcaspmm_plan *plan, const void *dB, int64_t ldb, void *dC, int64_t ldc,
                                   void *stream, const tcaspmm_epilogue *ep)
{
    if (!plan) return fail(TCASPMM_ERR_INVALID_ARG, "execute1: plan is NULL");
    if (plan->shards.size() != 1)
        return fail(TCASPMM_ERR_INVALID_ARG, "execute1: plan has %zu shards", plan->shards.size());
    return tcaspmm_execute_ex(plan, &dB, &ldb, &dC, &ldc, &stream, ep);
}

tcaspmm_status tcaspmm_execute1(tcaspmm_plan *plan, const void *dB, int64_t ldb, float *dC, int64_t ldc, void *stream)
{
    return tcaspmm_execute1_ex(plan, dB, ldb, dC, ldc, stream, nullptr);
}

tcaspmm_status tcaspmm_plan_sync_check(tcaspmm_plan *plan)
{
    if (!plan) return fail(TCASPMM_ERR_INVALID_ARG, "plan_sync_check: plan is NULL");
    for (auto &up : plan->shards) {
        Shard &sh = *up;
        DeviceGuard g(sh.device);
        cudaError_t e = cudaDeviceSynchronize();
        if (e != cudaSuccess) return cuda_fail(e, "synchronize");
        int err[6] = {0, 0, 0, 0, 0, 0};
        e = cudaMemcpy(err, sh.err, sizeof(err), cudaMemcpyDeviceToHost);
        if (e != cudaSuccess) return cuda_fail(e, "read error word");
        if (err[0] != 0) {
            cudaMemset(sh.err, 0, sizeof(err));
            // An aborted launch may have left split windows part-counted: start
            // the next launch from zero.
            if (sh.tc_counters)
                cudaMemset(sh.tc_counters, 0,
                           sizeof(unsigned int) * (size_t)sh.n_split_groups * ((sh.ncols + 127) / 128) * 4);
            return fail(TCASPMM_ERR_TIMEOUT,
                        "device %d: tensor-core kernel gave up waiting (codes 0x%x; first: code %d on the barrier at "
                        "shared address 0x%x, parity %d, CTA %d, thread %d)",
                        sh.device, err[0], err[1], err[2], err[3], err[4], err[5]);
        }
    }
    return TCASPMM_OK;
}

}  // extern "C"

// Device CSR arrays of a shard, for baselines that run on the same upload.
extern "C" tcaspmm_status tcaspmm_plan_device_csr(const tcaspmm_plan *plan, int shard, const int32_t **row_ptr,
                                                  const int32_t **col, const void **val)
{
    if (!plan || shard < 0 || shard >= (int)plan->shards.size())
        return fail(TCASPMM_ERR_INVALID_ARG, "plan_device_csr: bad shard");
    const Shard &s = *plan->shards[shard];
    if (row_ptr) *row_ptr = s.row_ptr;
    if (col) *col = s.col;
    if (val) *val = s.val;
    return TCASPMM_OK;
}
