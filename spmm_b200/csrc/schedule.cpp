// Host preprocessor: splits A into tensor-core windows (dense condensed column
// tiles) and CUDA-core residue work balanced by nonzeros.
//
// Replaces workload_manager (src/our_spmm.cu:353-477), which buckets rows by
// nnz into 1/2/4/8 warps or several 8-warp blocks and packs them first-fit.
// Here:
//   * rows are grouped into windows of R rows; a window whose condensed tiles
//     move fewer bytes than gathering its rows one nonzero at a time becomes a
//     tensor-core window (16-bit dtypes and TF32); optionally, rows left over
//     that are long are grouped by length into further windows with row lists
//     (the long-row half of workload_manager, src/our_spmm.cu:392-395);
//   * every other row belongs to exactly one contiguous row range, and ranges
//     carry about the same cost (nnz + per-row overhead) per warp;
//   * a row longer than twice the per-warp budget is cut into segments whose
//     partial sums are reduced in a fixed order (deterministic), so one hub row
//     never serialises a warp.
// Every nonzero lands in exactly one tile cell, one row range or one segment;
// tcaspmm_schedule_coverage checks that integer invariant.
#include <algorithm>
#include <chrono>
#include <cmath>
#include <cstdlib>
#include <cstring>

#include <omp.h>

#include "internal.h"

namespace tca {

void residue_shape(int64_t ncols, tcaspmm_dtype dt, bool vector_path, int *G, int *VEC)
{
    const int vec = vector_path ? 16 / dtype_size(dt) : 1;
    const int64_t nvec = (ncols + vec - 1) / vec;
    int g = 1;
    while (g < nvec && g < 32) g *= 2;
    *G = g;
    *VEC = vec;
}

// Integer tuning variable, clamped to [lo, hi]; unset, empty or not a whole
// number (trailing characters included) gives the default.
int64_t env_int(const char *name, int64_t dflt, int64_t lo, int64_t hi)
{
    const char *s = std::getenv(name);
    if (!s || !*s) return dflt;
    char *end = nullptr;
    const long long v = std::strtoll(s, &end, 10);
    if (end == s || *end != '\0') return dflt;
    return std::min<int64_t>(std::max<int64_t>(v, lo), hi);
}

// The sorted union of the columns of `rows` (n of them) and their nonzero
// count.  Small groups sort their columns; a group of more than 8192 nonzeros
// marks them in `marks` (one byte per column of A, allocated on first use and
// left zeroed), which costs O(nonzeros) instead of a sort of all of them.
static void column_union(const tcaspmm_csr &A, const int32_t *rows, int n, std::vector<uint8_t> &marks,
                         std::vector<int32_t> *cols_u, int64_t *nnz_w)
{
    cols_u->clear();
    int64_t nz = 0;
    for (int i = 0; i < n; i++) nz += A.row_ptr[rows[i] + 1] - A.row_ptr[rows[i]];
    *nnz_w = nz;
    if (nz <= 8192) {
        for (int i = 0; i < n; i++)
            cols_u->insert(cols_u->end(), A.col_idx + A.row_ptr[rows[i]], A.col_idx + A.row_ptr[rows[i] + 1]);
        std::sort(cols_u->begin(), cols_u->end());
        cols_u->erase(std::unique(cols_u->begin(), cols_u->end()), cols_u->end());
        return;
    }
    if (marks.empty()) marks.assign((size_t)A.ncol, 0);
    for (int i = 0; i < n; i++) {
        for (int64_t j = A.row_ptr[rows[i]]; j < A.row_ptr[rows[i] + 1]; j++) {
            const int32_t c = A.col_idx[j];
            if (!marks[c]) {
                marks[c] = 1;
                cols_u->push_back(c);
            }
        }
    }
    for (int32_t c : *cols_u) marks[c] = 0;
    std::sort(cols_u->begin(), cols_u->end());
}

// Bytes moved by a window of `nrows` rows as condensed tiles (16 gathered B rows
// and an R x KT value tile per tile) against per-nonzero gathers on the CUDA cores.
static bool tiles_pay(int64_t ucols, int64_t nz, int KT, int R, int64_t ncols, int elem)
{
    if (nz == 0) return false;
    const int64_t ntiles = (ucols + KT - 1) / KT;
    const double row_bytes = (double)ncols * elem;
    const double tc_bytes = (double)ntiles * KT * (row_bytes + 4) + (double)ntiles * R * KT * elem;
    const double res_bytes = (double)nz * (row_bytes + 4 + elem);
    return tc_bytes < 0.8 * res_bytes;
}

// Appends a window over rows[0..n) (x as in TileSchedule::windows) whose
// condensed columns are cols_u, and marks its rows as tensor-core rows.
static void add_window(const int32_t *rows, int n, int32_t x, const std::vector<int32_t> &cols_u, int64_t nz,
                       Schedule *S)
{
    TileSchedule &T = S->tc;
    const int KT = T.KT;
    const int64_t ntiles = ((int64_t)cols_u.size() + KT - 1) / KT;
    const int64_t t_first = (int64_t)T.tile_cols.size() / KT;
    T.windows.push_back(Int4{x, (int32_t)t_first, (int32_t)ntiles, (int32_t)n});
    const size_t cbase = T.tile_cols.size();
    T.tile_cols.resize(cbase + ntiles * KT);
    for (int64_t q = 0; q < ntiles * KT; q++) T.tile_cols[cbase + q] = q < (int64_t)cols_u.size() ? cols_u[q] : cols_u.back();
    for (int i = 0; i < n; i++) S->row_tc[rows[i]] = 1;
    T.nnz += nz;
}

tcaspmm_status build_schedule(const tcaspmm_csr &A, int64_t ncols, tcaspmm_dtype dt,
                              const ScheduleOptions &opt, Schedule *out)
{
    auto t0 = std::chrono::steady_clock::now();
    Schedule &S = *out;
    S = Schedule();
    S.M = A.nrow;
    S.K = A.ncol;
    S.nnz = A.nnz;
    S.ncols = ncols;
    S.dt = dt;
    const int elem = dtype_size(dt);
    const int64_t M = A.nrow;

    // ---- tensor-core windows (16-bit dtypes and TF32) ----
    const int R = 32;
    S.tc.R = R;
    S.tc.KT = 16;
    S.row_tc.assign((size_t)M, 0);
    const bool tc_ok = opt.allow_tc && dt != TCASPMM_F32 && ncols > 0 && ncols % 8 == 0 &&
                       env_int("TCASPMM_DISABLE_TC", 0, 0, 1) == 0;
    if (tc_ok) {
        const int nth = omp_get_max_threads();
        std::vector<std::vector<uint8_t>> marks((size_t)nth);  // per thread, allocated when a large group needs it
        // (1) Consecutive windows: blocks of R rows whose condensed tiles move fewer
        // bytes, are at least 1/32 dense (TCASPMM_TC_DENSITY) and have at most 256
        // tiles.  Evaluated in parallel, appended in order.  The density floor was
        // measured over the pruned-weight sweep (3 shapes x 4 sparsities x 2
        // structures x N = 128 / 512, f16): 1/32 within 1% of the best floor per
        // case on geometric mean (1/16: 12%, 1/8: 25%).
        const int64_t nwin = (M + R - 1) / R;
        const double density_div = (double)env_int("TCASPMM_TC_DENSITY", 32, 1, 1024);
        std::vector<std::vector<int32_t>> ok_cols((size_t)nwin);
        std::vector<int64_t> ok_nz((size_t)nwin, -1);
#pragma omp parallel for schedule(dynamic, 64)
        for (int64_t w = 0; w < nwin; w++) {
            const int64_t r0 = w * R;
            const int n = (int)std::min<int64_t>(R, M - r0);
            int32_t rows[32];
            for (int i = 0; i < n; i++) rows[i] = (int32_t)(r0 + i);
            std::vector<int32_t> cols_u;
            int64_t nz;
            column_union(A, rows, n, marks[omp_get_thread_num()], &cols_u, &nz);
            const int64_t ntiles = ((int64_t)cols_u.size() + S.tc.KT - 1) / S.tc.KT;
            if (nz == 0 || ntiles > 256 || (double)nz < (double)ntiles * S.tc.KT * n / density_div ||
                !tiles_pay((int64_t)cols_u.size(), nz, S.tc.KT, R, ncols, elem))
                continue;
            ok_cols[w] = std::move(cols_u);
            ok_nz[w] = nz;
        }
        for (int64_t w = 0; w < nwin; w++) {
            if (ok_nz[w] < 0) continue;
            const int n = (int)std::min<int64_t>(R, M - w * R);
            int32_t rows[32];
            for (int i = 0; i < n; i++) rows[i] = (int32_t)(w * R + i);
            add_window(rows, n, (int32_t)(w * R), ok_cols[w], ok_nz[w], &S);
            std::vector<int32_t>().swap(ok_cols[w]);
        }
        // (2) Gathered windows of long rows: the remaining rows of at least
        // 2 * KT nonzeros, longest first, taken R at a time while their condensed
        // tiles pay (hub rows share their hub columns, so the union is smaller
        // than the nonzero count); shorter rows pay less, so the first window that
        // does not pay ends the search.  Their tile chains are split across CTAs
        // at upload, so there is no tile cap.  Windows are evaluated in parallel
        // batches and appended in order.
        if (env_flag("TCASPMM_HUB_WINDOWS", false)) {
            std::vector<int32_t> cand;
            for (int64_t r = 0; r < M; r++)
                if (!S.row_tc[r] && A.row_ptr[r + 1] - A.row_ptr[r] >= 2 * S.tc.KT) cand.push_back((int32_t)r);
            std::stable_sort(cand.begin(), cand.end(), [&](int32_t a, int32_t b) {
                return A.row_ptr[a + 1] - A.row_ptr[a] > A.row_ptr[b + 1] - A.row_ptr[b];
            });
            const int64_t ncw = ((int64_t)cand.size() + R - 1) / R;
            bool stop = false;
            for (int64_t b0 = 0; b0 < ncw && !stop; b0 += 2 * nth) {
                const int64_t b1 = std::min<int64_t>(ncw, b0 + 2 * nth);
                std::vector<std::vector<int32_t>> cu((size_t)(b1 - b0));
                std::vector<int64_t> nzs((size_t)(b1 - b0));
                std::vector<char> pays((size_t)(b1 - b0));
#pragma omp parallel for schedule(dynamic, 1)
                for (int64_t w = b0; w < b1; w++) {
                    const int64_t c0 = w * R;
                    const int n = (int)std::min<int64_t>(R, (int64_t)cand.size() - c0);
                    column_union(A, cand.data() + c0, n, marks[omp_get_thread_num()], &cu[w - b0], &nzs[w - b0]);
                    pays[w - b0] = tiles_pay((int64_t)cu[w - b0].size(), nzs[w - b0], S.tc.KT, R, ncols, elem);
                }
                for (int64_t w = b0; w < b1; w++) {
                    if (!pays[w - b0]) {
                        stop = true;
                        break;
                    }
                    const int64_t c0 = w * R;
                    const int n = (int)std::min<int64_t>(R, (int64_t)cand.size() - c0);
                    const int32_t x = -(int32_t)(S.tc.rows.size() + 1);
                    S.tc.rows.insert(S.tc.rows.end(), cand.begin() + c0, cand.begin() + c0 + n);
                    add_window(cand.data() + c0, n, x, cu[w - b0], nzs[w - b0], &S);
                    S.tc.gathered++;
                }
            }
        }
    }

    // ---- residue rows ----
    ResidueSchedule &RS = S.res;
    residue_shape(ncols, dt, true, &RS.G, &RS.VEC);
    RS.P = 32 / RS.G;
    const int P = RS.P;
    const int64_t BETA = 2;  // per-row cost (row_ptr read, C row write) in nonzero units
    auto in_tc = [&](int64_t r) { return S.row_tc[r] != 0; };
    int64_t W = 0;
    for (int64_t r = 0; r < M; r++)
        if (!in_tc(r)) W += (A.row_ptr[r + 1] - A.row_ptr[r]) + BETA;
    const int64_t target_warps = (int64_t)opt.num_sms * env_int("TCASPMM_WARPS_PER_SM", 32, 1, 1024);
    // Per-group budget: W spread over the target warps, within [lo, hi].  With
    // one or two groups per warp hi is 1024 per group; with more, hi keeps a
    // warp's total near 1024 nonzeros (measured on GCN: N = 16, P = 8, 0.55 ms
    // against 0.67 ms with 1024 per group; N = 32, P = 4, 0.71 against 0.79; but
    // P = 2 is faster at 1024 per group: f16 N = 128 1.45 against 1.59 ms).
    // With eight or more groups per warp a warp's total is kept near 512
    // (GCN N = 16 with the prefetching stream: 0.487 against 0.506 ms at 1024;
    // N = 128 and SAGE are fastest at the 1024 caps, 2048 and 512 both slower).
    int64_t base = W / std::max<int64_t>(1, (int64_t)P * target_warps);
    const int64_t bmax = env_int("TCASPMM_BUDGET_MAX", 1024, 16, 1 << 20);
    const int64_t hi = P <= 2 ? bmax : std::max<int64_t>(16, (P >= 8 ? bmax / 2 : bmax) / P);
    const int64_t lo = std::min<int64_t>(env_int("TCASPMM_BUDGET_MIN", 128, 1, 1 << 20), hi);
    base = std::min<int64_t>(std::max<int64_t>(base, lo), hi);
    const int64_t warp_budget = base * P;  // a warp runs P rows (or P nnz streams) at once
    RS.long_thr = (int32_t)std::min<int64_t>(INT32_MAX, 2 * base);
    const int64_t seg_len = warp_budget;

    // Long rows -> segments (issued first so they start early).
    for (int64_t r = 0; r < M; r++) {
        if (in_tc(r)) continue;
        const int64_t b = A.row_ptr[r], e = A.row_ptr[r + 1], L = e - b;
        if (L <= RS.long_thr) continue;
        const int64_t nseg = (L + seg_len - 1) / seg_len;
        const int32_t long_id = (int32_t)RS.longs.size();
        RS.longs.push_back(Int4{(int32_t)r, (int32_t)RS.segs.size(), (int32_t)nseg, 0});
        for (int64_t k = 0; k < nseg; k++)
            RS.segs.push_back(Int4{(int32_t)r, (int32_t)(b + L * k / nseg), (int32_t)(b + L * (k + 1) / nseg), long_id});
        RS.nnz += L;
    }
    // Row ranges: runs of rows that are neither tensor-core rows nor long rows,
    // cut every warp_budget of cost.
    int64_t start = -1, acc = 0;
    for (int64_t r = 0; r < M; r++) {
        const int64_t L = A.row_ptr[r + 1] - A.row_ptr[r];
        if (in_tc(r) || L > RS.long_thr) {
            if (start >= 0) RS.ranges.push_back(Int2{(int32_t)start, (int32_t)r});
            start = -1;
            acc = 0;
            continue;
        }
        if (start < 0) start = r;
        acc += L + BETA;
        RS.nnz += L;
        if (acc >= warp_budget) {
            RS.ranges.push_back(Int2{(int32_t)start, (int32_t)(r + 1)});
            start = -1;
            acc = 0;
        }
    }
    if (start >= 0) RS.ranges.push_back(Int2{(int32_t)start, (int32_t)M});

    S.build_ms = std::chrono::duration<double, std::milli>(std::chrono::steady_clock::now() - t0).count();
    return TCASPMM_OK;
}

}  // namespace tca

using namespace tca;

extern "C" tcaspmm_status tcaspmm_schedule_coverage(const tcaspmm_csr *A, int64_t N, tcaspmm_dtype dt,
                                                    int32_t *cover, int8_t *kind, tcaspmm_plan_stats *stats)
{
    if (!A || !cover || !kind || N < 0 || !dtype_valid(dt))
        return fail(TCASPMM_ERR_INVALID_ARG, "schedule_coverage: bad arguments");
    tcaspmm_status s = tcaspmm_csr_validate(A);
    if (s != TCASPMM_OK) return s;
    Schedule S;
    ScheduleOptions opt;
    s = build_schedule(*A, N, dt, opt, &S);
    if (s != TCASPMM_OK) return s;
    std::memset(cover, 0, sizeof(int32_t) * A->nnz);
    std::memset(kind, 0, (size_t)A->nnz);
    auto mark = [&](int64_t j, int8_t k) {
        cover[j]++;
        kind[j] = k;
    };
    // Tile cells: every nonzero of a tc window's rows must find its column in the
    // window's condensed columns (its value tile is built from that position).
    const int R = S.tc.R, KT = S.tc.KT;
    for (const Int4 &w : S.tc.windows) {
        const int32_t *tc = S.tc.tile_cols.data() + (int64_t)w.y * KT;
        const int64_t ncond = (int64_t)w.z * KT;
        for (int64_t q = 1; q < ncond; q++)
            if (tc[q] < tc[q - 1]) return fail(TCASPMM_ERR_FORMAT, "window columns not ascending");
        for (int i = 0; i < w.w; i++) {
            const int64_t r = S.tc.row(w, i);
            for (int64_t j = A->row_ptr[r]; j < A->row_ptr[r + 1]; j++) {
                const int32_t c = A->col_idx[j];
                int64_t p = std::lower_bound(tc, tc + ncond, c) - tc;
                if (p >= ncond || tc[p] != c) continue;  // not covered: reported by cover[j] == 0
                mark(j, 3);
            }
        }
    }
    // Residue, walked exactly as the kernel walks it.
    const ResidueSchedule &RS = S.res;
    for (const Int2 &rg : RS.ranges) {
        for (int64_t r = rg.x; r < rg.y; r++) {
            if (S.row_tc[r])
                return fail(TCASPMM_ERR_FORMAT, "row range holds tensor-core row %lld", (long long)r);
            for (int64_t j = A->row_ptr[r]; j < A->row_ptr[r + 1]; j++) mark(j, 1);
        }
    }
    for (const Int4 &g : RS.segs) {
        const Int4 &L = RS.longs[g.w];
        if (L.x != g.x || g.y < A->row_ptr[g.x] || g.z > A->row_ptr[g.x + 1] || g.y > g.z)
            return fail(TCASPMM_ERR_FORMAT, "segment outside its row");
        for (int64_t j = g.y; j < g.z; j++) mark(j, 2);
    }
    if (stats) {
        std::memset(stats, 0, sizeof(*stats));
        stats->nrow = A->nrow;
        stats->ncol = A->ncol;
        stats->nnz = A->nnz;
        stats->ncols_total = N;
        stats->num_shards = 1;
        stats->window_rows = R;
        stats->tc_windows = (int64_t)S.tc.windows.size();
        stats->tc_gathered_windows = S.tc.gathered;
        stats->tc_tiles = (int64_t)S.tc.tile_cols.size() / (KT ? KT : 1);
        stats->tc_nnz = S.tc.nnz;
        stats->residue_nnz = RS.nnz;
        stats->residue_row_warps = (int64_t)RS.ranges.size();
        stats->residue_segments = (int64_t)RS.segs.size();
        stats->long_rows = (int64_t)RS.longs.size();
        stats->preprocess_ms = S.build_ms;
        stats->algorithmic_bytes = algorithmic_bytes(A->nrow, A->ncol, A->nnz, N, dt);
    }
    return TCASPMM_OK;
}
