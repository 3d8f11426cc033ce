// Per-device state of a plan and the launchers shared by plan.cu and tc.cu.
#pragma once

#include <cuda_runtime.h>

#include <vector>

#include "internal.h"

namespace tca {

struct Shard {
    int device = 0;
    int64_t col_begin = 0, ncols = 0;  // column block of B and C
    int64_t row_begin = 0, nrows = 0;  // row block of A and C (all rows unless row-split)
    int64_t K = 0;  // rows of B
    Schedule sched;  // host schedule; large arrays are released after upload
    std::vector<void *> allocs;
    int64_t bytes = 0;

    // A in CSR on the device.
    int32_t *row_ptr = nullptr;
    int32_t *col = nullptr;
    void *val = nullptr;

    // Residue schedule + scratch.
    Int2 *ranges = nullptr;
    Int4 *segs = nullptr;
    Int4 *longs = nullptr;
    int n_ranges = 0, n_segs = 0, n_longs = 0;
    int long_thr = 0;
    float *partials = nullptr;
    int pstride = 0;
    unsigned int *counters = nullptr;

    // Tensor-core windows and the tasks they are cut into.
    int n_windows = 0;
    int n_tasks = 0;              // work items per column block
    int n_split_groups = 0;       // gathered windows cut into several tasks
    int n_fallback = 0;
    int num_sms = 148;
    int tc_ctas_per_sm = 1;       // resident tc-kernel CTAs per SM (persistent grid)
    Int4 *tc_tasks = nullptr;     // {x, first tile, tiles, rows}, by decreasing tile count
    Int4 *tc_splits = nullptr;    // per task {split window id or -1, part, parts, first partial slot}
    int32_t *tc_rows = nullptr;   // row lists of the gathered windows
    float *tc_partials = nullptr; // partial tiles of split windows (scratch)
    unsigned int *tc_counters = nullptr;  // parts counted in per split window, zero between launches
    int32_t *tc_dense = nullptr;  // per task: first column of its consecutive run, or -1
    int32_t *tc_cols = nullptr;   // KT B-row indices per tile
    void *tc_vals = nullptr;      // R x KT values per tile, shared-memory image
    Int2 *tc_fallback = nullptr;  // row ranges covering the tc rows (unaligned B: CUDA cores)
    // Tensor maps over the last B block launched (rebuilt when B or ldb change);
    // opaque storage for three 128-byte CUtensorMap objects.
    alignas(64) mutable unsigned char maps[384] = {};
    mutable bool maps_valid = false;
    mutable const void *maps_ptr = nullptr;
    mutable int64_t maps_ldb = 0;
    // Tensor map over the last C block written by bulk stores (one CUtensorMap).
    alignas(64) mutable unsigned char cmap[128] = {};
    mutable bool cmap_valid = false;
    mutable const void *cmap_ptr = nullptr;
    mutable int64_t cmap_ldc = 0;
    mutable int cmap_out = 0;

    int *err = nullptr;  // device error words: codes of bounded waits that ran out, and where the first did

    // When a shard has both tensor-core tasks and residue work, the tensor-core
    // kernel runs on this (high-priority) stream beside the residue kernel on the
    // caller's stream, forked and joined by the two events.
    cudaStream_t side = nullptr;
    cudaEvent_t ev_fork = nullptr, ev_join = nullptr;
};

// Fused output epilogue of one launch (tcaspmm_epilogue after validation):
// C = relu?(row_scale[r] * (A B)[r][c] + bias[c]) stored as fp32 (out 0), fp16
// (1) or bf16 (2).
struct Epilogue {
    const float *row_scale = nullptr;
    const float *bias = nullptr;
    int relu = 0;
    int out = 0;
    int out_size() const { return out == 0 ? 4 : 2; }
};

struct ResidueParams;

tcaspmm_status cuda_fail(cudaError_t e, const char *what);
void free_shard(Shard &sh);

// Tensor-core path (tc.cu).
bool tc_supported();
tcaspmm_status tc_upload(const tcaspmm_csr &A, tcaspmm_dtype dt, Shard *sh);
// `ep` NULL: plain fp32 C.  ldc counts elements of the output type.
tcaspmm_status launch_tc(const Shard &sh, tcaspmm_dtype dt, const void *dB, int64_t ldb, void *dC, int64_t ldc,
                         const Epilogue *ep, cudaStream_t st);
// CUDA-core residue kernel over the shard's row ranges and segments, or, with
// `ranges` given, over those ranges only (whole rows of any length, no segments).
tcaspmm_status launch_residue(const Shard &sh, tcaspmm_dtype dt, const void *dB, int64_t ldb, void *dC, int64_t ldc,
                              const Epilogue *ep, cudaStream_t st, const Int2 *ranges = nullptr, int n_ranges = 0);
// The epilogue instantiations of the residue kernel (residue_epi.cu).
void launch_residue_epi(tcaspmm_dtype dt, bool vec, int G, const ResidueParams &p, int total_warps, cudaStream_t st);

}  // namespace tca
