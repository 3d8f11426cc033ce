// Internal declarations shared by the host sources of libtcaspmm.
#pragma once

#include <cstdarg>
#include <cstdint>
#include <string>
#include <vector>

#include "tcaspmm.h"

namespace tca {

// ---- error reporting (thread-local message behind tcaspmm_last_error) ----
tcaspmm_status fail(tcaspmm_status s, const char *fmt, ...);
void clear_error();

// ---- dtype helpers ----
inline bool dtype_fp32(tcaspmm_dtype dt) { return dt == TCASPMM_F32 || dt == TCASPMM_TF32; }  // fp32 storage
inline int dtype_size(tcaspmm_dtype dt) { return dtype_fp32(dt) ? 4 : 2; }
inline bool dtype_valid(int dt)
{
    return dt == TCASPMM_F32 || dt == TCASPMM_F16 || dt == TCASPMM_BF16 || dt == TCASPMM_TF32;
}
uint16_t float_to_half_bits(float f);
uint16_t float_to_bf16_bits(float f);
float half_bits_to_float(uint16_t h);
inline float bf16_bits_to_float(uint16_t b)
{
    const uint32_t u = (uint32_t)b << 16;
    float f;
    __builtin_memcpy(&f, &u, 4);
    return f;
}

// ---- tuning variables (read when a plan is created) ----
// Integer variable clamped to [lo, hi]; unset or not a whole number: dflt.
int64_t env_int(const char *name, int64_t dflt, int64_t lo, int64_t hi);
inline bool env_flag(const char *name, bool dflt) { return env_int(name, dflt ? 1 : 0, 0, 1) != 0; }

// ---- counter-based random streams (SplitMix64 finaliser over a counter) ----
inline uint64_t mix64(uint64_t z)
{
    // SplitMix64 output function (Steele, Lea & Flood, OOPSLA 2014).
    z = (z ^ (z >> 30)) * 0xbf58476d1ce4e5b9ULL;
    z = (z ^ (z >> 27)) * 0x94d049bb133111ebULL;
    return z ^ (z >> 31);
}
inline uint64_t rng_u64(uint64_t seed, uint64_t stream, uint64_t i)
{
    const uint64_t g = 0x9e3779b97f4a7c15ULL;
    return mix64(mix64(seed * g + stream) + (i + 1) * g);
}
inline double rng_unit(uint64_t seed, uint64_t stream, uint64_t i)
{
    return (double)(rng_u64(seed, stream, i) >> 11) * (1.0 / 9007199254740992.0);
}
double rng_normal(uint64_t seed, uint64_t stream, uint64_t i);

// ---- host CSR helpers ----
tcaspmm_status csr_from_rows(int64_t nrow, int64_t ncol, const std::vector<int64_t> &row_ptr,
                             const std::vector<int32_t> &col, const std::vector<float> *val,
                             tcaspmm_csr *out);

// ---- schedule (host preprocessor) ----
struct Int2 { int32_t x, y; };
struct Int4 { int32_t x, y, z, w; };

// Tensor-core window tiles.  A window is up to `R` rows -- consecutive rows, or
// a gathered list of long rows grouped by length -- whose condensed columns (the
// sorted union of the rows' columns) are split into tiles of KT columns.  For
// tile t of window w, tile_cols[t * KT + k] is the B row index of condensed
// column k (padding columns repeat the last index and get zero values); the
// R x KT value tile (row i of the window, k) is built from A at upload.
// windows[w] = {x, first tile, number of tiles, rows in window}: x >= 0 is the
// first of consecutive rows; x < 0 means rows[-(x + 1) + i] is the window's row i.
struct TileSchedule {
    int R = 0;
    int KT = 0;
    std::vector<Int4> windows;
    std::vector<int32_t> rows;     // row lists of the gathered windows
    std::vector<int32_t> tile_cols;
    int64_t nnz = 0;
    int64_t gathered = 0;          // gathered windows among `windows`
    // Row i of window w.
    int32_t row(const Int4 &w, int i) const { return w.x >= 0 ? w.x + i : rows[(size_t)(-(w.x + 1)) + i]; }
};

// CUDA-core residue work.  Row ranges are runs of rows that are neither in
// tensor-core windows nor longer than long_thr; each is handled whole by its
// range's warp.  Rows longer than long_thr are split into segments.
struct ResidueSchedule {
    int G = 32;                      // lanes per row slice
    int VEC = 4;                     // elements per lane load
    int P = 1;                       // rows (or nnz streams) per warp = 32 / G
    int32_t long_thr = 0;
    std::vector<Int2> ranges;        // {first row, end row} per row warp
    std::vector<Int4> segs;          // {row, begin, end, long_id}
    std::vector<Int4> longs;         // {row, first seg, number of segs, 0}
    int64_t nnz = 0;
};

struct Schedule {
    int64_t M = 0, K = 0, nnz = 0, ncols = 0;
    tcaspmm_dtype dt = TCASPMM_F32;
    TileSchedule tc;
    std::vector<uint8_t> row_tc;  // per row: 1 = in a tensor-core window
    ResidueSchedule res;
    double build_ms = 0.0;
};

struct ScheduleOptions {
    int num_sms = 148;
    bool allow_tc = true;
};

tcaspmm_status build_schedule(const tcaspmm_csr &A, int64_t ncols, tcaspmm_dtype dt,
                              const ScheduleOptions &opt, Schedule *out);
// Lanes per row slice / elements per lane for a shard of `ncols` columns.
void residue_shape(int64_t ncols, tcaspmm_dtype dt, bool vector_path, int *G, int *VEC);

int64_t algorithmic_bytes(int64_t M, int64_t K, int64_t nnz, int64_t N, tcaspmm_dtype dt);

}  // namespace tca
