// Residue-kernel launch dispatch over (dtype, vector width, lane-group size),
// instantiated once without and once with the fused epilogue (plan.cu,
// residue_epi.cu), so the two sets of kernels compile in parallel.
#pragma once

#include "plan.h"
#include "residue.cuh"

namespace tca {

// Nonzeros in flight per lane group: 8, or 6 for the 16-bit epilogue kernels,
// whose extra live values would otherwise spill at 64 registers (measured on
// GCN: 1.58 ms at 6 against 1.63 ms at 8).
template <typename T, bool EPI> constexpr int unroll() { return EPI && sizeof(T) < 4 ? 6 : 8; }

// Launch shape of the residue kernel: BLOCK threads per block, U nonzeros in
// flight per lane group, PF = columns and row ends loaded one chunk / one row
// ahead (64 registers hold PF only with U = 6).
template <typename T, int VEC, int G, bool EPI, bool PF, int BLOCK, int U = unroll<T, EPI>()>
void launch_res_v(const ResidueParams &p, int total_warps, cudaStream_t st)
{
    constexpr int W = BLOCK / 32;
    const int blocks = (total_warps + W - 1) / W;
    residue_kernel<T, VEC, G, U, EPI, PF, BLOCK><<<blocks, BLOCK, 0, st>>>(p);
}

// Vector paths run 128-thread blocks (a finished block's slot is refilled
// sooner than with 256: 27.3 against 25.8 resident warps per SM on GCN) and the
// prefetching stream, except with one 16-bit group per warp and, for 16-bit
// types, with the epilogue (its operands leave no registers for the prefetch;
// GCN f16 with the epilogue 1.56 -> 1.42 ms from the 128-thread blocks and the
// 32-bit addressing).  fp32 without the epilogue keeps 7 nonzeros in flight
// per lane (the most that 64 registers hold with the prefetch): GCN f32 1.765 ->
// 1.70 ms against 6; 16-bit types keep 6.
// Measured on one B200 against 256 threads, U = 8, no prefetch (ms):
//   GCN f32 N = 128: 1.92 -> 1.86 (prefetch, two runs averaged; 1.89 without)
//   GCN f16 N = 128: 1.46 -> 1.35;  GCN f32 N = 64 / 32 / 16: 1.15 / 0.70 /
//   0.55 -> 1.07 / 0.63 / 0.51;  skew f16 N = 64: 1.26 -> 1.24;
//   SAGE f16 N = 256 (one 16-bit group per warp): 5.17 -> 5.17 without
//   prefetch, 5.40 with it.
template <typename T, int VEC, int G, bool EPI>
void launch_res(const ResidueParams &p, int total_warps, cudaStream_t st)
{
    if constexpr (VEC > 1 && !EPI) {
        if constexpr (sizeof(T) == 4)
            launch_res_v<T, VEC, G, EPI, true, 128, 7>(p, total_warps, st);
        else if constexpr (G == 32)
            launch_res_v<T, VEC, G, EPI, false, 128>(p, total_warps, st);
        else
            launch_res_v<T, VEC, G, EPI, true, 128, 6>(p, total_warps, st);
    } else if constexpr (VEC > 1) {
        // Epilogue kernels: the prefetch fits 64 registers only for fp32.
        if constexpr (sizeof(T) == 4)
            launch_res_v<T, VEC, G, EPI, true, 128, 6>(p, total_warps, st);
        else
            launch_res_v<T, VEC, G, EPI, false, 128>(p, total_warps, st);
    } else {
        launch_res_v<T, VEC, G, EPI, false, 256>(p, total_warps, st);
    }
}

template <typename T, int VEC, bool EPI>
void launch_res_g(int G, const ResidueParams &p, int total_warps, cudaStream_t st)
{
    switch (G) {
    case 1: launch_res<T, VEC, 1, EPI>(p, total_warps, st); break;
    case 2: launch_res<T, VEC, 2, EPI>(p, total_warps, st); break;
    case 4: launch_res<T, VEC, 4, EPI>(p, total_warps, st); break;
    case 8: launch_res<T, VEC, 8, EPI>(p, total_warps, st); break;
    case 16: launch_res<T, VEC, 16, EPI>(p, total_warps, st); break;
    default: launch_res<T, VEC, 32, EPI>(p, total_warps, st); break;
    }
}

template <typename T, bool EPI>
void launch_res_t(bool vec, int G, const ResidueParams &p, int total_warps, cudaStream_t st)
{
    if (vec)
        launch_res_g<T, 16 / sizeof(T), EPI>(G, p, total_warps, st);
    else
        launch_res_g<T, 1, EPI>(G, p, total_warps, st);
}

template <bool EPI>
void launch_res_dt(tcaspmm_dtype dt, bool vec, int G, const ResidueParams &p, int total_warps, cudaStream_t st)
{
    if (dt == TCASPMM_F32 || dt == TCASPMM_TF32)
        launch_res_t<float, EPI>(vec, G, p, total_warps, st);
    else if (dt == TCASPMM_F16)
        launch_res_t<__half, EPI>(vec, G, p, total_warps, st);
    else
        launch_res_t<__nv_bfloat16, EPI>(vec, G, p, total_warps, st);
}

}  // namespace tca
