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
// ahead.  With PF, 64 registers hold U = 7 for fp32 and U = 6 for 16-bit types
// (6 for fp32 with the epilogue); beyond that the kernels spill.
template <typename T, int VEC, int G, bool EPI, bool PF, int BLOCK, int U = unroll<T, EPI>()>
void launch_res_v(const ResidueParams &p, int total_warps, cudaStream_t st)
{
    constexpr int W = BLOCK / 32;
    const int blocks = (total_warps + W - 1) / W;
    residue_kernel<T, VEC, G, U, EPI, PF, BLOCK><<<blocks, BLOCK, 0, st>>>(p);
}

// Shapes used (all measured on one B200, outputs bit-identical across shapes):
//   vector paths run 128-thread blocks: a finished block's slot is refilled
//   sooner than with 256 (27.3 against 25.8 resident warps per SM on GCN);
//   fp32: prefetch, U = 7 (GCN N = 128: 256 threads / U = 8 / no prefetch 1.92
//   ms, 128 threads / prefetch / U = 6 1.86, with 32-bit addressing 1.77, U = 7
//   1.70; N = 64 / 32 / 16: 1.15 / 0.70 / 0.55 -> 1.07 / 0.63 / 0.48);
//   16-bit, two or more groups per warp: prefetch, U = 6 (GCN f16 N = 128 1.46
//   -> 1.26 with the addressing; skew N = 64 1.26 -> 1.23);
//   16-bit, one group per warp (SAGE N = 256): no prefetch, U = 8 (5.17 -> 4.79;
//   the prefetch at U = 6 was 5.40 before the addressing change, a tie after);
//   epilogue kernels: prefetch, U = 6 for fp32, none for 16-bit, whose epilogue
//   operands leave no registers for it (GCN f32 / f16 with the epilogue 1.90 /
//   1.56 -> 1.68 / 1.42).
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
