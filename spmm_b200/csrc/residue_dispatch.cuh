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

template <typename T, int VEC, int G, bool EPI>
void launch_res(const ResidueParams &p, int total_warps, cudaStream_t st)
{
    const int blocks = (total_warps + 7) / 8;
    residue_kernel<T, VEC, G, unroll<T, EPI>(), EPI><<<blocks, 256, 0, st>>>(p);
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
