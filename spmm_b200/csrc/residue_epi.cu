// Residue kernels with the fused output epilogue (row scale, bias, ReLU, 16-bit C).
#include "residue_dispatch.cuh"

namespace tca {

void launch_residue_epi(tcaspmm_dtype dt, bool vec, int G, const ResidueParams &p, int total_warps, cudaStream_t st)
{
    launch_res_dt<true>(dt, vec, G, p, total_warps, st);
}

}  // namespace tca
