// Tensor-core path for dense windows (tcgen05).  Not enabled yet: every
// window is scheduled on the CUDA-core residue kernel.
#include "plan.h"

namespace tca {

bool tc_supported() { return false; }

tcaspmm_status tc_upload(const tcaspmm_csr &, tcaspmm_dtype, Shard *) { return TCASPMM_OK; }

tcaspmm_status launch_tc(const Shard &, tcaspmm_dtype, const void *, int64_t, float *, int64_t, cudaStream_t)
{
    return TCASPMM_OK;
}

}  // namespace tca
