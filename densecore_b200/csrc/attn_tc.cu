// attn_tc.cu -- tcgen05 tensor-core attention kernels (sm_100a).
#include "common.cuh"
#include "kernels.h"

namespace dc {

bool tc_forward_supported(const AttnProblem &) { return false; }
int tc_forward(const AttnProblem &, int, cudaStream_t) {
    return fail(DC_ERR_UNSUPPORTED, "tensor-core forward is not built");
}
bool tc_backward_supported(const AttnProblem &) { return false; }
int tc_backward(const AttnProblem &, const AttnGrads &, int, cudaStream_t) {
    return fail(DC_ERR_UNSUPPORTED, "tensor-core backward is not built");
}

}  // namespace dc
