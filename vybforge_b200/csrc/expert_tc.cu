// Tensor-core (tcgen05) grouped expert GEMMs.
#include "expert_tc.h"

namespace vfmoe {

int tc_plan_create(const vfmoe_layer_desc &, TcPlan &plan) {
    plan.ready = 0;
    return VFMOE_OK;
}

bool tc_supported(const TcPlan &plan, const MoeArgs &) { return plan.ready != 0; }

int launch_experts_tc(const TcPlan &, const MoeArgs &, cudaStream_t, const std::function<void()> &) {
    set_error("tensor-core expert path not built");
    return VFMOE_ERR_UNSUPPORTED;
}

}  // namespace vfmoe
