// Tensor-core (tcgen05) grouped expert GEMMs: launch state and entry points.
#pragma once

#include "kernels.h"

namespace vfmoe {

struct TcPlan {
    int ready = 0;
};

int tc_plan_create(const vfmoe_layer_desc &d, TcPlan &plan);
bool tc_supported(const TcPlan &plan, const MoeArgs &a);
int launch_experts_tc(const TcPlan &plan, const MoeArgs &a, cudaStream_t st, const std::function<void()> &mid);

}  // namespace vfmoe
