// Tensor-core (tcgen05) grouped expert GEMMs: launch state and entry points.
#pragma once

#include <cuda.h>

#include "kernels.h"

namespace vfmoe {

struct TcPlan {
    int ready = 0;
    int num_sms = 0;
    // Q8_0 weight tensor maps (3D: [experts][rows][row bytes as u16]).
    CUtensorMap gate, up, down;          // routed, stacked
    CUtensorMap sh_gate, sh_up, sh_down; // shared expert (one "expert")
};

int tc_plan_create(const vfmoe_layer_desc &d, TcPlan &plan);
bool tc_supported(const TcPlan &plan, const MoeArgs &a);
int launch_experts_tc(const TcPlan &plan, const MoeArgs &a, cudaStream_t st, const std::function<void()> &mid);

// Workspace the tensor-core path needs beyond MoeArgs: tile lists for both GEMMs.
int64_t tc_tiles_capacity(int T, int k, int E);

}  // namespace vfmoe
