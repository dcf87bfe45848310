// Layer handle state shared by the C-ABI translation units (api.cu, ep.cu).
#pragma once

#include <cstdint>
#include <functional>
#include <vector>

#include "common.cuh"
#include "kernels.h"
#include "expert_tc.h"

namespace vfmoe {

// Expert-parallel placement of one layer (vfmoe_ep_set_placement): which rank owns each
// virtual expert (the E routed experts plus R copies of hot experts), the local slot of each
// virtual expert on its owner, and the copy of each expert (or -1).  Device arrays.
struct EpPlacement {
    int ready = 0;
    int n_ranks = 0, rank = 0;
    int n_virtual = 0;            // E + R
    int32_t *owner = nullptr;     // [n_virtual]
    int32_t *local_slot = nullptr;  // [n_virtual]
    int32_t *copy_of = nullptr;   // [E]: virtual id of expert e's copy, -1 if none
};

struct Layer {
    vfmoe_layer_desc d;
    int device = 0;
    int H = 0, I = 0, E = 0, k = 0;
    int n_local = 0;             // routed experts whose weights this handle holds (E unless expert-parallel)
    int has_shared = 0;
    int64_t q8_row_gate = 0, q8_row_down = 0;
    int *dev_err = nullptr;      // device error word (allocated at create)
    float *nw = nullptr;         // |W_r row|_2 upper bounds (allocated at create)
    __nv_bfloat16 *wr_split = nullptr;  // W_r as bf16 hi and lo parts [2][E][H] for the tensor-core
                                        // router logits (bf16 x, H and E multiples of 128), else 0
    void *own_ws = nullptr;      // internal workspace when the caller passes none
    int64_t own_ws_bytes = 0;
    int num_sms = 0;
    // dense shared expert (shared_format VFMOE_WFMT_BF16): fp16 copies [I][H], [I][H], [H][I] in one
    // allocation, and their tensor maps; the routed launches then run without the shared expert
    int dense_sh = 0;
    __half *sh_dense = nullptr;
    CUtensorMap dsh_gate, dsh_up, dsh_down;
    TcPlan tc;                   // tensor-core launch state (tensor maps)
    Exl3Plan x3;                 // EXL3 trellis tensor maps
    uint64_t wait_ns = 2000000000ull;  // decode GEMV mbarrier wait bound (vfmoe_debug_inject)
    int inject = VFMOE_INJECT_NONE;
    // profiling (vfmoe_profile_enable / vfmoe_profile_read)
    int prof = 0;
    std::vector<cudaEvent_t> ev_pool;         // free events
    std::vector<std::vector<cudaEvent_t>> ev_pending;  // per forward: kNumStages + 1 events
    double stage_ms[8] = {0};
    int64_t n_fwd = 0, launches = 0;
    EpPlacement ep;               // expert-parallel placement (vfmoe_ep_set_placement)
};

struct WsLayout {
    int64_t counts, offsets, perm_tok, pos_of, idx, w, part, xp, act, y, tiles, tile_counts, tiles_cap;
    int64_t xs, act_s, y_s;  // dense shared expert: fp16 x [T][H], fp16 act [T][I], fp32 y [T][H]
    int64_t total;
};

Layer *get_layer(int64_t h);
// A timing event from the handle's pool (nullptr if none could be made).
cudaEvent_t take_event(Layer &L);
int layer_prec(const Layer &L);
WsLayout ws_layout(const Layer &L, int64_t T, int k = -1);
// Workspace base for a call: the caller's (checked against ws_layout) or the handle's own.
int ensure_ws(Layer &L, int64_t T, int64_t ws, int64_t ws_bytes, char **base, int k = -1);
MatrixRef mref(const vfmoe_matrix &m);
// Router of one call into the workspace layout `lay` at base; *idx_p / *w_p = 0: use the workspace's.
int route_impl(Layer &L, int64_t x, int64_t T, char *base, const WsLayout &lay, int32_t **idx_p, float **w_p,
               cudaStream_t st);
// y_out[i] = sum_l w[i,l] * FFN_{slots[i,l]}(rows[i]) (see vfmoe_forward_routed).
int rows_impl(Layer &L, int64_t rows, int64_t rows_dtype, const int32_t *sl, int64_t n, int k, const float *w,
              int64_t y_out, int y_dtype, int skip_negative, int64_t workspace, int64_t ws_bytes, cudaStream_t st);

}  // namespace vfmoe
