// Tensor-core (tcgen05) grouped expert GEMMs: launch state and entry points.
#pragma once

#include <cuda.h>

#include "kernels.h"
#include "sm100.cuh"

namespace vfmoe {

struct TcPlan {
    int ready = 0;
    int num_sms = 0;
    int path = VFMOE_PATH_AUTO;  // the descriptor's expert_path
    // Q8_0 weight tensor maps (3D: [experts][rows][row bytes as u16]).
    CUtensorMap gate, up, down;          // routed, stacked
    CUtensorMap sh_gate, sh_up, sh_down; // shared expert (one "expert")
    // 64-row boxes for the decode GEMV's gate/up tiles
    CUtensorMap gate64, up64, sh_gate64, sh_up64;
    // VFMOE_WFMT_Q8_0_TILED: weight bases and expert strides, read by 1D bulk copies
    // (no tensor maps)
    int tiled = 0;
    const uint8_t *p_gate = nullptr, *p_up = nullptr, *p_down = nullptr;
    const uint8_t *p_sh_gate = nullptr, *p_sh_up = nullptr, *p_sh_down = nullptr;
    int64_t s_gate = 0, s_up = 0, s_down = 0;
};

// Kernel parameters shared by the tcgen05 GEMM and the decode GEMV (passed __grid_constant__).
struct TcParams {
    CUtensorMap wa, wb, swa, swb;   // weights: routed A/B matrices, shared A/B (3D u16 maps)
    CUtensorMap xt;                 // token rows, fp16 [rows][K], SWIZZLE_128B
    // tiled != 0: the weights are VFMOE_WFMT_Q8_0_TILED and read from these bases instead of
    // the maps (routed A/B with expert strides, shared A/B)
    const uint8_t *pa, *pb, *spa, *spb;
    int64_t sa, sb;
    int tiled;
    const int4 *tiles;              // {expert, row0, nrows, 0}
    const int32_t *n_tiles;
    int E, K, M;
    int ld_out;
    void *out;
    float limit;
    int *err;
    // decode GEMV only:
    // prec != 0 (fp32 activations): xt2 maps the second fp16 plane of the token rows (the
    // residual x - fp16(x), times 2^12); gate/up write act as two fp16 planes, the second at
    // out + out_plane elements
    CUtensorMap xt2;
    int prec;
    int64_t out_plane;
    uint64_t wait_ns;  // bound of every mbarrier wait (2 s unless a test shortens it)
    int stall;         // test-only injection: the producer issues no loads (VFMOE_INJECT_STALL_LOADS)
    // dense fp16 weights (a shared expert stored as bf16, converted at create): wa / wb map the
    // single matrices [rows][K] with 64 x ROWS boxes, SWIZZLE_128B; no tile list: dense_T token
    // rows of the token map, tiles of N rows in order
    int dense_T;
};

int tc_plan_create(const vfmoe_layer_desc &d, TcPlan &plan);

// VFMOE_WFMT_Q8_0_TILED: a Q8_0 matrix [rows][K] is stored as tiles of 64 rows x 256 K
// (64 x 272 B = 17,408 B; each tile row is that row's 8 GGUF blocks), tile (rt, kr) at
// byte ((rt * K/256) + kr) * 17,408.  One weight stage of a 64-row tile is one contiguous
// copy: the TMA tensor path moves GGUF's 272-byte row pieces at about 70 GB/s per SM, a
// contiguous bulk copy at about 117 GB/s.
constexpr int kQ8Tile = 64 * 272;

// Weight stage (rows m0 .. m0 + rows - 1, K = 256 * kr .. + 255) of expert z of a tiled
// matrix into dst as rows / 64 bulk copies, completion on bar.
__device__ __forceinline__ void load_q8_tiled(uint8_t *dst, const uint8_t *base, int64_t estride, int z, int m0,
                                              int rows, int KR, int kr, uint64_t *bar) {
    const uint8_t *src = base + (int64_t)z * estride + ((int64_t)(m0 >> 6) * KR + kr) * kQ8Tile;
    for (int h = 0; h < (rows >> 6); ++h)
        sm100::bulk_load(dst + h * kQ8Tile, src + (int64_t)h * KR * kQ8Tile, kQ8Tile, bar);
}
bool tc_supported(const TcPlan &plan, const MoeArgs &a);
// launch_experts_tc runs the decode GEMV (few rows per expert, forced GEMV, or fp32 activations).
bool tc_decode_gemv(const TcPlan &plan, const MoeArgs &a);
int launch_experts_tc(const TcPlan &plan, const MoeArgs &a, cudaStream_t st, const std::function<void()> &mid);

// Dense fp16 expert (expert_gemv.cu): gate/up + SwiGLU then down over T token rows of xs
// (fp16 [T][H]), act_s fp16 [T][I], y_s fp32 [T][H]; maps from make_dense_map.
int make_dense_map(CUtensorMap *m, const void *base, int64_t rows, int64_t k, int box_rows);
int launch_dense_expert(const CUtensorMap &gate, const CUtensorMap &up, const CUtensorMap &down, const __half *xs,
                        int T, int H, int I, __half *act_s, float *y_s, float limit, int *err, int num_sms,
                        uint64_t wait_ns, cudaStream_t st);

// Decode path (few tokens per expert): TMA + register-operand MMA GEMV (expert_gemv.cu).
int gemv_tokens_per_tile(int T, int k, int E);
// a.prec: tok_gu2 / tok_dn2 map the second fp16 planes of xp and act.
int launch_experts_gemv(const TcPlan &plan, const MoeArgs &a, cudaStream_t st, const std::function<void()> &mid,
                        const CUtensorMap &tok_gu, const CUtensorMap &tok_dn, const CUtensorMap *tok_gu2 = nullptr,
                        const CUtensorMap *tok_dn2 = nullptr);

// Builds the (expert, token-tile) lists for both GEMMs on the device (n_gu / n_dn rows per tile).
int launch_tc_plan(const MoeArgs &a, int n_gu, int n_dn, cudaStream_t st);

// EXL3 3-bpw experts (exl3.cu): trellis tensor maps, one per projection.
struct Exl3Plan {
    int ready = 0;
    int num_sms = 0;
    int bits = 3;  // 3 (this library's layout) or 4 (the reference's)
    CUtensorMap gate, up, down;
    CUtensorMap sh_gate, sh_up, sh_down;
};
int exl3_plan_create(const vfmoe_layer_desc &d, Exl3Plan &plan);
// Gathers and rotates the token rows itself (x_perm holds two rotated copies per row:
// gate and up input bases), then the decode GEMVs.  `x` = the rows in caller order.
int launch_experts_exl3(const Exl3Plan &plan, const MoeArgs &a, const void *x, int x_dtype, cudaStream_t st,
                        const std::function<void()> &mid);

// Workspace the tensor-core path needs beyond MoeArgs: tile lists for both GEMMs.
int64_t tc_tiles_capacity(int T, int k, int E);

}  // namespace vfmoe
