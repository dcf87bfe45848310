// Internal launch interface between the C-ABI layer (api.cu) and the kernels.
#pragma once

#include <functional>

#include "common.cuh"

namespace vfmoe {

struct MatrixRef {
    const uint8_t *data;     // Q8_0 rows or EXL3 trellis of expert 0
    int64_t expert_stride;   // bytes
    const __half *suh;       // EXL3 only
    int64_t suh_stride;      // bytes
    const __half *svh;
    int64_t svh_stride;
};

// Everything the expert kernels need for one forward (passed by value).
struct MoeArgs {
    int T, H, I, E, k;
    int has_shared;
    int fmt, exl3_bits;
    float limit;
    MatrixRef gate, up, down, sh_gate, sh_up, sh_down;
    const int32_t *offsets;    // [E+2]: segment e = rows [offsets[e], offsets[e+1]); E = shared;
                               // offsets[E+1] = rows dispatched
    const int32_t *perm_tok;   // [T*k + T]
    const __half *xp;          // [T*k + T, H] gathered activations (fp16)
    __half *act;               // [T*k + T, I] SwiGLU output (fp16)
    float *y;                  // [T*k + T, H] expert outputs (fp32)
    int *err;
    int prec;                  // fp32 activations: split-precision decode GEMV (two fp16 planes per
                               // row of xp and act, the second at + rows * H / + rows * I elements)
    uint64_t wait_ns;          // bound of the decode GEMV's mbarrier waits
    int inject;                // VFMOE_INJECT_* (tests only; 0 in production)
    int4 *tiles;               // tensor-core path: two tile lists of tiles_cap entries each
    int32_t *tile_counts;      // [2]
    int64_t tiles_cap;
    int plan_ready;            // the decode front end already wrote the decode GEMV's tile lists
};

// Router: fp32 logits -> candidate filter -> float-float / f64 refinement (exact f64 ordering).
// nw = |W_r row|_2 upper bounds (launch_router_norms, once per layer); logits = scratch of
// router_logit_floats(T, H, E, wr_split != 0) floats.  wr_split (bf16 [2][E][H], w_hi then w_lo,
// launch_router_split once per layer; may be 0) enables the tensor-core logits for bf16 x at T > 32.
// counts [E + 2] is zeroed here (by the first level's kernel at T <= 32, else a memset) and then
// accumulates the selections per expert.
int launch_router(const void *x, int x_dtype, const float *wr, const __nv_bfloat16 *wr_split, const float *nw,
                  const float *bias, int T, int H, int E, int k, double scale, float *logits, int32_t *idx, float *w,
                  int32_t *counts, int *err, cudaStream_t st);
int launch_router_norms(const float *wr, int H, int E, float *nw, cudaStream_t st);
int64_t router_logit_floats(int T, int H, int E, bool tc);
// First level only: fp32 logits [T][E] into out (partials in part), and the constant c1 with
// |logit - exact| <= c1 * |x_t|_2 * |w_e|_2.
int launch_route_logits(const void *x, int x_dtype, const float *wr, const __nv_bfloat16 *wr_split, int T, int H,
                        int E, float *part, float *out, int *err, cudaStream_t st, float *c1);
// tensor-core logits (router_tc.cu)
bool router_tc_shape(int T, int H, int E);
int router_tc_splits(int T, int H, int E);
float router_tc_bound(int H);
int launch_router_split(const float *wr, int64_t n, __nv_bfloat16 *hi, __nv_bfloat16 *lo, cudaStream_t st);
int launch_router_logits_tc(const void *x, const __nv_bfloat16 *wr_split, int T, int H, int E, float *logits, int *err,
                            cudaStream_t st);

int launch_dispatch(const int32_t *idx, const int32_t *counts, int T, int E, int k, int has_shared, int32_t *perm_tok,
                    int32_t *pos_of, int32_t *offsets, int *err, cudaStream_t st);
int launch_count(const int32_t *ids, int64_t n, int nb, int32_t *counts, int *err, cudaStream_t st,
                 int skip_negative = 0);
// rows = launch size (an upper bound); *n_rows (device) = rows the dispatch produced.
// planes = 2 (fp32 x): xp + rows * H receives fp16((x - fp16(x)) * 2^12) of every row.
int launch_gather(const void *x, int x_dtype, const int32_t *perm_tok, int64_t rows, int H, __half *xp,
                  const int32_t *n_rows, cudaStream_t st, int planes = 1);
int launch_combine(const void *y, int y_dtype, const int32_t *pos_of, const float *w, int T, int H, int k,
                   const void *y_shared, void *out, int out_dtype, cudaStream_t st);
// Decode front end (T <= kDecodeFrontMaxT, E <= 1024): launch_dispatch + launch_gather + the decode
// GEMV's tile lists (ng rows per tile, both lists) in one launch, with the same results.
constexpr int kDecodeFrontMaxT = 64;
int launch_decode_front(const int32_t *idx, const int32_t *counts, int T, int E, int k, int has_shared, const void *x,
                        int x_dtype, int H, int32_t *perm_tok, int32_t *pos_of, int32_t *offsets, __half *xp, int planes,
                        int ng, int4 *tiles, int64_t cap, int32_t *tile_counts, int *err, cudaStream_t st);

// `mid` runs between the gate/up and the down launches (profiling marks).
int launch_experts_simt(const MoeArgs &a, cudaStream_t st, const std::function<void()> &mid);

// Hyper-connections (hc.cu): streams fp32 [R, 4, D], D in {2048, 4096, 6144, 8192}.
int launch_hc_mix(const float *streams, int64_t R, int D, const void *fn, int fn_dtype, const float *base,
                  const float *scale, float rms_eps, double hc_eps, int iters, const float *norm_w, float norm_eps,
                  void *h_out, int h_dtype, float *post, float *comb, cudaStream_t st);
int launch_hc_apply(const float *streams, const void *y, int y_dtype, const float *post, const float *comb, int64_t R,
                    int D, float *out, cudaStream_t st);

// dst[i] = fp16(src[i]), src BF16 / F16 / F32.
int launch_to_f16(const void *src, int dtype, int64_t n, __half *dst, cudaStream_t st);

int launch_rmsnorm(const void *x, const float *w, void *y, int64_t S, int D, float eps, int dtype,
                   cudaStream_t st);
int launch_residual_rmsnorm(const void *x, const void *y, const float *w, void *x_out, void *h, int64_t S, int D,
                            float eps, int dtype, cudaStream_t st);
int launch_q8_0_dequant(const uint8_t *src, void *dst, int64_t rows, int64_t k, int dst_dtype,
                        cudaStream_t st);
int launch_q8_0_quantize(const float *src, uint8_t *dst, int64_t rows, int64_t k, cudaStream_t st);
int launch_q8_0_tile(const uint8_t *src, uint8_t *dst, int64_t rows, int64_t k, int64_t n_mats, cudaStream_t st);
int launch_exl3_decode(const uint16_t *trellis, __half *dst, int64_t K, int64_t N, int bits,
                       cudaStream_t st);

}  // namespace vfmoe
