// Sigmoid + selection-bias top-k router (native/glm53/moe_ref.py:64-78,
// native/kernels/moe.vyb:32-95).
//
// Expert ids must match a float64 numpy oracle bit for bit, and selection is
// chaotically sensitive (one bf16 ulp on the router input moved a reference MoE
// output by 335%, native/glm53/README.md:367-379), so logits are accumulated in
// float64 from the exact bf16/fp32 inputs.
//
//   router_logits_small  T <= 32 (decode): 2 experts per CTA, K split over 4 warps,
//                        all T tokens per pass; reads W_r once (HBM-bound).
//   router_logits_tiled  T > 32 (prefill): 64x64 output tiles, fp64 FMA.
//   router_topk          warp per token: sigmoid, k rounds of warp argmax (ties -> lowest id),
//                        renormalise, per-expert counts for dispatch.
#include "common.cuh"
#include "kernels.h"

namespace vfmoe {

// Decode shapes (T <= 32): two experts per CTA, each expert's K split over 4 warps;
// every lane keeps TB token accumulators in fp64.  Partials are reduced in a fixed order
// through shared memory, so logits are deterministic and written once (no K-split pass).
template <int TB>
__global__ void __launch_bounds__(256) router_logits_small(const void *__restrict__ x, int x_dtype,
                                                           const float *__restrict__ wr, int T, int H,
                                                           int E, double *__restrict__ logits) {
    __shared__ double red[2][4][TB];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int le = warp >> 2, kq = warp & 3;
    const int e = blockIdx.x * 2 + le;
    const int kc = H / 4;  // H % 512 == 0 -> kc % 128 == 0
    double acc[TB];
#pragma unroll
    for (int t = 0; t < TB; ++t) acc[t] = 0.0;
    if (e < E) {
        const float *wrow = wr + (int64_t)e * H;
        for (int k = kq * kc + lane * 4; k < (kq + 1) * kc; k += 128) {
            const float4 w4 = *reinterpret_cast<const float4 *>(wrow + k);
#pragma unroll
            for (int t = 0; t < TB; ++t) {
                if (t < T) {
                    float xv[4];
                    if (x_dtype == VFMOE_DT_BF16) {
                        const uint2 raw = *reinterpret_cast<const uint2 *>(
                            reinterpret_cast<const __nv_bfloat16 *>(x) + (int64_t)t * H + k);
                        xv[0] = __uint_as_float(raw.x << 16);
                        xv[1] = __uint_as_float(raw.x & 0xFFFF0000u);
                        xv[2] = __uint_as_float(raw.y << 16);
                        xv[3] = __uint_as_float(raw.y & 0xFFFF0000u);
                    } else {
                        const float4 f = *reinterpret_cast<const float4 *>(
                            reinterpret_cast<const float *>(x) + (int64_t)t * H + k);
                        xv[0] = f.x; xv[1] = f.y; xv[2] = f.z; xv[3] = f.w;
                    }
                    double a = acc[t];
                    a = fma((double)xv[0], (double)w4.x, a);
                    a = fma((double)xv[1], (double)w4.y, a);
                    a = fma((double)xv[2], (double)w4.z, a);
                    a = fma((double)xv[3], (double)w4.w, a);
                    acc[t] = a;
                }
            }
        }
    }
#pragma unroll
    for (int t = 0; t < TB; ++t) {
        const double v = warp_sum_f64(acc[t]);
        if (lane == 0) red[le][kq][t] = v;
    }
    __syncthreads();
    if (threadIdx.x < 2 * TB) {
        const int l2 = threadIdx.x / TB, t = threadIdx.x % TB;
        const int e2 = blockIdx.x * 2 + l2;
        if (t < T && e2 < E)
            logits[(int64_t)t * E + e2] = ((red[l2][0][t] + red[l2][1][t]) + red[l2][2][t]) + red[l2][3][t];
    }
}

// 64 tokens x 64 experts per CTA, 256 threads, each 4 tokens x 4 experts, K in chunks of 16.
__global__ void __launch_bounds__(256) router_logits_tiled(const void *__restrict__ x, int x_dtype,
                                                           const float *__restrict__ wr, int T, int H,
                                                           int E, double *__restrict__ part) {
    constexpr int BT = 64, BE = 64, KC = 16;
    __shared__ double xs[KC][BT + 1];
    __shared__ double ws[KC][BE + 1];
    const int t0 = blockIdx.y * BT, e0 = blockIdx.x * BE;
    const int tid = threadIdx.x;
    const int tx = tid & 15, ty = tid >> 4;  // experts e0 + tx + 16j, tokens t0 + ty + 16i
    double acc[4][4];
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[i][j] = 0.0;
    for (int kb = 0; kb < H; kb += KC) {
        // 64 rows x 16 k for each operand = 1024 values; 4 per thread.
#pragma unroll
        for (int r = 0; r < 4; ++r) {
            const int idx = tid + r * 256;
            const int row = idx >> 4, kk = idx & 15;
            const int k = kb + kk;
            const int t = t0 + row;
            double xv = 0.0;
            if (t < T && k < H) xv = (double)ld_act(x, (int64_t)t * H + k, x_dtype);
            xs[kk][row] = xv;
            const int e = e0 + row;
            double wv = 0.0;
            if (e < E && k < H) wv = (double)wr[(int64_t)e * H + k];
            ws[kk][row] = wv;
        }
        __syncthreads();
#pragma unroll
        for (int kk = 0; kk < KC; ++kk) {
            double xr[4], wc[4];
#pragma unroll
            for (int i = 0; i < 4; ++i) xr[i] = xs[kk][ty + 16 * i];
#pragma unroll
            for (int j = 0; j < 4; ++j) wc[j] = ws[kk][tx + 16 * j];
#pragma unroll
            for (int i = 0; i < 4; ++i)
#pragma unroll
                for (int j = 0; j < 4; ++j) acc[i][j] = fma(xr[i], wc[j], acc[i][j]);
        }
        __syncthreads();
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const int t = t0 + ty + 16 * i;
        if (t >= T) continue;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const int e = e0 + tx + 16 * j;
            if (e < E) part[(int64_t)t * E + e] = acc[i][j];
        }
    }
}

// Warp per token.  NPL = experts per lane (E <= 32 * NPL).
template <int NPL>
__global__ void __launch_bounds__(256) router_topk(const double *__restrict__ logits, int T, int E,
                                                   int k, const float *__restrict__ bias, double scale,
                                                   int32_t *__restrict__ idx_out, float *__restrict__ w_out,
                                                   int32_t *__restrict__ counts) {
    const int lane = threadIdx.x & 31;
    const int t = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    if (t >= T) return;
    double score[NPL], choice[NPL];
#pragma unroll
    for (int j = 0; j < NPL; ++j) {
        const int e = lane + 32 * j;
        if (e < E) {
            const double logit = logits[(int64_t)t * E + e];
            const double sc = 1.0 / (1.0 + exp(-logit));
            score[j] = sc;
            const double c = sc + (double)bias[e];
            choice[j] = isnan(c) ? -INFINITY : c;  // NaN never wins; keeps the argmax total
        } else {
            score[j] = 0.0;
            choice[j] = -INFINITY;
        }
    }
    unsigned taken = 0;  // bit j: this lane's expert lane+32j already selected
    int my_e = -1;
    double my_s = 0.0, sum = 0.0;
    for (int r = 0; r < k; ++r) {
        double bv = -INFINITY;
        int bi = 0x7fffffff, bj = -1;
#pragma unroll
        for (int j = 0; j < NPL; ++j) {
            const int e = lane + 32 * j;
            if (e < E && !((taken >> j) & 1u)) {
                if (choice[j] > bv || bj < 0) {  // ascending e within a lane: strict > keeps lowest
                    bv = choice[j];
                    bi = e;
                    bj = j;
                }
            }
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            const double ov = __shfl_xor_sync(0xffffffffu, bv, o);
            const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
            if (ov > bv || (ov == bv && oi < bi)) {
                bv = ov;
                bi = oi;
            }
        }
        // bi is now warp-uniform: the winner.
        const int owner = bi & 31, wj = bi >> 5;
        double ws = 0.0;
#pragma unroll
        for (int j = 0; j < NPL; ++j)
            if (j == wj) ws = score[j];
        ws = __shfl_sync(0xffffffffu, ws, owner);
        if (lane == owner) taken |= 1u << wj;
        sum += ws;
        if (lane == r) {
            my_e = bi;
            my_s = ws;
        }
    }
    if (lane < k) {
        const double wv = my_s / (sum + 1e-20) * scale;
        idx_out[(int64_t)t * k + lane] = my_e;
        w_out[(int64_t)t * k + lane] = (float)wv;
        if (my_e >= 0 && my_e < E) atomicAdd(&counts[my_e], 1);
    }
}

int launch_router(const void *x, int x_dtype, const float *wr, const float *bias, int T, int H, int E,
                  int k, double scale, double *part, int32_t *idx, float *w, int32_t *counts,
                  cudaStream_t st) {
    if (T <= 32 && H % 512 == 0) {
        const unsigned grid = (unsigned)cdiv(E, 2);
        if (T <= 8)
            router_logits_small<8><<<grid, 256, 0, st>>>(x, x_dtype, wr, T, H, E, part);
        else
            router_logits_small<32><<<grid, 256, 0, st>>>(x, x_dtype, wr, T, H, E, part);
        VF_LAUNCH_CHECK("router_logits_small");
    } else {
        dim3 grid((unsigned)cdiv(E, 64), (unsigned)cdiv(T, 64));
        router_logits_tiled<<<grid, 256, 0, st>>>(x, x_dtype, wr, T, H, E, part);
        VF_LAUNCH_CHECK("router_logits_tiled");
    }
    const unsigned tb = (unsigned)cdiv(T, 8);
    const int npl = (int)cdiv(E, 32);
#define VF_TOPK(NPL) router_topk<NPL><<<tb, 256, 0, st>>>(part, T, E, k, bias, scale, idx, w, counts)
    if (npl <= 1) VF_TOPK(1);
    else if (npl <= 2) VF_TOPK(2);
    else if (npl <= 4) VF_TOPK(4);
    else if (npl <= 8) VF_TOPK(8);
    else if (npl <= 16) VF_TOPK(16);
    else VF_TOPK(32);
#undef VF_TOPK
    VF_LAUNCH_CHECK("router_topk");
    return VFMOE_OK;
}

int64_t router_partial_doubles(int T, int H, int E) { return (int64_t)T * E; }

}  // namespace vfmoe
