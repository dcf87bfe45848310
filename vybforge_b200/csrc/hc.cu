// Hyper-connections around the MoE sublayer of a GLM-5.3 layer (multi-stream residual, "mHC").
//
// Reference: hc_glue / hc_apply (native/glm53/glm_engine.vyb:437-612, :783-809) and their numpy
// definition native/glm53/hc_ref.py:27-63 (mix, apply_), used by tail_site around the MoE
// (glm_engine.vyb:1922-1952 shows the same pattern at the attention site).  Per token row r
// the layer keeps HC = 4 residual streams of width D (fp32):
//
//   flat      = streams[r] / rms(streams[r])                      (unweighted, over HC*D)
//   mv        = flat . fn^T                                       (24 = HC + HC + HC*HC values)
//   pre[h]    = sigmoid(mv[h] * scale0 + base[h]) + hc_eps
//   post[h]   = 2 sigmoid(mv[HC+h] * scale1 + base[HC+h])
//   comb      = softmax_rows(mv[2HC..] * scale2 + base[2HC..]) + hc_eps, then column-normalised,
//               then (iters - 1) x {row-normalise, column-normalise}     (Sinkhorn)
//   collapsed = sum_h pre[h] * streams[r, h]                       (the sublayer's input)
//   h         = RMSNorm_w(collapsed)                               (the post-attention layernorm)
// and after the sublayer (y = MoE(h)):
//   streams'[r, h] = post[h] * y[r] + sum_j comb[j, h] * streams[r, j]
//
// hc_mix_kernel: one CTA (512 threads) per row, the whole mix fused.  Thread t holds the four
// streams' values at d = 4t + 2048q (q < D/2048) in registers, so the collapse and both norms
// need no exchange beyond two block reductions; fn (bf16 or fp32 [24][HC*D]) is read once per
// row (L2-resident across rows).  Per-thread partial sums are fp32; the block reductions are
// float-float.  The gates and the 4x4 normalisation run in fp32 on warp 0, one matrix entry per
// lane (row and column sums by shuffles).
// hc_apply_kernel: streaming, HBM-bound (HC*D reads + D reads + HC*D writes per row).
#include "common.cuh"
#include "kernels.h"

namespace vfmoe {

constexpr int kHc = 4;                 // streams (hc_mult of GLM-5.3)
constexpr int kHcMix = 2 * kHc + kHc * kHc;   // 24 mix values per row
constexpr int kHcThreads = 512;

__device__ __forceinline__ float4 ld_fn4(const void *fn, int fn_dtype, int64_t i) {
    if (fn_dtype == VFMOE_DT_BF16) {
        const uint2 u = *reinterpret_cast<const uint2 *>(reinterpret_cast<const __nv_bfloat16 *>(fn) + i);
        return make_float4(__uint_as_float(u.x << 16), __uint_as_float(u.x & 0xFFFF0000u), __uint_as_float(u.y << 16),
                           __uint_as_float(u.y & 0xFFFF0000u));
    }
    return *reinterpret_cast<const float4 *>(reinterpret_cast<const float *>(fn) + i);
}

// Block-wide sums of NV fp32 values per thread (512 threads), in float-float: a TwoSum butterfly
// per warp, then threads 0..NV-1 add the 16 warps' (hi, lo) pairs in warp order; the totals
// (hi + lo, about 48 bits) land in out[] (shared memory) for every thread to read.  All of it runs on the fp32
// pipe: fp64 arithmetic on this part issues at a small fraction of the fp32 rate.
__device__ __forceinline__ void two_sum_f(float a, float b, float &s, float &t) {
    s = a + b;
    const float bb = s - a;
    t = (a - (s - bb)) + (b - bb);
}

template <int NV>
__device__ __forceinline__ void block_sum(const float (&v)[NV], float2 *red /* [16][NV] */, double *out /* [NV] */) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
    for (int i = 0; i < NV; ++i) {
        float hi = v[i], lo = 0.f;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            const float oh = __shfl_xor_sync(0xffffffffu, hi, o), ol = __shfl_xor_sync(0xffffffffu, lo, o);
            float sm, r;
            two_sum_f(hi, oh, sm, r);
            hi = sm;
            lo = lo + ol + r;
        }
        if (lane == 0) red[warp * NV + i] = make_float2(hi, lo);
    }
    __syncthreads();
    if (threadIdx.x < NV) {
        const int i = threadIdx.x;
        float hi = red[i].x, lo = red[i].y;
        for (int w = 1; w < kHcThreads / 32; ++w) {
            float sm, r;
            two_sum_f(hi, red[w * NV + i].x, sm, r);
            hi = sm;
            lo = lo + red[w * NV + i].y + r;
        }
        out[i] = (double)hi + (double)lo;
    }
    __syncthreads();
}

template <int VPT>
__global__ void __launch_bounds__(kHcThreads) hc_mix_kernel(const float *__restrict__ streams, int D,
                                                            const void *__restrict__ fn, int fn_dtype,
                                                            const float *__restrict__ base, const float *__restrict__ scale,
                                                            float rms_eps, double hc_eps, int iters,
                                                            const float *__restrict__ norm_w, float norm_eps,
                                                            void *__restrict__ h_out, int h_dtype,
                                                            float *__restrict__ post_out, float *__restrict__ comb_out) {
    __shared__ float2 red[16 * (kHcMix + 1)];
    __shared__ double s_tot[kHcMix + 1];
    __shared__ float s_pre[kHc];
    const int64_t r = blockIdx.x;
    const int t = threadIdx.x;
    const float *row = streams + r * kHc * D;
    float4 x[kHc][VPT];
    float ss = 0.f;
#pragma unroll
    for (int h = 0; h < kHc; ++h)
#pragma unroll
        for (int q = 0; q < VPT; ++q) {
            x[h][q] = *reinterpret_cast<const float4 *>(row + h * D + 4 * t + 2048 * q);
            ss += x[h][q].x * x[h][q].x + x[h][q].y * x[h][q].y + x[h][q].z * x[h][q].z + x[h][q].w * x[h][q].w;
        }
    // mix values of the raw row (the 1/rms factor is applied to the totals); per-thread partial
    // sums in fp32 (64 VPT products), the block reduction in fp64
    float part[kHcMix + 1];
#pragma unroll
    for (int j = 0; j < kHcMix; ++j) {
        float a = 0.f;
#pragma unroll
        for (int h = 0; h < kHc; ++h)
#pragma unroll
            for (int q = 0; q < VPT; ++q) {
                const float4 f = ld_fn4(fn, fn_dtype, (int64_t)j * kHc * D + h * D + 4 * t + 2048 * q);
                a = fmaf(x[h][q].x, f.x, a);
                a = fmaf(x[h][q].y, f.y, a);
                a = fmaf(x[h][q].z, f.z, a);
                a = fmaf(x[h][q].w, f.w, a);
            }
        part[j] = a;
    }
    part[kHcMix] = ss;
    block_sum<kHcMix + 1>(part, red, s_tot);
    if (t < 32) {
        // warp 0: lane 4a + b holds comb[a][b] (rows: shuffles over lane bits 0-1, columns: bits
        // 2-3); lanes 16-19 pre[h], lanes 20-23 post[h].  fp32 from the float-float totals: the
        // 20 normalisation rounds add about 20 roundings of 2^-24 each.
        const int lane = t;
        const float inv = (float)(1.0 / sqrt(s_tot[kHcMix] / (double)(kHc * D) + (double)rms_eps));
        const float s0 = scale[0], s1 = scale[1], s2 = scale[2];
        const float eps = (float)hc_eps;
        const int a = (lane >> 2) & 3, b = lane & 3;
        float c = (float)s_tot[2 * kHc + a * kHc + b] * inv * s2 + base[2 * kHc + a * kHc + b];
        float mx = c;
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
        c = expf(c - mx);
        float sm = c + __shfl_xor_sync(0xffffffffu, c, 1);
        sm += __shfl_xor_sync(0xffffffffu, sm, 2);
        c = c / sm + eps;
        for (int it = 0; it < iters; ++it) {
            if (it > 0) {
                float rs = c + __shfl_xor_sync(0xffffffffu, c, 1);
                rs += __shfl_xor_sync(0xffffffffu, rs, 2);
                c /= rs + eps;
            }
            float cs = c + __shfl_xor_sync(0xffffffffu, c, 4);
            cs += __shfl_xor_sync(0xffffffffu, cs, 8);
            c /= cs + eps;
        }
        const int h = lane & 3;
        const float zp = (float)s_tot[h] * inv * s0 + base[h];
        const float zq = (float)s_tot[kHc + h] * inv * s1 + base[kHc + h];
        if (lane < 16) {
            comb_out[(r * kHc + a) * kHc + b] = c;
        } else if (lane < 20) {
            s_pre[h] = 1.f / (1.f + expf(-zp)) + eps;
        } else if (lane < 24) {
            post_out[r * kHc + h] = 2.f / (1.f + expf(-zq));
        }
    }
    __syncthreads();
    // collapse, then the weighted RMSNorm over D
    float4 col[VPT];
    float ss2[1] = {0.f};
#pragma unroll
    for (int q = 0; q < VPT; ++q) {
        float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
        for (int h = 0; h < kHc; ++h) {
            const float p = s_pre[h];
            v.x = fmaf(p, x[h][q].x, v.x);
            v.y = fmaf(p, x[h][q].y, v.y);
            v.z = fmaf(p, x[h][q].z, v.z);
            v.w = fmaf(p, x[h][q].w, v.w);
        }
        col[q] = v;
        ss2[0] += v.x * v.x + v.y * v.y + v.z * v.z + v.w * v.w;
    }
    float inv2 = 1.f;
    if (norm_w) {
        block_sum<1>(ss2, red, s_tot);
        if (t == 0) s_pre[0] = (float)(1.0 / sqrt(s_tot[0] / (double)D + (double)norm_eps));  // s_pre is free now
        __syncthreads();
        inv2 = s_pre[0];
    }
#pragma unroll
    for (int q = 0; q < VPT; ++q) {
        const int d = 4 * t + 2048 * q;
        float4 wv = norm_w ? *reinterpret_cast<const float4 *>(norm_w + d) : make_float4(1.f, 1.f, 1.f, 1.f);
        const float o[4] = {col[q].x * inv2 * wv.x, col[q].y * inv2 * wv.y, col[q].z * inv2 * wv.z,
                            col[q].w * inv2 * wv.w};
#pragma unroll
        for (int i = 0; i < 4; ++i) st_act(h_out, r * D + d + i, o[i], h_dtype);
    }
}

// grid (R, D / 1024), 256 threads x 4 columns.  out may alias streams: every thread reads its
// four streams' values at its columns before writing them.
__global__ void __launch_bounds__(256) hc_apply_kernel(const float *__restrict__ streams, const void *__restrict__ y,
                                                       int y_dtype, const float *__restrict__ post,
                                                       const float *__restrict__ comb, int D, float *out) {
    const int64_t r = blockIdx.x;
    const int d = (blockIdx.y * 256 + threadIdx.x) * 4;
    if (d >= D) return;
    float p[kHc], c[kHc][kHc];
#pragma unroll
    for (int h = 0; h < kHc; ++h) p[h] = post[r * kHc + h];
#pragma unroll
    for (int j = 0; j < kHc; ++j)
#pragma unroll
        for (int h = 0; h < kHc; ++h) c[j][h] = comb[(r * kHc + j) * kHc + h];
    float4 s[kHc];
#pragma unroll
    for (int j = 0; j < kHc; ++j) s[j] = *reinterpret_cast<const float4 *>(streams + (r * kHc + j) * D + d);
    const float yv[4] = {ld_act(y, r * D + d, y_dtype), ld_act(y, r * D + d + 1, y_dtype),
                         ld_act(y, r * D + d + 2, y_dtype), ld_act(y, r * D + d + 3, y_dtype)};
#pragma unroll
    for (int h = 0; h < kHc; ++h) {
        float4 o = make_float4(p[h] * yv[0], p[h] * yv[1], p[h] * yv[2], p[h] * yv[3]);
#pragma unroll
        for (int j = 0; j < kHc; ++j) {
            o.x = fmaf(c[j][h], s[j].x, o.x);
            o.y = fmaf(c[j][h], s[j].y, o.y);
            o.z = fmaf(c[j][h], s[j].z, o.z);
            o.w = fmaf(c[j][h], s[j].w, o.w);
        }
        *reinterpret_cast<float4 *>(out + (r * kHc + h) * D + d) = o;
    }
}

// hc_mix_rows_kernel: the same mix for large batches, kHcRows rows per CTA (256 threads, two CTAs
// per SM), so that every hc_fn load serves kHcRows rows (hc_mix_kernel reads all of hc_fn, 24 x 4D
// values, once per row).  Thread t owns float4 chunks g = t + 256 i of the flattened 4 x D row and
// keeps kHcRows x 25 partial sums; the collapse then re-reads the block's rows (L2-resident)
// twice: for the RMSNorm's sum of squares, then for the output.  R = 4096, H = 6144: 0.51 ms
// (one row per CTA: 0.61 ms; four rows per CTA at 255 registers, one CTA per SM: 0.59 ms).  Both
// forms wait on the 24 hc_fn loads of every chunk (L2 latency), not on HBM.
constexpr int kHcRows = 2;
constexpr int64_t kHcRowsMinR = 1024;  // below this, one row per CTA keeps more SMs busy

// The gates and the 4x4 normalisation of one row on one warp (fp32; lane 4a + b holds comb[a][b]).
__device__ __forceinline__ void hc_tail_warp(const double *tot /* 25 */, int D, const float *base, const float *scale,
                                             float rms_eps, double hc_eps, int iters, int64_t r, bool valid,
                                             float *post_out, float *comb_out, float *pre_smem) {
    const int lane = threadIdx.x & 31;
    const float inv = (float)(1.0 / sqrt(tot[kHcMix] / (double)(kHc * D) + (double)rms_eps));
    const float s0 = scale[0], s1 = scale[1], s2 = scale[2];
    const float eps = (float)hc_eps;
    const int a = (lane >> 2) & 3, b = lane & 3;
    float c = (float)tot[2 * kHc + a * kHc + b] * inv * s2 + base[2 * kHc + a * kHc + b];
    float mx = c;
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
    c = expf(c - mx);
    float sm = c + __shfl_xor_sync(0xffffffffu, c, 1);
    sm += __shfl_xor_sync(0xffffffffu, sm, 2);
    c = c / sm + eps;
    for (int it = 0; it < iters; ++it) {
        if (it > 0) {
            float rs = c + __shfl_xor_sync(0xffffffffu, c, 1);
            rs += __shfl_xor_sync(0xffffffffu, rs, 2);
            c /= rs + eps;
        }
        float cs = c + __shfl_xor_sync(0xffffffffu, c, 4);
        cs += __shfl_xor_sync(0xffffffffu, cs, 8);
        c /= cs + eps;
    }
    const int h = lane & 3;
    const float zp = (float)tot[h] * inv * s0 + base[h];
    const float zq = (float)tot[kHc + h] * inv * s1 + base[kHc + h];
    if (lane < 16) {
        if (valid) comb_out[(r * kHc + a) * kHc + b] = c;
    } else if (lane < 20) {
        pre_smem[h] = 1.f / (1.f + expf(-zp)) + eps;
    } else if (lane < 24) {
        if (valid) post_out[r * kHc + h] = 2.f / (1.f + expf(-zq));
    }
}

__global__ void __launch_bounds__(256, 2) hc_mix_rows_kernel(const float *__restrict__ streams, int64_t R, int D,
                                                          const void *__restrict__ fn, int fn_dtype,
                                                          const float *__restrict__ base, const float *__restrict__ scale,
                                                          float rms_eps, double hc_eps, int iters,
                                                          const float *__restrict__ norm_w, float norm_eps,
                                                          void *__restrict__ h_out, int h_dtype,
                                                          float *__restrict__ post_out, float *__restrict__ comb_out) {
    constexpr int NV = kHcRows * (kHcMix + 1);
    __shared__ float2 red[8 * NV];
    __shared__ double s_tot[NV];
    __shared__ float s_pre[kHcRows][kHc];
    __shared__ float s_inv2[kHcRows];
    const int t = threadIdx.x, lane = t & 31, warp = t >> 5;
    const int64_t r0 = (int64_t)blockIdx.x * kHcRows;
    const int nch = kHc * D / 4;  // float4 chunks of a row
    float part[kHcRows][kHcMix + 1];
#pragma unroll
    for (int rb = 0; rb < kHcRows; ++rb)
#pragma unroll
        for (int j = 0; j <= kHcMix; ++j) part[rb][j] = 0.f;
    for (int g = t; g < nch; g += 256) {
        float4 xv[kHcRows];
#pragma unroll
        for (int rb = 0; rb < kHcRows; ++rb) {
            xv[rb] = r0 + rb < R ? *reinterpret_cast<const float4 *>(streams + (r0 + rb) * kHc * D + 4 * (int64_t)g)
                                 : make_float4(0.f, 0.f, 0.f, 0.f);
            part[rb][kHcMix] += xv[rb].x * xv[rb].x + xv[rb].y * xv[rb].y + xv[rb].z * xv[rb].z + xv[rb].w * xv[rb].w;
        }
#pragma unroll
        for (int j = 0; j < kHcMix; ++j) {
            const float4 f = ld_fn4(fn, fn_dtype, (int64_t)j * kHc * D + 4 * (int64_t)g);
#pragma unroll
            for (int rb = 0; rb < kHcRows; ++rb) {
                float a = part[rb][j];
                a = fmaf(xv[rb].x, f.x, a);
                a = fmaf(xv[rb].y, f.y, a);
                a = fmaf(xv[rb].z, f.z, a);
                a = fmaf(xv[rb].w, f.w, a);
                part[rb][j] = a;
            }
        }
    }
    // float-float block sums of the kHcRows x 25 values (8 warps)
#pragma unroll
    for (int rb = 0; rb < kHcRows; ++rb)
#pragma unroll
        for (int j = 0; j <= kHcMix; ++j) {
            float hi = part[rb][j], lo = 0.f;
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) {
                const float oh = __shfl_xor_sync(0xffffffffu, hi, o), ol = __shfl_xor_sync(0xffffffffu, lo, o);
                float sm, rr;
                two_sum_f(hi, oh, sm, rr);
                hi = sm;
                lo = lo + ol + rr;
            }
            if (lane == 0) red[warp * NV + rb * (kHcMix + 1) + j] = make_float2(hi, lo);
        }
    __syncthreads();
    if (t < NV) {
        float hi = red[t].x, lo = red[t].y;
        for (int w = 1; w < 8; ++w) {
            float sm, rr;
            two_sum_f(hi, red[w * NV + t].x, sm, rr);
            hi = sm;
            lo = lo + red[w * NV + t].y + rr;
        }
        s_tot[t] = (double)hi + (double)lo;
    }
    __syncthreads();
    if (warp < kHcRows)
        hc_tail_warp(s_tot + warp * (kHcMix + 1), D, base, scale, rms_eps, hc_eps, iters, r0 + warp, r0 + warp < R,
                     post_out, comb_out, s_pre[warp]);
    __syncthreads();
    // collapse: sum of squares per row (first pass), then the normalised output (second pass)
    auto collapsed = [&](int rb, int d) {
        float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
        for (int h = 0; h < kHc; ++h) {
            const float p = s_pre[rb][h];
            const float4 x = *reinterpret_cast<const float4 *>(streams + ((r0 + rb) * kHc + h) * D + d);
            v.x = fmaf(p, x.x, v.x);
            v.y = fmaf(p, x.y, v.y);
            v.z = fmaf(p, x.z, v.z);
            v.w = fmaf(p, x.w, v.w);
        }
        return v;
    };
    if (norm_w) {
        float ss2[kHcRows];
#pragma unroll
        for (int rb = 0; rb < kHcRows; ++rb) {
            ss2[rb] = 0.f;
            if (r0 + rb < R)
                for (int d = 4 * t; d < D; d += 1024) {
                    const float4 v = collapsed(rb, d);
                    ss2[rb] += v.x * v.x + v.y * v.y + v.z * v.z + v.w * v.w;
                }
        }
#pragma unroll
        for (int rb = 0; rb < kHcRows; ++rb) {
            float hi = ss2[rb], lo = 0.f;
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) {
                const float oh = __shfl_xor_sync(0xffffffffu, hi, o), ol = __shfl_xor_sync(0xffffffffu, lo, o);
                float sm, rr;
                two_sum_f(hi, oh, sm, rr);
                hi = sm;
                lo = lo + ol + rr;
            }
            if (lane == 0) red[warp * kHcRows + rb] = make_float2(hi, lo);
        }
        __syncthreads();
        if (t < kHcRows) {
            float hi = red[t].x, lo = red[t].y;
            for (int w = 1; w < 8; ++w) {
                float sm, rr;
                two_sum_f(hi, red[w * kHcRows + t].x, sm, rr);
                hi = sm;
                lo = lo + red[w * kHcRows + t].y + rr;
            }
            s_inv2[t] = (float)(1.0 / sqrt(((double)hi + (double)lo) / (double)D + (double)norm_eps));
        }
        __syncthreads();
    }
#pragma unroll
    for (int rb = 0; rb < kHcRows; ++rb) {
        if (r0 + rb >= R) continue;
        const float inv2 = norm_w ? s_inv2[rb] : 1.f;
        for (int d = 4 * t; d < D; d += 1024) {
            const float4 v = collapsed(rb, d);
            const float4 wv = norm_w ? *reinterpret_cast<const float4 *>(norm_w + d) : make_float4(1.f, 1.f, 1.f, 1.f);
            const float o[4] = {v.x * inv2 * wv.x, v.y * inv2 * wv.y, v.z * inv2 * wv.z, v.w * inv2 * wv.w};
#pragma unroll
            for (int i = 0; i < 4; ++i) st_act(h_out, (r0 + rb) * D + d + i, o[i], h_dtype);
        }
    }
}

// hc_mix_tc_kernel: the mix for batches of rows with a bf16 hc_fn, the 24 dot products on the
// tensor pipe.  A CTA takes kHcTcRows = 16 rows (one m16 tile); warp w takes the flattened K = 4D
// range [w K/8, (w + 1) K/8) of all 16 rows, so every hc_fn value loaded serves 16 rows.
//   mma.sync m16n8k8 tf32, three n8 tiles (the 24 mix values): A = stream values, B = hc_fn rows.
//   A value x is split into hi = x with the low 13 mantissa bits cleared (exact in tf32) and
//   lo = tf32_rn(x - hi) (x - hi is exact in fp32, |x - hi| < 2^-10 |x|), so x = hi + lo to
//   about 2^-21 |x|; bf16 hc_fn is exact in tf32 and every product exact in fp32.
//   K permutation inside a k16 chunk: thread (g, c) loads the float4 at k = 4c of rows g and g + 8
//   and the four bf16 at k = 4c of hc_fn row 8 nt + g; its MMA slots c and c + 4 of step s take
//   k = 4c + 2s and 4c + 2s + 1, the same for A and B, so the products are those of the plain
//   dot product.
//   Accuracy: the fp32 accumulators restart every 64 K (16 MMAs) and are added into float-float
//   totals (TwoSum); the sum of squares likewise.  The warps' totals are added in warp order.
// Then, as hc_mix_rows_kernel: the gates and the normalisation (hc_tail_warp, two rows per warp),
// and the collapse with its RMSNorm, one row at a time from registers.  The collapse re-reads the
// block's 16 rows after every CTA has streamed its own, so most of that re-read comes from HBM
// (about 845 MB of DRAM traffic for 453 MB of data at R = 4096, D = 6144).
constexpr int kHcTcRows = 16;
constexpr int64_t kHcTcMinR = 256;

__device__ __forceinline__ void mma_tf32_16808(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                               uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k8.row.col.f32.tf32.tf32.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
        "{%0, %1, %2, %3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

__device__ __forceinline__ uint32_t tf32_rn(float x) {
    uint32_t r;
    asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(r) : "f"(x));
    return r;
}

__device__ __forceinline__ void ff_acc(float &hi, float &lo, float v) {
    float sm, r;
    two_sum_f(hi, v, sm, r);
    hi = sm;
    lo += r;
}

template <int CH>  // D / 1024
__global__ void __launch_bounds__(256, 2) hc_mix_tc_kernel(const float *__restrict__ streams, int64_t R, int D,
                                                         const __nv_bfloat16 *__restrict__ fn,
                                                         const float *__restrict__ base, const float *__restrict__ scale,
                                                         float rms_eps, double hc_eps, int iters,
                                                         const float *__restrict__ norm_w, float norm_eps,
                                                         void *__restrict__ h_out, int h_dtype,
                                                         float *__restrict__ post_out, float *__restrict__ comb_out) {
    constexpr int NV = kHcMix + 1;
    __shared__ float2 red[8][kHcTcRows][NV];
    __shared__ double s_tot[kHcTcRows][NV];
    __shared__ float s_pre[kHcTcRows][kHc];
    __shared__ float s_inv2[kHcTcRows];
    const int t = threadIdx.x, lane = t & 31, warp = t >> 5;
    const int g = lane >> 2, c = lane & 3;
    const int64_t r0 = (int64_t)blockIdx.x * kHcTcRows;
    const int64_t K = (int64_t)kHc * D;
    const int kw = (int)(K / 8);
    const bool va = r0 + g < R, vb = r0 + g + 8 < R;
    const float *xa = streams + (va ? (r0 + g) * K : 0) + (int64_t)warp * kw + 4 * c;
    const float *xb = streams + (vb ? (r0 + g + 8) * K : 0) + (int64_t)warp * kw + 4 * c;
    const __nv_bfloat16 *f0 = fn + (int64_t)g * K + (int64_t)warp * kw + 4 * c;  // n tile nt: + 8 nt K

    float acc[3][4], fh[3][4], fl[3][4];
#pragma unroll
    for (int nt = 0; nt < 3; ++nt)
#pragma unroll
        for (int e = 0; e < 4; ++e) acc[nt][e] = fh[nt][e] = fl[nt][e] = 0.f;
    float ssa = 0.f, ssb = 0.f, sha = 0.f, sla = 0.f, shb = 0.f, slb = 0.f;
    for (int k = 0; k < kw; k += 64) {
        float4 xv[2][4];
        uint2 fv[3][4];
#pragma unroll
        for (int q = 0; q < 4; ++q) {
            xv[0][q] = va ? *reinterpret_cast<const float4 *>(xa + k + 16 * q) : make_float4(0.f, 0.f, 0.f, 0.f);
            xv[1][q] = vb ? *reinterpret_cast<const float4 *>(xb + k + 16 * q) : make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
            for (int nt = 0; nt < 3; ++nt)
                fv[nt][q] = *reinterpret_cast<const uint2 *>(f0 + 8 * nt * K + k + 16 * q);
        }
#pragma unroll
        for (int q = 0; q < 4; ++q) {
            ssa = fmaf(xv[0][q].x, xv[0][q].x, fmaf(xv[0][q].y, xv[0][q].y, fmaf(xv[0][q].z, xv[0][q].z, fmaf(xv[0][q].w, xv[0][q].w, ssa))));
            ssb = fmaf(xv[1][q].x, xv[1][q].x, fmaf(xv[1][q].y, xv[1][q].y, fmaf(xv[1][q].z, xv[1][q].z, fmaf(xv[1][q].w, xv[1][q].w, ssb))));
#pragma unroll
            for (int s2 = 0; s2 < 2; ++s2) {
                const float a0 = s2 ? xv[0][q].z : xv[0][q].x, a1 = s2 ? xv[0][q].w : xv[0][q].y;
                const float b0 = s2 ? xv[1][q].z : xv[1][q].x, b1 = s2 ? xv[1][q].w : xv[1][q].y;
                const uint32_t ha0 = __float_as_uint(a0) & 0xFFFFE000u, ha1 = __float_as_uint(a1) & 0xFFFFE000u;
                const uint32_t hb0 = __float_as_uint(b0) & 0xFFFFE000u, hb1 = __float_as_uint(b1) & 0xFFFFE000u;
                const uint32_t la0 = tf32_rn(a0 - __uint_as_float(ha0)), la1 = tf32_rn(a1 - __uint_as_float(ha1));
                const uint32_t lb0 = tf32_rn(b0 - __uint_as_float(hb0)), lb1 = tf32_rn(b1 - __uint_as_float(hb1));
#pragma unroll
                for (int nt = 0; nt < 3; ++nt) {
                    const uint32_t w = s2 ? fv[nt][q].y : fv[nt][q].x;
                    const uint32_t f_lo = w << 16, f_hi = w & 0xFFFF0000u;  // k = 4c + 2 s2, 4c + 2 s2 + 1
                    // A slots: (row g, c) (row g + 8, c) (row g, c + 4) (row g + 8, c + 4)
                    mma_tf32_16808(acc[nt], ha0, hb0, ha1, hb1, f_lo, f_hi);
                    mma_tf32_16808(acc[nt], la0, lb0, la1, lb1, f_lo, f_hi);
                }
            }
        }
#pragma unroll
        for (int nt = 0; nt < 3; ++nt)
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                ff_acc(fh[nt][e], fl[nt][e], acc[nt][e]);
                acc[nt][e] = 0.f;
            }
        ff_acc(sha, sla, ssa);
        ff_acc(shb, slb, ssb);
        ssa = ssb = 0.f;
    }
    // sums of squares: the quad's four threads share a row pair
#pragma unroll
    for (int o = 1; o < 4; o <<= 1) {
        float oh = __shfl_xor_sync(0xffffffffu, sha, o), ol = __shfl_xor_sync(0xffffffffu, sla, o);
        float sm, rr;
        two_sum_f(sha, oh, sm, rr);
        sha = sm;
        sla = sla + ol + rr;
        oh = __shfl_xor_sync(0xffffffffu, shb, o);
        ol = __shfl_xor_sync(0xffffffffu, slb, o);
        two_sum_f(shb, oh, sm, rr);
        shb = sm;
        slb = slb + ol + rr;
    }
    // accumulator element e of tile nt: row g + 8 (e >> 1), mix value 8 nt + 2c + (e & 1)
#pragma unroll
    for (int nt = 0; nt < 3; ++nt)
#pragma unroll
        for (int e = 0; e < 4; ++e) red[warp][g + 8 * (e >> 1)][8 * nt + 2 * c + (e & 1)] = make_float2(fh[nt][e], fl[nt][e]);
    if (c == 0) {
        red[warp][g][kHcMix] = make_float2(sha, sla);
        red[warp][g + 8][kHcMix] = make_float2(shb, slb);
    }
    __syncthreads();
    for (int i = t; i < kHcTcRows * NV; i += 256) {
        const int rr = i / NV, j = i % NV;
        float hi = red[0][rr][j].x, lo = red[0][rr][j].y;
#pragma unroll
        for (int w = 1; w < 8; ++w) {
            float sm, e2;
            two_sum_f(hi, red[w][rr][j].x, sm, e2);
            hi = sm;
            lo = lo + red[w][rr][j].y + e2;
        }
        s_tot[rr][j] = (double)hi + (double)lo;
    }
    __syncthreads();
    for (int rr = warp; rr < kHcTcRows; rr += 8)
        hc_tail_warp(s_tot[rr], D, base, scale, rms_eps, hc_eps, iters, r0 + rr, r0 + rr < R, post_out, comb_out,
                     s_pre[rr]);
    __syncthreads();
    // collapse and RMSNorm, one row at a time: thread t holds the row's collapsed values at
    // d = 4t + 1024q (q < CH) in registers, its loads issued in batches of four chunks (16 float4)
    // before they are used; one float-float block sum for the row's sum of squares, then the
    // normalised output from the same registers.
    const int nrow = (int)(R - r0 < kHcTcRows ? R - r0 : kHcTcRows);
    float2 *red2 = &red[0][0][0];  // [8 warps], per row
    for (int rb = 0; rb < nrow; ++rb) {
        float4 hv[CH];
        float ss2 = 0.f;
        const float *rowp = streams + (r0 + rb) * K + 4 * t;
#pragma unroll
        for (int q0 = 0; q0 < CH; q0 += 4) {
            float4 xs[4][kHc];
#pragma unroll
            for (int qq = 0; qq < 4; ++qq)
                if (q0 + qq < CH)
#pragma unroll
                    for (int h = 0; h < kHc; ++h)
                        xs[qq][h] = *reinterpret_cast<const float4 *>(rowp + (int64_t)h * D + 1024 * (q0 + qq));
#pragma unroll
            for (int qq = 0; qq < 4; ++qq)
                if (q0 + qq < CH) {
                    float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
                    for (int h = 0; h < kHc; ++h) {
                        const float p = s_pre[rb][h];
                        v.x = fmaf(p, xs[qq][h].x, v.x);
                        v.y = fmaf(p, xs[qq][h].y, v.y);
                        v.z = fmaf(p, xs[qq][h].z, v.z);
                        v.w = fmaf(p, xs[qq][h].w, v.w);
                    }
                    hv[q0 + qq] = v;
                    ss2 += v.x * v.x + v.y * v.y + v.z * v.z + v.w * v.w;
                }
        }
        float inv2 = 1.f;
        if (norm_w) {
            float hi = ss2, lo = 0.f;
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) {
                const float oh = __shfl_xor_sync(0xffffffffu, hi, o), ol = __shfl_xor_sync(0xffffffffu, lo, o);
                float sm, rr;
                two_sum_f(hi, oh, sm, rr);
                hi = sm;
                lo = lo + ol + rr;
            }
            if (lane == 0) red2[(rb & 1) * 8 + warp] = make_float2(hi, lo);  // two buffers: no second barrier
            __syncthreads();
            hi = red2[(rb & 1) * 8].x;
            lo = red2[(rb & 1) * 8].y;
#pragma unroll
            for (int w = 1; w < 8; ++w) {
                float sm, rr;
                two_sum_f(hi, red2[(rb & 1) * 8 + w].x, sm, rr);
                hi = sm;
                lo = lo + red2[(rb & 1) * 8 + w].y + rr;
            }
            inv2 = (float)(1.0 / sqrt(((double)hi + (double)lo) / (double)D + (double)norm_eps));
        }
#pragma unroll
        for (int q = 0; q < CH; ++q) {
            const int d = 4 * t + 1024 * q;
            const float4 wv = norm_w ? *reinterpret_cast<const float4 *>(norm_w + d) : make_float4(1.f, 1.f, 1.f, 1.f);
            const float o[4] = {hv[q].x * inv2 * wv.x, hv[q].y * inv2 * wv.y, hv[q].z * inv2 * wv.z,
                                hv[q].w * inv2 * wv.w};
#pragma unroll
            for (int i = 0; i < 4; ++i) st_act(h_out, (r0 + rb) * D + d + i, o[i], h_dtype);
        }
    }
}

int launch_hc_mix(const float *streams, int64_t R, int D, const void *fn, int fn_dtype, const float *base,
                  const float *scale, float rms_eps, double hc_eps, int iters, const float *norm_w, float norm_eps,
                  void *h_out, int h_dtype, float *post, float *comb, cudaStream_t st) {
    if (R == 0) return VFMOE_OK;
    if (fn_dtype == VFMOE_DT_BF16 && R >= kHcTcMinR && D % 2048 == 0 && D >= 2048 && D <= 8192) {
        const dim3 grid((unsigned)cdiv(R, kHcTcRows));
        const __nv_bfloat16 *f = reinterpret_cast<const __nv_bfloat16 *>(fn);
        switch (D / 1024) {
#define VF_HC_TC(CH)                                                                                                 \
    case CH:                                                                                                        \
        hc_mix_tc_kernel<CH><<<grid, 256, 0, st>>>(streams, R, D, f, base, scale, rms_eps, hc_eps, iters, norm_w,      \
                                                   norm_eps, h_out, h_dtype, post, comb);                           \
        break;
            VF_HC_TC(2)
            VF_HC_TC(4)
            VF_HC_TC(6)
            VF_HC_TC(8)
#undef VF_HC_TC
        }
        VF_LAUNCH_CHECK("hc_mix_tc_kernel");
        return VFMOE_OK;
    }
    if (R >= kHcRowsMinR && D % 1024 == 0) {
        hc_mix_rows_kernel<<<(unsigned)cdiv(R, kHcRows), 256, 0, st>>>(streams, R, D, fn, fn_dtype, base, scale, rms_eps,
                                                                      hc_eps, iters, norm_w, norm_eps, h_out, h_dtype,
                                                                      post, comb);
        VF_LAUNCH_CHECK("hc_mix_rows_kernel");
        return VFMOE_OK;
    }
    switch (D / 2048) {
        case 1: hc_mix_kernel<1><<<(unsigned)R, kHcThreads, 0, st>>>(streams, D, fn, fn_dtype, base, scale, rms_eps, hc_eps, iters, norm_w, norm_eps, h_out, h_dtype, post, comb); break;
        case 2: hc_mix_kernel<2><<<(unsigned)R, kHcThreads, 0, st>>>(streams, D, fn, fn_dtype, base, scale, rms_eps, hc_eps, iters, norm_w, norm_eps, h_out, h_dtype, post, comb); break;
        case 3: hc_mix_kernel<3><<<(unsigned)R, kHcThreads, 0, st>>>(streams, D, fn, fn_dtype, base, scale, rms_eps, hc_eps, iters, norm_w, norm_eps, h_out, h_dtype, post, comb); break;
        case 4: hc_mix_kernel<4><<<(unsigned)R, kHcThreads, 0, st>>>(streams, D, fn, fn_dtype, base, scale, rms_eps, hc_eps, iters, norm_w, norm_eps, h_out, h_dtype, post, comb); break;
        default:
            set_error("hyper-connection mix: D = %d (2048, 4096, 6144 or 8192 supported)", D);
            return VFMOE_ERR_UNSUPPORTED;
    }
    VF_LAUNCH_CHECK("hc_mix_kernel");
    return VFMOE_OK;
}

int launch_hc_apply(const float *streams, const void *y, int y_dtype, const float *post, const float *comb, int64_t R,
                    int D, float *out, cudaStream_t st) {
    if (R == 0) return VFMOE_OK;
    dim3 grid((unsigned)R, (unsigned)cdiv(D, 1024));
    hc_apply_kernel<<<grid, 256, 0, st>>>(streams, y, y_dtype, post, comb, D, out);
    VF_LAUNCH_CHECK("hc_apply_kernel");
    return VFMOE_OK;
}

}  // namespace vfmoe
