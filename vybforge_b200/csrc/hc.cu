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

int launch_hc_mix(const float *streams, int64_t R, int D, const void *fn, int fn_dtype, const float *base,
                  const float *scale, float rms_eps, double hc_eps, int iters, const float *norm_w, float norm_eps,
                  void *h_out, int h_dtype, float *post, float *comb, cudaStream_t st) {
    if (R == 0) return VFMOE_OK;
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
