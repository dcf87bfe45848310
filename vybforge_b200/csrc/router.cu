// Sigmoid + selection-bias top-k router (native/glm53/moe_ref.py:64-78,
// native/kernels/moe.vyb:32-95).
//
// Expert ids must equal those of a float64 numpy oracle, and selection is chaotically
// sensitive (one bf16 ulp on the router input moved a reference MoE output by 335%,
// native/glm53/README.md:367-379).  Vector fp64 on this part runs at ~2 FMA/clk/SM,
// so the router establishes the f64 ordering in three levels, each with a rigorous
// error bound:
//
//   L1  router_logits_f32_*  fp32 logits for every (token, expert).  Error bound
//       |L1 - exact| <= c1 * |x_t|_2 * |w_e|_2 (Cauchy-Schwarz on sum |x_i w_i|, c1 = the
//       gamma_n of the kernel's summation depth, doubled for safety).
//   L2  router_refine        keeps every expert that can still be in the top k
//       (approx choice + bound >= k-th largest of approx choice - bound), recomputes
//       their logits with float-float arithmetic (TwoProduct + TwoSum, error
//       <= c2 * |x|*|w| with c2 ~ 1e-9) and sorts them in f64.
//   L3  (same kernel)        if two neighbours among the top k+1 are closer than the L2
//       bound, their logits are recomputed with fp64 FMA and re-sorted (lowest id wins
//       exact ties).  Rare: ~1e-4 of tokens on random inputs; exact ties always take it.
//
// Weights w = score / (sum + 1e-20) * scale use the L2/L3 f64 scores.
#include <algorithm>

#include "common.cuh"
#include "kernels.h"

namespace vfmoe {

constexpr int kMaxCand = 128;
constexpr int kMaxH = 16384;     // router_refine keeps x_t in shared memory (fp32)
constexpr int kMaxChunks = 32;   // L1 decode partial-sum chunks (H / 512)
// router_refine_warp (one warp per token) from this batch size up.  Its per-token latency is
// longer (one warp streams every candidate row of W_r) but it has no block barriers and no
// all-pairs ranking, so it wins once the batch fills the GPU several times over (C1 shapes:
// T = 2048 148 vs 179 us, T = 4096 276 vs 236 us, T = 8192 516 vs 378 us for the whole route).
constexpr int kRefineWarpMinT = 3072;

// Packed pairs of fp32 (sm_100 f32x2 arithmetic, round to nearest even in each lane).
__device__ __forceinline__ uint64_t f2_pack(float lo, float hi) {
    uint64_t d;
    asm("mov.b64 %0, {%1, %2};" : "=l"(d) : "f"(lo), "f"(hi));
    return d;
}
__device__ __forceinline__ void f2_unpack(uint64_t v, float &lo, float &hi) {
    asm("mov.b64 {%0, %1}, %2;" : "=f"(lo), "=f"(hi) : "l"(v));
}
__device__ __forceinline__ uint64_t f2_add(uint64_t a, uint64_t b) {
    uint64_t d;
    asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
    return d;
}
__device__ __forceinline__ uint64_t f2_sub(uint64_t a, uint64_t b) {
    uint64_t d;
    asm("sub.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
    return d;
}
__device__ __forceinline__ uint64_t f2_mul(uint64_t a, uint64_t b) {
    uint64_t d;
    asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
    return d;
}
__device__ __forceinline__ uint64_t f2_fma(uint64_t a, uint64_t b, uint64_t c) {
    uint64_t d;
    asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
    return d;
}

__device__ __forceinline__ void two_sum(float a, float b, float &s, float &t) {
    s = a + b;
    const float bb = s - a;
    t = (a - (s - bb)) + (b - bb);
}

__device__ __forceinline__ void ld_x4(const void *x, int x_dtype, int64_t off, float (&v)[4]) {
    if (x_dtype == VFMOE_DT_BF16) {
        const uint2 raw = *reinterpret_cast<const uint2 *>(reinterpret_cast<const __nv_bfloat16 *>(x) + off);
        v[0] = __uint_as_float(raw.x << 16);
        v[1] = __uint_as_float(raw.x & 0xFFFF0000u);
        v[2] = __uint_as_float(raw.y << 16);
        v[3] = __uint_as_float(raw.y & 0xFFFF0000u);
    } else {
        const float4 f = *reinterpret_cast<const float4 *>(reinterpret_cast<const float *>(x) + off);
        v[0] = f.x; v[1] = f.y; v[2] = f.z; v[3] = f.w;
    }
}

// Unsigned keys that order floats as their values (-0 below +0); the inverse.  Selection keys put
// the key in the high word and ~expert id in the low word: ties by value go to the lowest id.
__device__ __forceinline__ uint32_t f32_order_key(float f) {
    const uint32_t u = __float_as_uint(f);
    return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}
__device__ __forceinline__ float f32_from_order_key(uint32_t key) {
    return __uint_as_float((key & 0x80000000u) ? (key & 0x7FFFFFFFu) : ~key);
}

// ----------------------------------------------------------------------------- L1, decode
// T <= 32: CTA = 16 experts x one K chunk of KCH (768 or 512) x TB tokens (grid z: token groups
// t0 = TB z, so each thread keeps 2 x TB accumulators and several CTAs fit an SM); x[t0..t0+TB)
// [chunk] is staged in shared memory as fp32, each thread issues all of its W loads before any
// FMA.  Lane l owns k = 4l + 128j + i of the chunk.  Per-chunk partials part[chunk][t][e] are
// summed in chunk order by router_refine.  Summation depth: KCH/32 sequential FMAs + 5 (warp
// tree) + nchunk.  CTA (0, 0, 0) also zeroes zero[0..nzero) (the per-expert counts that the
// refinement accumulates), in place of a memset before the launch.
template <int TB, int KCH>
__global__ void __launch_bounds__(256) router_logits_f32_small(const void *__restrict__ x, int x_dtype,
                                                               const float *__restrict__ wr, int T_all, int H, int E,
                                                               float *__restrict__ part, int32_t *__restrict__ zero,
                                                               int nzero) {
    pdl_wait_then_release();
    if (zero && (blockIdx.x | blockIdx.y | blockIdx.z) == 0)
        for (int i = threadIdx.x; i < nzero; i += 256) zero[i] = 0;
    int T = T_all;
    extern __shared__ float xs[];  // [TB][KCH]
    constexpr int J = KCH / 128;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int kc = blockIdx.y, k0 = kc * KCH;
    const int t0 = blockIdx.z * TB;
    x = x_dtype == VFMOE_DT_BF16 ? (const void *)(reinterpret_cast<const __nv_bfloat16 *>(x) + (int64_t)t0 * H)
                                 : (const void *)(reinterpret_cast<const float *>(x) + (int64_t)t0 * H);
    T = min(T - t0, TB);  // tokens of this group; rows below are relative to t0
    // stage x[0..T)[chunk] as fp32: all loads of a thread are issued before any store
    {
        constexpr int PER = (TB * KCH / 8 + 255) / 256;  // 8-element groups per thread
        uint4 raw[PER];
        float4 rawf[2 * PER];
#pragma unroll
        for (int i = 0; i < PER; ++i) {
            const int gi = (threadIdx.x + 256 * i) * 8;
            const int t = gi / KCH, kk = gi % KCH;
            if (t < T) {
                if (x_dtype == VFMOE_DT_BF16) {
                    raw[i] = *reinterpret_cast<const uint4 *>(reinterpret_cast<const __nv_bfloat16 *>(x) + (int64_t)t * H + k0 + kk);
                } else {
                    const float4 *src = reinterpret_cast<const float4 *>(reinterpret_cast<const float *>(x) + (int64_t)t * H + k0 + kk);
                    rawf[2 * i] = src[0];
                    rawf[2 * i + 1] = src[1];
                }
            }
        }
#pragma unroll
        for (int i = 0; i < PER; ++i) {
            const int gi = (threadIdx.x + 256 * i) * 8;
            if (gi / KCH < T) {
                float4 a, b;
                if (x_dtype == VFMOE_DT_BF16) {
                    a = make_float4(__uint_as_float(raw[i].x << 16), __uint_as_float(raw[i].x & 0xFFFF0000u),
                                    __uint_as_float(raw[i].y << 16), __uint_as_float(raw[i].y & 0xFFFF0000u));
                    b = make_float4(__uint_as_float(raw[i].z << 16), __uint_as_float(raw[i].z & 0xFFFF0000u),
                                    __uint_as_float(raw[i].w << 16), __uint_as_float(raw[i].w & 0xFFFF0000u));
                } else {
                    a = rawf[2 * i];
                    b = rawf[2 * i + 1];
                }
                *reinterpret_cast<float4 *>(xs + gi) = a;
                *reinterpret_cast<float4 *>(xs + gi + 4) = b;
            }
        }
    }
    const int e0 = blockIdx.x * 16 + warp * 2;
    float4 w4[2][J];
#pragma unroll
    for (int a = 0; a < 2; ++a)
#pragma unroll
        for (int j = 0; j < J; ++j)
            w4[a][j] = (e0 + a < E) ? *reinterpret_cast<const float4 *>(wr + (int64_t)(e0 + a) * H + k0 + 4 * lane + 128 * j)
                                    : make_float4(0.f, 0.f, 0.f, 0.f);
    __syncthreads();
    float acc[2][TB];
#pragma unroll
    for (int a = 0; a < 2; ++a)
#pragma unroll
        for (int t = 0; t < TB; ++t) acc[a][t] = 0.f;
#pragma unroll
    for (int j = 0; j < J; ++j) {
#pragma unroll
        for (int t = 0; t < TB; ++t) {
            if (t < T) {
                const float4 xv = *reinterpret_cast<const float4 *>(xs + t * KCH + 4 * lane + 128 * j);
#pragma unroll
                for (int a = 0; a < 2; ++a) {
                    float v = acc[a][t];
                    v = fmaf(xv.x, w4[a][j].x, v);
                    v = fmaf(xv.y, w4[a][j].y, v);
                    v = fmaf(xv.z, w4[a][j].z, v);
                    v = fmaf(xv.w, w4[a][j].w, v);
                    acc[a][t] = v;
                }
            }
        }
    }
#pragma unroll
    for (int a = 0; a < 2; ++a)
#pragma unroll
        for (int t = 0; t < TB; ++t) {
            if (t < T) {
                const float v = warp_sum_f32(acc[a][t]);
                if (lane == 0 && e0 + a < E) part[((int64_t)kc * T_all + t0 + t) * E + e0 + a] = v;
            }
        }
}

// ----------------------------------------------------------------------------- L1, prefill
// 128 tokens x 128 experts per CTA, 256 threads x (8 tokens x 8 experts), K in chunks of 16
// staged k-major in a double-buffered shared-memory tile (one barrier per chunk; the next
// chunk is loaded into registers while the current one is consumed): 4 float4 reads per 64
// FMAs.  Each chunk is summed on its own and then added to the running total, so the
// summation depth is 16 + HS/16 over the CTA's K slice of HS = H / gridDim.z.  Slice z
// writes partial logits to logits + z*T*E, added in slice order by router_refine.
__global__ void __launch_bounds__(256, 1) router_logits_f32_wide(const void *__restrict__ x, int x_dtype,
                                                                 const float *__restrict__ wr, int T, int H, int E,
                                                                 float *__restrict__ logits) {
    constexpr int BT = 128, BE = 128, KC = 16;
    __shared__ __align__(16) float xs[2][KC][BT];
    __shared__ __align__(16) float ws[2][KC][BE];
    const int t0 = blockIdx.y * BT, e0 = blockIdx.x * BE;
    const int tid = threadIdx.x;
    const int tx = tid & 15, ty = tid >> 4;  // experts e0 + 4tx.., e0 + 64 + 4tx..; tokens t0 + 8ty ..
    const int HS = H / gridDim.z, k0 = blockIdx.z * HS;
    logits += (int64_t)blockIdx.z * T * E;
    const int lrow = tid >> 1, lkq = (tid & 1) * 8;  // loader: one row of the x or W tile, 8 k
    float xr[8], wv[8];
    auto load = [&](int kb) {
        const int t = t0 + lrow;
        if (t < T) {
            if (x_dtype == VFMOE_DT_BF16) {
                const uint4 u = *reinterpret_cast<const uint4 *>(reinterpret_cast<const __nv_bfloat16 *>(x) +
                                                                 (int64_t)t * H + kb + lkq);
                const uint32_t uu[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    xr[2 * i] = __uint_as_float(uu[i] << 16);
                    xr[2 * i + 1] = __uint_as_float(uu[i] & 0xFFFF0000u);
                }
            } else {
                const float4 *src =
                    reinterpret_cast<const float4 *>(reinterpret_cast<const float *>(x) + (int64_t)t * H + kb + lkq);
                const float4 a = src[0], b = src[1];
                xr[0] = a.x; xr[1] = a.y; xr[2] = a.z; xr[3] = a.w;
                xr[4] = b.x; xr[5] = b.y; xr[6] = b.z; xr[7] = b.w;
            }
        } else {
#pragma unroll
            for (int i = 0; i < 8; ++i) xr[i] = 0.f;
        }
        const int e = e0 + lrow;
        if (e < E) {
            const float4 *src = reinterpret_cast<const float4 *>(wr + (int64_t)e * H + kb + lkq);
            const float4 a = src[0], b = src[1];
            wv[0] = a.x; wv[1] = a.y; wv[2] = a.z; wv[3] = a.w;
            wv[4] = b.x; wv[5] = b.y; wv[6] = b.z; wv[7] = b.w;
        } else {
#pragma unroll
            for (int i = 0; i < 8; ++i) wv[i] = 0.f;
        }
    };
    auto store = [&](int buf) {
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            xs[buf][lkq + i][lrow] = xr[i];
            ws[buf][lkq + i][lrow] = wv[i];
        }
    };
    float acc[8][8];
#pragma unroll
    for (int i = 0; i < 8; ++i)
#pragma unroll
        for (int j = 0; j < 8; ++j) acc[i][j] = 0.f;
    load(k0);
    store(0);
    __syncthreads();
    const int nch = HS / KC;
    for (int c = 0; c < nch; ++c) {
        const int buf = c & 1;
        const bool more = c + 1 < nch;
        if (more) load(k0 + (c + 1) * KC);
        float part[8][8];
#pragma unroll
        for (int i = 0; i < 8; ++i)
#pragma unroll
            for (int j = 0; j < 8; ++j) part[i][j] = 0.f;
#pragma unroll
        for (int kk = 0; kk < KC; ++kk) {
            const float4 xa = *reinterpret_cast<const float4 *>(&xs[buf][kk][8 * ty]);
            const float4 xb = *reinterpret_cast<const float4 *>(&xs[buf][kk][8 * ty + 4]);
            const float4 wa = *reinterpret_cast<const float4 *>(&ws[buf][kk][4 * tx]);
            const float4 wb = *reinterpret_cast<const float4 *>(&ws[buf][kk][64 + 4 * tx]);
            const float xv[8] = {xa.x, xa.y, xa.z, xa.w, xb.x, xb.y, xb.z, xb.w};
            const float wc[8] = {wa.x, wa.y, wa.z, wa.w, wb.x, wb.y, wb.z, wb.w};
#pragma unroll
            for (int i = 0; i < 8; ++i)
#pragma unroll
                for (int j = 0; j < 8; ++j) part[i][j] = fmaf(xv[i], wc[j], part[i][j]);
        }
#pragma unroll
        for (int i = 0; i < 8; ++i)
#pragma unroll
            for (int j = 0; j < 8; ++j) acc[i][j] += part[i][j];
        if (more) store(buf ^ 1);
        __syncthreads();
    }
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        const int t = t0 + 8 * ty + i;
        if (t >= T) continue;
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            const int e = e0 + 64 * h + 4 * tx;
            float *dst = logits + (int64_t)t * E + e;
            if (e + 3 < E && (E & 3) == 0) {
                *reinterpret_cast<float4 *>(dst) =
                    make_float4(acc[i][4 * h], acc[i][4 * h + 1], acc[i][4 * h + 2], acc[i][4 * h + 3]);
            } else {
#pragma unroll
                for (int j = 0; j < 4; ++j)
                    if (e + j < E) dst[j] = acc[i][4 * h + j];
            }
        }
    }
}

// ----------------------------------------------------------------------------- |w_e|_2
__global__ void __launch_bounds__(256) row_norms_kernel(const float *__restrict__ wr, int H, int E,
                                                        float *__restrict__ nw) {
    const int e = blockIdx.x * 8 + (threadIdx.x >> 5), lane = threadIdx.x & 31;
    if (e >= E) return;
    double s = 0.0;
    for (int k = lane; k < H; k += 32) {
        const double v = wr[(int64_t)e * H + k];
        s = fma(v, v, s);
    }
    s = warp_sum_f64(s);
    if (lane == 0) nw[e] = (float)(sqrt(s) * (1.0 + 1e-6));  // rounded up: an upper bound
}

// ----------------------------------------------------------------------------- L2 + L3
// One CTA (256 threads) per token.  NPL = experts per lane (E <= 32 * NPL).
template <int NPL, int CPP, int MINB>
__global__ void __launch_bounds__(256, MINB) router_refine(const void *__restrict__ x, int x_dtype,
                                                     const float *__restrict__ wr, const float *__restrict__ logits,
                                                     int nchunk,
                                                     const float *__restrict__ nw, const float *__restrict__ bias,
                                                     int T, int H, int E, int k, float c1, float c2, double scale,
                                                     int32_t *__restrict__ idx_out, float *__restrict__ w_out,
                                                     int32_t *__restrict__ counts, int *__restrict__ err) {
    extern __shared__ float s_x[];  // [H] fp32 copy of x_t
    __shared__ float s_red[8];
    __shared__ int s_cand[kMaxCand];
    __shared__ double s_logit[kMaxCand];   // L2/L3 logit, then the choice (score + bias)
    __shared__ double s_score[kMaxCand];   // sigmoid(logit)
    __shared__ int s_ncand, s_amb;
    __shared__ uint64_t s_keys[8 * 32];             // every warp's k largest keys (orderable lo, ~id)
    __shared__ float s_tau;
    __shared__ int s_wcnt[8];
    __shared__ int s_order[kMaxCand];
    __shared__ unsigned char s_redo[kMaxCand];
    __shared__ float s_phi[8][8], s_plo[8][8];
    __shared__ double s_pd[8][8];
    const int t = blockIdx.x;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

    // x_t -> shared memory as fp32 (16-byte loads, issued four at a time) and |x_t|_2 (upper bound).
    // This runs before the wait on the first level: x comes from a kernel before that one, which
    // released this launch only after its own wait on x's producer (pdl_wait_then_release), or
    // ran to completion first.
    float ss = 0.f;
    if (x_dtype == VFMOE_DT_BF16) {
        for (int i0 = 0; i0 < kMaxH / 2048; i0 += 4) {
            uint4 u[4];
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const int h = (threadIdx.x + 256 * (i0 + i)) * 8;
                if (h < H) u[i] = *reinterpret_cast<const uint4 *>(reinterpret_cast<const __nv_bfloat16 *>(x) + (int64_t)t * H + h);
            }
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const int h = (threadIdx.x + 256 * (i0 + i)) * 8;
                if (h < H) {
                    const float4 a = make_float4(__uint_as_float(u[i].x << 16), __uint_as_float(u[i].x & 0xFFFF0000u),
                                                 __uint_as_float(u[i].y << 16), __uint_as_float(u[i].y & 0xFFFF0000u));
                    const float4 b = make_float4(__uint_as_float(u[i].z << 16), __uint_as_float(u[i].z & 0xFFFF0000u),
                                                 __uint_as_float(u[i].w << 16), __uint_as_float(u[i].w & 0xFFFF0000u));
                    *reinterpret_cast<float4 *>(s_x + h) = a;
                    *reinterpret_cast<float4 *>(s_x + h + 4) = b;
                    ss = fmaf(a.x, a.x, fmaf(a.y, a.y, fmaf(a.z, a.z, fmaf(a.w, a.w, ss))));
                    ss = fmaf(b.x, b.x, fmaf(b.y, b.y, fmaf(b.z, b.z, fmaf(b.w, b.w, ss))));
                }
            }
        }
    } else {
        for (int i0 = 0; i0 < kMaxH / 1024; i0 += 4) {
            float4 f[4];
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const int h = (threadIdx.x + 256 * (i0 + i)) * 4;
                if (h < H) f[i] = *reinterpret_cast<const float4 *>(reinterpret_cast<const float *>(x) + (int64_t)t * H + h);
            }
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const int h = (threadIdx.x + 256 * (i0 + i)) * 4;
                if (h < H) {
                    *reinterpret_cast<float4 *>(s_x + h) = f[i];
                    ss = fmaf(f[i].x, f[i].x, fmaf(f[i].y, f[i].y, fmaf(f[i].z, f[i].z, fmaf(f[i].w, f[i].w, ss))));
                }
            }
        }
    }
    ss = warp_sum_f32(ss);
    if (lane == 0) s_red[warp] = ss;
    __syncthreads();
    float tot = 0.f;
#pragma unroll
    for (int i = 0; i < 8; ++i) tot += s_red[i];
    const float nx = sqrtf(tot) * 1.001f;
    pdl_wait_then_release();  // the first level's partial logits and the zeroed counts

    // ---- L2 candidate selection, all threads: thread i owns experts i, i + 256, ...
    // lo/hi = choice -/+ the L1 bound.  tau = the k-th largest lo in the order (lo desc, id
    // asc): every warp finds its k largest 64-bit keys (orderable lo, ~id) in k rounds of a
    // warp-wide max, and warp 0 takes the k-th largest of those 8 k keys.  Candidates = experts
    // with hi >= tau, compacted in ascending id order.  All partial loads of a thread are issued
    // before they are summed.
    constexpr int EPT = (32 * NPL + 255) / 256;  // experts per thread
    float lo[EPT], hi[EPT];
#pragma unroll
    for (int i = 0; i < EPT; ++i) {
        const int e = threadIdx.x + 256 * i;
        lo[i] = hi[i] = -INFINITY;
        if (e < E) {
            float l = 0.f;
            for (int c0 = 0; c0 < nchunk; c0 += 8) {  // 8 partial loads in flight, summed in chunk order
                float pv[8];
#pragma unroll
                for (int c = 0; c < 8; ++c) pv[c] = c0 + c < nchunk ? logits[((int64_t)(c0 + c) * T + t) * E + e] : 0.f;
#pragma unroll
                for (int c = 0; c < 8; ++c)
                    if (c0 + c < nchunk) l += pv[c];
            }
            const float b1 = 0.25f * c1 * nx * nw[e] + 4e-6f;  // sigmoid slope <= 1/4; fp32 sigmoid + bias slack
            float ca = 1.f / (1.f + expf(-l)) + bias[e];
            if (isnan(ca)) ca = -INFINITY;
            lo[i] = ca - b1;
            hi[i] = ca + b1;
        }
    }
    {
        uint64_t key[EPT];
        bool bad = false;
#pragma unroll
        for (int i = 0; i < EPT; ++i) {
            const int e = threadIdx.x + 256 * i;
            key[i] = 0ull;  // below every real expert's key
            if (e < E) {
                key[i] = ((uint64_t)f32_order_key(lo[i]) << 32) | (uint64_t)(~(uint32_t)e);
                bad |= isnan(lo[i]);
            }
        }
        for (int r = 0; r < k; ++r) {
            uint64_t m = 0ull;
#pragma unroll
            for (int i = 0; i < EPT; ++i) m = key[i] > m ? key[i] : m;
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) {
                const uint64_t v = __shfl_xor_sync(0xffffffffu, m, o);
                m = v > m ? v : m;
            }
#pragma unroll
            for (int i = 0; i < EPT; ++i)
                if (m != 0ull && key[i] == m) key[i] = 0ull;
            if (lane == 0) s_keys[warp * 32 + r] = m;
        }
        const int nbad = __syncthreads_count(bad);
        if (warp == 0) {
            // the k-th largest of the 8 warps' k keys each (lane l holds keys l, l + 32, ...)
            uint64_t kk[8];
#pragma unroll
            for (int i = 0; i < 8; ++i) {
                const int w2 = i, r = lane;
                kk[i] = r < k ? s_keys[w2 * 32 + r] : 0ull;
            }
            uint64_t kth = 0ull;
            for (int r = 0; r < k; ++r) {
                uint64_t m = 0ull;
#pragma unroll
                for (int i = 0; i < 8; ++i) m = kk[i] > m ? kk[i] : m;
#pragma unroll
                for (int o = 16; o > 0; o >>= 1) {
                    const uint64_t v = __shfl_xor_sync(0xffffffffu, m, o);
                    m = v > m ? v : m;
                }
#pragma unroll
                for (int i = 0; i < 8; ++i)
                    if (m != 0ull && kk[i] == m) kk[i] = 0ull;
                kth = m;
            }
            if (lane == 0) {
                s_amb = 0;
                // no k-th expert, or a NaN bound somewhere: every expert is a candidate
                s_tau = (kth == 0ull || nbad) ? -INFINITY : f32_from_order_key((uint32_t)(kth >> 32));
            }
        }
    }
    __syncthreads();
    const float tau = s_tau;
    int nbase = 0;
#pragma unroll
    for (int i = 0; i < EPT; ++i) {
        const int e = threadIdx.x + 256 * i;
        const bool c = e < E && hi[i] >= tau;
        const unsigned m = __ballot_sync(0xffffffffu, c);
        if (lane == 0) s_wcnt[warp] = __popc(m);
        __syncthreads();
        int before = nbase, total = 0;
#pragma unroll
        for (int w = 0; w < 8; ++w) {
            before += w < warp ? s_wcnt[w] : 0;
            total += s_wcnt[w];
        }
        if (c) {
            const int pos = before + __popc(m & ((1u << lane) - 1u));
            if (pos < kMaxCand) s_cand[pos] = e;
        }
        nbase += total;
        __syncthreads();
    }
    if (threadIdx.x == 0) {
        int n = nbase;
        if (n > kMaxCand) {
            raise_dev_error(err, DEV_BAD_COUNT);
            n = kMaxCand;
        }
        s_ncand = n;
    }
    __syncthreads();
    const int nc = s_ncand;

    // ---- L2 float-float logits of the candidates: thread owns k = 4*tid + 1024*j + i,
    // 8 candidates per pass (all loads of a pass are independent); then a fixed-order
    // TwoSum tree over lanes and warps.
    for (int c0 = 0; c0 < nc; c0 += CPP) {
        float shi[CPP], slo[CPP];
#pragma unroll
        for (int c = 0; c < CPP; ++c) shi[c] = slo[c] = 0.f;
        int ec[CPP];
#pragma unroll
        for (int c = 0; c < CPP; ++c) ec[c] = (c0 + c < nc) ? s_cand[c0 + c] : -1;
        for (int hb = 0; hb < H; hb += 3072) {          // 3 float4 per candidate per batch
            float4 w4[CPP][3];
#pragma unroll
            for (int c = 0; c < CPP; ++c)
#pragma unroll
                for (int j = 0; j < 3; ++j) {
                    const int h = hb + threadIdx.x * 4 + 1024 * j;
                    w4[c][j] = (ec[c] >= 0 && h < H) ? *reinterpret_cast<const float4 *>(wr + (int64_t)ec[c] * H + h)
                                                     : make_float4(0.f, 0.f, 0.f, 0.f);
                }
#pragma unroll
            for (int j = 0; j < 3; ++j) {
                const int h = hb + threadIdx.x * 4 + 1024 * j;
                if (h >= H) break;
                const float4 x4 = *reinterpret_cast<const float4 *>(s_x + h);
                const float xv[4] = {x4.x, x4.y, x4.z, x4.w};
                // two candidates per instruction (packed f32x2, each lane an IEEE fp32 op):
                // the same operations in the same order as the scalar TwoProduct / TwoSum
#pragma unroll
                for (int c = 0; c < CPP; c += 2) {
                    const float wa[4] = {w4[c][j].x, w4[c][j].y, w4[c][j].z, w4[c][j].w};
                    const float wb[4] = {w4[c + 1][j].x, w4[c + 1][j].y, w4[c + 1][j].z, w4[c + 1][j].w};
                    uint64_t sh = f2_pack(shi[c], shi[c + 1]), sl = f2_pack(slo[c], slo[c + 1]);
#pragma unroll
                    for (int i = 0; i < 4; ++i) {
                        const uint64_t x2 = f2_pack(xv[i], xv[i]), w2 = f2_pack(wa[i], wb[i]);
                        const uint64_t pp = f2_mul(x2, w2);
                        const uint64_t pe = f2_fma(x2, w2, pp ^ 0x8000000080000000ull);  // exact: x*w = p + pe
                        const uint64_t sum = f2_add(sh, pp);
                        const uint64_t bb = f2_sub(sum, sh);
                        const uint64_t r = f2_add(f2_sub(sh, f2_sub(sum, bb)), f2_sub(pp, bb));
                        sh = sum;
                        sl = f2_add(sl, f2_add(r, pe));
                    }
                    f2_unpack(sh, shi[c], shi[c + 1]);
                    f2_unpack(sl, slo[c], slo[c + 1]);
                }
            }
        }
#pragma unroll
        for (int c = 0; c < CPP; ++c) {
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) {
                const float oh = __shfl_xor_sync(0xffffffffu, shi[c], o);
                const float ol = __shfl_xor_sync(0xffffffffu, slo[c], o);
                float sum, r;
                two_sum(shi[c], oh, sum, r);
                shi[c] = sum;
                slo[c] = slo[c] + ol + r;
            }
            if (lane == 0) {
                s_phi[warp][c] = shi[c];
                s_plo[warp][c] = slo[c];
            }
        }
        __syncthreads();
        if (threadIdx.x < CPP && c0 + threadIdx.x < nc) {
            const int c = threadIdx.x;
            float hi = s_phi[0][c], lo = s_plo[0][c];
            for (int w = 1; w < 8; ++w) {
                float sum, r;
                two_sum(hi, s_phi[w][c], sum, r);
                hi = sum;
                lo = lo + s_plo[w][c] + r;
            }
            s_logit[c0 + c] = (double)hi + (double)lo;
        }
        __syncthreads();
    }

    // ---- order candidates in f64; flag neighbours closer than the L2 bound (warp 0)
    if (warp == 0) {
        // rank of candidate c = #candidates strictly better (choice desc, id asc)
        for (int c = lane; c < nc; c += 32) {
            const int e = s_cand[c];
            const double sc = 1.0 / (1.0 + exp(-s_logit[c]));
            s_score[c] = sc;
            s_logit[c] = sc + (double)bias[e];  // reuse: now the choice
            s_order[c] = -1;                    // stays -1 where NaN choices collide in rank
        }
        __syncwarp();
        for (int c = lane; c < nc; c += 32) {
            const double ch = s_logit[c];
            const int e = s_cand[c];
            int rank = 0;
            for (int o = 0; o < nc; ++o) {
                const double oc = s_logit[o];
                rank += (oc > ch || (oc == ch && s_cand[o] < e)) ? 1 : 0;
            }
            s_order[rank] = c;
            s_redo[c] = 0;
        }
        __syncwarp();
        for (int r = lane; r < k && r + 1 < nc; r += 32) {
            const int a = s_order[r], b = s_order[r + 1];
            if (a < 0 || b < 0) continue;
            const double ba = 0.25 * (double)c2 * nx * nw[s_cand[a]], bb = 0.25 * (double)c2 * nx * nw[s_cand[b]];
            if (s_logit[a] - s_logit[b] <= 2.0 * (ba + bb) + 1e-15) {
                s_redo[a] = 1;
                s_redo[b] = 1;
                s_amb = 1;
            }
        }
    }
    __syncthreads();

    // ---- L3: fp64 logits for ambiguous neighbours (rare); same decomposition as L2
    if (s_amb) {
        for (int c0 = 0; c0 < nc; c0 += 8) {
            double acc[8];
#pragma unroll
            for (int c = 0; c < 8; ++c) acc[c] = 0.0;
            for (int h = threadIdx.x * 4; h < H; h += 1024) {
                const float4 x4 = *reinterpret_cast<const float4 *>(s_x + h);
                const float xv[4] = {x4.x, x4.y, x4.z, x4.w};
#pragma unroll
                for (int c = 0; c < 8; ++c) {
                    if (c0 + c < nc && s_redo[c0 + c]) {
                        const float4 w4 = *reinterpret_cast<const float4 *>(wr + (int64_t)s_cand[c0 + c] * H + h);
                        acc[c] = fma((double)xv[0], (double)w4.x, acc[c]);
                        acc[c] = fma((double)xv[1], (double)w4.y, acc[c]);
                        acc[c] = fma((double)xv[2], (double)w4.z, acc[c]);
                        acc[c] = fma((double)xv[3], (double)w4.w, acc[c]);
                    }
                }
            }
#pragma unroll
            for (int c = 0; c < 8; ++c) {
                const double v = warp_sum_f64(acc[c]);
                if (lane == 0) s_pd[warp][c] = v;
            }
            __syncthreads();
            if (threadIdx.x < 8 && c0 + threadIdx.x < nc && s_redo[c0 + threadIdx.x]) {
                const int c = threadIdx.x;
                double v = 0.0;
                for (int w = 0; w < 8; ++w) v += s_pd[w][c];
                const int e = s_cand[c0 + c];
                const double sc = 1.0 / (1.0 + exp(-v));
                s_score[c0 + c] = sc;
                s_logit[c0 + c] = sc + (double)bias[e];
            }
            __syncthreads();
        }
        if (warp == 0) {
            for (int c = lane; c < nc; c += 32) {
                const double ch = s_logit[c];
                const int e = s_cand[c];
                int rank = 0;
                for (int o = 0; o < nc; ++o) {
                    const double oc = s_logit[o];
                    rank += (oc > ch || (oc == ch && s_cand[o] < e)) ? 1 : 0;
                }
                s_order[rank] = c;
            }
        }
        __syncthreads();
    }

    // ---- final top-k and weights (warp 0): scores = choice - bias, in f64
    if (warp == 0) {
        double sc = 0.0;
        int e = -1;
        if (lane < k && lane < nc) {
            const int c = s_order[lane];
            if (c >= 0) {
                e = s_cand[c];
                sc = s_score[c];
            }
        }
        double sum = 0.0;
        for (int r = 0; r < k; ++r) sum += __shfl_sync(0xffffffffu, sc, r);
        if (lane < k) {
            idx_out[(int64_t)t * k + lane] = e;
            w_out[(int64_t)t * k + lane] = (float)(sc / (sum + 1e-20) * scale);
            if (e >= 0 && e < E)
                atomicAdd(&counts[e], 1);
            else
                raise_dev_error(err, DEV_BAD_EXPERT_ID);
        }
    }
}

// ----------------------------------------------------------------------------- L2 + L3, one warp per token
// The same three levels as router_refine, for batches large enough to fill the GPU with one warp
// per token (four tokens per CTA), so that no step waits on a block barrier:
//   * tau, the k-th largest lower bound in the order (lo desc, id asc), is the k-th of k rounds
//     of a warp-wide max over 64-bit keys (orderable lo, ~id): about 40 instructions per lane and
//     round, where router_refine ranks every expert against every other;
//   * a candidate's float-float logit is accumulated by the 32 lanes over H (lane l holds
//     h = 4 l + 128 j, two candidates per packed f32x2 instruction) and reduced by a TwoSum
//     butterfly across the lanes;
//   * the f64 ordering, the f64 level for close neighbours and the weights run on the same warp.
// Lane l owns experts l, l + 32, ... (NPL of them, E <= 32 NPL).  Candidate lists, f64 logits and
// scores live in the warp's slice of shared memory.
constexpr int kRwWarps = 4;


template <int NPL>
__global__ void __launch_bounds__(32 * kRwWarps) router_refine_warp(
    const void *__restrict__ x, int x_dtype, const float *__restrict__ wr, const float *__restrict__ logits,
    int nchunk, const float *__restrict__ nw, const float *__restrict__ bias, int T, int H, int E, int k, float c1,
    float c2, double scale, int32_t *__restrict__ idx_out, float *__restrict__ w_out, int32_t *__restrict__ counts,
    int *__restrict__ err) {
    __shared__ int s_cand[kRwWarps][kMaxCand];
    __shared__ double s_logit[kRwWarps][kMaxCand];   // L2/L3 logit, then the choice (score + bias)
    __shared__ double s_score[kRwWarps][kMaxCand];   // sigmoid(logit)
    __shared__ int s_order[kRwWarps][kMaxCand];
    __shared__ unsigned char s_redo[kRwWarps][kMaxCand];
    pdl_wait_then_release();
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int t = blockIdx.x * kRwWarps + warp;
    if (t >= T) return;
    int *cand = s_cand[warp];
    double *lg = s_logit[warp];
    double *scr = s_score[warp];
    int *order = s_order[warp];
    unsigned char *redo = s_redo[warp];
    const int64_t xrow = (int64_t)t * H;

    // |x_t|_2, rounded up
    float ss = 0.f;
#pragma unroll 4
    for (int h = 4 * lane; h < H; h += 128) {
        float v[4];
        ld_x4(x, x_dtype, xrow + h, v);
        ss = fmaf(v[0], v[0], fmaf(v[1], v[1], fmaf(v[2], v[2], fmaf(v[3], v[3], ss))));
    }
    const float nx = sqrtf(warp_sum_f32(ss)) * 1.001f;

    // ---- L1 intervals [lo, hi] of every expert's choice, and tau
    float hi[NPL];
    uint64_t key[NPL];
    bool bad = false;
#pragma unroll
    for (int i = 0; i < NPL; ++i) {
        const int e = lane + 32 * i;
        hi[i] = -INFINITY;
        key[i] = 0ull;  // below every real expert's key
        if (e < E) {
            float l = 0.f;
#pragma unroll 4
            for (int c = 0; c < nchunk; ++c) l += logits[((int64_t)c * T + t) * E + e];  // chunk order
            const float b1 = 0.25f * c1 * nx * nw[e] + 4e-6f;  // sigmoid slope <= 1/4; fp32 sigmoid + bias slack
            float ca = 1.f / (1.f + expf(-l)) + bias[e];
            if (isnan(ca)) ca = -INFINITY;
            const float lo = ca - b1;
            hi[i] = ca + b1;
            bad |= isnan(lo);
            key[i] = ((uint64_t)f32_order_key(lo) << 32) | (uint64_t)(~(uint32_t)e);
        }
    }
    uint64_t kth = 0ull;
    for (int r = 0; r < k; ++r) {
        uint64_t m = 0ull;
#pragma unroll
        for (int i = 0; i < NPL; ++i) m = key[i] > m ? key[i] : m;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            const uint64_t v = __shfl_xor_sync(0xffffffffu, m, o);
            m = v > m ? v : m;
        }
#pragma unroll
        for (int i = 0; i < NPL; ++i)
            if (m != 0ull && key[i] == m) key[i] = 0ull;
        kth = m;
    }
    // no k-th expert, or a NaN bound somewhere: every expert is a candidate
    const float tau = (kth == 0ull || __any_sync(0xffffffffu, bad)) ? -INFINITY : f32_from_order_key((uint32_t)(kth >> 32));

    // ---- candidates (hi >= tau) in ascending id order
    int nc = 0;
#pragma unroll
    for (int i = 0; i < NPL; ++i) {
        const int e = lane + 32 * i;
        const bool c = e < E && hi[i] >= tau;
        const unsigned m = __ballot_sync(0xffffffffu, c);
        const int pos = nc + __popc(m & ((1u << lane) - 1u));
        if (c && pos < kMaxCand) cand[pos] = e;
        nc += __popc(m);
    }
    if (nc > kMaxCand) {
        if (lane == 0) raise_dev_error(err, DEV_BAD_COUNT);
        nc = kMaxCand;
    }
    __syncwarp();

    // ---- L2 float-float logits, two candidates at a time (a lone last candidate is paired with
    // itself and its second copy discarded)
    for (int c0 = 0; c0 < nc; c0 += 2) {
        const int ea = cand[c0];
        const int eb = c0 + 1 < nc ? cand[c0 + 1] : ea;
        const float *wa = wr + (int64_t)ea * H;
        const float *wb = wr + (int64_t)eb * H;
        uint64_t sh = 0ull, sl = 0ull;  // packed {candidate a, candidate b}
        for (int h0 = 4 * lane; h0 < H; h0 += 512) {
            float4 va[4], vb[4];
            float xv[4][4];
#pragma unroll
            for (int u = 0; u < 4; ++u) {
                const int h = h0 + 128 * u;
                if (h < H) {
                    va[u] = *reinterpret_cast<const float4 *>(wa + h);
                    vb[u] = *reinterpret_cast<const float4 *>(wb + h);
                    ld_x4(x, x_dtype, xrow + h, xv[u]);
                } else {
                    va[u] = vb[u] = make_float4(0.f, 0.f, 0.f, 0.f);
                    xv[u][0] = xv[u][1] = xv[u][2] = xv[u][3] = 0.f;
                }
            }
#pragma unroll
            for (int u = 0; u < 4; ++u) {
                const float a4[4] = {va[u].x, va[u].y, va[u].z, va[u].w};
                const float b4[4] = {vb[u].x, vb[u].y, vb[u].z, vb[u].w};
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    // TwoProduct (x*w = p + pe exactly) and TwoSum (sh + p = sum + r exactly), per lane of the pair
                    const uint64_t x2 = f2_pack(xv[u][i], xv[u][i]), w2 = f2_pack(a4[i], b4[i]);
                    const uint64_t pp = f2_mul(x2, w2);
                    const uint64_t pe = f2_fma(x2, w2, pp ^ 0x8000000080000000ull);
                    const uint64_t sum = f2_add(sh, pp);
                    const uint64_t bb = f2_sub(sum, sh);
                    const uint64_t r = f2_add(f2_sub(sh, f2_sub(sum, bb)), f2_sub(pp, bb));
                    sh = sum;
                    sl = f2_add(sl, f2_add(r, pe));
                }
            }
        }
        float ha, hb, la, lb;
        f2_unpack(sh, ha, hb);
        f2_unpack(sl, la, lb);
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            const float oha = __shfl_xor_sync(0xffffffffu, ha, o), ola = __shfl_xor_sync(0xffffffffu, la, o);
            const float ohb = __shfl_xor_sync(0xffffffffu, hb, o), olb = __shfl_xor_sync(0xffffffffu, lb, o);
            float s, r;
            two_sum(ha, oha, s, r);
            ha = s;
            la = la + ola + r;
            two_sum(hb, ohb, s, r);
            hb = s;
            lb = lb + olb + r;
        }
        if (lane == 0) {
            lg[c0] = (double)ha + (double)la;
            if (c0 + 1 < nc) lg[c0 + 1] = (double)hb + (double)lb;
        }
    }
    __syncwarp();

    // ---- order candidates in f64 (choice desc, id asc); flag neighbours closer than the L2 bound
    for (int c = lane; c < nc; c += 32) {
        const double sc = 1.0 / (1.0 + exp(-lg[c]));
        scr[c] = sc;
        lg[c] = sc + (double)bias[cand[c]];
    }
    for (int c = lane; c < nc; c += 32) order[c] = -1;  // stays -1 where NaN choices collide in rank
    __syncwarp();
    for (int c = lane; c < nc; c += 32) {
        const double ch = lg[c];
        const int e = cand[c];
        int rank = 0;
        for (int o = 0; o < nc; ++o) {
            const double oc = lg[o];
            rank += (oc > ch || (oc == ch && cand[o] < e)) ? 1 : 0;
        }
        order[rank] = c;
        redo[c] = 0;
    }
    __syncwarp();
    bool amb = false;
    for (int r = lane; r < k && r + 1 < nc; r += 32) {
        const int a = order[r], b = order[r + 1];
        if (a < 0 || b < 0) continue;
        const double ba = 0.25 * (double)c2 * nx * nw[cand[a]], bb = 0.25 * (double)c2 * nx * nw[cand[b]];
        if (lg[a] - lg[b] <= 2.0 * (ba + bb) + 1e-15) {
            redo[a] = 1;
            redo[b] = 1;
            amb = true;
        }
    }
    amb = __any_sync(0xffffffffu, amb);
    __syncwarp();

    // ---- L3: fp64 logits of the flagged candidates (rare), then reorder
    if (amb) {
        for (int c = 0; c < nc; ++c) {
            if (!redo[c]) continue;
            const float *wc = wr + (int64_t)cand[c] * H;
            double acc = 0.0;
            for (int h = 4 * lane; h < H; h += 128) {
                float v[4];
                ld_x4(x, x_dtype, xrow + h, v);
                const float4 w4 = *reinterpret_cast<const float4 *>(wc + h);
                acc = fma((double)v[0], (double)w4.x, acc);
                acc = fma((double)v[1], (double)w4.y, acc);
                acc = fma((double)v[2], (double)w4.z, acc);
                acc = fma((double)v[3], (double)w4.w, acc);
            }
            acc = warp_sum_f64(acc);
            if (lane == 0) {
                const double sc = 1.0 / (1.0 + exp(-acc));
                scr[c] = sc;
                lg[c] = sc + (double)bias[cand[c]];
            }
        }
        __syncwarp();
        for (int c = lane; c < nc; c += 32) {
            const double ch = lg[c];
            const int e = cand[c];
            int rank = 0;
            for (int o = 0; o < nc; ++o) {
                const double oc = lg[o];
                rank += (oc > ch || (oc == ch && cand[o] < e)) ? 1 : 0;
            }
            order[rank] = c;
        }
        __syncwarp();
    }

    // ---- top-k and weights: scores = choice - bias, in f64
    double sc = 0.0;
    int e = -1;
    if (lane < k && lane < nc) {
        const int c = order[lane];
        if (c >= 0) {
            e = cand[c];
            sc = scr[c];
        }
    }
    double sum = 0.0;
    for (int r = 0; r < k; ++r) sum += __shfl_sync(0xffffffffu, sc, r);
    if (lane < k) {
        idx_out[(int64_t)t * k + lane] = e;
        w_out[(int64_t)t * k + lane] = (float)(sc / (sum + 1e-20) * scale);
        if (e >= 0 && e < E)
            atomicAdd(&counts[e], 1);
        else
            raise_dev_error(err, DEV_BAD_EXPERT_ID);
    }
}

// Router summation-depth error constants (gamma_n with u = 2^-24, doubled for safety).
static float gamma_bound(int depth) { return 2.0f * (float)depth * 5.9604645e-8f / (1.0f - (float)depth * 5.96e-8f); }

int launch_router_norms(const float *wr, int H, int E, float *nw, cudaStream_t st) {
    row_norms_kernel<<<(unsigned)cdiv(E, 8), 256, 0, st>>>(wr, H, E, nw);
    VF_LAUNCH_CHECK("row_norms_kernel");
    return VFMOE_OK;
}

template <int TB, int KCH>
static int launch_l1_small(const void *x, int x_dtype, const float *wr, int T, int H, int E, float *part,
                           int32_t *zero, int nzero, cudaStream_t st) {
    const int smem = TB * KCH * 4;
    int rc = set_smem_attr_once(reinterpret_cast<const void *>(router_logits_f32_small<TB, KCH>), smem);
    if (rc) return rc;
    dim3 grid((unsigned)cdiv(E, 16), (unsigned)(H / KCH), (unsigned)cdiv(T, TB));
    VF_CUDA(launch_pdl(router_logits_f32_small<TB, KCH>, grid, dim3(256), (size_t)smem, st, x, x_dtype, wr, T, H, E,
                       part, zero, nzero));
    VF_LAUNCH_CHECK("router_logits_f32_small");
    return VFMOE_OK;
}

// K slices of the prefill logits kernel: enough CTAs (one per SM) for about two waves on
// 148 SMs, at most kMaxChunks, each slice a multiple of 16 columns of H.
static int tiled_splits(int T, int H, int E) {
    const int64_t base = cdiv(E, 128) * cdiv(T, 128);
    const int want = (int)std::min<int64_t>(kMaxChunks, cdiv(296, base));
    int s = 1;
    for (int c = 1; c <= want; ++c)
        if ((H / 16) % c == 0) s = c;
    return s;
}

// The decode logits kernel (T <= 32) takes H in chunks of 768 or 512 columns, one partial sum per
// chunk; 0 = H is a multiple of neither and the tiled kernel runs at every T.
static int router_l1_chunk(int H) { return H % 768 == 0 ? 768 : (H % 512 == 0 ? 512 : 0); }

// Partial-sum slices the logits kernel writes for (T, H, E): H / chunk on the decode kernel, else
// tiled_splits.  launch_router and the scratch sizing (router_logit_floats) both use this count.
static int router_splits(int T, int H, int E, bool tc) {
    if (tc && router_tc_shape(T, H, E)) return router_tc_splits(T, H, E);
    const int kch = router_l1_chunk(H);
    return (T <= 32 && kch) ? H / kch : tiled_splits(T, H, E);
}

int launch_router_l1(const void *x, int x_dtype, const float *wr, const __nv_bfloat16 *wr_split, int T, int H, int E,
                     float *logits, int *err, cudaStream_t st, int *nchunk_out, float *c1_out, int32_t *zero,
                     int nzero) {
    if (H > kMaxH || H / 512 > kMaxChunks) {
        set_error("router: hidden size %d exceeds %d", H, kMaxH);
        return VFMOE_ERR_UNSUPPORTED;
    }
    float c1;
    int rc = VFMOE_OK;
    const int kch = router_l1_chunk(H);
    const bool tc = wr_split && x_dtype == VFMOE_DT_BF16 && router_tc_shape(T, H, E) &&
                    (reinterpret_cast<uintptr_t>(x) & 15) == 0;
    const int nchunk = router_splits(T, H, E, tc);
    if (zero && !(T <= 32 && kch && !tc)) VF_CUDA(cudaMemsetAsync(zero, 0, (size_t)nzero * sizeof(int32_t), st));
    if (tc) {
        rc = launch_router_logits_tc(x, wr_split, T, H, E, logits, err, st);
        if (rc) return rc;
        c1 = router_tc_bound(H);
    } else if (T <= 32 && kch) {
        if (kch == 768)
            rc = launch_l1_small<8, 768>(x, x_dtype, wr, T, H, E, logits, zero, nzero, st);
        else
            rc = launch_l1_small<8, 512>(x, x_dtype, wr, T, H, E, logits, zero, nzero, st);
        if (rc) return rc;
        c1 = gamma_bound(kch / 32 + 5 + nchunk);
    } else {
        dim3 grid((unsigned)cdiv(E, 128), (unsigned)cdiv(T, 128), (unsigned)nchunk);
        router_logits_f32_wide<<<grid, 256, 0, st>>>(x, x_dtype, wr, T, H, E, logits);
        VF_LAUNCH_CHECK("router_logits_f32_wide");
        c1 = gamma_bound(16 + H / nchunk / 16 + nchunk);
    }
    *nchunk_out = nchunk;
    *c1_out = c1;
    return VFMOE_OK;
}

int launch_router(const void *x, int x_dtype, const float *wr, const __nv_bfloat16 *wr_split, const float *nw,
                  const float *bias, int T, int H, int E, int k, double scale, float *logits, int32_t *idx, float *w,
                  int32_t *counts, int *err, cudaStream_t st) {
    int nchunk = 1;
    float c1 = 0.f;
    int rc = launch_router_l1(x, x_dtype, wr, wr_split, T, H, E, logits, err, st, &nchunk, &c1, counts, E + 2);
    if (rc) return rc;
    // L2: thread owns n = H/256 terms.  hi + sum(r) = sum(p) exactly (TwoSum) and x*w = p + pe
    // exactly (TwoProduct), so the only error is lo's fp32 summation of the r and pe values,
    // sum(|r| + |pe|) <= (n + 1) u S:  |err| <= gamma_{2n} (n + 1) u S; the 5 + 7 level lane and
    // warp trees add terms of the same size (bounded with gamma_{2n+24}).  hi + lo is exact in f64.
    const int n2 = H / 256;
    const float c2 = gamma_bound(2 * n2 + 24) * (float)(n2 + 1 + 24) * 5.9604645e-8f;
    const int npl = (int)cdiv(E, 32);
    if (T >= kRefineWarpMinT && npl <= 16) {
        // One warp per token: a lane owns nl = 4 ceil(H / 128) terms; the 5-level lane butterfly adds
        // 31 TwoSum error terms (each <= u S) and 10 fp32 additions of depth to lo's summation:
        // |err| <= gamma_{2 nl + 10} (nl + 32) u S.
        const int nl = 4 * (int)cdiv(H, 128);
        const float c2w = gamma_bound(2 * nl + 10) * (float)(nl + 32) * 5.9604645e-8f;
        const dim3 grid((unsigned)cdiv(T, kRwWarps));
#define VF_REFINE_W(NPL)                                                                                           \
    VF_CUDA(launch_pdl(router_refine_warp<NPL>, grid, dim3(32 * kRwWarps), 0, st, x, x_dtype, wr, (const float *)logits, \
                       nchunk, nw, bias, T, H, E, k, c1, c2w, scale, idx, w, counts, err))
        if (npl <= 1) VF_REFINE_W(1);
        else if (npl <= 2) VF_REFINE_W(2);
        else if (npl <= 4) VF_REFINE_W(4);
        else if (npl <= 8) VF_REFINE_W(8);
        else VF_REFINE_W(16);
#undef VF_REFINE_W
        VF_LAUNCH_CHECK("router_refine_warp");
        return VFMOE_OK;
    }
    if (H * 4 > 48 * 1024) {
        if ((rc = set_smem_attr_once(reinterpret_cast<const void *>(router_refine<1, 8, 1>), kMaxH * 4))) return rc;
        if ((rc = set_smem_attr_once(reinterpret_cast<const void *>(router_refine<1, 4, 3>), kMaxH * 4))) return rc;
        if ((rc = set_smem_attr_once(reinterpret_cast<const void *>(router_refine<2, 8, 1>), kMaxH * 4))) return rc;
        if ((rc = set_smem_attr_once(reinterpret_cast<const void *>(router_refine<2, 4, 3>), kMaxH * 4))) return rc;
        if ((rc = set_smem_attr_once(reinterpret_cast<const void *>(router_refine<4, 8, 1>), kMaxH * 4))) return rc;
        if ((rc = set_smem_attr_once(reinterpret_cast<const void *>(router_refine<4, 4, 3>), kMaxH * 4))) return rc;
        if ((rc = set_smem_attr_once(reinterpret_cast<const void *>(router_refine<8, 8, 1>), kMaxH * 4))) return rc;
        if ((rc = set_smem_attr_once(reinterpret_cast<const void *>(router_refine<8, 4, 3>), kMaxH * 4))) return rc;
        if ((rc = set_smem_attr_once(reinterpret_cast<const void *>(router_refine<16, 8, 1>), kMaxH * 4))) return rc;
        if ((rc = set_smem_attr_once(reinterpret_cast<const void *>(router_refine<16, 4, 3>), kMaxH * 4))) return rc;
        if ((rc = set_smem_attr_once(reinterpret_cast<const void *>(router_refine<32, 8, 1>), kMaxH * 4))) return rc;
        if ((rc = set_smem_attr_once(reinterpret_cast<const void *>(router_refine<32, 4, 3>), kMaxH * 4))) return rc;
    }
#define VF_REFINE(NPL)                                                                                              \
    do {                                                                                                           \
        if (T <= 64)                                                                                               \
            VF_CUDA(launch_pdl(router_refine<NPL, 8, 1>, dim3((unsigned)T), dim3(256), (size_t)H * 4, st, x, x_dtype, \
                               wr, (const float *)logits, nchunk, nw, bias, T, H, E, k, c1, c2, scale, idx, w, counts, \
                               err));                                                                              \
        else                                                                                                       \
            VF_CUDA(launch_pdl(router_refine<NPL, 4, 3>, dim3((unsigned)T), dim3(256), (size_t)H * 4, st, x, x_dtype, \
                               wr, (const float *)logits, nchunk, nw, bias, T, H, E, k, c1, c2, scale, idx, w, counts, \
                               err));                                                                              \
    } while (0)
    if (npl <= 1) VF_REFINE(1);
    else if (npl <= 2) VF_REFINE(2);
    else if (npl <= 4) VF_REFINE(4);
    else if (npl <= 8) VF_REFINE(8);
    else if (npl <= 16) VF_REFINE(16);
    else VF_REFINE(32);
#undef VF_REFINE
    VF_LAUNCH_CHECK("router_refine");
    return VFMOE_OK;
}

// out[i] = sum over c < nchunk of part[c * n + i], in chunk order (as router_refine sums them).
__global__ void sum_partials_kernel(const float *__restrict__ part, int nchunk, int64_t n, float *__restrict__ out) {
    const int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
    if (i >= n) return;
    float s = 0.f;
    for (int c = 0; c < nchunk; ++c) s += part[c * n + i];
    out[i] = s;
}

int launch_route_logits(const void *x, int x_dtype, const float *wr, const __nv_bfloat16 *wr_split, int T, int H,
                        int E, float *part, float *out, int *err, cudaStream_t st, float *c1) {
    int nchunk = 1;
    int rc = launch_router_l1(x, x_dtype, wr, wr_split, T, H, E, part, err, st, &nchunk, c1, nullptr, 0);
    if (rc) return rc;
    const int64_t n = (int64_t)T * E;
    sum_partials_kernel<<<(unsigned)cdiv(n, 256), 256, 0, st>>>(part, nchunk, n, out);
    VF_LAUNCH_CHECK("sum_partials_kernel");
    return VFMOE_OK;
}

int64_t router_logit_floats(int T, int H, int E, bool tc) {
    return (int64_t)T * E * std::max(router_splits(T, H, E, tc), router_splits(T, H, E, false));
}

}  // namespace vfmoe
