// Plain-SIMT expert FFN kernels: the simple, obviously-correct CUDA path that the
// tensor-core kernels are checked against on the GPU.  Same numerics as the
// tensor-core path: each Q8_0 weight becomes fp16(d * q) (one rounding), activations
// are fp16, products are exact in fp32, accumulation is fp32.
//
//   gate_up_simt: act[pos, r] = fp16(swiglu(x_pos . Wg[r], x_pos . Wu[r]))   (moe.vyb:98-134)
//   down_simt:    y[pos, r]   = act_pos . Wd[r]  (fp32)                      (moe.vyb:137-170)
// One warp per weight row, lanes over Q8_0 blocks, up to 8 tokens per pass.
#include "common.cuh"
#include "kernels.h"

namespace vfmoe {

__device__ __forceinline__ void q8_block_fp16(const uint8_t *blk, float w[32]) {
    const float d = q8_scale(blk);
    const uint16_t *q2 = reinterpret_cast<const uint16_t *>(blk + 2);
#pragma unroll
    for (int i = 0; i < 16; ++i) {
        const uint16_t v = q2[i];
        const float q0 = (float)(int8_t)(v & 0xFF), q1 = (float)(int8_t)(v >> 8);
        w[2 * i] = __half2float(__float2half_rn(d * q0));
        w[2 * i + 1] = __half2float(__float2half_rn(d * q1));
    }
}

__device__ __forceinline__ void ld_x32(const __half *p, float x[32]) {
#pragma unroll
    for (int c = 0; c < 4; ++c) {
        const uint4 raw = reinterpret_cast<const uint4 *>(p)[c];
        const __half2 *h = reinterpret_cast<const __half2 *>(&raw);
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const float2 f = __half22float2(h[i]);
            x[8 * c + 2 * i] = f.x;
            x[8 * c + 2 * i + 1] = f.y;
        }
    }
}

struct SegInfo {
    int seg, n;
    const uint8_t *base;
};

__device__ __forceinline__ SegInfo seg_of(const MoeArgs &a, int e, const MatrixRef &routed, const MatrixRef &shared) {
    SegInfo s;
    s.seg = a.offsets[e];
    s.n = a.offsets[e + 1] - s.seg;
    s.base = (e < a.E) ? routed.data + (int64_t)e * routed.expert_stride : shared.data;
    return s;
}

__global__ void __launch_bounds__(256) gate_up_simt(MoeArgs a) {
    const int e = blockIdx.y;
    if (e == a.E && !a.has_shared) return;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int r = blockIdx.x * 8 + warp;
    if (r >= a.I) return;
    const SegInfo sg = seg_of(a, e, a.gate, a.sh_gate);
    const SegInfo su = seg_of(a, e, a.up, a.sh_up);
    if (sg.n <= 0) return;
    const int nb = a.H / 32;
    const int64_t row_bytes = (int64_t)nb * 34;
    const uint8_t *grow = sg.base + r * row_bytes;
    const uint8_t *urow = su.base + r * row_bytes;
    for (int tc = 0; tc < sg.n; tc += 8) {
        float ag[8], au[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) ag[j] = au[j] = 0.f;
        for (int b = lane; b < nb; b += 32) {
            float wg[32], wu[32];
            q8_block_fp16(grow + b * 34, wg);
            q8_block_fp16(urow + b * 34, wu);
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                if (tc + j < sg.n) {
                    float xv[32];
                    ld_x32(a.xp + (int64_t)(sg.seg + tc + j) * a.H + b * 32, xv);
                    float g = 0.f, u = 0.f;
#pragma unroll
                    for (int i = 0; i < 32; ++i) {
                        g = fmaf(wg[i], xv[i], g);
                        u = fmaf(wu[i], xv[i], u);
                    }
                    ag[j] += g;
                    au[j] += u;
                }
            }
        }
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            const float g = warp_sum_f32(ag[j]), u = warp_sum_f32(au[j]);
            if (lane == 0 && tc + j < sg.n)
                a.act[(int64_t)(sg.seg + tc + j) * a.I + r] = __float2half_rn(swiglu_clamped(g, u, a.limit));
        }
    }
}

__global__ void __launch_bounds__(256) down_simt(MoeArgs a) {
    const int e = blockIdx.y;
    if (e == a.E && !a.has_shared) return;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int r = blockIdx.x * 8 + warp;
    if (r >= a.H) return;
    const SegInfo sd = seg_of(a, e, a.down, a.sh_down);
    if (sd.n <= 0) return;
    const int nb = a.I / 32;
    const uint8_t *drow = sd.base + (int64_t)r * nb * 34;
    for (int tc = 0; tc < sd.n; tc += 8) {
        float ay[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) ay[j] = 0.f;
        for (int b = lane; b < nb; b += 32) {
            float wd[32];
            q8_block_fp16(drow + b * 34, wd);
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                if (tc + j < sd.n) {
                    float xv[32];
                    ld_x32(a.act + (int64_t)(sd.seg + tc + j) * a.I + b * 32, xv);
                    float s = 0.f;
#pragma unroll
                    for (int i = 0; i < 32; ++i) s = fmaf(wd[i], xv[i], s);
                    ay[j] += s;
                }
            }
        }
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            const float s = warp_sum_f32(ay[j]);
            if (lane == 0 && tc + j < sd.n) a.y[(int64_t)(sd.seg + tc + j) * a.H + r] = s;
        }
    }
}

int launch_experts_simt(const MoeArgs &a, cudaStream_t st, const std::function<void()> &mid) {
    dim3 g1((unsigned)cdiv(a.I, 8), (unsigned)(a.E + 1));
    gate_up_simt<<<g1, 256, 0, st>>>(a);
    VF_LAUNCH_CHECK("gate_up_simt");
    mid();
    dim3 g2((unsigned)cdiv(a.H, 8), (unsigned)(a.E + 1));
    down_simt<<<g2, 256, 0, st>>>(a);
    VF_LAUNCH_CHECK("down_simt");
    return VFMOE_OK;
}

}  // namespace vfmoe
