// Weight-format kernels: Q8_0 quantize/dequantize, EXL3 trellis decode, RMSNorm.
#include <algorithm>
#include "common.cuh"
#include "kernels.h"

namespace vfmoe {

// ----------------------------------------------------------------------------- Q8_0
// One thread per output value.  dst_dtype F32: exact d*q; F16: fp16(d*q) (the value
// the tensor-core kernels feed to the MMA).  native/kernels/q8_0.vyb:11-30.
__global__ void q8_0_dequant_kernel(const uint8_t *__restrict__ src, void *__restrict__ dst, int64_t rows,
                                    int64_t k, int dst_dtype) {
    const int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
    if (i >= rows * k) return;
    const int64_t r = i / k, c = i % k;
    const uint8_t *blk = src + r * (k / 32) * 34 + (c / 32) * 34;
    const float d = q8_scale(blk);
    const float v = d * (float)(int8_t)blk[2 + (c % 32)];
    if (dst_dtype == VFMOE_DT_F16)
        reinterpret_cast<__half *>(dst)[i] = __float2half_rn(v);
    else
        reinterpret_cast<float *>(dst)[i] = v;
}

// One thread per 32-value block (ggml quantize_row_q8_0_ref): d = amax/127,
// q = sign(v) * (floor|v| + floor(2(|v| - floor|v|))) with v = x * (1/d), all fp32.
__global__ void q8_0_quantize_kernel(const float *__restrict__ src, uint8_t *__restrict__ dst, int64_t nblk) {
    const int64_t b = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
    if (b >= nblk) return;
    const float *x = src + b * 32;
    float v[32];
    float amax = 0.f;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        const float4 f = reinterpret_cast<const float4 *>(x)[i];
        v[4 * i] = f.x; v[4 * i + 1] = f.y; v[4 * i + 2] = f.z; v[4 * i + 3] = f.w;
    }
#pragma unroll
    for (int i = 0; i < 32; ++i) amax = fmaxf(amax, fabsf(v[i]));
    const float d = __fdiv_rn(amax, 127.0f);
    const float inv = d == 0.f ? 0.f : __fdiv_rn(1.0f, d);
    // The 34-byte block is 2-byte aligned: write it as 17 little-endian 16-bit words
    // (word 0 = fp16 d, word 1+j = q[2j] | q[2j+1] << 8).
    uint16_t *o = reinterpret_cast<uint16_t *>(dst + b * 34);
    o[0] = __half_as_ushort(__float2half_rn(d));
#pragma unroll
    for (int j = 0; j < 16; ++j) {
        uint32_t pair = 0;
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            const float s = __fmul_rn(v[2 * j + h], inv);
            const float a = fabsf(s);
            const float fl = floorf(a);
            float q = __fadd_rn(fl, floorf(__fmul_rn(2.0f, __fsub_rn(a, fl))));
            q = s < 0.f ? -q : q;
            pair |= ((uint32_t)(int)q & 0xFFu) << (8 * h);
        }
        o[1 + j] = (uint16_t)pair;
    }
}

// ----------------------------------------------------------------------------- EXL3
// 3 bpw layout (defined by this library; the reference has only 4 bpw): a 16x16 tile is
// 48 uint16 words = a 768-bit circular stream, LSB-first.  Window j = bits [3j, 3j+16)
// (mod 768) decodes the weight at tile row r = j % 16, column c = j / 16, so column c's
// 16 rows are the consecutive windows 16c..16c+15 = bits [48c, 48c+61).
__device__ __forceinline__ uint64_t exl3_col_bits_3bpw(const uint16_t *tile, int c) {
    const int w0 = 3 * c;  // 48c / 16
    uint64_t v = 0;
#pragma unroll
    for (int i = 0; i < 4; ++i) v |= (uint64_t)tile[(w0 + i) % 48] << (16 * i);
    return v;
}

// One thread per (tile, column): writes the 16 values of W^[16kb + r][16nb + c].
__global__ void exl3_decode_kernel(const uint16_t *__restrict__ trellis, __half *__restrict__ dst, int64_t K,
                                   int64_t N, int bits) {
    const int64_t g = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
    const int64_t nbk = N / 16;
    const int64_t ntiles = (K / 16) * nbk;
    if (g >= ntiles * 16) return;
    const int c = (int)(g & 15);
    const int64_t tile = g >> 4;
    const int64_t kb = tile / nbk, nb = tile % nbk;
    const uint16_t *tp = trellis + tile * (16 * bits);
    if (bits == 3) {
        const uint64_t v = exl3_col_bits_3bpw(tp, c);
#pragma unroll
        for (int r = 0; r < 16; ++r) {
            const uint32_t w16 = (uint32_t)(v >> (3 * r)) & 0xFFFFu;
            dst[(kb * 16 + r) * N + nb * 16 + c] = exl3_mcg(w16);
        }
    } else {
        uint32_t v[4];
        exl3_col4_pairs(reinterpret_cast<const uint32_t *>(tp), c, v);
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const int rows[4] = {9, 8, 1, 0};
#pragma unroll
            for (int t = 0; t < 4; ++t)
                dst[(kb * 16 + 2 * j + rows[t]) * N + nb * 16 + c] = exl3_mcg((v[j] >> (4 * t)) & 0xFFFFu);
        }
    }
}

// ----------------------------------------------------------------------------- RMSNorm
// One CTA (256 threads) per row: fp32 sum of squares, y = x * rsqrt(mean + eps) * w
// (native/kernels/rmsnorm.vyb; reference recomputes the row stat per element).
__global__ void __launch_bounds__(256) rmsnorm_kernel(const void *__restrict__ x, const float *__restrict__ w,
                                                      void *__restrict__ y, int D, float eps, int dtype) {
    __shared__ float red[8];
    const int64_t row = blockIdx.x;
    float ss = 0.f;
    for (int c = threadIdx.x; c < D; c += 256) {
        const float v = ld_act(x, row * D + c, dtype);
        ss = fmaf(v, v, ss);
    }
    ss = warp_sum_f32(ss);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
    __syncthreads();
    float tot = 0.f;
#pragma unroll
    for (int i = 0; i < 8; ++i) tot += red[i];
    const float r = rsqrtf(tot / (float)D + eps);
    for (int c = threadIdx.x; c < D; c += 256) {
        const float v = ld_act(x, row * D + c, dtype);
        st_act(y, row * D + c, v * r * w[c], dtype);
    }
}

// Residual stream step of a pre-norm stack, one CTA per row:
//   x_out = x + y            (y optional; rounded to dtype)
//   h     = rmsnorm(x_out)   (w optional; statistics over the rounded x_out)
// so the residual add of layer l and the norm of layer l + 1 share one pass.
__global__ void __launch_bounds__(256) residual_rmsnorm_kernel(const void *__restrict__ x, const void *__restrict__ y,
                                                               const float *__restrict__ w, void *__restrict__ x_out,
                                                               void *__restrict__ h, int D, float eps, int dtype) {
    __shared__ float red[8];
    const int64_t row = blockIdx.x;
    float ss = 0.f;
    for (int c = threadIdx.x; c < D; c += 256) {
        float v = ld_act(x, row * D + c, dtype);
        if (y) {
            v += ld_act(y, row * D + c, dtype);
            st_act(x_out, row * D + c, v, dtype);
            v = ld_act(x_out, row * D + c, dtype);  // the rounded value
        }
        ss = fmaf(v, v, ss);
    }
    if (!w) return;
    ss = warp_sum_f32(ss);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
    __syncthreads();
    float tot = 0.f;
#pragma unroll
    for (int i = 0; i < 8; ++i) tot += red[i];
    const float r = rsqrtf(tot / (float)D + eps);
    const void *src = y ? x_out : x;
    for (int c = threadIdx.x; c < D; c += 256) st_act(h, row * D + c, ld_act(src, row * D + c, dtype) * r * w[c], dtype);
}

int launch_residual_rmsnorm(const void *x, const void *y, const float *w, void *x_out, void *h, int64_t S, int D,
                            float eps, int dtype, cudaStream_t st) {
    if (S == 0) return VFMOE_OK;
    residual_rmsnorm_kernel<<<(unsigned)S, 256, 0, st>>>(x, y, w, x_out, h, D, eps, dtype);
    VF_LAUNCH_CHECK("residual_rmsnorm_kernel");
    return VFMOE_OK;
}

int launch_q8_0_dequant(const uint8_t *src, void *dst, int64_t rows, int64_t k, int dst_dtype, cudaStream_t st) {
    const int64_t n = rows * k;
    if (n == 0) return VFMOE_OK;
    q8_0_dequant_kernel<<<(unsigned)cdiv(n, 256), 256, 0, st>>>(src, dst, rows, k, dst_dtype);
    VF_LAUNCH_CHECK("q8_0_dequant_kernel");
    return VFMOE_OK;
}

int launch_q8_0_quantize(const float *src, uint8_t *dst, int64_t rows, int64_t k, cudaStream_t st) {
    const int64_t nblk = rows * (k / 32);
    if (nblk == 0) return VFMOE_OK;
    q8_0_quantize_kernel<<<(unsigned)cdiv(nblk, 128), 128, 0, st>>>(src, dst, nblk);
    VF_LAUNCH_CHECK("q8_0_quantize_kernel");
    return VFMOE_OK;
}

// GGUF Q8_0 rows -> stage-tiled order (VFMOE_WFMT_Q8_0_TILED), one 16-byte chunk per
// thread step, destination order: chunk o of a matrix lies in tile o / 1088 (tile rt, stage
// kr; 17,408 B = 1088 chunks), tile row (o % 1088) / 17, chunk (o % 1088) % 17 of that row's
// 272-byte stage kr.
__global__ void q8_0_tile_kernel(const uint4 *__restrict__ src, uint4 *__restrict__ dst, int64_t n_chunks,
                                 int64_t mat_chunks, int64_t KR) {
    const int64_t row_chunks = 17 * KR;
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n_chunks;
         i += (int64_t)gridDim.x * blockDim.x) {
        const int64_t m = i / mat_chunks, o = i - m * mat_chunks;
        const int64_t tile = o / 1088, w = o - tile * 1088;
        const int64_t rt = tile / KR, kr = tile - rt * KR;
        const int64_t r = w / 17, b = w - r * 17;
        dst[i] = src[m * mat_chunks + (rt * 64 + r) * row_chunks + kr * 17 + b];
    }
}

int launch_q8_0_tile(const uint8_t *src, uint8_t *dst, int64_t rows, int64_t k, int64_t n_mats, cudaStream_t st) {
    const int64_t mat_chunks = rows * (k / 32 * 34) / 16;
    const int64_t n = mat_chunks * n_mats;
    if (n == 0) return VFMOE_OK;
    const int64_t blocks = std::min<int64_t>(cdiv(n, 256), 148 * 16);
    q8_0_tile_kernel<<<(unsigned)blocks, 256, 0, st>>>(reinterpret_cast<const uint4 *>(src),
                                                        reinterpret_cast<uint4 *>(dst), n, mat_chunks, k / 256);
    VF_LAUNCH_CHECK("q8_0_tile_kernel");
    return VFMOE_OK;
}

int launch_exl3_decode(const uint16_t *trellis, __half *dst, int64_t K, int64_t N, int bits, cudaStream_t st) {
    const int64_t n = (K / 16) * (N / 16) * 16;
    if (n == 0) return VFMOE_OK;
    exl3_decode_kernel<<<(unsigned)cdiv(n, 256), 256, 0, st>>>(trellis, dst, K, N, bits);
    VF_LAUNCH_CHECK("exl3_decode_kernel");
    return VFMOE_OK;
}

int launch_rmsnorm(const void *x, const float *w, void *y, int64_t S, int D, float eps, int dtype,
                   cudaStream_t st) {
    if (S == 0) return VFMOE_OK;
    rmsnorm_kernel<<<(unsigned)S, 256, 0, st>>>(x, w, y, D, eps, dtype);
    VF_LAUNCH_CHECK("rmsnorm_kernel");
    return VFMOE_OK;
}

// dst[i] = fp16(src[i]) for src of dtype BF16, F16 or F32 (round to nearest even).
__global__ void to_f16_kernel(const void *__restrict__ src, int dtype, int64_t n, __half *__restrict__ dst) {
    const int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
    if (i < n) dst[i] = __float2half_rn(ld_act(src, i, dtype));
}

int launch_to_f16(const void *src, int dtype, int64_t n, __half *dst, cudaStream_t st) {
    if (n == 0) return VFMOE_OK;
    to_f16_kernel<<<(unsigned)cdiv(n, 256), 256, 0, st>>>(src, dtype, n, dst);
    VF_LAUNCH_CHECK("to_f16_kernel");
    return VFMOE_OK;
}

}  // namespace vfmoe
