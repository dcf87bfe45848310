// Router logits on the tensor cores (tcgen05) for prefill batches: the first level of the
// router's exact selection (router.cu), logits = x . W_r^T in fp32 with a rigorous error bound.
//
// Reference: moe_route / route (native/kernels/moe.vyb:32-95; native/glm53/moe_ref.py:68-78),
// whose logits are exact (f64).  The selection here must equal the exact one, so this kernel only
// has to produce logits whose error is bounded; router_refine re-ranks every expert whose
// bounded interval reaches the k-th largest (float-float, then fp64 for near ties).
//
// Operands: x is bf16 (exact).  W_r (fp32) is split once per layer into bf16 parts
// w = w_hi + w_lo + r with w_hi = bf16(w), w_lo = bf16(w - w_hi), |r| <= 2^-18 |w|.  Every
// product x_i * w_part is exact in fp32 (8-bit by 8-bit significands), so the only errors are the
// tensor core's fp32 accumulation, the dropped residual r and the fp32 sum of the K slices.
//
// Tile: M = 128 tokens (A = x rows, K-major) x N = 128 experts (B = w_hi / w_lo rows, K-major),
// K in slices of 128: each slice is accumulated from zero in TMEM (16 MMAs: 8 k16 steps x 2 parts)
// and added in fp32 to the epilogue's registers, so no accumulator ever sums more than one
// slice.  Two TMEM accumulators alternate, so the MMAs of slice j + 1 overlap the epilogue of j.
//
// Error bound per logit (the constant router_tc_bound returns, times ||x_t||_2 ||w_e||_2):
//   * accumulation: each MMA adds 16 exact products to the accumulator.  The model is that all
//     17 terms are aligned to the largest and each loses less than one unit of the 24-bit
//     result, plus the final rounding: <= 18 * 2^-23 (|acc| + sum |p|) per MMA; the bound uses
//     2^-22 (one bit of margin).  Over the 16 MMAs of a slice |acc| <= the slice's sum |p|, so a
//     slice errs by at most 18 * 17 * 2^-22 * sum_slice |x_i w_i|;
//   * the residual: 2^-18 * sum |x_i| |w_i|;
//   * the fp32 sum of the S slices: gamma_S * sum |x_i w_i| (S = H / 128);
// and sum |x_i w_i| <= ||x|| ||w||.  tests/test_gpu_numerics.py measures the error of this kernel
// against fp64 logits, adversarial cancellation included, and checks it stays far inside.
//
// Warp roles (320 threads): warp 0 TMA producer, warp 1 MMA issuer and TMEM owner, warps 2..9
// epilogue (warp w reads TMEM lanes 32 (w % 4) .. + 31 = tokens, columns 64 ((w - 2) / 4) .. + 63
// = experts).  Every mbarrier wait is bounded (2 s).
#include <cudaTypedefs.h>

#include <algorithm>
#include <cmath>

#include "common.cuh"
#include "kernels.h"
#include "sm100.cuh"

namespace vfmoe {

using namespace sm100;

constexpr int kRtThreads = 320;
constexpr int kRtBox = 128 * 128;             // one 64-K x 128-row bf16 box (SWIZZLE_128B), bytes
constexpr int kRtStage = 6 * kRtBox;          // x, w_hi, w_lo: two 64-K boxes each
constexpr int kRtStages = 2;
constexpr int kRtSmem = kRtStages * kRtStage + 1024 + 256;

// kind::f16 instruction descriptor with bf16 A and B, fp32 D, K-major, M x N.
__host__ __device__ constexpr uint32_t idesc_bf16_f32(int M, int N) {
    return (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}

__device__ __forceinline__ void mma_bf16_ss(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                            uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
        "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
        : "memory");
}

__device__ __forceinline__ void tmem_ld_32x32b_x32(uint32_t taddr, uint32_t (&v)[32]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
        "%15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
        : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]), "=r"(v[8]),
          "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15]), "=r"(v[16]),
          "=r"(v[17]), "=r"(v[18]), "=r"(v[19]), "=r"(v[20]), "=r"(v[21]), "=r"(v[22]), "=r"(v[23]), "=r"(v[24]),
          "=r"(v[25]), "=r"(v[26]), "=r"(v[27]), "=r"(v[28]), "=r"(v[29]), "=r"(v[30]), "=r"(v[31])
        : "r"(taddr)
        : "memory");
}

struct RtParams {
    CUtensorMap xm, whm, wlm;  // x [T][H], w_hi / w_lo [E][H]; bf16, box 64 x 128, SWIZZLE_128B
    int T, H, E;
    int ks;                    // K split: CTA z sums slices [z S / ks, (z + 1) S / ks)
    float *logits;             // [ks][T][E] partial logits (router_refine sums them)
    int *err;
};

__global__ void __launch_bounds__(kRtThreads, 1) router_logits_tc(const __grid_constant__ RtParams p) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint64_t *bars = reinterpret_cast<uint64_t *>(smem + kRtStages * kRtStage);
    uint64_t *full = bars, *empty = bars + kRtStages;       // smem stages
    uint64_t *accf = bars + 2 * kRtStages, *acce = accf + 2;  // TMEM accumulators
    uint64_t *mma_done = acce + 2;
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(mma_done + 1);
    volatile int *abort = reinterpret_cast<volatile int *>(tmem_slot + 1);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int t0 = blockIdx.x * 128, e0 = blockIdx.y * 128;
    const int S_all = p.H / 128;
    const int j0 = blockIdx.z * S_all / p.ks, S = (blockIdx.z + 1) * S_all / p.ks - j0;  // this CTA's slices

    if (threadIdx.x == 0) {
        for (int i = 0; i < kRtStages; ++i) {
            mbar_init(&full[i], 1);
            mbar_init(&empty[i], 1);
        }
        for (int i = 0; i < 2; ++i) {
            mbar_init(&accf[i], 1);
            mbar_init(&acce[i], 8);
        }
        mbar_init(mma_done, 1);
        *abort = 0;
        fence_mbar_init();
    }
    if (warp == 0 && lane == 0) {
        prefetch_tmap(&p.xm);
        prefetch_tmap(&p.whm);
        prefetch_tmap(&p.wlm);
    }
    if (warp == 1) {
        tmem_alloc(tmem_slot, 256);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    pdl_wait_then_release();  // x may come from the previous kernel on the stream

    if (warp == 0) {
        // ---------------------------------------------------------------- TMA producer
        if (lane == 0) {
            bool ok = true;
            int j = 0;
            for (; j < S && ok; ++j) {
                const int s = j % kRtStages;
                if (!(ok = mbar_wait(&empty[s], ((j / kRtStages) & 1) ^ 1, abort))) break;
                uint8_t *st = smem + s * kRtStage;
                mbar_arrive_expect_tx(&full[s], kRtStage);
#pragma unroll
                for (int b = 0; b < 2; ++b) {
                    const int kx = (j0 + j) * 128 + 64 * b;
                    tma_load_2d(st + b * kRtBox, &p.xm, &full[s], kx, t0);
                    tma_load_2d(st + (2 + b) * kRtBox, &p.whm, &full[s], kx, e0);
                    tma_load_2d(st + (4 + b) * kRtBox, &p.wlm, &full[s], kx, e0);
                }
            }
            if (!ok) {
                atomicCAS(p.err, 0, DEV_WAIT_TIMEOUT);
                int dummy = 0;
                for (int i = (j > kRtStages ? j - kRtStages : 0); i < j; ++i)
                    mbar_wait(&full[i % kRtStages], (i / kRtStages) & 1, (volatile int *)&dummy, 100000000ull);
            }
        }
    } else if (warp == 1) {
        // ---------------------------------------------------------------- MMA issuer
        if (lane == 0) {
            const uint32_t idesc = idesc_bf16_f32(128, 128);
            bool ok = true;
            for (int j = 0; j < S && ok; ++j) {
                const int s = j % kRtStages, a = j & 1;
                if (!(ok = mbar_wait(&full[s], (j / kRtStages) & 1, abort))) break;
                if (!(ok = mbar_wait(&acce[a], ((j >> 1) & 1) ^ 1, abort))) break;
                tc_fence_after();
                const uint32_t st = smem_u32(smem + s * kRtStage);
                const uint32_t d = tmem + a * 128;
#pragma unroll
                for (int b = 0; b < 2; ++b)
#pragma unroll
                    for (int k = 0; k < 4; ++k) {
                        const uint64_t ad = smem_desc_sw128(st + b * kRtBox + 32 * k);
                        mma_bf16_ss(d, ad, smem_desc_sw128(st + (2 + b) * kRtBox + 32 * k), idesc, (b | k) != 0);
                        mma_bf16_ss(d, ad, smem_desc_sw128(st + (4 + b) * kRtBox + 32 * k), idesc, 1);
                    }
                mma_commit(&empty[s]);
                mma_commit(&accf[a]);
            }
            mma_commit(mma_done);
            int dummy = 0;
            mbar_wait(mma_done, 0, (volatile int *)&dummy, 200000000ull);
            if (!ok) atomicCAS(p.err, 0, DEV_WAIT_TIMEOUT);
        }
    } else {
        // ---------------------------------------------------------------- epilogue
        const int q = warp & 3, h = (warp - 2) >> 2;
        const uint32_t lane_base = (uint32_t)(32 * q) << 16;
        float run[64];
#pragma unroll
        for (int i = 0; i < 64; ++i) run[i] = 0.f;
        bool ok = true;
        for (int j = 0; j < S && ok; ++j) {
            const int a = j & 1;
            if (!(ok = mbar_wait(&accf[a], (j >> 1) & 1, abort))) break;
            tc_fence_after();
            uint32_t v[32];
#pragma unroll
            for (int c = 0; c < 2; ++c) {
                tmem_ld_32x32b_x32(tmem + lane_base + a * 128 + 64 * h + 32 * c, v);
                tmem_wait_ld();
#pragma unroll
                for (int i = 0; i < 32; ++i) run[32 * c + i] += __uint_as_float(v[i]);
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&acce[a]);
        }
        if (ok) {
            const int t = t0 + 32 * q + lane;
            if (t < p.T) {
                float *o = p.logits + ((int64_t)blockIdx.z * p.T + t) * p.E + e0 + 64 * h;
#pragma unroll
                for (int i = 0; i < 64; i += 4) *reinterpret_cast<float4 *>(o + i) = make_float4(run[i], run[i + 1], run[i + 2], run[i + 3]);
            }
        } else {
            atomicCAS(p.err, 0, DEV_WAIT_TIMEOUT);
        }
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (warp == 1) tmem_dealloc(tmem, 256);
}

// w (fp32 [n]) -> w_hi = bf16(w), w_lo = bf16(w - w_hi), both round-to-nearest-even.
__global__ void router_split_kernel(const float *__restrict__ w, int64_t n, __nv_bfloat16 *__restrict__ hi,
                                    __nv_bfloat16 *__restrict__ lo) {
    const int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
    if (i >= n) return;
    const float v = w[i];
    const __nv_bfloat16 a = __float2bfloat16_rn(v);
    hi[i] = a;
    lo[i] = __float2bfloat16_rn(v - __bfloat162float(a));
}

static PFN_cuTensorMapEncodeTiled_v12000 rt_encode() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    if (!fn) {
        void *ptr = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(ptr);
    }
    return fn;
}

// bf16 [rows][cols] (row-major), box 64 columns x 128 rows, SWIZZLE_128B; rows beyond the matrix
// read as zero.
static int make_bf16_map(CUtensorMap *m, const void *base, int64_t rows, int64_t cols) {
    auto enc = rt_encode();
    if (!enc) {
        set_error("cuTensorMapEncodeTiled unavailable from the driver");
        return VFMOE_ERR_CUDA;
    }
    cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
    cuuint64_t strides[1] = {(cuuint64_t)(cols * 2)};
    cuuint32_t box[2] = {64, 128};
    cuuint32_t es[2] = {1, 1};
    CUresult r = enc(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void *>(base), dims, strides, box, es,
                     CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                     CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) {
        set_error("cuTensorMapEncodeTiled (router operands) failed: %d", (int)r);
        return VFMOE_ERR_CUDA;
    }
    return VFMOE_OK;
}

bool router_tc_shape(int T, int H, int E) { return T > 32 && H % 128 == 0 && E % 128 == 0; }

// K split: enough CTAs for about two waves on 148 SMs, at most 8, at least 4 slices per CTA.
int router_tc_splits(int T, int H, int E) {
    const int64_t tiles = cdiv(T, 128) * (E / 128);
    int ks = (int)std::min<int64_t>(8, cdiv(296, tiles));
    ks = std::max(1, std::min(ks, H / 128 / 4));
    return ks;
}

float router_tc_bound(int H) {
    const double acc = 18.0 * 17.0 * std::ldexp(1.0, -22);         // per 128-K slice, 16 MMAs
    const double res = std::ldexp(1.0, -18);                         // dropped residual of the split
    const double S = H / 128;
    const double sum = S * std::ldexp(1.0, -24) / (1.0 - S * std::ldexp(1.0, -24));  // slice sum
    return (float)((acc + res + sum) * 1.01);
}

int launch_router_split(const float *wr, int64_t n, __nv_bfloat16 *hi, __nv_bfloat16 *lo, cudaStream_t st) {
    router_split_kernel<<<(unsigned)cdiv(n, 256), 256, 0, st>>>(wr, n, hi, lo);
    VF_LAUNCH_CHECK("router_split_kernel");
    return VFMOE_OK;
}

int launch_router_logits_tc(const void *x, const __nv_bfloat16 *wr_split, int T, int H, int E, float *logits, int *err,
                            cudaStream_t st) {
    RtParams p{};
    int rc;
    if ((rc = make_bf16_map(&p.xm, x, T, H))) return rc;
    if ((rc = make_bf16_map(&p.whm, wr_split, E, H))) return rc;
    if ((rc = make_bf16_map(&p.wlm, wr_split + (int64_t)E * H, E, H))) return rc;
    p.T = T;
    p.H = H;
    p.E = E;
    p.ks = router_tc_splits(T, H, E);
    p.logits = logits;
    p.err = err;
    if ((rc = set_smem_attr_once(reinterpret_cast<const void *>(router_logits_tc), kRtSmem))) return rc;
    dim3 grid((unsigned)cdiv(T, 128), (unsigned)(E / 128), (unsigned)p.ks);
    VF_CUDA(launch_pdl(router_logits_tc, grid, dim3(kRtThreads), (size_t)kRtSmem, st, p));
    VF_LAUNCH_CHECK("router_logits_tc");
    return VFMOE_OK;
}

}  // namespace vfmoe
