// EXL3 expert products (3 bits/weight trellis, mcg codebook), decode path.
//
// The reference reconstructs each weight matrix as W = diag(suh) Hb W^ Hb diag(svh) with
// Hb = blockdiag(H128 / sqrt(128)) (native/exl3/exl3_ref.py:84-120), two dense 128-tap
// transforms per block that dominated its MoE time.  Here the Hadamard moves to the
// activations (H is symmetric and orthogonal):
//
//     y = x W = ((x * suh) Hb) W^ Hb * svh
//
// so the GEMV only decodes trellis windows into W^ (fp16 values, exact) and the two
// rotations are 128-point fast Walsh-Hadamard transforms on activations:
//   gather_exl3   x_perm[row][gate|up] = fp16(FWHT(x * suh_{gate|up,e}) / sqrt(128))
//   gemv (gate/up) z = x' W^ per 128-channel tile; epilogue: y = FWHT(z)/sqrt(128) * svh,
//                 act = swiglu(y_g, y_u), act' = fp16(FWHT(act * suh_down)/sqrt(128))
//   gemv (down)   z = act' W^_d; epilogue y = FWHT(z)/sqrt(128) * svh_down (fp32)
//
// 3-bpw layout (defined here; the reference has 4 bpw only): a 16x16 tile is 48 uint16
// words = a 768-bit circular stream, LSB-first; window j = bits [3j, 3j+16) decodes the
// weight at tile row r = j % 16 (input k), column c = j / 16 (output n).  Output column c
// of a tile is 16 consecutive windows at bits [48c, 48c+61).
//
// The GEMV follows expert_gemv.cu: TMA producer warp, 8 consumer warps, mma.sync
// m16n8k16 with decoded fp16 fragments in registers; K permutation: thread c of the MMA
// quad owns the 16 k of one trellis tile (k-tile 4p + c of each 64-K group p).
#include <cudaTypedefs.h>

#include <algorithm>

#include "expert_tc.h"
#include "sm100.cuh"

namespace vfmoe {

using namespace sm100;

constexpr float kRScale = 0.08838834764831845f;  // 1/sqrt(128)
constexpr int kXcon = 8;                           // consumer warps
constexpr int kXthreads = 32 * (kXcon + 1);
constexpr int kKT = 16;                            // k-tiles (of 16) per stage = 256 K
constexpr int kTileBytes3 = 96;                    // 48 uint16 words

// ----------------------------------------------------------------------------- FWHT helpers
// 128-point unnormalised Walsh-Hadamard transform of v[q] = element (lane + 32q), q = 0..3,
// across one warp (natural / Sylvester order: butterflies at strides 1..64).
__device__ __forceinline__ void fwht128_warp(float (&v)[4]) {
#pragma unroll
    for (int s = 1; s < 32; s <<= 1) {
#pragma unroll
        for (int q = 0; q < 4; ++q) {
            const float o = __shfl_xor_sync(0xffffffffu, v[q], s);
            v[q] = (threadIdx.x & s) ? (o - v[q]) : (v[q] + o);
        }
    }
    // strides 32 and 64: between the q slots of one lane
    float a0 = v[0] + v[1], a1 = v[0] - v[1], a2 = v[2] + v[3], a3 = v[2] - v[3];
    v[0] = a0 + a2;
    v[1] = a1 + a3;
    v[2] = a0 - a2;
    v[3] = a1 - a3;
}

__device__ __forceinline__ int segment_of(const int32_t *offsets, int nseg, int pos) {
    int lo = 0, hi = nseg - 1;  // largest e with offsets[e] <= pos
    while (lo < hi) {
        const int mid = (lo + hi + 1) >> 1;
        if (offsets[mid] <= pos) lo = mid; else hi = mid - 1;
    }
    return lo;
}

// One CTA (256 threads = 8 warps) per permuted row: both rotated versions (gate, up).
__global__ void __launch_bounds__(256) gather_exl3_kernel(const void *__restrict__ x, int x_dtype,
                                                          const int32_t *__restrict__ perm_tok,
                                                          const int32_t *__restrict__ offsets, int nseg, int E, int H,
                                                          MatrixRef gate, MatrixRef up, MatrixRef sh_gate,
                                                          MatrixRef sh_up, __half *__restrict__ xp) {
    const int pos = blockIdx.x;
    const int t = perm_tok[pos];
    const int e = segment_of(offsets, nseg, pos);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    for (int ver = 0; ver < 2; ++ver) {
        const MatrixRef &m = (e < E) ? (ver ? up : gate) : (ver ? sh_up : sh_gate);
        const __half *suh = reinterpret_cast<const __half *>(reinterpret_cast<const uint8_t *>(m.suh) +
                                                             (e < E ? (int64_t)e * m.suh_stride : 0));
        __half *dst = xp + ((int64_t)pos * 2 + ver) * H;
        for (int b = warp; b < H / 128; b += 8) {
            float v[4];
#pragma unroll
            for (int q = 0; q < 4; ++q) {
                const int k = 128 * b + lane + 32 * q;
                v[q] = ld_act(x, (int64_t)t * H + k, x_dtype) * __half2float(suh[k]);
            }
            fwht128_warp(v);
#pragma unroll
            for (int q = 0; q < 4; ++q) dst[128 * b + lane + 32 * q] = __float2half_rn(v[q] * kRScale);
        }
    }
}

// ----------------------------------------------------------------------------- decode GEMV
template <bool GATEUP, int NT>
struct XCfg {
    static constexpr int N = 8 * NT;
    static constexpr int MATS = GATEUP ? 2 : 1;
    static constexpr int WBYTES = MATS * kKT * 8 * kTileBytes3;   // trellis per stage
    static constexpr int TOKROWS = GATEUP ? 2 * N : N;            // gate/up: two rotated versions
    static constexpr int TOK = TOKROWS * 512;                      // 256 K fp16
    static constexpr int STAGE = ((WBYTES + TOK) + 1023) / 1024 * 1024;
    static constexpr int XLD = 132;                                // exchange row stride (floats)
    static constexpr int XCH = MATS * N * XLD * 4;                 // epilogue exchange [m][token][channel]
    static constexpr int SW = (220000 - XCH) / STAGE > 6 ? 6 : (220000 - XCH) / STAGE;
    static constexpr int SMEM = SW * STAGE + XCH + 2 * SW * 8 + 16 + 1024;
    static_assert(SW >= 2, "double buffering");
    static_assert(SMEM <= 232448, "shared memory");
};

struct XParams {
    CUtensorMap wa, wb, swa, swb;  // trellis [E][K/16][N/16*24 u32] (routed) / shared
    CUtensorMap xt;                // token rows fp16
    const int4 *tiles;
    const int32_t *n_tiles;
    int E, K, M;
    MatrixRef ma, mb, sma, smb;    // suh/svh of the tile's matrices (routed, shared)
    MatrixRef mdown, smdown;       // gate/up epilogue: suh of the down projection
    int ld_out;
    void *out;
    float limit;
    int *err;
};

// 16 decoded weights (one tile column, k = 0..15) -> 8 packed fp16 pairs.
__device__ __forceinline__ void exl3_col16(const uint16_t *tile, int c, uint32_t (&out)[8]) {
    const int w0 = 3 * c;
    uint64_t v = 0;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const int wi = w0 + i;
        v |= (uint64_t)tile[wi >= 48 ? wi - 48 : wi] << (16 * i);
    }
#pragma unroll
    for (int p = 0; p < 8; ++p) {
        const uint32_t wa = (uint32_t)(v >> (6 * p)) & 0xFFFFu;
        const uint32_t wb = (uint32_t)(v >> (6 * p + 3)) & 0xFFFFu;
        const uint32_t ya = ((wa * 0xCBAC1FEDu) & 0x8FFF8FFFu) ^ 0x3B603B60u;
        const uint32_t yb = ((wb * 0xCBAC1FEDu) & 0x8FFF8FFFu) ^ 0x3B603B60u;
        const uint32_t lo = __byte_perm(ya, yb, 0x5410), hi = __byte_perm(ya, yb, 0x7632);
        const __half2 s = __hadd2(*reinterpret_cast<const __half2 *>(&lo), *reinterpret_cast<const __half2 *>(&hi));
        out[p] = *reinterpret_cast<const uint32_t *>(&s);
    }
}

template <bool GATEUP, int NT>
__global__ void __launch_bounds__(kXthreads, 1) expert_gemv_exl3(const __grid_constant__ XParams p) {
    using C = XCfg<GATEUP, NT>;
    constexpr int SW = C::SW, N = C::N, MATS = C::MATS;
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    float *xch = reinterpret_cast<float *>(smem + SW * C::STAGE);
    uint64_t *full = reinterpret_cast<uint64_t *>(smem + SW * C::STAGE + C::XCH);
    uint64_t *empty = full + SW;
    volatile int *abort = reinterpret_cast<volatile int *>(empty + SW);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int MT = p.M / 128;
    const int KR = p.K / 256;
    if (threadIdx.x == 0) {
        for (int i = 0; i < SW; ++i) {
            mbar_init(&full[i], 1);
            mbar_init(&empty[i], kXcon);
        }
        *abort = 0;
        fence_mbar_init();
    }
    __syncthreads();
    const int n_items = (*p.n_tiles) * MT;

    if (warp == kXcon) {
        if (lane == 0) {
            prefetch_tmap(&p.wa);
            prefetch_tmap(&p.xt);
            uint32_t n = 0;
            bool ok = true;
            for (int item = blockIdx.x; item < n_items && ok; item += gridDim.x) {
                const int4 t = p.tiles[item / MT];
                const int nb0 = (item % MT) * 8;  // first 16-column block of the tile
                const bool sh = t.x == p.E;
                const CUtensorMap *ma = sh ? &p.swa : &p.wa;
                const CUtensorMap *mb = sh ? &p.swb : &p.wb;
                const int z = sh ? 0 : t.x;
                for (int kr = 0; kr < KR; ++kr, ++n) {
                    const uint32_t s = n % SW;
                    if (!(ok = mbar_wait(&empty[s], ((n / SW) & 1) ^ 1, abort))) break;
                    uint8_t *st = smem + s * C::STAGE;
                    mbar_arrive_expect_tx(&full[s], C::WBYTES + C::TOK);
                    tma_load_3d(st, ma, &full[s], nb0 * 24, kr * kKT, z);
                    if (GATEUP) tma_load_3d(st + kKT * 8 * kTileBytes3, mb, &full[s], nb0 * 24, kr * kKT, z);
#pragma unroll
                    for (int q = 0; q < 4; ++q)
                        tma_load_2d(st + C::WBYTES + q * (C::TOKROWS * 128), &p.xt, &full[s], kr * 256 + 64 * q,
                                    GATEUP ? 2 * t.y : t.y);
                }
            }
            if (!ok) {
                atomicCAS(p.err, 0, DEV_WAIT_TIMEOUT);
                int dummy = 0;
                for (uint32_t i = (n > (uint32_t)SW ? n - SW : 0); i < n; ++i)
                    mbar_wait(&full[i % SW], (i / SW) & 1, (volatile int *)&dummy, 100000000ull);
            }
        }
        return;
    }

    // ------------------------------------------------------------------ consumers
    const int g = lane >> 2, c = lane & 3;
    const int r0 = 16 * warp;  // channels r0 + g, r0 + g + 8 of the 128-channel tile
    uint32_t n = 0;
    bool ok = true;
    for (int item = blockIdx.x; item < n_items && ok; item += gridDim.x) {
        const int4 t = p.tiles[item / MT];
        const int ntv = (t.z + 7) >> 3;
        float acc[MATS][NT][4];
#pragma unroll
        for (int m = 0; m < MATS; ++m)
#pragma unroll
            for (int j = 0; j < NT; ++j) acc[m][j][0] = acc[m][j][1] = acc[m][j][2] = acc[m][j][3] = 0.f;
        for (int kr = 0; kr < KR; ++kr, ++n) {
            const uint32_t s = n % SW;
            if (!(ok = mbar_wait(&full[s], (n / SW) & 1, abort))) break;
            const uint8_t *st = smem + s * C::STAGE;
#pragma unroll
            for (int pq = 0; pq < 4; ++pq) {
                const int kt = 4 * pq + c;  // this thread's k-tile in the stage
                const uint8_t *tq = st + C::WBYTES + pq * (C::TOKROWS * 128);
#pragma unroll
                for (int m = 0; m < MATS; ++m) {
                    const uint8_t *wbase = st + m * (kKT * 8 * kTileBytes3) + kt * (8 * kTileBytes3);
                    uint32_t wa[8], wb[8];
                    const int ra = r0 + g, rb = r0 + g + 8;
                    exl3_col16(reinterpret_cast<const uint16_t *>(wbase + (ra >> 4) * kTileBytes3), ra & 15, wa);
                    exl3_col16(reinterpret_cast<const uint16_t *>(wbase + (rb >> 4) * kTileBytes3), rb & 15, wb);
#pragma unroll
                    for (int j = 0; j < NT; ++j) {
                        if (j < ntv) {
                            const int rr = GATEUP ? 2 * (8 * j + g) + m : 8 * j + g;  // token row in the tile
                            const uint4 x0 = *reinterpret_cast<const uint4 *>(tq + rr * 128 + (((2 * c) ^ (rr & 7)) << 4));
                            const uint4 x1 = *reinterpret_cast<const uint4 *>(tq + rr * 128 + (((2 * c + 1) ^ (rr & 7)) << 4));
                            const uint32_t xb[8] = {x0.x, x0.y, x0.z, x0.w, x1.x, x1.y, x1.z, x1.w};
#pragma unroll
                            for (int s4 = 0; s4 < 4; ++s4) {
                                const uint32_t a[4] = {wa[2 * s4], wb[2 * s4], wa[2 * s4 + 1], wb[2 * s4 + 1]};
                                asm volatile(
                                    "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0, %1, %2, %3}, {%4, %5, %6, "
                                    "%7}, {%8, %9}, {%0, %1, %2, %3};"
                                    : "+f"(acc[m][j][0]), "+f"(acc[m][j][1]), "+f"(acc[m][j][2]), "+f"(acc[m][j][3])
                                    : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(xb[2 * s4]), "r"(xb[2 * s4 + 1]));
                            }
                        }
                    }
                }
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&empty[s]);
        }
        if (!ok) break;
        // ---------------------------------------------------------------- epilogue
        // z -> shared memory [m][token][channel], then one warp per token: FWHT over
        // the 128 channels, * svh, (gate/up) swiglu, * suh_down, FWHT, fp16 store.
#pragma unroll
        for (int m = 0; m < MATS; ++m)
#pragma unroll
            for (int j = 0; j < NT; ++j)
#pragma unroll
                for (int e4 = 0; e4 < 4; ++e4) {
                    const int ch = r0 + g + 8 * (e4 >> 1), tok = 8 * j + 2 * c + (e4 & 1);
                    xch[(m * N + tok) * C::XLD + ch] = acc[m][j][e4];
                }
        asm volatile("bar.sync 1, %0;" ::"r"(32 * kXcon) : "memory");
        const int e = t.x;
        const bool sh = e == p.E;
        const int ch0 = (item % MT) * 128;
        for (int tok = warp; tok < t.z; tok += kXcon) {
            float v[MATS][4];
#pragma unroll
            for (int m = 0; m < MATS; ++m) {
#pragma unroll
                for (int q = 0; q < 4; ++q) v[m][q] = xch[(m * N + tok) * C::XLD + lane + 32 * q];
                fwht128_warp(v[m]);
                const MatrixRef &mr = sh ? (m ? p.smb : p.sma) : (m ? p.mb : p.ma);
                const __half *svh = reinterpret_cast<const __half *>(reinterpret_cast<const uint8_t *>(mr.svh) +
                                                                     (sh ? 0 : (int64_t)e * mr.svh_stride));
#pragma unroll
                for (int q = 0; q < 4; ++q) v[m][q] *= kRScale * __half2float(svh[ch0 + lane + 32 * q]);
            }
            if (GATEUP) {
                const MatrixRef &md = sh ? p.smdown : p.mdown;
                const __half *suh = reinterpret_cast<const __half *>(reinterpret_cast<const uint8_t *>(md.suh) +
                                                                     (sh ? 0 : (int64_t)e * md.suh_stride));
                float a[4];
#pragma unroll
                for (int q = 0; q < 4; ++q)
                    a[q] = swiglu_clamped(v[0][q], v[MATS - 1][q], p.limit) * __half2float(suh[ch0 + lane + 32 * q]);
                fwht128_warp(a);
                __half *out = reinterpret_cast<__half *>(p.out);
#pragma unroll
                for (int q = 0; q < 4; ++q)
                    out[(int64_t)(t.y + tok) * p.ld_out + ch0 + lane + 32 * q] = __float2half_rn(a[q] * kRScale);
            } else {
                float *out = reinterpret_cast<float *>(p.out);
#pragma unroll
                for (int q = 0; q < 4; ++q) out[(int64_t)(t.y + tok) * p.ld_out + ch0 + lane + 32 * q] = v[0][q];
            }
        }
        asm volatile("bar.sync 1, %0;" ::"r"(32 * kXcon) : "memory");
    }
    if (!ok) atomicCAS(p.err, 0, DEV_WAIT_TIMEOUT);
}

// ----------------------------------------------------------------------------- host
static PFN_cuTensorMapEncodeTiled_v12000 x_encode() {
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

// Trellis stack [experts][K/16][N/16][48 u16] as u32 elements; box = 8 column blocks x kKT k-tiles.
static int make_trellis_map(CUtensorMap *m, const void *base, int64_t K, int64_t N, int64_t experts, int64_t stride) {
    auto enc = x_encode();
    if (!enc) {
        set_error("cuTensorMapEncodeTiled unavailable from the driver");
        return VFMOE_ERR_CUDA;
    }
    const int64_t row_u32 = (N / 16) * 24;
    if (experts <= 1) stride = (K / 16) * row_u32 * 4;
    cuuint64_t dims[3] = {(cuuint64_t)row_u32, (cuuint64_t)(K / 16), (cuuint64_t)experts};
    cuuint64_t strides[2] = {(cuuint64_t)(row_u32 * 4), (cuuint64_t)stride};
    cuuint32_t box[3] = {8 * 24, (cuuint32_t)kKT, 1};
    cuuint32_t es[3] = {1, 1, 1};
    CUresult r = enc(m, CU_TENSOR_MAP_DATA_TYPE_UINT32, 3, const_cast<void *>(base), dims, strides, box, es,
                     CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                     CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) {
        set_error("cuTensorMapEncodeTiled (EXL3 trellis) failed: %d", (int)r);
        return VFMOE_ERR_CUDA;
    }
    return VFMOE_OK;
}

static int make_rows_map(CUtensorMap *m, const void *base, int64_t rows, int64_t k, int box_rows) {
    auto enc = x_encode();
    if (!enc) {
        set_error("cuTensorMapEncodeTiled unavailable from the driver");
        return VFMOE_ERR_CUDA;
    }
    cuuint64_t dims[2] = {(cuuint64_t)k, (cuuint64_t)rows};
    cuuint64_t strides[1] = {(cuuint64_t)(k * 2)};
    cuuint32_t box[2] = {64, (cuuint32_t)box_rows};
    cuuint32_t es[2] = {1, 1};
    CUresult r = enc(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void *>(base), dims, strides, box, es,
                     CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                     CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) {
        set_error("cuTensorMapEncodeTiled (EXL3 token rows) failed: %d", (int)r);
        return VFMOE_ERR_CUDA;
    }
    return VFMOE_OK;
}

int exl3_plan_create(const vfmoe_layer_desc &d, Exl3Plan &plan) {
    plan.ready = 0;
    if (d.weight_format != VFMOE_WFMT_EXL3 || d.exl3_bits != 3) return VFMOE_OK;
    int dev = 0;
    VF_CUDA(cudaGetDevice(&dev));
    VF_CUDA(cudaDeviceGetAttribute(&plan.num_sms, cudaDevAttrMultiProcessorCount, dev));
    const int64_t H = d.hidden, I = d.inter, E = d.n_local_experts ? d.n_local_experts : d.n_experts;
    int rc;
    if ((rc = make_trellis_map(&plan.gate, (void *)d.gate.data, H, I, E, d.gate.expert_stride))) return rc;
    if ((rc = make_trellis_map(&plan.up, (void *)d.up.data, H, I, E, d.up.expert_stride))) return rc;
    if ((rc = make_trellis_map(&plan.down, (void *)d.down.data, I, H, E, d.down.expert_stride))) return rc;
    const bool sh = d.sh_gate.data != 0;
    if ((rc = make_trellis_map(&plan.sh_gate, (void *)(sh ? d.sh_gate.data : d.gate.data), H, I, 1, 0))) return rc;
    if ((rc = make_trellis_map(&plan.sh_up, (void *)(sh ? d.sh_up.data : d.up.data), H, I, 1, 0))) return rc;
    if ((rc = make_trellis_map(&plan.sh_down, (void *)(sh ? d.sh_down.data : d.down.data), I, H, 1, 0))) return rc;
    plan.ready = 1;
    return VFMOE_OK;
}

template <bool GATEUP, int NT>
static int launch_x(const XParams &prm, int grid, cudaStream_t st) {
    using C = XCfg<GATEUP, NT>;
    static bool attr_done = false;
    if (!attr_done) {
        VF_CUDA(cudaFuncSetAttribute(expert_gemv_exl3<GATEUP, NT>, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM));
        attr_done = true;
    }
    expert_gemv_exl3<GATEUP, NT><<<grid, kXthreads, C::SMEM, st>>>(prm);
    VF_LAUNCH_CHECK(GATEUP ? "expert_gemv_exl3<gate_up>" : "expert_gemv_exl3<down>");
    return VFMOE_OK;
}

int launch_experts_exl3(const Exl3Plan &plan, const MoeArgs &a, const void *x, int x_dtype,
                        cudaStream_t st, const std::function<void()> &mid) {
    const int N = gemv_tokens_per_tile(a.T, a.k, a.E);
    const int64_t rows = (int64_t)a.T * a.k + (a.has_shared ? a.T : 0);
    int rc = launch_tc_plan(a, N, N, st);
    if (rc) return rc;
    if (rows > 0) {
        gather_exl3_kernel<<<(unsigned)rows, 256, 0, st>>>(x, x_dtype, a.perm_tok, a.offsets, a.E + (a.has_shared ? 1 : 0),
                                                           a.E, a.H, a.gate, a.up, a.sh_gate, a.sh_up,
                                                           const_cast<__half *>(a.xp));
        VF_LAUNCH_CHECK("gather_exl3_kernel");
    }
    const int64_t cap_rows = (int64_t)a.T * a.k + a.T;
    XParams g{};
    g.wa = plan.gate;
    g.wb = plan.up;
    g.swa = plan.sh_gate;
    g.swb = plan.sh_up;
    if ((rc = make_rows_map(&g.xt, a.xp, 2 * cap_rows, a.H, 2 * N))) return rc;
    g.tiles = a.tiles;
    g.n_tiles = a.tile_counts;
    g.E = a.E;
    g.K = a.H;
    g.M = a.I;
    g.ma = a.gate;
    g.mb = a.up;
    g.sma = a.sh_gate;
    g.smb = a.sh_up;
    g.mdown = a.down;
    g.smdown = a.sh_down;
    g.ld_out = a.I;
    g.out = a.act;
    g.limit = a.limit;
    g.err = a.err;
    const int grid = plan.num_sms;
    switch (N) {
        case 8: rc = launch_x<true, 1>(g, grid, st); break;
        case 16: rc = launch_x<true, 2>(g, grid, st); break;
        default: rc = launch_x<true, 4>(g, grid, st); break;
    }
    if (rc) return rc;
    mid();
    XParams dn{};
    dn.wa = plan.down;
    dn.wb = plan.down;
    dn.swa = plan.sh_down;
    dn.swb = plan.sh_down;
    if ((rc = make_rows_map(&dn.xt, a.act, cap_rows, a.I, N))) return rc;
    dn.tiles = a.tiles;
    dn.n_tiles = a.tile_counts;
    dn.E = a.E;
    dn.K = a.I;
    dn.M = a.H;
    dn.ma = a.down;
    dn.mb = a.down;
    dn.sma = a.sh_down;
    dn.smb = a.sh_down;
    dn.ld_out = a.H;
    dn.out = a.y;
    dn.limit = a.limit;
    dn.err = a.err;
    switch (N) {
        case 8: return launch_x<false, 1>(dn, grid, st);
        case 16: return launch_x<false, 2>(dn, grid, st);
        default: return launch_x<false, 4>(dn, grid, st);
    }
}

}  // namespace vfmoe
