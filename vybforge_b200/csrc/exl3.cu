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
    if (pos >= offsets[nseg]) return;  // launch size is an upper bound on the rows dispatched
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
// Shared-memory trellis layout per stage and matrix: [nb 0..7][kt 0..15][48 u16] (a 4D TMA
// box over the global [K/16][N/16][48] order), so the four threads of an MMA quad (four
// k-tiles of one column block, 96 B apart) and its eight row groups hit 32 distinct banks.
// MMA row g of a warp's 16-channel block is channel 2g, row g + 8 is channel 2g + 1: one
// thread decodes two adjacent trellis columns, 14 bytes at u16 word 6g, with 4 LDS.32.
//
// Each window decodes to fp16(lo + hi) of the two halves of its mcg word, as the reference
// does (one fp16 add per pair of weights, HADD2), so the GEMV multiplies exactly the
// reference's decoded weights.
//
// CW consumer warps: 8 own 16 channels each over the whole 256-K stage; with 16 the second
// group takes the upper half of every stage (k-tiles 8..15) and the two partial sums meet
// in the epilogue exchange buffer.
template <bool GATEUP, int NT, int CW>
struct XCfg {
    static constexpr int N = 8 * NT;
    static constexpr int MATS = GATEUP ? 2 : 1;
    static constexpr int KG = CW / 8;                              // k groups
    static constexpr int PQ = 4 / KG;                              // 64-K quarters per warp and stage
    static constexpr int THREADS = 32 * (CW + 1);
    static constexpr int WBYTES = MATS * kKT * 8 * kTileBytes3;   // trellis per stage
    static constexpr int TOKROWS = GATEUP ? 2 * N : N;            // gate/up: two rotated versions
    static constexpr int TOK = TOKROWS * 512;                      // 256 K fp16
    static constexpr int STAGE = ((WBYTES + TOK) + 1023) / 1024 * 1024;
    static constexpr int XLD = 132;                                // exchange row stride (floats)
    static constexpr int XCH = MATS * N * XLD * 4;                 // epilogue exchange [m][token][channel]
    static constexpr int SW = (220000 - XCH) / STAGE > 6 ? 6 : (220000 - XCH) / STAGE;
    static constexpr int SMEM = SW * STAGE + XCH + 2 * SW * 8 + 16 + 1024;
    static_assert(CW == 8 || CW == 16, "consumer warps");
    static_assert(SW >= 2, "double buffering");
    static_assert(SMEM <= 232448, "shared memory");
};

struct XParams {
    CUtensorMap wa, wb, swa, swb;  // trellis 4D maps (routed, shared): {24 u32, K/16, N/16, experts}
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
    uint32_t k65536;               // 65536 as a run-time value: its multiplies stay IMADs
    uint32_t kxor;                 // 0x3B603B60 in a register: mask and xor in one LOP3
};

// Window at absolute bit O of the 128-bit little-endian stream w[0..3], as a clean 16-bit
// value.  The extraction is spread over the ALU and IMAD pipes (both limit this kernel):
//   byte-aligned inside a word     PRMT with zero fill                 1 ALU
//   inside one word                SHL to the top, IMAD.HI by 2^16     1 ALU + 1 IMAD
//   across two words, O >= 81      funnel shift, AND                   2 ALU
//   across two words, otherwise    funnel shift, IMAD.LO/HI by 2^16    1 ALU + 2 IMAD
template <int O>
__device__ __forceinline__ uint32_t window16(const uint32_t (&w)[4], uint32_t k65536) {
    constexpr int j = O >> 5, s = O & 31;
    if constexpr (s % 8 == 0 && s <= 16) {
        return __byte_perm(w[j], 0u, (s / 8) | ((s / 8 + 1) << 4) | (4 << 8) | (4 << 12));
    } else if constexpr (s < 16) {
        return __umulhi(w[j] << (16 - s), k65536);
    } else {
        const uint32_t u = __funnelshift_r(w[j], w[j + 1], s);
        if constexpr (O >= 81) {
            return u & 0xFFFFu;
        } else {
            return __umulhi(u * k65536, k65536);
        }
    }
}

// mcg codebook of two windows -> one packed fp16 pair (first window in the low half):
// hash, halves of both words regrouped (PRMT), mask/xor, fp16(lo + hi) per weight.
__device__ __forceinline__ uint32_t mcg_pair(uint32_t wa, uint32_t wb, uint32_t kxor) {
    const uint32_t pa = wa * 0xCBAC1FEDu, pb = wb * 0xCBAC1FEDu;
    const uint32_t lo = (__byte_perm(pa, pb, 0x5410) & 0x8FFF8FFFu) ^ kxor;
    const uint32_t hi = (__byte_perm(pa, pb, 0x7632) & 0x8FFF8FFFu) ^ kxor;
    const __half2 s = __hadd2(*reinterpret_cast<const __half2 *>(&lo), *reinterpret_cast<const __half2 *>(&hi));
    return *reinterpret_cast<const uint32_t *>(&s);
}

// Columns 2g (bits 0..63 of w) and 2g + 1 (bits 48..111): 16 weights each, k = 0..15,
// as 8 fp16 pairs (k = 2p, 2p + 1).
template <int P>
__device__ __forceinline__ void decode_pairs(const uint32_t (&w)[4], uint32_t k65536, uint32_t kxor, uint32_t (&a)[8],
                                             uint32_t (&b)[8]) {
    a[P] = mcg_pair(window16<6 * P>(w, k65536), window16<6 * P + 3>(w, k65536), kxor);
    b[P] = mcg_pair(window16<48 + 6 * P>(w, k65536), window16<48 + 6 * P + 3>(w, k65536), kxor);
    if constexpr (P < 7) decode_pairs<P + 1>(w, k65536, kxor, a, b);
}

template <bool GATEUP, int NT, int CW>
__global__ void __launch_bounds__(32 * (CW + 1), 1) expert_gemv_exl3(const __grid_constant__ XParams p) {
    using C = XCfg<GATEUP, NT, CW>;
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
            mbar_init(&empty[i], CW);
        }
        *abort = 0;
        fence_mbar_init();
    }
    __syncthreads();
    const int n_items = (*p.n_tiles) * MT;

    if (warp == CW) {
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
                    tma_load_4d(st, ma, &full[s], 0, kr * kKT, nb0, z);
                    if (GATEUP) tma_load_4d(st + kKT * 8 * kTileBytes3, mb, &full[s], 0, kr * kKT, nb0, z);
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
    const int wl = warp & 7, kg = warp >> 3;   // channel block, k group
    const int r0 = 16 * wl;                    // channels r0 + 2g, r0 + 2g + 1 of the 128-channel tile
    // u32 offsets of this thread's 14 trellis bytes inside a tile (word 6g .. 6g+6, circular)
    const int wo0 = 3 * g, wo3 = (3 * g + 3) % 24;
    const uint32_t k65536 = p.k65536, kxor = p.kxor;
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
            for (int pi = 0; pi < C::PQ; ++pi) {
                const int pq = kg * C::PQ + pi;
                const int kt = 4 * pq + c;  // this thread's k-tile in the stage
                const uint8_t *tq = st + C::WBYTES + pq * (C::TOKROWS * 128);
#pragma unroll
                for (int m = 0; m < MATS; ++m) {
                    const uint32_t *tile = reinterpret_cast<const uint32_t *>(
                        st + m * (kKT * 8 * kTileBytes3) + (wl * kKT + kt) * kTileBytes3);
                    const uint32_t w[4] = {tile[wo0], tile[wo0 + 1], tile[wo0 + 2], tile[wo3]};
                    uint32_t wa[8], wb[8];
                    decode_pairs<0>(w, k65536, kxor, wa, wb);
#pragma unroll
                    for (int j = 0; j < NT; ++j) {
                        if (j < ntv) {
                            const int rr = GATEUP ? 2 * (8 * j + g) + m : 8 * j + g;  // token row in the tile
                            const uint4 x0 = *reinterpret_cast<const uint4 *>(tq + rr * 128 + (((2 * c) ^ (rr & 7)) << 4));
                            const uint4 x1 = *reinterpret_cast<const uint4 *>(tq + rr * 128 + (((2 * c + 1) ^ (rr & 7)) << 4));
                            const uint32_t xb[8] = {x0.x, x0.y, x0.z, x0.w, x1.x, x1.y, x1.z, x1.w};
#pragma unroll
                            for (int s4 = 0; s4 < 4; ++s4) {
                                asm("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0, %1, %2, %3}, {%4, %5, %6, "
                                    "%7}, {%8, %9}, {%0, %1, %2, %3};"
                                    : "+f"(acc[m][j][0]), "+f"(acc[m][j][1]), "+f"(acc[m][j][2]), "+f"(acc[m][j][3])
                                    : "r"(wa[2 * s4]), "r"(wb[2 * s4]), "r"(wa[2 * s4 + 1]), "r"(wb[2 * s4 + 1]),
                                      "r"(xb[2 * s4]), "r"(xb[2 * s4 + 1]));
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
        // z -> shared memory [m][token][channel] (k groups summed), then one warp per token:
        // FWHT over the 128 channels, * svh, (gate/up) swiglu, * suh_down, FWHT, store.
        // acc[m][j]: rows g (e 0,1) / g + 8 (e 2,3) = channels r0 + 2g / r0 + 2g + 1,
        // tokens 8j + 2c + (e & 1).
        for (int pass = C::KG - 1; pass >= 0; --pass) {
            if (kg == pass) {
#pragma unroll
                for (int m = 0; m < MATS; ++m)
#pragma unroll
                    for (int j = 0; j < NT; ++j)
#pragma unroll
                        for (int e4 = 0; e4 < 4; ++e4) {
                            const int ch = r0 + 2 * g + (e4 >> 1), tok = 8 * j + 2 * c + (e4 & 1);
                            float *d = &xch[(m * N + tok) * C::XLD + ch];
                            *d = (pass == C::KG - 1) ? acc[m][j][e4] : *d + acc[m][j][e4];
                        }
            }
            asm volatile("bar.sync 1, %0;" ::"r"(32 * CW) : "memory");
        }
        const int e = t.x;
        const bool sh = e == p.E;
        const int ch0 = (item % MT) * 128;
        for (int tok = warp; tok < t.z; tok += CW) {
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
        asm volatile("bar.sync 1, %0;" ::"r"(32 * CW) : "memory");
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

// Trellis stack [experts][K/16][N/16][48 u16] as u32 elements, viewed as 4D
// {24 words, K/16 k-tiles, N/16 column blocks, experts} so that a box of 16 k-tiles x
// 8 column blocks lands in shared memory as [column block][k-tile][96 B].
static int make_trellis_map(CUtensorMap *m, const void *base, int64_t K, int64_t N, int64_t experts, int64_t stride) {
    auto enc = x_encode();
    if (!enc) {
        set_error("cuTensorMapEncodeTiled unavailable from the driver");
        return VFMOE_ERR_CUDA;
    }
    const int64_t row_u32 = (N / 16) * 24;
    if (experts <= 1) stride = (K / 16) * row_u32 * 4;
    cuuint64_t dims[4] = {24, (cuuint64_t)(K / 16), (cuuint64_t)(N / 16), (cuuint64_t)experts};
    cuuint64_t strides[3] = {(cuuint64_t)(row_u32 * 4), (cuuint64_t)kTileBytes3, (cuuint64_t)stride};
    cuuint32_t box[4] = {24, (cuuint32_t)kKT, 8, 1};
    cuuint32_t es[4] = {1, 1, 1, 1};
    CUresult r = enc(m, CU_TENSOR_MAP_DATA_TYPE_UINT32, 4, const_cast<void *>(base), dims, strides, box, es,
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

template <bool GATEUP, int NT, int CW>
static int launch_x(const XParams &prm, int grid, cudaStream_t st) {
    using C = XCfg<GATEUP, NT, CW>;
    static bool attr_done = false;
    if (!attr_done) {
        VF_CUDA(cudaFuncSetAttribute(expert_gemv_exl3<GATEUP, NT, CW>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     C::SMEM));
        attr_done = true;
    }
    expert_gemv_exl3<GATEUP, NT, CW><<<grid, C::THREADS, C::SMEM, st>>>(prm);
    VF_LAUNCH_CHECK(GATEUP ? "expert_gemv_exl3<gate_up>" : "expert_gemv_exl3<down>");
    return VFMOE_OK;
}

int launch_experts_exl3(const Exl3Plan &plan, const MoeArgs &a, const void *x, int x_dtype,
                        cudaStream_t st, const std::function<void()> &mid) {
    const int N = gemv_tokens_per_tile(a.T, a.k, a.E);
    const int64_t rows = (int64_t)a.T * a.k + (a.has_shared ? a.T : 0);  // upper bound
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
    g.k65536 = 65536u;
    g.kxor = 0x3B603B60u;
    const int grid = plan.num_sms;
    switch (N) {
        case 8: rc = launch_x<true, 1, 16>(g, grid, st); break;
        case 16: rc = launch_x<true, 2, 16>(g, grid, st); break;
        default: rc = launch_x<true, 4, 8>(g, grid, st); break;
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
    dn.k65536 = 65536u;
    dn.kxor = 0x3B603B60u;
    switch (N) {
        case 8: return launch_x<false, 1, 16>(dn, grid, st);
        case 16: return launch_x<false, 2, 16>(dn, grid, st);
        default: return launch_x<false, 4, 16>(dn, grid, st);
    }
}

}  // namespace vfmoe
