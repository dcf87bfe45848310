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
template <int BITS>
constexpr int kTileBytes = 32 * BITS;             // 3 bpw: 96 B (48 words), 4 bpw: 128 B (64 words)

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
    pdl_wait_then_release();
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
template <bool GATEUP, int NT, int CW, int BITS>
struct XCfg {
    static constexpr int N = 8 * NT;
    static constexpr int MATS = GATEUP ? 2 : 1;
    static constexpr int KG = CW / 8;                              // k groups
    static constexpr int PQ = 4 / KG;                              // 64-K quarters per warp and stage
    static constexpr int THREADS = 32 * (CW + 1);
    static constexpr int WBYTES = MATS * kKT * 8 * kTileBytes<BITS>;  // trellis per stage
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

// 4 bpw (the reference's format): one output column c of a tile -> 8 fp16 pairs
// (k = 2p, 2p + 1).  The column's 16 windows come from four 32-bit values v_j
// (exl3_col4_pairs); rows 2j + (9, 8, 1, 0)[t] take bits [4t, 4t + 16) of v_j, so pair p
// (rows 2p, 2p + 1) is v_{p & 3} at shifts (12, 8) for p < 4 and (4, 0) otherwise.
__device__ __forceinline__ void decode_col4(const uint32_t *t32, int c, uint32_t kxor, uint32_t *out) {
    uint32_t v[4];
    exl3_col4_pairs(t32, c, v);
#pragma unroll
    for (int p = 0; p < 8; ++p) {
        const uint32_t vj = v[p & 3];
        const int slo = p < 4 ? 12 : 4, shi = p < 4 ? 8 : 0;
        out[p] = mcg_pair((vj >> slo) & 0xFFFFu, (vj >> shi) & 0xFFFFu, kxor);
    }
}

template <bool GATEUP, int NT, int CW, int BITS>
__global__ void __launch_bounds__(32 * (CW + 1), 1) expert_gemv_exl3(const __grid_constant__ XParams p) {
    using C = XCfg<GATEUP, NT, CW, BITS>;
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
    // programmatic dependent launch: the set-up above overlaps the previous kernel; every thread
    // waits for it before reading the tile list or issuing a load of its rows
    griddep_wait();
    if (threadIdx.x == 0) griddep_launch_dependents();
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
                    if (GATEUP) tma_load_4d(st + kKT * 8 * kTileBytes<BITS>, mb, &full[s], 0, kr * kKT, nb0, z);
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
                        st + m * (kKT * 8 * kTileBytes<BITS>) + (wl * kKT + kt) * kTileBytes<BITS>);
                    uint32_t wa[8], wb[8];
                    if constexpr (BITS == 3) {
                        const uint32_t w[4] = {tile[wo0], tile[wo0 + 1], tile[wo0 + 2], tile[wo3]};
                        decode_pairs<0>(w, k65536, kxor, wa, wb);
                    } else {
                        decode_col4(tile, 2 * g, kxor, wa);
                        decode_col4(tile, 2 * g + 1, kxor, wb);
                    }
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

// ----------------------------------------------------------------------------- prefill (tcgen05)
// Many tokens per expert: the trellis of a 128-channel tile is decoded once per tile of up to
// N token rows and fed to tcgen05.mma, as in the Q8_0 tensor-core GEMM (expert_tc.cu):
//   A = decoded Ŵ columns, one output channel per TMEM lane, written with tcgen05.st by 16
//       decode warps (4 sub-stage slots of 64 K in TMEM);
//   B = rotated token rows (fp16, SWIZZLE_128B TMA tiles; gate/up read the gate and the up
//       rotation of each row through a 3D view of the interleaved x_perm);
//   D = fp32 accumulators in TMEM.
// The trellis streams in by TMA as 16 k-tiles x 8 column blocks per matrix and stage (12 KB,
// [column block][k-tile][96 B] as for the decode GEMV).  The epilogue applies the output
// Hadamard across the 128 channels = TMEM lanes: butterflies of stride 1..16 by warp
// shuffles, strides 32 and 64 through shared memory among the four quarter warps of a group.
// Warp roles as expert_tc.cu: 0 TMA, 1 MMA issuer, 2 TMEM allocator, 4..19 decode + epilogue.
// Every mbarrier wait is bounded (2 s).
constexpr int kXtThreads = 640;
constexpr int kXtDq = 16;
constexpr int kXtSA = 4;                           // TMEM A ring slots (64 K each)
constexpr int kXchLd = 9;                          // exchange row stride (floats), 8 columns + pad

template <bool GATEUP, int N, int BITS>
struct XtCfg {
    static constexpr int MATS = GATEUP ? 2 : 1;
    static constexpr int RAW_MAT = kKT * 8 * kTileBytes<BITS>;  // one matrix, one 256-K stage (12 / 16 KB)
    static constexpr int TOK_BOX = N * 128;                 // N rows x 64 K fp16
    static constexpr int TOK_STAGE = MATS * TOK_BOX;        // gate/up: both rotations
    static constexpr int RAW_STAGE = MATS * RAW_MAT;
    static constexpr int XCH = 4 * 128 * kXchLd * 4;        // one [128][9] buffer per epilogue group
    static constexpr int BUDGET = 232448 - 1024 - 256 - XCH;
    static constexpr int SB = kXtSA;  // token stages = TMEM A slots: one full/empty barrier pair per slot
    static constexpr int SW_FIT = (BUDGET - SB * TOK_STAGE) / RAW_STAGE;
    static constexpr int SW = SW_FIT > 4 ? 4 : SW_FIT;
    static constexpr int RAW_BYTES = SW * RAW_STAGE;
    static constexpr int TOK_BYTES = SB * TOK_STAGE;
    static constexpr int XCH_OFF = RAW_BYTES + TOK_BYTES;
    static constexpr int BAR_OFF = XCH_OFF + XCH;
    static constexpr int NBAR = 2 * SW + 2 * kXtSA + 3;
    static constexpr int SMEM = BAR_OFF + NBAR * 8 + 16 + 1024;
    static constexpr int D_COLS = MATS * N;
    static constexpr int A_COL0 = D_COLS;
    static constexpr int DQ_PER_SUB = 4;   // one decode group (four lane-quarter warps) per sub-stage
    static constexpr int TOK_ISSUERS = 1;  // its first warp issues the sub-stage's token loads
    static_assert(SW >= 2, "double-buffered trellis stages");
    static_assert(D_COLS + kXtSA * MATS * 32 <= 512, "TMEM budget");
    static_assert(SMEM <= 232448, "shared memory budget");
};

// Window at bit O of the 64-bit little-endian stream (lo, hi), 16 bits.
template <int O>
__device__ __forceinline__ uint32_t win64(uint32_t lo, uint32_t hi) {
    if constexpr (O == 0) {
        return lo & 0xFFFFu;
    } else if constexpr (O < 32) {
        return __funnelshift_r(lo, hi, O) & 0xFFFFu;
    } else {
        return (hi >> (O - 32)) & 0xFFFFu;
    }
}

// One trellis column c (16 windows at bits [48c, 48c+61) of the tile's circular stream) ->
// 8 fp16 pairs (k = 2p, 2p + 1), decoded exactly as the reference (fp16(lo + hi)).
template <int P>
__device__ __forceinline__ void decode_col(uint32_t lo, uint32_t hi, uint32_t kxor, uint32_t *out) {
    out[P] = mcg_pair(win64<6 * P>(lo, hi), win64<6 * P + 3>(lo, hi), kxor);
    if constexpr (P < 7) decode_col<P + 1>(lo, hi, kxor, out);
}

__device__ __forceinline__ void trellis_column(const uint8_t *tile, int c, uint32_t kxor, uint32_t *out) {
    const uint32_t *tw = reinterpret_cast<const uint32_t *>(tile);
    const int i0 = (3 * c) >> 1;                      // u32 holding u16 word 3c
    const uint32_t a = tw[i0], b = tw[i0 + 1], d = tw[i0 + 2 < 24 ? i0 + 2 : i0 + 2 - 24];
    const uint32_t lo = (c & 1) ? __funnelshift_r(a, b, 16) : a;
    const uint32_t hi = (c & 1) ? __funnelshift_r(b, d, 16) : b;
    decode_col<0>(lo, hi, kxor, out);
}

// 128-point FWHT over the channels of a group's four quarter warps (channel r = 32q + lane),
// for 8 columns per thread.  xb: the group's [128][kXchLd] exchange buffer; bar_id: its
// named barrier (128 threads).
__device__ __forceinline__ void fwht128_lanes(float (&v)[8], float *xb, int q, int lane, int bar_id) {
#pragma unroll
    for (int s = 1; s < 32; s <<= 1) {
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            const float o = __shfl_xor_sync(0xffffffffu, v[j], s);
            v[j] = (lane & s) ? (o - v[j]) : (v[j] + o);
        }
    }
    asm volatile("bar.sync %0, 128;" ::"r"(bar_id) : "memory");  // buffer free
#pragma unroll
    for (int j = 0; j < 8; ++j) xb[(32 * q + lane) * kXchLd + j] = v[j];
    asm volatile("bar.sync %0, 128;" ::"r"(bar_id) : "memory");
#pragma unroll
    for (int j = 0; j < 8; ++j) {
        const float x0 = xb[lane * kXchLd + j], x1 = xb[(32 + lane) * kXchLd + j];
        const float x2 = xb[(64 + lane) * kXchLd + j], x3 = xb[(96 + lane) * kXchLd + j];
        // 4-point Sylvester Hadamard over the stride-32 / stride-64 index bits (q)
        const float s01 = (q & 1) ? (x0 - x1) : (x0 + x1);
        const float s23 = (q & 1) ? (x2 - x3) : (x2 + x3);
        v[j] = (q & 2) ? (s01 - s23) : (s01 + s23);
    }
}

template <bool GATEUP, int N, int BITS>
__global__ void __launch_bounds__(kXtThreads, 1) expert_gemm_exl3_tc(const __grid_constant__ XParams p) {
    using C = XtCfg<GATEUP, N, BITS>;
    constexpr int MATS = C::MATS, SW = C::SW, SB = C::SB;
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t *raw = smem;
    uint8_t *tok = smem + C::RAW_BYTES;
    float *xch = reinterpret_cast<float *>(smem + C::XCH_OFF);
    uint64_t *bars = reinterpret_cast<uint64_t *>(smem + C::BAR_OFF);
    uint64_t *raw_full = bars, *raw_empty = bars + SW;
    uint64_t *full = bars + 2 * SW, *empty = full + kXtSA;
    uint64_t *d_full = empty + kXtSA, *d_empty = d_full + 1, *mma_done = d_full + 2;
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(bars + C::NBAR);
    volatile int *abort = reinterpret_cast<volatile int *>(tmem_slot + 1);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int MT = p.M / 128;
    const int KR = p.K / 256;

    if (threadIdx.x == 0) {
        for (int i = 0; i < SW; ++i) {
            mbar_init(&raw_full[i], MATS);  // one producer thread per matrix (+ tx bytes)
            mbar_init(&raw_empty[i], kXtDq);
        }
        for (int i = 0; i < kXtSA; ++i) {
            mbar_init(&full[i], C::DQ_PER_SUB + C::TOK_ISSUERS);  // decode warps + token loads (+ tx bytes)
            mbar_init(&empty[i], 2);                              // one tcgen05.commit per MMA issuer
        }
        mbar_init(d_full, 2);
        mbar_init(d_empty, kXtDq);
        mbar_init(mma_done, 2);
        *abort = 0;
        fence_mbar_init();
    }
    if (warp == 0 && lane == 0) {
        prefetch_tmap(&p.wa);
        prefetch_tmap(&p.swa);
        prefetch_tmap(&p.xt);
    }
    if (warp == 2) {
        tmem_alloc(tmem_slot, 512);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    const int n_items = (*p.n_tiles) * MT;

    if (warp == 0 || (GATEUP && warp == 3)) {
        // ------------------------------------------------------------------ TMA producers: trellis
        // One thread per matrix (warp 0: gate or down, warp 3: up): a thread sustains only
        // about one TMA load per ~500 clocks.
        if (lane == 0) {
            const int mat = warp == 0 ? 0 : 1;
            uint32_t nraw = 0;
            bool ok = true;
            for (int item = blockIdx.x; item < n_items && ok; item += gridDim.x) {
                const int4 t = p.tiles[item / MT];
                const int nb0 = (item % MT) * 8;
                const bool sh = t.x == p.E;
                const CUtensorMap *mp = mat == 0 ? (sh ? &p.swa : &p.wa) : (sh ? &p.swb : &p.wb);
                const int z = sh ? 0 : t.x;
                for (int kr = 0; kr < KR && ok; ++kr) {
                    const uint32_t rs = nraw % SW;
                    if (!(ok = mbar_wait(&raw_empty[rs], ((nraw / SW) & 1) ^ 1, abort))) break;
                    mbar_arrive_expect_tx(&raw_full[rs], C::RAW_MAT);
                    tma_load_4d(raw + rs * C::RAW_STAGE + mat * C::RAW_MAT, mp, &raw_full[rs], 0, kr * kKT, nb0, z);
                    ++nraw;
                }
            }
            if (!ok) {
                atomicCAS(p.err, 0, DEV_WAIT_TIMEOUT);
                int dummy = 0;
                for (uint32_t i = (nraw > (uint32_t)SW ? nraw - SW : 0); i < nraw; ++i)
                    mbar_wait(&raw_full[i % SW], (i / SW) & 1, (volatile int *)&dummy, 100000000ull);
            }
        }
    } else if (warp == 1 || warp == 2) {
        // ------------------------------------------------------------------ MMA issuers
        // Two issuing threads (gate/up: one per matrix; down: one per half of the token
        // columns), one barrier check and one commit per sub-stage each: every barrier
        // operation in an issuer's instruction stream stalls its next tcgen05.mma.
        if (lane == 0) {
            const int iss = warp - 1;
            uint32_t n = 0, it = 0;
            bool ok = true;
            for (int item = blockIdx.x; item < n_items && ok; item += gridDim.x, ++it) {
                const int n16 = (p.tiles[item / MT].z + 15) >> 4;
                int c_lo = 0, c_n = 16 * n16;
                if (!GATEUP) {
                    const int h0 = 16 * ((n16 + 1) >> 1);
                    c_lo = iss ? h0 : 0;
                    c_n = iss ? 16 * n16 - h0 : h0;
                }
                const int m = GATEUP ? iss : 0;
                const uint32_t idesc = idesc_f16_f32(128, c_n > 0 ? c_n : 16);
                if (!(ok = mbar_wait(d_empty, (it & 1) ^ 1, abort))) break;
                tc_fence_after();
                for (int kr = 0; kr < KR && ok; ++kr) {
                    for (int s = 0; s < 4; ++s) {
                        const uint32_t sl = n % kXtSA;
                        if (!(ok = mbar_wait(&full[sl], (n / kXtSA) & 1, abort))) break;
                        tc_fence_after();
                        if (c_n > 0) {
                            const uint32_t bsm = smem_u32(tok + sl * C::TOK_STAGE + m * C::TOK_BOX + c_lo * 128);
#pragma unroll
                            for (int j = 0; j < 4; ++j) {
                                const uint32_t a_t = tmem + C::A_COL0 + (sl * MATS + m) * 32 + 8 * j;
                                mma_f16_ts(tmem + m * N + c_lo, a_t, smem_desc_sw128(bsm + 32 * j), idesc,
                                           (kr | s | j) != 0);
                            }
                        }
                        mma_commit(&empty[sl]);
                        ++n;
                    }
                }
                if (ok) mma_commit(d_full);
            }
            mma_commit(mma_done);
            int dummy = 0;
            mbar_wait(mma_done, 0, (volatile int *)&dummy, 200000000ull);
            if (!ok) atomicCAS(p.err, 0, DEV_WAIT_TIMEOUT);
        }
    } else if (warp >= 4) {
        // ------------------------------------------------------------------ decode + epilogue
        const int q = warp & 3;            // TMEM lane quarter
        const int grp = (warp - 4) >> 2;   // 0..3
        const int r = 32 * q + lane;       // output channel within the tile = TMEM lane
        const int nb = r >> 4, c = r & 15; // trellis column block and column
        const uint32_t lane_base = (uint32_t)(32 * q) << 16;
        const uint32_t kxor = p.kxor;
        float *xb = xch + grp * 128 * kXchLd;
        // group g decodes sub-stage g of every raw stage: K = 64 of its 32 channels for every
        // matrix (four independent column decodes per thread), and its first warp issues the
        // sub-stage's token loads, one 16-row box per lane in one instruction.
        const bool tok_issuer = q == 0;
        uint32_t nraw = 0, na = 0, it = 0, tok_issued = 0;
        bool ok = true;
        // Epilogue of item `eitem` (the it-th of this CTA): 8-column chunks, chunk c0 handled by
        // group c0/8 % 4 (4 warps = 128 lanes), read from TMEM in batches; the accumulators
        // are released (d_empty) once the last batch is in registers, before its Hadamard
        // transforms and stores, so the next item's MMAs do not wait for them.
        auto epilogue = [&](int eitem, uint32_t eit) -> bool {
            if (!mbar_wait(d_full, eit & 1, abort)) return false;
            tc_fence_after();
            const int4 t = p.tiles[eitem / MT];
            const int e = t.x;
            const bool sh = e == p.E;
            const int ch = (eitem % MT) * 128 + r;
            auto vec = [&](const __half *base, int64_t stride) {
                return reinterpret_cast<const __half *>(reinterpret_cast<const uint8_t *>(base) +
                                                        (sh ? 0 : (int64_t)e * stride));
            };
            const MatrixRef &m0 = sh ? p.sma : p.ma;
            const float svh0 = kRScale * __half2float(vec(m0.svh, m0.svh_stride)[ch]);
            float svh1 = 0.f, suhd = 0.f;
            if (GATEUP) {
                const MatrixRef &m1 = sh ? p.smb : p.mb;
                const MatrixRef &md = sh ? p.smdown : p.mdown;
                svh1 = kRScale * __half2float(vec(m1.svh, m1.svh_stride)[ch]);
                suhd = __half2float(vec(md.suh, md.suh_stride)[ch]);
            }
            constexpr int NCH = (N + 31) / 32;                                     // chunks per group
            constexpr int G = GATEUP ? 1 : (NCH < 4 ? NCH : 4);  // chunks per batch
#pragma unroll
            for (int b0 = 0; b0 < NCH; b0 += G) {
                uint32_t dg[G][8];
                uint32_t du[GATEUP ? G : 1][8];
#pragma unroll
                for (int i = 0; i < G; ++i) {
                    const int c0 = 8 * grp + 32 * (b0 + i);
                    if (c0 < N && c0 < t.z) {
                        tmem_ld_32x32b_x8(tmem + lane_base + c0, dg[i]);
                        if constexpr (GATEUP) tmem_ld_32x32b_x8(tmem + lane_base + N + c0, du[i]);
                    }
                }
                tmem_wait_ld();
                if (b0 + G >= NCH) {
                    tc_fence_before();
                    __syncwarp();
                    if (lane == 0) mbar_arrive(d_empty);
                }
#pragma unroll
                for (int i = 0; i < G; ++i) {
                    const int c0 = 8 * grp + 32 * (b0 + i);
                    if (c0 < N && c0 < t.z) {
                        float vg[8];
#pragma unroll
                        for (int j = 0; j < 8; ++j) vg[j] = __uint_as_float(dg[i][j]);
                        if constexpr (GATEUP) {
                            float vu[8];
#pragma unroll
                            for (int j = 0; j < 8; ++j) vu[j] = __uint_as_float(du[i][j]);
                            fwht128_lanes(vg, xb, q, lane, 1 + grp);
                            fwht128_lanes(vu, xb, q, lane, 1 + grp);
#pragma unroll
                            for (int j = 0; j < 8; ++j)
                                vg[j] = swiglu_clamped(vg[j] * svh0, vu[j] * svh1, p.limit) * suhd;
                            fwht128_lanes(vg, xb, q, lane, 1 + grp);
                            __half *out = reinterpret_cast<__half *>(p.out);
#pragma unroll
                            for (int j = 0; j < 8; ++j)
                                if (c0 + j < t.z)
                                    out[(int64_t)(t.y + c0 + j) * p.ld_out + ch] = __float2half_rn(vg[j] * kRScale);
                        } else {
                            fwht128_lanes(vg, xb, q, lane, 1 + grp);
                            float *out = reinterpret_cast<float *>(p.out);
#pragma unroll
                            for (int j = 0; j < 8; ++j)
                                if (c0 + j < t.z) out[(int64_t)(t.y + c0 + j) * p.ld_out + ch] = vg[j] * svh0;
                        }
                    }
                }
            }
            return true;
        };
        // Item i's epilogue runs after this warp's share of item i+1's first raw stage (whose
        // TMEM slots and token stages item i's last MMAs freed): the next item's first
        // sub-stages are decoded and their token rows in flight while item i's accumulators
        // drain.  Deferring further would deadlock (item i+1's second raw stage needs slots
        // that only item i+1's MMAs free, and those wait for d_empty).
        for (int item = blockIdx.x; item < n_items && ok; item += gridDim.x, ++it) {
            const int4 tt = p.tiles[item / MT];
            const int t_y = tt.y, n16t = (tt.z + 15) >> 4;
            for (int kr = 0; kr < KR && ok; ++kr) {
                const uint32_t rs = nraw % SW;
                if (!(ok = mbar_wait(&raw_full[rs], (nraw / SW) & 1, abort))) break;
#pragma unroll 1
                for (int s = 0; s < 4; ++s) {
                    if (s == grp) {
                        const uint32_t as = na % kXtSA;
                        if (!(ok = mbar_wait(&empty[as], ((na / kXtSA) & 1) ^ 1, abort))) break;
                        if (tok_issuer) {
                            if (lane == 0) mbar_arrive_expect_tx(&full[as], MATS * n16t * 2048);
                            __syncwarp();
                            if (lane < MATS * n16t) {
                                const int m = lane / n16t, b = lane - m * n16t;
                                uint8_t *tdst = tok + as * C::TOK_STAGE + m * C::TOK_BOX + b * 2048;
                                if (GATEUP)
                                    tma_load_3d(tdst, &p.xt, &full[as], kr * 256 + 64 * s, m, t_y + 16 * b);
                                else
                                    tma_load_2d(tdst, &p.xt, &full[as], kr * 256 + 64 * s, t_y + 16 * b);
                            }
                            tok_issued = na + 1;
                        }
#pragma unroll
                        for (int m = 0; m < MATS; ++m) {
                            const uint8_t *stg = raw + rs * C::RAW_STAGE + m * C::RAW_MAT;
                            uint32_t v[32];
#pragma unroll
                            for (int kt = 0; kt < 4; ++kt) {
                                const uint8_t *tl = stg + (nb * kKT + 4 * s + kt) * kTileBytes<BITS>;
                                if constexpr (BITS == 3)
                                    trellis_column(tl, c, kxor, v + 8 * kt);
                                else
                                    decode_col4(reinterpret_cast<const uint32_t *>(tl), c, kxor, v + 8 * kt);
                            }
                            tmem_st_32x32b_x32(tmem + lane_base + C::A_COL0 + (as * MATS + m) * 32, v);
                        }
                        tmem_wait_st();
                        tc_fence_before();
                        __syncwarp();
                        if (lane == 0) mbar_arrive(&full[as]);
                    }
                    ++na;
                }
                if (!ok) break;
                __syncwarp();
                if (lane == 0) mbar_arrive(&raw_empty[rs]);
                ++nraw;
                if (kr == 0 && it > 0 && !(ok = epilogue(item - gridDim.x, it - 1))) break;
            }
        }
        // the last item's epilogue
        if (ok && it > 0) ok = epilogue(blockIdx.x + (it - 1) * gridDim.x, it - 1);
        if (!ok) {
            atomicCAS(p.err, 0, DEV_WAIT_TIMEOUT);
            // token loads this warp issued land before the CTA exits (bounded: the slot's phase
            // also needs the decode arrivals, which may never come after an abort)
            if (tok_issuer && tok_issued > 0) {
                int dummy = 0;
                const uint32_t i = tok_issued - 1;
                mbar_wait(&full[i % kXtSA], (i / kXtSA) & 1, (volatile int *)&dummy, 100000000ull);
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (warp == 2) tmem_dealloc(tmem, 512);
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
static int make_trellis_map(CUtensorMap *m, const void *base, int64_t K, int64_t N, int64_t experts, int64_t stride,
                            int bits) {
    auto enc = x_encode();
    if (!enc) {
        set_error("cuTensorMapEncodeTiled unavailable from the driver");
        return VFMOE_ERR_CUDA;
    }
    const int64_t tile_u32 = 8 * bits;  // 24 (3 bpw) or 32 (4 bpw) words of 32 bits
    const int64_t row_u32 = (N / 16) * tile_u32;
    if (experts <= 1) stride = (K / 16) * row_u32 * 4;
    cuuint64_t dims[4] = {(cuuint64_t)tile_u32, (cuuint64_t)(K / 16), (cuuint64_t)(N / 16), (cuuint64_t)experts};
    cuuint64_t strides[3] = {(cuuint64_t)(row_u32 * 4), (cuuint64_t)(tile_u32 * 4), (cuuint64_t)stride};
    cuuint32_t box[4] = {(cuuint32_t)tile_u32, (cuuint32_t)kKT, 8, 1};
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

// x_perm as [rows][2 rotations][K] fp16 viewed 3D {K, rotation, row}: a box of 64 K x one
// rotation x 16 rows loads one rotation's rows (SWIZZLE_128B).
static int make_rot_map(CUtensorMap *m, const void *base, int64_t rows, int64_t k) {
    auto enc = x_encode();
    if (!enc) {
        set_error("cuTensorMapEncodeTiled unavailable from the driver");
        return VFMOE_ERR_CUDA;
    }
    cuuint64_t dims[3] = {(cuuint64_t)k, 2, (cuuint64_t)rows};
    cuuint64_t strides[2] = {(cuuint64_t)(k * 2), (cuuint64_t)(k * 4)};
    cuuint32_t box[3] = {64, 1, 16};
    cuuint32_t es[3] = {1, 1, 1};
    CUresult r = enc(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3, const_cast<void *>(base), dims, strides, box, es,
                     CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                     CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) {
        set_error("cuTensorMapEncodeTiled (EXL3 rotated rows) failed: %d", (int)r);
        return VFMOE_ERR_CUDA;
    }
    return VFMOE_OK;
}

int exl3_plan_create(const vfmoe_layer_desc &d, Exl3Plan &plan) {
    plan.ready = 0;
    if (d.weight_format != VFMOE_WFMT_EXL3 || (d.exl3_bits != 3 && d.exl3_bits != 4)) return VFMOE_OK;
    plan.bits = (int)d.exl3_bits;
    const int b = plan.bits;
    int dev = 0;
    VF_CUDA(cudaGetDevice(&dev));
    VF_CUDA(cudaDeviceGetAttribute(&plan.num_sms, cudaDevAttrMultiProcessorCount, dev));
    const int64_t H = d.hidden, I = d.inter, E = d.n_local_experts ? d.n_local_experts : d.n_experts;
    int rc;
    if ((rc = make_trellis_map(&plan.gate, (void *)d.gate.data, H, I, E, d.gate.expert_stride, b))) return rc;
    if ((rc = make_trellis_map(&plan.up, (void *)d.up.data, H, I, E, d.up.expert_stride, b))) return rc;
    if ((rc = make_trellis_map(&plan.down, (void *)d.down.data, I, H, E, d.down.expert_stride, b))) return rc;
    const bool sh = d.sh_gate.data != 0;
    if ((rc = make_trellis_map(&plan.sh_gate, (void *)(sh ? d.sh_gate.data : d.gate.data), H, I, 1, 0, b))) return rc;
    if ((rc = make_trellis_map(&plan.sh_up, (void *)(sh ? d.sh_up.data : d.up.data), H, I, 1, 0, b))) return rc;
    if ((rc = make_trellis_map(&plan.sh_down, (void *)(sh ? d.sh_down.data : d.down.data), I, H, 1, 0, b))) return rc;
    plan.ready = 1;
    return VFMOE_OK;
}

template <bool GATEUP, int NT, int CW, int BITS>
static int launch_x1(const XParams &prm, int grid, cudaStream_t st) {
    using C = XCfg<GATEUP, NT, CW, BITS>;
    if (int rc_attr = set_smem_attr_once(reinterpret_cast<const void *>(expert_gemv_exl3<GATEUP, NT, CW, BITS>), C::SMEM)) return rc_attr;
    VF_CUDA(launch_pdl(expert_gemv_exl3<GATEUP, NT, CW, BITS>, dim3(grid), dim3(C::THREADS), (size_t)C::SMEM, st, prm));
    VF_LAUNCH_CHECK(GATEUP ? "expert_gemv_exl3<gate_up>" : "expert_gemv_exl3<down>");
    return VFMOE_OK;
}

template <bool GATEUP, int NT, int CW>
static int launch_x(const XParams &prm, int bits, int grid, cudaStream_t st) {
    return bits == 4 ? launch_x1<GATEUP, NT, CW, 4>(prm, grid, st) : launch_x1<GATEUP, NT, CW, 3>(prm, grid, st);
}

template <bool GATEUP, int N, int BITS>
static int launch_xt1(const XParams &prm, int grid, cudaStream_t st) {
    using C = XtCfg<GATEUP, N, BITS>;
    if (int rc_attr = set_smem_attr_once(reinterpret_cast<const void *>(expert_gemm_exl3_tc<GATEUP, N, BITS>), C::SMEM)) return rc_attr;
    expert_gemm_exl3_tc<GATEUP, N, BITS><<<grid, kXtThreads, C::SMEM, st>>>(prm);
    VF_LAUNCH_CHECK(GATEUP ? "expert_gemm_exl3_tc<gate_up>" : "expert_gemm_exl3_tc<down>");
    return VFMOE_OK;
}

template <bool GATEUP, int N>
static int launch_xt(const XParams &prm, int bits, int grid, cudaStream_t st) {
    return bits == 4 ? launch_xt1<GATEUP, N, 4>(prm, grid, st) : launch_xt1<GATEUP, N, 3>(prm, grid, st);
}

// Prefill (more than 16 rows per expert on average): gather + tile plan + tcgen05 GEMMs with
// 128-row gate/up tiles and 256-row down tiles.
static int launch_exl3_tc(const Exl3Plan &plan, const MoeArgs &a, cudaStream_t st, const std::function<void()> &mid) {
    const int64_t cap_rows = (int64_t)a.T * a.k + a.T;
    int rc;
    XParams g{};
    g.wa = plan.gate;
    g.wb = plan.up;
    g.swa = plan.sh_gate;
    g.swb = plan.sh_up;
    if ((rc = make_rot_map(&g.xt, a.xp, cap_rows, a.H))) return rc;
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
    g.kxor = 0x3B603B60u;
    const int grid = plan.num_sms;
    if ((rc = launch_xt<true, 128>(g, plan.bits, grid, st))) return rc;
    mid();
    XParams dn{};
    dn.wa = plan.down;
    dn.wb = plan.down;
    dn.swa = plan.sh_down;
    dn.swb = plan.sh_down;
    if ((rc = make_rows_map(&dn.xt, a.act, cap_rows, a.I, 16))) return rc;
    dn.tiles = a.tiles + a.tiles_cap;
    dn.n_tiles = a.tile_counts + 1;
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
    dn.kxor = 0x3B603B60u;
    return launch_xt<false, 256>(dn, plan.bits, grid, st);
}

int launch_experts_exl3(const Exl3Plan &plan, const MoeArgs &a, const void *x, int x_dtype,
                        cudaStream_t st, const std::function<void()> &mid) {
    const bool prefill = (double)a.T * a.k / a.E > 16.0;
    const int N = gemv_tokens_per_tile(a.T, a.k, a.E);
    const int64_t rows = (int64_t)a.T * a.k + (a.has_shared ? a.T : 0);  // upper bound
    int rc = prefill ? launch_tc_plan(a, 128, 256, st) : launch_tc_plan(a, N, N, st);
    if (rc) return rc;
    if (rows > 0) {
        VF_CUDA(launch_pdl(gather_exl3_kernel, dim3((unsigned)rows), dim3(256), 0, st, x, x_dtype, a.perm_tok,
                           (const int32_t *)a.offsets, a.E + (a.has_shared ? 1 : 0), a.E, a.H, a.gate, a.up, a.sh_gate,
                           a.sh_up, const_cast<__half *>(a.xp)));
        VF_LAUNCH_CHECK("gather_exl3_kernel");
    }
    if (prefill) return launch_exl3_tc(plan, a, st, mid);
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
        case 8: rc = launch_x<true, 1, 16>(g, plan.bits, grid, st); break;
        case 16: rc = launch_x<true, 2, 16>(g, plan.bits, grid, st); break;
        default: rc = launch_x<true, 4, 8>(g, plan.bits, grid, st); break;
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
        case 8: return launch_x<false, 1, 16>(dn, plan.bits, grid, st);
        case 16: return launch_x<false, 2, 16>(dn, plan.bits, grid, st);
        default: return launch_x<false, 4, 16>(dn, plan.bits, grid, st);
    }
}

}  // namespace vfmoe
