// Grouped expert GEMMs on the 5th-generation tensor cores (tcgen05), Q8_0 weights.
//
// One persistent kernel serves the decode and the prefill shapes (N = tokens per tile):
//   gate/up:  act[rows, ch] = fp16(swiglu(x . Wg[ch], x . Wu[ch]))  (moe.vyb:98-134)
//   down:     y[rows, ch]   = act . Wd[ch]                          (moe.vyb:137-170)
//
// Operand placement (per CTA tile of 128 output channels x N token rows):
//   A = weights, M = 128 channels, dequantized Q8_0 -> fp16 by 8 "dequant" warps and
//       written straight into TMEM with tcgen05.st (no shared-memory round trip);
//   B = token rows (fp16), N x 64 per sub-stage, TMA SWIZZLE_128B tiles in shared memory;
//   D = fp32 accumulators in TMEM (gate and up side by side for the fused SwiGLU).
// Raw Q8_0 bytes stream in as 128 rows x 272 B (8 GGUF blocks = 256 K) per stage: one TMA
// box from GGUF rows, or two contiguous bulk copies from stage-tiled weights.
//
// Warp roles (640 threads): warps 0 and 3 TMA producers of the weight stages (one matrix
// each), warps 1 and 2 MMA issuers (one thread each; warp 2 also allocates TMEM), warps
// 4..19 dequant + epilogue; the first warp of each dequant group also issues its sub-stage's
// token-row loads (one 16-row box per lane).  Dequant warp w owns TMEM lanes 32*(w%4)..+31
// (= weight rows of the tile) and belongs to group g = (w-4)/4, which converts sub-stage g of
// every raw stage (each raw stage holds 4 sub-stages of K = 64), for both matrices of
// gate/up.  A group therefore has four sub-stages of MMA time to fill its TMEM slot.
// Sub-stage slot i has one "full" barrier (its dequant group's four warps + the token TMA
// bytes) and one "empty" barrier (one commit per issuer), so an issuer checks one barrier
// and commits once per sub-stage: each barrier operation in an issuer's instruction stream
// stalls its next tcgen05.mma, and a single issuer with two waits and two commits per
// sub-stage kept the tensor pipe under 60 % busy even with all data in place.
// A work item's epilogue runs after the dequant warps' share of their next item's first raw
// stage and releases the accumulators as soon as they are read into registers, so the MMAs
// of the next item start with four sub-stages converted and their token rows landed.
// Every mbarrier wait is bounded (2 s); on expiry the CTA raises DEV_WAIT_TIMEOUT,
// drains what it issued and returns.
//
// Work list: the (expert, token-tile) list built on the device by tc_plan_kernel, times
// the M/128 channel tiles, strided over a grid of one CTA per SM.
#include <cudaTypedefs.h>

#include <algorithm>
#include <cstdlib>
#include <mutex>

#include "expert_tc.h"
#include "sm100.cuh"

namespace vfmoe {

using namespace sm100;

constexpr int kThreads = 640;
constexpr int kDqWarps = 16;
constexpr int kRawRow = 272;            // 8 Q8_0 blocks = 256 K values
constexpr int kRawMat = 128 * kRawRow;  // one matrix, one stage
constexpr int kSlots = 4;               // sub-stage ring (K = 64 each): TMEM A slots + token stages

template <bool GATEUP, int N>
struct TcCfg {
    static constexpr int MATS = GATEUP ? 2 : 1;
    static constexpr int SW = GATEUP ? (N <= 32 ? 3 : 2) : (N <= 32 ? 5 : (N == 64 ? 4 : (N == 128 ? 3 : 2)));
    static constexpr int RAW_BYTES = SW * MATS * kRawMat;
    static constexpr int TOK_STAGE = N * 128;
    static constexpr int TOK_BYTES = kSlots * TOK_STAGE;
    static constexpr int BAR_OFF = RAW_BYTES + TOK_BYTES;
    static constexpr int NBAR = 2 * SW + 2 * kSlots + 3;
    static constexpr int SMEM = BAR_OFF + NBAR * 8 + 16 + 1024;  // + alignment slack
    static constexpr int D_COLS = MATS * N;
    static constexpr int A_COL0 = D_COLS;
    static_assert(D_COLS + kSlots * MATS * 32 <= 512, "TMEM budget");
    static_assert(SMEM <= 232448, "shared memory budget");
};

// ----------------------------------------------------------------------------- dequant
// 68 bytes = two Q8_0 blocks (K = 64) of one weight row -> 32 packed fp16 pairs
// (column c holds k = 2c in the low half, 2c + 1 in the high half), value fp16(d * q).
// g[0..16] are the 17 little-endian words of the two blocks.
__device__ __forceinline__ uint32_t q8_pair(uint32_t word, uint32_t sel, __half2 d2) {
    const uint32_t h = __byte_perm(word, 0x64646464u, sel);  // {0x64, q_hi, 0x64, q_lo}: 1024 + (q ^ 0x80)
    __half2 v = *reinterpret_cast<const __half2 *>(&h);
    v = __hsub2(v, __half2half2(__ushort_as_half(0x6480)));  // - 1152 -> exact q
    v = __hmul2(v, d2);                                      // one rounding: fp16(d * q)
    return *reinterpret_cast<const uint32_t *>(&v);
}

__device__ __forceinline__ void q8_two_blocks(const uint32_t (&g)[17], uint32_t (&v)[32]) {
    const __half2 d0 = __half2half2(__ushort_as_half((unsigned short)(g[0] & 0xFFFFu)));
    const __half2 d1 = __half2half2(__ushort_as_half((unsigned short)(g[8] >> 16)));
    uint32_t x[17];
    x[0] = g[0] ^ 0x80800000u;
#pragma unroll
    for (int i = 1; i < 8; ++i) x[i] = g[i] ^ 0x80808080u;
    x[8] = g[8] ^ 0x00008080u;
#pragma unroll
    for (int i = 9; i < 17; ++i) x[i] = g[i] ^ 0x80808080u;
    // block 0: pair c = bytes 2+2c, 3+2c of the group
#pragma unroll
    for (int c = 0; c < 16; ++c) {
        const int b = 2 + 2 * c;
        v[c] = q8_pair(x[b >> 2], (b & 3) ? 0x4342u : 0x4140u, d0);
    }
    // block 1: pair c = bytes 36+2c, 37+2c
#pragma unroll
    for (int c = 0; c < 16; ++c) {
        const int b = 36 + 2 * c;
        v[16 + c] = q8_pair(x[b >> 2], (b & 3) ? 0x4342u : 0x4140u, d1);
    }
}

// ----------------------------------------------------------------------------- plan
// Token tiles of at most N rows for every expert segment (routed experts ascending, then
// shared); an expert's rows are split into equal-size tiles.
__global__ void __launch_bounds__(1024) tc_plan_kernel(const int32_t *__restrict__ offsets, int E, int has_shared,
                                                       int n_gu, int n_dn, int4 *__restrict__ tiles, int64_t cap,
                                                       int32_t *__restrict__ counts, int *__restrict__ err) {
    __shared__ int wsum[2][32];
    pdl_wait_then_release();
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int nexp = E + (has_shared ? 1 : 0);
    const int per = (nexp + 1023) / 1024;  // each thread owns experts [tid*per, (tid+1)*per)
    const int Ns[2] = {n_gu, n_dn};
    // tiles of this thread's experts for both lists, then one block-wide exclusive scan of both
    // (warp shuffles; the 32 warp totals are scanned by warp 0)
    int mine[2] = {0, 0};
    for (int i = 0; i < per; ++i) {
        const int e = tid * per + i;
        if (e < nexp) {
            const int n = offsets[e + 1] - offsets[e];
            mine[0] += (n + Ns[0] - 1) / Ns[0];
            mine[1] += (n + Ns[1] - 1) / Ns[1];
        }
    }
    int inc[2] = {mine[0], mine[1]};
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
#pragma unroll
        for (int l = 0; l < 2; ++l) {
            const int v = __shfl_up_sync(0xffffffffu, inc[l], o);
            if (lane >= o) inc[l] += v;
        }
    }
    if (lane == 31) {
        wsum[0][warp] = inc[0];
        wsum[1][warp] = inc[1];
    }
    __syncthreads();
    if (warp == 0) {
#pragma unroll
        for (int l = 0; l < 2; ++l) {
            int v = wsum[l][lane];
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const int u = __shfl_up_sync(0xffffffffu, v, o);
                if (lane >= o) v += u;
            }
            wsum[l][lane] = v;  // inclusive over warps
        }
    }
    __syncthreads();
#pragma unroll
    for (int l = 0; l < 2; ++l) {
        const int N = Ns[l];
        int4 *out = tiles + l * cap;
        int pos = inc[l] - mine[l] + (warp > 0 ? wsum[l][warp - 1] : 0);
        for (int i = 0; i < per; ++i) {
            const int e = tid * per + i;
            if (e < nexp) {
                // ceil(n / N) tiles of near-equal size (no mostly-empty tail tile)
                const int r0 = offsets[e], n = offsets[e + 1] - r0;
                const int nt = (n + N - 1) / N;
                int row = r0;
                for (int j = 0; j < nt; ++j) {
                    const int rows = n / nt + (j < n % nt ? 1 : 0);
                    if (pos < cap) out[pos] = make_int4(e, row, rows, 0);
                    row += rows;
                    ++pos;
                }
            }
        }
        if (tid == 0) {
            const int tot = wsum[l][31];
            counts[l] = (int32_t)(tot < cap ? tot : cap);
            if (tot > cap) raise_dev_error(err, DEV_BAD_COUNT);
        }
    }
}

// ----------------------------------------------------------------------------- GEMM
template <bool GATEUP, int N>
__global__ void __launch_bounds__(kThreads, 1) expert_gemm_tc(const __grid_constant__ TcParams p) {
    using C = TcCfg<GATEUP, N>;
    constexpr int MATS = C::MATS, SW = C::SW;
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t *raw = smem;
    uint8_t *tok = smem + C::RAW_BYTES;
    uint64_t *bars = reinterpret_cast<uint64_t *>(smem + C::BAR_OFF);
    uint64_t *raw_full = bars, *raw_empty = bars + SW;
    uint64_t *full = bars + 2 * SW, *empty = full + kSlots;
    uint64_t *d_full = empty + kSlots, *d_empty = d_full + 1, *mma_done = d_full + 2;
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(bars + C::NBAR);
    volatile int *abort = reinterpret_cast<volatile int *>(tmem_slot + 1);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int MT = p.M / 128;
    const int KR = p.K / 256;

    if (threadIdx.x == 0) {
        for (int i = 0; i < SW; ++i) {
            mbar_init(&raw_full[i], MATS);  // one producer thread per matrix (+ tx bytes)
            mbar_init(&raw_empty[i], kDqWarps);
        }
        for (int i = 0; i < kSlots; ++i) {
            mbar_init(&full[i], 4 + 1);  // the four warps of one dequant group + its token loads (+ tx bytes)
            mbar_init(&empty[i], 2);     // one tcgen05.commit per MMA issuer
        }
        mbar_init(d_full, 2);
        mbar_init(d_empty, kDqWarps);
        mbar_init(mma_done, 2);
        *abort = 0;
        fence_mbar_init();
    }
    if (warp == 0 && lane == 0) {
        prefetch_tmap(&p.xt);
        if (!p.tiled) {
            prefetch_tmap(&p.wa);
            prefetch_tmap(&p.swa);
            if (GATEUP) {
                prefetch_tmap(&p.wb);
                prefetch_tmap(&p.swb);
            }
        }
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
        // ------------------------------------------------------------------ TMA producers: weights
        // One thread per matrix (warp 0: A / gate or down, warp 3: B / up): a thread sustains
        // only about one TMA load per ~500 clocks however many it has in flight, so the two
        // matrices' loads are issued from different threads.
        if (lane == 0) {
            const int mat = warp == 0 ? 0 : 1;
            uint32_t nraw = 0;
            bool ok = true;
            for (int item = blockIdx.x; item < n_items && ok; item += gridDim.x) {
                const int4 t = p.tiles[item / MT];
                const int m0 = (item % MT) * 128;
                const bool sh = t.x == p.E;
                const CUtensorMap *mp = mat == 0 ? (sh ? &p.swa : &p.wa) : (sh ? &p.swb : &p.wb);
                const int z = sh ? 0 : t.x;
                for (int kr = 0; kr < KR && ok; ++kr) {
                    const uint32_t rs = nraw % SW;
                    if (!(ok = mbar_wait(&raw_empty[rs], ((nraw / SW) & 1) ^ 1, abort))) break;
                    mbar_arrive_expect_tx(&raw_full[rs], kRawMat);
                    uint8_t *dst = raw + rs * (MATS * kRawMat) + mat * kRawMat;
                    if (p.tiled)
                        load_q8_tiled(dst, mat == 0 ? (sh ? p.spa : p.pa) : (sh ? p.spb : p.pb), mat == 0 ? p.sa : p.sb,
                                      z, m0, 128, KR, kr, &raw_full[rs]);
                    else
                        tma_load_3d(dst, mp, &raw_full[rs], kr * (kRawRow / 2), m0, z);
                    ++nraw;
                }
            }
            if (!ok) {
                // drain copies still in flight before the CTA exits (bounded)
                atomicCAS(p.err, 0, DEV_WAIT_TIMEOUT);
                int dummy = 0;
                for (uint32_t i = (nraw > (uint32_t)SW ? nraw - SW : 0); i < nraw; ++i)
                    mbar_wait(&raw_full[i % SW], (i / SW) & 1, (volatile int *)&dummy, 100000000ull);
            }
        }
    } else if (warp == 1 || warp == 2) {
        // ------------------------------------------------------------------ MMA issuers
        // Two issuing threads keep the tensor pipe fed: every barrier check in an issuer's
        // instruction stream stalls its next MMA.  Gate/up: issuer i owns matrix i.  Down:
        // issuer i owns one half of the token columns (in 16-column units).
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
                const int mat = GATEUP ? iss : 0;
                const uint32_t idesc = idesc_f16_f32(128, c_n > 0 ? c_n : 16);
                if (!(ok = mbar_wait(d_empty, (it & 1) ^ 1, abort))) break;
                tc_fence_after();
                for (int kr = 0; kr < KR && ok; ++kr) {
                    for (int s = 0; s < 4; ++s) {
                        const uint32_t sl = n % kSlots;
                        if (!(ok = mbar_wait(&full[sl], (n / kSlots) & 1, abort))) break;
                        tc_fence_after();
                        if (c_n > 0) {
                            const uint32_t bsm = smem_u32(tok + sl * C::TOK_STAGE + c_lo * 128);
#pragma unroll
                            for (int j = 0; j < 4; ++j) {
                                const uint32_t a_t = tmem + C::A_COL0 + (sl * MATS + mat) * 32 + 8 * j;
                                mma_f16_ts(tmem + mat * N + c_lo, a_t, smem_desc_sw128(bsm + 32 * j), idesc,
                                           (kr | s | j) != 0);
                            }
                        }
                        mma_commit(&empty[sl]);
                        ++n;
                    }
                }
                if (ok) mma_commit(d_full);
            }
            // all issued MMAs complete before TMEM is released
            mma_commit(mma_done);
            int dummy = 0;
            mbar_wait(mma_done, 0, (volatile int *)&dummy, 200000000ull);
            if (!ok) atomicCAS(p.err, 0, DEV_WAIT_TIMEOUT);
        }
    } else if (warp >= 4) {
        // ------------------------------------------------------------------ dequant + epilogue
        const int q = warp & 3;            // TMEM lane quarter
        const int grp = (warp - 4) >> 2;   // 0..3
        const int r = 32 * q + lane;       // weight row within the tile = TMEM lane
        const uint32_t lane_base = (uint32_t)(32 * q) << 16;
        uint32_t nraw = 0, n = 0, it = 0;
        bool ok = true;
        uint32_t tok_issued = 0;  // sub-stages whose token loads this warp issued
        // Epilogue of item `eitem` (the it-th of this CTA): 8-column chunks of the N token
        // columns, chunk c handled by group c % 4, read from TMEM in batches of 32 registers.
        // The accumulators are released (d_empty) once the last batch is in registers, before
        // its SwiGLU and stores, so the next item's MMAs do not wait for them.
        auto epilogue = [&](int eitem, uint32_t eit) -> bool {
            if (!mbar_wait(d_full, eit & 1, abort)) return false;
            tc_fence_after();
            const int4 t = p.tiles[eitem / MT];
            const int ch = (eitem % MT) * 128 + r;
            constexpr int NCH = (N + 31) / 32;                     // chunks per group
            constexpr int G = GATEUP ? 1 : (NCH < 4 ? NCH : 4);  // chunks per batch (register budget)
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
                        if constexpr (GATEUP) {
                            __half *out = reinterpret_cast<__half *>(p.out);
#pragma unroll
                            for (int j = 0; j < 8; ++j) {
                                if (c0 + j < t.z) {
                                    const float a = swiglu_clamped_fast(__uint_as_float(dg[i][j]),
                                                                   __uint_as_float(du[i][j]), p.limit);
                                    out[(int64_t)(t.y + c0 + j) * p.ld_out + ch] = __float2half_rn(a);
                                }
                            }
                        } else {
                            float *out = reinterpret_cast<float *>(p.out);
#pragma unroll
                            for (int j = 0; j < 8; ++j)
                                if (c0 + j < t.z)
                                    out[(int64_t)(t.y + c0 + j) * p.ld_out + ch] = __uint_as_float(dg[i][j]);
                        }
                    }
                }
            }
            return true;
        };
        // Item i's epilogue runs after this warp's share of item i+1's first raw stage.  That
        // share's TMEM slots and token stages were freed by item i's last MMAs, so the next
        // item's first sub-stages are converted and their token rows in flight while item i's
        // accumulators drain.  Deferring further would deadlock: item i+1's second raw stage
        // needs slots that only item i+1's MMAs free, and those wait for d_empty.
        for (int item = blockIdx.x; item < n_items && ok; item += gridDim.x, ++it) {
            const int4 tt = p.tiles[item / MT];
            const int t_y = tt.y, n16 = (tt.z + 15) >> 4;  // 16-row token boxes actually needed
            for (int kr = 0; kr < KR && ok; ++kr) {
                const uint32_t rs = nraw % SW;
                if (!(ok = mbar_wait(&raw_full[rs], (nraw / SW) & 1, abort))) break;
                const uint8_t *row = raw + rs * (MATS * kRawMat) + r * kRawRow;
#pragma unroll
                for (int s = 0; s < 4; ++s) {
                    if (s == grp) {
                        // group g converts sub-stage g of every raw stage: K = 64 (two Q8_0
                        // blocks) of its 32 rows, for each matrix.  The warp reads its raw
                        // words into registers and releases the raw stage, and converts the
                        // first matrix, before it waits for its TMEM slot: the stage's lifetime
                        // is its load latency plus four reads, and after the slot frees only
                        // one conversion is left before the MMAs can use it.
                        auto load_words = [&](int m, uint32_t (&w)[20]) {
#pragma unroll
                            for (int c = 0; c < 5; ++c) {
                                const uint4 v4 =
                                    *reinterpret_cast<const uint4 *>(row + m * kRawMat + 64 * s + 16 * c);
                                w[4 * c] = v4.x;
                                w[4 * c + 1] = v4.y;
                                w[4 * c + 2] = v4.z;
                                w[4 * c + 3] = v4.w;
                            }
                        };
                        auto convert = [&](const uint32_t (&w)[20], uint32_t (&v)[32]) {
                            uint32_t g[17];
#pragma unroll
                            for (int j = 0; j < 17; ++j) g[j] = w[s + j];
                            q8_two_blocks(g, v);
                        };
                        uint32_t w0[20], w1[20], v[32];
                        load_words(0, w0);
                        if (GATEUP) load_words(1, w1);
                        __syncwarp();
                        if (lane == 0) mbar_arrive(&raw_empty[rs]);
                        convert(w0, v);
                        const uint32_t sl = n % kSlots;
                        if (!(ok = mbar_wait(&empty[sl], ((n / kSlots) & 1) ^ 1, abort))) break;
                        if (q == 0) {
                            // the group's token rows for this sub-stage: one 16-row box per lane,
                            // all issued by one instruction
                            if (lane == 0) mbar_arrive_expect_tx(&full[sl], n16 * 16 * 128);
                            __syncwarp();
                            if (lane < n16)
                                tma_load_2d(tok + sl * C::TOK_STAGE + lane * 2048, &p.xt, &full[sl], kr * 256 + 64 * s,
                                            t_y + 16 * lane);
                            tok_issued = n + 1;
                        }
                        const uint32_t tcol = tmem + lane_base + C::A_COL0 + sl * MATS * 32;
                        tmem_st_32x32b_x32(tcol, v);
                        if (GATEUP) {
                            convert(w1, v);
                            tmem_st_32x32b_x32(tcol + 32, v);
                        }
                        tmem_wait_st();
                        tc_fence_before();
                        __syncwarp();
                        if (lane == 0) mbar_arrive(&full[sl]);
                    }
                    ++n;
                }
                if (!ok) break;
                ++nraw;
                if (kr == 0 && it > 0 && !(ok = epilogue(item - gridDim.x, it - 1))) break;
            }
        }
        // the last item's epilogue
        if (ok && it > 0) ok = epilogue(blockIdx.x + (it - 1) * gridDim.x, it - 1);
        if (!ok) {
            atomicCAS(p.err, 0, DEV_WAIT_TIMEOUT);
            // token loads this warp issued land before the CTA exits (bounded: the slot's phase
            // also needs the dequant arrivals, which may never come after an abort)
            if (q == 0 && tok_issued > 0) {
                int dummy = 0;
                const uint32_t i = tok_issued - 1;
                mbar_wait(&full[i % kSlots], (i / kSlots) & 1, (volatile int *)&dummy, 100000000ull);
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (warp == 2) tmem_dealloc(tmem, 512);
}

// ----------------------------------------------------------------------------- GEMM over CTA pairs
// The same grouped GEMM with every work item spread over a cluster of two CTAs on two SMs
// (tcgen05 cta_group::2).  A pair covers 256 output channels x N token rows: each CTA converts
// and holds (TMEM) its own 128 weight rows and accumulators, and loads half of the token rows
// (N / 2, shared memory); one thread of the even CTA issues every MMA with M = 256.  Each MMA and
// each barrier operation of an issuer thus carries twice the work of the single-CTA kernel,
// whose issuers' per-instruction cost was the limit (about 860 clocks per 64-K sub-stage where
// the tensor pipe needs 512).  D column j is token j of the tile: the MMA takes B columns
// [0, N/2) from the even CTA's shared memory and [N/2, N) from the odd CTA's.
// Cross-CTA barriers (all in the even CTA unless noted): a sub-stage's "full" barrier counts both
// CTAs' dequant warps and token-load bytes; the accumulator "empty" barrier counts both CTAs'
// epilogue warps; the issuers' commits arrive on the "empty" and accumulator "full" barriers of
// both CTAs (multicast commit).  Weight stages (raw_full / raw_empty) stay per CTA.  Every
// mbarrier wait is bounded; the two cluster barriers (after set-up, before TMEM release) are
// reached by every thread of both CTAs on every path.  No load uses multicast.
template <bool GATEUP, int N>
struct TcPairCfg {
    static constexpr int MATS = GATEUP ? 2 : 1;
    static constexpr int NH = N / 2;                // token rows per CTA and sub-stage
    static constexpr int TOK_STAGE = NH * 128;
    static constexpr int TOK_BYTES = kSlots * TOK_STAGE;
    static constexpr int SW_FIT = (225000 - TOK_BYTES - 2048) / (MATS * kRawMat);
    static constexpr int SW = SW_FIT > 5 ? 5 : SW_FIT;
    static constexpr int RAW_BYTES = SW * MATS * kRawMat;
    static constexpr int BAR_OFF = RAW_BYTES + TOK_BYTES;
    static constexpr int NBAR = 2 * SW + 2 * kSlots + 3;
    static constexpr int SMEM = BAR_OFF + NBAR * 8 + 16 + 1024;
    static constexpr int ISSUERS = GATEUP ? 2 : 1;  // gate/up: one per matrix; down: one
    static constexpr int D_COLS = MATS * N;
    static constexpr int A_COL0 = D_COLS;
    static_assert(N % 32 == 0 && N >= 32 && N <= 256, "pair MMA: N a multiple of 32 in [32, 256]");
    static_assert(D_COLS + kSlots * MATS * 32 <= 512, "TMEM budget");
    static_assert(SW >= 2, "at least two weight stages");
    static_assert(TOK_STAGE % 1024 == 0 && (MATS * kRawMat) % 1024 == 0, "1024-byte aligned token stages");
    static_assert(SMEM <= 232448, "shared memory budget");
};

template <bool GATEUP, int N>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kThreads, 1)
    expert_gemm_tc_pair(const __grid_constant__ TcParams p) {
    using C = TcPairCfg<GATEUP, N>;
    constexpr int MATS = C::MATS, SW = C::SW;
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t *raw = smem;
    uint8_t *tok = smem + C::RAW_BYTES;
    uint64_t *bars = reinterpret_cast<uint64_t *>(smem + C::BAR_OFF);
    uint64_t *raw_full = bars, *raw_empty = bars + SW;
    uint64_t *full = bars + 2 * SW, *empty = full + kSlots;
    uint64_t *d_full = empty + kSlots, *d_empty = d_full + 1, *mma_done = d_full + 2;
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(bars + C::NBAR);
    volatile int *abort = reinterpret_cast<volatile int *>(tmem_slot + 1);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t rank = cluster_ctarank();
    const int cid = (int)cluster_id_x(), ncl = (int)cluster_count_x();
    const int MT = p.M / 256;
    const int KR = p.K / 256;

    if (threadIdx.x == 0) {
        for (int i = 0; i < SW; ++i) {
            mbar_init(&raw_full[i], MATS);
            mbar_init(&raw_empty[i], kDqWarps);
        }
        for (int i = 0; i < kSlots; ++i) {
            mbar_init(&full[i], 2 * (4 + 1));  // both CTAs: a dequant group's four warps + its token loads
            mbar_init(&empty[i], C::ISSUERS);  // one commit per issuer (arrives in both CTAs)
        }
        mbar_init(d_full, C::ISSUERS);
        mbar_init(d_empty, 2 * kDqWarps);      // both CTAs' epilogue warps
        mbar_init(mma_done, C::ISSUERS);
        *abort = 0;
        fence_mbar_init();
    }
    if (warp == 0 && lane == 0) {
        prefetch_tmap(&p.xt);
        if (!p.tiled) {
            prefetch_tmap(&p.wa);
            prefetch_tmap(&p.swa);
            if (GATEUP) {
                prefetch_tmap(&p.wb);
                prefetch_tmap(&p.swb);
            }
        }
    }
    if (warp == 2) {
        tmem_alloc_pair(tmem_slot, 512);
        tmem_relinquish_pair();
    }
    tc_fence_before();
    cluster_sync_all();  // both CTAs' barriers initialised and TMEM allocated before any cross-CTA use
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    const int n_items = (*p.n_tiles) * MT;
    const uint32_t full0 = mapa_shared(full, 0);      // the even CTA's full[i] at full0 + 8 i
    const uint32_t d_empty0 = mapa_shared(d_empty, 0);

    if (warp == 0 || (GATEUP && warp == 3)) {
        // ------------------------------------------------------------------ TMA producers: this CTA's weight rows
        if (lane == 0) {
            const int mat = warp == 0 ? 0 : 1;
            uint32_t nraw = 0;
            bool ok = true;
            for (int item = cid; item < n_items && ok; item += ncl) {
                const int4 t = p.tiles[item / MT];
                const int m0 = (item % MT) * 256 + 128 * (int)rank;
                const bool sh = t.x == p.E;
                const CUtensorMap *mp = mat == 0 ? (sh ? &p.swa : &p.wa) : (sh ? &p.swb : &p.wb);
                const int z = sh ? 0 : t.x;
                for (int kr = 0; kr < KR && ok; ++kr) {
                    const uint32_t rs = nraw % SW;
                    if (!(ok = mbar_wait(&raw_empty[rs], ((nraw / SW) & 1) ^ 1, abort))) break;
                    mbar_arrive_expect_tx(&raw_full[rs], kRawMat);
                    uint8_t *dst = raw + rs * (MATS * kRawMat) + mat * kRawMat;
                    if (p.tiled)
                        load_q8_tiled(dst, mat == 0 ? (sh ? p.spa : p.pa) : (sh ? p.spb : p.pb), mat == 0 ? p.sa : p.sb,
                                      z, m0, 128, KR, kr, &raw_full[rs]);
                    else
                        tma_load_3d(dst, mp, &raw_full[rs], kr * (kRawRow / 2), m0, z);
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
    } else if (warp == 1 || (GATEUP && warp == 2)) {
        // ------------------------------------------------------------------ MMA issuers (even CTA)
        if (lane == 0 && rank == 0) {
            const int mat = warp - 1;
            uint32_t n = 0, it = 0;
            bool ok = true;
            for (int item = cid; item < n_items && ok; item += ncl, ++it) {
                const int c_n = 32 * ((p.tiles[item / MT].z + 31) >> 5);  // <= N: the plan's tiles hold <= N rows
                const uint32_t idesc = idesc_f16_f32(256, c_n);
                if (!(ok = mbar_wait(d_empty, (it & 1) ^ 1, abort))) break;
                tc_fence_after();
                for (int kr = 0; kr < KR && ok; ++kr) {
                    for (int s = 0; s < 4; ++s) {
                        const uint32_t sl = n % kSlots;
                        if (!(ok = mbar_wait(&full[sl], (n / kSlots) & 1, abort))) break;
                        tc_fence_after();
                        const uint32_t bsm = smem_u32(tok + sl * C::TOK_STAGE);
#pragma unroll
                        for (int j = 0; j < 4; ++j) {
                            const uint32_t a_t = tmem + C::A_COL0 + (sl * MATS + mat) * 32 + 8 * j;
                            mma_f16_ts_pair(tmem + mat * N, a_t, smem_desc_sw128(bsm + 32 * j), idesc,
                                            (kr | s | j) != 0);
                        }
                        mma_commit_pair_both(&empty[sl]);
                        ++n;
                    }
                }
                if (ok) mma_commit_pair_both(d_full);
            }
            mma_commit_pair(mma_done);
            int dummy = 0;
            mbar_wait(mma_done, 0, (volatile int *)&dummy, 200000000ull);
            if (!ok) atomicCAS(p.err, 0, DEV_WAIT_TIMEOUT);
        }
    } else if (warp >= 4) {
        // ------------------------------------------------------------------ dequant + epilogue (both CTAs)
        const int q = warp & 3;
        const int grp = (warp - 4) >> 2;
        const int r = 32 * q + lane;
        const uint32_t lane_base = (uint32_t)(32 * q) << 16;
        uint32_t nraw = 0, n = 0, it = 0;
        bool ok = true;
        uint32_t tok_issued = 0;
        auto epilogue = [&](int eitem, uint32_t eit) -> bool {
            if (!mbar_wait(d_full, eit & 1, abort)) return false;
            tc_fence_after();
            const int4 t = p.tiles[eitem / MT];
            const int ch = (eitem % MT) * 256 + 128 * (int)rank + r;
            constexpr int NCH = (N + 31) / 32;
            constexpr int G = GATEUP ? 1 : (NCH < 4 ? NCH : 4);
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
                    if (lane == 0) mbar_arrive_cl(d_empty0);
                }
#pragma unroll
                for (int i = 0; i < G; ++i) {
                    const int c0 = 8 * grp + 32 * (b0 + i);
                    if (c0 < N && c0 < t.z) {
                        if constexpr (GATEUP) {
                            __half *out = reinterpret_cast<__half *>(p.out);
#pragma unroll
                            for (int j = 0; j < 8; ++j) {
                                if (c0 + j < t.z) {
                                    const float a = swiglu_clamped_fast(__uint_as_float(dg[i][j]),
                                                                       __uint_as_float(du[i][j]), p.limit);
                                    out[(int64_t)(t.y + c0 + j) * p.ld_out + ch] = __float2half_rn(a);
                                }
                            }
                        } else {
                            float *out = reinterpret_cast<float *>(p.out);
#pragma unroll
                            for (int j = 0; j < 8; ++j)
                                if (c0 + j < t.z)
                                    out[(int64_t)(t.y + c0 + j) * p.ld_out + ch] = __uint_as_float(dg[i][j]);
                        }
                    }
                }
            }
            return true;
        };
        for (int item = cid; item < n_items && ok; item += ncl, ++it) {
            const int4 tt = p.tiles[item / MT];
            const int n32 = (tt.z + 31) >> 5;              // 16-row token boxes per CTA
            const int y0 = tt.y + (int)rank * 16 * n32;    // this CTA's half of the token rows
            for (int kr = 0; kr < KR && ok; ++kr) {
                const uint32_t rs = nraw % SW;
                if (!(ok = mbar_wait(&raw_full[rs], (nraw / SW) & 1, abort))) break;
                const uint8_t *row = raw + rs * (MATS * kRawMat) + r * kRawRow;
#pragma unroll
                for (int s = 0; s < 4; ++s) {
                    if (s == grp) {
                        auto load_words = [&](int m, uint32_t (&w)[20]) {
#pragma unroll
                            for (int c = 0; c < 5; ++c) {
                                const uint4 v4 =
                                    *reinterpret_cast<const uint4 *>(row + m * kRawMat + 64 * s + 16 * c);
                                w[4 * c] = v4.x;
                                w[4 * c + 1] = v4.y;
                                w[4 * c + 2] = v4.z;
                                w[4 * c + 3] = v4.w;
                            }
                        };
                        auto convert = [&](const uint32_t (&w)[20], uint32_t (&v)[32]) {
                            uint32_t g[17];
#pragma unroll
                            for (int j = 0; j < 17; ++j) g[j] = w[s + j];
                            q8_two_blocks(g, v);
                        };
                        uint32_t w0[20], w1[20], v[32];
                        load_words(0, w0);
                        if (GATEUP) load_words(1, w1);
                        __syncwarp();
                        if (lane == 0) mbar_arrive(&raw_empty[rs]);
                        convert(w0, v);
                        const uint32_t sl = n % kSlots;
                        if (!(ok = mbar_wait(&empty[sl], ((n / kSlots) & 1) ^ 1, abort))) break;
                        if (q == 0) {
                            // this CTA's token rows of the sub-stage, counted on the even CTA's barrier
                            if (lane == 0) mbar_arrive_expect_tx_cl(full0 + 8 * sl, (uint32_t)n32 * 16 * 128);
                            __syncwarp();
                            if (lane < n32)
                                tma_load_2d_pair(tok + sl * C::TOK_STAGE + lane * 2048, &p.xt, full0 + 8 * sl,
                                                 kr * 256 + 64 * s, y0 + 16 * lane);
                            tok_issued = n + 1;
                        }
                        const uint32_t tcol = tmem + lane_base + C::A_COL0 + sl * MATS * 32;
                        tmem_st_32x32b_x32(tcol, v);
                        if (GATEUP) {
                            convert(w1, v);
                            tmem_st_32x32b_x32(tcol + 32, v);
                        }
                        tmem_wait_st();
                        tc_fence_before();
                        __syncwarp();
                        if (lane == 0) mbar_arrive_cl(full0 + 8 * sl);
                    }
                    ++n;
                }
                if (!ok) break;
                ++nraw;
                if (kr == 0 && it > 0 && !(ok = epilogue(item - ncl, it - 1))) break;
            }
        }
        if (ok && it > 0) ok = epilogue(cid + (int)(it - 1) * ncl, it - 1);
        if (!ok) {
            atomicCAS(p.err, 0, DEV_WAIT_TIMEOUT);
            // token loads in flight land before the pair releases its memory: the even CTA's
            // barrier counts both CTAs' bytes (bounded: after an abort its phase may never complete)
            if (rank == 0 && q == 0 && tok_issued > 0) {
                int dummy = 0;
                const uint32_t i = tok_issued - 1;
                mbar_wait(&full[i % kSlots], (i / kSlots) & 1, (volatile int *)&dummy, 100000000ull);
            }
        }
    }
    tc_fence_before();
    cluster_sync_all();  // every MMA of the pair complete and no cross-CTA access left
    tc_fence_after();
    if (warp == 2) tmem_dealloc_pair(tmem, 512);
}

// ----------------------------------------------------------------------------- host
static PFN_cuTensorMapEncodeTiled_v12000 get_encode() {
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

// Q8_0 matrix stack [experts][rows][row_bytes] as u16 elements; box = 128 rows x 272 B.
static int make_q8_map(CUtensorMap *m, const void *base, int64_t rows, int64_t k, int64_t experts,
                       int64_t expert_stride, int box_rows = 128) {
    auto enc = get_encode();
    if (!enc) {
        set_error("cuTensorMapEncodeTiled unavailable from the driver");
        return VFMOE_ERR_CUDA;
    }
    const int64_t row_bytes = k / 32 * 34;
    if (experts <= 1) expert_stride = rows * row_bytes;
    cuuint64_t dims[3] = {(cuuint64_t)(row_bytes / 2), (cuuint64_t)rows, (cuuint64_t)experts};
    cuuint64_t strides[2] = {(cuuint64_t)row_bytes, (cuuint64_t)expert_stride};
    cuuint32_t box[3] = {kRawRow / 2, (cuuint32_t)box_rows, 1};
    cuuint32_t es[3] = {1, 1, 1};
    CUresult r = enc(m, CU_TENSOR_MAP_DATA_TYPE_UINT16, 3, const_cast<void *>(base), dims, strides, box, es,
                     CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                     CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) {
        set_error("cuTensorMapEncodeTiled (Q8_0 weights) failed: %d", (int)r);
        return VFMOE_ERR_CUDA;
    }
    return VFMOE_OK;
}

// fp16 token rows [rows][k]; box = N rows x 64 halves (128 B), SWIZZLE_128B.
static int make_tok_map(CUtensorMap *m, const void *base, int64_t rows, int64_t k, int n) {
    auto enc = get_encode();
    if (!enc) {
        set_error("cuTensorMapEncodeTiled unavailable from the driver");
        return VFMOE_ERR_CUDA;
    }
    cuuint64_t dims[2] = {(cuuint64_t)k, (cuuint64_t)rows};
    cuuint64_t strides[1] = {(cuuint64_t)(k * 2)};
    cuuint32_t box[2] = {64, (cuuint32_t)n};
    cuuint32_t es[2] = {1, 1};
    CUresult r = enc(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void *>(base), dims, strides, box, es,
                     CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                     CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) {
        set_error("cuTensorMapEncodeTiled (token rows) failed: %d", (int)r);
        return VFMOE_ERR_CUDA;
    }
    return VFMOE_OK;
}

int tc_plan_create(const vfmoe_layer_desc &d, TcPlan &plan) {
    plan.ready = 0;
    const bool tiled = d.weight_format == VFMOE_WFMT_Q8_0_TILED;
    if (d.weight_format != VFMOE_WFMT_Q8_0 && !tiled) return VFMOE_OK;
    plan.path = (int)d.expert_path;
    if (d.expert_path == VFMOE_PATH_SIMT) {
        if (!tiled) return VFMOE_OK;
        set_error("VFMOE_PATH_SIMT: the SIMT expert path reads GGUF row order, not VFMOE_WFMT_Q8_0_TILED");
        return VFMOE_ERR_UNSUPPORTED;
    }
    int dev = 0;
    VF_CUDA(cudaGetDevice(&dev));
    VF_CUDA(cudaDeviceGetAttribute(&plan.num_sms, cudaDevAttrMultiProcessorCount, dev));
    const int64_t H = d.hidden, I = d.inter, E = d.n_local_experts ? d.n_local_experts : d.n_experts;
    const bool sh = d.sh_gate.data != 0;
    if (tiled) {
        plan.tiled = 1;
        plan.p_gate = reinterpret_cast<const uint8_t *>(d.gate.data);
        plan.p_up = reinterpret_cast<const uint8_t *>(d.up.data);
        plan.p_down = reinterpret_cast<const uint8_t *>(d.down.data);
        plan.p_sh_gate = reinterpret_cast<const uint8_t *>(sh ? d.sh_gate.data : d.gate.data);
        plan.p_sh_up = reinterpret_cast<const uint8_t *>(sh ? d.sh_up.data : d.up.data);
        plan.p_sh_down = reinterpret_cast<const uint8_t *>(sh ? d.sh_down.data : d.down.data);
        plan.s_gate = E > 1 ? d.gate.expert_stride : 0;
        plan.s_up = E > 1 ? d.up.expert_stride : 0;
        plan.s_down = E > 1 ? d.down.expert_stride : 0;
        plan.ready = 1;
        return VFMOE_OK;
    }
    int rc;
    if ((rc = make_q8_map(&plan.gate, (void *)d.gate.data, I, H, E, d.gate.expert_stride))) return rc;
    if ((rc = make_q8_map(&plan.up, (void *)d.up.data, I, H, E, d.up.expert_stride))) return rc;
    if ((rc = make_q8_map(&plan.down, (void *)d.down.data, H, I, E, d.down.expert_stride))) return rc;
    if ((rc = make_q8_map(&plan.sh_gate, (void *)(sh ? d.sh_gate.data : d.gate.data), I, H, 1, 0))) return rc;
    if ((rc = make_q8_map(&plan.sh_up, (void *)(sh ? d.sh_up.data : d.up.data), I, H, 1, 0))) return rc;
    if ((rc = make_q8_map(&plan.sh_down, (void *)(sh ? d.sh_down.data : d.down.data), H, I, 1, 0))) return rc;
    if ((rc = make_q8_map(&plan.gate64, (void *)d.gate.data, I, H, E, d.gate.expert_stride, 64))) return rc;
    if ((rc = make_q8_map(&plan.up64, (void *)d.up.data, I, H, E, d.up.expert_stride, 64))) return rc;
    if ((rc = make_q8_map(&plan.sh_gate64, (void *)(sh ? d.sh_gate.data : d.gate.data), I, H, 1, 0, 64))) return rc;
    if ((rc = make_q8_map(&plan.sh_up64, (void *)(sh ? d.sh_up.data : d.up.data), I, H, 1, 0, 64))) return rc;
    plan.ready = 1;
    return VFMOE_OK;
}

bool tc_supported(const TcPlan &plan, const MoeArgs &a) {
    return plan.ready && (a.fmt == VFMOE_WFMT_Q8_0 || a.fmt == VFMOE_WFMT_Q8_0_TILED) && a.tiles != nullptr && a.H % 256 == 0 && a.I % 256 == 0;
}

// Tiles of at least 8 rows (the decode GEMV's smallest): sum_e ceil(n_e / 8) <= rows / 8 + segments.
int64_t tc_tiles_capacity(int T, int k, int E) { return ((int64_t)T * k + T) / 8 + E + 2; }

int launch_tc_plan(const MoeArgs &a, int n_gu, int n_dn, cudaStream_t st) {
    VF_CUDA(launch_pdl(tc_plan_kernel, dim3(1), dim3(1024), 0, st, (const int32_t *)a.offsets, a.E, a.has_shared, n_gu,
                       n_dn, a.tiles, a.tiles_cap, a.tile_counts, a.err));
    VF_LAUNCH_CHECK("tc_plan_kernel");
    return VFMOE_OK;
}

static int pick_n(int T, int k, int E) {
    const double avg = (double)T * k / E;
    const int want = (int)std::max(2.0 * avg, (double)std::min(T, 32));
    int n = 16;
    while (n < want && n < 256) n <<= 1;
    return n;
}

template <bool GATEUP, int N>
static int launch_one(const TcParams &prm, int grid, cudaStream_t st) {
    using C = TcCfg<GATEUP, N>;
    if (int rc_attr = set_smem_attr_once(reinterpret_cast<const void *>(expert_gemm_tc<GATEUP, N>), C::SMEM)) return rc_attr;
    expert_gemm_tc<GATEUP, N><<<grid, kThreads, C::SMEM, st>>>(prm);
    VF_LAUNCH_CHECK(GATEUP ? "expert_gemm_tc<gate_up>" : "expert_gemm_tc<down>");
    return VFMOE_OK;
}

// Grid of a CTA-pair launch: every pair resident at once (the kernel is persistent), as many as
// the device holds with this kernel's shared memory; 0 if the query fails.
template <bool GATEUP, int N>
static int pair_grid() {
    static std::mutex mu;
    static int dev_cached = -1, grid_cached = 0;
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return 0;
    std::lock_guard<std::mutex> lk(mu);
    if (dev == dev_cached) return grid_cached;
    using C = TcPairCfg<GATEUP, N>;
    if (set_smem_attr_once(reinterpret_cast<const void *>(expert_gemm_tc_pair<GATEUP, N>), C::SMEM)) return 0;
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3(2);
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = C::SMEM;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 2;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    int nc = 0;
    if (cudaOccupancyMaxActiveClusters(&nc, reinterpret_cast<const void *>(expert_gemm_tc_pair<GATEUP, N>), &cfg) !=
        cudaSuccess) {
        cudaGetLastError();
        nc = 0;
    }
    dev_cached = dev;
    grid_cached = 2 * nc;
    return grid_cached;
}

template <bool GATEUP, int N>
static int launch_pair(const TcParams &prm, cudaStream_t st, bool *launched) {
    using C = TcPairCfg<GATEUP, N>;
    *launched = false;
    const int grid = pair_grid<GATEUP, N>();
    if (grid < 2) return VFMOE_OK;  // the caller runs the single-CTA kernel
    expert_gemm_tc_pair<GATEUP, N><<<grid, kThreads, C::SMEM, st>>>(prm);
    VF_LAUNCH_CHECK(GATEUP ? "expert_gemm_tc_pair<gate_up>" : "expert_gemm_tc_pair<down>");
    *launched = true;
    return VFMOE_OK;
}

bool tc_decode_gemv(const TcPlan &plan, const MoeArgs &a) {
    const bool decode = (double)a.T * a.k / a.E <= 16.0;
    const bool forced_tc = plan.path == VFMOE_PATH_TC || plan.path == VFMOE_PATH_TC1;
    return a.prec || plan.path == VFMOE_PATH_GEMV || (decode && !forced_tc);
}

int launch_experts_tc(const TcPlan &plan, const MoeArgs &a, cudaStream_t st, const std::function<void()> &mid) {
    const int64_t rows = (int64_t)a.T * a.k + a.T;
    if (tc_decode_gemv(plan, a)) {
        // decode: register-operand GEMV, one token-tile size for both GEMMs (fp32 activations:
        // its split-precision form at every T)
        const int ng = gemv_tokens_per_tile(a.T, a.k, a.E);
        if (!a.plan_ready) {
            VF_CUDA(launch_pdl(tc_plan_kernel, dim3(1), dim3(1024), 0, st, (const int32_t *)a.offsets, a.E, a.has_shared,
                               ng, ng, a.tiles, a.tiles_cap, a.tile_counts, a.err));
            VF_LAUNCH_CHECK("tc_plan_kernel");
        }
        CUtensorMap tg, td, tg2, td2;
        int rc;
        if ((rc = make_tok_map(&tg, a.xp, rows, a.H, ng))) return rc;
        if ((rc = make_tok_map(&td, a.act, rows, a.I, ng))) return rc;
        if (a.prec) {
            if ((rc = make_tok_map(&tg2, a.xp + rows * a.H, rows, a.H, ng))) return rc;
            if ((rc = make_tok_map(&td2, a.act + rows * a.I, rows, a.I, ng))) return rc;
        }
        return launch_experts_gemv(plan, a, st, mid, tg, td, a.prec ? &tg2 : nullptr, a.prec ? &td2 : nullptr);
    }
    const int n = pick_n(a.T, a.k, a.E);
    const int n_gu = std::min(n, 128);
    const int n_dn = n;
    VF_CUDA(launch_pdl(tc_plan_kernel, dim3(1), dim3(1024), 0, st, (const int32_t *)a.offsets, a.E, a.has_shared, n_gu,
                       n_dn, a.tiles, a.tiles_cap, a.tile_counts, a.err));
    VF_LAUNCH_CHECK("tc_plan_kernel");
    int rc;
    TcParams g{};
    g.wa = plan.gate;
    g.wb = plan.up;
    g.swa = plan.sh_gate;
    g.swb = plan.sh_up;
    g.tiled = plan.tiled;
    g.pa = plan.p_gate;
    g.pb = plan.p_up;
    g.spa = plan.p_sh_gate;
    g.spb = plan.p_sh_up;
    g.sa = plan.s_gate;
    g.sb = plan.s_up;
    if ((rc = make_tok_map(&g.xt, a.xp, rows, a.H, 16))) return rc;
    g.tiles = a.tiles;
    g.n_tiles = a.tile_counts;
    g.E = a.E;
    g.K = a.H;
    g.M = a.I;
    g.ld_out = a.I;
    g.out = a.act;
    g.limit = a.limit;
    g.err = a.err;
    const int grid = plan.num_sms;
    // CTA pairs (M = 256 per MMA) whenever the tiles allow their N (a multiple of 32); single-CTA
    // tiles for N = 16, when forced (VFMOE_PATH_TC1), or if the device holds no pair
    const bool try_pair = n_gu >= 32 && plan.path != VFMOE_PATH_TC1;
    bool paired = false;
    if (try_pair) {
        switch (n_gu) {
            case 32: rc = launch_pair<true, 32>(g, st, &paired); break;
            case 64: rc = launch_pair<true, 64>(g, st, &paired); break;
            default: rc = launch_pair<true, 128>(g, st, &paired); break;
        }
        if (rc) return rc;
    }
    if (!paired) {
        switch (n_gu) {
            case 16: rc = launch_one<true, 16>(g, grid, st); break;
            case 32: rc = launch_one<true, 32>(g, grid, st); break;
            case 64: rc = launch_one<true, 64>(g, grid, st); break;
            default: rc = launch_one<true, 128>(g, grid, st); break;
        }
        if (rc) return rc;
    }
    mid();
    TcParams dn{};
    dn.wa = plan.down;
    dn.wb = plan.down;
    dn.swa = plan.sh_down;
    dn.swb = plan.sh_down;
    dn.tiled = plan.tiled;
    dn.pa = dn.pb = plan.p_down;
    dn.spa = dn.spb = plan.p_sh_down;
    dn.sa = dn.sb = plan.s_down;
    if ((rc = make_tok_map(&dn.xt, a.act, rows, a.I, 16))) return rc;
    dn.tiles = a.tiles + a.tiles_cap;
    dn.n_tiles = a.tile_counts + 1;
    dn.E = a.E;
    dn.K = a.I;
    dn.M = a.H;
    dn.ld_out = a.H;
    dn.out = a.y;
    dn.limit = a.limit;
    dn.err = a.err;
    if (try_pair) {
        bool dn_paired = false;
        switch (n_dn) {
            case 32: rc = launch_pair<false, 32>(dn, st, &dn_paired); break;
            case 64: rc = launch_pair<false, 64>(dn, st, &dn_paired); break;
            case 128: rc = launch_pair<false, 128>(dn, st, &dn_paired); break;
            default: rc = launch_pair<false, 256>(dn, st, &dn_paired); break;
        }
        if (rc || dn_paired) return rc;
    }
    switch (n_dn) {
        case 16: return launch_one<false, 16>(dn, grid, st);
        case 32: return launch_one<false, 32>(dn, grid, st);
        case 64: return launch_one<false, 64>(dn, grid, st);
        case 128: return launch_one<false, 128>(dn, grid, st);
        default: return launch_one<false, 256>(dn, grid, st);
    }
}

}  // namespace vfmoe
