// Decode expert GEMV (few tokens per expert): TMA-fed, register-operand tensor-core MMA.
//
//   gate/up:  act[rows, ch] = fp16(swiglu(x . Wg[ch], x . Wu[ch]))  (moe.vyb:98-134)
//   down:     y[rows, ch]   = act . Wd[ch]                          (moe.vyb:137-170)
//
// At decode every Q8_0 weight byte is used by only a handful of tokens, so the kernel is
// HBM-bound: its job is to stream the weights once at full bandwidth.  A tcgen05 MMA
// reads its whole A tile from TMEM or shared memory per instruction; at N <= 32 tokens
// that operand traffic, not HBM, becomes the limit.  Here the dequantized weights go from
// registers straight into mma.sync m16n8k16 (fp16 x fp16 -> fp32), so weights are read
// from shared memory exactly once, as raw Q8_0 bytes.
//
// Data path per CTA (one per SM, persistent over (expert, token tile, channel tile)):
//   warp 16      TMA producer: per stage, 8 Q8_0 blocks (272 B) of each weight row of the
//                tile (a TMA box from GGUF rows, or one bulk copy per 64 rows from
//                stage-tiled weights) plus the 256-K slice of the tile's N token rows
//                (fp16, SWIZZLE_128B).
//   warps 0..15  consumers in two K halves: warps 8h..8h+7 take the 64-K pairs 2h and 2h+1 of
//                every stage, 16 weight rows each: LDS raw bytes -> fp16(d*q) fragments in
//                registers -> mma.sync against token fragments -> fp32 accumulators.  The
//                second half's partial sums join the first half's in the epilogue (shared
//                memory).  gate/up tile = 64 channels x (gate, up): warps 0-3 gate, 4-7 up,
//                SwiGLU after an exchange through shared memory; down tile = 128 channels.
//                Two warps per scheduler left the kernel stalled on the fixed latency between
//                the Q8_0 -> fp16 conversion and its mma.sync (0.77 of HBM); four reach 0.92.
//                (The split-precision form keeps 8 consumers, one K range: warp 8 produces.)
// K permutation: within each 64-K pair of Q8_0 blocks, thread (g, c) of the MMA quad owns
// actual k in [16c, 16c + 16) for both A and B, so each thread converts 16 consecutive
// quants of a row and loads 32 consecutive token bytes.
//
// Split precision (PREC, fp32 activations): a Q8_0 weight d*q is exact in fp32; it is carried
// as w_hi = fp16(d*q) and w_lo = fp16((d*q - w_hi) * 2^12), a token value as x_hi = fp16(x) and
// x_lo = fp16((x - x_hi) * 2^12) (a second fp16 plane of the token rows).  Each MMA step then
// issues w_hi.x_hi into one accumulator and w_hi.x_lo + w_lo.x_hi into a second, which is
// scaled by 2^-12 at the end: the products lose only the w_lo.x_lo term (~2^-24 relative) and
// the result is close to fp32 arithmetic.  The gate/up epilogue writes act as two planes the
// same way, so the down GEMV sees act to about fp32 precision too.
//
// Every mbarrier wait is bounded (2 s, or p.wait_ns); on expiry the CTA raises DEV_WAIT_TIMEOUT
// and exits after draining its TMA loads.  p.stall (tests only) makes the producer issue no
// loads at all, so the consumers' first waits expire with nothing in flight.
#include <cudaTypedefs.h>

#include <algorithm>

#include "expert_tc.h"
#include "sm100.cuh"

namespace vfmoe {

using namespace sm100;

constexpr int kRow = 272;            // 8 Q8_0 blocks (256 K) of one weight row
constexpr int kWBytes = 128 * kRow;  // weights per stage: 64 rows x 2 matrices or 128 rows

template <bool GATEUP, int NT, bool PREC, bool DENSE = false>
struct GvCfg {
    // consumer warps: 16 split each stage's K in two halves (pairs 0-1 and 2-3), whose partial
    // sums meet in the epilogue; the split-precision form keeps 8 (its three accumulators need
    // the registers)
    static constexpr int CONS = PREC ? 8 : 16;
    static constexpr int HALVES = CONS / 8;
    static constexpr int THREADS = 32 * (CONS + 1);
    static constexpr int N = 8 * NT;
    static constexpr int ROWS = GATEUP ? 64 : 128;  // channels per tile
    static constexpr int TOK1 = N * 512;            // N rows x 256 K fp16: one plane
    static constexpr int TOK = PREC ? 2 * TOK1 : TOK1;
    // weight bytes of a stage: Q8_0 rows of 272 B, or dense fp16 as 4 boxes of 64 K x ROWS rows
    // per matrix (128-byte rows, SWIZZLE_128B)
    static constexpr int WBOX = ROWS * 128;
    static constexpr int WB = DENSE ? (GATEUP ? 2 : 1) * 4 * WBOX : kWBytes;
    static constexpr int STAGE = WB + TOK;
    // epilogue exchange, fp32 [rows of the tile][N]: the second K half's partial sums, then (gate/up)
    // the up rows for the SwiGLU.  With two halves it is double-buffered by item parity, so the
    // second half starts its next item while the first writes this item's outputs.
    static constexpr int XBUF = (GATEUP ? 2 : 1) * ROWS * N;  // floats per buffer
    static constexpr int XCH = HALVES == 2 ? 2 * XBUF * 4 : (GATEUP ? ROWS * N * 4 : 0);
    static constexpr int SW = (230000 - XCH - 1024) / STAGE > 6 ? 6 : (230000 - XCH - 1024) / STAGE;
    static constexpr int SMEM = SW * STAGE + XCH + 2 * SW * 8 + 16 + 1024;
    static_assert(SW >= 2, "at least double buffering");
    static_assert(SMEM <= 232448, "shared memory budget");
};

__device__ __forceinline__ void mma_16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
        "{%0, %1, %2, %3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

__device__ __forceinline__ uint32_t q8_pair16(uint32_t word, uint32_t sel, __half2 d2) {
    const uint32_t h = __byte_perm(word, 0x64646464u, sel);  // 1024 + (q ^ 0x80) per half
    __half2 v = *reinterpret_cast<const __half2 *>(&h);
    v = __hsub2(v, __half2half2(__ushort_as_half(0x6480)));  // exact q
    v = __hmul2(v, d2);                                      // fp16(d * q), one rounding
    return *reinterpret_cast<const uint32_t *>(&v);
}

// 16 consecutive quants of one row inside a 64-K pair (thread c of the quad) -> 8 fp16
// pairs.  `row` points at the row's 272-byte stage slice, p = pair (0..3), c = 0..3.
// Quants start at byte 68p + 34*(c>>1) + 2 + 16*(c&1); the scale d at 68p + 34*(c>>1).
__device__ __forceinline__ void q8_frag(const uint8_t *row, int p, int c, uint32_t (&out)[8]) {
    const int blk = 68 * p + 34 * (c >> 1);
    const int qb = blk + 2 + 16 * (c & 1);            // first quant byte (2 mod 4 for c<2)
    const int w0 = qb >> 2;                            // aligned word holding it
    const uint32_t *rw = reinterpret_cast<const uint32_t *>(row);
    uint32_t w[5];
#pragma unroll
    for (int i = 0; i < 5; ++i) w[i] = rw[w0 + i];
    const uint32_t dw = rw[blk >> 2];
    const unsigned short dbits = (blk & 2) ? (unsigned short)(dw >> 16) : (unsigned short)(dw & 0xFFFFu);
    const __half2 d2 = __half2half2(__ushort_as_half(dbits));
    const int sh = qb & 3;                             // 0 or 2
    uint32_t q[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) q[i] = (sh ? __funnelshift_r(w[i], w[i + 1], 16) : w[i]) ^ 0x80808080u;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        out[2 * i] = q8_pair16(q[i], 0x4140u, d2);
        out[2 * i + 1] = q8_pair16(q[i], 0x4342u, d2);
    }
}

// q8_frag for the split-precision GEMV: the same 16 quants as fp16 pairs hi = fp16(d*q) and
// lo = fp16((d*q - hi) * 2^12).  d*q is exact in fp32 (11-bit d times 8-bit q).
__device__ __forceinline__ void q8_frag_prec(const uint8_t *row, int p, int c, uint32_t (&hi)[8],
                                             uint32_t (&lo)[8]) {
    const int blk = 68 * p + 34 * (c >> 1);
    const int qb = blk + 2 + 16 * (c & 1);
    const int w0 = qb >> 2;
    const uint32_t *rw = reinterpret_cast<const uint32_t *>(row);
    uint32_t w[5];
#pragma unroll
    for (int i = 0; i < 5; ++i) w[i] = rw[w0 + i];
    const uint32_t dw = rw[blk >> 2];
    const unsigned short dbits = (blk & 2) ? (unsigned short)(dw >> 16) : (unsigned short)(dw & 0xFFFFu);
    const float d = __half2float(__ushort_as_half(dbits));
    const int sh = qb & 3;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const uint32_t q = (sh ? __funnelshift_r(w[i], w[i + 1], 16) : w[i]);
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            const float a = d * (float)(int8_t)(q >> (16 * h)), b = d * (float)(int8_t)(q >> (16 * h + 8));
            const __half2 vh = __floats2half2_rn(a, b);
            const float2 back = __half22float2(vh);
            const __half2 vl = __floats2half2_rn((a - back.x) * 4096.f, (b - back.y) * 4096.f);
            hi[2 * i + h] = *reinterpret_cast<const uint32_t *>(&vh);
            lo[2 * i + h] = *reinterpret_cast<const uint32_t *>(&vl);
        }
    }
}

template <bool GATEUP, int NT, bool PREC, bool DENSE>
__global__ void __launch_bounds__(GvCfg<GATEUP, NT, PREC, DENSE>::THREADS, 1)
    expert_gemv_mma(const __grid_constant__ TcParams p) {
    using C = GvCfg<GATEUP, NT, PREC, DENSE>;
    constexpr int SW = C::SW, N = C::N, ROWS = C::ROWS, CONS = C::CONS;
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    float *xch = reinterpret_cast<float *>(smem + SW * C::STAGE);
    uint64_t *full = reinterpret_cast<uint64_t *>(smem + SW * C::STAGE + C::XCH);
    uint64_t *empty = full + SW;
    volatile int *abort = reinterpret_cast<volatile int *>(empty + SW);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int MT = p.M / ROWS;
    const int KR = p.K / 256;
    if (threadIdx.x == 0) {
        for (int i = 0; i < SW; ++i) {
            mbar_init(&full[i], 1);
            mbar_init(&empty[i], CONS);
        }
        *abort = 0;
        fence_mbar_init();
    }
    __syncthreads();
    // Programmatic dependent launch: the routed gate/up reads the tile list that the kernel
    // before it writes, so every thread waits for that kernel first (the barriers and the tensor
    // maps above are set up while it runs).  The down GEMV reads a tile list written two kernels
    // back and waits only before its token rows (below).  The next kernel (the down GEMV after
    // gate/up) may be scheduled onto SMs as this grid retires; it reads this grid's output only
    // after griddepcontrol.wait.
    if constexpr (GATEUP && !DENSE) griddep_wait();
    if (threadIdx.x == 0) griddep_launch_dependents();
    const int n_items = (DENSE ? (p.dense_T + N - 1) / N : *p.n_tiles) * MT;
    // the item's token tile: the tile list, or for a dense expert tiles of N rows in order
    auto tile_of = [&](int item) -> int4 {
        if constexpr (DENSE) {
            const int y = (item / MT) * N;
            return make_int4(p.E, y, min(N, p.dense_T - y), 0);
        } else {
            return p.tiles[item / MT];
        }
    };

    if (warp == CONS) {
        // ------------------------------------------------------------------ TMA producer
        if (lane == 0 && !p.stall) {
            if (PREC) prefetch_tmap(&p.xt2);
            if (!p.tiled) {
                prefetch_tmap(&p.wa);
                prefetch_tmap(&p.swa);
            }
            prefetch_tmap(&p.xt);
            // The first SW stages are free at start: their weights are requested before the
            // wait on the previous kernel (programmatic dependent launch: the token rows it
            // writes are read only after griddepcontrol.wait), their token rows after it.
            // Without a programmatic launch the wait returns at once.
            const int my_items = blockIdx.x < n_items ? (n_items - 1 - blockIdx.x) / gridDim.x + 1 : 0;
            const int pre = my_items * KR < SW ? my_items * KR : SW;
            for (int i = 0; i < pre; ++i) {
                const int item = blockIdx.x + (i / KR) * gridDim.x, kr = i % KR;
                const int4 t = tile_of(item);
                const bool sh = t.x == p.E;
                uint8_t *st = smem + i * C::STAGE;
                mbar_arrive_expect_tx(&full[i], C::STAGE);
                if constexpr (DENSE) {
#pragma unroll
                    for (int q = 0; q < 4; ++q) {
                        tma_load_2d(st + q * C::WBOX, &p.wa, &full[i], kr * 256 + 64 * q, (item % MT) * ROWS);
                        if (GATEUP)
                            tma_load_2d(st + (4 + q) * C::WBOX, &p.wb, &full[i], kr * 256 + 64 * q, (item % MT) * ROWS);
                    }
                } else if (p.tiled) {
                    load_q8_tiled(st, sh ? p.spa : p.pa, p.sa, sh ? 0 : t.x, (item % MT) * ROWS, ROWS, KR, kr, &full[i]);
                    if (GATEUP)
                        load_q8_tiled(st + ROWS * kRow, sh ? p.spb : p.pb, p.sb, sh ? 0 : t.x, (item % MT) * ROWS, ROWS,
                                      KR, kr, &full[i]);
                } else {
                    tma_load_3d(st, sh ? &p.swa : &p.wa, &full[i], kr * (kRow / 2), (item % MT) * ROWS, sh ? 0 : t.x);
                    if (GATEUP)
                        tma_load_3d(st + ROWS * kRow, sh ? &p.swb : &p.wb, &full[i], kr * (kRow / 2),
                                    (item % MT) * ROWS, sh ? 0 : t.x);
                }
            }
            griddep_wait();
            for (int i = 0; i < pre; ++i) {
                const int item = blockIdx.x + (i / KR) * gridDim.x, kr = i % KR;
                const int4 t = tile_of(item);
                uint8_t *st = smem + i * C::STAGE;
#pragma unroll
                for (int q = 0; q < 4; ++q) tma_load_2d(st + C::WB + q * (N * 128), &p.xt, &full[i], kr * 256 + 64 * q, t.y);
                if (PREC) {
#pragma unroll
                    for (int q = 0; q < 4; ++q)
                        tma_load_2d(st + C::WB + C::TOK1 + q * (N * 128), &p.xt2, &full[i], kr * 256 + 64 * q, t.y);
                }
            }
            uint32_t n = 0;
            bool ok = true;
            for (int item = blockIdx.x; item < n_items && ok; item += gridDim.x) {
                const int4 t = tile_of(item);
                const int m0 = (item % MT) * ROWS;
                const bool sh = t.x == p.E;
                const CUtensorMap *ma = sh ? &p.swa : &p.wa;
                const CUtensorMap *mb = sh ? &p.swb : &p.wb;
                const int z = sh ? 0 : t.x;
                for (int kr = 0; kr < KR; ++kr, ++n) {
                    if (n < (uint32_t)pre) continue;  // issued above
                    const uint32_t s = n % SW;
                    if (!(ok = mbar_wait(&empty[s], ((n / SW) & 1) ^ 1, abort, p.wait_ns))) break;
                    uint8_t *st = smem + s * C::STAGE;
                    mbar_arrive_expect_tx(&full[s], C::STAGE);
                    if constexpr (DENSE) {
#pragma unroll
                        for (int q = 0; q < 4; ++q) {
                            tma_load_2d(st + q * C::WBOX, &p.wa, &full[s], kr * 256 + 64 * q, m0);
                            if (GATEUP) tma_load_2d(st + (4 + q) * C::WBOX, &p.wb, &full[s], kr * 256 + 64 * q, m0);
                        }
                    } else if (p.tiled) {
                        load_q8_tiled(st, sh ? p.spa : p.pa, p.sa, z, m0, ROWS, KR, kr, &full[s]);
                        if (GATEUP) load_q8_tiled(st + ROWS * kRow, sh ? p.spb : p.pb, p.sb, z, m0, ROWS, KR, kr, &full[s]);
                    } else {
                        tma_load_3d(st, ma, &full[s], kr * (kRow / 2), m0, z);
                        if (GATEUP) tma_load_3d(st + ROWS * kRow, mb, &full[s], kr * (kRow / 2), m0, z);
                    }
#pragma unroll
                    for (int q = 0; q < 4; ++q) tma_load_2d(st + C::WB + q * (N * 128), &p.xt, &full[s], kr * 256 + 64 * q, t.y);
                    if (PREC) {
#pragma unroll
                        for (int q = 0; q < 4; ++q)
                            tma_load_2d(st + C::WB + C::TOK1 + q * (N * 128), &p.xt2, &full[s], kr * 256 + 64 * q,
                                        t.y);
                    }
                }
            }
            if (!ok) {
                atomicCAS(p.err, 0, DEV_WAIT_TIMEOUT);
                int dummy = 0;
                for (uint32_t i = (n > (uint32_t)SW ? n - SW : 0); i < n; ++i)
                    mbar_wait(&full[i % SW], (i / SW) & 1, (volatile int *)&dummy, 100000000ull);
            }
        }
    } else {
        // ------------------------------------------------------------------ consumers
        const int g = lane >> 2, c = lane & 3;
        const int half = warp >> 3, lw = warp & 7;            // K half (pairs 2 half .. 2 half + 4 / HALVES - 1)
        const int mat = GATEUP ? (lw >> 2) : 0;
        const int r0 = GATEUP ? 16 * (lw & 3) : 16 * lw;      // first row of this warp in its matrix tile
        const int xrow0 = mat * ROWS + r0;                    // the warp's rows in the exchange buffer
        uint32_t n = 0, it = 0;
        bool ok = true;
        for (int item = blockIdx.x; item < n_items && ok; item += gridDim.x, ++it) {
            const int4 t = tile_of(item);
            const int m0 = (item % MT) * ROWS;
            const int ntv = (t.z + 7) >> 3;                     // n8 tiles with valid token rows
            float acc[NT][4];
            float acc2[PREC ? NT : 1][4];                       // PREC: w_hi.x_lo + w_lo.x_hi, x 2^12
#pragma unroll
            for (int j = 0; j < NT; ++j) acc[j][0] = acc[j][1] = acc[j][2] = acc[j][3] = 0.f;
#pragma unroll
            for (int j = 0; j < (PREC ? NT : 1); ++j) acc2[j][0] = acc2[j][1] = acc2[j][2] = acc2[j][3] = 0.f;
            for (int kr = 0; kr < KR; ++kr, ++n) {
                const uint32_t s = n % SW;
                if (!(ok = mbar_wait(&full[s], (n / SW) & 1, abort, p.wait_ns))) break;
                const uint8_t *st = smem + s * C::STAGE;
                const uint8_t *rowA = st + (mat * ROWS + r0 + g) * kRow;
                const uint8_t *rowB = rowA + 8 * kRow;
#pragma unroll
                for (int pi = 0; pi < 4 / C::HALVES; ++pi) {
                    const int pq = half * (4 / C::HALVES) + pi;
                    uint32_t wa[8], wb[8], la[PREC ? 8 : 1], lb[PREC ? 8 : 1];
                    if constexpr (DENSE) {
                        // rows r0+g and r0+g+8 of this matrix's box pq, 16-byte chunks 2c and 2c+1
                        const uint8_t *box = st + (mat * 4 + pq) * C::WBOX;
                        const int ra = r0 + g, rb = ra + 8;
                        const uint4 a0 = *reinterpret_cast<const uint4 *>(box + ra * 128 + (((2 * c) ^ (ra & 7)) << 4));
                        const uint4 a1 = *reinterpret_cast<const uint4 *>(box + ra * 128 + (((2 * c + 1) ^ (ra & 7)) << 4));
                        const uint4 b0 = *reinterpret_cast<const uint4 *>(box + rb * 128 + (((2 * c) ^ (rb & 7)) << 4));
                        const uint4 b1 = *reinterpret_cast<const uint4 *>(box + rb * 128 + (((2 * c + 1) ^ (rb & 7)) << 4));
                        wa[0] = a0.x; wa[1] = a0.y; wa[2] = a0.z; wa[3] = a0.w;
                        wa[4] = a1.x; wa[5] = a1.y; wa[6] = a1.z; wa[7] = a1.w;
                        wb[0] = b0.x; wb[1] = b0.y; wb[2] = b0.z; wb[3] = b0.w;
                        wb[4] = b1.x; wb[5] = b1.y; wb[6] = b1.z; wb[7] = b1.w;
                    } else if constexpr (PREC) {
                        q8_frag_prec(rowA, pq, c, wa, la);
                        q8_frag_prec(rowB, pq, c, wb, lb);
                    } else {
                        q8_frag(rowA, pq, c, wa);
                        q8_frag(rowB, pq, c, wb);
                    }
                    const uint8_t *tq = st + C::WB + pq * (N * 128);
#pragma unroll
                    for (int j = 0; j < NT; ++j) {
                        if (j < ntv) {
                            // token row 8j+g, 16-byte chunks 2c and 2c+1 (SWIZZLE_128B: chunk ^ (row & 7))
                            const int rr = 8 * j + g;
                            const int o0 = rr * 128 + (((2 * c) ^ (rr & 7)) << 4);
                            const int o1 = rr * 128 + (((2 * c + 1) ^ (rr & 7)) << 4);
                            const uint4 x0 = *reinterpret_cast<const uint4 *>(tq + o0);
                            const uint4 x1 = *reinterpret_cast<const uint4 *>(tq + o1);
                            const uint32_t xb[8] = {x0.x, x0.y, x0.z, x0.w, x1.x, x1.y, x1.z, x1.w};
                            if constexpr (PREC) {
                                const uint4 y0 = *reinterpret_cast<const uint4 *>(tq + C::TOK1 + o0);
                                const uint4 y1 = *reinterpret_cast<const uint4 *>(tq + C::TOK1 + o1);
                                const uint32_t xl[8] = {y0.x, y0.y, y0.z, y0.w, y1.x, y1.y, y1.z, y1.w};
#pragma unroll
                                for (int s4 = 0; s4 < 4; ++s4) {
                                    const uint32_t a[4] = {wa[2 * s4], wb[2 * s4], wa[2 * s4 + 1], wb[2 * s4 + 1]};
                                    const uint32_t al[4] = {la[2 * s4], lb[2 * s4], la[2 * s4 + 1], lb[2 * s4 + 1]};
                                    mma_16816(acc[j], a, xb[2 * s4], xb[2 * s4 + 1]);
                                    mma_16816(acc2[j], a, xl[2 * s4], xl[2 * s4 + 1]);
                                    mma_16816(acc2[j], al, xb[2 * s4], xb[2 * s4 + 1]);
                                }
                            } else {
#pragma unroll
                                for (int s4 = 0; s4 < 4; ++s4) {
                                    const uint32_t a[4] = {wa[2 * s4], wb[2 * s4], wa[2 * s4 + 1], wb[2 * s4 + 1]};
                                    mma_16816(acc[j], a, xb[2 * s4], xb[2 * s4 + 1]);
                                }
                            }
                        }
                    }
                }
                __syncwarp();
                if (lane == 0) mbar_arrive(&empty[s]);
            }
            if (!ok) break;
            if constexpr (PREC) {
#pragma unroll
                for (int j = 0; j < NT; ++j)
#pragma unroll
                    for (int e = 0; e < 4; ++e) acc[j][e] = fmaf(acc2[j][e], 1.0f / 4096.f, acc[j][e]);
            }
            // ---------------------------------------------------------------- epilogue
            // acc[j]: rows r0+g (0,1) and r0+g+8 (2,3) x tokens 8j+2c, 8j+2c+1
            auto store_gate_up = [&](const float *xup) {
                __half *out = reinterpret_cast<__half *>(p.out);
#pragma unroll
                for (int j = 0; j < NT; ++j)
#pragma unroll
                    for (int e = 0; e < 4; ++e) {
                        const int rr = r0 + g + 8 * (e >> 1), tok = 8 * j + 2 * c + (e & 1);
                        if (tok < t.z) {
                            const float a = swiglu_clamped(acc[j][e], xup[rr * N + tok], p.limit);
                            const int64_t o = (int64_t)(t.y + tok) * p.ld_out + m0 + rr;
                            const __half ah = __float2half_rn(a);
                            out[o] = ah;
                            if (PREC) out[o + p.out_plane] = __float2half_rn((a - __half2float(ah)) * 4096.f);
                        }
                    }
            };
            auto store_down = [&]() {
                float *out = reinterpret_cast<float *>(p.out);
#pragma unroll
                for (int j = 0; j < NT; ++j)
#pragma unroll
                    for (int e = 0; e < 4; ++e) {
                        const int rr = r0 + g + 8 * (e >> 1), tok = 8 * j + 2 * c + (e & 1);
                        if (tok < t.z) out[(int64_t)(t.y + tok) * p.ld_out + m0 + rr] = acc[j][e];
                    }
            };
            auto put_up = [&](float *xup) {
#pragma unroll
                for (int j = 0; j < NT; ++j)
#pragma unroll
                    for (int e = 0; e < 4; ++e) xup[(r0 + g + 8 * (e >> 1)) * N + 8 * j + 2 * c + (e & 1)] = acc[j][e];
            };
            if constexpr (C::HALVES == 2) {
                // The second K half hands its partial sums to the first through this item's buffer
                // (one barrier of all consumers) and goes on to its next item, which uses the other
                // buffer; it can write this buffer again only after the next item's barrier, which
                // the first half reaches after it has finished reading it.  Gate/up: the first
                // half's up warps then pass their rows to its gate warps (a barrier of the first
                // half only).
                float *xb = xch + (it & 1) * C::XBUF;
                if (half == 1) {
#pragma unroll
                    for (int j = 0; j < NT; ++j)
#pragma unroll
                        for (int e = 0; e < 4; ++e)
                            xb[(xrow0 + g + 8 * (e >> 1)) * N + 8 * j + 2 * c + (e & 1)] = acc[j][e];
                }
                asm volatile("bar.sync 1, %0;" ::"r"(32 * CONS) : "memory");
                if (half == 0) {
#pragma unroll
                    for (int j = 0; j < NT; ++j)
#pragma unroll
                        for (int e = 0; e < 4; ++e)
                            acc[j][e] += xb[(xrow0 + g + 8 * (e >> 1)) * N + 8 * j + 2 * c + (e & 1)];
                    if (GATEUP) {
                        float *xup = xb + ROWS * N;  // each up warp overwrites only the rows it has just read
                        if (mat == 1) put_up(xup);
                        asm volatile("bar.sync 2, 256;" ::: "memory");
                        if (mat == 0) store_gate_up(xup);
                    } else {
                        store_down();
                    }
                }
            } else {
                if (GATEUP) {
                    if (mat == 1) put_up(xch);
                    asm volatile("bar.sync 1, %0;" ::"r"(32 * CONS) : "memory");
                    if (mat == 0) store_gate_up(xch);
                    asm volatile("bar.sync 1, %0;" ::"r"(32 * CONS) : "memory");
                } else {
                    store_down();
                }
            }
        }
        if (!ok) atomicCAS(p.err, 0, DEV_WAIT_TIMEOUT);
    }
}

template <bool GATEUP, int NT, bool PREC, bool DENSE = false>
static int launch_gv(const TcParams &prm, int grid, cudaStream_t st) {
    using C = GvCfg<GATEUP, NT, PREC, DENSE>;
    if (int rc_attr = set_smem_attr_once(reinterpret_cast<const void *>(expert_gemv_mma<GATEUP, NT, PREC, DENSE>),
                                         C::SMEM))
        return rc_attr;
    // programmatic dependent launch: gate/up sets up while the kernel before it finishes; the down
    // GEMV's CTAs start streaming weights on SMs the gate/up grid has released, before its act
    // rows are complete
    VF_CUDA(launch_pdl(expert_gemv_mma<GATEUP, NT, PREC, DENSE>, dim3(grid), dim3(C::THREADS), (size_t)C::SMEM, st,
                       prm));
    VF_LAUNCH_CHECK(GATEUP ? "expert_gemv_mma<gate_up>" : "expert_gemv_mma<down>");
    return VFMOE_OK;
}

static PFN_cuTensorMapEncodeTiled_v12000 gv_encode() {
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

// fp16 [rows][k], box 64 x box_rows, SWIZZLE_128B (dense weights and token rows alike).
int make_dense_map(CUtensorMap *m, const void *base, int64_t rows, int64_t k, int box_rows) {
    auto enc = gv_encode();
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
        set_error("cuTensorMapEncodeTiled (dense fp16) failed: %d", (int)r);
        return VFMOE_ERR_CUDA;
    }
    return VFMOE_OK;
}

template <bool GATEUP>
static int launch_gv_dense(int N, const TcParams &prm, int grid, cudaStream_t st) {
    switch (N) {
        case 8: return launch_gv<GATEUP, 1, false, true>(prm, grid, st);
        case 16: return launch_gv<GATEUP, 2, false, true>(prm, grid, st);
        default: return launch_gv<GATEUP, 4, false, true>(prm, grid, st);
    }
}

int launch_dense_expert(const CUtensorMap &gate, const CUtensorMap &up, const CUtensorMap &down, const __half *xs,
                        int T, int H, int I, __half *act_s, float *y_s, float limit, int *err, int num_sms,
                        uint64_t wait_ns, cudaStream_t st) {
    if (T == 0) return VFMOE_OK;
    const int N = T <= 8 ? 8 : (T <= 16 ? 16 : 32);
    int rc;
    TcParams g{};
    g.wa = gate;
    g.wb = up;
    if ((rc = make_dense_map(&g.xt, xs, T, H, N))) return rc;
    g.dense_T = T;
    g.E = -1;
    g.K = H;
    g.M = I;
    g.ld_out = I;
    g.out = act_s;
    g.limit = limit;
    g.err = err;
    g.wait_ns = wait_ns;
    if ((rc = launch_gv_dense<true>(N, g, num_sms, st))) return rc;
    TcParams dn{};
    dn.wa = down;
    dn.wb = down;
    if ((rc = make_dense_map(&dn.xt, act_s, T, I, N))) return rc;
    dn.dense_T = T;
    dn.E = -1;
    dn.K = I;
    dn.M = H;
    dn.ld_out = H;
    dn.out = y_s;
    dn.limit = limit;
    dn.err = err;
    dn.wait_ns = wait_ns;
    return launch_gv_dense<false>(N, dn, num_sms, st);
}

int gemv_tokens_per_tile(int T, int k, int E) {
    const double avg = (double)T * k / E;
    int nt = 1;
    while (8 * nt < 2 * avg && nt < 4) nt <<= 1;
    return 8 * nt;
}

template <bool PREC>
static int launch_gv_n(bool gateup, int N, const TcParams &prm, int grid, cudaStream_t st) {
    if (gateup) {
        switch (N) {
            case 8: return launch_gv<true, 1, PREC>(prm, grid, st);
            case 16: return launch_gv<true, 2, PREC>(prm, grid, st);
            default: return launch_gv<true, 4, PREC>(prm, grid, st);
        }
    }
    switch (N) {
        case 8: return launch_gv<false, 1, PREC>(prm, grid, st);
        case 16: return launch_gv<false, 2, PREC>(prm, grid, st);
        default: return launch_gv<false, 4, PREC>(prm, grid, st);
    }
}

int launch_experts_gemv(const TcPlan &plan, const MoeArgs &a, cudaStream_t st, const std::function<void()> &mid,
                        const CUtensorMap &tok_gu, const CUtensorMap &tok_dn, const CUtensorMap *tok_gu2,
                        const CUtensorMap *tok_dn2) {
    const int N = gemv_tokens_per_tile(a.T, a.k, a.E);
    const int64_t rows = (int64_t)a.T * a.k + a.T;
    TcParams g{};
    g.wa = plan.gate64;
    g.wb = plan.up64;
    g.swa = plan.sh_gate64;
    g.swb = plan.sh_up64;
    g.tiled = plan.tiled;
    g.pa = plan.p_gate;
    g.pb = plan.p_up;
    g.spa = plan.p_sh_gate;
    g.spb = plan.p_sh_up;
    g.sa = plan.s_gate;
    g.sb = plan.s_up;
    g.xt = tok_gu;
    g.tiles = a.tiles;
    g.n_tiles = a.tile_counts;
    g.E = a.E;
    g.K = a.H;
    g.M = a.I;
    g.ld_out = a.I;
    g.out = a.act;
    g.limit = a.limit;
    g.err = a.err;
    g.prec = a.prec;
    if (a.prec) g.xt2 = *tok_gu2;
    g.out_plane = rows * a.I;
    g.wait_ns = a.wait_ns;
    g.stall = a.inject == VFMOE_INJECT_STALL_LOADS;
    const int grid = plan.num_sms;
    int rc = a.prec ? launch_gv_n<true>(true, N, g, grid, st) : launch_gv_n<false>(true, N, g, grid, st);
    if (rc) return rc;
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
    dn.xt = tok_dn;
    dn.tiles = a.tiles;            // same token tiles as gate/up (same N)
    dn.n_tiles = a.tile_counts;
    dn.E = a.E;
    dn.K = a.I;
    dn.M = a.H;
    dn.ld_out = a.H;
    dn.out = a.y;
    dn.limit = a.limit;
    dn.err = a.err;
    dn.prec = a.prec;
    if (a.prec) dn.xt2 = *tok_dn2;
    dn.out_plane = 0;
    dn.wait_ns = a.wait_ns;
    dn.stall = g.stall;
    return a.prec ? launch_gv_n<true>(false, N, dn, grid, st) : launch_gv_n<false>(false, N, dn, grid, st);
}

}  // namespace vfmoe
