// Token dispatch (permutation + gather) and weighted combine.
//
// Canonical order follows the reference host gather (native/glm53/glm_engine.vyb:2827-2845):
// for each expert e ascending, the tokens t ascending with idx[t, l] == e.  The shared
// expert is segment E and holds every token in order (glm_engine.vyb:2955-2989).
//
//   dispatch_kernel  one CTA per expert (+1 for the shared expert): offset = sum of lower
//                    counts, then a block-wide ordered compaction of the tokens that chose e
//                    (ballot + prefix), writing perm_tok[pos] and pos_of[t*k + l].
//   gather_kernel    x_perm[pos] = fp16(x[perm_tok[pos]]): 16-byte vector copies.
//   combine_kernel   out[t] = sum_l w[t,l] * y[pos_of[t,l]] + y[shared row of t]
//                    (glm_engine.vyb:2925-2938, :2991), lanes summed in lane order.
#include "common.cuh"
#include "kernels.h"

namespace vfmoe {

constexpr int kFrontMaxE = 1024;  // decode_front_kernel: experts scanned in shared memory

__global__ void __launch_bounds__(256) dispatch_kernel(const int32_t *__restrict__ idx, const int32_t *__restrict__ counts,
                                                       int T, int E, int k, int has_shared, int32_t *__restrict__ perm_tok,
                                                       int32_t *__restrict__ pos_of, int32_t *__restrict__ offsets,
                                                       int *__restrict__ err) {
    __shared__ int red[8];
    __shared__ int warp_tot[8];
    pdl_wait_then_release();
    const int e = blockIdx.x;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int64_t tk = (int64_t)T * k;
    if (e == E) {  // shared expert: identity segment after the routed rows
        // routed rows = sum of counts (T*k unless some lanes carry no expert, id < 0)
        int s = 0;
        for (int i = tid; i < E; i += 256) s += counts[i];
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
        if (lane == 0) red[warp] = s;
        __syncthreads();
        int routed = 0;
#pragma unroll
        for (int w = 0; w < 8; ++w) routed += red[w];
        if (has_shared)
            for (int t = tid; t < T; t += 256) perm_tok[routed + t] = t;
        if (tid == 0) {
            offsets[E] = routed;
            offsets[E + 1] = routed + (has_shared ? T : 0);
        }
        (void)tk;
        return;
    }
    int s = 0;
    for (int i = tid; i < e; i += 256) s += counts[i];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    if (lane == 0) red[warp] = s;
    __syncthreads();
    int off = 0;
#pragma unroll
    for (int w = 0; w < 8; ++w) off += red[w];
    if (tid == 0) offsets[e] = off;
    const int ne = counts[e];
    if (ne == 0) return;
    int running = 0;
    for (int base = 0; base < T; base += 256) {
        const int t = base + tid;
        int hit_lane = -1;
        if (t < T) {
            for (int l = 0; l < k; ++l)
                if (idx[(int64_t)t * k + l] == e) hit_lane = l;
        }
        const unsigned m = __ballot_sync(0xffffffffu, hit_lane >= 0);
        if (lane == 0) warp_tot[warp] = __popc(m);
        __syncthreads();
        int before = 0, total = 0;
#pragma unroll
        for (int w = 0; w < 8; ++w) {
            const int c = warp_tot[w];
            before += (w < warp) ? c : 0;
            total += c;
        }
        if (hit_lane >= 0) {
            const int pos = off + running + before + __popc(m & ((1u << lane) - 1u));
            perm_tok[pos] = t;
            pos_of[(int64_t)t * k + hit_lane] = pos;
        }
        running += total;
        __syncthreads();
    }
    if (tid == 0 && running != ne) raise_dev_error(err, DEV_BAD_COUNT);
}

// x[t] -> x_perm[pos] as fp16 by `nth` threads (tid = 0 .. nth - 1); H % 8 == 0.  With
// plane2 != 0 (fp32 x), plane2[pos * H + c] = fp16((x - fp16(x)) * 2^12): the residual that the
// split-precision decode GEMV multiplies as a second operand plane.
__device__ __forceinline__ void gather_row(const void *__restrict__ x, int x_dtype, int t, int64_t pos, int H,
                                           __half *__restrict__ xp, __half *__restrict__ plane2, int tid, int nth) {
    __half *dst = xp + pos * H;
    if (plane2 && x_dtype == VFMOE_DT_F32) {
        const float *src = reinterpret_cast<const float *>(x) + (int64_t)t * H;
        __half *dst2 = plane2 + pos * H;
        for (int c = tid * 4; c < H; c += nth * 4) {
            const float4 a = *reinterpret_cast<const float4 *>(src + c);
            const __half2 h0 = __floats2half2_rn(a.x, a.y), h1 = __floats2half2_rn(a.z, a.w);
            const float2 b0 = __half22float2(h0), b1 = __half22float2(h1);
            const __half2 l0 = __floats2half2_rn((a.x - b0.x) * 4096.f, (a.y - b0.y) * 4096.f);
            const __half2 l1 = __floats2half2_rn((a.z - b1.x) * 4096.f, (a.w - b1.y) * 4096.f);
            *reinterpret_cast<uint2 *>(dst + c) =
                make_uint2(*reinterpret_cast<const uint32_t *>(&h0), *reinterpret_cast<const uint32_t *>(&h1));
            *reinterpret_cast<uint2 *>(dst2 + c) =
                make_uint2(*reinterpret_cast<const uint32_t *>(&l0), *reinterpret_cast<const uint32_t *>(&l1));
        }
        return;
    }
    if (x_dtype == VFMOE_DT_BF16) {
        const __nv_bfloat16 *src = reinterpret_cast<const __nv_bfloat16 *>(x) + (int64_t)t * H;
        for (int c = tid * 8; c < H; c += nth * 8) {
            const uint4 raw = *reinterpret_cast<const uint4 *>(src + c);
            const uint32_t in[4] = {raw.x, raw.y, raw.z, raw.w};
            uint32_t o[4];
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const float a = __uint_as_float(in[i] << 16), b = __uint_as_float(in[i] & 0xFFFF0000u);
                const __half2 h = __floats2half2_rn(a, b);
                o[i] = *reinterpret_cast<const uint32_t *>(&h);
            }
            *reinterpret_cast<uint4 *>(dst + c) = make_uint4(o[0], o[1], o[2], o[3]);
        }
    } else {
        const float *src = reinterpret_cast<const float *>(x) + (int64_t)t * H;
        for (int c = tid * 8; c < H; c += nth * 8) {
            const float4 a = *reinterpret_cast<const float4 *>(src + c);
            const float4 b = *reinterpret_cast<const float4 *>(src + c + 4);
            const __half2 h0 = __floats2half2_rn(a.x, a.y), h1 = __floats2half2_rn(a.z, a.w);
            const __half2 h2 = __floats2half2_rn(b.x, b.y), h3 = __floats2half2_rn(b.z, b.w);
            *reinterpret_cast<uint4 *>(dst + c) =
                make_uint4(*reinterpret_cast<const uint32_t *>(&h0), *reinterpret_cast<const uint32_t *>(&h1),
                           *reinterpret_cast<const uint32_t *>(&h2), *reinterpret_cast<const uint32_t *>(&h3));
        }
    }
}

// One CTA (128 threads) per permuted row.  The grid may exceed the rows the dispatch produced
// (*n_rows, device-side); the extra CTAs exit.
__global__ void __launch_bounds__(128) gather_kernel(const void *__restrict__ x, int x_dtype,
                                                     const int32_t *__restrict__ perm_tok, int H,
                                                     __half *__restrict__ xp, const int32_t *__restrict__ n_rows,
                                                     __half *__restrict__ plane2) {
    pdl_wait_then_release();
    const int64_t pos = blockIdx.x;
    if (pos >= *n_rows) return;
    gather_row(x, x_dtype, perm_tok[pos], pos, H, xp, plane2, threadIdx.x, 128);
}

// Decode front end: dispatch, gather and the decode GEMV's token-tile list in one launch (the
// three launches above plus tc_plan_kernel cost a launch boundary each, most of their time at
// decode sizes).  One CTA of 256 threads per permuted row (grid T*k + T; CTAs past the rows
// exit).  Every CTA scans counts[0..E) into the segment offsets in shared memory, finds the
// segment e of its row pos and the row's token: the j-th token in ascending order that chose e,
// j = pos - offset(e) (the shared segment E holds every token in order).  It writes perm_tok[pos]
// and pos_of[t*k + l] and gathers x[t] into x_perm[pos], so the permutation is the one
// dispatch_kernel writes.  CTA 0 also writes offsets[0..E+1] and the tile lists of
// tc_plan_kernel for n_gu = n_dn = ng: ceil(n / ng) near-equal tiles per segment, segments in
// ascending order with the shared expert last.
__global__ void __launch_bounds__(256) decode_front_kernel(
    const int32_t *__restrict__ idx, const int32_t *__restrict__ counts, int T, int E, int k, int has_shared,
    const void *__restrict__ x, int x_dtype, int H, int32_t *__restrict__ perm_tok, int32_t *__restrict__ pos_of,
    int32_t *__restrict__ offsets, __half *__restrict__ xp, __half *__restrict__ plane2, int ng,
    int4 *__restrict__ tiles, int64_t cap, int32_t *__restrict__ tile_counts, int *__restrict__ err) {
    __shared__ int s_off[kFrontMaxE + 1];  // exclusive offsets of the routed segments, then their total
    __shared__ int s_wsum[8], s_wcnt[8];
    __shared__ int s_e, s_t, s_l;
    pdl_wait_then_release();
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;

    // exclusive scan of counts over the experts: thread owns experts [tid*per, tid*per + per)
    const int per = (E + 255) / 256;
    int cnt[kFrontMaxE / 256];
    int mine = 0;
#pragma unroll
    for (int i = 0; i < kFrontMaxE / 256; ++i) {
        const int e = tid * per + i;
        cnt[i] = (i < per && e < E) ? counts[e] : 0;
        mine += cnt[i];
    }
    int inc = mine;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const int v = __shfl_up_sync(0xffffffffu, inc, o);
        if (lane >= o) inc += v;
    }
    if (lane == 31) s_wsum[warp] = inc;
    if (tid == 0) s_e = s_t = s_l = -1;
    __syncthreads();
    int ex = inc - mine, routed = 0;
#pragma unroll
    for (int w = 0; w < 8; ++w) {
        ex += w < warp ? s_wsum[w] : 0;
        routed += s_wsum[w];
    }
#pragma unroll
    for (int i = 0; i < kFrontMaxE / 256; ++i) {
        const int e = tid * per + i;
        if (i < per && e < E) s_off[e] = ex;
        ex += cnt[i];
    }
    if (tid == 0) s_off[E] = routed;
    __syncthreads();
    const int rows = routed + (has_shared ? T : 0);

    if (blockIdx.x == 0) {
        for (int e = tid; e <= E; e += 256) offsets[e] = s_off[e];
        if (tid == 0) offsets[E + 1] = rows;
        // tile lists: thread owns segments [tid*per2, tid*per2 + per2) of E + has_shared
        const int nseg = E + (has_shared ? 1 : 0);
        const int per2 = (nseg + 255) / 256;
        int ntl = 0;
        for (int i = 0; i < per2; ++i) {
            const int e = tid * per2 + i;
            if (e < nseg) ntl += ((e < E ? s_off[e + 1] - s_off[e] : T) + ng - 1) / ng;
        }
        int ti = ntl;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const int v = __shfl_up_sync(0xffffffffu, ti, o);
            if (lane >= o) ti += v;
        }
        if (lane == 31) s_wcnt[warp] = ti;
        __syncthreads();
        int tp = ti - ntl, ttot = 0;
#pragma unroll
        for (int w = 0; w < 8; ++w) {
            tp += w < warp ? s_wcnt[w] : 0;
            ttot += s_wcnt[w];
        }
        for (int i = 0; i < per2; ++i) {
            const int e = tid * per2 + i;
            if (e >= nseg) break;
            const int r0 = e < E ? s_off[e] : routed, n = e < E ? s_off[e + 1] - s_off[e] : T;
            const int nt = (n + ng - 1) / ng;
            int row = r0;
            for (int j = 0; j < nt; ++j) {
                const int nr = n / nt + (j < n % nt ? 1 : 0);
                if (tp < cap) tiles[tp] = tiles[cap + tp] = make_int4(e, row, nr, 0);
                row += nr;
                ++tp;
            }
        }
        if (tid == 0) {
            tile_counts[0] = tile_counts[1] = (int32_t)(ttot < cap ? ttot : cap);
            if (ttot > cap) raise_dev_error(err, DEV_BAD_COUNT);
        }
        __syncthreads();  // s_wcnt is reused below
    }

    const int pos = blockIdx.x;
    if (pos >= rows) return;
    if (pos >= routed) {  // shared expert: token pos - routed
        if (tid == 0) perm_tok[pos] = pos - routed;
        gather_row(x, x_dtype, pos - routed, pos, H, xp, plane2, tid, 256);
        return;
    }
    // the routed segment holding pos (empty segments hold nothing)
    for (int e = tid; e < E; e += 256)
        if (s_off[e] <= pos && pos < s_off[e + 1]) s_e = e;
    __syncthreads();
    const int e = s_e;
    if (e < 0) return;  // unreachable: pos < routed lies in some segment
    const int j = pos - s_off[e];
    // the j-th token (ascending) with a lane on e: one thread per token, 256 tokens a round
    int seen = 0;
    for (int base = 0; base < T; base += 256) {
        const int t = base + tid;
        int hl = -1;
        if (t < T)
            for (int l = 0; l < k; ++l)
                if (idx[(int64_t)t * k + l] == e) hl = l;
        const unsigned m = __ballot_sync(0xffffffffu, hl >= 0);
        if (lane == 0) s_wcnt[warp] = __popc(m);
        __syncthreads();
        int before = seen, total = 0;
#pragma unroll
        for (int w = 0; w < 8; ++w) {
            before += w < warp ? s_wcnt[w] : 0;
            total += s_wcnt[w];
        }
        if (hl >= 0 && before + __popc(m & ((1u << lane) - 1u)) == j) {
            s_t = t;
            s_l = hl;
        }
        seen += total;
        __syncthreads();
        if (s_t >= 0) break;
    }
    const int t = s_t;
    if (t < 0) {  // counts and idx disagree
        if (tid == 0) raise_dev_error(err, DEV_BAD_COUNT);
        return;
    }
    if (tid == 0) {
        perm_tok[pos] = t;
        pos_of[(int64_t)t * k + s_l] = pos;
    }
    gather_row(x, x_dtype, t, pos, H, xp, plane2, tid, 256);
}

// grid (T, H / 1024): 256 threads x 4 columns; H % 4 == 0.  The token's k row positions and
// weights are staged in shared memory so the k row loads are independent of each other.
// y and y_shared are fp32 or fp16 (y_dtype); a negative position skips its lane.
__device__ __forceinline__ float4 ld4(const void *p, int64_t i, int dtype) {
    if (dtype == VFMOE_DT_F16) {
        const uint2 u = *reinterpret_cast<const uint2 *>(reinterpret_cast<const __half *>(p) + i);
        const float2 a = __half22float2(*reinterpret_cast<const __half2 *>(&u.x));
        const float2 b = __half22float2(*reinterpret_cast<const __half2 *>(&u.y));
        return make_float4(a.x, a.y, b.x, b.y);
    }
    return *reinterpret_cast<const float4 *>(reinterpret_cast<const float *>(p) + i);
}

__global__ void __launch_bounds__(256) combine_kernel(const void *__restrict__ y, int y_dtype,
                                                      const int32_t *__restrict__ pos_of, const float *__restrict__ w,
                                                      int T, int H, int k, const void *__restrict__ y_shared,
                                                      void *__restrict__ out, int out_dtype) {
    __shared__ int64_t sp[33];
    __shared__ float sw[32];
    pdl_wait_then_release();
    const int t = blockIdx.x;
    if (threadIdx.x < k) {
        const int32_t p = pos_of[(int64_t)t * k + threadIdx.x];
        sp[threadIdx.x] = p < 0 ? -1 : (int64_t)p * H;
        sw[threadIdx.x] = w ? w[(int64_t)t * k + threadIdx.x] : 1.0f;
    }
    __syncthreads();
    const int c = (blockIdx.y * 256 + threadIdx.x) * 4;
    if (c >= H) return;
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll 8
    for (int l = 0; l < k; ++l) {
        if (sp[l] < 0) continue;
        const float wl = sw[l];
        const float4 v = ld4(y, sp[l] + c, y_dtype);
        acc.x = fmaf(wl, v.x, acc.x);
        acc.y = fmaf(wl, v.y, acc.y);
        acc.z = fmaf(wl, v.z, acc.z);
        acc.w = fmaf(wl, v.w, acc.w);
    }
    if (y_shared) {
        const float4 v = ld4(y_shared, (int64_t)t * H + c, y_dtype);
        acc.x += v.x;
        acc.y += v.y;
        acc.z += v.z;
        acc.w += v.w;
    }
    const int64_t o = (int64_t)t * H + c;
    if (out_dtype == VFMOE_DT_BF16) {
        const __nv_bfloat162 lo = __floats2bfloat162_rn(acc.x, acc.y), hi = __floats2bfloat162_rn(acc.z, acc.w);
        uint2 pk;
        pk.x = *reinterpret_cast<const uint32_t *>(&lo);
        pk.y = *reinterpret_cast<const uint32_t *>(&hi);
        *reinterpret_cast<uint2 *>(reinterpret_cast<__nv_bfloat16 *>(out) + o) = pk;
    } else if (out_dtype == VFMOE_DT_F16) {
        const __half2 lo = __floats2half2_rn(acc.x, acc.y), hi = __floats2half2_rn(acc.z, acc.w);
        uint2 pk;
        pk.x = *reinterpret_cast<const uint32_t *>(&lo);
        pk.y = *reinterpret_cast<const uint32_t *>(&hi);
        *reinterpret_cast<uint2 *>(reinterpret_cast<__half *>(out) + o) = pk;
    } else {
        *reinterpret_cast<float4 *>(reinterpret_cast<float *>(out) + o) = acc;
    }
}

// Per-bucket counts of n ids in [0, nb): counts[b] += 1 (caller zeroes counts).  With
// skip_negative, ids < 0 mean "no bucket" and are not counted.
__global__ void count_kernel(const int32_t *__restrict__ ids, int64_t n, int nb, int32_t *__restrict__ counts,
                             int *__restrict__ err, int skip_negative) {
    const int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
    if (i >= n) return;
    const int b = ids[i];
    if (b >= 0 && b < nb)
        atomicAdd(&counts[b], 1);
    else if (!(skip_negative && b < 0))
        raise_dev_error(err, DEV_BAD_EXPERT_ID);
}

int launch_count(const int32_t *ids, int64_t n, int nb, int32_t *counts, int *err, cudaStream_t st,
                 int skip_negative) {
    if (n == 0) return VFMOE_OK;
    count_kernel<<<(unsigned)cdiv(n, 256), 256, 0, st>>>(ids, n, nb, counts, err, skip_negative);
    VF_LAUNCH_CHECK("count_kernel");
    return VFMOE_OK;
}

int launch_dispatch(const int32_t *idx, const int32_t *counts, int T, int E, int k, int has_shared, int32_t *perm_tok,
                    int32_t *pos_of, int32_t *offsets, int *err, cudaStream_t st) {
    VF_CUDA(launch_pdl(dispatch_kernel, dim3(E + 1), dim3(256), 0, st, idx, counts, T, E, k, has_shared, perm_tok, pos_of,
                       offsets, err));
    VF_LAUNCH_CHECK("dispatch_kernel");
    return VFMOE_OK;
}

int launch_gather(const void *x, int x_dtype, const int32_t *perm_tok, int64_t rows, int H, __half *xp,
                  const int32_t *n_rows, cudaStream_t st, int planes) {
    if (rows == 0) return VFMOE_OK;
    __half *plane2 = planes == 2 ? xp + rows * H : nullptr;
    VF_CUDA(launch_pdl(gather_kernel, dim3((unsigned)rows), dim3(128), 0, st, x, x_dtype, perm_tok, H, xp, n_rows,
                       plane2));
    VF_LAUNCH_CHECK("gather_kernel");
    return VFMOE_OK;
}

int launch_decode_front(const int32_t *idx, const int32_t *counts, int T, int E, int k, int has_shared, const void *x,
                        int x_dtype, int H, int32_t *perm_tok, int32_t *pos_of, int32_t *offsets, __half *xp, int planes,
                        int ng, int4 *tiles, int64_t cap, int32_t *tile_counts, int *err, cudaStream_t st) {
    if (T <= 0) return VFMOE_OK;
    if (E > kFrontMaxE || T > kDecodeFrontMaxT || H % 8 != 0) {
        set_error("decode front end: E=%d, T=%d, H=%d out of range", E, T, H);
        return VFMOE_ERR_UNSUPPORTED;
    }
    const int64_t rows = (int64_t)T * k + T;
    __half *plane2 = planes == 2 ? xp + rows * H : nullptr;
    VF_CUDA(launch_pdl(decode_front_kernel, dim3((unsigned)rows), dim3(256), 0, st, idx, counts, T, E, k, has_shared, x,
                       x_dtype, H, perm_tok, pos_of, offsets, xp, plane2, ng, tiles, cap, tile_counts, err));
    VF_LAUNCH_CHECK("decode_front_kernel");
    return VFMOE_OK;
}

int launch_combine(const void *y, int y_dtype, const int32_t *pos_of, const float *w, int T, int H, int k,
                   const void *y_shared, void *out, int out_dtype, cudaStream_t st) {
    if (T == 0) return VFMOE_OK;
    dim3 grid((unsigned)T, (unsigned)cdiv(H, 1024));
    VF_CUDA(launch_pdl(combine_kernel, grid, dim3(256), 0, st, y, y_dtype, pos_of, w, T, H, k, y_shared, out, out_dtype));
    VF_LAUNCH_CHECK("combine_kernel");
    return VFMOE_OK;
}

}  // namespace vfmoe
