// Expert parallelism behind the C ABI: token-level dispatch/combine over a fixed-capacity
// exchange, with NCCL send/recv inside the library (vfmoe_ep_forward) or a caller's own
// transport between the phase entry points (vfmoe_ep_prepare / _shared / _experts / _combine).
//
// The reference has no multi-GPU code; its callers that would run expert-parallel are the
// tail_site router, expert loop and shared expert (native/glm53/glm_engine.vyb:2728-2991) and the
// prefill driver (native/host/glm_prefill.vyb:1458).
//
// One layer forward on rank r of N, all on the caller's stream, no host synchronization:
//   prepare  route the rank's T tokens; plan one send entry per (token, destination rank that owns
//            one of its k experts), entries of destination d at d*cap + i, i < count[d] <= T <= cap;
//            pack the send rows.  Entries i >= count[d] carry slot -1 in every lane.  The block
//            for d == r goes straight into the receive buffers.
//   exchange rows, lane slots and lane weights of block d to rank d (NCCL send/recv, every peer
//            block is cap entries whatever its count, so no count crosses to the host).
//   shared   the shared expert on the rank's own tokens (overlaps the exchange on a second stream).
//   experts  the rank's experts on the N*cap received rows, each row's local lanes summed with
//            their weights into one partial row (fp16, or fp32 for fp32 layers); padding rows
//            have no lanes and cost nothing in the expert kernels.
//   exchange partial rows back (block d to rank d).
//   combine  out[t] = sum over destinations of the returned partial + shared(x[t]).
// The capacity cap (>= every rank's T, equal on all ranks) fixes the exchange sizes: each
// rank sends N-1 blocks of cap rows each way, 1.0-1.5x the rows a count-exact exchange would
// move at 2-8 ranks, in exchange for no host round trip between route and exchange.
#include <dlfcn.h>
#include <nccl.h>

#include <chrono>
#include <cstring>
#include <mutex>
#include <string>
#include <thread>
#include <type_traits>
#include <unordered_map>
#include <vector>

#include "layer.h"

namespace vfmoe {

// ----------------------------------------------------------------------------- kernels
// Virtual expert of lane (t, l): expert e, or its copy when e has one and t + l is odd, so a
// copy takes about half of its expert's lanes even at one token per rank.
__device__ __forceinline__ int virtual_expert(int e, int t, int l, const int32_t *copy_of) {
    if (copy_of) {
        const int c = copy_of[e];
        if (c >= 0 && ((t + l) & 1)) return c;
    }
    return e;
}

// Fixed-capacity token-level send plan (one CTA, 1024 threads).  For every destination d:
// the tokens t (ascending) with a lane whose virtual expert d owns get entries d*cap + i;
// entry lanes carry (owner-local slot, weight) or (-1, 0).  Entries i >= count[d] get slot -1.
// The block of d == my_rank is written into the receive arrays (recv_slot, recv_w).
// pos_of[t * n_ranks + d] = d*cap + i or -1.
__global__ void __launch_bounds__(1024) ep_plan_fixed_kernel(
    const int32_t *__restrict__ idx, const float *__restrict__ w, int T, int k, int E, const int32_t *__restrict__ owner,
    const int32_t *__restrict__ local_slot, const int32_t *__restrict__ copy_of, int n_ranks, int my_rank, int cap,
    int32_t *__restrict__ send_counts, int32_t *__restrict__ send_tok, int32_t *__restrict__ send_slot,
    float *__restrict__ send_w, int32_t *__restrict__ recv_slot, float *__restrict__ recv_w,
    int32_t *__restrict__ pos_of, int *__restrict__ err) {
    __shared__ int warp_tot[32];
    pdl_wait_then_release();
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    for (int d = 0; d < n_ranks; ++d) {
        int32_t *slot_dst = (d == my_rank ? recv_slot : send_slot) + (int64_t)d * cap * k;
        float *w_dst = (d == my_rank ? recv_w : send_w) + (int64_t)d * cap * k;
        int running = 0;
        for (int c = 0; c < T; c += 1024) {
            const int t = c + tid;
            bool hit = false;
            if (t < T) {
                for (int l = 0; l < k; ++l) {
                    const int e = idx[(int64_t)t * k + l];
                    int o = -1;
                    if (e >= 0 && e < E) o = owner[virtual_expert(e, t, l, copy_of)];
                    if (o < 0 || o >= n_ranks) {
                        if (d == 0) raise_dev_error(err, DEV_BAD_EXPERT_ID);
                    } else if (o == d) {
                        hit = true;
                    }
                }
            }
            const unsigned m = __ballot_sync(0xffffffffu, hit);
            if (lane == 0) warp_tot[warp] = __popc(m);
            __syncthreads();
            int before = 0, total = 0;
            for (int q = 0; q < 32; ++q) {
                const int v = warp_tot[q];
                before += q < warp ? v : 0;
                total += v;
            }
            if (t < T) {
                int pos = -1;
                if (hit) {
                    const int i = running + before + __popc(m & ((1u << lane) - 1u));
                    pos = d * cap + i;
                    send_tok[pos] = t;
                    for (int l = 0; l < k; ++l) {
                        const int e = idx[(int64_t)t * k + l];
                        int sl = -1;
                        float wt = 0.f;
                        if (e >= 0 && e < E) {
                            const int v = virtual_expert(e, t, l, copy_of);
                            if (owner[v] == d) {
                                sl = local_slot[v];
                                wt = w[(int64_t)t * k + l];
                            }
                        }
                        slot_dst[(int64_t)i * k + l] = sl;
                        w_dst[(int64_t)i * k + l] = wt;
                    }
                }
                pos_of[(int64_t)t * n_ranks + d] = pos;
            }
            running += total;
            __syncthreads();
        }
        // padding entries: no lanes
        for (int64_t q = (int64_t)running * k + tid; q < (int64_t)cap * k; q += 1024) {
            slot_dst[q] = -1;
            w_dst[q] = 0.f;
        }
        if (tid == 0) send_counts[d] = running;
    }
}

// Send rows: grid (cap, n_ranks), 128 threads; entry (d, i) with i < count[d] copies
// x[send_tok[d*cap+i]] into send_rows (recv_rows for d == my_rank) at row d*cap + i.
__global__ void __launch_bounds__(128) ep_pack_fixed_kernel(const uint8_t *__restrict__ x, int64_t row_bytes, int cap,
                                                            int my_rank, const int32_t *__restrict__ send_counts,
                                                            const int32_t *__restrict__ send_tok,
                                                            uint8_t *__restrict__ send_rows,
                                                            uint8_t *__restrict__ recv_rows) {
    pdl_wait_then_release();
    const int i = blockIdx.x, d = blockIdx.y;
    if (i >= send_counts[d]) return;
    const int64_t e = (int64_t)d * cap + i;
    const int t = send_tok[e];
    const uint4 *src = reinterpret_cast<const uint4 *>(x + (int64_t)t * row_bytes);
    uint4 *dst = reinterpret_cast<uint4 *>((d == my_rank ? recv_rows : send_rows) + e * row_bytes);
    for (int64_t q = threadIdx.x; q < row_bytes / 16; q += 128) dst[q] = src[q];
}

__global__ void fill_i32_kernel(int32_t *p, int64_t n, int32_t v) {
    const int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
    if (i < n) p[i] = v;
}

// ----------------------------------------------------------------------------- workspace
// Byte offsets of the expert-parallel workspace (vfmoe_ep_buffers exposes the exchange buffers).
struct EpLayout {
    int64_t idx, w, counts, send_tok, pos_of, shared_slot;
    int64_t send_slot, recv_slot, send_w, recv_w;      // [N][cap][k]
    int64_t send_rows, recv_rows, y_part, y_back;      // [N][cap][H]
    int64_t y_shared;                                  // [cap][H]
    int64_t inner, inner_bytes, total;
    int64_t row_bytes, part_bytes;                     // bytes of one row: x dtype, partial dtype
};

static int part_dtype(const Layer &L) { return L.d.out_dtype == VFMOE_DT_F32 ? VFMOE_DT_F32 : VFMOE_DT_F16; }

static EpLayout ep_layout(const Layer &L, int64_t cap) {
    EpLayout o{};
    const int64_t N = L.ep.n_ranks, k = L.k, H = L.H;
    o.row_bytes = H * (L.d.x_dtype == VFMOE_DT_F32 ? 4 : 2);
    o.part_bytes = H * (part_dtype(L) == VFMOE_DT_F32 ? 4 : 2);
    int64_t p = 0;
    auto take = [&](int64_t bytes) {
        const int64_t at = p;
        p = align_up(p + bytes, 256);
        return at;
    };
    o.idx = take(cap * k * 4);
    o.w = take(cap * k * 4);
    o.counts = take(N * 4);
    o.send_tok = take(N * cap * 4);
    o.pos_of = take(cap * N * 4);
    o.shared_slot = take(cap * 4);
    o.send_slot = take(N * cap * k * 4);
    o.recv_slot = take(N * cap * k * 4);
    o.send_w = take(N * cap * k * 4);
    o.recv_w = take(N * cap * k * 4);
    o.send_rows = take(N * cap * o.row_bytes);
    o.recv_rows = take(N * cap * o.row_bytes);
    o.y_part = take(N * cap * o.part_bytes);
    o.y_back = take(N * cap * o.part_bytes);
    o.y_shared = take(cap * o.part_bytes);
    const int64_t a = ws_layout(L, cap).total, b = ws_layout(L, N * cap, (int)k).total, c = ws_layout(L, cap, 1).total;
    o.inner_bytes = std::max(a, std::max(b, c));
    o.inner = take(o.inner_bytes);
    o.total = p;
    return o;
}

static int ep_check(Layer *L, int64_t T, int64_t cap, const char *who) {
    if (!L->ep.ready) {
        set_error("%s: no expert-parallel placement on this layer (vfmoe_ep_set_placement)", who);
        return VFMOE_ERR_INVALID;
    }
    if (T < 0 || cap <= 0 || T > cap || cap > ((int64_t)1 << 22) || (int64_t)L->ep.n_ranks * cap > ((int64_t)1 << 24)) {
        set_error("%s: need 0 <= T <= t_cap, t_cap * n_ranks <= 2^24 (T=%lld, t_cap=%lld)", who, (long long)T,
                  (long long)cap);
        return VFMOE_ERR_INVALID;
    }
    return VFMOE_OK;
}

// Workspace base for an expert-parallel call (caller's, or the handle's own grown on demand).
static int ep_ws(Layer &L, const EpLayout &lay, int64_t ws, int64_t ws_bytes, char **base) {
    if (ws) {
        if (ws_bytes < lay.total) {
            set_error("expert-parallel workspace too small: %lld < %lld bytes", (long long)ws_bytes,
                      (long long)lay.total);
            return VFMOE_ERR_WORKSPACE;
        }
        if (ws % 256) {
            set_error("workspace must be 256-byte aligned");
            return VFMOE_ERR_INVALID;
        }
        *base = reinterpret_cast<char *>(ws);
        return VFMOE_OK;
    }
    if (L.own_ws_bytes < lay.total) {
        if (L.own_ws) VF_CUDA(cudaFree(L.own_ws));
        L.own_ws = nullptr;
        L.own_ws_bytes = 0;
        VF_CUDA(cudaMalloc(&L.own_ws, lay.total));
        L.own_ws_bytes = lay.total;
    }
    *base = reinterpret_cast<char *>(L.own_ws);
    return VFMOE_OK;
}

static int ep_prepare_impl(Layer &L, int64_t x, int64_t T, int64_t cap, char *base, const EpLayout &lay,
                           int32_t *idx, float *w, cudaStream_t st) {
    const WsLayout rl = ws_layout(L, T);
    int rc;
    if (T > 0 && (rc = route_impl(L, x, T, base + lay.inner, rl, &idx, &w, st))) return rc;
    const EpPlacement &P = L.ep;
    auto at = [&](int64_t off) { return base + off; };
    VF_CUDA(launch_pdl(ep_plan_fixed_kernel, dim3(1), dim3(1024), 0, st, (const int32_t *)idx, (const float *)w, (int)T,
                       L.k, L.E, (const int32_t *)P.owner, (const int32_t *)P.local_slot, (const int32_t *)P.copy_of,
                       P.n_ranks, P.rank, (int)cap, (int32_t *)at(lay.counts), (int32_t *)at(lay.send_tok),
                       (int32_t *)at(lay.send_slot), (float *)at(lay.send_w), (int32_t *)at(lay.recv_slot),
                       (float *)at(lay.recv_w), (int32_t *)at(lay.pos_of), L.dev_err));
    VF_LAUNCH_CHECK("ep_plan_fixed_kernel");
    if (T == 0) return VFMOE_OK;
    VF_CUDA(launch_pdl(ep_pack_fixed_kernel, dim3((unsigned)T, (unsigned)P.n_ranks), dim3(128), 0, st,
                       (const uint8_t *)x, lay.row_bytes, (int)cap, P.rank, (const int32_t *)at(lay.counts),
                       (const int32_t *)at(lay.send_tok), (uint8_t *)at(lay.send_rows), (uint8_t *)at(lay.recv_rows)));
    VF_LAUNCH_CHECK("ep_pack_fixed_kernel");
    return VFMOE_OK;
}

static int ep_shared_impl(Layer &L, int64_t x, int64_t T, char *base, const EpLayout &lay, cudaStream_t st) {
    if (T == 0) return VFMOE_OK;
    if (!L.has_shared) {
        VF_CUDA(cudaMemsetAsync(base + lay.y_shared, 0, T * lay.part_bytes, st));
        return VFMOE_OK;
    }
    if (L.dense_sh) {
        // the bf16-stored shared expert runs its own dense GEMVs (workspace regions of a T-row
        // forward inside the inner workspace), then its rows become partial rows
        char *in = base + lay.inner;
        const WsLayout wl = ws_layout(L, T);
        __half *xs = reinterpret_cast<__half *>(in + wl.xs);
        float *ys = reinterpret_cast<float *>(in + wl.y_s);
        int rc = launch_to_f16(reinterpret_cast<const void *>(x), (int)L.d.x_dtype, T * L.H, xs, st);
        if (!rc)
            rc = launch_dense_expert(L.dsh_gate, L.dsh_up, L.dsh_down, xs, (int)T, L.H, L.I,
                                     reinterpret_cast<__half *>(in + wl.act_s), ys, (float)L.d.swiglu_limit, L.dev_err,
                                     L.num_sms, L.wait_ns, st);
        if (rc) return rc;
        if (part_dtype(L) == VFMOE_DT_F32) {
            VF_CUDA(cudaMemcpyAsync(base + lay.y_shared, ys, T * lay.part_bytes, cudaMemcpyDeviceToDevice, st));
            return VFMOE_OK;
        }
        return launch_to_f16(ys, VFMOE_DT_F32, T * L.H, reinterpret_cast<__half *>(base + lay.y_shared), st);
    }
    int32_t *ss = reinterpret_cast<int32_t *>(base + lay.shared_slot);
    fill_i32_kernel<<<(unsigned)cdiv(T, 256), 256, 0, st>>>(ss, T, L.n_local);
    VF_LAUNCH_CHECK("fill_i32_kernel");
    return rows_impl(L, x, L.d.x_dtype, ss, T, 1, nullptr, reinterpret_cast<int64_t>(base + lay.y_shared),
                     part_dtype(L), 1, reinterpret_cast<int64_t>(base + lay.inner), lay.inner_bytes, st);
}

static int ep_experts_impl(Layer &L, int64_t cap, char *base, const EpLayout &lay, cudaStream_t st) {
    const int64_t n = (int64_t)L.ep.n_ranks * cap;
    int rc = rows_impl(L, reinterpret_cast<int64_t>(base + lay.recv_rows), L.d.x_dtype,
                       reinterpret_cast<const int32_t *>(base + lay.recv_slot), n, L.k,
                       reinterpret_cast<const float *>(base + lay.recv_w), reinterpret_cast<int64_t>(base + lay.y_part),
                       part_dtype(L), 1, reinterpret_cast<int64_t>(base + lay.inner), lay.inner_bytes, st);
    if (rc) return rc;
    // this rank's own block returns without crossing a link
    const int64_t blk = cap * lay.part_bytes, off = (int64_t)L.ep.rank * blk;
    VF_CUDA(cudaMemcpyAsync(base + lay.y_back + off, base + lay.y_part + off, blk, cudaMemcpyDeviceToDevice, st));
    return VFMOE_OK;
}

static int ep_combine_impl(Layer &L, int64_t T, char *base, const EpLayout &lay, int64_t out, cudaStream_t st) {
    if (T == 0) return VFMOE_OK;
    return launch_combine(base + lay.y_back, part_dtype(L), reinterpret_cast<const int32_t *>(base + lay.pos_of),
                          nullptr, (int)T, L.H, L.ep.n_ranks, base + lay.y_shared, reinterpret_cast<void *>(out),
                          (int)L.d.out_dtype, st);
}

// ----------------------------------------------------------------------------- NCCL (loaded at run time)
// The library does not link NCCL: vfmoe_ep_init opens libnccl.so.2 (the copy already loaded in
// the process, if any), so a host that never runs expert-parallel needs no NCCL at all.
struct NcclApi {
    bool ok = false;
    std::string why;
    ncclResult_t (*GetUniqueId)(ncclUniqueId *);
    ncclResult_t (*CommInitRankConfig)(ncclComm_t *, int, ncclUniqueId, int, ncclConfig_t *);
    ncclResult_t (*CommGetAsyncError)(ncclComm_t, ncclResult_t *);
    ncclResult_t (*CommAbort)(ncclComm_t);
    ncclResult_t (*CommDestroy)(ncclComm_t);
    ncclResult_t (*Send)(const void *, size_t, ncclDataType_t, int, ncclComm_t, cudaStream_t);
    ncclResult_t (*Recv)(void *, size_t, ncclDataType_t, int, ncclComm_t, cudaStream_t);
    ncclResult_t (*GroupStart)();
    ncclResult_t (*GroupEnd)();
    const char *(*GetErrorString)(ncclResult_t);
    ncclResult_t (*GetVersion)(int *);
};

static NcclApi &nccl() {
    static NcclApi api;
    static std::once_flag once;
    std::call_once(once, []() {
        void *h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_LOCAL);
        if (!h) h = dlopen("libnccl.so", RTLD_NOW | RTLD_LOCAL);
        if (!h) {
            const char *e = dlerror();
            api.why = std::string("cannot open libnccl.so.2: ") + (e ? e : "?");
            return;
        }
        bool all = true;
        auto sym = [&](auto &fp, const char *name) {
            void *p = dlsym(h, name);
            if (!p) all = false;
            fp = reinterpret_cast<std::remove_reference_t<decltype(fp)>>(p);
        };
        sym(api.GetUniqueId, "ncclGetUniqueId");
        sym(api.CommInitRankConfig, "ncclCommInitRankConfig");
        sym(api.CommGetAsyncError, "ncclCommGetAsyncError");
        sym(api.CommAbort, "ncclCommAbort");
        sym(api.CommDestroy, "ncclCommDestroy");
        sym(api.Send, "ncclSend");
        sym(api.Recv, "ncclRecv");
        sym(api.GroupStart, "ncclGroupStart");
        sym(api.GroupEnd, "ncclGroupEnd");
        sym(api.GetErrorString, "ncclGetErrorString");
        sym(api.GetVersion, "ncclGetVersion");
        if (!all) {
            api.why = "libnccl.so.2 lacks a required symbol (NCCL >= 2.14 needed)";
            return;
        }
        api.ok = true;
    });
    return api;
}

static int nccl_fail(ncclResult_t r, const char *what) {
    set_error("%s failed: %s", what, nccl().GetErrorString ? nccl().GetErrorString(r) : "?");
    return VFMOE_ERR_NCCL;
}

struct EpComm {
    ncclComm_t comm = nullptr;
    int nranks = 0, rank = 0, device = 0;
    int64_t timeout_ms = 0;
    cudaStream_t side = nullptr;
    cudaEvent_t ev_fork = nullptr, ev_join = nullptr;
};

static std::mutex g_comm_mu;
static std::unordered_map<int64_t, EpComm *> g_comms;
static int64_t g_next_comm = 1;

static EpComm *get_comm(int64_t h) {
    std::lock_guard<std::mutex> lk(g_comm_mu);
    auto it = g_comms.find(h);
    if (it == g_comms.end()) {
        set_error("unknown expert-parallel communicator %lld", (long long)h);
        return nullptr;
    }
    return it->second;
}

// A non-blocking communicator: wait (bounded) until its pending host-side work is done.
static int nccl_settle(EpComm &c, const char *what) {
    const auto t0 = std::chrono::steady_clock::now();
    while (true) {
        ncclResult_t st = ncclInProgress;
        ncclResult_t r = nccl().CommGetAsyncError(c.comm, &st);
        if (r != ncclSuccess) return nccl_fail(r, what);
        if (st == ncclSuccess) return VFMOE_OK;
        if (st != ncclInProgress) return nccl_fail(st, what);
        if (c.timeout_ms > 0 &&
            std::chrono::duration_cast<std::chrono::milliseconds>(std::chrono::steady_clock::now() - t0).count() >
                c.timeout_ms) {
            set_error("%s: NCCL did not finish within %lld ms", what, (long long)c.timeout_ms);
            return VFMOE_ERR_NCCL;
        }
        std::this_thread::yield();
    }
}

// Block d (bytes each) of send to rank d, block d of recv from rank d, for every peer d != rank.
static void exchange_blocks(EpComm &c, const char *send, char *recv, int64_t blk, cudaStream_t st,
                            ncclResult_t &r) {
    for (int d = 0; d < c.nranks && r == ncclSuccess; ++d) {
        if (d == c.rank) continue;
        r = nccl().Send(send + d * blk, (size_t)blk, ncclUint8, d, c.comm, st);
        if (r == ncclSuccess) r = nccl().Recv(recv + d * blk, (size_t)blk, ncclUint8, d, c.comm, st);
    }
}

}  // namespace vfmoe

using namespace vfmoe;

extern "C" {

int vfmoe_ep_unique_id(void *id_out, int64_t n) {
    if (!id_out || n < (int64_t)sizeof(ncclUniqueId)) {
        set_error("vfmoe_ep_unique_id: need a buffer of %d bytes", (int)sizeof(ncclUniqueId));
        return VFMOE_ERR_INVALID;
    }
    NcclApi &api = nccl();
    if (!api.ok) {
        set_error("vfmoe_ep_unique_id: %s", api.why.c_str());
        return VFMOE_ERR_NCCL;
    }
    ncclUniqueId id;
    ncclResult_t r = api.GetUniqueId(&id);
    if (r != ncclSuccess) return nccl_fail(r, "ncclGetUniqueId");
    memcpy(id_out, &id, sizeof(id));
    return VFMOE_OK;
}

int64_t vfmoe_ep_init(int64_t nranks, int64_t rank, const void *unique_id, int64_t timeout_ms) {
    if (nranks <= 0 || nranks > 32 || rank < 0 || rank >= nranks || !unique_id || timeout_ms < 0) {
        set_error("vfmoe_ep_init: bad arguments (1 <= nranks <= 32, 0 <= rank < nranks, id required)");
        return VFMOE_ERR_INVALID;
    }
    NcclApi &api = nccl();
    if (!api.ok) {
        set_error("vfmoe_ep_init: %s", api.why.c_str());
        return VFMOE_ERR_NCCL;
    }
    EpComm *c = new EpComm();
    c->nranks = (int)nranks;
    c->rank = (int)rank;
    c->timeout_ms = timeout_ms;
    cudaError_t e = cudaGetDevice(&c->device);
    if (e == cudaSuccess) e = cudaStreamCreateWithFlags(&c->side, cudaStreamNonBlocking);
    if (e == cudaSuccess) e = cudaEventCreateWithFlags(&c->ev_fork, cudaEventDisableTiming);
    if (e == cudaSuccess) e = cudaEventCreateWithFlags(&c->ev_join, cudaEventDisableTiming);
    if (e != cudaSuccess) {
        cuda_fail(e, "vfmoe_ep_init (stream, events)", __FILE__, __LINE__);
        if (c->side) cudaStreamDestroy(c->side);
        if (c->ev_fork) cudaEventDestroy(c->ev_fork);
        delete c;
        return VFMOE_ERR_CUDA;
    }
    ncclUniqueId id;
    memcpy(&id, unique_id, sizeof(id));
    ncclConfig_t cfg = NCCL_CONFIG_INITIALIZER;
    cfg.blocking = 0;  // init returns at once; the wait for the other ranks is bounded below
    ncclResult_t r = api.CommInitRankConfig(&c->comm, (int)nranks, id, (int)rank, &cfg);
    int rc = VFMOE_OK;
    if (r != ncclSuccess && r != ncclInProgress)
        rc = nccl_fail(r, "ncclCommInitRankConfig");
    else
        rc = nccl_settle(*c, "vfmoe_ep_init (waiting for every rank to join)");
    if (rc) {
        if (c->comm) api.CommAbort(c->comm);
        cudaEventDestroy(c->ev_fork);
        cudaEventDestroy(c->ev_join);
        cudaStreamDestroy(c->side);
        delete c;
        return rc;
    }
    std::lock_guard<std::mutex> lk(g_comm_mu);
    const int64_t h = g_next_comm++;
    g_comms[h] = c;
    return h;
}

int vfmoe_ep_destroy(int64_t comm) {
    EpComm *c;
    {
        std::lock_guard<std::mutex> lk(g_comm_mu);
        auto it = g_comms.find(comm);
        if (it == g_comms.end()) {
            set_error("unknown expert-parallel communicator %lld", (long long)comm);
            return VFMOE_ERR_HANDLE;
        }
        c = it->second;
        g_comms.erase(it);
    }
    int rc = VFMOE_OK;
    if (c->comm) {
        cudaStreamSynchronize(c->side);
        ncclResult_t r = nccl().CommDestroy(c->comm);
        if (r != ncclSuccess && r != ncclInProgress) rc = nccl_fail(r, "ncclCommDestroy");
    }
    cudaEventDestroy(c->ev_fork);
    cudaEventDestroy(c->ev_join);
    cudaStreamDestroy(c->side);
    delete c;
    return rc;
}

int vfmoe_ep_set_placement(int64_t handle, int64_t n_ranks, int64_t rank, const int32_t *owner, int64_t n_virtual,
                           const int32_t *replica_of, int64_t n_replicas) {
    Layer *L = get_layer(handle);
    if (!L) return VFMOE_ERR_HANDLE;
    if (n_ranks <= 0 || n_ranks > 32 || rank < 0 || rank >= n_ranks || !owner || n_replicas < 0 ||
        n_virtual != L->E + n_replicas || (n_replicas > 0 && !replica_of)) {
        set_error("vfmoe_ep_set_placement: bad arguments (n_virtual must be n_experts + n_replicas)");
        return VFMOE_ERR_INVALID;
    }
    std::vector<int32_t> slot(n_virtual), copy(L->E, -1);
    std::vector<int> seen(n_ranks, 0);
    for (int64_t v = 0; v < n_virtual; ++v) {
        const int o = owner[v];
        if (o < 0 || o >= n_ranks) {
            set_error("vfmoe_ep_set_placement: owner[%lld] = %d is not a rank", (long long)v, o);
            return VFMOE_ERR_INVALID;
        }
        slot[v] = seen[o]++;
    }
    if (seen[rank] != L->n_local) {
        set_error("vfmoe_ep_set_placement: rank %lld owns %d virtual experts but the layer holds %d", (long long)rank,
                  seen[rank], L->n_local);
        return VFMOE_ERR_INVALID;
    }
    for (int64_t j = 0; j < n_replicas; ++j) {
        const int e = replica_of[j];
        if (e < 0 || e >= L->E || copy[e] >= 0) {
            set_error("vfmoe_ep_set_placement: replica_of[%lld] = %d invalid or repeated", (long long)j, e);
            return VFMOE_ERR_INVALID;
        }
        copy[e] = (int32_t)(L->E + j);
    }
    EpPlacement &P = L->ep;
    if (!P.owner) {
        VF_CUDA(cudaMalloc(&P.owner, (L->E + 1024) * 4 * 2 + L->E * 4));  // room for any n_virtual <= E + 1024
        P.local_slot = P.owner + (L->E + 1024);
        P.copy_of = P.local_slot + (L->E + 1024);
    }
    if (n_virtual > L->E + 1024) {
        set_error("vfmoe_ep_set_placement: more than 1024 replicas");
        return VFMOE_ERR_INVALID;
    }
    VF_CUDA(cudaMemcpy(P.owner, owner, n_virtual * 4, cudaMemcpyHostToDevice));
    VF_CUDA(cudaMemcpy(P.local_slot, slot.data(), n_virtual * 4, cudaMemcpyHostToDevice));
    VF_CUDA(cudaMemcpy(P.copy_of, copy.data(), L->E * 4, cudaMemcpyHostToDevice));
    P.n_ranks = (int)n_ranks;
    P.rank = (int)rank;
    P.n_virtual = (int)n_virtual;
    P.ready = 1;
    return VFMOE_OK;
}

int64_t vfmoe_ep_workspace_bytes(int64_t handle, int64_t t_cap) {
    Layer *L = get_layer(handle);
    if (!L) return VFMOE_ERR_HANDLE;
    if (int rc = ep_check(L, 0, t_cap, "vfmoe_ep_workspace_bytes")) return rc;
    return ep_layout(*L, t_cap).total;
}

int vfmoe_ep_buffers(int64_t handle, int64_t t_cap, int64_t *offsets, int64_t n) {
    Layer *L = get_layer(handle);
    if (!L) return VFMOE_ERR_HANDLE;
    if (int rc = ep_check(L, 0, t_cap, "vfmoe_ep_buffers")) return rc;
    if (!offsets || n < VFMOE_EP_BUF_COUNT) {
        set_error("vfmoe_ep_buffers: need room for %d values", VFMOE_EP_BUF_COUNT);
        return VFMOE_ERR_INVALID;
    }
    const EpLayout o = ep_layout(*L, t_cap);
    const int64_t k = L->k;
    offsets[VFMOE_EP_SEND_ROWS] = o.send_rows;
    offsets[VFMOE_EP_RECV_ROWS] = o.recv_rows;
    offsets[VFMOE_EP_ROWS_BLOCK] = t_cap * o.row_bytes;
    offsets[VFMOE_EP_SEND_SLOTS] = o.send_slot;
    offsets[VFMOE_EP_RECV_SLOTS] = o.recv_slot;
    offsets[VFMOE_EP_SEND_WEIGHTS] = o.send_w;
    offsets[VFMOE_EP_RECV_WEIGHTS] = o.recv_w;
    offsets[VFMOE_EP_LANES_BLOCK] = t_cap * k * 4;
    offsets[VFMOE_EP_SEND_PARTIALS] = o.y_part;
    offsets[VFMOE_EP_RECV_PARTIALS] = o.y_back;
    offsets[VFMOE_EP_PARTIALS_BLOCK] = t_cap * o.part_bytes;
    offsets[VFMOE_EP_SEND_COUNTS] = o.counts;
    return VFMOE_OK;
}

int vfmoe_ep_prepare(int64_t handle, int64_t x, int64_t T, int64_t t_cap, int64_t idx_out, int64_t w_out,
                     int64_t workspace, int64_t ws_bytes, int64_t stream) {
    Layer *L = get_layer(handle);
    if (!L) return VFMOE_ERR_HANDLE;
    if (int rc = ep_check(L, T, t_cap, "vfmoe_ep_prepare")) return rc;
    if (T > 0 && (!x || (x & 15))) {
        set_error("vfmoe_ep_prepare: x must be non-null and 16-byte aligned");
        return VFMOE_ERR_INVALID;
    }
    const EpLayout lay = ep_layout(*L, t_cap);
    char *base;
    if (int rc = ep_ws(*L, lay, workspace, ws_bytes, &base)) return rc;
    int32_t *idx = idx_out ? reinterpret_cast<int32_t *>(idx_out) : reinterpret_cast<int32_t *>(base + lay.idx);
    float *w = w_out ? reinterpret_cast<float *>(w_out) : reinterpret_cast<float *>(base + lay.w);
    return ep_prepare_impl(*L, x, T, t_cap, base, lay, idx, w, reinterpret_cast<cudaStream_t>(stream));
}

int vfmoe_ep_shared(int64_t handle, int64_t x, int64_t T, int64_t t_cap, int64_t workspace, int64_t ws_bytes,
                    int64_t stream) {
    Layer *L = get_layer(handle);
    if (!L) return VFMOE_ERR_HANDLE;
    if (int rc = ep_check(L, T, t_cap, "vfmoe_ep_shared")) return rc;
    const EpLayout lay = ep_layout(*L, t_cap);
    char *base;
    if (int rc = ep_ws(*L, lay, workspace, ws_bytes, &base)) return rc;
    return ep_shared_impl(*L, x, T, base, lay, reinterpret_cast<cudaStream_t>(stream));
}

int vfmoe_ep_experts(int64_t handle, int64_t t_cap, int64_t workspace, int64_t ws_bytes, int64_t stream) {
    Layer *L = get_layer(handle);
    if (!L) return VFMOE_ERR_HANDLE;
    if (int rc = ep_check(L, 0, t_cap, "vfmoe_ep_experts")) return rc;
    const EpLayout lay = ep_layout(*L, t_cap);
    char *base;
    if (int rc = ep_ws(*L, lay, workspace, ws_bytes, &base)) return rc;
    return ep_experts_impl(*L, t_cap, base, lay, reinterpret_cast<cudaStream_t>(stream));
}

int vfmoe_ep_combine(int64_t handle, int64_t T, int64_t t_cap, int64_t out, int64_t workspace, int64_t ws_bytes,
                     int64_t stream) {
    Layer *L = get_layer(handle);
    if (!L) return VFMOE_ERR_HANDLE;
    if (int rc = ep_check(L, T, t_cap, "vfmoe_ep_combine")) return rc;
    if (T > 0 && !out) {
        set_error("vfmoe_ep_combine: out is null");
        return VFMOE_ERR_INVALID;
    }
    const EpLayout lay = ep_layout(*L, t_cap);
    char *base;
    if (int rc = ep_ws(*L, lay, workspace, ws_bytes, &base)) return rc;
    return ep_combine_impl(*L, T, base, lay, out, reinterpret_cast<cudaStream_t>(stream));
}

int vfmoe_ep_forward(int64_t comm, int64_t handle, int64_t x, int64_t T, int64_t t_cap, int64_t out, int64_t idx_out,
                     int64_t w_out, int64_t workspace, int64_t ws_bytes, int64_t stream) {
    EpComm *c = get_comm(comm);
    if (!c) return VFMOE_ERR_HANDLE;
    Layer *L = get_layer(handle);
    if (!L) return VFMOE_ERR_HANDLE;
    if (int rc = ep_check(L, T, t_cap, "vfmoe_ep_forward")) return rc;
    if (L->ep.n_ranks != c->nranks || L->ep.rank != c->rank) {
        set_error("vfmoe_ep_forward: the layer's placement is for rank %d of %d, the communicator is rank %d of %d",
                  L->ep.rank, L->ep.n_ranks, c->rank, c->nranks);
        return VFMOE_ERR_INVALID;
    }
    if ((T > 0 && (!x || !out || (x & 15)))) {
        set_error("vfmoe_ep_forward: x and out must be non-null, x 16-byte aligned");
        return VFMOE_ERR_INVALID;
    }
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    const EpLayout lay = ep_layout(*L, t_cap);
    char *base;
    int rc = ep_ws(*L, lay, workspace, ws_bytes, &base);
    if (rc) return rc;
    int32_t *idx = idx_out ? reinterpret_cast<int32_t *>(idx_out) : reinterpret_cast<int32_t *>(base + lay.idx);
    float *w = w_out ? reinterpret_cast<float *>(w_out) : reinterpret_cast<float *>(base + lay.w);
    // vfmoe_profile_enable: events on `stream` after each phase (stages 0 prepare, 1 shared expert,
    // 2 wait for the dispatch exchange, 3 experts, 4 return exchange, 5 combine)
    std::vector<cudaEvent_t> ev;
    auto mark = [&]() {
        if (!L->prof) return;
        cudaEvent_t e = take_event(*L);
        if (e) {
            cudaEventRecord(e, st);
            ev.push_back(e);
        }
    };
    mark();
    if ((rc = ep_prepare_impl(*L, x, T, t_cap, base, lay, idx, w, st))) return rc;
    mark();
    NcclApi &api = nccl();
    // dispatch on the side stream, the shared expert meanwhile on the caller's stream
    VF_CUDA(cudaEventRecord(c->ev_fork, st));
    VF_CUDA(cudaStreamWaitEvent(c->side, c->ev_fork, 0));
    ncclResult_t r = api.GroupStart();
    if (r == ncclSuccess) exchange_blocks(*c, base + lay.send_rows, base + lay.recv_rows, t_cap * lay.row_bytes, c->side, r);
    if (r == ncclSuccess)
        exchange_blocks(*c, base + lay.send_slot, base + lay.recv_slot, t_cap * L->k * 4, c->side, r);
    if (r == ncclSuccess) exchange_blocks(*c, base + lay.send_w, base + lay.recv_w, t_cap * L->k * 4, c->side, r);
    const ncclResult_t r_end = api.GroupEnd();
    if (r != ncclSuccess) return nccl_fail(r, "dispatch ncclSend/ncclRecv");
    if (r_end != ncclSuccess && r_end != ncclInProgress) return nccl_fail(r_end, "dispatch ncclGroupEnd");
    if ((rc = nccl_settle(*c, "dispatch exchange"))) return rc;
    VF_CUDA(cudaEventRecord(c->ev_join, c->side));
    if ((rc = ep_shared_impl(*L, x, T, base, lay, st))) return rc;
    mark();
    VF_CUDA(cudaStreamWaitEvent(st, c->ev_join, 0));
    mark();
    if ((rc = ep_experts_impl(*L, t_cap, base, lay, st))) return rc;
    mark();
    // partial rows back, on the caller's stream
    r = api.GroupStart();
    if (r == ncclSuccess) exchange_blocks(*c, base + lay.y_part, base + lay.y_back, t_cap * lay.part_bytes, st, r);
    const ncclResult_t r_end2 = api.GroupEnd();
    if (r != ncclSuccess) return nccl_fail(r, "return ncclSend/ncclRecv");
    if (r_end2 != ncclSuccess && r_end2 != ncclInProgress) return nccl_fail(r_end2, "return ncclGroupEnd");
    if ((rc = nccl_settle(*c, "return exchange"))) return rc;
    mark();
    if ((rc = ep_combine_impl(*L, T, base, lay, out, st))) return rc;
    mark();
    if (L->prof) {
        if (ev.size() == 7)
            L->ev_pending.push_back(ev);
        else
            for (auto e : ev) L->ev_pool.push_back(e);
    }
    return VFMOE_OK;
}

}  // extern "C"
