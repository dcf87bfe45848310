// C-ABI entry points of libvfmoe.so (declared in include/vfmoe.h).
//
// Host orchestration of one MoE layer forward (the reference does this with host
// loops in native/glm53/glm_engine.vyb:2728-2991 and three PTX launches in
// native/host/moe_driver.vyb:150-160).  Here every step is a kernel enqueued on the
// caller's stream, with no host synchronization:
//
//   router (fp64 logits, top-k, counts) -> dispatch (canonical permutation)
//   -> gather (fp16 rows) -> gate/up + SwiGLU -> down -> weighted combine.
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <set>
#include <tuple>
#include <string>
#include <unordered_map>
#include <vector>

#include "common.cuh"
#include "kernels.h"
#include "expert_tc.h"
#include "layer.h"

namespace vfmoe {

static thread_local std::string g_last_error;

void set_error(const char *fmt, ...) {
    char buf[1024];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof(buf), fmt, ap);
    va_end(ap);
    g_last_error = buf;
}

int cuda_fail(cudaError_t e, const char *what, const char *file, int line) {
    set_error("%s failed: %s (%s:%d)", what, cudaGetErrorString(e), file, line);
    return e == cudaErrorMemoryAllocation ? VFMOE_ERR_NOMEM : VFMOE_ERR_CUDA;
}

int set_smem_attr_once(const void *func, int bytes) {
    static std::mutex mu;
    static std::set<std::tuple<const void *, int, int>> done;
    int dev = 0;
    VF_CUDA(cudaGetDevice(&dev));
    std::lock_guard<std::mutex> lk(mu);
    if (done.count({func, dev, bytes})) return VFMOE_OK;
    VF_CUDA(cudaFuncSetAttribute(func, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes));
    done.insert({func, dev, bytes});
    return VFMOE_OK;
}


static constexpr int kNumStages = 5;

cudaEvent_t take_event(Layer &L) {
    cudaEvent_t e = nullptr;
    if (!L.ev_pool.empty()) {
        e = L.ev_pool.back();
        L.ev_pool.pop_back();
    } else if (cudaEventCreate(&e) != cudaSuccess) {
        e = nullptr;
    }
    return e;
}

static std::mutex g_mu;
static std::unordered_map<int64_t, Layer *> g_layers;
static int64_t g_next_handle = 1;

Layer *get_layer(int64_t h) {
    std::lock_guard<std::mutex> lk(g_mu);
    auto it = g_layers.find(h);
    if (it == g_layers.end()) {
        set_error("unknown layer handle %lld", (long long)h);
        return nullptr;
    }
    return it->second;
}

// ----------------------------------------------------------------------------- workspace

// Q8_0 layers with fp32 activations run the split-precision decode GEMV (unless the descriptor
// forces the tcgen05 or SIMT kernels).
int layer_prec(const Layer &L) {
    return L.d.x_dtype == VFMOE_DT_F32 && L.d.weight_format != VFMOE_WFMT_EXL3 &&
           L.d.expert_path != VFMOE_PATH_TC && L.d.expert_path != VFMOE_PATH_TC1 && L.d.expert_path != VFMOE_PATH_SIMT;
}

WsLayout ws_layout(const Layer &L, int64_t T, int k) {
    WsLayout o{};
    if (k < 0) k = L.k;
    const int64_t rows = T * k + T;
    const int nb = (L.E > L.n_local ? L.E : L.n_local) + 2;
    int64_t p = 0;
    auto take = [&](int64_t bytes) {
        const int64_t at = p;
        p = align_up(p + bytes, 256);
        return at;
    };
    o.counts = take((nb + 1) * 4);
    o.offsets = take((nb + 1) * 4);
    o.perm_tok = take(rows * 4);
    o.pos_of = take(T * k * 4);
    o.idx = take(T * k * 4);
    o.w = take(T * k * 4);
    o.part = take(router_logit_floats((int)T, L.H, L.E, L.wr_split != nullptr) * 4);
    // EXL3 keeps two rotated copies of every row (gate and up input bases); fp32 activations on
    // Q8_0 keep two fp16 planes of every row of xp and act (split-precision decode GEMV)
    const int prec = layer_prec(L);
    o.xp = take(rows * L.H * 2 * (L.d.weight_format == VFMOE_WFMT_EXL3 || prec ? 2 : 1));
    o.act = take(rows * L.I * 2 * (prec ? 2 : 1));
    o.y = take(rows * L.H * 4);
    o.tiles_cap = tc_tiles_capacity((int)T, k, L.n_local > L.E ? L.n_local : L.E);
    o.tiles = take(2 * o.tiles_cap * 16);
    o.tile_counts = take(2 * 4);
    if (L.dense_sh) {
        o.xs = take(T * L.H * 2);
        o.act_s = take(T * L.I * 2);
        o.y_s = take(T * L.H * 4);
    }
    o.total = p;
    return o;
}

int ensure_ws(Layer &L, int64_t T, int64_t ws, int64_t ws_bytes, char **base, int k) {
    const WsLayout lay = ws_layout(L, T, k);
    if (ws) {
        if (ws_bytes < lay.total) {
            set_error("workspace too small: %lld < %lld bytes for T=%lld", (long long)ws_bytes,
                      (long long)lay.total, (long long)T);
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

MatrixRef mref(const vfmoe_matrix &m) {
    MatrixRef r;
    r.data = reinterpret_cast<const uint8_t *>(m.data);
    r.expert_stride = m.expert_stride;
    r.suh = reinterpret_cast<const __half *>(m.suh);
    r.suh_stride = m.suh_stride;
    r.svh = reinterpret_cast<const __half *>(m.svh);
    r.svh_stride = m.svh_stride;
    return r;
}

static bool aligned16(int64_t p) { return (p & 15) == 0; }

static int validate(const vfmoe_layer_desc &d) {
    auto bad = [](const char *m) {
        set_error("invalid layer descriptor: %s", m);
        return VFMOE_ERR_INVALID;
    };
    if (d.hidden <= 0 || d.inter <= 0 || d.n_experts <= 0 || d.topk <= 0) return bad("non-positive shape");
    if (d.hidden % 256 || d.inter % 256) return bad("hidden and inter must be multiples of 256");
    if (d.n_experts > 1024) return bad("n_experts > 1024");
    if (d.n_local_experts < 0 || d.n_local_experts > 1024) return bad("n_local_experts out of range");
    if (d.topk > 32 || d.topk > d.n_experts) return bad("topk must be <= 32 and <= n_experts");
    if (d.x_dtype != VFMOE_DT_BF16 && d.x_dtype != VFMOE_DT_F32) return bad("x_dtype must be BF16 or F32");
    if (d.expert_path < VFMOE_PATH_AUTO || d.expert_path > VFMOE_PATH_TC1) return bad("expert_path out of range");
    if (d.out_dtype != VFMOE_DT_BF16 && d.out_dtype != VFMOE_DT_F32) return bad("out_dtype must be BF16 or F32");
    if (!d.router_w || !d.router_bias) return bad("router weights missing");
    if (!aligned16(d.router_w)) return bad("router_w must be 16-byte aligned");
    if (d.shared_format != 0 && d.shared_format != d.weight_format && d.shared_format != VFMOE_WFMT_BF16)
        return bad("shared_format must be 0, the routed format or VFMOE_WFMT_BF16");
    const bool dense_sh = d.shared_format == VFMOE_WFMT_BF16;
    if (dense_sh) {
        if (!d.sh_gate.data || !d.sh_up.data || !d.sh_down.data) return bad("bf16 shared expert incomplete");
        if (!aligned16(d.sh_gate.data) || !aligned16(d.sh_up.data) || !aligned16(d.sh_down.data))
            return bad("shared expert pointers must be 16-byte aligned");
    }
    if (d.weight_format == VFMOE_WFMT_Q8_0 || d.weight_format == VFMOE_WFMT_Q8_0_TILED) {
        const int64_t rg = d.hidden / 32 * 34, rd = d.inter / 32 * 34;
        if (!d.gate.data || !d.up.data || !d.down.data) return bad("routed expert weights missing");
        const int64_t nl = d.n_local_experts ? d.n_local_experts : d.n_experts;
        if (nl > 1 && (d.gate.expert_stride < d.inter * rg || d.up.expert_stride < d.inter * rg ||
                       d.down.expert_stride < d.hidden * rd))
            return bad("expert_stride smaller than one expert matrix");
        const int64_t ptrs[6] = {d.gate.data, d.up.data, d.down.data, d.sh_gate.data, d.sh_up.data, d.sh_down.data};
        for (int i = 0; i < 6; ++i)
            if (ptrs[i] && !aligned16(ptrs[i])) return bad("weight pointers must be 16-byte aligned");
        if ((d.gate.expert_stride | d.up.expert_stride | d.down.expert_stride) & 15)
            return bad("expert strides must be multiples of 16 bytes");
        if (d.sh_gate.data && (!d.sh_up.data || !d.sh_down.data)) return bad("shared expert incomplete");
    } else if (d.weight_format == VFMOE_WFMT_EXL3) {
        if (d.exl3_bits != 3 && d.exl3_bits != 4) return bad("exl3_bits must be 3 or 4");
        const vfmoe_matrix *ms[6] = {&d.gate, &d.up, &d.down, &d.sh_gate, &d.sh_up, &d.sh_down};
        const int64_t kk[3] = {d.hidden, d.hidden, d.inter}, nn[3] = {d.inter, d.inter, d.hidden};
        const int64_t nl = d.n_local_experts ? d.n_local_experts : d.n_experts;
        if (!d.gate.data || !d.up.data || !d.down.data) return bad("routed expert weights missing");
        if (d.sh_gate.data && (!d.sh_up.data || !d.sh_down.data)) return bad("shared expert incomplete");
        for (int i = 0; i < 6; ++i) {
            const vfmoe_matrix &m = *ms[i];
            if (!m.data || (i >= 3 && dense_sh)) continue;
            const int64_t K = kk[i % 3], N = nn[i % 3];
            if (!m.suh || !m.svh) return bad("EXL3 matrices need suh and svh");
            if (!aligned16(m.data) || (m.suh & 1) || (m.svh & 1)) return bad("EXL3 trellis must be 16-byte aligned");
            if (i < 3 && nl > 1 &&
                (m.expert_stride < K / 16 * N / 16 * 2 * 16 * d.exl3_bits || (m.expert_stride & 15) ||
                 m.suh_stride < K * 2 || m.svh_stride < N * 2 || (m.suh_stride & 1) || (m.svh_stride & 1)))
                return bad("EXL3 expert strides too small or misaligned");
        }
    } else {
        return bad("unknown weight_format");
    }
    return VFMOE_OK;
}

}  // namespace vfmoe

using namespace vfmoe;

extern "C" {

int vfmoe_version(void) { return VFMOE_ABI_VERSION; }

int vfmoe_last_error(char *buf, int64_t n) {
    const int len = (int)g_last_error.size();
    if (buf && n > 0) {
        const int64_t c = len < n - 1 ? len : n - 1;
        memcpy(buf, g_last_error.data(), (size_t)c);
        buf[c] = 0;
    }
    return len;
}

int vfmoe_init(int device) {
    int n = 0;
    VF_CUDA(cudaGetDeviceCount(&n));
    if (device < 0 || device >= n) {
        set_error("device %d out of range (%d devices)", device, n);
        return VFMOE_ERR_INVALID;
    }
    VF_CUDA(cudaSetDevice(device));
    cudaDeviceProp p;
    VF_CUDA(cudaGetDeviceProperties(&p, device));
    if (p.major != 10) {
        set_error("device %d is sm_%d%d; libvfmoe is built for sm_100a", device, p.major, p.minor);
        return VFMOE_ERR_UNSUPPORTED;
    }
    return VFMOE_OK;
}

int64_t vfmoe_layer_create(const vfmoe_layer_desc *desc) {
    if (!desc) {
        set_error("null descriptor");
        return VFMOE_ERR_INVALID;
    }
    int rc = validate(*desc);
    if (rc) return rc;
    Layer *L = new Layer();
    L->d = *desc;
    L->H = (int)desc->hidden;
    L->I = (int)desc->inter;
    L->E = (int)desc->n_experts;
    L->k = (int)desc->topk;
    L->n_local = (int)(desc->n_local_experts ? desc->n_local_experts : desc->n_experts);
    L->has_shared = desc->sh_gate.data != 0;
    L->q8_row_gate = desc->hidden / 32 * 34;
    L->q8_row_down = desc->inter / 32 * 34;
    cudaGetDevice(&L->device);
    cudaError_t e = cudaMalloc(&L->dev_err, sizeof(int));
    if (e == cudaSuccess) e = cudaMemset(L->dev_err, 0, sizeof(int));
    if (e == cudaSuccess) e = cudaMalloc(&L->nw, L->E * sizeof(float));
    if (e == cudaSuccess && launch_router_norms(reinterpret_cast<const float *>(desc->router_w), L->H, L->E, L->nw, 0))
        e = cudaErrorLaunchFailure;
    if (e == cudaSuccess && desc->x_dtype == VFMOE_DT_BF16 && L->H % 128 == 0 && L->E % 128 == 0) {
        const int64_t n = (int64_t)L->E * L->H;
        e = cudaMalloc(&L->wr_split, 2 * n * sizeof(__nv_bfloat16));
        if (e == cudaSuccess &&
            launch_router_split(reinterpret_cast<const float *>(desc->router_w), n, L->wr_split, L->wr_split + n, 0))
            e = cudaErrorLaunchFailure;
    }
    if (e == cudaSuccess) e = cudaDeviceSynchronize();
    if (e != cudaSuccess) {
        cuda_fail(e, "layer set-up (error word, router norms and split)", __FILE__, __LINE__);
        if (L->dev_err) cudaFree(L->dev_err);
        if (L->nw) cudaFree(L->nw);
        if (L->wr_split) cudaFree(L->wr_split);
        delete L;
        return VFMOE_ERR_CUDA;
    }
    cudaDeviceGetAttribute(&L->num_sms, cudaDevAttrMultiProcessorCount, L->device);
    vfmoe_layer_desc dplan = L->d;  // the routed kernels' plans never see a dense shared expert
    if (desc->shared_format == VFMOE_WFMT_BF16) {
        L->dense_sh = 1;
        dplan.sh_gate = dplan.sh_up = dplan.sh_down = vfmoe_matrix{};
        const int64_t gi = (int64_t)L->I * L->H;
        cudaError_t e2 = cudaMalloc(&L->sh_dense, 3 * gi * sizeof(__half));
        rc = e2 == cudaSuccess ? VFMOE_OK : cuda_fail(e2, "dense shared expert copy", __FILE__, __LINE__);
        const int64_t src[3] = {desc->sh_gate.data, desc->sh_up.data, desc->sh_down.data};
        for (int i = 0; i < 3 && !rc; ++i)
            rc = launch_to_f16(reinterpret_cast<const void *>(src[i]), VFMOE_DT_BF16, gi, L->sh_dense + i * gi, 0);
        if (!rc) rc = make_dense_map(&L->dsh_gate, L->sh_dense, L->I, L->H, 64);
        if (!rc) rc = make_dense_map(&L->dsh_up, L->sh_dense + gi, L->I, L->H, 64);
        if (!rc) rc = make_dense_map(&L->dsh_down, L->sh_dense + 2 * gi, L->H, L->I, 128);
        if (!rc && (e2 = cudaDeviceSynchronize()) != cudaSuccess)
            rc = cuda_fail(e2, "dense shared expert conversion", __FILE__, __LINE__);
    }
    if (!rc) rc = tc_plan_create(dplan, L->tc);
    if (!rc) rc = exl3_plan_create(dplan, L->x3);
    if (rc) {
        if (L->sh_dense) cudaFree(L->sh_dense);
        cudaFree(L->dev_err);
        cudaFree(L->nw);
        if (L->wr_split) cudaFree(L->wr_split);
        delete L;
        return rc;
    }
    std::lock_guard<std::mutex> lk(g_mu);
    const int64_t h = g_next_handle++;
    g_layers[h] = L;
    return h;
}

int vfmoe_layer_destroy(int64_t handle) {
    Layer *L;
    {
        std::lock_guard<std::mutex> lk(g_mu);
        auto it = g_layers.find(handle);
        if (it == g_layers.end()) {
            set_error("unknown layer handle %lld", (long long)handle);
            return VFMOE_ERR_HANDLE;
        }
        L = it->second;
        g_layers.erase(it);
    }
    if (L->own_ws) cudaFree(L->own_ws);
    if (L->dev_err) cudaFree(L->dev_err);
    if (L->nw) cudaFree(L->nw);
    if (L->wr_split) cudaFree(L->wr_split);
    if (L->sh_dense) cudaFree(L->sh_dense);
    if (L->ep.owner) cudaFree(L->ep.owner);
    for (auto &ev : L->ev_pending)
        for (auto e : ev) L->ev_pool.push_back(e);
    for (auto e : L->ev_pool) cudaEventDestroy(e);
    delete L;
    return VFMOE_OK;
}

int64_t vfmoe_workspace_bytes(int64_t handle, int64_t t_max) {
    Layer *L = get_layer(handle);
    if (!L) return VFMOE_ERR_HANDLE;
    if (t_max < 0) {
        set_error("negative t_max");
        return VFMOE_ERR_INVALID;
    }
    return ws_layout(*L, t_max).total;
}

}  // extern "C"

int vfmoe::route_impl(Layer &L, int64_t x, int64_t T, char *base, const WsLayout &lay, int32_t **idx_p,
                      float **w_p, cudaStream_t st) {
    int32_t *counts = reinterpret_cast<int32_t *>(base + lay.counts);  // zeroed by launch_router
    int32_t *idx = *idx_p ? *idx_p : reinterpret_cast<int32_t *>(base + lay.idx);
    float *w = *w_p ? *w_p : reinterpret_cast<float *>(base + lay.w);
    int rc = launch_router(reinterpret_cast<const void *>(x), (int)L.d.x_dtype,
                           reinterpret_cast<const float *>(L.d.router_w), L.wr_split, L.nw,
                           reinterpret_cast<const float *>(L.d.router_bias), (int)T, L.H, L.E, L.k,
                           L.d.routed_scale, reinterpret_cast<float *>(base + lay.part), idx, w, counts, L.dev_err,
                           st);
    *idx_p = idx;
    *w_p = w;
    return rc;
}

extern "C" {

int vfmoe_route(int64_t handle, int64_t x, int64_t T, int64_t idx_out, int64_t w_out, int64_t workspace,
                int64_t ws_bytes, int64_t stream) {
    Layer *L = get_layer(handle);
    if (!L) return VFMOE_ERR_HANDLE;
    if (T < 0 || (T > 0 && (!x || !idx_out || !w_out))) {
        set_error("vfmoe_route: bad arguments");
        return VFMOE_ERR_INVALID;
    }
    if (T == 0) return VFMOE_OK;
    if (T > (int64_t)1 << 24) {
        set_error("vfmoe_route: T=%lld exceeds 2^24", (long long)T);
        return VFMOE_ERR_UNSUPPORTED;
    }
    char *base;
    int rc = ensure_ws(*L, T, workspace, ws_bytes, &base);
    if (rc) return rc;
    const WsLayout lay = ws_layout(*L, T);
    int32_t *idx = reinterpret_cast<int32_t *>(idx_out);
    float *w = reinterpret_cast<float *>(w_out);
    return route_impl(*L, x, T, base, lay, &idx, &w, reinterpret_cast<cudaStream_t>(stream));
}

}  // extern "C"

// Q8_0 expert products on gathered fp16 rows: tensor-core path (decode GEMV or tcgen05
// grouped GEMM) unless the descriptor asks for the SIMT kernels (VFMOE_PATH_SIMT).
static int forward_experts(Layer &L, const MoeArgs &a, cudaStream_t st, const std::function<void()> &mid,
                           int64_t &nlaunch) {
    int rc;
    if (tc_supported(L.tc, a)) {
        rc = launch_experts_tc(L.tc, a, st, mid);
        nlaunch += 3;
    } else if (a.fmt == VFMOE_WFMT_Q8_0_TILED) {
        set_error("VFMOE_WFMT_Q8_0_TILED weights need the tensor-core expert path");
        return VFMOE_ERR_UNSUPPORTED;
    } else {
        rc = launch_experts_simt(a, st, mid);
        nlaunch += 2;
    }
    return rc;
}

extern "C" {

int vfmoe_forward(int64_t handle, int64_t x, int64_t T, int64_t out, int64_t idx_out, int64_t w_out,
                  int64_t workspace, int64_t ws_bytes, int64_t stream) {
    Layer *L = get_layer(handle);
    if (!L) return VFMOE_ERR_HANDLE;
    if (T < 0 || (T > 0 && (!x || !out))) {
        set_error("vfmoe_forward: bad arguments");
        return VFMOE_ERR_INVALID;
    }
    if (T == 0) return VFMOE_OK;
    if (T > (int64_t)1 << 24) {
        set_error("vfmoe_forward: T=%lld exceeds 2^24", (long long)T);
        return VFMOE_ERR_UNSUPPORTED;
    }
    if (L->n_local != L->E) {
        set_error("vfmoe_forward: this handle holds %d of %d experts (expert-parallel); use vfmoe_forward_rows",
                  L->n_local, L->E);
        return VFMOE_ERR_UNSUPPORTED;
    }
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    char *base;
    int rc = ensure_ws(*L, T, workspace, ws_bytes, &base);
    if (rc) return rc;
    const WsLayout lay = ws_layout(*L, T);
    int32_t *idx = reinterpret_cast<int32_t *>(idx_out);
    float *w = reinterpret_cast<float *>(w_out);
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
    rc = route_impl(*L, x, T, base, lay, &idx, &w, st);
    if (rc) return rc;
    mark();
    int64_t nlaunch = 2;

    MoeArgs a{};
    a.T = (int)T;
    a.H = L->H;
    a.I = L->I;
    a.E = L->E;
    a.k = L->k;
    const int fused_shared = L->has_shared && !L->dense_sh;  // shared expert inside the routed launches
    a.has_shared = fused_shared;
    a.fmt = (int)L->d.weight_format;
    a.exl3_bits = (int)L->d.exl3_bits;
    a.limit = (float)L->d.swiglu_limit;
    a.prec = layer_prec(*L);
    a.wait_ns = L->wait_ns;
    a.inject = L->inject;
    a.gate = mref(L->d.gate);
    a.up = mref(L->d.up);
    a.down = mref(L->d.down);
    a.sh_gate = mref(L->d.sh_gate);
    a.sh_up = mref(L->d.sh_up);
    a.sh_down = mref(L->d.sh_down);
    int32_t *counts = reinterpret_cast<int32_t *>(base + lay.counts);
    int32_t *offsets = reinterpret_cast<int32_t *>(base + lay.offsets);
    int32_t *perm_tok = reinterpret_cast<int32_t *>(base + lay.perm_tok);
    int32_t *pos_of = reinterpret_cast<int32_t *>(base + lay.pos_of);
    a.offsets = offsets;
    a.perm_tok = perm_tok;
    a.xp = reinterpret_cast<__half *>(base + lay.xp);
    a.act = reinterpret_cast<__half *>(base + lay.act);
    a.y = reinterpret_cast<float *>(base + lay.y);
    a.err = L->dev_err;
    a.tiles = reinterpret_cast<int4 *>(base + lay.tiles);
    a.tile_counts = reinterpret_cast<int32_t *>(base + lay.tile_counts);
    a.tiles_cap = lay.tiles_cap;

    // decode sizes on the GEMV path: dispatch, gather and the GEMV's tile lists in one launch
    const bool front = !L->x3.ready && L->tc.path == VFMOE_PATH_AUTO && tc_supported(L->tc, a) &&
                       tc_decode_gemv(L->tc, a) && T <= kDecodeFrontMaxT && L->E <= 1024;
    if (front) {
        a.plan_ready = 1;
        rc = launch_decode_front(idx, counts, (int)T, L->E, L->k, fused_shared, reinterpret_cast<const void *>(x),
                                 (int)L->d.x_dtype, L->H, perm_tok, pos_of, offsets,
                                 reinterpret_cast<__half *>(base + lay.xp), a.prec ? 2 : 1,
                                 gemv_tokens_per_tile((int)T, L->k, L->E), a.tiles, a.tiles_cap, a.tile_counts,
                                 L->dev_err, st);
    } else {
        rc = launch_dispatch(idx, counts, (int)T, L->E, L->k, fused_shared, perm_tok, pos_of, offsets, L->dev_err, st);
    }
    if (rc) return rc;
    if (L->dense_sh) {
        // the bf16-stored shared expert: its own dense GEMVs on fp16 x, ahead of the routed experts
        __half *xs = reinterpret_cast<__half *>(base + lay.xs);
        if ((rc = launch_to_f16(reinterpret_cast<const void *>(x), (int)L->d.x_dtype, T * L->H, xs, st))) return rc;
        if ((rc = launch_dense_expert(L->dsh_gate, L->dsh_up, L->dsh_down, xs, (int)T, L->H, L->I,
                                      reinterpret_cast<__half *>(base + lay.act_s), reinterpret_cast<float *>(base + lay.y_s),
                                      a.limit, L->dev_err, L->num_sms, L->wait_ns, st)))
            return rc;
        nlaunch += 3;
    }
    if (L->x3.ready) {
        // EXL3: the expert path gathers and rotates the rows itself
        nlaunch += 1;
        mark();
        rc = launch_experts_exl3(L->x3, a, reinterpret_cast<const void *>(x), (int)L->d.x_dtype, st,
                                 [&]() { mark(); });
        nlaunch += 4;
    } else {
        // launch bound T*k + T whether or not there is a shared expert: the second plane of a
        // split-precision layer starts at that row count, as the expert kernels expect
        if (!front) {
            rc = launch_gather(reinterpret_cast<const void *>(x), (int)L->d.x_dtype, perm_tok, T * L->k + T, L->H,
                               reinterpret_cast<__half *>(base + lay.xp), offsets + L->E + 1, st, a.prec ? 2 : 1);
            if (rc) return rc;
        }
        nlaunch += front ? 1 : 2;
        mark();
        rc = forward_experts(*L, a, st, [&]() { mark(); }, nlaunch);
        if (front) nlaunch -= 1;  // no tile-plan launch
    }
    if (rc) return rc;
    mark();
    rc = launch_combine(a.y, VFMOE_DT_F32, pos_of, w, (int)T, L->H, L->k,
                        L->dense_sh ? reinterpret_cast<float *>(base + lay.y_s)
                                    : (fused_shared ? a.y + T * L->k * L->H : nullptr),
                        reinterpret_cast<void *>(out),
                        (int)L->d.out_dtype, st);
    if (rc) return rc;
    nlaunch += 1;
    mark();
    if (L->prof) {
        if ((int)ev.size() == kNumStages + 1) {
            L->ev_pending.push_back(ev);
        } else {
            for (auto e : ev) L->ev_pool.push_back(e);
        }
        L->launches += nlaunch;
    }
    return VFMOE_OK;
}

int vfmoe_profile_enable(int64_t handle, int enable) {
    Layer *L = get_layer(handle);
    if (!L) return VFMOE_ERR_HANDLE;
    L->prof = enable ? 1 : 0;
    return VFMOE_OK;
}

int vfmoe_profile_read(int64_t handle, double *stage_ms, int64_t n, int64_t *launches) {
    Layer *L = get_layer(handle);
    if (!L) return VFMOE_ERR_HANDLE;
    for (auto &ev : L->ev_pending) {
        VF_CUDA(cudaEventSynchronize(ev.back()));
        for (int s = 0; s + 1 < (int)ev.size() && s < 8; ++s) {
            float ms = 0.f;
            VF_CUDA(cudaEventElapsedTime(&ms, ev[s], ev[s + 1]));
            L->stage_ms[s] += ms;
        }
        for (auto e : ev) L->ev_pool.push_back(e);
        L->n_fwd += 1;
    }
    L->ev_pending.clear();
    for (int64_t s = 0; s < n && s < 8; ++s) stage_ms[s] = L->stage_ms[s];
    if (launches) *launches = L->launches;
    const int nf = (int)L->n_fwd;
    for (int s = 0; s < 8; ++s) L->stage_ms[s] = 0;
    L->n_fwd = 0;
    L->launches = 0;
    return nf;
}

int64_t vfmoe_rows_workspace_bytes(int64_t handle, int64_t n_max) {
    Layer *L = get_layer(handle);
    if (!L) return VFMOE_ERR_HANDLE;
    if (n_max < 0) {
        set_error("negative n_max");
        return VFMOE_ERR_INVALID;
    }
    return ws_layout(*L, n_max, 1).total;
}

}  // extern "C"

// Expert products on caller-provided rows with caller-provided routing: slots [n, k] are
// local expert slots (n_local = the shared expert; < 0 = no expert when skip_negative),
// w [n, k] their weights (0 = weight 1).  y_out[i] = sum_l w[i,l] * FFN_{slots[i,l]}(rows[i]).
int vfmoe::rows_impl(Layer &L, int64_t rows, int64_t rows_dtype, const int32_t *sl, int64_t n, int k, const float *w,
                     int64_t y_out, int y_dtype, int skip_negative, int64_t workspace, int64_t ws_bytes,
                     cudaStream_t st) {
    if (n == 0) return VFMOE_OK;
    if (n * k > (int64_t)1 << 24) {
        set_error("expert rows: n*k=%lld exceeds 2^24", (long long)(n * k));
        return VFMOE_ERR_UNSUPPORTED;
    }
    char *base;
    int rc = ensure_ws(L, n, workspace, ws_bytes, &base, k);
    if (rc) return rc;
    const WsLayout lay = ws_layout(L, n, k);
    const int nl = L.n_local;
    // slot nl = the shared expert: an ordinary bucket of a dispatch over nl + 1 buckets
    const int nb = nl + (L.has_shared && !L.dense_sh ? 1 : 0);
    int32_t *counts = reinterpret_cast<int32_t *>(base + lay.counts);
    int32_t *offsets = reinterpret_cast<int32_t *>(base + lay.offsets);
    int32_t *perm_tok = reinterpret_cast<int32_t *>(base + lay.perm_tok);
    int32_t *pos_of = reinterpret_cast<int32_t *>(base + lay.pos_of);
    VF_CUDA(cudaMemsetAsync(counts, 0, (nb + 2) * sizeof(int32_t), st));
    if ((rc = launch_count(sl, n * k, nb, counts, L.dev_err, st, skip_negative))) return rc;
    // -1: no row (a lane with no expert, or a slot out of range that the count flagged)
    VF_CUDA(cudaMemsetAsync(pos_of, 0xFF, n * k * sizeof(int32_t), st));
    if ((rc = launch_dispatch(sl, counts, (int)n, nb, k, 0, perm_tok, pos_of, offsets, L.dev_err, st))) return rc;
    MoeArgs a{};
    a.T = (int)n;
    a.H = L.H;
    a.I = L.I;
    a.E = nl;
    a.k = k;
    a.has_shared = L.has_shared && !L.dense_sh;
    a.fmt = (int)L.d.weight_format;
    a.exl3_bits = (int)L.d.exl3_bits;
    a.limit = (float)L.d.swiglu_limit;
    a.prec = layer_prec(L) && rows_dtype == VFMOE_DT_F32;
    a.wait_ns = L.wait_ns;
    a.inject = L.inject;
    a.gate = mref(L.d.gate);
    a.up = mref(L.d.up);
    a.down = mref(L.d.down);
    a.sh_gate = mref(L.d.sh_gate);
    a.sh_up = mref(L.d.sh_up);
    a.sh_down = mref(L.d.sh_down);
    a.offsets = offsets;
    a.perm_tok = perm_tok;
    a.xp = reinterpret_cast<__half *>(base + lay.xp);
    a.act = reinterpret_cast<__half *>(base + lay.act);
    a.y = reinterpret_cast<float *>(base + lay.y);
    a.err = L.dev_err;
    a.tiles = reinterpret_cast<int4 *>(base + lay.tiles);
    a.tile_counts = reinterpret_cast<int32_t *>(base + lay.tile_counts);
    a.tiles_cap = lay.tiles_cap;
    int64_t nlaunch = 0;
    if (L.x3.ready) {
        rc = launch_experts_exl3(L.x3, a, reinterpret_cast<const void *>(rows), (int)rows_dtype, st, []() {});
    } else {
        if ((rc = launch_gather(reinterpret_cast<const void *>(rows), (int)rows_dtype, perm_tok, n * k + n, L.H,
                                reinterpret_cast<__half *>(base + lay.xp), offsets + nb + 1, st, a.prec ? 2 : 1)))
            return rc;
        rc = forward_experts(L, a, st, []() {}, nlaunch);
    }
    if (rc) return rc;
    // back to the callers' row order: y_out[i] = sum_l w[i,l] * y[pos_of[i*k+l]]
    return launch_combine(a.y, VFMOE_DT_F32, pos_of, w, (int)n, L.H, k, nullptr, reinterpret_cast<void *>(y_out),
                          y_dtype, st);
}

extern "C" {

int vfmoe_forward_rows(int64_t handle, int64_t rows, int64_t rows_dtype, int64_t slots, int64_t n, int64_t y_out,
                       int64_t workspace, int64_t ws_bytes, int64_t stream) {
    Layer *L = get_layer(handle);
    if (!L) return VFMOE_ERR_HANDLE;
    if (n < 0 || (n > 0 && (!rows || !slots || !y_out)) || (rows & 15) ||
        (rows_dtype != VFMOE_DT_BF16 && rows_dtype != VFMOE_DT_F32)) {
        set_error("vfmoe_forward_rows: bad arguments");
        return VFMOE_ERR_INVALID;
    }
    return rows_impl(*L, rows, rows_dtype, reinterpret_cast<const int32_t *>(slots), n, 1, nullptr, y_out,
                     VFMOE_DT_F32, 0, workspace, ws_bytes, reinterpret_cast<cudaStream_t>(stream));
}

int64_t vfmoe_routed_workspace_bytes(int64_t handle, int64_t n_max, int64_t k) {
    Layer *L = get_layer(handle);
    if (!L) return VFMOE_ERR_HANDLE;
    if (n_max < 0 || k <= 0 || k > 32) {
        set_error("vfmoe_routed_workspace_bytes: bad arguments");
        return VFMOE_ERR_INVALID;
    }
    return ws_layout(*L, n_max, (int)k).total;
}

int vfmoe_forward_routed(int64_t handle, int64_t rows, int64_t rows_dtype, int64_t n, int64_t k, int64_t slots,
                         int64_t w, int64_t y_out, int64_t y_dtype, int64_t workspace, int64_t ws_bytes,
                         int64_t stream) {
    Layer *L = get_layer(handle);
    if (!L) return VFMOE_ERR_HANDLE;
    if (n < 0 || k <= 0 || k > 32 || (n > 0 && (!rows || !slots || !y_out)) || (rows & 15) ||
        (rows_dtype != VFMOE_DT_BF16 && rows_dtype != VFMOE_DT_F32) ||
        (y_dtype != VFMOE_DT_F32 && y_dtype != VFMOE_DT_F16 && y_dtype != VFMOE_DT_BF16)) {
        set_error("vfmoe_forward_routed: bad arguments");
        return VFMOE_ERR_INVALID;
    }
    return rows_impl(*L, rows, rows_dtype, reinterpret_cast<const int32_t *>(slots), n, (int)k,
                     reinterpret_cast<const float *>(w), y_out, (int)y_dtype, 1, workspace, ws_bytes,
                     reinterpret_cast<cudaStream_t>(stream));
}

int vfmoe_combine(int64_t y, int64_t y_dtype, int64_t pos_of, int64_t w, int64_t T, int64_t k, int64_t H,
                  int64_t y_shared, int64_t out, int64_t out_dtype, int64_t stream) {
    if (T < 0 || k <= 0 || k > 32 || H <= 0 || H % 4 || (y_dtype != VFMOE_DT_F32 && y_dtype != VFMOE_DT_F16) ||
        (out_dtype != VFMOE_DT_F32 && out_dtype != VFMOE_DT_BF16 && out_dtype != VFMOE_DT_F16) ||
        (T > 0 && (!y || !pos_of || !out)) || (y & 15) || (y_shared & 15)) {
        set_error("vfmoe_combine: bad arguments");
        return VFMOE_ERR_INVALID;
    }
    return launch_combine(reinterpret_cast<const void *>(y), (int)y_dtype, reinterpret_cast<const int32_t *>(pos_of),
                          reinterpret_cast<const float *>(w), (int)T, (int)H, (int)k,
                          reinterpret_cast<const void *>(y_shared), reinterpret_cast<void *>(out), (int)out_dtype,
                          reinterpret_cast<cudaStream_t>(stream));
}

int vfmoe_dispatch(int64_t idx, int64_t T, int64_t k, int64_t n_experts, int64_t counts, int64_t offsets,
                   int64_t perm_tok, int64_t pos_of, int64_t err_word, int64_t stream) {
    if (T < 0 || k <= 0 || k > 32 || n_experts <= 0 || n_experts > 1024 || T * k > ((int64_t)1 << 30) ||
        !counts || !offsets || (T > 0 && (!idx || !perm_tok || !pos_of))) {
        set_error("vfmoe_dispatch: bad arguments");
        return VFMOE_ERR_INVALID;
    }
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    int32_t *cnt = reinterpret_cast<int32_t *>(counts);
    int32_t *pos = reinterpret_cast<int32_t *>(pos_of);
    VF_CUDA(cudaMemsetAsync(cnt, 0, (n_experts + 2) * sizeof(int32_t), st));
    if (T == 0) {
        VF_CUDA(cudaMemsetAsync(reinterpret_cast<void *>(offsets), 0, (n_experts + 2) * sizeof(int32_t), st));
        return VFMOE_OK;
    }
    // a lane whose id is out of range is counted nowhere and keeps pos_of = -1
    VF_CUDA(cudaMemsetAsync(pos, 0xFF, T * k * sizeof(int32_t), st));
    int *err = reinterpret_cast<int *>(err_word);
    int rc = launch_count(reinterpret_cast<const int32_t *>(idx), T * k, (int)n_experts, cnt, err, st);
    if (rc) return rc;
    return launch_dispatch(reinterpret_cast<const int32_t *>(idx), cnt, (int)T, (int)n_experts, (int)k, 0,
                           reinterpret_cast<int32_t *>(perm_tok), pos, reinterpret_cast<int32_t *>(offsets), err, st);
}

int vfmoe_route_logits(int64_t handle, int64_t x, int64_t T, int64_t logits_out, double *bound_out,
                       int64_t workspace, int64_t ws_bytes, int64_t stream) {
    Layer *L = get_layer(handle);
    if (!L) return VFMOE_ERR_HANDLE;
    if (T <= 0 || T > ((int64_t)1 << 24) || !x || !logits_out || !bound_out) {
        set_error("vfmoe_route_logits: bad arguments");
        return VFMOE_ERR_INVALID;
    }
    char *base;
    int rc = ensure_ws(*L, T, workspace, ws_bytes, &base);
    if (rc) return rc;
    const WsLayout lay = ws_layout(*L, T);
    float c1 = 0.f;
    rc = launch_route_logits(reinterpret_cast<const void *>(x), (int)L->d.x_dtype,
                             reinterpret_cast<const float *>(L->d.router_w), L->wr_split, (int)T, L->H, L->E,
                             reinterpret_cast<float *>(base + lay.part), reinterpret_cast<float *>(logits_out),
                             L->dev_err, reinterpret_cast<cudaStream_t>(stream), &c1);
    *bound_out = c1;
    return rc;
}

int vfmoe_debug_inject(int64_t handle, int64_t kind, int64_t wait_ns) {
    Layer *L = get_layer(handle);
    if (!L) return VFMOE_ERR_HANDLE;
    if ((kind != VFMOE_INJECT_NONE && kind != VFMOE_INJECT_STALL_LOADS) || wait_ns < 0) {
        set_error("vfmoe_debug_inject: bad arguments");
        return VFMOE_ERR_INVALID;
    }
    L->inject = (int)kind;
    L->wait_ns = wait_ns ? (uint64_t)wait_ns : 2000000000ull;
    return VFMOE_OK;
}

int vfmoe_check_device_error(int64_t handle, int64_t stream) {
    Layer *L = get_layer(handle);
    if (!L) return VFMOE_ERR_HANDLE;
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    VF_CUDA(cudaStreamSynchronize(st));
    int h = 0;
    VF_CUDA(cudaMemcpy(&h, L->dev_err, sizeof(int), cudaMemcpyDeviceToHost));
    if (h) {
        VF_CUDA(cudaMemset(L->dev_err, 0, sizeof(int)));
        set_error("device-side error code %d", h);
        return VFMOE_ERR_DEVICE;
    }
    return VFMOE_OK;
}

int vfmoe_rmsnorm(int64_t x, int64_t w, int64_t y, int64_t S, int64_t D, double eps, int64_t dtype,
                  int64_t stream) {
    if (S < 0 || D <= 0 || (S > 0 && (!x || !w || !y)) ||
        (dtype != VFMOE_DT_BF16 && dtype != VFMOE_DT_F32 && dtype != VFMOE_DT_F16)) {
        set_error("vfmoe_rmsnorm: bad arguments");
        return VFMOE_ERR_INVALID;
    }
    return launch_rmsnorm(reinterpret_cast<const void *>(x), reinterpret_cast<const float *>(w),
                          reinterpret_cast<void *>(y), S, (int)D, (float)eps, (int)dtype,
                          reinterpret_cast<cudaStream_t>(stream));
}

int vfmoe_residual_rmsnorm(int64_t x, int64_t y, int64_t w, int64_t x_out, int64_t h, int64_t S, int64_t D,
                           double eps, int64_t dtype, int64_t stream) {
    if (S < 0 || D <= 0 || (S > 0 && (!x || (y && !x_out) || (w && !h) || (!y && !w))) ||
        (dtype != VFMOE_DT_BF16 && dtype != VFMOE_DT_F32)) {
        set_error("vfmoe_residual_rmsnorm: bad arguments");
        return VFMOE_ERR_INVALID;
    }
    return launch_residual_rmsnorm(reinterpret_cast<const void *>(x), reinterpret_cast<const void *>(y),
                                   reinterpret_cast<const float *>(w), reinterpret_cast<void *>(x_out),
                                   reinterpret_cast<void *>(h), S, (int)D, (float)eps, (int)dtype,
                                   reinterpret_cast<cudaStream_t>(stream));
}

int vfmoe_hc_mix(const vfmoe_hc_desc *d, int64_t streams, int64_t R, int64_t h_out, int64_t h_dtype,
                 int64_t post_out, int64_t comb_out, int64_t stream) {
    if (!d || d->n_streams != 4 || d->hidden <= 0 || d->hidden % 2048 || d->hidden > 8192 || !d->fn || !d->base ||
        !d->scale || (d->fn_dtype != VFMOE_DT_BF16 && d->fn_dtype != VFMOE_DT_F32) || d->sinkhorn_iters < 1 ||
        d->sinkhorn_iters > 1000 || d->rms_eps < 0 || d->hc_eps < 0 || d->norm_eps < 0 || R < 0 ||
        (R > 0 && (!streams || !h_out || !post_out || !comb_out)) || (streams & 15) || (d->fn & 15) ||
        (d->norm_w & 15) || (h_dtype != VFMOE_DT_BF16 && h_dtype != VFMOE_DT_F32)) {
        set_error("vfmoe_hc_mix: bad arguments (4 streams, hidden a multiple of 2048 up to 8192, 16-byte aligned "
                  "streams / fn / norm_w)");
        return VFMOE_ERR_INVALID;
    }
    return launch_hc_mix(reinterpret_cast<const float *>(streams), R, (int)d->hidden, reinterpret_cast<const void *>(d->fn),
                         (int)d->fn_dtype, reinterpret_cast<const float *>(d->base),
                         reinterpret_cast<const float *>(d->scale), (float)d->rms_eps, d->hc_eps, (int)d->sinkhorn_iters,
                         reinterpret_cast<const float *>(d->norm_w), (float)d->norm_eps, reinterpret_cast<void *>(h_out),
                         (int)h_dtype, reinterpret_cast<float *>(post_out), reinterpret_cast<float *>(comb_out),
                         reinterpret_cast<cudaStream_t>(stream));
}

int vfmoe_hc_apply(int64_t streams, int64_t y, int64_t y_dtype, int64_t post, int64_t comb, int64_t R,
                   int64_t n_streams, int64_t hidden, int64_t out, int64_t stream) {
    if (n_streams != 4 || hidden <= 0 || hidden % 4 || R < 0 || (y_dtype != VFMOE_DT_BF16 && y_dtype != VFMOE_DT_F32) ||
        (R > 0 && (!streams || !y || !post || !comb || !out)) || (streams & 15) || (out & 15)) {
        set_error("vfmoe_hc_apply: bad arguments (4 streams, hidden a multiple of 4, 16-byte aligned streams/out)");
        return VFMOE_ERR_INVALID;
    }
    return launch_hc_apply(reinterpret_cast<const float *>(streams), reinterpret_cast<const void *>(y), (int)y_dtype,
                           reinterpret_cast<const float *>(post), reinterpret_cast<const float *>(comb), R, (int)hidden,
                           reinterpret_cast<float *>(out), reinterpret_cast<cudaStream_t>(stream));
}

int vfmoe_q8_0_dequant(int64_t src, int64_t dst, int64_t rows, int64_t k, int64_t dst_dtype, int64_t stream) {
    if (rows < 0 || k <= 0 || k % 32 || (rows > 0 && (!src || !dst)) ||
        (dst_dtype != VFMOE_DT_F32 && dst_dtype != VFMOE_DT_F16)) {
        set_error("vfmoe_q8_0_dequant: bad arguments");
        return VFMOE_ERR_INVALID;
    }
    return launch_q8_0_dequant(reinterpret_cast<const uint8_t *>(src), reinterpret_cast<void *>(dst), rows, k,
                               (int)dst_dtype, reinterpret_cast<cudaStream_t>(stream));
}

int vfmoe_q8_0_quantize(int64_t src_f32, int64_t dst, int64_t rows, int64_t k, int64_t stream) {
    if (rows < 0 || k <= 0 || k % 32 || (rows > 0 && (!src_f32 || !dst)) || (src_f32 & 15)) {
        set_error("vfmoe_q8_0_quantize: bad arguments");
        return VFMOE_ERR_INVALID;
    }
    return launch_q8_0_quantize(reinterpret_cast<const float *>(src_f32), reinterpret_cast<uint8_t *>(dst), rows,
                                k, reinterpret_cast<cudaStream_t>(stream));
}

int vfmoe_q8_0_tile(int64_t src, int64_t dst, int64_t rows, int64_t k, int64_t n_mats, int64_t stream) {
    if (rows < 0 || n_mats < 0 || k <= 0 || k % 256 || rows % 64) {
        set_error("vfmoe_q8_0_tile: rows must be a multiple of 64 and k of 256");
        return VFMOE_ERR_INVALID;
    }
    const int64_t bytes = rows * (k / 32 * 34) * n_mats;
    if (bytes == 0) return VFMOE_OK;
    if (!src || !dst || (src & 15) || (dst & 15)) {
        set_error("vfmoe_q8_0_tile: src and dst must be non-null and 16-byte aligned");
        return VFMOE_ERR_INVALID;
    }
    if (src < dst + bytes && dst < src + bytes) {
        set_error("vfmoe_q8_0_tile: dst overlaps src");
        return VFMOE_ERR_INVALID;
    }
    return launch_q8_0_tile(reinterpret_cast<const uint8_t *>(src), reinterpret_cast<uint8_t *>(dst), rows, k,
                            n_mats, reinterpret_cast<cudaStream_t>(stream));
}

int vfmoe_exl3_decode(int64_t trellis, int64_t dst_f16, int64_t K, int64_t N, int64_t bits, int64_t stream) {
    if (K <= 0 || N <= 0 || K % 16 || N % 16 || !trellis || !dst_f16) {
        set_error("vfmoe_exl3_decode: bad arguments");
        return VFMOE_ERR_INVALID;
    }
    if (bits != 3 && bits != 4) {
        set_error("vfmoe_exl3_decode: bits=%lld (3 or 4 expected)", (long long)bits);
        return VFMOE_ERR_INVALID;
    }
    if (trellis & 15) {
        set_error("vfmoe_exl3_decode: trellis must be 16-byte aligned");
        return VFMOE_ERR_INVALID;
    }
    return launch_exl3_decode(reinterpret_cast<const uint16_t *>(trellis), reinterpret_cast<__half *>(dst_f16), K,
                              N, (int)bits, reinterpret_cast<cudaStream_t>(stream));
}

}  // extern "C"

namespace vfmoe {

// Router into a caller-provided device scratch range (no allocation, no workspace layout):
// router logits/partials, then the per-expert counts.  Used by vfmoe_route_noalloc.
int route_into_scratch(int64_t handle, int64_t x, int64_t T, int64_t idx_out, int64_t w_out, char *scratch,
                       int64_t scratch_bytes, int64_t stream) {
    Layer *L = get_layer(handle);
    if (!L) return VFMOE_ERR_HANDLE;
    int dev = -1;
    VF_CUDA(cudaGetDevice(&dev));
    if (dev != L->device) {
        // the scratch address belongs to the current device, the layer's weights to its own
        set_error("vfmoe_route_noalloc: the current device is %d but the layer lives on device %d", dev, L->device);
        return VFMOE_ERR_INVALID;
    }
    if (T > (int64_t)1 << 24) {
        set_error("vfmoe_route_noalloc: T=%lld exceeds 2^24", (long long)T);
        return VFMOE_ERR_UNSUPPORTED;
    }
    const int64_t logit_bytes = align_up(router_logit_floats((int)T, L->H, L->E, L->wr_split != nullptr) * 4, 256);
    const int64_t need = logit_bytes + align_up((L->E + 2) * 4, 256);
    if (need > scratch_bytes) {
        set_error("vfmoe_route_noalloc: T=%lld needs %lld bytes of router scratch; the static scratch holds %lld "
                  "(use vfmoe_route with a workspace for this size)",
                  (long long)T, (long long)need, (long long)scratch_bytes);
        return VFMOE_ERR_UNSUPPORTED;
    }
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    int32_t *counts = reinterpret_cast<int32_t *>(scratch + logit_bytes);
    VF_CUDA(cudaMemsetAsync(counts, 0, (L->E + 2) * sizeof(int32_t), st));
    return launch_router(reinterpret_cast<const void *>(x), (int)L->d.x_dtype,
                         reinterpret_cast<const float *>(L->d.router_w), L->wr_split, L->nw,
                         reinterpret_cast<const float *>(L->d.router_bias), (int)T, L->H, L->E, L->k,
                         L->d.routed_scale, reinterpret_cast<float *>(scratch), reinterpret_cast<int32_t *>(idx_out),
                         reinterpret_cast<float *>(w_out), counts, L->dev_err, st);
}

}  // namespace vfmoe
