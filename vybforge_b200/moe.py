"""Host-side mirror of the reference MoE interface over libvfmoe.so.

The reference's operator surface for this path is the numpy gate
(native/glm53/moe_ref.py: ``route``, ``ffn``, ``moe_block``) and the three PTX
kernels of native/kernels/moe.vyb (``moe_route``, ``moe_act``, ``moe_down``)
driven by native/host/moe_driver.vyb.  ``MoELayer`` keeps those names and
argument meanings:

* ``MoELayer.route(x)``    -> (idx int32 [T,k], w fp32 [T,k])   (moe_ref.route)
* ``MoELayer.moe_block(x)`` -> (out [T,H], idx, w)               (moe_ref.moe_block)

Device memory and streams come from torch; every computation is a libvfmoe
kernel reached through the C ABI.  A missing library raises on import.
"""

from __future__ import annotations

import ctypes as C

import torch

from . import _lib
from ._lib import check, DT_BF16, DT_F16, DT_F32, WFMT_Q8_0, WFMT_EXL3, WFMT_Q8_0_TILED
from ._lib import PATH_AUTO, PATH_SIMT, PATH_TC, PATH_GEMV, PATH_TC1

_PATHS = {"auto": PATH_AUTO, "simt": PATH_SIMT, "tc": PATH_TC, "gemv": PATH_GEMV, "tc1": PATH_TC1}

_DT = {torch.float32: DT_F32, torch.float16: DT_F16, torch.bfloat16: DT_BF16}


def _ptr(t) -> int:
    return 0 if t is None else int(t.data_ptr())


def _stream() -> int:
    return int(torch.cuda.current_stream().cuda_stream)


def init(device: int = 0) -> None:
    check(_lib.load().vfmoe_init(device))


def q8_0_tile(w: torch.Tensor) -> torch.Tensor:
    """Stage-tiled copy (VFMOE_WFMT_Q8_0_TILED) of Q8_0 matrices in GGUF row order:
    uint8 [..., rows, k/32*34] on the GPU, rows % 64 == 0, k % 256 == 0."""
    assert w.dtype == torch.uint8 and w.is_cuda and w.is_contiguous()
    rows, rb = w.shape[-2], w.shape[-1]
    k = rb // 34 * 32
    n = w.numel() // (rows * rb)
    out = torch.empty_like(w)
    check(_lib.load().vfmoe_q8_0_tile(_ptr(w), _ptr(out), rows, k, n, _stream()))
    return out


class MoELayer:
    """One GLM-style MoE layer (router + routed experts + shared expert) on one GPU.

    Q8_0 weights: ``gate``/``up`` uint8 [E, I, H/32*34], ``down`` uint8 [E, H, I/32*34]
    (GGUF block rows = output channels); ``shared`` = (gate [I, ...], up, down) or None.
    fmt="q8_0_tiled": the same tensors after ``q8_0_tile`` (stage-tiled byte order).
    EXL3 weights: each projection is a tuple (trellis int16 [E, K/16, N/16, 16*bits],
    suh fp16 [E, K], svh fp16 [E, N]); shared likewise without the leading E.
    path: expert kernels, "auto" (default), "tc", "tc1" (tcgen05 with single-CTA tiles only), "gemv"
        or "simt" (vfmoe_layer_desc.expert_path).
    shared_format="bf16": the shared expert is (gate, up, down) bf16 [out, in] matrices as a Hugging
    Face checkpoint stores them (GLM-5.3: EXL3 routed experts, bf16 shared expert).
    """

    def __init__(self, *, hidden, inter, n_experts, topk, router_w, router_bias, gate, up, down,
                 shared=None, fmt="q8_0", exl3_bits=3, x_dtype=torch.bfloat16, out_dtype=torch.bfloat16,
                 scale=2.5, limit=10.0, n_local_experts=0, path="auto", shared_format=None):
        self.lib = _lib.load()
        self.H, self.I, self.E, self.k = hidden, inter, n_experts, topk
        self.x_dtype, self.out_dtype = x_dtype, out_dtype
        self.fmt = fmt
        d = _lib.LayerDesc()
        d.hidden, d.inter, d.n_experts, d.topk = hidden, inter, n_experts, topk
        d.n_local_experts = n_local_experts
        d.expert_path = _PATHS[path]
        self.n_local = n_local_experts or n_experts
        d.weight_format = {"q8_0": WFMT_Q8_0, "q8_0_tiled": WFMT_Q8_0_TILED, "exl3": WFMT_EXL3}[fmt]
        d.exl3_bits = exl3_bits
        d.x_dtype, d.out_dtype = _DT[x_dtype], _DT[out_dtype]
        d.routed_scale, d.swiglu_limit = scale, limit
        d.router_w, d.router_bias = _ptr(router_w), _ptr(router_bias)
        self._keep = [router_w, router_bias, gate, up, down, shared]

        def fill(m, w, stacked):
            if fmt in ("q8_0", "q8_0_tiled"):
                m.data = _ptr(w)
                m.expert_stride = w[0].numel() * w.element_size() if stacked else 0
            else:
                tr, suh, svh = w
                m.data, m.suh, m.svh = _ptr(tr), _ptr(suh), _ptr(svh)
                if stacked:
                    m.expert_stride = tr[0].numel() * tr.element_size()
                    m.suh_stride = suh[0].numel() * suh.element_size()
                    m.svh_stride = svh[0].numel() * svh.element_size()

        fill(d.gate, gate, True)
        fill(d.up, up, True)
        fill(d.down, down, True)
        if shared is not None and shared_format == "bf16":
            d.shared_format = _lib.WFMT_BF16
            for m, w in zip((d.sh_gate, d.sh_up, d.sh_down), shared):
                assert w.dtype == torch.bfloat16 and w.is_contiguous()
                m.data = _ptr(w)
        elif shared is not None:
            fill(d.sh_gate, shared[0], False)
            fill(d.sh_up, shared[1], False)
            fill(d.sh_down, shared[2], False)
        self.desc = d
        self.handle = check(self.lib.vfmoe_layer_create(C.byref(d)))
        self._ws = None
        self._rows_ws = None

    # ------------------------------------------------------------------ packed files
    def save_packed(self, path: str) -> None:
        """Write this layer's weights to a packed layer file (vfmoe_pack_save)."""
        check(self.lib.vfmoe_pack_save(path.encode(), C.byref(self.desc)))

    @classmethod
    def from_packed(cls, path: str):
        """A layer whose weights live in one device buffer read from a packed layer file
        (vfmoe_pack_load + vfmoe_layer_create)."""
        lib = _lib.load()
        need = check(lib.vfmoe_pack_bytes(path.encode()))
        buf = torch.empty(need, dtype=torch.uint8, device="cuda")
        d = _lib.LayerDesc()
        check(lib.vfmoe_pack_load(path.encode(), _ptr(buf), need, C.byref(d)))
        self = cls.__new__(cls)
        self.lib = lib
        self.H, self.I, self.E, self.k = d.hidden, d.inter, d.n_experts, d.topk
        inv = {v: k for k, v in _DT.items()}
        self.x_dtype, self.out_dtype = inv[d.x_dtype], inv[d.out_dtype]
        self.fmt = {WFMT_Q8_0: "q8_0", WFMT_Q8_0_TILED: "q8_0_tiled", WFMT_EXL3: "exl3"}[d.weight_format]
        self.n_local = d.n_local_experts or d.n_experts
        self._keep = [buf]
        self.desc = d
        self.handle = check(lib.vfmoe_layer_create(C.byref(d)))
        self._ws = None
        self._rows_ws = None
        return self

    # ------------------------------------------------------------------ workspace
    def workspace_bytes(self, T: int) -> int:
        return check(self.lib.vfmoe_workspace_bytes(self.handle, T))

    def workspace(self, T: int) -> torch.Tensor:
        need = self.workspace_bytes(T)
        if self._ws is None or self._ws.numel() < need:
            self._ws = torch.empty(need, dtype=torch.uint8, device="cuda")
        return self._ws

    # ------------------------------------------------------------------ ops
    def route(self, x: torch.Tensor):
        T = x.shape[0]
        idx = torch.empty((T, self.k), dtype=torch.int32, device=x.device)
        w = torch.empty((T, self.k), dtype=torch.float32, device=x.device)
        ws = self.workspace(T)
        check(self.lib.vfmoe_route(self.handle, _ptr(x), T, _ptr(idx), _ptr(w), _ptr(ws), ws.numel(), _stream()))
        return idx, w

    def route_logits(self, x: torch.Tensor):
        """(fp32 logits [T, E] of the router's first level, c) with |logit - exact| <= c |x_t| |w_e|
        (vfmoe_route_logits; diagnostics)."""
        T = x.shape[0]
        out = torch.empty((T, self.E), dtype=torch.float32, device=x.device)
        ws = self.workspace(T)
        c = C.c_double(0.0)
        check(self.lib.vfmoe_route_logits(self.handle, _ptr(x), T, _ptr(out), C.byref(c), _ptr(ws), ws.numel(),
                                          _stream()))
        return out, c.value

    def forward(self, x: torch.Tensor, out: torch.Tensor | None = None, idx=None, w=None,
                workspace: torch.Tensor | None = None):
        assert x.dtype == self.x_dtype and x.is_contiguous() and x.shape[1] == self.H
        T = x.shape[0]
        if out is None:
            out = torch.empty((T, self.H), dtype=self.out_dtype, device=x.device)
        ws = workspace if workspace is not None else self.workspace(T)
        check(self.lib.vfmoe_forward(self.handle, _ptr(x), T, _ptr(out), _ptr(idx), _ptr(w), _ptr(ws),
                                     ws.numel(), _stream()))
        return out

    def moe_block(self, x: torch.Tensor):
        """(out, idx, w) like native/glm53/moe_ref.py:92-112."""
        T = x.shape[0]
        idx = torch.empty((T, self.k), dtype=torch.int32, device=x.device)
        w = torch.empty((T, self.k), dtype=torch.float32, device=x.device)
        out = self.forward(x, idx=idx, w=w)
        return out, idx, w

    def forward_rows(self, rows: torch.Tensor, slots: torch.Tensor, y: torch.Tensor | None = None):
        """y[i] = FFN_{slots[i]}(rows[i]) in fp32; slot n_local = shared expert."""
        n = rows.shape[0]
        if y is None:
            y = torch.empty((n, self.H), dtype=torch.float32, device=rows.device)
        need = check(self.lib.vfmoe_rows_workspace_bytes(self.handle, n))
        if self._rows_ws is None or self._rows_ws.numel() < need:
            self._rows_ws = torch.empty(need, dtype=torch.uint8, device=rows.device)
        check(self.lib.vfmoe_forward_rows(self.handle, _ptr(rows), _DT[rows.dtype], _ptr(slots), n, _ptr(y),
                                          _ptr(self._rows_ws), self._rows_ws.numel(), _stream()))
        return y

    def forward_routed(self, rows: torch.Tensor, slots: torch.Tensor, w: torch.Tensor, y_dtype=torch.float16,
                       y: torch.Tensor | None = None):
        """y[i] = sum_l w[i,l] * FFN_{slots[i,l]}(rows[i]) over lanes with slots >= 0; slot n_local =
        shared expert."""
        n, k = slots.shape
        if y is None:
            y = torch.empty((n, self.H), dtype=y_dtype, device=rows.device)
        need = check(self.lib.vfmoe_routed_workspace_bytes(self.handle, n, k))
        if self._rows_ws is None or self._rows_ws.numel() < need:
            self._rows_ws = torch.empty(need, dtype=torch.uint8, device=rows.device)
        check(self.lib.vfmoe_forward_routed(self.handle, _ptr(rows), _DT[rows.dtype], n, k, _ptr(slots), _ptr(w),
                                            _ptr(y), _DT[y.dtype], _ptr(self._rows_ws), self._rows_ws.numel(),
                                            _stream()))
        return y

    def check_device_error(self):
        check(self.lib.vfmoe_check_device_error(self.handle, _stream()))

    def debug_inject(self, kind: int, wait_ns: int = 0):
        """Failure injection for tests (vfmoe_debug_inject); kind _lib.INJECT_NONE restores."""
        check(self.lib.vfmoe_debug_inject(self.handle, kind, wait_ns))

    def close(self):
        if getattr(self, "handle", 0) > 0:
            self.lib.vfmoe_layer_destroy(self.handle)
            self.handle = 0

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


# ---------------------------------------------------------------------- standalone ops
def q8_0_quantize(src_f32: torch.Tensor, dst_u8: torch.Tensor) -> None:
    rows, k = src_f32.shape
    check(_lib.load().vfmoe_q8_0_quantize(_ptr(src_f32), _ptr(dst_u8), rows, k, _stream()))


def q8_0_dequant(src_u8: torch.Tensor, rows: int, k: int, dtype=torch.float32) -> torch.Tensor:
    out = torch.empty((rows, k), dtype=dtype, device=src_u8.device)
    check(_lib.load().vfmoe_q8_0_dequant(_ptr(src_u8), _ptr(out), rows, k, _DT[dtype], _stream()))
    return out


def exl3_decode(trellis: torch.Tensor, K: int, N: int, bits: int) -> torch.Tensor:
    out = torch.empty((K, N), dtype=torch.float16, device=trellis.device)
    check(_lib.load().vfmoe_exl3_decode(_ptr(trellis), _ptr(out), K, N, bits, _stream()))
    return out


def dispatch(idx: torch.Tensor, n_experts: int, err: torch.Tensor | None = None):
    """Canonical permutation of idx int32 [T, k] (vfmoe_dispatch): (perm_tok [T*k], pos_of [T*k],
    offsets [E+1], counts [E]) on the device; err (int32 [1], device) records an id out of range."""
    T, k = idx.shape
    dev = idx.device
    counts = torch.empty(n_experts + 2, dtype=torch.int32, device=dev)
    offsets = torch.empty(n_experts + 2, dtype=torch.int32, device=dev)
    perm = torch.empty(T * k, dtype=torch.int32, device=dev)
    pos = torch.empty(T * k, dtype=torch.int32, device=dev)
    check(_lib.load().vfmoe_dispatch(_ptr(idx), T, k, n_experts, _ptr(counts), _ptr(offsets), _ptr(perm), _ptr(pos),
                                     _ptr(err), _stream()))
    return perm, pos, offsets[:n_experts + 1], counts[:n_experts]


def combine(y: torch.Tensor, pos_of: torch.Tensor, w, T: int, k: int, y_shared=None,
            out_dtype=torch.bfloat16) -> torch.Tensor:
    """out[t] = sum_l w[t,l] * y[pos_of[t*k+l]] (+ y_shared[t]); y fp32 or fp16; pos < 0 skips."""
    H = y.shape[1]
    out = torch.empty((T, H), dtype=out_dtype, device=y.device)
    if y_shared is not None:
        assert y_shared.dtype == y.dtype
    check(_lib.load().vfmoe_combine(_ptr(y), _DT[y.dtype], _ptr(pos_of), _ptr(w), T, k, H, _ptr(y_shared), _ptr(out),
                                    _DT[out_dtype], _stream()))
    return out


def rmsnorm(x: torch.Tensor, w: torch.Tensor, eps: float = 1e-5) -> torch.Tensor:
    y = torch.empty_like(x)
    S, D = x.shape
    check(_lib.load().vfmoe_rmsnorm(_ptr(x), _ptr(w), _ptr(y), S, D, eps, _DT[x.dtype], _stream()))
    return y


def residual_rmsnorm(x: torch.Tensor, y: torch.Tensor | None, w: torch.Tensor | None, eps: float = 1e-5,
                     x_out: torch.Tensor | None = None, h: torch.Tensor | None = None):
    """(x + y, RMSNorm_w(x + y)) in one pass; y=None -> (x, RMSNorm_w(x)); w=None -> (x + y, None)."""
    S, D = x.shape
    if y is not None and x_out is None:
        x_out = torch.empty_like(x)
    if w is not None and h is None:
        h = torch.empty_like(x)
    check(_lib.load().vfmoe_residual_rmsnorm(_ptr(x), _ptr(y), _ptr(w), _ptr(x_out), _ptr(h), S, D, eps,
                                             _DT[x.dtype], _stream()))
    return (x_out if y is not None else x), h


class HyperConnection:
    """One hyper-connection site of a GLM-5.3 layer (the multi-stream residual around the MoE):
    fn [24, 4*D] (bf16 or fp32), base fp32 [24], scale fp32 [3], and the RMSNorm weight fp32 [D]
    that feeds the sublayer (None: collapsed streams unnormalised).  Streams are fp32 [R, 4, D].
    Mirrors hc_glue / hc_apply (native/glm53/glm_engine.vyb:437, :783)."""

    def __init__(self, fn, base, scale, norm_w=None, rms_eps=1e-5, hc_eps=1e-6, sinkhorn_iters=20,
                 norm_eps=1e-5):
        D = fn.shape[1] // 4
        d = _lib.HcDesc()
        d.n_streams, d.hidden = 4, D
        d.fn, d.fn_dtype = _ptr(fn), _DT[fn.dtype]
        d.base, d.scale = _ptr(base), _ptr(scale)
        d.rms_eps, d.hc_eps, d.sinkhorn_iters = rms_eps, hc_eps, sinkhorn_iters
        d.norm_w, d.norm_eps = _ptr(norm_w), norm_eps
        self.desc, self.D = d, D
        self._keep = (fn, base, scale, norm_w)
        self.lib = _lib.load()

    def mix(self, streams: torch.Tensor, h_dtype=torch.bfloat16):
        """(h [R, D] h_dtype, post fp32 [R, 4], comb fp32 [R, 4, 4]) from streams fp32 [R, 4, D]."""
        R = streams.shape[0]
        h = torch.empty((R, self.D), dtype=h_dtype, device=streams.device)
        post = torch.empty((R, 4), dtype=torch.float32, device=streams.device)
        comb = torch.empty((R, 4, 4), dtype=torch.float32, device=streams.device)
        check(self.lib.vfmoe_hc_mix(C.byref(self.desc), _ptr(streams), R, _ptr(h), _DT[h_dtype], _ptr(post),
                                    _ptr(comb), _stream()))
        return h, post, comb

    def apply(self, streams: torch.Tensor, y: torch.Tensor, post, comb, out: torch.Tensor | None = None):
        """post * y + comb^T streams -> fp32 [R, 4, D] (out may be streams: in place)."""
        R = streams.shape[0]
        if out is None:
            out = torch.empty_like(streams)
        check(self.lib.vfmoe_hc_apply(_ptr(streams), _ptr(y), _DT[y.dtype], _ptr(post), _ptr(comb), R, 4, self.D,
                                      _ptr(out), _stream()))
        return out


def hc_moe_site(site: HyperConnection, layer: MoELayer, streams: torch.Tensor, out: torch.Tensor | None = None):
    """The MoE site of a GLM-5.3 layer (tail_site, native/glm53/glm_engine.vyb:2562-3019): mix the
    streams, normalise, MoE, then the residual update of the streams."""
    h, post, comb = site.mix(streams, h_dtype=layer.x_dtype)
    y = layer.forward(h)
    return site.apply(streams, y, post, comb, out=out)


class _Quantizer:
    """Adapter used by synth.expert_q8_cuda."""

    @staticmethod
    def q8_0_quantize(src, dst):
        q8_0_quantize(src, dst.view(src.shape[0], -1))


quantizer = _Quantizer()
