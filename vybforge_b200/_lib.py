"""ctypes binding of libvfmoe.so (the C ABI in include/vfmoe.h).

This is the same binding a non-Python host makes (a Vyb host declares the same functions
in an ``extern "C"`` block): plain int64 addresses, int status codes.  If the library
is missing the import fails loudly -- there is no CPU fallback.
"""

from __future__ import annotations

import ctypes as C
import os

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libvfmoe.so")

# status codes (vfmoe.h)
OK = 0
ERR_INVALID = -1
ERR_CUDA = -2
ERR_NOMEM = -3
ERR_HANDLE = -4
ERR_WORKSPACE = -5
ERR_DEVICE = -6
ERR_UNSUPPORTED = -7
ERR_NCCL = -8

# dtype ids (native/dtype/dtype.vyb:26-28)
DT_F32, DT_F16, DT_BF16 = 0, 1, 2
# weight formats
WFMT_Q8_0, WFMT_EXL3, WFMT_Q8_0_TILED, WFMT_BF16 = 1, 2, 3, 4
# expert kernel families (vfmoe_layer_desc.expert_path)
PATH_AUTO, PATH_SIMT, PATH_TC, PATH_GEMV, PATH_TC1 = 0, 1, 2, 3, 4
# failure injection (vfmoe_debug_inject)
INJECT_NONE, INJECT_STALL_LOADS = 0, 1
ABI_VERSION = 3


class VfmoeError(RuntimeError):
    def __init__(self, code: int, msg: str):
        super().__init__(f"vfmoe error {code}: {msg}")
        self.code = code


class Matrix(C.Structure):
    _fields_ = [("data", C.c_int64), ("expert_stride", C.c_int64), ("suh", C.c_int64),
                ("suh_stride", C.c_int64), ("svh", C.c_int64), ("svh_stride", C.c_int64)]


class LayerDesc(C.Structure):
    _fields_ = [("hidden", C.c_int64), ("inter", C.c_int64), ("n_experts", C.c_int64), ("topk", C.c_int64),
                ("weight_format", C.c_int64), ("exl3_bits", C.c_int64), ("x_dtype", C.c_int64),
                ("out_dtype", C.c_int64), ("routed_scale", C.c_double), ("swiglu_limit", C.c_double),
                ("router_w", C.c_int64), ("router_bias", C.c_int64),
                ("gate", Matrix), ("up", Matrix), ("down", Matrix),
                ("sh_gate", Matrix), ("sh_up", Matrix), ("sh_down", Matrix), ("n_local_experts", C.c_int64),
                ("expert_path", C.c_int64), ("shared_format", C.c_int64)]


class HcDesc(C.Structure):
    _fields_ = [("n_streams", C.c_int64), ("hidden", C.c_int64), ("fn", C.c_int64), ("fn_dtype", C.c_int64),
                ("base", C.c_int64), ("scale", C.c_int64), ("rms_eps", C.c_double), ("hc_eps", C.c_double),
                ("sinkhorn_iters", C.c_int64), ("norm_w", C.c_int64), ("norm_eps", C.c_double)]


class TensorInfo(C.Structure):
    _fields_ = [("dtype", C.c_int64), ("ndim", C.c_int64), ("shape", C.c_int64 * 8), ("nbytes", C.c_int64),
                ("file_offset", C.c_int64), ("shard", C.c_int64)]


# safetensors dtype ids (vfmoe.h VFMOE_ST_*)
ST_NAMES = ["F32", "F16", "BF16", "F64", "I64", "I32", "I16", "I8", "U8", "BOOL", "U16", "U32", "U64", "F8_E4M3",
            "F8_E5M2"]

I64 = C.c_int64
_SIGS = {
    "vfmoe_version": (C.c_int, []),
    "vfmoe_init": (C.c_int, [C.c_int]),
    "vfmoe_last_error": (C.c_int, [C.c_char_p, I64]),
    "vfmoe_layer_create": (I64, [C.POINTER(LayerDesc)]),
    "vfmoe_layer_destroy": (C.c_int, [I64]),
    "vfmoe_workspace_bytes": (I64, [I64, I64]),
    "vfmoe_route": (C.c_int, [I64] * 8),
    "vfmoe_route_noalloc": (C.c_int, [I64] * 6),
    "vfmoe_route_logits": (C.c_int, [I64, I64, I64, I64, C.POINTER(C.c_double), I64, I64, I64]),
    "vfmoe_forward": (C.c_int, [I64] * 9),
    "vfmoe_check_device_error": (C.c_int, [I64, I64]),
    "vfmoe_dispatch": (C.c_int, [I64] * 10),
    "vfmoe_ep_unique_id": (C.c_int, [C.c_void_p, I64]),
    "vfmoe_ep_init": (I64, [I64, I64, C.c_void_p, I64]),
    "vfmoe_ep_destroy": (C.c_int, [I64]),
    "vfmoe_ep_set_placement": (C.c_int, [I64, I64, I64, C.POINTER(C.c_int32), I64, C.POINTER(C.c_int32), I64]),
    "vfmoe_ep_workspace_bytes": (I64, [I64, I64]),
    "vfmoe_ep_buffers": (C.c_int, [I64, I64, C.POINTER(I64), I64]),
    "vfmoe_ep_prepare": (C.c_int, [I64] * 9),
    "vfmoe_ep_shared": (C.c_int, [I64] * 7),
    "vfmoe_ep_experts": (C.c_int, [I64] * 5),
    "vfmoe_ep_combine": (C.c_int, [I64] * 7),
    "vfmoe_ep_forward": (C.c_int, [I64] * 11),
    "vfmoe_debug_inject": (C.c_int, [I64, I64, I64]),
    "vfmoe_rows_workspace_bytes": (I64, [I64, I64]),
    "vfmoe_forward_rows": (C.c_int, [I64] * 9),
    "vfmoe_combine": (C.c_int, [I64] * 11),
    "vfmoe_routed_workspace_bytes": (I64, [I64, I64, I64]),
    "vfmoe_forward_routed": (C.c_int, [I64] * 12),
    "vfmoe_profile_enable": (C.c_int, [I64, C.c_int]),
    "vfmoe_profile_read": (C.c_int, [I64, C.POINTER(C.c_double), I64, C.POINTER(I64)]),
    "vfmoe_rmsnorm": (C.c_int, [I64, I64, I64, I64, I64, C.c_double, I64, I64]),
    "vfmoe_hc_mix": (C.c_int, [C.POINTER(HcDesc), I64, I64, I64, I64, I64, I64, I64]),
    "vfmoe_hc_apply": (C.c_int, [I64] * 10),
    "vfmoe_ckpt_open": (I64, [C.c_char_p]),
    "vfmoe_ckpt_close": (C.c_int, [I64]),
    "vfmoe_ckpt_find": (C.c_int, [I64, C.c_char_p, C.POINTER(TensorInfo)]),
    "vfmoe_ckpt_read": (C.c_int, [I64, C.c_char_p, I64, I64, I64]),
    "vfmoe_pack_save": (C.c_int, [C.c_char_p, C.POINTER(LayerDesc)]),
    "vfmoe_pack_bytes": (I64, [C.c_char_p]),
    "vfmoe_pack_load": (C.c_int, [C.c_char_p, I64, I64, C.POINTER(LayerDesc)]),
    "vfmoe_residual_rmsnorm": (C.c_int, [I64, I64, I64, I64, I64, I64, I64, C.c_double, I64, I64]),
    "vfmoe_q8_0_dequant": (C.c_int, [I64] * 6),
    "vfmoe_q8_0_quantize": (C.c_int, [I64] * 5),
    "vfmoe_q8_0_tile": (C.c_int, [I64] * 6),
    "vfmoe_exl3_decode": (C.c_int, [I64] * 6),
}

_lib = None


def load():
    """Load libvfmoe.so once (raises if it has not been built)."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            # a checkout without the built library compiles it from csrc/ (nvcc, sm_100a); a
            # failed build raises: there is no CPU fallback for the MoE path
            from . import build
            build.build()
        lib = C.CDLL(LIB_PATH)
        for name, (res, args) in _SIGS.items():
            f = getattr(lib, name)
            f.restype = res
            f.argtypes = args
        if lib.vfmoe_version() != ABI_VERSION:
            raise RuntimeError(f"{LIB_PATH} has ABI version {lib.vfmoe_version()}, this binding expects "
                               f"{ABI_VERSION}: rebuild with `python -m vybforge_b200.build`")
        _lib = lib
    return _lib


def last_error() -> str:
    lib = load()
    buf = C.create_string_buffer(2048)
    lib.vfmoe_last_error(buf, 2048)
    return buf.value.decode(errors="replace")


def check(rc: int) -> int:
    if rc < 0:
        raise VfmoeError(rc, last_error())
    return rc
