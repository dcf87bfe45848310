"""CPU checks of the C ABI: libvfmoe.so loads, exports every symbol that
include/*.h declares, and rejects bad input with status codes (no GPU work)."""

import ctypes as C
import glob
import os
import re

import pytest

from vybforge_b200 import _lib

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def header_functions():
    names = set()
    for h in glob.glob(os.path.join(REPO, "include", "*.h")):
        src = open(h).read()
        src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
        for m in re.finditer(r"^\s*(?:int|int64_t|void|const char\s*\*)\s+(vfmoe_\w+)\s*\(", src, re.M):
            names.add(m.group(1))
    return sorted(names)


def header_defines():
    src = open(os.path.join(REPO, "include", "vfmoe.h")).read()
    return {m.group(1): int(m.group(2)) for m in re.finditer(r"#define\s+(VFMOE_\w+)\s+\(?(-?\d+)\)?", src)}


def test_library_exports_every_header_symbol(built_lib):
    names = header_functions()
    assert "vfmoe_forward" in names and "vfmoe_route" in names
    missing = [n for n in names if not hasattr(built_lib, n)]
    assert not missing, missing


def test_python_binding_covers_header():
    assert set(header_functions()) <= set(_lib._SIGS)


def test_constants_match_header():
    d = header_defines()
    assert d["VFMOE_ABI_VERSION"] == _lib.ABI_VERSION == 3
    for k in ("OK", "ERR_INVALID", "ERR_CUDA", "ERR_NOMEM", "ERR_HANDLE", "ERR_WORKSPACE", "ERR_DEVICE",
              "ERR_UNSUPPORTED", "ERR_NCCL"):
        assert d["VFMOE_" + k] == getattr(_lib, k)
    assert (d["VFMOE_DT_F32"], d["VFMOE_DT_F16"], d["VFMOE_DT_BF16"]) == (0, 1, 2)  # native/dtype/dtype.vyb
    assert (d["VFMOE_WFMT_Q8_0"], d["VFMOE_WFMT_EXL3"]) == (_lib.WFMT_Q8_0, _lib.WFMT_EXL3)
    assert (d["VFMOE_PATH_AUTO"], d["VFMOE_PATH_SIMT"], d["VFMOE_PATH_TC"], d["VFMOE_PATH_GEMV"], d["VFMOE_PATH_TC1"]) == (
        _lib.PATH_AUTO, _lib.PATH_SIMT, _lib.PATH_TC, _lib.PATH_GEMV, _lib.PATH_TC1)
    assert (d["VFMOE_INJECT_NONE"], d["VFMOE_INJECT_STALL_LOADS"]) == (_lib.INJECT_NONE, _lib.INJECT_STALL_LOADS)


def test_descriptor_is_a_block_of_8_byte_words():
    assert C.sizeof(_lib.Matrix) == 6 * 8
    assert C.sizeof(_lib.LayerDesc) == (12 + 6 * 6 + 3) * 8


def test_version(built_lib):
    assert built_lib.vfmoe_version() == 3


def _desc(**kw):
    d = _lib.LayerDesc()
    d.hidden, d.inter, d.n_experts, d.topk = 1024, 512, 16, 4
    d.weight_format, d.x_dtype, d.out_dtype = _lib.WFMT_Q8_0, _lib.DT_F32, _lib.DT_F32
    d.routed_scale, d.swiglu_limit = 2.5, 10.0
    d.router_w, d.router_bias = 4096, 8192
    d.gate.data, d.up.data, d.down.data = 1 << 20, 2 << 20, 3 << 20
    d.gate.expert_stride = d.up.expert_stride = 512 * 1088
    d.down.expert_stride = 1024 * 544
    for k, v in kw.items():
        setattr(d, k, v)
    return d


@pytest.mark.parametrize("field,value", [("hidden", 1000), ("topk", 40), ("topk", 0), ("x_dtype", 7),
                                         ("weight_format", 9), ("n_experts", 0), ("router_w", 0)])
def test_invalid_descriptor_rejected(built_lib, field, value):
    d = _desc(**{field: value})
    rc = built_lib.vfmoe_layer_create(C.byref(d))
    assert rc == _lib.ERR_INVALID
    assert "invalid layer descriptor" in _lib.last_error()


def _exl3_desc(bits):
    d = _desc(weight_format=_lib.WFMT_EXL3, exl3_bits=bits)
    for m, (k, n) in ((d.gate, (1024, 512)), (d.up, (1024, 512)), (d.down, (512, 1024))):
        m.expert_stride = k // 16 * n // 16 * 2 * 16 * bits
        m.suh, m.svh = 16 << 20, 17 << 20
        m.suh_stride, m.svh_stride = 2 * k, 2 * n
    return d


def test_exl3_descriptors(built_lib):
    assert built_lib.vfmoe_layer_create(C.byref(_exl3_desc(5))) == _lib.ERR_INVALID
    assert "exl3_bits must be 3 or 4" in _lib.last_error()
    d = _exl3_desc(3)
    d.up.suh = 0
    assert built_lib.vfmoe_layer_create(C.byref(d)) == _lib.ERR_INVALID
    assert "suh and svh" in _lib.last_error()
    d = _exl3_desc(3)
    d.down.expert_stride -= 16
    assert built_lib.vfmoe_layer_create(C.byref(d)) == _lib.ERR_INVALID


def test_null_descriptor_and_unknown_handle(built_lib):
    assert built_lib.vfmoe_layer_create(None) == _lib.ERR_INVALID
    assert built_lib.vfmoe_layer_destroy(12345) == _lib.ERR_HANDLE
    assert built_lib.vfmoe_workspace_bytes(12345, 8) == _lib.ERR_HANDLE
    assert built_lib.vfmoe_forward(12345, 0, 1, 0, 0, 0, 0, 0, 0) == _lib.ERR_HANDLE
    assert "unknown layer handle" in _lib.last_error()


def test_standalone_ops_validate_arguments(built_lib):
    assert built_lib.vfmoe_q8_0_dequant(0, 0, 4, 33, 0, 0) == _lib.ERR_INVALID
    assert built_lib.vfmoe_q8_0_quantize(0, 0, 4, 30, 0) == _lib.ERR_INVALID
    assert built_lib.vfmoe_exl3_decode(0, 0, 15, 16, 3, 0) == _lib.ERR_INVALID
    assert built_lib.vfmoe_q8_0_tile(4096, 1 << 30, 96, 512, 1, 0) == _lib.ERR_INVALID       # rows % 64
    assert built_lib.vfmoe_q8_0_tile(4096, 1 << 30, 64, 288, 1, 0) == _lib.ERR_INVALID       # k % 256
    assert built_lib.vfmoe_q8_0_tile(4104, 1 << 30, 64, 512, 1, 0) == _lib.ERR_INVALID       # misaligned
    assert built_lib.vfmoe_q8_0_tile(4096, 4096 + 16, 64, 512, 1, 0) == _lib.ERR_INVALID     # overlap
    assert "overlaps" in _lib.last_error()
    assert built_lib.vfmoe_q8_0_tile(0, 0, 64, 512, 0, 0) == _lib.OK                          # nothing to do
    assert built_lib.vfmoe_rmsnorm(0, 0, 0, 2, 0, 1e-5, 0, 0) == _lib.ERR_INVALID
    assert built_lib.vfmoe_residual_rmsnorm(0, 0, 0, 0, 0, 2, 64, 1e-5, 2, 0) == _lib.ERR_INVALID       # no x
    assert built_lib.vfmoe_residual_rmsnorm(4096, 0, 0, 0, 0, 2, 64, 1e-5, 2, 0) == _lib.ERR_INVALID    # no y, no w
    assert built_lib.vfmoe_residual_rmsnorm(4096, 8192, 0, 0, 0, 2, 64, 1e-5, 2, 0) == _lib.ERR_INVALID  # y, no x_out
    assert built_lib.vfmoe_residual_rmsnorm(4096, 0, 8192, 0, 0, 2, 64, 1e-5, 1, 0) == _lib.ERR_INVALID  # f16


def test_init_without_device_returns_status(built_lib):
    import torch
    if torch.cuda.is_available():
        pytest.skip("has a GPU")
    rc = built_lib.vfmoe_init(0)
    assert rc < 0
    assert _lib.last_error()


def test_pack_load_rejects_a_file_that_is_not_a_pack(built_lib, tmp_path):
    p = tmp_path / "junk.vfpk"
    p.write_bytes(b"not a pack" * 1000)
    assert built_lib.vfmoe_pack_bytes(str(p).encode()) == _lib.ERR_INVALID
    assert "not a version-1 vfmoe pack" in _lib.last_error()
    assert built_lib.vfmoe_pack_bytes(str(tmp_path / "missing").encode()) == _lib.ERR_INVALID
