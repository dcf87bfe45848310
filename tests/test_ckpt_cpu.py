"""The checkpoint reader (vfmoe_ckpt_*, include/vfmoe.h) on CPU: synthetic safetensors shards
behind an index, read into host memory through the C ABI and compared byte for byte; the
errors a broken checkpoint must give (missing name, index naming a shard that lacks the tensor,
a hollow shard whose data region is shorter than its header says)."""

import json
import os

import numpy as np
import pytest

from vybforge_b200 import _lib
from vybforge_b200.ckpt import Checkpoint

from ckpt_writer import write_safetensors, write_sharded


@pytest.fixture
def tensors():
    rng = np.random.default_rng(0)
    return {"a.weight": ("BF16", rng.integers(0, 1 << 16, (4, 8), dtype=np.uint16)),
            "a.bias": ("F32", rng.standard_normal(8).astype(np.float32)),
            "b.trellis": ("I16", rng.integers(-32768, 32768, (2, 3, 64), dtype=np.int16)),
            "b.mcg": ("I32", np.array([7], np.int32)),
            "c.scale": ("F16", rng.standard_normal(5).astype(np.float16)),
            "empé.w": ("F32", np.zeros((0, 3), np.float32))}


def test_sharded_checkpoint_reads_every_tensor(tmp_path, tensors):
    write_sharded(str(tmp_path), tensors, n_shards=3)
    ck = Checkpoint(str(tmp_path))
    for name, (dt, a) in tensors.items():
        info = ck.info(name)
        assert info["dtype"] == dt and info["shape"] == a.shape and info["nbytes"] == a.nbytes
        got = ck.read_numpy(name)
        np.testing.assert_array_equal(got.view(a.dtype), a)
    assert not ck.has("missing.weight")
    ck.close()


def test_single_file_checkpoint(tmp_path, tensors):
    write_safetensors(str(tmp_path / "model.safetensors"), tensors)
    ck = Checkpoint(str(tmp_path))
    np.testing.assert_array_equal(ck.read_numpy("b.trellis"), tensors["b.trellis"][1])
    ck.close()


def test_missing_and_misplaced_tensors_are_errors(tmp_path, tensors):
    write_sharded(str(tmp_path), tensors, n_shards=2)
    idx = json.load(open(tmp_path / "model.safetensors.index.json"))
    other = {f for f in idx["weight_map"].values() if f != idx["weight_map"]["a.bias"]}.pop()
    idx["weight_map"]["a.bias"] = other                  # the index points at a shard without it
    json.dump(idx, open(tmp_path / "model.safetensors.index.json", "w"))
    ck = Checkpoint(str(tmp_path))
    with pytest.raises(_lib.VfmoeError, match="lacks it"):
        ck.info("a.bias")
    with pytest.raises(_lib.VfmoeError, match="no tensor"):
        ck.info("nope")
    ck.close()


def test_hollow_shard_is_rejected(tmp_path, tensors):
    """A shard whose file is shorter than its header's data region (a copied tree of dangling links
    or a partial download) is refused when a name first resolves to it."""
    write_sharded(str(tmp_path), tensors, n_shards=2)
    shard = tmp_path / json.load(open(tmp_path / "model.safetensors.index.json"))["weight_map"]["b.trellis"]
    data = shard.read_bytes()
    shard.write_bytes(data[:-10])
    ck = Checkpoint(str(tmp_path))
    with pytest.raises(_lib.VfmoeError, match="beyond the file"):
        ck.info("b.trellis")
    ck.close()


def test_destination_too_small_is_an_error(tmp_path, tensors):
    write_sharded(str(tmp_path), tensors, n_shards=1)
    ck = Checkpoint(str(tmp_path))
    buf = np.empty(3, np.float32)
    rc = ck.lib.vfmoe_ckpt_read(ck.handle, b"a.bias", buf.ctypes.data, buf.nbytes, 0)
    assert rc == _lib.ERR_INVALID
    ck.close()
