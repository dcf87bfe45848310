"""vybforge_b200 -- B200-native (sm_100a) GLM-style MoE layer behind a C ABI.

The compute lives in ``libvfmoe.so`` (``vybforge_b200/csrc``, built by
``python -m vybforge_b200.build``); ``include/vfmoe.h`` is its contract.
``vybforge_b200.moe`` is the Python host mirror used by the tests and bench.
"""

from ._lib import LIB_PATH, load, VfmoeError  # noqa: F401

__all__ = ["LIB_PATH", "load", "VfmoeError"]
