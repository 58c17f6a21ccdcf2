"""kushkash_b200: B200-native (sm_100a) kernels for kushkash's two hot paths -- quantize-on-write into int4/int8
page records and fused dequant paged decode attention -- behind kushkash's operator surface (Ops, KushCache).

The kernels live in libkush_sm100.so (C ABI: include/kushkash_b200.h), built in-tree by `python -m kushkash_b200.build`.
"""
from ._build import PAGE, BuildError, GpuConfig
from ._ops import Ops, cached_kv, dequant_records, pages_touched, record_bytes, rotation_enabled

__all__ = ["PAGE", "BuildError", "GpuConfig", "Ops", "KushCache", "MemoryStats", "cached_kv", "dequant_records",
           "pages_touched", "record_bytes", "rotation_enabled"]
__version__ = "0.1.0"


def __getattr__(name):
    if name in ("KushCache", "MemoryStats"):
        from . import cache
        return getattr(cache, name)
    raise AttributeError(name)

