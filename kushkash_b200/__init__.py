"""kushkash_b200: B200-native (sm_100a) kernels for kushkash's two hot paths -- quantize-on-write into int4/int8
page records and fused dequant paged decode attention.

The kernels live in libkush_sm100.so (C ABI: include/kushkash_b200.h), built in-tree by `python -m kushkash_b200.build`.
Two ways in:
  * kushkash_b200.dropin.install() binds an installed kushkash package (its Ops, KushCache, HF / vLLM / SGLang
    integrations, unchanged) to these kernels through the drop-in loader kushkash_b200._cuda;
  * kushkash_b200.Ops calls the C ABI directly (page size 16 or 32, fused rotation, launch order, split partials).
"""
from ._build import PAGE, BuildError, GpuConfig
from ._ops import Ops, record_bytes, split_factor

__all__ = ["PAGE", "BuildError", "GpuConfig", "Ops", "record_bytes", "split_factor"]
__version__ = "0.2.0"
