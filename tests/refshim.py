"""pytest plugin (`-p refshim`) that runs the kushkash reference package and its own test files over this repository.

TEST INFRASTRUCTURE.  Before the reference's tests import kushkash, it binds the package's two back ends:
  * GPU: kushkash._cuda / kushkash._build.GpuConfig -> kushkash_b200 (the product: libkush_sm100.so), through
    kushkash_b200.dropin.install(), the binding a user of the reference makes;
  * CPU: kushkash._cpu (the Mojo-built CPU library, which cannot be built without the mojo compiler) -> the C
    oracle under oracle/, which exports the same kush_cpu_* C ABI (kushkash/_cpu.py:10-40).
KUSHKASH_PAGE=16 runs everything at 16-token pages: the drop-in sets kushkash's PAGE constants and GpuConfig, and the
oracle takes the reference's CPU calls through its page-size variants.
So the reference's GPU tests compare this library against the oracle exactly where they compare the Mojo GPU
kernels against the Mojo CPU library, and its CPU tests check the oracle against the reference's PyTorch pins.
The kushkash package and its tests are read from where the caller's PYTHONPATH and command line point (a local
install of the unmodified reference); nothing of them is copied into this repository.
"""
import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parents[1]
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))

import os  # noqa: E402
import types  # noqa: E402

from oracle import kush_oracle  # noqa: E402

PAGE = int(os.environ.get("KUSHKASH_PAGE", "32"))


def _paged_cpu(page: int) -> types.ModuleType:
    """kushkash._cpu for `page`-token records: the oracle's kush_cpu_* entry points, through their `_p` variants (the
    page size first) when page != 32 (the reference's CPU ABI, kushkash/_cpu.py:10-40, has no page argument)."""
    if page == 32:
        return kush_oracle
    mod = types.ModuleType("kushkash._cpu")
    paged = {"kush_cpu_append", "kush_cpu_write", "kush_cpu_decode", "kush_cpu_unpack"}

    def call(name, *args):
        if name in paged:
            return kush_oracle.call(name + "_p", page, *args)
        return kush_oracle.call(name, *args)

    mod.call = call
    return mod


sys.modules["kushkash._cpu"] = _paged_cpu(PAGE)

import kushkash_b200.dropin  # noqa: E402

kushkash_b200.dropin.install(page=PAGE)


def _transformers_compat() -> None:
    """transformers 5.5 (the version installed here) declares CacheLayerMixin.get_max_cache_shape abstract; kushkash
    0.6's cache layer (kushkash/hf.py:34-59) implements that contract under the older name get_max_length, so the
    reference's HF integration cannot be instantiated on this transformers at all.  Alias the method (nothing else
    of the reference changes)."""
    try:
        import kushkash.hf as hf
    except ImportError:                     # no transformers: the HF tests skip or fail on their own
        return
    layer = hf._KushLayer
    if "get_max_cache_shape" in getattr(layer, "__abstractmethods__", ()):
        layer.get_max_cache_shape = layer.get_max_length
        layer.__abstractmethods__ = frozenset(layer.__abstractmethods__ - {"get_max_cache_shape"})


_transformers_compat()
