"""Route an installed kushkash package's GPU path to libkush_sm100.so, optionally at 16-token pages.

kushkash's own operator layer (kushkash/_ops.py:42-213, class Ops) reaches the GPU through exactly two names:
`from . import _cuda` (the kernel loader: `kernels(device, cfg)`, `arch(device)`, `sm_count(device)`,
kushkash/_cuda.py:106-117) and `from ._build import GpuConfig` (kushkash/_build.py:112-149).  `install()` puts this
package's ctypes shim in place of the first and its GpuConfig in place of the second, so that the unmodified
kushkash.Ops, kushkash.KushCache (cache.py), the Hugging Face cache and generate (hf.py, _generate.py) and the vLLM
and SGLang backends launch the sm_100a kernels of this library instead of Mojo-built PTX.  Nothing of kushkash is
edited or copied; its CPU path (kushkash._cpu, the Mojo CPU library) is left as it is.

Page size.  kushkash fixes 32 tokens per page record (kushkash/kush/quant.mojo:16) and every Python module of it
reads that size from a module constant PAGE: kushkash/_ops.py:25 and _build.py:26, the copies bound by
`from kushkash._ops import PAGE` (cache.py:20, sglang/pool.py:15, sglang/backend.py:25, vllm/backend.py:55) and
the SGLang plugin's own (sglang/__init__.py:22, which declares SGLang's page_size from it).  `install(page=16)` (or
KUSHKASH_PAGE=16 in the environment) sets all of them to 16 and makes GpuConfig default to 16-token kernels, so the
record spec (record_bytes), the block tables (one entry per 16 tokens), the exact-K tails [slots, Hkv, 16, D], the
SGLang page_size declaration and KV-pool sizing, vLLM's kernel block size and spec, and the kernels all agree on
16-token pages.  The Mojo CPU library stays 32-token only: at page 16 only CUDA devices are supported.

    import kushkash_b200.dropin
    kushkash = kushkash_b200.dropin.install()              # before the first kushkash.Ops / KushCache is built
    kushkash = kushkash_b200.dropin.install(page=16)       # the same at 16-token pages
"""
from __future__ import annotations

import importlib
import os
import sys
from types import ModuleType

from . import _build, _cuda

# modules of kushkash that define or bind PAGE, imported by install() so that a later import cannot bring back 32
# (the SGLang and vLLM plugin packages import their frameworks lazily; a missing framework is skipped)
_PAGE_MODULES = ("_build", "_ops", "cache", "sglang", "sglang.pool", "sglang.backend", "vllm", "vllm.backend")


def install(package: str = "kushkash", page: int | None = None) -> ModuleType:
    """Bind `package` (an importable kushkash distribution) to this library's kernels and return it.

    page: tokens per page record, 32 (kushkash's) or 16; None reads KUSHKASH_PAGE (default 32).  Idempotent for a
    given page.  Must run before the package's Ops objects for CUDA devices are constructed (each Ops resolves its
    loader and configuration once, in __init__).  The package must be kushkash >= 0.6 (the loader contract of
    kushkash/_cuda.py)."""
    if page is None:
        page = int(os.environ.get("KUSHKASH_PAGE", str(_build.PAGE)))
    if page not in (16, 32):
        raise ValueError(f"install: page must be 16 or 32, got {page}")
    sys.modules[f"{package}._cuda"] = _cuda
    build = importlib.import_module(f"{package}._build")        # imports the package itself first (torch only)
    build.GpuConfig = _build.config_class(page)
    pkg = importlib.import_module(package)
    pkg._cuda = _cuda
    set_page(package, page)
    return pkg


def set_page(package: str, page: int) -> list[str]:
    """Set PAGE in every loaded module of `package` that has it, importing the known ones first; returns the names
    of the modules changed or already at `page`."""
    for name in _PAGE_MODULES:
        try:
            importlib.import_module(f"{package}.{name}")
        except Exception:                   # noqa: BLE001 -- a plugin whose framework is absent or incompatible
            continue
    done = []
    for name, mod in list(sys.modules.items()):
        if (name == package or name.startswith(package + ".")) and isinstance(getattr(mod, "PAGE", None), int):
            mod.PAGE = page
            done.append(name)
    return sorted(done)


def installed(package: str = "kushkash") -> bool:
    """Whether `package`'s GPU loader is this library's shim."""
    return sys.modules.get(f"{package}._cuda") is _cuda


def page(package: str = "kushkash") -> int:
    """The page size `package` is running with (its kushkash._ops.PAGE)."""
    return importlib.import_module(f"{package}._ops").PAGE
