"""Route an installed kushkash package's GPU path to libkush_sm100.so.

kushkash's own operator layer (kushkash/_ops.py:42-213, class Ops) reaches the GPU through exactly two names:
`from . import _cuda` (the kernel loader: `kernels(device, cfg)`, `arch(device)`, `sm_count(device)`,
kushkash/_cuda.py:106-117) and `from ._build import GpuConfig` (kushkash/_build.py:112-149).  `install()` puts this
package's ctypes shim in place of the first and its GpuConfig in place of the second, so that the unmodified
kushkash.Ops, kushkash.KushCache (cache.py), the Hugging Face cache and generate (hf.py, _generate.py) and the vLLM
and SGLang backends launch the sm_100a kernels of this library instead of Mojo-built PTX.  Nothing of kushkash is
edited or copied; its CPU path (kushkash._cpu, the Mojo CPU library) is left as it is.

    import kushkash_b200.dropin
    kushkash = kushkash_b200.dropin.install()      # before the first kushkash.Ops / KushCache is built on a GPU
"""
from __future__ import annotations

import importlib
import sys
from types import ModuleType

from . import _build, _cuda


def install(package: str = "kushkash") -> ModuleType:
    """Bind `package` (an importable kushkash distribution) to this library's kernels and return it.

    Idempotent.  Must run before the package's Ops objects for CUDA devices are constructed (each Ops resolves its
    loader once, in __init__).  The package must be kushkash >= 0.6 (the loader contract of kushkash/_cuda.py)."""
    sys.modules[f"{package}._cuda"] = _cuda
    build = importlib.import_module(f"{package}._build")        # imports the package itself first (torch only)
    build.GpuConfig = _build.GpuConfig
    pkg = importlib.import_module(package)
    pkg._cuda = _cuda
    return pkg


def installed(package: str = "kushkash") -> bool:
    """Whether `package`'s GPU loader is this library's shim."""
    return sys.modules.get(f"{package}._cuda") is _cuda
