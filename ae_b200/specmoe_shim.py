"""Point SpecMoE's MoE modules at this library.

SpecMoE imports its expert layer as ``from specmoe.layers.FusedMoE import FusedMoE``
(``specmoe/models/mixtral.py:54``, ``specmoe/optimizer/performance_simulator/operators/gpu_fused_moe.py:13``)
and the kernel driver as ``specmoe.layers.fused_moe_kernel`` (``specmoe/layers/FusedMoE.py:23``).
``install()`` registers this package's drop-ins under those two module names, so the
reference's model and engine code run unchanged on the B200 kernels.  Call it before the
reference's model modules are imported.
"""
from __future__ import annotations

import importlib
import sys
import types

from .layers import FusedMoE as _fused_moe_module
from .layers import fused_moe_kernel as _fused_moe_kernel_module

TARGETS = {
    "specmoe.layers.FusedMoE": _fused_moe_module,
    "specmoe.layers.fused_moe_kernel": _fused_moe_kernel_module,
}


def install() -> list:
    """Register the drop-ins; returns the module names that now resolve here."""
    for parent in ("specmoe", "specmoe.layers"):
        if parent not in sys.modules:
            try:
                importlib.import_module(parent)
            except ImportError:
                stub = types.ModuleType(parent)
                stub.__path__ = []  # a package, so submodule imports are looked up in sys.modules
                sys.modules[parent] = stub
    layers_pkg = sys.modules["specmoe.layers"]
    for name, module in TARGETS.items():
        sys.modules[name] = module
        setattr(layers_pkg, name.rsplit(".", 1)[1], module)
    return sorted(TARGETS)


def installed() -> bool:
    return all(sys.modules.get(n) is m for n, m in TARGETS.items())
