"""ctypes binding of the C ABI in ``include/ae_b200.h`` (``ae_b200/libae_b200.so``).

There is no CPU fallback: if the library is missing or the device is not a B200, the
calls raise.  Build the library with ``python -m ae_b200.build``.
"""
from __future__ import annotations

import ctypes
import os
import threading

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libae_b200.so")

DTYPE_F16, DTYPE_BF16, DTYPE_F32 = 0, 1, 2

# Every entry point declared in include/ae_b200.h, with (restype, argtypes).
_P = ctypes.c_void_p
_I = ctypes.c_int
_L = ctypes.c_int64
_S = ctypes.c_size_t
SIGNATURES = {
    "smb_version": (_I, []),
    "smb_strerror": (ctypes.c_char_p, [_I]),
    "smb_last_cuda_error": (ctypes.c_char_p, []),
    "smb_moe_workspace_bytes": (_S, [_I, _I, _I, _I, _I, _I]),
    "smb_moe_splits": (_I, [_I, _I, _I, _I]),
    "smb_moe_ep_workspace_bytes": (_S, [_I, _I, _I, _I, _I, _I]),
    "smb_moe_route": (_I, [_P, _I, _P, _I, _I, _I, _I, _I, _I, _I, _P, _P, _P, _S, _P]),
    "smb_moe_permute": (_I, [_P, _P, _P, _I, _I, _I, _I, _I, _I, _P, _S, _P]),
    "smb_moe_ffn": (_I, [_P, _P, _L, _P, _I, _I, _I, _I, _I, _I, _P, _S, _P]),
    "smb_moe_gate_up": (_I, [_P, _P, _L, _P, _I, _I, _I, _I, _I, _I, _P, _S, _P]),
    "smb_moe_down": (_I, [_P, _L, _P, _I, _I, _I, _I, _I, _I, _P, _S, _P]),
    "smb_moe_combine": (_I, [_P, _I, _I, _I, _I, _I, _I, _P, _S, _P]),
    "smb_moe_combine_rows": (_I, [_P, _P, _I, _I, _I, _I, _I, _I, _P, _S, _P]),
    "smb_moe_ep_dispatch": (_I, [_P, _I, _P, _I, _I, _I, _I, _I, _I, _I, _I, _I, _P, _P, _P, _P, _S, _P]),
    "smb_moe_ep_experts": (_I, [_P, _I, _I, _P, _L, _P, _I, _I, _I, _I, _P, _P, _S, _P]),
    "smb_moe_ep_combine": (_I, [_P, _P, _I, _I, _I, _I, _I, _I, _I, _I, _P, _S, _P]),
    "smb_moe_forward": (_I, [_P, _P, _I, _P, _L, _P, _I, _I, _I, _I, _I, _I, _I, _P, _P, _P, _P, _S, _P]),
    "smb_moe_forward_routed": (_I, [_P, _P, _P, _P, _L, _P, _I, _I, _I, _I, _I, _I, _P, _P, _S, _P]),
    "smb_moe_forward_noalloc": (_I, [_P, _P, _I, _P, _L, _P, _I, _I, _I, _I, _I, _I, _I, _P, _P, _P, _P]),
    "smb_moe_page_copy": (_I, [_P, _P, _S, _P, _I, _P]),
    "smb_moe_forward_streamed": (_I, [_P, _P, _I, _P, _L, _P, _P, _I, _I, _I, _I, _I, _I, _I, _I, _P, _P, _P, _P,
                                      _S, _P]),
    "smb_ep_arena_bytes": (_S, [_I, _I, _I, _I]),
    "smb_ep_ipc_alloc": (_I, [_S, ctypes.POINTER(ctypes.c_void_p), _P]),
    "smb_ep_ipc_open": (_I, [_P, ctypes.POINTER(ctypes.c_void_p)]),
    "smb_ep_ipc_close": (_I, [_P]),
    "smb_ep_ipc_free": (_I, [_P]),
    "smb_ep_arena_reset": (_I, [_P, _I, _I, _I, _I, _P]),
    "smb_moe_ep_dispatch_p2p": (_I, [_P, _I, _P, _I, _I, _I, _I, _I, _I, _I, _I, _I, _I, _P, _P, _P, _P, _S, _P]),
    "smb_moe_ep_experts_p2p": (_I, [_I, _I, _I, _P, _P, _L, _P, _I, _I, _I, _I, _P, _S, _P]),
    "smb_moe_ep_combine_p2p": (_I, [_P, _I, _I, _I, _I, _I, _I, _I, _I, _I, _P, _P, _S, _P]),
    "smb_moe_forward_shared": (_I, [_P, _P, _I, _P, _P, _L, _P, _I, _I, _I, _I, _I, _I, _I, _I, _P, _P, _P, _P,
                                    _S, _P]),
    "smb_moe_workspace_init": (_I, [_P, _S, _P]),
    "smb_moe_gate": (_I, [_P, _P, _I, _I, _I, _I, _P, _P]),
    "smb_moe_forward_gated": (_I, [_P, _P, _P, _L, _P, _I, _I, _I, _I, _I, _I, _I, _P, _P, _P, _P, _P, _S, _P]),
    "smb_moe_align_block_size": (_I, [_P, _I, _I, _I, _P, _P, _P, _P]),
    "smb_moe_topk": (_I, [_P, _I, _I, _I, _I, _I, _P, _P, _P]),
    "smb_moe_read_status": (_I, [_P, _S, _I, _I, _I, _I, _I, _I, _P]),
    "smb_moe_read_timers": (_I, [_P, _S, _I, _P, _P]),
    "smb_moe_noalloc_read_status": (_I, [_P]),
}


class Timers(ctypes.Structure):
    """``smb_timers_t`` of ``include/ae_b200.h``: device-side kernel timers of a workspace."""

    _fields_ = [("ffn_ns", ctypes.c_uint64), ("recv_wait_ns", ctypes.c_uint64),
                ("combine_wait_ns", ctypes.c_uint64), ("ffn_launches", ctypes.c_uint32),
                ("recv_waits", ctypes.c_uint32), ("combine_waits", ctypes.c_uint32),
                ("reserved", ctypes.c_uint32), ("stage_ns", ctypes.c_uint64 * 5),
                ("stage_calls", ctypes.c_uint32 * 5), ("reserved2", ctypes.c_uint32),
                ("stage_busy_ns", ctypes.c_uint64 * 5)]

    STAGES = ("route", "reserved", "ffn", "combine", "final_combine")

    def as_dict(self):
        d = {f[0]: int(getattr(self, f[0])) for f in self._fields_[:6]}
        d["stage_ns"] = {n: int(v) for n, v in zip(self.STAGES, self.stage_ns)}
        d["stage_calls"] = {n: int(v) for n, v in zip(self.STAGES, self.stage_calls)}
        d["stage_busy_ns"] = {n: int(v) for n, v in zip(self.STAGES, self.stage_busy_ns)}
        return d

_lock = threading.Lock()
_lib = None


class NativeError(RuntimeError):
    """An ``smb_*`` call returned a negative status."""

    def __init__(self, fn: str, code: int, detail: str = ""):
        self.code = code
        msg = f"{fn} failed: {strerror(code)} (code {code})"
        if detail:
            msg += f": {detail}"
        super().__init__(msg)


def load(path: str | None = None):
    """Load the library once; raises if it is absent (no fallback path exists)."""
    global _lib
    with _lock:
        if _lib is not None:
            return _lib
        # SMB_LIB: load another build of the same ABI (side-by-side comparisons)
        p = path or os.environ.get("SMB_LIB") or LIB_PATH
        if not os.path.exists(p):
            raise RuntimeError(
                f"ae_b200 CUDA library not found at {p}; build it with `python -m ae_b200.build`")
        lib = ctypes.CDLL(p)
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(lib, name)
            fn.restype = res
            fn.argtypes = args
        _lib = lib
        return lib


def exported_symbols(path: str | None = None):
    lib = load(path)
    return {name: hasattr(lib, name) for name in SIGNATURES}


def strerror(code: int) -> str:
    lib = load()
    s = lib.smb_strerror(int(code))
    return s.decode() if s else "?"


def check(fn: str, code: int):
    if code < 0:
        detail = ""
        if code == -5:  # SMB_ERR_CUDA
            d = load().smb_last_cuda_error()
            detail = d.decode() if d else ""
        raise NativeError(fn, code, detail)
    return code


def call(name: str, *args):
    lib = load()
    return check(name, getattr(lib, name)(*args))
