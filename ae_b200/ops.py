"""Torch-tensor wrappers around the C ABI (``include/ae_b200.h``).

These functions take CUDA tensors, check them, find a workspace and call the library on
the current CUDA stream.  They never compute anything on the host: the library is the
only implementation, and a missing library or a non-B200 device raises.
"""
from __future__ import annotations

import os
import threading

import torch

from . import _native
from ._native import DTYPE_BF16, DTYPE_F16, DTYPE_F32

_STORAGE = {torch.float16: DTYPE_F16, torch.bfloat16: DTYPE_BF16}
_LOGITS = {torch.float16: DTYPE_F16, torch.bfloat16: DTYPE_BF16, torch.float32: DTYPE_F32}

DEBUG = os.environ.get("SMB_DEBUG", "0") == "1"


def storage_code(dtype: torch.dtype) -> int:
    try:
        return _STORAGE[dtype]
    except KeyError:
        raise NotImplementedError(f"storage dtype {dtype} (supported: float16, bfloat16)") from None


def logits_code(dtype: torch.dtype) -> int:
    try:
        return _LOGITS[dtype]
    except KeyError:
        raise NotImplementedError(f"router logits dtype {dtype}") from None


def _ptr(t: torch.Tensor | None):
    return None if t is None else t.data_ptr()


def _stream_ptr(device: torch.device):
    return torch.cuda.current_stream(device).cuda_stream


def _need_cuda(name: str, t: torch.Tensor):
    if not t.is_cuda:
        raise ValueError(f"{name} must be a CUDA tensor (no host path exists)")
    if not t.is_contiguous():
        raise ValueError(f"{name} must be contiguous")


class Workspace:
    """Per (device, stream) scratch buffer, grown on demand and reused across calls."""

    _lock = threading.Lock()
    _bufs: dict = {}

    @classmethod
    def get(cls, device: torch.device, nbytes: int) -> torch.Tensor:
        device = torch.device(device)
        if device.index is None:
            device = torch.device("cuda", torch.cuda.current_device())
        key = (device.index, torch.cuda.current_stream(device).cuda_stream)
        with cls._lock:
            buf = cls._bufs.get(key)
            if buf is None or buf.numel() < nbytes:
                buf = new_workspace(max(nbytes, 1 << 20), device)
                cls._bufs[key] = buf
            return buf

    @classmethod
    def lookup(cls, device: torch.device, stream=None) -> torch.Tensor | None:
        """The buffer that calls on ``stream`` (default: the current stream) of ``device``
        use, or None before the first call there."""
        device = torch.device(device)
        if device.index is None:
            device = torch.device("cuda", torch.cuda.current_device())
        s = stream if stream is not None else torch.cuda.current_stream(device)
        with cls._lock:
            return cls._bufs.get((device.index, s.cuda_stream))

    @classmethod
    def clear(cls):
        with cls._lock:
            cls._bufs.clear()


def new_workspace(nbytes: int, device) -> torch.Tensor:
    """A workspace buffer with its control block initialised (``smb_moe_workspace_init``)."""
    buf = torch.empty(max(int(nbytes), 256), dtype=torch.uint8, device=device)
    _native.call("smb_moe_workspace_init", buf.data_ptr(), buf.numel(), _stream_ptr(buf.device))
    return buf


def workspace_bytes(T: int, E: int, k: int, H: int, I: int, dtype: torch.dtype) -> int:
    n = _native.load().smb_moe_workspace_bytes(T, E, k, H, I, storage_code(dtype))
    if n == 0:
        raise NotImplementedError(
            f"unsupported MoE sizes T={T} E={E} k={k} H={H} I={I} dtype={dtype}: "
            + _native.strerror(-1))
    return int(n)


def splits(E: int, H: int, I: int, Tk: int) -> int:
    return _native.call("smb_moe_splits", E, H, I, Tk)


def ep_workspace_bytes(G: int, C: int, E_loc: int, H: int, I: int, dtype: torch.dtype) -> int:
    """Workspace of the expert side of a G-rank exchange with C slots per pair
    (``smb_moe_ep_workspace_bytes``)."""
    n = _native.load().smb_moe_ep_workspace_bytes(G, C, E_loc, H, I, storage_code(dtype))
    if n == 0:
        raise NotImplementedError(f"unsupported expert-parallel sizes G={G} C={C} E_loc={E_loc} H={H} I={I}")
    return int(n)


def pool_geometry(pool: torch.Tensor, H: int):
    """(num_pages, I) of a page pool [P, 3*I*H]."""
    if pool.dim() != 2:
        raise ValueError("expert pool must be [num_pages, 3*I*H]")
    P, page = pool.shape
    if page % (3 * H):
        raise ValueError(f"page size {page} is not 3*I*H for H={H}")
    return P, page // (3 * H)


def read_timers(ws: torch.Tensor, reset: bool = False) -> dict:
    """Device-side kernel timers accumulated in workspace ``ws`` (``smb_moe_read_timers``):
    ``ffn_ns`` / ``ffn_launches`` (FFN kernel launches, first CTA past its wait on the
    router to the last CTA done), the flag-wait times of the expert-parallel exchange and
    the per-stage times of the calls (``stage_ns`` / ``stage_calls``).  Synchronises the
    current stream; ``reset`` then zeroes them, stream-ordered."""
    return read_timers_at(ws.data_ptr(), ws.numel(), ws.device, reset)


def read_timers_at(ptr: int, nbytes: int, device, reset: bool = False) -> dict:
    """``read_timers`` on a raw control block (a workspace, or an exchange arena)."""
    import ctypes
    t = _native.Timers()
    _native.call("smb_moe_read_timers", ptr, nbytes, int(bool(reset)), ctypes.byref(t),
                 _stream_ptr(torch.device(device)))
    return t.as_dict()


def _status(ws: torch.Tensor, T, E, k, H, I, code, stream) -> int:
    """Device status of the last call on ``ws`` (0 or a negative SMB_ERR_* code); syncs."""
    return int(_native.load().smb_moe_read_status(ws.data_ptr(), ws.numel(), T, E, k, H, I, code, stream))


def moe_forward(x: torch.Tensor, router_logits: torch.Tensor, pool: torch.Tensor,
                page_of_expert: torch.Tensor, top_k: int, renormalize: bool = True,
                out: torch.Tensor | None = None, topk_weights: torch.Tensor | None = None,
                topk_ids: torch.Tensor | None = None) -> torch.Tensor:
    """Whole MoE layer on the GPU: route, gate/up GEMM + SiLU*mul, down GEMM, combine.

    ``out`` may be ``x`` (in-place, as the reference does).  Returns ``out``.
    """
    for n, t in (("hidden_states", x), ("router_logits", router_logits), ("expert pool", pool),
                 ("expert_cache_indices", page_of_expert)):
        _need_cuda(n, t)
    T, H = x.shape
    E = router_logits.shape[1]
    if router_logits.shape[0] != T:
        raise ValueError("Number of tokens mismatch")
    if page_of_expert.dtype != torch.int64 or page_of_expert.numel() != E:
        raise ValueError("expert_cache_indices must be int64 [E]")
    if pool.dtype != x.dtype:
        raise ValueError("expert pool and hidden_states dtypes differ")
    P, I = pool_geometry(pool, H)
    code = storage_code(x.dtype)
    if out is None:
        out = torch.empty_like(x)
    nbytes = workspace_bytes(T, E, top_k, H, I, x.dtype)
    ws = Workspace.get(x.device, nbytes)
    stream = _stream_ptr(x.device)
    _native.call("smb_moe_forward", x.data_ptr(), router_logits.data_ptr(), logits_code(router_logits.dtype),
                 pool.data_ptr(), P, page_of_expert.data_ptr(), code, T, E, top_k, H, I, int(bool(renormalize)),
                 out.data_ptr(), _ptr(topk_weights), _ptr(topk_ids), ws.data_ptr(), ws.numel(), stream)
    if DEBUG:
        _native.check("smb_moe_forward (device status)", _status(ws, T, E, top_k, H, I, code, stream))
    return out


def shared_expert_pages(w1: torch.Tensor, w3: torch.Tensor, w2: torch.Tensor, I: int) -> torch.Tensor:
    """A shared expert (w1, w3 [I_s, H], w2 [H, I_s]) as ceil(I_s / I) pages of the routed
    experts' page layout [w1 | w3 | w2] with intermediate size I: page q holds rows
    [q*I, (q+1)*I) of w1 / w3 and those columns of w2, zero-padded past I_s.  Returns
    [n_shared, 3*I*H] on the device of w1 (a load-time repacking, like weight_loader)."""
    Is, H = w1.shape
    if w3.shape != (Is, H) or w2.shape != (H, Is):
        raise ValueError("shared expert weights must be w1, w3 [I_s, H] and w2 [H, I_s]")
    n = -(-Is // I)
    pages = torch.zeros(n, 3 * I * H, dtype=w1.dtype, device=w1.device)
    for q in range(n):
        r0, r1 = q * I, min(Is, (q + 1) * I)
        p = pages[q]
        p[: I * H].view(I, H)[: r1 - r0] = w1[r0:r1]
        p[I * H: 2 * I * H].view(I, H)[: r1 - r0] = w3[r0:r1]
        p[2 * I * H:].view(H, I)[:, : r1 - r0] = w2[:, r0:r1]
    return pages


def moe_forward_shared(x: torch.Tensor, router_logits: torch.Tensor, pool: torch.Tensor,
                       page_of_expert: torch.Tensor, top_k: int, n_shared: int,
                       shared_weight: torch.Tensor | None = None, renormalize: bool = True,
                       out: torch.Tensor | None = None, topk_weights: torch.Tensor | None = None,
                       topk_ids: torch.Tensor | None = None) -> torch.Tensor:
    """Routed top-k experts plus a shared expert (``n_shared`` pseudo-expert pages from
    :func:`shared_expert_pages`, at ``page_of_expert[E:]``), scaled per token by
    ``shared_weight`` fp32 [T] (None: 1).  ``router_logits`` [T, E] cover the routed experts."""
    for n, t in (("hidden_states", x), ("router_logits", router_logits), ("expert pool", pool),
                 ("page_of_expert", page_of_expert)):
        _need_cuda(n, t)
    T, H = x.shape
    E = router_logits.shape[1]
    if router_logits.shape[0] != T:
        raise ValueError("Number of tokens mismatch")
    if page_of_expert.dtype != torch.int64 or page_of_expert.numel() != E + n_shared:
        raise ValueError("page_of_expert must be int64 [E + n_shared]")
    if shared_weight is not None:
        _need_cuda("shared_weight", shared_weight)
        if shared_weight.dtype != torch.float32 or shared_weight.numel() != T:
            raise ValueError("shared_weight must be float32 [T]")
    if pool.dtype != x.dtype:
        raise ValueError("expert pool and hidden_states dtypes differ")
    P, I = pool_geometry(pool, H)
    code = storage_code(x.dtype)
    if out is None:
        out = torch.empty_like(x)
    nbytes = workspace_bytes(T, E + n_shared, top_k + n_shared, H, I, x.dtype)
    ws = Workspace.get(x.device, nbytes)
    stream = _stream_ptr(x.device)
    _native.call("smb_moe_forward_shared", x.data_ptr(), router_logits.data_ptr(), logits_code(router_logits.dtype),
                 _ptr(shared_weight), pool.data_ptr(), P, page_of_expert.data_ptr(), code, T, E, top_k, n_shared,
                 H, I, int(bool(renormalize)), out.data_ptr(), _ptr(topk_weights), _ptr(topk_ids), ws.data_ptr(),
                 ws.numel(), stream)
    if DEBUG:
        _native.check("smb_moe_forward_shared (device status)",
                      _status(ws, T, E + n_shared, top_k + n_shared, H, I, code, stream))
    return out


def moe_forward_routed(x: torch.Tensor, topk_weights: torch.Tensor, topk_ids: torch.Tensor,
                       pool: torch.Tensor, page_of_expert: torch.Tensor, num_experts: int,
                       out: torch.Tensor | None = None) -> torch.Tensor:
    """MoE layer from a given routing (``stack_fused_moe``)."""
    for n, t in (("hidden_states", x), ("topk_weights", topk_weights), ("topk_ids", topk_ids),
                 ("expert pool", pool), ("indicies", page_of_expert)):
        _need_cuda(n, t)
    if topk_weights.dtype != torch.float32 or topk_ids.dtype != torch.int32:
        raise ValueError("topk_weights must be float32 and topk_ids int32")
    T, H = x.shape
    k = topk_ids.shape[1]
    E = int(num_experts)
    if page_of_expert.dtype != torch.int64 or page_of_expert.numel() < E:
        raise ValueError("indicies must be int64 [E]")
    P, I = pool_geometry(pool, H)
    code = storage_code(x.dtype)
    if out is None:
        out = torch.empty_like(x)
    nbytes = workspace_bytes(T, E, k, H, I, x.dtype)
    ws = Workspace.get(x.device, nbytes)
    stream = _stream_ptr(x.device)
    _native.call("smb_moe_forward_routed", x.data_ptr(), topk_weights.data_ptr(), topk_ids.data_ptr(),
                 pool.data_ptr(), P, page_of_expert.data_ptr(), code, T, E, k, H, I, out.data_ptr(),
                 ws.data_ptr(), ws.numel(), stream)
    if DEBUG:
        _native.check("smb_moe_forward_routed (device status)", _status(ws, T, E, k, H, I, code, stream))
    return out


def gate(x: torch.Tensor, gate_weight: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
    """Router logits [T, E] = x [T, H] @ gate_weight [E, H]^T in the storage dtype
    (``MixtralMoE.gate``, specmoe/models/mixtral.py:85-92)."""
    _need_cuda("hidden_states", x)
    _need_cuda("gate weight", gate_weight)
    T, H = x.shape
    E = gate_weight.shape[0]
    if gate_weight.shape[1] != H or gate_weight.dtype != x.dtype:
        raise ValueError("gate weight must be [E, H] in the dtype of hidden_states")
    if out is None:
        out = torch.empty(T, E, dtype=x.dtype, device=x.device)
    _native.call("smb_moe_gate", x.data_ptr(), gate_weight.data_ptr(), storage_code(x.dtype), T, E, H,
                 out.data_ptr(), _stream_ptr(x.device))
    return out


def moe_forward_gated(x: torch.Tensor, gate_weight: torch.Tensor, pool: torch.Tensor,
                      page_of_expert: torch.Tensor, top_k: int, renormalize: bool = True,
                      out: torch.Tensor | None = None, router_logits: torch.Tensor | None = None,
                      topk_weights: torch.Tensor | None = None,
                      topk_ids: torch.Tensor | None = None) -> torch.Tensor:
    """MixtralMoE block (gate + experts, specmoe/models/mixtral.py:106-115 without the
    TP all-reduce): the gate GEMV and the routing in one launch, then FFN and combine.
    ``out`` may be ``x``.  Optional outputs: ``router_logits`` [T, E] (storage dtype),
    ``topk_weights`` fp32 / ``topk_ids`` int32 [T, k]."""
    for n, t in (("hidden_states", x), ("gate weight", gate_weight), ("expert pool", pool),
                 ("expert_cache_indices", page_of_expert)):
        _need_cuda(n, t)
    T, H = x.shape
    E = gate_weight.shape[0]
    if gate_weight.shape[1] != H or gate_weight.dtype != x.dtype:
        raise ValueError("gate weight must be [E, H] in the dtype of hidden_states")
    if page_of_expert.dtype != torch.int64 or page_of_expert.numel() != E:
        raise ValueError("expert_cache_indices must be int64 [E]")
    if pool.dtype != x.dtype:
        raise ValueError("expert pool and hidden_states dtypes differ")
    P, I = pool_geometry(pool, H)
    code = storage_code(x.dtype)
    if out is None:
        out = torch.empty_like(x)
    nbytes = workspace_bytes(T, E, top_k, H, I, x.dtype)
    ws = Workspace.get(x.device, nbytes)
    stream = _stream_ptr(x.device)
    _native.call("smb_moe_forward_gated", x.data_ptr(), gate_weight.data_ptr(), pool.data_ptr(), P,
                 page_of_expert.data_ptr(), code, T, E, top_k, H, I, int(bool(renormalize)), out.data_ptr(),
                 _ptr(router_logits), _ptr(topk_weights), _ptr(topk_ids), ws.data_ptr(), ws.numel(), stream)
    if DEBUG:
        _native.check("smb_moe_forward_gated (device status)", _status(ws, T, E, top_k, H, I, code, stream))
    return out


def topk(router_logits: torch.Tensor, top_k: int, renormalize: bool = True):
    """(topk_weights fp32 [T,k], topk_ids int32 [T,k]) on the GPU."""
    _need_cuda("router_logits", router_logits)
    T, E = router_logits.shape
    w = torch.empty(T, top_k, dtype=torch.float32, device=router_logits.device)
    ids = torch.empty(T, top_k, dtype=torch.int32, device=router_logits.device)
    _native.call("smb_moe_topk", router_logits.data_ptr(), logits_code(router_logits.dtype), T, E, top_k,
                 int(bool(renormalize)), w.data_ptr(), ids.data_ptr(), _stream_ptr(router_logits.device))
    return w, ids


def align_block_size(topk_ids: torch.Tensor, block_size: int, num_experts: int):
    """(sorted_ids, expert_ids, num_tokens_post_pad) of moe_align_block_size."""
    _need_cuda("topk_ids", topk_ids)
    ids = topk_ids if topk_ids.dtype == torch.int32 else topk_ids.to(torch.int32)
    numel = ids.numel()
    max_padded = numel + num_experts * (block_size - 1)
    dev = ids.device
    sorted_ids = torch.empty(max_padded, dtype=torch.int32, device=dev)
    n_blocks = -(-max_padded // block_size)
    expert_ids = torch.empty(n_blocks, dtype=torch.int32, device=dev)
    npost = torch.empty(1, dtype=torch.int32, device=dev)
    _native.call("smb_moe_align_block_size", ids.data_ptr(), numel, num_experts, block_size,
                 sorted_ids.data_ptr(), expert_ids.data_ptr(), npost.data_ptr(), _stream_ptr(dev))
    return sorted_ids, expert_ids, npost


class StagedLayer:
    """The four stages as separate calls on one workspace (tests and profiling)."""

    def __init__(self, T, E, k, H, I, dtype, device):
        self.T, self.E, self.k, self.H, self.I = T, E, k, H, I
        self.dtype = dtype
        self.code = storage_code(dtype)
        self.nbytes = workspace_bytes(T, E, k, H, I, dtype)
        self.ws = new_workspace(self.nbytes, device)
        self.device = torch.device(device)

    def _s(self):
        return _stream_ptr(self.device)

    def route(self, router_logits, x, renormalize=True, topk_weights=None, topk_ids=None):
        _native.call("smb_moe_route", router_logits.data_ptr(), logits_code(router_logits.dtype), x.data_ptr(),
                     self.code, self.T, self.E, self.k, self.H, self.I, int(bool(renormalize)),
                     _ptr(topk_weights), _ptr(topk_ids), self.ws.data_ptr(), self.nbytes, self._s())

    def permute(self, topk_weights, topk_ids, x):
        _native.call("smb_moe_permute", topk_weights.data_ptr(), topk_ids.data_ptr(), x.data_ptr(), self.code,
                     self.T, self.E, self.k, self.H, self.I, self.ws.data_ptr(), self.nbytes, self._s())

    def ffn(self, pool, page_of_expert, x):
        _native.call("smb_moe_ffn", x.data_ptr(), pool.data_ptr(), pool.shape[0], page_of_expert.data_ptr(), self.code,
                     self.T, self.E, self.k, self.H, self.I, self.ws.data_ptr(), self.nbytes, self._s())

    def gate_up(self, pool, page_of_expert, x):
        _native.call("smb_moe_gate_up", x.data_ptr(), pool.data_ptr(), pool.shape[0], page_of_expert.data_ptr(), self.code,
                     self.T, self.E, self.k, self.H, self.I, self.ws.data_ptr(), self.nbytes, self._s())

    def down(self, pool, page_of_expert):
        _native.call("smb_moe_down", pool.data_ptr(), pool.shape[0], page_of_expert.data_ptr(), self.code,
                     self.T, self.E, self.k, self.H, self.I, self.ws.data_ptr(), self.nbytes, self._s())

    def combine(self, out):
        _native.call("smb_moe_combine", out.data_ptr(), self.code, self.T, self.E, self.k, self.H, self.I,
                     self.ws.data_ptr(), self.nbytes, self._s())

    def combine_rows(self, rows, out):
        _native.call("smb_moe_combine_rows", rows.data_ptr(), out.data_ptr(), self.code, self.T, self.E, self.k,
                     self.H, self.I, self.ws.data_ptr(), self.nbytes, self._s())

    def status(self):
        return _status(self.ws, self.T, self.E, self.k, self.H, self.I, self.code, self._s())

    # views of the workspace, following WsLayout in csrc/layout.h
    def views(self):
        Tk = self.T * self.k
        E, H, I = self.E, self.H, self.I
        A = 256

        def up(v):
            return (v + A - 1) // A * A

        rows = up_to(Tk, 64) + 64
        S = splits(E, H, I, Tk)
        ntc = -(-Tk // 256) if Tk > 256 else 1
        ndone = 2 + E * (S + -(-H // 256)) * ntc
        o = 0
        off = {}
        # mirrors ae_b200/csrc/layout.h::make_ws_layout (checked against its total below)
        for name, nb in (("status", 4 * 64), ("expert_off", 4 * (E + 1)), ("done", 4 * ndone),
                         ("perm", 4 * Tk), ("inv", 4 * Tk), ("w", 4 * Tk), ("ids", 4 * Tk),
                         ("logits", 4 * self.T * E), ("xp", 2 * rows * H), ("a2", 2 * rows * I),
                         ("part", 4 * S * Tk * H)):
            off[name] = (o, nb)
            o = up(o + nb)
        if o != self.nbytes:
            raise RuntimeError(f"workspace layout mirror out of date ({o} != {self.nbytes} bytes)")
        ws = self.ws

        def view(name, dtype, shape):
            o, nb = off[name]
            return ws[o:o + nb].view(dtype).view(*shape)

        return {
            "expert_off": view("expert_off", torch.int32, (E + 1,)),
            "status": view("status", torch.int32, (64,)),
            "done": view("done", torch.int32, (ndone,)),
            "perm": view("perm", torch.int32, (Tk,)),
            "inv": view("inv", torch.int32, (Tk,)),
            "w": view("w", torch.float32, (Tk,)),
            "ids": view("ids", torch.int32, (Tk,)),
            "logits": view("logits", torch.float32, (self.T, E)),
            "xp": view("xp", self.dtype, (rows, H)),
            "a2": view("a2", self.dtype, (rows, I)),
            "part": view("part", torch.float32, (S, Tk, H)),
        }


def up_to(v: int, a: int) -> int:
    return (v + a - 1) // a * a
