"""Expert pages streamed from host memory into the GPU page pool while the layer runs.

The reference keeps every expert in page-locked host memory (``FusedMoE.ws``, pinned when
``pin_experts_when_load_weight``, ``specmoe/layers/FusedMoE.py:68-97``) and copies the
pages a layer needs into its GPU expert cache before the layer runs
(``HtoDTransferEngine`` / ``StreamPriorityEngine.decode_load_weight``,
``specmoe/backend/htod_transfer_engine.py:260-341``, ``specmoe/engine.py:143-154,549-588``;
with ``decode_weight_cache_ratio=0`` every layer's experts cross PCIe).  Here the copies and
the layer overlap: each page's copy (one ``cudaMemcpyAsync`` on a copy stream) is followed
by a stream-ordered write of an epoch number into that page's ready flag, and the FFN
kernel of ``smb_moe_forward_streamed`` starts at once and waits, per unit of work, for the
flag of the page it is about to read, so the first experts are computed while the others
are still in flight.
"""
from __future__ import annotations

import torch

from . import _native, ops


class ExpertPageStreamer:
    """A GPU page pool fed from page-locked host expert pages.

    ``host_pages``: [E, 3*I*H] in page-locked host memory (page layout of
    ``FusedMoE.weight_loader``).  ``num_pages``: pages of the GPU pool (>= the experts one
    layer call uses)."""

    def __init__(self, host_pages: torch.Tensor, num_pages: int, device, copy_stream=None):
        if host_pages.is_cuda or not host_pages.is_pinned():
            raise ValueError("host expert pages must be in page-locked host memory (pin_memory=True)")
        if host_pages.dim() != 2 or not host_pages.is_contiguous():
            raise ValueError("host expert pages must be a contiguous [E, 3*I*H] tensor")
        self.device = torch.device(device)
        if self.device.type == "cuda" and self.device.index is None:
            self.device = torch.device("cuda", torch.cuda.current_device())
        self.host = host_pages
        self.page_bytes = host_pages.shape[1] * host_pages.element_size()
        self.pool = torch.empty(num_pages, host_pages.shape[1], dtype=host_pages.dtype, device=self.device)
        self.ready = torch.zeros(num_pages, dtype=torch.int32, device=self.device)
        self.epoch = 0
        self.stream = copy_stream or torch.cuda.Stream(self.device)

    def load(self, experts, pages=None) -> int:
        """Queue the copies of ``experts`` (host page indices) into ``pages`` of the pool
        (default 0, 1, ...).  Returns the epoch that marks them ready.  The copies start
        after the work already queued on the current stream (which may still read the
        pool)."""
        experts = [int(e) for e in experts]
        pages = list(range(len(experts))) if pages is None else [int(p) for p in pages]
        if len(pages) != len(experts):
            raise ValueError("one pool page per expert")
        if any(p < 0 or p >= self.pool.shape[0] for p in pages):
            raise ValueError("page index outside the pool")
        if any(e < 0 or e >= self.host.shape[0] for e in experts):
            raise ValueError("expert index outside the host store")
        self.epoch += 1
        self.stream.wait_stream(torch.cuda.current_stream(self.device))
        st = self.stream.cuda_stream
        for e, p in zip(experts, pages):
            _native.call("smb_moe_page_copy", self.pool[p].data_ptr(), self.host[e].data_ptr(), self.page_bytes,
                         self.ready[p:p + 1].data_ptr(), self.epoch, st)
        return self.epoch

    def forward(self, x: torch.Tensor, router_logits: torch.Tensor, top_k: int, page_of_expert: torch.Tensor,
                epoch: int | None = None, renormalize: bool = True, out: torch.Tensor | None = None) -> torch.Tensor:
        """The layer on the current stream, reading each expert's page once its copy of
        ``epoch`` (default: the last ``load``) has landed."""
        for n, t in (("hidden_states", x), ("router_logits", router_logits), ("page_of_expert", page_of_expert)):
            ops._need_cuda(n, t)
        T, H = x.shape
        E = router_logits.shape[1]
        if page_of_expert.dtype != torch.int64 or page_of_expert.numel() != E:
            raise ValueError("page_of_expert must be int64 [E]")
        P, I = ops.pool_geometry(self.pool, H)
        code = ops.storage_code(x.dtype)
        if out is None:
            out = torch.empty_like(x)
        nbytes = ops.workspace_bytes(T, E, top_k, H, I, x.dtype)
        ws = ops.Workspace.get(x.device, nbytes)
        stream = torch.cuda.current_stream(x.device).cuda_stream
        _native.call("smb_moe_forward_streamed", x.data_ptr(), router_logits.data_ptr(),
                     ops.logits_code(router_logits.dtype), self.pool.data_ptr(), P, page_of_expert.data_ptr(),
                     self.ready.data_ptr(), self.epoch if epoch is None else int(epoch), code, T, E, top_k, H, I,
                     int(bool(renormalize)), out.data_ptr(), None, None, ws.data_ptr(), ws.numel(), stream)
        if ops.DEBUG:
            _native.check("smb_moe_forward_streamed (device status)",
                          ops._status(ws, T, E, top_k, H, I, code, stream))
        return out

    def status(self, x: torch.Tensor, E: int, top_k: int) -> int:
        """Device status of the last ``forward`` with inputs shaped like ``x`` (0 or a
        negative SMB_ERR_* code; syncs)."""
        T, H = x.shape
        _, I = ops.pool_geometry(self.pool, H)
        nbytes = ops.workspace_bytes(T, E, top_k, H, I, x.dtype)
        ws = ops.Workspace.get(self.device, nbytes)
        return ops._status(ws, T, E, top_k, H, I, ops.storage_code(x.dtype),
                           torch.cuda.current_stream(self.device).cuda_stream)
