"""Expert-parallel MoE layer: experts sharded over the ranks of a process group, tokens
dispatched and combined with NCCL all-to-all.

The reference scales the layer by tensor parallelism only (intermediate dimension sharded,
then an all-reduce of [T, H]: ``specmoe/layers/FusedMoE.py:295-302,529-530``,
``specmoe/models/mixtral.py:113-114``); its expert-parallel flags are parsed but never
used (``specmoe/utils/server_args.py:148,202``).  Here rank r owns experts
[r*E/G, (r+1)*E/G) and its own verify tokens:

1. route the local tokens (softmax / top-k over all E experts) and gather their rows into
   the exchange layout: one chunk per destination rank, a header row with the chunk's
   per-expert counts and a fixed capacity of max_tokens * k payload rows (the worst case,
   so nothing overflows and no count has to reach the host);
2. one all-to-all moves counts and rows;
3. the local experts run on the received payload rows (expert ids come from the headers;
   rows past a chunk's counts are skipped);
4. one all-to-all returns the expert outputs;
5. the routing-weighted combine on the token's home rank reads them in place.

One process per GPU; the compute steps go through a backend object, so the exchange logic
runs the same with the CUDA library (``CudaBackend``) or with any other implementation of
the three steps.

``transport="p2p"`` moves the rows without a collective library: every rank owns an
exchange arena that its peers map through CUDA IPC (``PeerTransport``); the dispatch
kernel writes each destination's rows straight into that destination's arena over NVLink
and raises a flag there, the expert kernels wait for the flags, run the local experts and
write every row's output back into its source's arena (another flag), and the combine
waits for those.  Three library calls per layer call, no NCCL launch, graph-capturable.
"""
from __future__ import annotations

import ctypes

import torch
import torch.distributed as dist


def _ptr(t):
    return None if t is None else t.data_ptr()


class CudaBackend:
    """The three compute steps on the sm_100a library (``smb_moe_ep_dispatch``,
    ``smb_moe_ep_experts``, ``smb_moe_ep_combine`` in ``include/ae_b200.h``).  Buffers and
    workspaces are allocated on first use for each shape and reused, so a layer call can be
    captured in a CUDA graph after one warm call."""

    def __init__(self, E: int, k: int, H: int, I: int, dtype: torch.dtype, device, renormalize: bool = True):
        from . import ops
        self.E, self.k, self.H, self.I = E, k, H, I
        self.dtype = dtype
        self.code = ops.storage_code(dtype)
        self.device = torch.device(device)
        self.renormalize = renormalize
        self._bufs = {}

    def _buf(self, key, nbytes=None, shape=None, dtype=None):
        b = self._bufs.get(key)
        if b is None:
            if nbytes is not None:
                from . import ops
                b = ops.new_workspace(nbytes, self.device)
            else:
                b = torch.empty(*shape, dtype=dtype, device=self.device)
            self._bufs[key] = b
        return b

    def _stream(self):
        return torch.cuda.current_stream(self.device).cuda_stream

    def dispatch(self, x: torch.Tensor, logits: torch.Tensor, G: int, C: int, topk_weights=None, topk_ids=None):
        """Route the local tokens and gather them into the exchange layout [G*(C+1), H];
        optional routing outputs topk_weights fp32 / topk_ids int32 [T, k]."""
        from . import _native, ops
        T = x.shape[0]
        nbytes = ops.workspace_bytes(T, self.E, self.k, self.H, self.I, self.dtype)
        ws = self._buf(("ws_src", T), nbytes=nbytes)
        send = self._buf(("send", G, C), shape=(G * (C + 1), self.H), dtype=self.dtype)
        _native.call("smb_moe_ep_dispatch", logits.data_ptr(), ops.logits_code(logits.dtype), x.data_ptr(),
                     self.code, T, self.E, self.k, self.H, self.I, int(self.renormalize), G, C, send.data_ptr(),
                     _ptr(topk_weights), _ptr(topk_ids), ws.data_ptr(), ws.numel(), self._stream())
        return send, (ws, T)

    def experts(self, recv: torch.Tensor, G: int, C: int, pool: torch.Tensor, pages: torch.Tensor,
                num_local: int) -> torch.Tensor:
        """Expert output of every payload row of the received chunks, [G*C, H]."""
        from . import _native, ops
        nbytes = ops.ep_workspace_bytes(G, C, num_local, self.H, self.I, self.dtype)
        ws = self._buf(("ws_exp", G, C), nbytes=nbytes)
        out = self._buf(("y", G, C), shape=(G * C, self.H), dtype=self.dtype)
        _native.call("smb_moe_ep_experts", recv.data_ptr(), G, C, pool.data_ptr(), pool.shape[0], pages.data_ptr(),
                     self.code, num_local, self.H, self.I, out.data_ptr(), ws.data_ptr(), ws.numel(), self._stream())
        return out

    def combine(self, back: torch.Tensor, state, T: int, G: int, C: int) -> torch.Tensor:
        from . import _native
        ws, T0 = state
        out = self._buf(("out", T), shape=(T, self.H), dtype=self.dtype)
        if T > 0:
            _native.call("smb_moe_ep_combine", back.data_ptr(), out.data_ptr(), self.code, T, self.E, self.k, self.H,
                         self.I, G, C, ws.data_ptr(), ws.numel(), self._stream())
        return out


class PeerTransport:
    """This rank's exchange arena plus its peers' arenas mapped through CUDA IPC
    (``smb_ep_ipc_*`` in ``include/ae_b200.h``).  Collective: every rank of ``group``
    constructs it with the same (C, H, dtype)."""

    def __init__(self, C: int, H: int, dtype: torch.dtype, device, group=None):
        from . import _native, ops
        self.group = group
        self.G = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.C, self.H, self.code = C, H, ops.storage_code(dtype)
        self.device = torch.device(device)
        lib = _native.load()
        nbytes = int(lib.smb_ep_arena_bytes(self.G, C, H, ops.storage_code(dtype)))
        if nbytes == 0:
            raise ValueError(f"no exchange arena for G={self.G} C={C} H={H} (at most 8 ranks)")
        own = ctypes.c_void_p()
        handle = (ctypes.c_uint8 * 64)()
        with torch.cuda.device(device):
            _native.check("smb_ep_ipc_alloc", lib.smb_ep_ipc_alloc(nbytes, ctypes.byref(own), handle))
        self.own = own.value
        handles = [None] * self.G
        dist.all_gather_object(handles, bytes(handle), group=group)
        self.arenas = (ctypes.c_void_p * self.G)()
        self.opened = []
        with torch.cuda.device(device):
            for r in range(self.G):
                if r == self.rank:
                    self.arenas[r] = self.own
                    continue
                h = (ctypes.c_uint8 * 64).from_buffer_copy(handles[r])
                peer = ctypes.c_void_p()
                _native.check("smb_ep_ipc_open", lib.smb_ep_ipc_open(h, ctypes.byref(peer)))
                self.arenas[r] = peer.value
                self.opened.append(peer.value)
        self.arenas_ptr = ctypes.cast(self.arenas, ctypes.c_void_p)
        dist.barrier(group)

    def resync(self):
        """Bring every rank's exchange state back to epoch 0 (collective, between calls).

        After a call in which a wait ran out (a rank that skipped the call, or one that was
        late by more than the wait budget) the ranks' epochs disagree and every later call
        would time out too.  Each rank finishes its queued work, the ranks meet, each zeroes
        its own arena's control block and flags (``smb_ep_arena_reset``), and they meet
        again, so that no rank's next dispatch can reach a peer before that peer's reset."""
        from . import _native
        torch.cuda.synchronize(self.device)
        dist.barrier(self.group)
        with torch.cuda.device(self.device):
            _native.call("smb_ep_arena_reset", ctypes.c_void_p(self.own), self.G, self.C, self.H, self.code,
                         torch.cuda.current_stream(self.device).cuda_stream)
        torch.cuda.synchronize(self.device)
        dist.barrier(self.group)

    def close(self):
        """Unmap the peers' arenas and free this rank's (collective)."""
        from . import _native
        lib = _native.load()
        torch.cuda.synchronize()
        dist.barrier(self.group)
        for p in self.opened:
            lib.smb_ep_ipc_close(ctypes.c_void_p(p))
        self.opened = []
        dist.barrier(self.group)
        if self.own:
            lib.smb_ep_ipc_free(ctypes.c_void_p(self.own))
            self.own = None


class P2PBackend(CudaBackend):
    """The three steps over peer memory (``smb_moe_ep_*_p2p``): the exchange happens inside
    the kernels, so ``ExpertParallelMoE`` makes no collective call."""

    def __init__(self, E, k, H, I, dtype, device, transport: PeerTransport, renormalize: bool = True):
        super().__init__(E, k, H, I, dtype, device, renormalize)
        self.t = transport

    def layer(self, x, logits, G, C, pool, pages, num_local, topk_weights=None, topk_ids=None):
        from . import _native, ops
        T = x.shape[0]
        nb = ops.workspace_bytes(max(T, 1), self.E, self.k, self.H, self.I, self.dtype)
        ws = self._buf(("ws_src", T), nbytes=nb)
        nbe = ops.ep_workspace_bytes(G, C, num_local, self.H, self.I, self.dtype)
        wse = self._buf(("ws_exp", G, C), nbytes=nbe)
        out = self._buf(("out", T), shape=(T, self.H), dtype=self.dtype)
        st = self._stream()
        a = self.t.arenas_ptr
        _native.call("smb_moe_ep_dispatch_p2p", logits.data_ptr() if T else None, ops.logits_code(logits.dtype),
                     x.data_ptr() if T else None, self.code, T, self.E, self.k, self.H, self.I,
                     int(self.renormalize), G, self.t.rank, C, a, _ptr(topk_weights), _ptr(topk_ids), ws.data_ptr(),
                     ws.numel(), st)
        _native.call("smb_moe_ep_experts_p2p", G, self.t.rank, C, a, pool.data_ptr(), pool.shape[0],
                     pages.data_ptr(), self.code, num_local, self.H, self.I, wse.data_ptr(), wse.numel(), st)
        _native.call("smb_moe_ep_combine_p2p", out.data_ptr() if T else None, self.code, T, self.E, self.k,
                     self.H, self.I, G, self.t.rank, C, a, ws.data_ptr(), ws.numel(), st)
        return out


class ExpertParallelMoE:
    """MoE layer over G ranks, E/G experts each (``pool`` holds this rank's pages).

    The exchange uses fixed-capacity all-to-alls: every (source, destination) pair
    reserves ``max_tokens * top_k`` payload rows, the worst case, plus one header row of
    counts, so no count ever has to reach the host and nothing can overflow.  A layer
    call is free of host synchronisation and can be captured in a CUDA graph.

    Buffers are allocated on the first call with a given token count and kept (a captured
    graph keeps pointing at them): the returned [T, H] tensor is such a buffer and the next
    call with the same T overwrites it (clone it to keep it), and a caller that uses many
    different token counts holds one workspace per count.
    """

    def __init__(self, num_experts: int, top_k: int, hidden_size: int, intermediate_size: int,
                 pool: torch.Tensor, max_tokens: int, group=None, backend=None, renormalize: bool = True,
                 transport: str = "nccl"):
        self.group = group
        self.G = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        if num_experts % self.G:
            raise ValueError(f"{num_experts} experts do not shard over {self.G} ranks")
        self.E, self.k, self.H, self.I = num_experts, top_k, hidden_size, intermediate_size
        self.E_loc = num_experts // self.G
        self.first_expert = self.rank * self.E_loc
        if pool.shape[0] < self.E_loc or pool.shape[1] != 3 * intermediate_size * hidden_size:
            raise ValueError("pool must hold this rank's E/G expert pages [E/G, 3*I*H]")
        self.pool = pool
        self.device = pool.device
        self.pages = torch.arange(self.E_loc, dtype=torch.int64, device=pool.device)
        self.max_tokens = int(max_tokens)
        self.C = self.max_tokens * top_k  # rows reserved per (source, destination) pair
        self.transport = None
        if transport == "p2p":
            if backend is not None:
                raise ValueError("transport='p2p' runs the library's own kernels; no backend can be given")
            self.transport = PeerTransport(self.C, hidden_size, pool.dtype, pool.device, group)
            backend = P2PBackend(num_experts, top_k, hidden_size, intermediate_size, pool.dtype, pool.device,
                                 self.transport, renormalize)
        elif transport != "nccl":
            raise ValueError(f"transport must be 'nccl' or 'p2p', not {transport!r}")
        self.backend = backend or CudaBackend(num_experts, top_k, hidden_size, intermediate_size, pool.dtype,
                                              pool.device, renormalize)

    def forward(self, x: torch.Tensor, router_logits: torch.Tensor, events=None, topk_weights=None,
                topk_ids=None) -> torch.Tensor:
        """``events``: optional pair of CUDA events recorded around the local expert FFN
        (NCCL transport); ``topk_weights`` fp32 / ``topk_ids`` int32 [T, k]: optional outputs
        of the local tokens' routing."""
        T = x.shape[0]
        if T > self.max_tokens:
            raise ValueError(f"{T} tokens exceed max_tokens={self.max_tokens} of this layer")
        G, C = self.G, self.C
        if self.transport is not None:
            return self.backend.layer(x, router_logits, G, C, self.pool, self.pages, self.E_loc, topk_weights,
                                      topk_ids)
        # routing + gather into [G][1 header + C payload rows][H]; the headers carry the
        # per-expert counts, so one all-to-all moves counts and rows together
        if topk_weights is None and topk_ids is None:
            send, state = self.backend.dispatch(x, router_logits, G, C)
        else:
            send, state = self.backend.dispatch(x, router_logits, G, C, topk_weights=topk_weights, topk_ids=topk_ids)
        recv = torch.empty_like(send)
        dist.all_to_all_single(recv, send, group=self.group)
        if events is not None:
            events[0].record()
        y = self.backend.experts(recv, G, C, self.pool, self.pages, self.E_loc)
        if events is not None:
            events[1].record()
        back = torch.empty_like(y)
        dist.all_to_all_single(back, y, group=self.group)
        return self.backend.combine(back, state, T, G, C)

    __call__ = forward

    def timers(self, reset: bool = False) -> dict:
        """This rank's device-side timers (``smb_moe_read_timers``) over the calls so far:
        the local FFN kernel launches and, over peer memory, the time the FFN kernel waited
        for the sources' rows and the final combine for the returned rows."""
        from . import ops
        out = {}
        for key, buf in self.backend._bufs.items():
            if key[0] in ("ws_exp", "ws_src"):
                t = ops.read_timers(buf, reset)
                for name, v in t.items():
                    if not isinstance(v, dict):
                        out[name] = out.get(name, 0) + v
        if self.transport is not None:
            # over peer memory every kernel of a call stamps the stage clock of this rank's arena
            t = ops.read_timers_at(self.transport.own, 256, self.device, reset)
            out["stage_ns"], out["stage_calls"] = t["stage_ns"], t["stage_calls"]
            out["stage_busy_ns"] = t["stage_busy_ns"]
        return out

    def status(self) -> int:
        """Device status of this rank's last call (0, or a negative SMB_ERR_* code such as
        SMB_ERR_DEVICE_TIMEOUT when a wait for a peer ran out); synchronises."""
        from . import _native
        lib = _native.load()
        worst = 0
        st = torch.cuda.current_stream(self.device).cuda_stream
        for key, buf in self.backend._bufs.items():
            if key[0] == "ws_src":
                T = key[1]
                rc = lib.smb_moe_read_status(buf.data_ptr(), buf.numel(), T, self.E, self.k, self.H, self.I,
                                             self.backend.code, st)
            elif key[0] == "ws_exp":
                rc = lib.smb_moe_read_status(buf.data_ptr(), buf.numel(), key[1] * key[2], self.E_loc, 1, self.H,
                                             self.I, self.backend.code, st)
            else:
                continue
            if rc != 0 and worst == 0:
                worst = int(rc)
        return worst

    def resync(self):
        """Reset the peer-memory exchange of every rank to a common state after a failed
        call (collective; see ``PeerTransport.resync``).  No-op for the NCCL transport,
        whose collectives carry no state between calls."""
        if self.transport is not None:
            self.transport.resync()

    def close(self):
        """Release the exchange arenas of the p2p transport (collective)."""
        if self.transport is not None:
            self.transport.close()
            self.transport = None
