"""Expert-parallel MoE layer: experts sharded over the ranks of a process group, tokens
dispatched and combined with NCCL all-to-all.

The reference scales the layer by tensor parallelism only (intermediate dimension sharded,
then an all-reduce of [T, H]: ``specmoe/layers/FusedMoE.py:295-302,529-530``,
``specmoe/models/mixtral.py:113-114``); its expert-parallel flags are parsed but never
used (``specmoe/utils/server_args.py:148,202``).  Here rank r owns experts
[r*E/G, (r+1)*E/G) and its own verify tokens:

1. route the local tokens (softmax / top-k over all E experts).  The permuted rows are
   expert-major, and experts are contiguous per rank, so they are already grouped by
   destination rank;
2. all-to-all of the per-expert counts (E/G per destination), then one copy of the split
   sizes to the host (the only synchronisation of a layer call);
3. all-to-all of the token rows;
4. the local experts on the received rows: the same kernels as the single-GPU layer, as a
   routed problem with k = 1 (each received row has one local expert, weight 1), so each
   row's expert output comes back in received order;
5. the reverse all-to-all of those rows;
6. the routing-weighted combine on the token's home rank.

One process per GPU; the compute steps go through a backend object, so the exchange logic
runs the same with the CUDA library (``CudaBackend``) or with any other implementation of
the three steps.
"""
from __future__ import annotations

import torch
import torch.distributed as dist


class CudaBackend:
    """The three compute steps on the sm_100a library (``include/ae_b200.h``)."""

    def __init__(self, E: int, k: int, H: int, I: int, dtype: torch.dtype, device, renormalize: bool = True):
        self.E, self.k, self.H, self.I = E, k, H, I
        self.dtype = dtype
        self.device = torch.device(device)
        self.renormalize = renormalize
        self._layers = {}

    def _layer(self, T):
        from .ops import StagedLayer
        L = self._layers.get(T)
        if L is None:
            L = StagedLayer(T, self.E, self.k, self.H, self.I, self.dtype, self.device)
            self._layers[T] = L
        return L

    def route(self, x: torch.Tensor, logits: torch.Tensor):
        """Returns (rows [T*k, H] expert-major, counts [E] int32, state)."""
        T = x.shape[0]
        L = self._layer(T)
        L.route(logits, x, self.renormalize)
        v = L.views()
        off = v["expert_off"]
        counts = (off[1:] - off[:-1]).to(torch.int32)
        return v["xp"][: T * self.k], counts, L

    def experts(self, rows: torch.Tensor, local_ids: torch.Tensor, pool: torch.Tensor,
                pages: torch.Tensor, num_local: int) -> torch.Tensor:
        """Expert output of each received row (weight 1), in received order."""
        from . import ops
        N = rows.shape[0]
        out = torch.empty_like(rows)
        if N == 0:
            return out
        w = torch.ones(N, 1, dtype=torch.float32, device=rows.device)
        return ops.moe_forward_routed(rows, w, local_ids.view(N, 1), pool, pages, num_local, out=out)

    def combine(self, rows_back: torch.Tensor, state, T: int) -> torch.Tensor:
        out = torch.empty(T, self.H, dtype=self.dtype, device=self.device)
        if T > 0:
            state.combine_rows(rows_back, out)
        return out


class ExpertParallelMoE:
    """MoE layer over G ranks, E/G experts each (``pool`` holds this rank's pages)."""

    def __init__(self, num_experts: int, top_k: int, hidden_size: int, intermediate_size: int,
                 pool: torch.Tensor, group=None, backend=None, renormalize: bool = True):
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
        self.pages = torch.arange(self.E_loc, dtype=torch.int64, device=pool.device)
        self.backend = backend or CudaBackend(num_experts, top_k, hidden_size, intermediate_size, pool.dtype,
                                              pool.device, renormalize)

    def split_sizes(self, counts: torch.Tensor):
        """All-to-all of per-expert counts; returns (send_splits, recv_splits, recv_counts)
        with the split lists on the host."""
        recv_counts = torch.empty(self.G * self.E_loc, dtype=torch.int32, device=counts.device)
        dist.all_to_all_single(recv_counts, counts.contiguous(), group=self.group)
        both = torch.cat([counts, recv_counts]).cpu()
        send = both[: self.E].view(self.G, self.E_loc).sum(1).tolist()
        recv = both[self.E:].view(self.G, self.E_loc).sum(1).tolist()
        return [int(s) for s in send], [int(r) for r in recv], recv_counts

    def forward(self, x: torch.Tensor, router_logits: torch.Tensor) -> torch.Tensor:
        T = x.shape[0]
        rows, counts, state = self.backend.route(x, router_logits)
        send, recv, recv_counts = self.split_sizes(counts)
        N = sum(recv)
        recv_rows = torch.empty(N, self.H, dtype=rows.dtype, device=rows.device)
        dist.all_to_all_single(recv_rows, rows.contiguous(), recv, send, group=self.group)
        # local expert of each received row: per source, E/G runs of recv_counts rows
        local_ids = torch.repeat_interleave(
            torch.arange(self.E_loc, dtype=torch.int32, device=rows.device).repeat(self.G),
            recv_counts.to(torch.int64), output_size=N)
        y = self.backend.experts(recv_rows, local_ids, self.pool, self.pages, self.E_loc)
        back = torch.empty(T * self.k, self.H, dtype=rows.dtype, device=rows.device)
        dist.all_to_all_single(back, y.contiguous(), send, recv, group=self.group)
        return self.backend.combine(back, state, T)

    __call__ = forward
