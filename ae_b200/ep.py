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
2. all-to-all of the per-expert counts and of the token rows, each (source, destination)
   pair with a fixed capacity of max_tokens * k rows (the worst case), so the split sizes
   never have to reach the host;
3. the local experts on the received rows: the same kernels as the single-GPU layer, as a
   routed problem with k = 1 (each received row has one local expert and weight 1; the
   unused capacity rows carry expert -1 and are skipped);
4. the reverse all-to-all of the expert outputs;
5. the routing-weighted combine on the token's home rank.

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
    """MoE layer over G ranks, E/G experts each (``pool`` holds this rank's pages).

    The exchange uses fixed-capacity all-to-alls: every (source, destination) pair
    reserves ``max_tokens * top_k`` rows, the worst case, so no count ever has to reach
    the host and nothing can overflow; the unused rows of a pair carry expert id -1 and
    are skipped by the kernels.  A layer call is therefore free of host synchronisation
    and can be captured in a CUDA graph.
    """

    def __init__(self, num_experts: int, top_k: int, hidden_size: int, intermediate_size: int,
                 pool: torch.Tensor, max_tokens: int, group=None, backend=None, renormalize: bool = True):
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
        self.backend = backend or CudaBackend(num_experts, top_k, hidden_size, intermediate_size, pool.dtype,
                                              pool.device, renormalize)
        self._slot = torch.arange(self.C, device=pool.device)

    def forward(self, x: torch.Tensor, router_logits: torch.Tensor, events=None) -> torch.Tensor:
        """``events``: optional pair of CUDA events recorded around the local expert FFN."""
        T = x.shape[0]
        if T > self.max_tokens:
            raise ValueError(f"{T} tokens exceed max_tokens={self.max_tokens} of this layer")
        G, E_loc, C, H = self.G, self.E_loc, self.C, self.H
        Tk = T * self.k
        rows, counts, state = self.backend.route(x, router_logits)
        # rows are expert-major, hence destination-major: destination d owns rows
        # [off[d], off[d] + n[d])
        n_dst = counts.view(G, E_loc).sum(1)
        end_dst = torch.cumsum(n_dst, 0)
        off_dst = end_dst - n_dst
        if Tk > 0:
            idx = (off_dst.unsqueeze(1) + self._slot.unsqueeze(0)).clamp_(max=Tk - 1).reshape(-1)
            send = rows.index_select(0, idx)
        else:
            send = torch.zeros(G * C, H, dtype=x.dtype, device=x.device)
        recv_counts = torch.empty(G * E_loc, dtype=torch.int32, device=x.device)
        dist.all_to_all_single(recv_counts, counts.to(torch.int32).contiguous(), group=self.group)
        recv = torch.empty(G * C, H, dtype=x.dtype, device=x.device)
        dist.all_to_all_single(recv, send, group=self.group)
        # local expert of received row i of source s: the run of recv_counts[s] holding
        # i, or -1 past the rows that source actually sent
        cum = torch.cumsum(recv_counts.view(G, E_loc).to(torch.int64), 1)
        slots = self._slot.unsqueeze(0).expand(G, C).contiguous()
        ids = torch.searchsorted(cum, slots, right=True)
        ids = torch.where(slots < cum[:, -1:], ids, torch.full_like(ids, -1)).to(torch.int32).reshape(-1)
        if events is not None:
            events[0].record()
        y = self.backend.experts(recv, ids, self.pool, self.pages, E_loc)
        if events is not None:
            events[1].record()
        back = torch.empty(G * C, H, dtype=x.dtype, device=x.device)
        dist.all_to_all_single(back, y.contiguous(), group=self.group)
        if Tk == 0:
            return self.backend.combine(back[:0], state, T)
        # back row of permuted position p: destination d holding p, slot p - off[d]
        pos = torch.arange(Tk, device=x.device)
        d = torch.searchsorted(end_dst, pos, right=True)
        back_rows = back.index_select(0, d * C + pos - off_dst[d])
        return self.backend.combine(back_rows, state, T)

    __call__ = forward
