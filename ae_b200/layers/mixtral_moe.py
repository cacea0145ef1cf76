"""Drop-in for ``MixtralMoE`` (``specmoe/models/mixtral.py:59-115``): the router gate
(``ReplicatedLinear(H, E, bias=False)``, ``:85-92``) and the ``FusedMoE`` experts
(``:93-104``), with the gate fused into the routing launch.

The reference computes ``router_logits, _ = self.gate(hidden_states)`` (a half-precision
GEMM whose [T, E] output goes back to HBM) and then calls the experts.  Here
``forward`` makes one library call, ``smb_moe_forward_gated``: the gate GEMV and the
softmax/top-k/permutation run in one kernel, followed by the expert FFN and the combine.
Kept from the reference: the constructor signature, the ``gate.weight`` [E, H] and
``experts`` parameters (so checkpoint names ``block_sparse_moe.gate.weight`` and
``block_sparse_moe.experts.*`` load unchanged), ``forward(hidden_states,
experts_mapping)`` with 1-D or 2-D input, the in-place write into ``hidden_states``
(``FusedMoE`` runs with ``inplace=True``) and the tensor-parallel all-reduce when
``tp_size > 1`` (``:113-114``).
"""
from __future__ import annotations

from typing import Optional

import torch
import torch.distributed as dist

from .. import ops
from .FusedMoE import FusedMoE, _tp_world_size, expert_pool


class GateLinear(torch.nn.Module):
    """The router gate: ``weight`` [E, H] in the params dtype, no bias.  ``forward``
    returns ``(logits, None)`` like ``ReplicatedLinear``."""

    def __init__(self, input_size: int, output_size: int, params_dtype: torch.dtype):
        super().__init__()
        self.input_size = input_size
        self.output_size = output_size
        self.weight = torch.nn.Parameter(torch.empty(output_size, input_size, dtype=params_dtype),
                                         requires_grad=False)
        self.weight.weight_loader = self.weight_loader

    @staticmethod
    def weight_loader(param: torch.nn.Parameter, loaded_weight: torch.Tensor) -> None:
        if param.shape != loaded_weight.shape:
            raise ValueError(f"gate weight shape {tuple(loaded_weight.shape)} != {tuple(param.shape)}")
        param.data.copy_(loaded_weight)

    def forward(self, x: torch.Tensor):
        return ops.gate(x.contiguous(), self.weight), None


class MixtralMoE(torch.nn.Module):
    """Gate + experts of one Mixtral decoder layer (same constructor as the reference)."""

    def __init__(self, num_experts: int, top_k: int, hidden_size: int, intermediate_size: int,
                 params_dtype: Optional[torch.dtype] = None, quant_config=None,
                 tp_size: Optional[int] = None, prefix: str = "",
                 pin_experts_when_load_weight: bool = False):
        super().__init__()
        if params_dtype is None:
            params_dtype = torch.get_default_dtype()
        self.tp_size = _tp_world_size()
        self.hidden_size = hidden_size
        self.gate = GateLinear(hidden_size, num_experts, params_dtype)
        self.experts = FusedMoE(num_experts=num_experts, top_k=top_k, hidden_size=hidden_size,
                                intermediate_size=intermediate_size, params_dtype=params_dtype,
                                renormalize=True, quant_config=quant_config, tp_size=tp_size,
                                prefix=f"{prefix}.experts" if prefix else "experts",
                                pin_experts_when_load_weight=pin_experts_when_load_weight)

    def forward(self, hidden_states: torch.Tensor, experts_mapping: torch.Tensor) -> torch.Tensor:
        orig_shape = hidden_states.shape
        h = hidden_states.view(-1, self.hidden_size)
        out = ops.moe_forward_gated(h, self.gate.weight, expert_pool(self.experts), experts_mapping,
                                    self.experts.top_k, renormalize=True, out=h)
        if self.tp_size > 1:
            dist.all_reduce(out)
        return out.view(orig_shape)
