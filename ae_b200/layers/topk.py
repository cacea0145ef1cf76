"""``select_experts`` for the path SpecMoE uses (sglang==0.4.5.post3 semantics).

Reference call: ``specmoe/layers/FusedMoE.py:174-185`` with ``use_grouped_topk=False``,
no custom routing function and no correction bias (Mixtral, ``renormalize=True`` at
``specmoe/models/mixtral.py:99``).  The other routing variants sglang offers are not on
this path and raise ``NotImplementedError``.
"""
from __future__ import annotations

from typing import Callable, Optional

import torch

from .. import ops


def select_experts(hidden_states: torch.Tensor, router_logits: torch.Tensor, top_k: int,
                   use_grouped_topk: bool, renormalize: bool, topk_group: Optional[int] = None,
                   num_expert_group: Optional[int] = None,
                   custom_routing_function: Optional[Callable] = None,
                   correction_bias: Optional[torch.Tensor] = None,
                   torch_native: bool = False,
                   routed_scaling_factor: Optional[float] = None):
    """softmax -> top-k -> optional renormalise on the GPU.

    Returns ``(topk_weights fp32 [T,k], topk_ids int32 [T,k])``; ties go to the lower
    expert index.
    """
    if use_grouped_topk or custom_routing_function is not None or correction_bias is not None:
        raise NotImplementedError("only plain softmax top-k routing is on the SpecMoE verify path")
    if routed_scaling_factor is not None:
        raise NotImplementedError("routed_scaling_factor is not used on the SpecMoE verify path")
    if hidden_states.shape[0] != router_logits.shape[0]:
        raise ValueError("Number of tokens mismatch")
    return ops.topk(router_logits.contiguous(), top_k, renormalize)
