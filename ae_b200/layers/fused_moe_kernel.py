"""Drop-in for ``specmoe/layers/fused_moe_kernel.py`` backed by the sm_100a library.

Public surface kept from the reference:

* ``moe_align_block_size(topk_ids, block_size, num_experts)`` (reference ``:16-85``);
* ``stack_fused_moe(hidden_states, w1, indicies, gating_output, topk_weights, topk_ids,
  renormalize, inplace=False)`` (reference ``:253-349``): ``w1`` is the expert page pool
  ``[P, 3*I*H]`` with pages ``[w1 | w3 | w2]``, ``indicies`` the int64 page of each
  expert, ``gating_output`` supplies E, and the routing is taken from ``topk_weights`` /
  ``topk_ids``.  With ``inplace=True`` the result is written into ``hidden_states``.

The Triton kernel, its launcher and the three intermediate caches of the reference are
replaced by four library kernels (permute+gather, gate/up GEMM with SiLU*mul epilogue,
split-K down GEMM, combine) that share one reusable workspace.
"""
from __future__ import annotations

from typing import Tuple

import torch

from .. import ops


def moe_align_block_size(topk_ids: torch.Tensor, block_size: int,
                         num_experts: int) -> Tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    """Block-padded expert-major layout (pad value ``topk_ids.numel()``).

    ``expert_ids`` entries past the last used block are -1 (left uninitialised by the
    reference).
    """
    return ops.align_block_size(topk_ids, block_size, num_experts)


def stack_fused_moe(hidden_states: torch.Tensor, w1: torch.Tensor, indicies: torch.Tensor,
                    gating_output: torch.Tensor, topk_weights: torch.Tensor, topk_ids: torch.Tensor,
                    renormalize: bool, inplace: bool = False) -> torch.Tensor:
    """Mixture-of-experts layer from a given routing (reference ``:253-349``)."""
    if hidden_states.shape[0] != gating_output.shape[0]:
        raise AssertionError("Number of tokens mismatch")
    if not hidden_states.is_contiguous():
        raise AssertionError("Hidden_states must be contiguous")
    if not w1.is_contiguous():
        raise AssertionError("Expert weights1 must be contiguous")
    if hidden_states.dtype not in (torch.float16, torch.bfloat16):
        raise NotImplementedError("storage dtype must be float16 or bfloat16 on this path")
    E = gating_output.shape[1]
    w = topk_weights if topk_weights.dtype == torch.float32 else topk_weights.float()
    ids = topk_ids if topk_ids.dtype == torch.int32 else topk_ids.to(torch.int32)
    out = hidden_states if inplace else None
    return ops.moe_forward_routed(hidden_states, w.contiguous(), ids.contiguous(), w1, indicies, E, out=out)
