"""Drop-in for ``specmoe/layers/FusedMoE.py`` (the ``FusedMoE`` module SpecMoE's Mixtral
builds, ``specmoe/models/mixtral.py:93-104``), backed by the sm_100a library.

Kept from the reference:

* constructor signature and attributes (``FusedMoE.py:265-338``);
* ``ws``: the page-packed CPU expert store ``[E, 3*I_p*H]`` (pinned when
  ``pin_experts_when_load_weight``), page = ``[w1 | w3 | w2]`` (``:68-97``), with the GPU
  page pool hung on ``ws.gpu_cache`` by the engine (``mixtral.py:554-557``);
* ``weight_loader(param, loaded_weight, weight_name, shard_id, expert_id)`` with the same
  tensor-parallel slicing (``:485-505``) and ``make_expert_params_mapping`` (``:534-559``);
* ``forward(hidden_states, router_logits, expert_cache_indices)`` (``:508-532``): routing
  (softmax, top-k, renormalise), expert FFN and combine, written in place into
  ``hidden_states``; optional tensor-parallel all-reduce when ``reduce_results``.

Options the reference accepts but this path does not compute (grouped top-k, custom
routing, correction bias, quantisation, non-SiLU activations, router weight on input,
``no_combine``, ``routed_scaling_factor``) raise ``NotImplementedError`` instead of being
silently ignored.
"""
from __future__ import annotations

from typing import Callable, List, Optional, Tuple

import torch
import torch.distributed as dist

from .. import ops


def _tp_world_size() -> int:
    if dist.is_available() and dist.is_initialized():
        return dist.get_world_size()
    return 1


def _tp_rank() -> int:
    if dist.is_available() and dist.is_initialized():
        return dist.get_rank()
    return 0


def _make_pinned(nbytes: int, dtype: torch.dtype) -> torch.Tensor:
    # fp16/fp32/bf16 page store in page-locked host memory (the reference allocates it
    # with cudaMallocHost, specmoe/backend/pin_memory_allocator.py:10-55)
    elem = torch.tensor([], dtype=dtype).element_size()
    return torch.empty(nbytes // elem, dtype=dtype, pin_memory=True)


def expert_pool(layer: torch.nn.Module) -> torch.Tensor:
    """The GPU page pool of a FusedMoE: ``ws.gpu_cache`` as linked by the engine
    (``specmoe/models/mixtral.py:554-557``), or ``ws`` itself when it lives on the GPU."""
    pool = getattr(layer.ws, "gpu_cache", None)
    if pool is None:
        if not layer.ws.is_cuda:
            raise RuntimeError("FusedMoE.ws has no gpu_cache: the engine links the GPU expert pool "
                               "(MixtralForCausalLMOff.link_gpu_experts_cache) before forward")
        pool = layer.ws.data
    return pool


class UnquantizedFusedMoEMethod:
    """Weights and forward of the unquantised MoE (``FusedMoE.py:65-240``)."""

    def create_weights(self, layer: torch.nn.Module, num_experts: int, hidden_size: int,
                       intermediate_size: int, params_dtype: torch.dtype, **extra_weight_attrs):
        page = 3 * intermediate_size * hidden_size
        if layer.pin_experts_when_load_weight:
            elem = torch.tensor([], dtype=params_dtype).element_size()
            data = _make_pinned(num_experts * page * elem, params_dtype).reshape(num_experts, page)
        else:
            data = torch.empty(num_experts, page, dtype=params_dtype, device="cpu")
        ws = torch.nn.Parameter(data, requires_grad=False)
        layer.register_parameter("ws", ws)
        for k, v in extra_weight_attrs.items():
            setattr(ws, k, v)

    def apply(self, layer: torch.nn.Module, x: torch.Tensor, router_logits: torch.Tensor,
              expert_cache_indices: torch.Tensor, top_k: int, renormalize: bool,
              use_grouped_topk: bool, topk_group: Optional[int] = None,
              num_expert_group: Optional[int] = None,
              custom_routing_function: Optional[Callable] = None,
              correction_bias: Optional[torch.Tensor] = None, activation: str = "silu",
              apply_router_weight_on_input: bool = False, inplace: bool = True,
              no_combine: bool = False, routed_scaling_factor: Optional[float] = None) -> torch.Tensor:
        return self.forward_cuda(layer, x, expert_cache_indices, use_grouped_topk, top_k, router_logits,
                                 renormalize, topk_group, num_expert_group, custom_routing_function,
                                 correction_bias, activation, apply_router_weight_on_input, inplace,
                                 no_combine, routed_scaling_factor)

    def forward_cuda(self, layer, x, expert_cache_indices, use_grouped_topk, top_k, router_logits,
                     renormalize, topk_group=None, num_expert_group=None, custom_routing_function=None,
                     correction_bias=None, activation="silu", apply_router_weight_on_input=False,
                     inplace=True, no_combine=False, routed_scaling_factor=None) -> torch.Tensor:
        if use_grouped_topk or custom_routing_function is not None or correction_bias is not None:
            raise NotImplementedError("only plain softmax top-k routing is on the SpecMoE verify path")
        if activation != "silu":
            raise NotImplementedError(f"activation {activation!r} (only silu)")
        if apply_router_weight_on_input or no_combine:
            raise NotImplementedError("apply_router_weight_on_input / no_combine")
        if routed_scaling_factor is not None:
            raise NotImplementedError("routed_scaling_factor")
        pool = expert_pool(layer)
        # routing, permutation, expert FFN and combine; written in place like the
        # reference (stack_fused_moe(..., inplace=True), FusedMoE.py:187-196)
        return ops.moe_forward(x, router_logits.contiguous(), pool, expert_cache_indices, top_k,
                               renormalize, out=x)

    forward_native = forward_cuda


class FusedMoE(torch.nn.Module):
    """MoE layer: router top-k, per-expert SwiGLU FFN, weighted combine (in place)."""

    def __init__(self, num_experts: int, top_k: int, hidden_size: int, intermediate_size: int,
                 params_dtype: Optional[torch.dtype] = None, reduce_results: bool = False,
                 renormalize: bool = True, use_grouped_topk: bool = False,
                 num_expert_group: Optional[int] = None, topk_group: Optional[int] = None,
                 quant_config=None, tp_size: Optional[int] = None, prefix: str = "",
                 custom_routing_function: Optional[Callable] = None,
                 correction_bias: Optional[torch.Tensor] = None, activation: str = "silu",
                 apply_router_weight_on_input: bool = False, use_presharded_weights: bool = False,
                 inplace: bool = True, no_combine: bool = False,
                 routed_scaling_factor: Optional[float] = None,
                 pin_experts_when_load_weight: bool = False):
        super().__init__()
        if params_dtype is None:
            params_dtype = torch.get_default_dtype()
        self.tp_size = tp_size if tp_size is not None else _tp_world_size()
        self.routed_scaling_factor = routed_scaling_factor
        self.top_k = top_k
        self.num_experts = num_experts
        if intermediate_size % self.tp_size != 0:
            raise AssertionError("intermediate_size must divide by tp_size")
        self.intermediate_size_per_partition = intermediate_size // self.tp_size
        self.hidden_size = hidden_size
        self.reduce_results = reduce_results
        self.renormalize = renormalize
        self.use_grouped_topk = use_grouped_topk
        if self.use_grouped_topk:
            assert num_expert_group is not None and topk_group is not None
        self.num_expert_group = num_expert_group
        self.topk_group = topk_group
        self.custom_routing_function = custom_routing_function
        self.correction_bias = correction_bias
        self.activation = activation
        self.apply_router_weight_on_input = apply_router_weight_on_input
        self.use_presharded_weights = use_presharded_weights
        self.inplace = inplace
        self.no_combine = no_combine
        self.local_num_experts = num_experts
        self.pin_experts_when_load_weight = pin_experts_when_load_weight
        if quant_config is not None:
            raise NotImplementedError("quantised experts are not on this path")
        self.quant_method = UnquantizedFusedMoEMethod()
        self.quant_method.create_weights(layer=self, num_experts=num_experts, hidden_size=hidden_size,
                                         intermediate_size=self.intermediate_size_per_partition,
                                         params_dtype=params_dtype, weight_loader=self.weight_loader)

    def weight_loader(self, param: torch.nn.Parameter, loaded_weight: torch.Tensor, weight_name: str,
                      shard_id: str, expert_id: int) -> None:
        """Copy one checkpoint tensor into its slice of the expert's page (``:485-505``)."""
        tp_rank = _tp_rank() if self.tp_size > 1 else 0
        data = param.data
        shard_size = self.intermediate_size_per_partition
        shard = slice(tp_rank * shard_size, (tp_rank + 1) * shard_size)
        w3_offset = shard_size * self.hidden_size
        w2_offset = 2 * shard_size * self.hidden_size
        if weight_name.endswith("w1.weight"):
            data[expert_id, 0:w3_offset] = loaded_weight[shard, :].reshape(-1)
        if weight_name.endswith("w3.weight"):
            data[expert_id, w3_offset:w2_offset] = loaded_weight[shard, :].reshape(-1)
        if weight_name.endswith("w2.weight"):
            data[expert_id, w2_offset:] = loaded_weight[:, shard].reshape(-1)

    def forward(self, hidden_states: torch.Tensor, router_logits: torch.Tensor,
                expert_cache_indices: torch.Tensor) -> torch.Tensor:
        out = self.quant_method.apply(
            layer=self, x=hidden_states, router_logits=router_logits,
            expert_cache_indices=expert_cache_indices, top_k=self.top_k, renormalize=self.renormalize,
            use_grouped_topk=self.use_grouped_topk, topk_group=self.topk_group,
            num_expert_group=self.num_expert_group, custom_routing_function=self.custom_routing_function,
            correction_bias=self.correction_bias, activation=self.activation,
            apply_router_weight_on_input=self.apply_router_weight_on_input,
            routed_scaling_factor=self.routed_scaling_factor)
        if self.reduce_results and self.tp_size > 1:
            dist.all_reduce(out)
        return out

    @classmethod
    def make_expert_params_mapping(cls, ckpt_gate_proj_name: str, ckpt_down_proj_name: str,
                                   ckpt_up_proj_name: str, num_experts: int) -> List[Tuple[str, str, int, str]]:
        """(param_name, weight_name, expert_id, shard_id) tuples (``:534-559``)."""
        return [("experts.ws", f"experts.{expert_id}.{weight_name}.weight", expert_id, shard_id)
                for expert_id in range(num_experts)
                for shard_id, weight_name in [("w1", ckpt_gate_proj_name), ("w2", ckpt_down_proj_name),
                                              ("w3", ckpt_up_proj_name)]]
