"""MoE layer shapes of the benchmark configurations and their seeded synthetic inputs.

Shapes follow the reference's model configs (Mixtral reads H / I / E / k from the HF
config, ``specmoe/utils/hf_transformers_utils.py:142-170``).  Inputs are synthetic and
seeded (no checkpoints or datasets are available): expert weights ~ N(0, 0.02) stored
in bf16, hidden states ~ N(0, 1), router logits = x @ Wr^T with a config-specific router
scale.  The page pool follows ``FusedMoE.weight_loader`` (page = [w1 | w3 | w2]).
"""
from __future__ import annotations

import dataclasses
import math

import torch


@dataclasses.dataclass(frozen=True)
class MoEConfig:
    name: str
    H: int            # hidden size
    I: int            # expert intermediate size
    E: int            # routed experts
    k: int            # top-k
    T: int            # tokens per layer call (verify batch)
    router_std: float  # std of the router weight entries
    renormalize: bool = True
    zipf_s: float = 0.0  # > 0: router bias making expert popularity ~ Zipf(s)
    shared_I: int = 0    # shared-expert intermediate size (0: none)

    @property
    def page_elems(self) -> int:
        return 3 * self.I * self.H

    def weight_bytes(self, touched: int | None = None, elem: int = 2) -> int:
        e = self.E if touched is None else touched
        return e * self.page_elems * elem


# configs of BASELINE.json, indexed like its "configs" list
C1 = MoEConfig("C1 scaled Mixtral H1024 I3584 E8 k2 T32", 1024, 3584, 8, 2, 32, router_std=0.02)
C2_T16 = MoEConfig("C2 Mixtral-8x7B H4096 I14336 E8 k2 T16", 4096, 14336, 8, 2, 16,
                   router_std=0.1 / math.sqrt(4096))
C2_T64 = dataclasses.replace(C2_T16, name="C2 Mixtral-8x7B H4096 I14336 E8 k2 T64", T=64)
C2_T256 = dataclasses.replace(C2_T16, name="C2 Mixtral-8x7B H4096 I14336 E8 k2 T256", T=256)
C3 = MoEConfig("C3 Qwen2-MoE-style H2048 I1408 E60 k4 T128 zipf1.1", 2048, 1408, 60, 4, 128,
               router_std=0.1 / math.sqrt(2048), zipf_s=1.1, shared_I=5632)
C4_LAYER = dataclasses.replace(C2_T16, name="C4 Mixtral-8x7B verify layer 4x32 draft tokens", T=128)
C5 = MoEConfig("C5 Mixtral-8x22B H6144 I16384 E8 k2 T512", 6144, 16384, 8, 2, 512,
               router_std=0.1 / math.sqrt(6144))

# prefill-sized batches through the same Mixtral-8x7B layer (tensor-core bound: 256+
# tokens per expert)
C2_T1024 = dataclasses.replace(C2_T16, name="C2 Mixtral-8x7B H4096 I14336 E8 k2 T1024 (prefill-sized)", T=1024)
C2_T2048 = dataclasses.replace(C2_T16, name="C2 Mixtral-8x7B H4096 I14336 E8 k2 T2048 (prefill-sized)", T=2048)

BY_KEY = {"c1": C1, "c2-16": C2_T16, "c2-64": C2_T64, "c2-256": C2_T256, "c3": C3, "c4": C4_LAYER,
          "c5": C5, "c2-1024": C2_T1024, "c2-2048": C2_T2048}


def make_pool(cfg: MoEConfig, device, dtype=torch.bfloat16, seed: int = 0, num_pages: int | None = None,
              experts=None):
    """Page pool [P, 3*I*H] ~ N(0, 0.02), generated page by page on ``device``.  Page p
    holds expert ``experts[p]`` (default: expert p); an expert's page is the same whichever
    pool (a rank's shard or the whole set) it is generated into."""
    ids = list(experts) if experts is not None else list(range(num_pages or cfg.E))
    pool = torch.empty(len(ids), cfg.page_elems, dtype=dtype, device=device)
    g = torch.Generator(device=device)
    for p, e in enumerate(ids):
        g.manual_seed(seed * 1000003 + e)
        pool[p].normal_(0.0, 0.02, generator=g)
    return pool


def make_inputs(cfg: MoEConfig, device, dtype=torch.bfloat16, seed: int = 0, T: int | None = None):
    """(x [T,H], router_logits [T,E]) with the config's router statistics."""
    T = cfg.T if T is None else T
    g = torch.Generator(device=device)
    g.manual_seed(seed * 7919 + 17)
    x = torch.randn(T, cfg.H, generator=g, device=device, dtype=torch.float32)
    wr = torch.randn(cfg.E, cfg.H, generator=g, device=device, dtype=torch.float32) * cfg.router_std
    logits = x @ wr.t()
    if cfg.zipf_s > 0:
        # expert popularity ~ Zipf(s) over a seeded rank order: bias -s*log(rank+1) plus
        # Gumbel(0,1) noise per (token, expert), so the top-1 choice is expert e with
        # probability (rank_e+1)^-s / sum (Gumbel-max) and the top-k choices follow it
        ranks = torch.randperm(cfg.E, generator=g, device=device).float()
        u = torch.rand(T, cfg.E, generator=g, device=device).clamp_(1e-12, 1.0 - 1e-7)
        logits = logits + (-cfg.zipf_s * torch.log(ranks + 1.0)).unsqueeze(0) - torch.log(-torch.log(u))
    return x.to(dtype), logits.to(dtype)


def make_gate_inputs(cfg: MoEConfig, device, dtype=torch.bfloat16, seed: int = 0, T: int | None = None):
    """(x [T,H], gate weight [E,H]) in the storage dtype for the gated block
    (``MixtralMoE``: router logits = x @ W^T computed by the layer itself); same statistics
    as :func:`make_inputs` without the Zipf bias (the reference gate has no bias)."""
    T = cfg.T if T is None else T
    g = torch.Generator(device=device)
    g.manual_seed(seed * 7919 + 17)
    x = torch.randn(T, cfg.H, generator=g, device=device, dtype=torch.float32)
    wr = torch.randn(cfg.E, cfg.H, generator=g, device=device, dtype=torch.float32) * cfg.router_std
    return x.to(dtype), wr.to(dtype)
