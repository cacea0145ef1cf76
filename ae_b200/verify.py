"""Speculative-verification step of a Mixtral-architecture decoder around the MoE layer.

The reference runs this step inside its engine (sglang model runner, paged KV cache,
EAGLE draft trees: ``specmoe/engine.py``, ``specmoe/models/mixtral.py:118-330``), which
cannot run here.  This module is the minimal decoder that puts the layer in its real
context for the 32-layer verify configuration: per layer RMSNorm -> grouped-query
attention with rotary embeddings over a KV cache plus the draft tree (tree mask: a draft
token sees the cache, its ancestors and itself) -> RMSNorm -> MoE block (gate + experts,
``ae_b200.ops.moe_forward_gated``), residual adds as in ``MixtralDecoderLayer``
(``mixtral.py:226-268``); then the final norm, the LM head and greedy acceptance of the
draft tree.  Weights are random (no checkpoints); shapes follow Mixtral-8x7B.

The MoE calls can be bracketed by CUDA events (``moe_events``) so that the MoE layers'
share of the step is measured on the device.
"""
from __future__ import annotations

import dataclasses
import math
from typing import Callable, List, Optional

import torch

from . import ops


@dataclasses.dataclass(frozen=True)
class DecoderConfig:
    layers: int = 32
    H: int = 4096
    I: int = 14336
    E: int = 8
    k: int = 2
    heads: int = 32
    kv_heads: int = 8
    head_dim: int = 128
    vocab: int = 32000
    rope_theta: float = 1e6
    eps: float = 1e-5


MIXTRAL_8X7B = DecoderConfig()


def tree_mask(parents: List[int]) -> torch.Tensor:
    """[n, n] bool: entry (i, j) is True when draft token j is token i or an ancestor of it
    (parents[i] < i, -1 for a child of the last verified token)."""
    n = len(parents)
    m = torch.zeros(n, n, dtype=torch.bool)
    for i, p in enumerate(parents):
        if p >= i:
            raise ValueError("parents must point to earlier tokens")
        m[i, i] = True
        if p >= 0:
            m[i] |= m[p]
    return m


def tree_depths(parents: List[int]) -> List[int]:
    d = []
    for p in parents:
        d.append(0 if p < 0 else d[p] + 1)
    return d


def rope(x: torch.Tensor, pos: torch.Tensor, theta: float) -> torch.Tensor:
    """Rotary embedding (rotate-half form used by Mixtral/Llama) of x [..., n, d] at
    positions pos [n]."""
    d = x.shape[-1]
    inv = 1.0 / (theta ** (torch.arange(0, d, 2, device=x.device, dtype=torch.float32) / d))
    ang = pos.to(torch.float32)[:, None] * inv[None, :]
    cos = torch.cat([ang.cos(), ang.cos()], dim=-1)
    sin = torch.cat([ang.sin(), ang.sin()], dim=-1)
    xf = x.float()
    x1, x2 = xf[..., : d // 2], xf[..., d // 2:]
    rot = torch.cat([-x2, x1], dim=-1)
    return (xf * cos + rot * sin).to(x.dtype)


def rms_norm(x: torch.Tensor, w: torch.Tensor, eps: float) -> torch.Tensor:
    xf = x.float()
    return (xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + eps) * w.float()).to(x.dtype)


class VerifyDecoder:
    """Random-init Mixtral-architecture decoder with a KV cache of ``cache_len`` tokens per
    sequence (filled with random keys/values) and room for ``max_draft`` draft tokens.

    ``moe`` computes one MoE block in place: ``moe(layer, h [N, H]) -> h``; by default the
    sm_100a library (gate fused into the routing launch).  The expert pools are held per
    layer on the device: ``pools[l]`` [E, 3*I*H], page table identity."""

    def __init__(self, cfg: DecoderConfig, batch: int, cache_len: int, max_draft: int, device,
                 dtype=torch.bfloat16, seed: int = 0, moe: Optional[Callable] = None):
        self.cfg, self.batch, self.cache_len, self.max_draft = cfg, batch, cache_len, max_draft
        self.device = torch.device(device)
        self.dtype = dtype
        c = cfg
        g = torch.Generator(device=self.device)
        g.manual_seed(seed)

        def rnd(*shape, std):
            return (torch.randn(*shape, generator=g, device=self.device, dtype=torch.float32) * std).to(dtype)

        qd, kvd = c.heads * c.head_dim, c.kv_heads * c.head_dim
        self.embed = rnd(c.vocab, c.H, std=1.0)
        self.lm_head = rnd(c.vocab, c.H, std=1.0 / math.sqrt(c.H))
        self.final_norm = torch.ones(c.H, dtype=dtype, device=self.device)
        self.layers = []
        for _ in range(c.layers):
            pool = torch.empty(c.E, 3 * c.I * c.H, dtype=dtype, device=self.device)
            pool.normal_(0.0, 0.02, generator=g)
            self.layers.append({
                "wqkv": rnd(qd + 2 * kvd, c.H, std=1.0 / math.sqrt(c.H)),
                "wo": rnd(c.H, qd, std=1.0 / math.sqrt(qd)),
                "norm1": torch.ones(c.H, dtype=dtype, device=self.device),
                "norm2": torch.ones(c.H, dtype=dtype, device=self.device),
                "gate": rnd(c.E, c.H, std=1.0 / math.sqrt(c.H)),
                "pool": pool,
            })
        self.pages = torch.arange(c.E, dtype=torch.int64, device=self.device)
        S = cache_len + max_draft
        self.k_cache = [rnd(batch, c.kv_heads, S, c.head_dim, std=1.0) for _ in range(c.layers)]
        self.v_cache = [rnd(batch, c.kv_heads, S, c.head_dim, std=1.0) for _ in range(c.layers)]
        self.moe = moe or self._library_moe

    def _library_moe(self, layer: int, h: torch.Tensor) -> torch.Tensor:
        L = self.layers[layer]
        return ops.moe_forward_gated(h, L["gate"], L["pool"], self.pages, self.cfg.k, True, out=h)

    def attention(self, layer: int, h: torch.Tensor, pos: torch.Tensor, mask: torch.Tensor) -> torch.Tensor:
        """h [B, n, H] -> [B, n, H]; writes the draft tokens' keys/values into the cache at
        [cache_len, cache_len + n)."""
        c, L = self.cfg, self.layers[layer]
        B, n, _ = h.shape
        qd, kvd = c.heads * c.head_dim, c.kv_heads * c.head_dim
        qkv = h @ L["wqkv"].t()
        q = qkv[..., :qd].view(B, n, c.heads, c.head_dim).transpose(1, 2)
        k = qkv[..., qd:qd + kvd].view(B, n, c.kv_heads, c.head_dim).transpose(1, 2)
        v = qkv[..., qd + kvd:].view(B, n, c.kv_heads, c.head_dim).transpose(1, 2)
        q = rope(q, pos, c.rope_theta)
        k = rope(k, pos, c.rope_theta)
        s0 = self.cache_len
        self.k_cache[layer][:, :, s0:s0 + n] = k
        self.v_cache[layer][:, :, s0:s0 + n] = v
        keys = self.k_cache[layer][:, :, :s0 + n]
        vals = self.v_cache[layer][:, :, :s0 + n]
        full = torch.ones(n, s0 + n, dtype=torch.bool, device=h.device)
        full[:, s0:] = mask
        o = torch.nn.functional.scaled_dot_product_attention(q, keys, vals, attn_mask=full, enable_gqa=True)
        return o.transpose(1, 2).reshape(B, n, qd) @ L["wo"].t()

    def forward(self, tokens: torch.Tensor, parents: List[int], moe_events=None) -> torch.Tensor:
        """Logits [B, n, vocab] of the draft tree ``tokens`` [B, n] (same tree shape
        ``parents`` for every sequence).  ``moe_events``: optional list of (start, end)
        CUDA event pairs, one per layer, recorded around each MoE call."""
        c = self.cfg
        B, n = tokens.shape
        if n > self.max_draft:
            raise ValueError("more draft tokens than the cache has room for")
        mask = tree_mask(parents).to(self.device)
        pos = torch.tensor(tree_depths(parents), device=self.device) + self.cache_len
        h = self.embed[tokens]
        for li in range(c.layers):
            L = self.layers[li]
            h = h + self.attention(li, rms_norm(h, L["norm1"], c.eps), pos, mask)
            y = rms_norm(h, L["norm2"], c.eps).reshape(B * n, c.H).contiguous()
            if moe_events is not None:
                moe_events[li][0].record()
            y = self.moe(li, y)
            if moe_events is not None:
                moe_events[li][1].record()
            h = h + y.view(B, n, c.H)
        return rms_norm(h, self.final_norm, c.eps) @ self.lm_head.t()


def accept_greedy(logits: torch.Tensor, tokens: torch.Tensor, parents: List[int], root_logits: torch.Tensor):
    """Greedy verification of a draft tree: a draft token is accepted when it equals the
    argmax of its parent's logits (``root_logits`` [B, vocab] for children of the last
    verified token) and its parent was accepted.  Returns (accepted [B, n] bool, number of
    tokens on the longest accepted path [B])."""
    B, n = tokens.shape
    pred = logits.argmax(-1)           # [B, n]
    root_pred = root_logits.argmax(-1)  # [B]
    acc = torch.zeros(B, n, dtype=torch.bool, device=tokens.device)
    depth = torch.zeros(B, n, dtype=torch.int64, device=tokens.device)
    for i, p in enumerate(parents):
        if p < 0:
            acc[:, i] = tokens[:, i] == root_pred
            depth[:, i] = acc[:, i].long()
        else:
            acc[:, i] = acc[:, p] & (tokens[:, i] == pred[:, p])
            depth[:, i] = torch.where(acc[:, i], depth[:, p] + 1, torch.zeros_like(depth[:, p]))
    return acc, depth.max(dim=1).values


def random_tree(n: int, seed: int = 0, max_children: int = 4) -> List[int]:
    """A seeded draft-tree shape of n tokens (parents[i] < i), breadth-first like the
    top-k expansion of an EAGLE-style drafter."""
    g = torch.Generator().manual_seed(seed)
    parents = []
    children = {-1: 0}
    frontier = [-1]
    i = 0
    while i < n:
        p = frontier[0]
        limit = max_children if p < 0 else int(torch.randint(1, max_children + 1, (1,), generator=g))
        if children.get(p, 0) >= limit:
            frontier.pop(0)
            continue
        parents.append(p)
        children[p] = children.get(p, 0) + 1
        frontier.append(i)
        i += 1
    return parents
