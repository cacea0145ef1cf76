"""CPU oracle for the SpecMoE verify-layer MoE path.  TEST INFRASTRUCTURE ONLY.

This module restates, on the CPU, the arithmetic of the reference layer so that the
CUDA path can be checked against it.  Only ``tests/``, ``__graft_entry__.smoke()`` and
the ``cpu_baseline`` / ``--impl reference`` legs of ``bench.py`` may import it; the
product package (``ae_b200``) never does.

What it follows, in the reference tree (zzhbrr/ae):

* routing: ``select_experts`` of sglang==0.4.5.post3 as called from
  ``specmoe/layers/FusedMoE.py:174-185`` with ``use_grouped_topk=False``, no custom
  routing function and no correction bias: softmax over the E experts in fp32, top-k,
  and (``renormalize=True`` for Mixtral, ``specmoe/models/mixtral.py:99``) division of
  the k selected probabilities by their sum.  Output: weights fp32 [T,k], ids int32
  [T,k].  sglang is not vendored; its published algorithm is restated here.  Ties are
  broken towards the lower expert index.  Selection is done on the fp32 logits (the
  softmax is monotone, so this equals selection on the probabilities whenever the
  probabilities are distinct).
* permutation: the ``moe_align_block_size`` contract documented at
  ``specmoe/layers/fused_moe_kernel.py:16-55`` (sgl-kernel==0.1.2): flat assignment
  index f = t*k + j, bucketed by expert, ascending f inside an expert, each expert padded
  to a multiple of ``block_size`` with the value T*k.
* page layout: ``FusedMoE.weight_loader`` (``specmoe/layers/FusedMoE.py:485-505``): one
  flat page per expert ``[w1 (I x H) | w3 (I x H) | w2 (H x I)]``, all row-major.
* FFN: ``stack_fused_moe`` (``specmoe/layers/fused_moe_kernel.py:253-349``) and the
  Triton ``fused_moe_kernel`` it launches twice (``:88-210``):
  GEMM1 ``c1[f, n] = sum_h x[f // k, h] * page[n*H + h]`` for n < 2I (pool viewed as
  ``[P, 3I, H]``, ``:332``), ``silu_and_mul`` (``:337``), GEMM2 over the pool viewed as
  ``[P, 3H, I]`` starting at row 2H (``:339-342``) multiplied by the routing weight of
  the flat slot (``:197-201``), then ``torch.sum`` over the k slots (``:344-349``).

Two numeric modes:

* ``rounding="fp32"``: everything in fp32, no intermediate rounding.  This is the fp32
  reference the tolerances are stated against (max-abs <= 2e-2, rel-L2 <= 1e-2).
* ``rounding="reference"``: rounds to the storage dtype exactly where the Triton path
  does: after GEMM1 (``:203``, cache1), after SiLU*mul (cache2), after weight*GEMM2
  (``:201-203``, cache3) and after the sum over k (``:344``).

Parity pin: the ``stack_fused_moe`` arithmetic is pinned by golden vectors produced by
the reference's own Triton kernel (run by the Triton CPU interpreter, fp16 and fp32;
``tests/golden/make_golden.py``), and the permutation by the known-answer example in the
``moe_align_block_size`` docstring.  Routing (sglang) has no reference-side vector and is
restated from its published algorithm.
"""
from __future__ import annotations

import numpy as np
import torch

__all__ = [
    "select_experts",
    "permutation",
    "moe_align_block_size",
    "page_views",
    "stack_fused_moe",
    "fused_moe_forward",
    "pack_page",
]


def select_experts(logits, top_k: int, renormalize: bool = True):
    """softmax -> top-k -> optional renormalise; ties go to the lower expert index.

    Follows sglang ``select_experts`` as called at ``specmoe/layers/FusedMoE.py:174-185``.
    Returns ``(weights fp32 [T,k], ids int32 [T,k])`` as numpy arrays.
    """
    lg = np.asarray(torch.as_tensor(logits).float().numpy(), dtype=np.float32)
    T, E = lg.shape
    if not 1 <= top_k <= E:
        raise ValueError("top_k must be in [1, E]")
    m = lg.max(axis=1, keepdims=True)
    ex = np.exp((lg - m).astype(np.float32), dtype=np.float32)
    p = (ex * (np.float32(1.0) / ex.sum(axis=1, keepdims=True, dtype=np.float32))).astype(np.float32)
    # stable sort on -logit keeps the lower index first among equal logits
    order = np.argsort(-lg, axis=1, kind="stable")[:, :top_k]
    ids = order.astype(np.int32)
    w = np.take_along_axis(p, order, axis=1).astype(np.float32)
    if renormalize:
        w = (w / w.sum(axis=1, keepdims=True, dtype=np.float32)).astype(np.float32)
    return w, ids


def permutation(topk_ids, num_experts: int):
    """Unpadded expert-major permutation.

    ``perm[p]`` is the flat index f = t*k + j placed at position p; positions of expert
    e are ``[off[e], off[e+1])`` and, inside an expert, f ascends (the order of the
    ``moe_align_block_size`` docstring, ``specmoe/layers/fused_moe_kernel.py:41-54``,
    with the pad entries removed).  Also returns ``inv`` with ``inv[f] = p``.
    """
    ids = np.asarray(topk_ids).reshape(-1).astype(np.int64)
    if ids.size and (ids.min() < 0 or ids.max() >= num_experts):
        raise ValueError("expert id out of range")
    perm = np.argsort(ids, kind="stable").astype(np.int32)
    counts = np.bincount(ids, minlength=num_experts).astype(np.int64)
    off = np.zeros(num_experts + 1, dtype=np.int32)
    off[1:] = np.cumsum(counts)
    inv = np.empty_like(perm)
    inv[perm] = np.arange(perm.size, dtype=np.int32)
    return perm, off, inv


def moe_align_block_size(topk_ids, block_size: int, num_experts: int):
    """Block-padded layout of ``specmoe/layers/fused_moe_kernel.py:16-85``.

    Returns ``(sorted_ids int32 [numel + E*(block-1)], expert_ids int32
    [cdiv(len(sorted_ids), block)], num_tokens_post_pad int32 [1])``.  Entries past the
    padded end keep the fill value T*k; ``expert_ids`` past the last used block are left
    at -1 (the reference leaves them uninitialised).
    """
    ids = np.asarray(topk_ids).reshape(-1).astype(np.int64)
    numel = ids.size
    max_padded = numel + num_experts * (block_size - 1)
    sorted_ids = np.full(max_padded, numel, dtype=np.int32)
    n_blocks = -(-max_padded // block_size)
    expert_ids = np.full(n_blocks, -1, dtype=np.int32)
    pos = 0
    for e in range(num_experts):
        sel = np.nonzero(ids == e)[0].astype(np.int32)
        n = sel.size
        sorted_ids[pos:pos + n] = sel
        nb = -(-n // block_size)
        expert_ids[pos // block_size: pos // block_size + nb] = e
        pos += nb * block_size
    return sorted_ids, expert_ids, np.array([pos], dtype=np.int32)


def pack_page(w1, w3, w2):
    """One expert page ``[w1 | w3 | w2]`` flattened row-major (``FusedMoE.py:497-505``).

    w1, w3: [I, H] (gate_proj, up_proj); w2: [H, I] (down_proj).
    """
    w1 = torch.as_tensor(w1)
    return torch.cat([w1.reshape(-1), torch.as_tensor(w3).reshape(-1),
                      torch.as_tensor(w2).reshape(-1)])


def page_views(page, H: int, I: int):
    """Split one flat page into (w1 [I,H], w3 [I,H], w2 [H,I]) views."""
    w1 = page[: I * H].view(I, H)
    w3 = page[I * H: 2 * I * H].view(I, H)
    w2 = page[2 * I * H:].view(H, I)
    return w1, w3, w2


def _round(t, dt):
    return t.to(dt).float()


def stack_fused_moe(hidden_states, pool, page_of_expert, topk_weights, topk_ids,
                    rounding: str = "fp32", compute_dtype=None, threads: int | None = None):
    """CPU restatement of ``stack_fused_moe`` (``specmoe/layers/fused_moe_kernel.py:253-349``).

    hidden_states [T,H]; pool [P, 3*I*H] page-packed; page_of_expert int [E] (the
    ``indicies`` argument); topk_weights fp32 [T,k]; topk_ids int [T,k].

    rounding="fp32": fp32 result (torch.float32 tensor [T,H]).
    rounding="reference": rounds at the reference's four points, returns the storage
    dtype.  compute_dtype=torch.bfloat16 runs each expert's matmuls on the storage dtype
    (fp32 accumulation inside torch's CPU GEMM): the timed CPU baseline, not a checker.
    """
    if threads is not None:
        torch.set_num_threads(int(threads))
    x = torch.as_tensor(hidden_states)
    pool = torch.as_tensor(pool)
    dt = x.dtype
    T, H = x.shape
    P, page = pool.shape
    if page % (3 * H):
        raise ValueError("page size must be 3*I*H")
    I = page // (3 * H)
    pidx = torch.as_tensor(page_of_expert).to(torch.int64).cpu()
    w = torch.as_tensor(np.asarray(topk_weights, dtype=np.float32))
    ids = torch.as_tensor(np.asarray(topk_ids)).to(torch.int64)
    k = ids.shape[1]
    E = pidx.numel()
    flat = ids.reshape(-1)
    wf = w.reshape(-1)
    ref_round = rounding == "reference"
    if rounding not in ("fp32", "reference"):
        raise ValueError(rounding)
    cache3 = torch.zeros(T * k, H, dtype=torch.float32)
    for e in range(E):
        fsel = torch.nonzero(flat == e).flatten()
        if fsel.numel() == 0:
            continue
        pg = int(pidx[e])
        if not 0 <= pg < P:
            raise ValueError("page id out of range")
        w1, w3, w2 = page_views(pool[pg], H, I)
        xe = x[fsel // k]
        if compute_dtype is not None:
            g = xe.to(compute_dtype) @ w1.to(compute_dtype).T
            u = xe.to(compute_dtype) @ w3.to(compute_dtype).T
            a = (torch.nn.functional.silu(g.float()) * u.float()).to(compute_dtype)
            y = (a @ w2.to(compute_dtype).T).float()
        else:
            xf = xe.float()
            g = xf @ w1.float().T
            u = xf @ w3.float().T
            if ref_round:
                g, u = _round(g, dt), _round(u, dt)
            a = torch.nn.functional.silu(g) * u
            if ref_round:
                a = _round(a, dt)
            y = a @ w2.float().T
        y = y * wf[fsel].unsqueeze(1)
        if ref_round:
            y = _round(y, dt)
        cache3[fsel] = y
    out = cache3.view(T, k, H).sum(dim=1)
    if ref_round or compute_dtype is not None:
        return out.to(dt)
    return out


def fused_moe_forward(hidden_states, router_logits, pool, page_of_expert, top_k: int,
                      renormalize: bool = True, rounding: str = "fp32"):
    """``FusedMoE.forward`` (``specmoe/layers/FusedMoE.py:508-532``) without TP reduce:
    routing (``select_experts``) followed by ``stack_fused_moe``.  Returns
    ``(out, topk_weights, topk_ids)``.
    """
    w, ids = select_experts(router_logits, top_k, renormalize)
    out = stack_fused_moe(hidden_states, pool, page_of_expert, w, ids, rounding=rounding)
    return out, w, ids


def gate_logits(hidden_states, gate_weight):
    """Router logits of ``MixtralMoE.gate`` (``specmoe/models/mixtral.py:85-92``, called at
    ``:111``): ``ReplicatedLinear(H, E, bias=False)`` in the params dtype, i.e.
    ``x @ W^T`` accumulated in high precision (fp64 here) and rounded once to the storage
    dtype of ``hidden_states``.  Returns the logits in that dtype."""
    x = torch.as_tensor(hidden_states)
    w = torch.as_tensor(gate_weight)
    return (x.double() @ w.double().t()).to(x.dtype)


def mixtral_moe_forward(hidden_states, gate_weight, pool, page_of_expert, top_k: int,
                        rounding: str = "fp32"):
    """``MixtralMoE.forward`` (``specmoe/models/mixtral.py:106-115``) without the TP
    all-reduce: the gate, then ``FusedMoE.forward`` with ``renormalize=True`` (``:99``).
    Returns ``(out, router_logits, topk_weights, topk_ids)``."""
    logits = gate_logits(hidden_states, gate_weight)
    out, w, ids = fused_moe_forward(hidden_states, logits.float(), pool, page_of_expert, top_k, True,
                                    rounding=rounding)
    return out, logits, w, ids


def shared_expert_forward(hidden_states, w1, w3, w2, shared_weight=None):
    """A shared expert computed directly, in fp32: ``s_t * w2 (silu(w1 x_t) * (w3 x_t))``
    with w1, w3 [I_s, H], w2 [H, I_s] and ``s_t = shared_weight[t]`` (1 when None).  The
    reference (SpecMoE) has no shared expert; this states the Qwen2-MoE-style block the
    fine-grained benchmark configuration names (shared expert output added to the routed
    experts' sum, scaled by the sigmoid of a shared gate)."""
    x = torch.as_tensor(hidden_states).float()
    g = x @ torch.as_tensor(w1).float().t()
    u = x @ torch.as_tensor(w3).float().t()
    y = (torch.nn.functional.silu(g) * u) @ torch.as_tensor(w2).float().t()
    if shared_weight is not None:
        y = y * torch.as_tensor(shared_weight).float().view(-1, 1)
    return y


def error_metrics(got, ref):
    """(max-abs error, relative-L2 error) of ``got`` against the fp32 ``ref``."""
    g = torch.as_tensor(got).double()
    r = torch.as_tensor(ref).double()
    d = g - r
    max_abs = float(d.abs().max()) if d.numel() else 0.0
    den = float(r.norm())
    rel = float(d.norm()) / den if den > 0 else float(d.norm())
    return max_abs, rel
