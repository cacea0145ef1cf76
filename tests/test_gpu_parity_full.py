"""Parity at the headline and full expert sizes, through the same call the bench times.

The bench line's workload (Mixtral-8x7B, T = 256: split-K S = 2, 64-token tiles), a
smaller verify batch of the same layer (T = 64) and Mixtral-8x22B at T = 512 (128+ tokens
per expert: the TMA token-tile path) run through ``ops.moe_forward`` (``smb_moe_forward``)
on the bench's own seeded inputs (``ae_b200.configs``) and are checked against the fp32
CPU oracle (``oracle.stack_fused_moe``, restating
specmoe/layers/fused_moe_kernel.py:253-349):

* routing ids, weights and the expert-major permutation bit-exact (ids / permutation) and
  to fp32 rounding (weights);
* hidden states: relative-L2 <= 1e-2 and max-abs <= 2e-2, or, where larger, the error of
  the reference's own arithmetic at these sizes (the oracle's reference-rounding mode,
  which stores the SiLU*mul activations and each expert's weighted output in bf16 like the
  reference's cache2 / cache3, against fp32).  Each case prints its measured errors next
  to that bar (``PARITY`` lines, ``pytest -s``).
"""
import numpy as np
import pytest
import torch

from oracle import moe_oracle as mo

pytestmark = pytest.mark.gpu

MAX_ABS, REL_L2 = 2e-2, 1e-2


@pytest.mark.parametrize("key,T", [("c2-256", 256), ("c2-256", 64), ("c5", 512)])
def test_headline_layer_vs_oracle(key, T):
    from ae_b200 import configs, ops
    cfg = configs.BY_KEY[key]
    dev = torch.device("cuda", 0)
    pool = configs.make_pool(cfg, dev, seed=0)
    pages = torch.arange(cfg.E, device=dev, dtype=torch.int64)
    x, logits = configs.make_inputs(cfg, dev, seed=0, T=T)
    w = torch.empty(T, cfg.k, dtype=torch.float32, device=dev)
    ids = torch.empty(T, cfg.k, dtype=torch.int32, device=dev)
    out = ops.moe_forward(x, logits, pool, pages, cfg.k, cfg.renormalize, topk_weights=w, topk_ids=ids)
    # the permutation of the same routing, from the router alone
    L = ops.StagedLayer(T, cfg.E, cfg.k, cfg.H, cfg.I, x.dtype, dev)
    L.route(logits, x, cfg.renormalize)
    torch.cuda.synchronize()
    v = L.views()
    rw, rids = mo.select_experts(logits.cpu(), cfg.k, cfg.renormalize)
    perm, off, inv = mo.permutation(rids, cfg.E)
    assert (ids.cpu().numpy() == rids).all(), "routing ids differ"
    np.testing.assert_allclose(w.cpu().numpy(), rw, rtol=2e-6, atol=1e-7)
    assert (v["expert_off"].cpu().numpy() == off).all()
    assert (v["perm"].cpu().numpy() == perm).all()
    assert (v["inv"].cpu().numpy() == inv).all()
    assert L.status() == 0
    del L
    xc, pc, gc = x.cpu(), pool.cpu(), pages.cpu()
    got = out.float().cpu()
    del pool, out
    torch.cuda.empty_cache()
    ref = mo.stack_fused_moe(xc, pc, gc, rw, rids, rounding="fp32").float()
    ref_r = mo.stack_fused_moe(xc, pc, gc, rw, rids, rounding="reference").float()
    ref_err = float((ref_r - ref).abs().max())
    ref_rel = mo.error_metrics(ref_r, ref)[1]
    bar = max(MAX_ABS, ref_err)
    max_abs, rel = mo.error_metrics(got, ref)
    splits = ops.splits(cfg.E, cfg.H, cfg.I, T * cfg.k)
    print(f"PARITY {cfg.name.split(' T')[0]} T={T} S={splits}: max_abs={max_abs:.4e} rel_l2={rel:.4e} | "
          f"reference arithmetic vs fp32: max_abs={ref_err:.4e} rel_l2={ref_rel:.4e} | bar max_abs={bar:.4e}")
    assert max_abs <= bar and rel <= REL_L2, f"max_abs={max_abs:.3e} (bar {bar:.3e}) rel_l2={rel:.3e}"


@pytest.mark.parametrize("E,k,H,I,T", [
    (1, 1, 4096, 14336, 64),   # one Mixtral-8x7B expert (an 8-rank expert-parallel layer's share)
    (2, 1, 1024, 3584, 40),    # two small experts, fewer gate/up units than SMs
])
def test_few_experts_vs_oracle(E, k, H, I, T):
    """Layers with one or two experts (fewer gate/up units than SMs, a large down split-K)."""
    from ae_b200 import ops
    dev = torch.device("cuda", 0)
    g = torch.Generator(device=dev)
    g.manual_seed(E * 100 + T)
    pool = (torch.randn(E, 3 * I * H, generator=g, device=dev) * 0.02).to(torch.bfloat16)
    x = torch.randn(T, H, generator=g, device=dev).to(torch.bfloat16)
    logits = torch.randn(T, E, generator=g, device=dev).to(torch.bfloat16)
    pages = torch.arange(E, device=dev, dtype=torch.int64)
    ids = torch.empty(T, k, dtype=torch.int32, device=dev)
    out = ops.moe_forward(x, logits, pool, pages, k, True, topk_ids=ids)
    torch.cuda.synchronize()
    rw, rids = mo.select_experts(logits.cpu(), k, True)
    assert (ids.cpu().numpy() == rids).all()
    xc, pc = x.cpu(), pool.cpu()
    ref = mo.stack_fused_moe(xc, pc, pages.cpu(), rw, rids, rounding="fp32").float()
    ref_r = mo.stack_fused_moe(xc, pc, pages.cpu(), rw, rids, rounding="reference").float()
    bar = max(MAX_ABS, float((ref_r - ref).abs().max()))
    max_abs, rel = mo.error_metrics(out.float().cpu(), ref)
    S = ops.splits(E, H, I, T * k)
    print(f"PARITY E={E} H={H} I={I} T={T} S={S}: max_abs={max_abs:.4e} rel_l2={rel:.4e} bar={bar:.4e}")
    assert max_abs <= bar and rel <= REL_L2, (max_abs, bar, rel)


def test_prefill_sized_token_tiles_vs_oracle():
    """512 tokens per expert: two 256-token tiles per expert, each its own unit (TMA token
    tiles), down units per token tile."""
    from ae_b200 import ops
    E, k, H, I, T = 8, 2, 1024, 3584, 2048
    dev = torch.device("cuda", 0)
    g = torch.Generator(device=dev)
    g.manual_seed(2048)
    pool = (torch.randn(E, 3 * I * H, generator=g, device=dev) * 0.02).to(torch.bfloat16)
    x = torch.randn(T, H, generator=g, device=dev).to(torch.bfloat16)
    logits = (torch.randn(T, E, generator=g, device=dev) * 0.1).to(torch.bfloat16)
    pages = torch.arange(E, device=dev, dtype=torch.int64)
    ids = torch.empty(T, k, dtype=torch.int32, device=dev)
    out = ops.moe_forward(x, logits, pool, pages, k, True, topk_ids=ids)
    torch.cuda.synchronize()
    rw, rids = mo.select_experts(logits.cpu(), k, True)
    assert (ids.cpu().numpy() == rids).all()
    assert np.bincount(rids.reshape(-1), minlength=E).max() > 256  # several token tiles per expert
    xc, pc = x.cpu(), pool.cpu()
    ref = mo.stack_fused_moe(xc, pc, pages.cpu(), rw, rids, rounding="fp32").float()
    max_abs, rel = mo.error_metrics(out.float().cpu(), ref)
    print(f"PARITY prefill-sized E={E} H={H} I={I} T={T}: max_abs={max_abs:.4e} rel_l2={rel:.4e}")
    assert max_abs <= MAX_ABS and rel <= REL_L2, (max_abs, rel)


def test_device_timers_count_the_calls():
    """smb_moe_read_timers: the FFN kernel timer counts every launch on the workspace and the
    stage clock charges each stage of the route -> FFN -> combine chain once per call."""
    from ae_b200 import configs, ops
    dev = torch.device("cuda", 0)
    cfg = configs.BY_KEY["c1"]
    pool = configs.make_pool(cfg, dev, seed=0)
    pages = torch.arange(cfg.E, device=dev, dtype=torch.int64)
    x, logits = configs.make_inputs(cfg, dev, seed=0)
    ops.moe_forward(x, logits, pool, pages, cfg.k, True)
    ws = ops.Workspace.lookup(dev)
    ops.read_timers(ws, reset=True)
    for _ in range(4):
        ops.moe_forward(x, logits, pool, pages, cfg.k, True)
    tm = ops.read_timers(ws)
    assert tm["ffn_launches"] == 4 and tm["ffn_ns"] > 0
    # each stage is charged when the next one starts: route and FFN four times, the
    # combine three times (the fourth call's combine ends no stage yet)
    assert tm["stage_calls"]["route"] == 4 and tm["stage_calls"]["ffn"] == 4
    assert tm["stage_calls"]["combine"] == 3
    assert tm["stage_calls"]["reserved"] == 0 and tm["stage_calls"]["final_combine"] == 0
    ffn_stage = tm["stage_ns"]["ffn"] / 4
    ffn_kernel = tm["ffn_ns"] / 4
    assert ffn_kernel <= ffn_stage * 1.05 + 2000, (ffn_kernel, ffn_stage)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("T,E,k,H,I", [
    (1024, 8, 2, 256, 128),    # pair tiles wider than I and H (rows past them never stored)
    (1200, 6, 2, 512, 384),    # partial last token tiles of 256 (N a multiple of 32 < 256)
])
def test_cta_pair_path_vs_oracle(dtype, T, E, k, H, I):
    """Prefill-sized calls (>= 256 routed slots per expert) run on CTA pairs with the 2-SM
    MMA; checked against the fp32 oracle like the verify path."""
    from ae_b200 import ops
    dev = torch.device("cuda", 0)
    assert T * k >= 256 * E
    g = torch.Generator(device=dev)
    g.manual_seed(T + H)
    pool = (torch.randn(E + 2, 3 * I * H, generator=g, device=dev) * 0.05).to(dtype)
    x = torch.randn(T, H, generator=g, device=dev).to(dtype)
    logits = torch.randn(T, E, generator=g, device=dev).to(dtype)
    pages = torch.randperm(E + 2, generator=g, device=dev)[:E].to(torch.int64)
    ids = torch.empty(T, k, dtype=torch.int32, device=dev)
    out = ops.moe_forward(x, logits, pool, pages, k, True, topk_ids=ids)
    torch.cuda.synchronize()
    rw, rids = mo.select_experts(logits.cpu(), k, True)
    assert (ids.cpu().numpy() == rids).all()
    ref = mo.stack_fused_moe(x.cpu(), pool.cpu(), pages.cpu(), rw, rids, rounding="fp32").float()
    max_abs, rel = mo.error_metrics(out.float().cpu(), ref)
    print(f"PARITY pair path {dtype} T={T} E={E} H={H} I={I}: max_abs={max_abs:.4e} rel_l2={rel:.4e}")
    assert max_abs <= MAX_ABS and rel <= REL_L2, (max_abs, rel)
