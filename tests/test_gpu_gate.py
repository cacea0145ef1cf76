"""GPU parity of the fused router gate (``MixtralMoE.gate`` + routing in one launch,
``smb_moe_gate`` / ``smb_moe_forward_gated``) against the CPU oracle.

Bars: the gate's logits equal the oracle's (fp64 dot products rounded once to the storage
dtype) except where the fp32 sum lands within its own rounding error of a rounding
boundary, which may move one logit by one unit in the last place (at most 1 % of the
logits); routing from the kernel's logits is bit-exact; hidden states max-abs <= 2e-2 and
relative-L2 <= 1e-2 against the fp32 oracle.
"""
import pytest
import torch

from oracle import moe_oracle as mo

pytestmark = pytest.mark.gpu

MAX_ABS, REL_L2 = 2e-2, 1e-2


def _gen(seed):
    g = torch.Generator(device="cuda")
    g.manual_seed(seed)
    return g


def _ulp(t: torch.Tensor) -> torch.Tensor:
    """Spacing of the storage dtype at |t| (fp32 result)."""
    f = t.float().abs()
    mant = 8 if t.dtype == torch.bfloat16 else 11
    e = torch.floor(torch.log2(torch.clamp(f, min=2.0 ** -14)))
    return torch.pow(2.0, e - (mant - 1))


def make_gated(T, E, H, I, dtype=torch.bfloat16, seed=0, gate_std=0.02):
    g = _gen(seed)
    x = torch.randn(T, H, generator=g, device="cuda").to(dtype)
    wg = (torch.randn(E, H, generator=g, device="cuda") * gate_std).to(dtype)
    pool = (torch.randn(E, 3 * I * H, generator=g, device="cuda") * 0.02).to(dtype)
    pages = torch.randperm(E, generator=g, device="cuda").to(torch.int64)
    return x, wg, pool, pages


def check_logits(got, x, wg):
    ref = mo.gate_logits(x.cpu(), wg.cpu())
    got = got.cpu()
    diff = (got.float() - ref.float()).abs()
    assert bool((diff <= _ulp(ref) * 1.0001).all()), f"logit off by more than one ulp: {diff.max()}"
    frac_exact = float((diff == 0).float().mean())
    assert frac_exact >= 0.99, f"only {frac_exact:.4f} of the logits round like the oracle's"


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("T,E,H", [(1, 8, 4096), (5, 8, 1024), (33, 60, 2048), (256, 8, 4096), (600, 16, 1024),
                                   (7, 256, 128)])
def test_gate_logits(dtype, T, E, H):
    from ae_b200 import ops
    x, wg, _, _ = make_gated(T, E, H, 64, dtype, seed=T + E)
    got = ops.gate(x, wg)
    torch.cuda.synchronize()
    check_logits(got, x, wg)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("T,E,k,H,I", [(32, 8, 2, 1024, 3584), (3, 8, 2, 256, 128), (128, 60, 4, 2048, 1408),
                                       (300, 8, 2, 512, 256)])
def test_forward_gated_matches_oracle(dtype, T, E, k, H, I):
    from ae_b200 import ops
    x, wg, pool, pages = make_gated(T, E, H, I, dtype, seed=3 * T + E)
    logits = torch.empty(T, E, dtype=dtype, device="cuda")
    w = torch.empty(T, k, dtype=torch.float32, device="cuda")
    ids = torch.empty(T, k, dtype=torch.int32, device="cuda")
    out = ops.moe_forward_gated(x, wg, pool, pages, k, True, router_logits=logits, topk_weights=w, topk_ids=ids)
    torch.cuda.synchronize()
    check_logits(logits, x, wg)
    # routing from the kernel's own logits: bit-exact ids
    rw, rids = mo.select_experts(logits.cpu(), k, True)
    assert (ids.cpu().numpy() == rids).all()
    torch.testing.assert_close(w.cpu(), torch.as_tensor(rw), rtol=2e-6, atol=1e-7)
    ref = mo.stack_fused_moe(x.cpu(), pool.cpu(), pages.cpu(), rw, rids, rounding="fp32")
    max_abs, rel = mo.error_metrics(out.float().cpu(), ref)
    assert max_abs <= MAX_ABS and rel <= REL_L2, (max_abs, rel)


def test_forward_gated_repeat_and_ticket_reset():
    """Repeated calls (ticket back at 0 after each) and a changed token count on the same
    workspace give identical results."""
    from ae_b200 import ops
    x, wg, pool, pages = make_gated(64, 8, 1024, 512, seed=5)
    a = ops.moe_forward_gated(x, wg, pool, pages, 2)
    b = ops.moe_forward_gated(x[:9], wg, pool, pages, 2)
    c = ops.moe_forward_gated(x, wg, pool, pages, 2)
    d = ops.moe_forward_gated(x[:9], wg, pool, pages, 2)
    torch.cuda.synchronize()
    assert torch.equal(a, c)
    assert torch.equal(b, d)
    assert torch.equal(a[:9], b) or mo.error_metrics(a[:9].float().cpu(), b.float().cpu())[0] < 1e-2
    ws = ops.Workspace.get(x.device, 1)
    assert int(ws[4:8].view(torch.int32).item()) == 0


def test_forward_gated_cuda_graph():
    from ae_b200 import ops
    x, wg, pool, pages = make_gated(16, 8, 1024, 512, seed=9)
    eager = ops.moe_forward_gated(x, wg, pool, pages, 2)
    out = torch.empty_like(x)
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        ops.moe_forward_gated(x, wg, pool, pages, 2, out=out)
    torch.cuda.current_stream().wait_stream(s)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=s):
        ops.moe_forward_gated(x, wg, pool, pages, 2, out=out)
    out.zero_()
    g.replay()
    g.replay()
    torch.cuda.synchronize()
    assert torch.equal(out, eager)


def test_mixtral_moe_module_drop_in():
    """MixtralMoE built like specmoe/models/mixtral.py:68-104, weights through the
    reference's loader entry points, forward in place on a 3-D view."""
    from ae_b200.layers.mixtral_moe import MixtralMoE
    E, k, H, I, T = 8, 2, 512, 256, 24
    g = torch.Generator().manual_seed(21)
    w1 = [(torch.randn(I, H, generator=g) * 0.02).to(torch.bfloat16) for _ in range(E)]
    w3 = [(torch.randn(I, H, generator=g) * 0.02).to(torch.bfloat16) for _ in range(E)]
    w2 = [(torch.randn(H, I, generator=g) * 0.02).to(torch.bfloat16) for _ in range(E)]
    wg = (torch.randn(E, H, generator=g) * 0.05).to(torch.bfloat16)
    x = torch.randn(2, T // 2, H, generator=g).to(torch.bfloat16)
    moe = MixtralMoE(E, k, H, I, params_dtype=torch.bfloat16, tp_size=1)
    moe.gate.weight.weight_loader(moe.gate.weight, wg)
    for e in range(E):
        moe.experts.weight_loader(moe.experts.ws, w1[e], f"experts.{e}.w1.weight", "w1", e)
        moe.experts.weight_loader(moe.experts.ws, w3[e], f"experts.{e}.w3.weight", "w3", e)
        moe.experts.weight_loader(moe.experts.ws, w2[e], f"experts.{e}.w2.weight", "w2", e)
    moe = moe.cuda()
    moe.experts.ws.gpu_cache = moe.experts.ws.data
    mapping = torch.arange(E, dtype=torch.int64, device="cuda")
    hx = x.cuda()
    out = moe(hx, mapping)
    torch.cuda.synchronize()
    assert out.shape == x.shape and out.data_ptr() == hx.data_ptr()
    # reference routing from the module's own gate output (recomputed from the original x)
    logits_gpu, bias = moe.gate(x.view(-1, H).cuda())
    assert bias is None
    check_logits(logits_gpu, x.view(-1, H), wg)
    pool = torch.stack([mo.pack_page(w1[e], w3[e], w2[e]) for e in range(E)])
    rw, rids = mo.select_experts(logits_gpu.cpu(), k, True)
    ref = mo.stack_fused_moe(x.view(-1, H), pool, torch.arange(E), rw, rids, rounding="fp32")
    max_abs, rel = mo.error_metrics(out.view(-1, H).float().cpu(), ref)
    assert max_abs <= MAX_ABS and rel <= REL_L2, (max_abs, rel)
