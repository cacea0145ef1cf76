"""GPU parity of the layer with a shared expert (``smb_moe_forward_shared``): routed top-k
experts plus one shared expert split into pseudo-experts of the routed intermediate size,
against the fp32 oracle that computes the shared expert directly.

Includes the fine-grained benchmark shape (H 2048, 60 routed experts of I 1408, top-4,
shared expert of I 5632, Zipf(1.1)-skewed router, T 128).  Bars: routing ids bit-exact;
hidden states max-abs <= 2e-2 and relative-L2 <= 1e-2 against the fp32 oracle.
"""
import pytest
import torch

from oracle import moe_oracle as mo

pytestmark = pytest.mark.gpu

MAX_ABS, REL_L2 = 2e-2, 1e-2


def run_case(T, E, k, H, I, Is, dtype, seed, logits=None, x=None, sigmoid_gate=True):
    from ae_b200 import ops
    g = torch.Generator(device="cuda")
    g.manual_seed(seed)
    if x is None:
        x = torch.randn(T, H, generator=g, device="cuda").to(dtype)
    if logits is None:
        logits = torch.randn(T, E, generator=g, device="cuda").to(dtype)
    pool_r = (torch.randn(E, 3 * I * H, generator=g, device="cuda") * 0.02).to(dtype)
    w1 = (torch.randn(Is, H, generator=g, device="cuda") * 0.02).to(dtype)
    w3 = (torch.randn(Is, H, generator=g, device="cuda") * 0.02).to(dtype)
    w2 = (torch.randn(H, Is, generator=g, device="cuda") * 0.02).to(dtype)
    shared = ops.shared_expert_pages(w1, w3, w2, I)
    n_shared = shared.shape[0]
    pool = torch.cat([pool_r, shared])
    # routed experts on shuffled pages, the shared pieces after them
    pages = torch.cat([torch.randperm(E, generator=g, device="cuda"),
                       torch.arange(E, E + n_shared, device="cuda")]).to(torch.int64)
    sw = None
    if sigmoid_gate:
        wsg = (torch.randn(H, generator=g, device="cuda") * 0.05).to(dtype)
        sw = torch.sigmoid(x.float() @ wsg.float()).contiguous()
    w = torch.empty(T, k, dtype=torch.float32, device="cuda")
    ids = torch.empty(T, k, dtype=torch.int32, device="cuda")
    out = ops.moe_forward_shared(x, logits, pool, pages, k, n_shared, sw, True, topk_weights=w, topk_ids=ids)
    torch.cuda.synchronize()
    rw, rids = mo.select_experts(logits.cpu(), k, True)
    assert (ids.cpu().numpy() == rids).all()
    routed = mo.stack_fused_moe(x.cpu(), pool.cpu(), pages[:E].cpu(), rw, rids, rounding="fp32")
    ref = routed + mo.shared_expert_forward(x.cpu(), w1.cpu(), w3.cpu(), w2.cpu(),
                                            None if sw is None else sw.cpu())
    max_abs, rel = mo.error_metrics(out.float().cpu(), ref)
    assert max_abs <= MAX_ABS and rel <= REL_L2, (max_abs, rel)
    return out


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("T,E,k,H,I,Is", [(37, 8, 2, 256, 128, 320), (5, 4, 1, 128, 64, 64), (64, 16, 4, 512, 192, 768)])
def test_shared_expert_small(dtype, T, E, k, H, I, Is):
    run_case(T, E, k, H, I, Is, dtype, seed=T + E + Is)


def test_shared_expert_weight_one():
    run_case(20, 8, 2, 256, 128, 256, torch.bfloat16, seed=4, sigmoid_gate=False)


def test_qwen2_moe_style_config():
    """H 2048, 60 routed experts (I 1408) top-4 + shared expert (I 5632 = 4 pieces), T 128,
    router logits with the Zipf(1.1) popularity bias of the benchmark configuration."""
    from ae_b200 import configs
    cfg = configs.BY_KEY["c3"]
    dev = torch.device("cuda", 0)
    x, logits = configs.make_inputs(cfg, dev, seed=3)
    counts = torch.bincount(torch.topk(logits.float(), cfg.k, dim=1).indices.flatten(), minlength=cfg.E)
    assert int(counts.max()) > 4 * int(counts.float().mean())  # skewed popularity
    run_case(cfg.T, cfg.E, cfg.k, cfg.H, cfg.I, cfg.shared_I, torch.bfloat16, seed=11, logits=logits, x=x)
