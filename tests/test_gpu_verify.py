"""The verify-step decoder (ae_b200/verify.py) on the GPU: with the library MoE (gate fused
into the routing launch) against the same decoder whose MoE blocks are a plain torch fp32
restatement (routing from the library gate's logits, so both take the same experts).
Bar: relative-L2 of the final logits <= 2e-2 after two bf16 layers."""
import pytest
import torch

pytestmark = pytest.mark.gpu


def torch_fp32_moe(dec):
    from ae_b200 import ops
    c = dec.cfg

    def moe(layer, h):
        L = dec.layers[layer]
        logits = ops.gate(h, L["gate"])
        p = torch.softmax(logits.float(), dim=-1)
        w, ids = torch.topk(p, c.k, dim=-1)
        w = w / w.sum(-1, keepdim=True)
        x = h.float()
        out = torch.zeros_like(x)
        for e in range(c.E):
            page = L["pool"][int(dec.pages[e])].float()
            w1 = page[: c.I * c.H].view(c.I, c.H)
            w3 = page[c.I * c.H: 2 * c.I * c.H].view(c.I, c.H)
            w2 = page[2 * c.I * c.H:].view(c.H, c.I)
            y = (torch.nn.functional.silu(x @ w1.t()) * (x @ w3.t())) @ w2.t()
            out += (w * (ids == e)).sum(-1, keepdim=True) * y
        h.copy_(out.to(h.dtype))
        return h
    return moe


def test_verify_decoder_library_moe_matches_fp32_moe():
    from ae_b200.verify import DecoderConfig, VerifyDecoder, accept_greedy, random_tree
    cfg = DecoderConfig(layers=2, H=512, I=256, E=8, k=2, heads=4, kv_heads=2, head_dim=128, vocab=1000)
    parents = random_tree(32, seed=2)
    g = torch.Generator(device="cuda").manual_seed(1)
    tokens = torch.randint(0, cfg.vocab, (2, 32), generator=g, device="cuda")
    ours = VerifyDecoder(cfg, batch=2, cache_len=64, max_draft=32, device="cuda", seed=7)
    ref = VerifyDecoder(cfg, batch=2, cache_len=64, max_draft=32, device="cuda", seed=7)
    ref.moe = torch_fp32_moe(ref)
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(cfg.layers)]
    a = ours.forward(tokens, parents, moe_events=ev)
    b = ref.forward(tokens, parents)
    torch.cuda.synchronize()
    rel = float((a.float() - b.float()).norm() / b.float().norm())
    assert rel <= 2e-2, rel
    assert all(s.elapsed_time(e) > 0 for s, e in ev)
    acc, n = accept_greedy(a, tokens, parents, a[:, 0])
    assert acc.shape == tokens.shape and n.shape == (2,)
