"""The verify-step decoder (ae_b200/verify.py) on CPU with a torch MoE: tree attention is
consistent with running each root-to-node path as a plain causal sequence, and the greedy
acceptance follows the tree.  No GPU needed (the MoE is injected)."""
import torch

from oracle import moe_oracle as mo


def _cfg():
    from ae_b200.verify import DecoderConfig
    return DecoderConfig(layers=2, H=64, I=32, E=4, k=2, heads=4, kv_heads=2, head_dim=16, vocab=50)


def _oracle_moe(dec):
    def moe(layer, h):
        L = dec.layers[layer]
        logits = mo.gate_logits(h, L["gate"])
        out, _, _ = mo.fused_moe_forward(h, logits.float(), L["pool"], dec.pages, dec.cfg.k, True)
        h.copy_(out.to(h.dtype))
        return h
    return moe


def _decoder(seed=0, cache_len=5, max_draft=12):
    from ae_b200.verify import VerifyDecoder
    dec = VerifyDecoder(_cfg(), batch=2, cache_len=cache_len, max_draft=max_draft, device="cpu",
                        dtype=torch.float32, seed=seed)
    dec.moe = _oracle_moe(dec)
    return dec


def test_tree_mask_and_depths():
    from ae_b200.verify import random_tree, tree_depths, tree_mask
    parents = [-1, -1, 0, 0, 1, 2, 2, 4]
    m = tree_mask(parents)
    assert m[5].nonzero().flatten().tolist() == [0, 2, 5]
    assert m[7].nonzero().flatten().tolist() == [1, 4, 7]
    assert tree_depths(parents) == [0, 0, 1, 1, 1, 2, 2, 2]
    t = random_tree(32, seed=1)
    assert len(t) == 32 and all(p < i for i, p in enumerate(t))


def test_tree_attention_matches_path_sequences():
    from ae_b200.verify import tree_mask
    parents = [-1, -1, 0, 0, 1, 2, 2, 4]
    g = torch.Generator().manual_seed(3)
    tokens = torch.randint(0, 50, (2, len(parents)), generator=g)
    tree_logits = _decoder().forward(tokens, parents)
    m = tree_mask(parents)
    for node in (3, 5, 6, 7):
        path = m[node].nonzero().flatten().tolist()   # ancestors then the node, ascending
        chain = [-1] + list(range(len(path) - 1))      # the path as a causal chain
        chain_logits = _decoder().forward(tokens[:, path], chain)
        torch.testing.assert_close(chain_logits[:, -1], tree_logits[:, node], rtol=1e-4, atol=1e-4)


def test_greedy_acceptance():
    from ae_b200.verify import accept_greedy
    parents = [-1, -1, 0, 1, 2]
    V = 10
    logits = torch.full((1, 5, V), -1.0)
    root = torch.full((1, V), -1.0)
    root[0, 7] = 1.0          # root predicts 7
    logits[0, 0, 3] = 1.0     # after token 0 comes 3
    logits[0, 2, 4] = 1.0     # after token 2 comes 4
    tokens = torch.tensor([[7, 8, 3, 1, 4]])
    acc, n = accept_greedy(logits, tokens, parents, root)
    assert acc[0].tolist() == [True, False, True, False, True]
    assert n.tolist() == [3]
