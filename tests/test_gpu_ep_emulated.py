"""Expert-parallel layer with G ranks emulated on one GPU, through the NCCL-style entry
points (``smb_moe_ep_dispatch`` / ``smb_moe_ep_experts`` / ``smb_moe_ep_combine``).

Each emulated rank has its own backend (buffers, workspaces) and its E/G experts' pages;
the exchange is done by copying chunks between the ranks' buffers, in the layout the
all-to-all moves: source s's send chunk d becomes destination d's receive chunk s, and
destination d's output chunk s becomes source s's returned chunk d.  Every rank's output
is checked against the fp32 CPU oracle of the whole layer on that rank's tokens
(``oracle.stack_fused_moe``), its routing ids bit-exact.  The expert side exercises the
FFN kernel's exchange output (split-K fix-up units writing the returned rows), also at
the full Mixtral-8x7B expert size with one expert per rank (S = 9) and with S forced to
16 (two batches of loads per fix-up row).
"""

import pytest
import torch

from oracle import moe_oracle as mo

pytestmark = pytest.mark.gpu


def _emulate(G, E, k, H, I, tokens, pool_full, xs, logits, backs=None, C=None):
    from ae_b200.ep import CudaBackend
    dev = pool_full.device
    E_loc = E // G
    C = C or max(1, max(tokens)) * k
    if backs is None:
        backs = [CudaBackend(E, k, H, I, torch.bfloat16, dev) for _ in range(G)]
    sends, states = [], []
    for r in range(G):
        send, state = backs[r].dispatch(xs[r], logits[r], G, C)
        sends.append(send.clone())
        states.append(state)
    outs = []
    for d in range(G):
        recv = torch.cat([sends[s][d * (C + 1):(d + 1) * (C + 1)] for s in range(G)])
        pool = pool_full[d * E_loc:(d + 1) * E_loc].contiguous()
        pages = torch.arange(E_loc, device=dev, dtype=torch.int64)
        outs.append(backs[d].experts(recv, G, C, pool, pages, E_loc).clone())
    res = []
    for s in range(G):
        back = torch.cat([outs[d][s * C:(s + 1) * C] for d in range(G)])
        res.append(backs[s].combine(back, states[s], tokens[s], G, C).clone())
    torch.cuda.synchronize()
    return res


def _check(res, E, k, pool_full, xs, logits, bar_max_abs):
    pc = pool_full.cpu()
    pages = torch.arange(E)
    for r, out in enumerate(res):
        if xs[r].shape[0] == 0:
            assert out.shape[0] == 0
            continue
        w, ids = mo.select_experts(logits[r].cpu(), k, True)
        ref = mo.stack_fused_moe(xs[r].cpu(), pc, pages, w, ids, rounding="fp32").float()
        bar = bar_max_abs
        if bar is None:
            ref_r = mo.stack_fused_moe(xs[r].cpu(), pc, pages, w, ids, rounding="reference").float()
            bar = max(2e-2, float((ref_r - ref).abs().max()))
        max_abs, rel = mo.error_metrics(out.float().cpu(), ref)
        print(f"PARITY emulated rank {r}/{len(res)}: max_abs={max_abs:.4e} rel_l2={rel:.4e} bar={bar:.4e}")
        assert max_abs <= bar and rel <= 1e-2, (r, max_abs, bar, rel)


@pytest.mark.parametrize("G,split_k", [(2, None), (4, None), (8, None), (8, 16)])
def test_emulated_ranks_small_experts(G, split_k, monkeypatch):
    """Three calls on the same buffers (the expert side leaves its counters at zero for the
    next call), uneven token counts, a rank without tokens in the first call."""
    from ae_b200.ep import CudaBackend
    if split_k is not None:
        monkeypatch.setenv("SMB_SPLIT_K", str(split_k))
    E, k, H, I = 8, 2, 1024, 3584
    dev = torch.device("cuda", 0)
    g = torch.Generator(device=dev).manual_seed(11 * G)
    pool = (torch.randn(E, 3 * I * H, generator=g, device=dev) * 0.03).to(torch.bfloat16)
    backs = [CudaBackend(E, k, H, I, torch.bfloat16, dev) for _ in range(G)]
    for call in range(3):
        tokens = [24 - (5 * r + 3 * call) % 11 for r in range(G)]
        if call == 0 and G > 2:
            tokens[-1] = 0  # one rank without tokens
        xs = [torch.randn(t, H, generator=g, device=dev).to(torch.bfloat16) for t in tokens]
        logits = [torch.randn(t, E, generator=g, device=dev).to(torch.bfloat16) for t in tokens]
        res = _emulate(G, E, k, H, I, tokens, pool, xs, logits, backs=backs, C=24 * k)
        _check(res, E, k, pool, xs, logits, 2e-2)


@pytest.mark.parametrize("G", [2, 8])
def test_emulated_ranks_full_size_experts(G):
    """Mixtral-8x7B experts, 32 tokens per rank (the C2 T=256 layer over 8 ranks)."""
    from ae_b200 import configs
    cfg = configs.BY_KEY["c2-256"]
    dev = torch.device("cuda", 0)
    pool = configs.make_pool(cfg, dev, seed=0)
    tokens = [32] * G
    xs, logits = [], []
    for r in range(G):
        x, lg = configs.make_inputs(cfg, dev, seed=r, T=32)
        xs.append(x)
        logits.append(lg)
    res = _emulate(G, cfg.E, cfg.k, cfg.H, cfg.I, tokens, pool, xs, logits)
    _check(res, cfg.E, cfg.k, pool, xs, logits, None)


@pytest.mark.parametrize("T,k,H", [(37, 2, 1024), (300, 2, 4096), (5, 8, 512)])
def test_combine_rows_expert_major(T, k, H):
    """smb_moe_combine_rows (the same kernel as the exchange's final combine) on per-slot
    rows in expert-major order: out[t] = sum_j w[t, j] * rows[inv[t*k + j]], fp32 sums in
    slot order, checked against torch in fp32."""
    from ae_b200 import ops
    dev = torch.device("cuda", 0)
    E, I = 16, 256
    g = torch.Generator(device=dev).manual_seed(T * k)
    x = torch.randn(T, H, generator=g, device=dev).to(torch.bfloat16)
    logits = torch.randn(T, E, generator=g, device=dev).to(torch.bfloat16)
    L = ops.StagedLayer(T, E, k, H, I, torch.bfloat16, dev)
    L.route(logits, x, True)
    rows = torch.randn(T * k, H, generator=g, device=dev).to(torch.bfloat16)
    out = torch.empty(T, H, dtype=torch.bfloat16, device=dev)
    L.combine_rows(rows, out)
    torch.cuda.synchronize()
    v = L.views()
    inv = v["inv"].long()
    w = v["w"].float()
    ref = (rows.float()[inv].view(T, k, H) * w.view(T, k, 1)).sum(1)
    assert L.status() == 0
    torch.testing.assert_close(out.float(), ref, atol=2e-2, rtol=1e-2)


def test_emulated_ranks_prefill_sized_dispatch():
    """1250-1300 tokens per rank with H = 4096: a dispatch CTA's token rows no longer fit its
    shared-memory staging (more than 64 KB), so the rows are copied straight from global
    memory after the routing; the expert side then has 256-token tiles (TMA token tiles)."""
    from ae_b200.ep import CudaBackend
    E, k, H, I, G = 8, 2, 4096, 256, 2
    dev = torch.device("cuda", 0)
    g = torch.Generator(device=dev).manual_seed(1300)
    pool = (torch.randn(E, 3 * I * H, generator=g, device=dev) * 0.02).to(torch.bfloat16)
    tokens = [1300, 1250]
    xs = [torch.randn(t, H, generator=g, device=dev).to(torch.bfloat16) for t in tokens]
    logits = [torch.randn(t, E, generator=g, device=dev).to(torch.bfloat16) for t in tokens]
    backs = [CudaBackend(E, k, H, I, torch.bfloat16, dev) for _ in range(G)]
    res = _emulate(G, E, k, H, I, tokens, pool, xs, logits, backs=backs)
    _check(res, E, k, pool, xs, logits, 2e-2)
