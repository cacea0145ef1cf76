"""Expert-parallel exchange logic on CPU: 2 and 4 gloo ranks, compute steps done by the
CPU oracle, result compared with the single-process oracle layer (no GPU needed).

Covers uneven per-rank token counts (including a rank with no tokens), experts that
receive nothing, and the exact split bookkeeping of the count and row all-to-alls.
"""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from oracle import moe_oracle as mo


class OracleBackend:
    """The three compute steps of ae_b200.ep.CudaBackend, restated on the CPU, with the same
    exchange layout: G chunks of [1 header row of int32 counts | C payload rows]."""

    def __init__(self, E, k, H, I, renormalize=True):
        self.E, self.k, self.H, self.I = E, k, H, I
        self.renormalize = renormalize

    def dispatch(self, x, logits, G, C):
        T = x.shape[0]
        E_loc = self.E // G
        send = torch.zeros(G * (C + 1), self.H)
        w, ids = mo.select_experts(logits, self.k, self.renormalize)
        perm, off, inv = mo.permutation(ids, self.E)
        for d in range(G):
            hdr = send[d * (C + 1)].view(torch.int32)
            for el in range(E_loc):
                e = d * E_loc + el
                hdr[el] = int(off[e + 1] - off[e])
            for p in range(off[d * E_loc], off[(d + 1) * E_loc]):
                send[d * (C + 1) + 1 + p - off[d * E_loc]] = x[int(perm[p]) // self.k]
        return send, (w, ids, inv, off)

    def experts(self, recv, G, C, pool, pages, num_local):
        out = torch.zeros(G * C, self.H)
        for s in range(G):
            counts = recv[s * (C + 1)].view(torch.int32)[:num_local].tolist()
            i = 0
            for el, c in enumerate(counts):
                w1, w3, w2 = mo.page_views(pool[int(pages[el])], self.H, self.I)
                for _ in range(c):
                    row = recv[s * (C + 1) + 1 + i]
                    out[s * C + i] = w2 @ (torch.nn.functional.silu(w1 @ row) * (w3 @ row))
                    i += 1
        return out

    def combine(self, back, state, T, G, C):
        w, ids, inv, off = state
        E_loc = self.E // G
        out = torch.zeros(T, self.H)
        for t in range(T):
            for j in range(self.k):
                f = t * self.k + j
                d = int(ids[t, j]) // E_loc
                out[t] += float(w[t, j]) * back[d * C + int(inv[f]) - int(off[d * E_loc])]
        return out


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _worker(rank, world, port, tokens, E, k, H, I, q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from ae_b200.ep import ExpertParallelMoE
        g = torch.Generator().manual_seed(1234)
        full_pool = torch.randn(E, 3 * I * H, generator=g) * 0.3
        E_loc = E // world
        pool = full_pool[rank * E_loc:(rank + 1) * E_loc].clone()
        T = tokens[rank]
        gx = torch.Generator().manual_seed(100 + rank)
        x = torch.randn(T, H, generator=gx)
        logits = torch.randn(T, E, generator=gx) * 2
        if T > 0 and rank == 0:
            logits[:, E - 1] -= 100.0  # last expert never chosen by rank 0's tokens
        moe = ExpertParallelMoE(E, k, H, I, pool, max_tokens=max(tokens), backend=OracleBackend(E, k, H, I))
        out = moe(x, logits)
        if T > 0:
            w, ids = mo.select_experts(logits, k, True)
            ref = mo.stack_fused_moe(x, full_pool, torch.arange(E), w, ids, rounding="fp32")
            err = float((out - ref).abs().max())
        else:
            err = 0.0 if out.shape == (0, H) else 1.0
        q.put((rank, err))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world,tokens", [(2, [7, 5]), (2, [0, 9]), (4, [6, 3, 0, 11])])
def test_expert_parallel_matches_single_process(world, tokens):
    E, k, H, I = 8, 2, 16, 8
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, tokens, E, k, H, I, q)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=180)
    for p in procs:
        if p.is_alive():
            p.kill()
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    res = dict(q.get(timeout=5) for _ in range(world))
    for r in range(world):
        assert res[r] < 1e-4, (r, res[r])


def _single_rank_group():
    if not dist.is_initialized():
        os.environ["MASTER_ADDR"] = "127.0.0.1"
        os.environ["MASTER_PORT"] = str(_free_port())
        dist.init_process_group("gloo", rank=0, world_size=1)


def test_expert_parallel_argument_checks():
    """Checks that run before any device work: transport names, a backend with the p2p
    transport, experts that do not shard over the ranks, pool shapes, too many tokens."""
    from ae_b200.ep import ExpertParallelMoE
    _single_rank_group()
    E, k, H, I = 4, 2, 16, 8
    pool = torch.zeros(E, 3 * I * H)
    with pytest.raises(ValueError):
        ExpertParallelMoE(E, k, H, I, pool, max_tokens=4, transport="tcp")
    with pytest.raises(ValueError):
        ExpertParallelMoE(E, k, H, I, pool, max_tokens=4, transport="p2p", backend=OracleBackend(E, k, H, I))
    with pytest.raises(ValueError):
        ExpertParallelMoE(E, k, H, I, torch.zeros(E, 3 * I * H + 1), max_tokens=4, backend=OracleBackend(E, k, H, I))
    moe = ExpertParallelMoE(E, k, H, I, pool, max_tokens=4, backend=OracleBackend(E, k, H, I))
    with pytest.raises(ValueError):
        moe(torch.zeros(5, H), torch.zeros(5, E))
    out = moe(torch.zeros(3, H), torch.zeros(3, E))
    assert out.shape == (3, H)
