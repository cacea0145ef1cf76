"""Expert-parallel layer on 2 GPUs over NCCL (skipped with fewer than 2 GPUs).

Each rank runs its own tokens through ExpertParallelMoE (experts sharded 4 + 4); the
result is checked against the fp32 CPU oracle of the full layer on that rank's tokens.
"""
import os
import socket
import datetime

import pytest
import torch
import torch.multiprocessing as mp

from oracle import moe_oracle as mo

pytestmark = pytest.mark.gpu


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _worker(rank, world, port, q):
    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=dev)
    try:
        from ae_b200.ep import ExpertParallelMoE
        E, k, H, I = 8, 2, 256, 128
        T = [40, 23][rank]
        g = torch.Generator().manual_seed(7)
        full = (torch.randn(E, 3 * I * H, generator=g) * 0.05).to(torch.bfloat16)
        E_loc = E // world
        pool = full[rank * E_loc:(rank + 1) * E_loc].contiguous().to(dev)
        gx = torch.Generator().manual_seed(50 + rank)
        x = torch.randn(T, H, generator=gx).to(torch.bfloat16)
        logits = torch.randn(T, E, generator=gx).to(torch.bfloat16)
        moe = ExpertParallelMoE(E, k, H, I, pool, max_tokens=40)
        out = moe(x.to(dev), logits.to(dev))
        out2 = moe(x.to(dev), logits.to(dev))
        torch.cuda.synchronize()
        w, ids = mo.select_experts(logits, k, True)
        ref = mo.stack_fused_moe(x, full, torch.arange(E), w, ids, rounding="fp32")
        max_abs, rel = mo.error_metrics(out.float().cpu(), ref)
        same = bool(torch.equal(out, out2))
        q.put((rank, max_abs, rel, same))
        dist.barrier()
    finally:
        dist.destroy_process_group()


def test_expert_parallel_two_gpus():
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=240)
    for p in procs:
        if p.is_alive():
            p.kill()
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    for _ in range(2):
        rank, max_abs, rel, same = q.get(timeout=5)
        assert max_abs <= 2e-2 and rel <= 1e-2, (rank, max_abs, rel)
        assert same, f"rank {rank}: repeated call differs"
