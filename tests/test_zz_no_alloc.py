"""smb_moe_forward_noalloc: the layer call for callers that cannot allocate device memory.

Such callers (a host whose allocator owns the HBM, a latency-critical path that may not
call cudaMalloc, a binding without a device allocator) pass only inputs and outputs; the
library runs on its own 64 MiB static device scratch.  These checks call the entry point
through the C ABI and compare it with smb_moe_forward (caller-provided workspace), within
the layer tolerance (max-abs <= 2e-2, relative-L2 <= 1e-2; in practice identical), on two
calls in a row with different batches, so stale scratch contents from the first call
would show in the second.  The file sorts last so a stop-at-first-failure run has already
run every other test.
"""
import ctypes

import pytest
import torch

pytestmark = pytest.mark.gpu

MAX_ABS, REL_L2 = 2e-2, 1e-2


def _batch(T, E, H, seed, dtype=torch.bfloat16):
    g = torch.Generator(device="cuda")
    g.manual_seed(seed)
    x = torch.randn(T, H, generator=g, device="cuda").to(dtype)
    logits = torch.randn(T, E, generator=g, device="cuda").to(dtype)
    return x, logits


def _noalloc(lib, x, logits, pool, pages, k, out, w, ids):
    T, H = x.shape
    E = logits.shape[1]
    I = pool.shape[1] // (3 * H)
    stream = torch.cuda.current_stream().cuda_stream
    return lib.smb_moe_forward_noalloc(x.data_ptr(), logits.data_ptr(), 1, pool.data_ptr(), pool.shape[0],
                                       pages.data_ptr(), 1, T, E, k, H, I, 1, out.data_ptr(), w.data_ptr(),
                                       ids.data_ptr(), ctypes.c_void_p(stream))


def _diff(a, b):
    d = (a.float() - b.float())
    return d.abs().max().item(), (d.norm() / b.float().norm().clamp_min(1e-30)).item()


def test_noalloc_matches_workspace_entry_point_two_calls():
    from ae_b200 import _native, ops
    lib = _native.load()
    E, k, H, I = 8, 2, 1024, 3584
    g = torch.Generator(device="cuda")
    g.manual_seed(123)
    pool = (torch.randn(E + 4, 3 * I * H, generator=g, device="cuda") * 0.02).to(torch.bfloat16)
    pages = torch.tensor([3, 0, 5, 1, 11, 7, 2, 9], dtype=torch.int64, device="cuda")
    for call, (T, seed) in enumerate([(96, 1), (33, 2)]):
        x, logits = _batch(T, E, H, seed)
        ref_w = torch.empty(T, k, dtype=torch.float32, device="cuda")
        ref_ids = torch.empty(T, k, dtype=torch.int32, device="cuda")
        ref = ops.moe_forward(x, logits, pool, pages, k, True, topk_weights=ref_w, topk_ids=ref_ids)
        out = torch.full_like(x, float("nan"))
        w = torch.empty_like(ref_w)
        ids = torch.empty_like(ref_ids)
        rc = _noalloc(lib, x, logits, pool, pages, k, out, w, ids)
        assert rc == 0, f"call {call}: {_native.strerror(rc)}"
        torch.cuda.synchronize()
        assert torch.equal(ids, ref_ids), f"call {call}: routing differs"
        max_abs, rel = _diff(out, ref)
        assert max_abs <= MAX_ABS and rel <= REL_L2, f"call {call}: max_abs={max_abs} rel={rel}"


def test_noalloc_rejects_sizes_beyond_its_scratch():
    from ae_b200 import _native
    lib = _native.load()
    E, k, H, I = 8, 2, 4096, 14336  # Mixtral-8x7B layer
    T = 1024                         # needs ~138 MiB of workspace
    x = torch.empty(T, H, dtype=torch.bfloat16, device="cuda")
    logits = torch.empty(T, E, dtype=torch.bfloat16, device="cuda")
    pool = torch.empty(1, 3 * I * H, dtype=torch.bfloat16, device="cuda")
    pages = torch.zeros(E, dtype=torch.int64, device="cuda")
    out = torch.empty_like(x)
    w = torch.empty(T, k, dtype=torch.float32, device="cuda")
    ids = torch.empty(T, k, dtype=torch.int32, device="cuda")
    rc = _noalloc(lib, x, logits, pool, pages, k, out, w, ids)
    assert rc == -12, _native.strerror(rc)  # SMB_ERR_SCRATCH_LIMIT
    assert "64 MiB" in _native.strerror(rc)
