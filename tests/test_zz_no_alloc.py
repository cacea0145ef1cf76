"""smb_moe_forward_noalloc: the layer call for callers that cannot allocate device memory.

Such callers (a host whose allocator owns the HBM, a latency-critical path that may not
call cudaMalloc, a binding without a device allocator) pass only inputs and outputs; the
library runs on its own 64 MiB static device scratch.  These checks call the entry point
through the C ABI on two calls in a row with different batches (stale scratch contents
from the first call would show in the second) and compare each with the fp32 CPU oracle
(max-abs <= 2e-2, relative-L2 <= 1e-2, routing ids bit-exact) and with smb_moe_forward
(caller-provided workspace, the same kernels: identical results); that a call leaves the
device's free memory unchanged; the size limit; and that the scratch's status word,
read with smb_moe_noalloc_read_status, reports a page id out of range.  The file sorts
last so a stop-at-first-failure run has already run every other test.
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


def test_noalloc_matches_oracle_and_workspace_entry_point_two_calls():
    from ae_b200 import _native, ops
    from oracle import moe_oracle as mo
    lib = _native.load()
    E, k, H, I = 8, 2, 1024, 3584
    g = torch.Generator(device="cuda")
    g.manual_seed(123)
    pool = (torch.randn(E + 4, 3 * I * H, generator=g, device="cuda") * 0.02).to(torch.bfloat16)
    pages = torch.tensor([3, 0, 5, 1, 11, 7, 2, 9], dtype=torch.int64, device="cuda")
    pool_cpu, pages_cpu = pool.cpu(), pages.cpu()
    for call, (T, seed) in enumerate([(96, 1), (33, 2)]):
        x, logits = _batch(T, E, H, seed)
        out = torch.full_like(x, float("nan"))
        w = torch.empty(T, k, dtype=torch.float32, device="cuda")
        ids = torch.empty(T, k, dtype=torch.int32, device="cuda")
        rc = _noalloc(lib, x, logits, pool, pages, k, out, w, ids)
        assert rc == 0, f"call {call}: {_native.strerror(rc)}"
        assert lib.smb_moe_noalloc_read_status(ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)) == 0
        rw, rids = mo.select_experts(logits.cpu(), k, True)
        assert (ids.cpu().numpy() == rids).all(), f"call {call}: routing ids differ from the oracle"
        ref = mo.stack_fused_moe(x.cpu(), pool_cpu, pages_cpu, rw, rids, rounding="fp32")
        max_abs, rel = mo.error_metrics(out.float().cpu(), ref)
        assert max_abs <= MAX_ABS and rel <= REL_L2, f"call {call}: max_abs={max_abs} rel={rel}"
        # the workspace entry point runs the same kernels: the same bits
        same = ops.moe_forward(x, logits, pool, pages, k, True)
        torch.cuda.synchronize()
        assert torch.equal(same, out), f"call {call}: differs from smb_moe_forward"


def test_noalloc_large_batches_two_calls():
    """Batches of 2048+ routed slots take the router over many CTAs, whose ticket and
    generation words live in the scratch's control block: two such calls in a row (and the
    smaller calls of the other tests before them, on the same scratch) against the oracle
    and against smb_moe_forward."""
    from ae_b200 import _native, ops
    from oracle import moe_oracle as mo
    lib = _native.load()
    E, k, H, I = 8, 2, 512, 256
    g = torch.Generator(device="cuda")
    g.manual_seed(77)
    pool = (torch.randn(E, 3 * I * H, generator=g, device="cuda") * 0.03).to(torch.bfloat16)
    pages = torch.arange(E, dtype=torch.int64, device="cuda")
    pool_cpu, pages_cpu = pool.cpu(), pages.cpu()
    for call, (T, seed) in enumerate([(1100, 3), (1700, 4)]):
        assert T * k >= 2048
        x, logits = _batch(T, E, H, seed)
        out = torch.full_like(x, float("nan"))
        w = torch.empty(T, k, dtype=torch.float32, device="cuda")
        ids = torch.empty(T, k, dtype=torch.int32, device="cuda")
        rc = _noalloc(lib, x, logits, pool, pages, k, out, w, ids)
        assert rc == 0, f"call {call}: {_native.strerror(rc)}"
        assert lib.smb_moe_noalloc_read_status(ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)) == 0
        rw, rids = mo.select_experts(logits.cpu(), k, True)
        assert (ids.cpu().numpy() == rids).all(), f"call {call}: routing ids differ from the oracle"
        ref = mo.stack_fused_moe(x.cpu(), pool_cpu, pages_cpu, rw, rids, rounding="fp32")
        max_abs, rel = mo.error_metrics(out.float().cpu(), ref)
        assert max_abs <= MAX_ABS and rel <= REL_L2, f"call {call}: max_abs={max_abs} rel={rel}"
        same = ops.moe_forward(x, logits, pool, pages, k, True)
        torch.cuda.synchronize()
        assert torch.equal(same, out), f"call {call}: differs from smb_moe_forward"


def test_noalloc_call_allocates_no_device_memory():
    from ae_b200 import _native
    lib = _native.load()
    E, k, H, I, T = 8, 2, 1024, 3584, 64
    g = torch.Generator(device="cuda")
    g.manual_seed(5)
    pool = (torch.randn(E, 3 * I * H, generator=g, device="cuda") * 0.02).to(torch.bfloat16)
    pages = torch.arange(E, dtype=torch.int64, device="cuda")
    x, logits = _batch(T, E, H, 6)
    out = torch.empty_like(x)
    w = torch.empty(T, k, dtype=torch.float32, device="cuda")
    ids = torch.empty(T, k, dtype=torch.int32, device="cuda")
    assert _noalloc(lib, x, logits, pool, pages, k, out, w, ids) == 0  # first call: address lookup
    torch.cuda.synchronize()
    free0, _ = torch.cuda.mem_get_info()
    for _ in range(3):
        assert _noalloc(lib, x, logits, pool, pages, k, out, w, ids) == 0
    torch.cuda.synchronize()
    free1, _ = torch.cuda.mem_get_info()
    assert free1 == free0, f"device free memory changed by {free0 - free1} bytes"


def test_noalloc_status_reports_bad_page():
    from ae_b200 import _native
    lib = _native.load()
    E, k, H, I, T = 4, 2, 128, 64, 16
    g = torch.Generator(device="cuda")
    g.manual_seed(3)
    pool = (torch.randn(E, 3 * I * H, generator=g, device="cuda") * 0.02).to(torch.bfloat16)
    x = torch.randn(T, H, generator=g, device="cuda").to(torch.bfloat16)
    logits = torch.zeros(T, E, dtype=torch.bfloat16, device="cuda")  # ties: experts 0 and 1 for every token
    out = torch.empty_like(x)
    w = torch.empty(T, k, dtype=torch.float32, device="cuda")
    ids = torch.empty(T, k, dtype=torch.int32, device="cuda")
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    bad = torch.tensor([0, 99, 2, 3], dtype=torch.int64, device="cuda")  # page of expert 1 out of range
    assert _noalloc(lib, x, logits, pool, bad, k, out, w, ids) == 0  # queued; the kernels skip the page
    assert lib.smb_moe_noalloc_read_status(stream) == -10  # SMB_ERR_BAD_PAGE
    good = torch.arange(E, dtype=torch.int64, device="cuda")
    assert _noalloc(lib, x, logits, pool, good, k, out, w, ids) == 0
    assert lib.smb_moe_noalloc_read_status(stream) == 0


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
