"""CPU-side checks of the C ABI library and the host logic (no GPU needed)."""
import os
import re

import pytest
import torch

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _declared_symbols():
    src = open(os.path.join(ROOT, "include", "ae_b200.h")).read()
    return sorted(set(re.findall(r"SMB_API\s+[\w\s\*]+?\b(smb_\w+)\s*\(", src)))


@pytest.fixture(scope="module")
def lib():
    from ae_b200 import build, _native
    build.build()
    return _native.load()


def test_library_exports_every_declared_symbol(lib):
    from ae_b200 import _native
    declared = _declared_symbols()
    assert len(declared) >= 14
    for name in declared:
        assert hasattr(lib, name), name
    # the ctypes signature table covers the header exactly
    assert sorted(_native.SIGNATURES) == declared


def test_error_strings_and_version(lib):
    from ae_b200 import _native
    assert lib.smb_version() >= 100
    for code in range(0, -12, -1):
        assert _native.strerror(code) != "unknown error"
    assert _native.strerror(-999) == "unknown error"


def test_argument_checks_without_gpu(lib):
    # size / dtype validation happens before any device call
    assert lib.smb_moe_align_block_size(None, 4, 0, 4, None, None, None, None) == -1
    assert lib.smb_moe_topk(None, 7, 1, 8, 2, 1, None, None, None) == -2
    assert lib.smb_moe_topk(None, 1, 1, 8, 9, 1, None, None, None) == -1
    assert lib.smb_moe_topk(None, 1, 0, 8, 2, 1, None, None, None) == 0  # T = 0: nothing to do
    assert lib.smb_moe_splits(8, 100, 3584, 64) == -1
    assert lib.smb_moe_gate(None, None, 7, 4, 8, 1024, None, None) == -2
    assert lib.smb_moe_gate(None, None, 1, 4, 8, 100, None, None) == -1
    assert lib.smb_moe_gate(None, None, 1, 4, 257, 1024, None, None) == -1
    assert lib.smb_moe_gate(None, None, 1, 0, 8, 1024, None, None) == 0   # T = 0: nothing to do
    assert lib.smb_moe_workspace_init(None, 1 << 20, None) == -8
    assert lib.smb_moe_workspace_init(16, 1 << 20, None) == -3            # not 256-byte aligned


def test_no_host_fallback_in_product_path():
    """The product package never imports the oracle."""
    pkg = os.path.join(ROOT, "ae_b200")
    for dirpath, _, files in os.walk(pkg):
        for f in files:
            if f.endswith(".py"):
                src = open(os.path.join(dirpath, f)).read()
                assert "oracle" not in src, f


def test_ops_refuse_cpu_tensors(lib):
    from ae_b200 import ops
    x = torch.zeros(4, 128, dtype=torch.bfloat16)
    with pytest.raises(ValueError):
        ops.moe_forward(x, torch.zeros(4, 8), torch.zeros(8, 3 * 64 * 128, dtype=torch.bfloat16),
                        torch.arange(8), 2)


def test_fusedmoe_weight_loader_layout_and_tp_slicing():
    from ae_b200.layers.FusedMoE import FusedMoE
    E, k, H, I = 3, 2, 8, 6
    moe = FusedMoE(E, k, H, I, params_dtype=torch.float32, tp_size=2)
    assert moe.intermediate_size_per_partition == 3
    w1 = torch.arange(I * H, dtype=torch.float32).view(I, H)
    w3 = 1000 + torch.arange(I * H, dtype=torch.float32).view(I, H)
    w2 = 5000 + torch.arange(H * I, dtype=torch.float32).view(H, I)
    moe.weight_loader(moe.ws, w1, "experts.1.w1.weight", "w1", 1)
    moe.weight_loader(moe.ws, w3, "experts.1.w3.weight", "w3", 1)
    moe.weight_loader(moe.ws, w2, "experts.1.w2.weight", "w2", 1)
    page = moe.ws.data[1]
    Ip = 3
    assert torch.equal(page[: Ip * H].view(Ip, H), w1[:Ip])       # rank 0 slice of rows
    assert torch.equal(page[Ip * H: 2 * Ip * H].view(Ip, H), w3[:Ip])
    assert torch.equal(page[2 * Ip * H:].view(H, Ip), w2[:, :Ip])  # rank 0 slice of columns
    m = FusedMoE.make_expert_params_mapping("w1", "w2", "w3", 2)
    assert m[0] == ("experts.ws", "experts.0.w1.weight", 0, "w1")
    assert len(m) == 6


def test_unsupported_options_raise():
    from ae_b200.layers.FusedMoE import FusedMoE
    with pytest.raises(NotImplementedError):
        FusedMoE(4, 2, 128, 64, torch.bfloat16, tp_size=1, quant_config=object())


def test_specmoe_shim_routes_reference_imports():
    """`from specmoe.layers.FusedMoE import FusedMoE` (mixtral.py:54) resolves to the drop-in."""
    import importlib
    import sys
    from ae_b200 import specmoe_shim
    from ae_b200.layers import FusedMoE as ours_mod
    from ae_b200.layers import fused_moe_kernel as ours_k
    saved = {k: sys.modules.get(k) for k in ("specmoe", "specmoe.layers", "specmoe.layers.FusedMoE",
                                            "specmoe.layers.fused_moe_kernel")}
    try:
        names = specmoe_shim.install()
        assert names == ["specmoe.layers.FusedMoE", "specmoe.layers.fused_moe_kernel"]
        mod = importlib.import_module("specmoe.layers.FusedMoE")
        assert mod.FusedMoE is ours_mod.FusedMoE
        from specmoe.layers.fused_moe_kernel import moe_align_block_size, stack_fused_moe  # noqa: F401
        assert stack_fused_moe is ours_k.stack_fused_moe
        assert specmoe_shim.installed()
    finally:
        for k, v in saved.items():
            if v is None:
                sys.modules.pop(k, None)
            else:
                sys.modules[k] = v


def test_page_streamer_needs_pinned_host_pages():
    from ae_b200.streaming import ExpertPageStreamer
    with pytest.raises(ValueError):
        ExpertPageStreamer(torch.zeros(2, 3 * 64 * 128, dtype=torch.bfloat16), 2, "cpu")


def test_exchange_arena_layout(lib):
    """Arena of the peer-memory transport: 1 KiB control + flag block, then recv [G][C+1][H]
    and back [G][C][H], each rounded up to 256 bytes; at most 8 ranks."""
    def up(v):
        return (v + 255) // 256 * 256
    for G, C, H in [(2, 64, 4096), (8, 64, 4096), (4, 17, 128)]:
        want = 1024 + up(G * (C + 1) * H * 2) + up(G * C * H * 2)
        assert lib.smb_ep_arena_bytes(G, C, H, 1) == want
    assert lib.smb_ep_arena_bytes(9, 64, 4096, 1) == 0
    assert lib.smb_ep_arena_bytes(2, 64, 4096, 7) == 0
    assert lib.smb_ep_ipc_alloc(0, None, None) == -8
    assert lib.smb_moe_page_copy(None, None, 16, None, 1, None) == -8
