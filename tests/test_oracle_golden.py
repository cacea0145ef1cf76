"""The CPU oracle pinned against the reference's own outputs (no GPU).

Golden vectors come from the reference's Triton ``fused_moe_kernel`` /
``stack_fused_moe`` (specmoe/layers/fused_moe_kernel.py:88-349) run by the Triton CPU
interpreter (tests/golden/make_golden.py); the permutation known-answer test is the
example in the ``moe_align_block_size`` docstring (fused_moe_kernel.py:41-54).
"""
import numpy as np
import pytest
import torch

from oracle import moe_oracle as mo
from tests.golden.make_golden import CASES, make_pool, pool_sha256

GOLDEN = np.load(__import__("os").path.join(__import__("os").path.dirname(__file__), "golden", "moe_golden.npz"))

KAT_IDS = np.array([[2, 3, 4], [1, 2, 4], [1, 3, 4], [1, 2, 3]], dtype=np.int32)
KAT_SORTED = np.array([3, 6, 9, 12, 0, 4, 10, 12, 1, 7, 11, 12, 2, 5, 8, 12], dtype=np.int32)


def test_kat_align_as_written():
    # ids 1..4 with E=5 (expert 0 empty -> no block); same vector as the docstring.
    s, eids, npost = mo.moe_align_block_size(KAT_IDS, 4, 5)
    assert npost[0] == 16
    assert (s[:16] == KAT_SORTED).all()
    assert (s[16:] == 12).all()
    assert list(eids[:4]) == [1, 2, 3, 4]


def test_kat_align_zero_based():
    s, eids, npost = mo.moe_align_block_size(KAT_IDS - 1, 4, 4)
    assert npost[0] == 16
    assert (s[:16] == KAT_SORTED).all()
    assert list(eids[:4]) == [0, 1, 2, 3]


def test_kat_unpadded_permutation():
    perm, off, inv = mo.permutation(KAT_IDS - 1, 4)
    assert list(perm) == [3, 6, 9, 0, 4, 10, 1, 7, 11, 2, 5, 8]
    assert list(off) == [0, 3, 6, 9, 12]
    assert (perm[inv] == np.arange(12)).all()
    assert (GOLDEN["kat/sorted"] == KAT_SORTED).all()


def test_select_experts_ties_go_low():
    lg = torch.zeros(3, 6)
    lg[1, 4] = 1.0
    w, ids = mo.select_experts(lg, 2, True)
    assert ids[0].tolist() == [0, 1]
    assert ids[1].tolist() == [4, 0]
    assert np.allclose(w[0], [0.5, 0.5])


@pytest.mark.parametrize("case", CASES, ids=[c[0] for c in CASES])
def test_oracle_matches_reference_kernel(case):
    name, T, H, I, E, k, P, pidx, dtype, seed, renorm, scale = case
    pool = make_pool(seed, P, 3 * I * H, dtype)
    assert pool_sha256(pool) == str(GOLDEN[name + "/pool_sha256"]), "pool regeneration drifted"
    x = torch.from_numpy(GOLDEN[name + "/x"]).to(getattr(torch, dtype))
    w, ids = mo.select_experts(torch.from_numpy(GOLDEN[name + "/logits"]), k, renorm)
    assert (ids == GOLDEN[name + "/topk_ids"]).all()
    assert (w == GOLDEN[name + "/topk_weights"]).all()
    ref = torch.from_numpy(GOLDEN[name + "/out"])
    got_r = mo.stack_fused_moe(x, pool, pidx, w, ids, rounding="reference").float()
    got_f = mo.stack_fused_moe(x, pool, pidx, w, ids, rounding="fp32")
    if dtype == "float16":
        # Same rounding points as the Triton path.  The accumulation order inside the
        # dot products differs, so an intermediate may round the other way: at least
        # 99% of outputs are bit-identical and the rest are a few fp16 ulps apart
        # (one per rounded slot).
        eps = torch.finfo(torch.float16).eps
        d = (got_r - ref).abs()
        assert (d == 0).float().mean() >= 0.99
        assert (d <= 2 * k * eps * ref.abs() + eps * 2.0 ** -4 * ref.abs().max()).all()
    # and the fp32 oracle is within the layer tolerance of the reference kernel
    # (fp32 inputs go through tl.dot's TF32 path in the reference)
    max_abs, rel = mo.error_metrics(ref, got_f)
    assert max_abs <= 2e-2 and rel <= 1e-2


def test_permutation_is_stable_and_complete():
    rng = np.random.default_rng(0)
    ids = rng.integers(0, 7, size=(50, 3)).astype(np.int32)
    perm, off, inv = mo.permutation(ids, 7)
    flat = ids.reshape(-1)
    assert sorted(perm.tolist()) == list(range(150))
    for e in range(7):
        seg = perm[off[e]:off[e + 1]]
        assert (flat[seg] == e).all()
        assert (np.diff(seg) > 0).all()


def test_gate_logits_oracle_rounds_once():
    """The gate restatement rounds the exact dot products once to the storage dtype."""
    g = torch.Generator().manual_seed(3)
    x = torch.randn(6, 256, generator=g).to(torch.bfloat16)
    w = (torch.randn(8, 256, generator=g) * 0.05).to(torch.bfloat16)
    got = mo.gate_logits(x, w)
    assert got.dtype == torch.bfloat16 and got.shape == (6, 8)
    exact = x.double() @ w.double().t()
    assert torch.equal(got, exact.to(torch.bfloat16))
    # fp32 accumulation in another order differs from the exact sum by far less than a bf16 ulp
    assert float((exact - (x.float() @ w.float().t()).double()).abs().max()) < 1e-4


@pytest.mark.parametrize("Is,I", [(320, 128), (256, 128), (64, 64), (5632, 1408)])
def test_shared_expert_pages_split_is_exact(Is, I):
    """A shared expert cut into ceil(Is/I) zero-padded pages of intermediate I gives the same
    FFN as the whole expert (SwiGLU is separable along the intermediate dimension)."""
    from ae_b200.ops import shared_expert_pages
    H = 128
    g = torch.Generator().manual_seed(Is)
    w1 = torch.randn(Is, H, generator=g) * 0.05
    w3 = torch.randn(Is, H, generator=g) * 0.05
    w2 = torch.randn(H, Is, generator=g) * 0.05
    x = torch.randn(9, H, generator=g)
    pages = shared_expert_pages(w1, w3, w2, I)
    assert pages.shape == (-(-Is // I), 3 * I * H)
    direct = mo.shared_expert_forward(x, w1, w3, w2)
    pieces = torch.zeros_like(direct)
    for p in pages:
        a, b, c = mo.page_views(p, H, I)
        pieces += (torch.nn.functional.silu(x @ a.t()) * (x @ b.t())) @ c.t()
    torch.testing.assert_close(pieces, direct, rtol=1e-4, atol=1e-5)
