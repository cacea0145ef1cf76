"""Property tests of the oracle's routing and permutation restatements (CPU, hypothesis):
the invariants the reference's contracts state, on random shapes and values including
ties and empty experts.  They pin the oracle beyond the fixed golden vectors."""
import numpy as np
import torch
from hypothesis import given, settings
from hypothesis import strategies as st

from oracle import moe_oracle as mo


@st.composite
def routing_case(draw):
    T = draw(st.integers(1, 40))
    E = draw(st.integers(1, 64))
    k = draw(st.integers(1, min(E, 8)))
    seed = draw(st.integers(0, 2 ** 31 - 1))
    # coarse values make ties frequent
    coarse = draw(st.booleans())
    g = np.random.default_rng(seed)
    logits = (g.integers(-3, 4, size=(T, E)) if coarse else g.standard_normal((T, E))).astype(np.float32)
    return logits, k


@settings(max_examples=150, deadline=None)
@given(routing_case(), st.booleans())
def test_select_experts_invariants(case, renorm):
    logits, k = case
    w, ids = mo.select_experts(torch.from_numpy(logits), k, renorm)
    T, E = logits.shape
    assert w.shape == (T, k) and ids.shape == (T, k)
    assert w.dtype == np.float32 and ids.dtype == np.int32
    for t in range(T):
        row = ids[t]
        assert len(set(row.tolist())) == k and row.min() >= 0 and row.max() < E
        chosen = logits[t, row]
        # the k largest logits, in descending order; among equal logits the lower index first
        assert np.all(np.diff(chosen) <= 0)
        rest = np.setdiff1d(np.arange(E), row)
        if rest.size:
            assert chosen.min() >= logits[t, rest].max()
            tied_rest = rest[logits[t, rest] == chosen.min()]
            tied_in = row[chosen == chosen.min()]
            if tied_rest.size:
                assert tied_in.max() < tied_rest.min()
        for a in range(k - 1):
            if chosen[a] == chosen[a + 1]:
                assert row[a] < row[a + 1]
        assert np.all(w[t] > 0)
        if renorm:
            assert abs(float(w[t].sum()) - 1.0) < 1e-5
        else:
            assert float(w[t].sum()) <= 1.0 + 1e-5


@settings(max_examples=150, deadline=None)
@given(st.integers(0, 60), st.integers(1, 32), st.integers(1, 8), st.integers(0, 2 ** 31 - 1))
def test_permutation_invariants(T, E, k, seed):
    g = np.random.default_rng(seed)
    ids = g.integers(0, E, size=(T, k)).astype(np.int32)
    perm, off, inv = mo.permutation(ids, E)
    flat = ids.reshape(-1)
    n = flat.size
    assert sorted(perm.tolist()) == list(range(n))            # a permutation of the flat slots
    assert off[0] == 0 and off[-1] == n and np.all(np.diff(off) >= 0)
    for e in range(E):
        seg = perm[off[e]:off[e + 1]]
        assert np.all(flat[seg] == e)                          # expert-major
        assert np.all(np.diff(seg) > 0)                        # ascending flat index inside
        assert off[e + 1] - off[e] == int((flat == e).sum())
    assert np.array_equal(inv[perm], np.arange(n))             # inv is the inverse


@settings(max_examples=100, deadline=None)
@given(st.integers(1, 40), st.integers(1, 16), st.integers(1, 4), st.sampled_from([1, 4, 16, 64]),
       st.integers(0, 2 ** 31 - 1))
def test_align_block_size_invariants(T, E, k, block, seed):
    g = np.random.default_rng(seed)
    ids = g.integers(0, E, size=(T, k)).astype(np.int32)
    s, e_ids, npad = mo.moe_align_block_size(ids, block, E)
    numel = T * k
    total = int(npad[0])
    assert total % block == 0 and total <= numel + E * (block - 1)
    perm, off, _ = mo.permutation(ids, E)
    # stripping the pad value leaves exactly the unpadded permutation
    assert np.array_equal(s[s != numel], perm)
    assert np.all(s[total:] == numel)
    pos = 0
    for e in range(E):
        cnt = int(off[e + 1] - off[e])
        nb = -(-cnt // block)
        assert np.all(e_ids[pos // block:pos // block + nb] == e)
        assert np.all(s[pos + cnt:pos + nb * block] == numel)   # each expert padded to a block multiple
        pos += nb * block
    assert pos == total and np.all(e_ids[total // block:] == -1)
