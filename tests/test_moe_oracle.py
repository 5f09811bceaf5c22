"""The MoE routing oracle (oracle/moe_oracle.c) on the CPU: the reference has
no MoE forward, so these pin the oracle to independent numpy statements of
the same rules (stable sort by expert, top-k with lower-id ties, softmax over
the k, fma-ordered combine) and check the expert-parallel layout's
invariants."""
import numpy as np
import pytest


def test_sort_is_stable_argsort(oracle_mod):
    rng = np.random.default_rng(0)
    for P, E in [(0, 3), (1, 1), (100, 7), (5000, 256)]:
        ids = rng.integers(0, E, size=P).astype(np.int32)
        offs, srt, prow, bad = oracle_mod.moe_sort(ids, E)
        assert bad == 0
        assert np.array_equal(srt, np.argsort(ids, kind="stable"))
        assert np.array_equal(offs, np.concatenate([[0], np.cumsum(np.bincount(ids, minlength=E))]))
        assert np.array_equal(srt[prow], np.arange(P))


def test_sort_drops_bad_ids(oracle_mod):
    ids = np.array([2, -1, 2, 5, 0], dtype=np.int32)
    offs, srt, prow, bad = oracle_mod.moe_sort(ids, 3)
    assert bad == 2 and list(offs) == [0, 1, 1, 3] and list(srt) == [4, 0, 2]
    assert list(prow) == [1, -1, 2, -1, 0]


def test_topk_softmax(oracle_mod):
    rng = np.random.default_rng(1)
    l = rng.standard_normal((50, 64)).astype(np.float32)
    l[0, 10] = l[0, 20] = l[0, 30] = 9.0
    ids, w = oracle_mod.moe_topk_softmax(l, 5)
    order = np.lexsort((np.arange(64)[None].repeat(50, 0), -l), axis=1)[:, :5]
    assert np.array_equal(ids, order)
    assert list(ids[0, :3]) == [10, 20, 30]
    v = np.take_along_axis(l, ids, 1).astype(np.float64)
    ex = np.exp(v - v[:, :1])
    np.testing.assert_allclose(w, ex / ex.sum(1, keepdims=True), rtol=1e-6)


def test_combine_matches_float64(oracle_mod):
    rng = np.random.default_rng(2)
    T, k, H = 9, 3, 17
    Ys = rng.standard_normal((T * k, H)).astype(np.float32)
    prow = rng.permutation(T * k).astype(np.int32)
    prow[4] = -1
    w = rng.random((T, k)).astype(np.float32)
    got = oracle_mod.moe_combine(Ys, prow, w, T, k, H)
    want = np.zeros((T, H))
    for t in range(T):
        for j in range(k):
            if prow[t * k + j] >= 0:
                want[t] += float(w[t, j]) * Ys[prow[t * k + j]].astype(np.float64)
    np.testing.assert_allclose(got, want, rtol=1e-5, atol=1e-6)


@pytest.mark.parametrize("world", [1, 2, 4])
def test_ep_layout_partitions_pairs(oracle_mod, world):
    rng = np.random.default_rng(world)
    E, k = 8 * world, 3
    ids = [np.stack([rng.permutation(E)[:k] for _ in range(int(rng.integers(0, 20)))]).astype(np.int32)
           if True else None for _ in range(world)]
    ids = [i if i.size else np.zeros((0, k), np.int32) for i in ids]
    lay = oracle_mod.ep_layout(ids, E, world)
    seen = set()
    for d, L in enumerate(lay):
        assert L["loff"][0] == 0 and np.all(np.diff(L["loff"]) >= 0) and L["loff"][-1] == len(L["tags"])
        for s, i in L["tags"]:
            seen.add((s, i))
    assert seen == {(s, i) for s in range(world) for i in range(ids[s].size)}
