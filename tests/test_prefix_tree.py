"""Host logic of the prefix-tree cascade: ckl_prefix_tree against the brute-force checker.

ckl_prefix_tree (csrc/cascade.cu) builds the compressed trie of a batch's page lists in
one sort and one stack pass; oracle.prefix_tree_ref enumerates every depth. Both keep a
node when its own run, from the nearest kept ancestor, holds >= min_pages pages. No GPU.
"""
import numpy as np
import pytest


def tree_of(ckl, indptr, indices, min_pages):
    perm, nodes, start = ckl.prefix_tree(indptr, indices, min_pages)
    B = len(indptr) - 1
    assert sorted(perm.tolist()) == list(range(B)), "perm is not a permutation"
    got = set()
    for i, (first, end, m0, m1, parent) in enumerate(nodes.tolist()):
        assert m1 - m0 >= 2 and end - first >= max(1, min_pages)
        members = frozenset(perm[m0:m1].tolist())
        if parent >= 0:
            assert parent < i, "parents come first"
            pf, pe, pm0, pm1, _ = nodes[parent].tolist()
            assert pm0 <= m0 and m1 <= pm1 and (pm0, pm1) != (m0, m1)
            assert pe == first, "a node begins where its kept parent ends"
        else:
            assert first == 0
        # every member really holds the run, and it is never a member's last page
        b0 = perm[m0]
        run = indices[indptr[b0] + first:indptr[b0] + end]
        for b in members:
            assert end <= indptr[b + 1] - indptr[b] - 1
            assert np.array_equal(indices[indptr[b] + first:indptr[b] + end], run)
        got.add((members, first, end))
    return got, start


def check(ckl, oracle, indptr, indices, min_pages=1):
    indptr = np.asarray(indptr, np.int32)
    indices = np.asarray(indices, np.int32)
    got, start = tree_of(ckl, indptr, indices, min_pages)
    want, want_start = oracle.prefix_tree_ref(indptr, indices, min_pages)
    assert got == want
    assert np.array_equal(start, want_start)
    return got


def table(lists):
    indptr = np.zeros(len(lists) + 1, np.int32)
    indptr[1:] = np.cumsum([len(pl) for pl in lists])
    return indptr, np.array([p for pl in lists for p in pl], np.int32)


def test_empty_and_single(ckl, oracle):
    assert check(ckl, oracle, [0], []) == set()
    assert check(ckl, oracle, [0, 5], [1, 2, 3, 4, 5]) == set()
    assert check(ckl, oracle, [0, 0, 0], []) == set()


def test_whole_batch_prefix_matches_shared_prefix_pages(ckl, oracle):
    bt = oracle.shared_prefix_batch(1024, [77, 5, 300, 16], 32, 8, 13, fill=False)
    P = ckl.shared_prefix_pages(bt.indptr, bt.indices)
    got = check(ckl, oracle, bt.indptr, bt.indices)
    assert (frozenset(range(4)), 0, P) in got


def test_nested_groups(ckl, oracle):
    # system prompt (pages 0-3) for all; document A (10-12) for b0..b2, B (20-21) for b3, b4
    lists = [[0, 1, 2, 3, 10, 11, 12, 100], [0, 1, 2, 3, 10, 11, 12, 101, 102],
             [0, 1, 2, 3, 10, 11, 12, 103], [0, 1, 2, 3, 20, 21, 104],
             [0, 1, 2, 3, 20, 21, 105, 106], [0, 1, 2, 3, 107], [50, 51, 108]]
    got = check(ckl, oracle, *table(lists))
    assert got == {(frozenset(range(6)), 0, 4), (frozenset({0, 1, 2}), 4, 7),
                   (frozenset({3, 4}), 4, 6)}
    # a 3-page minimum drops document B: its members start after the system prompt
    got = check(ckl, oracle, *table(lists), min_pages=3)
    assert got == {(frozenset(range(6)), 0, 4), (frozenset({0, 1, 2}), 4, 7)}
    # a 5-page minimum drops the system prompt: document A then covers pages 0-7
    got = check(ckl, oracle, *table(lists), min_pages=5)
    assert got == {(frozenset({0, 1, 2}), 0, 7), (frozenset({3, 4}), 0, 6)}


def test_identical_and_prefix_keys(ckl, oracle):
    lists = [[1, 2, 3, 9], [1, 2, 3, 8], [1, 2, 3, 4, 5, 7], [1, 2, 6], [1, 2, 3]]
    got = check(ckl, oracle, *table(lists))
    assert (frozenset({0, 1, 2}), 2, 3) in got and (frozenset({0, 1, 2, 3, 4}), 0, 2) in got


@pytest.mark.parametrize("seed", range(12))
def test_random_forests(ckl, oracle, seed):
    rng = np.random.default_rng(seed)
    # a random forest of runs: each sequence walks down from a root, extending or branching
    runs = {}
    lists = []
    nxt = 0
    for b in range(int(rng.integers(2, 40))):
        path, node = [], ()
        for _ in range(int(rng.integers(0, 4))):
            kids = runs.setdefault(node, [])
            if kids and rng.random() < 0.7:
                node = kids[int(rng.integers(len(kids)))]
            else:
                ln = int(rng.integers(1, 6))
                node = node + (tuple(range(nxt, nxt + ln)),)
                nxt += ln
                kids.append(node)
        for run in node:
            path += list(run)
        npriv = int(rng.integers(1, 4))
        lists.append(path + list(range(10_000 + nxt, 10_000 + nxt + npriv)))
        nxt += npriv
    for min_pages in (1, 2, 4, 7):
        check(ckl, oracle, *table(lists), min_pages=min_pages)


def test_bad_table_is_rejected(ckl):
    with pytest.raises(ckl.CklError):
        ckl.prefix_tree(np.array([0, 3, 2], np.int32), np.arange(3, dtype=np.int32))


def test_empty_batch_plans_are_no_ops(ckl):
    """Both cascade planners accept B = 0 (the decode call is then a no-op) without a GPU."""
    base = ckl.DecodeParams()
    base.B, base.Hq, base.Hkv, base.num_pages = 0, 32, 8, 4
    base.num_chunks, base.chunk_tokens, base.part_stride = 1, 16, 1
    base.sm_scale = 128 ** -0.5
    e = np.zeros(0, np.int32)
    cp = ckl.plan_cascade(base, np.zeros(1, np.int32), e, e)
    assert cp.use == 0 and cp.suffix.num_chunks == 1 and cp.suffix.part_stride == 1
    tp = ckl.plan_cascade_tree(base, np.zeros(1, np.int32), e, e)
    assert tp.use == 0 and tp.tables is None and tp.suffix.num_chunks == 1
