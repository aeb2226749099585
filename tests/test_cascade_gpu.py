"""GPU parity of the shared-prefix cascade against the fp64 oracle.

Cases are the reference's (01_decode_attention.cu:782-815, seed 13, min_prefix 16), its
golden output for the first case, the unshared-batch fallback, and BASELINE config 3 at full
size (64 requests x (4096 shared + 256 private), and the ragged suffix variant) checked on
sampled sequences. Tolerance: out max-abs <= 2e-3 (north star), lse <= 2e-3 abs + 1e-3 rel
(the reference's cascade lse tolerance, 01_decode_attention.cu:808).
"""
import os

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

OUT_ATOL = 2e-3
LSE_ATOL, LSE_RTOL = 2e-3, 1e-3


def to_dev(bt, dev):
    import torch
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(dev)
    return dict(q=t(bt.q), k_cache=t(bt.k), v_cache=t(bt.v), kv_indptr=t(bt.indptr),
                kv_indices=t(bt.indices), kv_last_page_len=t(bt.last))


def check(out, lse, ref_o, ref_l, tag):
    o = out.float().cpu().numpy()
    l = lse.cpu().numpy()
    err = np.abs(o - ref_o).max()
    assert err <= OUT_ATOL, f"{tag}: out max-abs {err:.3e}"
    lerr = np.abs(l - ref_l)
    assert np.all(lerr <= LSE_ATOL + LSE_RTOL * np.abs(ref_l)), f"{tag}: lse {lerr.max():.3e}"


def run_cascade(ckl, bt, d, min_prefix):
    base = ckl.make_params(**d, num_chunks=1, chunk_tokens=16)
    cp = ckl.plan_cascade(base, bt.indptr, bt.indices, bt.lens, min_prefix)
    out, lse = ckl.cascade_decode(cp)
    return cp, out, lse


SCASES = [(64, [1, 17, 40], 8, 8), (48, [5, 300, 33, 16, 2], 32, 8),
          (1024, [77] * 40, 32, 8), (256, [100, 3], 16, 2)]


@pytest.mark.parametrize("Lp,suffix,Hq,Hkv", SCASES)
def test_reference_cascade_cases(ckl, oracle, dev, Lp, suffix, Hq, Hkv):
    bt = oracle.shared_prefix_batch(Lp, suffix, Hq, Hkv, 13)
    ref_o, ref_l = oracle.attention_ref(bt)
    cp, out, lse = run_cascade(ckl, bt, to_dev(bt, dev), 16)
    assert cp.use == 1 and cp.suffix.kv_start == Lp, "shared prefix not detected"
    assert cp.prefix_pages == Lp // 16
    check(out, lse, ref_o, ref_l, f"cascade Lp={Lp}")


def test_cascade_against_reference_golden(ckl, oracle, dev):
    g = np.load(os.path.join(os.path.dirname(__file__), "golden", "cascade_case1.npz"))
    bt = oracle.shared_prefix_batch(64, [1, 17, 40], 8, 8, 13)
    cp, out, lse = run_cascade(ckl, bt, to_dev(bt, dev), 16)
    assert cp.use == 1
    check(out, lse, g["out"], g["lse"], "golden cascade case 1")


def test_unshared_batch_falls_back_to_plain_decode(ckl, oracle, dev):
    bt = oracle.batch([1000] * 4, 32, 8, 3)
    assert ckl.shared_prefix_pages(bt.indptr, bt.indices) == 0
    ref_o, ref_l = oracle.attention_ref(bt)
    cp, out, lse = run_cascade(ckl, bt, to_dev(bt, dev), 256)
    assert cp.use == 0
    check(out, lse, ref_o, ref_l, "unshared")


def test_short_prefix_below_min_prefix_is_plain(ckl, oracle, dev):
    bt = oracle.shared_prefix_batch(64, [10, 20, 30], 32, 8, 5)
    ref_o, ref_l = oracle.attention_ref(bt)
    cp, out, lse = run_cascade(ckl, bt, to_dev(bt, dev), 256)
    assert cp.use == 0
    check(out, lse, ref_o, ref_l, "below min_prefix")


def test_cascade_matches_plain_decode_and_is_deterministic(ckl, oracle, dev):
    bt = oracle.shared_prefix_batch(1024, [77] * 40, 32, 8, 13)
    d = to_dev(bt, dev)
    _, o1, l1 = run_cascade(ckl, bt, d, 16)
    _, o2, l2 = run_cascade(ckl, bt, d, 16)
    assert bool((o1 == o2).all()) and bool((l1 == l2).all())
    po, pl = ckl.decode_attention(**d)
    assert float((o1.float() - po.float()).abs().max()) <= 2 * OUT_ATOL
    assert float((l1 - pl).abs().max()) <= 2 * LSE_ATOL


def _config3(ckl, oracle, dev, suffix, sample, seed=21):
    import torch
    Lp, Hq, Hkv = 4096, 32, 8
    bt = oracle.shared_prefix_batch(Lp, suffix, Hq, Hkv, seed, fill=False)
    g = torch.Generator(device=dev)
    g.manual_seed(seed)
    shape = (bt.num_pages, 16, Hkv, 128)
    k = (torch.rand(shape, generator=g, device=dev) * 2 - 1).half()
    v = (torch.rand(shape, generator=g, device=dev) * 2 - 1).half()
    q = (torch.rand((bt.B, Hq, 128), generator=g, device=dev) * 2 - 1).half()
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(dev)
    d = dict(q=q, k_cache=k, v_cache=v, kv_indptr=t(bt.indptr), kv_indices=t(bt.indices),
             kv_last_page_len=t(bt.last))
    cp, out, lse = run_cascade(ckl, bt, d, 256)
    assert cp.use == 1 and cp.prefix_len == Lp
    out, lse = out.float().cpu().numpy(), lse.cpu().numpy()
    for b in sample:
        pages = bt.indices[bt.indptr[b]:bt.indptr[b + 1]]
        pi = torch.from_numpy(pages.astype(np.int64)).to(dev)
        sb = oracle.Batch([bt.lens[b]], Hq, Hkv, np.array([0, len(pages)], np.int32),
                          np.arange(len(pages), dtype=np.int32), bt.last[b:b + 1],
                          q[b:b + 1].cpu().numpy(), k.index_select(0, pi).cpu().numpy(),
                          v.index_select(0, pi).cpu().numpy())
        ro, rl = oracle.attention_ref(sb)
        check_np(out[b], lse[b], ro[0], rl[0], f"config3 b={b}")


def check_np(o, l, ro, rl, tag):
    assert np.abs(o - ro).max() <= OUT_ATOL, tag
    assert np.all(np.abs(l - rl) <= LSE_ATOL + LSE_RTOL * np.abs(rl)), tag


def test_config3_uniform_suffix_sampled(ckl, oracle, dev):
    _config3(ckl, oracle, dev, [256] * 64, sample=(0, 31, 63))


def test_config3_ragged_suffix_sampled(ckl, oracle, dev):
    suffix = np.random.default_rng(77).integers(1, 1025, size=64)
    _config3(ckl, oracle, dev, suffix, sample=(0, 17, 63))


# ------------------------------------------------------------------ prefix-tree cascade
def run_tree(ckl, bt, d, min_prefix):
    base = ckl.make_params(**d, num_chunks=1, chunk_tokens=16)
    tp = ckl.plan_cascade_tree(base, bt.indptr, bt.indices, bt.lens, min_prefix)
    out, lse = ckl.cascade_tree_decode(tp)
    return tp, out, lse


# (segments in pages, sequences as (segment list, private tokens), Hq, Hkv): a system
# prompt under two documents, sequences outside every group, and a second unrelated tree
TREE_CASES = [
    ([8, 12, 6, 20],
     [([0, 1], 40), ([0, 1], 3), ([0, 1], 17), ([0, 2], 100), ([0, 2], 1), ([0], 70), ([], 300),
      ([3], 16), ([3], 9)], 32, 8),
    ([4, 16], [([0, 1], 5), ([0, 1], 50), ([0], 33), ([0], 1)], 16, 2),
    ([30], [([0], 1), ([0], 2), ([0], 700)], 8, 8),
]


@pytest.mark.parametrize("segments,seqs,Hq,Hkv", TREE_CASES)
def test_tree_cascade_against_oracle(ckl, oracle, dev, segments, seqs, Hq, Hkv):
    bt = oracle.prefix_tree_batch(segments, seqs, Hq, Hkv, 31)
    ref_o, ref_l = oracle.attention_ref(bt)
    tp, out, lse = run_tree(ckl, bt, to_dev(bt, dev), 16)
    want, _ = oracle.prefix_tree_ref(bt.indptr, bt.indices, 1)
    assert tp.use == 1 and tp.nodes == len(want)
    check(out, lse, ref_o, ref_l, f"tree {segments}")


def test_tree_cascade_min_prefix_and_fallback(ckl, oracle, dev):
    segments, seqs, Hq, Hkv = TREE_CASES[0]
    bt = oracle.prefix_tree_batch(segments, seqs, Hq, Hkv, 32)
    ref_o, ref_l = oracle.attention_ref(bt)
    d = to_dev(bt, dev)
    tp, out, lse = run_tree(ckl, bt, d, 256)        # 16 pages: only the 20-page segment and 0+1
    assert tp.use == 1 and tp.nodes == 2
    check(out, lse, ref_o, ref_l, "tree min_prefix 256")
    tp, out, lse = run_tree(ckl, bt, d, 1 << 20)    # nothing long enough: plain split-KV
    assert tp.use == 0
    check(out, lse, ref_o, ref_l, "tree fallback")
    bt = oracle.batch([1000] * 4, 32, 8, 3)
    tp, out, lse = run_tree(ckl, bt, to_dev(bt, dev), 16)
    assert tp.use == 0
    ref_o, ref_l = oracle.attention_ref(bt)
    check(out, lse, ref_o, ref_l, "tree unshared")


def test_tree_cascade_whole_batch_prefix_matches_cascade(ckl, oracle, dev):
    bt = oracle.shared_prefix_batch(1024, [77] * 40, 32, 8, 13)
    d = to_dev(bt, dev)
    tp, o1, l1 = run_tree(ckl, bt, d, 16)
    assert tp.use == 1 and tp.nodes == 1
    _, o2, l2 = run_tree(ckl, bt, d, 16)
    assert bool((o1 == o2).all()) and bool((l1 == l2).all()), "not deterministic"
    _, co, cl = run_cascade(ckl, bt, d, 16)
    assert float((o1.float() - co.float()).abs().max()) <= 2 * OUT_ATOL
    ref_o, ref_l = oracle.attention_ref(bt)
    check(o1, l1, ref_o, ref_l, "tree whole-batch prefix")


def tree_config(n_groups=4, per_group=16, system=1024, doc=4096, suffix=256):
    """Config-3-sized prefix tree: a system prompt shared by all sequences, one document per
    group of sequences, private suffixes (token counts)."""
    segments = [system // 16] + [doc // 16] * n_groups
    suffix = np.broadcast_to(np.asarray(suffix), (n_groups * per_group,))
    seqs = [([0, 1 + g], int(suffix[g * per_group + i]))
            for g in range(n_groups) for i in range(per_group)]
    return segments, seqs


def test_tree_config_sampled(ckl, oracle, dev):
    import torch
    Hq, Hkv = 32, 8
    segments, seqs = tree_config(suffix=np.random.default_rng(5).integers(1, 1025, size=64))
    bt = oracle.prefix_tree_batch(segments, seqs, Hq, Hkv, 41, fill=False)
    g = torch.Generator(device=dev)
    g.manual_seed(41)
    shape = (bt.num_pages, 16, Hkv, 128)
    k = (torch.rand(shape, generator=g, device=dev) * 2 - 1).half()
    v = (torch.rand(shape, generator=g, device=dev) * 2 - 1).half()
    q = (torch.rand((bt.B, Hq, 128), generator=g, device=dev) * 2 - 1).half()
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(dev)
    d = dict(q=q, k_cache=k, v_cache=v, kv_indptr=t(bt.indptr), kv_indices=t(bt.indices),
             kv_last_page_len=t(bt.last))
    tp, out, lse = run_tree(ckl, bt, d, 256)
    assert tp.use == 1 and tp.nodes == 5
    po, pl = ckl.decode_attention(**d)
    assert float((out.float() - po.float()).abs().max()) <= 2 * OUT_ATOL
    out, lse = out.float().cpu().numpy(), lse.cpu().numpy()
    for b in (0, 17, 40, 63):
        pages = bt.indices[bt.indptr[b]:bt.indptr[b + 1]]
        pi = torch.from_numpy(pages.astype(np.int64)).to(dev)
        sb = oracle.Batch([bt.lens[b]], Hq, Hkv, np.array([0, len(pages)], np.int32),
                          np.arange(len(pages), dtype=np.int32), bt.last[b:b + 1],
                          q[b:b + 1].cpu().numpy(), k.index_select(0, pi).cpu().numpy(),
                          v.index_select(0, pi).cpu().numpy())
        ro, rl = oracle.attention_ref(sb)
        check_np(out[b], lse[b], ro[0], rl[0], f"tree config b={b}")


def test_tree_prefix_alone_fills_each_members_node_slots(ckl, oracle, dev):
    """ckl_cascade_tree_prefix alone: every member row gets a finite partial in each of its
    nodes' chunk slots, and the merge of prefix + suffix slots (cascade_tree_decode) equals
    the oracle; G = 16 (Hq=32, Hkv=2) stacks 16 rows per sequence."""
    import torch
    segments, seqs = [10, 20], [([0, 1], 33), ([0, 1], 2), ([0], 70), ([0], 1), ([], 40)]
    bt = oracle.prefix_tree_batch(segments, seqs, 32, 2, 9)
    d = to_dev(bt, dev)
    base = ckl.make_params(**d, num_chunks=1, chunk_tokens=16)
    tp = ckl.plan_cascade_tree(base, bt.indptr, bt.indices, bt.lens, 16)
    assert tp.use == 1 and tp.nodes == 2
    sp = tp.suffix
    po = torch.full((sp.B * sp.Hq * sp.part_stride * 128,), float("nan"), device=dev)
    pl = torch.full((sp.B * sp.Hq * sp.part_stride,), float("nan"), device=dev)
    ckl.cascade_tree_prefix(tp, po, pl)
    torch.cuda.synchronize()
    ckl.check_device_error()
    pl = pl.view(sp.B, sp.Hq, sp.part_stride).cpu().numpy()
    want, start = oracle.prefix_tree_ref(bt.indptr, bt.indices, 1)
    for b in range(sp.B):
        n_prefix = int(start[b] > 0) + int(start[b] > 10)   # nodes on b's path
        # a member's prefix slots hold finite lse; the rest stay untouched (NaN)
        assert np.isfinite(pl[b, :, :1]).all() == (n_prefix > 0), b
    out, lse = ckl.cascade_tree_decode(tp)
    ref_o, ref_l = oracle.attention_ref(bt)
    check(out, lse, ref_o, ref_l, "tree G=16")
