"""CPU tests: the oracle restatement is pinned against the reference itself.

Two anchors: (1) golden fixtures committed under tests/golden/ (made by
tests/golden/make_golden.py from the reference's own compiled host code and its published
results), which need nothing at run time; (2) when oracle/_ref was built here, a live
value-for-value comparison with the reference's generators and cpu_reference.
"""
import hashlib
import json
import os

import numpy as np
import pytest

GOLDEN = os.path.join(os.path.dirname(__file__), "golden")


def _sha(a):
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


def test_fp16_conversion_matches_numpy(oracle):
    rng = np.random.default_rng(0)
    x = np.concatenate([rng.uniform(-1, 1, 100000), rng.standard_normal(100000) * 1e-5,
                        rng.standard_normal(1000) * 7e4,
                        [0.0, -0.0, 65504.0, 65519.0, 65520.0, 2.0**-24, 2.0**-25, 3 * 2.0**-26,
                         np.inf, -np.inf]]).astype(np.float32)
    out = np.empty(x.size, np.uint16)
    oracle.lib().ora_f32_to_f16(oracle._p(x), oracle._p(out), x.size)
    assert np.array_equal(out, x.astype(np.float16).view(np.uint16))
    back = np.empty(x.size, np.float32)
    oracle.lib().ora_f16_to_f32(oracle._p(out), oracle._p(back), x.size)
    assert np.array_equal(back, out.view(np.float16).astype(np.float32))


def test_config1_generator_and_reference_golden(oracle):
    """Batch({1000,777}, Hq=32, Hkv=8, seed 7)."""
    g = np.load(os.path.join(GOLDEN, "attn_config1.npz"))
    bt = oracle.batch([1000, 777], 32, 8, 7)
    for name in ("indptr", "indices", "last", "q", "k", "v"):
        assert _sha(getattr(bt, name)) == str(g["sha_" + name]), name
    out, lse = oracle.attention_ref(bt)
    assert np.array_equal(out.view(np.uint32), g["out"].view(np.uint32))
    assert np.array_equal(lse.view(np.uint32), g["lse"].view(np.uint32))


def test_cascade_generator_golden(oracle):
    g = np.load(os.path.join(GOLDEN, "cascade_case1.npz"))
    bt = oracle.shared_prefix_batch(64, [1, 17, 40], 8, 8, 13)
    for name in ("indptr", "indices", "last", "q", "k", "v"):
        assert _sha(getattr(bt, name)) == str(g["sha_" + name]), name
    out, lse = oracle.attention_ref(bt)
    assert np.array_equal(out.view(np.uint32), g["out"].view(np.uint32))
    assert np.array_equal(lse.view(np.uint32), g["lse"].view(np.uint32))
    assert oracle.shared_prefix_pages(bt.indptr, bt.indices) == 4


def test_unshared_batch_known_answer(oracle):
    known = json.load(open(os.path.join(GOLDEN, "known_answers.json")))
    bt = oracle.batch([1000] * 4, 32, 8, 3, fill=False)
    assert oracle.shared_prefix_pages(bt.indptr, bt.indices) == \
        known["unshared_batch_4x1000_seed3_shared_pages"] == 0


def test_routing_reproduces_published_counts(oracle):
    """make_logits(T,E,9) + top-k routing reproduce results/moe_decode_counts.txt exactly
    (MSVC normal-draw order, the build that produced the published results)."""
    rows = json.load(open(os.path.join(GOLDEN, "moe_decode_counts.json")))["rows"]
    assert len(rows) == 5
    for r in rows:
        lg = oracle.make_logits(r["T"], r["E"], r["seed"], msvc_pair_order=True)
        ids, wts = oracle.route(lg, r["k"])
        counts, offsets, tiles, inv = oracle.permute(ids, r["E"])
        assert counts.tolist() == r["counts"], (r["T"], r["E"])
        assert np.allclose(wts.sum(1), 1.0)


def test_permute_is_stable_rank(oracle):
    rng = np.random.default_rng(1)
    ids = rng.integers(0, 16, size=(37, 4)).astype(np.int32)
    counts, offsets, tiles, inv = oracle.permute(ids, 16, bm=64)
    flat = ids.reshape(-1)
    assert np.array_equal(counts, np.bincount(flat, minlength=16))
    assert offsets[0] == 0 and offsets[-1] == flat.size
    order = np.argsort(flat, kind="stable")          # rank by (expert, token, slot)
    expect = np.empty_like(order)
    expect[order] = np.arange(flat.size)
    assert np.array_equal(inv, expect)
    assert np.array_equal(np.diff(tiles), (counts + 63) // 64)


def test_plan_chunks_restatement(oracle):
    # 01_decode_attention.cu:292-312 with 148 SMs x 2 resident blocks
    assert oracle.plan_chunks(1, 8, 32768, 0, 296) == (37, 896)
    assert oracle.plan_chunks(8, 8, 8192, 0, 296) == (4, 2048)
    assert oracle.plan_chunks(64, 8, 1024, 0, 296) == (1, 1024)
    assert oracle.plan_chunks(2, 8, 1000, 7, 296) == (7, 160)


def test_quantizers_roundtrip(oracle):
    W = oracle.normal((2, 256, 48), seed=3, std=0.02)
    codes, scales, zeros = oracle.quant_asym4(W)
    assert codes.max() <= 15 and zeros.max() <= 15
    Wq = oracle.dequant(codes, scales, zeros, 4)
    err = np.abs(Wq - W.astype(np.float32))
    # rounding to the grid costs at most half a step; rounding the zero point can leave a
    # group extreme up to half a step outside the 16-level grid, so clamping costs <= 1 step
    step = np.repeat(scales.astype(np.float32), 128, axis=1)
    assert np.all(err <= step + 1e-7)
    assert np.mean(err <= 0.5 * step + 1e-7) > 0.999
    c8, s8 = oracle.quant_sym(W, 8, group=256)
    W8 = oracle.dequant(c8, s8, None, 8, group=256)
    assert np.all(np.abs(W8 - W.astype(np.float32)) <= 0.5 * s8.astype(np.float32) + 1e-7)


@pytest.mark.skipif(not os.path.exists(os.path.join(os.path.dirname(__file__), "..", "oracle",
                                                    "_ref", "libref01.so")),
                    reason="reference not compiled here")
def test_live_reference_attention_cases(oracle):
    """The reference's four correctness cases (01_decode_attention.cu:750-755, seed 7) and
    four cascade cases (:782-787, seed 13): generators and cpu_reference agree bit for bit."""
    cases = [([1, 17, 1000], 8, 8), ([5, 300, 2049, 4096], 32, 8), ([33, 777], 16, 2),
             ([16, 32, 48, 4097], 4, 2)]
    for lens, Hq, Hkv in cases:
        a, b = oracle.batch(lens, Hq, Hkv, 7), oracle.ref_batch(lens, Hq, Hkv, 7)
        for n in ("indptr", "indices", "last", "q", "k", "v"):
            assert np.array_equal(getattr(a, n), getattr(b, n)), (lens, n)
        o1, l1 = oracle.attention_ref(a)
        o2, l2 = oracle.ref_cpu_reference(b)
        assert np.array_equal(o1, o2) and np.array_equal(l1, l2)
    scases = [(64, [1, 17, 40], 8, 8), (48, [5, 300, 33, 16, 2], 32, 8),
              (1024, [77] * 40, 32, 8), (256, [100, 3], 16, 2)]
    for Lp, suf, Hq, Hkv in scases:
        a = oracle.shared_prefix_batch(Lp, suf, Hq, Hkv, 13)
        b = oracle.ref_shared_prefix_batch(Lp, suf, Hq, Hkv, 13)
        for n in ("indptr", "indices", "last", "q", "k", "v"):
            assert np.array_equal(getattr(a, n), getattr(b, n)), (Lp, n)
        assert oracle.shared_prefix_pages(a.indptr, a.indices) == \
            oracle.ref01().ref01_shared_prefix_pages(oracle._p(b.indptr), oracle._p(b.indices), b.B)


@pytest.mark.skipif(not os.path.exists(os.path.join(os.path.dirname(__file__), "..", "oracle",
                                                    "_ref", "libref03.so")),
                    reason="reference not compiled here")
def test_live_reference_logits(oracle):
    for T, E, seed, dis in [(16, 64, 9, -1), (40, 8, 5, 3), (100, 8, 5, -1), (37, 16, 5, 3)]:
        assert np.array_equal(oracle.make_logits(T, E, seed, dis), oracle.ref_make_logits(T, E, seed, dis))
