"""GPU parity of the balanced split (ckl_decode_attention_balanced) against the fp64 oracle:
the reference's correctness cases (01_decode_attention.cu:750-776)
against the reference's golden output, every GQA group size, empty sequences, batches with
fewer pages than CTAs, runs that cross many short units, and the large config-2 shapes
checked against the chunked decode. Tolerances as for the chunked decode (out max-abs 2e-3,
lse 1e-4 abs + 1e-4 rel)."""
import os

import numpy as np
import pytest

from test_decode_gpu import CASES, check, to_dev

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("lens,Hq,Hkv", CASES)
def test_reference_cases(ckl, oracle, dev, lens, Hq, Hkv):
    bt = oracle.batch(lens, Hq, Hkv, 7)
    ref_o, ref_l = oracle.attention_ref(bt)
    out, lse = ckl.decode_attention_balanced(**to_dev(bt, dev))
    check(out, lse, ref_o, ref_l, f"balanced {lens} G={Hq // Hkv}")


def test_config1_against_reference_golden(ckl, oracle, dev):
    g = np.load(os.path.join(os.path.dirname(__file__), "golden", "attn_config1.npz"))
    bt = oracle.batch([1000, 777], 32, 8, 7)
    out, lse = ckl.decode_attention_balanced(**to_dev(bt, dev))
    check(out, lse, g["out"], g["lse"], "balanced config1")


@pytest.mark.parametrize("G", [1, 2, 4, 8, 16])
def test_group_sizes(ckl, oracle, dev, G):
    bt = oracle.batch([1, 15, 16, 17, 300], G * 2, 2, 11)
    ref_o, ref_l = oracle.attention_ref(bt)
    out, lse = ckl.decode_attention_balanced(**to_dev(bt, dev))
    check(out, lse, ref_o, ref_l, f"balanced G={G}")


@pytest.mark.parametrize("lens", [[0, 5, 40, 1], [0, 0, 3], [1] * 300, [20], [0] * 3 + [4096] + [0] * 2])
def test_empty_tiny_and_many_short_units(ckl, oracle, dev, lens):
    # [20]: 2 pages x 8 heads = 16 pages < one wave of CTAs; [1]*300: 2400 one-page units,
    # so one CTA's run crosses several units; empty sequences give out = 0, lse = -inf
    bt = oracle.batch(lens, 32, 8, 5)
    ref_o, ref_l = oracle.attention_ref(bt)
    out, lse = ckl.decode_attention_balanced(**to_dev(bt, dev))
    check(out, lse, ref_o, ref_l, f"balanced {lens[:6]}")


def test_ragged_against_oracle_sampled(ckl, oracle, dev):
    rng = np.random.default_rng(3)
    lens = rng.integers(1, 3000, size=40).tolist()
    bt = oracle.batch(lens, 32, 8, 13)
    rows = np.arange(0, 40 * 32, 7)
    ref_o, ref_l = oracle.attention_ref(bt, rows=rows)
    out, lse = ckl.decode_attention_balanced(**to_dev(bt, dev))
    o = out.float().cpu().numpy().reshape(-1, 128)[rows]
    assert np.abs(o - ref_o.reshape(-1, 128)[rows]).max() <= 2e-3


@pytest.mark.parametrize("shape", [(1, 32768), (8, 8192), (64, 1024)])
def test_config2_shapes_match_chunked_decode(ckl, dev, shape):
    import torch
    B, L = shape
    import bench as Bm
    d, _ = Bm.paged_batch([L] * B, dev, seed=9)
    ref, ref_lse = ckl.decode_attention(**d)
    out, lse = ckl.decode_attention_balanced(**d)
    torch.cuda.synchronize()
    ckl.check_device_error()
    assert float((out.float() - ref.float()).abs().max()) <= 2e-3
    assert float((lse - ref_lse).abs().max()) <= 1e-4
    again, _ = ckl.decode_attention_balanced(**d)
    assert torch.equal(again, out)                       # deterministic
