"""GPU parity against the reference's OWN GPU kernels (built from its unmodified sources for
sm_100a into oracle/_ref): the same inputs through the reference's decode_attention
(01_decode_attention.cu:316-331), cascade_decode (01:703-712) and QuantWeights::run
(03_moe_wq_decode.cu:318-332) and through this library. A second pin besides the fp64 oracle;
the rows are those of tests/ref_gpu_compare.py, untimed.
"""
import os

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

REF = os.path.join(os.path.dirname(__file__), "..", "oracle", "_ref")
need_ref = pytest.mark.skipif(not (os.path.exists(os.path.join(REF, "libref01.so")) and
                                   os.path.exists(os.path.join(REF, "libref03.so"))),
                              reason="reference not compiled here")


@need_ref
@pytest.mark.parametrize("name", ["64x1024", "1x32768"])
def test_decode_matches_reference_gpu_kernel(ckl, oracle, dev, name):
    import bench
    from ref_gpu_compare import decode_row
    row = decode_row(ckl, oracle, bench, dev, None, name, timed=False)
    assert row["max_abs_diff"] <= 2e-3, row


@need_ref
def test_cascade_matches_reference_gpu_kernel(ckl, oracle, dev):
    import bench
    from ref_gpu_compare import cascade_row
    row = cascade_row(ckl, oracle, bench, dev, None, np.full(64, 256), timed=False)
    assert row["max_abs_diff"] <= 2e-3, row


@need_ref
@pytest.mark.parametrize("T", [1, 16])
def test_int4_gemm_matches_reference_gpu_kernel(ckl, oracle, dev, T):
    from ref_gpu_compare import gemm_row
    row = gemm_row(ckl, oracle, dev, None, T, timed=False)
    assert row["max_abs_diff"] <= 1e-2, row
