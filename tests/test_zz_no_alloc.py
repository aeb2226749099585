"""GPU test of ckl_decode_attention_noalloc.

Some hosts cannot give this library device memory: a plugin whose host process has already
reserved the GPU's memory in its own pool, or a decode loop that may not call cudaMalloc or
cudaFree because those calls can synchronise the device. ckl_decode_attention_noalloc serves
them with a scratch array compiled into the library instead of a caller workspace.

Through the C ABI, two calls in a row (different batches and split plans, so the second call
runs on scratch that still holds the first call's partials) must match
ckl_decode_attention with a caller workspace within the parity tolerance of the decode tests,
and a launch that needs more scratch than the built-in array must be refused on the host.
This file is collected last so that a run stopping at its first failure has already run
every other test.
"""
import ctypes as C

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

OUT_ATOL = 2e-3                 # same tolerances as tests/test_decode_gpu.py
LSE_ATOL, LSE_RTOL = 1e-4, 1e-4


def _device_batch(oracle, dev, lens, Hq, Hkv, seed):
    import torch
    bt = oracle.batch(lens, Hq, Hkv, seed)
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(dev)
    return dict(q=t(bt.q), k_cache=t(bt.k), v_cache=t(bt.v), kv_indptr=t(bt.indptr),
                kv_indices=t(bt.indices), kv_last_page_len=t(bt.last))


def _noalloc_vs_workspace(ckl, d, force):
    import torch
    B, Hq, _ = d["q"].shape
    Hkv = d["k_cache"].shape[2]
    lens_max = int(((d["kv_indptr"][1:] - d["kv_indptr"][:-1] - 1) * 16 +
                    d["kv_last_page_len"]).max())
    nc, ct = ckl.plan_chunks(Hq // Hkv, B, Hkv, lens_max, force_chunks=force)
    assert nc > 1, "the plan must split so that the scratch is used"
    p = ckl.make_params(**d, num_chunks=nc, chunk_tokens=ct)
    assert 0 < ckl.workspace_size(p) <= ckl.NOALLOC_SCRATCH_BYTES

    # the existing entry point, with a caller-allocated workspace
    want_o, want_l = ckl.decode_attention(**d, num_chunks=nc, chunk_tokens=ct)

    out = torch.full_like(d["q"], float("nan"))
    lse = torch.full((B, Hq), float("nan"), dtype=torch.float32, device=d["q"].device)
    st = ckl.lib().ckl_decode_attention_noalloc(
        C.byref(p), C.c_void_p(out.data_ptr()), C.c_void_p(lse.data_ptr()),
        C.c_void_p(torch.cuda.current_stream().cuda_stream))
    assert st == 0, ckl.lib().ckl_last_error_string()
    torch.cuda.synchronize()
    ckl.check_device_error()

    o, wo = out.float().cpu().numpy(), want_o.float().cpu().numpy()
    l, wl = lse.cpu().numpy(), want_l.cpu().numpy()
    assert np.isfinite(o).all()
    assert np.abs(o - wo).max() <= OUT_ATOL
    fin = np.isfinite(wl)
    assert np.array_equal(fin, np.isfinite(l))
    assert np.all(np.abs(l[fin] - wl[fin]) <= LSE_ATOL + LSE_RTOL * np.abs(wl[fin]))


def test_noalloc_matches_workspace_entry_point_twice(ckl, oracle, dev):
    d1 = _device_batch(oracle, dev, [5, 300, 2049, 4096], 32, 8, 7)
    _noalloc_vs_workspace(ckl, d1, force=7)
    d2 = _device_batch(oracle, dev, [33, 777, 1000], 16, 2, 9)
    _noalloc_vs_workspace(ckl, d2, force=3)


def test_noalloc_refuses_launches_beyond_the_scratch(ckl, dev):
    import torch
    B, Hq, Hkv = 1024, 32, 8
    q = torch.zeros((B, Hq, 128), dtype=torch.float16, device=dev)
    kv = torch.zeros((1, 16, Hkv, 128), dtype=torch.float16, device=dev)
    ip = torch.zeros(B + 1, dtype=torch.int32, device=dev)
    ix = torch.zeros(1, dtype=torch.int32, device=dev)
    last = torch.ones(B, dtype=torch.int32, device=dev)
    p = ckl.make_params(q, kv, kv, ip, ix, last, num_chunks=16, chunk_tokens=256)
    assert ckl.workspace_size(p) > ckl.NOALLOC_SCRATCH_BYTES
    out = torch.empty_like(q)
    lse = torch.empty((B, Hq), dtype=torch.float32, device=dev)
    st = ckl.lib().ckl_decode_attention_noalloc(C.byref(p), C.c_void_p(out.data_ptr()),
                                                C.c_void_p(lse.data_ptr()), None)
    assert st == 6   # CKL_WORKSPACE_TOO_SMALL, before any launch
    assert b"built-in scratch" in ckl.lib().ckl_last_error_string()
