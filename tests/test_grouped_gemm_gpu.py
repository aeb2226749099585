"""GPU parity of the dense grouped expert GEMM (ckl_moe_grouped_gemm, tcgen05), the path of
02_moe_grouped_gemm.cu for batches with tens of tokens or more per expert.

The reference's correctness cases (02:310-314, full layer: route + permute + grouped GEMM +
combine) are checked against the fp64 oracle with the reference's tolerance (rtol 1e-2,
atol 5e-3, 02:326-330); its prefill shapes (02:342-344) at full size against a fp32 torch
GEMM per expert on the same fp16 inputs; experts with more than 256 rows (several row
chunks), empty experts, and run-to-run bit identity; the persistent stream-K schedule's
cut items (partial tiles, flags cleared for the next launch) and its workspace check."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _close(got, ref, rtol=1e-2, atol=5e-3):
    got = np.asarray(got, np.float64)
    ref = np.asarray(ref, np.float64)
    bad = np.abs(got - ref) > atol + rtol * np.abs(ref)
    return int(bad.sum()), float(np.abs(got - ref).max())


def T_(a, dev):
    import torch
    return torch.from_numpy(np.ascontiguousarray(a)).to(dev)


@pytest.mark.parametrize("T,E,k,d,f,disable", [(100, 8, 2, 256, 384, -1), (37, 16, 4, 128, 256, 3),
                                               (64, 64, 6, 128, 128, -1), (600, 2, 1, 128, 256, -1)])
def test_layer_with_grouped_gemm_against_fp64(ckl, oracle, dev, T, E, k, d, f, disable):
    import torch
    lg = oracle.make_logits(T, E, 5, disable=disable)
    X = oracle.normal((T, d), seed=21, std=0.5)
    W = oracle.normal((E, d, f), seed=22, std=0.05)
    r = ckl.route_and_permute(T_(lg, dev), T_(X, dev), k)
    Wd = T_(W, dev)
    Yp = ckl.grouped_gemm(r["Xp"], Wd, r["offsets"])
    out = ckl.combine(Yp, r["inv_perm"], r["wts"], T, k)
    torch.cuda.synchronize()
    ckl.check_device_error()
    ids, wts = oracle.route(lg, k)
    assert np.array_equal(r["ids"].cpu().numpy(), ids)
    counts, offsets, _, inv = oracle.permute(ids, E)
    Xp = np.empty((T * k, d), np.float16)
    Xp[inv] = X[np.arange(T * k) // k]
    Y = oracle.expert_gemm(Xp, W.astype(np.float32), offsets)
    ref = oracle.combine(Y, inv, wts, T, k)
    nbad, err = _close(out.float().cpu().numpy(), ref)
    assert nbad == 0, (nbad, err)
    # the expert GEMM itself, row by row
    nbad, err = _close(Yp.float().cpu().numpy(), Y)
    assert nbad == 0, (nbad, err)
    again = ckl.grouped_gemm(r["Xp"], Wd, r["offsets"])
    assert torch.equal(again, Yp)


@pytest.mark.parametrize("T,E,k,d,f", [(512, 8, 2, 4096, 14336), (512, 64, 6, 2048, 1408),
                                       (16, 64, 6, 2048, 1408)])
def test_reference_prefill_shapes_full_size(ckl, oracle, dev, T, E, k, d, f):
    import torch
    g = torch.Generator(device=dev)
    g.manual_seed(T + E)
    lg = torch.randn((T, E), generator=g, device=dev)
    X = (torch.rand((T, d), generator=g, device=dev) * 2 - 1).half()
    W = ((torch.rand((E, d, f), generator=g, device=dev) * 2 - 1) / d ** 0.5).half()
    r = ckl.route_and_permute(lg, X, k)
    Yp = ckl.grouped_gemm(r["Xp"], W, r["offsets"])
    torch.cuda.synchronize()
    ckl.check_device_error()
    off = r["offsets"].cpu().numpy()
    worst = 0.0
    for e in range(E):
        a, b = int(off[e]), int(off[e + 1])
        if a == b:
            continue
        ref = r["Xp"][a:b].float() @ W[e].float()
        got = Yp[a:b].float()
        bad = (got - ref).abs() > 5e-3 + 1e-2 * ref.abs()
        assert int(bad.sum()) == 0, (e, float((got - ref).abs().max()))
        worst = max(worst, float((got - ref).abs().max()))
    del W
    torch.cuda.empty_cache()


def _torch_ref(Xp, W, off):
    import torch
    Y = torch.zeros((Xp.shape[0], W.shape[2]), dtype=torch.float32, device=Xp.device)
    for e in range(W.shape[0]):
        a, b = int(off[e]), int(off[e + 1])
        if b > a:
            Y[a:b] = Xp[a:b].float() @ W[e].float()
    return Y


def _case(dev, T, E, k, d, f, seed):
    import torch
    g = torch.Generator(device=dev)
    g.manual_seed(seed)
    lg = torch.randn((T, E), generator=g, device=dev)
    X = (torch.rand((T, d), generator=g, device=dev) * 2 - 1).half()
    W = ((torch.rand((E, d, f), generator=g, device=dev) * 2 - 1) / d ** 0.5).half()
    return lg, X, W


@pytest.mark.parametrize("T,E,k,d,f", [(3, 2, 1, 4096, 256), (2, 1, 1, 8192, 128),
                                       (5, 3, 2, 2048, 384)])
def test_items_cut_across_many_ctas(ckl, dev, T, E, k, d, f):
    """Few items with long k: one item's k blocks are spread over up to 128 CTAs (stream-K
    writers and one finisher), ranges of one k block, empty ranges."""
    import torch
    lg, X, W = _case(dev, T, E, k, d, f, seed=d + f)
    r = ckl.route_and_permute(lg, X, k)
    ws = ckl.grouped_workspace(dev)
    Yp = ckl.grouped_gemm(r["Xp"], W, r["offsets"], workspace=ws)
    torch.cuda.synchronize()
    ckl.check_device_error()
    ref = _torch_ref(r["Xp"], W, r["offsets"].cpu().numpy())
    bad = (Yp.float() - ref).abs() > 5e-3 + 1e-2 * ref.abs()
    assert int(bad.sum()) == 0, float((Yp.float() - ref).abs().max())
    assert int(ws[:1024].count_nonzero()) == 0          # every flag cleared by its finisher
    again = ckl.grouped_gemm(r["Xp"], W, r["offsets"], workspace=ws)
    assert torch.equal(again, Yp)


def test_changing_routings_reuse_one_workspace(ckl, dev):
    """Launches with different expert counts back to back on one workspace (the flags each
    launch leaves must be the zeros the next one needs); the first result is reproduced."""
    import torch
    ws = ckl.grouped_workspace(dev)
    cases = [(64, 8, 2, 1024, 2048, 1), (300, 16, 3, 512, 1152, 2), (7, 4, 2, 2048, 512, 3)]
    first = {}
    for rep in range(2):
        for T, E, k, d, f, seed in cases:
            lg, X, W = _case(dev, T, E, k, d, f, seed)
            r = ckl.route_and_permute(lg, X, k)
            Yp = ckl.grouped_gemm(r["Xp"], W, r["offsets"], workspace=ws)
            torch.cuda.synchronize()
            ckl.check_device_error()
            if rep == 0:
                ref = _torch_ref(r["Xp"], W, r["offsets"].cpu().numpy())
                bad = (Yp.float() - ref).abs() > 5e-3 + 1e-2 * ref.abs()
                assert int(bad.sum()) == 0, (T, E, float((Yp.float() - ref).abs().max()))
                first[seed] = Yp
            else:
                assert torch.equal(first[seed], Yp), (T, E)
    assert int(ws[:1024].count_nonzero()) == 0


def test_workspace_too_small_is_refused(ckl, dev):
    import torch
    lg, X, W = _case(dev, 8, 4, 2, 128, 128, seed=5)
    r = ckl.route_and_permute(lg, X, 2)
    small = torch.zeros(1024, dtype=torch.uint8, device=dev)
    with pytest.raises(ckl.CklError) as ei:
        ckl.grouped_gemm(r["Xp"], W, r["offsets"], workspace=small)
    assert ei.value.status == ckl.CKL_WORKSPACE_TOO_SMALL
