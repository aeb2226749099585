"""GPU parity of the weight-only MoE decode layer.

Bars (north star): dequantised weights, routing ids, counts, offsets, tile offsets and
inv_perm bit-exact against the host restatement; expert-GEMM / layer outputs within 1e-2
relative RMS of the fp64 oracle over the identical dequantised weights (the reference's own
GEMM test also used max-abs 2e-3 + 1e-2 rel, 03_moe_wq_decode.cu:483). Routing weights are
fp32 on the device and fp64 in the oracle: compared at 2e-6 relative.
"""
import os

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

REF03 = os.path.join(os.path.dirname(__file__), "..", "oracle", "_ref", "libref03.so")
REL_RMS = 1e-2


def rel_rms(got, ref):
    got = np.asarray(got, np.float64)
    ref = np.asarray(ref, np.float64)
    return float(np.linalg.norm(got - ref) / max(np.linalg.norm(ref), 1e-30))


def T_(a, dev):
    import torch
    return torch.from_numpy(np.ascontiguousarray(a)).to(dev)


@pytest.mark.parametrize("bits,group,asym", [(4, 128, False), (4, 128, True), (8, 128, False),
                                             (8, 0, False), (16, 0, False)])
def test_quantizer_bit_exact(ckl, oracle, dev, bits, group, asym):
    E, K, N = 3, 384, 56
    W = oracle.normal((E, K, N), seed=7, std=0.02)
    g = group or K
    q = ckl.QuantWeights(bits, T_(W, dev), group=g, asym=asym)
    got = q.dequant().cpu().numpy()
    if bits == 16:
        assert np.array_equal(got, W.astype(np.float32))
        return
    if asym:
        codes, scales, zeros = oracle.quant_asym4(W)
    else:
        codes, scales = oracle.quant_sym(W, bits, group=g)
        zeros = None
    want = oracle.dequant(codes, scales, zeros, bits, group=g)
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))
    assert np.array_equal(q.scales[:scales.size].cpu().numpy().reshape(scales.shape).view(np.uint16),
                          scales.view(np.uint16))
    if asym:
        zw = q.zeros[:E * (K // 128) * N // 8].cpu().numpy().view(np.uint32)
        nib = np.stack([(zw >> (4 * c)) & 15 for c in range(8)], -1).reshape(zeros.shape)
        assert np.array_equal(nib.astype(np.uint8), zeros)


@pytest.mark.skipif(not os.path.exists(REF03), reason="reference not compiled here")
@pytest.mark.parametrize("bits", [4, 8, 16])
def test_packing_matches_reference_pack_weights(ckl, oracle, dev, bits):
    """The reference's own pack_weights<bits> kernel (03_moe_wq_decode.cu:49-87) on the
    reference test's weights: identical scales, and our dequantised weights equal its
    host_weight (03:336-348) bit for bit."""
    import ctypes as C
    import torch
    E, d, f = 8, 2048, 200
    W = oracle.init_uniform((E, d, f), 5 + 2, 1.0 / np.sqrt(d))     # m.init(5): W seed + 2
    dW = T_(W, dev)
    cpt = 32 // bits
    P = torch.empty(E * d * (f // cpt), dtype=torch.int32, device=dev)
    ns = E * (d // 128) * f if bits < 16 else 1
    Sc = torch.empty(ns, dtype=torch.float16, device=dev)
    L = oracle.ref03()
    assert L.ref03_pack_weights_device(bits, C.c_void_p(dW.data_ptr()), C.c_void_p(P.data_ptr()),
                                       C.c_void_p(Sc.data_ptr()), E, d, f) == 0
    Pn = P.cpu().numpy().view(np.uint32)
    Scn = Sc.cpu().numpy()
    ref_w = np.empty((E, d, f), np.float32)
    L.ref03_host_weight_all(bits, oracle._p(Pn), Pn.size, oracle._p(Scn), Scn.size, E, d, f,
                            oracle._p(ref_w))
    q = ckl.QuantWeights(bits, dW, group=128)
    got = q.dequant().cpu().numpy()
    assert np.array_equal(got.view(np.uint32), ref_w.view(np.uint32))
    if bits < 16:
        assert np.array_equal(q.scales.cpu().numpy().view(np.uint16), Scn.view(np.uint16))


@pytest.mark.skipif(not os.path.exists(REF03), reason="reference not compiled here")
@pytest.mark.parametrize("bits", [4, 8, 16])
def test_import_reference_packed_weights(ckl, oracle, dev, bits):
    """Weights packed by the reference's own pack_weights<bits> (03_moe_wq_decode.cu:49-87),
    imported through ckl_moe_import_reference_packed: the dequantised weights equal the
    reference's host_weight (03:336-348) bit for bit, the packed records equal our own
    packer's from the same fp16 weights, and the expert GEMM over the imported weights
    matches the fp64 oracle on the reference's GEMM case (T=40 tokens, top-2, 8 experts,
    one of them empty)."""
    import ctypes as C
    import torch
    E, d, f = 8, 2048, 200
    W = oracle.init_uniform((E, d, f), 5 + 2, 1.0 / np.sqrt(d))
    dW = T_(W, dev)
    cpt = 32 // bits
    P = torch.empty(E * d * (f // cpt), dtype=torch.int32, device=dev)
    ns = E * (d // 128) * f if bits < 16 else 1
    Sc = torch.empty(ns, dtype=torch.float16, device=dev)
    L = oracle.ref03()
    assert L.ref03_pack_weights_device(bits, C.c_void_p(dW.data_ptr()), C.c_void_p(P.data_ptr()),
                                       C.c_void_p(Sc.data_ptr()), E, d, f) == 0
    Pn = P.cpu().numpy().view(np.uint32)
    Scn = Sc.cpu().numpy()
    ref_w = np.empty((E, d, f), np.float32)
    L.ref03_host_weight_all(bits, oracle._p(Pn), Pn.size, oracle._p(Scn), Scn.size, E, d, f,
                            oracle._p(ref_w))
    imp = ckl.QuantWeights.from_reference_packed(bits, P, Sc, E, d, f)
    torch.cuda.synchronize()
    got = imp.dequant().cpu().numpy()
    assert np.array_equal(got.view(np.uint32), ref_w.view(np.uint32))
    own = ckl.QuantWeights(bits, dW, group=128)
    assert torch.equal(imp.packed, own.packed)
    # expert GEMM over the imported weights: the reference's correctness case shape
    T, k = 40, 2
    lg = oracle.make_logits(T, E, 5, 3)                 # expert 3 receives no tokens
    X = oracle.init_uniform((T, d), 5 + 1, 1.0)
    r = ckl.route_and_permute(T_(lg, dev), T_(X, dev), k)
    A = T * k
    Yp = torch.empty((A, f), dtype=torch.float16, device=dev)
    imp.run(r["Xp"], Yp, r["offsets"], A)
    torch.cuda.synchronize()
    ref = oracle.expert_gemm(r["Xp"].cpu().numpy(), ref_w, r["offsets"].cpu().numpy())
    assert rel_rms(Yp.float().cpu().numpy(), ref) <= REL_RMS


ROUTE_CASES = [(40, 8, 2, 3, 5), (64, 64, 6, -1, 9), (1, 64, 6, -1, 9), (16, 8, 2, -1, 9),
               (100, 8, 2, -1, 5), (37, 16, 4, 3, 5), (300, 256, 8, -1, 1)]


@pytest.mark.parametrize("T,E,k,disable,seed", ROUTE_CASES)
def test_routing_bit_exact(ckl, oracle, dev, T, E, k, disable, seed):
    lg = oracle.make_logits(T, E, seed, disable)
    X = oracle.normal((T, 128), seed=3)
    r = ckl.route_and_permute(T_(lg, dev), T_(X, dev), k, bm=64)
    ids, wts = oracle.route(lg, k)
    counts, offsets, tiles, inv = oracle.permute(ids, E, bm=64)
    assert np.array_equal(r["ids"].cpu().numpy(), ids)
    assert np.allclose(r["wts"].cpu().numpy(), wts, rtol=2e-6, atol=0)
    assert np.array_equal(r["counts"].cpu().numpy(), counts)
    assert np.array_equal(r["offsets"].cpu().numpy(), offsets)
    assert np.array_equal(r["tiles"].cpu().numpy(), tiles)
    assert np.array_equal(r["inv_perm"].cpu().numpy(), inv)
    Xp = r["Xp"].cpu().numpy()
    flat = np.arange(T * k) // k
    assert np.array_equal(Xp[inv], X[flat])


@pytest.mark.parametrize("T,E,k", [(64, 64, 6), (33, 8, 2), (16, 256, 8)])
def test_routing_ties_go_to_the_lower_id(ckl, oracle, dev, T, E, k):
    """Logits drawn from 5 integer values (many exact ties), a quarter of the zeros negative:
    slot order is larger logit first, equal logits (-0 equal to +0) to the lower expert id,
    as in the reference (common/moe.cuh:55-59); ids bit-exact against the host restatement
    and, where it was compiled, the reference's own router_topk."""
    rng = np.random.default_rng(T * 1000 + E)
    lg = rng.integers(-2, 3, size=(T, E)).astype(np.float32)
    neg0 = (lg == 0) & (rng.random((T, E)) < 0.25)
    lg[neg0] = -0.0
    assert np.any(np.signbit(lg) & (lg == 0))
    r = ckl.route_and_permute(T_(lg, dev), None, k, permute=False)
    ids, wts = oracle.route(lg, k)
    assert np.array_equal(r["ids"].cpu().numpy(), ids)
    assert np.allclose(r["wts"].cpu().numpy(), wts, rtol=2e-6, atol=0)
    if os.path.exists(REF03):
        import ctypes as C
        import torch
        rid = torch.empty((T, k), dtype=torch.int32, device=dev)
        rw = torch.empty((T, k), dtype=torch.float32, device=dev)
        d_lg = T_(lg, dev)
        assert oracle.ref03().ref03_router_topk_device(C.c_void_p(d_lg.data_ptr()), C.c_void_p(rid.data_ptr()),
                                                       C.c_void_p(rw.data_ptr()), T, E, k) == 0
        assert torch.equal(r["ids"], rid)


@pytest.mark.skipif(not os.path.exists(REF03), reason="reference not compiled here")
def test_routing_matches_reference_router_kernel(ckl, oracle, dev):
    """Same ids as the reference's own router_topk kernel (common/moe.cuh:23-72)."""
    import ctypes as C
    import torch
    for T, E, k, seed in [(64, 64, 6, 9), (40, 8, 2, 5), (16, 64, 6, 9)]:
        lg = T_(oracle.make_logits(T, E, seed), dev)
        ids = torch.empty((T, k), dtype=torch.int32, device=dev)
        wts = torch.empty((T, k), dtype=torch.float32, device=dev)
        assert oracle.ref03().ref03_router_topk_device(C.c_void_p(lg.data_ptr()), C.c_void_p(ids.data_ptr()),
                                                       C.c_void_p(wts.data_ptr()), T, E, k) == 0
        r = ckl.route_and_permute(lg, None, k, permute=False)
        assert torch.equal(r["ids"], ids)
        assert torch.allclose(r["wts"], wts, rtol=1e-5, atol=1e-7)


@pytest.mark.parametrize("bits", [16, 8, 4])
@pytest.mark.parametrize("ks", [1, 4])
def test_expert_gemm_reference_case(ckl, oracle, dev, bits, ks):
    """03_moe_wq_decode.cu:449-485: T=40, E=8, k=2, d=2048, f=200 (tail column tile), one
    empty expert, inputs from the reference's generators (make_logits seed 5 disable 3,
    init_uniform X seed 6, W seed 7 scaled 1/sqrt(d)); K split 1 and 4 ways."""
    T, E, k, d, f = 40, 8, 2, 2048, 200
    lg = oracle.make_logits(T, E, 5, 3)
    X = oracle.init_uniform((T, d), 6, 1.0)
    W = oracle.init_uniform((E, d, f), 7, 1.0 / np.sqrt(d))
    r = ckl.route_and_permute(T_(lg, dev), T_(X, dev), k)
    offs = r["offsets"].cpu().numpy()
    assert offs[4] == offs[3]                 # expert 3 is empty
    q = ckl.QuantWeights(bits, T_(W, dev), group=128)
    import torch
    Yp = torch.zeros((T * k, f), dtype=torch.float16, device=dev)
    q.run(r["Xp"], Yp, r["offsets"], T * k, force_ksplit=ks)
    torch.cuda.synchronize()
    ckl.check_device_error()
    ref = oracle.expert_gemm(r["Xp"].cpu().numpy(), q.dequant().cpu().numpy(), offs)
    got = Yp.float().cpu().numpy()
    assert rel_rms(got, ref) <= REL_RMS
    assert np.all(np.abs(got - ref) <= 2e-3 + 1e-2 * np.abs(ref))


@pytest.mark.parametrize("asym", [True, False])
@pytest.mark.parametrize("ks", [1, 2, 4])
def test_expert_gemm_int4_tile_multiple_width(ckl, oracle, dev, asym, ks):
    """int4 at a width of whole 64-column quads: the reference case's generators at d=1024,
    f=384, T=40, E=8, top-2 -- experts with more than 16 rows run in several passes, expert
    3 is empty -- K split 1, 2 and 4 ways, asymmetric and symmetric codes."""
    T, E, k, d, f = 40, 8, 2, 1024, 384
    lg = oracle.make_logits(T, E, 5, 3)
    X = oracle.init_uniform((T, d), 6, 1.0)
    W = oracle.init_uniform((E, d, f), 7, 1.0 / np.sqrt(d))
    r = ckl.route_and_permute(T_(lg, dev), T_(X, dev), k)
    offs = r["offsets"].cpu().numpy()
    assert offs[4] == offs[3] and np.diff(offs).max() > 16
    q = ckl.QuantWeights(4, T_(W, dev), group=128, asym=asym)
    import torch
    Yp = torch.zeros((T * k, f), dtype=torch.float16, device=dev)
    q.run(r["Xp"], Yp, r["offsets"], T * k, force_ksplit=ks)
    torch.cuda.synchronize()
    ckl.check_device_error()
    ref = oracle.expert_gemm(r["Xp"].cpu().numpy(), q.dequant().cpu().numpy(), offs)
    got = Yp.float().cpu().numpy()
    assert rel_rms(got, ref) <= REL_RMS
    assert np.all(np.abs(got - ref) <= 2e-3 + 1e-2 * np.abs(ref))


def _layer_weights(ckl, oracle, dev, E, d, F, mode, seed=11):
    import torch
    Wg = oracle.normal((E, d, F), seed=seed, std=0.02)
    Wu = oracle.normal((E, d, F), seed=seed + 1, std=0.02)
    Wd = oracle.normal((E, F, d), seed=seed + 2, std=0.02)
    kw = dict(int4=dict(bits=4, group=128, asym=True), int8pc=dict(bits=8, group=0),
              fp16=dict(bits=16, group=0), int4sym=dict(bits=4, group=128))[mode]
    def q(W):
        g = kw.get("group") or W.shape[1]
        return ckl.QuantWeights(kw["bits"], T_(W, dev), group=g, asym=kw.get("asym", False))
    return q(Wg), q(Wu), q(Wd)


@pytest.mark.parametrize("mode", ["int4", "int8pc", "fp16", "int4sym"])
@pytest.mark.parametrize("T", [1, 5, 33])
def test_moe_layer_against_fp64_oracle(ckl, oracle, dev, mode, T):
    import torch
    E, k, d, F = 8, 2, 256, 384
    gq, uq, dq = _layer_weights(ckl, oracle, dev, E, d, F, mode)
    lg = oracle.normal((T, E), seed=100 + T, fp16=False)
    X = oracle.normal((T, d), seed=200 + T)
    layer = ckl.MoeLayer(gq, uq, dq)
    ids = torch.empty((T, k), dtype=torch.int32, device=dev)
    wts = torch.empty((T, k), dtype=torch.float32, device=dev)
    out = layer.forward(T_(lg, dev), T_(X, dev), k, ids=ids, wts=wts)
    torch.cuda.synchronize()
    ckl.check_device_error()
    rids, rwts = oracle.route(lg, k)
    assert np.array_equal(ids.cpu().numpy(), rids)
    ref = oracle.moe_layer(X, rids, rwts, gq.dequant().cpu().numpy(), uq.dequant().cpu().numpy(),
                           dq.dequant().cpu().numpy())
    assert rel_rms(out.float().cpu().numpy(), ref) <= REL_RMS
    again = layer.forward(T_(lg, dev), T_(X, dev), k)
    assert torch.equal(out, again)                     # deterministic


@pytest.mark.parametrize("T", [1, 4, 16, 64])
def test_config4_w4a16_layer_full_size(ckl, oracle, dev, T):
    """E=64, top-6, d=2048, F=1408, asymmetric int4 g128, weights
    N(0,0.02), activations and logits N(0,1). Routing ids bit-exact for the whole batch;
    the output of up to 8 sampled tokens against the fp64 oracle (rel-RMS <= 1e-2)."""
    import torch
    from moe_ref import rel_rms as rr, sample_tokens, sampled_layer_ref
    E, k, d, F = 64, 6, 2048, 1408
    g = torch.Generator(device=dev)
    g.manual_seed(4)
    mk = lambda *s: (torch.randn(*s, generator=g, device=dev) * 0.02).half()
    gq = ckl.QuantWeights(4, mk(E, d, F), group=128, asym=True)
    uq = ckl.QuantWeights(4, mk(E, d, F), group=128, asym=True)
    dq = ckl.QuantWeights(4, mk(E, F, d), group=128, asym=True)
    lg = torch.randn((T, E), generator=g, device=dev)
    X = torch.randn((T, d), generator=g, device=dev).half()
    ids = torch.empty((T, k), dtype=torch.int32, device=dev)
    wts = torch.empty((T, k), dtype=torch.float32, device=dev)
    out = ckl.MoeLayer(gq, uq, dq).forward(lg, X, k, ids=ids, wts=wts)
    torch.cuda.synchronize()
    ckl.check_device_error()
    tok = sample_tokens(T)
    ref, rids = sampled_layer_ref(oracle, lg.cpu().numpy(), X.cpu().numpy(), k, gq, uq, dq, tok)
    assert np.array_equal(ids.cpu().numpy(), rids)
    assert rr(out.float().cpu().numpy()[tok], ref) <= REL_RMS


def test_config5_w8a16_moe_full_size(ckl, oracle, dev):
    """BASELINE config 5 MoE block: E=8, top-2, d=4096, F=14336, int8 per output channel,
    weights N(0,0.02), T=32. Routing ids bit-exact; 8 sampled tokens against the fp64
    oracle (rel-RMS <= 1e-2)."""
    import torch
    from moe_ref import rel_rms as rr, sample_tokens, sampled_layer_ref
    E, k, d, F, T = 8, 2, 4096, 14336, 32
    g = torch.Generator(device=dev)
    g.manual_seed(5)
    mk = lambda *s: (torch.randn(*s, generator=g, device=dev) * 0.02).half()
    gq = ckl.QuantWeights(8, mk(E, d, F), group=d)
    uq = ckl.QuantWeights(8, mk(E, d, F), group=d)
    dq = ckl.QuantWeights(8, mk(E, F, d), group=F)
    lg = torch.randn((T, E), generator=g, device=dev)
    X = torch.randn((T, d), generator=g, device=dev).half()
    ids = torch.empty((T, k), dtype=torch.int32, device=dev)
    wts = torch.empty((T, k), dtype=torch.float32, device=dev)
    out = ckl.MoeLayer(gq, uq, dq).forward(lg, X, k, ids=ids, wts=wts)
    torch.cuda.synchronize()
    ckl.check_device_error()
    tok = sample_tokens(T)
    ref, rids = sampled_layer_ref(oracle, lg.cpu().numpy(), X.cpu().numpy(), k, gq, uq, dq, tok)
    assert np.array_equal(ids.cpu().numpy(), rids)
    assert rr(out.float().cpu().numpy()[tok], ref) <= REL_RMS
    del gq, uq, dq
    torch.cuda.empty_cache()


@pytest.mark.parametrize("mode", ["int4", "int8pc", "fp16", "int4sym"])
def test_packed_weights_file_round_trip(ckl, oracle, dev, tmp_path, mode):
    """ckl_moe_weights_save / _file_info / _load: the buffers come back bit for bit and the
    layer computes the same output from the loaded weights."""
    import torch
    E, k, d, F, T = 8, 2, 256, 384, 5
    gq, uq, dq = _layer_weights(ckl, oracle, dev, E, d, F, mode)
    paths = [tmp_path / f"{n}.ckw" for n in ("gate", "up", "down")]
    for q, pth in zip((gq, uq, dq), paths):
        q.save(pth)
    lq = [ckl.QuantWeights.load(pth, device=dev) for pth in paths]
    for a, b in zip((gq, uq, dq), lq):
        assert (a.bits, a.E, a.K, a.N, a.group, a.asym) == (b.bits, b.E, b.K, b.N, b.group, b.asym)
        assert torch.equal(a.packed, b.packed)
        if a.bits != 16:
            assert torch.equal(a.scales, b.scales)
        if a.asym:
            assert torch.equal(a.zeros, b.zeros)
    lg = T_(oracle.normal((T, E), seed=7, fp16=False), dev)
    X = T_(oracle.normal((T, d), seed=8), dev)
    ref = ckl.MoeLayer(gq, uq, dq).forward(lg, X, k)
    got = ckl.MoeLayer(*lq).forward(lg, X, k)
    torch.cuda.synchronize()
    assert torch.equal(ref, got)
