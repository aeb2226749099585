"""GPU parity of paged split-KV decode attention against the fp64 oracle.

Cases are the reference's own (01_decode_attention.cu:750-776): every case under three
split settings {no split, heuristic, 7 chunks}. Tolerances: out max-abs <= 2e-3 (north
star; the reference used atol 2e-3 + rtol 1e-2) and lse within 1e-4 abs + 1e-4 rel
(01_decode_attention.cu:776). BASELINE sizes are checked on sampled sequences.
"""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

OUT_ATOL = 2e-3
LSE_ATOL, LSE_RTOL = 1e-4, 1e-4


def to_dev(bt, dev):
    import torch
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(dev)
    return dict(q=t(bt.q), k_cache=t(bt.k), v_cache=t(bt.v), kv_indptr=t(bt.indptr),
                kv_indices=t(bt.indices), kv_last_page_len=t(bt.last))


def check(out, lse, ref_o, ref_l, tag):
    o = out.float().cpu().numpy()
    l = lse.cpu().numpy()
    assert np.isfinite(o).all(), tag
    err = np.abs(o - ref_o).max()
    assert err <= OUT_ATOL, f"{tag}: out max-abs {err:.3e}"
    fin = np.isfinite(ref_l)
    assert np.array_equal(fin, np.isfinite(l)), tag
    lerr = np.abs(l[fin] - ref_l[fin])
    assert np.all(lerr <= LSE_ATOL + LSE_RTOL * np.abs(ref_l[fin])), f"{tag}: lse {lerr.max():.3e}"
    return err


CASES = [([1, 17, 1000], 8, 8), ([5, 300, 2049, 4096], 32, 8), ([33, 777], 16, 2),
         ([16, 32, 48, 4097], 4, 2)]


@pytest.mark.parametrize("lens,Hq,Hkv", CASES)
@pytest.mark.parametrize("force", [1, 0, 7])
def test_reference_cases(ckl, oracle, dev, lens, Hq, Hkv, force):
    bt = oracle.batch(lens, Hq, Hkv, 7)
    ref_o, ref_l = oracle.attention_ref(bt)
    d = to_dev(bt, dev)
    out, lse = ckl.decode_attention(**d, force_chunks=force)
    check(out, lse, ref_o, ref_l, f"{lens} G={Hq // Hkv} force={force}")


def test_config1_against_reference_golden(ckl, oracle, dev):
    """BASELINE config 1 against the reference's own cpu_reference output."""
    import os
    g = np.load(os.path.join(os.path.dirname(__file__), "golden", "attn_config1.npz"))
    bt = oracle.batch([1000, 777], 32, 8, 7)
    d = to_dev(bt, dev)
    for force in (1, 0, 3):
        out, lse = ckl.decode_attention(**d, force_chunks=force)
        check(out, lse, g["out"], g["lse"], f"config1 force={force}")


@pytest.mark.parametrize("G", [1, 2, 4, 8, 16])
def test_group_sizes(ckl, oracle, dev, G):
    Hkv = 2
    bt = oracle.batch([1, 15, 16, 17, 300], G * Hkv, Hkv, 11)
    ref_o, ref_l = oracle.attention_ref(bt)
    d = to_dev(bt, dev)
    for force in (1, 2):
        out, lse = ckl.decode_attention(**d, force_chunks=force)
        check(out, lse, ref_o, ref_l, f"G={G} force={force}")


def test_empty_sequences_and_empty_chunks(ckl, oracle, dev):
    # a zero-length sequence gives out = 0, lse = -inf; 9 chunks over 40 keys leave most
    # chunks of the short sequences empty
    bt = oracle.batch([0, 5, 40, 1], 32, 8, 5)
    ref_o, ref_l = oracle.attention_ref(bt)
    d = to_dev(bt, dev)
    for force in (1, 9):
        out, lse = ckl.decode_attention(**d, force_chunks=force)
        check(out, lse, ref_o, ref_l, f"empty force={force}")
        assert float(out[0].abs().max()) == 0.0
        assert np.isneginf(lse[0].cpu().numpy()).all()


def test_deterministic_repeat(ckl, oracle, dev):
    bt = oracle.batch([5, 300, 2049, 4096], 32, 8, 7)
    d = to_dev(bt, dev)
    a = ckl.decode_attention(**d, force_chunks=5)
    b = ckl.decode_attention(**d, force_chunks=5)
    assert bool((a[0] == b[0]).all()) and bool((a[1] == b[1]).all())


@pytest.mark.parametrize("force", [0, 5])
def test_cache_ready_chain_equals_plain(ckl, oracle, dev, force):
    """ckl_decode_attention_ex with CKL_DECODE_CACHE_READY in a chain where each call's q is
    the previous call's output (written by the kernel it starts behind): every output equals
    the plain entry point's bit for bit, launched back to back on one stream and replayed
    from a CUDA graph; the first layer is checked against the fp64 oracle. The caches and
    page tables are written before the chain starts, as the flag requires."""
    import torch
    lens = [5, 300, 2049, 4096]
    layers = [to_dev(oracle.batch(lens, 32, 8, 40 + l), dev) for l in range(4)]
    q0 = layers[0]["q"]

    def run(ready, outs):
        x = q0
        for l, d in enumerate(layers):
            dd = dict(d, q=x)
            ckl.decode_attention(**dd, max_len=max(lens), force_chunks=force, out=outs[l][0],
                                 lse=outs[l][1], workspace=ws, cache_ready=ready)
            x = outs[l][0]

    ws = torch.empty(64 << 20, dtype=torch.uint8, device=dev)
    mk = lambda: [(torch.empty_like(q0), torch.empty((len(lens), 32), dtype=torch.float32,
                                                     device=dev)) for _ in layers]
    plain, ready, graphed = mk(), mk(), mk()
    run(False, plain)
    run(True, ready)
    torch.cuda.synchronize()
    ckl.check_device_error()
    s = torch.cuda.Stream(device=dev)
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        run(True, graphed)                              # warm-up outside the capture
    torch.cuda.current_stream().wait_stream(s)
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        run(True, graphed)
    for o, l in graphed:
        o.zero_()
        l.zero_()
    g.replay()
    torch.cuda.synchronize()
    ckl.check_device_error()
    for l in range(len(layers)):
        for got in (ready[l], graphed[l]):
            assert torch.equal(got[0], plain[l][0]) and torch.equal(got[1], plain[l][1]), l
    bt = oracle.batch(lens, 32, 8, 40)
    ref_o, ref_l = oracle.attention_ref(bt)
    check(plain[0][0], plain[0][1], ref_o, ref_l, "cache-ready chain, layer 0")


def test_partial_and_merge_entry_points(ckl, oracle, dev):
    """decode_partial + merge_states driven separately (the cascade suffix pattern:
    kv_start > 0, chunk_base > 0) against the oracle over the suffix keys."""
    import torch
    Lp = 64
    bt = oracle.batch([Lp + 1, Lp + 40, Lp + 300], 32, 8, 3)
    d = to_dev(bt, dev)
    # reference over the suffix only: drop the first Lp/16 pages of every sequence
    sub = oracle.Batch(bt.lens - Lp, 32, 8, None, None, None, bt.q, bt.k, bt.v)
    sub.indptr = (bt.indptr - np.arange(bt.B + 1) * (Lp // 16)).astype(np.int32)
    sub.indices = np.concatenate([bt.indices[bt.indptr[b] + Lp // 16:bt.indptr[b + 1]]
                                  for b in range(bt.B)]).astype(np.int32)
    ref_o, ref_l = oracle.attention_ref(sub)
    base, nc = 2, 3
    stride = base + nc
    part_o = torch.full((bt.B * 32, stride, 128), float("nan"), device=dev)
    part_lse = torch.full((bt.B * 32, stride), float("-inf"), device=dev)
    p = ckl.make_params(**d, num_chunks=nc, chunk_tokens=128, kv_start=Lp, chunk_base=base,
                        part_stride=stride, part_o=part_o, part_lse=part_lse)
    ckl.decode_partial(p)
    part_o[:, :base] = 0.0   # unused slots: o = 0, lse = -inf (ignored by the merge)
    out = torch.empty_like(d["q"])
    lse = torch.empty((bt.B, 32), device=dev)
    ckl.merge_states(part_o, part_lse, out, lse)
    torch.cuda.synchronize()
    check(out, lse, ref_o, ref_l, "suffix via partial+merge")


def _sampled_full_size(ckl, oracle, dev, lens, Hq=32, Hkv=8, sample=(0,), seed=11):
    """A BASELINE-size batch with device-filled U(-1,1) K/V; the oracle checks the sampled
    sequences (their pages gathered to the host)."""
    import torch
    lens = np.asarray(lens, np.int32)
    bt = oracle.batch(lens, Hq, Hkv, seed, fill=False)
    g = torch.Generator(device=dev)
    g.manual_seed(seed)
    shape = (bt.num_pages, 16, Hkv, 128)
    k = (torch.rand(shape, generator=g, device=dev, dtype=torch.float32) * 2 - 1).half()
    v = (torch.rand(shape, generator=g, device=dev, dtype=torch.float32) * 2 - 1).half()
    q = (torch.rand((bt.B, Hq, 128), generator=g, device=dev) * 2 - 1).half()
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(dev)
    out, lse = ckl.decode_attention(q, k, v, t(bt.indptr), t(bt.indices), t(bt.last))
    out, lse = out.float().cpu().numpy(), lse.cpu().numpy()
    for b in sample:
        pages = bt.indices[bt.indptr[b]:bt.indptr[b + 1]]
        pi = torch.from_numpy(pages.astype(np.int64)).to(dev)
        sb = oracle.Batch([lens[b]], Hq, Hkv, np.array([0, len(pages)], np.int32),
                          np.arange(len(pages), dtype=np.int32), bt.last[b:b + 1],
                          q[b:b + 1].cpu().numpy(), k.index_select(0, pi).cpu().numpy(),
                          v.index_select(0, pi).cpu().numpy())
        ro, rl = oracle.attention_ref(sb)
        assert np.abs(out[b] - ro[0]).max() <= OUT_ATOL
        assert np.all(np.abs(lse[b] - rl[0]) <= LSE_ATOL + LSE_RTOL * np.abs(rl[0]))
    del k, v
    torch.cuda.empty_cache()


@pytest.mark.parametrize("B,L", [(1, 32768), (8, 8192), (64, 1024), (256, 4096)])
def test_config2_sweep_sampled(ckl, oracle, dev, B, L):
    _sampled_full_size(ckl, oracle, dev, [L] * B, sample=sorted({0, B // 2, B - 1}))


def test_config2_ragged_sampled(ckl, oracle, dev):
    rng = np.random.default_rng(2024)
    lens = rng.integers(128, 8193, size=256)
    _sampled_full_size(ckl, oracle, dev, lens, sample=(0, 77, 255))


def test_stream_read_probe(ckl, dev):
    import torch
    buf = torch.ones(1 << 26, dtype=torch.uint8, device=dev)
    sink = torch.zeros(1, dtype=torch.int32, device=dev)
    ckl.stream_read(buf, sink)
    torch.cuda.synchronize()
    ckl.check_device_error()
