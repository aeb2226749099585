"""Head-sharded decode attention with the output rows placed in a wider buffer
(ckl_decode_attention_gather), on one GPU: every KV-head shard decoded on its own and
written into its rows of the full output must reproduce the full decode exactly (a head's
rows do not depend on other heads), in the direct single-chunk mode and through the LSE
merge. The gather-completion wait must give up on a flag nothing sets."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _dev_batch(oracle, dev, lens, seed=31):
    import torch
    bt = oracle.batch(lens, 32, 8, seed)
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(dev)
    return bt, dict(q=t(bt.q), k=t(bt.k), v=t(bt.v), indptr=t(bt.indptr),
                    indices=t(bt.indices), last=t(bt.last))


@pytest.mark.parametrize("lens,force", [([1000, 777], 3), ([1000, 777], 1), ([64, 1, 300, 4096], 0)])
@pytest.mark.parametrize("nshard", [2, 4, 8])
def test_head_shards_reassemble_the_full_decode(ckl, oracle, dev, lens, force, nshard):
    import torch
    bt, d = _dev_batch(oracle, dev, lens)
    B = len(lens)
    nc, ct = ckl.plan_chunks(4, B, 8, int(max(lens)), force_chunks=force or 0)
    ref, ref_lse = ckl.decode_attention(d["q"], d["k"], d["v"], d["indptr"], d["indices"],
                                        d["last"], num_chunks=nc, chunk_tokens=ct)
    out = torch.full((B, 32, 128), float("nan"), dtype=torch.float16, device=dev)
    lse = torch.full((B, 32), float("nan"), dtype=torch.float32, device=dev)
    hk, hq = 8 // nshard, 32 // nshard
    for r in range(nshard):
        ks = d["k"][:, :, r * hk:(r + 1) * hk].contiguous()
        vs = d["v"][:, :, r * hk:(r + 1) * hk].contiguous()
        qs = d["q"][:, r * hq:(r + 1) * hq].contiguous()
        p = ckl.make_params(qs, ks, vs, d["indptr"], d["indices"], d["last"], num_chunks=nc,
                            chunk_tokens=ct)
        ws = torch.empty(max(ckl.workspace_size(p), 256), dtype=torch.uint8, device=dev)
        ckl.decode_attention_gather(p, out.data_ptr(), lse.data_ptr(), 32, r * hq, workspace=ws)
    torch.cuda.synchronize()
    ckl.check_device_error()
    assert torch.equal(out, ref)
    assert torch.equal(lse, ref_lse)


def test_gather_rejects_rows_outside_the_output(ckl, oracle, dev):
    bt, d = _dev_batch(oracle, dev, [40])
    p = ckl.make_params(d["q"], d["k"], d["v"], d["indptr"], d["indices"], d["last"],
                        num_chunks=1, chunk_tokens=48)
    import torch
    out = torch.empty((1, 32, 128), dtype=torch.float16, device=dev)
    lse = torch.empty((1, 32), dtype=torch.float32, device=dev)
    with pytest.raises(ckl.CklError):
        ckl.decode_attention_gather(p, out.data_ptr(), lse.data_ptr(), 32, 4)   # 4 + 32 > 32


def test_gather_wait_gives_up_on_a_flag_nothing_sets(ckl, dev):
    import torch
    L = ckl._LibWindows
    w0, _ = L.alloc(ckl.PEER_WINDOW_BYTES)
    w1, _ = L.alloc(ckl.PEER_WINDOW_BYTES)
    try:
        g = ckl.PeerGroup(0, 2, (ckl.C.c_void_p * ckl.EP_MAX_RANKS)(w0, w1))
        ckl.set_spin_timeout_ns(20_000_000)
        ckl.check(ckl.lib().ckl_gather_signal(ckl.C.byref(g), 0, None), "signal")
        ckl.check(ckl.lib().ckl_gather_wait(ckl.C.byref(g), None), "wait")   # rank 1 never signals
        torch.cuda.synchronize()
        with pytest.raises(ckl.CklError) as e:
            ckl.check_device_error()
        assert e.value.status == 5
        # a one-rank group completes at once
        g1 = ckl.PeerGroup(0, 1, (ckl.C.c_void_p * ckl.EP_MAX_RANKS)(w1))
        for _ in range(3):
            ckl.check(ckl.lib().ckl_gather_signal(ckl.C.byref(g1), 0, None), "signal")
            ckl.check(ckl.lib().ckl_gather_wait(ckl.C.byref(g1), None), "wait")
        torch.cuda.synchronize()
        ckl.check_device_error()
    finally:
        ckl.set_spin_timeout_ns(1_000_000_000)
        torch.cuda.synchronize()
        L.free(w0)
        L.free(w1)


def test_peer_barrier_gives_up_on_a_rank_that_never_arrives(ckl, dev):
    """ckl_peer_barrier with a second window that no other rank writes: the barrier's bounded
    wait gives up (CKL_TIMEOUT) and the context stays usable; a one-rank group passes its
    barriers at once, many times in a row (epochs)."""
    import torch
    L = ckl._LibWindows
    w0, _ = L.alloc(ckl.PEER_WINDOW_BYTES)
    w1, _ = L.alloc(ckl.PEER_WINDOW_BYTES)
    try:
        g = ckl.PeerGroup(0, 2, (ckl.C.c_void_p * ckl.EP_MAX_RANKS)(w0, w1))
        ckl.set_spin_timeout_ns(20_000_000)
        ckl.check(ckl.lib().ckl_peer_barrier(ckl.C.byref(g), None), "barrier")  # rank 1 absent
        torch.cuda.synchronize()
        with pytest.raises(ckl.CklError) as e:
            ckl.check_device_error()
        assert e.value.status == 5
        g1 = ckl.PeerGroup(0, 1, (ckl.C.c_void_p * ckl.EP_MAX_RANKS)(w1))
        for _ in range(5):
            ckl.check(ckl.lib().ckl_peer_barrier(ckl.C.byref(g1), None), "barrier")
        torch.cuda.synchronize()
        ckl.check_device_error()
    finally:
        ckl.set_spin_timeout_ns(1_000_000_000)
        torch.cuda.synchronize()
        L.free(w0)
        L.free(w1)
