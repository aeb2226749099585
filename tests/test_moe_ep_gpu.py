"""GPU tests of the expert-parallel MoE layer (ckl_moe_ep_layer) on one device.

world = 1 runs the whole exchange through the rank's own window (dispatch to itself,
receive, GEMMs, pull-back combine): with the same token capacity as the batch, the row
order and split-K choice equal the single-GPU layer's, so the output must be bit-identical
to ckl_moe_layer. The bounded waits are checked with a flag that nothing sets: a world-2
communicator whose second window is a local buffer no other rank writes; the wait must
give up with CKL_TIMEOUT and leave the context usable. The multi-GPU path runs in
test_moe_ep_multi_gpu.py.
"""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

REL_RMS = 1e-2


def rel_rms(got, ref):
    got, ref = np.asarray(got, np.float64), np.asarray(ref, np.float64)
    return float(np.linalg.norm(got - ref) / max(np.linalg.norm(ref), 1e-30))


def _weights(ckl, dev, E, d, F, bits, seed):
    import torch
    g = torch.Generator(device=dev)
    g.manual_seed(seed)
    mk = lambda *s: (torch.randn(*s, generator=g, device=dev) * 0.02).half()
    kw = dict(group=128, asym=True) if bits == 4 else dict(group=None)
    def q(W):
        return ckl.QuantWeights(bits, W, group=kw["group"] or W.shape[1], asym=kw.get("asym", False))
    return q(mk(E, d, F)), q(mk(E, d, F)), q(mk(E, F, d))


def _one_rank(ckl, T_cap, k, E, d):
    return ckl.EpWindows(0, 1, T_cap, k, E, d, lambda h: [h])


@pytest.mark.parametrize("E,k,d,F,bits,T", [(64, 6, 2048, 1408, 4, 1), (64, 6, 2048, 1408, 4, 16),
                                             (64, 6, 2048, 1408, 4, 64), (8, 2, 512, 768, 8, 5),
                                             (8, 2, 512, 768, 16, 33)])
def test_world1_equals_single_gpu_layer(ckl, dev, E, k, d, F, bits, T):
    import torch
    gq, uq, dq = _weights(ckl, dev, E, d, F, bits, seed=E + T)
    g = torch.Generator(device=dev)
    g.manual_seed(100 + T)
    lg = torch.randn((T, E), generator=g, device=dev)
    X = torch.randn((T, d), generator=g, device=dev).half()
    ref = ckl.MoeLayer(gq, uq, dq).forward(lg, X, k)
    win = _one_rank(ckl, T, k, E, d)
    try:
        layer = ckl.MoeEpLayer(win, gq, uq, dq)
        ids = torch.empty((T, k), dtype=torch.int32, device=dev)
        wts = torch.empty((T, k), dtype=torch.float32, device=dev)
        outs = [layer.forward(lg, X, ids=ids, wts=wts) for _ in range(3)]   # epochs 1..3
        torch.cuda.synchronize()
        ckl.check_device_error()
        for o in outs:
            assert torch.equal(o, ref)
    finally:
        torch.cuda.synchronize()
        win.close()


def test_world1_fewer_tokens_than_capacity_and_graph_replay(ckl, oracle, dev):
    import torch
    E, k, d, F, T_cap = 64, 6, 2048, 1408, 64
    gq, uq, dq = _weights(ckl, dev, E, d, F, 4, seed=7)
    win = _one_rank(ckl, T_cap, k, E, d)
    try:
        layer = ckl.MoeEpLayer(win, gq, uq, dq)
        g = torch.Generator(device=dev)
        g.manual_seed(8)
        for T in (0, 3, 17):
            lg = torch.randn((max(T, 1), E), generator=g, device=dev)[:T].contiguous()
            X = torch.randn((max(T, 1), d), generator=g, device=dev).half()[:T].contiguous()
            out = layer.forward(lg, X)
            torch.cuda.synchronize()
            ckl.check_device_error()
            if T:
                ref = ckl.MoeLayer(gq, uq, dq).forward(lg, X, k)
                assert rel_rms(out.float().cpu(), ref.float().cpu()) < 1e-3
        # the epochs live on the device: a captured call replays correctly
        T = 9
        lg = torch.randn((T, E), generator=g, device=dev)
        X = torch.randn((T, d), generator=g, device=dev).half()
        out = torch.empty((T, d), dtype=torch.float16, device=dev)
        ws = torch.empty(layer.workspace_size(), dtype=torch.uint8, device=dev)
        s = torch.cuda.Stream()
        s.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(s):
            layer.forward(lg, X, out=out, workspace=ws, stream=s)
        torch.cuda.current_stream().wait_stream(s)
        first = out.clone()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=s):
            layer.forward(lg, X, out=out, workspace=ws, stream=s)
        for _ in range(3):
            out.zero_()
            graph.replay()
            torch.cuda.synchronize()
            ckl.check_device_error()
            assert torch.equal(out, first)
        del graph
    finally:
        torch.cuda.synchronize()
        win.close()


def test_wait_gives_up_on_a_flag_nothing_sets(ckl, dev):
    """A world-2 communicator whose rank-1 window is a local buffer: nobody raises rank 1's
    dispatch or ready flags, so the receive and combine waits must time out (bounded), the
    error word must report CKL_TIMEOUT, and the device must stay usable."""
    import torch
    E, k, d, F, T = 8, 2, 256, 256, 4
    gq, uq, dq = _weights(ckl, dev, E // 2, d, F, 4, seed=3)
    L = ckl._LibWindows
    nbytes = ckl.ep_window_bytes(2, T, k, E, d)
    w0, _ = L.alloc(nbytes)
    w1, _ = L.alloc(nbytes)
    try:
        win = type("W", (), {})()
        win.d = d
        wins = (ckl.C.c_void_p * ckl.EP_MAX_RANKS)(w0, w1)
        win.comm = ckl.MoeEpComm(0, 2, T, k, E, d, wins)
        layer = ckl.MoeEpLayer(win, gq, uq, dq)
        lg = torch.randn((T, E), device=dev)
        X = torch.randn((T, d), device=dev).half()
        ckl.set_spin_timeout_ns(20_000_000)            # 20 ms
        layer.forward(lg, X)
        torch.cuda.synchronize()
        with pytest.raises(ckl.CklError) as e:
            ckl.check_device_error()
        assert e.value.status == 5                      # CKL_TIMEOUT
    finally:
        ckl.set_spin_timeout_ns(1_000_000_000)
        torch.cuda.synchronize()
        L.free(w0)
        L.free(w1)
    # the context is still usable
    win = _one_rank(ckl, T, k, E // 2, d)
    try:
        lg = torch.randn((T, E // 2), device=dev)
        X = torch.randn((T, d), device=dev).half()
        out = ckl.MoeEpLayer(win, gq, uq, dq).forward(lg, X)
        ref = ckl.MoeLayer(gq, uq, dq).forward(lg, X, k)
        torch.cuda.synchronize()
        ckl.check_device_error()
        assert torch.equal(out, ref)
    finally:
        torch.cuda.synchronize()
        win.close()


def test_world1_token_bound(ckl, dev):
    """ckl_moe_ep_layer_ex: with T_max the GEMM grids are sized for world * T_max * min(k,
    E_loc) rows; the output equals the unbounded layer's. A bound below the rows a rank
    actually receives is refused on the host when it is the rank's own T, and recorded on
    the device (CKL_INVALID_ARG from ckl_check_device_error) when it is another rank's."""
    import torch
    E, k, d, F, T_cap = 64, 6, 2048, 1408, 64
    gq, uq, dq = _weights(ckl, dev, E, d, F, 4, seed=11)
    win = _one_rank(ckl, T_cap, k, E, d)
    try:
        layer = ckl.MoeEpLayer(win, gq, uq, dq)
        g = torch.Generator(device=dev)
        g.manual_seed(12)
        for T in (1, 4, 16):
            lg = torch.randn((T, E), generator=g, device=dev)
            X = torch.randn((T, d), generator=g, device=dev).half()
            ref = layer.forward(lg, X)
            got = layer.forward(lg, X, T_max=T)
            torch.cuda.synchronize()
            ckl.check_device_error()
            assert torch.equal(got, ref), T
        with pytest.raises(ckl.CklError) as ei:            # T above this call's bound
            layer.forward(lg, X, T_max=T - 1)
        assert ei.value.status == 1
        with pytest.raises(ckl.CklError):                   # bound above the capacity
            layer.forward(lg, X, T_max=T_cap + 1)
        torch.cuda.synchronize()
        ckl.check_device_error()                            # nothing recorded by the refusals
    finally:
        torch.cuda.synchronize()
        win.close()
