"""CPU tests of the expert-parallel MoE path over two gloo ranks (no GPU).

The GPU layer (ckl_moe_ep_layer) moves rows through IPC-mapped windows; here the same
placement -- dispatch slab positions, the owner's gather map, the pull-back for the
combine -- is restated with numpy (oracle.ep_dispatch / ep_receive), the rows are exchanged
with gloo collectives, and the result must equal the single-process oracle layer
(03_moe_wq_decode.cu:471-479 semantics, SwiGLU). The window handle exchange of
ckl.EpWindows is checked with a fake IPC backend over the same process group.
"""
import ctypes as C
import os
import socket
import sys
from datetime import timedelta

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _problem(E=8, d=256, F=256, k=2, T_all=(5, 3)):
    import oracle as O
    T = sum(T_all)
    logits = O.normal((T, E), seed=3, fp16=False).astype(np.float32)
    X = O.normal((T, d), seed=4)
    mats = []
    for i, (K, N) in enumerate(((d, F), (d, F), (F, d))):
        W = O.normal((E, K, N), seed=10 + i, std=0.02)
        codes, s, z = O.quant_asym4(W)
        mats.append(O.dequant(codes, s, z, 4))
    return logits, X, mats


class _FakeIpc:
    """Stands in for CUDA IPC: rank r's window is 0x1000*(r+1); handles name the rank."""

    def __init__(self, rank):
        self.rank, self.closed, self.freed = rank, [], []

    def alloc(self, nbytes):
        return 0x1000 * (self.rank + 1), b"win%d" % self.rank

    def open(self, handle):
        return 0x1000 * (int(handle[3:]) + 1)

    def close(self, p):
        self.closed.append(p)

    def free(self, p):
        self.freed.append(p)


def _worker(rank, world, port, T_all, out_q):
    import torch.distributed as dist
    sys.path[:0] = [os.path.join(ROOT, "oracle"), os.path.join(ROOT, "cuda-kernel-lab_b200")]
    import oracle as O
    import ckl
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank,
                            world_size=world, timeout=timedelta(seconds=60))
    try:
        E, k = 8, 2
        logits, X, (Wg, Wu, Wd) = _problem(E=E, k=k, T_all=T_all)
        d = X.shape[1]
        E_loc = E // world
        T_cap = max(T_all)
        cap = T_cap * min(k, E_loc)
        t0 = sum(T_all[:rank])
        T = T_all[rank]
        lg, x = logits[t0:t0 + T], X[t0:t0 + T]

        # ---- route this rank's tokens; dispatch placement
        ids, wts = O.route(lg, k)
        counts, offsets, _, inv = O.permute(ids, E)
        owner, pos = O.ep_dispatch(ids, inv, offsets, E_loc)
        assert (pos >= 0).all() and (pos < cap).all()
        slabs = {}
        for o in range(world):
            rows = np.zeros((cap, d), np.float16)
            sel = np.nonzero(owner == o)[0]
            assert len(set(pos[sel].tolist())) == len(sel)       # positions unique per owner
            rows[pos[sel]] = x[sel // k]
            slabs[o] = (rows, counts[o * E_loc:(o + 1) * E_loc].copy())
        sent = [None] * world
        dist.all_gather_object(sent, slabs)

        # ---- owner: receive, gather, local experts, outputs at slab positions
        counts_from = np.stack([sent[s][rank][1] for s in range(world)])
        off_loc, row_src = O.ep_receive(counts_from, cap)
        recv = np.concatenate([sent[s][rank][0] for s in range(world)])
        Xg = recv[row_src]
        e_of_row = np.searchsorted(off_loc, np.arange(len(row_src)), side="right") - 1
        lo = rank * E_loc
        y = O.moe_layer(Xg, e_of_row[:, None].astype(np.int32), np.ones((len(row_src), 1)),
                        Wg[lo:lo + E_loc], Wu[lo:lo + E_loc], Wd[lo:lo + E_loc]) \
            if len(row_src) else np.zeros((0, d), np.float32)
        ywin = np.zeros((world * cap, d), np.float32)
        ywin[row_src] = y
        ys = [None] * world
        dist.all_gather_object(ys, ywin)

        # ---- source: pull its rows back, fixed-order combine
        out = np.zeros((T, d), np.float64)
        for i in range(T * k):
            out[i // k] += wts.reshape(-1)[i] * ys[owner[i]][rank * cap + pos[i]]

        # ---- the window handle exchange of ckl.EpWindows (fake IPC, same group)
        fake = _FakeIpc(rank)
        win = ckl.EpWindows(rank, world, T_cap, k, E, d, ckl.torch_exchange(), ipc=fake)
        ptrs = [win.comm.windows[i] for i in range(world)]
        win.close()
        out_q.put((rank, out, ids, wts, ptrs, fake.closed, fake.freed))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("T_all", [(5, 3), (4, 0)])
def test_expert_parallel_two_ranks_matches_single_process(T_all, oracle):
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, T_all, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = {}
    for _ in procs:
        r, *rest = q.get(timeout=240)
        res[r] = rest
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0

    E, k = 8, 2
    logits, X, (Wg, Wu, Wd) = _problem(E=E, k=k, T_all=T_all)
    ids, wts = oracle.route(logits, k)
    ref = oracle.moe_layer(X, ids, wts, Wg, Wu, Wd)
    t0 = 0
    for r in range(2):
        out, rids, rwts, ptrs, closed, freed = res[r]
        T = T_all[r]
        np.testing.assert_array_equal(rids, ids[t0:t0 + T])          # routing per token
        np.testing.assert_array_equal(rwts, wts[t0:t0 + T])
        if T:
            err = np.abs(out - ref[t0:t0 + T]).max() / max(np.abs(ref).max(), 1e-30)
            assert err < 1e-6, err
        assert ptrs == [0x1000, 0x2000]                              # windows in rank order
        assert closed == [0x2000 if r == 0 else 0x1000] and freed == [0x1000 * (r + 1)]
        t0 += T


def test_ep_window_layout_and_argument_checks(ckl):
    # world 8, T_cap 64, k 6, E 64, d 2048: cap = 64 * min(6, 8) = 384 rows per source
    cap, A = 384, 8 * 384
    rows = (256 + 8 * 8 * 4 + 255) // 256 * 256
    y = rows + A * 2048 * 2
    assert ckl.ep_window_bytes(8, 64, 6, 64, 2048) == y + A * 2048 * 4
    assert ckl.ep_window_bytes(3, 64, 6, 64, 2048) == 0            # E % world != 0
    assert ckl.ep_window_bytes(9, 64, 6, 72, 2048) == 0            # world > 8
    lib = ckl.lib()
    comm = ckl.MoeEpComm(0, 2, 4, 2, 8, 256)
    w = ckl.MoeWeights(4, 4, 256, 256, 128, 1, None, None, None)
    args = (None, None, 1, C.byref(w), C.byref(w), C.byref(w), None, None, None, None, 0, None)
    assert lib.ckl_moe_ep_layer(C.byref(comm), *args) == 1         # NULL windows
    comm.windows[0], comm.windows[1] = 0x10000, 0x20000
    comm.E = 7
    assert lib.ckl_moe_ep_layer(C.byref(comm), *args) == 2         # E % world
    comm.E = 8
    comm.world = 9
    assert lib.ckl_moe_ep_layer(C.byref(comm), *args) == 1         # world > 8
    comm.world = 2
    comm.T_cap = 0
    with pytest.raises(ckl.CklError):
        ckl.check(lib.ckl_moe_ep_layer(C.byref(comm), *args), "ep")
    comm.T_cap = 4
    args_big = (None, None, 5) + args[3:]                          # T > T_cap
    assert lib.ckl_moe_ep_layer(C.byref(comm), *args_big) == 1


class _HostOps:
    """The library calls the NCCL expert-parallel designs of bench.py make, restated on the
    host (routing and slot order from the oracle; the SwiGLU intermediate rounded to fp16
    and the down projection kept in fp32, as the GPU GEMMs write them). Rows the offsets do
    not cover stay NaN, so a design that reads one fails."""

    class W:
        def __init__(self, W):
            self.W, self.E, self.N = W, W.shape[0], W.shape[2]

    def __init__(self, oracle):
        self.O = oracle

    def route_and_permute(self, lg, X, k):
        import torch
        ids, wts = self.O.route(lg.numpy(), k)
        counts, offsets, _, inv = self.O.permute(ids, lg.shape[1])
        Xp = torch.empty((X.shape[0] * k, X.shape[1]), dtype=torch.float16)
        Xp[torch.from_numpy(inv).long()] = X.repeat_interleave(k, 0)
        t = lambda a: torch.from_numpy(np.ascontiguousarray(a))
        return dict(ids=t(ids), wts=t(wts.astype(np.float32)), counts=t(counts),
                    offsets=t(offsets), inv_perm=t(inv), Xp=Xp)

    def expert_gemm_ex(self, X, row_src, offsets, A, gate, up=None, y_f32=False):
        import torch
        Y = torch.full((A, gate.N), float("nan"),
                       dtype=torch.float32 if y_f32 else torch.float16)
        off = offsets.tolist()
        for e in range(gate.E):
            rows = torch.arange(off[e], off[e + 1])
            if not len(rows):
                continue
            x = (X[row_src[rows].long()] if row_src is not None else X[rows]).double().numpy()
            if up is not None:
                g, u = x @ gate.W[e], x @ up.W[e]
                y = (g / (1 + np.exp(-g)) * u).astype(np.float16)
            else:
                y = (x @ gate.W[e]).astype(np.float32 if y_f32 else np.float16)
            Y[rows] = torch.from_numpy(y)
        return Y

    def combine(self, Yp, inv_perm, wts, T, k):
        import torch
        y = Yp.double()[inv_perm.long()].view(T, k, -1)
        return (y * wts.double().unsqueeze(2)).sum(1).half()


def _designs_worker(rank, world, port, T_all, out_q):
    import torch
    import torch.distributed as dist
    sys.path[:0] = [os.path.join(ROOT, "oracle"), ROOT]
    import oracle as O
    import bench
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank,
                            world_size=world, timeout=timedelta(seconds=60))
    try:
        E, k = 8, 3
        logits, X, mats = _problem(E=E, k=k, T_all=T_all)
        E_loc = E // world
        ops = _HostOps(O)
        q = [_HostOps.W(m[rank * E_loc:(rank + 1) * E_loc]) for m in mats]
        t0, T = sum(T_all[:rank]), T_all[rank]
        lg = torch.from_numpy(logits[t0:t0 + T].copy())
        x = torch.from_numpy(X[t0:t0 + T].copy())
        Tmax = max(T_all)
        a2a = bench.ep_a2a_layer(ops, q, lg, x, k, world, Tmax * min(k, E_loc))
        rep = bench.ep_replicated_layer(ops, q, lg, x, k, rank, world, Tmax)
        out_q.put((rank, a2a.float().numpy(), rep.float().numpy()))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("T_all", [(5, 3), (4, 0), (1, 1)])
def test_nccl_ep_designs_two_ranks_match_single_process(T_all, oracle):
    """bench.py's NCCL all-to-all and replicated + reduce-scatter expert-parallel layers (the
    designs timed beside ckl_moe_ep_layer) on two gloo ranks against the single-process
    layer with the same roundings."""
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_designs_worker, args=(r, 2, port, T_all, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = {}
    for _ in procs:
        r, *rest = q.get(timeout=240)
        res[r] = rest
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0

    E, k = 8, 3
    logits, X, (Wg, Wu, Wd) = _problem(E=E, k=k, T_all=T_all)
    ids, wts = oracle.route(logits, k)
    x = X.astype(np.float64)
    ref = np.zeros((len(X), Wd.shape[2]))
    for t in range(len(X)):
        for j in range(k):
            e = ids[t, j]
            g, u = x[t] @ Wg[e], x[t] @ Wu[e]
            h = (g / (1 + np.exp(-g)) * u).astype(np.float16).astype(np.float64)
            ref[t] += wts[t, j].astype(np.float32) * (h @ Wd[e]).astype(np.float32)
    t0 = 0
    for r in range(2):
        T = T_all[r]
        for out in res[r]:
            assert out.shape == (T, Wd.shape[2]) and np.isfinite(out).all()
            if T:
                err = np.abs(out - ref[t0:t0 + T]).max() / np.abs(ref).max()
                assert err < 2e-3, err
        t0 += T
