"""One rank of the multi-GPU tests (run by test_multi_gpu.py under torchrun, one process
per GPU). Every rank builds the same seeded problems on its own device.

Attention by KV head: each rank decodes its heads' shard and writes the rows straight into
rank 0's output (ckl_decode_attention_gather over a peer-mapped buffer), signals, and rank 0
waits (ckl_gather_wait) and compares the gathered output with the full single-GPU decode
under the same split: a head's rows do not depend on other heads, so they must be equal.
One long sequence (B=1) by its chunks: each rank holds only its run of the plan's chunks,
writes those partial slots into rank 0's buffers, and rank 0 merges them (bit-identical to
the single-GPU decode with the same plan).

MoE by expert: each rank packs only its own experts, runs ckl_moe_ep_layer on its share of
the tokens and checks the routing against the oracle, the output against the single-GPU
layer over all experts (ckl_moe_layer, same device) and a fp32 torch reference,
repeatability across calls and CUDA-graph replay.

On success each rank writes its results to $CKL_EP_RESULT_DIR/rank<r>.json."""
import json
import os
import sys
from datetime import timedelta

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path[:0] = [os.path.join(ROOT, "cuda-kernel-lab_b200"), os.path.join(ROOT, "oracle")]


def rel_rms(got, ref):
    got, ref = np.asarray(got, np.float64), np.asarray(ref, np.float64)
    return float(np.linalg.norm(got - ref) / max(np.linalg.norm(ref), 1e-30))


def torch_ref(X, ids, wts, Wg, Wu, Wd):
    import torch
    out = torch.zeros((X.shape[0], Wd.shape[2]), dtype=torch.float32, device=X.device)
    for t in range(X.shape[0]):
        for j in range(ids.shape[1]):
            e = int(ids[t, j])
            g, u = X[t].float() @ Wg[e], X[t].float() @ Wu[e]
            h = (torch.nn.functional.silu(g) * u).half().float()
            out[t] += wts[t, j] * (h @ Wd[e])
    return out


def case(ckl, oracle, rank, world, dev, name, E, k, d, F, bits, T_all, exchange):
    import torch
    g = torch.Generator(device=dev)
    g.manual_seed(1234)
    mk = lambda *s: (torch.randn(*s, generator=g, device=dev) * 0.02).half()
    W = [mk(E, d, F), mk(E, d, F), mk(E, F, d)]
    T = sum(T_all)
    lg_all = torch.randn((T, E), generator=g, device=dev)
    X_all = torch.randn((T, d), generator=g, device=dev).half()
    E_loc = E // world
    lo = rank * E_loc
    q = lambda w: ckl.QuantWeights(bits, w.contiguous(), group=128 if bits == 4 else w.shape[1],
                                   asym=bits == 4)
    loc = [q(w[lo:lo + E_loc]) for w in W]
    full = [q(w) for w in W]
    del W
    t0 = sum(T_all[:rank])
    Tr = T_all[rank]
    lg, X = lg_all[t0:t0 + Tr].contiguous(), X_all[t0:t0 + Tr].contiguous()

    win = ckl.EpWindows(rank, world, max(T_all), k, E, d, exchange)
    res = {"case": name}
    try:
        layer = ckl.MoeEpLayer(win, *loc)
        ids = torch.empty((Tr, k), dtype=torch.int32, device=dev)
        wts = torch.empty((Tr, k), dtype=torch.float32, device=dev)
        outs = [layer.forward(lg, X, ids=ids, wts=wts).clone() for _ in range(3)]
        torch.cuda.synchronize()
        ckl.check_device_error()
        for o in outs[1:]:
            assert torch.equal(o, outs[0]), "EP layer not repeatable"
        # graph replay (every rank captures and replays the same number of calls)
        out = torch.empty((Tr, d), dtype=torch.float16, device=dev)
        ws = torch.empty(layer.workspace_size(), dtype=torch.uint8, device=dev)
        s = torch.cuda.Stream()
        s.wait_stream(torch.cuda.current_stream())
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=s):
            layer.forward(lg, X, out=out, workspace=ws, stream=s)
        for _ in range(3):
            graph.replay()
        torch.cuda.synchronize()
        ckl.check_device_error()
        assert torch.equal(out, outs[0]), "graph replay differs"
        del graph
        # the per-call token bound (ckl_moe_ep_layer_ex) sizes the grids; same result
        bounded = layer.forward(lg, X, T_max=max(T_all))
        torch.cuda.synchronize()
        ckl.check_device_error()
        assert torch.equal(bounded, outs[0]), "T_max-bounded layer differs"
        if Tr:
            rids, _ = oracle.route(lg.cpu().numpy(), k)
            assert np.array_equal(ids.cpu().numpy(), rids), "routing"
            single = ckl.MoeLayer(*full).forward(lg, X, k)
            res["rel_rms_vs_single_gpu"] = rel_rms(outs[0].float().cpu(), single.float().cpu())
            ref = torch_ref(X, ids, wts, *[f.dequant() for f in full])
            res["rel_rms_vs_fp32"] = rel_rms(outs[0].float().cpu(), ref.cpu())
            assert res["rel_rms_vs_single_gpu"] < 1e-3, res
            assert res["rel_rms_vs_fp32"] <= 1e-2, res
    finally:
        torch.cuda.synchronize()
        import torch.distributed as dist
        dist.barrier()             # no rank unmaps a window a peer may still touch
        win.close()
    return res


def attention_case(ckl, oracle, rank, world, dev, name, lens, force_chunks, exchange):
    import torch
    HQ, HKV, D = 32, 8, 128
    bt = oracle.batch(lens, HQ, HKV, seed=77)               # host arrays, every rank the same
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(dev)
    k_all, v_all, q_all = t(bt.k).view(-1, 16, HKV, D), t(bt.v).view(-1, 16, HKV, D), t(bt.q)
    hk, hq = HKV // world, HQ // world
    ks = k_all[:, :, rank * hk:(rank + 1) * hk].contiguous()
    vs = v_all[:, :, rank * hk:(rank + 1) * hk].contiguous()
    qs = q_all[:, rank * hq:(rank + 1) * hq].contiguous()
    B = len(lens)
    nc, ct = ckl.plan_chunks(4, B, HKV, int(max(lens)), force_chunks=force_chunks)
    indptr, indices, last = t(bt.indptr), t(bt.indices), t(bt.last)
    p = ckl.make_params(qs, ks, vs, indptr, indices, last, num_chunks=nc, chunk_tokens=ct)
    ws = torch.empty(max(ckl.workspace_size(p), 256), dtype=torch.uint8, device=dev)
    out_bytes = (B * HQ * D * 2 + 255) // 256 * 256
    win = ckl.IpcWindows(rank, world, out_bytes + B * HQ * 4, exchange)
    grp = ckl.GatherGroup(rank, world, exchange)
    res = {"case": name}
    try:
        root_out, root_lse = win.ptrs[0], win.ptrs[0] + out_bytes
        for _ in range(2):                                   # the epochs advance per call
            ckl.decode_attention_gather(p, root_out, root_lse, HQ, rank * hq, workspace=ws)
            grp.signal(0)
            if rank == 0:
                grp.wait()
        torch.cuda.synchronize()
        ckl.check_device_error()
        if rank == 0:
            got = ckl.device_view(root_out, (B, HQ, D), torch.float16)
            got_lse = ckl.device_view(root_lse, (B, HQ), torch.float32)
            ref, ref_lse = ckl.decode_attention(q_all, k_all, v_all, indptr, indices, last,
                                                force_chunks=nc)
            torch.cuda.synchronize()
            assert torch.equal(got, ref), "gathered out differs from the single-GPU decode"
            assert torch.equal(got_lse, ref_lse), "gathered lse differs"
            ora = oracle.attention_ref(bt)
            res["max_abs_vs_fp64"] = float(np.abs(got.float().cpu().numpy() - ora[0]).max())
            assert res["max_abs_vs_fp64"] <= 2e-3, res
    finally:
        torch.cuda.synchronize()
        win.close()
        grp.close()
    return res


def seqsplit_case(ckl, oracle, rank, world, dev, name, L, exchange):
    """One long sequence split by its chunks over the ranks (B=1): rank r holds only the
    pages of its chunk run [lo_r, hi_r) of the single-GPU plan, runs the partial kernel over
    them (ckl_decode_partial with chunk_base = lo_r, part_stride = all chunks) with the
    partial buffers in rank 0's window, signals; rank 0 waits and runs the LSE merge. The
    slots are the single-GPU decode's slots, so the result equals it bit for bit."""
    import torch
    HQ, HKV, D, PAGE = 32, 8, 128, 16
    bt = oracle.batch([L], HQ, HKV, seed=91)
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(dev)
    k_all, v_all, q = t(bt.k).view(-1, PAGE, HKV, D), t(bt.v).view(-1, PAGE, HKV, D), t(bt.q)
    nc, ct = ckl.plan_chunks(HQ // HKV, 1, HKV, L)
    assert nc >= world, (nc, world)
    lo, hi = rank * nc // world, (rank + 1) * nc // world
    t0, t1 = lo * ct, min(hi * ct, L)
    pages = bt.indices[t0 // PAGE:(t1 + PAGE - 1) // PAGE]
    pi = torch.from_numpy(pages.astype(np.int64)).to(dev)
    kl, vl = k_all.index_select(0, pi).contiguous(), v_all.index_select(0, pi).contiguous()
    n = len(pages)
    ip = t(np.array([0, n], np.int32))
    ix = t(np.arange(n, dtype=np.int32))
    ls = t(np.array([t1 - t0 - (n - 1) * PAGE], np.int32))
    p = ckl.make_params(q, kl, vl, ip, ix, ls, num_chunks=hi - lo, chunk_tokens=ct,
                        chunk_base=lo, part_stride=nc)
    o_bytes = (HQ * nc * D * 4 + 255) // 256 * 256
    win = ckl.IpcWindows(rank, world, o_bytes + HQ * nc * 4, exchange)
    grp = ckl.GatherGroup(rank, world, exchange)
    res = {"case": name, "chunks": nc, "rank_chunks": [lo, hi]}
    try:
        p.part_o, p.part_lse = win.ptrs[0], win.ptrs[0] + o_bytes
        out = torch.empty((1, HQ, D), dtype=torch.float16, device=dev)
        lse = torch.empty((1, HQ), dtype=torch.float32, device=dev)
        for _ in range(2):                                   # the epochs advance per call
            ckl.decode_partial(p)
            grp.signal(0)
            if rank == 0:
                grp.wait()
                po = ckl.device_view(win.ptrs[0], (HQ, nc, D), torch.float32)
                pl = ckl.device_view(win.ptrs[0] + o_bytes, (HQ, nc), torch.float32)
                ckl.merge_states(po, pl, out, lse)
        torch.cuda.synchronize()
        ckl.check_device_error()
        if rank == 0:
            ref, ref_lse = ckl.decode_attention(q, k_all, v_all, t(bt.indptr), t(bt.indices),
                                                t(bt.last), num_chunks=nc, chunk_tokens=ct)
            torch.cuda.synchronize()
            assert torch.equal(out, ref), "sequence-split out differs from the single-GPU decode"
            assert torch.equal(lse, ref_lse), "sequence-split lse differs"
            ora = oracle.attention_ref(bt)
            res["max_abs_vs_fp64"] = float(np.abs(out.float().cpu().numpy() - ora[0]).max())
            assert res["max_abs_vs_fp64"] <= 2e-3, res
    finally:
        torch.cuda.synchronize()
        win.close()
        grp.close()
    return res


def main():
    import torch
    import torch.distributed as dist
    import ckl
    import oracle
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    local = int(os.environ.get("LOCAL_RANK", rank))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist.init_process_group("gloo", timeout=timedelta(seconds=120))
    ex = ckl.torch_exchange()
    out = []
    out.append(attention_case(ckl, oracle, rank, world, dev, "attn_config1_3chunks",
                              [1000, 777], 3, ex))
    out.append(attention_case(ckl, oracle, rank, world, dev, "attn_64x1024_direct",
                              [1024] * 64, 1, ex))
    out.append(seqsplit_case(ckl, oracle, rank, world, dev, "attn_B1_seqsplit_8000", 8000, ex))
    T4 = [64] * world
    out.append(case(ckl, oracle, rank, world, dev, "config4_T64_per_rank", 64, 6, 2048, 1408, 4, T4, ex))
    ragged = [(5 * r + 1) % 17 for r in range(world)]
    ragged[-1] = 0                                         # a rank with no tokens
    out.append(case(ckl, oracle, rank, world, dev, "config4_ragged", 64, 6, 2048, 1408, 4, ragged, ex))
    out.append(case(ckl, oracle, rank, world, dev, "config5_T32", 8, 2, 4096, 14336, 8,
                    [32 // world + (r < 32 % world) for r in range(world)], ex))
    dist.barrier()
    rdir = os.environ.get("CKL_EP_RESULT_DIR")
    if rdir:
        with open(os.path.join(rdir, f"rank{rank}.json"), "w") as f:
            json.dump(out, f)
    print("EP_OK", rank, json.dumps(out), flush=True)
    dist.destroy_process_group()


if __name__ == "__main__":
    try:
        main()
    except BaseException:
        import traceback
        r = os.environ.get("RANK", "?")
        for line in traceback.format_exc().splitlines():
            print(f"[rank{r}] {line}", flush=True)
        raise
