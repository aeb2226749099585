"""Same-box comparator: this library's kernels against the reference's OWN GPU kernels, built
from its unmodified sources for sm_100a (oracle/_ref, through oracle/ref_shim_01.cu and
oracle/ref_shim_03.cu), on the same inputs, the same B200 and the same timing method.

TEST INFRASTRUCTURE, not the product: it loads the reference-compiled libraries and is run by
hand on a GPU box (its summary is profiles/ref_gpu_comparator.md):

    python tests/ref_gpu_compare.py [--out result.json] [--iters 31]

Rows (cold L2: 512 MB memset before every sample, median of --iters, CUDA events):
  * decode: the reference's decode_attention (01_decode_attention.cu:316-331, its best
    variant decode_partial<4,3> + merge_states, planned by its plan_chunks) against
    ckl_decode_attention on every BASELINE config-2 shape;
  * cascade: the reference's cascade_decode (01:703-712, planned by plan_cascade) against
    ckl_cascade_decode on BASELINE config 3 (64 x (4096 + 256) and a ragged suffix);
  * int4 expert GEMM: the reference's QuantWeights::run (03:318-332, symmetric int4 g128)
    against ckl_moe_expert_gemm on the same symmetric codes (E=64, d=2048 -> f=1408,
    T in {1, 4, 16, 64} routed top-6).
Every row also reports the largest difference between the two outputs.
"""
import argparse
import json
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
for p in (os.path.join(ROOT, "cuda-kernel-lab_b200"), os.path.join(ROOT, "oracle"), ROOT):
    if p not in sys.path:
        sys.path.insert(0, p)

HQ, HKV, D = 32, 8, 128


def _vp(t):
    import ctypes as C
    return C.c_void_p(0 if t is None else t.data_ptr())


def decode_row(ckl, O, bench, dev, timer, name, timed=True):
    import torch
    lens = bench.lengths(name)
    d, _ = bench.paged_batch(lens, dev, seed=7)
    B = len(lens)
    nc, ct = ckl.plan_chunks(HQ // HKV, B, HKV, int(lens.max()))
    p = ckl.make_params(**d, num_chunks=nc, chunk_tokens=ct)
    out = torch.empty_like(d["q"])
    lse = torch.empty((B, HQ), dtype=torch.float32, device=dev)
    ws = torch.empty(max(ckl.workspace_size(p), 256), dtype=torch.uint8, device=dev)
    ours = lambda: ckl.decode_attention(**d, num_chunks=nc, chunk_tokens=ct, out=out, lse=lse,
                                        workspace=ws)
    L = O.ref01()
    plan = L.ref01_decode_plan(_vp(d["q"]), _vp(d["k_cache"]), _vp(d["v_cache"]), _vp(d["kv_indptr"]),
                               _vp(d["kv_indices"]), _vp(d["kv_last_page_len"]), B, HQ, HKV,
                               int(lens.max()), 3)
    rout = torch.empty_like(out)
    rlse = torch.empty_like(lse)
    stream = torch.cuda.current_stream().cuda_stream
    import ctypes as C
    ref = lambda: L.ref01_decode_run(plan, _vp(rout), _vp(rlse), C.c_void_p(stream))
    try:
        ours()
        ref()
        torch.cuda.synchronize()
        diff = float((out.float() - rout.float()).abs().max())
        row = {"max_abs_diff": diff, "ref_chunks": L.ref01_decode_plan_chunks(plan), "our_chunks": nc}
        if timed:
            t_o, t_r = timer(ours), timer(ref)
            byts = bench.algorithmic_bytes(lens)
            row.update({"ours_us": round(t_o * 1e3, 1), "reference_us": round(t_r * 1e3, 1),
                        "ours_GB/s": round(byts / (t_o * 1e-3) / 1e9, 1),
                        "reference_GB/s": round(byts / (t_r * 1e-3) / 1e9, 1),
                        "speedup": round(t_r / t_o, 2)})
        return row
    finally:
        torch.cuda.synchronize()
        L.ref01_decode_free(plan)


def cascade_row(ckl, O, bench, dev, timer, suffix, timed=True):
    import ctypes as C
    import torch
    Lp = 4096
    lens = (Lp + np.asarray(suffix)).astype(np.int32)
    d, (lens, indptr, indices) = bench.paged_batch(lens, dev, seed=21, Lp=Lp)
    B = len(lens)
    base = ckl.make_params(**d, num_chunks=1, chunk_tokens=16)
    cp = ckl.plan_cascade(base, indptr, indices, lens, 256)
    ws = torch.empty(max(ckl.cascade_workspace_size(cp), 256), dtype=torch.uint8, device=dev)
    out = torch.empty_like(d["q"])
    lse = torch.empty((B, HQ), dtype=torch.float32, device=dev)
    ours = lambda: ckl.cascade_decode(cp, out=out, lse=lse, workspace=ws)
    L = O.ref01()
    hi, hx, hl = (np.ascontiguousarray(a, dtype=np.int32) for a in (indptr, indices, lens))
    plan = L.ref01_cascade_plan(_vp(d["q"]), _vp(d["k_cache"]), _vp(d["v_cache"]), _vp(d["kv_indptr"]),
                                _vp(d["kv_indices"]), _vp(d["kv_last_page_len"]),
                                hi.ctypes.data_as(C.c_void_p), hx.ctypes.data_as(C.c_void_p),
                                hl.ctypes.data_as(C.c_void_p), B, HQ, HKV, 256)
    rout = torch.empty_like(out)
    rlse = torch.empty_like(lse)
    stream = torch.cuda.current_stream().cuda_stream
    ref = lambda: L.ref01_cascade_run(plan, _vp(rout), _vp(rlse), C.c_void_p(stream))
    try:
        assert cp.use == 1 and L.ref01_cascade_use(plan) == 1
        ours()
        ref()
        torch.cuda.synchronize()
        row = {"max_abs_diff": float((out.float() - rout.float()).abs().max())}
        if timed:
            t_o, t_r = timer(ours), timer(ref)
            row.update({"ours_us": round(t_o * 1e3, 1), "reference_us": round(t_r * 1e3, 1),
                        "speedup": round(t_r / t_o, 2)})
        return row
    finally:
        torch.cuda.synchronize()
        L.ref01_cascade_free(plan)


def gemm_row(ckl, O, dev, timer, T, timed=True, E=64, k=6, d=2048, f=1408):
    import ctypes as C
    import torch
    g = torch.Generator(device=dev)
    g.manual_seed(900 + T)
    W = (torch.randn((E, d, f), generator=g, device=dev) * 0.02).half()
    lg = torch.randn((T, E), generator=g, device=dev)
    X = torch.randn((T, d), generator=g, device=dev).half()
    r = ckl.route_and_permute(lg, X, k)
    A = T * k
    q = ckl.QuantWeights(4, W, group=128)                 # symmetric, the reference's codes
    Y = torch.empty((A, f), dtype=torch.float16, device=dev)
    ws = torch.empty(max(q.workspace_size(A), 256), dtype=torch.uint8, device=dev)
    ours = lambda: q.run(r["Xp"], Y, r["offsets"], A, workspace=ws)
    L = O.ref03()
    qw = L.ref03_quant_make(4, _vp(W), E, d, f)
    RY = torch.empty_like(Y)
    stream = torch.cuda.current_stream().cuda_stream
    ref = lambda: L.ref03_quant_run(qw, _vp(r["Xp"]), _vp(RY), _vp(r["offsets"]), A, E, d, f, 0,
                                    C.c_void_p(stream))
    try:
        ours()
        ref()
        torch.cuda.synchronize()
        active = int((r["counts"] > 0).sum())
        row = {"active_experts": active, "max_abs_diff": float((Y.float() - RY.float()).abs().max())}
        if timed:
            t_o, t_r = timer(ours), timer(ref)
            byts = active * q.bytes_per_expert() + A * (d + f) * 2
            row.update({"ours_us": round(t_o * 1e3, 1), "reference_us": round(t_r * 1e3, 1),
                        "ours_GB/s": round(byts / (t_o * 1e-3) / 1e9, 1),
                        "speedup": round(t_r / t_o, 2)})
        return row
    finally:
        torch.cuda.synchronize()
        L.ref03_quant_free(qw)


def main():
    import torch
    import bench
    import ckl
    import oracle as O
    ap = argparse.ArgumentParser()
    ap.add_argument("--out", default="")
    ap.add_argument("--iters", type=int, default=31)
    args = ap.parse_args()
    if O.ref01() is None or O.ref03() is None:
        sys.exit("oracle/_ref not built: make -C oracle REF=<reference tree>")
    dev = torch.device("cuda", 0)
    base_timer = bench.ColdTimer(dev)
    timer = lambda fn: base_timer(fn, iters=args.iters)
    res = {"method": f"cold L2 (512 MB memset before each sample), median of {args.iters}, "
                     "CUDA events, same inputs; the reference built from its sources for sm_100a",
           "decode": {}, "cascade": {}, "int4_expert_gemm": {}}
    for name in ("256x4096", "ragged256", "64x1024", "8x8192", "1x32768"):
        res["decode"][name] = decode_row(ckl, O, bench, dev, timer, name)
        torch.cuda.empty_cache()
    res["cascade"]["64x(4096+256)"] = cascade_row(ckl, O, bench, dev, timer, np.full(64, 256))
    res["cascade"]["64x(4096+U[1,1024])"] = cascade_row(
        ckl, O, bench, dev, timer, np.random.default_rng(77).integers(1, 1025, 64))
    for T in (1, 4, 16, 64):
        res["int4_expert_gemm"][f"T={T}"] = gemm_row(ckl, O, dev, timer, T)
        torch.cuda.empty_cache()
    line = json.dumps(res)
    print(line)
    if args.out:
        with open(args.out, "w") as f:
            f.write(line + "\n")


if __name__ == "__main__":
    main()
