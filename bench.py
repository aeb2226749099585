#!/usr/bin/env python
"""bench.py -- paged split-KV decode attention on B200: HBM GB/s.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--workload 256x4096|1x32768|8x8192|64x1024|ragged256]

One step = one ckl_decode_attention call (the C-ABI entry point; partial kernel + LSE
merge when the batch is split) over one synthetic paged batch: Hq=32, Hkv=8, d=128, page
16, shuffled page table, K/V U(-1,1) fp16 filled on the device. The default workload is
B=256 x L=4096 (4.3 GB of KV, larger than the 126 MB L2, so no flush is needed between
steps). Under torchrun (N>1) the KV heads are sharded N ways and the batch grows to
B = 256*N sequences, so every GPU streams the single-GPU workload's KV bytes (weak
scaling); each GPU's decode kernels store its output rows straight into rank 0's output
over NVLink (the gather), and rank 0 waits on per-rank epoch flags before the step ends.
Timing is CUDA events, max over ranks.

Rank 0 prints one JSON line. `value` = algorithmic bytes of all ranks / max step time
(sum of K+V of every token + q + out + lse); `e2e` = the same metric with the per-step
host->device copy of q and the page table from pinned memory and the device->host read of
out and lse inside the timed region; `roofline` = the partial kernel's achieved GB/s
against the measured HBM copy bandwidth (MEASURED_PEAKS.json); `cpu_baseline` = the
reference's own fp64 cpu_reference (oracle/_ref) on the host cores, on a bounded sample.

--impl reference times the reference's CPU implementation of the path (the same
cpu_reference) on the same workload shape, one bounded sample per step, all host threads.
"""
from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import sys
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(ROOT, "cuda-kernel-lab_b200"))

HQ, HKV, D, PAGE = 32, 8, 128, 16
WORKLOADS = {
    "256x4096": dict(B=256, L=4096),
    "1x32768": dict(B=1, L=32768),
    "8x8192": dict(B=8, L=8192),
    "64x1024": dict(B=64, L=1024),
    "ragged256": dict(B=256, L=None),   # lengths U[128, 8192], seeded
}
METRIC = "decode-attn HBM GB/s"


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--workload", choices=sorted(WORKLOADS), default="256x4096")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-extras", action="store_true",
                    help="skip the extra rows (sweep, cascades, MoE, Mixtral, grouped GEMM)")
    ap.add_argument("--extras", default="",
                    help="comma-separated names of the extra rows to run (default: all)")
    ap.add_argument("--probe", default="",
                    help="run one small fixed workload a few times (L2 flushed between calls) "
                         "for a profiler and exit: " + ", ".join(sorted(PROBES)))
    return ap.parse_args()


def lengths(workload, seed=2024):
    import numpy as np
    w = WORKLOADS[workload]
    if w["L"] is None:
        return np.random.default_rng(seed).integers(128, 8193, size=w["B"]).astype(np.int32)
    return np.full(w["B"], w["L"], np.int32)


def algorithmic_bytes(lens):
    kv = int(sum(int(L) for L in lens)) * HKV * D * 2 * 2
    return kv + len(lens) * HQ * D * 2 * 2 + len(lens) * HQ * 4


def config_of(workload, lens, n):
    c = {"workload": f"paged GQA decode attention {workload}", "B": int(len(lens)),
         "L": "U[128,8192]" if WORKLOADS[workload]["L"] is None else int(lens[0]),
         "Hq": HQ, "Hkv": HKV, "head_dim": D, "page": PAGE, "page_table": "shuffled",
         "kv_dtype": "fp16",
         "l2": "inputs larger than L2 (KV %.2f GB per GPU > 126 MB), no flush" %
               (algorithmic_bytes(lens) / 1e9 / n)}
    if n == 1:
        c["parallelism"] = "single GPU"
    else:
        c["parallelism"] = (f"KV heads sharded {n} ways ({HKV // n} KV / {HQ // n} q heads per "
                            "GPU), page table replicated; each GPU's output rows stored into "
                            "rank 0's output by the decode kernels (fused gather) + epoch-flag "
                            "completion wait on rank 0")
        c["per_gpu"] = (f"weak scaling: B = {len(lens) // n} x {n} sequences, so every GPU "
                        "streams the KV bytes of the single-GPU workload")
    return c


# ------------------------------------------------------------------ clocks
class Clocks:
    """Samples SM clock and throttle reasons through NVML on a background thread during the
    timed region (nvidia-smi's 200 ms period is longer than a decode step loop)."""

    REASONS = {"hw_slowdown": 0x8, "sw_thermal_slowdown": 0x20, "hw_thermal_slowdown": 0x40,
               "sw_power_cap": 0x4}

    def __init__(self, gpu_index):
        import threading
        self.samples = []
        self.active = False
        self.stop_flag = False
        try:
            import pynvml
            pynvml.nvmlInit()
            self.nv = pynvml
            bus = None
            try:   # NVML wants the "DDDDDDDD:BB:DD.0" string, torch gives the numbers
                import torch
                pr = torch.cuda.get_device_properties(gpu_index)
                ids = (pr.pci_domain_id, pr.pci_bus_id, pr.pci_device_id)
                if all(isinstance(x, int) for x in ids):
                    bus = "%08X:%02X:%02X.0" % ids
            except Exception:
                bus = None
            self.h = (pynvml.nvmlDeviceGetHandleByPciBusId(bus.encode()) if bus
                      else pynvml.nvmlDeviceGetHandleByIndex(gpu_index))
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self.h, pynvml.NVML_CLOCK_SM)
        except Exception:
            self.nv = None
            return
        self.t = threading.Thread(target=self._run, daemon=True)
        self.t.start()

    def _run(self):
        import time as _t
        while not self.stop_flag:
            if self.active:
                try:
                    mhz = self.nv.nvmlDeviceGetClockInfo(self.h, self.nv.NVML_CLOCK_SM)
                    rs = self.nv.nvmlDeviceGetCurrentClocksEventReasons(self.h)
                    self.samples.append((mhz, rs))
                except Exception:
                    pass
            _t.sleep(0.0005)

    def start(self):
        self.active = True

    def stop(self):
        if self.nv is None:
            return None
        self.active = False
        self.stop_flag = True
        self.t.join(timeout=2)
        if not self.samples:
            return None
        reasons = set()
        for _, rs in self.samples:
            for n, bit in self.REASONS.items():
                if rs & bit:
                    reasons.add(n)
        return {"sm_mhz": statistics.median(m for m, _ in self.samples),
                "sm_max_mhz": self.max_mhz, "reasons": sorted(reasons),
                "samples": len(self.samples), "source": "NVML during the timed region"}


# ------------------------------------------------------------------ distributed plumbing
def dist_setup(n):
    import torch
    import torch.distributed as dist
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world != n:
        sys.exit(f"--gpus {n} but WORLD_SIZE={world}")
    torch.cuda.set_device(local)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=180),
                                device_id=torch.device("cuda", local))
    return rank, world, local


def barrier(world):
    import torch
    import torch.distributed as dist
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()


def max_over_ranks(x, world):
    import torch
    import torch.distributed as dist
    if world == 1:
        return x
    t = torch.tensor([x], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def measured_peak():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            pk = json.load(f)
        return float(pk["hbm_gbs"]), "measured"
    except (OSError, KeyError, ValueError):
        return 6650.0, "fallback"


NOMINAL_HBM_GBS = 7700.0     # B200 HBM3e, HGX figure (8000 on DGX)


def stream_read_ceiling(ckl, dev, gib=2, iters=10):
    """The reference's own bandwidth denominator: its stream_read probe
    (01_decode_attention.cu:257-265, ckl_stream_read) over a gib-GiB buffer, GB/s (CUDA
    events on the launching stream, after 3 warm-up reads; the buffer is 16x L2)."""
    import torch
    buf = torch.zeros(gib << 30, dtype=torch.uint8, device=dev)
    sink = torch.zeros(4, dtype=torch.int32, device=dev)
    stream = torch.cuda.current_stream()
    for _ in range(3):
        ckl.stream_read(buf, sink, stream)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    e0.record(stream)
    for _ in range(iters):
        ckl.stream_read(buf, sink, stream)
    e1.record(stream)
    torch.cuda.synchronize()
    gbs = buf.numel() / (e0.elapsed_time(e1) / iters * 1e-3) / 1e9
    del buf
    torch.cuda.empty_cache()
    return gbs


def committed_traffic(kernel, workload):
    """DRAM bytes per launch from a committed ncu summary (profiles/traffic.json)."""
    try:
        with open(os.path.join(ROOT, "profiles", "traffic.json")) as f:
            t = json.load(f)
        e = t.get(kernel, {}).get(workload)
        return None if e is None else float(e)
    except (OSError, ValueError):
        return None


# ------------------------------------------------------------------ CPU baselines
def cpu_model():
    """The host CPU's model string (/proc/cpuinfo), or the platform's processor name."""
    try:
        with open("/proc/cpuinfo") as f:
            for line in f:
                if line.startswith("model name"):
                    return line.split(":", 1)[1].strip()
    except OSError:
        pass
    import platform
    return platform.processor() or "unknown"


def cpu_baseline_sample(L, threads, min_seqs=64):
    """The reference's cpu_reference (oracle/_ref) on `threads` threads over a bounded
    sample of ~min_seqs sequences of length L; returns the cpu_baseline object."""
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle as O
    if O.ref01() is not None:
        bpt = max(1, math.ceil(min_seqs / threads))
        s = O.RefCpuSample(threads, bpt, L, HQ, HKV, seed=11)
        try:
            sec, kvb = s.run()
        finally:
            s.close()
        nseq = threads * bpt
        byts = kvb + nseq * HQ * D * 2 * 2 + nseq * HQ * 4
        return {"value": byts / sec / 1e9, "unit": "GB/s", "cores": threads, "kind": "reference",
                "cpu_model": cpu_model(),
                "sample": f"{nseq} sequences x L={L} (Hq={HQ}, Hkv={HKV}), {threads} threads x "
                          f"{bpt}; cpu_reference 01_decode_attention.cu:371-400 compiled from "
                          f"the reference sources; {sec:.2f} s"}
    bt = O.batch([L] * 8, HQ, HKV, 11)
    sec = O.port_attention_seconds(bt, threads)
    return {"value": algorithmic_bytes([L] * 8) / sec / 1e9, "unit": "GB/s", "cores": threads,
            "kind": "port", "cpu_model": cpu_model(), "sample": f"8 sequences x L={L}, oracle port, {sec:.2f} s"}


def run_reference(args):
    rank, world, local = int(os.environ.get("RANK", "0")), int(os.environ.get("WORLD_SIZE", "1")), 0
    if rank != 0:
        return 0
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle as O
    lens = lengths(args.workload)
    L = int(lens.max()) if WORKLOADS[args.workload]["L"] is None else int(lens[0])
    threads = os.cpu_count() or 1
    if O.ref01() is None:
        print(json.dumps({"impl": "reference", "unavailable": "oracle/_ref not built (the reference "
                          "sources were not present when this tree was built)"}))
        return 0
    s = O.RefCpuSample(threads, 1, L, HQ, HKV, seed=11)
    try:
        for _ in range(args.warmup):
            s.run()
        secs = []
        kvb = 0.0
        for _ in range(args.steps):
            sec, kvb = s.run()
            secs.append(sec)
    finally:
        s.close()
    nseq = threads
    byts = kvb + nseq * HQ * D * 2 * 2 + nseq * HQ * 4
    tot = sum(secs)
    val = byts * len(secs) / tot / 1e9
    line = {"metric": METRIC, "value": val, "unit": "GB/s", "impl": "reference",
            "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": tot / len(secs) * 1e3, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "f64", "data": "synthetic (reference generator)",
            "config": config_of(args.workload, lens, args.gpus),
            "cpu_baseline": {"value": val, "unit": "GB/s", "cores": threads, "kind": "reference",
                             "cpu_model": cpu_model(),
                             "sample": f"per step {nseq} sequences x L={L} (one per thread) of "
                                       "the workload; cpu_reference compiled from the reference"},
            "e2e": {"value": val, "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line))
    return 0


# ------------------------------------------------------------------ extra rows (N=1)
def _fill_uniform(t, g):
    import torch
    flat = t.view(-1)
    step = 1 << 28
    for s0 in range(0, flat.numel(), step):
        n = min(step, flat.numel() - s0)
        flat[s0:s0 + n] = (torch.rand(n, generator=g, device=t.device) * 2 - 1).half()


class ColdTimer:
    """Median CUDA-event time of fn with L2 overwritten (512 MB memset, > 4x L2) before
    every sample, as the reference's Bench::time_cold (common/bench.cuh:111-131). The
    memset keeps the GPU busy for ~80 us, so the host has enqueued fn's launches before the
    start event runs and host-side call overhead stays outside the timed region. With
    world > 1 every rank calls it: the ranks start each sample together (host barrier after
    the flush) and the result is the max over ranks of the per-rank medians."""

    def __init__(self, dev, world=1):
        import torch
        self.flush = torch.empty(512 << 20, dtype=torch.uint8, device=dev)
        self.world = world

    def __call__(self, fn, iters=31, warmup=3):
        import torch
        for _ in range(warmup):
            fn()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        ts = []
        for i in range(iters):
            self.flush.fill_(i & 0xFF)
            if self.world > 1:
                barrier(self.world)
            e0.record()
            fn()
            e1.record()
            e1.synchronize()
            ts.append(e0.elapsed_time(e1))
        ts.sort()
        return max_over_ranks(ts[len(ts) // 2], self.world)


def paged_batch(lens, dev, seed, Lp=0):
    """A shuffled paged batch filled U(-1,1) on the device; Lp > 0 makes every sequence share
    its first Lp tokens' physical pages (prefix caching)."""
    import numpy as np
    import torch
    lens = np.asarray(lens, np.int32)
    B = len(lens)
    npg = (lens + PAGE - 1) // PAGE
    indptr = np.zeros(B + 1, np.int32)
    indptr[1:] = np.cumsum(npg)
    last = (lens - (npg - 1) * PAGE).astype(np.int32)
    pp = Lp // PAGE
    total = pp + int(np.sum(npg - pp))
    perm = np.random.default_rng(seed).permutation(total).astype(np.int32)
    indices = np.empty(int(indptr[-1]), np.int32)
    nxt = pp
    for b in range(B):
        n = int(npg[b])
        indices[indptr[b]:indptr[b] + pp] = perm[:pp]
        indices[indptr[b] + pp:indptr[b] + n] = perm[nxt:nxt + n - pp]
        nxt += n - pp
    g = torch.Generator(device=dev)
    g.manual_seed(seed)
    k = torch.empty((total, PAGE, HKV, D), dtype=torch.float16, device=dev)
    v = torch.empty_like(k)
    _fill_uniform(k, g)
    _fill_uniform(v, g)
    q = (torch.rand((B, HQ, D), generator=g, device=dev) * 2 - 1).half()
    t = lambda a: torch.from_numpy(a).to(dev)
    return dict(q=q, k_cache=k, v_cache=v, kv_indptr=t(indptr), kv_indices=t(indices),
                kv_last_page_len=t(last)), (lens, indptr, indices)


def sweep_config2(ckl, dev, timer, peak):
    """Every config-2 shape through ckl_decode_attention (the reference's chunked split) and
    ckl_decode_attention_balanced, cold L2, median of 31."""
    import torch
    rows = {}
    for name in ("1x32768", "8x8192", "64x1024", "256x4096", "ragged256"):
        lens = lengths(name)
        d, _ = paged_batch(lens, dev, seed=7)
        nc, ct = ckl.plan_chunks(HQ // HKV, len(lens), HKV, int(lens.max()))
        p = ckl.make_params(**d, num_chunks=nc, chunk_tokens=ct)
        out = torch.empty_like(d["q"])
        lse = torch.empty((len(lens), HQ), dtype=torch.float32, device=dev)
        ws = torch.empty(max(ckl.workspace_size(p), 256), dtype=torch.uint8, device=dev)
        ms = timer(lambda: ckl.decode_attention(**d, num_chunks=nc, chunk_tokens=ct, out=out,
                                                lse=lse, workspace=ws))
        gbs = algorithmic_bytes(lens) / (ms * 1e-3) / 1e9
        rows[name] = {"ms": round(ms, 4), "GB/s": round(gbs, 1),
                      "frac_of_measured_hbm": round(gbs / peak, 3), "chunks": nc}
        # the balanced split (ckl_decode_attention_balanced), the path for ragged batches
        pb = ckl.make_params(**d, num_chunks=1, chunk_tokens=16)
        wsb = torch.empty(max(ckl.lib().ckl_decode_balanced_workspace_size(ckl.C.byref(pb)), 256),
                          dtype=torch.uint8, device=dev)
        msb = timer(lambda: ckl.decode_attention_balanced(**d, out=out, lse=lse, workspace=wsb))
        gbb = algorithmic_bytes(lens) / (msb * 1e-3) / 1e9
        rows[name]["balanced_split"] = {"ms": round(msb, 4), "GB/s": round(gbb, 1),
                                        "frac_of_measured_hbm": round(gbb / peak, 3)}
        del d, out, lse, ws, wsb
        torch.cuda.empty_cache()
    return rows


def bench_decode_multilayer(ckl, dev, timer, peak):
    """Every config-2 shape as a multi-layer decode step: n layers, each with its own paged KV
    cache, layer l's output [B, Hq, 128] is layer l+1's q (a real dependency), all captured in
    one CUDA graph and replayed with a cold L2 (512 MB memset before each replay); the figure
    is per layer. Consecutive calls overlap only their launch and set-up (the partial kernel
    starts behind the previous merge and waits for it before reading anything); the
    `cache_ready` figure is the same chain through ckl_decode_attention_ex with
    CKL_DECODE_CACHE_READY, whose producer warp reads the page table and streams the first
    pages before that wait (the caches here are written before the step, as in decode)."""
    import torch
    rows = {}
    for name in ("1x32768", "8x8192", "64x1024", "256x4096", "ragged256"):
        lens = lengths(name)
        n = 4 if len(lens) >= 256 else 8
        layers = [paged_batch(lens, dev, seed=300 + l)[0] for l in range(n)]
        nc, ct = ckl.plan_chunks(HQ // HKV, len(lens), HKV, int(lens.max()))
        p = ckl.make_params(**layers[0], num_chunks=nc, chunk_tokens=ct)
        ws = torch.empty(max(ckl.workspace_size(p), 256), dtype=torch.uint8, device=dev)
        outs = [torch.empty_like(layers[0]["q"]) for _ in range(n)]
        lses = [torch.empty((len(lens), HQ), dtype=torch.float32, device=dev) for _ in range(n)]
        q0 = layers[0]["q"]

        def chain(ready):
            def step():
                x = q0
                for l, d in enumerate(layers):
                    dd = dict(d)
                    dd["q"] = x
                    ckl.decode_attention(**dd, num_chunks=nc, chunk_tokens=ct, out=outs[l],
                                         lse=lses[l], workspace=ws, cache_ready=ready)
                    x = outs[l]
            return step

        ms = timer(GraphStep(chain(False), dev)) / n
        ms_r = timer(GraphStep(chain(True), dev)) / n
        gbs = algorithmic_bytes(lens) / (ms * 1e-3) / 1e9
        gbs_r = algorithmic_bytes(lens) / (ms_r * 1e-3) / 1e9
        rows[name] = {"layers": n, "ms_per_layer": round(ms, 4), "GB/s": round(gbs, 1),
                      "frac_of_measured_hbm": round(gbs / peak, 3), "chunks": nc,
                      "cache_ready": {"ms_per_layer": round(ms_r, 4), "GB/s": round(gbs_r, 1),
                                      "frac_of_measured_hbm": round(gbs_r / peak, 3)}}
        del layers, outs, lses, ws
        torch.cuda.empty_cache()
    rows["method"] = ("n layers with distinct KV caches in one CUDA graph, each layer's output "
                      "the next layer's q, L2 flushed before each replay, per-layer median of 31")
    return rows


def plain_split_kv(ckl, d, lens, out, lse):
    """ckl_decode_attention on a batch, planned (plan_chunks) and given its workspace
    outside the timed call, so the timed call is the launches alone."""
    import torch
    nc, ct = ckl.plan_chunks(HQ // HKV, len(lens), HKV, int(max(lens)), 0)
    p = ckl.make_params(**d, num_chunks=nc, chunk_tokens=ct)
    ws = torch.empty(max(ckl.workspace_size(p), 256), dtype=torch.uint8, device=out.device)
    return lambda: ckl.decode_attention(**d, num_chunks=nc, chunk_tokens=ct, out=out, lse=lse,
                                        workspace=ws)


def bench_cascade(ckl, dev, timer, peak):
    """64 requests x (4096 shared + 256 private) tokens, and the ragged
    variant (suffix U[1,1024]); cascade vs plain split-KV on the same batch, cold L2."""
    import numpy as np
    import torch
    res = {}
    for name, suffix in (("64x(4096+256)", np.full(64, 256)),
                         ("64x(4096+U[1,1024])", np.random.default_rng(77).integers(1, 1025, 64))):
        Lp = 4096
        lens = (Lp + suffix).astype(np.int32)
        d, (lens, indptr, indices) = paged_batch(lens, dev, seed=21, Lp=Lp)
        base = ckl.make_params(**d, num_chunks=1, chunk_tokens=16)
        cp = ckl.plan_cascade(base, indptr, indices, lens, 256)
        assert cp.use == 1 and cp.prefix_len == Lp
        ws = torch.empty(max(ckl.cascade_workspace_size(cp), 256), dtype=torch.uint8, device=dev)
        out = torch.empty_like(d["q"])
        lse = torch.empty((len(lens), HQ), dtype=torch.float32, device=dev)
        t_cas = timer(lambda: ckl.cascade_decode(cp, out=out, lse=lse, workspace=ws))
        o_cas = out.clone()
        t_plain = timer(plain_split_kv(ckl, d, lens, out, lse))
        err = float((o_cas.float() - out.float()).abs().max())
        naive = algorithmic_bytes(lens)
        unique = (Lp + int(np.sum(lens - Lp))) * HKV * D * 2 * 2 + len(lens) * HQ * (D * 4 + 4)
        bound_ms = naive / (peak * 1e9) * 1e3
        res[name] = {"ms_cascade": round(t_cas, 4), "ms_plain_split_kv": round(t_plain, 4),
                     "naive_bytes": naive, "unique_bytes": unique,
                     "naive_bw_bound_ms": round(bound_ms, 4),
                     "speedup_vs_bw_bound": round(bound_ms / t_cas, 2),
                     "speedup_vs_plain": round(t_plain / t_cas, 2),
                     "naive_equiv_GB/s": round(naive / (t_cas * 1e-3) / 1e9, 1),
                     "max_abs_diff_vs_plain": err, "prefix_chunks": cp.prefix_chunks,
                     "suffix_chunks": cp.suffix.num_chunks}
        del d, ws, out, lse
        torch.cuda.empty_cache()
    return res


def tree_batch(system, doc, n_groups, suffix, dev, seed):
    """A shuffled paged batch shaped as a prefix tree: every sequence starts with the same
    `system` tokens, the sequences of each of n_groups equal groups then share one `doc`-token
    document, and each ends with its own suffix[b] tokens; filled U(-1,1) on the device."""
    import numpy as np
    import torch
    suffix = np.asarray(suffix, np.int32)
    B = len(suffix)
    sp, dp = system // PAGE, doc // PAGE
    spg = (suffix + PAGE - 1) // PAGE
    total = sp + n_groups * dp + int(spg.sum())
    perm = np.random.default_rng(seed).permutation(total).astype(np.int32)
    lists, nxt = [], sp + n_groups * dp
    for b in range(B):
        g = b * n_groups // B
        own = list(range(nxt, nxt + int(spg[b])))
        nxt += int(spg[b])
        lists.append(list(range(sp)) + list(range(sp + g * dp, sp + (g + 1) * dp)) + own)
    indptr = np.zeros(B + 1, np.int32)
    indptr[1:] = np.cumsum([len(x) for x in lists])
    indices = perm[np.array([p for x in lists for p in x], np.int64)]
    lens = (system + doc + suffix).astype(np.int32)
    last = (suffix - (spg - 1) * PAGE).astype(np.int32)
    g = torch.Generator(device=dev)
    g.manual_seed(seed)
    k = torch.empty((total, PAGE, HKV, D), dtype=torch.float16, device=dev)
    v = torch.empty_like(k)
    _fill_uniform(k, g)
    _fill_uniform(v, g)
    q = (torch.rand((B, HQ, D), generator=g, device=dev) * 2 - 1).half()
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(dev)
    return (dict(q=q, k_cache=k, v_cache=v, kv_indptr=t(indptr), kv_indices=t(indices),
                 kv_last_page_len=t(last)), (lens, indptr, indices), total)


def bench_cascade_tree(ckl, dev, timer, peak):
    """Prefix tree (the reference's cascade needs one prefix shared by the whole batch): 64
    requests = a 1024-token system prompt shared by all, 4 groups of 16 sharing a
    4096-token document each, private suffixes of 256 tokens (and U[1,1024]). The tree
    cascade against the whole-batch cascade (which finds only the system prompt) and plain
    split-KV on the same batch, cold L2."""
    import numpy as np
    import torch
    res = {}
    for name, suffix in (("64x(1024+4x4096+256)", np.full(64, 256)),
                         ("64x(1024+4x4096+U[1,1024])",
                          np.random.default_rng(78).integers(1, 1025, 64))):
        d, (lens, indptr, indices), total = tree_batch(1024, 4096, 4, suffix, dev, seed=23)
        base = ckl.make_params(**d, num_chunks=1, chunk_tokens=16)
        tp = ckl.plan_cascade_tree(base, indptr, indices, lens, 256)
        assert tp.use == 1 and tp.nodes == 5
        cp = ckl.plan_cascade(base, indptr, indices, lens, 256)
        nbytes = max(ckl.cascade_tree_workspace_size(tp), ckl.cascade_workspace_size(cp), 256)
        ws = torch.empty(nbytes, dtype=torch.uint8, device=dev)
        out = torch.empty_like(d["q"])
        lse = torch.empty((len(lens), HQ), dtype=torch.float32, device=dev)
        t_tree = timer(lambda: ckl.cascade_tree_decode(tp, out=out, lse=lse, workspace=ws))
        o_tree = out.clone()
        t_cas = timer(lambda: ckl.cascade_decode(cp, out=out, lse=lse, workspace=ws))
        t_plain = timer(plain_split_kv(ckl, d, lens, out, lse))
        err = float((o_tree.float() - out.float()).abs().max())
        naive = algorithmic_bytes(lens)
        unique = total * PAGE * HKV * D * 2 * 2 + len(lens) * HQ * (D * 4 + 4)
        bound_ms = naive / (peak * 1e9) * 1e3
        unique_ms = unique / (peak * 1e9) * 1e3
        res[name] = {"ms_tree_cascade": round(t_tree, 4), "ms_whole_batch_cascade": round(t_cas, 4),
                     "ms_plain_split_kv": round(t_plain, 4), "naive_bytes": naive,
                     "unique_bytes": unique, "naive_bw_bound_ms": round(bound_ms, 4),
                     "unique_bw_bound_ms": round(unique_ms, 4),
                     "speedup_vs_bw_bound": round(bound_ms / t_tree, 2),
                     "speedup_vs_plain": round(t_plain / t_tree, 2),
                     "speedup_vs_whole_batch_cascade": round(t_cas / t_tree, 2),
                     "unique_GB/s": round(unique / (t_tree * 1e-3) / 1e9, 1),
                     "max_abs_diff_vs_plain": err, "tree_nodes": tp.nodes,
                     "prefix_items_per_kv_head": tp.items, "suffix_chunks": tp.suffix.num_chunks}
        del d, ws, out, lse
        torch.cuda.empty_cache()
    return res


def _moe_active_bytes(q, ids_np):
    """Algorithmic bytes of one layer step: packed weights + scales + zeros of every active
    expert (gate, up, down) + X in + out (the reference credits the active experts' weight
    bytes, 03_moe_wq_decode.cu:527,551)."""
    import numpy as np
    active = len(np.unique(ids_np))
    return active * sum(w.bytes_per_expert() for w in q)


class GraphStep:
    """The step captured once in a CUDA graph and replayed (the layer never syncs the host
    and never allocates, so it is capturable)."""

    def __init__(self, fn, dev):
        import torch
        s = torch.cuda.Stream(device=dev)
        s.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(s):
            for _ in range(2):
                fn()
        torch.cuda.current_stream().wait_stream(s)
        torch.cuda.synchronize()
        self.g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.g):
            fn()
        torch.cuda.synchronize()

    def __call__(self):
        self.g.replay()


def bench_moe(ckl, dev, timer, peak, n_layers=8):
    """W4A16 (asym int4 g128) SwiGLU MoE layer, E=64, top-6, d=2048,
    F=1408, T in {1,4,16,64}; weights N(0,0.02), X and logits N(0,1).

    Timed like the reference's multi-layer decode step (03_moe_wq_decode.cu:651-681):
    n_layers layers, each with its own weights (2.2 GB in all, so a layer's weights are not
    in L2 when it runs), captured in one CUDA graph, L2 flushed before every replay; the
    figure is per layer. Also the single layer replayed alone with a cold L2."""
    import torch
    E, k, d, F = 64, 6, 2048, 1408
    g = torch.Generator(device=dev)
    g.manual_seed(44)
    mk = lambda *sh: (torch.randn(*sh, generator=g, device=dev) * 0.02).half()
    layers = []
    for _ in range(n_layers):
        q = [ckl.QuantWeights(4, mk(E, d, F), group=128, asym=True) for _ in range(2)]
        q.append(ckl.QuantWeights(4, mk(E, F, d), group=128, asym=True))
        layers.append((q, ckl.MoeLayer(*q)))
    res = {}
    for T in (1, 4, 16, 64):
        lg = [torch.randn((T, E), generator=g, device=dev) for _ in range(n_layers)]
        X = torch.randn((T, d), generator=g, device=dev).half()
        outs = [torch.empty((T, d), dtype=torch.float16, device=dev) for _ in range(n_layers)]
        ids = [torch.empty((T, k), dtype=torch.int32, device=dev) for _ in range(n_layers)]
        ws = torch.empty(layers[0][1].workspace_size(T, k), dtype=torch.uint8, device=dev)

        def step():
            x = X
            for l, (_, layer) in enumerate(layers):
                layer.forward(lg[l], x, k, out=outs[l], ids=ids[l], workspace=ws)
                x = outs[l]

        def one():
            layers[0][1].forward(lg[0], X, k, out=outs[0], ids=ids[0], workspace=ws)

        t_step = timer(GraphStep(step, dev)) / n_layers
        t_one = timer(GraphStep(one, dev))
        byts = sum(_moe_active_bytes(layers[l][0], ids[l].cpu().numpy()) for l in range(n_layers))
        byts = byts / n_layers + T * d * 2 * 2
        res[f"T={T}"] = {"us_per_layer": round(t_step * 1e3, 2),
                         "us_single_layer_cold": round(t_one * 1e3, 2),
                         "active_experts_avg": round(sum(len(set(i.cpu().numpy().ravel().tolist()))
                                                         for i in ids) / n_layers, 1),
                         "bytes_per_layer": int(byts),
                         "GB/s": round(byts / (t_step * 1e-3) / 1e9, 1),
                         "frac_of_measured_hbm": round(byts / (t_step * 1e-3) / 1e9 / peak, 3),
                         "kernels_per_layer": 4 + sum(1 for w, sw in ((layers[0][0][0], True),
                                                                      (layers[0][0][2], False))
                                                      if w.workspace_size(T * k, sw) > 0)}
    res["method"] = (f"{n_layers} layers with distinct weights in one CUDA graph, L2 flushed "
                     "before each replay, per-layer median of 31; PDL between the layer's kernels")
    del layers
    torch.cuda.empty_cache()
    return res


def bench_mixtral_layer(ckl, dev, timer, peak):
    """paged GQA attention (B=32, L=4096, Hq=32, Hkv=8) followed by the
    MoE block (E=8, top-2, d=4096, F=14336, SwiGLU, int8 per output channel), T=32 tokens;
    one step = attention + MoE, replayed from one CUDA graph; cold L2."""
    import torch
    B, L = 32, 4096
    E, k, d, F = 8, 2, 4096, 14336
    d_attn, _ = paged_batch([L] * B, dev, seed=55)
    nc, ct = ckl.plan_chunks(HQ // HKV, B, HKV, L)
    pa = ckl.make_params(**d_attn, num_chunks=nc, chunk_tokens=ct)
    a_out = torch.empty_like(d_attn["q"])
    a_lse = torch.empty((B, HQ), dtype=torch.float32, device=dev)
    a_ws = torch.empty(max(ckl.workspace_size(pa), 256), dtype=torch.uint8, device=dev)
    g = torch.Generator(device=dev)
    g.manual_seed(55)
    mk = lambda *sh: (torch.randn(*sh, generator=g, device=dev) * 0.02).half()
    q = [ckl.QuantWeights(8, mk(E, d, F), group=d), ckl.QuantWeights(8, mk(E, d, F), group=d),
         ckl.QuantWeights(8, mk(E, F, d), group=F)]
    layer = ckl.MoeLayer(*q)
    lg = torch.randn((B, E), generator=g, device=dev)
    X = torch.randn((B, d), generator=g, device=dev).half()
    out = torch.empty((B, d), dtype=torch.float16, device=dev)
    ids = torch.empty((B, k), dtype=torch.int32, device=dev)
    ws = torch.empty(layer.workspace_size(B, k), dtype=torch.uint8, device=dev)

    def attn():
        ckl.decode_attention(**d_attn, num_chunks=nc, chunk_tokens=ct, out=a_out, lse=a_lse,
                             workspace=a_ws)

    def moe():
        layer.forward(lg, X, k, out=out, ids=ids, workspace=ws)

    def step():
        attn()
        moe()

    t_attn = timer(GraphStep(attn, dev))
    t_moe = timer(GraphStep(moe, dev))
    t_step = timer(GraphStep(step, dev))
    attn_bytes = algorithmic_bytes([L] * B)
    moe_bytes = _moe_active_bytes(q, ids.cpu().numpy()) + B * d * 2 * 2
    res = {"us_step": round(t_step * 1e3, 2), "us_attention": round(t_attn * 1e3, 2),
           "us_moe": round(t_moe * 1e3, 2), "attention_bytes": attn_bytes, "moe_bytes": moe_bytes,
           "GB/s_step": round((attn_bytes + moe_bytes) / (t_step * 1e-3) / 1e9, 1),
           "frac_of_measured_hbm": round((attn_bytes + moe_bytes) / (t_step * 1e-3) / 1e9 / peak, 3),
           "moe_active_experts": int(len(set(ids.cpu().numpy().ravel().tolist())))}
    del q, layer, d_attn
    torch.cuda.empty_cache()
    return res


class CublasGrouped:
    """The reference's baseline (c), cublasGemmGroupedBatchedEx with one group per non-empty
    expert (02_moe_grouped_gemm.cu:397-423), called through ctypes on the cuBLAS library torch
    loads: column-major C[f x n_e] = W_e[f x d] . Xp_e[d x n_e], fp16 in and out, fp32
    compute. The host-side arrays are built once (not timed), as the reference does. A
    baseline leg only: never on the library's path."""

    def __init__(self, Xp, W, Y, offs):
        import ctypes as C
        import torch
        import nvidia.cublas
        path = os.path.join(list(nvidia.cublas.__path__)[0], "lib", "libcublas.so.12")
        self.L = L = C.CDLL(path)
        self.h = C.c_void_p()
        if L.cublasCreate_v2(C.byref(self.h)) != 0:
            raise RuntimeError("cublasCreate failed")
        E, d, f = W.shape
        act = [e for e in range(E) if offs[e + 1] > offs[e]]
        G = len(act)
        I = C.c_int * G
        self.keep = dict(
            ta=I(*[0] * G), tb=I(*[0] * G), m=I(*[f] * G), n=I(*[offs[e + 1] - offs[e] for e in act]),
            k=I(*[d] * G), lda=I(*[f] * G), ldb=I(*[d] * G), ldc=I(*[f] * G),
            alpha=(C.c_float * G)(*[1.0] * G), beta=(C.c_float * G)(*[0.0] * G), size=I(*[1] * G))
        ptr = lambda base, e, stride: base.data_ptr() + e * stride
        self.pa = torch.tensor([ptr(W, e, d * f * 2) for e in act], dtype=torch.int64, device=W.device)
        self.pb = torch.tensor([ptr(Xp, offs[e], d * 2) for e in act], dtype=torch.int64, device=W.device)
        self.pc = torch.tensor([ptr(Y, offs[e], f * 2) for e in act], dtype=torch.int64, device=W.device)
        self.G = G
        L.cublasGemmGroupedBatchedEx.restype = C.c_int

    def __call__(self):
        import ctypes as C
        import torch
        k = self.keep
        self.L.cublasSetStream_v2(self.h, C.c_void_p(torch.cuda.current_stream().cuda_stream))
        vp = lambda t: C.c_void_p(t.data_ptr())
        st = self.L.cublasGemmGroupedBatchedEx(
            self.h, k["ta"], k["tb"], k["m"], k["n"], k["k"], k["alpha"], vp(self.pa), 2, k["lda"],
            vp(self.pb), 2, k["ldb"], k["beta"], vp(self.pc), 2, k["ldc"], self.G, k["size"], 68)
        if st != 0:
            raise RuntimeError(f"cublasGemmGroupedBatchedEx status {st}")

    def close(self):
        self.L.cublasDestroy_v2(self.h)


def bench_grouped_gemm(ckl, dev, timer, peak):
    """The dense grouped expert GEMM (ckl_moe_grouped_gemm, tcgen05) on the reference's
    performance shapes (02_moe_grouped_gemm.cu:342-344): routed and permuted once, then the
    GEMM alone with a cold L2. Bound: HBM (every shape streams more weight bytes than the
    tensor cores need time for); both fractions are reported. Beside it the reference's
    three cuBLAS baselines (02:367-423): (a) one GEMM per expert (torch.matmul), (b) every
    expert padded to the largest count, one strided-batched GEMM (torch.bmm; padding copy
    not timed), (c) cublasGemmGroupedBatchedEx (CublasGrouped)."""
    import torch
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as fh:
            tf_peak = float(json.load(fh)["bf16_tflops"])
    except (OSError, KeyError, ValueError):
        tf_peak = 1590.0
    res = {}
    for name, (T, E, k, d, f) in {"mixtral_prefill_T512": (512, 8, 2, 4096, 14336),
                                  "finegrained_prefill_T512": (512, 64, 6, 2048, 1408),
                                  "finegrained_decode_T16": (16, 64, 6, 2048, 1408)}.items():
        g = torch.Generator(device=dev)
        g.manual_seed(T + E)
        lg = torch.randn((T, E), generator=g, device=dev)
        X = (torch.rand((T, d), generator=g, device=dev) * 2 - 1).half()
        W = ((torch.rand((E, d, f), generator=g, device=dev) * 2 - 1) / d ** 0.5).half()
        r = ckl.route_and_permute(lg, X, k)
        Xp, off = r["Xp"], r["offsets"]
        Yp = torch.empty((T * k, f), dtype=torch.float16, device=dev)
        offs = off.cpu().numpy().tolist()
        active = sum(1 for e in range(E) if offs[e + 1] > offs[e])
        A = T * k
        byts = active * d * f * 2 + A * d * 2 + A * f * 2
        flops = 2.0 * A * d * f
        t = timer(lambda: ckl.grouped_gemm(Xp, W, off, out=Yp))

        def per_expert():
            for e in range(E):
                if offs[e + 1] > offs[e]:
                    torch.matmul(Xp[offs[e]:offs[e + 1]], W[e], out=Yp[offs[e]:offs[e + 1]])
        t_ref = timer(per_expert)
        Yg = torch.empty_like(Yp)
        cg = CublasGrouped(Xp, W, Yg, offs)
        cg()
        torch.cuda.synchronize()
        grouped_diff = float((Yg.float() - Yp.float()).abs().max())
        t_grouped = timer(cg)
        cg.close()
        max_n = max(offs[e + 1] - offs[e] for e in range(E))
        Xpad = torch.zeros((E, max_n, d), dtype=torch.float16, device=dev)
        for e in range(E):
            Xpad[e, :offs[e + 1] - offs[e]] = Xp[offs[e]:offs[e + 1]]
        Ypad = torch.empty((E, max_n, f), dtype=torch.float16, device=dev)
        t_padded = timer(lambda: torch.bmm(Xpad, W, out=Ypad))
        del Xpad, Ypad, Yg
        res[name] = {"us": round(t * 1e3, 1), "active_experts": active,
                     "tokens_per_expert": round(A / E, 1),
                     "GB/s": round(byts / (t * 1e-3) / 1e9, 1),
                     "frac_of_measured_hbm": round(byts / (t * 1e-3) / 1e9 / peak, 3),
                     "TFLOP/s": round(flops / (t * 1e-3) / 1e12, 1),
                     "frac_of_measured_bf16_tensor": round(flops / (t * 1e-3) / 1e12 / tf_peak, 3),
                     "us_cublas_per_expert_loop": round(t_ref * 1e3, 1),
                     "us_cublas_padded_batched": round(t_padded * 1e3, 1),
                     "us_cublas_grouped_batched_ex": round(t_grouped * 1e3, 1),
                     "max_abs_diff_vs_cublas_grouped": grouped_diff}
        del W, Xp, Yp, r
        torch.cuda.empty_cache()
    res["method"] = "cold L2 (512 MB memset before each sample), median of 31; bytes = active experts' fp16 weights + Xp + Yp"
    return res


def bench_decode_step(ckl, dev, timer, peak, n_layers=4):
    """A decode step of n_layers config-5 layers in one CUDA graph: each layer its own paged
    KV cache (B=32 x 4096) and its own W8A16 experts (E=8, top-2, d=4096, F=14336); the
    attention output [32, 4096] is the MoE input and the MoE output the next layer's q (the
    projections between them are outside the reference's layer). Cold L2 before the step;
    the figure is per layer."""
    import torch
    B, L = 32, 4096
    E, k, d, F = 8, 2, 4096, 14336
    g = torch.Generator(device=dev)
    g.manual_seed(77)
    mk = lambda *sh: (torch.randn(*sh, generator=g, device=dev) * 0.02).half()
    layers = []
    for l in range(n_layers):
        d_attn, _ = paged_batch([L] * B, dev, seed=100 + l)
        nc, ct = ckl.plan_chunks(HQ // HKV, B, HKV, L)
        pa = ckl.make_params(**d_attn, num_chunks=nc, chunk_tokens=ct)
        q = [ckl.QuantWeights(8, mk(E, d, F), group=d), ckl.QuantWeights(8, mk(E, d, F), group=d),
             ckl.QuantWeights(8, mk(E, F, d), group=F)]
        layers.append(dict(attn=d_attn, nc=nc, ct=ct,
                           a_ws=torch.empty(max(ckl.workspace_size(pa), 256), dtype=torch.uint8, device=dev),
                           moe=ckl.MoeLayer(*q), q=q,
                           lg=torch.randn((B, E), generator=g, device=dev)))
    q0 = layers[0]["attn"]["q"].clone()
    a_out = torch.empty((B, HQ, D), dtype=torch.float16, device=dev)
    a_lse = torch.empty((B, HQ), dtype=torch.float32, device=dev)
    h = torch.empty((B, d), dtype=torch.float16, device=dev)
    m_ws = torch.empty(layers[0]["moe"].workspace_size(B, k), dtype=torch.uint8, device=dev)
    ids = torch.empty((B, k), dtype=torch.int32, device=dev)

    def chain(ready):
        def step():
            x = q0
            for ly in layers:
                dd = dict(ly["attn"])
                dd["q"] = x.view(B, HQ, D)
                ckl.decode_attention(**dd, num_chunks=ly["nc"], chunk_tokens=ly["ct"], out=a_out,
                                     lse=a_lse, workspace=ly["a_ws"], cache_ready=ready)
                ly["moe"].forward(ly["lg"], a_out.view(B, d), k, out=h, ids=ids, workspace=m_ws)
                x = h
        return step

    t = timer(GraphStep(chain(False), dev)) / n_layers
    t_r = timer(GraphStep(chain(True), dev)) / n_layers
    attn_bytes = algorithmic_bytes([L] * B)
    moe_bytes = E * sum(w.bytes_per_expert() for w in layers[0]["q"]) + B * d * 2 * 2
    gbs = lambda tt: (attn_bytes + moe_bytes) / (tt * 1e-3) / 1e9
    res = {"layers": n_layers, "us_per_layer": round(t * 1e3, 2),
           "GB/s": round(gbs(t), 1), "frac_of_measured_hbm": round(gbs(t) / peak, 3),
           "cache_ready": {"us_per_layer": round(t_r * 1e3, 2), "GB/s": round(gbs(t_r), 1),
                           "frac_of_measured_hbm": round(gbs(t_r) / peak, 3)},
           "method": "one CUDA graph for the whole step (attention -> MoE per layer, each layer "
                     "its own KV cache and experts: 1.95 GB per layer), L2 flushed before "
                     "each replay, per-layer median; cache_ready: the attention calls through "
                     "ckl_decode_attention_ex with CKL_DECODE_CACHE_READY"}
    del layers
    torch.cuda.empty_cache()
    return res


def _split(T, world, rank):
    return T // world + (1 if rank < T % world else 0)


def bench_moe_ep(ckl, dev, timer, peak, rank, world, exchange, n_layers=8):
    """BASELINE config 4 expert-parallel: experts [r*E/n, (r+1)*E/n) on GPU r, tokens routed
    on their own GPU and exchanged through IPC-mapped windows by the layer's kernels
    (ckl_moe_ep_layer). Same methodology as the single-GPU figure: n_layers layers with
    distinct weights in one CUDA graph, L2 flushed before every replay, per-layer time, max
    over ranks. T is the layer's whole batch split over the GPUs (the single-GPU config);
    "T=64/GPU" keeps 64 tokens on every GPU."""
    import numpy as np
    import torch
    E, k, d, F, T_cap = 64, 6, 2048, 1408, 64
    E_loc = E // world
    g = torch.Generator(device=dev)
    g.manual_seed(4400 + rank)
    mk = lambda *sh: (torch.randn(*sh, generator=g, device=dev) * 0.02).half()
    win = ckl.EpWindows(rank, world, T_cap, k, E, d, exchange)
    layers = []
    for _ in range(n_layers):
        q = [ckl.QuantWeights(4, mk(E_loc, d, F), group=128, asym=True) for _ in range(2)]
        q.append(ckl.QuantWeights(4, mk(E_loc, F, d), group=128, asym=True))
        layers.append((q, ckl.MoeEpLayer(win, *q)))
    ws = torch.empty(layers[0][1].workspace_size(), dtype=torch.uint8, device=dev)
    res = {}
    for name, T in [("T=1", 1), ("T=4", 4), ("T=16", 16), ("T=64", 64), ("T=64/GPU", 64 * world)]:
        Tr = _split(T, world, rank)
        T_max = _split(T, world, 0)                      # tokens on the busiest rank
        lg = [torch.randn((max(Tr, 1), E), generator=g, device=dev)[:Tr].contiguous()
              for _ in range(n_layers)]
        X = torch.randn((max(Tr, 1), d), generator=g, device=dev).half()[:Tr].contiguous()
        outs = [torch.empty((Tr, d), dtype=torch.float16, device=dev) for _ in range(n_layers)]
        ids = [torch.empty((Tr, k), dtype=torch.int32, device=dev) for _ in range(n_layers)]

        def step():
            x = X
            for l, (_, layer) in enumerate(layers):
                layer.forward(lg[l], x, out=outs[l], ids=ids[l], workspace=ws, T_max=T_max)
                x = outs[l]

        t = timer(GraphStep(step, dev)) / n_layers
        # algorithmic bytes: the local experts that received rows, summed over the GPUs
        act = []
        for l in range(n_layers):
            e_all = [None] * world
            import torch.distributed as dist
            dist.all_gather_object(e_all, ids[l].cpu().numpy().ravel().tolist())
            act.append(len(set(sum(e_all, []))))
        per_exp = sum(w.bytes_per_expert() for w in layers[0][0])
        byts = per_exp * sum(act) / n_layers + T * d * 2 * 2
        res[name] = {"us_per_layer": round(t * 1e3, 2), "tokens_per_gpu": Tr,
                     "active_experts_avg": round(sum(act) / n_layers, 1),
                     "bytes_per_layer_all_gpus": int(byts),
                     "GB/s_all_gpus": round(byts / (t * 1e-3) / 1e9, 1),
                     "frac_of_measured_hbm_all_gpus": round(byts / (t * 1e-3) / 1e9 / (peak * world), 3)}
    res["method"] = (f"{n_layers} layers with distinct weights ({E_loc} experts each per GPU) in "
                     "one CUDA graph per GPU, L2 flushed before each replay, per-layer time, max "
                     "over GPUs; dispatch/combine by the layer's kernels over NVLink (no NCCL)")
    torch.cuda.synchronize()
    del layers
    win.close()
    torch.cuda.empty_cache()
    return res


def ep_a2a_layer(ckl, q, lg, X, k, world, cap):
    """One expert-parallel MoE layer with NCCL all-to-all moving the rows: route on the
    token's GPU, scatter the permuted rows into fixed-capacity per-owner slabs [world][cap]
    (cap >= rows any GPU sends one owner), all_to_all_single the rows and the per-expert
    counts, build the owner's gather map on the device (no host sync), run the owner's
    experts (q = gate, up, down over E/world experts), send the fp32 rows back with a
    second all_to_all_single and combine. Every GPU makes the same collective calls."""
    import torch
    import torch.distributed as dist
    dev, d = X.device, X.shape[1]
    Tr, E_loc = X.shape[0], q[0].E
    i32 = dict(dtype=torch.int32, device=dev)
    S = torch.zeros((world * cap, d), dtype=torch.float16, device=dev)
    if Tr:
        r = ckl.route_and_permute(lg, X, k)
        rows = torch.arange(Tr * k, **i32)
        expert = torch.searchsorted(r["offsets"], rows, right=True) - 1
        owner = torch.div(expert, E_loc, rounding_mode="floor")
        slot_send = owner * cap + (rows - r["offsets"][owner * E_loc])          # [Tr*k]
        S.index_copy_(0, slot_send, r["Xp"])
        counts = r["counts"]
    else:
        counts = torch.zeros(world * E_loc, **i32)
    R = torch.empty_like(S)
    dist.all_to_all_single(R, S)
    cnt = torch.empty(world * E_loc, **i32)
    dist.all_to_all_single(cnt, counts.contiguous())
    cnt = cnt.view(world, E_loc).long()                                     # [src][expert]
    ends = torch.cumsum(cnt, 1)                                             # per src slab
    loc_off = torch.zeros(E_loc + 1, dtype=torch.long, device=dev)
    loc_off[1:] = torch.cumsum(cnt.sum(0), 0)
    before = torch.cumsum(cnt, 0) - cnt                                     # earlier srcs' rows
    sl = torch.arange(cap, device=dev).unsqueeze(0).expand(world, cap).contiguous()
    j = torch.searchsorted(ends, sl, right=True).clamp(max=E_loc - 1)       # expert of slot
    src = torch.arange(world, device=dev).unsqueeze(1).expand(world, cap)
    pos = loc_off[j] + before[src, j] + sl - (ends - cnt)[src, j]           # GEMM row of slot
    A = world * cap
    pos = torch.where(sl < ends[:, -1:], pos, torch.full_like(pos, A)).view(-1)   # empty -> spare
    row_src = torch.zeros(A + 1, **i32)
    row_src.index_copy_(0, pos, torch.arange(A, **i32))
    off = loc_off.int()
    h = ckl.expert_gemm_ex(R, row_src, off, A, q[0], q[1])
    y = ckl.expert_gemm_ex(h, None, off, A, q[2], None, y_f32=True)
    Sb = torch.cat([y, torch.zeros((1, d), dtype=torch.float32, device=dev)])[pos]
    Rb = torch.empty_like(Sb)
    dist.all_to_all_single(Rb, Sb)
    if not Tr:
        return torch.empty((0, d), dtype=torch.float16, device=dev)
    return ckl.combine(Rb[slot_send], r["inv_perm"], r["wts"], Tr, k)


def ep_replicated_layer(ckl, q, lg, X, k, rank, world, Tmax):
    """One expert-parallel MoE layer with replicated tokens: X and the logits all-gathered
    (every GPU's batch padded to Tmax rows; padding routes to some expert and is computed
    and discarded), every GPU runs its own experts (q over E/world experts) for the rows
    routed to them, the fp32 weighted partial outputs of all tokens are reduce-scattered
    back to the tokens' GPUs."""
    import torch
    import torch.distributed as dist
    dev, d = X.device, X.shape[1]
    Tr, E, E_loc = X.shape[0], lg.shape[1], q[0].E
    Xpad = torch.zeros((Tmax, d), dtype=torch.float16, device=dev)
    Xpad[:Tr] = X
    Lpad = torch.zeros((Tmax, E), dtype=torch.float32, device=dev)
    Lpad[:Tr] = lg
    T = world * Tmax
    Xall = torch.empty((T, d), dtype=torch.float16, device=dev)
    Lall = torch.empty((T, E), dtype=torch.float32, device=dev)
    dist.all_gather_into_tensor(Xall, Xpad)
    dist.all_gather_into_tensor(Lall, Lpad)
    r = ckl.route_and_permute(Lall, Xall, k)
    A = T * k
    off = r["offsets"][rank * E_loc:(rank + 1) * E_loc + 1]                  # rows of my experts
    h = ckl.expert_gemm_ex(r["Xp"], None, off, A, q[0], q[1])
    y = ckl.expert_gemm_ex(h, None, off, A, q[2], None, y_f32=True)
    rows = torch.arange(A, device=dev)
    mine = ((rows >= off[0]) & (rows < off[-1])).unsqueeze(1)
    y = torch.where(mine, y, torch.zeros((), dtype=y.dtype, device=dev))
    part = (y[r["inv_perm"].long()].view(T, k, d) * r["wts"].unsqueeze(2)).sum(1)
    out = torch.empty((Tmax, d), dtype=torch.float32, device=dev)
    dist.reduce_scatter_tensor(out, part)
    return out[:Tr].half()


def bench_seqsplit(ckl, dev, timer, peak, rank, world, exchange, L=32768):
    """Config 2's B=1 shape (1 x 32768) split by sequence over the GPUs: the single-GPU plan's
    chunks cut into one run per rank, each rank holding only its run's pages and writing its
    partial slots into rank 0's buffers (ckl_decode_partial over a peer-mapped buffer), a
    gather signal, then rank 0's wait and LSE merge. Cold L2 on every rank, ranks start each
    sample together, max over ranks."""
    import numpy as np
    import torch
    lens = np.array([L], np.int32)
    d, (lens, indptr, indices) = paged_batch(lens, dev, seed=7)
    nc, ct = ckl.plan_chunks(HQ // HKV, 1, HKV, L)
    lo, hi = rank * nc // world, (rank + 1) * nc // world
    t0, t1 = lo * ct, min(hi * ct, L)
    pages = torch.from_numpy(np.asarray(indices[t0 // PAGE:(t1 + PAGE - 1) // PAGE], np.int64)).to(dev)
    kl = d["k_cache"].index_select(0, pages).contiguous()
    vl = d["v_cache"].index_select(0, pages).contiguous()
    del d["k_cache"], d["v_cache"]
    n = pages.numel()
    t = lambda a: torch.tensor(a, dtype=torch.int32, device=dev)
    p = ckl.make_params(d["q"], kl, vl, t([0, n]), t(list(range(n))), t([t1 - t0 - (n - 1) * PAGE]),
                        num_chunks=hi - lo, chunk_tokens=ct, chunk_base=lo, part_stride=nc)
    o_bytes = (HQ * nc * D * 4 + 255) // 256 * 256
    win = ckl.IpcWindows(rank, world, o_bytes + HQ * nc * 4, exchange)
    grp = ckl.GatherGroup(rank, world, exchange)
    p.part_o, p.part_lse = win.ptrs[0], win.ptrs[0] + o_bytes
    out = torch.empty((1, HQ, D), dtype=torch.float16, device=dev)
    lse = torch.empty((1, HQ), dtype=torch.float32, device=dev)
    po = ckl.device_view(win.ptrs[0], (HQ, nc, D), torch.float32) if rank == 0 else None
    pl = ckl.device_view(win.ptrs[0] + o_bytes, (HQ, nc), torch.float32) if rank == 0 else None

    def step():
        ckl.decode_partial(p)
        grp.signal(0)
        if rank == 0:
            grp.wait()
            ckl.merge_states(po, pl, out, lse)

    ms = timer(step)
    byts = algorithmic_bytes(lens)
    torch.cuda.synchronize()
    res = {"1x32768": {"us": round(ms * 1e3, 1), "chunks": nc, "chunks_per_gpu": [lo, hi],
                       "GB/s_all_gpus": round(byts / (ms * 1e-3) / 1e9, 1),
                       "frac_of_measured_hbm_all_gpus": round(byts / (ms * 1e-3) / 1e9 / (peak * world), 3)},
           "method": "cold L2 (512 MB memset) on every rank, ranks start each sample together, "
                     "median of 31, max over ranks; partial slots over NVLink into rank 0, "
                     "gather flags, LSE merge on rank 0"}
    win.close()
    grp.close()
    del kl, vl
    torch.cuda.empty_cache()
    return res


def bench_moe_ep_designs(ckl, dev, timer, peak, rank, world, exchange, n_layers=8):
    """BASELINE config 4 expert-parallel, three ways of moving the tokens on the same local
    expert weights (experts [r*E/n, (r+1)*E/n) on GPU r) and the same inputs, each timed as
    n_layers layers in one CUDA graph (L2 flushed before every replay, per-layer time, max
    over GPUs):
      * ipc_kernels: ckl_moe_ep_layer, dispatch and combine by the layer's own kernels
        through IPC-mapped windows (this library's design);
      * nccl_all_to_all: ep_a2a_layer (fixed-capacity slabs, two NCCL all-to-alls);
      * nccl_replicated_reduce_scatter: ep_replicated_layer (all-gather, reduce-scatter);
      * *_collectives_only: each NCCL design's collectives alone, same sizes, no compute (the
        floor of that design whatever its glue).
    Each NCCL design's first-layer output is compared with the IPC layer's (relative RMS)."""
    import torch
    import torch.distributed as dist
    E, k, d, F, T_cap = 64, 6, 2048, 1408, 64
    E_loc = E // world
    g = torch.Generator(device=dev)
    g.manual_seed(4500 + rank)
    mk = lambda *sh: (torch.randn(*sh, generator=g, device=dev) * 0.02).half()
    win = ckl.EpWindows(rank, world, T_cap, k, E, d, exchange)
    layers = []
    for _ in range(n_layers):
        q = [ckl.QuantWeights(4, mk(E_loc, d, F), group=128, asym=True) for _ in range(2)]
        q.append(ckl.QuantWeights(4, mk(E_loc, F, d), group=128, asym=True))
        layers.append((q, ckl.MoeEpLayer(win, *q)))
    ws = torch.empty(layers[0][1].workspace_size(), dtype=torch.uint8, device=dev)
    res = {}
    for name, T in [("T=1", 1), ("T=16", 16), ("T=64", 64), ("T=64/GPU", 64 * world)]:
        Tc = [_split(T, world, rr) for rr in range(world)]
        Tr, Tmax = Tc[rank], max(Tc)
        cap = Tmax * min(k, E_loc)
        lg = [torch.randn((max(Tr, 1), E), generator=g, device=dev)[:Tr].contiguous()
              for _ in range(n_layers)]
        X = torch.randn((max(Tr, 1), d), generator=g, device=dev).half()[:Tr].contiguous()
        outs = {}
        ipc_out = [torch.empty((Tr, d), dtype=torch.float16, device=dev) for _ in range(n_layers)]

        def step_ipc():
            x = X
            for l, (_, layer) in enumerate(layers):
                layer.forward(lg[l], x, out=ipc_out[l], workspace=ws, T_max=Tmax)
                x = ipc_out[l]
            outs["ipc_kernels"] = ipc_out[0]

        def chain(key, fn):
            def step():
                x = X
                for l, (q, _) in enumerate(layers):
                    x = fn(q, lg[l], x)
                    if l == 0:
                        outs[key] = x
            return step

        steps = {"ipc_kernels": step_ipc,
                 "nccl_all_to_all": chain("nccl_all_to_all", lambda q, l_, x: ep_a2a_layer(
                     ckl, q, l_, x, k, world, cap)),
                 "nccl_replicated_reduce_scatter": chain(
                     "nccl_replicated_reduce_scatter",
                     lambda q, l_, x: ep_replicated_layer(ckl, q, l_, x, k, rank, world, Tmax))}
        # the NCCL designs' collectives alone (no routing, GEMMs or glue): their floor
        S16 = torch.zeros((world * cap, d), dtype=torch.float16, device=dev)
        R16, S32 = torch.empty_like(S16), torch.zeros((world * cap, d), dtype=torch.float32, device=dev)
        R32 = torch.empty_like(S32)
        cs, cr = (torch.zeros(E, dtype=torch.int32, device=dev) for _ in range(2))
        Xg, Lg = (torch.zeros((Tmax, n), dtype=t, device=dev) for n, t in ((d, torch.float16),
                                                                           (E, torch.float32)))
        Xa = torch.empty((world * Tmax, d), dtype=torch.float16, device=dev)
        La = torch.empty((world * Tmax, E), dtype=torch.float32, device=dev)
        P, O = torch.zeros((world * Tmax, d), dtype=torch.float32, device=dev), torch.empty(
            (Tmax, d), dtype=torch.float32, device=dev)

        def a2a_only():
            for _ in range(n_layers):
                dist.all_to_all_single(R16, S16)
                dist.all_to_all_single(cr, cs)
                dist.all_to_all_single(R32, S32)

        def replicated_only():
            for _ in range(n_layers):
                dist.all_gather_into_tensor(Xa, Xg)
                dist.all_gather_into_tensor(La, Lg)
                dist.reduce_scatter_tensor(O, P)

        steps["nccl_all_to_all_collectives_only"] = a2a_only
        steps["nccl_replicated_collectives_only"] = replicated_only
        row = {"tokens_per_gpu": Tr}
        graphs = {}
        for key, fn in steps.items():
            graphs[key] = GraphStep(fn, dev)
            row[key + "_us_per_layer"] = round(timer(graphs[key]) / n_layers * 1e3, 2)
        if Tr:
            ref = outs["ipc_kernels"].float()
            for key in ("nccl_all_to_all", "nccl_replicated_reduce_scatter"):
                row[key + "_rel_rms_vs_ipc"] = float(
                    (outs[key].float() - ref).norm() / max(float(ref.norm()), 1e-30))
        torch.cuda.synchronize()
        del graphs, outs
        res[name] = row
    res["method"] = (f"{n_layers} layers with distinct weights ({E_loc} experts per GPU) in one "
                     "CUDA graph per design and GPU, L2 flushed before each replay, per-layer "
                     "time, max over GPUs; rel_rms: first layer's output against the IPC "
                     "layer's, on rank 0")
    torch.cuda.synchronize()
    dist.barrier()
    del layers
    win.close()
    torch.cuda.empty_cache()
    return res


def bench_mixtral_ep(ckl, dev, timer, peak, rank, world, exchange):
    """BASELINE config 5 on several GPUs: attention of B=32 sequences of 4096 with the KV
    heads sharded over the GPUs (each GPU decodes its 8/n KV heads for all sequences), then
    the MoE block (E=8, top-2, d=4096, F=14336, int8 per channel) expert-parallel with the
    T=32 tokens split over the GPUs. One step = attention + MoE from one CUDA graph, cold L2,
    max over GPUs. (The o_proj GEMM and its reduce-scatter between them are outside the
    reference's layer and not run.)"""
    import numpy as np
    import torch
    B, L = 32, 4096
    E, k, d, F = 8, 2, 4096, 14336
    hk = HKV // world
    lens = np.full(B, L, np.int32)
    npg = (lens + PAGE - 1) // PAGE
    indptr = np.zeros(B + 1, np.int32)
    indptr[1:] = np.cumsum(npg)
    last = (lens - (npg - 1) * PAGE).astype(np.int32)
    indices = np.random.default_rng(55).permutation(int(indptr[-1])).astype(np.int32)
    g = torch.Generator(device=dev)
    g.manual_seed(5500 + rank)
    kc = torch.empty((int(indptr[-1]), PAGE, hk, D), dtype=torch.float16, device=dev)
    vc = torch.empty_like(kc)
    _fill_uniform(kc, g)
    _fill_uniform(vc, g)
    t_ = lambda a: torch.from_numpy(a).to(dev)
    d_attn = dict(q=(torch.rand((B, HQ // world, D), generator=g, device=dev) * 2 - 1).half(),
                  k_cache=kc, v_cache=vc, kv_indptr=t_(indptr), kv_indices=t_(indices),
                  kv_last_page_len=t_(last))
    nc, ct = ckl.plan_chunks(HQ // HKV, B, hk, L)
    pa = ckl.make_params(**d_attn, num_chunks=nc, chunk_tokens=ct)
    a_out = torch.empty_like(d_attn["q"])
    a_lse = torch.empty((B, HQ // world), dtype=torch.float32, device=dev)
    a_ws = torch.empty(max(ckl.workspace_size(pa), 256), dtype=torch.uint8, device=dev)
    mk = lambda *sh: (torch.randn(*sh, generator=g, device=dev) * 0.02).half()
    E_loc = E // world
    q = [ckl.QuantWeights(8, mk(E_loc, d, F), group=d), ckl.QuantWeights(8, mk(E_loc, d, F), group=d),
         ckl.QuantWeights(8, mk(E_loc, F, d), group=F)]
    Tr = _split(B, world, rank)
    win = ckl.EpWindows(rank, world, (B + world - 1) // world, k, E, d, exchange)
    layer = ckl.MoeEpLayer(win, *q)
    lg = torch.randn((max(Tr, 1), E), generator=g, device=dev)[:Tr].contiguous()
    X = torch.randn((max(Tr, 1), d), generator=g, device=dev).half()[:Tr].contiguous()
    out = torch.empty((Tr, d), dtype=torch.float16, device=dev)
    ids = torch.empty((Tr, k), dtype=torch.int32, device=dev)
    ws = torch.empty(layer.workspace_size(), dtype=torch.uint8, device=dev)

    def attn():
        ckl.decode_attention(**d_attn, num_chunks=nc, chunk_tokens=ct, out=a_out, lse=a_lse,
                             workspace=a_ws)

    def moe():
        layer.forward(lg, X, out=out, ids=ids, workspace=ws, T_max=_split(B, world, 0))

    def step():
        attn()
        moe()

    t_attn = timer(GraphStep(attn, dev))
    t_moe = timer(GraphStep(moe, dev))
    t_step = timer(GraphStep(step, dev))
    import torch.distributed as dist
    e_all = [None] * world
    dist.all_gather_object(e_all, ids.cpu().numpy().ravel().tolist())
    active = len(set(sum(e_all, [])))
    attn_bytes = algorithmic_bytes(lens)
    moe_bytes = active * sum(w.bytes_per_expert() for w in q) + B * d * 2 * 2
    res = {"us_step": round(t_step * 1e3, 2), "us_attention": round(t_attn * 1e3, 2),
           "us_moe": round(t_moe * 1e3, 2), "attention_bytes_all_gpus": attn_bytes,
           "moe_bytes_all_gpus": moe_bytes, "moe_active_experts": active,
           "GB/s_step_all_gpus": round((attn_bytes + moe_bytes) / (t_step * 1e-3) / 1e9, 1),
           "frac_of_measured_hbm_all_gpus":
               round((attn_bytes + moe_bytes) / (t_step * 1e-3) / 1e9 / (peak * world), 3)}
    torch.cuda.synchronize()
    del layer, q, d_attn
    win.close()
    torch.cuda.empty_cache()
    return res


# ------------------------------------------------------------------ our arm
def run_ours(args):
    import numpy as np
    import torch
    import ckl

    rank, world, local = dist_setup(args.gpus)
    dev = torch.device("cuda", local)
    if HKV % world:
        sys.exit(f"--gpus {world}: the {HKV} KV heads do not shard {world} ways")
    hk, hq = HKV // world, HQ // world              # this GPU's KV / q heads
    lens = np.tile(lengths(args.workload), world)    # weak scaling: B grows with the GPUs
    B = len(lens)
    npg = (lens + PAGE - 1) // PAGE
    indptr = np.zeros(B + 1, np.int32)
    indptr[1:] = np.cumsum(npg)
    last = (lens - (npg - 1) * PAGE).astype(np.int32)
    num_pages = int(indptr[-1])
    rng = np.random.default_rng(1000)                # the page table is replicated
    indices = rng.permutation(num_pages).astype(np.int32)

    g = torch.Generator(device=dev)
    g.manual_seed(1000 + rank)
    k = torch.empty((num_pages, PAGE, hk, D), dtype=torch.float16, device=dev)
    v = torch.empty_like(k)
    _fill_uniform(k, g)
    _fill_uniform(v, g)
    q_host = (torch.rand((B, hq, D), generator=g, device=dev) * 2 - 1).half().cpu().pin_memory()
    d_q = q_host.to(dev)
    d_indptr = torch.from_numpy(indptr).to(dev)
    d_indices = torch.from_numpy(indices).to(dev)
    d_last = torch.from_numpy(last).to(dev)
    nc, ct = ckl.plan_chunks(HQ // HKV, B, hk, int(lens.max()))
    p = ckl.make_params(d_q, k, v, d_indptr, d_indices, d_last, num_chunks=nc, chunk_tokens=ct)
    ws_n = ckl.workspace_size(p)
    ws = torch.empty(max(ws_n, 256), dtype=torch.uint8, device=dev)
    stream = torch.cuda.current_stream()
    byts = algorithmic_bytes(lens) // world          # this GPU's share (its heads)

    import ctypes as C
    L = ckl.lib()
    sptr = C.c_void_p(stream.cuda_stream)
    if world == 1:
        out = torch.empty((B, HQ, D), dtype=torch.float16, device=dev)
        lse = torch.empty((B, HQ), dtype=torch.float32, device=dev)
        out_ptr, lse_ptr, win, grp = out.data_ptr(), lse.data_ptr(), None, None
        launches_per_step = 1 if nc == 1 else 2
    else:
        # rank 0's output [B, Hq, 128] + lse lives in an IPC window every rank maps
        ex = ckl.torch_exchange()
        out_bytes = (B * HQ * D * 2 + 255) // 256 * 256
        win = ckl.IpcWindows(rank, world, out_bytes + B * HQ * 4, ex)
        grp = ckl.GatherGroup(rank, world, ex)
        out_ptr, lse_ptr = win.ptrs[0], win.ptrs[0] + out_bytes
        out = ckl.device_view(win.ptrs[rank], (B, HQ, D), torch.float16) if rank == 0 else None
        lse = ckl.device_view(win.ptrs[rank] + out_bytes, (B, HQ), torch.float32) if rank == 0 else None
        launches_per_step = (1 if nc == 1 else 2) + 1 + (1 if rank == 0 else 0)

    def step():
        if world == 1:
            ckl.check(L.ckl_decode_attention(C.byref(p), C.c_void_p(out_ptr),
                                             C.c_void_p(lse_ptr), C.c_void_p(ws.data_ptr()),
                                             ws.numel(), sptr), "ckl_decode_attention")
            return
        ckl.check(L.ckl_decode_attention_gather(C.byref(p), C.c_void_p(out_ptr),
                                                C.c_void_p(lse_ptr), HQ, rank * hq,
                                                C.c_void_p(ws.data_ptr()), ws.numel(), sptr),
                  "ckl_decode_attention_gather")
        grp.signal(0, stream)
        if rank == 0:
            grp.wait(stream)

    # ---- device-resident timing (value)
    for _ in range(args.warmup):
        step()
    barrier(world)
    clocks = Clocks(local)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier(world)
    clocks.start()
    e0.record(stream)
    for _ in range(args.steps):
        step()
    e1.record(stream)
    barrier(world)
    clk = clocks.stop()
    ms = e0.elapsed_time(e1) / args.steps
    ms_max = max_over_ranks(ms, world)
    ckl.check_device_error()

    # ---- dominant kernel alone (the partial kernel), for the roofline
    if nc == 1:
        kern_ms = ms
    else:
        pp = ckl.make_params(d_q, k, v, d_indptr, d_indices, d_last, num_chunks=nc,
                             chunk_tokens=ct)
        po_bytes = ((B * hq * nc * D * 4 + 255) // 256) * 256   # workspace layout
        pp.part_o = ws.data_ptr()
        pp.part_lse = ws.data_ptr() + po_bytes
        for _ in range(3):
            ckl.decode_partial(pp)
        torch.cuda.synchronize()
        e0.record(stream)
        for _ in range(args.steps):
            ckl.decode_partial(pp)
        e1.record(stream)
        torch.cuda.synchronize()
        kern_ms = e0.elapsed_time(e1) / args.steps

    # ---- end to end through the C-ABI with host buffers (every GPU copies its q shard and
    # the page table in; rank 0 reads the gathered output and lse back)
    h_indptr = torch.from_numpy(indptr).pin_memory()
    h_indices = torch.from_numpy(indices).pin_memory()
    h_last = torch.from_numpy(last).pin_memory()
    h_out = torch.empty((B, HQ, D), dtype=torch.float16).pin_memory() if rank == 0 else None
    h_lse = torch.empty((B, HQ), dtype=torch.float32).pin_memory() if rank == 0 else None
    h2d = q_host.numel() * 2 + h_indptr.numel() * 4 + h_indices.numel() * 4 + h_last.numel() * 4
    d2h = B * HQ * D * 2 + B * HQ * 4 if rank == 0 else 0

    out_final = out
    if world == 1:
        # One GPU: double-buffered, as a serving loop runs it. Step s's q and page table go in
        # on one copy stream and its out and lse come back on another (PCIe is full duplex),
        # while the neighbouring steps' kernels run; every step still copies all of its
        # inputs from pinned host memory and reads all of its results back, inside the timed
        # region. Buffer set s % 2 is rewritten only after step s-2's kernels and readback.
        sets = []
        for _ in range(2):
            bq, bip, bix, bl = (torch.empty_like(t) for t in (d_q, d_indptr, d_indices, d_last))
            bp = ckl.make_params(bq, k, v, bip, bix, bl, num_chunks=nc, chunk_tokens=ct)
            bo, bs = torch.empty_like(out), torch.empty_like(lse)
            sets.append((bq, bip, bix, bl, bp, bo, bs, torch.empty_like(h_out).pin_memory(),
                         torch.empty_like(h_lse).pin_memory()))
        up, down = torch.cuda.Stream(dev), torch.cuda.Stream(dev)
        ev_in, ev_done, ev_back = ([torch.cuda.Event() for _ in range(2)] for _ in range(3))

        def e2e_run(n, start=None):
            for s_ in range(n):
                b = s_ % 2
                bq, bip, bix, bl, bp, bo, bs, ho, hs = sets[b]
                if s_ >= 2:
                    up.wait_event(ev_done[b])
                elif start is not None:
                    up.wait_event(start)
                with torch.cuda.stream(up):
                    bq.copy_(q_host, non_blocking=True)
                    bip.copy_(h_indptr, non_blocking=True)
                    bix.copy_(h_indices, non_blocking=True)
                    bl.copy_(h_last, non_blocking=True)
                ev_in[b].record(up)
                stream.wait_event(ev_in[b])
                if s_ >= 2:
                    stream.wait_event(ev_back[b])
                ckl.check(L.ckl_decode_attention(C.byref(bp), C.c_void_p(bo.data_ptr()),
                                                 C.c_void_p(bs.data_ptr()), C.c_void_p(ws.data_ptr()),
                                                 ws.numel(), sptr), "ckl_decode_attention")
                ev_done[b].record(stream)
                down.wait_event(ev_done[b])
                with torch.cuda.stream(down):
                    ho.copy_(bo, non_blocking=True)
                    hs.copy_(bs, non_blocking=True)
                ev_back[b].record(down)
            for b in range(min(n, 2)):                   # the last readbacks have landed
                stream.wait_event(ev_back[b])

        e2e_run(args.warmup)
        torch.cuda.synchronize()
        e0.record(stream)
        e2e_run(args.steps, start=e0)
        e1.record(stream)
        torch.cuda.synchronize()
        e2e_ms = e0.elapsed_time(e1) / args.steps
        out_final = sets[(args.steps - 1) % 2][5]
    else:
        # N GPUs: double-buffered too. Two output windows on rank 0 (each rank's kernels store
        # their head rows into window s % 2), per-rank input sets on an upload stream, rank 0
        # reading window s % 2 back on a download stream while step s+1 runs. Before any rank
        # writes a window again (step s+2), every rank passes a peer barrier (ckl_peer_barrier)
        # that rank 0 reaches only after its readback of step s has landed.
        out_bytes2 = (B * HQ * D * 2 + 255) // 256 * 256
        win2 = ckl.IpcWindows(rank, world, out_bytes2 + B * HQ * 4, ex)
        wins = [(win.ptrs[0], win.ptrs[0] + out_bytes), (win2.ptrs[0], win2.ptrs[0] + out_bytes2)]
        sets = []
        for b_ in range(2):
            bq, bip, bix, bl = (torch.empty_like(t) for t in (d_q, d_indptr, d_indices, d_last))
            bp = ckl.make_params(bq, k, v, bip, bix, bl, num_chunks=nc, chunk_tokens=ct)
            ho = torch.empty_like(h_out).pin_memory() if rank == 0 else None
            hs = torch.empty_like(h_lse).pin_memory() if rank == 0 else None
            src = None
            if rank == 0:
                src = (ckl.device_view(wins[b_][0], (B, HQ, D), torch.float16),
                       ckl.device_view(wins[b_][1], (B, HQ), torch.float32))
            sets.append((bq, bip, bix, bl, bp, ho, hs, src))
        up, down = torch.cuda.Stream(dev), torch.cuda.Stream(dev)
        ev_in, ev_done, ev_back = ([torch.cuda.Event() for _ in range(2)] for _ in range(3))

        def e2e_run(n, start=None):
            for s_ in range(n):
                b_ = s_ % 2
                bq, bip, bix, bl, bp, ho, hs, src = sets[b_]
                if s_ >= 2:
                    up.wait_event(ev_done[b_])
                elif start is not None:
                    up.wait_event(start)
                with torch.cuda.stream(up):
                    bq.copy_(q_host, non_blocking=True)
                    bip.copy_(h_indptr, non_blocking=True)
                    bix.copy_(h_indices, non_blocking=True)
                    bl.copy_(h_last, non_blocking=True)
                ev_in[b_].record(up)
                stream.wait_event(ev_in[b_])
                if s_ >= 2:
                    if rank == 0:
                        stream.wait_event(ev_back[b_])
                    grp.barrier(stream)
                ckl.check(L.ckl_decode_attention_gather(C.byref(bp), C.c_void_p(wins[b_][0]),
                                                        C.c_void_p(wins[b_][1]), HQ, rank * hq,
                                                        C.c_void_p(ws.data_ptr()), ws.numel(), sptr),
                          "ckl_decode_attention_gather")
                grp.signal(0, stream)
                if rank == 0:
                    grp.wait(stream)
                ev_done[b_].record(stream)
                if rank == 0:
                    down.wait_event(ev_done[b_])
                    with torch.cuda.stream(down):
                        ho.copy_(src[0], non_blocking=True)
                        hs.copy_(src[1], non_blocking=True)
                    ev_back[b_].record(down)
            if rank == 0:
                for b_ in range(min(n, 2)):               # the last readbacks have landed
                    stream.wait_event(ev_back[b_])

        e2e_run(args.warmup)
        torch.cuda.synchronize()
        barrier(world)
        e0.record(stream)
        e2e_run(args.steps, start=e0)
        e1.record(stream)
        torch.cuda.synchronize()
        barrier(world)
        e2e_ms = max_over_ranks(e0.elapsed_time(e1) / args.steps, world)
        if rank == 0:
            out_final = sets[(args.steps - 1) % 2][7][0]

    # correctness of what was timed: the last sequence's rows, read from the (gathered)
    # output on rank 0, against a plain fp32 torch check that every GPU computes for its own
    # heads from its own K/V shard (torch only ever touches local memory)
    b0 = B - 1
    pages = indices[indptr[b0]:indptr[b0 + 1]]
    kk = k[torch.from_numpy(pages.astype(np.int64)).to(dev)].reshape(-1, hk, D)[:lens[b0]].float()
    vv = v[torch.from_numpy(pages.astype(np.int64)).to(dev)].reshape(-1, hk, D)[:lens[b0]].float()
    qq = d_q[b0].float().view(hk, HQ // HKV, D)
    s_ = torch.einsum("hgd,lhd->hgl", qq, kk) / math.sqrt(D)
    ref = torch.einsum("hgl,lhd->hgd", torch.softmax(s_, -1), vv).reshape(hq, D).cpu()
    if world > 1:
        import torch.distributed as dist
        refs = [None] * world
        dist.all_gather_object(refs, ref)
        ref = torch.cat(refs)
    chk_err = float((out_final[b0].float().cpu() - ref).abs().max()) if rank == 0 else 0.0

    peak, peak_kind = measured_peak()
    achieved = byts / (kern_ms * 1e-3) / 1e9
    srd = stream_read_ceiling(ckl, dev)
    extras = {}
    if not args.no_extras:
        del k, v
        torch.cuda.empty_cache()
        timer = ColdTimer(dev, world)
        want = set(filter(None, args.extras.split(",")))
        run = lambda name: not want or name in want
        if world == 1:
            rows = (("config2_sweep", sweep_config2), ("config2_multilayer", bench_decode_multilayer),
                    ("config3_cascade", bench_cascade),
                    ("prefix_tree_cascade", bench_cascade_tree),
                    ("config4_moe_w4a16_layer", bench_moe),
                    ("config5_mixtral_layer", bench_mixtral_layer),
                    ("grouped_gemm_tcgen05", bench_grouped_gemm),
                    ("decode_step_4_layers_config5", bench_decode_step))
            for name, fn in rows:
                if run(name):
                    extras[name] = fn(ckl, dev, timer, peak)
        else:
            ex = ckl.torch_exchange()
            if run("config2_1x32768_seqsplit"):
                extras["config2_1x32768_seqsplit"] = bench_seqsplit(ckl, dev, timer, peak, rank,
                                                                    world, ex)
            if "config4_moe_ep_designs" in want:           # opt-in: NCCL designs compared
                extras["config4_moe_ep_designs"] = bench_moe_ep_designs(ckl, dev, timer, peak, rank,
                                                                        world, ex)
            if run("config4_moe_w4a16_layer_ep"):
                extras["config4_moe_w4a16_layer_ep"] = bench_moe_ep(ckl, dev, timer, peak, rank,
                                                                    world, ex)
            if run("config5_mixtral_layer_tp_ep"):
                extras["config5_mixtral_layer_tp_ep"] = bench_mixtral_ep(ckl, dev, timer, peak,
                                                                         rank, world, ex)
        extras["extras_timing"] = ("cold L2 (512 MB memset before each sample), median of 31"
                                   + ("; ranks start each sample together (barrier), max over "
                                      "ranks" if world > 1 else ""))
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        cpu = cpu_baseline_sample(int(lens.max()), os.cpu_count() or 1)
    if rank == 0:
        line = {
            "metric": METRIC, "value": byts * world / (ms_max * 1e-3) / 1e9, "unit": "GB/s",
            "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms_max,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "fp16",
            "data": "synthetic: U(-1,1) fp16 K/V/q filled on device, seeded shuffled page table",
            "config": config_of(args.workload, lens, world),
            "frac_of_hbm": byts * world / (ms_max * 1e-3) / 1e9 / (peak * world),
            "denominators": {"measured_copy_gbs": peak, "reference_stream_read_gbs": srd,
                             "nominal_hbm_gbs": NOMINAL_HBM_GBS,
                             "frac_of_stream_read": byts / (ms_max * 1e-3) / 1e9 / srd,
                             "frac_of_nominal": byts / (ms_max * 1e-3) / 1e9 / NOMINAL_HBM_GBS,
                             "stream_read": "this GPU, 2 GiB, ckl_stream_read (the reference's "
                                            "stream_read probe), mean of 10 reads after 3 warm-up"},
            "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                         "frac": achieved / peak, "peak_source": peak_kind,
                         "kernel": "decode_partial_kernel<4>",
                         "algorithmic_bytes_per_launch": byts,
                         "traffic": committed_traffic("decode_partial_kernel<4>", args.workload)
                                    if world == 1 else None},
            "e2e": {"value": byts * world / (e2e_ms * 1e-3) / 1e9, "unit": "GB/s",
                    "ms_per_step": e2e_ms, "h2d_bytes_per_step": h2d * world,
                    "d2h_bytes_per_step": d2h,
                    "copies": ("double-buffered: each step's H2D and D2H on two copy streams, "
                               "overlapping the neighbouring steps' kernels") if world == 1 else
                              ("double-buffered: every rank's H2D on an upload stream, rank 0's "
                               "D2H of the gathered output (two output windows) on a download "
                               "stream overlapping the next step; a peer barrier before a window "
                               "is written again")},
            "gpu_launches": launches_per_step * args.steps,
            "plan": {"num_chunks": nc, "chunk_tokens": ct},
            "check_max_abs_err_vs_fp32": chk_err,
            "cpu_baseline": cpu,
            "clocks": clk,
        }
        line.update(extras)
        print(json.dumps(line))
    if world > 1:
        import torch.distributed as dist
        torch.cuda.synchronize()
        win.close()
        win2.close()
        grp.close()
        dist.barrier()
        dist.destroy_process_group()
    return 0


# ------------------------------------------------------------------ profiler probes
# Each probe builds one workload of the bench rows above, calls it `calls` times with a 512 MB
# memset between calls (cold L2, as in the timed rows) and prints the CUDA-event median. They
# are the commands behind the ncu summaries in profiles/ (run them under ncu with -k / -s / -c
# to pick the launches), small enough for a multi-pass capture: a few hundred MB on the device.
def _probe_moe_layer(ckl, dev, T, calls):
    import torch
    E, k, d, F = 64, 6, 2048, 1408
    g = torch.Generator(device=dev)
    g.manual_seed(44)
    mk = lambda *sh: (torch.randn(*sh, generator=g, device=dev) * 0.02).half()
    q = [ckl.QuantWeights(4, mk(E, d, F), group=128, asym=True) for _ in range(2)]
    q.append(ckl.QuantWeights(4, mk(E, F, d), group=128, asym=True))
    layer = ckl.MoeLayer(*q)
    lg = torch.randn((T, E), generator=g, device=dev)
    X = torch.randn((T, d), generator=g, device=dev).half()
    out = torch.empty((T, d), dtype=torch.float16, device=dev)
    ws = torch.empty(layer.workspace_size(T, k), dtype=torch.uint8, device=dev)
    return lambda: layer.forward(lg, X, k, out=out, workspace=ws)


def _probe_moe_gemms(ckl, dev, T, calls):
    """The layer's two expert GEMMs through the single-GEMM entry point (moe_gemm.cu)."""
    import torch
    E, k, d, F = 64, 6, 2048, 1408
    g = torch.Generator(device=dev)
    g.manual_seed(44)
    mk = lambda *sh: (torch.randn(*sh, generator=g, device=dev) * 0.02).half()
    gq, uq = (ckl.QuantWeights(4, mk(E, d, F), group=128, asym=True) for _ in range(2))
    dq = ckl.QuantWeights(4, mk(E, F, d), group=128, asym=True)
    lg = torch.randn((T, E), generator=g, device=dev)
    X = torch.randn((T, d), generator=g, device=dev).half()
    r = ckl.route_and_permute(lg, X, k)
    A = T * k

    def run():
        h = ckl.expert_gemm_ex(r["Xp"], None, r["offsets"], A, gq, uq)
        ckl.expert_gemm_ex(h, None, r["offsets"], A, dq, None, y_f32=True)
    return run


def _probe_cascade_tree(ckl, dev, calls):
    import numpy as np
    import torch
    d, (lens, indptr, indices), _ = tree_batch(1024, 4096, 4, np.full(64, 256), dev, seed=23)
    base = ckl.make_params(**d, num_chunks=1, chunk_tokens=16)
    tp = ckl.plan_cascade_tree(base, indptr, indices, lens, 256)
    ws = torch.empty(max(ckl.cascade_tree_workspace_size(tp), 256), dtype=torch.uint8, device=dev)
    out = torch.empty_like(d["q"])
    lse = torch.empty((len(lens), HQ), dtype=torch.float32, device=dev)
    return lambda: ckl.cascade_tree_decode(tp, out=out, lse=lse, workspace=ws)


def _probe_cascade_config3(ckl, dev, calls):
    import numpy as np
    import torch
    lens = (4096 + np.full(64, 256)).astype(np.int32)
    d, (lens, indptr, indices) = paged_batch(lens, dev, seed=21, Lp=4096)
    base = ckl.make_params(**d, num_chunks=1, chunk_tokens=16)
    cp = ckl.plan_cascade(base, indptr, indices, lens, 256)
    ws = torch.empty(max(ckl.cascade_workspace_size(cp), 256), dtype=torch.uint8, device=dev)
    out = torch.empty_like(d["q"])
    lse = torch.empty((len(lens), HQ), dtype=torch.float32, device=dev)
    return lambda: ckl.cascade_decode(cp, out=out, lse=lse, workspace=ws)


def _probe_grouped(ckl, dev, calls):
    import torch
    T, E, k, d, f = 512, 8, 2, 4096, 14336
    g = torch.Generator(device=dev)
    g.manual_seed(T + E)
    lg = torch.randn((T, E), generator=g, device=dev)
    X = (torch.rand((T, d), generator=g, device=dev) * 2 - 1).half()
    W = ((torch.rand((E, d, f), generator=g, device=dev) * 2 - 1) / d ** 0.5).half()
    r = ckl.route_and_permute(lg, X, k)
    out = torch.empty((T * k, f), dtype=torch.float16, device=dev)
    return lambda: ckl.grouped_gemm(r["Xp"], W, r["offsets"], out=out)


def _probe_decode(ckl, dev, name, calls):
    import torch
    lens = lengths(name)
    d, _ = paged_batch(lens, dev, seed=7)
    nc, ct = ckl.plan_chunks(HQ // HKV, len(lens), HKV, int(lens.max()))
    p = ckl.make_params(**d, num_chunks=nc, chunk_tokens=ct)
    out = torch.empty_like(d["q"])
    lse = torch.empty((len(lens), HQ), dtype=torch.float32, device=dev)
    ws = torch.empty(max(ckl.workspace_size(p), 256), dtype=torch.uint8, device=dev)
    return lambda: ckl.decode_attention(**d, num_chunks=nc, chunk_tokens=ct, out=out, lse=lse,
                                        workspace=ws)


PROBES = {
    **{f"moe_layer_T{T}": (lambda T: lambda ckl, dev, c: _probe_moe_layer(ckl, dev, T, c))(T)
       for T in (1, 4, 16, 64)},
    **{f"moe_gemms_T{T}": (lambda T: lambda ckl, dev, c: _probe_moe_gemms(ckl, dev, T, c))(T)
       for T in (1, 64)},
    "cascade_tree": _probe_cascade_tree,
    "cascade_config3": _probe_cascade_config3,
    "grouped_mixtral_T512": _probe_grouped,
    "decode_64x1024": lambda ckl, dev, c: _probe_decode(ckl, dev, "64x1024", c),
    "decode_1x32768": lambda ckl, dev, c: _probe_decode(ckl, dev, "1x32768", c),
}


def run_probe(args, calls=6):
    import torch
    import ckl
    dev = torch.device("cuda", 0)
    fn = PROBES[args.probe](ckl, dev, calls)
    timer = ColdTimer(dev)
    ms = timer(fn, iters=calls, warmup=3)
    torch.cuda.synchronize()
    ckl.check_device_error()
    print(json.dumps({"probe": args.probe, "calls": calls + 3, "median_ms_cold": ms}))
    return 0


def main():
    args = parse()
    if args.probe:
        return run_probe(args)
    if args.impl == "reference":
        return run_reference(args)
    return run_ours(args)


if __name__ == "__main__":
    sys.exit(main())
