"""ctypes binding of the CPU oracle (test infrastructure, never the product).

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg import this module.
It wraps oracle/libckl_oracle.so (the C++ restatement of the reference's generators and
fp64 CPU references, see ckl_oracle.cpp) and, when it was built, oracle/_ref/libref01.so /
libref03.so (the reference's own host code compiled from its sources).

All arrays are numpy; fp16 tensors travel as numpy.float16 (bit-identical to the uint16
patterns the C side uses).
"""
from __future__ import annotations

import ctypes as C
import os

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
HEAD_DIM = 128
PAGE = 16
GS = 128

_lib = None
_ref01 = None
_ref03 = None


def _p(a):
    return None if a is None else a.ctypes.data_as(C.c_void_p)


def lib():
    global _lib
    if _lib is None:
        path = os.path.join(HERE, "libckl_oracle.so")
        if not os.path.exists(path):
            raise RuntimeError(f"oracle library missing: {path} (run make -C oracle)")
        L = C.CDLL(path)
        vp, i, u, f, sz = C.c_void_p, C.c_int, C.c_uint, C.c_float, C.c_size_t
        sig = {
            "ora_f32_to_f16": (None, [vp, vp, sz]),
            "ora_f16_to_f32": (None, [vp, vp, sz]),
            "ora_batch_layout": (i, [vp, i, vp, vp]),
            "ora_batch_generate": (None, [vp, i, i, i, u, i, vp, vp, vp, vp, vp, vp]),
            "ora_shared_prefix_num_pages": (i, [i, vp, i]),
            "ora_shared_prefix_generate": (None, [i, vp, i, i, i, u, i, vp, vp, vp, vp, vp, vp]),
            "ora_attention_ref": (None, [i, i, i, vp, vp, vp, vp, vp, vp, vp, vp, vp, i, i]),
            "ora_plan_chunks": (None, [i, i, i, i, i, vp, vp]),
            "ora_shared_prefix_pages": (i, [vp, vp, i]),
            "ora_make_logits": (None, [i, i, u, i, i, vp]),
            "ora_normal": (None, [sz, u, f, f, vp, vp]),
            "ora_init_uniform": (None, [vp, sz, u, f]),
            "ora_route": (None, [vp, i, i, i, vp, vp]),
            "ora_permute": (None, [vp, i, i, i, vp, vp, vp, vp]),
            "ora_quant_sym": (None, [vp, i, i, i, i, i, vp, vp, i]),
            "ora_quant_asym4": (None, [vp, i, i, i, vp, vp, vp, i]),
            "ora_dequant": (None, [vp, vp, vp, i, i, i, i, i, vp]),
            "ora_expert_gemm": (None, [vp, vp, vp, i, i, i, vp, i]),
            "ora_moe_layer": (None, [vp, i, i, i, i, i, vp, vp, vp, vp, vp, vp, vp, i]),
            "ora_combine": (None, [vp, vp, vp, i, i, i, vp]),
        }
        for name, (res, args) in sig.items():
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _lib = L
    return _lib


def nthreads():
    return max(1, os.cpu_count() or 1)


# ------------------------------------------------------------------ attention
class Batch:
    """A generated paged batch (restates Batch / make_shared_prefix_batch)."""

    def __init__(self, lens, Hq, Hkv, indptr, indices, last, q, k, v):
        self.lens = np.asarray(lens, dtype=np.int32)
        self.B = len(self.lens)
        self.Hq, self.Hkv = Hq, Hkv
        self.indptr, self.indices, self.last = indptr, indices, last
        self.q, self.k, self.v = q, k, v
        self.num_pages = int(indptr[-1]) if k is None else k.shape[0]
        self.max_len = int(self.lens.max()) if self.B else 0


def batch(lens, Hq, Hkv, seed, fill=True):
    lens = np.ascontiguousarray(lens, dtype=np.int32)
    B = len(lens)
    indptr = np.zeros(B + 1, np.int32)
    last = np.zeros(B, np.int32)
    npages = int(np.sum((lens + PAGE - 1) // PAGE))
    indices = np.zeros(max(npages, 1), np.int32)[:npages]
    q = np.zeros((B, Hq, HEAD_DIM), np.float16)
    k = v = None
    if fill:
        k = np.empty((npages, PAGE, Hkv, HEAD_DIM), np.float16)
        v = np.empty_like(k)
    lib().ora_batch_generate(_p(lens), B, Hq, Hkv, seed, int(fill), _p(indptr), _p(indices),
                             _p(last), _p(q), _p(k), _p(v))
    return Batch(lens, Hq, Hkv, indptr, indices, last, q, k, v)


def shared_prefix_batch(Lp, suffix, Hq, Hkv, seed, fill=True):
    suffix = np.ascontiguousarray(suffix, dtype=np.int32)
    B = len(suffix)
    total = lib().ora_shared_prefix_num_pages(Lp, _p(suffix), B)
    lens = Lp + suffix
    npages_list = int(np.sum((lens + PAGE - 1) // PAGE))
    indptr = np.zeros(B + 1, np.int32)
    last = np.zeros(B, np.int32)
    indices = np.zeros(npages_list, np.int32)
    q = np.zeros((B, Hq, HEAD_DIM), np.float16)
    k = v = None
    if fill:
        k = np.empty((total, PAGE, Hkv, HEAD_DIM), np.float16)
        v = np.empty_like(k)
    lib().ora_shared_prefix_generate(Lp, _p(suffix), B, Hq, Hkv, seed, int(fill), _p(indptr),
                                     _p(indices), _p(last), _p(q), _p(k), _p(v))
    bt = Batch(lens, Hq, Hkv, indptr, indices, last, q, k, v)
    bt.num_pages = total
    return bt


def attention_ref(bt: Batch, rows=None, threads=None):
    """fp64 attention (restates cpu_reference). Returns (out fp32 [B,Hq,128], lse [B,Hq]).
    rows: optional flat list of b*Hq+h rows to compute (others stay NaN)."""
    out = np.full((bt.B, bt.Hq, HEAD_DIM), np.nan, np.float32)
    lse = np.full((bt.B, bt.Hq), np.nan, np.float32)
    rl = None if rows is None else np.ascontiguousarray(rows, dtype=np.int32)
    lib().ora_attention_ref(bt.B, bt.Hq, bt.Hkv, _p(bt.indptr), _p(bt.indices), _p(bt.lens),
                            _p(bt.q), _p(bt.k), _p(bt.v), _p(out), _p(lse), _p(rl),
                            0 if rl is None else len(rl), threads or nthreads())
    return out, lse


def plan_chunks(B, Hkv, max_len, force_chunks, wave_slots):
    nc, ct = C.c_int(), C.c_int()
    lib().ora_plan_chunks(B, Hkv, max_len, force_chunks, wave_slots, C.byref(nc), C.byref(ct))
    return nc.value, ct.value


def shared_prefix_pages(indptr, indices):
    indptr = np.ascontiguousarray(indptr, dtype=np.int32)
    indices = np.ascontiguousarray(indices, dtype=np.int32)
    return lib().ora_shared_prefix_pages(_p(indptr), _p(indices), len(indptr) - 1)


# ------------------------------------------------------------------ MoE
def prefix_tree_batch(segments, seqs, Hq, Hkv, seed, fill=True):
    """A paged batch whose sequences share runs of physical pages (a prefix tree).

    No reference generator exists for it (the reference lists prefix trees as not done,
    README.md:73); this follows make_shared_prefix_batch (01:446-484) in spirit: segment i
    is segments[i] pages stored once, sequence b = its segment list seqs[b][0] followed by
    seqs[b][1] >= 1 private tokens, physical page ids shuffled, K/V/q U(-1,1) fp16 from a
    numpy generator seeded with `seed`."""
    rng = np.random.default_rng(seed)
    seg_base, n = [], 0
    for pages in segments:
        seg_base.append(n)
        n += pages
    lists, lens, last = [], [], []
    for segs, priv in seqs:
        assert priv >= 1
        pl = [seg_base[i] + j for i in segs for j in range(segments[i])]
        npriv = (priv + PAGE - 1) // PAGE
        pl += list(range(n, n + npriv))
        n += npriv
        lists.append(pl)
        lens.append(PAGE * sum(segments[i] for i in segs) + priv)
        last.append(priv - (npriv - 1) * PAGE)
    phys = rng.permutation(n).astype(np.int32)
    indptr = np.zeros(len(seqs) + 1, np.int32)
    indptr[1:] = np.cumsum([len(pl) for pl in lists])
    indices = np.array([phys[i] for pl in lists for i in pl], np.int32)
    q = (rng.random((len(seqs), Hq, HEAD_DIM), np.float32) * 2 - 1).astype(np.float16)
    k = v = None
    if fill:
        k = (rng.random((n, PAGE, Hkv, HEAD_DIM), np.float32) * 2 - 1).astype(np.float16)
        v = (rng.random((n, PAGE, Hkv, HEAD_DIM), np.float32) * 2 - 1).astype(np.float16)
    bt = Batch(lens, Hq, Hkv, indptr, indices, np.array(last, np.int32), q, k, v)
    bt.num_pages = n
    return bt


def prefix_tree_ref(indptr, indices, min_pages=1):
    """Brute-force prefix tree of a page table (checker for ckl_prefix_tree).

    Each sequence's key is its page list but the last page. A node is a maximal set of >= 2
    sequences whose keys share their first `end` pages; taken by increasing depth, a node is
    kept when end - first >= min_pages, first being the end of its nearest kept ancestor
    (a kept node whose members strictly include its own). Returns ({(members, first, end)},
    start_pages[B] = end of each sequence's deepest kept node, else 0)."""
    ip = np.asarray(indptr)
    B = len(ip) - 1
    keys = [tuple(int(x) for x in indices[ip[b]:max(ip[b], ip[b + 1] - 1)]) for b in range(B)]
    best = {}
    for depth in range(1, max((len(k) for k in keys), default=0) + 1):
        groups = {}
        for b in range(B):
            if len(keys[b]) >= depth:
                groups.setdefault(keys[b][:depth], []).append(b)
        for g in groups.values():
            if len(g) >= 2:
                best[frozenset(g)] = depth
    kept = []
    for members, end in sorted(best.items(), key=lambda kv: kv[1]):
        anc = [e for (m, f, e) in kept if members < m]
        first = max(anc, default=0)
        if end - first >= max(1, min_pages):
            kept.append((members, first, end))
    start = np.zeros(B, np.int32)
    for members, first, end in kept:
        for b in members:
            start[b] = max(start[b], end)
    return set(kept), start


def make_logits(T, E, seed, disable=-1, msvc_pair_order=False):
    """Restates make_logits; msvc_pair_order reproduces the MSVC build that produced the
    reference's published results (see ckl_oracle.cpp)."""
    out = np.empty((T, E), np.float32)
    lib().ora_make_logits(T, E, seed, disable, int(msvc_pair_order), _p(out))
    return out


def normal(shape, seed, mean=0.0, std=1.0, fp16=True):
    n = int(np.prod(shape))
    if fp16:
        a = np.empty(shape, np.float16)
        lib().ora_normal(n, seed, mean, std, _p(a), None)
    else:
        a = np.empty(shape, np.float32)
        lib().ora_normal(n, seed, mean, std, None, _p(a))
    return a


def init_uniform(shape, seed, scale):
    """The reference's init_uniform hash generator (common/moe.cuh:131-138), fp16."""
    a = np.empty(shape, np.float16)
    lib().ora_init_uniform(_p(a), a.size, seed, scale)
    return a


def route(logits, k):
    logits = np.ascontiguousarray(logits, dtype=np.float32)
    T, E = logits.shape
    ids = np.empty((T, k), np.int32)
    wts = np.empty((T, k), np.float64)
    lib().ora_route(_p(logits), T, E, k, _p(ids), _p(wts))
    return ids, wts


def permute(ids, E, bm=128):
    ids = np.ascontiguousarray(ids, dtype=np.int32).reshape(-1)
    A = ids.size
    counts = np.empty(E, np.int32)
    offsets = np.empty(E + 1, np.int32)
    tiles = np.empty(E + 1, np.int32)
    inv = np.empty(A, np.int32)
    lib().ora_permute(_p(ids), A, E, bm, _p(counts), _p(offsets), _p(tiles), _p(inv))
    return counts, offsets, tiles, inv


def quant_sym(W, bits, group=GS):
    """W fp16 [E,d,f] -> (codes uint8 [E,d,f] offset-binary, scales fp16 [E,d/group,f])."""
    W = np.ascontiguousarray(W, dtype=np.float16)
    E, d, f = W.shape
    codes = np.empty((E, d, f), np.uint8)
    scales = np.empty((E, d // group, f), np.float16)
    lib().ora_quant_sym(_p(W), E, d, f, bits, group, _p(codes), _p(scales), nthreads())
    return codes, scales


def quant_asym4(W):
    """W fp16 [E,d,f] -> (codes uint8 q, scales fp16 [E,d/128,f], zeros uint8 [E,d/128,f])."""
    W = np.ascontiguousarray(W, dtype=np.float16)
    E, d, f = W.shape
    codes = np.empty((E, d, f), np.uint8)
    scales = np.empty((E, d // GS, f), np.float16)
    zeros = np.empty((E, d // GS, f), np.uint8)
    lib().ora_quant_asym4(_p(W), E, d, f, _p(codes), _p(scales), _p(zeros), nthreads())
    return codes, scales, zeros


def dequant(codes, scales, zeros, bits, group=GS):
    E, d, f = codes.shape
    out = np.empty((E, d, f), np.float32)
    lib().ora_dequant(_p(np.ascontiguousarray(codes)), _p(np.ascontiguousarray(scales)),
                      _p(None if zeros is None else np.ascontiguousarray(zeros)), E, d, f, bits,
                      group, _p(out))
    return out


def expert_gemm(X, Wdq, offsets):
    X = np.ascontiguousarray(X, dtype=np.float16)
    Wdq = np.ascontiguousarray(Wdq, dtype=np.float32)
    offsets = np.ascontiguousarray(offsets, dtype=np.int32)
    E, d, f = Wdq.shape
    A = int(offsets[E])
    Y = np.zeros((A, f), np.float32)
    lib().ora_expert_gemm(_p(X), _p(Wdq), _p(offsets), E, d, f, _p(Y), nthreads())
    return Y


def moe_layer(X, ids, wts, Wg, Wu, Wd, return_h=False):
    X = np.ascontiguousarray(X, dtype=np.float16)
    T, d = X.shape
    E, _, F = Wg.shape
    k = ids.shape[1]
    out = np.empty((T, d), np.float32)
    h = np.empty((T * k, F), np.float16) if return_h else None
    lib().ora_moe_layer(_p(X), T, d, F, E, k, _p(np.ascontiguousarray(ids, dtype=np.int32)),
                        _p(np.ascontiguousarray(wts, dtype=np.float64)),
                        _p(np.ascontiguousarray(Wg, dtype=np.float32)),
                        _p(np.ascontiguousarray(Wu, dtype=np.float32)),
                        _p(np.ascontiguousarray(Wd, dtype=np.float32)), _p(out), _p(h),
                        nthreads())
    return (out, h) if return_h else out


def combine(Y, inv_perm, wts, T, k):
    Y = np.ascontiguousarray(Y, dtype=np.float32)
    f = Y.shape[1]
    out = np.empty((T, f), np.float32)
    lib().ora_combine(_p(Y), _p(np.ascontiguousarray(inv_perm, dtype=np.int32)),
                      _p(np.ascontiguousarray(wts, dtype=np.float64)), T, k, f, _p(out))
    return out


# ------------------------------------------------------------------ the reference's own code
def ref01():
    """The reference's attention host code (oracle/_ref/libref01.so) or None if not built."""
    global _ref01
    if _ref01 is None:
        path = os.path.join(HERE, "_ref", "libref01.so")
        if not os.path.exists(path):
            return None
        L = C.CDLL(path)
        vp, i, u = C.c_void_p, C.c_int, C.c_uint
        L.ref01_batch_generate.restype = i
        L.ref01_batch_generate.argtypes = [vp, i, i, i, u, i, vp, vp, vp, vp, vp, vp]
        L.ref01_shared_prefix_generate.restype = i
        L.ref01_shared_prefix_generate.argtypes = [i, vp, i, i, i, u, i, vp, vp, vp, vp, vp, vp]
        L.ref01_cpu_reference.restype = None
        L.ref01_cpu_reference.argtypes = [i, i, i, vp, vp, vp, vp, vp, vp, vp, vp]
        L.ref01_shared_prefix_pages.restype = i
        L.ref01_shared_prefix_pages.argtypes = [vp, vp, i]
        L.ref01_sample_make.restype = vp
        L.ref01_sample_make.argtypes = [i, i, i, i, i, u]
        L.ref01_sample_run.restype = C.c_double
        L.ref01_sample_run.argtypes = [vp, C.POINTER(C.c_double)]
        L.ref01_sample_free.restype = None
        L.ref01_sample_free.argtypes = [vp]
        # the reference's GPU path (same-box comparator; needs a GPU)
        L.ref01_decode_plan.restype = vp
        L.ref01_decode_plan.argtypes = [vp, vp, vp, vp, vp, vp, i, i, i, i, i]
        L.ref01_decode_plan_chunks.restype = i
        L.ref01_decode_plan_chunks.argtypes = [vp]
        L.ref01_decode_run.restype = None
        L.ref01_decode_run.argtypes = [vp, vp, vp, vp]
        L.ref01_decode_free.restype = None
        L.ref01_decode_free.argtypes = [vp]
        L.ref01_cascade_plan.restype = vp
        L.ref01_cascade_plan.argtypes = [vp, vp, vp, vp, vp, vp, vp, vp, vp, i, i, i, i]
        L.ref01_cascade_use.restype = i
        L.ref01_cascade_use.argtypes = [vp]
        L.ref01_cascade_run.restype = None
        L.ref01_cascade_run.argtypes = [vp, vp, vp, vp]
        L.ref01_cascade_free.restype = None
        L.ref01_cascade_free.argtypes = [vp]
        _ref01 = L
    return _ref01


def ref03():
    """The reference's MoE code (oracle/_ref/libref03.so) or None if not built."""
    global _ref03
    if _ref03 is None:
        path = os.path.join(HERE, "_ref", "libref03.so")
        if not os.path.exists(path):
            return None
        L = C.CDLL(path)
        vp, i, u, sz = C.c_void_p, C.c_int, C.c_uint, C.c_size_t
        L.ref03_make_logits.restype = None
        L.ref03_make_logits.argtypes = [i, i, u, i, vp]
        L.ref03_host_weight_all.restype = None
        L.ref03_host_weight_all.argtypes = [i, vp, sz, vp, sz, i, i, i, vp]
        L.ref03_pack_weights_device.restype = i
        L.ref03_pack_weights_device.argtypes = [i, vp, vp, vp, i, i, i]
        L.ref03_router_topk_device.restype = i
        L.ref03_router_topk_device.argtypes = [vp, vp, vp, i, i, i]
        L.ref03_quant_make.restype = vp
        L.ref03_quant_make.argtypes = [i, vp, i, i, i]
        L.ref03_quant_run.restype = None
        L.ref03_quant_run.argtypes = [vp, vp, vp, vp, i, i, i, i, i, vp]
        L.ref03_quant_free.restype = None
        L.ref03_quant_free.argtypes = [vp]
        _ref03 = L
    return _ref03


def ref_batch(lens, Hq, Hkv, seed, fill=True):
    """Batch generated by the reference's own Batch constructor."""
    L = ref01()
    lens = np.ascontiguousarray(lens, dtype=np.int32)
    B = len(lens)
    npages = int(np.sum((lens + PAGE - 1) // PAGE))
    indptr = np.zeros(B + 1, np.int32)
    last = np.zeros(B, np.int32)
    indices = np.zeros(npages, np.int32)
    q = np.zeros((B, Hq, HEAD_DIM), np.float16)
    k = v = None
    if fill:
        k = np.empty((npages, PAGE, Hkv, HEAD_DIM), np.float16)
        v = np.empty_like(k)
    L.ref01_batch_generate(_p(lens), B, Hq, Hkv, seed, int(fill), _p(indptr), _p(indices),
                           _p(last), _p(q), _p(k), _p(v))
    return Batch(lens, Hq, Hkv, indptr, indices, last, q, k, v)


def ref_shared_prefix_batch(Lp, suffix, Hq, Hkv, seed, fill=True):
    L = ref01()
    suffix = np.ascontiguousarray(suffix, dtype=np.int32)
    B = len(suffix)
    lens = Lp + suffix
    total = lib().ora_shared_prefix_num_pages(Lp, _p(suffix), B)
    npl = int(np.sum((lens + PAGE - 1) // PAGE))
    indptr = np.zeros(B + 1, np.int32)
    last = np.zeros(B, np.int32)
    indices = np.zeros(npl, np.int32)
    q = np.zeros((B, Hq, HEAD_DIM), np.float16)
    k = v = None
    if fill:
        k = np.empty((total, PAGE, Hkv, HEAD_DIM), np.float16)
        v = np.empty_like(k)
    L.ref01_shared_prefix_generate(Lp, _p(suffix), B, Hq, Hkv, seed, int(fill), _p(indptr),
                                   _p(indices), _p(last), _p(q), _p(k), _p(v))
    bt = Batch(lens, Hq, Hkv, indptr, indices, last, q, k, v)
    bt.num_pages = total
    return bt


def ref_cpu_reference(bt: Batch):
    L = ref01()
    out = np.empty((bt.B, bt.Hq, HEAD_DIM), np.float32)
    lse = np.empty((bt.B, bt.Hq), np.float32)
    L.ref01_cpu_reference(bt.B, bt.Hq, bt.Hkv, _p(bt.lens), _p(bt.indptr), _p(bt.indices),
                          _p(bt.q), _p(bt.k), _p(bt.v), _p(out), _p(lse))
    return out, lse


def ref_make_logits(T, E, seed, disable=-1):
    out = np.empty((T, E), np.float32)
    ref03().ref03_make_logits(T, E, seed, disable, _p(out))
    return out


class RefCpuSample:
    """Timing sample of the reference's cpu_reference (oracle/_ref): nthreads threads, each
    with its own Batch(b_per_thread x L) from the reference's generator."""

    def __init__(self, nthreads, b_per_thread, L, Hq=32, Hkv=8, seed=11):
        self.h = ref01().ref01_sample_make(nthreads, b_per_thread, L, Hq, Hkv, seed)
        self.nthreads, self.b_per_thread, self.L = nthreads, b_per_thread, L

    def run(self):
        """Returns (seconds, kv_bytes) of one concurrent pass."""
        kvb = C.c_double()
        s = ref01().ref01_sample_run(self.h, C.byref(kvb))
        return s, kvb.value

    def close(self):
        if self.h:
            ref01().ref01_sample_free(self.h)
            self.h = None


def port_attention_seconds(bt, threads):
    """Times the oracle port (ora_attention_ref) on `threads` threads; returns seconds."""
    import time
    t0 = time.perf_counter()
    attention_ref(bt, threads=threads)
    return time.perf_counter() - t0


# ------------------------------------------------------------------ expert parallelism
# Restatement, for the tests, of where the expert-parallel layer (ckl_moe_ep_layer) puts
# rows. The reference is single-GPU; its layer (MoeDecode, 03_moe_wq_decode.cu:350-391) is
# the oracle the partitioned result is compared with.
def ep_dispatch(ids, inv_perm, offsets, E_loc):
    """Owner rank and slab position of every assignment i = t*k + j of one rank's tokens:
    owner = ids[i] // E_loc, pos = inv_perm[i] - offsets[owner * E_loc] (expert order
    within the rank's slab on the owner)."""
    ids = np.asarray(ids, np.int64).reshape(-1)
    owner = ids // E_loc
    pos = np.asarray(inv_perm, np.int64) - np.asarray(offsets, np.int64)[owner * E_loc]
    return owner, pos


def ep_receive(counts_from, cap):
    """counts_from [world][E_loc] (rows source s sent for each local expert) -> the expert
    offsets [E_loc + 1] over all received rows and the gather map row_src[a] = s*cap + slab
    position, ordered by expert, then source, then slab position."""
    counts_from = np.asarray(counts_from, np.int64)
    world, E_loc = counts_from.shape
    soff = np.zeros_like(counts_from)
    soff[:, 1:] = np.cumsum(counts_from, axis=1)[:, :-1]
    offsets = np.zeros(E_loc + 1, np.int64)
    offsets[1:] = np.cumsum(counts_from.sum(axis=0))
    row_src = []
    for e in range(E_loc):
        for s in range(world):
            row_src.extend(range(s * cap + soff[s, e], s * cap + soff[s, e] + counts_from[s, e]))
    return offsets.astype(np.int32), np.asarray(row_src, np.int32)
