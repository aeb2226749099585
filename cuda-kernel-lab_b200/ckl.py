"""Python host mirror of the reference's decode-layer interface, over the C ABI.

Every call goes through libckl.so (include/ckl.h); there is no CPU or PyTorch fallback:
if the library is missing or a call fails, a CklError is raised. PyTorch is used only as
plumbing -- device tensors, streams -- and tensors cross the boundary as raw pointers.

This module is the mirror the tests and bench.py drive the library through; it needs torch
to allocate buffers. libckl.so itself does not depend on torch: its C ABI takes plain
device pointers, sizes and a cudaStream_t, and a C/C++ host calls it directly.

Names follow the reference (01_decode_attention.cu, 03_moe_wq_decode.cu, common/moe.cuh):
plan_chunks, decode_attention, merge_states, shared_prefix_pages, plan_cascade,
cascade_decode, ...
"""
from __future__ import annotations

import ctypes as C
import math
import os

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libckl.so")
HEAD_DIM = 128
PAGE = 16

CKL_OK = 0
CKL_WORKSPACE_TOO_SMALL = 6
CKL_DECODE_CACHE_READY = 1     # ckl_decode_attention_ex flag (see include/ckl.h)
STATUS = {0: "CKL_OK", 1: "CKL_INVALID_ARG", 2: "CKL_UNSUPPORTED_SHAPE", 3: "CKL_CUDA_ERROR",
          4: "CKL_NCCL_ERROR", 5: "CKL_TIMEOUT", 6: "CKL_WORKSPACE_TOO_SMALL"}


class CklError(RuntimeError):
    def __init__(self, status, where, msg):
        self.status = status
        super().__init__(f"{where}: {STATUS.get(status, status)}: {msg}")


class DecodeParams(C.Structure):
    """ckl_decode_params (mirrors DecodeParams, 01_decode_attention.cu:51-65)."""
    _fields_ = [("q", C.c_void_p), ("k_cache", C.c_void_p), ("v_cache", C.c_void_p),
                ("kv_indptr", C.c_void_p), ("kv_indices", C.c_void_p),
                ("kv_last_page_len", C.c_void_p), ("part_o", C.c_void_p),
                ("part_lse", C.c_void_p), ("B", C.c_int), ("Hq", C.c_int), ("Hkv", C.c_int),
                ("num_chunks", C.c_int), ("chunk_tokens", C.c_int), ("kv_start", C.c_int),
                ("chunk_base", C.c_int), ("part_stride", C.c_int), ("sm_scale", C.c_float),
                ("num_pages", C.c_int)]


class CascadePlan(C.Structure):
    """ckl_cascade_plan_t (mirrors CascadePlan, 01_decode_attention.cu:656-662)."""
    _fields_ = [("use", C.c_int), ("prefix_pages", C.c_int), ("prefix_len", C.c_int),
                ("prefix_chunks", C.c_int), ("prefix_chunk_tokens", C.c_int),
                ("qtiles", C.c_int), ("prefix_page_ids", C.c_void_p),
                ("suffix", DecodeParams)]


class CascadeTreePlan(C.Structure):
    """ckl_cascade_tree_plan_t (the prefix-tree cascade; no reference counterpart)."""
    _fields_ = [("use", C.c_int), ("nodes", C.c_int), ("items", C.c_int),
                ("chunk_pages", C.c_int), ("max_path_slots", C.c_int), ("reserved", C.c_int),
                ("table_bytes", C.c_size_t), ("suffix", DecodeParams)]


class MoeWeights(C.Structure):
    """ckl_moe_weights (the packed buffers of QuantWeights, 03_moe_wq_decode.cu:281-333)."""
    _fields_ = [("bits", C.c_int), ("E", C.c_int), ("K", C.c_int), ("N", C.c_int),
                ("group", C.c_int), ("asym", C.c_int), ("packed", C.c_void_p),
                ("scales", C.c_void_p), ("zeros", C.c_void_p)]


EP_MAX_RANKS = 8
IPC_HANDLE_BYTES = 64


class MoeEpComm(C.Structure):
    """ckl_moe_ep_comm: rank, world, token capacity, top-k, experts, d_model and every
    rank's communication window as mapped in this process."""
    _fields_ = [("rank", C.c_int), ("world", C.c_int), ("T_cap", C.c_int), ("k", C.c_int),
                ("E", C.c_int), ("d", C.c_int), ("windows", C.c_void_p * EP_MAX_RANKS)]


class PeerGroup(C.Structure):
    """ckl_peer_group: rank, world and every rank's flag window as mapped here."""
    _fields_ = [("rank", C.c_int), ("world", C.c_int), ("windows", C.c_void_p * EP_MAX_RANKS)]


PEER_WINDOW_BYTES = 256

_lib = None

# name -> (restype, argtypes); every function declared in include/ckl.h
_SIGS = {
    "ckl_last_error_string": (C.c_char_p, []),
    "ckl_version": (C.c_char_p, []),
    "ckl_check_device_error": (C.c_int, []),
    "ckl_set_spin_timeout_ns": (None, [C.c_uint64]),
    "ckl_decode_plan": (C.c_int, [C.c_int, C.c_int, C.c_int, C.c_int, C.c_int,
                                  C.POINTER(C.c_int), C.POINTER(C.c_int)]),
    "ckl_decode_workspace_size": (C.c_size_t, [C.POINTER(DecodeParams)]),
    "ckl_decode_partial": (C.c_int, [C.POINTER(DecodeParams), C.c_void_p]),
    "ckl_merge_states": (C.c_int, [C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p, C.c_int,
                                   C.c_int, C.c_void_p]),
    "ckl_decode_attention": (C.c_int, [C.POINTER(DecodeParams), C.c_void_p, C.c_void_p,
                                       C.c_void_p, C.c_size_t, C.c_void_p]),
    "ckl_decode_attention_ex": (C.c_int, [C.POINTER(DecodeParams), C.c_void_p, C.c_void_p,
                                          C.c_void_p, C.c_size_t, C.c_uint, C.c_void_p]),
    "ckl_decode_balanced_workspace_size": (C.c_size_t, [C.POINTER(DecodeParams)]),
    "ckl_decode_attention_balanced": (C.c_int, [C.POINTER(DecodeParams), C.c_void_p, C.c_void_p,
                                                C.c_void_p, C.c_size_t, C.c_void_p]),
    "ckl_decode_attention_noalloc": (C.c_int, [C.POINTER(DecodeParams), C.c_void_p,
                                               C.c_void_p, C.c_void_p]),
    "ckl_validate_page_table": (C.c_int, [C.c_void_p, C.c_void_p, C.c_void_p, C.c_int,
                                          C.c_int]),
    "ckl_stream_read": (C.c_int, [C.c_void_p, C.c_size_t, C.c_void_p, C.c_void_p]),
    "ckl_shared_prefix_pages": (C.c_int, [C.c_void_p, C.c_void_p, C.c_int]),
    "ckl_cascade_plan": (C.c_int, [C.POINTER(DecodeParams), C.c_void_p, C.c_void_p, C.c_void_p,
                                   C.c_int, C.POINTER(CascadePlan)]),
    "ckl_cascade_workspace_size": (C.c_size_t, [C.POINTER(CascadePlan)]),
    "ckl_cascade_prefix": (C.c_int, [C.POINTER(CascadePlan), C.c_void_p, C.c_void_p,
                                     C.c_void_p]),
    "ckl_prefix_tree": (C.c_int, [C.c_void_p, C.c_void_p, C.c_int, C.c_int, C.c_void_p,
                                  C.c_void_p, C.c_void_p]),
    "ckl_cascade_tree_plan": (C.c_int, [C.POINTER(DecodeParams), C.c_void_p, C.c_void_p,
                                        C.c_void_p, C.c_int, C.POINTER(CascadeTreePlan),
                                        C.c_void_p, C.c_size_t]),
    "ckl_cascade_tree_workspace_size": (C.c_size_t, [C.POINTER(CascadeTreePlan)]),
    "ckl_cascade_tree_prefix": (C.c_int, [C.POINTER(CascadeTreePlan), C.c_void_p, C.c_void_p,
                                          C.c_void_p, C.c_void_p]),
    "ckl_cascade_tree_decode": (C.c_int, [C.POINTER(CascadeTreePlan), C.c_void_p, C.c_void_p,
                                          C.c_void_p, C.c_void_p, C.c_size_t, C.c_void_p]),
    "ckl_cascade_decode": (C.c_int, [C.POINTER(CascadePlan), C.c_void_p, C.c_void_p,
                                     C.c_void_p, C.c_size_t, C.c_void_p]),
    "ckl_moe_packed_bytes": (C.c_size_t, [C.c_int, C.c_int, C.c_int, C.c_int, C.c_int]),
    "ckl_moe_scale_count": (C.c_size_t, [C.c_int, C.c_int, C.c_int, C.c_int]),
    "ckl_moe_zero_words": (C.c_size_t, [C.c_int, C.c_int, C.c_int, C.c_int]),
    "ckl_moe_pack_weights": (C.c_int, [C.c_void_p, C.POINTER(MoeWeights), C.c_void_p]),
    "ckl_moe_dequant_weights": (C.c_int, [C.POINTER(MoeWeights), C.c_void_p, C.c_void_p]),
    "ckl_moe_import_reference_packed": (C.c_int, [C.c_void_p, C.c_void_p, C.POINTER(MoeWeights),
                                                  C.c_void_p]),
    "ckl_moe_gemm_workspace_size": (C.c_size_t, [C.POINTER(MoeWeights), C.c_int, C.c_int,
                                                 C.c_int]),
    "ckl_moe_expert_gemm": (C.c_int, [C.c_void_p, C.c_void_p, C.c_void_p, C.c_int,
                                      C.POINTER(MoeWeights), C.c_int, C.c_void_p, C.c_size_t,
                                      C.c_void_p]),
    "ckl_moe_expert_gemm_ex": (C.c_int, [C.c_void_p, C.c_void_p, C.c_void_p, C.c_int,
                                         C.POINTER(MoeWeights), C.POINTER(MoeWeights),
                                         C.c_void_p, C.c_int, C.c_int, C.c_void_p, C.c_size_t,
                                         C.c_void_p]),
    "ckl_moe_route_permute": (C.c_int, [C.c_void_p, C.c_void_p, C.c_int, C.c_int, C.c_int,
                                        C.c_int, C.c_void_p, C.c_void_p, C.c_void_p,
                                        C.c_void_p, C.c_void_p, C.c_void_p, C.c_int,
                                        C.c_void_p, C.c_void_p]),
    "ckl_moe_combine": (C.c_int, [C.c_void_p, C.c_int, C.c_void_p, C.c_void_p, C.c_void_p,
                                  C.c_int, C.c_int, C.c_int, C.c_void_p]),
    "ckl_moe_grouped_gemm_workspace_size": (C.c_size_t, []),
    "ckl_moe_grouped_gemm": (C.c_int, [C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p, C.c_int,
                                       C.c_int, C.c_int, C.c_int, C.c_void_p, C.c_size_t,
                                       C.c_void_p]),
    "ckl_moe_weights_save": (C.c_int, [C.c_char_p, C.POINTER(MoeWeights), C.c_void_p]),
    "ckl_moe_weights_file_info": (C.c_int, [C.c_char_p, C.POINTER(MoeWeights)]),
    "ckl_moe_weights_load": (C.c_int, [C.c_char_p, C.POINTER(MoeWeights), C.c_void_p]),
    "ckl_moe_layer_workspace_size": (C.c_size_t, [C.c_int, C.c_int, C.POINTER(MoeWeights),
                                                  C.POINTER(MoeWeights)]),
    "ckl_moe_layer": (C.c_int, [C.c_void_p, C.c_void_p, C.c_int, C.c_int,
                                C.POINTER(MoeWeights), C.POINTER(MoeWeights),
                                C.POINTER(MoeWeights), C.c_void_p, C.c_void_p, C.c_void_p,
                                C.c_void_p, C.c_size_t, C.c_void_p]),
    "ckl_decode_attention_gather": (C.c_int, [C.POINTER(DecodeParams), C.c_void_p, C.c_void_p,
                                              C.c_int, C.c_int, C.c_void_p, C.c_size_t,
                                              C.c_void_p]),
    "ckl_gather_signal": (C.c_int, [C.POINTER(PeerGroup), C.c_int, C.c_void_p]),
    "ckl_gather_wait": (C.c_int, [C.POINTER(PeerGroup), C.c_void_p]),
    "ckl_peer_barrier": (C.c_int, [C.POINTER(PeerGroup), C.c_void_p]),
    "ckl_moe_ep_window_bytes": (C.c_size_t, [C.c_int, C.c_int, C.c_int, C.c_int, C.c_int]),
    "ckl_ep_window_alloc": (C.c_int, [C.c_size_t, C.POINTER(C.c_void_p), C.c_void_p]),
    "ckl_ep_window_open": (C.c_int, [C.c_void_p, C.POINTER(C.c_void_p)]),
    "ckl_ep_window_close": (C.c_int, [C.c_void_p]),
    "ckl_ep_window_free": (C.c_int, [C.c_void_p]),
    "ckl_moe_ep_workspace_size": (C.c_size_t, [C.POINTER(MoeEpComm), C.POINTER(MoeWeights),
                                               C.POINTER(MoeWeights)]),
    "ckl_moe_ep_layer": (C.c_int, [C.POINTER(MoeEpComm), C.c_void_p, C.c_void_p, C.c_int,
                                   C.POINTER(MoeWeights), C.POINTER(MoeWeights),
                                   C.POINTER(MoeWeights), C.c_void_p, C.c_void_p, C.c_void_p,
                                   C.c_void_p, C.c_size_t, C.c_void_p]),
    "ckl_moe_ep_layer_ex": (C.c_int, [C.POINTER(MoeEpComm), C.c_int, C.c_void_p, C.c_void_p,
                                      C.c_int, C.POINTER(MoeWeights), C.POINTER(MoeWeights),
                                      C.POINTER(MoeWeights), C.c_void_p, C.c_void_p, C.c_void_p,
                                      C.c_void_p, C.c_size_t, C.c_void_p]),
}


def lib():
    """Loads libckl.so (raises if it was not built: there is no fallback)."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise CklError(3, "load", f"{LIB_PATH} not built (run make -C cuda-kernel-lab_b200)")
        L = C.CDLL(LIB_PATH)
        for name, (res, args) in _SIGS.items():
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _lib = L
    return _lib


def check(status, where):
    if status != CKL_OK:
        msg = lib().ckl_last_error_string().decode(errors="replace")
        raise CklError(status, where, msg)


def version():
    return lib().ckl_version().decode()


def check_device_error():
    check(lib().ckl_check_device_error(), "ckl_check_device_error")


def set_spin_timeout_ns(ns):
    lib().ckl_set_spin_timeout_ns(int(ns))


# ------------------------------------------------------------------ torch plumbing
def _torch():
    import torch
    return torch


def _ptr(t):
    return None if t is None else C.c_void_p(t.data_ptr())


def _stream(stream):
    torch = _torch()
    s = stream if stream is not None else torch.cuda.current_stream()
    return C.c_void_p(s.cuda_stream)


def _need(t, dtype, name):
    torch = _torch()
    if t is None or not isinstance(t, torch.Tensor) or not t.is_cuda:
        raise CklError(1, name, "expected a CUDA tensor")
    if t.dtype != dtype or not t.is_contiguous():
        raise CklError(1, name, f"expected contiguous {dtype}, got {t.dtype}")
    return t


class _CudaArray:
    def __init__(self, ptr, shape, typestr):
        self.__cuda_array_interface__ = {"data": (int(ptr), False), "shape": tuple(shape),
                                         "typestr": typestr, "strides": None, "version": 2}


def device_view(ptr, shape, dtype):
    """A torch tensor viewing raw device memory (a library-allocated window, own or
    peer-mapped) without a copy; the memory must outlive the view."""
    torch = _torch()
    ts = {torch.float16: "<f2", torch.float32: "<f4", torch.int32: "<i4", torch.uint8: "|u1"}[dtype]
    return torch.as_tensor(_CudaArray(ptr, shape, ts), device="cuda")


# ------------------------------------------------------------------ decode attention
def plan_chunks(G, B, Hkv, max_len, force_chunks=0):
    """plan_chunks (01_decode_attention.cu:292-312) -> (num_chunks, chunk_tokens)."""
    nc, ct = C.c_int(), C.c_int()
    check(lib().ckl_decode_plan(G, B, Hkv, max_len, force_chunks, C.byref(nc), C.byref(ct)),
          "ckl_decode_plan")
    return nc.value, ct.value


def make_params(q, k_cache, v_cache, kv_indptr, kv_indices, kv_last_page_len, *, num_chunks,
                chunk_tokens, kv_start=0, chunk_base=0, part_stride=None, sm_scale=None,
                part_o=None, part_lse=None):
    torch = _torch()
    _need(q, torch.float16, "q")
    _need(k_cache, torch.float16, "k_cache")
    _need(v_cache, torch.float16, "v_cache")
    for t, n in ((kv_indptr, "kv_indptr"), (kv_indices, "kv_indices"),
                 (kv_last_page_len, "kv_last_page_len")):
        _need(t, torch.int32, n)
    B, Hq, D = q.shape
    num_pages, page, Hkv, D2 = k_cache.shape
    if D != HEAD_DIM or D2 != HEAD_DIM or page != PAGE or v_cache.shape != k_cache.shape:
        raise CklError(2, "make_params", f"q {tuple(q.shape)} / cache {tuple(k_cache.shape)}")
    p = DecodeParams()
    p.q, p.k_cache, p.v_cache = q.data_ptr(), k_cache.data_ptr(), v_cache.data_ptr()
    p.kv_indptr, p.kv_indices = kv_indptr.data_ptr(), kv_indices.data_ptr()
    p.kv_last_page_len = kv_last_page_len.data_ptr()
    p.part_o = None if part_o is None else part_o.data_ptr()
    p.part_lse = None if part_lse is None else part_lse.data_ptr()
    p.B, p.Hq, p.Hkv = B, Hq, Hkv
    p.num_chunks, p.chunk_tokens = num_chunks, chunk_tokens
    p.kv_start, p.chunk_base = kv_start, chunk_base
    p.part_stride = num_chunks + chunk_base if part_stride is None else part_stride
    p.sm_scale = 1.0 / math.sqrt(HEAD_DIM) if sm_scale is None else sm_scale
    p.num_pages = num_pages
    return p


def workspace_size(p: DecodeParams):
    return lib().ckl_decode_workspace_size(C.byref(p))


def decode_partial(p: DecodeParams, stream=None):
    check(lib().ckl_decode_partial(C.byref(p), _stream(stream)), "ckl_decode_partial")


def merge_states(part_o, part_lse, out, lse, stream=None):
    rows, slots = part_lse.shape[0], part_lse.shape[1]
    check(lib().ckl_merge_states(_ptr(part_o), _ptr(part_lse), _ptr(out), _ptr(lse), rows,
                                 slots, _stream(stream)), "ckl_merge_states")


def decode_attention(q, k_cache, v_cache, kv_indptr, kv_indices, kv_last_page_len, *,
                     max_len=None, force_chunks=0, num_chunks=None, chunk_tokens=None,
                     out=None, lse=None, workspace=None, sm_scale=None, stream=None,
                     cache_ready=False):
    """decode_attention (01_decode_attention.cu:316-331): returns (out fp16 [B,Hq,128],
    lse fp32 [B,Hq]). Plans the split like the reference (plan_chunks) unless num_chunks /
    chunk_tokens are given; max_len defaults to the longest sequence (read from the page
    table on the host, which synchronises). cache_ready: ckl_decode_attention_ex with
    CKL_DECODE_CACHE_READY (the page table and all but each sequence's last page were written
    before the stream's previous kernel began)."""
    torch = _torch()
    B, Hq, _ = q.shape
    Hkv = k_cache.shape[2]
    if num_chunks is None:
        if max_len is None:
            ip = kv_indptr.cpu()
            lp = kv_last_page_len.cpu()
            np_ = ip[1:] - ip[:-1]
            lens = torch.where(np_ > 0, (np_ - 1) * PAGE + lp, torch.zeros_like(np_))
            max_len = int(lens.max()) if B else 0
        num_chunks, chunk_tokens = plan_chunks(Hq // Hkv, B, Hkv, max_len, force_chunks)
    p = make_params(q, k_cache, v_cache, kv_indptr, kv_indices, kv_last_page_len,
                    num_chunks=num_chunks, chunk_tokens=chunk_tokens, sm_scale=sm_scale)
    if out is None:
        out = torch.empty_like(q)
    if lse is None:
        lse = torch.empty((B, Hq), dtype=torch.float32, device=q.device)
    need = workspace_size(p)
    if need and (workspace is None or workspace.numel() * workspace.element_size() < need):
        workspace = torch.empty(need, dtype=torch.uint8, device=q.device)
    ws_bytes = 0 if workspace is None else workspace.numel() * workspace.element_size()
    if cache_ready:
        check(lib().ckl_decode_attention_ex(C.byref(p), _ptr(out), _ptr(lse), _ptr(workspace),
                                            ws_bytes, CKL_DECODE_CACHE_READY, _stream(stream)),
              "ckl_decode_attention_ex")
    else:
        check(lib().ckl_decode_attention(C.byref(p), _ptr(out), _ptr(lse), _ptr(workspace),
                                         ws_bytes, _stream(stream)), "ckl_decode_attention")
    return out, lse


def decode_attention_balanced(q, k_cache, v_cache, kv_indptr, kv_indices, kv_last_page_len, *,
                              out=None, lse=None, workspace=None, sm_scale=None, stream=None):
    """The balanced split (ckl_decode_attention_balanced): returns (out, lse)."""
    torch = _torch()
    B, Hq, _ = q.shape
    p = make_params(q, k_cache, v_cache, kv_indptr, kv_indices, kv_last_page_len, num_chunks=1,
                    chunk_tokens=16, sm_scale=sm_scale)
    if out is None:
        out = torch.empty_like(q)
    if lse is None:
        lse = torch.empty((B, Hq), dtype=torch.float32, device=q.device)
    need = lib().ckl_decode_balanced_workspace_size(C.byref(p))
    if workspace is None or workspace.numel() * workspace.element_size() < need:
        workspace = torch.empty(max(need, 256), dtype=torch.uint8, device=q.device)
    check(lib().ckl_decode_attention_balanced(C.byref(p), _ptr(out), _ptr(lse), _ptr(workspace),
                                              workspace.numel() * workspace.element_size(),
                                              _stream(stream)), "ckl_decode_attention_balanced")
    return out, lse


NOALLOC_SCRATCH_BYTES = 16 << 20   # CKL_NOALLOC_SCRATCH_BYTES


def decode_attention_noalloc(p: DecodeParams, out, lse, stream=None):
    """ckl_decode_attention_noalloc: decode with the library's built-in scratch instead of a
    caller workspace, for hosts that cannot allocate device memory (see include/ckl.h)."""
    check(lib().ckl_decode_attention_noalloc(C.byref(p), _ptr(out), _ptr(lse), _stream(stream)),
          "ckl_decode_attention_noalloc")


def validate_page_table(indptr, indices, last, num_pages):
    """Host validation of a page table given as numpy int32 arrays."""
    import numpy as np
    ip = np.ascontiguousarray(indptr, dtype=np.int32)
    ix = np.ascontiguousarray(indices, dtype=np.int32)
    ls = np.ascontiguousarray(last, dtype=np.int32)
    check(lib().ckl_validate_page_table(ip.ctypes.data_as(C.c_void_p),
                                        ix.ctypes.data_as(C.c_void_p),
                                        ls.ctypes.data_as(C.c_void_p), len(ip) - 1, num_pages),
          "ckl_validate_page_table")


def stream_read(buf, sink, stream=None):
    check(lib().ckl_stream_read(_ptr(buf), buf.numel() * buf.element_size(), _ptr(sink),
                                _stream(stream)), "ckl_stream_read")


# ------------------------------------------------------------------ cascade
def _np_i32(a):
    import numpy as np
    return np.ascontiguousarray(a, dtype=np.int32)


def shared_prefix_pages(indptr, indices):
    """shared_prefix_pages (01_decode_attention.cu:636-646) on host int32 arrays."""
    ip, ix = _np_i32(indptr), _np_i32(indices)
    return lib().ckl_shared_prefix_pages(ip.ctypes.data_as(C.c_void_p),
                                         ix.ctypes.data_as(C.c_void_p), len(ip) - 1)


def plan_cascade(base: DecodeParams, h_indptr, h_indices, h_lens, min_prefix=256):
    """plan_cascade (01_decode_attention.cu:666-701) from host copies of the page table."""
    ip, ix, ln = _np_i32(h_indptr), _np_i32(h_indices), _np_i32(h_lens)
    cp = CascadePlan()
    check(lib().ckl_cascade_plan(C.byref(base), ip.ctypes.data_as(C.c_void_p),
                                 ix.ctypes.data_as(C.c_void_p), ln.ctypes.data_as(C.c_void_p),
                                 min_prefix, C.byref(cp)), "ckl_cascade_plan")
    cp._keep = (base,)
    return cp


def cascade_workspace_size(cp: CascadePlan):
    return lib().ckl_cascade_workspace_size(C.byref(cp))


def cascade_prefix(cp: CascadePlan, part_o, part_lse, stream=None):
    check(lib().ckl_cascade_prefix(C.byref(cp), _ptr(part_o), _ptr(part_lse), _stream(stream)),
          "ckl_cascade_prefix")


def cascade_decode(cp: CascadePlan, out=None, lse=None, workspace=None, stream=None):
    """cascade_decode (01_decode_attention.cu:703-712) -> (out, lse)."""
    torch = _torch()
    sp = cp.suffix
    dev = torch.device("cuda", torch.cuda.current_device())
    if out is None:
        out = torch.empty((sp.B, sp.Hq, HEAD_DIM), dtype=torch.float16, device=dev)
    if lse is None:
        lse = torch.empty((sp.B, sp.Hq), dtype=torch.float32, device=dev)
    need = cascade_workspace_size(cp)
    if need and (workspace is None or workspace.numel() * workspace.element_size() < need):
        workspace = torch.empty(need, dtype=torch.uint8, device=dev)
    ws_bytes = 0 if workspace is None else workspace.numel() * workspace.element_size()
    check(lib().ckl_cascade_decode(C.byref(cp), _ptr(out), _ptr(lse), _ptr(workspace), ws_bytes,
                                   _stream(stream)), "ckl_cascade_decode")
    return out, lse


def prefix_tree(indptr, indices, min_pages=1):
    """ckl_prefix_tree on host int32 arrays -> (perm [B], nodes [n, 5] = {first page, end
    page, m0, m1, parent}, start_pages [B])."""
    import numpy as np
    ip, ix = _np_i32(indptr), _np_i32(indices)
    B = len(ip) - 1
    perm = np.zeros(max(B, 1), np.int32)
    start = np.zeros(max(B, 1), np.int32)
    nodes = np.zeros((max(B - 1, 1), 5), np.int32)
    vp = lambda a: a.ctypes.data_as(C.c_void_p)
    n = lib().ckl_prefix_tree(vp(ip), vp(ix), B, min_pages, vp(perm), vp(nodes), vp(start))
    if n < 0:
        raise CklError(1, "ckl_prefix_tree", "bad page table")
    return perm[:B], nodes[:n].copy(), start[:B]


def plan_cascade_tree(base: DecodeParams, h_indptr, h_indices, h_lens, min_prefix=256):
    """Plans the prefix-tree cascade from host copies of the page table and uploads its
    tables (plan.tables, a device uint8 tensor)."""
    import numpy as np
    torch = _torch()
    ip, ix, ln = _np_i32(h_indptr), _np_i32(h_indices), _np_i32(h_lens)
    vp = lambda a: a.ctypes.data_as(C.c_void_p)
    tp = CascadeTreePlan()
    st = lib().ckl_cascade_tree_plan(C.byref(base), vp(ip), vp(ix), vp(ln), min_prefix,
                                     C.byref(tp), None, 0)
    tp.tables = None
    if st == CKL_WORKSPACE_TOO_SMALL and tp.use:
        host = np.zeros(tp.table_bytes, np.uint8)
        check(lib().ckl_cascade_tree_plan(C.byref(base), vp(ip), vp(ix), vp(ln), min_prefix,
                                          C.byref(tp), vp(host), host.nbytes),
              "ckl_cascade_tree_plan")
        dev = torch.device("cuda", torch.cuda.current_device())
        tp.tables = torch.from_numpy(host).to(dev)
    else:
        check(st, "ckl_cascade_tree_plan")
    tp._keep = (base,)
    return tp


def cascade_tree_workspace_size(tp: CascadeTreePlan):
    return lib().ckl_cascade_tree_workspace_size(C.byref(tp))


def cascade_tree_prefix(tp: CascadeTreePlan, part_o, part_lse, stream=None):
    check(lib().ckl_cascade_tree_prefix(C.byref(tp), _ptr(tp.tables), _ptr(part_o),
                                        _ptr(part_lse), _stream(stream)), "ckl_cascade_tree_prefix")


def cascade_tree_decode(tp: CascadeTreePlan, out=None, lse=None, workspace=None, stream=None):
    """Prefix-tree cascade decode -> (out fp16 [B,Hq,128], lse fp32 [B,Hq])."""
    torch = _torch()
    sp = tp.suffix
    dev = torch.device("cuda", torch.cuda.current_device())
    if out is None:
        out = torch.empty((sp.B, sp.Hq, HEAD_DIM), dtype=torch.float16, device=dev)
    if lse is None:
        lse = torch.empty((sp.B, sp.Hq), dtype=torch.float32, device=dev)
    need = cascade_tree_workspace_size(tp)
    if need and (workspace is None or workspace.numel() * workspace.element_size() < need):
        workspace = torch.empty(need, dtype=torch.uint8, device=dev)
    ws_bytes = 0 if workspace is None else workspace.numel() * workspace.element_size()
    check(lib().ckl_cascade_tree_decode(C.byref(tp), _ptr(tp.tables), _ptr(out), _ptr(lse),
                                        _ptr(workspace), ws_bytes, _stream(stream)),
          "ckl_cascade_tree_decode")
    return out, lse


# ------------------------------------------------------------------ MoE
class QuantWeights:
    """QuantWeights (03_moe_wq_decode.cu:281-333): packs fp16 W [E][K][N] (a CUDA tensor)
    into the library's format. bits 4 (group 128; asym=True adds zero points), 8 (group 128
    or group=K per output channel) or 16."""

    def __init__(self, bits, W, group=128, asym=False, stream=None):
        torch = _torch()
        _need(W, torch.float16, "W")
        E, K, N = W.shape
        dev = W.device
        if bits == 16:
            group = K
        self.bits, self.E, self.K, self.N, self.group, self.asym = bits, E, K, N, group, asym
        L = lib()
        self.packed = torch.empty(L.ckl_moe_packed_bytes(bits, E, K, N, group), dtype=torch.uint8,
                                  device=dev)
        ns = L.ckl_moe_scale_count(E, K, N, group) if bits != 16 else 1
        self.scales = torch.empty(max(ns, 1), dtype=torch.float16, device=dev)
        nz = L.ckl_moe_zero_words(E, K, N, group) if asym else 1
        self.zeros = torch.zeros(max(nz, 1), dtype=torch.int32, device=dev)
        self.w = MoeWeights(bits, E, K, N, group, int(asym), self.packed.data_ptr(),
                            self.scales.data_ptr() if bits != 16 else None,
                            self.zeros.data_ptr() if asym else None)
        check(L.ckl_moe_pack_weights(_ptr(W), C.byref(self.w), _stream(stream)),
              "ckl_moe_pack_weights")

    @classmethod
    def from_reference_packed(cls, bits, P, Sc, E, K, N, stream=None):
        """Weights the reference's QuantWeights packed (P uint32 words in widx order and
        Sc fp16 [E][K/128][N], 03_moe_wq_decode.cu:43-87), re-laid on the device
        (ckl_moe_import_reference_packed). P and Sc are CUDA tensors."""
        torch = _torch()
        group = K if bits == 16 else 128
        self = cls.__new__(cls)
        self.bits, self.E, self.K, self.N, self.group, self.asym = bits, E, K, N, group, False
        L = lib()
        dev = P.device
        self.packed = torch.empty(L.ckl_moe_packed_bytes(bits, E, K, N, group), dtype=torch.uint8,
                                  device=dev)
        ns = L.ckl_moe_scale_count(E, K, N, group) if bits != 16 else 1
        self.scales = torch.empty(max(ns, 1), dtype=torch.float16, device=dev)
        self.zeros = torch.zeros(1, dtype=torch.int32, device=dev)
        self.w = MoeWeights(bits, E, K, N, group, 0, self.packed.data_ptr(),
                            self.scales.data_ptr() if bits != 16 else None, None)
        check(L.ckl_moe_import_reference_packed(_ptr(P), _ptr(Sc) if bits != 16 else None,
                                                C.byref(self.w), _stream(stream)),
              "ckl_moe_import_reference_packed")
        return self

    def dequant(self, stream=None):
        torch = _torch()
        out = torch.empty((self.E, self.K, self.N), dtype=torch.float32, device=self.packed.device)
        check(lib().ckl_moe_dequant_weights(C.byref(self.w), _ptr(out), _stream(stream)),
              "ckl_moe_dequant_weights")
        return out

    def save(self, path, stream=None):
        """Writes the packed weights to `path` (ckl_moe_weights_save)."""
        check(lib().ckl_moe_weights_save(os.fsencode(path), C.byref(self.w), _stream(stream)),
              "ckl_moe_weights_save")

    @classmethod
    def load(cls, path, device="cuda", stream=None):
        """Packed weights read back from `path` (ckl_moe_weights_file_info + _load)."""
        torch = _torch()
        info = MoeWeights()
        check(lib().ckl_moe_weights_file_info(os.fsencode(path), C.byref(info)),
              "ckl_moe_weights_file_info")
        self = cls.__new__(cls)
        self.bits, self.E, self.K, self.N = info.bits, info.E, info.K, info.N
        self.group, self.asym = info.group, bool(info.asym)
        L = lib()
        self.packed = torch.empty(L.ckl_moe_packed_bytes(info.bits, info.E, info.K, info.N, info.group),
                                  dtype=torch.uint8, device=device)
        ns = L.ckl_moe_scale_count(info.E, info.K, info.N, info.group) if info.bits != 16 else 1
        self.scales = torch.empty(max(ns, 1), dtype=torch.float16, device=device)
        nz = L.ckl_moe_zero_words(info.E, info.K, info.N, info.group) if info.asym else 1
        self.zeros = torch.zeros(max(nz, 1), dtype=torch.int32, device=device)
        self.w = MoeWeights(info.bits, info.E, info.K, info.N, info.group, info.asym,
                            self.packed.data_ptr(),
                            self.scales.data_ptr() if info.bits != 16 else None,
                            self.zeros.data_ptr() if info.asym else None)
        check(L.ckl_moe_weights_load(os.fsencode(path), C.byref(self.w), _stream(stream)),
              "ckl_moe_weights_load")
        return self

    def expert(self, e):
        """Expert e alone (E=1), a view sharing this object's device buffers: the packed
        codes, the scales and the zero points are all laid out expert-major."""
        L = lib()
        v = QuantWeights.__new__(QuantWeights)
        v.bits, v.E, v.K, v.N, v.group, v.asym = self.bits, 1, self.K, self.N, self.group, self.asym
        pb = L.ckl_moe_packed_bytes(self.bits, 1, self.K, self.N, self.group)
        v.packed = self.packed[e * pb:(e + 1) * pb]
        v.scales, v.zeros = self.scales, self.zeros
        if self.bits != 16:
            ns = L.ckl_moe_scale_count(1, self.K, self.N, self.group)
            v.scales = self.scales[e * ns:(e + 1) * ns]
        if self.asym:
            nz = L.ckl_moe_zero_words(1, self.K, self.N, self.group)
            v.zeros = self.zeros[e * nz:(e + 1) * nz]
        v.w = MoeWeights(v.bits, 1, v.K, v.N, v.group, int(v.asym), v.packed.data_ptr(),
                         v.scales.data_ptr() if v.bits != 16 else None,
                         v.zeros.data_ptr() if v.asym else None)
        return v

    def bytes_per_expert(self):
        """Algorithmic bytes of one expert: codes + scales (+ zero points), the bytes a
        decode step must stream for it (03_moe_wq_decode.cu:527,551 credit the same)."""
        b = self.K * self.N * self.bits // 8
        if self.bits != 16:
            b += (self.K // self.group) * self.N * 2
        if self.asym:
            b += (self.K // self.group) * self.N // 2
        return b

    def workspace_size(self, A, swiglu=False, force_ksplit=0):
        return lib().ckl_moe_gemm_workspace_size(C.byref(self.w), A, int(swiglu), force_ksplit)

    def run(self, Xp, Yp, offsets, A, force_ksplit=0, workspace=None, stream=None):
        """QuantWeights::run: Yp[r] = Xp[r] . W_e for the rows of each expert."""
        torch = _torch()
        need = self.workspace_size(A, False, force_ksplit)
        if need and (workspace is None or workspace.numel() * workspace.element_size() < need):
            workspace = torch.empty(need, dtype=torch.uint8, device=Xp.device)
        wsb = 0 if workspace is None else workspace.numel() * workspace.element_size()
        check(lib().ckl_moe_expert_gemm(_ptr(Xp), _ptr(Yp), _ptr(offsets), A, C.byref(self.w),
                                        force_ksplit, _ptr(workspace), wsb, _stream(stream)),
              "ckl_moe_expert_gemm")


def expert_gemm_ex(X, row_src, offsets, A, gate, up=None, y_f32=False, force_ksplit=0,
                   stream=None):
    torch = _torch()
    N = gate.N
    Y = torch.empty((A, N), dtype=torch.float32 if y_f32 else torch.float16, device=X.device)
    need = gate.workspace_size(A, up is not None, force_ksplit)
    ws = torch.empty(max(need, 1), dtype=torch.uint8, device=X.device)
    check(lib().ckl_moe_expert_gemm_ex(_ptr(X), _ptr(row_src), _ptr(offsets), A, C.byref(gate.w),
                                       None if up is None else C.byref(up.w), _ptr(Y), int(y_f32),
                                       force_ksplit, _ptr(ws), need, _stream(stream)),
          "ckl_moe_expert_gemm_ex")
    return Y


_GROUPED_WS = {}


def grouped_workspace(dev):
    """A zeroed ckl_moe_grouped_gemm workspace for device dev (every completed launch leaves
    its flag words zero, so it is reused; one launch at a time)."""
    torch = _torch()
    key = torch.device(dev).index if torch.device(dev).index is not None else torch.cuda.current_device()
    ws = _GROUPED_WS.get(key)
    if ws is None:
        n = lib().ckl_moe_grouped_gemm_workspace_size()
        if n == C.c_size_t(-1).value:
            raise CklError(3, "ckl_moe_grouped_gemm_workspace_size", "no CUDA device")
        ws = _GROUPED_WS[key] = torch.zeros(n, dtype=torch.uint8, device=dev)
    return ws


def grouped_gemm(Xp, W, offsets, out=None, workspace=None, stream=None):
    """moe_grouped_gemm (02_moe_grouped_gemm.cu:86-186): Yp[r] = Xp[r] . W[e] over the
    expert-sorted rows, fp16 [A][f] (tcgen05). W fp16 [E][d][f]. workspace: a zeroed
    ckl_moe_grouped_gemm_workspace_size() buffer (default: one cached per device)."""
    torch = _torch()
    _need(Xp, torch.float16, "Xp")
    _need(W, torch.float16, "W")
    A, d = Xp.shape
    E, _, f = W.shape
    if out is None:
        out = torch.empty((A, f), dtype=torch.float16, device=Xp.device)
    if workspace is None:
        workspace = grouped_workspace(Xp.device)
    check(lib().ckl_moe_grouped_gemm(_ptr(Xp), _ptr(W), _ptr(out), _ptr(offsets), A, E, d, f,
                                     _ptr(workspace), workspace.numel() * workspace.element_size(),
                                     _stream(stream)), "ckl_moe_grouped_gemm")
    return out


def route_and_permute(logits, X, k, bm=0, permute=True, stream=None):
    """MoeDecode::route_and_permute (03_moe_wq_decode.cu:382-389) -> dict of device tensors
    ids, wts, counts, offsets, inv_perm, Xp (None unless permute), tiles (None unless bm)."""
    torch = _torch()
    T, E = logits.shape
    dev = logits.device
    d = X.shape[1] if X is not None else 0
    i32 = dict(dtype=torch.int32, device=dev)
    r = dict(ids=torch.empty((T, k), **i32), wts=torch.empty((T, k), dtype=torch.float32, device=dev),
             counts=torch.empty(E, **i32), offsets=torch.empty(E + 1, **i32),
             inv_perm=torch.empty(T * k, **i32), Xp=None, tiles=None)
    if permute:
        r["Xp"] = torch.empty((T * k, d), dtype=torch.float16, device=dev)
    if bm:
        r["tiles"] = torch.empty(E + 1, **i32)
    check(lib().ckl_moe_route_permute(_ptr(logits), _ptr(X), T, E, k, d, _ptr(r["ids"]),
                                      _ptr(r["wts"]), _ptr(r["counts"]), _ptr(r["offsets"]),
                                      _ptr(r["inv_perm"]), _ptr(r["Xp"]), bm, _ptr(r["tiles"]),
                                      _stream(stream)), "ckl_moe_route_permute")
    return r


def combine(Yp, inv_perm, wts, T, k, stream=None):
    """moe_combine (common/moe.cuh:97-119) -> out fp16 [T][f]."""
    torch = _torch()
    f = Yp.shape[1]
    out = torch.empty((T, f), dtype=torch.float16, device=Yp.device)
    check(lib().ckl_moe_combine(_ptr(Yp), int(Yp.dtype == torch.float32), _ptr(inv_perm),
                                _ptr(wts), _ptr(out), T, k, f, _stream(stream)), "ckl_moe_combine")
    return out


class MoeLayer:
    """The SwiGLU MoE decode layer over packed gate/up [E][d][F] and down [E][F][d]."""

    def __init__(self, gate: QuantWeights, up: QuantWeights, down: QuantWeights):
        self.gate, self.up, self.down = gate, up, down

    def workspace_size(self, T, k):
        return lib().ckl_moe_layer_workspace_size(T, k, C.byref(self.gate.w), C.byref(self.down.w))

    def forward(self, logits, X, k, out=None, ids=None, wts=None, workspace=None, stream=None):
        torch = _torch()
        T = X.shape[0]
        dev = X.device
        if out is None:
            out = torch.empty((T, self.down.N), dtype=torch.float16, device=dev)
        need = self.workspace_size(T, k)
        if workspace is None or workspace.numel() * workspace.element_size() < need:
            workspace = torch.empty(need, dtype=torch.uint8, device=dev)
        check(lib().ckl_moe_layer(_ptr(logits), _ptr(X), T, k, C.byref(self.gate.w),
                                  C.byref(self.up.w), C.byref(self.down.w), _ptr(out), _ptr(ids),
                                  _ptr(wts), _ptr(workspace),
                                  workspace.numel() * workspace.element_size(), _stream(stream)),
              "ckl_moe_layer")
        return out


# ------------------------------------------------------------------ expert parallelism
def ep_window_bytes(world, T_cap, k, E, d):
    return lib().ckl_moe_ep_window_bytes(world, T_cap, k, E, d)


class _LibWindows:
    """CUDA IPC through the library: allocate + zero an own window, map / unmap peers."""

    @staticmethod
    def alloc(nbytes):
        ptr, h = C.c_void_p(), (C.c_char * IPC_HANDLE_BYTES)()
        check(lib().ckl_ep_window_alloc(nbytes, C.byref(ptr), h), "ckl_ep_window_alloc")
        return ptr.value, bytes(h)

    @staticmethod
    def open(handle):
        ptr = C.c_void_p()
        check(lib().ckl_ep_window_open(C.c_char_p(handle), C.byref(ptr)), "ckl_ep_window_open")
        return ptr.value

    @staticmethod
    def close(ptr):
        check(lib().ckl_ep_window_close(C.c_void_p(ptr)), "ckl_ep_window_close")

    @staticmethod
    def free(ptr):
        check(lib().ckl_ep_window_free(C.c_void_p(ptr)), "ckl_ep_window_free")


def torch_exchange(group=None):
    """exchange(handle) over a torch.distributed process group: every rank's bytes, in rank
    order (all_gather_object; any backend)."""
    import torch.distributed as dist

    def exchange(blob):
        out = [None] * dist.get_world_size(group)
        dist.all_gather_object(out, blob, group=group)
        return out
    return exchange


class IpcWindows:
    """One device window per rank, allocated and zeroed here, every peer's mapped from its
    IPC handle (windows in rank order in self.ptrs). `exchange(bytes) -> [bytes per rank]`
    moves the handles (e.g. torch_exchange()); it is also the barrier that makes every
    window zero before any rank uses one."""

    def __init__(self, rank, world, nbytes, exchange, ipc=_LibWindows):
        if not (1 <= world <= EP_MAX_RANKS and 0 <= rank < world):
            raise CklError(1, "IpcWindows", f"rank {rank} of world {world} (<= {EP_MAX_RANKS})")
        self.rank, self.world, self.nbytes = rank, world, nbytes
        self._ipc, self._exchange = ipc, exchange
        self.own, handle = ipc.alloc(nbytes)
        handles = exchange(handle)
        if len(handles) != world:
            raise CklError(1, "IpcWindows", f"exchange returned {len(handles)} handles, not {world}")
        self.ptrs, self._opened = [], []
        for r, h in enumerate(handles):
            if r == rank:
                self.ptrs.append(self.own)
            else:
                p = ipc.open(h)
                self.ptrs.append(p)
                self._opened.append(p)

    def _array(self):
        return (C.c_void_p * EP_MAX_RANKS)(*(self.ptrs + [None] * (EP_MAX_RANKS - self.world)))

    def close(self):
        """Collective: unmaps the peers' windows, waits until every rank has done so (an
        empty exchange), then frees the own window. No layer call may be in flight."""
        for p in self._opened:
            self._ipc.close(p)
        self._opened = []
        self._exchange(b"")
        if self.own is not None:
            self._ipc.free(self.own)
            self.own = None


class EpWindows(IpcWindows):
    """The communication windows of an expert-parallel group (ckl_moe_ep_comm). All ranks
    construct theirs collectively before any rank's first layer call."""

    def __init__(self, rank, world, T_cap, k, E, d, exchange, ipc=_LibWindows):
        if E % world:
            raise CklError(2, "EpWindows", f"E={E} does not divide by world={world}")
        nbytes = ep_window_bytes(world, T_cap, k, E, d) if ipc is _LibWindows else 0
        super().__init__(rank, world, nbytes, exchange, ipc)
        self.T_cap, self.k, self.E, self.d = T_cap, k, E, d
        self.E_loc = E // world
        self.comm = MoeEpComm(rank, world, T_cap, k, E, d, self._array())

    def experts(self):
        """Global expert ids owned by this rank."""
        return range(self.rank * self.E_loc, (self.rank + 1) * self.E_loc)


class GatherGroup(IpcWindows):
    """Flag windows for gathers into one rank's buffers (ckl_peer_group): signal() on every
    rank after its writes, wait() on the root before it reads."""

    def __init__(self, rank, world, exchange, ipc=_LibWindows):
        super().__init__(rank, world, PEER_WINDOW_BYTES, exchange, ipc)
        self.group = PeerGroup(rank, world, self._array())

    def signal(self, root=0, stream=None):
        check(lib().ckl_gather_signal(C.byref(self.group), root, _stream(stream)),
              "ckl_gather_signal")

    def wait(self, stream=None):
        check(lib().ckl_gather_wait(C.byref(self.group), _stream(stream)), "ckl_gather_wait")

    def barrier(self, stream=None):
        check(lib().ckl_peer_barrier(C.byref(self.group), _stream(stream)), "ckl_peer_barrier")


def decode_attention_gather(p: DecodeParams, out_full_ptr, lse_full_ptr, Hq_total, head_offset,
                            workspace=None, stream=None):
    """ckl_decode_attention_gather: this rank's head shard written into rows
    [head_offset, head_offset + p.Hq) of a [B, Hq_total] output given by raw device
    pointers (own or peer-mapped)."""
    wsb = 0 if workspace is None else workspace.numel() * workspace.element_size()
    check(lib().ckl_decode_attention_gather(C.byref(p), C.c_void_p(out_full_ptr),
                                            C.c_void_p(lse_full_ptr), Hq_total, head_offset,
                                            _ptr(workspace), wsb, _stream(stream)),
          "ckl_decode_attention_gather")


class MoeEpLayer:
    """The expert-parallel SwiGLU MoE layer (ckl_moe_ep_layer): this rank's experts
    gate/up [E/world][d][F], down [E/world][F][d]; forward() takes this rank's tokens."""

    def __init__(self, windows: EpWindows, gate: QuantWeights, up: QuantWeights,
                 down: QuantWeights):
        self.win, self.gate, self.up, self.down = windows, gate, up, down

    def workspace_size(self):
        return lib().ckl_moe_ep_workspace_size(C.byref(self.win.comm), C.byref(self.gate.w),
                                               C.byref(self.down.w))

    def forward(self, logits, X, out=None, ids=None, wts=None, workspace=None, stream=None,
                T_max=0):
        """T_max: an upper bound of the tokens on every rank this call (0: T_cap), which
        sizes the expert GEMMs' grids (ckl_moe_ep_layer_ex)."""
        torch = _torch()
        T = X.shape[0]
        dev = X.device
        if out is None:
            out = torch.empty((T, self.win.d), dtype=torch.float16, device=dev)
        need = self.workspace_size()
        if workspace is None or workspace.numel() * workspace.element_size() < need:
            workspace = torch.empty(need, dtype=torch.uint8, device=dev)
        check(lib().ckl_moe_ep_layer_ex(C.byref(self.win.comm), T_max, _ptr(logits), _ptr(X), T,
                                        C.byref(self.gate.w), C.byref(self.up.w),
                                        C.byref(self.down.w), _ptr(out), _ptr(ids), _ptr(wts),
                                        _ptr(workspace), workspace.numel() * workspace.element_size(),
                                        _stream(stream)), "ckl_moe_ep_layer_ex")
        return out
