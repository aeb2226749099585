"""CPU tests of the C ABI boundary: the library loads, exports every symbol include/ckl.h
declares, and rejects bad arguments with a status (no device needed for these calls)."""
import ctypes as C
import os
import re
import subprocess

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared_symbols():
    names = set()
    for fn in os.listdir(os.path.join(ROOT, "include")):
        if fn.endswith(".h"):
            src = open(os.path.join(ROOT, "include", fn)).read()
            names |= set(re.findall(r"CKL_API\s+[\w\s\*]+?\b(ckl_\w+)\s*\(", src))
    return names


def test_library_exports_every_declared_symbol(ckl):
    names = declared_symbols()
    assert len(names) >= 10
    out = subprocess.run(["nm", "-D", "--defined-only", ckl.LIB_PATH], capture_output=True,
                         text=True, check=True).stdout
    exported = set(re.findall(r"\bT (ckl_\w+)", out))
    missing = names - exported
    assert not missing, missing
    lib = ckl.lib()
    for n in names:
        assert getattr(lib, n) is not None
    # the python mirror binds every declared function too
    assert names <= set(ckl._SIGS), names - set(ckl._SIGS)


def test_decode_attention_ex_rejects_unknown_flags(ckl):
    # checked on the host before anything else (no device needed)
    st = ckl.lib().ckl_decode_attention_ex(None, None, None, None, 0, 0x2, None)
    assert st == 1   # CKL_INVALID_ARG


def test_version_and_error_string(ckl):
    assert "sm_100a" in ckl.version()
    assert isinstance(ckl.lib().ckl_last_error_string(), bytes)


def test_plan_force_chunks_is_host_only(ckl):
    # force_chunks > 0 needs no device (01_decode_attention.cu:295-296, 309-311)
    assert ckl.plan_chunks(4, 2, 8, 1000, force_chunks=7) == (7, 160)
    assert ckl.plan_chunks(4, 2, 8, 1000, force_chunks=1) == (1, 1024)
    with pytest.raises(ckl.CklError) as e:
        ckl.plan_chunks(3, 2, 8, 1000, force_chunks=1)
    assert e.value.status == 2   # unsupported group size


def test_validate_page_table(ckl, oracle):
    bt = oracle.batch([1, 17, 1000], 8, 8, 7, fill=False)
    ckl.validate_page_table(bt.indptr, bt.indices, bt.last, bt.num_pages)
    bad = bt.indices.copy()
    bad[3] = bt.num_pages
    with pytest.raises(ckl.CklError):
        ckl.validate_page_table(bt.indptr, bad, bt.last, bt.num_pages)
    bad_last = bt.last.copy()
    bad_last[0] = 17
    with pytest.raises(ckl.CklError):
        ckl.validate_page_table(bt.indptr, bt.indices, bad_last, bt.num_pages)


def test_invalid_params_rejected_before_any_launch(ckl):
    p = ckl.DecodeParams()
    p.B, p.Hq, p.Hkv = 2, 32, 7        # Hq % Hkv != 0
    st = ckl.lib().ckl_decode_partial(C.byref(p), None)
    assert st == 1
    p.Hkv = 8
    p.num_chunks, p.chunk_tokens, p.part_stride, p.num_pages = 1, 24, 1, 10   # not 16-aligned
    st = ckl.lib().ckl_decode_partial(C.byref(p), None)
    assert st == 1
    assert ckl.lib().ckl_decode_workspace_size(C.byref(p)) == 0
    p.num_chunks, p.part_stride = 4, 4
    # part_o [B*Hq, slots, 128] fp32 + part_lse [B*Hq, slots] fp32, each 256-byte aligned
    assert ckl.lib().ckl_decode_workspace_size(C.byref(p)) == 2 * 32 * 4 * 128 * 4 + 2 * 32 * 4 * 4


def test_no_fallback_when_library_missing(tmp_path, monkeypatch):
    import ckl as m
    monkeypatch.setattr(m, "LIB_PATH", str(tmp_path / "missing.so"))
    monkeypatch.setattr(m, "_lib", None)
    with pytest.raises(m.CklError):
        m.lib()
    # monkeypatch restores the loaded library (and its bound signatures) afterwards


def _weights_header(bits=4, E=2, K=256, N=128, group=128, asym=1, crc=0, magic=b"CKLMOEW1",
                    version=1, sizes=None):
    import struct
    import ckl
    L = ckl.lib()
    p = L.ckl_moe_packed_bytes(bits, E, K, N, group)
    s = L.ckl_moe_scale_count(E, K, N, group) if bits != 16 else 0
    z = L.ckl_moe_zero_words(E, K, N, group) if asym else 0
    if sizes:
        p, s, z = sizes
    return struct.pack("<8sIiiiiiiIQQQ", magic, version, bits, E, K, N, group, asym, crc, p, s, z), p, s, z


def test_packed_weights_file_header(ckl, tmp_path):
    """The on-disk format of packed weights (ckl_moe_weights_file_info): the documented
    64-byte header is read back field for field; wrong magic, version or section sizes
    are refused; a payload that fails its checksum is refused before any device copy."""
    hdr, p, s, z = _weights_header()
    assert len(hdr) == 64
    f = tmp_path / "w.bin"
    f.write_bytes(hdr + bytes(p + 2 * s + 4 * z))
    w = ckl.MoeWeights()
    ckl.check(ckl.lib().ckl_moe_weights_file_info(str(f).encode(), C.byref(w)), "info")
    assert (w.bits, w.E, w.K, w.N, w.group, w.asym) == (4, 2, 256, 128, 128, 1)
    assert w.packed is None and w.scales is None
    for bad in (_weights_header(magic=b"CKLMOEW0")[0], _weights_header(version=2)[0],
                _weights_header(sizes=(p + 16, s, z))[0]):
        g = tmp_path / "bad.bin"
        g.write_bytes(bad + bytes(p + 2 * s + 4 * z))
        assert ckl.lib().ckl_moe_weights_file_info(str(g).encode(), C.byref(w)) != 0
    # checksum of an all-zero payload is not 0: the load stops at the check
    w2 = ckl.MoeWeights(4, 2, 256, 128, 128, 1, 0x1000, 0x2000, 0x3000)
    st = ckl.lib().ckl_moe_weights_load(str(f).encode(), C.byref(w2), None)
    assert st == 1 and b"checksum" in ckl.lib().ckl_last_error_string()
