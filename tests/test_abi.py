"""The C-ABI library loads, exports every declared symbol and fails cleanly without a GPU."""
import ctypes
import os
import re

import pytest

import qllama_b200 as qb

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared_symbols():
    text = "".join(open(os.path.join(ROOT, "include", h)).read()
                   for h in ("qllama_attn.h", "qllama_model.h"))
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(ql_[a-z0-9_]+)\s*\(", text)))


def test_library_exports_every_declared_symbol():
    L = qb.load()
    names = declared_symbols()
    assert len(names) >= 15
    assert set(names) == set(qb.EXPORTS)
    for name in names:
        assert hasattr(L, name), name
    assert b"sm_100a" in L.ql_version()


def test_null_arguments_are_rejected_without_a_device():
    L = qb.load()
    assert L.ql_ctx_create(0, None) == qb.ERR_INVALID
    assert b"NULL" in L.ql_last_error()
    assert L.ql_attn_forward(None, None, None) == qb.ERR_INVALID
    assert L.ql_kv_create(None, None, None) == qb.ERR_INVALID
    assert L.ql_ctx_destroy(None) == qb.OK


@pytest.mark.skipif(__import__("torch").cuda.is_available(), reason="host has a GPU")
def test_context_reports_missing_device():
    L = qb.load()
    h = ctypes.c_void_p()
    rc = L.ql_ctx_create(0, ctypes.byref(h))
    assert rc == qb.ERR_NO_DEVICE
    assert b"no CUDA device" in L.ql_last_error()
    with pytest.raises(qb.QllamaError) as e:
        qb.Context(0)
    assert e.value.code == qb.ERR_NO_DEVICE


def test_comm_entry_points_validate_before_any_device_work():
    L = qb.load()
    cid = qb.CommId()
    out = ctypes.c_void_p()
    assert L.ql_comm_create(None, 2, 0, ctypes.byref(cid), 1 << 20, qb.COMM_P2P,
                            ctypes.byref(out)) == qb.ERR_INVALID
    assert b"NULL" in L.ql_last_error()
    assert L.ql_comm_unique_id(None) == qb.ERR_INVALID
    assert L.ql_comm_destroy(None) == qb.ERR_INVALID
    assert L.ql_comm_buffer(None, None, None) == qb.ERR_INVALID
    assert L.ql_attn_forward_sharded(None, None, None, None) == qb.ERR_INVALID


def test_comm_unique_id_keeps_all_bytes():
    """The id is opaque binary (NUL bytes included) and must cross the ABI whole."""
    a, b = qb.comm_unique_id(), qb.comm_unique_id()
    assert len(a) == len(b) == qb.COMM_ID_BYTES and a != b
    cid = qb.CommId()
    ctypes.memmove(ctypes.addressof(cid), a, qb.COMM_ID_BYTES)
    assert ctypes.string_at(ctypes.addressof(cid), qb.COMM_ID_BYTES) == a
