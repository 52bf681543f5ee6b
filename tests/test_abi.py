"""The C-ABI library without a GPU: it loads, exports every entry point that
include/b2engine.h declares, and rejects bad arguments before touching the
device."""
import os
import re

import b2engine as b2

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared_entry_points():
    names = set()
    for fn in os.listdir(os.path.join(ROOT, "include")):
        if fn.endswith(".h"):
            text = open(os.path.join(ROOT, "include", fn)).read()
            text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
            names |= set(re.findall(r"\b(b2_\w+)\s*\(", text))
    return names


def test_library_loads_and_reports_version():
    assert b"sm_100a" in b2.lib().b2_version()


def test_every_declared_symbol_is_exported():
    lib = b2.lib()
    declared = declared_entry_points()
    assert len(declared) > 30
    missing = [n for n in sorted(declared) if not hasattr(lib, n)]
    assert not missing, missing
    # and the Python binding types every one of them
    assert not sorted(declared - set(b2.exported_symbols()))


def test_status_strings():
    assert b2.status_string(0) == "ok"
    assert b2.status_string(-1) == "invalid argument"
    assert b2.status_string(-2).startswith("unsupported")
    assert "illegal memory access" in b2.status_string(700)


def test_invalid_arguments_rejected_without_device():
    L = b2.lib()
    assert L.b2_gemv(None, None, None, 8, 8, None) == -1
    assert L.b2_rmsnorm(None, None, None, 4, 4, 1e-5, None) == -1
    assert L.b2_decode_gqa_split(None, b2.KVView(), b2.KVView(), None, None, 1, 4, 2, 64, 10, None, 0, None) == -1
    assert L.b2_model_create(None, 0, 1, None, None) == -1
    # empty work is a successful no-op
    assert L.b2_gemv(None, None, None, 0, 8, None) == 0
    assert L.b2_embedding_lookup(None, None, None, 0, 8, None) == 0
