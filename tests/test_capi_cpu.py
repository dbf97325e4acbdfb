"""The C-ABI library without a GPU: it loads, exports every function include/xtagger_b200.h declares, and the
engine's host-side checks fail cleanly (-1 / NULL with an "eva:" line) before any device work."""
import ctypes as C
import struct

import pytest


def test_every_declared_symbol_is_exported(xlib):
    from xtagger_b200 import lib as L
    names = L.header_symbols()
    assert len(names) >= 30
    missing = [n for n in names if not hasattr(xlib, n)]
    assert not missing, missing


def test_open_rejects_missing_and_bad_files(xlib, tmp_path):
    from xtagger_b200 import lib as L
    e = L.Eva()
    assert xlib.eva_open(C.byref(e), str(tmp_path / "nope.bin").encode(), 0, None, 0, 0) == -1
    bad = tmp_path / "bad.bin"
    bad.write_bytes(struct.pack("<4sIII", b"EVA1", 3, 10, 0) + b"\0" * 300)
    assert xlib.eva_open(C.byref(e), str(bad).encode(), 0, None, 0, 0) == -1
    v9 = tmp_path / "v9.bin"
    v9.write_bytes(struct.pack("<4sIII", b"EVA2", 9, 10, 0) + b"\0" * 300)
    assert xlib.eva_open(C.byref(e), str(v9).encode(), 0, None, 0, 0) == -1
    nan = tmp_path / "nan.bin"
    nan.write_bytes(struct.pack("<4sIIIII", b"EVA2", 4, 10, 0, 1, 0) + b"\0" * 232 + struct.pack("<12f", *([float("nan")] * 12)))
    assert xlib.eva_open(C.byref(e), str(nan).encode(), 0, None, 0, 0) == -1
    # a failed open leaves a handle that the other calls treat as closed
    xlib.eva_close(C.byref(e))
    assert xlib.eva_wait(C.byref(e), 0) is None or not xlib.eva_wait(C.byref(e), 0)
    assert xlib.eva_query(C.byref(e), 0) == 1
    assert xlib.eva_ready(C.byref(e)) == -1


def test_open_ex_argument_checks(xlib, tmp_path):
    from xtagger_b200 import lib as L
    e = L.Eva()
    devs = (C.c_int * 9)(*range(9))
    assert xlib.eva_open_ex(C.byref(e), b"x.bin", devs, 9, 64, None, 0, 0) == -1     # more than EVA_MAXDEV
    assert xlib.eva_open_ex(C.byref(e), b"x.bin", devs, 0, 64, None, 0, 0) == -1     # no device
    assert xlib.eva_open_ex(C.byref(e), b"x.bin", devs, 4, 2, None, 0, 0) == -1      # batch < devices


def test_prof_names(xlib):
    names = [xlib.eva_prof_name(i) for i in range(9)]
    assert all(names) and xlib.eva_prof_name(9) is None
    assert names[2] == b"qkv" and names[3] == b"attention"
