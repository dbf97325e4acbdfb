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


def test_px_open_multi_argument_checks(xlib):
    from xtagger_b200 import lib as L
    p = L.Px()
    devs = (C.c_int * 9)(*range(9))
    assert xlib.px_open_multi(C.byref(p), b"x.bin", devs, 9, 64, None, 0) == -1      # more than 8 devices
    assert xlib.px_open_multi(C.byref(p), b"x.bin", devs, 0, 4, None, 0) == -1       # no device
    assert xlib.px_open_multi(C.byref(p), b"x.bin", devs, 4, 2, None, 0) == -1       # batch < devices
    assert xlib.px_open_multi(C.byref(p), b"x.bin", devs, 2, 129, None, 0) == -1     # more than 64 per device
    assert xlib.px_open_multi(C.byref(p), b"x.bin", None, 2, 4, None, 0) == -1       # no device list
    assert p.impl is None


def test_prof_names(xlib):
    names = [xlib.eva_prof_name(i) for i in range(9)]
    assert all(names) and xlib.eva_prof_name(9) is None
    assert names[2] == b"qkv" and names[3] == b"attention"


def test_scale_factor_image_layout(xlib):
    """xtb_sf_image (host code): records [k block][n block, count padded to even][512 bytes], every byte of a record
    the UE8M0 exponent of that block's power-of-two scale; the padding block's record is 2^0, so a 256-column tile of
    the CTA-pair kernel always has a record for its second weight block. Scales that are not positive normal powers
    of two are refused and leave the image untouched."""
    import numpy as np
    n, k = 5472, 1024                                     # 43 weight blocks (padded to 44) x 8 K blocks
    nbn, nbk, nbp = 43, 8, 44
    assert xlib.xtb_sf_image_bytes(n, k) == nbk * nbp * 512
    rng = np.random.default_rng(5)
    e = rng.integers(100, 140, size=(nbn, nbk))
    ws = np.ldexp(1.0, e - 127).astype(np.float32)
    img = np.zeros(nbk * nbp * 512, np.uint8)
    assert xlib.xtb_sf_image(ws.ctypes.data, n, k, img.ctypes.data) == 0
    rec = img.reshape(nbk, nbp, 512)
    assert np.all(rec == rec[:, :, :1])                   # uniform records
    np.testing.assert_array_equal(rec[:, :nbn, 0], e.T)
    assert np.all(rec[:, nbn, 0] == 127)
    for bad in (3.0, 0.0, -0.5, np.inf, 2.0 ** -130):     # not a power of two / zero / negative / inf / subnormal
        w2 = ws.copy()
        w2[7, 3] = bad
        img2 = np.full_like(img, 0xAB)
        assert xlib.xtb_sf_image(w2.ctypes.data, n, k, img2.ctypes.data) == -1
        assert np.all(img2 == 0xAB)


def test_block_scaled_gemm_argument_checks(xlib):
    """xtb_gemm_mx_f32 refuses bad arguments on the host, before any device work: no scale image, K not a multiple
    of 16, an unknown kernel form (pair outside 0..2), no rows, an output stride below N."""
    import numpy as np
    buf = np.zeros(1 << 16, np.uint8)
    p = buf.ctypes.data
    assert xlib.xtb_gemm_mx_f32(p, 16, 64, p, 256, None, 1, 1.0, p, 256, None) == -1
    assert xlib.xtb_gemm_mx_f32(p, 16, 60, p, 256, p, 1, 1.0, p, 256, None) == -1
    assert xlib.xtb_gemm_mx_f32(p, 16, 64, p, 256, p, 3, 1.0, p, 256, None) == -1
    assert xlib.xtb_gemm_mx_f32(p, 16, 64, p, 256, p, -1, 1.0, p, 256, None) == -1
    assert xlib.xtb_gemm_mx_f32(p, 0, 64, p, 256, p, 1, 1.0, p, 256, None) == -1
    assert xlib.xtb_gemm_mx_f32(p, 16, 64, p, 256, p, 1, 1.0, p, 128, None) == -1
