"""The reference's own kernels (eva_kernels.cu: k_ln, k_qkv, k_oproj, k_fc1 + k_fc2, built by oracle/Makefile `ref`
and driven by oracle/ref_kernels.cu) against the oracle's restatement and this library's kernels, on the same seeded
inputs with per-tensor weight scales (the reference's v3 format): it pins each piece of the oracle to the
reference's code, and checks this library against the reference directly.

Remaining differences are rounding decisions at representable-value boundaries: each implementation sums the FP8
products in its own order, the GPU kernels use tanh.approx where the oracle uses libm, and this library adds the
residual update as x + fp16(delta). E4M3 outputs are compared code for code (identical or one step apart), fp16
outputs within 1e-2 relative."""
import ctypes as C
import os

import numpy as np
import pytest

from tests import _gpu as G

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
REF_SO = os.path.join(ROOT, "oracle", "_ref", "libref_kernels.so")
NIMG = 2
ROWS = NIMG * 1025
D, HIDP, N12, TP = 1024, 2736, 5472, 1152

_u8 = np.ctypeslib.ndpointer(np.uint8, flags="C_CONTIGUOUS")
_u16 = np.ctypeslib.ndpointer(np.uint16, flags="C_CONTIGUOUS")
_f32 = np.ctypeslib.ndpointer(np.float32, flags="C_CONTIGUOUS")
_f64 = np.ctypeslib.ndpointer(np.float64, flags="C_CONTIGUOUS")


@pytest.fixture(scope="module")
def ref():
    if not os.path.exists(REF_SO):
        pytest.skip("oracle/_ref/libref_kernels.so not built (python -c 'import __graft_entry__ as g; g.build()' "
                    "where the reference sources are present)")
    lib = C.CDLL(REF_SO)
    f = C.c_float
    sigs = {
        "ref_ln": [_u16, _f32, _f32, C.c_int, f, _u8],
        "ref_qkv": [_u8, C.c_int, _u8, _f32, f, f, f, f, _u8, _u8, _u8, C.c_int],
        "ref_oproj": [_u8, C.c_int, _u8, f, _u16],
        "ref_mlp": [_u8, C.c_int, _u8, _f32, f, _u8, _f32, _f32, f, _u8, _f64, _f64, _u16],
    }
    for name, args in sigs.items():
        getattr(lib, name).restype = C.c_int
        getattr(lib, name).argtypes = args
    return lib


@pytest.fixture(scope="module")
def O():
    from oracle import oracle
    return oracle


def _act8(rng, rows, k, O, sd=1.0):
    return O.e4m3(rng.standard_normal((rows, k), dtype=np.float32) * sd * (448 / 8))


def _w8_tensor(rng, n, k, O, src=None):
    """E4M3 weights with one fp32 scale per tensor (v3), plus the same scale as a block-scale grid."""
    w = rng.standard_normal((n, k), dtype=np.float32) * 0.02 if src is None else src
    wdq = float(np.abs(w).max()) / 448
    w8 = O.e4m3(w / wdq)
    return w8, np.full(((n + 127) // 128, (k + 127) // 128), wdq, np.float32), wdq


def _report(name, a, b):
    d = np.abs(G.e4m3_ordinal(a) - G.e4m3_ordinal(b))
    print(f"{name}: {(d == 0).mean():.5f} identical, max {d.max()} steps")


def test_layernorm(xlib, ref, cuda, O):
    rng = np.random.default_rng(50)
    x = (rng.standard_normal((ROWS, D), dtype=np.float32) * 3).astype(np.float16).view(np.uint16)
    g = (1 + 0.2 * rng.standard_normal(D)).astype(np.float32)
    b = (0.1 * rng.standard_normal(D)).astype(np.float32)
    qs = 448 / 5.0
    r = np.empty((ROWS, D), np.uint8)
    assert ref.ref_ln(x, g, b, ROWS, qs, r) == 0
    w = np.empty((ROWS, D), np.uint8)
    O.lib().or_ln_e4m3(x, g, b, ROWS, qs, w)
    y = G.dev(np.zeros((ROWS, D), np.uint8))
    assert xlib.xtb_ln_e4m3(G.P(G.dev(x)), G.P(G.dev(g)), G.P(G.dev(b)), G.P(y), ROWS, qs, None) == 0
    _report("ln reference vs oracle", r, w)
    _report("ln kernel vs reference", G.host(y), r)
    G.assert_e4m3_close(r, w, 1, 0.999, "ln reference vs oracle")
    G.assert_e4m3_close(G.host(y), r, 1, 0.999, "ln kernel vs reference")


def test_qkv(xlib, ref, cuda, O):
    from xtagger_b200 import model as M
    rng = np.random.default_rng(51)
    h = _act8(rng, ROWS, D, O)
    w8, ws, wdq = _w8_tensor(rng, 3 * D, D, O)
    adq, cq, ck, cv = 10 / 448, 448 / 2.0, 448 / 4.0, 448 / 3.0
    cs = np.ascontiguousarray(M.rope_table(), np.float32)
    shp = (NIMG, 16, TP, 64)
    rq, rk, rv = (np.zeros(shp, np.uint8) for _ in range(3))
    assert ref.ref_qkv(h, ROWS, w8, cs.ravel(), wdq * adq, cq, ck, cv, rq, rk, rv, TP) == 0
    oq, ok_, ov = (np.zeros(shp, np.uint8) for _ in range(3))
    O.lib().or_qkv_epilogue(O.gemm_e4m3(h, w8, ws, adq), ROWS, cs, cq, ck, cv, oq, ok_, ov)
    import torch
    gq, gk, gv = (G.zeros(shp, torch.uint8) for _ in range(3))
    assert xlib.xtb_qkv(G.P(G.dev(h)), ROWS, G.P(G.dev(w8)), G.P(G.dev(ws)), adq, G.P(gq), G.P(gk), G.P(gv),
                        G.P(G.dev(cs)), cq, ck, cv, None) == 0
    G.check_error_word(xlib)
    for nm, r, o, g_ in (("q", rq, oq, gq), ("k", rk, ok_, gk), ("v", rv, ov, gv)):
        _report(f"{nm} reference vs oracle", r, o)
        _report(f"{nm} kernel vs reference", G.host(g_), r)
        G.assert_e4m3_close(r, o, 1, 0.999, f"{nm} reference vs oracle")
        G.assert_e4m3_close(G.host(g_), r, 1, 0.999, f"{nm} kernel vs reference")


def test_oproj(xlib, ref, cuda, O):
    rng = np.random.default_rng(52)
    a = _act8(rng, ROWS, D, O)
    w8, ws, wdq = _w8_tensor(rng, D, D, O)
    adq = 4 / 448
    x0 = (rng.standard_normal((ROWS, D), dtype=np.float32) * 2).astype(np.float16).view(np.uint16)
    r = x0.copy()
    assert ref.ref_oproj(a, ROWS, w8, wdq * adq, r) == 0
    o = x0.copy()
    O.lib().or_resid_add(o, O.gemm_e4m3(a, w8, ws, adq), ROWS)
    x = G.dev(x0)
    assert xlib.xtb_oproj(G.P(G.dev(a)), ROWS, G.P(G.dev(w8)), G.P(G.dev(ws)), adq, G.P(x), None) == 0
    G.check_error_word(xlib)
    G.assert_f16_close(r, o, 1e-2, "oproj reference vs oracle")
    G.assert_f16_close(G.host(x).view(np.uint16), r, 1e-2, "oproj kernel vs reference")


def test_mlp(xlib, ref, cuda, O):
    import torch
    from xtagger_b200 import model as M
    rng = np.random.default_rng(53)
    h = _act8(rng, ROWS, D, O)
    w12 = np.zeros((N12, D), np.float32)
    w12[:2730] = rng.standard_normal((2730, D), dtype=np.float32) * 0.02
    w12[HIDP:HIDP + 2730] = rng.standard_normal((2730, D), dtype=np.float32) * 0.02
    w12_8, ws12, wdq12 = _w8_tensor(rng, N12, D, O, M.interleave_gx(w12))
    w2 = np.zeros((D, HIDP), np.float32)
    w2[:, :2730] = rng.standard_normal((D, 2730), dtype=np.float32) * 0.02
    w2_8, ws2, wdq2 = _w8_tensor(rng, D, HIDP, O, w2)
    adq12, adq2 = 10 / 448, 3 / 448
    rs = np.full(HIDP, 1 / adq2, np.float32)
    cn = (rng.standard_normal(D) * 0.3).astype(np.float32)
    dn = (rng.standard_normal(D) * 0.1).astype(np.float32)
    x0 = (rng.standard_normal((ROWS, D), dtype=np.float32) * 2).astype(np.float16).view(np.uint16)
    # reference: k_fc1 then k_fc2 (fc2 on the reference's own fc1 outputs)
    rh8 = np.empty((ROWS, HIDP), np.uint8)
    rsum, rsq = np.empty(ROWS), np.empty(ROWS)
    rx = x0.copy()
    assert ref.ref_mlp(h, ROWS, w12_8, rs, wdq12 * adq12, w2_8, cn, dn, wdq2 * adq2, rh8, rsum, rsq, rx) == 0
    # oracle fc1
    oh8 = np.empty((ROWS, HIDP), np.uint8)
    osum, osq = np.empty(ROWS), np.empty(ROWS)
    O.lib().or_fc1_epilogue(O.gemm_e4m3(h, w12_8, ws12, adq12), ROWS, rs, oh8, osum, osq)
    # this library's fc1
    gh8 = G.zeros((ROWS, HIDP), torch.uint8)
    stat = G.zeros((43, ROWS, 2), torch.float32)
    assert xlib.xtb_fc1(G.P(G.dev(h)), ROWS, G.P(G.dev(w12_8)), G.P(G.dev(ws12)), adq12, G.P(gh8), G.P(stat),
                        G.P(G.dev(rs)), None) == 0
    gst = G.host(stat).astype(np.float64).sum(0)
    _report("h8 reference vs oracle", rh8, oh8)
    _report("h8 kernel vs reference", G.host(gh8), rh8)
    G.assert_e4m3_close(rh8, oh8, 1, 0.99, "h8 reference vs oracle")
    G.assert_e4m3_close(G.host(gh8), rh8, 1, 0.99, "h8 kernel vs reference")
    np.testing.assert_allclose(rsum, osum, rtol=1e-3, atol=1e-3 * np.abs(osum).max())
    np.testing.assert_allclose(rsq, osq, rtol=1e-3)
    np.testing.assert_allclose(gst[:, 0], rsum, rtol=1e-3, atol=1e-3 * np.abs(rsum).max())
    np.testing.assert_allclose(gst[:, 1], rsq, rtol=1e-3)
    # fc2 on the same operands (the reference's h8 and row sums): a code that fc1 rounded the other way would
    # otherwise carry one rounding decision through a whole GEMM row
    ox = x0.copy()
    O.lib().or_fc2_epilogue(ox, O.gemm_e4m3(rh8, w2_8, ws2, adq2), ROWS, rsum, rsq, cn, dn)
    st0 = np.zeros((43, ROWS, 2), np.float32)
    st0[0, :, 0], st0[0, :, 1] = rsum, rsq
    gx = G.dev(x0)
    assert xlib.xtb_fc2(G.P(G.dev(rh8)), ROWS, G.P(G.dev(w2_8)), G.P(G.dev(ws2)), adq2, G.P(gx), G.P(G.dev(st0)),
                        G.P(G.dev(cn)), G.P(G.dev(dn)), None) == 0
    G.check_error_word(xlib)
    G.assert_f16_close(rx, ox, 1e-2, "fc2 reference vs oracle")
    G.assert_f16_close(G.host(gx).view(np.uint16), rx, 1e-2, "fc2 kernel vs reference")
