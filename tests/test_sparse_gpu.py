"""The 2:4-sparse projections (tcgen05.mma.sp, xtb_*_sp) against the dense kernels (xtb_*) and the CPU oracle on
the same pruned weights. The reference runs pruned weights (prune24.py's output) through its dense kernels, so the
dense product on pruned weights is the ground truth; the sparse MMA multiplies the same nonzero products and only
the order of the fp32 sums inside a 128-k block differs, so outputs agree code for code except at rounding
boundaries (E4M3: identical or one step apart; fp16: within 1e-3 relative of the dense kernel, 1e-2 of the
oracle, as the dense tests)."""
import ctypes as C

import numpy as np
import pytest

from tests import _gpu as G

pytestmark = pytest.mark.gpu

NIMG = 2
ROWS = NIMG * 1025
D, HIDP, N12, TP = 1024, 2736, 5472, 1152


@pytest.fixture(scope="module")
def O():
    from oracle import oracle
    return oracle


def _act8(rng, rows, k, O, sd=1.0):
    return O.e4m3(rng.standard_normal((rows, k), dtype=np.float32) * sd * (448 / 8))


def _pruned(rng, n, k, src=None):
    from xtagger_b200 import model as M
    w = rng.standard_normal((n, k), dtype=np.float32) * 0.02 if src is None else src
    q, s = M.quant_blocks(w)
    return M.prune24_codes(q), s


def _sparse(xlib, w):
    """Compressed weight on the device: (values, metadata)."""
    n, k = w.shape
    npad, kp = -(-n // 128) * 128, -(-k // 128) * 128
    vals = np.empty(npad * kp // 2, np.uint8)
    meta = np.empty(npad * kp // 8, np.uint8)
    assert xlib.xtb_sparse24_compress(C.c_void_p(w.ctypes.data), n, k, C.c_void_p(vals.ctypes.data),
                                      C.c_void_p(meta.ctypes.data)) == 0
    return G.dev(vals), G.dev(meta)


@pytest.mark.parametrize("m", [1025, 300])
def test_gemm_sp_f32(xlib, cuda, O, m):
    import torch
    rng = np.random.default_rng(70 + m)
    af = rng.standard_normal((m, D), dtype=np.float32)
    ascale = float(np.abs(af).max()) / 448
    a8 = O.e4m3(af / ascale)
    w, ws = _pruned(rng, 2730, D)
    want = O.gemm_e4m3(a8, w, ws, ascale)
    vals, meta = _sparse(xlib, w)
    da, dws = G.dev(a8), G.dev(ws)
    sp = G.zeros((m, 2730), torch.float32)
    dn = G.zeros((m, 2730), torch.float32)
    assert xlib.xtb_gemm_sp_e4m3_f32(G.P(da), m, D, G.P(vals), G.P(meta), 2730, G.P(dws), ascale, G.P(sp), None) == 0
    assert xlib.xtb_gemm_e4m3_f32(G.P(da), m, D, G.P(G.dev(w)), 2730, G.P(dws), ascale, G.P(dn), None) == 0
    G.check_error_word(xlib)
    sp, dn = G.host(sp), G.host(dn)
    scale = np.abs(want).max()
    assert np.abs(sp - want).max() <= 1e-5 * scale, f"sparse vs oracle {np.abs(sp - want).max() / scale:.2e}"
    assert np.abs(sp - dn).max() <= 1e-5 * scale, f"sparse vs dense {np.abs(sp - dn).max() / scale:.2e}"


def test_qkv_sp(xlib, cuda, O):
    import torch
    from xtagger_b200 import model as M
    rng = np.random.default_rng(71)
    h = _act8(rng, ROWS, D, O)
    w, ws = _pruned(rng, 3 * D, D)
    adq, cq, ck, cv = 10 / 448, 448 / 2.0, 448 / 4.0, 448 / 3.0
    cs = M.rope_table()
    shp = (NIMG, 16, TP, 64)
    want = [np.zeros(shp, np.uint8) for _ in range(3)]
    O.lib().or_qkv_epilogue(O.gemm_e4m3(h, w, ws, adq), ROWS, cs, cq, ck, cv, *want)
    vals, meta = _sparse(xlib, w)
    dh, dws, dcs = G.dev(h), G.dev(ws), G.dev(cs)
    sp = [G.zeros(shp, torch.uint8) for _ in range(3)]
    dn = [G.zeros(shp, torch.uint8) for _ in range(3)]
    assert xlib.xtb_qkv_sp(G.P(dh), ROWS, G.P(vals), G.P(meta), G.P(dws), adq, *(G.P(t) for t in sp), G.P(dcs), cq, ck,
                           cv, None) == 0
    assert xlib.xtb_qkv(G.P(dh), ROWS, G.P(G.dev(w)), G.P(dws), adq, *(G.P(t) for t in dn), G.P(dcs), cq, ck, cv,
                        None) == 0
    G.check_error_word(xlib)
    for name, s, d, o in zip("qkv", sp, dn, want):
        s, d = G.host(s), G.host(d)
        G.assert_e4m3_close(s, d, 1, 0.999, f"{name} sparse vs dense")
        G.assert_e4m3_close(s, o, 1, 0.99, f"{name} sparse vs oracle")
        assert not s[:, :, 1025:].any(), f"{name}: padding rows written"


def test_oproj_sp(xlib, cuda, O):
    rng = np.random.default_rng(72)
    a = _act8(rng, ROWS, D, O)
    w, ws = _pruned(rng, D, D)
    adq = 4 / 448
    x0 = (rng.standard_normal((ROWS, D), dtype=np.float32) * 2).astype(np.float16).view(np.uint16)
    want = x0.copy()
    O.lib().or_resid_add(want, O.gemm_e4m3(a, w, ws, adq), ROWS)
    vals, meta = _sparse(xlib, w)
    da, dws = G.dev(a), G.dev(ws)
    xs, xd = G.dev(x0), G.dev(x0)
    assert xlib.xtb_oproj_sp(G.P(da), ROWS, G.P(vals), G.P(meta), G.P(dws), adq, G.P(xs), None) == 0
    assert xlib.xtb_oproj(G.P(da), ROWS, G.P(G.dev(w)), G.P(dws), adq, G.P(xd), None) == 0
    G.check_error_word(xlib)
    G.assert_f16_close(G.host(xs), G.host(xd), 1e-3, "oproj sparse vs dense")
    G.assert_f16_close(G.host(xs), want, 1e-2, "oproj sparse vs oracle")


def test_fc1_sp(xlib, cuda, O):
    import torch
    from xtagger_b200 import model as M
    rng = np.random.default_rng(73)
    h = _act8(rng, ROWS, D, O)
    w12 = np.zeros((N12, D), np.float32)
    w12[:2730] = rng.standard_normal((2730, D), dtype=np.float32) * 0.02
    w12[HIDP:HIDP + 2730] = rng.standard_normal((2730, D), dtype=np.float32) * 0.02
    w, ws = _pruned(rng, N12, D, M.interleave_gx(w12))
    adq = 10 / 448
    rs = np.full(HIDP, 448 / 3.0, np.float32)
    want = np.empty((ROWS, HIDP), np.uint8)
    s, q = np.empty(ROWS), np.empty(ROWS)
    O.lib().or_fc1_epilogue(O.gemm_e4m3(h, w, ws, adq), ROWS, rs, want, s, q)
    vals, meta = _sparse(xlib, w)
    dh, dws, drs = G.dev(h), G.dev(ws), G.dev(rs)
    h8s, h8d = G.zeros((ROWS, HIDP), torch.uint8), G.zeros((ROWS, HIDP), torch.uint8)
    sts, std = G.zeros((43, ROWS, 2), torch.float32), G.zeros((43, ROWS, 2), torch.float32)
    assert xlib.xtb_fc1_sp(G.P(dh), ROWS, G.P(vals), G.P(meta), G.P(dws), adq, G.P(h8s), G.P(sts), G.P(drs), None) == 0
    assert xlib.xtb_fc1(G.P(dh), ROWS, G.P(G.dev(w)), G.P(dws), adq, G.P(h8d), G.P(std), G.P(drs), None) == 0
    G.check_error_word(xlib)
    G.assert_e4m3_close(G.host(h8s), G.host(h8d), 1, 0.999, "h8 sparse vs dense")
    G.assert_e4m3_close(G.host(h8s), want, 1, 0.99, "h8 sparse vs oracle")
    ps, pd = G.host(sts).astype(np.float64), G.host(std).astype(np.float64)
    np.testing.assert_allclose(ps, pd, rtol=1e-4, atol=1e-5 * np.abs(pd).max())  # each of the 43 partials
    st = ps.sum(0)
    np.testing.assert_allclose(st[:, 0], s, rtol=1e-3, atol=1e-3 * np.abs(s).max())
    np.testing.assert_allclose(st[:, 1], q, rtol=1e-3)


def test_fc2_sp(xlib, cuda, O):
    rng = np.random.default_rng(74)
    h8 = _act8(rng, ROWS, HIDP, O, 0.5)
    h8[:, 2730:] = 0
    w, ws = _pruned(rng, D, HIDP)
    adq = 3 / 448
    c = (rng.standard_normal(D) * 0.3).astype(np.float32)
    d = (rng.standard_normal(D) * 0.1).astype(np.float32)
    s = rng.standard_normal(ROWS) * 5
    q = s * s / 2730 + np.abs(rng.standard_normal(ROWS)) * 2730 * 0.5 + 1
    x0 = (rng.standard_normal((ROWS, D), dtype=np.float32) * 2).astype(np.float16).view(np.uint16)
    want = x0.copy()
    O.lib().or_fc2_epilogue(want, O.gemm_e4m3(h8, w, ws, adq), ROWS, s, q, c, d)
    stat = np.zeros((43, ROWS, 2), np.float32)
    stat[0, :, 0], stat[0, :, 1] = s, q
    vals, meta = _sparse(xlib, w)
    dh, dws, dc, dd = G.dev(h8), G.dev(ws), G.dev(c), G.dev(d)
    xs, xd = G.dev(x0), G.dev(x0)
    assert xlib.xtb_fc2_sp(G.P(dh), ROWS, G.P(vals), G.P(meta), G.P(dws), adq, G.P(xs), G.P(G.dev(stat)), G.P(dc),
                           G.P(dd), None) == 0
    assert xlib.xtb_fc2(G.P(dh), ROWS, G.P(G.dev(w)), G.P(dws), adq, G.P(xd), G.P(G.dev(stat)), G.P(dc), G.P(dd),
                        None) == 0
    G.check_error_word(xlib)
    G.assert_f16_close(G.host(xs), G.host(xd), 1e-3, "fc2 sparse vs dense")
    G.assert_f16_close(G.host(xs), want, 1e-2, "fc2 sparse vs oracle")
