"""Every hot-path kernel through its C-ABI entry point against the CPU oracle on the same seeded inputs.

Integer / layout work is compared code for code; rounding decisions at representable-value boundaries may differ
by one E4M3 step (the GPU accumulates in fp32 in a different order, and uses the hardware exp2 / tanh
approximations the reference also uses), and fp16 / fp32 values within 1e-2 relative.
"""
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
    """E4M3 activations as the LayerNorm kernel would produce them (|x| up to ~448)."""
    return O.e4m3(rng.standard_normal((rows, k), dtype=np.float32) * sd * (448 / 8))


def _w8(rng, n, k):
    from xtagger_b200 import model as M
    return M.quant_blocks(rng.standard_normal((n, k), dtype=np.float32) * 0.02)


def test_ln_e4m3(xlib, cuda, O):
    rng = np.random.default_rng(11)
    x = (rng.standard_normal((ROWS, D), dtype=np.float32) * 3 + rng.standard_normal((ROWS, 1), dtype=np.float32))
    xh = x.astype(np.float16).view(np.uint16)
    g = (1 + 0.2 * rng.standard_normal(D)).astype(np.float32)
    b = (0.1 * rng.standard_normal(D)).astype(np.float32)
    qs = 448 / 10.0
    want = np.empty((ROWS, D), np.uint8)
    O.lib().or_ln_e4m3(xh, g, b, ROWS, qs, want)
    y = G.zeros((ROWS, D), __import__("torch").uint8)
    assert xlib.xtb_ln_e4m3(G.P(G.dev(xh)), G.P(G.dev(g)), G.P(G.dev(b)), G.P(y), ROWS, qs, None) == 0
    G.check_error_word(xlib)
    G.assert_e4m3_close(G.host(y), want, 1, 0.995, "ln")


def test_qkv_epilogue_layouts(xlib, cuda, O):
    import torch
    from xtagger_b200 import model as M
    rng = np.random.default_rng(12)
    h = _act8(rng, ROWS, D, O)
    w, ws = _w8(rng, 3 * D, D)
    adq, cq, ck, cv = 10 / 448, 448 / 2.0, 448 / 4.0, 448 / 3.0
    cs = M.rope_table()
    acc = O.gemm_e4m3(h, w, ws, adq)
    qw = np.zeros((NIMG, 16, TP, 64), np.uint8)
    kw, vw = np.zeros_like(qw), np.zeros((NIMG, 16, TP, 64), np.uint8)
    O.lib().or_qkv_epilogue(acc, ROWS, cs, cq, ck, cv, qw, kw, vw)
    q8, k8, vt8 = (G.zeros(a.shape, torch.uint8) for a in (qw, kw, vw))
    rc = xlib.xtb_qkv(G.P(G.dev(h)), ROWS, G.P(G.dev(w)), G.P(G.dev(ws)), adq, G.P(q8), G.P(k8), G.P(vt8),
                      G.P(G.dev(cs)), cq, ck, cv, None)
    assert rc == 0
    G.check_error_word(xlib)
    for name, got, want in (("q", q8, qw), ("k", k8, kw), ("vt", vt8, vw)):
        got = G.host(got)
        G.assert_e4m3_close(got, want, 1, 0.99, name)
    # padded key rows / columns untouched (zero)
    assert not G.host(q8)[:, :, 1025:].any() and not G.host(vt8)[:, :, 1025:].any()


@pytest.mark.parametrize("peaked", [False, True])
def test_attention(xlib, cuda, O, peaked):
    import torch
    rng = np.random.default_rng(13 + peaked)
    shape = (NIMG, 16, TP, 64)
    sd = 3.0 if peaked else 1.0   # peaked: large scores, so lazy rescales and dead tiles occur
    q = np.zeros(shape, np.uint8)
    k = np.zeros(shape, np.uint8)
    vt = np.zeros((NIMG, 16, TP, 64), np.uint8)
    q[:, :, :1025] = O.e4m3(rng.standard_normal((NIMG, 16, 1025, 64), dtype=np.float32) * 60 * sd)
    k[:, :, :1025] = O.e4m3(rng.standard_normal((NIMG, 16, 1025, 64), dtype=np.float32) * 60 * sd)
    vt[:, :, :1025] = O.e4m3(rng.standard_normal((NIMG, 16, 1025, 64), dtype=np.float32) * 100)
    sinv = (0.8 / 448) * (4.0 / 448)
    vo = (448 / 3.0) * (3.0 / 448) * 0.9
    want = np.empty((ROWS, D), np.uint8)
    O.lib().or_attention(q, k, vt, NIMG, sinv, vo, 64, 16, want)   # the reference's tiling and slices
    out = G.zeros((ROWS, D), torch.uint8)
    assert xlib.xtb_attention(G.P(G.dev(q)), G.P(G.dev(k)), G.P(G.dev(vt)), NIMG, G.P(out), sinv, vo, None) == 0
    G.check_error_word(xlib)
    G.assert_attention_close(G.host(out), want)


def test_oproj_residual(xlib, cuda, O):
    rng = np.random.default_rng(14)
    a = _act8(rng, ROWS, D, O)
    w, ws = _w8(rng, D, D)
    adq = 4 / 448
    x0 = (rng.standard_normal((ROWS, D), dtype=np.float32) * 2).astype(np.float16).view(np.uint16)
    want = x0.copy()
    O.lib().or_resid_add(want, O.gemm_e4m3(a, w, ws, adq), ROWS)
    x = G.dev(x0)
    assert xlib.xtb_oproj(G.P(G.dev(a)), ROWS, G.P(G.dev(w)), G.P(G.dev(ws)), adq, G.P(x), None) == 0
    G.check_error_word(xlib)
    G.assert_f16_close(G.host(x), want, 1e-2, "oproj")


def test_fc1_swiglu_stats(xlib, cuda, O):
    import torch
    from xtagger_b200 import model as M
    rng = np.random.default_rng(15)
    h = _act8(rng, ROWS, D, O)
    w12 = np.zeros((N12, D), np.float32)
    w12[:2730] = rng.standard_normal((2730, D), dtype=np.float32) * 0.02
    w12[HIDP:HIDP + 2730] = rng.standard_normal((2730, D), dtype=np.float32) * 0.02
    w, ws = M.quant_blocks(M.interleave_gx(w12))
    adq = 10 / 448
    rs = np.full(HIDP, 448 / 3.0, np.float32)
    acc = O.gemm_e4m3(h, w, ws, adq)
    want = np.empty((ROWS, HIDP), np.uint8)
    s, q = np.empty(ROWS), np.empty(ROWS)
    O.lib().or_fc1_epilogue(acc, ROWS, rs, want, s, q)
    h8 = G.zeros((ROWS, HIDP), torch.uint8)
    stat = G.zeros((43, ROWS, 2), torch.float32)
    assert xlib.xtb_fc1(G.P(G.dev(h)), ROWS, G.P(G.dev(w)), G.P(G.dev(ws)), adq, G.P(h8), G.P(stat), G.P(G.dev(rs)),
                        None) == 0
    G.check_error_word(xlib)
    G.assert_e4m3_close(G.host(h8), want, 1, 0.99, "h8")
    st = G.host(stat).astype(np.float64).sum(0)
    np.testing.assert_allclose(st[:, 0], s, rtol=1e-3, atol=1e-3 * np.abs(s).max())
    np.testing.assert_allclose(st[:, 1], q, rtol=1e-3)


def test_fc2_folded_ln(xlib, cuda, O):
    import torch
    rng = np.random.default_rng(16)
    h8 = _act8(rng, ROWS, HIDP, O, 0.5)
    h8[:, 2730:] = 0
    w, ws = _w8(rng, D, HIDP)
    adq = 3 / 448
    c = (rng.standard_normal(D) * 0.3).astype(np.float32)
    d = (rng.standard_normal(D) * 0.1).astype(np.float32)
    s = rng.standard_normal(ROWS) * 5
    q = s * s / 2730 + np.abs(rng.standard_normal(ROWS)) * 2730 * 0.5 + 1
    x0 = (rng.standard_normal((ROWS, D), dtype=np.float32) * 2).astype(np.float16).view(np.uint16)
    want = x0.copy()
    O.lib().or_fc2_epilogue(want, O.gemm_e4m3(h8, w, ws, adq), ROWS, s, q, c, d)
    # the kernel reads 43 partials per row: put the sums in partial 0
    stat = np.zeros((43, ROWS, 2), np.float32)
    stat[0, :, 0], stat[0, :, 1] = s, q
    x = G.dev(x0)
    assert xlib.xtb_fc2(G.P(G.dev(h8)), ROWS, G.P(G.dev(w)), G.P(G.dev(ws)), adq, G.P(x), G.P(G.dev(stat)),
                        G.P(G.dev(c)), G.P(G.dev(d)), None) == 0
    G.check_error_word(xlib)
    G.assert_f16_close(G.host(x), want, 1e-2, "fc2")


def test_patch_embed(xlib, cuda, O):
    import torch
    from xtagger_b200 import model as M
    rng = np.random.default_rng(17)
    inp = M.synthetic_inputs(NIMG, seed=3)
    pe = np.zeros((D, 592), np.float32)
    pe[:, :588] = rng.standard_normal((D, 588), dtype=np.float32) * 0.02
    pe = pe.astype(np.float16).view(np.uint16)
    pos = (rng.standard_normal((1025, D), dtype=np.float32) * 0.02).astype(np.float32)
    want = np.empty((ROWS, D), np.uint16)
    O.lib().or_patch_embed(inp, NIMG, pe, pos, want)
    x = G.zeros((ROWS, D), torch.int16)
    assert xlib.xtb_patch_embed(G.P(G.dev(inp)), NIMG, G.P(G.dev(pe)), G.P(G.dev(pos)), G.P(x), None) == 0
    G.check_error_word(xlib)
    G.assert_f16_close(G.host(x).view(np.uint16), want, 1e-2, "patch embed")


@pytest.mark.parametrize("head8", [False, True])
def test_pool_ln_head(xlib, cuda, O, head8):
    import torch
    from xtagger_b200 import model as M
    rng = np.random.default_rng(18 + head8)
    nt = 10861
    x = (rng.standard_normal((ROWS, D), dtype=np.float32) * 2 + 0.3).astype(np.float16).view(np.uint16)
    g = (1 + 0.1 * rng.standard_normal(D)).astype(np.float32)
    b = (0.1 * rng.standard_normal(D)).astype(np.float32)
    hw = rng.standard_normal((nt, D), dtype=np.float32) * 0.02
    hb = (rng.standard_normal(nt) * 0.5).astype(np.float32)
    qs = 448 / 10.0
    pool = np.empty((NIMG, D), np.float32)
    pn = np.empty((NIMG, D), np.uint16)
    pn8 = np.empty((NIMG, D), np.uint8)
    O.lib().or_pool_ln(x, NIMG, g, b, pool, pn, pn8.ctypes.data, qs)
    want = np.empty((NIMG, nt), np.float32)
    dpool, dpn, dpn8 = G.zeros((NIMG, D), torch.float32), G.zeros((NIMG, D), torch.int16), G.zeros((NIMG, D), torch.uint8)
    assert xlib.xtb_pool_ln(G.P(G.dev(x)), NIMG, G.P(G.dev(g)), G.P(G.dev(b)), G.P(dpool), G.P(dpn), G.P(dpn8), qs,
                            None) == 0
    out = G.zeros((NIMG, nt), torch.float32)
    if head8:
        w8, ws = M.quant_blocks(hw)
        O.lib().or_head_e4m3(pn8, NIMG, w8, ws, 1 / qs, hb, nt, want)
        rc = xlib.xtb_head_e4m3(G.P(G.dev(w8)), nt, G.P(G.dev(ws)), G.P(dpn8), NIMG, 1 / qs, G.P(G.dev(hb)), G.P(out),
                                None)
    else:
        w16 = hw.astype(np.float16).view(np.uint16)
        O.lib().or_head_f16(pn, NIMG, w16, hb, nt, want)
        rc = xlib.xtb_head_f16(G.P(G.dev(w16)), nt, G.P(dpn), NIMG, G.P(G.dev(hb)), G.P(out), None)
    assert rc == 0
    G.check_error_word(xlib)
    np.testing.assert_allclose(G.host(dpool), pool, rtol=1e-4, atol=1e-4)
    G.assert_f16_close(G.host(dpn).view(np.uint16), pn, 1e-2, "pn")
    np.testing.assert_allclose(G.host(out), want, atol=2e-3)


def test_fc1_mx_block_scale(xlib, cuda, O):
    """Power-of-two block scales on the tensor core's own block scaling (kind::mxf8f6f4.block_scale): the same h8
    as the oracle (and as the promoting kernel on the same weights), codes equal or one step apart."""
    import ctypes as C
    import torch
    from xtagger_b200 import model as M
    rng = np.random.default_rng(17)
    h = _act8(rng, ROWS, D, O)
    w12 = np.zeros((N12, D), np.float32)
    w12[:2730] = rng.standard_normal((2730, D), dtype=np.float32) * 0.02
    w12[HIDP:HIDP + 2730] = rng.standard_normal((2730, D), dtype=np.float32) * 0.02
    w12[:, :128] *= 8.0                              # block scales that differ across K blocks and N blocks
    w12[1000:1200] *= 0.25
    w, ws = M.quant_blocks(M.interleave_gx(w12), pow2=True)
    assert len(np.unique(ws)) > 2
    adq = 10 / 448
    rs = np.full(HIDP, 448 / 3.0, np.float32)
    acc = O.gemm_e4m3(h, w, ws, adq)
    want = np.empty((ROWS, HIDP), np.uint8)
    s, q = np.empty(ROWS), np.empty(ROWS)
    O.lib().or_fc1_epilogue(acc, ROWS, rs, want, s, q)
    img = np.zeros(xlib.xtb_sf_image_bytes(N12, D), np.uint8)
    assert xlib.xtb_sf_image(ws.ctypes.data_as(C.c_void_p), N12, D, img.ctypes.data_as(C.c_void_p)) == 0
    bad = ws.copy()
    bad[0, 0] *= 1.5
    assert xlib.xtb_sf_image(bad.ctypes.data_as(C.c_void_p), N12, D, img.copy().ctypes.data_as(C.c_void_p)) == -1
    outs = []
    for mx in (False, True):
        h8 = G.zeros((ROWS, HIDP), torch.uint8)
        stat = G.zeros((43, ROWS, 2), torch.float32)
        if mx:
            rc = xlib.xtb_fc1_mx(G.P(G.dev(h)), ROWS, G.P(G.dev(w)), G.P(G.dev(img)), adq, G.P(h8), G.P(stat),
                                 G.P(G.dev(rs)), None)
        else:
            rc = xlib.xtb_fc1(G.P(G.dev(h)), ROWS, G.P(G.dev(w)), G.P(G.dev(ws)), adq, G.P(h8), G.P(stat),
                              G.P(G.dev(rs)), None)
        assert rc == 0
        G.check_error_word(xlib)
        got = G.host(h8)
        G.assert_e4m3_close(got, want, 1, 0.99, f"h8 (mx {mx})")
        st = G.host(stat).astype(np.float64).sum(0)
        np.testing.assert_allclose(st[:, 1], q, rtol=1e-3)
        outs.append(got)
    G.assert_e4m3_close(outs[1], outs[0], 1, 0.99, "mx vs promote")
