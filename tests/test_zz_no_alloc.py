"""xtb_fc2_noalloc -- fc2 with its scratch in a static device array, for callers that cannot let the library
allocate device memory -- against xtb_fc2 through the C ABI, on two calls in a row (the second with fewer rows,
so a stale tail of the shared array from the first call would show)."""
import numpy as np
import pytest

from tests import _gpu as G

pytestmark = pytest.mark.gpu

D, HIDP, HID, NSTAT = 1024, 2736, 2730, 43


def _case(rng, rows):
    from oracle import oracle as O
    from xtagger_b200 import model as M
    u = rng.standard_normal((rows, HID)).astype(np.float32) * 0.3
    h8 = np.zeros((rows, HIDP), np.uint8)
    h8[:, :HID] = O.e4m3(u * (448 / 3.0))
    w, ws = M.quant_blocks(rng.standard_normal((D, HIDP)).astype(np.float32) * 0.02)
    stat = np.zeros((NSTAT, rows, 2), np.float32)
    up = np.zeros((rows, NSTAT * 64), np.float32)
    up[:, :HID] = u
    g = up.reshape(rows, NSTAT, 64)
    stat[:, :, 0] = g.sum(2).T
    stat[:, :, 1] = (g * g).sum(2).T
    c = (rng.standard_normal(D) * 0.3).astype(np.float32)
    d = (rng.standard_normal(D) * 0.1).astype(np.float32)
    x0 = (rng.standard_normal((rows, D)) * 2).astype(np.float16).view(np.uint16)
    return h8, w, ws, stat, c, d, x0


def test_noalloc_matches_fc2_on_two_calls(xlib, cuda):
    rng = np.random.default_rng(31)
    for rows in (2 * 1025, 1025 + 77):
        h8, w, ws, stat, c, d, x0 = _case(rng, rows)
        args = lambda x, st: (G.P(G.dev(h8)), rows, G.P(G.dev(w)), G.P(G.dev(ws)), 3 / 448, G.P(x), G.P(st),
                              G.P(G.dev(c)), G.P(G.dev(d)), None)
        x_ref, st_ref = G.dev(x0), G.dev(stat)
        assert xlib.xtb_fc2(*args(x_ref, st_ref)) == 0
        x_na, st_na = G.dev(x0), G.dev(stat)
        assert xlib.xtb_fc2_noalloc(*args(x_na, st_na)) == 0
        G.check_error_word(xlib)
        got, want = G.host(x_na).view(np.uint16), G.host(x_ref).view(np.uint16)
        G.assert_f16_close(got, want, 1e-2, f"noalloc fc2 ({rows} rows)")
        assert np.array_equal(G.host(st_na), stat)          # the caller's partials are only read
        G.release()


def test_noalloc_rejects_rows_beyond_the_static_scratch(xlib, cuda):
    import torch
    rows = 16 * 1025 + 1
    x = G.zeros((8, D), torch.int16)
    assert xlib.xtb_fc2_noalloc(G.P(x), rows, G.P(x), G.P(x), 1.0, G.P(x), G.P(x), G.P(x), G.P(x), None) == -1
    assert xlib.xtb_fc2_noalloc(G.P(x), 0, G.P(x), G.P(x), 1.0, G.P(x), G.P(x), G.P(x), G.P(x), None) == -1
