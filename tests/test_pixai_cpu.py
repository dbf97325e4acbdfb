"""PixAI tagger host side on the CPU: the window-major token order, the weight file the synthetic writer produces
(read back by the oracle's reader, whose layout check covers every tensor of px.h:196-245), the global-block rule,
the oracle's head on hand-made inputs, and the engine's header validation (no device needed)."""
import ctypes as C

import numpy as np
import pytest


def test_window_perm_is_a_permutation():
    from xtagger_b200 import pixai as P
    perm = P.window_perm()
    assert sorted(perm.tolist()) == list(range(P.T))
    # window 1 starts at grid row 0, column 24; window 3 at grid row 24, column 0
    assert perm[576] == 24 and perm[3 * 576] == 24 * 72
    # within a window tokens run row-major over 24 x 24
    assert perm[1] == 1 and perm[24] == 72


def test_global_blocks():
    from xtagger_b200 import pixai as P
    assert [i for i in range(32) if P.is_global(i)] == [7, 15, 23, 31]
    assert [i for i in range(4) if P.is_global(i, 4, 0b0110)] == [1, 2]


def test_patch_operand_layout():
    from xtagger_b200 import pixai as P
    img = np.zeros((1008, 1008, 3), np.float32)
    img[14 * 0 + 3, 14 * 24 + 5, 1] = 1.0   # grid (0, 24) = window 1, local token 0; pixel (3, 5) of channel G
    op = P.patch_operand(img)
    assert op.shape == (P.T, P.K0P)
    t = 576
    assert op[t, 1 * 196 + 3 * 14 + 5] == 1.0
    assert (op[:, 588:] == 0).all()
    assert op.astype(np.float32).min() == -1.0


def test_synthetic_file_reads_back(tmp_path):
    from oracle import oracle as O
    from xtagger_b200 import pixai as P
    p = P.write_synthetic(str(tmp_path / "px.bin"), seed=1, nt=77, nl=2, gmask=2)
    assert O.lib().or_px_model_nt(p.encode()) == 77
    hdr = np.fromfile(p, np.uint32, 6)
    assert bytes(hdr[:1].tobytes()) == b"PXAI" and hdr[1] == 3 and hdr[2] == 77 and hdr[4] == 2 and hdr[5] == 2


def test_oracle_head_uniform_pool():
    """With y constant over tokens the pool weights cancel: o = fp16(Wv . y), whatever the scores."""
    from oracle import oracle as O
    rng = np.random.default_rng(2)
    T, D = 5184, 1024
    x = np.zeros((T, D), np.float16)
    x[:] = rng.standard_normal(D).astype(np.float16)
    w = np.ones(D, np.float32)
    b = np.zeros(D, np.float32)
    U = rng.standard_normal((16, D)).astype(np.float32) * 0.01
    hpos = np.zeros((T, D), np.float16)
    wv = (rng.standard_normal((D, D)) * 0.02).astype(np.float16)
    hw = (rng.standard_normal((8, D)) * 0.02).astype(np.float16)
    hb = np.zeros(8, np.float32)
    scores = np.empty((1, 8), np.float32)
    o = np.empty((1, D), np.uint16)
    O.lib().or_px_head(x.view(np.uint16), 1, w, b, U, hpos.view(np.uint16), wv.view(np.uint16), hw.view(np.uint16),
                       hb, 8, scores, o.ctypes.data_as(C.c_void_p))
    xf = x[0].astype(np.float64)
    y = ((xf - xf.mean()) / np.sqrt(xf.var() + 1e-5)).astype(np.float16).astype(np.float64)
    want = wv.astype(np.float64) @ y
    got = o.view(np.float16)[0].astype(np.float64)
    assert np.abs(got - want).max() <= 2e-3 * np.abs(want).max() + 1e-3
    logits = hw.astype(np.float64) @ got
    np.testing.assert_allclose(scores[0], 1 / (1 + np.exp(-logits)), rtol=1e-4, atol=1e-5)


def test_px_open_rejects_bad_files(xlib, tmp_path):
    from xtagger_b200 import lib as L
    p = L.Px()
    assert xlib.px_open(C.byref(p), str(tmp_path / "missing.bin").encode(), 0, None, 0) == -1
    bad = tmp_path / "bad.bin"
    bad.write_bytes(b"EVA2" + b"\0" * 300)
    assert xlib.px_open(C.byref(p), str(bad).encode(), 0, None, 0) == -1
    v2 = tmp_path / "v2.bin"
    v2.write_bytes(b"PXAI" + (2).to_bytes(4, "little") + b"\0" * 300)   # the fp16 calibration format
    assert xlib.px_open(C.byref(p), str(v2).encode(), 0, None, 0) == -1
