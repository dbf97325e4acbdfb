"""GPU preprocessing (xtb_prep_ingest / xtb_prep_crop) against the CPU oracle's restatement of procimg.h's wd path,
bit for bit: every output half, and the image modified in place by alpha over white. Cases cover the scale-1 path
(whole 448-pixel sides, a 448 crop, vertical white pad), upscaling with white borders, downscaling from level 0 and
from pyramid levels 1 and 2, crops, an extreme aspect ratio and padded row strides. Then directly against the
reference's own preprocessing functions (procimg.h compiled with the reference's flags by
tests/golden/make_prep_golden.py): the sha256 of every output of tests/golden/golden_prep.json."""
import ctypes as C
import hashlib
import json
import os

import numpy as np
import pytest

from tests import _gpu as G

pytestmark = pytest.mark.gpu

CASES = [  # w, h, alpha, rect (x0, y0, cw, ch) or None for the whole image, extra stride bytes
    (448, 448, 0, None, 0),
    (448, 300, 1, None, 0),
    (897, 897, 0, (100, 200, 448, 448), 0),
    (300, 200, 1, None, 0),
    (1000, 700, 1, None, 64),
    (2000, 1500, 0, None, 0),
    (2000, 1500, 1, (100, 50, 900, 1200), 0),
    (4000, 3000, 0, None, 16),
    (4000, 3000, 1, (500, 300, 2400, 1800), 0),
    (1600, 30, 0, None, 0),
    (13, 977, 1, None, 4),
]


@pytest.mark.parametrize("w,h,alpha,rect,pad", CASES)
def test_prep_matches_oracle(xlib, cuda, w, h, alpha, rect, pad):
    import torch
    from oracle import oracle as O
    rng = np.random.default_rng(90 + w + h)
    stride = 4 * w + pad
    img = rng.integers(0, 256, (h, stride), dtype=np.uint8)
    if alpha:  # some fully transparent and fully opaque pixels too
        a = img[:, 3:4 * w:4]
        a[::5, ::3] = 0
        a[1::7, ::2] = 255
    x0, y0, cw, ch = rect or (0, 0, w, h)
    want_img = img.copy()
    want = np.zeros(1024 * 592, np.uint16)
    O.lib().or_prep(want_img, w, h, stride, alpha, x0, y0, cw, ch, want)
    dimg = G.dev(img)
    scratch = G.zeros((xlib.xtb_prep_scratch_bytes(w, h),), torch.uint8)
    out = G.zeros((1024 * 592,), torch.int16)
    out.fill_(0x5555)  # every half must be written (pad columns included)
    assert xlib.xtb_prep_ingest(G.P(dimg), w, h, stride, alpha, G.P(scratch), None) == 0
    assert xlib.xtb_prep_crop(G.P(dimg), w, h, stride, x0, y0, cw, ch, G.P(scratch), G.P(out), None) == 0
    got = G.host(out).view(np.uint16)
    gimg = G.host(dimg)
    assert np.array_equal(gimg[:, :4 * w], want_img[:, :4 * w]), "alpha over white differs"
    assert np.array_equal(gimg[:, 4 * w:], img[:, 4 * w:]), "bytes past the row written"
    diff = got != want
    assert not diff.any(), f"{int(diff.sum())} of {diff.size} halves differ (first at {np.argmax(diff)})"


def test_prep_rejects_bad_arguments(xlib, cuda):
    import torch
    img = G.zeros((10, 40), torch.uint8)
    scratch = G.zeros((xlib.xtb_prep_scratch_bytes(10, 10),), torch.uint8)
    out = G.zeros((1024 * 592,), torch.int16)
    assert xlib.xtb_prep_ingest(G.P(img), 10, 10, 38, 0, G.P(scratch), None) == -1      # stride < 4 w
    assert xlib.xtb_prep_crop(G.P(img), 10, 10, 40, 5, 0, 6, 10, G.P(scratch), G.P(out), None) == -1  # rect
    assert xlib.xtb_prep_crop(G.P(img), 10, 10, 40, 0, 0, 10, 10, None, G.P(out), None) == -1


def test_mixed_views_match_oracle(xlib, cuda):
    """The PixAI-style batch (whole images and quadrant crops of 896^2 sources, xtagger_b200.views) made on the
    device equals the oracle's preprocessing of every view."""
    from oracle import oracle as O
    from xtagger_b200 import views as V
    views = V.mix_views(7)  # one source x (whole + 4 quadrants), then two whole images
    nsrc = V.num_sources(views)
    src = V.mix_sources(nsrc, seed=9)
    dsrc = G.dev(src)
    prep = V.DevicePrep(V.SIDE, V.SIDE, nsrc)
    out = G.zeros((len(views), 1024 * 592), __import__("torch").int16)
    nk = prep.run([dsrc[i].data_ptr() for i in range(nsrc)], views, out.data_ptr(), 0)
    assert nk == nsrc * 1 + 3 * 3 + 4 * 1  # ingest 1 each; whole images 3 kernels; quadrants 1
    got = G.host(out).view(np.uint16)
    for i, (s, x0, y0, cw, ch) in enumerate(views):
        want = np.zeros(1024 * 592, np.uint16)
        O.lib().or_prep(src[s].copy(), V.SIDE, V.SIDE, 4 * V.SIDE, 0, x0, y0, cw, ch, want)
        assert np.array_equal(got[i], want), f"view {i} {views[i]} differs"


def test_prep_feeds_engine_in_place(xlib, cuda, tmp_path):
    """Preprocessing written straight into the engine's resident inputs (eva_input) and the scores read back from
    eva_output (xtb_copy_async) give the same scores as eva_submit of the same inputs from the host."""
    import torch
    from xtagger_b200 import lib as L
    from xtagger_b200 import model as M
    from xtagger_b200 import views as V
    from xtagger_b200.engine import Engine
    path = M.write_synthetic(str(tmp_path / "m.bin"), seed=7, nl=2, nt=300, ln_noise=1.0)
    views = V.mix_views(5)
    src = V.mix_sources(1, seed=10)
    dsrc = G.dev(src)
    prep = V.DevicePrep(V.SIDE, V.SIDE, 1)
    eng = Engine(path, nb=len(views))
    try:
        eng.ready()
        st = eng.stream(0)
        prep.run([dsrc[0].data_ptr()], views, eng.device_input(0), st)
        eng.forward_resident()
        scores = torch.empty((len(views), eng.nt), dtype=torch.float32).pin_memory()
        assert xlib.xtb_copy_async(C.c_void_p(scores.data_ptr()), C.c_void_p(eng.device_output(0)),
                                   scores.numel() * 4, C.c_void_p(st)) == 0
        torch.cuda.synchronize()
        got = scores.numpy().copy()
        ops = np.zeros((len(views), 1024, 592), np.uint16)
        torch.cuda.synchronize()
        assert xlib.xtb_copy_async(C.c_void_p(ops.ctypes.data), C.c_void_p(eng.device_input(0)),
                                   ops.nbytes, C.c_void_p(st)) == 0
        torch.cuda.synchronize()
        want = eng.run(ops)
        assert eng.device_input(1) is None and eng.device_output(-1) is None
    finally:
        eng.close()
    assert np.isfinite(got).all()
    assert np.array_equal(got, want)
    assert L.EVA_IN == 1024 * 592


def test_prep_matches_the_reference_preprocessing(xlib, cuda):
    import torch
    from tests.golden.prep_case import cases, image
    want = json.load(open(os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "golden_prep.json")))
    bad = []
    for name, w, h, alpha, seed, rects in cases():
        for i, (x0, y0, cw, ch) in enumerate(rects):
            dimg = G.dev(image(w, h, alpha, seed))
            scratch = G.zeros((xlib.xtb_prep_scratch_bytes(w, h),), torch.uint8)
            out = G.zeros((1024 * 592,), torch.int16)
            assert xlib.xtb_prep_ingest(G.P(dimg), w, h, 4 * w, alpha, G.P(scratch), None) == 0
            assert xlib.xtb_prep_crop(G.P(dimg), w, h, 4 * w, x0, y0, cw, ch, G.P(scratch), G.P(out), None) == 0
            if hashlib.sha256(G.host(out).tobytes()).hexdigest() != want[name][i]:
                bad.append((name, i))
            G.release()
    assert not bad, f"GPU outputs that differ from the reference's preprocessing: {bad}"
