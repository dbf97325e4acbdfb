"""The preprocessing oracle (oracle/prep_oracle.c, a restatement of src/core/procimg.h's wd path) pinned by exact
known answers on the CPU: the /255 rounding over its whole domain, alpha over white, the box pyramid's rounding
rules, the scale-1 path for every byte value, the level choice, and the bicubic resample against an independent
float64 implementation of the same filter; and bit for bit against the reference's own preprocessing functions, cut
out of procimg.h and compiled by tests/golden/make_prep_golden.py (procimg.h as a whole needs the Windows-only engine
headers and cannot be built here)."""
import os

import numpy as np
import pytest


@pytest.fixture(scope="module")
def O():
    from oracle import oracle
    return oracle


def test_div255_exact(O):
    lib = O.lib()
    xs = np.arange(0, 65026)
    got = np.array([lib.or_div255(int(x)) for x in xs])
    want = np.floor(xs / 255 + 0.5)
    np.testing.assert_array_equal(got, want)


def test_over_white(O):
    rng = np.random.default_rng(80)
    img = rng.integers(0, 256, (7, 9, 4), dtype=np.uint8)
    img[0, :4, 3] = (0, 255, 1, 254)
    a = img[..., 3:].astype(np.float64)
    want = np.floor((img[..., :3] * a + 255 * (255 - a)) / 255 + 0.5).astype(np.uint8)
    got = img.copy()
    O.lib().or_over_white(got, 9, 7, 36, 1)
    np.testing.assert_array_equal(got[..., :3], want)
    assert (got[..., 3] == 255).all()
    got = img.copy()
    O.lib().or_over_white(got, 9, 7, 36, 0)  # no alpha: colours untouched, X = 255
    np.testing.assert_array_equal(got[..., :3], img[..., :3])
    assert (got[..., 3] == 255).all()


def test_half_rounding(O):
    # rows average rounding up, then columns rounding down: (1, 2 / 2, 2) -> rows 2, 2 -> 2; (0, 1 / 0, 0) -> 1, 0 -> 0
    s = np.zeros((2, 4, 4), np.uint8)
    s[0, 0, 0], s[1, 0, 0], s[0, 1, 0], s[1, 1, 0] = 1, 2, 2, 2
    s[0, 0, 1], s[1, 0, 1], s[0, 1, 1], s[1, 1, 1] = 0, 0, 1, 0
    s[0, 0, 2], s[1, 0, 2], s[0, 1, 2], s[1, 1, 2] = 255, 254, 254, 254
    d = np.zeros((1, 2, 4), np.uint8)
    O.lib().or_half(s, 4, 2, 16, d, 8)
    assert tuple(d[0, 0, :3]) == (2, 0, 254)
    rng = np.random.default_rng(81)
    s = rng.integers(0, 256, (9, 11, 4), dtype=np.uint8)
    d = np.zeros((4, 5, 4), np.uint8)
    O.lib().or_half(s, 11, 9, 44, d, 20)
    t = s[:8, :10].astype(np.int32)
    rows = (t[0::2] + t[1::2] + 1) >> 1
    np.testing.assert_array_equal(d, (rows[:, 0::2] + rows[:, 1::2]) >> 1)


def test_scale_one_every_byte(O):
    """A 448 x 448 image is only normalised: fp16(fp32(v * fl(1/127.5) - 1)) with one rounding to fp32 (an FMA)."""
    v = np.arange(448 * 448 * 4, dtype=np.int64).reshape(448, 448, 4) % 256
    img = v.astype(np.uint8)
    img[..., 3] = 255
    out = np.zeros(1024 * 592, np.uint16)
    O.lib().or_prep(img.copy(), 448, 448, 448 * 4, 0, 0, 0, 448, 448, out)
    sc = float(np.float32(1.0) / np.float32(127.5))
    want = (v[..., :3] * sc - 1.0).astype(np.float32).astype(np.float16).view(np.uint16)
    o = out.reshape(32, 32, 592)  # [patch row][patch col][column]
    for q, c in ((0, 2), (1, 1), (2, 0)):  # planes B, G, R
        plane = o[:, :, q * 196:(q + 1) * 196].reshape(32, 32, 14, 14).transpose(0, 2, 1, 3).reshape(448, 448)
        np.testing.assert_array_equal(plane, want[..., c])
    assert not o[:, :, 588:].any()


@pytest.mark.parametrize("w,h,side,level", [(448, 448, 448, 0), (1000, 700, 1000, 0), (2000, 1500, 2000, 1),
                                            (4000, 3000, 4000, 2), (4000, 3000, 1200, 0), (4000, 3000, 2400, 1),
                                            (30000, 3, 30000, 1)])
def test_level_choice(O, w, h, side, level):
    assert O.lib().or_prep_level(w, h, side) == level


def _bicubic64(x):
    x = np.abs(x)
    return np.where(x < 1, (1.5 * x - 2.5) * x * x + 1, np.where(x < 2, ((-0.5 * x + 2.5) * x - 4) * x + 2, 0.0))


def _resample64(img, S=448):
    """Independent float64 statement of the filter: content centred in a white square of side max(w, h), Keys
    bicubic stretched by the downscale factor (antialiasing), weights normalised over the square."""
    h, w = img.shape[:2]
    side = max(w, h)
    scale = side / S
    fs = max(scale, 1.0)

    def axis(off, length):
        m = np.zeros((S, side))
        for i in range(S):
            c = (i + 0.5) * scale
            j = np.arange(int(max(0, c - 2 * fs + 0.5)), int(min(side, c + 2 * fs + 0.5)))
            wt = _bicubic64((j - c + 0.5) / fs)
            m[i, j] = wt / wt.sum()
        return m

    sq = np.full((side, side, 3), 255.0)
    oy, ox = (side - h) // 2, (side - w) // 2
    sq[oy:oy + h, ox:ox + w] = img[..., :3]
    my, mx = axis(oy, h), axis(ox, w)
    out = np.stack([my @ sq[..., c] @ mx.T for c in range(3)], axis=2)
    return np.clip(out / 127.5 - 1, -1, 1)


@pytest.mark.parametrize("w,h", [(300, 200), (1000, 700)])
def test_resample_matches_float64_filter(O, w, h):
    rng = np.random.default_rng(82 + w)
    img = rng.integers(0, 256, (h, w, 4), dtype=np.uint8)
    img[..., 3] = 255
    out = np.zeros(1024 * 592, np.uint16)
    O.lib().or_prep(img.copy(), w, h, w * 4, 0, 0, 0, w, h, out)
    o = out.reshape(32, 32, 592)
    want = _resample64(img)
    for q, c in ((0, 2), (1, 1), (2, 0)):
        plane = o[:, :, q * 196:(q + 1) * 196].reshape(32, 32, 14, 14).transpose(0, 2, 1, 3).reshape(448, 448)
        got = plane.view(np.float16).astype(np.float64)
        assert np.abs(got - want[..., c]).max() <= 2.5e-3  # fp16 steps of 2^-11 near 1 plus fp32 sums


def test_mix_views_layout():
    """32 inputs = 6 sources x (whole image + 4 quadrants) + 2 whole images, every rect inside its 896^2 source."""
    from xtagger_b200 import views as V
    v = V.mix_views(32)
    assert len(v) == 32 and V.num_sources(v) == 8
    assert sum(1 for x in v if x[3] == V.SIDE) == 8
    for s in range(6):
        quads = sorted((x0, y0) for (t, x0, y0, cw, ch) in v if t == s and cw == V.SIDE // 2)
        assert quads == [(0, 0), (0, 448), (448, 0), (448, 448)]
    assert all(0 <= x0 and 0 <= y0 and x0 + cw <= V.SIDE and y0 + ch <= V.SIDE for _, x0, y0, cw, ch in v)
    src = V.mix_sources(2, seed=3)
    assert src.shape == (2, 896, 896 * 4) and (src.reshape(2, 896, 896, 4)[..., 3] == 255).all()


@pytest.mark.parametrize("args,n", [((896, 896, 0, 0, 0, 0), 1), ((4000, 3000, 0, 0, 0, 0), 3),
                                    ((896, 896, 0, 0, 896, 896), 3), ((896, 896, 448, 448, 448, 448), 1),
                                    ((897, 897, 100, 200, 448, 448), 1), ((896, 896, 500, 0, 448, 10), -1),
                                    ((0, 896, 0, 0, 0, 0), -1)])
def test_prep_kernel_counts(xlib, args, n):
    """Kernels per call: ingest = alpha pass + one per pyramid level above 0; crop = 1 on the normalise-only path,
    3 (tables, vertical, horizontal) when resampling; bad rects -1. Host arithmetic only, no device."""
    assert xlib.xtb_prep_kernels(*args) == n


def test_oracle_matches_the_reference_preprocessing():
    """The oracle against the reference's own preprocessing: procimg.h's pi_row_rgbx / pi_pyramid / pi_prep (and the
    functions they call), extracted from the reference at generation time and compiled with its release flags
    (tests/golden/make_prep_golden.py), on seeded images through the identity path, resamples up and down from level
    0 and from pyramid levels 1 and 2, odd sizes and rects, with and without alpha: every output bit-identical (sha256
    of each model input in tests/golden/golden_prep.json)."""
    import hashlib
    import json

    from oracle import oracle as O
    from tests.golden.prep_case import cases, image
    want = json.load(open(os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "golden_prep.json")))
    bad = []
    for name, w, h, alpha, seed, rects in cases():
        for i, (x0, y0, cw, ch) in enumerate(rects):
            img = image(w, h, alpha, seed)
            out = np.zeros((1024, 592), np.uint16)
            O.lib().or_prep(img.reshape(-1), w, h, 4 * w, alpha, x0, y0, cw, ch, out.reshape(-1))
            if hashlib.sha256(out.tobytes()).hexdigest() != want[name][i]:
                bad.append((name, i))
    assert not bad, f"oracle outputs that differ from the reference's preprocessing: {bad}"
