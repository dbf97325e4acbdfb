"""The seeded images and crop rects on which the preprocessing oracle (oracle/prep_oracle.c) and the GPU kernels
(xtb_prep_*) are pinned to the reference's own preprocessing (make_prep_golden.py, golden_prep.json).
TEST INFRASTRUCTURE ONLY."""
import numpy as np


def cases():
    """(name, w, h, alpha, image seed, rects): sizes that take the identity path, one resample from level 0 (up and
    down), pyramid levels 1 and 2, odd sizes and rects, fully transparent and opaque pixels."""
    return [
        ("ident_448", 448, 448, 1, 1, [(0, 0, 448, 448)]),
        ("ident_tall", 300, 448, 0, 2, [(0, 0, 300, 448)]),
        ("up_200x130", 200, 130, 1, 3, [(0, 0, 200, 130), (17, 5, 101, 77)]),
        ("down_896", 896, 896, 1, 4, [(0, 0, 896, 896), (0, 0, 448, 448), (448, 448, 448, 448), (100, 37, 613, 501)]),
        ("down_1023x777", 1023, 777, 0, 5, [(0, 0, 1023, 777), (511, 0, 512, 777), (3, 11, 999, 700)]),
        ("pyr_2000x1500", 2000, 1500, 1, 6, [(0, 0, 2000, 1500), (1000, 750, 1000, 750), (13, 29, 1801, 1203)]),
        ("pyr_3601x1207", 3601, 1207, 1, 7, [(0, 0, 3601, 1207), (1800, 0, 1801, 1207)]),
    ]


def image(w, h, alpha, seed):
    """Seeded RGBA bytes: smooth gradients plus noise, alpha mixing 0, 255 and partial values (X = 255 without alpha)."""
    rng = np.random.default_rng(seed)
    yy, xx = np.mgrid[0:h, 0:w].astype(np.float32)
    img = np.empty((h, w, 4), np.uint8)
    for c in range(3):
        g = 127 + 100 * np.sin(xx / (17 + 9 * c) + yy / (23 + 5 * c) + c) + rng.normal(0, 20, (h, w))
        img[:, :, c] = np.clip(g, 0, 255).astype(np.uint8)
    a = rng.integers(0, 256, (h, w))
    a[rng.random((h, w)) < 0.3] = 255
    a[rng.random((h, w)) < 0.1] = 0
    img[:, :, 3] = a if alpha else 255
    return np.ascontiguousarray(img)
