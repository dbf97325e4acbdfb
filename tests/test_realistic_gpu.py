"""The north-star rule end to end on a 24-layer model whose FP8 forward is stable: final sigmoid scores within 2e-3
absolute and the same above-threshold tag sets (0.35 general, 0.85 character, procimg.h:435-436), for this library's
engine against the oracle and against the reference's own kernels run whole (eva_forward's sequence, eva.h:252-307,
oracle/ref_kernels.cu), and for the reference against the oracle.

The model (xtagger_b200.calib.realistic_model) is built the way a real one is: a float model calibrated by the float
forward (FloatEva), its head fitted as a linear probe on the float model's features, converted by the reference's
export_eva.py steps (convert.py) to the reference's v3 format (per-tensor E4M3) or to the block-scaled v4 format the
benchmark runs. Inputs are structured synthetic images (model.structured_inputs). On the random-init model of the
other whole-forward tests the forward is chaotic at E4M3's resolution and no implementation pair agrees to 2e-3;
this one is not, so the north-star tolerance is asserted as stated.

Images whose oracle scores put a tag within 2e-3 of a threshold would make the tag-set rule depend on which side of
the tolerance a score lands, so the inputs are the first images of a seeded pool with no such tag (at least three)."""
import ctypes as C
import os

import numpy as np
import pytest

from tests import _gpu as G

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
REF_SO = os.path.join(ROOT, "oracle", "_ref", "libref_kernels.so")
TOL = 2e-3
THRESHOLDS = (0.35, 0.85)


@pytest.fixture(scope="module")
def models(tmp_path_factory):
    import torch
    from xtagger_b200 import calib as CB
    d = tmp_path_factory.mktemp("realistic")
    out = {"v3": CB.realistic_model(str(d / "v3.bin"), seed=0, nl=24, version=3),
           "v4": CB.realistic_model(str(d / "v4.bin"), seed=0, nl=24, version=4, pow2=True),
           "v4_free": CB.realistic_model(str(d / "v4f.bin"), seed=0, nl=24, version=4, pow2=False)}
    torch.cuda.empty_cache()
    return out


def _pick_inputs(path, n=3, pool=8, seed=41):
    """The first n images of a seeded pool whose oracle scores keep every tag TOL away from each threshold."""
    from oracle import oracle as O
    from xtagger_b200 import model as M
    x = M.structured_inputs(pool, seed=seed)
    want = O.forward(path, x)
    ok = [i for i in range(pool) if all(np.abs(want[i] - t).min() > TOL for t in THRESHOLDS)]
    assert len(ok) >= n, f"only {len(ok)} of {pool} images keep their scores {TOL} away from the thresholds"
    keep = ok[:n]
    return np.ascontiguousarray(x[keep]), want[keep]


def _engine(path, x):
    from xtagger_b200.engine import Engine
    eng = Engine(path, nb=x.shape[0])
    try:
        return eng.run(x)
    finally:
        eng.close()


def _assert_north_star(a, b, what):
    assert np.isfinite(a).all() and np.isfinite(b).all(), what
    e = np.abs(a - b)
    sets = [int(((a > t) != (b > t)).sum()) for t in THRESHOLDS]
    print(f"{what}: max |diff| {e.max():.2e} mean {e.mean():.2e}; tags above 0.35 per image "
          f"{(b > 0.35).sum(1).tolist()}; set differences {sets}")
    assert e.max() <= TOL, f"{what}: max |score difference| {e.max():.2e} > {TOL}"
    assert sets == [0, 0], f"{what}: above-threshold tag sets differ ({sets})"


@pytest.mark.parametrize("name", ["v3", "v4", "v4_free"])
def test_engine_matches_oracle_at_north_star_tolerance(xlib, cuda, models, name):
    from oracle import oracle as O
    x, want = _pick_inputs(models[name])
    got = _engine(models[name], x)
    assert xlib.xtb_error_word(0) == 0
    alt = O.forward(models[name], x, key_tile=128, slice_rows=1)
    print(f"{name}: oracle tiling sensitivity max {np.abs(alt - want).max():.2e}")
    _assert_north_star(got, want, f"{name} engine-vs-oracle")


def test_reference_kernels_engine_and_oracle_agree(xlib, cuda, models):
    if not os.path.exists(REF_SO):
        pytest.skip("oracle/_ref/libref_kernels.so not built (the reference's sources were not present at build)")
    lib = C.CDLL(REF_SO)
    lib.ref_forward.restype = C.c_int
    lib.ref_forward.argtypes = [C.c_char_p, np.ctypeslib.ndpointer(np.uint16, flags="C_CONTIGUOUS"), C.c_int,
                                np.ctypeslib.ndpointer(np.float32, flags="C_CONTIGUOUS")]
    path = models["v3"]
    x, want = _pick_inputs(path)
    ref = np.empty(want.shape, np.float32)
    assert lib.ref_forward(path.encode(), x, x.shape[0], ref) == 0
    got = _engine(path, x)
    assert xlib.xtb_error_word(0) == 0
    _assert_north_star(ref, want, "reference-vs-oracle")
    _assert_north_star(got, ref, "engine-vs-reference")
