"""The reference's own PixAI forward (px_forward, px.h:115-190: its kernels from px_kernels.cu and kern_common.cuh,
built by oracle/Makefile `ref` into oracle/_ref/ and driven by oracle/ref_px.cu) on a reduced pixai.bin v3 (one
windowed and one global block), next to the oracle (oracle/px_oracle.c) and this library's px_* engine on the same
inputs. This pins the PixAI oracle to the reference's code: each pair agrees within 1.5x of the sensitivity two
tilings of the oracle's own attention already show (the forward is chaotic at the E4M3 quantisation points)."""
import ctypes as C
import os

import numpy as np
import pytest

from tests import _gpu as G

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
REF_SO = os.path.join(ROOT, "oracle", "_ref", "libref_px.so")


@pytest.fixture(scope="module")
def ref():
    if not os.path.exists(REF_SO):
        pytest.skip("oracle/_ref/libref_px.so not built (python -c 'import __graft_entry__ as g; g.build()' where the "
                    "reference sources are present)")
    lib = C.CDLL(REF_SO)
    lib.ref_px_forward.restype = C.c_int
    lib.ref_px_forward.argtypes = [C.c_char_p, np.ctypeslib.ndpointer(np.uint16, flags="C_CONTIGUOUS"), C.c_int,
                                   np.ctypeslib.ndpointer(np.float32, flags="C_CONTIGUOUS"), C.c_void_p]
    return lib


@pytest.mark.parametrize("nl,gmask", [(2, 2), (8, 0)])
def test_reference_px_forward_oracle_and_engine_agree(xlib, ref, cuda, tmp_path, nl, gmask):
    from oracle import oracle as O
    from xtagger_b200 import pixai as P
    from xtagger_b200.pxengine import PxEngine
    path = P.write_synthetic(str(tmp_path / "px.bin"), seed=13, nt=500, nl=nl, gmask=gmask)
    nimg = 2
    x = np.ascontiguousarray(P.synthetic_inputs(nimg, seed=24))
    r = np.empty((nimg, 500), np.float32)
    ro = np.empty((nimg, 1024), np.uint16)
    assert ref.ref_px_forward(path.encode(), x, nimg, r, ro.ctypes.data_as(C.c_void_p)) == 0
    want, wo = O.px_forward(path, x, want_o=True)
    alt = O.px_forward(path, x, key_tile=128, slice_rows=1)
    eng = PxEngine(path, nb=nimg)
    try:
        got = eng.run(x)
    finally:
        eng.close()
    G.check_error_word(xlib)
    assert np.isfinite(r).all() and np.isfinite(got).all()
    floor = float(np.abs(alt - want).max())
    pairs = {"reference-vs-oracle": (r, want), "engine-vs-reference": (got, r), "engine-vs-oracle": (got, want)}
    for name, (a, b) in pairs.items():
        e = float(np.abs(a - b).max())
        print(f"nl {nl}: {name}: max {e:.2e} (oracle tiling sensitivity {floor:.2e})")
        assert e <= max(2e-3, 1.5 * floor), name
    g, w = G.f16(ro), G.f16(wo)
    assert np.corrcoef(g.ravel(), w.ravel())[0, 1] > 0.9999
