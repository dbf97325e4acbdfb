"""The reference's whole FP8 forward (eva_forward, eva.h:252-307: its own kernels from eva_kernels.cu, built by
oracle/Makefile `ref` into oracle/_ref/ and driven by oracle/ref_kernels.cu) on a 24-layer v3 model, next to the
oracle and this library's engine on the same inputs.

On random-init weights the forward is chaotic at the E4M3 quantisation points (a rounding decision that a
floating-point order flips changes an element by 6-12 % and the difference grows layer by layer), so end to end
the three agree only to the scale that two tilings of the oracle's own attention already differ by; each pair is
asserted within 1.5x of that measured sensitivity. Per-kernel agreement is pinned elsewhere (teacher-forced layers,
the reference's attention kernel)."""
import ctypes as C
import os

import numpy as np
import pytest

from tests import _gpu as G

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
REF_SO = os.path.join(ROOT, "oracle", "_ref", "libref_kernels.so")
NT = 10861


@pytest.fixture(scope="module")
def ref():
    if not os.path.exists(REF_SO):
        pytest.skip("oracle/_ref/libref_kernels.so not built (python -c 'import __graft_entry__ as g; g.build()' "
                    "where the reference sources are present)")
    lib = C.CDLL(REF_SO)
    lib.ref_forward.restype = C.c_int
    lib.ref_forward.argtypes = [C.c_char_p, np.ctypeslib.ndpointer(np.uint16, flags="C_CONTIGUOUS"), C.c_int,
                                np.ctypeslib.ndpointer(np.float32, flags="C_CONTIGUOUS")]
    return lib


def test_reference_forward_oracle_and_engine_agree(xlib, ref, cuda, tmp_path):
    from oracle import oracle as O
    from xtagger_b200 import model as M
    from xtagger_b200.engine import Engine
    path = M.write_synthetic(str(tmp_path / "v3.bin"), seed=7, nl=24, version=3, head_fp8=False)
    nimg = 2
    x = np.ascontiguousarray(M.synthetic_inputs(nimg, seed=23))
    r = np.empty((nimg, NT), np.float32)
    assert ref.ref_forward(path.encode(), x, nimg, r) == 0
    want = O.forward(path, x)
    alt = O.forward(path, x, key_tile=128, slice_rows=1)
    eng = Engine(path, nb=nimg)
    try:
        got = eng.run(x)
    finally:
        eng.close()
    G.check_error_word(xlib)
    assert np.isfinite(r).all() and np.isfinite(got).all()
    floor_max, floor_mean = float(np.abs(alt - want).max()), float(np.abs(alt - want).mean())
    pairs = {"reference-vs-oracle": (r, want), "engine-vs-reference": (got, r), "engine-vs-oracle": (got, want)}
    for name, (a, b) in pairs.items():
        e = np.abs(a - b)
        print(f"{name}: max {e.max():.2e} mean {e.mean():.2e} (oracle tiling sensitivity max {floor_max:.2e} "
              f"mean {floor_mean:.2e})")
        assert e.max() <= max(2e-3, 1.5 * floor_max), name
        assert e.mean() <= max(2e-4, 1.5 * floor_mean), name
