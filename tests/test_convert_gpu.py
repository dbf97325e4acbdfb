"""Calibration and conversion end to end on the GPU: a float EVA02-L tagger (random init) runs through the
calibration forward (fp16, the reference's -DEVA_CALIB engine restated in xtagger_b200/calib.py, statistics by this
library's xtb_amax_f16 kernel), is converted to eva02.bin (xtagger_b200/convert.py, the steps of export_eva.py) and
then runs on the FP8 engine. The FP8 scores must track the float model's: the differences are the E4M3 quantisation
of weights and activations the format implies (reported, and bounded in the test)."""
import ctypes as C

import numpy as np
import pytest

from tests import _gpu as G

pytestmark = pytest.mark.gpu


def test_amax_kernel(xlib, cuda):
    import torch
    rng = np.random.default_rng(7)
    x = (rng.standard_normal((3000, 2736)) * rng.uniform(0.1, 50, 2736)).astype(np.float16)
    amax = G.zeros((2736,), torch.float32)
    assert xlib.xtb_amax_f16(G.P(G.dev(x.view(np.uint16))), 2736, 3000, G.P(amax), None) == 0
    np.testing.assert_array_equal(G.host(amax), np.abs(x.astype(np.float32)).max(0))
    # folds into existing values: a larger previous max stays
    big = np.full(2736, 1e4, np.float32)
    amax2 = G.dev(big)
    assert xlib.xtb_amax_f16(G.P(G.dev(x.view(np.uint16))), 2736, 3000, G.P(amax2), None) == 0
    np.testing.assert_array_equal(G.host(amax2), big)


@pytest.mark.parametrize("nl,version", [(2, 4), (24, 3)])
def test_calibrate_convert_run(xlib, cuda, tmp_path, nl, version):
    from xtagger_b200 import calib as CB
    from xtagger_b200 import convert as CV
    from xtagger_b200 import model as M
    from xtagger_b200.engine import Engine
    f = CB.synthetic_float(seed=6, nt=1000, nl=nl)
    fe = CB.FloatEva(f)
    stats = fe.calibrate(M.synthetic_inputs(4, seed=11), batch=4)
    assert all(np.isfinite(s).all() for s in stats)
    path = str(tmp_path / "conv.bin")
    CV.convert(f, stats, path, version=version)
    x = M.synthetic_inputs(3, seed=12)
    want = fe.forward(x)
    eng = Engine(path, nb=3)
    try:
        got = eng.run(x)
    finally:
        eng.close()
    assert xlib.xtb_error_word(0) == 0
    err = np.abs(got - want)
    print(f"nl {nl} v{version}: FP8 engine vs float model: max {err.max():.3e} mean {err.mean():.3e}; "
          f"score spread {want.std():.3e}; correlation {np.corrcoef(got.ravel(), want.ravel())[0, 1]:.5f}")
    assert np.isfinite(got).all()
    # measured on B200: 2 layers (v4) max 2.5e-2 mean 4.6e-3 corr 0.9992; 24 layers (v3) max 4.2e-2 mean 8.9e-3
    # corr 0.997 (score spread ~0.15)
    assert err.mean() <= 0.015 and err.max() <= 0.08
    assert np.corrcoef(got.ravel(), want.ravel())[0, 1] >= 0.99
