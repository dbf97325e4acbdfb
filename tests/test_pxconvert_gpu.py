"""PixAI calibration and conversion end to end on the GPU: a float ViTDet-L tagger (random init, one windowed and
one global block) runs through the calibration forward (fp16, the reference's -DPX_CALIB engine restated in
xtagger_b200/pxconvert.py, statistics by this library's xtb_amax_f16 kernel), is converted to pixai.bin v3 (the steps
of export_pixai.py: SmoothQuant folds, per-tensor E4M3, the attention-pool head folded) and then runs on the FP8
px_* engine. The FP8 scores must track the float model's: the differences are the E4M3 quantisation of weights and
activations the format implies (reported, and bounded in the test)."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def test_px_calibrate_convert_run(xlib, cuda, tmp_path):
    from oracle import oracle as O
    from xtagger_b200 import pixai as P
    from xtagger_b200 import pxconvert as PC
    from xtagger_b200.pxengine import PxEngine
    f = PC.synthetic_float(seed=6, nt=1000, nl=2, glob=[1])
    fp = PC.FloatPx(f)
    stats = fp.calibrate(P.synthetic_inputs(2, seed=11), batch=2)
    assert all(np.isfinite(s).all() for s in stats)
    assert (stats[0][:, :3, 1024:] == 0).all() and (stats[0][:, 3] > 0).all()
    path = str(tmp_path / "px_conv.bin")
    PC.convert(f, stats, path)
    hdr = np.fromfile(path, np.uint32, 6)
    assert hdr[4] == 2 and hdr[5] == 2          # 2 blocks, block 1 global
    x = P.synthetic_inputs(2, seed=12)
    want = fp.forward(x)
    eng = PxEngine(path, nb=2)
    try:
        got = eng.run(x)
    finally:
        eng.close()
    assert xlib.xtb_error_word(0) == 0
    ref = O.px_forward(path, x)                 # the converted file on the oracle: the engine's own parity
    err, perr = np.abs(got - want), np.abs(got - ref)
    corr = np.corrcoef(got.ravel(), want.ravel())[0, 1]
    print(f"FP8 engine vs float model: max {err.max():.3e} mean {err.mean():.3e}, score spread {want.std():.3e}, "
          f"correlation {corr:.5f}; vs oracle on the converted file: max {perr.max():.3e}")
    assert np.isfinite(got).all()
    assert perr.max() <= 2e-3
    assert err.mean() <= 0.015 and err.max() <= 0.08
    assert corr >= 0.99
