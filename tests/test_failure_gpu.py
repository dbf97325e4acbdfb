"""Failure detection on the GPU without a fault: a kernel's bounded wait on a barrier nothing arrives on runs out
(xtb_selftest_wait), sets its bit in the device error word and returns normally; the host reads the status, the
context keeps running kernels, and the engine reports the affected batch as failed (eva_wait returns NULL, as the
reference's eva_wait does on a device error) until the error word is cleared."""
import time

import numpy as np
import pytest

from tests import _gpu as G

pytestmark = pytest.mark.gpu
SELFTEST_BIT = 16


def test_bounded_wait_reports_and_context_survives(xlib, cuda):
    import torch
    xlib.xtb_error_clear(0)
    assert xlib.xtb_selftest_wait(20000, 1, None) == 0  # arrived: the wait completes
    torch.cuda.synchronize()
    assert xlib.xtb_error_word(0) == 0
    t0 = time.perf_counter()
    assert xlib.xtb_selftest_wait(20000, 0, None) == 0  # nothing arrives: runs out after 20 ms
    torch.cuda.synchronize()
    assert time.perf_counter() - t0 >= 0.019
    assert xlib.xtb_error_word(0) & SELFTEST_BIT
    xlib.xtb_error_clear(0)
    assert xlib.xtb_error_word(0) == 0
    # the context is intact: a kernel runs and matches the oracle
    from oracle import oracle as O
    rng = np.random.default_rng(3)
    x = (rng.standard_normal((64, 1024)) * 2).astype(np.float16).view(np.uint16)
    g, b = np.ones(1024, np.float32), np.zeros(1024, np.float32)
    y = G.zeros((64, 1024), torch.uint8)
    assert xlib.xtb_ln_e4m3(G.P(G.dev(x)), G.P(G.dev(g)), G.P(G.dev(b)), G.P(y), 64, 40.0, None) == 0
    want = np.empty((64, 1024), np.uint8)
    O.lib().or_ln_e4m3(x, g, b, 64, 40.0, want)
    G.assert_e4m3_close(G.host(y), want, 1, 0.99, "ln after the self-test")
    assert xlib.xtb_error_word(0) == 0


def test_engine_reports_a_device_timeout(xlib, cuda, tmp_path):
    import torch
    from xtagger_b200 import model as M
    from xtagger_b200.engine import Engine
    path = M.write_synthetic(str(tmp_path / "m.bin"), seed=5, nl=2, ln_noise=1.0)
    x = M.synthetic_inputs(2, seed=21)
    xlib.xtb_error_clear(0)
    eng = Engine(path, nb=2)
    try:
        good = eng.run(x)
        assert xlib.xtb_selftest_wait(1000, 0, None) == 0  # a wait runs out on the engine's device
        torch.cuda.synchronize()
        with pytest.raises(RuntimeError):
            eng.run(x)
        xlib.xtb_error_clear(0)
        again = eng.run(x)
    finally:
        eng.close()
        xlib.xtb_error_clear(0)
    np.testing.assert_array_equal(good, again)
