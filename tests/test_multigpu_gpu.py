"""The engines on two GPUs of one process: eva_open_ex with a device list (one replica, stream and graph per device, a
submit's inputs split into contiguous shards, the scores gathered into one host slot) and px_open_multi (one PixAI
engine replica per device, the same split and gather). Images are independent units and every kernel keeps rows
and images independent, so each image's scores must be bit-identical to a single-device engine's on the same
inputs; distinct images make a misplaced or duplicated shard row visible. Submits of the full batch and of fewer
inputs than the batch (a partial last shard, an idle second device) are both checked. Skipped below two devices."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def two_gpus(cuda):
    import torch
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two CUDA devices")
    return (0, 1)


def test_eva_two_devices_bit_identical(xlib, two_gpus, tmp_path):
    from xtagger_b200 import model as M
    from xtagger_b200.engine import Engine
    path = M.write_synthetic(str(tmp_path / "m.bin"), seed=13, nl=4, ln_noise=1.0, head_fp8=True, pow2=True)
    x = M.structured_inputs(16, seed=5)
    one = Engine(path, devices=(0,), nb=16)
    try:
        want = one.run(x)
        want11 = one.run(x[:11], buf=1)
    finally:
        one.close()
    two = Engine(path, devices=two_gpus, nb=16)
    try:
        got = two.run(x)
        got11 = two.run(x[:11], buf=1)        # shard 0 full (8), shard 1 partial (3)
        got5 = two.run(x[:5], buf=2)          # shard 0 partial, shard 1 idle
    finally:
        two.close()
    assert xlib.xtb_error_word(0) == 0 and xlib.xtb_error_word(1) == 0
    assert len({row.tobytes() for row in want}) == 16, "inputs should give distinct scores"
    assert np.array_equal(got, want), f"{int((got != want).any(1).sum())} of 16 images differ"
    assert np.array_equal(got11, want11) and np.array_equal(got11, want[:11])
    assert np.array_equal(got5, want[:5])


def test_pixai_two_devices_bit_identical(xlib, two_gpus, tmp_path):
    from xtagger_b200 import pixai as P
    from xtagger_b200.pxengine import PxEngine
    path = P.write_synthetic(str(tmp_path / "px.bin"), seed=3, nt=300, nl=2, gmask=2)
    x = P.synthetic_inputs(4, seed=8)
    one = PxEngine(path, device=0, nb=4)
    try:
        want = one.run(x)
    finally:
        one.close()
    two = PxEngine(path, nb=4, devices=two_gpus)
    try:
        got = two.run(x)
        got3 = two.run(x[:3], buf=1)
    finally:
        two.close()
    assert xlib.xtb_error_word(0) == 0 and xlib.xtb_error_word(1) == 0
    assert len({row.tobytes() for row in want}) == 4
    assert np.array_equal(got, want), f"{int((got != want).any(1).sum())} of 4 images differ"
    assert np.array_equal(got3, want[:3])
