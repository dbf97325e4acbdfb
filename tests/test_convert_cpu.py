"""The weight converter (xtagger_b200/convert.py, restating src/tools/export_eva.py) on the CPU: the written file
parses as eva02.bin, its static scales follow the calibration statistics through the SmoothQuant factors, the
folds are exact where the reference's are (position table, fc1 g / x interleave, d = W2 beta), and the quantised
weights dequantise to the smoothed float weights within E4M3 precision."""
import numpy as np
import pytest


@pytest.fixture(scope="module")
def conv(tmp_path_factory):
    from xtagger_b200 import calib as CB
    from xtagger_b200 import convert as CV
    f = CB.synthetic_float(seed=3, nt=64, nl=2)
    rng = np.random.default_rng(4)
    amax = np.abs(rng.standard_normal((2, 4, 2736))).astype(np.float32) * 3 + 0.1
    qkv = np.abs(rng.standard_normal((2, 3, 1024))).astype(np.float32) * 5 + 0.1
    h = np.abs(rng.standard_normal((2, 2736))).astype(np.float32) + 0.05
    h[:, 2730:] = 0
    path = str(tmp_path_factory.mktemp("conv") / "m.bin")
    CV.convert(f, (amax, qkv, h), path, version=4)
    return f, (amax, qkv, h), path


def test_structure_and_folds(conv):
    from xtagger_b200 import model as M
    f, (amax, qkv, h), path = conv
    m = M.read_model(path)
    assert m["version"] == 4 and m["nt"] == 64 and m["nl"] == 2 and not m["head8"]
    pos = f["pos_embed"].copy()
    pos[0] += f["cls_token"]
    pos[1:] += f["patch_embed.bias"]
    np.testing.assert_array_equal(m["pos"], pos)
    np.testing.assert_array_equal(m["pe"][:, :588], f["patch_embed.weight"].astype(np.float16).view(np.uint16))
    assert not m["pe"][:, 588:].any()
    L0 = m["layers"][0]
    d = f["blocks.0.mlp.fc2.weight"] @ f["blocks.0.mlp.norm.bias"]
    np.testing.assert_allclose(L0["d"], d, rtol=1e-5, atol=1e-6)


def test_smoothing_keeps_the_products(conv):
    """LN1 (gamma / s, beta / s) followed by the dequantised Wqkv (columns x s) equals LN1 followed by the original
    Wqkv (q rows x softmax scale x log2 e) up to E4M3 weight precision."""
    from xtagger_b200 import model as M
    f, _, path = conv
    m = M.read_model(path)
    L0 = m["layers"][0]
    rng = np.random.default_rng(5)
    z = rng.standard_normal((16, 1024))
    z = (z - z.mean(1, keepdims=True)) / z.std(1, keepdims=True)
    wq = np.concatenate([f["blocks.0.attn.q_proj.weight"] * (0.125 * np.log2(np.e)), f["blocks.0.attn.k_proj.weight"],
                         f["blocks.0.attn.v_proj.weight"]], 0)
    want = (z * f["blocks.0.norm1.weight"] + f["blocks.0.norm1.bias"]) @ wq.T
    wdq = M.dequant_blocks(L0["qkv"], L0["qkv_s"])
    got = (z * L0["ln1w"] + L0["ln1b"]) @ wdq.T
    # v rows also carry 1 / s of the out-projection smoothing: compare q and k exactly, v up to that factor
    err = np.abs(got[:, :2048] - want[:, :2048]).max() / np.abs(want[:, :2048]).max()
    assert err < 0.05, err


def test_static_scales_follow_calibration(conv):
    from xtagger_b200 import convert as CV
    from xtagger_b200 import model as M
    f, (amax, qkv, h), path = conv
    m = M.read_model(path)
    t = m["table"][0]
    assert np.allclose(t[:4], 1.0)  # v4: the weight scales live in the block arrays
    # q / k scales: calibrated max x 1.25 / 448 (no smoothing on q, k)
    np.testing.assert_allclose(t[8], qkv[0, 0].max() * 1.25 / 448, rtol=1e-6)
    np.testing.assert_allclose(t[9], qkv[0, 1].max() * 1.25 / 448, rtol=1e-6)
    wq = np.concatenate([f["blocks.0.attn.q_proj.weight"] * (0.125 * np.log2(np.e)), f["blocks.0.attn.k_proj.weight"],
                         f["blocks.0.attn.v_proj.weight"]], 0)
    s0 = CV.smooth(amax[0, 0, :1024], wq)
    np.testing.assert_allclose(t[4], (amax[0, 0, :1024] / s0).max() * 1.25 / 448, rtol=1e-5)
