"""PixAI tagger (ViTDet-L at 1008^2) on the GPU against the CPU oracle's restatement of the reference's FP8 engine
(oracle/px_oracle.c: px.h + px_kernels.cu + kern_common.cuh): the tcgen05 attention over 576-token windows and
5184-token global sequences, and the whole engine (px_open / px_submit / px_wait) on a reduced model with one
windowed and one global block."""
import numpy as np
import pytest

from tests import _gpu as G

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def O():
    from oracle import oracle
    return oracle


@pytest.mark.parametrize("L,nseq,peaked", [(576, 9, 0), (576, 9, 1), (5184, 1, 0), (5184, 1, 1)])
def test_px_attention(xlib, cuda, O, L, nseq, peaked):
    import torch
    rng = np.random.default_rng(40 + L + peaked)
    shape = (nseq, 16, L, 64)
    sd = 3.0 if peaked else 1.0   # peaked: large scores, so lazy rescales and dead tiles occur
    q = O.e4m3(rng.standard_normal(shape, dtype=np.float32) * 60 * sd)
    k = O.e4m3(rng.standard_normal(shape, dtype=np.float32) * 60 * sd)
    v = O.e4m3(rng.standard_normal(shape, dtype=np.float32) * 100)
    sinv = (0.8 / 448) * (4.0 / 448)
    vo = 0.9
    want = np.empty((nseq * L, 1024), np.uint8)
    O.lib().or_px_attention(q, k, v, nseq, L, sinv, vo, 64, 16, want)
    out = G.zeros((nseq * L, 1024), torch.uint8)
    assert xlib.xtb_px_attention(G.P(G.dev(q)), G.P(G.dev(k)), G.P(G.dev(v)), nseq, L, G.P(out), sinv, vo, None) == 0
    G.check_error_word(xlib)
    G.assert_attention_close(G.host(out), want, f"px attention L={L}")


@pytest.fixture(scope="module")
def px_model(tmp_path_factory):
    from xtagger_b200 import pixai as P
    d = tmp_path_factory.mktemp("px")
    return P.write_synthetic(str(d / "px_l2.bin"), seed=3, nt=300, nl=2, gmask=2)


def test_px_engine_matches_oracle(xlib, cuda, O, px_model):
    from xtagger_b200 import pixai as P
    from xtagger_b200.pxengine import PxEngine
    x = P.synthetic_inputs(2, seed=4)
    eng = PxEngine(px_model, nb=2)
    try:
        got = eng.run(x)
        o = eng.head_input(2)
        assert eng.launches_per_forward() == 2 + 7 * 2 + 5
    finally:
        eng.close()
    want, wo = O.px_forward(px_model, x, want_o=True)                           # the reference's attention tiling
    alt, ao = O.px_forward(px_model, x, key_tile=128, slice_rows=1, want_o=True)  # another tiling, same arithmetic
    floor = float(np.abs(alt - want).max())
    err = float(np.abs(got - want).max())
    assert np.isfinite(got).all()
    assert err <= max(2e-3, 1.5 * floor), f"scores: max |diff| {err:.3e} (oracle tiling noise floor {floor:.3e})"
    # the head vector: FP8 rounding flips inside the forward move it by about as much as another attention tiling
    g, w, a = G.f16(o), G.f16(wo), G.f16(ao)
    scale = float(np.abs(w).max())
    err_o, floor_o = float(np.abs(g - w).max()), float(np.abs(a - w).max())
    assert err_o <= max(2e-3 * scale, 2.0 * floor_o), f"o: max |diff| {err_o:.3e}, tiling floor {floor_o:.3e}"
    assert np.corrcoef(g.ravel(), w.ravel())[0, 1] > 0.9999


def test_px_engine_submit_slots(xlib, cuda, px_model):
    """Every slot returns the same scores for the same inputs; adjacent pool inputs go in one copy."""
    from xtagger_b200 import pixai as P
    from xtagger_b200.pxengine import PxEngine
    pool = P.synthetic_inputs(3, seed=5)
    eng = PxEngine(px_model, nb=3, pool=pool)
    try:
        first = eng.run([pool[i] for i in range(3)], buf=0)
        for b in range(1, 4):
            eng.submit(b, [pool[i] for i in range(3)])
        for b in range(1, 4):
            assert np.array_equal(eng.wait(b, 3), first)
        part = eng.run([pool[1]], buf=2)
        assert np.array_equal(part[0], first[1])
    finally:
        eng.close()


def test_px_fc1_gelu(xlib, cuda, O):
    """fc1 GEMM + bias + exact-erf GELU + rs -> E4M3 against the oracle (libm erff): codes equal or one step apart
    (a product on a rounding boundary), at least 99 % identical."""
    import torch
    rng = np.random.default_rng(44)
    rows = 1000                                   # a partial last row tile
    h = O.e4m3(rng.standard_normal((rows, 1024), dtype=np.float32) * 60)
    w = O.e4m3(rng.standard_normal((4736, 1024), dtype=np.float32) * 100)
    wscale, ascale = 0.02 / 100, 1.0 / 60
    b1 = (rng.standard_normal(4736) * 0.5).astype(np.float32)
    rs = (40 + 20 * rng.random(4736)).astype(np.float32)
    acc = np.empty((rows, 4736), np.float32)
    O.lib().or_gemm_e4m3(h, rows, 1024, w, 4736, np.ones((37, 8), np.float32), np.float32(wscale) * np.float32(ascale), acc)
    want = np.empty((rows, 4736), np.uint8)
    O.lib().or_px_fc1_epilogue(acc, rows, b1, rs, want)
    out = G.zeros((rows, 4736), torch.uint8)
    assert xlib.xtb_px_fc1(G.P(G.dev(h)), rows, G.P(G.dev(w)), wscale, ascale, G.P(G.dev(b1)), G.P(G.dev(rs)),
                           G.P(out), None) == 0
    G.check_error_word(xlib)
    G.assert_e4m3_close(G.host(out), want, 1, 0.99, "px fc1")


def test_px_full_model_batch_invariance(xlib, cuda, O, tmp_path_factory):
    """The full PixAI model (32 blocks, 30877 tags) at batch 8: bit-identical scores for the same image at two batch
    positions and alone, and image 0 against the oracle within its tiling noise floor."""
    from xtagger_b200 import pixai as P
    from xtagger_b200.pxengine import PxEngine
    d = str(tmp_path_factory.mktemp("pxfull"))
    path = P.cached_synthetic(d, seed=0, nt=30877)
    x = P.synthetic_inputs(8, seed=1)
    x[7] = x[2]
    eng = PxEngine(path, nb=8)
    try:
        got = eng.run(x)
    finally:
        eng.close()
    one = PxEngine(path, nb=1)
    try:
        alone = one.run(x[2:3])
    finally:
        one.close()
    assert xlib.xtb_error_word(0) == 0
    assert np.isfinite(got).all()
    assert np.array_equal(got[7], got[2]) and np.array_equal(alone[0], got[2])
    want = O.px_forward(path, x[:1])
    alt = O.px_forward(path, x[:1], key_tile=128, slice_rows=1)
    floor = float(np.abs(alt - want).max())
    err = float(np.abs(got[:1] - want).max())
    assert err <= max(2e-3, 1.5 * floor), f"image 0: {err:.3e} against floor {floor:.3e}"
