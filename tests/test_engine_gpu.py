"""The engine (eva_open / eva_submit / eva_wait ...) end to end against the oracle's whole forward, plus a
teacher-forced per-layer check of every kernel in forward order.

Tolerances. Teacher-forced (each GPU step and the oracle fed the same GPU intermediate): E4M3 outputs identical
or one representable value apart (a rounding decision at a boundary; attention two), fp16 within 1e-2 relative.
Whole forward: the reference's attention quantises P to E4M3 (kern_common.cuh:509-513) after a lazily refreshed
running max (RESCALE, kern_common.cuh:480-493), so its result depends on the key tiling; on random-init weights
(flat attention, ~4 % relative E4M3 noise on every attention output, coherent across tokens) two valid tilings
of the same semantics -- the reference's 64-key tiles and this library's 128-key tiles, both restated by the
oracle -- already differ by ~2e-2 in final scores. End-to-end parity is therefore asserted against that measured
noise floor of the semantics (max and mean |score difference| within 1.5x of oracle64-vs-oracle128), and the
above-threshold tag sets must agree outside a band of that width. The north-star 2e-3 score tolerance holds
wherever the semantics themselves are stable to 2e-3.
"""
import os

import numpy as np
import pytest

from tests import _gpu as G

pytestmark = pytest.mark.gpu

THRESH = 0.5


def _mx_kinds():
    """Projection kinds the engine runs on the block-scaled MMA for a model whose block scales are all powers of two:
    its default (all four: QKV, out-projection, fc1, fc2), or the XTB_MX / XTB_MX_KINDS overrides the engine reads
    from the environment."""
    if os.environ.get("XTB_MX", "1").startswith("0"):
        return 0
    return int(os.environ.get("XTB_MX_KINDS", "F"), 16) & 0xF


@pytest.fixture(scope="module")
def models(tmp_path_factory):
    from xtagger_b200 import model as M
    d = str(tmp_path_factory.mktemp("models"))
    return {
        "v4_l2_h8": M.write_synthetic(os.path.join(d, "a.bin"), seed=5, nl=2, ln_noise=1.0, head_fp8=True),
        "v4_l2_h16": M.write_synthetic(os.path.join(d, "b.bin"), seed=6, nl=2, ln_noise=1.0, head_fp8=False),
        "v4_l24_h8": M.write_synthetic(os.path.join(d, "c.bin"), seed=0, nl=24, head_fp8=True),
        "v3_l24": M.write_synthetic(os.path.join(d, "d.bin"), seed=7, nl=24, version=3, head_fp8=False),
        # 2:4-pruned projections (config 5): the engine runs them on the sparse tensor-core kernels
        "v4_l2_p": M.write_synthetic(os.path.join(d, "e.bin"), seed=8, nl=2, ln_noise=1.0, head_fp8=True, prune24=True),
        "v4_l24_p": M.write_synthetic(os.path.join(d, "f.bin"), seed=9, nl=24, head_fp8=True, prune24=True),
        # the reference's format pruned as prune24.py does: the sparse kernels without block-scale promotion
        "v3_l24_p": M.write_synthetic(os.path.join(d, "g.bin"), seed=10, nl=24, version=3, head_fp8=False,
                                      prune24=True),
        # power-of-two block scales: fc1 on the tensor core's own block scaling
        "v4_l2_pow2": M.write_synthetic(os.path.join(d, "h.bin"), seed=11, nl=2, ln_noise=1.0, head_fp8=True, pow2=True),
        "v4_l24_pow2": M.write_synthetic(os.path.join(d, "i.bin"), seed=12, nl=24, head_fp8=True, pow2=True),
    }


@pytest.mark.parametrize("name,nimg", [("v4_l2_h8", 3), ("v4_l2_h16", 2), ("v4_l24_h8", 1), ("v3_l24", 1),
                                       ("v4_l2_p", 3), ("v4_l24_p", 1), ("v3_l24_p", 1), ("v4_l2_pow2", 3),
                                       ("v4_l24_pow2", 1)])
def test_forward_matches_oracle(xlib, cuda, models, name, nimg):
    from oracle import oracle as O
    from xtagger_b200 import model as M
    from xtagger_b200.engine import Engine
    x = M.synthetic_inputs(nimg, seed=21)
    want = O.forward(models[name], x)                     # the reference's attention: 64-key tiles, 16-row slices
    alt = O.forward(models[name], x, key_tile=128, slice_rows=1)   # another tiling of the same arithmetic
    floor_max = float(np.abs(alt - want).max())
    floor_mean = float(np.abs(alt - want).mean())
    if name.endswith("_p"):
        os.environ["XTB_SPARSE"] = "1"  # pruned models: the sparse kernels (opt-in)
    try:
        eng = Engine(models[name], nb=max(nimg, 2))
        try:
            got = eng.run(x)
            assert eng.sparse_kinds() == (15 if name.endswith("_p") else 0)
            assert eng.block_scale_kinds() == (_mx_kinds() if name.endswith("_pow2") else 0)
        finally:
            eng.close()
    finally:
        os.environ.pop("XTB_SPARSE", None)
    assert xlib.xtb_error_word(0) == 0
    assert np.isfinite(got).all()
    err = np.abs(got - want)
    print(f"{name}: engine-vs-oracle max {err.max():.2e} mean {err.mean():.2e}; "
          f"oracle tiling sensitivity max {floor_max:.2e} mean {floor_mean:.2e}")
    tol_max = max(2e-3, 1.5 * floor_max)
    assert err.max() <= tol_max
    assert err.mean() <= max(2e-4, 1.5 * floor_mean)
    band = np.abs(want - THRESH) > tol_max
    assert ((got > THRESH) == (want > THRESH))[band].all()


def test_sparse_engine_matches_dense_engine(xlib, cuda, models):
    """The same pruned 2-layer model through the sparse kernels and (XTB_SPARSE=0) through the dense ones: the same
    products in another fp32 summation order. A sum that lands on the other side of an E4M3 rounding boundary is
    carried through the attention like any other rounding difference, so the two engines are held to half of the
    semantics' own tiling sensitivity (oracle 64-key tiles vs 128-key tiles on the same inputs), a third of the
    bound the oracle comparisons allow."""
    from oracle import oracle as O
    from xtagger_b200 import model as M
    from xtagger_b200.engine import Engine
    x = M.synthetic_inputs(3, seed=25)
    floor = np.abs(O.forward(models["v4_l2_p"], x) - O.forward(models["v4_l2_p"], x, key_tile=128, slice_rows=1))
    out = {}
    for mode in ("1", "0"):
        os.environ["XTB_SPARSE"] = mode
        try:
            eng = Engine(models["v4_l2_p"], nb=3)
            try:
                out[mode] = eng.run(x)
                assert eng.sparse_kinds() == (15 if mode == "1" else 0)
            finally:
                eng.close()
        finally:
            del os.environ["XTB_SPARSE"]
    err = np.abs(out["1"] - out["0"])
    print(f"sparse vs dense engine: max {err.max():.2e} mean {err.mean():.2e}; "
          f"tiling sensitivity max {floor.max():.2e} mean {floor.mean():.2e}")
    assert err.max() <= max(2e-3, 0.5 * floor.max()) and err.mean() <= max(2e-4, 0.5 * floor.mean())


def test_teacher_forced_layers(xlib, cuda, models):
    """Each kernel, in forward order over a 2-layer model, against the oracle on the GPU's own intermediates."""
    import torch
    from oracle import oracle as O
    from xtagger_b200 import model as M
    m = M.read_model(models["v4_l2_h8"])
    nimg, rows = 2, 2 * 1025
    lib = O.lib()
    x_in = M.synthetic_inputs(nimg, seed=24)
    c = np.ascontiguousarray
    x = G.zeros((rows, 1024), torch.int16)
    assert xlib.xtb_patch_embed(G.P(G.dev(x_in)), nimg, G.P(G.dev(m["pe"])), G.P(G.dev(m["pos"])), G.P(x), None) == 0
    want = np.empty((rows, 1024), np.uint16)
    lib.or_patch_embed(x_in, nimg, c(m["pe"]), c(m["pos"]), want)
    G.assert_f16_close(G.host(x).view(np.uint16), want, 1e-2, "patch")
    cs = c(m["cs"])
    for i, L in enumerate(m["layers"]):
        xh = G.host(x).view(np.uint16).copy()
        h = G.zeros((rows, 1024), torch.uint8)
        assert xlib.xtb_ln_e4m3(G.P(x), G.P(G.dev(L["ln1w"])), G.P(G.dev(L["ln1b"])), G.P(h), rows,
                                float(1 / L["adq"][0]), None) == 0
        w = np.empty((rows, 1024), np.uint8)
        lib.or_ln_e4m3(xh, c(L["ln1w"]), c(L["ln1b"]), rows, float(1 / L["adq"][0]), w)
        G.assert_e4m3_close(G.host(h), w, 1, 0.999, f"L{i} ln1")
        hh = G.host(h).copy()
        shp, shv = (nimg, 16, 1152, 64), (nimg, 16, 1152, 64)
        q8, k8, vt8 = G.zeros(shp, torch.uint8), G.zeros(shp, torch.uint8), G.zeros(shv, torch.uint8)
        assert xlib.xtb_qkv(G.P(h), rows, G.P(G.dev(L["qkv"])), G.P(G.dev(L["qkv_s"])), float(L["adq"][0]), G.P(q8),
                            G.P(k8), G.P(vt8), G.P(G.dev(cs)), float(L["cq"]), float(L["ck"]), float(L["cv"]), None) == 0
        acc = O.gemm_e4m3(hh, c(L["qkv"]), c(L["qkv_s"]), float(L["adq"][0]))
        qw, kw, vw = np.zeros(shp, np.uint8), np.zeros(shp, np.uint8), np.zeros(shv, np.uint8)
        lib.or_qkv_epilogue(acc, rows, cs, float(L["cq"]), float(L["ck"]), float(L["cv"]), qw, kw, vw)
        qg, kg, vg = G.host(q8).copy(), G.host(k8).copy(), G.host(vt8).copy()
        for nm, g_, w_ in (("q", qg, qw), ("k", kg, kw), ("v", vg, vw)):
            G.assert_e4m3_close(g_, w_, 1, 0.999, f"L{i} {nm}")
        att = G.zeros((rows, 1024), torch.uint8)
        assert xlib.xtb_attention(G.P(q8), G.P(k8), G.P(vt8), nimg, G.P(att), float(L["sinv"]), float(L["vo"]),
                                  None) == 0
        aw = np.empty((rows, 1024), np.uint8)
        lib.or_attention(qg, kg, vg, nimg, float(L["sinv"]), float(L["vo"]), 64, 16, aw)
        G.assert_attention_close(G.host(att), aw, f"L{i} attention")
        ag = G.host(att).copy()
        assert xlib.xtb_oproj(G.P(att), rows, G.P(G.dev(L["o"])), G.P(G.dev(L["o_s"])), float(L["adq"][1]), G.P(x),
                              None) == 0
        w = xh.copy()
        lib.or_resid_add(w, O.gemm_e4m3(ag, c(L["o"]), c(L["o_s"]), float(L["adq"][1])), rows)
        G.assert_f16_close(G.host(x).view(np.uint16), w, 1e-2, f"L{i} oproj")
        xh = G.host(x).view(np.uint16).copy()
        assert xlib.xtb_ln_e4m3(G.P(x), G.P(G.dev(L["ln2w"])), G.P(G.dev(L["ln2b"])), G.P(h), rows,
                                float(1 / L["adq"][2]), None) == 0
        w = np.empty((rows, 1024), np.uint8)
        lib.or_ln_e4m3(xh, c(L["ln2w"]), c(L["ln2b"]), rows, float(1 / L["adq"][2]), w)
        G.assert_e4m3_close(G.host(h), w, 1, 0.999, f"L{i} ln2")
        hh = G.host(h).copy()
        h8 = G.zeros((rows, 2736), torch.uint8)
        stat = G.zeros((43, rows, 2), torch.float32)
        assert xlib.xtb_fc1(G.P(h), rows, G.P(G.dev(L["w12"])), G.P(G.dev(L["w12_s"])), float(L["adq"][2]), G.P(h8),
                            G.P(stat), G.P(G.dev(L["rs"])), None) == 0
        acc = O.gemm_e4m3(hh, c(L["w12"]), c(L["w12_s"]), float(L["adq"][2]))
        w = np.empty((rows, 2736), np.uint8)
        s, q = np.empty(rows), np.empty(rows)
        lib.or_fc1_epilogue(acc, rows, c(L["rs"]), w, s, q)
        G.assert_e4m3_close(G.host(h8), w, 1, 0.999, f"L{i} h8")
        st = G.host(stat).astype(np.float64).sum(0)
        np.testing.assert_allclose(st[:, 1], q, rtol=1e-3)
        h8g = G.host(h8).copy()
        assert xlib.xtb_fc2(G.P(h8), rows, G.P(G.dev(L["w2"])), G.P(G.dev(L["w2_s"])), float(L["adq"][3]), G.P(x),
                            G.P(stat), G.P(G.dev(L["c"])), G.P(G.dev(L["d"])), None) == 0
        w = xh.copy()
        lib.or_fc2_epilogue(w, O.gemm_e4m3(h8g, c(L["w2"]), c(L["w2_s"]), float(L["adq"][3])), rows, c(st[:, 0]),
                            c(st[:, 1]), c(L["c"]), c(L["d"]))
        G.assert_f16_close(G.host(x).view(np.uint16), w, 1e-2, f"L{i} fc2")
    G.check_error_word(xlib)


def test_submit_ring_and_adjacent_inputs(xlib, cuda, models):
    """Several slots in flight; inputs adjacent in a pool go in one copy; an image's scores do not depend on its
    position in the batch or on the other images."""
    from xtagger_b200 import model as M
    from xtagger_b200.engine import Engine
    pool = M.synthetic_inputs(6, seed=22)
    eng = Engine(models["v4_l2_h8"], nb=3, pool=pool)
    try:
        eng.submit(0, [pool[0], pool[1], pool[2]])
        eng.submit(1, [pool[3], pool[5], pool[4]])
        a, b = eng.wait(0, 3), eng.wait(1, 3)
        c = eng.run([pool[5]], buf=2)
    finally:
        eng.close()
    np.testing.assert_array_equal(c[0], b[1])
    assert not np.array_equal(a[0], a[1])


def test_head_put_get(xlib, cuda, models):
    from xtagger_b200 import model as M
    from xtagger_b200.engine import Engine
    x = M.synthetic_inputs(2, seed=23)
    eng = Engine(models["v4_l2_h16"], nb=2, extra=3)
    try:
        assert eng.nt == 10861 + 3
        base = eng.run(x)
        assert np.all(base[:, 10861:] < 1e-6)          # unwritten extra rows never fire (bias -16)
        w, b = eng.head_get()
        assert w.shape == (10861, 1024)
        eng.head_put(10861, w[7], float(b[7]))         # copy tag 7 into the first extra row
        got = eng.run(x, buf=1)
        pn = eng.hpn(1, 2)
    finally:
        eng.close()
    np.testing.assert_array_equal(got[:, 10861], got[:, 7])
    assert pn is not None and np.isfinite(pn.view(np.float16)).all()


def test_head_put_fp8_head(xlib, cuda, models):
    """FP8 head: a row written with eva_head_put is quantised with its block's scales; copying a row onto itself
    (after a read-back) reproduces the same scores."""
    from xtagger_b200 import model as M
    from xtagger_b200.engine import Engine
    x = M.synthetic_inputs(2, seed=25)
    eng = Engine(models["v4_l2_h8"], nb=2, extra=1)
    try:
        base = eng.run(x)
        w, b = eng.head_get()
        eng.head_put(3, w[3], float(b[3]))             # fp16 read-back -> E4M3 with the same block scales
        again = eng.run(x, buf=1)
    finally:
        eng.close()
    np.testing.assert_array_equal(again[:, 3], base[:, 3])


def test_full_size_batch_invariance(xlib, cuda, tmp_path_factory):
    """Config 3 at full size (the bench's 24-layer model with power-of-two block scales, batch 64): an image's
    scores do not depend on its batch neighbours or the batch size (bit-identical at positions 5 and 63 of a batch
    of 64 and alone), and image 0 matches the oracle within the tiling noise floor."""
    from oracle import oracle as O
    from xtagger_b200 import model as M
    from xtagger_b200.engine import Engine
    d = str(tmp_path_factory.mktemp("full"))
    path = M.cached_synthetic(d, seed=0, nt=10861, nl=24, version=4, head_fp8=True, pow2=True)
    x = M.synthetic_inputs(64, seed=1)
    x[63] = x[5]
    eng = Engine(path, nb=64)
    try:
        got = eng.run(x)
        assert eng.block_scale_kinds() == _mx_kinds()
    finally:
        eng.close()
    one = Engine(path, nb=1)
    try:
        alone = one.run(x[5:6])
    finally:
        one.close()
    assert xlib.xtb_error_word(0) == 0
    assert np.isfinite(got).all()
    assert np.array_equal(got[63], got[5])
    assert np.array_equal(alone[0], got[5])
    want = O.forward(path, x[:1])
    alt = O.forward(path, x[:1], key_tile=128, slice_rows=1)
    floor = float(np.abs(alt - want).max())
    err = float(np.abs(got[:1] - want).max())
    assert err <= max(2e-3, 1.5 * floor), f"image 0: {err:.3e} against floor {floor:.3e}"
