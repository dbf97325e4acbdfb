"""The CPU oracle pinned against the reference's own code (golden vectors from tests/golden/make_golden.py) and
against independent numpy statements of the same arithmetic. No GPU needed."""
import hashlib
import json
import os

import numpy as np
import pytest

HERE = os.path.dirname(os.path.abspath(__file__))
GOLD = os.path.join(HERE, "golden")


@pytest.fixture(scope="module")
def O():
    from oracle import oracle
    oracle.lib()
    return oracle


def test_e4m3_encode_matches_reference_quantiser(O):
    """or_e4m3 == export_eva.py's fp8() (clip, ml_dtypes float8_e4m3fn), bit for bit, over every code, every tie
    between neighbouring codes (round half to even), saturation, subnormals and signed zero."""
    g = np.load(os.path.join(GOLD, "golden_e4m3.npz"))
    got = O.e4m3(g["x"])
    bad = np.nonzero(got != g["codes"])[0]
    assert bad.size == 0, f"{bad.size} mismatches, first x={g['x'][bad[:5]]} got={got[bad[:5]]} want={g['codes'][bad[:5]]}"


def test_e4m3_saturates_and_keeps_nan(O):
    x = np.array([1e6, -1e6, np.inf, -np.inf, np.nan, 449, 464, 480], np.float32)
    got = O.e4m3(x)
    assert list(got[:4]) == [0x7E, 0xFE, 0x7E, 0xFE]          # SATFINITE
    assert got[4] & 0x7F == 0x7F                               # NaN stays NaN
    assert list(got[5:]) == [0x7E, 0x7E, 0x7E]


def test_e4m3_decode_all_codes(O):
    import ml_dtypes
    codes = np.arange(256, dtype=np.uint8)
    want = codes.view(ml_dtypes.float8_e4m3fn).astype(np.float32)
    got = O.e4m3_dec(codes)
    assert np.array_equal(np.isnan(got), np.isnan(want))
    fin = ~np.isnan(want)
    assert np.array_equal(got[fin], want[fin])


def test_fp16_codec(O):
    rng = np.random.default_rng(3)
    x = np.concatenate([rng.standard_normal(100000).astype(np.float32) * s for s in (1e-6, 1e-3, 1, 100, 3e4)])
    y = np.empty(x.size, np.uint16)
    O.lib().or_f2h_n(x, y, x.size)
    assert np.array_equal(y, x.astype(np.float16).view(np.uint16))


def test_interleave_matches_reference():
    from xtagger_b200 import model as M
    perm = np.load(os.path.join(GOLD, "golden_interleave.npz"))["perm"]
    rows = np.arange(2 * 2736, dtype=np.int64)[:, None]
    assert np.array_equal(M.interleave_gx(rows)[:, 0], perm)


def test_prune24_matches_reference(O, tmp_path):
    """or_prune24 reproduces src/tools/prune24.py's 2:4 selection bit for bit (Wanda and magnitude scores, ties to
    the lower index, NaN codes as zero) on every block-GEMM matrix of a seeded random v3 blob."""
    from tests.golden.make_golden import blob_matrices, random_v3_blob
    g = json.load(open(os.path.join(GOLD, "golden_prune24.json")))
    src = str(tmp_path / "rand.bin")
    random_v3_blob(src, seed=g["seed"], nt=g["nt"])
    shapes = {"qkv": (3072, 1024), "oproj": (1024, 1024), "fc1": (5472, 1024), "fc2": (1024, 2736)}
    mats = blob_matrices(src)
    for mode, wanda in (("wanda", 1), ("mag", 0)):
        for name, i, b in mats:
            w = np.frombuffer(b, np.uint8).copy()
            n, k = shapes[name]
            O.lib().or_prune24(w, n, k, wanda)
            assert hashlib.sha256(w.tobytes()).hexdigest() == g["digests"][mode][f"{name}.{i}"], (mode, name, i)
        # and the 2:4 property itself
    wq = np.frombuffer(mats[0][2], np.uint8).copy()
    O.lib().or_prune24(wq, 3072, 1024, 0)
    assert ((wq.reshape(3072, 256, 4) != 0).sum(-1) <= 2).all()


def test_gemm_blockscaled_matches_numpy(O):
    from xtagger_b200 import model as M
    rng = np.random.default_rng(5)
    m, n, k = 37, 300, 400
    a8 = O.e4m3(rng.standard_normal((m, k)).astype(np.float32) * 50)
    w8, ws = M.quant_blocks(rng.standard_normal((n, k)).astype(np.float32) * 0.02)
    want = (O.e4m3_dec(a8).astype(np.float64) * 0.01) @ M.dequant_blocks(w8, ws).astype(np.float64).T
    got = O.gemm_e4m3(a8, w8, ws, 0.01)
    np.testing.assert_allclose(got, want, rtol=1e-5, atol=1e-6 * np.abs(want).max())


def _attention_numpy(O, q, k, v, sinv, vo, key_tile, slice_rows, head):
    """flash8's algorithm (kern_common.cuh:403-543) for one head, vectorised over slices of slice_rows query rows:
    decisions (lazy rescale, dead tile) per slice and key tile, as the oracle's C restatement."""
    TP, T = q.shape[2], 1025
    ns = -(-T // slice_rows)
    R = ns * slice_rows                                  # rows past 1024 are the zero padding of q
    Q = O.e4m3_dec(q[0, head, :R]).astype(np.float32)
    K, V = (O.e4m3_dec(a[0, head, :T]).astype(np.float32) for a in (k, v))
    S = (Q @ K.T).reshape(ns, slice_rows, T)
    m = np.full((ns, slice_rows), -1e30, np.float32)
    l = np.zeros((ns, slice_rows), np.float32)
    acc = np.zeros((ns, slice_rows, 64), np.float32)
    thr, dthr = np.float32(8.0 / sinv), np.float32(10.0 / sinv)
    with np.errstate(over="ignore", invalid="ignore"):
        for t0 in range(0, T, key_tile):
            s = S[:, :, t0:t0 + key_tile]
            tm = s.max(2)
            mn = np.maximum(m, tm)
            re = (mn > m + thr).any(1)                   # per slice
            sc = np.exp2((m - mn) * np.float32(sinv)).astype(np.float32)
            l = np.where(re[:, None], l * sc, l)
            acc = np.where(re[:, None, None], acc * sc[:, :, None], acc)
            m = np.where(re[:, None], mn, m)
            live = ~(tm < m - dthr).all(1)               # per slice
            p = np.exp2(s * np.float32(sinv) - (m * np.float32(sinv))[:, :, None]).astype(np.float32)
            p = np.where(live[:, None, None], p, 0)
            l = l + p.sum(2)
            acc = acc + O.e4m3_dec(O.e4m3(p)) @ V[t0:t0 + key_tile]
    out = (acc * (vo / l)[:, :, None]).reshape(R, 64)[:T]
    return O.e4m3(out.astype(np.float16).astype(np.float32))


@pytest.mark.parametrize("key_tile,slice_rows", [(64, 16), (128, 1)])
def test_attention_matches_numpy_restatement(O, key_tile, slice_rows):
    """The oracle's flash attention (tiles, lazy rescale and dead tiles decided per slice of query rows, E4M3 P,
    fp16-staged output) against a vectorised numpy statement of the same algorithm, for one head: the reference's
    64-key tiles with 16-row slices, and 128-key tiles decided per row."""
    rng = np.random.default_rng(6)
    TP, T = 1152, 1025
    q = np.zeros((1, 16, TP, 64), np.uint8)
    k = np.zeros_like(q)
    v = np.zeros_like(q)
    q[:, :, :T] = O.e4m3(rng.standard_normal((1, 16, T, 64)).astype(np.float32) * 120)
    k[:, :, :T] = O.e4m3(rng.standard_normal((1, 16, T, 64)).astype(np.float32) * 120)
    v[:, :, :T] = O.e4m3(rng.standard_normal((1, 16, T, 64)).astype(np.float32) * 60)
    sinv, vo = 3e-4, 0.7
    out = np.empty((T, 1024), np.uint8)
    O.lib().or_attention(q, k, v, 1, sinv, vo, key_tile, slice_rows, out)
    want = _attention_numpy(O, q, k, v, sinv, vo, key_tile, slice_rows, 3)
    got = out[:, 3 * 64:4 * 64]
    from tests._gpu import e4m3_ordinal
    d = np.abs(e4m3_ordinal(got) - e4m3_ordinal(want))
    assert (d == 0).mean() > 0.99 and d.max() <= 1
