"""2:4 weights on the host (no GPU): the selection (xtagger_b200.model.prune24_codes, used to build the pruned
synthetic model, against the oracle's restatement of prune24.py:44-56, which the golden vectors pin) and the
compressed form the sparse tensor-core path reads (xtb_sparse24_check / xtb_sparse24_compress, host code of the
library), decoded here independently from its documented layout: values [np][kp / 2] = the two kept bytes of
every group of four; metadata [np][kp / 8] = per group i0 | i1 << 2 (i0 < i1), two groups per byte, low nibble
first; np / kp = n / k rounded up to 128, padding groups zero with indices 0 and 1."""
import ctypes as C

import numpy as np
import pytest


def _ptr(a):
    return C.c_void_p(a.ctypes.data)


def _r128(x):
    return -(-x // 128) * 128


def _decompress(vals, meta, n, k):
    npad, kp = _r128(n), _r128(k)
    v = vals.reshape(npad, kp // 2)
    m = meta.reshape(npad, kp // 8)
    nib = np.stack([m & 15, m >> 4], axis=2).reshape(npad, kp // 4)
    i0, i1 = nib & 3, nib >> 2
    assert (i0 < i1).all(), "metadata with i0 >= i1"
    out = np.zeros((npad, kp // 4, 4), np.uint8)
    rows = np.arange(npad)[:, None]
    grp = np.arange(kp // 4)[None, :]
    out[rows, grp, i0] = v[:, 0::2]
    out[rows, grp, i1] = v[:, 1::2]
    return out.reshape(npad, kp), nib


def _compress(xlib, w):
    n, k = w.shape
    vals = np.full(_r128(n) * _r128(k) // 2, 0xAB, np.uint8)
    meta = np.full(_r128(n) * _r128(k) // 8, 0xAB, np.uint8)
    rc = xlib.xtb_sparse24_compress(_ptr(w), n, k, _ptr(vals), _ptr(meta))
    return rc, vals, meta


def _zero_sign(a):
    a = np.asarray(a, np.uint8)
    return np.where((a & 0x7F) == 0, 0, a)


def _codes(rng, n, k):
    from xtagger_b200 import model as M
    q, _ = M.quant_blocks(rng.standard_normal((n, k), dtype=np.float32) * 0.02)
    q[:3] = q[:3] & 0xF8  # coarser codes: ties between members of a group
    q[3, :8] = 0x80       # negative zeros
    return q


def test_prune24_codes_matches_oracle():
    from oracle import oracle as O
    from xtagger_b200 import model as M
    rng = np.random.default_rng(60)
    q = _codes(rng, 300, 2736)
    want = q.copy()
    O.lib().or_prune24(want, 300, 2736, 0)
    np.testing.assert_array_equal(M.prune24_codes(q), want)


@pytest.mark.parametrize("n,k", [(300, 2736), (128, 1024), (5472, 1024)])
def test_compress_roundtrip(xlib, n, k):
    from xtagger_b200 import model as M
    rng = np.random.default_rng(61 + n)
    w = M.prune24_codes(_codes(rng, n, k))
    assert xlib.xtb_sparse24_check(_ptr(w), n, k) == 1
    rc, vals, meta = _compress(xlib, w)
    assert rc == 0
    full, nib = _decompress(vals, meta, n, k)
    np.testing.assert_array_equal(_zero_sign(full[:n, :k]), _zero_sign(w))
    assert not full[n:].any() and not full[:, k:].any()
    assert (nib[n:] == 4).all() and (nib[:, k // 4:] == 4).all()


def test_compress_group_patterns(xlib):
    """Every group shape: empty, one nonzero at each position, two at each of the six position pairs; kept codes
    land at their own indices, fillers take the lowest free positions."""
    groups = [[0, 0, 0, 0]]
    for i in range(4):
        g = [0, 0, 0, 0]
        g[i] = 0x41
        groups.append(g)
    for i in range(4):
        for j in range(i + 1, 4):
            g = [0x80, 0x80, 0x80, 0x80]
            g[i], g[j] = 0x3A, 0xC5
            groups.append(g)
    w = np.zeros((1, 128), np.uint8)
    w[0, :4 * len(groups)] = np.array(groups, np.uint8).ravel()
    rc, vals, meta = _compress(xlib, w)
    assert rc == 0
    full, nib = _decompress(vals, meta, 1, 128)
    np.testing.assert_array_equal(_zero_sign(full[0]), _zero_sign(w[0]))
    want_nib = [0 | 1 << 2, 0 | 1 << 2, 0 | 1 << 2, 0 | 2 << 2, 0 | 3 << 2]
    want_nib += [i | j << 2 for i in range(4) for j in range(i + 1, 4)]
    np.testing.assert_array_equal(nib[0, :len(groups)], want_nib)


def test_rejects_dense_weights(xlib):
    rng = np.random.default_rng(62)
    w = _codes(rng, 130, 1024)
    assert xlib.xtb_sparse24_check(_ptr(w), 130, 1024) == 0
    rc, _, _ = _compress(xlib, w)
    assert rc == -1
    w = np.zeros((4, 1024), np.uint8)
    w[2, 8:11] = 0x30  # a single group with three nonzero codes
    assert xlib.xtb_sparse24_check(_ptr(w), 4, 1024) == 0
    assert xlib.xtb_sparse24_check(_ptr(w[:, :1022].copy()), 4, 1022) == 0  # k not a multiple of 4
