"""Helpers for the GPU parity tests: numpy <-> device buffers (torch is only the allocator here) and the
comparison rules for E4M3 / fp16 outputs."""
import ctypes as C

import numpy as np


_keep = []


def dev(a):
    """Device copy of a numpy array. The tensor is kept alive until release() so that a pointer taken from a
    temporary cannot be recycled by the caching allocator before the kernel that reads it has run."""
    import torch
    t = torch.from_numpy(np.ascontiguousarray(a)).cuda()
    _keep.append(t)
    return t


def release():
    import torch
    torch.cuda.synchronize()
    _keep.clear()


def zeros(shape, dtype):
    import torch
    t = torch.zeros(shape, dtype=dtype, device="cuda")
    _keep.append(t)
    return t


def P(t):
    return C.c_void_p(t.data_ptr())


def host(t):
    import torch
    torch.cuda.synchronize()
    return t.cpu().numpy()


def e4m3_ordinal(b):
    """Signed position of an E4M3 code on the number line (adjacent finite values differ by 1; +-0 -> 0)."""
    b = np.asarray(b, np.int32)
    mag = b & 0x7F
    return np.where(b & 0x80, -mag, mag)


def assert_e4m3_close(got, want, max_steps=1, min_exact=0.99, what=""):
    """Codes equal, or at most max_steps representable values apart (a rounding decision at a boundary)."""
    d = np.abs(e4m3_ordinal(got) - e4m3_ordinal(want))
    exact = float((d == 0).mean())
    assert d.max() <= max_steps, f"{what}: {int((d > max_steps).sum())} codes more than {max_steps} apart (max {d.max()})"
    assert exact >= min_exact, f"{what}: only {exact:.4f} of codes identical"


def f16(a):
    return np.asarray(a, np.uint16).view(np.float16).astype(np.float32)


def assert_f16_close(got, want, rel=1e-2, what=""):
    g, w = f16(got), f16(want)
    assert np.isfinite(g).all(), f"{what}: non-finite output"
    scale = np.abs(w).max() + 1e-30
    err = np.abs(g - w)
    assert (err <= rel * np.abs(w) + 1e-3 * scale).all(), f"{what}: max err {err.max()} (scale {scale})"


def check_error_word(xlib):
    import torch
    torch.cuda.synchronize()
    assert xlib.xtb_error_word(0) == 0, "a kernel's bounded wait ran out"


def assert_attention_close(got, want, what="attention"):
    """Attention outputs: scores come from the tensor core's fp32 accumulation and exp2 from ex2.approx, so a p on
    an E4M3 rounding boundary, or a row's tile max on the lazy-rescale threshold, can round either way. Near zero
    such a flip spans several finely spaced small codes, so the step bound applies to outputs of at least 1/16 of
    the range; everywhere else the mean deviation is bounded."""
    from oracle import oracle as O
    d = np.abs(e4m3_ordinal(got) - e4m3_ordinal(want))
    gv, wv = O.e4m3_dec(got), O.e4m3_dec(want)
    rng = np.abs(wv).max()
    big = np.abs(wv) >= rng / 16
    assert (d == 0).mean() >= 0.95, f"{what}: only {(d == 0).mean():.4f} identical"
    assert d[big].max() <= 2, f"{what}: codes of large outputs up to {d[big].max()} steps apart"
    assert np.abs(gv - wv).mean() <= 2e-3 * rng, f"{what}: mean deviation {np.abs(gv - wv).mean() / rng:.2e} of range"
