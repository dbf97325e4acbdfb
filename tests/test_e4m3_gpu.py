"""The device E4M3 encoder (e4m3x2: __nv_cvt_float2_to_fp8x2 with __NV_SATFINITE / __NV_E4M3, the reference's q2,
kern_common.cuh:96-100), through xtb_e4m3_encode, against the oracle's or_e4m3 -- which tests/test_oracle_pins.py
pins bit for bit to the reference's weight quantiser (export_eva.py:64-66) -- on every fp16 value, every tie between
adjacent E4M3 values (and the floats either side of it), the saturation boundary (448, 464, 480, inf) and a sweep of
float bit patterns over every exponent. The attention output's fp16 staging (kern_common.cuh:527-541) is checked the
same way against fp16 round-to-nearest-even followed by or_e4m3.

Bit-exact everywhere except the sign of the NaN code: both sides must give a NaN code (0x7F / 0xFF) for a NaN
input, the only input the forward never produces."""
import numpy as np
import pytest

from tests import _gpu as G

pytestmark = pytest.mark.gpu


def _inputs():
    from oracle import oracle as O
    f16 = np.arange(1 << 16, dtype=np.uint32).astype(np.uint16).view(np.float16).astype(np.float32)
    codes = np.arange(0x7F, dtype=np.uint8)                        # every finite non-negative E4M3 code
    vals = O.e4m3_dec(codes).astype(np.float64)
    mids = ((vals[:-1] + vals[1:]) / 2).astype(np.float32)           # exact in fp32
    assert np.array_equal(mids.astype(np.float64), (vals[:-1] + vals[1:]) / 2)
    ties = np.concatenate([mids, np.nextafter(mids, np.float32(np.inf)), np.nextafter(mids, np.float32(0))])
    edge = np.array([448, 464, np.nextafter(np.float32(464), np.float32(0)), np.nextafter(np.float32(464),
                     np.float32(np.inf)), 480, 1e30, np.inf, 2.0 ** -10, 3 * 2.0 ** -10, 2.0 ** -12, 1e-30, 0.0],
                    np.float32)
    rng = np.random.default_rng(0)
    bits = rng.integers(0, 1 << 32, 1 << 22, dtype=np.uint64).astype(np.uint32).view(np.float32)
    dense = np.exp2(np.linspace(-14, 9.5, 1 << 20)).astype(np.float32)
    x = np.concatenate([f16, ties, edge, bits, dense])
    return np.ascontiguousarray(np.concatenate([x, -x]), np.float32)


def _compare(got, want, x, what):
    nan = np.isnan(x)
    assert ((got[nan] & 0x7F) == 0x7F).all() and ((want[nan] & 0x7F) == 0x7F).all(), f"{what}: NaN codes"
    bad = (got != want) & ~nan
    assert not bad.any(), (f"{what}: {int(bad.sum())} of {x.size} codes differ, e.g. x={x[bad][:4]} "
                           f"device={got[bad][:4]} oracle={want[bad][:4]}")


@pytest.mark.parametrize("via_f16", [0, 1])
def test_device_encoder_matches_oracle(xlib, cuda, via_f16):
    import torch
    from oracle import oracle as O
    x = _inputs()
    if via_f16:
        h = np.empty(x.shape, np.uint16)
        O.lib().or_f2h_n(x, h, x.size)
        r = np.empty(x.shape, np.float32)
        O.lib().or_h2f_n(h, r, x.size)
        want = O.e4m3(r)
    else:
        want = O.e4m3(x)
    y = G.zeros(x.shape, torch.uint8)
    assert xlib.xtb_e4m3_encode(G.P(G.dev(x)), G.P(y), x.size, via_f16, None) == 0
    G.check_error_word(xlib)
    _compare(G.host(y), want, x, "e4m3x2_via_f16" if via_f16 else "e4m3x2")


def test_device_encoder_odd_length(xlib, cuda):
    """A last unpaired element is encoded and nothing past the end is written."""
    import torch
    from oracle import oracle as O
    x = np.array([0.3, -1.7, 500.0], np.float32)
    y = G.zeros((4,), torch.uint8)
    y.fill_(0xAB)
    assert xlib.xtb_e4m3_encode(G.P(G.dev(x)), G.P(y), 3, 0, None) == 0
    out = G.host(y)
    assert np.array_equal(out[:3], O.e4m3(x)) and out[3] == 0xAB
