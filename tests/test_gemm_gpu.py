"""Block-scaled E4M3 GEMM on tcgen05 (xtb_gemm_e4m3_f32) against a plain fp32 dequantize-then-matmul.

Tolerance (north star): every output within 1e-2 relative. The kernel multiplies the same E4M3 products in fp32,
so in practice only the summation order differs.
"""
import ctypes as C

import pytest

pytestmark = pytest.mark.gpu


def _quant_blocks(w, blk=128):
    """E4M3 with one fp32 scale per blk x blk block (scale = max|block| / 448), like the synthetic model writer."""
    import torch
    n, k = w.shape
    nb, kb = (n + blk - 1) // blk, (k + blk - 1) // blk
    wp = torch.zeros(nb * blk, kb * blk, dtype=torch.float32, device=w.device)
    wp[:n, :k] = w
    blocks = wp.view(nb, blk, kb, blk)
    s = blocks.abs().amax(dim=(1, 3)).clamp_min(1e-12) / 448.0
    q = (blocks / s[:, None, :, None]).clamp(-448, 448).to(torch.float8_e4m3fn)
    deq = q.float() * s[:, None, :, None]
    return (q.view(nb * blk, kb * blk)[:n, :k].contiguous(), s.contiguous(),
            deq.view(nb * blk, kb * blk)[:n, :k].contiguous())


def _run(xlib, m, n, k, seed):
    import torch
    g = torch.Generator(device="cuda").manual_seed(seed)
    a = torch.randn(m, k, generator=g, device="cuda")
    asc = a.abs().max().item() / 448.0
    a8 = (a / asc).clamp(-448, 448).to(torch.float8_e4m3fn)
    w = torch.randn(n, k, generator=g, device="cuda") * 0.02
    w8, ws, wdeq = _quant_blocks(w)
    out = torch.full((m, n), float("nan"), device="cuda")
    rc = xlib.xtb_gemm_e4m3_f32(C.c_void_p(a8.data_ptr()), m, k, C.c_void_p(w8.data_ptr()), n,
                                C.c_void_p(ws.data_ptr()), C.c_float(asc), C.c_void_p(out.data_ptr()), None)
    assert rc == 0
    torch.cuda.synchronize()
    assert xlib.xtb_error_word(0) == 0
    ref = (a8.float() * asc) @ wdeq.t()
    return out, ref


@pytest.mark.parametrize("m,n,k", [(128, 256, 128), (1025, 2730, 1024), (300, 100, 256), (8200, 5472, 1024),
                                   (257, 1024, 2736), (64, 10861, 1024)])
def test_gemm_blockscaled_matches_fp32(xlib, cuda, m, n, k):
    import torch
    out, ref = _run(xlib, m, n, k, seed=m + n + k)
    assert torch.isfinite(out).all()
    err = (out - ref).abs()
    scale = ref.abs().max().item()
    assert err.max().item() <= 1e-2 * scale, (err.max().item(), scale)
    # elementwise: relative 1e-2 with a floor at 1e-3 of the output range
    assert bool((err <= 1e-2 * ref.abs() + 1e-3 * scale).all())


@pytest.mark.parametrize("pair", [0, 1, 2])
@pytest.mark.parametrize("m,n,k", [(2050, 5472, 1024), (1000, 1024, 2736), (300, 3072, 1024)])
def test_gemm_block_scale_mma(xlib, cuda, m, n, k, pair):
    """The block-scaled MMA kernels (single CTA, CTA pair, CTA pair on 256-column tiles) against the oracle's
    dequantize-then-matmul on power-of-two block scales that vary across N and K blocks, adjacent 128-row weight
    blocks included (a wide tile spans two): the same sums up to the fp32 order."""
    import ctypes as C
    import numpy as np
    import torch
    from oracle import oracle as O
    from xtagger_b200 import model as M
    from tests import _gpu as G
    rng = np.random.default_rng(m + n + k + pair)
    a = O.e4m3(rng.standard_normal((m, k), dtype=np.float32) * 40)
    w = rng.standard_normal((n, k), dtype=np.float32) * 0.02
    w[:, : k // 3] *= 16.0
    w[n // 2:] *= 0.125
    w[(np.arange(n) // 128) % 2 == 1] *= 4.0    # odd weight blocks four times their neighbours
    wq, ws = M.quant_blocks(w, pow2=True)
    assert np.all(ws[1::2, 0][: (n // 128) // 2] != ws[0::2, 0][: (n // 128) // 2])
    assert len(np.unique(ws)) > 2
    img = np.zeros(xlib.xtb_sf_image_bytes(n, k), np.uint8)
    assert xlib.xtb_sf_image(ws.ctypes.data_as(C.c_void_p), n, k, img.ctypes.data_as(C.c_void_p)) == 0
    ascale = 1.0 / 40
    want = O.gemm_e4m3(a, wq, ws, ascale)
    out = G.zeros((m, n), torch.float32)
    assert xlib.xtb_gemm_mx_f32(G.P(G.dev(a)), m, k, G.P(G.dev(wq)), n, G.P(G.dev(img)), pair, ascale, G.P(out), n,
                                None) == 0
    G.check_error_word(xlib)
    got = G.host(out)
    scale = np.abs(want).max()
    err = np.abs(got - want)
    assert err.max() <= 1e-5 * scale, (err.max(), scale)
