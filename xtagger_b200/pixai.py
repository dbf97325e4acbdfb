"""PixAI tagger (ViTDet-L at 1008^2) weight format, input layout and the seeded synthetic-model writer.

Format (reader: csrc/px_engine.cu and oracle/px_oracle.c; reference: src/engine/px.h:196-245, writer
src/tools/export_pixai.py:119-146): 16-byte header ``"PXAI", version 3, nt, blob bytes`` zero-padded to 256 bytes,
then 256-byte-aligned tensors:

  table f32 [nl][12]       per block: weight dequant x4 (QKV, O, fc1, fc2), activation dequant x4, q, k, v, 0
  pe f16 [1024][592]       patch embedding, column c*196 + ky*14 + kx (RGB), 588..591 zero
  pos f32 [5184][1024]     absolute position table, tiled 3 x 3 and permuted to window-major token order
  ln_pre w, b f32 [1024]
  cs_win f32 [576][32][2]  RoPE (cos, sin) of the windowed blocks (window-local token order)
  cs_glob f32 [5184][32][2] RoPE of the global blocks (window-major token order)
  per block: ln1 w, b; Wqkv u8 [3072][1024]; bqkv f32 [3072]; Wo u8 [1024][1024]; bo; ln2 w, b;
             W1 u8 [4736][1024]; b1 f32 [4736]; rs f32 [4736]; W2 u8 [1024][4736]; b2 f32 [1024]
  head: norm w, b f32 [1024]; U f32 [16][1024]; hpos f16 [5184][1024]; Wv f16 [1024][1024];
        hw f16 [ntp][1024]; hb f32 [ntp]                                          (ntp = nt rounded up to 8)

Wq rows and the q bias carry 1/8 x log2(e) (scores in the exp2 domain). Tokens are window-major throughout: 72 x 72
patches = 9 windows of 24 x 24, window w = tokens 576 w .. 576 w + 575 (export_pixai.py:39-42). Blocks 7, 15, 23 and
31 attend over all 5184 tokens, the others within their window.

This library's extension of the header (zero in the reference's files, which then read as the reference's model):
word 4 = number of blocks (0 = 32), word 5 = bit mask of the global blocks (0 = block i is global when i % 8 == 7).
"""
import os
import struct

import numpy as np

from . import model as M

D, T, LW, HID, NL, K0, K0P, NH, HD = 1024, 5184, 576, 4736, 32, 588, 592, 16, 64
WS, GRID, NWIN = 24, 72, 9
PX_IN = T * K0P          # halves per model input
E4M3_MAX = 448.0
HEADROOM = 1.25


def window_perm():
    """perm[i] = row-major token (72 x 72 grid) of window-major token i (export_pixai.py:39-42)."""
    i = np.arange(T)
    wi, l = i // (WS * WS), i % (WS * WS)
    return ((wi // 3) * WS + l // WS) * GRID + (wi % 3) * WS + l % WS


def is_global(i, nl=NL, gmask=0):
    """Whether block i attends over all tokens (px.h:37: blocks 7, 15, 23, 31), or per the file's mask."""
    return bool((gmask >> i) & 1) if gmask else (i & 7) == 7


def axial_rope(grid, theta=10000.0):
    """2D axial rotary table [grid^2][32][2] = (cos, sin) per token (row-major) and rotary pair: pairs 0..15
    rotate with the token's row, 16..31 with its column, frequencies theta^(-2i / 32)."""
    freqs = 1.0 / theta ** (np.arange(0, 32, 2, dtype=np.float64) / 32)
    t = np.arange(grid, dtype=np.float64)
    fy, fx = np.meshgrid(t, t, indexing="ij")
    ang = np.concatenate([fy.reshape(-1, 1) * freqs[None], fx.reshape(-1, 1) * freqs[None]], 1)
    return np.stack([np.cos(ang), np.sin(ang)], -1).astype(np.float32)


def patch_operand(img_rgb):
    """1008 x 1008 x 3 RGB image in [0, 1] -> the engine's input: fp16 [5184 window-major patches][592], RGB,
    (x - 0.5) / 0.5, column c*196 + ky*14 + kx (px.h:9-10)."""
    a = (np.asarray(img_rgb, np.float32) - 0.5) / 0.5
    p = a.reshape(GRID, 14, GRID, 14, 3).transpose(0, 2, 4, 1, 3).reshape(GRID * GRID, K0)  # row-major patches
    out = np.zeros((T, K0P), np.float16)
    out[:, :K0] = p[window_perm()]
    return out


def synthetic_inputs(n, seed=1):
    """n seeded synthetic images (uniform [0, 1] pixels) as patch operands, uint16 view [n][5184][592]."""
    rng = np.random.default_rng(seed)
    return np.stack([patch_operand(rng.random((GRID * 14, GRID * 14, 3), dtype=np.float32))
                     for _ in range(n)]).view(np.uint16)


def write_synthetic(path, seed=0, nt=30877, nl=NL, gmask=0, ln_noise=1.0, std=0.02):
    """Random-init PixAI tagger in pixai.bin v3 format (E4M3 weights with one scale per tensor, as export_pixai.py
    writes them). Linears and biases N(0, std); LayerNorm gamma 1 + N(0, 0.1 ln_noise), beta N(0, 0.1 ln_noise);
    pos, pe, U, hpos, Wv, head N(0, std); axial RoPE tables. Static activation scales in closed form from the
    random-init statistics (LayerNorm outputs have unit variance per row): LN outputs amax 8; q / k / v amax
    6 ||W row||_2 + |bias|; attention output bounded by v; GELU output 6 ||W1 row||_2; 1.25 headroom."""
    rng = np.random.default_rng(seed)
    ntp = (nt + 7) & ~7

    def randn(*shape):
        return rng.standard_normal(shape, dtype=np.float32) * std

    def ln_pair(n):
        return ((1 + 0.1 * ln_noise * rng.standard_normal(n, dtype=np.float32)).astype(np.float32),
                (0.1 * ln_noise * rng.standard_normal(n, dtype=np.float32)).astype(np.float32))

    qs = (1.0 / 8.0) * np.log2(np.e)
    perm = window_perm()
    blob = M._Blob()
    table = np.zeros((nl, 12), np.float32)
    pe = np.zeros((D, K0P), np.float32)
    pe[:, :K0] = randn(D, K0)
    pos = randn(T, D)
    lnp = ln_pair(D)
    cs_win = axial_rope(WS)
    cs_glob = axial_rope(GRID)[perm]
    layers = []
    for i in range(nl):
        ln1 = ln_pair(D)
        wqkv = randn(3 * D, D)
        bqkv = randn(3 * D)
        wqkv[:D] *= qs
        bqkv[:D] *= qs
        wo, bo = randn(D, D), randn(D)
        ln2 = ln_pair(D)
        w1, b1 = randn(HID, D), randn(HID)
        w2, b2 = randn(D, HID), randn(D)
        rn = np.sqrt((wqkv.reshape(3, D, D) ** 2).sum(2)).max(1)            # max row norm of q, k, v
        bq = np.abs(bqkv.reshape(3, D)).max(1)
        amax_q, amax_k, amax_v = (6 * rn + bq).tolist()
        amax_u = 6 * float(np.sqrt((w1 ** 2).sum(1)).max()) + float(np.abs(b1).max())
        adq = [8.0, amax_v, 8.0, amax_u]
        table[i, 4:8] = [a * HEADROOM / E4M3_MAX for a in adq]
        table[i, 8:11] = [a * HEADROOM / E4M3_MAX for a in (amax_q, amax_k, amax_v)]
        mats = []
        for g, w in enumerate((wqkv, wo, w1, w2)):
            q, sc = M.quant_tensor(w)
            table[i, g] = sc
            mats.append(q)
        rs = np.full(HID, 1.0 / table[i, 7], np.float32)
        layers.append((ln1, mats, bqkv, bo, ln2, b1, rs, b2))
    hn = ln_pair(D)
    U = randn(NH, D)
    hpos = randn(T, D)
    wv = randn(D, D)
    hw = np.zeros((ntp, D), np.float32)
    hw[:nt] = randn(nt, D)
    hb = np.zeros(ntp, np.float32)
    hb[:nt] = randn(nt)

    blob.put(table, np.float32)
    blob.put(pe, np.float16)
    blob.put(pos, np.float32)
    blob.put(lnp[0], np.float32)
    blob.put(lnp[1], np.float32)
    blob.put(cs_win, np.float32)
    blob.put(cs_glob, np.float32)
    for ln1, mats, bqkv, bo, ln2, b1, rs, b2 in layers:
        blob.put(ln1[0], np.float32)
        blob.put(ln1[1], np.float32)
        blob.put(mats[0], np.uint8)
        blob.put(bqkv, np.float32)
        blob.put(mats[1], np.uint8)
        blob.put(bo, np.float32)
        blob.put(ln2[0], np.float32)
        blob.put(ln2[1], np.float32)
        blob.put(mats[2], np.uint8)
        blob.put(b1, np.float32)
        blob.put(rs, np.float32)
        blob.put(mats[3], np.uint8)
        blob.put(b2, np.float32)
    blob.put(hn[0], np.float32)
    blob.put(hn[1], np.float32)
    blob.put(U, np.float32)
    blob.put(hpos, np.float16)
    blob.put(wv, np.float16)
    blob.put(hw, np.float16)
    blob.put(hb, np.float32)
    hdr = struct.pack("<4sIIIII", b"PXAI", 3, nt, blob.n, 0 if nl == NL else nl, gmask)
    tmp = path + ".tmp"
    with open(tmp, "wb") as f:
        f.write(hdr + b"\0" * (256 - len(hdr)))
        for p in blob.parts:
            f.write(p)
    os.replace(tmp, path)
    return path


def cached_synthetic(d, **kw):
    """write_synthetic into directory d once per parameter set (the file name encodes them)."""
    os.makedirs(d, exist_ok=True)
    name = "px_" + "_".join(f"{k}{v}" for k, v in sorted(kw.items())) + ".bin"
    p = os.path.join(d, name)
    if not os.path.exists(p):
        write_synthetic(p, **kw)
    return p
