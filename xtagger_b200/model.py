"""Weight format (eva02.bin v3 / block-scaled v4), input layout, and the seeded synthetic-model writer.

Format (reader: engine.cpp; reference: src/engine/eva.h:378-430, writer src/tools/export_eva.py:119-153):
16-byte header ``"EVA2", version, nt, blob bytes`` zero-padded to 256 bytes, then 256-byte-aligned tensors:

  table f32 [nl][12]   per layer: weight dequant x4 (QKV, O, W12, W2), activation dequant x4, q, k, v dequant, pad
  pe f16 [1024][592]   patch embedding, column c*196 + ky*14 + kx (BGR), 588..591 zero
  pos f32 [1025][1024] position table, cls folded into row 0, conv bias into rows 1..
  cs f32 [1024][32][2] RoPE (cos, sin) per patch token and rotary pair
  per layer: ln1 g, b f32 [1024]; Wqkv u8 [3072][1024]; Wo u8 [1024][1024]; ln2 g, b; W12 u8 [5472][1024]
             (g / x interleaved in 16-unit chunks); rs f32 [2736]; W~2 u8 [1024][2736]; c f32 [1024]; d f32 [1024]
  fc_norm g, b f32 [1024]; head hw f16 [ntp][1024]; hb f32 [ntp]          (ntp = nt rounded up to 8)

v3 (the reference's production format): E4M3 weights with one fp32 scale per tensor (table columns 0..3).
v4 (this library): header word 4 = number of layers (0 = 24), word 5 = flags (bit 0: FP8 head); every E4M3 matrix
is followed by fp32 scales, one per 128 x 128 block ([ceil(n/128)][ceil(k/128)]); table columns 0..3 are unused.
With an FP8 head the head reads: f32[4] {head activation dequant, 0, 0, 0}; hw u8 [ntp][1024]; hw scales
[ceil(ntp/128)][8]; hb f32 [ntp].
"""
import os
import struct

import numpy as np

D, T, NP, HID, HIDP, K0, K0P, NH = 1024, 1025, 1024, 2730, 2736, 588, 592, 16
N12 = 2 * HIDP
E4M3_MAX = 448.0
HEADROOM = 1.25          # activation scale margin, as export_eva.py:20


def _e4m3(x):
    """float32 -> E4M3 bytes, round to nearest even, after clipping to +-448 (export_eva.py:64-66)."""
    import ml_dtypes
    return np.clip(x, -E4M3_MAX, E4M3_MAX).astype(ml_dtypes.float8_e4m3fn).view(np.uint8)


def e4m3_decode(b):
    """E4M3 bytes -> float32 (NaN codes decode to NaN)."""
    import ml_dtypes
    return np.asarray(b, np.uint8).view(ml_dtypes.float8_e4m3fn).astype(np.float32)


def quant_blocks(w, blk=128, pow2=False):
    """E4M3 with one fp32 scale per blk x blk block: scale = max|block| / 448 (1 for an all-zero block); with pow2 the
    scale is rounded up to a power of two (the block's largest value then lands in [224, 448]), which the tensor
    core applies itself as an UE8M0 scale factor."""
    n, k = w.shape
    nb, kb = -(-n // blk), -(-k // blk)
    wp = np.zeros((nb * blk, kb * blk), np.float32)
    wp[:n, :k] = w
    v = wp.reshape(nb, blk, kb, blk)
    s = np.abs(v).max(axis=(1, 3)).astype(np.float32) / E4M3_MAX
    s[s == 0] = 1.0
    if pow2:
        s = np.exp2(np.ceil(np.log2(s.astype(np.float64)))).astype(np.float32)
    q = _e4m3(v / s[:, None, :, None]).reshape(nb * blk, kb * blk)[:n, :k]
    return np.ascontiguousarray(q), s


def dequant_blocks(q, s, blk=128):
    n, k = q.shape
    f = e4m3_decode(q)
    return f * np.repeat(np.repeat(s, blk, 0), blk, 1)[:n, :k]


def quant_tensor(w):
    """The reference's per-tensor E4M3 (export_eva.py:64-66): scale = max|w| / 448."""
    sc = float(np.abs(w).max()) / E4M3_MAX
    return _e4m3(w / sc), sc


def interleave_gx(gx):
    """[g (HIDP rows) | x (HIDP rows)] -> 16-unit chunks [g_c | x_c] (export_eva.py:60-62)."""
    return gx.reshape(2, HIDP // 16, 16, -1).transpose(1, 0, 2, 3).reshape(2 * HIDP, -1)


def prune24_codes(q):
    """2:4 selection by magnitude on E4M3 codes (prune24.py:44-56, "mag" mode): in every group of four consecutive
    k of each row the two codes of smallest |value| become zero; among equal values the lower index is dropped first
    (a stable sort, as numpy's argsort is for four elements). The scale of a 128 x 128 block is common to a group,
    so ranking codes ranks the dequantised weights."""
    q = np.ascontiguousarray(q, np.uint8)
    n, k = q.shape
    assert k % 4 == 0
    v = np.abs(e4m3_decode(q)).reshape(n, k // 4, 4)
    v[np.isnan(v)] = 0.0  # NaN codes score 0, as in prune24.py's E4 table
    drop = np.argsort(v, axis=2, kind="stable")[:, :, :2]
    keep = np.ones(v.shape, bool)
    np.put_along_axis(keep, drop, False, axis=2)
    return np.where(keep.reshape(n, k), q, 0).astype(np.uint8)


def rope_table(theta=10000.0, grid=32, pt_seq=16):
    """EVA02 2D axial rotary table [1024][32][2] = (cos, sin) per patch token and rotary pair: pairs 0..15 rotate
    with the token's row coordinate, 16..31 with its column, frequencies theta^(-2i/32), coordinates scaled by
    pt_seq / grid (EVA02's fine-tuning interpolation)."""
    freqs = 1.0 / theta ** (np.arange(0, 32, 2, dtype=np.float64) / 32)
    t = np.arange(grid, dtype=np.float64) * (pt_seq / grid)
    fy, fx = np.meshgrid(t, t, indexing="ij")
    ang = np.concatenate([fy.reshape(-1, 1) * freqs[None], fx.reshape(-1, 1) * freqs[None]], 1)  # [1024][32]
    return np.stack([np.cos(ang), np.sin(ang)], -1).astype(np.float32)


def patch_operand(img_rgb):
    """HxWx3 RGB image in [0, 1] (448 x 448) -> the engine's input: fp16 [1024][592], BGR, (x - 0.5) / 0.5,
    column c*196 + ky*14 + kx, patch index py*32 + px (eva.h:15-16)."""
    a = np.asarray(img_rgb, np.float32)[:, :, ::-1]                       # BGR
    a = (a - 0.5) / 0.5
    p = a.reshape(32, 14, 32, 14, 3).transpose(0, 2, 4, 1, 3).reshape(NP, K0)
    out = np.zeros((NP, K0P), np.float16)
    out[:, :K0] = p
    return out


def synthetic_inputs(n, seed=1):
    """n seeded synthetic images (uniform [0, 1] pixels) as patch operands, uint16 view [n][1024][592]."""
    rng = np.random.default_rng(seed)
    return np.stack([patch_operand(rng.random((448, 448, 3), dtype=np.float32)) for _ in range(n)]).view(np.uint16)


def structured_image(rng, side=448, grid=8, amp=0.25, noise=0.05):
    """One seeded synthetic image with image-level content, RGB in [0, 1]: a base colour U[0.15, 0.85] per channel,
    a smooth field (N(0, 1) on a grid x grid lattice, bilinearly interpolated) times amp, and N(0, noise) pixel
    noise, clipped. Unlike uniform-noise pixels, the token mean of such an image differs from image to image."""
    base = rng.uniform(0.15, 0.85, 3)
    g = rng.standard_normal((grid, grid, 3))
    t = np.clip((np.arange(side) + 0.5) * grid / side - 0.5, 0, grid - 1)
    i0 = np.minimum(t.astype(np.int64), grid - 2)
    w = (t - i0)[:, None]
    rows = g[i0] * (1 - w)[:, :, None] + g[i0 + 1] * w[:, :, None]                       # [side][grid][3]
    field = rows[:, i0] * (1 - w.T)[:, :, None] + rows[:, i0 + 1] * w.T[:, :, None]      # [side][side][3]
    img = base + amp * field + noise * rng.standard_normal((side, side, 3))
    return np.clip(img, 0, 1).astype(np.float32)


def structured_inputs(n, seed=1):
    """n seeded structured_image()s as patch operands, uint16 view [n][1024][592]."""
    rng = np.random.default_rng(seed)
    return np.stack([patch_operand(structured_image(rng)) for _ in range(n)]).view(np.uint16)


class _Blob:
    def __init__(self):
        self.parts, self.n = [], 0

    def put(self, a, dt):
        pad = -self.n % 256
        if pad:
            self.parts.append(b"\0" * pad)
            self.n += pad
        b = np.ascontiguousarray(a, dtype=dt).tobytes()
        self.parts.append(b)
        self.n += len(b)


def write_synthetic(path, seed=0, nt=10861, nl=24, version=4, head_fp8=True, ln_noise=0.0, std=0.02, prune24=False,
                    pow2=False):
    """Random-init EVA02-L tagger in eva02.bin format.

    Linears N(0, std) quantised to E4M3 (v4: per 128 x 128 block; v3: per tensor); LayerNorm gamma = 1 and
    beta = 0, perturbed by N(0, 0.1 ln_noise) when ln_noise > 0 (so that every folded term is exercised);
    pos, cls, patch embedding N(0, std); EVA02 RoPE table; head bias 0. prune24: the four projections of every
    layer (QKV, O, W12, W2) made 2:4 sparse along k after quantisation (prune24_codes); the folded MLP term c is
    computed from the pruned W2. pow2 (v4): the four projections' block scales are powers of two (quant_blocks).
    Static activation scales: closed-form statistics of the random-init network, since LayerNorm outputs have
    unit variance per row: LN outputs amax 8; q / k / v amax 6 ||W row||_2 (max over rows); attention output
    bounded by v's; SwiGLU output 16 sigma_x sigma_g; every one times the reference's 1.25 headroom.
    """
    assert version in (3, 4)
    if version == 3:
        assert nl == 24 and not head_fp8, "v3 files always hold 24 layers and an fp16 head"
    rng = np.random.default_rng(seed)
    ntp = (nt + 7) & ~7

    def randn(*shape):
        return rng.standard_normal(shape, dtype=np.float32) * std

    def ln_pair(n):
        if ln_noise:
            return (1 + 0.1 * ln_noise * rng.standard_normal(n, dtype=np.float32)).astype(np.float32), \
                (0.1 * ln_noise * rng.standard_normal(n, dtype=np.float32)).astype(np.float32)
        return np.ones(n, np.float32), np.zeros(n, np.float32)

    qscale = (1.0 / np.sqrt(64.0)) * np.log2(np.e)   # softmax scale * log2(e) in Wq (export_eva.py:70-71, 86)
    blob = _Blob()
    table = np.zeros((nl, 12), np.float32)
    pe = np.zeros((D, K0P), np.float32)
    pe[:, :K0] = randn(D, K0)
    pos = randn(T, D)
    cs = rope_table()
    layers = []
    for i in range(nl):
        ln1 = ln_pair(D)
        wq = randn(D, D) * qscale
        wk, wv = randn(D, D), randn(D, D)
        wqkv = np.concatenate([wq, wk, wv], 0)
        wo = randn(D, D)
        ln2 = ln_pair(D)
        w12 = np.zeros((N12, D), np.float32)
        w12[:HID] = randn(HID, D)
        w12[HIDP:HIDP + HID] = randn(HID, D)
        mw, mb = ln_pair(HID)
        w2 = np.zeros((D, HIDP), np.float32)
        w2[:, :HID] = randn(D, HID)
        rown = np.sqrt((w12[:HID] ** 2).sum(1)).max(), np.sqrt((w12[HIDP:HIDP + HID] ** 2).sum(1)).max()
        w12 = interleave_gx(w12)
        mwp = np.zeros(HIDP, np.float32)
        mwp[:HID] = mw
        mbp = np.zeros(HIDP, np.float32)
        mbp[:HID] = mb
        dn = (w2 @ mbp).astype(np.float32)                 # d = W2 beta (export_eva.py:102)
        wt2 = w2 * mwp[None, :]                            # W~ = W2 gamma
        # activation amax (static, closed form) -> table
        amax_ln = 8.0
        amax_q = 6 * np.sqrt((wq ** 2).sum(1)).max()
        amax_k = 6 * np.sqrt((wk ** 2).sum(1)).max()
        amax_v = 6 * np.sqrt((wv ** 2).sum(1)).max()
        amax_h = 16 * rown[0] * rown[1]
        adq = [amax_ln, amax_v, amax_ln, amax_h]
        table[i, 4:8] = [a * HEADROOM / E4M3_MAX for a in adq]
        table[i, 8:11] = [amax_q * HEADROOM / E4M3_MAX, amax_k * HEADROOM / E4M3_MAX, amax_v * HEADROOM / E4M3_MAX]
        mats = []
        for g, w in enumerate((wqkv, wo, w12, wt2)):
            if version == 4:
                q, s = quant_blocks(w, pow2=pow2)
                if prune24:
                    q = prune24_codes(q)
                table[i, g] = 1.0
                mats.append((q, s, dequant_blocks(q, s)))
            else:
                q, sc = quant_tensor(w)
                if prune24:
                    q = prune24_codes(q)
                table[i, g] = sc
                mats.append((q, None, e4m3_decode(q) * sc))
        rs = np.full(HIDP, 1.0 / table[i, 7], np.float32)  # raw h -> E4M3 operand (no smoothing)
        c = mats[3][2].sum(1).astype(np.float32)           # c = W~ 1, from the quantised W~ (export_eva.py:118)
        layers.append((ln1, mats[0], mats[1], ln2, mats[2], rs, mats[3], c, dn))
    fw, fb = ln_pair(D)
    hw = np.zeros((ntp, D), np.float32)
    hw[:nt] = randn(nt, D)
    hb = np.zeros(ntp, np.float32)

    blob.put(table, np.float32)
    blob.put(pe, np.float16)
    blob.put(pos, np.float32)
    blob.put(cs, np.float32)

    def put_mat(m):
        blob.put(m[0], np.uint8)
        if version == 4:
            blob.put(m[1], np.float32)

    for ln1, mq, mo, ln2, m12, rs, m2, c, dn in layers:
        blob.put(ln1[0], np.float32)
        blob.put(ln1[1], np.float32)
        put_mat(mq)
        put_mat(mo)
        blob.put(ln2[0], np.float32)
        blob.put(ln2[1], np.float32)
        put_mat(m12)
        blob.put(rs, np.float32)
        put_mat(m2)
        blob.put(c, np.float32)
        blob.put(dn, np.float32)
    blob.put(fw, np.float32)
    blob.put(fb, np.float32)
    if head_fp8:
        amax_pn = 8.0
        blob.put(np.array([amax_pn * HEADROOM / E4M3_MAX, 0, 0, 0], np.float32), np.float32)
        q, s = quant_blocks(hw)
        blob.put(q, np.uint8)
        blob.put(s, np.float32)
    else:
        blob.put(hw, np.float16)
    blob.put(hb, np.float32)
    hdr = struct.pack("<4sIII", b"EVA2", version, nt, blob.n)
    if version == 4:
        hdr += struct.pack("<II", 0 if nl == 24 else nl, 1 if head_fp8 else 0)
    tmp = path + ".tmp"
    with open(tmp, "wb") as f:
        f.write(hdr + b"\0" * (256 - len(hdr)))
        for p in blob.parts:
            f.write(p)
    os.replace(tmp, path)
    return path


def cached_synthetic(directory, **kw):
    """Path of a synthetic model with these parameters, written once into `directory`."""
    key = "_".join(f"{k}{v}" for k, v in sorted(kw.items()))
    path = os.path.join(directory, f"eva_synth_{key}.bin")
    if not os.path.exists(path):
        os.makedirs(directory, exist_ok=True)
        write_synthetic(path, **kw)
    return path


def read_model(path):
    """Parse an eva02.bin (v3 / v4) into numpy arrays (views of the file bytes). Layout as in the module doc."""
    raw = np.fromfile(path, np.uint8)
    magic, ver, nt, nbytes = struct.unpack("<4sIII", raw[:16].tobytes())
    assert magic == b"EVA2" and ver in (3, 4), f"{path}: not an eva02.bin v3 / v4"
    nl, flags = (struct.unpack("<II", raw[16:24].tobytes()) if ver == 4 else (0, 0))
    nl = nl or 24
    head8 = ver == 4 and bool(flags & 1)
    ntp = (nt + 7) & ~7
    blob = raw[256:256 + nbytes]
    off = [0]

    def take(nb, dt, shape):
        o = (off[0] + 255) & ~255
        off[0] = o + nb
        return blob[o:o + nb].view(dt).reshape(shape)

    def kb(x):
        return -(-x // 128)

    m = {"version": ver, "nt": nt, "ntp": ntp, "nl": nl, "head8": head8}
    m["table"] = take(nl * 48, np.float32, (nl, 12))
    m["pe"] = take(D * K0P * 2, np.uint16, (D, K0P))
    m["pos"] = take(T * D * 4, np.float32, (T, D))
    m["cs"] = take(NP * 32 * 8, np.float32, (NP, 32, 2))
    layers = []
    for i in range(nl):
        L = {}
        L["ln1w"] = take(D * 4, np.float32, (D,))
        L["ln1b"] = take(D * 4, np.float32, (D,))
        for name, n, k in (("qkv", 3 * D, D), ("o", D, D)):
            L[name] = take(n * k, np.uint8, (n, k))
            L[name + "_s"] = (take(kb(n) * kb(k) * 4, np.float32, (kb(n), kb(k))) if ver == 4 else
                              np.full((kb(n), kb(k)), m["table"][i, ("qkv", "o").index(name)], np.float32))
        L["ln2w"] = take(D * 4, np.float32, (D,))
        L["ln2b"] = take(D * 4, np.float32, (D,))
        L["w12"] = take(N12 * D, np.uint8, (N12, D))
        L["w12_s"] = (take(kb(N12) * kb(D) * 4, np.float32, (kb(N12), kb(D))) if ver == 4 else
                      np.full((kb(N12), kb(D)), m["table"][i, 2], np.float32))
        L["rs"] = take(HIDP * 4, np.float32, (HIDP,))
        L["w2"] = take(D * HIDP, np.uint8, (D, HIDP))
        L["w2_s"] = (take(kb(D) * kb(HIDP) * 4, np.float32, (kb(D), kb(HIDP))) if ver == 4 else
                     np.full((kb(D), kb(HIDP)), m["table"][i, 3], np.float32))
        L["c"] = take(D * 4, np.float32, (D,))
        L["d"] = take(D * 4, np.float32, (D,))
        t = m["table"][i]
        L["adq"] = t[4:8].copy()
        L["cq"], L["ck"], L["cv"] = 1 / t[8], 1 / t[9], 1 / t[10]
        L["sinv"] = t[8] * t[9]
        L["vo"] = (1 / t[5]) * t[10]
        layers.append(L)
    m["layers"] = layers
    m["fnw"] = take(D * 4, np.float32, (D,))
    m["fnb"] = take(D * 4, np.float32, (D,))
    if head8:
        m["head_adq"] = float(take(16, np.float32, (4,))[0])
        m["hw"] = take(ntp * D, np.uint8, (ntp, D))
        m["hw_s"] = take(kb(ntp) * 8 * 4, np.float32, (kb(ntp), 8))
    else:
        m["hw"] = take(ntp * D * 2, np.uint16, (ntp, D))
    m["hb"] = take(ntp * 4, np.float32, (ntp,))
    assert off[0] == nbytes, f"layout mismatch ({off[0]} vs {nbytes} bytes)"
    return m
