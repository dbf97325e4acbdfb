"""Weight converter: a float EVA02-L tagger (the dict format of xtagger_b200.calib) plus its calibration statistics ->
eva02.bin, restating the reference's src/tools/export_eva.py step by step (the reference reads the float weights
from the upstream ONNX graph, absent here; everything after that is the same):

  * linear weights [out][in]; QKV fused with the softmax scale x log2 e folded into Wq (scores in the exp2 domain,
    export_eva.py:70-71, 86); fc1 g / x fused and interleaved in 16-unit chunks (export_eva.py:60-62); cls and the
    patch-embedding bias folded into the position table; RoPE table [1024][32] of (cos, sin) (export_eva.py:68-74);
  * SmoothQuant (alpha 0.5, s = clip(amax_act^alpha / amax_wcol^(1 - alpha), 1e-3, 1e3)) folded exactly into the
    producers: LN1 gamma / beta and the QKV columns, the Wv rows and the out-projection columns, LN2 and the fc1
    columns, the SwiGLU output and the fc2 columns (export_eva.py:52-58, 100-108);
  * the MLP LayerNorm folded into fc2: W~ = gamma W2, d = W2 beta, c = W~ 1 from the quantised W~ (export_eva.py:98-
    118), rs = 448 / (1.25 amax(h / s));
  * E4M3 with one scale per tensor (v3, export_eva.py:64-66), or with one fp32 scale per 128 x 128 block (v4, this
    library's block-scaled format; powers of two by default, which the tensor core applies itself); table [24][12] =
    w_dq x 4, a_dq x 4 (calibrated amax x 1.25 / 448), q, k, v;
  * every tensor on a 256-byte boundary, header "EVA2", version, tags, bytes, zero padding to 256 (export_eva.py:
    119-153); the head stays fp16.

    python -m xtagger_b200.convert float_model.npz eva02.bin float_model.calib [--v4]
"""
import argparse
import os
import struct

import numpy as np

from xtagger_b200 import model as M

D, T, NP, HID, HIDP, K0, K0P = 1024, 1025, 1024, 2730, 2736, 588, 592
E4M3 = 448.0
HEADROOM = 1.25   # export_eva.py:20
ALPHA = 0.5       # export_eva.py:21


def smooth(a, w):
    """SmoothQuant factors per input channel k: sqrt(amax_act[k] / amax over rows of |w[:, k]|) (export_eva.py:52-58)."""
    wa = np.abs(w).max(0)
    ok = (a > 0) & (wa > 0)
    s = np.ones_like(a)
    s[ok] = np.clip(a[ok] ** ALPHA / wa[ok] ** (1 - ALPHA), 1e-3, 1e3)
    return s


def fp8_tensor(w):
    """E4M3 with one scale per tensor (export_eva.py:64-66): codes, scale."""
    sc = float(np.abs(w).max()) / E4M3
    return M._e4m3(w / sc), sc


def convert(f, calib, path, version=3, pow2=True):
    """Write eva02.bin (version 3: per-tensor E4M3; 4: 128 x 128 block scales, powers of two unless pow2 is false, so
    that the engine's block-scaled MMA applies them) from the float model f and the calibration statistics (amax
    [nl][4][2736], qkv [nl][3][1024], h [nl][2736])."""
    assert version in (3, 4)
    from xtagger_b200 import calib as CB
    amax, qkvmax, hmax = calib
    nl = CB.num_layers(f)
    assert version == 4 or nl == 24, "v3 files hold 24 layers"
    qscale = float(f["attn_scale"]) * np.log2(np.e)
    cos, sin = f["rope.cos"], f["rope.sin"]
    assert (cos[:, 0::2] == cos[:, 1::2]).all() and (sin[:, 0::2] == sin[:, 1::2]).all()
    rope = np.stack([cos[:, 0::2], sin[:, 0::2]], -1).astype(np.float32)
    pe = np.zeros((D, K0P), np.float32)
    pe[:, :K0] = f["patch_embed.weight"]
    pos = f["pos_embed"].astype(np.float32).copy()
    pos[0] += f["cls_token"]
    pos[1:] += f["patch_embed.bias"][None, :]
    table = np.zeros((nl, 12), np.float32)
    layers = []
    for b in range(nl):
        p = f"blocks.{b}."
        w1, b1 = f[p + "norm1.weight"].astype(np.float32).copy(), f[p + "norm1.bias"].astype(np.float32).copy()
        wqkv = np.concatenate([f[p + "attn.q_proj.weight"] * qscale, f[p + "attn.k_proj.weight"],
                               f[p + "attn.v_proj.weight"]], 0).astype(np.float32)
        wo = f[p + "attn.proj.weight"].astype(np.float32).copy()
        w2, b2 = f[p + "norm2.weight"].astype(np.float32).copy(), f[p + "norm2.bias"].astype(np.float32).copy()
        w12 = np.zeros((2 * HIDP, D), np.float32)
        w12[:HID] = f[p + "mlp.fc1_g.weight"]
        w12[HIDP:HIDP + HID] = f[p + "mlp.fc1_x.weight"]
        mwp = np.zeros(HIDP, np.float32)
        mwp[:HID] = f[p + "mlp.norm.weight"]
        mbp = np.zeros(HIDP, np.float32)
        mbp[:HID] = f[p + "mlp.norm.bias"]
        wf2 = np.zeros((D, HIDP), np.float32)
        wf2[:, :HID] = f[p + "mlp.fc2.weight"]
        w12 = M.interleave_gx(w12)
        dn = (wf2 @ mbp).astype(np.float32)
        wf2 = wf2 * mwp[None, :]
        a = [amax[b, 0, :D], amax[b, 1, :D], amax[b, 2, :D], hmax[b]]
        s = [smooth(a[0], wqkv), smooth(a[1], wo), smooth(a[2], w12), smooth(a[3], wf2)]
        w1 /= s[0]
        b1 /= s[0]
        wqkv *= s[0]
        wqkv[2 * D:] /= s[1][:, None]
        wo *= s[1]
        w2 /= s[2]
        b2 /= s[2]
        w12 *= s[2]
        wf2 *= s[3]
        mats = []
        for k, w in enumerate((wqkv, wo, w12, wf2)):
            if version == 3:
                q, table[b, k] = fp8_tensor(w)
                mats.append((q, None, M.e4m3_decode(q) * table[b, k]))
            else:
                q, sc = M.quant_blocks(w, pow2=pow2)
                table[b, k] = 1.0
                mats.append((q, sc, M.dequant_blocks(q, sc)))
            table[b, 4 + k] = float((a[k] / s[k]).max()) * HEADROOM / E4M3
        table[b, 8] = float(qkvmax[b, 0].max()) * HEADROOM / E4M3
        table[b, 9] = float(qkvmax[b, 1].max()) * HEADROOM / E4M3
        table[b, 10] = float((qkvmax[b, 2] / s[1]).max()) * HEADROOM / E4M3
        rs = ((1.0 / table[b, 7]) / s[3]).astype(np.float32)           # raw h -> E4M3 operand
        c = (mats[3][2] / s[3][None, :]).sum(1).astype(np.float32)      # W~ 1 from the quantised W~
        layers.append((w1, b1, mats, w2, b2, rs, c, dn))
    nt = f["head.weight"].shape[0]
    ntp = (nt + 7) & ~7
    hw = np.zeros((ntp, D), np.float32)
    hw[:nt] = f["head.weight"]
    hb = np.zeros(ntp, np.float32)
    hb[:nt] = f["head.bias"]

    blob = M._Blob()
    blob.put(table, np.float32)
    blob.put(pe, np.float16)
    blob.put(pos, np.float32)
    blob.put(rope, np.float32)

    def put_mat(m):
        blob.put(m[0], np.uint8)
        if version == 4:
            blob.put(m[1], np.float32)

    for w1, b1, mats, w2, b2, rs, c, dn in layers:
        blob.put(w1, np.float32)
        blob.put(b1, np.float32)
        put_mat(mats[0])
        put_mat(mats[1])
        blob.put(w2, np.float32)
        blob.put(b2, np.float32)
        put_mat(mats[2])
        blob.put(rs, np.float32)
        put_mat(mats[3])
        blob.put(c, np.float32)
        blob.put(dn, np.float32)
    blob.put(f["fc_norm.weight"], np.float32)
    blob.put(f["fc_norm.bias"], np.float32)
    blob.put(hw, np.float16)
    blob.put(hb, np.float32)
    hdr = struct.pack("<4sIII", b"EVA2", version, nt, blob.n)
    if version == 4:
        hdr += struct.pack("<II", 0 if nl == 24 else nl, 0)  # fp16 head
    tmp = path + ".tmp"
    with open(tmp, "wb") as fh:
        fh.write(hdr + b"\0" * (256 - len(hdr)))
        for part in blob.parts:
            fh.write(part)
    os.replace(tmp, path)
    return path


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("model", help="float model: .npz of the arrays named in xtagger_b200.calib")
    ap.add_argument("out", help="eva02.bin to write")
    ap.add_argument("calib", help="calibration statistics (.calib, as written by xtagger_b200.calib.write_calib)")
    ap.add_argument("--v4", action="store_true", help="128 x 128 block scales instead of one scale per tensor")
    ap.add_argument("--free-scales", action="store_true", help="v4 block scales max / 448, not powers of two")
    a = ap.parse_args()
    from xtagger_b200 import calib as CB
    f = dict(np.load(a.model))
    convert(f, CB.read_calib(a.calib, CB.num_layers(f)), a.out, 4 if a.v4 else 3, pow2=not a.free_scales)
    print(f"{a.out}: v{4 if a.v4 else 3}, {f['head.weight'].shape[0]} tags")


if __name__ == "__main__":
    main()
