"""PixAI weight production: the fp16 calibration forward of the float ViTDet-L tagger (the reference's -DPX_CALIB
build of px.h, px.h:120-190 with cuBLAS GEMMs) and the converter to pixai.bin v3 (export_pixai.py:44-146; the
reference reads the float weights from the upstream ONNX graph, absent here; everything after that is the same).

Float model: a dict of float32 arrays (linear weights [out][in] as in PyTorch):
  patch_embed.weight [1024][588] (column c*196 + ky*14 + kx, RGB), pos_embed [576][1024] (one 24 x 24 window,
  tiled 3 x 3 over the 72 x 72 grid), ln_pre.weight / .bias, rope_win.cos / .sin [576][32] (window-local, row-major
  over 24 x 24), rope_glob.cos / .sin [5184][32] (row-major over 72 x 72), attn_scale (1/8);
  per block b: blocks.b.norm1.weight / .bias, blocks.b.attn.qkv.weight [3072][1024] / .bias, blocks.b.attn.proj.weight
  / .bias, blocks.b.norm2.weight / .bias, blocks.b.mlp.fc1.weight [4736][1024] / .bias, blocks.b.mlp.fc2.weight
  [1024][4736] / .bias; head_pool.norm.weight / .bias, head_pool.q [16][64] (the constant query), head_pool.scale,
  head_pool.kv.weight [2048][1024] / .bias (k | v), head_pool.pos_embed [5184][1024] (row-major),
  head_pool.proj.weight [1024][1024] / .bias, head.weight [nt][1024], head.bias [nt].
The block indices of the global blocks: global_blocks (default 7, 15, 23, 31).

Calibration statistics, as px_calib_dump writes <weights>.calib (px.h:436-453): amax [nl][4][4736] (QKV input = LN1
output, out-projection input = attention output, fc1 input = LN2 output, fc2 input = GELU output; the first three
use 1024 entries), then [nl][3 x 1024]: rotated q (carrying the softmax scale x log2 e) | rotated k | v.

    python -m xtagger_b200.pxconvert float_px.npz pixai.bin float_px.calib
"""
import argparse
import ctypes as C
import math
import os
import struct

import numpy as np

from . import model as M
from . import pixai as P

D, T, LW, HID, NH, HD, K0 = 1024, 5184, 576, 4736, 16, 64, 588
E4M3 = 448.0
HEADROOM = 1.25   # export_pixai.py:24
ALPHA = 0.5       # export_pixai.py:25


def num_layers(f):
    return sum(1 for k in f if k.endswith(".norm1.weight"))


def global_blocks(f):
    nl = num_layers(f)
    g = f.get("global_blocks")
    return [int(i) for i in g] if g is not None else [i for i in range(nl) if P.is_global(i)]


def synthetic_float(seed=0, nt=30877, nl=32, glob=None, std=0.02, ln_noise=1.0):
    """Random-init float PixAI tagger in the dict format above (seeded)."""
    rng = np.random.default_rng(seed)

    def randn(*shape):
        return rng.standard_normal(shape, dtype=np.float32) * std

    def ln(n):
        return ((1 + 0.1 * ln_noise * rng.standard_normal(n, dtype=np.float32)).astype(np.float32),
                (0.1 * ln_noise * rng.standard_normal(n, dtype=np.float32)).astype(np.float32))

    cw, cg = P.axial_rope(P.WS), P.axial_rope(P.GRID)
    f = {"patch_embed.weight": randn(D, K0), "pos_embed": randn(LW, D), "attn_scale": np.float32(1.0 / 8.0),
         "rope_win.cos": cw[:, :, 0].copy(), "rope_win.sin": cw[:, :, 1].copy(),
         "rope_glob.cos": cg[:, :, 0].copy(), "rope_glob.sin": cg[:, :, 1].copy()}
    f["ln_pre.weight"], f["ln_pre.bias"] = ln(D)
    for b in range(nl):
        p = f"blocks.{b}."
        f[p + "norm1.weight"], f[p + "norm1.bias"] = ln(D)
        f[p + "attn.qkv.weight"], f[p + "attn.qkv.bias"] = randn(3 * D, D), randn(3 * D)
        f[p + "attn.proj.weight"], f[p + "attn.proj.bias"] = randn(D, D), randn(D)
        f[p + "norm2.weight"], f[p + "norm2.bias"] = ln(D)
        f[p + "mlp.fc1.weight"], f[p + "mlp.fc1.bias"] = randn(HID, D), randn(HID)
        f[p + "mlp.fc2.weight"], f[p + "mlp.fc2.bias"] = randn(D, HID), randn(D)
    f["head_pool.norm.weight"], f["head_pool.norm.bias"] = ln(D)
    f["head_pool.q"] = rng.standard_normal((NH, HD), dtype=np.float32)
    f["head_pool.scale"] = np.float32(1.0 / math.sqrt(8.0))
    f["head_pool.kv.weight"], f["head_pool.kv.bias"] = randn(2 * D, D), randn(2 * D)
    f["head_pool.pos_embed"] = randn(T, D)
    f["head_pool.proj.weight"], f["head_pool.proj.bias"] = randn(D, D), randn(D)
    f["head.weight"], f["head.bias"] = randn(nt, D), randn(nt)
    if glob is not None:
        f["global_blocks"] = np.asarray(glob, np.int32)
    return f


def _tiled_pos(f):
    """pos [576] of one window tiled over the 3 x 3 windows, in window-major order (export_pixai.py:73-74)."""
    pos = f["pos_embed"].reshape(P.WS, P.WS, D)
    return np.tile(pos, (3, 3, 1)).reshape(T, D)[P.window_perm()].astype(np.float32)


class FloatPx:
    """The float model on one GPU: fp16 GEMMs (fp32 accumulation), fp32 LayerNorms and residual, fp16 attention,
    window-major tokens. forward() returns the tag scores; with calibrate=True it also folds the activation ranges
    into self.amax / self.qkv."""

    def __init__(self, f, device="cuda"):
        import torch
        self.torch = torch
        self.dev = torch.device(device)
        self.nl = num_layers(f)
        self.glob = set(global_blocks(f))
        t = lambda a, dt=torch.float16: torch.from_numpy(np.ascontiguousarray(a, np.float32)).to(self.dev, dt)  # noqa
        f32 = torch.float32
        self.qs = float(f["attn_scale"]) * math.log2(math.e)
        self.pe = t(f["patch_embed.weight"])
        self.pos = t(_tiled_pos(f), f32)
        self.lnp = (t(f["ln_pre.weight"], f32), t(f["ln_pre.bias"], f32))
        perm = P.window_perm()
        self.cs_w = (t(f["rope_win.cos"], f32), t(f["rope_win.sin"], f32))
        self.cs_g = (t(f["rope_glob.cos"][perm], f32), t(f["rope_glob.sin"][perm], f32))
        self.L = []
        for b in range(self.nl):
            p = f"blocks.{b}."
            wqkv = f[p + "attn.qkv.weight"].copy()
            bqkv = f[p + "attn.qkv.bias"].copy()
            wqkv[:D] *= self.qs
            bqkv[:D] *= self.qs
            self.L.append(dict(
                n1=(t(f[p + "norm1.weight"], f32), t(f[p + "norm1.bias"], f32)),
                wqkv=t(wqkv), bqkv=t(bqkv, f32), wo=t(f[p + "attn.proj.weight"]), bo=t(f[p + "attn.proj.bias"], f32),
                n2=(t(f[p + "norm2.weight"], f32), t(f[p + "norm2.bias"], f32)),
                w1=t(f[p + "mlp.fc1.weight"]), b1=t(f[p + "mlp.fc1.bias"], f32),
                w2=t(f[p + "mlp.fc2.weight"]), b2=t(f[p + "mlp.fc2.bias"], f32)))
        self.hn = (t(f["head_pool.norm.weight"], f32), t(f["head_pool.norm.bias"], f32))
        self.hpos = t(f["head_pool.pos_embed"][perm], f32)
        kvw, kvb = f["head_pool.kv.weight"], f["head_pool.kv.bias"]
        self.hq = t(f["head_pool.q"], f32)
        self.hscale = float(f["head_pool.scale"])
        self.wk, self.bk = t(kvw[:D], f32), t(kvb[:D], f32)
        self.wv, self.bv = t(kvw[D:], f32), t(kvb[D:], f32)
        self.wp, self.bp = t(f["head_pool.proj.weight"], f32), t(f["head_pool.proj.bias"], f32)
        self.hw, self.hb = t(f["head.weight"], f32), t(f["head.bias"], f32)
        self.amax = torch.zeros((self.nl, 4, HID), dtype=f32, device=self.dev)
        self.qkv = torch.zeros((self.nl, 3, D), dtype=f32, device=self.dev)

    def _amax(self, x16, out):
        """out[:k] = max(out, max over rows |x16|): this library's xtb_amax_f16 kernel."""
        from xtagger_b200 import lib as L
        torch = self.torch
        x16 = x16.reshape(-1, x16.shape[-1]).contiguous()
        st = C.c_void_p(torch.cuda.current_stream(self.dev).cuda_stream)
        rc = L.lib().xtb_amax_f16(C.c_void_p(x16.data_ptr()), x16.shape[1], x16.shape[0], C.c_void_p(out.data_ptr()), st)
        assert rc == 0, "xtb_amax_f16 failed"

    def _ln(self, x, wb, eps):
        return self.torch.nn.functional.layer_norm(x, (x.shape[-1],), wb[0], wb[1], eps)

    def forward(self, inputs, calibrate=False):
        """inputs: uint16 patch operands [n][5184][592] (fp16 bits, window-major). Returns fp32 scores [n][nt]."""
        torch = self.torch
        F = torch.nn.functional
        n = inputs.shape[0]
        a = torch.from_numpy(np.ascontiguousarray(inputs).view(np.float16)).to(self.dev)[:, :, :K0]
        x = (a @ self.pe.t()).half().float() + self.pos
        x = self._ln(x, self.lnp, 1e-5).half().float()
        for i, L in enumerate(self.L):
            glob = i in self.glob
            Ls = T if glob else LW
            cos, sin = self.cs_g if glob else self.cs_w
            h = self._ln(x, L["n1"], 1e-6).half()
            if calibrate:
                self._amax(h, self.amax[i, 0, :D])
            qkv = ((h @ L["wqkv"].t()).float() + L["bqkv"]).view(n * T // Ls, Ls, 3, NH, HD)
            q, k, v = qkv[:, :, 0], qkv[:, :, 1], qkv[:, :, 2]
            c = cos.view(1, Ls, 1, 32).repeat_interleave(2, -1)
            s = sin.view(1, Ls, 1, 32).repeat_interleave(2, -1)
            for u in (q, k):  # interleaved RoPE on every token: (f0, f1) -> (f0 c - f1 s, f1 c + f0 s)
                rot = torch.stack([-u[..., 1::2], u[..., 0::2]], -1).flatten(-2)
                u.copy_(u * c + rot * s)
            q, k, v = q.half(), k.half(), v.half()
            if calibrate:
                for j, u in enumerate((q, k, v)):
                    self._amax(u.reshape(-1, D), self.qkv[i, j])
            # q carries scale x log2 e: softmax(q k^T ln 2) = 2^s / sum 2^s, the reference's exp2-domain softmax
            o = F.scaled_dot_product_attention(q.transpose(1, 2), k.transpose(1, 2), v.transpose(1, 2),
                                               scale=math.log(2.0))
            o = o.transpose(1, 2).reshape(n * T, D).contiguous()
            if calibrate:
                self._amax(o, self.amax[i, 1, :D])
            x = x.view(n * T, D) + (o @ L["wo"].t()).float() + L["bo"]
            h = self._ln(x, L["n2"], 1e-6).half()
            if calibrate:
                self._amax(h, self.amax[i, 2, :D])
            u = F.gelu((h @ L["w1"].t()).float() + L["b1"]).half()
            if calibrate:
                self._amax(u, self.amax[i, 3])
            x = (x + (u @ L["w2"].t()).float() + L["b2"]).half().float()
        x = x.view(n, T, D)
        y = self._ln(x, self.hn, 1e-5) + self.hpos
        kk = (y @ self.wk.t() + self.bk).view(n, T, NH, HD)
        sc = torch.einsum("nthd,hd->nht", kk, self.hq) * self.hscale
        pw = torch.softmax(sc, -1)                                       # [n][16][T]
        vv = (y @ self.wv.t() + self.bv).view(n, T, NH, HD)
        pooled = torch.einsum("nht,nthd->nhd", pw, vv).reshape(n, D)
        logits = (pooled @ self.wp.t() + self.bp) @ self.hw.t() + self.hb
        return torch.sigmoid(logits).cpu().numpy()

    def calibrate(self, inputs, batch=2):
        for s in range(0, inputs.shape[0], batch):
            self.forward(inputs[s:s + batch], calibrate=True)
        self.torch.cuda.synchronize(self.dev)
        return self.amax.cpu().numpy(), self.qkv.cpu().numpy()


def write_calib(path, amax, qkv):
    """px_calib_dump's layout: float [nl][4][4736], then [nl][3 x 1024]."""
    with open(path, "wb") as fh:
        for a in (amax, qkv):
            fh.write(np.ascontiguousarray(a, np.float32).tobytes())


def read_calib(path, nl=32):
    raw = np.fromfile(path, np.float32)
    na = nl * 4 * HID
    return raw[:na].reshape(nl, 4, HID), raw[na:na + nl * 3 * D].reshape(nl, 3, D)


def smooth(a, w):
    """SmoothQuant factors per input channel (export_pixai.py:49-54)."""
    wa = np.abs(w).max(0)
    ok = (a > 0) & (wa > 0)
    s = np.ones_like(a)
    s[ok] = np.clip(a[ok] ** ALPHA / wa[ok] ** (1 - ALPHA), 1e-3, 1e3)
    return s


def convert(f, calib, path):
    """Write pixai.bin v3 from the float model f and its calibration statistics (amax [nl][4][4736],
    qkv [nl][3][1024]), step by step as export_pixai.py:66-146."""
    amax, qkvmax = calib
    nl = num_layers(f)
    glob = global_blocks(f)
    gmask = 0 if glob == [i for i in range(nl) if P.is_global(i)] else sum(1 << i for i in glob)
    qs = float(f["attn_scale"]) * np.log2(np.e)
    perm = P.window_perm()
    pe = np.zeros((D, P.K0P), np.float32)
    pe[:, :K0] = f["patch_embed.weight"]
    cs_win = np.stack([f["rope_win.cos"], f["rope_win.sin"]], -1).astype(np.float32)
    cs_glob = np.stack([f["rope_glob.cos"], f["rope_glob.sin"]], -1).astype(np.float32)[perm]
    table = np.zeros((nl, 12), np.float32)
    layers = []
    for b in range(nl):
        p = f"blocks.{b}."
        w1, b1 = f[p + "norm1.weight"].astype(np.float32).copy(), f[p + "norm1.bias"].astype(np.float32).copy()
        wqkv, bqkv = f[p + "attn.qkv.weight"].astype(np.float32).copy(), f[p + "attn.qkv.bias"].astype(np.float32).copy()
        wqkv[:D] *= qs
        bqkv[:D] *= qs
        wo, bo = f[p + "attn.proj.weight"].astype(np.float32).copy(), f[p + "attn.proj.bias"].astype(np.float32)
        w2, b2 = f[p + "norm2.weight"].astype(np.float32).copy(), f[p + "norm2.bias"].astype(np.float32).copy()
        wf1, bf1 = f[p + "mlp.fc1.weight"].astype(np.float32).copy(), f[p + "mlp.fc1.bias"].astype(np.float32)
        wf2, bf2 = f[p + "mlp.fc2.weight"].astype(np.float32).copy(), f[p + "mlp.fc2.bias"].astype(np.float32)
        a = [amax[b, 0, :D], amax[b, 1, :D], amax[b, 2, :D], amax[b, 3]]
        s = [smooth(a[0], wqkv), smooth(a[1], wo), smooth(a[2], wf1), smooth(a[3], wf2)]
        w1 /= s[0]
        b1 /= s[0]
        wqkv *= s[0]
        wqkv[2 * D:] /= s[1][:, None]
        bqkv[2 * D:] /= s[1]
        wo *= s[1]
        w2 /= s[2]
        b2 /= s[2]
        wf1 *= s[2]
        wf2 *= s[3]
        mats = []
        for k, w in enumerate((wqkv, wo, wf1, wf2)):
            q, table[b, k] = M.quant_tensor(w)
            mats.append(q)
            table[b, 4 + k] = float((a[k] / s[k]).max()) * HEADROOM / E4M3
        table[b, 8] = float(qkvmax[b, 0].max()) * HEADROOM / E4M3
        table[b, 9] = float(qkvmax[b, 1].max()) * HEADROOM / E4M3
        table[b, 10] = float((qkvmax[b, 2] / s[1]).max()) * HEADROOM / E4M3
        rs = ((1.0 / table[b, 7]) / s[3]).astype(np.float32)
        layers.append((w1, b1, mats, bqkv, bo, w2, b2, bf1, rs, bf2))
    # attention-pool head (export_pixai.py:106-122): the constant query folds into the key projection
    hq = f["head_pool.q"].astype(np.float64)
    kvw, kvb = f["head_pool.kv.weight"].astype(np.float64), f["head_pool.kv.bias"].astype(np.float64)
    ks = float(f["head_pool.scale"]) * np.log2(np.e)
    U = np.stack([kvw[HD * h:HD * h + HD].T @ hq[h] for h in range(NH)]) * ks      # [16][1024]; q . bk cancels
    hpos = f["head_pool.pos_embed"][perm]
    wv, bv = kvw[D:], kvb[D:]
    wp, bp = f["head_pool.proj.weight"].astype(np.float64), f["head_pool.proj.bias"].astype(np.float64)
    hw, hb = f["head.weight"].astype(np.float64), f["head.bias"].astype(np.float64)
    hb = hw @ (wp @ bv + bp) + hb
    hw = hw @ wp
    nt = hw.shape[0]
    ntp = (nt + 7) & ~7
    hwp = np.zeros((ntp, D), np.float32)
    hwp[:nt] = hw
    hbp = np.zeros(ntp, np.float32)
    hbp[:nt] = hb

    blob = M._Blob()
    blob.put(table, np.float32)
    blob.put(pe, np.float16)
    blob.put(_tiled_pos(f), np.float32)
    blob.put(f["ln_pre.weight"], np.float32)
    blob.put(f["ln_pre.bias"], np.float32)
    blob.put(cs_win, np.float32)
    blob.put(cs_glob, np.float32)
    for w1, b1, mats, bqkv, bo, w2, b2, bf1, rs, bf2 in layers:
        blob.put(w1, np.float32)
        blob.put(b1, np.float32)
        blob.put(mats[0], np.uint8)
        blob.put(bqkv, np.float32)
        blob.put(mats[1], np.uint8)
        blob.put(bo, np.float32)
        blob.put(w2, np.float32)
        blob.put(b2, np.float32)
        blob.put(mats[2], np.uint8)
        blob.put(bf1, np.float32)
        blob.put(rs, np.float32)
        blob.put(mats[3], np.uint8)
        blob.put(bf2, np.float32)
    blob.put(f["head_pool.norm.weight"], np.float32)
    blob.put(f["head_pool.norm.bias"], np.float32)
    blob.put(U, np.float32)
    blob.put(hpos, np.float16)
    blob.put(wv, np.float16)
    blob.put(hwp, np.float16)
    blob.put(hbp, np.float32)
    hdr = struct.pack("<4sIIIII", b"PXAI", 3, nt, blob.n, 0 if nl == P.NL else nl, gmask)
    tmp = path + ".tmp"
    with open(tmp, "wb") as fh:
        fh.write(hdr + b"\0" * (256 - len(hdr)))
        for part in blob.parts:
            fh.write(part)
    os.replace(tmp, path)
    return path


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("model", help="float model: .npz of the arrays named in xtagger_b200.pxconvert")
    ap.add_argument("out", help="pixai.bin to write")
    ap.add_argument("calib", help="calibration statistics (.calib, as written by write_calib)")
    a = ap.parse_args()
    f = dict(np.load(a.model))
    convert(f, read_calib(a.calib, num_layers(f)), a.out)
    print(f"{a.out}: v3, {f['head.weight'].shape[0]} tags")


if __name__ == "__main__":
    main()
