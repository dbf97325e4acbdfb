"""Calibration engine: the fp16 forward of the float EVA02-L tagger that records the static activation ranges the
FP8 weight file needs (the reference's -DEVA_CALIB build of eva.h, which runs the fp16 "v2" weights with cuBLAS
GEMMs and records per-channel |max| with k_amax, eva.h:226-310, kern_common.cuh:194-217).

Recorded per layer, as eva_calib_dump (eva.h:682-701) writes them to <weights>.calib:
  amax[l][0][:1024]  LN1 output (QKV input)          amax[l][1][:1024]  attention output (out-projection input)
  amax[l][2][:1024]  LN2 output (fc1 input)          amax[l][3][:2730]  MLP-LayerNorm output (fc2 input)
  qkv[l][0 | 1 | 2]  rotated q (carrying the softmax scale x log2 e, as the v2 weights do) | rotated k | v
  h[l][:2730]        raw SwiGLU output silu(g) x
The statistic itself is this library's xtb_amax_f16 kernel on the fp16 tensors; the GEMMs, LayerNorms and the
attention are PyTorch's (library kernels, as the reference's calibration engine uses cuBLAS): this is the offline
float reference of the model, not the FP8 hot path.

The float model is a dict of float32 arrays (names below; linear weights [out][in] as in PyTorch, so the tensors
export_eva.py reads from the ONNX graph, transposed): patch_embed.weight [1024][588] (column c * 196 + ky * 14 + kx
in the patch operand's BGR order), patch_embed.bias, cls_token [1024], pos_embed [1025][1024], rope.cos / rope.sin
[1024][64] (pairs 2j, 2j + 1 share an angle), attn_scale (1 / sqrt(64)), and per block b: blocks.b.norm1.weight /
.bias, blocks.b.attn.{q,k,v}_proj.weight, blocks.b.attn.proj.weight, blocks.b.norm2.weight / .bias,
blocks.b.mlp.fc1_g.weight / fc1_x.weight [2730][1024], blocks.b.mlp.norm.weight / .bias [2730],
blocks.b.mlp.fc2.weight [1024][2730]; then fc_norm.weight / .bias, head.weight [nt][1024], head.bias [nt].
"""
import ctypes as C
import math

import numpy as np

D, T, NP, HID, HIDP, K0, NH, HD = 1024, 1025, 1024, 2730, 2736, 588, 16, 64
EPS = 1e-6


def synthetic_float(seed=0, nt=10861, nl=24, std=0.02, ln_noise=1.0, qk_std=None, out_std=None):
    """Random-init float EVA02-L tagger in the dict format above (seeded). Every weight is N(0, std) unless
    qk_std / out_std give the query and key projections or the two residual-branch outputs (attention output
    projection, fc2) their own standard deviation (see realistic_float)."""
    from xtagger_b200 import model as M
    rng = np.random.default_rng(seed)

    def randn(*shape, s=std):
        return rng.standard_normal(shape, dtype=np.float32) * s

    def ln(n):
        return ((1 + 0.1 * ln_noise * rng.standard_normal(n, dtype=np.float32)).astype(np.float32),
                (0.1 * ln_noise * rng.standard_normal(n, dtype=np.float32)).astype(np.float32))

    f = {"patch_embed.weight": randn(D, K0), "patch_embed.bias": randn(D), "cls_token": randn(D),
         "pos_embed": randn(T, D), "attn_scale": np.float32(1.0 / math.sqrt(HD))}
    cs = M.rope_table()  # [1024][32][2]
    f["rope.cos"] = np.repeat(cs[:, :, 0], 2, axis=1).astype(np.float32)
    f["rope.sin"] = np.repeat(cs[:, :, 1], 2, axis=1).astype(np.float32)
    for b in range(nl):
        p = f"blocks.{b}."
        f[p + "norm1.weight"], f[p + "norm1.bias"] = ln(D)
        for n, s in (("q_proj", qk_std), ("k_proj", qk_std), ("v_proj", None), ("proj", out_std)):
            f[p + f"attn.{n}.weight"] = randn(D, D, s=std if s is None else s)
        f[p + "norm2.weight"], f[p + "norm2.bias"] = ln(D)
        f[p + "mlp.fc1_g.weight"] = randn(HID, D)
        f[p + "mlp.fc1_x.weight"] = randn(HID, D)
        f[p + "mlp.norm.weight"], f[p + "mlp.norm.bias"] = ln(HID)
        f[p + "mlp.fc2.weight"] = randn(D, HID, s=std if out_std is None else out_std)
    f["fc_norm.weight"], f["fc_norm.bias"] = ln(D)
    f["head.weight"] = randn(nt, D)
    f["head.bias"] = np.zeros(nt, np.float32)
    return f


def num_layers(f):
    return sum(1 for k in f if k.endswith(".norm1.weight"))


class FloatEva:
    """The float model on one GPU: fp16 GEMMs (fp32 accumulation), fp32 LayerNorms and residual, fp16 attention.
    forward() returns the tag scores; with calibrate=True it also folds the activation ranges into self.amax,
    self.qkv, self.h (numpy views of the device statistics after sync()).
    device="cpu" runs the same model on the host (fp16-rounded operands, fp32 products, torch's own max for the
    statistics) for small test fixtures that should launch nothing on the GPU."""

    def __init__(self, f, device="cuda"):
        import torch
        self.torch = torch
        self.dev = torch.device(device)
        self.cpu = self.dev.type == "cpu"
        self.nl = num_layers(f)

        def t(a, dt=torch.float16):
            w = torch.from_numpy(np.ascontiguousarray(a, np.float32)).to(dt)
            return (w.float() if self.cpu else w).to(self.dev)
        self.qscale = float(f["attn_scale"]) * math.log2(math.e)
        self.pe_w, self.pe_b = t(f["patch_embed.weight"]), t(f["patch_embed.bias"], torch.float32)
        pos = f["pos_embed"].astype(np.float32).copy()
        pos[0] += f["cls_token"]
        self.pos = t(pos, torch.float32)
        self.cos = t(f["rope.cos"], torch.float32)
        self.sin = t(f["rope.sin"], torch.float32)
        self.L = []
        for b in range(self.nl):
            p = f"blocks.{b}."
            self.L.append(dict(
                n1=(t(f[p + "norm1.weight"], torch.float32), t(f[p + "norm1.bias"], torch.float32)),
                wqkv=t(np.concatenate([f[p + "attn.q_proj.weight"] * self.qscale, f[p + "attn.k_proj.weight"],
                                       f[p + "attn.v_proj.weight"]], 0)),
                wo=t(f[p + "attn.proj.weight"]),
                n2=(t(f[p + "norm2.weight"], torch.float32), t(f[p + "norm2.bias"], torch.float32)),
                wg=t(f[p + "mlp.fc1_g.weight"]), wx=t(f[p + "mlp.fc1_x.weight"]),
                nm=(t(f[p + "mlp.norm.weight"], torch.float32), t(f[p + "mlp.norm.bias"], torch.float32)),
                w2=t(f[p + "mlp.fc2.weight"])))
        self.fn = (t(f["fc_norm.weight"], torch.float32), t(f["fc_norm.bias"], torch.float32))
        self.hw, self.hb = t(f["head.weight"]), t(f["head.bias"], torch.float32)
        self.amax = torch.zeros((self.nl, 4, HIDP), dtype=torch.float32, device=self.dev)
        self.qkv = torch.zeros((self.nl, 3, D), dtype=torch.float32, device=self.dev)
        self.h = torch.zeros((self.nl, HIDP), dtype=torch.float32, device=self.dev)

    def _half(self, x):
        """Round to fp16 (kept in fp32 on the host)."""
        return x.half().float() if self.cpu else x.half()

    def _amax(self, x16, out):
        """out[:k] = max(out, max over rows |x16|): the xtb_amax_f16 kernel (columns padded to a multiple of 8)."""
        from xtagger_b200 import lib as L
        torch = self.torch
        if self.cpu:
            m = x16.reshape(-1, x16.shape[-1]).abs().amax(0)
            out[:m.shape[0]] = torch.maximum(out[:m.shape[0]], m)
            return
        x16 = x16.reshape(-1, x16.shape[-1])
        k = x16.shape[1]
        if k % 8:
            x16 = torch.nn.functional.pad(x16, (0, 8 - k % 8))
        x16 = x16.contiguous()
        st = C.c_void_p(torch.cuda.current_stream(self.dev).cuda_stream)
        rc = L.lib().xtb_amax_f16(C.c_void_p(x16.data_ptr()), x16.shape[1], x16.shape[0], C.c_void_p(out.data_ptr()), st)
        assert rc == 0, "xtb_amax_f16 failed"

    def _ln(self, x, wb):
        return self.torch.nn.functional.layer_norm(x, (x.shape[-1],), wb[0], wb[1], EPS)

    def forward(self, inputs, calibrate=False):
        """inputs: uint16 patch operands [n][1024][592] (fp16 bits). Returns fp32 scores [n][nt]."""
        pn = self._trunk(inputs, calibrate)
        logits = (pn @ self.hw.t()).float() + self.hb
        return self.torch.sigmoid(logits).cpu().numpy()

    def features(self, inputs, batch=8):
        """The head's input: fc_norm of the token mean, fp32 [n][1024] (fp16 values)."""
        return np.concatenate([self._trunk(inputs[s:s + batch]).float().cpu().numpy()
                               for s in range(0, inputs.shape[0], batch)])

    def _trunk(self, inputs, calibrate=False):
        torch = self.torch
        F = torch.nn.functional
        n = inputs.shape[0]
        a = torch.from_numpy(np.ascontiguousarray(inputs).view(np.float16)).to(self.dev)[:, :, :K0]
        if self.cpu:
            a = a.float()
        xp = (a @ self.pe_w.t()).float() + self.pe_b
        x = torch.empty((n, T, D), dtype=torch.float32, device=self.dev)
        x[:, 0] = 0
        x[:, 1:] = xp
        x += self.pos
        for i, L in enumerate(self.L):
            h = self._half(self._ln(x, L["n1"]))
            if calibrate:
                self._amax(h, self.amax[i, 0])
            qkv = (h @ L["wqkv"].t()).float().view(n, T, 3, NH, HD)
            q, k, v = qkv[:, :, 0], qkv[:, :, 1], qkv[:, :, 2]
            for u in (q, k):  # interleaved RoPE on the patch tokens: (f0, f1) -> (f0 c - f1 s, f1 c + f0 s)
                pt = u[:, 1:]
                c = self.cos.view(1, NP, 1, HD)
                s = self.sin.view(1, NP, 1, HD)
                rot = torch.stack([-pt[..., 1::2], pt[..., 0::2]], -1).flatten(-2)
                u[:, 1:] = pt * c + rot * s
            q, k, v = self._half(q), self._half(k), self._half(v)
            if calibrate:
                for j, u in enumerate((q, k, v)):
                    self._amax(u.reshape(n * T, D), self.qkv[i, j])
            # q carries scale x log2 e: softmax(q k^T ln 2) = 2^s / sum 2^s, the reference's exp2-domain softmax
            o = F.scaled_dot_product_attention(q.transpose(1, 2), k.transpose(1, 2), v.transpose(1, 2),
                                               scale=math.log(2.0))
            o = self._half(o.transpose(1, 2).reshape(n, T, D).contiguous())
            if calibrate:
                self._amax(o, self.amax[i, 1])
            x += (o @ L["wo"].t()).float()
            h = self._half(self._ln(x, L["n2"]))
            if calibrate:
                self._amax(h, self.amax[i, 2])
            g = (h @ L["wg"].t()).float()
            u = F.silu(g) * (h @ L["wx"].t()).float()
            m = self._half(self._ln(u, L["nm"]))
            if calibrate:
                self._amax(self._half(u), self.h[i])
                self._amax(m, self.amax[i, 3])
            x += (m @ L["w2"].t()).float()
        pooled = x[:, 1:].mean(1)
        return self._half(self._ln(pooled, self.fn))

    def calibrate(self, inputs, batch=8):
        """Fold the activation ranges of these inputs into the statistics; returns (amax, qkv, h) as numpy."""
        for s in range(0, inputs.shape[0], batch):
            self.forward(inputs[s:s + batch], calibrate=True)
        if not self.cpu:
            self.torch.cuda.synchronize(self.dev)
        return self.amax.cpu().numpy(), self.qkv.cpu().numpy(), self.h.cpu().numpy()


def write_calib(path, amax, qkv, h):
    """The reference's <weights>.calib layout: float [nl][4][2736], then [nl][3 x 1024], then [nl][2736]."""
    with open(path, "wb") as fh:
        for a in (amax, qkv, h):
            fh.write(np.ascontiguousarray(a, np.float32).tobytes())


def read_calib(path, nl=24):
    raw = np.fromfile(path, np.float32)
    na, nq = nl * 4 * HIDP, nl * 3 * D
    return (raw[:na].reshape(nl, 4, HIDP), raw[na:na + nq].reshape(nl, 3, D),
            raw[na + nq:na + nq + nl * HIDP].reshape(nl, HIDP))


# ---- a float model with a stable FP8 forward, for end-to-end parity at the score tolerance ----
#
# On the random-init model (every weight N(0, 0.02), head bias 0, uniform-noise images) the FP8 forward is chaotic:
# every GEMM input and every attention probability is re-quantised to E4M3 (3 mantissa bits), so a difference in the
# last bit of an fp32 sum flips a rounding decision with probability (difference / step), and a flip costs a whole
# step. The root-mean-square difference after one quantisation is sqrt(step x difference): two implementations that
# differ only in summation order reach the E4M3 noise level within a few layers. What reaches the scores is that noise
# over the head's input: uniform-noise images have no image-level content (the token mean barely moves between
# images), flat attention makes the attention noise the same for every token (it does not average out in the pool),
# and a head spread over all 1024 directions picks up all of it. A trained tagger differs on all three counts, and
# realistic_model() builds one that does too:
#   * inputs with image-level statistics (model.structured_inputs): the token mean carries the image;
#   * query / key projections N(0, 0.06): attention over some 50 keys instead of all 1025, so rounding noise differs
#     between tokens and averages out in the pool;
#   * residual-branch outputs (attention output projection, fc2) N(0, 0.0005): over 24 layers the blocks add about a
#     fifth of the residual stream's variance instead of dominating it;
#   * the head fitted as a linear probe on the float model's features: tag rows in the span of the top principal
#     directions of the head input over a set of images, each scaled to a logit spread of 1.5 between images, biases
#     centred to -5 +- 0.7 (between a few and a few dozen of the 10861 tags above 0.35 per image, most near zero).
# On this model the oracle on inputs one fp16 ulp apart differs by about 2e-4 in the 24-layer scores (on the
# random-init model: 4e-2), a tenth of the north-star tolerance.

def realistic_float(seed=0, nt=10861, nl=24):
    """The float model of realistic_model() before its head is fitted (probe_head)."""
    return synthetic_float(seed=seed, nt=nt, nl=nl, qk_std=0.06, out_std=0.0005)


def probe_head(f, pn, k=3, spread=1.5, base=-5.0, base_std=0.7, seed=0):
    """Fit the tag head of float model f as a linear probe on its features pn [n][1024] (FloatEva.features): every
    row a random combination of the top k principal directions of pn, scaled so that its logit has standard
    deviation `spread` over these images, with the bias centring the logit at base + N(0, base_std)."""
    pn = np.asarray(pn, np.float64)
    mu = pn.mean(0)
    _, _, vt = np.linalg.svd(pn - mu, full_matrices=False)
    rng = np.random.default_rng(seed)
    nt = f["head.weight"].shape[0]
    hw = rng.standard_normal((nt, k)) @ vt[:k]
    hw *= (spread / ((pn - mu) @ hw.T).std(0))[:, None]
    f["head.weight"] = hw.astype(np.float32)
    f["head.bias"] = (base - hw @ mu + base_std * rng.standard_normal(nt)).astype(np.float32)
    return f


def realistic_model(path, seed=0, nl=24, version=3, nt=10861, pow2=True, device="cuda", ncal=4, nprobe=16):
    """Write an eva02.bin of the stable model described above: float model -> calibration on ncal structured images
    (FloatEva, the fp16 float forward, on `device`) -> linear-probe head on nprobe more -> convert (the reference's
    export_eva.py steps: SmoothQuant, per-tensor E4M3 for version 3, 128 x 128 block scales for version 4)."""
    from xtagger_b200 import convert as CV
    from xtagger_b200 import model as M
    f = realistic_float(seed=seed, nt=nt, nl=nl)
    fe = FloatEva(f, device=device)
    stats = fe.calibrate(M.structured_inputs(ncal, seed=seed + 100), batch=4)
    pn = fe.features(M.structured_inputs(nprobe, seed=seed + 200))
    del fe
    probe_head(f, pn, seed=seed + 9)
    return CV.convert(f, stats, path, version=version, pow2=pow2)
