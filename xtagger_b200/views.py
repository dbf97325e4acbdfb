"""Mixed whole-image / detail-crop batches built on the device with the GPU preprocessing (xtb_prep_ingest +
xtb_prep_crop): the PixAI-style workload, where every source image is tagged whole and as its four quadrant
crops, each view resampled to the 448^2 patch operand with the reference's antialiased bicubic (procimg.h:750-793
for the resample, the crop rectangles handed to pi_prep the same way procimg.h:1083-1124's crop selector hands
them over).

    views = mix_views(32)             # (source, x0, y0, cw, ch) per input
    prep = DevicePrep(896, 896, nsrc) # scratch for every source
    prep.run(src_ptrs, views, out_ptr, stream)
"""
import ctypes as C

import numpy as np

from . import lib as L

SIDE = 896
PER_SOURCE = 5  # the whole image, then its four quadrants


def mix_views(n, side=SIDE):
    """(source, x0, y0, cw, ch) for n inputs: n // 5 sources give their whole image and their four quadrants
    (top-left, top-right, bottom-left, bottom-right), then n % 5 further sources give their whole image only
    (32 inputs: 6 sources x 5 views + 2 whole images)."""
    full, extra = divmod(n, PER_SOURCE)
    half = side // 2
    out = []
    for s in range(full):
        out.append((s, 0, 0, side, side))
        for y0 in (0, half):
            for x0 in (0, half):
                out.append((s, x0, y0, half, half))
    for s in range(full, full + extra):
        out.append((s, 0, 0, side, side))
    return out


def mix_sources(nsrc, seed=1, side=SIDE):
    """nsrc seeded decoded images: side x side RGBX, uniform bytes (pixels uniform on [0, 1] in 1/255 steps), X = 255,
    uint8 [nsrc][side][4 side]."""
    rng = np.random.default_rng(seed)
    img = rng.integers(0, 256, (nsrc, side, side, 4), dtype=np.uint8)
    img[..., 3] = 255
    return img.reshape(nsrc, side, side * 4)


def num_sources(views):
    return 1 + max(v[0] for v in views) if views else 0


class DevicePrep:
    """Device scratch for nsrc decoded w x h images, and the launches that turn them into model inputs."""

    def __init__(self, w, h, nsrc, device=None):
        import torch
        self.lib = L.lib()
        self.w, self.h, self.stride = w, h, 4 * w
        self.nscr = self.lib.xtb_prep_scratch_bytes(w, h)
        self.scratch = torch.empty((max(1, nsrc), self.nscr), dtype=torch.uint8,
                                   device=device if device is not None else "cuda")

    def run(self, src_ptrs, views, out_ptr, stream, alpha=0):
        """Ingest every source that a view reads (alpha over white when `alpha`, the box pyramid), then write view i's
        input (EVA_IN halves) at out_ptr + i EVA_IN halves. src_ptrs[s]: device address of source s; stream: the
        cudaStream_t the launches are ordered on. Returns the number of kernels launched."""
        st = C.c_void_p(stream)
        used = sorted({v[0] for v in views})
        n = 0
        for s in used:
            scr = C.c_void_p(self.scratch[s].data_ptr())
            rc = self.lib.xtb_prep_ingest(C.c_void_p(src_ptrs[s]), self.w, self.h, self.stride, alpha, scr, st)
            L.check(rc, "xtb_prep_ingest")
            n += self.lib.xtb_prep_kernels(self.w, self.h, 0, 0, 0, 0)
        for i, (s, x0, y0, cw, ch) in enumerate(views):
            scr = C.c_void_p(self.scratch[s].data_ptr())
            dst = C.c_void_p(out_ptr + i * L.EVA_IN * 2)
            rc = self.lib.xtb_prep_crop(C.c_void_p(src_ptrs[s]), self.w, self.h, self.stride, x0, y0, cw, ch, scr,
                                        dst, st)
            L.check(rc, "xtb_prep_crop")
            n += self.lib.xtb_prep_kernels(self.w, self.h, x0, y0, cw, ch)
        return n
