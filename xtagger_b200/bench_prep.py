"""Throughput of the GPU preprocessing (xtb_prep_ingest + xtb_prep_crop: decoded RGBA image -> model input) on
seeded synthetic images, through the C ABI. Per workload (image size, alpha) one JSON line:
  device_img_s   images/s with the decoded images resident in HBM (a CUDA graph of `batch` images, CUDA events);
  e2e_img_s      the same including the copy of each decoded image from pinned host memory (H2D on the stream);
  gbs            decoded-image bytes read per second (device-resident);
  level          the pyramid level the whole-image resample reads from.
The reference does this step on the host (src/core/procimg.h, AVX2 per worker thread).

    python -m xtagger_b200.bench_prep [--batch 64] [--iters 10] [--sizes 0,1,2,3]
"""
import argparse
import ctypes as C
import json
import os
import sys

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
WORKLOADS = [(1024, 1024, 1), (1600, 1200, 0), (3000, 2000, 1), (448, 448, 0)]


def _level(w, h, S=448):
    """Pyramid level a whole-image resample reads from: halve while the next level's long side stays >= 2 S, then the
    coarsest level that still leaves a factor >= 2 (procimg.h:665-697)."""
    lw, lh, nlv = w, h, 1
    while nlv < 12 and (max(lw, lh) >> 1) >= 2 * S and lw >= 2 and lh >= 2:
        lw, lh, nlv = lw >> 1, lh >> 1, nlv + 1
    side, L = max(w, h), 0
    while L + 1 < nlv and (side >> (L + 1)) >= 2 * S:
        L += 1
    return L


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--batch", type=int, default=64)
    ap.add_argument("--iters", type=int, default=10)
    ap.add_argument("--sizes", default="", help="indices into the workload list (default: all)")
    a = ap.parse_args()
    sys.path.insert(0, ROOT)
    import torch
    from xtagger_b200 import lib as L
    xl = L.lib()
    rng = np.random.default_rng(5)
    pick = [int(i) for i in a.sizes.split(",") if i] or range(len(WORKLOADS))
    for w, h, alpha in (WORKLOADS[i] for i in pick):
        stride = 4 * w
        host = torch.from_numpy(rng.integers(0, 256, (a.batch, h, stride), dtype=np.uint8)).pin_memory()
        dev = host.cuda()
        nscr = xl.xtb_prep_scratch_bytes(w, h)
        scratch = torch.empty((a.batch, nscr), dtype=torch.uint8, device="cuda")
        out = torch.empty((a.batch, 1024 * 592), dtype=torch.int16, device="cuda")

        def step(copy):
            s = C.c_void_p(torch.cuda.current_stream().cuda_stream)
            for i in range(a.batch):
                if copy:
                    dev[i].copy_(host[i], non_blocking=True)
                p = C.c_void_p(dev[i].data_ptr())
                assert xl.xtb_prep_ingest(p, w, h, stride, alpha, C.c_void_p(scratch[i].data_ptr()), s) == 0
                assert xl.xtb_prep_crop(p, w, h, stride, 0, 0, w, h, C.c_void_p(scratch[i].data_ptr()),
                                        C.c_void_p(out[i].data_ptr()), s) == 0

        res = {}
        for copy in (False, True):
            step(copy)
            torch.cuda.synchronize()
            g = torch.cuda.CUDAGraph()
            st = torch.cuda.Stream()
            with torch.cuda.stream(st):
                with torch.cuda.graph(g, stream=st):
                    step(copy)
            g.replay()
            torch.cuda.synchronize()
            ts = []
            for _ in range(a.iters):
                e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                e0.record()
                g.replay()
                e1.record()
                torch.cuda.synchronize()
                ts.append(e0.elapsed_time(e1) * 1e-3)
            res[copy] = float(np.median(ts))
            del g
        assert xl.xtb_error_word(0) == 0
        print(json.dumps({"workload": f"{w}x{h} RGBA{' with alpha' if alpha else ''}, whole image -> 448^2 input",
                          "batch": a.batch, "level": _level(w, h),
                          "device_img_s": a.batch / res[False], "e2e_img_s": a.batch / res[True],
                          "us_per_img": res[False] / a.batch * 1e6,
                          "gbs": a.batch * h * stride / res[False] / 1e9,
                          "h2d_bytes_per_img": h * stride}), flush=True)


if __name__ == "__main__":
    main()
