"""Device time of the reference's own FP8 forward on this GPU (baseline infrastructure; run on the GPU box).

The reference's kernels (eva_kernels.cu, built by oracle/Makefile `ref` into oracle/_ref/libref_kernels.so) replay
eva_forward (eva.h:252-307) on a random-init 24-layer v3 model with seeded synthetic inputs, captured in a CUDA
graph as the reference does; CUDA events around `iters` graph launches after `warmup`. Prints one JSON line per
batch size: images/s with inputs resident on the device, the same measurement bench.py's `value` makes.

    python oracle/ref_time.py [--batch 8 64] [--iters 10] [--warmup 3]
    python oracle/ref_time.py --pixai [--batch 4 8]    # the reference's PixAI forward (px_kernels.cu, px.h:115-190)
"""
import argparse
import ctypes as C
import json
import os
import sys
import tempfile

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--batch", type=int, nargs="+", default=[8, 64])
    ap.add_argument("--iters", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--nt", type=int, default=None)
    ap.add_argument("--pixai", action="store_true", help="the PixAI forward (full 32-block model, 30877 tags)")
    a = ap.parse_args()
    if a.pixai:
        return pixai(a)
    a.nt = a.nt or 10861
    for line in reference_kernels(a.batch, a.warmup, a.iters, a.nt):
        print(json.dumps(line), flush=True)


def reference_kernels(batches, warmup=3, iters=10, nt=10861):
    """One dict per batch size: the reference's eva_forward replayed as a CUDA graph on GPU 0 (inputs resident)."""
    import torch
    if not torch.cuda.is_available():
        raise RuntimeError("no CUDA device")
    from xtagger_b200 import model as M
    so = os.path.join(ROOT, "oracle", "_ref", "libref_kernels.so")
    if not os.path.exists(so):
        raise FileNotFoundError(so + " not built (oracle/Makefile ref, where the reference sources are present)")
    lib = C.CDLL(so)
    lib.ref_forward_time.restype = C.c_int
    lib.ref_forward_time.argtypes = [C.c_char_p, np.ctypeslib.ndpointer(np.uint16, flags="C_CONTIGUOUS"), C.c_int,
                                     C.c_int, C.c_int, C.POINTER(C.c_float)]
    path = M.write_synthetic(os.path.join(tempfile.mkdtemp(), "v3.bin"), seed=0, nt=nt, nl=24, version=3,
                             head_fp8=False)
    out = []
    try:
        for nb in batches:
            x = np.ascontiguousarray(M.synthetic_inputs(nb, seed=1))
            ms = C.c_float(0)
            if lib.ref_forward_time(path.encode(), x, nb, warmup, iters, C.byref(ms)):
                raise RuntimeError("reference forward failed")
            out.append({"impl": "reference kernels (eva_kernels.cu, mma.sync E4M3) on this GPU", "batch": nb,
                        "ms_per_forward": ms.value, "images_per_s": nb / (ms.value * 1e-3),
                        "model": f"v3, 24 layers, fp16 head, {nt} tags, random-init"})
    finally:
        os.remove(path)
    return out


def pixai(a):
    from xtagger_b200 import pixai as P
    lib = C.CDLL(os.path.join(ROOT, "oracle", "_ref", "libref_px.so"))
    lib.ref_px_forward_time.restype = C.c_int
    lib.ref_px_forward_time.argtypes = [C.c_char_p, np.ctypeslib.ndpointer(np.uint16, flags="C_CONTIGUOUS"), C.c_int,
                                        C.c_int, C.c_int, C.POINTER(C.c_float)]
    nt = a.nt or 30877
    path = P.write_synthetic(os.path.join(tempfile.mkdtemp(), "px.bin"), seed=0, nt=nt)
    for nb in a.batch:
        x = np.ascontiguousarray(P.synthetic_inputs(nb, seed=1))
        ms = C.c_float(0)
        if lib.ref_px_forward_time(path.encode(), x, nb, a.warmup, a.iters, C.byref(ms)):
            raise SystemExit("reference PixAI forward failed")
        print(json.dumps({"impl": "reference PixAI kernels (px_kernels.cu, mma.sync E4M3) on this GPU", "batch": nb,
                          "ms_per_forward": ms.value, "images_per_s": nb / (ms.value * 1e-3),
                          "model": f"pixai.bin v3, 32 blocks, {nt} tags, random-init"}), flush=True)


if __name__ == "__main__":
    main()
