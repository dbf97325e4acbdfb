"""Throughput of the PixAI tagger forward (ViTDet-L at 1008^2: 5184 window-major tokens, 32 blocks of which 4 attend
globally, GELU MLP 4736, attention-pool head, 30877 tags) on one B200 through the px_* engine, random-init
pixai.bin v3 weights (E4M3, one scale per tensor), seeded synthetic 1008^2 images. One JSON line:
  value        images/s with the inputs resident (CUDA events around K graph launches on the engine's stream);
  e2e          images/s through px_submit / px_wait with the inputs in a pinned host pool (H2D of 6.1 MB per
               image and D2H of the scores every step), wall clock;
  roofline     fc1 (the largest GEMM): dense FP8 FLOPs per launch over its time in one direct forward with events
               after every kernel, against 2x the measured bf16 sustained peak;
  profile_ms   per-kind kernel times of that forward;

    python -m xtagger_b200.bench_pixai [--batch 8] [--steps 10] [--warmup 3]
"""
import argparse
import json
import os
import tempfile
import time

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
T, D, HID, NL = 5184, 1024, 4736, 32
LIN_FLOP = 2.0 * T * NL * (3 * D * D + D * D + 2 * HID * D)                      # 4.610 TFLOP
ATT_FLOP = 28 * 9 * 16 * 4.0 * 576 * 576 * 64 + 4 * 16 * 4.0 * T * T * 64         # 0.783 TFLOP
FLOP_PER_IMAGE = LIN_FLOP + ATT_FLOP + 2.0 * T * D * 588
FC1_FLOP_PER_ROW = 2.0 * HID * D


def peak():
    try:
        j = json.load(open(os.path.join(ROOT, "MEASURED_PEAKS.json")))
        return 2 * float(j["bf16_tflops_sustained"]), "2x measured bf16 sustained (MEASURED_PEAKS.json)"
    except (OSError, KeyError, ValueError):
        return 2 * 1.4e3, "2x fallback bf16 sustained 1.4 PF/s"


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--batch", type=int, default=8)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--nt", type=int, default=30877)
    a = ap.parse_args()
    import sys
    sys.path.insert(0, ROOT)
    import torch
    from xtagger_b200 import pixai as P
    from xtagger_b200.pxengine import PxEngine

    d = os.environ.get("XTB_BENCH_DIR", os.path.join(tempfile.gettempdir(), "xtb_bench"))
    model = P.cached_synthetic(d, seed=0, nt=a.nt)
    pool = P.synthetic_inputs(a.batch, seed=1)
    eng = PxEngine(model, nb=a.batch, pool=pool)
    eng.ready()
    st = torch.cuda.ExternalStream(eng.stream())
    eng.upload(pool)
    for _ in range(a.warmup):
        eng.forward_resident()
    torch.cuda.synchronize()
    from xtagger_b200.clocks import Clocks
    clk = Clocks(torch.cuda.current_device())
    clk.start()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(st)
    for _ in range(a.steps):
        eng.forward_resident()
    e1.record(st)
    torch.cuda.synchronize()
    clocks = clk.stop()
    t = e0.elapsed_time(e1) / 1e3
    value = a.batch * a.steps / t
    inputs = [pool[i] for i in range(a.batch)]
    eng.run(inputs)
    t0 = time.perf_counter()
    for k in range(a.steps):
        eng.submit(k % 2, inputs)
        if k >= 1:
            eng.wait((k - 1) % 2, a.batch)
    eng.wait((a.steps - 1) % 2, a.batch)
    e2e = a.batch * a.steps / (time.perf_counter() - t0)
    prof = eng.profile()
    launches = eng.launches_per_forward()
    eng.close()
    fc1_ms = prof["fc1"] / NL
    achieved = FC1_FLOP_PER_ROW * a.batch * T / (fc1_ms * 1e-3) / 1e12
    pk, src = peak()
    line = {"metric": "images/sec PixAI (ViTDet-L 1008^2, 32 blocks, 30877 tags), 1 B200", "value": value,
            "unit": "images/s", "batch": a.batch, "steps": a.steps, "warmup": a.warmup,
            "ms_per_step": 1e3 * t / a.steps, "dtype": "e4m3", "data": "synthetic",
            "weights": "random-init pixai.bin v3 (E4M3, one scale per tensor)",
            "e2e": {"value": e2e, "unit": "images/s", "h2d_bytes_per_step": a.batch * P.PX_IN * 2,
                    "d2h_bytes_per_step": a.batch * a.nt * 4},
            "forward_tflops": FLOP_PER_IMAGE * value / 1e12, "flop_per_image": FLOP_PER_IMAGE,
            "roofline": {"bound": "tensor", "kernel": "fc1 (tcgen05 E4M3 GEMM + bias / GELU epilogue)",
                         "achieved": achieved, "peak": pk, "unit": "TFLOP/s", "frac": achieved / pk,
                         "peak_source": src, "launch_ms": fc1_ms},
            "profile_ms": prof, "gpu_launches_per_forward": launches, "clocks": clocks}
    print(json.dumps(line), flush=True)


if __name__ == "__main__":
    main()
