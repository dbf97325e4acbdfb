"""Config 1 of the benchmark plan: the EVA02-L MLP up-projection alone, A [M][1024] x W [2730][1024]^T, E4M3 with
fp32 scales per 128 x 128 weight block, fp32 output, through the C-ABI entry point xtb_gemm_e4m3_f32.

A ~ N(0, 1) quantised with one scale from max |A|; W ~ N(0, 0.02) quantised per block; seed 0. Device time from
CUDA-graph replays (the entry point encodes its TMA descriptors on the host at every call, which a graph captures
once): "hot" = a graph of `reps` back-to-back launches, "cold" = a graph of `reps` x (write a 256 MB buffer, launch)
minus a graph of the writes alone (L2 flushed before each launch); median over `iters` replays. One JSON line per M (1025 = one image, 8200 = eight) with the roofline of both
bounds against the measured peaks (MEASURED_PEAKS.json: copy bandwidth; dense FP8 as 2x the bf16 GEMM rate), and
the largest deviation from a float64 dequantise-then-matmul of the same operands in PyTorch at M = 1025.

    python -m xtagger_b200.bench_gemm [--iters 20] [--reps 50]
"""
import argparse
import ctypes as C
import json
import os

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _peaks():
    try:
        j = json.load(open(os.path.join(ROOT, "MEASURED_PEAKS.json")))
        return float(j["hbm_gbs"]), 2 * float(j["bf16_tflops"]), "MEASURED_PEAKS.json (burst)"
    except (OSError, KeyError, ValueError):
        return 6650.0, 2 * 1590.0, "fallback"


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--iters", type=int, default=20)
    ap.add_argument("--reps", type=int, default=50)
    a = ap.parse_args()
    import sys
    sys.path.insert(0, ROOT)
    import torch
    from xtagger_b200 import lib as L
    from xtagger_b200 import model as M
    xl = L.lib()
    K, N = 1024, 2730
    rng = np.random.default_rng(0)
    w8, ws = M.quant_blocks(rng.standard_normal((N, K), dtype=np.float32) * 0.02)
    hbm, fp8, src = _peaks()
    dw, dws = torch.from_numpy(w8).cuda(), torch.from_numpy(ws).cuda()
    flush = torch.empty(256 << 20, dtype=torch.uint8, device="cuda")
    for m in (1025, 8200):
        af = rng.standard_normal((m, K), dtype=np.float32)
        ascale = float(np.abs(af).max()) / 448
        a8 = M._e4m3(af / ascale)
        da = torch.from_numpy(a8).cuda()
        out = torch.empty((m, N), dtype=torch.float32, device="cuda")
        args = (C.c_void_p(da.data_ptr()), m, K, C.c_void_p(dw.data_ptr()), N, C.c_void_p(dws.data_ptr()),
                C.c_float(ascale), C.c_void_p(out.data_ptr()), None)
        for _ in range(5):
            assert xl.xtb_gemm_e4m3_f32(*args) == 0
        torch.cuda.synchronize()

        def graph(fn):
            g = torch.cuda.CUDAGraph()
            st = torch.cuda.Stream()
            with torch.cuda.stream(st):
                with torch.cuda.graph(g, stream=st):
                    for _ in range(a.reps):
                        fn()
            return g

        def gemm():
            xl.xtb_gemm_e4m3_f32(*args[:-1], C.c_void_p(torch.cuda.current_stream().cuda_stream))

        g_hot = graph(gemm)
        g_cold = graph(lambda: (flush.zero_(), gemm()))
        g_flush = graph(lambda: flush.zero_())

        def replay(g):
            ts = []
            for _ in range(a.iters):
                e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                e0.record()
                g.replay()
                e1.record()
                torch.cuda.synchronize()
                ts.append(e0.elapsed_time(e1) * 1e-3)
            return float(np.median(ts))
        res = {"hot": replay(g_hot) / a.reps, "cold": (replay(g_cold) - replay(g_flush)) / a.reps}
        assert xl.xtb_error_word(0) == 0
        flop = 2.0 * m * K * N
        byts = m * K + N * K + ws.size * 4 + m * N * 4
        if m == 1025:
            want = (torch.from_numpy(M.e4m3_decode(a8).astype(np.float64) * ascale).cuda() @
                    torch.from_numpy(M.dequant_blocks(w8, ws).astype(np.float64)).cuda().T)
            err = float((out.double() - want).abs().max() / want.abs().max())
        line = {"config": 1, "workload": f"{m} x {K} x {N} E4M3 block-scaled GEMM, fp32 out", "M": m,
                "flop": flop, "algorithmic_bytes": byts, "peaks": {"hbm_gbs": hbm, "fp8_tflops": fp8, "source": src}}
        for mode, t in res.items():
            line[mode] = {"us": t * 1e6, "tflops": flop / t / 1e12, "gbs": byts / t / 1e9,
                          "frac_tensor": flop / t / 1e12 / fp8, "frac_hbm": byts / t / 1e9 / hbm}
        if m == 1025:
            line["max_abs_err_over_max_abs_ref"] = err
        print(json.dumps(line), flush=True)


if __name__ == "__main__":
    main()
