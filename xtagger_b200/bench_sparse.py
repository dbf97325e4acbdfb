"""Per-projection timing of the 2:4-sparse kernels (xtb_*_sp, tcgen05.mma.sp) against the dense ones (xtb_*) on the
same pruned weights, through the C ABI: device time per launch from CUDA-graph replays of `reps` back-to-back
launches (median of `iters` replays). Inputs: `batch` images of activations (rows = batch x 1025), seeded random
E4M3 weights N(0, 0.02) with 128 x 128 block scales, 2:4-pruned by magnitude. One JSON line per (projection, kind)
with the dense-equivalent TFLOP/s. Also the target of the ncu captures of the sparse kernels (--only, --reps 1).

    python -m xtagger_b200.bench_sparse [--batch 64] [--iters 10] [--reps 5] [--only fc1_sp,fc1]
"""
import argparse
import ctypes as C
import json
import os
import sys

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
D, HIDP, N12, T, TP, NH = 1024, 2736, 5472, 1025, 1152, 16


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--batch", type=int, default=64)
    ap.add_argument("--iters", type=int, default=10)
    ap.add_argument("--reps", type=int, default=5)
    ap.add_argument("--only", default="")
    a = ap.parse_args()
    sys.path.insert(0, ROOT)
    import torch
    from xtagger_b200 import lib as L
    from xtagger_b200 import model as M
    xl = L.lib()
    rows = a.batch * T
    rng = np.random.default_rng(3)
    P = lambda t: C.c_void_p(t.data_ptr())  # noqa: E731

    def weight(n, k):
        q, s = M.quant_blocks(rng.standard_normal((n, k), dtype=np.float32) * 0.02)
        q = M.prune24_codes(q)
        npad, kp = -(-n // 128) * 128, -(-k // 128) * 128
        vals = np.empty(npad * kp // 2, np.uint8)
        meta = np.empty(npad * kp // 8, np.uint8)
        assert xl.xtb_sparse24_compress(C.c_void_p(q.ctypes.data), n, k, C.c_void_p(vals.ctypes.data),
                                        C.c_void_p(meta.ctypes.data)) == 0
        cuda = lambda x: torch.from_numpy(x).cuda()  # noqa: E731
        return cuda(q), cuda(s), cuda(vals), cuda(meta)

    def act(n, k):
        return torch.randint(0, 0x7F, (n, k), dtype=torch.uint8, device="cuda") & 0x6F  # finite E4M3 codes

    h = act(rows, D)
    h8 = act(rows, HIDP)
    x = torch.zeros((rows, D), dtype=torch.float16, device="cuda")
    q8, k8, v8 = (torch.zeros((a.batch, NH, TP, 64), dtype=torch.uint8, device="cuda") for _ in range(3))
    hout = torch.zeros((rows, HIDP), dtype=torch.uint8, device="cuda")
    stat = torch.zeros((43, rows, 2), dtype=torch.float32, device="cuda")
    cs = torch.from_numpy(np.ascontiguousarray(M.rope_table(), np.float32)).cuda()
    rs = torch.full((HIDP,), 30.0, dtype=torch.float32, device="cuda")
    cvec = torch.zeros(D, dtype=torch.float32, device="cuda")
    wq, wo, w12, w2 = weight(3 * D, D), weight(D, D), weight(N12, D), weight(D, HIDP)
    s0 = None

    def stream():
        return C.c_void_p(torch.cuda.current_stream().cuda_stream)

    cases = {
        "qkv": (2.0 * rows * 3 * D * D, lambda: xl.xtb_qkv(P(h), rows, P(wq[0]), P(wq[1]), 0.02, P(q8), P(k8), P(v8), P(cs),
                                                           1.0, 1.0, 1.0, stream())),
        "qkv_sp": (2.0 * rows * 3 * D * D, lambda: xl.xtb_qkv_sp(P(h), rows, P(wq[2]), P(wq[3]), P(wq[1]), 0.02, P(q8), P(k8),
                                                                 P(v8), P(cs), 1.0, 1.0, 1.0, stream())),
        "oproj": (2.0 * rows * D * D, lambda: xl.xtb_oproj(P(h), rows, P(wo[0]), P(wo[1]), 1e-4, P(x), stream())),
        "oproj_sp": (2.0 * rows * D * D, lambda: xl.xtb_oproj_sp(P(h), rows, P(wo[2]), P(wo[3]), P(wo[1]), 1e-4, P(x),
                                                                 stream())),
        "fc1": (2.0 * rows * N12 * D, lambda: xl.xtb_fc1(P(h), rows, P(w12[0]), P(w12[1]), 0.02, P(hout), P(stat), P(rs),
                                                         stream())),
        "fc1_sp": (2.0 * rows * N12 * D, lambda: xl.xtb_fc1_sp(P(h), rows, P(w12[2]), P(w12[3]), P(w12[1]), 0.02, P(hout),
                                                               P(stat), P(rs), stream())),
        "fc2": (2.0 * rows * D * HIDP, lambda: xl.xtb_fc2(P(h8), rows, P(w2[0]), P(w2[1]), 1e-4, P(x), P(stat), P(cvec),
                                                          P(cvec), stream())),
        "fc2_sp": (2.0 * rows * D * HIDP, lambda: xl.xtb_fc2_sp(P(h8), rows, P(w2[2]), P(w2[3]), P(w2[1]), 1e-4, P(x),
                                                                P(stat), P(cvec), P(cvec), stream())),
    }
    only = [s for s in a.only.split(",") if s]
    for name, (flop, fn) in cases.items():
        if only and name not in only:
            continue
        for _ in range(2):
            assert fn() == 0
        torch.cuda.synchronize()
        g = torch.cuda.CUDAGraph()
        st = torch.cuda.Stream()
        with torch.cuda.stream(st):
            with torch.cuda.graph(g, stream=st):
                for _ in range(a.reps):
                    fn()
        ts = []
        for _ in range(a.iters):
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            g.replay()
            e1.record()
            torch.cuda.synchronize()
            ts.append(e0.elapsed_time(e1) * 1e-3 / a.reps)
        t = float(np.median(ts))
        assert xl.xtb_error_word(0) == 0
        print(json.dumps({"kernel": name, "batch": a.batch, "rows": rows, "us": t * 1e6,
                          "dense_equiv_tflops": flop / t / 1e12}), flush=True)
        del g
    del s0


if __name__ == "__main__":
    main()
