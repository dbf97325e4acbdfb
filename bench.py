"""Benchmark of the EVA02-L tagger forward: global batch 64 of synthetic 448^2 images,
split across N GPUs (one process per GPU, launched by torch.distributed.run for N > 1), random-init block-scaled
E4M3 weights (24 layers, 10861 tags, FP8 head).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference] [--batch 64] [--nt 10861] [--sparse]

--v3 runs the same forward on weights in the reference's own eva02.bin v3 format (one E4M3 scale per tensor, fp16
head): the GEMMs then accumulate the whole K range in TMEM and scale once, as the reference's kernels do. This is
the format oracle/ref_time.py times the reference's kernels on.
Block scales are powers of two by default (max / 448 rounded up, the convention of the tensor core's own block
scaling): QKV and fc1 then run on tcgen05.mma kind::mxf8f6f4.block_scale with the whole K range in one accumulator;
--free-scales writes max / 448 scales instead, and every projection promotes its 128-deep K blocks in the epilogue.
--sparse is config 5: the four projections of every layer 2:4-pruned by magnitude (prune24.py's rule), which the
engine runs on the sparse tensor cores (tcgen05.mma.sp); global batch 128 unless --batch is given.
--nt 13461 --batch 32 is config 4 (implies --mix): the inputs are views of seeded 896^2 sources (per source the
whole image and its four quadrants, 6 x 5 + 2 whole images), made by the GPU preprocessing, and the line gains
e2e_decoded: images/s from decoded RGBX sources in pinned host memory through H2D, the preprocessing kernels, the
forward and the scores' D2H, all on the engine's stream.

Prints one JSON line (rank 0):
  value       whole-job images/s with inputs resident on the devices (CUDA events around K graph launches on the
              engine's stream, max over ranks);
  e2e         the same metric through the engine's public calls (eva_submit / eva_wait) with host buffers: every
              step copies its inputs from a pinned host pool and its scores back (wall clock, max over ranks);
  roofline    the dominant kernel by time, attention (36 % of the step): algorithmic FLOPs per launch over its
              average launch time from one direct (non-graph) forward timed with events on the launching stream,
              against the FP8 dense peak taken as 2x the measured bf16 peak, with its exp2 count and the floor those
              exponentials set on the MUFU unit; roofline_fc1 the same for fc1 (38 % of the FLOPs);
  free_scales   the resident forward on max / 448 block scales (the promoting kernels), single GPU;
  gemm_config1  BASELINE config 1 (1025 x 2730 x 1024 block-scaled E4M3 GEMM) cold, single GPU;
  cpu_baseline  the CPU oracle (plain C, OpenMP) on a bounded sample, rank 0 at N = 1.
--impl reference times the CPU restatement of the reference's forward (the reference has no CPU path of its
own and its host engine is Windows-only) on the same config and prints the same line with "impl": "reference".
"""
import argparse
import ctypes
import json
import os
import sys
import tempfile
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "images/sec EVA02-L 448² (1/2/4/8 B200) + FP8 GEMM % of tensor peak"
NT = 10861
MODEL_KW = dict(seed=0, nt=NT, nl=24, version=4, head_fp8=True, pow2=True)
FC1_FLOP_PER_ROW = 2.0 * 5472 * 1024
# DRAM bytes (dram__bytes_read.sum + dram__bytes_write.sum) of one fc1 launch (k_gemm2_mx<EpiFC1, 2>, the CTA pair on
# 256 x 256 block-scaled tiles) in an ncu capture at batch 32 (32 x 1025 rows): 39.48 MB + 48.74 MB; the launch at
# another batch is scaled by the rows it processes. The single-CTA block-scaled and the promoting fc1 kernels moved
# 87.2 MB in the same capture, within 1 % of this, so the figure stands for the dense fc1 under every scale format.
FC1_TRAFFIC_PER_ROW = (39.4752e6 + 48.742912e6) / (32 * 1025)
FLOP_PER_IMAGE = 723.5e9
# attention per layer and image: QK^T and PV over 16 heads of 64 (2 x 2 x 1025^2 x 64 x 16 FLOPs), one exp2 per score
# (16 x 1025^2), algorithmic bytes = q8 / k8 / v8 read once (3 x 16 x 1025 x 64) + the E4M3 output (1025 x 1024);
# DRAM bytes per image from the ncu capture of k_attention at batch 32 (109.09 MB read + 15.34 MB written).
ATT_FLOP_PER_IMAGE = 4.0 * 1025 * 1025 * 64 * 16
ATT_EXP_PER_IMAGE = 16.0 * 1025 * 1025
ATT_BYTES_PER_IMAGE = 3.0 * 16 * 1025 * 64 + 1025 * 1024
ATT_TRAFFIC_PER_IMAGE = (109.09e6 + 15.34e6) / 32


from xtagger_b200.clocks import Clocks  # noqa: E402


def dist_env():
    return int(os.environ.get("RANK", 0)), int(os.environ.get("WORLD_SIZE", 1)), int(os.environ.get("LOCAL_RANK", 0))


def model_path(rank, world, barrier):
    from xtagger_b200 import model as M
    d = os.environ.get("XTB_BENCH_DIR", os.path.join(tempfile.gettempdir(), "xtb_bench"))
    if rank == 0:
        p = M.cached_synthetic(d, **MODEL_KW)
    barrier()
    if rank != 0:
        p = M.cached_synthetic(d, **MODEL_KW)
    return p


def peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        j = json.load(open(p))
        return float(j["bf16_tflops_sustained"]), "2x measured bf16 sustained (MEASURED_PEAKS.json)"
    except (OSError, KeyError, ValueError):
        return 1.4e3, "2x fallback bf16 sustained 1.4 PF/s"


def cpu_sample(model, nimg=1):
    from oracle import oracle as O
    from xtagger_b200 import model as M
    x = M.synthetic_inputs(nimg, seed=1)
    cores = O.use_all_cores()   # not OMP_NUM_THREADS, which torch.distributed.run sets to 1
    t0 = time.perf_counter()
    O.forward(model, x)   # the reference's attention tiling (64-key tiles, 16-row slices)
    dt = time.perf_counter() - t0
    return nimg / dt, cores, dt


def num_sms():
    import torch
    return torch.cuda.get_device_properties(torch.cuda.current_device()).multi_processor_count


def time_free_scales(args, pool, nb, local, steps=5, warmup=3):
    """The same device-resident forward on weights whose 128 x 128 block scales are max / 448 (the quantiser's natural
    output) instead of powers of two: every projection then promotes its 128-deep K blocks in the epilogue."""
    import torch
    from xtagger_b200 import model as M
    from xtagger_b200.engine import Engine
    d = os.environ.get("XTB_BENCH_DIR", os.path.join(tempfile.gettempdir(), "xtb_bench"))
    kw = dict(MODEL_KW, pow2=False)
    eng = Engine(M.cached_synthetic(d, **kw), devices=(local,), nb=nb)
    try:
        eng.ready()
        eng.upload(pool)
        st = torch.cuda.ExternalStream(eng.stream(0), device=torch.device("cuda", local))
        for _ in range(warmup):
            eng.forward_resident()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(st)
        for _ in range(steps):
            eng.forward_resident()
        e1.record(st)
        torch.cuda.synchronize()
        t = e0.elapsed_time(e1) / 1e3
        return {"value": nb * steps / t, "unit": "images/s", "steps": steps, "block_scale_kinds":
                eng.block_scale_kinds(), "weights": "random-init, E4M3 with fp32 scales per 128x128 block (max / 448)"}
    finally:
        eng.close()


def time_gemm_config1(local, reps=50):
    """BASELINE config 1 on the device through xtb_gemm_e4m3_f32: A [1025][1024] ~ N(0, 1) in E4M3 with one scale
    max|A| / 448, W [2730][1024] ~ N(0, 0.02) in E4M3 with fp32 scales per 128 x 128 block (max / 448), fp32 out, seed
    0. Cold: L2 flushed (a 256 MB write) before every launch; each launch timed alone with CUDA events. Error against
    a float64 dequantise-then-matmul in PyTorch."""
    import numpy as np
    import torch
    from xtagger_b200 import lib as XL
    from xtagger_b200 import model as M
    dev = torch.device("cuda", local)
    rng = np.random.default_rng(0)
    a = rng.standard_normal((1025, 1024), dtype=np.float32)
    ascale = float(np.abs(a).max()) / 448.0
    a8 = M._e4m3(a / ascale)
    w8, ws = M.quant_blocks(rng.standard_normal((2730, 1024), dtype=np.float32) * 0.02)
    da, dw, dws = (torch.from_numpy(np.ascontiguousarray(v)).to(dev) for v in (a8, w8, ws))
    out = torch.empty((1025, 2730), dtype=torch.float32, device=dev)
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
    xl = XL.lib()
    st = torch.cuda.current_stream(dev)
    P = lambda t: ctypes.c_void_p(t.data_ptr())  # noqa: E731

    def launch():
        XL.check(xl.xtb_gemm_e4m3_f32(P(da), 1025, 1024, P(dw), 2730, P(dws), ascale, P(out),
                                      ctypes.c_void_p(st.cuda_stream)), "xtb_gemm_e4m3_f32")
    for _ in range(5):
        launch()
    times = []
    for _ in range(reps):
        flush.fill_(1)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(st)
        launch()
        e1.record(st)
        torch.cuda.synchronize()
        times.append(e0.elapsed_time(e1) * 1e3)
    us = float(np.median(times))
    ref = (torch.from_numpy(M.e4m3_decode(a8).astype(np.float64) * ascale).to(dev) @
           torch.from_numpy(M.dequant_blocks(w8, ws).astype(np.float64)).to(dev).T)
    err = float((out.double() - ref).abs().max() / ref.abs().max())
    flop, nbytes = 2.0 * 1025 * 1024 * 2730, 1025 * 1024 + 2730 * 1024 + ws.size * 4 + 1025 * 2730 * 4
    hbm = None
    try:
        hbm = float(json.load(open(os.path.join(ROOT, "MEASURED_PEAKS.json")))["hbm_gbs"])
    except (OSError, KeyError, ValueError):
        pass
    return {"cold_us_median": us, "cold_us_min": float(min(times)), "tflops": flop / (us * 1e-6) / 1e12,
            "gb_per_s": nbytes / (us * 1e-6) / 1e9, "hbm_frac": (nbytes / (us * 1e-6) / 1e9 / hbm) if hbm else None,
            "algorithmic_bytes": nbytes, "max_abs_err_over_max_abs_ref": err,
            "what": "1025x2730x1024 E4M3 block-scaled GEMM, fp32 out, L2 flushed before each of the timed launches, "
                    "median of " + str(reps)}


def run_reference(args, rank, world):
    """CPU restatement of the reference's forward (its attention tiling), bounded sample per step."""
    if rank != 0:
        return
    model = model_path(0, 1, lambda: None)
    for _ in range(args.warmup):
        cpu_sample(model)
    vals, cores = [], 1
    t0 = time.perf_counter()
    for _ in range(args.steps):
        v, cores, _ = cpu_sample(model)
        vals.append(v)
    el = time.perf_counter() - t0
    v = args.steps / el
    line = {"metric": METRIC, "value": v, "unit": "images/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": 1e3 * el / args.steps, "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "e4m3", "data": "synthetic", "impl": "reference",
            "config": {"workload": f"{config_name(args)} (EVA02-L 448^2 forward, 24 layers, {args.nt} tags); each step a bounded "
                                   "sample of 1 image on the host cores", "global_batch": args.batch},
            "cpu_baseline": {"value": v, "unit": "images/s", "cores": cores, "kind": "port",
                             "sample": "1 image per step, full 24-layer forward, CPU restatement (oracle/) of the "
                                       "reference's GPU forward; the reference ships no CPU path"},
            "e2e": {"value": v, "unit": "images/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    if not args.no_extra:
        # The reference's own GPU kernels (compiled from its sources into oracle/_ref) on GPU 0 of this box, at the
        # same batch: its eva_forward replayed as a CUDA graph with the inputs resident, on its v3 weight format.
        try:
            from oracle import ref_time as RT
            line["reference_gpu_kernels"] = RT.reference_kernels([args.batch], warmup=3, iters=10, nt=args.nt)[0]
        except Exception as e:  # no GPU, or the reference library not built here
            line["reference_gpu_kernels"] = {"unavailable": f"{type(e).__name__}: {e}"[:300]}
    print(json.dumps(line), flush=True)


def run_ours(args, rank, world, local):
    import numpy as np
    import torch
    from xtagger_b200 import model as M
    from xtagger_b200.engine import Engine
    from xtagger_b200.lib import EVA_IN

    torch.cuda.set_device(local)
    pg = None
    if world > 1:
        import datetime
        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=600), device_id=torch.device("cuda", local))
        pg = dist

    def barrier():
        if pg:
            pg.barrier()

    from xtagger_b200.dist import allmax, shard_bounds
    model = model_path(rank, world, barrier)
    lo, hi = shard_bounds(args.batch, world, rank)
    nb = hi - lo
    dev = torch.device("cuda", local)
    if args.mix:
        # config 4: the whole images and quadrant crops of 896^2 sources, resampled on the device by the GPU
        # preprocessing (the same kernels the decoded-image e2e below times)
        from xtagger_b200 import views as V
        views_all = V.mix_views(args.batch)
        views = views_all[lo:hi]
        nsrc = V.num_sources(views_all)
        used = sorted({v[0] for v in views})
        src_host = torch.from_numpy(V.mix_sources(nsrc, seed=1)).pin_memory()
        src_dev = src_host.to(dev)
        src_ptrs = [src_dev[i].data_ptr() for i in range(nsrc)]
        prep = V.DevicePrep(V.SIDE, V.SIDE, nsrc, device=dev)
        ops = torch.empty((max(nb, 1), EVA_IN), dtype=torch.int16, device=dev)
        prep.run(src_ptrs, views, ops.data_ptr(), torch.cuda.current_stream(dev).cuda_stream)
        torch.cuda.synchronize()
        pool = np.ascontiguousarray(ops[:nb].cpu().numpy().view(np.uint16).reshape(nb, 1024, 592))
    else:
        allx = M.synthetic_inputs(args.batch, seed=1)
        pool = np.ascontiguousarray(allx[lo:hi])
    eng = Engine(model, devices=(local,), nb=nb, pool=pool)
    eng.ready()
    st = torch.cuda.ExternalStream(eng.stream(0), device=torch.device("cuda", local))
    launches = eng.launches_per_forward()

    # ---- device-resident throughput ----
    eng.upload(pool)
    for _ in range(args.warmup):
        eng.forward_resident()
    torch.cuda.synchronize()
    barrier()
    torch.cuda.synchronize()
    clk = Clocks(local)
    clk.start()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(st)
    for _ in range(args.steps):
        eng.forward_resident()
    e1.record(st)
    torch.cuda.synchronize()
    clocks = clk.stop()
    barrier()
    t = allmax(e0.elapsed_time(e1) / 1e3)
    value = args.batch * args.steps / t

    # ---- end to end through eva_submit / eva_wait (pinned host inputs in, scores out, every step) ----
    # wall clock from an idle device to the last eva_wait: the copies run on the engine's copy stream, so device
    # events on the compute stream would not bracket them
    inputs = [pool[i] for i in range(nb)]
    for s in range(min(args.warmup, 2)):
        eng.submit(s, inputs)
    for s in range(min(args.warmup, 2)):
        eng.wait(s, nb)
    torch.cuda.synchronize()
    barrier()
    t0 = time.perf_counter()
    for k in range(args.steps):       # two slots in flight: copies of one batch overlap the other's forward
        eng.submit(k % 2, inputs)
        if k >= 1:
            eng.wait((k - 1) % 2, nb)
    eng.wait((args.steps - 1) % 2, nb)
    torch.cuda.synchronize()
    te = allmax(time.perf_counter() - t0)
    barrier()
    e2e = args.batch * args.steps / te

    # ---- config 4, end to end from decoded images: every step copies the 896^2 RGBX sources from pinned host memory,
    # preprocesses them on the device into the engine's resident inputs (xtb_prep_ingest / xtb_prep_crop), runs the
    # forward and copies the scores back to pinned host memory; all on the engine's stream, timed by CUDA events ----
    decoded = None
    if args.mix:
        from xtagger_b200 import lib as XL
        xl = XL.lib()
        din, dout, est = eng.device_input(0), eng.device_output(0), eng.stream(0)
        scores = torch.empty((max(nb, 1), eng.nt), dtype=torch.float32).pin_memory()
        nk = [0]

        def dstep():
            for i in used:
                XL.check(xl.xtb_copy_async(ctypes.c_void_p(src_ptrs[i]), ctypes.c_void_p(src_host[i].data_ptr()),
                                           src_host[i].numel(), ctypes.c_void_p(est)), "xtb_copy_async")
            nk[0] = prep.run(src_ptrs, views, din, est)
            eng.forward_resident()
            XL.check(xl.xtb_copy_async(ctypes.c_void_p(scores.data_ptr()), ctypes.c_void_p(dout), nb * eng.nt * 4,
                                       ctypes.c_void_p(est)), "xtb_copy_async")

        for _ in range(args.warmup):
            dstep()
        torch.cuda.synchronize()
        barrier()
        torch.cuda.synchronize()
        e0.record(st)
        for _ in range(args.steps):
            dstep()
        e1.record(st)
        torch.cuda.synchronize()
        td = allmax(e0.elapsed_time(e1) / 1e3)
        barrier()
        # the scores of the last step equal the resident forward's on the same inputs (prep is deterministic)
        assert np.isfinite(scores[:nb].numpy()).all()
        decoded = {"value": args.batch * args.steps / td, "unit": "images/s",
                   "h2d_bytes_per_step": sum(src_host[i].numel() for i in used) * world,
                   "d2h_bytes_per_step": args.batch * eng.nt * 4,
                   "prep_kernels_per_step": nk[0] * world,
                   "what": "decoded 896^2 RGBX sources (pinned host) -> H2D -> GPU preprocessing (whole image: "
                           "antialiased bicubic 896 -> 448; quadrants: normalise) -> forward -> scores D2H, CUDA "
                           "events on the engine stream, max over ranks"}

    # ---- rooflines from one direct (non-graph) forward with per-kernel events on the engine's stream: attention, the
    # dominant kernel by time, and fc1, the dominant one by FLOPs ----
    prof = eng.profile()
    sparse_kinds = eng.sparse_kinds()
    block_scale_kinds = eng.block_scale_kinds()
    fc1_sparse = bool(sparse_kinds & 4)
    rows = nb * 1025
    bf16, peak_src = peaks()
    fc1_ms = prof["fc1"] / 24
    achieved = FC1_FLOP_PER_ROW * rows / (fc1_ms * 1e-3) / 1e12   # dense-equivalent FLOPs
    fc1_peak = (4 if fc1_sparse else 2) * bf16
    fc1_src = peak_src
    if fc1_sparse:
        fc1_src = peak_src.replace("2x", "4x") + "; 2:4-sparse FP8 runs at twice the dense FP8 rate"
    att_ms = prof["attention"] / 24
    att_flop = ATT_FLOP_PER_IMAGE * nb
    att_exp = ATT_EXP_PER_IMAGE * nb
    sm_mhz = clocks.get("sm_mhz") or 1965.0
    exp_floor_ms = att_exp / (16 * num_sms() * sm_mhz * 1e6) * 1e3   # every exponential on the MUFU unit
    roof_att = {"bound": "tensor", "kernel": "attention (k_attention + k_attention_last: tcgen05 QK^T / PV, "
                "exp2 softmax, E4M3 P)", "achieved": att_flop / (att_ms * 1e-3) / 1e12, "peak": 2 * bf16,
                "unit": "TFLOP/s", "frac": att_flop / (att_ms * 1e-3) / 1e12 / (2 * bf16), "peak_source": peak_src,
                "flop_per_launch": att_flop, "launch_ms": att_ms,
                "traffic": ATT_TRAFFIC_PER_IMAGE * nb,
                "traffic_unit": "bytes per launch (ncu DRAM read + write at batch 32, scaled by images)",
                "algorithmic_bytes": ATT_BYTES_PER_IMAGE * nb,
                "exp2_per_launch": att_exp, "exp2_floor_ms": exp_floor_ms,
                "frac_of_exp2_floor": exp_floor_ms / att_ms,
                "exp2_floor_source": f"16 exp2 per clock per SM x {num_sms()} SMs at the median SM clock {sm_mhz:.0f} MHz"}
    roof_fc1 = {"bound": "tensor",
                "kernel": "fc1 (tcgen05.mma.sp 2:4-sparse E4M3 GEMM + SwiGLU epilogue)" if fc1_sparse
                else "fc1 (tcgen05 E4M3 GEMM + SwiGLU epilogue)",
                "achieved": achieved, "peak": fc1_peak, "unit": "TFLOP/s", "frac": achieved / fc1_peak,
                "peak_source": fc1_src, "flop_per_launch": FC1_FLOP_PER_ROW * rows, "launch_ms": fc1_ms,
                "traffic": None if fc1_sparse else FC1_TRAFFIC_PER_ROW * rows,
                "traffic_unit": "bytes per launch (ncu DRAM read + write at batch 32, scaled by rows)"}
    free_scales = None
    if rank == 0 and world == 1 and not args.no_extra and not (args.v3 or args.free_scales or args.sparse or args.mix):
        free_scales = time_free_scales(args, pool, nb, local)
    gemm1 = None
    if rank == 0 and world == 1 and not args.no_extra:
        gemm1 = time_gemm_config1(local)
    out = None
    if rank == 0 and world == 1 and not args.no_cpu:
        v, cores, dt = cpu_sample(model, nimg=4)
        out = {"value": v, "unit": "images/s", "cores": cores, "kind": "port",
               "sample": f"4 images, full 24-layer forward ({dt:.1f} s), CPU oracle (plain C + OpenMP)"}
    eng.close()
    if rank == 0:
        line = {"metric": METRIC, "value": value, "unit": "images/s", "n_gpus": world, "steps": args.steps,
                "warmup": args.warmup, "ms_per_step": 1e3 * t / args.steps, "higher_is_better": True,
                "scaling": "strong", "vs_baseline": None, "dtype": "e4m3", "data": "synthetic",
                "config": {"workload": f"{config_name(args)}: EVA02-L 448^2 forward (24 layers, d 1024, 1025 tokens, {args.nt}-tag "
                                       f"{'fp16' if args.v3 else 'FP8'} head), global batch split across the GPUs" +
                                       (f"; inputs: {len(views_all)} views of {nsrc} seeded 896^2 sources (whole "
                                        "image + 4 quadrant crops per source, the rest whole images), "
                                        "preprocessed on the device" if args.mix else ""),
                           "global_batch": args.batch, "per_gpu_batch_rank0": nb, "parallelism": f"dp{world}",
                           "weights": ("random-init, E4M3 with one fp32 scale per tensor (eva02.bin v3), fp16 head"
                                       if args.v3 else "random-init, E4M3 with fp32 scales per 128x128 block" +
                                       (" (max / 448)" if args.free_scales else
                                        " (powers of two, max / 448 rounded up)")) +
                                      (", QKV / O / W12 / W2 2:4-pruned by magnitude" if args.sparse else ""),
                           "sparse_kinds": sparse_kinds, "block_scale_kinds": block_scale_kinds,
                           "l2": "no flush: the working set per step (0.33 GB weights + activations) exceeds L2"},
                "e2e": {"value": e2e, "unit": "images/s", "h2d_bytes_per_step": args.batch * 1024 * 592 * 2,
                        "d2h_bytes_per_step": args.batch * args.nt * 4},
                "roofline": roof_att,
                "roofline_fc1": roof_fc1,
                "value_clock_normalised": (value * clocks["sm_max_mhz"] / clocks["sm_mhz"]
                                           if clocks.get("sm_mhz") and clocks.get("sm_max_mhz") else None),
                "value_clock_normalised_how": "value x max SM clock / median SM clock during the timed region (for "
                                              "comparing runs at different clocks, e.g. across GPU counts)",
                "free_scales": free_scales,
                "gemm_config1": gemm1,
                "forward_tflops": FLOP_PER_IMAGE * value / 1e12,
                "e2e_decoded": decoded,
                "profile_ms": prof,
                "clocks": clocks,
                "gpu_launches": launches * args.steps * world}
        if out:
            line["cpu_baseline"] = out
        print(json.dumps(line), flush=True)
    if pg:
        pg.destroy_process_group()


def config_name(args):
    """The benchmark-plan config a run corresponds to (2: batch 1; 3: batch 64; 4: batch 32 with 13461 tags;
    5: 2:4-sparse projections)."""
    if args.sparse:
        return "config 5"
    if args.v3:
        return f"batch {args.batch}, {args.nt} tags, reference v3 weights"
    if args.nt == NT and args.batch == 1:
        return "config 2"
    if args.nt == NT and args.batch == 64:
        return "config 3"
    if args.nt == 13461 and args.batch == 32:
        return "config 4"
    return f"batch {args.batch}, {args.nt} tags"


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--batch", type=int, default=None, help="global batch (default 64; 128 with --sparse)")
    ap.add_argument("--no-cpu", action="store_true", help="skip the CPU baseline sample")
    ap.add_argument("--no-extra", action="store_true",
                    help="skip the extra single-GPU keys (free_scales forward, config-1 GEMM)")
    ap.add_argument("--nt", type=int, default=NT, help="head size (tags): 10861, or 13461 for the PixAI-style config")
    ap.add_argument("--sparse", action="store_true", help="config 5: 2:4-pruned projections on the sparse kernels")
    ap.add_argument("--v3", action="store_true", help="weights in the reference's v3 format (per-tensor scales)")
    ap.add_argument("--free-scales", action="store_true",
                    help="block scales max / 448 instead of powers of two: every projection on the promoting kernels")
    ap.add_argument("--mix", action="store_true",
                    help="inputs: whole images + quadrant crops of 896^2 sources, preprocessed on the device (the "
                         "default for config 4: --nt 13461 --batch 32)")
    args = ap.parse_args()
    rank, world, local = dist_env()
    MODEL_KW["nt"] = args.nt
    if args.batch is None:
        args.batch = 128 if args.sparse else 64
    args.mix = args.mix or (args.nt == 13461 and args.batch == 32)
    if args.v3:
        MODEL_KW.update(version=3, head_fp8=False)
    if args.free_scales or args.v3:
        MODEL_KW["pow2"] = False
    if args.sparse:
        MODEL_KW["prune24"] = True
        os.environ.setdefault("XTB_SPARSE", "1")  # the engine's sparse kernels are opt-in
    if args.impl == "reference":
        run_reference(args, rank, world)
    else:
        run_ours(args, rank, world, local)


if __name__ == "__main__":
    main()
