"""ctypes binding of the CPU oracle (liboracle.so) — TEST INFRASTRUCTURE ONLY.

Imported by tests/, by __graft_entry__.smoke() and by bench.py's CPU-baseline leg, and nowhere else: the oracle
is the checker, never the thing measured or shipped.
"""
import ctypes as C
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB = os.path.join(HERE, "liboracle.so")
_lib = None

_u8 = np.ctypeslib.ndpointer(np.uint8, flags="C_CONTIGUOUS")
_u16 = np.ctypeslib.ndpointer(np.uint16, flags="C_CONTIGUOUS")
_f32 = np.ctypeslib.ndpointer(np.float32, flags="C_CONTIGUOUS")
_f64 = np.ctypeslib.ndpointer(np.float64, flags="C_CONTIGUOUS")


def build():
    subprocess.run(["make", "-s", "-C", HERE], check=True)
    return LIB


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(LIB):
            build()
        l = C.CDLL(LIB)
        sig = {
            "or_e4m3": (C.c_uint8, [C.c_float]),
            "or_e4m3_dec": (C.c_float, [C.c_uint8]),
            "or_e4m3_n": (None, [_f32, _u8, C.c_size_t]),
            "or_e4m3_dec_n": (None, [_u8, _f32, C.c_size_t]),
            "or_f2h_n": (None, [_f32, _u16, C.c_size_t]),
            "or_h2f_n": (None, [_u16, _f32, C.c_size_t]),
            "or_gemm_e4m3": (None, [_u8, C.c_int, C.c_int, _u8, C.c_int, _f32, C.c_float, _f32]),
            "or_gemm_f16": (None, [_u16, C.c_int, C.c_int, _u16, C.c_int, _f32]),
            "or_ln_e4m3": (None, [_u16, _f32, _f32, C.c_int, C.c_float, _u8]),
            "or_qkv_epilogue": (None, [_f32, C.c_int, _f32, C.c_float, C.c_float, C.c_float, _u8, _u8, _u8]),
            "or_attention": (None, [_u8, _u8, _u8, C.c_int, C.c_float, C.c_float, C.c_int, C.c_int, _u8]),
            "or_resid_add": (None, [_u16, _f32, C.c_int]),
            "or_fc1_epilogue": (None, [_f32, C.c_int, _f32, _u8, _f64, _f64]),
            "or_fc2_epilogue": (None, [_u16, _f32, C.c_int, _f64, _f64, _f32, _f32]),
            "or_patch_embed": (None, [_u16, C.c_int, _u16, _f32, _u16]),
            "or_pool_ln": (None, [_u16, C.c_int, _f32, _f32, _f32, _u16, C.c_void_p, C.c_float]),
            "or_head_f16": (None, [_u16, C.c_int, _u16, _f32, C.c_int, _f32]),
            "or_head_e4m3": (None, [_u8, C.c_int, _u8, _f32, C.c_float, _f32, C.c_int, _f32]),
            "or_forward": (C.c_int, [C.c_char_p, _u16, C.c_int, C.c_int, C.c_int, _f32, C.c_void_p]),
            "or_model_nt": (C.c_int, [C.c_char_p]),
            "or_prune24": (None, [_u8, C.c_int, C.c_int, C.c_int]),
            "or_threads": (C.c_int, []),
            "or_set_threads": (C.c_int, [C.c_int]),
            "or_div255": (C.c_uint32, [C.c_uint32]),
            "or_over_white": (None, [_u8, C.c_int, C.c_int, C.c_int, C.c_int]),
            "or_half": (None, [_u8, C.c_int, C.c_int, C.c_int, _u8, C.c_int]),
            "or_prep": (None, [_u8, C.c_int, C.c_int, C.c_int, C.c_int, C.c_int, C.c_int, C.c_int, C.c_int, _u16]),
            "or_prep_level": (C.c_int, [C.c_int, C.c_int, C.c_int]),
            "or_px_embed": (None, [_u16, C.c_int, _u16, _f32, _f32, _f32, _u16]),
            "or_px_qkv_epilogue": (None, [_f32, C.c_int, C.c_int, _f32, _f32, C.c_float, C.c_float, C.c_float, _u8,
                                          _u8, _u8]),
            "or_px_attention": (None, [_u8, _u8, _u8, C.c_int, C.c_int, C.c_float, C.c_float, C.c_int, C.c_int,
                                       _u8]),
            "or_px_resid_bias": (None, [_u16, _f32, _f32, C.c_int]),
            "or_px_fc1_epilogue": (None, [_f32, C.c_int, _f32, _f32, _u8]),
            "or_px_head": (None, [_u16, C.c_int, _f32, _f32, _f32, _u16, _u16, _u16, _f32, C.c_int, _f32,
                                  C.c_void_p]),
            "or_px_forward": (C.c_int, [C.c_char_p, _u16, C.c_int, C.c_int, C.c_int, _f32, C.c_void_p]),
            "or_px_model_nt": (C.c_int, [C.c_char_p]),
        }
        for name, (res, args) in sig.items():
            f = getattr(l, name)
            f.restype = res
            f.argtypes = args
        _lib = l
    return _lib


def use_all_cores():
    """Run the oracle's parallel regions on every core this process may use (torch.distributed.run sets
    OMP_NUM_THREADS=1 for its workers); returns the thread count."""
    return lib().or_set_threads(len(os.sched_getaffinity(0)))


def e4m3(x):
    x = np.ascontiguousarray(x, np.float32)
    y = np.empty(x.shape, np.uint8)
    lib().or_e4m3_n(x.ravel(), y.ravel(), x.size)
    return y


def e4m3_dec(b):
    b = np.ascontiguousarray(b, np.uint8)
    y = np.empty(b.shape, np.float32)
    lib().or_e4m3_dec_n(b.ravel(), y.ravel(), b.size)
    return y


def gemm_e4m3(a, w, ws, ascale):
    m, k = a.shape
    n = w.shape[0]
    out = np.empty((m, n), np.float32)
    lib().or_gemm_e4m3(np.ascontiguousarray(a), m, k, np.ascontiguousarray(w), n,
                       np.ascontiguousarray(ws, np.float32), ascale, out)
    return out


def gemm_f16(a, w):
    m, k = a.shape
    n = w.shape[0]
    out = np.empty((m, n), np.float32)
    lib().or_gemm_f16(np.ascontiguousarray(a), m, k, np.ascontiguousarray(w), n, out)
    return out


def forward(model, inputs, key_tile=64, slice_rows=16, want_pn=False):
    """Scores [nimg][nt] (and fp16 pn [nimg][1024]) of the whole forward on the CPU. The defaults are the
    reference's attention: 64-key tiles, lazy-rescale / dead-tile decisions per 16-row warp slice."""
    inputs = np.ascontiguousarray(inputs, np.uint16)
    nimg = inputs.shape[0]
    nt = lib().or_model_nt(model.encode())
    if nt <= 0:
        raise RuntimeError(f"oracle cannot read {model}")
    scores = np.empty((nimg, nt), np.float32)
    pn = np.empty((nimg, 1024), np.uint16) if want_pn else None
    rc = lib().or_forward(model.encode(), inputs.ravel(), nimg, key_tile, slice_rows, scores,
                          pn.ctypes.data_as(C.c_void_p) if want_pn else None)
    if rc:
        raise RuntimeError("oracle forward failed")
    return (scores, pn) if want_pn else scores


def px_forward(model, inputs, key_tile=64, slice_rows=16, want_o=False):
    """PixAI scores [nimg][nt] (and the head's fp16 o [nimg][1024]) of the whole forward on the CPU; the defaults
    are the reference's attention tiling."""
    inputs = np.ascontiguousarray(inputs, np.uint16)
    nimg = inputs.shape[0]
    nt = lib().or_px_model_nt(model.encode())
    if nt <= 0:
        raise RuntimeError(f"oracle cannot read {model}")
    scores = np.empty((nimg, nt), np.float32)
    o = np.empty((nimg, 1024), np.uint16) if want_o else None
    rc = lib().or_px_forward(model.encode(), inputs.ravel(), nimg, key_tile, slice_rows, scores,
                             o.ctypes.data_as(C.c_void_p) if want_o else None)
    if rc:
        raise RuntimeError("oracle PixAI forward failed")
    return (scores, o) if want_o else scores
