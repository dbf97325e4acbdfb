"""ctypes binding of libxtagger_b200.so (the C ABI declared in include/xtagger_b200.h).

The library is built in-tree by ``python -m xtagger_b200.build``. There is no fallback: if the shared library is
missing or does not load, every call raises.
"""
import ctypes as C
import os
import re

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libxtagger_b200.so")
HEADER = os.path.join(os.path.dirname(HERE), "include", "xtagger_b200.h")

EVA_NB, EVA_NBUF, EVA_D, EVA_T, EVA_NP, EVA_K0P = 8, 8, 1024, 1025, 1024, 592
EVA_IN = EVA_NP * EVA_K0P


class Eva(C.Structure):
    """Mirror of `struct eva` in include/xtagger_b200.h."""
    _fields_ = [
        ("nt", C.c_uint32), ("ntp", C.c_uint32), ("nt0", C.c_uint32), ("nb", C.c_uint32),
        ("hout", C.POINTER(C.c_float) * EVA_NBUF),
        ("hpn", C.POINTER(C.c_uint16) * EVA_NBUF),
        ("impl", C.c_void_p),
    ]


PX_NB, PX_NBUF, PX_T = 4, 4, 5184
PX_IN = PX_T * EVA_K0P


class Px(C.Structure):
    """Mirror of `struct px` in include/xtagger_b200.h."""
    _fields_ = [
        ("nt", C.c_uint32), ("ntp", C.c_uint32), ("nb", C.c_uint32),
        ("hout", C.POINTER(C.c_float) * PX_NBUF),
        ("impl", C.c_void_p),
    ]


_lib = None

_P = C.c_void_p
_PX = C.POINTER(Px)
_SIGS = {
    "px_open": (C.c_int, [_PX, C.c_char_p, C.c_int, _P, C.c_size_t]),
    "px_open_ex": (C.c_int, [_PX, C.c_char_p, C.c_int, C.c_uint32, _P, C.c_size_t]),
    "px_open_multi": (C.c_int, [_PX, C.c_char_p, C.POINTER(C.c_int), C.c_int, C.c_uint32, _P, C.c_size_t]),
    "px_ready": (C.c_int, [_PX]),
    "px_poll": (C.c_int, [_PX]),
    "px_submit": (C.c_int, [_PX, C.c_uint32, C.POINTER(_P), C.c_uint32]),
    "px_query": (C.c_int, [_PX, C.c_uint32]),
    "px_wait": (C.POINTER(C.c_float), [_PX, C.c_uint32]),
    "px_close": (None, [_PX]),
    "px_forward_resident": (C.c_int, [_PX]),
    "px_upload": (C.c_int, [_PX, C.POINTER(_P), C.c_uint32]),
    "px_download": (C.c_int, [_PX, _P, C.c_uint32]),
    "px_head_input": (C.c_int, [_PX, _P, C.c_uint32]),
    "px_stream": (_P, [_PX]),
    "px_input": (_P, [_PX]),
    "px_launches_per_forward": (C.c_int, [_PX]),
    "px_profile": (C.c_int, [_PX, _P, C.c_int]),
    "px_prof_name": (C.c_char_p, [C.c_int]),
    "xtb_px_attention": (C.c_int, [_P, _P, _P, C.c_int, C.c_int, _P, C.c_float, C.c_float, _P]),
    "xtb_px_fc1": (C.c_int, [_P, C.c_int, _P, C.c_float, C.c_float, _P, _P, _P, _P]),
    "eva_open": (C.c_int, [C.POINTER(Eva), C.c_char_p, C.c_int, _P, C.c_size_t, C.c_uint32]),
    "eva_open_ex": (C.c_int, [C.POINTER(Eva), C.c_char_p, C.POINTER(C.c_int), C.c_int, C.c_uint32, _P, C.c_size_t,
                              C.c_uint32]),
    "eva_ready": (C.c_int, [C.POINTER(Eva)]),
    "eva_poll": (C.c_int, [C.POINTER(Eva)]),
    "eva_submit": (C.c_int, [C.POINTER(Eva), C.c_uint32, C.POINTER(_P), C.c_uint32]),
    "eva_query": (C.c_int, [C.POINTER(Eva), C.c_uint32]),
    "eva_wait": (C.POINTER(C.c_float), [C.POINTER(Eva), C.c_uint32]),
    "eva_head_put": (C.c_int, [C.POINTER(Eva), C.c_uint32, _P, C.c_float]),
    "eva_head_get": (C.c_int, [C.POINTER(Eva), _P, _P]),
    "eva_close": (None, [C.POINTER(Eva)]),
    "eva_forward_resident": (C.c_int, [C.POINTER(Eva)]),
    "eva_upload": (C.c_int, [C.POINTER(Eva), C.POINTER(_P), C.c_uint32]),
    "eva_download": (C.c_int, [C.POINTER(Eva), _P, C.c_uint32]),
    "eva_stream": (_P, [C.POINTER(Eva), C.c_int]),
    "eva_input": (_P, [C.POINTER(Eva), C.c_int]),
    "eva_output": (_P, [C.POINTER(Eva), C.c_int]),
    "eva_launches_per_forward": (C.c_int, [C.POINTER(Eva)]),
    "eva_sparse_kinds": (C.c_int, [C.POINTER(Eva)]),
    "eva_block_scale_kinds": (C.c_int, [C.POINTER(Eva)]),
    "eva_profile": (C.c_int, [C.POINTER(Eva), _P, C.c_int]),
    "eva_prof_name": (C.c_char_p, [C.c_int]),
    "xtb_gemm_e4m3_f32": (C.c_int, [_P, C.c_int, C.c_int, _P, C.c_int, _P, C.c_float, _P, _P]),
    "xtb_ln_e4m3": (C.c_int, [_P, _P, _P, _P, C.c_int, C.c_float, _P]),
    "xtb_qkv": (C.c_int, [_P, C.c_int, _P, _P, C.c_float, _P, _P, _P, _P, C.c_float, C.c_float, C.c_float, _P]),
    "xtb_attention": (C.c_int, [_P, _P, _P, C.c_int, _P, C.c_float, C.c_float, _P]),
    "xtb_oproj": (C.c_int, [_P, C.c_int, _P, _P, C.c_float, _P, _P]),
    "xtb_fc1": (C.c_int, [_P, C.c_int, _P, _P, C.c_float, _P, _P, _P, _P]),
    "xtb_sf_image_bytes": (C.c_size_t, [C.c_int, C.c_int]),
    "xtb_sf_image": (C.c_int, [_P, C.c_int, C.c_int, _P]),
    "xtb_fc1_mx": (C.c_int, [_P, C.c_int, _P, _P, C.c_float, _P, _P, _P, _P]),
    "xtb_gemm_mx_f32": (C.c_int, [_P, C.c_int, C.c_int, _P, C.c_int, _P, C.c_int, C.c_float, _P, C.c_int, _P]),
    "xtb_fc2": (C.c_int, [_P, C.c_int, _P, _P, C.c_float, _P, _P, _P, _P, _P]),
    "xtb_patch_embed": (C.c_int, [_P, C.c_int, _P, _P, _P, _P]),
    "xtb_pool_ln": (C.c_int, [_P, C.c_int, _P, _P, _P, _P, _P, C.c_float, _P]),
    "xtb_head_f16": (C.c_int, [_P, C.c_int, _P, C.c_int, _P, _P, _P]),
    "xtb_head_e4m3": (C.c_int, [_P, C.c_int, _P, _P, C.c_int, C.c_float, _P, _P, _P]),
    "xtb_fc2_noalloc": (C.c_int, [_P, C.c_int, _P, _P, C.c_float, _P, _P, _P, _P, _P]),
    "xtb_amax_f16": (C.c_int, [_P, C.c_int, C.c_int, _P, _P]),
    "xtb_e4m3_encode": (C.c_int, [_P, _P, C.c_size_t, C.c_int, _P]),
    "xtb_sparse24_check": (C.c_int, [_P, C.c_int, C.c_int]),
    "xtb_sparse24_compress": (C.c_int, [_P, C.c_int, C.c_int, _P, _P]),
    "xtb_gemm_sp_e4m3_f32": (C.c_int, [_P, C.c_int, C.c_int, _P, _P, C.c_int, _P, C.c_float, _P, _P]),
    "xtb_qkv_sp": (C.c_int, [_P, C.c_int, _P, _P, _P, C.c_float, _P, _P, _P, _P, C.c_float, C.c_float, C.c_float, _P]),
    "xtb_oproj_sp": (C.c_int, [_P, C.c_int, _P, _P, _P, C.c_float, _P, _P]),
    "xtb_fc1_sp": (C.c_int, [_P, C.c_int, _P, _P, _P, C.c_float, _P, _P, _P, _P]),
    "xtb_fc2_sp": (C.c_int, [_P, C.c_int, _P, _P, _P, C.c_float, _P, _P, _P, _P, _P]),
    "xtb_prep_scratch_bytes": (C.c_size_t, [C.c_int, C.c_int]),
    "xtb_prep_ingest": (C.c_int, [_P, C.c_int, C.c_int, C.c_int, C.c_int, _P, _P]),
    "xtb_prep_crop": (C.c_int, [_P, C.c_int, C.c_int, C.c_int, C.c_int, C.c_int, C.c_int, C.c_int, _P, _P, _P]),
    "xtb_prep_kernels": (C.c_int, [C.c_int] * 6),
    "xtb_copy_async": (C.c_int, [_P, _P, C.c_size_t, _P]),
    "xtb_error_word": (C.c_uint32, [C.c_int]),
    "xtb_error_clear": (None, [C.c_int]),
    "xtb_selftest_wait": (C.c_int, [C.c_uint32, C.c_int, _P]),
}


def header_symbols():
    """Names of every function declared in include/xtagger_b200.h."""
    src = open(HEADER).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return sorted(set(re.findall(r"\b((?:eva|xtb|px)_[a-z0-9_]+)\s*\(", src)))


def lib():
    """The loaded library with argtypes set. Raises OSError if it is missing (no fallback path exists)."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise OSError(f"{LIB_PATH} is missing: run `python -m xtagger_b200.build` (no CPU fallback exists)")
        l = C.CDLL(LIB_PATH)
        for name, (res, args) in _SIGS.items():
            f = getattr(l, name, None)
            if f is None:
                continue
            f.restype = res
            f.argtypes = args
        _lib = l
    return _lib


def check(rc, what):
    if rc != 0:
        raise RuntimeError(f"{what} failed (rc {rc}); see the 'eva:' line on stderr")
