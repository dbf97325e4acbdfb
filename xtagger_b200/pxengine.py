"""Python view of the px_* engine (include/xtagger_b200.h), for tests and the benchmark.

Mirrors the reference's PixAI engine calls one to one (px_open / px_submit / px_query / px_wait / px_close,
src/engine/px.h:355-492); errors raise RuntimeError where the C call returns -1 / NULL.
"""
import ctypes as C

import numpy as np

from . import lib as L

PX_IN = L.PX_IN


class PxEngine:
    def __init__(self, weights, device=0, nb=L.PX_NB, pool=None, devices=None):
        """Open the engine on `device` (or on every device of `devices`, px_open_multi) with nb inputs per submit.
        `pool`: optional uint16 numpy array holding the inputs (page-locked in place by the bring-up, like the
        reference's input pool)."""
        self.lib = L.lib()
        self.p = L.Px()
        self.pool = pool
        pptr = pool.ctypes.data_as(C.c_void_p) if pool is not None else None
        pbytes = pool.nbytes if pool is not None else 0
        if devices is not None:
            devs = (C.c_int * len(devices))(*devices)
            L.check(self.lib.px_open_multi(C.byref(self.p), str(weights).encode(), devs, len(devices), nb, pptr,
                                           pbytes), "px_open_multi")
        else:
            L.check(self.lib.px_open_ex(C.byref(self.p), str(weights).encode(), device, nb, pptr, pbytes),
                    "px_open_ex")
        self.open = True

    @property
    def nt(self):
        return self.p.nt

    @property
    def nb(self):
        return self.p.nb

    def ready(self):
        L.check(self.lib.px_ready(C.byref(self.p)), "px_ready")

    def _ptrs(self, inputs):
        """inputs: list of uint16 arrays of PX_IN halves (or a [n][5184][592] array)."""
        if isinstance(inputs, np.ndarray) and inputs.ndim == 3:
            inputs = [inputs[i] for i in range(inputs.shape[0])]
        for a in inputs:
            assert a.dtype == np.uint16 and a.size == PX_IN and a.flags["C_CONTIGUOUS"]
        arr = (C.c_void_p * max(1, len(inputs)))(*[a.ctypes.data for a in inputs])
        return arr, len(inputs)

    def submit(self, buf, inputs):
        arr, n = self._ptrs(inputs)
        self._keep = inputs
        L.check(self.lib.px_submit(C.byref(self.p), buf, arr, n), "px_submit")
        return n

    def query(self, buf):
        return bool(self.lib.px_query(C.byref(self.p), buf))

    def wait(self, buf, n):
        ptr = self.lib.px_wait(C.byref(self.p), buf)
        if not ptr:
            raise RuntimeError("px_wait failed")
        return np.ctypeslib.as_array(ptr, shape=(n, self.nt)).copy()

    def run(self, inputs, buf=0):
        n = self.submit(buf, inputs)
        return self.wait(buf, n)

    def upload(self, inputs):
        arr, n = self._ptrs(inputs)
        L.check(self.lib.px_upload(C.byref(self.p), arr, n), "px_upload")

    def forward_resident(self):
        L.check(self.lib.px_forward_resident(C.byref(self.p)), "px_forward_resident")

    def download(self, n):
        out = np.empty((n, self.nt), np.float32)
        L.check(self.lib.px_download(C.byref(self.p), out.ctypes.data_as(C.c_void_p), n), "px_download")
        return out

    def head_input(self, n):
        """The head's pooled-and-projected vectors o [n][1024] (fp16 bits) of the last forward."""
        o = np.empty((n, 1024), np.uint16)
        L.check(self.lib.px_head_input(C.byref(self.p), o.ctypes.data_as(C.c_void_p), n), "px_head_input")
        return o

    def stream(self):
        return self.lib.px_stream(C.byref(self.p))

    def device_input(self):
        return self.lib.px_input(C.byref(self.p))

    def launches_per_forward(self):
        return self.lib.px_launches_per_forward(C.byref(self.p))

    def profile(self):
        """Per-kind kernel milliseconds of one direct forward (events after every launch)."""
        ms = np.zeros(16, np.float32)
        k = self.lib.px_profile(C.byref(self.p), ms.ctypes.data_as(C.c_void_p), 16)
        L.check(0 if k > 0 else -1, "px_profile")
        return {self.lib.px_prof_name(i).decode(): float(ms[i]) for i in range(k)}

    def close(self):
        if getattr(self, "open", False):
            self.lib.px_close(C.byref(self.p))
            self.open = False

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
