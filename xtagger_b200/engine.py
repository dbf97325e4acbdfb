"""Python view of the eva_* engine (include/xtagger_b200.h), for tests and the benchmark.

Mirrors the reference's engine calls one to one (eva_open / eva_submit / eva_wait / eva_head_put / eva_head_get /
eva_close, src/engine/eva.h:573-745); errors raise RuntimeError where the C call returns -1 / NULL.
"""
import ctypes as C

import numpy as np

from . import lib as L

EVA_IN = L.EVA_IN


class Engine:
    def __init__(self, weights, devices=(0,), nb=L.EVA_NB, pool=None, extra=0):
        """Open the engine on `devices` with nb inputs per submit. `pool`: optional uint16 numpy array holding the
        inputs (page-locked in place by the bring-up, like the reference's input pool)."""
        self.lib = L.lib()
        self.e = L.Eva()
        self.pool = pool
        devs = (C.c_int * len(devices))(*devices)
        pptr = pool.ctypes.data_as(C.c_void_p) if pool is not None else None
        pbytes = pool.nbytes if pool is not None else 0
        rc = self.lib.eva_open_ex(C.byref(self.e), str(weights).encode(), devs, len(devices), nb, pptr, pbytes, extra)
        L.check(rc, "eva_open_ex")
        self.open = True

    @property
    def nt(self):
        return self.e.nt

    @property
    def nb(self):
        return self.e.nb

    def ready(self):
        L.check(self.lib.eva_ready(C.byref(self.e)), "eva_ready")

    def _ptrs(self, inputs):
        """inputs: list of uint16 arrays of EVA_IN halves (or a [n][1024][592] array)."""
        if isinstance(inputs, np.ndarray) and inputs.ndim == 3:
            inputs = [inputs[i] for i in range(inputs.shape[0])]
        for a in inputs:
            assert a.dtype == np.uint16 and a.size == EVA_IN and a.flags["C_CONTIGUOUS"]
        arr = (C.c_void_p * max(1, len(inputs)))(*[a.ctypes.data for a in inputs])
        return arr, len(inputs)

    def submit(self, buf, inputs):
        arr, n = self._ptrs(inputs)
        self._keep = inputs
        L.check(self.lib.eva_submit(C.byref(self.e), buf, arr, n), "eva_submit")
        return n

    def query(self, buf):
        return bool(self.lib.eva_query(C.byref(self.e), buf))

    def wait(self, buf, n):
        p = self.lib.eva_wait(C.byref(self.e), buf)
        if not p:
            raise RuntimeError("eva_wait failed")
        return np.ctypeslib.as_array(p, shape=(n, self.nt)).copy()

    def hpn(self, buf, n):
        p = self.e.hpn[buf]
        if not p:
            return None
        return np.ctypeslib.as_array(p, shape=(n, 1024)).copy()

    def run(self, inputs, buf=0):
        n = self.submit(buf, inputs)
        return self.wait(buf, n)

    def head_put(self, j, w16, bias):
        w16 = np.ascontiguousarray(w16, np.uint16)
        L.check(self.lib.eva_head_put(C.byref(self.e), j, w16.ctypes.data_as(C.c_void_p), bias), "eva_head_put")

    def head_get(self):
        nt0 = self.e.nt0
        w = np.empty((nt0, 1024), np.uint16)
        b = np.empty(nt0, np.float32)
        L.check(self.lib.eva_head_get(C.byref(self.e), w.ctypes.data_as(C.c_void_p), b.ctypes.data_as(C.c_void_p)),
                "eva_head_get")
        return w, b

    def upload(self, inputs):
        arr, n = self._ptrs(inputs)
        L.check(self.lib.eva_upload(C.byref(self.e), arr, n), "eva_upload")

    def forward_resident(self):
        L.check(self.lib.eva_forward_resident(C.byref(self.e)), "eva_forward_resident")

    def download(self, n):
        out = np.empty((n, self.nt), np.float32)
        L.check(self.lib.eva_download(C.byref(self.e), out.ctypes.data_as(C.c_void_p), n), "eva_download")
        return out

    def stream(self, i=0):
        return self.lib.eva_stream(C.byref(self.e), i)

    def device_input(self, i=0):
        """Device address of the i-th device's resident inputs (what forward_resident reads)."""
        return self.lib.eva_input(C.byref(self.e), i)

    def device_output(self, i=0):
        """Device address of the i-th device's resident scores (what forward_resident writes)."""
        return self.lib.eva_output(C.byref(self.e), i)

    def block_scale_kinds(self):
        return self.lib.eva_block_scale_kinds(C.byref(self.e))

    def launches_per_forward(self):
        return self.lib.eva_launches_per_forward(C.byref(self.e))

    def sparse_kinds(self):
        """Bit mask of the projections on the 2:4-sparse kernels (1 QKV, 2 O, 4 W12, 8 W2)."""
        return self.lib.eva_sparse_kinds(C.byref(self.e))

    def profile(self):
        ms = np.zeros(16, np.float32)
        k = self.lib.eva_profile(C.byref(self.e), ms.ctypes.data_as(C.c_void_p), 16)
        if k < 0:
            raise RuntimeError("eva_profile failed")
        return {self.lib.eva_prof_name(i).decode(): float(ms[i]) for i in range(k)}

    def close(self):
        if getattr(self, "open", False):
            self.lib.eva_close(C.byref(self.e))
            self.open = False

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
