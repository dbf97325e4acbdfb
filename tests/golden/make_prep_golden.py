"""Run the reference's own preprocessing (src/core/procimg.h's wd path) on seeded images and record digests of its
outputs (golden_prep.json), against which tests/test_prep_cpu.py checks the oracle (oracle/prep_oracle.c) and
tests/test_prep_gpu.py the GPU kernels, bit for bit.

procimg.h cannot be compiled whole here (it includes the Windows-only engine headers), but the functions of this path
are self-contained static inline C with AVX2 / FMA / F16C intrinsics. At generation time this script cuts them out of
procimg.h where it lies (pi_row_rgbx, pi_half, pi_pyramid, pi_level, pi_lsrc, pi_cubic, pi_axis, pi_vrow, pi_hrow,
pi_idrow, pi_stream, pi_prep and the macros and the pi_pyr type they use), places them in a temporary translation unit
after a preamble of this file's own (the two engine constants, the fields of the tagger state pi_prep touches) and a
driver of this file's own (level 0 with alpha over white as pi_ingest does, the pyramid, one pi_prep per rect), and
compiles it with the reference's release flags (src/CMakeLists.txt:38,73: -O3, -march=native, here x86-64-v3: AVX2,
FMA, F16C). Nothing of procimg.h is written into this repository.

Run where the reference tree is available (its path in $XTAGGER_REF, default: a checkout named "reference" beside
this repository):

    python tests/golden/make_prep_golden.py
TEST INFRASTRUCTURE ONLY."""
import ctypes as C
import hashlib
import json
import os
import re
import subprocess
import sys
import tempfile

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, REPO)
REF = os.environ.get("XTAGGER_REF", os.path.join(os.path.dirname(REPO), "reference"))

FUNCS = ["pi_row_rgbx", "pi_half", "pi_pyramid", "pi_level", "pi_lsrc", "pi_cubic", "pi_axis", "pi_vrow", "pi_hrow",
         "pi_idrow", "pi_stream", "pi_prep"]
MACROS = ["PI_DIV255", "PI_OVER", "PI_OVER_X", "PI_U8F", "PI_BGR", "PI_RGB", "PI_BANDH", "PI_SMAX", "PI_PXRUN", "PI_A32",
          "PI_GROW", "PI_LV", "PI_PYRMIN"]

PREAMBLE = r"""
#include <immintrin.h>
#include <stdint.h>
#include <stddef.h>
#include <stdlib.h>
#include <string.h>
#define EVA_S 448
#define EVA_K0P 592
typedef struct pi_tagger {
    uint32_t S, mt_cap;
    size_t tmp_cap;
    float *tmp, *wx, *wy, *kx, *ky;
    int32_t *sx, *nx, *sy, *ny;
    uint32_t *jo;
    uint16_t *band;
} pi_tagger;
"""

DRIVER = r"""
/* The generator's driver: image rows w * 4 bytes apart at level 0 (64 bytes of slack), alpha over white in place when
 * `alpha` (as pi_ingest), the pyramid, then one pi_prep per rect into out (EVA_IN halves each). */
int gen_prep(const uint8_t *rgba, uint32_t w, uint32_t h, uint32_t alpha, const uint32_t *rects, int nrect,
             uint16_t *out)
{
    pi_pyr p;
    pi_tagger t;
    uint32_t y, j;
    int r;
    memset(&p, 0, sizeof(p));
    memset(&t, 0, sizeof(t));
    p.lw[0] = w;
    p.lh[0] = h;
    p.ls[0] = (size_t)w * 4;
    p.lv[0] = malloc((size_t)w * 4 * h + 64);
    if (!p.lv[0]) return -1;
    memcpy(p.lv[0], rgba, (size_t)w * 4 * h);
    if (alpha)
        for (y = 0; y < h; y++) pi_row_rgbx(p.lv[0] + y * p.ls[0], p.lv[0] + y * p.ls[0], w, 1);
    pi_pyramid(&p);
    t.S = EVA_S;
    t.kx = malloc(PI_SMAX * sizeof(float));
    t.ky = malloc(PI_SMAX * sizeof(float));
    t.sx = malloc(PI_SMAX * sizeof(int32_t));
    t.nx = malloc(PI_SMAX * sizeof(int32_t));
    t.sy = malloc(PI_SMAX * sizeof(int32_t));
    t.ny = malloc(PI_SMAX * sizeof(int32_t));
    t.jo = malloc(PI_SMAX * sizeof(uint32_t));
    for (j = 0; j < PI_SMAX; j++) t.jo[j] = (j / 14) * EVA_K0P + j % 14;
    t.band = _mm_malloc(3 * PI_PXRUN * 2, 64);
    memset(t.band, 0, 3 * PI_PXRUN * 2);
    for (r = 0; r < nrect; r++)
        pi_prep(&t, &p, rects[4 * r], rects[4 * r + 1], rects[4 * r + 2], rects[4 * r + 3],
                out + (size_t)r * 1024 * EVA_K0P);
    free(p.lv[0]);
    if (p.nlv > 1) _mm_free(p.lv[1]);
    _mm_free(t.band);
    _mm_free(t.wx);
    _mm_free(t.wy);
    _mm_free(t.tmp);
    free(t.kx), free(t.ky), free(t.sx), free(t.nx), free(t.sy), free(t.ny), free(t.jo);
    return 0;
}
"""


def _macro(src, name):
    m = re.search(r"^#define " + name + r"\b.*?(?<!\\)\n", src, re.M | re.S)
    assert m, name
    return m.group(0)


def _func(src, name):
    m = re.search(r"^static inline [^;{]*?\b" + name + r"\(", src, re.M)
    assert m, name
    i = src.index("{", m.end())
    depth = 0
    for k in range(i, len(src)):
        depth += {"{": 1, "}": -1}.get(src[k], 0)
        if depth == 0:
            return src[m.start():k + 1] + "\n"
    raise ValueError(name)


def _pyr_type(src):
    m = re.search(r"typedef struct \{[^}]*\} pi_pyr;", src, re.S)
    assert m
    return m.group(0) + "\n"


def build_reference(outdir):
    src = open(os.path.join(REF, "src", "core", "procimg.h")).read()
    tu = PREAMBLE + "".join(_macro(src, n) for n in MACROS) + _pyr_type(src) + "".join(_func(src, n) for n in FUNCS)
    tu += DRIVER
    c = os.path.join(outdir, "ref_prep.c")
    so = os.path.join(outdir, "libref_prep.so")
    open(c, "w").write(tu)
    subprocess.run(["gcc", "-O3", "-march=x86-64-v3", "-fno-semantic-interposition", "-fPIC", "-shared", "-w",
                    "-o", so, c], check=True)
    lib = C.CDLL(so)
    lib.gen_prep.restype = C.c_int
    lib.gen_prep.argtypes = [C.c_void_p, C.c_uint32, C.c_uint32, C.c_uint32, C.c_void_p, C.c_int, C.c_void_p]
    return lib


def _aligned(shape, align=64):
    n = int(np.prod(shape))
    buf = np.zeros(n + align // 2, np.uint16)
    off = (-buf.ctypes.data % align) // 2
    return buf[off:off + n].reshape(shape)


def main():
    from tests.golden.prep_case import cases, image
    with tempfile.TemporaryDirectory() as d:
        lib = build_reference(d)
        out = {}
        for name, w, h, alpha, seed, rects in cases():
            img = image(w, h, alpha, seed)
            r = np.ascontiguousarray(np.array(rects, np.uint32).ravel())
            res = _aligned((len(rects), 1024, 592))          # pi_prep streams 32-byte-aligned stores
            assert lib.gen_prep(img.ctypes.data, w, h, alpha, r.ctypes.data, len(rects), res.ctypes.data) == 0
            out[name] = [hashlib.sha256(res[i].tobytes()).hexdigest() for i in range(len(rects))]
            print(name, [s[:12] for s in out[name]])
    out["generated_by"] = ("procimg.h's pi_row_rgbx / pi_pyramid / pi_prep (and the functions they call), extracted at "
                           "generation time, gcc -O3 -march=x86-64-v3")
    with open(os.path.join(HERE, "golden_prep.json"), "w") as fh:
        json.dump(out, fh, indent=0, sort_keys=True)


if __name__ == "__main__":
    main()
