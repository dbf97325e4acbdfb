"""Generate the golden vectors that pin the CPU oracle to the reference's own code.

Run in a container where the reference tree is available (its path in $XTAGGER_REF, default: a checkout named "reference" beside this repository);
the outputs are small committed fixtures in this directory, so the tests never need the reference at run time.

  golden_e4m3.npz      inputs and E4M3 codes of the reference's weight quantiser (src/tools/export_eva.py:64-66,
                       `fp8`: clip to +-448, ml_dtypes float8_e4m3fn cast), executed from the reference source
  golden_interleave.npz  row permutation of the reference's fc1 g / x interleave (export_eva.py:60-62)
  golden_prune24.json  sha256 of every pruned matrix of a seeded random v3 blob after the reference's
                       src/tools/prune24.py (magnitude and Wanda modes, all four block GEMMs), run as a subprocess

    python tests/golden/make_golden.py
"""
import ast
import hashlib
import json
import os
import struct
import subprocess
import sys
import tempfile

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))
REF = os.environ.get("XTAGGER_REF", os.path.join(os.path.dirname(REPO), "reference"))

D, T, NP, K0P, HIDP, NL = 1024, 1025, 1024, 592, 2736, 24


def ref_functions(names):
    """Top-level function definitions and constants of export_eva.py, without running its ONNX-loading body."""
    src = open(os.path.join(REF, "src/tools/export_eva.py")).read()
    tree = ast.parse(src)
    def const(v):
        return isinstance(v, ast.Constant) or (isinstance(v, ast.Tuple) and all(isinstance(e, ast.Constant) for e in v.elts))
    keep = [n for n in tree.body if (isinstance(n, ast.FunctionDef) and n.name in names)
            or (isinstance(n, ast.Assign) and const(n.value))]
    mod = ast.Module(body=keep, type_ignores=[])
    import ml_dtypes
    ns = {"np": np, "ml_dtypes": ml_dtypes, "os": os}
    exec(compile(mod, "export_eva.py", "exec"), ns)
    return ns


def e4m3_sweep():
    """Inputs covering every E4M3 code, the ties between neighbours, saturation, subnormals and signed zero."""
    import ml_dtypes
    codes = np.arange(256, dtype=np.uint8)
    vals = codes.view(ml_dtypes.float8_e4m3fn).astype(np.float32)
    fin = np.sort(np.unique(vals[np.isfinite(vals)]))
    mids = (fin[:-1] + fin[1:]) / 2                       # exact ties: round half to even
    rng = np.random.default_rng(0)
    rnd = np.concatenate([rng.standard_normal(20000).astype(np.float32) * s for s in (0.001, 0.05, 1, 30, 300)])
    x = np.concatenate([fin, mids, np.nextafter(mids, np.float32(np.inf)), np.nextafter(mids, np.float32(-np.inf)),
                        rnd, np.array([440, 447.9, 448, -448, 464, 1e4, -1e4, 2 ** -10, 2 ** -9.5, -0.0, 0.0],
                                      np.float32)]).astype(np.float32)
    x = np.clip(x, -448, 448)                              # export_eva.py clips before the cast
    return np.concatenate([x, np.array([448.0, -448.0], np.float32)])  # max |x| = 448: fp8()'s scale is exactly 1


def random_v3_blob(path, seed=11, nt=16):
    """A v3-layout blob with random bytes everywhere (what prune24.py reads: only the layout and the E4M3 matrices)."""
    rng = np.random.default_rng(seed)
    ntp = (nt + 7) & ~7
    sizes = [NL * 12 * 4, D * K0P * 2, T * D * 4, NP * 32 * 2 * 4]
    for _ in range(NL):
        sizes += [D * 4, D * 4, 3 * D * D, D * D, D * 4, D * 4, 2 * HIDP * D, HIDP * 4, D * HIDP, D * 4, D * 4]
    sizes += [D * 4, D * 4, ntp * D * 2, ntp * 4]
    off = 0
    parts = []
    for n in sizes:
        pad = -off % 256
        parts.append(b"\0" * pad)
        off += pad
        parts.append(rng.integers(0, 256, n, dtype=np.uint8).tobytes())
        off += n
    with open(path, "wb") as f:
        f.write(struct.pack("<4sIII", b"EVA2", 3, nt, off) + b"\0" * 240)
        for p in parts:
            f.write(p)


def blob_matrices(path):
    """(name, layer, bytes) of every block-GEMM matrix in a v3 blob, in file order (layout of prune24.py:24-40)."""
    raw = open(path, "rb").read()
    off = 0

    def take(n):
        nonlocal off
        off = (off + 255) & ~255
        o = off
        off += n
        return 256 + o

    take(NL * 12 * 4); take(D * K0P * 2); take(T * D * 4); take(NP * 32 * 2 * 4)
    out = []
    for i in range(NL):
        take(D * 4); take(D * 4)
        o = take(3 * D * D); out.append(("qkv", i, raw[o:o + 3 * D * D]))
        o = take(D * D); out.append(("oproj", i, raw[o:o + D * D]))
        take(D * 4); take(D * 4)
        o = take(2 * HIDP * D); out.append(("fc1", i, raw[o:o + 2 * HIDP * D]))
        take(HIDP * 4)
        o = take(D * HIDP); out.append(("fc2", i, raw[o:o + D * HIDP]))
        take(D * 4); take(D * 4)
    return out


def main():
    ns = ref_functions({"fp8", "interleave"})
    x = e4m3_sweep()
    codes, sc = ns["fp8"](x)
    assert sc == 1.0
    np.savez_compressed(os.path.join(HERE, "golden_e4m3.npz"), x=x, codes=np.asarray(codes, np.uint8))
    rows = np.arange(2 * HIDP, dtype=np.int64)[:, None] * np.ones((1, 2), np.int64)
    perm = ns["interleave"](rows)[:, 0]
    np.savez_compressed(os.path.join(HERE, "golden_interleave.npz"), perm=perm)
    with tempfile.TemporaryDirectory() as d:
        src = os.path.join(d, "rand.bin")
        random_v3_blob(src)
        digests = {}
        for mode in ("wanda", "mag"):
            dst = os.path.join(d, f"pruned_{mode}.bin")
            cmd = [sys.executable, os.path.join(REF, "src/tools/prune24.py"), src, dst, "fc1,fc2,qkv,oproj"]
            if mode == "mag":
                cmd.append("mag")
            subprocess.run(cmd, check=True, capture_output=True)
            digests[mode] = {f"{n}.{i}": hashlib.sha256(b).hexdigest() for n, i, b in blob_matrices(dst)}
    json.dump({"seed": 11, "nt": 16, "digests": digests}, open(os.path.join(HERE, "golden_prune24.json"), "w"),
              indent=0, sort_keys=True)
    print("golden vectors written to", HERE)


if __name__ == "__main__":
    main()
