"""The seeded case on which the weight converter (xtagger_b200/convert.py) is pinned to the reference's own converter
(src/tools/export_eva.py, run unmodified by make_export_golden.py through the `onnx` stand-in in onnx_stub/):
a 24-layer float EVA02-L tagger (xtagger_b200.calib.synthetic_float, 1000 tags) and seeded calibration statistics
in the reference's .calib layout. TEST INFRASTRUCTURE ONLY."""
import json

import numpy as np

NT = 1000
SEED = 17
D, HIDP, HID = 1024, 2736, 2730


def float_model():
    """The float model; its softmax scale is the square of a float32 constant, as the ONNX graph carries sqrt(scale)
    for q and k each (export_eva.py:70-71 squares it back)."""
    from xtagger_b200 import calib as CB
    f = CB.synthetic_float(seed=SEED, nt=NT, nl=24)
    f["attn_scale"] = np.float64(float(np.float32(np.sqrt(1.0 / 64))) ** 2)
    f["head.bias"] = np.random.default_rng(SEED + 1).standard_normal(NT).astype(np.float32)
    return f


def calib_stats():
    """(amax [24][4][2736], qkv [24][3][1024], h [24][2736]) as eva_calib_dump writes them (eva.h:682-701): GEMM-input
    |max| per channel (first 1024 channels for the three d-wide inputs, 2730 for the MLP-LN output), rotated q / k and
    v |max|, raw SwiGLU |max| (pad units zero)."""
    rng = np.random.default_rng(SEED + 2)
    amax = np.zeros((24, 4, HIDP), np.float32)
    amax[:, :3, :D] = np.abs(rng.standard_normal((24, 3, D))) * 2 + 0.5
    amax[:, 3, :HID] = np.abs(rng.standard_normal((24, HID))) * 2 + 0.5
    qkv = (np.abs(rng.standard_normal((24, 3, D))) * 3 + 1).astype(np.float32)
    h = np.zeros((24, HIDP), np.float32)
    h[:, :HID] = np.abs(rng.standard_normal((24, HID))) * 4 + 0.25
    return amax, qkv, h


def write_onnx_npz(f, path):
    """The float model under the ONNX initializer / node / constant names export_eva.py reads (for onnx_stub)."""
    arr, nodes = {}, []

    def init(name, a):
        arr["init/" + name] = np.ascontiguousarray(a)

    def ln(node, prefix):
        init(prefix + ".weight", f[prefix + ".weight"])
        init(prefix + ".bias", f[prefix + ".bias"])
        nodes.append({"name": node, "op_type": "LayerNormalization", "input": ["x", prefix + ".weight",
                                                                              prefix + ".bias"], "output": [node]})

    def mm(node, weight):
        wname = "onnx::MatMul_" + node
        init(wname, np.ascontiguousarray(f[weight].T))                  # MatMul operand: [in][out]
        nodes.append({"name": node, "op_type": "MatMul", "input": ["x", wname], "output": [node]})

    init("core_model.patch_embed.proj.weight", f["patch_embed.weight"].reshape(D, 3, 14, 14))
    init("core_model.patch_embed.proj.bias", f["patch_embed.bias"])
    init("core_model.pos_embed", f["pos_embed"].reshape(1, 1025, D))
    init("core_model.cls_token", f["cls_token"].reshape(1, 1, D))
    init("core_model.head.weight", f["head.weight"])
    init("core_model.head.bias", f["head.bias"])
    arr["const//core_model/blocks.0/attn/Constant_17_output_0"] = f["rope.cos"].astype(np.float32)
    arr["const//core_model/blocks.0/attn/Constant_32_output_0"] = f["rope.sin"].astype(np.float32)
    arr["const//core_model/blocks.0/attn/Sqrt_1_output_0"] = np.array(
        [np.float32(np.sqrt(float(f["attn_scale"])))], np.float32)
    for b in range(24):
        p, q = f"/core_model/blocks.{b}", f"blocks.{b}."
        ln(f"{p}/norm1/LayerNormalization", q + "norm1")
        for n in ("q_proj", "k_proj", "v_proj", "proj"):
            mm(f"{p}/attn/{n}/MatMul", q + f"attn.{n}.weight")
        ln(f"{p}/norm2/LayerNormalization", q + "norm2")
        mm(f"{p}/mlp/fc1_g/MatMul", q + "mlp.fc1_g.weight")
        mm(f"{p}/mlp/fc1_x/MatMul", q + "mlp.fc1_x.weight")
        ln(f"{p}/mlp/norm/LayerNormalization", q + "mlp.norm")
        mm(f"{p}/mlp/fc2/MatMul", q + "mlp.fc2.weight")
    ln("/core_model/fc_norm/LayerNormalization", "fc_norm")
    arr["__nodes__"] = np.array(json.dumps(nodes))
    np.savez(path, **arr)


def section_digests(path):
    """sha256 of the whole file and of every tensor it holds (names of xtagger_b200.model.read_model; per layer l:
    "l.ln1w", "l.qkv", ... ), so that a mismatch names the tensor that differs."""
    import hashlib

    from xtagger_b200 import model as M
    raw = open(path, "rb").read()
    m = M.read_model(path)
    dig = {"file": hashlib.sha256(raw).hexdigest(), "bytes": len(raw), "version": m["version"], "nt": m["nt"]}
    h = lambda a: hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()[:16]  # noqa: E731
    for k in ("table", "pe", "pos", "cs", "fnw", "fnb", "hw", "hb"):
        dig[k] = h(m[k])
    for i, L in enumerate(m["layers"]):
        for k in ("ln1w", "ln1b", "qkv", "o", "ln2w", "ln2b", "w12", "rs", "w2", "c", "d"):
            dig[f"{i}.{k}"] = h(L[k])
    return dig
