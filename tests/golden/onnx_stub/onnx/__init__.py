"""A stand-in for the `onnx` package, just enough for the reference's src/tools/export_eva.py to run unmodified on a
synthetic float model: onnx.load(path) returns an object with .graph.initializer (tensors with .name) and .graph.node
(nodes with .name, .op_type, .input, .output, .attribute), which is all export_eva.py:23-31 reads; the tensors'
values come back through onnx.numpy_helper.to_array. TEST INFRASTRUCTURE ONLY (tests/golden/make_export_golden.py).

`path` is an .npz written by tests/golden/export_case.py: "init/<name>" arrays are initializers, "const/<output>"
arrays are the values of Constant nodes, and "__nodes__" is a JSON list of the other nodes."""
import json

import numpy as np

from . import numpy_helper  # noqa: F401  (export_eva.py imports it from here)


class _Obj:
    def __init__(self, **kw):
        self.__dict__.update(kw)


def load(path):
    z = np.load(path, allow_pickle=False)
    inits = [_Obj(name=k[5:], value=z[k]) for k in z.files if k.startswith("init/")]
    nodes = [_Obj(name=f"Constant_{i}", op_type="Constant", input=[], output=[k[6:]],
                  attribute=[_Obj(name="value", t=_Obj(name=k[6:], value=z[k]))])
             for i, k in enumerate(k for k in z.files if k.startswith("const/"))]
    for n in json.loads(str(z["__nodes__"])):
        nodes.append(_Obj(name=n["name"], op_type=n["op_type"], input=n["input"], output=n["output"], attribute=[]))
    return _Obj(graph=_Obj(initializer=inits, node=nodes))
