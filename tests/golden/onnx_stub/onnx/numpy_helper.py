"""onnx.numpy_helper stand-in: to_array(tensor) -> the numpy value the stub attached (see __init__.py)."""


def to_array(t):
    return t.value
