"""This library's weight converter (xtagger_b200/convert.py) against the reference's own (src/tools/export_eva.py):
on the seeded 24-layer float model and calibration statistics of tests/golden/export_case.py, convert.py --v3 must
write the same eva02.bin, byte for byte, as export_eva.py did when run unmodified on them
(tests/golden/make_export_golden.py, digests in tests/golden/golden_export_eva.json). That pins the v3 format (header,
256-byte tensor alignment, order), the folds (cls / conv bias into the position table, softmax scale x log2 e into
Wq, the MLP LayerNorm into fc2), SmoothQuant, per-tensor E4M3, the scale table and the reading of the .calib layout
(eva.h:682-701) to the reference's code. The CPU oracle then reads the file."""
import json
import os

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))


def test_convert_writes_the_reference_converters_bytes(tmp_path):
    from tests.golden import export_case as E
    from xtagger_b200 import calib as CB
    from xtagger_b200 import convert as CV
    want = json.load(open(os.path.join(HERE, "golden", "golden_export_eva.json")))
    f = E.float_model()
    cal = str(tmp_path / "model.calib")
    CB.write_calib(cal, *E.calib_stats())             # through the .calib file, as the reference reads it
    path = CV.convert(f, CB.read_calib(cal), str(tmp_path / "eva02.bin"), version=3)
    got = E.section_digests(path)
    diff = sorted(k for k in want if k != "generated_by" and got.get(k) != want[k])
    assert not diff, f"tensors that differ from export_eva.py's output: {diff[:12]}"
    from oracle import oracle as O
    assert O.lib().or_model_nt(path.encode()) == E.NT
    assert np.isfinite(np.fromfile(path, np.float32, 24 * 12, offset=256)).all()
