"""Run the reference's weight converter, unmodified, on the seeded case of export_case.py and record digests of what
it writes (golden_export_eva.json), against which tests/test_export_pin_cpu.py checks this library's converter.

src/tools/export_eva.py reads the float weights from the upstream ONNX graph with `onnx` (absent from this image);
onnx_stub/ stands in for that package and serves the synthetic float model under the graph's names. Run where the
reference tree is available (its path in $XTAGGER_REF, default: a checkout named "reference" beside this repository):

    python tests/golden/make_export_golden.py
TEST INFRASTRUCTURE ONLY."""
import json
import os
import subprocess
import sys
import tempfile

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, REPO)
REF = os.environ.get("XTAGGER_REF", os.path.join(os.path.dirname(REPO), "reference"))


def main():
    from tests.golden import export_case as E
    from xtagger_b200 import calib as CB
    script = os.path.join(REF, "src", "tools", "export_eva.py")
    assert os.path.exists(script), f"{script} not found (set XTAGGER_REF)"
    f = E.float_model()
    with tempfile.TemporaryDirectory() as d:
        npz, cal, out = os.path.join(d, "model.npz"), os.path.join(d, "model.calib"), os.path.join(d, "eva02.bin")
        E.write_onnx_npz(f, npz)
        CB.write_calib(cal, *E.calib_stats())
        env = dict(os.environ, PYTHONPATH=os.path.join(HERE, "onnx_stub"))
        r = subprocess.run([sys.executable, script, npz, out, cal], env=env, capture_output=True, text=True)
        assert r.returncode == 0, r.stderr
        print(r.stdout.strip())
        dig = E.section_digests(out)
    dig["generated_by"] = "src/tools/export_eva.py (unmodified) on tests/golden/export_case.py through onnx_stub/"
    with open(os.path.join(HERE, "golden_export_eva.json"), "w") as fh:
        json.dump(dig, fh, indent=0, sort_keys=True)
    print("golden_export_eva.json:", dig["file"], dig["bytes"])


if __name__ == "__main__":
    main()
