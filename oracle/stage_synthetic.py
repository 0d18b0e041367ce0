"""Build step of the test infrastructure (not the product): stages the reference's own synthetic
generality models and their float64 goldens under oracle/_ref/synthetic/, for the test that runs the
reference's unmodified varda-parity app on this backend (tests/test_reference_harness.py).

The models are written by the reference's python/tests/synthetic.py, imported from the reference
checkout, with the tolerance tables tolerances/synthetic-<name>.json copied beside them. The staged
files are git-ignored and travel with the working tree to the GPU box, where the reference checkout
does not exist. Only the models that keep that tree small are staged: a, f, g and h (about 80 MB in
all). The suite's d (C = 2048, 370 MB) and e (C = 1024, 329 MB) are left out for size; those widths
are covered by this repository's own t2048 / t1024 goldens from the reference's CPU backend.

    python oracle/stage_synthetic.py REFERENCE_TREE [OUT_DIR]
"""
import importlib.util
import os
import shutil
import sys

STAGED = ["a", "f", "g", "h"]


def stage(ref, out):
    os.makedirs(out, exist_ok=True)
    spec = importlib.util.spec_from_file_location("ref_synthetic", os.path.join(ref, "python", "tests", "synthetic.py"))
    syn = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(syn)
    for name in STAGED:
        have = all(os.path.exists(os.path.join(out, f"{name}.{k}.safetensors")) for k in ("model", "golden"))
        if not have:
            syn.generate(name, out)
        shutil.copyfile(os.path.join(ref, "tolerances", f"synthetic-{name}.json"),
                        os.path.join(out, f"synthetic-{name}.json"))


if __name__ == "__main__":
    if len(sys.argv) < 2:
        raise SystemExit(__doc__)
    here = os.path.dirname(os.path.abspath(__file__))
    stage(sys.argv[1], sys.argv[2] if len(sys.argv) > 2 else os.path.join(here, "_ref", "synthetic"))
