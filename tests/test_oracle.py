"""The CPU oracle (oracle/), pinned to the reference's own numbers. CPU only.

* against the committed goldens of this repo's seeded models, produced by the reference CPU backend
  compiled from its sources (tests/golden/make_golden.py);
* against the reference's own synthetic generality models a-h and their float64 goldens
  (python/tests/synthetic.py of the reference), when the reference tree is present;
* against the compiled reference itself (oracle/_ref/ref_dump), when built.
"""
import json
import os
import subprocess

import numpy as np
import pytest

import oracle
from conftest import GOLDEN, REFERENCE, REPO, golden
from varda_b200 import safetensors as st

MODELS = ["c0", "t128", "t256", "t512", "t768", "t1024", "t384i", "t2048"]
FP32_TOL = 1e-5


@pytest.mark.parametrize("name", MODELS)
def test_oracle_matches_reference_goldens(name, seeded_model):
    mp, xp = seeded_model(name)
    gold = golden(name)
    x = st.read(xp)[0]["in.x"]
    got = {}
    oracle.OracleModel(mp).predict_step(x, lambda k, a: got.__setitem__(k, a))
    for k, ref in gold.items():
        err = oracle.rel_absmax(got[k], ref)
        assert err <= FP32_TOL, f"{name} {k}: rel_absmax {err:.3e}"


def test_synthetic_pin_summary():
    """The committed record of the pin against the reference's own float64 goldens."""
    pin = json.load(open(os.path.join(GOLDEN, "synthetic_pin.json")))
    assert sorted(pin) == list("abcdefgh")
    for name, rec in pin.items():
        assert rec["worst"] <= rec["tolerance_fp32"], name


@pytest.mark.skipif(not os.path.exists(os.path.join(REFERENCE, "python/tests/synthetic.py")),
                    reason="reference sources not present")
@pytest.mark.parametrize("name", ["a", "b", "f", "h"])
def test_oracle_vs_reference_synthetic_live(name, tmp_path):
    import importlib.util
    spec = importlib.util.spec_from_file_location("ref_syn", os.path.join(REFERENCE, "python/tests/synthetic.py"))
    syn = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(syn)
    syn.generate(name, str(tmp_path))
    from varda_b200 import synth
    pin = json.load(open(os.path.join(GOLDEN, "synthetic_pin.json")))[name]
    mp = str(tmp_path / f"{name}.model.safetensors")
    assert synth.sha256_file(mp) == pin["model_sha256"]
    gold, _ = oracle.read_safetensors(str(tmp_path / f"{name}.golden.safetensors"))
    errs = {}
    oracle.OracleModel(mp).predict_step(gold["in.x"], lambda k, a: errs.__setitem__(k, oracle.rel_absmax(a, gold[k])))
    assert set(errs) == set(gold)
    assert max(errs.values()) <= FP32_TOL, errs


REF_DUMP = os.path.join(REPO, "oracle", "_ref", "ref_dump")


@pytest.mark.skipif(not os.path.exists(REF_DUMP), reason="oracle/_ref not built")
def test_oracle_vs_compiled_reference_live(seeded_model, tmp_path):
    mp, xp = seeded_model("t256")
    dump = str(tmp_path / "d.safetensors")
    subprocess.run([REF_DUMP, "--model", mp, "--input", xp, "--dump", dump, "--threads", "4"], check=True,
                   capture_output=True)
    ref = st.read(dump)[0]
    x = st.read(xp)[0]["in.x"]
    errs = {}
    oracle.OracleModel(mp).predict_step(x, lambda k, a: errs.__setitem__(k, oracle.rel_absmax(a, ref[k])))
    assert len(errs) == len(ref)
    assert max(errs.values()) <= FP32_TOL, errs


def test_csr_oracle_is_stable_counting_sort():
    rng = np.random.default_rng(3)
    E, ns, nd = 5000, 300, 200
    ei = np.stack([rng.integers(0, ns, E), rng.integers(0, nd, E)]).astype(np.int64)
    ea = rng.normal(size=(E, 3)).astype(np.float32)
    rp, src, eid, at = oracle.build_csr(ei, ea, ns, nd)
    order = np.argsort(ei[1], kind="stable")
    assert np.array_equal(eid, order)
    assert np.array_equal(src, ei[0][order])
    assert np.array_equal(at, ea[order])
    assert np.array_equal(rp, np.concatenate([[0], np.cumsum(np.bincount(ei[1], minlength=nd))]))
