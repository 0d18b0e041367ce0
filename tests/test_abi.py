"""The C ABI boundary, on CPU: the library loads and exports every declared symbol, the host-side
parts (CSR build, edge packing, strict model loading) behave like the reference's. No GPU."""
import json
import os
import re

import numpy as np
import pytest

import oracle
import varda_b200 as vb
from conftest import REPO
from varda_b200 import safetensors as st

HEADER = os.path.join(REPO, "include", "varda_b200.h")


def declared_functions():
    text = open(HEADER).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(vb_[a-z0-9_]+)\s*\(", text)))


def test_library_exports_every_declared_symbol():
    names = declared_functions()
    assert len(names) >= 25
    for n in names:
        assert hasattr(vb.lib, n), f"{n} declared in include/varda_b200.h but not exported"


def random_graph(rng, ns, nd, E):
    return np.stack([rng.integers(0, ns, E), rng.integers(0, nd, E)]).astype(np.int64)


@pytest.mark.parametrize("seed,ns,nd,E,A", [(0, 50, 40, 0, 3), (1, 300, 200, 5000, 3), (2, 7, 1000, 30000, 2),
                                             (3, 10000, 97, 20000, 1)])
def test_build_csr_bit_exact(seed, ns, nd, E, A):
    rng = np.random.default_rng(seed)
    ei = random_graph(rng, ns, nd, E)
    ea = rng.normal(size=(E, A)).astype(np.float32)
    got = vb.build_csr(ei, ea, ns, nd)
    ref = oracle.build_csr(ei, ea, ns, nd)
    for g, r in zip(got, ref):
        assert g.dtype == r.dtype and np.array_equal(g, r)


def test_build_csr_rejects_out_of_range():
    ei = np.array([[0, 5], [0, 1]], np.int64)
    with pytest.raises(vb.VardaError) as e:
        vb.build_csr(ei, np.zeros((2, 3), np.float32), 5, 2)
    assert e.value.code == 2 and "out of range" in str(e.value)


def test_pack_edges_layout_and_rounding():
    src = np.array([3, 0, 7], np.int32)
    at = np.array([[0.1, 1.0 / 3, 2.0], [5.0, -1.5, 0.2], [1e-3, 7.7, -2.2]], np.float32)
    p = vb.pack_edges(src, at[:, :2], round_fp16=False)
    assert np.array_equal(p[:, :2], at[:, :2]) and np.all(p[:, 2] == 0)
    assert np.array_equal(p[:, 3].view(np.int32), src)
    p16 = vb.pack_edges(src, at, round_fp16=True)
    assert np.array_equal(p16[:, :3], at.astype(np.float16).astype(np.float32))


def _small_model(tmp_path, mutate=None, cfg_mutate=None):
    from varda_b200 import synth
    cfg, t, x = synth.config_test("t128")
    if mutate:
        mutate(t)
    if cfg_mutate:
        cfg_mutate(cfg)
    p = str(tmp_path / "m.safetensors")
    synth.write_model(p, cfg, t)
    return p


def _load_error(path):
    with pytest.raises(vb.VardaError) as e:
        vb.Model.load(path, precision=vb.FP32)
    return e.value


def test_load_rejects_missing_tensor(tmp_path):
    err = _load_error(_small_model(tmp_path, mutate=lambda t: t.pop("proc.0.mlp1.weight")))
    assert err.code == 2 and "no tensor 'proc.0.mlp1.weight'" in str(err)


def test_load_rejects_unconsumed_tensor(tmp_path):
    err = _load_error(_small_model(tmp_path, mutate=lambda t: t.__setitem__("extra.thing", np.zeros(3, np.float32))))
    assert err.code == 2 and "extra.thing" in str(err)


@pytest.mark.parametrize("edit,msg", [
    (lambda c: c["architecture"]["processor"].__setitem__("kind", "gnn"), "architecture.processor.kind"),
    (lambda c: c["dims"].__setitem__("gelu_approximate", "erf2"), "gelu_approximate"),
    (lambda c: c.__setitem__("format_version", 2), "format_version"),
    (lambda c: c["bounding"].append({"type": "softplus", "index": [0]}), "softplus"),
    (lambda c: c["residual"].__setitem__("step", 5), "residual.step"),
])
def test_load_rejects_bad_config(tmp_path, edit, msg):
    err = _load_error(_small_model(tmp_path, cfg_mutate=edit))
    assert err.code == 2 and msg in str(err)


def test_load_rejects_missing_file(tmp_path):
    err = _load_error(str(tmp_path / "nope.safetensors"))
    assert err.code == 2 and "cannot open" in str(err)


def test_python_binding_requires_library():
    assert os.path.exists(vb.LIB_PATH)


def test_build_csr_bit_exact_threaded():
    """Above 2^20 edges the CSR build runs on several threads (per-thread counts, slots handed out in
    range order): still the one-pass stable counting sort, bit for bit."""
    rng = np.random.default_rng(11)
    ns, nd, E, A = 50000, 30000, 3_000_000, 3
    ei = random_graph(rng, ns, nd, E)
    ea = rng.normal(size=(E, A)).astype(np.float32)
    rp, src, eid, attr = vb.build_csr(ei, ea, ns, nd)
    order = np.argsort(ei[1], kind="stable")
    assert np.array_equal(eid, order)
    assert np.array_equal(src, ei[0][order])
    assert np.array_equal(attr, ea[order])
    assert np.array_equal(rp, np.concatenate([[0], np.cumsum(np.bincount(ei[1], minlength=nd))]))
    packed = vb.pack_edges(src, attr, round_fp16=True)
    assert np.array_equal(packed[:, :3], attr.astype(np.float16).astype(np.float32))
    assert np.array_equal(packed[:, 3].view(np.int32), src)


def test_output_arrays_are_checked_before_the_library_writes_them():
    """Arrays the library writes through a raw pointer (predict_step's y) must be fp32, C-contiguous,
    writable and of the output's size; anything else is rejected in Python, before the call."""
    ok = np.zeros((1, 2, 1, 5, 3), np.float32)
    vb._check_out(ok, 30, "y")
    bad = [np.zeros(30, np.float64), np.zeros((3, 20), np.float32)[:, :10], np.zeros(29, np.float32), [0.0] * 30]
    ro = np.zeros(30, np.float32)
    ro.flags.writeable = False
    for a in bad + [ro]:
        with pytest.raises(ValueError, match="y "):
            vb._check_out(a, 30, "y")
