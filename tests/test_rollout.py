"""The rollout's state update and host loop in the CPU oracle (oracle.StateUpdate / oracle.rollout),
pinned to the reference. CPU only.

The reference's tests/test_rollout.cpp strategy: tiny windows whose values differ per (slot, point,
channel), so a value taken from the wrong slot shows; three consecutive updates, each bitwise equal to
the two upstream definitions executed literally on whole slots (anemoi-inference's advance_map for the
default in-place constants, roll(-1) for the oldest-slot constants); explicit per-slot expectations;
invalid index sets rejected. Then the whole rollout against the reference's own host rollout
(varda::Rollout::run on the CPU backend, committed goldens from oracle/_ref/ref_rollout, and live when
built).
"""
import os
import subprocess

import numpy as np
import pytest

import oracle
from conftest import REPO, rollout_golden
from varda_b200 import safetensors as st
from varda_b200 import synth

G, V_IN, V_OUT = 3, 7, 5
PROG_IN, PROG_OUT, DYN_IN, CONST_IN = [0, 3, 6], [2, 0, 4], [1, 4], [2, 5]


def wval(t, g, c):
    return 1000.0 * (t + 1) + 10.0 * g + c + 0.125


def window(T, G=G, const_equal=False):
    w = np.empty((T, G, V_IN), np.float32)
    for t in range(T):
        for g in range(G):
            for c in range(V_IN):
                w[t, g, c] = wval(0 if (const_equal and c in CONST_IN) else t, g, c)
    return w


def yf(G=G):
    y = np.array([[-(100.0 * g + o) - 0.5 for o in range(V_OUT)] for g in range(G)], np.float32)
    f = np.array([[0.25 + g + 0.0625 * k for k in range(len(DYN_IN))] for g in range(G)], np.float32)
    return y, f


def literal_update(w, y, f, oldest):
    """The two upstream definitions on whole slots (m = 1 output step, n = T input slots):
    advance_map: inin = [(i, i - 1) for i in 1..n-1] applied in order, then outin writes the newest
    slot's prognostic inputs and forcings; roll: the window rolled by -1, then the same writes."""
    T = w.shape[0]
    w = w.copy()
    if oldest:
        w = np.roll(w, -1, axis=0)
    else:
        for i in range(1, T):
            w[i - 1] = w[i]
    for i, o in zip(PROG_IN, PROG_OUT):
        w[T - 1, :, i] = y[:, o]
    for k, c in enumerate(DYN_IN):
        w[T - 1, :, c] = f[:, k]
    return w


@pytest.mark.parametrize("oldest", [False, True])
@pytest.mark.parametrize("T", [1, 2, 3, 4, 5])
def test_update_matches_literal_definitions(T, oldest):
    u = oracle.StateUpdate(T, G, V_IN, V_OUT, PROG_IN, PROG_OUT, DYN_IN, CONST_IN, oldest)
    assert u.F == 2
    w = window(T)
    y, f = yf()
    want = w.copy()
    for rep in range(3):
        want = literal_update(want, y, f, oldest)
        u.apply(w, y, f)
        assert np.array_equal(w.view(np.uint32), want.view(np.uint32)), f"update {rep + 1}"


@pytest.mark.parametrize("oldest", [False, True])
@pytest.mark.parametrize("T", [2, 3, 5])
def test_update_explicit_slots(T, oldest):
    u = oracle.StateUpdate(T, G, V_IN, V_OUT, PROG_IN, PROG_OUT, DYN_IN, CONST_IN, oldest)
    w = window(T)
    y, f = yf()
    u.apply(w, y, f)
    n = T - 1
    for t in range(n):
        for g in range(G):
            for c in range(V_IN):
                assert w[t, g, c] == np.float32(wval(t + 1, g, c)), "slot t is the old slot t+1"
    for g in range(G):
        for i, o in zip(PROG_IN, PROG_OUT):
            assert w[n, g, i] == y[g, o]
        for k, c in enumerate(DYN_IN):
            assert w[n, g, c] == f[g, k]
        for c in CONST_IN:
            want = wval(0, g, c) if oldest else wval(n, g, c)
            assert w[n, g, c] == np.float32(want)
    # second update: in place keeps the newest slot's constants; roll brings the original slot 1 round
    u.apply(w, y, f)
    for g in range(G):
        for c in CONST_IN:
            assert w[n, g, c] == np.float32(wval(1, g, c) if oldest else wval(n, g, c))


@pytest.mark.parametrize("T", [2, 3, 4])
def test_equal_constants_make_both_sources_agree(T):
    a = oracle.StateUpdate(T, 5, V_IN, V_OUT, PROG_IN, PROG_OUT, DYN_IN, CONST_IN, False)
    b = oracle.StateUpdate(T, 5, V_IN, V_OUT, PROG_IN, PROG_OUT, DYN_IN, CONST_IN, True)
    wa = window(T, 5, const_equal=True)
    wb = wa.copy()
    y, f = yf(5)
    for _ in range(3):
        a.apply(wa, y, f)
        b.apply(wb, y, f)
    assert np.array_equal(wa.view(np.uint32), wb.view(np.uint32))


def test_invalid_index_sets_rejected():
    with pytest.raises(ValueError, match="channel 3"):
        oracle.StateUpdate(2, 1, 4, 2, [0], [0], [1], [2])
    with pytest.raises(ValueError, match="twice"):
        oracle.StateUpdate(2, 1, 3, 2, [0], [0], [0], [1, 2])
    with pytest.raises(ValueError, match="out of range"):
        oracle.StateUpdate(2, 1, 3, 2, [0], [5], [1], [2])
    with pytest.raises(ValueError, match="out of range"):
        oracle.StateUpdate(2, 1, 3, 2, [0], [0], [7], [1, 2])
    with pytest.raises(ValueError, match="differ in length"):
        oracle.StateUpdate(2, 1, 3, 2, [0, 1], [0], [], [2])
    cfg, _, _ = synth.config_test("t256")
    with pytest.raises(ValueError, match="forcings"):
        oracle.StateUpdate.from_config(cfg)


def test_update_missing_forcings_rejected():
    u = oracle.StateUpdate(2, G, V_IN, V_OUT, PROG_IN, PROG_OUT, DYN_IN, CONST_IN)
    y, _ = yf()
    with pytest.raises(ValueError, match="forcings missing"):
        u.apply(window(2), y, None)


ROLLOUT_MODELS = ["t256r", "t128r"]
FP32_TOL = 1e-5


@pytest.mark.parametrize("name", ROLLOUT_MODELS)
def test_oracle_rollout_matches_reference_goldens(name, seeded_model):
    mp, xp = seeded_model(name)
    gold = rollout_golden(name)
    x = st.read(xp)[0]["in.x"]
    om = oracle.OracleModel(mp)
    n = gold["y_newest"].shape[0]
    for tag, oldest in (("newest", False), ("oldest", True)):
        y = oracle.rollout(om, x, n, gold["forcings"], oldest)
        for s in range(n):
            err = oracle.rel_absmax(y[s], gold[f"y_{tag}"][s])
            assert err <= FP32_TOL, f"{name} {tag} step {s}: {err:.3e}"
    # the constant source matters on these inputs (constants differ between slots)
    assert not np.array_equal(gold["y_newest"][1:], gold["y_oldest"][1:])


REF_ROLLOUT = os.path.join(REPO, "oracle", "_ref", "ref_rollout")


@pytest.mark.skipif(not os.path.exists(REF_ROLLOUT), reason="oracle/_ref not built")
def test_oracle_rollout_vs_compiled_reference_live(seeded_model, tmp_path):
    mp, xp = seeded_model("t128r")
    x = st.read(xp)[0]["in.x"]
    om = oracle.OracleModel(mp)
    n = 3
    f = synth.replay_forcings(n, om.G, 3, seed=11)
    rp, out = str(tmp_path / "in.safetensors"), str(tmp_path / "y.safetensors")
    st.write(rp, {"in.x": x, "forcings": f}, {})
    subprocess.run([REF_ROLLOUT, "--model", mp, "--input", rp, "--steps", str(n), "--threads", "4", "--oldest",
                    "--out", out], check=True, capture_output=True)
    ref = st.read(out)[0]["y"]
    y = oracle.rollout(om, x, n, f, True)
    assert max(oracle.rel_absmax(y[s], ref[s]) for s in range(n)) <= FP32_TOL
