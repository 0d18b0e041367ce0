"""The B200 device rollout (vb_rollout) and its state-update kernel (vb_rollout_update), through the
C ABI. The reference's tests/test_rollout_cuda.cu strategy: the device loop is bitwise equal to the host
loop on the same backend (predict_step + the update, here the CPU oracle's restatement of
StateUpdate::apply), with CUDA graphs and without, both constant sources; plus parity of the whole
rollout with the reference's own host rollout on the CPU backend (committed goldens,
tests/golden/*.rollout.npz) and the update kernel bitwise against the oracle.
"""
import numpy as np
import pytest

import oracle
import varda_b200 as vb
from conftest import rollout_golden
from varda_b200 import safetensors as st

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")

MODELS = ["t256r", "t128r"]
# rel_absmax against the reference CPU fp32 rollout: step 0 is a predict_step and has its bar (1e-5
# fp32, 3e-3 fp16); later steps feed the outputs back (step_bars).
STEP0 = {vb.FP32: 1e-5, vb.FP16: 3e-3}


def step_bars(mp, x, f, n, oldest, step0):
    """Per-step bars from the model's own error growth, measured on the CPU oracle: g_k = the relative
    difference at step k between two oracle rollouts whose inputs differ by a seeded relative perturbation
    of size step0, divided by that difference at step 0 (for the synthetic models here g_k stays within
    0.77-1.08 over 4 steps). Each step adds at most one predict_step's error (step0), and the error added
    at step j has grown by g_(s-j) by step s, so bar_s = step0 x sum_(k<=s) max(1, g_k). Nothing here
    depends on the B200 path."""
    om = oracle.OracleModel(mp)
    base = oracle.rollout(om, x, n, f, oldest)
    rng = np.random.default_rng(123)
    xq = (x * (1.0 + step0 * rng.uniform(-1.0, 1.0, x.shape))).astype(np.float32)
    pert = oracle.rollout(om, xq, n, f, oldest)
    e = [oracle.rel_absmax(pert[s], base[s]) for s in range(n)]
    g = [max(1.0, v / e[0]) for v in e]
    return [step0 * sum(g[:s + 1]) for s in range(n)], g


def bits(a):
    return np.ascontiguousarray(a, np.float32).view(np.uint32)


@pytest.mark.parametrize("oldest", [False, True])
@pytest.mark.parametrize("T", [1, 2, 3])
def test_update_kernel_bitwise(T, oldest):
    rng = np.random.default_rng(T)
    rows, n_own, V_in, V_out, F = 1000, 700, 11, 9, 3
    prog_in, prog_out, dyn_in, const_in = [0, 4, 7, 10], [8, 1, 3, 0], [2, 5, 9], [1, 3, 6, 8]
    u = oracle.StateUpdate(T, rows, V_in, V_out, prog_in, prog_out, dyn_in, const_in, oldest)
    w = rng.standard_normal((T, rows, V_in)).astype(np.float32)
    y = rng.standard_normal((rows, V_out)).astype(np.float32)
    f = rng.standard_normal((rows, F)).astype(np.float32)
    kind = u.kind.copy()
    if oldest:
        kind[kind == 0] = 3
    dev = lambda a: torch.from_numpy(np.ascontiguousarray(a)).cuda()
    dw, dyo, dyh, df = dev(w), dev(y[:n_own]), dev(y[n_own:]), dev(f)
    dk, ds = dev(kind), dev(u.src)
    for _ in range(3):
        u.apply(w, y, f)
        vb.rollout_update(dw, T, rows, V_in, dyo, dyh, n_own, V_out, df, F, dk, ds)
    torch.cuda.synchronize()
    assert np.array_equal(bits(dw.cpu().numpy()), bits(w))


class HostLoop:
    """The host rollout on the same backend: predict_step of the B200 model plus the oracle's
    StateUpdate::apply (Rollout::run, rollout.cpp:116-155)."""

    def __init__(self, m, cfg):
        self.m, self.cfg = m, cfg

    def predict_step(self, x):
        return self.m.predict_step(x)


@pytest.mark.parametrize("oldest", [False, True])
@pytest.mark.parametrize("dt", [vb.FP32, vb.FP16])
@pytest.mark.parametrize("name", MODELS)
def test_rollout_parity_and_host_loop_bitwise(name, dt, oldest, seeded_model):
    mp, xp = seeded_model(name)
    x = np.array(st.read(xp)[0]["in.x"])
    gold = rollout_golden(name)
    f = gold["forcings"]
    n = gold["y_newest"].shape[0]
    m = vb.Model.load(mp, precision=dt)
    seen = []
    y, ms = m.rollout(x, n, f, constants_oldest=oldest, on_step=lambda s, a: seen.append((s, a.copy())))
    assert [s for s, _ in seen] == list(range(n))
    for s, a in seen:
        assert np.array_equal(bits(a), bits(y[s])), "callback rows == returned rows"
    assert (ms > 0).all()
    ref = gold["y_oldest" if oldest else "y_newest"]
    errs = [oracle.rel_absmax(y[s], ref[s]) for s in range(n)]
    bars, growth = step_bars(mp, x, f, n, oldest, STEP0[dt])
    assert all(e <= b for e, b in zip(errs, bars)), f"per-step errors {errs} against bars {bars} (growth {growth})"
    # device loop == host loop on the same backend, bitwise
    host = oracle.rollout(HostLoop(m, oracle.OracleModel(mp).cfg), x, n, f, oldest)
    assert np.array_equal(bits(y), bits(host))


@pytest.mark.parametrize("dt", [vb.FP32, vb.FP16])
def test_rollout_graph_equals_eager_and_repeats(dt, seeded_model):
    mp, xp = seeded_model("t256r")
    x = np.array(st.read(xp)[0]["in.x"])
    f = rollout_golden("t256r")["forcings"]
    a = vb.Model.load(mp, precision=dt, cuda_graph=True)
    b = vb.Model.load(mp, precision=dt, cuda_graph=False)
    ya, _ = a.rollout(x, 4, f)
    yb, _ = b.rollout(x, 4, f)
    assert np.array_equal(bits(ya), bits(yb))
    ya2, _ = a.rollout(x, 4, f)             # a second run restarts from x0
    assert np.array_equal(bits(ya), bits(ya2))
    ya3, _ = a.rollout(x, 3, f[:2])          # a shorter run is a prefix
    assert np.array_equal(bits(ya[:3]), bits(ya3))


def test_rollout_one_step_is_predict_step(seeded_model):
    mp, xp = seeded_model("t128r")
    x = np.array(st.read(xp)[0]["in.x"])
    m = vb.Model.load(mp, precision=vb.FP16)
    y, _ = m.rollout(x, 1, None)
    assert np.array_equal(bits(y[0]), bits(m.predict_step(x).reshape(y[0].shape)))


def test_rollout_errors(seeded_model):
    mp, xp = seeded_model("t128r")
    x = np.array(st.read(xp)[0]["in.x"])
    m = vb.Model.load(mp, precision=vb.FP16)
    with pytest.raises(vb.VardaError, match="forcings missing"):
        m.rollout(x, 3, None)
    mp2, xp2 = seeded_model("t128")
    m2 = vb.Model.load(mp2, precision=vb.FP16)
    with pytest.raises(vb.VardaError, match="forcings"):
        m2.rollout(np.array(st.read(xp2)[0]["in.x"]), 2, None)
    # the model still works after the failed calls
    y, _ = m.rollout(x, 2, rollout_golden("t128r")["forcings"][:1])
    assert np.isfinite(y).all()
