"""Failure paths, exercised from the host without a GPU fault (on the B200, through the C ABI).

* A CUDA graph capture that fails (VB_DEBUG_CAPTURE_FAIL=1 makes every capture fail as a throwing
  launch inside it would; the reference's own hook is VARDA_DEBUG_CAPTURE_THROW,
  src/varda/cuda/backend_cuda.cu:170-172): the engine reports it on stderr and runs eagerly, with the
  same bits as a model whose captures succeed: predict_step through host buffers (eager, then the
  graph or pipelined path), the device entry point, and the device rollout.
* A bounded device-side wait that runs out: the tensor-core attention's consumer warps wait for a head
  stage that its producer, by a test flag (VB_DEBUG_TC_WITHHOLD=1), never fills, under a 20 ms limit
  (VB_DEBUG_WAIT_NS). The kernel gives up, the host reads VB_ERR_TIMEOUT (code 6) from
  vb_check_device, and the device stays usable: the same launch without the flag then matches the
  gather kernel.
"""
import numpy as np
import pytest

import oracle
import varda_b200 as vb
from varda_b200 import safetensors as st

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")


@pytest.mark.parametrize("name", ["t256", "t1024"])
def test_capture_failure_falls_back_to_eager(name, seeded_model, monkeypatch, capfd):
    mp, xp = seeded_model(name)
    x = np.array(st.read(xp)[0]["in.x"])
    good = vb.Model.load(mp, precision=vb.FP16)
    want = [good.predict_step(x) for _ in range(3)]
    good.free()
    monkeypatch.setenv("VB_DEBUG_CAPTURE_FAIL", "1")
    m = vb.Model.load(mp, precision=vb.FP16)
    got = [m.predict_step(x) for _ in range(3)]  # eager, then the capture attempts fail
    vb.check_device()
    for g, w in zip(got, want):
        assert np.array_equal(g, w), "the eager fallback gives the graph path's bits"
    assert "capture failed" in capfd.readouterr().err
    # the device entry point
    xd = torch.from_numpy(x).cuda()
    yd = torch.empty(m.output_shape, device="cuda")
    m.predict_step_device(xd, yd)
    torch.cuda.synchronize()
    assert np.array_equal(yd.cpu().numpy(), want[0])
    m.free()


def test_capture_failure_rollout(seeded_model, monkeypatch):
    from conftest import rollout_golden
    mp, xp = seeded_model("t256r")
    x = np.array(st.read(xp)[0]["in.x"])
    f = rollout_golden("t256r")["forcings"]
    good = vb.Model.load(mp, precision=vb.FP16)
    want, _ = good.rollout(x, f.shape[0] + 1, f)
    good.free()
    monkeypatch.setenv("VB_DEBUG_CAPTURE_FAIL", "1")
    m = vb.Model.load(mp, precision=vb.FP16)
    got, _ = m.rollout(x, f.shape[0] + 1, f)
    vb.check_device()
    assert np.array_equal(got, want), "the rollout's eager fallback gives the graph path's bits"
    m.free()


def _unique_local_graph(rng, n, A, window=40):
    s, d = [], []
    for i in range(n):
        deg = int(rng.integers(0, 30))
        off = rng.choice(np.arange(-window, window + 1), deg, replace=False)
        s += list(np.unique(np.clip(i + off, 0, n - 1)))
        d += [i] * (len(s) - len(d))
    return np.stack([np.array(s, np.int64), np.array(d, np.int64)]), rng.normal(size=(len(s), A)).astype(np.float32)


def test_bounded_wait_runs_out_and_the_device_stays_usable(monkeypatch):
    rng = np.random.default_rng(3)
    C, heads, A, n = 1024, 16, 3, 600
    hd = C // heads
    ei, ea = _unique_local_graph(rng, n, A)
    rp, src, _, attr = vb.build_csr(ei, ea, n, n)
    attr = attr.astype(np.float16).astype(np.float32)
    T = torch.float16
    ld = C
    q, k, v, xr = (torch.from_numpy(rng.normal(size=(n, ld)).astype(np.float16)).cuda() for _ in range(4))
    w4 = np.zeros((4, C), np.float32)
    w4[:A] = (rng.normal(size=(C, A)) * 0.5).astype(np.float16).astype(np.float32).T
    w4[3] = (rng.normal(size=C) * 0.5).astype(np.float16).astype(np.float32)
    d_w = torch.from_numpy(w4).cuda()
    tiles = vb.Tiles(rp, src, attr, n, hd, kind=vb.Tiles.TC)
    out = torch.full((n, C), float("nan"), device="cuda", dtype=T)
    monkeypatch.setenv("VB_DEBUG_WAIT_NS", "20000000")
    monkeypatch.setenv("VB_DEBUG_TC_WITHHOLD", "1")
    tiles.attention(0, n, q, ld, k, v, ld, xr, ld, out, C, d_w, C, heads, hd)
    torch.cuda.synchronize()
    with pytest.raises(vb.VardaError) as e:
        vb.check_device()
    assert e.value.code == 6, "a wait that runs out is reported as VB_ERR_TIMEOUT"
    vb.check_device()  # reading the flag clears it
    monkeypatch.delenv("VB_DEBUG_TC_WITHHOLD")
    monkeypatch.delenv("VB_DEBUG_WAIT_NS")
    tiles.attention(0, n, q, ld, k, v, ld, xr, ld, out, C, d_w, C, heads, hd)
    ref = torch.full_like(out, float("nan"))
    edges = vb.pack_edges(src, attr, round_fp16=True)
    vb.attention(vb.FP16, torch.from_numpy(rp).cuda(), torch.from_numpy(edges).cuda(), 0, n, q, ld, k, v, ld, xr, ld,
                 ref, C, d_w, C, heads, hd)
    torch.cuda.synchronize()
    vb.check_device()
    assert oracle.rel_absmax(out.float().cpu().numpy(), ref.float().cpu().numpy()) <= 2e-3
