"""Parity at the shapes the benchmark runs (C1 widths and depth, the C2 graph, full C1), through the C ABI.

* c1s: C1's architecture (C = 1024, 16 heads, mlp 4096, 16 processor blocks, T_in = 2, V_in = 90,
  V_out = 80) on 1/64 of its nodes. Every contract key of the hooked predict_step against the
  reference CPU backend's own values (tests/golden/c1s.sampled.npz: seeded rows and columns of every
  key, from oracle/_ref/ref_dump), with the reference's tolerances (3e-3 fp16, 1e-5 fp32 rel_absmax),
  input keys within 1e-6. The reference's bitwise self-checks too (hook inert, graph replay == eager).
* C2: the isolated processor block's graph (189,809 rows, 2,561,682 edges, C = 1024, 16 heads, fp16):
  the tile-sparse tensor-core, gather, shared-memory-tiled and no-allocation split attention paths
  against the oracle's restatement of cpu::graph_attention on 4,096 seeded rows (16 runs of 256
  consecutive rows), and the paths against each other on every row. Exercises the 64-bit row offsets
  of the [H, 4C] buffer.
* c1: the full Varda-shaped model (G = 1,688,650) in fp16: out.y at 8,192 seeded data nodes against
  one predict_step of the reference's CPU backend on the same model and input
  (tests/golden/c1.y_sample.npz), 3e-3 rel_absmax; graph replay bitwise equal to the eager call.
"""
import os

import numpy as np
import pytest

import oracle
import varda_b200 as vb
from conftest import GOLDEN
from varda_b200 import safetensors as st

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")

TOL = {vb.FP32: 1e-5, vb.FP16: 3e-3}
EXACT = ("in.x", "in.x_norm", "enc.x_src", "enc.x_dst")


def sampled(name):
    z = np.load(os.path.join(GOLDEN, f"{name}.sampled.npz"))
    out = {}
    for k in z.files:
        if k.startswith("__") or k.endswith((".rows", ".cols", ".shape")):
            continue
        out[k] = (z[k], z[k + ".rows"], z[k + ".cols"], tuple(z[k + ".shape"]))
    return out


@pytest.mark.parametrize("dt", [vb.FP16, vb.FP32])
def test_c1s_parity_against_reference(dt, seeded_model):
    mp, xp = seeded_model("c1s")
    ref = sampled("c1s")
    x = np.array(st.read(xp)[0]["in.x"])
    m = vb.Model.load(mp, precision=dt)
    errs, seen = {}, []

    def hook(k, a):
        seen.append(k)
        g, rows, cols, shape = ref[k]
        assert a.shape == shape, (k, a.shape, shape)
        a2 = a.reshape(-1, a.shape[-1])
        got = a2[rows][:, cols]
        assert not np.isnan(got).any(), k
        errs[k] = oracle.rel_absmax(got, g)

    y = m.predict_step(x, hook=hook)
    assert sorted(seen) == sorted(ref), "every contract key of the reference, once"
    assert len(seen) == len(set(seen))
    bad = {k: e for k, e in errs.items() if e > (1e-6 if k in EXACT else TOL[dt])}
    assert not bad, f"over tolerance: {bad} (all: {errs})"
    y2 = m.predict_step(x)
    y3 = m.predict_step(x)
    assert np.array_equal(y2, y), "a hooked run must not change the output"
    assert np.array_equal(y3, y2), "graph replay must equal the eager run"
    vb.check_device()
    m.free()


@pytest.fixture(scope="module")
def c2_graph():
    from varda_b200 import synth
    pos, e, attr = synth.graph_c2()
    H = len(pos)
    rp, src, _, at = vb.build_csr(e.T, attr, H, H)
    at16 = at.astype(np.float16).astype(np.float32)  # fp16 mode: attributes rounded as autocast does
    return H, rp, src, at16


def test_c2_attention_parity(c2_graph):
    H, rp, src, at = c2_graph
    C, heads = 1024, 16
    hd = C // heads
    assert rp[-1] == 2_561_682 and H == 189_809
    rng = np.random.default_rng(22)
    qkvs = rng.standard_normal((H, 4 * C), dtype=np.float32).astype(np.float16)
    we = (rng.standard_normal((C, 3)) / np.sqrt(3)).astype(np.float16).astype(np.float32)
    be = (rng.standard_normal(C) * 0.1).astype(np.float16).astype(np.float32)
    w4 = np.zeros((4, C), np.float32)
    w4[:3], w4[3] = we.T, be
    edges = vb.pack_edges(src, at, round_fp16=True)
    d = torch.from_numpy(qkvs).cuda()
    ld = 4 * C
    q, k, v, xr = d[:, :C], d[:, C:], d[:, 2 * C:], d[:, 3 * C:]
    d_rp = torch.from_numpy(rp).cuda()
    d_ed = torch.from_numpy(edges).cuda()
    d_w = torch.from_numpy(w4).cuda()
    outs = {}
    for path in ("tc", "gather", "tiled", "split"):
        o = torch.full((H, C), float("nan"), device="cuda", dtype=torch.float16)
        if path == "tc":
            tiles = vb.Tiles(rp, src, at, H, hd, kind=vb.Tiles.TC)
            tiles.attention(0, H, q, ld, k, v, ld, xr, ld, o, C, d_w, C, heads, hd)
        elif path == "gather":
            vb.attention(vb.FP16, d_rp, d_ed, 0, H, q, ld, k, v, ld, xr, ld, o, C, d_w, C, heads, hd)
        elif path == "tiled":
            tiles = vb.Tiles(rp, src, at, H, hd)
            tiles.attention(0, H, q, ld, k, v, ld, xr, ld, o, C, d_w, C, heads, hd)
        else:
            vb.attention_split_noalloc(vb.FP16, d_rp, d_ed, 0, H, q, ld, k, v, ld, xr, ld, o, C, d_w, C, heads, hd,
                                       splits=4)
        torch.cuda.synchronize()
        outs[path] = o
    vb.check_device()
    # the oracle on 16 runs of 256 consecutive rows
    starts = np.sort(rng.choice(H - 256, 16, replace=False))
    starts[0], starts[-1] = 0, H - 256
    qf = qkvs[:, :C].astype(np.float32)
    kf = np.ascontiguousarray(qkvs[:, C:2 * C].astype(np.float32))
    vf = np.ascontiguousarray(qkvs[:, 2 * C:3 * C].astype(np.float32))
    xf = qkvs[:, 3 * C:].astype(np.float32)
    for s0 in starts:
        ref = oracle.graph_attention((rp, src, None, at), int(s0), 256, qf[s0:s0 + 256], kf, vf,
                                     np.ascontiguousarray(we.T), be, heads, hd) + xf[s0:s0 + 256]
        for path, o in outs.items():
            got = o[s0:s0 + 256].float().cpu().numpy()
            e = oracle.rel_absmax(got, ref)
            assert e <= TOL[vb.FP16], f"{path} rows [{s0}, {s0 + 256}): rel_absmax {e:.3e}"
    zero = np.where(rp[1:] == rp[:-1])[0]
    assert len(zero) == 0  # the C2 graph has in-degree 11..54
    base = outs["gather"].float()
    for path in ("tc", "tiled", "split"):
        e = ((outs[path].float() - base).abs().max() / base.abs().max()).item()
        assert e <= TOL[vb.FP16], f"{path} vs gather on every row: {e:.3e}"


def test_c1_full_out_y_against_reference(tmp_path):
    g = np.load(os.path.join(GOLDEN, "c1.y_sample.npz"))
    from varda_b200 import synth
    mp, xp = synth.generate("c1", str(tmp_path))
    assert synth.sha256_file(mp) == bytes(g["__model_sha256__"]).decode(), "c1 model drifted from the golden's"
    assert synth.sha256_file(xp) == bytes(g["__input_sha256__"]).decode(), "c1 input drifted from the golden's"
    x = np.array(st.read(xp)[0]["in.x"])
    m = vb.Model.load(mp, precision=vb.FP16)
    assert (m.T_out, m.G, m.V_out) == tuple(g["shape"][[1, 3, 4]])
    y = m.predict_step(x)
    got = y[0, :, 0][:, g["rows"]]
    e = oracle.rel_absmax(got, g["y"])
    assert e <= TOL[vb.FP16], f"out.y at {len(g['rows'])} rows: rel_absmax {e:.3e}"
    y2 = m.predict_step(x)
    y3 = m.predict_step(x)
    assert np.array_equal(y2, y) and np.array_equal(y3, y), "graph replay == eager, repeat calls identical"
    vb.check_device()
    m.free()
