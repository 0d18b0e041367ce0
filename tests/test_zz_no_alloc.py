"""The no-allocation attention entry point (vb_attention_split_noalloc) against the existing one
(vb_attention), through the C ABI, on the B200. Named to be collected last, so it also runs after every
other test in the session has used the device; it passes alone as well.

Two calls in a row on the same inputs (the second reuses the static scratch the first wrote) must both
match vb_attention: within 1e-5 rel_absmax in fp32 (the summation order differs), and in fp16 within
the fp16 bar with nearly every element bitwise equal (only outputs near an fp16 rounding boundary may
differ by one unit). In fp32 the output is also checked against the CPU oracle's restatement of the
reference's graph attention, plus x_r. The device's free memory is the same before and after the
second call (the entry point allocates nothing). Cases cover every degree class incl. zero in-degree,
a destination sub-range, several split counts, and a graph large enough to need several scratch-sized
batches.
"""
import numpy as np
import pytest

import oracle
import varda_b200 as vb

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")

DEGREES = [0, 1, 2, 3, 5, 8, 17, 33, 64, 300]


def dev(a, dtype):
    return torch.from_numpy(np.ascontiguousarray(a)).to(device="cuda", dtype=dtype)


def rounded(a, dt):
    return a.astype(np.float32) if dt == vb.FP32 else a.astype(np.float16).astype(np.float32)


def setup(rng, C, heads, A, n_src, n_dst, dt):
    s, d = [], []
    for i in range(n_dst):
        deg = DEGREES[i] if i < len(DEGREES) else DEGREES[int(rng.integers(len(DEGREES) - 1))]
        s += list(rng.integers(0, n_src, deg))
        d += [i] * deg
    perm = rng.permutation(len(s))
    ei = np.stack([np.array(s, np.int64)[perm], np.array(d, np.int64)[perm]])
    ea = rng.normal(size=(ei.shape[1], A)).astype(np.float32)
    rp, src, _, attr = vb.build_csr(ei, ea, n_src, n_dst)
    attr = rounded(attr, dt)
    ld = C + 8
    T = torch.float32 if dt == vb.FP32 else torch.float16
    q, k, v, xr = (dev(rounded(rng.normal(size=(n, ld)), dt), T) for n in (n_dst, n_src, n_src, n_dst))
    w4 = np.zeros((4, C), np.float32)
    w4[:A] = rounded(rng.normal(size=(C, A)) * 0.5, dt).T
    w4[3] = rounded(rng.normal(size=C) * 0.5, dt)
    edges = vb.pack_edges(src, attr, round_fp16=False)
    return dict(rp=dev(rp, torch.int32), ed=dev(edges, torch.float32), w=dev(w4, torch.float32), q=q, k=k, v=v,
                xr=xr, ld=ld, T=T, rp_host=rp, csr=(rp, src, None, attr), w4=w4, A=A)


def run_both(g, dt, C, heads, lo, n, splits):
    hd = C // heads
    ref = torch.full((n, C), float("nan"), device="cuda", dtype=g["T"])
    vb.attention(dt, g["rp"], g["ed"], lo, n, g["q"][lo:], g["ld"], g["k"], g["v"], g["ld"], g["xr"][lo:], g["ld"],
                 ref, C, g["w"], C, heads, hd)
    outs = []
    for i in range(2):  # two calls in a row: the second reuses the scratch the first wrote
        o = torch.full((n, C), float("nan"), device="cuda", dtype=g["T"])
        torch.cuda.synchronize()
        free0 = torch.cuda.mem_get_info()[0]
        vb.attention_split_noalloc(dt, g["rp"], g["ed"], lo, n, g["q"][lo:], g["ld"], g["k"], g["v"], g["ld"],
                                   g["xr"][lo:], g["ld"], o, C, g["w"], C, heads, hd, splits)
        torch.cuda.synchronize()
        if i == 1:  # the first call on a device may load the module; the second must take no memory
            assert torch.cuda.mem_get_info()[0] == free0, "the no-allocation entry point took device memory"
        outs.append(o)
    return ref.float().cpu().numpy(), [o.float().cpu().numpy() for o in outs]


def check(ref, outs, dt, g, lo, n):
    assert not np.isnan(ref).any()
    for got in outs:
        assert not np.isnan(got).any()
        if dt == vb.FP32:
            assert oracle.rel_absmax(got, ref) <= 1e-5
        else:
            assert oracle.rel_absmax(got, ref) <= 3e-3
            assert np.mean(got != ref) < 0.02, "fp16: all but a few boundary cases bitwise equal"
        rp = g["rp_host"][lo:lo + n + 1]
        zero = np.where(rp[1:] == rp[:-1])[0]
        xr = g["xr"][lo:lo + n].float().cpu().numpy()[:, :got.shape[1]]
        assert np.array_equal(got[zero], xr[zero]), "zero in-degree gives x_r exactly"
    assert np.array_equal(outs[0], outs[1]), "repeat calls are deterministic"
    if dt == vb.FP32:  # the CPU oracle (the reference's graph attention restated), plus x_r
        C = outs[0].shape[1]
        heads = g["heads"]
        ld = g["ld"]
        q = g["q"].float().cpu().numpy()[:, :C]
        k = g["k"].float().cpu().numpy()[:, :C]
        v = g["v"].float().cpu().numpy()[:, :C]
        xr = g["xr"].float().cpu().numpy()[:, :C]
        we = np.ascontiguousarray(g["w4"][:g["A"]])
        o = oracle.graph_attention(g["csr"], lo, n, q[lo:lo + n], k, v, we, g["w4"][3], heads, C // heads)
        assert oracle.rel_absmax(outs[0], o + xr[lo:lo + n]) <= 1e-5, "against the CPU oracle"
        del ld


@pytest.mark.parametrize("dt", [vb.FP32, vb.FP16])
@pytest.mark.parametrize("C,heads,A,splits", [(1024, 16, 3, 1), (1024, 16, 3, 4), (256, 8, 3, 3), (512, 4, 2, 8),
                                              (128, 4, 3, 2), (384, 6, 3, 5), (2048, 8, 3, 4), (256, 32, 1, 64)])
def test_matches_existing_entry_point(C, heads, A, splits, dt):
    rng = np.random.default_rng(C + heads + splits + dt)
    g = setup(rng, C, heads, A, 131, 97, dt)
    g["heads"] = heads
    ref, outs = run_both(g, dt, C, heads, 0, 97, splits)
    check(ref, outs, dt, g, 0, 97)
    lo, n = 13, 51  # a destination sub-range, rows local
    ref, outs = run_both(g, dt, C, heads, lo, n, splits)
    check(ref, outs, dt, g, lo, n)


@pytest.mark.parametrize("dt", [vb.FP32, vb.FP16])
def test_many_batches(dt):
    """2,500 rows x 8 splits x (1024 + 80) floats: about six scratch-sized batches."""
    rng = np.random.default_rng(5 + dt)
    g = setup(rng, 1024, 16, 3, 700, 2500, dt)
    g["heads"] = 16
    ref, outs = run_both(g, dt, 1024, 16, 0, 2500, 8)
    check(ref, outs, dt, g, 0, 2500)


def test_rejects_what_does_not_fit():
    rp = torch.zeros(2, dtype=torch.int32, device="cuda")
    ed = torch.zeros(1, 4, dtype=torch.float32, device="cuda")
    C = 65536
    row = torch.zeros(1, C, dtype=torch.float32, device="cuda")  # one row of q, k, v, x_r, out
    w = torch.zeros(4, C, dtype=torch.float32, device="cuda")
    # one row: 64 splits x (65536 + 5 x 1024) floats > the 16 MiB scratch; rejected before any launch
    with pytest.raises(vb.VardaError, match="static scratch"):
        vb.attention_split_noalloc(vb.FP32, rp, ed, 0, 1, row, C, row, row, C, row, C, row, C, w, C, 1024, 64, 64)
    with pytest.raises(vb.VardaError, match="splits"):
        vb.attention_split_noalloc(vb.FP32, rp, ed, 0, 1, row, 256, row, row, 256, row, 256, row, 256, w, 256, 4, 64, 0)
    with pytest.raises(vb.VardaError, match="non-null"):
        vb.attention_split_noalloc(vb.FP32, rp, ed, 0, 1, None, 256, row, row, 256, row, 256, row, 256, w, 256, 4, 64, 2)
    with pytest.raises(vb.VardaError, match="at least C"):
        vb.attention_split_noalloc(vb.FP32, rp, ed, 0, 1, row, 128, row, row, 256, row, 256, row, 256, w, 256, 4, 64, 2)
    vb.check_device()
