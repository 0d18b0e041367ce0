"""Kernel parity on the B200, through the C ABI (device memory via torch as plumbing).

Attention follows the reference's own unit test (tests/test_cuda_kernels.cu:98-233 of varda.cpp): a
graph with every degree class {0,1,2,3,5,8,17,33,64} in shuffled stored order, the layouts
(C, heads, A) it uses plus this repo's C=128/384/2048, a float64 reference with the edge term
materialised and a two-pass softmax; tolerance 1e-5 (fp32) and 2e-3 (fp16) as there; zero in-degree
gives x_r exactly; a destination sub-range is bitwise equal to the full launch. GEMM and LayerNorm are
checked against float64 references of the same fp32 / autocast-fp16 arithmetic.
"""
import math

import numpy as np
import pytest

import oracle
import varda_b200 as vb

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")

DEGREES = [0, 1, 2, 3, 5, 8, 17, 33, 64]


def dev(a, dtype):
    t = torch.from_numpy(np.ascontiguousarray(a))
    return t.to(device="cuda", dtype=dtype)


def tname(dt):
    return torch.float32 if dt == vb.FP32 else torch.float16


def rounded(a, dt):
    return a.astype(np.float32) if dt == vb.FP32 else a.astype(np.float16).astype(np.float32)


def make_graph(rng, n_src, n_dst, A):
    s, d = [], []
    for i in range(n_dst):
        deg = DEGREES[i] if i < len(DEGREES) else DEGREES[int(rng.integers(len(DEGREES)))]
        s += list(rng.integers(0, n_src, deg))
        d += [i] * deg
    perm = rng.permutation(len(s))
    ei = np.stack([np.array(s, np.int64)[perm], np.array(d, np.int64)[perm]])
    ea = rng.normal(size=(ei.shape[1], A)).astype(np.float32)
    return ei, ea


def attention_reference(rp, src, attr, q, k, v, xr, we, be, heads, hd):
    """float64, e materialised and added to k and v, two-pass softmax (the reference test's maths)."""
    C = heads * hd
    nd = len(rp) - 1
    out = np.zeros((nd, C))
    for d in range(nd):
        b0, b1 = rp[d], rp[d + 1]
        if b1 == b0:
            out[d] = xr[d]
            continue
        e = attr[b0:b1].astype(np.float64) @ we.T.astype(np.float64) + be  # [deg, C]
        kk = k[src[b0:b1]] + e
        vv = v[src[b0:b1]] + e
        for h in range(heads):
            sl = slice(h * hd, (h + 1) * hd)
            sc = (kk[:, sl] @ q[d, sl]) / math.sqrt(hd)
            p = np.exp(sc - sc.max())
            p /= p.sum()
            out[d, sl] = p @ vv[:, sl] + xr[d, sl]
    return out


LAYOUTS = [(1024, 16, 3), (256, 8, 3), (512, 4, 2), (256, 32, 1), (768, 12, 3), (128, 4, 3), (384, 6, 3),
           (2048, 8, 3)]


@pytest.mark.parametrize("dt", [vb.FP32, vb.FP16])
@pytest.mark.parametrize("C,heads,A", LAYOUTS)
def test_attention(C, heads, A, dt):
    rng = np.random.default_rng(C * 7 + heads + A + dt)
    hd = C // heads
    n_src, n_dst, ld = 131, 97, C + 8
    ei, ea = make_graph(rng, n_src, n_dst, A)
    rp, src, _, attr = vb.build_csr(ei, ea, n_src, n_dst)
    attr = rounded(attr, dt)
    q, k, v, xr = (rounded(rng.normal(size=(n, ld)), dt) for n in (n_dst, n_src, n_src, n_dst))
    we = rounded(rng.normal(size=(C, A)) * 0.5, dt)
    be = rounded(rng.normal(size=C) * 0.5, dt)
    w4 = np.zeros((4, C), np.float32)
    w4[:A] = we.T
    w4[3] = be
    edges = vb.pack_edges(src, attr, round_fp16=False)
    T = tname(dt)
    d_rp, d_ed, d_w = dev(rp, torch.int32), dev(edges, torch.float32), dev(w4, torch.float32)
    d_q, d_k, d_v, d_x = dev(q, T), dev(k, T), dev(v, T), dev(xr, T)
    out = torch.full((n_dst, C), float("nan"), device="cuda", dtype=T)
    vb.attention(dt, d_rp, d_ed, 0, n_dst, d_q, ld, d_k, d_v, ld, d_x, ld, out, C, d_w, C, heads, hd)
    torch.cuda.synchronize()
    got = out.float().cpu().numpy()
    ref = attention_reference(rp, src, attr, q[:, :C].astype(np.float64), k[:, :C].astype(np.float64),
                              v[:, :C].astype(np.float64), xr[:, :C].astype(np.float64), we, be.astype(np.float64),
                              heads, hd)
    err = oracle.rel_absmax(got, ref)
    tol = 1e-5 if dt == vb.FP32 else 2e-3
    assert err <= tol, f"rel_absmax {err:.3e} > {tol}"
    zero = np.where(rp[1:] == rp[:-1])[0]
    assert len(zero) > 0
    assert np.array_equal(got[zero], xr[zero, :C]), "zero in-degree must give x_r exactly"
    if dt == vb.FP32:
        # the oracle's restatement of cpu::graph_attention, plus x_r
        o = oracle.graph_attention((rp, src, None, attr), 0, n_dst, q[:, :C], k[:, :C], v[:, :C],
                                   np.ascontiguousarray(we.T), be, heads, hd) + xr[:, :C]
        assert oracle.rel_absmax(got, o) <= 1e-5
    # destination sub-range [13, 64): rows local, bitwise equal to the full launch
    lo, n = 13, 51
    out2 = torch.empty((n, C), device="cuda", dtype=T)
    vb.attention(dt, d_rp, d_ed, lo, n, d_q[lo:], ld, d_k, d_v, ld, d_x[lo:], ld, out2, C, d_w, C, heads, hd)
    torch.cuda.synchronize()
    assert torch.equal(out2, out[lo:lo + n])


def gemm_reference(A, W, b, R, epi, gelu_tanh, fp16):
    acc = A.astype(np.float64) @ W.astype(np.float64).T
    rnd = (lambda x: x.astype(np.float16).astype(np.float64)) if fp16 else (lambda x: x)
    y = acc + (b.astype(np.float64) if b is not None else 0)
    y = rnd(y)
    if epi == 1:
        if gelu_tanh:
            y = 0.5 * y * (1 + np.tanh(math.sqrt(2 / math.pi) * (y + 0.044715 * y ** 3)))
        else:
            from scipy.special import erf
            y = 0.5 * y * (1 + erf(y / math.sqrt(2)))
        y = rnd(y)
    elif epi == 2:
        y = rnd(y + R.astype(np.float64))
    return y


GEMM_SHAPES = [(1, 8, 8, 8), (77, 67, 168, 168), (300, 1024, 1024, 1024), (1000, 4096, 1024, 1024),
               (513, 1024, 4096, 4096), (1031, 80, 1024, 1024), (4000, 2048, 184, 192), (2562, 128, 4, 8),
               (129, 256, 64, 64)]


@pytest.mark.parametrize("M,N,K,lda", GEMM_SHAPES)
@pytest.mark.parametrize("epi", [0, 1, 2])
@pytest.mark.parametrize("dt,engine", [(vb.FP32, 1), (vb.FP16, 1), (vb.FP16, 2)])
def test_gemm(M, N, K, lda, epi, dt, engine):
    rng = np.random.default_rng(M + N + K + epi)
    fp16 = dt == vb.FP16
    A = np.zeros((M, lda), np.float32)
    A[:, :K] = rounded(rng.normal(size=(M, K)), dt)
    ldw = lda
    W = np.zeros((N, ldw), np.float32)
    W[:, :K] = rounded(rng.normal(size=(N, K)) / math.sqrt(K), dt)
    b = rounded(rng.normal(size=N) * 0.2, dt)
    ldy = (N + 7) // 8 * 8  # 16-byte row strides, as the engine lays out its buffers
    R = np.zeros((M, ldy), np.float32)
    R[:, :N] = rounded(rng.normal(size=(M, N)), dt)
    T = tname(dt)
    dA, dW, db, dR = dev(A, T), dev(W, T), dev(b, T), dev(R, T)
    Y = torch.full((M, ldy), float("nan"), device="cuda", dtype=T)
    vb.gemm(dt, engine, dA, lda, dW, ldw, db, Y, ldy, dR if epi == 2 else None, ldy, M, N, K, epi,
            gelu_tanh=(N % 2 == 1))
    torch.cuda.synchronize()
    vb.check_device()
    got = Y.float().cpu().numpy()[:, :N]
    ref = gemm_reference(A[:, :K], W[:, :K], b, R[:, :N], epi, N % 2 == 1, fp16)
    err = oracle.rel_absmax(got, ref)
    tol = 1e-5 if dt == vb.FP32 else 2e-3
    assert err <= tol, f"rel_absmax {err:.3e}"


def test_gemm_tensor_core_matches_cuda_core():
    rng = np.random.default_rng(5)
    M, N, K = 3000, 4096, 1024
    A = dev(rng.normal(size=(M, K)), torch.float16)
    W = dev(rng.normal(size=(N, K)) / 32, torch.float16)
    b = dev(rng.normal(size=N), torch.float16)
    Y1 = torch.empty((M, N), device="cuda", dtype=torch.float16)
    Y2 = torch.empty_like(Y1)
    vb.gemm(vb.FP16, 1, A, K, W, K, b, Y1, N, None, N, M, N, K, 0)
    vb.gemm(vb.FP16, 2, A, K, W, K, b, Y2, N, None, N, M, N, K, 0)
    torch.cuda.synchronize()
    vb.check_device()
    d = (Y1.float() - Y2.float()).abs().max().item() / Y1.float().abs().max().item()
    assert d <= 2e-3
    # repeatability: the same launch twice is bitwise equal
    Y3 = torch.empty_like(Y1)
    vb.gemm(vb.FP16, 2, A, K, W, K, b, Y3, N, None, N, M, N, K, 0)
    torch.cuda.synchronize()
    assert torch.equal(Y2, Y3)


def seg_records_reference(y, segw):
    """float64 {mean, M2} of every run of segw columns of every row of y."""
    M, N = y.shape
    s = y.astype(np.float64).reshape(M, N // segw, segw)
    m = s.mean(2)
    return np.stack([m, ((s - m[..., None]) ** 2).sum(2)], -1)


@pytest.mark.parametrize("M,N,K,epi", [(1000, 1024, 1024, 2), (700, 384, 256, 0), (333, 128, 512, 2),
                                       (2000, 1024, 184, 0), (513, 2048, 1024, 2), (300, 256, 64, 0)])
def test_gemm_ln_records(M, N, K, epi):
    """LayerNorm records written by the GEMM epilogue (vb_gemm_ln st_out): the output is bitwise the
    plain GEMM's, each record is the float64 {mean, M2} of its fp16 segment within fp32 rounding (rows
    with a mean of several standard deviations), and row_seg_stats of the stored output gives the
    same bits (the engine uses it for rows no GEMM produced)."""
    rng = np.random.default_rng(M + N + K)
    A = dev(rng.normal(size=(M, K)), torch.float16)
    W = dev(rng.normal(size=(N, K)) / math.sqrt(K), torch.float16)
    b = dev(rng.normal(size=N) * 0.2 + 4.0, torch.float16)
    R = dev(rng.normal(size=(M, N)) + rng.normal(size=(M, 1)) * 3, torch.float16)
    segw = vb.ln_segment_width(N)
    assert segw == (64 if N <= 128 else 128)
    Y0 = torch.empty((M, N), device="cuda", dtype=torch.float16)
    Y1 = torch.full((M, N), float("nan"), device="cuda", dtype=torch.float16)
    st1 = torch.full((M, N // segw, 2), float("nan"), device="cuda", dtype=torch.float32)
    st2 = torch.full_like(st1, float("nan"))
    Rp = R if epi == 2 else None
    vb.gemm(vb.FP16, 2, A, K, W, K, b, Y0, N, Rp, N, M, N, K, epi)
    vb.gemm_ln(A, K, W, K, b, Y1, N, Rp, N, M, N, K, epi, st_out=st1)
    vb.row_seg_stats(Y1, N, M, N, segw, st2)
    torch.cuda.synchronize()
    vb.check_device()
    assert torch.equal(Y0, Y1), "writing the records must not change the output"
    assert torch.equal(st1, st2), "epilogue records and row_seg_stats must agree bitwise"
    got = st1.cpu().numpy().astype(np.float64)
    ref = seg_records_reference(Y1.float().cpu().numpy(), segw)
    scale = np.abs(ref[..., 0]).max() + np.sqrt(ref[..., 1].max() / segw)
    assert np.abs(got[..., 0] - ref[..., 0]).max() <= 1e-6 * scale
    assert np.all(np.abs(got[..., 1] - ref[..., 1]) <= 1e-4 * ref[..., 1] + 1e-6 * segw * scale ** 2)
    with pytest.raises(vb.VardaError):  # GELU epilogues write no records
        vb.gemm_ln(A, K, W, K, b, Y1, N, None, N, M, N, K, 1, st_out=st1)


@pytest.mark.parametrize("M,N,C,epi,shift", [(1000, 4096, 1024, 0, 0.0), (1000, 4096, 1024, 1, 3.0),
                                             (777, 2048, 384, 0, 8.0), (500, 80, 1024, 0, 1.0),
                                             (300, 512, 128, 1, 0.0), (1200, 1024, 2048, 0, 2.0)])
def test_gemm_ln_fold(M, N, C, epi, shift):
    """A LayerNorm folded into the Linear after it: vb_fold_layernorm on (W, b) with the LN's weight and
    bias, then vb_gemm_ln on the raw rows and their records (row_seg_stats): against float64
    LN(x) W^T + b (GELU: exact erf) at the fp16 tolerance, and against the unfused fp16 path (LN kernel,
    then the GEMM) at the same bar; rows whose mean is `shift` standard deviations off zero, where the
    fold's two terms cancel the most."""
    rng = np.random.default_rng(M + N + C)
    x = rounded(rng.normal(size=(M, C)) * 1.5 + shift * 1.5 * rng.uniform(0.5, 1.0, size=(M, 1)), vb.FP16)
    g = rng.uniform(0.5, 1.5, C).astype(np.float32)
    be = (rng.normal(size=C) * 0.3).astype(np.float32)
    W = rounded(rng.normal(size=(N, C)) / math.sqrt(C), vb.FP16)
    b = rounded(rng.normal(size=N) * 0.2, vb.FP16)
    segw = vb.ln_segment_width(C)
    dx, dg, dbe = dev(x, torch.float16), dev(g, torch.float32), dev(be, torch.float32)
    ldy = (N + 7) // 8 * 8
    # unfused: LN kernel then the GEMM
    t = torch.empty((M, C), device="cuda", dtype=torch.float16)
    Y0 = torch.zeros((M, ldy), device="cuda", dtype=torch.float16)
    vb.layernorm(vb.FP16, dx, C, dg, dbe, t, C, M, C, 1e-5)
    vb.gemm(vb.FP16, 2, t, C, dev(W, torch.float16), C, dev(b, torch.float16), Y0, ldy, None, ldy, M, N, C, epi)
    # folded
    Wf, bf = dev(W, torch.float16), dev(b, torch.float16)
    cs = torch.empty(N, device="cuda", dtype=torch.float32)
    st = torch.empty((M, C // segw, 2), device="cuda", dtype=torch.float32)
    vb.fold_layernorm(Wf, C, N, C, dg, dbe, bf, cs)
    vb.row_seg_stats(dx, C, M, C, segw, st)
    Y = torch.full((M, ldy), float("nan"), device="cuda", dtype=torch.float16)
    vb.gemm_ln(dx, C, Wf, C, bf, Y, ldy, None, 0, M, N, C, epi, st_in=st, colsum=cs, nseg_in=C // segw,
               segw_in=segw, eps=1e-5)
    torch.cuda.synchronize()
    vb.check_device()
    xd = x.astype(np.float64)
    m = xd.mean(1, keepdims=True)
    ln = (xd - m) / np.sqrt(((xd - m) ** 2).mean(1, keepdims=True) + 1e-5) * g + be
    ref = gemm_reference(ln, W, b, None, epi, False, True)
    got = Y.float().cpu().numpy()[:, :N]
    assert oracle.rel_absmax(got, ref) <= 2e-3
    assert oracle.rel_absmax(got, Y0.float().cpu().numpy()[:, :N]) <= 2e-3
    # the folded weights and sums
    Wg = (W.astype(np.float32) * g).astype(np.float16)  # fp32 product, rounded once to fp16
    assert np.array_equal(Wf.cpu().numpy(), Wg)
    assert np.allclose(cs.cpu().numpy(), Wg.astype(np.float64).sum(1), rtol=1e-5, atol=1e-5)
    bref = b.astype(np.float64) + W.astype(np.float64) @ be.astype(np.float64)
    assert np.allclose(bf.float().cpu().numpy(), bref, rtol=2e-3, atol=2e-3)


@pytest.mark.parametrize("dt", [vb.FP32, vb.FP16])
@pytest.mark.parametrize("C", [128, 256, 384, 768, 1024, 2048])
def test_layernorm(C, dt):
    rng = np.random.default_rng(C)
    rows = 333
    x = rounded(rng.normal(size=(rows, C)) * 3 + 1, dt)
    r = rounded(rng.normal(size=(rows, C)), dt)
    w = rng.uniform(0.5, 1.5, C).astype(np.float32)
    b = rng.normal(size=C).astype(np.float32)
    T = tname(dt)
    dx, dr, y, o1 = dev(x, T), dev(r, T), torch.empty((rows, C), device="cuda", dtype=T), \
        torch.empty((rows, C), device="cuda", dtype=T)
    vb.layernorm(dt, dx, C, dev(w, torch.float32), dev(b, torch.float32), y, C, rows, C, 1e-5)
    torch.cuda.synchronize()

    def ln(a):
        a = a.astype(np.float64)
        m = a.mean(1, keepdims=True)
        return (a - m) / np.sqrt(((a - m) ** 2).mean(1, keepdims=True) + 1e-5) * w + b

    tol = 1e-5 if dt == vb.FP32 else 2e-3
    assert oracle.rel_absmax(y.float().cpu().numpy(), ln(x)) <= tol
    vb.layernorm(dt, dx, C, dev(w, torch.float32), None, y, C, rows, C, 1e-5)
    torch.cuda.synchronize()
    assert oracle.rel_absmax(y.float().cpu().numpy(), ln(x) - b) <= tol
    vb.add_layernorm(dt, dx, dr, o1, dev(w, torch.float32), dev(b, torch.float32), y, C, rows, C, 1e-5)
    torch.cuda.synchronize()
    s = rounded(x + r, dt)
    assert np.array_equal(o1.float().cpu().numpy(), s), "residual sum must be the rounded fp32 sum"
    assert oracle.rel_absmax(y.float().cpu().numpy(), ln(s)) <= tol


@pytest.mark.parametrize("C,heads,A", [(1024, 16, 3), (256, 8, 3), (512, 4, 2), (256, 32, 1), (768, 12, 3),
                                       (2048, 8, 3)])
def test_attention_tiled(C, heads, A):
    """The shared-memory-staged fp16 attention (tiles + heavy rows on the gather kernel): same graphs
    and reference as test_attention, plus rows far wider than a tile (degree 300)."""
    rng = np.random.default_rng(C * 11 + heads + A)
    hd = C // heads
    n_src, n_dst, ld = 131, 97, C + 8
    ei, ea = make_graph(rng, n_src, n_dst, A)
    wide = np.stack([rng.integers(0, n_src, 300), np.full(300, 50)]).astype(np.int64)  # a heavy row
    ei = np.concatenate([ei, wide], 1)
    ea = np.concatenate([ea, rng.normal(size=(300, A)).astype(np.float32)])
    rp, src, _, attr = vb.build_csr(ei, ea, n_src, n_dst)
    attr = rounded(attr, vb.FP16)
    q, k, v, xr = (rounded(rng.normal(size=(n, ld)), vb.FP16) for n in (n_dst, n_src, n_src, n_dst))
    we = rounded(rng.normal(size=(C, A)) * 0.5, vb.FP16)
    be = rounded(rng.normal(size=C) * 0.5, vb.FP16)
    w4 = np.zeros((4, C), np.float32)
    w4[:A] = we.T
    w4[3] = be
    tiles = vb.Tiles(rp, src, attr, n_src, hd)
    T = torch.float16
    d_q, d_k, d_v, d_x = dev(q, T), dev(k, T), dev(v, T), dev(xr, T)
    out = torch.full((n_dst, C), float("nan"), device="cuda", dtype=T)
    tiles.attention(0, n_dst, d_q, ld, d_k, d_v, ld, d_x, ld, out, C, dev(w4, torch.float32), C, heads, hd)
    torch.cuda.synchronize()
    vb.check_device()
    got = out.float().cpu().numpy()
    ref = attention_reference(rp, src, attr, q[:, :C].astype(np.float64), k[:, :C].astype(np.float64),
                              v[:, :C].astype(np.float64), xr[:, :C].astype(np.float64), we, be.astype(np.float64),
                              heads, hd)
    err = oracle.rel_absmax(got, ref)
    assert err <= 2e-3, f"rel_absmax {err:.3e}"
    zero = np.where(rp[1:] == rp[:-1])[0]
    assert np.array_equal(got[zero], xr[zero, :C]), "zero in-degree must give x_r exactly"


def local_graph(rng, n, A, window=40, unique=False):
    """Destinations drawing their sources from a window around their own index, so runs of
    consecutive rows share sources (multi-row tiles); with unique=False sources may repeat within a
    row, with unique=True they do not (rows the tensor-core kernel tiles)."""
    s, d = [], []
    for i in range(n):
        deg = DEGREES[i % len(DEGREES)] if i < 3 * len(DEGREES) else int(rng.integers(0, 30))
        if unique:
            off = rng.choice(np.arange(-window, window + 1), min(deg, 2 * window + 1), replace=False)
            s += list(np.unique(np.clip(i + off, 0, n - 1)))
        else:
            s += list(np.clip(i + rng.integers(-window, window + 1, deg), 0, n - 1))
        d += [i] * (len(s) - len(d))
    perm = rng.permutation(len(s))
    ei = np.stack([np.array(s, np.int64)[perm], np.array(d, np.int64)[perm]])
    return ei, rng.normal(size=(ei.shape[1], A)).astype(np.float32)


@pytest.mark.parametrize("graph", ["random", "local", "unique"])
@pytest.mark.parametrize("C,heads,A", [(1024, 16, 3), (512, 8, 2), (256, 4, 3), (128, 2, 1), (2048, 32, 3)])
def test_attention_tc(C, heads, A, graph):
    """The tile-sparse tensor-core attention (vb_tiles_create_kind VB_TILES_TC: per 16-row block and
    head, q.k and the value sums as mma.sync products over the column blocks that hold edges; heavy rows
    on the gather kernel): the float64 reference within the reference unit test's fp16 bar (2e-3), the
    gather kernel within the same bar, zero in-degree rows give x_r exactly, a row range starting at a
    tile gives the same bits as the full launch, and a second launch gives the same bits. Graphs: every
    degree class with repeated sources (mostly heavy rows) plus a row of 300 edges, a local graph with
    repeats, and a local graph of distinct sources whose tiles fill 64 rows."""
    rng = np.random.default_rng(C * 13 + heads + A + len(graph))
    hd = C // heads
    if graph == "random":
        n_src, n_dst = 400, 97
        ei, ea = make_graph(rng, n_src, n_dst, A)
        wide = np.stack([rng.integers(0, n_src, 300), np.full(300, 50)]).astype(np.int64)
        ei = np.concatenate([ei, wide], 1)
        ea = np.concatenate([ea, rng.normal(size=(300, A)).astype(np.float32)])
    else:
        n_src = n_dst = 1500
        ei, ea = local_graph(rng, n_dst, A, unique=graph == "unique")
    ld = C + 8
    rp, src, _, attr = vb.build_csr(ei, ea, n_src, n_dst)
    attr = rounded(attr, vb.FP16)
    q, k, v, xr = (rounded(rng.normal(size=(n, ld)), vb.FP16) for n in (n_dst, n_src, n_src, n_dst))
    we = rounded(rng.normal(size=(C, A)) * 0.5, vb.FP16)
    be = rounded(rng.normal(size=C) * 0.5, vb.FP16)
    w4 = np.zeros((4, C), np.float32)
    w4[:A] = we.T
    w4[3] = be
    tiles = vb.Tiles(rp, src, attr, n_src, hd, kind=vb.Tiles.TC)
    plan = vb.tile_plan(rp, src, attr, n_src, vb.Tiles.TC)
    if graph == "unique":
        assert len(plan["heavy"]) == 0 and plan["tiles"][:, 1].mean() > 30
    T = torch.float16
    d_q, d_k, d_v, d_x, d_w = dev(q, T), dev(k, T), dev(v, T), dev(xr, T), dev(w4, torch.float32)
    out = torch.full((n_dst, C), float("nan"), device="cuda", dtype=T)
    tiles.attention(0, n_dst, d_q, ld, d_k, d_v, ld, d_x, ld, out, C, d_w, C, heads, hd)
    again = torch.full_like(out, float("nan"))
    tiles.attention(0, n_dst, d_q, ld, d_k, d_v, ld, d_x, ld, again, C, d_w, C, heads, hd)
    gat = torch.full((n_dst, C), float("nan"), device="cuda", dtype=T)
    edges = vb.pack_edges(src, attr, round_fp16=True)
    vb.attention(vb.FP16, dev(rp, torch.int32), dev(edges, torch.float32), 0, n_dst, d_q, ld, d_k, d_v, ld, d_x, ld,
                 gat, C, d_w, C, heads, hd)
    torch.cuda.synchronize()
    vb.check_device()
    got, g = out.float().cpu().numpy(), gat.float().cpu().numpy()
    ref = attention_reference(rp, src, attr, q[:, :C].astype(np.float64), k[:, :C].astype(np.float64),
                              v[:, :C].astype(np.float64), xr[:, :C].astype(np.float64), we, be.astype(np.float64),
                              heads, hd)
    assert not np.isnan(got).any()
    err = oracle.rel_absmax(got, ref)
    assert err <= 2e-3, f"rel_absmax {err:.3e}"
    assert oracle.rel_absmax(got, g) <= 2e-3
    assert torch.equal(out, again), "a second launch gives the same bits"
    zero = np.where(rp[1:] == rp[:-1])[0]
    assert len(zero) > 0
    assert np.array_equal(got[zero], xr[zero, :C]), "zero in-degree must give x_r exactly"
    # rows from the start of a middle tile to the end: the same bits as the full launch
    t = plan["tiles"]
    lo = int(t[len(t) // 2, 0]) if len(t) > 1 else 0
    n = n_dst - lo
    part = torch.full((n, C), float("nan"), device="cuda", dtype=T)
    tiles.attention(lo, n, d_q[lo:], ld, d_k, d_v, ld, d_x[lo:], ld, part, C, d_w, C, heads, hd)
    torch.cuda.synchronize()
    assert torch.equal(part, out[lo:]), "a row range gives the full launch's bits"


@pytest.mark.parametrize("variant", ["1", "2", "3", "4"])
@pytest.mark.parametrize("C,heads", [(1024, 16), (2048, 8), (1024, 32)])
def test_attention_variants(C, heads, variant, monkeypatch):
    """The gather kernel's alternative launch shapes (VB_ATT_VARIANT: 1 = 16 channels per lane at 2
    blocks per SM, 2 = 8 channels with two edges per pipeline stage at 3, 3 = 8 channels at 5, 4 = 4
    channels at 4) against the float64 reference with the fp16 bar, zero in-degree giving x_r exactly;
    variants that keep the default's summation order (2, 3) are bitwise equal to it. A shape whose
    head would need more than 32 lanes (4 channels per lane, head_dim 256) is rejected."""
    monkeypatch.setenv("VB_ATT_VARIANT", variant)
    dt, A = vb.FP16, 3
    rng = np.random.default_rng(C + heads + int(variant))
    hd = C // heads
    n_src, n_dst, ld = 131, 97, C + 8
    ei, ea = make_graph(rng, n_src, n_dst, A)
    rp, src, _, attr = vb.build_csr(ei, ea, n_src, n_dst)
    attr = rounded(attr, dt)
    q, k, v, xr = (rounded(rng.normal(size=(n, ld)), dt) for n in (n_dst, n_src, n_src, n_dst))
    we = rounded(rng.normal(size=(C, A)) * 0.5, dt)
    be = rounded(rng.normal(size=C) * 0.5, dt)
    w4 = np.zeros((4, C), np.float32)
    w4[:A] = we.T
    w4[3] = be
    edges = vb.pack_edges(src, attr, round_fp16=False)
    T = tname(dt)
    d_rp, d_ed, d_w = dev(rp, torch.int32), dev(edges, torch.float32), dev(w4, torch.float32)
    d_q, d_k, d_v, d_x = dev(q, T), dev(k, T), dev(v, T), dev(xr, T)
    out = torch.full((n_dst, C), float("nan"), device="cuda", dtype=T)
    if variant == "4" and hd // 4 > 32:
        with pytest.raises(vb.VardaError, match="power of two <= 32"):
            vb.attention(dt, d_rp, d_ed, 0, n_dst, d_q, ld, d_k, d_v, ld, d_x, ld, out, C, d_w, C, heads, hd)
        return
    vb.attention(dt, d_rp, d_ed, 0, n_dst, d_q, ld, d_k, d_v, ld, d_x, ld, out, C, d_w, C, heads, hd)
    monkeypatch.setenv("VB_ATT_VARIANT", "0")
    dflt = torch.full((n_dst, C), float("nan"), device="cuda", dtype=T)
    vb.attention(dt, d_rp, d_ed, 0, n_dst, d_q, ld, d_k, d_v, ld, d_x, ld, dflt, C, d_w, C, heads, hd)
    torch.cuda.synchronize()
    vb.check_device()
    got = out.float().cpu().numpy()
    ref = attention_reference(rp, src, attr, q[:, :C].astype(np.float64), k[:, :C].astype(np.float64),
                              v[:, :C].astype(np.float64), xr[:, :C].astype(np.float64), we, be.astype(np.float64),
                              heads, hd)
    assert oracle.rel_absmax(got, ref) <= 2e-3
    zero = np.where(rp[1:] == rp[:-1])[0]
    assert np.array_equal(got[zero], xr[zero, :C])
    if variant in ("2", "3"):
        assert torch.equal(out, dflt), "same summation order as the default shape: bitwise equal"


@pytest.mark.parametrize("M,N,K,lda", [(300, 1024, 1024, 1024), (1000, 4096, 1024, 1024), (513, 1024, 4096, 4096),
                                       (4000, 2048, 184, 192), (256, 256, 64, 64), (777, 512, 320, 320)])
@pytest.mark.parametrize("epi", [0, 1, 2])
def test_gemm_cta_pair(M, N, K, lda, epi, monkeypatch):
    """The tensor-core GEMM on CTA pairs (VB_GEMM_PAIR=1: tcgen05.mma.cta_group::2, 256-row tiles over
    two SMs, each CTA loading its 128 rows of A and half of W): the float64 reference of the fp16
    arithmetic within the fp16 bar, and the single-CTA kernel's result within one fp16 rounding."""
    rng = np.random.default_rng(M + N + K + epi + 7)
    A = np.zeros((M, lda), np.float32)
    A[:, :K] = rounded(rng.normal(size=(M, K)), vb.FP16)
    W = np.zeros((N, lda), np.float32)
    W[:, :K] = rounded(rng.normal(size=(N, K)) / math.sqrt(K), vb.FP16)
    b = rounded(rng.normal(size=N) * 0.2, vb.FP16)
    R = rounded(rng.normal(size=(M, N)), vb.FP16)
    T = torch.float16
    dA, dW, db, dR = dev(A, T), dev(W, T), dev(b, T), dev(R, T)
    outs = []
    for pair in ("1", "0"):
        monkeypatch.setenv("VB_GEMM_PAIR", pair)
        Y = torch.full((M, N), float("nan"), device="cuda", dtype=T)
        vb.gemm(vb.FP16, 2, dA, lda, dW, lda, db, Y, N, dR if epi == 2 else None, N, M, N, K, epi)
        torch.cuda.synchronize()
        vb.check_device()
        outs.append(Y.float().cpu().numpy())
    ref = gemm_reference(A[:, :K], W[:, :K], b, R, epi, False, True)
    assert not np.isnan(outs[0]).any()
    assert oracle.rel_absmax(outs[0], ref) <= 2e-3
    assert oracle.rel_absmax(outs[0], outs[1]) <= 2e-3


@pytest.mark.parametrize("M,N,K,epi", [(20000, 1024, 256, 2), (9000, 4096, 128, 1), (300, 2048, 512, 0),
                                       (70000, 256, 64, 0), (5000, 128, 192, 2)])
@pytest.mark.parametrize("pair", ["1", "0"])
def test_gemm_tile_order_bitwise(M, N, K, epi, pair, monkeypatch):
    """Dynamic tile order (each CTA or CTA pair takes its next tile from a counter; through vb_gemm with
    VB_GEMM_SCHED=1, a counter per stream) against the static order (vb_gemm's default): the same tiles
    with the same k order, so bitwise equal; repeated launches (the counter is zeroed by each launch's
    last CTA) and launches interleaved on two streams (a counter each) too."""
    rng = np.random.default_rng(M + N + K + epi)
    T = torch.float16
    A = dev(rounded(rng.normal(size=(M, K)), vb.FP16), T)
    W = dev(rounded(rng.normal(size=(N, K)) / math.sqrt(K), vb.FP16), T)
    b = dev(rounded(rng.normal(size=N) * 0.2, vb.FP16), T)
    R = dev(rounded(rng.normal(size=(M, N)), vb.FP16), T) if epi == 2 else None
    monkeypatch.setenv("VB_GEMM_PAIR", pair)

    def run(stream=None):
        Y = torch.full((M, N), float("nan"), device="cuda", dtype=T)
        kw = {}
        if stream is not None:
            stream.wait_stream(torch.cuda.current_stream())  # the fill above is on the current stream
            kw = {"stream": stream.cuda_stream}
        vb.gemm(vb.FP16, 2, A, K, W, K, b, Y, N, R, N, M, N, K, epi, **kw)
        return Y

    monkeypatch.setenv("VB_GEMM_SCHED", "0")
    ref = run()
    torch.cuda.synchronize()
    vb.check_device()
    assert not torch.isnan(ref.float()).any()
    monkeypatch.setenv("VB_GEMM_SCHED", "1")
    outs = [run() for _ in range(3)]
    s1, s2 = torch.cuda.Stream(), torch.cuda.Stream()
    for _ in range(2):
        outs.append(run(s1))
        outs.append(run(s2))
    torch.cuda.synchronize()
    vb.check_device()
    for o in outs:
        assert torch.equal(o, ref)


@pytest.mark.parametrize("dt", [vb.FP32, vb.FP16])
@pytest.mark.parametrize("C,heads", [(128, 4), (1024, 16)])
def test_attention_row_list_bitwise(C, heads, dt):
    """The gather attention over an explicit row list (the engine's interior / boundary split) is bitwise
    the range launch on those rows."""
    rng = np.random.default_rng(C + dt)
    hd, A = C // heads, 3
    n_src, n_dst, ld = 131, 97, C + 8
    ei, ea = make_graph(rng, n_src, n_dst, A)
    rp, src, _, attr = vb.build_csr(ei, ea, n_src, n_dst)
    attr = rounded(attr, dt)
    q, k, v, xr = (rounded(rng.normal(size=(n, ld)), dt) for n in (n_dst, n_src, n_src, n_dst))
    w4 = np.zeros((4, C), np.float32)
    w4[:A] = rounded(rng.normal(size=(C, A)) * 0.5, dt).T
    edges = vb.pack_edges(src, attr, round_fp16=False)
    T = tname(dt)
    d_rp, d_ed, d_w = dev(rp, torch.int32), dev(edges, torch.float32), dev(w4, torch.float32)
    d_q, d_k, d_v, d_x = dev(q, T), dev(k, T), dev(v, T), dev(xr, T)
    ref = torch.full((n_dst, C), float("nan"), device="cuda", dtype=T)
    vb.attention(dt, d_rp, d_ed, 0, n_dst, d_q, ld, d_k, d_v, ld, d_x, ld, ref, C, d_w, C, heads, hd)
    rows = rng.permutation(n_dst).astype(np.int32)
    got = torch.full((n_dst, C), float("nan"), device="cuda", dtype=T)
    for part in (rows[:40], rows[40:]):
        vb.attention_rows(dt, d_rp, d_ed, dev(np.sort(part), torch.int32), len(part), d_q, ld, d_k, d_v, ld, d_x, ld,
                          got, C, d_w, C, heads, hd)
    torch.cuda.synchronize()
    assert torch.equal(got, ref)
