"""Destination tiles of the shared-memory (CUDA-core) and tensor-core attention kernels, on the host
(vb_tile_plan, no GPU): the properties the kernels rely on.

* The tiles and the heavy rows partition the destination rows, in increasing order.
* A tile stays within its kernel's limits: rows, distinct sources, edges.
* A tile's sources are distinct and increasing, and every tiled edge's slot names its own source.
* A heavy row has more distinct sources or more edges than a tile holds. Its records keep their
  sources and their stored order.
* Attributes are rounded to fp16.
* Tiled rows keep their records in stored order.
* Tensor-core tiles: slots number a tile's sources by the first, then the last 16-row block of the tile
  that reads them, then by first appearance along its edges (padded with the last source to a
  multiple of 4), so the plan does not depend on how the source
  nodes are numbered; a row with a repeated source is heavy; tiles restart at multiples of 64 rows.
"""
import numpy as np
import pytest

import varda_b200 as vb

LIMITS = {vb.Tiles.SMEM: dict(rows=64, src=80, edges=1024), vb.Tiles.TC: dict(rows=64, src=128, edges=1024)}
DEGREES = [0, 1, 2, 3, 5, 8, 17, 33, 64]


def random_graph(rng, n_src, n_dst, A, heavy=True):
    s, d = [], []
    for i in range(n_dst):
        deg = DEGREES[i % len(DEGREES)] if i < 3 * len(DEGREES) else int(rng.integers(0, 40))
        s += list(rng.integers(0, n_src, deg))
        d += [i] * deg
    if heavy:  # one row over more distinct sources than any tile holds, one over more edges
        s += list(rng.permutation(n_src)[:150]) + list(rng.integers(0, 10, 1100))
        d += [n_dst // 2] * 150 + [n_dst // 3] * 1100
    ei = np.stack([np.array(s, np.int64), np.array(d, np.int64)])
    perm = rng.permutation(ei.shape[1])
    return ei[:, perm], rng.normal(size=(ei.shape[1], A)).astype(np.float32)


def local_graph(rng, n, A, window=40):
    s, d = [], []
    for i in range(n):
        deg = int(rng.integers(0, 30))
        s += list(np.clip(i + rng.integers(-window, window + 1, deg), 0, n - 1))
        d += [i] * deg
    ei = np.stack([np.array(s, np.int64), np.array(d, np.int64)])
    perm = rng.permutation(ei.shape[1])
    return ei[:, perm], rng.normal(size=(ei.shape[1], A)).astype(np.float32)


def f16(a):
    return a.astype(np.float16).astype(np.float32)


def unique_local_graph(rng, n, A, window=40):
    """Like local_graph with distinct sources per row (the tensor-core kernel's tiled rows)."""
    s, d = [], []
    for i in range(n):
        deg = int(rng.integers(0, 30))
        s += list(np.clip(i + rng.choice(np.arange(-window, window + 1), deg, replace=False), 0, n - 1))
        d += [i] * deg
    ei = np.unique(np.stack([np.array(s, np.int64), np.array(d, np.int64)], 1), axis=0).T
    perm = rng.permutation(ei.shape[1])
    return ei[:, perm], rng.normal(size=(ei.shape[1], A)).astype(np.float32)


def make(graph, rng, A):
    if graph == "random":
        n_src, n_dst = 300, 400
        ei, ea = random_graph(rng, n_src, n_dst, A)
    elif graph == "local":
        n_src = n_dst = 3000
        ei, ea = local_graph(rng, n_dst, A)
    else:
        n_src = n_dst = 3000
        ei, ea = unique_local_graph(rng, n_dst, A)
    return n_src, n_dst, ei, ea


@pytest.mark.parametrize("kind", [vb.Tiles.SMEM, vb.Tiles.TC])
@pytest.mark.parametrize("graph", ["random", "local", "unique"])
def test_tile_plan_properties(kind, graph):
    rng = np.random.default_rng(7 + kind + len(graph))
    A = 3
    n_src, n_dst, ei, ea = make(graph, rng, A)
    rp, src, _, attr = vb.build_csr(ei, ea, n_src, n_dst)
    plan = vb.tile_plan(rp, src, attr, n_src, kind)
    tiles, srcs, heavy, edges = plan["tiles"], plan["srcs"], plan["heavy"], plan["edges"]
    lim = LIMITS[kind]
    slot_or_src = edges[:, 3].view(np.int32)
    if kind == vb.Tiles.SMEM:  # records in stored order, attributes rounded to fp16
        np.testing.assert_array_equal(edges[:, :3], f16(attr))

    covered = np.zeros(n_dst, np.int32)
    tiled_rows = set()
    for r0, nr, s0, ns in tiles:
        assert 1 <= nr <= lim["rows"] and ns <= lim["src"]
        assert rp[r0 + nr] - rp[r0] <= lim["edges"]
        ts = srcs[s0:s0 + ns]
        if kind == vb.Tiles.TC:
            assert len(np.unique(ts)) == ns, "a tile's sources are distinct"
            first = list(dict.fromkeys(src[rp[r0]:rp[r0 + nr]].tolist()))
            fb, lb = {}, {}
            for i in range(nr):
                for s_ in src[rp[r0 + i]:rp[r0 + i + 1]].tolist():
                    fb.setdefault(s_, i // 16)
                    lb[s_] = i // 16
            want_order = sorted(first, key=lambda s_: (fb[s_], lb[s_]))  # stable: first appearance breaks ties
            assert ts.tolist() == want_order, "slots by first block, last block, first appearance"
            pad = srcs[s0 + ns:s0 + ((ns + 3) // 4) * 4]
            assert ns == 0 or np.all(pad == ts[-1]), "padded with the last source to a multiple of 4"
            assert r0 // 64 == (r0 + nr - 1) // 64, "tiles restart at multiples of 64 rows"
        else:
            assert np.all(np.diff(ts) > 0), "a tile's sources are distinct and increasing"
        for r in range(r0, r0 + nr):
            covered[r] += 1
            tiled_rows.add(r)
            b, e = rp[r], rp[r + 1]
            slots = slot_or_src[b:e]
            assert np.all((slots >= 0) & (slots < ns))
            got = sorted(zip(ts[slots].tolist(), map(tuple, edges[b:e, :3].tolist())))
            want = sorted(zip(src[b:e].tolist(), map(tuple, f16(attr[b:e]).tolist())))
            assert got == want, "every tiled edge's slot names its own source (with its attributes)"
            np.testing.assert_array_equal(ts[slots], src[b:e])  # stored order kept
            np.testing.assert_array_equal(edges[b:e, :3], f16(attr[b:e]))
    for r in heavy:
        covered[r] += 1
        b, e = rp[r], rp[r + 1]
        np.testing.assert_array_equal(edges[b:e, :3], f16(attr[b:e]))
        distinct = len(np.unique(src[b:e]))
        fits = distinct <= lim["src"] and e - b <= lim["edges"]
        if kind == vb.Tiles.TC:
            fits = fits and distinct == e - b
        assert not fits, "heavy only when it cannot fit a tile"
        np.testing.assert_array_equal(slot_or_src[b:e], src[b:e])
    assert np.all(covered == 1), "tiles and heavy rows partition the destinations"
    starts = sorted([int(t[0]) for t in tiles] + [int(h) for h in heavy])
    assert starts == sorted(starts) and len(set(starts)) == len(starts)
    assert np.all(np.diff(tiles[:, 0]) > 0), "tiles in row order"
    if graph != "random":
        assert tiles[:, 1].mean() > 8 or kind == vb.Tiles.TC and graph == "local", "multi-row tiles"
    if kind == vb.Tiles.TC and graph == "unique":
        assert len(heavy) == 0 and tiles[:, 1].mean() > 8


def test_tc_plan_independent_of_node_numbering():
    """Renumbering the source nodes (as a destination split over GPUs does with its local ids) leaves
    the tensor-core tiles, their slots and the heavy rows unchanged: the bits of the kernel's sums do
    not depend on the split."""
    rng = np.random.default_rng(5)
    n_src, n_dst, ei, ea = make("unique", rng, 3)
    rp, src, _, attr = vb.build_csr(ei, ea, n_src, n_dst)
    a = vb.tile_plan(rp, src, attr, n_src, vb.Tiles.TC)
    perm = rng.permutation(n_src).astype(np.int32)
    b = vb.tile_plan(rp, perm[src], attr, n_src, vb.Tiles.TC)
    np.testing.assert_array_equal(a["tiles"], b["tiles"])
    np.testing.assert_array_equal(a["heavy"], b["heavy"])
    np.testing.assert_array_equal(a["edges"], b["edges"])
    np.testing.assert_array_equal(perm[a["srcs"]], b["srcs"])


def test_tile_plan_rejects_unknown_kind():
    rp = np.array([0, 1], np.int32)
    with pytest.raises(vb.VardaError, match="tiles kind"):
        vb.tile_plan(rp, np.array([0], np.int32), np.zeros((1, 3), np.float32), 1, kind=7)
