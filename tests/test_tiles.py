"""Destination tiles of the shared-memory (CUDA-core) and tensor-core attention kernels, on the host
(vb_tile_plan, no GPU): the properties the kernels rely on.

* The tiles and the heavy rows partition the destination rows, in increasing order.
* A tile stays within its kernel's limits: rows, distinct sources, edges.
* A tile's sources are distinct and increasing, and every tiled edge's slot names its own source.
* A heavy row has more distinct sources or more edges than a tile holds. Its records keep their
  sources and their stored order.
* Attributes are rounded to fp16.
* Tiled rows keep their records in stored order for the shared-memory kernel. For the tensor-core
  kernel they are stably sorted by slot (duplicates adjacent, equal slots in stored order).
"""
import numpy as np
import pytest

import varda_b200 as vb

LIMITS = {vb.Tiles.SMEM: dict(rows=64, src=80, edges=1024), vb.Tiles.MMA: dict(rows=128, src=112, edges=1024)}
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


@pytest.mark.parametrize("kind", [vb.Tiles.SMEM, vb.Tiles.MMA])
@pytest.mark.parametrize("graph", ["random", "local"])
def test_tile_plan_properties(kind, graph):
    rng = np.random.default_rng(7 + kind + len(graph))
    A = 3
    if graph == "random":
        n_src, n_dst = 300, 400
        ei, ea = random_graph(rng, n_src, n_dst, A)
    else:
        n_src = n_dst = 3000
        ei, ea = local_graph(rng, n_dst, A)
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
            if kind == vb.Tiles.MMA:
                assert np.all(np.diff(slots) >= 0), "tensor-core tiles: records sorted by slot"
                # stable: records of one slot keep their stored order (here: same attribute sequence)
                for sl in np.unique(slots):
                    rows_at = np.where(slots == sl)[0]
                    stored = [i for i in range(b, e) if src[i] == ts[sl]]
                    np.testing.assert_array_equal(edges[b + rows_at, :3], f16(attr[stored]))
            else:
                np.testing.assert_array_equal(ts[slots], src[b:e])  # stored order kept
    for r in heavy:
        covered[r] += 1
        b, e = rp[r], rp[r + 1]
        np.testing.assert_array_equal(edges[b:e, :3], f16(attr[b:e]))
        assert len(np.unique(src[b:e])) > lim["src"] or e - b > lim["edges"], "heavy only when it cannot fit a tile"
        np.testing.assert_array_equal(slot_or_src[b:e], src[b:e])
    assert np.all(covered == 1), "tiles and heavy rows partition the destinations"
    starts = sorted([int(t[0]) for t in tiles] + [int(h) for h in heavy])
    assert starts == sorted(starts) and len(set(starts)) == len(starts)
    assert np.all(np.diff(tiles[:, 0]) > 0), "tiles in row order"
    if graph == "local":
        assert tiles[:, 1].mean() > 8, "local graphs give multi-row tiles"


def test_tile_plan_rejects_unknown_kind():
    rp = np.array([0, 1], np.int32)
    with pytest.raises(vb.VardaError, match="tiles kind"):
        vb.tile_plan(rp, np.array([0], np.int32), np.zeros((1, 3), np.float32), 1, kind=7)
