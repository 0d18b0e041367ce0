"""Seeded synthetic GraphTransformer models in varda.cpp's converted-model format.

The reference runs real checkpoints; none are available here, so the benchmark and parity models are
built from a seed (numpy default_rng). The format is the reference's model-file contract: safetensors
with metadata {"varda_format": "1", "config": <format v3 JSON>} and the tensor names of its format
description (graph.{enc,proc,dec}.edge_index I64 [2, E], edge_attr F32 [E, A_e], nodes.*.attr,
norm.*, per block q/k/v/self/edge/proj/mlp1/mlp2 Linears and ln_* LayerNorms, enc.emb_src,
enc.emb_dst, dec.emb_dst, dec.out_norm, dec.out_proj).

Configurations (the benchmark's C0-C4):
  c0   icosphere refinement 5 data nodes (10,242) and refinement 4 hidden nodes (2,562); encoder:
       each hidden node receives from its 12 nearest data nodes; processor: bidirectional
       multi-scale icosphere edges of levels 0-4; decoder: each data node receives from its 3
       nearest hidden nodes. C=128, 4 heads, mlp 512, 2 processor blocks, T=2, V_in=10, V_out=8.
  c1   Varda-shaped: 1,688,650 data nodes on a stretched grid (a ~1 km lat-lon patch over
       43-50N, 3-14E plus a ~31 km Fibonacci lattice elsewhere) and 189,809 hidden nodes on a
       stretched icosphere (refinement 7 everywhere, refinement 8-9 in a cap around the patch).
       Encoder kNN-4 data->hidden, decoder kNN-3 hidden->data, multi-scale processor edges.
       C=1024, 16 heads, mlp 4096, 16 blocks, T=2, V_in=90, V_out=80, fp32 weights.
  c3   c1 as a temporal downscaler (interpolator kind, T_out=6).
  c1s  c1's architecture (C=1024, 16 heads, mlp 4096, 16 blocks, T=2, V_in=90, V_out=80) on 1/64 of
       its nodes (G=26,385, H=2,965 on Fibonacci lattices) with c1's per-node edge counts: encoder
       kNN-4, processor kNN-14, decoder kNN-3. The reference CPU backend runs it in seconds, so it is
       the parity model at the benchmark's widths and depth and the CPU baseline's sample.
  Small random-graph models (`test_*`) cover every degree class, absent biases, the three
       boundings, tanh/erf GELU, latent skip on/off and T_out>1 for the parity tests.

Node numbering follows a 3-D Morton (Z-order) curve of the unit-sphere positions, so nodes close in
index are close in space: the CSR rows of neighbouring destinations then share sources, which is what
lets the attention's gathers hit in L2, and contiguous index ranges are compact regions for the
multi-GPU partition. Edge attributes: great-circle length (normalised by the graph's longest edge)
and the 2-D unit direction from destination to source in the destination's east/north tangent plane.
"""
from __future__ import annotations

import argparse
import hashlib
import json
import math
import os

import numpy as np

from . import safetensors as st

# ------------------------------------------------------------------ sphere geometry


def latlon_to_xyz(lat_deg, lon_deg):
    la, lo = np.deg2rad(lat_deg), np.deg2rad(lon_deg)
    return np.stack([np.cos(la) * np.cos(lo), np.cos(la) * np.sin(lo), np.sin(la)], -1)


def xyz_to_latlon(v):
    lat = np.rad2deg(np.arcsin(np.clip(v[:, 2], -1, 1)))
    lon = np.rad2deg(np.arctan2(v[:, 1], v[:, 0]))
    return lat, lon


def morton_order(v):
    """Stable argsort of 3-D Morton codes (21 bits per axis) of unit vectors."""
    q = np.clip(((v + 1.0) * 0.5 * (1 << 21)).astype(np.int64), 0, (1 << 21) - 1).astype(np.uint64)

    def spread(x):
        x = x & np.uint64(0x1FFFFF)
        x = (x | (x << np.uint64(32))) & np.uint64(0x1F00000000FFFF)
        x = (x | (x << np.uint64(16))) & np.uint64(0x1F0000FF0000FF)
        x = (x | (x << np.uint64(8))) & np.uint64(0x100F00F00F00F00F)
        x = (x | (x << np.uint64(4))) & np.uint64(0x10C30C30C30C30C3)
        x = (x | (x << np.uint64(2))) & np.uint64(0x1249249249249249)
        return x

    code = spread(q[:, 0]) | (spread(q[:, 1]) << np.uint64(1)) | (spread(q[:, 2]) << np.uint64(2))
    return np.argsort(code, kind="stable")


def icosahedron():
    t = (1.0 + 5 ** 0.5) / 2.0
    v = np.array([[-1, t, 0], [1, t, 0], [-1, -t, 0], [1, -t, 0], [0, -1, t], [0, 1, t], [0, -1, -t],
                  [0, 1, -t], [t, 0, -1], [t, 0, 1], [-t, 0, -1], [-t, 0, 1]], np.float64)
    v /= np.linalg.norm(v, axis=1, keepdims=True)
    f = np.array([[0, 11, 5], [0, 5, 1], [0, 1, 7], [0, 7, 10], [0, 10, 11], [1, 5, 9], [5, 11, 4],
                  [11, 10, 2], [10, 7, 6], [7, 1, 8], [3, 9, 4], [3, 4, 2], [3, 2, 6], [3, 6, 8],
                  [3, 8, 9], [4, 9, 5], [2, 4, 11], [6, 2, 10], [8, 6, 7], [9, 8, 1]], np.int64)
    return v, f


def refine(verts, faces):
    """Splits every face into four through the (re-normalised) edge midpoints. New vertices are
    appended, so the vertices of coarser levels keep their indices."""
    e = np.concatenate([faces[:, [0, 1]], faces[:, [1, 2]], faces[:, [2, 0]]])
    lo, hi = np.minimum(e[:, 0], e[:, 1]), np.maximum(e[:, 0], e[:, 1])
    big = np.int64(len(verts) + 1)
    uniq, inv = np.unique(lo * big + hi, return_inverse=True)
    a, b = uniq // big, uniq % big
    mid = verts[a] + verts[b]
    mid /= np.linalg.norm(mid, axis=1, keepdims=True)
    ids = (len(verts) + np.arange(len(uniq), dtype=np.int64))[inv].reshape(3, -1).T
    m01, m12, m20 = ids[:, 0], ids[:, 1], ids[:, 2]
    v0, v1, v2 = faces[:, 0], faces[:, 1], faces[:, 2]
    nf = np.concatenate([np.stack([v0, m01, m20], 1), np.stack([v1, m12, m01], 1),
                         np.stack([v2, m20, m12], 1), np.stack([m01, m12, m20], 1)])
    return np.concatenate([verts, mid]), nf


def face_edges(faces):
    """Unique undirected edges (lo, hi) of a face list."""
    e = np.concatenate([faces[:, [0, 1]], faces[:, [1, 2]], faces[:, [2, 0]]])
    lo, hi = np.minimum(e[:, 0], e[:, 1]), np.maximum(e[:, 0], e[:, 1])
    k = np.unique(np.stack([lo, hi], 1), axis=0)
    return k


def icosphere_levels(level):
    """Vertices of the level-`level` icosphere and the face list of every level 0..level."""
    v, f = icosahedron()
    faces = [f]
    for _ in range(level):
        v, f = refine(v, f)
        faces.append(f)
    return v, faces


def edge_attributes(pos_src, pos_dst, src, dst):
    """[length / max length, east, north]: great-circle length and the unit direction from the
    destination to the source in the destination's tangent plane."""
    ps, pd = pos_src[src], pos_dst[dst]
    ang = np.arccos(np.clip(np.einsum("ij,ij->i", ps, pd), -1.0, 1.0))
    lat, lon = xyz_to_latlon(pd)
    la, lo = np.deg2rad(lat), np.deg2rad(lon)
    east = np.stack([-np.sin(lo), np.cos(lo), np.zeros_like(lo)], 1)
    north = np.stack([-np.sin(la) * np.cos(lo), -np.sin(la) * np.sin(lo), np.cos(la)], 1)
    d = ps - pd
    de, dn = np.einsum("ij,ij->i", d, east), np.einsum("ij,ij->i", d, north)
    nrm = np.sqrt(de * de + dn * dn)
    nrm[nrm == 0] = 1.0
    mx = ang.max() if ang.size else 1.0
    return np.stack([ang / (mx if mx > 0 else 1.0), de / nrm, dn / nrm], 1).astype(np.float32)


def node_attributes(pos):
    lat, lon = xyz_to_latlon(pos)
    la, lo = np.deg2rad(lat), np.deg2rad(lon)
    return np.stack([np.sin(la), np.cos(la), np.sin(lo), np.cos(lo)], 1).astype(np.float32)


def knn(tree_pos, query_pos, k):
    from scipy.spatial import cKDTree
    _, idx = cKDTree(tree_pos).query(query_pos, k=k, workers=-1)
    return np.asarray(idx, np.int64).reshape(len(query_pos), k)


def renumber(edges, perm_of):
    """Maps node ids through `perm_of` (old -> new)."""
    return perm_of[edges]


# ------------------------------------------------------------------ graphs


def graph_c0():
    """C0: icosphere refinement 5 (data) and 4 (hidden)."""
    v5, faces = icosphere_levels(5)
    data = v5
    hidden = v5[: 10 * 4 ** 4 + 2]
    proc = np.concatenate([face_edges(faces[l]) for l in range(5)])       # levels 0-4, undirected
    proc = np.concatenate([proc, proc[:, ::-1]])                          # bidirectional
    enc_src = knn(data, hidden, 12)                                        # [H, 12] data ids
    enc = np.stack([enc_src.ravel(), np.repeat(np.arange(len(hidden)), 12)], 1)
    dec_src = knn(hidden, data, 3)                                         # [G, 3] hidden ids
    dec = np.stack([dec_src.ravel(), np.repeat(np.arange(len(data)), 3)], 1)
    return data, hidden, enc, proc[:, [0, 1]], dec


def stretched_data_nodes(G, lat0=43.0, lat1=50.0, lon0=3.0, lon1=14.0, n_lat=1033, n_lon=1120):
    """A regular lat-lon patch (cell centres) plus a Fibonacci lattice outside it, G points."""
    la = lat0 + (np.arange(n_lat) + 0.5) * (lat1 - lat0) / n_lat
    lo = lon0 + (np.arange(n_lon) + 0.5) * (lon1 - lon0) / n_lon
    LA, LO = np.meshgrid(la, lo, indexing="ij")
    lam = latlon_to_xyz(LA.ravel(), LO.ravel())
    need = G - len(lam)
    assert need > 0
    n = int(need * 1.01) + 1000
    while True:
        i = np.arange(n) + 0.5
        z = 1 - 2 * i / n
        phi = i * math.pi * (3 - 5 ** 0.5)
        r = np.sqrt(1 - z * z)
        p = np.stack([r * np.cos(phi), r * np.sin(phi), z], 1)
        lat, lon = xyz_to_latlon(p)
        out = ~((lat >= lat0) & (lat <= lat1) & (lon >= lon0) & (lon <= lon1))
        if out.sum() >= need:
            glob = p[out][:need]
            break
        n = int(n * 1.01) + 100
    return np.concatenate([lam, glob])


def stretched_hidden(H, center=(46.5, 8.5), global_level=7, fine_levels=2, refine_deg=14.0):
    """Icosphere refinement `global_level` everywhere plus the vertices of finer refinements
    nearest to `center` (all levels nested), H vertices in total. Returns positions, the node id
    of each kept vertex, and the multi-scale edge list (both directions)."""
    v, faces = icosphere_levels(global_level)
    n_glob = len(v)
    c = latlon_to_xyz(np.array([center[0]]), np.array([center[1]]))[0]
    cos_ref = math.cos(math.radians(refine_deg))
    fine_faces = []
    f = faces[-1]
    for _ in range(fine_levels):
        cen = v[f].mean(1)
        cen /= np.linalg.norm(cen, axis=1, keepdims=True)
        f = f[cen @ c >= cos_ref]
        v, f = refine(v, f)
        fine_faces.append(f)
    extra = H - n_glob
    cand = np.arange(n_glob, len(v))
    order = np.argsort(-(v[cand] @ c), kind="stable")
    keep = np.concatenate([np.arange(n_glob), cand[order[:extra]]])
    assert len(keep) == H
    new_id = np.full(len(v), -1, np.int64)
    new_id[keep] = np.arange(H)
    und = [face_edges(fc) for fc in faces] + [face_edges(fc) for fc in fine_faces]
    und = np.concatenate(und)
    und = new_id[und]
    und = und[(und >= 0).all(1)]
    und = np.unique(und, axis=0)
    return v[keep], und


def _processor_edges(hidden, und, knn_extra):
    """The multi-scale edges `und` (undirected pairs) plus each node's knn_extra nearest hidden nodes,
    deduplicated, in both directions: (source, destination) rows."""
    H = len(hidden)
    nb = knn(hidden, hidden, knn_extra + 1)[:, 1:]
    kn = np.stack([nb.ravel(), np.repeat(np.arange(H), knn_extra)], 1)
    pairs = np.concatenate([und, kn])  # as (lo, hi): each undirected edge once, whichever list it came from
    und = np.unique(np.stack([pairs.min(1), pairs.max(1)], 1), axis=0)
    return np.concatenate([und, und[:, ::-1]])


def graph_c2(H=189_809, knn_extra=11, seed=2):
    """C2, the isolated processor block: c1's hidden nodes and processor graph alone (same node numbering
    as c1's hidden nodes, edges sorted by destination then source), with edge attributes uniform on
    [0, 1) from `seed` as the benchmark's config states. Returns (positions [H, 3], edges [E, 2] as
    (source, destination), attributes [E, 3] float32)."""
    hidden, und = stretched_hidden(H)
    proc = _processor_edges(hidden, und, knn_extra)
    ph = morton_order(hidden)
    inv_h = np.empty_like(ph)
    inv_h[ph] = np.arange(len(ph))
    proc = np.stack([inv_h[proc[:, 0]], inv_h[proc[:, 1]]], 1)
    proc = proc[np.lexsort((proc[:, 0], proc[:, 1]))]
    attr = np.random.default_rng(seed).uniform(0.0, 1.0, size=(len(proc), 3)).astype(np.float32)
    return hidden[ph], proc, attr


def graph_c1(G=1_688_650, H=189_809, knn_extra=11):
    """C1 graph (see module docstring). Processor edges: the multi-scale icosphere edges (one hop at
    every refinement level a node belongs to) plus each node's `knn_extra` nearest hidden nodes,
    deduplicated, in both directions."""
    data = stretched_data_nodes(G)
    hidden, und = stretched_hidden(H)
    proc = _processor_edges(hidden, und, knn_extra)
    enc_dst = knn(hidden, data, 4)                                         # data g -> its 4 nearest hidden
    enc = np.stack([np.repeat(np.arange(G), 4), enc_dst.ravel()], 1)
    dec_src = knn(hidden, data, 3)                                         # data g <- its 3 nearest hidden
    dec = np.stack([dec_src.ravel(), np.repeat(np.arange(G), 3)], 1)
    return data, hidden, enc, proc, dec


def random_graph(rng, n_src, n_dst, degrees, zero_every=7):
    """Random bipartite graph: destination d takes a degree from `degrees` (every class once among
    the first destinations), every `zero_every`-th destination none; shuffled stored order."""
    src, dst = [], []
    for d in range(n_dst):
        if zero_every and d % zero_every == zero_every - 4:
            continue
        k = degrees[d] if d < len(degrees) else degrees[int(rng.integers(len(degrees)))]
        src.append(rng.integers(0, n_src, k))
        dst.append(np.full(k, d))
    s, t = np.concatenate(src), np.concatenate(dst)
    perm = rng.permutation(len(s))
    return np.stack([s[perm], t[perm]], 1)


# ------------------------------------------------------------------ model assembly


def _sort_nodes(data, hidden, enc, proc, dec):
    """Renumbers data and hidden nodes along the Morton curve and sorts each edge list by
    (destination, source) so that the stored order is already destination-major."""
    pd, ph = morton_order(data), morton_order(hidden)
    inv_d = np.empty_like(pd); inv_d[pd] = np.arange(len(pd))
    inv_h = np.empty_like(ph); inv_h[ph] = np.arange(len(ph))
    enc = np.stack([inv_d[enc[:, 0]], inv_h[enc[:, 1]]], 1)
    proc = np.stack([inv_h[proc[:, 0]], inv_h[proc[:, 1]]], 1)
    dec = np.stack([inv_h[dec[:, 0]], inv_d[dec[:, 1]]], 1)

    def srt(e):
        return e[np.lexsort((e[:, 0], e[:, 1]))]

    return data[pd], hidden[ph], srt(enc), srt(proc), srt(dec)


def make_model(*, seed, C, heads, mlp, n_proc, T, Vd, Vi, Vo, norm_input, norm_output, res_in, res_out,
               bounding, data_pos=None, hidden_pos=None, enc=None, proc=None, dec=None, G=None, H=None,
               A=4, Ae=3, gelu="none", latent_skip=True, res_step=-1, absent=(), T_out=1, times=None,
               forcings=None, xavier=True, edge_attr="geometric", var_names=None, uuid=None,
               node_attr=None, weight_scale=1.0):
    """Returns (config dict, tensor dict, x) of a model in the reference format."""
    rng = np.random.default_rng(seed)
    t = {}
    if data_pos is not None:
        G, H = len(data_pos), len(hidden_pos)
    t["norm.mul"] = rng.uniform(0.5, 2.0, Vd).astype(np.float32)
    t["norm.add"] = rng.normal(0.0, 0.3, Vd).astype(np.float32)
    if node_attr is None:
        if data_pos is not None and A == 4:
            t["nodes.data.attr"] = node_attributes(data_pos)
            t["nodes.hidden.attr"] = node_attributes(hidden_pos)
        else:
            t["nodes.data.attr"] = rng.normal(0, 1, (G, A)).astype(np.float32)
            t["nodes.hidden.attr"] = rng.normal(0, 1, (H, A)).astype(np.float32)
    else:
        t["nodes.data.attr"], t["nodes.hidden.attr"] = node_attr
    for name, e, ps, pdst in (("enc", enc, data_pos, hidden_pos), ("proc", proc, hidden_pos, hidden_pos),
                              ("dec", dec, hidden_pos, data_pos)):
        t[f"graph.{name}.edge_index"] = np.ascontiguousarray(e.T.astype(np.int64))
        if edge_attr == "geometric" and ps is not None and Ae == 3:
            t[f"graph.{name}.edge_attr"] = edge_attributes(ps, pdst, e[:, 0], e[:, 1])
        elif edge_attr == "uniform":
            t[f"graph.{name}.edge_attr"] = rng.uniform(0, 1, (len(e), Ae)).astype(np.float32)
        else:
            t[f"graph.{name}.edge_attr"] = rng.normal(0, 1, (len(e), Ae)).astype(np.float32)
    F = T * Vi + A
    absent = set(absent)
    absent_list = []
    blocks = ["enc.block"] + [f"proc.{i}" for i in range(n_proc)] + ["dec.block"]

    def lin(name, o, i):
        std = math.sqrt(2.0 / (i + o)) if xavier else 1.0 / math.sqrt(i)
        t[name + ".weight"] = (rng.standard_normal((o, i), dtype=np.float32) * np.float32(std * weight_scale))
        if name + ".bias" in absent:
            absent_list.append(name + ".bias")
        else:
            t[name + ".bias"] = rng.normal(0, 0.1, o).astype(np.float32)

    def ln(name):
        t[name + ".weight"] = rng.uniform(0.7, 1.3, C).astype(np.float32)
        if name + ".bias" in absent:
            absent_list.append(name + ".bias")
        else:
            t[name + ".bias"] = rng.normal(0, 0.1, C).astype(np.float32)

    lin("enc.emb_src", C, F)
    lin("enc.emb_dst", C, A)
    lin("dec.emb_dst", C, F)
    ln("dec.out_norm")
    lin("dec.out_proj", T_out * Vo, C)
    for b in blocks:
        for l in ("q", "k", "v", "self", "proj"):
            lin(f"{b}.{l}", C, C)
        lin(f"{b}.edge", C, Ae)
        lin(f"{b}.mlp1", mlp, C)
        lin(f"{b}.mlp2", C, mlp)
        ln(f"{b}.ln_dst")
        ln(f"{b}.ln_mlp")
        if b in ("enc.block", "dec.block"):
            ln(f"{b}.ln_src")
    names = var_names or [f"v{i}" for i in range(Vd)]
    cfg = {
        "format_version": 3,
        "source": {"checkpoint": "synthetic (varda_b200.synth)", "uuid": uuid or f"b200-synthetic-{seed}"},
        "architecture": {
            "model": {"kind": "enc_proc_dec" if times is None else "enc_proc_dec_interpolator"},
            "encoder": {"kind": "graph_transformer_forward_mapper"},
            "processor": {"kind": "graph_transformer_processor"},
            "decoder": {"kind": "graph_transformer_backward_mapper"}},
        "dims": {"num_channels": C, "num_heads": heads, "head_dim": C // heads, "mlp_hidden": mlp,
                 "num_processor_layers": n_proc, "n_input_steps": T, "n_output_steps": T_out,
                 "n_data_vars": Vd, "n_input_vars": Vi, "n_output_vars": Vo, "n_data_nodes": int(G),
                 "n_hidden_nodes": int(H), "node_attr_dim": A, "edge_attr_dim": Ae, "layer_norm_eps": 1e-5,
                 "gelu_approximate": gelu, "latent_skip": bool(latent_skip)},
        "variables": {"data": names, "input": [names[i] for i in norm_input],
                      "output": [names[i] for i in norm_output]},
        "indices": {"norm_input": list(norm_input), "norm_output": list(norm_output),
                    "residual_input": list(res_in), "residual_output": list(res_out)},
        "residual": {"type": "skip", "step": res_step},
        "bounding": bounding,
        "mappers": {"enc": {"num_chunks": 1}, "dec": {"num_chunks": 1}},
        "blocks": {b: {"kind": "graph_transformer_mapper_block" if b in ("enc.block", "dec.block")
                       else "graph_transformer_processor_block"} for b in blocks},
        "absent": absent_list,
        "unused": [],
    }
    if times is not None:
        cfg["times"] = times
    if forcings is not None:
        cfg["forcings"] = forcings
    x = rng.standard_normal((1, T, G, Vi), dtype=np.float32)
    return cfg, t, x


def write_model(path, cfg, t):
    st.write(path, t, {"varda_format": "1", "config": json.dumps(cfg)})


def write_input(path, x):
    st.write(path, {"in.x": x}, {"producer": "varda_b200.synth"})


def _vars(Vd, Vi, Vo, n_prog):
    """Variable layout: data vars 0..Vd-1; inputs are the first Vi, outputs the first Vo; the
    first n_prog are prognostic (residual pairs). Boundings on outputs 3..7: relu, hardtanh,
    fraction with the hardtanh output as total."""
    b = [{"type": "relu", "index": [3]},
         {"type": "hardtanh", "index": [4], "min": 0.0, "max": 1.0},
         {"type": "fraction", "index": [5, 6, 7], "min": 0.0, "max": 1.0, "total_index": [4]}]
    return dict(Vd=Vd, Vi=Vi, Vo=Vo, norm_input=list(range(Vi)), norm_output=list(range(Vo)),
                res_in=list(range(n_prog)), res_out=list(range(n_prog)), bounding=b)


def config_c0(seed=0):
    data, hidden, enc, proc, dec = _sort_nodes(*graph_c0())
    v = _vars(10, 10, 8, 8)
    return make_model(seed=seed, C=128, heads=4, mlp=512, n_proc=2, T=2, data_pos=data, hidden_pos=hidden,
                      enc=enc, proc=proc, dec=dec, A=4, Ae=3, uuid="b200-c0", **v)


_C1_CACHE = {}


def c1_graph(seed_unused=0):
    if "g" not in _C1_CACHE:
        _C1_CACHE["g"] = _sort_nodes(*graph_c1())
    return _C1_CACHE["g"]


def _c1_forcings():
    dyn = list(range(80, 86))
    const = list(range(86, 90))
    names = [f"v{i}" for i in range(80)] + [f"f{i}" for i in range(10)]
    return names, {"dynamic": [names[i] for i in dyn], "dynamic_input_index": dyn,
                   "constant": [names[i] for i in const], "constant_input_index": const,
                   "timestep_hours": 6, "source": "varda_b200.synth"}


def config_c1(seed=1, n_proc=16, T_out=1, G=None):
    data, hidden, enc, proc, dec = c1_graph()
    names, forc = _c1_forcings()
    v = _vars(90, 90, 80, 80)
    kw = {}
    if T_out > 1:
        kw = dict(T_out=T_out, times={"input": [0, T_out], "target": list(range(1, T_out + 1)),
                                      "frequency_hours": 1}, res_step=0, latent_skip=False)
    return make_model(seed=seed, C=1024, heads=16, mlp=4096, n_proc=n_proc, T=2, data_pos=data,
                      hidden_pos=hidden, enc=enc, proc=proc, dec=dec, A=4, Ae=3, var_names=names,
                      forcings=forc if T_out == 1 else None, uuid=f"b200-c1-T{T_out}", **v, **kw)


TEST_DEGREES = [0, 1, 2, 3, 5, 8, 17, 33, 64]


def config_test(name):
    """Small random-graph models for GPU parity tests (own choice of shapes)."""
    specs = {
        # C, heads, mlp, n_proc, T, A, Ae, gelu, skip, res_step, absent?, G, H, T_out
        "t256": (11, 256, 8, 520, 2, 2, 4, 3, "none", True, -1, False, 300, 70, 1),
        "t512": (12, 512, 4, 1024, 1, 3, 5, 2, "tanh", False, 0, True, 260, 61, 1),
        "t1024": (13, 1024, 16, 4096, 2, 2, 4, 3, "none", True, -1, False, 301, 67, 1),
        "t128": (14, 128, 4, 512, 2, 2, 4, 3, "none", True, -1, False, 333, 90, 1),
        "t768": (15, 768, 12, 1536, 1, 2, 3, 1, "tanh", True, -2, True, 211, 47, 1),
        "t384i": (16, 384, 6, 768, 2, 2, 4, 3, "none", False, 0, False, 257, 53, 6),
        "t2048": (17, 2048, 8, 512, 1, 2, 4, 3, "tanh", True, -1, True, 120, 30, 1),
    }
    rollout = name.endswith("r") and name[:-1] in specs
    base = name[:-1] if rollout else name
    (seed, C, heads, mlp, n_proc, T, A, Ae, gelu, skip, rs, absent_kind, G, H, T_out) = specs[base]
    rng = np.random.default_rng(1000 + seed)
    enc = random_graph(rng, G, H, [0, 1, 2, 3, 5, 8, 17, 33, 64, 9, 12])
    proc = random_graph(rng, H, H, [0, 1, 2, 3, 5, 8, 17, 33, 64, 6])
    dec = random_graph(rng, H, G, [0, 1, 2, 3, 4])
    absent = []
    if absent_kind:
        for b in ["enc.block"] + [f"proc.{i}" for i in range(n_proc)] + ["dec.block"]:
            absent += [f"{b}.{l}.bias" for l in ("q", "k", "v", "self", "edge")]
        absent += ["dec.out_norm.bias", "enc.block.ln_mlp.bias"]
    v = _vars(12, 10, 8, 6)
    kw = {}
    if T_out > 1:
        kw = dict(T_out=T_out, times={"input": [0, T_out], "target": list(range(1, T_out + 1)),
                                      "frequency_hours": 1})
    if rollout:
        # 6 prognostic inputs (0..5 <- outputs 0..5), dynamic forcings 6..8, constant 9
        names = [f"v{i}" for i in range(12)]
        kw["var_names"] = names
        kw["forcings"] = {"dynamic": [names[i] for i in (6, 7, 8)], "dynamic_input_index": [6, 7, 8],
                          "constant": [names[9]], "constant_input_index": [9], "timestep_hours": 6,
                          "source": "varda_b200.synth"}
    cfg, t, x = make_model(seed=seed, C=C, heads=heads, mlp=mlp, n_proc=n_proc, T=T, G=G, H=H, enc=enc, proc=proc,
                           dec=dec, A=A, Ae=Ae, gelu=gelu, latent_skip=skip, res_step=rs, absent=absent,
                           edge_attr="normal", xavier=False, uuid=f"b200-{name}", **v, **kw)
    if rollout:
        g = np.random.default_rng(2000 + seed)
        t["grid.latitudes"] = g.uniform(-80.0, 80.0, G).astype(np.float64)
        t["grid.longitudes"] = g.uniform(0.0, 360.0, G).astype(np.float64)
    return cfg, t, x


def replay_forcings(n_steps, G, F, timestep_hours=6, seed=0):
    """Synthetic dynamic forcings to replay in a rollout: (n_steps - 1, G, F) fp32 sin/cos waves of the
    valid time of each step (forcing s belongs to the output of step s) with a per-node phase."""
    rng = np.random.default_rng(seed)
    phase = rng.uniform(0.0, 2.0 * np.pi, (G, 1))
    s = np.arange(1, max(n_steps, 1), dtype=np.float64)[:, None, None]
    hours = s * timestep_hours
    k = np.arange(F, dtype=np.float64)[None, None, :]
    period = np.where(k % 2 == 0, 24.0, 24.0 * 365.25)
    f = np.where(k % 3 == 2, np.cos(2 * np.pi * hours / period + phase[None]),
                 np.sin(2 * np.pi * hours / period + phase[None] + k))
    return np.ascontiguousarray(f.astype(np.float32))


def sha256_file(path, chunk=1 << 24):
    h = hashlib.sha256()
    with open(path, "rb") as f:
        while True:
            b = f.read(chunk)
            if not b:
                break
            h.update(b)
    return h.hexdigest()


C1_SAMPLE_FACTOR = 64
C2_SAMPLE_FACTOR = 8


def fibonacci_sphere(n):
    """n nearly uniform unit vectors (the Fibonacci lattice)."""
    i = np.arange(n) + 0.5
    z = 1 - 2 * i / n
    phi = i * np.pi * (3 - 5 ** 0.5)
    r = np.sqrt(1 - z * z)
    return np.stack([r * np.cos(phi), r * np.sin(phi), z], 1)


def config_c2(seed=2, n_proc=1, sample=1, G=4096):
    """c2: the isolated processor block (C2) as a complete model file. Hidden nodes and processor graph
    of graph_c2 (edge attributes U[0, 1) from `seed`), C=1024, 16 heads of 64, mlp 4096, `n_proc`
    processor blocks. The data grid only completes the file: G Fibonacci-lattice nodes, each sending to
    its 4 nearest hidden nodes and receiving from its 3 nearest. With sample > 1 the hidden nodes are
    the first 1/sample of graph_c2's (Morton order, so a compact region) with the edges among them: the
    bounded sample the reference CPU backend is timed on."""
    hidden, proc, attr = graph_c2(seed=seed)
    if sample > 1:
        Hs = len(hidden) // sample
        keep = (proc[:, 0] < Hs) & (proc[:, 1] < Hs)
        hidden, proc, attr = hidden[:Hs], proc[keep], attr[keep]
    data = fibonacci_sphere(G)
    data = data[morton_order(data)]

    def srt(e):
        return e[np.lexsort((e[:, 0], e[:, 1]))]

    enc = srt(np.stack([np.repeat(np.arange(G), 4), knn(hidden, data, 4).ravel()], 1))
    dec = srt(np.stack([knn(hidden, data, 3).ravel(), np.repeat(np.arange(G), 3)], 1))
    v = _vars(8, 8, 8, 8)
    cfg, t, x = make_model(seed=seed, C=1024, heads=16, mlp=4096, n_proc=n_proc, T=2, data_pos=data,
                           hidden_pos=hidden, enc=enc, proc=proc, dec=dec, A=4, Ae=3,
                           uuid=f"b200-c2-p{n_proc}-s{sample}", **v)
    t["graph.proc.edge_attr"] = attr
    return cfg, t, x


def c2_features(rows, C=1024, seed=2):
    """C2's node features: N(0, 1) float32 [rows, C] from `seed`."""
    return np.random.default_rng(seed + 1000).standard_normal((rows, C), dtype=np.float32)


def config_c1_sample(factor=C1_SAMPLE_FACTOR):
    """c1s: C1's architecture on 1/factor of its nodes, with the same per-node edge counts."""
    G, H = 1_688_650 // factor, 189_809 // factor
    fib = fibonacci_sphere

    data, hidden = fib(G), fib(H)
    enc = np.stack([np.repeat(np.arange(G), 4), knn(hidden, data, 4).ravel()], 1)
    nb = knn(hidden, hidden, 15)[:, 1:]
    proc = np.stack([nb.ravel(), np.repeat(np.arange(H), 14)], 1)
    dec = np.stack([knn(hidden, data, 3).ravel(), np.repeat(np.arange(G), 3)], 1)
    data, hidden, enc, proc, dec = _sort_nodes(data, hidden, enc, proc, dec)
    names, forc = _c1_forcings()
    v = _vars(90, 90, 80, 80)
    return make_model(seed=1, C=1024, heads=16, mlp=4096, n_proc=16, T=2, data_pos=data, hidden_pos=hidden,
                      enc=enc, proc=proc, dec=dec, A=4, Ae=3, var_names=names, forcings=forc,
                      uuid="b200-c1-sample", **v)


def generate(name, out_dir, **kw):
    """Writes <out_dir>/<name>.model.safetensors and <name>.input.safetensors; returns the paths."""
    os.makedirs(out_dir, exist_ok=True)
    mp = os.path.join(out_dir, f"{name}.model.safetensors")
    xp = os.path.join(out_dir, f"{name}.input.safetensors")
    if name == "c0":
        cfg, t, x = config_c0(**kw)
    elif name == "c1":
        cfg, t, x = config_c1(**kw)
    elif name == "c3":
        cfg, t, x = config_c1(T_out=6, **kw)
    elif name == "c1s":
        cfg, t, x = config_c1_sample(**kw)
    elif name == "c2":
        cfg, t, x = config_c2(**kw)
    elif name in ("c2s1", "c2s3"):  # the CPU baseline's sample: 1 and 3 processor blocks
        cfg, t, x = config_c2(n_proc=int(name[-1]), sample=C2_SAMPLE_FACTOR, **kw)
    else:
        cfg, t, x = config_test(name)
    write_model(mp, cfg, t)
    write_input(xp, x)
    return mp, xp


def main():
    ap = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    ap.add_argument("name")
    ap.add_argument("--out", required=True)
    ap.add_argument("--n-proc", type=int, default=None)
    a = ap.parse_args()
    kw = {} if a.n_proc is None else {"n_proc": a.n_proc}
    print(generate(a.name, a.out, **kw))


if __name__ == "__main__":
    main()
