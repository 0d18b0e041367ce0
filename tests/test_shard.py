"""The destination partition for multi-GPU runs, on CPU.

* plans for 1..4 ranks are consistent (ranges cover every node once, what r sends to p is what p
  expects from r, local graphs keep every destination's stored edge order), with and without the
  encoder split (VB_SHARD_ENC=1: the encoder's own hidden ranges, whose output rows then move to
  their processor owners);
* two `gloo` ranks exchange K|V halo rows by the plan and compute the graph attention of their own
  destination rows on their local graphs with the CPU oracle: every row is bitwise equal to the
  single-process result, which is what makes the sharded GPU result independent of the GPU count;
* with the encoder split, three `gloo` ranks compute the encoder attention of their encoder rows and
  move them to their processor owners by the plan: again bitwise the single-process rows.
"""
import os

import numpy as np
import pytest

import oracle
import varda_b200 as vb
from varda_b200 import safetensors as st


def plans(path, world):
    return [vb.shard_plan(path, world, r) for r in range(world)]


def rows(lo, hi):
    """A row range [lo, hi), or None when it is empty."""
    return (lo, hi) if hi > lo else None


@pytest.mark.parametrize("enc_split", [False, True])
@pytest.mark.parametrize("name", ["t256", "c0"])
@pytest.mark.parametrize("world", [1, 2, 3, 4, 8])
def test_plan_consistency(name, world, enc_split, seeded_model, monkeypatch):
    mp, _ = seeded_model(name)
    monkeypatch.setenv("VB_SHARD_ENC", "1" if enc_split else "0")
    t, meta = st.read(mp)
    import json
    d = json.loads(meta["config"])["dims"]
    G, H = d["n_data_nodes"], d["n_hidden_nodes"]
    ps = plans(mp, world)
    hs, gs = ps[0]["h_split"], ps[0]["g_split"]
    assert hs[0] == 0 and hs[-1] == H and gs[0] == 0 and gs[-1] == G
    assert all(np.diff(hs) >= 0) and all(np.diff(gs) >= 0)
    full = {g: oracle.build_csr(t[f"graph.{g}.edge_index"], t[f"graph.{g}.edge_attr"], *ns)
            for g, ns in (("enc", (G, H)), ("proc", (H, H)), ("dec", (H, G)))}
    es = ps[0]["e_split"]
    assert es[0] == 0 and es[-1] == H and all(np.diff(es) >= 0)
    if not enc_split or world == 1:
        assert es == hs
    else:  # the processor's and decoder's ranges do not depend on the encoder split
        monkeypatch.setenv("VB_SHARD_ENC", "0")
        base = vb.shard_plan(mp, world, 0)
        monkeypatch.setenv("VB_SHARD_ENC", "1")
        assert base["h_split"] == hs and base["g_split"] == gs and base["e_split"] == hs
        assert all(np.diff(es) > 0), "every encoder range is non-empty"
    for r, p in enumerate(ps):
        assert p["h_split"] == hs and p["g_split"] == gs and p["e_split"] == es
        # encoder output rows: what r sends p is what p receives from r; the received ranges (and
        # the kept one) tile r's hidden range, the sent ones r's encoder range
        m = p["enc_move"]
        for q in range(world):
            mq = ps[q]["enc_move"]
            assert rows(m["send_lo"][q], m["send_hi"][q]) == rows(mq["recv_lo"][r], mq["recv_hi"][r])
        for lo_key, hi_key, (lo, hi) in (("recv_lo", "recv_hi", hs[r:r + 2]), ("send_lo", "send_hi", es[r:r + 2])):
            cover = sorted((m[lo_key][q], m[hi_key][q]) for q in range(world) if m[hi_key][q] > m[lo_key][q])
            pos = lo
            for a, b in cover:
                assert a == pos, "row ranges tile the range without gaps or overlaps"
                pos = b
            assert pos == hi
        for key in ("proc", "dec"):
            halo = p[key]["halo"]
            assert halo == sorted(set(halo))
            for q in range(world):
                mine = [s for s in halo if hs[q] <= s < hs[q + 1]]
                assert len(mine) == p[key]["recv_count"][q]
                if q != r:
                    assert ps[q][key]["send"][r] == mine, f"{key}: rank {q} must send rank {r} exactly its halo"
                else:
                    assert mine == []
        # local graphs: own rows, stored edge order kept, sources mapped back to the same global ids
        for key, gname, (lo, hi), (slo, shi), halo in (
                ("proc_g", "proc", hs[r:r + 2], hs[r:r + 2], p["proc"]["halo"]),
                ("dec_g", "dec", gs[r:r + 2], hs[r:r + 2], p["dec"]["halo"]),
                ("enc", "enc", es[r:r + 2], gs[r:r + 2], p["enc_halo"])):
            lg = p[key]
            rp, src, eid, _ = full[gname]
            e0, e1 = rp[lo], rp[hi]
            assert np.array_equal(np.array(lg["row_ptr"]) + e0, rp[lo:hi + 1])
            assert np.array_equal(lg["edge_id"], eid[e0:e1])
            own = shi - slo
            loc = np.array(lg["src"], np.int64)
            back = np.where(loc < own, loc + slo, np.array(halo + [0], np.int64)[np.clip(loc - own, 0, None)])
            assert np.array_equal(back, src[e0:e1])


def _rank_main(rank, world, mp, port, out_dir):
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    import sys
    here = os.path.dirname(os.path.abspath(__file__))
    sys.path.insert(0, os.path.join(os.path.dirname(here), "oracle"))
    t, meta = st.read(mp)
    import json
    d = json.loads(meta["config"])["dims"]
    H, C, heads = d["n_hidden_nodes"], d["num_channels"], d["num_heads"]
    p = vb.shard_plan(mp, world, rank)
    hs = p["h_split"]
    lo, hi = hs[rank], hs[rank + 1]
    rng = np.random.default_rng(7)  # the same global tensors on every rank
    q, k, v = (rng.normal(size=(H, C)).astype(np.float32) for _ in range(3))
    we = rng.normal(size=(3, C)).astype(np.float32)
    be = rng.normal(size=C).astype(np.float32)
    kv_own = np.concatenate([k[lo:hi], v[lo:hi]], 1)
    # halo exchange by the plan: send own rows each peer needs, receive the halo in peer order
    reqs = []
    for peer in range(world):
        if peer == rank:
            continue
        send = p["proc"]["send"][peer]
        if send:
            import torch
            buf = torch.from_numpy(np.ascontiguousarray(kv_own[np.array(send) - lo]))
            reqs.append(dist.isend(buf, peer))
    import torch
    halo_parts = []
    for peer in range(world):
        n = p["proc"]["recv_count"][peer]
        if peer == rank or n == 0:
            continue
        buf = torch.empty((n, 2 * C), dtype=torch.float32)
        dist.recv(buf, peer)
        halo_parts.append(buf.numpy())
    for rq in reqs:
        rq.wait()
    kv_loc = np.concatenate([kv_own] + halo_parts, 0)
    lg = p["proc_g"]
    rp = np.array(lg["row_ptr"], np.int32)
    src = np.array(lg["src"], np.int32)
    attr = t["graph.proc.edge_attr"][np.array(lg["edge_id"], np.int64)]
    out = oracle.graph_attention((rp, src, None, np.ascontiguousarray(attr)), 0, hi - lo, q[lo:hi],
                                 kv_loc[:, :C], kv_loc[:, C:], we.T.copy(), be, heads, C // heads)
    np.save(os.path.join(out_dir, f"rank{rank}.npy"), out)
    dist.barrier()
    dist.destroy_process_group()


def test_gloo_two_ranks_halo_exchange_matches_single_process(seeded_model, tmp_path):
    import torch.multiprocessing as mp_
    mp, _ = seeded_model("c0")
    world = 2
    port = 29500 + os.getpid() % 1000
    mp_.start_processes(_rank_main, args=(world, mp, port, str(tmp_path)), nprocs=world, join=True,
                        start_method="spawn")
    t, meta = st.read(mp)
    import json
    d = json.loads(meta["config"])["dims"]
    H, C, heads = d["n_hidden_nodes"], d["num_channels"], d["num_heads"]
    rng = np.random.default_rng(7)
    q, k, v = (rng.normal(size=(H, C)).astype(np.float32) for _ in range(3))
    we = rng.normal(size=(3, C)).astype(np.float32)
    be = rng.normal(size=C).astype(np.float32)
    csr = oracle.build_csr(t["graph.proc.edge_index"], t["graph.proc.edge_attr"], H, H)
    full = oracle.graph_attention(csr, 0, H, q, k, v, we.T.copy(), be, heads, C // heads)
    hs = vb.shard_plan(mp, world, 0)["h_split"]
    for r in range(world):
        part = np.load(tmp_path / f"rank{r}.npy")
        assert np.array_equal(part, full[hs[r]:hs[r + 1]]), f"rank {r} rows differ from the single-process result"


def _enc_rank_main(rank, world, mp, port, out_dir):
    """Encoder split on `gloo`: the encoder attention of this rank's encoder rows, then every row to its
    processor owner by the plan's row ranges."""
    import json
    import torch
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), VB_SHARD_ENC="1")
    dist.init_process_group("gloo", rank=rank, world_size=world)
    t, meta = st.read(mp)
    d = json.loads(meta["config"])["dims"]
    G, H, C, heads = d["n_data_nodes"], d["n_hidden_nodes"], d["num_channels"], d["num_heads"]
    p = vb.shard_plan(mp, world, rank)
    gs, hs, es = p["g_split"], p["h_split"], p["e_split"]
    q, k, v, we, be = _enc_tensors(G, H, C)
    # local sources: own data rows, then the encoder halo (global ids, ascending)
    srcs = np.concatenate([np.arange(gs[rank], gs[rank + 1]), np.array(p["enc_halo"], np.int64)])
    lg = p["enc"]
    attr = t["graph.enc.edge_attr"][np.array(lg["edge_id"], np.int64)]
    e_lo, e_hi = es[rank], es[rank + 1]
    out = oracle.graph_attention((np.array(lg["row_ptr"], np.int32), np.array(lg["src"], np.int32), None,
                                  np.ascontiguousarray(attr)), 0, e_hi - e_lo, q[e_lo:e_hi], k[srcs], v[srcs],
                                 we.T.copy(), be, heads, C // heads)
    m = p["enc_move"]
    h_lo, h_hi = hs[rank], hs[rank + 1]
    mine = np.full((h_hi - h_lo, C), np.nan, np.float32)
    reqs = []
    for peer in range(world):
        a, b = m["send_lo"][peer], m["send_hi"][peer]
        if b <= a:
            continue
        if peer == rank:
            mine[a - h_lo:b - h_lo] = out[a - e_lo:b - e_lo]
        else:
            reqs.append(dist.isend(torch.from_numpy(np.ascontiguousarray(out[a - e_lo:b - e_lo])), peer))
    for peer in range(world):
        a, b = m["recv_lo"][peer], m["recv_hi"][peer]
        if peer == rank or b <= a:
            continue
        buf = torch.empty((b - a, C), dtype=torch.float32)
        dist.recv(buf, peer)
        mine[a - h_lo:b - h_lo] = buf.numpy()
    for rq in reqs:
        rq.wait()
    np.save(os.path.join(out_dir, f"enc{rank}.npy"), mine)
    dist.barrier()
    dist.destroy_process_group()


def _enc_tensors(G, H, C):
    rng = np.random.default_rng(11)  # the same global tensors on every rank
    q = rng.normal(size=(H, C)).astype(np.float32)
    k, v = (rng.normal(size=(G, C)).astype(np.float32) for _ in range(2))
    return q, k, v, rng.normal(size=(3, C)).astype(np.float32), rng.normal(size=C).astype(np.float32)


def test_gloo_encoder_split_moves_rows_to_their_owners(seeded_model, tmp_path, monkeypatch):
    import json
    import torch.multiprocessing as mp_
    mp, _ = seeded_model("t256")
    world = 3
    monkeypatch.setenv("VB_SHARD_ENC", "1")
    p0 = vb.shard_plan(mp, world, 0)
    assert p0["e_split"] != p0["h_split"], "the test model must move encoder rows between ranks"
    port = 29500 + (os.getpid() + 500) % 1000
    mp_.start_processes(_enc_rank_main, args=(world, mp, port, str(tmp_path)), nprocs=world, join=True,
                        start_method="spawn")
    t, meta = st.read(mp)
    d = json.loads(meta["config"])["dims"]
    G, H, C, heads = d["n_data_nodes"], d["n_hidden_nodes"], d["num_channels"], d["num_heads"]
    q, k, v, we, be = _enc_tensors(G, H, C)
    csr = oracle.build_csr(t["graph.enc.edge_index"], t["graph.enc.edge_attr"], G, H)
    full = oracle.graph_attention(csr, 0, H, q, k, v, we.T.copy(), be, heads, C // heads)
    hs = p0["h_split"]
    for r in range(world):
        part = np.load(tmp_path / f"enc{r}.npy")
        assert np.array_equal(part, full[hs[r]:hs[r + 1]]), f"rank {r}: encoder rows differ from the single process"
