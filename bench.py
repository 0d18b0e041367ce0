"""Benchmark: ms per fp16 predict_step at the Varda shape (the benchmark's config C1), plus edge-attention
HBM GB/s, on N B200s of one node.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference] [--workload c1|c0|c2|c3|c4]

Prints one JSON line (rank 0). `value` is the device-resident time of one predict_step (the model's
own input/output buffers, CUDA-graph replay, CUDA events on the model's stream, max over ranks);
`e2e` is the same through the public host API vb_predict_step with pinned host buffers (H2D of x and
D2H of y inside the timed region; the library overlaps them with the compute in row chunks). `roofline` describes the dominant kernel class and
`edge_attention` the processor-block attention (compulsory bytes; on one GPU also the K|V bytes its
edges gather, mostly L2 hits), both from one eager pass with a CUDA event pair around every launch
(vb_profile_forward). `cpu_baseline` is the reference's own CPU fp32 backend
(oracle/_ref/ref_dump, built from the reference's sources) timed on this host on a bounded sample.

--workload c2 is the isolated processor block (the benchmark's config C2: the C1 hidden graph, 189,809 rows,
2.63M edges with U[0,1) attributes, C=1024, fp16, N(0,1) node features) through vb_processor_block:
`value` = device ms per block run (LN_dst + the block, K runs on the same input, sharded runs exchanging
the K|V halo every run), `e2e` = the same with the host fp32 features copied in and the output copied
back every run. Its `cpu_baseline` / reference arm is the reference CPU backend's time per processor
block: ref_dump on models with 3 and with 1 block over the same 1/8 sample of the graph, half the
difference, scaled by the row count (C2_SAMPLE_FACTOR).

--workload c4 is the 24-step autoregressive rollout of C1 (the benchmark's config C4): K rollout steps through
vb_rollout (CUDA graph per step, forcings replayed from the host, every step's output copied back to
pinned host memory), `value` = device ms per rollout step, `e2e` = wall time of the whole rollout call
per step.

--impl reference times that reference CPU backend alone (rank 0; other ranks exit 0).
Inputs and activations (tens of GB) are far larger than the 126 MB L2, so no L2 flush is needed.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(HERE, "varda.cpp_b200"))

PEAKS_FALLBACK = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}
CACHE = os.environ.get("VB_BENCH_CACHE", os.path.join(tempfile.gettempdir(), "varda_b200_bench"))
REF_DUMP = os.path.join(HERE, "oracle", "_ref", "ref_dump")
SAMPLE_FACTOR = 64  # the CPU baseline runs the C1 architecture on 1/64 of its nodes (synth "c1s")


def peaks():
    p = os.path.join(HERE, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        d = json.load(open(p))
        return d, "measured"
    return PEAKS_FALLBACK, "fallback"


def log(*a):
    print(*a, file=sys.stderr, flush=True)


# ------------------------------------------------------------------ models
def model_paths(workload):
    from varda_b200 import synth
    os.makedirs(CACHE, exist_ok=True)
    mp = os.path.join(CACHE, f"{workload}.model.safetensors")
    xp = os.path.join(CACHE, f"{workload}.input.safetensors")
    if not (os.path.exists(mp) and os.path.exists(xp)):
        t0 = time.time()
        synth.generate(workload, CACHE)
        log(f"bench: generated {workload} in {time.time() - t0:.1f} s")
    return mp, xp


def sample_model():
    """c1s: C1's architecture on 1/SAMPLE_FACTOR of its nodes with the same per-node edge counts
    (varda_b200.synth.config_c1_sample)."""
    from varda_b200 import synth
    os.makedirs(CACHE, exist_ok=True)
    mp = os.path.join(CACHE, "c1s.model.safetensors")
    xp = os.path.join(CACHE, "c1s.input.safetensors")
    if not (os.path.exists(mp) and os.path.exists(xp)):
        synth.generate("c1s", CACHE)
    return mp, xp


def ref_env():
    """Environment for the reference CPU runs. The OpenBLAS 0.3.15 its build links does not recognise
    some recent Xeons and then runs its generic kernels (5x slower on this pool's CPU container); unless
    OPENBLAS_CORETYPE is set, name the core type from the CPU's flags so the reference gets its fast
    kernels."""
    env = dict(os.environ)
    if not env.get("OPENBLAS_CORETYPE"):
        try:
            flags = open("/proc/cpuinfo").read()
        except OSError:
            flags = ""
        if " avx512f" in flags:
            env["OPENBLAS_CORETYPE"] = "SkylakeX"
        elif " avx2" in flags:
            env["OPENBLAS_CORETYPE"] = "Haswell"
    return env


def reference_cpu(steps, warmup, threads=0):
    """The reference's CPU fp32 backend on the bounded sample; per-step seconds, scaled to the full
    C1 node count (every op of the forward pass is linear in node and edge counts)."""
    if not os.path.exists(REF_DUMP):
        raise FileNotFoundError(f"{REF_DUMP} missing (make -C oracle with the reference sources)")
    mp, xp = sample_model()
    cmd = [REF_DUMP, "--model", mp, "--input", xp, "--steps", str(warmup + steps)]
    if threads:
        cmd += ["--threads", str(threads)]
    r = subprocess.run(cmd, capture_output=True, text=True, check=True, env=ref_env())
    rec = json.loads(r.stdout.strip().splitlines()[-1])
    times = rec["steps_s"][warmup:]
    return times, rec["threads"], SAMPLE_FACTOR


def reference_cpu_c2(steps, warmup):
    """The reference's CPU fp32 backend per processor block of C2: ref_dump on the c2s1 and c2s3 models
    (1 and 3 processor blocks over the first 1/8 of the C2 graph's rows with the edges among them; the
    encoder, decoder and I/O identical in both), half the per-step difference, scaled by the row count
    (the block's GEMMs, which dominate it on the CPU, are linear in rows)."""
    if not os.path.exists(REF_DUMP):
        raise FileNotFoundError(f"{REF_DUMP} missing (make -C oracle with the reference sources)")
    from varda_b200 import safetensors as st
    recs = {}
    for name in ("c2s1", "c2s3"):
        mp, xp = model_paths(name)
        r = subprocess.run([REF_DUMP, "--model", mp, "--input", xp, "--steps", str(warmup + steps)],
                           capture_output=True, text=True, check=True, env=ref_env())
        recs[name] = json.loads(r.stdout.strip().splitlines()[-1])
    hs = int(json.loads(st.read(model_paths("c2s1")[0])[1]["config"])["dims"]["n_hidden_nodes"])
    f = 189_809 / hs
    t1, t3 = recs["c2s1"]["steps_s"][warmup:], recs["c2s3"]["steps_s"][warmup:]
    times = [(b - a) / 2 * f for a, b in zip(t1, t3)]
    return times, recs["c2s1"]["threads"], hs


# ------------------------------------------------------------------ clocks
class Clocks:
    def __init__(self, device):
        self.f = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)
        self.p = subprocess.Popen(
            ["nvidia-smi", "-i", str(device), "--query-gpu=index,clocks.sm,clocks.max.sm,power.draw,"
             "clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap",
             "--format=csv,noheader,nounits", "-lms", "100"], stdout=self.f, stderr=subprocess.DEVNULL)

    def start_region(self, timeout=5.0):
        """Waits (outside the timed region) until nvidia-smi, which takes a moment to start, has written
        a row, and marks where the region's rows begin: a region of a few hundred ms is then sampled too."""
        t0 = time.time()
        while time.time() - t0 < timeout and os.path.getsize(self.f.name) == 0:
            time.sleep(0.02)
        self.f.flush()
        with open(self.f.name) as f:
            self.skip = sum(1 for l in f if l.strip())

    def stop(self):
        self.p.terminate()
        try:
            self.p.wait(5)
        except Exception:
            self.p.kill()
        self.f.seek(0)
        rows = [l.split(",") for l in self.f.read().strip().splitlines() if l.strip()]
        skip = getattr(self, "skip", 0)
        if len(rows) > skip:  # the rows taken before the region (kept only if the region got none)
            rows = rows[skip:]
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for r in rows:
            try:
                sm.append(float(r[1]))
                mx = float(r[2])
                for n, v in zip(names, r[5:9]):
                    if v.strip() == "Active":
                        reasons.add(n)
            except (ValueError, IndexError):
                pass
        os.unlink(self.f.name)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx, "samples": len(sm),
                "reasons": sorted(reasons)}


# ------------------------------------------------------------------ ours
def load_model(args, rank, world, local_rank):
    import torch
    import varda_b200 as vb

    torch.cuda.set_device(local_rank)
    dist = None
    if world > 1:
        import torch.distributed as dist
        import datetime
        dist.init_process_group("gloo", timeout=datetime.timedelta(seconds=600))
    if rank == 0:
        mp, xp = model_paths(args.workload)
    if dist:
        dist.barrier()
    mp, xp = model_paths(args.workload)
    t0 = time.time()
    if world > 1:
        obj = [vb.nccl_unique_id() if rank == 0 else None]
        dist.broadcast_object_list(obj, src=0)
        m = vb.Model.load_sharded(mp, rank, world, obj[0], precision=vb.FP16, cuda_device=local_rank)
    else:
        m = vb.Model.load(mp, precision=vb.FP16, cuda_device=local_rank)
    load_s = time.time() - t0
    return m, mp, xp, dist, load_s


def run_ours(args, rank, world, local_rank):
    import torch
    import varda_b200 as vb
    from varda_b200 import safetensors as st

    m, mp, xp, dist, load_s = load_model(args, rank, world, local_rank)
    x = np.array(st.read(xp)[0]["in.x"])
    stream = torch.cuda.ExternalStream(m.stream(), device=f"cuda:{local_rank}")
    xh = torch.from_numpy(x).pin_memory().numpy()
    yh = torch.empty(m.output_shape, dtype=torch.float32).pin_memory().numpy()

    # warm-up through the host API: fills the model's own (this rank's) input buffer, runs the first
    # (eager) forward and captures the CUDA graph; the timed steps replay it on that input
    for _ in range(args.warmup):
        m.predict_step(xh, yh)
    torch.cuda.synchronize()
    # ... and the timed path itself (its first call captures the step's CUDA graph)
    for i in range(args.warmup):
        t0 = time.perf_counter()
        m.enqueue_predict()
        torch.cuda.synchronize()
        if i == 0:
            log(f"bench: first graph step (capture + run) {time.perf_counter() - t0:.3f} s")
    clk = Clocks(local_rank)
    clk.start_region()
    if dist:
        dist.barrier()
    n_launch0 = vb.launch_count()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    ev0.record(stream)
    for _ in range(args.steps):
        m.enqueue_predict()
    ev1.record(stream)
    torch.cuda.synchronize()
    clocks = clk.stop()
    ms = ev0.elapsed_time(ev1) / args.steps
    if dist:
        dist.barrier()

    # e2e through the host API: pinned x, y; H2D of this rank's input rows + forward + D2H of its
    # output rows every step (one untimed call first: on one GPU the host path is pipelined, and its
    # first call captures the pieces' graphs)
    for i in range(2):
        t0 = time.perf_counter()
        m.predict_step(xh, yh)
        torch.cuda.synchronize()
        log(f"bench: untimed host-API step {i} {time.perf_counter() - t0:.3f} s")
    if dist:
        dist.barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(args.steps):
        m.predict_step(xh, yh)
    e1.record(stream)
    torch.cuda.synchronize()
    e2e_ms = e0.elapsed_time(e1) / args.steps
    h2d = (m.data_hi - m.data_lo) * m.T_in * m.V_in * 4  # this rank's own input rows (halo rows come over NVLink)
    d2h = m.device_output_numel * 4  # this rank's output rows

    # one profiled eager pass: per-launch device times
    prof = m.profile()
    vb.check_device()
    launches_per_step = sum(1 for r in prof)  # every launch of one forward is profiled once
    if dist:
        t = torch.tensor([ms, e2e_ms], dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms, e2e_ms = t.tolist()
    return dict(m=m, ms=ms, e2e_ms=e2e_ms, clocks=clocks, prof=prof, load_s=load_s, h2d=h2d, d2h=d2h,
                launches=launches_per_step + 2, dist=dist, n_launch_timed=vb.launch_count() - n_launch0)


def run_rollout(args, rank, world, local_rank):
    """C4: K steps of the device rollout of C1 (vb_rollout), after a W-step warm-up rollout."""
    import torch
    import varda_b200 as vb
    from varda_b200 import safetensors as st, synth

    m, mp, xp, dist, load_s = load_model(args, rank, world, local_rank)
    x = torch.from_numpy(np.array(st.read(xp)[0]["in.x"])).pin_memory().numpy()
    cfg = json.loads(st.read(mp)[1]["config"])
    F = len(cfg["forcings"]["dynamic_input_index"])
    n = args.steps
    t0 = time.time()
    f = synth.replay_forcings(max(n, args.warmup), m.G, F, cfg["forcings"]["timestep_hours"], seed=3)
    f = torch.from_numpy(f).pin_memory().numpy()
    log(f"bench: forcings {f.shape} in {time.time() - t0:.1f} s")
    sums = []

    def on_step(s, rows):  # a light consumer of every step's output rows on the host
        sums.append(float(rows[::997].sum()))

    m.rollout(x, args.warmup, f[:max(args.warmup - 1, 0)], keep=False, on_step=on_step)
    torch.cuda.synchronize()
    clk = Clocks(local_rank)
    clk.start_region()
    if dist:
        dist.barrier()
    n_launch0 = vb.launch_count()
    sums.clear()
    t0 = time.perf_counter()
    _, step_ms = m.rollout(x, n, f[:n - 1], keep=False, on_step=on_step)
    wall = time.perf_counter() - t0
    clocks = clk.stop()
    assert len(sums) == n and all(np.isfinite(sums)), "rollout outputs not finite"
    ms = float(np.mean(step_ms))
    e2e_ms = wall * 1000 / n
    prof = m.profile()
    vb.check_device()
    if dist:
        t = torch.tensor([ms, e2e_ms], dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms, e2e_ms = t.tolist()
    own = m.data_hi - m.data_lo  # own rows: x0 once, one forcing row per own row and step
    h2d = (own * m.T_in * m.V_in * 4 + (n - 1) * own * F * 4) / n
    d2h = m.device_output_numel * 4
    return dict(m=m, ms=ms, e2e_ms=e2e_ms, clocks=clocks, prof=prof, load_s=load_s, h2d=h2d, d2h=d2h,
                launches=len(prof) + 2 + (1 if n > 1 else 0) + (1 if world > 1 else 0), dist=dist,
                step_ms=[round(float(v), 3) for v in step_ms], wall_s=wall,
                n_launch_timed=vb.launch_count() - n_launch0)


def run_c2(args, rank, world, local_rank):
    """C2: the isolated processor block through vb_processor_block on this rank's hidden rows."""
    import torch
    import varda_b200 as vb
    from varda_b200 import synth

    m, mp, xp, dist, load_s = load_model(args, rank, world, local_rank)
    rows = m.hidden_hi - m.hidden_lo
    z = synth.c2_features(m.H, m.C)[m.hidden_lo:m.hidden_hi]
    zin = torch.from_numpy(np.ascontiguousarray(z)).pin_memory().numpy()
    zout = torch.empty((rows, m.C), dtype=torch.float32).pin_memory().numpy()
    stream = torch.cuda.ExternalStream(m.stream(), device=f"cuda:{local_rank}")
    # the timed runs are short: the clock sampler runs from before the warm-up through the e2e runs
    clk = Clocks(local_rank)
    clk.start_region()
    time.sleep(0.5)
    for _ in range(args.warmup):
        m.processor_block(0, zin, zout)
    assert np.isfinite(zout).all(), "processor block output not finite"
    torch.cuda.synchronize()
    if dist:
        dist.barrier()
    n_launch0 = vb.launch_count()
    _, total_ms = m.processor_block(0, None, None, repeats=args.steps)
    ms = total_ms / args.steps
    n_launch = vb.launch_count() - n_launch0
    if dist:
        dist.barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(args.steps):
        m.processor_block(0, zin, zout)
    e1.record(stream)
    torch.cuda.synchronize()
    e2e_ms = e0.elapsed_time(e1) / args.steps
    clocks = clk.stop()
    clocks["window"] = "warm-up through the e2e runs"
    prof = m.profile_block(0)
    vb.check_device()
    if dist:
        t = torch.tensor([ms, e2e_ms], dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms, e2e_ms = t.tolist()
    return dict(m=m, ms=ms, e2e_ms=e2e_ms, clocks=clocks, prof=prof, load_s=load_s, h2d=rows * m.C * 4,
                d2h=rows * m.C * 4, launches=n_launch / args.steps, dist=dist, n_launch_timed=n_launch,
                rows=rows)


def halo_ms_per_rank(prof, dist):
    """Milliseconds each rank spent in the halo records (pack, NCCL exchange including the wait for
    the slowest peer, unpack) of its profiled pass; rank 0 gets the list."""
    own = round(sum(r["ms"] for r in prof if r["name"].startswith("halo")), 3)
    if not dist:
        return [own]
    out = [None] * dist.get_world_size()
    dist.all_gather_object(out, own)
    return out


TRAFFIC = os.path.join(HERE, "profiles", "traffic.json")


def proc_gathered_bytes(workload, C):
    """K|V bytes the processor attention gathers per launch, one 2C-wide fp16 row per edge (E * 2C * 2):
    the L2-reuse figure reported beside the compulsory bytes."""
    from varda_b200 import safetensors as st
    mp, _ = model_paths("c1" if workload == "c4" else workload)
    return int(st.read(mp)[0]["graph.proc.edge_index"].shape[1]) * 2 * int(C) * 2


def traffic_for(kind, records):
    """DRAM bytes (read + write) per launch of a kernel class, averaged over the class's launches in
    `records`, from the single-kernel ncu captures in profiles/traffic.json scaled to each launch as its
    `method` says; (None, None) when a launch has no capture to scale."""
    if not os.path.exists(TRAFFIC):
        return None, None
    d = json.load(open(TRAFFIC))
    ent = d.get(kind)
    if ent is None or not records:
        return None, None
    total = 0.0
    if kind == "gemm_tc":
        for r in records:
            f = dict(kv.split("=") for kv in r["name"].split(" ")[1:] if "=" in kv)  # ("+ln": LayerNorm folded in)
            sh = ent["shapes"].get(f"N={f['N']} K={f['K']} epi={f['epi']}")
            M, N, K = int(f["M"]), int(f["N"]), int(f["K"])
            if sh is None:  # a shape without a capture (the K = 4 embeddings): its algorithmic bytes
                total += 2 * (M * K + N * K + M * N * (2 if f["epi"] == "2" else 1))
                continue
            total += sh["weight"] + (sh["read"] - sh["weight"]) * M / ent["M"] + M * N * 2
    else:
        for r in records:
            total += (ent["read"] + ent["write"]) * r["bytes"] / ent["compulsory"]
    return int(total / len(records)), f"{ent.get('capture')} ({ent['method']})"


def summarise(prof, pk, src):
    by, recs = {}, {}
    for r in prof:
        cls = r["name"].split(" ")[0]
        if r["name"].startswith("attention"):
            cls = r["name"]
        d = by.setdefault(cls, {"ms": 0.0, "flop": 0.0, "bytes": 0.0, "n": 0})
        d["ms"] += r["ms"]
        d["flop"] += r["flop"]
        d["bytes"] += r["bytes"]
        d["n"] += 1
        recs.setdefault(cls, []).append(r)
    total = sum(d["ms"] for d in by.values())
    # the dominant compute kernel class (halo_* records of a sharded run are communication and waits)
    dom = max((k for k in by if not k.startswith("halo")), key=lambda k: by[k]["ms"])
    d = by[dom]
    tr, tr_src = traffic_for(dom, recs.get(dom))
    if d["flop"] > 0:
        ach = d["flop"] / (d["ms"] * 1e-3) / 1e12
        peak = pk["bf16_tflops_sustained"]
        roof = {"kernel": dom, "bound": "tensor", "achieved": round(ach, 1), "peak": peak, "unit": "TFLOP/s",
                "frac": round(ach / peak, 4), "traffic": tr, "launches_per_step": d["n"],
                "share": round(d["ms"] / total, 4), "peak_source": f"{src} (sustained bf16, kernel inside a long step)",
                "traffic_source": tr_src, "flop_per_launch": d["flop"] / d["n"]}
    else:
        ach = d["bytes"] / (d["ms"] * 1e-3) / 1e9
        peak = pk["hbm_gbs"]
        roof = {"kernel": dom, "bound": "hbm", "achieved": round(ach, 1), "peak": peak, "unit": "GB/s",
                "frac": round(ach / peak, 4), "traffic": tr, "launches_per_step": d["n"],
                "share": round(d["ms"] / total, 4), "peak_source": src, "traffic_source": tr_src}
    att = by.get("attention proc")
    edge = None
    if att:
        per = att["ms"] / att["n"]
        gbs = att["bytes"] / (att["ms"] * 1e-3) / 1e9
        atr, atr_src = traffic_for("attention proc", recs.get("attention proc"))
        edge = {"kernel": "attention proc", "bound": "hbm", "ms_per_launch": round(per, 4),
                "bytes_per_launch": att["bytes"] / att["n"], "achieved": round(gbs, 1), "peak": pk["hbm_gbs"],
                "unit": "GB/s", "frac": round(gbs / pk["hbm_gbs"], 4), "traffic": atr,
                "peak_source": src, "traffic_source": atr_src}
    shares = {k: {"ms": round(v["ms"], 3), "share": round(v["ms"] / total, 4), "launches": v["n"]}
              for k, v in sorted(by.items(), key=lambda kv: -kv[1]["ms"])}
    return roof, edge, shares, total


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--workload", default="c1", choices=["c1", "c0", "c2", "c3", "c4"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--profile-out", default=None, help="write the per-launch profile records (JSON) here")
    args = ap.parse_args()
    rank = int(os.environ.get("RANK", 0))
    world = int(os.environ.get("WORLD_SIZE", args.gpus))
    local_rank = int(os.environ.get("LOCAL_RANK", 0))
    if "WORLD_SIZE" not in os.environ and args.gpus > 1:
        raise SystemExit("for --gpus > 1 launch with torch.distributed.run (one process per GPU)")
    config = {"workload": "C1: one predict_step of the full Varda-shaped GraphTransformer forecaster (varda.cpp "
                          "format v3, random-init seeded weights; G=1,688,650 data nodes, H=189,809 hidden, C=1024, "
                          "16 heads, 16 processor blocks, T_in=2, V_in=90, V_out=80)",
              "parallelism": f"graph partition by destination x{world}",
              "l2": "inputs and activations >> 126 MB L2 (no flush needed)"}
    if args.workload == "c0":
        config["workload"] = "C0: icosphere r5/r4 model, C=128"
    if args.workload == "c3":
        config["workload"] = ("C3: one call of the temporal-downscaler shape (C1 graph and width, fp16, two input "
                              "states, 6 output steps of 1,688,650 x 80)")
    pk, src = peaks()
    metric = "ms/predict_step fp16 at Varda shape"
    if args.workload == "c4":
        config["workload"] = (f"C4: {args.steps}-step autoregressive rollout of C1 in fp16 (CUDA graph per step, "
                              "synthetic sin/cos forcings replayed from the host, outputs streamed back)")
        metric = "ms/rollout step fp16 at Varda shape"
    if args.workload == "c2":
        config["workload"] = ("C2: one isolated processor block, fp16 (LN_dst + q|k|v|self GEMM + edge attention + "
                              "proj/residual + LN + MLP), H=189,809 hidden rows, 2,561,682 edges (in-degree 11-54), "
                              "U[0,1) edge attributes, C=1024, 16 heads of 64, N(0,1) node features")
        metric = "ms/processor block fp16 at C2 shape"

    if args.impl == "reference" and args.workload == "c2":
        if rank != 0:
            return
        times, threads, hs = reference_cpu_c2(args.steps, args.warmup)
        v = statistics.median(times) * 1000
        line = {"impl": "reference", "metric": metric, "value": round(v, 2), "unit": "ms", "n_gpus": world,
                "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(v, 2), "higher_is_better": False,
                "scaling": "strong", "vs_baseline": None, "dtype": "f32", "data": "synthetic (seeded)",
                "config": config,
                "cpu_baseline": {"value": round(v, 2), "unit": "ms", "cores": threads, "kind": "reference",
                                 "sample": f"reference CPU fp32 backend (oracle/_ref/ref_dump) on 1/8 of the C2 rows "
                                           f"({hs} rows): (3-block step - 1-block step) / 2, x {189809 / hs:.3f}; "
                                           f"median of {len(times)}"},
                "e2e": {"value": round(v, 2), "unit": "ms", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
        print(json.dumps(line), flush=True)
        return
    if args.impl == "reference":
        if rank != 0:
            return
        times, threads, f = reference_cpu(args.steps, args.warmup)
        v = statistics.median(times) * f * 1000
        line = {"impl": "reference", "metric": metric, "value": round(v, 2), "unit": "ms", "n_gpus": world,
                "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(v, 2), "higher_is_better": False,
                "scaling": "strong", "vs_baseline": None, "dtype": "f32", "data": "synthetic (seeded)",
                "config": config,
                "cpu_baseline": {"value": round(v, 2), "unit": "ms", "cores": threads, "kind": "reference",
                                 "sample": f"reference CPU fp32 backend (oracle/_ref/ref_dump, unmodified sources) on "
                                           f"the C1 architecture with 1/{f} of its nodes (G={1688650 // f}, "
                                           f"H={189809 // f}, same per-node edge counts); median of {len(times)} "
                                           f"steps x {f}"},
                "e2e": {"value": round(v, 2), "unit": "ms", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
        print(json.dumps(line), flush=True)
        return

    if args.workload == "c4":
        args.workload = "c1"  # the rollout runs the C1 model
        r = run_rollout(args, rank, world, local_rank)
        args.workload = "c4"
    elif args.workload == "c2":
        r = run_c2(args, rank, world, local_rank)
    else:
        r = run_ours(args, rank, world, local_rank)
    halo = halo_ms_per_rank(r["prof"], r["dist"]) if world > 1 else None
    roof, edge, shares, prof_total = summarise(r["prof"], pk, src)
    if edge is not None and world == 1:
        try:  # secondary figure: never in the way of the bench line
            gb = proc_gathered_bytes(args.workload, r["m"].C)
            edge["gathered_bytes_per_launch"] = gb
            edge["gathered_gbs"] = round(gb / (edge["ms_per_launch"] * 1e-3) / 1e9, 1)
        except Exception as e:
            log(f"bench: gathered bytes unavailable ({e})")
    if args.profile_out and rank == 0:
        with open(args.profile_out, "w") as fh:
            json.dump(r["prof"], fh, indent=0)
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline and args.workload == "c2":
        try:
            times, threads, hs = reference_cpu_c2(2, 1)
            cpu = {"value": round(statistics.median(times) * 1000, 1), "unit": "ms", "cores": threads,
                   "kind": "reference", "sample": f"reference CPU fp32 backend (oracle/_ref/ref_dump) per processor "
                   f"block on 1/8 of the C2 rows ({hs}): (3-block - 1-block step) / 2, scaled by rows"}
        except Exception as e:
            cpu = {"value": None, "unit": "ms", "error": str(e)[:200]}
    if rank == 0 and world == 1 and not args.no_cpu_baseline and args.workload in ("c1", "c4"):
        try:
            times, threads, f = reference_cpu(2, 1)
            v = statistics.median(times) * f * 1000
            cpu = {"value": round(v, 1), "unit": "ms", "cores": threads, "kind": "reference",
                   "sample": f"reference CPU fp32 backend (oracle/_ref/ref_dump) on the C1 architecture with 1/{f} of "
                             f"its nodes, median of {len(times)} steps x {f}"}
        except Exception as e:  # the baseline is reported, never the product
            cpu = {"value": None, "unit": "ms", "error": str(e)[:200]}
    if rank == 0:
        line = {"metric": metric, "value": round(r["ms"], 3), "unit": "ms", "n_gpus": world, "steps": args.steps,
                "warmup": args.warmup, "ms_per_step": round(r["ms"], 3), "higher_is_better": False,
                "scaling": "strong", "vs_baseline": None, "dtype": "f16", "data": "synthetic (seeded graph, inputs "
                "and random-init weights)", "config": config, "roofline": roof, "edge_attention": edge,
                "cpu_baseline": cpu, "clocks": r["clocks"],
                "e2e": {"value": round(r["e2e_ms"], 3), "unit": "ms", "h2d_bytes_per_step": int(r["h2d"]),
                        "d2h_bytes_per_step": int(r["d2h"])},
                "gpu_launches": int(r["launches"] * args.steps),
                "kernel_shares": shares, "profiled_forward_ms": round(prof_total, 3), "load_s": round(r["load_s"], 1)}
        if "step_ms" in r:
            line["rollout"] = {"step_ms": r["step_ms"], "wall_s": round(r["wall_s"], 3)}
        if halo is not None:
            line["halo_ms_per_rank"] = halo
        if args.workload == "c2":
            line["gpu_launches"] = int(round(r["launches"] * args.steps))
        print(json.dumps(line), flush=True)
    if r["dist"]:
        r["dist"].barrier()
        r["dist"].destroy_process_group()


if __name__ == "__main__":
    main()
