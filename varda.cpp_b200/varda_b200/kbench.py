"""Kernel microbenchmarks through the C ABI (CUDA events on the launching stream, after warm-up).

    python -m varda_b200.kbench gemm --M 189809 --N 4096 --K 1024 --epi 1 [--engine 2] [--iters 20] [--library]
    python -m varda_b200.kbench attention [--config c2] [--dtype fp16] [--impl tc,tiled,gather] [--iters 20]

`attention --config c2` is the benchmark's config C2, the isolated processor graph-attention block: the
hidden graph of C1 (189,809 nodes, ~2.6M directed multi-scale edges in CSR by destination), C=1024,
16 heads of 64, 3-dim edge attributes uniform[0,1], node features N(0,1), seeded. q, k, v and x_r
are column slices of one [H, 4C] buffer as in the processor block. Reported: ms per launch, and the
compulsory bytes per launch (q, x_r, out per destination, k and v per source, 16 bytes per edge,
row_ptr, edge weights) divided by it.
"""
from __future__ import annotations

import argparse
import json
import math
import os
import sys

import numpy as np

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
import varda_b200 as vb  # noqa: E402


def _peaks():
    p = os.path.join(os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__)))),
                     "MEASURED_PEAKS.json")
    return json.load(open(p)) if os.path.exists(p) else {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0}


def time_launches(fn, iters, warmup=3):
    import torch
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(iters):
        fn()
    e1.record()
    torch.cuda.synchronize()
    vb.check_device()
    return e0.elapsed_time(e1) / iters


def gemm(a):
    import torch
    g = torch.Generator(device="cuda").manual_seed(0)
    A = torch.randn(a.M, a.K, device="cuda", generator=g).half()
    W = (torch.randn(a.N, a.K, device="cuda", generator=g) / math.sqrt(a.K)).half()
    b = torch.randn(a.N, device="cuda", generator=g).half()
    R = torch.randn(a.M, a.N, device="cuda", generator=g).half() if a.epi == 2 else None
    Y = torch.empty(a.M, a.N, device="cuda", dtype=torch.float16)
    s = torch.cuda.current_stream().cuda_stream
    fn = lambda: vb.gemm(vb.FP16, a.engine, A, a.K, W, a.K, b, Y, a.N, R, a.N, a.M, a.N, a.K, a.epi, stream=s)  # noqa
    if a.ln == "stats":  # + the output rows' LayerNorm records
        st = torch.empty(a.M, a.N // vb.ln_segment_width(a.N), 2, device="cuda")
        fn = lambda: vb.gemm_ln(A, a.K, W, a.K, b, Y, a.N, R, a.N, a.M, a.N, a.K, a.epi, st_out=st, stream=s)  # noqa
    elif a.ln == "fold":  # a LayerNorm over A's rows folded into W and b
        segw = vb.ln_segment_width(a.K)
        st = torch.empty(a.M, a.K // segw, 2, device="cuda")
        cs = torch.empty(a.N, device="cuda")
        ones = torch.ones(a.K, device="cuda")
        vb.fold_layernorm(W, a.K, a.N, a.K, ones, None, b, cs, stream=s)
        vb.row_seg_stats(A, a.K, a.M, a.K, segw, st, stream=s)
        fn = lambda: vb.gemm_ln(A, a.K, W, a.K, b, Y, a.N, None, 0, a.M, a.N, a.K, a.epi, st_in=st, colsum=cs,  # noqa
                                nseg_in=a.K // segw, segw_in=segw, eps=1e-5, stream=s)
    pk = _peaks()
    if a.library:  # the library GEMM (cuBLAS through torch.matmul, fp16, no fused epilogue) on the same shape
        ms = time_launches(lambda: torch.matmul(A, W.t(), out=Y), a.iters, a.warmup)
        tf = 2.0 * a.M * a.N * a.K / (ms * 1e-3) / 1e12
        print(json.dumps({"kernel": "library matmul (cuBLAS)", "M": a.M, "N": a.N, "K": a.K, "ms": round(ms, 4),
                          "tflops": round(tf, 1), "frac_of_burst": round(tf / pk["bf16_tflops"], 3)}))
    # --modes: comma-separated CTA-pair / tile-order settings timed one after another in this process
    # (pair|single)_(dyn|static) -> VB_GEMM_PAIR, VB_GEMM_SCHED; default: the library's defaults
    for mode in (a.modes.split(",") if a.modes else [""]):
        if mode:
            cta, order = mode.split("_")
            os.environ["VB_GEMM_PAIR"] = "1" if cta == "pair" else "0"
            os.environ["VB_GEMM_SCHED"] = "1" if order == "dyn" else "0"
        ms = time_launches(fn, a.iters, a.warmup)
        tf = 2.0 * a.M * a.N * a.K / (ms * 1e-3) / 1e12
        print(json.dumps({"kernel": "gemm", "M": a.M, "N": a.N, "K": a.K, "epi": a.epi, "ln": a.ln,
                          "engine": a.engine, "mode": mode or "default", "ms": round(ms, 4), "tflops": round(tf, 1),
                          "frac_of_burst": round(tf / pk["bf16_tflops"], 3)}))


def c2_graph():
    from varda_b200 import synth
    hidden, proc, attr = synth.graph_c2()
    return len(hidden), np.ascontiguousarray(proc.T), attr


def attention(a):
    import torch
    dt = vb.FP16 if a.dtype == "fp16" else vb.FP32
    T = torch.float16 if dt == vb.FP16 else torch.float32
    H, ei, ea = c2_graph()
    rp, src, _, at = vb.build_csr(ei, ea, H, H)
    edges = vb.pack_edges(src, at, round_fp16=dt == vb.FP16)
    C, heads = 1024, 16
    g = torch.Generator(device="cuda").manual_seed(1)
    qkvs = torch.randn(H, 4 * C, device="cuda", generator=g).to(T)
    w4 = torch.zeros(4, C, device="cuda")
    w4[:3] = torch.randn(3, C, device="cuda", generator=g) * 0.3
    w4[3] = torch.randn(C, device="cuda", generator=g) * 0.1
    d_rp = torch.from_numpy(rp).cuda()
    d_ed = torch.from_numpy(edges).cuda()
    out = torch.empty(H, C, device="cuda", dtype=T)
    s = torch.cuda.current_stream().cuda_stream
    q, k, v, xr = (qkvs[:, i * C:] for i in range(4))
    E = len(src)
    es = 2 if dt == vb.FP16 else 4
    byt = es * C * (3.0 * H + 2.0 * H) + 16.0 * E + 4.0 * (H + 1) + 16.0 * C
    pk = _peaks()
    for impl in a.impl.split(","):
        if impl in ("tiled", "tc"):
            tiles = vb.Tiles(rp, src, at, H, C // heads, kind=vb.Tiles.TC if impl == "tc" else vb.Tiles.SMEM)
            fn = lambda: tiles.attention(0, H, q, 4 * C, k, v, 4 * C, xr, 4 * C, out, C, w4, C, heads,  # noqa
                                         C // heads, stream=s)
        else:
            fn = lambda: vb.attention(dt, d_rp, d_ed, 0, H, q, 4 * C, k, v, 4 * C, xr, 4 * C, out, C, w4, C,  # noqa
                                      heads, C // heads, stream=s)
        ms = time_launches(fn, a.iters, a.warmup)
        gbs = byt / (ms * 1e-3) / 1e9
        print(json.dumps({"kernel": "attention", "impl": impl, "config": "c2", "dtype": a.dtype, "H": H, "E": E,
                          "ms": round(ms, 4), "bytes": byt, "gbs": round(gbs, 1),
                          "frac_of_hbm": round(gbs / pk["hbm_gbs"], 4), "gathered_bytes": 2.0 * E * C * es}),
              flush=True)


def main():
    ap = argparse.ArgumentParser()
    sub = ap.add_subparsers(dest="cmd", required=True)
    g = sub.add_parser("gemm")
    g.add_argument("--M", type=int, default=189809)
    g.add_argument("--N", type=int, default=4096)
    g.add_argument("--K", type=int, default=1024)
    g.add_argument("--epi", type=int, default=0)
    g.add_argument("--engine", type=int, default=2)
    g.add_argument("--iters", type=int, default=20)
    g.add_argument("--warmup", type=int, default=3)
    g.add_argument("--modes", default="", help="e.g. pair_dyn,pair_static,single_dyn,single_static")
    g.add_argument("--library", action="store_true", help="also time cuBLAS (torch.matmul) on the shape")
    g.add_argument("--ln", default="none", choices=["none", "stats", "fold"],
                   help="LayerNorm fusion: write the output's records, or apply an LN of A folded into W")
    t = sub.add_parser("attention")
    t.add_argument("--config", default="c2")
    t.add_argument("--dtype", default="fp16")
    t.add_argument("--impl", default="tc", help="comma-separated: tc, tiled, gather")
    t.add_argument("--iters", type=int, default=20)
    t.add_argument("--warmup", type=int, default=3)
    a = ap.parse_args()
    {"gemm": gemm, "attention": attention}[a.cmd](a)


if __name__ == "__main__":
    main()
