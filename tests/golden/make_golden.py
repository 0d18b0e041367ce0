"""Generates the committed golden fixtures of tests/golden/ (run in a container that has the reference
sources and oracle/_ref built; the fixtures then travel, the reference does not).

1. synthetic_pin.json: for the reference's own synthetic models a-h (python/tests/synthetic.py of
   varda.cpp, imported from the reference tree), the sha256 of the model file and the worst
   rel_absmax of this repo's oracle restatement (oracle/oracle.py) against the reference's float64
   goldens, per key.
2. <name>.golden.npz for this repo's seeded models (varda_b200.synth: c0 and the t* parity models):
   contract activations computed by the UNMODIFIED reference CPU backend (oracle/_ref/ref_dump,
   compiled from the reference's sources), the model file's sha256, and the input's sha256.
3. <name>.rollout.npz for the rollout variants of the parity models (t*r: a `forcings` section):
   ROLLOUT_STEPS steps of the reference's host rollout (varda::Rollout::run on the CPU backend,
   oracle/_ref/ref_rollout) with replayed synthetic forcings, both constant sources.
4. <name>.sampled.npz for the benchmark-width models whose activations are too large to keep whole
   (c1s: C1's architecture, 16 blocks of C = 1024, on 1/64 of its nodes): every contract key of the
   reference's hooked predict_step, viewed as rows of its last axis, at SAMPLE_ROWS seeded rows and
   SAMPLE_COLS seeded columns (indices stored beside the values as <key>.rows and <key>.cols).
5. c1.y_sample.npz: the reference's out.y on the full C1 model (one predict_step of its CPU backend,
   `ref_dump --y-out`, about 26 GB of host memory and minutes), at C1_Y_ROWS seeded data nodes, with
   the wall time of that step. Only with --c1-y Y MODEL INPUT: the file such a run wrote, and the
   model and input it ran (synth "c1"; their sha256 are kept to detect drift).

    python tests/golden/make_golden.py [--reference REFERENCE_TREE] [--only NAME ...]
                                       [--c1-y Y MODEL INPUT --c1-step-s S --c1-threads N --c1-rss-gb GB]
"""
from __future__ import annotations

import argparse
import importlib.util
import json
import os
import subprocess
import sys
import tempfile

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, os.path.join(REPO, "varda.cpp_b200"))
sys.path.insert(0, os.path.join(REPO, "oracle"))

from varda_b200 import safetensors as st, synth  # noqa: E402
import oracle  # noqa: E402

MODELS = ["c0", "t128", "t256", "t512", "t768", "t1024", "t384i", "t2048"]
# keys kept in the fixtures (the small ones; [H, C] / [G, C] keys only for small models)
KEEP_ALWAYS = ["dec.out", "out.pre_bound", "out.norm", "out.y"]
KEEP_SMALL = ["enc.out", "latent"]
ROLLOUT_MODELS = ["t256r", "t128r"]
ROLLOUT_STEPS = 4
SAMPLED_MODELS = ["c1s"]
SAMPLE_ROWS = 128
SAMPLE_COLS = 128
C1_Y_ROWS = 8192


def sample_rows(n_rows, k, seed):
    """k distinct row indices of n_rows (all of them when n_rows <= k), ascending; always includes the
    first and the last row."""
    if n_rows <= k:
        return np.arange(n_rows, dtype=np.int64)
    r = np.random.default_rng(seed).choice(n_rows, size=k - 2, replace=False)
    return np.unique(np.concatenate([r, [0, n_rows - 1]])).astype(np.int64)


def sampled_golden(name, work, ref_dump):
    mp, xp = synth.generate(name, work)
    dump = os.path.join(work, f"{name}.dump.safetensors")
    r = subprocess.run([ref_dump, "--model", mp, "--input", xp, "--dump", dump, "--threads", "8"],
                       capture_output=True, text=True, check=True)
    acts, _ = st.read(dump)
    keep = {}
    for i, (k, a) in enumerate(sorted(acts.items())):
        a2 = np.asarray(a, np.float32).reshape(-1, a.shape[-1])
        rows = sample_rows(a2.shape[0], SAMPLE_ROWS, seed=1000 + i)
        cols = sample_rows(a2.shape[1], SAMPLE_COLS, seed=2000 + i)
        keep[k] = a2[rows][:, cols]
        keep[k + ".rows"] = rows
        keep[k + ".cols"] = cols
        keep[k + ".shape"] = np.array(a.shape, np.int64)
    keep["__model_sha256__"] = np.frombuffer(synth.sha256_file(mp).encode(), np.uint8)
    keep["__input_sha256__"] = np.frombuffer(synth.sha256_file(xp).encode(), np.uint8)
    np.savez_compressed(os.path.join(HERE, f"{name}.sampled.npz"), **keep)
    print(f"{name}: reference ref_dump {r.stdout.strip()}; {len(acts)} keys sampled")
    return {}


def c1_y_sample(y_path, model_path, input_path, seconds, threads, peak_rss_gb):
    y = np.asarray(st.read(y_path)[0]["y"], np.float32)  # (1, T_out, 1, G, V_out)
    G = y.shape[3]
    rows = sample_rows(G, C1_Y_ROWS, seed=2024)
    np.savez_compressed(os.path.join(HERE, "c1.y_sample.npz"), rows=rows, y=y[0, :, 0][:, rows],
                        shape=np.array(y.shape, np.int64), step_s=np.float64(seconds),
                        threads=np.int64(threads), peak_rss_gb=np.float64(peak_rss_gb),
                        __model_sha256__=np.frombuffer(synth.sha256_file(model_path).encode(), np.uint8),
                        __input_sha256__=np.frombuffer(synth.sha256_file(input_path).encode(), np.uint8))
    print(f"c1: {len(rows)} of {G} rows of out.y kept")


def pin_synthetic(ref_root, work):
    spec = importlib.util.spec_from_file_location("ref_synthetic", os.path.join(ref_root, "python/tests/synthetic.py"))
    syn = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(syn)
    out = {}
    for name in sorted(syn.CONFIGS):
        syn.generate(name, work)
        mp = os.path.join(work, f"{name}.model.safetensors")
        gold, _ = oracle.read_safetensors(os.path.join(work, f"{name}.golden.safetensors"))
        m = oracle.OracleModel(mp)
        res = {}
        m.predict_step(gold["in.x"], lambda k, a: res.__setitem__(k, oracle.rel_absmax(a, gold[k])))
        out[name] = {"model_sha256": synth.sha256_file(mp), "rel_absmax": res,
                     "worst": max(res.values()), "tolerance_fp32": 1e-5}
        print(f"synthetic {name}: worst {out[name]['worst']:.3e}")
    return out


def ref_golden(name, work, ref_dump):
    mp, xp = synth.generate(name, work)
    dump = os.path.join(work, f"{name}.dump.safetensors")
    r = subprocess.run([ref_dump, "--model", mp, "--input", xp, "--dump", dump, "--threads", "8"],
                       capture_output=True, text=True, check=True)
    acts, _ = st.read(dump)
    keep = {k: np.array(acts[k], np.float32) for k in KEEP_ALWAYS}
    for k in KEEP_SMALL:
        if acts[k].size <= 300_000:
            keep[k] = np.array(acts[k], np.float32)
    # the oracle restatement against the reference, same inputs (printed, and checked by the tests)
    x = st.read(xp)[0]["in.x"]
    om = oracle.OracleModel(mp)
    worst = {}
    om.predict_step(x, lambda k, a: worst.__setitem__(k, oracle.rel_absmax(a, acts[k])))
    keep["__model_sha256__"] = np.frombuffer(synth.sha256_file(mp).encode(), np.uint8)
    keep["__input_sha256__"] = np.frombuffer(synth.sha256_file(xp).encode(), np.uint8)
    np.savez_compressed(os.path.join(HERE, f"{name}.golden.npz"), **keep)
    print(f"{name}: reference ref_dump {r.stdout.strip()} ; oracle vs reference worst {max(worst.values()):.3e}")
    return {k: float(v) for k, v in worst.items()}


def rollout_golden(name, work, ref_rollout):
    mp, xp = synth.generate(name, work)
    x = st.read(xp)[0]["in.x"]
    om = oracle.OracleModel(mp)
    F = len(om.cfg["forcings"]["dynamic_input_index"])
    f = synth.replay_forcings(ROLLOUT_STEPS, om.G, F, om.cfg["forcings"]["timestep_hours"], seed=7)
    rp = os.path.join(work, f"{name}.rollout_in.safetensors")
    st.write(rp, {"in.x": x, "forcings": f}, {"producer": "tests/golden/make_golden.py"})
    keep, worst = {}, {}
    for oldest in (False, True):
        out = os.path.join(work, f"{name}.{int(oldest)}.rollout.safetensors")
        cmd = [ref_rollout, "--model", mp, "--input", rp, "--steps", str(ROLLOUT_STEPS), "--threads", "8",
               "--out", out] + (["--oldest"] if oldest else [])
        r = subprocess.run(cmd, capture_output=True, text=True, check=True)
        y = np.array(st.read(out)[0]["y"], np.float32)
        tag = "oldest" if oldest else "newest"
        keep[f"y_{tag}"] = y
        yo = oracle.rollout(om, x, ROLLOUT_STEPS, f, oldest)
        worst[f"rollout.{tag}"] = max(oracle.rel_absmax(yo[s], y[s]) for s in range(ROLLOUT_STEPS))
        print(f"{name} rollout ({tag}): reference {r.stdout.strip()} ; oracle vs reference "
              f"worst {worst[f'rollout.{tag}']:.3e}")
    keep["forcings"] = f
    keep["__model_sha256__"] = np.frombuffer(synth.sha256_file(mp).encode(), np.uint8)
    keep["__input_sha256__"] = np.frombuffer(synth.sha256_file(xp).encode(), np.uint8)
    np.savez_compressed(os.path.join(HERE, f"{name}.rollout.npz"), **keep)
    return worst


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=os.environ.get("VARDA_REFERENCE")
                    or os.path.join(os.path.dirname(REPO), "reference"),
                    help="the reference checkout ($VARDA_REFERENCE, else `reference` beside the repository)")
    ap.add_argument("--only", nargs="*")
    ap.add_argument("--skip-synthetic", action="store_true")
    ap.add_argument("--c1-y", nargs=3, metavar=("Y", "MODEL", "INPUT"),
                    help="out.y of a full-C1 ref_dump run (--y-out) and the model and input it ran; "
                         "writes c1.y_sample.npz")
    ap.add_argument("--c1-step-s", type=float, default=0.0, help="that run's step wall time (s)")
    ap.add_argument("--c1-threads", type=int, default=0, help="that run's thread count")
    ap.add_argument("--c1-rss-gb", type=float, default=0.0, help="that run's peak resident memory (GB)")
    a = ap.parse_args()
    if a.c1_y:
        c1_y_sample(*a.c1_y, a.c1_step_s, a.c1_threads, a.c1_rss_gb)
        return
    ref_dump = os.path.join(REPO, "oracle", "_ref", "ref_dump")
    if not os.path.exists(ref_dump):
        subprocess.run(["make", "-C", os.path.join(REPO, "oracle"), f"REF={a.reference}"], check=True)
    with tempfile.TemporaryDirectory() as work:
        summary_path = os.path.join(HERE, "oracle_vs_reference.json")
        summary = json.load(open(summary_path)) if os.path.exists(summary_path) else {}
        if not a.skip_synthetic:
            pin = pin_synthetic(a.reference, work)
            with open(os.path.join(HERE, "synthetic_pin.json"), "w") as f:
                json.dump(pin, f, indent=1, sort_keys=True)
        for name in a.only or MODELS + ROLLOUT_MODELS + SAMPLED_MODELS:
            if name in SAMPLED_MODELS:
                sampled_golden(name, work, ref_dump)
                continue
            if name in ROLLOUT_MODELS:
                summary[name] = rollout_golden(name, work, os.path.join(REPO, "oracle", "_ref", "ref_rollout"))
            else:
                summary[name] = ref_golden(name, work, ref_dump)
        with open(summary_path, "w") as f:
            json.dump(summary, f, indent=1, sort_keys=True)


if __name__ == "__main__":
    main()
