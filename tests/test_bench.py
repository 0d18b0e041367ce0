"""The benchmark's host-side bookkeeping, on CPU: how the per-launch profile records of one forward
become the `roofline`, `edge_attention` and `kernel_shares` objects of the JSON line, and the
gathered-bytes figure. No GPU (the records are made up; the GPU run produces them)."""
import os
import sys

import pytest

from conftest import REPO

sys.path.insert(0, REPO)
import bench  # noqa: E402


def records():
    # two GEMM launches, two processor attention launches, one LayerNorm, one halo wait
    return [
        {"name": "gemm_tc M=1000 N=4096 K=1024 epi=0 +ln", "ms": 1.0, "flop": 2e12, "bytes": 0.0},
        {"name": "gemm_tc M=1000 N=1024 K=4096 epi=2", "ms": 1.0, "flop": 1e12, "bytes": 0.0},
        {"name": "attention proc", "ms": 0.5, "flop": 0.0, "bytes": 1e9},
        {"name": "attention proc", "ms": 0.5, "flop": 0.0, "bytes": 1e9},
        {"name": "layernorm", "ms": 0.2, "flop": 0.0, "bytes": 4e8},
        {"name": "halo_exchange", "ms": 5.0, "flop": 0.0, "bytes": 1e6},
    ]


def test_summarise_picks_the_dominant_compute_kernel():
    pk = {"hbm_gbs": 6000.0, "bf16_tflops": 1600.0, "bf16_tflops_sustained": 1500.0}
    roof, edge, shares, total = bench.summarise(records(), pk, "measured")
    # halo_* records are communication and waits, never the dominant kernel
    assert roof["kernel"] == "gemm_tc" and roof["bound"] == "tensor" and roof["unit"] == "TFLOP/s"
    assert roof["achieved"] == pytest.approx(3e12 / 2e-3 / 1e12)  # 1500 TFLOP/s
    assert roof["peak"] == 1500.0 and roof["frac"] == pytest.approx(1.0)
    assert roof["launches_per_step"] == 2 and roof["flop_per_launch"] == pytest.approx(1.5e12)
    assert edge["kernel"] == "attention proc" and edge["bound"] == "hbm"
    assert edge["ms_per_launch"] == pytest.approx(0.5) and edge["bytes_per_launch"] == pytest.approx(1e9)
    assert edge["achieved"] == pytest.approx(2000.0) and edge["frac"] == pytest.approx(2000.0 / 6000.0, abs=1e-4)
    assert total == pytest.approx(8.2)
    assert list(shares)[0] == "halo_exchange" and shares["gemm_tc"]["launches"] == 2
    assert sum(v["share"] for v in shares.values()) == pytest.approx(1.0, abs=1e-3)


def test_summarise_hbm_bound_when_no_flops():
    pk = {"hbm_gbs": 6000.0, "bf16_tflops": 1600.0, "bf16_tflops_sustained": 1500.0}
    recs = [r for r in records() if not r["name"].startswith("gemm")]
    roof, edge, _, _ = bench.summarise(recs, pk, "fallback")
    assert roof["kernel"] == "attention proc" and roof["bound"] == "hbm" and roof["unit"] == "GB/s"
    assert roof["achieved"] == pytest.approx(2000.0) and roof["peak_source"] == "fallback"


def test_peaks_file_is_read():
    pk, src = bench.peaks()
    assert {"hbm_gbs", "bf16_tflops_sustained"} <= set(pk)
    assert src == ("measured" if os.path.exists(os.path.join(REPO, "MEASURED_PEAKS.json")) else "fallback")


def test_gathered_bytes_of_the_processor_attention(tmp_path, monkeypatch):
    """E_proc * 2C * 2 bytes: one fp16 K|V row per processor edge (C0: 20,460 edges, C = 128)."""
    monkeypatch.setattr(bench, "CACHE", str(tmp_path))
    assert bench.proc_gathered_bytes("c0", 128) == 20460 * 2 * 128 * 2


def test_traffic_scales_the_captures_to_each_launch():
    """profiles/traffic.json: a GEMM launch of M rows gets the capture's weight bytes once, its reads per
    row times M and its output once; a shape without a capture its algorithmic bytes; the processor
    attention the capture's traffic in proportion to the launch's compulsory bytes."""
    import json
    d = json.load(open(bench.TRAFFIC))
    sh = d["gemm_tc"]["shapes"]["N=4096 K=1024 epi=0"]
    m0 = d["gemm_tc"]["M"]
    rec = {"name": "gemm_tc M=65536 N=4096 K=1024 epi=0", "ms": 1.0, "flop": 1.0, "bytes": 0.0}
    t, src = bench.traffic_for("gemm_tc", [rec])
    assert t == int(sh["weight"] + (sh["read"] - sh["weight"]) * 65536 / m0 + 65536 * 4096 * 2)
    assert "gemm_tc_dram" in src
    other = {"name": "gemm_tc M=100 N=1024 K=4 epi=0", "ms": 1.0, "flop": 1.0, "bytes": 0.0}
    t2, _ = bench.traffic_for("gemm_tc", [other])
    assert t2 == 2 * (100 * 4 + 1024 * 4 + 100 * 1024)
    a = d["attention proc"]
    att = {"name": "attention proc", "ms": 1.0, "flop": 0.0, "bytes": a["compulsory"] / 2}
    t3, _ = bench.traffic_for("attention proc", [att])
    assert t3 == int((a["read"] + a["write"]) / 2)
    assert bench.traffic_for("layernorm", [att]) == (None, None)


def test_reference_env_names_an_openblas_core_type(monkeypatch):
    monkeypatch.delenv("OPENBLAS_CORETYPE", raising=False)
    env = bench.ref_env()
    flags = open("/proc/cpuinfo").read() if os.path.exists("/proc/cpuinfo") else ""
    if " avx512f" in flags:
        assert env["OPENBLAS_CORETYPE"] == "SkylakeX"
    elif " avx2" in flags:
        assert env["OPENBLAS_CORETYPE"] == "Haswell"
    monkeypatch.setenv("OPENBLAS_CORETYPE", "Zen")
    assert bench.ref_env()["OPENBLAS_CORETYPE"] == "Zen", "a caller's choice is kept"


class _FakeSmi:
    """Stands in for the nvidia-smi sampler process: writes rows into its stdout file on demand."""
    def __init__(self, args, stdout=None, stderr=None):
        self.out = stdout

    def row(self, mhz, cap="Not Active"):
        self.out.write(f"0, {mhz}, 1965, 900.0, 0x0, Not Active, Not Active, Not Active, {cap}\n")
        self.out.flush()

    def terminate(self):
        pass

    def wait(self, timeout=None):
        return 0


def test_clock_sampler_keeps_the_timed_region_rows(monkeypatch):
    """Clocks.start_region waits for the sampler's first row and drops the rows taken before the timed
    region; with no row inside the region the earlier ones are kept (a median of something)."""
    monkeypatch.setattr(bench.subprocess, "Popen", _FakeSmi)
    c = bench.Clocks(0)
    c.p.row(1965)  # idle, before the region
    c.start_region()
    assert c.skip == 1
    c.p.row(1400, "Active")
    c.p.row(1420, "Active")
    r = c.stop()
    assert r["samples"] == 2 and r["sm_mhz"] == 1410 and r["reasons"] == ["sw_power_cap"]
    c = bench.Clocks(0)
    c.p.row(1900)
    c.start_region()
    r = c.stop()
    assert r["samples"] == 1 and r["sm_mhz"] == 1900
