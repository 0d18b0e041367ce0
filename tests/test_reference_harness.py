"""The reference's own parity harness driving this backend (the drop-in proof).

oracle/_ref/b200/varda-parity is the reference's UNMODIFIED apps/varda-parity.cpp, compiled with its
core (config, format, graph, model, CPU backend) and with the CUDA backend taken from libvarda_b200
through include/varda_b200_backend.hpp (oracle/Makefile, target b200apps). It loads the model with
varda::Model::load(path, {Device::CUDA}), runs one hooked predict_step comparing every contract key
with the golden file under the named tolerance table, checks that a hook-free run is bitwise equal
(hook inert) and that the returned y matches out.y.

Models: the reference's synthetic generality suite a-h (python/tests/synthetic.py of the reference,
float64 goldens, tolerances/synthetic-*.json: 1e-5 fp32, 3e-3 fp16), staged under
oracle/_ref/synthetic/ by a container that has the reference sources (make_golden.py does not commit
them: they are several hundred MB). The reference runs this suite for its own CUDA backend in fp32,
fp32 with 128-row decoder chunks, and fp16; so does this test. Skipped when the staged files or the
apps are absent.
"""
import os
import subprocess

import pytest

from conftest import REPO

pytestmark = pytest.mark.gpu
SYN = os.path.join(REPO, "oracle", "_ref", "synthetic")
PARITY = os.path.join(REPO, "oracle", "_ref", "b200", "varda-parity")
MODELS = [m for m in "abcdefgh" if os.path.exists(os.path.join(SYN, f"{m}.model.safetensors"))]


@pytest.mark.skipif(not (os.path.exists(PARITY) and MODELS), reason="reference apps / synthetic suite not staged")
@pytest.mark.parametrize("name", MODELS or ["none"])
@pytest.mark.parametrize("mode", ["fp32", "fp32-chunk128", "fp16"])
def test_reference_varda_parity_on_b200(name, mode):
    prec = "fp16" if mode == "fp16" else "fp32"
    table = "synthetic-fp16" if prec == "fp16" else "synthetic-fp32"
    env = dict(os.environ)
    if mode == "fp32-chunk128":
        env["VB_DEC_CHUNK_ROWS"] = "128"
    r = subprocess.run([PARITY, "--model", os.path.join(SYN, f"{name}.model.safetensors"), "--check",
                        os.path.join(SYN, f"{name}.golden.safetensors") + "=" + table, "--device", "cuda",
                        "--precision", prec, "--tolerances", os.path.join(SYN, f"synthetic-{name}.json")],
                       capture_output=True, text=True, timeout=600, env=env)
    out = r.stdout + r.stderr
    assert r.returncode == 0 and out.strip().endswith("PASS"), out[-3000:]
