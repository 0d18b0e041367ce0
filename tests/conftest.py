import os
import sys

import numpy as np
import pytest

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, os.path.join(REPO, "varda.cpp_b200"))
sys.path.insert(0, os.path.join(REPO, "oracle"))
GOLDEN = os.path.join(REPO, "tests", "golden")
# The reference checkout (sources of varda.cpp) when this container has one: $VARDA_REFERENCE, else a
# `reference` directory beside the repository. Tests that need it skip when it is absent (the GPU box).
REFERENCE = os.environ.get("VARDA_REFERENCE") or os.path.join(os.path.dirname(REPO), "reference")


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (runs the CUDA library)")


def have_gpu():
    try:
        import torch
        return torch.cuda.is_available()
    except Exception:
        return False


@pytest.fixture(scope="session")
def model_dir(tmp_path_factory):
    return str(tmp_path_factory.mktemp("models"))


_MODELS = {}


@pytest.fixture(scope="session")
def seeded_model(model_dir):
    """seeded_model(name) -> (model path, input path), generated once per session and checked
    against the sha256 recorded with the golden fixture."""
    from varda_b200 import synth

    def get(name):
        if name not in _MODELS:
            mp, xp = synth.generate(name, model_dir)
            for kind in ("golden", "rollout", "sampled"):
                g = os.path.join(GOLDEN, f"{name}.{kind}.npz")
                if os.path.exists(g):
                    z = np.load(g)
                    assert synth.sha256_file(mp) == bytes(z["__model_sha256__"]).decode(), f"{name}: model drifted"
                    assert synth.sha256_file(xp) == bytes(z["__input_sha256__"]).decode(), f"{name}: input drifted"
            _MODELS[name] = (mp, xp)
        return _MODELS[name]

    return get


def rollout_golden(name):
    z = np.load(os.path.join(GOLDEN, f"{name}.rollout.npz"))
    return {k: z[k] for k in z.files if not k.startswith("__")}


def golden(name):
    z = np.load(os.path.join(GOLDEN, f"{name}.golden.npz"))
    return {k: z[k] for k in z.files if not k.startswith("__")}
