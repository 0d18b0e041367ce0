"""Multi-GPU destination partition on B200s (skipped with fewer than 2 visible GPUs): one process per
GPU, NCCL halo exchange; every rank's output rows (of predict_step, and of the isolated processor
block vb_processor_block with its K|V halo exchange) must be bitwise equal to the single-GPU result
(the partition keeps every destination's edge order and every GEMM row's arithmetic, and, on graphs of
at least 128 hidden rows per GPU, the tensor-core attention's tiles), with and without the encoder
split. On smaller graphs the hidden ranges are not on the tiles' 64-row grid, so those models run the
processor on the gather kernel here (VB_ATT_TC=none)."""
import os

import numpy as np
import pytest

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")


def _worker(rank, world, mp, xp, dtype, uid_path, out_dir):
    import time
    import varda_b200 as vb
    from varda_b200 import safetensors as st
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    torch.cuda.set_device(rank)
    if rank == 0:
        with open(uid_path + ".tmp", "wb") as f:
            f.write(vb.nccl_unique_id())
        os.replace(uid_path + ".tmp", uid_path)
    t0 = time.time()
    while not os.path.exists(uid_path):
        if time.time() - t0 > 60:
            raise TimeoutError("no NCCL id")
        time.sleep(0.05)
    uid = open(uid_path, "rb").read()
    m = vb.Model.load_sharded(mp, rank, world, uid, precision=dtype, cuda_device=rank)
    x = np.array(st.read(xp)[0]["in.x"])
    ys = []
    for _ in range(3):  # eager, capture + replay, replay
        y = np.full(m.output_shape, np.nan, np.float32)
        m.predict_step(x, y)
        ys.append(y[:, :, :, m.data_lo:m.data_hi].copy())
    zb, _ = m.processor_block(0, _block_input(m)[m.hidden_lo:m.hidden_hi], True)  # the isolated block (C2)
    vb.check_device()
    np.savez(os.path.join(out_dir, f"r{rank}.npz"), y0=ys[0], y1=ys[1], y2=ys[2], lo=m.data_lo, hi=m.data_hi,
             zb=zb, hlo=m.hidden_lo, hhi=m.hidden_hi)
    m.free()


def _block_input(m):
    return np.random.default_rng(5).standard_normal((m.H, m.C), dtype=np.float32)


def _single(mp, xp, dtype, out):
    import varda_b200 as vb
    from varda_b200 import safetensors as st
    torch.cuda.set_device(0)
    m = vb.Model.load(mp, precision=dtype)
    y = m.predict_step(np.array(st.read(xp)[0]["in.x"]))
    np.save(out, y)
    np.save(out + ".block.npy", m.processor_block(0, _block_input(m), True)[0])


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
@pytest.mark.parametrize("name,enc_split", [("c0", 0), ("t256", 0), ("c0", 1), ("t1024", 1), ("c1s", 0), ("c1s", 1)])
@pytest.mark.parametrize("dtype", [0, 1])
def test_sharded_equals_single_gpu(name, enc_split, dtype, seeded_model, tmp_path, monkeypatch):
    """enc_split: the encoder on its own hidden ranges (VB_SHARD_ENC=1, the default), its output rows moved to their
    processor owners; c0 and t1024 move rows between ranks at 2-4 GPUs. c1s (C1's widths, 2,965 hidden
    rows) runs its processor on the tensor-core attention (fp16)."""
    import torch.multiprocessing as tmp
    if name == "c1s" and dtype == 0:
        pytest.skip("c1s: the fp16 tensor-core path is what it covers")
    monkeypatch.setenv("VB_SHARD_ENC", str(enc_split))
    mp, xp = seeded_model(name)
    world = min(torch.cuda.device_count(), 4)
    from varda_b200 import safetensors as st
    import json
    H = json.loads(st.read(mp)[1]["config"])["dims"]["n_hidden_nodes"]
    if H < 128 * world:
        monkeypatch.setenv("VB_ATT_TC", "none")
    ctx = tmp.get_context("spawn")
    p = ctx.Process(target=_single, args=(mp, xp, dtype, str(tmp_path / "single.npy")))
    p.start()
    p.join(300)
    assert p.exitcode == 0
    y1 = np.load(tmp_path / "single.npy")
    zb1 = np.load(str(tmp_path / "single.npy") + ".block.npy")
    tmp.start_processes(_worker, args=(world, mp, xp, dtype, str(tmp_path / "uid"), str(tmp_path)), nprocs=world,
                        join=True, start_method="spawn")
    covered = hidden = 0
    for r in range(world):
        z = np.load(tmp_path / f"r{r}.npz")
        lo, hi = int(z["lo"]), int(z["hi"])
        covered += hi - lo
        for k in ("y0", "y1", "y2"):
            assert np.array_equal(z[k], y1[:, :, :, lo:hi]), f"rank {r} {k} differs from one GPU"
        hlo, hhi = int(z["hlo"]), int(z["hhi"])
        hidden += hhi - hlo
        assert np.array_equal(z["zb"], zb1[hlo:hhi]), f"rank {r}: the isolated block differs from one GPU"
    assert covered == y1.shape[3] and hidden == zb1.shape[0]


def _rollout_worker(rank, world, mp, xp, fp, dtype, uid_path, out_dir):
    import time
    import varda_b200 as vb
    from varda_b200 import safetensors as st
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    torch.cuda.set_device(rank)
    if rank == 0:
        with open(uid_path + ".tmp", "wb") as f:
            f.write(vb.nccl_unique_id())
        os.replace(uid_path + ".tmp", uid_path)
    t0 = time.time()
    while not os.path.exists(uid_path):
        if time.time() - t0 > 60:
            raise TimeoutError("no NCCL id")
        time.sleep(0.05)
    m = vb.Model.load_sharded(mp, rank, world, open(uid_path, "rb").read(), precision=dtype, cuda_device=rank)
    x = np.array(st.read(xp)[0]["in.x"])
    f = np.load(fp)
    y, _ = m.rollout(x, f.shape[0] + 1, f)
    vb.check_device()
    np.savez(os.path.join(out_dir, f"ro{rank}.npz"), y=y[:, m.data_lo:m.data_hi], lo=m.data_lo, hi=m.data_hi)
    m.free()


def _rollout_single(mp, xp, fp, dtype, out):
    import varda_b200 as vb
    from varda_b200 import safetensors as st
    torch.cuda.set_device(0)
    m = vb.Model.load(mp, precision=dtype)
    f = np.load(fp)
    y, _ = m.rollout(np.array(st.read(xp)[0]["in.x"]), f.shape[0] + 1, f)
    np.save(out, y)


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
@pytest.mark.parametrize("enc_split", [0, 1])
@pytest.mark.parametrize("dtype", [0, 1])
def test_sharded_rollout_equals_single_gpu(dtype, enc_split, seeded_model, tmp_path, monkeypatch):
    """The rollout's per-step exchange of the encoder-halo rows' outputs: every rank's rows of every
    step bitwise equal to the single-GPU rollout, with and without the encoder's own split."""
    import torch.multiprocessing as tmp
    from conftest import rollout_golden
    monkeypatch.setenv("VB_SHARD_ENC", str(enc_split))
    mp, xp = seeded_model("t256r")
    fp = str(tmp_path / "f.npy")
    np.save(fp, rollout_golden("t256r")["forcings"])
    world = min(torch.cuda.device_count(), 4)
    ctx = tmp.get_context("spawn")
    p = ctx.Process(target=_rollout_single, args=(mp, xp, fp, dtype, str(tmp_path / "single.npy")))
    p.start()
    p.join(300)
    assert p.exitcode == 0
    y1 = np.load(tmp_path / "single.npy")
    tmp.start_processes(_rollout_worker, args=(world, mp, xp, fp, dtype, str(tmp_path / "uid"), str(tmp_path)),
                        nprocs=world, join=True, start_method="spawn")
    covered = 0
    for r in range(world):
        z = np.load(tmp_path / f"ro{r}.npz")
        lo, hi = int(z["lo"]), int(z["hi"])
        covered += hi - lo
        assert np.array_equal(z["y"], y1[:, lo:hi]), f"rank {r} differs from one GPU"
    assert covered == y1.shape[1]


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_two_devices_in_one_process(seeded_model):
    """Models on two devices of one process: kernel attributes and SM counts are set up per device, so
    the second device's launches run as the first's do (same bits)."""
    import varda_b200 as vb
    from varda_b200 import safetensors as st
    mp, xp = seeded_model("t1024")
    x = np.array(st.read(xp)[0]["in.x"])
    ys = []
    for dev in (0, 1):
        m = vb.Model.load(mp, precision=1, cuda_device=dev)
        ys.append(m.predict_step(x))
        m.free()
    vb.check_device()
    assert np.array_equal(ys[0], ys[1])
