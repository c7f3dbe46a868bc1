"""Data-parallel tests.

CPU (gloo, world size 2): the data-parallel arithmetic the trainer relies on — averaging the
ranks' gradients of equal-sized micro-batches gives the full batch's gradient (the loss is a
mean over lanes), and clip + AdamW on the averaged gradient equals the single-process step;
and failure detection: a rank that dies makes the survivor's next collective fail within the
process-group timeout instead of hanging.

GPU (>= 2 devices): tests/dp_worker.py under torchrun, two ranks training through the C++
trainer with its NCCL bucketed all-reduce, against the oracle's full-batch step.
"""
import os
import socket
import subprocess
import sys
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parent.parent
ADAM = dict(learning_rate=1e-3, beta1=0.9, beta2=0.95, eps=1e-8, weight_decay=0.1)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _dp_math_worker(rank, world, port, out_dir):
    import torch
    import torch.distributed as dist
    sys.path.insert(0, str(ROOT))
    from oracle import veda_oracle as O
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank,
                            world_size=world)
    cfg = O.ModelConfig(vocab=64, hidden=32, intermediate=48, layers=1, heads=4, kv_heads=2,
                        head_dim=8, eps=1e-6, theta=1e4)
    params = O.init_params(cfg, 1)
    ids, tg = O.synthetic_batch(cfg, 2 * world, 8, 1)      # the global batch
    mine = slice(2 * rank, 2 * rank + 2)                    # this rank's micro-batch
    _, grads = O.forward_backward(cfg, params, ids[mine], tg[mine])
    flat = torch.from_numpy(np.concatenate([g.ravel() for g in grads]).astype(np.float64))
    dist.all_reduce(flat)                                   # the trainer's sum ...
    flat /= world                                           # ... and its 1/world
    if rank == 0:
        np.save(Path(out_dir) / "avg.npy", flat.numpy())
    dist.barrier()
    dist.destroy_process_group()


@pytest.mark.timeout(300)
def test_gloo_two_ranks_average_equals_full_batch(tmp_path):
    import torch.multiprocessing as mp
    from oracle import veda_oracle as O
    port = _free_port()
    mp.spawn(_dp_math_worker, args=(2, port, str(tmp_path)), nprocs=2, join=True)
    avg = np.load(tmp_path / "avg.npy")
    cfg = O.ModelConfig(vocab=64, hidden=32, intermediate=48, layers=1, heads=4, kv_heads=2,
                        head_dim=8, eps=1e-6, theta=1e4)
    params = O.init_params(cfg, 1)
    ids, tg = O.synthetic_batch(cfg, 4, 8, 1)
    _, full = O.forward_backward(cfg, params, ids, tg)
    full = np.concatenate([g.ravel() for g in full])
    assert O.max_abs_rel(avg, full) < 1e-5
    # clip + AdamW on the averaged gradient: the same update on every rank as one process
    p1 = [p.copy() for p in params]
    p2 = [p.copy() for p in params]
    at, ga = 0, []
    for p in params:
        ga.append(avg[at:at + p.size].reshape(p.shape).astype(np.float32))
        at += p.size
    gf = [g.copy() for g in O.forward_backward(cfg, params, ids, tg)[1]]
    O.clip_gradient_norm(ga, 1.0)
    O.clip_gradient_norm(gf, 1.0)
    O.AdamW(p1, O.AdamWConfig(**ADAM)).step(ga)
    O.AdamW(p2, O.AdamWConfig(**ADAM)).step(gf)
    for a, b in zip(p1, p2):
        assert O.max_abs_rel(a, b) < 1e-3


def _failure_worker(rank, world, port, out_dir):
    import datetime
    import time
    import torch
    import torch.distributed as dist
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank,
                            world_size=world, timeout=datetime.timedelta(seconds=5))
    t = torch.ones(4)
    dist.all_reduce(t)                      # one healthy step
    if rank == 1:
        os._exit(0)                         # the rank leaves between steps, nothing in flight
    start = time.time()
    try:
        dist.all_reduce(t)                  # the survivor's next collective
        outcome = "completed"
    except Exception as e:  # noqa: BLE001
        outcome = f"error: {type(e).__name__}"
    (Path(out_dir) / "outcome.txt").write_text(f"{outcome} after {time.time() - start:.1f}s")
    os._exit(0)


@pytest.mark.timeout(120)
def test_gloo_dead_rank_is_detected_not_hung(tmp_path):
    import torch.multiprocessing as mp
    port = _free_port()
    ctx = mp.start_processes(_failure_worker, args=(2, port, str(tmp_path)), nprocs=2,
                             join=False, start_method="spawn")
    for p in ctx.processes:
        p.join(timeout=90)
    for p in ctx.processes:
        if p.is_alive():
            p.kill()
    outcome = (tmp_path / "outcome.txt").read_text()
    assert outcome.startswith("error"), outcome
    assert float(outcome.split("after ")[1].rstrip("s")) < 60


@pytest.mark.gpu
@pytest.mark.timeout(900)
def test_nccl_two_gpus_match_full_batch():
    import torch
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    env = dict(os.environ, NCCL_NVLS_ENABLE="0", PYTHONPATH=str(ROOT))
    cmd = ["timeout", "-k", "30", "600", sys.executable, "-m", "torch.distributed.run",
           "--nnodes=1", "--nproc-per-node", "2", "--master-addr", "127.0.0.1",
           "--master-port", str(_free_port()), str(ROOT / "tests" / "dp_worker.py")]
    r = subprocess.run(cmd, capture_output=True, text=True, env=env, cwd=str(ROOT))
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-3000:]
    assert "DP OK" in r.stdout, r.stdout[-2000:]
    assert "SHARDED OK" in r.stdout, r.stdout[-2000:]


@pytest.mark.gpu
@pytest.mark.timeout(600)
def test_nccl_two_gpus_lost_peer_is_detected_and_aborted():
    """A rank leaves between steps; the survivor learns of it on the host, aborts its NCCL
    communicator (nothing in flight), gets an error from its next step instead of a hang, and
    keeps a working CUDA context. NVLS is off (no multicast memory bound to the leaving rank)."""
    import torch
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    env = dict(os.environ, NCCL_NVLS_ENABLE="0", PYTHONPATH=str(ROOT), VEDA_DP_MODE="lost_peer")
    cmd = ["timeout", "-k", "30", "300", sys.executable, "-m", "torch.distributed.run",
           "--nnodes=1", "--nproc-per-node", "2", "--master-addr", "127.0.0.1",
           "--master-port", str(_free_port()), str(ROOT / "tests" / "dp_worker.py")]
    r = subprocess.run(cmd, capture_output=True, text=True, env=env, cwd=str(ROOT))
    assert "LOST PEER OK" in r.stdout, r.stdout[-3000:] + r.stderr[-3000:]


@pytest.mark.gpu
@pytest.mark.timeout(900)
def test_nccl_two_gpus_graph_replay_matches_eager(tmp_path):
    """The data-parallel steps captured into CUDA graphs (VEDA_DP_GRAPH=1; NCCL calls inside the
    graph) give the same weights, bit for bit, as the eager steps."""
    import torch
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    results = []
    for graph in ("0", "1"):
        out = tmp_path / f"w{graph}.npy"
        env = dict(os.environ, NCCL_NVLS_ENABLE="0", PYTHONPATH=str(ROOT), VEDA_DP_GRAPH=graph,
                   VEDA_DP_OUT=str(out))
        cmd = ["timeout", "-k", "30", "600", sys.executable, "-m", "torch.distributed.run",
               "--nnodes=1", "--nproc-per-node", "2", "--master-addr", "127.0.0.1",
               "--master-port", str(_free_port()), str(ROOT / "tests" / "dp_worker.py")]
        r = subprocess.run(cmd, capture_output=True, text=True, env=env, cwd=str(ROOT))
        assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-3000:]
        results.append(np.load(out))
    assert np.array_equal(results[0], results[1])
