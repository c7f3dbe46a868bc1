"""One rank of the 2-GPU data-parallel parity check (launched by tests/test_dp.py under torchrun).

Each rank trains the Qwen3-shaped bf16 decoder through the C++ trainer on its own micro-batch
(B 2 x T 128) with the library's NCCL bucketed all-reduce (small 1 MB buckets, so many are in
flight during the backward). Rank 0 compares the averaged gradient with the oracle's gradient of
the full batch (both micro-batches, B 4) and every rank checks that the updated weights are the
same on both ranks. The same step with the optimizer state sharded across the ranks must give the
same gradients, norm and weights. With VEDA_DP_OUT set, rank 0 saves the sharded trainer's
weights after its three steps there."""
import datetime
import os
import sys
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent.parent
sys.path.insert(0, str(ROOT))


def main():
    import torch
    import torch.distributed as dist
    from oracle import veda_oracle as O
    from veda_b200 import train_abi as TA

    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    local = int(os.environ["LOCAL_RANK"])
    torch.cuda.set_device(local)
    dist.init_process_group("gloo", timeout=datetime.timedelta(seconds=120))
    cfg = O.ModelConfig(vocab=2048, hidden=256, intermediate=512, layers=2, heads=4, kv_heads=2,
                        head_dim=128, eps=1e-6, theta=1e6)
    B, T = 2, 128
    params = O.init_params(cfg, 3, bf16=True)
    ids, tg = O.synthetic_batch(cfg, B * world, T, 7)
    mine = slice(B * rank, B * rank + B)
    t = TA.Trainer(cfg, lr=1e-3, betas=(0.9, 0.95), eps=1e-8, weight_decay=0.1, max_norm=1.0,
                   dtype=1, batch=B, seq_len=T, seed=3)
    t.set_params(np.concatenate([p.ravel() for p in params]))
    uid = [TA.nccl_unique_id() if rank == 0 else None]
    dist.broadcast_object_list(uid, src=0)
    t.init_dp(uid[0], rank, world, 1 << 20)
    loss, norm = t.step_host(ids[mine], tg[mine])
    grads_sum = t.get_grads()
    w = t.get_params()
    # identical weights on every rank
    wt = torch.from_numpy(w.astype(np.float64))
    w0 = wt.clone()
    dist.broadcast(w0, src=0)
    assert torch.equal(wt, w0), "ranks diverged"
    if rank == 0:
        ref = [p.copy() for p in params]
        _, rnorm, rgrads = O.train_step(cfg, ref, ids, tg, 1.0,
                                        O.AdamW(ref, O.AdamWConfig(1e-3, 0.9, 0.95, 1e-8, 0.1)))
        avg = grads_sum / world
        at, worst = 0, 0.0
        for g in rgrads:
            worst = max(worst, O.max_abs_rel(avg[at:at + g.size].reshape(g.shape), g))
            at += g.size
        assert worst <= 2e-2, worst
        assert abs(norm - rnorm) <= 2e-2 * rnorm, (norm, rnorm)
        print(f"DP OK worst grad err {worst:.2e} norm {norm:.4f} vs {rnorm:.4f}", flush=True)
    # The same step with the optimizer state sharded across the ranks (reduce-scatter, per-rank
    # clip + AdamW on 1/world of the parameters, all-gather of the updated weights): the same
    # gradient sums, norm and updated weights as the all-reduce run above.
    ts = TA.Trainer(cfg, lr=1e-3, betas=(0.9, 0.95), eps=1e-8, weight_decay=0.1, max_norm=1.0,
                    dtype=1, batch=B, seq_len=T, seed=3)
    ts.set_params(np.concatenate([p.ravel() for p in params]))
    uid = [TA.nccl_unique_id() if rank == 0 else None]
    dist.broadcast_object_list(uid, src=0)
    ts.init_dp(uid[0], rank, world, 1 << 20, sharded=True)
    for step in range(3):
        l_s, n_s = ts.step_host(ids[mine], tg[mine])
        if step == 0:
            assert abs(l_s - loss) <= 1e-6 * abs(loss), (l_s, loss)
            assert abs(n_s - norm) <= 1e-5 * norm, (n_s, norm)
            g_s = ts.get_grads()
            assert np.max(np.abs(g_s - grads_sum)) <= 1e-6 * np.max(np.abs(grads_sum)), "gradients"
            w_s = ts.get_params()
            assert np.max(np.abs(w_s - w)) <= 1e-5, np.max(np.abs(w_s - w))
    # the second step ran on the all-gathered bf16 weights: identical on every rank
    wfin = ts.get_params()
    w2 = torch.from_numpy(wfin.astype(np.float64))
    w20 = w2.clone()
    dist.broadcast(w20, src=0)
    assert torch.equal(w2, w20), "sharded ranks diverged"
    if rank == 0:
        out = os.environ.get("VEDA_DP_OUT")
        if out:
            np.save(out, wfin)
        print(f"SHARDED OK loss {l_s:.4f}", flush=True)
    dist.barrier()
    ts.close()
    t.close()
    dist.destroy_process_group()


def lost_peer():
    """Rank 1 leaves between steps (after a host barrier: none of its work is in flight). Rank 0
    learns of it on the host (a monitored barrier that times out) before its next launch, aborts
    its communicator without waiting for the peer, gets an error from the next step instead of a
    hang, and its CUDA context still runs kernels."""
    import torch
    import torch.distributed as dist
    from oracle import veda_oracle as O
    from veda_b200 import train_abi as TA

    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    torch.cuda.set_device(int(os.environ["LOCAL_RANK"]))
    dist.init_process_group("gloo", timeout=datetime.timedelta(seconds=60))
    cfg = O.ModelConfig(vocab=2048, hidden=256, intermediate=512, layers=2, heads=4, kv_heads=2,
                        head_dim=128, eps=1e-6, theta=1e6)
    B, T = 2, 128
    ids, tg = O.synthetic_batch(cfg, B * world, T, 7)
    mine = slice(B * rank, B * rank + B)
    t = TA.Trainer(cfg, lr=1e-3, betas=(0.9, 0.95), eps=1e-8, weight_decay=0.1, max_norm=1.0,
                   dtype=1, batch=B, seq_len=T, seed=3)
    uid = [TA.nccl_unique_id() if rank == 0 else None]
    dist.broadcast_object_list(uid, src=0)
    t.init_dp(uid[0], rank, world, 1 << 20)
    t.set_comm_timeout(30.0)
    t.step_host(ids[mine], tg[mine])          # one healthy step; last_stats waited for it
    dist.barrier()                            # both ranks are past the step: nothing in flight
    if rank == 1:
        os._exit(0)                           # the rank leaves between steps
    try:
        dist.monitored_barrier(timeout=datetime.timedelta(seconds=10))
        print("LOST PEER NOT DETECTED", flush=True)
        os._exit(1)
    except Exception:  # noqa: BLE001 - the host learns the peer is gone
        pass
    t.abort_comm()                            # nothing of ours is in flight either
    try:
        t.step_host(ids[mine], tg[mine])
        print("STEP AFTER ABORT DID NOT FAIL", flush=True)
        os._exit(1)
    except RuntimeError as e:
        assert "abort" in str(e), str(e)
    x = torch.ones(1 << 20, device="cuda")    # the context still runs kernels
    assert float(x.sum().item()) == float(1 << 20)
    print("LOST PEER OK", flush=True)
    os._exit(0)


if __name__ == "__main__":
    if os.environ.get("VEDA_DP_MODE") == "lost_peer":
        lost_peer()
    else:
        main()
