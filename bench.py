"""Training-step throughput of the B200 path (train tokens/s: forward + backward + clip + AdamW).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--workload qwen3-0.6b|qwen3-1.7b|tiny]
    python -m torch.distributed.run --nproc-per-node N ... bench.py --gpus N   (N > 1)
    python bench.py --impl reference ...   (the reference's own CPU implementation)

One step = one full training step of the named config on one synthetic micro-batch per GPU
(data-parallel: 25 MB gradient buckets reduce-scattered by NCCL while the backward runs, the
optimizer state sharded across the ranks and the updated weights all-gathered; --dp allreduce
keeps the optimizer replicated and all-reduces the buckets instead), inputs
uniform random token ids with shifted-by-one targets. Prints one JSON line (rank 0).
"""
from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

# name -> (config kwargs, micro-batch, seq_len, weight seed)
WORKLOADS = {
    "qwen3-0.6b": (dict(vocab=151936, hidden=1024, intermediate=3072, layers=28, heads=16,
                        kv_heads=8, head_dim=128, eps=1e-6, theta=1e6), 4, 2048, 3),
    "qwen3-1.7b": (dict(vocab=151936, hidden=2048, intermediate=6144, layers=28, heads=16,
                        kv_heads=8, head_dim=128, eps=1e-6, theta=1e6), 2, 4096, 4),
    "tiny": (dict(vocab=512, hidden=64, intermediate=192, layers=2, heads=4, kv_heads=2,
                  head_dim=16, eps=1e-6, theta=1e4), 4, 32, 0),
}
METRIC = "train tokens/s (fwd+bwd+AdamW) at 1/2/4/8 B200; bwd kernels % of roofline"


def load_peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return d["hbm_gbs"], d["bf16_tflops"], d.get("bf16_tflops_sustained", d["bf16_tflops"]), "measured"
    return 6650.0, 1590.0, 1400.0, "fallback"


def model_flops_per_token(c, seq_len):
    """Model FLOPs per token: 6 x matmul parameters (tied LM head counted once as the head) plus
    causal attention 3.5 x 2 x T x H x Dh per layer (forward 2, backward 5 products of T*Dh per
    query, halved by the mask)."""
    D, F, H, Hk, Dh, V, L = (c["hidden"], c["intermediate"], c["heads"], c["kv_heads"],
                             c["head_dim"], c["vocab"], c["layers"])
    per_layer = D * (H + 2 * Hk) * Dh + H * Dh * D + 3 * D * F
    matmul_params = L * per_layer + V * D
    attn = L * 3.5 * 2 * seq_len * H * Dh
    return 6.0 * matmul_params + attn


# ------------------------------------------------------------------------------------------
# clocks during the timed region
# ------------------------------------------------------------------------------------------
class ClockSampler:
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index):
        self.gpu = gpu_index
        self.proc = None
        self.path = None

    def start(self):
        try:
            import tempfile
            self.f = tempfile.NamedTemporaryFile("w+", prefix=f"veda_clocks_gpu{self.gpu}_",
                                                 suffix=".csv", delete=False)
            self.path = Path(self.f.name)
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "200", "-i", str(self.gpu)], stdout=self.f, stderr=subprocess.DEVNULL)
        except Exception:
            self.proc = None

    def stop(self):
        if self.proc is None:
            return None
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        self.f.close()
        rows = []
        text = self.path.read_text()
        try:
            self.path.unlink()
        except OSError:
            pass
        for line in text.splitlines():
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                rows.append((float(parts[1]), float(parts[2]), parts[4:]))
            except ValueError:
                continue
        if not rows:
            return None
        load = [r for r in rows if r[0] > 0.5 * r[1]] or rows
        reasons = set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for r in rows:
            for name, v in zip(names, r[2][1:5]):
                if v.lower() == "active":
                    reasons.add(name)
        return {"sm_mhz": statistics.median(r[0] for r in load), "sm_max_mhz": rows[0][1],
                "reasons": sorted(reasons), "samples": len(rows)}


# ------------------------------------------------------------------------------------------
# the reference's CPU path (oracle/_ref: the reference compiled from its own sources)
# ------------------------------------------------------------------------------------------
def _ref_step_seconds(cfg_kwargs, T, threads):
    """Wall time of one reference CPU training step (vref_train_step: forward, CE, backward, clip,
    AdamW through the reference's own autograd / optim code) on a 1 x T window."""
    from oracle import ref as R
    from oracle import veda_oracle as O
    R.set_threads(threads)
    cfg = O.ModelConfig(**cfg_kwargs)
    params = O.init_params(cfg, 3)
    ids, tg = O.synthetic_batch(cfg, 1, T, 3)
    t0 = time.perf_counter()
    R.train_steps(cfg, params, ids, tg, 1.0, O.AdamWConfig(1e-3, 0.9, 0.95, 1e-8, 0.1), 1)
    return time.perf_counter() - t0


def cpu_reference_sample(c, T, threads):
    """The reference's CPU training step at full width and full sequence length T, from parts
    each measured where it is exact:
      * one decoder layer at T (quadratic attention included): a 1-layer minus a 0-layer model,
        both with a 512-token vocabulary so the difference is the layer alone;
      * the embedding / final norm / LM head / cross-entropy part at the full vocabulary, linear
        in tokens: a 0-layer model at 32 and 160 tokens, fitted as fixed + per-token cost;
    step(T) = head(T) + layers x layer(T). Returns (tokens/s, description, seconds spent)."""
    from oracle import ref as R
    if not R.available():
        raise RuntimeError("oracle/_ref/libveda_ref.so is not built")
    t_start = time.perf_counter()
    small = {**c, "vocab": 512}
    layer = (_ref_step_seconds({**small, "layers": 1}, T, threads) -
             _ref_step_seconds({**small, "layers": 0}, T, threads))
    h_lo = _ref_step_seconds({**c, "layers": 0}, 32, threads)
    h_hi = _ref_step_seconds({**c, "layers": 0}, 160, threads)
    per_token = max(h_hi - h_lo, 0.0) / 128.0
    head = h_lo + (T - 32) * per_token
    step = head + c["layers"] * layer
    desc = (f"reference CPU step (oracle/_ref, {threads} threads), full width, 1 x {T} tokens: one "
            f"decoder layer measured at T = {T} ({layer:.2f} s, attention included), the "
            f"full-vocabulary head fitted from 32- and 160-token windows ({h_lo:.2f} s, "
            f"{h_hi:.2f} s; {head:.1f} s at {T}); {c['layers']} layers + head = {step:.1f} s "
            f"per {T} tokens")
    return T / step, desc, time.perf_counter() - t_start


def cpu_tiny_sample(threads, steps=20):
    """The tiny decoder config (fp32, d_model 64, 2 layers, GQA 4/2, B 4 x T 32) timed in full on
    the reference's CPU path: median of `steps` whole steps. Returns (tokens/s, description)."""
    c, B, T, _ = WORKLOADS["tiny"]
    from oracle import ref as R
    from oracle import veda_oracle as O
    R.set_threads(threads)
    cfg = O.ModelConfig(**c)
    params = O.init_params(cfg, 0)
    ids, tg = O.synthetic_batch(cfg, B, T, 0)
    adam = O.AdamWConfig(1e-3, 0.9, 0.95, 1e-8, 0.1)
    times = []
    for _ in range(steps):
        t0 = time.perf_counter()
        R.train_steps(cfg, params, ids, tg, 1.0, adam, 1)
        times.append(time.perf_counter() - t0)
    med = statistics.median(times)
    return B * T / med, (f"tiny config, fp32, B {B} x T {T}, full steps on the reference's CPU path "
                         f"({threads} threads), median of {steps}: {1000 * med:.1f} ms per step")


def run_reference(args):
    """The reference arm: the reference's own CPU training step (oracle/_ref, all host threads) on
    this workload. A sample times every part once (about two to three minutes at Qwen3 sizes), so
    samples are repeated only while the whole run stays within about four minutes; the line
    reports how many were taken."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return 0
    c, B, T, _ = WORKLOADS[args.workload]
    threads = os.cpu_count() or 1
    vals, desc, spent = [], "", 0.0
    for i in range(max(1, args.steps)):
        if args.workload == "tiny":
            v, desc = cpu_tiny_sample(threads)
            vals.append(v)
            continue
        v, desc, took = cpu_reference_sample(c, T, threads)
        vals.append(v)
        spent += took
        if spent + took > 240.0:
            break
    value = statistics.median(vals)
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": "tokens/s",
        "n_gpus": args.gpus, "steps": len(vals), "warmup": 0,
        "ms_per_step": 1000.0 * B * T * args.gpus / value if value > 0 else None,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic",
        "config": {"workload": args.workload, "global_batch": B * args.gpus, "seq_len": T,
                   "parallelism": "cpu"},
        "cpu_baseline": {"value": value, "unit": "tokens/s", "cores": threads,
                         "kind": "reference", "sample": desc},
        "e2e": {"value": value, "unit": "tokens/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }
    if args.workload != "tiny":
        tv, tdesc = cpu_tiny_sample(threads)
        line["cpu_baseline_tiny"] = {"value": tv, "unit": "tokens/s", "cores": threads,
                                     "kind": "reference", "sample": tdesc}
    emit(line)
    return 0


# ------------------------------------------------------------------------------------------
# the B200 path
# ------------------------------------------------------------------------------------------
def run_veda(args):
    import torch
    import torch.distributed as dist

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    if world > 1:
        os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
        import datetime
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                device_id=torch.device("cuda", local))

    import veda_b200 as V
    from oracle import veda_oracle as O  # noqa: F401  (configs only; not on the timed path)
    from veda_b200 import train_abi as TA

    c, B, T, seed = WORKLOADS[args.workload]
    cfg = O.ModelConfig(**c)
    stream = torch.cuda.Stream()
    tr = TA.Trainer(cfg, lr=1e-3, betas=(0.9, 0.95), eps=1e-8, weight_decay=0.1, max_norm=1.0,
                    dtype=0 if args.workload == "tiny" else 1, batch=B, seq_len=T, seed=seed,
                    stream=stream.cuda_stream)
    recompute = args.recompute == "on" or (args.recompute == "auto" and args.workload == "qwen3-1.7b")
    tr.set_recompute_attention(recompute)
    if world > 1:
        obj = [TA.nccl_unique_id() if rank == 0 else None]
        dist.broadcast_object_list(obj, src=0)
        tr.init_dp(obj[0], rank, world, args.bucket_mb << 20, sharded=args.dp == "sharded")

    # synthetic batches (per rank, per step), pinned on the host and resident on the device
    nb = 4
    rng = np.random.default_rng(1000 * seed + rank)
    windows = [rng.integers(0, cfg.vocab, size=(B, T + 1), dtype=np.int64) for _ in range(nb)]
    host_ids = [torch.from_numpy(np.ascontiguousarray(w[:, :-1])).pin_memory() for w in windows]
    host_tg = [torch.from_numpy(np.ascontiguousarray(w[:, 1:])).pin_memory() for w in windows]
    dev_ids = [h.to(f"cuda:{local}") for h in host_ids]
    dev_tg = [h.to(f"cuda:{local}") for h in host_tg]
    torch.cuda.synchronize()

    def barrier():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()

    def max_over_ranks(x):
        if world == 1:
            return x
        t = torch.tensor([x], dtype=torch.float64, device=f"cuda:{local}")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    with torch.cuda.stream(stream):
        for i in range(args.warmup):
            tr.step_device(dev_ids[i % nb].data_ptr(), dev_tg[i % nb].data_ptr())
        tr.last_stats()

        # ---- value: device-resident inputs, no instrumentation in the timed steps ------------
        sampler = ClockSampler(local) if rank == 0 else None
        barrier()
        if sampler:
            sampler.start()
        launches0 = V.lib().veda_launch_count()
        start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        start.record(stream)
        for i in range(args.steps):
            tr.step_device(dev_ids[i % nb].data_ptr(), dev_tg[i % nb].data_ptr())
        tr.sync()   # the last step's weight all-gather (sharded optimizer) is inside the region
        stop.record(stream)
        stop.synchronize()
        launches = V.lib().veda_launch_count() - launches0
        ms = max_over_ranks(start.elapsed_time(stop))
        loss, norm = tr.last_stats()
        barrier()
        clocks = sampler.stop() if sampler else None

        # ---- per-kernel-class device time: the same steps again with CUDA-event scopes on the
        # trainer's stream (the event pairs cost ~2 ms a step, so they stay out of `value`) -----
        TA.profile_enable(True)
        for i in range(args.steps):
            tr.step_device(dev_ids[i % nb].data_ptr(), dev_tg[i % nb].data_ptr())
        TA.profile_enable(False)
        prof = TA.profile_collect()
        barrier()

        # ---- e2e: host buffers through the public step call (H2D in, loss/norm D2H out) -------
        barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for i in range(args.steps):
            tr.step_host(host_ids[i % nb].numpy(), host_tg[i % nb].numpy())
        tr.sync()
        e1.record(stream)
        e1.synchronize()
        e2e_ms = max_over_ranks(e0.elapsed_time(e1))
    barrier()

    tokens = world * B * T * args.steps
    value = tokens / (ms / 1000.0)
    e2e = tokens / (e2e_ms / 1000.0)
    hbm, tf_burst, tf_sus, peak_kind = load_peaks()

    gemm = [(k, prof[k]) for k in ("gemm_fwd", "gemm_dx", "gemm_dw", "gemm_bwd") if k in prof]
    g_ms = sum(p[0] for _, p in gemm)
    g_fl = sum(p[1] for _, p in gemm)
    g_n = sum(p[3] * (2 if k == "gemm_bwd" else 1) for k, p in gemm)   # a gemm_bwd scope = 2 GEMMs
    achieved = g_fl / (g_ms / 1000.0) / 1e12 if g_ms > 0 else None
    kernels = {k: {"ms_per_step": v[0] / args.steps, "launches_per_step": v[3] / args.steps,
                   "tflops": (v[1] / (v[0] / 1000.0) / 1e12) if v[1] and v[0] else None,
                   "gbs": (v[2] / (v[0] / 1000.0) / 1e9) if v[2] and v[0] else None}
               for k, v in sorted(prof.items())}
    # DRAM bytes (read + write) per GEMM launch, averaged over the 339 GEMM launches of one step,
    # from one ncu capture of the same step
    traffic = GEMM_DRAM_BYTES_PER_LAUNCH.get(args.workload)

    line = {
        "metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms / args.steps,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "f32" if args.workload == "tiny" else "bf16", "data": "synthetic",
        "config": {"workload": args.workload, "model": args.workload, "global_batch": B * world,
                   "micro_batch": B, "seq_len": T, "parallelism": f"dp{world}",
                   "params": tr.n, "l2": "inputs and the step's working set exceed L2",
                   "buckets_mb": args.bucket_mb, "attention_recompute": recompute,
                   "optimizer_state": ("sharded (ZeRO-1)" if world > 1 and args.dp == "sharded"
                                       else "replicated")},
        "mfu_model_tflops": model_flops_per_token(c, T) * value / 1e12,
        "roofline": {"bound": "tensor", "kernel": "tcgen05 GEMM (gemm_fwd + gemm_bwd: dX beside dW)",
                     "achieved": achieved, "peak": tf_sus, "unit": "TFLOP/s",
                     "peak_kind": f"{peak_kind} bf16 sustained",
                     "frac": (achieved / tf_sus) if achieved else None,
                     "launches_per_step": g_n / args.steps, "traffic": traffic},
        "kernels": kernels,
        "gpu_launches": int(launches),
        "e2e": {"value": e2e, "unit": "tokens/s", "h2d_bytes_per_step": 2 * B * T * 8,
                "d2h_bytes_per_step": 4 + 8},
        "loss": loss, "grad_norm": norm,
        "clocks": clocks,
    }
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        threads = os.cpu_count() or 1
        try:
            if args.workload == "tiny":
                v, desc = cpu_tiny_sample(threads)
            else:
                v, desc, _ = cpu_reference_sample(c, T, threads)
            line["cpu_baseline"] = {"value": v, "unit": "tokens/s", "cores": threads,
                                    "kind": "reference", "sample": desc}
            if args.workload != "tiny":
                tv, tdesc = cpu_tiny_sample(threads)
                line["cpu_baseline_tiny"] = {"value": tv, "unit": "tokens/s", "cores": threads,
                                             "kind": "reference", "sample": tdesc}
        except Exception as e:  # the reference build is missing: report, do not fail
            line["cpu_baseline"] = {"value": None, "unit": "tokens/s", "cores": 0,
                                    "kind": "reference", "sample": f"unavailable: {e}"}
    if rank == 0:
        emit(line)
    tr.close()
    if world > 1:
        dist.destroy_process_group()
    return 0


_JSON_OUT = None
GEMM_DRAM_BYTES_PER_LAUNCH = {"qwen3-0.6b": 116.57e6}


def emit(line: dict):
    """Writes the one JSON line to the real stdout (everything else goes to stderr)."""
    os.write(_JSON_OUT if _JSON_OUT is not None else 1, (json.dumps(line) + "\n").encode())


def main():
    global _JSON_OUT
    # Libraries (NCCL, torch.distributed) may print to stdout from native code; keep stdout for
    # the JSON line alone by pointing fd 1 at stderr and keeping a private copy of the original.
    sys.stdout.flush()
    _JSON_OUT = os.dup(1)
    os.dup2(2, 1)
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="veda", choices=["veda", "reference"])
    ap.add_argument("--workload", default="qwen3-0.6b", choices=sorted(WORKLOADS))
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--bucket-mb", type=int, default=25,
                    help="N > 1: gradient bucket size in MiB")
    ap.add_argument("--recompute", default="auto", choices=["auto", "on", "off"],
                    help="activation recompute of attention (auto: on for qwen3-1.7b, the config "
                         "that names it)")
    ap.add_argument("--dp", default="sharded", choices=["sharded", "allreduce"],
                    help="N > 1: optimizer state sharded across ranks (reduce-scatter + all-gather) "
                         "or replicated (all-reduce)")
    args = ap.parse_args()
    if args.impl == "reference":
        return run_reference(args)
    return run_veda(args)


if __name__ == "__main__":
    sys.exit(main())
