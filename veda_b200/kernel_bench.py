"""Isolated kernel timings through the C ABI (CUDA events on one stream, inputs larger than L2).

    python -m veda_b200.kernel_bench mm-sweep [--reps 10]
        the matmul-backward sweep: for X[M,K], W[K,N], dY[M,N] (bf16, ~N(0,1)/sqrt(K), seed 1)
        time dX = dY W^T and dW = X^T dY (fp32 out) for (M,K,N) in the five sweep shapes, the
        pair as one CUDA graph replayed after an L2-clearing read; 4*M*K*N FLOP per shape.
    python -m veda_b200.kernel_bench attn-bwd [--seq 1024 4096] [--reps 5] [--modes 0 1]
        causal GQA attention backward, B 8, H 16, Hkv 8, Dh 128, bf16, seed 2; 5*B*H*T^2*Dh FLOP.
    python -m veda_b200.kernel_bench gemm --op nt --m 8192 --n 151936 --k 1024 [--reps 3]
        one GEMM shape (used for the ncu captures).
    python -m veda_b200.kernel_bench bw [--tokens 8192] [--reps 20]
        the bandwidth-bound kernels of one Qwen3-0.6B layer at `tokens` tokens (hidden 1024,
        16 query / 8 KV heads of 128, FFN 3072, vocab 151936 for the cross-entropy): RMSNorm
        forward / backward (with residual gradient and dgamma), QK-norm+RoPE forward / backward,
        SwiGLU forward / backward, cross-entropy; GB/s from the algorithmic bytes (each tensor
        read or written once). --kernels NAME... runs a subset (names as printed). Each kernel is
        timed as a CUDA graph of 24 calls over 6 rotating input sets (so launch latency is not
        counted and every call reads HBM).
Prints one JSON line per measurement.
"""
from __future__ import annotations

import argparse
import json
import math

import numpy as np

SWEEP = [(4096, 1024, 1024), (4096, 1024, 3072), (4096, 3072, 1024), (8192, 2048, 6144),
         (8192, 1024, 151936)]


def _peaks():
    from pathlib import Path
    p = Path(__file__).resolve().parent.parent / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return d["bf16_tflops"], d["hbm_gbs"], "measured"
    return 1590.0, 6650.0, "fallback"


def _time(fn, reps, stream, flush=None):
    """Mean CUDA-event time of fn over reps. With `flush` (a device tensor larger than L2), each
    rep first reads it (a sum), so L2 holds clean lines of no use to fn: fn's reads come from
    HBM without also paying write-backs of dirty lines a writing flush would leave behind."""
    import torch
    fn()
    torch.cuda.synchronize()
    total = 0.0
    for _ in range(reps):
        if flush is not None:
            flush.sum()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record(stream)
        fn()
        b.record(stream)
        b.synchronize()
        total += a.elapsed_time(b)
    return total / reps


def mm_sweep(reps):
    """dX and dW of each shape as one CUDA graph (so the host's launch latency is not timed),
    replayed after an L2-clearing read; parity spot-checked against fp64."""
    import torch
    import veda_b200 as V
    L = V.lib()
    s = torch.cuda.Stream()     # graphs are captured on a non-default stream
    torch.cuda.set_stream(s)
    peak, _, kind = _peaks()
    flush = torch.ones(64 << 20, dtype=torch.float32, device="cuda")   # 256 MB > L2, read per rep
    g = torch.Generator(device="cuda").manual_seed(1)
    for (M, K, N) in SWEEP:
        x = (torch.randn(M, K, device="cuda", generator=g) / math.sqrt(K)).to(torch.bfloat16)
        w = (torch.randn(K, N, device="cuda", generator=g) / math.sqrt(K)).to(torch.bfloat16)
        dy = (torch.randn(M, N, device="cuda", generator=g) / math.sqrt(K)).to(torch.bfloat16)
        dx = torch.empty(M, K, dtype=torch.float32, device="cuda")
        dw = torch.empty(K, N, dtype=torch.float32, device="cuda")

        def run():
            # dX[M,K] = dY[M,N] . W[K,N]^T  (NT) ; dW[K,N] = X[M,K]^T . dY[M,N]  (TN)
            V.check(L.veda_gemm_nt(M, K, N, dy.data_ptr(), N, w.data_ptr(), N, dx.data_ptr(), K,
                                   V.BF16, V.F32, 1.0, 0.0, s.cuda_stream))
            V.check(L.veda_gemm_tn(K, N, M, x.data_ptr(), K, dy.data_ptr(), N, dw.data_ptr(), N,
                                   V.BF16, V.F32, 1.0, 0.0, s.cuda_stream))
        run()                   # first calls (attributes, cluster occupancy) outside the capture
        torch.cuda.synchronize()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=s):
            run()
        ms = _time(graph.replay, reps, s, flush)
        del graph
        flops = 4.0 * M * K * N
        tf = flops / (ms / 1e3) / 1e12
        print(json.dumps({"bench": "mm-sweep", "M": M, "K": K, "N": N, "ms": ms,
                          "tflops": tf, "peak": peak, "frac": tf / peak,
                          "peak_kind": f"{kind} bf16 burst"}), flush=True)
        # parity spot check of the two products on a row/column sample (fp64 on the host)
        rows = torch.arange(0, M, max(1, M // 64), device="cuda")
        cols = torch.arange(0, N, max(1, N // 64), device="cuda")
        ref_dx = (dy[rows].double() @ w.double().T)
        ref_dw = (x.double().T @ dy[:, cols].double())
        e1 = float((dx[rows].double() - ref_dx).abs().max() / ref_dx.abs().max())
        e2 = float((dw[:, cols].double() - ref_dw).abs().max() / ref_dw.abs().max())
        assert e1 < 1e-3 and e2 < 1e-3, (M, K, N, e1, e2)   # fp32 accumulation over K
        del x, w, dy, dx, dw
        torch.cuda.empty_cache()


def attn_bwd(seqs, reps, modes=(0, 1), B=8):
    """Attention fwd and bwd at B x H16 / Hkv8 x Dh128; each backward mode: 0 the fused kernel,
    1 the deterministic two-kernel path."""
    import torch
    import veda_b200 as V
    L = V.lib()
    s = torch.cuda.current_stream()
    peak, _, kind = _peaks()
    H, Hk, Dh = 16, 8, 128
    g = torch.Generator(device="cuda").manual_seed(2)
    for T, mode in [(T, m) for T in seqs for m in modes]:
        L.veda_attention_set_deterministic(mode)
        q = torch.randn(B * T, H * Dh, device="cuda", generator=g).to(torch.bfloat16)
        k = torch.randn(B * T, Hk * Dh, device="cuda", generator=g).to(torch.bfloat16)
        v = torch.randn(B * T, Hk * Dh, device="cuda", generator=g).to(torch.bfloat16)
        do = torch.randn(B * T, H * Dh, device="cuda", generator=g).to(torch.bfloat16)
        o = torch.empty_like(q)
        lse = torch.empty(B * H * T, dtype=torch.float32, device="cuda")
        dq, dk, dv = torch.empty_like(q), torch.empty_like(k), torch.empty_like(v)
        ws = torch.empty(L.veda_attention_bwd_workspace(B, T, H, Hk, Dh, V.BF16), dtype=torch.uint8,
                         device="cuda")
        scale = 1.0 / math.sqrt(Dh)
        V.check(L.veda_attention_fwd(q.data_ptr(), H * Dh, k.data_ptr(), Hk * Dh, v.data_ptr(),
                                     Hk * Dh, o.data_ptr(), H * Dh, lse.data_ptr(), B, T, H, Hk, Dh,
                                     scale, 1, V.BF16, s.cuda_stream))

        def fwd():
            V.check(L.veda_attention_fwd(q.data_ptr(), H * Dh, k.data_ptr(), Hk * Dh, v.data_ptr(),
                                         Hk * Dh, o.data_ptr(), H * Dh, lse.data_ptr(), B, T, H, Hk,
                                         Dh, scale, 1, V.BF16, s.cuda_stream))

        def bwd():
            V.check(L.veda_attention_bwd(q.data_ptr(), H * Dh, k.data_ptr(), Hk * Dh, v.data_ptr(),
                                         Hk * Dh, o.data_ptr(), H * Dh, do.data_ptr(), H * Dh,
                                         lse.data_ptr(), dq.data_ptr(), H * Dh, dk.data_ptr(),
                                         Hk * Dh, dv.data_ptr(), Hk * Dh, ws.data_ptr(), ws.numel(),
                                         B, T, H, Hk, Dh, scale, 1, V.BF16, s.cuda_stream))
        ms_b = _time(bwd, reps, s)
        ms_f = _time(fwd, reps, s)
        fl_b = 5.0 * B * H * T * T * Dh
        fl_f = 2.0 * B * H * T * T * Dh
        print(json.dumps({"bench": "attn", "mode": ["fused", "deterministic"][mode], "B": B,
                          "H": H, "Hkv": Hk, "Dh": Dh, "T": T,
                          "bwd_ms": ms_b, "bwd_tflops": fl_b / (ms_b / 1e3) / 1e12,
                          "fwd_ms": ms_f, "fwd_tflops": fl_f / (ms_f / 1e3) / 1e12,
                          "peak": peak, "bwd_frac": fl_b / (ms_b / 1e3) / 1e12 / peak,
                          "peak_kind": f"{kind} bf16 burst"}), flush=True)
        del q, k, v, do, o, lse, dq, dk, dv, ws
        torch.cuda.empty_cache()


def bandwidth_kernels(tokens, reps, only=None):
    """Each kernel is captured in a CUDA graph of 24 calls rotating over 6 input sets (together far
    larger than L2, so every call reads HBM), replayed `reps` times; per-call time = graph time /
    24. Timing a single call between two events would measure the host's launch latency for
    these ~10-50 us kernels. The cross-entropy (~1.4 ms a call) is timed directly."""
    import torch
    import veda_b200 as V
    L = V.lib()
    s = torch.cuda.Stream()     # graphs are captured on a non-default stream
    torch.cuda.set_stream(s)
    _, hbm, kind = _peaks()
    g = torch.Generator(device="cuda").manual_seed(3)
    T, D, H, Hk, F, Vv = 2048, 1024, 16, 8, 3072, 151936
    bf = torch.bfloat16
    B2 = 2
    SETS, CALLS = 6, 24
    rn = lambda *shape: torch.randn(*shape, device="cuda", generator=g).to(bf)  # noqa: E731
    st = s.cuda_stream
    gam, gq = rn(D), rn(128)
    cos = torch.randn(T, 128, device="cuda", generator=g)
    sin = torch.randn(T, 128, device="cuda", generator=g)
    dg = torch.zeros(D, dtype=torch.float32, device="cuda")
    dgq = torch.zeros(128, dtype=torch.float32, device="cuda")
    ws = torch.empty(L.veda_rmsnorm_bwd_workspace(tokens, D), dtype=torch.uint8, device="cuda")
    wsq = torch.empty(L.veda_qknorm_rope_bwd_workspace(tokens, H, 128), dtype=torch.uint8,
                      device="cuda")

    def want(name):
        return only is None or name in only

    sets = []
    for _ in range(SETS):
        d = {}
        if want("rmsnorm_fwd") or want("rmsnorm_bwd"):
            d.update(x=rn(tokens, D), dy=rn(tokens, D), dr=rn(tokens, D),
                     y=torch.empty(tokens, D, dtype=bf, device="cuda"),
                     dx=torch.empty(tokens, D, dtype=bf, device="cuda"))
        if want("qknorm_rope_fwd_q") or want("qknorm_rope_bwd_q"):
            d.update(qkv=rn(tokens, (H + 2 * Hk) * 128), dqkv=rn(tokens, H * 128),
                     qo=torch.empty(tokens, H * 128, dtype=bf, device="cuda"))
        if want("swiglu_fwd") or want("swiglu_bwd"):
            d.update(gu=rn(tokens, 2 * F), dh=rn(tokens, F),
                     hh=torch.empty(tokens, F, dtype=bf, device="cuda"),
                     dgu=torch.empty(tokens, 2 * F, dtype=bf, device="cuda"))
        sets.append(d)

    def rms_fwd(d):
        V.check(L.veda_rmsnorm_fwd(d["x"].data_ptr(), D, gam.data_ptr(), d["y"].data_ptr(), D, tokens, D,
                                   1e-6, V.BF16, st))

    def rms_bwd(d):
        V.check(L.veda_rmsnorm_bwd(d["x"].data_ptr(), D, gam.data_ptr(), d["dy"].data_ptr(), D,
                                   d["dr"].data_ptr(), D, d["dx"].data_ptr(), D, dg.data_ptr(),
                                   ws.data_ptr(), ws.numel(), tokens, D, 1e-6, V.BF16, st))

    def qk_fwd(d):
        q = d["qkv"]
        V.check(L.veda_qknorm_rope_fwd(q.data_ptr(), q.shape[1], gq.data_ptr(), cos.data_ptr(),
                                       sin.data_ptr(), d["qo"].data_ptr(), H * 128, tokens, H, T, 128,
                                       1e-6, V.BF16, st))

    def qk_bwd(d):
        q = d["qkv"]
        V.check(L.veda_qknorm_rope_bwd(q.data_ptr(), q.shape[1], gq.data_ptr(), cos.data_ptr(),
                                       sin.data_ptr(), d["dqkv"].data_ptr(), H * 128, d["qo"].data_ptr(),
                                       H * 128, dgq.data_ptr(), wsq.data_ptr(), wsq.numel(), tokens, H, T,
                                       128, 1e-6, V.BF16, st))

    def sw_fwd(d):
        gu = d["gu"]
        V.check(L.veda_swiglu_fwd(gu.data_ptr(), 2 * F, gu.data_ptr() + F * B2, 2 * F, d["hh"].data_ptr(),
                                  F, tokens, F, V.BF16, st))

    def sw_bwd(d):
        gu, dgu = d["gu"], d["dgu"]
        V.check(L.veda_swiglu_bwd(gu.data_ptr(), 2 * F, gu.data_ptr() + F * B2, 2 * F, d["dh"].data_ptr(), F,
                                  dgu.data_ptr(), 2 * F, dgu.data_ptr() + F * B2, 2 * F, tokens, F, V.BF16,
                                  st))

    cases = {
        "rmsnorm_fwd": (rms_fwd, 2 * tokens * D * B2),
        "rmsnorm_bwd": (rms_bwd, 4 * tokens * D * B2),
        "qknorm_rope_fwd_q": (qk_fwd, 2 * tokens * H * 128 * B2),
        "qknorm_rope_bwd_q": (qk_bwd, 3 * tokens * H * 128 * B2),
        "swiglu_fwd": (sw_fwd, 3 * tokens * F * B2),
        "swiglu_bwd": (sw_bwd, 5 * tokens * F * B2),
    }
    for name, (fn, nbytes) in cases.items():
        if not want(name):
            continue
        for d in sets:          # warm-up outside the capture (first-call set-up, attributes)
            fn(d)
        torch.cuda.synchronize()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=s):
            for k in range(CALLS):
                fn(sets[k % SETS])
        graph.replay()
        torch.cuda.synchronize()
        ms = _time(graph.replay, reps, s) / CALLS
        print(json.dumps({"bench": "bw", "kernel": name, "tokens": tokens, "ms": ms,
                          "gbs": nbytes / (ms / 1e3) / 1e9, "peak_gbs": hbm, "peak_kind": kind,
                          "frac": nbytes / (ms / 1e3) / 1e9 / hbm}), flush=True)
        del graph
    del sets
    torch.cuda.empty_cache()
    if want("cross_entropy"):
        logits = rn(tokens, Vv)
        tgt = torch.randint(0, Vv, (tokens,), device="cuda", generator=g)
        rl = torch.empty(tokens, dtype=torch.float32, device="cuda")
        dl = torch.empty_like(logits)
        flush = torch.ones(64 << 20, dtype=torch.float32, device="cuda")   # 256 MB > L2, read per rep

        def ce():
            V.check(L.veda_cross_entropy(logits.data_ptr(), Vv, tgt.data_ptr(), rl.data_ptr(), dl.data_ptr(),
                                         Vv, tokens, Vv, 1.0 / tokens, 0, V.BF16, st))
        ms = _time(ce, reps, s, flush)
        nbytes = 2 * tokens * Vv * B2
        print(json.dumps({"bench": "bw", "kernel": "cross_entropy", "tokens": tokens, "ms": ms,
                          "gbs": nbytes / (ms / 1e3) / 1e9, "peak_gbs": hbm, "peak_kind": kind,
                          "frac": nbytes / (ms / 1e3) / 1e9 / hbm}), flush=True)


def one_gemm(op, M, N, K, reps, out=None):
    import torch
    import veda_b200 as V
    L = V.lib()
    s = torch.cuda.current_stream()
    a = torch.randn(*((K, M) if op == "tn" else (M, K)), device="cuda").to(torch.bfloat16)
    b = torch.randn(*((N, K) if op == "nt" else (K, N)), device="cuda").to(torch.bfloat16)
    # C in bf16 for nt (a forward layer) and fp32 otherwise (a gradient), unless `out` says
    bf = out == "bf16" if out is not None else op == "nt"
    c = torch.empty(M, N, dtype=torch.bfloat16 if bf else torch.float32, device="cuda")
    dc = V.BF16 if bf else V.F32
    fn = getattr(L, f"veda_gemm_{op}")

    def run():
        V.check(fn(M, N, K, a.data_ptr(), a.shape[1], b.data_ptr(), b.shape[1], c.data_ptr(), N,
                   V.BF16, dc, 1.0, 0.0, s.cuda_stream))
    ms = _time(run, reps, s)
    tf = 2.0 * M * N * K / (ms / 1e3) / 1e12
    print(json.dumps({"bench": "gemm", "op": op, "M": M, "N": N, "K": K, "ms": ms, "tflops": tf}),
          flush=True)


def swiglu_gemms(rows, F, D, reps, profile=False):
    """The MLP's GEMMs with SwiGLU in the epilogue (veda_gemm_swiglu_fwd / _bwd) against the GEMM
    followed by the stand-alone SwiGLU kernel, each timed as a CUDA graph of `reps` launches
    (median of 7 replays). With `profile`, two rounds of the fused forward and backward run once
    each, untimed (for ncu: the second round is launches 2 and 3)."""
    import torch
    import veda_b200 as V
    L = V.lib()
    s = torch.cuda.Stream()
    torch.cuda.set_stream(s)
    st = s.cuda_stream
    bf = torch.bfloat16
    g = torch.Generator(device="cuda").manual_seed(7)
    x = torch.randn(rows, D, device="cuda", generator=g).to(bf)
    wgu = (torch.randn(2 * F, D, device="cuda", generator=g) / math.sqrt(D)).to(bf)
    wd = (torch.randn(D, F, device="cuda", generator=g) / math.sqrt(F)).to(bf)
    dy = torch.randn(rows, D, device="cuda", generator=g).to(bf)
    gu = torch.empty(rows, 2 * F, device="cuda", dtype=bf)
    h = torch.empty(rows, F, device="cuda", dtype=bf)
    dh = torch.empty(rows, F, device="cuda", dtype=bf)
    dgu = torch.empty(rows, 2 * F, device="cuda", dtype=bf)
    es = 2

    def fwd_fused():
        V.check(L.veda_gemm_swiglu_fwd(rows, F, D, x.data_ptr(), D, wgu.data_ptr(), D, gu.data_ptr(),
                                       2 * F, h.data_ptr(), F, st))

    def bwd_fused():
        V.check(L.veda_gemm_swiglu_bwd(rows, F, D, dy.data_ptr(), D, wd.data_ptr(), F, gu.data_ptr(),
                                       2 * F, dgu.data_ptr(), 2 * F, st))

    def fwd_two():
        V.check(L.veda_gemm_nt(rows, 2 * F, D, x.data_ptr(), D, wgu.data_ptr(), D, gu.data_ptr(),
                               2 * F, V.BF16, V.BF16, 1.0, 0.0, st))
        V.check(L.veda_swiglu_fwd(gu.data_ptr(), 2 * F, gu.data_ptr() + F * es, 2 * F, h.data_ptr(), F,
                                  rows, F, V.BF16, st))

    def bwd_two():
        V.check(L.veda_gemm_nn(rows, F, D, dy.data_ptr(), D, wd.data_ptr(), F, dh.data_ptr(), F,
                               V.BF16, V.BF16, 1.0, 0.0, st))
        V.check(L.veda_swiglu_bwd(gu.data_ptr(), 2 * F, gu.data_ptr() + F * es, 2 * F, dh.data_ptr(),
                                  F, dgu.data_ptr(), 2 * F, dgu.data_ptr() + F * es, 2 * F, rows, F,
                                  V.BF16, st))

    if profile:
        for _ in range(2):
            fwd_fused()
            bwd_fused()
        torch.cuda.synchronize()
        return

    def graph_us(fn):
        fn()
        torch.cuda.synchronize()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=s):
            for _ in range(reps):
                fn()
        graph.replay()
        torch.cuda.synchronize()
        ts = []
        for _ in range(7):
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record(s)
            graph.replay()
            b.record(s)
            b.synchronize()
            ts.append(a.elapsed_time(b) / reps * 1e3)
        del graph
        return sorted(ts)[3]

    out = {"bench": "swiglu-gemms", "rows": rows, "F": F, "D": D,
           "fwd_fused_us": graph_us(fwd_fused), "fwd_gemm_then_swiglu_us": graph_us(fwd_two),
           "bwd_fused_us": graph_us(bwd_fused), "bwd_gemm_then_swiglu_us": graph_us(bwd_two)}
    out["fwd_fused_tflops"] = 4.0 * rows * F * D / out["fwd_fused_us"] / 1e6
    out["bwd_fused_tflops"] = 2.0 * rows * F * D / out["bwd_fused_us"] / 1e6
    print(json.dumps(out), flush=True)


def decode(prompt_len, new_tokens):
    """Greedy generation with the KV cache on the Qwen3-0.6B-shaped model (random weights, batch 1):
    decode tokens/s after the prefill, against the HBM roofline of one step (every weight read
    once, plus the cache rows attended to)."""
    import time
    import types
    import torch
    from veda_b200 import train_abi as TA
    _, hbm, kind = _peaks()
    cfg = types.SimpleNamespace(vocab=151936, hidden=1024, intermediate=3072, layers=28, heads=16,
                                kv_heads=8, head_dim=128, eps=1e-6, theta=1e6)
    t = TA.Trainer(cfg, dtype=1, batch=1, seq_len=8, seed=3)
    prompt = list(np.random.default_rng(0).integers(0, cfg.vocab, prompt_len))
    base = 8
    t.generate(prompt, 2, cached=True)   # warm-up
    torch.cuda.synchronize()
    # two generations that differ only in their number of new tokens: the prefill and the step's
    # recording cancel in the difference
    t0 = time.perf_counter()
    short, _, _ = t.generate(prompt, base, cached=True)
    t1 = time.perf_counter()
    toks, _, passes = t.generate(prompt, base + new_tokens, cached=True)
    t2 = time.perf_counter()
    extra = max(1, len(toks) - len(short))
    per_token = ((t2 - t1) - (t1 - t0)) / extra
    weights = t.n * 2.0
    kv = 2 * cfg.layers * cfg.kv_heads * cfg.head_dim * 2.0 * (prompt_len + base + new_tokens / 2)
    gbs = (weights + kv) / per_token / 1e9
    print(json.dumps({"bench": "decode", "model": "qwen3-0.6b", "prompt": prompt_len,
                      "new_tokens": extra, "ms_per_token": per_token * 1e3,
                      "tokens_per_s": 1.0 / per_token, "bytes_per_token": weights + kv,
                      "gbs": gbs, "frac": gbs / hbm, "peak_kind": kind,
                      "timing": "host wall clock per token: generations of 8 and 8 + N new tokens, "
                                "differenced (each token is read back to pick the next)"}),
          flush=True)
    t.close()
    # the step's projections alone: one activation row against each weight matrix, L2 flushed
    import veda_b200 as V
    s = torch.cuda.current_stream()
    flush = torch.empty(256 << 20, dtype=torch.float32, device="cuda")
    x = torch.randn(cfg.intermediate, device="cuda").to(torch.bfloat16)
    W = (cfg.heads + 2 * cfg.kv_heads) * cfg.head_dim
    shapes = [("qkv", W, cfg.hidden, False), ("o", cfg.hidden, cfg.heads * cfg.head_dim, False),
              ("gate_up+swiglu", cfg.intermediate, cfg.hidden, True),
              ("down", cfg.hidden, cfg.intermediate, False), ("lm_head", cfg.vocab, cfg.hidden, False)]
    for name, n, k, swiglu in shapes:
        rows = 2 * n if swiglu else n
        w = torch.randn(rows, k, device="cuda").to(torch.bfloat16)
        y = torch.empty(n, dtype=torch.bfloat16, device="cuda")
        fn = V.lib().veda_gemv_swiglu if swiglu else V.lib().veda_gemv_nt

        def run():
            V.check(fn(x.data_ptr(), w.data_ptr(), k, y.data_ptr(), n, k, V.BF16, s.cuda_stream))
        ms = _time(run, 20, s, flush)
        gbs = rows * k * 2.0 / (ms / 1e3) / 1e9
        print(json.dumps({"bench": "gemv", "layer": name, "n": n, "k": k, "us": ms * 1e3, "gbs": gbs,
                          "frac": gbs / hbm, "peak_kind": kind}), flush=True)
        del w


def main():
    ap = argparse.ArgumentParser()
    sub = ap.add_subparsers(dest="cmd", required=True)
    a = sub.add_parser("mm-sweep")
    a.add_argument("--reps", type=int, default=10)
    b = sub.add_parser("attn-bwd")
    b.add_argument("--seq", type=int, nargs="+", default=[1024, 4096])
    b.add_argument("--reps", type=int, default=5)
    b.add_argument("--modes", type=int, nargs="+", default=[0, 1])
    b.add_argument("--batch", type=int, default=8)
    c = sub.add_parser("gemm")
    c.add_argument("--op", default="nt", choices=["nt", "nn", "tn"])
    c.add_argument("--m", type=int, default=8192)
    c.add_argument("--n", type=int, default=151936)
    c.add_argument("--k", type=int, default=1024)
    c.add_argument("--reps", type=int, default=3)
    c.add_argument("--out", choices=["bf16", "f32"], default=None)
    d = sub.add_parser("bw")
    d.add_argument("--tokens", type=int, default=8192)
    d.add_argument("--reps", type=int, default=20)
    d.add_argument("--kernels", nargs="+", default=None)
    f = sub.add_parser("swiglu")
    f.add_argument("--rows", type=int, default=8192)
    f.add_argument("--f", type=int, default=3072)
    f.add_argument("--d", type=int, default=1024)
    f.add_argument("--reps", type=int, default=8)
    f.add_argument("--profile", action="store_true")
    e = sub.add_parser("decode")
    e.add_argument("--prompt", type=int, default=128)
    e.add_argument("--new-tokens", type=int, default=64)
    args = ap.parse_args()
    if args.cmd == "decode":
        decode(args.prompt, args.new_tokens)
        return
    if args.cmd == "swiglu":
        swiglu_gemms(args.rows, args.f, args.d, args.reps, args.profile)
        return
    if args.cmd == "mm-sweep":
        mm_sweep(args.reps)
    elif args.cmd == "attn-bwd":
        attn_bwd(args.seq, args.reps, args.modes, args.batch)
    elif args.cmd == "bw":
        bandwidth_kernels(args.tokens, args.reps, args.kernels)
    else:
        one_gemm(args.op, args.m, args.n, args.k, args.reps, args.out)


if __name__ == "__main__":
    main()
