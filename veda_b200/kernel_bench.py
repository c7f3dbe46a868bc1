"""Isolated kernel timings through the C ABI (CUDA events on one stream, inputs larger than L2).

    python -m veda_b200.kernel_bench mm-sweep [--reps 10]
        the matmul-backward sweep: for X[M,K], W[K,N], dY[M,N] (bf16, ~N(0,1)/sqrt(K), seed 1)
        time dX = dY W^T and dW = X^T dY (fp32 out) for (M,K,N) in the five sweep shapes;
        4*M*K*N FLOP per shape.
    python -m veda_b200.kernel_bench attn-bwd [--seq 1024 4096] [--reps 5]
        causal GQA attention backward, B 8, H 16, Hkv 8, Dh 128, bf16, seed 2; 5*B*H*T^2*Dh FLOP.
    python -m veda_b200.kernel_bench gemm --op nt --m 8192 --n 151936 --k 1024 [--reps 3]
        one GEMM shape (used for the ncu captures).
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
    import torch
    fn()
    torch.cuda.synchronize()
    total = 0.0
    for _ in range(reps):
        if flush is not None:
            flush.zero_()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record(stream)
        fn()
        b.record(stream)
        b.synchronize()
        total += a.elapsed_time(b)
    return total / reps


def mm_sweep(reps):
    import torch
    import veda_b200 as V
    L = V.lib()
    s = torch.cuda.current_stream()
    peak, _, kind = _peaks()
    flush = torch.empty(256 << 20, dtype=torch.uint8, device="cuda")   # > L2, cleared per rep
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
        ms = _time(run, reps, s, flush)
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


def attn_bwd(seqs, reps):
    import torch
    import veda_b200 as V
    L = V.lib()
    s = torch.cuda.current_stream()
    peak, _, kind = _peaks()
    B, H, Hk, Dh = 8, 16, 8, 128
    g = torch.Generator(device="cuda").manual_seed(2)
    for T in seqs:
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
        print(json.dumps({"bench": "attn", "B": B, "H": H, "Hkv": Hk, "Dh": Dh, "T": T,
                          "bwd_ms": ms_b, "bwd_tflops": fl_b / (ms_b / 1e3) / 1e12,
                          "fwd_ms": ms_f, "fwd_tflops": fl_f / (ms_f / 1e3) / 1e12,
                          "peak": peak, "bwd_frac": fl_b / (ms_b / 1e3) / 1e12 / peak,
                          "peak_kind": f"{kind} bf16 burst"}), flush=True)
        del q, k, v, do, o, lse, dq, dk, dv, ws
        torch.cuda.empty_cache()


def one_gemm(op, M, N, K, reps):
    import torch
    import veda_b200 as V
    L = V.lib()
    s = torch.cuda.current_stream()
    a = torch.randn(*((K, M) if op == "tn" else (M, K)), device="cuda").to(torch.bfloat16)
    b = torch.randn(*((N, K) if op == "nt" else (K, N)), device="cuda").to(torch.bfloat16)
    c = torch.empty(M, N, dtype=torch.bfloat16 if op == "nt" else torch.float32, device="cuda")
    dc = V.BF16 if op == "nt" else V.F32
    fn = getattr(L, f"veda_gemm_{op}")

    def run():
        V.check(fn(M, N, K, a.data_ptr(), a.shape[1], b.data_ptr(), b.shape[1], c.data_ptr(), N,
                   V.BF16, dc, 1.0, 0.0, s.cuda_stream))
    ms = _time(run, reps, s)
    tf = 2.0 * M * N * K / (ms / 1e3) / 1e12
    print(json.dumps({"bench": "gemm", "op": op, "M": M, "N": N, "K": K, "ms": ms, "tflops": tf}),
          flush=True)


def main():
    ap = argparse.ArgumentParser()
    sub = ap.add_subparsers(dest="cmd", required=True)
    a = sub.add_parser("mm-sweep")
    a.add_argument("--reps", type=int, default=10)
    b = sub.add_parser("attn-bwd")
    b.add_argument("--seq", type=int, nargs="+", default=[1024, 4096])
    b.add_argument("--reps", type=int, default=5)
    c = sub.add_parser("gemm")
    c.add_argument("--op", default="nt", choices=["nt", "nn", "tn"])
    c.add_argument("--m", type=int, default=8192)
    c.add_argument("--n", type=int, default=151936)
    c.add_argument("--k", type=int, default=1024)
    c.add_argument("--reps", type=int, default=3)
    args = ap.parse_args()
    if args.cmd == "mm-sweep":
        mm_sweep(args.reps)
    elif args.cmd == "attn-bwd":
        attn_bwd(args.seq, args.reps)
    else:
        one_gemm(args.op, args.m, args.n, args.k, args.reps)


if __name__ == "__main__":
    main()
