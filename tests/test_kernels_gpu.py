"""Parity of every kernel behind include/veda_cuda.h with the oracle, through the C ABI.

Tolerances (max-abs-relative error per tensor): 1e-4 for fp32, 2e-2 for bf16; integer and index
work (gathers, deterministic scatter, argmax) and the AdamW update on equal gradients are
compared bit for bit."""
import math

import numpy as np
import pytest

import veda_b200 as V
from oracle import veda_oracle as O
from tests.gpu_util import (bf, call, dev, empty, host, ptr, rel, stream, sync, torch, workspace,
                            zeros)

pytestmark = pytest.mark.gpu
F32 = np.float32
TOL = {V.F32: 1e-4, V.BF16: 2e-2}


@pytest.fixture(autouse=True)
def _lib(cuda):
    yield


def rng(seed):
    return np.random.default_rng(seed)


# ---------------------------------------------------------------------------------------------
# RMSNorm
# ---------------------------------------------------------------------------------------------
@pytest.mark.parametrize("dtype,rows,n", [(V.F32, 128, 64), (V.F32, 37, 100), (V.BF16, 8192, 1024),
                                          (V.BF16, 33, 2048), (V.F32, 8192, 1024),
                                          (V.BF16, 1001, 512), (V.F32, 77, 2048),
                                          (V.BF16, 300, 256), (V.BF16, 20001, 1024)])
def test_rmsnorm_fwd_bwd(dtype, rows, n):
    r = rng(rows + n)
    x = r.standard_normal((rows, n)).astype(F32)
    gam = (1 + 0.1 * r.standard_normal(n)).astype(F32)
    g = r.standard_normal((rows, n)).astype(F32)
    res = r.standard_normal((rows, n)).astype(F32)
    if dtype == V.BF16:
        x, gam, g, res = bf(x), bf(gam), bf(g), bf(res)
    y_ref, _, _ = O.rms_norm_gamma(x, gam, 1e-6)
    dx_ref, dgam_ref = O.rms_norm_gamma_backward(x, gam, g, 1e-6)
    dx_ref = dx_ref + res
    dx_, gam_, g_, res_ = dev(x, dtype), dev(gam, dtype), dev(g, dtype), dev(res, dtype)
    y = empty((rows, n), dtype)
    call("veda_rmsnorm_fwd", ptr(dx_), n, ptr(gam_), ptr(y), n, rows, n, 1e-6, dtype, stream())
    dx = empty((rows, n), dtype)
    dgam = dev(np.full(n, 0.5, F32))   # accumulates onto an existing gradient
    ws = workspace(V.lib().veda_rmsnorm_bwd_workspace(rows, n))
    call("veda_rmsnorm_bwd", ptr(dx_), n, ptr(gam_), ptr(g_), n, ptr(res_), n, ptr(dx), n,
         ptr(dgam), ptr(ws), ws.numel(), rows, n, 1e-6, dtype, stream())
    sync()
    assert rel(host(y), y_ref) <= TOL[dtype]
    assert rel(host(dx), dx_ref) <= TOL[dtype]
    assert rel(host(dgam), dgam_ref + 0.5) <= (1e-4 if dtype == V.F32 else 1e-3)


@pytest.mark.parametrize("dtype,rows,n", [(V.BF16, 1001, 1024), (V.BF16, 77, 2048),
                                          (V.BF16, 9, 256), (V.BF16, 5, 300), (V.F32, 33, 512)])
def test_add_rmsnorm_fwd(dtype, rows, n):
    """The residual add fused with the next norm: the sum is the add's result exactly (fp32 add
    rounded to the dtype, Variable.cpp:195-216) and the output is the norm of that sum."""
    r = rng(rows * 3 + n)
    x = r.standard_normal((rows, n)).astype(F32)
    res = r.standard_normal((rows, n)).astype(F32)
    gam = (1 + 0.1 * r.standard_normal(n)).astype(F32)
    if dtype == V.BF16:
        x, res, gam = bf(x), bf(res), bf(gam)
    s_ref = x + res
    if dtype == V.BF16:
        s_ref = bf(s_ref)
    y_ref, _, _ = O.rms_norm_gamma(s_ref, gam, 1e-6)
    xd, rd, gd = dev(x, dtype), dev(res, dtype), dev(gam, dtype)
    total, y = empty((rows, n), dtype), empty((rows, n), dtype)
    call("veda_add_rmsnorm_fwd", ptr(xd), n, ptr(rd), n, ptr(gd), ptr(total), n, ptr(y), n, rows,
         n, 1e-6, dtype, stream())
    sync()
    assert np.array_equal(host(total), s_ref)
    assert rel(host(y), y_ref) <= TOL[dtype]


@pytest.mark.parametrize("with_dgamma", [True, False])
def test_rmsnorm_bwd_without_residual(with_dgamma):
    """The backward without a residual gradient, with and without the gain gradient."""
    rows, n = 515, 1024
    r = rng(71)
    x = bf(r.standard_normal((rows, n)).astype(F32))
    gam = bf((1 + 0.1 * r.standard_normal(n)).astype(F32))
    g = bf(r.standard_normal((rows, n)).astype(F32))
    dx_ref, dgam_ref = O.rms_norm_gamma_backward(x, gam, g, 1e-6)
    xd, gamd, gd = dev(x, V.BF16), dev(gam, V.BF16), dev(g, V.BF16)
    dx = empty((rows, n), V.BF16)
    dgam = zeros(n) if with_dgamma else None
    ws = workspace(V.lib().veda_rmsnorm_bwd_workspace(rows, n)) if with_dgamma else None
    call("veda_rmsnorm_bwd", ptr(xd), n, ptr(gamd), ptr(gd), n, None, 0, ptr(dx), n,
         ptr(dgam) if with_dgamma else None, ptr(ws) if with_dgamma else None,
         ws.numel() if with_dgamma else 0, rows, n, 1e-6, V.BF16, stream())
    sync()
    assert rel(host(dx), dx_ref) <= TOL[V.BF16]
    if with_dgamma:
        assert rel(host(dgam), dgam_ref) <= 1e-3


def test_rmsnorm_plain_matches_golden():
    from pathlib import Path
    ops = np.load(Path(__file__).parent / "golden" / "ops_small.npz")
    x, gam, g = ops["rms_x"], ops["rms_gamma"], ops["rms_g"]
    rows, n = x.shape
    y = empty((rows, n))
    dx = empty((rows, n))
    dgam = zeros(n)
    xd, gd, gg = dev(x), dev(gam), dev(g)
    call("veda_rmsnorm_fwd", ptr(xd), n, ptr(gd), ptr(y), n, rows, n, 1e-6, V.F32, stream())
    ws = workspace(V.lib().veda_rmsnorm_bwd_workspace(rows, n))
    call("veda_rmsnorm_bwd", ptr(xd), n, ptr(gd), ptr(gg), n, None, 0, ptr(dx), n, ptr(dgam),
         ptr(ws), ws.numel(), rows, n, 1e-6, V.F32, stream())
    sync()
    assert rel(host(y), ops["rms_y"]) <= 1e-6
    assert rel(host(dx), ops["rms_dx"]) <= 1e-5
    assert rel(host(dgam), ops["rms_dgamma"]) <= 1e-5


# ---------------------------------------------------------------------------------------------
# QK-norm + RoPE
# ---------------------------------------------------------------------------------------------
@pytest.mark.parametrize("dtype,B,T,H,Dh,theta", [(V.F32, 4, 32, 4, 16, 1e4),
                                                 (V.BF16, 2, 256, 16, 128, 1e6),
                                                 (V.BF16, 3, 100, 3, 128, 1e6),
                                                 (V.F32, 1, 64, 8, 128, 1e6),
                                                 # many rows per warp: positions and heads stepped
                                                 # across the sequence and token boundaries
                                                 (V.BF16, 8, 2048, 8, 128, 1e6),
                                                 (V.BF16, 40, 100, 3, 128, 1e6)])
def test_qknorm_rope(dtype, B, T, H, Dh, theta):
    r = rng(T + H)
    N = B * T
    ld = H * Dh + 8 * 3  # a column slice of a wider fused buffer
    buf = r.standard_normal((N, ld)).astype(F32)
    if dtype == V.BF16:
        buf = bf(buf)
    gam = (1 + 0.1 * r.standard_normal(Dh)).astype(F32)
    if dtype == V.BF16:
        gam = bf(gam)
    g = r.standard_normal((N, H * Dh)).astype(F32)
    if dtype == V.BF16:
        g = bf(g)
    x = buf[:, 8:8 + H * Dh]
    cos, sin = O.rope_tables(T, Dh, theta)
    xh = x.reshape(B, T, H, Dh).transpose(0, 2, 1, 3)
    gh = g.reshape(B, T, H, Dh).transpose(0, 2, 1, 3)
    yn, _, _ = O.rms_norm_gamma(xh, gam, 1e-6)
    y_ref = O.rope(yn, cos, sin).transpose(0, 2, 1, 3).reshape(N, H * Dh)
    dyn = O.rope_backward(gh, cos, sin)
    dx_ref, dgam_ref = O.rms_norm_gamma_backward(xh, gam, dyn, 1e-6)
    dx_ref = dx_ref.transpose(0, 2, 1, 3).reshape(N, H * Dh)
    bufd = dev(buf, dtype)
    base = bufd.data_ptr() + 8 * (2 if dtype == V.BF16 else 4)
    gamd, gd = dev(gam, dtype), dev(g, dtype)
    cd, sd = dev(cos), dev(sin)
    y = empty((N, H * Dh), dtype)
    call("veda_qknorm_rope_fwd", base, ld, ptr(gamd), ptr(cd), ptr(sd), ptr(y), H * Dh, N, H, T,
         Dh, 1e-6, dtype, stream())
    dx = empty((N, H * Dh), dtype)
    dgam = zeros(Dh)
    ws = workspace(V.lib().veda_qknorm_rope_bwd_workspace(N, H, Dh))
    call("veda_qknorm_rope_bwd", base, ld, ptr(gamd), ptr(cd), ptr(sd), ptr(gd), H * Dh, ptr(dx),
         H * Dh, ptr(dgam), ptr(ws), ws.numel(), N, H, T, Dh, 1e-6, dtype, stream())
    sync()
    assert rel(host(y), y_ref) <= TOL[dtype]
    assert rel(host(dx), dx_ref) <= TOL[dtype]
    assert rel(host(dgam), dgam_ref) <= (1e-4 if dtype == V.F32 else 1e-3)


@pytest.mark.parametrize("dtype,B,T,H,Hk", [(V.BF16, 4, 2048, 16, 8), (V.BF16, 3, 100, 6, 2),
                                             (V.F32, 2, 64, 4, 2)])
def test_qknorm_rope_fwd_q_and_k_in_one_launch(dtype, B, T, H, Hk):
    """veda_qknorm_rope_fwd_qk (the q and k heads of a layer in one launch) equals two
    veda_qknorm_rope_fwd calls bit for bit."""
    r = rng(3 * T + H)
    Dh, N = 128, B * T
    W = (H + 2 * Hk) * Dh
    buf = r.standard_normal((N, W)).astype(F32)
    qg = (1 + 0.1 * r.standard_normal(Dh)).astype(F32)
    kg = (1 + 0.1 * r.standard_normal(Dh)).astype(F32)
    if dtype == V.BF16:
        buf, qg, kg = bf(buf), bf(qg), bf(kg)
    cos, sin = O.rope_tables(T, Dh, 1e6)
    es = 2 if dtype == V.BF16 else 4
    bufd, qgd, kgd, cd, sd = dev(buf, dtype), dev(qg, dtype), dev(kg, dtype), dev(cos), dev(sin)
    xq, xk = bufd.data_ptr(), bufd.data_ptr() + H * Dh * es
    yq, yk = empty((N, H * Dh), dtype), empty((N, Hk * Dh), dtype)
    call("veda_qknorm_rope_fwd_qk", xq, xk, W, ptr(qgd), ptr(kgd), ptr(cd), ptr(sd), ptr(yq), H * Dh,
         ptr(yk), Hk * Dh, N, H, Hk, T, Dh, 1e-6, dtype, stream())
    yq2, yk2 = empty((N, H * Dh), dtype), empty((N, Hk * Dh), dtype)
    call("veda_qknorm_rope_fwd", xq, W, ptr(qgd), ptr(cd), ptr(sd), ptr(yq2), H * Dh, N, H, T, Dh, 1e-6,
         dtype, stream())
    call("veda_qknorm_rope_fwd", xk, W, ptr(kgd), ptr(cd), ptr(sd), ptr(yk2), Hk * Dh, N, Hk, T, Dh, 1e-6,
         dtype, stream())
    sync()
    assert np.array_equal(host(yq), host(yq2))
    assert np.array_equal(host(yk), host(yk2))


@pytest.mark.parametrize("dtype,B,T,H,Hk,with_k_gain", [(V.BF16, 2, 256, 16, 8, True),
                                                        (V.BF16, 4, 2048, 16, 8, True),
                                                        (V.BF16, 3, 100, 6, 2, False),
                                                        (V.F32, 2, 64, 4, 2, True)])
def test_qknorm_rope_bwd_q_and_k_in_one_launch(dtype, B, T, H, Hk, with_k_gain):
    """veda_qknorm_rope_bwd_qk (the q and k heads of a layer in one launch) against two
    veda_qknorm_rope_bwd calls: dx bit for bit, the gain gradients to rounding; and the oracle."""
    r = rng(7 * T + H + Hk)
    Dh = 128
    N = B * T
    W = (H + 2 * Hk) * Dh   # the fused q|k|v projection
    buf = r.standard_normal((N, W)).astype(F32)
    qg = (1 + 0.1 * r.standard_normal(Dh)).astype(F32)
    kg = (1 + 0.1 * r.standard_normal(Dh)).astype(F32)
    gq = r.standard_normal((N, H * Dh)).astype(F32)
    gk = r.standard_normal((N, Hk * Dh)).astype(F32)
    if dtype == V.BF16:
        buf, qg, kg, gq, gk = bf(buf), bf(qg), bf(kg), bf(gq), bf(gk)
    cos, sin = O.rope_tables(T, Dh, 1e6)
    es = 2 if dtype == V.BF16 else 4
    bufd = dev(buf, dtype)
    xq, xk = bufd.data_ptr(), bufd.data_ptr() + H * Dh * es
    qgd, kgd, gqd, gkd = dev(qg, dtype), dev(kg, dtype), dev(gq, dtype), dev(gk, dtype)
    cd, sd = dev(cos), dev(sin)
    lib = V.lib()
    # one launch: results into the q and k columns of one fused gradient
    dx = empty((N, W), dtype)
    dqg, dkg = dev(np.full(Dh, 0.25, F32)), dev(np.full(Dh, -0.5, F32))
    ws = workspace(lib.veda_qknorm_rope_bwd_qk_workspace(N, H, Hk, Dh))
    call("veda_qknorm_rope_bwd_qk", xq, xk, W, ptr(qgd), ptr(kgd), ptr(cd), ptr(sd), ptr(gqd), H * Dh,
         0, 1.0, ptr(gkd), Hk * Dh, ptr(dx), ptr(dx) + H * Dh * es, W, ptr(dqg),
         ptr(dkg) if with_k_gain else None, ptr(ws), ws.numel(), N, H, Hk, T, Dh, 1e-6, dtype, stream())
    # two calls
    dxq, dxk = empty((N, H * Dh), dtype), empty((N, Hk * Dh), dtype)
    dqg2, dkg2 = dev(np.full(Dh, 0.25, F32)), dev(np.full(Dh, -0.5, F32))
    for x0, gd, g0, nh, out, dg in ((xq, qgd, gqd, H, dxq, dqg2), (xk, kgd, gkd, Hk, dxk, dkg2)):
        w1 = workspace(lib.veda_qknorm_rope_bwd_workspace(N, nh, Dh))
        call("veda_qknorm_rope_bwd", x0, W, ptr(gd), ptr(cd), ptr(sd), ptr(g0), nh * Dh, ptr(out), nh * Dh,
             ptr(dg) if (dg is dqg2 or with_k_gain) else None, ptr(w1), w1.numel(), N, nh, T, Dh, 1e-6,
             dtype, stream())
    sync()
    got = host(dx)
    assert np.array_equal(got[:, :H * Dh], host(dxq))
    assert np.array_equal(got[:, H * Dh:(H + Hk) * Dh], host(dxk))
    assert rel(host(dqg), host(dqg2)) <= 1e-5
    assert rel(host(dkg), host(dkg2)) <= 1e-5
    if not with_k_gain:
        assert np.array_equal(host(dkg), np.full(Dh, -0.5, F32))
    # the oracle, per set
    for x, g, gam, nh, got_x, got_g, base in ((buf[:, :H * Dh], gq, qg, H, got[:, :H * Dh], dqg, 0.25),
                                               (buf[:, H * Dh:(H + Hk) * Dh], gk, kg, Hk,
                                                got[:, H * Dh:(H + Hk) * Dh], dkg, -0.5)):
        xh = x.reshape(B, T, nh, Dh).transpose(0, 2, 1, 3)
        gh = g.reshape(B, T, nh, Dh).transpose(0, 2, 1, 3)
        dyn = O.rope_backward(gh, cos, sin)
        dx_ref, dg_ref = O.rms_norm_gamma_backward(xh, gam, dyn, 1e-6)
        assert rel(got_x, dx_ref.transpose(0, 2, 1, 3).reshape(N, nh * Dh)) <= TOL[dtype]
        if base > 0 or with_k_gain:
            assert rel(host(got_g), dg_ref + base) <= (1e-4 if dtype == V.F32 else 1e-3)


def test_rope_plain_matches_golden():
    from pathlib import Path
    ops = np.load(Path(__file__).parent / "golden" / "ops_small.npz")
    x, g = ops["rope_x"], ops["rope_g"]
    lanes, T, Dh = x.shape
    cd, sd = dev(ops["rope_cos"]), dev(ops["rope_sin"])
    y, dx = empty(x.shape), empty(x.shape)
    call("veda_rope", ptr(dev(x)), ptr(y), ptr(cd), ptr(sd), lanes, T, Dh, 0, V.F32, stream())
    call("veda_rope", ptr(dev(g)), ptr(dx), ptr(cd), ptr(sd), lanes, T, Dh, 1, V.F32, stream())
    sync()
    assert rel(host(y), ops["rope_y"]) <= 1e-6
    assert rel(host(dx), ops["rope_dx"]) <= 1e-6


# ---------------------------------------------------------------------------------------------
# SwiGLU
# ---------------------------------------------------------------------------------------------
@pytest.mark.parametrize("dtype,rows,F", [(V.F32, 128, 192), (V.BF16, 4096, 3072), (V.F32, 7, 13)])
def test_swiglu(dtype, rows, F):
    r = rng(F)
    gu = (2 * r.standard_normal((rows, 2 * F))).astype(F32)
    dh = r.standard_normal((rows, F)).astype(F32)
    if dtype == V.BF16:
        gu, dh = bf(gu), bf(dh)
    gate, up = gu[:, :F], gu[:, F:]
    h_ref = O.swiglu(gate, up)
    dg_ref, du_ref = O.swiglu_backward(gate, up, dh)
    gud, dhd = dev(gu, dtype), dev(dh, dtype)
    es = 2 if dtype == V.BF16 else 4
    h = empty((rows, F), dtype)
    call("veda_swiglu_fwd", ptr(gud), 2 * F, gud.data_ptr() + F * es, 2 * F, ptr(h), F, rows, F,
         dtype, stream())
    dgu = empty((rows, 2 * F), dtype)
    call("veda_swiglu_bwd", ptr(gud), 2 * F, gud.data_ptr() + F * es, 2 * F, ptr(dhd), F,
         ptr(dgu), 2 * F, dgu.data_ptr() + F * es, 2 * F, rows, F, dtype, stream())
    sync()
    out = host(dgu)
    assert rel(host(h), h_ref) <= TOL[dtype]
    assert rel(out[:, :F], dg_ref) <= TOL[dtype]
    assert rel(out[:, F:], du_ref) <= TOL[dtype]


# The MLP's projections with SwiGLU fused into their GEMMs give the bits of the GEMM followed by
# the stand-alone SwiGLU kernel: the Qwen3-0.6B shape, and ragged rows and K.
@pytest.mark.parametrize("rows,F,D", [(8192, 3072, 1024), (300, 256, 64), (1000, 384, 136)])
def test_gemm_swiglu_fwd_is_gemm_then_swiglu(rows, F, D):
    t = torch()
    g = t.Generator(device="cuda").manual_seed(rows + F + D)
    x = t.randn(rows, D, device="cuda", generator=g).to(t.bfloat16)
    w = (t.randn(2 * F, D, device="cuda", generator=g) / math.sqrt(D)).to(t.bfloat16)
    gu_ref, h_ref = empty((rows, 2 * F), V.BF16), empty((rows, F), V.BF16)
    call("veda_gemm_nt", rows, 2 * F, D, ptr(x), D, ptr(w), D, ptr(gu_ref), 2 * F, V.BF16, V.BF16,
         1.0, 0.0, stream())
    call("veda_swiglu_fwd", ptr(gu_ref), 2 * F, gu_ref.data_ptr() + 2 * F, 2 * F, ptr(h_ref), F,
         rows, F, V.BF16, stream())
    gu, h = empty((rows, 2 * F), V.BF16), empty((rows, F), V.BF16)
    call("veda_gemm_swiglu_fwd", rows, F, D, ptr(x), D, ptr(w), D, ptr(gu), 2 * F, ptr(h), F,
         stream())
    sync()
    assert t.equal(gu, gu_ref)
    assert t.equal(h, h_ref)


@pytest.mark.parametrize("rows,F,D", [(8192, 3072, 1024), (300, 256, 64), (1000, 512, 136)])
def test_gemm_swiglu_bwd_is_gemm_then_swiglu_bwd(rows, F, D):
    t = torch()
    g = t.Generator(device="cuda").manual_seed(rows * 3 + F + D)
    dy = t.randn(rows, D, device="cuda", generator=g).to(t.bfloat16)
    w = (t.randn(D, F, device="cuda", generator=g) / math.sqrt(F)).to(t.bfloat16)
    gu = (2 * t.randn(rows, 2 * F, device="cuda", generator=g)).to(t.bfloat16)
    dh, dgu_ref = empty((rows, F), V.BF16), empty((rows, 2 * F), V.BF16)
    call("veda_gemm_nn", rows, F, D, ptr(dy), D, ptr(w), F, ptr(dh), F, V.BF16, V.BF16, 1.0, 0.0,
         stream())
    call("veda_swiglu_bwd", ptr(gu), 2 * F, gu.data_ptr() + 2 * F, 2 * F, ptr(dh), F, ptr(dgu_ref),
         2 * F, dgu_ref.data_ptr() + 2 * F, 2 * F, rows, F, V.BF16, stream())
    dgu = empty((rows, 2 * F), V.BF16)
    call("veda_gemm_swiglu_bwd", rows, F, D, ptr(dy), D, ptr(w), F, ptr(gu), 2 * F, ptr(dgu), 2 * F,
         stream())
    sync()
    assert t.equal(dgu, dgu_ref)


def test_gemm_swiglu_rejects_what_it_cannot_tile():
    a = empty((512, 512), V.BF16)
    L = V.lib()
    # F not a multiple of 128 (forward) or 256 (backward), fewer than 256 rows: nothing runs
    assert L.veda_gemm_swiglu_fwd(300, 200, 64, ptr(a), 64, ptr(a), 64, ptr(a), 400, ptr(a), 200,
                                  stream()) == -4
    assert L.veda_gemm_swiglu_bwd(300, 128, 64, ptr(a), 64, ptr(a), 128, ptr(a), 256, ptr(a), 256,
                                  stream()) == -4
    assert L.veda_gemm_swiglu_fwd(200, 128, 64, ptr(a), 64, ptr(a), 64, ptr(a), 256, ptr(a), 128,
                                  stream()) == -4
    sync()


# ---------------------------------------------------------------------------------------------
# Cross-entropy
# ---------------------------------------------------------------------------------------------
# rows of >= 128 KB take the cluster form (a row split over 8 CTAs); (BF16, 37, 65544) leaves the
# last CTA a shorter slice, (BF16, 3, 70001) is not a whole number of 16-byte vectors (one-CTA
# form), and 1000 rows make every cluster loop over several rows
@pytest.mark.parametrize("dtype,rows,Vv,inplace", [(V.F32, 128, 512, False), (V.F32, 9, 77, False),
                                                   (V.BF16, 64, 151936, False),
                                                   (V.F32, 16, 151936, False),
                                                   (V.BF16, 1000, 151936, True),
                                                   (V.BF16, 37, 65544, True),
                                                   (V.BF16, 3, 70001, False)])
def test_cross_entropy(dtype, rows, Vv, inplace):
    r = rng(rows * 7 + Vv)
    lg = (3 * r.standard_normal((rows, Vv))).astype(F32)
    if dtype == V.BF16:
        lg = bf(lg)
    t = r.integers(0, Vv, rows).astype(np.int64)
    loss_ref, d_ref = O.cross_entropy(lg, t)
    rows_ref = O.cross_entropy_rows(lg, t)
    lgd, td = dev(lg, dtype), dev(t)
    row_loss = empty(rows)
    d = lgd if inplace else lgd.clone()
    status = zeros(1).int()
    call("veda_cross_entropy", ptr(lgd), Vv, ptr(td), ptr(row_loss), ptr(d), Vv, rows, Vv,
         1.0 / rows, ptr(status), dtype, stream())
    mean = empty(1)
    call("veda_mean_f64", ptr(row_loss), rows, ptr(mean), None, stream())
    sync()
    assert int(host(status)[0]) == 0
    assert rel(host(row_loss), rows_ref) <= 1e-5
    assert abs(float(host(mean)[0]) - loss_ref) <= 1e-5 * abs(loss_ref)
    assert rel(host(d), d_ref) <= TOL[dtype]


def test_cross_entropy_golden_and_out_of_range():
    from pathlib import Path
    ops = np.load(Path(__file__).parent / "golden" / "ops_small.npz")
    lg, t = ops["ce_logits"], ops["ce_targets"]
    rows, Vv = lg.shape
    lgd, td = dev(lg), dev(t)
    row_loss, d, mean = empty(rows), empty((rows, Vv)), empty(1)
    status = zeros(1).int()
    call("veda_cross_entropy", ptr(lgd), Vv, ptr(td), ptr(row_loss), ptr(d), Vv, rows, Vv,
         1.0 / rows, ptr(status), V.F32, stream())
    call("veda_mean_f64", ptr(row_loss), rows, ptr(mean), None, stream())
    sync()
    assert abs(float(host(mean)[0]) - float(ops["ce_loss"][0])) <= 1e-6
    assert rel(host(d), ops["ce_dlogits"]) <= 1e-6
    bad = t.copy()
    bad[3] = Vv
    call("veda_cross_entropy", ptr(lgd), Vv, ptr(dev(bad)), ptr(row_loss), ptr(d), Vv, rows, Vv,
         1.0, ptr(status), V.F32, stream())
    sync()
    assert int(host(status)[0]) == V.ERR_OUT_OF_RANGE


def test_cross_entropy_cluster_out_of_range_target():
    rows, Vv = 6, 151936
    r = rng(11)
    lg = bf((3 * r.standard_normal((rows, Vv))).astype(F32))
    t = r.integers(0, Vv, rows).astype(np.int64)
    t[2] = -1
    ok = np.arange(rows) != 2
    rows_ref = O.cross_entropy_rows(lg[ok], t[ok])
    lgd, td = dev(lg, V.BF16), dev(t)
    row_loss, status = empty(rows), zeros(1).int()
    d = lgd.clone()
    call("veda_cross_entropy", ptr(lgd), Vv, ptr(td), ptr(row_loss), ptr(d), Vv, rows, Vv,
         1.0 / rows, ptr(status), V.BF16, stream())
    sync()
    assert int(host(status)[0]) == V.ERR_OUT_OF_RANGE
    got = host(row_loss)
    assert np.isnan(got[2])
    assert rel(got[ok], rows_ref) <= 1e-5


# ---------------------------------------------------------------------------------------------
# Embedding
# ---------------------------------------------------------------------------------------------
@pytest.mark.parametrize("dtype,count,Vv,D", [(V.F32, 128, 512, 64), (V.BF16, 8192, 151936, 1024),
                                              (V.F32, 20000, 300, 24)])
def test_embedding(dtype, count, Vv, D):
    r = rng(count + D)
    table = r.standard_normal((Vv, D)).astype(F32)
    if dtype == V.BF16:
        table = bf(table)
    ids = r.integers(0, min(Vv, max(8, count // 4)), count).astype(np.int64)  # many repeats
    g = r.standard_normal((count, D)).astype(F32)
    if dtype == V.BF16:
        g = bf(g)
    start = r.standard_normal((Vv, D)).astype(F32)   # e.g. the tied LM-head contribution
    out_ref = O.embedding(table, ids)
    dt_ref = O.embedding_backward(start.copy(), ids, g)
    tabd, idd, gd = dev(table, dtype), dev(ids), dev(g, dtype)
    out = empty((count, D), dtype)
    status = zeros(1).int()
    call("veda_embedding_fwd", ptr(idd), count, ptr(tabd), Vv, D, ptr(out), D, ptr(status), dtype,
         stream())
    dt = dev(start)
    ws = workspace(V.lib().veda_embedding_bwd_workspace(count))
    call("veda_embedding_bwd", ptr(idd), count, ptr(gd), D, Vv, D, ptr(dt), 1, ptr(ws), ws.numel(),
         dtype, stream())
    dta = dev(start)
    call("veda_embedding_bwd", ptr(idd), count, ptr(gd), D, Vv, D, ptr(dta), 0, None, 0, dtype,
         stream())
    sync()
    assert np.array_equal(host(out), out_ref), "gather must be bit-exact"
    assert np.array_equal(host(dt), dt_ref), "deterministic scatter must be bit-exact"
    assert rel(host(dta), dt_ref) <= 1e-5
    assert int(host(status)[0]) == 0
    call("veda_embedding_fwd", ptr(dev(np.array([0, Vv], np.int64))), 2, ptr(tabd), Vv, D,
         ptr(out), D, ptr(status), dtype, stream())
    sync()
    assert int(host(status)[0]) == V.ERR_OUT_OF_RANGE


# ---------------------------------------------------------------------------------------------
# Clip + AdamW
# ---------------------------------------------------------------------------------------------
def test_clip_kat_thirteen():
    g = dev(np.array([3.0, 4.0, 12.0], F32))
    ss = zeros(1).double()
    ws = workspace(V.lib().veda_sumsq_workspace(3))
    call("veda_sumsq", ptr(g), 3, ptr(ss), 0, ptr(ws), ws.numel(), stream())
    call("veda_clip_apply", ptr(g), 3, ptr(ss), 6.5, stream())
    sync()
    assert abs(math.sqrt(float(host(ss)[0])) - 13.0) < 1e-9
    np.testing.assert_allclose(host(g), [1.5, 2.0, 6.0], atol=1e-6)
    g2 = dev(np.array([3.0, 4.0, 12.0], F32))
    call("veda_sumsq", ptr(g2), 3, ptr(ss), 0, ptr(ws), ws.numel(), stream())
    call("veda_clip_apply", ptr(g2), 3, ptr(ss), 13.0, stream())
    sync()
    assert np.array_equal(host(g2), np.array([3.0, 4.0, 12.0], F32)), "no-op must be bitwise"


@pytest.mark.parametrize("n,clip", [(1000003, 1.0), (4096, 1e9)])
def test_adamw_bit_exact_with_clip(n, clip):
    r = rng(n)
    w = r.standard_normal(n).astype(F32)
    grads = [(r.standard_normal(n) * 0.01).astype(F32) for _ in range(3)]
    cfg = O.AdamWConfig(1e-3, 0.9, 0.95, 1e-8, 0.1)
    ref_w = w.copy()
    opt = O.AdamW([ref_w], cfg)
    wd, md, vd = dev(w), zeros(n), zeros(n)
    lowp = empty(n, V.BF16)
    ss = zeros(1).double()
    ws = workspace(V.lib().veda_sumsq_workspace(n))
    for s, g in enumerate(grads, start=1):
        gc = [g.copy()]
        O.clip_gradient_norm(gc, clip)
        opt.step(gc)
        gd = dev(g)
        call("veda_sumsq", ptr(gd), n, ptr(ss), 0, ptr(ws), ws.numel(), stream())
        b1 = 1.0 - math.pow(float(F32(0.9)), s)
        b2 = 1.0 - math.pow(float(F32(0.95)), s)
        call("veda_adamw_step", ptr(wd), ptr(md), ptr(vd), ptr(gd), ptr(lowp), n, 1e-3, 0.9, 0.95,
             1e-8, 0.1, b1, b2, ptr(ss), clip, 1.0, 1, stream())
        sync()
        assert np.array_equal(host(gd), gc[0]), "clipped gradient must equal the CPU's"
    assert np.array_equal(host(wd), ref_w), "AdamW on equal gradients must be bit-exact"
    assert np.array_equal(host(lowp), bf(ref_w))


def test_adamw_kat_point_nine():
    w, m, v, g = dev(np.array([1.0], F32)), zeros(1), zeros(1), dev(np.array([2.0], F32))
    call("veda_adamw_step", ptr(w), ptr(m), ptr(v), ptr(g), None, 1, 0.1, 0.9, 0.999, 1e-8, 0.0,
         1 - 0.9, 1 - 0.999, None, 1.0, 1.0, 0, stream())
    sync()
    assert abs(float(host(w)[0]) - 0.9) < 1e-5


# ---------------------------------------------------------------------------------------------
# GEMM
# ---------------------------------------------------------------------------------------------
def _gemm_case(op, M, N, K, dtype_c, seed, beta=0.0):
    r = rng(seed)
    a = bf(r.standard_normal((K, M) if op == "tn" else (M, K)).astype(F32) / math.sqrt(K))
    b = bf(r.standard_normal((N, K) if op == "nt" else (K, N)).astype(F32))
    c0 = r.standard_normal((M, N)).astype(F32)
    am = a.T if op == "tn" else a
    bm = b.T if op == "nt" else b
    ref = (am.astype(np.float64) @ bm.astype(np.float64)).astype(F32)
    if beta != 0.0:
        ref = ref + beta * (bf(c0) if dtype_c == V.BF16 else c0)
    ad, bd = dev(a, V.BF16), dev(b, V.BF16)
    c = dev(c0, dtype_c)
    lda = a.shape[1]
    ldb = b.shape[1]
    call(f"veda_gemm_{op}", M, N, K, ptr(ad), lda, ptr(bd), ldb, ptr(c), N, V.BF16, dtype_c, 1.0,
         beta, stream())
    sync()
    return host(c), ref


@pytest.mark.parametrize("op", ["nt", "nn", "tn"])
@pytest.mark.parametrize("M,N,K", [(128, 256, 64), (256, 512, 1024), (300, 200, 136),
                                   (4096, 1024, 1024), (128, 128, 8192)])
def test_gemm_bf16_fp32_out(op, M, N, K):
    c, ref = _gemm_case(op, M, N, K, V.F32, M + N + K)
    # fp32 accumulation of bf16 products against a float64 product of the same bf16 values
    assert rel(c, ref) <= 3e-5, rel(c, ref)


@pytest.mark.parametrize("op", ["nt", "nn", "tn"])
@pytest.mark.parametrize("M,N,K", [(300, 520, 200), (520, 776, 72), (256, 256, 8192),
                                   (1000, 1000, 1000)])
def test_gemm_cta_pair_tiles(op, M, N, K):
    """M, N >= 256 run as 256 x 256 tiles on CTA pairs: ragged edges in M, N and K, a split-K
    case (one tile, K = 8192), and the bf16 output of the same tiles."""
    c, ref = _gemm_case(op, M, N, K, V.F32, M * 7 + N + K)
    assert rel(c, ref) <= 3e-5, rel(c, ref)
    c, ref = _gemm_case(op, M, N, K, V.BF16, M * 7 + N + K + 1)
    assert rel(c, ref) <= 1e-2, rel(c, ref)


@pytest.mark.parametrize("op", ["nt", "nn", "tn"])
def test_gemm_bf16_out_and_accumulate(op):
    c, ref = _gemm_case(op, 512, 768, 320, V.BF16, 5)
    assert rel(c, ref) <= 1e-2
    c, ref = _gemm_case(op, 1024, 1024, 4096, V.F32, 6, beta=1.0)   # split-K path + accumulate
    assert rel(c, ref) <= 1e-5


def test_gemm_fp32_is_bit_exact_with_reference_loop(ref_lib):
    r = rng(9)
    a = r.standard_normal((70, 45)).astype(F32)
    b = r.standard_normal((33, 45)).astype(F32)
    want = ref_lib.gemm_nt(a, b)
    c = empty((70, 33))
    ad, bd = dev(a), dev(b)
    call("veda_gemm_nt", 70, 33, 45, ptr(ad), 45, ptr(bd), 45, ptr(c), 33, V.F32, V.F32,
         1.0, 0.0, stream())
    sync()
    assert np.array_equal(host(c), want)


@pytest.mark.parametrize("op", ["nt", "nn", "tn"])
def test_gemm_fp32_small_shapes(op):
    r = rng(3)
    M, N, K = 96, 40, 17
    a = r.standard_normal((K, M) if op == "tn" else (M, K)).astype(F32)
    b = r.standard_normal((N, K) if op == "nt" else (K, N)).astype(F32)
    am = a.T if op == "tn" else a
    bm = b.T if op == "nt" else b
    c = empty((M, N))
    ad, bd = dev(a), dev(b)
    call(f"veda_gemm_{op}", M, N, K, ptr(ad), a.shape[1], ptr(bd), b.shape[1], ptr(c), N,
         V.F32, V.F32, 1.0, 0.0, stream())
    sync()
    assert rel(host(c), am @ bm) <= 1e-6


@pytest.mark.parametrize("M,K,N", [(8192, 2048, 6144), (8192, 1024, 151936)])
def test_matmul_backward_sweep_shapes_against_fp64(M, K, N):
    """The two largest shapes of the isolated matmul-backward sweep: dX = dY W^T (NT) and
    dW = X^T dY (TN), bf16 inputs ~ N(0,1)/sqrt(K) (seed 1), fp32 outputs, checked against fp64
    products on a slab of dX rows and a slab of dW columns (src/libs/autograd/Variable.cpp:325-346
    is the reference's backward of matmul_nt)."""
    t = torch()
    g = t.Generator(device="cuda").manual_seed(1)
    x = (t.randn(M, K, device="cuda", generator=g) / math.sqrt(K)).to(t.bfloat16)
    w = (t.randn(K, N, device="cuda", generator=g) / math.sqrt(K)).to(t.bfloat16)
    dy = (t.randn(M, N, device="cuda", generator=g) / math.sqrt(K)).to(t.bfloat16)
    dx = t.empty(M, K, dtype=t.float32, device="cuda")
    dw = t.empty(K, N, dtype=t.float32, device="cuda")
    call("veda_gemm_nt", M, K, N, dy.data_ptr(), N, w.data_ptr(), N, dx.data_ptr(), K, V.BF16, V.F32,
         1.0, 0.0, stream())
    call("veda_gemm_tn", K, N, M, x.data_ptr(), K, dy.data_ptr(), N, dw.data_ptr(), N, V.BF16, V.F32,
         1.0, 0.0, stream())
    sync()
    rows = t.arange(0, M, M // 16, device="cuda")
    cols = t.arange(0, N, max(1, N // 64), device="cuda")
    ref_dx = (dy[rows].double() @ w.double().T).cpu().numpy()
    ref_dw = (x.double().T @ dy[:, cols].double()).cpu().numpy()
    assert rel(dx[rows].double().cpu().numpy(), ref_dx) <= 1e-4
    assert rel(dw[:, cols].double().cpu().numpy(), ref_dw) <= 1e-4


@pytest.mark.parametrize("op,dtype,M,N,K", [(0, V.BF16, 70, 136, 48), (1, V.BF16, 70, 136, 48),
                                            (2, V.BF16, 70, 136, 48), (1, V.F32, 70, 136, 48),
                                            (0, V.BF16, 256, 384, 128), (1, V.BF16, 256, 384, 128),
                                            (2, V.BF16, 256, 384, 128)])
def test_gemm_batched_against_oracle(op, dtype, M, N, K):
    """veda_gemm_batched, the products of autograd::matmul on batched operands (P.V of attention
    and its backward: src/libs/autograd/Variable.cpp:300-323), with an operand broadcast over the
    batch (stride 0, the weight of a batched matmul): every batch entry against numpy. Ragged
    shapes take the CUDA-core kernel, 16-byte-aligned ones the tensor-core kernel."""
    r = rng(21 + op)
    batch = 3
    shp_a = (batch, K, M) if op == 2 else (batch, M, K)
    shp_b = (N, K) if op == 0 else (K, N)        # broadcast over the batch
    a = r.standard_normal(shp_a).astype(F32)
    b = r.standard_normal(shp_b).astype(F32)
    c0 = r.standard_normal((batch, M, N)).astype(F32)
    if dtype == V.BF16:
        a, b = bf(a), bf(b)
    ad, bd = dev(a, dtype), dev(b, dtype)
    c = dev(c0)
    lda = shp_a[2]
    ldb = shp_b[1]
    call("veda_gemm_batched", op, batch, M, N, K, ptr(ad), lda, M * K, ptr(bd), ldb, 0, ptr(c), N,
         M * N, dtype, V.F32, 0.5, 1.0, stream())
    sync()
    am = np.transpose(a, (0, 2, 1)) if op == 2 else a
    bm = b.T if op == 0 else b
    want = 0.5 * (am.astype(np.float64) @ bm.astype(np.float64)) + c0
    assert rel(host(c), want) <= (1e-5 if dtype == V.F32 else 1e-4)


@pytest.mark.parametrize("dtype", [V.F32, V.BF16])
def test_scale_and_accumulate(dtype):
    """veda_scale (autograd::mul by a scalar, src/libs/autograd/Variable.cpp:241-258) and
    veda_accumulate (the gradient += of Variable.cpp:27-38), fp32 and bf16, ragged length."""
    r = rng(5)
    n = 100003
    x = r.standard_normal(n).astype(F32)
    d0 = r.standard_normal(n).astype(F32)
    if dtype == V.BF16:
        x = bf(x)
    xd = dev(x, dtype)
    out = empty(n, dtype)
    call("veda_scale", ptr(xd), 0.125, ptr(out), n, dtype, stream())
    dst = dev(d0)
    call("veda_accumulate", ptr(dst), V.F32, ptr(xd), dtype, n, stream())
    sync()
    want = x * np.float32(0.125)
    assert np.array_equal(host(out), bf(want) if dtype == V.BF16 else want)   # exact: a power of 2
    assert np.array_equal(host(dst), d0 + x)


# ---------------------------------------------------------------------------------------------
# Attention
# ---------------------------------------------------------------------------------------------
def _attention_case(dtype, B, T, H, Hk, Dh, seed):
    r = rng(seed)
    q = r.standard_normal((B, H, T, Dh)).astype(F32)
    k = r.standard_normal((B, Hk, T, Dh)).astype(F32)
    v = r.standard_normal((B, Hk, T, Dh)).astype(F32)
    do = r.standard_normal((B, H, T, Dh)).astype(F32)
    if dtype == V.BF16:
        q, k, v, do = bf(q), bf(k), bf(v), bf(do)
    o_ref, lse_ref, p = O.attention(q, k, v)
    dq_ref, dk_ref, dv_ref = O.attention_backward(q, k, v, p, do)
    tok = lambda a: np.ascontiguousarray(a.transpose(0, 2, 1, 3)).reshape(B * T, -1)  # noqa: E731
    qd, kd, vd, dod = dev(tok(q), dtype), dev(tok(k), dtype), dev(tok(v), dtype), dev(tok(do), dtype)
    o = empty((B * T, H * Dh), dtype)
    lse = empty(B * H * T)
    scale = 1.0 / math.sqrt(Dh)
    call("veda_attention_fwd", ptr(qd), H * Dh, ptr(kd), Hk * Dh, ptr(vd), Hk * Dh, ptr(o), H * Dh,
         ptr(lse), B, T, H, Hk, Dh, scale, 1, dtype, stream())
    # the backward runs on the reference's O (rounded like ours would be) to isolate its error
    od = dev(tok(o_ref), dtype)
    dq, dk, dv = empty((B * T, H * Dh), dtype), empty((B * T, Hk * Dh), dtype), empty((B * T, Hk * Dh), dtype)
    ws = workspace(V.lib().veda_attention_bwd_workspace(B, T, H, Hk, Dh, dtype))
    call("veda_attention_bwd", ptr(qd), H * Dh, ptr(kd), Hk * Dh, ptr(vd), Hk * Dh, ptr(od), H * Dh,
         ptr(dod), H * Dh, ptr(lse), ptr(dq), H * Dh, ptr(dk), Hk * Dh, ptr(dv), Hk * Dh, ptr(ws),
         ws.numel(), B, T, H, Hk, Dh, scale, 1, dtype, stream())
    sync()
    return (host(o), tok(o_ref), host(lse).reshape(B, H, T), lse_ref, host(dq), tok(dq_ref),
            host(dk), tok(dk_ref), host(dv), tok(dv_ref))


def test_attention_bwd_dq_f32_feeds_the_norm_backward():
    """veda_attention_bwd_dq_f32 leaves dQ unscaled in the fp32 accumulator of its workspace and
    writes dK, dV like veda_attention_bwd; the q+k norm backward reading that accumulator
    (dyq_f32, the attention scale) gives bit for bit what it gives on bf16(scale * accumulator),
    the dQ veda_attention_bwd would have written."""
    import torch as T_
    B, T, H, Hk, Dh = 2, 256, 16, 8, 128
    o, o_ref, lse, lse_ref, dq, dq_ref, dk, dk_ref, dv, dv_ref = _attention_case(V.BF16, B, T, H, Hk, Dh, 11)
    lib = V.lib()
    r = rng(11)   # the same inputs as _attention_case drew
    q = bf(r.standard_normal((B, H, T, Dh)).astype(F32))
    k = bf(r.standard_normal((B, Hk, T, Dh)).astype(F32))
    v = bf(r.standard_normal((B, Hk, T, Dh)).astype(F32))
    do = bf(r.standard_normal((B, H, T, Dh)).astype(F32))
    tok = lambda a: np.ascontiguousarray(a.transpose(0, 2, 1, 3)).reshape(B * T, -1)  # noqa: E731
    qd, kd, vd, dod = dev(tok(q), V.BF16), dev(tok(k), V.BF16), dev(tok(v), V.BF16), dev(tok(do), V.BF16)
    od, lsed = dev(o_ref, V.BF16), dev(lse_ref.reshape(-1).astype(F32))
    scale = 1.0 / math.sqrt(Dh)
    ws = workspace(lib.veda_attention_bwd_workspace(B, T, H, Hk, Dh, V.BF16))
    dk2, dv2 = empty((B * T, Hk * Dh), V.BF16), empty((B * T, Hk * Dh), V.BF16)
    call("veda_attention_bwd_dq_f32", ptr(qd), H * Dh, ptr(kd), Hk * Dh, ptr(vd), Hk * Dh, ptr(od), H * Dh,
         ptr(dod), H * Dh, ptr(lsed), ptr(dk2), Hk * Dh, ptr(dv2), Hk * Dh, ptr(ws), ws.numel(), B, T, H, Hk,
         Dh, scale, 1, V.BF16, stream())
    sync()
    off = lib.veda_attention_bwd_dq_offset(B, T, H)
    acc = ws[off:off + B * T * H * Dh * 4].view(T_.float32).reshape(B * T, H * Dh)
    assert rel(host(dk2), dk_ref) <= TOL[V.BF16] and rel(host(dv2), dv_ref) <= TOL[V.BF16]
    assert rel(acc.cpu().numpy() * scale, dq_ref) <= TOL[V.BF16]
    # the norm backward on the accumulator and on its rounded copy
    x = bf(r.standard_normal((B * T, (H + 2 * Hk) * Dh)).astype(F32))
    W = x.shape[1]
    xd = dev(x, V.BF16)
    qg, kg = dev(bf((1 + 0.1 * r.standard_normal(Dh)).astype(F32)), V.BF16), dev(bf((1 + 0.1 * r.standard_normal(Dh)).astype(F32)), V.BF16)
    cos, sin = O.rope_tables(T, Dh, 1e6)
    cd, sd = dev(cos), dev(sin)
    dkd = dev(bf(r.standard_normal((B * T, Hk * Dh)).astype(F32)), V.BF16)
    dq_bf = (acc * scale).to(T_.bfloat16).contiguous()
    outs = []
    for f32 in (1, 0):
        dx = empty((B * T, W), V.BF16)
        dgq, dgk = dev(np.zeros(Dh, F32)), dev(np.zeros(Dh, F32))
        w2 = workspace(lib.veda_qknorm_rope_bwd_qk_workspace(B * T, H, Hk, Dh))
        src = acc.data_ptr() if f32 else dq_bf.data_ptr()
        call("veda_qknorm_rope_bwd_qk", ptr(xd), ptr(xd) + H * Dh * 2, W, ptr(qg), ptr(kg), ptr(cd), ptr(sd),
             src, H * Dh, f32, scale if f32 else 1.0, ptr(dkd), Hk * Dh, ptr(dx), ptr(dx) + H * Dh * 2, W,
             ptr(dgq), ptr(dgk), ptr(w2), w2.numel(), B * T, H, Hk, T, Dh, 1e-6, V.BF16, stream())
        sync()
        outs.append((host(dx)[:, :(H + Hk) * Dh], host(dgq), host(dgk)))   # the q and k columns
    for a_, b_ in zip(outs[0], outs[1]):
        assert np.array_equal(a_, b_)


@pytest.mark.parametrize("dtype,B,T,H,Hk,Dh", [(V.F32, 4, 32, 4, 2, 16), (V.F32, 2, 70, 4, 1, 64),
                                              (V.BF16, 2, 256, 16, 8, 128),
                                              (V.BF16, 1, 200, 4, 2, 128),
                                              (V.BF16, 1, 136, 4, 1, 128),
                                              (V.BF16, 1, 100, 2, 2, 128)])
def test_attention(dtype, B, T, H, Hk, Dh):
    o, o_ref, lse, lse_ref, dq, dq_ref, dk, dk_ref, dv, dv_ref = _attention_case(
        dtype, B, T, H, Hk, Dh, T + Dh)
    tol = TOL[dtype]
    assert rel(o, o_ref) <= tol
    assert rel(lse, lse_ref) <= (1e-5 if dtype == V.F32 else 1e-3)
    assert rel(dq, dq_ref) <= tol
    assert rel(dk, dk_ref) <= tol
    assert rel(dv, dv_ref) <= tol


@pytest.fixture
def deterministic_attention():
    """Runs a test with the two-kernel (bit-reproducible) attention backward, then restores."""
    prev = V.lib().veda_attention_set_deterministic(1)
    yield
    V.lib().veda_attention_set_deterministic(prev)


@pytest.mark.parametrize("B,T,H,Hk", [(2, 256, 16, 8), (1, 200, 4, 2)])
def test_attention_deterministic_mode(deterministic_attention, B, T, H, Hk):
    o, o_ref, lse, lse_ref, dq, dq_ref, dk, dk_ref, dv, dv_ref = _attention_case(
        V.BF16, B, T, H, Hk, 128, T + 7)
    for got, want in ((dq, dq_ref), (dk, dk_ref), (dv, dv_ref)):
        assert rel(got, want) <= TOL[V.BF16]


@pytest.mark.parametrize("mode", [0, 1])
def test_attention_bwd_t1024_h16_against_oracle(mode):
    """Attention backward at T 1024 with 16 query heads over 8 KV heads, head_dim 128 (one batch
    row of the isolated attention-backward config): dQ, dK and dV against the oracle, for the
    fused kernel (mode 0) and the two-kernel path (mode 1). Reference: the softmax backward of
    src/libs/autograd/NonLinear.cpp:123-133 inside the composition of src/libs/train/Model.cpp:182-189."""
    prev = V.lib().veda_attention_set_deterministic(mode)
    try:
        _, _, _, _, dq, dq_ref, dk, dk_ref, dv, dv_ref = _attention_case(V.BF16, 1, 1024, 16, 8, 128, 2)
    finally:
        V.lib().veda_attention_set_deterministic(prev)
    assert rel(dq, dq_ref) <= TOL[V.BF16]
    assert rel(dk, dk_ref) <= TOL[V.BF16]
    assert rel(dv, dv_ref) <= TOL[V.BF16]


@pytest.mark.parametrize("B,T", [(8, 1024), (2, 4096)])
def test_attention_fused_equals_deterministic(B, T):
    """The fused backward against the two-kernel one on the same inputs at the isolated config's
    sizes (B 8 x T 1024, and T 4096): dV comes from the same bf16 P and the same products in the
    same order, so it is bit-identical; dK differs in that the fused kernel forms dS from the
    bf16 P (the two-kernel path from fp32 P), and dQ also in the order key tiles are summed."""
    H, Hk, Dh = 16, 8, 128
    r = rng(2)
    tok = (B * T, H * Dh)
    q, do = bf(r.standard_normal(tok)), bf(r.standard_normal(tok))
    k, v = bf(r.standard_normal((B * T, Hk * Dh))), bf(r.standard_normal((B * T, Hk * Dh)))
    qd, kd, vd, dod = dev(q, V.BF16), dev(k, V.BF16), dev(v, V.BF16), dev(do, V.BF16)
    o, lse = empty(tok, V.BF16), empty(B * H * T)
    scale = 1.0 / math.sqrt(Dh)
    call("veda_attention_fwd", ptr(qd), H * Dh, ptr(kd), Hk * Dh, ptr(vd), Hk * Dh, ptr(o), H * Dh,
         ptr(lse), B, T, H, Hk, Dh, scale, 1, V.BF16, stream())
    out = []
    for mode in (0, 1):
        prev = V.lib().veda_attention_set_deterministic(mode)
        try:
            dq, dk, dv = empty(tok, V.BF16), empty((B * T, Hk * Dh), V.BF16), empty((B * T, Hk * Dh), V.BF16)
            ws = workspace(V.lib().veda_attention_bwd_workspace(B, T, H, Hk, Dh, V.BF16))
            call("veda_attention_bwd", ptr(qd), H * Dh, ptr(kd), Hk * Dh, ptr(vd), Hk * Dh, ptr(o),
                 H * Dh, ptr(dod), H * Dh, ptr(lse), ptr(dq), H * Dh, ptr(dk), Hk * Dh, ptr(dv),
                 Hk * Dh, ptr(ws), ws.numel(), B, T, H, Hk, Dh, scale, 1, V.BF16, stream())
            sync()
            out.append((host(dq), host(dk), host(dv)))
            del ws
        finally:
            V.lib().veda_attention_set_deterministic(prev)
    (dq0, dk0, dv0), (dq1, dk1, dv1) = out
    assert np.array_equal(dv0, dv1)
    assert np.isfinite(dq0).all() and np.isfinite(dk0).all()
    assert rel(dk0, dk1) <= 1e-2
    assert rel(dq0, dq1) <= 1e-2


def test_attention_golden():
    from pathlib import Path
    ops = np.load(Path(__file__).parent / "golden" / "ops_small.npz")
    q, k, v, g = ops["att_q"], ops["att_k"], ops["att_v"], ops["att_g"]
    B, H, T, Dh = q.shape
    Hk = k.shape[1]
    tok = lambda a: np.ascontiguousarray(a.transpose(0, 2, 1, 3)).reshape(B * T, -1)  # noqa: E731
    qd, kd, vd, gd = dev(tok(q)), dev(tok(k)), dev(tok(v)), dev(tok(g))
    o, lse = empty((B * T, H * Dh)), empty(B * H * T)
    call("veda_attention_fwd", ptr(qd), H * Dh, ptr(kd), Hk * Dh, ptr(vd), Hk * Dh, ptr(o), H * Dh,
         ptr(lse), B, T, H, Hk, Dh, 0.25, 1, V.F32, stream())
    dq, dk, dv = empty((B * T, H * Dh)), empty((B * T, Hk * Dh)), empty((B * T, Hk * Dh))
    ws = workspace(V.lib().veda_attention_bwd_workspace(B, T, H, Hk, Dh, V.F32))
    call("veda_attention_bwd", ptr(qd), H * Dh, ptr(kd), Hk * Dh, ptr(vd), Hk * Dh, ptr(o), H * Dh,
         ptr(gd), H * Dh, ptr(lse), ptr(dq), H * Dh, ptr(dk), Hk * Dh, ptr(dv), Hk * Dh, ptr(ws),
         ws.numel(), B, T, H, Hk, Dh, 0.25, 1, V.F32, stream())
    sync()
    assert rel(host(o), tok(ops["att_o"])) <= 1e-5
    assert rel(host(dq), tok(ops["att_dq"])) <= 1e-5
    assert rel(host(dk), tok(ops["att_dk"])) <= 1e-5
    assert rel(host(dv), tok(ops["att_dv"])) <= 1e-5


# ---------------------------------------------------------------------------------------------
# Element-wise ops of the fine-grained API
# ---------------------------------------------------------------------------------------------
def test_binary_broadcast_and_unbroadcast():
    r = rng(21)
    a = r.standard_normal((3, 4, 5)).astype(F32)
    b = r.standard_normal((5,)).astype(F32)
    shape = np.array([3, 4, 5], np.int64)
    sa = np.array([20, 5, 1], np.int64)
    sb = np.array([0, 0, 1], np.int64)
    out = empty((3, 4, 5))
    ad, bd = dev(a), dev(b)   # held: a freed temporary could be reused before the launch runs
    for op, ref in ((0, a + b), (1, a * b)):
        call("veda_binary", op, ptr(ad), sa.ctypes.data, ptr(bd), sb.ctypes.data, ptr(out),
             shape.ctypes.data, 3, V.F32, stream())
        sync()
        assert np.array_equal(host(out), ref.astype(F32))
    g = r.standard_normal((3, 4, 5)).astype(F32)
    red = empty((1, 4, 1))
    tgt = np.array([1, 4, 1], np.int64)
    gd = dev(g)
    call("veda_unbroadcast", ptr(gd), shape.ctypes.data, tgt.ctypes.data, 3, ptr(red), V.F32,
         stream())
    sync()
    assert rel(host(red).ravel(), g.sum(axis=(0, 2))) <= 1e-6


def test_softmax_silu_sum_copy():
    from pathlib import Path
    ops = np.load(Path(__file__).parent / "golden" / "ops_small.npz")
    x, g = ops["softmax_x"], ops["softmax_g"]
    lanes, n = x.shape
    y, dx = empty(x.shape), empty(x.shape)
    yd, gd = dev(x), dev(g)
    call("veda_softmax_fwd", ptr(yd), ptr(y), lanes, n, V.F32, stream())
    call("veda_softmax_bwd", ptr(y), ptr(gd), ptr(dx), lanes, n, V.F32, stream())
    sync()
    assert rel(host(y), ops["softmax_y"]) <= 1e-6
    assert rel(host(dx), ops["softmax_dx"]) <= 1e-5
    xs = dev(np.array([0.0, 1.0, -1.0], F32))
    ones = dev(np.ones(3, F32))
    d = empty(3)
    call("veda_silu_bwd", ptr(xs), ptr(ones), ptr(d), 3, V.F32, stream())
    s = empty(1)
    ar = dev(np.arange(10, dtype=F32))
    call("veda_sum", ptr(ar), 10, ptr(s), V.F32, stream())
    m = np.arange(12, dtype=F32).reshape(3, 4)
    t = empty((4, 3))
    shape = np.array([4, 3], np.int64)
    strides = np.array([1, 4], np.int64)
    md = dev(m)
    call("veda_copy_strided", ptr(md), V.F32, strides.ctypes.data, 0, ptr(t), V.F32,
         shape.ctypes.data, 2, stream())
    sync()
    np.testing.assert_allclose(host(d), [0.5, 0.9277, 0.0723], atol=1e-3)
    assert float(host(s)[0]) == 45.0
    assert np.array_equal(host(t), m.T)


def test_argmax_ties_and_nan():
    x = np.array([[1.0, 3.0, 3.0, 2.0], [5.0, 5.0, 5.0, 5.0], [0.0, np.nan, 1.0, 2.0]], F32)
    out = torch_long(3)
    status = zeros(1).int()
    call("veda_argmax", ptr(dev(x[:2])), 4, 2, 4, ptr(out), ptr(status), V.F32, stream())
    sync()
    assert list(host(out)[:2]) == [1, 0] and int(host(status)[0]) == 0
    call("veda_argmax", ptr(dev(x)), 4, 3, 4, ptr(out), ptr(status), V.F32, stream())
    sync()
    assert int(host(status)[0]) == V.ERR_INVALID_ARGUMENT


def torch_long(n):
    from tests.gpu_util import torch
    t = torch()
    return t.zeros(n, dtype=t.int64, device="cuda")


def test_randn_statistics():
    n = 1 << 20
    x = empty(n)
    call("veda_randn", ptr(x), n, 0.02, 3, V.F32, stream())
    sync()
    h = host(x)
    assert abs(h.mean()) < 1e-4 and abs(h.std() - 0.02) < 2e-4


def test_bounded_wait_gives_up_with_timeout_status_and_context_survives():
    """The bounded mbarrier wait of the tensor-core and streaming kernels, driven to its limit on a
    barrier nothing arrives on (veda_wait_timeout_check, a small spin budget): the device status
    word reads VEDA_ERR_TIMEOUT, the reset clears it, and the context still runs kernels."""
    lib = V.lib()
    lib.veda_kernel_status(1)
    call("veda_wait_timeout_check", 1 << 20, stream())
    torch().cuda.synchronize()
    assert lib.veda_kernel_status(1) == V.ERR_TIMEOUT
    assert lib.veda_kernel_status(0) == 0
    x = dev(np.arange(1000, dtype=F32))
    out = empty(1000)
    call("veda_scale", ptr(x), 2.0, ptr(out), 1000, V.F32, stream())
    sync()
    assert np.array_equal(host(out), np.arange(1000, dtype=F32) * 2)
