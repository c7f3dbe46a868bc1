"""Greedy generation on the device (src/libs/generate/Generator.cpp:20-109, Sampling.cpp:97-113)
against the oracle's uncached loop, and the KV-cached loop against the uncached one (the
reference's acceptance rule for its cache)."""
import math

import numpy as np
import pytest

from oracle import veda_oracle as O

pytestmark = pytest.mark.gpu

QWEN_SMALL = O.ModelConfig(vocab=2048, hidden=256, intermediate=512, layers=2, heads=4,
                           kv_heads=2, head_dim=128, eps=1e-6, theta=1e6)


@pytest.fixture(autouse=True)
def _gpu(cuda):
    yield


def trainer(cfg, dtype, params):
    from veda_b200.train_abi import Trainer
    t = Trainer(cfg, dtype=dtype, batch=1, seq_len=8, seed=1)
    t.set_params(np.concatenate([p.ravel() for p in params]))
    return t


@pytest.mark.parametrize("dtype,heads,kv,dh,length", [(0, 4, 2, 16, 1), (0, 4, 2, 16, 37),
                                                      (1, 16, 8, 128, 1000), (1, 4, 4, 64, 5)])
def test_attention_decode_matches_softmax_row(dtype, heads, kv, dh, length):
    import torch
    import veda_b200 as V
    from tests.gpu_util import bf, call, stream
    r = np.random.default_rng(length + dh)
    q = r.standard_normal((heads, dh)).astype(np.float32)
    k = r.standard_normal((length, kv * dh)).astype(np.float32)
    v = r.standard_normal((length, kv * dh)).astype(np.float32)
    if dtype == 1:
        q, k, v = bf(q), bf(k), bf(v)
    scale = 1.0 / math.sqrt(dh)
    ref = np.empty((heads, dh), np.float32)
    for h in range(heads):
        g = h // (heads // kv)
        kh, vh = k[:, g * dh:(g + 1) * dh], v[:, g * dh:(g + 1) * dh]
        s = (kh @ q[h]) * scale
        p = np.exp(s - s.max())
        ref[h] = (p / p.sum()) @ vh
    tdt = torch.float32 if dtype == 0 else torch.bfloat16
    dq, dk, dv = (torch.from_numpy(a).to("cuda").to(tdt) for a in (q, k, v))
    out = torch.empty((heads, dh), dtype=tdt, device="cuda")
    call("veda_attention_decode", dq.data_ptr(), dk.data_ptr(), dv.data_ptr(), kv * dh, length, heads,
         kv, dh, scale, out.data_ptr(), V.F32 if dtype == 0 else V.BF16, stream())
    got = out.float().cpu().numpy()
    assert O.max_abs_rel(got, ref) <= (1e-5 if dtype == 0 else 2e-2)


def test_tiny_fp32_generation_matches_oracle_and_cache():
    cfg = O.TINY
    params = O.init_params(cfg, 0)
    t = trainer(cfg, 0, params)
    prompt = [5, 77, 300, 12, 1, 480, 33]
    logits = t.last_logits(prompt)
    assert O.max_abs_rel(logits, O.forward_logits(cfg, params, prompt)[-1]) <= 1e-4
    ref, ref_stopped, ref_passes = O.generate(cfg, params, prompt, 12)
    toks, stopped, passes = t.generate(prompt, 12, cached=False)
    assert toks == ref and not stopped and passes == ref_passes == 12
    toks_c, stopped_c, passes_c = t.generate(prompt, 12, cached=True)
    assert toks_c == ref and not stopped_c and passes_c == 13   # the limit still runs the last feed
    # a stop token ends the loop and is never emitted
    stop = ref[2]
    first = ref.index(stop)
    toks_s, stopped_s, _ = t.generate(prompt, 12, stop_tokens=[stop], cached=True)
    assert toks_s == ref[:first] and stopped_s
    with pytest.raises(ValueError):
        t.generate([], 4)
    with pytest.raises(ValueError):
        t.generate([cfg.vocab], 4)
    t.close()


def test_qwen_shaped_bf16_cached_generation_matches_uncached():
    cfg = QWEN_SMALL
    params = O.init_params(cfg, 3, bf16=True)
    t = trainer(cfg, 1, params)
    prompt = list(np.random.default_rng(4).integers(0, cfg.vocab, 40))
    logits = t.last_logits(prompt)
    assert O.max_abs_rel(logits, O.forward_logits(cfg, params, prompt)[-1]) <= 2e-2
    toks, _, _ = t.generate(prompt, 16, cached=False)
    toks_c, _, _ = t.generate(prompt, 16, cached=True)
    assert len(toks) == 16 and toks_c == toks
    t.close()


@pytest.mark.parametrize("dtype,heads,kv,dh,pos", [(0, 4, 2, 16, 0), (1, 16, 8, 128, 37), (0, 4, 4, 128, 5),
                                                  (1, 16, 4, 128, 300), (1, 32, 4, 128, 50), (1, 16, 8, 128, 0),
                                                  (1, 16, 8, 128, 1000), (0, 8, 4, 128, 200),
                                                  # eight query heads a KV head over several slices;
                                                  # capacity 257, one row past single-slice decode
                                                  (1, 32, 4, 128, 300), (1, 16, 8, 128, 254)])
def test_decode_step_kernels_read_the_device_position(dtype, heads, kv, dh, pos):
    """One token's QK-norm + RoPE at the position held in device memory, its K/V rows written into
    the cache at that position, and attention over positions 0..pos: the two-launch path against
    the oracle and the length-argument kernel, the fused launch (head_dim 128) against both; the
    position then advances by one on the device."""
    import torch
    import veda_b200 as V
    from tests.gpu_util import bf, call, stream
    r = np.random.default_rng(pos + dh + heads)
    cap = pos + 3
    W = (heads + 2 * kv) * dh
    qkv = r.standard_normal((1, W)).astype(np.float32)
    qg = (1 + 0.1 * r.standard_normal(dh)).astype(np.float32)
    kg = (1 + 0.1 * r.standard_normal(dh)).astype(np.float32)
    kc = r.standard_normal((cap, kv * dh)).astype(np.float32)
    vc = r.standard_normal((cap, kv * dh)).astype(np.float32)
    if dtype == 1:
        qkv, qg, kg, kc, vc = bf(qkv), bf(qg), bf(kg), bf(kc), bf(vc)
    cos, sin = O.rope_tables(cap, dh, 1e6)
    q = qkv[0, :heads * dh].reshape(heads, dh)
    k = qkv[0, heads * dh:(heads + kv) * dh].reshape(kv, dh)
    v = qkv[0, (heads + kv) * dh:].reshape(kv * dh)
    q_ref = O.rope(O.rms_norm_gamma(q, qg, 1e-6)[0], cos[pos], sin[pos])
    k_ref = O.rope(O.rms_norm_gamma(k, kg, 1e-6)[0], cos[pos], sin[pos]).reshape(-1)
    scale = 1.0 / math.sqrt(dh)
    keys, vals = kc[:pos + 1].copy(), vc[:pos + 1].copy()
    keys[pos], vals[pos] = k_ref, v
    att_ref = np.empty((heads, dh), np.float32)
    for h in range(heads):
        g = h // (heads // kv)
        sc = (keys[:, g * dh:(g + 1) * dh] @ q_ref[h]) * scale
        e = np.exp(sc - sc.max())
        att_ref[h] = (e / e.sum()) @ vals[:, g * dh:(g + 1) * dh]
    tdt = torch.float32 if dtype == 0 else torch.bfloat16
    d = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to("cuda").to(tdt)
    dqkv, dqg, dkg = d(qkv), d(qg), d(kg)
    dcos, dsin = (torch.from_numpy(a).to("cuda") for a in (cos, sin))
    dpos = torch.tensor([pos], dtype=torch.int64, device="cuda")
    dt = V.F32 if dtype == 0 else V.BF16
    tol = 1e-5 if dtype == 0 else 2e-2
    rows = [i for i in range(cap) if i != pos]

    def check_cache(dk, dv):
        kc_got, vc_got = dk.float().cpu().numpy(), dv.float().cpu().numpy()
        assert O.max_abs_rel(kc_got[pos], k_ref) <= tol
        assert np.array_equal(vc_got[pos], v.astype(np.float32))
        assert np.array_equal(kc_got[rows], kc[rows].astype(np.float32))   # other rows untouched
        assert np.array_equal(vc_got[rows], vc[rows].astype(np.float32))

    # two launches: q/k/v at the position, then attention reading it
    dk, dv = d(kc), d(vc)
    qr = torch.empty((heads * dh,), dtype=tdt, device="cuda")
    call("veda_decode_qkv_at", dqkv.data_ptr(), dqg.data_ptr(), dkg.data_ptr(), dcos.data_ptr(),
         dsin.data_ptr(), dpos.data_ptr(), qr.data_ptr(), dk.data_ptr(), dv.data_ptr(), kv * dh, heads,
         kv, dh, 1e-6, dt, stream())
    assert O.max_abs_rel(qr.float().cpu().numpy(), q_ref.reshape(-1)) <= tol
    check_cache(dk, dv)
    out_at = torch.empty((heads, dh), dtype=tdt, device="cuda")
    out_len = torch.empty((heads, dh), dtype=tdt, device="cuda")
    call("veda_attention_decode_at", qr.data_ptr(), dk.data_ptr(), dv.data_ptr(), kv * dh, dpos.data_ptr(),
         heads, kv, dh, scale, out_at.data_ptr(), dt, stream())
    call("veda_attention_decode", qr.data_ptr(), dk.data_ptr(), dv.data_ptr(), kv * dh, pos + 1, heads, kv,
         dh, scale, out_len.data_ptr(), dt, stream())
    assert torch.equal(out_at, out_len)
    assert O.max_abs_rel(out_at.float().cpu().numpy(), att_ref) <= tol
    # one launch, the positions split across CTAs by the capacity (cap rows) and merged through the
    # workspace; a second call on the same workspace gives the same result (its counters reset)
    ws = V.lib().veda_decode_attention_workspace(heads, kv, cap)
    work = torch.zeros(ws, dtype=torch.uint8, device="cuda")
    for _ in range(2):
        dk2, dv2 = d(kc), d(vc)
        out_f = torch.empty((heads, dh), dtype=tdt, device="cuda")
        args = (dqkv.data_ptr(), dqg.data_ptr(), dkg.data_ptr(), dcos.data_ptr(), dsin.data_ptr(),
                dpos.data_ptr(), dk2.data_ptr(), dv2.data_ptr(), kv * dh, cap, heads, kv, dh, 1e-6, scale,
                out_f.data_ptr(), work.data_ptr(), ws, dt, stream())
        if dh != 128:
            assert V.lib().veda_decode_attention_at(*args) == V.ERR_UNSUPPORTED
            break
        call("veda_decode_attention_at", *args)
        check_cache(dk2, dv2)
        assert O.max_abs_rel(out_f.float().cpu().numpy(), att_ref) <= tol
        assert O.max_abs_rel(out_f.float().cpu().numpy(), out_at.float().cpu().numpy()) <= tol
    if dh == 128:
        assert not bool(work[:256].any())   # the merge counters are back at zero
        small = args[:16] + (work.data_ptr(), ws - 4) + args[18:]
        assert V.lib().veda_decode_attention_at(*small) == V.ERR_INVALID_ARGUMENT
    call("veda_decode_advance", dpos.data_ptr(), stream())
    assert int(dpos.item()) == pos + 1


@pytest.mark.parametrize("dtype,k,with_r", [(1, 1024, True), (1, 1024, False), (1, 2048, True),
                                            (0, 96, True), (1, 200, True),
                                            (1, 12032, True)])   # the largest row and gain staged
def test_gemv_with_rmsnorm_prologue(dtype, k, with_r):
    """The pre-norm computed inside the projection equals the separate add + RMSNorm then the
    projection: the residual sum bit for bit, the outputs within one rounding of the dtype."""
    import torch
    import veda_b200 as V
    from tests.gpu_util import bf, call, stream
    r = np.random.default_rng(k + with_r)
    n = 3 * 96
    x = r.standard_normal(k).astype(np.float32)
    dlt = r.standard_normal(k).astype(np.float32)
    gam = (1 + 0.1 * r.standard_normal(k)).astype(np.float32)
    w = r.standard_normal((2 * n, k)).astype(np.float32)
    if dtype == 1:
        x, dlt, gam, w = bf(x), bf(dlt), bf(gam), bf(w)
    tdt = torch.float32 if dtype == 0 else torch.bfloat16
    dt = V.F32 if dtype == 0 else V.BF16
    dx, dr, dg, dw = (torch.from_numpy(a).to("cuda").to(tdt) for a in (x, dlt, gam, w))
    rp = dr.data_ptr() if with_r else None
    s_sep, a_sep = torch.empty(k, dtype=tdt, device="cuda"), torch.empty(k, dtype=tdt, device="cuda")
    if with_r:
        call("veda_add_rmsnorm_fwd", dx.data_ptr(), k, dr.data_ptr(), k, dg.data_ptr(), s_sep.data_ptr(), k,
             a_sep.data_ptr(), k, 1, k, 1e-6, dt, stream())
    else:
        s_sep.copy_(dx)
        call("veda_rmsnorm_fwd", dx.data_ptr(), k, dg.data_ptr(), a_sep.data_ptr(), k, 1, k, 1e-6, dt, stream())
    y_sep = torch.empty(2 * n, dtype=tdt, device="cuda")
    call("veda_gemv_nt", a_sep.data_ptr(), dw.data_ptr(), k, y_sep.data_ptr(), 2 * n, k, dt, stream())
    h_sep = torch.empty(n, dtype=tdt, device="cuda")
    call("veda_gemv_swiglu", a_sep.data_ptr(), dw.data_ptr(), k, h_sep.data_ptr(), n, k, dt, stream())
    s = torch.zeros(k, dtype=tdt, device="cuda")
    y = torch.empty(2 * n, dtype=tdt, device="cuda")
    call("veda_gemv_rmsnorm", dx.data_ptr(), rp, dg.data_ptr(), 1e-6, s.data_ptr() if with_r else None,
         dw.data_ptr(), k, y.data_ptr(), 2 * n, k, dt, stream())
    h = torch.empty(n, dtype=tdt, device="cuda")
    call("veda_gemv_rmsnorm_swiglu", dx.data_ptr(), rp, dg.data_ptr(), 1e-6, None, dw.data_ptr(), k,
         h.data_ptr(), n, k, dt, stream())
    if with_r:
        assert torch.equal(s, s_sep)
    tol = 1e-5 if dtype == 0 else 1e-2
    assert O.max_abs_rel(y.float().cpu().numpy(), y_sep.float().cpu().numpy()) <= tol
    assert O.max_abs_rel(h.float().cpu().numpy(), h_sep.float().cpu().numpy()) <= tol
    # the oracle: s = x + r rounded, RMSNorm * gamma, then the product
    sr = (x + dlt) if with_r else x
    if dtype == 1:
        sr = bf(sr)
    a_ref = O.rms_norm_gamma(sr[None, :], gam, 1e-6)[0][0]
    assert O.max_abs_rel(y.float().cpu().numpy(), w.astype(np.float64) @ a_ref.astype(np.float64)) <= \
        (1e-4 if dtype == 0 else 2e-2)
    assert V.lib().veda_gemv_rmsnorm(dx.data_ptr(), rp, dg.data_ptr(), 1e-6, dx.data_ptr(), dw.data_ptr(), k,
                                     y.data_ptr(), 2 * n, k, dt, stream()) == V.ERR_INVALID_ARGUMENT
    if k == 12032:   # one more 16-byte chunk of row and gain no longer fits the staged 47 KB
        assert V.lib().veda_gemv_rmsnorm(dx.data_ptr(), rp, dg.data_ptr(), 1e-6, None, dw.data_ptr(), k,
                                         y.data_ptr(), 2 * n, k + 8, dt, stream()) == V.ERR_INVALID_ARGUMENT


@pytest.mark.parametrize("dtype,n,k,ldw", [(0, 37, 24, 24), (1, 1024, 3072, 3072), (1, 9000, 1024, 1032),
                                          (1, 5, 19, 21), (0, 8200, 96, 100), (1, 300, 2048, 2048),
                                          (0, 100, 1536, 1540), (1, 7, 2056, 2056),
                                          (1, 64, 24064, 24064)])   # the largest row staged
def test_gemv_matches_row_product(dtype, n, k, ldw):
    """One activation row through a Linear layer (both rows-per-warp variants, rows split across 1, 2
    or 4 warps, the 16-byte and the element-wise paths) against the float64 product; gate/up + SwiGLU in one pass equals
    the projection followed by veda_swiglu_fwd bit for bit."""
    import torch
    import veda_b200 as V
    from tests.gpu_util import bf, call, stream
    r = np.random.default_rng(n + k)
    x = r.standard_normal(k).astype(np.float32)
    w = r.standard_normal((2 * n, ldw)).astype(np.float32)
    if dtype == 1:
        x, w = bf(x), bf(w)
    tdt = torch.float32 if dtype == 0 else torch.bfloat16
    dt = V.F32 if dtype == 0 else V.BF16
    dx, dw = (torch.from_numpy(a).to("cuda").to(tdt) for a in (x, w))
    y = torch.empty(2 * n, dtype=tdt, device="cuda")
    call("veda_gemv_nt", dx.data_ptr(), dw.data_ptr(), ldw, y.data_ptr(), 2 * n, k, dt, stream())
    ref = w[:, :k].astype(np.float64) @ x.astype(np.float64)
    tol = 1e-5 if dtype == 0 else 8e-3
    assert O.max_abs_rel(y.float().cpu().numpy(), ref) <= tol
    h = torch.empty(n, dtype=tdt, device="cuda")
    call("veda_gemv_swiglu", dx.data_ptr(), dw.data_ptr(), ldw, h.data_ptr(), n, k, dt, stream())
    h2 = torch.empty(n, dtype=tdt, device="cuda")
    call("veda_swiglu_fwd", y.data_ptr(), n, y[n:].data_ptr(), n, h2.data_ptr(), n, 1, n, dt, stream())
    assert torch.equal(h, h2)


@pytest.mark.parametrize("dtype,n,k", [(1, 151936, 1024), (1, 3000, 256), (0, 9000, 64)])
def test_lm_head_gemv_with_greedy_choice(dtype, n, k):
    """The norm + LM head with the argmax fused in: the logits equal the unfused projection's bit
    for bit, the token equals veda_argmax over them, ties go to the lower index, a NaN sets the
    status; the merge workspace is left ready for the next call."""
    import torch
    import veda_b200 as V
    from tests.gpu_util import bf, call, stream
    r = np.random.default_rng(n)
    x = r.standard_normal(k).astype(np.float32)
    dlt = r.standard_normal(k).astype(np.float32)
    gam = (1 + 0.1 * r.standard_normal(k)).astype(np.float32)
    w = r.standard_normal((n, k)).astype(np.float32)
    if dtype == 1:
        x, dlt, gam, w = bf(x), bf(dlt), bf(gam), bf(w)
    tdt = torch.float32 if dtype == 0 else torch.bfloat16
    dt = V.F32 if dtype == 0 else V.BF16
    dx, dr, dg = (torch.from_numpy(a).to("cuda").to(tdt) for a in (x, dlt, gam))
    ws = V.lib().veda_gemv_argmax_workspace(n)
    work = torch.zeros(ws, dtype=torch.uint8, device="cuda")

    def both(wt):
        y_sep = torch.empty(n, dtype=tdt, device="cuda")
        call("veda_gemv_rmsnorm", dx.data_ptr(), dr.data_ptr(), dg.data_ptr(), 1e-6, None, wt.data_ptr(), k,
             y_sep.data_ptr(), n, k, dt, stream())
        ref = torch.zeros(1, dtype=torch.int64, device="cuda")
        ref_status = torch.zeros(1, dtype=torch.int32, device="cuda")
        call("veda_argmax", y_sep.data_ptr(), n, 1, n, ref.data_ptr(), ref_status.data_ptr(), dt, stream())
        y = torch.empty(n, dtype=tdt, device="cuda")
        tok = torch.zeros(1, dtype=torch.int64, device="cuda")
        status = torch.zeros(1, dtype=torch.int32, device="cuda")
        call("veda_gemv_rmsnorm_argmax", dx.data_ptr(), dr.data_ptr(), dg.data_ptr(), 1e-6, None, wt.data_ptr(),
             k, y.data_ptr(), n, k, tok.data_ptr(), status.data_ptr(), work.data_ptr(), ws, dt, stream())
        assert torch.allclose(y, y_sep, rtol=0, atol=0, equal_nan=True)   # bit for bit, NaN where NaN
        return int(tok.item()), int(status.item()), int(ref.item()), y_sep

    dw = torch.from_numpy(w).to("cuda").to(tdt)
    tok, status, ref, y = both(dw)
    assert tok == ref and status == 0
    assert tok == int(np.argmax(y.float().cpu().numpy()))
    # copies of the winning row further down and further up: the lowest index wins
    lo, hi = min(5, tok), n - 3
    dw[5] = dw[tok]
    dw[hi] = dw[tok]
    tok2, status2, ref2, _ = both(dw)
    assert tok2 == ref2 == lo and status2 == 0
    assert not bool(work[:4].any())
    # a NaN weight row makes one logit NaN: no token, the status set
    dw[n // 2] = float("nan")
    tok3, status3, ref3, _ = both(dw)
    assert tok3 == -1 and status3 == V.ERR_INVALID_ARGUMENT and ref3 == -1


def test_decode_graph_and_per_launch_decode_agree(tmp_path):
    """VEDA_DECODE_GRAPH=0 (each decode step an eager one-token forward through the prefill's
    kernels) generates the same tokens as the replayed graph, in fp32 and bf16."""
    import os
    import subprocess
    import sys
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    script = (
        "import sys, json, numpy as np\n"
        "from oracle import veda_oracle as O\n"
        "from veda_b200.train_abi import Trainer\n"
        "out = {}\n"
        "for name, cfg, dtype, seed in [('tiny', O.TINY, 0, 0), ('qwen', O.ModelConfig(vocab=2048, hidden=256, "
        "intermediate=512, layers=2, heads=4, kv_heads=2, head_dim=128, eps=1e-6, theta=1e6), 1, 3)]:\n"
        "    params = O.init_params(cfg, seed, bf16=(dtype == 1))\n"
        "    t = Trainer(cfg, dtype=dtype, batch=1, seq_len=8, seed=1)\n"
        "    t.set_params(np.concatenate([p.ravel() for p in params]))\n"
        "    prompt = [int(v) for v in np.random.default_rng(4).integers(0, cfg.vocab, 24)]\n"
        "    out[name] = t.generate(prompt, 12, cached=True)[0]\n"
        "    t.close()\n"
        "print(json.dumps(out))\n")
    runs = []
    for flag in ("1", "0"):
        env = dict(os.environ, VEDA_DECODE_GRAPH=flag)
        r = subprocess.run([sys.executable, "-c", script], cwd=root, env=env, capture_output=True, text=True,
                           timeout=600)
        assert r.returncode == 0, r.stderr[-2000:]
        runs.append(r.stdout.strip().splitlines()[-1])
    assert runs[0] == runs[1]
