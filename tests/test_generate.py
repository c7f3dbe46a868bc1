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


@pytest.mark.parametrize("dtype,heads,kv,dh,pos", [(0, 4, 2, 16, 0), (1, 16, 8, 128, 37)])
def test_decode_step_kernels_read_the_device_position(dtype, heads, kv, dh, pos):
    """One token's QK-norm + RoPE at the position held in device memory, its K/V rows written into
    the cache at that position, and attention over positions 0..pos, against the oracle and the
    length-argument kernel; the position then advances by one on the device."""
    import torch
    import veda_b200 as V
    from tests.gpu_util import bf, call, stream
    r = np.random.default_rng(pos + dh)
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
    q_ref = O.rope(O.rms_norm_gamma(q, qg, 1e-6)[0], cos[pos], sin[pos]).reshape(-1)
    k_ref = O.rope(O.rms_norm_gamma(k, kg, 1e-6)[0], cos[pos], sin[pos]).reshape(-1)
    tdt = torch.float32 if dtype == 0 else torch.bfloat16
    d = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to("cuda").to(tdt)
    dqkv, dqg, dkg, dk, dv = d(qkv), d(qg), d(kg), d(kc), d(vc)
    dcos, dsin = (torch.from_numpy(a).to("cuda") for a in (cos, sin))
    dpos = torch.tensor([pos], dtype=torch.int64, device="cuda")
    qr = torch.empty((heads * dh,), dtype=tdt, device="cuda")
    dt = V.F32 if dtype == 0 else V.BF16
    call("veda_decode_qkv_at", dqkv.data_ptr(), dqg.data_ptr(), dkg.data_ptr(), dcos.data_ptr(),
         dsin.data_ptr(), dpos.data_ptr(), qr.data_ptr(), dk.data_ptr(), dv.data_ptr(), kv * dh, heads,
         kv, dh, 1e-6, dt, stream())
    tol = 1e-5 if dtype == 0 else 2e-2
    assert O.max_abs_rel(qr.float().cpu().numpy(), q_ref) <= tol
    kc_got, vc_got = dk.float().cpu().numpy(), dv.float().cpu().numpy()
    assert O.max_abs_rel(kc_got[pos], k_ref) <= tol
    assert np.array_equal(vc_got[pos], v.astype(np.float32))
    rows = [i for i in range(cap) if i != pos]
    assert np.array_equal(kc_got[rows], kc[rows].astype(np.float32))   # other rows untouched
    assert np.array_equal(vc_got[rows], vc[rows].astype(np.float32))
    scale = 1.0 / math.sqrt(dh)
    out_at = torch.empty((heads, dh), dtype=tdt, device="cuda")
    out_len = torch.empty((heads, dh), dtype=tdt, device="cuda")
    call("veda_attention_decode_at", qr.data_ptr(), dk.data_ptr(), dv.data_ptr(), kv * dh, dpos.data_ptr(),
         heads, kv, dh, scale, out_at.data_ptr(), dt, stream())
    call("veda_attention_decode", qr.data_ptr(), dk.data_ptr(), dv.data_ptr(), kv * dh, pos + 1, heads, kv,
         dh, scale, out_len.data_ptr(), dt, stream())
    assert torch.equal(out_at, out_len)
    call("veda_decode_advance", dpos.data_ptr(), stream())
    assert int(dpos.item()) == pos + 1


@pytest.mark.parametrize("dtype,n,k,ldw", [(0, 37, 24, 24), (1, 1024, 3072, 3072), (1, 9000, 1024, 1032),
                                          (1, 5, 19, 21), (0, 8200, 96, 100)])
def test_gemv_matches_row_product(dtype, n, k, ldw):
    """One activation row through a Linear layer (both rows-per-warp variants, the 16-byte and the
    element-wise paths) against the float64 product; gate/up + SwiGLU in one pass equals
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
