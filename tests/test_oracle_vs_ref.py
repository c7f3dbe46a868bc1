"""Pins the numpy oracle against the reference itself: the golden fixtures that
tests/golden/make_golden.py produced from the reference compiled from its sources, and — when
oracle/_ref/libveda_ref.so is present — live calls into that library on fresh seeded inputs."""
from pathlib import Path

import numpy as np
import pytest

from oracle import veda_oracle as O

F32 = np.float32
GOLDEN = Path(__file__).resolve().parent / "golden"
ADAM = O.AdamWConfig(1e-3, 0.9, 0.95, 1e-8, 0.1)


@pytest.fixture(scope="module")
def ops():
    return dict(np.load(GOLDEN / "ops_small.npz"))


@pytest.fixture(scope="module")
def tiny():
    return dict(np.load(GOLDEN / "tiny_step.npz"))


def close(a, b, tol):
    err = O.max_abs_rel(a, b)
    assert err <= tol, f"max-abs-rel {err:.3e} > {tol:.0e}"


def test_golden_rms_norm_gamma(ops):
    x, gam, g = ops["rms_x"], ops["rms_gamma"], ops["rms_g"]
    y, _, _ = O.rms_norm_gamma(x, gam, 1e-6)
    dx, dgam = O.rms_norm_gamma_backward(x, gam, g, 1e-6)
    close(y, ops["rms_y"], 1e-6)
    close(dx, ops["rms_dx"], 1e-5)
    close(dgam, ops["rms_dgamma"], 1e-5)


def test_golden_swiglu(ops):
    ga, up, g = ops["swiglu_gate"], ops["swiglu_up"], ops["swiglu_g"]
    close(O.swiglu(ga, up), ops["swiglu_y"], 1e-6)
    dga, dup = O.swiglu_backward(ga, up, g)
    close(dga, ops["swiglu_dgate"], 1e-6)
    close(dup, ops["swiglu_dup"], 1e-6)


def test_golden_softmax(ops):
    y = O.softmax(ops["softmax_x"])
    close(y, ops["softmax_y"], 1e-6)
    close(O.softmax_backward(y, ops["softmax_g"]), ops["softmax_dx"], 1e-5)


def test_golden_cross_entropy(ops):
    loss, d = O.cross_entropy(ops["ce_logits"], ops["ce_targets"])
    assert abs(loss - ops["ce_loss"][0]) <= 1e-6 * max(1.0, abs(loss))
    close(d, ops["ce_dlogits"], 1e-6)


def test_golden_embedding_bit_exact(ops):
    rows = O.embedding(ops["emb_table"], ops["emb_ids"])
    assert np.array_equal(rows, ops["emb_rows"])
    dt = O.embedding_backward(np.zeros_like(ops["emb_table"]), ops["emb_ids"], ops["emb_g"])
    assert np.array_equal(dt, ops["emb_dtable"]), "sequential scatter-add must be bit-exact"


def test_golden_rope(ops):
    c, s = O.rope_tables(10, 16, 10000.0)
    assert np.array_equal(c, ops["rope_cos"]) and np.array_equal(s, ops["rope_sin"])
    c6, s6 = O.rope_tables(64, 128, 1e6)
    assert np.array_equal(c6, ops["rope6_cos"]) and np.array_equal(s6, ops["rope6_sin"])
    close(O.rope(ops["rope_x"], c, s), ops["rope_y"], 1e-6)
    close(O.rope_backward(ops["rope_g"], c, s), ops["rope_dx"], 1e-6)


def test_golden_matmul_nt(ops):
    a, b, g = ops["mm_a"], ops["mm_b"], ops["mm_g"]
    close(a @ b.T, ops["mm_y"], 1e-6)
    close(g @ b, ops["mm_da"], 1e-6)
    close(g.T @ a, ops["mm_db"], 1e-6)


def test_golden_attention_gqa(ops):
    q, k, v, g = ops["att_q"], ops["att_k"], ops["att_v"], ops["att_g"]
    o, _, p = O.attention(q, k, v)
    close(o, ops["att_o"], 1e-5)
    dq, dk, dv = O.attention_backward(q, k, v, p, g)
    close(dq, ops["att_dq"], 1e-5)
    close(dk, ops["att_dk"], 1e-5)
    close(dv, ops["att_dv"], 1e-5)


def test_golden_tiny_step(tiny):
    c = O.TINY
    n = len(O.param_specs(c))
    params = [tiny[f"w0_{i:03d}"].copy() for i in range(n)]
    fresh = O.init_params(c, 0)
    assert all(np.array_equal(a, b) for a, b in zip(params, fresh)), "seeded init drifted"
    ids, tg = O.synthetic_batch(c, 4, 32, 0)
    assert np.array_equal(ids, tiny["ids"]) and np.array_equal(tg, tiny["targets"])
    opt = O.AdamW(params, ADAM)
    loss, norm, grads = O.train_step(c, params, ids, tg, 1.0, opt)
    assert abs(loss - tiny["loss"][0]) <= 1e-6 * abs(loss)
    assert abs(norm - tiny["norm"][0]) <= 1e-5 * abs(norm)
    for i in range(n):
        close(grads[i], tiny[f"g_{i:03d}"], 1e-5)
        # updated weights: AdamW's g / (sqrt(v) + eps) turns last-bit gradient differences into
        # visible weight differences where |g| is about eps, hence the looser bound
        close(params[i], tiny[f"w1_{i:03d}"], 2e-4)


def test_live_reference_ops(ref_lib):
    rng = np.random.default_rng(11)
    x, g = rng.standard_normal((5, 64)).astype(F32), rng.standard_normal((5, 64)).astype(F32)
    gam = (1 + 0.1 * rng.standard_normal(64)).astype(F32)
    y, dx, dg = ref_lib.rms_norm_gamma(x, gam, g, 1e-6)
    close(O.rms_norm_gamma(x, gam, 1e-6)[0], y, 1e-6)
    dx2, dg2 = O.rms_norm_gamma_backward(x, gam, g, 1e-6)
    close(dx2, dx, 1e-5)
    close(dg2, dg, 1e-5)
    lg = rng.standard_normal((3, 1000)).astype(F32)
    t = rng.integers(0, 1000, 3)
    loss, d = ref_lib.cross_entropy(lg, t)
    loss2, d2 = O.cross_entropy(lg, t)
    assert abs(loss - loss2) < 1e-6
    close(d2, d, 1e-6)
    with pytest.raises(ValueError):
        ref_lib.cross_entropy(lg, np.array([0, 1, 1000]))
    with pytest.raises(IndexError):
        ref_lib.embedding(np.zeros((4, 2), F32), np.array([4]), np.zeros((1, 2), F32))


def test_live_reference_clip_and_adamw(ref_lib):
    norm, out = ref_lib.clip([np.array([3.0, 4.0], F32), np.array([12.0], F32)], 6.5)
    assert abs(norm - 13.0) < 1e-5
    np.testing.assert_allclose(out[0], [1.5, 2.0], atol=1e-6)
    rng = np.random.default_rng(12)
    w = rng.standard_normal(100).astype(F32)
    gs = rng.standard_normal((3, 100)).astype(F32)
    got = ref_lib.adamw(w, gs, 1e-2, 0.9, 0.95, 1e-8, 0.1)
    mine = w.copy()
    opt = O.AdamW([mine], O.AdamWConfig(1e-2, 0.9, 0.95, 1e-8, 0.1))
    for s in range(3):
        opt.step([gs[s]])
    assert np.array_equal(mine, got), "AdamW restatement must be bit-exact on equal gradients"


def test_live_reference_two_steps_gqa(ref_lib):
    # a second, Qwen3-proportioned shape (H/Hkv = 2, theta 1e6) and two steps
    c = O.ModelConfig(vocab=96, hidden=32, intermediate=48, layers=2, heads=4, kv_heads=2,
                      head_dim=8, eps=1e-6, theta=1e6)
    params = O.init_params(c, 5)
    ids, tg = O.synthetic_batch(c, 2, 16, 5)
    w, losses, norms, grads = ref_lib.train_steps(c, [p.copy() for p in params], ids, tg, 0.5,
                                                  ADAM, steps=2)
    mine = [p.copy() for p in params]
    opt = O.AdamW(mine, ADAM)
    O.train_step(c, mine, ids, tg, 0.5, opt)
    loss, norm, g2 = O.train_step(c, mine, ids, tg, 0.5, opt)
    assert abs(loss - losses[1]) < 1e-5
    assert abs(norm - norms[1]) < 1e-5 * norm
    for a, b in zip(g2, grads):
        close(a, b, 1e-4)
