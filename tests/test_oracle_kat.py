"""Pins the numpy oracle (oracle/veda_oracle.py) to the known answers of the reference's own
tests. Each case names the reference test file:line whose hand arithmetic it restates."""
import math

import numpy as np
import pytest

from oracle import veda_oracle as O

F32 = np.float32


def test_adamw_one_step_by_hand():
    # tests/AdamWTest.cpp:45-63 — theta 1, g 2, lr 0.1: m=0.2, v=0.008, m_hat=2, v_hat=4 -> 0.9
    w = np.array([1.0], F32)
    opt = O.AdamW([w], O.AdamWConfig(0.1, 0.9, 0.999, 1e-8, 0.0))
    opt.step([np.array([2.0], F32)])
    assert abs(w[0] - 0.9) < 1e-5
    assert opt.steps == 1


def test_adamw_first_step_is_the_learning_rate():
    # tests/AdamWTest.cpp:65-85 — gradients a million apart both move by lr
    tiny, huge, neg = np.zeros(1, F32), np.zeros(1, F32), np.zeros(1, F32)
    opt = O.AdamW([tiny, huge, neg], O.AdamWConfig(0.1, 0.9, 0.999, 1e-8, 0.0))
    opt.step([np.array([0.001], F32), np.array([1000.0], F32), np.array([-5.0], F32)])
    assert abs(tiny[0] + 0.1) < 1e-5 and abs(huge[0] + 0.1) < 1e-5
    assert abs(neg[0] - 0.1) < 1e-5


def test_adamw_decay_alone():
    # tests/AdamWTest.cpp:100-112 — g = 0: theta (1 - lr wd) per step -> 0.999, 0.999^2
    w = np.array([1.0], F32)
    opt = O.AdamW([w], O.AdamWConfig(0.1, 0.9, 0.999, 1e-8, 0.01))
    opt.step([np.zeros(1, F32)])
    assert abs(w[0] - 0.999) < 1e-6
    opt.step([np.zeros(1, F32)])
    assert abs(w[0] - 0.999 * 0.999) < 1e-6


def test_adamw_decoupled_decay():
    # tests/AdamWTest.cpp:114-141 — decay contribution lr*wd*theta, independent of the gradient
    def run(wd):
        a, b = np.array([2.0], F32), np.array([2.0], F32)
        O.AdamW([a, b], O.AdamWConfig(0.1, 0.9, 0.999, 1e-8, wd)).step(
            [np.array([0.001], F32), np.array([500.0], F32)])
        return a[0], b[0]
    a, b = run(0.05)
    ap, bp = run(0.0)
    assert abs((ap - a) - 0.1 * 0.05 * 2.0) < 1e-6
    assert abs((ap - a) - (bp - b)) < 1e-6


def test_adamw_rejects_bad_config():
    # src/libs/optim/AdamW.cpp:18-26
    with pytest.raises(ValueError):
        O.AdamW([np.zeros(1, F32)], O.AdamWConfig(0.1, 1.0, 0.999, 1e-8, 0.0))
    with pytest.raises(ValueError):
        O.AdamW([np.zeros(1, F32)], O.AdamWConfig(0.1, 0.9, 0.999, 0.0, 0.0))


def test_clip_thirteen_to_six_and_a_half():
    # tests/GradientClipTest.cpp:51-72 — [3,4],[12] -> norm 13; clipped to 6.5 -> [1.5,2],[6]
    a, b = np.array([3.0, 4.0], F32), np.array([12.0], F32)
    norm = O.clip_gradient_norm([a, b], 6.5)
    assert abs(norm - 13.0) < 1e-5
    np.testing.assert_allclose(a, [1.5, 2.0], atol=1e-5)
    np.testing.assert_allclose(b, [6.0], atol=1e-5)


def test_clip_no_op_at_or_below_threshold_is_bitwise():
    # tests/GradientClipTest.cpp:74-87
    a, b = np.array([3.0, 4.0], F32), np.array([12.0], F32)
    assert abs(O.clip_gradient_norm([a, b], 20.0) - 13.0) < 1e-5
    assert a[0] == F32(3.0) and b[0] == F32(12.0)
    assert abs(O.clip_gradient_norm([a, b], 13.0) - 13.0) < 1e-5
    assert a[0] == F32(3.0) and b[0] == F32(12.0)


def test_clip_non_finite_is_reported_not_spread():
    # tests/GradientClipTest.cpp:89-101
    good, bad = np.array([1.0, 1.0], F32), np.array([np.nan], F32)
    assert not math.isfinite(O.clip_gradient_norm([good, bad], 1.0))
    assert good[0] == 1.0 and good[1] == 1.0
    inf = np.array([np.inf], F32)
    assert not math.isfinite(O.clip_gradient_norm([good, inf], 1.0))
    assert good[0] == 1.0


def test_log_softmax_and_cross_entropy_by_hand():
    # tests/CrossEntropyTest.cpp:56-62, 119-150
    lp = O.log_softmax(np.array([1.0, 2.0, 3.0], F32))
    np.testing.assert_allclose(lp, [-2.4076, -1.4076, -0.4076], atol=1e-3)
    loss, d = O.cross_entropy(np.array([[1.0, 2.0, 3.0]], F32), [2])
    assert abs(loss - 0.4076) < 1e-3
    np.testing.assert_allclose(d[0], [0.0900, 0.2447, -0.3348], atol=1e-3)
    assert abs(float(d.sum())) < 1e-5
    loss, d = O.cross_entropy(np.array([[1.0, 2.0, 3.0]], F32), [0])
    assert abs(loss - 2.4076) < 1e-3
    np.testing.assert_allclose(d[0], [-0.9100, 0.2447, 0.6652], atol=1e-3)


def test_log_softmax_extremes():
    # tests/CrossEntropyTest.cpp:73-110 — large logits stay finite; all -inf lane stays -inf
    lp = O.log_softmax(np.array([0.0, 200.0], F32))
    assert abs(lp[0] + 200.0) < 1e-2 and abs(lp[1]) < 1e-2
    lp = O.log_softmax(np.array([-np.inf, 0.0, -np.inf], F32))
    assert abs(lp[1]) < 1e-6
    lp = O.log_softmax(np.array([[-np.inf, -np.inf]], F32))
    assert np.all(np.isneginf(lp))


def test_cross_entropy_uniform_is_log_v_and_mean_over_lanes():
    # tests/CrossEntropyTest.cpp:160-214
    V = 151936
    loss, _ = O.cross_entropy(np.zeros((1, V), F32), [7])
    assert abs(loss - math.log(V)) < 1e-4
    rng = np.random.default_rng(1)
    x = rng.standard_normal((4, 3)).astype(F32)
    t = np.array([0, 2, 1, 1])
    loss, d = O.cross_entropy(x, t)
    by_hand = sum(-O.log_softmax(x[i])[t[i]] for i in range(4)) / 4.0
    assert abs(loss - by_hand) < 1e-5
    _, alone = O.cross_entropy(x[:1], t[:1])
    assert abs(alone[0, 0] - d[0, 0] * 4.0) < 1e-5


def test_cross_entropy_refusals():
    # src/libs/autograd/Loss.cpp:21-47
    with pytest.raises(ValueError):
        O.cross_entropy(np.zeros((2, 3), F32), [0])
    with pytest.raises(ValueError):
        O.cross_entropy(np.zeros((1, 3), F32), [3])
    with pytest.raises(ValueError):
        O.cross_entropy(np.zeros((1, 3), F32), [-1])


def test_silu_gradient_values():
    # tests/AutogradNonLinearTest.cpp:55-66
    d = O.silu_backward(np.array([0.0, 1.0, -1.0], F32), np.ones(3, F32))
    assert abs(d[0] - 0.5) < 1e-4
    assert abs(d[1] - 0.9277) < 1e-3
    assert abs(d[2] - 0.0723) < 1e-3


def test_softmax_gradient_values_and_zero_sum():
    # tests/AutogradNonLinearTest.cpp:91-109
    y = O.softmax(np.array([1.0, 2.0, 3.0], F32))
    d = O.softmax_backward(y, np.array([1.0, 0.0, 0.0], F32))
    np.testing.assert_allclose(d, [0.0819, -0.0220, -0.0599], atol=1e-3)
    assert abs(float(d.sum())) < 1e-5


def test_embedding_scatter_add_accumulates_repeats():
    # tests/AutogradNonLinearTest.cpp:186-209 — ids {2,0,2}, weights 1,2,4 -> row2 = 5, row0 = 2
    rng = np.random.default_rng(3)
    table = rng.standard_normal((4, 3)).astype(F32)
    ids = [2, 0, 2]
    rows = O.embedding(table, ids)
    assert rows[0, 1] == table[2, 1] and rows[1, 2] == table[0, 2]
    g = np.array([[1, 1, 1], [2, 2, 2], [4, 4, 4]], F32)
    d = O.embedding_backward(np.zeros_like(table), ids, g)
    assert abs(d[2, 0] - 5.0) < 1e-5 and abs(d[2, 2] - 5.0) < 1e-5
    assert abs(d[0, 0] - 2.0) < 1e-5
    assert d[1, 0] == 0.0 and d[3, 2] == 0.0
    with pytest.raises(IndexError):
        O.embedding(table, [4])


def test_rope_quarter_turn_and_backward():
    # tests/AutogradViewsTest.cpp:114-134
    cos = np.zeros((1, 2), F32)
    sin = np.ones((1, 2), F32)
    out = O.rope(np.array([[1.0, 0.0]], F32), cos, sin)
    np.testing.assert_allclose(out, [[0.0, 1.0]], atol=1e-6)
    d = O.rope_backward(np.array([[1.0, 0.0]], F32), cos, sin)
    np.testing.assert_allclose(d, [[0.0, -1.0]], atol=1e-6)


def test_rope_preserves_norm():
    # tests/AutogradViewsTest.cpp:137-166
    c, s = O.rope_tables(6, 8, 10000.0)
    rng = np.random.default_rng(4)
    x = rng.standard_normal((2, 6, 8)).astype(F32)
    g = rng.standard_normal((2, 6, 8)).astype(F32)
    assert abs(np.linalg.norm(O.rope(x, c, s)) - np.linalg.norm(x)) < 1e-3
    assert abs(np.linalg.norm(O.rope_backward(g, c, s)) - np.linalg.norm(g)) < 1e-3


def test_matmul_backward_two_by_two():
    # tests/AutogradMatmulTest.cpp:48-75 — dA = G B^T = [[11,15],..]; dB = A^T G = [[4,4],[6,6]]
    a = np.array([[1, 2], [3, 4]], F32)
    b = np.array([[5, 6], [7, 8]], F32)
    g = np.ones((2, 2), F32)
    assert (a @ b)[0, 0] == 19 and (a @ b)[1, 1] == 50
    np.testing.assert_allclose(g @ b.T, [[11, 15], [11, 15]])
    np.testing.assert_allclose(a.T @ g, [[4, 4], [6, 6]])


def test_bf16_rounding_is_nearest_even():
    x = np.array([1.0, 1.00390625, 1.01171875, -2.5, 3.0e38, np.inf], F32)
    r = O.bf16_round(x)
    # 1 + 2^-8 is a tie between 1 and 1 + 2^-7 -> even (1.0); 1 + 3*2^-8 -> 1 + 2^-6
    assert r[0] == 1.0 and r[1] == 1.0 and r[2] == F32(1.015625)
    assert r[3] == -2.5 and np.isinf(r[5])
    assert np.isnan(O.bf16_round(np.array([np.nan], F32))[0])


def test_tiny_step_learns_and_is_deterministic():
    # tests/TinyModelTest.cpp:276-305 in miniature: loss at init ~ log V and decreasing
    c = O.TINY
    params = O.init_params(c, 0)
    ids, tg = O.synthetic_batch(c, 4, 32, 0)
    opt = O.AdamW(params, O.AdamWConfig(1e-2, 0.9, 0.95, 1e-8, 0.0))
    first, _, _ = O.train_step(c, params, ids, tg, 1.0, opt)
    assert abs(first - math.log(c.vocab)) < 0.3
    for _ in range(5):
        last, _, _ = O.train_step(c, params, ids, tg, 1.0, opt)
    assert last < first
