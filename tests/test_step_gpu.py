"""Parity of the full training step (forward, cross-entropy, backward, clip, AdamW) run by the
C++ trainer (libveda.so, include/veda_train.h) against the reference.

* fp32, the tiny decoder config: against tests/golden/tiny_step.npz, produced by the reference
  compiled from its sources (tolerance 1e-4 max-abs-relative per tensor);
* bf16, Qwen3-shaped (head_dim 128, GQA 2:1, QK-norm, RoPE theta 1e6), reduced width and depth:
  against the oracle's fp32 step on the same bf16-rounded weights (tolerance 2e-2).
"""
import math
from pathlib import Path

import numpy as np
import pytest

from oracle import veda_oracle as O

pytestmark = pytest.mark.gpu
GOLDEN = Path(__file__).resolve().parent / "golden"
ADAM = O.AdamWConfig(1e-3, 0.9, 0.95, 1e-8, 0.1)


@pytest.fixture(autouse=True)
def _gpu(cuda):
    yield


def make_trainer(cfg, dtype, batch, seq_len, seed=0):
    from veda_b200.train_abi import Trainer
    return Trainer(cfg, lr=ADAM.learning_rate, betas=(ADAM.beta1, ADAM.beta2), eps=ADAM.eps,
                   weight_decay=ADAM.weight_decay, max_norm=1.0, dtype=dtype, batch=batch,
                   seq_len=seq_len, seed=seed)


def split(cfg, flat):
    out, at = [], 0
    for _, shape in O.param_specs(cfg):
        n = int(np.prod(shape))
        out.append(flat[at:at + n].reshape(shape))
        at += n
    return out


def test_tiny_fp32_step_matches_reference_golden():
    g = dict(np.load(GOLDEN / "tiny_step.npz"))
    cfg = O.TINY
    n = len(O.param_specs(cfg))
    w0 = np.concatenate([g[f"w0_{i:03d}"].ravel() for i in range(n)])
    t = make_trainer(cfg, 0, 4, 32)
    t.set_params(w0)
    assert np.array_equal(t.get_params(), w0)
    loss, norm = t.step_host(g["ids"], g["targets"])
    assert abs(loss - g["loss"][0]) <= 1e-5 * abs(g["loss"][0]), (loss, g["loss"][0])
    assert abs(norm - g["norm"][0]) <= 1e-4 * g["norm"][0], (norm, g["norm"][0])
    grads = split(cfg, t.get_grads())
    w1 = split(cfg, t.get_params())
    specs = O.param_specs(cfg)
    worst_g = max((O.max_abs_rel(grads[i], g[f"g_{i:03d}"]), specs[i][0]) for i in range(n))
    worst_w = max((O.max_abs_rel(w1[i], g[f"w1_{i:03d}"]), specs[i][0]) for i in range(n))
    assert worst_g[0] <= 1e-4, worst_g
    # AdamW's g / (|g| + eps) amplifies last-bit gradient differences where |g| ~ eps; the
    # reference compiled twice with different summation orders differs by the same amount
    assert worst_w[0] <= 2e-4, worst_w
    t.close()


def test_tiny_fp32_loss_decreases_and_is_log_v_at_init():
    cfg = O.TINY
    ids, tg = O.synthetic_batch(cfg, 4, 32, 0)
    t = make_trainer(cfg, 0, 4, 32)
    t.set_params(np.concatenate([p.ravel() for p in O.init_params(cfg, 0)]))
    first, _ = t.step_host(ids, tg)
    assert abs(first - math.log(cfg.vocab)) < 0.3
    last = first
    for _ in range(10):
        last, norm = t.step_host(ids, tg)
        assert math.isfinite(norm)
    assert last < first - 0.05
    t.close()


QWEN_SMALL = O.ModelConfig(vocab=2048, hidden=256, intermediate=512, layers=2, heads=4,
                           kv_heads=2, head_dim=128, eps=1e-6, theta=1e6)
# the Qwen3-1.7B widths (d_model 2048, SwiGLU 6144, 16/8 heads) at one layer and a small vocabulary
QWEN_WIDE = O.ModelConfig(vocab=2048, hidden=2048, intermediate=6144, layers=1, heads=16,
                          kv_heads=8, head_dim=128, eps=1e-6, theta=1e6)


# the full Qwen3-0.6B width and vocabulary (d_model 1024, SwiGLU 3072, 16/8 heads, head_dim 128,
# vocab 151936 with the tied embedding) at two layers
QWEN06_FULL_WIDTH = O.ModelConfig(vocab=151936, hidden=1024, intermediate=3072, layers=2, heads=16,
                                  kv_heads=8, head_dim=128, eps=1e-6, theta=1e6)


@pytest.mark.parametrize("cfg,B,T,recompute", [(QWEN_SMALL, 2, 128, False),
                                               (QWEN_WIDE, 1, 128, False),
                                               (QWEN_WIDE, 1, 256, True),
                                               (QWEN06_FULL_WIDTH, 1, 512, False)])
def test_qwen_shaped_bf16_step_matches_oracle(cfg, B, T, recompute):
    """One bf16 step (forward, cross-entropy, backward, clip, AdamW) against the oracle's fp32
    step on the same bf16-rounded weights and batch (src/libs/train/Model.cpp:206-255,
    src/libs/autograd/Loss.cpp:18-103, src/libs/optim/AdamW.cpp:38-93): loss, norm, every
    gradient and every updated weight. QWEN_WIDE with recompute is the Qwen3-1.7B layer width with
    activation recompute of attention; the last case is the Qwen3-0.6B width and vocabulary."""
    params = O.init_params(cfg, 3, bf16=True)
    ids, tg = O.synthetic_batch(cfg, B, T, 3)
    t = make_trainer(cfg, 1, B, T)
    t.set_recompute_attention(recompute)
    t.set_params(np.concatenate([p.ravel() for p in params]))
    loss, norm = t.step_host(ids, tg)
    ref = [p.copy() for p in params]
    opt = O.AdamW(ref, ADAM)
    rloss, rnorm, rgrads = O.train_step(cfg, ref, ids, tg, 1.0, opt)
    assert abs(loss - rloss) <= 2e-2 * abs(rloss)
    assert abs(norm - rnorm) <= 2e-2 * rnorm
    grads = split(cfg, t.get_grads())
    w1 = split(cfg, t.get_params())
    specs = O.param_specs(cfg)
    errs = sorted(((O.max_abs_rel(grads[i], rgrads[i]), specs[i][0]) for i in range(len(specs))),
                  reverse=True)
    assert errs[0][0] <= 2e-2, errs[:4]
    # Updated weights. AdamW's first step moves every element by about lr * sign(g), so an
    # element whose gradient is below bf16 resolution can take the opposite sign on the GPU and
    # land 2*lr away from the fp32 reference (measured: 0.2-0.8% of elements per tensor, which
    # puts the per-tensor max-abs-relative error at up to 2.4e-2 for matrices with |w| ~ 0.09).
    # Checked: the difference never exceeds those flips; a flip happens only where the reference
    # gradient is within the gradient tolerance (2e-2 of the tensor's largest gradient) of zero,
    # so its sign is not resolved at the stated precision; flips stay rare; and apart from them
    # the weights agree to 2e-2.
    lr = ADAM.learning_rate
    for i in range(len(specs)):
        dw_gpu, dw_ref = w1[i] - params[i], ref[i] - params[i]
        flips = np.sign(dw_gpu) != np.sign(dw_ref)
        assert np.max(np.abs(dw_gpu - dw_ref)) <= 2.02 * lr, specs[i][0]
        g_scale = np.abs(rgrads[i]).max()
        assert np.all(np.abs(rgrads[i])[flips] <= 2e-2 * g_scale), specs[i][0]
        assert flips.mean() <= 0.05, (specs[i][0], flips.mean())
        keep = ~flips
        den = np.abs(ref[i]).max()
        assert np.max(np.abs(w1[i] - ref[i])[keep], initial=0.0) <= 2e-2 * den, specs[i][0]
    t.close()


@pytest.mark.parametrize("cfg,B,T,seed", [(O.QWEN3_06B, 4, 2048, 3), (O.QWEN3_17B, 2, 4096, 4)])
def test_qwen_full_shape_step_properties(cfg, B, T, seed):
    """The Qwen3-0.6B (B 4 x T 2048) and Qwen3-1.7B (B 2 x T 4096) shaped steps at full size: the
    CPU oracle cannot run them, so check size-independent properties: initial loss ~ log V,
    finite grad norm, and a second step on the same batch lowering the loss."""
    ids, tg = O.synthetic_batch(cfg, B, T, seed)
    t = make_trainer(cfg, 1, B, T, seed=seed)
    t.set_recompute_attention(cfg is O.QWEN3_17B)   # the 1.7B step recomputes attention
    l1, n1 = t.step_host(ids, tg)
    l2, n2 = t.step_host(ids, tg)
    assert abs(l1 - math.log(cfg.vocab)) < 0.5, l1
    assert math.isfinite(n1) and math.isfinite(n2) and n1 > 0
    assert l2 < l1
    t.close()


def test_checkpoint_resume_is_bit_exact(tmp_path):
    """Save after one step, load into a fresh trainer, take the next step: the same loss, norm,
    gradients and weights as continuing without the checkpoint. The model file, read by the
    reference's own safetensors reader, holds the bf16 weights under the reference's names."""
    from oracle import ref as R
    cfg = QWEN_SMALL
    B, T = 2, 128
    params = O.init_params(cfg, 3, bf16=True)
    b1, b2 = O.synthetic_batch(cfg, B, T, 3), O.synthetic_batch(cfg, B, T, 4)
    t = make_trainer(cfg, 1, B, T)
    t.set_params(np.concatenate([p.ravel() for p in params]))
    t.step_host(*b1)
    w1 = t.get_params()
    ck = tmp_path / "ck"
    t.save(ck)
    loss, norm = t.step_host(*b2)
    w2, g2 = t.get_params(), t.get_grads()
    u = make_trainer(cfg, 1, B, T, seed=9)
    u.load(ck)
    assert np.array_equal(u.get_params(), w1)
    loss_u, norm_u = u.step_host(*b2)
    assert loss_u == loss and norm_u == norm
    assert np.array_equal(u.get_grads(), g2)
    assert np.array_equal(u.get_params(), w2)
    if R.available():
        got = R.read_safetensors(ck / "model.safetensors")
        specs = O.param_specs(cfg)
        assert [name for name, _ in got] == [name for name, _ in specs]
        for (name, arr), ref in zip(got, split(cfg, O.bf16_round(w1))):
            assert arr.shape == ref.shape and np.array_equal(arr, ref), name
    # weights only (no optimizer file): the bf16 weights, the optimizer starting afresh
    (ck / "optimizer.safetensors").unlink()
    v = make_trainer(cfg, 1, B, T, seed=11)
    v.load(ck)
    assert np.array_equal(v.get_params(), O.bf16_round(w1))
    for x in (t, u, v):
        x.close()


def test_nonfinite_step_is_skipped_and_not_counted():
    """set_skip_nonfinite: a step whose gradient norm is not finite (here an infinite final-norm
    gain makes the loss NaN) updates nothing and is reported as skipped; the step after it, with
    finite weights again, equals a fresh trainer's first step bit for bit (the skipped step was
    not counted, so the bias corrections are those of step 1)."""
    cfg = O.TINY
    ids, tg = O.synthetic_batch(cfg, 4, 32, 0)
    flat = np.concatenate([p.ravel() for p in O.init_params(cfg, 0)])
    bad = flat.copy()
    names = [name for name, _ in O.param_specs(cfg)]
    at = sum(int(np.prod(shape)) for name, shape in O.param_specs(cfg)[:names.index("model.norm.weight")])
    bad[at] = np.inf
    t = make_trainer(cfg, 0, 4, 32)
    t.set_skip_nonfinite(True)
    t.set_params(bad)
    loss, norm = t.step_host(ids, tg)
    assert not math.isfinite(norm) and t.step_skipped()
    got = t.get_params()
    assert np.array_equal(got[np.isfinite(got)], bad[np.isfinite(bad)])   # nothing was updated
    t.set_params(flat)
    loss2, norm2 = t.step_host(ids, tg)
    assert math.isfinite(norm2) and not t.step_skipped()
    fresh = make_trainer(cfg, 0, 4, 32)
    fresh.set_params(flat)
    loss3, norm3 = fresh.step_host(ids, tg)
    assert loss2 == loss3 and norm2 == norm3
    assert np.array_equal(t.get_params(), fresh.get_params())
    t.close()
    fresh.close()


def test_recompute_attention_is_bit_exact():
    """Activation recompute of attention forms q, k and the attention output again with the same
    deterministic kernels, so a trainer that recomputes (its step replayed from a CUDA graph) and
    one that keeps them (eager) agree bit for bit: losses, norms, gradients and weights. Switching
    recompute off mid-run drops the captured graph and the steps still agree."""
    cfg, B, T = QWEN_SMALL, 2, 128
    flat = np.concatenate([p.ravel() for p in O.init_params(cfg, 3, bf16=True)])
    a, b = make_trainer(cfg, 1, B, T), make_trainer(cfg, 1, B, T)
    a.set_params(flat)
    b.set_params(flat)
    a.set_recompute_attention(True)
    b.set_step_graph(False)
    for s in range(6):
        if s == 4:
            a.set_recompute_attention(False)
        ids, tg = O.synthetic_batch(cfg, B, T, 20 + s)
        la, na = a.step_host(ids, tg)
        lb, nb = b.step_host(ids, tg)
        assert la == lb and na == nb, (s, la, lb, na, nb)
    assert np.array_equal(a.get_grads(), b.get_grads())
    assert np.array_equal(a.get_params(), b.get_params())
    a.close()
    b.close()


def test_fused_mlp_is_bit_exact(monkeypatch):
    """The feed-forward block with SwiGLU in the GEMM epilogues (the bf16 default) and run as its
    three ops (VEDA_FUSED_MLP=0) give the same losses, norms, gradients and weights, bit for bit."""
    cfg, B, T = QWEN_SMALL, 2, 128
    flat = np.concatenate([p.ravel() for p in O.init_params(cfg, 3, bf16=True)])
    a, b = make_trainer(cfg, 1, B, T), make_trainer(cfg, 1, B, T)
    for t in (a, b):
        t.set_params(flat)
        t.set_step_graph(False)
    for s in range(3):
        ids, tg = O.synthetic_batch(cfg, B, T, 40 + s)
        monkeypatch.setenv("VEDA_FUSED_MLP", "1")
        la, na = a.step_host(ids, tg)
        monkeypatch.setenv("VEDA_FUSED_MLP", "0")
        lb, nb = b.step_host(ids, tg)
        assert la == lb and na == nb, (s, la, lb, na, nb)
    assert np.array_equal(a.get_grads(), b.get_grads())
    assert np.array_equal(a.get_params(), b.get_params())
    a.close()
    b.close()


@pytest.mark.parametrize("dtype", [0, 1])
def test_step_graph_replay_matches_eager(dtype):
    """A trainer replaying its step from a CUDA graph (captured at the second step) gives the same
    losses, norms, gradients and weights, bit for bit, as one launching every kernel eagerly."""
    cfg = O.TINY if dtype == 0 else QWEN_SMALL
    B, T = (4, 32) if dtype == 0 else (2, 128)
    flat = np.concatenate([p.ravel() for p in O.init_params(cfg, 3, bf16=dtype == 1)])
    a, b = make_trainer(cfg, dtype, B, T), make_trainer(cfg, dtype, B, T)
    a.set_params(flat)
    b.set_params(flat)
    b.set_step_graph(False)
    for s in range(5):
        ids, tg = O.synthetic_batch(cfg, B, T, 10 + s)
        la, na = a.step_host(ids, tg)
        lb, nb = b.step_host(ids, tg)
        assert la == lb and na == nb, (s, la, lb, na, nb)
    assert np.array_equal(a.get_grads(), b.get_grads())
    assert np.array_equal(a.get_params(), b.get_params())
    a.close()
    b.close()
