"""Test infrastructure only: the oracle for the training-step hot path.

A numpy restatement of the reference's CPU training path (pictaile/veda, fp32 throughout, with
double precision exactly where the reference uses it). Only the tests, ``__graft_entry__.smoke()``
and ``bench.py``'s CPU-baseline leg may import this module, and only as the checker: the product
path never calls it and has no CPU fallback.

Every function cites the reference file:line it restates. Parity of this restatement is pinned two
ways (see tests/test_oracle_*.py):
  * against the known-answer values of the reference's own tests (AdamWTest, CrossEntropyTest,
    GradientClipTest, AutogradNonLinearTest, AutogradViewsTest, AutogradMatmulTest);
  * against the reference itself, compiled from its sources into oracle/_ref/libveda_ref.so by
    oracle/Makefile and driven through oracle/ref_driver.cpp (oracle/ref.py loads it).

Layouts: activations are token-major ``[N, features]`` with N = B*T and token n = b*T + t, the
layout the reference's ``[B, T, D]`` tensors have in memory. Weights are ``[out, in]``
(src/libs/nn/Linear.cpp:57; y = x W^T).
"""
from __future__ import annotations

from dataclasses import dataclass, field
import math

import numpy as np

F32 = np.float32


# ---------------------------------------------------------------------------------------------
# bf16 helpers. The reference has no fp32->bf16 narrowing at all (it only widens at load,
# src/libs/tensor/BFloat16.h:26-41); this is round-to-nearest-even on the bit pattern.
# ---------------------------------------------------------------------------------------------
def bf16_round(x: np.ndarray) -> np.ndarray:
    """Round fp32 values to the nearest bf16 (ties to even); returns fp32 holding bf16 values."""
    a = np.ascontiguousarray(x, dtype=F32)
    bits = a.view(np.uint32).astype(np.uint64)
    rounding = ((bits >> 16) & 1) + 0x7FFF
    out = ((bits + rounding) >> 16) << 16
    out = out.astype(np.uint32)
    nan = np.isnan(a)
    if nan.any():
        out[nan] = 0x7FC00000
    return out.view(F32).reshape(a.shape)


def bf16_bits(x: np.ndarray) -> np.ndarray:
    """The uint16 bf16 encodings of fp32 values (rounded to nearest even)."""
    return (bf16_round(x).view(np.uint32) >> 16).astype(np.uint16)


def bf16_from_bits(b: np.ndarray) -> np.ndarray:
    return (b.astype(np.uint32) << 16).view(F32)


# ---------------------------------------------------------------------------------------------
# Element-wise and per-lane ops
# ---------------------------------------------------------------------------------------------
def rms_normalize(x: np.ndarray, eps: float):
    """y = x / sqrt(mean(x^2) + eps) over the last dim, fp32.  Returns (y, r).

    src/libs/ops/Normalize.cpp:18-70 (eps inside the root, :58-59).
    """
    x = x.astype(F32, copy=False)
    n = x.shape[-1]
    ss = np.sum(x * x, axis=-1, dtype=F32, keepdims=True)
    r = np.sqrt(ss / F32(n) + F32(eps)).astype(F32)
    return (x / r).astype(F32), r


def rms_normalize_backward(x: np.ndarray, g: np.ndarray, eps: float) -> np.ndarray:
    """dx = g/r - x * sum(g x) / (n r^3).   src/libs/autograd/NonLinear.cpp:153-201."""
    x = x.astype(F32, copy=False)
    g = g.astype(F32, copy=False)
    n = x.shape[-1]
    ss = np.sum(x * x, axis=-1, dtype=F32, keepdims=True)
    w = np.sum(g * x, axis=-1, dtype=F32, keepdims=True)
    r = np.sqrt(ss / F32(n) + F32(eps)).astype(F32)
    coupling = (w / (F32(n) * r * r * r)).astype(F32)
    return (g / r - x * coupling).astype(F32)


def rms_norm_gamma(x, gamma, eps):
    """mul(rms_normalize(x), gamma) — the pre-norm of src/libs/train/Model.cpp:242-243."""
    y, r = rms_normalize(x, eps)
    return (y * gamma.astype(F32)).astype(F32), y, r


def rms_norm_gamma_backward(x, gamma, g, eps):
    """Returns (dx, dgamma). The gamma mul's backward is mul + unbroadcast
    (src/libs/autograd/Variable.cpp:218-239, 48-87): dgamma = sum over rows of g * x_hat."""
    xhat, _ = rms_normalize(x, eps)
    lead = tuple(range(x.ndim - 1))
    dgamma = np.sum((g * xhat).astype(F32), axis=lead, dtype=F32)
    dx = rms_normalize_backward(x, (g * gamma).astype(F32), eps)
    return dx, dgamma.astype(F32)


def sigmoid(x):
    return (F32(1) / (F32(1) + np.exp(-x.astype(F32)))).astype(F32)


def silu(x):
    """x / (1 + exp(-x)).   src/libs/ops/Activations.cpp:13-16."""
    x = x.astype(F32, copy=False)
    return (x / (F32(1) + np.exp(-x))).astype(F32)


def silu_backward(x, g):
    """g * s * (1 + x (1 - s)).   src/libs/autograd/NonLinear.cpp:47-63."""
    s = sigmoid(x)
    return (g * s * (F32(1) + x * (F32(1) - s))).astype(F32)


def swiglu(gate, up):
    """mul(silu(gate), up).   src/libs/train/Model.cpp:201-202."""
    return (silu(gate) * up).astype(F32)


def swiglu_backward(gate, up, g):
    """Returns (dgate, dup).   Variable.cpp:218-239 (mul) and NonLinear.cpp:47-63 (silu)."""
    dgate = silu_backward(gate, (g * up).astype(F32))
    dup = (g * silu(gate)).astype(F32)
    return dgate, dup


def softmax(x, axis=-1):
    """max, exp(x - max), sum, divide; fp32.   src/libs/ops/Softmax.cpp:20-80."""
    x = x.astype(F32, copy=False)
    m = np.max(x, axis=axis, keepdims=True)
    e = np.exp(x - m).astype(F32)
    return (e / np.sum(e, axis=axis, dtype=F32, keepdims=True)).astype(F32)


def softmax_backward(y, g, axis=-1):
    """y * (g - sum(g y)).   src/libs/autograd/NonLinear.cpp:89-151."""
    w = np.sum((g * y).astype(F32), axis=axis, dtype=F32, keepdims=True)
    return (y * (g - w)).astype(F32)


def log_softmax(x, axis=-1):
    """x - max - log(sum exp(x - max)); an all -inf lane stays -inf.
    src/libs/ops/Softmax.cpp:82-151."""
    x = x.astype(F32, copy=False)
    m = np.max(x, axis=axis, keepdims=True)
    with np.errstate(invalid="ignore", divide="ignore"):
        s = np.sum(np.exp(x - m), axis=axis, dtype=F32, keepdims=True)
        out = (x - m - np.log(s)).astype(F32)
    dead = np.isneginf(m).squeeze(axis)
    if np.any(dead):
        out[dead] = -np.inf
    return out


def cross_entropy(logits, targets):
    """Mean CE over lanes (sum in double), and dlogits for an upstream seed of 1.

    src/libs/autograd/Loss.cpp:18-103: loss = mean(-log_softmax[target]) accumulated in double
    (:52-60); backward = (p - onehot) * (g / lanes) with p = exp(log_softmax) (:69-99).
    Raises ValueError on a target outside [0, V) or a count mismatch (:21-47).
    """
    logits = logits.astype(F32, copy=False)
    V = logits.shape[-1]
    lp = log_softmax(logits.reshape(-1, V))
    lanes = lp.shape[0]
    targets = np.asarray(targets, dtype=np.int64).reshape(-1)
    if targets.size != lanes:
        raise ValueError(f"cross_entropy: {targets.size} targets for {lanes} lanes")
    if lanes == 0:
        raise ValueError("cross_entropy: nothing to average over")
    if np.any(targets < 0) or np.any(targets >= V):
        raise ValueError("cross_entropy: target outside [0, V)")
    picked = lp[np.arange(lanes), targets].astype(np.float64)
    loss = F32(np.sum(-picked) / float(lanes))
    seed = F32(1.0) / F32(lanes)
    p = np.exp(lp).astype(F32)
    d = (seed * p).astype(F32)
    d[np.arange(lanes), targets] -= seed
    return loss, d.reshape(logits.shape)


def cross_entropy_rows(logits, targets):
    """Per-row -log p_target (fp32) — the quantity a row-parallel kernel produces before the
    double-precision mean of Loss.cpp:52-60."""
    V = logits.shape[-1]
    lp = log_softmax(logits.reshape(-1, V))
    t = np.asarray(targets, dtype=np.int64).reshape(-1)
    return (-lp[np.arange(lp.shape[0]), t]).astype(F32)


def embedding(table, ids):
    """Row gather, bit-exact.   src/libs/autograd/NonLinear.cpp:203-236."""
    ids = np.asarray(ids, dtype=np.int64).reshape(-1)
    V = table.shape[0]
    if np.any(ids < 0) or np.any(ids >= V):
        raise IndexError("embedding: token id outside the vocabulary")
    return table[ids].copy()


def embedding_backward(dtable, ids, g):
    """dtable[id[p]] += g[p], positions in ascending order, fp32 — the sequential loop of
    src/libs/autograd/NonLinear.cpp:245-252. Mutates and returns dtable."""
    ids = np.asarray(ids, dtype=np.int64).reshape(-1)
    g = g.reshape(ids.size, -1).astype(F32, copy=False)
    for p in range(ids.size):
        dtable[ids[p]] += g[p]
    return dtable


def rope_tables(positions: int, head_dim: int, theta: float):
    """cos/sin [T, Dh]: angle = t * theta^(-2i/Dh) in double, cast to fp32 per element, each
    angle written to both halves (i and i + Dh/2).   src/libs/model/Rope.cpp:17-63."""
    if head_dim == 0 or head_dim % 2:
        raise ValueError("rope_tables: head_dim must be even")
    pairs = head_dim // 2
    i = np.arange(pairs, dtype=np.float64)
    freq = np.power(np.float64(np.float32(theta)), -2.0 * i / float(head_dim))
    ang = np.arange(positions, dtype=np.float64)[:, None] * freq[None, :]
    c = np.cos(ang).astype(F32)
    s = np.sin(ang).astype(F32)
    return np.concatenate([c, c], axis=1), np.concatenate([s, s], axis=1)


def rope(x, cos, sin):
    """Half-split rotation on [..., T, Dh]: out_i = x_i c - x_{i+p} s; out_{i+p} = x_{i+p} c +
    x_i s.   src/libs/autograd/Views.cpp:78-134."""
    p = x.shape[-1] // 2
    a, b = x[..., :p], x[..., p:]
    c, s = cos[..., :p], sin[..., :p]
    return np.concatenate([a * c - b * s, b * c + a * s], axis=-1).astype(F32)


def rope_backward(g, cos, sin):
    """Rotation by -theta.   src/libs/autograd/Views.cpp:136-171."""
    p = g.shape[-1] // 2
    a, b = g[..., :p], g[..., p:]
    c, s = cos[..., :p], sin[..., :p]
    return np.concatenate([a * c + b * s, b * c - a * s], axis=-1).astype(F32)


# ---------------------------------------------------------------------------------------------
# Attention (causal, GQA with contiguous groups kv = h // (H/Hkv), src/libs/model/Attention.cpp:191)
# composed as src/libs/train/Model.cpp:182-189: scores = q k^T * (1/sqrt(Dh)); + mask; softmax; @ v
# ---------------------------------------------------------------------------------------------
def attention(q, k, v, scale=None):
    """q [B,H,T,Dh], k/v [B,Hkv,T,Dh] -> (out [B,H,T,Dh], lse [B,H,T], P [B,H,T,T])."""
    B, H, T, Dh = q.shape
    Hk = k.shape[1]
    rep = H // Hk
    if scale is None:
        scale = F32(1.0) / F32(math.sqrt(Dh))
    kx = np.repeat(k, rep, axis=1)
    vx = np.repeat(v, rep, axis=1)
    s = (np.matmul(q, np.swapaxes(kx, -1, -2)).astype(F32) * F32(scale)).astype(F32)
    mask = np.triu(np.ones((T, T), dtype=bool), 1)
    s = np.where(mask, -np.inf, s).astype(F32)
    m = np.max(s, axis=-1, keepdims=True)
    e = np.exp(s - m).astype(F32)
    z = np.sum(e, axis=-1, dtype=F32, keepdims=True)
    p = (e / z).astype(F32)
    lse = (m + np.log(z)).astype(F32)[..., 0]
    return np.matmul(p, vx).astype(F32), lse, p


def attention_backward(q, k, v, p, do, scale=None):
    """dq, dk, dv; dk/dv summed over the H/Hkv query heads of each group (the unbroadcast of the
    KV expansion). Softmax backward NonLinear.cpp:123-133, matmul backwards Variable.cpp:300-346."""
    B, H, T, Dh = q.shape
    Hk = k.shape[1]
    rep = H // Hk
    if scale is None:
        scale = F32(1.0) / F32(math.sqrt(Dh))
    kx = np.repeat(k, rep, axis=1)
    vx = np.repeat(v, rep, axis=1)
    dvx = np.matmul(np.swapaxes(p, -1, -2), do).astype(F32)
    dp = np.matmul(do, np.swapaxes(vx, -1, -2)).astype(F32)
    ds = softmax_backward(p, dp) * F32(scale)
    ds = ds.astype(F32)
    dq = np.matmul(ds, kx).astype(F32)
    dkx = np.matmul(np.swapaxes(ds, -1, -2), q).astype(F32)
    dk = dkx.reshape(B, Hk, rep, T, Dh).sum(axis=2, dtype=F32)
    dv = dvx.reshape(B, Hk, rep, T, Dh).sum(axis=2, dtype=F32)
    return dq, dk.astype(F32), dv.astype(F32)


# ---------------------------------------------------------------------------------------------
# Optimiser
# ---------------------------------------------------------------------------------------------
def clip_gradient_norm(grads: list, max_norm: float) -> float:
    """Global-norm clip in place; returns the pre-clip norm.   src/libs/optim/Clip.cpp:12-61.

    sum of g^2 in double; non-finite total -> returned, nothing scaled; total <= max -> nothing
    written; else every g *= float(max / total) in fp32."""
    if not (max_norm > 0):
        raise ValueError("clip_gradient_norm: max_norm must be positive")
    sq = 0.0
    for g in grads:
        gd = g.astype(np.float64).ravel()
        sq += float(np.dot(gd, gd))
    total = math.sqrt(sq) if sq == sq else float("nan")
    if not math.isfinite(total):
        return F32(total)
    if total <= float(np.float32(max_norm)):
        return F32(total)
    scale = F32(float(np.float32(max_norm)) / total)
    for g in grads:
        g *= scale
    return F32(total)


@dataclass
class AdamWConfig:
    """src/libs/optim/AdamW.h:23-30 (defaults are the reference's)."""
    learning_rate: float = 1e-3
    beta1: float = 0.9
    beta2: float = 0.999
    eps: float = 1e-8
    weight_decay: float = 0.01


@dataclass
class AdamW:
    """Decoupled AdamW, fp32 moments, double bias correction and m_hat/v_hat.
    src/libs/optim/AdamW.cpp:15-109."""
    params: list
    config: AdamWConfig = field(default_factory=AdamWConfig)
    steps: int = 0

    def __post_init__(self):
        c = self.config
        if c.learning_rate < 0 or c.eps <= 0 or c.weight_decay < 0:
            raise ValueError("AdamW: learning rate, eps and weight decay must be positive")
        if not (0 <= c.beta1 < 1 and 0 <= c.beta2 < 1):
            raise ValueError("AdamW: betas must lie in [0, 1)")
        self.m = [np.zeros_like(p, dtype=F32) for p in self.params]
        self.v = [np.zeros_like(p, dtype=F32) for p in self.params]

    def step(self, grads: list, frozen=()):
        self.steps += 1
        c = self.config
        b1, b2 = F32(c.beta1), F32(c.beta2)
        lr, wd, eps = F32(c.learning_rate), F32(c.weight_decay), F32(c.eps)
        bias1 = 1.0 - math.pow(float(b1), float(self.steps))
        bias2 = 1.0 - math.pow(float(b2), float(self.steps))
        for i, (w, g) in enumerate(zip(self.params, grads)):
            if i in frozen:
                continue
            g = g.astype(F32, copy=False)
            self.m[i] = (b1 * self.m[i] + (F32(1) - b1) * g).astype(F32)
            self.v[i] = (b2 * self.v[i] + (F32(1) - b2) * g * g).astype(F32)
            m_hat = self.m[i].astype(np.float64) / bias1
            v_hat = self.v[i].astype(np.float64) / bias2
            adaptive = (m_hat / (np.sqrt(v_hat) + float(eps))).astype(F32)
            w -= (lr * wd * w).astype(F32)
            w -= (lr * adaptive).astype(F32)


# ---------------------------------------------------------------------------------------------
# The Qwen3-shaped decoder step (src/libs/train/Model.cpp:154-255 with GQA), forward + manual
# backward + clip + AdamW. Parameter order and names: Model.cpp:120-140.
# ---------------------------------------------------------------------------------------------
@dataclass
class ModelConfig:
    vocab: int
    hidden: int
    intermediate: int
    layers: int
    heads: int
    kv_heads: int
    head_dim: int
    eps: float = 1e-6
    theta: float = 10000.0


TINY = ModelConfig(vocab=512, hidden=64, intermediate=192, layers=2, heads=4, kv_heads=2,
                   head_dim=16, eps=1e-6, theta=10000.0)
QWEN3_06B = ModelConfig(vocab=151936, hidden=1024, intermediate=3072, layers=28, heads=16,
                        kv_heads=8, head_dim=128, eps=1e-6, theta=1e6)
QWEN3_17B = ModelConfig(vocab=151936, hidden=2048, intermediate=6144, layers=28, heads=16,
                        kv_heads=8, head_dim=128, eps=1e-6, theta=1e6)


def param_specs(c: ModelConfig):
    """(name, shape) in the order of src/libs/train/Model.cpp:120-140 (k/v are [Hkv*Dh, D])."""
    D, F, H, Hk, Dh, V = c.hidden, c.intermediate, c.heads, c.kv_heads, c.head_dim, c.vocab
    specs = [("model.embed_tokens.weight", (V, D))]
    for l in range(c.layers):
        pre = f"model.layers.{l}."
        specs += [
            (pre + "input_layernorm.weight", (D,)),
            (pre + "self_attn.q_proj.weight", (H * Dh, D)),
            (pre + "self_attn.k_proj.weight", (Hk * Dh, D)),
            (pre + "self_attn.v_proj.weight", (Hk * Dh, D)),
            (pre + "self_attn.o_proj.weight", (D, H * Dh)),
            (pre + "self_attn.q_norm.weight", (Dh,)),
            (pre + "self_attn.k_norm.weight", (Dh,)),
            (pre + "post_attention_layernorm.weight", (D,)),
            (pre + "mlp.gate_proj.weight", (F, D)),
            (pre + "mlp.up_proj.weight", (F, D)),
            (pre + "mlp.down_proj.weight", (D, F)),
        ]
    specs.append(("model.norm.weight", (D,)))
    return specs


def init_params(c: ModelConfig, seed: int, bf16: bool = False):
    """Seeded weights: matrices ~ N(0, 0.02), norm gains 1; optionally rounded to bf16 values so
    an fp32 CPU run and a bf16 GPU run start from identical numbers."""
    rng = np.random.default_rng(seed)
    out = []
    for name, shape in param_specs(c):
        if len(shape) == 1:
            w = np.ones(shape, dtype=F32)
        else:
            w = (rng.standard_normal(shape, dtype=F32) * F32(0.02)).astype(F32)
            if bf16:
                w = bf16_round(w)
        out.append(w)
    return out


def synthetic_batch(c: ModelConfig, batch: int, length: int, seed: int):
    """ids uniform in [0, V) over windows of T+1 tokens; inputs are the first T, targets the next
    T (the shifted-by-one rule of src/libs/data/Corpus.cpp:99-103)."""
    rng = np.random.default_rng(seed)
    window = rng.integers(0, c.vocab, size=(batch, length + 1), dtype=np.int64)
    return window[:, :-1].copy(), window[:, 1:].copy()


def _unpack(c: ModelConfig, params):
    it = iter(params)
    embed = next(it)
    layers = []
    for _ in range(c.layers):
        layers.append({k: next(it) for k in ("in_norm", "q", "k", "v", "o", "q_norm", "k_norm",
                                             "post_norm", "gate", "up", "down")})
    final = next(it)
    return embed, layers, final


def forward_backward(c: ModelConfig, params, ids, targets):
    """One forward + cross-entropy + full backward. Returns (loss, grads in parameter order).
    Activations fp32; the op order of src/libs/train/Model.cpp:206-255."""
    ids = np.asarray(ids, dtype=np.int64)
    B, T = ids.shape
    N = B * T
    D, H, Hk, Dh = c.hidden, c.heads, c.kv_heads, c.head_dim
    rep = H // Hk
    eps = c.eps
    embed, layers, final = _unpack(c, params)
    cos, sin = rope_tables(T, Dh, c.theta)
    scale = F32(1.0) / F32(math.sqrt(Dh))

    def heads_of(a, nh):  # [N, nh*Dh] -> [B, nh, T, Dh]
        return a.reshape(B, T, nh, Dh).transpose(0, 2, 1, 3)

    def tokens_of(a):  # [B, nh, T, Dh] -> [N, nh*Dh]
        return np.ascontiguousarray(a.transpose(0, 2, 1, 3)).reshape(N, -1)

    x = embedding(embed, ids)
    saved = []
    for L in layers:
        s = {"x": x}
        a, s["xhat1"], _ = rms_norm_gamma(x, L["in_norm"], eps)
        s["a"] = a
        q = (a @ L["q"].T).astype(F32)
        k = (a @ L["k"].T).astype(F32)
        v = (a @ L["v"].T).astype(F32)
        qh, kh, vh = heads_of(q, H), heads_of(k, Hk), heads_of(v, Hk)
        s["qh"], s["kh"], s["vh"] = qh, kh, vh
        qn, _, _ = rms_norm_gamma(qh, L["q_norm"], eps)
        kn, _, _ = rms_norm_gamma(kh, L["k_norm"], eps)
        qr, kr = rope(qn, cos, sin), rope(kn, cos, sin)
        s["qr"], s["kr"] = qr, kr
        ctx, _, p = attention(qr, kr, vh, scale)
        s["p"] = p
        ctx_t = tokens_of(ctx)
        s["ctx"] = ctx_t
        x1 = (x + ctx_t @ L["o"].T).astype(F32)
        s["x1"] = x1
        b, _, _ = rms_norm_gamma(x1, L["post_norm"], eps)
        s["b"] = b
        g = (b @ L["gate"].T).astype(F32)
        u = (b @ L["up"].T).astype(F32)
        s["g"], s["u"] = g, u
        h = swiglu(g, u)
        s["h"] = h
        x = (x1 + h @ L["down"].T).astype(F32)
        saved.append(s)
    xf, _, _ = rms_norm_gamma(x, final, eps)
    logits = (xf @ embed.T).astype(F32)
    loss, dlogits = cross_entropy(logits, targets)

    grads = {}
    d_embed = (dlogits.T @ xf).astype(F32)
    dxf = (dlogits @ embed).astype(F32)
    dx, d_final = rms_norm_gamma_backward(x, final, dxf, eps)
    layer_grads = []
    for L, s in zip(reversed(layers), reversed(saved)):
        G = {}
        # x = x1 + h W_down^T
        G["down"] = (dx.T @ s["h"]).astype(F32)
        dh = (dx @ L["down"]).astype(F32)
        dg, du = swiglu_backward(s["g"], s["u"], dh)
        G["gate"] = (dg.T @ s["b"]).astype(F32)
        G["up"] = (du.T @ s["b"]).astype(F32)
        db = (dg @ L["gate"] + du @ L["up"]).astype(F32)
        dx1n, G["post_norm"] = rms_norm_gamma_backward(s["x1"], L["post_norm"], db, eps)
        dx1 = (dx + dx1n).astype(F32)
        # x1 = x + ctx W_o^T
        G["o"] = (dx1.T @ s["ctx"]).astype(F32)
        dctx = heads_of((dx1 @ L["o"]).astype(F32), H)
        dqr, dkr, dvh = attention_backward(s["qr"], s["kr"], s["vh"], s["p"], dctx, scale)
        dqn, dkn = rope_backward(dqr, cos, sin), rope_backward(dkr, cos, sin)
        dqh, G["q_norm"] = rms_norm_gamma_backward(s["qh"], L["q_norm"], dqn, eps)
        dkh, G["k_norm"] = rms_norm_gamma_backward(s["kh"], L["k_norm"], dkn, eps)
        dq, dk, dv = tokens_of(dqh), tokens_of(dkh), tokens_of(dvh)
        G["q"] = (dq.T @ s["a"]).astype(F32)
        G["k"] = (dk.T @ s["a"]).astype(F32)
        G["v"] = (dv.T @ s["a"]).astype(F32)
        da = (dq @ L["q"] + dk @ L["k"] + dv @ L["v"]).astype(F32)
        dxn, G["in_norm"] = rms_norm_gamma_backward(s["x"], L["in_norm"], da, eps)
        dx = (dx1 + dxn).astype(F32)
        layer_grads.append(G)
    layer_grads.reverse()
    embedding_backward(d_embed, ids, dx)

    out = [d_embed]
    for G in layer_grads:
        out += [G[k] for k in ("in_norm", "q", "k", "v", "o", "q_norm", "k_norm", "post_norm",
                               "gate", "up", "down")]
    out.append(d_final)
    del grads
    return loss, out


def train_step(c: ModelConfig, params, ids, targets, max_norm: float, opt: AdamW):
    """zero_grad, forward, CE, backward, clip, AdamW — tests/TinyModelTest.cpp:290-299.
    Mutates params through opt; returns (loss, pre-clip norm, pre-clip grads)."""
    loss, grads = forward_backward(c, params, ids, targets)
    pre = [g.copy() for g in grads]
    norm = clip_gradient_norm(grads, max_norm)
    opt.step(grads)
    return loss, norm, pre


def max_abs_rel(a, b) -> float:
    """Per-tensor max-abs-relative error: max|a - b| / max|b| (0 when both are all zero)."""
    a = np.asarray(a, dtype=np.float64)
    b = np.asarray(b, dtype=np.float64)
    den = float(np.max(np.abs(b))) if b.size else 0.0
    num = float(np.max(np.abs(a - b))) if a.size else 0.0
    if den == 0.0:
        return num
    return num / den


# ---- corpus batcher ----------------------------------------------------------------------------
_U64 = (1 << 64) - 1
_GOLDEN = 0x9E3779B97F4A7C15


class Corpus:
    """The reference's batcher, restated (src/libs/data/Corpus.cpp:25-107): contiguous split at
    int(size * (1 - validation_fraction)); splitmix64 (state += 0x9E3779B97F4A7C15, then the
    published mix) with seed 0 meaning 0x9E3779B97F4A7C15; one draw per row, start = begin +
    draw % (available - window + 1); targets are the inputs' successors."""

    def __init__(self, ids, validation_fraction, seed):
        if not 0.0 <= validation_fraction <= 1.0:
            raise ValueError("Corpus: validation_fraction must lie in [0, 1]")
        self.ids = np.asarray(ids, dtype=np.int64)
        self.boundary = min(int(float(len(self.ids)) * (1.0 - validation_fraction)), len(self.ids))
        self.state = _GOLDEN if seed == 0 else seed & _U64

    def _next_random(self):
        # Corpus.cpp:55-64
        self.state = (self.state + _GOLDEN) & _U64
        z = self.state
        z = ((z ^ (z >> 30)) * 0xBF58476D1CE4E5B9) & _U64
        z = ((z ^ (z >> 27)) * 0x94D049BB133111EB) & _U64
        return z ^ (z >> 31)

    def next_batch(self, batch, length, split="train"):
        # Corpus.cpp:66-107
        if batch == 0 or length == 0:
            raise ValueError("Corpus: batch size and length must be positive")
        begin, end = (0, self.boundary) if split == "train" else (self.boundary, len(self.ids))
        window = length + 1
        if end - begin < window:
            raise ValueError("Corpus: the split is shorter than one window")
        offsets = end - begin - window + 1
        inputs = np.empty((batch, length), np.int64)
        targets = np.empty((batch, length), np.int64)
        for row in range(batch):
            start = begin + self._next_random() % offsets
            inputs[row] = self.ids[start:start + length]
            targets[row] = self.ids[start + 1:start + length + 1]
        return inputs, targets


# ---- generation --------------------------------------------------------------------------------
def forward_logits(c: ModelConfig, params, ids):
    """Logits [T, V] of one sequence (the forward of forward_backward, Model.cpp:206-255)."""
    ids = np.asarray(ids, dtype=np.int64).reshape(1, -1)
    T = ids.shape[1]
    D, H, Hk, Dh = c.hidden, c.heads, c.kv_heads, c.head_dim
    embed, layers, final = _unpack(c, params)
    cos, sin = rope_tables(T, Dh, c.theta)
    scale = F32(1.0) / F32(math.sqrt(Dh))

    def heads_of(a, nh):
        return a.reshape(1, T, nh, Dh).transpose(0, 2, 1, 3)

    x = embedding(embed, ids)
    for L in layers:
        a, _, _ = rms_norm_gamma(x, L["in_norm"], c.eps)
        q, k, v = ((a @ L[n].T).astype(F32) for n in ("q", "k", "v"))
        qn, _, _ = rms_norm_gamma(heads_of(q, H), L["q_norm"], c.eps)
        kn, _, _ = rms_norm_gamma(heads_of(k, Hk), L["k_norm"], c.eps)
        ctx, _, _ = attention(rope(qn, cos, sin), rope(kn, cos, sin), heads_of(v, Hk), scale)
        ctx = np.ascontiguousarray(ctx.transpose(0, 2, 1, 3)).reshape(T, -1)
        x = (x + ctx @ L["o"].T).astype(F32)
        b, _, _ = rms_norm_gamma(x, L["post_norm"], c.eps)
        h = swiglu((b @ L["gate"].T).astype(F32), (b @ L["up"].T).astype(F32))
        x = (x + h @ L["down"].T).astype(F32)
    xf, _, _ = rms_norm_gamma(x, final, c.eps)
    return (xf @ embed.T).astype(F32)


def greedy(logits):
    """The first index of the largest logit; NaN raises (Sampling.cpp:97-113)."""
    logits = np.asarray(logits, dtype=F32).ravel()
    if np.isnan(logits).any():
        raise ValueError("generate: a logit is NaN")
    return int(np.argmax(logits))   # numpy returns the first maximum


def generate(c: ModelConfig, params, prompt, max_new_tokens, stop_tokens=()):
    """The uncached generation loop of Generator.cpp:20-55 with greedy sampling: (tokens,
    stopped_on_token, forward_passes)."""
    ids = list(prompt)
    out, passes = [], 0
    for _ in range(max_new_tokens):
        nxt = greedy(forward_logits(c, params, ids)[-1])
        passes += 1
        if nxt in stop_tokens:
            return out, True, passes
        out.append(nxt)
        ids.append(nxt)
    return out, False, passes
