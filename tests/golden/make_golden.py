"""Generates the golden fixtures in this folder from the reference itself.

Runs the reference's CPU training path, compiled from its sources by oracle/Makefile into
oracle/_ref/libveda_ref.so, on seeded inputs and stores inputs and outputs as .npz files:

  tiny_step.npz      one full training step of the tiny decoder config (fp32; vocab 512, d 64,
                     2 layers, 4 query / 2 KV heads, head_dim 16, SwiGLU 192, tied embedding;
                     weights N(0, 0.02) seed 0, batch 4 x 32; clip 1.0; AdamW 1e-3, 0.9/0.95,
                     1e-8, wd 0.1): loss, pre-clip norm, pre-clip gradients, updated weights.
  ops_small.npz      per-op forward/backward cases (rms norm with gain, swiglu, softmax, CE,
                     embedding with repeats, rope, matmul_nt, causal GQA attention).

Usage:  python tests/golden/make_golden.py    (needs oracle/_ref built: make -C oracle)
"""
from __future__ import annotations

import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE.parent.parent))

from oracle import ref as R  # noqa: E402
from oracle import veda_oracle as O  # noqa: E402

F32 = np.float32
ADAM = O.AdamWConfig(1e-3, 0.9, 0.95, 1e-8, 0.1)


def tiny_step():
    c = O.TINY
    params = O.init_params(c, 0)
    ids, tg = O.synthetic_batch(c, 4, 32, 0)
    w, losses, norms, grads = R.train_steps(c, params, ids, tg, 1.0, ADAM, steps=1)
    out = {"ids": ids, "targets": tg, "loss": losses, "norm": norms}
    for i, (p, g, nw) in enumerate(zip(params, grads, w)):
        out[f"w0_{i:03d}"] = p
        out[f"g_{i:03d}"] = g
        out[f"w1_{i:03d}"] = nw
    np.savez_compressed(HERE / "tiny_step.npz", **out)


def ops_small():
    rng = np.random.default_rng(7)
    r = lambda *s: rng.standard_normal(s).astype(F32)  # noqa: E731
    out = {}
    x, gam, g = r(6, 40), (1 + 0.1 * r(40)).astype(F32), r(6, 40)
    y, dx, dg = R.rms_norm_gamma(x, gam, g, 1e-6)
    out.update(rms_x=x, rms_gamma=gam, rms_g=g, rms_y=y, rms_dx=dx, rms_dgamma=dg)

    ga, up, g = r(5, 24), r(5, 24), r(5, 24)
    y, dga, dup = R.swiglu(ga, up, g)
    out.update(swiglu_gate=ga, swiglu_up=up, swiglu_g=g, swiglu_y=y, swiglu_dgate=dga,
               swiglu_dup=dup)

    x, g = r(4, 33), r(4, 33)
    y, dx = R.softmax(x, g)
    out.update(softmax_x=x, softmax_g=g, softmax_y=y, softmax_dx=dx)

    lg = (3 * r(9, 77)).astype(F32)
    t = rng.integers(0, 77, size=9).astype(np.int64)
    loss, d = R.cross_entropy(lg, t)
    out.update(ce_logits=lg, ce_targets=t, ce_loss=np.array([loss]), ce_dlogits=d)

    table = r(11, 8)
    ids = np.array([3, 1, 3, 10, 0, 3, 7, 1], dtype=np.int64)
    g = r(8, 8)
    rows, dt = R.embedding(table, ids, g)
    out.update(emb_table=table, emb_ids=ids, emb_g=g, emb_rows=rows, emb_dtable=dt)

    x, g = r(3, 10, 16), r(3, 10, 16)
    y, dx = R.rope(x, g, 10000.0)
    cs, sn = R.rope_tables(10, 16, 10000.0)
    out.update(rope_x=x, rope_g=g, rope_y=y, rope_dx=dx, rope_cos=cs, rope_sin=sn)
    cs, sn = R.rope_tables(64, 128, 1e6)
    out.update(rope6_cos=cs, rope6_sin=sn)

    a, b, g = r(12, 20), r(9, 20), r(12, 9)
    y, da, db = R.matmul_nt(a, b, g)
    out.update(mm_a=a, mm_b=b, mm_g=g, mm_y=y, mm_da=da, mm_db=db)

    q, k, v, g = r(2, 4, 12, 16), r(2, 2, 12, 16), r(2, 2, 12, 16), r(2, 4, 12, 16)
    o, dq, dk, dv = R.attention(q, k, v, g)
    out.update(att_q=q, att_k=k, att_v=v, att_g=g, att_o=o, att_dq=dq, att_dk=dk, att_dv=dv)
    np.savez_compressed(HERE / "ops_small.npz", **out)


if __name__ == "__main__":
    if not R.available():
        sys.exit("oracle/_ref/libveda_ref.so is not built: make -C oracle")
    tiny_step()
    ops_small()
    print("wrote", sorted(p.name for p in HERE.glob("*.npz")))
