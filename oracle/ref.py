"""Test infrastructure only: numpy wrappers over the reference compiled from its own sources.

oracle/Makefile compiles the reference's CPU training path (src/libs/{tensor,ops,autograd,optim,
train} and model/Rope.cpp) together with oracle/ref_driver.cpp into oracle/_ref/libveda_ref.so.
This module loads that library with ctypes. ``available()`` is False when it has not been built
(the build needs the reference checkout; the built .so travels with the repository snapshot).
"""
from __future__ import annotations

import ctypes as C
import os
from pathlib import Path

import numpy as np

_HERE = Path(__file__).resolve().parent
LIB_PATH = _HERE / "_ref" / "libveda_ref.so"
_lib = None

F32P = np.ctypeslib.ndpointer(dtype=np.float32, flags="C_CONTIGUOUS")
I64P = np.ctypeslib.ndpointer(dtype=np.int64, flags="C_CONTIGUOUS")


class VrefModelConfig(C.Structure):
    _fields_ = [("vocab", C.c_int64), ("hidden", C.c_int64), ("intermediate", C.c_int64),
                ("layers", C.c_int64), ("heads", C.c_int64), ("kv_heads", C.c_int64),
                ("head_dim", C.c_int64), ("eps", C.c_float), ("theta", C.c_float)]


class VrefAdamConfig(C.Structure):
    _fields_ = [("lr", C.c_float), ("beta1", C.c_float), ("beta2", C.c_float),
                ("eps", C.c_float), ("weight_decay", C.c_float)]


def build(ref_dir: str | None = None) -> bool:
    """Run oracle/Makefile when the reference checkout (ref_dir, else $VEDA_REF_DIR) is present.
    Returns True if the library exists afterwards."""
    import subprocess
    ref_dir = ref_dir or os.environ.get("VEDA_REF_DIR")
    if not ref_dir or not Path(ref_dir, "src", "libs", "autograd", "Variable.cpp").exists():
        return LIB_PATH.exists()
    subprocess.run(["make", "-s", "-C", str(_HERE), f"VEDA_REF_DIR={ref_dir}",
                    f"-j{os.cpu_count() or 4}"], check=True)
    return LIB_PATH.exists()


def available() -> bool:
    return LIB_PATH.exists()


def lib():
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            raise FileNotFoundError(f"{LIB_PATH} is not built (make -C oracle)")
        L = C.CDLL(str(LIB_PATH))
        L.vref_last_error.restype = C.c_char_p
        L.vref_param_count.restype = C.c_int64
        L.vref_param_count.argtypes = [C.POINTER(VrefModelConfig)]
        L.vref_set_threads.argtypes = [C.c_int64]
        _lib = L
    return _lib


def _check(rc):
    if rc != 0:
        msg = lib().vref_last_error().decode()
        if rc == -5:
            raise IndexError(msg)
        if rc == -1:
            raise ValueError(msg)
        raise RuntimeError(msg)


def _f(a):
    return np.ascontiguousarray(a, dtype=np.float32)


def _p(a):
    return a.ctypes.data_as(C.c_void_p)


def set_threads(n: int):
    lib().vref_set_threads(int(n))


def rms_normalize(x, g, eps):
    x, g = _f(x), _f(g)
    rows, n = x.reshape(-1, x.shape[-1]).shape
    y, dx = np.empty_like(x), np.empty_like(x)
    _check(lib().vref_rms_normalize(_p(x), _p(g), C.c_int64(rows), C.c_int64(n), C.c_float(eps),
                                    _p(y), _p(dx)))
    return y, dx


def rms_norm_gamma(x, gamma, g, eps):
    x, gamma, g = _f(x), _f(gamma), _f(g)
    rows, n = x.reshape(-1, x.shape[-1]).shape
    y, dx, dgamma = np.empty_like(x), np.empty_like(x), np.empty_like(gamma)
    _check(lib().vref_rms_norm_gamma(_p(x), _p(gamma), _p(g), C.c_int64(rows), C.c_int64(n),
                                     C.c_float(eps), _p(y), _p(dx), _p(dgamma)))
    return y, dx, dgamma


def silu(x, g):
    x, g = _f(x), _f(g)
    y, dx = np.empty_like(x), np.empty_like(x)
    _check(lib().vref_silu(_p(x), _p(g), C.c_int64(x.size), _p(y), _p(dx)))
    return y, dx


def swiglu(gate, up, g):
    gate, up, g = _f(gate), _f(up), _f(g)
    rows, n = gate.reshape(-1, gate.shape[-1]).shape
    y, dg, du = np.empty_like(gate), np.empty_like(gate), np.empty_like(gate)
    _check(lib().vref_swiglu(_p(gate), _p(up), _p(g), C.c_int64(rows), C.c_int64(n), _p(y),
                             _p(dg), _p(du)))
    return y, dg, du


def softmax(x, g):
    x, g = _f(x), _f(g)
    lanes, n = x.reshape(-1, x.shape[-1]).shape
    y, dx = np.empty_like(x), np.empty_like(x)
    _check(lib().vref_softmax(_p(x), _p(g), C.c_int64(lanes), C.c_int64(n), _p(y), _p(dx)))
    return y, dx


def cross_entropy(logits, targets):
    logits = _f(logits)
    V = logits.shape[-1]
    lanes = logits.size // V
    t = np.ascontiguousarray(targets, dtype=np.int64).reshape(-1)
    loss = C.c_float(0)
    d = np.empty_like(logits)
    _check(lib().vref_cross_entropy(_p(logits), _p(t), C.c_int64(lanes), C.c_int64(V),
                                    C.byref(loss), _p(d)))
    return np.float32(loss.value), d


def embedding(table, ids, g, dtable=None):
    table = _f(table)
    V, D = table.shape
    ids = np.ascontiguousarray(ids, dtype=np.int64).reshape(-1)
    g = _f(g).reshape(ids.size, D)
    out = np.empty((ids.size, D), dtype=np.float32)
    dt = np.zeros_like(table) if dtable is None else _f(dtable).copy()
    _check(lib().vref_embedding(_p(table), _p(ids), C.c_int64(ids.size), C.c_int64(V),
                                C.c_int64(D), _p(g), _p(out), _p(dt)))
    return out, dt


def rope_tables(T, Dh, theta):
    c = np.empty((T, Dh), dtype=np.float32)
    s = np.empty((T, Dh), dtype=np.float32)
    _check(lib().vref_rope_tables(C.c_int64(T), C.c_int64(Dh), C.c_float(theta), _p(c), _p(s)))
    return c, s


def rope(x, g, theta):
    x, g = _f(x), _f(g)
    T, Dh = x.shape[-2], x.shape[-1]
    lanes = x.size // (T * Dh)
    y, dx = np.empty_like(x), np.empty_like(x)
    _check(lib().vref_rope(_p(x), _p(g), C.c_int64(lanes), C.c_int64(T), C.c_int64(Dh),
                           C.c_float(theta), _p(y), _p(dx)))
    return y, dx


def matmul_nt(a, b, g):
    a, b, g = _f(a), _f(b), _f(g)
    M, K = a.shape
    N = b.shape[0]
    y = np.empty((M, N), np.float32)
    da, db = np.empty_like(a), np.empty_like(b)
    _check(lib().vref_matmul_nt(_p(a), _p(b), _p(g), C.c_int64(M), C.c_int64(N), C.c_int64(K),
                                _p(y), _p(da), _p(db)))
    return y, da, db


def matmul(a, b, g):
    a, b, g = _f(a), _f(b), _f(g)
    M, K = a.shape
    N = b.shape[1]
    y = np.empty((M, N), np.float32)
    da, db = np.empty_like(a), np.empty_like(b)
    _check(lib().vref_matmul(_p(a), _p(b), _p(g), C.c_int64(M), C.c_int64(N), C.c_int64(K),
                             _p(y), _p(da), _p(db)))
    return y, da, db


def gemm_nt(a, b):
    a, b = _f(a), _f(b)
    M, K = a.shape
    N = b.shape[0]
    y = np.empty((M, N), np.float32)
    _check(lib().vref_gemm_nt(_p(a), _p(b), C.c_int64(M), C.c_int64(N), C.c_int64(K), _p(y)))
    return y


def attention(q, k, v, g):
    q, k, v, g = _f(q), _f(k), _f(v), _f(g)
    B, H, T, Dh = q.shape
    Hk = k.shape[1]
    o, dq = np.empty_like(q), np.empty_like(q)
    dk, dv = np.empty_like(k), np.empty_like(v)
    _check(lib().vref_attention(_p(q), _p(k), _p(v), _p(g), C.c_int64(B), C.c_int64(H),
                                C.c_int64(Hk), C.c_int64(T), C.c_int64(Dh), _p(o), _p(dq), _p(dk),
                                _p(dv)))
    return o, dq, dk, dv


def clip(grads: list, max_norm: float):
    sizes = np.array([g.size for g in grads], dtype=np.int64)
    flat = np.concatenate([_f(g).ravel() for g in grads]) if grads else np.zeros(0, np.float32)
    norm = C.c_float(0)
    _check(lib().vref_clip(_p(flat), _p(sizes), C.c_int64(len(grads)), C.c_float(max_norm),
                           C.byref(norm)))
    out, at = [], 0
    for g in grads:
        out.append(flat[at:at + g.size].reshape(g.shape))
        at += g.size
    return np.float32(norm.value), out


def adamw(value, grads_seq, lr, beta1, beta2, eps, wd):
    value = _f(value).copy()
    grads_seq = _f(grads_seq)
    steps = grads_seq.shape[0]
    cfg = VrefAdamConfig(lr, beta1, beta2, eps, wd)
    _check(lib().vref_adamw(_p(value), _p(grads_seq), C.c_int64(value.size), C.c_int64(steps),
                            cfg, None, None))
    return value


def model_config(c) -> VrefModelConfig:
    return VrefModelConfig(c.vocab, c.hidden, c.intermediate, c.layers, c.heads, c.kv_heads,
                           c.head_dim, c.eps, c.theta)


def train_steps(c, params, ids, targets, max_norm, adam, steps=1):
    """Runs `steps` reference training steps on one batch. Returns (weights list, losses, norms,
    pre-clip grads of the last step)."""
    cfg = model_config(c)
    flat = np.concatenate([_f(p).ravel() for p in params])
    assert flat.size == lib().vref_param_count(C.byref(cfg))
    ids = np.ascontiguousarray(ids, dtype=np.int64)
    targets = np.ascontiguousarray(targets, dtype=np.int64)
    B, T = ids.shape
    losses = np.zeros(steps, np.float32)
    norms = np.zeros(steps, np.float32)
    grads = np.zeros_like(flat)
    a = VrefAdamConfig(adam.learning_rate, adam.beta1, adam.beta2, adam.eps, adam.weight_decay)
    _check(lib().vref_train_step(C.byref(cfg), _p(flat), _p(ids), _p(targets), C.c_int64(B),
                                 C.c_int64(T), C.c_float(max_norm), a, C.c_int64(steps),
                                 _p(losses), _p(norms), _p(grads)))

    def split(v):
        out, at = [], 0
        for p in params:
            out.append(v[at:at + p.size].reshape(p.shape))
            at += p.size
        return out
    return split(flat), losses, norms, split(grads)


def read_safetensors(path):
    """Every tensor of a safetensors file as the reference's reader returns it (widened to fp32),
    in header order: [(name, array)] (src/libs/io/Safetensors.cpp:106-257)."""
    L = lib()
    fn = L.vref_read_safetensors
    fn.restype = C.c_int64
    fn.argtypes = [C.c_char_p, C.c_int64, C.c_char_p, C.c_int64, C.POINTER(C.c_int64),
                   C.POINTER(C.c_int64), C.c_void_p, C.c_int64]
    name = C.create_string_buffer(512)
    rank = C.c_int64(0)
    dims = (C.c_int64 * 8)()
    count = fn(str(path).encode(), -1, name, 512, C.byref(rank), dims, None, 0)
    if count < 0:
        raise RuntimeError(L.vref_last_error().decode())
    out = []
    for i in range(count):
        fn(str(path).encode(), i, name, 512, C.byref(rank), dims, None, 0)
        shape = tuple(dims[j] for j in range(rank.value))
        vals = np.empty(int(np.prod(shape)) if shape else 1, np.float32)
        rc = fn(str(path).encode(), i, name, 512, C.byref(rank), dims, vals.ctypes.data, vals.size)
        if rc < 0:
            raise RuntimeError(L.vref_last_error().decode())
        out.append((name.value.decode(), vals.reshape(shape)))
    return out


class RefCorpus:
    """The reference's data::Corpus (src/libs/data/Corpus.cpp), compiled from its sources."""

    def __init__(self, ids, validation_fraction, seed):
        L = lib()
        L.vref_corpus_create.restype = C.c_void_p
        L.vref_corpus_create.argtypes = [I64P, C.c_int64, C.c_double, C.c_uint64]
        L.vref_corpus_next_batch.argtypes = [C.c_void_p, C.c_int64, C.c_int64, C.c_int, I64P, I64P]
        L.vref_corpus_boundary.restype = C.c_int64
        L.vref_corpus_boundary.argtypes = [C.c_void_p]
        L.vref_corpus_destroy.argtypes = [C.c_void_p]
        self.L = L
        ids = np.ascontiguousarray(ids, dtype=np.int64)
        self.h = L.vref_corpus_create(ids, ids.size, validation_fraction, seed)
        if not self.h:
            raise ValueError(L.vref_last_error().decode())

    @property
    def boundary(self):
        return self.L.vref_corpus_boundary(self.h)

    def next_batch(self, batch, length, split="train"):
        inputs = np.empty(batch * length, np.int64)
        targets = np.empty(batch * length, np.int64)
        rc = self.L.vref_corpus_next_batch(self.h, batch, length, 1 if split == "validation" else 0,
                                           inputs, targets)
        if rc != 0:
            raise ValueError(self.L.vref_last_error().decode())
        return inputs.reshape(batch, length), targets.reshape(batch, length)

    def __del__(self):
        if getattr(self, "h", None):
            self.L.vref_corpus_destroy(self.h)
            self.h = None
