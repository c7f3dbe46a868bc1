"""ctypes binding of include/veda_train.h (libveda.so) and a thin Python handle around it, used
by the tests and bench.py. The training step itself runs in the C++ library."""
from __future__ import annotations

import ctypes as C

import numpy as np

_p, _i, _i64, _f, _sz, _u64 = C.c_void_p, C.c_int, C.c_int64, C.c_float, C.c_size_t, C.c_uint64


class ModelConfig(C.Structure):
    _fields_ = [("vocab", _i64), ("hidden", _i64), ("intermediate", _i64), ("layers", _i64),
                ("heads", _i64), ("kv_heads", _i64), ("head_dim", _i64), ("eps", _f),
                ("theta", _f)]


class OptimConfig(C.Structure):
    _fields_ = [("lr", _f), ("beta1", _f), ("beta2", _f), ("eps", _f), ("weight_decay", _f),
                ("max_norm", _f)]


SIGNATURES = {
    "veda_train_last_error": (C.c_char_p, []),
    "veda_train_set_stream": (_i, [_p]),
    "veda_trainer_create": (_i, [C.POINTER(ModelConfig), C.POINTER(OptimConfig), _i, _i64, _i64,
                                 _u64, C.POINTER(_p)]),
    "veda_trainer_destroy": (_i, [_p]),
    "veda_trainer_param_count": (_i64, [_p]),
    "veda_trainer_set_params": (_i, [_p, _p]),
    "veda_trainer_get_params": (_i, [_p, _p]),
    "veda_trainer_get_grads": (_i, [_p, _p]),
    "veda_nccl_unique_id": (_i, [_p]),
    "veda_trainer_init_dp": (_i, [_p, _p, _i, _i, _sz]),
    "veda_trainer_init_dp_sharded": (_i, [_p, _p, _i, _i, _sz]),
    "veda_trainer_sync": (_i, [_p]),
    "veda_trainer_generate": (_i, [_p, _p, _i64, _i64, _p, _i64, _i, _p, _p, _p, _p]),
    "veda_trainer_last_logits": (_i, [_p, _p, _i64, _p]),
    "veda_trainer_set_step_graph": (_i, [_p, _i]),
    "veda_corpus_create": (_i, [_p, _i64, C.c_double, C.c_uint64, _p]),
    "veda_corpus_destroy": (_i, [_p]),
    "veda_corpus_boundary": (_i64, [_p]),
    "veda_corpus_next_batch": (_i, [_p, _i64, _i64, _i, _p, _p]),
    "veda_trainer_save_checkpoint": (_i, [_p, C.c_char_p]),
    "veda_trainer_load_checkpoint": (_i, [_p, C.c_char_p]),
    "veda_safetensors_write": (_i, [C.c_char_p, _i64, _p, _p, _p, _p, _p, _i64, _p, _p]),
    "veda_trainer_step_host": (_i, [_p, _p, _p, _p, _p]),
    "veda_trainer_step_device": (_i, [_p, _p, _p]),
    "veda_trainer_last_stats": (_i, [_p, _p, _p]),
    "veda_trainer_set_comm_timeout": (_i, [_p, C.c_double]),
    "veda_trainer_abort_comm": (_i, [_p]),
    "veda_trainer_set_skip_nonfinite": (_i, [_p, _i]),
    "veda_trainer_set_recompute_attention": (_i, [_p, _i]),
    "veda_trainer_step_skipped": (_i, [_p, _p]),
    "veda_profile_enable": (_i, [_i]),
    "veda_profile_collect": (_i, [_p, _p, _p, _p, _p, _i]),
}


def load(path):
    L = C.CDLL(str(path))
    for name, (res, args) in SIGNATURES.items():
        fn = getattr(L, name)
        fn.restype = res
        fn.argtypes = args
    return L


class TrainError(RuntimeError):
    pass


def _check(L, rc):
    if rc < 0:
        msg = L.veda_train_last_error().decode(errors="replace")
        if rc == -5:
            raise IndexError(msg)
        if rc == -1:
            raise ValueError(msg)
        raise TrainError(f"[{rc}] {msg}")
    return rc


class Trainer:
    """A veda::train::Trainer on the current CUDA device (C++ object behind the C ABI)."""

    def __init__(self, cfg, lr=1e-3, betas=(0.9, 0.95), eps=1e-8, weight_decay=0.1, max_norm=1.0,
                 dtype=1, batch=1, seq_len=1, seed=0, stream=None):
        from . import host_lib
        self.L = host_lib()
        if stream is not None:
            _check(self.L, self.L.veda_train_set_stream(stream))
        m = ModelConfig(cfg.vocab, cfg.hidden, cfg.intermediate, cfg.layers, cfg.heads,
                        cfg.kv_heads, cfg.head_dim, cfg.eps, cfg.theta)
        o = OptimConfig(lr, betas[0], betas[1], eps, weight_decay, max_norm)
        h = _p()
        _check(self.L, self.L.veda_trainer_create(C.byref(m), C.byref(o), dtype, batch, seq_len,
                                                  seed, C.byref(h)))
        self.h = h
        self.batch, self.seq_len = batch, seq_len
        self.n = int(self.L.veda_trainer_param_count(h))
        self.cfg_vocab = int(cfg.vocab)

    def close(self):
        if self.h:
            _check(self.L, self.L.veda_trainer_destroy(self.h))
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def set_params(self, flat: np.ndarray):
        flat = np.ascontiguousarray(flat, dtype=np.float32)
        assert flat.size == self.n
        _check(self.L, self.L.veda_trainer_set_params(self.h, flat.ctypes.data))

    def get_params(self) -> np.ndarray:
        out = np.empty(self.n, np.float32)
        _check(self.L, self.L.veda_trainer_get_params(self.h, out.ctypes.data))
        return out

    def get_grads(self) -> np.ndarray:
        out = np.empty(self.n, np.float32)
        _check(self.L, self.L.veda_trainer_get_grads(self.h, out.ctypes.data))
        return out

    def init_dp(self, unique_id: bytes, rank: int, world: int, bucket_bytes=25 << 20,
                sharded=False):
        """NCCL data parallelism; sharded=True splits the optimizer state across the ranks
        (get_params / get_grads then have to be called on every rank together)."""
        buf = C.create_string_buffer(bytes(unique_id), 128)
        fn = self.L.veda_trainer_init_dp_sharded if sharded else self.L.veda_trainer_init_dp
        _check(self.L, fn(self.h, buf, rank, world, bucket_bytes))

    def save(self, directory: str):
        """dir/model.safetensors + dir/optimizer.safetensors (collective when sharded)."""
        _check(self.L, self.L.veda_trainer_save_checkpoint(self.h, str(directory).encode()))

    def load(self, directory: str):
        _check(self.L, self.L.veda_trainer_load_checkpoint(self.h, str(directory).encode()))

    def set_step_graph(self, on: bool):
        _check(self.L, self.L.veda_trainer_set_step_graph(self.h, 1 if on else 0))

    def generate(self, prompt, max_new_tokens, stop_tokens=(), cached=True):
        """Greedy generation: (tokens, stopped_on_token, forward_passes)."""
        p = np.ascontiguousarray(prompt, dtype=np.int32)
        st = np.ascontiguousarray(list(stop_tokens) or [0], dtype=np.int32)
        out = np.empty(max(1, max_new_tokens), np.int32)
        cnt, stopped, passes = C.c_int64(0), C.c_int(0), C.c_int64(0)
        _check(self.L, self.L.veda_trainer_generate(self.h, p.ctypes.data if p.size else None, p.size,
                                                    max_new_tokens, st.ctypes.data, len(stop_tokens),
                                                    1 if cached else 0, out.ctypes.data, C.byref(cnt),
                                                    C.byref(stopped), C.byref(passes)))
        return out[:cnt.value].tolist(), bool(stopped.value), passes.value

    def last_logits(self, ids):
        ids = np.ascontiguousarray(ids, dtype=np.int32)
        out = np.empty(self.cfg_vocab, np.float32)
        _check(self.L, self.L.veda_trainer_last_logits(self.h, ids.ctypes.data, ids.size, out.ctypes.data))
        return out

    def sync(self):
        """The current stream waits for the trainer's queued communication."""
        _check(self.L, self.L.veda_trainer_sync(self.h))

    def step_host(self, ids: np.ndarray, targets: np.ndarray):
        ids = np.ascontiguousarray(ids, dtype=np.int64)
        targets = np.ascontiguousarray(targets, dtype=np.int64)
        loss, norm = C.c_float(0), C.c_float(0)
        _check(self.L, self.L.veda_trainer_step_host(self.h, ids.ctypes.data, targets.ctypes.data,
                                                     C.byref(loss), C.byref(norm)))
        return float(loss.value), float(norm.value)

    def step_device(self, ids_ptr: int, targets_ptr: int):
        _check(self.L, self.L.veda_trainer_step_device(self.h, ids_ptr, targets_ptr))

    def last_stats(self):
        loss, norm = C.c_float(0), C.c_float(0)
        _check(self.L, self.L.veda_trainer_last_stats(self.h, C.byref(loss), C.byref(norm)))
        return float(loss.value), float(norm.value)

    def set_comm_timeout(self, seconds: float):
        _check(self.L, self.L.veda_trainer_set_comm_timeout(self.h, float(seconds)))

    def abort_comm(self):
        _check(self.L, self.L.veda_trainer_abort_comm(self.h))

    def set_skip_nonfinite(self, on: bool):
        _check(self.L, self.L.veda_trainer_set_skip_nonfinite(self.h, 1 if on else 0))

    def set_recompute_attention(self, on: bool):
        _check(self.L, self.L.veda_trainer_set_recompute_attention(self.h, 1 if on else 0))

    def step_skipped(self) -> bool:
        out = C.c_int(0)
        _check(self.L, self.L.veda_trainer_step_skipped(self.h, C.byref(out)))
        return bool(out.value)


def nccl_unique_id() -> bytes:
    from . import host_lib
    L = host_lib()
    buf = C.create_string_buffer(128)
    _check(L, L.veda_nccl_unique_id(buf))
    return buf.raw


def profile_enable(on: bool):
    from . import host_lib
    host_lib().veda_profile_enable(1 if on else 0)


def profile_collect():
    """{class: (ms, flops, bytes, launches)} since the last collect (synchronises)."""
    from . import host_lib
    L = host_lib()
    cap = 64
    names = (C.c_char * 32 * cap)()
    ms = (C.c_double * cap)()
    fl = (C.c_double * cap)()
    by = (C.c_double * cap)()
    la = (C.c_uint64 * cap)()
    n = _check(L, L.veda_profile_collect(names, ms, fl, by, la, cap))
    return {names[i].value.decode(): (ms[i], fl[i], by[i], int(la[i])) for i in range(min(n, cap))}


def write_safetensors(path, tensors, metadata=None):
    """Writes host arrays with the library's safetensors writer. tensors: list of (name, dtype
    name, numpy array holding the raw little-endian values)."""
    from . import host_lib
    L = host_lib()
    names = [n.encode() for n, _, _ in tensors]
    dtypes = [d.encode() for _, d, _ in tensors]
    arrays = [np.ascontiguousarray(a) for _, _, a in tensors]
    ranks = np.array([a.ndim for a in arrays], np.int64)
    dims = np.array([x for a in arrays for x in a.shape], np.int64)
    meta = list((metadata or {}).items())
    strs = lambda xs: (C.c_char_p * max(1, len(xs)))(*xs)  # noqa: E731
    ptrs = (C.c_void_p * max(1, len(arrays)))(*[a.ctypes.data for a in arrays])
    _check(L, L.veda_safetensors_write(str(path).encode(), len(arrays), strs(names), strs(dtypes),
                                       ranks.ctypes.data, dims.ctypes.data if dims.size else None,
                                       ptrs, len(meta), strs([k.encode() for k, _ in meta]),
                                       strs([v.encode() for _, v in meta])))


class Corpus:
    """data::Corpus on the current CUDA device; next_batch fills device int64 buffers."""

    def __init__(self, ids, validation_fraction, seed):
        from . import host_lib
        self.L = host_lib()
        ids = np.ascontiguousarray(ids, dtype=np.int64)
        h = C.c_void_p()
        _check(self.L, self.L.veda_corpus_create(ids.ctypes.data if ids.size else None, ids.size,
                                                 float(validation_fraction), int(seed),
                                                 C.byref(h)))
        self.h = h

    @property
    def boundary(self):
        return self.L.veda_corpus_boundary(self.h)

    def next_batch(self, batch, length, split, inputs_ptr, targets_ptr):
        _check(self.L, self.L.veda_corpus_next_batch(self.h, batch, length,
                                                     1 if split == "validation" else 0,
                                                     inputs_ptr, targets_ptr))

    def close(self):
        if self.h:
            self.L.veda_corpus_destroy(self.h)
            self.h = None
