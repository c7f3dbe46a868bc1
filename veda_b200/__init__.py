"""veda_b200 — B200-native training backward path for Veda's autograd.

The product is two in-tree shared libraries:
  * libveda_cuda.so — hand-written sm_100a kernels behind the C ABI of include/veda_cuda.h;
  * libveda.so      — the C++23 host library (veda::core::Tensor on device memory,
                      veda::autograd, veda::optim, veda::train) behind include/veda/*.hpp,
                      with a C ABI for the trainer in include/veda_train.h.
This module only loads them (ctypes) for the tests and bench.py. There is no CPU fallback: if the
libraries are missing, loading fails loudly.
"""
from __future__ import annotations

import ctypes as C
from pathlib import Path

PKG = Path(__file__).resolve().parent
CUDA_LIB_PATH = PKG / "libveda_cuda.so"
HOST_LIB_PATH = PKG / "libveda.so"

F32, BF16 = 0, 1
OK = 0
ERR_INVALID_ARGUMENT, ERR_CUDA, ERR_TIMEOUT, ERR_UNSUPPORTED, ERR_OUT_OF_RANGE = -1, -2, -3, -4, -5

_p = C.c_void_p
_i64 = C.c_int64
_i = C.c_int
_f = C.c_float
_d = C.c_double
_sz = C.c_size_t
_u64 = C.c_uint64

# name -> (restype, argtypes), in the order of include/veda_cuda.h
SIGNATURES = {
    "veda_last_error": (C.c_char_p, []),
    "veda_device_info": (_i, [_p, _p, _p]),
    "veda_launch_count": (_u64, []),
    "veda_kernel_status": (_i, [_i]),
    "veda_wait_timeout_check": (_i, [C.c_longlong, _p]),
    "veda_set_reserved_sms": (_i, [_i]),
    "veda_gemm_nt": (_i, [_i64, _i64, _i64, _p, _i64, _p, _i64, _p, _i64, _i, _i, _f, _f, _p]),
    "veda_gemm_nn": (_i, [_i64, _i64, _i64, _p, _i64, _p, _i64, _p, _i64, _i, _i, _f, _f, _p]),
    "veda_gemm_tn": (_i, [_i64, _i64, _i64, _p, _i64, _p, _i64, _p, _i64, _i, _i, _f, _f, _p]),
    "veda_gemm_swiglu_fwd": (_i, [_i64, _i64, _i64, _p, _i64, _p, _i64, _p, _i64, _p, _i64, _p]),
    "veda_gemm_swiglu_bwd": (_i, [_i64, _i64, _i64, _p, _i64, _p, _i64, _p, _i64, _p, _i64, _p]),
    "veda_gemm_batched": (_i, [_i, _i64, _i64, _i64, _i64, _p, _i64, _i64, _p, _i64, _i64, _p,
                               _i64, _i64, _i, _i, _f, _f, _p]),
    "veda_rmsnorm_fwd": (_i, [_p, _i64, _p, _p, _i64, _i64, _i64, _f, _i, _p]),
    "veda_add_rmsnorm_fwd": (_i, [_p, _i64, _p, _i64, _p, _p, _i64, _p, _i64, _i64, _i64, _f, _i,
                                  _p]),
    "veda_rmsnorm_bwd": (_i, [_p, _i64, _p, _p, _i64, _p, _i64, _p, _i64, _p, _p, _sz, _i64,
                              _i64, _f, _i, _p]),
    "veda_rmsnorm_bwd_workspace": (_sz, [_i64, _i64]),
    "veda_rmsnorm_bwd_noalloc": (_i, [_p, _i64, _p, _p, _i64, _p, _i64, _p, _i64, _p, _i64, _i64,
                                      _f, _i, _p]),
    "veda_qknorm_rope_fwd": (_i, [_p, _i64, _p, _p, _p, _p, _i64, _i64, _i64, _i64, _i64, _f,
                                  _i, _p]),
    "veda_qknorm_rope_fwd_qk": (_i, [_p, _p, _i64, _p, _p, _p, _p, _p, _i64, _p, _i64, _i64, _i64,
                                     _i64, _i64, _i64, _f, _i, _p]),
    "veda_qknorm_rope_bwd": (_i, [_p, _i64, _p, _p, _p, _p, _i64, _p, _i64, _p, _p, _sz, _i64,
                                  _i64, _i64, _i64, _f, _i, _p]),
    "veda_qknorm_rope_bwd_workspace": (_sz, [_i64, _i64, _i64]),
    "veda_qknorm_rope_bwd_qk": (_i, [_p, _p, _i64, _p, _p, _p, _p, _p, _i64, _i, _f, _p, _i64,
                                     _p, _p, _i64, _p, _p, _p, _sz, _i64, _i64, _i64, _i64, _i64,
                                     _f, _i, _p]),
    "veda_qknorm_rope_bwd_qk_workspace": (_sz, [_i64, _i64, _i64, _i64]),
    "veda_rope": (_i, [_p, _p, _p, _p, _i64, _i64, _i64, _i, _i, _p]),
    "veda_swiglu_fwd": (_i, [_p, _i64, _p, _i64, _p, _i64, _i64, _i64, _i, _p]),
    "veda_swiglu_bwd": (_i, [_p, _i64, _p, _i64, _p, _i64, _p, _i64, _p, _i64, _i64, _i64, _i,
                             _p]),
    "veda_cross_entropy": (_i, [_p, _i64, _p, _p, _p, _i64, _i64, _i64, _f, _p, _i, _p]),
    "veda_mean_f64": (_i, [_p, _i64, _p, _p, _p]),
    "veda_embedding_fwd": (_i, [_p, _i64, _p, _i64, _i64, _p, _i64, _p, _i, _p]),
    "veda_embedding_bwd": (_i, [_p, _i64, _p, _i64, _i64, _i64, _p, _i, _p, _sz, _i, _p]),
    "veda_embedding_bwd_workspace": (_sz, [_i64]),
    "veda_embedding_sort": (_i, [_p, _i64, _i64, _p, _p]),
    "veda_embedding_apply_sorted": (_i, [_p, _i64, _p, _i64, _i64, _i64, _i64, _p, _i, _p]),
    "veda_sumsq": (_i, [_p, _i64, _p, _i, _p, _sz, _p]),
    "veda_sumsq_workspace": (_sz, [_i64]),
    "veda_clip_apply": (_i, [_p, _i64, _p, _f, _p]),
    "veda_adamw_step": (_i, [_p, _p, _p, _p, _p, _i64, _f, _f, _f, _f, _f, _d, _d, _p, _f, _f,
                             _i, _p]),
    "veda_adamw_step_dev": (_i, [_p, _p, _p, _p, _p, _i64, _f, _f, _f, _f, _f, _p, _p, _f, _f, _i, _p]),
    "veda_launch_count_add": (_i, [_i64]),
    "veda_binary": (_i, [_i, _p, _p, _p, _p, _p, _p, _i, _i, _p]),
    "veda_scale": (_i, [_p, _f, _p, _i64, _i, _p]),
    "veda_accumulate": (_i, [_p, _i, _p, _i, _i64, _p]),
    "veda_copy_strided": (_i, [_p, _i, _p, _i64, _p, _i, _p, _i, _p]),
    "veda_unbroadcast": (_i, [_p, _p, _p, _i, _p, _i, _p]),
    "veda_sum": (_i, [_p, _i64, _p, _i, _p]),
    "veda_fill": (_i, [_p, _f, _i64, _i, _p]),
    "veda_softmax_fwd": (_i, [_p, _p, _i64, _i64, _i, _p]),
    "veda_softmax_bwd": (_i, [_p, _p, _p, _i64, _i64, _i, _p]),
    "veda_silu_fwd": (_i, [_p, _p, _i64, _i, _p]),
    "veda_silu_bwd": (_i, [_p, _p, _p, _i64, _i, _p]),
    "veda_gelu_fwd": (_i, [_p, _p, _i64, _i, _p]),
    "veda_gelu_bwd": (_i, [_p, _p, _p, _i64, _i, _p]),
    "veda_argmax": (_i, [_p, _i64, _i64, _i64, _p, _p, _i, _p]),
    "veda_attention_decode": (_i, [_p, _p, _p, _i64, _i64, _i64, _i64, _i64, _f, _p, _i, _p]),
    "veda_attention_decode_at": (_i, [_p, _p, _p, _i64, _p, _i64, _i64, _i64, _f, _p, _i, _p]),
    "veda_decode_qkv_at": (_i, [_p, _p, _p, _p, _p, _p, _p, _p, _p, _i64, _i64, _i64, _i64, _f, _i,
                                _p]),
    "veda_decode_advance": (_i, [_p, _p]),
    "veda_gemv_nt": (_i, [_p, _p, _i64, _p, _i64, _i64, _i, _p]),
    "veda_gemv_swiglu": (_i, [_p, _p, _i64, _p, _i64, _i64, _i, _p]),
    "veda_gemv_rmsnorm": (_i, [_p, _p, _p, _f, _p, _p, _i64, _p, _i64, _i64, _i, _p]),
    "veda_gemv_rmsnorm_swiglu": (_i, [_p, _p, _p, _f, _p, _p, _i64, _p, _i64, _i64, _i, _p]),
    "veda_decode_attention_workspace": (_i64, [_i64, _i64, _i64]),
    "veda_gemv_argmax_workspace": (_i64, [_i64]),
    "veda_gemv_rmsnorm_argmax": (_i, [_p, _p, _p, _f, _p, _p, _i64, _p, _i64, _i64, _p, _p, _p, _i64, _i,
                                      _p]),
    "veda_decode_attention_at": (_i, [_p, _p, _p, _p, _p, _p, _p, _p, _i64, _i64, _i64, _i64, _i64, _f, _f,
                                      _p, _p, _i64, _i, _p]),
    "veda_randn": (_i, [_p, _i64, _f, _u64, _i, _p]),
    "veda_f32_to_bf16": (_i, [_p, _p, _i64, _p]),
    "veda_corpus_gather": (_i, [_p, _i64, _i64, C.c_uint64, _i64, _i64, _p, _p, _p]),
    "veda_attention_fwd": (_i, [_p, _i64, _p, _i64, _p, _i64, _p, _i64, _p, _i64, _i64, _i64,
                                _i64, _i64, _f, _i, _i, _p]),
    "veda_attention_bwd": (_i, [_p, _i64, _p, _i64, _p, _i64, _p, _i64, _p, _i64, _p, _p, _i64,
                                _p, _i64, _p, _i64, _p, _sz, _i64, _i64, _i64, _i64, _i64, _f,
                                _i, _i, _p]),
    "veda_attention_bwd_workspace": (_sz, [_i64, _i64, _i64, _i64, _i64, _i]),
    "veda_attention_bwd_dq_f32": (_i, [_p, _i64, _p, _i64, _p, _i64, _p, _i64, _p, _i64, _p, _p,
                                       _i64, _p, _i64, _p, _sz, _i64, _i64, _i64, _i64, _i64, _f,
                                       _i, _i, _p]),
    "veda_attention_bwd_dq_offset": (_sz, [_i64, _i64, _i64]),
    "veda_attention_set_deterministic": (_i, [_i]),
    "veda_log_softmax_fwd": (_i, [_p, _p, _i64, _i64, _i, _p]),
}

_cuda = None
_host = None


class VedaError(RuntimeError):
    def __init__(self, code, message):
        super().__init__(f"[{code}] {message}")
        self.code = code


def lib():
    """libveda_cuda.so with every entry point of include/veda_cuda.h typed."""
    global _cuda
    if _cuda is None:
        if not CUDA_LIB_PATH.exists():
            raise FileNotFoundError(
                f"{CUDA_LIB_PATH} is not built; run python -m veda_b200.build "
                "(there is no CPU fallback)")
        L = C.CDLL(str(CUDA_LIB_PATH))
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _cuda = L
    return _cuda


def check(rc: int):
    """Raise VedaError carrying veda_last_error() for a non-zero status."""
    if rc != OK:
        raise VedaError(rc, lib().veda_last_error().decode(errors="replace"))
    return rc


def host_lib():
    """libveda.so (the C++ host library) with the trainer C ABI of include/veda_train.h."""
    global _host
    if _host is None:
        lib()
        if not HOST_LIB_PATH.exists():
            raise FileNotFoundError(f"{HOST_LIB_PATH} is not built; run python -m veda_b200.build")
        from . import train_abi
        _host = train_abi.load(HOST_LIB_PATH)
    return _host
