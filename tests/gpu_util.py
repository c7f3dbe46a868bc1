"""Helpers for the GPU parity tests: numpy <-> torch device buffers (torch is only the allocator
and stream here) and calls through the C ABI of libveda_cuda.so."""
import numpy as np

import veda_b200 as V
from oracle import veda_oracle as O


def torch():
    import torch as t
    return t


def dev(a, dtype=V.F32):
    """Device copy of a numpy array; bf16 rounds to nearest even."""
    t = torch()
    a = np.ascontiguousarray(a)
    if a.dtype == np.int64:
        return t.from_numpy(a).cuda()
    if dtype == V.BF16:
        return t.from_numpy(np.ascontiguousarray(a, dtype=np.float32)).cuda().to(t.bfloat16)
    return t.from_numpy(np.ascontiguousarray(a, dtype=np.float32)).cuda()


def host(x):
    t = torch()
    if x.dtype == t.bfloat16:
        x = x.float()
    return x.detach().cpu().numpy()


def empty(shape, dtype=V.F32):
    t = torch()
    return t.empty(shape, dtype=t.bfloat16 if dtype == V.BF16 else t.float32, device="cuda")


def zeros(shape, dtype=V.F32):
    t = torch()
    return t.zeros(shape, dtype=t.bfloat16 if dtype == V.BF16 else t.float32, device="cuda")


def ptr(x):
    return None if x is None else x.data_ptr()


def stream():
    return torch().cuda.current_stream().cuda_stream


def workspace(nbytes):
    t = torch()
    return t.empty(max(int(nbytes), 16), dtype=t.uint8, device="cuda")


def call(name, *args):
    rc = getattr(V.lib(), name)(*args)
    V.check(rc)
    return rc


def sync():
    torch().cuda.synchronize()
    status = V.lib().veda_kernel_status(1)
    assert status == 0, f"device status word {status}: {V.lib().veda_last_error().decode()}"


def rel(a, b):
    return O.max_abs_rel(a, b)


def bf(a):
    """fp32 array holding the bf16-rounded values (what a bf16 device copy holds)."""
    return O.bf16_round(np.asarray(a, dtype=np.float32))
