"""veda_rmsnorm_bwd_noalloc: the RMSNorm backward for callers that cannot allocate device memory
(a workspace costs a cudaMalloc, which synchronises the device and can fail under an engine that
reserves its memory up front; a caller using only the C ABI may have no device allocator). It
takes its scratch from a fixed array inside the library. This file is collected last on purpose,
and its test must pass both alone in a fresh process and after every other test."""
import numpy as np
import pytest

import veda_b200 as V
from oracle import veda_oracle as O
from tests.gpu_util import bf, dev, empty, host, ptr, rel, stream, sync, workspace

pytestmark = pytest.mark.gpu
TOL = {V.F32: 1e-4, V.BF16: 2e-2}


@pytest.fixture(autouse=True)
def _gpu(cuda):
    yield


@pytest.mark.parametrize("dtype,rows,n", [(V.BF16, 8192, 1024), (V.F32, 300, 2048)])
def test_noalloc_matches_workspace_entry_point_twice(dtype, rows, n):
    lib = V.lib()
    r = np.random.default_rng(rows + n)
    x = r.standard_normal((rows, n)).astype(np.float32)
    gam = (1 + 0.1 * r.standard_normal(n)).astype(np.float32)
    g = r.standard_normal((rows, n)).astype(np.float32)
    res = r.standard_normal((rows, n)).astype(np.float32)
    if dtype == V.BF16:
        x, gam, g, res = bf(x), bf(gam), bf(g), bf(res)
    xd, gd, gyd, rd = dev(x, dtype), dev(gam, dtype), dev(g, dtype), dev(res, dtype)

    # the existing entry point with a caller-allocated workspace
    dx_ref = empty((rows, n), dtype)
    dg_ref = dev(np.zeros(n, np.float32))
    ws = workspace(lib.veda_rmsnorm_bwd_workspace(rows, n))
    V.check(lib.veda_rmsnorm_bwd(ptr(xd), n, ptr(gd), ptr(gyd), n, ptr(rd), n, ptr(dx_ref), n,
                                 ptr(dg_ref), ptr(ws), ws.numel(), rows, n, 1e-6, dtype, stream()))
    sync()
    want_dx, want_dg = host(dx_ref), host(dg_ref)

    # the allocation-free entry point, two calls in a row (the shared scratch is reused)
    for _ in range(2):
        dx = empty((rows, n), dtype)
        dg = dev(np.zeros(n, np.float32))
        V.check(lib.veda_rmsnorm_bwd_noalloc(ptr(xd), n, ptr(gd), ptr(gyd), n, ptr(rd), n, ptr(dx),
                                             n, ptr(dg), rows, n, 1e-6, dtype, stream()))
        sync()
        assert rel(host(dx), want_dx) <= TOL[dtype]
        assert rel(host(dg), want_dg) <= 1e-4
    # and both agree with the oracle
    dx_o, dg_o = O.rms_norm_gamma_backward(x, gam, g, 1e-6)
    assert rel(host(dx), dx_o + res) <= TOL[dtype]
    assert rel(host(dg), dg_o) <= (1e-4 if dtype == V.F32 else 1e-3)


def test_noalloc_rejects_rows_beyond_its_scratch():
    lib = V.lib()
    rows, n = 8192, 8192   # needs 2 x SMs x 8192 floats of scratch: above the fixed 4 MiB
    rc = lib.veda_rmsnorm_bwd_noalloc(None, n, None, None, n, None, n, None, n, 1, rows, n, 1e-6,
                                      V.BF16, stream())
    assert rc == V.ERR_INVALID_ARGUMENT
    assert "scratch" in lib.veda_last_error().decode()
