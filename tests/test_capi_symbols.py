"""The C-ABI libraries load on a machine without a GPU and export every symbol the headers in
include/ declare (no kernel is launched here)."""
import re
from pathlib import Path

import pytest

import veda_b200 as V

ROOT = Path(__file__).resolve().parent.parent


def declared(header: Path):
    text = header.read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(veda_[a-z0-9_]+)\s*\(", text)))


def test_cuda_header_symbols_are_exported():
    names = declared(ROOT / "include" / "veda_cuda.h")
    assert len(names) > 30
    lib = V.lib()
    missing = [n for n in names if not hasattr(lib, n)]
    assert not missing, f"declared but not exported: {missing}"
    assert set(names) == set(V.SIGNATURES), "ctypes signature table out of sync with the header"


def test_host_header_symbols_are_exported():
    header = ROOT / "include" / "veda_train.h"
    if not header.exists():
        pytest.skip("no trainer header yet")
    names = declared(header)
    lib = V.host_lib()
    missing = [n for n in names if not hasattr(lib, n)]
    assert not missing, f"declared but not exported: {missing}"


def test_library_is_sm100a_only():
    # the fat binary carries sm_100a code only (no PTX for other targets): the build flags say so
    from veda_b200 import build
    assert build.ARCH == ["-gencode", "arch=compute_100a,code=sm_100a"]


def test_argument_errors_without_a_gpu():
    # argument validation runs on the host before any launch, so it works without a device
    lib = V.lib()
    rc = lib.veda_rmsnorm_fwd(None, 4, None, None, 4, 2, 8, 1e-6, 0, None)
    assert rc == V.ERR_INVALID_ARGUMENT
    assert "leading dimension" in lib.veda_last_error().decode() or "shape" in lib.veda_last_error().decode()
    rc = lib.veda_adamw_step(None, None, None, None, None, 4, 1e-3, 1.0, 0.9, 1e-8, 0.0, 1.0, 1.0,
                             None, 1.0, 1.0, 0, None)
    assert rc == V.ERR_INVALID_ARGUMENT and "betas" in lib.veda_last_error().decode()
    rc = lib.veda_attention_fwd(None, 64, None, 32, None, 32, None, 64, None, 1, 4, 3, 2, 16,
                                0.25, 1, 0, None)
    assert rc == V.ERR_INVALID_ARGUMENT and "multiple" in lib.veda_last_error().decode()


def test_decode_workspace_sizes_and_argument_errors_without_a_gpu():
    # the decode step's workspace sizes are host arithmetic: one 256-position slice (no merge) up to
    # 256 cache rows, 128-position slices beyond, at most 64 slices; counters padded to 256 bytes
    lib = V.lib()
    per_slice = lambda heads, kv: kv * (heads // kv) * 130 * 4
    assert lib.veda_decode_attention_workspace(16, 8, 200) == 256 + 1 * per_slice(16, 8)
    assert lib.veda_decode_attention_workspace(16, 8, 256) == 256 + 1 * per_slice(16, 8)
    assert lib.veda_decode_attention_workspace(16, 8, 257) == 256 + 3 * per_slice(16, 8)
    assert lib.veda_decode_attention_workspace(32, 4, 1000) == 256 + 8 * per_slice(32, 4)
    big = lib.veda_decode_attention_workspace(16, 8, 100000)
    assert big <= 256 + 64 * per_slice(16, 8)
    assert lib.veda_decode_attention_workspace(16, 6, 100) == -1      # heads not a multiple
    assert lib.veda_decode_attention_workspace(16, 8, 0) == -1
    # the GEMV entries check their arguments before any launch
    rc = lib.veda_gemv_nt(None, None, 8, None, 4, 8, 1, None)
    assert rc == V.ERR_INVALID_ARGUMENT and "null" in lib.veda_last_error().decode()
    # a 16000-element bf16 row fits the staged 48 KB alone, not together with its gain
    rc = lib.veda_gemv_rmsnorm(8, None, 8, 1e-6, None, 8, 16000, 8, 4, 16000, 1, None)
    assert rc == V.ERR_INVALID_ARGUMENT and "gain exceed" in lib.veda_last_error().decode()
