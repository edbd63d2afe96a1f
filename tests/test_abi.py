"""CPU tests of the C ABI boundary: the library loads, exports every function
that include/continuum_attention_b200.h declares, and rejects bad arguments
before touching a GPU (the checks return status codes and messages, like the
reference binding's TORCH_CHECKs, cuda/continuum_attention.py:460-605).
"""
import ctypes
import os
import re
import subprocess

import pytest

from continuum_attention_b200 import _native

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "continuum_attention_b200.h")


def _declared_functions():
    text = open(HEADER).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"^\s*(?:const\s+)?[A-Za-z_][A-Za-z0-9_]*\s*\**\s*(ca_[a-z0-9_]+)\s*\(",
                                 text, flags=re.M)))


def test_header_declares_the_abi():
    names = _declared_functions()
    assert {"ca_forward", "ca_backward", "ca_backward_workspace_size", "ca_abi_version",
            "ca_last_error", "ca_row_stats_floats", "ca_device_status"} <= set(names)


def test_library_exports_every_declared_symbol():
    lib = _native.lib()
    for name in _declared_functions():
        assert hasattr(lib, name), f"{name} missing from {_native.LIB_PATH}"
        assert name in _native.SIGNATURES, f"{name} has no ctypes signature"
    out = subprocess.run(["nm", "-D", "--defined-only", _native.LIB_PATH], capture_output=True, text=True)
    if out.returncode == 0:
        exported = set(re.findall(r"\bT (ca_[a-z0-9_]+)\b", out.stdout))
        assert set(_declared_functions()) <= exported


def test_abi_version_matches_header():
    m = re.search(r"#define\s+CA_ABI_VERSION\s+(\d+)", open(HEADER).read())
    assert _native.lib().ca_abi_version() == int(m.group(1))
    assert _native.lib().ca_row_stats_floats() == 2


def test_workspace_size_formula():
    lib = _native.lib()
    assert lib.ca_backward_workspace_size(0, 1, 1, 1, 1) == 0
    B, H, T, D = 2, 16, 2048, 64
    n = lib.ca_backward_workspace_size(B, H, T, D, 1)
    rows = B * H * T
    assert n >= rows * 4 + rows * D * 4 + B * H * (T // 64) * 4
    assert n % 256 == 0
    # grows with T
    assert lib.ca_backward_workspace_size(B, H, 4096, D, 1) > n


def _status_and_msg(st):
    return st, _native.lib().ca_last_error().decode()


def test_argument_checks_need_no_gpu():
    lib = _native.lib()
    st, msg = _status_and_msg(lib.ca_forward(None, None, None, None, None, None, None, 1, 2, -3, 64, 1, 0, None))
    assert st == 1 and "negative shape" in msg
    st, msg = _status_and_msg(lib.ca_forward(None, None, None, None, None, None, None, 1, 2, 8, 64, 7, 0, None))
    assert st == 1 and "dtype" in msg
    st, msg = _status_and_msg(lib.ca_forward(None, None, None, None, None, None, None, 1, 2, 8, 256, 1, 0, None))
    assert st == 2 and "D=256" in msg
    st, msg = _status_and_msg(lib.ca_forward(None, None, None, None, None, None, None, 1, 2, 8, 64, 1, 0, None))
    assert st == 1 and "null" in msg
    st, msg = _status_and_msg(lib.ca_forward(None, None, None, None, None, None, None, 1, 2, 8, 64, 1, 9, None))
    assert st == 1 and "impl" in msg
    # a zero-size problem is a successful no-op
    st, msg = _status_and_msg(lib.ca_forward(None, None, None, None, None, None, None, 0, 2, 8, 64, 1, 0, None))
    assert st == 0 and msg == ""
    fake = ctypes.c_void_p(256)
    st, msg = _status_and_msg(lib.ca_backward(fake, fake, fake, fake, None, fake, fake, fake, fake, fake, fake,
                                              None, fake, 16, 1, 2, 8, 64, 1, 0, None))
    assert st == 4 and "workspace" in msg


def test_python_wrapper_rejects_cpu_tensors_without_fallback():
    import torch
    import continuum_attention_b200 as ca
    q = torch.randn(1, 2, 4, 8)
    with pytest.raises(RuntimeError, match="CUDA"):
        ca.continuum_attention(q, q, q, torch.zeros(2))
    with pytest.raises(ValueError, match="must share dtype"):
        ca.continuum_attention(q, q.double(), q, torch.zeros(2))


def test_rmsnorm_argument_checks_on_cpu():
    lib = _native.lib()
    # rejected before any device work: unsupported width, unsupported dtype, null pointers
    assert lib.ca_rmsnorm_forward(None, None, None, None, 4, 768, 1e-6, 0, 1, None) == 2
    assert lib.ca_rmsnorm_forward(None, None, None, None, 4, 1024, 1e-6, 2, 1, None) == 2
    assert lib.ca_rmsnorm_forward(None, None, None, None, 4, 1024, 1e-6, 0, 1, None) == 1
    assert b"null" in lib.ca_last_error()
    assert lib.ca_rmsnorm_forward(None, None, None, None, 0, 1024, 1e-6, 0, 1, None) == 0
    assert lib.ca_rmsnorm_workspace_size(0, 1024) == 0


def test_gelu_argument_checks_on_cpu():
    lib = _native.lib()
    # rejected before any device work: unknown dtype, ragged length, null pointers
    assert lib.ca_gelu_tanh_forward(None, None, 8, 7, None) == 1
    assert lib.ca_gelu_tanh_forward(None, None, 6, 1, None) == 2
    assert lib.ca_gelu_tanh_forward(None, None, 6, 0, None) == 2
    assert lib.ca_gelu_tanh_forward(None, None, 8, 1, None) == 1
    assert b"null" in lib.ca_last_error()
    assert lib.ca_gelu_tanh_backward(None, None, None, 4, 0, None) == 1
    assert lib.ca_gelu_tanh_forward(None, None, 0, 1, None) == 0
    assert lib.ca_gelu_tanh_backward(None, None, None, 0, 2, None) == 0


def test_rope_argument_checks_on_cpu():
    lib = _native.lib()
    fake = ctypes.c_void_p(256)
    # token and head counts beyond the kernels' 32-bit indexing are rejected before any device work
    st, msg = _status_and_msg(lib.ca_rope_qkv_forward(fake, fake, fake, fake, fake, 2, 1 << 30, 1, 8, 1, None))
    assert st == 2 and "2^31-1" in msg
    st, msg = _status_and_msg(lib.ca_rope_qkv_backward(fake, fake, fake, fake, fake, 1, 1 << 31, 1, 8, 1, None))
    assert st == 2 and "2^31-1" in msg
    st, msg = _status_and_msg(lib.ca_rope_qkv_forward(fake, fake, fake, fake, fake, 1, 4, (1 << 20) + 1, 8, 1, None))
    assert st == 2 and "heads" in msg
    st, msg = _status_and_msg(lib.ca_rope_qkv_forward(fake, fake, fake, fake, fake, 1, 4, 2, 12, 1, None))
    assert st == 2 and "multiple of 8" in msg
    assert lib.ca_rope_qkv_forward(None, None, None, None, None, 0, 4, 2, 8, 1, None) == 0


def test_backward_flags_checked_on_cpu():
    lib = _native.lib()
    fake = ctypes.c_void_p(256)
    args = (fake, fake, fake, fake, None, fake, fake, fake, fake, fake, fake, None, fake, 1 << 20,
            1, 2, 256, 64, 1, 0, 0)
    st, msg = _status_and_msg(lib.ca_backward_ex2(*args, 4, None))
    assert st == 1 and "flags" in msg
    # deterministic dQ needs the tcgen05 kernels: the CUDA-core family is refused up front
    st, msg = _status_and_msg(lib.ca_backward_ex2(*args[:-2], 1, 0, _native.CA_BWD_DETERMINISTIC, None))
    assert st == 2 and "deterministic" in msg
    st, msg = _status_and_msg(lib.ca_backward_ex2(fake, fake, fake, fake, None, fake, fake, fake, fake, fake, fake,
                                                  None, fake, 1 << 20, 1, 2, 256, 32, 1, 0, 0,
                                                  _native.CA_BWD_DETERMINISTIC, None))
    assert st == 2 and "deterministic" in msg
