"""The C ABI library loads and exports every function its header declares."""

import ctypes
import os
import re

import pytest

from conftest import ROOT
from triton_pesq_b200 import _lib

HEADER = os.path.join(ROOT, "include", "pesq_cuda.h")


def declared_functions():
    text = open(HEADER).read()
    return sorted(set(re.findall(r"^\s*(?:int|size_t|const char\*)\s+(pesq_\w+)\s*\(", text, re.M)))


def test_header_declares_the_entry_points():
    names = declared_functions()
    for want in ("pesq_plan_create", "pesq_forward", "pesq_backward", "pesq_workspace_size", "pesq_last_error",
                 "pesq_resampler_create", "pesq_resample_forward", "pesq_iir_create", "pesq_iir_workspace_bytes",
                 "pesq_iir_filter", "pesq_forward_noalloc"):
        assert want in names


def test_library_exports_every_declared_symbol():
    lib = ctypes.CDLL(_lib.LIB_PATH)
    for name in declared_functions():
        assert hasattr(lib, name), name
    assert set(_lib.SIGNATURES) >= set(declared_functions())


def test_abi_version_and_error_string():
    lib = _lib.library()
    assert lib.pesq_abi_version() == _lib.ABI_VERSION
    # a call rejected before touching the GPU sets a message
    assert lib.pesq_plan_create(None, None) == _lib.PESQ_ERR_INVALID_ARGUMENT
    assert "NULL" in _lib.last_error()


def test_torch_ops_register_without_a_gpu():
    import torch

    _lib.load_ops()
    assert hasattr(torch.ops.pesq_cuda, "forward")
    assert hasattr(torch.ops.pesq_cuda, "backward")


def test_cpu_input_raises():
    import torch

    from triton_pesq_b200 import PesqLossCuda

    model = PesqLossCuda(1.0, sample_rate=16000)
    with pytest.raises(RuntimeError):
        model(torch.randn(1, 16000), torch.randn(1, 16000))
    with pytest.raises(ValueError):
        model(torch.randn(1, 16000), torch.randn(1, 15000))
