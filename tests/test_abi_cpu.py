"""The C-ABI library: it builds, loads, and exports every declared entry point.

No compute runs here (no GPU on this host); creating a backend must fail
with a typed error rather than crash.
"""
import os

import pytest

from runtime_b200 import _lib

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "mfcuda.h")


@pytest.fixture(scope="module")
def lib():
    from runtime_b200 import build

    build.build()
    return _lib.load()


def test_every_header_symbol_is_exported(lib):
    declared = _lib.exported_symbols(HEADER)
    assert len(declared) > 60
    missing = [name for name in declared if not hasattr(lib, name)]
    assert not missing, missing
    # and every declared symbol has a Python signature
    assert set(declared) <= set(_lib.SIGNATURES), set(declared) - set(_lib.SIGNATURES)


def test_abi_version(lib):
    assert lib.mf_abi_version() == 1


def test_no_gpu_backend_create_is_a_typed_error(lib):
    import torch

    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    from runtime_b200.backend import CudaBackend, ExecutorError

    with pytest.raises(ExecutorError) as e:
        CudaBackend(0)
    assert e.value.kind in ("BackendFailure", "InvalidArgument")
