"""The C-ABI library loads and exports every entry point include/smallm_cuda.h
declares; without a GPU every compute call fails cleanly (no CPU fallback)."""
import ctypes
import subprocess

import pytest

from smallm_engine_b200 import _lib


def test_library_exports_every_declared_symbol():
    declared = _lib.declared_symbols()
    assert len(declared) >= 30
    out = subprocess.run(["nm", "-D", "--defined-only", str(_lib.LIB_PATH)], capture_output=True, text=True,
                         check=True).stdout
    exported = {line.split()[-1] for line in out.splitlines() if " T " in line}
    missing = [s for s in declared if s not in exported]
    assert not missing, missing
    L = _lib.lib()
    for s in declared:
        assert getattr(L, s) is not None
    assert set(_lib.SIGNATURES) == set(declared)


def test_version_and_error_string():
    L = _lib.lib()
    assert L.smallm_version() >= 100
    assert isinstance(L.smallm_last_error(), bytes)


def _has_gpu():
    try:
        import torch
        return torch.cuda.is_available()
    except Exception:
        return False


@pytest.mark.skipif(_has_gpu(), reason="checks the no-GPU failure mode")
def test_no_gpu_fails_loudly():
    from smallm_engine_b200 import CUDABackend, CudaModel, SmallmError
    with pytest.raises(SmallmError) as e:
        CUDABackend(0)
    assert e.value.code == _lib.ERR_CUDA
    with pytest.raises(SmallmError):
        CudaModel("/nonexistent.gguf")


def test_null_arguments_rejected():
    L = _lib.lib()
    assert L.smallm_ctx_create(0, None) == _lib.ERR_INVALID
    assert L.smallm_model_forward(None, 0, 0, None, None) == _lib.ERR_INVALID
    assert L.smallm_qmatrix_bytes(None, None, None) == _lib.ERR_INVALID
