"""The tensor-core (tcgen05) GEMM of the batched prefill, through the C ABI
(smallm_gemm_f16), against a float64 product of the same f16 operands.

The products of f16 values are exact in f32, so the only difference is the
accumulation order and rounding of the f32 sum:
    |y - y_ref| <= 1e-4 * sum_k |x_k * w_k|
(an operand-layout mistake gives errors of the size of y itself).  Shapes
cover one tile, ragged N/K/T (partial tiles and a partial last K stage that
the tensor map zero-fills), the prefill shapes of the Qwen2-1.5B and
Llama-3-8B decoders (many trips around the stage ring), all three token-tile
widths and persistent CTAs that take several tiles."""
import ctypes

import numpy as np
import pytest
import torch

from smallm_engine_b200 import SmallmError
from smallm_engine_b200 import _lib

pytestmark = pytest.mark.gpu


def gemm(be, w, x, y, ldy=None):
    """One launch on the context stream, waited for (torch's stream does not
    order with it)."""
    N, K = w.shape
    T = x.shape[0]
    torch.cuda.synchronize()
    _lib.check(_lib.lib().smallm_gemm_f16(be.h, w.data_ptr(), x.data_ptr(), N, K, T, y.data_ptr(),
                                          ldy if ldy is not None else N, be.stream))
    be.synchronize()


def device_errors(be, clear=True):
    f = ctypes.c_uint32()
    _lib.check(_lib.lib().smallm_ctx_device_errors(be.h, ctypes.byref(f), 1 if clear else 0))
    return f.value


def operands(N, K, T, seed):
    g = torch.Generator(device="cuda").manual_seed(seed)
    w = (torch.randn(N, K, device="cuda", generator=g) * 0.02).half()
    x = torch.randn(T, K, device="cuda", generator=g).half()
    return w, x


def check(y, w, x):
    wd, xd = w.double(), x.double()
    want = xd @ wd.T
    bound = 1e-4 * (xd.abs() @ wd.abs().T) + 1e-30
    err = (y.double() - want).abs()
    assert bool((err <= bound).all()), float((err / bound).max())


@pytest.mark.parametrize("N,K,T", [
    (128, 64, 64),       # one tile, one stage
    (300, 200, 37),      # ragged rows, K (a partial last stage) and tokens
    (2048, 1536, 512),   # Qwen2-1.5B QKV over a 512-token prompt (64-token tiles)
    (4096, 14336, 128),  # Llama-3-8B down: 224 K stages around the ring
    (4096, 1024, 384),   # 128-token tiles
    (28672, 4096, 256),  # Llama-3-8B gate/up: 256-token tiles, some CTAs take two
    (17920, 1536, 2048), # Qwen2-1.5B gate/up over 4 x 512 tokens: ~8 tiles per CTA,
                         # both accumulators reused several times
])
def test_tc_gemm_matches_f64(be, N, K, T):
    w, x = operands(N, K, T, seed=N + K + T)
    y = torch.full((T, N), float("nan"), device="cuda")
    device_errors(be)
    gemm(be, w, x, y)
    torch.cuda.synchronize()
    assert device_errors(be) == 0
    check(y, w, x)


def test_tc_gemm_row_stride_and_repeat(be):
    N, K, T, ldy = 256, 128, 100, 300
    w, x = operands(N, K, T, seed=5)
    y = torch.full((T, ldy), -7.0, device="cuda")
    gemm(be, w, x, y, ldy)
    first = y.clone()
    gemm(be, w, x, y, ldy)
    torch.cuda.synchronize()
    check(y[:, :N], w, x)
    assert bool((y[:, N:] == -7.0).all())          # columns past N untouched
    assert torch.equal(y, first)                    # deterministic


def test_tc_gemm_rejects_bad_shapes(be):
    w, x = operands(128, 64, 16, seed=1)
    y = torch.empty(16, 128, device="cuda")
    L = _lib.lib()
    s = torch.cuda.current_stream().cuda_stream
    with pytest.raises(SmallmError):   # K not a multiple of 8
        _lib.check(L.smallm_gemm_f16(be.h, w.data_ptr(), x.data_ptr(), 128, 60, 16, y.data_ptr(), 128, s))
    with pytest.raises(SmallmError):   # ldy < N
        _lib.check(L.smallm_gemm_f16(be.h, w.data_ptr(), x.data_ptr(), 128, 64, 16, y.data_ptr(), 100, s))
    with pytest.raises(SmallmError):   # misaligned operand
        _lib.check(L.smallm_gemm_f16(be.h, w.data_ptr() + 2, x.data_ptr(), 128, 64, 16, y.data_ptr(), 128, s))
    # empty products are no-ops
    _lib.check(L.smallm_gemm_f16(be.h, w.data_ptr(), x.data_ptr(), 0, 64, 16, y.data_ptr(), 128, s))
    _lib.check(L.smallm_gemm_f16(be.h, w.data_ptr(), x.data_ptr(), 128, 64, 0, y.data_ptr(), 128, s))
    torch.cuda.synchronize()
