"""GPU parity of the op-level kernels against the reference (golden
fixtures) and the pinned oracle.

Bars: integer/byte work (dequantization, repacking) is bit-exact; RoPE is
bit-exact (host table computed with the reference's arithmetic); the GEMV
and reductions are floating point with a per-row bound
    |y_gpu - y_ref| <= 1e-5 * sum_i |w_i * x_i| + sum_i |w_i| * r_i
(f32 accumulation in another order; the reference's own rounding error is
~1e-7 of the same sum).  r_i is the representation error of x_i in the
GEMV's block fixed point, one unit 2^(e-21) for a 32-block whose maximum lies
in [2^(e-1), 2^e) (zero for F32 weights, which meet x in f32)."""
import numpy as np
import pytest
import torch

import oracle as O
from smallm_engine_b200 import SmallmError, synth
from smallm_engine_b200 import _lib

pytestmark = pytest.mark.gpu

TYPES = [O.F32, O.Q4_0, O.Q8_0, O.Q6_K, O.Q4_K]


def x_rep_err(t, x):
    """Per-element bound on |x_i - X_i 2^(e-21)| (one unit of the 21-bit block
    fixed point, twice the rounding error); zero for F32 weights."""
    x = np.asarray(x, np.float64)
    out = np.zeros_like(x)
    if t == O.F32:
        return out
    n = x.size // 32 * 32
    m = np.abs(x[:n]).reshape(-1, 32).max(axis=1)
    e = np.frexp(m)[1]
    out[:n] = np.repeat(np.where(m >= 1e-30, np.ldexp(1.0, e - 21), 1e-30), 32)
    return out


def gemv_bound(orc, W, t, x, rows, cols):
    wd = np.abs(orc.dequantize(t, W, rows * cols).reshape(rows, cols).astype(np.float64))
    return 1e-5 * (wd @ np.abs(x.astype(np.float64))) + wd @ x_rep_err(t, x) + 1e-30


@pytest.mark.parametrize("t", [O.Q4_0, O.Q8_0, O.Q6_K, O.Q4_K])
def test_dequant_bit_exact(be, golden, t):
    g = golden("dequant")
    raw, want = g[f"raw_{t}"], g[f"out_{t}"].astype(np.float32)
    got = be.dequantize(t, raw, want.size)
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))


def assert_bits_equal_nan_aware(got, want):
    """Bit-identical except for the payload of NaN results: x86 propagates an
    input NaN's payload (and returns 0xFFC00000 for inf * 0) where the GPU
    returns its canonical NaN; NaN positions must still agree."""
    gn, wn = np.isnan(got), np.isnan(want)
    assert np.array_equal(gn, wn)
    assert np.array_equal(got[~gn].view(np.uint32), want[~wn].view(np.uint32))


@pytest.mark.parametrize("t", [O.Q4_0, O.Q8_0, O.Q6_K])
def test_dequant_random_bytes_bit_exact(be, orc, t):
    """Arbitrary block bytes (NaN/Inf/subnormal scales included)."""
    rng = np.random.default_rng(3 + t)
    be_, bb = {O.Q4_0: (32, 18), O.Q8_0: (32, 34), O.Q6_K: (256, 210)}[t]
    raw = rng.integers(0, 256, size=bb * 200, dtype=np.uint8)
    want = orc.dequantize(t, raw, 200 * be_)
    got = be.dequantize(t, raw, 200 * be_)
    assert_bits_equal_nan_aware(got, want)


@pytest.mark.parametrize("t,rows,cols", [(O.Q4_0, 37, 512), (O.Q4_0, 21, 96), (O.Q8_0, 9, 896),
                                         (O.Q6_K, 13, 2048), (O.Q4_K, 21, 1024), (O.F32, 5, 64)])
def test_repacked_layout_dequant_bit_exact(be, orc, t, rows, cols):
    """The device layout (split streams, Q6_K re-encoding, row padding) holds
    exactly the reference's values."""
    rng = np.random.default_rng(rows)
    w = (rng.standard_normal(rows * cols) * 0.02).astype(np.float32)
    W = synth.quantize(t, w) if t != O.F32 else w.view(np.uint8)
    qm = be.upload(W, t, rows, cols)
    y = torch.empty(rows * cols, dtype=torch.float32, device="cuda")
    qm.dequantize_to(y.data_ptr())
    be.synchronize()
    want = orc.dequantize(t, W, rows * cols)
    assert np.array_equal(y.cpu().numpy().view(np.uint32), want.view(np.uint32))
    g, d = qm.bytes()
    assert g == orc_bytes(t, rows, cols)


def orc_bytes(t, rows, cols):
    return rows * O.type_nbytes(t, cols)


@pytest.mark.parametrize("t", TYPES)
def test_matmul_quantized_vs_golden(be, orc, golden, t):
    g = golden("matmul")
    rows, cols = (int(v) for v in g[f"shape_{t}"])
    W, x, want = g[f"W_{t}"], g[f"x_{t}"], g[f"y_{t}"]
    y = be.matmul_quantized(W, t, x, rows, cols)
    assert np.all(np.abs(y.astype(np.float64) - want) <= gemv_bound(orc, W, t, x, rows, cols))


@pytest.mark.parametrize("t,rows,cols", [(O.Q4_0, 14336, 4096), (O.Q4_0, 4096, 14336), (O.Q8_0, 4864, 896),
                                         (O.Q8_0, 896, 4864), (O.Q6_K, 2048, 5632), (O.Q4_K, 5632, 2048),
                                         (O.Q4_0, 1000, 4096), (O.Q8_0, 3, 32), (O.Q4_0, 3, 32),
                                         (O.Q4_0, 33, 96), (O.Q4_0, 100, 4128), (O.Q4_0, 6144, 4096)])
def test_gemv_shapes_vs_oracle(be, orc, t, rows, cols):
    """Model shapes (config 2's Q4_0 matrices included) and ragged row counts."""
    rng = np.random.default_rng(rows + cols)
    w = (rng.standard_normal(rows * cols) * 0.02).astype(np.float32)
    W = synth.quantize(t, w)
    x = rng.standard_normal(cols).astype(np.float32)
    y = be.matmul_quantized(W, t, x, rows, cols)
    want = orc.matmul_quantized(W, t, x, rows, cols)
    assert np.all(np.abs(y.astype(np.float64) - want) <= gemv_bound(orc, W, t, x, rows, cols))


@pytest.mark.parametrize("t,rows,cols", [(O.Q8_0, 5, 40), (O.Q4_0, 6, 70), (O.Q6_K, 3, 300), (O.Q8_0, 4, 20),
                                         (O.Q4_0, 2, 0), (O.F32, 3, 0), (O.F32, 4, 1), (O.F32, 7, 45),
                                         (O.F32, 33, 301)])
def test_backend_matmul_partial_blocks_vs_oracle(be, orc, t, rows, cols):
    """Backend::matmul takes any column count; matmul_quantized covers whole
    blocks only (the tail of x is ignored, no whole block gives 0)."""
    from test_oracle import partial_case
    W, x = partial_case(t, rows, cols)
    want = orc.matmul_quantized(W, t, x, rows, cols)
    if t == O.F32:
        y = be.matmul(W.view(np.float32) if cols else np.zeros(1, np.float32), x, rows, cols)
    else:
        y = be.matmul_quantized(W, t, x, rows, cols)
    ce = cols if t == O.F32 else cols // (256 if t == O.Q6_K else 32) * (256 if t == O.Q6_K else 32)
    if ce == 0:
        assert np.array_equal(y, np.zeros(rows, np.float32)) and np.array_equal(want, y)
        return
    wd = np.abs(orc.dequantize(t, W, rows * ce).reshape(rows, ce).astype(np.float64))
    bound = 1e-5 * (wd @ np.abs(x[:ce].astype(np.float64))) + wd @ x_rep_err(t, x[:ce]) + 1e-30
    assert np.all(np.abs(y.astype(np.float64) - want) <= bound)


def test_backend_matmul_zero_rows(be):
    y = np.full(3, 7.0, np.float32)
    _lib.check(_lib.lib().smallm_backend_matmul(be.h, None, None, 0, 64, y.ctypes.data))
    assert np.all(y == 7.0)


def test_gemv_device_pointers_and_linearity(be, orc):
    """Device-resident GEMV: W(a x1 + b x2) = a W x1 + b W x2 within rounding
    and the representation error of each x."""
    rows, cols = 4096, 4096
    rng = np.random.default_rng(9)
    W = synth.quantize(O.Q4_0, (rng.standard_normal(rows * cols) * 0.02).astype(np.float32))
    qm = be.upload(W, O.Q4_0, rows, cols)
    x1 = torch.randn(cols, device="cuda")
    x2 = torch.randn(cols, device="cuda")
    ys = [torch.empty(rows, device="cuda") for _ in range(3)]
    s = torch.cuda.current_stream().cuda_stream
    qm.gemv(x1.data_ptr(), ys[0].data_ptr(), s)
    qm.gemv(x2.data_ptr(), ys[1].data_ptr(), s)
    x3 = 2.0 * x1 - 0.5 * x2
    qm.gemv(x3.data_ptr(), ys[2].data_ptr(), s)
    torch.cuda.synchronize()
    lhs = ys[2].double()
    rhs = 2.0 * ys[0].double() - 0.5 * ys[1].double()
    scale = ys[0].abs().max().item() + ys[1].abs().max().item()
    wd = np.abs(orc.dequantize(O.Q4_0, W, rows * cols).reshape(rows, cols).astype(np.float64))
    rep = wd @ (x_rep_err(O.Q4_0, x3.cpu().numpy()) + 2.0 * x_rep_err(O.Q4_0, x1.cpu().numpy()) +
                0.5 * x_rep_err(O.Q4_0, x2.cpu().numpy()))
    assert np.all((lhs - rhs).abs().cpu().numpy() <= 1e-5 * scale + rep)
    # split tiles are summed in a fixed order and their tickets reset: a
    # repeated launch gives the same bits
    again = torch.empty(rows, device="cuda")
    qm.gemv(x1.data_ptr(), again.data_ptr(), s)
    torch.cuda.synchronize()
    assert torch.equal(again, ys[0])


def test_matmul_weight_cache_reused(be):
    rng = np.random.default_rng(10)
    W = synth.quantize(O.Q8_0, (rng.standard_normal(64 * 256) * 0.02).astype(np.float32))
    x = rng.standard_normal(256).astype(np.float32)
    a = be.matmul_quantized(W, O.Q8_0, x, 64, 256)
    b = be.matmul_quantized(W, O.Q8_0, x, 64, 256)
    assert np.array_equal(a, b)


def test_unsupported_type_rejected(be):
    W = np.zeros(64 * 2 * 4, dtype=np.uint8)
    with pytest.raises(SmallmError) as e:
        be.matmul_quantized(W, 1, np.zeros(64, np.float32), 4, 64)  # F16: not implemented
    assert e.value.code == _lib.ERR_UNSUPPORTED_TYPE
    with pytest.raises(SmallmError) as e:
        be.matmul_quantized(W, 3, np.zeros(64, np.float32), 4, 64)
    assert e.value.code == _lib.ERR_UNSUPPORTED_TYPE


def test_ops_vs_golden(be, golden):
    g = golden("ops")
    for n in (1, 7, 64, 896, 4096):
        x, w = g[f"rms_x_{n}"], g[f"rms_w_{n}"]
        y = be.rmsnorm(x, w, n, 1e-6)
        assert np.allclose(y, g[f"rms_y_{n}"], rtol=1e-5, atol=1e-6)
        s = g[f"sm_x_{n}"].copy()
        be.softmax(s)
        assert np.allclose(s, g[f"sm_y_{n}"], rtol=1e-5, atol=1e-7)
        v = (x * 4).astype(np.float32)
        be.silu(v)
        assert np.allclose(v, g[f"silu_y_{n}"], rtol=1e-5, atol=1e-6)
    for k in [k[len("rope_x_"):] for k in g if k.startswith("rope_x_")]:
        nh, hd, pos, base = g[f"rope_args_{k}"]
        v = g[f"rope_x_{k}"].copy()
        be.rope(v, int(nh), int(hd), int(pos), float(base))
        assert np.array_equal(v, g[f"rope_y_{k}"]), k   # bit-exact


def test_softmax_empty_is_noop(be):
    x = np.zeros(0, dtype=np.float32)
    be.softmax(x)


def _residual_sum(be, qm, x_res, parts, flags, epoch, norm_w, eps, x_out, y):
    import ctypes
    _lib.check(_lib.lib().smallm_gemv_residual_sum(
        be.h, qm.h, x_res.data_ptr(), parts.data_ptr(), parts.shape[0], flags.data_ptr(), epoch.data_ptr(),
        norm_w.data_ptr(), ctypes.c_float(eps), x_out.data_ptr(), y.data_ptr(), None))


def _device_errors(be, clear=True):
    import ctypes
    f = ctypes.c_uint32(0)
    _lib.check(_lib.lib().smallm_ctx_device_errors(be.h, ctypes.byref(f), 1 if clear else 0))
    return f.value


def test_gemv_residual_sum_vs_oracle(be, orc):
    """The tensor-parallel residual step: x_out = x_res + parts in rank order
    (bit-exact f32 adds), then the reference's RMSNorm and the GEMV, once
    every arrival flag reads epoch + 1."""
    rows, cols, n, eps = 96, 2048, 3, 1e-5
    rng = np.random.default_rng(21)
    W = synth.quantize(O.Q4_0, (rng.standard_normal(rows * cols) * 0.02).astype(np.float32))
    qm = be.upload(W, O.Q4_0, rows, cols)
    xr = rng.standard_normal(cols).astype(np.float32)
    P = rng.standard_normal((n, cols)).astype(np.float32)
    nw = (1.0 + 0.1 * rng.standard_normal(cols)).astype(np.float32)
    dev = lambda a: torch.from_numpy(a).cuda()
    epoch = torch.tensor([41], dtype=torch.int32, device="cuda")
    flags = torch.full((n,), 42, dtype=torch.int32, device="cuda")
    x_out = torch.empty(cols, device="cuda")
    y = torch.empty(rows, device="cuda")
    assert _device_errors(be) == 0
    _residual_sum(be, qm, dev(xr), dev(P), flags, epoch, dev(nw), eps, x_out, y)
    torch.cuda.synchronize()
    assert _device_errors(be) == 0
    want_x = xr.copy()
    for r in range(n):
        want_x = (want_x + P[r]).astype(np.float32)
    assert np.array_equal(x_out.cpu().numpy().view(np.uint32), want_x.view(np.uint32))
    xn = orc.rmsnorm(want_x, nw, eps)
    want = orc.matmul_quantized(W, O.Q4_0, xn, rows, cols)
    got = y.cpu().numpy().astype(np.float64)
    # the GEMV bound plus the norm's own f32 rounding (1/rms applied to the row sums)
    bound = gemv_bound(orc, W, O.Q4_0, xn, rows, cols) + 1e-6 * np.abs(want)
    assert np.all(np.abs(got - want) <= bound)


def test_gemv_residual_sum_flag_wait_gives_up(be, orc):
    """A part whose arrival flag never comes up: the kernel's bounded wait
    (about a second) gives up, raises bit 3 of the device error word and the
    kernel ends; the context stays usable."""
    rows, cols = 32, 512
    rng = np.random.default_rng(22)
    W = synth.quantize(O.Q4_0, (rng.standard_normal(rows * cols) * 0.02).astype(np.float32))
    qm = be.upload(W, O.Q4_0, rows, cols)
    x_res = torch.randn(cols, device="cuda")
    parts = torch.randn(2, cols, device="cuda")
    norm_w = torch.ones(cols, device="cuda")
    epoch = torch.tensor([7], dtype=torch.int32, device="cuda")
    flags = torch.tensor([8, 0], dtype=torch.int32, device="cuda")  # the second sender never arrives
    x_out = torch.empty(cols, device="cuda")
    y = torch.empty(rows, device="cuda")
    assert _device_errors(be) == 0
    _residual_sum(be, qm, x_res, parts, flags, epoch, norm_w, 1e-5, x_out, y)
    torch.cuda.synchronize()
    assert _device_errors(be) & 8
    assert _device_errors(be) == 0  # cleared by the read above
    # the context still runs kernels, with correct results
    x = rng.standard_normal(cols).astype(np.float32)
    xd = torch.from_numpy(x).cuda()
    qm.gemv(xd.data_ptr(), y.data_ptr(), torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    want = orc.matmul_quantized(W, O.Q4_0, x, rows, cols)
    assert np.all(np.abs(y.cpu().numpy().astype(np.float64) - want) <= gemv_bound(orc, W, O.Q4_0, x, rows, cols))
    assert _device_errors(be) == 0
