"""smallm_attention_noalloc: the split-K decode attention with its scratch in a
static device array of the library (no allocation per call or per context).

It is compared with the same attention computed through the existing Backend
entry points, composed the way the reference's forward composes its ops
(src/model/qwen2/qwen2_model.cpp:111-133: a dot per cached position, scale,
softmax, then the weighted sum of V rows): smallm_backend_matmul for the
scores and for V^T . p, smallm_backend_softmax in between.  Two calls run back
to back on one stream before a single synchronise, so the second reuses the
tickets the first put back to zero.  The file name sorts last so the test also
runs after every other GPU test in the same process.
"""
from __future__ import annotations

import ctypes
import math

import numpy as np
import pytest

from smallm_engine_b200 import SmallmError, _lib

pytestmark = pytest.mark.gpu


def _call(be, q, kc, vc, n_heads, n_kv, hd, max_ctx, pos, out, stream):
    _lib.check(_lib.lib().smallm_attention_noalloc(be.h, q.data_ptr(), kc.data_ptr(), vc.data_ptr(), n_heads,
                                                   n_kv, hd, max_ctx, pos, out.data_ptr(), stream))


def _via_backend_ops(be, q, kc, vc, n_heads, n_kv, hd, pos):
    """Attention from smallm_backend_matmul + smallm_backend_softmax (host in,
    host out)."""
    group = n_heads // n_kv
    n = pos + 1
    n_pad = (n + 31) // 32 * 32  # V^T . p with zero columns appended (they add nothing)
    scale = np.float32(1.0 / math.sqrt(hd))
    out = np.empty((n_heads, hd), dtype=np.float32)
    for h in range(n_heads):
        g = h // group
        K = np.ascontiguousarray(kc[g, :n])
        s = be.matmul(K, q[h], n, hd) * scale
        be.softmax(s)
        Vt = np.zeros((hd, n_pad), dtype=np.float32)
        Vt[:, :n] = vc[g, :n].T
        p = np.zeros(n_pad, dtype=np.float32)
        p[:n] = s
        out[h] = be.matmul(Vt, p, hd, n_pad)
    return out


@pytest.mark.parametrize("n_heads,n_kv,hd,max_ctx,positions", [
    (32, 8, 128, 512, (300, 301)),     # Llama-3-8B attention shape
    (14, 2, 64, 512, (0, 37)),         # Qwen2-0.5B attention shape
])
def test_noalloc_attention_matches_backend_ops(be, n_heads, n_kv, hd, max_ctx, positions):
    import torch
    rng = np.random.default_rng(11)
    kc = rng.standard_normal((n_kv, max_ctx, hd), dtype=np.float32)
    vc = rng.standard_normal((n_kv, max_ctx, hd), dtype=np.float32)
    qs = [rng.standard_normal((n_heads, hd), dtype=np.float32) for _ in positions]
    dev = torch.device("cuda", 0)
    kc_d, vc_d = torch.from_numpy(kc).to(dev), torch.from_numpy(vc).to(dev)
    qs_d = [torch.from_numpy(q).to(dev) for q in qs]
    outs = [torch.full((n_heads * hd,), float("nan"), device=dev) for _ in range(len(positions) + 1)]
    stream = torch.cuda.current_stream(dev).cuda_stream
    for q_d, pos, out in zip(qs_d, positions, outs):
        _call(be, q_d, kc_d, vc_d, n_heads, n_kv, hd, max_ctx, pos, out, stream)
    # a third call repeats the first: the same partition, so the same bits
    _call(be, qs_d[0], kc_d, vc_d, n_heads, n_kv, hd, max_ctx, positions[0], outs[-1], stream)
    torch.cuda.synchronize(dev)
    got = [o.cpu().numpy().reshape(n_heads, hd) for o in outs]
    for q, pos, g in zip(qs, positions, got):
        want = _via_backend_ops(be, q, kc, vc, n_heads, n_kv, hd, pos)
        # f32 throughout; only the summation order differs
        np.testing.assert_allclose(g, want, rtol=1e-4, atol=1e-5)
    assert np.array_equal(got[0], got[-1])


def test_noalloc_attention_rejects_out_of_range(be):
    import torch
    dev = torch.device("cuda", 0)
    buf = torch.zeros(16, device=dev)
    p = buf.data_ptr()
    L = _lib.lib()
    # partials for max_ctx 65536 at 32 heads of 128 need ~17 MB > 4 MiB
    rc = L.smallm_attention_noalloc(be.h, p, p, p, 32, 8, 128, 65536, 0, p, None)
    assert rc == _lib.ERR_RANGE and b"static scratch" in L.smallm_last_error()
    assert L.smallm_attention_noalloc(be.h, p, p, p, 32, 8, 128, 512, 512, p, None) == _lib.ERR_RANGE
    assert L.smallm_attention_noalloc(be.h, p, p, p, 32, 8, 96, 512, 0, p, None) == _lib.ERR_INVALID
    assert L.smallm_attention_noalloc(be.h, p, p, p, 30, 8, 128, 512, 0, p, None) == _lib.ERR_INVALID
    assert L.smallm_attention_noalloc(be.h, None, p, p, 32, 8, 128, 512, 0, p, None) == _lib.ERR_INVALID
    torch.cuda.synchronize(dev)
    assert not torch.isnan(buf).any() and float(buf.abs().sum()) == 0.0  # nothing was launched
    with pytest.raises(SmallmError):
        _lib.check(rc)
