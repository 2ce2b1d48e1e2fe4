"""smallm_attention_noalloc: the split-K decode attention with its scratch in a
static device array of the library (no allocation per call or per context).

Some callers cannot let the library allocate: a serving engine that has given
all of the GPU's memory to its own KV-block pool leaves nothing for cudaMalloc
to find, and a latency-bound decode loop cannot absorb the device
synchronisation cudaMalloc / cudaFree may cause.  This entry point serves them.

Its output is compared with the oracle's restatement of the reference's
attention loop (src/model/qwen2_model.cpp:111-133: a dot per cached position,
scale, softmax, then the weighted sum of V rows; oracle.c orc_attention), on
the same seeded q / K / V.  Two calls run back to back on one stream before a
single synchronise, so the second reuses the tickets the first put back to
zero, and a third call repeating the first must give the same bits.  The cases
cover the Llama-3-8B and Qwen2-0.5B attention shapes, a context whose K/V
chunk needs more than 48 KiB of shared memory (max_ctx 4096), and the largest
context whose partials fit the 4 MiB array at 32 heads of 128 (max_ctx 16128,
positions near its end).  The file name sorts last so the test also runs
after every other GPU test in the same process.
"""
from __future__ import annotations

import numpy as np
import pytest

from smallm_engine_b200 import SmallmError, _lib

pytestmark = pytest.mark.gpu


def _call(be, q, kc, vc, n_heads, n_kv, hd, max_ctx, pos, out, stream):
    _lib.check(_lib.lib().smallm_attention_noalloc(be.h, q.data_ptr(), kc.data_ptr(), vc.data_ptr(), n_heads,
                                                   n_kv, hd, max_ctx, pos, out.data_ptr(), stream))


@pytest.mark.parametrize("n_heads,n_kv,hd,max_ctx,positions", [
    (32, 8, 128, 512, (300, 301)),         # Llama-3-8B attention shape
    (14, 2, 64, 512, (0, 37)),             # Qwen2-0.5B attention shape
    (32, 8, 128, 4096, (2303, 4095)),      # K/V chunk over 48 KiB of shared memory
    (32, 8, 128, 16128, (16000, 16127)),   # partials just inside the 4 MiB array
])
def test_noalloc_attention_matches_oracle(be, orc, n_heads, n_kv, hd, max_ctx, positions):
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
    got = [o.cpu().numpy() for o in outs]
    # the reference's cache layout, [position][kv head][head_dim]
    kc_ref = np.ascontiguousarray(kc.transpose(1, 0, 2))
    vc_ref = np.ascontiguousarray(vc.transpose(1, 0, 2))
    for q, pos, g in zip(qs, positions, got):
        want = orc.attention(q.ravel(), kc_ref, vc_ref, n_heads, n_kv, hd, pos)
        # f32 throughout; only the summation order differs
        np.testing.assert_allclose(g, want, rtol=1e-4, atol=2e-5)
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
    # one split more than max_ctx 16128 needs: the partials pass 4 MiB
    assert L.smallm_attention_noalloc(be.h, p, p, p, 32, 8, 128, 16192, 0, p, None) == _lib.ERR_RANGE
    # K/V rows are bulk-copied: their base pointers must be 16-byte aligned
    assert L.smallm_attention_noalloc(be.h, p, p + 4, p, 32, 8, 128, 512, 0, p, None) == _lib.ERR_INVALID
    assert L.smallm_attention_noalloc(be.h, p, p, p + 8, 32, 8, 128, 512, 0, p, None) == _lib.ERR_INVALID
    torch.cuda.synchronize(dev)
    assert not torch.isnan(buf).any() and float(buf.abs().sum()) == 0.0  # nothing was launched
    with pytest.raises(SmallmError):
        _lib.check(rc)
