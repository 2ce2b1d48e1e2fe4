"""Batched prefill (smallm_model_prefill: the GEMMs on the backend's tcgen05
tensor-core kernel over f16 weight copies) against the oracle's restatement
of the token-by-token forward (the reference's Generator prefill,
src/runtime/generator.cpp:47-51): the last token's logits within
1e-2 * max|logit|, the same greedy id, the greedy ids of the decode that
continues from the prefilled cache identical, and prefix reuse (two prefill
segments) equal to one pass."""
import numpy as np
import pytest

import oracle as O
from smallm_engine_b200 import CudaModel, SmallmError, synth

pytestmark = pytest.mark.gpu

TOL = 1e-2


def close(a, b, tol=TOL):
    return np.abs(a.astype(np.float64) - b).max() <= tol * np.abs(b).max()


def _oracle_last(ref, toks):
    want = None
    for p, t in enumerate(toks):
        want = ref.forward(int(t), p)
    return want


@pytest.mark.parametrize("kind,seed", [("qwen2", 7), ("llama-q4_0", 8), ("llama-kq", 9)])
def test_prefill_matches_token_by_token(orc, gguf_dir, kind, seed):
    spec = synth.tiny_spec(kind)
    path = synth.write_gguf(spec, seed, gguf_dir / f"pre-{kind}.gguf")
    ref = O.OracleModel(path, orc)
    rng = np.random.default_rng(seed)
    toks = [int(t) for t in rng.integers(0, spec.vocab, size=21)]
    want = _oracle_last(ref, toks)
    m = CudaModel(path)
    got, am = m.prefill(toks, 0)
    assert close(got, want)
    assert am == int(np.argmax(got)) == int(np.argmax(want))
    assert m.cached_length() == len(toks)
    # decode continues from the prefilled cache
    ids = m.decode_greedy(am, len(toks), 12)
    pos, n = len(toks), am
    for k in range(12):
        l = ref.forward(n, pos)
        pos += 1
        n = int(np.argmax(l))
        assert int(ids[k]) == n


def test_prefill_in_segments_equals_one_pass(gguf_dir):
    spec = synth.tiny_spec("llama-q4_0")
    path = synth.write_gguf(spec, 8, gguf_dir / "pre-seg.gguf")
    toks = list(range(3, 40, 2))
    m = CudaModel(path)
    one, _ = m.prefill(toks, 0)
    m.reset_cache()
    m.prefill(toks[:7], 0, want_logits=False)
    two, _ = m.prefill(toks[7:], 7)
    assert close(two, one)
    # a forward after a prefill sees the same cache as forwards all along
    m.truncate_cache(len(toks) - 1)
    again = m.forward(toks[-1], len(toks) - 1)
    assert close(again, one)


def test_prefill_long_prompt_key_splits(orc, gguf_dir):
    """A 130-token prompt: few token blocks, so the attention splits each
    block's keys over several CTAs and merges the partials.  One pass and two
    segments (the second starting at position 60) against the token-by-token
    restatement."""
    spec = synth.tiny_spec("llama-q4_0", ctx=256)
    path = synth.write_gguf(spec, 12, gguf_dir / "pre-long.gguf")
    toks = [int(t) for t in np.random.default_rng(12).integers(0, spec.vocab, size=130)]
    ref = O.OracleModel(path, orc)
    want = _oracle_last(ref, toks)
    m = CudaModel(path)
    got, am = m.prefill(toks, 0)
    assert close(got, want)
    assert am == int(np.argmax(want))
    m.reset_cache()
    m.prefill(toks[:60], 0, want_logits=False)
    two, am2 = m.prefill(toks[60:], 60)
    assert close(two, want)
    assert am2 == am


def test_prefill_wide_model_vs_oracle(orc, gguf_dir):
    """A wider model and a 300-token prompt (several row and token tiles per
    GEMM) against the oracle's token-by-token forward, in one pass and in two
    segments (the attention then splits the keys over a different number of
    CTAs: another f32 summation order, which the f16 rounding of the GEMM
    inputs can turn into 2^-11 steps; both stay inside the model bar)."""
    spec = synth.tiny_spec("llama-q4_0", embd=1024, heads=8, kv_heads=2, ffn=2816, vocab=1024, ctx=512)
    path = synth.write_gguf(spec, 11, gguf_dir / "pre-tc-wide.gguf")
    toks = [int(t) for t in np.random.default_rng(11).integers(0, spec.vocab, size=300)]
    want = _oracle_last(O.OracleModel(path, orc), toks)
    m = CudaModel(path)
    one, am_one = m.prefill(toks, 0)
    assert close(one, want)
    assert am_one == int(np.argmax(want))
    m.reset_cache()
    m.prefill(toks[:170], 0, want_logits=False)
    two, am_two = m.prefill(toks[170:], 170)
    assert close(two, want)
    assert am_two == am_one


def test_prefill_rejects_unknown_flags(gguf_dir):
    import ctypes
    from smallm_engine_b200 import _lib
    spec = synth.tiny_spec("llama-q4_0")
    path = synth.write_gguf(spec, 8, gguf_dir / "pre-flags.gguf")
    m = CudaModel(path)
    toks = np.array([1, 2, 3], np.uint32)
    rc = _lib.lib().smallm_model_prefill(m.h, toks.ctypes.data, 3, 0, None, None, 1)
    assert rc == _lib.ERR_INVALID
    assert _lib.lib().smallm_model_prefill(m.h, toks.ctypes.data, 3, 0, None, None, 2) == 0  # the named default


def test_prefill_errors(gguf_dir):
    spec = synth.tiny_spec("llama-q4_0")
    path = synth.write_gguf(spec, 8, gguf_dir / "pre-err.gguf")
    m = CudaModel(path, max_ctx=32)
    with pytest.raises(SmallmError):
        m.prefill([1] * 40, 0)           # past the context
    with pytest.raises(SmallmError):
        m.prefill([spec.vocab], 0)       # id out of range
    with pytest.raises(SmallmError):
        m.prefill([], 0)
