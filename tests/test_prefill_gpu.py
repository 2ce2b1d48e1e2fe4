"""Batched prefill (smallm_model_prefill) against the restatement's
token-by-token forward (the reference's Generator prefill,
src/runtime/generator.cpp:47-51): the last token's logits within
1e-2 * max|logit| (exact-f32 GEMMs land near 1e-5), the greedy ids of the
decode that continues from the prefilled cache identical, and prefix reuse
(two prefill segments) equal to one pass."""
import numpy as np
import pytest

import oracle as O
from smallm_engine_b200 import CudaModel, SmallmError, synth

pytestmark = pytest.mark.gpu

TOL = 1e-2


def close(a, b, tol=TOL):
    return np.abs(a.astype(np.float64) - b).max() <= tol * np.abs(b).max()


@pytest.mark.parametrize("kind,seed", [("qwen2", 7), ("llama-q4_0", 8), ("llama-kq", 9)])
def test_prefill_matches_token_by_token(orc, gguf_dir, kind, seed):
    spec = synth.tiny_spec(kind)
    path = synth.write_gguf(spec, seed, gguf_dir / f"pre-{kind}.gguf")
    ref = O.OracleModel(path, orc)
    rng = np.random.default_rng(seed)
    toks = [int(t) for t in rng.integers(0, spec.vocab, size=21)]
    want = None
    for p, t in enumerate(toks):
        want = ref.forward(t, p)
    m = CudaModel(path)
    got, am = m.prefill(toks, 0)
    assert close(got, want)
    assert np.abs(got.astype(np.float64) - want).max() <= 1e-4 * np.abs(want).max()  # exact-f32 GEMMs
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
    assert close(two, one, 1e-5)
    # a forward after a prefill sees the same cache as forwards all along
    m.truncate_cache(len(toks) - 1)
    again = m.forward(toks[-1], len(toks) - 1)
    assert close(again, one, 1e-4)


def test_prefill_tf32(orc, gguf_dir):
    spec = synth.tiny_spec("llama-q4_0")
    path = synth.write_gguf(spec, 8, gguf_dir / "pre-tf32.gguf")
    ref = O.OracleModel(path, orc)
    toks = [5, 9, 200, 31, 7, 64, 2, 150]
    want = None
    for p, t in enumerate(toks):
        want = ref.forward(t, p)
    got, _ = CudaModel(path).prefill(toks, 0, tf32=True)
    assert close(got, want)


@pytest.mark.parametrize("kind,seed", [("qwen2", 7), ("llama-q4_0", 8), ("llama-kq", 9)])
def test_prefill_tensor_cores(orc, gguf_dir, kind, seed):
    """The GEMMs on the backend's tcgen05 kernel over f16 weight copies: the
    last logits within 1e-2 * max|logit| of the token-by-token restatement,
    the same greedy id, and decode continuing from that cache matching it."""
    spec = synth.tiny_spec(kind)
    path = synth.write_gguf(spec, seed, gguf_dir / f"pre-tc-{kind}.gguf")
    ref = O.OracleModel(path, orc)
    rng = np.random.default_rng(seed)
    toks = [int(t) for t in rng.integers(0, spec.vocab, size=21)]
    want = None
    for p, t in enumerate(toks):
        want = ref.forward(t, p)
    m = CudaModel(path)
    got, am = m.prefill(toks, 0, tensor_cores=True)
    assert close(got, want)
    assert am == int(np.argmax(got)) == int(np.argmax(want))
    ids = m.decode_greedy(am, len(toks), 8)
    pos, n = len(toks), am
    for k in range(8):
        l = ref.forward(n, pos)
        pos += 1
        n = int(np.argmax(l))
        assert int(ids[k]) == n


@pytest.mark.parametrize("tensor_cores", [False, True])
def test_prefill_long_prompt_key_splits(orc, gguf_dir, tensor_cores):
    """A 130-token prompt: few token blocks, so the attention splits each
    block's keys over several CTAs and merges the partials.  One pass and two
    segments (the second starting at position 60) against the token-by-token
    restatement."""
    spec = synth.tiny_spec("llama-q4_0", ctx=256)
    path = synth.write_gguf(spec, 12, gguf_dir / "pre-long.gguf")
    toks = [int(t) for t in np.random.default_rng(12).integers(0, spec.vocab, size=130)]
    ref = O.OracleModel(path, orc)
    want = None
    for p, t in enumerate(toks):
        want = ref.forward(t, p)
    m = CudaModel(path)
    got, am = m.prefill(toks, 0, tensor_cores=tensor_cores)
    assert close(got, want, TOL if tensor_cores else 1e-4)
    assert am == int(np.argmax(want))
    m.reset_cache()
    m.prefill(toks[:60], 0, want_logits=False, tensor_cores=tensor_cores)
    two, am2 = m.prefill(toks[60:], 60, tensor_cores=tensor_cores)
    assert close(two, want, TOL if tensor_cores else 1e-4)
    assert am2 == am


def test_prefill_tensor_cores_wide(gguf_dir):
    """A wider model and a 300-token prompt (several row and token tiles per
    GEMM): tensor-core prefill against the exact-f32 prefill."""
    spec = synth.tiny_spec("llama-q4_0", embd=1024, heads=8, kv_heads=2, ffn=2816, vocab=1024, ctx=512)
    path = synth.write_gguf(spec, 11, gguf_dir / "pre-tc-wide.gguf")
    toks = [int(t) for t in np.random.default_rng(11).integers(0, spec.vocab, size=300)]
    m = CudaModel(path)
    exact, am_exact = m.prefill(toks, 0)
    m.reset_cache()
    tc, am_tc = m.prefill(toks, 0, tensor_cores=True)
    assert close(tc, exact)
    assert am_tc == am_exact
    # two tensor-core segments against one pass: the attention splits the keys
    # over a different number of CTAs in each (another f32 summation order),
    # and the f16 rounding of the GEMM inputs turns such last-bit differences
    # into 2^-11 steps, so the bound is the tensor-core one
    m.reset_cache()
    m.prefill(toks[:170], 0, want_logits=False, tensor_cores=True)
    two, am_two = m.prefill(toks[170:], 170, tensor_cores=True)
    assert close(two, tc)
    assert am_two == am_tc


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
