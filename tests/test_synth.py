"""Synthetic GGUF inputs: quantizers match gguf-py byte for byte (Q8_0,
Q4_0), K-quant encoders round-trip through the oracle's dequantizers, and
written files load in gguf-py and in the reference."""
import numpy as np
import pytest

import oracle as O
from smallm_engine_b200 import synth


@pytest.mark.parametrize("t", [synth.Q8_0, synth.Q4_0])
def test_quantizer_matches_gguf_py(t):
    import gguf
    rng = np.random.default_rng(5)
    x = (rng.standard_normal(32 * 300) * 0.02).astype(np.float32)
    x[:32] = 0.0                        # all-zero block
    x[32:64] = np.linspace(-1, 1, 32)   # exact ties in |x|
    x[64] = 70000.0                     # scale overflows f16
    ours = synth.quantize(t, x)
    theirs = gguf.quants.quantize(x.reshape(-1, 32), gguf.GGMLQuantizationType(t)).ravel()
    assert np.array_equal(ours, theirs)


def test_f16_rounding_matches_numpy():
    rng = np.random.default_rng(6)
    v = np.concatenate([rng.standard_normal(20000) * 10.0 ** rng.integers(-9, 6, 20000),
                        [0.0, -0.0, 65504.0, 65520.0, 1e-8, 2.0 ** -24, 2.0 ** -25, 3 * 2.0 ** -26]]).astype(np.float32)
    lib = synth._synth_lib()
    ours = np.array([lib.synth_f32_to_f16(float(a)) for a in v], dtype=np.uint16)
    assert np.array_equal(ours, v.astype(np.float16).view(np.uint16))


@pytest.mark.parametrize("t,sub,levels,rms", [(synth.Q6_K, 16, 62, 0.03), (synth.Q4_K, 32, 15, 0.12)])
def test_kquant_roundtrip(orc, t, sub, levels, rms):
    rng = np.random.default_rng(7)
    x = (rng.standard_normal(256 * 64) * 0.02).astype(np.float32)
    q = synth.quantize(t, x)
    y = orc.dequantize(t, q, x.size)
    blk = x.reshape(-1, sub)
    # quantization step of each sub-block (value range / number of levels)
    step = ((blk.max(axis=1) - np.minimum(blk.min(axis=1), 0)) / levels).repeat(sub)
    assert np.all(np.abs(y - x) <= 1.5 * step + 1e-4)
    assert np.sqrt(np.mean((y - x) ** 2)) / np.sqrt(np.mean(x ** 2)) < rms


def test_gguf_file_readable(gguf_dir):
    import gguf
    spec = synth.tiny_spec("llama-kq")
    p = synth.write_gguf(spec, 3, gguf_dir / "r.gguf")
    r = gguf.GGUFReader(str(p))
    names = {t.name: t for t in r.tensors}
    assert set(names) == {n for n, *_ in spec.tensors()}
    assert int(names["blk.0.attn_v.weight"].tensor_type) == synth.Q6_K
    assert int(names["blk.0.attn_q.weight"].tensor_type) == synth.Q4_K
    f = O.GGUFFile(p)
    assert f.meta["llama.block_count"] == spec.layers
    assert len(f.meta["tokenizer.ggml.tokens"]) == spec.vocab


def test_gguf_loads_in_reference(ref, gguf_dir):
    spec = synth.tiny_spec("qwen2")
    p = synth.write_gguf(spec, 1, gguf_dir / "q.gguf")
    m = ref.load(p)
    assert (m.n_layers, m.embd, m.n_heads, m.n_kv, m.vocab, m.ctx) == (
        spec.layers, spec.embd, spec.heads, spec.kv_heads, spec.vocab, spec.ctx)
    assert np.isfinite(m.forward(1, 0)).all()


def test_workload_bytes():
    s = synth.WORKLOADS["llama3-8b-q4_0"]
    wb = s.weight_bytes_per_token()
    # 32 layers of Q4_0 linears + Q8_0 lm_head (about 4.48 GB)
    assert 4.40e9 < wb < 4.50e9
