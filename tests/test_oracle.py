"""The CPU oracle is pinned before anything is checked against it: the C
restatement must reproduce the reference's outputs (golden fixtures made by
the reference build, tests/golden/make_golden.py) bit for bit, and where the
reference build is present, on fresh random inputs too."""
import hashlib

import numpy as np
import pytest

import oracle as O
from smallm_engine_b200 import synth


def test_f16_table_matches_reference(orc, golden):
    g = golden("f16")
    bits = np.array([orc.f16_to_f32(int(c)) for c in range(65536)], dtype=np.float32).view(np.uint32)
    assert hashlib.sha256(bits.tobytes()).hexdigest() == str(g["sha256"])
    assert np.array_equal(bits[g["codes"]], g["bits"])


@pytest.mark.parametrize("t", [O.Q4_0, O.Q8_0, O.Q6_K, O.Q4_K])
def test_dequant_matches_golden(orc, golden, t):
    g = golden("dequant")
    raw, want = g[f"raw_{t}"], g[f"out_{t}"]
    got = orc.dequantize(t, raw, want.size)
    assert np.array_equal(got.view(np.uint32), want.astype(np.float32).view(np.uint32))


@pytest.mark.parametrize("t", [O.F32, O.Q4_0, O.Q8_0, O.Q6_K])
def test_matmul_bit_exact_vs_golden(orc, golden, t):
    g = golden("matmul")
    rows, cols = g[f"shape_{t}"]
    y = orc.matmul_quantized(g[f"W_{t}"], t, g[f"x_{t}"], int(rows), int(cols))
    assert np.array_equal(y.view(np.uint32), g[f"y_{t}"].view(np.uint32))


def test_matmul_q4k_vs_gguf_py(orc, golden):
    g = golden("matmul")
    rows, cols = g[f"shape_{O.Q4_K}"]
    W, x = g[f"W_{O.Q4_K}"], g[f"x_{O.Q4_K}"]
    y = orc.matmul_quantized(W, O.Q4_K, x, int(rows), int(cols))
    wd = orc.dequantize(O.Q4_K, W, int(rows * cols)).reshape(int(rows), int(cols))
    bound = 1e-6 * (np.abs(wd) @ np.abs(x)) + 1e-12
    assert np.all(np.abs(y - g[f"y_{O.Q4_K}"]) <= bound)


def test_ops_bit_exact_vs_golden(orc, golden):
    g = golden("ops")
    for n in (1, 7, 64, 896, 4096):
        assert np.array_equal(orc.rmsnorm(g[f"rms_x_{n}"], g[f"rms_w_{n}"], 1e-6), g[f"rms_y_{n}"])
        assert np.array_equal(orc.softmax(g[f"sm_x_{n}"]), g[f"sm_y_{n}"])
        assert np.array_equal(orc.silu(g[f"rms_x_{n}"] * 4), g[f"silu_y_{n}"])
    for k in [k[len("rope_x_"):] for k in g if k.startswith("rope_x_")]:
        nh, hd, pos, base = g[f"rope_args_{k}"]
        y = orc.rope(g[f"rope_x_{k}"], int(nh), int(hd), int(pos), float(base))
        assert np.array_equal(y, g[f"rope_y_{k}"])


@pytest.mark.parametrize("kind,seed", [("qwen2", 7), ("llama-q4_0", 8)])
def test_model_restatement_bit_exact_vs_golden(orc, golden, gguf_dir, kind, seed):
    g = golden(f"model_{kind}")
    spec = synth.tiny_spec(kind)
    path = synth.write_gguf(spec, seed, gguf_dir / f"{spec.name}-{seed}.gguf")
    assert hashlib.sha256(path.read_bytes()).hexdigest() == str(g["sha256"]), "synthetic GGUF generator drifted"
    m = O.OracleModel(path, orc)
    pos = 0
    for t in g["prompt"]:
        l = m.forward(int(t), pos)
        pos += 1
    assert np.array_equal(l, g["logits"][0])
    for i, nxt in enumerate(g["ids"]):
        assert orc.argmax(l) == nxt
        l = m.forward(int(nxt), pos)
        pos += 1
        assert np.array_equal(l, g["logits"][i + 1])


def test_argmax_first_max(orc):
    x = np.array([1.0, 3.0, 2.0, 3.0], dtype=np.float32)
    assert orc.argmax(x) == 1


# ---- against the reference build itself (present where it was compiled) ----

@pytest.mark.parametrize("t", [O.Q4_0, O.Q8_0, O.Q6_K])
def test_dequant_random_vs_reference(orc, ref, t):
    rng = np.random.default_rng(31 + t)
    be, bb = {O.Q4_0: (32, 18), O.Q8_0: (32, 34), O.Q6_K: (256, 210)}[t]
    raw = rng.integers(0, 256, size=bb * 50, dtype=np.uint8)
    n = 50 * be
    a, b = orc.dequantize(t, raw, n), ref.dequantize(t, raw, n)
    assert np.array_equal(a.view(np.uint32), b.view(np.uint32))  # NaN payloads included


@pytest.mark.parametrize("t,rows,cols", [(O.Q4_0, 97, 4096), (O.Q8_0, 33, 896), (O.Q6_K, 17, 2048),
                                         (O.F32, 9, 100)])
def test_matmul_random_vs_reference(orc, ref, t, rows, cols):
    rng = np.random.default_rng(41)
    w = (rng.standard_normal(rows * cols) * 0.02).astype(np.float32)
    W = synth.quantize(t, w) if t != O.F32 else w.view(np.uint8)
    x = rng.standard_normal(cols).astype(np.float32)
    a = orc.matmul_quantized(W, t, x, rows, cols)
    b = ref.matmul_quantized(W, t, x, rows, cols)
    assert np.array_equal(a.view(np.uint32), b.view(np.uint32))


# rows of whole blocks only: trailing columns ignored, no whole block -> 0
PARTIAL_SHAPES = [(O.Q8_0, 5, 40), (O.Q4_0, 6, 70), (O.Q6_K, 3, 300), (O.Q8_0, 4, 20), (O.Q4_0, 2, 0),
                  (O.F32, 3, 0), (O.F32, 4, 1), (O.F32, 7, 45)]


def partial_case(t, rows, cols, seed=43):
    rng = np.random.default_rng(seed)
    ce = cols if t == O.F32 else cols // (256 if t == O.Q6_K else 32) * (256 if t == O.Q6_K else 32)
    w = (rng.standard_normal(rows * ce) * 0.02).astype(np.float32)
    W = (synth.quantize(t, w) if t != O.F32 else w.view(np.uint8)) if ce else np.zeros(1, np.uint8)
    x = rng.standard_normal(max(cols, 1)).astype(np.float32)
    return W, x


@pytest.mark.parametrize("t,rows,cols", PARTIAL_SHAPES)
def test_matmul_partial_blocks_vs_reference(orc, ref, t, rows, cols):
    W, x = partial_case(t, rows, cols)
    a = orc.matmul_quantized(W, t, x, rows, cols)
    b = ref.matmul_quantized(W, t, x, rows, cols)
    assert np.array_equal(a.view(np.uint32), b.view(np.uint32))


def test_model_llama_kq_restatement_runs(orc, gguf_dir):
    """Q4_K/Q6_K model: the reference cannot run it (no Q4_K); the
    restatement must at least be self-consistent across cache truncation."""
    spec = synth.tiny_spec("llama-kq")
    p = synth.write_gguf(spec, 9, gguf_dir / "kq.gguf")
    m = O.OracleModel(p, orc)
    toks = [3, 17, 200, 5, 9]
    outs = [m.forward(t, i) for i, t in enumerate(toks)]
    m.truncate_cache(2)
    again = [m.forward(t, i) for i, t in enumerate(toks[2:], start=2)]
    for a, b in zip(outs[2:], again):
        assert np.array_equal(a, b)
    assert np.isfinite(outs[-1]).all()


def test_mt19937_matches_reference_temperature_sampler(golden):
    """The host-drawn uniform (std::mt19937 + uniform_real_distribution<float>)
    that feeds stochastic sampling reproduces the reference sampler's choices."""
    g = golden("samplers")
    k, p, temp, seed = g["args_1"]
    rng = O.MT19937(int(seed))
    got = []
    for l in g["logits"]:
        m = l.max()
        e = np.exp((l - m) / np.float32(temp)).astype(np.float32)
        s = np.float32(0)
        for v in e:
            s = np.float32(s + v)
        probs = (e / s).astype(np.float32)
        r = np.float32(rng.uniform01())
        c = np.float32(0)
        pick = len(l) - 1
        for i, v in enumerate(probs):
            c = np.float32(c + v)
            if r <= c:
                pick = i
                break
        got.append(pick)
    assert got == list(g["ids_1"])
