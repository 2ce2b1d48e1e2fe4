"""Generate the golden fixtures in this directory from the reference itself.

    make -C oracle            # builds oracle/_ref/libsmallm_ref.so from the reference sources
    python tests/golden/make_golden.py

Every expected output here comes from the smallm-engine reference compiled
from its unmodified sources (oracle/_ref/libsmallm_ref.so), except Q4_K,
which the reference does not implement: its expected dequantization comes
from gguf-py 0.19.0 (gguf.quants.dequantize), the published GGUF Q4_K
definition.  Inputs are seeded, and synthetic GGUF files are identified by
their SHA-256 so a test can tell if the generator drifted.
"""
from __future__ import annotations

import hashlib
import sys
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parents[2]
sys.path.insert(0, str(ROOT))
sys.path.insert(0, str(ROOT / "oracle"))

import oracle as O  # noqa: E402
from smallm_engine_b200 import synth  # noqa: E402

OUT = Path(__file__).resolve().parent


def random_blocks(rng, t, nblocks):
    """Random block bytes of type t with finite, moderate f16 scales."""
    be, bb = synth.BLOCK[t]
    raw = rng.integers(0, 256, size=nblocks * bb, dtype=np.uint8)
    for i in range(nblocks):
        o = i * bb
        if t in (synth.Q4_0, synth.Q8_0):
            raw[o:o + 2] = np.frombuffer(np.float16(rng.uniform(-0.05, 0.05)).tobytes(), np.uint8)
        elif t == synth.Q6_K:
            raw[o + 208:o + 210] = np.frombuffer(np.float16(rng.uniform(-0.01, 0.01)).tobytes(), np.uint8)
        elif t == synth.Q4_K:
            raw[o:o + 2] = np.frombuffer(np.float16(rng.uniform(0, 0.01)).tobytes(), np.uint8)
            raw[o + 2:o + 4] = np.frombuffer(np.float16(rng.uniform(0, 0.01)).tobytes(), np.uint8)
    return raw


def f16_fixture(ref):
    codes = np.arange(65536, dtype=np.uint32)
    bits = np.array([ref.f16_to_f32(int(c)) for c in codes], dtype=np.float32).view(np.uint32)
    pick = np.unique(np.concatenate([np.arange(0, 1100), np.arange(0x7BF0, 0x7E10), np.arange(0x8000, 0x8410),
                                     np.arange(0xFBF0, 0x10000), np.random.default_rng(11).integers(0, 65536, 600)]))
    np.savez_compressed(OUT / "f16.npz", sha256=hashlib.sha256(bits.tobytes()).hexdigest(),
                        codes=pick.astype(np.uint32), bits=bits[pick])


def dequant_fixture(ref):
    import gguf
    rng = np.random.default_rng(20)
    d = {}
    for t, nb in [(synth.Q4_0, 64), (synth.Q8_0, 64), (synth.Q6_K, 12)]:
        raw = random_blocks(rng, t, nb)
        n = nb * synth.BLOCK[t][0]
        d[f"raw_{t}"] = raw
        d[f"out_{t}"] = ref.dequantize(t, raw, n)
    raw = random_blocks(rng, synth.Q4_K, 12)
    d[f"raw_{synth.Q4_K}"] = raw
    d[f"out_{synth.Q4_K}"] = gguf.quants.dequantize(raw.reshape(12, 144), gguf.GGMLQuantizationType.Q4_K).ravel()
    np.savez_compressed(OUT / "dequant.npz", **d)


def matmul_fixture(ref):
    import gguf
    rng = np.random.default_rng(21)
    d = {}
    shapes = {synth.F32: (40, 96), synth.Q4_0: (72, 512), synth.Q8_0: (72, 512), synth.Q6_K: (40, 1024),
              synth.Q4_K: (40, 1024)}
    for t, (rows, cols) in shapes.items():
        w = (rng.standard_normal(rows * cols) * 0.02).astype(np.float32)
        W = synth.quantize(t, w) if t != synth.F32 else w.view(np.uint8)
        x = rng.standard_normal(cols).astype(np.float32)
        d[f"W_{t}"] = W
        d[f"x_{t}"] = x
        d[f"shape_{t}"] = np.array([rows, cols])
        if t == synth.Q4_K:
            wd = gguf.quants.dequantize(W.reshape(-1, 144), gguf.GGMLQuantizationType.Q4_K).reshape(rows, cols)
            d[f"y_{t}"] = (wd.astype(np.float64) @ x.astype(np.float64)).astype(np.float32)
        else:
            d[f"y_{t}"] = ref.matmul_quantized(W, t, x, rows, cols)
    np.savez_compressed(OUT / "matmul.npz", **d)


def ops_fixture(ref):
    rng = np.random.default_rng(22)
    d = {}
    for n in (1, 7, 64, 896, 4096):
        x = rng.standard_normal(n).astype(np.float32)
        w = rng.standard_normal(n).astype(np.float32)
        d[f"rms_x_{n}"], d[f"rms_w_{n}"] = x, w
        d[f"rms_y_{n}"] = ref.rmsnorm(x, w, 1e-6)
        d[f"sm_x_{n}"] = x * 3
        d[f"sm_y_{n}"] = ref.softmax(x * 3)
        d[f"silu_y_{n}"] = ref.silu(x * 4)
    for (nh, hd, pos, base) in [(14, 64, 0, 1e6), (2, 64, 159, 1e6), (32, 128, 383, 5e5), (4, 64, 2303, 1e4)]:
        x = rng.standard_normal(nh * hd).astype(np.float32)
        key = f"{nh}_{hd}_{pos}"
        d[f"rope_x_{key}"] = x
        d[f"rope_y_{key}"] = ref.rope(x, nh, hd, pos, base)
        d[f"rope_args_{key}"] = np.array([nh, hd, pos, base], dtype=np.float64)
    np.savez_compressed(OUT / "ops.npz", **d)


def model_fixture(ref, kind, seed, n_prompt=8, n_steps=24):
    spec = synth.tiny_spec(kind)
    path = synth.write_gguf(spec, seed, Path("/tmp/smallm_golden") / f"{spec.name}-s{seed}.gguf")
    sha = hashlib.sha256(path.read_bytes()).hexdigest()
    m = ref.load(path)
    rng = np.random.default_rng(seed + 100)
    prompt = rng.integers(0, spec.vocab, size=n_prompt).astype(np.uint32)
    logits = []
    pos = 0
    for t in prompt:
        l = m.forward(int(t), pos)
        pos += 1
    logits.append(l)
    ids = []
    for _ in range(n_steps):
        nxt = int(np.argmax(l))
        ids.append(nxt)
        l = m.forward(nxt, pos)
        pos += 1
        logits.append(l)
    np.savez_compressed(OUT / f"model_{kind}.npz", sha256=sha, seed=seed, prompt=prompt,
                        ids=np.array(ids, dtype=np.uint32), logits=np.stack(logits))


def sampler_fixture(ref):
    rng = np.random.default_rng(23)
    logits = (rng.standard_normal((6, 1000)) * 3).astype(np.float32)
    d = {"logits": logits}
    for kind, k, p, temp, seed in [(1, 0, 0.0, 0.8, 5), (2, 40, 0.0, 1.0, 6), (3, 0, 0.9, 0.7, 7), (0, 0, 0, 1, 0)]:
        s = ref.sampler(kind, k, p, temp, seed)
        d[f"ids_{kind}"] = np.array([s.sample(l) for l in logits], dtype=np.uint32)
        d[f"args_{kind}"] = np.array([k, p, temp, seed], dtype=np.float64)
    # raw mt19937 stream and its uniform_real_distribution<float> for seed 5
    np.savez_compressed(OUT / "samplers.npz", **d)


def main():
    ref = O.Reference()
    f16_fixture(ref)
    dequant_fixture(ref)
    matmul_fixture(ref)
    ops_fixture(ref)
    model_fixture(ref, "qwen2", 7)
    model_fixture(ref, "llama-q4_0", 8)
    sampler_fixture(ref)
    for p in sorted(OUT.glob("*.npz")):
        print(f"{p.name}: {p.stat().st_size} bytes")


if __name__ == "__main__":
    main()
