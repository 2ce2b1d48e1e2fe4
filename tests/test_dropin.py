"""The C++ adapters (include/smallm/backend/cuda_backend.h,
include/smallm/model/cuda_model.h) inside the reference engine: the
reference's own Generator, GreedySampler, GGUF loader and config reader
(unmodified sources, src/runtime/generator.cpp:22-72) drive CudaModel,
CPUBackend is compared with CUDABackend op by op, and the reference's own
Qwen2Model / LlamaModel run their forward pass on CUDABackend (the compat
driver, whose two model files see CPUBackend as CUDABackend through an
include shim).  The driver binaries (oracle/_ref/dropin_driver,
oracle/_ref/compat_driver) are built where the reference sources are present.

Generator semantics checked: the first prompt is prefilled token by token
and continued greedily; the second prompt shares a prefix with the cached
tokens, so the Generator truncates the cache to the shared length and
prefills only the rest (generator.cpp:33-51).  The ids must equal the
oracle's greedy continuation of each prompt from an empty cache."""
import subprocess

import numpy as np
import pytest

import oracle as O
from smallm_engine_b200 import synth


def _has_gpu():
    try:
        import torch
        return torch.cuda.is_available()
    except Exception:
        return False


@pytest.fixture(scope="module")
def compat():
    if O.reference_sources_present():
        return O.build_compat()
    if not O.COMPAT.exists():
        pytest.skip("compat driver not built (reference sources absent)")
    return O.COMPAT


@pytest.fixture(scope="module")
def driver():
    if O.reference_sources_present():
        return O.build_dropin()
    if not O.DROPIN.exists():
        pytest.skip("drop-in driver not built (reference sources absent)")
    return O.DROPIN


def run(driver, *args):
    return subprocess.run([str(driver), *map(str, args)], capture_output=True, text=True, timeout=600)


@pytest.mark.skipif(_has_gpu(), reason="checks the no-GPU failure mode")
def test_dropin_fails_loudly_without_gpu(driver, gguf_dir):
    path = synth.write_gguf(synth.tiny_spec("llama-q4_0"), 8, gguf_dir / "dropin-cpu.gguf")
    r = run(driver, "generate", path, 4, "5 9 200", "5 9 7")
    assert r.returncode == 2 and r.stderr.startswith("error: CudaModel:"), r.stderr
    r = run(driver, "ops", 1)
    assert r.returncode == 2 and r.stderr.startswith("error: CUDABackend:"), r.stderr


@pytest.mark.skipif(_has_gpu(), reason="checks the no-GPU failure mode")
def test_compat_model_code_constructs_cuda_backend(compat, gguf_dir, tmp_path):
    """The reference's Qwen2Model / LlamaModel, compiled against the compat
    shim, construct CUDABackend: without a GPU their constructor throws from
    it (the stock build would run on the CPU)."""
    for kind, seed in (("qwen2", 7), ("llama-q4_0", 8)):
        path = synth.write_gguf(synth.tiny_spec(kind), seed, gguf_dir / f"compat-cpu-{kind}.gguf")
        r = run(compat, path, 2, "5 9 200", tmp_path / "l.f32")
        assert r.returncode == 2 and r.stderr.startswith("error: CUDABackend:"), r.stderr


def greedy(path, orc, prompt, n):
    m = O.OracleModel(path, orc)
    logits = None
    for p, t in enumerate(prompt):
        logits = m.forward(t, p)
    out, pos = [], len(prompt)
    for _ in range(n):
        nxt = int(np.argmax(logits))
        out.append(nxt)
        logits = m.forward(nxt, pos)
        pos += 1
    return out


@pytest.mark.gpu
@pytest.mark.parametrize("kind,seed", [("qwen2", 7), ("llama-q4_0", 8)])
def test_reference_generator_drives_cuda_model(driver, orc, gguf_dir, kind, seed):
    path = synth.write_gguf(synth.tiny_spec(kind), seed, gguf_dir / f"dropin-{kind}.gguf")
    p1, p2, n = [5, 9, 200, 31, 7], [5, 9, 200, 77, 3, 11], 10
    r = run(driver, "generate", path, n, " ".join(map(str, p1)), " ".join(map(str, p2)))
    assert r.returncode == 0, r.stderr
    lines = [l.split() for l in r.stdout.splitlines() if l.startswith("ids ")]
    assert len(lines) == 2
    (_, reused1, pre1, *ids1), (_, reused2, pre2, *ids2) = lines
    assert (int(reused1), int(pre1)) == (0, len(p1))
    assert (int(reused2), int(pre2)) == (3, len(p2) - 3)  # shared prefix 5 9 200
    assert [int(i) for i in ids1] == greedy(path, orc, p1, n)
    assert [int(i) for i in ids2] == greedy(path, orc, p2, n)


@pytest.mark.gpu
@pytest.mark.parametrize("kind,seed", [("qwen2", 7), ("llama-q4_0", 8)])
def test_cuda_model_generate_greedy(driver, orc, gguf_dir, kind, seed):
    """CudaModel::generate_greedy: one-pass prefill (exact f32 GEMMs, flags 0)
    and device-chained greedy steps give the oracle's greedy continuation."""
    path = synth.write_gguf(synth.tiny_spec(kind), seed, gguf_dir / f"fastgen-{kind}.gguf")
    p, n = [5, 9, 200, 31, 7], 12
    r = run(driver, "fastgen", path, n, " ".join(map(str, p)), 0)
    assert r.returncode == 0, r.stderr
    line = [l.split() for l in r.stdout.splitlines() if l.startswith("fast")]
    assert len(line) == 1
    assert [int(i) for i in line[0][1:]] == greedy(path, orc, p, n)


@pytest.mark.gpu
@pytest.mark.parametrize("kind,seed", [("qwen2", 7), ("llama-q4_0", 8)])
def test_compat_reference_model_on_cuda_backend(compat, orc, gguf_dir, tmp_path, kind, seed):
    """The reference's own forward pass (qwen2_model.cpp / llama_model.cpp,
    unmodified) with every Backend call on the GPU: the last prompt token's
    logits within 1e-2 * max|logit| of the restatement and the greedy ids
    identical."""
    path = synth.write_gguf(synth.tiny_spec(kind), seed, gguf_dir / f"compat-{kind}.gguf")
    p, n = [5, 9, 200, 31, 7], 8
    out = tmp_path / "logits.f32"
    r = run(compat, path, n, " ".join(map(str, p)), out)
    assert r.returncode == 0, r.stderr
    got = np.fromfile(out, dtype=np.float32)
    ref = O.OracleModel(path, orc)
    want = None
    for pos, t in enumerate(p):
        want = ref.forward(t, pos)
    assert got.shape == want.shape
    assert np.abs(got.astype(np.float64) - want).max() <= 1e-2 * np.abs(want).max()
    line = [l.split() for l in r.stdout.splitlines() if l.startswith("ids")]
    assert [int(i) for i in line[0][1:]] == greedy(path, orc, p, n)


@pytest.mark.gpu
def test_cpu_backend_vs_cuda_backend(driver):
    r = run(driver, "ops", 3)
    assert r.returncode == 0, r.stderr
    ops = {l.split()[1]: l.split()[2:] for l in r.stdout.splitlines() if l.startswith("op ")}
    assert set(ops) == {"rmsnorm", "softmax", "silu", "rope", "matmul"}
    diff = {k: float(v[0]) for k, v in ops.items()}
    mag = {k: float(v[1]) for k, v in ops.items()}
    assert ops["rope"][2] == "1"                       # host table with the reference's arithmetic
    assert diff["rmsnorm"] <= 1e-5 * mag["rmsnorm"]
    assert diff["softmax"] <= 1e-5 * mag["softmax"]
    assert diff["silu"] <= 1e-5 * mag["silu"]
    assert diff["matmul"] <= 1e-4 * mag["matmul"]      # f32 sums of 1000 products, other order
