"""The persistent decode step (csrc/step.cu): the whole token step as one
cooperative kernel, for models whose layer matrices share one of the
32-element block formats (Q4_0, Q8_0); selected at load with
SMALLM_STEP=persistent.

Checked against the oracle's restatement of the reference's forward pass
(src/model/qwen2_model.cpp:163-198, src/model/llama_model.cpp:148-177) with
the model-level bar (logits within 1e-2 * max|logit| per step, observed far
inside it, and identical greedy ids), and against the per-op kernel path of
the same library on the same model (the default at load)."""
import os

import numpy as np
import pytest

import oracle as O
from smallm_engine_b200 import CudaModel, synth

pytestmark = pytest.mark.gpu


def _load(path, per_op: bool = False, **kw) -> CudaModel:
    if not per_op:
        os.environ["SMALLM_STEP"] = "persistent"
    try:
        return CudaModel(path, **kw)
    finally:
        os.environ.pop("SMALLM_STEP", None)


@pytest.mark.parametrize("kind,seed", [("qwen2", 21), ("llama-q4_0", 22)])
def test_tiny_models_persistent_step_vs_oracle(orc, gguf_dir, kind, seed):
    spec = synth.tiny_spec(kind)
    path = synth.write_gguf(spec, seed, gguf_dir / f"step-{kind}-{seed}.gguf")
    m = _load(path)
    assert m.config().step_launches == 1  # the persistent step runs this model
    ref = O.OracleModel(path, orc)
    rng = np.random.default_rng(seed)
    pos = 0
    for t in rng.integers(0, spec.vocab, size=5):
        a, b = m.forward(int(t), pos), ref.forward(int(t), pos)
        pos += 1
    worst = 0.0
    for step in range(24):
        err = float(np.abs(a.astype(np.float64) - b).max())
        worst = max(worst, err / float(np.abs(b).max()))
        assert err <= 1e-2 * float(np.abs(b).max()), f"step {step}"
        nxt = int(np.argmax(b))
        assert int(np.argmax(a)) == nxt, f"greedy id differs at step {step}"
        a, b = m.forward(nxt, pos), ref.forward(nxt, pos)
        pos += 1
    assert worst < 1e-4
    m.close()


@pytest.mark.parametrize("name", ["qwen2-0.5b-q8_0", "llama3-8b-q4_0"])
def test_real_shapes_persistent_vs_per_op_kernels(gguf_dir, name):
    """The workload shapes with 2 layers: the persistent step and the per-op
    kernels give the same greedy ids over 48 device-chained steps and logits
    that agree to f32 rounding; the device-chained ids equal the ids of
    step-by-step forward calls."""
    from dataclasses import replace
    spec = replace(synth.WORKLOADS[name], layers=2, name=name + "-2l-step", ctx=256)
    path = synth.write_gguf(spec, 31, gguf_dir / f"{name}-2l-step.gguf")
    ms = _load(path)
    mk = _load(path, per_op=True)
    assert ms.config().step_launches == 1 and mk.config().step_launches > 1
    rng = np.random.default_rng(3)
    prompt = rng.integers(0, spec.vocab, size=9)
    for pos, t in enumerate(prompt):
        a = ms.forward(int(t), pos)
        b = mk.forward(int(t), pos)
    scale = float(np.abs(b).max())
    assert float(np.abs(a - b).max()) <= 1e-4 * scale
    tok, pos = int(np.argmax(b)), len(prompt)
    ids_s = ms.decode_greedy(tok, pos, 48)
    ids_k = mk.decode_greedy(tok, pos, 48)
    assert np.array_equal(ids_s, ids_k)
    # the same steps one forward() at a time
    ms.truncate_cache(pos)
    t, ids_f = tok, []
    for i in range(48):
        t = ms.forward_into(t, pos + i, None)
        ids_f.append(t)
    assert np.array_equal(np.array(ids_f, np.uint32), ids_s)
    ms.close()
    mk.close()


def test_long_context_persistent_attention(orc, gguf_dir):
    """Positions up to ~700 on a 2-layer Llama-shaped Q4_0 model: the step's
    attention splits every KV head over many CTAs and merges their partials
    (atomic ticket); checked against the oracle at the last positions."""
    spec = synth.tiny_spec("llama-q4_0", ctx=768, name="tiny-llama-q4_0-768")
    path = synth.write_gguf(spec, 23, gguf_dir / "step-long.gguf")
    m = _load(path)
    assert m.config().step_launches == 1
    ref = O.OracleModel(path, orc)
    rng = np.random.default_rng(5)
    toks = rng.integers(0, spec.vocab, size=700)
    for pos, t in enumerate(toks):
        a = m.forward(int(t), pos, want_logits=pos >= 690)
        b = ref.forward(int(t), pos)
        if pos >= 690:
            assert float(np.abs(a - b).max()) <= 1e-3 * float(np.abs(b).max()), pos
            assert int(np.argmax(a)) == int(np.argmax(b))
    m.close()


@pytest.mark.parametrize("ctx,n_pos", [(768, 700), (8192, 3300)])
def test_long_context_cluster_attention(orc, gguf_dir, ctx, n_pos):
    """The per-op step's cluster attention sized for max_ctx (head_dim 64,
    2 KV heads, 16-CTA clusters).  At 768: one cluster per KV head, 64-position
    chunks, each CTA's range in one chunk copied before the dependency wait.
    At 8192: four clusters per KV head, each over a quarter of the positions,
    their normalised outputs merged by the O GEMV as it stages x; checked
    also at the first positions, where some parts are still empty.  Checked
    against the oracle."""
    spec = synth.tiny_spec("llama-q4_0", ctx=ctx, name=f"tiny-llama-q4_0-{ctx}")
    path = synth.write_gguf(spec, 24, gguf_dir / f"ring-{ctx}.gguf")
    m = _load(path, per_op=True)
    assert m.config().step_launches > 1  # the per-op kernels
    ref = O.OracleModel(path, orc)
    rng = np.random.default_rng(6)
    toks = rng.integers(0, spec.vocab, size=n_pos)
    for pos, t in enumerate(toks):
        last = pos >= n_pos - 6 or pos < 3
        a = m.forward(int(t), pos, want_logits=last)
        b = ref.forward(int(t), pos)
        if last:
            assert float(np.abs(a - b).max()) <= 1e-3 * float(np.abs(b).max()), pos
            assert int(np.argmax(a)) == int(np.argmax(b))
    m.close()
