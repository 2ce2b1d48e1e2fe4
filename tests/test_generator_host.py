"""The host-side Generator mirror (smallm_engine_b200.Generator) against the
reference's own Generator (src/runtime/generator.cpp:22-72, compiled from its
sources), on CPU: both drive a CPU model of the same GGUF (the mirror the
oracle's restatement, the reference its own Qwen2Model / LlamaModel, whose
logits the restatement reproduces bit for bit), with first-maximum greedy
sampling.  Across a sequence of calls the generated ids and the statistics
(prompt, reused, prefilled and generated tokens) must be identical: a first
prompt, a prompt that extends the cached tokens, the same prompt again
(shared prefix capped at len - 1), an unrelated prompt, and an end-of-sequence
stop."""
import numpy as np
import pytest

import oracle as O
from smallm_engine_b200 import Generator, synth


class OracleAsModel:
    """The restatement behind the mirror's model interface."""

    def __init__(self, path, orc):
        self.m = O.OracleModel(path, orc)

    def config(self):
        return self

    @property
    def n_layers(self):
        return self.m.n_layers

    def forward(self, token, pos, want_logits=True):
        return self.m.forward(token, pos)

    def truncate_cache(self, n):
        self.m.truncate_cache(n)


class FirstMax:
    """greedy_sampler.cpp:8-14 on host logits."""

    def sample(self, logits):
        return int(np.argmax(logits))


def ours_stats(g):
    s = g.stats
    return {"prompt_tokens": s.prompt_tokens, "reused_tokens": s.reused_tokens,
            "prefill_tokens": s.prefill_tokens, "generated_tokens": s.generated_tokens}


@pytest.mark.parametrize("kind,seed", [("qwen2", 7), ("llama-q4_0", 8)])
def test_generator_mirror_matches_reference(ref, orc, gguf_dir, kind, seed):
    path = synth.write_gguf(synth.tiny_spec(kind), seed, gguf_dir / f"gen-{kind}.gguf")
    rm = ref.load(path)
    theirs = O.RefGenerator(ref, rm, ref.sampler(0))
    ours = Generator(OracleAsModel(path, orc), FirstMax(), batched_prefill=False)
    n = 6
    p1 = [5, 9, 200, 31, 7]
    a, sa = theirs.generate(p1, n)
    b = ours.generate(p1, n)
    assert b == a and ours_stats(ours) == sa
    assert sa["reused_tokens"] == 0 and sa["generated_tokens"] == n
    p2 = p1 + a[:2] + [11]          # extends the cached tokens
    a, sa = theirs.generate(p2, n)
    b = ours.generate(p2, n)
    assert b == a and ours_stats(ours) == sa
    assert sa["reused_tokens"] == len(p1) + 2
    a, sa = theirs.generate(p2, n)  # the same prompt: reuse capped at len - 1
    b = ours.generate(p2, n)
    assert b == a and ours_stats(ours) == sa
    assert sa["reused_tokens"] == len(p2) - 1 and sa["prefill_tokens"] == 1
    p3 = [3, 1, 4]                  # nothing shared
    a, sa = theirs.generate(p3, n)
    b = ours.generate(p3, n)
    assert b == a and ours_stats(ours) == sa
    assert sa["reused_tokens"] == 0


def test_generator_mirror_stops_at_eos_like_reference(ref, orc, gguf_dir):
    path = synth.write_gguf(synth.tiny_spec("llama-q4_0"), 8, gguf_dir / "gen-eos.gguf")
    p = [5, 9, 200, 31, 7]
    free, _ = O.RefGenerator(ref, ref.load(path), ref.sampler(0)).generate(p, 8)
    k = next((i for i in range(1, len(free)) if free[i] not in free[:i]), None)
    if k is None:
        pytest.skip("the greedy continuation repeats one token; no distinct stop id")
    eos = free[k]
    a, sa = O.RefGenerator(ref, ref.load(path), ref.sampler(0), eos=eos).generate(p, 8)
    ours = Generator(OracleAsModel(path, orc), FirstMax(), eos_id=eos, batched_prefill=False)
    b = ours.generate(p, 8)
    assert a == free[:k] and b == a and ours_stats(ours) == sa
