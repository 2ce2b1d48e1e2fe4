"""Device-resident Qwen2/Llama models behind the reference's ``Model``
contract (include/smallm/model/common/model.h:16-43), the samplers
(src/runtime/sampler/*.cpp) and the ``Generator`` loop
(src/runtime/generator.cpp:22-72).

``CudaModel(path)`` plays the role of ``Qwen2Model(load_gguf(path))`` /
``LlamaModel(...)``: ``forward(token, pos)`` returns the vocab logits,
``reset_cache``/``truncate_cache``/``cached_length`` keep the reference's
prefix-reuse bookkeeping.  ``decode_greedy`` runs many steps entirely on the
GPU (argmax feeds the next step) for throughput.
"""
from __future__ import annotations

import ctypes
import math
from dataclasses import dataclass

import numpy as np

from ._lib import ModelInfo, ModelOpts, check, lib


@dataclass
class ModelConfig:
    """Fields of smallm::ModelConfig (src/config/common/config.h:15-46)."""
    architecture: str
    n_layers: int
    embd_dim: int
    ffn_dim: int
    n_heads: int
    n_kv_heads: int
    vocab_size: int
    context_length: int
    rope_freq_base: float
    rms_eps: float
    head_dim: int
    max_ctx: int
    weight_bytes_per_token: int
    device_bytes: int
    step_launches: int = 0


class CudaModel:
    def __init__(self, path, device: int = 0, max_ctx: int = 0, tp_rank: int = 0, tp_size: int = 1,
                 nccl_id: bytes | None = None):
        opts = ModelOpts(device, max_ctx, tp_rank, tp_size, None, 0)
        self.tp_size = tp_size
        self._id = None
        if nccl_id is not None:
            self._id = ctypes.create_string_buffer(bytes(nccl_id), 128)
            opts.nccl_id = ctypes.cast(self._id, ctypes.c_void_p)
        h = ctypes.c_void_p()
        check(lib().smallm_model_load(str(path).encode(), ctypes.byref(opts), ctypes.byref(h)))
        self.h = h
        info = ModelInfo()
        check(lib().smallm_model_get_info(self.h, ctypes.byref(info)))
        self._config = ModelConfig(info.arch.decode(), info.n_layers, info.embd, info.ffn, info.n_heads,
                                   info.n_kv_heads, info.vocab, info.context_length, info.rope_freq_base,
                                   info.rms_eps, info.head_dim, info.max_ctx, info.weight_bytes_per_token,
                                   info.device_bytes, info.step_launches)
        self._logits = np.empty(self._config.vocab_size, dtype=np.float32)

    def config(self) -> ModelConfig:
        return self._config

    @property
    def stream(self) -> int:
        return lib().smallm_model_stream(self.h) or 0

    # ---- Model (model.h:22-34) ----
    def forward(self, token_id: int, pos: int, want_logits: bool = True) -> np.ndarray | None:
        out = np.empty(self._config.vocab_size, dtype=np.float32) if want_logits else None
        check(lib().smallm_model_forward(self.h, int(token_id), int(pos),
                                         out.ctypes.data if want_logits else None, None))
        return out

    def forward_into(self, token_id: int, pos: int, logits_ptr: int | None) -> int:
        """forward() writing logits to a caller buffer (e.g. pinned memory);
        returns the greedy argmax."""
        am = ctypes.c_uint32()
        check(lib().smallm_model_forward(self.h, int(token_id), int(pos), logits_ptr, ctypes.byref(am)))
        return am.value

    def reset_cache(self):
        check(lib().smallm_model_reset_cache(self.h))

    def truncate_cache(self, n: int):
        check(lib().smallm_model_truncate_cache(self.h, int(n)))

    def cached_length(self) -> int:
        return int(lib().smallm_model_cached_length(self.h))

    # ---- device-side decode ----
    def decode_greedy_async(self, token: int, pos: int, n_steps: int):
        check(lib().smallm_model_decode_greedy_async(self.h, int(token), int(pos), int(n_steps)))

    def decode_ids(self, n: int) -> np.ndarray:
        ids = np.empty(n, dtype=np.uint32)
        check(lib().smallm_model_decode_ids(self.h, ids.ctypes.data, n))
        return ids

    def decode_greedy(self, token: int, pos: int, n_steps: int) -> np.ndarray:
        self.decode_greedy_async(token, pos, n_steps)
        return self.decode_ids(n_steps)

    def prefill(self, tokens, start_pos: int, want_logits: bool = True):
        """Batched prefill (smallm_model_prefill): tokens at positions
        start_pos.. in one pass per layer, the GEMMs on the backend's tcgen05
        tensor-core kernel over f16 weight copies.  Returns (last logits or
        None, greedy id of the last token)."""
        toks = np.ascontiguousarray(tokens, dtype=np.uint32)
        out = np.empty(self._config.vocab_size, dtype=np.float32) if want_logits else None
        am = ctypes.c_uint32()
        check(lib().smallm_model_prefill(self.h, toks.ctypes.data, toks.size, int(start_pos),
                                         out.ctypes.data if want_logits else None, ctypes.byref(am), 0))
        return out, int(am.value)

    def logits_device_ptr(self) -> int:
        return lib().smallm_model_logits_device(self.h) or 0

    TRACE_KINDS = {1: "embed", 2: "qkv", 3: "v", 4: "attention", 5: "o", 6: "gate_up", 7: "down",
                   8: "lm_head", 9: "finalize", 1000: "piece", 1001: "piece_done"}

    def trace_step(self, token: int, pos: int) -> list[dict]:
        """One step with GPU timestamps per kernel (ns from the step start)."""
        cap = 16 + 6 * self._config.n_layers + 2 * 8192  # persistent step: ops, then CTA 0's pieces
        buf = np.zeros(4 * cap, dtype=np.uint64)
        n = ctypes.c_uint32()
        check(lib().smallm_model_trace_step(self.h, int(token), int(pos), buf.ctypes.data, cap, ctypes.byref(n)))
        r = buf[:4 * min(n.value, cap)].reshape(-1, 4)
        return [{"kind": self.TRACE_KINDS.get(int(k), str(int(k))), "start": int(s), "ready": int(rd),
                 "end": int(e)} for s, rd, e, k in r]

    def close(self):
        if getattr(self, "h", None):
            lib().smallm_model_free(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


# ------------------------------------------------------------- samplers --

class MT19937:
    """std::mt19937 seeded with one integer (numpy's legacy MT19937 seeding is
    the same init_genrand)."""

    def __init__(self, seed: int):
        self.bg = np.random.MT19937(0)
        self.bg._legacy_seeding(int(seed) & 0xFFFFFFFF)

    def uniform01(self) -> float:
        """std::uniform_real_distribution<float>(0,1)(mt19937) under libstdc++:
        one 32-bit draw / 2^32 in float, 1.0 clamped to the float below."""
        r = np.float32(int(self.bg.random_raw())) / np.float32(4294967296.0)
        if r >= np.float32(1.0):
            r = np.nextafter(np.float32(1.0), np.float32(0.0))
        return float(r)


class _DeviceSampler:
    """A reference sampler (src/runtime/sampler/*.cpp) whose arithmetic runs on
    the GPU (csrc/sampler.cu) and whose random stream is the reference's: one
    std::uniform_real_distribution<float>(0, 1) draw from its std::mt19937 per
    sample, made here on the host."""
    KIND = 0
    DRAWS = True

    def __init__(self, k: int = 0, p: float = 0.0, temperature: float = 1.0, seed: int = 0, device: int = 0):
        self.k, self.p, self.temperature = int(k), float(p), float(temperature)
        self.rng = MT19937(seed)
        self.device = device
        self._ctx = None

    def _u(self) -> float:
        return self.rng.uniform01() if self.DRAWS else 0.0

    def sample(self, logits: np.ndarray) -> int:
        """Sampler::sample(const std::vector<float>& logits) on host logits."""
        if self._ctx is None:
            h = ctypes.c_void_p()
            check(lib().smallm_ctx_create(self.device, ctypes.byref(h)))
            self._ctx = h
        logits = np.ascontiguousarray(logits, dtype=np.float32)
        tok = ctypes.c_uint32()
        check(lib().smallm_sample(self._ctx, logits.ctypes.data, logits.size, self.KIND, self.k, self.p,
                                  self.temperature, self._u(), ctypes.byref(tok)))
        return int(tok.value)

    def sample_model(self, model: "CudaModel") -> int:
        """The same on the model's last logits, which stay on the device."""
        tok = ctypes.c_uint32()
        check(lib().smallm_model_sample(model.h, self.KIND, self.k, self.p, self.temperature, self._u(),
                                        ctypes.byref(tok)))
        return int(tok.value)

    def __del__(self):
        if getattr(self, "_ctx", None):
            try:
                lib().smallm_ctx_destroy(self._ctx)
            except Exception:
                pass
            self._ctx = None


class GreedySampler(_DeviceSampler):
    """src/runtime/sampler/greedy_sampler.cpp:8-14: the first index of the
    maximum, no random draw."""
    KIND, DRAWS = 0, False

    def __init__(self, device: int = 0):
        super().__init__(device=device)


class TemperatureSampler(_DeviceSampler):
    """src/runtime/sampler/temperature_sampler.cpp: softmax(logits / T), then
    the first index whose cumulative probability reaches the draw."""
    KIND = 1

    def __init__(self, temperature: float, seed: int, device: int = 0):
        super().__init__(temperature=temperature, seed=seed, device=device)


class TopKSampler(_DeviceSampler):
    """src/runtime/sampler/top_k_sampler.cpp: the k largest logits only."""
    KIND = 2

    def __init__(self, k: int, temperature: float, seed: int, device: int = 0):
        super().__init__(k=k, temperature=temperature, seed=seed, device=device)


class TopPSampler(_DeviceSampler):
    """src/runtime/sampler/top_p_sampler.cpp: the smallest prefix of the sorted
    distribution whose mass reaches p, the draw scaled by that mass."""
    KIND = 3

    def __init__(self, p: float, temperature: float, seed: int, device: int = 0):
        super().__init__(p=p, temperature=temperature, seed=seed, device=device)


def _seq_sum(a: np.ndarray) -> float:
    """Left-to-right f32 sum, the order of the reference's loops."""
    return float(np.cumsum(a, dtype=np.float32)[-1]) if a.size else 0.0


# ------------------------------------------------------------- generator --

@dataclass
class GenerationStats:
    """include/smallm/runtime/generation_stats.h:12-28."""
    prompt_tokens: int = 0
    reused_tokens: int = 0
    prefill_tokens: int = 0
    generated_tokens: int = 0
    prefill_ms: float = 0.0
    decode_ms: float = 0.0

    def prefill_tokens_per_sec(self) -> float:
        return self.prefill_tokens / (self.prefill_ms / 1000.0) if self.prefill_ms > 0 else 0.0

    def decode_tokens_per_sec(self) -> float:
        return self.generated_tokens / (self.decode_ms / 1000.0) if self.decode_ms > 0 else 0.0


class Generator:
    """src/runtime/generator.cpp:22-72 over token ids (tokenisation is outside
    this backend): prefix reuse against the previous call, one forward per
    new prompt token, then sample / forward until max_new or EOS."""

    def __init__(self, model: CudaModel, sampler, eos_id: int = -1, batched_prefill: bool = True):
        self.model, self.sampler, self.eos = model, sampler, eos_id
        # the prompt in one pass per layer (smallm_model_prefill) instead of
        # one forward per token; single GPU only
        self.batched_prefill = batched_prefill and model.config().n_layers > 0
        self.cached_tokens: list[int] = []
        self.stats = GenerationStats()

    def generate(self, prompt: list[int], max_new_tokens: int) -> list[int]:
        import time
        self.stats = GenerationStats()
        tokens = [int(t) for t in prompt]
        if not tokens:
            return []
        self.stats.prompt_tokens = len(tokens)
        shared = 0
        while shared < min(len(tokens), len(self.cached_tokens)) and tokens[shared] == self.cached_tokens[shared]:
            shared += 1
        if shared >= len(tokens):
            shared = len(tokens) - 1
        self.stats.reused_tokens = shared
        self.model.truncate_cache(shared)
        pos = shared
        # samplers that run on the device read the model's logits in place
        on_device = hasattr(self.sampler, "sample_model")
        t0 = time.perf_counter()
        logits = None
        if self.batched_prefill and getattr(self.model, "tp_size", 1) == 1:
            logits, _ = self.model.prefill(tokens[shared:], pos, want_logits=not on_device)
            self.stats.prefill_tokens += len(tokens) - shared
            pos = len(tokens)
        else:
            for i in range(shared, len(tokens)):
                logits = self.model.forward(tokens[i], pos, want_logits=not on_device)
                pos += 1
                self.stats.prefill_tokens += 1
        self.stats.prefill_ms = (time.perf_counter() - t0) * 1e3
        out: list[int] = []
        generated = list(tokens)
        t0 = time.perf_counter()
        for _ in range(max_new_tokens):
            nxt = self.sampler.sample_model(self.model) if on_device else self.sampler.sample(logits)
            if self.eos >= 0 and nxt == self.eos:
                break
            out.append(nxt)
            generated.append(nxt)
            logits = self.model.forward(nxt, pos, want_logits=not on_device)
            pos += 1
            self.stats.generated_tokens += 1
        self.stats.decode_ms = (time.perf_counter() - t0) * 1e3
        self.cached_tokens = generated
        return out
