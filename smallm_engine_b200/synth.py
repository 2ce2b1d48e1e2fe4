"""Seeded synthetic GGUF models for the decode workloads.

There are no checkpoints or datasets on the machines this runs on, so every
model is random-init weights of the named architecture, written as a real
GGUF v3 file that both this backend and the reference engine load with
their own loaders.

Layout rules the reference needs (it has no fallbacks):
* ``<arch>.block_count`` etc. are stored as exactly ``uint32``
  (src/config/common/config.cpp:28-32 via meta_read.h:14-20);
* ``vocab_size`` is the length of ``tokenizer.ggml.tokens``
  (config.cpp:42-47), so a V-long token list is written;
* ``output.weight`` must exist (src/model/qwen2_model.cpp:42); for
  tied-embedding models it is a byte copy of ``token_embd.weight``;
* weights are ``[out, in]`` with GGUF dims fastest-first, i.e. dims
  ``(in, out)`` (include/smallm/core/gguf.h:49).

Values: matrices and biases ~ N(0, 0.02) from a counter-based generator keyed
by (seed, tensor name), quantized per tensor type; norms are 1.0.
"""
from __future__ import annotations

import ctypes
import hashlib
import os
import struct
from dataclasses import dataclass, field, replace
from pathlib import Path

import numpy as np

F32, F16, Q4_0, Q8_0, Q4_K, Q6_K = 0, 1, 2, 8, 12, 14
TYPE_NAMES = {F32: "F32", F16: "F16", Q4_0: "Q4_0", Q8_0: "Q8_0", Q4_K: "Q4_K", Q6_K: "Q6_K"}
BLOCK = {F32: (1, 4), Q4_0: (32, 18), Q8_0: (32, 34), Q4_K: (256, 144), Q6_K: (256, 210)}

ROLES = ("token_embd", "output", "attn_q", "attn_k", "attn_v", "attn_output",
         "ffn_gate", "ffn_up", "ffn_down")


def nbytes(type_: int, count: int) -> int:
    be, bb = BLOCK[type_]
    if count % be:
        raise ValueError(f"{count} elements is not a whole number of {TYPE_NAMES[type_]} blocks")
    return count // be * bb


@dataclass(frozen=True)
class ModelSpec:
    """Shape and quantization recipe of a synthetic Qwen2/Llama decoder."""
    name: str
    arch: str                      # "qwen2" or "llama"
    embd: int
    layers: int
    heads: int
    kv_heads: int
    ffn: int
    vocab: int
    ctx: int
    rope_base: float
    eps: float
    bias: bool                     # Qwen2 QKV biases
    tied: bool                     # output.weight = copy of token_embd.weight
    types: dict = field(default_factory=dict)   # role -> GGML type
    std: float = 0.02

    @property
    def head_dim(self) -> int:
        return self.embd // self.heads

    def type_of(self, role: str) -> int:
        return self.types.get(role, self.types.get("default", Q8_0))

    def tensors(self):
        """[(name, dims fastest-first, type, source)] in file order.
        source: ("normal", std) | ("ones",) | ("alias", name)."""
        hd = self.head_dim
        qd, kvd = self.heads * hd, self.kv_heads * hd
        out = [("token_embd.weight", (self.embd, self.vocab), self.type_of("token_embd"),
                ("normal", self.std)),
               ("output_norm.weight", (self.embd,), F32, ("ones",))]
        if self.tied:
            out.append(("output.weight", (self.embd, self.vocab), self.type_of("token_embd"),
                        ("alias", "token_embd.weight")))
        else:
            out.append(("output.weight", (self.embd, self.vocab), self.type_of("output"),
                        ("normal", self.std)))
        for i in range(self.layers):
            p = f"blk.{i}."
            out.append((p + "attn_norm.weight", (self.embd,), F32, ("ones",)))
            out.append((p + "attn_q.weight", (self.embd, qd), self.type_of("attn_q"), ("normal", self.std)))
            out.append((p + "attn_k.weight", (self.embd, kvd), self.type_of("attn_k"), ("normal", self.std)))
            out.append((p + "attn_v.weight", (self.embd, kvd), self.type_of("attn_v"), ("normal", self.std)))
            if self.bias:
                out.append((p + "attn_q.bias", (qd,), F32, ("normal", self.std)))
                out.append((p + "attn_k.bias", (kvd,), F32, ("normal", self.std)))
                out.append((p + "attn_v.bias", (kvd,), F32, ("normal", self.std)))
            out.append((p + "attn_output.weight", (qd, self.embd), self.type_of("attn_output"),
                        ("normal", self.std)))
            out.append((p + "ffn_norm.weight", (self.embd,), F32, ("ones",)))
            out.append((p + "ffn_gate.weight", (self.embd, self.ffn), self.type_of("ffn_gate"),
                        ("normal", self.std)))
            out.append((p + "ffn_up.weight", (self.embd, self.ffn), self.type_of("ffn_up"),
                        ("normal", self.std)))
            out.append((p + "ffn_down.weight", (self.ffn, self.embd), self.type_of("ffn_down"),
                        ("normal", self.std)))
        return out

    def weight_bytes_per_token(self) -> int:
        """Quantized bytes of every matrix one decode step reads: all linears
        plus lm_head in their GGUF size, plus one embedding row."""
        total = 0
        for name, dims, t, _ in self.tensors():
            n = int(np.prod(dims))
            if name == "token_embd.weight":
                total += nbytes(t, dims[0])
            elif len(dims) == 2:
                total += nbytes(t, n)
            else:
                total += 4 * n            # norms / biases (f32, read once)
        return total

    def kv_bytes_per_token(self, pos: int) -> int:
        """f32 KV bytes read at position `pos` (positions 0..pos) plus the
        K and V rows written."""
        kvd = self.kv_heads * self.head_dim
        return self.layers * 2 * kvd * 4 * (pos + 1) + self.layers * 2 * kvd * 4


# The decode workloads (seeded shapes of the named model families).
WORKLOADS = {
    "qwen2-0.5b-q8_0": ModelSpec("qwen2-0.5b-q8_0", "qwen2", 896, 24, 14, 2, 4864, 151936, 512,
                                 1e6, 1e-6, True, True, {"default": Q8_0}),
    "tinyllama-1.1b-q4_k": ModelSpec("tinyllama-1.1b-q4_k", "llama", 2048, 22, 32, 4, 5632, 32000,
                                     2304, 1e4, 1e-5, False, False,
                                     {"default": Q4_K, "attn_v": Q6_K, "ffn_down": Q6_K,
                                      "output": Q6_K}),
    "llama3-8b-q4_0": ModelSpec("llama3-8b-q4_0", "llama", 4096, 32, 32, 8, 14336, 128256, 512,
                                5e5, 1e-5, False, False,
                                {"default": Q4_0, "token_embd": Q8_0, "output": Q8_0}),
    "qwen2-1.5b-q8_0": ModelSpec("qwen2-1.5b-q8_0", "qwen2", 1536, 28, 12, 2, 8960, 151936, 1024,
                                 1e6, 1e-6, True, True, {"default": Q8_0}),
}
WORKLOAD_SEEDS = {"qwen2-0.5b-q8_0": 0, "tinyllama-1.1b-q4_k": 3, "llama3-8b-q4_0": 4,
                  "qwen2-1.5b-q8_0": 5}


def tiny_spec(kind: str, **over) -> ModelSpec:
    """Small models with the same structure, for tests that the CPU oracles
    finish in seconds."""
    base = {
        "qwen2": ModelSpec("tiny-qwen2", "qwen2", 128, 2, 4, 2, 256, 512, 64, 1e6, 1e-6, True, True,
                           {"default": Q8_0}),
        "llama-q4_0": ModelSpec("tiny-llama-q4_0", "llama", 256, 2, 4, 2, 512, 384, 64, 5e5, 1e-5,
                                False, False, {"default": Q4_0, "token_embd": Q8_0, "output": Q8_0}),
        "llama-kq": ModelSpec("tiny-llama-kq", "llama", 256, 2, 4, 1, 512, 320, 96, 1e4, 1e-5,
                              False, False, {"default": Q4_K, "attn_v": Q6_K, "ffn_down": Q6_K,
                                             "output": Q6_K}),
    }[kind]
    return replace(base, **over) if over else base


# ---------------------------------------------------------------- native --

_lib = None


def _synth_lib():
    global _lib
    if _lib is None:
        from . import build
        path = build.build_synth()
        lib = ctypes.CDLL(str(path))
        lib.synth_fill.argtypes = [ctypes.c_uint32, ctypes.c_uint64, ctypes.c_uint64,
                                   ctypes.c_float, ctypes.c_float, ctypes.c_void_p]
        lib.synth_fill.restype = ctypes.c_int
        lib.synth_quantize.argtypes = [ctypes.c_uint32, ctypes.c_void_p, ctypes.c_uint64,
                                       ctypes.c_void_p]
        lib.synth_quantize.restype = ctypes.c_int
        lib.synth_normals.argtypes = [ctypes.c_uint64, ctypes.c_uint64, ctypes.c_float,
                                      ctypes.c_float, ctypes.c_void_p]
        lib.synth_f32_to_f16.argtypes = [ctypes.c_float]
        lib.synth_f32_to_f16.restype = ctypes.c_uint16
        _lib = lib
    return _lib


def stream_key(seed: int, name: str) -> int:
    """64-bit generator key of one tensor: FNV-1a of the name mixed with the seed."""
    h = 0xCBF29CE484222325
    for b in name.encode():
        h = ((h ^ b) * 0x100000001B3) & 0xFFFFFFFFFFFFFFFF
    return h ^ ((seed * 0x9E3779B97F4A7C15 + 0x632BE59BD9B4E019) & 0xFFFFFFFFFFFFFFFF)


def normals(seed: int, name: str, count: int, std: float = 1.0, mean: float = 0.0) -> np.ndarray:
    out = np.empty(count, dtype=np.float32)
    _synth_lib().synth_normals(stream_key(seed, name), count, mean, std, out.ctypes.data)
    return out


def quantize(type_: int, x: np.ndarray) -> np.ndarray:
    """Quantize f32 values into GGUF blocks of `type_` (Q8_0/Q4_0 match gguf-py byte for byte)."""
    x = np.ascontiguousarray(x, dtype=np.float32).ravel()
    out = np.empty(nbytes(type_, x.size), dtype=np.uint8)
    if _synth_lib().synth_quantize(type_, x.ctypes.data, x.size, out.ctypes.data) != 0:
        raise ValueError("bad quantize arguments")
    return out


def fill(type_: int, seed: int, name: str, count: int, std: float) -> np.ndarray:
    out = np.empty(nbytes(type_, count), dtype=np.uint8)
    if _synth_lib().synth_fill(type_, stream_key(seed, name), count, 0.0, std,
                               out.ctypes.data) != 0:
        raise ValueError("bad fill arguments")
    return out


# ------------------------------------------------------------------ GGUF --

def _s(v: str) -> bytes:
    b = v.encode()
    return struct.pack("<Q", len(b)) + b


def _kv_u32(k, v):
    return _s(k) + struct.pack("<II", 4, v)


def _kv_f32(k, v):
    return _s(k) + struct.pack("<If", 6, v)


def _kv_str(k, v):
    return _s(k) + struct.pack("<I", 8) + _s(v)


def _kv_strs(k, vs):
    return _s(k) + struct.pack("<IIQ", 9, 8, len(vs)) + b"".join(_s(v) for v in vs)


ALIGN = 32


def write_gguf(spec: ModelSpec, seed: int, path: str | os.PathLike) -> Path:
    """Write `spec` with weights from `seed` to `path` (atomically)."""
    path = Path(path)
    a = spec.arch
    kv = [_kv_str("general.architecture", a),
          _kv_str("general.name", spec.name),
          _kv_u32("general.alignment", ALIGN),
          _kv_u32(f"{a}.block_count", spec.layers),
          _kv_u32(f"{a}.embedding_length", spec.embd),
          _kv_u32(f"{a}.feed_forward_length", spec.ffn),
          _kv_u32(f"{a}.attention.head_count", spec.heads),
          _kv_u32(f"{a}.attention.head_count_kv", spec.kv_heads),
          _kv_u32(f"{a}.context_length", spec.ctx),
          _kv_f32(f"{a}.rope.freq_base", spec.rope_base),
          _kv_f32(f"{a}.attention.layer_norm_rms_epsilon", spec.eps),
          _kv_str("tokenizer.ggml.model", "none"),
          _kv_strs("tokenizer.ggml.tokens", [f"<{i}>" for i in range(spec.vocab)])]
    tensors = spec.tensors()
    infos, offsets, off = [], [], 0
    for name, dims, t, _ in tensors:
        offsets.append(off)
        infos.append(_s(name) + struct.pack("<I", len(dims)) +
                     b"".join(struct.pack("<Q", d) for d in dims) + struct.pack("<IQ", t, off))
        off += nbytes(t, int(np.prod(dims)))
        off = (off + ALIGN - 1) // ALIGN * ALIGN
    head = b"GGUF" + struct.pack("<IQQ", 3, len(tensors), len(kv)) + b"".join(kv) + b"".join(infos)
    head += b"\0" * ((-len(head)) % ALIGN)
    tmp = path.with_name(path.name + f".tmp{os.getpid()}")
    path.parent.mkdir(parents=True, exist_ok=True)
    with open(tmp, "wb") as f:
        f.write(head)
        base = f.tell()
        for (name, dims, t, src), o in zip(tensors, offsets):
            n = int(np.prod(dims))
            if src[0] == "ones":
                data = np.ones(n, dtype=np.float32).view(np.uint8)
            elif src[0] == "alias":
                data = fill(t, seed, src[1], n, spec.std)
            else:
                data = fill(t, seed, name, n, src[1])
            f.seek(base + o)
            f.write(memoryview(data))
        end = base + off
        f.truncate(end)
    os.replace(tmp, path)
    return path


def default_cache_dir() -> Path:
    return Path(os.environ.get("SMALLM_GGUF_CACHE", "/tmp/smallm_gguf"))


def spec_digest(spec: ModelSpec, seed: int) -> str:
    return hashlib.sha1(repr((spec, seed, ALIGN, 1)).encode()).hexdigest()[:12]


def ensure_gguf(spec: ModelSpec | str, seed: int | None = None,
                cache_dir: str | os.PathLike | None = None) -> Path:
    """Path of the GGUF for (spec, seed), writing it once into the cache."""
    if isinstance(spec, str):
        if seed is None:
            seed = WORKLOAD_SEEDS[spec]
        spec = WORKLOADS[spec]
    if seed is None:
        seed = 0
    d = Path(cache_dir) if cache_dir is not None else default_cache_dir()
    p = d / f"{spec.name}-s{seed}-{spec_digest(spec, seed)}.gguf"
    if not p.exists():
        write_gguf(spec, seed, p)
    return p
