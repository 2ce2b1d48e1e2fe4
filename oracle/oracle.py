"""CPU oracle for the smallm-engine decode path -- TEST INFRASTRUCTURE ONLY.

Only tests, the smoke check and the benchmark's CPU-baseline leg import this
module; the product never does.

Two checkers live here:

* ``Oracle``     -- the plain-C restatement (oracle.c, built into
                    oracle/_build/liboracle.so) plus a numpy/C restatement of
                    the Qwen2/Llama forward pass (``OracleModel``), following
                    src/model/qwen2_model.cpp:163-198 and
                    src/model/llama_model.cpp:148-177.  It also covers Q4_K,
                    which the reference lacks.
* ``Reference``  -- the reference engine itself, compiled from its unmodified
                    sources into oracle/_ref/libsmallm_ref.so (see Makefile),
                    driven through ref_harness.cpp.  Present wherever it was
                    built; the restatement is pinned against it.
"""
from __future__ import annotations

import ctypes
import os
import math
import struct
import subprocess
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
ORACLE_SO = HERE / "_build" / "liboracle.so"
REF_SO = HERE / "_ref" / "libsmallm_ref.so"

F32, F16, Q4_0, Q8_0, Q4_K, Q6_K = 0, 1, 2, 8, 12, 14
_BLOCK = {F32: (1, 4), F16: (1, 2), Q4_0: (32, 18), Q8_0: (32, 34), Q4_K: (256, 144), Q6_K: (256, 210)}

_fp = ctypes.POINTER(ctypes.c_float)


def _ptr(a: np.ndarray):
    return a.ctypes.data_as(ctypes.c_void_p)


def build(ref: bool = True) -> None:
    """make -C oracle (the reference part only where its sources exist)."""
    target = "all" if ref else "oracle"
    r = subprocess.run(["make", "-s", "-C", str(HERE), f"REF={REF_SRC}", target], capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError("oracle build failed:\n" + r.stdout + r.stderr)


DROPIN = HERE / "_ref" / "dropin_driver"


def build_dropin() -> Path:
    """make -C oracle dropin: the reference's sources + dropin_driver.cpp +
    the C++ adapters, linked against the already built CUDA backend."""
    r = subprocess.run(["make", "-s", "-C", str(HERE), f"REF={REF_SRC}", "dropin"], capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError("drop-in driver build failed:\n" + r.stdout + r.stderr)
    return DROPIN


COMPAT = HERE / "_ref" / "compat_driver"


def build_compat() -> Path:
    """make -C oracle compat: the reference's sources with its two model files
    compiled against compat/ (CPUBackend -> the CUDABackend adapter)."""
    r = subprocess.run(["make", "-s", "-C", str(HERE), f"REF={REF_SRC}", "compat"], capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError("compat driver build failed:\n" + r.stdout + r.stderr)
    return COMPAT


# Where the reference's sources are read from when its build (oracle/_ref) is
# made: $SMALLM_REF_SRC, by default the read-only checkout beside this repo.
REF_SRC = Path(os.environ.get("SMALLM_REF_SRC", "/root/reference"))


def reference_sources_present() -> bool:
    return (REF_SRC / "src" / "core" / "ops.cpp").exists()


def type_nbytes(t: int, count: int) -> int:
    be, bb = _BLOCK[t]
    return count // be * bb


class Oracle:
    """ctypes view of oracle/_build/liboracle.so."""

    def __init__(self):
        if not ORACLE_SO.exists():
            build(ref=False)
        L = ctypes.CDLL(str(ORACLE_SO))
        L.orc_f16_to_f32.argtypes = [ctypes.c_uint16]
        L.orc_f16_to_f32.restype = ctypes.c_float
        L.orc_dequantize.argtypes = [ctypes.c_uint32, ctypes.c_void_p, ctypes.c_uint64, ctypes.c_void_p]
        L.orc_matmul_quantized.argtypes = [ctypes.c_void_p, ctypes.c_uint32, ctypes.c_void_p,
                                           ctypes.c_uint32, ctypes.c_uint32, ctypes.c_void_p]
        L.orc_rmsnorm.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_uint32, ctypes.c_float,
                                  ctypes.c_void_p]
        L.orc_softmax.argtypes = [ctypes.c_void_p, ctypes.c_uint32]
        L.orc_silu.argtypes = [ctypes.c_void_p, ctypes.c_uint32]
        L.orc_rope.argtypes = [ctypes.c_void_p, ctypes.c_uint32, ctypes.c_uint32, ctypes.c_uint32,
                               ctypes.c_float]
        L.orc_dot.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_uint32]
        L.orc_dot.restype = ctypes.c_float
        L.orc_axpy.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_float, ctypes.c_uint32]
        L.orc_mul.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_uint32]
        L.orc_attention.argtypes = [ctypes.c_void_p] * 3 + [ctypes.c_uint32] * 4 + [ctypes.c_void_p] * 2
        L.orc_argmax.argtypes = [ctypes.c_void_p, ctypes.c_uint32]
        L.orc_argmax.restype = ctypes.c_uint32
        self.L = L

    def f16_to_f32(self, h: int) -> float:
        return self.L.orc_f16_to_f32(h)

    def dequantize(self, t: int, raw: np.ndarray, count: int) -> np.ndarray:
        out = np.empty(count, dtype=np.float32)
        raw = np.ascontiguousarray(raw, dtype=np.uint8)
        if self.L.orc_dequantize(t, _ptr(raw), count, _ptr(out)) != 0:
            raise ValueError(f"unsupported tensor type: {t}")
        return out

    def matmul_quantized(self, W: np.ndarray, t: int, x: np.ndarray, rows: int, cols: int) -> np.ndarray:
        y = np.empty(rows, dtype=np.float32)
        x = np.ascontiguousarray(x, dtype=np.float32)
        W = np.ascontiguousarray(W)
        if self.L.orc_matmul_quantized(_ptr(W), t, _ptr(x), rows, cols, _ptr(y)) != 0:
            raise ValueError(f"unsupported tensor type: {t}")
        return y

    def rmsnorm(self, x, w, eps):
        x = np.ascontiguousarray(x, np.float32)
        w = np.ascontiguousarray(w, np.float32)
        y = np.empty_like(x)
        self.L.orc_rmsnorm(_ptr(x), _ptr(w), x.size, eps, _ptr(y))
        return y

    def softmax(self, x):
        x = np.array(x, dtype=np.float32)
        self.L.orc_softmax(_ptr(x), x.size)
        return x

    def silu(self, x):
        x = np.array(x, dtype=np.float32)
        self.L.orc_silu(_ptr(x), x.size)
        return x

    def rope(self, x, n_heads, head_dim, pos, base):
        x = np.array(x, dtype=np.float32)
        self.L.orc_rope(_ptr(x), n_heads, head_dim, pos, base)
        return x

    def axpy(self, y, v, s):
        self.L.orc_axpy(_ptr(y), _ptr(np.ascontiguousarray(v, np.float32)), s, y.size)

    def mul(self, y, v):
        self.L.orc_mul(_ptr(y), _ptr(np.ascontiguousarray(v, np.float32)), y.size)

    def attention(self, q, kc, vc, n_head, n_kv, hd, pos):
        out = np.empty(n_head * hd, dtype=np.float32)
        scratch = np.empty(pos + 1, dtype=np.float32)
        self.L.orc_attention(_ptr(q), _ptr(kc), _ptr(vc), n_head, n_kv, hd, pos, _ptr(out), _ptr(scratch))
        return out

    def argmax(self, logits):
        logits = np.ascontiguousarray(logits, np.float32)
        return int(self.L.orc_argmax(_ptr(logits), logits.size))


class Reference:
    """ctypes view of the reference engine compiled from its own sources."""

    @staticmethod
    def available() -> bool:
        return REF_SO.exists()

    def __init__(self):
        if not REF_SO.exists():
            raise FileNotFoundError(f"{REF_SO} not built (needs the reference sources)")
        L = ctypes.CDLL(str(REF_SO))
        L.ref_last_error.restype = ctypes.c_char_p
        L.ref_f16_to_f32.argtypes = [ctypes.c_uint16]
        L.ref_f16_to_f32.restype = ctypes.c_float
        L.ref_matmul_quantized.argtypes = [ctypes.c_void_p, ctypes.c_uint32, ctypes.c_void_p,
                                           ctypes.c_uint32, ctypes.c_uint32, ctypes.c_void_p]
        L.ref_rmsnorm.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_uint32, ctypes.c_float,
                                  ctypes.c_void_p]
        L.ref_softmax.argtypes = [ctypes.c_void_p, ctypes.c_uint32]
        L.ref_silu.argtypes = [ctypes.c_void_p, ctypes.c_uint32]
        L.ref_rope.argtypes = [ctypes.c_void_p, ctypes.c_uint32, ctypes.c_uint32, ctypes.c_uint32,
                               ctypes.c_float]
        L.ref_dot.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_uint32]
        L.ref_dot.restype = ctypes.c_float
        L.ref_axpy.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_float, ctypes.c_uint32]
        L.ref_dequantize.argtypes = [ctypes.c_uint32, ctypes.c_void_p, ctypes.c_uint64, ctypes.c_void_p]
        L.ref_model_load.argtypes = [ctypes.c_char_p]
        L.ref_model_load.restype = ctypes.c_void_p
        L.ref_model_free.argtypes = [ctypes.c_void_p]
        L.ref_model_config.argtypes = [ctypes.c_void_p, ctypes.c_void_p]
        L.ref_model_forward.argtypes = [ctypes.c_void_p, ctypes.c_uint32, ctypes.c_uint32, ctypes.c_void_p]
        L.ref_model_reset.argtypes = [ctypes.c_void_p]
        L.ref_model_truncate.argtypes = [ctypes.c_void_p, ctypes.c_uint32]
        L.ref_model_cached_length.argtypes = [ctypes.c_void_p]
        L.ref_model_cached_length.restype = ctypes.c_uint32
        L.ref_sampler_new.argtypes = [ctypes.c_int, ctypes.c_uint32, ctypes.c_float, ctypes.c_float,
                                      ctypes.c_uint64]
        L.ref_sampler_new.restype = ctypes.c_void_p
        L.ref_sampler_free.argtypes = [ctypes.c_void_p]
        L.ref_sampler_sample.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_uint32, ctypes.c_void_p]
        L.ref_generator_new.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int32]
        L.ref_generator_new.restype = ctypes.c_void_p
        L.ref_generator_free.argtypes = [ctypes.c_void_p]
        L.ref_generate.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_uint32, ctypes.c_uint32,
                                   ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p]
        L.ref_decode_timed.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_uint32, ctypes.c_uint32,
                                       ctypes.c_uint32, ctypes.c_void_p, ctypes.c_void_p]
        self.L = L

    def _check(self, rc):
        if rc != 0:
            raise RuntimeError(self.L.ref_last_error().decode())

    def f16_to_f32(self, h):
        return self.L.ref_f16_to_f32(h)

    def matmul_quantized(self, W, t, x, rows, cols):
        y = np.empty(rows, dtype=np.float32)
        x = np.ascontiguousarray(x, np.float32)
        W = np.ascontiguousarray(W)
        self._check(self.L.ref_matmul_quantized(_ptr(W), t, _ptr(x), rows, cols, _ptr(y)))
        return y

    def dequantize(self, t, raw, count):
        out = np.empty(count, dtype=np.float32)
        raw = np.ascontiguousarray(raw, dtype=np.uint8)
        self._check(self.L.ref_dequantize(t, _ptr(raw), count, _ptr(out)))
        return out

    def rmsnorm(self, x, w, eps):
        x = np.ascontiguousarray(x, np.float32)
        y = np.empty_like(x)
        self._check(self.L.ref_rmsnorm(_ptr(x), _ptr(np.ascontiguousarray(w, np.float32)), x.size, eps, _ptr(y)))
        return y

    def softmax(self, x):
        x = np.array(x, dtype=np.float32)
        self._check(self.L.ref_softmax(_ptr(x), x.size))
        return x

    def silu(self, x):
        x = np.array(x, dtype=np.float32)
        self._check(self.L.ref_silu(_ptr(x), x.size))
        return x

    def rope(self, x, n_heads, head_dim, pos, base):
        x = np.array(x, dtype=np.float32)
        self._check(self.L.ref_rope(_ptr(x), n_heads, head_dim, pos, base))
        return x

    def load(self, path) -> "RefModel":
        return RefModel(self, path)

    def sampler(self, kind: int, k=0, p=0.0, temp=1.0, seed=0) -> "RefSampler":
        return RefSampler(self, kind, k, p, temp, seed)


class RefModel:
    def __init__(self, ref: Reference, path):
        self.ref = ref
        self.h = ref.L.ref_model_load(str(path).encode())
        if not self.h:
            raise RuntimeError(ref.L.ref_last_error().decode())
        c = np.zeros(10, dtype=np.uint32)
        ref._check(ref.L.ref_model_config(self.h, _ptr(c)))
        self.n_layers, self.embd, self.ffn, self.n_heads, self.n_kv, self.vocab, self.ctx, self.hd = map(int, c[:8])
        self.rope_base = float(c[8:9].view(np.float32)[0])
        self.eps = float(c[9:10].view(np.float32)[0])

    def forward(self, token: int, pos: int) -> np.ndarray:
        out = np.empty(self.vocab, dtype=np.float32)
        self.ref._check(self.ref.L.ref_model_forward(self.h, token, pos, _ptr(out)))
        return out

    def reset_cache(self):
        self.ref._check(self.ref.L.ref_model_reset(self.h))

    def truncate_cache(self, n):
        self.ref._check(self.ref.L.ref_model_truncate(self.h, n))

    def cached_length(self):
        return int(self.ref.L.ref_model_cached_length(self.h))

    def decode_timed(self, prompt, steps, warmup=0):
        """Prompt token by token, `warmup` untimed greedy steps, then `steps`
        timed ones: (all warmup + steps ids, ms of the timed steps)."""
        prompt = np.ascontiguousarray(prompt, np.uint32)
        ids = np.empty(warmup + steps, dtype=np.uint32)
        ms = ctypes.c_double()
        self.ref._check(self.ref.L.ref_decode_timed(self.h, _ptr(prompt), prompt.size, warmup, steps, _ptr(ids),
                                                    ctypes.byref(ms)))
        return ids, ms.value

    def __del__(self):
        if getattr(self, "h", None):
            self.ref.L.ref_model_free(self.h)
            self.h = None


class RefGenerator:
    """The reference's own smallm::Generator (src/runtime/generator.cpp:22-72)
    over `model` and `sampler`, with the harness's id tokenizer (prompt and
    output are token ids; `eos` < 0 disables the stop)."""

    def __init__(self, ref: Reference, model: "RefModel", sampler: "RefSampler", eos: int = -1):
        self.ref = ref
        self.h = ref.L.ref_generator_new(model.h, sampler.h, eos)
        if not self.h:
            raise RuntimeError(ref.L.ref_last_error().decode())
        self._keep = (model, sampler)

    def generate(self, prompt, max_new: int):
        """(generated ids, stats dict) of one Generator::generate call."""
        p = np.ascontiguousarray(prompt, dtype=np.uint32)
        out = np.zeros(max_new + 1, dtype=np.uint32)
        n = np.zeros(1, dtype=np.uint32)
        st = np.zeros(6, dtype=np.float64)
        self.ref._check(self.ref.L.ref_generate(self.h, _ptr(p), p.size, max_new, _ptr(out), _ptr(n), _ptr(st)))
        keys = ("prompt_tokens", "reused_tokens", "prefill_tokens", "generated_tokens")
        return [int(i) for i in out[:int(n[0])]], {k: int(v) for k, v in zip(keys, st[:4])}

    def __del__(self):
        try:
            if self.h:
                self.ref.L.ref_generator_free(self.h)
        except Exception:
            pass


class RefSampler:
    def __init__(self, ref, kind, k, p, temp, seed):
        self.ref = ref
        self.h = ref.L.ref_sampler_new(kind, k, p, temp, seed)

    def sample(self, logits) -> int:
        logits = np.ascontiguousarray(logits, np.float32)
        out = ctypes.c_uint32()
        self.ref._check(self.ref.L.ref_sampler_sample(self.h, _ptr(logits), logits.size, ctypes.byref(out)))
        return int(out.value)

    def __del__(self):
        if getattr(self, "h", None):
            self.ref.L.ref_sampler_free(self.h)
            self.h = None


# ------------------------------------------------------------- GGUF read --

class GGUFFile:
    """Minimal GGUF v2/v3 reader over a numpy memmap, restating
    src/core/gguf.cpp:116-183 (header, typed metadata, tensor table,
    data offset aligned to general.alignment, default 32)."""

    _SCALARS = {0: "<B", 1: "<b", 2: "<H", 3: "<h", 4: "<I", 5: "<i", 6: "<f", 7: "<?",
                10: "<Q", 11: "<q", 12: "<d"}

    def __init__(self, path):
        self.path = str(path)
        self.buf = np.memmap(self.path, dtype=np.uint8, mode="r")
        self.pos = 0
        if bytes(self.buf[:4]) != b"GGUF":
            raise ValueError("gguf: bad magic, not a GGUF file")
        self.pos = 4
        self.version = self._u("<I")
        n_t = self._u("<Q")
        n_kv = self._u("<Q")
        self.meta = {}
        for _ in range(n_kv):
            k = self._str()
            t = self._u("<I")
            self.meta[k] = self._val(t)
        self.tensors = {}
        for _ in range(n_t):
            name = self._str()
            nd = self._u("<I")
            dims = [self._u("<Q") for _ in range(nd)]
            t = self._u("<I")
            off = self._u("<Q")
            self.tensors[name] = (dims, t, off)
        align = self.meta.get("general.alignment", 32)
        self.data_offset = (self.pos + align - 1) // align * align

    def _u(self, fmt):
        n = struct.calcsize(fmt)
        v = struct.unpack_from(fmt, self.buf, self.pos)[0]
        self.pos += n
        return v

    def _str(self):
        n = self._u("<Q")
        s = bytes(self.buf[self.pos:self.pos + n]).decode("utf-8", "replace")
        self.pos += n
        return s

    def _val(self, t):
        if t in self._SCALARS:
            return self._u(self._SCALARS[t])
        if t == 8:
            return self._str()
        if t == 9:
            et = self._u("<I")
            n = self._u("<Q")
            return [self._val(et) for _ in range(n)]
        raise ValueError("gguf: unknown metadata value type")

    def raw(self, name) -> np.ndarray:
        dims, t, off = self.tensors[name]
        n = int(np.prod(dims))
        start = self.data_offset + off
        return self.buf[start:start + type_nbytes(t, n)]

    def info(self, name):
        return self.tensors[name]


# ---------------------------------------------------- model restatement --

class OracleModel:
    """Restatement of Qwen2Model / LlamaModel (qwen2_model.cpp:78-198,
    llama_model.cpp:71-177) over the C restatement's kernels.  Handles every
    type the CUDA backend does, Q4_K included."""

    def __init__(self, path, orc: Oracle | None = None):
        self.o = orc or Oracle()
        g = GGUFFile(path)
        self.g = g
        a = g.meta["general.architecture"]
        if a not in ("qwen2", "llama"):
            raise ValueError(f"config: unsupported architecture: {a}")
        self.arch = a
        m = g.meta
        self.n_layers = m[f"{a}.block_count"]
        self.embd = m[f"{a}.embedding_length"]
        self.ffn = m[f"{a}.feed_forward_length"]
        self.n_heads = m[f"{a}.attention.head_count"]
        self.ctx = m[f"{a}.context_length"]
        self.n_kv = m.get(f"{a}.attention.head_count_kv", self.n_heads)
        self.rope_base = float(np.float32(m.get(f"{a}.rope.freq_base", 10000.0)))
        self.eps = float(np.float32(m.get(f"{a}.attention.layer_norm_rms_epsilon", 1e-5)))
        self.vocab = len(m.get("tokenizer.ggml.tokens", []))
        self.hd = self.embd // self.n_heads

        def deq(name):
            dims, t, _ = g.info(name)
            return self.o.dequantize(t, g.raw(name), int(np.prod(dims)))

        def qt(name):
            dims, t, _ = g.info(name)
            return (np.ascontiguousarray(g.raw(name)), t)

        self.token_embd = deq("token_embd.weight").reshape(self.vocab, self.embd)
        self.output_norm = deq("output_norm.weight")
        self.output = qt("output.weight")
        self.layers = []
        for i in range(self.n_layers):
            p = f"blk.{i}."
            L = {"attn_norm": deq(p + "attn_norm.weight"), "ffn_norm": deq(p + "ffn_norm.weight")}
            for k in ("attn_q", "attn_k", "attn_v", "attn_output", "ffn_gate", "ffn_up", "ffn_down"):
                L[k] = qt(p + k + ".weight")
            if a == "qwen2":
                for k in ("attn_q", "attn_k", "attn_v"):
                    L[k + "_b"] = deq(p + k + ".bias")
            self.layers.append(L)
        kvd = self.n_kv * self.hd
        self.kc = np.zeros((self.n_layers, self.ctx, kvd), dtype=np.float32)
        self.vc = np.zeros((self.n_layers, self.ctx, kvd), dtype=np.float32)
        self.cached_length = 0

    def reset_cache(self):
        self.cached_length = 0

    def truncate_cache(self, n):
        if n < self.cached_length:
            self.cached_length = n

    def _mm(self, wt, x, rows, cols):
        return self.o.matmul_quantized(wt[0], wt[1], x, rows, cols)

    def forward(self, token: int, pos: int) -> np.ndarray:
        o, e = self.o, self.embd
        hd, nh, nkv = self.hd, self.n_heads, self.n_kv
        qd, kvd = nh * hd, nkv * hd
        x = self.token_embd[token].copy()
        for li, L in enumerate(self.layers):
            h = o.rmsnorm(x, L["attn_norm"], self.eps)
            q = self._mm(L["attn_q"], h, qd, e)
            k = self._mm(L["attn_k"], h, kvd, e)
            v = self._mm(L["attn_v"], h, kvd, e)
            if self.arch == "qwen2":
                o.axpy(q, L["attn_q_b"], 1.0)
                o.axpy(k, L["attn_k_b"], 1.0)
                o.axpy(v, L["attn_v_b"], 1.0)
            q = o.rope(q, nh, hd, pos, self.rope_base)
            k = o.rope(k, nkv, hd, pos, self.rope_base)
            self.kc[li, pos] = k
            self.vc[li, pos] = v
            att = o.attention(q, self.kc[li], self.vc[li], nh, nkv, hd, pos)
            proj = self._mm(L["attn_output"], att, e, qd)
            o.axpy(x, proj, 1.0)
            h = o.rmsnorm(x, L["ffn_norm"], self.eps)
            gate = self._mm(L["ffn_gate"], h, self.ffn, e)
            up = self._mm(L["ffn_up"], h, self.ffn, e)
            gate = o.silu(gate)
            o.mul(gate, up)
            down = self._mm(L["ffn_down"], gate, e, self.ffn)
            o.axpy(x, down, 1.0)
        h = o.rmsnorm(x, self.output_norm, self.eps)
        logits = self._mm(self.output, h, self.vocab, e)
        self.cached_length = pos + 1
        return logits


# ------------------------------------------------------ sampler restatement --

class MT19937:
    """std::mt19937 (32-bit Mersenne Twister, seeded like the C++ standard's
    single-integer constructor) -- numpy's legacy MT19937 uses the same
    init_genrand seeding."""

    def __init__(self, seed: int):
        self.bg = np.random.MT19937(0)
        self.bg._legacy_seeding(seed & 0xFFFFFFFF)

    def next_u32(self) -> int:
        return int(self.bg.random_raw())

    def uniform01(self) -> float:
        """std::uniform_real_distribution<float>(0, 1) on std::mt19937 with
        libstdc++: generate_canonical<float, 24> takes one 32-bit draw,
        divides by 2^32 in float and clamps a result of 1.0 down to the
        float just below 1."""
        r = np.float32(self.next_u32()) / np.float32(4294967296.0)
        if r >= np.float32(1.0):
            r = np.nextafter(np.float32(1.0), np.float32(0.0))
        return float(r)
