"""Prefill benchmark: the tensor-core GEMM alone and the batched prefill of a
whole model (the dense-contraction path).

    python -m smallm_engine_b200.prefill_bench [--workload qwen2-1.5b-q8_0]
        [--seqs 4] [--tokens 512] [--decode 64] [--gemm-only]

GEMM leg: smallm_gemm_f16 (tcgen05) on seeded f16 operands with the
workload's layer shapes over seqs x tokens rows, `iters` launches timed with
CUDA events on the launching stream after warm-up; TFLOP/s counts 2*N*K*T
per launch.  Model leg: `seqs` independent seeded prompts of `tokens` ids,
each prefilled in one pass (smallm_model_prefill on the tcgen05 GEMMs, after
reset_cache) and then decoded greedily for `decode` steps from its prefilled
cache; CUDA events on the model stream around each prefill and each decode.  Linear-layer FLOPs per
token are 2 x the layer weights (the lm_head runs once, for the last token).
One JSON line.
"""
from __future__ import annotations

import argparse
import json
import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parents[1]


def tensor_peak() -> tuple[float, str]:
    """Dense 16-bit tensor peak in TFLOP/s: the measured cuBLAS bf16 figure
    when the driver wrote one, else the pool's earlier measurement."""
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        try:
            return float(json.loads(p.read_text())["bf16_tflops"]), "measured"
        except Exception:
            pass
    return 1590.0, "fallback"


def layer_shapes(spec) -> list[tuple[str, int, int]]:
    """(name, rows, cols) of one layer's GEMMs as the prefill runs them."""
    hd = spec.head_dim
    q, kv = spec.heads * hd, spec.kv_heads * hd
    return [("qkv", q + 2 * kv, spec.embd), ("o", spec.embd, q), ("gate_up", 2 * spec.ffn, spec.embd),
            ("down", spec.embd, spec.ffn)]


def gemm_run(spec, T: int, iters: int = 20, device: int = 0) -> list[dict]:
    import torch

    from . import CUDABackend
    from . import _lib
    be = CUDABackend(device)
    dev = f"cuda:{device}"
    out = []
    for name, N, K in layer_shapes(spec):
        g = torch.Generator(device=dev).manual_seed(N * 7 + K)
        w = (torch.randn(N, K, device=dev, generator=g) * 0.02).half()
        x = torch.randn(T, K, device=dev, generator=g).half()
        y = torch.empty(T, N, device=dev)
        torch.cuda.synchronize(dev)
        s = torch.cuda.ExternalStream(be.stream, device=dev)  # the stream the kernel runs on

        def launch():
            _lib.check(_lib.lib().smallm_gemm_f16(be.h, w.data_ptr(), x.data_ptr(), N, K, T, y.data_ptr(), N,
                                                  be.stream))
        for _ in range(3):
            launch()
        be.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(s)
        for _ in range(iters):
            launch()
        e1.record(s)
        e1.synchronize()
        ms = e0.elapsed_time(e1) / iters
        flops = 2.0 * N * K * T
        out.append({"gemm": name, "N": N, "K": K, "T": T, "ms": ms, "tflops": flops / (ms / 1e3) / 1e12,
                    "operand_bytes": 2 * (N * K + T * K) + 4 * T * N})
        del w, x, y
    be.close()
    return out


def model_run(workload: str, seqs: int, tokens: int, decode: int, device: int = 0) -> dict:
    import numpy as np
    import torch

    from . import CudaModel, synth
    spec = synth.WORKLOADS[workload]
    path = synth.ensure_gguf(workload, synth.WORKLOAD_SEEDS[workload])
    m = CudaModel(path, device=device, max_ctx=tokens + decode)
    rng = np.random.default_rng(1)
    prompts = [rng.integers(0, spec.vocab, size=tokens).tolist() for _ in range(seqs)]
    s = torch.cuda.ExternalStream(m.stream, device=f"cuda:{device}")
    flops_tok = 2.0 * spec.layers * sum(r * c for _, r, c in layer_shapes(spec))
    m.reset_cache()
    m.prefill(prompts[0], 0, want_logits=False)  # makes the weight copies; warm-up
    ms, dec_ms, ids, heads = [], [], [], []
    for p in prompts:
        m.reset_cache()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(s)
        _, am = m.prefill(p, 0, want_logits=False)
        e1.record(s)
        e1.synchronize()
        ms.append(e0.elapsed_time(e1))
        ids.append(am)
        if decode:
            e0.record(s)
            m.decode_greedy_async(am, tokens, decode)
            e1.record(s)
            e1.synchronize()
            dec_ms.append(e0.elapsed_time(e1))
            heads.append([int(v) for v in m.decode_ids(decode)[:4]])
    m.close()
    tot = sum(ms)
    return {"workload": workload, "seqs": seqs, "tokens": tokens, "decode_steps": decode,
            "prefill_ms_per_seq": [round(v, 3) for v in ms],
            "prefill_tok_s": seqs * tokens / (tot / 1e3),
            "linear_tflops": flops_tok * seqs * tokens / (tot / 1e3) / 1e12,
            "decode_tok_s": (seqs * decode / (sum(dec_ms) / 1e3)) if dec_ms else None,
            "decode_ms_per_seq": [round(v, 3) for v in dec_ms],
            "first_ids": ids, "decode_ids_head": heads}


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--workload", default="qwen2-1.5b-q8_0")
    ap.add_argument("--seqs", type=int, default=4)
    ap.add_argument("--tokens", type=int, default=512)
    ap.add_argument("--decode", type=int, default=64)
    ap.add_argument("--iters", type=int, default=20)
    ap.add_argument("--gemm-only", action="store_true")
    a = ap.parse_args(argv)
    from . import synth
    spec = synth.WORKLOADS[a.workload]
    peak, kind = tensor_peak()
    g = gemm_run(spec, a.seqs * a.tokens, a.iters)
    for r in g:
        r["frac_of_" + kind + "_peak"] = r["tflops"] / peak
    line = {"gemm": g, "tensor_peak_tflops": peak, "peak_kind": kind}
    if not a.gemm_only:
        line["model"] = model_run(a.workload, a.seqs, a.tokens, a.decode)
        line["model"]["linear_frac_of_" + kind + "_peak"] = line["model"]["linear_tflops"] / peak
    print(json.dumps(line), flush=True)


if __name__ == "__main__":
    sys.exit(main())
