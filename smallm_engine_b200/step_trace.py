"""Per-kernel timeline of one decode step on the GPU.

    python -m smallm_engine_b200.step_trace --workload llama3-8b-q4_0 --prompt 128

Loads the workload's synthetic GGUF, runs a prompt, then traces a few steps
(smallm_model_trace_step) and prints, per kernel kind, the mean duration
(first CTA start to last CTA end), the mean time from start until the
dependency on the previous kernel released, the mean gap since the previous
kernel ended, and its share of the step.  Timestamps come from the GPU global
timer; the traced graph is a copy of the production step with stamping
enabled, so numbers include that small cost.
"""
from __future__ import annotations

import argparse
import collections
import json

import numpy as np


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--workload", default="llama3-8b-q4_0")
    ap.add_argument("--prompt", type=int, default=128)
    ap.add_argument("--steps", type=int, default=4)
    ap.add_argument("--json", action="store_true")
    a = ap.parse_args(argv)

    from . import CudaModel, synth
    path = synth.ensure_gguf(a.workload)
    m = CudaModel(path, max_ctx=max(512, a.prompt + a.steps + 8))
    vocab = m.config().vocab_size
    prompt = np.random.default_rng(1).integers(0, vocab, size=a.prompt)
    pos = 0
    for t in prompt[:-1]:
        m.forward(int(t), pos, want_logits=False)
        pos += 1
    tok = int(prompt[-1])
    agg = collections.OrderedDict()
    steps = []
    for _ in range(a.steps):
        tr = m.trace_step(tok, pos)
        pos += 1
        tok = int(np.argmax(m.forward(tok, pos - 1)))  # keep the cache consistent; feed greedy
        steps.append(tr)
        prev_end = 0
        pieces = [k for k in tr if k["kind"] in ("piece", "piece_done")]
        tr = [k for k in tr if k["kind"] not in ("piece", "piece_done")]
        steps[-1] = tr
        if pieces:
            # CTA 0's weight pieces: copy latency (start -> data seen), time to
            # the last warp's finish, and to retirement
            lat = [p["ready"] - p["start"] for p in pieces if p["kind"] == "piece"]
            ends = [p["end"] for p in pieces if p["kind"] == "piece"]
            dn = [p["start"] for p in pieces if p["kind"] == "piece_done"]
            rd = [p["ready"] for p in pieces if p["kind"] == "piece"]
            agg.setdefault("_pieces", []).append({
                "n": len(lat), "copy_to_seen_us": float(np.median(lat)) / 1e3,
                "seen_to_done_us": float(np.median(np.array(dn) - np.array(rd))) / 1e3,
                "done_to_retired_us": float(np.median(np.array(ends) - np.array(dn))) / 1e3,
                "interval_us": float(np.median(np.diff(ends))) / 1e3 if len(ends) > 1 else None})
        for k in tr:
            d = agg.setdefault(k["kind"], {"n": 0, "dur": 0.0, "wait": 0.0, "gap": 0.0})
            d["n"] += 1
            d["dur"] += k["end"] - k["start"]
            d["wait"] += max(0, k["ready"] - k["start"])
            d["gap"] += k["start"] - prev_end
            prev_end = k["end"]
    step_ns = np.mean([s[-1]["end"] for s in steps])
    out = {"workload": a.workload, "prompt": a.prompt, "step_us": step_ns / 1e3, "kernels": {}}
    if "_pieces" in agg:
        out["pieces_cta0"] = agg.pop("_pieces")[-1]
    for kind, d in agg.items():
        out["kernels"][kind] = {"per_step": d["n"] / a.steps, "mean_us": d["dur"] / d["n"] / 1e3,
                                "mean_wait_us": d["wait"] / d["n"] / 1e3, "mean_gap_us": d["gap"] / d["n"] / 1e3,
                                "share": d["dur"] / a.steps / step_ns}
    if a.json:
        print(json.dumps(out))
        return
    print(f"{a.workload}: step {out['step_us']:.1f} us (traced)")
    for kind, d in out["kernels"].items():
        print(f"  {kind:10s} x{d['per_step']:5.1f}  mean {d['mean_us']:7.2f} us  dep-wait {d['mean_wait_us']:6.2f} us"
              f"  gap {d['mean_gap_us']:6.2f} us  share {100 * d['share']:5.1f}%")


if __name__ == "__main__":
    main()
