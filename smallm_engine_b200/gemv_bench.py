"""Isolated quantized GEMV benchmark (the decode path's dominant kernel).

    python -m smallm_engine_b200.gemv_bench --type q4_0 --rows 14336 --cols 4096

Uploads `--copies` independent seeded matrices (enough that together they
exceed the 126 MB L2, so every launch streams from HBM), launches the GEMV
`--iters` times round-robin on the context stream, once from the host and
once replayed from a CUDA graph, and times both with CUDA events on that
stream (the graph figure is the device time; the host-launched one also
pays the Python launch cost).  Prints one JSON line: ms per launch and
the achieved bandwidth counted in ALGORITHMIC bytes (the GGUF bytes of the
matrix plus x and y), the same count as the reference's memory traffic.
"""
from __future__ import annotations

import argparse
import json
import sys

TYPES = {"f32": 0, "q4_0": 2, "q8_0": 8, "q4_k": 12, "q6_k": 14}


def run(type_: str, rows: int, cols: int, iters: int = 50, copies: int = 0, device: int = 0,
        warmup: int = 8) -> dict:
    import torch

    from . import CUDABackend, synth
    t = TYPES[type_]
    be = CUDABackend(device)
    per = synth.nbytes(t, rows * cols)
    if copies <= 0:
        copies = max(2, -(-300 * 2**20 // per))  # > 2x L2
    mats = []
    for i in range(copies):
        W = synth.fill(t, 1000 + i, "gemv_bench", rows * cols, 0.02)
        mats.append(be.upload(W, t, rows, cols))
    dev = f"cuda:{device}"
    x = torch.randn(cols, device=dev)
    y = torch.empty(rows, device=dev)
    s = torch.cuda.ExternalStream(be.stream, device=dev)
    for i in range(warmup):
        mats[i % copies].gemv(x.data_ptr(), y.data_ptr(), be.stream)
    be.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    # host-launched: includes the Python/ctypes cost of each launch
    e0.record(s)
    for i in range(iters):
        mats[i % copies].gemv(x.data_ptr(), y.data_ptr(), be.stream)
    e1.record(s)
    e1.synchronize()
    ms_stream = e0.elapsed_time(e1) / iters
    # the same launches captured in a CUDA graph: device time only
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=s):
        for i in range(iters):
            mats[i % copies].gemv(x.data_ptr(), y.data_ptr(), be.stream)
    with torch.cuda.stream(s):  # replay on the stream the events are recorded on
        g.replay()
        s.synchronize()
        e0.record(s)
        g.replay()
        e1.record(s)
    e1.synchronize()
    ms = e0.elapsed_time(e1) / iters
    del g
    algo = per + 4 * (rows + cols)
    for m in mats:
        m.free()
    be.close()
    return {"type": type_, "rows": rows, "cols": cols, "iters": iters, "copies": copies,
            "ms_per_launch": ms, "ms_per_launch_stream": ms_stream, "algorithmic_bytes": algo,
            "gbs": algo / (ms / 1e3) / 1e9}


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--type", default="q4_0", choices=sorted(TYPES))
    ap.add_argument("--rows", type=int, default=14336)
    ap.add_argument("--cols", type=int, default=4096)
    ap.add_argument("--iters", type=int, default=50)
    ap.add_argument("--copies", type=int, default=0)
    ap.add_argument("--warmup", type=int, default=8)
    a = ap.parse_args(argv)
    print(json.dumps(run(a.type, a.rows, a.cols, a.iters, a.copies, warmup=a.warmup)), flush=True)


if __name__ == "__main__":
    sys.exit(main())
