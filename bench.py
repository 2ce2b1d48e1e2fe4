"""Decode benchmark: batch-1 greedy decode tok/s of the Llama-3-8B-shaped
Q4_0 model (hidden 4096, 32 layers, 32/8 heads, FFN 14336, vocab 128256;
Q4_0 linears, Q8_0 embeddings/output; seeded synthetic weights), plus the
fraction of B200 HBM roofline.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

One JSON line on rank 0.  A step is one decode token.  Both arms run the same
sequence: the 128-token prompt through Model::forward token by token
(positions 0..127), W untimed greedy steps, then K timed greedy steps at
positions 128+W .. 128+W+K-1.  Under torchrun (N > 1) the model is
tensor-parallel over the N GPUs (heads / FFN rows split, the residual
all-reduced after attention and after the FFN); total work is fixed, so
scaling is "strong".

  value        K greedy steps enqueued as K CUDA-graph launches with the
               token fed back on the device; CUDA events on the model stream,
               max over ranks.  The weights (4.5 GB) are far larger than L2.
  e2e          the same K steps through the public Model::forward call
               (smallm_model_forward): per step the token/position state goes
               host->device from pinned memory and the full logits come back
               device->host into pinned memory.
  roofline     the dominant kernel, the Q4_0 GEMV, timed alone on the
               14336x4096 matrix (33.03 MB of Q4_0 blocks per launch, four
               copies rotated so every launch streams from HBM).
  gemv_q4_0    the isolated Q4_0 GEMV op on both of its matrices (14336x4096
               and 4096x14336, seed 2, x ~ N(0,1)): GPU time and GB/s, the
               reference's ops::matmul_quantized on the same matrix and x on
               the host cores, and the GPU result checked against the CPU one.
  cpu_baseline the reference's own CPU decode (compiled from its sources,
               oracle/_ref) on a bounded sample of the same sequence, all
               host cores.
  --impl reference  the reference's CPU decode alone on the same sequence:
               W untimed and K timed greedy steps, steady_clock around the loop.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

WORKLOAD = "llama3-8b-q4_0"
PROMPT = 128
METRIC = "decode tok/s @B=1 (Llama-3-8B-shaped, Q4_0) + % of HBM BW roofline"
# dram__bytes_read.sum + dram__bytes_write.sum of one Q4_0 GEMV launch on the
# 14336x4096 matrix, from one ncu capture of the Q4_0 GEMV kernel
# (profiles/gemv_q4_0_14336x4096.md): 33.091072 MB read, 0 written (the
# algorithmic bytes are 33.10 MB).
GEMV_NCU_TRAFFIC_BYTES = 33091072


def peaks() -> tuple[float, str]:
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        try:
            return float(json.loads(p.read_text())["hbm_gbs"]), "measured"
        except Exception:
            pass
    return 6650.0, "fallback"


class ClockSampler:
    """nvidia-smi clocks and throttle reasons sampled every 25 ms."""
    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index = index
        self.proc = None
        self.lines: list[str] = []

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", "-i", str(self.index), f"--query-gpu={self.Q}",
                                          "--format=csv,noheader,nounits", "-lms", "25"],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
        except Exception:
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def __exit__(self, *a):
        if self.proc:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()

    def summary(self) -> dict:
        sm, mx, reasons = [], 0.0, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for l in self.lines:
            f = [x.strip() for x in l.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx = max(mx, float(f[2]))
            except ValueError:
                continue
            for n, v in zip(names, f[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx or None,
                "reasons": sorted(reasons), "samples": len(sm)}


def dist_setup():
    ws = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if ws > 1:
        import datetime
        import torch
        import torch.distributed as dist
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=600),
                                device_id=torch.device("cuda", local))
    return ws, rank, local


def allreduce_max(v: float, ws: int) -> float:
    from smallm_engine_b200.tp import max_over_ranks
    return max_over_ranks(v, ws, device="cuda")


def barrier(ws: int):
    if ws > 1:
        import torch.distributed as dist
        dist.barrier()


def ensure_model(ws: int, rank: int, workload: str = WORKLOAD) -> Path:
    from smallm_engine_b200 import synth
    if rank == 0:
        p = synth.ensure_gguf(workload)
    barrier(ws)
    if rank != 0:
        p = synth.ensure_gguf(workload)  # already written by rank 0: just the path
    return p


def metric_for(workload: str) -> str:
    return METRIC if workload == WORKLOAD else f"decode tok/s @B=1 ({workload}) + % of HBM BW roofline"


def prompt_ids(vocab: int, n: int = PROMPT) -> np.ndarray:
    return np.random.default_rng(1).integers(0, vocab, size=max(n, PROMPT))


# ------------------------------------------------------------ CPU baseline --

def _cpu_model(path: Path):
    """The reference build (oracle/_ref) on the workload, else the pinned
    restatement (the reference cannot load every workload: it has no Q4_K)."""
    sys.path.insert(0, str(ROOT / "oracle"))
    import oracle as O
    cores = os.cpu_count() or 1
    os.environ.setdefault("OMP_NUM_THREADS", str(cores))
    if O.Reference.available():
        try:
            return O.Reference().load(path), "reference", cores
        except Exception:
            pass
    return O.OracleModel(path), "port", cores


def cpu_decode(path: Path, prompt: np.ndarray, warmup: int, steps: int) -> tuple[np.ndarray, float, str, int]:
    """The reference's decode loop on the host: the prompt token by token,
    `warmup` untimed greedy steps, `steps` timed ones.  Returns (all greedy
    ids from the first decode step, ms of the timed steps, kind, cores)."""
    m, kind, cores = _cpu_model(path)
    if kind == "reference":
        ids, ms = m.decode_timed(prompt, steps, warmup=warmup)
        return ids, ms, kind, cores
    ids = []
    l = None
    for pos, t in enumerate(prompt):
        l = m.forward(int(t), pos)
    pos = len(prompt)
    t0 = 0.0
    for s in range(warmup + steps):
        if s == warmup:
            t0 = time.perf_counter()
        nxt = int(np.argmax(l))
        ids.append(nxt)
        l = m.forward(nxt, pos)
        pos += 1
    return np.array(ids, np.uint32), (time.perf_counter() - t0) * 1e3, kind, cores


def cpu_decode_sample(path: Path, vocab: int, prompt_len: int, workload: str = WORKLOAD) -> dict:
    """Bounded CPU sample of the benchmark's sequence (about 10-20 s on a
    16-core host): the same prompt, 2 untimed and 8 timed greedy steps."""
    prompt = prompt_ids(vocab, prompt_len)[:prompt_len]
    ids, ms, kind, cores = cpu_decode(path, prompt, 2, 8)
    return {"value": 8 / (ms / 1e3), "unit": "tok/s", "cores": cores, "kind": kind,
            "sample": f"{workload}: {prompt_len}-token prompt, 2 untimed + 8 timed greedy steps at positions "
                      f"{prompt_len + 2}..{prompt_len + 9} (steady_clock around the decode loop), "
                      f"OMP_NUM_THREADS={os.environ['OMP_NUM_THREADS']}",
            "greedy_ids_head": [int(v) for v in ids[:8]]}


def decode_config(workload: str, prompt: int, warmup: int, steps: int) -> dict:
    """The `config` object both arms print (identical for the same run)."""
    return {"workload": f"{workload} greedy decode, batch 1",
            "prompt": prompt,
            "positions": f"{prompt + warmup}..{prompt + warmup + steps - 1}",
            "warmup_steps": warmup}


def reference_arm(args, ws, rank):
    if rank != 0:
        return
    from smallm_engine_b200 import synth
    path = ensure_model(1, 0, args.workload)
    vocab = synth.WORKLOADS[args.workload].vocab
    prompt = prompt_ids(vocab, args.prompt)[:args.prompt]
    ids, ms, kind, cores = cpu_decode(path, prompt, args.warmup, args.steps)
    value = args.steps / (ms / 1e3)
    sample = (f"{args.workload}: {args.prompt}-token prompt, {args.warmup} untimed + {args.steps} timed greedy "
              f"steps (steady_clock around the decode loop), OMP_NUM_THREADS={os.environ['OMP_NUM_THREADS']}")
    line = {"metric": metric_for(args.workload), "value": value, "unit": "tok/s", "n_gpus": args.gpus,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms / args.steps,
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic (seeded random weights, random token ids)", "impl": "reference",
            "config": decode_config(args.workload, args.prompt, args.warmup, args.steps),
            "executor": f"reference CPU build ({kind}), OpenMP on {cores} host cores",
            "cpu_baseline": {"value": value, "unit": "tok/s", "cores": cores, "kind": kind, "sample": sample},
            "e2e": {"value": value, "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
            "greedy_ids_head": [int(v) for v in ids[:8]]}
    emit(line)


# ------------------------------------------------------------------ ours --

def gemv_legs(device: int, iters: int = 50, cpu: bool = True) -> list[dict]:
    """The isolated Q4_0 GEMV op on its two matrices, 14336x4096 and
    4096x14336 (f32 values ~N(0, 0.02) quantized to Q4_0, seed 2; x ~ N(0, 1)).
    GPU: four seeded copies rotated (132 MB > L2), `iters` launches replayed
    from a CUDA graph and timed with CUDA events on the launching stream
    (device time per launch, no host launch cost).  CPU: the reference's
    ops::matmul_quantized (oracle/_ref, OpenMP on every host core) on the
    seed-2 matrix and the same x, and the GPU's y on that matrix checked
    against it with the GEMV parity bound of the tests."""
    import torch
    from smallm_engine_b200 import CUDABackend, synth
    be = CUDABackend(device)
    dev = f"cuda:{device}"
    s = torch.cuda.ExternalStream(be.stream, device=dev)
    O = None
    if cpu:
        sys.path.insert(0, str(ROOT / "oracle"))
        import oracle as O
        os.environ.setdefault("OMP_NUM_THREADS", str(os.cpu_count() or 1))
    out = []
    for rows, cols in ((14336, 4096), (4096, 14336)):
        Ws = [synth.fill(synth.Q4_0, 2 + i, f"gemv{rows}x{cols}", rows * cols, 0.02) for i in range(4)]
        mats = [be.upload(W, synth.Q4_0, rows, cols) for W in Ws]
        algo = mats[0].bytes()[0] + cols * 4 + rows * 4
        xh = synth.normals(2, f"gemv-x{cols}", cols)
        x = torch.from_numpy(xh).to(dev)
        y = torch.empty(rows, device=dev)
        for i in range(8):
            mats[i % 4].gemv(x.data_ptr(), y.data_ptr(), be.stream)
        be.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=s):
            for i in range(iters):
                mats[i % 4].gemv(x.data_ptr(), y.data_ptr(), be.stream)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        with torch.cuda.stream(s):  # replay on the stream the events are recorded on
            g.replay()
            s.synchronize()
            e0.record(s)
            g.replay()
            e1.record(s)
        e1.synchronize()
        ms = e0.elapsed_time(e1) / iters
        del g
        mats[0].gemv(x.data_ptr(), y.data_ptr(), be.stream)
        be.synchronize()
        yg = y.cpu().numpy().astype(np.float64)
        leg = {"shape": f"{rows}x{cols}", "bytes": algo, "gpu_us": ms * 1e3,
               "gpu_gbs": algo / (ms / 1e3) / 1e9}
        if O is not None:
            cpu_impl = O.Reference() if O.Reference.available() else O.Oracle()
            kind = "reference" if O.Reference.available() else "port"
            yc = cpu_impl.matmul_quantized(Ws[0], synth.Q4_0, xh, rows, cols)
            n, t0 = 0, time.perf_counter()
            while n < 20 or (time.perf_counter() - t0 < 1.0 and n < 200):
                cpu_impl.matmul_quantized(Ws[0], synth.Q4_0, xh, rows, cols)
                n += 1
            cms = (time.perf_counter() - t0) * 1e3 / n
            # the tests' GEMV bound: 1e-5 sum|w x| + sum|w| r, r = one unit of
            # x's 21-bit block fixed point
            wd = np.abs(O.Oracle().dequantize(synth.Q4_0, Ws[0], rows * cols).reshape(rows, cols))
            m = np.abs(xh.astype(np.float64)).reshape(-1, 32).max(axis=1)
            r = np.repeat(np.where(m >= 1e-30, np.ldexp(1.0, np.frexp(m)[1] - 21), 1e-30), 32)
            bound = 1e-5 * (wd @ np.abs(xh.astype(np.float64))) + wd @ r + 1e-30
            err = np.abs(yg - yc.astype(np.float64))
            leg.update({"cpu_kind": kind, "cpu_ms": cms, "cpu_gbs": algo / (cms / 1e3) / 1e9,
                        "cpu_cores": int(os.environ["OMP_NUM_THREADS"]), "cpu_iters": n,
                        "max_abs_err": float(err.max()), "max_err_over_bound": float((err / bound).max()),
                        "parity": bool((err <= bound).all())})
        out.append(leg)
        for mt in mats:
            mt.free()
    be.close()
    return out


def our_arm(args, ws, rank, local):
    import torch
    from smallm_engine_b200 import CudaModel
    from smallm_engine_b200 import _lib

    path = ensure_model(ws, rank, args.workload)
    from smallm_engine_b200.tp import share_nccl_id
    nccl_id = share_nccl_id(rank, ws)
    total_steps = args.prompt + args.warmup + 2 * args.steps + 8
    max_ctx = max(512, (total_steps + 255) // 256 * 256)
    m = CudaModel(path, device=local, max_ctx=max_ctx, tp_rank=rank, tp_size=ws, nccl_id=nccl_id)
    cfg = m.config()
    dev = f"cuda:{local}"
    s = torch.cuda.ExternalStream(m.stream, device=dev)

    # prompt: token by token through Model::forward, like the reference's
    # Generator; its last argmax is the first decode token
    prompt = prompt_ids(cfg.vocab_size, args.prompt)[:args.prompt]
    tok = 0
    for pos, t in enumerate(prompt):
        tok = m.forward_into(int(t), pos, None)
    pos = len(prompt)
    head = [tok]
    # warm-up
    m.decode_greedy_async(tok, pos, args.warmup)
    ids = m.decode_ids(args.warmup)
    head += [int(v) for v in ids]
    pos += args.warmup
    tok = int(ids[-1])

    # ---- value: K device-fed greedy steps (graph launches), CUDA events
    barrier(ws)
    torch.cuda.synchronize(dev)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clk:
        e0.record(s)
        m.decode_greedy_async(tok, pos, args.steps)
        e1.record(s)
        e1.synchronize()
        torch.cuda.synchronize(dev)
        barrier(ws)
        ms = allreduce_max(e0.elapsed_time(e1), ws)
        ids = m.decode_ids(args.steps)
        head += [int(v) for v in ids]
        pos_timed = pos
        pos += args.steps
        tok = int(ids[-1])

        # ---- e2e: public forward() with pinned host buffers, K steps
        import ctypes
        hbuf = ctypes.c_void_p()
        _lib.check(_lib.lib().smallm_host_alloc(4 * cfg.vocab_size, ctypes.byref(hbuf)))
        barrier(ws)
        torch.cuda.synchronize(dev)
        f0, f1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        f0.record(s)
        for _ in range(args.steps):
            tok = m.forward_into(tok, pos, hbuf.value)
            pos += 1
        f1.record(s)
        f1.synchronize()
    barrier(ws)
    e2e_ms = allreduce_max(f0.elapsed_time(f1), ws)
    _lib.lib().smallm_host_free(hbuf)

    # ---- roofline numbers
    from smallm_engine_b200 import synth
    spec = synth.WORKLOADS[args.workload]
    mid = pos_timed + args.steps // 2
    bytes_tok = spec.weight_bytes_per_token() + spec.kv_bytes_per_token(mid)
    peak, peak_kind = peaks()
    step_ms = ms / args.steps
    step_gbs = bytes_tok / (step_ms / 1e3) / 1e9 / ws
    if rank == 0:
        want_cpu = ws == 1 and not args.no_cpu_baseline
        legs = gemv_legs(local, cpu=want_cpu)
        g = legs[0]
        ach = g["gpu_gbs"]
        cpu = cpu_decode_sample(path, cfg.vocab_size, args.prompt, workload=args.workload) if want_cpu else None
        line = {
            "metric": metric_for(args.workload),
            "value": args.steps / (ms / 1e3),
            "unit": "tok/s",
            "n_gpus": ws,
            "steps": args.steps,
            "warmup": args.warmup,
            "ms_per_step": step_ms,
            "higher_is_better": True,
            "scaling": "strong",
            "vs_baseline": None,
            "dtype": "f32",
            "x_repr": "activations enter the GEMVs as 21-bit block fixed point per 32 elements (three "
                      "int8 digits, held to 2^-21 of the block maximum) for every weight format; exact int32 "
                      "dot per digit and block, f32 scale and accumulation; attention, norms and residual in f32",
            "data": "synthetic (seeded random weights, random token ids)",
            "config": decode_config(args.workload, args.prompt, args.warmup, args.steps),
            "executor": f"tp{ws}" if ws > 1 else "single GPU",
            "l2": f"inputs larger than L2 ({spec.weight_bytes_per_token() / 1e9:.2f} GB of weights per step, "
                  "126 MB L2): no flush needed",
            "e2e": {"value": args.steps / (e2e_ms / 1e3), "unit": "tok/s", "h2d_bytes_per_step": 16,
                    "d2h_bytes_per_step": 4 * cfg.vocab_size + 16},
            "roofline": {"bound": "hbm", "achieved": ach, "peak": peak, "unit": "GB/s", "frac": ach / peak,
                         "traffic": GEMV_NCU_TRAFFIC_BYTES, "peak_source": peak_kind,
                         "kernel": "Q4_0 GEMV 14336x4096 (33.03 MB/launch)", "ms_per_launch": g["gpu_us"] / 1e3},
            "gemv_q4_0": [dict(l, frac=l["gpu_gbs"] / peak) for l in legs],
            "step_roofline": {"bytes_per_token": bytes_tok, "achieved_gbs_per_gpu": step_gbs,
                              "frac": step_gbs / peak, "note": "weights + f32 KV at mid position; "
                              "per-GPU share under tensor parallelism"},
            "gpu_launches": args.steps * cfg.step_launches,
            "step_path": "persistent step kernel (one cooperative launch per token)" if cfg.step_launches == 1
                         else f"per-op kernels ({cfg.step_launches} launches per token)",
            "clocks": clk.summary(),
            "greedy_ids_head": head[:8],
        }
        if cpu:
            line["cpu_baseline"] = cpu
        emit(line)
    barrier(ws)
    m.close()


# The result line is the only thing on stdout: libraries loaded on the way
# (NCCL prints its version there when NCCL_DEBUG is set) write to the
# process's file descriptor 1, so fd 1 is pointed at stderr for the run and
# the line goes to the saved original.
_RESULT_FD = None


def emit(line: dict) -> None:
    data = (json.dumps(line) + "\n").encode()
    if _RESULT_FD is None:
        sys.stdout.write(data.decode())
        sys.stdout.flush()
    else:
        os.write(_RESULT_FD, data)


def main():
    global _RESULT_FD
    sys.stdout.flush()
    _RESULT_FD = os.dup(1)
    os.dup2(2, 1)
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=64)
    ap.add_argument("--warmup", type=int, default=8)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--prompt", type=int, default=PROMPT, help="prompt length before the timed steps")
    ap.add_argument("--workload", default=WORKLOAD, help="synthetic model (synth.WORKLOADS); the default is the headline one")
    ap.add_argument("--no-cpu-baseline", action="store_true", help="skip the CPU baseline leg (profiling runs)")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    ws, rank, local = dist_setup()
    try:
        if args.impl == "reference":
            reference_arm(args, ws, rank)
        else:
            our_arm(args, ws, rank, local)
    finally:
        if ws > 1:
            import torch.distributed as dist
            dist.destroy_process_group()


if __name__ == "__main__":
    main()
