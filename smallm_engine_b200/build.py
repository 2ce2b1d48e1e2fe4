"""In-tree build of the native libraries (no JIT cache, nothing installed).

    python -m smallm_engine_b200.build          # build what is out of date
    python -m smallm_engine_b200.build --force  # rebuild everything

Outputs, all under ``smallm_engine_b200/lib/``:

* ``libsmallm_cuda.so``  -- the CUDA backend: every sm_100a kernel plus the
  C-ABI declared in ``include/smallm_cuda.h``.  Built with
  ``nvcc -gencode arch=compute_100a,code=sm_100a`` and a static CUDA runtime.
* ``libsmallm_synth.so`` -- host-only seeded generator/quantizer used to write
  synthetic GGUF files.
"""
from __future__ import annotations

import argparse
import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / "csrc"
LIB = PKG / "lib"
OBJ = PKG / "_build"

CUDA_LIB = LIB / "libsmallm_cuda.so"
SYNTH_LIB = LIB / "libsmallm_synth.so"

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def _host_cc() -> str:
    # An alternative gcc exported through $CC may lack libgomp; prefer the
    # system compiler, which is also what nvcc uses as its host compiler.
    for c in ("/usr/bin/gcc", "gcc"):
        if shutil.which(c):
            return c
    raise RuntimeError("no host C compiler found")


def _host_cxx() -> str:
    for c in ("/usr/bin/g++", "g++"):
        if shutil.which(c):
            return c
    raise RuntimeError("no host C++ compiler found")


def _nvcc() -> str:
    for c in ("/usr/local/cuda/bin/nvcc", "nvcc"):
        if shutil.which(c):
            return c
    raise RuntimeError("nvcc not found: the CUDA backend cannot be built")


def nccl_paths() -> tuple[Path, Path]:
    """(include dir, library dir) of the NCCL that torch also loads."""
    import importlib.util

    spec = importlib.util.find_spec("nvidia.nccl")
    if spec is not None and spec.submodule_search_locations:
        base = Path(list(spec.submodule_search_locations)[0])
        if (base / "include" / "nccl.h").exists():
            return base / "include", base / "lib"
    return Path("/usr/include"), Path("/usr/lib/x86_64-linux-gnu")


def _stale(target: Path, sources: list[Path]) -> bool:
    if not target.exists():
        return True
    t = target.stat().st_mtime
    return any(s.stat().st_mtime > t for s in sources)


def _run(cmd: list[str]) -> None:
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        sys.stderr.write(r.stdout + r.stderr)
        raise RuntimeError(f"build step failed ({r.returncode}): {' '.join(cmd[:4])} ...")


def build_synth(force: bool = False) -> Path:
    src = CSRC / "synth.c"
    if force or _stale(SYNTH_LIB, [src]):
        LIB.mkdir(exist_ok=True)
        _run([_host_cc(), "-O2", "-fopenmp", "-fPIC", "-shared", "-ffp-contract=off",
              "-o", str(SYNTH_LIB), str(src), "-lm"])
    return SYNTH_LIB


def cuda_sources() -> list[Path]:
    return sorted(list(CSRC.glob("*.cu")) + list(CSRC.glob("*.cpp")))


def cuda_headers() -> list[Path]:
    return sorted(list(CSRC.glob("*.h")) + list(CSRC.glob("*.cuh")) +
                  list((ROOT / "include").glob("*.h")) + [CSRC / "exports.map"])


def build_cuda(force: bool = False, jobs: int | None = None) -> Path:
    srcs = cuda_sources()
    if not srcs:
        raise RuntimeError("no CUDA sources found")
    headers = cuda_headers()
    if not (force or _stale(CUDA_LIB, srcs + headers)):
        return CUDA_LIB
    LIB.mkdir(exist_ok=True)
    OBJ.mkdir(exist_ok=True)
    nvcc = _nvcc()
    inc_nccl, lib_nccl = nccl_paths()
    common = ["-std=c++17", "-O3", "-lineinfo", "-Xcompiler", "-fPIC",
              "-I", str(ROOT / "include"), "-I", str(CSRC), "-I", str(inc_nccl),
              "-ccbin", _host_cxx()]
    objs = []
    procs = []
    for s in srcs:
        o = OBJ / (s.name + ".o")
        objs.append(o)
        if not force and o.exists() and o.stat().st_mtime > max(
                [s.stat().st_mtime] + [h.stat().st_mtime for h in headers]):
            continue
        cmd = [nvcc, *ARCH, *common, "-Xptxas=-warn-spills", "-c", str(s), "-o", str(o)]
        procs.append((cmd, subprocess.Popen(cmd, stdout=subprocess.PIPE,
                                            stderr=subprocess.STDOUT, text=True)))
    failed = []
    for cmd, p in procs:
        out, _ = p.communicate()
        if p.returncode != 0:
            failed.append(out)
        elif "spill" in out and "0 bytes spill" not in out:
            sys.stderr.write(out)
    if failed:
        sys.stderr.write("\n".join(failed))
        raise RuntimeError("nvcc compilation failed")
    _run([nvcc, *ARCH, "-shared", "-cudart", "static", "-o", str(CUDA_LIB),
          *[str(o) for o in objs], "-L", str(lib_nccl), "-l:libnccl.so.2",
          "-Xlinker", f"-rpath={lib_nccl}",
          "-Xlinker", f"--version-script={CSRC / 'exports.map'}"])
    return CUDA_LIB


def build_all(force: bool = False) -> None:
    build_synth(force)
    build_cuda(force)


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    a = ap.parse_args()
    build_all(a.force)
    print(f"built {CUDA_LIB} and {SYNTH_LIB}")


if __name__ == "__main__":
    main()
