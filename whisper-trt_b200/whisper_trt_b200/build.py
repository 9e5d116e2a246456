"""Build the C-ABI library ``libwhisper_attn_b200.so`` from ``csrc/*.cu`` for sm_100a (in-tree).

    python -m whisper_trt_b200.build          (from the whisper-trt_b200/ directory), or
    python whisper-trt_b200/whisper_trt_b200/build.py

nvcc compiles each source with ``-gencode arch=compute_100a,code=sm_100a -lineinfo -O3`` into ``_build/`` and
links one shared library next to this file (the CUDA runtime linked statically, so the library needs only the
driver). Sources newer than their object are rebuilt; ``force=True`` rebuilds everything.
"""

from __future__ import annotations

import concurrent.futures as cf
import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent  # whisper-trt_b200/
CSRC = ROOT / "csrc"
INCLUDE = ROOT.parent / "include"
BUILD = ROOT / "_build"
LIB_NAME = "libwhisper_attn_b200.so"
LIB = PKG / LIB_NAME
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "--expt-relaxed-constexpr",
              "-Xptxas", "-v"]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found (set NVCC or put the CUDA toolkit's bin/ on PATH)")


def _compile(src: Path, obj: Path, log: Path) -> None:
    cmd = [nvcc(), *ARCH, *NVCC_FLAGS, "-I", str(INCLUDE), "-I", str(CSRC), "-c", str(src), "-o", str(obj)]
    res = subprocess.run(cmd, capture_output=True, text=True)
    log.write_text(" ".join(cmd) + "\n" + res.stdout + res.stderr)
    if res.returncode != 0:
        raise RuntimeError(f"nvcc failed on {src.name}:\n{res.stderr[-4000:]}")


def build(force: bool = False, verbose: bool = False) -> Path:
    """Compile every csrc/*.cu (if changed) and link the library; returns its path."""
    BUILD.mkdir(exist_ok=True)
    sources = sorted(CSRC.glob("*.cu"))
    headers = sorted(CSRC.glob("*.cuh")) + sorted(INCLUDE.glob("*.h"))
    newest_header = max((h.stat().st_mtime for h in headers), default=0.0)
    jobs = []
    for src in sources:
        obj = BUILD / (src.stem + ".o")
        stale = (force or not obj.exists() or obj.stat().st_mtime < src.stat().st_mtime
                 or obj.stat().st_mtime < newest_header)
        if stale:
            jobs.append((src, obj, BUILD / (src.stem + ".log")))
    with cf.ThreadPoolExecutor(max_workers=min(8, max(1, len(jobs)))) as ex:
        for f in [ex.submit(_compile, *j) for j in jobs]:
            f.result()
    objs = [BUILD / (s.stem + ".o") for s in sources]
    if jobs or not LIB.exists() or LIB.stat().st_mtime < max(o.stat().st_mtime for o in objs):
        tmp = LIB.with_suffix(".so.tmp")
        cmd = [nvcc(), *ARCH, "-shared", "-cudart", "static", "-o", str(tmp), *map(str, objs)]
        res = subprocess.run(cmd, capture_output=True, text=True)
        if res.returncode != 0:
            raise RuntimeError(f"link failed:\n{res.stderr[-4000:]}")
        os.replace(tmp, LIB)
    if verbose:
        for j in jobs:
            print(j[2].read_text())
    return LIB


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose="-v" in sys.argv))
