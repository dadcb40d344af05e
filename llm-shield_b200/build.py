"""Build the B200 Jevstral libraries in-tree.

libjv.so     CUDA kernels for sm_100a + the host runtime behind include/jv.h
             (nvcc -gencode arch=compute_100a,code=sm_100a, static CUDA runtime).
libjv_checked.so  the same with -DJV_BOUNDS_CHECK (index checks that fail the call instead of
             touching memory out of range; a diagnostic build, selected with JV_LIBRARY).
libjvsynth.so  the random-weight GGUF filler used by the tests and the benchmark.
jvsynth        the same filler as a stand-alone program (the benchmark's reference arm).

Usage: python llm-shield_b200/build.py [--verbose] [--ptxas]
"""
from __future__ import annotations

import concurrent.futures as cf
import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
CSRC = PKG / "csrc"
OUT = PKG / "_build"
OUT_CHECKED = PKG / "_build_checked"
LIB = PKG / "libjv.so"
LIB_CHECKED = PKG / "libjv_checked.so"
SYNTH = PKG / "libjvsynth.so"
SYNTH_EXE = PKG / "jvsynth"

NVCC = os.environ.get("NVCC", shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ARCH + ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC", "--expt-relaxed-constexpr",
                     "-Xcompiler", "-Wall,-Wno-unused-function", "-I", str(PKG.parent / "include")]

SOURCES = ["gguf.cpp", "qx.cpp", "runtime.cu", "kernels_quant.cu", "kernels_elem.cu", "kernels_attn.cu", "attn_tc.cu", "gemm_tc.cu",
           "quantmatmul.cu", "noalloc.cu", "kernels_decode.cu"]


def _run(cmd: list[str], verbose: bool) -> str:
    if verbose:
        print(" ".join(cmd), flush=True)
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"command failed ({r.returncode}): {' '.join(cmd)}\n{r.stdout}\n{r.stderr}")
    return r.stdout + r.stderr


def _stale(target: Path, deps: list[Path]) -> bool:
    if not target.exists():
        return True
    t = target.stat().st_mtime
    return any(d.stat().st_mtime > t for d in deps)


def build(verbose: bool = False, ptxas: bool = False, force: bool = False) -> Path:
    _build_lib(LIB, OUT, [], verbose, ptxas, force)
    _build_lib(LIB_CHECKED, OUT_CHECKED, ["-DJV_BOUNDS_CHECK"], verbose, False, force)
    _build_synth(force, verbose)
    return LIB


def _build_lib(lib: Path, out: Path, extra: list[str], verbose: bool, ptxas: bool, force: bool) -> None:
    out.mkdir(exist_ok=True)
    headers = list(CSRC.glob("*.h")) + list(CSRC.glob("*.cuh")) + [PKG.parent / "include" / "jv.h"]
    jobs = []
    objs = []
    for src in SOURCES:
        s = CSRC / src
        o = out / (src + ".o")
        objs.append(o)
        if force or _stale(o, [s] + headers):
            flags = list(NVCC_FLAGS) + extra
            if ptxas and src.endswith(".cu"):
                flags += ["-Xptxas", "-v"]
            jobs.append([NVCC] + flags + (["-x", "cu"] if src.endswith(".cu") else []) + ["-c", str(s), "-o", str(o)])
    logs = []
    with cf.ThreadPoolExecutor(max_workers=min(8, max(1, len(jobs)))) as ex:
        for out in ex.map(lambda c: _run(c, verbose), jobs):
            logs.append(out)
    if ptxas:
        for log in logs:
            print(log)
    if force or jobs or _stale(lib, objs):
        _run([NVCC] + ARCH + ["-shared", "-o", str(lib)] + [str(o) for o in objs] +
             ["-cudart", "static", "-lpthread", "-ldl", "-lrt"], verbose)


def _build_synth(force: bool, verbose: bool) -> None:
    synth_src = CSRC / "synth" / "gguf_synth.cpp"
    if force or _stale(SYNTH, [synth_src]):
        _run(["g++", "-O3", "-std=c++17", "-fPIC", "-ffp-contract=off", "-fno-fast-math", "-shared", "-o", str(SYNTH),
              str(synth_src), "-lpthread"], verbose)
    if force or _stale(SYNTH_EXE, [synth_src]):
        _run(["g++", "-O3", "-std=c++17", "-DJVS_MAIN", "-ffp-contract=off", "-fno-fast-math", "-o", str(SYNTH_EXE),
              str(synth_src), "-lpthread"], verbose)


if __name__ == "__main__":
    build(verbose="--verbose" in sys.argv, ptxas="--ptxas" in sys.argv, force="--force" in sys.argv)
    print(LIB)
