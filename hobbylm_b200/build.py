"""Build libhobbygpu.so in-tree (nvcc for sm_100a; host C++ through nvcc's g++).

    python -m hobbylm_b200.build [--force]

The library lands at hobbylm_b200/libhobbygpu.so; objects under hobbylm_b200/_build/.
"""
from __future__ import annotations

import argparse
import os
import shutil
import subprocess
import sys
from concurrent.futures import ThreadPoolExecutor

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")
BUILD = os.path.join(HERE, "_build")
LIB = os.path.join(HERE, "libhobbygpu.so")
INCLUDE = os.path.join(os.path.dirname(HERE), "include")

SOURCES = ["engine.cu", "decode.cu", "tc.cu", "ep.cu", "prefill.cu", "sample.cu", "noalloc.cu", "gguf.cpp", "sampler.cpp"]
HEADERS = ["hg_device.cuh", "hg_model.cuh", "hg_launch.h", "hg_host.h", "hg_ep.h"]

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
# --fmad=false: no implicit FMA contraction; kernels write every fused multiply-add explicitly so the
# arithmetic order matches the reference. IEEE division / sqrt stay on (nvcc defaults).
NVFLAGS = ["-O3", "-std=c++17", "-lineinfo", "--fmad=false", "-Xcompiler", "-fPIC,-fopenmp,-ffp-contract=off",
           f"-I{INCLUDE}", "--expt-relaxed-constexpr"]


def nvcc() -> str:
    for c in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if c and os.path.exists(c):
            return c
    raise RuntimeError("nvcc not found")


def _stale(out: str, deps: list[str]) -> bool:
    if not os.path.exists(out):
        return True
    t = os.path.getmtime(out)
    return any(os.path.getmtime(d) > t for d in deps)


def build(force: bool = False, verbose: bool = False, ptxas_verbose: bool = False) -> str:
    os.makedirs(BUILD, exist_ok=True)
    hdrs = [os.path.join(CSRC, h) for h in HEADERS] + [os.path.join(INCLUDE, "hobbygpu.h")]
    objs, jobs = [], []
    for src in SOURCES:
        s = os.path.join(CSRC, src)
        o = os.path.join(BUILD, src + ".o")
        objs.append(o)
        if force or _stale(o, [s, *hdrs]):
            cmd = [nvcc(), *ARCH, *NVFLAGS, "-c", s, "-o", o]
            if ptxas_verbose and src.endswith(".cu"):
                cmd.insert(1, "-Xptxas=-v")
            jobs.append(cmd)

    def run(cmd):
        if verbose:
            print(" ".join(cmd), flush=True)
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"compile failed: {' '.join(cmd)}\n{r.stdout}\n{r.stderr}")
        if ptxas_verbose:
            sys.stderr.write(r.stderr)
        return r

    with ThreadPoolExecutor(max_workers=min(8, max(1, len(jobs)))) as ex:
        list(ex.map(run, jobs))
    if force or jobs or _stale(LIB, objs):
        tmp = LIB + f".tmp{os.getpid()}"
        run([nvcc(), *ARCH, "-shared", "-Xcompiler", "-fopenmp", *objs, "-o", tmp, "-lgomp", "-lcudart", "-ldl"])
        os.replace(tmp, LIB)
    return LIB


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("-v", "--verbose", action="store_true")
    ap.add_argument("--ptxas", action="store_true", help="print registers / spills / shared memory per kernel")
    a = ap.parse_args()
    print(build(a.force, a.verbose, a.ptxas))


if __name__ == "__main__":
    main()
