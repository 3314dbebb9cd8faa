"""Build libhga_b200.so in-tree with nvcc for sm_100a (no torch headers: plain C ABI)."""
from __future__ import annotations

import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")
OUT = os.path.join(HERE, "libhga_b200.so")
SOURCES = ["abi.cu", "prologue.cu", "summaries.cu", "route_prefill.cu", "attend_simt.cu", "attend_tc.cu", "route_tc.cu", "decode.cu", "decode_fast.cu", "shard.cu", "bank.cu"]
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def nvcc() -> str:
    cand = os.path.join(os.environ.get("CUDA_HOME", "/usr/local/cuda"), "bin", "nvcc")
    return cand if os.path.exists(cand) else "nvcc"


def needs_build() -> bool:
    if not os.path.exists(OUT):
        return True
    t = os.path.getmtime(OUT)
    deps = [os.path.join(CSRC, f) for f in os.listdir(CSRC)] + [os.path.join(HERE, "..", "include", "hga_b200.h")]
    return any(os.path.getmtime(d) > t for d in deps)


def build(verbose: bool = False, force: bool = False) -> str:
    if not force and not needs_build():
        return OUT
    objdir = os.path.join(HERE, "_build")
    os.makedirs(objdir, exist_ok=True)
    objs = []
    procs = []
    for src in SOURCES:
        obj = os.path.join(objdir, src.replace(".cu", ".o"))
        cmd = [nvcc(), *ARCH, "-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "-c",
               os.path.join(CSRC, src), "-o", obj]
        if verbose:
            cmd.insert(1, "-Xptxas=-v")
        procs.append((src, cmd, subprocess.Popen(cmd, stdout=subprocess.PIPE, stderr=subprocess.STDOUT, text=True)))
        objs.append(obj)
    failed = False
    for src, cmd, pr in procs:
        out, _ = pr.communicate()
        if pr.returncode != 0 or verbose:
            sys.stderr.write(f"--- nvcc {src}\n{out}")
        failed |= pr.returncode != 0
    if failed:
        raise RuntimeError("nvcc failed")
    tmp = OUT + ".tmp"
    subprocess.check_call([nvcc(), *ARCH, "-shared", "-o", tmp, *objs, "-lcudart"])
    os.replace(tmp, OUT)
    return OUT


if __name__ == "__main__":
    build(verbose="-v" in sys.argv, force=True)
    print(OUT)
