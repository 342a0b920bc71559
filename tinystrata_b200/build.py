"""Build libtsb_moe.so in-tree for sm_100a (nvcc), after generating the GGUF codebook header.

``python -m tinystrata_b200.build`` or ``tinystrata_b200.build.build()``.  The library lands next to this file so it
travels with the source tree; nothing is installed into site-packages.
"""
from __future__ import annotations

import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")
LIB = os.path.join(HERE, "libtsb_moe.so")
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
SOURCES = ["tsb_moe.cu", "tsb_decode.cu", "tsb_decode_act.cu", "tsb_ep.cu", "tsb_staged.cu", "tsb_gguf.cpp"]
# every header of the sources: a change to any of them rebuilds both objects
HEADERS = sorted(f for f in os.listdir(CSRC) if f.endswith((".cuh", ".inc"))) + ["../../include/tsb_moe.h"]
FLAGS = ["-std=c++17", "-O3", "-gencode", "arch=compute_100a,code=sm_100a", "-lineinfo", "-Xcompiler", "-fPIC",
         "--expt-relaxed-constexpr"]


def _stale(target: str, deps: list[str]) -> bool:
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.exists(d) and os.path.getmtime(d) > t for d in deps)


def build(verbose: bool = False, force: bool = False) -> str:
    sys.path.insert(0, CSRC)
    try:
        import gen_codebooks
        gen_codebooks.main(os.path.join(CSRC, "codebooks.inc"))
    finally:
        sys.path.pop(0)
    srcs = [s for s in SOURCES if os.path.exists(os.path.join(CSRC, s))]
    deps = [os.path.join(CSRC, f) for f in srcs + HEADERS]
    objs = []
    os.makedirs(os.path.join(HERE, "_build"), exist_ok=True)
    procs = []
    for s in srcs:
        obj = os.path.join(HERE, "_build", os.path.splitext(s)[0] + ".o")
        objs.append(obj)
        if force or _stale(obj, deps):
            cmd = [NVCC, *FLAGS, "-c", os.path.join(CSRC, s), "-o", obj]
            if verbose:
                print(" ".join(cmd), flush=True)
            procs.append((s, subprocess.Popen(cmd, stdout=subprocess.PIPE, stderr=subprocess.STDOUT, text=True)))
    for s, p in procs:
        out, _ = p.communicate()
        if p.returncode != 0:
            raise RuntimeError(f"nvcc failed on {s}:\n{out}")
        if verbose and out.strip():
            print(out)
    if force or _stale(LIB, objs):
        cmd = [NVCC, "-shared", "-gencode", "arch=compute_100a,code=sm_100a", "-o", LIB, *objs, "-lcudart", "-ldl"]
        if verbose:
            print(" ".join(cmd), flush=True)
        subprocess.run(cmd, check=True)
    return LIB


if __name__ == "__main__":
    print(build(verbose=True, force="--force" in sys.argv))
