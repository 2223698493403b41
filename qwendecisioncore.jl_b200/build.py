"""Build libqdc_b200.so (sm_100a) in-tree with nvcc.

    python qwendecisioncore.jl_b200/build.py

Output: qwendecisioncore.jl_b200/_build/libqdc_b200.so.  The library is a
plain C ABI (include/qdc_b200.h) linked against the CUDA runtime only; it
has no torch types, so it is built by nvcc directly rather than as a torch
extension.  -Xptxas -v output goes to _build/ptxas.txt.
"""
import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
OUT_DIR = os.path.join(HERE, "_build")
LIB = os.path.join(OUT_DIR, "libqdc_b200.so")
SOURCES = [os.path.join(HERE, "csrc", "qdc_b200.cu"), os.path.join(HERE, "csrc", "qdc_noalloc.cu")]
DEPS = SOURCES + [os.path.join(HERE, "csrc", "qdc_kernels.cuh"),
                  os.path.join(ROOT, "include", "qdc_b200.h")]


def nvcc():
    for cand in (os.environ.get("NVCC"), "/usr/local/cuda/bin/nvcc", "nvcc"):
        if cand and (os.path.isabs(cand) and os.path.exists(cand) or not os.path.isabs(cand)):
            return cand
    return "nvcc"


def needs_build():
    if not os.path.exists(LIB):
        return True
    t = os.path.getmtime(LIB)
    return any(os.path.getmtime(p) > t for p in DEPS)


def build(force=False):
    if not force and not needs_build():
        return LIB
    os.makedirs(OUT_DIR, exist_ok=True)
    cmd = [nvcc(), "-gencode", "arch=compute_100a,code=sm_100a", "-lineinfo", "-O3",
           "-std=c++17", "-shared", "-Xcompiler", "-fPIC,-fvisibility=hidden",
           "-Xptxas", "-v", "--expt-relaxed-constexpr",
           "-I" + os.path.join(ROOT, "include"), "-I" + os.path.join(HERE, "csrc"),
           "-DQDC_B200_BUILD", "-o", LIB] + SOURCES + ["-lcudart"]
    res = subprocess.run(cmd, capture_output=True, text=True)
    with open(os.path.join(OUT_DIR, "ptxas.txt"), "w") as f:
        f.write(res.stdout + res.stderr)
    if res.returncode != 0:
        noise = ("ptxas info", "    0 bytes stack", "ptxas info    : Function properties")
        lines = [l for l in (res.stdout + res.stderr).splitlines() if not l.startswith(noise)]
        sys.stderr.write("\n".join(lines) + "\n")
        raise RuntimeError("nvcc failed building libqdc_b200.so (full log: _build/ptxas.txt)")
    return LIB


if __name__ == "__main__":
    print(build(force=True))
