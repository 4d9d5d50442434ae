"""Build libtinybrain_cuda.so in-tree with nvcc for sm_100a.

Usage: python -m tinybrain_b200.build  (or tinybrain_b200.build.build()).
The library is written next to this file so it travels with the source tree.
"""
import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")
ROOT = os.path.dirname(HERE)
LIB = os.path.join(HERE, "libtinybrain_cuda.so")
SOURCES = ["tb_gemv.cu", "tb_attention.cu", "tb_quant.cu", "tb_step.cu", "tb_flow.cu", "tb_nccl.cu", "tb_sampler.cu", "tb_runtime.cu"]
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def nvcc():
    for cand in (os.environ.get("NVCC"), "/usr/local/cuda/bin/nvcc", "nvcc"):
        if cand and (os.path.isabs(cand) and os.path.exists(cand) or not os.path.isabs(cand)):
            return cand
    return "nvcc"


def _stale(outputs, inputs):
    if not all(os.path.exists(o) for o in outputs):
        return True
    t = min(os.path.getmtime(o) for o in outputs)
    return any(os.path.getmtime(i) > t for i in inputs)


def build(verbose=False, force=False, jobs=None):
    build_dir = os.path.join(HERE, "_build")
    os.makedirs(build_dir, exist_ok=True)
    headers = [os.path.join(CSRC, h) for h in os.listdir(CSRC) if h.endswith((".h", ".cuh"))]
    headers.append(os.path.join(ROOT, "include", "tinybrain_cuda.h"))
    common = [nvcc(), *ARCH, "-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC",
              "-I", os.path.join(ROOT, "include"), "-Xptxas", "-v" if verbose else "-O3"]
    objs, procs = [], []
    for src in SOURCES:
        s = os.path.join(CSRC, src)
        o = os.path.join(build_dir, src.replace(".cu", ".o"))
        objs.append(o)
        if force or _stale([o], [s] + headers):
            cmd = common + ["-c", s, "-o", o]
            procs.append((src, subprocess.Popen(cmd, stdout=subprocess.PIPE, stderr=subprocess.STDOUT)))
    failed = []
    for src, p in procs:
        out, _ = p.communicate()
        if verbose or p.returncode != 0:
            sys.stdout.write(out.decode(errors="replace"))
        if p.returncode != 0:
            failed.append(src)
    if failed:
        raise RuntimeError("nvcc failed for: " + ", ".join(failed))
    if force or _stale([LIB], objs):
        cmd = [nvcc(), *ARCH, "-shared", "-cudart", "static", "-o", LIB, *objs, "-lpthread", "-ldl"]
        subprocess.check_call(cmd)
    return LIB


if __name__ == "__main__":
    print(build(verbose="-v" in sys.argv, force="-f" in sys.argv))
