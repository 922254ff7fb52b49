"""Builds the in-tree CUDA library ds_ocr_b200/libds_cuda.so for sm_100a.

nvcc compiles every .cu under csrc/ (plus the host C file synth.c) with
-gencode arch=compute_100a,code=sm_100a into one shared library exporting the
C ABI of include/ds_cuda.h. Runs without a GPU (cross-compilation).
"""
import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
LIB = os.path.join(HERE, "libds_cuda.so")
BUILD = os.path.join(ROOT, "_build")

NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC",
    "--expt-relaxed-constexpr",
]


def _nvcc():
    for c in (os.environ.get("NVCC"), "/usr/local/cuda/bin/nvcc", "nvcc"):
        if c and (os.path.isabs(c) and os.path.exists(c) or not os.path.isabs(c)):
            return c
    return "nvcc"


def sources():
    cu = sorted(f for f in os.listdir(CSRC) if f.endswith(".cu"))
    return [os.path.join(CSRC, f) for f in cu]


def _stale(out, deps):
    if not os.path.exists(out):
        return True
    t = os.path.getmtime(out)
    return any(os.path.getmtime(d) > t for d in deps)


def build(verbose=False, force=False):
    os.makedirs(BUILD, exist_ok=True)
    hdrs = [os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith((".cuh", ".h"))]
    hdrs.append(os.path.join(ROOT, "include", "ds_cuda.h"))
    objs = []
    procs = []
    for src in sources():
        obj = os.path.join(BUILD, os.path.basename(src) + ".o")
        objs.append(obj)
        if force or _stale(obj, [src] + hdrs):
            cmd = [_nvcc(), *NVCC_FLAGS, "-I", CSRC, "-I", os.path.join(ROOT, "include"), "-c", src, "-o", obj]
            if verbose:
                print(" ".join(cmd))
            procs.append((src, subprocess.Popen(cmd, stdout=subprocess.PIPE, stderr=subprocess.STDOUT)))
    synth_o = os.path.join(BUILD, "synth.c.o")
    synth_c = os.path.join(CSRC, "synth.c")
    if force or _stale(synth_o, [synth_c]):
        procs.append((synth_c, subprocess.Popen(
            ["gcc", "-O2", "-fPIC", "-c", synth_c, "-o", synth_o],
            stdout=subprocess.PIPE, stderr=subprocess.STDOUT)))
    failed = []
    for src, p in procs:
        out, _ = p.communicate()
        if p.returncode != 0:
            failed.append((src, out.decode(errors="replace")))
        elif verbose and out:
            print(out.decode(errors="replace"))
    if failed:
        for src, out in failed:
            sys.stderr.write(f"--- {src}\n{out}\n")
        raise RuntimeError("nvcc failed for: " + ", ".join(s for s, _ in failed))
    objs.append(synth_o)
    if force or _stale(LIB, objs):
        cmd = [_nvcc(), "-shared", "-gencode", "arch=compute_100a,code=sm_100a", "-o", LIB, *objs,
               "-lcudart", "-lcuda", "-lpthread", "-ldl", "-lm"]
        if verbose:
            print(" ".join(cmd))
        subprocess.check_call(cmd)
    return LIB


if __name__ == "__main__":
    build(verbose="-v" in sys.argv, force="-f" in sys.argv)
    print(LIB)
