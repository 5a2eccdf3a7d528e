"""Build the engine's C-ABI shared library, ``muon_sr_b200/libmuon_sr_b200.so``, with nvcc.

    python -m muon_sr_b200.build [--verbose-ptxas] [--force]

Every CUDA source under ``csrc/`` is compiled for sm_100a only
(``-gencode arch=compute_100a,code=sm_100a``) and linked with the static CUDA runtime into
one in-tree shared object that the Python layer loads with ctypes. The elementwise and
8-bit sources are compiled with ``--fmad=false`` so no multiply-add is contracted (their
results are bit-compared with the reference). nvcc cross-compiles without a GPU.
"""
import argparse
import concurrent.futures as cf
import os
import shutil
import subprocess
import sys

PKG = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(PKG, "csrc")
BUILD = os.path.join(PKG, "_build")
LIB = os.path.join(PKG, "libmuon_sr_b200.so")
INCLUDE = os.path.join(os.path.dirname(PKG), "include")

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
COMMON = ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC,-O2", "--expt-relaxed-constexpr", "-I", INCLUDE]
NO_FMA = {"elementwise.cu", "adamw8bit.cu"}


def nvcc():
    path = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not os.path.exists(path):
        raise RuntimeError("nvcc not found; the CUDA 12.9 toolkit is required to build muon_sr_b200")
    return path


def sources():
    return sorted(f for f in os.listdir(CSRC) if f.endswith(".cu"))


def _deps_mtime():
    files = [os.path.join(CSRC, f) for f in os.listdir(CSRC)] + [os.path.join(INCLUDE, f) for f in os.listdir(INCLUDE)]
    return max(os.path.getmtime(f) for f in files)


def build(force: bool = False, verbose_ptxas: bool = False) -> str:
    if not force and os.path.exists(LIB) and os.path.getmtime(LIB) >= _deps_mtime():
        return LIB
    os.makedirs(BUILD, exist_ok=True)
    cc = nvcc()

    def compile_one(src):
        obj = os.path.join(BUILD, src.replace(".cu", ".o"))
        cmd = [cc, *ARCH, *COMMON, "-c", os.path.join(CSRC, src), "-o", obj]
        if src in NO_FMA:
            cmd.insert(1, "--fmad=false")
        if verbose_ptxas:
            cmd.insert(1, "-Xptxas=-v")
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"nvcc failed on {src}:\n{r.stdout}\n{r.stderr}")
        return obj, r.stderr

    with cf.ThreadPoolExecutor(max_workers=min(8, os.cpu_count() or 1)) as ex:
        results = list(ex.map(compile_one, sources()))
    if verbose_ptxas:
        for obj, err in results:
            sys.stderr.write(f"== {os.path.basename(obj)}\n{err}")
    tmp = LIB + ".tmp"
    cmd = [cc, *ARCH, "-shared", "-cudart", "static", "-o", tmp, *[o for o, _ in results]]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc link failed:\n{r.stdout}\n{r.stderr}")
    os.replace(tmp, LIB)
    return LIB


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--verbose-ptxas", action="store_true")
    args = ap.parse_args()
    print(build(force=args.force, verbose_ptxas=args.verbose_ptxas))


if __name__ == "__main__":
    main()
