"""Builds libspeech_sampler_b200.so in-tree: every csrc/*.cu for sm_100a with nvcc, linked with the
static CUDA runtime and hidden visibility except the C ABI of include/speech_sampler_b200.h.

Also builds the wait-limit test library, libspeech_sampler_b200_waittest.so: the same sources with
SSB_WAIT_TEST defined, whose bounded waits give up after about 2 ms and whose top-k kernel never
issues one refill of row 0 (a stage that nothing fills), so that a test can check that a wait that runs
out becomes SSB_ROW_DEVICE_TIMEOUT without a fault or a hang. It is test infrastructure only.

    python speech.cpp_b200/speech_build.py          # incremental
    python speech.cpp_b200/speech_build.py --force  # rebuild everything
"""
from __future__ import annotations

import argparse
import concurrent.futures as cf
import os
import shutil
import subprocess
import sys

PKG = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG)
CSRC = os.path.join(PKG, "csrc")
OBJ = os.path.join(PKG, "_build")
LIB = os.path.join(PKG, "libspeech_sampler_b200.so")
OBJ_WAITTEST = os.path.join(PKG, "_build_waittest")
LIB_WAITTEST = os.path.join(PKG, "libspeech_sampler_b200_waittest.so")
INCLUDE = os.path.join(ROOT, "include")

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ARCH + ["-O3", "-lineinfo", "-std=c++17", "--expt-relaxed-constexpr", "-Xcompiler",
                     "-fPIC,-fvisibility=hidden", f"-I{INCLUDE}", f"-I{CSRC}"]


def nvcc() -> str:
    for c in (os.environ.get("NVCC"), "/usr/local/cuda/bin/nvcc", shutil.which("nvcc")):
        if c and os.path.exists(c):
            return c
    raise RuntimeError("nvcc not found")


def sources():
    return sorted(os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith(".cu"))


def headers():
    hs = [os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith((".cuh", ".h"))]
    hs += [os.path.join(INCLUDE, f) for f in os.listdir(INCLUDE) if f.endswith((".h", ".hpp"))]
    return hs


def _stale(target: str, deps) -> bool:
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(d) > t for d in deps)


def build(force: bool = False, verbose: bool = False, ptxas_info: bool = False, waittest: bool = False) -> str:
    objdir, lib = (OBJ_WAITTEST, LIB_WAITTEST) if waittest else (OBJ, LIB)
    os.makedirs(objdir, exist_ok=True)
    cc = nvcc()
    hdrs = headers()
    jobs = []
    extra = ["-DSSB_WAIT_TEST"] if waittest else []
    for src in sources():
        obj = os.path.join(objdir, os.path.basename(src)[:-3] + ".o")
        if force or ptxas_info or _stale(obj, [src] + hdrs):
            cmd = [cc] + NVCC_FLAGS + extra + (["-Xptxas", "-v"] if ptxas_info else []) + ["-c", src, "-o", obj]
            jobs.append((src, cmd))
    objs = [os.path.join(objdir, os.path.basename(s)[:-3] + ".o") for s in sources()]

    def run(job):
        src, cmd = job
        if verbose:
            print(" ".join(cmd), flush=True)
        r = subprocess.run(cmd, capture_output=True, text=True)
        return src, r

    if jobs:
        with cf.ThreadPoolExecutor(max_workers=min(8, len(jobs))) as ex:
            for src, r in ex.map(run, jobs):
                if r.returncode != 0:
                    sys.stderr.write(r.stdout + r.stderr)
                    raise RuntimeError(f"nvcc failed on {src}")
                if ptxas_info or verbose:
                    sys.stderr.write(r.stderr)
    if force or jobs or _stale(lib, objs):
        cmd = [cc] + ARCH + ["-shared", "-cudart", "static", "-o", lib] + objs + ["-lpthread"]
        if verbose:
            print(" ".join(cmd), flush=True)
        subprocess.run(cmd, check=True)
    return lib


NCCL_SRC = os.path.join(CSRC, "ssb_nccl.cpp")
LIB_NCCL = os.path.join(PKG, "libspeech_sampler_b200_nccl.so")


def nccl_dirs():
    """(include, lib) of the NCCL that torch.distributed loads (the wheel's), else the system's."""
    try:
        import nvidia.nccl as n
        base = os.path.dirname(n.__file__) if n.__file__ else list(n.__path__)[0]
        inc, lib = os.path.join(base, "include"), os.path.join(base, "lib")
        if os.path.exists(os.path.join(inc, "nccl.h")):
            return inc, lib
    except Exception:
        pass
    return "/usr/include", "/usr/lib/x86_64-linux-gnu"


def build_nccl(force: bool = False, verbose: bool = False) -> str:
    """libspeech_sampler_b200_nccl.so: the NCCL host code of the vocabulary-sharded draw, linked with the
    engine (found next to it at run time) and libnccl.so.2."""
    inc, libdir = nccl_dirs()
    deps = [NCCL_SRC, LIB, os.path.join(INCLUDE, "speech_sampler_b200_nccl.h"), os.path.join(INCLUDE, "speech_sampler_b200.h")]
    if not force and not _stale(LIB_NCCL, deps):
        return LIB_NCCL
    cmd = [nvcc()] + ARCH + ["-O2", "-std=c++17", "-shared", "-Xcompiler", "-fPIC", f"-I{INCLUDE}", f"-I{inc}", NCCL_SRC,
           "-o", LIB_NCCL, f"-L{PKG}", "-lspeech_sampler_b200", f"-L{libdir}", "-l:libnccl.so.2",
           "-Xlinker", "-rpath,$ORIGIN", "-Xlinker", f"-rpath,{libdir}"]
    if verbose:
        print(" ".join(cmd), flush=True)
    subprocess.run(cmd, check=True)
    return LIB_NCCL


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--verbose", action="store_true")
    ap.add_argument("--ptxas-info", action="store_true")
    args = ap.parse_args()
    print(build(force=args.force, verbose=args.verbose, ptxas_info=args.ptxas_info))
    print(build(force=args.force, verbose=args.verbose, waittest=True))
    print(build_nccl(force=args.force, verbose=args.verbose))
