"""Build recipe of the B200 GPT library: csrc/*.cu (nvcc, sm_100a) and
csrc/*.cpp (host C++17) -> libitts_gpt_b200.so next to this file.

Run ``python build.py`` (or call ``build()``); objects go to ``_build/`` and
are rebuilt when a source or header is newer.  nvcc cross-compiles for
sm_100a without a GPU.
"""
from __future__ import annotations

import concurrent.futures as cf
import glob
import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")
OUT_DIR = os.path.join(HERE, "_build")
LIB = os.path.join(HERE, "libitts_gpt_b200.so")
INCLUDE = os.path.join(os.path.dirname(HERE), "include")
CUDA = os.environ.get("CUDA_HOME", "/usr/local/cuda")
NVCC = os.path.join(CUDA, "bin", "nvcc")
# The system compiler: an environment CXX may point at a wrapper toolchain.
HOST_CXX = "/usr/bin/g++" if os.path.exists("/usr/bin/g++") else "g++"
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVFLAGS = ["-std=c++17", "-O3", "-lineinfo", "-Xcompiler", "-fPIC", "-ccbin", HOST_CXX, "--expt-relaxed-constexpr",
           "-I", INCLUDE, "-I", CSRC]
CXXFLAGS = ["-std=c++17", "-O2", "-fPIC", "-Wall", "-I", INCLUDE, "-I", CSRC, "-I", os.path.join(CUDA, "include")]


def _deps():
    return [p for ext in ("*.h", "*.hpp", "*.cuh") for p in glob.glob(os.path.join(CSRC, ext))] + \
        glob.glob(os.path.join(INCLUDE, "*.h"))


def _stale(obj, src, deps):
    if not os.path.exists(obj):
        return True
    t = os.path.getmtime(obj)
    return any(os.path.getmtime(p) > t for p in [src] + deps)


def _compile(src, obj, verbose):
    if src.endswith(".cu"):
        cmd = [NVCC, *ARCH, *NVFLAGS, "-c", src, "-o", obj]
        if verbose:
            cmd.insert(1, "-Xptxas=-v")
    else:
        cmd = [HOST_CXX, *CXXFLAGS, "-c", src, "-o", obj]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"compile failed: {' '.join(cmd)}\n{r.stdout}\n{r.stderr}")
    return r.stderr


def build(verbose: bool = False, force: bool = False) -> str:
    os.makedirs(OUT_DIR, exist_ok=True)
    deps = _deps()
    srcs = sorted(glob.glob(os.path.join(CSRC, "*.cu")) + glob.glob(os.path.join(CSRC, "*.cpp")))
    objs, jobs = [], []
    for s in srcs:
        o = os.path.join(OUT_DIR, os.path.basename(s) + ".o")
        objs.append(o)
        if force or _stale(o, s, deps):
            jobs.append((s, o))
    with cf.ThreadPoolExecutor(max_workers=min(8, max(1, len(jobs)))) as ex:
        for (s, _), log in zip(jobs, ex.map(lambda j: _compile(j[0], j[1], verbose), jobs)):
            if verbose and log:
                print(f"--- {os.path.basename(s)}\n{log}", file=sys.stderr)
    if force or jobs or not os.path.exists(LIB) or any(os.path.getmtime(o) > os.path.getmtime(LIB) for o in objs):
        cmd = [NVCC, *ARCH, "-shared", "-ccbin", HOST_CXX, "-o", LIB, *objs]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link failed: {' '.join(cmd)}\n{r.stdout}\n{r.stderr}")
    build_op_server(force)
    return LIB


SERVER_SRC = os.path.join(HERE, "host", "gpt_op_server.cpp")
SERVER = os.path.join(HERE, "itts_gpt_op_server")


def build_op_server(force: bool = False) -> str:
    """The line-protocol `gpt` op server (host/gpt_op_server.cpp), linked
    against the library next to it."""
    deps = [SERVER_SRC, LIB, os.path.join(HERE, "host", "gpt_decoder.hpp"), os.path.join(CSRC, "mit2_bundle.hpp"),
            os.path.join(INCLUDE, "itts_gpt.h")]
    if not force and os.path.exists(SERVER) and all(os.path.getmtime(d) <= os.path.getmtime(SERVER) for d in deps):
        return SERVER
    cmd = [HOST_CXX, "-std=c++17", "-O2", "-Wall", "-I", INCLUDE, "-I", os.path.join(HERE, "host"), "-I", CSRC,
           "-I", os.path.join(CUDA, "include"), SERVER_SRC, "-L", HERE, "-litts_gpt_b200", "-Wl,-rpath,$ORIGIN",
           "-o", SERVER]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"op server build failed: {' '.join(cmd)}\n{r.stdout}\n{r.stderr}")
    return SERVER


if __name__ == "__main__":
    print(build(verbose="-v" in sys.argv, force="-f" in sys.argv))
