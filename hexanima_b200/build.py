"""Build libhxdit.so in-tree with nvcc for sm_100a.

usage: python -m hexanima_b200.build [--force] [--jobs N]

Objects go to hexanima_b200/_build/ and are rebuilt when a source or header is newer.
"""
import argparse
import os
import subprocess
import sys
from concurrent.futures import ThreadPoolExecutor

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
BUILD = os.path.join(HERE, "_build")
LIB = os.path.join(HERE, "libhxdit.so")
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
SOURCES = ["gemm.cu", "gemm_wt.cu", "attn.cu", "attn_short.cu", "elem.cu", "repack.cu", "glue.cu", "sp.cu", "lora.cu", "lorasvd.cu", "adapter.cu", "expand.cu", "api.cpp"]
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC,-fvisibility=hidden", "-I" + os.path.join(ROOT, "include")]


def _headers():
    hs = [os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith((".h", ".cuh"))]
    hs.append(os.path.join(ROOT, "include", "hxdit.h"))
    return hs


def _stale(obj, src, headers):
    if not os.path.exists(obj):
        return True
    t = os.path.getmtime(obj)
    return any(os.path.getmtime(p) > t for p in [src] + headers)


def _compile(src, force, headers, verbose):
    obj = os.path.join(BUILD, os.path.splitext(src)[0] + ".o")
    path = os.path.join(CSRC, src)
    if not force and not _stale(obj, path, headers):
        return obj
    cmd = [NVCC] + ARCH + FLAGS + ["-c", path, "-o", obj]
    if verbose:
        cmd += ["-Xptxas", "-v"]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc failed for {src}:\n{r.stdout}\n{r.stderr}")
    if verbose and r.stderr:
        sys.stderr.write(r.stderr)
    return obj


def build(force=False, jobs=None, verbose=False):
    os.makedirs(BUILD, exist_ok=True)
    headers = _headers()
    with ThreadPoolExecutor(max_workers=jobs or len(SOURCES)) as ex:
        objs = list(ex.map(lambda s: _compile(s, force, headers, verbose), SOURCES))
    if force or not os.path.exists(LIB) or any(os.path.getmtime(o) > os.path.getmtime(LIB) for o in objs):
        cmd = [NVCC] + ARCH + ["-shared", "-cudart", "static", "-o", LIB] + objs + ["-ldl"]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
    _build_hxrun(force)
    return LIB


HXRUN = os.path.join(HERE, "hxrun")


def _build_hxrun(force=False):
    """The megarun-protocol CLI, linked against the in-tree libhxdit.so (rpath $ORIGIN)."""
    src = os.path.join(CSRC, "hxrun.cpp")
    if not force and os.path.exists(HXRUN) and os.path.getmtime(HXRUN) >= max(
            os.path.getmtime(src), os.path.getmtime(LIB), os.path.getmtime(os.path.join(ROOT, "include", "hxdit.h"))):
        return HXRUN
    cmd = ["g++", "-O2", "-std=c++17", "-I" + os.path.join(ROOT, "include"), src, "-L" + HERE, "-lhxdit",
           "-Wl,-rpath,$ORIGIN", "-o", HXRUN]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"hxrun build failed:\n{r.stdout}\n{r.stderr}")
    return HXRUN


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--jobs", type=int, default=None)
    ap.add_argument("-v", "--verbose", action="store_true")
    a = ap.parse_args()
    print(build(a.force, a.jobs, a.verbose))
