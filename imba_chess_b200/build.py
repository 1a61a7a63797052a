"""Build the in-tree shared library ``libimba_b200.so`` for sm_100a and the
host-path extension ``_hostpath``.

    python -m imba_chess_b200.build [--force] [--verbose]

Each ``csrc/*.cu`` is compiled by nvcc in parallel into ``_build/`` and the
objects are linked into ``imba_chess_b200/libimba_b200.so`` (a plain C-ABI
library; no torch headers).  Objects are rebuilt only when a source or header
is newer than the object.  ``host/hostpath.cpp`` (CPython API, the wave
service's request packing and response building) is compiled by g++ into
``imba_chess_b200/_hostpath<EXT_SUFFIX>``.
"""

from __future__ import annotations

import argparse
import concurrent.futures as cf
import glob
import os
import shutil
import subprocess
import sys
import sysconfig

PKG = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG)
CSRC = os.path.join(PKG, "csrc")
BUILD = os.path.join(PKG, "_build")
INCLUDE = os.path.join(ROOT, "include")
LIB = os.path.join(PKG, "libimba_b200.so")
HOST_SRC = os.path.join(PKG, "host", "hostpath.cpp")
HOST_EXT = os.path.join(PKG, "_hostpath" + (sysconfig.get_config_var("EXT_SUFFIX") or ".so"))
CHESS_SRC = os.path.join(PKG, "host", "chess.cpp")
CHESS_EXT = os.path.join(PKG, "_chess" + (sysconfig.get_config_var("EXT_SUFFIX") or ".so"))

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = [
    "-O3",
    "-std=c++17",
    "-lineinfo",
    "-Xcompiler",
    "-fPIC,-fvisibility=hidden",
    "-Xptxas",
    "-v",
    "--expt-relaxed-constexpr",
]


def nvcc_path() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found: the imba_b200 library cannot be built")


def _newest_header() -> float:
    hdrs = glob.glob(os.path.join(CSRC, "*.cuh")) + glob.glob(os.path.join(INCLUDE, "*.h"))
    return max((os.path.getmtime(h) for h in hdrs), default=0.0)


def _compile(nvcc: str, src: str, force: bool, verbose: bool) -> tuple[str, str]:
    obj = os.path.join(BUILD, os.path.basename(src)[:-3] + ".o")
    if not force and os.path.exists(obj):
        t = os.path.getmtime(obj)
        if t >= os.path.getmtime(src) and t >= _newest_header():
            return obj, ""
    cmd = [nvcc, *ARCH, *NVCC_FLAGS, "-I", INCLUDE, "-I", CSRC, "-c", src, "-o", obj]
    proc = subprocess.run(cmd, capture_output=True, text=True)
    if proc.returncode != 0:
        raise RuntimeError(f"nvcc failed for {src}:\n{proc.stdout}\n{proc.stderr}")
    return obj, (proc.stderr if verbose else "")


def build(force: bool = False, verbose: bool = False) -> str:
    """Compile every kernel source and link the shared library; returns its path."""
    nvcc = nvcc_path()
    os.makedirs(BUILD, exist_ok=True)
    sources = sorted(glob.glob(os.path.join(CSRC, "*.cu")))
    with cf.ThreadPoolExecutor(max_workers=min(8, len(sources))) as ex:
        results = list(ex.map(lambda s: _compile(nvcc, s, force, verbose), sources))
    objs = [o for o, _ in results]
    if verbose:
        for _, log in results:
            if log:
                sys.stderr.write(log)
    newest_obj = max(os.path.getmtime(o) for o in objs)
    if force or not os.path.exists(LIB) or os.path.getmtime(LIB) < newest_obj:
        tmp = LIB + ".tmp"
        cmd = [nvcc, *ARCH, "-shared", "-o", tmp, *objs, "-lcuda"]
        proc = subprocess.run(cmd, capture_output=True, text=True)
        if proc.returncode != 0:
            raise RuntimeError(f"link failed:\n{proc.stdout}\n{proc.stderr}")
        os.replace(tmp, LIB)
    return LIB


def _build_ext(src: str, ext: str, force: bool) -> str:
    if not force and os.path.exists(ext) and os.path.getmtime(ext) >= os.path.getmtime(src):
        return ext
    cxx = os.environ.get("CXX") or shutil.which("g++") or "g++"
    inc = sysconfig.get_paths()["include"]
    tmp = ext + ".tmp"
    cmd = [cxx, "-O2", "-std=c++17", "-shared", "-fPIC", "-fvisibility=hidden", "-pthread", "-I", inc, src, "-o", tmp]
    proc = subprocess.run(cmd, capture_output=True, text=True)
    if proc.returncode != 0:
        raise RuntimeError(f"host extension build failed ({src}):\n{proc.stdout}\n{proc.stderr}")
    os.replace(tmp, ext)
    return ext


def build_host(force: bool = False) -> str:
    """Compile the CPython host extensions (g++, -O2): the wave service's
    host path (``_hostpath``) and worker-side chess (``_chess``)."""
    _build_ext(CHESS_SRC, CHESS_EXT, force)
    return _build_ext(HOST_SRC, HOST_EXT, force)


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--verbose", action="store_true")
    a = ap.parse_args()
    print(build(force=a.force, verbose=a.verbose))
    print(build_host(force=a.force))


if __name__ == "__main__":
    main()
