"""Ahead-of-time build of the two native libraries of this package.

* ``libxdna_b200.so`` -- the C-ABI kernel library (``include/b2.h``), CUDA
  sources under ``csrc/abi`` compiled by nvcc for sm_100a only.
* ``_C.so`` -- the PyTorch extension (``csrc/torch``): the PrivateUse1
  allocator, guard, hooks, aten registrations and Python bindings.  It links
  ``libxdna_b200.so`` through an ``$ORIGIN`` rpath.

Both land inside the package directory, so they travel with the source tree
and are imported from there (no JIT cache).  The reference builds its single
extension at import time with ``torch.utils.cpp_extension.load``
(xdna_train/_build.py:29-79); here nvcc and g++ run once, in parallel, and a
rebuild happens only when a source, header or flag changes.

Run ``python -m xdna_train._build`` (from the ``pytorch-xdna2_b200``
directory or with it on ``sys.path``) to build.
"""
from __future__ import annotations

import concurrent.futures as cf
import hashlib
import json
import os
import shutil
import subprocess
import sys
import sysconfig
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent                      # pytorch-xdna2_b200/
REPO = ROOT.parent
CSRC = ROOT / "csrc"
INCLUDE = REPO / "include"
BUILD = ROOT / "_build"
ABI_LIB = PKG / "libxdna_b200.so"
EXT_LIB = PKG / "_C.so"

CUDA_HOME = Path(os.environ.get("CUDA_HOME", "/usr/local/cuda"))
NVCC = CUDA_HOME / "bin" / "nvcc"
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ARCH + ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC",
                     "--expt-relaxed-constexpr", f"-I{INCLUDE}", f"-I{CSRC / 'abi'}"]


def _torch_flags():
    import torch
    import torch.utils.cpp_extension as ce

    inc = list(ce.include_paths()) + [str(CUDA_HOME / "include"), sysconfig.get_paths()["include"],
                                      str(INCLUDE), str(CSRC / "torch")]
    abi = int(torch._C._GLIBCXX_USE_CXX11_ABI)
    cflags = ["-O2", "-std=c++17", "-fPIC", "-fvisibility=hidden", f"-D_GLIBCXX_USE_CXX11_ABI={abi}",
              "-DTORCH_API_INCLUDE_EXTENSION_H", "-DTORCH_EXTENSION_NAME=_C",
              "-Wno-unused-parameter"] + [f"-I{p}" for p in inc]
    libdirs = list(ce.library_paths())
    ldflags = [f"-L{d}" for d in libdirs] + [f"-Wl,-rpath,{d}" for d in libdirs] + [
        "-lc10", "-lc10_cuda", "-ltorch", "-ltorch_cpu", "-ltorch_cuda", "-ltorch_python",
        f"-L{PKG}", "-lxdna_b200", "-Wl,-rpath,$ORIGIN"]
    return cflags, ldflags


def _hash(paths, extra) -> str:
    h = hashlib.sha256()
    for p in sorted(paths):
        h.update(str(p.name).encode())
        h.update(p.read_bytes())
    h.update(json.dumps(extra).encode())
    return h.hexdigest()[:16]


def _run(cmd):
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"build step failed: {' '.join(map(str, cmd))}\n{r.stdout}\n{r.stderr}")
    return r.stdout + r.stderr


def _stamp_ok(stamp: Path, key: str, out: Path) -> bool:
    return out.is_file() and stamp.is_file() and stamp.read_text() == key


def build_abi(force: bool = False, verbose: bool = False) -> Path:
    srcs = sorted((CSRC / "abi").glob("*.cu"))
    deps = srcs + sorted((CSRC / "abi").glob("*.cuh")) + sorted(INCLUDE.glob("*.h"))
    key = _hash(deps, NVCC_FLAGS)
    stamp = BUILD / "abi.stamp"
    if not force and _stamp_ok(stamp, key, ABI_LIB):
        return ABI_LIB
    if not NVCC.is_file():
        raise RuntimeError(f"nvcc not found at {NVCC}")
    odir = BUILD / "abi"
    odir.mkdir(parents=True, exist_ok=True)
    extra = ["-Xptxas", "-v"] if verbose else []

    def one(src: Path) -> Path:
        obj = odir / (src.stem + ".o")
        out = _run([str(NVCC), *NVCC_FLAGS, *extra, "-c", str(src), "-o", str(obj)])
        if verbose and out.strip():
            print(out)
        return obj

    with cf.ThreadPoolExecutor(max_workers=min(8, os.cpu_count() or 4)) as ex:
        objs = list(ex.map(one, srcs))
    tmp = ABI_LIB.with_suffix(".so.tmp")
    _run([str(NVCC), *ARCH, "-shared", "-Xcompiler", "-fPIC", "-o", str(tmp), *map(str, objs)])
    os.replace(tmp, ABI_LIB)
    stamp.write_text(key)
    return ABI_LIB


def build_ext(force: bool = False) -> Path:
    build_abi(force=force)
    cflags, ldflags = _torch_flags()
    srcs = sorted((CSRC / "torch").glob("*.cpp"))
    deps = srcs + sorted((CSRC / "torch").glob("*.h")) + sorted(INCLUDE.glob("*.h"))
    key = _hash(deps, cflags + ldflags)
    stamp = BUILD / "ext.stamp"
    if not force and _stamp_ok(stamp, key, EXT_LIB):
        return EXT_LIB
    odir = BUILD / "ext"
    odir.mkdir(parents=True, exist_ok=True)
    cxx = os.environ.get("CXX_B2", shutil.which("g++") or "g++")
    if cxx.startswith("/opt/gcc"):
        cxx = "/usr/bin/g++"

    def one(src: Path) -> Path:
        obj = odir / (src.stem + ".o")
        _run([cxx, *cflags, "-c", str(src), "-o", str(obj)])
        return obj

    with cf.ThreadPoolExecutor(max_workers=min(8, os.cpu_count() or 4)) as ex:
        objs = list(ex.map(one, srcs))
    tmp = EXT_LIB.with_suffix(".so.tmp")
    _run([cxx, "-shared", "-o", str(tmp), *map(str, objs), *ldflags])
    os.replace(tmp, EXT_LIB)
    stamp.write_text(key)
    return EXT_LIB


def build(force: bool = False) -> None:
    build_abi(force=force)
    if sorted((CSRC / "torch").glob("*.cpp")):
        build_ext(force=force)


if __name__ == "__main__":
    build(force="--force" in sys.argv)
    print(ABI_LIB)
    print(EXT_LIB)
