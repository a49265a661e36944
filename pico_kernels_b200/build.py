"""Build libpico_b200.so in-tree with nvcc for sm_100a.

    python -m pico_kernels_b200.build [--force] [--verbose]

Each ``csrc/*.cu`` compiles to an object under ``_build/`` (in parallel, and
only when it or a header changed), then everything links into
``pico_kernels_b200/libpico_b200.so``. No fast-math: the quantizers rely on
IEEE fp32 division for bit-exact parity. Then ``csrc/pyfast.cpp`` compiles
with the host compiler into the CPython module ``_pkfast`` beside it, the
fast-call entry points of the hottest calls (ctypes remains the path for
the rest, and for all calls when Python's headers are missing), and
``csrc/pytorch_fast.cpp`` against torch's headers into ``_pktorch``, which
makes the tensor checks of ``int4_gemm`` / ``int4_gemm_host`` in C++.
"""

from __future__ import annotations

import argparse
import os
import shutil
import subprocess
import sys
import sysconfig
from concurrent.futures import ThreadPoolExecutor
from pathlib import Path

PKG = Path(__file__).resolve().parent
CSRC = PKG / "csrc"
INCLUDE = PKG.parent / "include"
BUILD = PKG.parent / "_build"
LIB = PKG / "libpico_b200.so"
FAST = PKG / ("_pkfast" + (sysconfig.get_config_var("EXT_SUFFIX") or ".so"))
TFAST = PKG / ("_pktorch" + (sysconfig.get_config_var("EXT_SUFFIX") or ".so"))

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = [
    "-O3", "-std=c++17", "-lineinfo", "--expt-relaxed-constexpr",
    "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden",
    "-Xptxas", "-warn-spills",
    f"-I{CSRC}", f"-I{INCLUDE}",
]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found; set NVCC")


def _headers_mtime() -> float:
    hs = list(CSRC.glob("*.h")) + list(CSRC.glob("*.cuh")) + list(INCLUDE.glob("*.h"))
    return max((h.stat().st_mtime for h in hs), default=0.0)


def build(force: bool = False, verbose: bool = False) -> Path:
    BUILD.mkdir(exist_ok=True)
    sources = sorted(CSRC.glob("*.cu"))
    hdr = _headers_mtime()
    cc = nvcc()

    def compile_one(src: Path) -> Path:
        obj = BUILD / (src.stem + ".o")
        if not force and obj.exists() and obj.stat().st_mtime >= max(src.stat().st_mtime, hdr):
            return obj
        cmd = [cc, *ARCH, *NVCC_FLAGS, "-c", str(src), "-o", str(obj)]
        if verbose:
            cmd += ["-Xptxas", "-v"]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"nvcc failed on {src.name}:\n{r.stdout}\n{r.stderr}")
        if verbose and (r.stdout or r.stderr):
            print(f"== {src.name}\n{r.stdout}{r.stderr}", file=sys.stderr)
        return obj

    with ThreadPoolExecutor(max_workers=min(8, len(sources))) as ex:
        objs = list(ex.map(compile_one, sources))
    if force or not LIB.exists() or LIB.stat().st_mtime < max(o.stat().st_mtime for o in objs):
        tmp = LIB.with_suffix(".so.tmp")
        cmd = [cc, *ARCH, "-shared", "-o", str(tmp), *map(str, objs), "-lcudart_static",
               "-ldl", "-lrt", "-lpthread", "-Xlinker", "-soname=libpico_b200.so"]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
        os.replace(tmp, LIB)
    build_fast(force)
    build_torch_fast(force)
    return LIB


def build_fast(force: bool = False) -> Path | None:
    """The CPython module _pkfast (csrc/pyfast.cpp), linked against the
    library by its soname with an $ORIGIN run path; None without headers."""
    src = CSRC / "pyfast.cpp"
    inc = sysconfig.get_paths().get("include")
    cxx = shutil.which("g++") or shutil.which("c++")
    if not inc or not (Path(inc) / "Python.h").exists() or cxx is None:
        return None
    newest = max(src.stat().st_mtime, LIB.stat().st_mtime, (INCLUDE / "pico_b200.h").stat().st_mtime)
    if not force and FAST.exists() and FAST.stat().st_mtime >= newest:
        return FAST
    tmp = FAST.with_suffix(".tmp")
    cmd = [cxx, "-O2", "-std=c++17", "-fPIC", "-shared", f"-I{inc}", f"-I{INCLUDE}", str(src),
           "-o", str(tmp), f"-L{PKG}", "-lpico_b200", "-Wl,-rpath,$ORIGIN"]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"host compiler failed on {src.name}:\n{r.stdout}\n{r.stderr}")
    os.replace(tmp, FAST)
    return FAST


def build_torch_fast(force: bool = False) -> Path | None:
    """The CPython module _pktorch (csrc/pytorch_fast.cpp): the tensor checks
    of int4_gemm / int4_gemm_host in C++ against torch's headers and
    libraries, linked like _pkfast; None without Python's or torch's headers."""
    import torch  # noqa: PLC0415

    src = CSRC / "pytorch_fast.cpp"
    inc = sysconfig.get_paths().get("include")
    cxx = shutil.which("g++") or shutil.which("c++")
    tdir = Path(torch.__file__).resolve().parent
    cuda_inc = Path(os.environ.get("CUDA_HOME", "/usr/local/cuda")) / "include"
    if (not inc or not (Path(inc) / "Python.h").exists() or cxx is None
            or not (tdir / "include" / "torch").is_dir() or not (cuda_inc / "cuda.h").exists()):
        return None
    newest = max(src.stat().st_mtime, LIB.stat().st_mtime, (INCLUDE / "pico_b200.h").stat().st_mtime)
    if not force and TFAST.exists() and TFAST.stat().st_mtime >= newest:
        return TFAST
    tmp = TFAST.with_suffix(".tmp")
    abi = int(bool(getattr(torch._C, "_GLIBCXX_USE_CXX11_ABI", True)))
    tlib = tdir / "lib"
    cmd = [cxx, "-O2", "-std=c++17", "-fPIC", "-shared", f"-D_GLIBCXX_USE_CXX11_ABI={abi}",
           f"-I{inc}", f"-I{INCLUDE}", f"-I{tdir / 'include'}",
           f"-I{tdir / 'include' / 'torch' / 'csrc' / 'api' / 'include'}", f"-I{cuda_inc}",
           str(src), "-o", str(tmp), f"-L{PKG}", "-lpico_b200", f"-L{tlib}", "-ltorch_python",
           "-ltorch", "-ltorch_cpu", "-lc10", "-lc10_cuda", "-Wl,-rpath,$ORIGIN",
           f"-Wl,-rpath,{tlib}"]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"host compiler failed on {src.name}:\n{r.stdout}\n{r.stderr}")
    os.replace(tmp, TFAST)
    return TFAST


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--verbose", action="store_true", help="print ptxas register/smem usage")
    args = ap.parse_args()
    print(build(force=args.force, verbose=args.verbose))


if __name__ == "__main__":
    main()
