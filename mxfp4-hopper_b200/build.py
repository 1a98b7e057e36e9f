"""In-tree build of the B200 library and its torch binding.

  lib/libmxfp4_b200.so   the C-ABI library (include/mxfp4_b200.h): every CUDA
                         kernel, compiled for sm_100a only.
  omo<ext-suffix>.so     the `omo` torch extension: C++ host code with the
                         reference's operator names and keyword arguments
                         (code/kernel/ops.cu:27-43), calling the C ABI.

Usage: python mxfp4-hopper_b200/build.py [--force] [--no-omo] [-j N]
"""
from __future__ import annotations

import argparse
import concurrent.futures as cf
import os
import subprocess
import sys
import sysconfig
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / "csrc"
INC = ROOT / "include"
LIBDIR = PKG / "lib"
LIB = LIBDIR / "libmxfp4_b200.so"
BUILD = PKG / "_build"

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "-Xcompiler", "-Wall",
              "--expt-relaxed-constexpr", f"-I{INC}", f"-I{CSRC}"] + ARCH
CU_SOURCES = ["quantize.cu", "dequant.cu", "convert_col.cu", "fp8_token.cu", "ep.cu", "ep_p2p.cu",
              "ep_nccl.cu", "gemm_mxfp4.cu"]
CPP_SOURCES = ["capi_util.cpp", "host_pipeline.cpp"]


def _nvcc() -> str:
    home = os.environ.get("CUDA_HOME", "/usr/local/cuda")
    p = Path(home) / "bin" / "nvcc"
    return str(p) if p.exists() else "nvcc"


def _cxx() -> str:
    # The image's CC/CXX may point at a wrapper without OpenMP specs; /usr/bin/g++ is plain.
    return "/usr/bin/g++" if Path("/usr/bin/g++").exists() else "g++"


def _run(cmd):
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"build failed:\n{' '.join(map(str, cmd))}\n{r.stdout}\n{r.stderr}")
    return r


def _stale(out: Path, deps) -> bool:
    if not out.exists():
        return True
    t = out.stat().st_mtime
    return any(Path(d).stat().st_mtime > t for d in deps)


def build_lib(force: bool = False, jobs: int = 8, verbose: bool = False) -> Path:
    BUILD.mkdir(exist_ok=True)
    LIBDIR.mkdir(exist_ok=True)
    headers = list(CSRC.glob("*.cuh")) + list(CSRC.glob("*.h")) + list(INC.glob("*.h"))
    cmds, objs = [], []
    for s in CU_SOURCES + CPP_SOURCES:
        src = CSRC / s
        obj = BUILD / (s + ".o")
        objs.append(obj)
        if force or _stale(obj, [src] + headers):
            cmds.append([_nvcc(), "-c", str(src), "-o", str(obj)] + NVCC_FLAGS +
                        (["-x", "cu"] if s.endswith(".cu") else []))
    with cf.ThreadPoolExecutor(max_workers=jobs) as ex:
        for r in ex.map(_run, cmds):
            if verbose and r.stderr:
                print(r.stderr, file=sys.stderr)
    if force or cmds or not LIB.exists():
        _run([_nvcc(), "-shared", "-o", str(LIB)] + [str(o) for o in objs] + ARCH +
             ["-lcudart", "-ldl"])
    return LIB


def omo_path() -> Path:
    return PKG / f"omo{sysconfig.get_config_var('EXT_SUFFIX')}"


def build_omo(force: bool = False) -> Path:
    from torch.utils import cpp_extension as ce

    src = PKG / "omo_src" / "omo_ext.cpp"
    out = omo_path()
    if not force and not _stale(out, [src, INC / "mxfp4_b200.h", LIB]):
        return out
    inc = ce.include_paths(device_type="cuda") + [sysconfig.get_paths()["include"], str(INC)]
    libs = ce.library_paths(device_type="cuda")
    cmd = [_cxx(), "-shared", "-fPIC", "-O2", "-std=c++17", "-D_GLIBCXX_USE_CXX11_ABI=1",
           "-DTORCH_API_INCLUDE_EXTENSION_H", "-DTORCH_EXTENSION_NAME=omo", str(src), "-o", str(out)]
    cmd += [f"-I{p}" for p in inc] + [f"-L{p}" for p in libs] + [f"-Wl,-rpath,{p}" for p in libs]
    cmd += [f"-L{LIBDIR}", "-Wl,-rpath,$ORIGIN/lib", "-lmxfp4_b200", "-lc10", "-lc10_cuda",
            "-ltorch", "-ltorch_cpu", "-ltorch_cuda", "-ltorch_python", "-lcudart"]
    _run(cmd)
    return out


def build(force: bool = False, omo: bool = True, jobs: int = 8) -> None:
    build_lib(force=force, jobs=jobs)
    if omo:
        build_omo(force=force)


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--no-omo", action="store_true")
    ap.add_argument("-j", type=int, default=8)
    a = ap.parse_args()
    build(force=a.force, omo=not a.no_omo, jobs=a.j)
    print("built", LIB, "" if a.no_omo else omo_path())
