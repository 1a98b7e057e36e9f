"""Test infrastructure only: build the reference's own CUDA kernels into a GPU oracle.

Compiles the six kernel sources of the reference (code/kernel/*.cu, unmodified,
read in place from the reference checkout) for sm_100a together with
`oracle/ref_shim/` (stand-ins for the two headers the reference includes but
does not ship) and `oracle/ref_bind.cpp` (a pybind module standing in for
code/kernel/ops.cu). The result is `oracle/_ref/omo_ref*.so`, which only the
GPU parity tests and the golden-fixture generator import. Nothing is copied
from the reference into this repository; the objects land under `oracle/_ref/`,
which git ignores.

Flags follow the reference build (code/kernel/setup.py:34-56 plus torch's
BuildExtension defaults): no fast-math, so log2f/exp2f/division are the
IEEE-accurate versions the reference kernels were written against.

Usage: python oracle/build_ref.py [--ref ROOT] [-j JOBS]
"""
from __future__ import annotations

import argparse
import concurrent.futures as cf
import os
import subprocess
import sys
import sysconfig
from pathlib import Path

HERE = Path(__file__).resolve().parent
OUT = HERE / "_ref"


def reference_root() -> Path:
    """Where the reference checkout is: $MXFP4_REFERENCE_ROOT, else a directory
    named `reference` next to this repository's own directory."""
    env = os.environ.get("MXFP4_REFERENCE_ROOT")
    return Path(env) if env else HERE.parent.parent / "reference"
KERNELS = [
    "per_token_quant_mxfp4.cu",
    "per_token_Mxfp4ToBf16_dequant.cu",
    "per_token_Mxfp4ToFp8.cu",
    "per_token_Mxfp4ToFp8_col.cu",
    "per_token_Mxfp4RowToBf16ToFp8Col.cu",
    "per_token_Mxfp4RowToBf16ToFp8Col_msplit.cu",
]


def _torch_paths():
    from torch.utils import cpp_extension as ce

    inc = ce.include_paths(device_type="cuda") + [sysconfig.get_paths()["include"]]
    lib = ce.library_paths(device_type="cuda")
    return inc, lib


def _run(cmd):
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"command failed: {' '.join(cmd)}\n{r.stdout}\n{r.stderr}")
    return r


def build(ref_root: Path, jobs: int = 6, verbose: bool = True) -> Path:
    src_dir = ref_root / "code" / "kernel"
    if not src_dir.is_dir():
        raise FileNotFoundError(f"reference kernel sources not found under {src_dir}")
    OUT.mkdir(parents=True, exist_ok=True)
    inc, lib = _torch_paths()
    incs = [f"-I{HERE / 'ref_shim'}", f"-I{src_dir}"] + [f"-I{p}" for p in inc]
    defs = ["-DTORCH_API_INCLUDE_EXTENSION_H", "-DTORCH_EXTENSION_NAME=omo_ref",
            "-D_GLIBCXX_USE_CXX11_ABI=1"]
    nvcc = [
        "nvcc", "-c", "-std=c++17", "-O3", "-Xcompiler", "-fPIC",
        "-gencode", "arch=compute_100a,code=sm_100a",
        "-D__CUDA_NO_HALF_OPERATORS__", "-D__CUDA_NO_HALF_CONVERSIONS__",
        "-D__CUDA_NO_BFLOAT16_CONVERSIONS__", "-D__CUDA_NO_HALF2_OPERATORS__",
        "--expt-relaxed-constexpr", "-DENABLE_BF16", "-DENABLE_FP16", "-DENABLE_FP8",
        "-w",
    ] + defs + incs

    jobs_list = []
    for k in KERNELS:
        src = src_dir / k
        obj = OUT / (k + ".o")
        if obj.exists() and obj.stat().st_mtime > src.stat().st_mtime and \
                obj.stat().st_mtime > (HERE / "ref_shim" / "utils.h").stat().st_mtime:
            continue
        jobs_list.append(nvcc + [str(src), "-o", str(obj)])
    bind_obj = OUT / "ref_bind.o"
    if not bind_obj.exists() or bind_obj.stat().st_mtime < (HERE / "ref_bind.cpp").stat().st_mtime:
        jobs_list.append(["g++", "-c", "-std=c++17", "-O2", "-fPIC", "-w"] + defs + incs +
                         [str(HERE / "ref_bind.cpp"), "-o", str(bind_obj)])
    with cf.ThreadPoolExecutor(max_workers=jobs) as ex:
        for cmd in jobs_list:
            if verbose:
                print("[build_ref]", os.path.basename(cmd[-3]), flush=True)
        list(ex.map(_run, jobs_list))

    suffix = sysconfig.get_config_var("EXT_SUFFIX")
    so = OUT / f"omo_ref{suffix}"
    objs = [str(OUT / (k + ".o")) for k in KERNELS] + [str(bind_obj)]
    link = ["g++", "-shared", "-o", str(so)] + objs + [f"-L{p}" for p in lib] + [
        f"-Wl,-rpath,{p}" for p in lib] + ["-lc10", "-lc10_cuda", "-ltorch", "-ltorch_cpu",
                                           "-ltorch_cuda", "-ltorch_python", "-lcudart"]
    _run(link)
    if verbose:
        print("[build_ref] wrote", so)
    return so


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref", default=str(reference_root()))
    ap.add_argument("-j", type=int, default=6)
    a = ap.parse_args()
    build(Path(a.ref), jobs=a.j)
    sys.exit(0)
