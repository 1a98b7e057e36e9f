"""B200 (sm_100a) MXFP4 quantize / dequantize / convert library.

Layers, bottom-up:
  lib/libmxfp4_b200.so  CUDA kernels behind the C ABI of include/mxfp4_b200.h
  mxfp4_b200.capi       ctypes binding of that C ABI (no torch types)
  omo                   C++ torch extension with the reference's op names
  omo_python_api        the reference's Python wrappers (allocation, padding,
                        splits) on top of `omo`
  mxfp4_b200.ep         MoE expert-parallel dispatch / combine with MXFP4
                        payloads over torch.distributed (NCCL)
"""
from __future__ import annotations

import sys
from pathlib import Path

PKG_DIR = Path(__file__).resolve().parent.parent

if str(PKG_DIR) not in sys.path:
    sys.path.insert(0, str(PKG_DIR))

__all__ = ["PKG_DIR", "build"]


def build(force: bool = False) -> None:
    """Compile libmxfp4_b200.so and the `omo` extension in-tree."""
    import importlib.util

    spec = importlib.util.spec_from_file_location("_mxb_build", PKG_DIR / "build.py")
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    mod.build(force=force)
