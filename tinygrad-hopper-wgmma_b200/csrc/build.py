"""Build ``hopper_wgmma/lib/libsm100_gemm.so`` from the CUDA sources in this directory (nvcc, sm_100a only).

    python tinygrad-hopper-wgmma_b200/csrc/build.py [--force]

The library links the CUDA runtime statically and fetches the one driver entry point it needs at run time, so it
loads on machines without a GPU driver (the CPU tests check its exports there)."""
from __future__ import annotations

import argparse
import os
import shutil
import subprocess
import sys
from pathlib import Path

CSRC = Path(__file__).resolve().parent
PKG = CSRC.parent / "hopper_wgmma"
INCLUDE = CSRC.parent.parent / "include"
OUT = PKG / "lib" / "libsm100_gemm.so"
SOURCES = [CSRC / "capi.cu"]
DEPS = SOURCES + [CSRC / "gemm_kernels.cuh", CSRC / "ptx.cuh", INCLUDE / "sm100_gemm.h"]
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def nvcc() -> str:
  for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
    if cand and Path(cand).exists(): return cand
  raise RuntimeError("nvcc not found (set NVCC or add /usr/local/cuda/bin to PATH)")


def up_to_date() -> bool:
  return OUT.exists() and all(OUT.stat().st_mtime >= d.stat().st_mtime for d in DEPS)


def build(force: bool = False, verbose: bool = False) -> Path:
  if not force and up_to_date(): return OUT
  OUT.parent.mkdir(parents=True, exist_ok=True)
  tmp = OUT.with_suffix(".so.tmp")
  cmd = [nvcc(), *ARCH, "-lineinfo", "-O3", "-std=c++17", "-shared", "-Xcompiler", "-fPIC,-O3", "-cudart", "static",
         f"-I{INCLUDE}", f"-I{CSRC}", "-o", str(tmp), *map(str, SOURCES)]
  if verbose: cmd.insert(1, "-Xptxas=-v")
  res = subprocess.run(cmd, capture_output=True, text=True)
  if res.returncode != 0:
    raise RuntimeError(f"nvcc failed ({res.returncode}):\n{' '.join(cmd)}\n{res.stdout}\n{res.stderr}")
  if verbose: sys.stderr.write(res.stderr)
  tmp.replace(OUT)
  return OUT


if __name__ == "__main__":
  ap = argparse.ArgumentParser()
  ap.add_argument("--force", action="store_true")
  ap.add_argument("-v", "--verbose", action="store_true")
  args = ap.parse_args()
  print(build(force=args.force, verbose=args.verbose))
