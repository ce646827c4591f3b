"""pytest setup: import paths, the ``gpu`` marker, and an in-tree build of the CUDA library when it is missing."""
from __future__ import annotations

import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent
PKG_ROOT = ROOT / "tinygrad-hopper-wgmma_b200"
for p in (str(PKG_ROOT), str(ROOT)):
  if p not in sys.path: sys.path.insert(0, p)


def pytest_configure(config):
  config.addinivalue_line("markers", "gpu: needs a B200 (sm_100a) GPU")
  lib = PKG_ROOT / "hopper_wgmma" / "lib" / "libsm100_gemm.so"
  if not lib.exists():
    sys.path.insert(0, str(PKG_ROOT / "csrc"))
    import build as csrc_build
    csrc_build.build()


@pytest.fixture(scope="session")
def golden():
  import json
  return json.loads((ROOT / "tests" / "golden" / "reference_host.json").read_text())


@pytest.fixture(scope="session")
def cuda_dev():
  import torch
  if not torch.cuda.is_available(): pytest.skip("no CUDA device")
  return torch.device("cuda:0")
