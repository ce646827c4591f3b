"""The tinygrad side of the boundary (the reference's own framework, hopper_wgmma/gemm.py:389 launches through
``Tensor.custom_kernel`` and scripts/ncu_workload.py:50 runs the stock ``a @ b``).

This records, on the GPU box, whether tinygrad is importable there. When it is not (this image ships no tinygrad and
has no network to fetch the reference's pinned submodule), the test is skipped with that reason. When it is:
  * the BASELINE oracle — tinygrad's CPU ``A @ B`` at 1024^3 on seeded bf16 inputs — is checked against the CPU
    restatement in oracle/gemm_ref.py, and
  * ``build_gemm_ws(...)(a, b, c)()`` runs over realized tinygrad CUDA Tensors (pointers read as
    hopper_wgmma/tensor_map.py:20-24 does) and is compared with the same oracle. tinygrad's own queue is drained
    before the launch and the launch is waited for before tinygrad reads C, because the GEMM is enqueued on the legacy
    default stream, which tinygrad's queue does not order against."""
from __future__ import annotations

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

TOL = 4e-3


def _tinygrad():
  try:
    import tinygrad
  except ImportError as exc:
    pytest.skip(f"tinygrad is not importable on this machine ({exc}); the tinygrad-Tensor boundary is untested here")
  return tinygrad


def test_tinygrad_cpu_matmul_matches_the_oracle(cuda_dev):
  _tinygrad()
  from tinygrad import Tensor, dtypes
  from oracle import gemm_ref
  M = N = K = 1024
  a_bits, b_bits = gemm_ref.randn_bf16_bits((M, K), 0), gemm_ref.randn_bf16_bits((K, N), 1)
  a = Tensor(gemm_ref.bf16_bits_to_f32(a_bits), device="CPU").cast(dtypes.bfloat16)
  b = Tensor(gemm_ref.bf16_bits_to_f32(b_bits), device="CPU").cast(dtypes.bfloat16)
  out = (a @ b).float().numpy()
  ref = gemm_ref.gemm_f32(a_bits, b_bits)
  rel = float(np.max(np.abs(out - ref)) / (np.max(np.abs(ref)) + 1e-9))
  assert rel <= TOL, rel


def test_launch_over_tinygrad_cuda_tensors(cuda_dev):
  _tinygrad()
  from tinygrad import Device, Tensor, dtypes
  from hopper_wgmma import WSCfg, build_gemm_ws
  from oracle import gemm_ref
  M, N, K = 512, 1024, 384
  a_bits, b_bits = gemm_ref.randn_bf16_bits((M, K), 3), gemm_ref.randn_bf16_bits((K, N), 4)
  a = Tensor(gemm_ref.bf16_bits_to_f32(a_bits), device="CUDA").cast(dtypes.bfloat16).contiguous().realize()
  b = Tensor(gemm_ref.bf16_bits_to_f32(b_bits), device="CUDA").cast(dtypes.bfloat16).contiguous().realize()
  c = Tensor.full((M, N), float("nan"), dtype=dtypes.bfloat16, device="CUDA").contiguous().realize()
  launch = build_gemm_ws(N, WSCfg(tma_store=True, cluster=2, hilbert=True), M, K)(a, b, c)
  Device["CUDA"].synchronize()
  launch()
  launch.check()
  out = c.float().numpy()
  ref = gemm_ref.gemm_f32(a_bits, b_bits)
  assert not np.isnan(out).any()
  rel = float(np.max(np.abs(out - ref)) / (np.max(np.abs(ref)) + 1e-9))
  assert rel <= TOL, rel
