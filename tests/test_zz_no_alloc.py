"""bg_gemm_noalloc: the GEMM entry point that allocates nothing, for callers that may not allocate device memory
themselves (for example a plugin whose host framework owns all device memory through its own pool). Called through
the C ABI on seeded bf16 inputs, on two calls in a row — the second call reuses the scratch array the first one left
behind — its output must match the CPU oracle (fp32 accumulation of the same bf16 inputs) within the tests' tolerance
and agree with the plan-based entry point (bg_plan_create + bg_plan_launch). The second call must leave the device's
free memory unchanged. With split_k = -1 (automatic) on a shape where the plan path would split K, it runs unsplit
(it has no split-K workspace) and still matches the oracle. A problem whose tile table does not fit its fixed scratch
is refused before anything is enqueued.

This file is named so that pytest collects it last: a failure here leaves every other test already run."""
from __future__ import annotations

import ctypes

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

TOL = 4e-3


def _lib():
  from hopper_wgmma import _capi
  lib = _capi.LIB
  lib.bg_gemm_noalloc.restype = ctypes.c_int32
  lib.bg_gemm_noalloc.argtypes = [ctypes.POINTER(_capi.BgCfg), ctypes.c_int64, ctypes.c_int64, ctypes.c_int64,
                                  ctypes.c_void_p, ctypes.c_int64, ctypes.c_void_p, ctypes.c_int64, ctypes.c_void_p,
                                  ctypes.c_int64, ctypes.c_int32, ctypes.c_void_p, ctypes.POINTER(ctypes.c_uint32)]
  return lib, _capi


def _operands(M, N, K, seed, dev):
  """Seeded bf16 A[M,K] and BT[N,K] on the device, with the same bits for the CPU oracle (A bits, B = BT^T bits)."""
  import torch
  from oracle import gemm_ref
  a_bits = gemm_ref.randn_bf16_bits((M, K), seed)
  b_bits = gemm_ref.randn_bf16_bits((K, N), seed + 1)
  to_dev = lambda bits: torch.from_numpy(np.ascontiguousarray(bits).view(np.int16)).view(torch.bfloat16).to(dev)
  return to_dev(a_bits), to_dev(np.ascontiguousarray(b_bits.T)), gemm_ref.gemm_f32(a_bits, b_bits)


def _bits(t):
  import torch
  return t.contiguous().view(torch.int16).cpu().numpy().view(np.uint16)


def _noalloc(lib, c_cfg, M, N, K, A, BT, out, dev, stream):
  err = ctypes.c_uint32(0xFFFFFFFF)
  st = lib.bg_gemm_noalloc(ctypes.byref(c_cfg), M, N, K, A.data_ptr(), K, BT.data_ptr(), K, out.data_ptr(), N,
                           dev.index or 0, ctypes.c_void_p(stream), ctypes.byref(err))
  return st, err.value


@pytest.mark.parametrize("case", ["pair_hilbert", "cta_bn128", "auto_split_k_runs_unsplit"])
def test_noalloc_matches_oracle_on_two_calls_in_a_row(case, cuda_dev):
  import torch
  from hopper_wgmma import WSCfg
  from oracle import gemm_ref
  lib, _capi = _lib()
  cfg, (M, N, K), seed = {
    "pair_hilbert": (WSCfg(tma_store=True, cluster=2, hilbert=True), (512, 1024, 256), 0),
    "cta_bn128": (WSCfg(BN=128, tma_store=True), (768, 512, 320), 1),
    # 4 tiles of 128 x 128 and 128 k-blocks: the plan path's automatic choice splits K four ways
    "auto_split_k_runs_unsplit": (WSCfg(BN=128, tma_store=True, split_k=-1), (256, 256, 8192), 2),
  }[case]
  stream = torch.cuda.current_stream(cuda_dev).cuda_stream
  A, BT, ref = _operands(M, N, K, seed, cuda_dev)
  c_cfg = cfg.to_c()

  # the plan-based entry point on the same inputs
  planned = torch.full((M, N), float("nan"), dtype=torch.bfloat16, device=cuda_dev)
  plan = _capi.Plan(c_cfg, M, N, K, A.data_ptr(), K, BT.data_ptr(), K, planned.data_ptr(), N, cuda_dev.index or 0)
  plan.launch(stream)
  plan.check_error(stream)
  if case == "auto_split_k_runs_unsplit": assert plan.info()["split_k"] > 1
  assert gemm_ref.rel_err(_bits(planned), ref) <= TOL

  outs = []
  for call in range(2):
    out = torch.full((M, N), float("nan"), dtype=torch.bfloat16, device=cuda_dev)
    torch.cuda.synchronize(cuda_dev)
    free_before = torch.cuda.mem_get_info(cuda_dev)[0]
    st, err = _noalloc(lib, c_cfg, M, N, K, A, BT, out, cuda_dev, stream)
    torch.cuda.synchronize(cuda_dev)
    free_after = torch.cuda.mem_get_info(cuda_dev)[0]
    assert st == 0, _capi.last_error()
    assert err == 0
    if call == 1:   # any device allocation takes at least one 2 MiB page
      assert free_after == free_before, (free_before, free_after)
    bits = _bits(out)
    assert gemm_ref.count_nan(bits) == 0
    rel = gemm_ref.rel_err(bits, ref)
    assert rel <= TOL, (case, call, rel)
    outs.append(bits)
  assert (outs[0] == outs[1]).all()
  if case != "auto_split_k_runs_unsplit":   # same kernel and schedule as the plan: the same bits
    assert (outs[1] == _bits(planned)).all()


def test_noalloc_rejects_a_tile_table_beyond_its_scratch(cuda_dev):
  import torch
  from hopper_wgmma import WSCfg
  lib, _capi = _lib()
  M, N, K = 65536, 4096, 64              # BN=16 tiles: 512 x 256 = 131072 entries > 65536
  A = torch.zeros((M, K), dtype=torch.bfloat16, device=cuda_dev)
  BT = torch.zeros((N, K), dtype=torch.bfloat16, device=cuda_dev)
  C = torch.zeros((M, N), dtype=torch.bfloat16, device=cuda_dev)
  c_cfg = WSCfg(BN=16).to_c()
  st = lib.bg_gemm_noalloc(ctypes.byref(c_cfg), M, N, K, A.data_ptr(), K, BT.data_ptr(), K, C.data_ptr(), N,
                           cuda_dev.index or 0, ctypes.c_void_p(torch.cuda.current_stream(cuda_dev).cuda_stream), None)
  assert st < 0
  assert "65536" in _capi.last_error()
  torch.cuda.synchronize(cuda_dev)
