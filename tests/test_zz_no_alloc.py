"""bg_gemm_noalloc: the GEMM entry point that allocates nothing, for callers that may not allocate device memory
themselves (for example a plugin whose host framework owns all device memory through its own pool). Called through
the C ABI, it must give the same output as the plan-based entry point (bg_plan_create + bg_plan_launch), within the
tests' tolerance, on two calls in a row — the second call reuses the scratch array the first one left behind — and
it must refuse a problem whose tile table does not fit its fixed scratch before it enqueues anything.

This file is named so that pytest collects it last: a failure here leaves every other test already run."""
from __future__ import annotations

import ctypes

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
  import torch
  g = torch.Generator(device=dev).manual_seed(seed)
  A = torch.randn((M, K), generator=g, device=dev).to(torch.bfloat16)
  BT = torch.randn((N, K), generator=g, device=dev).to(torch.bfloat16)
  return A, BT


def test_noalloc_matches_plan_entry_point_on_two_calls_in_a_row(cuda_dev):
  import torch
  from hopper_wgmma import WSCfg
  lib, _capi = _lib()
  stream = torch.cuda.current_stream(cuda_dev).cuda_stream
  cases = [(WSCfg(tma_store=True, cluster=2, hilbert=True), (512, 1024, 256), 0),
           (WSCfg(BN=128, tma_store=True), (768, 512, 320), 1)]
  for cfg, (M, N, K), seed in cases:
    A, BT = _operands(M, N, K, seed, cuda_dev)
    c_cfg = cfg.to_c()
    ref = torch.full((M, N), float("nan"), dtype=torch.bfloat16, device=cuda_dev)
    plan = _capi.Plan(c_cfg, M, N, K, A.data_ptr(), K, BT.data_ptr(), K, ref.data_ptr(), N, cuda_dev.index or 0)
    plan.launch(stream)
    plan.check_error(stream)
    out = torch.full((M, N), float("nan"), dtype=torch.bfloat16, device=cuda_dev)
    err = ctypes.c_uint32(0xFFFFFFFF)
    st = lib.bg_gemm_noalloc(ctypes.byref(c_cfg), M, N, K, A.data_ptr(), K, BT.data_ptr(), K, out.data_ptr(), N,
                             cuda_dev.index or 0, ctypes.c_void_p(stream), ctypes.byref(err))
    assert st == 0, _capi.last_error()
    assert err.value == 0
    assert not torch.isnan(out).any()
    r = ref.float()
    rel = float((out.float() - r).abs().max() / (r.abs().max() + 1e-9))
    assert rel <= TOL, (cfg.name, rel)


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
