"""The C ABI's argument checks, exercised on the CPU: a contract violation returns a negative status (ValueError in
Python, as the reference raises for config and shape errors) before any device call; a valid request on a machine
without a GPU driver comes back as a positive status (RuntimeError) instead of crashing."""
from __future__ import annotations

import ctypes

import pytest

FAKE_A, FAKE_B, FAKE_C = 0x10000, 0x20000, 0x30000   # aligned, never dereferenced: validation fails first


def _create(cfg, M, N, K, a=FAKE_A, b=FAKE_B, c=FAKE_C, lda=None, ldb=None, ldc=None):
  from hopper_wgmma import _capi
  h = ctypes.c_void_p()
  st = _capi.LIB.bg_plan_create(ctypes.byref(h), ctypes.byref(cfg), M, N, K, a, K if lda is None else lda, b,
                                K if ldb is None else ldb, c, N if ldc is None else ldc, 0)
  if st == 0: _capi.LIB.bg_plan_destroy(h)
  return st, _capi.last_error()


def _cfg(**kw):
  from hopper_wgmma import WSCfg
  c = WSCfg().to_c()
  for k, v in kw.items(): setattr(c, k, v)
  return c


@pytest.mark.parametrize("kw,shape,msg", [
  ({"BK": 32}, (512, 512, 512), "BK must be 64"),
  ({"BN": 24}, (512, 512, 512), "BN must be a multiple of 16"),
  ({"BN": 96, "tma_store": 1}, (512, 576, 512), "tma_store needs BN"),
  ({"stages": 1}, (512, 512, 512), "stages must be at least 2"),
  ({"consumers": 3}, (512, 512, 512), "consumers must be 1 or 2"),
  ({"cluster": 3}, (512, 512, 512), "cluster must be 1 or 2"),
  ({"num_sm": 1, "cluster": 2}, (512, 512, 512), "num_sm must be at least the cluster size"),
  ({"group_m": 0}, (512, 512, 512), "group_m and group_n must be positive"),
  ({"n_mma": 3}, (512, 512, 512), "n_mma must be 1 or 2"),
  ({"acc_bufs": 3}, (512, 512, 512), "acc_bufs"),
  ({}, (500, 512, 512), "not a multiple of tile"),
  ({}, (512, 512, 96), "not a multiple of tile"),
  ({"cluster": 2}, (128, 512, 512), "row tiles not divisible by cluster"),
  ({"ragged": 1}, (300, 522, 200), "multiples of 8"),
  ({"kind": 2, "consumers": 0, "cluster": 2}, (512, 512, 512), "need the persistent kernel"),
  ({"kind": 2, "consumers": 2}, (512, 512, 512), "consumers == 0"),
  ({"kind": 7}, (512, 512, 512), "unknown kernel kind"),
  ({"split_k": 65}, (512, 512, 4096 + 128), "split_k must be -1 (auto) or in [0, 64]"),
  ({"split_k": -2}, (512, 512, 512), "split_k must be -1 (auto)"),
  ({"split_k": 2, "kind": 1}, (512, 512, 512), "split_k needs the persistent kernel"),
  ({"split_k": 9}, (512, 512, 512), "exceeds the 8 k-blocks"),
  ({"split_k": 2, "BN": 48}, (512, 480, 512), "multiple of 32 columns"),
  ({"b_nmajor": 2}, (512, 512, 512), "b_nmajor must be 0 or 1"),
  ({"b_nmajor": 1, "kind": 1}, (512, 512, 512), "b_nmajor needs the warp-specialized kernel"),
  ({"b_nmajor": 1, "BN": 96}, (512, 576, 512), "b_nmajor needs BN a multiple of 64"),
  ({"b_nmajor": 1, "BN": 64, "cluster": 2}, (512, 512, 512), "b_nmajor needs BN / 2 a multiple of 64"),
  ({"wave_sync": 3}, (512, 512, 512), "wave_sync must be 0 (auto), 1 (on) or 2 (off)"),
  ({"split_k_cluster": 3}, (512, 512, 512), "split_k_cluster must be 0 (auto)"),
  ({"split_k_cluster": -1}, (512, 512, 512), "split_k_cluster must be 0 (auto)"),
])
def test_contract_violations_are_negative_status(kw, shape, msg):
  st, err = _create(_cfg(**kw), *shape)
  assert st < 0, (st, err)
  assert msg in err


def test_pointer_and_pitch_checks():
  assert _create(_cfg(), 512, 512, 512, a=0)[0] < 0
  st, err = _create(_cfg(), 512, 512, 512, b=FAKE_B + 8)
  assert st < 0 and "16-byte aligned" in err
  st, err = _create(_cfg(), 512, 512, 512, lda=256)
  assert st < 0 and "row pitches" in err
  st, err = _create(_cfg(), 512, 512, 512, ldc=516)
  assert st < 0 and "row pitches" in err
  # N-major B: its pitch covers N, not K
  st, err = _create(_cfg(b_nmajor=1), 512, 1024, 256, ldb=512)
  assert st < 0 and "row pitches" in err


def test_valid_request_without_driver_is_a_positive_status():
  import torch
  if torch.cuda.is_available(): pytest.skip("a device is present")
  st, err = _create(_cfg(), 512, 512, 512)
  assert st > 0 and err


def test_python_plan_maps_status_to_exceptions():
  import torch
  from hopper_wgmma import _capi
  with pytest.raises(ValueError, match="BN must be"):
    _capi.Plan(_cfg(BN=24), 512, 512, 512, FAKE_A, 512, FAKE_B, 512, FAKE_C, 512, 0)
  if not torch.cuda.is_available():
    with pytest.raises(RuntimeError):
      _capi.Plan(_cfg(), 512, 512, 512, FAKE_A, 512, FAKE_B, 512, FAKE_C, 512, 0)


def test_noalloc_entry_checks_arguments_first():
  from hopper_wgmma import _capi
  lib = _capi.LIB
  lib.bg_gemm_noalloc.restype = ctypes.c_int32
  lib.bg_gemm_noalloc.argtypes = [ctypes.POINTER(_capi.BgCfg), ctypes.c_int64, ctypes.c_int64, ctypes.c_int64,
                                  ctypes.c_void_p, ctypes.c_int64, ctypes.c_void_p, ctypes.c_int64, ctypes.c_void_p,
                                  ctypes.c_int64, ctypes.c_int32, ctypes.c_void_p, ctypes.POINTER(ctypes.c_uint32)]
  cfg = _cfg(BN=24)
  st = lib.bg_gemm_noalloc(ctypes.byref(cfg), 512, 512, 512, FAKE_A, 512, FAKE_B, 512, FAKE_C, 512, 0, None, None)
  assert st < 0 and "BN must be" in _capi.last_error()
  st = lib.bg_gemm_noalloc(None, 512, 512, 512, FAKE_A, 512, FAKE_B, 512, FAKE_C, 512, 0, None, None)
  assert st < 0
  cfg = _cfg(split_k=2)
  st = lib.bg_gemm_noalloc(ctypes.byref(cfg), 512, 512, 512, FAKE_A, 512, FAKE_B, 512, FAKE_C, 512, 0, None, None)
  assert st < 0 and "split-K" in _capi.last_error()


def test_plan_destructor_needs_no_module_globals(monkeypatch):
  """Plan.__del__ may run at interpreter exit, after the _capi module's globals (ctypes, LIB) have been set to None:
  it must destroy the handle with what the instance holds."""
  import ctypes
  from hopper_wgmma import _capi
  destroyed = []
  p = _capi.Plan.__new__(_capi.Plan)
  p._h = ctypes.c_void_p(1)
  p._destroy = destroyed.append
  monkeypatch.setattr(_capi, "ctypes", None)
  monkeypatch.setattr(_capi, "LIB", None)
  p.__del__()
  assert len(destroyed) == 1 and p._h is None
