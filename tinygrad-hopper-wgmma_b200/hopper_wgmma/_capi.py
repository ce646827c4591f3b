"""ctypes binding of the sm_100a GEMM library (``lib/libsm100_gemm.so``, C ABI in ``include/sm100_gemm.h``).

The library is the only compute path: there is no CPU or eager fallback. If it was not built, importing this module
raises ``ImportError`` naming the build command.
"""
from __future__ import annotations

import ctypes
import os
from pathlib import Path

LIB_DIR = Path(__file__).resolve().parent / "lib"
LIB_PATH = LIB_DIR / "libsm100_gemm.so"

KIND_WS, KIND_GATED, KIND_RING = 0, 1, 2

# Exported symbols; the CPU tests check that the library provides every one of them.
EXPORTS = ("bg_last_error", "bg_version", "bg_device_info", "bg_plan_create", "bg_plan_launch", "bg_plan_check_error",
           "bg_plan_get_info", "bg_plan_destroy", "bg_hilbert_order", "bg_grouped_order", "bg_encode_tensor_map_3d")


class BgCfg(ctypes.Structure):
  _fields_ = [("kind", ctypes.c_int32), ("BN", ctypes.c_int32), ("BK", ctypes.c_int32), ("stages", ctypes.c_int32),
              ("consumers", ctypes.c_int32), ("num_sm", ctypes.c_int32), ("group_m", ctypes.c_int32),
              ("group_n", ctypes.c_int32), ("tma_store", ctypes.c_int32), ("cluster", ctypes.c_int32),
              ("hilbert", ctypes.c_int32), ("acc_bufs", ctypes.c_int32), ("wait_budget_ns", ctypes.c_int64),
              ("debug_skip_job", ctypes.c_int32), ("n_mma", ctypes.c_int32),
              ("no_tail_split", ctypes.c_int32), ("ragged", ctypes.c_int32), ("split_k", ctypes.c_int32),
              ("no_k_serpentine", ctypes.c_int32), ("b_nmajor", ctypes.c_int32), ("wave_sync", ctypes.c_int32),
              ("split_k_cluster", ctypes.c_int32)]


class BgPlanInfo(ctypes.Structure):
  _fields_ = [("grid", ctypes.c_int32), ("threads", ctypes.c_int32), ("smem_bytes", ctypes.c_int32),
              ("stages", ctypes.c_int32), ("tiles", ctypes.c_int32), ("clusters", ctypes.c_int32),
              ("cluster", ctypes.c_int32), ("paired", ctypes.c_int32), ("bm", ctypes.c_int32), ("bn", ctypes.c_int32),
              ("acc_bufs", ctypes.c_int32), ("tmem_cols", ctypes.c_int32), ("max_active_clusters", ctypes.c_int32),
              ("narrow_tiles", ctypes.c_int32), ("split_k", ctypes.c_int32), ("kernel", ctypes.c_char * 96)]


def _load() -> ctypes.CDLL:
  if not LIB_PATH.exists():
    raise ImportError(f"{LIB_PATH} is missing: build it with `python -c 'import __graft_entry__ as g; g.build()'` "
                      "from the repository root (nvcc, sm_100a)")
  lib = ctypes.CDLL(str(LIB_PATH), mode=os.RTLD_LOCAL if hasattr(os, "RTLD_LOCAL") else 0)
  i32, i64, vp = ctypes.c_int32, ctypes.c_int64, ctypes.c_void_p
  lib.bg_last_error.restype = ctypes.c_char_p
  lib.bg_last_error.argtypes = []
  lib.bg_version.restype = i32
  lib.bg_device_info.restype = i32
  lib.bg_device_info.argtypes = [i32] + [ctypes.POINTER(i32)] * 4
  lib.bg_plan_create.restype = i32
  lib.bg_plan_create.argtypes = [ctypes.POINTER(vp), ctypes.POINTER(BgCfg), i64, i64, i64, vp, i64, vp, i64, vp, i64, i32]
  lib.bg_plan_launch.restype = i32
  lib.bg_plan_launch.argtypes = [vp, vp]
  lib.bg_plan_check_error.restype = i32
  lib.bg_plan_check_error.argtypes = [vp, vp, ctypes.POINTER(ctypes.c_uint32)]
  lib.bg_plan_get_info.restype = i32
  lib.bg_plan_get_info.argtypes = [vp, ctypes.POINTER(BgPlanInfo)]
  lib.bg_plan_destroy.restype = None
  lib.bg_plan_destroy.argtypes = [vp]
  lib.bg_hilbert_order.restype = i32
  lib.bg_hilbert_order.argtypes = [i32, i32, ctypes.POINTER(i32), i32]
  lib.bg_grouped_order.restype = i32
  lib.bg_grouped_order.argtypes = [i32, i32, i32, i32, ctypes.POINTER(i32), i32]
  lib.bg_encode_tensor_map_3d.restype = i32
  lib.bg_encode_tensor_map_3d.argtypes = [vp, vp, i64, i64, i32, i32]
  return lib


LIB = _load()


def last_error() -> str:
  return LIB.bg_last_error().decode(errors="replace")


def check(status: int, what: str) -> None:
  """Negative status: the arguments break the contract (ValueError). Positive: CUDA or device error (RuntimeError)."""
  if status < 0: raise ValueError(f"{what}: {last_error()}")
  if status > 0: raise RuntimeError(f"{what} failed with status {status}: {last_error()}")


def device_info(device: int) -> dict:
  vals = [ctypes.c_int32() for _ in range(4)]
  check(LIB.bg_device_info(device, *[ctypes.byref(v) for v in vals]), "bg_device_info")
  return dict(zip(("sm_count", "smem_optin", "cc_major", "cc_minor"), (v.value for v in vals)))


def hilbert_order(m_tiles: int, n_tiles: int) -> list[int]:
  cap = m_tiles * n_tiles
  buf = (ctypes.c_int32 * max(cap, 1))()
  n = LIB.bg_hilbert_order(m_tiles, n_tiles, buf, cap)
  check(n if n < 0 else 0, "bg_hilbert_order")
  return list(buf[:n])


def grouped_order(m_tiles: int, n_tiles: int, group_m: int, group_n: int) -> list[int]:
  cap = m_tiles * n_tiles
  buf = (ctypes.c_int32 * max(cap, 1))()
  n = LIB.bg_grouped_order(m_tiles, n_tiles, group_m, group_n, buf, cap)
  check(n if n < 0 else 0, "bg_grouped_order")
  return list(buf[:n])


class Plan:
  """Owns one ``bg_plan``: encoded tensor maps, the device tile table, the error word and any split-K workspace."""

  def __init__(self, cfg: BgCfg, M: int, N: int, K: int, a_ptr: int, lda: int, bt_ptr: int, ldb: int, c_ptr: int,
               ldc: int, device: int):
    self._h = ctypes.c_void_p()
    self._cfg = cfg
    self._destroy = LIB.bg_plan_destroy   # kept on the instance: module globals may be gone when __del__ runs at exit
    check(LIB.bg_plan_create(ctypes.byref(self._h), ctypes.byref(cfg), M, N, K, a_ptr, lda, bt_ptr, ldb, c_ptr, ldc,
                             device), "bg_plan_create")
    self.device = device

  def launch(self, stream: int) -> None:
    check(LIB.bg_plan_launch(self._h, ctypes.c_void_p(stream)), "bg_plan_launch")

  def check_error(self, stream: int) -> int:
    """Synchronize ``stream`` and raise RuntimeError if a device-side wait timed out (the word is then cleared)."""
    word = ctypes.c_uint32(0)
    st = LIB.bg_plan_check_error(self._h, ctypes.c_void_p(stream), ctypes.byref(word))
    check(st, "GEMM launch")
    return word.value

  def info(self) -> dict:
    inf = BgPlanInfo()
    check(LIB.bg_plan_get_info(self._h, ctypes.byref(inf)), "bg_plan_get_info")
    out = {name: getattr(inf, name) for name, _ in BgPlanInfo._fields_}
    out["kernel"] = inf.kernel.decode()
    return out

  def __del__(self):
    # may run at interpreter exit, after module globals (ctypes included) are gone: use only what the instance holds
    h = getattr(self, "_h", None)
    if h is not None and h.value:
      self._destroy(h)
      self._h = None
