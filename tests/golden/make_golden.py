"""Generate tests/golden/reference_host.json by running the reference's own host-side Python.

Run in a container that has the reference checkout, passing its root:

    python tests/golden/make_golden.py REFERENCE_ROOT

The reference package (hopper_wgmma/) imports tinygrad at module level, and tinygrad is not installable here. Its
host logic (config dataclasses and their validation, the shape contract and kernel naming of build_gemm_ws /
build_gated_gemm, grouped_tile_order, hilbert_schedule, Ring.slot, the ladder tables, make_tensor_map's argument
checks) uses tinygrad only for names at import time, so this script injects a minimal stand-in for those names,
loads the reference package under the alias ``ref_hopper_wgmma`` and records what the reference functions return
or raise. Nothing here launches a kernel. The JSON is committed; the GPU box never needs the reference.
"""
from __future__ import annotations

import importlib.util
import json
import sys
import types
from pathlib import Path

HERE = Path(__file__).resolve().parent


class _Name:
  """Placeholder for a tinygrad name that is only referenced, never used, by the host code exercised here."""
  def __init__(self, name: str): self._name = name
  def __getattr__(self, item): return _Name(f"{self._name}.{item}")
  def __call__(self, *a, **k): raise RuntimeError(f"tinygrad stand-in {self._name} called")
  def __repr__(self): return f"<stub {self._name}>"


class _Bool:
  """Comparison result supporting the ``cond.where(a, b)`` used by the 1-D GROUP_M order (gemm.py:212)."""
  def __init__(self, v: bool): self.v = v
  def where(self, a, b): return a if self.v else b


class I:
  """Integer with the UOp operators grouped_tile_order's 1-D branch applies to a tile id."""
  def __init__(self, v): self.v = int(v.v if isinstance(v, I) else v)
  def _o(self, x): return x.v if isinstance(x, I) else x
  def __floordiv__(self, x): return I(self.v // self._o(x))
  def __mod__(self, x): return I(self.v % self._o(x))
  def __add__(self, x): return I(self.v + self._o(x))
  __radd__ = __add__
  def __mul__(self, x): return I(self.v * self._o(x))
  __rmul__ = __mul__
  def __sub__(self, x): return I(self.v - self._o(x))
  def __rsub__(self, x): return I(self._o(x) - self.v)
  def __gt__(self, x): return _Bool(self.v > self._o(x))
  def __int__(self): return self.v


def _install_tinygrad_standin() -> None:
  tg = types.ModuleType("tinygrad")
  tg.Tensor, tg.UOp, tg.dtypes, tg.Device = _Name("Tensor"), _Name("UOp"), _Name("dtypes"), _Name("Device")
  dt = types.ModuleType("tinygrad.dtype")
  dt.AddrSpace = _Name("AddrSpace")
  uop = types.ModuleType("tinygrad.uop")
  ops = types.ModuleType("tinygrad.uop.ops")
  for n in ("AxisType", "KernelInfo", "Ops", "PatternMatcher", "UPat"): setattr(ops, n, _Name(n))
  sys.modules.update({"tinygrad": tg, "tinygrad.dtype": dt, "tinygrad.uop": uop, "tinygrad.uop.ops": ops})


def _load_reference(root: Path):
  _install_tinygrad_standin()
  pkg_dir = root / "hopper_wgmma"
  spec = importlib.util.spec_from_file_location("ref_hopper_wgmma", pkg_dir / "__init__.py",
                                                submodule_search_locations=[str(pkg_dir)])
  pkg = importlib.util.module_from_spec(spec)
  sys.modules["ref_hopper_wgmma"] = pkg
  spec.loader.exec_module(pkg)
  runtime = importlib.import_module("ref_hopper_wgmma.runtime")
  runtime.install_runtime_hooks = lambda: None      # process-global tinygrad patches: not needed for host logic
  gemm = importlib.import_module("ref_hopper_wgmma.gemm")
  gated = importlib.import_module("ref_hopper_wgmma.gated")
  ladder = importlib.import_module("ref_hopper_wgmma.ladder")
  tensor_map = importlib.import_module("ref_hopper_wgmma.tensor_map")
  return gemm, gated, ladder, tensor_map


def _outcome(fn):
  try:
    return {"ok": fn()}
  except ValueError as exc:
    return {"error": str(exc)}


def main(root: Path) -> dict:
  gemm, gated, ladder, tensor_map = _load_reference(root)
  out: dict = {"source": "narain1/tinygrad-hopper-wgmma host code, run by tests/golden/make_golden.py"}

  # hilbert_schedule(M, N, cores): even splits give the table, uneven ones raise
  hil = []
  for M, N, cores in [(1, 1, 1), (2, 2, 1), (2, 2, 4), (4, 4, 4), (4, 2, 8), (3, 5, 1), (3, 5, 3), (3, 5, 5),
                      (8, 8, 16), (16, 16, 128), (16, 8, 128), (32, 16, 128), (8, 4, 8), (6, 6, 4), (7, 3, 7),
                      (12, 12, 72), (16, 16, 74), (32, 32, 74), (5, 7, 2), (64, 32, 128)]:
    hil.append({"M": M, "N": N, "cores": cores, **_outcome(lambda: gemm.hilbert_schedule(M, N, cores))})
  out["hilbert_schedule"] = hil

  # grouped_tile_order(CMT, NT, GM, GN): coords of every tile id and the 2-D flag
  grp = []
  for CMT, NT, GM, GN in [(4, 2, 16, 8), (16, 16, 16, 8), (32, 16, 16, 8), (6, 2, 3, 8), (6, 2, 3, 2), (7, 5, 3, 2),
                          (5, 3, 2, 3), (8, 8, 8, 8), (32, 32, 8, 8), (3, 4, 1, 1), (10, 6, 4, 4), (64, 32, 16, 8)]:
    GMc, GNc = min(GM, CMT), min(GN, NT)
    coords, two_d = gemm.grouped_tile_order(CMT, NT, GMc, GNc)
    tiles = [coords(t) if two_d else coords(I(t)) for t in range(CMT * NT)]
    grp.append({"CMT": CMT, "NT": NT, "GM": GMc, "GN": GNc, "grouped_2d": two_d,
                "coords": [[int(r), int(c)] for r, c in tiles]})
  out["grouped_tile_order"] = grp

  # WSCfg validation and derived fields
  ws = []
  for kw in [{}, {"BK": 32}, {"BN": 0}, {"BN": 8}, {"BN": 272}, {"BN": 192}, {"BN": 192, "tma_store": True},
             {"BN": 128, "tma_store": True}, {"stages": 1}, {"stages": 2}, {"stages": 5}, {"consumers": 0},
             {"consumers": 3}, {"consumers": 1}, {"cluster": 3}, {"cluster": 2}, {"num_sm": 1, "cluster": 2},
             {"group_m": 0}, {"group_n": 0}, {"regs": (24, 240)}, {"regs": (20, 240)}, {"regs": (24, 264)},
             {"regs": (24,)}, {"tma_store": True, "hilbert": True, "cluster": 2}, {"BN": 16}]:
    def fields(kw=kw):
      c = gemm.WSCfg(**kw)
      return {"BM": c.BM, "threads": c.threads, "smem_bytes": c.smem_bytes, "name": c.name}
    ws.append({"kwargs": {k: list(v) if isinstance(v, tuple) else v for k, v in kw.items()}, **_outcome(fields)})
  out["WSCfg"] = ws

  gc = []
  for kw in [{}, {"BK": 128}, {"BN": 24}, {"stages": 1}, {"consumers": 3}, {"consumers": 0}, {"consumers": 1},
             {"BN": 128, "stages": 4, "consumers": 0}, {"stages": 6}]:
    def gfields(kw=kw):
      c = gated.GatedCfg(**kw)
      return {"BM": c.BM, "threads": c.threads, "smem_bytes": c.smem_bytes}
    gc.append({"kwargs": kw, **_outcome(gfields)})
  out["GatedCfg"] = gc

  # build_gemm_ws shape contract and kernel naming (no launch)
  bw = []
  for N, kw, M, K in [(512, {}, None, None), (512, {}, 256, 256), (500, {}, None, None), (512, {}, 100, 512),
                      (512, {}, 512, 96), (512, {"cluster": 2}, 128, 512), (512, {"cluster": 2}, 256, 512),
                      (1024, {"hilbert": True, "num_sm": 3}, 512, 512), (512, {"group_m": 3}, 768, 256),
                      (768, {"BN": 192, "tma_store": True}, 256, 256), (512, {"consumers": 1}, 64, 64),
                      (0, {}, None, None), (4096, {"tma_store": True, "hilbert": True}, None, None)]:
    def built(N=N, kw=kw, M=M, K=K):
      run = gemm.build_gemm_ws(N, gemm.WSCfg(**kw), M, K)
      return {"kernel_name": run.kernel_name}
    bw.append({"N": N, "kwargs": kw, "M": M, "K": K, **_outcome(built)})
  out["build_gemm_ws"] = bw

  bg = []
  for N, kw in [(512, {}), (500, {}), (128, {"stages": 3}), (256, {"BN": 128, "stages": 4, "consumers": 0}),
                (192, {"consumers": 0, "BN": 64, "stages": 4})]:
    def gbuilt(N=N, kw=kw):
      return {"kernel_name": gated.build_gated_gemm(N, gated.GatedCfg(**kw)).kernel_name}
    bg.append({"N": N, "kwargs": kw, **_outcome(gbuilt)})
  out["build_gated_gemm"] = bg

  def cfg_fields(c):
    d = {k: getattr(c, k) for k in c.__dataclass_fields__}
    return {"type": type(c).__name__, **{k: list(v) if isinstance(v, tuple) else v for k, v in d.items()}}
  out["LADDER"] = {k: cfg_fields(v) for k, v in ladder.LADDER.items()}
  out["SWEEP"] = {k: cfg_fields(v) for k, v in ladder.SWEEP.items()}
  out["EXTRA"] = {k: cfg_fields(v) for k, v in ladder.EXTRA.items()}
  out["ladder_build"] = [{"N": 512, "M": 256, "K": None, **_outcome(lambda: ladder.build(512, ladder.LADDER["gated_ws"], 256))}]

  ring = gemm.Ring(None, 0, 3, 2, 1)
  out["Ring_slot"] = {"stages": 3, "slots": [list(ring.slot(j)) for j in range(10)]}

  tm = []
  for args in [(0, 64, 64, 64), (64, 0, 64, 64), (64, 64, 0, 64), (64, 64, 64, 0), (64, 32, 64, 64),
               (64, 64, 64, 96)]:
    tm.append({"args": list(args), **_outcome(lambda args=args: tensor_map.make_tensor_map(None, *args))})
  out["make_tensor_map"] = tm
  return out


if __name__ == "__main__":
  if len(sys.argv) != 2: raise SystemExit("usage: python tests/golden/make_golden.py REFERENCE_ROOT")
  root = Path(sys.argv[1])
  data = main(root)
  (HERE / "reference_host.json").write_text(json.dumps(data, indent=1) + "\n")
  print(f"wrote {HERE / 'reference_host.json'}")
