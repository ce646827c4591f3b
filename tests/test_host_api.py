"""Host-side parity with the reference's operator API (no GPU needed): the C ABI library loads and exports what the
header declares; configs, shape contracts, tile orders, ladder tables and helper contracts match what the reference's
own code returns or raises (tests/golden/reference_host.json, made by tests/golden/make_golden.py)."""
from __future__ import annotations

import re
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent
SMEM_MSG = "needs "


# ----------------------------------------------------------------------------------------------------------------
# the C ABI library
# ----------------------------------------------------------------------------------------------------------------
def header_functions() -> set[str]:
  text = (ROOT / "include" / "sm100_gemm.h").read_text()
  text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
  return set(re.findall(r"\b(bg_[a-z0-9_]+)\s*\(", text))


def test_library_loads_and_exports_every_declared_symbol():
  from hopper_wgmma import _capi
  declared = header_functions()
  assert declared, "no declarations parsed from include/sm100_gemm.h"
  missing = [name for name in sorted(declared) if not hasattr(_capi.LIB, name)]
  assert not missing, f"library lacks {missing}"
  assert set(_capi.EXPORTS) <= declared
  assert _capi.LIB.bg_version() >= 100


def test_library_reports_missing_device_as_runtime_error_not_crash():
  import torch
  if torch.cuda.is_available(): pytest.skip("a device is present")
  from hopper_wgmma import _capi
  with pytest.raises(RuntimeError):
    _capi.device_info(0)


def test_cfg_struct_layout_matches_header():
  """The ctypes mirror of bg_cfg has the header's fields in order (12 int32, int64, 9 int32, padded to 8 bytes)."""
  import ctypes
  from hopper_wgmma import _capi
  text = (ROOT / "include" / "sm100_gemm.h").read_text()
  body = text[text.index("typedef struct bg_cfg {"):text.index("} bg_cfg;")]
  fields = re.findall(r"int(?:32|64)_t\s+(\w+);", body)
  assert [f for f, _ in _capi.BgCfg._fields_] == fields
  assert ctypes.sizeof(_capi.BgCfg) == 12 * 4 + 8 + 9 * 4 + 4


# ----------------------------------------------------------------------------------------------------------------
# configs
# ----------------------------------------------------------------------------------------------------------------
def _kw(d):
  return {k: tuple(v) if isinstance(v, list) else v for k, v in d.items()}


def test_wscfg_validation_matches_reference(golden):
  from hopper_wgmma import WSCfg
  for case in golden["WSCfg"]:
    kw = _kw(case["kwargs"])
    if "error" in case and not case["error"].startswith(SMEM_MSG):
      with pytest.raises(ValueError) as exc:
        WSCfg(**kw)
      assert str(exc.value) == case["error"], kw
    elif "error" in case:            # the reference's H200 shared-memory budget: ours must reject it too
      with pytest.raises(ValueError, match=SMEM_MSG):
        WSCfg(**kw)
    else:
      cfg = WSCfg(**kw)
      assert cfg.BM == case["ok"]["BM"], kw
      assert cfg.smem_bytes <= 227 * 1024


def test_gatedcfg_validation_matches_reference(golden):
  from hopper_wgmma import GatedCfg
  for case in golden["GatedCfg"]:
    kw = case["kwargs"]
    if "error" in case and not case["error"].startswith(SMEM_MSG):
      with pytest.raises(ValueError) as exc:
        GatedCfg(**kw)
      assert str(exc.value) == case["error"], kw
    elif "error" not in case:
      assert GatedCfg(**kw).BM == case["ok"]["BM"], kw


def test_b200_knobs_validate():
  from hopper_wgmma import WSCfg
  with pytest.raises(ValueError, match="n_mma"):
    WSCfg(n_mma=3)
  with pytest.raises(ValueError, match="acc_bufs"):
    WSCfg(acc_bufs=3)
  with pytest.raises(ValueError, match="tensor memory"):
    WSCfg(n_mma=2, acc_bufs=2)
  assert WSCfg(n_mma=2, cluster=2, tma_store=True).width == 512
  assert WSCfg().stages_used >= 2 and WSCfg(stages=3).stages_used == 3
  with pytest.raises(ValueError, match="split_k must be"):
    WSCfg(split_k=0)
  with pytest.raises(ValueError, match="multiple of 32"):
    WSCfg(BN=48, split_k=2)
  assert WSCfg(split_k=4).name.endswith("_sk4") and WSCfg(split_k=4).to_c().split_k == 4
  assert WSCfg(split_k=-1).name.endswith("_skA") and WSCfg(split_k=-1).to_c().split_k == -1
  # split_k_cluster: None = automatic (0), True = inside a cluster (1), False = through the workspace (2)
  assert WSCfg(split_k=2).to_c().split_k_cluster == 0
  assert WSCfg(split_k=2, split_k_cluster=True).name.endswith("_sk2_skc")
  assert WSCfg(split_k=2, split_k_cluster=True).to_c().split_k_cluster == 1
  assert WSCfg(split_k=2, split_k_cluster=False).name.endswith("_sk2_skw")
  assert WSCfg(split_k=2, split_k_cluster=False).to_c().split_k_cluster == 2


def test_which_configs_read_b_directly():
  """build_gemm_ws hands B[K,N] to the kernel uncopied when every CTA's share of a tile's columns, and of a
  half-width tail tile's, is whole 64-column boxes; by default CTA pairs and 128 x 256 single-CTA tiles do (smaller
  single-CTA tiles measured slower with N-major B). Otherwise it makes the reference's K-major copy."""
  import dataclasses
  from hopper_wgmma import WSCfg
  from hopper_wgmma.ladder import B200, LADDER
  for name in ("cluster", "cluster_hilbert"):
    assert LADDER[name].reads_b_directly, name                 # 256x256 pair tiles, 128 columns per CTA
  assert B200["pair_wide_hilbert"].reads_b_directly             # two N blocks of 128 columns per CTA
  for name in ("role_split", "tma_store", "hilbert"):
    assert LADDER[name].reads_b_directly, name                 # 128 x 256 single-CTA tiles read B directly ...
    assert not dataclasses.replace(LADDER[name], b_nmajor=False).reads_b_directly, name   # ... unless told not to
  for name in ("cta_n128", "cta_n64", "m64_n128"):
    assert not B200[name].reads_b_directly, name               # smaller single-CTA tiles copy by default
  assert not WSCfg(consumers=1).reads_b_directly                # 64 x 256: M = 64 MMAs, copied too
  forced = {k: dataclasses.replace(v, b_nmajor=True) for k, v in B200.items()}
  assert forced["cta_n128"].reads_b_directly and forced["m64_n128"].reads_b_directly
  assert not forced["cta_n64"].reads_b_directly                # its half-width tail tiles are 32 columns
  assert WSCfg(BN=64, tma_store=True, split_tail=False, b_nmajor=True).reads_b_directly
  assert not forced["pair_n128"].reads_b_directly              # 64 columns per CTA, 32 in a tail tile
  assert not forced["pair_n192"].reads_b_directly              # 96 columns per CTA
  assert not WSCfg(cluster=2, b_nmajor=False).reads_b_directly
  assert WSCfg(b_nmajor=False).name.endswith("_bT") and WSCfg(b_nmajor=True).name.endswith("_bN")
  assert not WSCfg().name.endswith(("_bT", "_bN"))
  assert WSCfg().to_c().b_nmajor == 0 and WSCfg().to_c(b_nmajor=True).b_nmajor == 1


# ----------------------------------------------------------------------------------------------------------------
# builders: shape contract and names (no launch)
# ----------------------------------------------------------------------------------------------------------------
def test_build_gemm_ws_shape_contract_matches_reference(golden):
  from hopper_wgmma import WSCfg, build_gemm_ws
  for case in golden["build_gemm_ws"]:
    kw = dict(case["kwargs"])
    N, M, K = case["N"], case["M"], case["K"]
    if "error" in case and "hilbert needs equal tiles" in case["error"]:
      # B200 deals Hilbert tiles raggedly over the device's clusters instead of refusing (documented difference)
      build_gemm_ws(N, WSCfg(**kw), M, K)
      continue
    if "error" in case:
      with pytest.raises(ValueError) as exc:
        build_gemm_ws(N, WSCfg(**kw), M, K)
      assert str(exc.value) == case["error"], case
    else:
      run = build_gemm_ws(N, WSCfg(**kw), M, K)
      ref_name = case["ok"]["kernel_name"]
      assert ("_g1d_" in run.kernel_name) == ("_g1d_" in ref_name)
      assert run.kernel_name.split("_")[1] == ref_name.split("_")[1]   # the shape token
      assert run.kernel_name.startswith("sm100_")


def test_build_gated_gemm_contract_matches_reference(golden):
  from hopper_wgmma import GatedCfg, build_gated_gemm
  for case in golden["build_gated_gemm"]:
    if "error" in case:
      with pytest.raises(ValueError) as exc:
        build_gated_gemm(case["N"], GatedCfg(**case["kwargs"]))
      assert str(exc.value) == case["error"]
    else:
      name = build_gated_gemm(case["N"], GatedCfg(**case["kwargs"])).kernel_name
      assert name.replace("sm100_", "hopper_") == case["ok"]["kernel_name"]


def test_ladder_tables_match_reference(golden):
  from hopper_wgmma.ladder import EXTRA, LADDER, SWEEP, build
  assert list(LADDER) == list(golden["LADDER"])
  assert list(SWEEP) == list(golden["SWEEP"])
  assert set(golden["EXTRA"]) <= set(EXTRA)
  b200_defaults = {"num_sm", "stages"}   # device SM count, fill shared memory
  for table, ref in ((LADDER, golden["LADDER"]), (SWEEP, golden["SWEEP"])):
    for name, fields in ref.items():
      cfg = table[name]
      assert type(cfg).__name__ == fields["type"]
      for k, v in fields.items():
        if k == "type" or (k in b200_defaults and type(cfg).__name__ == "WSCfg"): continue
        got = getattr(cfg, k)
        assert (list(got) if isinstance(got, tuple) else got) == v, (name, k)
  with pytest.raises(ValueError) as exc:
    build(512, LADDER["gated_ws"], 256)
  assert str(exc.value) == golden["ladder_build"][0]["error"]


def test_ring_slot_and_barrier_layout(golden):
  from hopper_wgmma import Ring
  ring = Ring(None, 0, golden["Ring_slot"]["stages"], 2, 1)
  assert [list(ring.slot(j)) for j in range(10)] == golden["Ring_slot"]["slots"]
  r = Ring(None, 1024, 4)
  assert [r.full(s) for s in range(4)] == [1024, 1032, 1040, 1048]
  assert r.empty(0) == 1024 + 32 and r.producer_parity(0) == 1


def test_region_semantics():
  from hopper_wgmma import region
  assert list(region(True, 0)) == [0] and list(region(False, 0)) == []


def test_make_tensor_map_argument_checks_match_reference(golden):
  from hopper_wgmma.tensor_map import make_tensor_map
  for case in golden["make_tensor_map"]:
    with pytest.raises(ValueError) as exc:
      make_tensor_map(None, *case["args"])
    assert str(exc.value) == case["error"]


def test_builders_register_their_shared_memory_and_run_honours_a_lower_budget():
  """build_gemm_ws / build_gated_gemm register their dynamic shared memory per kernel name, as the reference's
  builders do (gemm.py:316, gated.py:65); a lower registered size cuts the plan's ring to the stages that fit."""
  from hopper_wgmma import GatedCfg, WSCfg, build_gated_gemm, build_gemm_ws, runtime
  cfg = WSCfg(tma_store=True, cluster=2, hilbert=True)
  run = build_gemm_ws(4096, cfg)
  assert runtime.dynamic_smem_bytes(run.kernel_name) == cfg.smem_bytes
  gated = build_gated_gemm(512, GatedCfg())
  assert runtime.dynamic_smem_bytes(gated.kernel_name) == GatedCfg().smem_bytes
  small = cfg.within_smem(150_000)
  assert small.stages == 3 and small.smem_bytes <= 150_000 and cfg.within_smem(cfg.smem_bytes) is cfg
  with pytest.raises(ValueError, match="fewer than 2 stages"):
    cfg.within_smem(60_000)


def test_runtime_hooks_are_compatible_noops():
  from hopper_wgmma.runtime import install_runtime_hooks, set_dynamic_smem_bytes
  install_runtime_hooks()
  set_dynamic_smem_bytes("sm100_x", 1024)
  with pytest.raises(ValueError):
    set_dynamic_smem_bytes("other", 1024)
  with pytest.raises(ValueError):
    set_dynamic_smem_bytes("sm100_x", 300 * 1024)


# ----------------------------------------------------------------------------------------------------------------
# tile orders: Python API and the C++ builders the kernel uses, against the reference
# ----------------------------------------------------------------------------------------------------------------
def test_python_hilbert_schedule_matches_reference(golden):
  from hopper_wgmma import hilbert_schedule
  for case in golden["hilbert_schedule"]:
    if "error" in case:
      with pytest.raises(ValueError) as exc:
        hilbert_schedule(case["M"], case["N"], case["cores"])
      assert str(exc.value) == case["error"]
    else:
      assert hilbert_schedule(case["M"], case["N"], case["cores"]) == case["ok"]


def test_cpp_hilbert_order_deals_like_reference(golden):
  from hopper_wgmma import _capi
  from oracle import schedule_ref
  for case in golden["hilbert_schedule"]:
    curve = _capi.hilbert_order(case["M"], case["N"])
    assert curve == schedule_ref.hilbert_curve(case["M"], case["N"])
    if "ok" in case:
      dealt = schedule_ref.assignment(curve, case["cores"])
      assert [v for c in dealt for v in c] == case["ok"]


def test_pruned_hilbert_walks_match_the_full_square_walk():
  """The C++ and Python builders skip curve blocks outside the grid; the order must stay the one the full-square
  walk of the reference (gemm.py:222-235, restated in oracle/schedule_ref.py) gives, on square, tall and wide
  grids."""
  import itertools
  from hopper_wgmma import _capi
  from hopper_wgmma.gemm import hilbert_order
  from oracle import schedule_ref
  for M, N in itertools.chain(itertools.product((1, 2, 3, 5, 8, 13, 31, 33, 64, 100), (1, 2, 3, 4, 9, 17, 40)),
                              [(257, 1), (1, 300), (130, 7), (6, 129)]):
    full = schedule_ref.hilbert_curve(M, N)
    assert _capi.hilbert_order(M, N) == full, (M, N)
    assert hilbert_order(M, N) == full, (M, N)


def test_tall_grid_schedule_is_cheap():
  """2^20 rows of 128-row tiles and one column tile: the full-square walk would visit 8192^2 = 67 M cells."""
  import time
  from hopper_wgmma import _capi
  t0 = time.perf_counter()
  curve = _capi.hilbert_order(8192, 1)
  assert time.perf_counter() - t0 < 0.05
  assert sorted(e >> 16 for e in curve) == list(range(8192))


def test_cpp_and_python_grouped_orders_match_reference(golden):
  from hopper_wgmma import _capi
  from hopper_wgmma.gemm import grouped_tile_order
  for case in golden["grouped_tile_order"]:
    CMT, NT, GM, GN = case["CMT"], case["NT"], case["GM"], case["GN"]
    table = _capi.grouped_order(CMT, NT, GM, GN)
    assert [[e >> 16, e & 0xFFFF] for e in table] == case["coords"]
    coords, two_d = grouped_tile_order(CMT, NT, GM, GN)
    assert two_d == case["grouped_2d"]
    assert [list(coords(t)) for t in range(CMT * NT)] == case["coords"]


def test_cpp_schedule_builders_reject_bad_sizes():
  from hopper_wgmma import _capi
  with pytest.raises(ValueError):
    _capi.grouped_order(4, 4, 5, 1)
  with pytest.raises(ValueError):
    _capi.hilbert_order(0, 4)


def test_ragged_shape_contract():
  from hopper_wgmma import WSCfg, build_gemm_ws
  with pytest.raises(ValueError, match="not a multiple of tile"):
    build_gemm_ws(500, WSCfg())
  run = build_gemm_ws(520, WSCfg(ragged=True), 300, 200)
  assert run.kernel_name.startswith("sm100_300x520x200")
  with pytest.raises(ValueError, match="multiples of 8"):
    build_gemm_ws(522, WSCfg(ragged=True), 300, 200)
  with pytest.raises(ValueError, match="multiples of 8"):
    build_gemm_ws(520, WSCfg(ragged=True), 300, 201)


@pytest.mark.parametrize("splits,width", [(2, 64), (2, 128), (2, 256), (4, 128), (4, 256)])
def test_split_k_cluster_exchange_layout(splits, width):
  """The index arithmetic of the cluster split-K exchange (kc_epilogue in csrc/gemm_kernels.cuh), checked on the
  host: every 16-byte piece a CTA sends lands inside its owner's receive region ((splits - 1) x 128 lanes x
  width / splits x 4 bytes, the host's expect_tx count) at an offset no other piece uses, the owner reads each piece
  at the offset it was written to, and the owner sees every other split exactly once per owned chunk."""
  nch = width // 32
  per = nch // splits
  recv_bytes = (splits - 1) * 128 * (width // splits) * 4
  written = {}   # (owner, byte offset) -> (sender, chunk, warp, lane, piece)
  for ks in range(splits):                       # sender: its chunks owned by others
    for c in range(nch):
      g = c // per
      if g == ks: continue
      j = ks if ks < g else ks - 1
      for q in range(4):
        for lane in range(32):
          for e in range(8):
            off = ((j * 4 + q) * per + (c - g * per)) * 4096 + lane * 16 + 512 * e
            assert 0 <= off and off + 16 <= recv_bytes
            assert (g, off) not in written
            written[(g, off)] = (ks, c, q, lane, e)
  assert len(written) * 16 == splits * recv_bytes   # every byte of every receive region is written once
  for g in range(splits):                         # owner: its chunks, the other splits in split order
    for cc in range(per):
      for s in range(splits):
        if s == g: continue
        j = s if s < g else s - 1
        for q in range(4):
          for lane in range(32):
            for e in range(8):
              off = ((j * 4 + q) * per + cc) * 4096 + lane * 16 + 512 * e
              assert written[(g, off)] == (s, g * per + cc, q, lane, e)
