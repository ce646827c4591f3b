"""CPU restatement of the reference's tile orders. TEST INFRASTRUCTURE ONLY (see oracle/gemm_ref.py).

Restates, as plain Python integer arithmetic:
  * ``grouped_tile_order`` (hopper_wgmma/gemm.py:200-215): GM x GN super-tiles in row-major order when they divide
    the CMT x NT grid, else the 1-D GROUP_M order whose ``UOp.where`` (gemm.py:212) is the conditional below;
  * ``hilbert_schedule`` (hopper_wgmma/gemm.py:218-240): tiles of the smallest power-of-two square covering the grid,
    walked in Hilbert order, kept if inside the grid, dealt round-robin over ``cores``, returned core-major;
  * the persistent loop's dealing of tile ids to clusters (gemm.py:309-337: cluster ``cid`` runs tiles
    cid, cid+NCL, ...) as a flat "dealt" table: entry i runs on cluster i % NCL at slot i // NCL.
Pinned against tests/golden/reference_host.json, produced by running the reference's own functions
(tests/golden/make_golden.py).
"""
from __future__ import annotations


def grouped_coords(CMT: int, NT: int, GM: int, GN: int, tile: int) -> tuple[int, int]:
  if CMT % GM == 0 and NT % GN == 0:
    st, pos = tile // (GM * GN), tile % (GM * GN)
    return (st // (NT // GN)) * GM + pos // GN, (st % (NT // GN)) * GN + pos % GN
  first = (tile // (GM * NT)) * GM
  rows = (CMT - first) if first > CMT - GM else GM
  r = tile % (GM * NT)
  return first + r % rows, r // rows


def is_grouped_2d(CMT: int, NT: int, GM: int, GN: int) -> bool:
  return CMT % GM == 0 and NT % GN == 0


def d2xy(n: int, d: int) -> tuple[int, int]:
  x = y = 0
  s, t = 1, d
  while s < n:
    rx = 1 & (t // 2)
    ry = 1 & (t ^ rx)
    if ry == 0:
      if rx == 1:
        x, y = s - 1 - x, s - 1 - y
      x, y = y, x
    x += s * rx
    y += s * ry
    t //= 4
    s *= 2
  return x, y


def hilbert_curve(M: int, N: int) -> list[int]:
  dim = 1
  while dim < max(M, N):
    dim *= 2
  out = []
  for i in range(dim * dim):
    x, y = d2xy(dim, i)
    if x < M and y < N:
      out.append((x << 16) | y)
  return out


def hilbert_schedule(M: int, N: int, cores: int) -> list[int]:
  curve = hilbert_curve(M, N)
  per_core: list[list[int]] = [[] for _ in range(cores)]
  for p, v in enumerate(curve):
    per_core[p % cores].append(v)
  if any(len(c) != len(per_core[0]) for c in per_core):
    raise ValueError(f"hilbert needs an equal number of tiles per core ({M}x{N} tiles over {cores} cores)")
  return [v for c in per_core for v in c]


def dealt_grouped(CMT: int, NT: int, GM: int, GN: int) -> list[int]:
  """Dealt table of the persistent kernel with the grouped order: entry i = coords(i)."""
  out = []
  for t in range(CMT * NT):
    r, c = grouped_coords(CMT, NT, GM, GN, t)
    out.append((r << 16) | c)
  return out


def assignment(dealt: list[int], nclusters: int) -> list[list[int]]:
  """Per-cluster tile lists of a dealt table: cluster c runs entries c, c + nclusters, ..."""
  return [dealt[c::nclusters] for c in range(nclusters)]
