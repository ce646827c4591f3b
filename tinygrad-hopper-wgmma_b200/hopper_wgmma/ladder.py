"""The optimization ladder as named configs (the reference's hopper_wgmma/ladder.py:7-37), on B200.

Names and knob combinations are the reference's. Knobs the reference hard-coded for an H200 are left at their
B200 defaults: ``num_sm`` is the device's SM count and ``stages`` fills shared memory."""
from __future__ import annotations

from .gated import GatedCfg, build_gated_gemm
from .gemm import WSCfg, build_gemm_ws

LADDER = {
  "tma_ring": GatedCfg(BN=128, stages=4, consumers=0),            # one thread drives the TMA ring and the MMAs
  "gated_ws": GatedCfg(consumers=2),                              # warp specialization, one tile per CTA
  "role_split": WSCfg(),                                          # persistent, role-split, 16x8 tile order
  "role_split_regs": WSCfg(regs=(24, 240)),                       # role_split + register split knob
  "tma_store": WSCfg(tma_store=True),                             # + swizzled staging / TMA-store epilogue
  "hilbert": WSCfg(tma_store=True, hilbert=True),                 # + Hilbert tile order
  "cluster": WSCfg(tma_store=True, cluster=2),                    # CTA pairs on cta_group::2 (instead of Hilbert)
  "cluster_hilbert": WSCfg(tma_store=True, hilbert=True, cluster=2),
}


def build(N: int, cfg, M: int | None = None, K: int | None = None, **hooks):
  """Build the right GEMM for ``cfg``. Gated configs are square only."""
  if isinstance(cfg, GatedCfg):
    if (M, K) not in ((None, None), (N, N)): raise ValueError("the gated builder is square only")
    return build_gated_gemm(N, cfg, **hooks)
  return build_gemm_ws(N, cfg, M, K, **hooks)


# Tile shapes the shape sweep adds to the ladder's: 192-column tiles split widths such as 3072 into whole tiles.
SWEEP = {
  "tma_store": LADDER["tma_store"],
  "hilbert": LADDER["hilbert"],
  "tma_store_n192": WSCfg(BN=192, tma_store=True),
  "hilbert_n192": WSCfg(BN=192, tma_store=True, hilbert=True),
}

# B200 tile shapes beyond the reference's ladder: CTA pairs with 256 x 512 tiles (two N=256 MMAs per K step, one
# 512-column TMEM accumulator), which read a quarter fewer operand bytes per FLOP than 256 x 256.
B200 = {
  "pair_wide": WSCfg(tma_store=True, cluster=2, n_mma=2),
  "pair_wide_hilbert": WSCfg(tma_store=True, cluster=2, n_mma=2, hilbert=True),
  "pair_n128": WSCfg(BN=128, tma_store=True, cluster=2, hilbert=True),
  "pair_n192": WSCfg(BN=192, tma_store=True, cluster=2, hilbert=True),
  "pair_reg": WSCfg(cluster=2, hilbert=True),
  "cta_n128": WSCfg(BN=128, tma_store=True, hilbert=True),
  "cta_n64": WSCfg(BN=64, tma_store=True, hilbert=True),
  "m64_n128": WSCfg(consumers=1, BN=128, tma_store=True, hilbert=True),
}

# The shape sweep of the benchmark configuration (12 tile-multiple shapes) and the configs tried on each.
SWEEP_SHAPES = [(512, 512, 512), (1024, 1024, 1024), (1536, 1536, 1536), (2048, 2048, 2048), (3072, 3072, 3072),
                (6144, 6144, 6144), (12288, 12288, 12288), (16384, 16384, 16384), (16384, 4096, 4096),
                (4096, 16384, 4096), (8192, 8192, 2048), (2048, 2048, 16384)]
SWEEP_CONFIGS = ["cluster_hilbert", "hilbert", "pair_wide_hilbert", "pair_n128", "pair_n192", "cta_n128", "cta_n64",
                 "m64_n128", "hilbert_n192"]

# One-off comparisons quoted by the reference (all SMs vs 128 on an H200); here: 128 CTAs vs the device count.
EXTRA = {
  "tma_store_132": WSCfg(tma_store=True, num_sm=132),
  "tma_store_128": WSCfg(tma_store=True, num_sm=128),
}


def lookup(name: str):
  """A config by name from LADDER, SWEEP, B200 or EXTRA, with optional ``@`` modifiers so that sweeps can vary one
  knob on any tile shape: ``@sk<S>`` sets ``split_k=S`` (``@skA`` = automatic), ``@reg`` selects the register
  epilogue (``tma_store=False``), ``@s<N>`` sets the ring depth ``stages=N``, ``@bT`` makes build_gemm_ws copy B
  to a K-major BT first (``b_nmajor=False``, the reference's operand layout), ``@bN`` makes it read B[K,N]
  directly wherever the tile allows (``b_nmajor=True``) and ``@g<M>x<N>`` replaces the tile order by the grouped
  order with ``group_m=M, group_n=N`` (``hilbert=False``); ``@wsync`` / ``@nowsync`` force the wave barrier
  on or off (``wave_sync``); ``@skc`` / ``@skw`` make split-K meet inside a cluster or through the workspace
  (``split_k_cluster``). Example: ``cta_n128@sk2``, ``cta_n128@sk2@skw``, ``cta_n64@reg@skA``,
  ``pair_n128@s4``, ``cluster_hilbert@bT``, ``cta_n128@bN``, ``pair_wide@g64x8``."""
  import dataclasses
  base, *mods = name.split("@")
  cfg = {**LADDER, **SWEEP, **EXTRA, **B200}[base]
  for mod in mods:
    if not isinstance(cfg, WSCfg): raise ValueError(f"{base} is not a persistent config: no @{mod}")
    if mod == "reg":
      cfg = dataclasses.replace(cfg, tma_store=False)
    elif mod in ("skc", "skw"):
      cfg = dataclasses.replace(cfg, split_k_cluster=mod == "skc")
    elif mod.startswith("sk") and (mod[2:].isdigit() or mod[2:] == "A"):
      cfg = dataclasses.replace(cfg, split_k=-1 if mod[2:] == "A" else int(mod[2:]))
    elif mod in ("bT", "bN"):
      cfg = dataclasses.replace(cfg, b_nmajor=mod == "bN")
    elif mod in ("wsync", "nowsync"):
      cfg = dataclasses.replace(cfg, wave_sync=mod == "wsync")
    elif mod.startswith("g") and "x" in mod and all(p.isdigit() for p in mod[1:].split("x", 1)):
      gm, gn = (int(p) for p in mod[1:].split("x", 1))
      cfg = dataclasses.replace(cfg, group_m=gm, group_n=gn, hilbert=False)
    elif mod.startswith("s") and mod[1:].isdigit():
      cfg = dataclasses.replace(cfg, stages=int(mod[1:]))
    else:
      raise KeyError(f"unknown config modifier {mod!r} in {name!r}")
  return cfg


def best_config(M: int, N: int, K: int) -> WSCfg:
  """The config the B200 Nsight Compute shape sweep (``python -m hopper_wgmma.report ncu-sweep``) found fastest
  for a problem of this size:
  256x512 CTA-pair tiles once the GEMM is big enough to run at the power cap (M*N*K >= 6144^3), where they move a
  quarter fewer operand bytes per FLOP; 256x256 pair tiles from 2048^2 outputs up; 128x128 CTA tiles below, with
  split-K chosen automatically (it splits only shapes with few tiles and a long K). The pair tiles also read B as
  given (no transposed copy in ``run``). Tile-multiple shapes are assumed; pass ``ragged=True`` yourself otherwise."""
  import dataclasses
  if M * N * K >= 6144 ** 3: return B200["pair_wide_hilbert"]
  if M * N >= 2048 * 2048: return LADDER["cluster_hilbert"]
  return dataclasses.replace(B200["cta_n128"], split_k=-1)

