"""N-column sharding of one GEMM over the GPUs of a node: one process per GPU, A replicated, B and C split by
columns, no communication inside the GEMM. Rank r of W owns output columns [r*N/W, (r+1)*N/W): its B shard is that
column block of B, i.e. the contiguous row block BT[r*N/W : (r+1)*N/W, :] of the K-major copy, and its C shard is an
M x N/W block (its own buffer, or a column view of a full C written through the row pitch).

The reference has no multi-GPU path; the partitioning is the one its benchmark configuration names. The only
collectives are optional and outside the GEMM: an all-gather of the C shards and a max-reduction of per-rank kernel
times (whole-job throughput is total FLOPs over the slowest rank).
"""
from __future__ import annotations

from .gemm import WSCfg, plan_gemm_bt


def column_range(N: int, world: int, rank: int, BN: int = 1) -> tuple[int, int]:
  """Columns [start, stop) owned by ``rank``: equal shards, each a multiple of the tile width ``BN``."""
  if world < 1 or not 0 <= rank < world: raise ValueError(f"rank {rank} out of range for world size {world}")
  if N % world: raise ValueError(f"N={N} does not split into {world} equal column shards")
  n = N // world
  if n % BN: raise ValueError(f"column shard {n} is not a multiple of the tile width {BN}")
  return rank * n, (rank + 1) * n


def shard_bt(BT, world: int, rank: int, BN: int = 1):
  """This rank's rows of the K-major BT[N, K] (a view, no copy)."""
  c0, c1 = column_range(BT.shape[0], world, rank, BN)
  return BT[c0:c1]


def local_gemm(A, BT_shard, C_shard, cfg: WSCfg, **hooks):
  """The rank's GEMM C_shard[M, n] = A[M, K] @ BT_shard[n, K]^T on its own GPU; returns ``launch``."""
  return plan_gemm_bt(A, BT_shard, C_shard, cfg, **hooks)


def gather_columns(C_shard, world: int, group=None, as_row_major: bool = True):
  """All-gather the column shards of every rank. Returns the [M, N] matrix (or the [world, M, n] stack when
  ``as_row_major`` is False, which skips the final permute copy)."""
  import torch
  import torch.distributed as dist
  M, n = C_shard.shape
  stack = torch.empty((world, M, n), dtype=C_shard.dtype, device=C_shard.device)
  if dist.get_backend(group) == "nccl":
    dist.all_gather_into_tensor(stack, C_shard.contiguous(), group=group)
  else:                                  # gloo (CPU ranks): list form
    dist.all_gather(list(stack.unbind(0)), C_shard.contiguous(), group=group)
  if not as_row_major: return stack
  return stack.permute(1, 0, 2).reshape(M, world * n)


def max_over_ranks(value: float, device=None, group=None) -> float:
  """The maximum of a per-rank scalar over all ranks (whole-job time is the slowest rank's)."""
  import torch
  import torch.distributed as dist
  t = torch.tensor([float(value)], dtype=torch.float64, device=device)
  dist.all_reduce(t, op=dist.ReduceOp.MAX, group=group)
  return float(t.item())
