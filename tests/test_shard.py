"""Column sharding on CPU ranks (gloo, world size 2): the partition, the gather and the max-over-ranks timing, with
the per-rank GEMM stubbed by the CPU oracle; and failure detection on the host — a rank that raises before the
gather makes its peer's collective end with an error after the process group's short timeout instead of hanging."""
from __future__ import annotations

import os
import socket
import sys
import traceback
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent


def _free_port() -> int:
  with socket.socket() as s:
    s.bind(("127.0.0.1", 0))
    return s.getsockname()[1]


def _worker(rank: int, world: int, port: int, mode: str, out_dir: str):
  sys.path[:0] = [str(ROOT / "tinygrad-hopper-wgmma_b200"), str(ROOT)]
  from datetime import timedelta

  import numpy as np
  import torch
  import torch.distributed as dist

  from hopper_wgmma import shard
  from oracle import gemm_ref
  status = "ok"
  try:
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=6))
    M, N, K = 64, 128, 96
    a_bits, b_bits = gemm_ref.randn_bf16_bits((M, K), 0), gemm_ref.randn_bf16_bits((K, N), 1)
    c0, c1 = shard.column_range(N, world, rank, BN=16)
    bt_bits = np.ascontiguousarray(b_bits.T)
    bt_shard = shard.shard_bt(bt_bits, world, rank, BN=16)
    assert bt_shard.shape == (c1 - c0, K)
    c_shard = gemm_ref.gemm_f32(a_bits, np.ascontiguousarray(bt_shard.T))   # the rank's GEMM, oracle-stubbed
    if mode == "fail" and rank == 1:
      raise RuntimeError("injected rank failure before the gather")
    full = shard.gather_columns(torch.from_numpy(c_shard), world)
    assert torch.equal(full, torch.from_numpy(gemm_ref.gemm_f32(a_bits, b_bits)))
    stack = shard.gather_columns(torch.from_numpy(c_shard), world, as_row_major=False)
    assert tuple(stack.shape) == (world, M, N // world)
    assert shard.max_over_ranks(float(rank + 1)) == float(world)
    dist.barrier()
  except Exception as exc:
    status = f"error: {type(exc).__name__}: {exc}\n{traceback.format_exc()}"
  finally:
    Path(out_dir, f"rank{rank}.txt").write_text(status)
    if dist.is_initialized():
      try:
        dist.destroy_process_group()
      except Exception:
        pass


def _run(mode: str, tmp_path) -> dict[int, str]:
  import torch.multiprocessing as mp
  world, port = 2, _free_port()
  ctx = mp.get_context("spawn")
  procs = [ctx.Process(target=_worker, args=(r, world, port, mode, str(tmp_path))) for r in range(world)]
  for p in procs: p.start()
  for p in procs: p.join(timeout=120)
  for p in procs:
    if p.is_alive():
      p.kill()
      pytest.fail("a rank did not finish")
  return {r: (tmp_path / f"rank{r}.txt").read_text() for r in range(world)}


def test_column_shards_gather_to_the_full_product(tmp_path):
  res = _run("ok", tmp_path)
  assert res == {0: "ok", 1: "ok"}, res


def test_failed_rank_surfaces_as_error_on_peer(tmp_path):
  res = _run("fail", tmp_path)
  assert res[1].startswith("error: RuntimeError: injected")
  assert res[0].startswith("error:"), res[0]   # the peer's gather ended with an error instead of hanging


def test_column_range_contract():
  sys.path[:0] = [str(ROOT / "tinygrad-hopper-wgmma_b200")]
  from hopper_wgmma import shard
  assert [shard.column_range(32768, 8, r, 512) for r in (0, 7)] == [(0, 4096), (28672, 32768)]
  with pytest.raises(ValueError):
    shard.column_range(1000, 3, 0)
  with pytest.raises(ValueError):
    shard.column_range(1024, 4, 0, BN=512)
  with pytest.raises(ValueError):
    shard.column_range(1024, 4, 4)
