"""The first two ladder steps on B200: a TMA ring driven by one thread, then warp specialization without
persistence (the reference's hopper_wgmma/gated.py).

``consumers=0`` ("tma_ring"): one 128-thread CTA per tile; a single thread fills the shared-memory ring with TMA and
issues every ``tcgen05.mma`` itself, refilling each stage once the MMA has read it; all four warps then drain the
TMEM accumulator with register stores. ``consumers=1|2`` ("gated_ws"): the warp-specialized kernel (TMA warp, MMA
warp, epilogue warpgroup), one tile per CTA in row-major tile order (gated.py:81), one accumulator, register stores.
Square problems only, as in the reference (gated.py:56, :113)."""
from __future__ import annotations

from dataclasses import dataclass

from . import _capi, runtime
from .gemm import SMEM_ALIGN_SLACK, SMEM_LIMIT, Ring, _make_launch
from .tensors import current_stream, operand, transpose_contiguous


@dataclass(frozen=True)
class GatedCfg:
  """consumers=0: one thread drives both the TMA ring and the MMAs. consumers=1|2: warp-specialized roles."""
  BN: int = 256
  BK: int = 64
  stages: int = 3
  consumers: int = 2

  def __post_init__(self):
    if self.BK != 64: raise ValueError("BK must be 64 (one 128-byte swizzle atom)")
    if self.BN <= 0 or self.BN % 16 or self.BN > 256: raise ValueError("BN must be a multiple of 16 in (0, 256]")
    if self.stages < 2: raise ValueError("stages must be at least 2")
    if self.consumers not in (0, 1, 2): raise ValueError("consumers must be 0, 1 or 2")
    if self.smem_bytes > SMEM_LIMIT: raise ValueError(f"needs {self.smem_bytes} bytes of shared memory, the limit is {SMEM_LIMIT}")

  @property
  def ncons(self): return max(self.consumers, 1)
  @property
  def BM(self): return 64 * self.ncons
  @property
  def threads(self): return 256 if self.consumers else 128
  @property
  def tmem_cols(self): return self.BN
  @property
  def a_elems(self): return self.BM * self.BK
  @property
  def b_elems(self): return self.BN * self.BK
  @property
  def smem_bytes(self):
    fixed = SMEM_ALIGN_SLACK + (48 if self.consumers else 16)
    return fixed + ((self.a_elems + self.b_elems) * 2 + Ring.BYTES_PER_STAGE) * self.stages

  def to_c(self, wait_budget_ns: int = 0, debug_skip_job: int = -1) -> _capi.BgCfg:
    kind = _capi.KIND_GATED if self.consumers else _capi.KIND_RING
    return _capi.BgCfg(kind=kind, BN=self.BN, BK=self.BK, stages=self.stages, consumers=self.consumers, num_sm=0,
                       group_m=1, group_n=1, tma_store=0, cluster=1, hilbert=0, acc_bufs=1,
                       wait_budget_ns=wait_budget_ns, debug_skip_job=debug_skip_job, n_mma=1,
                       no_tail_split=1)


def build_gated_gemm(N: int, cfg: GatedCfg, *, wait_budget_ns: int = 0, debug_skip_job: int = -1):
  """C[N,N] (bf16) = A[N,N] @ B[N,N], one CTA per output tile. Same contract as ``build_gemm_ws``."""
  BM, BN, BK, QS = cfg.BM, cfg.BN, cfg.BK, cfg.stages
  if N <= 0 or N % BM or N % BN or N % BK: raise ValueError(f"N={N} must be a multiple of the tile {BM}x{BN}x{BK}")
  NK = N // BK
  if NK < QS: raise ValueError(f"K has {NK} blocks, fewer than {QS} stages")
  kernel_name = f"sm100_gated_{N}_c{cfg.consumers}_s{QS}_n{BN}"
  runtime.set_dynamic_smem_bytes(kernel_name, cfg.smem_bytes)   # as the reference's builder does (gated.py:65)

  def run(A, B, Cout):
    a, b, c = operand(A), operand(B), operand(Cout)
    if a.shape != (N, N) or b.shape != (N, N) or c.shape != (N, N): raise ValueError("A, B and C must be N x N")
    if not (a.bf16 and b.bf16 and c.bf16): raise ValueError("A, B and C must be bfloat16")
    if not (a.device == b.device == c.device): raise ValueError("A, B and C must be on the same device")
    BT = transpose_contiguous(B)   # keep alive: the tensor maps hold raw device pointers
    bt = operand(BT)
    plan = _capi.Plan(cfg.to_c(wait_budget_ns, debug_skip_job), N, N, N, a.ptr, a.row_pitch, bt.ptr, bt.row_pitch,
                      c.ptr, c.row_pitch, a.device)
    return _make_launch(plan, lambda: current_stream(Cout), Cout, (A, BT, Cout))
  run.out_dtype = "bfloat16"
  run.kernel_name = kernel_name
  run.cuda_kernel = "regex:sm100_gemm_ring" if cfg.consumers == 0 else "regex:sm100_gemm_ws"
  run.cfg = cfg
  return run
