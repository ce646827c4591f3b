"""Warp-specialized bf16 GEMM for B200 (sm_100a): the host layer over the hand-written tcgen05 kernel.

Same operator API as the reference's Hopper builder (hopper_wgmma/gemm.py): ``build_gemm_ws(N, WSCfg(...), M, K)``
returns ``run(A, B, C)``, which returns ``launch()``; ``launch()`` enqueues the GEMM and returns C. bf16 in, fp32
accumulate, bf16 out; A is M x K row-major, B is K x N and is transposed once in ``run`` to the K-major BT the kernel
reads (gemm.py:387); M, N and K are multiples of the tile.

What changed underneath, and why:
  * The kernel is CUDA C++ with inline PTX, compiled ahead of time for sm_100a (``csrc/``) and called through a C ABI
    (``include/sm100_gemm.h``), instead of tinygrad UOps rendered and compiled at first launch.
  * MMA is ``tcgen05.mma`` with fp32 accumulators in tensor memory (TMEM): one thread issues it, the epilogue warps
    read TMEM with ``tcgen05.ld``. BM is still ``64 * consumers`` rows per CTA (M = 64 or 128 per instruction).
  * ``cluster=2`` (with ``consumers=2``) pairs two CTAs on one M = 256 ``tcgen05.mma.cta_group::2``: each CTA loads its
    own A rows and half of the B tile. The reference multicasts B into the pair instead (gemm.py:90-94, 361); no load
    here is multicast.
  * ``num_sm=None`` (the default) uses the device's SM count, and a Hilbert order may deal tiles unevenly over the
    clusters; the reference hard-codes 128 CTAs (gemm.py:252) and rejects uneven Hilbert splits (gemm.py:311).
  * ``stages=None`` (the default) fills shared memory with as many stages as fit.
  * Every device-side wait is bounded; a timeout is reported through ``launch.check()`` instead of hanging the GPU.
"""
from __future__ import annotations

from dataclasses import dataclass

from . import _capi, runtime
from .tensors import current_stream, operand, transpose_contiguous

SMEM_LIMIT = 227 * 1024   # opt-in dynamic shared memory per block on B200 (the same figure as H100/H200)
SMEM_ALIGN_SLACK = 1024   # the kernel aligns its dynamic shared memory to 1024 bytes itself


# =============================================================================================================
# helpers: the shared-memory ring, warp-role regions, tile orders
# =============================================================================================================
def region(cond, axis: int = 0) -> range:
  """A loop that runs once when ``cond`` holds and zero times otherwise: the reference's way to give a warp role its
  own code block (gemm.py:151-154). In this build warp roles are plain C++ branches in the kernel; the helper keeps
  the name and meaning for host-side code written against it."""
  return range(1 if cond else 0)


class Ring:
  """Host model of the kernel's ``stages``-deep shared-memory queue (gemm.py:157-189 is the reference's).

  Stage s owns a FULL barrier (one arrival from the producer's expect_tx, completed by the TMA bytes; in a CTA pair
  the even CTA's barrier counts both CTAs' bytes) and an EMPTY barrier (one arrival: the ``tcgen05.commit`` issued
  after the stage's MMAs, sent to both CTAs of a pair). Iteration j uses stage ``j % stages`` with phase parity
  ``(j // stages) % 2``. The producer waits on EMPTY with the opposite parity, so a fresh ring starts out empty and
  needs no priming arrivals. Barrier byte offsets match the kernel's layout: FULL s at ``bar_off + 8 s``, EMPTY s at
  ``bar_off + 8 (stages + s)``."""
  BYTES_PER_STAGE = 16                                    # two 8-byte mbarriers

  def __init__(self, smem=None, bar_off: int = 0, stages: int = 2, consumers: int = 1, cluster: int = 1):
    if stages < 2: raise ValueError("stages must be at least 2")
    self.smem, self.bar_off, self.stages, self.consumers, self.cluster = smem, bar_off, stages, consumers, cluster

  def full(self, s: int, dep=None) -> int: return self.bar_off + 8 * s
  def empty(self, s: int, dep=None) -> int: return self.bar_off + 8 * (self.stages + s)
  def slot(self, j: int) -> tuple[int, int]: return j % self.stages, (j // self.stages) % 2
  def producer_parity(self, j: int) -> int: return self.slot(j)[1] ^ 1


def grouped_tile_order(CMT: int, NT: int, GM: int, GN: int):
  """Linear tile id -> (tile row, tile col) (gemm.py:200-215). If GM x GN super-tiles divide the grid: row-major over
  super-tiles, row-major inside one. Else GROUP_M: GM tile rows swept across all NT columns, column-major inside the
  group, the last group ragged. Returns ``(coords, grouped_2d)``."""
  if CMT % GM == 0 and NT % GN == 0:
    per_row = NT // GN

    def coords(tile: int) -> tuple[int, int]:
      st, pos = divmod(tile, GM * GN)
      return (st // per_row) * GM + pos // GN, (st % per_row) * GN + pos % GN
    return coords, True

  def coords1d(tile: int) -> tuple[int, int]:
    first = (tile // (GM * NT)) * GM
    rows = CMT - first if first > CMT - GM else GM
    r = tile % (GM * NT)
    return first + r % rows, r // rows
  return coords1d, False


def _hilbert_d2xy(n: int, d: int) -> tuple[int, int]:
  """Position d on the Hilbert curve over an n x n grid (n a power of two) -> (x, y); iterative walk."""
  x = y = 0
  s, t = 1, d
  while s < n:
    rx = 1 & (t // 2)
    ry = 1 & (t ^ rx)
    if ry == 0:
      if rx == 1: x, y = s - 1 - x, s - 1 - y
      x, y = y, x
    x, y = x + s * rx, y + s * ry
    t //= 4
    s *= 2
  return x, y


def hilbert_order(M: int, N: int) -> list[int]:
  """Tiles of an M x N tile grid in Hilbert-curve order, as (m << 16) | n: the order in which the curve over the
  smallest power-of-two square covering the grid visits them (gemm.py:222-235 walks the whole square and keeps the
  cells inside the grid). The curve covers each aligned s x s block in one run of s * s positions, so runs whose
  block lies outside the grid are skipped whole and tall or wide grids cost O(cells * log dim), not O(dim^2)."""
  dim = 1
  while dim < max(M, N): dim *= 2
  out: list[int] = []
  stack = [(0, dim)]                     # (first curve position of a block, block side), visited in curve order
  while stack:
    d0, s = stack.pop()
    x, y = _hilbert_d2xy(dim, d0)
    if (x & ~(s - 1)) >= M or (y & ~(s - 1)) >= N: continue
    if s == 1:
      out.append((x << 16) | y)
      continue
    q = (s // 2) * (s // 2)
    stack.extend((d0 + i * q, s // 2) for i in (3, 2, 1, 0))
  return out


def hilbert_schedule(M: int, N: int, cores: int) -> list[int]:
  """Walk an M x N tile grid along a Hilbert curve and deal the tiles round-robin to ``cores`` (gemm.py:218-240),
  so that at step i the cores work on curve positions [i*cores, (i+1)*cores). Returns a flat [cores][M*N/cores]
  table of (m << 16) | n and raises ValueError if the tiles do not split evenly, as the reference does. (The kernel
  itself deals the same curve without that restriction, see ``hilbert_order``.)"""
  curve = hilbert_order(M, N)
  if len(curve) % cores:
    raise ValueError(f"hilbert needs an equal number of tiles per core ({M}x{N} tiles over {cores} cores)")
  return [curve[p] for c in range(cores) for p in range(c, len(curve), cores)]


# =============================================================================================================
# configuration
# =============================================================================================================
def _device_sm_count(device: int | None = None) -> int:
  import torch
  dev = torch.cuda.current_device() if device is None else device
  return _capi.device_info(dev)["sm_count"]


@dataclass(frozen=True)
class WSCfg:
  BN: int = 256                # output columns per tile = tcgen05.mma N (a multiple of 16, up to 256)
  BK: int = 64                 # one 128-byte swizzle row along K (the only supported value)
  stages: int | None = None    # shared-memory ring depth; None = as many as fit
  consumers: int = 2           # BM = 64 * consumers rows per CTA (tcgen05.mma M = 64 or 128)
  num_sm: int | None = None    # persistent CTAs (upper bound); None = the device's SM count
  group_m: int = 16            # L2 tile order, super-tiles of group_m x group_n tiles
  group_n: int = 8
  tma_store: bool = False      # swizzled shared-memory staging + TMA store epilogue
  regs: tuple[int, int] | None = None   # register split (producer, consumer): validated, not applied (the
                                        # kernels need <= 100 registers per thread without it)
  cluster: int = 1             # 2: two CTAs share one M = 256 MMA (cta_group::2), each loading half of B
  hilbert: bool = False        # Hilbert tile order from a host-built table
  acc_bufs: int | None = None  # accumulator buffers in tensor memory; None = 2 when 2 * width <= 512 columns
  n_mma: int = 1               # tcgen05.mma instructions along N per K step: tiles are n_mma * BN columns wide
  split_tail: bool = True      # split a last wave that is at most half full into half-width tiles
  ragged: bool = False         # accept any M (and N, K multiples of 8): edge tiles are zero-filled / clipped
  split_k: int = 1             # K splits per output tile (fp32 partial sums reduced in-kernel by the last split);
                               # -1 = chosen per shape (only shapes with few tiles and long K are split)
  k_serpentine: bool = True    # alternate the K direction from tile to tile of a cluster (L2 reuse across waves)
  b_nmajor: bool | None = None # build_gemm_ws reads B[K,N] as given (MN-major tcgen05 operand) instead of making
                               # the K-major copy BT (gemm.py:382): True = wherever the tile allows it, False = never,
                               # None = for CTA-pair tiles only (see reads_b_directly)
  wave_sync: bool | None = None  # the TMA producers of all CTAs meet at every tile boundary, keeping a wave's tiles
                               # in step so that they share operand panels through L2: True = on, False = off,
                               # None = on when each cluster runs >= 4 tiles and a wave's K-long operand panels
                               # outgrow L2 (256x512 pair tiles from K = 8192; no split-K)
  split_k_cluster: bool | None = None  # how split-K meets: True = the splits of a tile are the CTAs of one cluster
                               # and add up through distributed shared memory (single-CTA tiles, split_k 2 or 4, one
                               # wave), False = through a global fp32 workspace, None = the cluster where it applies

  def __post_init__(self):
    if self.BK != 64: raise ValueError("BK must be 64 (one 128-byte swizzle atom)")
    if self.BN <= 0 or self.BN % 16 or self.BN > 256: raise ValueError("BN must be a multiple of 16 in (0, 256]")
    if self.tma_store and self.BN % 64: raise ValueError("tma_store needs BN to be a multiple of 64")
    if self.stages is not None and self.stages < 2: raise ValueError("stages must be at least 2")
    if self.consumers not in (1, 2): raise ValueError("consumers must be 1 or 2")
    if self.cluster not in (1, 2): raise ValueError("cluster must be 1 or 2")
    if self.num_sm is not None and self.num_sm < self.cluster: raise ValueError("num_sm must be at least the cluster size")
    if self.group_m < 1 or self.group_n < 1: raise ValueError("group_m and group_n must be positive")
    if self.regs is not None and (len(self.regs) != 2 or any(r % 8 or not 24 <= r <= 256 for r in self.regs)):
      raise ValueError("regs must be two multiples of 8 in [24, 256]")
    if self.n_mma not in (1, 2): raise ValueError("n_mma must be 1 or 2")
    if self.split_k != -1 and not 1 <= self.split_k <= 64: raise ValueError("split_k must be -1 (auto) or in [1, 64]")
    if self.split_k > 1 and self.width % 32: raise ValueError("split_k needs tiles a multiple of 32 columns wide")
    if self.acc_bufs is not None and self.acc_bufs not in (1, 2): raise ValueError("acc_bufs must be 1 or 2")
    if self.wave_sync and self.split_k > 1: raise ValueError("wave_sync needs split_k = 1")
    if self.acc_bufs == 2 and 2 * self.width > 512: raise ValueError("two accumulators of the tile width exceed tensor memory")
    if self.stages_used < 2: raise ValueError(f"not even 2 stages fit in {SMEM_LIMIT} bytes of shared memory")
    if self.smem_bytes > SMEM_LIMIT: raise ValueError(f"needs {self.smem_bytes} bytes of shared memory, the limit is {SMEM_LIMIT}")

  @property
  def BM(self): return 64 * self.consumers
  @property
  def width(self): return self.BN * self.n_mma            # output columns per tile
  @property
  def paired(self): return self.cluster == 2 and self.BM == 128   # cta_group::2 across the CTA pair
  @property
  def threads(self): return 256                         # warp 0 TMA, warp 1 TMEM + MMA, warps 4-7 epilogue
  @property
  def tmem_cols(self): return self.width                # fp32 accumulator columns per buffer (BM lanes)
  @property
  def a_elems(self): return self.BM * self.BK
  @property
  def b_elems(self): return (self.BN // 2 if self.paired else self.BN) * self.BK * self.n_mma   # this CTA's B share
  @property
  def c_elems(self): return self.BM * 128 if self.tma_store else 0   # 4 warps x 2 buffers x (BM/4 rows x 64 cols)
  @property
  def stage_bytes(self): return (self.a_elems + self.b_elems) * 2 + Ring.BYTES_PER_STAGE
  @property
  def fixed_bytes(self): return SMEM_ALIGN_SLACK + self.c_elems * 2 + 56   # + accumulator/drain/receive barriers, TMEM slot
  @property
  def stages_used(self):
    if self.stages is not None: return self.stages
    return min(8, (SMEM_LIMIT - self.fixed_bytes) // self.stage_bytes)
  @property
  def smem_bytes(self): return self.fixed_bytes + self.stage_bytes * self.stages_used
  def within_smem(self, nbytes: int) -> "WSCfg":
    """This config with its shared-memory ring cut to the stages that fit in ``nbytes`` of dynamic shared memory
    (unchanged when they all fit). ValueError if not even two stages fit."""
    import dataclasses
    if self.smem_bytes <= nbytes: return self
    stages = min(self.stages_used, (nbytes - self.fixed_bytes) // self.stage_bytes)
    if stages < 2: raise ValueError(f"{nbytes} bytes of dynamic shared memory hold fewer than 2 stages of {self.name}")
    return dataclasses.replace(self, stages=stages)

  @property
  def reads_b_directly(self):
    """True when build_gemm_ws hands B[K,N] to the kernel without a transposed copy. N-major B arrives in 64-column
    boxes, so each CTA's share of a tile's columns (and of a half-width tail tile's) must be whole boxes. By default
    (b_nmajor=None) B is read directly where the MMA asks shared memory for at most 96 bytes per cycle: CTA pairs
    (64 B/cycle; the same kernel time with either layout) and 128 x 256 single-CTA tiles (96 B/cycle; within
    -1.4 % / +2.8 % at 4096^3 / 2048^3). Smaller single-CTA tiles come close to the SM's 128 bytes per cycle of shared
    memory, where the MN-major operand reads cost 5-15 % (128 x 128: -8 %, 64 x 128: -15 % at 4096^3; Nsight
    Compute), so they keep the reference's K-major copy."""
    wide_cta = not self.paired and self.BM == 128 and self.BN >= 256
    if self.b_nmajor is False or (self.b_nmajor is None and not (self.paired or wide_cta)): return False
    share = self.BN // 2 if self.paired else self.BN
    return share % 64 == 0 and (self.n_mma == 2 or not self.split_tail or (share // 2) % 64 == 0)
  @property
  def name(self):
    st = self.stages if self.stages is not None else "A"
    sm = self.num_sm if self.num_sm is not None else "dev"
    return (f"ws_c{self.consumers}_s{st}_n{self.BN}_sm{sm}_g{self.group_m}x{self.group_n}"
            f"{'_tmast' if self.tma_store else ''}{'_hil' if self.hilbert else ''}"
            f"{f'_r{self.regs[0]}x{self.regs[1]}' if self.regs else ''}{f'_cl{self.cluster}' if self.cluster > 1 else ''}"
            f"{f'_x{self.n_mma}' if self.n_mma > 1 else ''}{f'_sk{self.split_k}' if self.split_k > 1 else '_skA' if self.split_k == -1 else ''}"
            f"{'' if self.k_serpentine else '_kfwd'}{'' if self.b_nmajor is None else '_bN' if self.b_nmajor else '_bT'}"
            f"{'' if self.wave_sync is None else '_wsync' if self.wave_sync else '_nowsync'}"
            f"{'' if self.split_k_cluster is None else '_skc' if self.split_k_cluster else '_skw'}")

  def to_c(self, kind: int = _capi.KIND_WS, num_sm: int | None = None, wait_budget_ns: int = 0,
           debug_skip_job: int = -1, b_nmajor: bool = False) -> _capi.BgCfg:
    """The C-ABI config. ``b_nmajor`` says how the caller passes B: B[K,N] itself (True) or BT[N,K] (False)."""
    return _capi.BgCfg(kind=kind, BN=self.BN, BK=self.BK, stages=self.stages or 0, consumers=self.consumers,
                       num_sm=num_sm or self.num_sm or 0, group_m=self.group_m, group_n=self.group_n,
                       tma_store=int(self.tma_store), cluster=self.cluster, hilbert=int(self.hilbert),
                       acc_bufs=self.acc_bufs or 0, wait_budget_ns=wait_budget_ns, debug_skip_job=debug_skip_job,
                       n_mma=self.n_mma, no_tail_split=0 if self.split_tail else 1, ragged=int(self.ragged),
                       split_k=self.split_k, no_k_serpentine=0 if self.k_serpentine else 1,
                       b_nmajor=int(b_nmajor), wave_sync={None: 0, True: 1, False: 2}[self.wave_sync],
                       split_k_cluster={None: 0, True: 1, False: 2}[self.split_k_cluster])


# =============================================================================================================
# builder
# =============================================================================================================
def _make_launch(plan: _capi.Plan, stream_of, out, keep):
  def launch(_keep=keep):
    plan.launch(stream_of())
    return out

  def check():
    """Wait for the launch's stream and raise RuntimeError if a device-side wait timed out."""
    plan.check_error(stream_of())
    return out
  launch.check = check
  launch.plan = plan
  launch.info = plan.info
  return launch


def plan_gemm_bt(A, BT, Cout, cfg: WSCfg, *, wait_budget_ns: int = 0, debug_skip_job: int = -1):
  """C[M,N] = A[M,K] @ BT[N,K]^T with B already K-major (no transpose): the entry the column-sharded path uses.
  C may be a column view of a wider matrix (its row pitch is passed to the kernel). Returns ``launch``."""
  a, bt, c = operand(A), operand(BT), operand(Cout)
  M, K = a.shape
  N = bt.shape[0]
  if bt.shape != (N, K) or c.shape != (M, N): raise ValueError("A, BT and C shapes do not match the GEMM")
  if not (a.bf16 and bt.bf16 and c.bf16): raise ValueError("A, B and C must be bfloat16")
  if not (a.device == bt.device == c.device): raise ValueError("A, B and C must be on the same device")
  plan = _capi.Plan(cfg.to_c(_capi.KIND_WS, wait_budget_ns=wait_budget_ns, debug_skip_job=debug_skip_job), M, N, K,
                    a.ptr, a.row_pitch, bt.ptr, bt.row_pitch, c.ptr, c.row_pitch, a.device)
  return _make_launch(plan, lambda: current_stream(Cout), Cout, (A, BT, Cout))


def plan_gemm_b(A, B, Cout, cfg: WSCfg, *, wait_budget_ns: int = 0, debug_skip_job: int = -1):
  """C[M,N] = A[M,K] @ B[K,N] with B read N-major as it is (no copy). B and C may be column views of wider
  matrices (their row pitches are passed to the kernel), so a rank's shard B[:, c0:c1] needs no copy either.
  Each CTA's share of the tile's columns (BN, or BN / 2 in a CTA pair) must be a multiple of 64, or the plan raises
  ValueError; half-width tail tiles are used only when their share is too. Returns ``launch``."""
  a, b, c = operand(A), operand(B), operand(Cout)
  M, K = a.shape
  N = b.shape[1]
  if b.shape != (K, N) or c.shape != (M, N): raise ValueError("A, B and C shapes do not match the GEMM")
  if not (a.bf16 and b.bf16 and c.bf16): raise ValueError("A, B and C must be bfloat16")
  if not (a.device == b.device == c.device): raise ValueError("A, B and C must be on the same device")
  plan = _capi.Plan(cfg.to_c(_capi.KIND_WS, wait_budget_ns=wait_budget_ns, debug_skip_job=debug_skip_job,
                             b_nmajor=True), M, N, K, a.ptr, a.row_pitch, b.ptr, b.row_pitch, c.ptr, c.row_pitch,
                    a.device)
  return _make_launch(plan, lambda: current_stream(Cout), Cout, (A, B, Cout))


def build_gemm_ws(N: int, cfg: WSCfg, M: int | None = None, K: int | None = None, *, wait_budget_ns: int = 0,
                  debug_skip_job: int = -1):
  """C[M,N] = A[M,K] @ B[K,N] (square by default), bf16 in, fp32 accumulate, bf16 out.
  M % BM, N % BN and K % BK must be 0. Returns ``run(A, B, C) -> launch()``; ``launch()`` enqueues the kernel on the
  current stream and returns C; ``launch.check()`` synchronizes and raises if a device wait timed out.
  ``run.kernel_name`` names the configuration; ``run.cuda_kernel`` is the regex Nsight Compute matches.
  ``wait_budget_ns`` / ``debug_skip_job`` are test hooks (per-wait time limit; a job the producer never loads)."""
  M, K = N if M is None else M, N if K is None else K
  if min(M, N, K) <= 0: raise ValueError("M, N and K must be positive")
  BM, BN, BK, CL = cfg.BM, cfg.width, cfg.BK, cfg.cluster
  if cfg.ragged:
    if N % 8 or K % 8: raise ValueError(f"ragged shapes need N and K to be multiples of 8, got N={N} K={K}")
    MT, NT = -(-M // BM), -(-N // BN)
    MT = -(-MT // CL) * CL
  else:
    if M % BM or N % BN or K % BK: raise ValueError(f"shape {M}x{N}x{K} not a multiple of tile {BM}x{BN}x{BK}")
    MT, NT = M // BM, N // BN
  if MT % CL: raise ValueError(f"{MT} row tiles not divisible by cluster {CL}")
  CMT = MT // CL
  _, grouped_2d = grouped_tile_order(CMT, NT, min(max(cfg.group_m // CL, 1), CMT), min(cfg.group_n, NT))
  shp = f"{N}" if M == N == K else f"{M}x{N}x{K}"
  kernel_name = f"sm100_{shp}_{'' if grouped_2d else 'g1d_'}{cfg.name}"
  runtime.set_dynamic_smem_bytes(kernel_name, cfg.smem_bytes)   # as the reference's builder does (gemm.py:316)

  def run(A, B, Cout):
    # the registered size is this kernel's shared-memory budget (a caller may have lowered it since the build)
    budget = runtime.dynamic_smem_bytes(kernel_name)
    plan_cfg = cfg if budget is None else cfg.within_smem(budget)
    a, b, c = operand(A), operand(B), operand(Cout)
    if a.shape != (M, K) or b.shape != (K, N) or c.shape != (M, N): raise ValueError("A, B and C shapes do not match the GEMM")
    if not (a.bf16 and b.bf16 and c.bf16): raise ValueError("A, B and C must be bfloat16")
    if not (a.device == b.device == c.device): raise ValueError("A, B and C must be on the same device")
    if plan_cfg.reads_b_directly:
      # B as given, N-major: no transposed copy (the reference makes one per run, gemm.py:382)
      plan = _capi.Plan(plan_cfg.to_c(_capi.KIND_WS, wait_budget_ns=wait_budget_ns, debug_skip_job=debug_skip_job,
                                 b_nmajor=True), M, N, K, a.ptr, a.row_pitch, b.ptr, b.row_pitch, c.ptr, c.row_pitch,
                        a.device)
      return _make_launch(plan, lambda: current_stream(Cout), Cout, (A, B, Cout))
    BT = transpose_contiguous(B)          # K-major B. Keep it alive: the tensor map holds its raw device pointer
    bt = operand(BT)
    plan = _capi.Plan(plan_cfg.to_c(_capi.KIND_WS, wait_budget_ns=wait_budget_ns, debug_skip_job=debug_skip_job), M, N, K,
                      a.ptr, a.row_pitch, bt.ptr, bt.row_pitch, c.ptr, c.row_pitch, a.device)
    return _make_launch(plan, lambda: current_stream(Cout), Cout, (A, BT, Cout))
  run.out_dtype = "bfloat16"
  run.kernel_name = kernel_name
  run.cuda_kernel = "regex:sm100_gemm_ws"
  run.cfg = cfg
  return run
