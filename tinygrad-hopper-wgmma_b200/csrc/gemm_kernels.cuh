// bf16 GEMM kernels for sm_100a: C[M,N] = A[M,K] * B[K,N], A K-major (row-major), B either K-major (given as
// BT[N,K]) or, for sm100_gemm_ws, N-major (B[K,N] as it is, read through MN-major tcgen05 descriptors), fp32
// accumulation in tensor memory, bf16 output. Shapes are tile multiples unless the host asks for ragged edges
// (TMA zero-fills loads past the operands; stores are clipped or masked).
//
//   sm100_gemm_ws    warp-specialized tcgen05 GEMM. Used for the reference's persistent ladder rungs
//                    (hopper_wgmma/gemm.py:293-398: role_split, tma_store, hilbert, cluster, cluster_hilbert) with
//                    one cluster per SM and a host-built tile table, and for the non-persistent warp-specialized
//                    rung (hopper_wgmma/gated.py:50-123 with consumers >= 1) with one tile per cluster.
//   sm100_gemm_ring  one thread issues both the TMA ring and the MMAs, one tile per CTA: the reference's "ring only"
//                    rung (gated.py with consumers = 0, ladder.py:8).
//
// Warp roles of sm100_gemm_ws (256 threads):
//   warp 0, lane 0   TMA producer: for every (tile, k-block) it waits for a free shared-memory stage, then loads the
//                    A tile (BM x 64) and its B tile (bn_local x 64) with 128-byte swizzle.
//   warp 1           allocates tensor memory; lane 0 issues tcgen05.mma (4 x K16 per stage) into one of two
//                    accumulator buffers and commits stage releases and "accumulator full" events to mbarriers.
//   warps 4-7        epilogue: warp w owns TMEM lane quadrant w % 4 (32 accumulator rows, or 16 for BM = 64),
//                    reads fp32 columns with tcgen05.ld, rounds to bf16 and writes C either directly
//                    (register epilogue) or through a 128B-swizzled staging buffer and a TMA store (per warp,
//                    double-buffered), then frees the accumulator buffer for the next tile.
// With two N blocks per tile and one 512-column accumulator (NB == 2, acc_bufs == 1) the accumulator is split in two
// 256-column halves with their own full/empty barriers: the MMA warp issues the half-0 MMAs of a tile's last k-blocks
// first and publishes half 0, so the epilogue drains it while half 1 finishes, and starts the next tile on half 0
// while the epilogue drains half 1.
// In a CTA pair (PAIRED, cta_group::2) both CTAs load their own A rows and their own half of the B tile; only the
// even CTA issues MMAs (M = 256 across the pair); the odd CTA's loads complete on the even CTA's barriers and the
// MMA commits arrive on both CTAs' barriers. No load is multicast.
// A persistent cluster walks K forwards on its even-numbered tiles and backwards on its odd-numbered ones (K
// serpentine). SPLITK selects split-K: with kSplitWorkspace the tile table may hold several entries per tile over
// disjoint K ranges, whose fp32 partial sums the epilogue warps combine through a global workspace; with
// kSplitCluster the CTAs of one cluster are the splits of one tile and combine their sums through distributed shared
// memory (see the split-K block of the epilogue).
//
// Every mbarrier wait is bounded (GemmParams::budget_ns). On expiry a thread writes a code into GemmParams::err and
// leaves its loop; all other roles then run out of work or time out too, the kernel drains what it issued, frees
// its tensor memory and returns, and the host turns the code into an error.
#pragma once
#include "ptx.cuh"

namespace sm100 {

constexpr int kBK = 64;           // K per pipeline stage: one 128-byte swizzle row of bf16
constexpr int kWsThreads = 256;   // warps 0-3 producer / MMA / idle, warps 4-7 epilogue
constexpr int kRingThreads = 128;
constexpr int kFirstWave = 160;   // first-wave tile entries passed in the kernel parameters (>= clusters on a B200)
constexpr int kSkSlots = 8;
constexpr int kSplitNone = 0, kSplitWorkspace = 1, kSplitCluster = 2;   // the kernel's SPLITK parameter
constexpr uint32_t kNmajorChunk = 64 * 128;   // one N-major B box in shared memory: 64 K rows x 64 columns of bf16       // split-K reduce: 4 KB shared-memory slots per epilogue warp (in the idle ring)

// Error word layout: role in bits 24-31, the role's job or tile counter (saturated) in bits 0-23.
enum : uint32_t {
  kErrProducer = 1u << 24,    // producer timed out waiting for a free stage
  kErrMmaFull = 2u << 24,     // MMA issuer timed out waiting for a loaded stage
  kErrMmaAcc = 3u << 24,      // MMA issuer timed out waiting for a free accumulator buffer
  kErrEpilogue = 4u << 24,    // epilogue timed out waiting for a finished accumulator
  kErrDrain = 5u << 24,       // final wait for outstanding MMAs timed out
  kErrLoadDrain = 6u << 24,   // producer's final wait for its in-flight loads timed out (after another error)
  kErrSplitK = 7u << 24,      // split-K (one wave): the other entries of a tile did not all publish in time
};

struct GemmParams {
  int num_kb;              // K / 64
  int bn;                  // MMA N: columns per tcgen05.mma (the whole pair's when PAIRED)
  int nblk;                // MMAs along N per K step: a tile is nblk * bn columns wide (1 or 2)
  int bn_local;            // rows of BT this CTA loads per N block and stage (bn / 2 when PAIRED)
  int stages;              // shared-memory ring depth
  int tiles;               // schedule entries (cluster tiles)
  int nclusters;           // clusters (persistent workers) in the grid
  int cl;                  // CTAs per cluster (1 or 2)
  int nt;                  // column tiles; used when sched == nullptr (row-major tile order)
  int acc_bufs;            // accumulator buffers in tensor memory (1 or 2)
  int acc_stride;          // TMEM columns between accumulator buffers
  uint32_t tmem_cols;      // TMEM columns allocated (power of two >= 32)
  uint32_t idesc;          // tcgen05 instruction descriptor (bf16 x bf16 -> f32, K-major, M, N)
  uint32_t tx_bytes;       // bytes that complete one stage's FULL barrier (both CTAs' loads when PAIRED)
  uint32_t tx_narrow;      // the same for a half-width tile
  uint32_t idesc_narrow;   // instruction descriptor of a half-width tile (N = bn / 2) when nblk == 1
  uint32_t a_stage_bytes;  // BM * 128
  uint32_t b_block_bytes;  // bn_local * 128: one N block of B in a stage
  uint32_t b_stage_bytes;  // nblk * b_block_bytes
  const int32_t* sched;    // [tiles] entries (cluster row tile << 16) | column tile; entry i runs on cluster
                           // i % nclusters as that cluster's (i / nclusters)-th tile. kNarrowTile in the column
                           // field marks a half-width tile whose column index counts half-width tiles
  __nv_bfloat16* C;        // output base (register epilogue)
  long long ldc;           // C row pitch in elements
  int m_valid;             // rows of C (the register epilogue masks rows >= m_valid; the TMA store clips them)
  int n_valid;             // columns of C (a multiple of 8; the same for columns)
  unsigned int* err;       // error word (0 = ok)
  unsigned long long budget_ns;  // per-wait time limit
  int look;                // split accumulator: k-blocks of the half-0-first phases at tile start and end (< stages)
  int skip_job;            // test hook: the producer never loads this job index (-1 = off); makes waits run out
  int split_k;             // K splits per output tile (1 = off): entry i computes split i % split_k of tile
                           // i / split_k, k-blocks [s * num_kb / split_k, (s + 1) * num_kb / split_k)
  float* partial;          // split-K: fp32 partial sums, one 32-lane x width slice per (entry, CTA of the pair, warp)
  unsigned int* tickets;   // split-K: one arrival word per (tile, CTA of the pair, warp), counting entries whose
                           // partial sums are written; zero between launches
  int sk_scatter;          // split-K with one entry per cluster, launched cooperatively: the reduce is shared out
  int k_serpentine;        // a cluster walks K backwards on its odd-numbered tiles (1) or always forwards (0)
  int b_nmajor;            // B is given as B[K,N] row-major (1; tmB/tmBn map it with 64 x 64 boxes) or as BT[N,K] (0)
  int wave_sync;           // 1: the producers of all CTAs meet at every tile boundary (see wave_barrier)
  unsigned long long* wave_ctr;   // wave barrier: arrivals, counted across launches (the plan's counter)
  unsigned long long wave_base;   // wave barrier: the counter's value when this launch starts
  unsigned long long wave_wait_ns;  // wave barrier: longest wait at one boundary before the CTA stops waiting
  int kc;                  // split-K inside a cluster (1 = off): the kc CTAs of a cluster run splits 0..kc-1 (their
                           // cluster rank) of the cluster's one tile and reduce through distributed shared memory
  uint32_t kc_recv_bytes;  // split-K inside a cluster: bytes each CTA receives from the others (its receive region)
  int32_t first_wave[kFirstWave];  // sched[0 .. min(tiles, kFirstWave)) again, delivered with the launch
};

// K range of schedule entry idx: k-blocks [kb0, kb0 + nk). Kernels built without split-K (kSplitNone) ignore
// p.split_k; the host never hands them a split schedule. Split-K inside a cluster runs split `ks` (the CTA's cluster
// rank) of every entry; through the workspace, entry idx is split idx % split_k of its tile.
template <int SPLITK>
__device__ __forceinline__ void k_range(const GemmParams& p, int idx, int ks, int& kb0, int& nk) {
  if (SPLITK != kSplitNone && p.split_k > 1) {
    const int s = SPLITK == kSplitCluster ? ks : idx % p.split_k;
    kb0 = s * p.num_kb / p.split_k;
    nk = (s + 1) * p.num_kb / p.split_k - kb0;
  } else {
    kb0 = 0;
    nk = p.num_kb;
  }
}

__device__ __forceinline__ void record_error(unsigned int* err, uint32_t role, uint32_t counter) {
  atomicCAS(err, 0u, role | (counter > 0xFFFFFFu ? 0xFFFFFFu : counter));
}

// Wave barrier (p.wave_sync): before loading its i-th tile (i >= 1), each CTA's producer counts itself on a
// GPU-wide counter and waits until every CTA that has an i-th tile has done the same. Without it, CTAs drift apart
// over many tiles (a few percent of speed accumulates to whole tiles), so the tiles of one wave that share an A or B
// panel no longer read its K-slabs at about the same time, and L2 no longer serves the later readers: at 32768^3 on
// one GPU (110 tiles per cluster) DRAM read 51x the compulsory bytes. The barrier keeps a wave's tiles within the
// last tile's spread of each other. It publishes no data (relaxed counting), so it is soft: a CTA that has waited
// p.wave_wait_ns at one boundary (the launch's CTAs are not all resident, e.g. beside another launch on the GPU)
// stops waiting for the rest of the launch (`waiting` turns false) but keeps counting its arrivals, so that the next
// launch's base stays right. The counter counts across launches: launch L starts at p.wave_base = L x (arrivals per
// launch), set by the host.
__device__ __forceinline__ void wave_barrier(const GemmParams& p, int i, int lane, bool& waiting) {
  if (lane == 0) {
    // arrivals at boundaries 1..i: every CTA of each cluster that has a j-th tile
    unsigned long long target = p.wave_base;
    for (int j = 1; j <= i; ++j) {
      const int left = p.tiles - j * p.nclusters;
      target += static_cast<unsigned long long>(left < p.nclusters ? left : p.nclusters) * p.cl;
    }
    atomicAdd(p.wave_ctr, 1ull);
    if (waiting && ld_relaxed_gpu_u64(p.wave_ctr) < target) {
      const uint64_t t0 = globaltimer_ns();
      while (ld_relaxed_gpu_u64(p.wave_ctr) < target) {
        if (globaltimer_ns() - t0 > p.wave_wait_ns) {
          waiting = false;
          break;
        }
        __nanosleep(64);
      }
    }
  }
  waiting = __shfl_sync(0xffffffffu, waiting ? 1u : 0u, 0) != 0;
}

constexpr int kNarrowTile = 0x8000;   // column-field flag of a half-width tile (the last wave's split tiles)

__device__ __forceinline__ void tile_coords(const GemmParams& p, int idx, int& cm, int& tn, bool& narrow) {
  if (p.sched != nullptr) {
    const int e = __ldg(p.sched + idx);
    cm = e >> 16;
    tn = e & 0x7FFF;
    narrow = (e & kNarrowTile) != 0;
  } else {
    cm = idx / p.nt;
    tn = idx - cm * p.nt;
    narrow = false;
  }
}

__device__ __forceinline__ void tile_coords(const GemmParams& p, int idx, int& cm, int& tn) {
  bool narrow;
  tile_coords(p, idx, cm, tn, narrow);
}

// The first tile of a persistent cluster comes from the kernel parameters (a copy of the table's first wave), so the
// first TMA load does not wait for a cold global-memory read of the tile table (about 1 us per launch, which matters
// for microsecond-scale problems).
struct FirstTile {
  int idx = -1;
  int entry = 0;
  __device__ __forceinline__ void load(const GemmParams& p, int cid) {
    if (p.sched != nullptr && cid < p.tiles && cid < kFirstWave) {
      idx = cid;
      entry = p.first_wave[cid];   // kernel-parameter space: no global-memory round trip before the first TMA
    }
  }
  __device__ __forceinline__ void coords(const GemmParams& p, int i, int& cm, int& tn, bool& narrow) const {
    if (i == idx) {
      cm = entry >> 16;
      tn = entry & 0x7FFF;
      narrow = (entry & kNarrowTile) != 0;
    } else {
      tile_coords(p, i, cm, tn, narrow);
    }
  }
};

// Round 2N fp32 accumulator words to bf16 and store N/2 packed words per 16-byte chunk.
template <int N>
__device__ __forceinline__ void store_row_global(__nv_bfloat16* dst, const uint32_t (&v)[N]) {
#pragma unroll
  for (int j = 0; j < N / 8; ++j)
    st_global_v4(dst + 8 * j, pack_bf16x2(v[8 * j + 0], v[8 * j + 1]), pack_bf16x2(v[8 * j + 2], v[8 * j + 3]),
                 pack_bf16x2(v[8 * j + 4], v[8 * j + 5]), pack_bf16x2(v[8 * j + 6], v[8 * j + 7]));
}

// Store the first `cols` (a multiple of 8) of N accumulator words as bf16; for tiles that overhang C's last column.
template <int N>
__device__ __forceinline__ void store_row_global_masked(__nv_bfloat16* dst, const uint32_t (&v)[N], int cols) {
#pragma unroll
  for (int j = 0; j < N / 8; ++j)
    if (8 * j < cols)
      st_global_v4(dst + 8 * j, pack_bf16x2(v[8 * j + 0], v[8 * j + 1]), pack_bf16x2(v[8 * j + 2], v[8 * j + 3]),
                   pack_bf16x2(v[8 * j + 4], v[8 * j + 5]), pack_bf16x2(v[8 * j + 6], v[8 * j + 7]));
}

// Register epilogue for one accumulator: this thread's row, columns [0, bn), 32 at a time plus a 16-column tail.
// Only the first `cols` columns exist in C (cols >= bn for an interior tile); TMEM reads stay warp-uniform.
__device__ __forceinline__ void epilogue_registers(uint32_t tacc, __nv_bfloat16* crow, int bn, bool active,
                                                   int cols) {
  const int n32 = bn >> 5;
#pragma unroll 1
  for (int c = 0; c < n32; ++c) {
    uint32_t v[32];
    tmem_ld_32x32b_x32(tacc + 32 * c, v);
    tmem_ld_wait();
    if (active) {
      if (cols >= 32 * c + 32) store_row_global<32>(crow + 32 * c, v);
      else if (cols > 32 * c) store_row_global_masked<32>(crow + 32 * c, v, cols - 32 * c);
    }
  }
  if (bn & 16) {
    uint32_t v[16];
    tmem_ld_32x32b_x16(tacc + 32 * n32, v);
    tmem_ld_wait();
    if (active && cols > 32 * n32) store_row_global_masked<16>(crow + 32 * n32, v, cols - 32 * n32);
  }
}

template <int BM, bool PAIRED, bool TMA_STORE, int NB, int SPLITK>
__global__ void __launch_bounds__(kWsThreads, 1)
    sm100_gemm_ws(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                  const __grid_constant__ CUtensorMap tmBn, const __grid_constant__ CUtensorMap tmC,
                  const __grid_constant__ GemmParams p) {
  static_assert(BM == 64 || BM == 128, "BM is 64 or 128 rows per CTA");
  static_assert(!PAIRED || BM == 128, "CTA pairs use M = 256 (128 rows per CTA)");
  static_assert(SPLITK != kSplitCluster || (!PAIRED && NB == 1), "split-K inside a cluster: single-CTA, one N block");
  constexpr int CG = PAIRED ? 2 : 1;
  constexpr int ROWS_W = BM / 4;                  // accumulator rows per epilogue warp
  constexpr uint32_t STAGE_C = ROWS_W * 128;      // one 64-column bf16 staging buffer of one warp
  extern __shared__ __align__(1024) uint8_t smem_raw[];

  const uint32_t raw = smem_u32(smem_raw);
  const uint32_t base = (raw + 1023u) & ~1023u;   // 128B-swizzled tiles need 1024-byte alignment
  const uint32_t sA = base;
  const uint32_t sB = sA + p.stages * p.a_stage_bytes;
  const uint32_t sC = sB + p.stages * p.b_stage_bytes;
  const uint32_t sR = sC + (TMA_STORE ? 4u * 2u * STAGE_C : 0u);   // split-K inside a cluster: receive region
  const uint32_t bars = sR + (SPLITK == kSplitCluster ? p.kc_recv_bytes : 0u);
  const uint32_t full0 = bars;
  const uint32_t empty0 = bars + 8u * p.stages;
  const uint32_t tfull0 = bars + 16u * p.stages;
  const uint32_t tempty0 = tfull0 + 16u;
  const uint32_t drain = tempty0 + 16u;
  const uint32_t tslot = drain + 8u;
  const uint32_t recvbar = tslot + 8u;   // split-K inside a cluster: the other splits' sums of this CTA's chunks
  volatile uint32_t* tslot_ptr = reinterpret_cast<volatile uint32_t*>(smem_raw + (tslot - raw));

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  // Launched clusters are CTA pairs (PAIRED: rank = the pair's row half) or, for split-K inside a cluster, the kc
  // splits of one tile (ks = the CTA's split; the host never combines the two).
  constexpr bool kcl = SPLITK == kSplitCluster;
  const int ccl = kcl ? p.kc : p.cl;
  const uint32_t crank = ccl > 1 ? cluster_ctarank() : 0u;
  const uint32_t rank = kcl ? 0u : crank;
  const int ks = static_cast<int>(crank);
  const int cid = static_cast<int>(blockIdx.x) / ccl;
  const bool leader = !PAIRED || rank == 0;
  bool kc_waiting = false;   // an epilogue warp whose wait for the other splits' sums timed out (see teardown)
  const uint64_t budget = p.budget_ns;
  FirstTile first;
  first.load(p, cid);

  if (threadIdx.x == 0) {
    for (int s = 0; s < p.stages; ++s) {
      mbar_init(full0 + 8u * s, 1);
      mbar_init(empty0 + 8u * s, 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(tfull0 + 8u * b, 1);
      mbar_init(tempty0 + 8u * b, 4 * CG);   // one arrival per epilogue warp of each CTA of the pair
    }
    mbar_init(drain, 1);
    if (kcl) mbar_init(recvbar, 1);
    fence_mbar_init();
    // the receive barrier's only arrival, with every byte the other splits will send (they may land first: the
    // phase cannot complete before this arrival)
    if (kcl) mbar_arrive_expect_tx(recvbar, p.kc_recv_bytes);
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_map(&tmA);
    tma_prefetch_map(&tmB);
    if (NB == 1) tma_prefetch_map(&tmBn);
    if (TMA_STORE) tma_prefetch_map(&tmC);
  }
  if (warp == 1) {
    tmem_alloc<CG>(tslot, p.tmem_cols);
    tmem_relinquish<CG>();
  }
  tc_fence_before();
  __syncthreads();
  if (PAIRED || kcl) cluster_sync_all();   // the peers' barriers and TMEM exist before anyone signals them
  tc_fence_after();
  const uint32_t tmem_base = *tslot_ptr;

  if (warp == 0) {
    // ------------------------------------------------------------------ TMA producer (one elected lane issues)
    uint32_t stage = 0, phase = 0;
    int job = 0;
    bool failed = false;
    bool wave_waiting = true;   // the wave barrier still waits (see wave_barrier)
    for (int i = 0; !failed; ++i) {
      const int idx = cid + i * p.nclusters;
      if (idx >= p.tiles) break;
      if (p.wave_sync && i > 0) wave_barrier(p, i, lane, wave_waiting);
      int cm, tn;
      bool narrow;
      first.coords(p, idx, cm, tn, narrow);
      // A half-width tile keeps NB == 2's MMA N and drops the second N block, or halves NB == 1's MMA N
      const int nblk = (narrow && NB == 2) ? 1 : NB;
      const CUtensorMap* mapB = (narrow && NB == 1) ? &tmBn : &tmB;
      const int bsub = (narrow && NB == 1) ? p.bn / 2 : p.bn;            // B rows of one N block (pair level)
      const int width = narrow ? p.bn * NB / 2 : p.bn * NB;
      const uint32_t tx = narrow ? p.tx_narrow : p.tx_bytes;
      const int row_a = (cm * p.cl + static_cast<int>(rank)) * BM;
      const int row_b = tn * width + (PAIRED ? static_cast<int>(rank) * (bsub / 2) : 0);
      int kb0, nk;
      k_range<SPLITK>(p, idx, ks, kb0, nk);
      // K serpentine: consecutive tiles of a cluster walk K in opposite directions, so a wave of tiles starts on
      // the K-slabs the previous wave read last, which are still in L2 (fewer DRAM reads, less power under the
      // cap). The MMA side counts k-blocks from the first one issued, whichever the direction.
      const bool reverse = p.k_serpentine != 0 && (i & 1) != 0;
      for (int kb = kb0; kb < kb0 + nk; ++kb, ++job) {
        const int kc = reverse ? 2 * kb0 + nk - 1 - kb : kb;   // the k-block this job loads
        if (!mbar_wait_warp(empty0 + 8u * stage, phase ^ 1u, budget)) {
          if (lane == 0) record_error(p.err, kErrProducer, job);
          failed = true;
          break;
        }
        if (job != p.skip_job && elect_one()) {
          const uint32_t fb = full0 + 8u * stage;
          const uint32_t a_dst = sA + stage * p.a_stage_bytes;
          const uint32_t b_dst = sB + stage * p.b_stage_bytes;
          // N-major B: this CTA's columns of an N block arrive as 64-column x 64-row boxes, 8 KB apart (the MMA's
          // leading byte offset); K-major B: one box of bn_local (or half that) rows of BT
          const int chunks = p.b_nmajor ? (bsub / CG) >> 6 : 0;
          if (PAIRED) {
            const uint32_t fb_leader = mapa_shared(fb, 0);
            if (leader) mbar_arrive_expect_tx(fb, tx);
            tma_load_2d_pair(a_dst, &tmA, fb_leader, kc * kBK, row_a);
#pragma unroll
            for (int nb = 0; nb < NB; ++nb) {
              if (nb >= nblk) continue;
              if (p.b_nmajor) {
                for (int j = 0; j < chunks; ++j)
                  tma_load_2d_pair(b_dst + nb * p.b_block_bytes + j * kNmajorChunk, mapB, fb_leader,
                                   row_b + nb * bsub + 64 * j, kc * kBK);
              } else {
                tma_load_2d_pair(b_dst + nb * p.b_block_bytes, mapB, fb_leader, kc * kBK, row_b + nb * bsub);
              }
            }
          } else {
            mbar_arrive_expect_tx(fb, tx);
            tma_load_2d(a_dst, &tmA, fb, kc * kBK, row_a);
#pragma unroll
            for (int nb = 0; nb < NB; ++nb) {
              if (nb >= nblk) continue;
              if (p.b_nmajor) {
                for (int j = 0; j < chunks; ++j)
                  tma_load_2d(b_dst + nb * p.b_block_bytes + j * kNmajorChunk, mapB, fb, row_b + nb * bsub + 64 * j,
                              kc * kBK);
              } else {
                tma_load_2d(b_dst + nb * p.b_block_bytes, mapB, fb, kc * kBK, row_b + nb * bsub);
              }
            }
          }
        }
        __syncwarp();
        if (++stage == static_cast<uint32_t>(p.stages)) {
          stage = 0;
          phase ^= 1u;
        }
      }
    }
    if (leader) {
      // Let the loads already issued land before shared memory goes away: the newest job of every stage. On the
      // normal path the MMA has consumed them all and these waits return at once; after an error elsewhere they
      // keep the CTA alive until its own copies have arrived. (A pair's FULL barriers live in the even CTA and
      // count both CTAs' bytes; the odd CTA leaves only after the cluster barrier below.)
      const int first = job - p.stages < 0 ? 0 : job - p.stages;
      for (int j = first; j < job; ++j) {
        if (j == p.skip_job) continue;
        const uint32_t s = static_cast<uint32_t>(j % p.stages), ph = static_cast<uint32_t>((j / p.stages) & 1);
        if (!mbar_wait_warp(full0 + 8u * s, ph, budget) && lane == 0) record_error(p.err, kErrLoadDrain, j);
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    // ------------------------------------------------------------------ MMA issuer (whole warp, one elected lane)
    if (leader) {
      uint32_t stage = 0, phase = 0, acc = 0, acc_phase = 0;
      int job = 0;
      bool failed = false;
      // Two N blocks sharing one 512-column accumulator ("split" mode): each half of TMEM has its own full/empty
      // barrier pair (the two pairs that otherwise serve two accumulator buffers), so the epilogue drains half 0
      // while the MMAs of half 1 still run, and the next tile starts on half 0 while the epilogue drains half 1.
      const bool split = NB == 2 && p.acc_bufs == 1;
      auto adv = [&](uint32_t& st, uint32_t& ph) {
        if (++st == static_cast<uint32_t>(p.stages)) {
          st = 0;
          ph ^= 1u;
        }
      };
      // B's K16 step in descriptor address units: +32 bytes inside a K-major swizzle row, or +16 rows of 128 bytes
      // (2048 bytes) for N-major B; the N-major descriptor's leading byte offset is the 8 KB between 64-column boxes
      const uint32_t b_kstep = p.b_nmajor ? 128u : 2u;
      const uint32_t b_lbo = p.b_nmajor ? (kNmajorChunk >> 4) : 1u;
      auto issue = [&](uint32_t st, int kb, int nb_lo, int nb_hi, uint32_t d, uint32_t idesc) {
        if (elect_one()) {
          const uint64_t ad = smem_desc_sw128(sA + st * p.a_stage_bytes);
          const uint64_t bd = smem_desc_sw128(sB + st * p.b_stage_bytes, b_lbo);
          // A: +32 bytes along K inside the swizzle row = +2 in the descriptor's address field; N block nb reads the
          // nb-th B sub-tile and accumulates into TMEM columns [nb * bn, (nb + 1) * bn)
#pragma unroll
          for (int k = 0; k < kBK / 16; ++k)
#pragma unroll
            for (int nb = 0; nb < NB; ++nb)
              if (nb >= nb_lo && nb < nb_hi)
                mma_bf16<CG>(d + static_cast<uint32_t>(nb * p.bn), ad + 2u * k,
                             bd + static_cast<uint64_t>((nb * p.b_block_bytes) >> 4) + b_kstep * k, idesc,
                             (kb | k) != 0 ? 1u : 0u);
        }
        __syncwarp();
      };
      auto commit_both = [&](uint32_t bar) {   // arrive on this CTA's barrier and, in a pair, on the peer's
        if (elect_one()) {
          mma_commit<CG>(bar);
          if (PAIRED) mma_commit<CG>(mapa_shared(bar, 1));
        }
        __syncwarp();
      };
      auto wait_full = [&](uint32_t st, uint32_t ph, int j) {
        if (!mbar_wait_warp(full0 + 8u * st, ph, budget)) {
          if (lane == 0) record_error(p.err, kErrMmaFull, j);
          return false;
        }
        tc_fence_after();
        return true;
      };
      auto wait_acc = [&](uint32_t bar, uint32_t parity, int i) {
        if (!mbar_wait_warp(bar, parity, budget)) {
          if (lane == 0) record_error(p.err, kErrMmaAcc, i);
          return false;
        }
        tc_fence_after();
        return true;
      };
      for (int i = 0; !failed; ++i) {
        const int idx = cid + i * p.nclusters;
        if (idx >= p.tiles) break;
        int cm, tn;
        bool narrow;
        first.coords(p, idx, cm, tn, narrow);
        const int nblk = (narrow && NB == 2) ? 1 : NB;
        const uint32_t idesc = (narrow && NB == 1) ? p.idesc_narrow : p.idesc;
        int kb0, nk;   // the MMAs count k-blocks from 0 within the entry's K range: the first one overwrites D
        k_range<SPLITK>(p, idx, ks, kb0, nk);
        if (!split) {
          if (!wait_acc(tempty0 + 8u * acc, acc_phase ^ 1u, i)) break;
          const uint32_t d = tmem_base + acc * static_cast<uint32_t>(p.acc_stride);
          for (int kb = 0; kb < nk; ++kb, ++job) {
            if (!wait_full(stage, phase, job)) {
              failed = true;
              break;
            }
            issue(stage, kb, 0, nblk, d, idesc);
            commit_both(empty0 + 8u * stage);
            adv(stage, phase);
          }
          if (failed) break;
          commit_both(tfull0 + 8u * acc);
          if (++acc == static_cast<uint32_t>(p.acc_bufs)) {
            acc = 0;
            acc_phase ^= 1u;
          }
          continue;
        }
        // split mode: tile i uses TMEM half h through tfull0/tempty0 + 8h, parity acc_phase (flips per tile)
        const uint32_t d = tmem_base;
        if (nblk == 1) {
          // a half-width tail tile: half 0 only, streamed like the unsplit path; half 1's barriers still take one
          // phase per tile so that both sides stay in step
          if (!wait_acc(tempty0, acc_phase ^ 1u, i)) break;
          for (int kb = 0; kb < nk; ++kb, ++job) {
            if (!wait_full(stage, phase, job)) {
              failed = true;
              break;
            }
            issue(stage, kb, 0, 1, d, idesc);
            commit_both(empty0 + 8u * stage);
            adv(stage, phase);
          }
          if (failed) break;
          commit_both(tfull0);
          if (!wait_acc(tempty0 + 8u, acc_phase ^ 1u, i)) break;
          commit_both(tfull0 + 8u);
          acc_phase ^= 1u;
          continue;
        }
        const int la = nk < p.look ? nk : p.look;                 // phase A k-blocks [0, la)
        const int lc = (nk - la) < p.look ? nk - la : p.look;     // phase C k-blocks [nk - lc, nk)
        // phase A: half 0 of k-blocks [0, la) as soon as half 0 is free (holding those la < stages stages), then
        // half 1 of the same k-blocks once half 1 is free, releasing each stage
        if (!wait_acc(tempty0, acc_phase ^ 1u, i)) break;
        uint32_t st = stage, ph = phase;
        for (int kb = 0; kb < la; ++kb) {
          if (!wait_full(st, ph, job + kb)) {
            failed = true;
            break;
          }
          issue(st, kb, 0, 1, d, idesc);
          adv(st, ph);
        }
        if (failed) break;
        if (la == nk) commit_both(tfull0);   // the whole tile was phase A: half 0 is complete
        if (!wait_acc(tempty0 + 8u, acc_phase ^ 1u, i)) break;
        st = stage;
        ph = phase;
        for (int kb = 0; kb < la; ++kb) {
          issue(st, kb, 1, 2, d, idesc);
          commit_both(empty0 + 8u * st);
          adv(st, ph);
        }
        if (la < nk) {
          // phase B: both halves per k-block
          for (int kb = la; kb < nk - lc; ++kb) {
            if (!wait_full(st, ph, job + kb)) {
              failed = true;
              break;
            }
            issue(st, kb, 0, 2, d, idesc);
            commit_both(empty0 + 8u * st);
            adv(st, ph);
          }
          if (failed) break;
          // phase C: half 0 of the last lc k-blocks (holding lc < stages stages), publish half 0, then half 1
          const uint32_t st_c = st, ph_c = ph;
          for (int kb = nk - lc; kb < nk; ++kb) {
            if (!wait_full(st, ph, job + kb)) {
              failed = true;
              break;
            }
            issue(st, kb, 0, 1, d, idesc);
            adv(st, ph);
          }
          if (failed) break;
          commit_both(tfull0);
          st = st_c;
          ph = ph_c;
          for (int kb = nk - lc; kb < nk; ++kb) {
            issue(st, kb, 1, 2, d, idesc);
            commit_both(empty0 + 8u * st);
            adv(st, ph);
          }
        }
        commit_both(tfull0 + 8u);
        stage = st;
        phase = ph;
        job += nk;
        acc_phase ^= 1u;
      }
      if (elect_one()) mma_commit<CG>(drain);   // every MMA issued above has finished once this arrives
      __syncwarp();
      if (!mbar_wait_warp(drain, 0, budget) && lane == 0) record_error(p.err, kErrDrain, 0);
    }
    __syncwarp();
  } else if (warp >= 4) {
    // ------------------------------------------------------------------ epilogue
    const int q = warp & 3;   // TMEM lane quadrant this warp may access
    const uint32_t lane_base = static_cast<uint32_t>(q * 32) << 16;
    const uint32_t my_stage = sC + static_cast<uint32_t>(q) * 2u * STAGE_C;
    const bool split = NB == 2 && p.acc_bufs == 1;
    uint32_t acc = 0, acc_phase = 0, chunk = 0;
    // Free an accumulator buffer for the MMA warp once this warp's tensor-memory reads of it have completed. The
    // arrive is relaxed: it hands back tensor memory and publishes no memory writes (C goes out through TMA stores
    // or plain stores that no one in the kernel reads). A release arrive here stalled each epilogue warp about 3000
    // cycles per 256-column half, which the MMA warp of a 256x512 pair tile waited out at every tile boundary. The
    // cluster's last entry skips the arrive: no MMA waits for that buffer again, and in a pair the remote arrive
    // would only delay the teardown (tensor memory is freed after the final CTA barrier, which also orders the last
    // TMEM reads).
    bool last_entry = false;
    auto release = [&](uint32_t bar) {
      if (last_entry) return;
      tc_fence_before();
      __syncwarp();
      if (lane == 0) {
        if (PAIRED)
          mbar_arrive_cluster_relaxed(mapa_shared(bar, 0));
        else
          mbar_arrive_local_relaxed(bar);
      }
    };
    // Write accumulator columns starting at TMEM address tacc (this warp's lanes) to C rows row0.., columns
    // [ccol, ccol + ncols), and release accumulator barrier rel_bar (0 = none) as soon as the last columns are in
    // registers, before their stores.
    auto drain = [&](uint32_t tacc, int row0, int ccol, int ncols, uint32_t rel_bar) {
      if constexpr (TMA_STORE) {
        const int nchunks = ncols >> 6;
#pragma unroll 1
        for (int c = 0; c < nchunks; ++c, ++chunk) {
          uint32_t v0[32], v1[32];
          tmem_ld_32x32b_x32(tacc + 64u * c, v0);
          tmem_ld_32x32b_x32(tacc + 64u * c + 32u, v1);
          tmem_ld_wait();
          if (!SPLITK && c + 1 == nchunks && rel_bar != 0u) release(rel_bar);
          const uint32_t buf = my_stage + (chunk & 1u) * STAGE_C;
          if (lane == 0) bulk_wait_group_read<1>();   // the store issued from this buffer two chunks ago has read it
          __syncwarp();
          if (lane < ROWS_W) {
            // row `lane` of the staging tile: 16-byte chunk j holds columns 8j..8j+7, stored at chunk j ^ (row % 8)
            const uint32_t rowaddr = buf + static_cast<uint32_t>(lane) * 128u;
            const uint32_t sw = static_cast<uint32_t>(lane) & 7u;
#pragma unroll
            for (int j = 0; j < 4; ++j)
              st_shared_v4(rowaddr + ((static_cast<uint32_t>(j) ^ sw) << 4), pack_bf16x2(v0[8 * j], v0[8 * j + 1]),
                           pack_bf16x2(v0[8 * j + 2], v0[8 * j + 3]), pack_bf16x2(v0[8 * j + 4], v0[8 * j + 5]),
                           pack_bf16x2(v0[8 * j + 6], v0[8 * j + 7]));
#pragma unroll
            for (int j = 0; j < 4; ++j)
              st_shared_v4(rowaddr + ((static_cast<uint32_t>(j + 4) ^ sw) << 4), pack_bf16x2(v1[8 * j], v1[8 * j + 1]),
                           pack_bf16x2(v1[8 * j + 2], v1[8 * j + 3]), pack_bf16x2(v1[8 * j + 4], v1[8 * j + 5]),
                           pack_bf16x2(v1[8 * j + 6], v1[8 * j + 7]));
          }
          fence_proxy_async_smem();
          __syncwarp();
          if (lane == 0) {
            tma_store_2d(&tmC, buf, ccol + 64 * c, row0);
            bulk_commit_group();
          }
        }
        if (SPLITK && rel_bar != 0u) release(rel_bar);   // (after the loop: no registers to spare in these kernels)
      } else {
        __nv_bfloat16* crow = p.C + static_cast<long long>(row0 + lane) * p.ldc + ccol;
        epilogue_registers(tacc, crow, ncols, lane < ROWS_W && row0 + lane < p.m_valid, p.n_valid - ccol);
        if (rel_bar != 0u) release(rel_bar);
      }
    };
    // Split-K (p.split_k > 1). The split_k entries of a tile run on different clusters, each into its own
    // accumulator, and meet through a workspace of fp32 slices (one per entry, CTA of the pair and warp; 32 lanes x
    // width columns, float4 g = column / 4 of lane l at (g * 32 + l) * 4) and one arrival word per (tile, CTA, warp).
    // The sum over the splits is always taken in split order 0, 1, ..., split_k - 1 (an entry's own values from its
    // tensor memory, in their place), so the rounding does not depend on the order in which the entries finish.
    //   * one wave (p.sk_scatter: every entry on its own cluster, all resident at once under a cooperative launch):
    //     the tile's 32-column chunks are shared out among its entries. Each entry publishes the chunks the others
    //     reduce, counts itself, waits (bounded) until all split_k entries have counted, then reduces its own chunks
    //     and stores them to C; a second count lets the last entry through reset the word.
    //   * otherwise: every entry publishes all its chunks and counts itself; the entry that sees the count reach
    //     split_k - 1 is the last, reduces the whole tile into its tensor memory, drains it as usual and resets the
    //     word. No entry waits for another.
    const size_t sk_slice = 32u * static_cast<size_t>(p.bn * NB);                 // floats per slice
    const size_t sk_stride = static_cast<size_t>(p.cl) * 4u * sk_slice;           // between consecutive splits
    int sk_own = 0;                    // this entry's split
    unsigned int* sk_word = nullptr;   // the tile's arrival word for this warp
    float* sk_src = nullptr;           // this warp's slice of split 0 of the tile
    auto sk_setup = [&](int idx) {
      const int tile = idx / p.split_k;
      sk_own = idx - tile * p.split_k;
      sk_word = p.tickets + (static_cast<size_t>(tile) * p.cl + rank) * 4u + static_cast<size_t>(q);
      sk_src = p.partial + ((static_cast<size_t>(tile) * p.split_k * p.cl + rank) * 4u + q) * sk_slice;
    };
    // Publish accumulator chunks [0, nch) except [skip_lo, skip_hi) (chunk c = 32 columns at TMEM tacc + 32 c).
    auto sk_publish = [&](uint32_t tacc, int nch, int skip_lo, int skip_hi) {
      float* d = sk_src + static_cast<size_t>(sk_own) * sk_stride + static_cast<size_t>(lane) * 4u;
#pragma unroll 1
      for (int c = 0; c < nch; ++c) {
        if (c >= skip_lo && c < skip_hi) continue;
        uint32_t v[32];
        tmem_ld_32x32b_x32(tacc + 32u * c, v);
        tmem_ld_wait();
#pragma unroll
        for (int i = 0; i < 8; ++i) st_global_v4(d + (8 * c + i) * 128, v[4 * i], v[4 * i + 1], v[4 * i + 2], v[4 * i + 3]);
      }
      __threadfence();   // this lane's partial sums are visible at gpu scope before the count
      __syncwarp();
    };
    // Last-arrival protocol: count this entry; true for the last entry of the tile (which then resets the word).
    auto sk_count = [&]() {
      uint32_t prev = 0;
      if (lane == 0) {
        prev = atomicAdd(sk_word, 1u);
        __threadfence();   // acquire: the partial sums counted before this entry are visible from here on
      }
      prev = __shfl_sync(0xffffffffu, prev, 0);
      __syncwarp();
      const bool last = static_cast<int>(prev) == p.split_k - 1;
      if (last && lane == 0) atomicExch(sk_word, 0u);   // every split has counted: free for the next launch
      return last;
    };
    // Scatter protocol: count this entry, then wait until every entry of the tile has counted. False on timeout.
    auto sk_count_all = [&](int i) {
      bool ok = true;
      if (lane == 0) {
        atomicAdd(sk_word, 1u);
        const uint32_t all = static_cast<uint32_t>(p.split_k);
        if (ld_acquire_gpu(sk_word) < all) {
          const uint64_t t0 = globaltimer_ns();
          while (ld_acquire_gpu(sk_word) < all) {
            if (globaltimer_ns() - t0 > budget) {
              ok = false;
              break;
            }
            __nanosleep(32);
          }
        }
        __threadfence();
        if (!ok) record_error(p.err, kErrSplitK, i);
      }
      ok = __shfl_sync(0xffffffffu, ok ? 1u : 0u, 0) != 0;
      __syncwarp();
      return ok;
    };
    // Scatter protocol, after the reduce: the last of the tile's 2 * split_k counts resets the word.
    auto sk_leave = [&]() {
      __syncwarp();
      if (lane == 0 && atomicAdd(sk_word, 1u) == 2u * static_cast<uint32_t>(p.split_k) - 1u) atomicExch(sk_word, 0u);
    };
    // Reduce chunks [c_begin, c_end) of the tile over all splits. Each finished chunk goes back into tensor memory
    // or, with `crow` set, is rounded and stored to C row crow (columns 32 c onwards; `cols_left` columns of C
    // from the tile's first, `row_ok` false for rows outside C). The other splits' slices are read in units of one
    // chunk of one split (4 KB per warp). With `staged` (the operand ring is idle: this is the cluster's last
    // entry and its accumulator is complete) each warp streams units through kSkSlots 4 KB slots of the ring with
    // cp.async, every lane copying and reading back only its own 16-byte pieces; otherwise two units at a time go
    // through registers (one at a time for wide tiles).
    auto sk_reduce = [&](uint32_t tacc, int c_begin, int c_end, bool staged, __nv_bfloat16* crow, bool row_ok,
                         int cols_left) {
      const int others = p.split_k - 1;
      const int units = (c_end - c_begin) * others;   // unit u: chunk c_begin + u / others, (u % others)-th other split
      auto src_of = [&](int u) {
        const int c = c_begin + u / others, j = u % others;
        const int s = j < sk_own ? j : j + 1;
        return sk_src + static_cast<size_t>(s) * sk_stride + (static_cast<size_t>(8 * c) * 32u + static_cast<size_t>(lane)) * 4u;
      };
      auto load = [&](int u, uint32_t (&x)[32]) {
        const float* src = src_of(u);
#pragma unroll
        for (int i = 0; i < 8; ++i) ld_global_cg_v4(src + i * 128, x[4 * i], x[4 * i + 1], x[4 * i + 2], x[4 * i + 3]);
      };
      float a[32];
      auto add_own = [&](int c, bool first) {
        uint32_t v[32];
        tmem_ld_32x32b_x32(tacc + 32u * c, v);
        tmem_ld_wait();
#pragma unroll
        for (int j = 0; j < 32; ++j) a[j] = first ? __uint_as_float(v[j]) : a[j] + __uint_as_float(v[j]);
      };
      // fold unit u (split s of chunk c) into the running sum in the order 0, 1, ..., split_k - 1
      auto consume = [&](int u, const uint32_t (&x)[32]) {
        const int c = c_begin + u / others, j = u % others;
        const int s = j < sk_own ? j : j + 1;
        if (j == 0 && sk_own == 0) add_own(c, true);
        else if (j > 0 && sk_own == s - 1) add_own(c, false);
        const bool first = j == 0 && sk_own != 0;   // split 0 starts the sum
#pragma unroll
        for (int e = 0; e < 32; ++e) a[e] = first ? __uint_as_float(x[e]) : a[e] + __uint_as_float(x[e]);
        if (j == others - 1) {
          if (sk_own == p.split_k - 1) add_own(c, false);
          uint32_t v[32];
#pragma unroll
          for (int e = 0; e < 32; ++e) v[e] = __float_as_uint(a[e]);
          if (crow == nullptr) {
            tmem_st_32x32b_x32(tacc + 32u * c, v);
          } else if (row_ok) {
            const int cols = cols_left - 32 * c;
            if (cols >= 32) store_row_global<32>(crow + 32 * c, v);
            else if (cols > 0) store_row_global_masked<32>(crow + 32 * c, v, cols);
          }
        }
      };
      if (staged) {
        const uint32_t wbase = sA + static_cast<uint32_t>(q) * (kSkSlots * 4096u) + static_cast<uint32_t>(lane) * 16u;
        auto issue = [&](int u) {   // one commit group per unit, empty past the end, so that groups stay in step
          if (u < units) {
            const float* src = src_of(u);
            const uint32_t dst = wbase + static_cast<uint32_t>(u % kSkSlots) * 4096u;
#pragma unroll
            for (int i = 0; i < 8; ++i) cp_async_16(dst + i * 512u, src + i * 128);
          }
          cp_async_commit();
        };
#pragma unroll 1
        for (int u = 0; u < kSkSlots; ++u) issue(u);
#pragma unroll 1
        for (int u = 0; u < units; ++u) {
          cp_async_wait<kSkSlots - 1>();   // unit u has landed
          uint32_t x[32];
          const uint32_t slot = wbase + static_cast<uint32_t>(u % kSkSlots) * 4096u;
#pragma unroll
          for (int i = 0; i < 8; ++i) ld_shared_v4(slot + i * 512u, x[4 * i], x[4 * i + 1], x[4 * i + 2], x[4 * i + 3]);
          consume(u, x);   // uses x, so the slot has been read before it is refilled below
          issue(u + kSkSlots);
        }
        cp_async_wait<0>();
      } else if constexpr (NB == 1) {
        uint32_t xa[32], xb[32];
        if (units > 0) load(0, xa);
#pragma unroll 1
        for (int u = 0; u < units; u += 2) {
          if (u + 1 < units) load(u + 1, xb);
          consume(u, xa);
          if (u + 2 < units) load(u + 2, xa);
          if (u + 1 < units) consume(u + 1, xb);
        }
      } else {   // wide tiles: one unit at a time (their kernels have no registers to spare for two)
#pragma unroll 1
        for (int u = 0; u < units; ++u) {
          uint32_t x[32];
          load(u, x);
          consume(u, x);
        }
      }
    };
    // The operand ring can stage the reduce: big enough for every warp's slots, and idle after the accumulator of
    // the cluster's last entry is complete (no loads follow, and the MMAs that read it have finished).
    const bool sk_ring_ok =
        static_cast<uint32_t>(p.stages) * (p.a_stage_bytes + p.b_stage_bytes) >= 4u * kSkSlots * 4096u;
    // Split-K inside a cluster (p.kc > 1): the cluster's kc CTAs hold the partial sums of one tile over disjoint K
    // ranges (split = cluster rank), and the tile's nch 32-column chunks are shared out, CTA g owning chunks
    // [g * per, (g + 1) * per). Each CTA sends every chunk it does not own from tensor memory straight into the
    // owner's receive region (st.async into the owner's shared memory, completing on the owner's receive barrier),
    // then waits (bounded) for the other kc - 1 CTAs' copies of its own chunks, adds them in split order
    // 0, 1, ..., kc - 1 (the order of the workspace protocols below, so the same bits), writes the sums back to
    // tensor memory and drains them to C. Receive region: slot j (the j-th other split in rank order) holds for each
    // warp q and owned chunk cc one 4 KB unit, in which lane l's 16-byte piece e (columns 4e..4e+3 of its row) sits
    // at e * 512 + l * 16: sender and owner lanes both move 512 contiguous bytes per instruction. No workspace, no
    // global-memory round trip: the exchange costs one pass through each SM's shared-memory intake.
    auto kc_epilogue = [&](int i, uint32_t tacc, int nch, int row0, int col0) {
      const int per = nch / p.kc;
      const uint32_t piece = static_cast<uint32_t>(lane) * 16u;
#pragma unroll 1
      for (int c = 0; c < nch; ++c) {
        const int g = c / per;   // the chunk's owner
        if (g == ks) continue;
        const int j = ks < g ? ks : ks - 1;   // this CTA's slot in the owner's receive region
        uint32_t v[32];
        tmem_ld_32x32b_x32(tacc + 32u * c, v);
        tmem_ld_wait();
        const uint32_t unit = sR + static_cast<uint32_t>(((j * 4 + q) * per + (c - g * per)) * 4096) + piece;
        const uint32_t dst = mapa_shared(unit, static_cast<uint32_t>(g));
        const uint32_t bar = mapa_shared(recvbar, static_cast<uint32_t>(g));
#pragma unroll
        for (int e = 0; e < 8; ++e)
          st_async_v4(dst + 512u * e, v[4 * e], v[4 * e + 1], v[4 * e + 2], v[4 * e + 3], bar);
      }
      if (!mbar_wait_warp(recvbar, 0, budget)) {
        if (lane == 0) record_error(p.err, kErrSplitK, i);
        kc_waiting = true;
        return false;
      }
      const int lo = ks * per;
#pragma unroll 1
      for (int cc = 0; cc < per; ++cc) {
        float a[32];
#pragma unroll 1
        for (int s = 0; s < p.kc; ++s) {
          uint32_t x[32];
          if (s == ks) {
            tmem_ld_32x32b_x32(tacc + 32u * (lo + cc), x);
            tmem_ld_wait();
          } else {
            const int j = s < ks ? s : s - 1;
            const uint32_t unit = sR + static_cast<uint32_t>(((j * 4 + q) * per + cc) * 4096) + piece;
#pragma unroll
            for (int e = 0; e < 8; ++e) ld_shared_v4(unit + 512u * e, x[4 * e], x[4 * e + 1], x[4 * e + 2], x[4 * e + 3]);
          }
#pragma unroll
          for (int e = 0; e < 32; ++e) a[e] = s == 0 ? __uint_as_float(x[e]) : a[e] + __uint_as_float(x[e]);
        }
        uint32_t w[32];
#pragma unroll
        for (int e = 0; e < 32; ++e) w[e] = __float_as_uint(a[e]);
        tmem_st_32x32b_x32(tacc + 32u * (lo + cc), w);
      }
      tmem_st_wait();
      drain(tacc + 32u * lo, row0, col0 + 32 * lo, 32 * per, 0u);
      return true;
    };
    // The split-K epilogue of entry idx, whose accumulator (nch chunks at TMEM tacc) is complete. False on timeout.
    auto sk_epilogue = [&](int idx, int i, uint32_t tacc, int nch, int row0, int col0) -> bool {
      if constexpr (kcl) {
        return kc_epilogue(i, tacc, nch, row0, col0);
      } else {
        sk_setup(idx);
        const bool staged = sk_ring_ok && idx + p.nclusters >= p.tiles;
        if (p.sk_scatter) {
          const int lo = sk_own * nch / p.split_k, hi = (sk_own + 1) * nch / p.split_k;
          sk_publish(tacc, nch, lo, hi);
          if (!sk_count_all(i)) return false;
          sk_reduce(tacc, lo, hi, staged, p.C + static_cast<long long>(row0 + lane) * p.ldc + col0,
                    lane < ROWS_W && row0 + lane < p.m_valid, p.n_valid - col0);
          sk_leave();
          return true;
        }
        sk_publish(tacc, nch, 0, 0);
        if (sk_count()) {
          sk_reduce(tacc, 0, nch, staged, nullptr, false, 0);
          tmem_st_wait();
          drain(tacc, row0, col0, nch * 32, 0u);
        }
        return true;
      }
    };
    for (int i = 0;; ++i) {
      const int idx = cid + i * p.nclusters;
      if (idx >= p.tiles) break;
      int cm, tn;
      bool narrow;
      first.coords(p, idx, cm, tn, narrow);
      last_entry = idx + p.nclusters >= p.tiles;
      const int row0 = (cm * p.cl + static_cast<int>(rank)) * BM + q * ROWS_W;   // first row of this warp
      const int width = narrow ? p.bn * NB / 2 : p.bn * NB;   // output columns of this tile
      const int col0 = tn * width;
      if (split) {
        // half h = TMEM columns [h * bn, (h + 1) * bn) with its own barriers; a half-width tile has only half 0.
        // Under split-K both halves are held until the entry has counted itself.
        bool ok = true;
        for (int h = 0; h < 2; ++h) {
          if (!mbar_wait_warp(tfull0 + 8u * h, acc_phase, budget)) {
            record_error(p.err, kErrEpilogue, i);
            ok = false;
            break;
          }
          tc_fence_after();
          if (SPLITK && p.split_k > 1) continue;   // both halves first, then the split-K epilogue on the whole tile
          const uint32_t tacc = tmem_base + lane_base + static_cast<uint32_t>(h * p.bn);
          if (h == 0 || !narrow)
            drain(tacc, row0, col0 + h * p.bn, p.bn, tempty0 + 8u * h);
          else
            release(tempty0 + 8u * h);
        }
        if (!ok) break;
        if (SPLITK && p.split_k > 1) {
          if (!sk_epilogue(idx, i, tmem_base + lane_base, width >> 5, row0, col0)) break;
          release(tempty0);
          release(tempty0 + 8u);
        }
        acc_phase ^= 1u;
        continue;
      }
      if (!mbar_wait_warp(tfull0 + 8u * acc, acc_phase, budget)) {
        record_error(p.err, kErrEpilogue, i);
        break;
      }
      tc_fence_after();
      const uint32_t tacc = tmem_base + lane_base + acc * static_cast<uint32_t>(p.acc_stride);
      if (SPLITK && p.split_k > 1) {
        if (!sk_epilogue(idx, i, tacc, width >> 5, row0, col0)) break;
      } else {
        drain(tacc, row0, col0, width, tempty0 + 8u * acc);
      }
      if (SPLITK && p.split_k > 1) release(tempty0 + 8u * acc);
      if (++acc == static_cast<uint32_t>(p.acc_bufs)) {
        acc = 0;
        acc_phase ^= 1u;
      }
    }
    // Shared memory must outlive the TMA engine's reads of the staging buffers; the global writes themselves are
    // complete when the grid is.
    if (TMA_STORE && lane == 0) bulk_wait_group_read<0>();
    __syncwarp();
  }

  // ------------------------------------------------------------------ teardown
  tc_fence_before();
  __syncthreads();
  if (PAIRED || kcl) cluster_sync_all();   // the cluster is done with each other's barriers and memory
  // A wait for the other splits' sums that timed out: every CTA of the cluster has now passed the barrier, so the
  // stores it sends here have been issued; let them land (bounded) before this CTA's shared memory goes away.
  if (kc_waiting && lane == 0) mbar_wait_bounded(recvbar, 0, budget);
  tc_fence_after();
  if (warp == 1) {
    __syncwarp();
    tmem_dealloc<CG>(tmem_base, p.tmem_cols);
  }
}

// One thread runs the whole mainloop: a prologue fills the ring, then each k-block waits for its stage, issues the
// MMAs, commits the stage's release and, once the MMA has read it, refills the stage with the k-block `stages`
// ahead. All four warps then drain the accumulator with the register epilogue. One tile per CTA, row-major order.
template <int BM>
__global__ void __launch_bounds__(kRingThreads, 1)
    sm100_gemm_ring(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                    const __grid_constant__ GemmParams p) {
  constexpr int ROWS_W = BM / 4;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  const uint32_t base = (raw + 1023u) & ~1023u;
  const uint32_t sA = base;
  const uint32_t sB = sA + p.stages * p.a_stage_bytes;
  const uint32_t bars = sB + p.stages * p.b_stage_bytes;
  const uint32_t full0 = bars;
  const uint32_t empty0 = bars + 8u * p.stages;
  const uint32_t tfull = bars + 16u * p.stages;
  const uint32_t tslot = tfull + 8u;
  volatile uint32_t* tslot_ptr = reinterpret_cast<volatile uint32_t*>(smem_raw + (tslot - raw));

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint64_t budget = p.budget_ns;

  if (threadIdx.x == 0) {
    for (int s = 0; s < p.stages; ++s) {
      mbar_init(full0 + 8u * s, 1);
      mbar_init(empty0 + 8u * s, 1);
    }
    mbar_init(tfull, 1);
    fence_mbar_init();
    tma_prefetch_map(&tmA);
    tma_prefetch_map(&tmB);
  }
  if (warp == 0) {
    tmem_alloc<1>(tslot, p.tmem_cols);
    tmem_relinquish<1>();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tslot_ptr;

  int cm, tn;
  tile_coords(p, static_cast<int>(blockIdx.x), cm, tn);
  const int row_a = cm * BM;
  const int row_b = tn * p.bn;

  if (threadIdx.x == 0) {
    const int pro = p.num_kb < p.stages ? p.num_kb : p.stages;
    for (int j = 0; j < pro; ++j) {
      if (j == p.skip_job) continue;
      mbar_arrive_expect_tx(full0 + 8u * j, p.tx_bytes);
      tma_load_2d(sA + j * p.a_stage_bytes, &tmA, full0 + 8u * j, j * kBK, row_a);
      tma_load_2d(sB + j * p.b_stage_bytes, &tmB, full0 + 8u * j, j * kBK, row_b);
    }
    bool failed = false;
    int issued = pro;   // loads issued so far (jobs 0 .. issued-1)
    for (int kb = 0; kb < p.num_kb; ++kb) {
      const uint32_t s = static_cast<uint32_t>(kb % p.stages), ph = static_cast<uint32_t>((kb / p.stages) & 1);
      if (!mbar_wait_bounded(full0 + 8u * s, ph, budget)) {
        record_error(p.err, kErrMmaFull, kb);
        failed = true;
        break;
      }
      tc_fence_after();
      const uint64_t ad = smem_desc_sw128(sA + s * p.a_stage_bytes);
      const uint64_t bd = smem_desc_sw128(sB + s * p.b_stage_bytes);
#pragma unroll
      for (int k = 0; k < kBK / 16; ++k) mma_bf16<1>(tmem_base, ad + 2u * k, bd + 2u * k, p.idesc, (kb | k) != 0);
      mma_commit<1>(empty0 + 8u * s);
      const int nxt = kb + p.stages;
      if (nxt < p.num_kb) {
        if (!mbar_wait_bounded(empty0 + 8u * s, ph, budget)) {   // the MMAs above have read stage s
          record_error(p.err, kErrProducer, nxt);
          failed = true;
          break;
        }
        if (nxt != p.skip_job) {
          mbar_arrive_expect_tx(full0 + 8u * s, p.tx_bytes);
          tma_load_2d(sA + s * p.a_stage_bytes, &tmA, full0 + 8u * s, nxt * kBK, row_a);
          tma_load_2d(sB + s * p.b_stage_bytes, &tmB, full0 + 8u * s, nxt * kBK, row_b);
        }
        issued = nxt + 1;
      }
    }
    mma_commit<1>(tfull);   // also the drain point for every MMA issued above
    if (failed) {
      const int first = issued - p.stages < 0 ? 0 : issued - p.stages;
      for (int j = first; j < issued; ++j) {
        if (j == p.skip_job) continue;
        const uint32_t s = static_cast<uint32_t>(j % p.stages), ph = static_cast<uint32_t>((j / p.stages) & 1);
        if (!mbar_wait_bounded(full0 + 8u * s, ph, budget)) record_error(p.err, kErrLoadDrain, j);
      }
    }
  }
  __syncwarp();

  const bool ready = mbar_wait_bounded(tfull, 0, budget);
  if (!ready) record_error(p.err, kErrEpilogue, 0);
  tc_fence_after();
  __syncwarp();
  {
    const int q = warp & 3;
    const uint32_t tacc = tmem_base + (static_cast<uint32_t>(q * 32) << 16);
    __nv_bfloat16* crow = p.C + static_cast<long long>(row_a + q * ROWS_W + lane) * p.ldc + row_b;
    // A failed tile leaves C unwritten (the host reports the error), but the TMEM reads stay warp-uniform.
    epilogue_registers(tacc, crow, p.bn, ready && lane < ROWS_W, p.bn);
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 0) {
    __syncwarp();
    tmem_dealloc<1>(tmem_base, p.tmem_cols);
  }
}

}  // namespace sm100
