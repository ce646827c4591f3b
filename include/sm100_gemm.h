/*
 * sm100_gemm.h — C ABI of the B200 (sm_100a) bf16 GEMM that stands in for the Hopper wgmma GEMM of
 * narain1/tinygrad-hopper-wgmma. Plain pointers, sizes and status codes; no framework types.
 *
 *   C[M,N] (bf16) = A[M,K] (bf16, row-major) x B[K,N], with B supplied K-major as BT[N,K] (row-major) or, with
 *   bg_cfg.b_nmajor = 1, as B[K,N] itself; fp32 accumulation, bf16 output rounded to nearest even. M, N and K are
 *   multiples of the tile unless bg_cfg.ragged is set.
 *
 * Status codes: 0 = ok; negative = the arguments break the operator's contract (the Python layer raises
 * ValueError, as the reference does for config and shape errors); positive = a CUDA / driver error or a device-side
 * timeout (RuntimeError). bg_last_error() returns the message of the last failing call on this thread.
 *
 * Threading: a plan is immutable after bg_plan_create and may be launched repeatedly on one stream at a time. Plans
 * on different devices or streams are independent. Launches are asynchronous on the given stream. One exception: a
 * split-K plan that reduces through the workspace with all its splits in one wave (the splits of a tile wait for
 * each other on different clusters) needs all its CTAs resident at once; launched beside other work that holds SMs,
 * its bounded wait can run out, and the launch then reports an error (bg_plan_check_error) instead of a result.
 * Split-K inside a cluster has no such need: the CTAs that wait for each other form one cluster, which the GPU
 * always schedules at once.
 */
#ifndef SM100_GEMM_H
#define SM100_GEMM_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Kernel families (the reference's ladder steps map onto these, see bg_cfg). */
enum {
  BG_KIND_WS = 0,    /* persistent warp-specialized kernel: one cluster per SM, host-built tile table          */
  BG_KIND_GATED = 1, /* same warp roles, one tile per cluster, row-major order (gated.py consumers >= 1)       */
  BG_KIND_RING = 2   /* one thread issues TMA and MMA, one tile per CTA (gated.py consumers == 0, "tma_ring")  */
};

/* Error-word roles (bits 24-31 of the word bg_plan_check_error returns; bits 0-23 hold the role's counter). */
enum {
  BG_ERR_PRODUCER = 1,   /* TMA producer timed out waiting for a free stage       */
  BG_ERR_MMA_FULL = 2,   /* MMA issuer timed out waiting for a loaded stage       */
  BG_ERR_MMA_ACC = 3,    /* MMA issuer timed out waiting for a free accumulator   */
  BG_ERR_EPILOGUE = 4,   /* epilogue timed out waiting for a finished accumulator */
  BG_ERR_DRAIN = 5,      /* final wait for outstanding MMAs timed out             */
  BG_ERR_LOAD_DRAIN = 6, /* wait for in-flight loads after another error timed out */
  BG_ERR_SPLIT_K = 7     /* split-K (one wave): a tile's other splits did not all publish in time */
};

/*
 * Knobs of one GEMM. Field names follow WSCfg / GatedCfg (hopper_wgmma/gemm.py:246-258, gated.py:18-25).
 *   BN          output columns per tile (MMA N): a multiple of 16 in [16, 256] (RING/GATED with BM = 64: of 8)
 *   BK          must be 64 (one 128-byte swizzle row of bf16)
 *   stages      shared-memory ring depth (>= 2); 0 = as many as fit
 *   consumers   0, 1 or 2: BM = 64 * max(consumers, 1) rows per CTA (M = 64 or 128 per tcgen05.mma)
 *   num_sm      persistent clusters * cluster size upper bound; <= 0 = the device's SM count
 *   group_m/n   grouped tile order (gemm.py:200-215)
 *   tma_store   1 = swizzled staging + TMA store epilogue (BN multiple of 64), 0 = direct register stores
 *   cluster     1 or 2; 2 with consumers == 2 pairs two CTAs on one M = 256 tcgen05.mma (cta_group::2)
 *   hilbert     1 = Hilbert tile order dealt round-robin over the clusters (gemm.py:218-240), ragged allowed
 *   acc_bufs    accumulator buffers in tensor memory: 0 = auto (2 when 2 * BN <= 512), 1 or 2
 *   wait_budget_ns  per-wait device time limit; 0 = 4 s
 *   n_mma       tcgen05.mma instructions along N per K step (1 or 2; persistent kernel only): a tile is n_mma * BN
 *               columns wide, so n_mma = 2 with BN = 256 gives 128 x 512 per CTA (256 x 512 per CTA pair), which
 *               reads 25% fewer operand bytes per FLOP than 256 x 256 at the cost of a single TMEM accumulator
 *   no_tail_split   0 (default): when the persistent schedule's last wave is at most half full, its tiles are split
 *                   into half-width tiles so that the tail costs about half a tile; 1: keep whole tiles
 *   ragged      0 (default): M, N, K must be multiples of the tile, as in the reference (gemm.py:303);
 *               1 (persistent kernel): any M, and N, K multiples of 8 — edge tiles are zero-filled on load and clipped
 *               or masked on store
 *   debug_skip_job  test hook: the producer never loads this job (-1 = off) so that the kernel's waits run out and
 *                   the launch reports an error instead of hanging
 *   split_k     0 or 1: off. -1: automatic (the most splits, up to 16, that keep all tiles' splits within one wave of
 *               clusters with at least 32 k-blocks each, 24 where they can meet inside a cluster; off otherwise).
 *               S in [2, 64] (persistent kernel, tiles a multiple of 32 columns wide, S <= K / 64):
 *               each output tile is computed by S entries of the schedule, each over a contiguous 1/S of K, on
 *               different clusters; fp32 partial sums meet in a plan-owned workspace and are added in split
 *               order (bitwise reproducible). When every entry has its own cluster (one wave) the plan launches
 *               cooperatively and the tile's entries share the reduction out; otherwise the entry that finishes
 *               last reduces the tile and no entry waits for another. For shapes with few tiles and long K. Not
 *               available through bg_gemm_noalloc (it owns no workspace).
 *   no_k_serpentine 0 (default): a persistent cluster walks K forwards on its even-numbered tiles and backwards on
 *               its odd-numbered ones, so each wave starts on the K-slabs the previous wave left in L2 (fewer DRAM
 *               reads); 1: always forwards (the fp32 accumulation order of every tile then runs along K)
 *   b_nmajor    0 (default): the B operand is BT[N,K] (K-major, row pitch ldb >= K), as the reference's kernel takes
 *               it after its transpose (gemm.py:382). 1 (warp-specialized kernel): the B operand is B[K,N] itself
 *               (N-major, row pitch ldb >= N; a column block of a wider B is allowed), read through MN-major
 *               tcgen05 descriptors, so the caller makes no transposed copy. Needs each CTA's share of a tile's
 *               columns (BN, or BN / 2 in a CTA pair) to be a multiple of 64; half-width tail tiles are used only
 *               when their share is too.
 *   wave_sync   0 (default): automatic — on for persistent schedules without split-K that give each cluster at
 *               least 4 tiles and whose waves touch operand panels too big to stay in L2 (at least 96 MB by the
 *               estimate 4 K sqrt(clusters x tile rows x tile columns) bytes: 256x512 pair tiles from K = 8192),
 *               off otherwise; 1: on (persistent kernel, no split-K); 2: off. When on, the TMA
 *               producers of all CTAs meet at every tile boundary (a wait on a plan-owned 64-bit counter), so the
 *               tiles of one wave stay in step and share their operand panels through L2; without it CTAs drift
 *               apart over many tiles and re-read the panels from DRAM. The barrier orders no data and is soft: a
 *               CTA that has waited 200 us at one boundary (its launch is not wholly resident, e.g. beside another
 *               launch on the same GPU) stops waiting for the rest of that launch; results never depend on it.
 *               Not used by bg_gemm_noalloc.
 *   split_k_cluster  how a split-K plan (split_k > 1, or chosen by -1) reduces its splits. 0 (default):
 *               automatic — inside a cluster when the plan allows it (below), through the workspace otherwise;
 *               1: inside a cluster, or fail; 2: through the workspace. Inside a cluster, the split_k splits of a
 *               tile run on the CTAs of one cluster of split_k CTAs (its ranks), and the tile's columns are shared
 *               out among them: each CTA sends the columns it does not own straight from tensor memory into their
 *               owner's shared memory (distributed shared memory, st.async), adds what it receives for its own
 *               columns in split order and stores them. No workspace and no global-memory round trip; the same
 *               bits as the workspace. Needs single-CTA tiles (cluster 1, n_mma 1), split_k 2 or 4, each CTA's
 *               share of the tile's columns a multiple of 64 (32 with the register epilogue), room for the
 *               received sums ((split_k - 1) * 128 * width / split_k * 4 bytes of shared memory) and every tile
 *               on its own cluster at once (one wave).
 */
typedef struct bg_cfg {
  int32_t kind;
  int32_t BN;
  int32_t BK;
  int32_t stages;
  int32_t consumers;
  int32_t num_sm;
  int32_t group_m;
  int32_t group_n;
  int32_t tma_store;
  int32_t cluster;
  int32_t hilbert;
  int32_t acc_bufs;
  int64_t wait_budget_ns;
  int32_t debug_skip_job;
  int32_t n_mma;
  int32_t no_tail_split;
  int32_t ragged;
  int32_t split_k;
  int32_t no_k_serpentine;
  int32_t b_nmajor;
  int32_t wave_sync;
  int32_t split_k_cluster;
} bg_cfg;

/* What a plan resolved to (for reports and tests). */
typedef struct bg_plan_info {
  int32_t grid;           /* CTAs launched                                   */
  int32_t threads;        /* threads per CTA                                 */
  int32_t smem_bytes;     /* dynamic shared memory per CTA                   */
  int32_t stages;         /* ring depth used                                 */
  int32_t tiles;          /* schedule entries (cluster tiles)                */
  int32_t clusters;       /* persistent clusters (or tiles, non-persistent)  */
  int32_t cluster;        /* CTAs per cluster                                */
  int32_t paired;         /* 1 = cta_group::2 MMA across the pair            */
  int32_t bm;             /* rows per CTA tile                               */
  int32_t bn;             /* columns per tile                                */
  int32_t acc_bufs;       /* accumulator buffers                             */
  int32_t tmem_cols;      /* tensor-memory columns allocated per CTA         */
  int32_t max_active_clusters; /* occupancy limit reported by the runtime (0 if not queried) */
  int32_t narrow_tiles;   /* half-width tiles in the last wave (0 = no tail split)             */
  int32_t split_k;        /* K splits per output tile (1 = off)                                */
  char kernel[96];        /* kernel family and template arguments            */
} bg_plan_info;

typedef struct bg_plan bg_plan;

/* Message of the last failing call on this thread ("" if none). */
const char* bg_last_error(void);

/* Library version: major * 10000 + minor * 100 + patch. */
int32_t bg_version(void);

/* Device properties the host layer needs (replaces the reference's hard-coded num_sm=128 and SMEM_LIMIT,
 * gemm.py:26, :252). */
int32_t bg_device_info(int32_t device, int32_t* sm_count, int32_t* smem_optin, int32_t* cc_major, int32_t* cc_minor);

/*
 * Build a GEMM plan for C[M,N] = A[M,K] x BT[N,K]^T. Replaces build_gemm_ws + run (gemm.py:293-398) and
 * build_gated_gemm + run (gated.py:50-123) on the host side: validates the shape contract (gemm.py:300-311), encodes
 * the tensor maps (tensor_map.py:13-33), builds the tile table (gemm.py:200-240) in device memory, allocates the
 * error word and sets the kernel's launch attributes (runtime.py:20-98).
 *   A   device pointer, M rows, row pitch lda elements (>= K)
 *   BT  device pointer, N rows, row pitch ldb elements (>= K); with cfg->b_nmajor = 1 it is B[K,N]: K rows, row
 *       pitch ldb elements (>= N), and a column block of a wider B is allowed
 *   C   device pointer, M rows, row pitch ldc elements (>= N); a column shard of a wider C is allowed
 * All pointers 16-byte aligned, all pitches multiples of 8 elements. The plan keeps the raw pointers: the caller keeps
 * the buffers alive for the plan's life (as the reference keeps A and BT alive in launch, gemm.py:394).
 */
int32_t bg_plan_create(bg_plan** out, const bg_cfg* cfg, int64_t M, int64_t N, int64_t K, const void* A, int64_t lda,
                       const void* BT, int64_t ldb, void* C, int64_t ldc, int32_t device);

/* Enqueue the GEMM on `stream` (a cudaStream_t; NULL = legacy default stream). Replaces launch() (gemm.py:394). */
int32_t bg_plan_launch(bg_plan* plan, void* stream);

/* Wait for `stream`, then read the plan's device error word into *err_word (0 = no error) and clear it.
 * Returns a positive status if the word is non-zero. */
int32_t bg_plan_check_error(bg_plan* plan, void* stream, uint32_t* err_word);

int32_t bg_plan_get_info(const bg_plan* plan, bg_plan_info* info);

void bg_plan_destroy(bg_plan* plan);

/*
 * bg_gemm_noalloc — the same GEMM as bg_plan_create + bg_plan_launch in one call that allocates no memory.
 * No counterpart in the reference: it exists for callers that may not allocate device memory themselves, such as a
 * plugin inside a framework that owns the whole device memory through its own pool allocator (an allocation behind
 * the pool's back can fail or fragment it), or code on a path where cudaMalloc / cudaFree would synchronize the
 * device. The caller still passes A, BT and C (as for bg_plan_create); the kernel's scratch — its tile table and
 * error word — lives in a fixed file-scope device array of this library (256 KiB + 256 bytes per GPU that loads the
 * library, held until the process exits), so a problem may have at most 65536 tiles (cluster tiles of the schedule);
 * larger ones are rejected with a negative status before anything is enqueued.
 *   The first call on a device looks up the array's device address (cudaGetSymbolAddress) with that device current;
 *   make that first call before any stream capture. (A lookup that fails is retried by the next call.)
 *   Every call reuses the same array and overwrites the previous call's tile table and error word (the error word is
 *   cleared on the stream before each launch). Calls whose kernels can overlap on the GPU — on different streams, or
 *   from different threads — race on that array: serialize them on one stream.
 *   The tile table is staged from host memory with cudaMemcpyAsync on `stream`, ordered after the stream's earlier
 *   work.
 *   split_k: values above 1 are rejected (a split schedule needs a workspace); -1 (automatic) runs unsplit here.
 *   err_word == NULL: returns once the GEMM is enqueued. Otherwise it waits for `stream`, stores the kernel's error
 *   word (0 = ok) and returns a positive status if a device-side wait timed out.
 */
int32_t bg_gemm_noalloc(const bg_cfg* cfg, int64_t M, int64_t N, int64_t K, const void* A, int64_t lda,
                        const void* BT, int64_t ldb, void* C, int64_t ldc, int32_t device, void* stream,
                        uint32_t* err_word);

/*
 * Host-only schedule builders (no device needed). Entries are (row tile << 16) | column tile.
 * bg_hilbert_order: the tiles of an M x N tile grid in Hilbert-curve order (the walk of gemm.py:222-240); dealing
 *   entry p to cluster p % clusters reproduces hilbert_schedule's assignment, ragged ends included.
 * bg_grouped_order: entry t = grouped_tile_order(CMT, NT, GM, GN)(t) (gemm.py:200-215).
 * Both return the number of entries written, or a negative status if `capacity` is too small or sizes are invalid.
 */
int32_t bg_hilbert_order(int32_t m_tiles, int32_t n_tiles, int32_t* out, int32_t capacity);
int32_t bg_grouped_order(int32_t m_tiles, int32_t n_tiles, int32_t group_m, int32_t group_n, int32_t* out,
                         int32_t capacity);

/*
 * Encode the reference's 3-D bf16 tensor map (tensor_map.py:13-33): dims (64, height, width/64), strides
 * (2*width, 128) bytes, box (64, box_h, box_w/64), 128-byte swizzle, into the 128 bytes at `out`.
 * Needs the CUDA driver (not a device context). The GEMM itself encodes its own 2-D maps.
 */
int32_t bg_encode_tensor_map_3d(void* out128, const void* base, int64_t height, int64_t width, int32_t box_h,
                                int32_t box_w);

#ifdef __cplusplus
}
#endif

#endif /* SM100_GEMM_H */
