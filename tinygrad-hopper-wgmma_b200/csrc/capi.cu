// Host side of the sm_100a GEMM behind the C ABI declared in include/sm100_gemm.h.
//
// It replaces three host pieces of the reference: the shape/schedule arithmetic of build_gemm_ws and
// build_gated_gemm (hopper_wgmma/gemm.py:300-319, gated.py:55-63), the tensor-map encoder (tensor_map.py:13-33, here
// 2-D maps passed as __grid_constant__ kernel parameters instead of 128-byte device tensors), and the
// process-global tinygrad runtime hooks (runtime.py:20-98), which become explicit launch attributes:
// cudaFuncSetAttribute for dynamic shared memory and a cluster-dimension attribute on cudaLaunchKernelEx.
#include <cuda.h>
#include <cuda_runtime.h>
#include <cudaTypedefs.h>

#include <algorithm>
#include <cmath>
#include <array>
#include <map>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <memory>
#include <mutex>
#include <vector>

#include "gemm_kernels.cuh"
#include "sm100_gemm.h"

using sm100::GemmParams;

namespace {

thread_local char g_err[512] = "";

int32_t fail(int32_t code, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_err, sizeof(g_err), fmt, ap);
  va_end(ap);
  return code;
}

int32_t cuda_fail(cudaError_t e, const char* what) {
  return fail(e == cudaSuccess ? 1 : static_cast<int32_t>(e), "%s failed: %s (%s)", what, cudaGetErrorName(e),
              cudaGetErrorString(e));
}

// ---------------------------------------------------------------------------------------------------------------
// Driver entry point for cuTensorMapEncodeTiled, fetched through the runtime so that the library does not link
// libcuda directly (it then loads on machines without a driver, e.g. for the CPU-side tests).
// ---------------------------------------------------------------------------------------------------------------
PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &p, 12000, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  });
  return fn;
}

int32_t encode_2d(CUtensorMap* map, const void* base, uint64_t inner, uint64_t outer, uint64_t pitch_elems,
                  uint32_t box_inner, uint32_t box_outer, const char* what) {
  auto fn = encode_fn();
  if (fn == nullptr) return fail(2, "cuTensorMapEncodeTiled is unavailable (no CUDA driver)");
  const cuuint64_t dims[2] = {inner, outer};
  const cuuint64_t strides[1] = {pitch_elems * 2};
  const cuuint32_t box[2] = {box_inner, box_outer};
  const cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(3, "cuTensorMapEncodeTiled(%s) failed with CUresult %d", what, static_cast<int>(r));
  return 0;
}

// ---------------------------------------------------------------------------------------------------------------
// Tile orders (host). Entries are (row tile << 16) | column tile.
// ---------------------------------------------------------------------------------------------------------------
// Hilbert index d -> (x, y) on an n x n grid (n a power of two), the iterative walk used by fast.cu's createHilbert
// and hilbert_schedule (gemm.py:222-230).
void hilbert_d2xy(int n, long long d, int& x, int& y) {
  x = y = 0;
  long long t = d;
  for (int s = 1; s < n; s *= 2) {
    const int rx = static_cast<int>(1 & (t / 2));
    const int ry = static_cast<int>(1 & (t ^ rx));
    if (ry == 0) {
      if (rx == 1) {
        x = s - 1 - x;
        y = s - 1 - y;
      }
      std::swap(x, y);
    }
    x += s * rx;
    y += s * ry;
    t /= 4;
  }
}

// The curve covers each aligned s x s block (s a power of two) in one run of s * s consecutive positions, so a run
// whose block lies outside the grid is skipped whole: the walk costs O(cells of the grid * log dim) instead of
// O(dim^2), which matters for tall or wide grids (2^20 rows of 128 give dim = 8192 for a single column of tiles).
void hilbert_walk(int dim, long long d0, int s, int mt, int nt, std::vector<int32_t>& out) {
  int x, y;
  hilbert_d2xy(dim, d0, x, y);   // a cell of the block; its corner is (x, y) rounded down to multiples of s
  if ((x & ~(s - 1)) >= mt || (y & ~(s - 1)) >= nt) return;
  if (s == 1) {
    out.push_back((x << 16) | y);
    return;
  }
  const long long quarter = static_cast<long long>(s / 2) * (s / 2);
  for (int i = 0; i < 4; ++i) hilbert_walk(dim, d0 + i * quarter, s / 2, mt, nt, out);
}

// Cells of the mt x nt grid in the order the Hilbert curve over the smallest power-of-two square covering it visits
// them (gemm.py:218-240 walks every cell of that square and keeps the ones inside the grid: the same order).
void hilbert_order(int mt, int nt, std::vector<int32_t>& out) {
  out.clear();
  out.reserve(static_cast<size_t>(mt) * nt);
  int dim = 1;
  while (dim < std::max(mt, nt)) dim *= 2;
  hilbert_walk(dim, 0, dim, mt, nt, out);
}

// grouped_tile_order (gemm.py:200-215): GM x GN super-tiles in row-major order when they divide the grid, else
// Triton-style GROUP_M (GM row tiles swept over all columns, column-major inside, ragged last group).
void grouped_order(int mt, int nt, int gm, int gn, std::vector<int32_t>& out) {
  out.resize(static_cast<size_t>(mt) * nt);
  const bool two_d = (mt % gm == 0) && (nt % gn == 0);
  for (int t = 0; t < mt * nt; ++t) {
    int r, c;
    if (two_d) {
      const int st = t / (gm * gn), pos = t % (gm * gn);
      r = (st / (nt / gn)) * gm + pos / gn;
      c = (st % (nt / gn)) * gn + pos % gn;
    } else {
      const int first = (t / (gm * nt)) * gm;
      const int rows = first > mt - gm ? mt - first : gm;
      const int rr = t % (gm * nt);
      r = first + rr % rows;
      c = rr / rows;
    }
    out[t] = (r << 16) | c;
  }
}

// ---------------------------------------------------------------------------------------------------------------
// Kernel table
// ---------------------------------------------------------------------------------------------------------------
using WsKernel = void (*)(const CUtensorMap, const CUtensorMap, const CUtensorMap, const CUtensorMap,
                          const GemmParams);
using RingKernel = void (*)(const CUtensorMap, const CUtensorMap, const GemmParams);

// Split-K is a template switch so that the kernels without it carry none of its code or registers.
template <int NB, int SK>
WsKernel pick_ws_nb(int bm, bool paired, bool tma_store) {
  using namespace sm100;
  if (bm == 128) {
    if (paired) return tma_store ? sm100_gemm_ws<128, true, true, NB, SK> : sm100_gemm_ws<128, true, false, NB, SK>;
    return tma_store ? sm100_gemm_ws<128, false, true, NB, SK> : sm100_gemm_ws<128, false, false, NB, SK>;
  }
  return tma_store ? sm100_gemm_ws<64, false, true, NB, SK> : sm100_gemm_ws<64, false, false, NB, SK>;
}

// split: sm100::kSplitNone, kSplitWorkspace or kSplitCluster (single-CTA tiles with one N block only)
WsKernel pick_ws(int bm, bool paired, bool tma_store, int nblk, int split) {
  using namespace sm100;
  if (split == kSplitCluster) {
    if (paired || nblk != 1) return nullptr;
    if (bm == 128) return tma_store ? sm100_gemm_ws<128, false, true, 1, kSplitCluster> : sm100_gemm_ws<128, false, false, 1, kSplitCluster>;
    return tma_store ? sm100_gemm_ws<64, false, true, 1, kSplitCluster> : sm100_gemm_ws<64, false, false, 1, kSplitCluster>;
  }
  if (split == kSplitWorkspace)
    return nblk == 2 ? pick_ws_nb<2, kSplitWorkspace>(bm, paired, tma_store) : pick_ws_nb<1, kSplitWorkspace>(bm, paired, tma_store);
  return nblk == 2 ? pick_ws_nb<2, kSplitNone>(bm, paired, tma_store) : pick_ws_nb<1, kSplitNone>(bm, paired, tma_store);
}

RingKernel pick_ring(int bm) { return bm == 128 ? sm100::sm100_gemm_ring<128> : sm100::sm100_gemm_ring<64>; }

uint32_t pow2_cols(int n) {
  uint32_t c = 32;
  while (c < static_cast<uint32_t>(n)) c *= 2;
  return c;
}

// tcgen05 instruction descriptor, kind::f16: D f32 (bits 4-5 = 1), A bf16 (bits 7-9 = 1), B bf16 (bits 10-12 = 1),
// both K-major (bits 15, 16 = 0), N >> 3 in bits 17-22, M >> 4 in bits 24-28. Bit 16 set = B is MN-major.
constexpr uint32_t kIdescBMajorMN = 1u << 16;
uint32_t make_idesc(int m, int n) {
  return (1u << 4) | (1u << 7) | (1u << 10) | (static_cast<uint32_t>(n >> 3) << 17) |
         (static_cast<uint32_t>(m >> 4) << 24);
}

}  // namespace

struct bg_plan {
  int device = 0;
  int kind = BG_KIND_WS;
  int bm = 128;
  bool paired = false;
  bool tma_store = false;
  int cl = 1;
  int kc = 1;   // split-K inside a cluster: CTAs per cluster that share a tile's K (launched cluster = cl * kc)
  int grid = 0;
  int threads = 0;
  size_t smem = 0;
  int max_active_clusters = 0;
  bool cooperative = false;   // split-K with one entry per cluster: all CTAs must be resident at once
  CUtensorMap tmA{}, tmB{}, tmBn{}, tmC{};
  int narrow_tiles = 0;
  GemmParams kp{};
  int32_t* d_sched = nullptr;
  bool holds_table = false;          // d_sched is a reference on the device store's table table_key
  std::array<int, 8> table_key{};
  unsigned int* d_err = nullptr;
  unsigned long long* d_wave = nullptr;   // wave-barrier counter (from the device store's slab), or null
  unsigned long long wave_per_launch = 0; // arrivals one launch adds to it
  unsigned long long launches = 0;        // launches enqueued since the counter was last zero
  size_t partial_bytes = 0;          // split-K workspace, owned by the plan
  size_t ticket_words = 0;
  float* d_partial = nullptr;
  unsigned int* d_tickets = nullptr;
  WsKernel ws = nullptr;
  RingKernel ring = nullptr;
  char name[128] = "";   // bg_plan_info.kernel receives its first 95 characters
};

namespace {

// Save / restore the caller's current device around work on the plan's device.
struct DeviceGuard {
  int prev = -1;
  bool changed = false;
  cudaError_t status = cudaSuccess;
  explicit DeviceGuard(int dev) {
    status = cudaGetDevice(&prev);
    if (status == cudaSuccess && prev != dev) {
      status = cudaSetDevice(dev);
      changed = status == cudaSuccess;
    }
  }
  ~DeviceGuard() {
    if (changed) cudaSetDevice(prev);
  }
};

// Device storage shared by the plans of one device, so that building a plan allocates nothing once warm (no
// cudaMalloc / cudaFree, which can synchronize the device, on the path of a caller that plans per batch):
//   * tile tables, one per distinct schedule, uploaded on first use and shared by every plan of that schedule
//     (reference-counted). A table no plan uses stays cached for the next plan of its schedule, up to
//     kIdleTables tables and kIdleTableBytes bytes per device; beyond that the least recently released ones are
//     freed, so a caller whose shapes keep changing (ragged batches) holds bounded device memory;
//   * error words, one per live plan, handed out from 4 KiB slabs and returned when the plan is destroyed.
constexpr size_t kIdleTables = 64;
constexpr size_t kIdleTableBytes = size_t{16} << 20;

struct TableEntry {
  int32_t* ptr = nullptr;
  size_t bytes = 0;
  int refs = 0;             // live plans using the table
  uint64_t released = 0;    // when the last plan let go of it (store clock), for eviction order
};

struct DeviceStore {
  std::mutex mu;
  std::map<std::array<int, 8>, TableEntry> tables;
  uint64_t clock = 0;
  std::vector<unsigned int*> free_words;
  std::vector<unsigned long long*> free_counters;
};

DeviceStore& device_store(int dev) {
  static DeviceStore stores[64];
  return stores[dev & 63];
}

// Free idle tables, least recently released first, until the idle ones fit the caps. Called with s.mu held and
// the store's device current.
void evict_idle_tables(DeviceStore& s) {
  for (;;) {
    size_t idle = 0, idle_bytes = 0;
    auto oldest = s.tables.end();
    for (auto it = s.tables.begin(); it != s.tables.end(); ++it) {
      if (it->second.refs > 0) continue;
      ++idle;
      idle_bytes += it->second.bytes;
      if (oldest == s.tables.end() || it->second.released < oldest->second.released) oldest = it;
    }
    if (idle <= kIdleTables && idle_bytes <= kIdleTableBytes) return;
    cudaFree(oldest->second.ptr);   // waits for work in flight, which may still read it
    s.tables.erase(oldest);
  }
}

// The device copy of schedule `key` (uploaded from `host` on first use), with one more reference on it.
int32_t acquire_table(int dev, const std::array<int, 8>& key, const std::vector<int32_t>& host, int32_t** out) {
  DeviceStore& s = device_store(dev);
  std::lock_guard<std::mutex> lock(s.mu);
  auto it = s.tables.find(key);
  if (it != s.tables.end()) {
    ++it->second.refs;
    *out = it->second.ptr;
    return 0;
  }
  int32_t* d = nullptr;
  const size_t bytes = host.size() * sizeof(int32_t);
  cudaError_t e = cudaMalloc(&d, bytes);
  if (e != cudaSuccess) return cuda_fail(e, "cudaMalloc(tile table)");
  e = cudaMemcpy(d, host.data(), bytes, cudaMemcpyHostToDevice);
  if (e != cudaSuccess) {
    cudaFree(d);
    return cuda_fail(e, "cudaMemcpy(tile table)");
  }
  TableEntry entry;
  entry.ptr = d;
  entry.bytes = bytes;
  entry.refs = 1;
  s.tables.emplace(key, entry);
  *out = d;
  return 0;
}

// Drop one reference on schedule `key`'s table; idle tables beyond the caps are freed.
void release_table(int dev, const std::array<int, 8>& key) {
  DeviceStore& s = device_store(dev);
  std::lock_guard<std::mutex> lock(s.mu);
  auto it = s.tables.find(key);
  if (it == s.tables.end()) return;
  if (--it->second.refs <= 0) {
    it->second.refs = 0;
    it->second.released = ++s.clock;
    evict_idle_tables(s);
  }
}

int32_t take_error_word(int dev, unsigned int** out) {
  DeviceStore& s = device_store(dev);
  std::lock_guard<std::mutex> lock(s.mu);
  if (s.free_words.empty()) {
    constexpr int kWords = 1024;
    unsigned int* slab = nullptr;
    cudaError_t e = cudaMalloc(&slab, kWords * sizeof(unsigned int));
    if (e != cudaSuccess) return cuda_fail(e, "cudaMalloc(error words)");
    for (int i = kWords - 1; i >= 0; --i) s.free_words.push_back(slab + i);
  }
  unsigned int* w = s.free_words.back();
  cudaError_t e = cudaMemset(w, 0, sizeof(unsigned int));
  if (e != cudaSuccess) return cuda_fail(e, "cudaMemset(error word)");
  s.free_words.pop_back();
  *out = w;
  return 0;
}

// A zeroed 64-bit counter (the wave barrier's), handed out from 4 KiB slabs like the error words.
int32_t take_counter(int dev, unsigned long long** out) {
  DeviceStore& s = device_store(dev);
  std::lock_guard<std::mutex> lock(s.mu);
  if (s.free_counters.empty()) {
    constexpr int kCounters = 512;
    unsigned long long* slab = nullptr;
    cudaError_t e = cudaMalloc(&slab, kCounters * sizeof(unsigned long long));
    if (e != cudaSuccess) return cuda_fail(e, "cudaMalloc(wave counters)");
    for (int i = kCounters - 1; i >= 0; --i) s.free_counters.push_back(slab + i);
  }
  unsigned long long* c = s.free_counters.back();
  cudaError_t e = cudaMemset(c, 0, sizeof(unsigned long long));
  if (e != cudaSuccess) return cuda_fail(e, "cudaMemset(wave counter)");
  s.free_counters.pop_back();
  *out = c;
  return 0;
}

void free_plan(bg_plan* p) {
  if (p == nullptr) return;
  if (p->d_partial || p->d_tickets || p->holds_table) {
    DeviceGuard guard(p->device);
    if (p->d_partial) cudaFree(p->d_partial);
    if (p->d_tickets) cudaFree(p->d_tickets);
    if (p->holds_table) release_table(p->device, p->table_key);
  }
  if (p->d_err || p->d_wave) {
    DeviceStore& s = device_store(p->device);
    std::lock_guard<std::mutex> lock(s.mu);
    if (p->d_err) s.free_words.push_back(p->d_err);
    if (p->d_wave) s.free_counters.push_back(p->d_wave);
  }
  delete p;
}

}  // namespace

extern "C" {

const char* bg_last_error(void) { return g_err; }

int32_t bg_version(void) { return 100; }

int32_t bg_device_info(int32_t device, int32_t* sm_count, int32_t* smem_optin, int32_t* cc_major, int32_t* cc_minor) {
  int v = 0;
  cudaError_t e;
  if ((e = cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, device)) != cudaSuccess)
    return cuda_fail(e, "cudaDeviceGetAttribute(MultiProcessorCount)");
  if (sm_count) *sm_count = v;
  if ((e = cudaDeviceGetAttribute(&v, cudaDevAttrMaxSharedMemoryPerBlockOptin, device)) != cudaSuccess)
    return cuda_fail(e, "cudaDeviceGetAttribute(MaxSharedMemoryPerBlockOptin)");
  if (smem_optin) *smem_optin = v;
  if ((e = cudaDeviceGetAttribute(&v, cudaDevAttrComputeCapabilityMajor, device)) != cudaSuccess)
    return cuda_fail(e, "cudaDeviceGetAttribute(ComputeCapabilityMajor)");
  if (cc_major) *cc_major = v;
  if ((e = cudaDeviceGetAttribute(&v, cudaDevAttrComputeCapabilityMinor, device)) != cudaSuccess)
    return cuda_fail(e, "cudaDeviceGetAttribute(ComputeCapabilityMinor)");
  if (cc_minor) *cc_minor = v;
  return 0;
}

int32_t bg_hilbert_order(int32_t m_tiles, int32_t n_tiles, int32_t* out, int32_t capacity) {
  if (m_tiles <= 0 || n_tiles <= 0 || m_tiles > 0xFFFF || n_tiles > 0xFFFF)
    return fail(-1, "tile grid %d x %d out of range", m_tiles, n_tiles);
  std::vector<int32_t> v;
  hilbert_order(m_tiles, n_tiles, v);
  if (static_cast<int64_t>(v.size()) > capacity) return fail(-2, "capacity %d < %zu entries", capacity, v.size());
  std::copy(v.begin(), v.end(), out);
  return static_cast<int32_t>(v.size());
}

int32_t bg_grouped_order(int32_t m_tiles, int32_t n_tiles, int32_t group_m, int32_t group_n, int32_t* out,
                         int32_t capacity) {
  if (m_tiles <= 0 || n_tiles <= 0 || m_tiles > 0xFFFF || n_tiles > 0xFFFF)
    return fail(-1, "tile grid %d x %d out of range", m_tiles, n_tiles);
  if (group_m < 1 || group_n < 1 || group_m > m_tiles || group_n > n_tiles)
    return fail(-1, "group %d x %d must be within the tile grid %d x %d", group_m, group_n, m_tiles, n_tiles);
  std::vector<int32_t> v;
  grouped_order(m_tiles, n_tiles, group_m, group_n, v);
  if (static_cast<int64_t>(v.size()) > capacity) return fail(-2, "capacity %d < %zu entries", capacity, v.size());
  std::copy(v.begin(), v.end(), out);
  return static_cast<int32_t>(v.size());
}

int32_t bg_encode_tensor_map_3d(void* out128, const void* base, int64_t height, int64_t width, int32_t box_h,
                                int32_t box_w) {
  // tensor_map.py:14-17: positive sizes; tile and width multiples of 64 elements.
  if (box_h <= 0 || box_w <= 0 || height <= 0 || width <= 0) return fail(-1, "tensor-map dimensions must be positive");
  if (box_w % 64 || width % 64) return fail(-1, "tensor-map tile and width must be multiples of 64 bf16 elements");
  if (out128 == nullptr || base == nullptr) return fail(-1, "null pointer");
  auto fn = encode_fn();
  if (fn == nullptr) return fail(2, "cuTensorMapEncodeTiled is unavailable (no CUDA driver)");
  const cuuint64_t dims[3] = {64, static_cast<cuuint64_t>(height), static_cast<cuuint64_t>(width / 64)};
  const cuuint64_t strides[2] = {static_cast<cuuint64_t>(2 * width), 128};
  const cuuint32_t box[3] = {64, static_cast<cuuint32_t>(box_h), static_cast<cuuint32_t>(box_w / 64)};
  const cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = fn(reinterpret_cast<CUtensorMap*>(out128), CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(base),
                  dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                  CU_TENSOR_MAP_L2_PROMOTION_NONE, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(3, "cuTensorMapEncodeTiled failed with CUresult %d", static_cast<int>(r));
  return 0;
}

}  // extern "C"

namespace {

// Everything a plan needs except device memory: validation of the knobs and the shape contract, shared-memory and
// tensor-memory sizing, kernel choice and launch attributes, tensor maps, and the host-side tile table (returned in
// `sched` with its cache key; empty for the non-persistent kernels). Runs with `device` current. Fills p->kp except
// its `sched` and `err` pointers, which the caller points at device memory of its own.
int32_t setup_plan(const bg_cfg& c, int64_t M, int64_t N, int64_t K, const void* A, int64_t lda, const void* BT,
                   int64_t ldb, void* C, int64_t ldc, int32_t device, bg_plan* p, std::vector<int32_t>& sched,
                   std::array<int, 8>& sched_key, bool validate_only = false) {
  // ---- knob validation (gemm.py:260-271, gated.py:27-32)
  if (c.kind != BG_KIND_WS && c.kind != BG_KIND_GATED && c.kind != BG_KIND_RING)
    return fail(-1, "unknown kernel kind %d", c.kind);
  if (c.BK != 64) return fail(-1, "BK must be 64 (one 128-byte swizzle atom)");
  if (c.BN <= 0 || c.BN % 16 || c.BN > 256) return fail(-1, "BN must be a multiple of 16 in (0, 256]");
  if (c.tma_store && c.BN % 64) return fail(-1, "tma_store needs BN to be a multiple of 64");
  if (c.stages != 0 && c.stages < 2) return fail(-1, "stages must be at least 2");
  if (c.kind == BG_KIND_RING ? c.consumers != 0 : (c.consumers != 1 && c.consumers != 2))
    return fail(-1, c.kind == BG_KIND_RING ? "the ring kernel has consumers == 0" : "consumers must be 1 or 2");
  if (c.cluster != 1 && c.cluster != 2) return fail(-1, "cluster must be 1 or 2");
  if (c.kind != BG_KIND_WS && (c.cluster != 1 || c.hilbert || c.tma_store))
    return fail(-1, "cluster, hilbert and tma_store need the persistent kernel");
  if (c.num_sm > 0 && c.num_sm < c.cluster) return fail(-1, "num_sm must be at least the cluster size");
  if (c.group_m < 1 || c.group_n < 1) return fail(-1, "group_m and group_n must be positive");
  if (c.acc_bufs < 0 || c.acc_bufs > 2) return fail(-1, "acc_bufs must be 0 (auto), 1 or 2");
  // split_k: -1 = choose below, once the cluster count is known; 0 or 1 = off
  if (c.split_k < -1 || c.split_k > 64) return fail(-1, "split_k must be -1 (auto) or in [0, 64]");
  const bool sk_auto = c.split_k == -1;
  int sk = c.split_k <= 1 ? 1 : c.split_k;
  if (sk > 1 && c.kind != BG_KIND_WS) return fail(-1, "split_k needs the persistent kernel");
  const bool nmajor = c.b_nmajor != 0;
  if (c.b_nmajor != 0 && c.b_nmajor != 1) return fail(-1, "b_nmajor must be 0 or 1");
  if (nmajor && c.kind != BG_KIND_WS) return fail(-1, "b_nmajor needs the warp-specialized kernel");
  if (c.wave_sync < 0 || c.wave_sync > 2) return fail(-1, "wave_sync must be 0 (auto), 1 (on) or 2 (off)");
  if (c.wave_sync == 1 && (c.kind != BG_KIND_WS || sk > 1))
    return fail(-1, "wave_sync needs the persistent kernel without split-K");
  if (c.split_k_cluster < 0 || c.split_k_cluster > 2)
    return fail(-1, "split_k_cluster must be 0 (auto), 1 (inside a cluster) or 2 (through the workspace)");

  const int bm = 64 * std::max(c.consumers, 1);
  const int cl = c.cluster;
  const bool paired = c.kind == BG_KIND_WS && cl == 2 && bm == 128;
  const int bn = c.BN;
  const int nblk = c.n_mma == 0 ? 1 : c.n_mma;
  if (nblk < 1 || nblk > 2 || (nblk > 1 && c.kind != BG_KIND_WS)) return fail(-1, "n_mma must be 1 or 2 (persistent kernel)");
  const int width = bn * nblk;   // output columns per tile
  const int bn_local = paired ? bn / 2 : bn;
  // N-major B arrives in 64-column boxes: every CTA's share of an N block must be whole boxes
  if (nmajor && bn_local % 64)
    return fail(-1, "b_nmajor needs %s a multiple of 64 columns (got %d)", paired ? "BN / 2" : "BN", bn_local);

  // ---- shape contract (gemm.py:300-311)
  if (M <= 0 || N <= 0 || K <= 0) return fail(-1, "M, N and K must be positive");
  const bool ragged = c.ragged != 0;
  if (ragged && c.kind != BG_KIND_WS) return fail(-1, "ragged shapes need the persistent kernel");
  if (!ragged && (M % bm || N % width || K % 64))
    return fail(-1, "shape %lldx%lldx%lld not a multiple of tile %dx%dx64", (long long)M, (long long)N, (long long)K, bm,
                width);
  if (ragged && (N % 8 || K % 8))
    return fail(-1, "ragged shapes need N and K to be multiples of 8 (16-byte rows), got N=%lld K=%lld", (long long)N,
                (long long)K);
  // Ragged shapes round the tile grid up: TMA loads zero-fill what lies beyond A, BT and K, the TMA store clips
  // and the register epilogue masks what lies beyond C; a pair's second row tile may lie wholly outside A.
  int64_t mt = (M + bm - 1) / bm;
  const int64_t nt = (N + width - 1) / width, nkb = (K + 63) / 64;
  if (ragged) mt = (mt + cl - 1) / cl * cl;
  if (mt % cl) return fail(-1, "%lld row tiles not divisible by cluster %d", (long long)mt, cl);
  const int64_t cmt = mt / cl;
  if (cmt > 0xFFFF || nt > 0xFFFF || cmt * nt * sk > (1ll << 30) || nkb * sk > (1ll << 30))
    return fail(-1, "problem too large for the tile table");
  if (sk > 1 && sk > nkb) return fail(-1, "split_k %d exceeds the %lld k-blocks of K", sk, (long long)nkb);
  if (sk > 1 && width % 32) return fail(-1, "split_k needs tiles a multiple of 32 columns wide (got %d)", width);
  if (A == nullptr || BT == nullptr || C == nullptr) return fail(-1, "null operand pointer");
  if ((reinterpret_cast<uintptr_t>(A) | reinterpret_cast<uintptr_t>(BT) | reinterpret_cast<uintptr_t>(C)) & 15)
    return fail(-1, "operand pointers must be 16-byte aligned");
  if (lda < K || ldb < (nmajor ? N : K) || ldc < N || lda % 8 || ldb % 8 || ldc % 8)
    return fail(-1, "row pitches must cover the row and be multiples of 8 elements (lda=%lld ldb=%lld ldc=%lld)",
                (long long)lda, (long long)ldb, (long long)ldc);

  if (validate_only) return 0;   // the argument checks above touch no device

  int sm_count = 0, smem_optin = 0, ccmaj = 0, ccmin = 0;
  int32_t st = bg_device_info(device, &sm_count, &smem_optin, &ccmaj, &ccmin);
  if (st) return st;
  if (ccmaj != 10) return fail(4, "device %d is sm_%d%d; this library is built for sm_100a", device, ccmaj, ccmin);

  // ---- shared memory: [A stages][B stages][C staging][barriers], +1024 bytes to align the base
  const uint32_t a_stage = static_cast<uint32_t>(bm) * 128u;
  const uint32_t b_block = static_cast<uint32_t>(bn_local) * 128u;
  const uint32_t b_stage = b_block * static_cast<uint32_t>(nblk);
  const uint32_t c_bytes = c.tma_store ? static_cast<uint32_t>(bm) * 256u : 0u;
  const uint32_t fixed = 1024u + c_bytes + (c.kind == BG_KIND_RING ? 16u : 56u);
  int stages = c.stages;
  if (stages == 0) {
    const int64_t fit = (static_cast<int64_t>(smem_optin) - fixed) / (a_stage + b_stage + 16);
    stages = static_cast<int>(std::min<int64_t>(fit, 8));
    if (stages < 2) return fail(-1, "not even 2 stages fit in %d bytes of shared memory", smem_optin);
  }
  size_t smem = fixed + static_cast<size_t>(stages) * (a_stage + b_stage + 16u);
  if (smem > static_cast<size_t>(smem_optin))
    return fail(-1, "needs %zu bytes of shared memory, the limit is %d", smem, smem_optin);

  // ---- accumulators in tensor memory
  int acc_bufs = c.acc_bufs;
  if (c.kind != BG_KIND_WS) acc_bufs = 1;
  if (acc_bufs == 0) acc_bufs = 2 * width <= 512 ? 2 : 1;
  if (acc_bufs * width > 512) return fail(-1, "%d accumulators of %d columns exceed tensor memory", acc_bufs, width);

  p->device = device;
  p->kind = c.kind;
  p->bm = bm;
  p->paired = paired;
  p->tma_store = c.tma_store != 0;
  p->cl = cl;
  p->smem = smem;
  p->threads = c.kind == BG_KIND_RING ? sm100::kRingThreads : sm100::kWsThreads;

  // ---- schedule
  const int64_t tiles = cmt * nt;
  int64_t nclusters = tiles;
  sched.clear();
  if (c.kind == BG_KIND_WS) {
    const int num_sm = c.num_sm > 0 ? c.num_sm : sm_count;
    nclusters = num_sm / cl;   // clusters available; the grid is cut to the schedule's entries below
    if (c.hilbert) {
      sched_key = {device, 1, static_cast<int>(cmt), static_cast<int>(nt), 0, 0, 0, 0};
      hilbert_order(static_cast<int>(cmt), static_cast<int>(nt), sched);
    } else {
      const int gm = std::min<int>(std::max(c.group_m / cl, 1), static_cast<int>(cmt));
      const int gn = std::min<int>(c.group_n, static_cast<int>(nt));
      sched_key = {device, 0, static_cast<int>(cmt), static_cast<int>(nt), gm, gn, 0, 0};
      grouped_order(static_cast<int>(cmt), static_cast<int>(nt), gm, gn, sched);
    }
  }

  // ---- automatic split-K: the most splits that still fit the tiles in one wave of clusters
  // (num_sm / cluster of them), each split keeping at least kAutoSplitMinKb k-blocks (below that the partial-sum
  // round trip costs more than the split saves), or kAutoSplitMinKbCluster where the splits can meet inside a
  // cluster (single-CTA tiles, 2 or 4 splits, each split's share of the columns whole 64- or 32-column chunks):
  // CUDA events, L2 flushed, 128x128 tiles with 2 splits inside a cluster against none: 16 k-blocks per split
  // even (1024x1024x2048, 512x512x2048), 24 per split 10 % faster (1024x1024x3072)
  if (sk_auto && c.kind == BG_KIND_WS && width % 32 == 0) {
    constexpr int kAutoSplitMinKb = 32, kAutoSplitMinKbCluster = 24, kAutoSplitMax = 16;
    const int num_sm = c.num_sm > 0 ? c.num_sm : sm_count;
    for (int s2 = 2; s2 <= kAutoSplitMax; ++s2) {
      const bool in_cluster = c.split_k_cluster != 2 && cl == 1 && nblk == 1 && (s2 == 2 || s2 == 4) &&
                              width % s2 == 0 && (width / s2) % (c.tma_store ? 64 : 32) == 0 && tiles * s2 <= num_sm;
      const int min_kb = in_cluster ? kAutoSplitMinKbCluster : kAutoSplitMinKb;
      if (tiles * s2 <= nclusters && nkb >= static_cast<int64_t>(min_kb) * s2 && nkb * s2 <= (1ll << 30)) sk = s2;
    }
  }

  // ---- kernel and launch attributes
  const void* fn = nullptr;
  if (c.kind == BG_KIND_RING) {
    p->ring = pick_ring(bm);
    fn = reinterpret_cast<const void*>(p->ring);
  } else {
    p->ws = pick_ws(bm, paired, p->tma_store, nblk, sk > 1 ? sm100::kSplitWorkspace : sm100::kSplitNone);
    fn = reinterpret_cast<const void*>(p->ws);
  }
  cudaError_t e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, smem_optin);
  if (e != cudaSuccess) return cuda_fail(e, "cudaFuncSetAttribute(MaxDynamicSharedMemorySize)");

  // ---- split-K inside a cluster (bg_cfg.split_k_cluster): the sk CTAs of one cluster share each tile and reduce
  // through distributed shared memory, each receiving (sk - 1) x 128 x (width / sk) fp32 sums (the 4 epilogue
  // warps' 32 tensor-memory lanes each, also when BM = 64 leaves half of them unused)
  int kc = 1;
  uint32_t recv_bytes = 0;
  if (sk > 1 && c.split_k_cluster != 2) {
    char why[160] = "";
    const int share = width % sk == 0 ? width / sk : 0;
    const int num_sm = c.num_sm > 0 ? c.num_sm : sm_count;
    int kc_stages = stages;
    size_t kc_smem = 0;
    WsKernel kc_fn = nullptr;
    if (cl != 1 || nblk != 1) {
      snprintf(why, sizeof(why), "single-CTA tiles (cluster 1, n_mma 1)");
    } else if (sk != 2 && sk != 4) {
      snprintf(why, sizeof(why), "split_k 2 or 4 (got %d)", sk);
    } else if (share == 0 || share % (c.tma_store ? 64 : 32)) {
      snprintf(why, sizeof(why), "each split's share of the %d tile columns a multiple of %d", width,
               c.tma_store ? 64 : 32);
    } else if (tiles * sk > num_sm) {
      snprintf(why, sizeof(why), "every tile on its own cluster at once (%lld tiles x %d splits > %d SMs)",
               (long long)tiles, sk, num_sm);
    } else {
      recv_bytes = static_cast<uint32_t>(sk - 1) * 128u * static_cast<uint32_t>(share) * 4u;
      if (c.stages == 0) {
        const int64_t fit = (static_cast<int64_t>(smem_optin) - fixed - recv_bytes) / (a_stage + b_stage + 16);
        kc_stages = static_cast<int>(std::min<int64_t>(fit, 8));
      }
      kc_smem = fixed + recv_bytes + static_cast<size_t>(kc_stages) * (a_stage + b_stage + 16u);
      kc_fn = pick_ws(bm, paired, p->tma_store, nblk, sm100::kSplitCluster);
      if (kc_stages < 2 || kc_smem > static_cast<size_t>(smem_optin)) {
        snprintf(why, sizeof(why), "room for %u bytes of received sums beside the ring", recv_bytes);
      } else {
        e = cudaFuncSetAttribute(reinterpret_cast<const void*>(kc_fn), cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 smem_optin);
        if (e != cudaSuccess) return cuda_fail(e, "cudaFuncSetAttribute(MaxDynamicSharedMemorySize)");
        cudaLaunchConfig_t lc = {};
        lc.gridDim = dim3(static_cast<unsigned>(sk * tiles));
        lc.blockDim = dim3(p->threads);
        lc.dynamicSmemBytes = kc_smem;
        cudaLaunchAttribute at[1];
        at[0].id = cudaLaunchAttributeClusterDimension;
        at[0].val.clusterDim.x = sk;
        at[0].val.clusterDim.y = 1;
        at[0].val.clusterDim.z = 1;
        lc.attrs = at;
        lc.numAttrs = 1;
        int maxc = 0;
        e = cudaOccupancyMaxActiveClusters(&maxc, reinterpret_cast<const void*>(kc_fn), &lc);
        if (e != cudaSuccess) return cuda_fail(e, "cudaOccupancyMaxActiveClusters");
        if (maxc < tiles)
          snprintf(why, sizeof(why), "every tile on its own cluster at once (%lld tiles, %d clusters of %d fit)",
                   (long long)tiles, maxc, sk);
      }
    }
    if (why[0] == '\0') {
      kc = sk;
      stages = kc_stages;
      smem = kc_smem;
      p->ws = kc_fn;
      fn = reinterpret_cast<const void*>(kc_fn);
    } else {
      recv_bytes = 0;
      if (c.split_k_cluster == 1) return fail(-1, "split_k_cluster = 1 needs %s", why);
    }
  }
  p->kc = kc;
  // Tensor memory is 512 columns per SM. CTAs that could share an SM must fit in it together, or a CTA would block
  // in tcgen05.alloc behind another (and CTA pairs waiting on each other could deadlock). Pad the shared-memory
  // request until the occupancy limit keeps co-resident CTAs within the SM's tensor memory.
  {
    const int tcols = static_cast<int>(pow2_cols(acc_bufs * width));
    const int allowed = 512 / tcols;
    for (;;) {
      int blocks = 0;
      e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&blocks, fn, p->threads, smem);
      if (e != cudaSuccess) return cuda_fail(e, "cudaOccupancyMaxActiveBlocksPerMultiprocessor");
      if (blocks <= allowed) break;
      if (smem >= static_cast<size_t>(smem_optin))
        return fail(5, "cannot limit residency to %d CTAs per SM for %d TMEM columns", allowed, tcols);
      smem = std::min<size_t>(smem + 8192, static_cast<size_t>(smem_optin));
    }
    p->smem = smem;
  }
  const int lcl = cl * kc;   // CTAs per launched cluster
  if (kc > 1) nclusters = (c.num_sm > 0 ? c.num_sm : sm_count) / lcl;
  if (lcl > 1) {
    // Persistent clusters must all be resident at once: cap their number at what the GPU can co-schedule.
    cudaLaunchConfig_t lc = {};
    lc.gridDim = dim3(static_cast<unsigned>(lcl * nclusters));
    lc.blockDim = dim3(p->threads);
    lc.dynamicSmemBytes = smem;
    cudaLaunchAttribute at[1];
    at[0].id = cudaLaunchAttributeClusterDimension;
    at[0].val.clusterDim.x = lcl;
    at[0].val.clusterDim.y = 1;
    at[0].val.clusterDim.z = 1;
    lc.attrs = at;
    lc.numAttrs = 1;
    int maxc = 0;
    e = cudaOccupancyMaxActiveClusters(&maxc, fn, &lc);
    if (e != cudaSuccess) return cuda_fail(e, "cudaOccupancyMaxActiveClusters");
    if (maxc <= 0) return fail(5, "no cluster of %d CTAs with %zu bytes of shared memory fits on the device", lcl, smem);
    p->max_active_clusters = maxc;
    if (c.kind == BG_KIND_WS) nclusters = std::min<int64_t>(nclusters, maxc);
  }
  // split-K inside a cluster runs exactly one tile per cluster (its receive barrier serves one phase)
  if (kc > 1 && nclusters < tiles)
    return fail(5, "split-K inside a cluster: %lld tiles but only %lld clusters of %d fit", (long long)tiles,
                (long long)nclusters, lcl);
  // ---- wave-quantization tail: the last, partial wave of the persistent schedule (entries [full, tiles) of the
  // dealt table) is split into half-width tiles when twice its size still fits in one wave, so that the tail takes
  // about half a tile's time instead of a whole one. Half width = one N block when nblk == 2, MMA N = BN/2 otherwise.
  const int half = nblk == 2 ? bn : bn / 2;
  const bool narrow_ok = nblk == 2 || (half % 16 == 0 && (!c.tma_store || half % 64 == 0) &&
                                       (!nmajor || (paired ? half / 2 : half) % 64 == 0));
  int64_t n_entries = tiles;
  if (c.kind == BG_KIND_WS && !c.no_tail_split && sk == 1 && narrow_ok && !sched.empty()) {
    const int64_t full = (tiles / nclusters) * nclusters;
    const int64_t tail = tiles - full;
    if (tail > 0 && 2 * tail <= nclusters) {
      std::vector<int32_t> split(sched.begin(), sched.begin() + full);
      for (int64_t i = full; i < tiles; ++i) {
        const int32_t cmi = sched[i] >> 16, tni = sched[i] & 0xFFFF;
        split.push_back((cmi << 16) | sm100::kNarrowTile | (2 * tni));
        split.push_back((cmi << 16) | sm100::kNarrowTile | (2 * tni + 1));
      }
      sched.swap(split);
      n_entries = static_cast<int64_t>(sched.size());
      p->narrow_tiles = static_cast<int>(2 * tail);
      sched_key[6] = static_cast<int>(nclusters);
      sched_key[7] = 1;
    }
  }
  if (nt * 2 > 0x7FFF) return fail(-1, "too many column tiles (%lld) for the tile table", (long long)nt);
  // ---- split-K through the workspace: every tile becomes sk consecutive entries (split s = entry % sk), dealt to
  // consecutive clusters. (Inside a cluster, each tile keeps one entry: its cluster's ranks are the splits.)
  if (sk > 1 && kc == 1) {
    std::vector<int32_t> ext;
    ext.reserve(sched.size() * sk);
    for (int32_t e : sched)
      for (int s = 0; s < sk; ++s) ext.push_back(e);
    sched.swap(ext);
    n_entries = static_cast<int64_t>(sched.size());
    sched_key[1] |= sk << 1;
    p->partial_bytes = static_cast<size_t>(n_entries) * cl * 4u * 32u * static_cast<size_t>(width) * sizeof(float);
    p->ticket_words = static_cast<size_t>(tiles) * cl * 4u;
  }
  // one entry per cluster: the tile's entries are all resident together (cooperative launch) and share the reduce
  const bool sk_scatter = sk > 1 && kc == 1 && n_entries <= nclusters;
  nclusters = std::min<int64_t>(nclusters, n_entries);
  p->grid = static_cast<int>(nclusters * (c.kind == BG_KIND_RING ? 1 : lcl));

  // ---- tensor maps: A[M,K] box (64, BM); BT[N,K] box (64, bn_local), or B[K,N] box (64, 64) when N-major;
  // C[M,N] box (64, BM/4) per epilogue warp
  if ((st = encode_2d(&p->tmA, A, K, M, lda, 64, bm, "A"))) return st;
  if (nmajor) {
    // 64-column x 64-row boxes (one 128-byte swizzle row of N per K row) serve full and half-width tiles alike
    if ((st = encode_2d(&p->tmB, BT, N, K, ldb, 64, 64, "B (N-major)"))) return st;
    p->tmBn = p->tmB;
  } else {
    if ((st = encode_2d(&p->tmB, BT, K, N, ldb, 64, bn_local, "BT"))) return st;
    if (nblk == 1 && p->narrow_tiles > 0) {
      if ((st = encode_2d(&p->tmBn, BT, K, N, ldb, 64, bn_local / 2, "BT half tiles"))) return st;
    } else {
      p->tmBn = p->tmB;
    }
  }
  if (p->tma_store) {
    if ((st = encode_2d(&p->tmC, C, N, M, ldc, 64, bm / 4, "C"))) return st;
  } else {
    p->tmC = p->tmA;   // unused by the register epilogue
  }

  // ---- wave barrier: on request, or automatically when (a) each cluster runs at least kAutoWaveSyncTiles tiles (the
  // drift the barrier removes builds up over a cluster's tiles) and (b) one wave's operand panels are too big to stay
  // in L2 between the reads of the tiles that share them: a wave of n cluster tiles (rows x cols, each tile BMp x W,
  // rows * cols = n) touches K-long panels of at least 2 * K * 2 * sqrt(n * BMp * W) bytes (the square-ish wave;
  // AM-GM). Measured under Nsight Compute: 256x512 pair tiles gain 1.4 % at 8192^3 (a 102 MB wave), 3.6 % at
  // 12288^3 and 7 % at 16384^3 and are even at 6144^3 (77 MB); 256x256 pair tiles lose 2 % at 4096^3 (36 MB), where
  // the waits cost more than the barrier saves.
  constexpr int64_t kAutoWaveSyncTiles = 4;
  constexpr double kAutoWaveSyncBytes = 96e6;   // about three quarters of the 126 MB L2
  const bool wave_ok = c.kind == BG_KIND_WS && sk == 1 && n_entries > nclusters;
  const double wave_bytes =
      4.0 * static_cast<double>(K) *
      std::sqrt(static_cast<double>(std::min<int64_t>(nclusters, n_entries)) * bm * cl * static_cast<double>(width));
  const bool wave_auto = n_entries >= kAutoWaveSyncTiles * nclusters && wave_bytes >= kAutoWaveSyncBytes;
  const bool wave = wave_ok && (c.wave_sync == 1 || (c.wave_sync == 0 && wave_auto));
  p->wave_per_launch = 0;
  if (wave) {
    for (int64_t j = 1; j * nclusters < n_entries; ++j)
      p->wave_per_launch += static_cast<unsigned long long>(std::min<int64_t>(nclusters, n_entries - j * nclusters)) *
                            static_cast<unsigned long long>(cl);
  }

  GemmParams& kp = p->kp;
  kp.num_kb = static_cast<int>(nkb);
  kp.bn = bn;
  kp.nblk = nblk;
  kp.bn_local = bn_local;
  kp.stages = stages;
  kp.tiles = static_cast<int>(n_entries);
  kp.nclusters = static_cast<int>(nclusters);
  kp.cl = c.kind == BG_KIND_RING ? 1 : cl;
  kp.nt = static_cast<int>(nt);
  kp.acc_bufs = acc_bufs;
  kp.acc_stride = width;
  kp.tmem_cols = pow2_cols(acc_bufs * width);
  const uint32_t b_mn = nmajor ? kIdescBMajorMN : 0u;
  kp.idesc = make_idesc(paired ? 2 * bm : bm, bn) | b_mn;
  kp.tx_bytes = (a_stage + b_stage) * (paired ? 2u : 1u);
  kp.tx_narrow = (a_stage + (nblk == 2 ? b_block : b_block / 2)) * (paired ? 2u : 1u);
  kp.idesc_narrow = make_idesc(paired ? 2 * bm : bm, nblk == 2 ? bn : bn / 2) | b_mn;
  kp.a_stage_bytes = a_stage;
  kp.b_block_bytes = b_block;
  kp.b_stage_bytes = b_stage;
  kp.sched = nullptr;
  kp.C = static_cast<__nv_bfloat16*>(C);
  kp.ldc = ldc;
  kp.m_valid = static_cast<int>(M);
  kp.n_valid = static_cast<int>(N);
  kp.err = nullptr;
  kp.budget_ns = c.wait_budget_ns > 0 ? static_cast<unsigned long long>(c.wait_budget_ns) : 4000000000ull;
  kp.skip_job = c.debug_skip_job;
  kp.split_k = sk;
  kp.partial = nullptr;
  kp.tickets = nullptr;
  kp.sk_scatter = sk_scatter ? 1 : 0;
  kp.k_serpentine = c.no_k_serpentine ? 0 : 1;
  kp.b_nmajor = nmajor ? 1 : 0;
  kp.wave_sync = wave ? 1 : 0;
  kp.wave_ctr = nullptr;
  kp.wave_base = 0;
  kp.wave_wait_ns = 200000;   // 200 us: a boundary's natural spread is a few us (a few % of one tile)
  kp.kc = kc;
  kp.kc_recv_bytes = recv_bytes;
  // A cooperative launch guarantees that every CTA is resident at once. It cannot be combined with cluster
  // dimensions here (such a launch fails under Nsight Compute), so CTA pairs rely on the persistent grid being
  // capped at what the GPU co-schedules, with the bounded wait reporting an error if other work holds SMs.
  p->cooperative = sk_scatter && cl == 1;
  // split accumulator (two N blocks, one 512-column buffer): how many k-blocks run on half 0 alone at a tile's start
  // and end; it must stay below the ring depth so the producer keeps a free stage
  kp.look = std::max(1, std::min(2, stages - 2));
  // the first wave of the tile table also travels in the kernel parameters (see FirstTile in the kernel)
  for (size_t i = 0; i < sched.size() && i < static_cast<size_t>(sm100::kFirstWave); ++i) kp.first_wave[i] = sched[i];

  snprintf(p->name, sizeof(p->name), "%s<BM=%d,%s,%s> BN=%dx%d stages=%d acc=%d tail=%d splitk=%d%s%s b=%s",
           c.kind == BG_KIND_RING ? "sm100_gemm_ring" : "sm100_gemm_ws", bm,
           paired ? "pair" : (cl == 2 ? "cluster2" : "cta"), p->tma_store ? "tma_store" : "reg_store", bn, nblk,
           stages, acc_bufs, p->narrow_tiles, sk, kc > 1 ? "/cluster" : "", wave ? " wavesync" : "",
           nmajor ? "N" : "K");
  return 0;
}

}  // namespace

extern "C" {

int32_t bg_plan_create(bg_plan** out, const bg_cfg* cfg, int64_t M, int64_t N, int64_t K, const void* A, int64_t lda,
                       const void* BT, int64_t ldb, void* C, int64_t ldc, int32_t device) {
  if (out == nullptr || cfg == nullptr) return fail(-1, "null plan or cfg pointer");
  *out = nullptr;
  std::unique_ptr<bg_plan, void (*)(bg_plan*)> p(new bg_plan, free_plan);
  std::vector<int32_t> sched;
  std::array<int, 8> sched_key{};
  int32_t st = setup_plan(*cfg, M, N, K, A, lda, BT, ldb, C, ldc, device, p.get(), sched, sched_key, true);
  if (st) return st;
  DeviceGuard guard(device);
  if (guard.status != cudaSuccess) return cuda_fail(guard.status, "cudaSetDevice");
  st = setup_plan(*cfg, M, N, K, A, lda, BT, ldb, C, ldc, device, p.get(), sched, sched_key);
  if (st) return st;
  // ---- device buffers: tile table (cached per schedule) and error word (from the device's slab)
  if (!sched.empty()) {
    if ((st = acquire_table(device, sched_key, sched, &p->d_sched))) return st;
    p->holds_table = true;
    p->table_key = sched_key;
  }
  if ((st = take_error_word(device, &p->d_err))) return st;
  if (p->kp.wave_sync && (st = take_counter(device, &p->d_wave))) return st;
  if (p->partial_bytes > 0) {
    // split-K workspace: partial sums (fully written before they are read) and zeroed arrival words
    cudaError_t e = cudaMalloc(&p->d_partial, p->partial_bytes);
    if (e != cudaSuccess) return cuda_fail(e, "cudaMalloc(split-K partial sums)");
    if ((e = cudaMalloc(&p->d_tickets, p->ticket_words * sizeof(unsigned int))) != cudaSuccess)
      return cuda_fail(e, "cudaMalloc(split-K arrival words)");
    if ((e = cudaMemset(p->d_tickets, 0, p->ticket_words * sizeof(unsigned int))) != cudaSuccess)
      return cuda_fail(e, "cudaMemset(split-K arrival words)");
  }
  p->kp.sched = p->d_sched;
  p->kp.err = p->d_err;
  p->kp.wave_ctr = p->d_wave;
  p->kp.partial = p->d_partial;
  p->kp.tickets = p->d_tickets;
  *out = p.release();
  return 0;
}


}  // extern "C"

// ---------------------------------------------------------------------------------------------------------------
// Allocation-free entry point (bg_gemm_noalloc)
// ---------------------------------------------------------------------------------------------------------------
namespace {

// Scratch of bg_gemm_noalloc: the persistent kernel's tile table (kNoAllocMaxTiles int32 entries) followed by its
// error word. It is a file-scope device array, so every GPU that loads this library holds these 256 KiB + 256 bytes
// until the process exits, and no call allocates anything.
constexpr int kNoAllocMaxTiles = 65536;
constexpr int kNoAllocErrOffset = kNoAllocMaxTiles;   // int32 index of the error word
static __device__ __align__(256) int32_t g_noalloc_scratch[kNoAllocMaxTiles + 64];

// In host code g_noalloc_scratch names a host-side stand-in, not device memory: its device address is looked up
// with the device current, on the first call that succeeds in doing so, and handed to the kernel. A failed lookup
// is not remembered, so a later call tries again.
struct NoAllocScratch {
  std::mutex mu;
  int32_t* ptr = nullptr;
};

NoAllocScratch& noalloc_scratch(int dev) {
  static NoAllocScratch s[64];
  return s[dev & 63];
}

}  // namespace

extern "C" {

int32_t bg_gemm_noalloc(const bg_cfg* cfg, int64_t M, int64_t N, int64_t K, const void* A, int64_t lda,
                        const void* BT, int64_t ldb, void* C, int64_t ldc, int32_t device, void* stream,
                        uint32_t* err_word) {
  if (cfg == nullptr) return fail(-1, "null cfg pointer");
  if (device < 0 || device >= 64) return fail(-1, "device %d out of range", device);
  if (cfg->split_k > 1)
    return fail(-1, "bg_gemm_noalloc has no split-K workspace (split_k = %d); use bg_plan_create", cfg->split_k);
  // The automatic choice (split_k = -1) would split some shapes (few tiles, long K), and a split schedule needs a
  // workspace this entry point does not have: here those shapes run unsplit.
  bg_cfg c = *cfg;
  if (c.split_k == -1) c.split_k = 1;
  c.wave_sync = 2;   // the wave barrier needs a counter this entry point does not have
  bg_plan plan;   // lives on this stack frame and owns no device memory
  std::vector<int32_t> sched;
  std::array<int, 8> sched_key{};
  int32_t st = setup_plan(c, M, N, K, A, lda, BT, ldb, C, ldc, device, &plan, sched, sched_key, true);
  if (st) return st;
  DeviceGuard guard(device);
  if (guard.status != cudaSuccess) return cuda_fail(guard.status, "cudaSetDevice");
  st = setup_plan(c, M, N, K, A, lda, BT, ldb, C, ldc, device, &plan, sched, sched_key);
  if (st) return st;
  if (plan.kp.split_k > 1 || plan.partial_bytes > 0)   // never reached with split_k <= 1; kept as the guard
    return fail(-1, "bg_gemm_noalloc: the plan needs a split-K workspace; use bg_plan_create");
  if (sched.size() > static_cast<size_t>(kNoAllocMaxTiles))
    return fail(-1, "bg_gemm_noalloc: %zu tiles exceed its fixed scratch of %d tile entries; use bg_plan_create or "
                "wider tiles", sched.size(), kNoAllocMaxTiles);
  int32_t* scratch = nullptr;
  {
    NoAllocScratch& ns = noalloc_scratch(device);
    std::lock_guard<std::mutex> lock(ns.mu);
    if (ns.ptr == nullptr) {
      int32_t* ptr = nullptr;
      const cudaError_t e = cudaGetSymbolAddress(reinterpret_cast<void**>(&ptr), g_noalloc_scratch);
      if (e != cudaSuccess) return cuda_fail(e, "cudaGetSymbolAddress(g_noalloc_scratch)");
      ns.ptr = ptr;
    }
    scratch = ns.ptr;
  }
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  unsigned int* err = reinterpret_cast<unsigned int*>(scratch + kNoAllocErrOffset);
  cudaError_t e;
  if (!sched.empty()) {
    // Staged from host memory on the stream, ordered after the stream's earlier work; the host vector may go away
    // once cudaMemcpyAsync has returned.
    e = cudaMemcpyAsync(scratch, sched.data(), sched.size() * sizeof(int32_t), cudaMemcpyHostToDevice, s);
    if (e != cudaSuccess) return cuda_fail(e, "cudaMemcpyAsync(tile table)");
  }
  if ((e = cudaMemsetAsync(err, 0, sizeof(unsigned int), s)) != cudaSuccess) return cuda_fail(e, "cudaMemsetAsync");
  plan.kp.sched = sched.empty() ? nullptr : scratch;
  plan.kp.err = err;
  if ((st = bg_plan_launch(&plan, stream))) return st;
  if (err_word == nullptr) return 0;
  if ((e = cudaStreamSynchronize(s)) != cudaSuccess) return cuda_fail(e, "cudaStreamSynchronize");
  uint32_t w = 0;
  if ((e = cudaMemcpy(&w, err, sizeof(w), cudaMemcpyDeviceToHost)) != cudaSuccess)
    return cuda_fail(e, "cudaMemcpy(error word)");
  *err_word = w;
  if (w != 0) return fail(6, "device wait timed out (error word 0x%08x)", w);
  return 0;
}

int32_t bg_plan_launch(bg_plan* p, void* stream) {
  if (p == nullptr) return fail(-1, "null plan");
  DeviceGuard guard(p->device);
  if (guard.status != cudaSuccess) return cuda_fail(guard.status, "cudaSetDevice");
  cudaLaunchConfig_t lc = {};
  lc.gridDim = dim3(static_cast<unsigned>(p->grid));
  lc.blockDim = dim3(static_cast<unsigned>(p->threads));
  lc.dynamicSmemBytes = p->smem;
  lc.stream = static_cast<cudaStream_t>(stream);
  cudaLaunchAttribute at[2];
  lc.attrs = at;
  lc.numAttrs = 0;
  if (p->cl * p->kc > 1 && p->kind == BG_KIND_WS) {
    at[lc.numAttrs].id = cudaLaunchAttributeClusterDimension;
    at[lc.numAttrs].val.clusterDim.x = p->cl * p->kc;
    at[lc.numAttrs].val.clusterDim.y = 1;
    at[lc.numAttrs].val.clusterDim.z = 1;
    ++lc.numAttrs;
  }
  if (p->cooperative) {
    at[lc.numAttrs].id = cudaLaunchAttributeCooperative;
    at[lc.numAttrs].val.cooperative = 1;
    ++lc.numAttrs;
  }
  // the wave barrier's counter keeps counting across launches: this launch starts where the previous ones left it
  if (p->kp.wave_sync) p->kp.wave_base = p->launches * p->wave_per_launch;
  cudaError_t e;
  if (p->kind == BG_KIND_RING)
    e = cudaLaunchKernelEx(&lc, p->ring, p->tmA, p->tmB, p->kp);
  else
    e = cudaLaunchKernelEx(&lc, p->ws, p->tmA, p->tmB, p->tmBn, p->tmC, p->kp);
  if (e != cudaSuccess) return cuda_fail(e, "cudaLaunchKernelEx");
  ++p->launches;
  return 0;
}

int32_t bg_plan_check_error(bg_plan* p, void* stream, uint32_t* err_word) {
  if (p == nullptr) return fail(-1, "null plan");
  DeviceGuard guard(p->device);
  if (guard.status != cudaSuccess) return cuda_fail(guard.status, "cudaSetDevice");
  cudaError_t e = cudaStreamSynchronize(static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "cudaStreamSynchronize");
  uint32_t w = 0;
  if ((e = cudaMemcpy(&w, p->d_err, sizeof(w), cudaMemcpyDeviceToHost)) != cudaSuccess)
    return cuda_fail(e, "cudaMemcpy(error word)");
  if (err_word) *err_word = w;
  if (w != 0) {
    cudaMemset(p->d_err, 0, sizeof(uint32_t));
    // an interrupted split-K launch can leave arrival words behind; the next launch needs them zero
    if (p->d_tickets) cudaMemset(p->d_tickets, 0, p->ticket_words * sizeof(unsigned int));
    // an interrupted launch leaves the wave barrier's count short: start counting afresh
    if (p->d_wave) {
      cudaMemset(p->d_wave, 0, sizeof(unsigned long long));
      p->launches = 0;
    }
    static const char* roles[] = {"?", "producer (free stage)", "MMA (loaded stage)", "MMA (free accumulator)",
                                  "epilogue (finished accumulator)", "MMA drain", "load drain",
                                  "split-K (partial sums of the tile's other splits)"};
    const uint32_t role = w >> 24;
    return fail(6, "device wait timed out: %s, counter %u (error word 0x%08x)", role < 8 ? roles[role] : "?",
                w & 0xFFFFFFu, w);
  }
  return 0;
}

int32_t bg_plan_get_info(const bg_plan* p, bg_plan_info* info) {
  if (p == nullptr || info == nullptr) return fail(-1, "null pointer");
  info->grid = p->grid;
  info->threads = p->threads;
  info->smem_bytes = static_cast<int32_t>(p->smem);
  info->stages = p->kp.stages;
  info->tiles = p->kp.tiles;
  info->clusters = p->kp.nclusters;
  info->cluster = p->cl;
  info->paired = p->paired ? 1 : 0;
  info->bm = p->bm;
  info->bn = p->kp.bn;
  info->acc_bufs = p->kp.acc_bufs;
  info->tmem_cols = static_cast<int32_t>(p->kp.tmem_cols);
  info->max_active_clusters = p->max_active_clusters;
  info->narrow_tiles = p->narrow_tiles;
  info->split_k = p->kp.split_k;
  snprintf(info->kernel, sizeof(info->kernel), "%.95s", p->name);
  return 0;
}

void bg_plan_destroy(bg_plan* p) { free_plan(p); }

}  // extern "C"
