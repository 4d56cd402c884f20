// tiles.cu -- tile counting, exclusive scan, key duplication, onesweep radix
// sort and tile ranges.
//
// Sort: a stable LSD radix sort with 8-bit digits in the "onesweep" style
// (one kernel per digit pass, single read and single write of the pairs per
// pass). One upfront kernel histograms every pass's digits in a single read
// of the keys. In a pass, each 256-thread block takes a 3840-pair tile
// (ticketed in start order), ranks its digits warp by warp with match.any
// (warp-striped layout keeps the ranking stable), publishes its per-digit
// counts, obtains the global per-digit prefix from its predecessors by
// decoupled look-back (bounded spins), shuffles the tile into digit order in
// shared memory and writes it out in coalesced runs.
//
// Only the significant key bits are sorted: 32 depth bits + ceil(log2 tiles)
// tile bits, i.e. 6 passes for up to 65536 tiles. The reference sorts all 64
// bits with CUB (ruguangyou/3dgs_from_scratch src/cuda/kernel.cu:1341-1388);
// the higher bits are zero, so the order is identical.
#include "gs_common.cuh"

namespace gs {

// ---- tile counts (kernel.cu:784-818) -------------------------------------

__global__ void __launch_bounds__(256) count_tiles_kernel(int n, const float2 *__restrict__ points,
                                                          const float2 *__restrict__ radii,
                                                          const uint8_t *__restrict__ mask,
                                                          int width, int height,
                                                          int32_t *__restrict__ counts) {
  int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n || !mask[i]) return;
  float2 p = points[i], r = radii[i];
  TileRect tr = tile_rect(p.x, p.y, r.x, r.y, width, height);
  counts[i] = tr.empty ? 0 : (tr.x1 - tr.x0 + 1) * (tr.y1 - tr.y0 + 1);
}

// ---- exclusive scan of int32 counts (decoupled look-back) ----------------

constexpr int kScanThreads = 256;
constexpr int kScanItems = 8;
constexpr int kScanTile = kScanThreads * kScanItems;

__device__ __forceinline__ uint64_t ld_vol64(const uint64_t *p) {
  uint64_t v;
  asm volatile("ld.volatile.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void st_vol64(uint64_t *p, uint64_t v) {
  asm volatile("st.volatile.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}

__global__ void __launch_bounds__(kScanThreads) scan_kernel(int n, const int32_t *__restrict__ in,
                                                            int32_t *__restrict__ out,
                                                            int64_t *__restrict__ total,
                                                            uint64_t *__restrict__ words,
                                                            int num_tiles, uint32_t *status) {
  __shared__ int s_tile;
  __shared__ long long s_warp[kScanThreads / 32 + 1];
  __shared__ unsigned long long s_prefix;
  const int t = threadIdx.x, lane = t & 31, warp = t >> 5;
  if (t == 0) s_tile = (int)atomicAdd((unsigned long long *)(words + num_tiles), 1ull);
  __syncthreads();
  const int tile = s_tile;
  const long long base = (long long)tile * kScanTile + (long long)t * kScanItems;
  int v[kScanItems];
  long long sum = 0;
#pragma unroll
  for (int k = 0; k < kScanItems; ++k) {
    long long idx = base + k;
    v[k] = idx < n ? in[idx] : 0;
    sum += v[k];
  }
  long long incl = sum;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    long long y = __shfl_up_sync(0xffffffffu, incl, o);
    if (lane >= o) incl += y;
  }
  if (lane == 31) s_warp[warp] = incl;
  __syncthreads();
  if (t == 0) {
    long long acc = 0;
    for (int w = 0; w < kScanThreads / 32; ++w) {
      long long x = s_warp[w];
      s_warp[w] = acc;
      acc += x;
    }
    s_warp[kScanThreads / 32] = acc;
    const uint64_t agg = (uint64_t)acc;
    uint64_t prefix = 0;
    if (tile == 0) {
      st_vol64(words, (2ull << 62) | agg);
    } else {
      st_vol64(words + tile, (1ull << 62) | agg);
      for (int j = tile - 1; j >= 0; --j) {
        uint64_t w;
        uint32_t spins = 0;
        do {
          w = ld_vol64(words + j);
        } while ((w >> 62) == 0 && ++spins < kSpinLimit);
        if ((w >> 62) == 0) {
          atomicExch(status, (uint32_t)GS_ERR_DEVICE_TIMEOUT);
          break;
        }
        prefix += w & ((1ull << 62) - 1);
        if ((w >> 62) == 2) break;
      }
      st_vol64(words + tile, (2ull << 62) | (prefix + agg));
    }
    s_prefix = prefix;
    if (tile == num_tiles - 1) *total = (int64_t)(prefix + agg);
  }
  __syncthreads();
  long long run = (long long)s_prefix + s_warp[warp] + (incl - sum);
#pragma unroll
  for (int k = 0; k < kScanItems; ++k) {
    long long idx = base + k;
    if (idx < n) out[idx] = (int32_t)run;
    run += v[k];
  }
}

// ---- key duplication (kernel.cu:820-873) ------------------------------------

__global__ void __launch_bounds__(256) keygen_kernel(int n, const float2 *__restrict__ points,
                                                     const float2 *__restrict__ radii,
                                                     const float *__restrict__ depths,
                                                     const uint8_t *__restrict__ mask,
                                                     const int32_t *__restrict__ offsets,
                                                     int width, int height, int64_t total,
                                                     uint64_t *__restrict__ keys,
                                                     int32_t *__restrict__ vals) {
  int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n || !mask[i]) return;
  float2 p = points[i], r = radii[i];
  TileRect tr = tile_rect(p.x, p.y, r.x, r.y, width, height);
  if (tr.empty) return;
  const int tx = tiles_x_of(width);
  const uint64_t dbits = (uint64_t)__float_as_uint(depths[i]);
  int64_t o = offsets[i];
  if (o < 0) return;
  for (int y = tr.y0; y <= tr.y1; ++y)
    for (int x = tr.x0; x <= tr.x1; ++x) {
      if (o >= total) return;  // only reachable if the offsets were corrupted
      uint64_t tid = (uint64_t)(y * tx + x);
      keys[o] = (tid << 32) | dbits;
      vals[o] = i;
      ++o;
    }
}

// ---- onesweep radix sort -----------------------------------------------------

constexpr int kSortThreads = 256;
constexpr int kSortWarps = kSortThreads / 32;
constexpr int kSortItems = 15;
constexpr int kSortTile = kSortThreads * kSortItems;  // 3840 pairs
constexpr int kMaxPasses = 8;
constexpr uint32_t kLbAgg = 1u << 30;
constexpr uint32_t kLbPrefix = 2u << 30;
constexpr uint32_t kLbValue = (1u << 30) - 1;

// Histogram of every pass's digits in one read of the keys.
__global__ void __launch_bounds__(256) sort_histogram_kernel(const uint64_t *__restrict__ keys,
                                                             int64_t n, int passes, int end_bit,
                                                             uint32_t *__restrict__ hist) {
  __shared__ uint32_t sh[kMaxPasses * 256];
  for (int k = threadIdx.x; k < passes * 256; k += blockDim.x) sh[k] = 0;
  __syncthreads();
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  const uint32_t lane = lane_id();
  for (int64_t base = (int64_t)blockIdx.x * blockDim.x; base < n; base += stride) {
    const int64_t idx = base + threadIdx.x;
    const bool valid = idx < n;
    const uint64_t key = valid ? keys[idx] : 0;
    for (int p = 0; p < passes; ++p) {
      const int bits = min(8, end_bit - 8 * p);
      const uint32_t d = valid ? (uint32_t)((key >> (8 * p)) & ((1u << bits) - 1u)) : 0x100u;
      const uint32_t peers = __match_any_sync(0xffffffffu, d);
      const uint32_t leader = 31 - __clz(peers);
      if (valid && lane == leader) atomicAdd(&sh[p * 256 + d], (uint32_t)__popc(peers));
    }
  }
  __syncthreads();
  for (int k = threadIdx.x; k < passes * 256; k += blockDim.x)
    if (sh[k]) atomicAdd(&hist[k], sh[k]);
}

// Block-wide exclusive scan of one uint32 per thread, blockDim == 256.
__device__ __forceinline__ uint32_t block_scan_256(uint32_t x, uint32_t *s_tmp) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  uint32_t incl = x;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    uint32_t y = __shfl_up_sync(0xffffffffu, incl, o);
    if (lane >= o) incl += y;
  }
  if (lane == 31) s_tmp[warp] = incl;
  __syncthreads();
  if (warp == 0) {
    uint32_t w = lane < kSortWarps ? s_tmp[lane] : 0u;
    uint32_t wi = w;
#pragma unroll
    for (int o = 1; o < kSortWarps; o <<= 1) {
      uint32_t y = __shfl_up_sync(0xffffffffu, wi, o);
      if (lane >= o) wi += y;
    }
    if (lane < kSortWarps) s_tmp[lane] = wi - w;
  }
  __syncthreads();
  uint32_t r = incl - x + s_tmp[warp];
  __syncthreads();
  return r;
}

struct SortSmem {
  uint64_t keys[kSortTile];
  int32_t vals[kSortTile];
  uint32_t whist[kSortWarps][256];
  uint32_t gbase[256];
  uint32_t lstart[256];
  uint32_t tmp[kSortWarps + 1];
  int tile;
};

__global__ void __launch_bounds__(kSortThreads, 2) onesweep_pass_kernel(
    const uint64_t *__restrict__ keys_in, const int32_t *__restrict__ vals_in,
    uint64_t *__restrict__ keys_out, int32_t *__restrict__ vals_out, int64_t n, int shift,
    uint32_t dmask, const uint32_t *__restrict__ hist, uint32_t *__restrict__ lookback,
    uint32_t *__restrict__ ticket, uint32_t *status) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  SortSmem &S = *reinterpret_cast<SortSmem *>(smem_raw);
  const int t = threadIdx.x, warp = t >> 5;
  const uint32_t lane = t & 31;
  if (t == 0) S.tile = (int)atomicAdd(ticket, 1u);
  for (int k = t; k < kSortWarps * 256; k += kSortThreads) (&S.whist[0][0])[k] = 0;
  __syncthreads();
  const int tile = S.tile;
  const int64_t base = (int64_t)tile * kSortTile + (int64_t)warp * (32 * kSortItems);

  // Load warp-striped: item k of lane l is element base + k*32 + l.
  uint64_t key[kSortItems];
  int32_t val[kSortItems];
#pragma unroll
  for (int k = 0; k < kSortItems; ++k) {
    const int64_t idx = base + k * 32 + lane;
    const bool valid = idx < n;
    key[k] = valid ? keys_in[idx] : ~0ull;
    val[k] = valid ? vals_in[idx] : 0;
  }

  // Stable warp-local ranks: running per-warp digit counts in shared memory.
  uint32_t rank[kSortItems];
  const uint32_t lt_mask = (1u << lane) - 1u;
#pragma unroll
  for (int k = 0; k < kSortItems; ++k) {
    const int64_t idx = base + k * 32 + lane;
    const bool valid = idx < n;
    const uint32_t d = valid ? (uint32_t)((key[k] >> shift) & dmask) : 0x100u;
    const uint32_t peers = __match_any_sync(0xffffffffu, d);
    const uint32_t leader = 31 - __clz(peers);
    uint32_t old = 0;
    if (valid && lane == leader) {
      old = S.whist[warp][d];
      S.whist[warp][d] = old + (uint32_t)__popc(peers);
    }
    old = __shfl_sync(0xffffffffu, old, leader);
    rank[k] = old + (uint32_t)__popc(peers & lt_mask);
    __syncwarp();
  }
  __syncthreads();

  // Thread t owns digit t: warp offsets, block count, look-back.
  const uint32_t d = (uint32_t)t;
  uint32_t cnt = 0;
#pragma unroll
  for (int w = 0; w < kSortWarps; ++w) {
    uint32_t c = S.whist[w][d];
    S.whist[w][d] = cnt;
    cnt += c;
  }
  uint32_t *my_lb = lookback + (size_t)tile * 256 + d;
  uint32_t excl = 0;
  if (tile == 0) {
    st_volatile_u32(my_lb, kLbPrefix | cnt);
  } else {
    st_volatile_u32(my_lb, kLbAgg | cnt);
    for (int j = tile - 1; j >= 0; --j) {
      const uint32_t *w = lookback + (size_t)j * 256 + d;
      uint32_t x;
      uint32_t spins = 0;
      do {
        x = ld_volatile_u32(w);
      } while ((x >> 30) == 0 && ++spins < kSpinLimit);
      if ((x >> 30) == 0) {
        atomicExch(status, (uint32_t)GS_ERR_DEVICE_TIMEOUT);
        break;
      }
      excl += x & kLbValue;
      if ((x >> 30) == 2) break;
    }
    st_volatile_u32(my_lb, kLbPrefix | ((excl + cnt) & kLbValue));
  }
  const uint32_t gdig = block_scan_256(hist[d], S.tmp);
  const uint32_t ldig = block_scan_256(cnt, S.tmp);
  S.gbase[d] = gdig + excl;
  S.lstart[d] = ldig;
  __syncthreads();

  // Shuffle into digit order in shared memory.
#pragma unroll
  for (int k = 0; k < kSortItems; ++k) {
    const int64_t idx = base + k * 32 + lane;
    if (idx < n) {
      const uint32_t dk = (uint32_t)((key[k] >> shift) & dmask);
      const uint32_t pos = S.lstart[dk] + S.whist[warp][dk] + rank[k];
      S.keys[pos] = key[k];
      S.vals[pos] = val[k];
    }
  }
  __syncthreads();

  const int64_t tile_base = (int64_t)tile * kSortTile;
  const int valid_count = (int)min((int64_t)kSortTile, n - tile_base);
  for (int p = t; p < valid_count; p += kSortThreads) {
    const uint64_t kk = S.keys[p];
    const uint32_t dk = (uint32_t)((kk >> shift) & dmask);
    const uint32_t out = S.gbase[dk] + ((uint32_t)p - S.lstart[dk]);
    if ((int64_t)out < n) {  // always true unless a look-back gave up
      keys_out[out] = kk;
      vals_out[out] = S.vals[p];
    }
  }
}

// ---- tile ranges (kernel.cu:875-914) -------------------------------------------

__global__ void __launch_bounds__(256) ranges_kernel(const uint64_t *__restrict__ keys,
                                                     int64_t n, int num_tiles,
                                                     int32_t *__restrict__ offsets) {
  const int64_t k = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (k >= n) return;
  const int tile = min((int)(keys[k] >> 32), num_tiles - 1);
  const int prev = (k == 0) ? -1 : min((int)(keys[k - 1] >> 32), num_tiles - 1);
  for (int g = prev + 1; g <= tile; ++g) offsets[g] = (int32_t)k;
  if (k == n - 1)
    for (int g = tile + 1; g < num_tiles; ++g) offsets[g] = (int32_t)n;
}

// ---- host-side sort driver -------------------------------------------------------

static inline size_t align_up(size_t x, size_t a) { return (x + a - 1) / a * a; }

struct SortLayout {
  size_t hist, lookback, tickets, total;
  int tiles;
};

static SortLayout sort_layout(int64_t n) {
  SortLayout L;
  L.tiles = (int)((n + kSortTile - 1) / kSortTile);
  L.hist = 0;
  L.lookback = align_up(L.hist + kMaxPasses * 256 * sizeof(uint32_t), 256);
  L.tickets = align_up(L.lookback + (size_t)kMaxPasses * L.tiles * 256 * sizeof(uint32_t), 256);
  L.total = align_up(L.tickets + kMaxPasses * sizeof(uint32_t), 256);
  return L;
}

// Sorts (keys, vals) on bits [0, end_bit) in ceil(end_bit / 8) passes; the
// result ends in the buffers selected by the parity of the pass count
// (even: keys/vals, odd: alt).
static int run_sort(int64_t n, uint64_t *keys, int32_t *vals, uint64_t *keys_alt,
                    int32_t *vals_alt, int end_bit, void *scratch, cudaStream_t st) {
  const int passes = (end_bit + 7) / 8;
  if (n <= 0 || passes <= 0) return GS_OK;
  if (n > (int64_t)kLbValue) return GS_ERR_CAPACITY;
  SortLayout L = sort_layout(n);
  unsigned char *base = reinterpret_cast<unsigned char *>(scratch);
  uint32_t *hist = reinterpret_cast<uint32_t *>(base + L.hist);
  uint32_t *lookback = reinterpret_cast<uint32_t *>(base + L.lookback);
  uint32_t *tickets = reinterpret_cast<uint32_t *>(base + L.tickets);
  int rc = cuda_status(cudaMemsetAsync(scratch, 0, L.total, st));
  if (rc) return rc;
  int dev = 0;
  cudaGetDevice(&dev);
  int sms = 148;
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  int64_t hb = (n + 255) / 256;
  int hblocks = (int)(hb < (int64_t)sms * 4 ? hb : (int64_t)sms * 4);
  sort_histogram_kernel<<<hblocks, 256, 0, st>>>(keys, n, passes, end_bit, hist);
  count_launch();
  static int attr_done[64] = {0};
  const size_t smem = sizeof(SortSmem);
  if (dev < 64 && !attr_done[dev]) {
    cudaFuncSetAttribute(onesweep_pass_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         (int)smem);
    attr_done[dev] = 1;
  }
  uint64_t *kin = keys, *kout = keys_alt;
  int32_t *vin = vals, *vout = vals_alt;
  for (int p = 0; p < passes; ++p) {
    const int bits = end_bit - 8 * p < 8 ? end_bit - 8 * p : 8;
    onesweep_pass_kernel<<<L.tiles, kSortThreads, smem, st>>>(
        kin, vin, kout, vout, n, 8 * p, (1u << bits) - 1u, hist + 256 * p,
        lookback + (size_t)p * L.tiles * 256,
        tickets + p, device_status_word());
    count_launch();
    uint64_t *tk = kin;
    kin = kout;
    kout = tk;
    int32_t *tv = vin;
    vin = vout;
    vout = tv;
  }
  return launch_status();
}

static int key_bits_for_tiles(int num_tiles) {
  int tile_bits = 0;
  while ((1ll << tile_bits) < (long long)num_tiles) ++tile_bits;
  return 32 + tile_bits;
}

}  // namespace gs

using namespace gs;

static inline cudaStream_t as_stream(void *s) { return reinterpret_cast<cudaStream_t>(s); }

extern "C" int gs_count_tiles(int n, const float *points_img, const float *radii,
                              const uint8_t *mask, int width, int height, int32_t *counts,
                              void *stream) {
  if (n < 0 || width <= 0 || height <= 0) return GS_ERR_INVALID_ARGUMENT;
  if (((uintptr_t)points_img & 7) || ((uintptr_t)radii & 7)) return GS_ERR_INVALID_ARGUMENT;
  if (n == 0) return GS_OK;
  count_tiles_kernel<<<(n + 255) / 256, 256, 0, as_stream(stream)>>>(
      n, reinterpret_cast<const float2 *>(points_img), reinterpret_cast<const float2 *>(radii),
      mask, width, height, counts);
  count_launch();
  return launch_status();
}

extern "C" size_t gs_scan_scratch_bytes(int n) {
  int tiles = (n + kScanTile - 1) / kScanTile;
  return (size_t)(tiles + 1) * sizeof(uint64_t);
}

extern "C" int gs_exclusive_scan(int n, const int32_t *counts, int32_t *offsets,
                                 int64_t *total_dev, void *scratch, size_t scratch_bytes,
                                 void *stream) {
  if (n < 0) return GS_ERR_INVALID_ARGUMENT;
  cudaStream_t st = as_stream(stream);
  if (n == 0) return cuda_status(cudaMemsetAsync(total_dev, 0, sizeof(int64_t), st));
  if (scratch == nullptr || scratch_bytes < gs_scan_scratch_bytes(n)) return GS_ERR_CAPACITY;
  int tiles = (n + kScanTile - 1) / kScanTile;
  int rc = cuda_status(cudaMemsetAsync(scratch, 0, gs_scan_scratch_bytes(n), st));
  if (rc) return rc;
  scan_kernel<<<tiles, kScanThreads, 0, st>>>(n, counts, offsets, total_dev,
                                              reinterpret_cast<uint64_t *>(scratch), tiles,
                                              device_status_word());
  count_launch();
  return launch_status();
}

extern "C" size_t gs_sort_scratch_bytes(int64_t n) { return sort_layout(n > 0 ? n : 1).total; }

extern "C" int gs_sort_pairs(int64_t n, uint64_t *keys, int32_t *vals, uint64_t *keys_alt,
                             int32_t *vals_alt, int end_bit, void *scratch,
                             size_t scratch_bytes, void *stream) {
  if (n < 0 || end_bit < 0 || end_bit > 64) return GS_ERR_INVALID_ARGUMENT;
  if (n == 0 || end_bit == 0) return GS_OK;
  if (scratch == nullptr || scratch_bytes < gs_sort_scratch_bytes(n)) return GS_ERR_CAPACITY;
  int passes = (end_bit + 7) / 8;
  cudaStream_t st = as_stream(stream);
  int rc = run_sort(n, keys, vals, keys_alt, vals_alt, end_bit, scratch, st);
  if (rc) return rc;
  if (passes & 1) {
    rc = cuda_status(cudaMemcpyAsync(keys, keys_alt, n * sizeof(uint64_t), cudaMemcpyDeviceToDevice, st));
    if (rc) return rc;
    rc = cuda_status(cudaMemcpyAsync(vals, vals_alt, n * sizeof(int32_t), cudaMemcpyDeviceToDevice, st));
  }
  return rc;
}

// Scratch of gs_tile_layout: key buffer A (unless the caller keeps the keys),
// key buffer B, value buffer B, sort state.
extern "C" size_t gs_tile_layout_scratch_bytes(int64_t total, int width, int height) {
  (void)width;
  (void)height;
  size_t t = (size_t)(total > 0 ? total : 1);
  size_t bytes = align_up(t * sizeof(uint64_t), 256) * 2 + align_up(t * sizeof(int32_t), 256);
  return bytes + gs_sort_scratch_bytes(total);
}

extern "C" int gs_tile_layout(int n, const float *points_img, const float *radii,
                              const float *depths, const uint8_t *mask, const int32_t *offsets,
                              int64_t total, int width, int height, int64_t *keys_sorted,
                              int32_t *ids_sorted, int32_t *indexing_offset, void *scratch,
                              size_t scratch_bytes, void *stream) {
  if (n < 0 || width <= 0 || height <= 0 || total < 0) return GS_ERR_INVALID_ARGUMENT;
  if (((uintptr_t)points_img & 7) || ((uintptr_t)radii & 7)) return GS_ERR_INVALID_ARGUMENT;
  if (total >= (int64_t)kLbValue) return GS_ERR_CAPACITY;
  cudaStream_t st = as_stream(stream);
  const int num_tiles = tiles_x_of(width) * tiles_y_of(height);
  // rasterizer.cpp:352: offsets start at zero; with no pairs they stay zero.
  int rc = cuda_status(cudaMemsetAsync(indexing_offset, 0, (size_t)num_tiles * sizeof(int32_t), st));
  if (rc || total == 0) return rc;
  if (scratch == nullptr || scratch_bytes < gs_tile_layout_scratch_bytes(total, width, height))
    return GS_ERR_CAPACITY;
  unsigned char *p = reinterpret_cast<unsigned char *>(scratch);
  const size_t kbytes = align_up((size_t)total * sizeof(uint64_t), 256);
  const size_t vbytes = align_up((size_t)total * sizeof(int32_t), 256);
  uint64_t *keys_a = keys_sorted ? reinterpret_cast<uint64_t *>(keys_sorted)
                                 : reinterpret_cast<uint64_t *>(p);
  uint64_t *keys_b = reinterpret_cast<uint64_t *>(p + kbytes);
  int32_t *vals_b = reinterpret_cast<int32_t *>(p + 2 * kbytes);
  void *sort_scratch = p + 2 * kbytes + vbytes;
  const int key_bits = key_bits_for_tiles(num_tiles);
  const int passes = (key_bits + 7) / 8;
  // Emit into the buffer pair that the final pass does not write, so the
  // sorted result lands in (keys_a, ids_sorted).
  uint64_t *k0 = (passes & 1) ? keys_b : keys_a;
  int32_t *v0 = (passes & 1) ? vals_b : ids_sorted;
  uint64_t *k1 = (passes & 1) ? keys_a : keys_b;
  int32_t *v1 = (passes & 1) ? ids_sorted : vals_b;
  if (n > 0) {
    keygen_kernel<<<(n + 255) / 256, 256, 0, st>>>(
        n, reinterpret_cast<const float2 *>(points_img), reinterpret_cast<const float2 *>(radii),
        depths, mask, offsets, width, height, total, k0, v0);
    count_launch();
  }
  rc = run_sort(total, k0, v0, k1, v1, key_bits, sort_scratch, st);
  if (rc) return rc;
  ranges_kernel<<<(unsigned)((total + 255) / 256), 256, 0, st>>>(keys_a, total, num_tiles,
                                                                  indexing_offset);
  count_launch();
  return launch_status();
}

// ---- exclusive scan without caller-provided scratch -----------------------
//
// For callers that can hand over their input and output buffers but may not
// allocate device memory themselves -- e.g. a host application that owns all
// GPU memory through its own allocator, or a frame loop where a cudaMalloc /
// cudaFree (which synchronise the device) is not allowed. The look-back state
// the scan needs lives in this fixed device array instead: 64 KiB, enough for
// up to kNoAllocScanMaxN counts, held by every GPU that loads the library
// until the process exits.
constexpr int kNoAllocScanMaxN = 1 << 24;  // 16,777,216 counts
constexpr int kNoAllocScanWords = (kNoAllocScanMaxN + kScanTile - 1) / kScanTile + 1;
static __device__ __align__(256) uint64_t g_noalloc_scan_words[kNoAllocScanWords];

static uint64_t *g_noalloc_scan_ptr[64] = {nullptr};

// Device address of g_noalloc_scan_words for the current device, looked up
// once per device (host code may not use the symbol itself as a pointer).
static int noalloc_scan_words(uint64_t **out) {
  int dev = 0;
  int rc = cuda_status(cudaGetDevice(&dev));
  if (rc) return rc;
  if (dev < 0 || dev >= 64) return GS_ERR_INVALID_ARGUMENT;
  if (g_noalloc_scan_ptr[dev] == nullptr) {
    void *p = nullptr;
    rc = cuda_status(cudaGetSymbolAddress(&p, g_noalloc_scan_words));
    if (rc) return rc;
    g_noalloc_scan_ptr[dev] = reinterpret_cast<uint64_t *>(p);
  }
  *out = g_noalloc_scan_ptr[dev];
  return GS_OK;
}

extern "C" int gs_exclusive_scan_noalloc(int n, const int32_t *counts, int32_t *offsets,
                                         int64_t *total_dev, void *stream) {
  if (n < 0 || total_dev == nullptr) return GS_ERR_INVALID_ARGUMENT;
  if (n > kNoAllocScanMaxN) return GS_ERR_CAPACITY;
  cudaStream_t st = as_stream(stream);
  if (n == 0) return cuda_status(cudaMemsetAsync(total_dev, 0, sizeof(int64_t), st));
  if (counts == nullptr || offsets == nullptr) return GS_ERR_INVALID_ARGUMENT;
  uint64_t *words = nullptr;
  int rc = noalloc_scan_words(&words);
  if (rc) return rc;
  const int tiles = (n + kScanTile - 1) / kScanTile;
  // The array keeps the previous call's look-back words and ticket: clear the
  // part this call uses (tiles + 1 words) before the launch, on the same stream.
  rc = cuda_status(cudaMemsetAsync(words, 0, (size_t)(tiles + 1) * sizeof(uint64_t), st));
  if (rc) return rc;
  scan_kernel<<<tiles, kScanThreads, 0, st>>>(n, counts, offsets, total_dev, words, tiles,
                                              device_status_word());
  count_launch();
  return launch_status();
}
