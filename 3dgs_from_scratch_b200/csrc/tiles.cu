// tiles.cu -- tile counting, exclusive scan, onesweep radix sort, tile layout.
//
// Sort: a stable LSD radix sort with 8-bit digits in the "onesweep" style
// (one kernel per digit pass, one read and one write of the pairs per pass),
// templated on the key width. One upfront kernel histograms every pass's
// digits in a single read of the keys. In a pass, each 256-thread block
// takes a tile of pairs (ticketed in start order), ranks its digits warp by
// warp (lanes with equal digits found with one ballot per digit bit; the
// warp-striped layout keeps the ranking stable),
// publishes its per-digit counts, obtains the global per-digit prefix from
// its predecessors by decoupled look-back (bounded spins), shuffles the tile
// into digit order in shared memory and writes it out in coalesced runs.
//
// Tile layout: the reference emits (tile << 32 | depth bits, id) pairs in
// Gaussian order and sorts all 64 key bits with CUB (ruguangyou/
// 3dgs_from_scratch src/cuda/kernel.cu:820-873,1341-1388). The same order
// comes out of two cheaper stable sorts: the N Gaussians by depth bits (4
// passes over N, ties keep Gaussian order), then the K pairs -- emitted in
// that depth order -- by tile id alone (2 passes of 16-bit keys up to 65536
// tiles). Within a tile the entries end up ordered by depth bits, ties by
// Gaussian id: exactly the reference's stable 64-bit order.
#include "gs_common.cuh"

namespace gs {

static inline size_t align_up(size_t x, size_t a) { return (x + a - 1) / a * a; }

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

// Warp-parallel look-back over 64-bit words (flag in bits 63..62: 1 =
// aggregate, 2 = inclusive prefix): lane i inspects predecessor tile-1-i,
// 32 predecessors per step; bounded spins record GS_ERR_DEVICE_TIMEOUT.
// Call with the whole warp; returns the exclusive prefix in every lane.
__device__ __forceinline__ uint64_t warp_lookback64(const uint64_t *__restrict__ words, int tile,
                                                    uint32_t *status) {
  const uint32_t lane = lane_id();
  uint64_t excl = 0;
  int top = tile - 1;
  while (top >= 0) {
    const int j = top - (int)lane;
    uint64_t w = 0;
    if (j >= 0) {
      uint32_t spins = 0;
      do {
        w = ld_vol64(words + j);
      } while ((w >> 62) == 0 && ++spins < kSpinLimit);
      if ((w >> 62) == 0) {
        atomicExch(status, (uint32_t)GS_ERR_DEVICE_TIMEOUT);
        w = 2ull << 62;  // give up: treat as a (wrong) prefix so the walk ends
      }
    } else {
      w = 2ull << 62;  // before tile 0: a zero prefix
    }
    const uint32_t prefix_lanes = __ballot_sync(0xffffffffu, (w >> 62) == 2);
    // nearest predecessor holding a prefix; with none in this window all 32
    // aggregates count and the walk moves 32 tiles further back
    const int stop = prefix_lanes ? __ffs(prefix_lanes) - 1 : 31;
    uint64_t v = ((int)lane <= stop) ? (w & ((1ull << 62) - 1)) : 0ull;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    excl += v;
    if (prefix_lanes) break;
    top -= 32;
  }
  return excl;
}

// Exclusive scan of n counts (optionally gathered: in[gather[i]]) into out,
// total into *total. words: one per tile plus the ticket counter at
// words[num_tiles], all zero on entry.
__global__ void __launch_bounds__(kScanThreads) scan_kernel(int n, const int32_t *__restrict__ in,
                                                            const int32_t *__restrict__ gather,
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
    int x = 0;
    if (idx < n) {
      if (gather) {
        const int g = gather[idx];
        x = (g >= 0 && g < n) ? in[g] : 0;  // out-of-range only with a corrupted permutation
      } else {
        x = in[idx];
      }
    }
    v[k] = x;
    sum += x;
  }
  long long incl = sum;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    long long y = __shfl_up_sync(0xffffffffu, incl, o);
    if (lane >= o) incl += y;
  }
  if (lane == 31) s_warp[warp] = incl;
  __syncthreads();
  if (warp == 0) {
    long long wv = lane < kScanThreads / 32 ? s_warp[lane] : 0;
    long long wi = wv;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      long long y = __shfl_up_sync(0xffffffffu, wi, o);
      if (lane >= o) wi += y;
    }
    const uint64_t agg = (uint64_t)__shfl_sync(0xffffffffu, wi, kScanThreads / 32 - 1);
    if (lane < kScanThreads / 32) s_warp[lane] = wi - wv;
    uint64_t prefix = 0;
    if (tile == 0) {
      if (lane == 0) st_vol64(words, (2ull << 62) | agg);
    } else {
      if (lane == 0) st_vol64(words + tile, (1ull << 62) | agg);
      prefix = warp_lookback64(words, tile, status);
      if (lane == 0) st_vol64(words + tile, (2ull << 62) | (prefix + agg));
    }
    if (lane == 0) {
      s_prefix = prefix;
      if (tile == num_tiles - 1) {
        *total = (int64_t)(prefix + agg);
        // the int32 offsets wrapped: the total (int64) stays exact, the
        // offsets past INT32_MAX do not
        if (prefix + agg > (uint64_t)INT32_MAX) atomicCAS(status, 0u, (uint32_t)GS_ERR_CAPACITY);
      }
    }
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

// Item count of the capacity form of the layout: *count_dev when it fits the
// capacity, else 0 (the lists are then empty and GS_ERR_CAPACITY is recorded
// by the pair emission).
__device__ __forceinline__ int64_t capped_count(const int64_t *count_dev, int64_t capacity) {
  const int64_t c = *count_dev;
  return (c >= 0 && c <= capacity) ? c : 0;
}

// ---- onesweep radix sort -----------------------------------------------------

constexpr int kSortThreads = 256;
#ifndef GS_SORT_LOOKBACK
#define GS_SORT_LOOKBACK 16  // predecessors inspected per look-back round trip
#endif
constexpr int kSortWarps = kSortThreads / 32;
constexpr int kMaxPasses = 8;
constexpr uint32_t kLbAgg = 1u << 30;
constexpr uint32_t kLbPrefix = 2u << 30;
constexpr uint32_t kLbValue = (1u << 30) - 1;

// Items per thread and resident blocks per SM by key width (shared memory per
// tile: items * 256 * (key + 4) B; registers capped at 65536 / (256 * blocks)).
template <typename KT> struct SortItems;
template <> struct SortItems<uint64_t> {
  static constexpr int value = 14, min_blocks = 2;
};
template <> struct SortItems<uint32_t> {
  static constexpr int value = 10, min_blocks = 3;
};
template <> struct SortItems<uint16_t> {
  static constexpr int value = 12, min_blocks = 3;
};

template <typename KT>
__device__ __forceinline__ uint32_t digit_of(KT key, int shift, uint32_t dmask) {
  return (uint32_t)((uint64_t)key >> shift) & dmask;
}

// Histogram of every pass's digits in one read of the keys (sub-histograms
// in shared memory shared by a few warps each, merged per block into global
// counts).
template <typename KT>
__global__ void __launch_bounds__(256) sort_histogram_kernel(const KT *__restrict__ keys,
                                                             int64_t n, int passes, int end_bit,
                                                             uint32_t *__restrict__ hist) {
  constexpr int kMaxP = (int)sizeof(KT);            // 8-bit digits per key
  constexpr int kCopies = sizeof(KT) == 8 ? 4 : 8;  // <= 32 KB of shared memory
  __shared__ uint32_t sh[kCopies][kMaxP * 256];
  const int copy = (threadIdx.x >> 5) % kCopies;
  for (int k = threadIdx.x; k < kCopies * kMaxP * 256; k += blockDim.x) (&sh[0][0])[k] = 0;
  __syncthreads();
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; idx < n; idx += stride) {
    const KT key = keys[idx];
    for (int p = 0; p < passes; ++p) {
      const int bits = min(8, end_bit - 8 * p);
      atomicAdd(&sh[copy][p * 256 + digit_of(key, 8 * p, (1u << bits) - 1u)], 1u);
    }
  }
  __syncthreads();
  for (int k = threadIdx.x; k < passes * 256; k += blockDim.x) {
    uint32_t c = 0;
#pragma unroll
    for (int w = 0; w < kCopies; ++w) c += sh[w][k];
    if (c) atomicAdd(&hist[k], c);
  }
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

template <typename KT, int ITEMS>
struct SortSmem {
  KT keys[kSortThreads * ITEMS];
  int32_t vals[kSortThreads * ITEMS];
  uint32_t whist[kSortWarps][256];
  uint32_t gbase[256];
  uint32_t lstart[256];
  uint32_t tmp[kSortWarps + 1];
  int tile;
};

// One digit pass. vals_in == nullptr means the identity (value = index).
template <typename KT, int ITEMS>
__global__ void __launch_bounds__(kSortThreads, SortItems<KT>::min_blocks) onesweep_pass_kernel(
    const KT *__restrict__ keys_in, const int32_t *__restrict__ vals_in,
    KT *__restrict__ keys_out, int32_t *__restrict__ vals_out, int64_t n, int shift,
    uint32_t dmask, const uint32_t *__restrict__ hist, uint32_t *__restrict__ lookback,
    uint32_t *__restrict__ ticket, uint32_t *status, const int64_t *__restrict__ n_dev) {
  constexpr int kTileItems = kSortThreads * ITEMS;
  extern __shared__ __align__(16) unsigned char smem_raw[];
  SortSmem<KT, ITEMS> &S = *reinterpret_cast<SortSmem<KT, ITEMS> *>(smem_raw);
  const int t = threadIdx.x, warp = t >> 5;
  const uint32_t lane = t & 31;
  // capacity form: n is the capacity the grid was sized for, *n_dev the
  // item count (0 when it exceeds the capacity)
  if (n_dev) n = capped_count(n_dev, n);
  if (t == 0) S.tile = (int)atomicAdd(ticket, 1u);
  for (int k = t; k < kSortWarps * 256; k += kSortThreads) (&S.whist[0][0])[k] = 0;
  __syncthreads();
  const int tile = S.tile;
  // tiles are ticketed in order, so the tiles past the items form the tail
  // of the ticket sequence: no tile that holds items looks back at them
  if ((int64_t)tile * kTileItems >= n) return;
  const int64_t base = (int64_t)tile * kTileItems + (int64_t)warp * (32 * ITEMS);

  // Load warp-striped: item k of lane l is element base + k*32 + l.
  KT key[ITEMS];
  int32_t val[ITEMS];
#pragma unroll
  for (int k = 0; k < ITEMS; ++k) {
    const int64_t idx = base + k * 32 + lane;
    const bool valid = idx < n;
    key[k] = valid ? keys_in[idx] : (KT)0;
    val[k] = valid ? (vals_in ? vals_in[idx] : (int32_t)idx) : 0;
  }

  // Stable warp-local ranks: running per-warp digit counts in shared memory.
  uint32_t rank[ITEMS];
  uint32_t lead_old[ITEMS];
  uint8_t leader_of[ITEMS];
  const uint32_t lt_mask = (1u << lane) - 1u;
#pragma unroll
  for (int k = 0; k < ITEMS; ++k) {
    const int64_t idx = base + k * 32 + lane;
    const bool valid = idx < n;
    const uint32_t d = valid ? digit_of(key[k], shift, dmask) : 0x100u;
    // Lanes with the same digit (and validity): one ballot per digit bit,
    // which issues faster than match.any.
    uint32_t peers = __ballot_sync(0xffffffffu, valid);
    if (!valid) peers = ~peers;
#pragma unroll
    for (int b = 0; b < 8; ++b) {
      const bool bit = (d >> b) & 1u;
      const uint32_t bal = __ballot_sync(0xffffffffu, bit);
      peers &= bit ? bal : ~bal;
    }
    const uint32_t leader = 31 - __clz(peers);
    // One shared-memory atomic per digit group: the returned count is only
    // needed in the scatter below, so the ITEMS atomics of a thread are
    // independent instructions that pipeline (a load/store pair per item
    // would serialise on the possible aliasing of consecutive items).
    uint32_t old = 0;
    if (valid && lane == leader) old = atomicAdd(&S.whist[warp][d], (uint32_t)__popc(peers));
    rank[k] = (uint32_t)__popc(peers & lt_mask);
    lead_old[k] = old;
    leader_of[k] = (uint8_t)leader;
  }
#pragma unroll
  for (int k = 0; k < ITEMS; ++k) rank[k] += __shfl_sync(0xffffffffu, lead_old[k], leader_of[k]);
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
    // Decoupled look-back over kLookback predecessors per step: their words
    // are loaded together (independent loads in flight), then consumed
    // nearest first, re-polling (bounded) only those not yet published.
    // Inspecting many predecessors per round trip keeps the first wave of
    // tiles from forming a chain of one L2 round trip per tile.
    constexpr int kLookback = GS_SORT_LOOKBACK;
    int top = tile - 1;
    bool found = false;
    while (!found && top >= 0) {
      uint32_t w[kLookback];
#pragma unroll
      for (int q = 0; q < kLookback; ++q) {
        const int j = top - q;
        w[q] = (j >= 0) ? ld_volatile_u32(lookback + (size_t)j * 256 + d) : kLbPrefix;
      }
#pragma unroll
      for (int q = 0; q < kLookback; ++q) {
        if (found) break;
        const int j = top - q;
        uint32_t x = w[q];
        uint32_t spins = 0;
        while ((x >> 30) == 0 && ++spins < kSpinLimit) x = ld_volatile_u32(lookback + (size_t)j * 256 + d);
        if ((x >> 30) == 0) {
          atomicExch(status, (uint32_t)GS_ERR_DEVICE_TIMEOUT);
          found = true;
          break;
        }
        excl += x & kLbValue;  // (j < 0 contributes a zero prefix)
        if ((x >> 30) == 2) found = true;
      }
      top -= kLookback;
    }
    st_volatile_u32(my_lb, kLbPrefix | ((excl + cnt) & kLbValue));
  }
  const uint32_t gdig = block_scan_256(hist[d], S.tmp);
  const uint32_t ldig = block_scan_256(cnt, S.tmp);
  S.gbase[d] = gdig + excl - ldig;  // output index = gbase[digit] + position in the tile
  S.lstart[d] = ldig;
  __syncthreads();

  // Shuffle into digit order in shared memory.
#pragma unroll
  for (int k = 0; k < ITEMS; ++k) {
    const int64_t idx = base + k * 32 + lane;
    if (idx < n) {
      const uint32_t dk = digit_of(key[k], shift, dmask);
      const uint32_t pos = S.lstart[dk] + S.whist[warp][dk] + rank[k];
      S.keys[pos] = key[k];
      S.vals[pos] = val[k];
    }
  }
  __syncthreads();

  const int64_t tile_base = (int64_t)tile * kTileItems;
  const int valid_count = (int)min((int64_t)kTileItems, n - tile_base);
#pragma unroll
  for (int k = 0; k < ITEMS; ++k) {
    const int p = t + k * kSortThreads;
    if (p < valid_count) {
      const KT kk = S.keys[p];
      const uint32_t out = S.gbase[digit_of(kk, shift, dmask)] + (uint32_t)p;
      if ((int64_t)out < n) {  // always true unless a look-back gave up
        keys_out[out] = kk;
        vals_out[out] = S.vals[p];
      }
    }
  }
}

// ---- tile layout kernels -------------------------------------------------------

// Pairs in depth order. Thread i takes the i-th Gaussian of the depth sort
// and its output range at offsets[i] (exclusive scan of the counts in depth
// order). Rectangles of up to kSmallRect tiles are written by their own
// thread; larger ones by the whole warp, one Gaussian at a time, lane q
// writing the rectangle's q-th tile in row-major order (contiguous stores). The digit
// histograms of the following tile-id sort (passes of 8 bits over tbits bits)
// are counted on the way (per-block shared counters, one global atomic per
// non-zero bin per block), which saves the sort a read of the keys.
constexpr int kSmallRect = 8;

template <typename KT>
__device__ __forceinline__ void emit_one(int64_t o, int tile, int g, KT *keys, int32_t *vals,
                                         uint32_t *s_hist, int tpasses) {
  keys[o] = (KT)tile;
  vals[o] = g;
  atomicAdd(&s_hist[tile & 255], 1u);
  if (tpasses > 1) atomicAdd(&s_hist[256 + ((tile >> 8) & 255)], 1u);
  if (tpasses > 2) atomicAdd(&s_hist[512 + ((tile >> 16) & 255)], 1u);
}

template <typename KT>
__global__ void __launch_bounds__(256) emit_pairs_kernel(int n, const int32_t *__restrict__ order,
                                                         const int32_t *__restrict__ counts,
                                                         const int32_t *__restrict__ offsets,
                                                         const float2 *__restrict__ points,
                                                         const float2 *__restrict__ radii,
                                                         int width, int height, int64_t total,
                                                         int tpasses, KT *__restrict__ keys,
                                                         int32_t *__restrict__ vals,
                                                         uint32_t *__restrict__ hist,
                                                         const int64_t *__restrict__ total_dev,
                                                         uint32_t *status) {
  // capacity form: `total` is the capacity of keys / vals and *total_dev the
  // scan's pair total; beyond the capacity nothing is emitted and the
  // status word records GS_ERR_CAPACITY
  if (total_dev) {
    const int64_t real = *total_dev;
    if (real > total || real < 0) {
      if (blockIdx.x == 0 && threadIdx.x == 0) atomicCAS(status, 0u, (uint32_t)GS_ERR_CAPACITY);
      return;
    }
    total = real;
  }
  __shared__ uint32_t s_hist[3 * 256];
  for (int k = threadIdx.x; k < tpasses * 256; k += blockDim.x) s_hist[k] = 0;
  __syncthreads();
  const int lane = threadIdx.x & 31;
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  const int tx = tiles_x_of(width);
  int g = -1, x0 = 0, y0 = 0, w = 0, h = 0;
  int64_t base = 0;
  if (i < n) {
    const int gg = order[i];
    if (gg >= 0 && gg < n && counts[gg] > 0) {
      const float2 p = points[gg], r = radii[gg];
      const TileRect tr = tile_rect(p.x, p.y, r.x, r.y, width, height);
      base = offsets[i];
      w = tr.x1 - tr.x0 + 1;
      h = tr.y1 - tr.y0 + 1;
      if (!tr.empty && base >= 0 && base + (int64_t)w * h <= total) {  // else: corrupted offsets
        g = gg;
        x0 = tr.x0;
        y0 = tr.y0;
      }
    }
  }
  const bool big = g >= 0 && w * h > kSmallRect;
  if (g >= 0 && !big) {
    int64_t o = base;
    for (int y = y0; y < y0 + h; ++y)
      for (int x = x0; x < x0 + w; ++x) emit_one<KT>(o++, y * tx + x, g, keys, vals, s_hist, tpasses);
  }
  uint32_t todo = __ballot_sync(0xffffffffu, big);
  while (todo) {
    const int j = __ffs(todo) - 1;
    todo &= todo - 1;
    const int gj = __shfl_sync(0xffffffffu, g, j);
    const int xj = __shfl_sync(0xffffffffu, x0, j), yj = __shfl_sync(0xffffffffu, y0, j);
    const int wj = __shfl_sync(0xffffffffu, w, j), hj = __shfl_sync(0xffffffffu, h, j);
    const int64_t bj = __shfl_sync(0xffffffffu, base, j);
    const int area = wj * hj;
    for (int q = lane; q < area; q += 32) {
      const int r = q / wj, c = q - r * wj;
      emit_one<KT>(bj + q, (yj + r) * tx + xj + c, gj, keys, vals, s_hist, tpasses);
    }
  }
  __syncthreads();
  for (int k = threadIdx.x; k < tpasses * 256; k += blockDim.x)
    if (s_hist[k]) atomicAdd(&hist[k], s_hist[k]);
}

// Per-tile start offsets from the sorted tile ids (kernel.cu:875-914): one
// thread per 8 consecutive ids (a 16-byte load for 16-bit ids), comparing
// each id with its predecessor and filling the offsets of the tiles in
// between.
template <typename KT>
__global__ void __launch_bounds__(256) ranges_kernel(const KT *__restrict__ tiles_sorted,
                                                     int64_t n, int num_tiles,
                                                     int32_t *__restrict__ offsets,
                                                     const int64_t *__restrict__ n_dev) {
  constexpr int kPer = 8;
  // capacity form: the count from the device, and offsets[num_tiles] = the
  // end of the last tile's list
  if (n_dev) {
    n = capped_count(n_dev, n);
    if (blockIdx.x == 0 && threadIdx.x == 0) offsets[num_tiles] = (int32_t)n;
  }
  const int64_t stride = (int64_t)gridDim.x * blockDim.x * kPer;
  for (int64_t k0 = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) * kPer; k0 < n; k0 += stride) {
    KT v[kPer];
    if (k0 + kPer <= n && sizeof(KT) * kPer == 16) {
      const uint4 raw = *reinterpret_cast<const uint4 *>(tiles_sorted + k0);
      const KT *pv = reinterpret_cast<const KT *>(&raw);
#pragma unroll
      for (int q = 0; q < kPer; ++q) v[q] = pv[q];
    } else {
#pragma unroll
      for (int q = 0; q < kPer; ++q) v[q] = (k0 + q < n) ? tiles_sorted[k0 + q] : (KT)0;
    }
    int prev = (k0 == 0) ? -1 : min((int)tiles_sorted[k0 - 1], num_tiles - 1);
#pragma unroll
    for (int q = 0; q < kPer; ++q) {
      const int64_t k = k0 + q;
      if (k >= n) break;
      const int tile = min((int)v[q], num_tiles - 1);
      for (int t = prev + 1; t <= tile; ++t) offsets[t] = (int32_t)k;
      prev = tile;
      if (k == n - 1)
        for (int t = tile + 1; t < num_tiles; ++t) offsets[t] = (int32_t)n;
    }
  }
}

// The reference's 64-bit keys (tile << 32 | depth bits) of the sorted pairs,
// for callers that ask for them.
template <typename KT>
__global__ void __launch_bounds__(256) full_keys_kernel(const KT *__restrict__ tiles_sorted,
                                                        const int32_t *__restrict__ ids,
                                                        const float *__restrict__ depths,
                                                        int64_t n, uint64_t *__restrict__ out) {
  const int64_t k = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (k >= n) return;
  out[k] = ((uint64_t)tiles_sorted[k] << 32) | (uint64_t)__float_as_uint(depths[ids[k]]);
}

// ---- host-side sort driver -------------------------------------------------------

struct SortLayout {
  size_t hist, lookback, tickets, total;
  int tiles;
};

template <typename KT>
static SortLayout sort_layout(int64_t n) {
  constexpr int kTileItems = kSortThreads * SortItems<KT>::value;
  SortLayout L;
  L.tiles = (int)((n + kTileItems - 1) / kTileItems);
  L.hist = 0;
  L.lookback = align_up(L.hist + kMaxPasses * 256 * sizeof(uint32_t), 256);
  L.tickets = align_up(L.lookback + (size_t)kMaxPasses * L.tiles * 256 * sizeof(uint32_t), 256);
  L.total = align_up(L.tickets + kMaxPasses * sizeof(uint32_t), 256);
  return L;
}

static int sm_count() {
  static int cached[64] = {0};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64) return 148;
  if (!cached[dev]) {
    int sms = 148;
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    cached[dev] = sms;
  }
  return cached[dev];
}

// Sorts (keys, vals) on bits [0, end_bit) in ceil(end_bit / 8) passes; the
// result ends in the buffers selected by the parity of the pass count (even:
// keys/vals, odd: alt). vals == nullptr sorts the identity permutation (the
// first pass generates it; vals must then not be read back for an even pass
// count unless it points at storage, so callers pass real buffers when they
// need the even-parity result).
template <typename KT>
static int run_sort(int64_t n, KT *keys, int32_t *vals, KT *keys_alt, int32_t *vals_alt,
                    int end_bit, void *scratch, cudaStream_t st, const int32_t *vals_first = nullptr,
                    bool identity_first = false, const uint32_t *hist_given = nullptr,
                    const int64_t *n_dev = nullptr) {
  constexpr int ITEMS = SortItems<KT>::value;
  const int passes = (end_bit + 7) / 8;
  if (n <= 0 || passes <= 0) return GS_OK;
  if (n > (int64_t)kLbValue) return GS_ERR_CAPACITY;
  SortLayout L = sort_layout<KT>(n);
  unsigned char *base = reinterpret_cast<unsigned char *>(scratch);
  uint32_t *hist = reinterpret_cast<uint32_t *>(base + L.hist);
  uint32_t *lookback = reinterpret_cast<uint32_t *>(base + L.lookback);
  uint32_t *tickets = reinterpret_cast<uint32_t *>(base + L.tickets);
  int rc = cuda_status(cudaMemsetAsync(scratch, 0, L.total, st));
  if (rc) return rc;
  if (hist_given) {
    hist = const_cast<uint32_t *>(hist_given);  // digit counts known in advance
  } else {
    const int64_t hb = (n + 255) / 256;
    const int hblocks = (int)(hb < (int64_t)sm_count() * 4 ? hb : (int64_t)sm_count() * 4);
    sort_histogram_kernel<KT><<<hblocks, 256, 0, st>>>(keys, n, passes, end_bit, hist);
    count_launch();
  }
  // the dynamic shared-memory opt-in is per context: set once per host
  // thread and context
  thread_local unsigned long long attr_ctx = 0;
  const size_t smem = sizeof(SortSmem<KT, ITEMS>);
  const unsigned long long ctx = current_context_id();
  if (ctx == 0 || attr_ctx != ctx) {
    rc = cuda_status(cudaFuncSetAttribute(onesweep_pass_kernel<KT, ITEMS>,
                                          cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    if (rc) return rc;
    attr_ctx = ctx;
  }
  KT *kin = keys, *kout = keys_alt;
  int32_t *vin = vals, *vout = vals_alt;
  for (int p = 0; p < passes; ++p) {
    const int bits = end_bit - 8 * p < 8 ? end_bit - 8 * p : 8;
    const int32_t *vsrc = (p == 0) ? (identity_first ? nullptr : (vals_first ? vals_first : vin)) : vin;
    onesweep_pass_kernel<KT, ITEMS><<<L.tiles, kSortThreads, smem, st>>>(
        kin, vsrc, kout, vout, n, 8 * p, (1u << bits) - 1u, hist + 256 * p,
        lookback + (size_t)p * L.tiles * 256, tickets + p, device_status_word(), n_dev);
    count_launch();
    KT *tk = kin;
    kin = kout;
    kout = tk;
    int32_t *tv = vin;
    vin = vout;
    vout = tv;
  }
  return launch_status();
}

static int bits_for(int64_t count) {
  int b = 0;
  while ((1ll << b) < count) ++b;
  return b;
}

// Scratch of the tile layout, carved in this order.
struct LayoutScratch {
  size_t dkeys_a, dkeys_b, dvals_a, dvals_b, offs, total8, thist, tkeys_a, tkeys_b, tvals_b, sort,
      total;
};

static LayoutScratch layout_scratch(int n, int64_t total, int num_tiles) {
  const size_t tk = num_tiles <= 65536 ? 2 : 4;
  const size_t nn = (size_t)(n > 0 ? n : 1), kk = (size_t)(total > 0 ? total : 1);
  LayoutScratch L;
  L.dkeys_a = 0;
  L.dkeys_b = align_up(L.dkeys_a + 4 * nn, 256);
  L.dvals_a = align_up(L.dkeys_b + 4 * nn, 256);
  L.dvals_b = align_up(L.dvals_a + 4 * nn, 256);
  L.offs = align_up(L.dvals_b + 4 * nn, 256);
  L.total8 = align_up(L.offs + 4 * nn, 256);  // the scan's int64 total (8-byte aligned)
  L.thist = align_up(L.total8 + 8, 256);
  L.tkeys_a = align_up(L.thist + kMaxPasses * 256 * 4, 256);
  L.tkeys_b = align_up(L.tkeys_a + tk * kk, 256);
  L.tvals_b = align_up(L.tkeys_b + tk * kk, 256);
  L.sort = align_up(L.tvals_b + 4 * kk, 256);
  const size_t s1 = sort_layout<uint32_t>((int64_t)nn).total;
  const size_t s2 = tk == 2 ? sort_layout<uint16_t>((int64_t)kk).total
                            : sort_layout<uint32_t>((int64_t)kk).total;
  const size_t scan = ((nn + kScanTile - 1) / kScanTile + 1) * sizeof(uint64_t);
  L.total = align_up(L.sort + (s1 > s2 ? (s1 > scan ? s1 : scan) : (s2 > scan ? s2 : scan)), 256);
  return L;
}

template <typename KT>
static int tile_layout_impl(int n, const float2 *points, const float2 *radii, const float *depths,
                            const int32_t *counts, int64_t total, int width, int height,
                            uint64_t *keys_sorted, int32_t *ids_sorted, int32_t *indexing_offset,
                            unsigned char *p, const LayoutScratch &L, cudaStream_t st,
                            bool capped = false, int64_t *total_out = nullptr) {
  // capped: `total` is the capacity of the pair buffers; the pair count is
  // the scan's device total, read by the kernels (no host synchronisation)
  const int num_tiles = tiles_x_of(width) * tiles_y_of(height);
  uint32_t *dk_a = reinterpret_cast<uint32_t *>(p + L.dkeys_a);
  uint32_t *dk_b = reinterpret_cast<uint32_t *>(p + L.dkeys_b);
  int32_t *dv_a = reinterpret_cast<int32_t *>(p + L.dvals_a);
  int32_t *dv_b = reinterpret_cast<int32_t *>(p + L.dvals_b);
  int32_t *offs = reinterpret_cast<int32_t *>(p + L.offs);
  KT *tk_a = reinterpret_cast<KT *>(p + L.tkeys_a);
  KT *tk_b = reinterpret_cast<KT *>(p + L.tkeys_b);
  int32_t *tv_b = reinterpret_cast<int32_t *>(p + L.tvals_b);
  void *sort_scratch = p + L.sort;

  // 1. Gaussians by depth bits (stable, identity values): the depth keys are
  //    copied first so the caller's depths stay untouched.
  int rc = cuda_status(cudaMemcpyAsync(dk_a, depths, (size_t)n * 4, cudaMemcpyDeviceToDevice, st));
  if (rc) return rc;
  rc = run_sort<uint32_t>(n, dk_a, dv_a, dk_b, dv_b, 32, sort_scratch, st, nullptr, true);
  if (rc) return rc;
  const int32_t *order = dv_a;  // 4 passes: even, the result is back in (dk_a, dv_a)

  // 2. exclusive scan of the counts in depth order
  const int stiles = (n + kScanTile - 1) / kScanTile;
  rc = cuda_status(cudaMemsetAsync(sort_scratch, 0, (size_t)(stiles + 1) * 8, st));
  if (rc) return rc;
  int64_t *tot_dev = total_out ? total_out : reinterpret_cast<int64_t *>(p + L.total8);
  scan_kernel<<<stiles, kScanThreads, 0, st>>>(n, counts, order, offs, tot_dev,
                                               reinterpret_cast<uint64_t *>(sort_scratch), stiles,
                                               device_status_word());
  count_launch();

  // 3. pairs in depth order (with the tile sort's digit histograms)
  const int tbits = bits_for(num_tiles) > 0 ? bits_for(num_tiles) : 1;
  const int tpasses = (tbits + 7) / 8;
  uint32_t *thist = reinterpret_cast<uint32_t *>(p + L.thist);
  rc = cuda_status(cudaMemsetAsync(thist, 0, kMaxPasses * 256 * 4, st));
  if (rc) return rc;
  KT *k0 = (tpasses & 1) ? tk_b : tk_a;
  int32_t *v0 = (tpasses & 1) ? tv_b : ids_sorted;
  KT *k1 = (tpasses & 1) ? tk_a : tk_b;
  int32_t *v1 = (tpasses & 1) ? ids_sorted : tv_b;
  emit_pairs_kernel<KT><<<(n + 255) / 256, 256, 0, st>>>(n, order, counts, offs, points, radii,
                                                         width, height, total, tpasses, k0, v0,
                                                         thist, capped ? tot_dev : nullptr,
                                                         device_status_word());
  count_launch();
  // 4. stable sort by tile id; the sorted ids land in (tk_a, ids_sorted)
  rc = run_sort<KT>(total, k0, v0, k1, v1, tbits, sort_scratch, st, nullptr, false, thist,
                    capped ? tot_dev : nullptr);
  if (rc) return rc;
  // 5. tile ranges
  {
    const int64_t want = (total + 256 * 8 - 1) / (256 * 8);
    const int grid = (int)(want < (int64_t)sm_count() * 16 ? want : (int64_t)sm_count() * 16);
    ranges_kernel<KT><<<grid, 256, 0, st>>>(tk_a, total, num_tiles, indexing_offset,
                                            capped ? tot_dev : nullptr);
    count_launch();
  }
  if (keys_sorted) {
    full_keys_kernel<KT><<<(unsigned)((total + 255) / 256), 256, 0, st>>>(tk_a, ids_sorted, depths,
                                                                          total, keys_sorted);
    count_launch();
  }
  return launch_status();
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
  scan_kernel<<<tiles, kScanThreads, 0, st>>>(n, counts, nullptr, offsets, total_dev,
                                              reinterpret_cast<uint64_t *>(scratch), tiles,
                                              device_status_word());
  count_launch();
  return launch_status();
}

extern "C" size_t gs_sort_scratch_bytes(int64_t n) {
  return sort_layout<uint64_t>(n > 0 ? n : 1).total;
}

extern "C" int gs_sort_pairs(int64_t n, uint64_t *keys, int32_t *vals, uint64_t *keys_alt,
                             int32_t *vals_alt, int end_bit, void *scratch,
                             size_t scratch_bytes, void *stream) {
  if (n < 0 || end_bit < 0 || end_bit > 64) return GS_ERR_INVALID_ARGUMENT;
  if (n == 0 || end_bit == 0) return GS_OK;
  if (scratch == nullptr || scratch_bytes < gs_sort_scratch_bytes(n)) return GS_ERR_CAPACITY;
  int passes = (end_bit + 7) / 8;
  cudaStream_t st = as_stream(stream);
  int rc = run_sort<uint64_t>(n, keys, vals, keys_alt, vals_alt, end_bit, scratch, st);
  if (rc) return rc;
  if (passes & 1) {
    rc = cuda_status(cudaMemcpyAsync(keys, keys_alt, n * sizeof(uint64_t), cudaMemcpyDeviceToDevice, st));
    if (rc) return rc;
    rc = cuda_status(cudaMemcpyAsync(vals, vals_alt, n * sizeof(int32_t), cudaMemcpyDeviceToDevice, st));
  }
  return rc;
}

extern "C" size_t gs_tile_layout_scratch_bytes(int n, int64_t total, int width, int height) {
  return layout_scratch(n, total, tiles_x_of(width) * tiles_y_of(height)).total;
}

extern "C" int gs_tile_layout(int n, const float *points_img, const float *radii,
                              const float *depths, const int32_t *counts, int64_t total,
                              int width, int height, int64_t *keys_sorted, int32_t *ids_sorted,
                              int32_t *indexing_offset, void *scratch, size_t scratch_bytes,
                              void *stream) {
  if (n < 0 || width <= 0 || height <= 0 || total < 0) return GS_ERR_INVALID_ARGUMENT;
  if (((uintptr_t)points_img & 7) || ((uintptr_t)radii & 7)) return GS_ERR_INVALID_ARGUMENT;
  if (total >= (int64_t)kLbValue) return GS_ERR_CAPACITY;
  cudaStream_t st = as_stream(stream);
  const int num_tiles = tiles_x_of(width) * tiles_y_of(height);
  if (num_tiles > (1 << 24)) return GS_ERR_CAPACITY;  // tile ids sorted in at most 3 passes
  // rasterizer.cpp:352: offsets start at zero; with no pairs they stay zero.
  int rc = cuda_status(cudaMemsetAsync(indexing_offset, 0, (size_t)num_tiles * sizeof(int32_t), st));
  if (rc || total == 0 || n == 0) return rc;
  const LayoutScratch L = layout_scratch(n, total, num_tiles);
  if (scratch == nullptr || scratch_bytes < L.total) return GS_ERR_CAPACITY;
  unsigned char *p = reinterpret_cast<unsigned char *>(scratch);
  const float2 *pts = reinterpret_cast<const float2 *>(points_img);
  const float2 *rad = reinterpret_cast<const float2 *>(radii);
  uint64_t *ks = reinterpret_cast<uint64_t *>(keys_sorted);
  if (num_tiles <= 65536)
    return tile_layout_impl<uint16_t>(n, pts, rad, depths, counts, total, width, height, ks,
                                      ids_sorted, indexing_offset, p, L, st);
  return tile_layout_impl<uint32_t>(n, pts, rad, depths, counts, total, width, height, ks,
                                    ids_sorted, indexing_offset, p, L, st);
}

extern "C" int gs_tile_layout_capped(int n, const float *points_img, const float *radii,
                                     const float *depths, const int32_t *counts,
                                     int64_t capacity, int width, int height,
                                     int32_t *ids_sorted, int32_t *indexing_offset,
                                     int64_t *total_dev, void *scratch, size_t scratch_bytes,
                                     void *stream) {
  if (n < 0 || width <= 0 || height <= 0 || capacity < 0) return GS_ERR_INVALID_ARGUMENT;
  if (((uintptr_t)points_img & 7) || ((uintptr_t)radii & 7) || ((uintptr_t)total_dev & 7))
    return GS_ERR_INVALID_ARGUMENT;
  if (total_dev == nullptr) return GS_ERR_INVALID_ARGUMENT;
  if (capacity >= (int64_t)kLbValue) return GS_ERR_CAPACITY;
  cudaStream_t st = as_stream(stream);
  const int num_tiles = tiles_x_of(width) * tiles_y_of(height);
  if (num_tiles > (1 << 24)) return GS_ERR_CAPACITY;
  // num_tiles start offsets and the end of the last list, zero until written
  int rc = cuda_status(
      cudaMemsetAsync(indexing_offset, 0, (size_t)(num_tiles + 1) * sizeof(int32_t), st));
  if (rc) return rc;
  rc = cuda_status(cudaMemsetAsync(total_dev, 0, sizeof(int64_t), st));
  if (rc || n == 0) return rc;
  const int64_t cap = capacity > 0 ? capacity : 1;
  const LayoutScratch L = layout_scratch(n, cap, num_tiles);
  if (scratch == nullptr || scratch_bytes < L.total) return GS_ERR_CAPACITY;
  unsigned char *p = reinterpret_cast<unsigned char *>(scratch);
  const float2 *pts = reinterpret_cast<const float2 *>(points_img);
  const float2 *rad = reinterpret_cast<const float2 *>(radii);
  if (num_tiles <= 65536)
    return tile_layout_impl<uint16_t>(n, pts, rad, depths, counts, cap, width, height, nullptr,
                                      ids_sorted, indexing_offset, p, L, st, true, total_dev);
  return tile_layout_impl<uint32_t>(n, pts, rad, depths, counts, cap, width, height, nullptr,
                                    ids_sorted, indexing_offset, p, L, st, true, total_dev);
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

// Device address of g_noalloc_scan_words in the current context (host code
// may not use the symbol itself as a pointer): cudaGetSymbolAddress, cached
// per host thread against the context's id.
static int noalloc_scan_words(uint64_t **out) {
  thread_local SymbolCache cache;
  void *p = nullptr;
  int rc = symbol_address(&g_noalloc_scan_words, &cache, &p);
  if (rc) return rc;
  *out = reinterpret_cast<uint64_t *>(p);
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
  scan_kernel<<<tiles, kScanThreads, 0, st>>>(n, counts, nullptr, offsets, total_dev, words,
                                              tiles, device_status_word());
  count_launch();
  return launch_status();
}
