// binning.cu -- the tile layout by binning: per-tile buckets, then a sort of
// each bucket on its own.
//
// The reference orders the (tile, Gaussian) pairs with one stable sort of 64-bit
// keys (tile << 32 | depth bits) over every pair of the view
// (ruguangyou/3dgs_from_scratch src/cuda/kernel.cu:820-873 key emission and
// the CUB sort of kernel.cu:1341-1388), then finds the tile ranges
// (kernel.cu:875-914). Within a tile that order is: depth bits ascending, ties
// by Gaussian id (the emission order, kept by the stable sort) -- i.e. the
// order of the unique 64-bit key (depth bits << 32 | id). This file gets the
// same lists without any sort over all pairs:
//   1. bin_count_kernel: every Gaussian adds one to the counter of each tile
//      its rectangle covers (a Gaussian per thread; rectangles of more than
//      kSmallRect tiles by the whole warp);
//   2. bin_scan_kernel (one block): exclusive scan of the tile counters --
//      the per-tile start offsets (indexing_offset), the total, and the
//      capacity check (beyond the capacity every list is left empty and
//      GS_ERR_CAPACITY recorded);
//   3. bin_scatter_kernel: every Gaussian takes a slot in each of its tiles'
//      buckets with an atomic cursor and writes its id there (the bucket is
//      then complete but in arbitrary order);
//   4. bin_sort_kernel: one block per tile sorts its bucket by the key
//      (depth bits << 32 | id), built from the view's depths: buckets of up
//      to 2048 entries by 256 threads as a block radix sort of the depth
//      bits (ties then put in id order); longer ones, listed by that kernel,
//      by 1024-thread blocks (bin_sort_long_kernel) up to 8192 entries in
//      registers and shared memory (a sorting network on each thread's 8
//      keys, then merge-path merges of sorted runs), beyond that as sorted
//      chunks merged run by run through global scratch.
// With up to kMaxPrivTiles tiles, steps 1 and 3 keep the tile counters in
// shared memory per block (bin_hist_kernel, bin_colscan_kernel,
// bin_place_kernel) instead of global atomics.
// Every key is unique, so any correct sort yields the reference's order bit
// for bit. No host synchronisation: the pair count stays on the device.
#include "gs_common.cuh"

namespace gs {
namespace binning {

constexpr int kItems = 8;
constexpr int kSmallRect = 8;
constexpr uint64_t kPad = ~0ull;  // sorts after every real key

struct Ctl {
  int32_t overflow;   // set by the scan when the total exceeds the capacity
  int32_t num_long;   // buckets longer than the mid sort's chunk, listed in long_tiles
  int32_t num_mid;    // buckets longer than the short sort's chunk, listed in mid_tiles
};

// The tiles of one Gaussian's rectangle, row-major, q-th of them.
__device__ __forceinline__ int rect_tile(const TileRect &r, int q, int tx) {
  const int w = r.x1 - r.x0 + 1;
  const int row = q / w, col = q - row * w;
  return (r.y0 + row) * tx + r.x0 + col;
}

// One Gaussian's inputs, loaded together (the three loads are independent).
struct PairSrc {
  float2 p, rd;
  int count;
};

__device__ __forceinline__ PairSrc load_pair_src(int i, bool valid,
                                                 const float2 *__restrict__ points,
                                                 const float2 *__restrict__ radii,
                                                 const int32_t *__restrict__ counts) {
  PairSrc g{make_float2(0.f, 0.f), make_float2(0.f, 0.f), 0};
  if (valid) {
    g.count = counts[i];
    g.p = points[i];
    g.rd = radii[i];
  }
  return g;
}

// Visits every (Gaussian, tile) pair of Gaussian i (valid: i < n): small
// rectangles by the calling thread, larger ones by the whole warp (lane q
// takes the rectangle's q-th, q+32-th, ... tile). f(tile, gaussian). Called
// by whole warps (every lane, valid or not).
template <typename F>
__device__ __forceinline__ void pairs_from(int i, bool valid, const PairSrc &g, int width,
                                           int height, F f) {
  const int lane = threadIdx.x & 31;
  const int tx = tiles_x_of(width);
  TileRect r{0, -1, 0, -1, true};
  int area = 0;
  if (valid && g.count > 0) {
    r = tile_rect(g.p.x, g.p.y, g.rd.x, g.rd.y, width, height);
    if (!r.empty) area = (r.x1 - r.x0 + 1) * (r.y1 - r.y0 + 1);
  }
  const bool big = area > kSmallRect;
  if (area > 0 && !big)
    for (int q = 0; q < area; ++q) f(rect_tile(r, q, tx), i);
  uint32_t todo = __ballot_sync(0xffffffffu, big);
  while (todo) {
    const int j = __ffs(todo) - 1;
    todo &= todo - 1;
    TileRect rj;
    rj.x0 = __shfl_sync(0xffffffffu, r.x0, j);
    rj.x1 = __shfl_sync(0xffffffffu, r.x1, j);
    rj.y0 = __shfl_sync(0xffffffffu, r.y0, j);
    rj.y1 = __shfl_sync(0xffffffffu, r.y1, j);
    const int aj = __shfl_sync(0xffffffffu, area, j);
    const int gj = __shfl_sync(0xffffffffu, i, j);
    for (int q = lane; q < aj; q += 32) f(rect_tile(rj, q, tx), gj);
  }
}

template <typename F>
__device__ __forceinline__ void pairs_of(int i, bool valid, const float2 *__restrict__ points,
                                         const float2 *__restrict__ radii,
                                         const int32_t *__restrict__ counts, int width,
                                         int height, F f) {
  pairs_from(i, valid, load_pair_src(i, valid, points, radii, counts), width, height, f);
}

// A block's contiguous range [lo, hi) of Gaussians, kPrivThreads at a time,
// the next Gaussian's inputs loaded while the current one's pairs are made.
template <int THREADS, typename F>
__device__ __forceinline__ void pairs_of_range(int lo, int hi, const float2 *__restrict__ points,
                                               const float2 *__restrict__ radii,
                                               const int32_t *__restrict__ counts, int width,
                                               int height, F f) {
  int i = lo + (int)threadIdx.x;
  PairSrc cur = load_pair_src(i, i < hi, points, radii, counts);
  for (int base = lo; base < hi; base += THREADS) {  // block-uniform trip count
    const int inext = i + THREADS;
    const PairSrc next = load_pair_src(inext, inext < hi, points, radii, counts);
    pairs_from(i, i < hi, cur, width, height, f);
    i = inext;
    cur = next;
  }
}

// One Gaussian per thread over the grid.
template <typename F>
__device__ __forceinline__ void for_each_pair(int n, const float2 *__restrict__ points,
                                              const float2 *__restrict__ radii,
                                              const int32_t *__restrict__ counts, int width,
                                              int height, F f) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  pairs_of(i, i < n, points, radii, counts, width, height, f);
}

__global__ void __launch_bounds__(256) bin_count_kernel(int n, const float2 *__restrict__ points,
                                                        const float2 *__restrict__ radii,
                                                        const int32_t *__restrict__ counts,
                                                        int width, int height,
                                                        uint32_t *__restrict__ tile_count) {
  for_each_pair(n, points, radii, counts, width, height,
                [&](int tile, int) { atomicAdd(tile_count + tile, 1u); });
}

// One block of 1024 threads: exclusive scan of the T tile counters into
// offsets[0..T-1], offsets[T] = total, cursor = offsets; *total_dev = total.
// A total beyond `capacity` leaves offsets (and the cursors) zero, raises
// ctl->overflow and records GS_ERR_CAPACITY.
constexpr int kScanThreads = 1024;
constexpr int kScanPer = 4;

__device__ __forceinline__ long long block_excl_scan_ll(long long x, long long *s_warp,
                                                        long long &block_total) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  long long incl = x;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const long long y = __shfl_up_sync(0xffffffffu, incl, o);
    if (lane >= o) incl += y;
  }
  if (lane == 31) s_warp[warp] = incl;
  __syncthreads();
  if (warp == 0) {
    const long long w = s_warp[lane];
    long long wi = w;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const long long y = __shfl_up_sync(0xffffffffu, wi, o);
      if (lane >= o) wi += y;
    }
    s_warp[lane] = wi - w;
    if (lane == 31) s_warp[32] = wi;
  }
  __syncthreads();
  const long long r = incl - x + s_warp[warp];
  block_total = s_warp[32];
  __syncthreads();
  return r;
}

__global__ void __launch_bounds__(kScanThreads) bin_scan_kernel(
    const uint32_t *__restrict__ tile_count, int T, int64_t capacity,
    int32_t *__restrict__ offsets, uint32_t *__restrict__ cursor, int64_t *__restrict__ total_dev,
    Ctl *ctl, uint32_t *status, int32_t *__restrict__ tile_order) {
  __shared__ long long s_warp[33];
  __shared__ uint32_t s_class[kOrderClasses];
  const int t = threadIdx.x;
  // pass 1: the total
  long long sum = 0;
  for (int k = t; k < T; k += kScanThreads) sum += tile_count[k];
  long long total = 0;
  block_excl_scan_ll(sum, s_warp, total);
  const bool over = total > capacity;
  if (t == 0) {
    *total_dev = total;
    ctl->overflow = over ? 1 : 0;
    if (over) atomicCAS(status, 0u, (uint32_t)GS_ERR_CAPACITY);
  }
  if (tile_order != nullptr)  // the blend order (every list empty beyond the capacity)
    tile_order_block(T, [&](int k) { return over ? 0 : (int)tile_count[k]; }, tile_order,
                     s_class);
  if (over) {  // block-uniform
    for (int k = t; k <= T; k += kScanThreads) offsets[k] = 0;
    return;
  }
  // pass 2: the offsets, kScanPer consecutive counters per thread per round
  long long carry = 0;
  for (int base = 0; base < T; base += kScanThreads * kScanPer) {
    const int k0 = base + t * kScanPer;
    uint32_t v[kScanPer];
    long long s = 0;
#pragma unroll
    for (int q = 0; q < kScanPer; ++q) {
      v[q] = (k0 + q < T) ? tile_count[k0 + q] : 0u;
      s += v[q];
    }
    long long round_total = 0;
    long long run = carry + block_excl_scan_ll(s, s_warp, round_total);
#pragma unroll
    for (int q = 0; q < kScanPer; ++q) {
      if (k0 + q < T) {
        offsets[k0 + q] = (int32_t)run;
        cursor[k0 + q] = (uint32_t)run;
      }
      run += v[q];
    }
    carry += round_total;
  }
  if (t == 0) offsets[T] = (int32_t)total;
}

__global__ void __launch_bounds__(256) bin_scatter_kernel(int n, const float2 *__restrict__ points,
                                                          const float2 *__restrict__ radii,
                                                          const int32_t *__restrict__ counts,
                                                          int width, int height, int64_t capacity,
                                                          uint32_t *__restrict__ cursor,
                                                          int32_t *__restrict__ ids,
                                                          const Ctl *ctl) {
  if (ctl->overflow) return;  // grid-uniform
  for_each_pair(n, points, radii, counts, width, height, [&](int tile, int g) {
    const uint32_t pos = atomicAdd(cursor + tile, 1u);
    if ((int64_t)pos < capacity) ids[pos] = g;  // always true unless the inputs changed
  });
}

// ---- privatised binning (no global atomics) -----------------------------------
//
// With up to kMaxPrivTiles tiles, every block keeps all the tile counters in
// shared memory: block b counts the pairs of its contiguous Gaussian range
// (bin_hist_kernel, one row hist[b][0..T) per block), a column scan turns the
// rows into each block's base within every tile (bin_colscan_kernel), and the
// placement (bin_place_kernel) hands out slots from shared-memory cursors
// started at offsets[t] + hist[b][t]. The global atomics of the direct kernels
// above, ~600 on each tile counter at config 1, serialise in L2; here each
// tile counter in global memory is read and written once per block.
constexpr int kPrivThreads = 512;
constexpr int kMaxPrivTiles = 24576;  // 96 KB of shared counters

__device__ __forceinline__ void block_gaussian_range(int n, int &lo, int &hi) {
  const int per = (n + gridDim.x - 1) / gridDim.x;
  lo = min(n, blockIdx.x * per);
  hi = min(n, lo + per);
}

__global__ void __launch_bounds__(kPrivThreads) bin_hist_kernel(
    int n, const float2 *__restrict__ points, const float2 *__restrict__ radii,
    const int32_t *__restrict__ counts, int width, int height, int T,
    uint32_t *__restrict__ hist) {
  extern __shared__ uint32_t s_cnt[];
  for (int k = threadIdx.x; k < T; k += kPrivThreads) s_cnt[k] = 0u;
  __syncthreads();
  int lo, hi;
  block_gaussian_range(n, lo, hi);
  pairs_of_range<kPrivThreads>(lo, hi, points, radii, counts, width, height,
                               [&](int tile, int) { atomicAdd(s_cnt + tile, 1u); });
  __syncthreads();
  uint32_t *row = hist + (size_t)blockIdx.x * T;
  for (int k = threadIdx.x; k < T; k += kPrivThreads) row[k] = s_cnt[k];
}

// The rows become exclusive prefixes over the blocks, the column totals the
// tiles' counts. A block takes 32 tiles (a warp's lanes, coalesced across
// each row) and splits the rows into kColSlices slices, one per warp: slice
// sums, their prefix over the slices in shared memory, then the rewrite.
constexpr int kColSlices = 16;

__global__ void __launch_bounds__(32 * kColSlices) bin_colscan_kernel(
    int T, int B, uint32_t *__restrict__ hist, uint32_t *__restrict__ tile_count) {
  __shared__ uint32_t s_part[kColSlices][32];
  const int lane = threadIdx.x & 31, slice = threadIdx.x >> 5;
  const int t = blockIdx.x * 32 + lane;
  const int per = (B + kColSlices - 1) / kColSlices;
  const int b0 = min(B, slice * per), b1 = min(B, b0 + per);
  uint32_t sum = 0;
  if (t < T)
    for (int b = b0; b < b1; ++b) sum += hist[(size_t)b * T + t];
  s_part[slice][lane] = sum;
  __syncthreads();
  uint32_t run = 0;
  for (int q = 0; q < slice; ++q) run += s_part[q][lane];
  if (t < T) {
    for (int b = b0; b < b1; ++b) {
      const uint32_t v = hist[(size_t)b * T + t];
      hist[(size_t)b * T + t] = run;
      run += v;
    }
    if (slice == kColSlices - 1) tile_count[t] = run;
  }
}

__global__ void __launch_bounds__(kPrivThreads) bin_place_kernel(
    int n, const float2 *__restrict__ points, const float2 *__restrict__ radii,
    const int32_t *__restrict__ counts, int width, int height, int T,
    const uint32_t *__restrict__ hist, const int32_t *__restrict__ offsets,
    int32_t *__restrict__ ids, const Ctl *ctl) {
  if (ctl->overflow) return;  // grid-uniform
  extern __shared__ uint32_t s_cur[];
  const uint32_t *row = hist + (size_t)blockIdx.x * T;
  for (int k = threadIdx.x; k < T; k += kPrivThreads) s_cur[k] = (uint32_t)offsets[k] + row[k];
  __syncthreads();
  int lo, hi;
  block_gaussian_range(n, lo, hi);
  pairs_of_range<kPrivThreads>(lo, hi, points, radii, counts, width, height,
                               [&](int tile, int g) { ids[atomicAdd(s_cur + tile, 1u)] = g; });
}

// ---- per-tile sort ---------------------------------------------------------

__device__ __forceinline__ void cswap(uint64_t &a, uint64_t &b) {
  const uint64_t lo = a < b ? a : b, hi = a < b ? b : a;
  a = lo;
  b = hi;
}

// Batcher's odd-even merge sort network for 8 keys (19 comparators).
__device__ __forceinline__ void sort8(uint64_t k[8]) {
  cswap(k[0], k[1]); cswap(k[2], k[3]); cswap(k[4], k[5]); cswap(k[6], k[7]);
  cswap(k[0], k[2]); cswap(k[1], k[3]); cswap(k[4], k[6]); cswap(k[5], k[7]);
  cswap(k[1], k[2]); cswap(k[5], k[6]);
  cswap(k[0], k[4]); cswap(k[1], k[5]); cswap(k[2], k[6]); cswap(k[3], k[7]);
  cswap(k[2], k[4]); cswap(k[3], k[5]);
  cswap(k[1], k[2]); cswap(k[3], k[4]); cswap(k[5], k[6]);
}

// Merge path: the number of elements taken from A (sorted, length la) among
// the first `diag` outputs of merge(A, B) (B sorted, length lb), ties to A.
template <typename LoadA, typename LoadB>
__device__ __forceinline__ int merge_path(LoadA a, int la, LoadB b, int lb, int diag) {
  int lo = diag > lb ? diag - lb : 0;
  int hi = diag < la ? diag : la;
  while (lo < hi) {
    const int mid = (lo + hi) >> 1;
    if (a(mid) <= b(diag - 1 - mid))
      lo = mid + 1;
    else
      hi = mid;
  }
  return lo;
}

// kItems outputs of merge(A, B) starting at (ai, bi).
template <typename LoadA, typename LoadB>
__device__ __forceinline__ void merge_items(LoadA a, int la, LoadB b, int lb, int ai, int bi,
                                            uint64_t out[kItems]) {
  uint64_t ka = ai < la ? a(ai) : kPad, kb = bi < lb ? b(bi) : kPad;
#pragma unroll
  for (int q = 0; q < kItems; ++q) {
    const bool takeA = (bi >= lb) || (ai < la && ka <= kb);
    out[q] = takeA ? ka : kb;
    if (takeA) {
      ++ai;
      ka = ai < la ? a(ai) : kPad;
    } else {
      ++bi;
      kb = bi < lb ? b(bi) : kPad;
    }
  }
}

// Shared-memory slot of logical position p of a THREADS * kItems chunk:
// item q of every thread is one contiguous row, so that the threads' stores
// of their q-th keys, and the reads of neighbouring merge positions by
// neighbouring threads, fall in distinct banks.
template <int THREADS>
__device__ __forceinline__ int slot_of(int p) {
  return (p & (kItems - 1)) * THREADS + (p >> 3);
}

// Sorts the block's THREADS * kItems keys (kItems per thread, thread t
// holding positions t*kItems..) up to runs of `span` (a power of two >=
// kItems, <= THREADS * kItems): on return thread t holds positions
// t*kItems.. of the sorted chunk. Two barriers per merge level: warp
// barriers while the merged runs fit in a warp, block barriers above.
// A merge level whose merged runs (2 * run keys) fit in one warp's
// 32 * kItems positions only exchanges keys within the warp: it needs a warp
// barrier, not a block barrier.
__device__ __forceinline__ bool warp_level(int run) { return 2 * run <= 32 * kItems; }

__device__ __forceinline__ void level_sync(int run) {
  if (warp_level(run))
    __syncwarp();
  else
    __syncthreads();
}

template <int THREADS>
__device__ __forceinline__ void block_sort(uint64_t k[kItems], int span, uint64_t *s_keys) {
  sort8(k);
  const int t = threadIdx.x;
  for (int run = kItems; run < span; run <<= 1) {
#pragma unroll
    for (int q = 0; q < kItems; ++q) s_keys[q * THREADS + t] = k[q];
    level_sync(run);
    const int pair = 2 * run;
    const int start = (t * kItems) / pair * pair;
    const int diag = t * kItems - start;
    auto la = [&](int i) { return s_keys[slot_of<THREADS>(start + i)]; };
    auto lb = [&](int i) { return s_keys[slot_of<THREADS>(start + run + i)]; };
    const int ai = merge_path(la, run, lb, run, diag);
    merge_items(la, run, lb, run, ai, diag - ai, k);
    level_sync(run);
  }
}

__device__ __forceinline__ uint64_t key_of(int id, const float *__restrict__ depths, int n) {
  const uint32_t d = (id >= 0 && id < n) ? __float_as_uint(depths[id]) : 0xffffffffu;
  return ((uint64_t)d << 32) | (uint32_t)id;
}

__device__ __forceinline__ int next_pow2(int x) {
  int p = kItems;
  while (p < x) p <<= 1;
  return p;
}

// The whole block sorts the bucket ids[beg .. beg + L) in place by (depth
// bits, id). Buckets of up to THREADS * kItems entries are sorted on chip;
// longer ones as sorted chunks of that size written to keys_a, merged run by
// run between keys_a and keys_b (global scratch at the bucket's own
// offsets), the ids taken from the last run. Every thread returns after the
// same barriers.
template <int THREADS>
__device__ void sort_bucket(int beg, int L, const float *__restrict__ depths, int n,
                            int32_t *__restrict__ ids, uint64_t *__restrict__ keys_a,
                            uint64_t *__restrict__ keys_b, uint64_t *s_keys) {
  constexpr int kCh = THREADS * kItems;
  const int t = threadIdx.x;
  uint64_t k[kItems];
  if (L <= kCh) {
    const int span = next_pow2(L);
    // A warp whose positions are all padding only takes part in the block
    // barriers (two per merge level above the warp levels). The test is per
    // warp, so that every barrier is reached by whole warps; threads of an
    // active warp past `span` merge padding (or stale shared memory), and
    // their results are dropped.
    if ((t & ~31) * kItems >= span) {
      for (int run = kItems; run < span; run <<= 1) {
        if (!warp_level(run)) {
          __syncthreads();
          __syncthreads();
        }
      }
      return;
    }
#pragma unroll
    for (int q = 0; q < kItems; ++q) {
      const int p = t * kItems + q;
      k[q] = p < L ? key_of(ids[beg + p], depths, n) : kPad;
    }
    block_sort<THREADS>(k, span, s_keys);
#pragma unroll
    for (int q = 0; q < kItems; ++q) {
      const int p = t * kItems + q;
      if (p < L) ids[beg + p] = (int32_t)(uint32_t)k[q];
    }
    return;
  }
  // long bucket: sorted chunks of kCh into keys_a
  uint64_t *ka = keys_a + beg, *kb = keys_b + beg;
  for (int c0 = 0; c0 < L; c0 += kCh) {
#pragma unroll
    for (int q = 0; q < kItems; ++q) {
      const int p = c0 + t * kItems + q;
      k[q] = p < L ? key_of(ids[beg + p], depths, n) : kPad;
    }
    block_sort<THREADS>(k, kCh, s_keys);
#pragma unroll
    for (int q = 0; q < kItems; ++q) {
      const int p = c0 + t * kItems + q;
      if (p < L) ka[p] = k[q];
    }
  }
  __syncthreads();
  // merge runs of kCh, 2 kCh, ... (ping-pong ka <-> kb)
  for (int run = kCh; run < L; run <<= 1) {
    for (int out0 = 0; out0 < L; out0 += kCh) {
      const int p0 = out0 + t * kItems;  // this thread's first output position
      if (p0 < L) {
        const int start = p0 / (2 * run) * (2 * run);
        const int la_n = min(run, L - start);
        const int lb_n = max(0, min(run, L - start - run));
        const uint64_t *A = ka + start, *B = ka + start + run;
        auto la = [&](int i) { return A[i]; };
        auto lb = [&](int i) { return B[i]; };
        const int diag = p0 - start;
        const int ai = merge_path(la, la_n, lb, lb_n, diag);
        merge_items(la, la_n, lb, lb_n, ai, diag - ai, k);
#pragma unroll
        for (int q = 0; q < kItems; ++q)
          if (p0 + q < L) kb[p0 + q] = k[q];
      }
    }
    __syncthreads();  // the level's writes are visible to the block
    uint64_t *tmp = ka;
    ka = kb;
    kb = tmp;
  }
  for (int p = t; p < L; p += THREADS) ids[beg + p] = (int32_t)(uint32_t)ka[p];
}

// ---- short buckets: block radix sort on the depth bits -----------------------
//
// A bucket of up to kRadChunk entries is sorted by one 256-thread block (up
// to kRadMidChunk by a 512-thread block) as a
// stable LSD radix sort of its 32-bit depth keys (8-bit digits) in shared
// memory. The keys are sorted as their offsets from the bucket's smallest
// key (an order-preserving shift for unsigned keys), so only the bits of the
// bucket's key range are sorted: a tile's depths spanning 5.0 to 12.0 give
// offsets below 2^24, 3 passes, where the bits in which the keys differ
// (their XOR) reach bit 24 and would take 4. Entries with an invalid id, and
// the padding up to whole warps, take a key above every valid one. Each pass ranks
// the digits warp by warp -- lanes with equal digits found with one ballot
// per digit bit, items taken in position order (position 32 (ipw w + k) +
// lane for item k of lane `lane` in warp w, ipw items per lane), so the
// ranking is stable -- scans the per-warp digit counts and
// scatters into the other buffer. Equal depth keys keep the bucket's
// (arbitrary) order, so runs of equal keys are then put in id order: the
// (depth bits, id) order of the reference's stable 64-bit sort.
constexpr int kRadThreads = 256;                    // buckets up to 2048 entries
constexpr int kRadMidThreads = 512;                 // 2049 to 4096 entries
constexpr int kRadItems = 8;
constexpr int kRadChunk = kRadThreads * kRadItems;  // 2048
constexpr int kRadMidChunk = kRadMidThreads * kRadItems;  // 4096

template <int THREADS>
struct RadSmem {
  uint32_t key[2][THREADS * kRadItems];
  int32_t val[2][THREADS * kRadItems];
  uint32_t whist[THREADS / 32][256];
  uint32_t gbase[256];
  uint32_t tmp[THREADS / 32 + 1];
  uint32_t kmin, kmax, invalid;
};

template <int THREADS>
__device__ __forceinline__ uint32_t rad_block_excl_scan(uint32_t x, uint32_t *s_tmp) {
  constexpr int kWarps = THREADS / 32;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  uint32_t incl = x;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const uint32_t y = __shfl_up_sync(0xffffffffu, incl, o);
    if (lane >= o) incl += y;
  }
  if (lane == 31) s_tmp[warp] = incl;
  __syncthreads();
  if (warp == 0) {
    const uint32_t w = lane < kWarps ? s_tmp[lane] : 0u;
    uint32_t wi = w;
#pragma unroll
    for (int o = 1; o < kWarps; o <<= 1) {
      const uint32_t y = __shfl_up_sync(0xffffffffu, wi, o);
      if (lane >= o) wi += y;
    }
    if (lane < kWarps) s_tmp[lane] = wi - w;
  }
  __syncthreads();
  const uint32_t r = incl - x + s_tmp[warp];
  __syncthreads();
  return r;
}

// THREADS = 256 or 512 threads sort a bucket of up to 8 THREADS entries;
// threads 0-255 own the 256 digits in each pass's digit scan.
template <int THREADS>
__device__ void radix_sort_bucket(int beg, int L, const float *__restrict__ depths, int n,
                                  int32_t *__restrict__ ids, RadSmem<THREADS> &S) {
  constexpr int kWarps = THREADS / 32;
  const int t = threadIdx.x, warp = t >> 5;
  const uint32_t lane = t & 31;
  const uint32_t lt_mask = (1u << lane) - 1u;
  // positions [0, 256 ipw): ipw items per lane in every warp (the bucket
  // spread over all warps, so a warp ranks as few items as the bucket
  // allows), the tail padded with a key that sorts after every real key
  // (stable, so the real keys stay first)
  const int ipw = (L + THREADS - 1) / THREADS;  // 1..kRadItems, block-uniform
  if (t == 0) {
    S.kmin = 0xffffffffu;
    S.kmax = 0u;
    S.invalid = 0u;
  }
  __syncthreads();
  uint32_t kmn = 0xffffffffu, kmx = 0u, bad = 0u;
  // positions t + 256 q, q < ipw: every id load first, then the depth loads
  // (one round trip each instead of two per position)
  int32_t vals[kRadItems];
#pragma unroll
  for (int q = 0; q < kRadItems; ++q) {
    if (q >= ipw) break;
    const int p = t + q * THREADS;
    vals[q] = p < L ? ids[beg + p] : -1;
  }
#pragma unroll
  for (int q = 0; q < kRadItems; ++q) {
    if (q >= ipw) break;
    const int p = t + q * THREADS;
    const int32_t val = vals[q];
    uint32_t key = 0xffffffffu;
    if (p < L) {
      if (val >= 0 && val < n) {
        key = __float_as_uint(depths[val]);
        kmn = min(kmn, key);
        kmx = max(kmx, key);
      } else {
        bad = 1u;
      }
    }
    S.key[0][p] = key;
    S.val[0][p] = val;
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    kmn = min(kmn, __shfl_xor_sync(0xffffffffu, kmn, o));
    kmx = max(kmx, __shfl_xor_sync(0xffffffffu, kmx, o));
    bad |= __shfl_xor_sync(0xffffffffu, bad, o);
  }
  if (lane == 0) {
    atomicMin(&S.kmin, kmn);
    atomicMax(&S.kmax, kmx);
    if (bad) S.invalid = 1u;
  }
  __syncthreads();
  // sorted key = key - kmin for a valid entry, `sent` for an invalid one or
  // padding; `bits` covers every sorted key. Padding sits after position L,
  // so with no invalid entry it may tie the largest valid key (the sort is
  // stable); an invalid entry needs a key above every valid one.
  uint32_t kmin = S.kmin;
  const uint32_t kmax = S.kmax;
  const bool has_invalid = S.invalid != 0u;
  int bits;
  if (kmin > kmax) {  // no valid entry: every key is the sentinel
    kmin = 0u;
    bits = 0;
  } else {
    const uint64_t top = (uint64_t)(kmax - kmin) + (has_invalid ? 1u : 0u);
    bits = top ? 64 - __clzll((long long)top) : 0;
    if (bits > 32) {  // keys spanning the whole 32-bit range: sort them as they are
      kmin = 0u;
      bits = 32;
    }
  }
  const uint32_t sent = bits >= 32 ? 0xffffffffu : ((1u << bits) - 1u);
  const int passes = (bits + 7) / 8;
  int cur = 0;
  for (int pass = 0; pass < passes; ++pass) {  // block-uniform
    const int shift = 8 * pass;
    for (int k = t; k < kWarps * 256; k += THREADS) (&S.whist[0][0])[k] = 0u;
    __syncthreads();
    uint32_t key[kRadItems], rank[kRadItems];
    int32_t val[kRadItems];
    {
      uint32_t lead_old[kRadItems];
      uint8_t leader_of[kRadItems];
#pragma unroll
      for (int q = 0; q < kRadItems; ++q) {
        if (q >= ipw) break;  // warp-uniform
        const int p = warp * 32 * ipw + q * 32 + (int)lane;
        key[q] = S.key[cur][p];
        val[q] = S.val[cur][p];
        if (pass == 0) key[q] = ((uint32_t)val[q] < (uint32_t)n) ? key[q] - kmin : sent;
        const uint32_t d = (key[q] >> shift) & 0xffu;
        uint32_t peers = 0xffffffffu;
#pragma unroll
        for (int b = 0; b < 8; ++b) {
          const bool bit = (d >> b) & 1u;
          const uint32_t bal = __ballot_sync(0xffffffffu, bit);
          peers &= bit ? bal : ~bal;
        }
        const uint32_t leader = 31 - __clz(peers);
        uint32_t old = 0;
        if (lane == leader) old = atomicAdd(&S.whist[warp][d], (uint32_t)__popc(peers));
        rank[q] = (uint32_t)__popc(peers & lt_mask);
        lead_old[q] = old;
        leader_of[q] = (uint8_t)leader;
      }
#pragma unroll
      for (int q = 0; q < kRadItems; ++q)
        if (q < ipw) rank[q] += __shfl_sync(0xffffffffu, lead_old[q], leader_of[q]);
    }
    __syncthreads();
    {  // thread t < 256 owns digit t: warp prefixes, then the digit prefix
      const int d = t;
      uint32_t c = 0;
      if (d < 256) {
#pragma unroll
        for (int w = 0; w < kWarps; ++w) {
          const uint32_t x = S.whist[w][d];
          S.whist[w][d] = c;
          c += x;
        }
      }
      const uint32_t g = rad_block_excl_scan<THREADS>(c, S.tmp);
      if (d < 256) S.gbase[d] = g;
    }
    __syncthreads();
    {
#pragma unroll
      for (int q = 0; q < kRadItems; ++q) {
        if (q >= ipw) break;
        const uint32_t d = (key[q] >> shift) & 0xffu;
        const uint32_t pos = S.gbase[d] + S.whist[warp][d] + rank[q];
        S.key[cur ^ 1][pos] = key[q];
        S.val[cur ^ 1][pos] = val[q];
      }
    }
    __syncthreads();
    cur ^= 1;
  }
  // runs of equal depth keys in id order, each by the thread at its start
  for (int p = t; p < L; p += THREADS) {
    const uint32_t kp = S.key[cur][p];
    if ((p == 0 || S.key[cur][p - 1] != kp) && p + 1 < L && S.key[cur][p + 1] == kp) {
      int e = p + 1;
      while (e < L && S.key[cur][e] == kp) ++e;
      for (int i = p + 1; i < e; ++i) {  // insertion sort of [p, e) by id
        const int32_t v = S.val[cur][i];
        int j = i - 1;
        while (j >= p && S.val[cur][j] > v) {
          S.val[cur][j + 1] = S.val[cur][j];
          --j;
        }
        S.val[cur][j + 1] = v;
      }
    }
  }
  __syncthreads();
  for (int p = t; p < L; p += THREADS) ids[beg + p] = S.val[cur][p];
}

// One block per tile sorts buckets of up to kRadChunk entries; longer
// buckets are listed: up to kRadMidChunk for bin_sort_mid_kernel
// (ctl->num_mid, mid_tiles), the rest for bin_sort_long_kernel
// (ctl->num_long, long_tiles).
#ifndef GS_BIN_SORT_MINB
#define GS_BIN_SORT_MINB 4  // blocks per SM the bucket sort's registers target (64 each)
#endif
__global__ void __launch_bounds__(kRadThreads, GS_BIN_SORT_MINB) bin_sort_kernel(const int32_t *__restrict__ offsets,
                                                               const float *__restrict__ depths,
                                                               int n, int32_t *__restrict__ ids,
                                                               Ctl *ctl,
                                                               int32_t *__restrict__ long_tiles,
                                                               int32_t *__restrict__ mid_tiles) {
  extern __shared__ __align__(16) unsigned char rad_raw[];
  RadSmem<kRadThreads> &S = *reinterpret_cast<RadSmem<kRadThreads> *>(rad_raw);
  const int tile = blockIdx.x;
  const int beg = offsets[tile], L = offsets[tile + 1] - beg;
  if (L <= 1) return;  // block-uniform
  if (L > kRadChunk) {
    if (threadIdx.x == 0) {
      if (L <= kRadMidChunk)
        mid_tiles[atomicAdd(&ctl->num_mid, 1)] = tile;
      else
        long_tiles[atomicAdd(&ctl->num_long, 1)] = tile;
    }
    return;
  }
  radix_sort_bucket<kRadThreads>(beg, L, depths, n, ids, S);
}

// The listed buckets of kRadChunk + 1 to kRadMidChunk entries, a 512-thread
// block at a time over the list (two blocks per SM).
__global__ void __launch_bounds__(kRadMidThreads, 2) bin_sort_mid_kernel(
    const int32_t *__restrict__ offsets, const float *__restrict__ depths, int n,
    int32_t *__restrict__ ids, const Ctl *ctl, const int32_t *__restrict__ mid_tiles) {
  extern __shared__ __align__(16) unsigned char rad_raw[];
  RadSmem<kRadMidThreads> &S = *reinterpret_cast<RadSmem<kRadMidThreads> *>(rad_raw);
  const int count = ctl->num_mid;
  for (int q = blockIdx.x; q < count; q += gridDim.x) {  // block-uniform
    const int tile = mid_tiles[q];
    const int beg = offsets[tile], L = offsets[tile + 1] - beg;
    radix_sort_bucket<kRadMidThreads>(beg, L, depths, n, ids, S);
    __syncthreads();  // the shared buffers are reused by the next bucket
  }
}

// The listed long buckets, a block at a time over the list.
template <int THREADS>
__global__ void __launch_bounds__(THREADS) bin_sort_long_kernel(
    const int32_t *__restrict__ offsets, const float *__restrict__ depths, int n,
    int32_t *__restrict__ ids, const Ctl *ctl, const int32_t *__restrict__ long_tiles,
    uint64_t *__restrict__ keys_a, uint64_t *__restrict__ keys_b) {
  extern __shared__ uint64_t s_keys[];  // THREADS * kItems keys
  const int count = ctl->num_long;
  for (int q = blockIdx.x; q < count; q += gridDim.x) {  // block-uniform
    const int tile = long_tiles[q];
    const int beg = offsets[tile], L = offsets[tile + 1] - beg;
    sort_bucket<THREADS>(beg, L, depths, n, ids, keys_a, keys_b, s_keys);
    __syncthreads();  // s_keys is reused by the next bucket
  }
}

constexpr int kSortLarge = 1024;  // buckets above kRadChunk: on chip up to 8192 entries

}  // namespace binning

// Scratch of gs_tile_bins, carved in this order.
struct BinScratch {
  size_t ctl, count, cursor, longs, mids, hist, keys_a, keys_b, total;
  int blocks;  // blocks of the privatised binning (0: direct global atomics)
};

static inline size_t bin_align(size_t x) { return (x + 255) / 256 * 256; }

static int bin_sm_count() {
  int dev = 0, sms = 148;
  if (cudaGetDevice(&dev) == cudaSuccess)
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  return sms > 0 ? sms : 148;
}

static BinScratch bin_scratch(int64_t capacity, int num_tiles) {
  const size_t cap = (size_t)(capacity > 0 ? capacity : 1);
  BinScratch L;
  L.blocks = num_tiles <= binning::kMaxPrivTiles ? 2 * bin_sm_count() : 0;
  L.ctl = 0;
  L.count = bin_align(sizeof(binning::Ctl));
  L.cursor = bin_align(L.count + 4 * (size_t)num_tiles);
  L.longs = bin_align(L.cursor + 4 * (size_t)num_tiles);
  L.mids = bin_align(L.longs + 4 * (size_t)num_tiles);
  L.hist = bin_align(L.mids + 4 * (size_t)num_tiles);
  L.keys_a = bin_align(L.hist + 4 * (size_t)num_tiles * (size_t)L.blocks);
  L.keys_b = bin_align(L.keys_a + 8 * cap);
  L.total = bin_align(L.keys_b + 8 * cap);
  return L;
}

}  // namespace gs

using namespace gs;

extern "C" size_t gs_tile_bins_scratch_bytes(int n, int64_t capacity, int width, int height) {
  if (n < 0 || capacity < 0 || width <= 0 || height <= 0) return 0;
  return bin_scratch(capacity, tiles_x_of(width) * tiles_y_of(height)).total;
}

extern "C" int gs_tile_bins(int n, const float *points_img, const float *radii,
                            const float *depths, const int32_t *counts, int64_t capacity,
                            int width, int height, int32_t *ids_sorted, int32_t *indexing_offset,
                            int64_t *total_dev, void *scratch, size_t scratch_bytes,
                            int32_t *tile_order, void *stream) {
  using namespace gs::binning;
  if (n < 0 || width <= 0 || height <= 0 || capacity < 0 || total_dev == nullptr)
    return GS_ERR_INVALID_ARGUMENT;
  if (((uintptr_t)points_img & 7) || ((uintptr_t)radii & 7) || ((uintptr_t)total_dev & 7))
    return GS_ERR_INVALID_ARGUMENT;
  if (capacity >= (1ll << 31) - 1) return GS_ERR_CAPACITY;  // int32 offsets
  const int T = tiles_x_of(width) * tiles_y_of(height);
  if (T > (1 << 24)) return GS_ERR_CAPACITY;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  const BinScratch L = bin_scratch(capacity, T);
  if (scratch == nullptr || scratch_bytes < L.total) return GS_ERR_CAPACITY;
  unsigned char *p = reinterpret_cast<unsigned char *>(scratch);
  Ctl *ctl = reinterpret_cast<Ctl *>(p + L.ctl);
  uint32_t *tcount = reinterpret_cast<uint32_t *>(p + L.count);
  uint32_t *cursor = reinterpret_cast<uint32_t *>(p + L.cursor);
  uint32_t *hist = reinterpret_cast<uint32_t *>(p + L.hist);
  // ctl and the tile counters start at zero
  int rc = zero_async(p, L.cursor, st);
  if (rc) return rc;
  const float2 *pts = reinterpret_cast<const float2 *>(points_img);
  const float2 *rad = reinterpret_cast<const float2 *>(radii);
  const int gblocks = (n + 255) / 256;
  const size_t priv_smem = sizeof(uint32_t) * (size_t)T;
  if (n > 0 && L.blocks > 0) {
    if (priv_smem > 48 * 1024) {
      cudaFuncSetAttribute(bin_hist_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           (int)priv_smem);
      cudaFuncSetAttribute(bin_place_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           (int)priv_smem);
    }
    bin_hist_kernel<<<L.blocks, kPrivThreads, priv_smem, st>>>(n, pts, rad, counts, width,
                                                                height, T, hist);
    bin_colscan_kernel<<<(T + 31) / 32, 32 * kColSlices, 0, st>>>(T, L.blocks, hist, tcount);
    count_launch(2);
  } else if (n > 0) {
    bin_count_kernel<<<gblocks, 256, 0, st>>>(n, pts, rad, counts, width, height, tcount);
    count_launch();
  }
  bin_scan_kernel<<<1, kScanThreads, 0, st>>>(tcount, T, capacity, indexing_offset, cursor,
                                              total_dev, ctl, device_status_word(), tile_order);
  count_launch();
  if (n > 0) {
    if (L.blocks > 0) {
      bin_place_kernel<<<L.blocks, kPrivThreads, priv_smem, st>>>(
          n, pts, rad, counts, width, height, T, hist, indexing_offset, ids_sorted, ctl);
    } else {
      bin_scatter_kernel<<<gblocks, 256, 0, st>>>(n, pts, rad, counts, width, height, capacity,
                                                  cursor, ids_sorted, ctl);
    }
    count_launch();
    uint64_t *ka = reinterpret_cast<uint64_t *>(p + L.keys_a);
    uint64_t *kb = reinterpret_cast<uint64_t *>(p + L.keys_b);
    int32_t *longs = reinterpret_cast<int32_t *>(p + L.longs);
    int32_t *mids = reinterpret_cast<int32_t *>(p + L.mids);
    const size_t smem_small = sizeof(RadSmem<kRadThreads>);
    const size_t smem_mid = sizeof(RadSmem<kRadMidThreads>);
    const size_t smem_large = sizeof(uint64_t) * kSortLarge * kItems;
    cudaFuncSetAttribute(bin_sort_long_kernel<kSortLarge>,
                         cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem_large);
    cudaFuncSetAttribute(bin_sort_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         (int)smem_small);
    cudaFuncSetAttribute(bin_sort_mid_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         (int)smem_mid);
    bin_sort_kernel<<<T, kRadThreads, smem_small, st>>>(indexing_offset, depths, n, ids_sorted,
                                                        ctl, longs, mids);
    bin_sort_mid_kernel<<<2 * bin_sm_count(), kRadMidThreads, smem_mid, st>>>(
        indexing_offset, depths, n, ids_sorted, ctl, mids);
    bin_sort_long_kernel<kSortLarge><<<2 * bin_sm_count(), kSortLarge, smem_large, st>>>(
        indexing_offset, depths, n, ids_sorted, ctl, longs, ka, kb);
    count_launch(3);
  }
  return launch_status();
}
