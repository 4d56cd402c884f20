// layout.cu -- the tile layout of a step's views in one persistent launch.
//
// For every view the rasterizer needs, per 16x16 tile, the list of the
// Gaussians that overlap it, ordered by depth bits with ties by Gaussian id
// (ruguangyou/3dgs_from_scratch src/cuda/kernel.cu:820-914 with the CUB sort
// of kernel.cu:1341-1388: key (tile << 32 | depth bits), stable over all 64
// bits), and the per-tile start offsets. As in tiles.cu the order comes from
// two stable LSD radix sorts: the Gaussians by depth bits, then the pairs --
// emitted in that depth order -- by tile id.
//
// This kernel runs the whole layout of up to kMaxViews views in one
// cooperative launch (all blocks resident, one or a few per SM), phase after
// phase, with grid-wide barriers between the phases instead of kernel
// boundaries:
//   * each view is a segment; a segment's items are split over a contiguous
//     group of blocks, one contiguous range per block;
//   * a radix pass is: (A) every block counts the digits of its range,
//     (B) one warp per (segment, digit) scans that digit's counts over the
//     segment's blocks, (C) every block re-reads its range in sub-tiles,
//     ranks each sub-tile stably (warp ballots, per-warp counters) and
//     writes it to its final place -- the block's base for the digit from
//     (B), advanced sub-tile by sub-tile. No decoupled look-back chain: the
//     prefix over the blocks is known before any block writes;
//   * between the sorts: the exclusive scan of the tile counts in depth
//     order (per-block sums, a per-segment scan of the sums, a rescan), then
//     the pair emission, where each warp writes the contiguous output span
//     of its 32 consecutive Gaussians lane by lane (coalesced stores);
//   * last, the per-tile start offsets from the sorted tile ids.
// Every grid barrier is bounded: a barrier that does not complete within the
// spin limit records GS_ERR_DEVICE_TIMEOUT in the status word and sets an
// abort flag, after which every phase and barrier is skipped (the outputs are
// then invalid and the step's optimizer update is gated off).
#include "gs_common.cuh"

namespace gs {

namespace layout {

constexpr int kThreads = 256;
constexpr int kWarps = kThreads / 32;
constexpr int kItems = 12;
constexpr int kTile = kThreads * kItems;
constexpr int kMaxViews = 64;
constexpr int kRadix = 256;

// Scratch words at the start of the scratch area.
struct Ctl {
  uint32_t arrive;  // grid-barrier arrival counter (monotonic)
  uint32_t abort;   // set when a barrier gave up
};

template <typename KT>
struct Args {
  int n, V, width, height, num_tiles;
  const float2 *points, *radii;  // (V, n)
  const uint32_t *depth_bits;    // (V, n)
  const int32_t *counts;         // (V, n)
  int32_t *ids_out;              // concatenated lists
  int32_t *offsets_out;          // (V, num_tiles)
  uint32_t *dk[2];
  int32_t *dv[2];
  int32_t *offs;                 // (V, n): pair offset of the i-th Gaussian in depth order
  KT *tk[2];
  int32_t *tv[2];                // tv[1] == ids_out
  uint32_t *H, *P;               // (grid, 256) per pass
  uint32_t *dtot;                // (V, 256)
  unsigned long long *bsum;      // (grid): per-block count sums of the scan
  Ctl *ctl;
  uint32_t *status;
  int dpasses, tpasses, tbits, emit_buf;
  int dseg[kMaxViews + 1];       // blocks of the depth segments: [dseg[s], dseg[s+1])
  int tseg[kMaxViews + 1];       // blocks of the pair segments
  long long pbase[kMaxViews + 1];  // pair offset of each view in the concatenation
};

__device__ __forceinline__ uint32_t ld_acquire_gpu(const uint32_t *p) {
  uint32_t v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// Grid-wide barrier number `k` (1, 2, ...): every block adds one arrival and
// waits until k * gridDim.x blocks have arrived. Bounded: on expiry the
// status word records GS_ERR_DEVICE_TIMEOUT and the abort flag is raised, so
// later barriers and phases return at once. Returns false after an abort.
__device__ bool grid_sync(Ctl *ctl, uint32_t k, uint32_t *status) {
  __shared__ int s_ok;
  __syncthreads();
  if (threadIdx.x == 0) {
    int ok = ld_volatile_u32(&ctl->abort) == 0u;
    if (ok) {
      __threadfence();
      atomicAdd(&ctl->arrive, 1u);
      const uint32_t target = k * gridDim.x;
      uint32_t spins = 0;
      while (ld_acquire_gpu(&ctl->arrive) < target) {
        if (ld_volatile_u32(&ctl->abort) != 0u || ++spins > (kSpinLimit << 2)) {
          ok = 0;
          break;
        }
        __nanosleep(32);
      }
      if (!ok) {
        atomicExch(status, (uint32_t)GS_ERR_DEVICE_TIMEOUT);
        atomicExch(&ctl->abort, 1u);
      }
      __threadfence();
    }
    s_ok = ok;
  }
  __syncthreads();
  return s_ok != 0;
}

// Segment of block b in a table of block starts, and the block's item range.
__device__ __forceinline__ int segment_of(const int *seg, int V, int b) {
  int s = 0;
  while (s + 1 < V && b >= seg[s + 1]) ++s;
  return s;
}

__device__ __forceinline__ void block_range(const int *seg, int s, int b, long long items,
                                            long long &lo, long long &hi) {
  const int nb = seg[s + 1] - seg[s];
  const long long per = nb > 0 ? (items + nb - 1) / nb : 0;
  lo = min(items, (long long)(b - seg[s]) * per);
  hi = min(items, lo + per);
}

// Exclusive scan of one uint32 per thread over the block (256 threads).
__device__ __forceinline__ uint32_t block_excl_scan(uint32_t x, uint32_t *s_tmp) {
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

template <typename KT>
struct Smem {
  KT keys[kTile];
  int32_t vals[kTile];
  uint32_t whist[kWarps][kRadix];
  uint32_t cursor[kRadix];
  uint32_t lstart[kRadix];
  uint32_t cnt[kRadix];
  uint32_t tmp[kWarps + 1];
};

// ---- one radix pass over every segment ------------------------------------

// (A) digit counts of this block's range into H[block].
template <typename KT, typename KeyAt>
__device__ void pass_count(KeyAt key_at, long long lo, long long hi, int shift, uint32_t *H,
                           uint32_t (*whist)[kRadix]) {
  const int warp = threadIdx.x >> 5;
  for (int k = threadIdx.x; k < kWarps * kRadix; k += kThreads) (&whist[0][0])[k] = 0u;
  __syncthreads();
  for (long long i = lo + threadIdx.x; i < hi; i += kThreads)
    atomicAdd(&whist[warp][(uint32_t)(key_at(i) >> shift) & 0xffu], 1u);
  __syncthreads();
  const int d = threadIdx.x;
  uint32_t c = 0;
#pragma unroll
  for (int w = 0; w < kWarps; ++w) c += whist[w][d];
  H[(size_t)blockIdx.x * kRadix + d] = c;
}

// (B) per (segment, digit): exclusive prefix of H over the segment's blocks
// into P, the digit's total into dtot[segment]. One warp per task.
__device__ void pass_scan(const int *seg, int V, const uint32_t *H, uint32_t *P,
                          uint32_t *dtot) {
  const int lane = threadIdx.x & 31;
  const int gwarp = blockIdx.x * kWarps + (threadIdx.x >> 5);
  const int nwarps = gridDim.x * kWarps;
  for (int task = gwarp; task < V * kRadix; task += nwarps) {
    const int s = task / kRadix, d = task - s * kRadix;
    uint32_t run = 0;
    for (int b0 = seg[s]; b0 < seg[s + 1]; b0 += 32) {
      const int b = b0 + lane;
      const uint32_t x = b < seg[s + 1] ? H[(size_t)b * kRadix + d] : 0u;
      uint32_t incl = x;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const uint32_t y = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += y;
      }
      if (b < seg[s + 1]) P[(size_t)b * kRadix + d] = run + incl - x;
      run += __shfl_sync(0xffffffffu, incl, 31);
    }
    if (lane == 0) dtot[s * kRadix + d] = run;
  }
}

// (C) this block's range in sub-tiles of kTile items, ranked stably and
// written to keys_out / vals_out at the block's per-digit cursors.
// key_at(i) / val_at(i) read item i (absolute index); out_base is added to
// every output index (the segment's start).
template <typename KT, typename KeyAt, typename ValAt>
__device__ void pass_scatter(KeyAt key_at, ValAt val_at, long long lo, long long hi,
                             long long out_base, int shift, int s, const uint32_t *P,
                             const uint32_t *dtot, KT *keys_out, int32_t *vals_out,
                             Smem<KT> &S) {
  const int t = threadIdx.x, warp = t >> 5;
  const uint32_t lane = t & 31;
  {
    const uint32_t total_d = dtot[s * kRadix + t];
    const uint32_t dex = block_excl_scan(total_d, S.tmp);
    S.cursor[t] = dex + P[(size_t)blockIdx.x * kRadix + t];
  }
  for (long long base = lo; base < hi; base += kTile) {
    for (int k = t; k < kWarps * kRadix; k += kThreads) (&S.whist[0][0])[k] = 0u;
    __syncthreads();
    const long long wbase = base + (long long)warp * (32 * kItems);
    KT key[kItems];
    int32_t val[kItems];
    uint32_t rank[kItems], lead_old[kItems];
    uint8_t leader_of[kItems];
    const uint32_t lt_mask = (1u << lane) - 1u;
#pragma unroll
    for (int k = 0; k < kItems; ++k) {
      const long long idx = wbase + k * 32 + lane;
      const bool valid = idx < hi;
      key[k] = valid ? key_at(idx) : (KT)0;
      val[k] = valid ? val_at(idx) : 0;
    }
#pragma unroll
    for (int k = 0; k < kItems; ++k) {
      const long long idx = wbase + k * 32 + lane;
      const bool valid = idx < hi;
      const uint32_t d = valid ? (((uint32_t)key[k] >> shift) & 0xffu) : 0x100u;
      uint32_t peers = __ballot_sync(0xffffffffu, valid);
      if (!valid) peers = ~peers;
#pragma unroll
      for (int bit = 0; bit < 8; ++bit) {
        const bool on = (d >> bit) & 1u;
        const uint32_t bal = __ballot_sync(0xffffffffu, on);
        peers &= on ? bal : ~bal;
      }
      const uint32_t leader = 31 - __clz(peers);
      uint32_t old = 0;
      if (valid && lane == leader) old = atomicAdd(&S.whist[warp][d], (uint32_t)__popc(peers));
      rank[k] = (uint32_t)__popc(peers & lt_mask);
      lead_old[k] = old;
      leader_of[k] = (uint8_t)leader;
    }
#pragma unroll
    for (int k = 0; k < kItems; ++k) rank[k] += __shfl_sync(0xffffffffu, lead_old[k], leader_of[k]);
    __syncthreads();
    {
      const int d = t;
      uint32_t c = 0;
#pragma unroll
      for (int w = 0; w < kWarps; ++w) {
        const uint32_t x = S.whist[w][d];
        S.whist[w][d] = c;
        c += x;
      }
      S.cnt[d] = c;
      S.lstart[d] = block_excl_scan(c, S.tmp);
    }
    __syncthreads();
#pragma unroll
    for (int k = 0; k < kItems; ++k) {
      const long long idx = wbase + k * 32 + lane;
      if (idx < hi) {
        const uint32_t d = ((uint32_t)key[k] >> shift) & 0xffu;
        const uint32_t pos = S.lstart[d] + S.whist[warp][d] + rank[k];
        S.keys[pos] = key[k];
        S.vals[pos] = val[k];
      }
    }
    __syncthreads();
    const int valid_count = (int)min((long long)kTile, hi - base);
#pragma unroll
    for (int k = 0; k < kItems; ++k) {
      const int p = t + k * kThreads;
      if (p < valid_count) {
        const KT kk = S.keys[p];
        const uint32_t d = ((uint32_t)kk >> shift) & 0xffu;
        const long long out = out_base + (long long)S.cursor[d] + (p - (int)S.lstart[d]);
        keys_out[out] = kk;
        vals_out[out] = S.vals[p];
      }
    }
    __syncthreads();
    S.cursor[t] += S.cnt[t];
  }
  __syncthreads();
}

template <typename KT>
__global__ void __launch_bounds__(kThreads, 3) layout_kernel(const Args<KT> A) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  Smem<KT> &S = *reinterpret_cast<Smem<KT> *>(smem_raw);
  // depth sort keys are u32; they share the stage with the tile keys, whose
  // Smem is at least as large (KT is u16 or u32)
  Smem<uint32_t> &SD = *reinterpret_cast<Smem<uint32_t> *>(smem_raw);
  const int b = blockIdx.x;
  uint32_t bar = 0;
  const int n = A.n;

  // ---- 1. the Gaussians of each view by depth bits (stable) ----------------
  const int ds = segment_of(A.dseg, A.V, b);
  long long dlo, dhi;
  block_range(A.dseg, ds, b, n, dlo, dhi);
  const long long dbase = (long long)ds * n;
  for (int p = 0; p < A.dpasses; ++p) {
    const int shift = 8 * p;
    const uint32_t *kin = p == 0 ? A.depth_bits + dbase : A.dk[(p - 1) & 1] + dbase;
    const int32_t *vin = p == 0 ? nullptr : A.dv[(p - 1) & 1] + dbase;
    auto key_at = [&](long long i) { return __ldg(kin + i); };
    auto val_at = [&](long long i) { return vin ? vin[i] : (int32_t)i; };
    if (!ld_volatile_u32(&A.ctl->abort)) pass_count<uint32_t>(key_at, dlo, dhi, shift, A.H, SD.whist);
    if (!grid_sync(A.ctl, ++bar, A.status)) return;
    pass_scan(A.dseg, A.V, A.H, A.P, A.dtot);
    if (!grid_sync(A.ctl, ++bar, A.status)) return;
    pass_scatter<uint32_t>(key_at, val_at, dlo, dhi, dbase, shift, ds, A.P, A.dtot, A.dk[p & 1],
                           A.dv[p & 1], SD);
    if (!grid_sync(A.ctl, ++bar, A.status)) return;
  }
  const int32_t *order = A.dv[(A.dpasses - 1) & 1] + dbase;
  const int32_t *counts = A.counts + dbase;

  // ---- 2. exclusive scan of the counts in depth order ------------------------
  {
    unsigned long long sum = 0;
    for (long long i = dlo + threadIdx.x; i < dhi; i += kThreads) {
      const int g = order[i];
      sum += (g >= 0 && g < n) ? (unsigned long long)counts[g] : 0ull;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
    __shared__ unsigned long long s_part[kWarps];
    if ((threadIdx.x & 31) == 0) s_part[threadIdx.x >> 5] = sum;
    __syncthreads();
    if (threadIdx.x == 0) {
      unsigned long long tsum = 0;
      for (int w = 0; w < kWarps; ++w) tsum += s_part[w];
      A.bsum[b] = tsum;
    }
  }
  if (!grid_sync(A.ctl, ++bar, A.status)) return;
  if (b < A.V && threadIdx.x < 32) {  // segment b: exclusive scan of its blocks' sums
    const int lane = threadIdx.x;
    unsigned long long run = 0;
    for (int b0 = A.dseg[b]; b0 < A.dseg[b + 1]; b0 += 32) {
      const int bb = b0 + lane;
      const unsigned long long x = bb < A.dseg[b + 1] ? A.bsum[bb] : 0ull;
      unsigned long long incl = x;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const unsigned long long y = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += y;
      }
      __syncwarp();
      if (bb < A.dseg[b + 1]) A.bsum[bb] = run + incl - x;
      run += __shfl_sync(0xffffffffu, incl, 31);
    }
  }
  if (!grid_sync(A.ctl, ++bar, A.status)) return;
  {
    // rescan: the block's range in chunks of kThreads, with a running carry
    unsigned long long carry = A.bsum[b];
    __shared__ unsigned long long s_w[kWarps];
    for (long long c0 = dlo; c0 < dhi; c0 += kThreads) {
      const long long i = c0 + threadIdx.x;
      uint32_t x = 0;
      if (i < dhi) {
        const int g = order[i];
        x = (g >= 0 && g < n) ? (uint32_t)counts[g] : 0u;
      }
      unsigned long long incl = x;
      const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const unsigned long long y = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += y;
      }
      if (lane == 31) s_w[warp] = incl;
      __syncthreads();
      unsigned long long wex = 0, all = 0;
      for (int w = 0; w < kWarps; ++w) {
        const unsigned long long sw = s_w[w];
        if (w < warp) wex += sw;
        all += sw;
      }
      if (i < dhi) A.offs[dbase + i] = (int32_t)(carry + wex + incl - x);
      carry += all;
      __syncthreads();
    }
  }
  if (!grid_sync(A.ctl, ++bar, A.status)) return;

  // ---- 3. pairs in depth order: each warp writes the contiguous span of its
  //         32 consecutive Gaussians lane by lane ---------------------------
  {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int tx = tiles_x_of(A.width);
    const long long pb = A.pbase[ds];
    const long long seg_pairs = A.pbase[ds + 1] - pb;
    KT *ko = A.tk[A.emit_buf];
    int32_t *vo = A.tv[A.emit_buf];
    for (long long w0 = dlo + (long long)warp * 32; w0 < dhi; w0 += kThreads) {
      const long long i = w0 + lane;
      int g = -1, x0 = 0, y0 = 0, w = 1;
      uint32_t c = 0;
      long long off = 0;
      if (i < dhi) {
        const int gg = order[i];
        if (gg >= 0 && gg < n && counts[gg] > 0) {
          const float2 pt = A.points[dbase + gg], r = A.radii[dbase + gg];
          const TileRect tr = tile_rect(pt.x, pt.y, r.x, r.y, A.width, A.height);
          off = A.offs[dbase + i];
          const int ww = tr.x1 - tr.x0 + 1, hh = tr.y1 - tr.y0 + 1;
          if (!tr.empty && off >= 0 && off + (long long)ww * hh <= seg_pairs &&
              ww * hh == counts[gg]) {  // else: corrupted input, nothing written
            g = gg;
            x0 = tr.x0;
            y0 = tr.y0;
            w = ww;
            c = (uint32_t)(ww * hh);
          }
        }
      }
      // the warp's span: lanes' pairs are contiguous in depth order
      uint32_t incl = c;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const uint32_t y = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += y;
      }
      const uint32_t excl = incl - c;
      const uint32_t span = __shfl_sync(0xffffffffu, incl, 31);
      if (span == 0) continue;
      for (uint32_t k0 = 0; k0 < span; k0 += 32) {
        const uint32_t k = k0 + lane;
        // owner: the last lane whose exclusive prefix is <= k (a lane without
        // pairs shares its successor's prefix, so the owner has pairs)
        int j = 0;
#pragma unroll
        for (int step = 16; step > 0; step >>= 1) {
          const uint32_t e = __shfl_sync(0xffffffffu, excl, j + step);
          if (e <= k) j += step;
        }
        const uint32_t ej = __shfl_sync(0xffffffffu, excl, j);
        const long long oj = __shfl_sync(0xffffffffu, off, j);
        const int gj = __shfl_sync(0xffffffffu, g, j);
        const int xj = __shfl_sync(0xffffffffu, x0, j), yj = __shfl_sync(0xffffffffu, y0, j);
        const int wj = __shfl_sync(0xffffffffu, w, j);
        if (k < span) {
          const uint32_t q = k - ej;
          const uint32_t row = q / (uint32_t)wj, col = q - row * (uint32_t)wj;
          const long long o = pb + oj + q;
          ko[o] = (KT)((yj + (int)row) * tx + xj + (int)col);
          vo[o] = gj;
        }
      }
    }
  }
  if (!grid_sync(A.ctl, ++bar, A.status)) return;

  // ---- 4. the pairs of each view by tile id (stable) -------------------------
  const int ts = segment_of(A.tseg, A.V, b);
  const bool has_pairs = A.tseg[ts + 1] > A.tseg[ts] && b >= A.tseg[ts] && b < A.tseg[ts + 1];
  long long tlo = 0, thi = 0;
  const long long tbase = A.pbase[ts];
  if (has_pairs) block_range(A.tseg, ts, b, A.pbase[ts + 1] - tbase, tlo, thi);
  for (int p = 0; p < A.tpasses; ++p) {
    const int shift = 8 * p;
    const int src = (A.emit_buf + p) & 1, dst = src ^ 1;
    const KT *kin = A.tk[src] + tbase;
    const int32_t *vin = A.tv[src] + tbase;
    auto key_at = [&](long long i) { return kin[i]; };
    auto val_at = [&](long long i) { return vin[i]; };
    if (!ld_volatile_u32(&A.ctl->abort)) pass_count<KT>(key_at, tlo, thi, shift, A.H, S.whist);
    if (!grid_sync(A.ctl, ++bar, A.status)) return;
    pass_scan(A.tseg, A.V, A.H, A.P, A.dtot);
    if (!grid_sync(A.ctl, ++bar, A.status)) return;
    if (has_pairs)
      pass_scatter<KT>(key_at, val_at, tlo, thi, tbase, shift, ts, A.P, A.dtot, A.tk[dst],
                       A.tv[dst], S);
    if (!grid_sync(A.ctl, ++bar, A.status)) return;
  }

  // ---- 5. per-tile start offsets (kernel.cu:875-914) --------------------------
  if (has_pairs) {
    const KT *keys = A.tk[(A.emit_buf + A.tpasses) & 1] + tbase;
    const long long K = A.pbase[ts + 1] - tbase;
    int32_t *offv = A.offsets_out + (size_t)ts * A.num_tiles;
    const int T = A.num_tiles;
    for (long long k = tlo + threadIdx.x; k < thi; k += kThreads) {
      const int tile = min((int)keys[k], T - 1);
      const int prev = k == 0 ? -1 : min((int)keys[k - 1], T - 1);
      for (int t = prev + 1; t <= tile; ++t) offv[t] = (int32_t)k;
      if (k == K - 1)
        for (int t = tile + 1; t < T; ++t) offv[t] = (int32_t)K;
    }
  }
}

}  // namespace layout

// ---- host side ------------------------------------------------------------------

namespace {

inline size_t align256(size_t x) { return (x + 255) / 256 * 256; }

struct LayoutPlan {
  int grid = 0;
  size_t smem = 0;
  // scratch offsets
  size_t ctl, dk0, dk1, dv0, dv1, offs, tk0, tk1, tv0, H, P, dtot, bsum, total;
};

template <typename KT>
int layout_grid(size_t smem) {
  // the shared-memory opt-in is per context: redone (with the occupancy
  // query) once per host thread and context
  thread_local unsigned long long cached_ctx = 0;
  thread_local int cached = 0;
  const unsigned long long ctx = current_context_id();
  if (ctx != 0 && cached_ctx == ctx && cached) return cached;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return 0;
  if (cudaFuncSetAttribute(layout::layout_kernel<KT>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           (int)smem) != cudaSuccess)
    return 0;
  int per_sm = 0, sms = 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, layout::layout_kernel<KT>,
                                                    layout::kThreads, smem) != cudaSuccess)
    return 0;
  if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) return 0;
  int g = sms * (per_sm < 3 ? per_sm : 3);
  cached = g;
  cached_ctx = ctx;
  return g;
}

template <typename KT>
LayoutPlan plan_layout(int n, int V, long long ktot, int grid) {
  LayoutPlan L;
  L.grid = grid;
  L.smem = sizeof(layout::Smem<KT>) > sizeof(layout::Smem<uint32_t>)
               ? sizeof(layout::Smem<KT>)
               : sizeof(layout::Smem<uint32_t>);
  const size_t vn = (size_t)V * (size_t)(n > 0 ? n : 1);
  const size_t kk = (size_t)(ktot > 0 ? ktot : 1);
  size_t o = 0;
  L.ctl = o;
  o = align256(o + sizeof(layout::Ctl));
  L.dk0 = o;
  o = align256(o + 4 * vn);
  L.dk1 = o;
  o = align256(o + 4 * vn);
  L.dv0 = o;
  o = align256(o + 4 * vn);
  L.dv1 = o;
  o = align256(o + 4 * vn);
  L.offs = o;
  o = align256(o + 4 * vn);
  L.tk0 = o;
  o = align256(o + sizeof(KT) * kk);
  L.tk1 = o;
  o = align256(o + sizeof(KT) * kk);
  L.tv0 = o;
  o = align256(o + 4 * kk);
  L.H = o;
  o = align256(o + 4 * (size_t)grid * layout::kRadix);
  L.P = o;
  o = align256(o + 4 * (size_t)grid * layout::kRadix);
  L.dtot = o;
  o = align256(o + 4 * (size_t)V * layout::kRadix);
  L.bsum = o;
  o = align256(o + 8 * (size_t)grid);
  L.total = o;
  return L;
}

// Blocks of `V` segments of sizes w[s] over `grid` blocks: proportional,
// at least one per non-empty segment, none for an empty one.
void split_blocks(int grid, int V, const long long *w, int *seg) {
  long long sum = 0;
  int nonempty = 0;
  for (int s = 0; s < V; ++s) {
    sum += w[s];
    nonempty += w[s] > 0;
  }
  seg[0] = 0;
  int left = grid - nonempty;  // blocks beyond the one every non-empty segment gets
  long long wleft = sum;
  for (int s = 0; s < V; ++s) {
    int nb = 0;
    if (w[s] > 0) {
      const long long extra = wleft > 0 ? (long long)left * w[s] / wleft : 0;
      nb = 1 + (int)extra;
      left -= (int)extra;
      wleft -= w[s];
    }
    seg[s + 1] = seg[s] + nb;
  }
}

template <typename KT>
int run_layout(int n, int V, const float *points, const float *radii, const float *depths,
               const int32_t *counts, const int64_t *totals, int width, int height,
               int32_t *ids_sorted, int32_t *indexing_offset, void *scratch,
               size_t scratch_bytes, cudaStream_t st) {
  const int num_tiles = tiles_x_of(width) * tiles_y_of(height);
  long long ktot = 0;
  for (int v = 0; v < V; ++v) ktot += totals[v];
  const size_t smem0 = sizeof(layout::Smem<KT>) > sizeof(layout::Smem<uint32_t>)
                           ? sizeof(layout::Smem<KT>)
                           : sizeof(layout::Smem<uint32_t>);
  const int grid = layout_grid<KT>(smem0);
  if (grid < V) return grid <= 0 ? GS_ERR_CUDA : GS_ERR_CAPACITY;
  const LayoutPlan L = plan_layout<KT>(n, V, ktot, grid);
  if (scratch == nullptr || scratch_bytes < L.total) return GS_ERR_CAPACITY;
  unsigned char *p = reinterpret_cast<unsigned char *>(scratch);
  int rc = cuda_status(cudaMemsetAsync(p + L.ctl, 0, sizeof(layout::Ctl), st));
  if (rc) return rc;
  layout::Args<KT> A{};
  A.n = n;
  A.V = V;
  A.width = width;
  A.height = height;
  A.num_tiles = num_tiles;
  A.points = reinterpret_cast<const float2 *>(points);
  A.radii = reinterpret_cast<const float2 *>(radii);
  A.depth_bits = reinterpret_cast<const uint32_t *>(depths);
  A.counts = counts;
  A.ids_out = ids_sorted;
  A.offsets_out = indexing_offset;
  A.dk[0] = reinterpret_cast<uint32_t *>(p + L.dk0);
  A.dk[1] = reinterpret_cast<uint32_t *>(p + L.dk1);
  A.dv[0] = reinterpret_cast<int32_t *>(p + L.dv0);
  A.dv[1] = reinterpret_cast<int32_t *>(p + L.dv1);
  A.offs = reinterpret_cast<int32_t *>(p + L.offs);
  A.tk[0] = reinterpret_cast<KT *>(p + L.tk0);
  A.tk[1] = reinterpret_cast<KT *>(p + L.tk1);
  A.tv[0] = reinterpret_cast<int32_t *>(p + L.tv0);
  A.tv[1] = ids_sorted;
  A.H = reinterpret_cast<uint32_t *>(p + L.H);
  A.P = reinterpret_cast<uint32_t *>(p + L.P);
  A.dtot = reinterpret_cast<uint32_t *>(p + L.dtot);
  A.bsum = reinterpret_cast<unsigned long long *>(p + L.bsum);
  A.ctl = reinterpret_cast<layout::Ctl *>(p + L.ctl);
  A.status = device_status_word();
  if (A.status == nullptr) return GS_ERR_CUDA;
  A.dpasses = 4;
  int tbits = 0;
  while ((1 << tbits) < num_tiles) ++tbits;
  A.tbits = tbits > 0 ? tbits : 1;
  A.tpasses = (A.tbits + 7) / 8;
  // the emission buffer is chosen so that the last pass writes ids_out (tv[1])
  A.emit_buf = (A.tpasses + 1) & 1;
  long long wn[layout::kMaxViews], wk[layout::kMaxViews];
  for (int v = 0; v < V; ++v) {
    wn[v] = n;
    wk[v] = totals[v];
  }
  split_blocks(grid, V, wn, A.dseg);
  split_blocks(grid, V, wk, A.tseg);
  A.pbase[0] = 0;
  for (int v = 0; v < V; ++v) A.pbase[v + 1] = A.pbase[v] + totals[v];
  void *args[] = {(void *)&A};
  rc = cuda_status(cudaLaunchCooperativeKernel((const void *)layout::layout_kernel<KT>, grid,
                                               layout::kThreads, args, L.smem, st));
  count_launch();
  return rc;
}

}  // namespace

}  // namespace gs

using namespace gs;

extern "C" size_t gs_tile_layout_views_scratch_bytes(int n, int num_views, const int64_t *totals,
                                                     int width, int height) {
  if (n < 0 || num_views < 1 || num_views > layout::kMaxViews || totals == nullptr || width <= 0 ||
      height <= 0)
    return 0;
  long long ktot = 0;
  for (int v = 0; v < num_views; ++v) ktot += totals[v] > 0 ? totals[v] : 0;
  const int num_tiles = tiles_x_of(width) * tiles_y_of(height);
  if (num_tiles <= 65536) {
    const size_t smem = sizeof(layout::Smem<uint32_t>);
    const int grid = layout_grid<uint16_t>(smem);
    return grid > 0 ? plan_layout<uint16_t>(n, num_views, ktot, grid).total : 0;
  }
  const int grid = layout_grid<uint32_t>(sizeof(layout::Smem<uint32_t>));
  return grid > 0 ? plan_layout<uint32_t>(n, num_views, ktot, grid).total : 0;
}

extern "C" int gs_tile_layout_views(int n, int num_views, const float *points_img,
                                    const float *radii, const float *depths,
                                    const int32_t *counts, const int64_t *totals, int width,
                                    int height, int32_t *ids_sorted, int32_t *indexing_offset,
                                    void *scratch, size_t scratch_bytes, void *stream) {
  if (n < 0 || num_views < 1 || num_views > layout::kMaxViews || width <= 0 || height <= 0 ||
      totals == nullptr || indexing_offset == nullptr)
    return GS_ERR_INVALID_ARGUMENT;
  if (((uintptr_t)points_img & 7) || ((uintptr_t)radii & 7)) return GS_ERR_INVALID_ARGUMENT;
  const int num_tiles = tiles_x_of(width) * tiles_y_of(height);
  if (num_tiles > (1 << 24)) return GS_ERR_CAPACITY;
  long long ktot = 0;
  for (int v = 0; v < num_views; ++v) {
    if (totals[v] < 0) return GS_ERR_INVALID_ARGUMENT;
    if (totals[v] >= (1ll << 31)) return GS_ERR_CAPACITY;  // int32 offsets within a view
    ktot += totals[v];
  }
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  // rasterizer.cpp:352: offsets start at zero; a view without pairs keeps them
  int rc = cuda_status(cudaMemsetAsync(indexing_offset, 0,
                                       sizeof(int32_t) * (size_t)num_tiles * num_views, st));
  if (rc || n == 0 || ktot == 0) return rc;
  if (points_img == nullptr || radii == nullptr || depths == nullptr || counts == nullptr ||
      ids_sorted == nullptr)
    return GS_ERR_INVALID_ARGUMENT;
  if (num_tiles <= 65536)
    return run_layout<uint16_t>(n, num_views, points_img, radii, depths, counts, totals, width,
                                height, ids_sorted, indexing_offset, scratch, scratch_bytes, st);
  return run_layout<uint32_t>(n, num_views, points_img, radii, depths, counts, totals, width,
                              height, ids_sorted, indexing_offset, scratch, scratch_bytes, st);
}
