// blend.cu -- per-tile alpha blending, forward and backward.
//
// One 128-thread block per 16x16 tile, two pixels per thread (two
// independent dependency chains per record). Warp w owns an 8x8 pixel block,
// so a warp's pixels are spatially compact. The tile's Gaussian list is
// streamed in batches of 256: each thread stages two Gaussians' records in
// shared memory, together with a 4-bit mask of the warp blocks whose pixels
// that Gaussian can reach (a conservative bound; see reach_mask), and then
// every warp walks the batch from shared memory, 32 records at a time: one
// ballot of their masks, then only the records its block can see. Per pixel the forward arithmetic is the
// reference's, operation for operation (ruguangyou/3dgs_from_scratch
// src/cuda/kernel.cu:954-982), so images match it bit for bit; a thread's
// two pixels (same column) run as fp32x2 pairs through Blackwell's packed
// FMA / MUL / ADD, which round exactly as the scalar forms (fwd_step2); the backward
// (kernel.cu:1066-1110) keeps the forward's skip tests and reorganises the
// gradient sums (see bwd_step).
//
// The forward records each pixel's final transmittance and the index one past
// its last contributing list entry, so the backward needs no forward replay.
// The backward walks each batch back to front, runs a thread's two pixels
// (same column) as fp32x2 pairs with Blackwell's packed FMA / MUL / ADD
// (bwd_step2: one instruction for both pixels' chains), sums them,
// pre-reduces the 9 gradient terms of a (warp, Gaussian) pair with a
// transposing warp-shuffle reduction (two visible records at a time: their
// 18 sums in 21 shuffles, against 45 per record for plain butterflies),
// accumulates warps into shared memory, and issues one vector atomic per
// gradient group per (tile, Gaussian).
#include "gs_common.cuh"

namespace gs {

constexpr int kBlendThreads = 128;  // 4 warps per 16x16 tile, 2 pixels per thread
constexpr int kBatch = 256;         // records staged per batch (2 per thread)
constexpr int kWarps = kBlendThreads / 32;
#ifndef GS_BWD_PAIRED
#define GS_BWD_PAIRED 1  // 1: the backward reduces two visible entries per step
#endif
#ifndef GS_BWD_F32X2
#define GS_BWD_F32X2 1  // 1: the backward runs a thread's two pixels as fp32x2 pairs
#endif
#ifndef GS_BWD_EX2
#define GS_BWD_EX2 1  // 1: the backward's exponential as 2^(x log2 e) with the scale folded
#endif

// Pixels owned by thread t: warp w covers the 8x8 block at (8*(w&1), 8*(w>>1));
// lane l takes column l&7 and rows (l>>3) and (l>>3)+4 of that block.
__device__ __forceinline__ int2 pixel_in_tile(int t) {
  int w = t >> 5, l = t & 31;
  return make_int2(8 * (w & 1) + (l & 7), 8 * (w >> 1) + (l >> 3));
}

// Gaussian record in shared memory: g0 = (u, v, A, B), g1 = (C, opacity, r, g), b.
struct Rec {
  float4 g0, g1;
  float b;
};

// Bitmask of the tile's 4 warp blocks (8x8 pixels each) that may hold a pixel
// with q <= q_cut, where q_cut = min(chi2, 2 ln(opacity / alpha_thr)) bounds
// both of the reference's skip tests (q > chi2, alpha < alpha_thr). A block
// is reached when the minimum m of the quadratic form q(d) = d^T Q d over the
// box of offsets d = pixel - mean spanned by the block's pixel centres is at
// most qc = 1.01 q_cut + 0.05: q is convex with its minimum at d = 0, so m is
// 0 if the box holds the origin and otherwise lies on one of the box's four
// edges, where it is a clamped 1-D quadratic minimum. The box contains every
// pixel offset of the block, so m bounds q at each of them from below.
// Rounding: with R = 2 (A + C)^2 / det (the ratio of the summed term
// magnitudes to q), both the kernels' float q at a pixel and the float m
// here are within 5e-4 R/2000 of exact (relative); an error in the clamped
// minimiser changes m only to second order. Conics with R >= 2000 reach
// everything; for the rest, m > qc implies the pixel's float q exceeds
// (1.01 q_cut + 0.05)(1 - 1e-3) > q_cut, so a skipped record fails one of the
// reference's tests at every pixel of the block. Non-finite input reaches
// everything.
__device__ __forceinline__ float box_min_q(float a, float b, float c, float dx0, float dx1,
                                           float dy0, float dy1, float inv_a, float inv_c) {
  if (dx0 <= 0.0f && dx1 >= 0.0f && dy0 <= 0.0f && dy1 >= 0.0f) return 0.0f;
  float best = INFINITY;
#pragma unroll
  for (int e = 0; e < 2; ++e) {
    const float X = e ? dx1 : dx0;
    const float dy = fminf(fmaxf(-b * X * inv_c, dy0), dy1);
    best = fminf(best, a * X * X + 2.0f * b * X * dy + c * dy * dy);
    const float Y = e ? dy1 : dy0;
    const float dx = fminf(fmaxf(-b * Y * inv_a, dx0), dx1);
    best = fminf(best, a * dx * dx + 2.0f * b * dx * Y + c * Y * Y);
  }
  return best;
}

__device__ __forceinline__ uint32_t reach_mask(float u, float v, float A, float B, float C,
                                               float opac, float alpha_thr, float chi_thr,
                                               int tile_x0, int tile_y0) {
  float q_cut = chi_thr;
  if (alpha_thr > 0.0f) {
    if (!(opac > 0.0f)) return 0xfu;  // degenerate opacity: evaluate normally
    q_cut = fminf(q_cut, 2.0f * logf(opac / alpha_thr));
  }
  const float det = A * C - B * B;
  if (!(A > 0.0f) || !(C > 0.0f) || !(det > 0.0f) || !isfinite(u) || !isfinite(v) ||
      !isfinite(q_cut) || !(2.0f * (A + C) * (A + C) < 2000.0f * det))
    return 0xfu;
  if (q_cut < -0.05f) return 0u;  // opacity below the alpha threshold: alpha < thr everywhere
  const float qc = fmaxf(q_cut, 0.0f) * 1.01f + 0.05f;
  const float inv_a = 1.0f / A, inv_c = 1.0f / C;
  uint32_t m = 0;
#pragma unroll
  for (int w = 0; w < kWarps; ++w) {
    const float dx0 = (float)(tile_x0 + 8 * (w & 1)) - u;
    const float dy0 = (float)(tile_y0 + 8 * (w >> 1)) - v;
    const bool hit = box_min_q(A, B, C, dx0, dx0 + 7.0f, dy0, dy0 + 7.0f, inv_a, inv_c) <= qc;
    m |= hit ? (1u << w) : 0u;
  }
  return m;
}

template <bool PACKED>
__device__ __forceinline__ Rec load_rec(int id, int n, const float2 *__restrict__ points,
                                        const float4 *__restrict__ splat,
                                        const float *__restrict__ conic,
                                        const float *__restrict__ opac,
                                        const float *__restrict__ colors) {
  Rec r;
  if (id < 0 || id >= n) {  // only reachable with a corrupted id list: contributes nothing
    r.g0 = make_float4(0.f, 0.f, 0.f, 0.f);
    r.g1 = make_float4(0.f, 0.f, 0.f, 0.f);
    r.b = 0.f;
    return r;
  }
  float2 p = __ldg(points + id);
  if (PACKED) {
    float4 s0 = __ldg(splat + 2 * (size_t)id);
    float4 s1 = __ldg(splat + 2 * (size_t)id + 1);
    r.g0 = make_float4(p.x, p.y, s0.x, s0.y);
    r.g1 = make_float4(s0.z, s0.w, s1.x, s1.y);
    r.b = s1.z;
  } else {
    size_t i3 = 3 * (size_t)id;
    r.g0 = make_float4(p.x, p.y, __ldg(conic + i3), __ldg(conic + i3 + 1));
    r.g1 = make_float4(__ldg(conic + i3 + 2), __ldg(opac + id), __ldg(colors + i3),
                       __ldg(colors + i3 + 1));
    r.b = __ldg(colors + i3 + 2);
  }
  return r;
}

__device__ __forceinline__ float2 f2(float x) { return make_float2(x, x); }

// Forward state of one pixel.
struct FwdPx {
  float fu, fv, T, r, g, b;
  int last;
  bool done;
};

// One list entry for one pixel: kernel.cu:955-981, operation for operation.
template <bool ACCUM>
__device__ __forceinline__ void fwd_step(FwdPx &p, const float4 &g0, const float4 &g1, float cb,
                                         int k, float alpha_thr, float trans_thr,
                                         float chi_thr) {
  const float du = p.fu - g0.x;
  const float dv = p.fv - g0.y;
  const float inv00 = g0.z, inv01 = g0.w, inv11 = g1.x;
  float exponent = inv00 * du * du + 2.0f * inv01 * du * dv + inv11 * dv * dv;
  if (exponent > chi_thr) return;
  float alpha = expf(-0.5f * exponent) * g1.y;
  if (alpha < alpha_thr) return;
  if (ACCUM) {
    float weight = alpha * p.T;
    p.r += weight * g1.z;
    p.g += weight * g1.w;
    p.b += weight * cb;
  }
  float one_minus_alpha = 1.0f - alpha + kTransEps;
  p.T *= one_minus_alpha;
  p.last = k + 1;
  if (p.T < trans_thr) p.done = true;
}

#ifndef GS_FWD_F32X2
#define GS_FWD_F32X2 1  // 1: the forward runs a thread's two pixels as fp32x2 pairs
#endif

// Forward state of a thread's two pixels as fp32x2 pairs (.x upper, .y lower).
struct FwdPx2 {
  float fu;
  float2 fv, T, r, g, b;
  int last0, last1;
  bool done0, done1;
};

// fwd_step for both pixels with packed fp32x2 instructions, rounding for
// rounding the scalar step as compiled (multiply-adds contracted): the
// exponent is fma(inv11 dv, dv, fma(inv00 du, du, (2 inv01 du) dv)), the
// colour updates fma(weight, colour, sum); the column terms (inv00 du,
// 2 inv01 du) are computed once for both pixels. -alpha is carried so that
// 1 - alpha and the colour updates stay single operations; a pixel that is
// done or cut gets -alpha = 0, which leaves its colour and (1 + 0 + 1e-10
// rounds to 1) its transmittance unchanged. Images, transmittances and end
// indices are identical to the scalar step's.
template <bool ACCUM>
__device__ __forceinline__ void fwd_step2(FwdPx2 &p, const float4 &g0, const float4 &g1, float cb,
                                          int k, float alpha_thr, float trans_thr,
                                          float chi_thr) {
  bool v0 = !p.done0, v1 = !p.done1;
  const float du = p.fu - g0.x;
  const float2 dv = __fadd2_rn(p.fv, f2(-g0.y));
  const float inv00 = g0.z, inv01 = g0.w, inv11 = g1.x;
  const float A = inv00 * du;
  const float B = 2.0f * inv01 * du;
  const float2 s1 = __ffma2_rn(f2(A), f2(du), __fmul2_rn(f2(B), dv));
  const float2 e = __ffma2_rn(__fmul2_rn(f2(inv11), dv), dv, s1);
  v0 = v0 && !(e.x > chi_thr);
  v1 = v1 && !(e.y > chi_thr);
  if (!(v0 || v1)) return;
  const float2 h = __fmul2_rn(e, f2(-0.5f));
  float2 nal = __fmul2_rn(make_float2(expf(h.x), expf(h.y)), f2(-g1.y));
  v0 = v0 && !(-nal.x < alpha_thr);
  v1 = v1 && !(-nal.y < alpha_thr);
  if (!(v0 || v1)) return;
  if (!v0) nal.x = 0.f;
  if (!v1) nal.y = 0.f;
  if (ACCUM) {
    const float2 nw = __fmul2_rn(nal, p.T);  // -weight
    p.r = __ffma2_rn(nw, f2(-g1.z), p.r);
    p.g = __ffma2_rn(nw, f2(-g1.w), p.g);
    p.b = __ffma2_rn(nw, f2(-cb), p.b);
  }
  const float2 oma = __fadd2_rn(__fadd2_rn(nal, f2(1.0f)), f2(kTransEps));
  p.T = __fmul2_rn(p.T, oma);
  if (v0) {
    p.last0 = k + 1;
    if (p.T.x < trans_thr) p.done0 = true;
  }
  if (v1) {
    p.last1 = k + 1;
    if (p.T.y < trans_thr) p.done1 = true;
  }
}

// Forward blend. With ACCUM = false only the transmittance bookkeeping is
// done (the replay used by the reference-API backward).
#ifndef GS_FWD_MINB
#define GS_FWD_MINB 8  // resident blocks per SM the forward's register budget targets
#endif
template <bool PACKED, bool ACCUM>
__global__ void __launch_bounds__(kBlendThreads, GS_FWD_MINB) blend_forward_kernel(
    int num_tiles, const int32_t *__restrict__ offsets, int64_t total,
    const int32_t *__restrict__ ids, int n, const float2 *__restrict__ points,
    const float4 *__restrict__ splat, const float *__restrict__ conic,
    const float *__restrict__ opac, const float *__restrict__ colors, int width, int height,
    float alpha_thr, float trans_thr, float chi_thr, float *__restrict__ image,
    float *__restrict__ final_t, int32_t *__restrict__ pixel_end, uint8_t *__restrict__ reach,
    const int32_t *__restrict__ order) {
  __shared__ float4 s_g0[kBatch];
  __shared__ float4 s_g1[kBatch];
  __shared__ float s_b[kBatch];
  __shared__ uint8_t s_mask[kBatch];

  // block b blends tile order[b] (longest lists first), or tile b
  const int tile = order != nullptr ? __ldg(order + blockIdx.x) : (int)blockIdx.x;
  const int tx = tiles_x_of(width);
  const int tile_x0 = (tile % tx) * GS_TILE, tile_y0 = (tile / tx) * GS_TILE;
  const int t = threadIdx.x, warp = t >> 5, lane = t & 31;
  const int2 pp = pixel_in_tile(t);
  const int u = tile_x0 + pp.x, v0 = tile_y0 + pp.y, v1 = v0 + 4;
  const bool in0 = (u < width) && (v0 < height);
  const bool in1 = (u < width) && (v1 < height);

  const int s = offsets[tile];
  // total < 0: the offsets hold num_tiles + 1 entries, the last one the end
  // of the last tile's list (the capacity form of the tile layout)
  const int e = (tile + 1 < num_tiles) ? offsets[tile + 1]
                                       : (total >= 0 ? (int)total : offsets[num_tiles]);

#if GS_FWD_F32X2
  FwdPx2 P{(float)u, make_float2((float)v0, (float)v1), make_float2(1.f, 1.f),
           make_float2(0.f, 0.f), make_float2(0.f, 0.f), make_float2(0.f, 0.f), s, s, !in0,
           !in1};
#define GS_ALL_DONE (P.done0 && P.done1)
#else
  FwdPx p0{(float)u, (float)v0, 1.0f, 0.f, 0.f, 0.f, s, !in0};
  FwdPx p1{(float)u, (float)v1, 1.0f, 0.f, 0.f, 0.f, s, !in1};
#define GS_ALL_DONE (p0.done && p1.done)
#endif

  for (int base = s; base < e; base += kBatch) {
    if (__syncthreads_count(!GS_ALL_DONE) == 0) break;
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const int slot = t + h * kBlendThreads;
      const int k = base + slot;
      if (k < e) {
        int id = __ldg(ids + k);
        Rec r = load_rec<PACKED>(id, n, points, splat, conic, opac, colors);
        s_g0[slot] = r.g0;
        s_g1[slot] = r.g1;
        s_b[slot] = r.b;
        const uint8_t m = (uint8_t)reach_mask(r.g0.x, r.g0.y, r.g0.z, r.g0.w, r.g1.x, r.g1.y,
                                              alpha_thr, chi_thr, tile_x0, tile_y0);
        s_mask[slot] = m;
        if (reach != nullptr) reach[k] = m;  // kept for the backward
      }
    }
    __syncthreads();
    const int cnt = min(kBatch, e - base);
    // 32 entries at a time: one ballot of the reach masks, then only the
    // entries this warp's block can see, in list order
    for (int j0 = 0; j0 < cnt; j0 += 32) {
      if (__all_sync(0xffffffffu, GS_ALL_DONE)) break;
      const int jl = j0 + lane;
      uint32_t todo = __ballot_sync(0xffffffffu, jl < cnt && ((s_mask[jl] >> warp) & 1u));
      // two visible records per step: both are read from shared memory up
      // front, then applied to each pixel in list order
      while (todo & (todo - 1)) {
        const int j = j0 + __ffs(todo) - 1;
        todo &= todo - 1;
        const int j2 = j0 + __ffs(todo) - 1;
        todo &= todo - 1;
        const float4 g0 = s_g0[j], h0 = s_g0[j2];
        const float4 g1 = s_g1[j], h1 = s_g1[j2];
        const float cb = ACCUM ? s_b[j] : 0.f, hb = ACCUM ? s_b[j2] : 0.f;
#if GS_FWD_F32X2
        fwd_step2<ACCUM>(P, g0, g1, cb, base + j, alpha_thr, trans_thr, chi_thr);
        fwd_step2<ACCUM>(P, h0, h1, hb, base + j2, alpha_thr, trans_thr, chi_thr);
#else
        if (!p0.done) fwd_step<ACCUM>(p0, g0, g1, cb, base + j, alpha_thr, trans_thr, chi_thr);
        if (!p1.done) fwd_step<ACCUM>(p1, g0, g1, cb, base + j, alpha_thr, trans_thr, chi_thr);
        if (!p0.done) fwd_step<ACCUM>(p0, h0, h1, hb, base + j2, alpha_thr, trans_thr, chi_thr);
        if (!p1.done) fwd_step<ACCUM>(p1, h0, h1, hb, base + j2, alpha_thr, trans_thr, chi_thr);
#endif
      }
      if (todo) {
        const int j = j0 + __ffs(todo) - 1;
        const float4 g0 = s_g0[j];
        const float4 g1 = s_g1[j];
        const float cb = ACCUM ? s_b[j] : 0.f;
#if GS_FWD_F32X2
        fwd_step2<ACCUM>(P, g0, g1, cb, base + j, alpha_thr, trans_thr, chi_thr);
#else
        if (!p0.done) fwd_step<ACCUM>(p0, g0, g1, cb, base + j, alpha_thr, trans_thr, chi_thr);
        if (!p1.done) fwd_step<ACCUM>(p1, g0, g1, cb, base + j, alpha_thr, trans_thr, chi_thr);
#endif
      }
    }
  }
#undef GS_ALL_DONE
#if GS_FWD_F32X2
  const FwdPx p0{P.fu, P.fv.x, P.T.x, P.r.x, P.g.x, P.b.x, P.last0, P.done0};
  const FwdPx p1{P.fu, P.fv.y, P.T.y, P.r.y, P.g.y, P.b.y, P.last1, P.done1};
#endif
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    const FwdPx &p = h ? p1 : p0;
    const int v = h ? v1 : v0;
    if (!(h ? in1 : in0)) continue;
    size_t px = (size_t)v * width + u;
    if (ACCUM && image) {
      image[3 * px] = p.r;
      image[3 * px + 1] = p.g;
      image[3 * px + 2] = p.b;
    }
    final_t[px] = p.T;
    pixel_end[px] = p.last;
  }
}

// Transposing warp reduction of 8 values: afterwards lane L holds the
// warp-wide sum of value index (L >> 2) & 7.
__device__ __forceinline__ float reduce8(const float v[8], uint32_t lane) {
  const unsigned FULL = 0xffffffffu;
  float a[4];
  const bool b4 = lane & 16;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    float send = b4 ? v[i] : v[i + 4];
    float keep = b4 ? v[i + 4] : v[i];
    a[i] = keep + __shfl_xor_sync(FULL, send, 16);
  }
  float c[2];
  const bool b3 = lane & 8;
#pragma unroll
  for (int i = 0; i < 2; ++i) {
    float send = b3 ? a[i] : a[i + 2];
    float keep = b3 ? a[i + 2] : a[i];
    c[i] = keep + __shfl_xor_sync(FULL, send, 8);
  }
  const bool b2 = lane & 4;
  float send = b2 ? c[0] : c[1];
  float keep = b2 ? c[1] : c[0];
  float d = keep + __shfl_xor_sync(FULL, send, 4);
  d += __shfl_xor_sync(FULL, d, 2);
  d += __shfl_xor_sync(FULL, d, 1);
  return d;
}

__device__ __forceinline__ float reduce1(float x) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) x += __shfl_xor_sync(0xffffffffu, x, o);
  return x;
}

// Transposing warp reduction of 16 values (16 shuffles): afterwards lane L
// holds the warp-wide sum of value index (L >> 1) & 15.
__device__ __forceinline__ float reduce16(const float v[16], uint32_t lane) {
  const unsigned FULL = 0xffffffffu;
  float a[8];
  const bool b4 = lane & 16;
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const float send = b4 ? v[i] : v[i + 8];
    const float keep = b4 ? v[i + 8] : v[i];
    a[i] = keep + __shfl_xor_sync(FULL, send, 16);
  }
  float c[4];
  const bool b3 = lane & 8;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float send = b3 ? a[i] : a[i + 4];
    const float keep = b3 ? a[i + 4] : a[i];
    c[i] = keep + __shfl_xor_sync(FULL, send, 8);
  }
  float d[2];
  const bool b2 = lane & 4;
#pragma unroll
  for (int i = 0; i < 2; ++i) {
    const float send = b2 ? c[i] : c[i + 2];
    const float keep = b2 ? c[i + 2] : c[i];
    d[i] = keep + __shfl_xor_sync(FULL, send, 4);
  }
  const bool b1 = lane & 2;
  const float send = b1 ? d[0] : d[1];
  const float keep = b1 ? d[1] : d[0];
  float e = keep + __shfl_xor_sync(FULL, send, 2);
  return e + __shfl_xor_sync(FULL, e, 1);
}

// Two values (5 shuffles): afterwards lane L holds the warp-wide sum of
// value (L >> 4) & 1.
__device__ __forceinline__ float reduce2(float x0, float x1, uint32_t lane) {
  const bool b4 = lane & 16;
  float x = (b4 ? x1 : x0) + __shfl_xor_sync(0xffffffffu, b4 ? x0 : x1, 16);
#pragma unroll
  for (int o = 8; o > 0; o >>= 1) x += __shfl_xor_sync(0xffffffffu, x, o);
  return x;
}

// Backward state of one pixel.
struct BwdPx {
  float fu, fv, gr, gg, gb, Ta, suffix;
  int end;
};

// One list entry for one pixel, back to front (kernel.cu:1068-1109). Adds the
// pixel's gradient terms into acc and returns whether it contributed. The
// terms that are a per-Gaussian constant times a per-pixel quantity are
// summed without the constant, which is applied once per (tile, Gaussian) in
// the flush: acc[0..4] = sum of du*ag, dv*ag, du*du*ag, du*dv*ag, dv*dv*ag
// (ag = alpha * dL/dalpha), from which d(u,v) = conic * (acc0, acc1) and
// d conic = (-acc2 / 2, -acc3, -acc4 / 2). The skip decisions (chi-square
// cut, alpha threshold) use the forward's expressions, with an approximate
// exponential (a few 1e-7 relative; in bwd_step2 exp(x) = 2^(x log2 e) by
// ex2.approx, the scale folded into the packed multiply): a pair whose alpha lies within
// that of the threshold may be decided differently from the forward, which
// changes the pixel's gradient by about alpha_thr relative; the two
// divisions by (1 - alpha) of the reference (kernel.cu:1088,1094) become one
// approximate reciprocal (rcp.approx, at most 1 ulp) and two products.
__device__ __forceinline__ float rcp_approx(float x) {
  float r;
  asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(r) : "f"(x));
  return r;
}

// 2^x by the PTX approximate base-2 exponential (flush-to-zero).
__device__ __forceinline__ float ex2_approx(float x) {
  float r;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(r) : "f"(x));
  return r;
}

__device__ __forceinline__ bool bwd_step(BwdPx &p, const float4 &g0, const float4 &g1, float c2,
                                         float alpha_thr, float chi_thr, float acc[9]) {
  const float du = p.fu - g0.x;
  const float dv = p.fv - g0.y;
  const float inv00 = g0.z, inv01 = g0.w, inv11 = g1.x;
  float exponent = inv00 * du * du + 2.0f * inv01 * du * dv + inv11 * dv * dv;
  if (exponent > chi_thr) return false;
  float density = __expf(-0.5f * exponent);
  float alpha = density * g1.y;
  if (alpha < alpha_thr) return false;
  float one_minus_alpha = 1.0f - alpha + kTransEps;
  float rcp = rcp_approx(one_minus_alpha);
  float prefix_t = p.Ta * rcp;
  float weight = alpha * prefix_t;
  const float c0 = g1.z, c1 = g1.w;
  float grad_rgb = p.gr * c0 + p.gg * c1 + p.gb * c2;
  float grad_alpha = prefix_t * grad_rgb - p.suffix * rcp;
  float ag = alpha * grad_alpha;
  const float au = du * ag, av = dv * ag;
  acc[0] += au;
  acc[1] += av;
  acc[2] = fmaf(au, du, acc[2]);
  acc[3] = fmaf(au, dv, acc[3]);
  acc[4] = fmaf(av, dv, acc[4]);
  acc[5] = fmaf(density, grad_alpha, acc[5]);
  acc[6] = fmaf(weight, p.gr, acc[6]);
  acc[7] = fmaf(weight, p.gg, acc[7]);
  acc[8] = fmaf(weight, p.gb, acc[8]);
  p.suffix += weight * grad_rgb;
  p.Ta = prefix_t;
  return true;
}

// Backward state of a thread's two pixels (same column, rows 4 apart) as
// fp32x2 pairs: .x the upper pixel, .y the lower one. nsuffix holds the
// negated suffix sum.
struct BwdPx2 {
  float fu;
  float2 fv, gr, gg, gb, Ta, nsuffix;
  int end0, end1;
};

// bwd_step for both pixels at once with the packed fp32x2 instructions
// (__ffma2_rn, __fmul2_rn, __fadd2_rn: two IEEE round-to-nearest operations
// per instruction, the same results as the scalar forms). The column terms of
// the exponent are computed once: inv00 du^2 + dv (2 inv01 du + inv11 dv).
// A pixel past its end or cut by the chi-square / alpha test gets alpha =
// density = 0, so it adds nothing and keeps its transmittance. acc receives
// the pair's sums (not accumulated): slots 0-4 and 6-8 negated (the sign
// comes from carrying -alpha, which turns the subtractions into fused
// multiply-adds; restored in the flush), slot 5 as is.
__device__ __forceinline__ bool bwd_step2(BwdPx2 &p, int k, const float4 &g0, const float4 &g1,
                                          float c2, float alpha_thr, float chi_thr,
                                          float acc[9]) {
  bool v0 = k < p.end0, v1 = k < p.end1;
  const float du = p.fu - g0.x;
  const float2 dv = __fadd2_rn(p.fv, f2(-g0.y));
  const float P = g0.z * du * du;
  const float Q = 2.0f * g0.w * du;
  const float2 e = __ffma2_rn(dv, __ffma2_rn(f2(g1.x), dv, f2(Q)), f2(P));
  v0 = v0 && !(e.x > chi_thr);
  v1 = v1 && !(e.y > chi_thr);
  if (!(v0 || v1)) return false;
#if GS_BWD_EX2
  // exp(-e/2) = 2^(e * (-log2(e) / 2)), the scale folded into one packed multiply
  const float2 h = __fmul2_rn(e, f2(-0.72134752044448170f));
  float2 dens = make_float2(ex2_approx(h.x), ex2_approx(h.y));
#else
  const float2 h = __fmul2_rn(e, f2(-0.5f));
  float2 dens = make_float2(__expf(h.x), __expf(h.y));
#endif
  float2 nal = __fmul2_rn(dens, f2(-g1.y));  // -alpha
  v0 = v0 && !(-nal.x < alpha_thr);
  v1 = v1 && !(-nal.y < alpha_thr);
  if (!(v0 || v1)) return false;
  if (!v0) dens.x = nal.x = 0.f;
  if (!v1) dens.y = nal.y = 0.f;
  const float2 oma = __fadd2_rn(__fadd2_rn(nal, f2(1.0f)), f2(kTransEps));
  const float2 rcp = make_float2(rcp_approx(oma.x), rcp_approx(oma.y));
  const float2 prefix = __fmul2_rn(p.Ta, rcp);
  const float2 nw = __fmul2_rn(nal, prefix);  // -weight
  const float2 grgb =
      __ffma2_rn(p.gb, f2(c2), __ffma2_rn(p.gg, f2(g1.w), __fmul2_rn(p.gr, f2(g1.z))));
  const float2 galpha = __ffma2_rn(prefix, grgb, __fmul2_rn(p.nsuffix, rcp));
  const float2 nag = __fmul2_rn(nal, galpha);
  const float2 nau = __fmul2_rn(f2(du), nag);
  const float2 nav = __fmul2_rn(dv, nag);
  acc[0] = nau.x + nau.y;
  acc[1] = nav.x + nav.y;
  acc[2] = du * acc[0];
  acc[3] = fmaf(nau.x, dv.x, nau.y * dv.y);
  acc[4] = fmaf(nav.x, dv.x, nav.y * dv.y);
  acc[5] = fmaf(dens.x, galpha.x, dens.y * galpha.y);
  acc[6] = fmaf(nw.x, p.gr.x, nw.y * p.gr.y);
  acc[7] = fmaf(nw.x, p.gg.x, nw.y * p.gg.y);
  acc[8] = fmaf(nw.x, p.gb.x, nw.y * p.gb.y);
  p.nsuffix = __ffma2_rn(nw, grgb, p.nsuffix);
  if (v0) p.Ta.x = prefix.x;
  if (v1) p.Ta.y = prefix.y;
  return true;
}

// Backward blend. Gradient slot order per Gaussian: 0,1 = d(u,v);
// 2,3,4 = d(conic a,b,c); 5 = d opacity; 6,7,8 = d colour.
template <bool PACKED>
#ifndef GS_BWD_MINB
#define GS_BWD_MINB 8  // resident blocks per SM the backward's register budget targets
#endif
__global__ void __launch_bounds__(kBlendThreads, GS_BWD_MINB) blend_backward_kernel(
    int num_tiles, const int32_t *__restrict__ offsets, int64_t total,
    const int32_t *__restrict__ ids, int n, const float2 *__restrict__ points,
    const float4 *__restrict__ splat, const float *__restrict__ conic,
    const float *__restrict__ opac, const float *__restrict__ colors,
    const float *__restrict__ grad_image, const float *__restrict__ final_t,
    const int32_t *__restrict__ pixel_end, int width, int height, float alpha_thr,
    float trans_thr, float chi_thr, float *__restrict__ g_points, float *__restrict__ g_splat,
    float *__restrict__ g_conic, float *__restrict__ g_opac, float *__restrict__ g_colors,
    const uint8_t *__restrict__ reach, const int32_t *__restrict__ order) {
  __shared__ float4 s_g0[kBatch];
  __shared__ float4 s_g1[kBatch];
  __shared__ float s_b[kBatch];
  __shared__ int32_t s_id[kBatch];
  __shared__ uint8_t s_mask[kBatch];
  __shared__ float s_acc[9 * kBatch];
  __shared__ int s_max_end;

  // block b blends tile order[b] (longest lists first), or tile b
  const int tile = order != nullptr ? __ldg(order + blockIdx.x) : (int)blockIdx.x;
  const int tx = tiles_x_of(width);
  const int tile_x0 = (tile % tx) * GS_TILE, tile_y0 = (tile / tx) * GS_TILE;
  const int t = threadIdx.x, warp = t >> 5;
  const uint32_t lane = t & 31;
  const int2 pp = pixel_in_tile(t);
  const int u = tile_x0 + pp.x;
  const int s = offsets[tile];

  BwdPx px[2];
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    const int v = tile_y0 + pp.y + 4 * h;
    BwdPx &p = px[h];
    p.fu = (float)u;
    p.fv = (float)v;
    p.gr = p.gg = p.gb = 0.f;
    p.Ta = 1.f;
    p.suffix = 0.f;
    p.end = s;
    if (u < width && v < height) {
      size_t q = (size_t)v * width + u;
      p.gr = grad_image[3 * q];
      p.gg = grad_image[3 * q + 1];
      p.gb = grad_image[3 * q + 2];
      // kernel.cu:1028: pixels with an all-zero upstream gradient are skipped.
      if (!(p.gr == 0.0f && p.gg == 0.0f && p.gb == 0.0f)) {
        p.Ta = final_t[q];
        p.end = pixel_end[q];
      }
    }
  }
#if GS_BWD_F32X2
  BwdPx2 P2;
  P2.fu = px[0].fu;
  P2.fv = make_float2(px[0].fv, px[1].fv);
  P2.gr = make_float2(px[0].gr, px[1].gr);
  P2.gg = make_float2(px[0].gg, px[1].gg);
  P2.gb = make_float2(px[0].gb, px[1].gb);
  P2.Ta = make_float2(px[0].Ta, px[1].Ta);
  P2.nsuffix = make_float2(0.f, 0.f);
  P2.end0 = px[0].end;
  P2.end1 = px[1].end;
#endif
  if (t == 0) s_max_end = s;
  __syncthreads();
  const int my_end = max(px[0].end, px[1].end);
  if (my_end > s) atomicMax(&s_max_end, my_end);
  __syncthreads();
  const int max_end = s_max_end;
  if (max_end <= s) return;
  int warp_end = my_end;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) warp_end = max(warp_end, __shfl_xor_sync(0xffffffffu, warp_end, o));

  for (int bend = max_end; bend > s; bend -= kBatch) {
    const int bstart = max(s, bend - kBatch);
    const int cnt = bend - bstart;
    __syncthreads();
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const int slot = t + h * kBlendThreads;
      if (slot < cnt) {
        const int k = bstart + slot;
        int id = __ldg(ids + k);
        Rec r = load_rec<PACKED>(id, n, points, splat, conic, opac, colors);
        s_g0[slot] = r.g0;
        s_g1[slot] = r.g1;
        s_b[slot] = r.b;
        s_id[slot] = id;
        // the forward's masks when it kept them (every entry below the
        // tile's largest pixel end was loaded, so its mask was written)
        s_mask[slot] = reach != nullptr
                           ? __ldg(reach + k)
                           : (uint8_t)reach_mask(r.g0.x, r.g0.y, r.g0.z, r.g0.w, r.g1.x, r.g1.y,
                                                 alpha_thr, chi_thr, tile_x0, tile_y0);
      }
#pragma unroll
      for (int q = 0; q < 9; ++q) s_acc[slot * 9 + q] = 0.f;
    }
    __syncthreads();
    const int jmax = min(cnt, warp_end - bstart);  // entries beyond every lane's end are idle
    // 32 entries at a time, back to front: one ballot of the reach masks
    // (bit b <-> entry j1 - 1 - b), then the visible entries highest first
    for (int j1 = jmax; j1 > 0; j1 -= 32) {
      const int jl = j1 - 1 - (int)lane;
      uint32_t todo = __ballot_sync(0xffffffffu, jl >= 0 && ((s_mask[jl] >> warp) & 1u));
#if GS_BWD_PAIRED
      // two visible entries per step, reduced together (21 shuffles for 18
      // sums instead of 28); their per-pixel updates stay in back-to-front
      // order (j before j2)
      while (todo & (todo - 1)) {
        const int j = j1 - __ffs(todo);
        todo &= todo - 1;
        const int j2 = j1 - __ffs(todo);
        todo &= todo - 1;
        float acc[18];
#pragma unroll
        for (int q = 0; q < 18; ++q) acc[q] = 0.f;
        bool contrib = false;
#if GS_BWD_F32X2
        contrib |= bwd_step2(P2, bstart + j, s_g0[j], s_g1[j], s_b[j], alpha_thr, chi_thr, acc);
        contrib |= bwd_step2(P2, bstart + j2, s_g0[j2], s_g1[j2], s_b[j2], alpha_thr, chi_thr,
                             acc + 9);
#else
        {
          const int k = bstart + j;
          const float4 g0 = s_g0[j];
          const float4 g1 = s_g1[j];
          const float c2 = s_b[j];
          if (k < px[0].end) contrib |= bwd_step(px[0], g0, g1, c2, alpha_thr, chi_thr, acc);
          if (k < px[1].end) contrib |= bwd_step(px[1], g0, g1, c2, alpha_thr, chi_thr, acc);
        }
        {
          const int k = bstart + j2;
          const float4 g0 = s_g0[j2];
          const float4 g1 = s_g1[j2];
          const float c2 = s_b[j2];
          if (k < px[0].end) contrib |= bwd_step(px[0], g0, g1, c2, alpha_thr, chi_thr, acc + 9);
          if (k < px[1].end) contrib |= bwd_step(px[1], g0, g1, c2, alpha_thr, chi_thr, acc + 9);
        }
#endif
        if (!__any_sync(0xffffffffu, contrib)) continue;
        float v16[16];
#pragma unroll
        for (int q = 0; q < 8; ++q) {
          v16[q] = acc[q];
          v16[q + 8] = acc[9 + q];
        }
        const float r16 = reduce16(v16, lane);
        const float r2 = reduce2(acc[8], acc[17], lane);
        const int q16 = (lane >> 1) & 15;
        if ((lane & 1) == 0)
          atomicAdd(&s_acc[(q16 < 8 ? j : j2) * 9 + (q16 & 7)], r16);
        if ((lane & 15) == 0) atomicAdd(&s_acc[((lane >> 4) ? j2 : j) * 9 + 8], r2);
      }
#endif
      while (todo) {
        const int j = j1 - __ffs(todo);
        todo &= todo - 1;
        const int k = bstart + j;
        const float4 g0 = s_g0[j];
        const float4 g1 = s_g1[j];
        const float c2 = s_b[j];
        float acc[9];
#pragma unroll
        for (int q = 0; q < 9; ++q) acc[q] = 0.f;
        bool contrib = false;
#if GS_BWD_F32X2
        contrib = bwd_step2(P2, k, g0, g1, c2, alpha_thr, chi_thr, acc);
#else
        if (k < px[0].end) contrib |= bwd_step(px[0], g0, g1, c2, alpha_thr, chi_thr, acc);
        if (k < px[1].end) contrib |= bwd_step(px[1], g0, g1, c2, alpha_thr, chi_thr, acc);
#endif
        if (!__any_sync(0xffffffffu, contrib)) continue;
        float r8 = reduce8(acc, lane);
        float r9 = reduce1(acc[8]);
        // [j][9] layout: the 8 writing lanes hit 8 consecutive words (distinct banks)
        if ((lane & 3) == 0) atomicAdd(&s_acc[j * 9 + ((lane >> 2) & 7)], r8);
        if (lane == 1) atomicAdd(&s_acc[j * 9 + 8], r9);
      }
    }
    __syncthreads();
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const int slot = t + h * kBlendThreads;
      if (slot < cnt && s_id[slot] >= 0 && s_id[slot] < n) {
        const int id = s_id[slot];
        float a[9];
#pragma unroll
        for (int q = 0; q < 9; ++q) a[q] = s_acc[slot * 9 + q];
        {  // apply the per-Gaussian constants factored out of bwd_step's sums
          const float4 g0 = s_g0[slot];
          const float inv00 = g0.z, inv01 = g0.w, inv11 = s_g1[slot].x;
#if GS_BWD_F32X2  // slots 0-4 and 6-8 were summed negated
          const float su = -a[0], sv = -a[1];
          a[0] = inv00 * su + inv01 * sv;
          a[1] = inv01 * su + inv11 * sv;
          a[2] = 0.5f * a[2];
          a[4] = 0.5f * a[4];
          a[6] = -a[6];
          a[7] = -a[7];
          a[8] = -a[8];
#else
          const float su = a[0], sv = a[1];
          a[0] = inv00 * su + inv01 * sv;
          a[1] = inv01 * su + inv11 * sv;
          a[2] = -0.5f * a[2];
          a[3] = -a[3];
          a[4] = -0.5f * a[4];
#endif
        }
        if (a[0] != 0.f || a[1] != 0.f)
          atomicAdd(reinterpret_cast<float2 *>(g_points) + id, make_float2(a[0], a[1]));
        if (PACKED) {
          float4 *gs4 = reinterpret_cast<float4 *>(g_splat) + 2 * (size_t)id;
          if (a[2] != 0.f || a[3] != 0.f || a[4] != 0.f || a[5] != 0.f)
            atomicAdd(gs4, make_float4(a[2], a[3], a[4], a[5]));
          if (a[6] != 0.f || a[7] != 0.f || a[8] != 0.f)
            atomicAdd(gs4 + 1, make_float4(a[6], a[7], a[8], 0.f));
        } else {
          size_t i3 = 3 * (size_t)id;
          if (a[2] != 0.f) atomicAdd(g_conic + i3, a[2]);
          if (a[3] != 0.f) atomicAdd(g_conic + i3 + 1, a[3]);
          if (a[4] != 0.f) atomicAdd(g_conic + i3 + 2, a[4]);
          if (a[5] != 0.f) atomicAdd(g_opac + id, a[5]);
          if (a[6] != 0.f) atomicAdd(g_colors + i3, a[6]);
          if (a[7] != 0.f) atomicAdd(g_colors + i3 + 1, a[7]);
          if (a[8] != 0.f) atomicAdd(g_colors + i3 + 2, a[8]);
        }
      }
    }
  }
}

// Blend order of the tiles: longest lists first, so that the blend's last
// wave holds short tiles instead of a few long ones that run on while most
// SMs idle (list scheduling, longest first). One block (tile_order_block).
constexpr int kOrderThreads = 1024;

__global__ void __launch_bounds__(kOrderThreads) tile_order_kernel(
    int num_tiles, const int32_t *__restrict__ offsets, int64_t total,
    int32_t *__restrict__ order) {
  __shared__ uint32_t s_count[kOrderClasses];
  tile_order_block(
      num_tiles,
      [&](int tile) {
        const int e = (tile + 1 < num_tiles) ? offsets[tile + 1]
                                             : (total >= 0 ? (int)total : offsets[num_tiles]);
        return e - offsets[tile];
      },
      order, s_count);
}

}  // namespace gs

using namespace gs;

extern "C" int gs_tile_order(int num_tiles, const int32_t *indexing_offset, int64_t total,
                             int32_t *order, void *stream) {
  if (num_tiles < 0 || total < -1 || total >= (1ll << 31) || indexing_offset == nullptr ||
      order == nullptr)
    return GS_ERR_INVALID_ARGUMENT;
  if (num_tiles == 0) return GS_OK;
  tile_order_kernel<<<1, kOrderThreads, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
      num_tiles, indexing_offset, total, order);
  count_launch();
  return launch_status();
}

static inline cudaStream_t as_stream(void *s) { return reinterpret_cast<cudaStream_t>(s); }

extern "C" int gs_rasterize(int num_tiles, const int32_t *indexing_offset, int64_t total,
                            const int32_t *ids_sorted, int n, const float *points_img,
                            const float *conic, const float *opacities, const float *colors,
                            int width, int height, float alpha_threshold,
                            float transmittance_threshold, float chi_squared_threshold,
                            float *image, float *work_final_t, int32_t *work_pixel_end,
                            void *stream) {
  if (num_tiles < 0 || n < 0 || width <= 0 || height <= 0 || total < 0 || total >= (1ll << 31))
    return GS_ERR_INVALID_ARGUMENT;
  if (((uintptr_t)points_img & 7)) return GS_ERR_INVALID_ARGUMENT;
  // rasterizer.cpp:424-428: nothing is drawn when there are no tiles or pairs.
  if (num_tiles == 0 || total == 0) return GS_OK;
  if (num_tiles > tiles_x_of(width) * tiles_y_of(height)) return GS_ERR_INVALID_ARGUMENT;
  blend_forward_kernel<false, true><<<num_tiles, kBlendThreads, 0, as_stream(stream)>>>(
      num_tiles, indexing_offset, total, ids_sorted, n, reinterpret_cast<const float2 *>(points_img),
      nullptr, conic, opacities, colors, width, height, alpha_threshold, transmittance_threshold,
      chi_squared_threshold, image, work_final_t, work_pixel_end, nullptr, nullptr);
  count_launch();
  return launch_status();
}

extern "C" int gs_rasterize_backward(int num_tiles, const int32_t *indexing_offset,
                                     int64_t total, const int32_t *ids_sorted, int n,
                                     const float *grad_image, const float *points_img,
                                     const float *conic, const float *opacities,
                                     const float *colors, int width, int height,
                                     float alpha_threshold, float transmittance_threshold,
                                     float chi_squared_threshold, float *grad_points_img,
                                     float *grad_conic, float *grad_opacities,
                                     float *grad_colors, float *work_final_t,
                                     int32_t *work_pixel_end, void *stream) {
  if (num_tiles < 0 || n < 0 || width <= 0 || height <= 0 || total < 0 || total >= (1ll << 31))
    return GS_ERR_INVALID_ARGUMENT;
  if (((uintptr_t)points_img & 7) || ((uintptr_t)grad_points_img & 7))
    return GS_ERR_INVALID_ARGUMENT;
  if (num_tiles == 0 || total == 0) return GS_OK;
  if (num_tiles > tiles_x_of(width) * tiles_y_of(height)) return GS_ERR_INVALID_ARGUMENT;
  cudaStream_t st = as_stream(stream);
  // The reference backward replays the forward per pixel (kernel.cu:1036-1060);
  // here the replay is a transmittance-only forward pass into the work buffers.
  blend_forward_kernel<false, false><<<num_tiles, kBlendThreads, 0, st>>>(
      num_tiles, indexing_offset, total, ids_sorted, n, reinterpret_cast<const float2 *>(points_img),
      nullptr, conic, opacities, colors, width, height, alpha_threshold, transmittance_threshold,
      chi_squared_threshold, nullptr, work_final_t, work_pixel_end, nullptr, nullptr);
  count_launch();
  blend_backward_kernel<false><<<num_tiles, kBlendThreads, 0, st>>>(
      num_tiles, indexing_offset, total, ids_sorted, n, reinterpret_cast<const float2 *>(points_img),
      nullptr, conic, opacities, colors, grad_image, work_final_t, work_pixel_end, width, height,
      alpha_threshold, transmittance_threshold, chi_squared_threshold, grad_points_img, nullptr,
      grad_conic, grad_opacities, grad_colors, nullptr, nullptr);
  count_launch();
  return launch_status();
}

extern "C" int gs_blend_forward(int num_tiles, const int32_t *indexing_offset, int64_t total,
                                const int32_t *ids_sorted, int n, const float *points_img,
                                const float *splat, int width, int height,
                                float alpha_threshold, float transmittance_threshold,
                                float chi_squared_threshold, float *image, float *final_t,
                                int32_t *pixel_end, uint8_t *reach, const int32_t *tile_order,
                                void *stream) {
  if (num_tiles < 0 || n < 0 || width <= 0 || height <= 0 || total < -1 || total >= (1ll << 31))
    return GS_ERR_INVALID_ARGUMENT;
  if (((uintptr_t)points_img & 7) || ((uintptr_t)splat & 15)) return GS_ERR_INVALID_ARGUMENT;
  if (num_tiles == 0) return GS_OK;
  if (num_tiles > tiles_x_of(width) * tiles_y_of(height)) return GS_ERR_INVALID_ARGUMENT;
  blend_forward_kernel<true, true><<<num_tiles, kBlendThreads, 0, as_stream(stream)>>>(
      num_tiles, indexing_offset, total, ids_sorted, n, reinterpret_cast<const float2 *>(points_img),
      reinterpret_cast<const float4 *>(splat), nullptr, nullptr, nullptr, width, height,
      alpha_threshold, transmittance_threshold, chi_squared_threshold, image, final_t,
      pixel_end, reach, tile_order);
  count_launch();
  return launch_status();
}

extern "C" int gs_blend_backward(int num_tiles, const int32_t *indexing_offset, int64_t total,
                                 const int32_t *ids_sorted, int n, const float *points_img,
                                 const float *splat, const float *grad_image,
                                 const float *final_t, const int32_t *pixel_end, int width,
                                 int height, float alpha_threshold,
                                 float transmittance_threshold, float chi_squared_threshold,
                                 float *grad_points_img, float *grad_splat,
                                 const uint8_t *reach, const int32_t *tile_order,
                                 void *stream) {
  if (num_tiles < 0 || n < 0 || width <= 0 || height <= 0 || total < -1 || total >= (1ll << 31))
    return GS_ERR_INVALID_ARGUMENT;
  if (((uintptr_t)points_img & 7) || ((uintptr_t)splat & 15) || ((uintptr_t)grad_points_img & 7) ||
      ((uintptr_t)grad_splat & 15))
    return GS_ERR_INVALID_ARGUMENT;
  if (num_tiles == 0 || total == 0) return GS_OK;
  if (num_tiles > tiles_x_of(width) * tiles_y_of(height)) return GS_ERR_INVALID_ARGUMENT;
  blend_backward_kernel<true><<<num_tiles, kBlendThreads, 0, as_stream(stream)>>>(
      num_tiles, indexing_offset, total, ids_sorted, n, reinterpret_cast<const float2 *>(points_img),
      reinterpret_cast<const float4 *>(splat), nullptr, nullptr, nullptr, grad_image, final_t,
      pixel_end, width, height, alpha_threshold, transmittance_threshold, chi_squared_threshold,
      grad_points_img, grad_splat, nullptr, nullptr, nullptr, reach, tile_order);
  count_launch();
  return launch_status();
}
