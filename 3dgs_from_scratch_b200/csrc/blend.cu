// blend.cu -- per-tile alpha blending, forward and backward.
//
// One 256-thread block per 16x16 tile, one thread per pixel. Warp w owns an
// 8x4 pixel sub-block (2 across, 4 down), so a warp's pixels are spatially
// compact. The tile's Gaussian list is streamed in batches of 256: each
// thread stages one Gaussian's record in shared memory, together with an
// 8-bit mask of the sub-blocks whose pixels that Gaussian can reach (a
// conservative bound; see reach_mask), and then every warp walks the batch
// from shared memory, skipping records its sub-block cannot see as one
// uniform branch. Per pixel the arithmetic is the reference's, operation for
// operation (ruguangyou/3dgs_from_scratch src/cuda/kernel.cu:954-982 forward,
// 1066-1110 backward), so images and per-pixel gradient terms match it.
//
// The forward records each pixel's final transmittance and the index one past
// its last contributing list entry, so the backward needs no forward replay.
// The backward walks each batch back to front, pre-reduces the 9 gradient
// terms of a (warp, Gaussian) pair with a transposing warp-shuffle reduction
// (14 shuffles instead of 45), accumulates warps into shared memory, and
// issues one vector atomic per gradient group per (tile, Gaussian).
#include "gs_common.cuh"

namespace gs {

constexpr int kBlendThreads = 256;
constexpr int kBatch = 256;

// Pixel owned by a thread: warp w -> 8x4 sub-block at (8*(w&1), 4*(w>>1)).
__device__ __forceinline__ int2 pixel_in_tile(int t) {
  int w = t >> 5, l = t & 31;
  return make_int2(8 * (w & 1) + (l & 7), 4 * (w >> 1) + (l >> 3));
}

// Gaussian record in shared memory: g0 = (u, v, A, B), g1 = (C, opacity, r, g), b.
struct Rec {
  float4 g0, g1;
  float b;
};

// Bitmask of the tile's 8 warp sub-blocks that may hold a pixel with
// q <= q_cut, where q_cut = min(chi2, 2 ln(opacity / alpha_thr)) bounds both
// of the reference's skip tests (q > chi2, alpha < alpha_thr). The ellipse
// {d : d^T Q d <= qc} lies in the box |dx| <= sqrt(qc C / det),
// |dy| <= sqrt(qc A / det). The float evaluation of q at a pixel has a
// relative error below 3e-7 * R with R = 2 (A + C)^2 / det (the ratio of the
// summed term magnitudes to q); conics with R >= 2000 reach everything, and
// for the rest qc = 1.01 q_cut + 0.05 exceeds q_cut by far more than that
// error, so a skipped record fails one of the reference's tests at every
// pixel of the sub-block. Non-finite input reaches everything.
__device__ __forceinline__ uint32_t reach_mask(float u, float v, float A, float B, float C,
                                               float opac, float alpha_thr, float chi_thr,
                                               int tile_x0, int tile_y0) {
  double q_cut = (double)chi_thr;
  if (alpha_thr > 0.0f) {
    if (!(opac > 0.0f)) return 0xffu;  // degenerate opacity: evaluate normally
    double qa = 2.0 * log((double)opac / (double)alpha_thr);
    q_cut = fmin(q_cut, qa);
  }
  double a = A, c = C, b = B;
  double det = a * c - b * b;
  if (!(A > 0.0f) || !(C > 0.0f) || !(det > 0.0) || !isfinite(u) || !isfinite(v) ||
      !isfinite(q_cut) || !(2.0 * (a + c) * (a + c) < 2000.0 * det))
    return 0xffu;
  if (q_cut < -0.05) return 0u;  // opacity below the alpha threshold: alpha < thr everywhere
  double qc = fmax(q_cut, 0.0) * 1.01 + 0.05;
  double hx = sqrt(qc * c / det);
  double hy = sqrt(qc * a / det);
  uint32_t m = 0;
#pragma unroll
  for (int w = 0; w < 8; ++w) {
    double bx0 = tile_x0 + 8 * (w & 1), by0 = tile_y0 + 4 * (w >> 1);
    bool hit = (u + hx >= bx0) && (u - hx <= bx0 + 7.0) && (v + hy >= by0) && (v - hy <= by0 + 3.0);
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

// Forward blend. With ACCUM = false only the transmittance bookkeeping is
// done (the replay used by the reference-API backward).
template <bool PACKED, bool ACCUM>
__global__ void __launch_bounds__(kBlendThreads) blend_forward_kernel(
    int num_tiles, const int32_t *__restrict__ offsets, int64_t total,
    const int32_t *__restrict__ ids, int n, const float2 *__restrict__ points,
    const float4 *__restrict__ splat, const float *__restrict__ conic,
    const float *__restrict__ opac, const float *__restrict__ colors, int width, int height,
    float alpha_thr, float trans_thr, float chi_thr, float *__restrict__ image,
    float *__restrict__ final_t, int32_t *__restrict__ pixel_end) {
  __shared__ float4 s_g0[kBatch];
  __shared__ float4 s_g1[kBatch];
  __shared__ float s_b[kBatch];
  __shared__ uint8_t s_mask[kBatch];

  const int tile = blockIdx.x;
  const int tx = tiles_x_of(width);
  const int tile_x0 = (tile % tx) * GS_TILE, tile_y0 = (tile / tx) * GS_TILE;
  const int t = threadIdx.x, warp = t >> 5;
  const int2 pp = pixel_in_tile(t);
  const int u = tile_x0 + pp.x, v = tile_y0 + pp.y;
  const bool inside = (u < width) && (v < height);
  const float fu = (float)u, fv = (float)v;

  const int s = offsets[tile];
  const int e = (tile + 1 < num_tiles) ? offsets[tile + 1] : (int)total;

  float T = 1.0f, cr = 0.f, cg = 0.f, cb = 0.f;
  int last = s;
  bool done = !inside;

  for (int base = s; base < e; base += kBatch) {
    if (__syncthreads_count(!done) == 0) break;
    const int k = base + t;
    if (k < e) {
      int id = __ldg(ids + k);
      Rec r = load_rec<PACKED>(id, n, points, splat, conic, opac, colors);
      s_g0[t] = r.g0;
      s_g1[t] = r.g1;
      s_b[t] = r.b;
      s_mask[t] = (uint8_t)reach_mask(r.g0.x, r.g0.y, r.g0.z, r.g0.w, r.g1.x, r.g1.y, alpha_thr,
                                      chi_thr, tile_x0, tile_y0);
    }
    __syncthreads();
    const int cnt = min(kBatch, e - base);
    if (!__all_sync(0xffffffffu, done)) {
      for (int j = 0; j < cnt; ++j) {
        if (!((s_mask[j] >> warp) & 1u)) continue;  // uniform across the warp
        if (done) break;
        const float4 g0 = s_g0[j];
        const float du = fu - g0.x;
        const float dv = fv - g0.y;
        const float4 g1 = s_g1[j];
        const float inv00 = g0.z, inv01 = g0.w, inv11 = g1.x;
        float exponent = inv00 * du * du + 2.0f * inv01 * du * dv + inv11 * dv * dv;
        if (exponent > chi_thr) continue;
        float alpha = expf(-0.5f * exponent) * g1.y;
        if (alpha < alpha_thr) continue;
        if (ACCUM) {
          float weight = alpha * T;
          cr += weight * g1.z;
          cg += weight * g1.w;
          cb += weight * s_b[j];
        }
        float one_minus_alpha = 1.0f - alpha + kTransEps;
        T *= one_minus_alpha;
        last = base + j + 1;
        if (T < trans_thr) done = true;
      }
    }
  }
  if (inside) {
    size_t px = (size_t)v * width + u;
    if (ACCUM && image) {
      image[3 * px] = cr;
      image[3 * px + 1] = cg;
      image[3 * px + 2] = cb;
    }
    final_t[px] = T;
    pixel_end[px] = last;
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

// Backward blend. Gradient slot order per Gaussian: 0,1 = d(u,v);
// 2,3,4 = d(conic a,b,c); 5 = d opacity; 6,7,8 = d colour.
template <bool PACKED>
__global__ void __launch_bounds__(kBlendThreads) blend_backward_kernel(
    int num_tiles, const int32_t *__restrict__ offsets, int64_t total,
    const int32_t *__restrict__ ids, int n, const float2 *__restrict__ points,
    const float4 *__restrict__ splat, const float *__restrict__ conic,
    const float *__restrict__ opac, const float *__restrict__ colors,
    const float *__restrict__ grad_image, const float *__restrict__ final_t,
    const int32_t *__restrict__ pixel_end, int width, int height, float alpha_thr,
    float trans_thr, float chi_thr, float *__restrict__ g_points, float *__restrict__ g_splat,
    float *__restrict__ g_conic, float *__restrict__ g_opac, float *__restrict__ g_colors) {
  __shared__ float4 s_g0[kBatch];
  __shared__ float4 s_g1[kBatch];
  __shared__ float s_b[kBatch];
  __shared__ int32_t s_id[kBatch];
  __shared__ uint8_t s_mask[kBatch];
  __shared__ float s_acc[kBatch * 9];
  __shared__ int s_max_end;

  const int tile = blockIdx.x;
  const int tx = tiles_x_of(width);
  const int tile_x0 = (tile % tx) * GS_TILE, tile_y0 = (tile / tx) * GS_TILE;
  const int t = threadIdx.x, warp = t >> 5;
  const uint32_t lane = t & 31;
  const int2 pp = pixel_in_tile(t);
  const int u = tile_x0 + pp.x, v = tile_y0 + pp.y;
  const bool inside = (u < width) && (v < height);
  const float fu = (float)u, fv = (float)v;

  const int s = offsets[tile];
  
  float gr = 0.f, gg = 0.f, gb = 0.f, Ta = 1.f;
  int my_end = s;
  if (inside) {
    size_t px = (size_t)v * width + u;
    gr = grad_image[3 * px];
    gg = grad_image[3 * px + 1];
    gb = grad_image[3 * px + 2];
    // kernel.cu:1028: pixels with an all-zero upstream gradient are skipped.
    if (!(gr == 0.0f && gg == 0.0f && gb == 0.0f)) {
      Ta = final_t[px];
      my_end = pixel_end[px];
    }
  }
  if (t == 0) s_max_end = s;
  __syncthreads();
  if (my_end > s) atomicMax(&s_max_end, my_end);
  __syncthreads();
  const int max_end = s_max_end;
  if (max_end <= s) return;
  int warp_end = my_end;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) warp_end = max(warp_end, __shfl_xor_sync(0xffffffffu, warp_end, o));

  float suffix = 0.0f;
  for (int bend = max_end; bend > s; bend -= kBatch) {
    const int bstart = max(s, bend - kBatch);
    const int cnt = bend - bstart;
    __syncthreads();
    if (t < cnt) {
      const int k = bstart + t;
      int id = __ldg(ids + k);
      Rec r = load_rec<PACKED>(id, n, points, splat, conic, opac, colors);
      s_g0[t] = r.g0;
      s_g1[t] = r.g1;
      s_b[t] = r.b;
      s_id[t] = id;
      s_mask[t] = (uint8_t)reach_mask(r.g0.x, r.g0.y, r.g0.z, r.g0.w, r.g1.x, r.g1.y, alpha_thr,
                                      chi_thr, tile_x0, tile_y0);
    }
#pragma unroll
    for (int q = 0; q < 9; ++q) s_acc[q * kBatch + t] = 0.f;
    __syncthreads();
    const int jmax = min(cnt, warp_end - bstart);  // entries beyond every lane's end are idle
    for (int j = jmax - 1; j >= 0; --j) {
      if (!((s_mask[j] >> warp) & 1u)) continue;  // uniform across the warp
      const int k = bstart + j;
      float vals[9];
      bool contrib = false;
      if (k < my_end) {
        const float4 g0 = s_g0[j];
        const float4 g1 = s_g1[j];
        const float du = fu - g0.x;
        const float dv = fv - g0.y;
        const float inv00 = g0.z, inv01 = g0.w, inv11 = g1.x;
        float exponent = inv00 * du * du + 2.0f * inv01 * du * dv + inv11 * dv * dv;
        if (exponent <= chi_thr) {
          float density = expf(-0.5f * exponent);
          float alpha = density * g1.y;
          if (alpha >= alpha_thr) {
            contrib = true;
            float one_minus_alpha = 1.0f - alpha + kTransEps;
            float prefix_t = Ta / one_minus_alpha;
            float weight = alpha * prefix_t;
            const float c0 = g1.z, c1 = g1.w, c2 = s_b[j];
            float grad_rgb = gr * c0 + gg * c1 + gb * c2;
            float grad_alpha = prefix_t * grad_rgb - suffix / one_minus_alpha;
            float grad_u = inv00 * du + inv01 * dv;
            float grad_v = inv01 * du + inv11 * dv;
            vals[0] = grad_u * alpha * grad_alpha;
            vals[1] = grad_v * alpha * grad_alpha;
            vals[2] = -0.5f * du * du * alpha * grad_alpha;
            vals[3] = -du * dv * alpha * grad_alpha;
            vals[4] = -0.5f * dv * dv * alpha * grad_alpha;
            vals[5] = density * grad_alpha;
            vals[6] = weight * gr;
            vals[7] = weight * gg;
            vals[8] = weight * gb;
            suffix += weight * grad_rgb;
            Ta = prefix_t;
          }
        }
      }
      if (!__any_sync(0xffffffffu, contrib)) continue;
      if (!contrib) {
#pragma unroll
        for (int q = 0; q < 9; ++q) vals[q] = 0.f;
      }
      float r8 = reduce8(vals, lane);
      float r9 = reduce1(vals[8]);
      if ((lane & 3) == 0) atomicAdd(&s_acc[((lane >> 2) & 7) * kBatch + j], r8);
      if (lane == 1) atomicAdd(&s_acc[8 * kBatch + j], r9);
    }
    __syncthreads();
    if (t < cnt && s_id[t] >= 0 && s_id[t] < n) {
      const int id = s_id[t];
      float a[9];
#pragma unroll
      for (int q = 0; q < 9; ++q) a[q] = s_acc[q * kBatch + t];
      if (a[0] != 0.f || a[1] != 0.f) atomicAdd(reinterpret_cast<float2 *>(g_points) + id, make_float2(a[0], a[1]));
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

}  // namespace gs

using namespace gs;

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
      chi_squared_threshold, image, work_final_t, work_pixel_end);
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
      chi_squared_threshold, nullptr, work_final_t, work_pixel_end);
  count_launch();
  blend_backward_kernel<false><<<num_tiles, kBlendThreads, 0, st>>>(
      num_tiles, indexing_offset, total, ids_sorted, n, reinterpret_cast<const float2 *>(points_img),
      nullptr, conic, opacities, colors, grad_image, work_final_t, work_pixel_end, width, height,
      alpha_threshold, transmittance_threshold, chi_squared_threshold, grad_points_img, nullptr,
      grad_conic, grad_opacities, grad_colors);
  count_launch();
  return launch_status();
}

extern "C" int gs_blend_forward(int num_tiles, const int32_t *indexing_offset, int64_t total,
                                const int32_t *ids_sorted, int n, const float *points_img,
                                const float *splat, int width, int height,
                                float alpha_threshold, float transmittance_threshold,
                                float chi_squared_threshold, float *image, float *final_t,
                                int32_t *pixel_end, void *stream) {
  if (num_tiles < 0 || n < 0 || width <= 0 || height <= 0 || total < 0 || total >= (1ll << 31))
    return GS_ERR_INVALID_ARGUMENT;
  if (((uintptr_t)points_img & 7) || ((uintptr_t)splat & 15)) return GS_ERR_INVALID_ARGUMENT;
  if (num_tiles == 0) return GS_OK;
  if (num_tiles > tiles_x_of(width) * tiles_y_of(height)) return GS_ERR_INVALID_ARGUMENT;
  blend_forward_kernel<true, true><<<num_tiles, kBlendThreads, 0, as_stream(stream)>>>(
      num_tiles, indexing_offset, total, ids_sorted, n, reinterpret_cast<const float2 *>(points_img),
      reinterpret_cast<const float4 *>(splat), nullptr, nullptr, nullptr, width, height,
      alpha_threshold, transmittance_threshold, chi_squared_threshold, image, final_t,
      pixel_end);
  count_launch();
  return launch_status();
}

extern "C" int gs_blend_backward(int num_tiles, const int32_t *indexing_offset, int64_t total,
                                 const int32_t *ids_sorted, int n, const float *points_img,
                                 const float *splat, const float *grad_image,
                                 const float *final_t, const int32_t *pixel_end, int width,
                                 int height, float alpha_threshold,
                                 float transmittance_threshold, float chi_squared_threshold,
                                 float *grad_points_img, float *grad_splat, void *stream) {
  if (num_tiles < 0 || n < 0 || width <= 0 || height <= 0 || total < 0 || total >= (1ll << 31))
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
      grad_points_img, grad_splat, nullptr, nullptr, nullptr);
  count_launch();
  return launch_status();
}
