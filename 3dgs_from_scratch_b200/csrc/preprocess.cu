// preprocess.cu -- per-Gaussian stages of the rasterizer.
//
// Two families of kernels:
//  * the reference module's per-function kernels (project, SH, their
//    backwards; ruguangyou/3dgs_from_scratch src/cuda/kernel.cu:411-782),
//    one thread per Gaussian, writing the reference's separate output arrays;
//  * the fused path used by render(): one forward kernel that does projection,
//    EWA covariance, conic, radii, SH colour and tile counts (plus their sum)
//    in a single pass, and one backward kernel for the whole projection +
//    covariance + SH chain.
//
// The fused kernels work on chunks of 128 Gaussians: each chunk's contiguous
// slice of the AoS parameter arrays (means, scales, quats, opacities, sh_dc,
// sh_rest: 236 B/Gaussian) is brought into shared memory by the TMA engine
// (cp.async.bulk, completion on an mbarrier) in persistent, double-buffered
// blocks, so the next chunk streams in while the current one is computed; the
// backward's 236 B/Gaussian of gradients leave through bulk stores. A tail
// chunk, or unaligned pointers, use a one-chunk-per-block variant that stages
// with 128-bit loads.
#include "gs_common.cuh"

namespace gs {

// ---------------------------------------------------------------------------
// reference per-function kernels
// ---------------------------------------------------------------------------

__global__ void __launch_bounds__(256) project_points_kernel(
    int n, const float *__restrict__ means, const float *__restrict__ scales,
    const float *__restrict__ quats, const float *__restrict__ opac,
    const float *__restrict__ w2c, const float *__restrict__ K, float near_plane,
    float far_plane, float min_opacity, float min_radius, float max_radius, int width,
    int height, float *__restrict__ points, float *__restrict__ depths,
    float *__restrict__ cov_out, float *__restrict__ conic_out, float *__restrict__ radii,
    uint8_t *__restrict__ mask) {
  int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  Cam c = load_cam(w2c, K);
  const float *q = quats + 4 * (size_t)i;
  Projected p = project_one(c, width, height, near_plane, far_plane, min_opacity, min_radius,
                            max_radius, means[3 * (size_t)i], means[3 * (size_t)i + 1],
                            means[3 * (size_t)i + 2], scales[3 * (size_t)i],
                            scales[3 * (size_t)i + 1], scales[3 * (size_t)i + 2], q[0], q[1],
                            q[2], q[3], opac[i]);
  if (p.cov_written) {
    cov_out[3 * (size_t)i] = p.cov.x;
    cov_out[3 * (size_t)i + 1] = p.cov.y;
    cov_out[3 * (size_t)i + 2] = p.cov.z;
  }
  if (!p.visible) {
    mask[i] = 0;
    return;
  }
  points[2 * (size_t)i] = p.u;
  points[2 * (size_t)i + 1] = p.v;
  depths[i] = p.depth;
  conic_out[3 * (size_t)i] = p.conic.x;
  conic_out[3 * (size_t)i + 1] = p.conic.y;
  conic_out[3 * (size_t)i + 2] = p.conic.z;
  radii[2 * (size_t)i] = p.ru;
  radii[2 * (size_t)i + 1] = p.rv;
}

__global__ void __launch_bounds__(256) project_points_backward_kernel(
    int n, const float *__restrict__ g_points, const float *__restrict__ g_conic,
    const float *__restrict__ means, const float *__restrict__ scales,
    const float *__restrict__ quats, const float *__restrict__ w2c,
    const float *__restrict__ K, const float *__restrict__ cov, const uint8_t *__restrict__ mask,
    int width, int height, float *__restrict__ g_means, float *__restrict__ g_scales,
    float *__restrict__ g_quats) {
  int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n || !mask[i]) return;
  Cam c = load_cam(w2c, K);
  size_t i3 = 3 * (size_t)i;
  float3 pc = to_camera(c, means[i3], means[i3 + 1], means[i3 + 2]);
  const float *q = quats + 4 * (size_t)i;
  float gm[3], gsc[3], gq[4];
  project_backward_one(c, width, height, pc, g_points[2 * (size_t)i], g_points[2 * (size_t)i + 1],
                       scales[i3], scales[i3 + 1], scales[i3 + 2], q[0], q[1], q[2], q[3],
                       make_float3(cov[i3], cov[i3 + 1], cov[i3 + 2]), g_conic[i3],
                       g_conic[i3 + 1], g_conic[i3 + 2], gm, gsc, gq);
  g_means[i3] = gm[0];
  g_means[i3 + 1] = gm[1];
  g_means[i3 + 2] = gm[2];
  g_scales[i3] = gsc[0];
  g_scales[i3 + 1] = gsc[1];
  g_scales[i3 + 2] = gsc[2];
  float *o = g_quats + 4 * (size_t)i;
  o[0] = gq[0];
  o[1] = gq[1];
  o[2] = gq[2];
  o[3] = gq[3];
}

__global__ void __launch_bounds__(256) sh_forward_kernel(
    int n, const float *__restrict__ campos, const float *__restrict__ means,
    const float *__restrict__ dc, const float *__restrict__ rest,
    const uint8_t *__restrict__ mask, int sh_sigmoid, float *__restrict__ colors) {
  int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n || !mask[i]) return;
  size_t i3 = 3 * (size_t)i;
  ViewDir d = view_dir(__ldg(campos), __ldg(campos + 1), __ldg(campos + 2), means[i3],
                       means[i3 + 1], means[i3 + 2]);
  float b[16];
  sh_basis(d.x, d.y, d.z, b);
  const float *r = rest + 45 * (size_t)i;
  float acc[3];
#pragma unroll
  for (int ch = 0; ch < 3; ++ch) {
    float a = b[0] * dc[i3 + ch];
#pragma unroll
    for (int k = 0; k < 15; ++k) a += b[k + 1] * r[k * 3 + ch];
    acc[ch] = a;
  }
#pragma unroll
  for (int ch = 0; ch < 3; ++ch) colors[i3 + ch] = sh_sigmoid ? ref_sigmoid(acc[ch]) : acc[ch];
}

__global__ void __launch_bounds__(256) sh_backward_kernel(
    int n, const float *__restrict__ g_colors, const float *__restrict__ campos,
    const float *__restrict__ means, const float *__restrict__ rest,
    const float *__restrict__ colors, const uint8_t *__restrict__ mask, int sh_sigmoid,
    float *__restrict__ g_means, float *__restrict__ g_dc, float *__restrict__ g_rest) {
  int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n || !mask[i]) return;
  size_t i3 = 3 * (size_t)i;
  ViewDir d = view_dir(__ldg(campos), __ldg(campos + 1), __ldg(campos + 2), means[i3],
                       means[i3 + 1], means[i3 + 2]);
  float b[16];
  sh_basis(d.x, d.y, d.z, b);
  float g[3];
#pragma unroll
  for (int ch = 0; ch < 3; ++ch) {
    g[ch] = g_colors[i3 + ch];
    if (sh_sigmoid) g[ch] *= colors[i3 + ch] * (1.0f - colors[i3 + ch]);
  }
#pragma unroll
  for (int ch = 0; ch < 3; ++ch) g_dc[i3 + ch] = g[ch] * b[0];
  const float *r = rest + 45 * (size_t)i;
  float *gr = g_rest + 45 * (size_t)i;
#pragma unroll
  for (int k = 0; k < 15; ++k)
#pragma unroll
    for (int ch = 0; ch < 3; ++ch) gr[k * 3 + ch] = g[ch] * b[k + 1];
  float3 gm = sh_dir_backward(d, g[0], g[1], g[2], [&](int k, int ch) { return r[k * 3 + ch]; });
  g_means[i3] = gm.x;
  g_means[i3 + 1] = gm.y;
  g_means[i3 + 2] = gm.z;
}

// ---------------------------------------------------------------------------
// fused path
// ---------------------------------------------------------------------------

constexpr int kPreBlock = 128;  // Gaussians (and threads) per chunk

// Shared-memory image of one chunk's parameter slice, AoS as in HBM. Every
// member starts on a 16-byte boundary (bulk-copy destinations).
struct PreSmem {  // stage_chunk relies on this order and on there being no padding
  float means[kPreBlock * 3];
  float scales[kPreBlock * 3];
  float quats[kPreBlock * 4];
  float opac[kPreBlock];
  float dc[kPreBlock * 3];
  float rest[kPreBlock * 45];
};

// Copy `count` floats global -> shared; 128-bit loads when both ends are
// 16-byte aligned and count % 4 == 0, else 32-bit loads.
__device__ __forceinline__ void stage(float *__restrict__ dst, const float *__restrict__ src,
                                      int count) {
  if ((((uintptr_t)src | (uintptr_t)dst) & 15) == 0 && (count & 3) == 0) {
    const float4 *s4 = reinterpret_cast<const float4 *>(src);
    float4 *d4 = reinterpret_cast<float4 *>(dst);
    for (int k = threadIdx.x; k < (count >> 2); k += blockDim.x) d4[k] = __ldg(s4 + k);
  } else {
    for (int k = threadIdx.x; k < count; k += blockDim.x) dst[k] = __ldg(src + k);
  }
}

// Stages one chunk's parameter slices (means, scales, quats, opacities if
// with_opac, dc, rest: count Gaussians from Gaussian `first`) as one index
// space of float4s, kStageBatch loads in flight per thread before their
// stores (the slices one after the other would wait on memory once per
// slice and loop trip). Falls back to stage() per slice unless every source
// slice is 16-byte aligned and count % 4 == 0.
constexpr int kStageBatch = 8;
static_assert(sizeof(PreSmem) == sizeof(float) * kPreBlock * (3 + 3 + 4 + 1 + 3 + 45),
              "PreSmem is the six slices back to back");

__device__ __forceinline__ void stage_chunk(PreSmem &S, const float *__restrict__ means,
                                            const float *__restrict__ scales,
                                            const float *__restrict__ quats,
                                            const float *__restrict__ opac,
                                            const float *__restrict__ dc,
                                            const float *__restrict__ rest, size_t first,
                                            int count, bool with_opac) {
  const float *p0 = means + 3 * first, *p1 = scales + 3 * first, *p2 = quats + 4 * first;
  const float *p3 = with_opac ? opac + first : nullptr, *p4 = dc + 3 * first;
  const float *p5 = rest + 45 * first;
  const uintptr_t bits = (uintptr_t)p0 | (uintptr_t)p1 | (uintptr_t)p2 | (uintptr_t)p3 |
                         (uintptr_t)p4 | (uintptr_t)p5;
  if ((bits & 15) != 0 || (count & 3) != 0) {
    stage(S.means, p0, 3 * count);
    stage(S.scales, p1, 3 * count);
    stage(S.quats, p2, 4 * count);
    if (with_opac) stage(S.opac, p3, count);
    stage(S.dc, p4, 3 * count);
    stage(S.rest, p5, 45 * count);
    return;
  }
  // float4 counts of the six slices and their running ends
  const int q = count >> 2;
  const int e0 = 3 * q, e1 = e0 + 3 * q, e2 = e1 + 4 * q, e3 = e2 + (with_opac ? q : 0),
            e4 = e3 + 3 * q, e5 = e4 + 45 * q;
  const float4 *s0 = reinterpret_cast<const float4 *>(p0), *s1 = reinterpret_cast<const float4 *>(p1),
               *s2 = reinterpret_cast<const float4 *>(p2), *s3 = reinterpret_cast<const float4 *>(p3),
               *s4 = reinterpret_cast<const float4 *>(p4), *s5 = reinterpret_cast<const float4 *>(p5);
  auto src_of = [&](int i) -> const float4 * {
    return i < e0 ? s0 + i
         : i < e1 ? s1 + (i - e0)
         : i < e2 ? s2 + (i - e1)
         : i < e3 ? s3 + (i - e2)
         : i < e4 ? s4 + (i - e3)
                  : s5 + (i - e4);
  };
  auto dst_of = [&](int i) -> float4 * {
    float *d = i < e0 ? S.means + 4 * i
             : i < e1 ? S.scales + 4 * (i - e0)
             : i < e2 ? S.quats + 4 * (i - e1)
             : i < e3 ? S.opac + 4 * (i - e2)
             : i < e4 ? S.dc + 4 * (i - e3)
                      : S.rest + 4 * (i - e4);
    return reinterpret_cast<float4 *>(d);
  };
  const int step = blockDim.x;
  // PreSmem holds the six slices back to back, each kPreBlock Gaussians long
  const bool dense = count == kPreBlock && with_opac;
  for (int i0 = threadIdx.x; i0 < e5; i0 += kStageBatch * step) {
    float4 v[kStageBatch];
#pragma unroll
    for (int u = 0; u < kStageBatch; ++u) {
      const int i = i0 + u * step;
      if (i < e5) v[u] = __ldg(src_of(i));
    }
#pragma unroll
    for (int u = 0; u < kStageBatch; ++u) {
      const int i = i0 + u * step;
      if (i < e5) *(dense ? reinterpret_cast<float4 *>(&S) + i : dst_of(i)) = v[u];
    }
  }
}

__device__ __forceinline__ void stage_out(float *__restrict__ dst, const float *__restrict__ src,
                                          int count) {
  if ((((uintptr_t)src | (uintptr_t)dst) & 15) == 0 && (count & 3) == 0) {
    const float4 *s4 = reinterpret_cast<const float4 *>(src);
    float4 *d4 = reinterpret_cast<float4 *>(dst);
    for (int k = threadIdx.x; k < (count >> 2); k += blockDim.x) d4[k] = s4[k];
  } else {
    for (int k = threadIdx.x; k < count; k += blockDim.x) dst[k] = src[k];
  }
}

__device__ __forceinline__ void stage_add(float *__restrict__ dst, const float *__restrict__ src,
                                          int count) {
  for (int k = threadIdx.x; k < count; k += blockDim.x) dst[k] += src[k];
}

// Views: camera v at w2c + 16 v, K + 9 v, campos + 3 v; its outputs at
// element offset v * n of each per-Gaussian output array, its pair total at
// total[v]. One staged chunk of parameters serves every view.
struct PreFwdArgs {
  const float *means, *scales, *quats, *opac, *dc, *rest, *w2c, *K, *campos;
  float near_plane, far_plane, min_opacity, min_radius, max_radius;
  int width, height, sh_sigmoid;
  int activate;  // parameters are raw (log-scales, unnormalised quats, logits)
  float2 *points;
  float *depths;
  float2 *radii;
  uint8_t *mask;
  float4 *splat;
  int32_t *tile_counts;
  unsigned long long *total;
  int num_views;
  int64_t n;  // per-view stride of the outputs, in Gaussians
};


// Per-view camera record staged in shared memory by the fused kernels: rows
// 0..2 of world_to_camera (12), fx, fy, cx, cy, camera position (3), pad.
constexpr int kCamFloats = 20;

__device__ __forceinline__ void stage_cameras(const float *w2c, const float *K,
                                              const float *campos, int num_views,
                                              float *s_cam) {
  for (int k = threadIdx.x; k < num_views * kCamFloats; k += blockDim.x) {
    const int v = k / kCamFloats, e = k - v * kCamFloats;
    float x = 0.f;
    if (e < 12)
      x = w2c[16 * v + e];
    else if (e == 12)
      x = K[9 * v + 0];
    else if (e == 13)
      x = K[9 * v + 4];
    else if (e == 14)
      x = K[9 * v + 2];
    else if (e == 15)
      x = K[9 * v + 5];
    else if (e < 19)
      x = campos[3 * v + (e - 16)];
    s_cam[k] = x;
  }
}

__device__ __forceinline__ Cam cam_from_smem(const float *sc) {
  Cam c;
#pragma unroll
  for (int k = 0; k < 12; ++k) c.W[k] = sc[k];
  c.fx = sc[12];
  c.fy = sc[13];
  c.cx = sc[14];
  c.cy = sc[15];
  return c;
}

// Forward for Gaussian i = first + t and view v from the staged chunk (the
// activated scale / quaternion / opacity and the world covariance computed
// once for all views); returns its tile count.
__device__ __forceinline__ int pre_fwd_one(const PreFwdArgs &A, const PreSmem &S,
                                           const float *s_cam, const float Cw[9], float op,
                                           int t, int i, int v) {
  const float *sc = s_cam + kCamFloats * v;
  const Cam c = cam_from_smem(sc);
  const int64_t o = (int64_t)v * A.n + i;
  const float *m = S.means + 3 * t;
  Projected p = project_one_cw(c, A.width, A.height, A.near_plane, A.far_plane, A.min_opacity,
                               A.min_radius, A.max_radius, m[0], m[1], m[2], Cw, op);
  float2 pt = make_float2(0.f, 0.f), rd = make_float2(0.f, 0.f);
  float depth = 0.f;
  float4 s0 = make_float4(0.f, 0.f, 0.f, 0.f), s1 = make_float4(0.f, 0.f, 0.f, 0.f);
  int count = 0;
  if (p.visible) {
    ViewDir d = view_dir(sc[16], sc[17], sc[18], m[0], m[1], m[2]);
    float b[16];
    sh_basis(d.x, d.y, d.z, b);
    const float *r = S.rest + 45 * t;
    float rgb[3];
#pragma unroll
    for (int ch = 0; ch < 3; ++ch) {
      float a = b[0] * S.dc[3 * t + ch];
#pragma unroll
      for (int k = 0; k < 15; ++k) a += b[k + 1] * r[k * 3 + ch];
      if (A.sh_sigmoid) {
        a = ref_sigmoid(a);
      } else {
        a = a + 0.5f;               // wrapper.py:264-265: clamp_min(colors + 0.5, 0)
        a = (a < 0.0f) ? 0.0f : a;  // NaN propagates, as in torch.clamp_min
      }
      rgb[ch] = a;
    }
    pt = make_float2(p.u, p.v);
    rd = make_float2(p.ru, p.rv);
    depth = p.depth;
    s0 = make_float4(p.conic.x, p.conic.y, p.conic.z, op);
    s1 = make_float4(rgb[0], rgb[1], rgb[2], 0.f);
    TileRect tr = tile_rect(p.u, p.v, p.ru, p.rv, A.width, A.height);
    count = tr.empty ? 0 : (tr.x1 - tr.x0 + 1) * (tr.y1 - tr.y0 + 1);
  }
  A.points[o] = pt;
  A.radii[o] = rd;
  A.depths[o] = depth;
  A.mask[o] = p.visible ? 1 : 0;
  A.splat[2 * o] = s0;
  A.splat[2 * o + 1] = s1;
  A.tile_counts[o] = count;
  return count;
}

// All views of one staged chunk. The pair counts go to the block's per-view
// partial sums in shared memory (s_tot, one warp-reduced shared atomic per
// warp and view; a chunk's sum is below 128 * 2^24 tiles, so 32 bits hold
// it), added to the global totals once per chunk: one global atomic per
// view per chunk rather than per warp (same-address atomics from every warp
// of every view serialise in L2).
__device__ __forceinline__ void pre_fwd_views(const PreFwdArgs &A, const PreSmem &S,
                                              const float *s_cam, int t, int i, bool active,
                                              uint32_t *s_tot) {
  float Cw[9];
  float op = 0.f;
  if (active) {
    const float *s = S.scales + 3 * t;
    const float4 q = reinterpret_cast<const float4 *>(S.quats)[t];
    float sx = s[0], sy = s[1], sz = s[2], qx = q.x, qy = q.y, qz = q.z, qw = q.w;
    op = S.opac[t];
    if (A.activate) {
      const Activated a = activate_params(sx, sy, sz, qx, qy, qz, qw, op);
      sx = a.sx; sy = a.sy; sz = a.sz;
      qx = a.qx; qy = a.qy; qz = a.qz; qw = a.qw;
      op = a.opac;
    }
    world_cov(sx, sy, sz, qx, qy, qz, qw, Cw);
  }
  for (int v = 0; v < A.num_views; ++v) {
    int count = active ? pre_fwd_one(A, S, s_cam, Cw, op, t, i, v) : 0;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) count += __shfl_xor_sync(0xffffffffu, count, o);
    if ((threadIdx.x & 31) == 0 && count) atomicAdd(s_tot + v, (uint32_t)count);
  }
}

__device__ __forceinline__ void flush_totals(const PreFwdArgs &A, const uint32_t *s_tot) {
  __syncthreads();
  for (int v = threadIdx.x; v < A.num_views; v += blockDim.x)
    if (s_tot[v]) atomicAdd(A.total + v, (unsigned long long)s_tot[v]);
}

__device__ __forceinline__ void zero_totals(const PreFwdArgs &A, uint32_t *s_tot) {
  for (int v = threadIdx.x; v < A.num_views; v += blockDim.x) s_tot[v] = 0u;
}

// Fused forward, one chunk per block, staged with 128-bit loads. Handles
// Gaussians [base, n) (any alignment); used for the tail of the pipelined
// kernel and when a pointer is not 16-byte aligned.
// One chunk per block. Dynamic shared memory: the chunk stage, then
// num_views per-view partial totals.
__global__ void __launch_bounds__(kPreBlock) preprocess_forward_kernel(PreFwdArgs A, int n, int base) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  PreSmem &S = *reinterpret_cast<PreSmem *>(smem_raw);
  uint32_t *s_tot = reinterpret_cast<uint32_t *>(smem_raw + sizeof(PreSmem));
  float *s_cam = reinterpret_cast<float *>(s_tot + A.num_views);
  zero_totals(A, s_tot);
  stage_cameras(A.w2c, A.K, A.campos, A.num_views, s_cam);
  const int t = threadIdx.x;
  const int first = base + blockIdx.x * kPreBlock;
  const int cnt = min(kPreBlock, n - first);
  const size_t f = (size_t)first;
  stage_chunk(S, A.means, A.scales, A.quats, A.opac, A.dc, A.rest, f, cnt, true);
  __syncthreads();
  pre_fwd_views(A, S, s_cam, t, first + t, t < cnt, s_tot);
  flush_totals(A, s_tot);
}

// Bulk loads of one full chunk (kPreBlock Gaussians from `first`) into S,
// completing on `bar`. With opac == nullptr the opacities are not loaded.
__device__ __forceinline__ void issue_chunk(PreSmem &S, uint64_t *bar, size_t f, const float *means,
                                            const float *scales, const float *quats,
                                            const float *opac, const float *dc,
                                            const float *rest) {
  const uint32_t bytes = kPreBlock * 4 * (3 + 3 + 4 + 3 + 45) + (opac ? kPreBlock * 4 : 0);
  mbar_expect_tx(bar, bytes);
  bulk_load(S.means, means + 3 * f, kPreBlock * 12, bar);
  bulk_load(S.scales, scales + 3 * f, kPreBlock * 12, bar);
  bulk_load(S.quats, quats + 4 * f, kPreBlock * 16, bar);
  if (opac) bulk_load(S.opac, opac + f, kPreBlock * 4, bar);
  bulk_load(S.dc, dc + 3 * f, kPreBlock * 12, bar);
  bulk_load(S.rest, rest + 45 * f, kPreBlock * 180, bar);
}

// Fused forward, persistent and double-buffered: while a block computes chunk
// c from one shared-memory stage, the TMA engine fills the other stage with
// chunk c + gridDim.x. Only full chunks; all parameter pointers 16-byte aligned.
__global__ void __launch_bounds__(kPreBlock) preprocess_forward_pipe_kernel(PreFwdArgs A,
                                                                           int num_chunks,
                                                                           uint32_t *status) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  PreSmem *stg = reinterpret_cast<PreSmem *>(smem_raw);
  uint32_t *s_tot = reinterpret_cast<uint32_t *>(smem_raw + 2 * sizeof(PreSmem));
  float *s_cam = reinterpret_cast<float *>(s_tot + A.num_views);
  __shared__ __align__(8) uint64_t bars[2];
  const int t = threadIdx.x;
  zero_totals(A, s_tot);
  stage_cameras(A.w2c, A.K, A.campos, A.num_views, s_cam);
  if (t == 0) {
    mbar_init(&bars[0], 1);
    mbar_init(&bars[1], 1);
    fence_mbar_init();
  }
  __syncthreads();
  int c = blockIdx.x;
  if (t == 0 && c < num_chunks)
    issue_chunk(stg[0], &bars[0], (size_t)c * kPreBlock, A.means, A.scales, A.quats, A.opac, A.dc,
                A.rest);
  uint32_t phase = 0;  // bit s: parity of the next completion of bars[s]
  int s = 0;
  for (; c < num_chunks; c += gridDim.x) {
    const int nc = c + gridDim.x;
    if (t == 0 && nc < num_chunks)
      issue_chunk(stg[s ^ 1], &bars[s ^ 1], (size_t)nc * kPreBlock, A.means, A.scales, A.quats,
                  A.opac, A.dc, A.rest);
    // every thread polls (bounded); the abort decision is made block-wide
    if (!__syncthreads_and(mbar_wait(&bars[s], (phase >> s) & 1u))) {
      if (t == 0) {
        atomicExch(status, (uint32_t)GS_ERR_DEVICE_TIMEOUT);
        // let the copies already issued land before the block exits (bounded)
        mbar_wait(&bars[s], (phase >> s) & 1u);
        if (nc < num_chunks) mbar_wait(&bars[s ^ 1], (phase >> (s ^ 1)) & 1u);
      }
      return;
    }
    phase ^= 1u << s;
    pre_fwd_views(A, stg[s], s_cam, t, c * kPreBlock + t, true, s_tot);
    flush_totals(A, s_tot);  // per chunk: the 32-bit partials cannot overflow
    __syncthreads();  // every thread is done with stg[s] (and s_tot) before reuse
    zero_totals(A, s_tot);
    s ^= 1;
  }
}

// Views: camera v at w2c + 16 v, K + 9 v, campos + 3 v; its culling mask at
// mask + v * n and its upstream gradients at g_points + v * gp_vstride,
// g_splat + v * gs_vstride. The gradients of all views are summed.
struct PreBwdArgs {
  const float *means, *scales, *quats, *opac, *dc, *rest, *w2c, *K, *campos;
  int width, height, sh_sigmoid;
  int activate;    // parameters are raw; gradients are w.r.t. the raw parameters
  int accumulate;  // add the gradients into the outputs instead of writing them
  const uint8_t *mask;
  const float *g_points;
  int gp_stride;
  const float *g_splat;
  int gs_stride;
  float *g_means, *g_scales, *g_quats, *g_opac, *g_dc, *g_rest;
  int num_views;
  int64_t n;
  int64_t gp_vstride, gs_vstride;
  int vec_upstream;  // upstream gradients loadable as float2 / float4
};

// One view's upstream values for one Gaussian: its culling mask, d loss /
// d points_img, and d loss / d splat record (conic a, b, c, opacity; r, g, b).
struct Upstream {
  float2 gp;
  float4 s0, s1;
  uint32_t mask;
};

__device__ __forceinline__ Upstream load_upstream(const PreBwdArgs &A, int v, int64_t i) {
  Upstream u;
  u.mask = A.mask[v * A.n + i];
  const float *gp = A.g_points + v * A.gp_vstride + i * A.gp_stride;
  const float *gsp = A.g_splat + v * A.gs_vstride + i * A.gs_stride;
  if (A.vec_upstream) {  // strides 2 and 8 floats, 8- and 16-byte aligned
    u.gp = __ldg(reinterpret_cast<const float2 *>(gp));
    u.s0 = __ldg(reinterpret_cast<const float4 *>(gsp));
    u.s1 = __ldg(reinterpret_cast<const float4 *>(gsp) + 1);
  } else {
    u.gp = make_float2(gp[0], gp[1]);
    u.s0 = make_float4(gsp[0], gsp[1], gsp[2], gsp[3]);
    u.s1 = make_float4(gsp[4], gsp[5], gsp[6], 0.f);
  }
  return u;
}

// Backward for Gaussian i = first + t over every view: reads the staged
// parameters and overwrites them in place with the summed gradients (zeros
// for a Gaussian culled in every view). Per view: the projection's and the
// image covariance's chain down to d loss / d (world covariance) and the
// mean, and the SH chain; once per Gaussian, after the views: the world
// covariance to scale and rotation (linear, so applied to the sum over the
// views) and the activation Jacobians (exp, quaternion normalisation,
// sigmoid; also linear). With several views the SH-rest gradient is summed
// in rest_acc (this thread's 45 floats) while the staged coefficients are
// still needed.
template <bool MULTI>
__device__ __forceinline__ void pre_bwd_one(const PreBwdArgs &A, PreSmem &S, const float *s_cam,
                                            float *rest_acc, int t, int i) {
  float *m = S.means + 3 * t;
  float *s = S.scales + 3 * t;
  float *qq = S.quats + 4 * t;
  float *dcc = S.dc + 3 * t;
  float *r = S.rest + 45 * t;
  const float px = m[0], py = m[1], pz = m[2];
  float sx = s[0], sy = s[1], sz = s[2];
  float4 q = reinterpret_cast<const float4 *>(S.quats)[t];
  Activated act;
  if (A.activate) {
    act = activate_params(sx, sy, sz, q.x, q.y, q.z, q.w, S.opac[t]);
    sx = act.sx;
    sy = act.sy;
    sz = act.sz;
    q = make_float4(act.qx, act.qy, act.qz, act.qw);
  }
  float Sg[6];
  world_cov_sym(sx, sy, sz, q.x, q.y, q.z, q.w, Sg);
  float gm[3] = {0.f, 0.f, 0.f}, gSg[6] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
  float gdc[3] = {0.f, 0.f, 0.f}, opac_grad = 0.f;
  bool any = false;
  const int views = MULTI ? A.num_views : 1;
  if (MULTI) {
#pragma unroll
    for (int k = 0; k < 45; ++k) rest_acc[k] = 0.f;
  }
  // The upstream gradients of view v + 1 are loaded while view v is computed
  // (their loads do not wait on the view's mask test).
  Upstream up = load_upstream(A, 0, i);
  for (int v = 0; v < views; ++v) {
    const Upstream cur = up;
    if (v + 1 < views) up = load_upstream(A, v + 1, i);
    if (!cur.mask) continue;
    any = true;
    const float *sc = s_cam + kCamFloats * v;
    const Cam c = cam_from_smem(sc);
    view_proj_backward(c, A.width, A.height, to_camera(c, px, py, pz), Sg, cur.gp.x, cur.gp.y,
                       cur.s0.x, cur.s0.y, cur.s0.z, gm, gSg);
    opac_grad += cur.s0.w;
    const ViewDir d = view_dir(sc[16], sc[17], sc[18], px, py, pz);
    float b[16];
    sh_basis(d.x, d.y, d.z, b);
    float g[3];
    sh_view_backward(d, b, dcc, [&](int k, int ch) { return r[k * 3 + ch]; }, cur.s1.x,
                     cur.s1.y, cur.s1.z, A.sh_sigmoid, g, gm, gdc);
    if (MULTI) {
#pragma unroll
      for (int k = 0; k < 15; ++k)
#pragma unroll
        for (int ch = 0; ch < 3; ++ch) rest_acc[k * 3 + ch] += g[ch] * b[k + 1];
    } else {
#pragma unroll
      for (int k = 0; k < 15; ++k)
#pragma unroll
        for (int ch = 0; ch < 3; ++ch) r[k * 3 + ch] = g[ch] * b[k + 1];
    }
  }
  float gsc[3] = {0.f, 0.f, 0.f}, gq[4] = {0.f, 0.f, 0.f, 0.f};
  if (any) {
    cov_backward(gSg, sx, sy, sz, q.x, q.y, q.z, q.w, gsc, gq);
    if (A.activate) {
      // exp backward (scale), normalisation backward (quaternion)
      gsc[0] *= act.sx;
      gsc[1] *= act.sy;
      gsc[2] *= act.sz;
      const float nq = fmaxf(act.qnorm, 1e-12f);
      if (act.qnorm >= 1e-12f) {
        const float dot = q.x * gq[0] + q.y * gq[1] + q.z * gq[2] + q.w * gq[3];
        gq[0] = (gq[0] - q.x * dot) / nq;
        gq[1] = (gq[1] - q.y * dot) / nq;
        gq[2] = (gq[2] - q.z * dot) / nq;
        gq[3] = (gq[3] - q.w * dot) / nq;
      } else {
        gq[0] /= nq;
        gq[1] /= nq;
        gq[2] /= nq;
        gq[3] /= nq;
      }
      opac_grad = opac_grad * (1.0f - act.opac) * act.opac;  // sigmoid backward
    }
    if (MULTI) {
#pragma unroll
      for (int k = 0; k < 45; ++k) r[k] = rest_acc[k];
    }
  } else {
#pragma unroll
    for (int k = 0; k < 45; ++k) r[k] = 0.f;
  }
#pragma unroll
  for (int k = 0; k < 3; ++k) {
    m[k] = gm[k];
    s[k] = gsc[k];
    dcc[k] = gdc[k];
  }
#pragma unroll
  for (int k = 0; k < 4; ++k) qq[k] = gq[k];
  if (A.g_opac) {
    if (A.accumulate)
      A.g_opac[i] += opac_grad;
    else
      A.g_opac[i] = opac_grad;
  }
}

// Shared memory of the multi-view backward beyond its stages: the SH-rest
// gradient accumulators, one row of 45 floats per thread.
constexpr size_t kPreRestAccBytes = sizeof(float) * kPreBlock * 45;

#ifndef GS_PRE_MULTI_MINB
#define GS_PRE_MULTI_MINB 3  // resident blocks per SM the multi-view register budget targets
#endif
#ifndef GS_PRE_MULTI_SIMPLE
#define GS_PRE_MULTI_SIMPLE 1  // 1: the multi-view backward stages chunks with plain loads
#endif

// Fused backward, one chunk per block (tail / unaligned fallback).
template <bool MULTI>
__global__ void __launch_bounds__(kPreBlock, MULTI ? GS_PRE_MULTI_MINB : 1)
    preprocess_backward_kernel(PreBwdArgs A, int n, int base) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  PreSmem &S = *reinterpret_cast<PreSmem *>(smem_raw);
  float *rest_acc = reinterpret_cast<float *>(smem_raw + sizeof(PreSmem));
  float *s_cam = reinterpret_cast<float *>(smem_raw + sizeof(PreSmem) +
                                           (MULTI ? kPreRestAccBytes : 0));
  stage_cameras(A.w2c, A.K, A.campos, A.num_views, s_cam);
  const int first = base + blockIdx.x * kPreBlock;
  const int cnt = min(kPreBlock, n - first);
  const size_t f = (size_t)first;
  stage_chunk(S, A.means, A.scales, A.quats, A.opac, A.dc, A.rest, f, cnt, A.activate != 0);
  __syncthreads();
  const int t = threadIdx.x;
  if (t < cnt) pre_bwd_one<MULTI>(A, S, s_cam, rest_acc + 45 * t, t, first + t);
  __syncthreads();
  if (A.accumulate) {
    stage_add(A.g_means + 3 * f, S.means, 3 * cnt);
    stage_add(A.g_scales + 3 * f, S.scales, 3 * cnt);
    stage_add(A.g_quats + 4 * f, S.quats, 4 * cnt);
    stage_add(A.g_dc + 3 * f, S.dc, 3 * cnt);
    stage_add(A.g_rest + 45 * f, S.rest, 45 * cnt);
  } else {
    stage_out(A.g_means + 3 * f, S.means, 3 * cnt);
    stage_out(A.g_scales + 3 * f, S.scales, 3 * cnt);
    stage_out(A.g_quats + 4 * f, S.quats, 4 * cnt);
    stage_out(A.g_dc + 3 * f, S.dc, 3 * cnt);
    stage_out(A.g_rest + 45 * f, S.rest, 45 * cnt);
  }
}

// Fused backward, persistent and double-buffered like the forward; the
// gradients leave shared memory through bulk stores. Before a stage is
// refilled its stores must have read their source (bulk wait_group.read).
template <bool MULTI>
__global__ void __launch_bounds__(kPreBlock) preprocess_backward_pipe_kernel(PreBwdArgs A,
                                                                            int num_chunks,
                                                                            uint32_t *status) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  PreSmem *stg = reinterpret_cast<PreSmem *>(smem_raw);
  float *rest_acc = reinterpret_cast<float *>(smem_raw + 2 * sizeof(PreSmem));
  float *s_cam = reinterpret_cast<float *>(smem_raw + 2 * sizeof(PreSmem) +
                                           (MULTI ? kPreRestAccBytes : 0));
  __shared__ __align__(8) uint64_t bars[2];
  const int t = threadIdx.x;
  stage_cameras(A.w2c, A.K, A.campos, A.num_views, s_cam);
  if (t == 0) {
    mbar_init(&bars[0], 1);
    mbar_init(&bars[1], 1);
    fence_mbar_init();
  }
  __syncthreads();
  int c = blockIdx.x;
  if (t == 0 && c < num_chunks)
    issue_chunk(stg[0], &bars[0], (size_t)c * kPreBlock, A.means, A.scales, A.quats,
                A.activate ? A.opac : nullptr, A.dc, A.rest);
  uint32_t phase = 0;
  int s = 0;
  for (; c < num_chunks; c += gridDim.x) {
    const int nc = c + gridDim.x;
    if (t == 0 && nc < num_chunks) {
      bulk_wait_read_all();  // stg[s ^ 1]'s stores from the previous chunk have read it
      issue_chunk(stg[s ^ 1], &bars[s ^ 1], (size_t)nc * kPreBlock, A.means, A.scales, A.quats,
                  A.activate ? A.opac : nullptr, A.dc, A.rest);
    }
    if (!__syncthreads_and(mbar_wait(&bars[s], (phase >> s) & 1u))) {
      if (t == 0) {
        atomicExch(status, (uint32_t)GS_ERR_DEVICE_TIMEOUT);
        mbar_wait(&bars[s], (phase >> s) & 1u);
        if (nc < num_chunks) mbar_wait(&bars[s ^ 1], (phase >> (s ^ 1)) & 1u);
        bulk_wait_all();
      }
      return;
    }
    phase ^= 1u << s;
    const int i0 = c * kPreBlock;
    pre_bwd_one<MULTI>(A, stg[s], s_cam, rest_acc + 45 * t, t, i0 + t);
    fence_proxy_async_smem();  // this thread's shared writes are visible to the bulk stores
    __syncthreads();
    if (t == 0) {
      const size_t f = (size_t)i0;
      PreSmem &S = stg[s];
      if (A.accumulate) {  // global += shared, performed by the TMA engine in L2
        bulk_reduce_add(A.g_means + 3 * f, S.means, kPreBlock * 12);
        bulk_reduce_add(A.g_scales + 3 * f, S.scales, kPreBlock * 12);
        bulk_reduce_add(A.g_quats + 4 * f, S.quats, kPreBlock * 16);
        bulk_reduce_add(A.g_dc + 3 * f, S.dc, kPreBlock * 12);
        bulk_reduce_add(A.g_rest + 45 * f, S.rest, kPreBlock * 180);
      } else {
        bulk_store(A.g_means + 3 * f, S.means, kPreBlock * 12);
        bulk_store(A.g_scales + 3 * f, S.scales, kPreBlock * 12);
        bulk_store(A.g_quats + 4 * f, S.quats, kPreBlock * 16);
        bulk_store(A.g_dc + 3 * f, S.dc, kPreBlock * 12);
        bulk_store(A.g_rest + 45 * f, S.rest, kPreBlock * 180);
      }
      bulk_commit();
    }
    s ^= 1;
  }
  if (t == 0) bulk_wait_all();
}

static bool aligned16(const void *p) { return ((uintptr_t)p & 15) == 0; }

// Grid of a persistent kernel: every SM filled to its occupancy for this
// kernel and shared-memory size (queried per call: both vary by caller).
static int pipe_grid(int num_chunks, const void *kernel, size_t smem) {
  int dev = 0;
  cudaGetDevice(&dev);
  int per_sm = 0;
  cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kernel, kPreBlock, smem);
  if (per_sm < 1) per_sm = 1;
  int sms = 148;
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const int g = sms * per_sm;
  return num_chunks < g ? num_chunks : g;
}

}  // namespace gs

// ---------------------------------------------------------------------------
// C ABI
// ---------------------------------------------------------------------------
using namespace gs;

static inline cudaStream_t as_stream(void *s) { return reinterpret_cast<cudaStream_t>(s); }

extern "C" int gs_project_points(int n, const float *means, const float *scales,
                                 const float *quats, const float *opacities,
                                 const float *world_to_camera, const float *intrinsic,
                                 float near_plane, float far_plane, float min_opacity,
                                 float min_radius, float max_radius, int width, int height,
                                 float *points_img, float *depths, float *cov_img, float *conic,
                                 float *radii, uint8_t *mask, void *stream) {
  if (n < 0 || width <= 0 || height <= 0) return GS_ERR_INVALID_ARGUMENT;
  if (n == 0) return GS_OK;
  int blocks = (n + 255) / 256;
  project_points_kernel<<<blocks, 256, 0, as_stream(stream)>>>(
      n, means, scales, quats, opacities, world_to_camera, intrinsic, near_plane, far_plane,
      min_opacity, min_radius, max_radius, width, height, points_img, depths, cov_img, conic,
      radii, mask);
  count_launch();
  return launch_status();
}

extern "C" int gs_project_points_backward(int n, const float *grad_points_img,
                                          const float *grad_conic, const float *means,
                                          const float *scales, const float *quats,
                                          const float *world_to_camera, const float *intrinsic,
                                          const float *cov_img, const uint8_t *mask, int width,
                                          int height, float *grad_means, float *grad_scales,
                                          float *grad_quats, void *stream) {
  if (n < 0 || width <= 0 || height <= 0) return GS_ERR_INVALID_ARGUMENT;
  if (n == 0) return GS_OK;
  int blocks = (n + 255) / 256;
  project_points_backward_kernel<<<blocks, 256, 0, as_stream(stream)>>>(
      n, grad_points_img, grad_conic, means, scales, quats, world_to_camera, intrinsic, cov_img,
      mask, width, height, grad_means, grad_scales, grad_quats);
  count_launch();
  return launch_status();
}

extern "C" int gs_evaluate_sh(int n, const float *camera_pos, const float *means,
                              const float *sh_dc, const float *sh_rest, const uint8_t *mask,
                              int sh_sigmoid, float *colors, void *stream) {
  if (n < 0) return GS_ERR_INVALID_ARGUMENT;
  if (n == 0) return GS_OK;
  int blocks = (n + 255) / 256;
  sh_forward_kernel<<<blocks, 256, 0, as_stream(stream)>>>(n, camera_pos, means, sh_dc, sh_rest,
                                                            mask, sh_sigmoid, colors);
  count_launch();
  return launch_status();
}

extern "C" int gs_evaluate_sh_backward(int n, const float *grad_colors, const float *camera_pos,
                                       const float *means, const float *sh_rest,
                                       const float *colors, const uint8_t *mask, int sh_sigmoid,
                                       float *grad_means, float *grad_dc, float *grad_rest,
                                       void *stream) {
  if (n < 0) return GS_ERR_INVALID_ARGUMENT;
  if (n == 0) return GS_OK;
  int blocks = (n + 255) / 256;
  sh_backward_kernel<<<blocks, 256, 0, as_stream(stream)>>>(n, grad_colors, camera_pos, means,
                                                             sh_rest, colors, mask, sh_sigmoid,
                                                             grad_means, grad_dc, grad_rest);
  count_launch();
  return launch_status();
}

#ifndef GS_PRE_FWD_MULTI_SIMPLE
#define GS_PRE_FWD_MULTI_SIMPLE 1  // 1: the multi-view forward stages chunks with plain loads
#endif

static int launch_preprocess_forward(const PreFwdArgs &A, int n, cudaStream_t st) {
  const bool pipe_ok = aligned16(A.means) && aligned16(A.scales) && aligned16(A.quats) &&
                       aligned16(A.opac) && aligned16(A.dc) && aligned16(A.rest) &&
                       !(A.num_views > 1 && GS_PRE_FWD_MULTI_SIMPLE);
  const int full = pipe_ok ? n / kPreBlock : 0;
  // per-view pair totals and staged cameras after the stage(s)
  const size_t tot_bytes = sizeof(uint32_t) * (size_t)A.num_views * (1 + kCamFloats);
  if (2 * sizeof(PreSmem) + tot_bytes > 200 * 1024) return GS_ERR_CAPACITY;  // views per launch
  if (full > 0) {
    const size_t smem = 2 * sizeof(PreSmem) + tot_bytes;
    cudaFuncSetAttribute(preprocess_forward_pipe_kernel,
                         cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    const int grid = pipe_grid(full, (const void *)preprocess_forward_pipe_kernel, smem);
    preprocess_forward_pipe_kernel<<<grid, kPreBlock, smem, st>>>(A, full, device_status_word());
    count_launch();
  }
  const int base = full * kPreBlock;
  if (base < n) {
    const size_t smem = sizeof(PreSmem) + tot_bytes;
    cudaFuncSetAttribute(preprocess_forward_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         (int)smem);
    const int blocks = (n - base + kPreBlock - 1) / kPreBlock;  // one chunk per block
    preprocess_forward_kernel<<<blocks, kPreBlock, smem, st>>>(A, n, base);
    count_launch();
  }
  return launch_status();
}

static int preprocess_forward_impl(int n, int num_views, const float *means, const float *scales,
                                   const float *quats, const float *opacities,
                                   const float *sh_dc, const float *sh_rest, const float *w2c,
                                   const float *K, const float *campos, float near_plane,
                                   float far_plane, float min_opacity, float min_radius,
                                   float max_radius, int width, int height, int sh_sigmoid,
                                   int activate, float *points_img, float *depths, float *radii,
                                   uint8_t *mask, float *splat, int32_t *tile_counts,
                                   int64_t *totals, void *stream) {
  if (n < 0 || num_views < 1 || width <= 0 || height <= 0 || totals == nullptr)
    return GS_ERR_INVALID_ARGUMENT;
  if (((uintptr_t)points_img & 7) || ((uintptr_t)radii & 7) || ((uintptr_t)splat & 15) ||
      ((uintptr_t)totals & 7))
    return GS_ERR_INVALID_ARGUMENT;
  cudaStream_t st = as_stream(stream);
  int rc = zero_async(totals, sizeof(int64_t) * num_views, st);
  if (rc || n == 0) return rc;
  if (tile_counts == nullptr) return GS_ERR_INVALID_ARGUMENT;
  PreFwdArgs A{means, scales, quats, opacities, sh_dc, sh_rest, w2c, K, campos, near_plane,
               far_plane, min_opacity, min_radius, max_radius, width, height, sh_sigmoid,
               activate, reinterpret_cast<float2 *>(points_img), depths,
               reinterpret_cast<float2 *>(radii), mask, reinterpret_cast<float4 *>(splat),
               tile_counts, reinterpret_cast<unsigned long long *>(totals), num_views,
               (int64_t)n};
  return launch_preprocess_forward(A, n, st);
}

extern "C" int gs_preprocess_forward(int n, const float *means, const float *scales,
                                     const float *quats, const float *opacities,
                                     const float *sh_dc, const float *sh_rest,
                                     const float *world_to_camera, const float *intrinsic,
                                     const float *camera_pos, float near_plane,
                                     float far_plane, float min_opacity, float min_radius,
                                     float max_radius, int width, int height, int sh_sigmoid,
                                     int activate, float *points_img, float *depths,
                                     float *radii, uint8_t *mask, float *splat,
                                     int32_t *tile_counts, int64_t *total_dev, void *stream) {
  return preprocess_forward_impl(n, 1, means, scales, quats, opacities, sh_dc, sh_rest,
                                 world_to_camera, intrinsic, camera_pos, near_plane, far_plane,
                                 min_opacity, min_radius, max_radius, width, height, sh_sigmoid,
                                 activate, points_img, depths, radii, mask, splat, tile_counts,
                                 total_dev, stream);
}

extern "C" int gs_preprocess_forward_views(
    int n, int num_views, const float *means, const float *scales, const float *quats,
    const float *opacities, const float *sh_dc, const float *sh_rest,
    const float *world_to_cameras, const float *intrinsics, const float *camera_positions,
    float near_plane, float far_plane, float min_opacity, float min_radius, float max_radius,
    int width, int height, int sh_sigmoid, int activate, float *points_img, float *depths,
    float *radii, uint8_t *mask, float *splat, int32_t *tile_counts, int64_t *totals,
    void *stream) {
  return preprocess_forward_impl(n, num_views, means, scales, quats, opacities, sh_dc, sh_rest,
                                 world_to_cameras, intrinsics, camera_positions, near_plane,
                                 far_plane, min_opacity, min_radius, max_radius, width, height,
                                 sh_sigmoid, activate, points_img, depths, radii, mask, splat,
                                 tile_counts, totals, stream);
}

template <bool MULTI>
static int launch_preprocess_backward(const PreBwdArgs &A, int n, cudaStream_t st) {
  const bool pipe_ok = aligned16(A.means) && aligned16(A.scales) && aligned16(A.quats) &&
                       (!A.activate || aligned16(A.opac)) && aligned16(A.dc) &&
                       aligned16(A.rest) && aligned16(A.g_means) && aligned16(A.g_scales) &&
                       aligned16(A.g_quats) && aligned16(A.g_dc) && aligned16(A.g_rest);
  const int full = (pipe_ok && !(MULTI && GS_PRE_MULTI_SIMPLE)) ? n / kPreBlock : 0;
  const size_t extra =
      (MULTI ? kPreRestAccBytes : 0) + sizeof(float) * kCamFloats * (size_t)A.num_views;
  if (sizeof(PreSmem) + extra > 200 * 1024) return GS_ERR_CAPACITY;  // views per launch
  if (full > 0) {
    const size_t smem = 2 * sizeof(PreSmem) + extra;
    cudaFuncSetAttribute(preprocess_backward_pipe_kernel<MULTI>,
                         cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    const int grid = pipe_grid(full, (const void *)preprocess_backward_pipe_kernel<MULTI>, smem);
    preprocess_backward_pipe_kernel<MULTI>
        <<<grid, kPreBlock, smem, st>>>(A, full, device_status_word());
    count_launch();
  }
  const int base = full * kPreBlock;
  if (base < n) {
    const size_t smem = sizeof(PreSmem) + extra;
    cudaFuncSetAttribute(preprocess_backward_kernel<MULTI>,
                         cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    const int blocks = (n - base + kPreBlock - 1) / kPreBlock;
    preprocess_backward_kernel<MULTI><<<blocks, kPreBlock, smem, st>>>(A, n, base);
    count_launch();
  }
  return launch_status();
}

// n Gaussians; the per-view upstream arrays (mask, grad_points_img,
// grad_splat) hold view_stride Gaussians per view (>= n: a sub-range of the
// views' arrays when the pointers are offset to its first Gaussian).
static int preprocess_backward_impl(int n, int num_views, const float *means,
                                    const float *scales, const float *quats,
                                    const float *opacities, const float *sh_dc,
                                    const float *sh_rest, const float *w2c, const float *K,
                                    const float *campos, int width, int height, int sh_sigmoid,
                                    int activate, int accumulate, const uint8_t *mask,
                                    const float *grad_points_img, int gp_stride,
                                    const float *grad_splat, int gs_stride, float *grad_means,
                                    float *grad_scales, float *grad_quats,
                                    float *grad_opacities, float *grad_dc, float *grad_rest,
                                    void *stream, int64_t view_stride = -1) {
  if (view_stride < 0) view_stride = n;
  if (n < 0 || num_views < 1 || width <= 0 || height <= 0 || gp_stride < 2 || gs_stride < 7 ||
      view_stride < n)
    return GS_ERR_INVALID_ARGUMENT;
  if (activate && opacities == nullptr) return GS_ERR_INVALID_ARGUMENT;
  if (n == 0) return GS_OK;
  cudaStream_t st = as_stream(stream);
  PreBwdArgs A{means, scales, quats, opacities, sh_dc, sh_rest, w2c, K, campos, width, height,
               sh_sigmoid, activate, accumulate, mask, grad_points_img, gp_stride, grad_splat,
               gs_stride, grad_means, grad_scales, grad_quats, grad_opacities, grad_dc,
               grad_rest, num_views, view_stride, view_stride * gp_stride,
               view_stride * gs_stride,
               (gp_stride == 2 && gs_stride == 8 && ((uintptr_t)grad_points_img & 7) == 0 &&
                ((uintptr_t)grad_splat & 15) == 0)
                   ? 1
                   : 0};
  return num_views > 1 ? launch_preprocess_backward<true>(A, n, st)
                       : launch_preprocess_backward<false>(A, n, st);
}

extern "C" int gs_preprocess_backward(int n, const float *means, const float *scales,
                                      const float *quats, const float *opacities,
                                      const float *sh_dc, const float *sh_rest,
                                      const float *world_to_camera, const float *intrinsic,
                                      const float *camera_pos, int width, int height,
                                      int sh_sigmoid, int activate, int accumulate,
                                      const uint8_t *mask, const float *grad_points_img,
                                      int gp_stride, const float *grad_splat, int gs_stride,
                                      float *grad_means, float *grad_scales, float *grad_quats,
                                      float *grad_opacities, float *grad_dc, float *grad_rest,
                                      void *stream) {
  return preprocess_backward_impl(n, 1, means, scales, quats, opacities, sh_dc, sh_rest,
                                  world_to_camera, intrinsic, camera_pos, width, height,
                                  sh_sigmoid, activate, accumulate, mask, grad_points_img,
                                  gp_stride, grad_splat, gs_stride, grad_means, grad_scales,
                                  grad_quats, grad_opacities, grad_dc, grad_rest, stream);
}

extern "C" int gs_preprocess_backward_views(
    int n, int num_views, const float *means, const float *scales, const float *quats,
    const float *opacities, const float *sh_dc, const float *sh_rest,
    const float *world_to_cameras, const float *intrinsics, const float *camera_positions,
    int width, int height, int sh_sigmoid, int activate, int accumulate, const uint8_t *mask,
    const float *grad_points_img, int gp_stride, const float *grad_splat, int gs_stride,
    float *grad_means, float *grad_scales, float *grad_quats, float *grad_opacities,
    float *grad_dc, float *grad_rest, void *stream) {
  return preprocess_backward_impl(n, num_views, means, scales, quats, opacities, sh_dc, sh_rest,
                                  world_to_cameras, intrinsics, camera_positions, width, height,
                                  sh_sigmoid, activate, accumulate, mask, grad_points_img,
                                  gp_stride, grad_splat, gs_stride, grad_means, grad_scales,
                                  grad_quats, grad_opacities, grad_dc, grad_rest, stream);
}

extern "C" int gs_preprocess_backward_views_range(
    int n_total, int first, int count, int num_views, const float *means, const float *scales,
    const float *quats, const float *opacities, const float *sh_dc, const float *sh_rest,
    const float *world_to_cameras, const float *intrinsics, const float *camera_positions,
    int width, int height, int sh_sigmoid, int activate, int accumulate, const uint8_t *mask,
    const float *grad_points_img, int gp_stride, const float *grad_splat, int gs_stride,
    float *grad_means, float *grad_scales, float *grad_quats, float *grad_opacities,
    float *grad_dc, float *grad_rest, void *stream) {
  if (n_total < 0 || first < 0 || count < 0 || (int64_t)first + count > n_total)
    return GS_ERR_INVALID_ARGUMENT;
  if (count == 0) return GS_OK;
  const size_t f = (size_t)first;
  return preprocess_backward_impl(
      count, num_views, means + 3 * f, scales + 3 * f, quats + 4 * f,
      opacities ? opacities + f : nullptr, sh_dc + 3 * f, sh_rest + 45 * f, world_to_cameras,
      intrinsics, camera_positions, width, height, sh_sigmoid, activate, accumulate, mask + f,
      grad_points_img + (size_t)gp_stride * f, gp_stride, grad_splat + (size_t)gs_stride * f,
      gs_stride, grad_means + 3 * f, grad_scales + 3 * f, grad_quats + 4 * f,
      grad_opacities ? grad_opacities + f : nullptr, grad_dc + 3 * f, grad_rest + 45 * f, stream,
      n_total);
}
