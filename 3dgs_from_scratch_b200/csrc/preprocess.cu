// preprocess.cu -- per-Gaussian stages of the rasterizer.
//
// Two families of kernels:
//  * the reference module's per-function kernels (project, SH, their
//    backwards; ruguangyou/3dgs_from_scratch src/cuda/kernel.cu:411-782),
//    one thread per Gaussian, writing the reference's separate output arrays;
//  * the fused path used by render(): one forward kernel that does projection,
//    EWA covariance, conic, radii, SH colour, tile count and the exclusive scan
//    of the tile counts (decoupled look-back) in a single pass, and one
//    backward kernel for the whole projection + covariance + SH chain.
//
// The fused kernels stage each block's contiguous slice of the AoS parameter
// arrays (means, scales, quats, opacities, sh_dc, sh_rest: 236 B/Gaussian)
// into shared memory with 128-bit coalesced loads, so every warp-wide global
// access is a full, aligned transaction even for the 180 B/Gaussian SH block.
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

constexpr int kPreBlock = 128;  // Gaussians (and threads) per block

// Shared-memory image of one block's parameter slice, AoS as in HBM.
struct PreSmem {
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

// Fused forward: one thread per Gaussian. Tile counts are written per
// Gaussian and their block sum is added into *total_out.
__global__ void __launch_bounds__(kPreBlock) preprocess_forward_kernel(
    int n, const float *__restrict__ means, const float *__restrict__ scales,
    const float *__restrict__ quats, const float *__restrict__ opac,
    const float *__restrict__ dc, const float *__restrict__ rest,
    const float *__restrict__ w2c, const float *__restrict__ K,
    const float *__restrict__ campos, float near_plane, float far_plane, float min_opacity,
    float min_radius, float max_radius, int width, int height, int sh_sigmoid,
    float2 *__restrict__ points, float *__restrict__ depths, float2 *__restrict__ radii,
    uint8_t *__restrict__ mask, float4 *__restrict__ splat, int32_t *__restrict__ tile_counts,
    unsigned long long *__restrict__ total_out) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  PreSmem &S = *reinterpret_cast<PreSmem *>(smem_raw);
  const int first = blockIdx.x * kPreBlock;
  const int cnt = min(kPreBlock, n - first);
  const size_t f = (size_t)first;
  stage(S.means, means + 3 * f, 3 * cnt);
  stage(S.scales, scales + 3 * f, 3 * cnt);
  stage(S.quats, quats + 4 * f, 4 * cnt);
  stage(S.opac, opac + f, cnt);
  stage(S.dc, dc + 3 * f, 3 * cnt);
  stage(S.rest, rest + 45 * f, 45 * cnt);
  __syncthreads();

  const int t = threadIdx.x;
  const int i = first + t;
  int count = 0;
  if (t < cnt) {
    Cam c = load_cam(w2c, K);
    const float *m = S.means + 3 * t;
    const float *s = S.scales + 3 * t;
    const float4 q = reinterpret_cast<const float4 *>(S.quats)[t];
    Projected p = project_one(c, width, height, near_plane, far_plane, min_opacity, min_radius,
                              max_radius, m[0], m[1], m[2], s[0], s[1], s[2], q.x, q.y, q.z, q.w,
                              S.opac[t]);
    float2 pt = make_float2(0.f, 0.f), rd = make_float2(0.f, 0.f);
    float depth = 0.f;
    float4 s0 = make_float4(0.f, 0.f, 0.f, 0.f), s1 = make_float4(0.f, 0.f, 0.f, 0.f);
    if (p.visible) {
      ViewDir d = view_dir(__ldg(campos), __ldg(campos + 1), __ldg(campos + 2), m[0], m[1], m[2]);
      float b[16];
      sh_basis(d.x, d.y, d.z, b);
      const float *r = S.rest + 45 * t;
      float rgb[3];
#pragma unroll
      for (int ch = 0; ch < 3; ++ch) {
        float a = b[0] * S.dc[3 * t + ch];
#pragma unroll
        for (int k = 0; k < 15; ++k) a += b[k + 1] * r[k * 3 + ch];
        if (sh_sigmoid) {
          a = ref_sigmoid(a);
        } else {
          a = a + 0.5f;                 // wrapper.py:264-265: clamp_min(colors + 0.5, 0)
          a = (a < 0.0f) ? 0.0f : a;    // NaN propagates, as in torch.clamp_min
        }
        rgb[ch] = a;
      }
      pt = make_float2(p.u, p.v);
      rd = make_float2(p.ru, p.rv);
      depth = p.depth;
      s0 = make_float4(p.conic.x, p.conic.y, p.conic.z, S.opac[t]);
      s1 = make_float4(rgb[0], rgb[1], rgb[2], 0.f);
      TileRect tr = tile_rect(p.u, p.v, p.ru, p.rv, width, height);
      count = tr.empty ? 0 : (tr.x1 - tr.x0 + 1) * (tr.y1 - tr.y0 + 1);
    }
    points[i] = pt;
    radii[i] = rd;
    depths[i] = depth;
    mask[i] = p.visible ? 1 : 0;
    splat[2 * (size_t)i] = s0;
    splat[2 * (size_t)i + 1] = s1;
    tile_counts[i] = count;
  }
  // Sum of the tile counts: warp reduction, one atomic per warp.
  unsigned long long c = (unsigned long long)count;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) c += __shfl_xor_sync(0xffffffffu, c, o);
  if ((t & 31) == 0 && c) atomicAdd(total_out, c);
}

// Fused backward: one thread per Gaussian. Writes every output element
// (zeros for Gaussians that were culled).
__global__ void __launch_bounds__(kPreBlock) preprocess_backward_kernel(
    int n, const float *__restrict__ means, const float *__restrict__ scales,
    const float *__restrict__ quats, const float *__restrict__ dc,
    const float *__restrict__ rest, const float *__restrict__ w2c,
    const float *__restrict__ K, const float *__restrict__ campos, int width, int height,
    int sh_sigmoid, const uint8_t *__restrict__ mask, const float *__restrict__ g_points,
    int gp_stride, const float *__restrict__ g_splat, int gs_stride,
    float *__restrict__ g_means, float *__restrict__ g_scales, float *__restrict__ g_quats,
    float *__restrict__ g_opac, float *__restrict__ g_dc, float *__restrict__ g_rest) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  PreSmem &S = *reinterpret_cast<PreSmem *>(smem_raw);
  const int first = blockIdx.x * kPreBlock;
  const int cnt = min(kPreBlock, n - first);
  const size_t f = (size_t)first;
  stage(S.means, means + 3 * f, 3 * cnt);
  stage(S.scales, scales + 3 * f, 3 * cnt);
  stage(S.quats, quats + 4 * f, 4 * cnt);
  stage(S.dc, dc + 3 * f, 3 * cnt);
  stage(S.rest, rest + 45 * f, 45 * cnt);
  __syncthreads();

  const int t = threadIdx.x;
  const int i = first + t;
  // Results for means/scales/quats/dc are staged in place of the inputs
  // (each thread only overwrites its own slots after reading them); the
  // 45 SH-rest gradients go to S.rest the same way.
  if (t < cnt) {
    float *m = S.means + 3 * t;
    float *s = S.scales + 3 * t;
    float *qq = S.quats + 4 * t;
    float *dcc = S.dc + 3 * t;
    float *r = S.rest + 45 * t;
    float opac_grad = 0.f;
    if (mask[i]) {
      Cam c = load_cam(w2c, K);
      float px = m[0], py = m[1], pz = m[2];
      float sx = s[0], sy = s[1], sz = s[2];
      float4 q = reinterpret_cast<const float4 *>(S.quats)[t];
      float3 pc = to_camera(c, px, py, pz);
      float3 cov = image_cov(c, width, height, pc, sx, sy, sz, q.x, q.y, q.z, q.w);
      const float *gp = g_points + (size_t)i * gp_stride;
      const float *gsp = g_splat + (size_t)i * gs_stride;
      float gm[3], gsc[3], gq[4];
      project_backward_one(c, width, height, pc, gp[0], gp[1], sx, sy, sz, q.x, q.y, q.z, q.w,
                           cov, gsp[0], gsp[1], gsp[2], gm, gsc, gq);
      opac_grad = gsp[3];

      ViewDir d = view_dir(__ldg(campos), __ldg(campos + 1), __ldg(campos + 2), px, py, pz);
      float b[16];
      sh_basis(d.x, d.y, d.z, b);
      float g[3];
#pragma unroll
      for (int ch = 0; ch < 3; ++ch) {
        float raw = b[0] * dcc[ch];
#pragma unroll
        for (int k = 0; k < 15; ++k) raw += b[k + 1] * r[k * 3 + ch];
        float gc = gsp[4 + ch];
        if (sh_sigmoid) {
          float col = ref_sigmoid(raw);
          gc *= col * (1.0f - col);
        } else {
          gc = (raw + 0.5f >= 0.0f) ? gc : 0.0f;  // clamp_min backward passes where >= 0
        }
        g[ch] = gc;
      }
      float3 gmsh = sh_dir_backward(d, g[0], g[1], g[2], [&](int k, int ch) { return r[k * 3 + ch]; });
#pragma unroll
      for (int k = 0; k < 15; ++k)
#pragma unroll
        for (int ch = 0; ch < 3; ++ch) r[k * 3 + ch] = g[ch] * b[k + 1];
#pragma unroll
      for (int ch = 0; ch < 3; ++ch) dcc[ch] = g[ch] * b[0];
      m[0] = gm[0] + gmsh.x;
      m[1] = gm[1] + gmsh.y;
      m[2] = gm[2] + gmsh.z;
      s[0] = gsc[0];
      s[1] = gsc[1];
      s[2] = gsc[2];
      qq[0] = gq[0];
      qq[1] = gq[1];
      qq[2] = gq[2];
      qq[3] = gq[3];
    } else {
#pragma unroll
      for (int k = 0; k < 3; ++k) m[k] = s[k] = dcc[k] = 0.f;
#pragma unroll
      for (int k = 0; k < 4; ++k) qq[k] = 0.f;
#pragma unroll
      for (int k = 0; k < 45; ++k) r[k] = 0.f;
    }
    if (g_opac) g_opac[i] = opac_grad;
  }
  __syncthreads();
  stage_out(g_means + 3 * f, S.means, 3 * cnt);
  stage_out(g_scales + 3 * f, S.scales, 3 * cnt);
  stage_out(g_quats + 4 * f, S.quats, 4 * cnt);
  stage_out(g_dc + 3 * f, S.dc, 3 * cnt);
  stage_out(g_rest + 45 * f, S.rest, 45 * cnt);
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

extern "C" int gs_preprocess_forward(int n, const float *means, const float *scales,
                                     const float *quats, const float *opacities,
                                     const float *sh_dc, const float *sh_rest,
                                     const float *world_to_camera, const float *intrinsic,
                                     const float *camera_pos, float near_plane,
                                     float far_plane, float min_opacity, float min_radius,
                                     float max_radius, int width, int height, int sh_sigmoid,
                                     float *points_img, float *depths, float *radii,
                                     uint8_t *mask, float *splat, int32_t *tile_counts,
                                     int64_t *total_dev, void *stream) {
  if (n < 0 || width <= 0 || height <= 0 || total_dev == nullptr) return GS_ERR_INVALID_ARGUMENT;
  if (((uintptr_t)points_img & 7) || ((uintptr_t)radii & 7) || ((uintptr_t)splat & 15) ||
      ((uintptr_t)total_dev & 7))
    return GS_ERR_INVALID_ARGUMENT;
  cudaStream_t st = as_stream(stream);
  int rc = cuda_status(cudaMemsetAsync(total_dev, 0, sizeof(int64_t), st));
  if (rc || n == 0) return rc;
  if (tile_counts == nullptr) return GS_ERR_INVALID_ARGUMENT;
  const int blocks = (n + kPreBlock - 1) / kPreBlock;
  preprocess_forward_kernel<<<blocks, kPreBlock, sizeof(PreSmem), st>>>(
      n, means, scales, quats, opacities, sh_dc, sh_rest, world_to_camera, intrinsic,
      camera_pos, near_plane, far_plane, min_opacity, min_radius, max_radius, width, height,
      sh_sigmoid, reinterpret_cast<float2 *>(points_img), depths,
      reinterpret_cast<float2 *>(radii), mask, reinterpret_cast<float4 *>(splat), tile_counts,
      reinterpret_cast<unsigned long long *>(total_dev));
  count_launch();
  return launch_status();
}

extern "C" int gs_preprocess_backward(int n, const float *means, const float *scales,
                                      const float *quats, const float *sh_dc,
                                      const float *sh_rest, const float *world_to_camera,
                                      const float *intrinsic, const float *camera_pos,
                                      int width, int height, int sh_sigmoid,
                                      const uint8_t *mask, const float *grad_points_img,
                                      int gp_stride, const float *grad_splat, int gs_stride,
                                      float *grad_means, float *grad_scales, float *grad_quats,
                                      float *grad_opacities, float *grad_dc, float *grad_rest,
                                      void *stream) {
  if (n < 0 || width <= 0 || height <= 0 || gp_stride < 2 || gs_stride < 7)
    return GS_ERR_INVALID_ARGUMENT;
  if (n == 0) return GS_OK;
  const size_t smem = sizeof(PreSmem);  // 30 KB: below the 48 KB default, no opt-in
  int blocks = (n + kPreBlock - 1) / kPreBlock;
  preprocess_backward_kernel<<<blocks, kPreBlock, smem, as_stream(stream)>>>(
      n, means, scales, quats, sh_dc, sh_rest, world_to_camera, intrinsic, camera_pos, width,
      height, sh_sigmoid, mask, grad_points_img, gp_stride, grad_splat, gs_stride, grad_means,
      grad_scales, grad_quats, grad_opacities, grad_dc, grad_rest);
  count_launch();
  return launch_status();
}
