// densify.cu -- adaptive density control (prune / clone / split / opacity
// reset) on the flat parameter and Adam-state buffers, on the device.
//
// The reference's Strategy (src/strategy.py:5-250) keeps, per Gaussian, the
// sum of the screen-space means-gradient norms and a visibility count
// (_update_state, :48-72), and every 100 steps between 500 and 15000
// (:22-42) prunes low-opacity (and, after step 3000, oversized) Gaussians
// (:74-111), clones small Gaussians with a high mean gradient and splits
// large ones into two samples of their own distribution (:113-233), each
// time rebuilding every parameter tensor and Adam state with torch.cat /
// index_select on the host's orders; every 3000 steps it clamps the opacity
// logits to logit(0.01) and zeroes their Adam moments (:235-250).
//
// Here the Gaussians live in one flat buffer of six groups (means, log-scales,
// raw quaternions, opacity logits, sh_dc, sh_rest; 3, 3, 4, 1, 3, 45 floats
// per Gaussian, each group padded to 4 floats) with Adam moments in the same
// layout, and a densification step is:
//   gs_densify_accumulate  per view: grad_accum += |(du W/2, dv H/2)|,
//                          count += 1 where both radii are positive;
//   gs_densify_plan        per Gaussian a code: 0 pruned, 1 kept, 2 kept and
//                          cloned, 3 split; plus 0/1 flag arrays whose
//                          exclusive scans (gs_exclusive_scan) give each
//                          survivor's, clone's and split's output slot;
//   gs_densify_apply       one thread per old Gaussian writes its outputs into
//                          the new flat buffers, in the reference's order:
//                          [kept, not split] [clones] [split sample 0]
//                          [split sample 1]; new Adam moments are zero for
//                          clones and split samples, copied for the rest.
//   gs_reset_opacities     clamp of the opacity logits, zeroed moments.
// Split samples: mean + R(q / |q|) (exp(log_scale) * z) for z ~ N(0, I_3),
// log-scale log(exp(log_scale) / 1.6), other parameters repeated
// (strategy.py:178-201). z comes from the caller (noise, 2 x n_split x 3,
// sample-major as the reference's torch.randn((2, n_split, 3))) or, when
// noise is NULL, from a counter-based Philox generator keyed by (seed, split
// index), so every rank of a data-parallel job draws the same samples.
#include <curand_kernel.h>

#include "gs_common.cuh"

namespace gs {

constexpr int kDensifyGroups = 6;
__constant__ int c_group_dims[kDensifyGroups] = {3, 3, 4, 1, 3, 45};

struct FlatLayout {
  int64_t off[kDensifyGroups];  // element offset of each group in the flat buffer
};

__global__ void __launch_bounds__(256) densify_accumulate_kernel(
    int n, const float2 *__restrict__ g_points, const float2 *__restrict__ radii, float half_w,
    float half_h, float *__restrict__ grad_accum, float *__restrict__ count,
    const uint32_t *__restrict__ status) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  // a step whose status word holds an error (e.g. a pair count beyond the
  // layout capacity, after which the step is repeated) adds no statistics
  if (status && ld_volatile_u32(status) != 0u) return;
  const float2 r = radii[i];
  if (!(r.x > 0.0f && r.y > 0.0f)) return;  // strategy.py:68
  const float2 g = g_points[i];
  const float gx = g.x * half_w, gy = g.y * half_h;  // strategy.py:62-63
  grad_accum[i] += sqrtf(gx * gx + gy * gy);
  count[i] += 1.0f;
}

// strategy.py:76-80 (prune) and :118-128 (grow decisions of the survivors).
__global__ void __launch_bounds__(256) densify_plan_kernel(
    int n, const float *__restrict__ params, FlatLayout L, const float *__restrict__ grad_accum,
    const float *__restrict__ count, float prune_opacity, int prune_by_scale, float prune_scale,
    float grow_grad, float split_scale, uint8_t *__restrict__ code, int32_t *__restrict__ keep,
    int32_t *__restrict__ clone, int32_t *__restrict__ split) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  const float opacity = 1.0f / (1.0f + expf(-params[L.off[3] + i]));
  const float *ls = params + L.off[1] + 3 * (int64_t)i;
  const float smax = fmaxf(fmaxf(expf(ls[0]), expf(ls[1])), expf(ls[2]));
  bool prune = opacity < prune_opacity;
  if (prune_by_scale) prune = prune || smax > prune_scale;
  uint8_t c = 0;
  if (!prune) {
    const float g = grad_accum[i] / fmaxf(count[i], 1.0f);
    const bool high = g > grow_grad;
    c = !high ? 1 : (smax < split_scale ? 2 : 3);
  }
  code[i] = c;
  keep[i] = (c == 1 || c == 2) ? 1 : 0;
  clone[i] = (c == 2) ? 1 : 0;
  split[i] = (c == 3) ? 1 : 0;
}

__device__ __forceinline__ void copy_gaussian(const float *__restrict__ src, FlatLayout Ls,
                                              int64_t i, float *__restrict__ dst, FlatLayout Ld,
                                              int64_t j, int first_group) {
  for (int gI = first_group; gI < kDensifyGroups; ++gI) {
    const int d = c_group_dims[gI];
    const float *s = src + Ls.off[gI] + d * i;
    float *t = dst + Ld.off[gI] + d * j;
    for (int k = 0; k < d; ++k) t[k] = s[k];
  }
}

__device__ __forceinline__ void zero_gaussian(float *__restrict__ dst, FlatLayout Ld, int64_t j) {
  for (int gI = 0; gI < kDensifyGroups; ++gI) {
    const int d = c_group_dims[gI];
    float *t = dst + Ld.off[gI] + d * j;
    for (int k = 0; k < d; ++k) t[k] = 0.0f;
  }
}

__global__ void __launch_bounds__(256) densify_apply_kernel(
    int n, const uint8_t *__restrict__ code, const int32_t *__restrict__ pos_keep,
    const int32_t *__restrict__ pos_clone, const int32_t *__restrict__ pos_split, int64_t n_keep,
    int64_t n_clone, int64_t n_split, const float *__restrict__ params, FlatLayout Lo,
    float *__restrict__ out, FlatLayout Ln, const float *__restrict__ m_old,
    const float *__restrict__ v_old, float *__restrict__ m_new, float *__restrict__ v_new,
    const float *__restrict__ noise, unsigned long long seed, float scale_div) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  const uint8_t c = code[i];
  if (c == 1 || c == 2) {
    const int64_t a = pos_keep[i];
    copy_gaussian(params, Lo, i, out, Ln, a, 0);
    if (m_new) copy_gaussian(m_old, Lo, i, m_new, Ln, a, 0);
    if (v_new) copy_gaussian(v_old, Lo, i, v_new, Ln, a, 0);
  }
  if (c == 2) {  // strategy.py:149-176: clone appended, zero moments
    const int64_t b = n_keep + pos_clone[i];
    copy_gaussian(params, Lo, i, out, Ln, b, 0);
    if (m_new) zero_gaussian(m_new, Ln, b);
    if (v_new) zero_gaussian(v_new, Ln, b);
  }
  if (c == 3) {  // strategy.py:178-226
    const int64_t s = pos_split[i];
    const float *q = params + Lo.off[2] + 4 * (int64_t)i;
    // F.normalize (eps 1e-12) and quaternion_to_rotation_matrix (x, y, z, w), gaussian.py:64-79
    const float qn = fmaxf(sqrtf(q[0] * q[0] + q[1] * q[1] + q[2] * q[2] + q[3] * q[3]), 1e-12f);
    const float x = q[0] / qn, y = q[1] / qn, z = q[2] / qn, w = q[3] / qn;
    const float R[3][3] = {{1 - 2 * (y * y + z * z), 2 * (x * y - z * w), 2 * (x * z + y * w)},
                           {2 * (x * y + z * w), 1 - 2 * (x * x + z * z), 2 * (y * z - x * w)},
                           {2 * (x * z - y * w), 2 * (y * z + x * w), 1 - 2 * (x * x + y * y)}};
    const float *ls = params + Lo.off[1] + 3 * (int64_t)i;
    const float sc[3] = {expf(ls[0]), expf(ls[1]), expf(ls[2])};
    const float *mu = params + Lo.off[0] + 3 * (int64_t)i;
    float zz[2][3];
    if (noise) {
      for (int k = 0; k < 2; ++k)
        for (int d = 0; d < 3; ++d) zz[k][d] = noise[((int64_t)k * n_split + s) * 3 + d];
    } else {
      curandStatePhilox4_32_10_t st;
      curand_init(seed, (unsigned long long)s, 0, &st);
      const float4 a = curand_normal4(&st);
      const float4 b = curand_normal4(&st);
      zz[0][0] = a.x; zz[0][1] = a.y; zz[0][2] = a.z;
      zz[1][0] = a.w; zz[1][1] = b.x; zz[1][2] = b.y;
    }
    for (int k = 0; k < 2; ++k) {
      const int64_t j = n_keep + n_clone + (int64_t)k * n_split + s;
      copy_gaussian(params, Lo, i, out, Ln, j, 2);  // quaternions, opacity, SH repeated
      float *mo = out + Ln.off[0] + 3 * j;
      for (int r = 0; r < 3; ++r) {
        const float v0 = sc[0] * zz[k][0], v1 = sc[1] * zz[k][1], v2 = sc[2] * zz[k][2];
        mo[r] = mu[r] + (R[r][0] * v0 + R[r][1] * v1 + R[r][2] * v2);
      }
      float *so = out + Ln.off[1] + 3 * j;
      for (int d = 0; d < 3; ++d) so[d] = logf(sc[d] / scale_div);
      if (m_new) zero_gaussian(m_new, Ln, j);
      if (v_new) zero_gaussian(v_new, Ln, j);
    }
  }
}

// strategy.py:235-250
__global__ void __launch_bounds__(256) reset_opacities_kernel(int n, float *__restrict__ logits,
                                                              float *__restrict__ m,
                                                              float *__restrict__ v,
                                                              float threshold) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  logits[i] = fminf(logits[i], threshold);
  if (m) m[i] = 0.0f;
  if (v) v[i] = 0.0f;
}

static bool read_layout(const int64_t *offsets, int64_t n, FlatLayout *L) {
  if (offsets == nullptr) return false;
  for (int g = 0; g < kDensifyGroups; ++g) {
    if (offsets[g] < 0 || (g > 0 && offsets[g] < offsets[g - 1] + 0)) return false;
    L->off[g] = offsets[g];
  }
  static const int dims[kDensifyGroups] = {3, 3, 4, 1, 3, 45};
  for (int g = 0; g + 1 < kDensifyGroups; ++g)
    if (offsets[g] + dims[g] * n > offsets[g + 1]) return false;  // groups must not overlap
  return true;
}

}  // namespace gs

using namespace gs;

static inline cudaStream_t as_stream(void *s) { return reinterpret_cast<cudaStream_t>(s); }

extern "C" int gs_densify_accumulate(int n, const float *grad_points, const float *radii,
                                     int width, int height, float *grad_accum, float *count,
                                     void *stream) {
  if (n < 0 || width <= 0 || height <= 0 || grad_accum == nullptr || count == nullptr)
    return GS_ERR_INVALID_ARGUMENT;
  if (((uintptr_t)grad_points & 7) || ((uintptr_t)radii & 7)) return GS_ERR_INVALID_ARGUMENT;
  if (n == 0) return GS_OK;
  densify_accumulate_kernel<<<(n + 255) / 256, 256, 0, as_stream(stream)>>>(
      n, reinterpret_cast<const float2 *>(grad_points), reinterpret_cast<const float2 *>(radii),
      (float)(width / 2.0), (float)(height / 2.0), grad_accum, count, device_status_word());
  count_launch();
  return launch_status();
}

extern "C" int gs_densify_plan(int n, const float *params, const int64_t *group_offsets,
                               const float *grad_accum, const float *count, float prune_opacity,
                               int prune_by_scale, float prune_scale, float grow_grad,
                               float split_scale, uint8_t *codes, int32_t *keep_flags,
                               int32_t *clone_flags, int32_t *split_flags, void *stream) {
  FlatLayout L;
  if (n < 0 || params == nullptr || !read_layout(group_offsets, n, &L) || grad_accum == nullptr ||
      count == nullptr || codes == nullptr || keep_flags == nullptr || clone_flags == nullptr ||
      split_flags == nullptr)
    return GS_ERR_INVALID_ARGUMENT;
  if (n == 0) return GS_OK;
  densify_plan_kernel<<<(n + 255) / 256, 256, 0, as_stream(stream)>>>(
      n, params, L, grad_accum, count, prune_opacity, prune_by_scale, prune_scale, grow_grad,
      split_scale, codes, keep_flags, clone_flags, split_flags);
  count_launch();
  return launch_status();
}

extern "C" int gs_densify_apply(int n, const uint8_t *codes, const int32_t *pos_keep,
                                const int32_t *pos_clone, const int32_t *pos_split,
                                int64_t n_keep, int64_t n_clone, int64_t n_split,
                                const float *params, const int64_t *group_offsets,
                                float *new_params, const int64_t *new_group_offsets,
                                const float *exp_avg, const float *exp_avg_sq, float *new_exp_avg,
                                float *new_exp_avg_sq, const float *noise, uint64_t seed,
                                float scale_div, void *stream) {
  FlatLayout Lo, Ln;
  const int64_t n_new = n_keep + n_clone + 2 * n_split;
  if (n < 0 || n_keep < 0 || n_clone < 0 || n_split < 0 || n_keep + n_split > n ||
      n_clone > n_keep || codes == nullptr || pos_keep == nullptr || pos_clone == nullptr ||
      pos_split == nullptr || params == nullptr || new_params == nullptr ||
      !read_layout(group_offsets, n, &Lo) || !read_layout(new_group_offsets, n_new, &Ln) ||
      !(scale_div > 0.0f))
    return GS_ERR_INVALID_ARGUMENT;
  if ((new_exp_avg != nullptr && exp_avg == nullptr) ||
      (new_exp_avg_sq != nullptr && exp_avg_sq == nullptr))
    return GS_ERR_INVALID_ARGUMENT;
  if (n == 0) return GS_OK;
  densify_apply_kernel<<<(n + 255) / 256, 256, 0, as_stream(stream)>>>(
      n, codes, pos_keep, pos_clone, pos_split, n_keep, n_clone, n_split, params, Lo, new_params,
      Ln, exp_avg, exp_avg_sq, new_exp_avg, new_exp_avg_sq, noise, (unsigned long long)seed,
      scale_div);
  count_launch();
  return launch_status();
}

extern "C" int gs_reset_opacities(int n, float *opacity_logits, float *exp_avg,
                                  float *exp_avg_sq, float threshold, void *stream) {
  if (n < 0 || opacity_logits == nullptr) return GS_ERR_INVALID_ARGUMENT;
  if (n == 0) return GS_OK;
  reset_opacities_kernel<<<(n + 255) / 256, 256, 0, as_stream(stream)>>>(
      n, opacity_logits, exp_avg, exp_avg_sq, threshold);
  count_launch();
  return launch_status();
}
