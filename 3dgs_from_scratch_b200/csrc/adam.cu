// adam.cu -- one-launch Adam over a flat fp32 parameter buffer.
//
// The training loop of the reference (scripts/train.py:17-44,219-221) runs
// six torch.optim.Adam instances, one per parameter group (means, scales,
// quaternions, opacities, sh_dc, sh_rest), each with its own learning rate
// and eps = 1e-15. When the six groups are laid out back to back in one flat
// buffer (as the data-parallel trainer does, so that one all-reduce covers
// every gradient), a single grid-stride kernel updates all of them: per
// element it reads param, grad, exp_avg, exp_avg_sq and writes param,
// exp_avg, exp_avg_sq (28 B), 128-bit vectorised. Arithmetic follows
// torch.optim.Adam's default (non-amsgrad, no weight decay) update:
//   m = b1 m + (1 - b1) g;  v = b2 v + (1 - b2) g^2
//   p -= lr / (1 - b1^t) * m / (sqrt(v) / sqrt(1 - b2^t) + eps)
#include "adam.cuh"

namespace gs {

// Gated on the device status word: when an earlier kernel of the step
// recorded an error (a bounded wait that gave up, a capacity overflow), the
// gradient may be incomplete, so the update is skipped and the parameters and
// moments stay as they were; the host reads the status with gs_check_status.
__global__ void __launch_bounds__(256) adam_kernel(float4 *__restrict__ p, const float4 *__restrict__ g,
                                                   float4 *__restrict__ m, float4 *__restrict__ v,
                                                   int64_t n4, AdamGroups G, float b1, float b2,
                                                   const uint32_t *status) {
  if (ld_volatile_u32(status) != 0u) return;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n4; i += stride) {
    float4 pp = p[i], gg = g[i], mm = m[i], vv = v[i];
    adam_float4(G, 4 * i, pp, gg, mm, vv, b1, b2);
    p[i] = pp;
    m[i] = mm;
    v[i] = vv;
  }
}

// The same update with the group table (and its folded bias corrections)
// read from device memory, so that a captured launch (CUDA graph) applies
// the step whose table the host uploaded before the replay.
__global__ void __launch_bounds__(256) adam_table_kernel(float4 *__restrict__ p,
                                                         const float4 *__restrict__ g,
                                                         float4 *__restrict__ m,
                                                         float4 *__restrict__ v, int64_t n4,
                                                         const AdamGroups *__restrict__ Gd,
                                                         float b1, float b2,
                                                         const uint32_t *status) {
  if (ld_volatile_u32(status) != 0u) return;
  const AdamGroups G = *Gd;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n4; i += stride) {
    float4 pp = p[i], gg = g[i], mm = m[i], vv = v[i];
    adam_float4(G, 4 * i, pp, gg, mm, vv, b1, b2);
    p[i] = pp;
    m[i] = mm;
    v[i] = vv;
  }
}

// Adam over up to kAdamMaxGroups disjoint element ranges of the flat buffer,
// range r belonging to group r of the device table (the step's bias
// corrections): a slice of every group -- e.g. the parameters of a range of
// Gaussians, each group holding them contiguously -- updated as soon as its
// gradient is complete.
struct AdamRanges {
  int64_t start4[kAdamMaxGroups];   // first float4 of each range
  int64_t prefix4[kAdamMaxGroups + 1];
  int count;
};

__global__ void __launch_bounds__(256) adam_ranges_kernel(float4 *__restrict__ p,
                                                          const float4 *__restrict__ g,
                                                          float4 *__restrict__ m,
                                                          float4 *__restrict__ v, AdamRanges R,
                                                          const AdamGroups *__restrict__ Gd,
                                                          float b1, float b2,
                                                          const uint32_t *status) {
  if (ld_volatile_u32(status) != 0u) return;
  const int64_t total = R.prefix4[R.count];
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t k = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; k < total; k += stride) {
    int r = 0;
#pragma unroll
    for (int q = 1; q < kAdamMaxGroups; ++q) r += (q < R.count && k >= R.prefix4[q]) ? 1 : 0;
    const int64_t i = R.start4[r] + (k - R.prefix4[r]);
    float4 pp = p[i], gg = g[i], mm = m[i], vv = v[i];
    const float st = Gd->step_size[r], ib = Gd->inv_bc2_sqrt[r], ep = Gd->eps[r];
    adam_one(pp.x, gg.x, mm.x, vv.x, b1, b2, st, ib, ep);
    adam_one(pp.y, gg.y, mm.y, vv.y, b1, b2, st, ib, ep);
    adam_one(pp.z, gg.z, mm.z, vv.z, b1, b2, st, ib, ep);
    adam_one(pp.w, gg.w, mm.w, vv.w, b1, b2, st, ib, ep);
    p[i] = pp;
    m[i] = mm;
    v[i] = vv;
  }
}

int build_adam_groups(int64_t n, int num_groups, const int64_t *group_ends, const float *lrs,
                      const float *eps, float beta1, float beta2, int64_t step, AdamGroups *G) {
  if (num_groups < 1 || num_groups > kAdamMaxGroups || step < 1 || group_ends == nullptr ||
      lrs == nullptr || eps == nullptr)
    return GS_ERR_INVALID_ARGUMENT;
  G->count = num_groups;
  const double bc1 = 1.0 - pow((double)beta1, (double)step);
  const double bc2 = 1.0 - pow((double)beta2, (double)step);
  int64_t prev = 0;
  for (int k = 0; k < kAdamMaxGroups; ++k) {
    if (k < num_groups) {
      if (group_ends[k] < prev || (group_ends[k] & 3)) return GS_ERR_INVALID_ARGUMENT;
      prev = group_ends[k];
      G->end[k] = group_ends[k];
      G->step_size[k] = (float)((double)lrs[k] / bc1);
      G->inv_bc2_sqrt[k] = (float)(1.0 / sqrt(bc2));
      G->eps[k] = eps[k];
    } else {
      G->end[k] = n;
      G->step_size[k] = 0.f;
      G->inv_bc2_sqrt[k] = 1.f;
      G->eps[k] = 1.f;
    }
  }
  return prev == n ? GS_OK : GS_ERR_INVALID_ARGUMENT;
}

}  // namespace gs

using namespace gs;

extern "C" int gs_adam_step(int64_t n, float *params, const float *grads, float *exp_avg,
                            float *exp_avg_sq, int num_groups, const int64_t *group_ends,
                            const float *lrs, const float *eps, float beta1, float beta2,
                            int64_t step, void *stream) {
  if (n < 0 || num_groups < 1 || num_groups > kAdamMaxGroups || step < 1 || (n & 3))
    return GS_ERR_INVALID_ARGUMENT;
  if ((((uintptr_t)params | (uintptr_t)grads | (uintptr_t)exp_avg | (uintptr_t)exp_avg_sq) & 15))
    return GS_ERR_INVALID_ARGUMENT;
  if (n == 0) return GS_OK;
  AdamGroups G;
  const int rc = build_adam_groups(n, num_groups, group_ends, lrs, eps, beta1, beta2, step, &G);
  if (rc) return rc;
  const int64_t n4 = n / 4;
  int dev = 0;
  cudaGetDevice(&dev);
  int sms = 148;
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const int64_t want = (n4 + 255) / 256;
  const int grid = (int)(want < (int64_t)sms * 8 ? want : (int64_t)sms * 8);
  uint32_t *status = device_status_word();
  if (status == nullptr) return GS_ERR_CUDA;
  adam_kernel<<<grid, 256, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
      reinterpret_cast<float4 *>(params), reinterpret_cast<const float4 *>(grads),
      reinterpret_cast<float4 *>(exp_avg), reinterpret_cast<float4 *>(exp_avg_sq), n4, G, beta1,
      beta2, status);
  count_launch();
  return launch_status();
}

extern "C" size_t gs_adam_table_bytes(void) { return sizeof(AdamGroups); }

extern "C" int gs_adam_table(int64_t n, int num_groups, const int64_t *group_ends,
                             const float *lrs, const float *eps, float beta1, float beta2,
                             int64_t step, void *table_host, size_t table_bytes) {
  if (table_host == nullptr || table_bytes < sizeof(AdamGroups) || n < 0 || (n & 3))
    return GS_ERR_INVALID_ARGUMENT;
  return build_adam_groups(n, num_groups, group_ends, lrs, eps, beta1, beta2, step,
                           reinterpret_cast<AdamGroups *>(table_host));
}

static int adam_grid(int64_t n4) {
  int dev = 0;
  cudaGetDevice(&dev);
  int sms = 148;
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const int64_t want = (n4 + 255) / 256;
  return (int)(want < (int64_t)sms * 8 ? want : (int64_t)sms * 8);
}

extern "C" int gs_adam_step_table(int64_t n, float *params, const float *grads, float *exp_avg,
                                  float *exp_avg_sq, const void *table_dev, float beta1,
                                  float beta2, void *stream) {
  if (n < 0 || (n & 3) || table_dev == nullptr || ((uintptr_t)table_dev & 7))
    return GS_ERR_INVALID_ARGUMENT;
  if ((((uintptr_t)params | (uintptr_t)grads | (uintptr_t)exp_avg | (uintptr_t)exp_avg_sq) & 15))
    return GS_ERR_INVALID_ARGUMENT;
  if (n == 0) return GS_OK;
  uint32_t *status = device_status_word();
  if (status == nullptr) return GS_ERR_CUDA;
  const int64_t n4 = n / 4;
  adam_table_kernel<<<adam_grid(n4), 256, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
      reinterpret_cast<float4 *>(params), reinterpret_cast<const float4 *>(grads),
      reinterpret_cast<float4 *>(exp_avg), reinterpret_cast<float4 *>(exp_avg_sq), n4,
      reinterpret_cast<const AdamGroups *>(table_dev), beta1, beta2, status);
  count_launch();
  return launch_status();
}

extern "C" int gs_adam_step_ranges(float *params, const float *grads, float *exp_avg,
                                   float *exp_avg_sq, int num_ranges, const int64_t *starts,
                                   const int64_t *counts, const void *table_dev, float beta1,
                                   float beta2, void *stream) {
  if (num_ranges < 1 || num_ranges > kAdamMaxGroups || starts == nullptr || counts == nullptr ||
      table_dev == nullptr || ((uintptr_t)table_dev & 7))
    return GS_ERR_INVALID_ARGUMENT;
  if ((((uintptr_t)params | (uintptr_t)grads | (uintptr_t)exp_avg | (uintptr_t)exp_avg_sq) & 15))
    return GS_ERR_INVALID_ARGUMENT;
  AdamRanges R{};
  R.count = num_ranges;
  R.prefix4[0] = 0;
  for (int r = 0; r < num_ranges; ++r) {
    if (starts[r] < 0 || counts[r] < 0 || (starts[r] & 3) || (counts[r] & 3))
      return GS_ERR_INVALID_ARGUMENT;
    R.start4[r] = starts[r] / 4;
    R.prefix4[r + 1] = R.prefix4[r] + counts[r] / 4;
  }
  for (int r = num_ranges; r < kAdamMaxGroups; ++r) {
    R.start4[r] = 0;
    R.prefix4[r + 1] = R.prefix4[num_ranges];
  }
  if (R.prefix4[num_ranges] == 0) return GS_OK;
  uint32_t *status = device_status_word();
  if (status == nullptr) return GS_ERR_CUDA;
  adam_ranges_kernel<<<adam_grid(R.prefix4[num_ranges]), 256, 0,
                       reinterpret_cast<cudaStream_t>(stream)>>>(
      reinterpret_cast<float4 *>(params), reinterpret_cast<const float4 *>(grads),
      reinterpret_cast<float4 *>(exp_avg), reinterpret_cast<float4 *>(exp_avg_sq), R,
      reinterpret_cast<const AdamGroups *>(table_dev), beta1, beta2, status);
  count_launch();
  return launch_status();
}
