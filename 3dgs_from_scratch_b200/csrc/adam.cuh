// adam.cuh -- the Adam update shared by the one-GPU optimizer (adam.cu) and
// the data-parallel optimizer step (dp_step.cu).
//
// The training loop of the reference (scripts/train.py:17-44,219-221) runs
// six torch.optim.Adam instances, one per parameter group (means, scales,
// quaternions, opacities, sh_dc, sh_rest), each with its own learning rate
// and eps = 1e-15. Laid out back to back in one flat buffer, one kernel
// updates all of them with torch.optim.Adam's default (non-amsgrad, no
// weight decay) arithmetic:
//   m = b1 m + (1 - b1) g;  v = b2 v + (1 - b2) g^2
//   p -= lr / (1 - b1^t) * m / (sqrt(v) / sqrt(1 - b2^t) + eps)
#pragma once
#include "gs_common.cuh"

namespace gs {

constexpr int kAdamMaxGroups = 8;

struct AdamGroups {
  int64_t end[kAdamMaxGroups];         // exclusive end (in elements) of each group, multiples of 4
  float step_size[kAdamMaxGroups];     // lr / (1 - b1^t)
  float inv_bc2_sqrt[kAdamMaxGroups];  // 1 / sqrt(1 - b2^t)
  float eps[kAdamMaxGroups];
  int count;
};

// Every rounding step is explicit (no contraction left to the compiler), so
// the one-GPU and the data-parallel kernels produce bit-identical updates.
__device__ __forceinline__ float adam_one(float &p, float g, float &m, float &v, float b1,
                                          float b2, float step, float ibc2, float eps) {
  m = __fmaf_rn(b1, m, __fmul_rn(1.0f - b1, g));
  v = __fmaf_rn(b2, v, __fmul_rn(__fmul_rn(1.0f - b2, g), g));
  const float denom = __fmaf_rn(__fsqrt_rn(v), ibc2, eps);
  p = __fmaf_rn(-step, __fdiv_rn(m, denom), p);
  return p;
}

// Group of flat element e (groups are contiguous and in order).
__device__ __forceinline__ int adam_group_of(const AdamGroups &G, int64_t e) {
  int grp = 0;
#pragma unroll
  for (int k = 0; k < kAdamMaxGroups - 1; ++k) grp += (k < G.count - 1 && e >= G.end[k]) ? 1 : 0;
  return grp;
}

__device__ __forceinline__ void adam_float4(const AdamGroups &G, int64_t e, float4 &p,
                                            const float4 &g, float4 &m, float4 &v, float b1,
                                            float b2) {
  const int grp = adam_group_of(G, e);
  const float st = G.step_size[grp], ib = G.inv_bc2_sqrt[grp], ep = G.eps[grp];
  adam_one(p.x, g.x, m.x, v.x, b1, b2, st, ib, ep);
  adam_one(p.y, g.y, m.y, v.y, b1, b2, st, ib, ep);
  adam_one(p.z, g.z, m.z, v.z, b1, b2, st, ib, ep);
  adam_one(p.w, g.w, m.w, v.w, b1, b2, st, ib, ep);
}

// Host: validate the group table and fold the bias corrections of step
// `step` into it. Returns GS_OK or GS_ERR_INVALID_ARGUMENT.
int build_adam_groups(int64_t n, int num_groups, const int64_t *group_ends, const float *lrs,
                      const float *eps, float beta1, float beta2, int64_t step, AdamGroups *G);

}  // namespace gs
