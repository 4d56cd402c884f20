// loss.cu -- the reference's per-view training loss and its gradient in one pass.
//
// The reference renders rendered = clamp(raw, 0, 1) * 255 (src/cuda/wrapper.py:294)
// and trains on l1 = mean(|rendered / 255 - target / 255|) (scripts/train.py:
// 187-191). This kernel reads the raw blended image and the target once,
// adds sum |.| into a double accumulator, and writes d l1 / d raw with Torch's
// chain (sign(d) / numel, then the / 255 and * 255 of the division and the
// scaling, then the clamp's pass-through mask 0 <= raw <= 1).
#include "gs_common.cuh"

namespace gs {

template <typename TT>
__device__ __forceinline__ float target_value(const TT *t, int64_t i);
template <>
__device__ __forceinline__ float target_value<float>(const float *t, int64_t i) {
  return t[i];
}
template <>
__device__ __forceinline__ float target_value<uint8_t>(const uint8_t *t, int64_t i) {
  return (float)t[i];
}

// The / 255 of the normalisation is a product with the rounded reciprocal,
// within an ulp of the reference's quotient: equal values still give d == 0,
// and only a difference within that rounding of zero can get another sign,
// which moves that element's gradient by 1 / n.
constexpr float kInv255 = 1.0f / 255.0f;

__device__ __forceinline__ float l1_elem(float r, float tv, float inv_n, float &grad) {
  const float c = fminf(fmaxf(r, 0.0f), 1.0f);
  const float rendered = c * 255.0f;
  const float d = rendered * kInv255 - tv * kInv255;
  const float sgn = (d > 0.0f) ? 1.0f : ((d < 0.0f) ? -1.0f : 0.0f);
  float g = (sgn * inv_n) * kInv255;
  g = g * 255.0f;
  grad = (r >= 0.0f && r <= 1.0f) ? g : 0.0f;
  return fabsf(d);
}

__device__ __forceinline__ float4 load4(const float *t, int64_t i) {
  return *reinterpret_cast<const float4 *>(t + i);
}
__device__ __forceinline__ float4 load4(const uint8_t *t, int64_t i) {
  const uchar4 u = *reinterpret_cast<const uchar4 *>(t + i);
  return make_float4((float)u.x, (float)u.y, (float)u.z, (float)u.w);
}

// Four elements per thread and step (128-bit raw and gradient accesses) when
// n % 4 == 0 and the pointers are aligned; per-thread partial sums in fp32,
// block sums in double.
template <typename TT, bool VEC>
__global__ void __launch_bounds__(256) l1_loss_grad_kernel(int64_t n, const float *__restrict__ raw,
                                                           const TT *__restrict__ target,
                                                           float inv_n, float *__restrict__ grad,
                                                           double *__restrict__ loss_sum) {
  float part = 0.0f;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  if (VEC) {
    for (int64_t q = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; 4 * q < n; q += stride) {
      const float4 r = load4(raw, 4 * q);
      const float4 tv = load4(target, 4 * q);
      float4 g;
      part += l1_elem(r.x, tv.x, inv_n, g.x);
      part += l1_elem(r.y, tv.y, inv_n, g.y);
      part += l1_elem(r.z, tv.z, inv_n, g.z);
      part += l1_elem(r.w, tv.w, inv_n, g.w);
      *reinterpret_cast<float4 *>(grad + 4 * q) = g;
    }
  } else {
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride) {
      float g;
      part += l1_elem(raw[i], target_value<TT>(target, i), inv_n, g);
      grad[i] = g;
    }
  }
  double acc = (double)part;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
  __shared__ double s_acc[8];
  if ((threadIdx.x & 31) == 0) s_acc[threadIdx.x >> 5] = acc;
  __syncthreads();
  if (threadIdx.x == 0) {
    double b = 0.0;
    for (int w = 0; w < (int)(blockDim.x >> 5); ++w) b += s_acc[w];
    atomicAdd(loss_sum, b);
  }
}

}  // namespace gs

using namespace gs;

extern "C" int gs_l1_loss_grad(int64_t n, const float *raw_image, const void *target,
                               int target_is_u8, float *grad_raw, double *loss_sum, void *stream) {
  if (n < 0 || raw_image == nullptr || target == nullptr || grad_raw == nullptr ||
      loss_sum == nullptr)
    return GS_ERR_INVALID_ARGUMENT;
  if (n == 0) return GS_OK;
  int dev = 0;
  cudaGetDevice(&dev);
  int sms = 148;
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const int tb = target_is_u8 ? 4 : 16;  // target alignment for 4-element loads
  const bool vec = (n % 4 == 0) && !(((uintptr_t)raw_image | (uintptr_t)grad_raw) & 15) &&
                   !((uintptr_t)target & (tb - 1));
  const int64_t want = ((vec ? n / 4 : n) + 255) / 256;
  const int grid = (int)(want < (int64_t)sms * 8 ? want : (int64_t)sms * 8);
  const float inv_n = (float)(1.0 / (double)n);
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  const uint8_t *t8 = reinterpret_cast<const uint8_t *>(target);
  const float *tf = reinterpret_cast<const float *>(target);
  if (target_is_u8 && vec)
    l1_loss_grad_kernel<uint8_t, true><<<grid, 256, 0, st>>>(n, raw_image, t8, inv_n, grad_raw,
                                                             loss_sum);
  else if (target_is_u8)
    l1_loss_grad_kernel<uint8_t, false><<<grid, 256, 0, st>>>(n, raw_image, t8, inv_n, grad_raw,
                                                              loss_sum);
  else if (vec)
    l1_loss_grad_kernel<float, true><<<grid, 256, 0, st>>>(n, raw_image, tf, inv_n, grad_raw,
                                                           loss_sum);
  else
    l1_loss_grad_kernel<float, false><<<grid, 256, 0, st>>>(n, raw_image, tf, inv_n, grad_raw,
                                                            loss_sum);
  count_launch();
  return launch_status();
}
