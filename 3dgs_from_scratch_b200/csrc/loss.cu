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

__device__ __forceinline__ float l1_elem(float r, float tv, float inv_n, float &grad) {
  const float c = fminf(fmaxf(r, 0.0f), 1.0f);
  const float rendered = c * 255.0f;
  const float d = rendered / 255.0f - tv / 255.0f;
  const float sgn = (d > 0.0f) ? 1.0f : ((d < 0.0f) ? -1.0f : 0.0f);
  float g = (sgn * inv_n) / 255.0f;
  g = g * 255.0f;
  grad = (r >= 0.0f && r <= 1.0f) ? g : 0.0f;
  return fabsf(d);
}

template <typename TT>
__global__ void __launch_bounds__(256) l1_loss_grad_kernel(int64_t n, const float *__restrict__ raw,
                                                           const TT *__restrict__ target,
                                                           float inv_n, float *__restrict__ grad,
                                                           double *__restrict__ loss_sum) {
  double acc = 0.0;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride) {
    float g;
    acc += (double)l1_elem(raw[i], target_value<TT>(target, i), inv_n, g);
    grad[i] = g;
  }
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
  const int64_t want = (n + 255) / 256;
  const int grid = (int)(want < (int64_t)sms * 8 ? want : (int64_t)sms * 8);
  const float inv_n = (float)(1.0 / (double)n);
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  if (target_is_u8)
    l1_loss_grad_kernel<uint8_t><<<grid, 256, 0, st>>>(
        n, raw_image, reinterpret_cast<const uint8_t *>(target), inv_n, grad_raw, loss_sum);
  else
    l1_loss_grad_kernel<float><<<grid, 256, 0, st>>>(
        n, raw_image, reinterpret_cast<const float *>(target), inv_n, grad_raw, loss_sum);
  count_launch();
  return launch_status();
}
