// ssim.cu -- SSIM (11x11 Gaussian window, sigma 1.5) with its gradient, and the
// reference's training loss (1 - lambda) * L1 + lambda * (1 - SSIM) fused with
// the clamp * 255 / 255 of the rendered image (scripts/train.py:183-203).
//
// The reference takes SSIM from the external package fused_ssim (pinned as
// fused-ssim==0.0.0 in environment.yml:56, not vendored), called at
// scripts/train.py:193-197 and scripts/evaluate.py:57-61. What is restated
// here is the published definition of Wang et al. (2004) that package
// implements: per channel, Gaussian-weighted local statistics
//   mu_x = G*x, mu_y = G*y, s_xx = G*(x^2) - mu_x^2, s_yy = ..., s_xy = G*(xy) - mu_x mu_y
// (G the normalised 11-tap Gaussian, sigma 1.5, outer product; zero padding),
// S = (2 mu_x mu_y + C1)(2 s_xy + C2) / ((mu_x^2 + mu_y^2 + C1)(s_xx + s_yy + C2)),
// C1 = 0.01^2, C2 = 0.03^2, and the loss value is the mean of S over every
// channel and pixel ("same") or over the pixels at least 5 from every border
// ("valid", the reference's choice).
//
// Two kernels, both tiled 32 x 32 output pixels per block with the 5-pixel
// halo staged in shared memory and the window applied separably, register
// blocked (a thread produces 8 consecutive outputs of a row, then 4 of a
// column, from a sliding window of loaded values, instead of one shared-memory
// load per multiply-add):
//   ssim_fwd_kernel  local statistics -> S (summed into a double) and the
//                    three partial derivatives of S at each pixel,
//                    dS/dmu_x, dS/dE[x^2], dS/dE[xy], already multiplied by
//                    the loss weight of that pixel (zero where not counted);
//   ssim_bwd_kernel  the same window applied to those three maps gives
//                    dL/dx(p) = G*m0 + 2 x(p) G*m1 + y(p) G*m2;
//                    in the fused-loss form it adds the L1 term, sums |d|,
//                    and chains through clamp * 255 / 255 to the raw image.
// Inputs are either planar (N, C, H, W) fp32 (the fused_ssim interface) or
// the rasterizer's (H, W, 3) raw image with an (H, W, 3) uint8 or fp32 target
// in [0, 255] (the training loss).
#include "gs_common.cuh"

namespace gs {

constexpr int kSsimTW = 32;                    // output tile width
constexpr int kSsimTH = 32;                    // output tile height
constexpr int kSsimR = 5;                      // window radius
constexpr int kSsimWin = 2 * kSsimR + 1;
constexpr int kSsimHW = kSsimTW + 2 * kSsimR;  // 42 staged columns
constexpr int kSsimHH = kSsimTH + 2 * kSsimR;  // 42 staged rows
constexpr int kSsimStride = kSsimHW + 1;       // 43: conflict-free row starts
constexpr int kSsimHRow = kSsimTW + 1;         // 33: conflict-free horizontal-pass stores
constexpr int kSsimRunH = 8;                   // outputs per thread, horizontal pass
constexpr int kSsimRunV = 4;                   // outputs per thread, vertical pass
constexpr int kSsimStageRows = 6;              // staged rows per step (6 x 42 threads)
constexpr int kSsimStageThreads = kSsimStageRows * kSsimHW;
constexpr int kSsimStageSteps = kSsimHH / kSsimStageRows;  // 7 staged rows per thread
static_assert(kSsimHH % kSsimStageRows == 0, "every staging thread takes kSsimStageSteps rows");
constexpr int kSsimThreads = 256;
constexpr float kSsimC1 = 0.01f * 0.01f;
constexpr float kSsimC2 = 0.03f * 0.03f;

__constant__ float c_ssim_win[kSsimWin];

// Where the two images of one plane come from.
//   HWC = false: planar fp32, plane p = n * C + c at offset p * H * W.
//   HWC = true : raw rendered (H, W, C) fp32 -> clamp(r, 0, 1) * 255 / 255,
//                target (H, W, C) of type TT -> t / 255; plane = channel.
// Index arithmetic is 32-bit: the host entry points reject images of 2^31
// or more elements. The / 255 of the reference's normalisation is a product
// with the rounded reciprocal (within an ulp of the division; the loss and
// its gradient do not need the quotient bit for bit).
constexpr float kInv255 = 1.0f / 255.0f;

template <bool HWC, typename TT>
struct SsimSrc {
  const float *a;
  const TT *b;
  int C, H, W;

  __device__ __forceinline__ int index(int plane, int y, int x) const {
    if (HWC) return (y * W + x) * C + plane;
    return (plane * H + y) * W + x;
  }
  __device__ __forceinline__ void load(int plane, int y, int x, float &xv, float &yv) const {
    const int i = index(plane, y, x);
    if (HWC) {
      const float c = fminf(fmaxf(a[i], 0.0f), 1.0f);
      xv = (c * 255.0f) * kInv255;
      yv = (float)b[i] * kInv255;
    } else {
      xv = a[i];
      yv = (float)b[i];
    }
  }
};

__device__ __forceinline__ double block_sum_double(double v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  __shared__ double s_part[kSsimThreads / 32];
  if ((threadIdx.x & 31) == 0) s_part[threadIdx.x >> 5] = v;
  __syncthreads();
  double t = 0.0;
  if (threadIdx.x == 0)
    for (int w = 0; w < kSsimThreads / 32; ++w) t += s_part[w];
  return t;  // valid in thread 0
}

// Grid: x = tiles_x * planes (plane fastest, so the blocks of the three
// channels of one tile run together and share the tile's cache lines),
// y = tiles_y.
// Horizontal pass of NQ quantities over one staged row: thread item = (row,
// group of kSsimRunH columns). val(k, q) gives quantity q at staged column
// c0 + k; the kSsimRunH window sums go to out[q][row][c0 + o].
template <int NQ, typename Val>
__device__ __forceinline__ void hpass_run(Val val, float (*out)[kSsimHH][kSsimHRow], int row,
                                          int c0) {
  float acc[kSsimRunH][NQ];
#pragma unroll
  for (int o = 0; o < kSsimRunH; ++o)
#pragma unroll
    for (int q = 0; q < NQ; ++q) acc[o][q] = 0.f;
#pragma unroll
  for (int k = 0; k < kSsimRunH + kSsimWin - 1; ++k) {
    float v[NQ];
    val(k, v);
#pragma unroll
    for (int o = 0; o < kSsimRunH; ++o) {
      const int t = k - o;
      if (t >= 0 && t < kSsimWin) {
#pragma unroll
        for (int q = 0; q < NQ; ++q) acc[o][q] = fmaf(c_ssim_win[t], v[q], acc[o][q]);
      }
    }
  }
#pragma unroll
  for (int o = 0; o < kSsimRunH; ++o)
#pragma unroll
    for (int q = 0; q < NQ; ++q) out[q][row][c0 + o] = acc[o][q];
}

// Vertical pass: kSsimRunV consecutive output rows r0.. of column c.
template <int NQ>
__device__ __forceinline__ void vpass_run(const float (*hs)[kSsimHH][kSsimHRow], int r0, int c,
                                          float (&acc)[kSsimRunV][NQ]) {
#pragma unroll
  for (int o = 0; o < kSsimRunV; ++o)
#pragma unroll
    for (int q = 0; q < NQ; ++q) acc[o][q] = 0.f;
#pragma unroll
  for (int k = 0; k < kSsimRunV + kSsimWin - 1; ++k) {
    float v[NQ];
#pragma unroll
    for (int q = 0; q < NQ; ++q) v[q] = hs[q][r0 + k][c];
#pragma unroll
    for (int o = 0; o < kSsimRunV; ++o) {
      const int t = k - o;
      if (t >= 0 && t < kSsimWin) {
#pragma unroll
        for (int q = 0; q < NQ; ++q) acc[o][q] = fmaf(c_ssim_win[t], v[q], acc[o][q]);
      }
    }
  }
}

constexpr int kSsimHItems = kSsimHH * (kSsimTW / kSsimRunH);  // 168
constexpr int kSsimVItems = kSsimTW * (kSsimTH / kSsimRunV);  // 256
static_assert(kSsimVItems == kSsimThreads, "one vertical run per thread");

// Grid: x = tiles_x * planes (plane fastest, so the blocks of the three
// channels of one tile run together and share the tile's cache lines),
// y = tiles_y.
template <bool HWC, typename TT>
__global__ void __launch_bounds__(kSsimThreads) ssim_fwd_kernel(SsimSrc<HWC, TT> src, int planes,
                                                                int valid, float wscale,
                                                                float *__restrict__ m0,
                                                                float *__restrict__ m1,
                                                                float *__restrict__ m2,
                                                                double *__restrict__ ssim_sum) {
  __shared__ float sx[kSsimHH * kSsimStride];
  __shared__ float sy[kSsimHH * kSsimStride];
  __shared__ float hs[5][kSsimHH][kSsimHRow];
  const int H = src.H, W = src.W;
  const int plane = blockIdx.x % planes;
  const int tx = blockIdx.x / planes;
  const int gx0 = tx * kSsimTW, gy0 = blockIdx.y * kSsimTH;
  if (threadIdx.x < kSsimStageThreads) {  // 6 rows of 42 columns per step
    const int c = threadIdx.x % kSsimHW, r0 = threadIdx.x / kSsimHW;
    const int gx = gx0 - kSsimR + c;
    const bool in_x = gx >= 0 && gx < W;
    // every load of the thread's 7 rows first, then the stores (one round
    // trip to memory instead of seven)
    float xv[kSsimStageSteps], yv[kSsimStageSteps];
#pragma unroll
    for (int i = 0; i < kSsimStageSteps; ++i) {
      const int gy = gy0 - kSsimR + r0 + i * kSsimStageRows;
      xv[i] = 0.0f;
      yv[i] = 0.0f;
      if (in_x && gy >= 0 && gy < H) src.load(plane, gy, gx, xv[i], yv[i]);
    }
#pragma unroll
    for (int i = 0; i < kSsimStageSteps; ++i) {
      const int r = r0 + i * kSsimStageRows;
      sx[r * kSsimStride + c] = xv[i];
      sy[r * kSsimStride + c] = yv[i];
    }
  }
  __syncthreads();
  if (threadIdx.x < kSsimHItems) {
    const int row = threadIdx.x >> 2, c0 = (threadIdx.x & 3) * kSsimRunH;
    const float *px = sx + row * kSsimStride + c0;
    const float *py = sy + row * kSsimStride + c0;
    hpass_run<5>(
        [&](int k, float *v) {
          const float x = px[k], y = py[k];
          v[0] = x;
          v[1] = y;
          v[2] = x * x;
          v[3] = y * y;
          v[4] = x * y;
        },
        hs, row, c0);
  }
  __syncthreads();
  const int c = threadIdx.x & 31, r0 = (threadIdx.x >> 5) * kSsimRunV;
  float st[kSsimRunV][5];
  vpass_run<5>(hs, r0, c, st);
  double acc = 0.0;
  const int gx = gx0 + c;
#pragma unroll
  for (int o = 0; o < kSsimRunV; ++o) {
    const int gy = gy0 + r0 + o;
    if (gy >= H || gx >= W) continue;
    const float mx = st[o][0], my = st[o][1], exx = st[o][2], eyy = st[o][3], exy = st[o][4];
    const bool counted =
        !valid || (gy >= kSsimR && gy < H - kSsimR && gx >= kSsimR && gx < W - kSsimR);
    float d_mu = 0.f, d_xx = 0.f, d_xy = 0.f;
    if (counted) {
      const float sxx = exx - mx * mx, syy = eyy - my * my, sxy = exy - mx * my;
      const float a1 = 2.f * mx * my + kSsimC1, a2 = 2.f * sxy + kSsimC2;
      const float b1 = mx * mx + my * my + kSsimC1, b2 = sxx + syy + kSsimC2;
      const float inv_b = 1.0f / (b1 * b2);
      const float s = a1 * a2 * inv_b;
      acc += (double)s;
      d_xy = 2.f * a1 * inv_b;  // dS/dE[xy]
      d_xx = -s / b2;           // dS/dE[x^2]
      d_mu = 2.f * my * a2 * inv_b - 2.f * mx * s / b1 - 2.f * mx * d_xx - my * d_xy;
      d_mu *= wscale;
      d_xx *= wscale;
      d_xy *= wscale;
    }
    const int oi = (plane * H + gy) * W + gx;
    m0[oi] = d_mu;
    m1[oi] = d_xx;
    m2[oi] = d_xy;
  }
  const double t = block_sum_double(acc);
  if (threadIdx.x == 0 && t != 0.0) atomicAdd(ssim_sum, t);
}

// FUSED = true: the training loss form (HWC only): grad_raw = chain of
// l1_weight * sign(x - y) / numel + (G*m0 + 2x G*m1 + y G*m2) through the
// / 255, * 255 and the clamp mask, and sum |x - y| into l1_sum.
// FUSED = false: grad (planar) = upstream * (G*m0 + 2x G*m1 + y G*m2).
template <bool HWC, typename TT, bool FUSED>
__global__ void __launch_bounds__(kSsimThreads) ssim_bwd_kernel(
    SsimSrc<HWC, TT> src, int planes, const float *__restrict__ m0, const float *__restrict__ m1,
    const float *__restrict__ m2, const float *__restrict__ upstream, float l1_weight,
    float inv_numel, float *__restrict__ grad, double *__restrict__ l1_sum) {
  __shared__ float sm[3][kSsimHH * kSsimStride];
  __shared__ float hs[3][kSsimHH][kSsimHRow];
  const int H = src.H, W = src.W;
  const int plane = blockIdx.x % planes;
  const int tx = blockIdx.x / planes;
  const int gx0 = tx * kSsimTW, gy0 = blockIdx.y * kSsimTH;
  const int pbase = plane * H * W;
  if (threadIdx.x < kSsimStageThreads) {  // 6 rows of 42 columns per step
    const int c = threadIdx.x % kSsimHW, r0 = threadIdx.x / kSsimHW;
    const int gx = gx0 - kSsimR + c;
    const bool in_x = gx >= 0 && gx < W;
    // every load of the thread's 7 rows first, then the stores
    float v0[kSsimStageSteps], v1[kSsimStageSteps], v2[kSsimStageSteps];
#pragma unroll
    for (int i = 0; i < kSsimStageSteps; ++i) {
      const int gy = gy0 - kSsimR + r0 + i * kSsimStageRows;
      v0[i] = v1[i] = v2[i] = 0.f;
      if (in_x && gy >= 0 && gy < H) {
        const int o = pbase + gy * W + gx;
        v0[i] = m0[o];
        v1[i] = m1[o];
        v2[i] = m2[o];
      }
    }
#pragma unroll
    for (int i = 0; i < kSsimStageSteps; ++i) {
      const int r = r0 + i * kSsimStageRows;
      sm[0][r * kSsimStride + c] = v0[i];
      sm[1][r * kSsimStride + c] = v1[i];
      sm[2][r * kSsimStride + c] = v2[i];
    }
  }
  __syncthreads();
  if (threadIdx.x < kSsimHItems) {
    const int row = threadIdx.x >> 2, c0 = (threadIdx.x & 3) * kSsimRunH;
    const int base = row * kSsimStride + c0;
    hpass_run<3>(
        [&](int k, float *v) {
          v[0] = sm[0][base + k];
          v[1] = sm[1][base + k];
          v[2] = sm[2][base + k];
        },
        hs, row, c0);
  }
  __syncthreads();
  const int c = threadIdx.x & 31, r0 = (threadIdx.x >> 5) * kSsimRunV;
  float cv[kSsimRunV][3];
  vpass_run<3>(hs, r0, c, cv);
  const float up = upstream ? *upstream : 1.0f;
  double acc = 0.0;
  const int gx = gx0 + c;
#pragma unroll
  for (int o = 0; o < kSsimRunV; ++o) {
    const int gy = gy0 + r0 + o;
    if (gy >= H || gx >= W) continue;
    float xv, yv;
    src.load(plane, gy, gx, xv, yv);
    const float gs = cv[o][0] + 2.f * xv * cv[o][1] + yv * cv[o][2];
    if (FUSED) {
      const int i = src.index(plane, gy, gx);
      const float d = xv - yv;
      acc += (double)fabsf(d);
      const float sgn = (d > 0.0f) ? 1.0f : ((d < 0.0f) ? -1.0f : 0.0f);
      const float gn = l1_weight * sgn * inv_numel + gs;  // d loss / d rendered_norm
      float g = gn * kInv255;                            // rendered_norm = rendered / 255
      g = g * 255.0f;                                    // rendered = clamp(raw) * 255
      const float raw = src.a[i];
      grad[i] = (raw >= 0.0f && raw <= 1.0f) ? g : 0.0f;
    } else {
      grad[pbase + gy * W + gx] = up * gs;
    }
  }
  if (FUSED) {
    const double t = block_sum_double(acc);
    if (threadIdx.x == 0 && t != 0.0) atomicAdd(l1_sum, t);
  }
}

// The normalised window exp(-(i - 5)^2 / (2 * 1.5^2)) / sum, computed in
// double and rounded to fp32, uploaded once per host thread and context (a
// synchronous copy: the first call on a thread must not be inside a stream
// capture).
static int ensure_window() {
  thread_local unsigned long long ready_ctx = 0;
  const unsigned long long ctx = current_context_id();
  if (ctx != 0 && ready_ctx == ctx) return GS_OK;
  int rc;
  double w[kSsimWin], sum = 0.0;
  for (int i = 0; i < kSsimWin; ++i) {
    const double d = (double)(i - kSsimR);
    w[i] = exp(-d * d / (2.0 * 1.5 * 1.5));
    sum += w[i];
  }
  float wf[kSsimWin];
  for (int i = 0; i < kSsimWin; ++i) wf[i] = (float)(w[i] / sum);
  rc = cuda_status(cudaMemcpyToSymbol(c_ssim_win, wf, sizeof(wf)));
  if (rc) return rc;
  ready_ctx = ctx != 0 ? ctx : current_context_id();
  return GS_OK;
}

static dim3 ssim_grid(int planes, int H, int W) {
  return dim3((unsigned)(((W + kSsimTW - 1) / kSsimTW) * planes),
              (unsigned)((H + kSsimTH - 1) / kSsimTH));
}

static bool ssim_grid_ok(int planes, int H, int W) {
  return (int64_t)((W + kSsimTW - 1) / kSsimTW) * planes < (int64_t)INT32_MAX &&
         (H + kSsimTH - 1) / kSsimTH <= 65535 &&
         (int64_t)planes * H * W < (int64_t)INT32_MAX;  // 32-bit element indices
}

static int64_t ssim_count(int planes, int H, int W, int valid) {
  if (!valid) return (int64_t)planes * H * W;
  return (int64_t)planes * (H - 2 * kSsimR) * (W - 2 * kSsimR);
}

}  // namespace gs

using namespace gs;

extern "C" size_t gs_ssim_scratch_bytes(int planes, int height, int width) {
  if (planes <= 0 || height <= 0 || width <= 0) return 0;
  return (size_t)3 * planes * height * width * sizeof(float);
}

extern "C" int gs_ssim_forward(int planes, int height, int width, const float *img1,
                               const float *img2, int valid, float *scratch,
                               size_t scratch_bytes, double *ssim_sum, void *stream) {
  if (planes <= 0 || height <= 0 || width <= 0 || img1 == nullptr || img2 == nullptr ||
      ssim_sum == nullptr)
    return GS_ERR_INVALID_ARGUMENT;
  if (valid && (height <= 2 * kSsimR || width <= 2 * kSsimR)) return GS_ERR_INVALID_ARGUMENT;
  if (!ssim_grid_ok(planes, height, width)) return GS_ERR_CAPACITY;
  if (scratch == nullptr || scratch_bytes < gs_ssim_scratch_bytes(planes, height, width))
    return GS_ERR_CAPACITY;
  int rc = ensure_window();
  if (rc) return rc;
  const int64_t plane_px = (int64_t)height * width;
  const float wscale = (float)(1.0 / (double)ssim_count(planes, height, width, valid));
  SsimSrc<false, float> src{img1, img2, 1, height, width};
  ssim_fwd_kernel<false, float><<<ssim_grid(planes, height, width), kSsimThreads, 0,
                                  reinterpret_cast<cudaStream_t>(stream)>>>(
      src, planes, valid, wscale, scratch, scratch + planes * plane_px,
      scratch + 2 * planes * plane_px, ssim_sum);
  count_launch();
  return launch_status();
}

extern "C" int gs_ssim_backward(int planes, int height, int width, const float *img1,
                                const float *img2, const float *scratch, const float *grad_out,
                                float *grad_img1, void *stream) {
  if (planes <= 0 || height <= 0 || width <= 0 || img1 == nullptr || img2 == nullptr ||
      scratch == nullptr || grad_img1 == nullptr)
    return GS_ERR_INVALID_ARGUMENT;
  if (!ssim_grid_ok(planes, height, width)) return GS_ERR_CAPACITY;
  int rc = ensure_window();
  if (rc) return rc;
  const int64_t plane_px = (int64_t)height * width;
  SsimSrc<false, float> src{img1, img2, 1, height, width};
  ssim_bwd_kernel<false, float, false><<<ssim_grid(planes, height, width), kSsimThreads, 0,
                                         reinterpret_cast<cudaStream_t>(stream)>>>(
      src, planes, scratch, scratch + planes * plane_px, scratch + 2 * planes * plane_px,
      grad_out, 0.0f, 0.0f, grad_img1, nullptr);
  count_launch();
  return launch_status();
}

extern "C" int gs_l1_ssim_loss_grad(int height, int width, const float *raw_image,
                                    const void *target, int target_is_u8, float ssim_lambda,
                                    float *grad_raw, double *sums, float *scratch,
                                    size_t scratch_bytes, void *stream) {
  if (height <= 2 * kSsimR || width <= 2 * kSsimR || raw_image == nullptr || target == nullptr ||
      grad_raw == nullptr || sums == nullptr)
    return GS_ERR_INVALID_ARGUMENT;
  if (!(ssim_lambda >= 0.0f && ssim_lambda <= 1.0f)) return GS_ERR_INVALID_ARGUMENT;
  if (scratch == nullptr || scratch_bytes < gs_ssim_scratch_bytes(3, height, width))
    return GS_ERR_CAPACITY;
  if (!ssim_grid_ok(3, height, width)) return GS_ERR_CAPACITY;
  int rc = ensure_window();
  if (rc) return rc;
  const int planes = 3;
  const int64_t plane_px = (int64_t)height * width;
  const int64_t numel = 3 * plane_px;
  const float wscale = (float)(-(double)ssim_lambda / (double)ssim_count(3, height, width, 1));
  const float l1_weight = 1.0f - ssim_lambda;
  const float inv_numel = (float)(1.0 / (double)numel);
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  float *m0 = scratch, *m1 = scratch + planes * plane_px, *m2 = scratch + 2 * planes * plane_px;
  const dim3 grid = ssim_grid(planes, height, width);
  if (target_is_u8) {
    SsimSrc<true, uint8_t> src{raw_image, reinterpret_cast<const uint8_t *>(target), 3, height,
                               width};
    ssim_fwd_kernel<true, uint8_t><<<grid, kSsimThreads, 0, st>>>(src, planes, 1, wscale, m0, m1,
                                                                  m2, sums + 1);
    ssim_bwd_kernel<true, uint8_t, true><<<grid, kSsimThreads, 0, st>>>(
        src, planes, m0, m1, m2, nullptr, l1_weight, inv_numel, grad_raw, sums);
  } else {
    SsimSrc<true, float> src{raw_image, reinterpret_cast<const float *>(target), 3, height, width};
    ssim_fwd_kernel<true, float><<<grid, kSsimThreads, 0, st>>>(src, planes, 1, wscale, m0, m1, m2,
                                                                sums + 1);
    ssim_bwd_kernel<true, float, true><<<grid, kSsimThreads, 0, st>>>(
        src, planes, m0, m1, m2, nullptr, l1_weight, inv_numel, grad_raw, sums);
  }
  count_launch();
  count_launch();
  return launch_status();
}
