// gs_common.cuh -- shared device math, status plumbing and launch accounting
// for the B200 Gaussian-splatting rasterizer.
//
// The per-Gaussian float expressions below keep the operand order of the
// reference kernels (ruguangyou/3dgs_from_scratch src/cuda/kernel.cu) so that
// nvcc contracts them into the same fused multiply-adds: depth bits and the
// pixel-space tile rectangle feed the sort keys, which must match the
// reference bit for bit. Everything else (memory layout, fusion, launch
// shape) is this library's own.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/gs_b200.h"

namespace gs {

constexpr float kLowPass = 0.3f;        // kernel.cu:23
constexpr float kFovClamp = 1.3f;       // kernel.cu:24
constexpr float kTransEps = 1e-10f;     // kernel.cu:25

// Real SH constants, degree 0..3 (kernel.cu:7-22).
constexpr float kC0 = 0.28209479177387814f;
constexpr float kC1 = 0.4886025119029199f;
constexpr float kC2xy = 1.0925484305920792f;
constexpr float kC2zz = 0.31539156525252005f;
constexpr float kC2xxyy = 0.5462742152960396f;
constexpr float kC3a = 0.5900435899266435f;
constexpr float kC3xyz = 2.890611442640554f;
constexpr float kC3c = 0.4570457994644658f;
constexpr float kC3zzz = 0.3731763325901154f;
constexpr float kC3zxx = 1.445305721320277f;

// ---- host-side plumbing (defined in capi.cu) ------------------------------
void count_launch(int n = 1);
int cuda_status(cudaError_t e);                 // maps and records a CUDA error
int launch_status();                            // cudaGetLastError after launches
uint32_t *device_status_word();                 // per-device status word (device ptr)
// Zero-fill of device memory by a kernel (a memset inside a CUDA graph can be
// queued on a copy engine behind a large host transfer; a kernel is not).
int zero_async(void *p, size_t bytes, cudaStream_t st);

// Device address of a __device__ symbol in the current context. Host code
// cannot use the symbol itself as a pointer; the address is looked up with
// cudaGetSymbolAddress and cached per host thread (the caller passes a
// thread_local cache) against the context's process-unique id, so a context
// torn down and re-created (cudaDeviceReset) or a switch of device gets a
// fresh lookup.
struct SymbolCache {
  unsigned long long context_id = 0;
  void *address = nullptr;
};
int symbol_address(const void *symbol, SymbolCache *cache, void **out);
// Process-unique id of the current CUDA context (0 when none is current yet);
// per-context set-up (function attributes, constant uploads) is keyed on it.
unsigned long long current_context_id();

// Bounded spin limit for look-back waits. A predecessor that is resident
// publishes within microseconds; this bound (~ tens of ms) only ends a wait
// that can never finish, which then records GS_ERR_DEVICE_TIMEOUT.
constexpr uint32_t kSpinLimit = 1u << 20;

__device__ __forceinline__ uint32_t ld_volatile_u32(const uint32_t *p) {
  uint32_t v;
  asm volatile("ld.volatile.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ void st_volatile_u32(uint32_t *p, uint32_t v) {
  asm volatile("st.volatile.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

__device__ __forceinline__ uint32_t lane_id() {
  uint32_t l;
  asm("mov.u32 %0, %%laneid;" : "=r"(l));
  return l;
}

// ---- bulk asynchronous copies (the TMA engine, 1-D, no tensor map) ----------
// Used without cluster multicast: every source is this GPU's own memory.

__device__ __forceinline__ uint32_t smem_addr(const void *p) {
  return (uint32_t)__cvta_generic_to_shared(p);
}

__device__ __forceinline__ void mbar_init(uint64_t *bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

// Arrive on the barrier and add `bytes` to the transaction count it waits for.
__device__ __forceinline__ void mbar_expect_tx(uint64_t *bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_addr(bar)),
               "r"(bytes)
               : "memory");
}

// Global -> shared bulk copy; completion is signalled on `bar`. dst, src and
// bytes must be multiples of 16.
__device__ __forceinline__ void bulk_load(void *smem_dst, const void *gsrc, uint32_t bytes,
                                          uint64_t *bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_addr(smem_dst)),
      "l"(gsrc), "r"(bytes), "r"(smem_addr(bar))
      : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t *bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(ok)
      : "r"(smem_addr(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Bounded wait for the barrier phase with parity `parity` to complete.
__device__ __forceinline__ bool mbar_wait(uint64_t *bar, uint32_t parity) {
  for (uint32_t i = 0; i < kSpinLimit; ++i)
    if (mbar_try_wait(bar, parity)) return true;
  return false;
}

// Shared -> global bulk copy, tracked by bulk groups.
__device__ __forceinline__ void bulk_store(void *gdst, const void *smem_src, uint32_t bytes) {
  asm volatile("cp.async.bulk.global.shared::cta.bulk_group [%0], [%1], %2;" ::"l"(gdst),
               "r"(smem_addr(smem_src)), "r"(bytes)
               : "memory");
}
// Shared -> global bulk reduction: global[i] += shared[i] (fp32), tracked by
// bulk groups like bulk_store.
__device__ __forceinline__ void bulk_reduce_add(float *gdst, const float *smem_src,
                                                uint32_t bytes) {
  asm volatile("cp.reduce.async.bulk.global.shared::cta.bulk_group.add.f32 [%0], [%1], %2;" ::"l"(
                   gdst),
               "r"(smem_addr(smem_src)), "r"(bytes)
               : "memory");
}
__device__ __forceinline__ void bulk_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
// Wait until the committed bulk stores have read their shared-memory source.
__device__ __forceinline__ void bulk_wait_read_all() {
  asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");
}
// Wait until the committed bulk stores are complete.
__device__ __forceinline__ void bulk_wait_all() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }
// Make this thread's generic-proxy shared-memory writes visible to bulk copies.
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// ---- projection -------------------------------------------------------------

struct Cam {
  float W[12];  // rows 0..2 of the row-major world_to_camera
  float fx, fy, cx, cy;
};

__device__ __forceinline__ Cam load_cam(const float *__restrict__ w2c,
                                        const float *__restrict__ K) {
  Cam c;
#pragma unroll
  for (int i = 0; i < 12; ++i) c.W[i] = __ldg(w2c + i);
  c.fx = __ldg(K + 0);
  c.cx = __ldg(K + 2);
  c.fy = __ldg(K + 4);
  c.cy = __ldg(K + 5);
  return c;
}

// Camera-space position (kernel.cu:27-44).
__device__ __forceinline__ float3 to_camera(const Cam &c, float px, float py, float pz) {
  float3 r;
  r.x = c.W[0] * px + c.W[1] * py + c.W[2] * pz + c.W[3];
  r.y = c.W[4] * px + c.W[5] * py + c.W[6] * pz + c.W[7];
  r.z = c.W[8] * px + c.W[9] * py + c.W[10] * pz + c.W[11];
  return r;
}

// Rotation of an (x, y, z, w) quaternion, row-major (kernel.cu:57-65).
__device__ __forceinline__ void quat_to_rot(float x, float y, float z, float w, float R[9]) {
  R[0] = 1 - 2 * y * y - 2 * z * z;
  R[1] = 2 * x * y - 2 * z * w;
  R[2] = 2 * x * z + 2 * y * w;
  R[3] = 2 * x * y + 2 * z * w;
  R[4] = 1 - 2 * x * x - 2 * z * z;
  R[5] = 2 * y * z - 2 * x * w;
  R[6] = 2 * x * z - 2 * y * w;
  R[7] = 2 * y * z + 2 * x * w;
  R[8] = 1 - 2 * x * x - 2 * y * y;
}

// Camera covariance Cc = W3 * A * W3^T for a symmetric world covariance A.
__device__ __forceinline__ void cam_cov(const Cam &c, const float A[9], float Cc[9]) {
  const float *W = c.W;
  float WA[9];
#pragma unroll
  for (int i = 0; i < 3; ++i)
#pragma unroll
    for (int j = 0; j < 3; ++j)
      WA[i * 3 + j] = W[i * 4] * A[j] + W[i * 4 + 1] * A[3 + j] + W[i * 4 + 2] * A[6 + j];
#pragma unroll
  for (int i = 0; i < 3; ++i)
#pragma unroll
    for (int j = 0; j < 3; ++j)
      Cc[i * 3 + j] = WA[i * 3] * W[j * 4] + WA[i * 3 + 1] * W[j * 4 + 1] + WA[i * 3 + 2] * W[j * 4 + 2];
}

struct Jac {
  float J0, J2, J4, J5, inv_z, x_ndc, y_ndc, xc, yc, lim_x, lim_y;
};

// Perspective Jacobian with the 1.3x FOV clamp (kernel.cu:110-127).
__device__ __forceinline__ Jac jacobian(const Cam &c, int width, int height, float3 p) {
  Jac j;
  j.lim_x = kFovClamp * fmaxf(c.cx, (float)width - c.cx) / c.fx;
  j.lim_y = kFovClamp * fmaxf(c.cy, (float)height - c.cy) / c.fy;
  j.inv_z = 1.0f / p.z;
  j.x_ndc = p.x * j.inv_z;
  j.y_ndc = p.y * j.inv_z;
  j.xc = fminf(j.lim_x, fmaxf(-j.lim_x, j.x_ndc));
  j.yc = fminf(j.lim_y, fmaxf(-j.lim_y, j.y_ndc));
  j.J0 = c.fx * j.inv_z;
  j.J2 = -c.fx * j.xc * j.inv_z;
  j.J4 = c.fy * j.inv_z;
  j.J5 = -c.fy * j.yc * j.inv_z;
  return j;
}

// World covariance R diag(s^2) R^T, full 3x3 (kernel.cu:66-80); view-independent.
__device__ __forceinline__ void world_cov(float sx, float sy, float sz, float qx, float qy,
                                          float qz, float qw, float Cw[9]) {
  float R[9];
  quat_to_rot(qx, qy, qz, qw, R);
  float s2[3] = {sx * sx, sy * sy, sz * sz};
#pragma unroll
  for (int i = 0; i < 3; ++i)
#pragma unroll
    for (int k = 0; k < 3; ++k)
      Cw[i * 3 + k] = R[i * 3] * s2[0] * R[k * 3] + R[i * 3 + 1] * s2[1] * R[k * 3 + 1] +
                      R[i * 3 + 2] * s2[2] * R[k * 3 + 2];
}

// Image-space covariance (a, b, c) with low-pass and symmetrisation from the
// world covariance (kernel.cu:82-155).
__device__ __forceinline__ float3 image_cov_from(const Cam &c, int width, int height, float3 p,
                                                 const float Cw[9]) {
  float Cc[9];
  cam_cov(c, Cw, Cc);
  Jac j = jacobian(c, width, height, p);
  float A0 = j.J0 * Cc[0] + j.J2 * Cc[6];
  float A1 = j.J0 * Cc[1] + j.J2 * Cc[7];
  float A2 = j.J0 * Cc[2] + j.J2 * Cc[8];
  float B0 = j.J4 * Cc[3] + j.J5 * Cc[6];
  float B1 = j.J4 * Cc[4] + j.J5 * Cc[7];
  float B2 = j.J4 * Cc[5] + j.J5 * Cc[8];
  float c00 = A0 * j.J0 + A2 * j.J2;
  float c01 = A1 * j.J4 + A2 * j.J5;
  float c10 = B0 * j.J0 + B2 * j.J2;
  float c11 = B1 * j.J4 + B2 * j.J5;
  return make_float3(c00 + kLowPass, 0.5f * (c01 + c10), c11 + kLowPass);
}

// Image-space covariance (a, b, c) with low-pass and symmetrisation
// (kernel.cu:46-155).
__device__ __forceinline__ float3 image_cov(const Cam &c, int width, int height, float3 p,
                                            float sx, float sy, float sz, float qx, float qy,
                                            float qz, float qw) {
  float Cw[9];
  world_cov(sx, sy, sz, qx, qy, qz, qw, Cw);
  return image_cov_from(c, width, height, p, Cw);
}

// Result of the per-Gaussian projection with the reference's culling order
// (kernel.cu:438-500). visible == false means mask = 0.
struct Projected {
  bool visible;
  bool cov_written;  // the reference writes cov_image before the radius cull
  float u, v, depth;
  float3 cov, conic;
  float ru, rv;
};

// project_one with the world covariance given (computed once per Gaussian
// when several views share it); covw == nullptr computes it from the scale
// and quaternion.
__device__ __forceinline__ Projected project_one_cw(const Cam &c, int width, int height,
                                                    float near_plane, float far_plane,
                                                    float min_opacity, float min_radius,
                                                    float max_radius, float px, float py,
                                                    float pz, const float covw[9], float opac) {
  Projected r;
  r.visible = false;
  r.cov_written = false;
  if (opac < min_opacity) return r;
  float3 pc = to_camera(c, px, py, pz);
  if (pc.z < near_plane || pc.z > far_plane) return r;
  r.u = c.fx * pc.x / pc.z + c.cx;
  r.v = c.fy * pc.y / pc.z + c.cy;
  r.depth = pc.z;
  r.cov = image_cov_from(c, width, height, pc, covw);
  r.cov_written = true;
  float det = r.cov.x * r.cov.z - r.cov.y * r.cov.y;
  float inv_det = 1.0f / fmaxf(det, 1e-12f);
  r.ru = fmaxf(sqrtf(r.cov.x), 1e-12f) * 3.0f;
  r.rv = fmaxf(sqrtf(r.cov.z), 1e-12f) * 3.0f;
  float radius = fmaxf(r.ru, r.rv);
  if (radius < min_radius || radius > max_radius) return r;
  if (r.u < -r.ru || r.u > (float)width + r.ru || r.v < -r.rv || r.v > (float)height + r.rv)
    return r;
  r.conic = make_float3(r.cov.z * inv_det, -r.cov.y * inv_det, r.cov.x * inv_det);
  r.visible = true;
  return r;
}

__device__ __forceinline__ Projected project_one(const Cam &c, int width, int height,
                                                 float near_plane, float far_plane,
                                                 float min_opacity, float min_radius,
                                                 float max_radius, float px, float py,
                                                 float pz, float sx, float sy, float sz,
                                                 float qx, float qy, float qz, float qw,
                                                 float opac) {
  float Cw[9];
  world_cov(sx, sy, sz, qx, qy, qz, qw, Cw);
  return project_one_cw(c, width, height, near_plane, far_plane, min_opacity, min_radius,
                        max_radius, px, py, pz, Cw, opac);
}

// Backward of projection + covariance for one Gaussian (kernel.cu:157-409).
// The off-diagonal conic gradient enters the Jacobian term as the full g01,
// as the reference does (kernel.cu:384-389).
__device__ __forceinline__ void project_backward_one(
    const Cam &c, int width, int height, float3 pc, float gu, float gv, float sx, float sy,
    float sz, float qi, float qj, float qk, float qr, float3 cov, float gA, float gB, float gC,
    float gm[3], float gs[3], float gq[4]) {
  const float *W = c.W;
  const float fx = c.fx, fy = c.fy;
  Jac j = jacobian(c, width, height, pc);
  float x = pc.x, y = pc.y, z = pc.z;
  float iz2 = j.inv_z * j.inv_z;
  float iz3 = iz2 * j.inv_z;
  bool xcl = fabsf(j.x_ndc) > j.lim_x;
  bool ycl = fabsf(j.y_ndc) > j.lim_y;
  float gm0 = (gu * fx * (W[0] * z - W[8] * x) + gv * fy * (W[4] * z - W[8] * y)) * iz2;
  float gm1 = (gu * fx * (W[1] * z - W[9] * x) + gv * fy * (W[5] * z - W[9] * y)) * iz2;
  float gm2 = (-gu * fx * (W[10] * x - W[2] * z) - gv * fy * (W[10] * y - W[6] * z)) * iz2;

  float U[6];
  U[0] = j.J0 * W[0] + j.J2 * W[8];
  U[1] = j.J0 * W[1] + j.J2 * W[9];
  U[2] = j.J0 * W[2] + j.J2 * W[10];
  U[3] = j.J4 * W[4] + j.J5 * W[8];
  U[4] = j.J4 * W[5] + j.J5 * W[9];
  U[5] = j.J4 * W[6] + j.J5 * W[10];

  float R[9];
  quat_to_rot(qi, qj, qk, qr, R);
  float M[9] = {R[0] * sx, R[1] * sy, R[2] * sz, R[3] * sx, R[4] * sy,
                R[5] * sz, R[6] * sx, R[7] * sy, R[8] * sz};

  float a = cov.x, b = cov.y, cc = cov.z;
  float det = a * cc - b * b;
  float id = 1.0f / fmaxf(det, 1e-12f);
  float id2 = id * id;
  float D[3][3] = {{-cc * cc * id2, b * cc * id2, -b * b * id2},
                   {2.0f * b * cc * id2, -(a * cc + b * b) * id2, 2.0f * a * b * id2},
                   {-b * b * id2, a * b * id2, -a * a * id2}};
  float gcon[3] = {gA, gB, gC};
  float gE2[3];
#pragma unroll
  for (int r = 0; r < 3; ++r) {
    gE2[r] = 0.0f;
#pragma unroll
    for (int k = 0; k < 3; ++k) gE2[r] += gcon[k] * D[r][k];
  }
  float gE[9];
#pragma unroll
  for (int r = 0; r < 3; ++r)
#pragma unroll
    for (int k = 0; k < 3; ++k) {
      float t0 = U[r] * U[k];
      float t1 = U[r] * U[3 + k];
      float t2 = U[k] * U[3 + r];
      float t3 = U[3 + r] * U[3 + k];
      gE[r * 3 + k] = gE2[0] * t0 + 0.5f * gE2[1] * (t1 + t2) + gE2[2] * t3;
    }
  float gM[9];
#pragma unroll
  for (int r = 0; r < 3; ++r)
#pragma unroll
    for (int col = 0; col < 3; ++col) {
      float acc = 0.0f;
#pragma unroll
      for (int k = 0; k < 3; ++k) acc += (gE[r * 3 + k] + gE[k * 3 + r]) * M[k * 3 + col];
      gM[r * 3 + col] = acc;
    }
  gs[0] = gM[0] * R[0] + gM[3] * R[3] + gM[6] * R[6];
  gs[1] = gM[1] * R[1] + gM[4] * R[4] + gM[7] * R[7];
  gs[2] = gM[2] * R[2] + gM[5] * R[5] + gM[8] * R[8];

  float dqi[9] = {0.0f, 2.0f * sy * qj, 2.0f * sz * qk, 2.0f * sx * qj, -4.0f * sy * qi,
                  -2.0f * sz * qr, 2.0f * sx * qk, 2.0f * sy * qr, -4.0f * sz * qi};
  float dqj[9] = {-4.0f * sx * qj, 2.0f * sy * qi, 2.0f * sz * qr, 2.0f * sx * qi, 0.0f,
                  2.0f * sz * qk, -2.0f * sx * qr, 2.0f * sy * qk, -4.0f * sz * qj};
  float dqk[9] = {-4.0f * sx * qk, -2.0f * sy * qr, 2.0f * sz * qi, 2.0f * sx * qr,
                  -4.0f * sy * qk, 2.0f * sz * qj, 2.0f * sx * qi, 2.0f * sy * qj, 0.0f};
  float dqr[9] = {0.0f, -2.0f * sy * qk, 2.0f * sz * qj, 2.0f * sx * qk, 0.0f,
                  -2.0f * sz * qi, -2.0f * sx * qj, 2.0f * sy * qi, 0.0f};
  float q0 = 0.f, q1 = 0.f, q2 = 0.f, q3 = 0.f;
#pragma unroll
  for (int k = 0; k < 9; ++k) {
    q0 += gM[k] * dqi[k];
    q1 += gM[k] * dqj[k];
    q2 += gM[k] * dqk[k];
    q3 += gM[k] * dqr[k];
  }
  gq[0] = q0;
  gq[1] = q1;
  gq[2] = q2;
  gq[3] = q3;

  float E[9];
#pragma unroll
  for (int r = 0; r < 3; ++r)
#pragma unroll
    for (int k = 0; k < 3; ++k)
      E[r * 3 + k] = M[r * 3] * M[k * 3] + M[r * 3 + 1] * M[k * 3 + 1] + M[r * 3 + 2] * M[k * 3 + 2];
  float Cc[9];
  cam_cov(c, E, Cc);

  float g00 = gE2[0], g01 = gE2[1], g11 = gE2[2];
  float GJ00 = g00 * j.J0;
  float GJ01 = g01 * j.J4;
  float GJ02 = g00 * j.J2 + g01 * j.J5;
  float GJ10 = g01 * j.J0;
  float GJ11 = g11 * j.J4;
  float GJ12 = g01 * j.J2 + g11 * j.J5;
  float dJ00 = 2.0f * (GJ00 * Cc[0] + GJ01 * Cc[3] + GJ02 * Cc[6]);
  float dJ02 = 2.0f * (GJ00 * Cc[2] + GJ01 * Cc[5] + GJ02 * Cc[8]);
  float dJ11 = 2.0f * (GJ10 * Cc[1] + GJ11 * Cc[4] + GJ12 * Cc[7]);
  float dJ12 = 2.0f * (GJ10 * Cc[2] + GJ11 * Cc[5] + GJ12 * Cc[8]);
  float gx = xcl ? 0.0f : dJ02 * (-fx * iz2);
  float gy = ycl ? 0.0f : dJ12 * (-fy * iz2);
  float dJ02dz = xcl ? (fx * j.xc * iz2) : (2.0f * fx * x * iz3);
  float dJ12dz = ycl ? (fy * j.yc * iz2) : (2.0f * fy * y * iz3);
  float gz = dJ00 * (-fx * iz2) + dJ11 * (-fy * iz2) + dJ02 * dJ02dz + dJ12 * dJ12dz;
  gm[0] = gm0 + (W[0] * gx + W[4] * gy + W[8] * gz);
  gm[1] = gm1 + (W[1] * gx + W[5] * gy + W[9] * gz);
  gm[2] = gm2 + (W[2] * gx + W[6] * gy + W[10] * gz);
}

// ---- fused backward: per-view and per-Gaussian parts ---------------------------
//
// project_backward_one's chain, split for the multi-view backward: the part
// from the conic gradient down to d loss / d (world covariance) and the
// mean's terms depend on the view; the part from d loss / d (world
// covariance) to the scale and rotation is linear and view-independent, so
// it runs once per Gaussian on the sum over views.

// World covariance Sigma = M M^T, M = R diag(s), symmetric: xx xy xz yy yz zz.
__device__ __forceinline__ void world_cov_sym(float sx, float sy, float sz, float qi, float qj,
                                              float qk, float qr, float Sg[6]) {
  float R[9];
  quat_to_rot(qi, qj, qk, qr, R);
  const float M[9] = {R[0] * sx, R[1] * sy, R[2] * sz, R[3] * sx, R[4] * sy,
                      R[5] * sz, R[6] * sx, R[7] * sy, R[8] * sz};
  Sg[0] = M[0] * M[0] + M[1] * M[1] + M[2] * M[2];
  Sg[1] = M[0] * M[3] + M[1] * M[4] + M[2] * M[5];
  Sg[2] = M[0] * M[6] + M[1] * M[7] + M[2] * M[8];
  Sg[3] = M[3] * M[3] + M[4] * M[4] + M[5] * M[5];
  Sg[4] = M[3] * M[6] + M[4] * M[7] + M[5] * M[8];
  Sg[5] = M[6] * M[6] + M[7] * M[7] + M[8] * M[8];
}

__device__ __forceinline__ constexpr int sym3(int r, int k) {
  return r <= k ? (r == 0 ? k : (r == 1 ? 2 + k : 5)) : (k == 0 ? r : (k == 1 ? 2 + r : 5));
}

// Camera covariance Cc = W3 Sigma W3^T of a symmetric Sigma (both as 6 values).
__device__ __forceinline__ void cam_cov_sym(const Cam &c, const float Sg[6], float Cc[6]) {
  const float *W = c.W;
  float WA[9];
#pragma unroll
  for (int i = 0; i < 3; ++i)
#pragma unroll
    for (int j = 0; j < 3; ++j)
      WA[i * 3 + j] = W[i * 4] * Sg[sym3(0, j)] + W[i * 4 + 1] * Sg[sym3(1, j)] +
                      W[i * 4 + 2] * Sg[sym3(2, j)];
#pragma unroll
  for (int i = 0; i < 3; ++i)
#pragma unroll
    for (int j = i; j < 3; ++j)
      Cc[sym3(i, j)] = WA[i * 3] * W[j * 4] + WA[i * 3 + 1] * W[j * 4 + 1] +
                       WA[i * 3 + 2] * W[j * 4 + 2];
}

// One view's part: adds d loss / d mean (projection and the Jacobian's
// dependence on the mean) to gm and d loss / d Sigma (symmetric) to gSg.
// Same formulas as project_backward_one (kernel.cu:157-409), including the
// full off-diagonal conic gradient in the Jacobian term (kernel.cu:384-389).
__device__ __forceinline__ void view_proj_backward(const Cam &c, int width, int height, float3 pc,
                                                   const float Sg[6], float gu, float gv,
                                                   float gA, float gB, float gC, float gm[3],
                                                   float gSg[6]) {
  const float *W = c.W;
  const float fx = c.fx, fy = c.fy;
  const Jac j = jacobian(c, width, height, pc);
  const float x = pc.x, y = pc.y, z = pc.z;
  const float iz2 = j.inv_z * j.inv_z;
  const float iz3 = iz2 * j.inv_z;
  const bool xcl = fabsf(j.x_ndc) > j.lim_x;
  const bool ycl = fabsf(j.y_ndc) > j.lim_y;
  const float gm0 = (gu * fx * (W[0] * z - W[8] * x) + gv * fy * (W[4] * z - W[8] * y)) * iz2;
  const float gm1 = (gu * fx * (W[1] * z - W[9] * x) + gv * fy * (W[5] * z - W[9] * y)) * iz2;
  const float gm2 = (-gu * fx * (W[10] * x - W[2] * z) - gv * fy * (W[10] * y - W[6] * z)) * iz2;

  float Cc[6];
  cam_cov_sym(c, Sg, Cc);
  // image covariance (image_cov)
  const float A0 = j.J0 * Cc[0] + j.J2 * Cc[2];
  const float A1 = j.J0 * Cc[1] + j.J2 * Cc[4];
  const float A2 = j.J0 * Cc[2] + j.J2 * Cc[5];
  const float B0 = j.J4 * Cc[1] + j.J5 * Cc[2];
  const float B1 = j.J4 * Cc[3] + j.J5 * Cc[4];
  const float B2 = j.J4 * Cc[4] + j.J5 * Cc[5];
  const float a = A0 * j.J0 + A2 * j.J2 + kLowPass;
  const float b = 0.5f * ((A1 * j.J4 + A2 * j.J5) + (B0 * j.J0 + B2 * j.J2));
  const float cc = B1 * j.J4 + B2 * j.J5 + kLowPass;
  const float det = a * cc - b * b;
  const float id = 1.0f / fmaxf(det, 1e-12f);
  const float id2 = id * id;
  // d loss / d (image covariance a, b, c) from the conic gradient
  const float g00 = (-cc * cc * gA + b * cc * gB - b * b * gC) * id2;
  const float g01 = (2.0f * b * cc * gA - (a * cc + b * b) * gB + 2.0f * a * b * gC) * id2;
  const float g11 = (-b * b * gA + a * b * gB - a * a * gC) * id2;
  float U[6];
  U[0] = j.J0 * W[0] + j.J2 * W[8];
  U[1] = j.J0 * W[1] + j.J2 * W[9];
  U[2] = j.J0 * W[2] + j.J2 * W[10];
  U[3] = j.J4 * W[4] + j.J5 * W[8];
  U[4] = j.J4 * W[5] + j.J5 * W[9];
  U[5] = j.J4 * W[6] + j.J5 * W[10];
#pragma unroll
  for (int r = 0; r < 3; ++r)
#pragma unroll
    for (int k = r; k < 3; ++k)
      gSg[sym3(r, k)] += g00 * (U[r] * U[k]) + 0.5f * g01 * (U[r] * U[3 + k] + U[k] * U[3 + r]) +
                         g11 * (U[3 + r] * U[3 + k]);
  const float GJ00 = g00 * j.J0;
  const float GJ01 = g01 * j.J4;
  const float GJ02 = g00 * j.J2 + g01 * j.J5;
  const float GJ10 = g01 * j.J0;
  const float GJ11 = g11 * j.J4;
  const float GJ12 = g01 * j.J2 + g11 * j.J5;
  const float dJ00 = 2.0f * (GJ00 * Cc[0] + GJ01 * Cc[1] + GJ02 * Cc[2]);
  const float dJ02 = 2.0f * (GJ00 * Cc[2] + GJ01 * Cc[4] + GJ02 * Cc[5]);
  const float dJ11 = 2.0f * (GJ10 * Cc[1] + GJ11 * Cc[3] + GJ12 * Cc[4]);
  const float dJ12 = 2.0f * (GJ10 * Cc[2] + GJ11 * Cc[4] + GJ12 * Cc[5]);
  const float gx = xcl ? 0.0f : dJ02 * (-fx * iz2);
  const float gy = ycl ? 0.0f : dJ12 * (-fy * iz2);
  const float dJ02dz = xcl ? (fx * j.xc * iz2) : (2.0f * fx * x * iz3);
  const float dJ12dz = ycl ? (fy * j.yc * iz2) : (2.0f * fy * y * iz3);
  const float gz = dJ00 * (-fx * iz2) + dJ11 * (-fy * iz2) + dJ02 * dJ02dz + dJ12 * dJ12dz;
  gm[0] += gm0 + (W[0] * gx + W[4] * gy + W[8] * gz);
  gm[1] += gm1 + (W[1] * gx + W[5] * gy + W[9] * gz);
  gm[2] += gm2 + (W[2] * gx + W[6] * gy + W[10] * gz);
}

// The view-independent part: d loss / d Sigma (symmetric, summed over the
// views) to the activated scale and the quaternion (kernel.cu:300-375).
__device__ __forceinline__ void cov_backward(const float gSg[6], float sx, float sy, float sz,
                                             float qi, float qj, float qk, float qr, float gs[3],
                                             float gq[4]) {
  float R[9];
  quat_to_rot(qi, qj, qk, qr, R);
  const float M[9] = {R[0] * sx, R[1] * sy, R[2] * sz, R[3] * sx, R[4] * sy,
                      R[5] * sz, R[6] * sx, R[7] * sy, R[8] * sz};
  float gM[9];
#pragma unroll
  for (int r = 0; r < 3; ++r)
#pragma unroll
    for (int col = 0; col < 3; ++col) {
      float acc = 0.0f;
#pragma unroll
      for (int k = 0; k < 3; ++k) acc += (2.0f * gSg[sym3(r, k)]) * M[k * 3 + col];
      gM[r * 3 + col] = acc;
    }
  gs[0] = gM[0] * R[0] + gM[3] * R[3] + gM[6] * R[6];
  gs[1] = gM[1] * R[1] + gM[4] * R[4] + gM[7] * R[7];
  gs[2] = gM[2] * R[2] + gM[5] * R[5] + gM[8] * R[8];
  const float dqi[9] = {0.0f, 2.0f * sy * qj, 2.0f * sz * qk, 2.0f * sx * qj, -4.0f * sy * qi,
                        -2.0f * sz * qr, 2.0f * sx * qk, 2.0f * sy * qr, -4.0f * sz * qi};
  const float dqj[9] = {-4.0f * sx * qj, 2.0f * sy * qi, 2.0f * sz * qr, 2.0f * sx * qi, 0.0f,
                        2.0f * sz * qk, -2.0f * sx * qr, 2.0f * sy * qk, -4.0f * sz * qj};
  const float dqk[9] = {-4.0f * sx * qk, -2.0f * sy * qr, 2.0f * sz * qi, 2.0f * sx * qr,
                        -4.0f * sy * qk, 2.0f * sz * qj, 2.0f * sx * qi, 2.0f * sy * qj, 0.0f};
  const float dqr[9] = {0.0f, -2.0f * sy * qk, 2.0f * sz * qj, 2.0f * sx * qk, 0.0f,
                        -2.0f * sz * qi, -2.0f * sx * qj, 2.0f * sy * qi, 0.0f};
  float q0 = 0.f, q1 = 0.f, q2 = 0.f, q3 = 0.f;
#pragma unroll
  for (int k = 0; k < 9; ++k) {
    q0 += gM[k] * dqi[k];
    q1 += gM[k] * dqj[k];
    q2 += gM[k] * dqk[k];
    q3 += gM[k] * dqr[k];
  }
  gq[0] = q0;
  gq[1] = q1;
  gq[2] = q2;
  gq[3] = q3;
}

// ---- parameter activations (scripts/train.py:135-140 of the reference) --------

// exp(log-scale), q / max(|q|, 1e-12), sigmoid(logit): the activations the
// reference applies in Torch before render().
struct Activated {
  float sx, sy, sz, qx, qy, qz, qw, opac, qnorm;
};

__device__ __forceinline__ Activated activate_params(float lsx, float lsy, float lsz, float qx,
                                                     float qy, float qz, float qw, float logit) {
  Activated a;
  a.sx = expf(lsx);
  a.sy = expf(lsy);
  a.sz = expf(lsz);
  a.qnorm = sqrtf(qx * qx + qy * qy + qz * qz + qw * qw);
  const float nq = fmaxf(a.qnorm, 1e-12f);
  a.qx = qx / nq;
  a.qy = qy / nq;
  a.qz = qz / nq;
  a.qw = qw / nq;
  a.opac = 1.0f / (1.0f + expf(-logit));
  return a;
}

// ---- spherical harmonics ----------------------------------------------------

struct ViewDir {
  float x, y, z, inv_norm;
};

__device__ __forceinline__ ViewDir view_dir(float cpx, float cpy, float cpz, float px,
                                            float py, float pz) {
  float dx = px - cpx, dy = py - cpy, dz = pz - cpz;
  float n = sqrtf(dx * dx + dy * dy + dz * dz);
  ViewDir d;
  d.inv_norm = 1.0f / (n + 1e-8f);
  d.x = dx * d.inv_norm;
  d.y = dy * d.inv_norm;
  d.z = dz * d.inv_norm;
  return d;
}

// Basis values 0..15 (kernel.cu:578-595).
__device__ __forceinline__ void sh_basis(float x, float y, float z, float b[16]) {
  float xx = x * x, yy = y * y, zz = z * z, xy = x * y, xz = x * z, yz = y * z;
  b[0] = kC0;
  b[1] = -kC1 * y;
  b[2] = kC1 * z;
  b[3] = -kC1 * x;
  b[4] = kC2xy * xy;
  b[5] = kC2xy * yz;
  b[6] = kC2zz * (3 * zz - 1);
  b[7] = kC2xy * xz;
  b[8] = kC2xxyy * (xx - yy);
  b[9] = kC3a * y * (xx - yy);
  b[10] = kC3xyz * (x * y * z);
  b[11] = kC3c * y * (4 * zz - xx - yy);
  b[12] = kC3zzz * z * (2 * zz - 3 * xx - 3 * yy);
  b[13] = kC3c * x * (4 * zz - xx - yy);
  b[14] = kC3zxx * z * (xx - yy);
  b[15] = kC3a * x * (xx - 3 * yy);
}

// Sigmoid the way the reference computes it (kernel.cu:608-610).
__device__ __forceinline__ float ref_sigmoid(float r) {
  return (float)(1.0 / (1.0 + (double)expf(-r)));
}

// d(view-dependent colour)/d(mean) through the normalised direction
// (kernel.cu:674-781); g is d loss / d raw colour, rest points at the 45
// coefficients (15 bases x rgb) of one Gaussian.
template <typename RestAt>
__device__ __forceinline__ float3 sh_dir_backward(const ViewDir &d, float g0, float g1,
                                                  float g2, RestAt rest) {
  float x = d.x, y = d.y, z = d.z;
  float xx = x * x, yy = y * y, zz = z * z, xy = x * y, xz = x * z, yz = y * z;
  float bx[15] = {0.0f, 0.0f, -kC1, kC2xy * y, 0.0f, 0.0f, kC2xy * z, 2.0f * kC2xxyy * x,
                  2.0f * kC3a * x * y, kC3xyz * y * z, -2.0f * kC3c * x * y,
                  -6.0f * kC3zzz * x * z, kC3c * (4.0f * zz - 3.0f * xx - yy),
                  2.0f * kC3zxx * x * z, 3.0f * kC3a * (xx - yy)};
  float by[15] = {-kC1, 0.0f, 0.0f, kC2xy * x, kC2xy * z, 0.0f, 0.0f, -2.0f * kC2xxyy * y,
                  kC3a * (xx - 3.0f * yy), kC3xyz * x * z, kC3c * (4.0f * zz - xx - 3.0f * yy),
                  -6.0f * kC3zzz * y * z, -2.0f * kC3c * x * y, -2.0f * kC3zxx * y * z,
                  -6.0f * kC3a * x * y};
  float bz[15] = {0.0f, kC1, 0.0f, 0.0f, kC2xy * y, 6.0f * kC2zz * z, kC2xy * x, 0.0f, 0.0f,
                  kC3xyz * x * y, 8.0f * kC3c * y * z, 3.0f * kC3zzz * (2.0f * zz - xx - yy),
                  8.0f * kC3c * x * z, kC3zxx * (xx - yy), 0.0f};
  float in = d.inv_norm;
  float j00 = (1.0f - xx) * in, j01 = -xy * in, j02 = -xz * in;
  float j11 = (1.0f - yy) * in, j12 = -yz * in, j22 = (1.0f - zz) * in;
  // d/d(unnormalised direction) = J^T d/d(unit direction), J symmetric: sum
  // the basis derivatives weighted by s_k = sum_ch g_ch rest[k][ch] first,
  // then apply J once
  float tx = 0.f, ty = 0.f, tz = 0.f;
#pragma unroll
  for (int k = 0; k < 15; ++k) {
    const float sk = g0 * rest(k, 0) + g1 * rest(k, 1) + g2 * rest(k, 2);
    tx += sk * bx[k];
    ty += sk * by[k];
    tz += sk * bz[k];
  }
  return make_float3(j00 * tx + j01 * ty + j02 * tz, j01 * tx + j11 * ty + j12 * tz,
                     j02 * tx + j12 * ty + j22 * tz);
}

// The SH part of one view of the fused backward in one pass over the 45 rest
// coefficients: raw colour (for the clamp / sigmoid backward) and, per
// channel, the direction-derivative sums T[ch] = sum_k d basis_{k+1} / d dir
// * rest[k][ch]; then g (d loss / d raw colour) from the upstream colour
// gradient, and d loss / d mean through the normalised direction. Same
// quantities as the raw-colour loop plus sh_dir_backward (kernel.cu:619-782),
// with the channel sum taken last. Adds into gm and gdc; returns g in g[3].
template <typename RestAt>
__device__ __forceinline__ void sh_view_backward(const ViewDir &d, const float b[16],
                                                 const float dc[3], RestAt rest, float up_r,
                                                 float up_g, float up_b, int sh_sigmoid,
                                                 float g[3], float gm[3], float gdc[3]) {
  const float x = d.x, y = d.y, z = d.z;
  const float xx = x * x, yy = y * y, zz = z * z, xy = x * y, xz = x * z, yz = y * z;
  const float bx[15] = {0.0f, 0.0f, -kC1, kC2xy * y, 0.0f, 0.0f, kC2xy * z, 2.0f * kC2xxyy * x,
                        2.0f * kC3a * x * y, kC3xyz * y * z, -2.0f * kC3c * x * y,
                        -6.0f * kC3zzz * x * z, kC3c * (4.0f * zz - 3.0f * xx - yy),
                        2.0f * kC3zxx * x * z, 3.0f * kC3a * (xx - yy)};
  const float by[15] = {-kC1, 0.0f, 0.0f, kC2xy * x, kC2xy * z, 0.0f, 0.0f, -2.0f * kC2xxyy * y,
                        kC3a * (xx - 3.0f * yy), kC3xyz * x * z,
                        kC3c * (4.0f * zz - xx - 3.0f * yy), -6.0f * kC3zzz * y * z,
                        -2.0f * kC3c * x * y, -2.0f * kC3zxx * y * z, -6.0f * kC3a * x * y};
  const float bz[15] = {0.0f, kC1, 0.0f, 0.0f, kC2xy * y, 6.0f * kC2zz * z, kC2xy * x, 0.0f, 0.0f,
                        kC3xyz * x * y, 8.0f * kC3c * y * z,
                        3.0f * kC3zzz * (2.0f * zz - xx - yy), 8.0f * kC3c * x * z,
                        kC3zxx * (xx - yy), 0.0f};
  float raw[3], Tx[3], Ty[3], Tz[3];
#pragma unroll
  for (int ch = 0; ch < 3; ++ch) {
    raw[ch] = b[0] * dc[ch];
    Tx[ch] = Ty[ch] = Tz[ch] = 0.0f;
  }
#pragma unroll
  for (int k = 0; k < 15; ++k)
#pragma unroll
    for (int ch = 0; ch < 3; ++ch) {
      const float r = rest(k, ch);
      raw[ch] += b[k + 1] * r;
      Tx[ch] += bx[k] * r;
      Ty[ch] += by[k] * r;
      Tz[ch] += bz[k] * r;
    }
  const float up[3] = {up_r, up_g, up_b};
  float tx = 0.f, ty = 0.f, tz = 0.f;
#pragma unroll
  for (int ch = 0; ch < 3; ++ch) {
    float gc = up[ch];
    if (sh_sigmoid) {
      const float col = ref_sigmoid(raw[ch]);
      gc *= col * (1.0f - col);
    } else {
      gc = (raw[ch] + 0.5f >= 0.0f) ? gc : 0.0f;  // clamp_min backward passes where >= 0
    }
    g[ch] = gc;
    gdc[ch] += gc * b[0];
    tx += gc * Tx[ch];
    ty += gc * Ty[ch];
    tz += gc * Tz[ch];
  }
  const float in = d.inv_norm;
  const float j00 = (1.0f - xx) * in, j01 = -xy * in, j02 = -xz * in;
  const float j11 = (1.0f - yy) * in, j12 = -yz * in, j22 = (1.0f - zz) * in;
  gm[0] += j00 * tx + j01 * ty + j02 * tz;
  gm[1] += j01 * tx + j11 * ty + j12 * tz;
  gm[2] += j02 * tx + j12 * ty + j22 * tz;
}

// ---- blend order of the tiles ---------------------------------------------------

// Length class of a tile list for the blend order: exact below 8 entries,
// then 8 classes per power of two (the leading bit's position and the next
// three bits), at most 8 * 30 + 7.
constexpr int kOrderClasses = 256;

__device__ __forceinline__ int length_class(int len) {
  if (len < 8) return max(len, 0);
  const int e = 31 - __clz(len);  // >= 3
  return (e << 3) | ((len >> (e - 3)) & 7);
}

// One block writes the num_tiles tile indices into `order`, longest lists
// first: a counting sort by descending length class (tiles of one class in
// any order), with lanes of a warp that share a class adding once. len(tile)
// gives a tile's list length; s_count is kOrderClasses words of shared
// memory. Every thread of the block calls it (blockDim.x a multiple of 32).
template <typename LenF>
__device__ void tile_order_block(int num_tiles, LenF len, int32_t *__restrict__ order,
                                 uint32_t *s_count) {
  const int t = threadIdx.x, lane = t & 31, nt = blockDim.x;
  const uint32_t lt_mask = (1u << lane) - 1u;
  for (int c = t; c < kOrderClasses; c += nt) s_count[c] = 0u;
  __syncthreads();
  const int rounds = (num_tiles + nt - 1) / nt;  // block-uniform
  for (int r = 0; r < rounds; ++r) {
    const int tile = r * nt + t;
    const int c = tile < num_tiles ? kOrderClasses - 1 - length_class(len(tile)) : -1;
    const uint32_t peers = __match_any_sync(0xffffffffu, c);
    if (c >= 0 && (peers & lt_mask) == 0u) atomicAdd(&s_count[c], (uint32_t)__popc(peers));
  }
  __syncthreads();
  if (t < 32) {  // exclusive scan of the class counts by one warp, 8 per lane
    uint32_t v[kOrderClasses / 32], sum = 0;
#pragma unroll
    for (int i = 0; i < kOrderClasses / 32; ++i) {
      v[i] = s_count[t * (kOrderClasses / 32) + i];
      sum += v[i];
    }
    uint32_t incl = sum;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const uint32_t y = __shfl_up_sync(0xffffffffu, incl, o);
      if (t >= o) incl += y;
    }
    uint32_t run = incl - sum;
#pragma unroll
    for (int i = 0; i < kOrderClasses / 32; ++i) {
      s_count[t * (kOrderClasses / 32) + i] = run;
      run += v[i];
    }
  }
  __syncthreads();
  for (int r = 0; r < rounds; ++r) {
    const int tile = r * nt + t;
    const int c = tile < num_tiles ? kOrderClasses - 1 - length_class(len(tile)) : -1;
    const uint32_t peers = __match_any_sync(0xffffffffu, c);
    const int leader = __ffs(peers) - 1;
    uint32_t base = 0;
    if (c >= 0 && lane == leader) base = atomicAdd(&s_count[c], (uint32_t)__popc(peers));
    base = __shfl_sync(0xffffffffu, base, leader);
    if (c >= 0) order[base + __popc(peers & lt_mask)] = tile;
  }
}

// ---- tiles --------------------------------------------------------------------

// floorf followed by the float->int32 conversion (kernel.cu:804-807).
__device__ __forceinline__ int floor_i32(float f) { return (int32_t)floorf(f); }

struct TileRect {
  int x0, x1, y0, y1;  // inclusive tile coordinates
  bool empty;
};

// Tile rectangle of a Gaussian (kernel.cu:799-816).
__device__ __forceinline__ TileRect tile_rect(float u, float v, float ru, float rv, int width,
                                              int height) {
  int u0 = min(max(0, floor_i32(u - ru)), width - 1);
  int u1 = min(max(0, floor_i32(u + ru)), width - 1);
  int v0 = min(max(0, floor_i32(v - rv)), height - 1);
  int v1 = min(max(0, floor_i32(v + rv)), height - 1);
  TileRect t;
  t.empty = (u0 > u1 || v0 > v1);
  t.x0 = u0 / GS_TILE;
  t.x1 = u1 / GS_TILE;
  t.y0 = v0 / GS_TILE;
  t.y1 = v1 / GS_TILE;
  return t;
}

__host__ __device__ __forceinline__ int tiles_x_of(int width) { return (width + GS_TILE - 1) / GS_TILE; }
__host__ __device__ __forceinline__ int tiles_y_of(int height) { return (height + GS_TILE - 1) / GS_TILE; }

}  // namespace gs
