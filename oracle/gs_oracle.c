/*
 * gs_oracle.c -- CPU restatement of the reference rasterizer's algorithm.
 *
 * TEST INFRASTRUCTURE ONLY. This file is the parity checker for the CUDA
 * kernels in the package and the timed CPU baseline of bench.py. The shipped
 * package never links, loads or calls it; only tests/, bench.py (cpu_baseline
 * leg and --impl reference) and __graft_entry__.smoke() do.
 *
 * Every function restates, in plain sequential C with IEEE single precision
 * (compiled with -ffp-contract=off, so no fused multiply-add), the behaviour
 * of one reference kernel of ruguangyou/3dgs_from_scratch:
 *
 *   or_project_points            src/cuda/kernel.cu:411-500 (+ 27-155)
 *   or_project_points_backward   src/cuda/kernel.cu:502-543 (+ 157-409)
 *   or_sh_forward                src/cuda/kernel.cu:545-617
 *   or_sh_backward               src/cuda/kernel.cu:619-782
 *   or_count_tiles               src/cuda/kernel.cu:784-818
 *   or_tile_layout               src/cuda/kernel.cu:820-914 +
 *                                src/cuda/rasterizer.cpp:292-359 (stable sort)
 *   or_rasterize                 src/cuda/kernel.cu:916-987
 *   or_rasterize_backward        src/cuda/kernel.cu:989-1111
 *
 * Outputs are written only where the reference kernel writes; callers pass
 * zero-initialised outputs (mask initialised to 1), exactly as
 * src/cuda/rasterizer.cpp allocates them with torch::zeros / torch::ones.
 *
 * Parity of this restatement is pinned against the reference's own Python
 * checks (scripts/check_cuda_gradients.py: rasterize_reference,
 * build_reference_tile_layout and the Torch autograd references) through the
 * golden vectors in tests/golden/, and against the reference CUDA extension
 * itself on the GPU box.
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

#define LOW_PASS 0.3f          /* kernel.cu:23 */
#define FOV_CLAMP 1.3f         /* kernel.cu:24 */
#define T_EPS 1e-10f           /* kernel.cu:25 */

static const float C0 = 0.28209479177387814f;
static const float C1 = 0.4886025119029199f;
static const float C2a = 1.0925484305920792f;   /* xy, xz, yz */
static const float C2b = 0.31539156525252005f;  /* zz */
static const float C2c = 0.5462742152960396f;   /* xx - yy */
static const float C3a = 0.5900435899266435f;   /* y(xx-yy), x(xx-3yy) */
static const float C3b = 2.890611442640554f;    /* xyz */
static const float C3c = 0.4570457994644658f;   /* y(4zz-xx-yy), x(4zz-xx-yy) */
static const float C3d = 0.3731763325901154f;   /* z(2zz-3xx-3yy) */
static const float C3e = 1.445305721320277f;    /* z(xx-yy) */

int or_num_threads(void) {
#ifdef _OPENMP
    return omp_get_max_threads();
#else
    return 1;
#endif
}

void or_set_num_threads(int n) {
#ifdef _OPENMP
    if (n > 0) omp_set_num_threads(n);
#else
    (void)n;
#endif
}

/* Camera-space point: rows 0..2 of the row-major 4x4 world_to_camera. */
static void to_camera(const float *W, const float *p, float *c) {
    c[0] = W[0] * p[0] + W[1] * p[1] + W[2] * p[2] + W[3];
    c[1] = W[4] * p[0] + W[5] * p[1] + W[6] * p[2] + W[7];
    c[2] = W[8] * p[0] + W[9] * p[1] + W[10] * p[2] + W[11];
}

/* Rotation matrix of an (x, y, z, w) quaternion, row-major. */
static void quat_rot(const float *q, float *R) {
    float x = q[0], y = q[1], z = q[2], w = q[3];
    R[0] = 1 - 2 * y * y - 2 * z * z; R[1] = 2 * x * y - 2 * z * w; R[2] = 2 * x * z + 2 * y * w;
    R[3] = 2 * x * y + 2 * z * w; R[4] = 1 - 2 * x * x - 2 * z * z; R[5] = 2 * y * z - 2 * x * w;
    R[6] = 2 * x * z - 2 * y * w; R[7] = 2 * y * z + 2 * x * w; R[8] = 1 - 2 * x * x - 2 * y * y;
}

/* out = A * B^T where B is 3x3 given by rows of the 4x4 W (columns 0..2). */
static void mat3_mul_wT(const float *A, const float *W, float *out) {
    for (int i = 0; i < 3; ++i)
        for (int j = 0; j < 3; ++j)
            out[i * 3 + j] = A[i * 3] * W[j * 4] + A[i * 3 + 1] * W[j * 4 + 1] + A[i * 3 + 2] * W[j * 4 + 2];
}

/* out = W3 * A where W3 is the upper-left 3x3 of the 4x4 W. */
static void w_mul(const float *W, const float *A, float *out) {
    for (int i = 0; i < 3; ++i)
        for (int j = 0; j < 3; ++j)
            out[i * 3 + j] = W[i * 4] * A[j] + W[i * 4 + 1] * A[3 + j] + W[i * 4 + 2] * A[6 + j];
}

/* Projection Jacobian entries (J0, J2, J4, J5) with the 1.3x FOV clamp of
 * kernel.cu:117-127; also reports the clamp state and the ndc values. */
typedef struct {
    float J0, J2, J4, J5;
    float inv_z, x_ndc, y_ndc, xc, yc, lim_x, lim_y;
} Jac;

static Jac jacobian(const float *K, int width, int height, const float *pc) {
    Jac j;
    float fx = K[0], fy = K[4], cx = K[2], cy = K[5];
    j.lim_x = FOV_CLAMP * fmaxf(cx, (float)width - cx) / fx;
    j.lim_y = FOV_CLAMP * fmaxf(cy, (float)height - cy) / fy;
    j.inv_z = 1.0f / pc[2];
    j.x_ndc = pc[0] * j.inv_z;
    j.y_ndc = pc[1] * j.inv_z;
    j.xc = fminf(j.lim_x, fmaxf(-j.lim_x, j.x_ndc));
    j.yc = fminf(j.lim_y, fmaxf(-j.lim_y, j.y_ndc));
    j.J0 = fx * j.inv_z;
    j.J2 = -fx * j.xc * j.inv_z;
    j.J4 = fy * j.inv_z;
    j.J5 = -fy * j.yc * j.inv_z;
    return j;
}

/* Σ2D = J W R S² Rᵀ Wᵀ Jᵀ with the 0.3 low-pass and symmetrisation
 * (kernel.cu:46-155). */
static void image_cov(const float *W, const float *K, int width, int height,
                      const float *s, const float *q, const float *pc, float *cov) {
    float R[9], Cw[9], WC[9], Cc[9];
    quat_rot(q, R);
    float s2[3] = {s[0] * s[0], s[1] * s[1], s[2] * s[2]};
    for (int i = 0; i < 3; ++i)
        for (int k = 0; k < 3; ++k)
            Cw[i * 3 + k] = R[i * 3] * s2[0] * R[k * 3] + R[i * 3 + 1] * s2[1] * R[k * 3 + 1] +
                            R[i * 3 + 2] * s2[2] * R[k * 3 + 2];
    w_mul(W, Cw, WC);
    mat3_mul_wT(WC, W, Cc);
    Jac j = jacobian(K, width, height, pc);
    /* J Cc: rows (J0, 0, J2) and (0, J4, J5) */
    float A0 = j.J0 * Cc[0] + j.J2 * Cc[6];
    float A1 = j.J0 * Cc[1] + j.J2 * Cc[7];
    float A2 = j.J0 * Cc[2] + j.J2 * Cc[8];
    float B1 = j.J4 * Cc[4] + j.J5 * Cc[7];
    float B2 = j.J4 * Cc[5] + j.J5 * Cc[8];
    float B0 = j.J4 * Cc[3] + j.J5 * Cc[6];
    float c00 = A0 * j.J0 + A2 * j.J2;
    float c01 = A1 * j.J4 + A2 * j.J5;
    float c10 = B0 * j.J0 + B2 * j.J2;
    float c11 = B1 * j.J4 + B2 * j.J5;
    cov[0] = c00 + LOW_PASS;
    cov[1] = 0.5f * (c01 + c10);
    cov[2] = c11 + LOW_PASS;
}

void or_project_points(int N, const float *means, const float *scales, const float *quats,
                       const float *opac, const float *W, const float *K, float near_plane,
                       float far_plane, float min_opacity, float min_radius, float max_radius,
                       int width, int height, float *points, float *depths, float *cov,
                       float *conic, float *radii, uint8_t *mask) {
#pragma omp parallel for schedule(static)
    for (int i = 0; i < N; ++i) {
        if (opac[i] < min_opacity) { mask[i] = 0; continue; }
        float pc[3];
        to_camera(W, means + 3 * i, pc);
        if (pc[2] < near_plane || pc[2] > far_plane) { mask[i] = 0; continue; }
        float u = K[0] * pc[0] / pc[2] + K[2];
        float v = K[4] * pc[1] / pc[2] + K[5];
        float *c = cov + 3 * i;
        image_cov(W, K, width, height, scales + 3 * i, quats + 4 * i, pc, c);
        float det = c[0] * c[2] - c[1] * c[1];
        float inv_det = 1.0f / fmaxf(det, 1e-12f);
        float ru = fmaxf(sqrtf(c[0]), 1e-12f) * 3.0f;
        float rv = fmaxf(sqrtf(c[2]), 1e-12f) * 3.0f;
        float r = fmaxf(ru, rv);
        if (r < min_radius || r > max_radius) { mask[i] = 0; continue; }
        if (u < -ru || u > (float)width + ru || v < -rv || v > (float)height + rv) {
            mask[i] = 0;
            continue;
        }
        points[2 * i] = u;
        points[2 * i + 1] = v;
        depths[i] = pc[2];
        conic[3 * i] = c[2] * inv_det;
        conic[3 * i + 1] = -c[1] * inv_det;
        conic[3 * i + 2] = c[0] * inv_det;
        radii[2 * i] = ru;
        radii[2 * i + 1] = rv;
    }
}

/* Chain rule of kernel.cu:157-409 for one Gaussian: d(u,v) and d(conic)
 * back to d(mean), d(scale), d(quat). The off-diagonal conic gradient enters
 * the Jacobian path as the full g01 (kernel.cu:384-389), as the reference does. */
static void proj_backward_one(const float *pc, const float *W, const float *K, int width,
                              int height, const float *g_uv, const float *s, const float *q,
                              const float *cov, const float *g_conic, float *g_mean,
                              float *g_scale, float *g_quat) {
    float fx = K[0], fy = K[4];
    Jac j = jacobian(K, width, height, pc);
    float x = pc[0], y = pc[1], z = pc[2];
    float iz2 = j.inv_z * j.inv_z;
    float iz3 = iz2 * j.inv_z;
    int xcl = fabsf(j.x_ndc) > j.lim_x;
    int ycl = fabsf(j.y_ndc) > j.lim_y;
    float gu = g_uv[0], gv = g_uv[1];
    float gm0 = (gu * fx * (W[0] * z - W[8] * x) + gv * fy * (W[4] * z - W[8] * y)) * iz2;
    float gm1 = (gu * fx * (W[1] * z - W[9] * x) + gv * fy * (W[5] * z - W[9] * y)) * iz2;
    float gm2 = (-gu * fx * (W[10] * x - W[2] * z) - gv * fy * (W[10] * y - W[6] * z)) * iz2;

    /* U = J W3 (2x3) */
    float U[6];
    U[0] = j.J0 * W[0] + j.J2 * W[8];
    U[1] = j.J0 * W[1] + j.J2 * W[9];
    U[2] = j.J0 * W[2] + j.J2 * W[10];
    U[3] = j.J4 * W[4] + j.J5 * W[8];
    U[4] = j.J4 * W[5] + j.J5 * W[9];
    U[5] = j.J4 * W[6] + j.J5 * W[10];

    float R[9];
    quat_rot(q, R);
    float qi = q[0], qj = q[1], qk = q[2], qr = q[3];
    float sx = s[0], sy = s[1], sz = s[2];
    float M[9] = {R[0] * sx, R[1] * sy, R[2] * sz, R[3] * sx, R[4] * sy,
                  R[5] * sz, R[6] * sx, R[7] * sy, R[8] * sz};

    /* d(conic)/d(cov) (kernel.cu:295-313) */
    float a = cov[0], b = cov[1], c = cov[2];
    float det = a * c - b * b;
    float id = 1.0f / fmaxf(det, 1e-12f);
    float id2 = id * id;
    float D[3][3] = {{-c * c * id2, b * c * id2, -b * b * id2},
                     {2.0f * b * c * id2, -(a * c + b * b) * id2, 2.0f * a * b * id2},
                     {-b * b * id2, a * b * id2, -a * a * id2}};
    float gE2[3];
    for (int r = 0; r < 3; ++r) {
        gE2[r] = 0.0f;
        for (int k = 0; k < 3; ++k) gE2[r] += g_conic[k] * D[r][k];
    }

    /* d(Σ2D)/d(Σ3D) entries, row-major over the 3x3 Σ3D (kernel.cu:282-292,316-322) */
    float gE[9];
    for (int r = 0; r < 3; ++r)
        for (int k = 0; k < 3; ++k) {
            float t0 = U[r] * U[k];
            float t1 = U[r] * U[3 + k];
            float t2 = U[k] * U[3 + r];
            float t3 = U[3 + r] * U[3 + k];
            gE[r * 3 + k] = gE2[0] * t0 + 0.5f * gE2[1] * (t1 + t2) + gE2[2] * t3;
        }
    float gM[9];
    for (int r = 0; r < 3; ++r)
        for (int col = 0; col < 3; ++col) {
            float acc = 0.0f;
            for (int k = 0; k < 3; ++k) acc += (gE[r * 3 + k] + gE[k * 3 + r]) * M[k * 3 + col];
            gM[r * 3 + col] = acc;
        }
    g_scale[0] = gM[0] * R[0] + gM[3] * R[3] + gM[6] * R[6];
    g_scale[1] = gM[1] * R[1] + gM[4] * R[4] + gM[7] * R[7];
    g_scale[2] = gM[2] * R[2] + gM[5] * R[5] + gM[8] * R[8];

    /* dM/dq for (x, y, z, w) = (qi, qj, qk, qr) (kernel.cu:260-279) */
    float dqi[9] = {0.0f, 2.0f * sy * qj, 2.0f * sz * qk, 2.0f * sx * qj, -4.0f * sy * qi,
                    -2.0f * sz * qr, 2.0f * sx * qk, 2.0f * sy * qr, -4.0f * sz * qi};
    float dqj[9] = {-4.0f * sx * qj, 2.0f * sy * qi, 2.0f * sz * qr, 2.0f * sx * qi, 0.0f,
                    2.0f * sz * qk, -2.0f * sx * qr, 2.0f * sy * qk, -4.0f * sz * qj};
    float dqk[9] = {-4.0f * sx * qk, -2.0f * sy * qr, 2.0f * sz * qi, 2.0f * sx * qr,
                    -4.0f * sy * qk, 2.0f * sz * qj, 2.0f * sx * qi, 2.0f * sy * qj, 0.0f};
    float dqr[9] = {0.0f, -2.0f * sy * qk, 2.0f * sz * qj, 2.0f * sx * qk, 0.0f,
                    -2.0f * sz * qi, -2.0f * sx * qj, 2.0f * sy * qi, 0.0f};
    float q0 = 0.f, q1 = 0.f, q2 = 0.f, q3 = 0.f;
    for (int k = 0; k < 9; ++k) {
        q0 += gM[k] * dqi[k];
        q1 += gM[k] * dqj[k];
        q2 += gM[k] * dqk[k];
        q3 += gM[k] * dqr[k];
    }
    g_quat[0] = q0; g_quat[1] = q1; g_quat[2] = q2; g_quat[3] = q3;

    /* Camera covariance rebuilt from M (kernel.cu:347-379) */
    float E[9], WE[9], Cc[9];
    for (int r = 0; r < 3; ++r)
        for (int k = 0; k < 3; ++k)
            E[r * 3 + k] = M[r * 3] * M[k * 3] + M[r * 3 + 1] * M[k * 3 + 1] + M[r * 3 + 2] * M[k * 3 + 2];
    w_mul(W, E, WE);
    mat3_mul_wT(WE, W, Cc);

    float g00 = gE2[0], g01 = gE2[1], g11 = gE2[2];
    /* G J with J = [[J0,0,J2],[0,J4,J5]] */
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
    g_mean[0] = gm0 + (W[0] * gx + W[4] * gy + W[8] * gz);
    g_mean[1] = gm1 + (W[1] * gx + W[5] * gy + W[9] * gz);
    g_mean[2] = gm2 + (W[2] * gx + W[6] * gy + W[10] * gz);
}

void or_project_points_backward(int N, const float *g_points, const float *g_conic,
                                const float *means, const float *scales, const float *quats,
                                const float *W, const float *K, const float *cov,
                                const uint8_t *mask, int width, int height, float *g_means,
                                float *g_scales, float *g_quats) {
#pragma omp parallel for schedule(static)
    for (int i = 0; i < N; ++i) {
        if (!mask[i]) continue;
        float pc[3];
        to_camera(W, means + 3 * i, pc);
        proj_backward_one(pc, W, K, width, height, g_points + 2 * i, scales + 3 * i,
                          quats + 4 * i, cov + 3 * i, g_conic + 3 * i, g_means + 3 * i,
                          g_scales + 3 * i, g_quats + 4 * i);
    }
}

/* The 16 real SH basis values for a unit direction (kernel.cu:578-595). */
static void sh_basis(float x, float y, float z, float *b) {
    float xx = x * x, yy = y * y, zz = z * z, xy = x * y, xz = x * z, yz = y * z;
    b[0] = C0;
    b[1] = -C1 * y;
    b[2] = C1 * z;
    b[3] = -C1 * x;
    b[4] = C2a * xy;
    b[5] = C2a * yz;
    b[6] = C2b * (3 * zz - 1);
    b[7] = C2a * xz;
    b[8] = C2c * (xx - yy);
    b[9] = C3a * y * (xx - yy);
    b[10] = C3b * (x * y * z);
    b[11] = C3c * y * (4 * zz - xx - yy);
    b[12] = C3d * z * (2 * zz - 3 * xx - 3 * yy);
    b[13] = C3c * x * (4 * zz - xx - yy);
    b[14] = C3e * z * (xx - yy);
    b[15] = C3a * x * (xx - 3 * yy);
}

static void view_dir(const float *campos, const float *p, float *d, float *inv_norm) {
    float dx = p[0] - campos[0], dy = p[1] - campos[1], dz = p[2] - campos[2];
    float n = sqrtf(dx * dx + dy * dy + dz * dz);
    float in = 1.0f / (n + 1e-8f);
    d[0] = dx * in; d[1] = dy * in; d[2] = dz * in;
    *inv_norm = in;
}

void or_sh_forward(int N, const float *campos, const float *means, const float *dc,
                   const float *rest, const uint8_t *mask, int sh_sigmoid, float *colors) {
#pragma omp parallel for schedule(static)
    for (int i = 0; i < N; ++i) {
        if (!mask[i]) continue;
        float d[3], in, b[16];
        view_dir(campos, means + 3 * i, d, &in);
        sh_basis(d[0], d[1], d[2], b);
        float rgb[3];
        for (int c = 0; c < 3; ++c) {
            float acc = b[0] * dc[3 * i + c];
            for (int k = 0; k < 15; ++k) acc += b[k + 1] * rest[(i * 15 + k) * 3 + c];
            rgb[c] = acc;
        }
        for (int c = 0; c < 3; ++c)
            colors[3 * i + c] = sh_sigmoid ? (float)(1.0 / (1.0 + (double)expf(-rgb[c]))) : rgb[c];
    }
}

void or_sh_backward(int N, const float *g_colors, const float *campos, const float *means,
                    const float *rest, const float *colors, const uint8_t *mask, int sh_sigmoid,
                    float *g_means, float *g_dc, float *g_rest) {
#pragma omp parallel for schedule(static)
    for (int i = 0; i < N; ++i) {
        if (!mask[i]) continue;
        float d[3], in, b[16];
        view_dir(campos, means + 3 * i, d, &in);
        float x = d[0], y = d[1], z = d[2];
        sh_basis(x, y, z, b);
        float xx = x * x, yy = y * y, zz = z * z, xy = x * y, xz = x * z, yz = y * z;
        /* derivatives of bases 1..15 w.r.t. the unit direction (kernel.cu:675-725) */
        float bx[15] = {0.0f, 0.0f, -C1, C2a * y, 0.0f, 0.0f, C2a * z, 2.0f * C2c * x,
                        2.0f * C3a * x * y, C3b * y * z, -2.0f * C3c * x * y, -6.0f * C3d * x * z,
                        C3c * (4.0f * zz - 3.0f * xx - yy), 2.0f * C3e * x * z,
                        3.0f * C3a * (xx - yy)};
        float by[15] = {-C1, 0.0f, 0.0f, C2a * x, C2a * z, 0.0f, 0.0f, -2.0f * C2c * y,
                        C3a * (xx - 3.0f * yy), C3b * x * z, C3c * (4.0f * zz - xx - 3.0f * yy),
                        -6.0f * C3d * y * z, -2.0f * C3c * x * y, -2.0f * C3e * y * z,
                        -6.0f * C3a * x * y};
        float bz[15] = {0.0f, C1, 0.0f, 0.0f, C2a * y, 6.0f * C2b * z, C2a * x, 0.0f, 0.0f,
                        C3b * x * y, 8.0f * C3c * y * z, 3.0f * C3d * (2.0f * zz - xx - yy),
                        8.0f * C3c * x * z, C3e * (xx - yy), 0.0f};
        float j00 = (1.0f - xx) * in, j01 = -xy * in, j02 = -xz * in;
        float j11 = (1.0f - yy) * in, j12 = -yz * in, j22 = (1.0f - zz) * in;
        float g[3];
        for (int c = 0; c < 3; ++c) {
            g[c] = g_colors[3 * i + c];
            if (sh_sigmoid) g[c] *= colors[3 * i + c] * (1.0f - colors[3 * i + c]);
        }
        for (int c = 0; c < 3; ++c) g_dc[3 * i + c] = g[c] * b[0];
        for (int k = 0; k < 15; ++k)
            for (int c = 0; c < 3; ++c) g_rest[(i * 15 + k) * 3 + c] = g[c] * b[k + 1];
        float gx = 0.f, gy = 0.f, gz = 0.f;
        for (int k = 0; k < 15; ++k) {
            float px = bx[k] * j00 + by[k] * j01 + bz[k] * j02;
            float py = bx[k] * j01 + by[k] * j11 + bz[k] * j12;
            float pz = bx[k] * j02 + by[k] * j12 + bz[k] * j22;
            const float *r = rest + (i * 15 + k) * 3;
            gx += g[0] * r[0] * px + g[1] * r[1] * px + g[2] * r[2] * px;
            gy += g[0] * r[0] * py + g[1] * r[1] * py + g[2] * r[2] * py;
            gz += g[0] * r[0] * pz + g[1] * r[1] * pz + g[2] * r[2] * pz;
        }
        g_means[3 * i] = gx;
        g_means[3 * i + 1] = gy;
        g_means[3 * i + 2] = gz;
    }
}

/* floorf then a saturating float->int32 conversion (NaN -> 0), the
 * behaviour of CUDA's (int32_t) cast of an out-of-range float. */
static int32_t floor_to_i32(float f) {
    float x = floorf(f);
    if (x != x) return 0;
    if (x >= 2147483647.0f) return INT32_MAX;
    if (x <= -2147483648.0f) return INT32_MIN;
    return (int32_t)x;
}

static int imin(int a, int b) { return a < b ? a : b; }
static int imax(int a, int b) { return a > b ? a : b; }

/* Tile rectangle of a Gaussian (kernel.cu:799-816); returns 0 if empty. */
static int tile_rect(const float *pts, const float *radii, int width, int height, int tile,
                     int *tu0, int *tu1, int *tv0, int *tv1) {
    float u = pts[0], v = pts[1], ru = radii[0], rv = radii[1];
    int u0 = imin(imax(0, floor_to_i32(u - ru)), width - 1);
    int u1 = imin(imax(0, floor_to_i32(u + ru)), width - 1);
    int v0 = imin(imax(0, floor_to_i32(v - rv)), height - 1);
    int v1 = imin(imax(0, floor_to_i32(v + rv)), height - 1);
    if (u0 > u1 || v0 > v1) return 0;
    *tu0 = u0 / tile; *tu1 = u1 / tile; *tv0 = v0 / tile; *tv1 = v1 / tile;
    return 1;
}

void or_count_tiles(int N, const float *points, const float *radii, const uint8_t *mask,
                    int width, int height, int tile, int32_t *counts) {
#pragma omp parallel for schedule(static)
    for (int i = 0; i < N; ++i) {
        if (!mask[i]) continue;
        int a, b, c, d;
        if (!tile_rect(points + 2 * i, radii + 2 * i, width, height, tile, &a, &b, &c, &d)) {
            counts[i] = 0;
            continue;
        }
        counts[i] = (b - a + 1) * (d - c + 1);
    }
}

/* Stable LSD radix sort of (key, value) pairs by the low `bits` bits of key. */
static void radix_sort_pairs(int64_t n, uint64_t *keys, int32_t *vals, int bits) {
    if (n <= 1) return;
    uint64_t *k2 = (uint64_t *)malloc((size_t)n * sizeof(uint64_t));
    int32_t *v2 = (int32_t *)malloc((size_t)n * sizeof(int32_t));
    uint64_t *ka = keys, *kb = k2;
    int32_t *va = vals, *vb = v2;
    for (int shift = 0; shift < bits; shift += 8) {
        int64_t hist[257];
        memset(hist, 0, sizeof(hist));
        for (int64_t i = 0; i < n; ++i) hist[((ka[i] >> shift) & 0xFF) + 1]++;
        for (int d = 0; d < 256; ++d) hist[d + 1] += hist[d];
        for (int64_t i = 0; i < n; ++i) {
            int64_t pos = hist[(ka[i] >> shift) & 0xFF]++;
            kb[pos] = ka[i];
            vb[pos] = va[i];
        }
        uint64_t *tk = ka; ka = kb; kb = tk;
        int32_t *tv = va; va = vb; vb = tv;
    }
    if (ka != keys) {
        memcpy(keys, ka, (size_t)n * sizeof(uint64_t));
        memcpy(vals, va, (size_t)n * sizeof(int32_t));
    }
    free(k2);
    free(v2);
}

/* Duplicate (tile << 32 | depth bits, id) pairs in Gaussian order, tile
 * row-major (kernel.cu:820-873), stable-sort them over all significant key
 * bits (the CUB DeviceRadixSort::SortPairs call of kernel.cu:1341-1388), and
 * derive the per-tile start offsets (kernel.cu:875-914).
 * `offsets` has num_tiles entries and must be zero on entry; keys_out and
 * ids_out have `total` entries, the sum of or_count_tiles' counts. */
void or_tile_layout(int N, const float *points, const float *radii, const float *depths,
                    const uint8_t *mask, const int32_t *counts, int width, int height, int tile,
                    int64_t total, int64_t *keys_out, int32_t *ids_out, int32_t *offsets) {
    int tiles_x = (width + tile - 1) / tile;
    int tiles_y = (height + tile - 1) / tile;
    int num_tiles = tiles_x * tiles_y;
    int64_t pos = 0;
    for (int i = 0; i < N; ++i) {
        if (!mask[i] || counts[i] == 0) continue;
        int a, b, c, d;
        if (!tile_rect(points + 2 * i, radii + 2 * i, width, height, tile, &a, &b, &c, &d)) continue;
        uint32_t dbits;
        memcpy(&dbits, depths + i, 4);
        for (int tv = c; tv <= d; ++tv)
            for (int tu = a; tu <= b; ++tu) {
                uint64_t t = (uint64_t)(tv * tiles_x + tu);
                keys_out[pos] = (int64_t)((t << 32) | (uint64_t)dbits);
                ids_out[pos] = i;
                ++pos;
            }
    }
    int tile_bits = 0;
    while ((1 << tile_bits) < num_tiles) ++tile_bits;
    radix_sort_pairs(total, (uint64_t *)keys_out, ids_out, 32 + tile_bits);
    if (total == 0) return;
    int prev = -1;
    for (int64_t k = 0; k < total; ++k) {
        int t = (int)(keys_out[k] >> 32);
        if (t != prev) {
            for (int g = prev + 1; g <= t; ++g) offsets[g] = (int32_t)k;
            prev = t;
        }
    }
    for (int g = prev + 1; g < num_tiles; ++g) offsets[g] = (int32_t)total;
}

static void tile_range(const int32_t *offsets, int num_tiles, int64_t total, int t,
                       int64_t *start, int64_t *end) {
    *start = offsets[t];
    *end = (t + 1 < num_tiles) ? offsets[t + 1] : total;
}

/* Front-to-back blend, one pixel at a time (kernel.cu:916-987). */
void or_rasterize(const int32_t *offsets, int num_tiles, const int32_t *ids, int64_t total,
                  const float *points, const float *conic, const float *opac,
                  const float *colors, int width, int height, int tile, float alpha_thr,
                  float trans_thr, float chi_thr, float *image) {
    int tiles_x = (width + tile - 1) / tile;
#pragma omp parallel for schedule(dynamic, 4)
    for (int t = 0; t < num_tiles; ++t) {
        int64_t s, e;
        tile_range(offsets, num_tiles, total, t, &s, &e);
        int row = t / tiles_x, col = t % tiles_x;
        for (int p = 0; p < tile * tile; ++p) {
            int u = col * tile + p % tile, v = row * tile + p / tile;
            if (u >= width || v >= height) continue;
            float T = 1.0f, r = 0.f, g = 0.f, b = 0.f;
            for (int64_t k = s; k < e; ++k) {
                int id = ids[k];
                float du = (float)u - points[2 * id];
                float dv = (float)v - points[2 * id + 1];
                float A = conic[3 * id], B = conic[3 * id + 1], C = conic[3 * id + 2];
                float q = A * du * du + 2.0f * B * du * dv + C * dv * dv;
                if (q > chi_thr) continue;
                float alpha = expf(-0.5f * q) * opac[id];
                if (alpha < alpha_thr) continue;
                float w = alpha * T;
                r += w * colors[3 * id];
                g += w * colors[3 * id + 1];
                b += w * colors[3 * id + 2];
                T *= 1.0f - alpha + T_EPS;
                if (T < trans_thr) break;
            }
            float *o = image + 3 * ((int64_t)v * width + u);
            o[0] = r; o[1] = g; o[2] = b;
        }
    }
}

/* Back-to-front gradient of one tile's pixels (kernel.cu:1025-1110).
 * Gradients are accumulated per thread and summed in thread order. */
void or_rasterize_backward(const float *g_image, const int32_t *offsets, int num_tiles,
                           const int32_t *ids, int64_t total, int N, const float *points,
                           const float *conic, const float *opac, const float *colors,
                           int width, int height, int tile, float alpha_thr, float trans_thr,
                           float chi_thr, float *g_points, float *g_conic, float *g_opac,
                           float *g_colors) {
    int tiles_x = (width + tile - 1) / tile;
    int nt = or_num_threads();
    float *acc = (float *)calloc((size_t)nt * (size_t)N * 9, sizeof(float));
#pragma omp parallel
    {
        int tid = 0;
#ifdef _OPENMP
        tid = omp_get_thread_num();
#endif
        float *A9 = acc + (size_t)tid * (size_t)N * 9;
#pragma omp for schedule(dynamic, 4)
        for (int t = 0; t < num_tiles; ++t) {
            int64_t s, e;
            tile_range(offsets, num_tiles, total, t, &s, &e);
            int row = t / tiles_x, col = t % tiles_x;
            for (int p = 0; p < tile * tile; ++p) {
                int u = col * tile + p % tile, v = row * tile + p / tile;
                if (u >= width || v >= height) continue;
                const float *gp = g_image + 3 * ((int64_t)v * width + u);
                float gr = gp[0], gg = gp[1], gb = gp[2];
                if (gr == 0.0f && gg == 0.0f && gb == 0.0f) continue;
                float Tf = 1.0f;
                int64_t end = e;
                for (int64_t k = s; k < e; ++k) {
                    int id = ids[k];
                    float du = (float)u - points[2 * id];
                    float dv = (float)v - points[2 * id + 1];
                    float A = conic[3 * id], B = conic[3 * id + 1], C = conic[3 * id + 2];
                    float q = A * du * du + 2.0f * B * du * dv + C * dv * dv;
                    if (q > chi_thr) continue;
                    float alpha = expf(-0.5f * q) * opac[id];
                    if (alpha < alpha_thr) continue;
                    Tf *= 1.0f - alpha + T_EPS;
                    if (Tf < trans_thr) { end = k + 1; break; }
                }
                if (end == s) continue;
                float suffix = 0.0f, Ta = Tf;
                for (int64_t k = end - 1; k >= s; --k) {
                    int id = ids[k];
                    float du = (float)u - points[2 * id];
                    float dv = (float)v - points[2 * id + 1];
                    float A = conic[3 * id], B = conic[3 * id + 1], C = conic[3 * id + 2];
                    float q = A * du * du + 2.0f * B * du * dv + C * dv * dv;
                    if (q > chi_thr) continue;
                    float dens = expf(-0.5f * q);
                    float alpha = dens * opac[id];
                    if (alpha < alpha_thr) continue;
                    float oma = 1.0f - alpha + T_EPS;
                    float Tp = Ta / oma;
                    float w = alpha * Tp;
                    const float *c = colors + 3 * id;
                    float grgb = gr * c[0] + gg * c[1] + gb * c[2];
                    float ga = Tp * grgb - suffix / oma;
                    float gu = A * du + B * dv;
                    float gv = B * du + C * dv;
                    float *a9 = A9 + (size_t)id * 9;
                    a9[0] += gu * alpha * ga;
                    a9[1] += gv * alpha * ga;
                    a9[2] += -0.5f * du * du * alpha * ga;
                    a9[3] += -du * dv * alpha * ga;
                    a9[4] += -0.5f * dv * dv * alpha * ga;
                    a9[5] += dens * ga;
                    a9[6] += w * gr;
                    a9[7] += w * gg;
                    a9[8] += w * gb;
                    suffix += w * grgb;
                    Ta = Tp;
                }
            }
        }
    }
    for (int th = 0; th < nt; ++th) {
        const float *A9 = acc + (size_t)th * (size_t)N * 9;
        for (int i = 0; i < N; ++i) {
            const float *a = A9 + (size_t)i * 9;
            g_points[2 * i] += a[0];
            g_points[2 * i + 1] += a[1];
            g_conic[3 * i] += a[2];
            g_conic[3 * i + 1] += a[3];
            g_conic[3 * i + 2] += a[4];
            g_opac[i] += a[5];
            g_colors[3 * i] += a[6];
            g_colors[3 * i + 1] += a[7];
            g_colors[3 * i + 2] += a[8];
        }
    }
    free(acc);
}
