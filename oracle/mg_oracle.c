/*
 * CPU ORACLE -- test infrastructure only. Nothing in the product links, loads
 * or calls this file; tests/, __graft_entry__.smoke() and bench.py's CPU
 * baseline use it as the checker.
 *
 * A plain-C restatement of nandometzger/metal-gauss's training hot path as
 * its Metal kernels define it (the reference's own torch_ref.py is pure
 * PyTorch and does not cover the kernels' SnugBox extent, validity rule, exact
 * ellipse binning, stop index or reverse-walk backward). Each function cites
 * the reference lines it follows. Built with -ffp-contract=off so every fp32
 * expression is a fixed sequence of correctly rounded operations; the
 * projection and binning use the operation order documented in
 * metal_gauss_b200/csrc/exact_math.cuh so their results can be compared bit
 * for bit with the GPU.
 *
 * Parity of this restatement against the reference itself is pinned by
 * tests/test_oracle_golden.py against fixtures produced by the reference's
 * torch_ref.render/project, sh.eval_sh, metal_backend.build_tile_lists,
 * metal_backend.antialias_scale, ssim.ssim and selective_adam.SelectiveAdam
 * (tests/golden/make_golden.py).
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#include "../include/mg_b200.h"

#define SH_C0 0.28209479177387814f
#define SH_C1 0.4886025119029199f
#define SH_C2_0 1.0925484305920792f
#define SH_C2_1 -1.0925484305920792f
#define SH_C2_2 0.31539156525252005f
#define SH_C2_3 -1.0925484305920792f
#define SH_C2_4 0.5462742152960396f
#define SH_C3_0 -0.5900435899266435f
#define SH_C3_1 2.890611442640554f
#define SH_C3_2 -0.4570457994644658f
#define SH_C3_3 0.3731763325901154f
#define SH_C3_4 -0.4570457994644658f
#define SH_C3_5 1.445305721320277f
#define SH_C3_6 -0.5900435899266435f

static inline float clampf(float v, float lo, float hi) { return fminf(fmaxf(v, lo), hi); }
static inline float log_f32(float x) { return (float)log((double)x); }

/* Real SH basis, degrees 0-3 (metal_gauss/sh.py:24-62; preprocess.metal:56-78). */
static void sh_basis(int deg, float x, float y, float z, float* B) {
    B[0] = SH_C0;
    if (deg < 1) return;
    B[1] = (-SH_C1) * y;
    B[2] = SH_C1 * z;
    B[3] = (-SH_C1) * x;
    if (deg < 2) return;
    const float xx = x * x, yy = y * y, zz = z * z;
    B[4] = (SH_C2_0 * x) * y;
    B[5] = (SH_C2_1 * y) * z;
    B[6] = SH_C2_2 * (((2.0f * zz) - xx) - yy);
    B[7] = (SH_C2_3 * x) * z;
    B[8] = SH_C2_4 * (xx - yy);
    if (deg < 3) return;
    B[9] = (SH_C3_0 * y) * ((3.0f * xx) - yy);
    B[10] = ((SH_C3_1 * x) * y) * z;
    B[11] = (SH_C3_2 * y) * (((4.0f * zz) - xx) - yy);
    B[12] = (SH_C3_3 * z) * (((2.0f * zz) - (3.0f * xx)) - (3.0f * yy));
    B[13] = (SH_C3_4 * x) * (((4.0f * zz) - xx) - yy);
    B[14] = (SH_C3_5 * z) * (xx - yy);
    B[15] = (SH_C3_6 * x) * (xx - (3.0f * yy));
}

/* d B_b / d dir (preprocess.metal:80-101). */
static void sh_basis_grad(int b, float x, float y, float z, float* g) {
    const float xx = x * x, yy = y * y, zz = z * z;
    g[0] = g[1] = g[2] = 0.0f;
    switch (b) {
        case 1: g[1] = -SH_C1; break;
        case 2: g[2] = SH_C1; break;
        case 3: g[0] = -SH_C1; break;
        case 4: g[0] = SH_C2_0 * y; g[1] = SH_C2_0 * x; break;
        case 5: g[1] = SH_C2_1 * z; g[2] = SH_C2_1 * y; break;
        case 6: g[0] = SH_C2_2 * (-2.f * x); g[1] = SH_C2_2 * (-2.f * y); g[2] = SH_C2_2 * (4.f * z); break;
        case 7: g[0] = SH_C2_3 * z; g[2] = SH_C2_3 * x; break;
        case 8: g[0] = SH_C2_4 * (2.f * x); g[1] = SH_C2_4 * (-2.f * y); break;
        case 9: g[0] = SH_C3_0 * (6.f * x * y); g[1] = SH_C3_0 * (3.f * xx - 3.f * yy); break;
        case 10: g[0] = SH_C3_1 * (y * z); g[1] = SH_C3_1 * (x * z); g[2] = SH_C3_1 * (x * y); break;
        case 11: g[0] = SH_C3_2 * (-2.f * x * y); g[1] = SH_C3_2 * (4.f * zz - xx - 3.f * yy); g[2] = SH_C3_2 * (8.f * y * z); break;
        case 12: g[0] = SH_C3_3 * (-6.f * x * z); g[1] = SH_C3_3 * (-6.f * y * z); g[2] = SH_C3_3 * (6.f * zz - 3.f * xx - 3.f * yy); break;
        case 13: g[0] = SH_C3_4 * (4.f * zz - 3.f * xx - yy); g[1] = SH_C3_4 * (-2.f * x * y); g[2] = SH_C3_4 * (8.f * x * z); break;
        case 14: g[0] = SH_C3_5 * (2.f * x * z); g[1] = SH_C3_5 * (-2.f * y * z); g[2] = SH_C3_5 * (xx - yy); break;
        case 15: g[0] = SH_C3_6 * (3.f * xx - 3.f * yy); g[1] = SH_C3_6 * (-6.f * x * y); break;
        default: break;
    }
}

static inline const float* sh_row(const float* dc, const float* rest, mg_sh_layout L,
                                  int64_t g, int i) {
    return i == 0 ? dc + g * L.stride_dc * 3
                  : rest + (g * L.stride_rest + L.offset_rest + (i - 1)) * 3;
}
static inline float* sh_row_w(float* dc, float* rest, mg_sh_layout L, int64_t g, int i) {
    return i == 0 ? dc + g * L.stride_dc * 3
                  : rest + (g * L.stride_rest + L.offset_rest + (i - 1)) * 3;
}

/* ------------------------------------------------------------------------ */
/* preprocess_forward (preprocess.metal:114-221)                            */
/* ------------------------------------------------------------------------ */
void mgo_preprocess_forward(const float* means, const float* quats, const float* scales,
                            const float* sh_dc, const float* sh_rest, mg_sh_layout shl,
                            const float* opacities, const mg_camera* cam, int sh_degree,
                            int64_t n, float* out_uv, float* out_conic, float* out_depth,
                            float* out_rxy, int32_t* out_valid, float* out_color) {
    const float* V = cam->viewmat;
    const float fx = cam->fx, fy = cam->fy, cx = cam->cx, cy = cam->cy;
    const int W = cam->width, H = cam->height;
#pragma omp parallel for schedule(static)
    for (int64_t g = 0; g < n; ++g) {
        const float mx = means[3 * g], my = means[3 * g + 1], mz = means[3 * g + 2];
        const float pcx = ((V[0] * mx + V[1] * my) + V[2] * mz) + V[3];
        const float pcy = ((V[4] * mx + V[5] * my) + V[6] * mz) + V[7];
        const float pcz = ((V[8] * mx + V[9] * my) + V[10] * mz) + V[11];
        const float z = pcz;
        const float zc = fmaxf(z, cam->near_plane);
        const float u = ((fx * pcx) / zc) + cx;
        const float v = ((fy * pcy) / zc) + cy;
        /* Jacobian evaluated at a point clamped to 1.3x the half-FOV
           (preprocess.metal:147-151; torch_ref.py:86-89). */
        const float lim_x = 1.3f * ((0.5f * (float)W) / fx);
        const float lim_y = 1.3f * ((0.5f * (float)H) / fy);
        const float tx = clampf(pcx / zc, -lim_x, lim_x) * zc;
        const float ty = clampf(pcy / zc, -lim_y, lim_y) * zc;

        const float qw0 = quats[4 * g], qx0 = quats[4 * g + 1], qy0 = quats[4 * g + 2],
                    qz0 = quats[4 * g + 3];
        const float qn = sqrtf(((qw0 * qw0 + qx0 * qx0) + qy0 * qy0) + qz0 * qz0);
        const float qd = fmaxf(qn, 1e-12f);
        const float w = qw0 / qd, x = qx0 / qd, y = qy0 / qd, zq = qz0 / qd;
        /* R(q) as torch_ref.quat_to_rotmat (torch_ref.py:31-39). */
        const float R00 = 1.0f - 2.0f * ((y * y) + (zq * zq));
        const float R01 = 2.0f * ((x * y) - (w * zq));
        const float R02 = 2.0f * ((x * zq) + (w * y));
        const float R10 = 2.0f * ((x * y) + (w * zq));
        const float R11 = 1.0f - 2.0f * ((x * x) + (zq * zq));
        const float R12 = 2.0f * ((y * zq) - (w * x));
        const float R20 = 2.0f * ((x * zq) - (w * y));
        const float R21 = 2.0f * ((y * zq) + (w * x));
        const float R22 = 1.0f - 2.0f * ((x * x) + (y * y));
        const float sx = scales[3 * g], sy = scales[3 * g + 1], sz = scales[3 * g + 2];
        /* Sigma = M M^T with M = R diag(s) (torch_ref.py:42-46). */
        const float M00 = R00 * sx, M01 = R01 * sy, M02 = R02 * sz;
        const float M10 = R10 * sx, M11 = R11 * sy, M12 = R12 * sz;
        const float M20 = R20 * sx, M21 = R21 * sy, M22 = R22 * sz;
        const float S00 = (M00 * M00 + M01 * M01) + M02 * M02;
        const float S01 = (M00 * M10 + M01 * M11) + M02 * M12;
        const float S02 = (M00 * M20 + M01 * M21) + M02 * M22;
        const float S11 = (M10 * M10 + M11 * M11) + M12 * M12;
        const float S12 = (M10 * M20 + M11 * M21) + M12 * M22;
        const float S22 = (M20 * M20 + M21 * M21) + M22 * M22;
        /* EWA: cov2d = T Sigma T^T, T = J R_w2c (torch_ref.py:92-100). */
        const float izc = 1.0f / zc, izc2 = izc * izc;
        const float J0x = fx * izc, J0z = ((-fx) * tx) * izc2;
        const float J1y = fy * izc, J1z = ((-fy) * ty) * izc2;
        const float T00 = (J0x * V[0] + 0.0f * V[4]) + J0z * V[8];
        const float T01 = (J0x * V[1] + 0.0f * V[5]) + J0z * V[9];
        const float T02 = (J0x * V[2] + 0.0f * V[6]) + J0z * V[10];
        const float T10 = (0.0f * V[0] + J1y * V[4]) + J1z * V[8];
        const float T11 = (0.0f * V[1] + J1y * V[5]) + J1z * V[9];
        const float T12 = (0.0f * V[2] + J1y * V[6]) + J1z * V[10];
        const float ST00 = (S00 * T00 + S01 * T01) + S02 * T02;
        const float ST01 = (S01 * T00 + S11 * T01) + S12 * T02;
        const float ST02 = (S02 * T00 + S12 * T01) + S22 * T02;
        const float ST10 = (S00 * T10 + S01 * T11) + S02 * T12;
        const float ST11 = (S01 * T10 + S11 * T11) + S12 * T12;
        const float ST12 = (S02 * T10 + S12 * T11) + S22 * T12;
        /* + blur on the diagonal (torch_ref.py:124) */
        const float a = ((T00 * ST00 + T01 * ST01) + T02 * ST02) + cam->blur;
        const float b = (T00 * ST10 + T01 * ST11) + T02 * ST12;
        const float c = ((T10 * ST10 + T11 * ST11) + T12 * ST12) + cam->blur;
        const float det = (a * c) - (b * b);
        const float dets = fmaxf(det, 1e-12f);
        /* 3-sigma radius from the larger eigenvalue (torch_ref.py:136-139). */
        const float mid = 0.5f * (a + c);
        const float disc = sqrtf(fmaxf((mid * mid) - dets, 0.0f));
        const float lam = fmaxf(mid + disc, 1e-12f);
        const float radius = 3.0f * sqrtf(lam);
        /* SnugBox: exact extent of the alpha = 1/255 level set
           (preprocess.metal:180-191). */
        const float twoL = 2.0f * log_f32(fmaxf(255.0f * opacities[g], 1.0f));
        const float rs = sqrtf(twoL);
        const float rx = fminf(rs * sqrtf(fmaxf(a, 0.0f)), radius);
        const float ry = fminf(rs * sqrtf(fmaxf(c, 0.0f)), radius);
        const int ok = (z > cam->near_plane) && (z < cam->far_plane) && (det > 1e-12f) &&
                       (radius < cam->max_radius) && (rx > 0.0f) && (ry > 0.0f) &&
                       (u + rx > 0.0f) && (u - rx < (float)W) && (v + ry > 0.0f) &&
                       (v - ry < (float)H);
        out_uv[2 * g] = u; out_uv[2 * g + 1] = v;
        out_conic[3 * g] = c / dets;
        out_conic[3 * g + 1] = (-b) / dets;
        out_conic[3 * g + 2] = a / dets;
        out_depth[g] = z;
        out_rxy[2 * g] = rx; out_rxy[2 * g + 1] = ry;
        out_valid[g] = ok ? 1 : 0;
        if (sh_degree < 0 || sh_dc == NULL) continue;
        /* Visibility-gated SH (preprocess.metal:203-220). */
        if (!ok) {
            out_color[3 * g] = out_color[3 * g + 1] = out_color[3 * g + 2] = 0.0f;
            continue;
        }
        const float dvx = mx - cam->cam_center[0], dvy = my - cam->cam_center[1],
                    dvz = mz - cam->cam_center[2];
        const float len = sqrtf((dvx * dvx + dvy * dvy) + dvz * dvz);
        const float invn = 1.0f / fmaxf(len, 1e-12f);
        float B[16];
        sh_basis(sh_degree, dvx * invn, dvy * invn, dvz * invn, B);
        const int nb = (sh_degree + 1) * (sh_degree + 1);
        float r = 0.0f, gg = 0.0f, bb = 0.0f;
        for (int i = 0; i < nb; ++i) {
            const float* row = sh_row(sh_dc, sh_rest, shl, g, i);
            r = r + B[i] * row[0];
            gg = gg + B[i] * row[1];
            bb = bb + B[i] * row[2];
        }
        r = r + 0.5f; gg = gg + 0.5f; bb = bb + 0.5f;
        out_color[3 * g] = fmaxf(r, 0.0f);
        out_color[3 * g + 1] = fmaxf(gg, 0.0f);
        out_color[3 * g + 2] = fmaxf(bb, 0.0f);
    }
}

/* ------------------------------------------------------------------------ */
/* preprocess_backward (preprocess.metal:223-411)                           */
/* ------------------------------------------------------------------------ */
void mgo_preprocess_backward(const float* means, const float* quats, const float* scales,
                             const float* sh_dc, const float* sh_rest, mg_sh_layout shl,
                             const float* d_uv, int64_t d_uv_stride, const float* d_conic,
                             int64_t d_conic_stride, const float* d_color,
                             int64_t d_color_stride, const int32_t* valid,
                             const mg_camera* cam, int sh_degree, int64_t n, float* d_means,
                             float* d_quats, float* d_scales, float* d_sh_dc,
                             float* d_sh_rest) {
    const float* V = cam->viewmat;
    const float fx = cam->fx, fy = cam->fy;
#pragma omp parallel for schedule(static)
    for (int64_t g = 0; g < n; ++g) {
        const float mx = means[3 * g], my = means[3 * g + 1], mz = means[3 * g + 2];
        float dm[3] = {0.f, 0.f, 0.f};
        if (sh_degree >= 0 && d_color != NULL && sh_dc != NULL) {
            const float* dcol = d_color + g * d_color_stride;
            const int nb = (sh_degree + 1) * (sh_degree + 1);
            if (dcol[0] == 0.f && dcol[1] == 0.f && dcol[2] == 0.f) {
                for (int i = 0; i < 16; ++i) {
                    float* r = sh_row_w(d_sh_dc, d_sh_rest, shl, g, i);
                    r[0] = r[1] = r[2] = 0.f;
                }
            } else {
                const float dvx = mx - cam->cam_center[0], dvy = my - cam->cam_center[1],
                            dvz = mz - cam->cam_center[2];
                const float len = fmaxf(sqrtf(dvx * dvx + dvy * dvy + dvz * dvz), 1e-12f);
                const float dir[3] = {dvx / len, dvy / len, dvz / len};
                float B[16];
                sh_basis(sh_degree, dir[0], dir[1], dir[2], B);
                float pre[3] = {0.f, 0.f, 0.f};
                for (int i = 0; i < nb; ++i) {
                    const float* row = sh_row(sh_dc, sh_rest, shl, g, i);
                    for (int k = 0; k < 3; ++k) pre[k] += B[i] * row[k];
                }
                float dpre[3];
                for (int k = 0; k < 3; ++k) dpre[k] = (pre[k] + 0.5f > 0.f) ? dcol[k] : 0.f;
                float ddir[3] = {0.f, 0.f, 0.f};
                for (int i = 0; i < nb; ++i) {
                    const float* row = sh_row(sh_dc, sh_rest, shl, g, i);
                    const float k = row[0] * dpre[0] + row[1] * dpre[1] + row[2] * dpre[2];
                    float gb[3];
                    sh_basis_grad(i, dir[0], dir[1], dir[2], gb);
                    for (int q = 0; q < 3; ++q) ddir[q] += gb[q] * k;
                    float* w = sh_row_w(d_sh_dc, d_sh_rest, shl, g, i);
                    for (int q = 0; q < 3; ++q) w[q] = B[i] * dpre[q];
                }
                for (int i = nb; i < 16; ++i) {
                    float* w = sh_row_w(d_sh_dc, d_sh_rest, shl, g, i);
                    w[0] = w[1] = w[2] = 0.f;
                }
                const float dd = dir[0] * ddir[0] + dir[1] * ddir[1] + dir[2] * ddir[2];
                for (int q = 0; q < 3; ++q) dm[q] += (ddir[q] - dir[q] * dd) / len;
            }
        }
        if (valid[g] != 0) {
            const float pc[3] = {V[0] * mx + V[1] * my + V[2] * mz + V[3],
                                 V[4] * mx + V[5] * my + V[6] * mz + V[7],
                                 V[8] * mx + V[9] * my + V[10] * mz + V[11]};
            const float z = pc[2], zc = fmaxf(z, cam->near_plane);
            const float izc = 1.0f / zc, izc2 = izc * izc;
            const float lim_x = 1.3f * (0.5f * (float)cam->width / fx);
            const float lim_y = 1.3f * (0.5f * (float)cam->height / fy);
            const float txn = pc[0] / zc, tyn = pc[1] / zc;
            const int clx = (txn < -lim_x) || (txn > lim_x);
            const int cly = (tyn < -lim_y) || (tyn > lim_y);
            const float tx = clampf(txn, -lim_x, lim_x) * zc;
            const float ty = clampf(tyn, -lim_y, lim_y) * zc;
            const float* q0 = quats + 4 * g;
            const float qn = sqrtf(q0[0] * q0[0] + q0[1] * q0[1] + q0[2] * q0[2] + q0[3] * q0[3]);
            const float qd = fmaxf(qn, 1e-12f);
            const float w = q0[0] / qd, x = q0[1] / qd, y = q0[2] / qd, zq = q0[3] / qd;
            const float R[3][3] = {
                {1.f - 2.f * (y * y + zq * zq), 2.f * (x * y - w * zq), 2.f * (x * zq + w * y)},
                {2.f * (x * y + w * zq), 1.f - 2.f * (x * x + zq * zq), 2.f * (y * zq - w * x)},
                {2.f * (x * zq - w * y), 2.f * (y * zq + w * x), 1.f - 2.f * (x * x + y * y)}};
            const float s[3] = {scales[3 * g], scales[3 * g + 1], scales[3 * g + 2]};
            float M[3][3], S[3][3];
            for (int i = 0; i < 3; ++i)
                for (int j = 0; j < 3; ++j) M[i][j] = R[i][j] * s[j];
            for (int i = 0; i < 3; ++i)
                for (int j = 0; j < 3; ++j)
                    S[i][j] = M[i][0] * M[j][0] + M[i][1] * M[j][1] + M[i][2] * M[j][2];
            const float Rw[3][3] = {{V[0], V[1], V[2]}, {V[4], V[5], V[6]}, {V[8], V[9], V[10]}};
            const float J0x = fx * izc, J0z = -fx * tx * izc2;
            const float J1y = fy * izc, J1z = -fy * ty * izc2;
            float T0[3], T1[3], ST0[3], ST1[3];
            for (int k = 0; k < 3; ++k) {
                T0[k] = J0x * Rw[0][k] + J0z * Rw[2][k];
                T1[k] = J1y * Rw[1][k] + J1z * Rw[2][k];
            }
            for (int i = 0; i < 3; ++i) {
                ST0[i] = S[i][0] * T0[0] + S[i][1] * T0[1] + S[i][2] * T0[2];
                ST1[i] = S[i][0] * T1[0] + S[i][1] * T1[1] + S[i][2] * T1[2];
            }
            const float a = T0[0] * ST0[0] + T0[1] * ST0[1] + T0[2] * ST0[2] + cam->blur;
            const float b = T0[0] * ST1[0] + T0[1] * ST1[1] + T0[2] * ST1[2];
            const float c = T1[0] * ST1[0] + T1[1] * ST1[1] + T1[2] * ST1[2] + cam->blur;
            const float det = a * c - b * b;
            const float id = 1.0f / fmaxf(det, 1e-12f);
            const float* dcn = d_conic + g * d_conic_stride;
            /* conic = (c, -b, a) / det (preprocess.metal:308-317) */
            const float ddet = -(dcn[0] * c - dcn[1] * b + dcn[2] * a) * id * id;
            float da = dcn[2] * id + ddet * c;
            float db = -dcn[1] * id - 2.0f * ddet * b;
            float dc = dcn[0] * id + ddet * a;
            if (det <= 1e-12f) da = db = dc = 0.f;
            float dS[3][3], dT0[3], dT1[3], dJ0[3], dJ1[3];
            for (int i = 0; i < 3; ++i)
                for (int j = 0; j < 3; ++j)
                    dS[i][j] = da * T0[i] * T0[j] + db * T0[i] * T1[j] + dc * T1[i] * T1[j];
            for (int k = 0; k < 3; ++k) {
                dT0[k] = 2.0f * (da * ST0[k]) + db * ST1[k];
                dT1[k] = 2.0f * (dc * ST1[k]) + db * ST0[k];
            }
            for (int r = 0; r < 3; ++r) {
                dJ0[r] = dT0[0] * Rw[r][0] + dT0[1] * Rw[r][1] + dT0[2] * Rw[r][2];
                dJ1[r] = dT1[0] * Rw[r][0] + dT1[1] * Rw[r][1] + dT1[2] * Rw[r][2];
            }
            const float dtx = -fx * izc2 * dJ0[2];
            const float dty = -fy * izc2 * dJ1[2];
            float dzc = -fx * izc2 * dJ0[0] - fy * izc2 * dJ1[1] +
                        2.0f * fx * tx * izc2 * izc * dJ0[2] + 2.0f * fy * ty * izc2 * izc * dJ1[2];
            const float* duv = d_uv + g * d_uv_stride;
            float dpx = fx * izc * duv[0];
            float dpy = fy * izc * duv[1];
            dzc += -fx * pc[0] * izc2 * duv[0] - fy * pc[1] * izc2 * duv[1];
            /* tx = clamp(px/zc) zc routes to px unclamped, to zc clamped
               (preprocess.metal:363-369) */
            if (!clx) dpx += dtx; else dzc += dtx * (tx * izc);
            if (!cly) dpy += dty; else dzc += dty * (ty * izc);
            const float dpz = (z > cam->near_plane) ? dzc : 0.0f;
            for (int k = 0; k < 3; ++k) dm[k] += Rw[0][k] * dpx + Rw[1][k] * dpy + Rw[2][k] * dpz;
            float dM[3][3];
            for (int i = 0; i < 3; ++i)
                for (int j = 0; j < 3; ++j) {
                    float acc = 0.f;
                    for (int k = 0; k < 3; ++k) acc += 0.5f * (dS[i][k] + dS[k][i]) * M[k][j];
                    dM[i][j] = 2.0f * acc;
                }
            for (int j = 0; j < 3; ++j)
                d_scales[3 * g + j] = dM[0][j] * R[0][j] + dM[1][j] * R[1][j] + dM[2][j] * R[2][j];
            float G[3][3];
            for (int i = 0; i < 3; ++i)
                for (int j = 0; j < 3; ++j) G[i][j] = dM[i][j] * s[j];
            /* VJP of R(q) then of the normalisation (preprocess.metal:384-404) */
            const float dw = 2.f * (x * (G[2][1] - G[1][2]) + y * (G[0][2] - G[2][0]) + zq * (G[1][0] - G[0][1]));
            const float dqx = 2.f * (w * (G[2][1] - G[1][2]) + y * (G[1][0] + G[0][1]) + zq * (G[2][0] + G[0][2]) - 2.f * x * (G[1][1] + G[2][2]));
            const float dqy = 2.f * (w * (G[0][2] - G[2][0]) + x * (G[1][0] + G[0][1]) + zq * (G[2][1] + G[1][2]) - 2.f * y * (G[0][0] + G[2][2]));
            const float dqz = 2.f * (w * (G[1][0] - G[0][1]) + x * (G[2][0] + G[0][2]) + y * (G[2][1] + G[1][2]) - 2.f * zq * (G[0][0] + G[1][1]));
            const float qdot = w * dw + x * dqx + y * dqy + zq * dqz;
            d_quats[4 * g] = (dw - w * qdot) / qd;
            d_quats[4 * g + 1] = (dqx - x * qdot) / qd;
            d_quats[4 * g + 2] = (dqy - y * qdot) / qd;
            d_quats[4 * g + 3] = (dqz - zq * qdot) / qd;
        } else {
            d_scales[3 * g] = d_scales[3 * g + 1] = d_scales[3 * g + 2] = 0.f;
            d_quats[4 * g] = d_quats[4 * g + 1] = d_quats[4 * g + 2] = d_quats[4 * g + 3] = 0.f;
        }
        d_means[3 * g] = dm[0];
        d_means[3 * g + 1] = dm[1];
        d_means[3 * g + 2] = dm[2];
    }
}

/* ------------------------------------------------------------------------ */
/* Binning (binning.metal:25-120; metal_backend.py:217-285)                 */
/* ------------------------------------------------------------------------ */
static float min_q_over_rect(float mux, float muy, float ca, float cb, float ccz, float x0,
                             float x1, float y0, float y1) {
    if (mux >= x0 && mux <= x1 && muy >= y0 && muy <= y1) return 0.0f;
    const float a = fmaxf(ca, 1e-12f), b = cb, cc = fmaxf(ccz, 1e-12f);
    float best = INFINITY;
    for (int e = 0; e < 2; ++e) {
        const float yc = e == 0 ? y0 : y1;
        const float xs = clampf(mux - ((b * (yc - muy)) / a), x0, x1);
        const float ex = xs - mux, ey = yc - muy;
        best = fminf(best, (((a * ex) * ex) + (((2.0f * b) * ex) * ey)) + ((cc * ey) * ey));
    }
    for (int e = 0; e < 2; ++e) {
        const float xc = e == 0 ? x0 : x1;
        const float ys = clampf(muy - ((b * (xc - mux)) / cc), y0, y1);
        const float ex = xc - mux, ey = ys - muy;
        best = fminf(best, (((a * ex) * ex) + (((2.0f * b) * ex) * ey)) + ((cc * ey) * ey));
    }
    return best;
}

static int clampi(int v, int lo, int hi) { return v < lo ? lo : (v > hi ? hi : v); }

/* Counts (keys == NULL) or writes the Gaussian's surviving tiles row-major. */
static int64_t bin_walk(int64_t g, const float* uv, const float* rxy, const float* conic,
                        const float* opacity, const float* depth, int W, int H, int tile,
                        int tiles_x, int tiles_y, uint64_t* keys, int32_t* ids,
                        int64_t write_at) {
    const float mux = uv[2 * g], muy = uv[2 * g + 1], rx = rxy[2 * g], ry = rxy[2 * g + 1];
    const float tf = (float)tile;
    const int x0 = clampi((int)floorf((mux - rx) / tf), 0, tiles_x - 1);
    const int x1 = clampi((int)floorf((mux + rx) / tf), 0, tiles_x - 1);
    const int y0 = clampi((int)floorf((muy - ry) / tf), 0, tiles_y - 1);
    const int y1 = clampi((int)floorf((muy + ry) / tf), 0, tiles_y - 1);
    const float oa = 255.0f * opacity[g];
    if (oa <= 1.0f) return 0;
    const float thr = 2.0f * log_f32(oa);
    uint32_t dbits = 0;
    if (keys) memcpy(&dbits, depth + g, 4);
    int64_t cnt = 0;
    for (int ty = y0; ty <= y1; ++ty) {
        const float ry0 = (float)(ty * tile);
        const float ry1 = fminf((float)((ty + 1) * tile), (float)H);
        for (int tx = x0; tx <= x1; ++tx) {
            const float rx0 = (float)(tx * tile);
            const float rx1 = fminf((float)((tx + 1) * tile), (float)W);
            if (min_q_over_rect(mux, muy, conic[3 * g], conic[3 * g + 1], conic[3 * g + 2], rx0,
                                rx1, ry0, ry1) >= thr)
                continue;
            if (keys) {
                keys[write_at + cnt] = ((uint64_t)(uint32_t)(ty * tiles_x + tx) << 32) | dbits;
                ids[write_at + cnt] = (int32_t)g;
            }
            ++cnt;
        }
    }
    return cnt;
}

void mgo_bin_count(const float* uv, const float* rxy, const float* conic, const float* opacity,
                   const int32_t* valid, int64_t n, int W, int H, int tile, int tiles_x,
                   int tiles_y, int32_t* counts) {
#pragma omp parallel for schedule(static)
    for (int64_t g = 0; g < n; ++g)
        counts[g] = valid[g] ? (int32_t)bin_walk(g, uv, rxy, conic, opacity, NULL, W, H, tile,
                                                 tiles_x, tiles_y, NULL, NULL, 0)
                             : 0;
}

void mgo_bin_write(const float* uv, const float* rxy, const float* conic, const float* opacity,
                   const int32_t* valid, const float* depth, const int64_t* offsets, int64_t n,
                   int W, int H, int tile, int tiles_x, int tiles_y, uint64_t* keys,
                   int32_t* ids) {
#pragma omp parallel for schedule(static)
    for (int64_t g = 0; g < n; ++g)
        if (valid[g])
            bin_walk(g, uv, rxy, conic, opacity, depth, W, H, tile, tiles_x, tiles_y, keys, ids,
                     offsets[g]);
}

/* Stable LSD radix sort of (key, id) on the low `bits` bits, 8 bits a pass:
   the order torch.argsort(keys, stable=True) gives (metal_backend.py:256). */
void mgo_sort_pairs_u64(uint64_t* keys, int32_t* ids, int64_t m, int bits) {
    if (m <= 1) return;
    uint64_t* k2 = (uint64_t*)malloc(sizeof(uint64_t) * m);
    int32_t* v2 = (int32_t*)malloc(sizeof(int32_t) * m);
    uint64_t *ka = keys, *kb = k2;
    int32_t *va = ids, *vb = v2;
    for (int shift = 0; shift < bits; shift += 8) {
        int64_t cnt[257];
        memset(cnt, 0, sizeof(cnt));
        for (int64_t i = 0; i < m; ++i) cnt[((ka[i] >> shift) & 0xff) + 1]++;
        for (int d = 0; d < 256; ++d) cnt[d + 1] += cnt[d];
        for (int64_t i = 0; i < m; ++i) {
            const int64_t p = cnt[(ka[i] >> shift) & 0xff]++;
            kb[p] = ka[i];
            vb[p] = va[i];
        }
        uint64_t* tk = ka; ka = kb; kb = tk;
        int32_t* tv = va; va = vb; vb = tv;
    }
    if (ka != keys) {
        memcpy(keys, ka, sizeof(uint64_t) * m);
        memcpy(ids, va, sizeof(int32_t) * m);
    }
    free(k2);
    free(v2);
}

/* offsets[t] = first index whose tile (key >> 32) is >= t; offsets[T] = m
   (the searchsorted of metal_backend.py:257-260). */
void mgo_tile_ranges(const uint64_t* keys, int64_t m, int n_tiles, int32_t* offsets) {
    int64_t i = 0;
    for (int t = 0; t <= n_tiles; ++t) {
        while (i < m && (int64_t)(keys[i] >> 32) < t) ++i;
        offsets[t] = (int32_t)i;
    }
}

/* ------------------------------------------------------------------------ */
/* rasterize_forward (rasterize.metal:61-167), one pixel at a time           */
/* ------------------------------------------------------------------------ */
void mgo_rasterize_forward(const float* uv, const float* conic, const float* opacity,
                           const float* color, const int32_t* ids, const int32_t* offsets,
                           int W, int H, int tile, const float* bg, float* out_rgb,
                           float* out_alpha, float* out_T, int32_t* out_stop) {
    const int tiles_x = (W + tile - 1) / tile;
#pragma omp parallel for schedule(dynamic, 16)
    for (int64_t p = 0; p < (int64_t)W * H; ++p) {
        const int px = (int)(p % W), py = (int)(p / W);
        const int t = (py / tile) * tiles_x + px / tile;
        const int start = offsets[t], end = offsets[t + 1];
        const float fx = (float)px + 0.5f, fy = (float)py + 0.5f;
        float T = 1.0f, acc[3] = {0.f, 0.f, 0.f}, a_acc = 0.f;
        int stop = start;
        for (int i = start; i < end; ++i) {
            const int64_t g = ids[i];
            const float dx = fx - uv[2 * g], dy = fy - uv[2 * g + 1];
            const float* c = conic + 3 * g;
            const float power = -0.5f * (c[0] * dx * dx + 2.0f * c[1] * dx * dy + c[2] * dy * dy);
            if (power > 0.0f) continue;
            const float alpha = fminf(0.999f, opacity[g] * expf(power));
            if (alpha < 1.0f / 255.0f) continue;
            const float w = alpha * T;
            for (int k = 0; k < 3; ++k) acc[k] += w * color[3 * g + k];
            a_acc += w;
            T *= (1.0f - alpha);
            stop = i + 1;
            if (T < 1e-4f) break;
        }
        if (bg) {
            const float kk = fmaxf(1.0f - a_acc, 0.0f);
            for (int k = 0; k < 3; ++k) acc[k] = acc[k] + kk * bg[k];
        }
        for (int k = 0; k < 3; ++k) out_rgb[3 * p + k] = acc[k];
        out_alpha[p] = a_acc;
        out_T[p] = T;
        out_stop[p] = stop;
    }
}

/* ------------------------------------------------------------------------ */
/* rasterize_backward (rasterize.metal:173-340): reverse walk from the stop */
/* index, T recovered by division; gradients ADDED into the packed g2d      */
/* records (MG_G2D_* layout).                                               */
/* ------------------------------------------------------------------------ */
void mgo_rasterize_backward(const float* uv, const float* conic, const float* opacity,
                            const float* color, const int32_t* ids, const int32_t* offsets,
                            const float* final_T, const int32_t* stop_idx,
                            const float* grad_rgb, const float* grad_alpha, int W, int H,
                            int tile, const float* bg, const float* alpha_fwd,
                            int want_absgrad, float* g2d) {
    const int tiles_x = (W + tile - 1) / tile;
#pragma omp parallel for schedule(dynamic, 16)
    for (int64_t p = 0; p < (int64_t)W * H; ++p) {
        const int px = (int)(p % W), py = (int)(p / W);
        const int t = (py / tile) * tiles_x + px / tile;
        const int start = offsets[t];
        const float fx = (float)px + 0.5f, fy = (float)py + 0.5f;
        float T = final_T[p];
        const float* dL_drgb = grad_rgb + 3 * p;
        float dL_da = grad_alpha ? grad_alpha[p] : 0.f;
        if (bg && 1.0f - alpha_fwd[p] >= 0.0f)
            dL_da -= dL_drgb[0] * bg[0] + dL_drgb[1] * bg[1] + dL_drgb[2] * bg[2];
        float suffix[3] = {0.f, 0.f, 0.f}, suffix_a = 0.f;
        for (int i = stop_idx[p] - 1; i >= start; --i) {
            const int64_t g = ids[i];
            const float dx = fx - uv[2 * g], dy = fy - uv[2 * g + 1];
            const float* c = conic + 3 * g;
            const float power = -0.5f * (c[0] * dx * dx + 2.0f * c[1] * dx * dy + c[2] * dy * dy);
            if (power > 0.0f) continue;
            const float gauss = expf(power);
            const float op = opacity[g];
            const float alpha_raw = op * gauss;
            const int clamped = alpha_raw > 0.999f;
            const float alpha = fminf(0.999f, alpha_raw);
            if (alpha < 1.0f / 255.0f) continue;
            const float om = fmaxf(1.0f - alpha, 1e-8f);
            T = T / om;
            const float inv = 1.0f / om;
            const float w = alpha * T;
            const float* col = color + 3 * g;
            float* out = g2d + MG_G2D_STRIDE * g;
            float dL_dalpha = dL_da * (T - suffix_a * inv);
            for (int k = 0; k < 3; ++k) {
#pragma omp atomic
                out[MG_G2D_COLOR + k] += w * dL_drgb[k];
                dL_dalpha += dL_drgb[k] * (T * col[k] - suffix[k] * inv);
            }
            for (int k = 0; k < 3; ++k) suffix[k] += alpha * T * col[k];
            suffix_a += alpha * T;
            if (!clamped) {
                const float dp = dL_dalpha * op * gauss;
                const float dux = dp * (c[0] * dx + c[1] * dy);
                const float duy = dp * (c[1] * dx + c[2] * dy);
#pragma omp atomic
                out[MG_G2D_OPACITY] += dL_dalpha * gauss;
#pragma omp atomic
                out[MG_G2D_UV] += dux;
#pragma omp atomic
                out[MG_G2D_UV + 1] += duy;
#pragma omp atomic
                out[MG_G2D_CONIC] += dp * (-0.5f * dx * dx);
#pragma omp atomic
                out[MG_G2D_CONIC + 1] += dp * (-1.0f * dx * dy);
#pragma omp atomic
                out[MG_G2D_CONIC + 2] += dp * (-0.5f * dy * dy);
                if (want_absgrad) {
#pragma omp atomic
                    out[MG_G2D_ABSUV] += sqrtf(dux * dux + duy * duy);
                }
            }
        }
    }
}

/* ------------------------------------------------------------------------ */
/* Adam (adam.metal:25-42, torch.optim.Adam order) and SelectiveAdam        */
/* (selective_adam.py:116-148)                                              */
/* ------------------------------------------------------------------------ */
void mgo_adam_step(float* p, const float* g, float* m, float* v, int64_t n, float lr, float b1,
                   float b2, float eps, float bc1, float sqrt_bc2) {
    const float w1 = 1.0f - b1, w2 = 1.0f - b2, ss = lr / bc1;
#pragma omp parallel for schedule(static)
    for (int64_t i = 0; i < n; ++i) {
        const float gi = g[i];
        const float mi = m[i] + w1 * (gi - m[i]);
        const float vi = v[i] * b2 + (w2 * gi) * gi;
        m[i] = mi;
        v[i] = vi;
        p[i] = p[i] + ((-ss) * mi) / (sqrtf(vi) / sqrt_bc2 + eps);
    }
}

void mgo_selective_adam_step(float* p, const float* g, float* m, float* v, float* steps,
                             const uint8_t* visible, int64_t n_visible, int64_t rows,
                             int64_t width, float lr, float b1, float b2, float eps) {
    const float w1 = (float)(1.0 - (double)b1), w2 = (float)(1.0 - (double)b2);
#pragma omp parallel for schedule(static)
    for (int64_t r = 0; r < rows; ++r) {
        if (r >= n_visible || !visible[r]) continue;
        const float k = steps[r] + 1.0f;
        const float bc1 = 1.0f - powf(b1, k), bc2 = 1.0f - powf(b2, k);
        const float step_size = lr * (sqrtf(bc2) / bc1);
        for (int64_t e = 0; e < width; ++e) {
            const int64_t i = r * width + e;
            const float mi = m[i] * b1 + g[i] * w1;
            const float vi = v[i] * b2 + (g[i] * g[i]) * w2;
            m[i] = mi;
            v[i] = vi;
            p[i] = p[i] - (step_size * mi) / (sqrtf(vi) + eps);
        }
        steps[r] = k;
    }
}

/* ------------------------------------------------------------------------ */
/* SSIM and the training loss (metal_gauss/ssim.py; train.py:52-105,389-393) */
/* ------------------------------------------------------------------------ */
#define SSIM_C1 (0.01f * 0.01f)
#define SSIM_C2 (0.03f * 0.03f)

/* Separable 11-tap blur with zero padding of one (H,W) plane. */
static void blur_plane(const float* src, float* dst, float* tmp, int W, int H, const float* w) {
    for (int y = 0; y < H; ++y)
        for (int x = 0; x < W; ++x) {
            float s = 0.f;
            for (int k = -5; k <= 5; ++k) {
                const int u = x + k;
                if (u >= 0 && u < W) s += w[k + 5] * src[(int64_t)y * W + u];
            }
            tmp[(int64_t)y * W + x] = s;
        }
    for (int y = 0; y < H; ++y)
        for (int x = 0; x < W; ++x) {
            float s = 0.f;
            for (int k = -5; k <= 5; ++k) {
                const int v = y + k;
                if (v >= 0 && v < H) s += w[k + 5] * tmp[(int64_t)v * W + x];
            }
            dst[(int64_t)y * W + x] = s;
        }
}

/* loss = w_l1 mean|x-y| + w_ssim (1 - mean SSIM); grad = d loss / d x.
   x, y are (H,W,3). Returns the loss; grad may be NULL. */
double mgo_l1_ssim_loss(const float* x, const float* y, const float* w, int H, int W,
                        float w_l1, float w_ssim, float* grad) {
    const int64_t np = (int64_t)W * H;
    const double inv_n = 1.0 / (double)(3 * np);
    double sum_s = 0.0, sum_l1 = 0.0;
#pragma omp parallel for reduction(+ : sum_s, sum_l1) schedule(static)
    for (int c = 0; c < 3; ++c) {
        float* buf = (float*)malloc(sizeof(float) * np * 14);
        float *xs = buf, *ys = buf + np, *q = buf + 2 * np, *mx = buf + 3 * np,
              *my = buf + 4 * np, *exx = buf + 5 * np, *eyy = buf + 6 * np, *exy = buf + 7 * np,
              *tmp = buf + 8 * np, *a0 = buf + 9 * np, *a1 = buf + 10 * np, *a2 = buf + 11 * np,
              *b = buf + 12 * np;
        for (int64_t i = 0; i < np; ++i) { xs[i] = x[3 * i + c]; ys[i] = y[3 * i + c]; }
        blur_plane(xs, mx, tmp, W, H, w);
        blur_plane(ys, my, tmp, W, H, w);
        for (int64_t i = 0; i < np; ++i) q[i] = xs[i] * xs[i];
        blur_plane(q, exx, tmp, W, H, w);
        for (int64_t i = 0; i < np; ++i) q[i] = ys[i] * ys[i];
        blur_plane(q, eyy, tmp, W, H, w);
        for (int64_t i = 0; i < np; ++i) q[i] = xs[i] * ys[i];
        blur_plane(q, exy, tmp, W, H, w);
        const float gs = (float)(-(double)w_ssim * inv_n);
        for (int64_t i = 0; i < np; ++i) {
            const float MX = mx[i], MY = my[i];
            const float sxx = exx[i] - MX * MX, syy = eyy[i] - MY * MY, sxy = exy[i] - MX * MY;
            const float A = 2.f * MX * MY + SSIM_C1, B = 2.f * sxy + SSIM_C2;
            const float C = MX * MX + MY * MY + SSIM_C1, D = sxx + syy + SSIM_C2;
            const float invCD = 1.0f / (C * D);
            const float S = A * B * invCD;
            sum_s += S;
            sum_l1 += fabsf(xs[i] - ys[i]);
            const float dA = B * invCD, dB = A * invCD, dC = -S / C, dD = -S / D;
            a0[i] = gs * (2.f * MY * (dA - dB) + 2.f * MX * (dC - dD));
            a1[i] = gs * dD;
            a2[i] = gs * (2.f * dB);
        }
        if (grad) {
            const float gl = (float)((double)w_l1 * inv_n);
            blur_plane(a0, mx, tmp, W, H, w);
            blur_plane(a1, exx, tmp, W, H, w);
            blur_plane(a2, exy, tmp, W, H, w);
            for (int64_t i = 0; i < np; ++i) {
                const float d = xs[i] - ys[i];
                const float sg = d > 0.f ? 1.f : (d < 0.f ? -1.f : 0.f);
                grad[3 * i + c] = mx[i] + 2.f * xs[i] * exx[i] + ys[i] * exy[i] + gl * sg;
            }
        }
        (void)b;
        free(buf);
    }
    return (double)w_l1 * sum_l1 * inv_n + (double)w_ssim * (1.0 - sum_s * inv_n);
}
