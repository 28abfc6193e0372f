// Per-Gaussian projection, SH colour and the ellipse-vs-rectangle test, in the
// exact operation order shared with the CPU restatement in oracle/mg_oracle.c.
//
// The translation units that include this header are compiled with
// -fmad=false (no multiply-add contraction) and IEEE division and square root,
// so every expression below is a fixed sequence of correctly rounded fp32
// operations. The oracle is compiled with -ffp-contract=off and evaluates the
// same sequence, which makes uv, conic, depth, rxy, valid, colour, the tile
// counts and the sort keys bit-identical between the two.
//
// Math follows metal_gauss/csrc/preprocess.metal:114-221 (projection, EWA
// covariance with the 1.3x Jacobian clamp, blur, conic, 3-sigma radius,
// SnugBox extent, validity, visibility-gated SH) and
// metal_gauss/csrc/binning.metal:25-90 (minimum of the conic's quadratic form
// over a tile rectangle, threshold 2 ln(255 op)).
#pragma once

#include "common.cuh"

namespace mg {

#define MG_SH_C0 0.28209479177387814f
#define MG_SH_C1 0.4886025119029199f
#define MG_SH_C2_0 1.0925484305920792f
#define MG_SH_C2_1 -1.0925484305920792f
#define MG_SH_C2_2 0.31539156525252005f
#define MG_SH_C2_3 -1.0925484305920792f
#define MG_SH_C2_4 0.5462742152960396f
#define MG_SH_C3_0 -0.5900435899266435f
#define MG_SH_C3_1 2.890611442640554f
#define MG_SH_C3_2 -0.4570457994644658f
#define MG_SH_C3_3 0.3731763325901154f
#define MG_SH_C3_4 -0.4570457994644658f
#define MG_SH_C3_5 1.445305721320277f
#define MG_SH_C3_6 -0.5900435899266435f

__device__ __forceinline__ float clampf(float v, float lo, float hi) {
    return fminf(fmaxf(v, lo), hi);
}

// Real SH basis, degrees 0-3, in the .ply / 3DGS coefficient order
// (metal_gauss/sh.py:11-62).
__device__ __forceinline__ void sh_basis(int deg, float x, float y, float z, float* B) {
    B[0] = MG_SH_C0;
    if (deg < 1) return;
    B[1] = (-MG_SH_C1) * y;
    B[2] = MG_SH_C1 * z;
    B[3] = (-MG_SH_C1) * x;
    if (deg < 2) return;
    const float xx = x * x, yy = y * y, zz = z * z;
    B[4] = (MG_SH_C2_0 * x) * y;
    B[5] = (MG_SH_C2_1 * y) * z;
    B[6] = MG_SH_C2_2 * (((2.0f * zz) - xx) - yy);
    B[7] = (MG_SH_C2_3 * x) * z;
    B[8] = MG_SH_C2_4 * (xx - yy);
    if (deg < 3) return;
    B[9] = (MG_SH_C3_0 * y) * ((3.0f * xx) - yy);
    B[10] = ((MG_SH_C3_1 * x) * y) * z;
    B[11] = (MG_SH_C3_2 * y) * (((4.0f * zz) - xx) - yy);
    B[12] = (MG_SH_C3_3 * z) * (((2.0f * zz) - (3.0f * xx)) - (3.0f * yy));
    B[13] = (MG_SH_C3_4 * x) * (((4.0f * zz) - xx) - yy);
    B[14] = (MG_SH_C3_5 * z) * (xx - yy);
    B[15] = (MG_SH_C3_6 * x) * (xx - (3.0f * yy));
}

// Everything preprocess_forward produces for one Gaussian except colour.
struct Projected {
    float u, v;
    float ca, cb, cc;  // conic
    float z;           // camera-space depth (unclamped)
    float rx, ry;      // SnugBox half extents
    bool ok;
    float a, b, c;     // dilated 2D covariance (used by the backward)
};

// The view-independent part of a projection: the 3D covariance from the
// quaternion and scales, and the opacity's radius factor sqrt(2 ln(255 op)).
struct GaussianCov {
    float S00, S01, S02, S11, S12, S22;
    float rs;
};

__device__ __forceinline__ GaussianCov gaussian_cov(float qw0, float qx0, float qy0, float qz0,
                                                    float sx, float sy, float sz, float op) {
    GaussianCov G;
    const float qn = sqrtf(((qw0 * qw0 + qx0 * qx0) + qy0 * qy0) + qz0 * qz0);
    const float qd = fmaxf(qn, 1e-12f);
    const float w = qw0 / qd, x = qx0 / qd, y = qy0 / qd, zq = qz0 / qd;
    const float R00 = 1.0f - 2.0f * ((y * y) + (zq * zq));
    const float R01 = 2.0f * ((x * y) - (w * zq));
    const float R02 = 2.0f * ((x * zq) + (w * y));
    const float R10 = 2.0f * ((x * y) + (w * zq));
    const float R11 = 1.0f - 2.0f * ((x * x) + (zq * zq));
    const float R12 = 2.0f * ((y * zq) - (w * x));
    const float R20 = 2.0f * ((x * zq) - (w * y));
    const float R21 = 2.0f * ((y * zq) + (w * x));
    const float R22 = 1.0f - 2.0f * ((x * x) + (y * y));

    // M = R diag(s); Sigma = M M^T
    const float M00 = R00 * sx, M01 = R01 * sy, M02 = R02 * sz;
    const float M10 = R10 * sx, M11 = R11 * sy, M12 = R12 * sz;
    const float M20 = R20 * sx, M21 = R21 * sy, M22 = R22 * sz;
    G.S00 = (M00 * M00 + M01 * M01) + M02 * M02;
    G.S01 = (M00 * M10 + M01 * M11) + M02 * M12;
    G.S02 = (M00 * M20 + M01 * M21) + M02 * M22;
    G.S11 = (M10 * M10 + M11 * M11) + M12 * M12;
    G.S12 = (M10 * M20 + M11 * M21) + M12 * M22;
    G.S22 = (M20 * M20 + M21 * M21) + M22 * M22;

    const float twoL = 2.0f * log_f32_via_f64(fmaxf(255.0f * op, 1.0f));
    G.rs = sqrtf(twoL);
    return G;
}

// The view-dependent part: everything preprocess_forward produces for one
// Gaussian and camera except colour, from its mean and GaussianCov.
__device__ __forceinline__ Projected project_with(const CamParams& P, float mx, float my,
                                                  float mz, const GaussianCov& G) {
    Projected o;
    const float S00 = G.S00, S01 = G.S01, S02 = G.S02, S11 = G.S11, S12 = G.S12, S22 = G.S22;
    const float pcx = ((P.R0.x * mx + P.R0.y * my) + P.R0.z * mz) + P.R0.w;
    const float pcy = ((P.R1.x * mx + P.R1.y * my) + P.R1.z * mz) + P.R1.w;
    const float pcz = ((P.R2.x * mx + P.R2.y * my) + P.R2.z * mz) + P.R2.w;
    const float z = pcz;
    const float zc = fmaxf(z, P.near_plane);

    const float u = ((P.fx * pcx) / zc) + P.cx;
    const float v = ((P.fy * pcy) / zc) + P.cy;

    const float lim_x = 1.3f * ((0.5f * (float)P.W) / P.fx);
    const float lim_y = 1.3f * ((0.5f * (float)P.H) / P.fy);
    const float tx = clampf(pcx / zc, -lim_x, lim_x) * zc;
    const float ty = clampf(pcy / zc, -lim_y, lim_y) * zc;

    const float izc = 1.0f / zc, izc2 = izc * izc;
    const float J0x = P.fx * izc, J0z = ((-P.fx) * tx) * izc2;
    const float J1y = P.fy * izc, J1z = ((-P.fy) * ty) * izc2;
    // T = J R_w2c (rows), with J0y = J1x = 0 written out as in the reference
    const float T00 = (J0x * P.R0.x + 0.0f * P.R1.x) + J0z * P.R2.x;
    const float T01 = (J0x * P.R0.y + 0.0f * P.R1.y) + J0z * P.R2.y;
    const float T02 = (J0x * P.R0.z + 0.0f * P.R1.z) + J0z * P.R2.z;
    const float T10 = (0.0f * P.R0.x + J1y * P.R1.x) + J1z * P.R2.x;
    const float T11 = (0.0f * P.R0.y + J1y * P.R1.y) + J1z * P.R2.y;
    const float T12 = (0.0f * P.R0.z + J1y * P.R1.z) + J1z * P.R2.z;

    const float ST00 = (S00 * T00 + S01 * T01) + S02 * T02;
    const float ST01 = (S01 * T00 + S11 * T01) + S12 * T02;
    const float ST02 = (S02 * T00 + S12 * T01) + S22 * T02;
    const float ST10 = (S00 * T10 + S01 * T11) + S02 * T12;
    const float ST11 = (S01 * T10 + S11 * T11) + S12 * T12;
    const float ST12 = (S02 * T10 + S12 * T11) + S22 * T12;

    const float a = ((T00 * ST00 + T01 * ST01) + T02 * ST02) + P.blur;
    const float b = (T00 * ST10 + T01 * ST11) + T02 * ST12;
    const float c = ((T10 * ST10 + T11 * ST11) + T12 * ST12) + P.blur;
    const float det = (a * c) - (b * b);
    const float dets = fmaxf(det, 1e-12f);

    const float mid = 0.5f * (a + c);
    const float disc = sqrtf(fmaxf((mid * mid) - dets, 0.0f));
    const float lam = fmaxf(mid + disc, 1e-12f);
    const float radius = 3.0f * sqrtf(lam);

    const float rs = G.rs;
    const float rx = fminf(rs * sqrtf(fmaxf(a, 0.0f)), radius);
    const float ry = fminf(rs * sqrtf(fmaxf(c, 0.0f)), radius);

    o.ok = (z > P.near_plane) && (z < P.far_plane) && (det > 1e-12f) &&
           (radius < P.max_radius) && (rx > 0.0f) && (ry > 0.0f) &&
           (u + rx > 0.0f) && (u - rx < (float)P.W) &&
           (v + ry > 0.0f) && (v - ry < (float)P.H);
    o.u = u; o.v = v;
    o.ca = c / dets; o.cb = (-b) / dets; o.cc = a / dets;
    o.z = z; o.rx = rx; o.ry = ry;
    o.a = a; o.b = b; o.c = c;
    return o;
}

__device__ __forceinline__ Projected project_one(
    const CamParams& P, float mx, float my, float mz,
    float qw0, float qx0, float qy0, float qz0,
    float sx, float sy, float sz, float op)
{
    return project_with(P, mx, my, mz, gaussian_cov(qw0, qx0, qy0, qz0, sx, sy, sz, op));
}

// Minimum of a x^2 + 2 b x y + c y^2 (x, y relative to mu) over the closed
// rectangle [x0,x1] x [y0,y1]: 0 with the centre inside, otherwise the
// smallest of the four edge minima (binning.metal:25-44).
__device__ __forceinline__ float min_q_over_rect(float mux, float muy, float ca,
                                                 float cb, float ccz, float x0,
                                                 float x1, float y0, float y1) {
    if (mux >= x0 && mux <= x1 && muy >= y0 && muy <= y1) return 0.0f;
    const float a = fmaxf(ca, 1e-12f), b = cb, cc = fmaxf(ccz, 1e-12f);
    float best = __int_as_float(0x7f800000);
#pragma unroll
    for (int e = 0; e < 2; ++e) {
        const float yc = (e == 0) ? y0 : y1;
        const float xs = clampf(mux - ((b * (yc - muy)) / a), x0, x1);
        const float ex = xs - mux, ey = yc - muy;
        best = fminf(best, (((a * ex) * ex) + (((2.0f * b) * ex) * ey)) + ((cc * ey) * ey));
    }
#pragma unroll
    for (int e = 0; e < 2; ++e) {
        const float xc = (e == 0) ? x0 : x1;
        const float ys = clampf(muy - ((b * (xc - mux)) / cc), y0, y1);
        const float ex = xc - mux, ey = ys - muy;
        best = fminf(best, (((a * ex) * ex) + (((2.0f * b) * ex) * ey)) + ((cc * ey) * ey));
    }
    return best;
}

// min_q_over_rect evaluated tile after tile along a row-major walk of a grid
// of tile rectangles. The terms that depend only on one row edge (y) or one
// column edge (x) -- among them the two divisions per edge -- are computed
// once per edge and shared by the tiles on either side of it. Each value is
// produced by the same operations on the same operands as min_q_over_rect,
// so the minima are bit-identical; only repeated work is removed.
struct RowEdge {
    float y, ey, s, tc;  // y, y - mu_y, b (y - mu_y) / a, c (y - mu_y)^2
};
struct ColEdge {
    float x, ex, s, ta;  // x, x - mu_x, b (x - mu_x) / c, a (x - mu_x)^2
};
struct RectQuadratic {
    float mux, muy, a, b, b2, c;
    __device__ __forceinline__ RectQuadratic(float mux_, float muy_, float ca, float cb,
                                             float ccz)
        : mux(mux_), muy(muy_), a(fmaxf(ca, 1e-12f)), b(cb), b2(2.0f * cb),
          c(fmaxf(ccz, 1e-12f)) {}
    __device__ __forceinline__ RowEdge row_edge(float y) const {
        RowEdge e;
        e.y = y;
        e.ey = y - muy;
        e.s = (b * e.ey) / a;
        e.tc = (c * e.ey) * e.ey;
        return e;
    }
    __device__ __forceinline__ ColEdge col_edge(float x) const {
        ColEdge e;
        e.x = x;
        e.ex = x - mux;
        e.s = (b * e.ex) / c;
        e.ta = (a * e.ex) * e.ex;
        return e;
    }
    // The candidate of min_q_over_rect on a vertical side at column edge e
    // between rows t and bt. A walk along a row computes it once per column
    // edge: the right side's candidate of one tile is the left side's of the
    // next (same operations on the same operands).
    __device__ __forceinline__ float side_q(const ColEdge& e, const RowEdge& t,
                                            const RowEdge& bt) const {
        const float ey = clampf(muy - e.s, t.y, bt.y) - muy;
        return (e.ta + ((b2 * e.ex) * ey)) + ((c * ey) * ey);
    }
    // min_q with the two vertical sides' candidates given (ql = side_q(l, t,
    // bt), qr = side_q(r, t, bt)): the same minimum of the same four values.
    __device__ __forceinline__ float min_q_sides(const ColEdge& l, const ColEdge& r,
                                                 const RowEdge& t, const RowEdge& bt, float ql,
                                                 float qr) const {
        if (mux >= l.x && mux <= r.x && muy >= t.y && muy <= bt.y) return 0.0f;
        float best = __int_as_float(0x7f800000);
        {
            const float ex = clampf(mux - t.s, l.x, r.x) - mux;
            best = fminf(best, (((a * ex) * ex) + ((b2 * ex) * t.ey)) + t.tc);
        }
        {
            const float ex = clampf(mux - bt.s, l.x, r.x) - mux;
            best = fminf(best, (((a * ex) * ex) + ((b2 * ex) * bt.ey)) + bt.tc);
        }
        best = fminf(best, ql);
        return fminf(best, qr);
    }
    // min_q_over_rect(mux, muy, ca, cb, ccz, l.x, r.x, t.y, bt.y)
    __device__ __forceinline__ float min_q(const ColEdge& l, const ColEdge& r, const RowEdge& t,
                                           const RowEdge& bt) const {
        if (mux >= l.x && mux <= r.x && muy >= t.y && muy <= bt.y) return 0.0f;
        float best = __int_as_float(0x7f800000);
        {
            const float ex = clampf(mux - t.s, l.x, r.x) - mux;
            best = fminf(best, (((a * ex) * ex) + ((b2 * ex) * t.ey)) + t.tc);
        }
        {
            const float ex = clampf(mux - bt.s, l.x, r.x) - mux;
            best = fminf(best, (((a * ex) * ex) + ((b2 * ex) * bt.ey)) + bt.tc);
        }
        {
            const float ey = clampf(muy - l.s, t.y, bt.y) - muy;
            best = fminf(best, (l.ta + ((b2 * l.ex) * ey)) + ((c * ey) * ey));
        }
        {
            const float ey = clampf(muy - r.s, t.y, bt.y) - muy;
            best = fminf(best, (r.ta + ((b2 * r.ex) * ey)) + ((c * ey) * ey));
        }
        return best;
    }
};

// Tile rectangle clamped to the grid, from the SnugBox extents
// (binning.metal:59-64).
struct TileRect {
    int x0, x1, y0, y1;
};

__device__ __forceinline__ TileRect tile_rect(float mux, float muy, float rx,
                                              float ry, int tile, int tiles_x,
                                              int tiles_y) {
    const float tf = (float)tile;
    float ex0, ex1, ey0, ey1;
    if ((tile & (tile - 1)) == 0) {
        // a power-of-two side: x * (1 / tile) is x / tile exactly (scaling by
        // a power of two rounds once, as the division does)
        const float inv = 1.0f / tf;
        ex0 = (mux - rx) * inv; ex1 = (mux + rx) * inv;
        ey0 = (muy - ry) * inv; ey1 = (muy + ry) * inv;
    } else {
        ex0 = (mux - rx) / tf; ex1 = (mux + rx) / tf;
        ey0 = (muy - ry) / tf; ey1 = (muy + ry) / tf;
    }
    TileRect r;
    r.x0 = min(max((int)floorf(ex0), 0), tiles_x - 1);
    r.x1 = min(max((int)floorf(ex1), 0), tiles_x - 1);
    r.y0 = min(max((int)floorf(ey0), 0), tiles_y - 1);
    r.y1 = min(max((int)floorf(ey1), 0), tiles_y - 1);
    return r;
}

}  // namespace mg
