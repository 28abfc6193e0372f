// Preprocess backward (preprocess.metal:223-411): SH adjoint gated on a
// non-zero colour gradient and the ReLU of the pre-clamp colour, then the
// projection adjoint (conic -> 2D covariance -> Sigma and J -> camera point,
// with the Jacobian clamp routing the gradient to zc) and the quaternion VJP
// through normalisation. Rows with valid == 0 get zero scale and quaternion
// gradients. One thread per Gaussian, no atomics.
//
// SH coefficient rows are staged per warp through shared memory: the split
// layout's (N,15,3) rows and the fused layout's (N,16,3) rows are 180 B and
// 192 B, so per-thread access would scatter every load and store across 32
// rows; the warp moves its 32 rows as one contiguous block instead.
#include "exact_math.cuh"
#include "filter3d.cuh"
#include "kernels.cuh"

namespace mg {

namespace {

constexpr int kBwdBlock = 128;
constexpr int kRowBlock = 48;  // floats staged per Gaussian (16 rows x 3)
constexpr mg_sh_layout SH_SPLIT_LAYOUT = {1, 15, 0, 0};

__device__ __forceinline__ void sh_basis_grad(int b, float x, float y, float z, float& gx,
                                              float& gy, float& gz) {
    const float xx = x * x, yy = y * y, zz = z * z;
    switch (b) {
        case 1: gx = 0.f; gy = -MG_SH_C1; gz = 0.f; break;
        case 2: gx = 0.f; gy = 0.f; gz = MG_SH_C1; break;
        case 3: gx = -MG_SH_C1; gy = 0.f; gz = 0.f; break;
        case 4: gx = MG_SH_C2_0 * y; gy = MG_SH_C2_0 * x; gz = 0.f; break;
        case 5: gx = 0.f; gy = MG_SH_C2_1 * z; gz = MG_SH_C2_1 * y; break;
        case 6: gx = MG_SH_C2_2 * (-2.f * x); gy = MG_SH_C2_2 * (-2.f * y); gz = MG_SH_C2_2 * (4.f * z); break;
        case 7: gx = MG_SH_C2_3 * z; gy = 0.f; gz = MG_SH_C2_3 * x; break;
        case 8: gx = MG_SH_C2_4 * (2.f * x); gy = MG_SH_C2_4 * (-2.f * y); gz = 0.f; break;
        case 9: gx = MG_SH_C3_0 * (6.f * x * y); gy = MG_SH_C3_0 * (3.f * xx - 3.f * yy); gz = 0.f; break;
        case 10: gx = MG_SH_C3_1 * (y * z); gy = MG_SH_C3_1 * (x * z); gz = MG_SH_C3_1 * (x * y); break;
        case 11: gx = MG_SH_C3_2 * (-2.f * x * y); gy = MG_SH_C3_2 * (4.f * zz - xx - 3.f * yy); gz = MG_SH_C3_2 * (8.f * y * z); break;
        case 12: gx = MG_SH_C3_3 * (-6.f * x * z); gy = MG_SH_C3_3 * (-6.f * y * z); gz = MG_SH_C3_3 * (6.f * zz - 3.f * xx - 3.f * yy); break;
        case 13: gx = MG_SH_C3_4 * (4.f * zz - 3.f * xx - yy); gy = MG_SH_C3_4 * (-2.f * x * y); gz = MG_SH_C3_4 * (8.f * x * z); break;
        case 14: gx = MG_SH_C3_5 * (2.f * x * z); gy = MG_SH_C3_5 * (-2.f * y * z); gz = MG_SH_C3_5 * (xx - yy); break;
        case 15: gx = MG_SH_C3_6 * (3.f * xx - 3.f * yy); gy = MG_SH_C3_6 * (-6.f * x * y); gz = 0.f; break;
        default: gx = gy = gz = 0.f;
    }
}

// The warp's SH block: row r (0 = DC, 1..15 = bands 1+) of lane `lane`.
struct ShBlock {
    float* s;        // shared memory, 32 x kRowBlock floats
    bool fused;      // fused: rows 0..15 staged; split: rows 1..15 staged
    __device__ __forceinline__ float* row(int lane, int r) const {
        return s + lane * kRowBlock + (fused ? r : r - 1) * 3;
    }
};

// Projection adjoint (preprocess.metal:265-411), in two parts: the incoming
// uv and conic gradients of one camera are carried through the conic inverse
// and the EWA covariance J W Sigma W^T J^T (with the Jacobian's clamp routing
// to zc) to the mean and to d Sigma; d Sigma goes through Sigma = R S S^T R^T
// and the quaternion normalisation to d scales and d quat. The second part is
// linear in d Sigma, so a Gaussian seen by several cameras sums their
// (symmetrised) d Sigma and runs it once; the view-independent rotation and
// covariance are formed once as well.
struct CovFrame {
    float w, x, y, zq, qd;  // normalised quaternion and the norm it was divided by
    float R[3][3], M[3][3], S[3][3];
};

__device__ __forceinline__ CovFrame cov_frame(const float4 q4, const float (&s)[3]) {
    CovFrame F;
    const float qn = sqrtf(q4.x * q4.x + q4.y * q4.y + q4.z * q4.z + q4.w * q4.w);
    F.qd = fmaxf(qn, 1e-12f);
    const float w = q4.x / F.qd, x = q4.y / F.qd, y = q4.z / F.qd, zq = q4.w / F.qd;
    F.w = w; F.x = x; F.y = y; F.zq = zq;
    F.R[0][0] = 1.f - 2.f * (y * y + zq * zq); F.R[0][1] = 2.f * (x * y - w * zq); F.R[0][2] = 2.f * (x * zq + w * y);
    F.R[1][0] = 2.f * (x * y + w * zq); F.R[1][1] = 1.f - 2.f * (x * x + zq * zq); F.R[1][2] = 2.f * (y * zq - w * x);
    F.R[2][0] = 2.f * (x * zq - w * y); F.R[2][1] = 2.f * (y * zq + w * x); F.R[2][2] = 1.f - 2.f * (x * x + y * y);
#pragma unroll
    for (int i = 0; i < 3; ++i)
#pragma unroll
        for (int j = 0; j < 3; ++j) F.M[i][j] = F.R[i][j] * s[j];
#pragma unroll
    for (int i = 0; i < 3; ++i)
#pragma unroll
        for (int j = 0; j < 3; ++j)
            F.S[i][j] = F.M[i][0] * F.M[j][0] + F.M[i][1] * F.M[j][1] + F.M[i][2] * F.M[j][2];
    return F;
}

// One camera: adds the mean gradient into dmx/dmy/dmz and the symmetrised
// covariance gradient (entries 00 01 02 11 12 22) into dSym.
__device__ __forceinline__ void projection_adjoint_view(const CamParams& P, float mx, float my,
                                                        float mz, const float (&S)[3][3],
                                                        float dux, float duy, float dcx,
                                                        float dcy, float dcz, float& dmx,
                                                        float& dmy, float& dmz,
                                                        float (&dSym)[6]) {
    const float fx = P.fx, fy = P.fy;
    const float pcx = P.R0.x * mx + P.R0.y * my + P.R0.z * mz + P.R0.w;
    const float pcy = P.R1.x * mx + P.R1.y * my + P.R1.z * mz + P.R1.w;
    const float pcz = P.R2.x * mx + P.R2.y * my + P.R2.z * mz + P.R2.w;
    const float z = pcz, zc = fmaxf(z, P.near_plane);
    const float izc = 1.0f / zc, izc2 = izc * izc;
    const float lim_x = 1.3f * (0.5f * (float)P.W / fx);
    const float lim_y = 1.3f * (0.5f * (float)P.H / fy);
    const float txn = pcx / zc, tyn = pcy / zc;
    const bool clx = (txn < -lim_x) || (txn > lim_x);
    const bool cly = (tyn < -lim_y) || (tyn > lim_y);
    const float tx = clampf(txn, -lim_x, lim_x) * zc;
    const float ty = clampf(tyn, -lim_y, lim_y) * zc;

    const float Rw[3][3] = {{P.R0.x, P.R0.y, P.R0.z}, {P.R1.x, P.R1.y, P.R1.z},
                            {P.R2.x, P.R2.y, P.R2.z}};
    const float J0x = fx * izc, J0z = -fx * tx * izc2;
    const float J1y = fy * izc, J1z = -fy * ty * izc2;
    float T0[3], T1[3], ST0[3], ST1[3];
#pragma unroll
    for (int k = 0; k < 3; ++k) {
        T0[k] = J0x * Rw[0][k] + J0z * Rw[2][k];
        T1[k] = J1y * Rw[1][k] + J1z * Rw[2][k];
    }
#pragma unroll
    for (int i = 0; i < 3; ++i) {
        ST0[i] = S[i][0] * T0[0] + S[i][1] * T0[1] + S[i][2] * T0[2];
        ST1[i] = S[i][0] * T1[0] + S[i][1] * T1[1] + S[i][2] * T1[2];
    }
    const float a = T0[0] * ST0[0] + T0[1] * ST0[1] + T0[2] * ST0[2] + P.blur;
    const float b = T0[0] * ST1[0] + T0[1] * ST1[1] + T0[2] * ST1[2];
    const float c = T1[0] * ST1[0] + T1[1] * ST1[1] + T1[2] * ST1[2] + P.blur;
    const float det = a * c - b * b;
    const float dets = fmaxf(det, 1e-12f);
    const float id = 1.0f / dets;
    const float ddet = -(dcx * c - dcy * b + dcz * a) * id * id;
    float da = dcz * id + ddet * c;
    float db = -dcy * id - 2.0f * ddet * b;
    float dc = dcx * id + ddet * a;
    if (det <= 1e-12f) { da = db = dc = 0.f; }

    // d Sigma = da T0 T0^T + db T0 T1^T + dc T1 T1^T, symmetrised
    const float hb = 0.5f * db;
    dSym[0] += da * T0[0] * T0[0] + db * T0[0] * T1[0] + dc * T1[0] * T1[0];
    dSym[1] += da * T0[0] * T0[1] + hb * (T0[0] * T1[1] + T0[1] * T1[0]) + dc * T1[0] * T1[1];
    dSym[2] += da * T0[0] * T0[2] + hb * (T0[0] * T1[2] + T0[2] * T1[0]) + dc * T1[0] * T1[2];
    dSym[3] += da * T0[1] * T0[1] + db * T0[1] * T1[1] + dc * T1[1] * T1[1];
    dSym[4] += da * T0[1] * T0[2] + hb * (T0[1] * T1[2] + T0[2] * T1[1]) + dc * T1[1] * T1[2];
    dSym[5] += da * T0[2] * T0[2] + db * T0[2] * T1[2] + dc * T1[2] * T1[2];
    float dT0[3], dT1[3];
#pragma unroll
    for (int k = 0; k < 3; ++k) {
        dT0[k] = 2.0f * (da * ST0[k]) + db * ST1[k];
        dT1[k] = 2.0f * (dc * ST1[k]) + db * ST0[k];
    }
    float dJ0[3], dJ1[3];
#pragma unroll
    for (int r = 0; r < 3; ++r) {
        dJ0[r] = dT0[0] * Rw[r][0] + dT0[1] * Rw[r][1] + dT0[2] * Rw[r][2];
        dJ1[r] = dT1[0] * Rw[r][0] + dT1[1] * Rw[r][1] + dT1[2] * Rw[r][2];
    }
    const float dtx = -fx * izc2 * dJ0[2];
    const float dty = -fy * izc2 * dJ1[2];
    float dzc = -fx * izc2 * dJ0[0] - fy * izc2 * dJ1[1] +
                2.0f * fx * tx * izc2 * izc * dJ0[2] + 2.0f * fy * ty * izc2 * izc * dJ1[2];
    float dpx = fx * izc * dux;
    float dpy = fy * izc * duy;
    dzc += -fx * pcx * izc2 * dux - fy * pcy * izc2 * duy;
    if (!clx) dpx += dtx; else dzc += dtx * (tx * izc);
    if (!cly) dpy += dty; else dzc += dty * (ty * izc);
    const float dpz = (z > P.near_plane) ? dzc : 0.0f;
    dmx += Rw[0][0] * dpx + Rw[1][0] * dpy + Rw[2][0] * dpz;
    dmy += Rw[0][1] * dpx + Rw[1][1] * dpy + Rw[2][1] * dpz;
    dmz += Rw[0][2] * dpx + Rw[1][2] * dpy + Rw[2][2] * dpz;
}

// From the (summed, symmetrised) covariance gradient to d scales and d quat.
__device__ __forceinline__ void covariance_adjoint(const CovFrame& F, const float (&s)[3],
                                                   const float (&dSym)[6], float (&ds)[3],
                                                   float4& dq) {
    const float D[3][3] = {{dSym[0], dSym[1], dSym[2]},
                           {dSym[1], dSym[3], dSym[4]},
                           {dSym[2], dSym[4], dSym[5]}};
    // dM = 2 sym(dSigma) M
    float dM[3][3];
#pragma unroll
    for (int i = 0; i < 3; ++i)
#pragma unroll
        for (int j = 0; j < 3; ++j)
            dM[i][j] = 2.0f * (D[i][0] * F.M[0][j] + D[i][1] * F.M[1][j] + D[i][2] * F.M[2][j]);
#pragma unroll
    for (int j = 0; j < 3; ++j)
        ds[j] = dM[0][j] * F.R[0][j] + dM[1][j] * F.R[1][j] + dM[2][j] * F.R[2][j];
    float G[3][3];  // dL/dR
#pragma unroll
    for (int i = 0; i < 3; ++i)
#pragma unroll
        for (int j = 0; j < 3; ++j) G[i][j] = dM[i][j] * s[j];
    const float w = F.w, x = F.x, y = F.y, zq = F.zq;
    const float dw = 2.f * (x * (G[2][1] - G[1][2]) + y * (G[0][2] - G[2][0]) + zq * (G[1][0] - G[0][1]));
    const float dqx = 2.f * (w * (G[2][1] - G[1][2]) + y * (G[1][0] + G[0][1]) + zq * (G[2][0] + G[0][2]) - 2.f * x * (G[1][1] + G[2][2]));
    const float dqy = 2.f * (w * (G[0][2] - G[2][0]) + x * (G[1][0] + G[0][1]) + zq * (G[2][1] + G[1][2]) - 2.f * y * (G[0][0] + G[2][2]));
    const float dqz = 2.f * (w * (G[1][0] - G[0][1]) + x * (G[2][0] + G[0][2]) + y * (G[2][1] + G[1][2]) - 2.f * zq * (G[0][0] + G[1][1]));
    const float qdot = w * dw + x * dqx + y * dqy + zq * dqz;
    dq = make_float4((dw - w * qdot) / F.qd, (dqx - x * qdot) / F.qd, (dqy - y * qdot) / F.qd,
                     (dqz - zq * qdot) / F.qd);
}

// Both parts for one camera. Adds the mean gradient into dmx/dmy/dmz;
// returns d scales and d quat.
__device__ __forceinline__ void projection_adjoint(const CamParams& P, float mx, float my,
                                                   float mz, const float4 q4, const float (&s)[3],
                                                   float dux, float duy, float dcx, float dcy,
                                                   float dcz, float& dmx, float& dmy,
                                                   float& dmz, float (&ds)[3], float4& dq) {
    const CovFrame F = cov_frame(q4, s);
    float dSym[6] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    projection_adjoint_view(P, mx, my, mz, F.S, dux, duy, dcx, dcy, dcz, dmx, dmy, dmz, dSym);
    covariance_adjoint(F, s, dSym, ds, dq);
}

// kAccum = false: the reference bridge's semantics (every output overwritten).
// kAccum = true: the training engine's form -- gradients are ADDED, the
// activation chain is applied (d_log_scales = d_scales * scales, d_logit =
// d_opacity * op (1 - op), with d_opacity read from `d_opac`), and rows that
// receive nothing are not written at all.
template <bool kAccum>
__global__ void __launch_bounds__(kBwdBlock)
preprocess_backward_kernel(const float* __restrict__ means, const float* __restrict__ quats,
                           const float* __restrict__ scales, const float* __restrict__ sh_dc,
                           const float* __restrict__ sh_rest, mg_sh_layout shl,
                           const float* __restrict__ d_uv, int64_t d_uv_stride,
                           const float* __restrict__ d_conic, int64_t d_conic_stride,
                           const float* __restrict__ d_color, int64_t d_color_stride,
                           const int32_t* __restrict__ valid, CamParams P, int sh_degree,
                           int64_t n, float* __restrict__ d_means,
                           float* __restrict__ d_quats, float* __restrict__ d_scales,
                           float* __restrict__ d_sh_dc, float* __restrict__ d_sh_rest,
                           int fused, int contiguous_rest,
                           const float* __restrict__ opac, const float* __restrict__ d_opac,
                           int64_t d_opac_stride, float* __restrict__ d_logit,
                           const float* __restrict__ color, float* __restrict__ dpre_out) {
    __shared__ float s_sh[kBwdBlock / 32][32 * kRowBlock];
    const int lane = threadIdx.x & 31, wib = threadIdx.x >> 5;
    const int64_t g = (int64_t)blockIdx.x * kBwdBlock + threadIdx.x;
    const int64_t g0 = g - lane;
    const bool in = g < n;
    const int64_t warp_n = min((int64_t)32, n - g0);

    float mx = 0.f, my = 0.f, mz = 0.f;
    if (in) { mx = means[3 * g]; my = means[3 * g + 1]; mz = means[3 * g + 2]; }
    float dmx = 0.f, dmy = 0.f, dmz = 0.f;

    // ---------------------------------------------------------- SH branch
    if (kAccum && dpre_out != nullptr) {
        // deferred: only the ReLU-gated colour gradient, for mg_sh_backward_views
        if (in) {
            float3 d = make_float3(0.f, 0.f, 0.f);
            if (d_color != nullptr) {
                const float* dc = d_color + g * d_color_stride;
                d = make_float3(color[3 * g] > 0.f ? dc[0] : 0.f,
                                color[3 * g + 1] > 0.f ? dc[1] : 0.f,
                                color[3 * g + 2] > 0.f ? dc[2] : 0.f);
            }
            dpre_out[3 * g] = d.x; dpre_out[3 * g + 1] = d.y; dpre_out[3 * g + 2] = d.z;
        }
    }
    const bool do_sh = sh_degree >= 0 && d_color != nullptr && sh_dc != nullptr &&
                       !(kAccum && dpre_out != nullptr);
    if (do_sh) {
        const ShBlock blk{s_sh[wib], fused != 0};
        const int nb = (sh_degree + 1) * (sh_degree + 1);
        float dcr = 0.f, dcg = 0.f, dcb = 0.f;
        if (in) {
            dcr = d_color[g * d_color_stride];
            dcg = d_color[g * d_color_stride + 1];
            dcb = d_color[g * d_color_stride + 2];
        }
        const bool need = in && !(dcr == 0.f && dcg == 0.f && dcb == 0.f);
        const bool staged = (fused != 0) || (contiguous_rest != 0);
        const unsigned any_need = __ballot_sync(0xffffffffu, need);
        // Stage coefficient rows (only when some lane reads them).
        if (staged && any_need) {
            const int per_g = fused ? 48 : 45;
            const float* src = fused ? sh_dc + g0 * 48 : sh_rest + g0 * 45;
            const int total = (int)warp_n * per_g;
            for (int i = lane; i < total; i += 32)
                blk.s[(i / per_g) * kRowBlock + (i % per_g)] = __ldg(src + i);
        }
        __syncwarp();
        // Row writer: the split layout's DC row goes straight to global memory
        // (12 B per Gaussian, coalesced across the warp); staged rows go to the
        // shared block; the rare unstaged layout writes in place.
        auto wr = [&](int i, float r0, float r1, float r2) {
            float* r;
            bool global = true;
            if (i == 0 && !blk.fused) r = d_sh_dc + g * (int64_t)shl.stride_dc * 3;
            else if (staged) { r = blk.row(lane, i); global = false; }
            else r = (i == 0) ? d_sh_dc + g * (int64_t)shl.stride_dc * 3
                              : d_sh_rest + (g * (int64_t)shl.stride_rest + shl.offset_rest + (i - 1)) * 3;
            if (kAccum && global) {
                if (r0 != 0.f || r1 != 0.f || r2 != 0.f) { r[0] += r0; r[1] += r1; r[2] += r2; }
            } else {
                r[0] = r0; r[1] = r1; r[2] = r2;
            }
        };
        if (need) {
            auto rd = [&](int i, int c) -> float {
                if (i == 0) return sh_dc[g * (int64_t)shl.stride_dc * 3 + c];
                if (staged) return blk.row(lane, i)[c];
                return sh_rest[(g * (int64_t)shl.stride_rest + shl.offset_rest + (i - 1)) * 3 + c];
            };
            const float dvx = mx - P.ccx, dvy = my - P.ccy, dvz = mz - P.ccz;
            const float len = fmaxf(sqrtf(dvx * dvx + dvy * dvy + dvz * dvz), 1e-12f);
            const float x = dvx / len, y = dvy / len, z = dvz / len;
            float B[16];
            sh_basis(sh_degree, x, y, z, B);
            float pr = 0.f, pg = 0.f, pb = 0.f;
#pragma unroll
            for (int i = 0; i < 16; ++i) {
                if (i < nb) { pr += B[i] * rd(i, 0); pg += B[i] * rd(i, 1); pb += B[i] * rd(i, 2); }
            }
            pr += 0.5f; pg += 0.5f; pb += 0.5f;
            const float er = pr > 0.f ? dcr : 0.f;
            const float eg = pg > 0.f ? dcg : 0.f;
            const float eb = pb > 0.f ? dcb : 0.f;
            float ddx = 0.f, ddy = 0.f, ddz = 0.f;
#pragma unroll
            for (int i = 0; i < 16; ++i) {
                if (i < nb) {
                    float gx, gy, gz;
                    sh_basis_grad(i, x, y, z, gx, gy, gz);
                    const float k = rd(i, 0) * er + rd(i, 1) * eg + rd(i, 2) * eb;
                    ddx += gx * k; ddy += gy * k; ddz += gz * k;
                    wr(i, B[i] * er, B[i] * eg, B[i] * eb);  // after this row's reads
                } else {
                    wr(i, 0.f, 0.f, 0.f);
                }
            }
            // dir = v/|v|: d v = (I - dir dir^T) d dir / |v|
            const float dd = x * ddx + y * ddy + z * ddz;
            dmx += (ddx - x * dd) / len;
            dmy += (ddy - y * dd) / len;
            dmz += (ddz - z * dd) / len;
        } else if (in && (!kAccum || (staged && any_need))) {
            // overwrite mode writes zeros; accumulate mode only clears this
            // lane's staged rows so the warp's block add below adds nothing
#pragma unroll
            for (int i = 0; i < 16; ++i) wr(i, 0.f, 0.f, 0.f);
        }
        __syncwarp();
        if (staged && (!kAccum || any_need)) {
            const int per_g = fused ? 48 : 45;
            float* dst = fused ? d_sh_dc + g0 * 48 : d_sh_rest + g0 * 45;
            const int total = (int)warp_n * per_g;
            for (int i = lane; i < total; i += 32) {
                const float x = blk.s[(i / per_g) * kRowBlock + (i % per_g)];
                if (kAccum) dst[i] += x; else dst[i] = x;
            }
        }
    }
    if (!in) return;

    // --------------------------------------------------- projection branch
    if (valid[g] != 0) {
        const float4 q4 = reinterpret_cast<const float4*>(quats)[g];
        const float s[3] = {scales[3 * g], scales[3 * g + 1], scales[3 * g + 2]};
        float ds[3];
        float4 dq;
        projection_adjoint(P, mx, my, mz, q4, s, d_uv[g * d_uv_stride],
                           d_uv[g * d_uv_stride + 1], d_conic[g * d_conic_stride],
                           d_conic[g * d_conic_stride + 1], d_conic[g * d_conic_stride + 2],
                           dmx, dmy, dmz, ds, dq);
        if (kAccum) {  // d log s = d s * s
            d_scales[3 * g + 0] += ds[0] * s[0];
            d_scales[3 * g + 1] += ds[1] * s[1];
            d_scales[3 * g + 2] += ds[2] * s[2];
            const float op = opac[g];
            d_logit[g] += d_opac[g * d_opac_stride] * (op * (1.0f - op));
        } else {
            d_scales[3 * g + 0] = ds[0];
            d_scales[3 * g + 1] = ds[1];
            d_scales[3 * g + 2] = ds[2];
        }
        float4* dqp = reinterpret_cast<float4*>(d_quats) + g;
        if (kAccum) {
            const float4 o = *dqp;
            *dqp = make_float4(o.x + dq.x, o.y + dq.y, o.z + dq.z, o.w + dq.w);
        } else {
            *dqp = dq;
        }
    } else if (!kAccum) {
        d_scales[3 * g + 0] = 0.f; d_scales[3 * g + 1] = 0.f; d_scales[3 * g + 2] = 0.f;
        reinterpret_cast<float4*>(d_quats)[g] = make_float4(0.f, 0.f, 0.f, 0.f);
    }
    if (kAccum) {
        if (dmx != 0.f || dmy != 0.f || dmz != 0.f) {
            d_means[3 * g + 0] += dmx;
            d_means[3 * g + 1] += dmy;
            d_means[3 * g + 2] += dmz;
        }
    } else {
        d_means[3 * g + 0] = dmx;
        d_means[3 * g + 1] = dmy;
        d_means[3 * g + 2] = dmz;
    }
}

constexpr int kMaxViewsPerLaunch = 16;
struct ViewCams {
    CamParams c[kMaxViewsPerLaunch];
};

// The projection half of preprocess_backward_kernel<true> (deferred SH) for
// several cameras at once: a Gaussian's parameters are read once, its
// per-view adjoints are summed in registers in view order and added into the
// gradient rows once, and each view's ReLU-gated colour gradient goes to
// dpre[v * view_stride + g] for sh_backward_views_kernel. View v's grad2d
// records, valid flags and forward colours start at v * view_stride rows.
// With `filt`, scales and opacities are the activations before Mip-Splatting's
// 3D filter: the projection adjoint runs at the widened scales and the summed
// gradients are carried back through the filter (filter_3d constant).
// Resident 128-thread CTAs per SM the multi-view adjoints' registers are
// held to (0: no cap). Both are bound by load latency, so occupancy pays: 5
// (96 registers, no spills) against none (123 / 105 registers) measured
// 0.257 -> 0.220 ms and 0.279 -> 0.254 ms per step of 8 views; 6 spills.
#ifndef MG_PRE_BWD_MIN_CTAS
#define MG_PRE_BWD_MIN_CTAS 5
#endif
__global__ void __launch_bounds__(kBwdBlock, MG_PRE_BWD_MIN_CTAS)
preprocess_backward_views_kernel(const float* __restrict__ means,
                                 const float* __restrict__ quats,
                                 const float* __restrict__ scales,
                                 const float* __restrict__ opac,
                                 const float* __restrict__ grad2d,
                                 const int32_t* __restrict__ valid,
                                 const float* __restrict__ color, ViewCams cams, int n_views,
                                 int64_t n, int64_t view_stride,
                                 const float* __restrict__ filt, float* __restrict__ d_means,
                                 float* __restrict__ d_quats, float* __restrict__ d_log_scales,
                                 float* __restrict__ d_logit, float* __restrict__ dpre) {
    const int64_t g = (int64_t)blockIdx.x * kBwdBlock + threadIdx.x;
    if (g >= n) return;
    const float mx = means[3 * g], my = means[3 * g + 1], mz = means[3 * g + 2];
    const float4 q4 = reinterpret_cast<const float4*>(quats)[g];
    const float s_act[3] = {scales[3 * g], scales[3 * g + 1], scales[3 * g + 2]};
    const float op = opac[g];
    float s[3] = {s_act[0], s_act[1], s_act[2]};  // the scales the forward projected
    Filter3d fl;
    float f = 0.0f;
    if (filt) {
        f = filt[g];
        fl = filter3d(s_act[0], s_act[1], s_act[2], f);
        s[0] = fl.s[0]; s[1] = fl.s[1]; s[2] = fl.s[2];
    }
    float dmx = 0.f, dmy = 0.f, dmz = 0.f, dop = 0.f;
    // the views' symmetrised covariance gradients, carried to the scales and
    // the quaternion once after the loop (that part is linear in them)
    float dSym[6] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    const CovFrame F = cov_frame(q4, s);
    bool any = false;
    static_assert(MG_G2D_STRIDE == 12 && MG_G2D_UV == 0 && MG_G2D_OPACITY == 2 &&
                      MG_G2D_CONIC == 4 && MG_G2D_COLOR == 8,
                  "the record is read as three float4: uv op abs | conic pad | colour pad");
    for (int v = 0; v < n_views; ++v) {
        const int64_t o = (int64_t)v * view_stride + g;
        // the record's three 16-byte words, the forward colour and the valid
        // flag are loaded together before any of them is used
        const float4* rec = reinterpret_cast<const float4*>(grad2d) + 3 * o;
        const float4 r0 = rec[0], r1 = rec[1], r2 = rec[2];
        const float c0 = color[3 * o + 0], c1 = color[3 * o + 1], c2 = color[3 * o + 2];
        const int32_t ok = valid[o];
        dpre[3 * o + 0] = c0 > 0.f ? r2.x : 0.f;
        dpre[3 * o + 1] = c1 > 0.f ? r2.y : 0.f;
        dpre[3 * o + 2] = c2 > 0.f ? r2.z : 0.f;
        if (ok == 0) continue;
        projection_adjoint_view(cams.c[v], mx, my, mz, F.S, r0.x, r0.y, r1.x, r1.y, r1.z, dmx,
                                dmy, dmz, dSym);
        dop += r0.z;
        any = true;
    }
    if (!any) return;
    float dsa[3];  // d loss / d (projected) scales, all views
    float4 dqa;
    covariance_adjoint(F, s, dSym, dsa, dqa);
    // activation chain: d log s = d s * s, d logit = d op * op (1 - op), through
    // the 3D filter when there is one (s' = sqrt(s^2 + f^2), op' = op coef)
    float dls[3], dl;
    if (filt) {
#pragma unroll
        for (int i = 0; i < 3; ++i)
            dls[i] = (dsa[i] * s_act[i] / fl.s[i] + filter3d_dcoef(fl, s_act[i], f) * (dop * op)) *
                     s_act[i];
        dl = dop * fl.coef * (op * (1.0f - op));
    } else {
#pragma unroll
        for (int i = 0; i < 3; ++i) dls[i] = dsa[i] * s_act[i];
        dl = dop * (op * (1.0f - op));
    }
    d_means[3 * g + 0] += dmx;
    d_means[3 * g + 1] += dmy;
    d_means[3 * g + 2] += dmz;
    float4* dqp = reinterpret_cast<float4*>(d_quats) + g;
    const float4 oq = *dqp;
    *dqp = make_float4(oq.x + dqa.x, oq.y + dqa.y, oq.z + dqa.z, oq.w + dqa.w);
    d_log_scales[3 * g + 0] += dls[0];
    d_log_scales[3 * g + 1] += dls[1];
    d_log_scales[3 * g + 2] += dls[2];
    d_logit[g] += dl;
}

constexpr int kMaxViews = 64;
struct ViewCentres {
    float c[kMaxViews][3];
};

// Deferred SH adjoint over all views of a step: per Gaussian, the
// coefficients are staged once (per warp, as in the per-view kernel), the
// gradient rows are summed over the views in registers and written once.
// The kernel waits on loads: four views' colour gradients in flight at once
// with 128 registers (4 CTAs of 128 threads per SM) measured 228 -> 174 us
// per step of 8 views against one view at a time at 96 registers; two at 96
// registers 181 us; four at 96 spill.
#ifndef MG_SH_BWD_MIN_CTAS
#define MG_SH_BWD_MIN_CTAS 4
#endif
__global__ void __launch_bounds__(kBwdBlock, MG_SH_BWD_MIN_CTAS)
sh_backward_views_kernel(const float* __restrict__ means, const float* __restrict__ sh_dc,
                         const float* __restrict__ sh_rest, int sh_degree, int64_t n,
                         ViewCentres centres, const float* __restrict__ dpre, int n_views,
                         int64_t view_stride, float* __restrict__ d_means,
                         float* __restrict__ d_sh_dc, float* __restrict__ d_sh_rest) {
    __shared__ __align__(16) float s_sh[kBwdBlock / 32][32 * 45];
    const int lane = threadIdx.x & 31, wib = threadIdx.x >> 5;
    const int64_t g = (int64_t)blockIdx.x * kBwdBlock + threadIdx.x;
    const int64_t g0 = g - lane;
    const bool in = g < n;
    const int64_t warp_n = min((int64_t)32, n - g0);
    float* blk = s_sh[wib];
    const int total = (int)max((int64_t)0, warp_n) * 45;
    warp_copy_to_shared(sh_rest + g0 * 45, total, blk, lane);
    const int nb = (sh_degree + 1) * (sh_degree + 1);
    float acc[16][3];
#pragma unroll
    for (int i = 0; i < 16; ++i) acc[i][0] = acc[i][1] = acc[i][2] = 0.f;
    float dmx = 0.f, dmy = 0.f, dmz = 0.f;
    if (in) {
        const float mx = means[3 * g], my = means[3 * g + 1], mz = means[3 * g + 2];
        const float* dc = sh_dc + 3 * g;
        const float* rest = blk + lane * 45;
        // the colour gradients of up to kShViewBatch views are loaded together
        // (their loads in flight at once) before any of them is used
        constexpr int kShViewBatch = 4;
        for (int v0 = 0; v0 < n_views; v0 += kShViewBatch) {
        float e[kShViewBatch][3];
#pragma unroll
        for (int j = 0; j < kShViewBatch; ++j) {
            e[j][0] = e[j][1] = e[j][2] = 0.f;
            if (v0 + j < n_views) {
                const float* dp = dpre + ((int64_t)(v0 + j) * view_stride + g) * 3;
                e[j][0] = dp[0]; e[j][1] = dp[1]; e[j][2] = dp[2];
            }
        }
#pragma unroll
        for (int j = 0; j < kShViewBatch; ++j) {
            const int v = v0 + j;
            const float er = e[j][0], eg = e[j][1], eb = e[j][2];
            if (v >= n_views || (er == 0.f && eg == 0.f && eb == 0.f)) continue;
            const float dvx = mx - centres.c[v][0], dvy = my - centres.c[v][1],
                        dvz = mz - centres.c[v][2];
            const float len = fmaxf(sqrtf(dvx * dvx + dvy * dvy + dvz * dvz), 1e-12f);
            const float inv_len = 1.0f / len;
            const float x = dvx * inv_len, y = dvy * inv_len, z = dvz * inv_len;
            float B[16];
            sh_basis(sh_degree, x, y, z, B);
            float ddx = 0.f, ddy = 0.f, ddz = 0.f;
#pragma unroll
            for (int i = 0; i < 16; ++i) {
                if (i < nb) {
                    const float* row = i == 0 ? dc : rest + (i - 1) * 3;
                    acc[i][0] += B[i] * er; acc[i][1] += B[i] * eg; acc[i][2] += B[i] * eb;
                    float gx, gy, gz;
                    sh_basis_grad(i, x, y, z, gx, gy, gz);
                    const float k = row[0] * er + row[1] * eg + row[2] * eb;
                    ddx += gx * k; ddy += gy * k; ddz += gz * k;
                }
            }
            const float dd = x * ddx + y * ddy + z * ddz;
            dmx += (ddx - x * dd) * inv_len;
            dmy += (ddy - y * dd) * inv_len;
            dmz += (ddz - z * dd) * inv_len;
        }
        }
        if (dmx != 0.f || dmy != 0.f || dmz != 0.f) {
            d_means[3 * g] += dmx; d_means[3 * g + 1] += dmy; d_means[3 * g + 2] += dmz;
        }
        d_sh_dc[3 * g] = acc[0][0]; d_sh_dc[3 * g + 1] = acc[0][1]; d_sh_dc[3 * g + 2] = acc[0][2];
    }
    __syncwarp();
    if (in) {
#pragma unroll
        for (int i = 1; i < 16; ++i) {
            float* r = blk + lane * 45 + (i - 1) * 3;
            r[0] = acc[i][0]; r[1] = acc[i][1]; r[2] = acc[i][2];
        }
    }
    __syncwarp();
    warp_copy_from_shared(blk, total, d_sh_rest + g0 * 45, lane);
}

}  // namespace

}  // namespace mg

using namespace mg;

extern "C" mg_status mg_preprocess_backward(
    const float* means, const float* quats, const float* scales, const float* sh_dc,
    const float* sh_rest, mg_sh_layout shl, const float* d_uv, int64_t d_uv_stride,
    const float* d_conic, int64_t d_conic_stride, const float* d_color,
    int64_t d_color_stride, const int32_t* valid, const mg_camera* cam, int32_t sh_degree,
    int64_t n, float* d_means, float* d_quats, float* d_scales, float* d_sh_dc,
    float* d_sh_rest, mg_stream_t stream) {
    MG_REQUIRE(cam != nullptr, "preprocess_backward: null camera");
    MG_REQUIRE(sh_degree <= 3, "preprocess_backward: sh_degree must be <= 3");
    if (n == 0) return MG_OK;
    MG_REQUIRE(means && quats && scales && d_uv && d_conic && valid && d_means && d_quats &&
                   d_scales,
               "preprocess_backward: null pointer");
    MG_REQUIRE((reinterpret_cast<uintptr_t>(quats) & 15u) == 0u &&
                   (reinterpret_cast<uintptr_t>(d_quats) & 15u) == 0u,
               "preprocess_backward: quats must be 16-byte aligned");
    const bool fused = shl.stride_dc == 16 && shl.stride_rest == 16 && shl.offset_rest == 1;
    const bool split = shl.stride_dc == 1 && shl.stride_rest == 15 && shl.offset_rest == 0;
    if (sh_degree >= 0 && d_color != nullptr) {
        MG_REQUIRE(fused || split,
                   "SH must be either one (N,16,3) tensor or (N,1,3)+(N,15,3)");
        MG_REQUIRE(sh_dc && sh_rest && d_sh_dc && d_sh_rest,
                   "preprocess_backward: null SH pointer");
        if (fused)
            MG_REQUIRE(sh_rest == sh_dc && d_sh_rest == d_sh_dc,
                       "preprocess_backward: the fused SH layout passes one tensor twice");
    }
    const CamParams P = make_cam_params(*cam);
    preprocess_backward_kernel<false><<<ceil_div(n, kBwdBlock), kBwdBlock, 0,
                                        reinterpret_cast<cudaStream_t>(stream)>>>(
        means, quats, scales, sh_dc, sh_rest, shl, d_uv, d_uv_stride, d_conic, d_conic_stride,
        d_color, d_color_stride, valid, P, sh_degree, n, d_means, d_quats, d_scales, d_sh_dc,
        d_sh_rest, fused ? 1 : 0, split ? 1 : 0, nullptr, nullptr, 0, nullptr, nullptr, nullptr);
    return check_launch("preprocess_backward");
}

extern "C" mg_status mg_preprocess_backward_accumulate(
    const float* means, const float* quats, const float* scales, const float* opacities,
    const float* sh_dc, const float* sh_rest, const float* grad2d, const int32_t* valid,
    const mg_camera* cam, int32_t sh_degree, int64_t n, float* d_means, float* d_quats,
    float* d_log_scales, float* d_logit_opac, float* d_sh_dc, float* d_sh_rest,
    const float* color, float* dpre_out, mg_stream_t stream) {
    MG_REQUIRE(cam != nullptr, "preprocess_backward_accumulate: null camera");
    MG_REQUIRE(sh_degree <= 3, "preprocess_backward_accumulate: sh_degree must be <= 3");
    if (n == 0) return MG_OK;
    MG_REQUIRE(means && quats && scales && opacities && grad2d && valid && d_means && d_quats &&
                   d_log_scales && d_logit_opac,
               "preprocess_backward_accumulate: null pointer");
    MG_REQUIRE((reinterpret_cast<uintptr_t>(quats) & 15u) == 0u &&
                   (reinterpret_cast<uintptr_t>(d_quats) & 15u) == 0u,
               "preprocess_backward_accumulate: quats must be 16-byte aligned");
    const bool deferred = dpre_out != nullptr;
    const bool with_sh = sh_degree >= 0 && sh_dc != nullptr;
    if (deferred)
        MG_REQUIRE(color != nullptr, "preprocess_backward_accumulate: deferred SH needs color");
    else if (with_sh)
        MG_REQUIRE(sh_rest && d_sh_dc && d_sh_rest,
                   "preprocess_backward_accumulate: null SH pointer");
    const CamParams P = make_cam_params(*cam);
    preprocess_backward_kernel<true><<<ceil_div(n, kBwdBlock), kBwdBlock, 0,
                                       reinterpret_cast<cudaStream_t>(stream)>>>(
        means, quats, scales, with_sh ? sh_dc : nullptr, sh_rest, SH_SPLIT_LAYOUT,
        grad2d + MG_G2D_UV, MG_G2D_STRIDE, grad2d + MG_G2D_CONIC, MG_G2D_STRIDE,
        (with_sh || deferred) ? grad2d + MG_G2D_COLOR : nullptr, MG_G2D_STRIDE, valid, P,
        with_sh ? sh_degree : -1, n, d_means, d_quats, d_log_scales, d_sh_dc, d_sh_rest, 0, 1,
        opacities, grad2d + MG_G2D_OPACITY, MG_G2D_STRIDE, d_logit_opac, color, dpre_out);
    return check_launch("preprocess_backward_accumulate");
}

extern "C" mg_status mg_preprocess_backward_views(
    const float* means, const float* quats, const float* scales, const float* opacities,
    const float* grad2d, const int32_t* valid, const float* color, const mg_camera* cams,
    int32_t n_views, int64_t n, int64_t view_stride, const float* filter_3d, float* d_means,
    float* d_quats, float* d_log_scales, float* d_logit_opac, float* dpre_out,
    mg_stream_t stream) {
    MG_REQUIRE(n_views >= 0, "preprocess_backward_views: negative view count");
    if (n == 0 || n_views == 0) return MG_OK;
    MG_REQUIRE(cams != nullptr, "preprocess_backward_views: null cameras");
    MG_REQUIRE(view_stride >= n, "preprocess_backward_views: view_stride below n");
    MG_REQUIRE(means && quats && scales && opacities && grad2d && valid && color && d_means &&
                   d_quats && d_log_scales && d_logit_opac && dpre_out,
               "preprocess_backward_views: null pointer");
    MG_REQUIRE((reinterpret_cast<uintptr_t>(quats) & 15u) == 0u &&
                   (reinterpret_cast<uintptr_t>(d_quats) & 15u) == 0u &&
                   (reinterpret_cast<uintptr_t>(grad2d) & 15u) == 0u,
               "preprocess_backward_views: quats and grad2d must be 16-byte aligned");
    const cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    for (int v0 = 0; v0 < n_views; v0 += kMaxViewsPerLaunch) {
        const int nv = n_views - v0 < kMaxViewsPerLaunch ? n_views - v0 : kMaxViewsPerLaunch;
        ViewCams vc;
        for (int k = 0; k < nv; ++k) vc.c[k] = make_cam_params(cams[v0 + k]);
        const int64_t o = (int64_t)v0 * view_stride;
        preprocess_backward_views_kernel<<<ceil_div(n, kBwdBlock), kBwdBlock, 0, st>>>(
            means, quats, scales, opacities, grad2d + o * MG_G2D_STRIDE, valid + o,
            color + 3 * o, vc, nv, n, view_stride, filter_3d, d_means, d_quats, d_log_scales,
            d_logit_opac, dpre_out + 3 * o);
        MG_TRY(check_launch("preprocess_backward_views"));
    }
    return MG_OK;
}

extern "C" mg_status mg_sh_backward_views(const float* means, const float* sh_dc,
                                          const float* sh_rest, int32_t sh_degree, int64_t n,
                                          const float* cam_centers, const float* dpre,
                                          int32_t n_views, int64_t view_stride, float* d_means,
                                          float* d_sh_dc, float* d_sh_rest, mg_stream_t stream) {
    MG_REQUIRE(n_views >= 0 && n_views <= kMaxViews, "sh_backward_views: at most 64 views");
    MG_REQUIRE(view_stride >= n, "sh_backward_views: view_stride below n");
    MG_REQUIRE(sh_degree >= 0 && sh_degree <= 3, "sh_backward_views: sh_degree must be 0..3");
    if (n == 0) return MG_OK;
    MG_REQUIRE(means && sh_dc && sh_rest && d_means && d_sh_dc && d_sh_rest &&
                   (n_views == 0 || (cam_centers && dpre)),
               "sh_backward_views: null pointer");
    ViewCentres c;
    for (int v = 0; v < n_views; ++v)
        for (int k = 0; k < 3; ++k) c.c[v][k] = cam_centers[3 * v + k];
    sh_backward_views_kernel<<<ceil_div(n, kBwdBlock), kBwdBlock, 0,
                               reinterpret_cast<cudaStream_t>(stream)>>>(
        means, sh_dc, sh_rest, sh_degree, n, c, dpre, n_views, view_stride, d_means, d_sh_dc,
        d_sh_rest);
    return check_launch("sh_backward_views");
}
