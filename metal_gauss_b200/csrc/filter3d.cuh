// Mip-Splatting 3D filter algebra (metal_gauss/mipfilter.py:79-93), shared by
// the filter entry points and the training engine's projection adjoint.
#pragma once

namespace mg {

struct Filter3d {
    float s[3];  // sqrt(scales^2 + f^2)
    float s2[3], s2f[3];
    float coef;  // sqrt(clamp(prod(scales^2) / prod(scales^2 + f^2), 0, 1))
};

// The widened scales and the opacity factor, in the reference's order of
// operations (squares, sums, left-to-right products, clamp, square root).
__device__ __forceinline__ Filter3d filter3d(float sx, float sy, float sz, float f) {
    Filter3d r;
    const float f2 = __fmul_rn(f, f);
    r.s2[0] = __fmul_rn(sx, sx);
    r.s2[1] = __fmul_rn(sy, sy);
    r.s2[2] = __fmul_rn(sz, sz);
#pragma unroll
    for (int i = 0; i < 3; ++i) {
        r.s2f[i] = __fadd_rn(r.s2[i], f2);
        r.s[i] = __fsqrt_rn(r.s2f[i]);
    }
    const float num = __fmul_rn(__fmul_rn(r.s2[0], r.s2[1]), r.s2[2]);
    const float den = __fmul_rn(__fmul_rn(r.s2f[0], r.s2f[1]), r.s2f[2]);
    r.coef = __fsqrt_rn(fminf(fmaxf(__fdiv_rn(num, den), 0.0f), 1.0f));
    return r;
}

// d coef / d scale_i = coef * f^2 / (scale_i * (scale_i^2 + f^2)).
__device__ __forceinline__ float filter3d_dcoef(const Filter3d& r, float s, float f) {
    return r.coef * (f * f) / (s * (s * s + f * f));
}

}  // namespace mg
