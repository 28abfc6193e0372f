// Mip-Splatting's 3D smoothing filter (metal_gauss/mipfilter.py): the
// per-Gaussian band limit of the training cameras and the reparameterisation
// of scales and opacity it defines, with its adjoint.
//
//   filter_3d = min over the cameras that see it of depth / max focal * sqrt(0.2)
//   scales'   = sqrt(scales^2 + filter_3d^2)
//   opacity'  = opacity * sqrt(clamp(prod(scales^2) / prod(scales'^2), 0, 1))
#include <algorithm>
#include <cmath>

#include "filter3d.cuh"
#include "kernels.cuh"

namespace mg {

namespace {

constexpr int kMaxFilterViews = 64;
struct FilterCams {
    float R[kMaxFilterViews][12];  // viewmat rows 0..2 (rotation | translation)
    float fx[kMaxFilterViews], fy[kMaxFilterViews], cx[kMaxFilterViews], cy[kMaxFilterViews];
    float W[kMaxFilterViews], H[kMaxFilterViews];
};

// Pass 1 (mipfilter.py:49-68): the smallest camera depth among the views in
// whose (margin-widened) frame the mean projects in front of `near`, +inf
// when none. Cameras come in chunks of at most kMaxFilterViews, each passed
// by value in the launch's parameters (4.6 KB; sm_100 takes up to 32 KB), so
// the launches need no device copy of them and no synchronisation: a chunk
// after the first continues from the running minimum in dist, and the last
// one puts the largest finite minimum over all Gaussians into *max_bits
// (positive floats order like their bit patterns).
__global__ void filter_depth_kernel(const float* __restrict__ means, int64_t n,
                                    const __grid_constant__ FilterCams cams, int n_views,
                                    float near, float margin, int first, int last,
                                    float* __restrict__ dist, uint32_t* __restrict__ max_bits) {
    __shared__ FilterCams s;
    for (int i = threadIdx.x; i < (int)(sizeof(FilterCams) / 4); i += blockDim.x)
        reinterpret_cast<float*>(&s)[i] = reinterpret_cast<const float*>(&cams)[i];
    __syncthreads();
    const int64_t g = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    float d = __int_as_float(0x7f800000);
    if (g < n) {
        if (!first) d = dist[g];
        const float x = means[3 * g], y = means[3 * g + 1], z = means[3 * g + 2];
        for (int v = 0; v < n_views; ++v) {
            const float* R = s.R[v];
            const float px = R[0] * x + R[1] * y + R[2] * z + R[3];
            const float py = R[4] * x + R[5] * y + R[6] * z + R[7];
            const float pz = R[8] * x + R[9] * y + R[10] * z + R[11];
            const float zc = fmaxf(pz, 1e-6f);
            const float u = s.fx[v] * px / zc + s.cx[v];
            const float w = s.fy[v] * py / zc + s.cy[v];
            const float Wv = s.W[v], Hv = s.H[v];
            const bool inview = pz > near && u > -margin * Wv && u < (1.0f + margin) * Wv &&
                                w > -margin * Hv && w < (1.0f + margin) * Hv;
            if (inview) d = fminf(d, pz);
        }
        dist[g] = d;
    }
    if (!last) return;  // (block-uniform)
    // block maximum of the finite depths, then one atomic
    uint32_t m = (g < n && d < __int_as_float(0x7f800000)) ? __float_as_uint(d) : 0u;
    m = __reduce_max_sync(0xffffffffu, m);
    __shared__ uint32_t s_max;
    if (threadIdx.x == 0) s_max = 0u;
    __syncthreads();
    if ((threadIdx.x & 31) == 0 && m) atomicMax(&s_max, m);
    __syncthreads();
    if (threadIdx.x == 0 && s_max) atomicMax(max_bits, s_max);
}

// Pass 2 (mipfilter.py:70-76): unseen Gaussians take the largest depth any
// Gaussian got (all take 1 when none was seen), then depth / focal *
// sqrt(0.2), rounded as the reference's float32 tensor arithmetic is.
__global__ void filter_finish_kernel(float* __restrict__ dist, int64_t n,
                                     const uint32_t* __restrict__ max_bits, float focal,
                                     float k) {
    const int64_t g = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (g >= n) return;
    const uint32_t mb = *max_bits;
    float d = dist[g];
    if (mb == 0u) d = 1.0f;
    else if (!(d < __int_as_float(0x7f800000))) d = __uint_as_float(mb);
    dist[g] = __fmul_rn(__fdiv_rn(d, focal), k);
}

__global__ void apply_filter_kernel(const float* __restrict__ scales,
                                    const float* __restrict__ opac,
                                    const float* __restrict__ filt, int64_t n,
                                    float* __restrict__ out_scales,
                                    float* __restrict__ out_opac) {
    const int64_t g = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (g >= n) return;
    const Filter3d f = filter3d(scales[3 * g], scales[3 * g + 1], scales[3 * g + 2], filt[g]);
    out_scales[3 * g] = f.s[0];
    out_scales[3 * g + 1] = f.s[1];
    out_scales[3 * g + 2] = f.s[2];
    out_opac[g] = opac[g] * f.coef;
}

__global__ void apply_filter_backward_kernel(const float* __restrict__ scales,
                                             const float* __restrict__ opac,
                                             const float* __restrict__ filt,
                                             const float* __restrict__ d_fs,
                                             const float* __restrict__ d_fo, int64_t n,
                                             float* __restrict__ d_scales,
                                             float* __restrict__ d_opac) {
    const int64_t g = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (g >= n) return;
    const float s[3] = {scales[3 * g], scales[3 * g + 1], scales[3 * g + 2]};
    const float f = filt[g];
    const Filter3d fl = filter3d(s[0], s[1], s[2], f);
    const float dfo = d_fo[g], op = opac[g];
#pragma unroll
    for (int i = 0; i < 3; ++i) {
        const float ds = d_fs[3 * g + i];
        d_scales[3 * g + i] = ds * s[i] / fl.s[i] + filter3d_dcoef(fl, s[i], f) * (dfo * op);
    }
    d_opac[g] = dfo * fl.coef;
}

}  // namespace

}  // namespace mg

using namespace mg;

extern "C" mg_status mg_compute_3d_filter(const float* means, int64_t n, const mg_camera* cams,
                                          int32_t n_views, float near_plane, float margin,
                                          float* filter_out, void* scratch, size_t scratch_bytes,
                                          mg_stream_t stream) {
    MG_REQUIRE(n >= 0 && n_views >= 0, "compute_3d_filter: negative count");
    if (n == 0) return MG_OK;
    MG_REQUIRE(means && filter_out && (n_views == 0 || cams), "compute_3d_filter: null pointer");
    MG_REQUIRE(scratch && scratch_bytes >= mg_compute_3d_filter_scratch_bytes(),
               "compute_3d_filter: scratch too small");
    float focal = 0.0f;
    for (int v = 0; v < n_views; ++v)
        focal = std::max(focal, std::max(cams[v].fx, cams[v].fy));
    if (!(focal > 0.0f)) focal = 1.0f;
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    uint32_t* max_bits = static_cast<uint32_t*>(scratch);
    if (cudaMemsetAsync(max_bits, 0, sizeof(uint32_t), st) != cudaSuccess)
        return check_launch("compute_3d_filter memset");
    // cameras in chunks of kMaxFilterViews (one launch each, the running
    // minimum carried in filter_out); no cameras: one launch that sees none
    const int chunks = std::max(1, (n_views + kMaxFilterViews - 1) / kMaxFilterViews);
    for (int c = 0; c < chunks; ++c) {
        const int v0 = c * kMaxFilterViews;
        const int nv = std::min(kMaxFilterViews, n_views - v0);
        FilterCams h{};
        for (int k = 0; k < nv; ++k) {
            const mg_camera& cm = cams[v0 + k];
            for (int r = 0; r < 3; ++r)
                for (int q = 0; q < 4; ++q) h.R[k][4 * r + q] = cm.viewmat[4 * r + q];
            h.fx[k] = cm.fx; h.fy[k] = cm.fy; h.cx[k] = cm.cx; h.cy[k] = cm.cy;
            h.W[k] = (float)cm.width; h.H[k] = (float)cm.height;
        }
        filter_depth_kernel<<<ceil_div(n, 256), 256, 0, st>>>(
            means, n, h, std::max(nv, 0), near_plane, margin, c == 0 ? 1 : 0,
            c == chunks - 1 ? 1 : 0, filter_out, max_bits);
        MG_TRY(check_launch("compute_3d_filter depth"));
    }
    filter_finish_kernel<<<ceil_div(n, 256), 256, 0, st>>>(filter_out, n, max_bits, focal,
                                                          std::sqrt(0.2f));
    return check_launch("compute_3d_filter finish");
}

extern "C" size_t mg_compute_3d_filter_scratch_bytes(void) { return 256; }

extern "C" mg_status mg_apply_3d_filter(const float* scales, const float* opacities,
                                        const float* filter_3d, int64_t n, float* out_scales,
                                        float* out_opacities, mg_stream_t stream) {
    MG_REQUIRE(n >= 0, "apply_3d_filter: negative count");
    if (n == 0) return MG_OK;
    MG_REQUIRE(scales && opacities && filter_3d && out_scales && out_opacities,
               "apply_3d_filter: null pointer");
    apply_filter_kernel<<<ceil_div(n, 256), 256, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
        scales, opacities, filter_3d, n, out_scales, out_opacities);
    return check_launch("apply_3d_filter");
}

extern "C" mg_status mg_apply_3d_filter_backward(const float* scales, const float* opacities,
                                                 const float* filter_3d,
                                                 const float* d_out_scales,
                                                 const float* d_out_opacities, int64_t n,
                                                 float* d_scales, float* d_opacities,
                                                 mg_stream_t stream) {
    MG_REQUIRE(n >= 0, "apply_3d_filter_backward: negative count");
    if (n == 0) return MG_OK;
    MG_REQUIRE(scales && opacities && filter_3d && d_out_scales && d_out_opacities && d_scales &&
                   d_opacities,
               "apply_3d_filter_backward: null pointer");
    apply_filter_backward_kernel<<<ceil_div(n, 256), 256, 0,
                                   reinterpret_cast<cudaStream_t>(stream)>>>(
        scales, opacities, filter_3d, d_out_scales, d_out_opacities, n, d_scales, d_opacities);
    return check_launch("apply_3d_filter_backward");
}
