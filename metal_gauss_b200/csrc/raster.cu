// Tile rasterisation, forward and backward (rasterize.metal:61-340).
//
// One CTA per screen tile. Full 8x4 pixel blocks per warp when the tile side
// is a multiple of 8 (compact warps see fewer Gaussians); otherwise row-major
// pixels with the CTA padded to whole warps. Each batch of up to kBatch
// Gaussians of the tile's depth-sorted list is staged into shared memory with
// one gather per Gaussian, then every pixel walks the batch from shared memory.
//
// Forward: front to back, alpha = min(0.999, op exp(power)), skip power > 0
// or alpha < 1/255, stop a pixel once T < 1e-4 and record the stop INDEX;
// the CTA leaves the list once every pixel has stopped.
//
// Backward: back to front from the CTA's largest stop index, recovering T by
// division. Per Gaussian, each warp reduces its 32 pixels' contributions with
// a 16-slot butterfly reduce-scatter (16 shuffles for all components instead
// of 5 per component), adds the result into a per-Gaussian shared-memory
// accumulator, and after the batch one thread per Gaussian adds the record
// to global memory with three 16-byte vector atomics.
#include "kernels.cuh"

namespace mg {

namespace {

constexpr int kBatch = 256;

struct __align__(16) StagedGauss {
    float u, v, op, pad;
    float ca, cb, cc, pad2;
    float r, g, b, pad3;
};

// Quadratic form and alpha for one (pixel, Gaussian) pair. Shared by the
// forward and the backward and written with explicitly rounded operations, so
// both passes take bit-identical blend decisions.
__device__ __forceinline__ float pair_power(float dx, float dy, float ca, float cb,
                                            float cc) {
    const float q = __fmaf_rn(ca, __fmul_rn(dx, dx),
                              __fmaf_rn(__fmul_rn(2.0f, cb), __fmul_rn(dx, dy),
                                        __fmul_rn(cc, __fmul_rn(dy, dy))));
    return __fmul_rn(-0.5f, q);
}

__device__ __forceinline__ float pair_gauss(float power) { return __expf(power); }

template <int TILE>
struct TileGeom {
    static constexpr int kPix = TILE * TILE;
    static constexpr int kThreads = (kPix + 31) / 32 * 32;
    __device__ __forceinline__ static void pixel(int tid, int& lx, int& ly) {
        if (TILE % 8 == 0) {
            const int warp = tid >> 5, lane = tid & 31, bx = TILE / 8;
            lx = (warp % bx) * 8 + (lane & 7);
            ly = (warp / bx) * 4 + (lane >> 3);
        } else if (tid < kPix) {
            lx = tid % TILE;
            ly = tid / TILE;
        } else {
            lx = TILE;  // padding thread, outside the tile
            ly = TILE;
        }
    }
};

template <int TILE>
__global__ void __launch_bounds__(TileGeom<TILE>::kThreads)
raster_forward_kernel(const float2* __restrict__ uv, const float* __restrict__ conic,
                      const float* __restrict__ opacity, const float* __restrict__ color,
                      const int32_t* __restrict__ ids,
                      const int32_t* __restrict__ offsets, int W, int H, int tiles_x,
                      int has_bg, float bg_r, float bg_g, float bg_b,
                      float* __restrict__ out_rgb, float* __restrict__ out_alpha,
                      float* __restrict__ out_T, int32_t* __restrict__ out_stop) {
    using G = TileGeom<TILE>;
    __shared__ StagedGauss s_g[kBatch];
    const int tid = threadIdx.x;
    const int tile_id = blockIdx.x;
    const int tx = tile_id % tiles_x, ty = tile_id / tiles_x;
    int lx, ly;
    G::pixel(tid, lx, ly);
    const bool in_tile = lx < TILE && ly < TILE;
    const int px = tx * TILE + lx, py = ty * TILE + ly;
    const bool inimg = in_tile && px < W && py < H;
    const int start = offsets[tile_id], end = offsets[tile_id + 1];
    const float fx = (float)px + 0.5f, fy = (float)py + 0.5f;

    float T = 1.0f, ar = 0.0f, ag = 0.0f, ab = 0.0f, aa = 0.0f;
    int stop = start;
    bool done = !inimg;

    for (int base = start; base < end; base += kBatch) {
        const int n = min(kBatch, end - base);
        for (int t = tid; t < n; t += G::kThreads) {
            const int g = ids[base + t];
            const float2 m = uv[g];
            StagedGauss s;
            s.u = m.x; s.v = m.y; s.op = opacity[g]; s.pad = 0.f;
            s.ca = conic[3 * g]; s.cb = conic[3 * g + 1]; s.cc = conic[3 * g + 2]; s.pad2 = 0.f;
            s.r = color[3 * g]; s.g = color[3 * g + 1]; s.b = color[3 * g + 2]; s.pad3 = 0.f;
            s_g[t] = s;
        }
        __syncthreads();
        if (!done) {
            for (int j = 0; j < n; ++j) {
                const StagedGauss& s = s_g[j];
                const float power = pair_power(fx - s.u, fy - s.v, s.ca, s.cb, s.cc);
                if (power > 0.0f) continue;
                const float alpha = fminf(0.999f, s.op * pair_gauss(power));
                if (alpha < 1.0f / 255.0f) continue;
                const float w = alpha * T;
                ar += w * s.r; ag += w * s.g; ab += w * s.b;
                aa += w;
                T *= (1.0f - alpha);
                stop = base + j + 1;
                if (T < 1e-4f) { done = true; break; }
            }
        }
        if (__syncthreads_count(done) == G::kThreads) break;
    }
    if (!inimg) return;
    const int64_t o = (int64_t)py * W + px;
    if (has_bg) {
        const float k = fmaxf(1.0f - aa, 0.0f);
        ar = ar + k * bg_r; ag = ag + k * bg_g; ab = ab + k * bg_b;
    }
    out_rgb[3 * o + 0] = ar;
    out_rgb[3 * o + 1] = ag;
    out_rgb[3 * o + 2] = ab;
    out_alpha[o] = aa;
    out_T[o] = T;
    out_stop[o] = stop;
}

// 16-slot butterfly reduce-scatter across the warp: on return, lanes 2s and
// 2s+1 hold the warp sum of slot s.
__device__ __forceinline__ float reduce_scatter16(float (&v)[16], int lane) {
#pragma unroll
    for (int k = 0; k < 8; ++k) {
        const bool hi = lane & 16;
        const float send = hi ? v[k] : v[k + 8];
        const float keep = hi ? v[k + 8] : v[k];
        v[k] = keep + __shfl_xor_sync(0xffffffffu, send, 16);
    }
#pragma unroll
    for (int k = 0; k < 4; ++k) {
        const bool hi = lane & 8;
        const float send = hi ? v[k] : v[k + 4];
        const float keep = hi ? v[k + 4] : v[k];
        v[k] = keep + __shfl_xor_sync(0xffffffffu, send, 8);
    }
#pragma unroll
    for (int k = 0; k < 2; ++k) {
        const bool hi = lane & 4;
        const float send = hi ? v[k] : v[k + 2];
        const float keep = hi ? v[k + 2] : v[k];
        v[k] = keep + __shfl_xor_sync(0xffffffffu, send, 4);
    }
    {
        const bool hi = lane & 2;
        const float send = hi ? v[0] : v[1];
        const float keep = hi ? v[1] : v[0];
        v[0] = keep + __shfl_xor_sync(0xffffffffu, send, 2);
    }
    return v[0] + __shfl_xor_sync(0xffffffffu, v[0], 1);
}

template <int TILE>
__global__ void __launch_bounds__(TileGeom<TILE>::kThreads)
raster_backward_kernel(const float2* __restrict__ uv, const float* __restrict__ conic,
                       const float* __restrict__ opacity, const float* __restrict__ color,
                       const int32_t* __restrict__ ids,
                       const int32_t* __restrict__ offsets,
                       const float* __restrict__ final_T,
                       const int32_t* __restrict__ stop_idx,
                       const float* __restrict__ grad_rgb,
                       const float* __restrict__ grad_alpha, int W, int H, int tiles_x,
                       int has_bg, float bg_r, float bg_g, float bg_b,
                       const float* __restrict__ alpha_fwd, int want_absgrad,
                       float* __restrict__ grad2d) {
    using G = TileGeom<TILE>;
    __shared__ StagedGauss s_g[kBatch];
    __shared__ int32_t s_id[kBatch];
    __shared__ __align__(16) float s_acc[kBatch][MG_G2D_STRIDE];
    __shared__ int s_max_stop;
    const int tid = threadIdx.x, lane = tid & 31;
    const int tile_id = blockIdx.x;
    const int tx = tile_id % tiles_x, ty = tile_id / tiles_x;
    int lx, ly;
    G::pixel(tid, lx, ly);
    const bool in_tile = lx < TILE && ly < TILE;
    const int px = tx * TILE + lx, py = ty * TILE + ly;
    const bool inimg = in_tile && px < W && py < H;
    const int start = offsets[tile_id], end = offsets[tile_id + 1];
    const float fx = (float)px + 0.5f, fy = (float)py + 0.5f;
    const int64_t o = inimg ? (int64_t)py * W + px : 0;

    float T = inimg ? final_T[o] : 1.0f;
    const int my_stop = inimg ? stop_idx[o] : start;
    float gr = 0.f, gg = 0.f, gb = 0.f, ga = 0.f;
    if (inimg) {
        gr = grad_rgb[3 * o]; gg = grad_rgb[3 * o + 1]; gb = grad_rgb[3 * o + 2];
        ga = grad_alpha ? grad_alpha[o] : 0.0f;
        // rgb_out = rgb + max(1 - alpha, 0) * bg  =>  d alpha -= <d rgb, bg>
        if (has_bg && 1.0f - alpha_fwd[o] >= 0.0f) ga -= gr * bg_r + gg * bg_g + gb * bg_b;
    }
    const int warp_stop = __reduce_max_sync(0xffffffffu, my_stop);
    if (tid == 0) s_max_stop = start;
    __syncthreads();
    if (lane == 0) atomicMax(&s_max_stop, warp_stop);
    __syncthreads();
    const int max_stop = s_max_stop;
    if (max_stop <= start) return;

    float sr = 0.f, sg = 0.f, sb = 0.f, sa = 0.f;  // suffix colour / alpha
    const int last_batch = (max_stop - 1 - start) / kBatch;
    for (int bi = last_batch; bi >= 0; --bi) {
        const int base = start + bi * kBatch;
        const int n = min(kBatch, end - base);
        __syncthreads();
        for (int t = tid; t < n; t += G::kThreads) {
            const int g = ids[base + t];
            const float2 m = uv[g];
            StagedGauss s;
            s.u = m.x; s.v = m.y; s.op = opacity[g]; s.pad = 0.f;
            s.ca = conic[3 * g]; s.cb = conic[3 * g + 1]; s.cc = conic[3 * g + 2]; s.pad2 = 0.f;
            s.r = color[3 * g]; s.g = color[3 * g + 1]; s.b = color[3 * g + 2]; s.pad3 = 0.f;
            s_g[t] = s;
            s_id[t] = g;
            float4* a = reinterpret_cast<float4*>(s_acc[t]);
            a[0] = a[1] = a[2] = make_float4(0.f, 0.f, 0.f, 0.f);
        }
        __syncthreads();
        const int jtop = min(n, warp_stop - base) - 1;
        for (int j = jtop; j >= 0; --j) {
            const int i = base + j;
            const StagedGauss& s = s_g[j];
            const float dx = fx - s.u, dy = fy - s.v;
            const float power = pair_power(dx, dy, s.ca, s.cb, s.cc);
            const float gauss = pair_gauss(fminf(power, 0.0f));
            const float alpha_raw = s.op * gauss;
            const bool clamped = alpha_raw > 0.999f;
            const float alpha = fminf(0.999f, alpha_raw);
            const bool active = inimg && (i < my_stop) && (power <= 0.0f) &&
                                (alpha >= 1.0f / 255.0f);
            if (__ballot_sync(0xffffffffu, active) == 0u) continue;
            float v[16];
#pragma unroll
            for (int k = 0; k < 16; ++k) v[k] = 0.0f;
            if (active) {
                const float om = fmaxf(1.0f - alpha, 1e-8f);
                T = T / om;
                const float inv = 1.0f / om;
                const float w = alpha * T;
                v[8] = w * gr; v[9] = w * gg; v[10] = w * gb;
                const float dL_dalpha = (gr * (T * s.r - sr * inv) + gg * (T * s.g - sg * inv) +
                                         gb * (T * s.b - sb * inv)) +
                                        ga * (T - sa * inv);
                sr += alpha * T * s.r; sg += alpha * T * s.g; sb += alpha * T * s.b;
                sa += alpha * T;
                if (!clamped) {
                    const float dp = dL_dalpha * s.op * gauss;
                    v[2] = dL_dalpha * gauss;
                    const float dux = dp * (s.ca * dx + s.cb * dy);
                    const float duy = dp * (s.cb * dx + s.cc * dy);
                    v[0] = dux; v[1] = duy;
                    v[4] = dp * (-0.5f * dx * dx);
                    v[5] = dp * (-1.0f * dx * dy);
                    v[6] = dp * (-0.5f * dy * dy);
                    if (want_absgrad) v[3] = sqrtf(dux * dux + duy * duy);
                }
            }
            const float r = reduce_scatter16(v, lane);
            const int slot = lane >> 1;
            if ((lane & 1) == 0 && slot < MG_G2D_STRIDE && r != 0.0f)
                atomicAdd(&s_acc[j][slot], r);
        }
        __syncthreads();
        for (int t = tid; t < n; t += G::kThreads) {
            const float4* a = reinterpret_cast<const float4*>(s_acc[t]);
            float4* dst = reinterpret_cast<float4*>(grad2d + (int64_t)s_id[t] * MG_G2D_STRIDE);
#pragma unroll
            for (int q = 0; q < 3; ++q) {
                const float4 x = a[q];
                if (x.x != 0.f || x.y != 0.f || x.z != 0.f || x.w != 0.f) atomicAdd(dst + q, x);
            }
        }
    }
}

__global__ void pack_intersections_kernel(const float2* __restrict__ uv,
                                          const float* __restrict__ conic,
                                          const float* __restrict__ opacity,
                                          const float* __restrict__ color,
                                          const int32_t* __restrict__ ids, int64_t m,
                                          float* __restrict__ p_xy_opac,
                                          float* __restrict__ p_conic,
                                          float* __restrict__ p_rgb) {
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= m) return;
    const int64_t g = ids[i];
    const float2 t = uv[g];
    p_xy_opac[3 * i] = t.x; p_xy_opac[3 * i + 1] = t.y; p_xy_opac[3 * i + 2] = opacity[g];
    p_conic[3 * i] = conic[3 * g]; p_conic[3 * i + 1] = conic[3 * g + 1];
    p_conic[3 * i + 2] = conic[3 * g + 2];
    p_rgb[3 * i] = color[3 * g]; p_rgb[3 * i + 1] = color[3 * g + 1];
    p_rgb[3 * i + 2] = color[3 * g + 2];
}

template <int TILE>
mg_status launch_fwd(const float* uv, const float* conic, const float* opacity,
                     const float* color, const int32_t* ids, const int32_t* offsets, int W,
                     int H, int tiles_x, int tiles_y, const float* bg, float* rgb,
                     float* alpha, float* T, int32_t* stop, cudaStream_t stream) {
    const int n_tiles = tiles_x * tiles_y;
    raster_forward_kernel<TILE><<<n_tiles, TileGeom<TILE>::kThreads, 0, stream>>>(
        reinterpret_cast<const float2*>(uv), conic, opacity, color, ids, offsets, W, H,
        tiles_x, bg != nullptr, bg ? bg[0] : 0.f, bg ? bg[1] : 0.f, bg ? bg[2] : 0.f, rgb,
        alpha, T, stop);
    return check_launch("rasterize_forward");
}

template <int TILE>
mg_status launch_bwd(const float* uv, const float* conic, const float* opacity,
                     const float* color, const int32_t* ids, const int32_t* offsets,
                     const float* final_T, const int32_t* stop, const float* grad_rgb,
                     const float* grad_alpha, int W, int H, int tiles_x, int tiles_y,
                     const float* bg, const float* alpha, int want_absgrad, float* grad2d,
                     cudaStream_t stream) {
    const int n_tiles = tiles_x * tiles_y;
    raster_backward_kernel<TILE><<<n_tiles, TileGeom<TILE>::kThreads, 0, stream>>>(
        reinterpret_cast<const float2*>(uv), conic, opacity, color, ids, offsets, final_T,
        stop, grad_rgb, grad_alpha, W, H, tiles_x, bg != nullptr, bg ? bg[0] : 0.f,
        bg ? bg[1] : 0.f, bg ? bg[2] : 0.f, alpha, want_absgrad, grad2d);
    return check_launch("rasterize_backward");
}

mg_status check_tile(int tile) {
    if (tile == 8 || tile == 12 || tile == 16 || tile == 32) return MG_OK;
    return fail(MG_ERR_INVALID_ARGUMENT,
                "tile " + std::to_string(tile) + " needs " + std::to_string(tile * tile) +
                    " threads per threadgroup (CUDA block); the rasteriser supports "
                    "tiles 8, 12, 16 and 32 (at most 1024 threads per block)");
}

}  // namespace

}  // namespace mg

using namespace mg;

extern "C" mg_status mg_rasterize_forward(const float* uv, const float* conic,
                                          const float* opacity, const float* color,
                                          const int32_t* gauss_ids,
                                          const int32_t* tile_offsets, int32_t width,
                                          int32_t height, int32_t tile, int32_t tiles_x,
                                          const float* background, float* out_rgb,
                                          float* out_alpha, float* out_T,
                                          int32_t* out_stop, mg_stream_t stream) {
    MG_TRY(check_tile(tile));
    MG_REQUIRE(width > 0 && height > 0, "rasterize_forward: empty image");
    const int tiles_y = (height + tile - 1) / tile;
    MG_REQUIRE(tiles_x == (width + tile - 1) / tile, "rasterize_forward: tiles_x mismatch");
    MG_REQUIRE(tile_offsets && out_rgb && out_alpha && out_T && out_stop,
               "rasterize_forward: null pointer");
    cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
    switch (tile) {
        case 8: return launch_fwd<8>(uv, conic, opacity, color, gauss_ids, tile_offsets, width, height, tiles_x, tiles_y, background, out_rgb, out_alpha, out_T, out_stop, s);
        case 12: return launch_fwd<12>(uv, conic, opacity, color, gauss_ids, tile_offsets, width, height, tiles_x, tiles_y, background, out_rgb, out_alpha, out_T, out_stop, s);
        case 16: return launch_fwd<16>(uv, conic, opacity, color, gauss_ids, tile_offsets, width, height, tiles_x, tiles_y, background, out_rgb, out_alpha, out_T, out_stop, s);
        default: return launch_fwd<32>(uv, conic, opacity, color, gauss_ids, tile_offsets, width, height, tiles_x, tiles_y, background, out_rgb, out_alpha, out_T, out_stop, s);
    }
}

extern "C" mg_status mg_rasterize_backward(
    const float* uv, const float* conic, const float* opacity, const float* color,
    const int32_t* gauss_ids, const int32_t* tile_offsets, const float* final_T,
    const int32_t* stop, const float* grad_rgb, const float* grad_alpha, int32_t width,
    int32_t height, int32_t tile, int32_t tiles_x, const float* background,
    const float* alpha, int32_t want_absgrad, int64_t n, float* grad2d,
    mg_stream_t stream) {
    MG_TRY(check_tile(tile));
    MG_REQUIRE(width > 0 && height > 0, "rasterize_backward: empty image");
    const int tiles_y = (height + tile - 1) / tile;
    MG_REQUIRE(tiles_x == (width + tile - 1) / tile, "rasterize_backward: tiles_x mismatch");
    MG_REQUIRE(final_T && stop && grad_rgb && tile_offsets, "rasterize_backward: null pointer");
    MG_REQUIRE(background == nullptr || alpha != nullptr,
               "rasterize_backward: the background blend needs the forward alpha");
    MG_REQUIRE((reinterpret_cast<uintptr_t>(grad2d) & 15u) == 0u,
               "rasterize_backward: grad2d must be 16-byte aligned");
    if (n == 0) return MG_OK;
    cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
    switch (tile) {
        case 8: return launch_bwd<8>(uv, conic, opacity, color, gauss_ids, tile_offsets, final_T, stop, grad_rgb, grad_alpha, width, height, tiles_x, tiles_y, background, alpha, want_absgrad, grad2d, s);
        case 12: return launch_bwd<12>(uv, conic, opacity, color, gauss_ids, tile_offsets, final_T, stop, grad_rgb, grad_alpha, width, height, tiles_x, tiles_y, background, alpha, want_absgrad, grad2d, s);
        case 16: return launch_bwd<16>(uv, conic, opacity, color, gauss_ids, tile_offsets, final_T, stop, grad_rgb, grad_alpha, width, height, tiles_x, tiles_y, background, alpha, want_absgrad, grad2d, s);
        default: return launch_bwd<32>(uv, conic, opacity, color, gauss_ids, tile_offsets, final_T, stop, grad_rgb, grad_alpha, width, height, tiles_x, tiles_y, background, alpha, want_absgrad, grad2d, s);
    }
}

extern "C" mg_status mg_pack_intersections(const float* uv, const float* conic,
                                           const float* opacity, const float* color,
                                           const int32_t* gauss_ids, int64_t m,
                                           float* p_xy_opac, float* p_conic, float* p_rgb,
                                           mg_stream_t stream) {
    if (m == 0) return MG_OK;
    pack_intersections_kernel<<<ceil_div(m, 256), 256, 0,
                                reinterpret_cast<cudaStream_t>(stream)>>>(
        reinterpret_cast<const float2*>(uv), conic, opacity, color, gauss_ids, m, p_xy_opac,
        p_conic, p_rgb);
    return check_launch("pack_intersections");
}
