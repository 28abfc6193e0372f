// Tile rasterisation, forward and backward (rasterize.metal:61-340).
//
// One CTA per screen tile; full 8x4 pixel blocks per warp when the tile side
// is a multiple of 8 (compact warps reach fewer Gaussians), otherwise
// row-major pixels with the CTA padded to whole warps.
//
// Every warp walks the tile's depth-sorted list ON ITS OWN, 32 entries at a
// time: each lane gathers one entry into warp-private shared memory and tests
// it against the warp's rectangle of pixel centres (the minimum of the conic's
// quadratic form over the rectangle against 2 ln(255 op), the reference's
// per-simdgroup cull, rasterize.metal:13-38); the warp then evaluates only the
// live entries (a ballot mask) and leaves the list as soon as its own 32
// pixels are done. There is no CTA barrier inside the walk, so a warp never
// waits for a slower one. Tiles are taken in a caller-given order (heaviest
// first, mg_tile_order) so long tiles do not form the kernel's tail.
//
// Forward: front to back, alpha = min(0.999, op exp(power)), skip power > 0
// or alpha < 1/255, stop a pixel once T < 1e-4 and record the stop INDEX.
//
// Backward: back to front from the warp's largest stop index, recovering T
// by division. Per live entry the warp reduces its 32 pixels' contributions
// with a 16-slot butterfly reduce-scatter (16 shuffles for all components
// instead of 5 per component) and three lanes add the 48-byte gradient record
// to global memory with three 16-byte vector atomics.
#include "kernels.cuh"

namespace mg {

namespace {

// One list entry as a warp stages it (36 B: two 16-byte and one 4-byte
// shared-memory words).
struct StagedGauss {
    float u, v, op, ca;
    float cb, cc, r, g;
    float b;
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

// Minimum of the conic's quadratic form over a rectangle (binning.metal:25-44),
// in ordinary fast arithmetic: it only decides a conservative skip.
__device__ __forceinline__ float min_q_rect_fast(float mux, float muy, float ca, float cb,
                                                 float cc, float x0, float x1, float y0,
                                                 float y1) {
    if (mux >= x0 && mux <= x1 && muy >= y0 && muy <= y1) return 0.0f;
    const float a = fmaxf(ca, 1e-12f), c = fmaxf(cc, 1e-12f);
    const float ia = 1.0f / a, ic = 1.0f / c;
    float best = __int_as_float(0x7f800000);
#pragma unroll
    for (int e = 0; e < 2; ++e) {
        const float yc = e == 0 ? y0 : y1;
        const float ey = yc - muy;
        const float ex = fminf(fmaxf(mux - cb * ey * ia, x0), x1) - mux;
        best = fminf(best, a * ex * ex + 2.0f * cb * ex * ey + c * ey * ey);
    }
#pragma unroll
    for (int e = 0; e < 2; ++e) {
        const float xc = e == 0 ? x0 : x1;
        const float ex = xc - mux;
        const float ey = fminf(fmaxf(muy - cb * ex * ic, y0), y1) - muy;
        best = fminf(best, a * ex * ex + 2.0f * cb * ex * ey + c * ey * ey);
    }
    return best;
}



__device__ __forceinline__ StagedGauss stage_one(const float2* __restrict__ uv,
                                                 const float* __restrict__ conic,
                                                 const float* __restrict__ opacity,
                                                 const float* __restrict__ color, int g) {
    const float2 m = uv[g];
    StagedGauss s;
    s.u = m.x; s.v = m.y; s.op = opacity[g];
    s.ca = conic[3 * g]; s.cb = conic[3 * g + 1]; s.cc = conic[3 * g + 2];
    s.r = color[3 * g]; s.g = color[3 * g + 1]; s.b = color[3 * g + 2];
    return s;
}

// Warp-private staging slots: float4 {u, v, op, ca}, float4 {cb, cc, r, g},
// float b.
struct WarpSlots {
    float4 a[32];
    float4 c[32];
    float b[32];
    int32_t id[32];
    __device__ __forceinline__ void put(int k, const StagedGauss& s, int gid) {
        a[k] = make_float4(s.u, s.v, s.op, s.ca);
        c[k] = make_float4(s.cb, s.cc, s.r, s.g);
        b[k] = s.b;
        id[k] = gid;
    }
    __device__ __forceinline__ StagedGauss get(int k) const {
        const float4 x = a[k], y = c[k];
        StagedGauss s;
        s.u = x.x; s.v = x.y; s.op = x.z; s.ca = x.w;
        s.cb = y.x; s.cc = y.y; s.r = y.z; s.g = y.w;
        s.b = b[k];
        return s;
    }
};

// Is this entry live for a warp whose pixel centres span [x0,x1] x [y0,y1]?
__device__ __forceinline__ bool live_for_rect(const StagedGauss& g, float x0, float x1,
                                              float y0, float y1) {
    const float oa = 255.0f * g.op;
    if (oa <= 1.0f || x0 > x1) return false;
    const float thr = 2.0f * __logf(oa) * 1.0001f + 1e-4f;
    return min_q_rect_fast(g.u, g.v, g.ca, g.cb, g.cc, x0, x1, y0, y1) < thr;
}

// Bounding rectangle of the warp's in-image pixel centres, in every lane
// (x0 > x1 when the warp has no pixel in the image).
__device__ __forceinline__ void warp_rect(bool inimg, float fx, float fy, float& x0, float& x1,
                                          float& y0, float& y1) {
    x0 = inimg ? fx : 3.0e38f; x1 = inimg ? fx : -3.0e38f;
    y0 = inimg ? fy : 3.0e38f; y1 = inimg ? fy : -3.0e38f;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        x0 = fminf(x0, __shfl_xor_sync(0xffffffffu, x0, o));
        x1 = fmaxf(x1, __shfl_xor_sync(0xffffffffu, x1, o));
        y0 = fminf(y0, __shfl_xor_sync(0xffffffffu, y0, o));
        y1 = fmaxf(y1, __shfl_xor_sync(0xffffffffu, y1, o));
    }
}

// Work split: a tile's pixels are 8x4 warp blocks (row-major pixels padded
// to whole warps when the side is not a multiple of 8). Warps walk the list
// independently, so a CTA is only a scheduling unit: two warps (an 8x8
// sub-block) per CTA when the side is a multiple of 8, which lets finished
// sub-blocks free their registers while a slow one is still walking.
template <int TILE>
struct TileGeom {
    static constexpr int kPix = TILE * TILE;
    static constexpr int kTileWarps = (kPix + 31) / 32;
    static constexpr int kWarps = (TILE % 8 == 0) ? 2 : kTileWarps;  // per CTA
    static constexpr int kThreads = kWarps * 32;
    static constexpr int kCtasPerTile = kTileWarps / kWarps;
    // pixel of lane `lane` in warp `wt` (0 .. kTileWarps-1) of the tile
    __device__ __forceinline__ static void pixel(int wt, int lane, int& lx, int& ly) {
        if (TILE % 8 == 0) {
            const int bx = TILE / 8;
            lx = (wt % bx) * 8 + (lane & 7);
            ly = (wt / bx) * 4 + (lane >> 3);
        } else {
            const int t = wt * 32 + lane;
            if (t < kPix) {
                lx = t % TILE;
                ly = t / TILE;
            } else {
                lx = TILE;  // padding thread, outside the tile
                ly = TILE;
            }
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
                      float* __restrict__ out_T, int32_t* __restrict__ out_stop,
                      const int32_t* __restrict__ tile_order, int32_t* __restrict__ tile_work) {
    using G = TileGeom<TILE>;
    __shared__ WarpSlots s_w[G::kWarps];
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int slot = blockIdx.x / G::kCtasPerTile;
    const int tile_id = tile_order ? tile_order[slot] : slot;
    const int tx = tile_id % tiles_x, ty = tile_id / tiles_x;
    int lx, ly;
    G::pixel((blockIdx.x % G::kCtasPerTile) * G::kWarps + warp, lane, lx, ly);
    const bool in_tile = lx < TILE && ly < TILE;
    const int px = tx * TILE + lx, py = ty * TILE + ly;
    const bool inimg = in_tile && px < W && py < H;
    const int start = offsets[tile_id], end = offsets[tile_id + 1];
    const float fx = (float)px + 0.5f, fy = (float)py + 0.5f;
    float rx0, rx1, ry0, ry1;
    warp_rect(inimg, fx, fy, rx0, rx1, ry0, ry1);
    WarpSlots& slots = s_w[warp];

    float T = 1.0f, ar = 0.0f, ag = 0.0f, ab = 0.0f, aa = 0.0f;
    int stop = start;
    bool done = !inimg;
    bool warp_done = __all_sync(0xffffffffu, done);
    for (int base = start; base < end && !warp_done; base += 32) {
        const int i = base + lane;
        bool lv = false;
        if (i < end) {
            const StagedGauss sg = stage_one(uv, conic, opacity, color, ids[i]);
            lv = live_for_rect(sg, rx0, rx1, ry0, ry1);
            if (lv) slots.put(lane, sg, 0);
        }
        uint32_t live = __ballot_sync(0xffffffffu, lv);
        __syncwarp();
        while (live) {
            const int k = __ffs(live) - 1;  // front to back
            live &= live - 1;
            if (done) continue;
            const StagedGauss sj = slots.get(k);
            const float power = pair_power(fx - sj.u, fy - sj.v, sj.ca, sj.cb, sj.cc);
            if (power > 0.0f) continue;
            const float alpha = fminf(0.999f, sj.op * pair_gauss(power));
            if (alpha < 1.0f / 255.0f) continue;
            const float w = alpha * T;
            ar += w * sj.r; ag += w * sj.g; ab += w * sj.b;
            aa += w;
            T *= (1.0f - alpha);
            stop = base + k + 1;
            if (T < 1e-4f) done = true;
        }
        warp_done = __all_sync(0xffffffffu, done);
        __syncwarp();  // slots are rewritten by the next chunk
    }
    if (tile_work) {  // zeroed by the launcher; the tile's walk = max stop - start
        const int ws = __reduce_max_sync(0xffffffffu, stop) - start;
        if (lane == 0 && ws > 0) atomicMax(&tile_work[tile_id], ws);
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
                       float* __restrict__ grad2d, const int32_t* __restrict__ tile_order) {
    using G = TileGeom<TILE>;
    __shared__ WarpSlots s_w[G::kWarps];
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int slot = blockIdx.x / G::kCtasPerTile;
    const int tile_id = tile_order ? tile_order[slot] : slot;
    const int tx = tile_id % tiles_x, ty = tile_id / tiles_x;
    int lx, ly;
    G::pixel((blockIdx.x % G::kCtasPerTile) * G::kWarps + warp, lane, lx, ly);
    const bool in_tile = lx < TILE && ly < TILE;
    const int px = tx * TILE + lx, py = ty * TILE + ly;
    const bool inimg = in_tile && px < W && py < H;
    const int start = offsets[tile_id];
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
    if (warp_stop <= start) return;  // this warp blended nothing
    float rx0, rx1, ry0, ry1;
    warp_rect(inimg, fx, fy, rx0, rx1, ry0, ry1);
    WarpSlots& slots = s_w[warp];

    float sr = 0.f, sg = 0.f, sb = 0.f, sa = 0.f;  // suffix colour / alpha
    for (int cbase = start + ((warp_stop - 1 - start) >> 5) * 32; cbase >= start; cbase -= 32) {
        const int i = cbase + lane;
        bool lv = false;
        if (i < warp_stop) {
            const int gid = ids[i];
            const StagedGauss st = stage_one(uv, conic, opacity, color, gid);
            lv = live_for_rect(st, rx0, rx1, ry0, ry1);
            if (lv) slots.put(lane, st, gid);
        }
        uint32_t live = __ballot_sync(0xffffffffu, lv);
        __syncwarp();
        while (live) {
            const int k = 31 - __clz(live);  // back to front
            live &= ~(1u << k);
            const StagedGauss s = slots.get(k);
            const float dx = fx - s.u, dy = fy - s.v;
            const float power = pair_power(dx, dy, s.ca, s.cb, s.cc);
            const float gauss = pair_gauss(fminf(power, 0.0f));
            const float alpha_raw = s.op * gauss;
            const bool clamped = alpha_raw > 0.999f;
            const float alpha = fminf(0.999f, alpha_raw);
            const bool active = inimg && (cbase + k < my_stop) && (power <= 0.0f) &&
                                (alpha >= 1.0f / 255.0f);
            const uint32_t act = __ballot_sync(0xffffffffu, active);
            if (act == 0u) continue;
            float v[16];
#pragma unroll
            for (int q = 0; q < 16; ++q) v[q] = 0.0f;
            if (active) {
                const float inv = __frcp_rn(fmaxf(1.0f - alpha, 1e-8f));
                T = T * inv;
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
            if (__popc(act) <= 2) {
                // few contributing pixels: each adds its own record (the warp
                // reduction costs more instructions than two sets of atomics)
                if (active) {
                    float4* dst =
                        reinterpret_cast<float4*>(grad2d + (int64_t)slots.id[k] * MG_G2D_STRIDE);
                    atomicAdd(dst, make_float4(v[0], v[1], v[2], v[3]));
                    if (v[4] != 0.f || v[5] != 0.f || v[6] != 0.f)
                        atomicAdd(dst + 1, make_float4(v[4], v[5], v[6], 0.f));
                    atomicAdd(dst + 2, make_float4(v[8], v[9], v[10], 0.f));
                }
                continue;
            }
            // lanes 2s, 2s+1 hold slot s; lanes 0, 8, 16 gather slots 0-3, 4-7, 8-11
            const float r = reduce_scatter16(v, lane);
            const float r1 = __shfl_down_sync(0xffffffffu, r, 2);
            const float r2 = __shfl_down_sync(0xffffffffu, r, 4);
            const float r3 = __shfl_down_sync(0xffffffffu, r, 6);
            if ((lane & 7) == 0 && lane < 24 && (r != 0.f || r1 != 0.f || r2 != 0.f || r3 != 0.f)) {
                float4* dst = reinterpret_cast<float4*>(grad2d + (int64_t)slots.id[k] * MG_G2D_STRIDE);
                atomicAdd(dst + (lane >> 3), make_float4(r, r1, r2, r3));
            }
        }
        __syncwarp();  // slots are rewritten by the next chunk
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

// Longest-first tile order: a one-CTA counting sort of the tiles by the
// bucket floor(log2(work)) + 1, heaviest bucket first.
__global__ void __launch_bounds__(1024)
tile_order_kernel(const int32_t* __restrict__ offsets, const int32_t* __restrict__ work,
                  int n_tiles, int32_t* __restrict__ order) {
    __shared__ int s_count[33];
    __shared__ int s_cursor[33];
    const int tid = threadIdx.x;
    if (tid < 33) s_count[tid] = 0;
    __syncthreads();
    for (int t = tid; t < n_tiles; t += 1024) {
        const int w = work ? work[t] : offsets[t + 1] - offsets[t];
        const int b = w > 0 ? 32 - __clz(w) : 0;       // 0..31
        atomicAdd(&s_count[31 - b], 1);                // heaviest bucket first
    }
    __syncthreads();
    if (tid == 0) {
        int run = 0;
        for (int b = 0; b < 33; ++b) { s_cursor[b] = run; run += s_count[b]; }
    }
    __syncthreads();
    for (int t = tid; t < n_tiles; t += 1024) {
        const int w = work ? work[t] : offsets[t + 1] - offsets[t];
        const int b = w > 0 ? 32 - __clz(w) : 0;
        order[atomicAdd(&s_cursor[31 - b], 1)] = t;
    }
}

template <int TILE>
mg_status launch_fwd(const float* uv, const float* conic, const float* opacity,
                     const float* color, const int32_t* ids, const int32_t* offsets, int W,
                     int H, int tiles_x, int tiles_y, const float* bg, float* rgb,
                     float* alpha, float* T, int32_t* stop, const int32_t* order,
                     int32_t* work, cudaStream_t stream) {
    const int n_tiles = tiles_x * tiles_y;
    if (work && cudaMemsetAsync(work, 0, sizeof(int32_t) * n_tiles, stream) != cudaSuccess)
        return check_launch("rasterize_forward tile_work memset");
    raster_forward_kernel<TILE><<<n_tiles * TileGeom<TILE>::kCtasPerTile,
                                  TileGeom<TILE>::kThreads, 0, stream>>>(
        reinterpret_cast<const float2*>(uv), conic, opacity, color, ids, offsets, W, H,
        tiles_x, bg != nullptr, bg ? bg[0] : 0.f, bg ? bg[1] : 0.f, bg ? bg[2] : 0.f, rgb,
        alpha, T, stop, order, work);
    return check_launch("rasterize_forward");
}

template <int TILE>
mg_status launch_bwd(const float* uv, const float* conic, const float* opacity,
                     const float* color, const int32_t* ids, const int32_t* offsets,
                     const float* final_T, const int32_t* stop, const float* grad_rgb,
                     const float* grad_alpha, int W, int H, int tiles_x, int tiles_y,
                     const float* bg, const float* alpha, int want_absgrad, float* grad2d,
                     const int32_t* order, cudaStream_t stream) {
    const int n_tiles = tiles_x * tiles_y;
    raster_backward_kernel<TILE><<<n_tiles * TileGeom<TILE>::kCtasPerTile,
                                   TileGeom<TILE>::kThreads, 0, stream>>>(
        reinterpret_cast<const float2*>(uv), conic, opacity, color, ids, offsets, final_T,
        stop, grad_rgb, grad_alpha, W, H, tiles_x, bg != nullptr, bg ? bg[0] : 0.f,
        bg ? bg[1] : 0.f, bg ? bg[2] : 0.f, alpha, want_absgrad, grad2d, order);
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
                                          int32_t* out_stop, const int32_t* tile_order,
                                          int32_t* tile_work, mg_stream_t stream) {
    MG_TRY(check_tile(tile));
    MG_REQUIRE(width > 0 && height > 0, "rasterize_forward: empty image");
    const int tiles_y = (height + tile - 1) / tile;
    MG_REQUIRE(tiles_x == (width + tile - 1) / tile, "rasterize_forward: tiles_x mismatch");
    MG_REQUIRE(tile_offsets && out_rgb && out_alpha && out_T && out_stop,
               "rasterize_forward: null pointer");
    cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
    switch (tile) {
        case 8: return launch_fwd<8>(uv, conic, opacity, color, gauss_ids, tile_offsets, width, height, tiles_x, tiles_y, background, out_rgb, out_alpha, out_T, out_stop, tile_order, tile_work, s);
        case 12: return launch_fwd<12>(uv, conic, opacity, color, gauss_ids, tile_offsets, width, height, tiles_x, tiles_y, background, out_rgb, out_alpha, out_T, out_stop, tile_order, tile_work, s);
        case 16: return launch_fwd<16>(uv, conic, opacity, color, gauss_ids, tile_offsets, width, height, tiles_x, tiles_y, background, out_rgb, out_alpha, out_T, out_stop, tile_order, tile_work, s);
        default: return launch_fwd<32>(uv, conic, opacity, color, gauss_ids, tile_offsets, width, height, tiles_x, tiles_y, background, out_rgb, out_alpha, out_T, out_stop, tile_order, tile_work, s);
    }
}

extern "C" mg_status mg_rasterize_backward(
    const float* uv, const float* conic, const float* opacity, const float* color,
    const int32_t* gauss_ids, const int32_t* tile_offsets, const float* final_T,
    const int32_t* stop, const float* grad_rgb, const float* grad_alpha, int32_t width,
    int32_t height, int32_t tile, int32_t tiles_x, const float* background,
    const float* alpha, int32_t want_absgrad, int64_t n, float* grad2d,
    const int32_t* tile_order, mg_stream_t stream) {
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
        case 8: return launch_bwd<8>(uv, conic, opacity, color, gauss_ids, tile_offsets, final_T, stop, grad_rgb, grad_alpha, width, height, tiles_x, tiles_y, background, alpha, want_absgrad, grad2d, tile_order, s);
        case 12: return launch_bwd<12>(uv, conic, opacity, color, gauss_ids, tile_offsets, final_T, stop, grad_rgb, grad_alpha, width, height, tiles_x, tiles_y, background, alpha, want_absgrad, grad2d, tile_order, s);
        case 16: return launch_bwd<16>(uv, conic, opacity, color, gauss_ids, tile_offsets, final_T, stop, grad_rgb, grad_alpha, width, height, tiles_x, tiles_y, background, alpha, want_absgrad, grad2d, tile_order, s);
        default: return launch_bwd<32>(uv, conic, opacity, color, gauss_ids, tile_offsets, final_T, stop, grad_rgb, grad_alpha, width, height, tiles_x, tiles_y, background, alpha, want_absgrad, grad2d, tile_order, s);
    }
}

extern "C" mg_status mg_tile_order(const int32_t* tile_offsets, const int32_t* work,
                                   int32_t n_tiles, int32_t* order, mg_stream_t stream) {
    MG_REQUIRE(n_tiles > 0 && order != nullptr, "tile_order: bad arguments");
    MG_REQUIRE(work != nullptr || tile_offsets != nullptr, "tile_order: no work measure");
    tile_order_kernel<<<1, 1024, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
        tile_offsets, work, n_tiles, order);
    return check_launch("tile_order");
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
