// Preprocess forward and the per-Gaussian binning kernels (count, 64-bit key
// write, the two-stage depth-key/count and pair emission used by
// mg_bin_prepare / mg_bin_emit). Built with -fmad=false: see exact_math.cuh.
//
// Layout notes. means/scales are (N,3) and quats (N,4) rows; a warp reads 32
// consecutive rows, so every load instruction touches one or two contiguous
// 128-byte segments. SH rows are 48 B (fused) or 12 B + 180 B (split): a warp
// stages its 32 Gaussians' coefficient block through shared memory with
// coalesced loads and each thread then reads its own row from there.
#include "exact_math.cuh"
#include "kernels.cuh"

namespace mg {

namespace {

constexpr int kPreBlock = 128;  // 4 warps

// Stage one warp's coefficient rows [g0, g0+32) of a (rows, stride) array of
// 3-float rows into shared memory (contiguous), skipping rows >= n.
__device__ __forceinline__ void stage_rows(const float* __restrict__ src,
                                           int64_t g0, int64_t n, int stride_rows,
                                           int offset_rows, int nrows,
                                           float* __restrict__ dst, int lane) {
    // Row g occupies floats [(g*stride + offset)*3, +nrows*3). With the split
    // layout (stride == nrows, offset 0) consecutive Gaussians are contiguous.
    const int64_t avail = min((int64_t)32, n - g0);
    const int per_g = nrows * 3;
    if (stride_rows == nrows && offset_rows == 0) {
        const float* base = src + g0 * (int64_t)per_g;
        const int total = (int)avail * per_g;
        for (int i = lane; i < total; i += 32) dst[i] = __ldg(base + i);
    } else {
        for (int k = 0; k < (int)avail; ++k) {
            const float* row = src + ((g0 + k) * stride_rows + offset_rows) * 3;
            for (int i = lane; i < per_g; i += 32) dst[k * per_g + i] = __ldg(row + i);
        }
    }
}

__global__ void __launch_bounds__(kPreBlock)
preprocess_forward_kernel(const float* __restrict__ means,
                          const float* __restrict__ quats,
                          const float* __restrict__ scales,
                          const float* __restrict__ sh_dc,
                          const float* __restrict__ sh_rest, mg_sh_layout shl,
                          const float* __restrict__ opacities, CamParams P,
                          int sh_degree, int64_t n, float2* __restrict__ out_uv,
                          float* __restrict__ out_conic,
                          float* __restrict__ out_depth,
                          float2* __restrict__ out_rxy,
                          int32_t* __restrict__ out_valid,
                          float* __restrict__ out_color) {
    // 32 Gaussians x 15 rest rows x 3 floats per warp.
    __shared__ float s_rest[kPreBlock / 32][32 * 15 * 3];
    const int lane = threadIdx.x & 31, wib = threadIdx.x >> 5;
    const int64_t g = (int64_t)blockIdx.x * kPreBlock + threadIdx.x;
    const int64_t g0 = g - lane;
    const bool in = g < n;

    Projected pr;
    pr.ok = false;
    float mx = 0.f, my = 0.f, mz = 0.f;
    if (in) {
        mx = means[3 * g + 0]; my = means[3 * g + 1]; mz = means[3 * g + 2];
        const float4 q = __ldg(reinterpret_cast<const float4*>(quats) + g);
        const float sx = scales[3 * g + 0], sy = scales[3 * g + 1], sz = scales[3 * g + 2];
        pr = project_one(P, mx, my, mz, q.x, q.y, q.z, q.w, sx, sy, sz, opacities[g]);
        out_uv[g] = make_float2(pr.u, pr.v);
        out_conic[3 * g + 0] = pr.ca;
        out_conic[3 * g + 1] = pr.cb;
        out_conic[3 * g + 2] = pr.cc;
        out_depth[g] = pr.z;
        out_rxy[g] = make_float2(pr.rx, pr.ry);
        out_valid[g] = pr.ok ? 1 : 0;
    }
    if (sh_degree < 0 || sh_dc == nullptr) return;  // explicit colours

    // Visibility-gated SH (preprocess.metal:203-207): only rows that will be
    // binned read their coefficients; the rest get colour 0.
    const unsigned any_ok = __ballot_sync(0xffffffffu, in && pr.ok);
    const int nb = (sh_degree + 1) * (sh_degree + 1);
    if (any_ok != 0u && nb > 1) {
        stage_rows(sh_rest, g0, n, shl.stride_rest, shl.offset_rest, nb - 1,
                   s_rest[wib], lane);
        __syncwarp();
    }
    if (!in) return;
    if (!pr.ok) {
        out_color[3 * g + 0] = 0.0f;
        out_color[3 * g + 1] = 0.0f;
        out_color[3 * g + 2] = 0.0f;
        return;
    }
    const float dvx = mx - P.ccx, dvy = my - P.ccy, dvz = mz - P.ccz;
    const float len = sqrtf((dvx * dvx + dvy * dvy) + dvz * dvz);
    const float invn = 1.0f / fmaxf(len, 1e-12f);
    float B[16];
    sh_basis(sh_degree, dvx * invn, dvy * invn, dvz * invn, B);
    const float* dc = sh_dc + g * (int64_t)shl.stride_dc * 3;
    float r = 0.0f, gg = 0.0f, bb = 0.0f;
    r = r + B[0] * dc[0];
    gg = gg + B[0] * dc[1];
    bb = bb + B[0] * dc[2];
    const float* rest = s_rest[wib] + lane * (nb - 1) * 3;
#pragma unroll
    for (int i = 1; i < 16; ++i) {
        if (i < nb) {
            r = r + B[i] * rest[(i - 1) * 3 + 0];
            gg = gg + B[i] * rest[(i - 1) * 3 + 1];
            bb = bb + B[i] * rest[(i - 1) * 3 + 2];
        }
    }
    r = r + 0.5f; gg = gg + 0.5f; bb = bb + 0.5f;
    out_color[3 * g + 0] = fmaxf(r, 0.0f);
    out_color[3 * g + 1] = fmaxf(gg, 0.0f);
    out_color[3 * g + 2] = fmaxf(bb, 0.0f);
}

// Walk the Gaussian's clamped tile rectangle row-major and count (or emit)
// the tiles that pass the exact ellipse test (binning.metal:46-90).
// With `rec` given (count walks), the walk also leaves a record of its
// decisions: rectangles of at most 64 tiles get the pass mask over the
// rectangle in row-major order plus the rectangle itself, so the emission
// can expand the mask instead of testing every tile again.
template <bool kEmit64, bool kEmitPair>
__device__ __forceinline__ uint32_t bin_walk(
    float mux, float muy, float rx, float ry, float ca, float cb, float cc,
    float op, uint32_t dbits, int tile, int tiles_x, int tiles_y, int W, int H,
    uint64_t* keys, int32_t* ids, uint32_t* pair_tiles, uint32_t* pair_ids,
    int64_t write_at, uint32_t cap, int32_t gid, uint4* rec = nullptr) {
    const TileRect tr = tile_rect(mux, muy, rx, ry, tile, tiles_x, tiles_y);
    const float oa = 255.0f * op;
    if (oa <= 1.0f) return 0u;
    const float thr = 2.0f * log_f32_via_f64(oa);
    const int rw = tr.x1 - tr.x0 + 1, rh = tr.y1 - tr.y0 + 1;
    const bool masked = rec != nullptr && rw * rh <= 64;
    uint64_t mask = 0ull;
    int bit = 0;
    uint32_t cnt = 0u;
    for (int ty = tr.y0; ty <= tr.y1; ++ty) {
        const float y0 = (float)(ty * tile);
        const float y1 = fminf((float)((ty + 1) * tile), (float)H);
        for (int tx = tr.x0; tx <= tr.x1; ++tx) {
            const float x0 = (float)(tx * tile);
            const float x1 = fminf((float)((tx + 1) * tile), (float)W);
            const int b = bit++;
            if (min_q_over_rect(mux, muy, ca, cb, cc, x0, x1, y0, y1) >= thr) continue;
            if (masked) mask |= 1ull << b;
            if (kEmit64 || kEmitPair) {
                if (cnt < cap) {
                    const uint32_t tid = (uint32_t)(ty * tiles_x + tx);
                    if (kEmit64) {
                        keys[write_at + cnt] = ((uint64_t)tid << 32) | (uint64_t)dbits;
                        ids[write_at + cnt] = gid;
                    } else {
                        pair_tiles[write_at + cnt] = tid;
                        pair_ids[write_at + cnt] = (uint32_t)gid;
                    }
                }
            }
            ++cnt;
        }
    }
    if (rec)  // width 0 marks a rectangle the emission must walk again
        *rec = make_uint4((uint32_t)mask, (uint32_t)(mask >> 32),
                          (uint32_t)tr.x0 | ((uint32_t)tr.y0 << 16),
                          masked ? ((uint32_t)rw | ((uint32_t)rh << 16)) : 0u);
    return cnt;
}

__global__ void bin_count_kernel(const float2* __restrict__ uv,
                                 const float2* __restrict__ rxy,
                                 const float* __restrict__ conic,
                                 const float* __restrict__ opacity,
                                 const int32_t* __restrict__ valid, int64_t n,
                                 int W, int H, int tile, int tiles_x, int tiles_y,
                                 int32_t* __restrict__ counts) {
    const int64_t g = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (g >= n) return;
    uint32_t c = 0u;
    if (valid[g] != 0) {
        const float2 mu = uv[g], r = rxy[g];
        c = bin_walk<false, false>(mu.x, mu.y, r.x, r.y, conic[3 * g], conic[3 * g + 1],
                                   conic[3 * g + 2], opacity[g], 0u, tile, tiles_x,
                                   tiles_y, W, H, nullptr, nullptr, nullptr, nullptr,
                                   0, 0u, 0);
    }
    counts[g] = (int32_t)c;
}

__global__ void bin_write_kernel(const float2* __restrict__ uv,
                                 const float2* __restrict__ rxy,
                                 const float* __restrict__ conic,
                                 const float* __restrict__ opacity,
                                 const int32_t* __restrict__ valid,
                                 const float* __restrict__ depth,
                                 const int32_t* __restrict__ offsets, int64_t total,
                                 int64_t n, int W, int H, int tile, int tiles_x,
                                 int tiles_y, uint64_t* __restrict__ keys,
                                 int32_t* __restrict__ ids) {
    const int64_t g = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (g >= n || valid[g] == 0) return;
    const int64_t at = offsets[g];
    if (at < 0 || at >= total) return;
    const uint32_t cap = (uint32_t)min((int64_t)0xffffffff, total - at);
    const float2 mu = uv[g], r = rxy[g];
    bin_walk<true, false>(mu.x, mu.y, r.x, r.y, conic[3 * g], conic[3 * g + 1],
                          conic[3 * g + 2], opacity[g], __float_as_uint(depth[g]), tile,
                          tiles_x, tiles_y, W, H, keys, ids, nullptr, nullptr, at, cap,
                          (int32_t)g);
}

// Stage A of the two-stage binning: tile counts plus the depth sort keys.
// Gaussians that claim no tile get key 0xffffffff and sort behind every
// positive depth (valid depths are > near > 0, whose bit patterns are below
// 0x7f800000).
__global__ void bin_count_depth_kernel(const float2* __restrict__ uv,
                                       const float2* __restrict__ rxy,
                                       const float* __restrict__ conic,
                                       const float* __restrict__ opacity,
                                       const int32_t* __restrict__ valid,
                                       const float* __restrict__ depth, int64_t n,
                                       int W, int H, int tile, int tiles_x,
                                       int tiles_y, uint32_t* __restrict__ counts,
                                       uint32_t* __restrict__ dkeys,
                                       uint32_t* __restrict__ dvals,
                                       uint4* __restrict__ recs) {
    const int64_t g = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (g >= n) return;
    uint32_t c = 0u;
    if (valid[g] != 0) {
        const float2 mu = uv[g], r = rxy[g];
        c = bin_walk<false, false>(mu.x, mu.y, r.x, r.y, conic[3 * g], conic[3 * g + 1],
                                   conic[3 * g + 2], opacity[g], 0u, tile, tiles_x,
                                   tiles_y, W, H, nullptr, nullptr, nullptr, nullptr,
                                   0, 0u, 0, recs + g);
    }
    counts[g] = c;
    dkeys[g] = c > 0u ? __float_as_uint(depth[g]) : 0xffffffffu;
    dvals[g] = (uint32_t)g;
}

// Stage B: emit every (tile, Gaussian) pair with Gaussians in depth order.
// offsets are the exclusive scan of the counts in that order; each thread
// writes at most its own count so a disagreement can never overrun.
__global__ void bin_emit_kernel(const float2* __restrict__ uv,
                                const float2* __restrict__ rxy,
                                const float* __restrict__ conic,
                                const float* __restrict__ opacity,
                                const uint32_t* __restrict__ sorted_gid,
                                const uint32_t* __restrict__ counts,
                                const uint32_t* __restrict__ offsets, int64_t n,
                                int64_t m, int W, int H, int tile, int tiles_x,
                                int tiles_y, const uint4* __restrict__ recs,
                                uint32_t* __restrict__ pair_tiles,
                                uint32_t* __restrict__ pair_ids) {
    const int64_t s = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (s >= n) return;
    const uint32_t g = sorted_gid[s];
    const uint32_t cnt = counts[g];
    if (cnt == 0u) return;
    const int64_t at = offsets[s];
    if (at + cnt > m) return;
    const uint4 rec = recs[g];
    const uint32_t rw = rec.w & 0xffffu, rh = rec.w >> 16;
    if (rw != 0u) {
        // the count walk's decisions: row-major bits over the rectangle
        uint64_t mask = (uint64_t)rec.x | ((uint64_t)rec.y << 32);
        const uint32_t x0 = rec.z & 0xffffu, y0 = rec.z >> 16;
        const uint64_t row_bits = rw == 64u ? ~0ull : (1ull << rw) - 1ull;
        uint32_t k = 0u;
        for (uint32_t r = 0; r < rh && mask; ++r) {
            uint64_t row = mask & row_bits;
            mask >>= rw;
            const uint32_t trow = (y0 + r) * (uint32_t)tiles_x + x0;
            while (row) {
                const uint32_t b = (uint32_t)__ffsll((long long)row) - 1u;
                row &= row - 1ull;
                if (k < cnt) {
                    pair_tiles[at + k] = trow + b;
                    pair_ids[at + k] = g;
                }
                ++k;
            }
        }
        return;
    }
    const float2 mu = uv[g], r = rxy[g];
    bin_walk<false, true>(mu.x, mu.y, r.x, r.y, conic[3 * (int64_t)g],
                          conic[3 * (int64_t)g + 1], conic[3 * (int64_t)g + 2],
                          opacity[g], 0u, tile, tiles_x, tiles_y, W, H, nullptr,
                          nullptr, pair_tiles, pair_ids, at, cnt, (int32_t)g);
}

}  // namespace

mg_status launch_preprocess_forward(const float* means, const float* quats,
                                    const float* scales, const float* sh_dc,
                                    const float* sh_rest, mg_sh_layout shl,
                                    const float* opacities, const mg_camera& cam,
                                    int sh_degree, int64_t n, float* uv, float* conic,
                                    float* depth, float* rxy, int32_t* valid,
                                    float* color, cudaStream_t stream) {
    if (n == 0) return MG_OK;
    const CamParams P = make_cam_params(cam);
    preprocess_forward_kernel<<<ceil_div(n, kPreBlock), kPreBlock, 0, stream>>>(
        means, quats, scales, sh_dc, sh_rest, shl, opacities, P, sh_degree, n,
        reinterpret_cast<float2*>(uv), conic, depth, reinterpret_cast<float2*>(rxy),
        valid, color);
    return check_launch("preprocess_forward");
}

mg_status launch_bin_count(const float* uv, const float* rxy, const float* conic,
                           const float* opacity, const int32_t* valid, int64_t n,
                           int W, int H, int tile, int tiles_x, int tiles_y,
                           int32_t* counts, cudaStream_t stream) {
    if (n == 0) return MG_OK;
    bin_count_kernel<<<ceil_div(n, 256), 256, 0, stream>>>(
        reinterpret_cast<const float2*>(uv), reinterpret_cast<const float2*>(rxy), conic,
        opacity, valid, n, W, H, tile, tiles_x, tiles_y, counts);
    return check_launch("bin_count");
}

mg_status launch_bin_write(const float* uv, const float* rxy, const float* conic,
                           const float* opacity, const int32_t* valid,
                           const float* depth, const int32_t* offsets, int64_t total,
                           int64_t n, int W, int H, int tile, int tiles_x,
                           int tiles_y, uint64_t* keys, int32_t* ids,
                           cudaStream_t stream) {
    if (n == 0 || total == 0) return MG_OK;
    bin_write_kernel<<<ceil_div(n, 256), 256, 0, stream>>>(
        reinterpret_cast<const float2*>(uv), reinterpret_cast<const float2*>(rxy), conic,
        opacity, valid, depth, offsets, total, n, W, H, tile, tiles_x, tiles_y, keys, ids);
    return check_launch("bin_write");
}

mg_status launch_bin_count_depth(const float* uv, const float* rxy, const float* conic,
                                 const float* opacity, const int32_t* valid,
                                 const float* depth, int64_t n, int W, int H, int tile,
                                 int tiles_x, int tiles_y, uint32_t* counts,
                                 uint32_t* dkeys, uint32_t* dvals, uint4* recs,
                                 cudaStream_t stream) {
    if (n == 0) return MG_OK;
    bin_count_depth_kernel<<<ceil_div(n, 256), 256, 0, stream>>>(
        reinterpret_cast<const float2*>(uv), reinterpret_cast<const float2*>(rxy), conic,
        opacity, valid, depth, n, W, H, tile, tiles_x, tiles_y, counts, dkeys, dvals, recs);
    return check_launch("bin_count_depth");
}

mg_status launch_bin_emit(const float* uv, const float* rxy, const float* conic,
                          const float* opacity, const uint32_t* sorted_gid,
                          const uint32_t* counts, const uint32_t* offsets, int64_t n,
                          int64_t m, int W, int H, int tile, int tiles_x, int tiles_y,
                          const uint4* recs, uint32_t* pair_tiles, uint32_t* pair_ids,
                          cudaStream_t stream) {
    if (n == 0 || m == 0) return MG_OK;
    bin_emit_kernel<<<ceil_div(n, 256), 256, 0, stream>>>(
        reinterpret_cast<const float2*>(uv), reinterpret_cast<const float2*>(rxy), conic,
        opacity, sorted_gid, counts, offsets, n, m, W, H, tile, tiles_x, tiles_y,
        recs, pair_tiles, pair_ids);
    return check_launch("bin_emit");
}

}  // namespace mg
