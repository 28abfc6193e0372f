// Preprocess forward and the per-Gaussian binning kernels (count, 64-bit key
// write, the two-stage depth-key/count and pair emission used by
// mg_bin_prepare / mg_bin_emit). Built with -fmad=false: see exact_math.cuh.
//
// Layout notes. means/scales are (N,3) and quats (N,4) rows; a warp reads 32
// consecutive rows, so every load instruction touches one or two contiguous
// 128-byte segments. SH rows are 48 B (fused) or 12 B + 180 B (split): a warp
// stages its 32 Gaussians' coefficient block through shared memory with
// coalesced loads and each thread then reads its own row from there.
#include <algorithm>

#include "exact_math.cuh"
#include "filter3d.cuh"
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
        warp_copy_to_shared(src + g0 * (int64_t)per_g, (int)avail * per_g, dst, lane);
    } else {
        for (int k = 0; k < (int)avail; ++k) {
            const float* row = src + ((g0 + k) * stride_rows + offset_rows) * 3;
            for (int i = lane; i < per_g; i += 32) dst[k * per_g + i] = __ldg(row + i);
        }
    }
}

// SH colour of one Gaussian seen along (dvx, dvy, dvz) (mean minus camera
// centre): DC row from global memory, rows 1.. from the warp's staged block,
// +0.5 and the clamp at 0 (preprocess.metal:203-221).
__device__ __forceinline__ float3 sh_colour(int sh_degree, int nb, float dvx, float dvy,
                                            float dvz, const float* __restrict__ dc,
                                            const float* rest) {
    const float len = sqrtf((dvx * dvx + dvy * dvy) + dvz * dvz);
    const float invn = 1.0f / fmaxf(len, 1e-12f);
    float B[16];
    sh_basis(sh_degree, dvx * invn, dvy * invn, dvz * invn, B);
    float r = 0.0f, gg = 0.0f, bb = 0.0f;
    r = r + B[0] * dc[0];
    gg = gg + B[0] * dc[1];
    bb = bb + B[0] * dc[2];
#pragma unroll
    for (int i = 1; i < 16; ++i) {
        if (i < nb) {
            r = r + B[i] * rest[(i - 1) * 3 + 0];
            gg = gg + B[i] * rest[(i - 1) * 3 + 1];
            bb = bb + B[i] * rest[(i - 1) * 3 + 2];
        }
    }
    r = r + 0.5f; gg = gg + 0.5f; bb = bb + 0.5f;
    return make_float3(fmaxf(r, 0.0f), fmaxf(gg, 0.0f), fmaxf(bb, 0.0f));
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
    __shared__ __align__(16) float s_rest[kPreBlock / 32][32 * 15 * 3];
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
    const float3 col = sh_colour(sh_degree, nb, mx - P.ccx, my - P.ccy, mz - P.ccz,
                                 sh_dc + g * (int64_t)shl.stride_dc * 3,
                                 s_rest[wib] + lane * (nb - 1) * 3);
    out_color[3 * g + 0] = col.x;
    out_color[3 * g + 1] = col.y;
    out_color[3 * g + 2] = col.z;
}

constexpr int kMaxViewsPerLaunch = 16;
struct ViewCams {
    CamParams c[kMaxViewsPerLaunch];
};

// preprocess_forward_kernel for several cameras at once: a Gaussian's
// parameters and SH rows are read (and staged) once and projected and
// coloured for every view; view v's outputs start at v * view_stride. With
// `vis` given, each Gaussian's count of views where it is valid is added to
// vis[g]. Per view the arithmetic is that of the single-view kernel.
// Resident 128-thread CTAs per SM the multi-view projection's registers are
// held to (it is bound by load latency, so occupancy pays): 6 / 7 / 8 (72 /
// 64 / 64 registers, no spills) measured 0.219 / 0.215 / 0.217 ms per step of
// 8 views.
#ifndef MG_PRE_FWD_MIN_CTAS
#define MG_PRE_FWD_MIN_CTAS 7
#endif
__global__ void __launch_bounds__(kPreBlock, MG_PRE_FWD_MIN_CTAS)
preprocess_forward_views_kernel(const float* __restrict__ means,
                                const float* __restrict__ quats,
                                const float* __restrict__ scales,
                                const float* __restrict__ sh_dc,
                                const float* __restrict__ sh_rest, mg_sh_layout shl,
                                const float* __restrict__ opacities, ViewCams cams,
                                int n_views, int sh_degree, int64_t n, int64_t view_stride,
                                float2* __restrict__ out_uv, float* __restrict__ out_conic,
                                float* __restrict__ out_depth, float2* __restrict__ out_rxy,
                                int32_t* __restrict__ out_valid,
                                float* __restrict__ out_color, float* __restrict__ vis,
                                const mg_step_prologue pro, bool with_prologue) {
    __shared__ __align__(16) float s_rest[kPreBlock / 32][32 * 15 * 3];
    const int lane = threadIdx.x & 31, wib = threadIdx.x >> 5;
    const int64_t g = (int64_t)blockIdx.x * kPreBlock + threadIdx.x;
    const int64_t g0 = g - lane;
    const bool in = g < n;
    const bool colour = sh_degree >= 0 && sh_dc != nullptr;
    const int nb = (sh_degree + 1) * (sh_degree + 1);

    float mx = 0.f, my = 0.f, mz = 0.f;
    GaussianCov gc{};  // view-independent: computed once for every view
    if (in) {
        mx = means[3 * g + 0]; my = means[3 * g + 1]; mz = means[3 * g + 2];
        const float4 q = __ldg(reinterpret_cast<const float4*>(quats) + g);
        float sx, sy, sz, op;
        if (with_prologue) {
            // the step's activations (train.py:221-222, torch's exp and
            // 1 / (1 + exp(-x))), then the 3D filter when one is set
            // (train.py:223-227, mipfilter.py:79-93)
            sx = expf(pro.log_scales[3 * g + 0]);
            sy = expf(pro.log_scales[3 * g + 1]);
            sz = expf(pro.log_scales[3 * g + 2]);
            op = 1.0f / (1.0f + expf(-pro.logit_opac[g]));
            pro.act_scales[3 * g + 0] = sx;
            pro.act_scales[3 * g + 1] = sy;
            pro.act_scales[3 * g + 2] = sz;
            pro.act_opac[g] = op;
            if (pro.filter_3d != nullptr) {
                const Filter3d f = filter3d(sx, sy, sz, pro.filter_3d[g]);
                sx = f.s[0]; sy = f.s[1]; sz = f.s[2];
                op = op * f.coef;
                pro.out_scales[3 * g + 0] = sx;
                pro.out_scales[3 * g + 1] = sy;
                pro.out_scales[3 * g + 2] = sz;
                pro.out_opac[g] = op;
            }
            // the gradient rows this step accumulates into start at zero
#pragma unroll
            for (int k = 0; k < 4; ++k) {
                float* z = pro.zero[k];
                if (z == nullptr) continue;
                const int w = pro.zero_width[k];
                for (int j = 0; j < w; ++j) z[g * w + j] = 0.0f;
            }
            if (g == 0 && pro.zero_word != nullptr) *pro.zero_word = 0.0f;
        } else {
            sx = scales[3 * g + 0]; sy = scales[3 * g + 1]; sz = scales[3 * g + 2];
            op = opacities[g];
        }
        gc = gaussian_cov(q.x, q.y, q.z, q.w, sx, sy, sz, op);
    }
    bool staged = false;  // warp-uniform: the SH rows are staged at first use
    int visible = 0;
    for (int v = 0; v < n_views; ++v) {
        const CamParams& P = cams.c[v];
        const int64_t o = (int64_t)v * view_stride + g;
        Projected pr;
        pr.ok = false;
        if (in) {
            pr = project_with(P, mx, my, mz, gc);
            out_uv[o] = make_float2(pr.u, pr.v);
            out_conic[3 * o + 0] = pr.ca;
            out_conic[3 * o + 1] = pr.cb;
            out_conic[3 * o + 2] = pr.cc;
            out_depth[o] = pr.z;
            out_rxy[o] = make_float2(pr.rx, pr.ry);
            out_valid[o] = pr.ok ? 1 : 0;
            visible += pr.ok ? 1 : 0;
        }
        if (!colour) continue;
        const unsigned any_ok = __ballot_sync(0xffffffffu, in && pr.ok);
        if (!staged && any_ok != 0u && nb > 1) {
            stage_rows(sh_rest, g0, n, shl.stride_rest, shl.offset_rest, nb - 1, s_rest[wib],
                       lane);
            __syncwarp();
            staged = true;
        }
        if (!in) continue;
        float3 col = make_float3(0.f, 0.f, 0.f);
        if (pr.ok)
            col = sh_colour(sh_degree, nb, mx - P.ccx, my - P.ccy, mz - P.ccz,
                            sh_dc + g * (int64_t)shl.stride_dc * 3,
                            s_rest[wib] + lane * (nb - 1) * 3);
        out_color[3 * o + 0] = col.x;
        out_color[3 * o + 1] = col.y;
        out_color[3 * o + 2] = col.z;
    }
    if (vis != nullptr && in) {
        if (with_prologue) vis[g] = (float)visible;  // the step's first count
        else if (visible > 0) vis[g] += (float)visible;
    }
}

// The colour half of preprocess_forward_views_kernel, for a projection that
// ran without it (SH pointers null): view v's colour of Gaussian g from its
// SH rows and the direction from camera centre v, or 0 where valid is 0.
// The rows are staged per warp and the arithmetic is sh_colour's, so the
// colours are bit-identical to the fused projection's.
constexpr int kMaxColourViews = 64;
struct ColourCentres {
    float c[kMaxColourViews][3];
};

__global__ void __launch_bounds__(kPreBlock)
sh_colour_views_kernel(const float* __restrict__ means, const float* __restrict__ sh_dc,
                       const float* __restrict__ sh_rest, mg_sh_layout shl, ColourCentres cc,
                       int n_views, int sh_degree, int64_t n, int64_t view_stride,
                       const int32_t* __restrict__ valid, float* __restrict__ out_color) {
    __shared__ __align__(16) float s_rest[kPreBlock / 32][32 * 15 * 3];
    const int lane = threadIdx.x & 31, wib = threadIdx.x >> 5;
    const int64_t g = (int64_t)blockIdx.x * kPreBlock + threadIdx.x;
    const int64_t g0 = g - lane;
    const bool in = g < n;
    const int nb = (sh_degree + 1) * (sh_degree + 1);
    float mx = 0.f, my = 0.f, mz = 0.f;
    if (in) { mx = means[3 * g + 0]; my = means[3 * g + 1]; mz = means[3 * g + 2]; }
    bool staged = false;
    for (int v = 0; v < n_views; ++v) {
        const int64_t o = (int64_t)v * view_stride + g;
        const bool ok = in && valid[o] != 0;
        const unsigned any_ok = __ballot_sync(0xffffffffu, ok);
        if (!staged && any_ok != 0u && nb > 1) {
            stage_rows(sh_rest, g0, n, shl.stride_rest, shl.offset_rest, nb - 1, s_rest[wib],
                       lane);
            __syncwarp();
            staged = true;
        }
        if (!in) continue;
        float3 col = make_float3(0.f, 0.f, 0.f);
        if (ok)
            col = sh_colour(sh_degree, nb, mx - cc.c[v][0], my - cc.c[v][1], mz - cc.c[v][2],
                            sh_dc + g * (int64_t)shl.stride_dc * 3,
                            s_rest[wib] + lane * (nb - 1) * 3);
        out_color[3 * o + 0] = col.x;
        out_color[3 * o + 1] = col.y;
        out_color[3 * o + 2] = col.z;
    }
}

// Walk the Gaussian's clamped tile rectangle row-major and count (or emit)
// the tiles that pass the exact ellipse test (binning.metal:46-90).
// Saturation cut (engine binning). A tile's pairs behind the depth at which
// Gaussians that cover the whole tile have certainly driven every pixel's
// transmittance below the rasteriser's 1e-4 stop are never read by either
// pass, so they need not be emitted or sorted. Per tile, a histogram over
// kCutBins log-spaced depth bins accumulates each covering Gaussian's optical
// depth -ln(1 - alpha_lb), alpha_lb being a lower bound of its alpha at every
// pixel centre of the tile; the cutoff bin is the first where the running sum
// reaches ln(1e4) + 1 (T <= 3.7e-5 with a margin for float rounding), and
// pairs in later bins are dropped. Kept pairs are a depth-order prefix of
// each tile's list, so images and gradients are unchanged.
// Resident 256-thread CTAs per SM the binning walks' register budget is held
// to (0: none).
#ifndef MG_BIN_MIN_CTAS
#define MG_BIN_MIN_CTAS 4
#endif
constexpr int kCutBins = kSaturationBins;
constexpr float kCutOdScale = 1048576.0f;  // optical depth quantum 2^-20
constexpr uint32_t kCutNeed = 10707140u;   // (ln(1e4) + 1) * 2^20, rounded up

struct CutArgs {
    uint32_t* hist;          // count walks: n_tiles * kCutBins optical depths
    const int32_t* cutoff;   // filtering walks: per-tile last kept bin
    int bin;                 // this Gaussian's depth bin
};

// Depth bin of a Gaussian: log-spaced over the view's depth range, given as
// the bit patterns of the smallest and largest visible depth.
__device__ __forceinline__ int cut_bin(float depth, uint32_t dmin_bits, uint32_t dmax_bits) {
    const float lo = __logf(__uint_as_float(dmin_bits));
    const float hi = __logf(__uint_as_float(dmax_bits));
    // fast division: any deterministic, monotone binning serves the cut
    const float inv = __fdividef((float)kCutBins, fmaxf(hi - lo, 1e-6f));
    const int b = (int)((__logf(depth) - lo) * inv);
    return min(max(b, 0), kCutBins - 1);
}

// Quantised lower bound of the optical depth -ln(1 - alpha) that a Gaussian
// adds at every pixel centre [x0+.5, x1-.5] x [y0+.5, y1-.5] of a tile, or 0
// when it may fall under 1/255 somewhere (then some pixel can skip it). The
// conic's quadratic form is convex, so it is largest at a corner; a corner
// at or past the 1/255 threshold `thr` (the pass test's) ends the search.
// The bound only decides how much of a list is kept, never a blend: fast
// exp/log with a 1e-3 margin on alpha and another on the optical depth.
__device__ __forceinline__ uint32_t tile_optical_depth(float mux, float muy, float ca,
                                                       float cb, float cc, float op, float thr,
                                                       float x0, float x1, float y0,
                                                       float y1) {
    float qmax = 0.0f;
#pragma unroll
    for (int e = 0; e < 4; ++e) {
        const float dx = ((e & 1) ? x1 - 0.5f : x0 + 0.5f) - mux;
        const float dy = ((e & 2) ? y1 - 0.5f : y0 + 0.5f) - muy;
        const float q = __fmaf_rn(ca * dx, dx, __fmaf_rn(2.0f * cb * dx, dy, cc * dy * dy));
        if (q >= thr) return 0u;
        qmax = fmaxf(qmax, q);
    }
    const float alb = fminf(op * __expf(-0.5f * qmax) * 0.999f, 0.999f);
    if (alb < 1.0f / 255.0f) return 0u;
    return (uint32_t)(-__logf(1.0f - alb) * (0.999f * kCutOdScale));
}

// With `rec` given (count walks), the walk also leaves a record of its
// decisions: rectangles of at most 64 tiles get the pass mask over the
// rectangle in row-major order plus the rectangle itself (and the Gaussian's
// depth bin), so the emission can expand the mask instead of testing every
// tile again. kCut: 1 adds covering Gaussians to the saturation histogram,
// 2 keeps only tiles whose cutoff bin is not before the Gaussian's bin.
// Emitted pair tiles are offset by tile_base (a view's first tile in a batch).
template <bool kEmit64, bool kEmitPair, int kCut = 0>
__device__ __forceinline__ uint32_t bin_walk(
    float mux, float muy, float rx, float ry, float ca, float cb, float cc,
    float op, uint32_t dbits, int tile, int tiles_x, int tiles_y, int W, int H,
    uint64_t* keys, int32_t* ids, uint32_t* pair_tiles, uint32_t* pair_ids,
    int64_t write_at, uint32_t cap, int32_t gid, uint4* rec = nullptr,
    CutArgs cut = CutArgs{nullptr, nullptr, 0}, uint32_t tile_base = 0u,
    const TileRect* known_rect = nullptr) {
    const TileRect tr =
        known_rect ? *known_rect : tile_rect(mux, muy, rx, ry, tile, tiles_x, tiles_y);
    const float oa = 255.0f * op;
    if (oa <= 1.0f) return 0u;
    const float thr = 2.0f * log_f32_via_f64(oa);
    const int rw = tr.x1 - tr.x0 + 1, rh = tr.y1 - tr.y0 + 1;
    const bool masked = rec != nullptr && rw * rh <= 64;
    // a tile fits in the 1/255 ellipse {q < thr} only if its inscribed circle
    // does: the ellipse's smaller semi-axis sqrt(thr / lambda_max(conic))
    // must reach half the side, lambda_max <= 4 thr / (tile - 1)^2
    bool can_cover = false;
    if (kCut == 1) {
        const float half_tr = 0.5f * (ca + cc);
        const float lmax = half_tr + sqrtf(fmaxf(half_tr * half_tr - (ca * cc - cb * cb), 0.0f));
        const float side = (float)(tile - 1);
        can_cover = lmax * side * side <= 4.0f * thr * 1.001f;
    }
    uint64_t mask = 0ull;
    int bit = 0;
    uint32_t cnt = 0u;
    // inside the rectangle a tile's bottom (right) edge is the next row's
    // top (next tile's left) edge: (ty + 1) * tile < H there
    const RectQuadratic rq(mux, muy, ca, cb, cc);
    RowEdge top = rq.row_edge((float)(tr.y0 * tile));
    for (int ty = tr.y0; ty <= tr.y1; ++ty) {
        const RowEdge bottom = rq.row_edge(fminf((float)((ty + 1) * tile), (float)H));
        const float y0 = top.y, y1 = bottom.y;
        ColEdge right = rq.col_edge((float)(tr.x0 * tile));
        float q_right = rq.side_q(right, top, bottom);
        for (int tx = tr.x0; tx <= tr.x1; ++tx) {
            const ColEdge left = right;
            const float q_left = q_right;
            right = rq.col_edge(fminf((float)((tx + 1) * tile), (float)W));
            q_right = rq.side_q(right, top, bottom);
            const float x0 = left.x, x1 = right.x;
            const int b = bit++;
            if (rq.min_q_sides(left, right, top, bottom, q_left, q_right) >= thr) continue;
            if (masked) mask |= 1ull << b;
            if (kCut == 1 && can_cover) {
                const uint32_t q =
                    tile_optical_depth(mux, muy, ca, cb, cc, op, thr, x0, x1, y0, y1);
                if (q) atomicAdd(&cut.hist[(ty * tiles_x + tx) * kCutBins + cut.bin], q);
            }
            if (kCut == 2 && cut.cutoff[ty * tiles_x + tx] < cut.bin) continue;
            if (kEmit64 || kEmitPair) {
                if (cnt < cap) {
                    const uint32_t tid = (uint32_t)(ty * tiles_x + tx);
                    if (kEmit64) {
                        keys[write_at + cnt] = ((uint64_t)tid << 32) | (uint64_t)dbits;
                        ids[write_at + cnt] = gid;
                    } else {
                        pair_tiles[write_at + cnt] = tile_base + tid;
                        pair_ids[write_at + cnt] = (uint32_t)gid;
                    }
                }
            }
            ++cnt;
        }
        top = bottom;
    }
    if (rec)  // width 0 marks a rectangle the emission must walk again
        *rec = make_uint4((uint32_t)mask, (uint32_t)(mask >> 32),
                          (uint32_t)tr.x0 | ((uint32_t)tr.y0 << 16),
                          (masked ? ((uint32_t)rw | ((uint32_t)rh << 8)) : 0u) |
                              ((uint32_t)cut.bin << 16));
    return cnt;
}

// Rectangles of more than kCoopTiles tiles (the largest whose pass mask a
// record holds) are walked by a whole warp, one Gaussian at a time: one lane
// walking hundreds of tiles would hold its warp, and at the end of a launch
// its SM, while the other lanes idle. Every lane calls warp_walk with the
// same Gaussian. The lanes form a grid of cw columns x ch rows (cw = the
// rectangle's width up to 32, ch = 32 / cw) stepped over the rectangle;
// each tile gets bin_walk's test on edges computed from the same
// coordinates, so the decisions, the histogram adds and the pair set are
// bin_walk's (a tile's top edge is the row above's bottom edge there, and a
// left edge the previous column's right edge). Pairs are written in the order
// the warp finds them, not row-major: a Gaussian's pairs lie in distinct
// tiles, so the stable tile sort puts them in the same places either way.
// Returns the count (kept pairs for kCut 2) in every lane.
constexpr int kCoopTiles = 64;

template <bool kEmitPair, int kCut>
__device__ __forceinline__ uint32_t warp_walk(int lane, float mux, float muy, float rx, float ry,
                                              float ca, float cb, float cc, float op, int tile,
                                              int tiles_x, int tiles_y, int W, int H,
                                              uint32_t* pair_tiles, uint32_t* pair_ids,
                                              int64_t write_at, uint32_t cap, uint32_t gid,
                                              CutArgs cut, uint32_t tile_base) {
    const TileRect tr = tile_rect(mux, muy, rx, ry, tile, tiles_x, tiles_y);
    const float oa = 255.0f * op;
    if (oa <= 1.0f) return 0u;
    const float thr = 2.0f * log_f32_via_f64(oa);
    const int rw = tr.x1 - tr.x0 + 1, rh = tr.y1 - tr.y0 + 1;
    bool can_cover = false;  // as in bin_walk
    if (kCut == 1) {
        const float half_tr = 0.5f * (ca + cc);
        const float lmax = half_tr + sqrtf(fmaxf(half_tr * half_tr - (ca * cc - cb * cb), 0.0f));
        const float side = (float)(tile - 1);
        can_cover = lmax * side * side <= 4.0f * thr * 1.001f;
    }
    const RectQuadratic rq(mux, muy, ca, cb, cc);
    const int cw = min(rw, 32), ch = 32 / cw;
    const int cx = lane % cw, cy = lane / cw;
    uint32_t cnt = 0u;
    for (int bx = 0; bx < rw; bx += cw) {
        const int tx = tr.x0 + bx + cx;
        const bool col = cy < ch && bx + cx < rw;
        ColEdge left{}, right{};
        if (col) {
            left = rq.col_edge((float)(tx * tile));
            right = rq.col_edge(fminf((float)((tx + 1) * tile), (float)W));
        }
        for (int by = 0; by < rh; by += ch) {
            const int ty = tr.y0 + by + cy;
            bool pass = false;
            if (col && by + cy < rh) {
                const RowEdge top = rq.row_edge((float)(ty * tile));
                const RowEdge bottom = rq.row_edge(fminf((float)((ty + 1) * tile), (float)H));
                pass = !(rq.min_q(left, right, top, bottom) >= thr);
                if (kCut == 1 && pass && can_cover) {
                    const uint32_t q = tile_optical_depth(mux, muy, ca, cb, cc, op, thr, left.x,
                                                          right.x, top.y, bottom.y);
                    if (q) atomicAdd(&cut.hist[(ty * tiles_x + tx) * kCutBins + cut.bin], q);
                }
                if (kCut == 2 && pass && cut.cutoff[ty * tiles_x + tx] < cut.bin) pass = false;
            }
            if (kEmitPair) {
                const uint32_t bal = __ballot_sync(0xffffffffu, pass);
                if (pass) {
                    const uint32_t k = cnt + (uint32_t)__popc(bal & ((1u << lane) - 1u));
                    if (k < cap) {
                        pair_tiles[write_at + k] = tile_base + (uint32_t)(ty * tiles_x + tx);
                        pair_ids[write_at + k] = gid;
                    }
                }
                cnt += (uint32_t)__popc(bal);
            } else {
                cnt += pass ? 1u : 0u;
            }
        }
    }
    if (!kEmitPair) cnt = __reduce_add_sync(0xffffffffu, cnt);
    return cnt;
}

__device__ __forceinline__ bool coop_rect(const TileRect& tr) {
    return (tr.x1 - tr.x0 + 1) * (tr.y1 - tr.y0 + 1) > kCoopTiles;
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

// Reorders a 256-thread block's work items by a cost class (a counting sort
// in shared memory): returns the block-local index this thread takes, so
// each warp holds items of similar cost instead of waiting on its largest.
// Every output is indexed by item, so the order changes nothing but the
// warps' divergence. `cls` is in [0, kCostClasses); put items past the end
// in the last class.
constexpr int kCostClasses = 160;  // 5 per lane of the scanning warp
__device__ __forceinline__ int block_sorted_slot(int cls) {
    static_assert(kCostClasses % 32 == 0, "whole classes per lane");
    constexpr int kPerLane = kCostClasses / 32;
    __shared__ int s_count[kCostClasses];
    __shared__ int s_slot[256];
    const int tid = threadIdx.x;
    for (int k = tid; k < kCostClasses; k += blockDim.x) s_count[k] = 0;
    __syncthreads();
    const int rank = atomicAdd(&s_count[cls], 1);
    __syncthreads();
    if (tid < 32) {  // exclusive prefix over the classes: kPerLane per lane
        int c[kPerLane], sum = 0;
#pragma unroll
        for (int k = 0; k < kPerLane; ++k) {
            c[k] = s_count[tid * kPerLane + k];
            sum += c[k];
        }
        int incl = sum;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const int t = __shfl_up_sync(0xffffffffu, incl, o);
            if (tid >= o) incl += t;
        }
        int run = incl - sum;
#pragma unroll
        for (int k = 0; k < kPerLane; ++k) {
            s_count[tid * kPerLane + k] = run;
            run += c[k];
        }
    }
    __syncthreads();
    s_slot[s_count[cls] + rank] = tid;
    __syncthreads();
    return s_slot[tid];
}

// Cost class of a Gaussian's count walk: the shape of its tile rectangle
// (rows, then columns), so a warp's lanes mostly run the same row and column
// loop trip counts; no tile (invalid) first, rectangles the whole warp walks
// (warp_walk) together, items past the end last.
__device__ __forceinline__ int64_t block_sorted_gaussian(const float2* __restrict__ uv,
                                                         const float2* __restrict__ rxy,
                                                         const int32_t* __restrict__ valid,
                                                         int64_t n, int tile, int tiles_x,
                                                         int tiles_y) {
    const int64_t own = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    int cls = kCostClasses - 1;
    if (own < n) {
        cls = 0;
        if (valid[own] != 0) {
            const float2 mu = uv[own], r = rxy[own];
            const TileRect tr = tile_rect(mu.x, mu.y, r.x, r.y, tile, tiles_x, tiles_y);
            const int rh = min(tr.y1 - tr.y0 + 1, 9), rw = min(tr.x1 - tr.x0 + 1, 16);
            cls = coop_rect(tr) ? 145 : 1 + (rh - 1) * 16 + (rw - 1);  // 1 .. 145
        }
    }
    return (int64_t)blockIdx.x * blockDim.x + block_sorted_slot(cls);
}

// Depth sort keys. Valid depths are positive, so their bit patterns order
// like the depths. When the view's depth range (range[0] = ~smallest bits,
// range[1] = largest, from the saturation cut's range pass) spans fewer than
// 2^24 - 1 patterns, keys are taken relative to the smallest: the same order,
// every key below 2^24, so the sort's top 8-bit pass finds one digit and only
// copies. Gaussians that claim no tile take the largest key and sort last.
__device__ __forceinline__ bool relative_depth_keys(const uint32_t* range) {
    return range != nullptr && range[1] != 0u && range[1] - ~range[0] < 0x00ffffffu;
}
__device__ __forceinline__ uint32_t depth_key(float d, const uint32_t* range) {
    return relative_depth_keys(range) ? __float_as_uint(d) - ~range[0] : __float_as_uint(d);
}
__device__ __forceinline__ uint32_t no_depth_key(const uint32_t* range) {
    return relative_depth_keys(range) ? 0x00ffffffu : 0xffffffffu;
}
// Batch keys (BinViews::batch_keys): the depth relative to the view's
// smallest, each view sorted as a segment of its own; rows without a pair
// take 2^24 - 1, so when a view's range spans fewer than 2^24 patterns the
// top 8-bit pass finds one digit in that view and only copies.
constexpr uint32_t kBatchNoDepthKey = 0x00ffffffu;
__device__ __forceinline__ uint32_t view_depth_key(float d, const uint32_t* range,
                                                   int batch_keys) {
    return batch_keys ? __float_as_uint(d) - ~range[0] : depth_key(d, range);
}
__device__ __forceinline__ uint32_t view_no_depth_key(const uint32_t* range, int batch_keys) {
    return batch_keys ? kBatchNoDepthKey : no_depth_key(range);
}

// Stage A of the two-stage binning: tile counts plus the depth sort keys
// (depth_key: Gaussians that claim no tile sort behind every valid depth).
__global__ void __launch_bounds__(256, MG_BIN_MIN_CTAS) bin_count_depth_kernel(const float2* __restrict__ uv,
                                       const float2* __restrict__ rxy,
                                       const float* __restrict__ conic,
                                       const float* __restrict__ opacity,
                                       const int32_t* __restrict__ valid,
                                       const float* __restrict__ depth, int64_t n,
                                       int W, int H, int tile, int tiles_x,
                                       int tiles_y, uint32_t* __restrict__ counts,
                                       uint32_t* __restrict__ dkeys,
                                       uint32_t* __restrict__ dvals,
                                       uint4* __restrict__ recs,
                                       const uint32_t* __restrict__ range,
                                       uint32_t* __restrict__ hist, BinViews bv) {
    const int v = blockIdx.y;
    {  // view v's slice of the batch
        const int64_t vin = (int64_t)v * bv.in_stride, vout = (int64_t)v * n;
        uv += vin; rxy += vin; conic += 3 * vin; valid += vin; depth += vin;
        opacity += (int64_t)v * bv.opac_stride;
        counts += vout; dkeys += vout; dvals += vout; recs += vout;
        if (range) range += 2 * v;
        if (hist) hist += (int64_t)v * tiles_x * tiles_y * kCutBins;
    }
    const int64_t g = block_sorted_gaussian(uv, rxy, valid, n, tile, tiles_x, tiles_y);
    const int lane = threadIdx.x & 31;
    uint32_t c = 0u;
    bool big = false;
    int gbin = 0;
    if (g < n && valid[g] != 0) {
        const float2 mu = uv[g], r = rxy[g];
        const TileRect tr = tile_rect(mu.x, mu.y, r.x, r.y, tile, tiles_x, tiles_y);
        big = coop_rect(tr);
        if (hist) gbin = cut_bin(depth[g], ~range[0], range[1]);
        if (!big) {
            if (hist)
                c = bin_walk<false, false, 1>(mu.x, mu.y, r.x, r.y, conic[3 * g],
                                              conic[3 * g + 1], conic[3 * g + 2], opacity[g],
                                              0u, tile, tiles_x, tiles_y, W, H, nullptr,
                                              nullptr, nullptr, nullptr, 0, 0u, 0, recs + g,
                                              CutArgs{hist, nullptr, gbin}, 0u, &tr);
            else
                c = bin_walk<false, false>(mu.x, mu.y, r.x, r.y, conic[3 * g],
                                           conic[3 * g + 1], conic[3 * g + 2], opacity[g], 0u,
                                           tile, tiles_x, tiles_y, W, H, nullptr, nullptr,
                                           nullptr, nullptr, 0, 0u, 0, recs + g,
                                           CutArgs{nullptr, nullptr, 0}, 0u, &tr);
        }
    }
    // the warp's large rectangles, one at a time (their records say: walk
    // again)
    for (uint32_t pend = __ballot_sync(0xffffffffu, big); pend; pend &= pend - 1u) {
        const int src = __ffs(pend) - 1;
        const int64_t gs = __shfl_sync(0xffffffffu, g, src);
        const int bin = __shfl_sync(0xffffffffu, gbin, src);
        const float2 mu = uv[gs], r = rxy[gs];
        const float ca = conic[3 * gs], cb = conic[3 * gs + 1], cc = conic[3 * gs + 2];
        const uint32_t k =
            hist ? warp_walk<false, 1>(lane, mu.x, mu.y, r.x, r.y, ca, cb, cc, opacity[gs], tile,
                                       tiles_x, tiles_y, W, H, nullptr, nullptr, 0, 0u, 0u,
                                       CutArgs{hist, nullptr, bin}, 0u)
                 : warp_walk<false, 0>(lane, mu.x, mu.y, r.x, r.y, ca, cb, cc, opacity[gs], tile,
                                       tiles_x, tiles_y, W, H, nullptr, nullptr, 0, 0u, 0u,
                                       CutArgs{nullptr, nullptr, 0}, 0u);
        if (lane == src) {
            c = k;
            recs[g] = make_uint4(0u, 0u, 0u, (uint32_t)bin << 16);
        }
    }
    if (g >= n) return;
    counts[g] = c;
    dkeys[g] = c > 0u ? view_depth_key(depth[g], range, bv.batch_keys)
                      : view_no_depth_key(range, bv.batch_keys);
    dvals[g] = (uint32_t)((int64_t)v * n + g);
}

// The keep bits of tiles x0 .. x0 + 63 of one (row, bin) entry of the keep
// table (bit i: tile x0 + i).
__device__ __forceinline__ uint64_t keep_bits(const uint64_t* __restrict__ words, uint32_t x0) {
    const uint32_t w = x0 >> 6, s = x0 & 63u;
    uint64_t bits = words[w] >> s;
    if (s) bits |= words[w + 1] << (64u - s);
    return bits;
}

// Stage B: emit every (tile, Gaussian) pair with Gaussians in depth order.
// offsets are the exclusive scan of the counts in that order; each thread
// writes at most its own count so a disagreement can never overrun.
__global__ void __launch_bounds__(256, MG_BIN_MIN_CTAS) bin_emit_kernel(const float2* __restrict__ uv,
                                const float2* __restrict__ rxy,
                                const float* __restrict__ conic,
                                const float* __restrict__ opacity,
                                const uint32_t* __restrict__ sorted_gid,
                                const uint32_t* __restrict__ counts,
                                const uint32_t* __restrict__ offsets, int64_t n,
                                int64_t m, int W, int H, int tile, int tiles_x,
                                int tiles_y, const uint4* __restrict__ recs,
                                const int32_t* __restrict__ cutoff,
                                const uint64_t* __restrict__ keep,
                                uint32_t* __restrict__ pair_tiles,
                                uint32_t* __restrict__ pair_ids, BinViews bv) {
    const int64_t sl = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    const int lane = threadIdx.x & 31;
    const int n_tiles = tiles_x * tiles_y;
    // view v owns the batch's sorted slots [v n, (v + 1) n); its pairs carry
    // tiles v * n_tiles + t and the Gaussian's index within the view
    const int v = blockIdx.y;
    const uint32_t tile_base = (uint32_t)v * (uint32_t)n_tiles;
    {
        const int64_t vin = (int64_t)v * bv.in_stride;
        uv += vin; rxy += vin; conic += 3 * vin;
        opacity += (int64_t)v * bv.opac_stride;
        if (cutoff) cutoff += (int64_t)v * n_tiles;
        if (keep) keep += (int64_t)v * tiles_y * kCutBins * cut_keep_stride(tiles_x);
    }
    int gbin = 0;
    uint32_t g = 0u, cnt = 0u;
    int64_t at = 0;
    bool again = false;
    if (sl < n) {
        const int64_t s = (int64_t)v * n + sl;
        const uint32_t gv = sorted_gid[s];
        g = gv - (uint32_t)v * (uint32_t)n;
        if ((int64_t)g < n) cnt = counts[gv];
        if (cnt != 0u) {
            at = offsets[s];
            if (at + cnt > m) cnt = 0u;
        }
        if (cnt != 0u) {
            const uint4 rec = recs[gv];
            const uint32_t rw = rec.w & 0xffu, rh = (rec.w >> 8) & 0xffu;
            gbin = (int)((rec.w >> 16) & 0xffu);
            again = rw == 0u;  // a large rectangle: the warp walks it again
            if (!again) {
                // the count walk's decisions: row-major bits over the rectangle
                uint64_t mask = (uint64_t)rec.x | ((uint64_t)rec.y << 32);
                const uint32_t x0 = rec.z & 0xffffu, y0 = rec.z >> 16;
                const uint64_t row_bits = rw == 64u ? ~0ull : (1ull << rw) - 1ull;
                uint32_t k = 0u;
                const int ks = cut_keep_stride(tiles_x);
                for (uint32_t r = 0; r < rh && mask; ++r) {
                    uint64_t row = mask & row_bits;
                    mask >>= rw;
                    if (keep)  // only the tiles the cut keeps
                        row &= keep_bits(keep + ((int64_t)(y0 + r) * kCutBins + gbin) * ks, x0);
                    const uint32_t trow = (y0 + r) * (uint32_t)tiles_x + x0;
                    while (row) {
                        const uint32_t b = (uint32_t)__ffsll((long long)row) - 1u;
                        row &= row - 1ull;
                        if (!keep && cutoff && cutoff[trow + b] < gbin) continue;
                        if (k < cnt) {
                            pair_tiles[at + k] = tile_base + trow + b;
                            pair_ids[at + k] = g;
                        }
                        ++k;
                    }
                }
            }
        }
    }
    for (uint32_t pend = __ballot_sync(0xffffffffu, again); pend; pend &= pend - 1u) {
        const int src = __ffs(pend) - 1;
        const uint32_t gs = __shfl_sync(0xffffffffu, g, src);
        const int bin = __shfl_sync(0xffffffffu, gbin, src);
        const int64_t ats = __shfl_sync(0xffffffffu, at, src);
        const uint32_t cap = __shfl_sync(0xffffffffu, cnt, src);
        const float2 mu = uv[gs], r = rxy[gs];
        const float ca = conic[3 * (int64_t)gs], cb = conic[3 * (int64_t)gs + 1],
                    cc = conic[3 * (int64_t)gs + 2];
        if (cutoff)
            warp_walk<true, 2>(lane, mu.x, mu.y, r.x, r.y, ca, cb, cc, opacity[gs], tile,
                               tiles_x, tiles_y, W, H, pair_tiles, pair_ids, ats, cap, gs,
                               CutArgs{nullptr, cutoff, bin}, tile_base);
        else
            warp_walk<true, 0>(lane, mu.x, mu.y, r.x, r.y, ca, cb, cc, opacity[gs], tile,
                               tiles_x, tiles_y, W, H, pair_tiles, pair_ids, ats, cap, gs,
                               CutArgs{nullptr, nullptr, 0}, tile_base);
    }
}

// Saturation cut, step 1: the view's visible depth range as bit patterns
// (range[0] holds the complement of the smallest, so both are maxima over
// zero-initialised words).
__global__ void __launch_bounds__(256)
bin_depth_range_kernel(const int32_t* __restrict__ valid, const float* __restrict__ depth,
                       int64_t n, uint32_t* __restrict__ range, int64_t in_stride) {
    valid += blockIdx.y * in_stride;  // view blockIdx.y of a batch
    depth += blockIdx.y * in_stride;
    range += 2 * blockIdx.y;
    __shared__ uint32_t s_lo[8], s_hi[8];
    uint32_t lo = 0u, hi = 0u;
    auto take = [&](int32_t ok, float d) {
        if (ok != 0) {
            const uint32_t bits = __float_as_uint(d);  // positive depths
            lo = max(lo, ~bits);
            hi = max(hi, bits);
        }
    };
    const int64_t tid = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    const int64_t nthreads = (int64_t)gridDim.x * blockDim.x;
    // 16-byte loads of both arrays when they share an alignment (four rows in
    // flight per load pair), single rows before and after the aligned body
    const uintptr_t av = reinterpret_cast<uintptr_t>(valid), ad = reinterpret_cast<uintptr_t>(depth);
    int64_t head = n, body = 0;
    if ((av & 15u) == (ad & 15u) && (av & 3u) == 0u) {
        const int64_t lead = (int64_t)(((16u - (av & 15u)) & 15u) >> 2);
        head = lead < n ? lead : n;
        body = (n - head) >> 2;
    }
    for (int64_t g = tid; g < head; g += nthreads) take(valid[g], depth[g]);
    const int4* v4 = reinterpret_cast<const int4*>(valid + head);
    const float4* d4 = reinterpret_cast<const float4*>(depth + head);
    for (int64_t i = tid; i < body; i += nthreads) {
        const int4 ok = v4[i];
        const float4 d = d4[i];
        take(ok.x, d.x); take(ok.y, d.y); take(ok.z, d.z); take(ok.w, d.w);
    }
    for (int64_t g = head + 4 * body + tid; g < n; g += nthreads) take(valid[g], depth[g]);
    lo = __reduce_max_sync(0xffffffffu, lo);
    hi = __reduce_max_sync(0xffffffffu, hi);
    const int warp = threadIdx.x >> 5;
    if ((threadIdx.x & 31) == 0) { s_lo[warp] = lo; s_hi[warp] = hi; }
    __syncthreads();
    if (threadIdx.x == 0) {
        for (int w = 1; w < (int)(blockDim.x >> 5); ++w) {
            lo = max(lo, s_lo[w]);
            hi = max(hi, s_hi[w]);
        }
        if (hi != 0u) {  // one pair of atomics per block
            atomicMax(&range[0], lo);
            atomicMax(&range[1], hi);
        }
    }
}

// Saturation cut, step 2: per tile, the first depth bin whose running optical
// depth reaches kCutNeed (the last bin when none does).
__global__ void bin_cutoff_kernel(const uint32_t* __restrict__ hist, int n_tiles,
                                  int32_t* __restrict__ cutoff) {
    static_assert(kCutBins == 64, "two bins per lane");
    const int t = (int)(((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5);
    const int lane = threadIdx.x & 31;
    if (t >= n_tiles) return;  // whole warps
    const uint2 h = reinterpret_cast<const uint2*>(hist + (int64_t)t * kCutBins)[lane];
    // inclusive running sums of bins 2*lane and 2*lane + 1
    unsigned long long a = h.x, b = (unsigned long long)h.x + h.y, incl = b;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const unsigned long long v = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += v;
    }
    const unsigned long long before = incl - b;
    a += before;
    b += before;
    const uint32_t hit_a = __ballot_sync(0xffffffffu, a >= kCutNeed);
    const uint32_t hit_b = __ballot_sync(0xffffffffu, b >= kCutNeed);
    if (lane == 0) {
        int cut = kCutBins - 1;
        if (hit_a | hit_b) {
            const int la = hit_a ? __ffs(hit_a) - 1 : 64, lb = hit_b ? __ffs(hit_b) - 1 : 64;
            cut = min(2 * la, 2 * lb + 1);
        }
        cutoff[t] = cut;
    }
}

// Saturation cut, step 2b: the keep table (see cut_keep_stride), one thread
// per (view, tile row, bin, word).
__global__ void bin_keep_kernel(const int32_t* __restrict__ cutoff, int tiles_x, int tiles_y,
                                int n_views, uint64_t* __restrict__ keep) {
    const int stride = cut_keep_stride(tiles_x);
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= (int64_t)n_views * tiles_y * kCutBins * stride) return;
    const int w = (int)(i % stride);
    const int64_t rb = i / stride;
    const int b = (int)(rb % kCutBins);
    const int64_t row = rb / kCutBins;  // view * tiles_y + tile row
    const int32_t* c = cutoff + row * tiles_x;
    uint64_t bits = 0ull;
    for (int k = 0; k < 64; ++k) {
        const int tx = w * 64 + k;
        if (tx < tiles_x && c[tx] >= b) bits |= 1ull << k;
    }
    keep[i] = bits;
}

// Saturation cut, step 3: per Gaussian, the pairs that survive the cut (its
// count and depth key are rewritten; the emission keeps the same pairs).
__global__ void __launch_bounds__(256, MG_BIN_MIN_CTAS) bin_recount_kernel(const float2* __restrict__ uv,
                                   const float2* __restrict__ rxy,
                                   const float* __restrict__ conic,
                                   const float* __restrict__ opacity,
                                   const float* __restrict__ depth, int64_t n, int W, int H,
                                   int tile, int tiles_x, int tiles_y,
                                   const uint4* __restrict__ recs,
                                   const int32_t* __restrict__ cutoff,
                                   const uint64_t* __restrict__ keep,
                                   const uint32_t* __restrict__ range,
                                   uint32_t* __restrict__ counts,
                                   uint32_t* __restrict__ dkeys, BinViews bv) {
    const int v = blockIdx.y;
    {  // view v's slice of the batch
        const int64_t vin = (int64_t)v * bv.in_stride, vout = (int64_t)v * n;
        uv += vin; rxy += vin; conic += 3 * vin; depth += vin;
        opacity += (int64_t)v * bv.opac_stride;
        counts += vout; dkeys += vout; recs += vout;
        cutoff += (int64_t)v * tiles_x * tiles_y;
        if (keep) keep += (int64_t)v * tiles_y * kCutBins * cut_keep_stride(tiles_x);
        range += 2 * v;
    }
    const int ks = cut_keep_stride(tiles_x);
    const int64_t g = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    const int lane = threadIdx.x & 31;
    const bool has = g < n && counts[g] != 0u;
    uint32_t kept = 0u;
    bool again = false;
    int gbin = 0;
    if (has) {
        const uint4 rec = recs[g];
        const uint32_t rw = rec.w & 0xffu, rh = (rec.w >> 8) & 0xffu;
        gbin = (int)((rec.w >> 16) & 0xffu);
        if (rw != 0u) {
            uint64_t mask = (uint64_t)rec.x | ((uint64_t)rec.y << 32);
            const uint32_t x0 = rec.z & 0xffffu, y0 = rec.z >> 16;
            const uint64_t row_bits = rw == 64u ? ~0ull : (1ull << rw) - 1ull;
            for (uint32_t r = 0; r < rh && mask; ++r) {
                uint64_t row = mask & row_bits;
                mask >>= rw;
                if (keep) {  // the row's kept tiles from the keep table
                    kept += __popcll(row & keep_bits(keep + ((int64_t)(y0 + r) * kCutBins + gbin) * ks, x0));
                    continue;
                }
                const uint32_t trow = (y0 + r) * (uint32_t)tiles_x + x0;
                while (row) {
                    const uint32_t b = (uint32_t)__ffsll((long long)row) - 1u;
                    row &= row - 1ull;
                    kept += cutoff[trow + b] >= gbin;
                }
            }
        } else {
            again = true;  // a large rectangle: the warp walks it again
        }
    }
    for (uint32_t pend = __ballot_sync(0xffffffffu, again); pend; pend &= pend - 1u) {
        const int src = __ffs(pend) - 1;
        const int64_t gs = __shfl_sync(0xffffffffu, g, src);
        const int bin = __shfl_sync(0xffffffffu, gbin, src);
        const float2 mu = uv[gs], r = rxy[gs];
        const uint32_t k = warp_walk<false, 2>(
            lane, mu.x, mu.y, r.x, r.y, conic[3 * gs], conic[3 * gs + 1], conic[3 * gs + 2],
            opacity[gs], tile, tiles_x, tiles_y, W, H, nullptr, nullptr, 0, 0u, 0u,
            CutArgs{nullptr, cutoff, bin}, 0u);
        if (lane == src) kept = k;
    }
    if (!has) return;
    counts[g] = kept;
    if (kept == 0u) dkeys[g] = view_no_depth_key(range, bv.batch_keys);
}

// Per-view pair totals of a batch: view v's pairs start at the scan value of
// its first sorted slot v * n.
__global__ void view_totals_kernel(const uint32_t* __restrict__ offsets, int64_t n,
                                   int n_views,
                                   int64_t* __restrict__ totals) {
    const int v = threadIdx.x;
    if (v > n_views) return;
    if (v == n_views) {
        totals[n_views + 1] = 0;
        return;
    }
    const int64_t next = v + 1 < n_views ? (int64_t)offsets[(int64_t)(v + 1) * n]
                                         : totals[n_views];
    totals[v] = next - (int64_t)offsets[(int64_t)v * n];
}

__global__ void view_tile_offsets_kernel(const int32_t* __restrict__ global, int n_tiles,
                                         int n_views, int32_t* __restrict__ local) {
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= (int64_t)n_views * (n_tiles + 1)) return;
    const int64_t v = i / (n_tiles + 1), t = i - v * (n_tiles + 1);
    local[i] = global[v * n_tiles + t] - global[v * n_tiles];
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

mg_status launch_preprocess_forward_views(const float* means, const float* quats,
                                          const float* scales, const float* sh_dc,
                                          const float* sh_rest, mg_sh_layout shl,
                                          const float* opacities, const mg_camera* cams,
                                          int n_views, int sh_degree, int64_t n,
                                          int64_t view_stride, float* uv, float* conic,
                                          float* depth, float* rxy, int32_t* valid,
                                          float* color, float* vis,
                                          const mg_step_prologue* prologue,
                                          cudaStream_t stream) {
    if (n == 0) return MG_OK;
    const mg_step_prologue none{};
    for (int v0 = 0; v0 < n_views; v0 += kMaxViewsPerLaunch) {
        const int nv = std::min(kMaxViewsPerLaunch, n_views - v0);
        ViewCams vc;
        for (int k = 0; k < nv; ++k) vc.c[k] = make_cam_params(cams[v0 + k]);
        const int64_t o = (int64_t)v0 * view_stride;
        // the prologue runs with the first launch; later launches (more than
        // 16 views) project the activations it wrote and add to the count
        const bool pro = prologue != nullptr && v0 == 0;
        const float* sc = scales;
        const float* op = opacities;
        if (prologue != nullptr && v0 > 0) {
            const bool filt = prologue->filter_3d != nullptr;
            sc = filt ? prologue->out_scales : prologue->act_scales;
            op = filt ? prologue->out_opac : prologue->act_opac;
        }
        preprocess_forward_views_kernel<<<ceil_div(n, kPreBlock), kPreBlock, 0, stream>>>(
            means, quats, sc, sh_dc, sh_rest, shl, op, vc, nv, sh_degree, n, view_stride,
            reinterpret_cast<float2*>(uv) + o, conic + 3 * o, depth + o,
            reinterpret_cast<float2*>(rxy) + o, valid + o, color ? color + 3 * o : nullptr, vis,
            pro ? *prologue : none, pro);
        MG_TRY(check_launch("preprocess_forward_views"));
    }
    return MG_OK;
}

mg_status launch_sh_colour_views(const float* means, const float* sh_dc, const float* sh_rest,
                                mg_sh_layout shl, const float* cam_centers, int n_views,
                                int sh_degree, int64_t n, int64_t view_stride,
                                const int32_t* valid, float* color, cudaStream_t stream) {
    if (n == 0 || n_views == 0) return MG_OK;
    ColourCentres cc;
    for (int v = 0; v < n_views; ++v)
        for (int k = 0; k < 3; ++k) cc.c[v][k] = cam_centers[3 * v + k];
    sh_colour_views_kernel<<<ceil_div(n, kPreBlock), kPreBlock, 0, stream>>>(
        means, sh_dc, sh_rest, shl, cc, n_views, sh_degree, n, view_stride, valid, color);
    return check_launch("sh_colour_views");
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
                                 uint32_t* cut_range, uint32_t* cut_hist, int32_t* cutoff,
                                 const BinViews& bv, cudaStream_t stream) {
    if (n == 0 || bv.n_views == 0) return MG_OK;
    const bool cut = cut_hist != nullptr;
    const int V = bv.n_views;
    if (cut_range) {
        const int per_view = (int)std::max<int64_t>(1, std::min<int64_t>(
                                 ceil_div(n, 256), ceil_div(148 * 4, V)));
        bin_depth_range_kernel<<<dim3(per_view, V), 256, 0, stream>>>(valid, depth, n,
                                                                       cut_range, bv.in_stride);
        MG_TRY(check_launch("bin_depth_range"));
    }
    const dim3 grid((unsigned)ceil_div(n, 256), (unsigned)V);
    bin_count_depth_kernel<<<grid, 256, 0, stream>>>(
        reinterpret_cast<const float2*>(uv), reinterpret_cast<const float2*>(rxy), conic,
        opacity, valid, depth, n, W, H, tile, tiles_x, tiles_y, counts, dkeys, dvals, recs,
        cut_range, cut_hist, bv);
    MG_TRY(check_launch("bin_count_depth"));
    if (!cut) return MG_OK;
    const int64_t cut_tiles = (int64_t)tiles_x * tiles_y * V;
    bin_cutoff_kernel<<<ceil_div(cut_tiles * 32, 256), 256, 0, stream>>>(cut_hist,
                                                                       (int)cut_tiles, cutoff);
    MG_TRY(check_launch("bin_cutoff"));
    uint64_t* keep = nullptr;
    if (cut_keep_fits(tiles_x)) {  // over the histogram, which the cutoff pass has consumed
        keep = reinterpret_cast<uint64_t*>(cut_hist);
        const int64_t words = (int64_t)V * tiles_y * kCutBins * cut_keep_stride(tiles_x);
        bin_keep_kernel<<<ceil_div(words, 256), 256, 0, stream>>>(cutoff, tiles_x, tiles_y, V,
                                                                  keep);
        MG_TRY(check_launch("bin_keep"));
    }
    bin_recount_kernel<<<grid, 256, 0, stream>>>(
        reinterpret_cast<const float2*>(uv), reinterpret_cast<const float2*>(rxy), conic,
        opacity, depth, n, W, H, tile, tiles_x, tiles_y, recs, cutoff, keep, cut_range, counts,
        dkeys, bv);
    return check_launch("bin_recount");
}

mg_status launch_bin_emit(const float* uv, const float* rxy, const float* conic,
                          const float* opacity, const uint32_t* sorted_gid,
                          const uint32_t* counts, const uint32_t* offsets, int64_t n,
                          int64_t m, int W, int H, int tile, int tiles_x, int tiles_y,
                          const uint4* recs, const int32_t* cutoff, const uint64_t* keep,
                          uint32_t* pair_tiles, uint32_t* pair_ids, const BinViews& bv,
                          cudaStream_t stream) {
    if (n == 0 || m == 0 || bv.n_views == 0) return MG_OK;
    bin_emit_kernel<<<dim3((unsigned)ceil_div(n, 256), (unsigned)bv.n_views), 256, 0, stream>>>(
        reinterpret_cast<const float2*>(uv), reinterpret_cast<const float2*>(rxy), conic,
        opacity, sorted_gid, counts, offsets, n, m, W, H, tile, tiles_x, tiles_y,
        recs, cutoff, cutoff ? keep : nullptr, pair_tiles, pair_ids, bv);
    return check_launch("bin_emit");
}

mg_status launch_view_totals(const uint32_t* offsets, int64_t n, int n_views,
                             int64_t* totals, cudaStream_t stream) {
    view_totals_kernel<<<1, ((n_views + 1 + 31) / 32) * 32, 0, stream>>>(offsets, n, n_views,
                                                                         totals);
    return check_launch("view_totals");
}

mg_status launch_view_tile_offsets(const int32_t* global, int n_tiles, int n_views,
                                   int32_t* local, cudaStream_t stream) {
    const int64_t count = (int64_t)n_views * (n_tiles + 1);
    view_tile_offsets_kernel<<<ceil_div(count, 256), 256, 0, stream>>>(global, n_tiles, n_views,
                                                                       local);
    return check_launch("view_tile_offsets");
}

}  // namespace mg
