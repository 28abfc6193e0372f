// Tile rasterisation, forward and backward (rasterize.metal:61-340).
//
// Splat records. Before rasterising, each splat is packed into one 48-byte
// record (mg_pack_splats): centre, the conic pre-scaled so the exponent is
// A dx^2 + B dx dy + C dy^2 (A = -ca/2, B = -cb, C = -cc/2 are exact power-of-
// two scalings), opacity, colour and the constants of the rectangle cull. A
// list entry then costs three 16-byte loads instead of eight scalar gathers.
//
// Work units. A tile's pixels are split into warp blocks of 32 pixels (8x4
// when the tile side is a multiple of 8, else row-major pixels padded to whole
// warps). Both kernels are persistent: every warp takes work items from a
// device counter until the list is exhausted, so a warp that finishes early
// takes more work instead of idling behind a slow one.
//
// Walk. A warp walks its tile's depth-sorted list 32 entries (a chunk) at a
// time. The records of the next chunk are copied into the warp's shared-memory
// double buffer with cp.async while the current chunk is processed, and the
// list ids two chunks ahead are loaded into registers, so one chunk's gather
// latency overlaps the previous chunk's arithmetic. Each lane tests its entry
// against the warp's rectangle of pixel centres (the reference's per-simdgroup
// cull, rasterize.metal:13-38, done as the largest exponent over the rectangle
// against -ln(255 op) with a margin); the warp then evaluates only the live
// entries (a ballot mask).
//
// Forward, front to back: alpha = min(0.999, op exp(power)), skip power > 0 or
// alpha < 1/255, stop a pixel once T < 1e-4 and record the stop INDEX. Live
// entries are taken two at a time: both exponentials are evaluated before
// either blend, so their latencies overlap, and the blends stay in list order
// and branch per pixel, so a warp skips the blend when no pixel takes it.
// Every MG_RASTER_SEGMENT entries of a tile's list the forward stores each
// pixel's running state (T, accumulated rgb, accumulated alpha): a checkpoint.
//
// Backward, back to front: work items are (warp block, segment) pairs, a
// segment being MG_RASTER_SEGMENT consecutive entries of the block's walk,
// which the forward appends as it finishes each block. A backward warp block
// is two vertically adjacent forward blocks when the tile side is a multiple
// of 8 (each lane holds two pixels, so the record loads, the cull and the
// gradient reduction are shared by both); the last of the pair to finish in
// the forward appends the pair's segments. A segment starts from
// the checkpoint at its upper end (T
// there; the colour behind it is the final colour minus the checkpointed one),
// so a long list is split over many warps instead of forming the kernel's
// tail. The colour and alpha behind an entry enter its gradient only through
// their dot product with the pixel's output gradient, so a pixel carries one
// running sum for them. Per live entry a lane sums, over its pixels, the raw
// moments of g = dL/dalpha * gauss (g dx, g dy, g, g dx^2, g dx dy, g dy^2)
// and the colour weights; the conic and opacity factors every pixel shares
// are applied once per entry, after the sum over lanes. An entry to which at
// most 24 of the warp's lanes contribute is added as per-lane 16-byte vector
// atomics; otherwise the warp reduces its lanes' sums with a 10-slot
// butterfly reduce-scatter (12 shuffles) and three lanes add the 48-byte
// gradient record with three vector atomics (the crossover measured on B200).
#include <mutex>
#include <unordered_map>

#include "kernels.cuh"

namespace mg {

namespace {

constexpr int kSeg = MG_RASTER_SEGMENT;
static_assert(kSeg % 32 == 0 && (kSeg & (kSeg - 1)) == 0,
              "segments are a power of two number of whole chunks");
#ifndef MG_RASTER_WARPS
#define MG_RASTER_WARPS 4
#endif
constexpr int kRasterWarps = MG_RASTER_WARPS;  // warps per CTA of the persistent kernels

inline size_t align256(size_t x) { return (x + 255) & ~(size_t)255; }

// ---------------------------------------------------------------- records

__global__ void pack_splats_kernel(const float2* __restrict__ uv,
                                   const float* __restrict__ conic,
                                   const float* __restrict__ opacity,
                                   const float* __restrict__ color, int64_t n,
                                   float4* __restrict__ out, float4* __restrict__ g2d_zero) {
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n) return;
    if (g2d_zero != nullptr) {  // the view's gradient records, before its backward
        const float4 z = make_float4(0.f, 0.f, 0.f, 0.f);
        g2d_zero[3 * i] = z;
        g2d_zero[3 * i + 1] = z;
        g2d_zero[3 * i + 2] = z;
    }
    const float2 m = uv[i];
    const float ca = conic[3 * i], cb = conic[3 * i + 1], cc = conic[3 * i + 2];
    const float op = opacity[i];
    const float oa = 255.0f * op;
    // live iff max exponent over a rectangle > pthr; -ln(255 op) is the exact
    // bound (alpha >= 1/255), widened by a relative and an absolute margin
    const float pthr = oa > 1.0f ? -(logf(oa) * 1.0001f + 5e-5f) : __int_as_float(0x7f800000);
    out[3 * i] = make_float4(m.x, m.y, -0.5f * ca, -cb);
    out[3 * i + 1] = make_float4(-0.5f * cc, op, color[3 * i], color[3 * i + 1]);
    out[3 * i + 2] = make_float4(color[3 * i + 2], cb / fmaxf(ca, 1e-12f),
                                 cb / fmaxf(cc, 1e-12f), pthr);
}

// Exponent of one (pixel, splat) pair with explicitly rounded operations, so
// the forward and the backward take bit-identical blend decisions.
__device__ __forceinline__ float pair_power(float dx, float dy, float A, float B, float C) {
    return __fmaf_rn(A, __fmul_rn(dx, dx),
                     __fmaf_rn(B, __fmul_rn(dx, dy), __fmul_rn(C, __fmul_rn(dy, dy))));
}

// Is the record live for a warp whose pixel centres span [x0,x1] x [y0,y1]?
// The largest exponent over the rectangle (binning.metal:25-44 for the
// quadratic form's minimum): at the centre when it lies inside, else on an
// edge at the clamped stationary point. q0 = {u, v, A, B}, C, q2 = {b, kx,
// ky, pthr} with kx = cb/ca, ky = cb/cc.
__device__ __forceinline__ bool rect_live(const float4 q0, const float C, const float4 q2,
                                          float x0, float x1, float y0, float y1) {
    const float u = q0.x, v = q0.y, A = q0.z, B = q0.w;
    const float kx = q2.y, ky = q2.z, pthr = q2.w;
    if (!(pthr < 0.0f)) return false;  // opacity at most 1/255
    if (u >= x0 && u <= x1 && v >= y0 && v <= y1) return true;
    float best = -3.0e38f;
#pragma unroll
    for (int e = 0; e < 2; ++e) {
        const float ey = (e == 0 ? y0 : y1) - v;
        const float ex = fminf(fmaxf(u - kx * ey, x0), x1) - u;
        best = fmaxf(best, A * ex * ex + B * ex * ey + C * ey * ey);
    }
#pragma unroll
    for (int e = 0; e < 2; ++e) {
        const float ex = (e == 0 ? x0 : x1) - u;
        const float ey = fminf(fmaxf(v - ky * ex, y0), y1) - v;
        best = fmaxf(best, A * ex * ex + B * ex * ey + C * ey * ey);
    }
    return best > pthr;
}

// Bounding rectangle of the warp's in-image pixel centres, in every lane.
template <int PX>
__device__ __forceinline__ void warp_rect(const bool (&inimg)[PX], const float (&fx)[PX],
                                          const float (&fy)[PX], float& x0, float& x1,
                                          float& y0, float& y1) {
    x0 = 3.0e38f; x1 = -3.0e38f; y0 = 3.0e38f; y1 = -3.0e38f;
#pragma unroll
    for (int p = 0; p < PX; ++p) {
        if (!inimg[p]) continue;
        x0 = fminf(x0, fx[p]); x1 = fmaxf(x1, fx[p]);
        y0 = fminf(y0, fy[p]); y1 = fmaxf(y1, fy[p]);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        x0 = fminf(x0, __shfl_xor_sync(0xffffffffu, x0, o));
        x1 = fmaxf(x1, __shfl_xor_sync(0xffffffffu, x1, o));
        y0 = fminf(y0, __shfl_xor_sync(0xffffffffu, y0, o));
        y1 = fmaxf(y1, __shfl_xor_sync(0xffffffffu, y1, o));
    }
}

__device__ __forceinline__ void warp_rect(bool inimg, float fx, float fy, float& x0, float& x1,
                                          float& y0, float& y1) {
    const bool in[1] = {inimg};
    const float x[1] = {fx}, y[1] = {fy};
    warp_rect<1>(in, x, y, x0, x1, y0, y1);
}

// ---------------------------------------------------------------- staging

__device__ __forceinline__ void cp_async16(void* smem, const void* gmem) {
    const uint32_t s = (uint32_t)__cvta_generic_to_shared(smem);
    asm volatile("cp.async.ca.shared.global [%0], [%1], 16;\n" ::"r"(s), "l"(gmem) : "memory");
}
__device__ __forceinline__ void cp_async_commit() {
    asm volatile("cp.async.commit_group;\n" ::: "memory");
}
template <int N>
__device__ __forceinline__ void cp_async_wait() {
    asm volatile("cp.async.wait_group %0;\n" ::"n"(N) : "memory");
}

// Chunks in flight per warp: the records of chunk i + stages - 1 are copied
// while chunk i is processed. The forward finds its records in L2 (packed
// just before), so two stages suffice there; the backward starts a new walk
// every segment and gains from a third.
#ifndef MG_FWD_STAGES
#define MG_FWD_STAGES 2
#endif
#ifndef MG_BWD_STAGES
#define MG_BWD_STAGES 3
#endif
constexpr int kFwdStages = MG_FWD_STAGES;
#ifndef MG_BWD_DIRECT_LANES
#define MG_BWD_DIRECT_LANES 24
#endif
// Up to this many lanes (of 32) with a contributing pixel, a live entry's
// gradient goes out as per-lane vector atomics instead of through the warp
// reduction (8 / 12 / 16 / 20 / 24 / 32 measured on the bench: 24 best; 32,
// atomics only, is 30% slower).
constexpr int kBwdDirectLanes = MG_BWD_DIRECT_LANES;
constexpr int kBwdStages = MG_BWD_STAGES;

// A warp's ring of chunk buffers: q[buffer][word][entry], so a lane's three
// copies land in consecutive 16-byte words of three rows and an entry is read
// back as three broadcast loads.
template <int kStages>
struct WarpStage {
    float4 q[kStages][3][32];
    int32_t id[kStages][32];
    __device__ __forceinline__ void fetch(int buf, int lane, const float4* splats, int gid,
                                          bool keep_id) {
        const float4* src = splats + 3 * (int64_t)gid;
        cp_async16(&q[buf][0][lane], src);
        cp_async16(&q[buf][1][lane], src + 1);
        cp_async16(&q[buf][2][lane], src + 2);
        if (keep_id) id[buf][lane] = gid;
    }
};

// Pixels of a tile in the forward's warp blocks: 8x4 when the side is a
// multiple of 8, otherwise row-major with the last block padded.
template <int TILE>
struct Blocks {
    static constexpr int kPix = TILE * TILE;
    static constexpr int kCount = (kPix + 31) / 32;
    static constexpr int kPixPad = kCount * 32;  // pixel slots of a checkpoint
    __device__ __forceinline__ static void pixel(int wb, int lane, int& lx, int& ly) {
        if (TILE % 8 == 0) {
            const int bx = TILE / 8;
            lx = (wb % bx) * 8 + (lane & 7);
            ly = (wb / bx) * 4 + (lane >> 3);
        } else {
            const int t = wb * 32 + lane;
            lx = t < kPix ? t % TILE : TILE;  // padding lanes sit outside the tile
            ly = t < kPix ? t / TILE : TILE;
        }
    }
};

// Forward blocks per backward warp block (1 or 2) when the tile side is a
// multiple of 8.
#ifndef MG_RASTER_PX
#define MG_RASTER_PX 2
#endif

// The backward's warp blocks: kPx vertically adjacent forward blocks (8 x 4
// kPx pixels when the side is a multiple of 8), lane l holding the pixel of
// lane l in each. A list entry's record, its cull vote and the warp reduction
// of its gradient are then shared by kPx pixels per lane. (The forward keeps
// 32-pixel blocks: its heaviest block's walk is a serial chain per warp, and
// two pixels per lane would double it.)
// Pixels per lane of the backward for a tile side: MG_RASTER_PX when the
// side is a multiple of 8 (at most the tile's forward blocks), else 1.
__host__ __device__ constexpr int bwd_px_for(int tile) {
    return tile % 8 != 0 ? 1
                         : ((tile * tile + 31) / 32 >= MG_RASTER_PX ? MG_RASTER_PX
                                                                   : (tile * tile + 31) / 32);
}

template <int TILE>
struct BwdBlocks {
    using F = Blocks<TILE>;
    static constexpr int kPx = bwd_px_for(TILE);
    static constexpr int kCount = F::kCount / kPx;
    static_assert(F::kCount % kPx == 0, "whole forward blocks per backward block");
    // forward block holding pixel p of backward block b
    __device__ __forceinline__ static int fwd_block(int b, int p) {
        if (kPx == 1) return b;
        const int bx = TILE / 8;
        return ((b / bx) * kPx + p) * bx + b % bx;
    }
    // backward block holding forward block wb
    __device__ __forceinline__ static int of_fwd(int wb) {
        if (kPx == 1) return wb;
        const int bx = TILE / 8;
        return ((wb / bx) / kPx) * bx + wb % bx;
    }
};

// Checkpoint slot of boundary j (1-based: the state before entry start + j *
// kSeg) of the tile whose list starts at `start`. Slots of consecutive tiles
// never overlap and stay below m / kSeg + n_tiles.
__device__ __forceinline__ int64_t ckpt_slot(int start, int tile_id, int j) {
    return (int64_t)(start / kSeg) + tile_id + j - 1;
}

__device__ __forceinline__ int pull_item(int32_t* counter, int lane) {
    int item = 0;
    if (lane == 0) item = atomicAdd(counter, 1);
    return __shfl_sync(0xffffffffu, item, 0);
}

// ---------------------------------------------------------------- forward

template <int TILE>
__global__ void __launch_bounds__(kRasterWarps * 32)
raster_forward_kernel(const float4* __restrict__ splats, const int32_t* __restrict__ ids,
                      const int32_t* __restrict__ offsets, int W, int H, int tiles_x,
                      int n_tiles, int has_bg, float bg_r, float bg_g, float bg_b,
                      float* __restrict__ out_rgb, float* __restrict__ out_alpha,
                      float* __restrict__ out_T, int32_t* __restrict__ out_stop,
                      const int32_t* __restrict__ order, int32_t* __restrict__ counter,
                      int32_t* __restrict__ block_work, int32_t* __restrict__ tile_work,
                      float* __restrict__ ckpt, int2* __restrict__ items,
                      int32_t* __restrict__ pair_done, int m_cap, int32_t* __restrict__ err) {
    using G = Blocks<TILE>;
    using B = BwdBlocks<TILE>;
    constexpr int kStages = kFwdStages;
    __shared__ WarpStage<kStages> s_stage[kRasterWarps];
    const int lane = threadIdx.x & 31;
    WarpStage<kStages>& st = s_stage[threadIdx.x >> 5];
    const int n_items = n_tiles * G::kCount;

    for (int item = pull_item(counter, lane); item < n_items; item = pull_item(counter, lane)) {
        const int tile_id = order[item / G::kCount];
        const int wb = item % G::kCount;
        int lx, ly;
        G::pixel(wb, lane, lx, ly);
        const int px = (tile_id % tiles_x) * TILE + lx, py = (tile_id / tiles_x) * TILE + ly;
        const bool inimg = lx < TILE && ly < TILE && px < W && py < H;
        const int start = offsets[tile_id];
        int end = offsets[tile_id + 1];
        if (end > m_cap) {  // lists beyond the sized pair count: report, render nothing
            if (lane == 0) record_device_error(err, DEV_ERR_INDEX);
            end = start;
        }
        const float fx = (float)px + 0.5f, fy = (float)py + 0.5f;

        float T = 1.0f, ar = 0.0f, ag = 0.0f, ab = 0.0f, aa = 0.0f;
        int stop = start;
        bool done = !inimg;
        if (start < end && !__all_sync(0xffffffffu, done)) {
            float rx0, rx1, ry0, ry1;
            warp_rect(inimg, fx, fy, rx0, rx1, ry0, ry1);
            float* ck = ckpt ? ckpt + wb * 32 + lane : nullptr;  // null: forward only
            const int n_chunks = (end - start + 31) >> 5;
            // ids of the first kStages chunks (all loads in flight together),
            // then the copies of the first kStages - 1
            int gid[kStages];
#pragma unroll
            for (int c = 0; c < kStages; ++c) {
                const int j = start + 32 * c + lane;
                gid[c] = j < end ? ids[j] : -1;
            }
#pragma unroll
            for (int c = 0; c < kStages - 1; ++c) {
                if (gid[c] >= 0) st.fetch(c, lane, splats, gid[c], false);
                cp_async_commit();
            }
            int gid_next = gid[kStages - 1];
            int buf = 0, ibuf = kStages - 1;  // buffers of chunk i and chunk i + kStages - 1
            for (int ci = 0;; ++ci) {
                const int base = start + 32 * ci;
                // ibuf held chunk ci - 1, released by that chunk's last vote
                if (gid_next >= 0) st.fetch(ibuf, lane, splats, gid_next, false);
                cp_async_commit();
                {
                    const int j = base + 32 * kStages + lane;
                    gid_next = j < end ? ids[j] : -1;
                }
                if (ck && ci != 0 && ((base - start) & (kSeg - 1)) == 0) {
                    float* c = ck + ckpt_slot(start, tile_id, (base - start) / kSeg) * 5 *
                                        G::kPixPad;
                    c[0] = T;
                    c[G::kPixPad] = ar;
                    c[2 * G::kPixPad] = ag;
                    c[3 * G::kPixPad] = ab;
                    c[4 * G::kPixPad] = aa;
                }
                cp_async_wait<kStages - 1>();
                __syncwarp();
                const bool lv = base + lane < end &&
                                rect_live(st.q[buf][0][lane], st.q[buf][1][lane].x,
                                          st.q[buf][2][lane], rx0, rx1, ry0, ry1);
                uint32_t live = __ballot_sync(0xffffffffu, lv);
                int round = 0;
                while (live) {
                    const int k1 = __ffs(live) - 1;
                    live &= live - 1;
                    const bool two = live != 0u;
                    const int k2 = two ? __ffs(live) - 1 : k1;
                    live &= live - 1;
                    const float4 a1 = st.q[buf][0][k1], b1 = st.q[buf][1][k1];
                    const float c1 = st.q[buf][2][k1].x;
                    const float4 a2 = st.q[buf][0][k2], b2 = st.q[buf][1][k2];
                    const float c2 = st.q[buf][2][k2].x;
                    const float p1 = pair_power(fx - a1.x, fy - a1.y, a1.z, a1.w, b1.x);
                    const float p2 = pair_power(fx - a2.x, fy - a2.y, a2.z, a2.w, b2.x);
                    const float al1 = fminf(0.999f, b1.y * __expf(p1));
                    const float al2 = fminf(0.999f, b2.y * __expf(p2));
                    if (!done && p1 <= 0.0f && al1 >= 1.0f / 255.0f) {
                        const float w = al1 * T;
                        ar += w * b1.z; ag += w * b1.w; ab += w * c1;
                        aa += w;
                        T *= (1.0f - al1);
                        stop = base + k1 + 1;
                        done = T < 1e-4f;
                    }
                    if (two && !done && p2 <= 0.0f && al2 >= 1.0f / 255.0f) {
                        const float w = al2 * T;
                        ar += w * b2.z; ag += w * b2.w; ab += w * c2;
                        aa += w;
                        T *= (1.0f - al2);
                        stop = base + k2 + 1;
                        done = T < 1e-4f;
                    }
                    // every other round: a round after every pixel stopped
                    // blends nothing, and the vote costs an instruction per
                    // round (launch lists: 348-363 us per view against
                    // 361-363 voting every round, within box-to-box noise)
                    if ((++round & 1) == 0 && __all_sync(0xffffffffu, done)) break;
                }
                const bool all_done = __all_sync(0xffffffffu, done);  // releases buffer buf
                if (all_done || ci + 1 >= n_chunks) break;
                buf = buf + 1 == kStages ? 0 : buf + 1;
                ibuf = ibuf + 1 == kStages ? 0 : ibuf + 1;
            }
            cp_async_wait<0>();
            __syncwarp();
        }
        const int walk = __reduce_max_sync(0xffffffffu, stop) - start;
        // the backward's work items for this block's backward block: one per
        // MG_RASTER_SEGMENT entries of its walk (the longest of its forward
        // blocks), appended by the last of those to finish (in completion
        // order; every item is at most one segment, so their order forms no
        // tail)
        const int bb = B::of_fwd(wb);
        int nseg = 0, ibase = 0;
        if (lane == 0) {
            block_work[tile_id * G::kCount + wb] = walk;
            if (tile_work && walk > 0) atomicMax(&tile_work[tile_id], walk);
            if (items) {
                int w = walk;
                bool last = true;
                if (B::kPx > 1) {
                    __threadfence();  // this walk is visible before the count
                    last = atomicAdd(&pair_done[tile_id * B::kCount + bb], 1) == B::kPx - 1;
                    if (last) {
                        __threadfence();
#pragma unroll
                        for (int p = 0; p < B::kPx; ++p)
                            w = max(w, *reinterpret_cast<volatile int32_t*>(
                                           &block_work[tile_id * G::kCount + B::fwd_block(bb, p)]));
                    }
                }
                if (last) {
                    nseg = (w + kSeg - 1) / kSeg;
                    if (nseg > 0) ibase = atomicAdd(&counter[2], nseg);
                }
            }
        }
        nseg = __shfl_sync(0xffffffffu, nseg, 0);
        ibase = __shfl_sync(0xffffffffu, ibase, 0);
        for (int sgi = lane; sgi < nseg; sgi += 32)
            items[ibase + sgi] = make_int2(tile_id * B::kCount + bb, sgi);
        if (inimg) {
            const int64_t o = (int64_t)py * W + px;
            if (has_bg) {
                const float k = fmaxf(1.0f - aa, 0.0f);
                ar = ar + k * bg_r; ag = ag + k * bg_g; ab = ab + k * bg_b;
            }
            out_rgb[3 * o + 0] = ar;
            out_rgb[3 * o + 1] = ag;
            out_rgb[3 * o + 2] = ab;
            out_alpha[o] = aa;
            if (out_T) {  // the backward's inputs; absent in forward-only renders
                out_T[o] = T;
                out_stop[o] = stop;
            }
        }
    }
}

// ---------------------------------------------------------------- backward

// 10-slot butterfly reduce-scatter across the warp in 12 shuffles (5 + 3 + 2
// + 1 exchanges, halving the slots a lane holds each round, padded where the
// count is odd, then one plain add). On return lanes 2p and 2p+1 hold the
// warp sum of slot s for (p, s) = (0,0) (1,1) (2,2) (4,3) (5,4) (8,5) (9,6)
// (10,7) (12,8) (13,9); the other pairs hold padding zeros.
__device__ __forceinline__ float reduce_scatter10(const float (&v)[10], int lane) {
    const bool h16 = lane & 16, h8 = lane & 8, h4 = lane & 4, h2 = lane & 2;
    float u[5];
#pragma unroll
    for (int k = 0; k < 5; ++k) {
        const float send = h16 ? v[k] : v[k + 5];
        const float keep = h16 ? v[k + 5] : v[k];
        u[k] = keep + __shfl_xor_sync(0xffffffffu, send, 16);
    }
    float w[3];
#pragma unroll
    for (int k = 0; k < 2; ++k) {
        const float send = h8 ? u[k] : u[k + 3];
        const float keep = h8 ? u[k + 3] : u[k];
        w[k] = keep + __shfl_xor_sync(0xffffffffu, send, 8);
    }
    w[2] = (h8 ? 0.0f : u[2]) + __shfl_xor_sync(0xffffffffu, h8 ? u[2] : 0.0f, 8);
    float x0, x1;
    {
        const float send = h4 ? w[0] : w[2];
        const float keep = h4 ? w[2] : w[0];
        x0 = keep + __shfl_xor_sync(0xffffffffu, send, 4);
    }
    x1 = (h4 ? 0.0f : w[1]) + __shfl_xor_sync(0xffffffffu, h4 ? w[1] : 0.0f, 4);
    const float send = h2 ? x0 : x1;
    const float keep = h2 ? x1 : x0;
    const float y = keep + __shfl_xor_sync(0xffffffffu, send, 2);
    return y + __shfl_xor_sync(0xffffffffu, y, 1);
}

// Source lanes from which lanes 0, 1, 2 gather the float4 words of the
// gradient record after reduce_scatter10 (slot s -> lane of its pair; lane 6
// holds a padding zero).
__device__ __forceinline__ void record_gather_lanes(int lane, int& s0, int& s1, int& s2,
                                                    int& s3) {
    s0 = lane == 0 ? 0 : lane == 1 ? 10 : lane == 2 ? 20 : lane;
    s1 = lane == 0 ? 2 : lane == 1 ? 16 : lane == 2 ? 24 : lane;
    s2 = lane == 0 ? 4 : lane == 1 ? 18 : lane == 2 ? 26 : lane;
    s3 = lane == 0 ? 8 : lane <= 2 ? 6 : lane;
}

// kSegmented: items are (block, segment) pairs and segments start from the
// forward's checkpoints; otherwise one item per block walks the whole list
// from the pixels' stop indices (no forward state needed). With kPx pixels
// per lane, a lane adds its pixels' contributions to an entry before the
// warp reduction (or its own atomics), so the reduction and the record loads
// are shared by kPx pixels.
template <int TILE, bool kSegmented>
__global__ void __launch_bounds__(kRasterWarps * 32)
raster_backward_kernel(const float4* __restrict__ splats, const int32_t* __restrict__ ids,
                       const int32_t* __restrict__ offsets, const float* __restrict__ out_rgb,
                       const float* __restrict__ out_alpha, const float* __restrict__ final_T,
                       const int32_t* __restrict__ stop_idx,
                       const float* __restrict__ grad_rgb,
                       const float* __restrict__ grad_alpha, int W, int H, int tiles_x,
                       int has_bg, float bg_r, float bg_g, float bg_b, int want_absgrad,
                       float* __restrict__ grad2d, const int2* __restrict__ items,
                       int32_t* __restrict__ counters, const float* __restrict__ ckpt,
                       int m_cap, int32_t* __restrict__ err) {
    using G = Blocks<TILE>;
    using B = BwdBlocks<TILE>;
    constexpr int PX = B::kPx;
    constexpr int kStages = kBwdStages;
    __shared__ WarpStage<kStages> s_stage[kRasterWarps];
    const int lane = threadIdx.x & 31;
    WarpStage<kStages>& st = s_stage[threadIdx.x >> 5];
    const int n_items = counters[2];
    int g0, g1, g2, g3;
    record_gather_lanes(lane, g0, g1, g2, g3);

    for (int item = pull_item(counters + 1, lane); item < n_items;
         item = pull_item(counters + 1, lane)) {
        const int2 it = items[item];
        const int tile_id = it.x / B::kCount, wb = it.x % B::kCount, seg = it.y;
        const int start = offsets[tile_id], end = offsets[tile_id + 1];
        if (end > m_cap) {
            if (lane == 0) record_device_error(err, DEV_ERR_INDEX);
            continue;
        }
        const int seg_lo = start + seg * kSeg;
        const int seg_top = kSegmented ? min(seg_lo + kSeg, end) : end;
        const int tx0 = (tile_id % tiles_x) * TILE, ty0 = (tile_id / tiles_x) * TILE;

        // S = <d L / d (rgb, alpha), colour and alpha blended behind the
        // current entry>: one running dot product instead of four suffix sums
        bool inimg[PX];
        float fx[PX], fy[PX], T[PX], S[PX], gr[PX], gg[PX], gb[PX], ga[PX];
        int my_stop[PX];
        int hi = seg_lo;
#pragma unroll
        for (int p = 0; p < PX; ++p) {
            const int fb = B::fwd_block(wb, p);
            int lx, ly;
            G::pixel(fb, lane, lx, ly);
            const int px = tx0 + lx, py = ty0 + ly;
            inimg[p] = lx < TILE && ly < TILE && px < W && py < H;
            fx[p] = (float)px + 0.5f;
            fy[p] = (float)py + 0.5f;
            T[p] = 1.0f; S[p] = 0.0f;
            gr[p] = gg[p] = gb[p] = ga[p] = 0.0f;
            my_stop[p] = start;
            if (!inimg[p]) continue;
            const int64_t o = (int64_t)py * W + px;
            my_stop[p] = stop_idx[o];
            gr[p] = grad_rgb[3 * o]; gg[p] = grad_rgb[3 * o + 1]; gb[p] = grad_rgb[3 * o + 2];
            ga[p] = grad_alpha ? grad_alpha[o] : 0.0f;
            const float a_fin = (has_bg || kSegmented) ? out_alpha[o] : 0.0f;
            const float kbg = fmaxf(1.0f - a_fin, 0.0f);
            // rgb_out = rgb + max(1 - alpha, 0) * bg  =>  d alpha -= <d rgb, bg>
            if (has_bg && 1.0f - a_fin >= 0.0f)
                ga[p] -= gr[p] * bg_r + gg[p] * bg_g + gb[p] * bg_b;
            if (kSegmented && my_stop[p] > seg_lo + kSeg) {
                const float* c = ckpt + ckpt_slot(start, tile_id, seg + 1) * 5 * G::kPixPad +
                                 fb * 32 + lane;
                float cr = out_rgb[3 * o], cg = out_rgb[3 * o + 1], cbl = out_rgb[3 * o + 2];
                if (has_bg) { cr -= kbg * bg_r; cg -= kbg * bg_g; cbl -= kbg * bg_b; }
                T[p] = c[0];
                S[p] = gr[p] * (cr - c[G::kPixPad]) + gg[p] * (cg - c[2 * G::kPixPad]) +
                       gb[p] * (cbl - c[3 * G::kPixPad]) + ga[p] * (a_fin - c[4 * G::kPixPad]);
            } else {
                T[p] = final_T[o];
            }
            hi = max(hi, min(my_stop[p], seg_top));
        }
        const int warp_hi = __reduce_max_sync(0xffffffffu, hi);
        if (warp_hi <= seg_lo) continue;
        float rx0, rx1, ry0, ry1;
        warp_rect<PX>(inimg, fx, fy, rx0, rx1, ry0, ry1);

        // chunks are aligned to the list start (seg_lo is a chunk boundary)
        // and walked from the top one down: chunk c starts at top - 32 c
        const int top = start + ((warp_hi - 1 - start) >> 5) * 32;
        const int n_chunks = ((top - seg_lo) >> 5) + 1;
        int gid[kStages];
#pragma unroll
        for (int c = 0; c < kStages; ++c) {
            const int j = top - 32 * c + lane;
            gid[c] = (c < n_chunks && j < warp_hi) ? ids[j] : -1;
        }
#pragma unroll
        for (int c = 0; c < kStages - 1; ++c) {
            if (gid[c] >= 0) st.fetch(c, lane, splats, gid[c], true);
            cp_async_commit();
        }
        int gid_next = gid[kStages - 1];
        int buf = 0, ibuf = kStages - 1;
        for (int ci = 0;; ++ci) {
            const int base = top - 32 * ci;
            if (gid_next >= 0) st.fetch(ibuf, lane, splats, gid_next, true);
            cp_async_commit();
            gid_next = ci + kStages < n_chunks ? ids[top - 32 * (ci + kStages) + lane] : -1;
            cp_async_wait<kStages - 1>();
            __syncwarp();
            const bool lv = base + lane < warp_hi &&
                            rect_live(st.q[buf][0][lane], st.q[buf][1][lane].x,
                                      st.q[buf][2][lane], rx0, rx1, ry0, ry1);
            uint32_t live = __ballot_sync(0xffffffffu, lv);
            while (live) {
                const int k = 31 - __clz(live);  // back to front
                live &= ~(1u << k);
                const float4 a = st.q[buf][0][k], b4 = st.q[buf][1][k];
                const float cbk = st.q[buf][2][k].x;
                // a = {u, v, A, B}, b4 = {C, op, r, g}, cbk = b
                float dx[PX], dy[PX], gauss[PX], alpha[PX];
                bool active[PX], unclamped[PX];
                bool any = false;
#pragma unroll
                for (int p = 0; p < PX; ++p) {
                    dx[p] = fx[p] - a.x;
                    dy[p] = fy[p] - a.y;
                    const float power = pair_power(dx[p], dy[p], a.z, a.w, b4.x);
                    gauss[p] = __expf(fminf(power, 0.0f));
                    const float alpha_raw = b4.y * gauss[p];
                    alpha[p] = fminf(0.999f, alpha_raw);
                    // the 0.999 clamp cuts the gradient to opacity and position
                    unclamped[p] = alpha_raw <= 0.999f;
                    active[p] = inimg[p] && (base + k < my_stop[p]) && (power <= 0.0f) &&
                                (alpha[p] >= 1.0f / 255.0f);
                    any = any || active[p];
                }
                const uint32_t lanes = __ballot_sync(0xffffffffu, any);
                if (lanes == 0u) continue;
                // Per lane, the raw moments of g = dL/dalpha * gauss over its
                // pixels (g dx, g dy, g, g dx^2, g dx dy, g dy^2) and the colour
                // weights; the conic and opacity factors common to every pixel
                // are applied once per entry after the reduction:
                //   d u = -op (2A Sx + B Sy),  d v = -op (B Sx + 2C Sy),
                //   d op = Sg,  d conic = -op (Sxx / 2, Sxy, Syy / 2),
                // since d power / d u = -(2A dx + B dy) and A = -ca/2, B = -cb,
                // C = -cc/2.
                float v[10];
#pragma unroll
                for (int i = 0; i < 10; ++i) v[i] = 0.0f;
#pragma unroll
                for (int p = 0; p < PX; ++p) {
                    const float om = fmaxf(1.0f - alpha[p], 1e-8f);
                    // segments bound the recovery chain to kSeg divisions
                    const float inv = kSegmented ? __fdividef(1.0f, om) : __frcp_rn(om);
                    const float Tn = T[p] * inv;
                    const float q = gr[p] * b4.z + gg[p] * b4.w + gb[p] * cbk + ga[p];
                    const float dL_dalpha = Tn * q - inv * S[p];
                    const float w = active[p] ? alpha[p] * Tn : 0.0f;
                    T[p] = active[p] ? Tn : T[p];
                    S[p] += w * q;
                    const float g = (active[p] && unclamped[p]) ? dL_dalpha * gauss[p] : 0.0f;
                    const float gx = g * dx[p], gy = g * dy[p];
                    v[0] += gx;
                    v[1] += gy;
                    v[2] += g;
                    if (want_absgrad) {  // per-pixel |d uv|, before the factors
                        const float ux = -(2.0f * a.z * dx[p] + a.w * dy[p]);
                        const float uy = -(a.w * dx[p] + 2.0f * b4.x * dy[p]);
                        v[3] += b4.y * fabsf(g) * sqrtf(ux * ux + uy * uy);
                    }
                    v[4] = fmaf(gx, dx[p], v[4]);
                    v[5] = fmaf(gx, dy[p], v[5]);
                    v[6] = fmaf(gy, dy[p], v[6]);
                    v[7] = fmaf(w, gr[p], v[7]);
                    v[8] = fmaf(w, gg[p], v[8]);
                    v[9] = fmaf(w, gb[p], v[9]);
                }
                float4* dst =
                    reinterpret_cast<float4*>(grad2d + (int64_t)st.id[buf][k] * MG_G2D_STRIDE);
                const float op = b4.y;
                if (__popc(lanes) <= kBwdDirectLanes) {
                    // few contributing lanes: each adds its own sums (the warp
                    // reduction costs more than a few sets of atomics)
                    if (any) {
                        atomicAdd(dst, make_float4(-op * (2.0f * a.z * v[0] + a.w * v[1]),
                                                   -op * (a.w * v[0] + 2.0f * b4.x * v[1]),
                                                   v[2], v[3]));
                        if (v[4] != 0.f || v[5] != 0.f || v[6] != 0.f)
                            atomicAdd(dst + 1, make_float4(-0.5f * op * v[4], -op * v[5],
                                                           -0.5f * op * v[6], 0.f));
                        atomicAdd(dst + 2, make_float4(v[7], v[8], v[9], 0.f));
                    }
                    continue;
                }
                const float r = reduce_scatter10(v, lane);
                float r0 = __shfl_sync(0xffffffffu, r, g0);
                float r1 = __shfl_sync(0xffffffffu, r, g1);
                float r2 = __shfl_sync(0xffffffffu, r, g2);
                const float r3 = __shfl_sync(0xffffffffu, r, g3);
                // lane 0 holds (Sx, Sy, Sg, |uv|), lane 1 (Sxx, Sxy, Syy, 0),
                // lane 2 the colour sums
                if (lane == 0) {
                    const float sx = r0, sy = r1;
                    r0 = -op * (2.0f * a.z * sx + a.w * sy);
                    r1 = -op * (a.w * sx + 2.0f * b4.x * sy);
                } else if (lane == 1) {
                    r0 = -0.5f * op * r0;
                    r1 = -op * r1;
                    r2 = -0.5f * op * r2;
                }
                if (lane < 3 && (r0 != 0.f || r1 != 0.f || r2 != 0.f || r3 != 0.f))
                    atomicAdd(dst + lane, make_float4(r0, r1, r2, r3));
            }
            __syncwarp();  // buffer buf is refilled kStages - 1 chunks on
            if (ci + 1 >= n_chunks) break;
            buf = buf + 1 == kStages ? 0 : buf + 1;
            ibuf = ibuf + 1 == kStages ? 0 : ibuf + 1;
        }
        cp_async_wait<0>();
        __syncwarp();
    }
}

// ---------------------------------------------------------------- ordering

// Inclusive prefix sum across the warp.
__device__ __forceinline__ int warp_incl_scan(int x, int lane) {
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const int t = __shfl_up_sync(0xffffffffu, x, o);
        if (lane >= o) x += t;
    }
    return x;
}

// One-CTA counting sort into K classes, class K-1 first. Each thread owns
// the elements tid, tid + 1024, ... and counts them per class in registers;
// per class, every warp scans its lanes' counts and reserves its range with
// one shared-memory atomic, so there is no per-element atomic. Returns, per
// class, this thread's first output position.
template <int K>
__device__ __forceinline__ void class_positions(const int (&cnt)[K], int (&pos)[K], int lane,
                                                int* s_total /* [K], zeroed */) {
    int wbase[K], excl[K];
#pragma unroll
    for (int c = 0; c < K; ++c) {
        const int incl = warp_incl_scan(cnt[c], lane);
        const int wtot = __shfl_sync(0xffffffffu, incl, 31);
        int b = 0;
        if (lane == 31 && wtot > 0) b = atomicAdd(&s_total[c], wtot);
        wbase[c] = __shfl_sync(0xffffffffu, b, 31);
        excl[c] = incl - cnt[c];
    }
    __syncthreads();  // class totals complete
    int run = 0;
#pragma unroll
    for (int c = K - 1; c >= 0; --c) {
        pos[c] = run + wbase[c] + excl[c];
        run += s_total[c];
    }
}

constexpr int kOrderClasses = 8;

// Length class of a tile: floor(log2(len)) - 6 clamped to [0, 7].
__device__ __forceinline__ int length_class(int w) {
    if (w <= 0) return 0;
    return min(kOrderClasses - 1, max(0, (31 - __clz(w)) - 6));
}

// Longest-first tile order by list-length class (order inside a class is
// unspecified). Optionally zeroes a work counter, a per-tile array and the
// per-backward-block completion counters for the kernel that follows.
__global__ void __launch_bounds__(1024)
tile_order_kernel(const int32_t* __restrict__ offsets, const int32_t* __restrict__ work,
                  int n_tiles, int32_t* __restrict__ order, int32_t* __restrict__ zero_word,
                  int32_t* __restrict__ zero_tiles, int32_t* __restrict__ zero_pairs,
                  int n_pairs) {
    __shared__ int s_total[kOrderClasses];
    const int tid = threadIdx.x, lane = tid & 31;
    if (tid < kOrderClasses) s_total[tid] = 0;
    if (tid < 4 && zero_word) zero_word[tid] = 0;  // a kernel's work counters
    __syncthreads();
    int cnt[kOrderClasses], pos[kOrderClasses];
#pragma unroll
    for (int c = 0; c < kOrderClasses; ++c) cnt[c] = 0;
    for (int t = tid; t < n_tiles; t += 1024) {
        const int cls = length_class(work ? work[t] : offsets[t + 1] - offsets[t]);
#pragma unroll
        for (int c = 0; c < kOrderClasses; ++c) cnt[c] += cls == c;
        if (zero_tiles) zero_tiles[t] = 0;
    }
    if (zero_pairs)
        for (int b = tid; b < n_pairs; b += 1024) zero_pairs[b] = 0;
    class_positions<kOrderClasses>(cnt, pos, lane, s_total);
    for (int t = tid; t < n_tiles; t += 1024) {
        const int cls = length_class(work ? work[t] : offsets[t + 1] - offsets[t]);
#pragma unroll
        for (int c = 0; c < kOrderClasses; ++c)
            if (cls == c) order[pos[c]++] = t;
    }
}

// Backward work items when there is no forward state (the segmented
// backward's items are appended by the forward itself): one item per block
// with a non-empty list, longest list first; with seg > 0 each block's walk
// would instead become floor(walk / seg) whole segments plus one partial
// segment, whole segments first. One CTA; also zeroes the backward's pull
// counter and publishes the item count.
__global__ void __launch_bounds__(1024)
backward_items_kernel(const int32_t* __restrict__ offsets,
                      const int32_t* __restrict__ block_work, int n_tiles, int blocks_per_tile,
                      int seg, int2* __restrict__ items, int32_t* __restrict__ counters) {
    __shared__ int s_total[2];
    const int tid = threadIdx.x, lane = tid & 31;
    const int n_blocks = n_tiles * blocks_per_tile;
    if (tid < 2) s_total[tid] = 0;
    __syncthreads();
    int cnt[2] = {0, 0}, pos[2];  // [0] partial segments, [1] whole segments
    for (int b = tid; b < n_blocks; b += 1024) {
        const int t = b / blocks_per_tile;
        const int w = block_work ? block_work[b] : offsets[t + 1] - offsets[t];
        if (w <= 0) continue;
        const int full = seg > 0 ? w / seg : 0;
        cnt[1] += full;
        cnt[0] += w - full * seg > 0;
    }
    class_positions<2>(cnt, pos, lane, s_total);
    if (tid == 0) {
        counters[1] = 0;
        counters[2] = s_total[0] + s_total[1];
    }
    for (int b = tid; b < n_blocks; b += 1024) {
        const int t = b / blocks_per_tile;
        const int w = block_work ? block_work[b] : offsets[t + 1] - offsets[t];
        if (w <= 0) continue;
        const int full = seg > 0 ? w / seg : 0;
        for (int k = 0; k < full; ++k) items[pos[1]++] = make_int2(b, k);
        if (w - full * seg > 0) items[pos[0]++] = make_int2(b, full);
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

// Mip-Splatting opacity compensation (metal_backend.py:367-393): the 2D
// covariance before the 0.3 px blur, recovered from the blurred conic, gives
// op * sqrt(clamp(det_before / det_after, 0, 1)).
// Every operation explicitly rounded, in the order of the reference's
// float32 expression (metal_backend.py:367-393), so the compensated opacity
// -- which decides the 1/255 binning and blending thresholds -- is
// bit-identical to the CPU restatement's.
__device__ __forceinline__ float antialias_factor(float cxx, float cxy, float cyy, float blur) {
    const float det_conic = fmaxf(__fsub_rn(__fmul_rn(cxx, cyy), __fmul_rn(cxy, cxy)), 1e-12f);
    const float det_after = __fdiv_rn(1.0f, det_conic);
    const float a = __fmul_rn(cyy, det_after), b = __fmul_rn(-cxy, det_after);
    const float c = __fmul_rn(cxx, det_after);
    const float det_before = __fsub_rn(__fmul_rn(__fsub_rn(a, blur), __fsub_rn(c, blur)),
                                       __fmul_rn(b, b));
    return __fsqrt_rn(fminf(fmaxf(__fdiv_rn(fmaxf(det_before, 0.0f), det_after), 0.0f), 1.0f));
}

__global__ void antialias_opacity_kernel(const float* __restrict__ conic,
                                         const float* __restrict__ opacity, int64_t n,
                                         float blur, float* __restrict__ out) {
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n) return;
    out[i] = opacity[i] * antialias_factor(conic[3 * i], conic[3 * i + 1], conic[3 * i + 2], blur);
}

// The same for a batch of views (blockIdx.y): view v's conics and outputs at
// rows v * view_stride, the opacities shared.
__global__ void antialias_opacity_views_kernel(const float* __restrict__ conic,
                                               const float* __restrict__ opacity, int64_t n,
                                               int64_t view_stride, float blur,
                                               float* __restrict__ out) {
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n) return;
    const int64_t o = (int64_t)blockIdx.y * view_stride + i;
    out[o] = opacity[i] * antialias_factor(conic[3 * o], conic[3 * o + 1], conic[3 * o + 2], blur);
}

// Adjoint of antialias_opacity_kernel. With beta the blur, the ratio
// det_before / det_after equals 1 - beta (cxx + cyy) + beta^2 (cxx cyy - cxy^2)
// (the blurred covariance is the conic's inverse), so with
// k = sqrt(clamp(ratio, 0, 1)): d op = g k and, where 0 < ratio < 1,
// d conic = g op / (2 k) * d ratio / d conic.
// d out -> (d conic, d opacity) of one Gaussian (conic c, opacity op).
struct AntialiasAdjoint {
    float d_op, dxx, dxy, dyy;
};
__device__ __forceinline__ AntialiasAdjoint antialias_adjoint(float cxx, float cxy, float cyy,
                                                              float op, float g, float blur) {
    const float det_after = 1.0f / fmaxf(cxx * cyy - cxy * cxy, 1e-12f);
    const float a = cyy * det_after, b = -cxy * det_after, c = cxx * det_after;
    const float ratio = ((a - blur) * (c - blur) - b * b) / det_after;
    const float k = sqrtf(fminf(fmaxf(ratio, 0.0f), 1.0f));
    AntialiasAdjoint r{g * k, 0.0f, 0.0f, 0.0f};
    if (ratio > 0.0f && ratio < 1.0f) {
        const float h = g * op / (2.0f * k);
        const float b2 = blur * blur;
        r.dxx = h * (b2 * cyy - blur);
        r.dyy = h * (b2 * cxx - blur);
        r.dxy = h * (-2.0f * b2 * cxy);
    }
    return r;
}

__global__ void antialias_opacity_backward_kernel(const float* __restrict__ conic,
                                                  const float* __restrict__ opacity,
                                                  const float* __restrict__ grad_out, int64_t n,
                                                  float blur, float* __restrict__ d_conic,
                                                  float* __restrict__ d_opacity) {
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n) return;
    const AntialiasAdjoint r = antialias_adjoint(conic[3 * i], conic[3 * i + 1],
                                                 conic[3 * i + 2], opacity[i], grad_out[i], blur);
    d_opacity[i] = r.d_op;
    d_conic[3 * i] = r.dxx;
    d_conic[3 * i + 1] = r.dxy;
    d_conic[3 * i + 2] = r.dyy;
}

// The adjoint in place on a batch of views' gradient records (MG_G2D_*,
// view v's conics and records at rows v * view_stride): the record's d
// opacity, taken against the compensated opacity, becomes the one against
// the opacity before compensation, and the compensation's conic term is
// added to its d conic.
__global__ void antialias_grad2d_views_kernel(const float* __restrict__ conic,
                                              const float* __restrict__ opacity, int64_t n,
                                              int64_t view_stride, float blur,
                                              float* __restrict__ grad2d) {
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n) return;
    const int64_t o = (int64_t)blockIdx.y * view_stride + i;
    float* rec = grad2d + o * MG_G2D_STRIDE;
    const float g = rec[MG_G2D_OPACITY];
    if (g == 0.0f) return;  // no pixel took it: nothing to carry
    const AntialiasAdjoint r = antialias_adjoint(conic[3 * o], conic[3 * o + 1],
                                                 conic[3 * o + 2], opacity[i], g, blur);
    rec[MG_G2D_OPACITY] = r.d_op;
    rec[MG_G2D_CONIC] += r.dxx;
    rec[MG_G2D_CONIC + 1] += r.dxy;
    rec[MG_G2D_CONIC + 2] += r.dyy;
}

// ---------------------------------------------------------------- host side

// Forward and backward warp blocks per tile (Blocks / BwdBlocks on the host).
int blocks_per_tile(int tile) { return (tile * tile + 31) / 32; }
int bwd_blocks_per_tile(int tile) { return blocks_per_tile(tile) / bwd_px_for(tile); }

// Scratch shared by one view's forward and backward.
struct RasterScratch {
    int32_t* counters;    // [0] forward pull, [1] backward pull, [2] backward item count
    int32_t* order;       // n_tiles, longest list first
    int32_t* block_work;  // n_blocks walk lengths (forward)
    int32_t* pair_done;   // per backward block: its forward blocks finished
    int2* items;          // backward work items
    float* ckpt;          // checkpoint slots x 5 x pixel slots
    size_t bytes;
};

RasterScratch carve_raster(void* base, int W, int H, int tile, int64_t m) {
    const int64_t tiles_x = (W + tile - 1) / tile, tiles_y = (H + tile - 1) / tile;
    const int64_t n_tiles = tiles_x * tiles_y;
    const int bpt = blocks_per_tile(tile), bbpt = bwd_blocks_per_tile(tile);
    const int64_t n_blocks = n_tiles * bpt, n_bwd = n_tiles * bbpt;
    const int64_t m1 = std::max<int64_t>(m, 1);
    // sum over backward blocks of ceil(walk / kSeg) <= n_bwd + bbpt * m / kSeg
    const int64_t n_items = n_bwd + (int64_t)bbpt * ((m1 + kSeg - 1) / kSeg);
    const int64_t slots = m1 / kSeg + n_tiles;
    RasterScratch s;
    char* p = static_cast<char*>(base);
    s.counters = reinterpret_cast<int32_t*>(p); p += 256;
    s.order = reinterpret_cast<int32_t*>(p); p += align256(sizeof(int32_t) * n_tiles);
    s.block_work = reinterpret_cast<int32_t*>(p); p += align256(sizeof(int32_t) * n_blocks);
    s.pair_done = reinterpret_cast<int32_t*>(p); p += align256(sizeof(int32_t) * n_bwd);
    s.items = reinterpret_cast<int2*>(p); p += align256(sizeof(int2) * n_items);
    s.ckpt = reinterpret_cast<float*>(p);
    p += align256(sizeof(float) * (size_t)slots * 5 * (size_t)bpt * 32);
    s.bytes = (size_t)(p - static_cast<char*>(base));
    return s;
}

// CTAs that fit on the device at once, per (kernel, device).
int persistent_grid(const void* kernel, int threads) {
    static std::mutex mu;
    static std::unordered_map<uint64_t, int> cache;
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return 0;
    const uint64_t key = (reinterpret_cast<uint64_t>(kernel) << 6) ^ (uint64_t)dev;
    std::lock_guard<std::mutex> lock(mu);
    auto it = cache.find(key);
    if (it != cache.end()) return it->second;
    int per_sm = 0, sms = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kernel, threads, 0) !=
            cudaSuccess ||
        cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess)
        return 0;
    const int grid = std::max(per_sm, 1) * sms;
    cache[key] = grid;
    return grid;
}

template <int TILE>
mg_status launch_fwd(const float4* splats, const int32_t* ids, const int32_t* offsets, int W,
                     int H, int tiles_x, int tiles_y, const float* bg, float* rgb,
                     float* alpha, float* T, int32_t* stop, int32_t* tile_work,
                     const RasterScratch& sc, int m_cap, cudaStream_t stream) {
    const int n_tiles = tiles_x * tiles_y;
    tile_order_kernel<<<1, 1024, 0, stream>>>(offsets, nullptr, n_tiles, sc.order, sc.counters,
                                              tile_work, T ? sc.pair_done : nullptr,
                                              n_tiles * BwdBlocks<TILE>::kCount);
    MG_TRY(check_launch("rasterize_forward order"));
    const void* k = reinterpret_cast<const void*>(&raster_forward_kernel<TILE>);
    const int grid = persistent_grid(k, kRasterWarps * 32);
    if (grid <= 0) return check_launch("rasterize_forward occupancy");
    raster_forward_kernel<TILE><<<grid, kRasterWarps * 32, 0, stream>>>(
        splats, ids, offsets, W, H, tiles_x, n_tiles, bg != nullptr, bg ? bg[0] : 0.f,
        bg ? bg[1] : 0.f, bg ? bg[2] : 0.f, rgb, alpha, T, stop, sc.order, sc.counters,
        sc.block_work, tile_work, T ? sc.ckpt : nullptr, T ? sc.items : nullptr, sc.pair_done,
        m_cap, device_error_word());
    return check_launch("rasterize_forward");
}

template <int TILE, bool kSegmented>
mg_status launch_bwd_mode(const float4* splats, const int32_t* ids, const int32_t* offsets,
                          const float* rgb, const float* alpha, const float* final_T,
                          const int32_t* stop, const float* grad_rgb, const float* grad_alpha,
                          int W, int H, int tiles_x, int tiles_y, const float* bg,
                          int want_absgrad, float* grad2d, const RasterScratch& sc,
                          int m_cap, cudaStream_t stream) {
    const int n_tiles = tiles_x * tiles_y;
    if (kSegmented) {
        // the forward of this view appended the items and their count; only
        // the pull counter starts over (a second backward reuses the items)
        if (cudaMemsetAsync(sc.counters + 1, 0, sizeof(int32_t), stream) != cudaSuccess)
            return check_launch("rasterize_backward counter");
    } else {
        backward_items_kernel<<<1, 1024, 0, stream>>>(offsets, nullptr, n_tiles,
                                                      BwdBlocks<TILE>::kCount, 0, sc.items,
                                                      sc.counters);
        MG_TRY(check_launch("rasterize_backward items"));
    }
    const void* k = reinterpret_cast<const void*>(&raster_backward_kernel<TILE, kSegmented>);
    const int grid = persistent_grid(k, kRasterWarps * 32);
    if (grid <= 0) return check_launch("rasterize_backward occupancy");
    raster_backward_kernel<TILE, kSegmented><<<grid, kRasterWarps * 32, 0, stream>>>(
        splats, ids, offsets, rgb, alpha, final_T, stop, grad_rgb, grad_alpha, W, H, tiles_x,
        bg != nullptr, bg ? bg[0] : 0.f, bg ? bg[1] : 0.f, bg ? bg[2] : 0.f, want_absgrad,
        grad2d, sc.items, sc.counters, sc.ckpt, m_cap, device_error_word());
    return check_launch("rasterize_backward");
}

template <int TILE>
mg_status launch_bwd(bool segmented, const float4* splats, const int32_t* ids,
                     const int32_t* offsets, const float* rgb, const float* alpha,
                     const float* final_T, const int32_t* stop, const float* grad_rgb,
                     const float* grad_alpha, int W, int H, int tiles_x, int tiles_y,
                     const float* bg, int want_absgrad, float* grad2d, const RasterScratch& sc,
                     int m_cap, cudaStream_t stream) {
    if (segmented)
        return launch_bwd_mode<TILE, true>(splats, ids, offsets, rgb, alpha, final_T, stop,
                                           grad_rgb, grad_alpha, W, H, tiles_x, tiles_y, bg,
                                           want_absgrad, grad2d, sc, m_cap, stream);
    return launch_bwd_mode<TILE, false>(splats, ids, offsets, rgb, alpha, final_T, stop,
                                        grad_rgb, grad_alpha, W, H, tiles_x, tiles_y, bg,
                                        want_absgrad, grad2d, sc, m_cap, stream);
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

extern "C" size_t mg_raster_scratch_bytes(int32_t width, int32_t height, int32_t tile,
                                          int64_t m) {
    if (width <= 0 || height <= 0 || tile <= 0 || m < 0) return 0;
    return carve_raster(nullptr, width, height, tile, m).bytes;
}

extern "C" mg_status mg_pack_splats(const float* uv, const float* conic, const float* opacity,
                                    const float* color, int64_t n, void* splats,
                                    float* grad2d_zero, mg_stream_t stream) {
    MG_REQUIRE(n >= 0, "pack_splats: negative count");
    if (n == 0) return MG_OK;
    MG_REQUIRE(uv && conic && opacity && color && splats, "pack_splats: null pointer");
    MG_REQUIRE((reinterpret_cast<uintptr_t>(splats) & 15u) == 0u &&
                   (reinterpret_cast<uintptr_t>(grad2d_zero) & 15u) == 0u,
               "pack_splats: splats and grad2d_zero must be 16-byte aligned");
    pack_splats_kernel<<<ceil_div(n, 256), 256, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
        reinterpret_cast<const float2*>(uv), conic, opacity, color, n,
        static_cast<float4*>(splats), reinterpret_cast<float4*>(grad2d_zero));
    return check_launch("pack_splats");
}

extern "C" mg_status mg_rasterize_forward(const void* splats, const int32_t* gauss_ids,
                                          const int32_t* tile_offsets, int64_t m,
                                          int32_t width, int32_t height, int32_t tile,
                                          int32_t tiles_x, const float* background,
                                          float* out_rgb, float* out_alpha, float* out_T,
                                          int32_t* out_stop, int32_t* tile_work,
                                          void* scratch, size_t scratch_bytes,
                                          mg_stream_t stream) {
    MG_TRY(check_tile(tile));
    MG_REQUIRE(width > 0 && height > 0, "rasterize_forward: empty image");
    const int tiles_y = (height + tile - 1) / tile;
    MG_REQUIRE(tiles_x == (width + tile - 1) / tile, "rasterize_forward: tiles_x mismatch");
    MG_REQUIRE(tile_offsets && out_rgb && out_alpha && scratch,
               "rasterize_forward: null pointer");
    MG_REQUIRE((out_T == nullptr) == (out_stop == nullptr),
               "rasterize_forward: give both out_T and out_stop, or neither (forward only)");
    MG_REQUIRE(m >= 0 && m < ((int64_t)1 << 31), "rasterize_forward: pair count out of range");
    MG_REQUIRE(m == 0 || (splats && gauss_ids), "rasterize_forward: null splats or ids");
    MG_REQUIRE((reinterpret_cast<uintptr_t>(splats) & 15u) == 0u &&
                   (reinterpret_cast<uintptr_t>(scratch) & 15u) == 0u,
               "rasterize_forward: splats and scratch must be 16-byte aligned");
    const RasterScratch sc = carve_raster(scratch, width, height, tile, m);
    MG_REQUIRE(scratch_bytes >= sc.bytes,
               "rasterize_forward: scratch too small (mg_raster_scratch_bytes)");
    cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
    const float4* sp = static_cast<const float4*>(splats);
    switch (tile) {
        case 8: return launch_fwd<8>(sp, gauss_ids, tile_offsets, width, height, tiles_x, tiles_y, background, out_rgb, out_alpha, out_T, out_stop, tile_work, sc, (int)m, s);
        case 12: return launch_fwd<12>(sp, gauss_ids, tile_offsets, width, height, tiles_x, tiles_y, background, out_rgb, out_alpha, out_T, out_stop, tile_work, sc, (int)m, s);
        case 16: return launch_fwd<16>(sp, gauss_ids, tile_offsets, width, height, tiles_x, tiles_y, background, out_rgb, out_alpha, out_T, out_stop, tile_work, sc, (int)m, s);
        default: return launch_fwd<32>(sp, gauss_ids, tile_offsets, width, height, tiles_x, tiles_y, background, out_rgb, out_alpha, out_T, out_stop, tile_work, sc, (int)m, s);
    }
}

extern "C" mg_status mg_rasterize_backward(
    const void* splats, const int32_t* gauss_ids, const int32_t* tile_offsets, int64_t m,
    const float* out_rgb, const float* out_alpha, const float* final_T, const int32_t* stop,
    const float* grad_rgb, const float* grad_alpha, int32_t width, int32_t height,
    int32_t tile, int32_t tiles_x, const float* background, int32_t want_absgrad, int64_t n,
    float* grad2d, int32_t segmented, void* scratch, size_t scratch_bytes,
    mg_stream_t stream) {
    MG_TRY(check_tile(tile));
    MG_REQUIRE(width > 0 && height > 0, "rasterize_backward: empty image");
    const int tiles_y = (height + tile - 1) / tile;
    MG_REQUIRE(tiles_x == (width + tile - 1) / tile, "rasterize_backward: tiles_x mismatch");
    MG_REQUIRE(final_T && stop && grad_rgb && tile_offsets && scratch,
               "rasterize_backward: null pointer");
    MG_REQUIRE(background == nullptr || out_alpha != nullptr,
               "rasterize_backward: the background blend needs the forward alpha");
    MG_REQUIRE(!segmented || (out_rgb && out_alpha),
               "rasterize_backward: segments need the forward's rgb and alpha");
    MG_REQUIRE(m >= 0 && m < ((int64_t)1 << 31), "rasterize_backward: pair count out of range");
    MG_REQUIRE((reinterpret_cast<uintptr_t>(grad2d) & 15u) == 0u &&
                   (reinterpret_cast<uintptr_t>(splats) & 15u) == 0u &&
                   (reinterpret_cast<uintptr_t>(scratch) & 15u) == 0u,
               "rasterize_backward: grad2d, splats and scratch must be 16-byte aligned");
    if (n == 0 || m == 0) return MG_OK;
    MG_REQUIRE(splats && gauss_ids && grad2d, "rasterize_backward: null splats, ids or grad2d");
    const RasterScratch sc = carve_raster(scratch, width, height, tile, m);
    MG_REQUIRE(scratch_bytes >= sc.bytes,
               "rasterize_backward: scratch too small (mg_raster_scratch_bytes)");
    cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
    const float4* sp = static_cast<const float4*>(splats);
    const bool seg = segmented != 0;
    switch (tile) {
        case 8: return launch_bwd<8>(seg, sp, gauss_ids, tile_offsets, out_rgb, out_alpha, final_T, stop, grad_rgb, grad_alpha, width, height, tiles_x, tiles_y, background, want_absgrad, grad2d, sc, (int)m, s);
        case 12: return launch_bwd<12>(seg, sp, gauss_ids, tile_offsets, out_rgb, out_alpha, final_T, stop, grad_rgb, grad_alpha, width, height, tiles_x, tiles_y, background, want_absgrad, grad2d, sc, (int)m, s);
        case 16: return launch_bwd<16>(seg, sp, gauss_ids, tile_offsets, out_rgb, out_alpha, final_T, stop, grad_rgb, grad_alpha, width, height, tiles_x, tiles_y, background, want_absgrad, grad2d, sc, (int)m, s);
        default: return launch_bwd<32>(seg, sp, gauss_ids, tile_offsets, out_rgb, out_alpha, final_T, stop, grad_rgb, grad_alpha, width, height, tiles_x, tiles_y, background, want_absgrad, grad2d, sc, (int)m, s);
    }
}

extern "C" mg_status mg_tile_order(const int32_t* tile_offsets, const int32_t* work,
                                   int32_t n_tiles, int32_t* order, mg_stream_t stream) {
    MG_REQUIRE(n_tiles > 0 && order != nullptr, "tile_order: bad arguments");
    MG_REQUIRE(work != nullptr || tile_offsets != nullptr, "tile_order: no work measure");
    tile_order_kernel<<<1, 1024, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
        tile_offsets, work, n_tiles, order, nullptr, nullptr, nullptr, 0);
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

extern "C" mg_status mg_antialias_opacity(const float* conic, const float* opacity, int64_t n,
                                          float blur, float* out, mg_stream_t stream) {
    MG_REQUIRE(n >= 0, "antialias_opacity: negative count");
    if (n == 0) return MG_OK;
    MG_REQUIRE(conic && opacity && out, "antialias_opacity: null pointer");
    antialias_opacity_kernel<<<ceil_div(n, 256), 256, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
        conic, opacity, n, blur, out);
    return check_launch("antialias_opacity");
}

extern "C" mg_status mg_antialias_opacity_views(const float* conic, const float* opacity,
                                                int64_t n, int32_t n_views, int64_t view_stride,
                                                float blur, float* out, mg_stream_t stream) {
    MG_REQUIRE(n >= 0 && n_views >= 0 && n_views <= 65535, "antialias_opacity_views: bad counts");
    MG_REQUIRE(view_stride >= n, "antialias_opacity_views: view_stride below n");
    if (n == 0 || n_views == 0) return MG_OK;
    MG_REQUIRE(conic && opacity && out, "antialias_opacity_views: null pointer");
    antialias_opacity_views_kernel<<<dim3((unsigned)ceil_div(n, 256), (unsigned)n_views), 256, 0,
                                     reinterpret_cast<cudaStream_t>(stream)>>>(
        conic, opacity, n, view_stride, blur, out);
    return check_launch("antialias_opacity_views");
}

extern "C" mg_status mg_antialias_grad2d_views(const float* conic, const float* opacity,
                                               int64_t n, int32_t n_views, int64_t view_stride,
                                               float blur, float* grad2d, mg_stream_t stream) {
    MG_REQUIRE(n >= 0 && n_views >= 0 && n_views <= 65535, "antialias_grad2d_views: bad counts");
    MG_REQUIRE(view_stride >= n, "antialias_grad2d_views: view_stride below n");
    if (n == 0 || n_views == 0) return MG_OK;
    MG_REQUIRE(conic && opacity && grad2d, "antialias_grad2d_views: null pointer");
    antialias_grad2d_views_kernel<<<dim3((unsigned)ceil_div(n, 256), (unsigned)n_views), 256, 0,
                                    reinterpret_cast<cudaStream_t>(stream)>>>(
        conic, opacity, n, view_stride, blur, grad2d);
    return check_launch("antialias_grad2d_views");
}

extern "C" mg_status mg_antialias_opacity_backward(const float* conic, const float* opacity,
                                                   const float* grad_out, int64_t n, float blur,
                                                   float* d_conic, float* d_opacity,
                                                   mg_stream_t stream) {
    MG_REQUIRE(n >= 0, "antialias_opacity_backward: negative count");
    if (n == 0) return MG_OK;
    MG_REQUIRE(conic && opacity && grad_out && d_conic && d_opacity,
               "antialias_opacity_backward: null pointer");
    antialias_opacity_backward_kernel<<<ceil_div(n, 256), 256, 0,
                                        reinterpret_cast<cudaStream_t>(stream)>>>(
        conic, opacity, grad_out, n, blur, d_conic, d_opacity);
    return check_launch("antialias_opacity_backward");
}
