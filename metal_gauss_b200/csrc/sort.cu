// Stable LSD radix sort (onesweep form), the gathered exclusive scan and the
// per-tile range extraction used by the binning.
//
// Onesweep: one histogram kernel counts the digits of every pass at once;
// then each 8-bit pass is ONE kernel that reads each key/value once, ranks it
// inside its CTA tile, learns the tile's global offset per digit through a
// decoupled look-back over the previous tiles, and writes each key/value
// once. Tiles are claimed through an atomic counter, so a CTA only ever waits
// for tiles already claimed by running CTAs; every wait is bounded and a
// timeout records DEV_ERR_SORT_LOOKBACK_TIMEOUT in the device error word
// instead of hanging.
//
// Ranking is stable: a warp ranks its 32 x ITEMS keys in input order with
// __match_any_sync peer groups and warp-private counters; warps are combined
// in warp order, tiles in tile order, so equal digits keep their input order
// and the sort is stable across passes.
//
// Segments: the input may be `segments` equal runs, each sorted on its own
// and kept in place (a batch of views sorting each view's rows). Tiles never
// straddle a segment, digits are counted per segment, and a tile looks back
// only over its own segment's tiles. A pass in which all of a segment's keys
// share one digit copies that segment's tiles through.
#include <algorithm>
#include <string>

#include "kernels.cuh"

namespace mg {

namespace {

constexpr int kRadixBits = 8;
constexpr int kRadix = 1 << kRadixBits;

// Bits per pass: the key bits split evenly over the fewest 8-bit-or-narrower
// passes (12-bit tile ids sort as 6 + 6, not 8 + 4: 64 bins per pass keep the
// scatter's runs longer than 256 would).
__host__ __device__ __forceinline__ int pass_bits(int bits) {
    const int passes = (bits + kRadixBits - 1) / kRadixBits;
    return (bits + passes - 1) / passes;
}
constexpr int kSortThreads = 256;
constexpr int kSortWarps = kSortThreads / 32;
constexpr int kHistPrivatePasses = 4;  // per-warp histogram copies up to this many passes

template <typename K> struct SortTraits;
#ifndef MG_SORT_ITEMS32
#define MG_SORT_ITEMS32 16
#endif
template <> struct SortTraits<uint32_t> { static constexpr int kItems = MG_SORT_ITEMS32; };
template <> struct SortTraits<uint64_t> { static constexpr int kItems = 10; };

template <typename K>
__host__ __device__ constexpr int tile_keys() { return kSortThreads * SortTraits<K>::kItems; }

constexpr uint32_t kFlagAgg = 1u << 30;
constexpr uint32_t kFlagInc = 2u << 30;
constexpr uint32_t kCountMask = (1u << 30) - 1u;
// Look-back rounds a tile waits on an unpublished predecessor before it gives
// up (a few milliseconds; a healthy predecessor publishes within microseconds).
constexpr uint32_t kLookbackSpinLimit = 1u << 22;
#ifndef MG_SORT_LOOKBACK
#define MG_SORT_LOOKBACK 4
#endif
constexpr int kLookback = MG_SORT_LOOKBACK;  // predecessor words read per round trip

struct SortScratch {
    uint32_t* hist;           // passes x 256 (x segments): histogram, then exclusive offsets
    uint32_t* tile_counter;   // passes
    uint32_t* status;         // passes x tiles x 256 look-back words
    uint32_t* one_digit;      // segmented: passes x segments flags (all keys share a digit)
    int tiles;                // segments x tiles_per_seg
    int tiles_per_seg;
    int passes;
    size_t bytes;
};

inline size_t align256(size_t x) { return (x + 255) & ~(size_t)255; }

// n keys in `segments` equal runs (segments divides n). With one segment the
// layout is hist | counters | status, as the allocation-free entry point's
// fixed array assumes.
SortScratch carve(void* base, int64_t n, int bits, int key_bytes, int segments = 1) {
    SortScratch s;
    s.passes = (bits + kRadixBits - 1) / kRadixBits;
    const int tk = key_bytes == 4 ? tile_keys<uint32_t>() : tile_keys<uint64_t>();
    segments = std::max(segments, 1);
    const int64_t seg_n = n / segments;
    s.tiles_per_seg = (int)std::max<int64_t>(1, (seg_n + tk - 1) / tk);
    s.tiles = s.tiles_per_seg * segments;
    char* p = static_cast<char*>(base);
    s.hist = reinterpret_cast<uint32_t*>(p);
    p += align256(sizeof(uint32_t) * kRadix * s.passes * segments);
    s.tile_counter = reinterpret_cast<uint32_t*>(p);
    p += align256(sizeof(uint32_t) * s.passes);
    s.status = reinterpret_cast<uint32_t*>(p);
    p += align256(sizeof(uint32_t) * (size_t)s.tiles * kRadix * s.passes);
    s.one_digit = nullptr;
    if (segments > 1) {
        s.one_digit = reinterpret_cast<uint32_t*>(p);
        p += align256(sizeof(uint32_t) * (size_t)s.passes * segments);
    }
    s.bytes = (size_t)(p - static_cast<char*>(base));
    return s;
}

size_t sort_scratch_size(int64_t n, int bits, int key_bytes, int segments = 1) {
    return carve(nullptr, n, bits, key_bytes, segments).bytes;
}

template <typename K>
__device__ __forceinline__ uint32_t digit_of(K key, int shift, uint32_t mask) {
    return (uint32_t)(key >> shift) & mask;
}

// Digit histograms of all passes in one read of the keys (blockIdx.y is the
// segment, of seg_n keys; hist is passes x segments x 256).
template <typename K>
__global__ void __launch_bounds__(kSortThreads)
radix_histogram_kernel(const K* __restrict__ keys, int64_t seg_n, int bits, int passes,
                       uint32_t* __restrict__ hist) {
    const int seg = blockIdx.y, segments = gridDim.y;
    keys += (int64_t)seg * seg_n;
    const int64_t n = seg_n;
    // One counter set per warp (keys with few distinct digits, such as the
    // high bits of tile ids, would otherwise serialise every warp of the
    // block on the same shared-memory words), when they fit.
    extern __shared__ uint32_t s_hist[];
    const bool per_warp = passes <= kHistPrivatePasses;
    const int sets = per_warp ? kSortWarps : 1;
    const int words = sets * passes * kRadix;
    for (int i = threadIdx.x; i < words; i += kSortThreads) s_hist[i] = 0u;
    __syncthreads();
    uint32_t* mine = s_hist + (per_warp ? (threadIdx.x >> 5) * passes * kRadix : 0);
    const int pb = pass_bits(bits);
    auto count = [&](K k) {
        for (int p = 0; p < passes; ++p) {
            const int shift = p * pb;
            atomicAdd(&mine[p * kRadix + digit_of(k, shift, (1u << min(pb, bits - shift)) - 1u)],
                      1u);
        }
    };
    // 16-byte loads over the aligned body (several keys in flight per
    // thread), single keys before and after it
    constexpr int VW = 16 / (int)sizeof(K);
    const int64_t lead =
        (VW - (int64_t)((reinterpret_cast<uintptr_t>(keys) / sizeof(K)) % VW)) % VW;
    const int64_t head = lead < n ? lead : n;
    const int64_t body = (n - head) / VW;
    const int64_t tid = (int64_t)blockIdx.x * kSortThreads + threadIdx.x;
    const int64_t nthreads = (int64_t)gridDim.x * kSortThreads;
    if (tid < head) count(keys[tid]);
    const uint4* vec = reinterpret_cast<const uint4*>(keys + head);
    for (int64_t i = tid; i < body; i += nthreads) {
        const uint4 q = vec[i];
        const K* kk = reinterpret_cast<const K*>(&q);
#pragma unroll
        for (int j = 0; j < VW; ++j) count(kk[j]);
    }
    for (int64_t i = head + body * VW + tid; i < n; i += nthreads) count(keys[i]);
    __syncthreads();
    for (int i = threadIdx.x; i < passes * kRadix; i += kSortThreads) {
        uint32_t c = 0u;
        for (int w = 0; w < sets; ++w) c += s_hist[w * passes * kRadix + i];
        const int p = i / kRadix, d = i % kRadix;
        if (c) atomicAdd(&hist[((int64_t)p * segments + seg) * kRadix + d], c);
    }
}

// Exclusive scan of each (pass, segment)'s 256 digit counts (one CTA each);
// with one_digit given, also whether one digit holds all seg_n keys.
__global__ void __launch_bounds__(kRadix) radix_offsets_kernel(uint32_t* hist,
                                                               uint32_t* one_digit,
                                                               int64_t seg_n) {
    __shared__ uint32_t s[kRadix];
    uint32_t* h = hist + blockIdx.x * kRadix;
    const int t = threadIdx.x;
    const uint32_t v = h[t];
    if (one_digit) {
        const int all = __syncthreads_or((int64_t)v == seg_n);
        if (t == 0) one_digit[blockIdx.x] = all ? 1u : 0u;
    }
    s[t] = v;
    __syncthreads();
    for (int off = 1; off < kRadix; off <<= 1) {
        const uint32_t add = t >= off ? s[t - off] : 0u;
        __syncthreads();
        s[t] += add;
        __syncthreads();
    }
    h[t] = s[t] - v;
}

constexpr int kMaxSortSegments = 256;

template <typename K>
struct OnesweepSmem {
    K keys[tile_keys<K>()];
    uint32_t vals[tile_keys<K>()];
    uint32_t warp_hist[kSortWarps][kRadix];
    uint32_t local_start[kRadix];
    uint32_t bin_offset[kRadix];
    uint32_t one_digit[kMaxSortSegments];  // segmented passes: the per-segment flags
    uint32_t tile_id;
};

// Resident 256-thread CTAs per SM the pass's registers are held to (0: none;
// 4 -- 64 registers, no spills -- measured the same on the bench).
#ifndef MG_SORT_MIN_CTAS
#define MG_SORT_MIN_CTAS 0
#endif
template <typename K, bool kSegmented = false>
__global__ void __launch_bounds__(kSortThreads, MG_SORT_MIN_CTAS)
onesweep_pass_kernel(const K* __restrict__ keys_in, const uint32_t* __restrict__ vals_in,
                     K* __restrict__ keys_out, uint32_t* __restrict__ vals_out,
                     int64_t n, int shift, int digit_bits,
                     const uint32_t* __restrict__ digit_offsets,
                     uint32_t* __restrict__ tile_counter, uint32_t* status,
                     int32_t* err_word, uint32_t spin_limit, int tiles_per_seg = 0,
                     const uint32_t* __restrict__ one_digit = nullptr,
                     bool write_keys = true) {
    // kSegmented: n keys per segment, tiles_per_seg tiles each, one_digit the
    // pass's per-segment flags; otherwise one segment of n keys. write_keys
    // false: only the values go out (a last pass whose keys nobody reads).
    constexpr int ITEMS = SortTraits<K>::kItems;
    constexpr int TK = tile_keys<K>();
    __shared__ OnesweepSmem<K> sm;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const uint32_t mask = (1u << digit_bits) - 1u;

    // A pass whose digit is the same for every key keeps the order: copy the
    // tile through (each block decides alike from the digit offsets). With
    // segments the test is per segment, after the claim.
    if (!kSegmented) {
        const uint32_t d0 = digit_of(keys_in[0], shift, mask);
        const uint32_t next = d0 + 1u < (uint32_t)kRadix ? digit_offsets[d0 + 1u] : (uint32_t)n;
        if (digit_offsets[d0] == 0u && (int64_t)next == n) {
            for (int64_t i = (int64_t)blockIdx.x * TK + tid;
                 i < min(n, (int64_t)(blockIdx.x + 1) * TK); i += kSortThreads) {
                if (write_keys) keys_out[i] = keys_in[i];
                vals_out[i] = vals_in[i];
            }
            return;
        }
    }

    for (int i = tid; i < kSortWarps * kRadix; i += kSortThreads)
        (&sm.warp_hist[0][0])[i] = 0u;
    // the segments' one-digit flags, read while the tile is claimed
    if (kSegmented && tid < (int)(gridDim.x / (unsigned)tiles_per_seg))
        sm.one_digit[tid] = one_digit[tid];
    if (tid == 0) sm.tile_id = atomicAdd(tile_counter, 1u);
    __syncthreads();
    const uint32_t tile = sm.tile_id;
    int tl = (int)tile;  // the tile's index within its segment
    int64_t seg_base = 0, end = n;
    if (kSegmented) {
        const int seg = (int)(tile / (uint32_t)tiles_per_seg);
        tl -= seg * tiles_per_seg;
        seg_base = (int64_t)seg * n;
        end = seg_base + n;
        digit_offsets += (int64_t)seg * kRadix;
        if (sm.one_digit[seg]) {  // block-uniform: copy the tile through
            for (int64_t i = seg_base + (int64_t)tl * TK + tid;
                 i < min(end, seg_base + (int64_t)(tl + 1) * TK); i += kSortThreads) {
                if (write_keys) keys_out[i] = keys_in[i];
                vals_out[i] = vals_in[i];
            }
            return;
        }
    }
    const int64_t base = seg_base + (int64_t)tl * TK;

    // Warp w owns input slots [w*32*ITEMS, (w+1)*32*ITEMS) of the tile; item i
    // of lane l is slot i*32 + l inside it, so (i, l) order is input order.
    K key[ITEMS];
    uint32_t val[ITEMS];
    uint32_t rank[ITEMS];
#pragma unroll
    for (int i = 0; i < ITEMS; ++i) {
        const int64_t idx = base + (int64_t)warp * 32 * ITEMS + i * 32 + lane;
        if (idx < end) {
            key[i] = keys_in[idx];
            val[i] = vals_in[idx];
        } else {
            key[i] = ~(K)0;  // max digit: ranks after every real key of the tile
            val[i] = 0u;
        }
    }
    const unsigned lt_mask = (1u << lane) - 1u;
#pragma unroll
    for (int i = 0; i < ITEMS; ++i) {
        const uint32_t d = digit_of(key[i], shift, mask);
        const unsigned peers = __match_any_sync(0xffffffffu, d);
        const int leader = __ffs(peers) - 1;
        uint32_t before = 0u;
        if (lane == leader) {
            before = sm.warp_hist[warp][d];
            sm.warp_hist[warp][d] = before + (uint32_t)__popc(peers);
        }
        before = __shfl_sync(0xffffffffu, before, leader);
        rank[i] = before + (uint32_t)__popc(peers & lt_mask);
        __syncwarp();
    }
    __syncthreads();

    // Per digit (one thread each): warp offsets inside the tile, tile count.
    const int d = tid;
    uint32_t tile_count = 0u;
    for (int w = 0; w < kSortWarps; ++w) {
        const uint32_t c = sm.warp_hist[w][d];
        sm.warp_hist[w][d] = tile_count;
        tile_count += c;
    }
    // Publish this tile's aggregate first so successors can proceed. Digits a
    // narrow pass cannot produce are empty in every tile: no tile publishes
    // or reads their words.
    const bool in_pass = d <= (int)mask;
    uint32_t* my_status = status + (int64_t)tile * kRadix + d;
    if (in_pass) {
        if (tl == 0) {
            atomicExch(my_status, kFlagInc | tile_count);
        } else {
            atomicExch(my_status, kFlagAgg | tile_count);
        }
    }
    // Exclusive scan of tile counts over digits -> local layout.
    sm.local_start[d] = tile_count;
    __syncthreads();
    for (int off = 1; off < kRadix; off <<= 1) {
        const uint32_t add = d >= off ? sm.local_start[d - off] : 0u;
        __syncthreads();
        sm.local_start[d] += add;
        __syncthreads();
    }
    sm.local_start[d] -= tile_count;

    // Decoupled look-back over previous tiles for this digit, kLookback
    // predecessors per round trip (independent loads): aggregates are added
    // up to the first inclusive prefix; a word not yet published ends the
    // round and is read again.
    uint32_t excl = 0u;
    if (tl > 0 && in_pass) {
        int64_t t = (int64_t)tile - 1;
        const int64_t first = (int64_t)tile - tl;  // the segment's first tile: inclusive
        uint32_t spins = 0u;
        for (;;) {
            uint32_t sv[kLookback];
#pragma unroll
            for (int k = 0; k < kLookback; ++k)  // never read past the first tile
                sv[k] = t - k >= first
                            ? (uint32_t)*(volatile uint32_t*)(status + (t - k) * kRadix + d)
                            : (uint32_t)kFlagInc;
            int k = 0;
            bool found = false;
#pragma unroll
            for (; k < kLookback; ++k) {
                const uint32_t flag = sv[k] & ~kCountMask;
                if (flag == 0u) break;
                excl += sv[k] & kCountMask;
                if (flag == kFlagInc) { found = true; break; }
            }
            if (found) break;
            if (k == 0 && ++spins > spin_limit) {
                record_device_error(err_word, DEV_ERR_SORT_LOOKBACK_TIMEOUT);
                break;
            }
            t -= k;
        }
        atomicExch(my_status, kFlagInc | ((excl + tile_count) & kCountMask));
    }
    sm.bin_offset[d] = digit_offsets[d] + excl;
    __syncthreads();

    // Scatter into shared memory in tile-sorted order...
#pragma unroll
    for (int i = 0; i < ITEMS; ++i) {
        const uint32_t dd = digit_of(key[i], shift, mask);
        const uint32_t pos = sm.local_start[dd] + sm.warp_hist[warp][dd] + rank[i];
        sm.keys[pos] = key[i];
        sm.vals[pos] = val[i];
    }
    __syncthreads();
    // ...and write out; consecutive positions of a digit run are consecutive
    // in the output. Padding keys land at or past the segment's end.
#pragma unroll
    for (int i = 0; i < ITEMS; ++i) {
        const int p = i * kSortThreads + tid;
        const K k = sm.keys[p];
        const uint32_t dd = digit_of(k, shift, mask);
        const int64_t out =
            seg_base + (int64_t)sm.bin_offset[dd] + (p - (int)sm.local_start[dd]);
        if (out < end) {
            if (write_keys) keys_out[out] = k;
            vals_out[out] = sm.vals[p];
        }
    }
}

// ------------------------------------------------------------------ scan

constexpr int kScanThreads = 1024;
constexpr int kScanItems = 4;
constexpr int kScanTile = kScanThreads * kScanItems;

__device__ __forceinline__ uint32_t gathered(const uint32_t* counts,
                                             const uint32_t* order, int64_t i,
                                             int64_t n) {
    if (i >= n) return 0u;
    return order ? counts[order[i]] : counts[i];
}

__device__ __forceinline__ unsigned long long block_sum_ull(unsigned long long v,
                                                            unsigned long long* s_warp) {
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
    if (lane == 0) s_warp[w] = v;
    __syncthreads();
    unsigned long long t = 0ull;
    if (threadIdx.x < 32) {
        t = threadIdx.x < (blockDim.x >> 5) ? s_warp[threadIdx.x] : 0ull;
        for (int o = 16; o > 0; o >>= 1) t += __shfl_xor_sync(0xffffffffu, t, o);
    }
    return t;  // valid in warp 0
}

__global__ void __launch_bounds__(kScanThreads)
scan_reduce_kernel(const uint32_t* __restrict__ counts, const uint32_t* __restrict__ order,
                   int64_t n, unsigned long long* __restrict__ partials) {
    __shared__ unsigned long long s_warp[32];
    const int64_t base = (int64_t)blockIdx.x * kScanTile;
    unsigned long long v = 0ull;
#pragma unroll
    for (int i = 0; i < kScanItems; ++i)
        v += gathered(counts, order, base + i * kScanThreads + threadIdx.x, n);
    const unsigned long long t = block_sum_ull(v, s_warp);
    if (threadIdx.x == 0) partials[blockIdx.x] = t;
}

// Exclusive scan of the per-block partials in place, one CTA, any length.
__global__ void __launch_bounds__(kScanThreads)
scan_partials_kernel(unsigned long long* partials, int nblocks) {
    __shared__ unsigned long long s[kScanThreads];
    __shared__ unsigned long long carry;
    if (threadIdx.x == 0) carry = 0ull;
    __syncthreads();
    for (int base = 0; base < nblocks; base += kScanThreads) {
        const int i = base + threadIdx.x;
        const unsigned long long v = i < nblocks ? partials[i] : 0ull;
        s[threadIdx.x] = v;
        __syncthreads();
        for (int off = 1; off < kScanThreads; off <<= 1) {
            const unsigned long long add = threadIdx.x >= off ? s[threadIdx.x - off] : 0ull;
            __syncthreads();
            s[threadIdx.x] += add;
            __syncthreads();
        }
        if (i < nblocks) partials[i] = carry + s[threadIdx.x] - v;
        __syncthreads();
        if (threadIdx.x == 0) carry += s[kScanThreads - 1];
        __syncthreads();
    }
}

__global__ void __launch_bounds__(kScanThreads)
scan_downsweep_kernel(const uint32_t* __restrict__ counts, const uint32_t* __restrict__ order,
                      int64_t n, const unsigned long long* __restrict__ partials,
                      uint32_t* __restrict__ out, int64_t* __restrict__ total_dev) {
    __shared__ unsigned long long s_warp[32];
    const int64_t base = (int64_t)blockIdx.x * kScanTile;
    // Blocked arrangement: thread t owns items [t*4, t*4+4) of the tile.
    uint32_t v[kScanItems];
    unsigned long long local = 0ull;
#pragma unroll
    for (int i = 0; i < kScanItems; ++i) {
        v[i] = gathered(counts, order, base + threadIdx.x * kScanItems + i, n);
        local += v[i];
    }
    // Block-wide exclusive scan of the per-thread sums.
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
    unsigned long long incl = local;
    for (int o = 1; o < 32; o <<= 1) {
        const unsigned long long y = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += y;
    }
    if (lane == 31) s_warp[w] = incl;
    __syncthreads();
    if (w == 0) {
        unsigned long long x = lane < (kScanThreads >> 5) ? s_warp[lane] : 0ull;
        for (int o = 1; o < 32; o <<= 1) {
            const unsigned long long y = __shfl_up_sync(0xffffffffu, x, o);
            if (lane >= o) x += y;
        }
        s_warp[lane] = x;  // inclusive over warps
    }
    __syncthreads();
    unsigned long long run = partials[blockIdx.x] + (w > 0 ? s_warp[w - 1] : 0ull) +
                             (incl - local);
#pragma unroll
    for (int i = 0; i < kScanItems; ++i) {
        const int64_t idx = base + threadIdx.x * kScanItems + i;
        if (idx < n) out[idx] = (uint32_t)run;
        run += v[i];
    }
    if (blockIdx.x == gridDim.x - 1 && threadIdx.x == kScanThreads - 1)
        *total_dev = (int64_t)run;
}

// ------------------------------------------------------------- tile ranges

__device__ __forceinline__ int64_t tile_at(const uint32_t* tiles, const uint64_t* keys64,
                                           int64_t i) {
    return tiles ? (int64_t)tiles[i] : (int64_t)(keys64[i] >> 32);
}

__global__ void tile_ranges_kernel(const uint32_t* __restrict__ tiles,
                                   const uint64_t* __restrict__ keys64, int64_t m,
                                   int n_tiles, int32_t* __restrict__ offsets) {
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= m) return;
    const int64_t t = min(tile_at(tiles, keys64, i), (int64_t)n_tiles);
    const int64_t prev = i == 0 ? -1 : min(tile_at(tiles, keys64, i - 1), (int64_t)n_tiles);
    for (int64_t tt = prev + 1; tt <= t; ++tt) offsets[tt] = (int32_t)i;
    if (i == m - 1)
        for (int64_t tt = t + 1; tt <= n_tiles; ++tt) offsets[tt] = (int32_t)m;
}

// Same as tile_ranges_kernel for 32-bit tile ids on a 16-byte boundary: each
// thread reads four consecutive ids with one vector load.
__global__ void tile_ranges4_kernel(const uint32_t* __restrict__ tiles, int64_t m, int n_tiles,
                                    int32_t* __restrict__ offsets) {
    const int64_t i0 = 4 * ((int64_t)blockIdx.x * blockDim.x + threadIdx.x);
    if (i0 >= m) return;
    uint32_t t[4];
    if (i0 + 3 < m) {
        const uint4 v = reinterpret_cast<const uint4*>(tiles)[i0 >> 2];
        t[0] = v.x; t[1] = v.y; t[2] = v.z; t[3] = v.w;
    } else {
        for (int k = 0; k < 4; ++k) t[k] = i0 + k < m ? tiles[i0 + k] : 0u;
    }
    int64_t prev = i0 == 0 ? -1 : min((int64_t)tiles[i0 - 1], (int64_t)n_tiles);
#pragma unroll
    for (int k = 0; k < 4; ++k) {
        const int64_t i = i0 + k;
        if (i >= m) break;
        const int64_t tk = min((int64_t)t[k], (int64_t)n_tiles);
        for (int64_t tt = prev + 1; tt <= tk; ++tt) offsets[tt] = (int32_t)i;
        if (i == m - 1)
            for (int64_t tt = tk + 1; tt <= n_tiles; ++tt) offsets[tt] = (int32_t)m;
        prev = tk;
    }
}

}  // namespace

size_t radix_sort_scratch_bytes(int64_t n, int bits, int key_bytes, int segments) {
    return sort_scratch_size(n, bits, key_bytes, segments);
}

template <typename K>
mg_status radix_sort_pairs(K* keys, uint32_t* vals, K* keys_alt, uint32_t* vals_alt,
                           int64_t n, int bits, void* scratch, size_t scratch_bytes,
                           bool* result_in_alt, cudaStream_t stream, int segments,
                           bool keys_out) {
    *result_in_alt = false;
    if (n <= 1 || bits <= 0) return MG_OK;
    if (bits > (int)(8 * sizeof(K)))
        return fail(MG_ERR_INVALID_ARGUMENT, "sort: bits exceeds the key width");
    if (n >= (int64_t)kCountMask)
        return fail(MG_ERR_CAPACITY, "sort: more than 2^30 elements");
    if (segments < 1 || segments > kMaxSortSegments || n % segments != 0)
        return fail(MG_ERR_INVALID_ARGUMENT, "sort: 1..256 segments that divide the key count");
    const size_t need = sort_scratch_size(n, bits, (int)sizeof(K), segments);
    if (scratch == nullptr || scratch_bytes < need)
        return fail(MG_ERR_INVALID_ARGUMENT, "sort: scratch buffer too small");
    SortScratch s = carve(scratch, n, bits, (int)sizeof(K), segments);
    if (cudaMemsetAsync(scratch, 0, need, stream) != cudaSuccess)
        return check_launch("sort scratch memset");
    const int64_t seg_n = n / segments;

    const int hist_blocks = (int)std::max<int64_t>(
        1, std::min<int64_t>((seg_n + 4095) / 4096, (148 * 4 + segments - 1) / segments));
    const size_t hist_smem = sizeof(uint32_t) * kRadix * s.passes *
                             (s.passes <= kHistPrivatePasses ? kSortWarps : 1);
    radix_histogram_kernel<K><<<dim3(hist_blocks, segments), kSortThreads, hist_smem, stream>>>(
        keys, seg_n, bits, s.passes, s.hist);
    MG_TRY(check_launch("radix_histogram"));
    radix_offsets_kernel<<<s.passes * segments, kRadix, 0, stream>>>(s.hist, s.one_digit, seg_n);
    MG_TRY(check_launch("radix_offsets"));

    int32_t* err = device_error_word();
    K* kin = keys; uint32_t* vin = vals;
    K* kout = keys_alt; uint32_t* vout = vals_alt;
    for (int p = 0; p < s.passes; ++p) {
        const int shift = p * pass_bits(bits);
        const int db = std::min(pass_bits(bits), bits - shift);
        const bool wk = keys_out || p + 1 < s.passes;
        if (segments > 1)
            onesweep_pass_kernel<K, true><<<s.tiles, kSortThreads, 0, stream>>>(
                kin, vin, kout, vout, seg_n, shift, db, s.hist + (size_t)p * segments * kRadix,
                s.tile_counter + p, s.status + (size_t)p * s.tiles * kRadix, err,
                kLookbackSpinLimit, s.tiles_per_seg, s.one_digit + (size_t)p * segments, wk);
        else
            onesweep_pass_kernel<K><<<s.tiles, kSortThreads, 0, stream>>>(
                kin, vin, kout, vout, n, shift, db, s.hist + p * kRadix, s.tile_counter + p,
                s.status + (size_t)p * s.tiles * kRadix, err, kLookbackSpinLimit, 0, nullptr,
                wk);
        MG_TRY(check_launch("onesweep_pass"));
        std::swap(kin, kout);
        std::swap(vin, vout);
    }
    *result_in_alt = (kin == keys_alt);
    return MG_OK;
}

template mg_status radix_sort_pairs<uint32_t>(uint32_t*, uint32_t*, uint32_t*, uint32_t*,
                                              int64_t, int, void*, size_t, bool*,
                                              cudaStream_t, int, bool);
template mg_status radix_sort_pairs<uint64_t>(uint64_t*, uint32_t*, uint64_t*, uint32_t*,
                                              int64_t, int, void*, size_t, bool*,
                                              cudaStream_t, int, bool);

size_t scan_scratch_bytes(int64_t n) {
    const int64_t blocks = std::max<int64_t>(1, (n + kScanTile - 1) / kScanTile);
    return align256(sizeof(unsigned long long) * blocks);
}

mg_status exclusive_scan_gather(const uint32_t* counts, const uint32_t* order, int64_t n,
                                uint32_t* out, int64_t* total_dev, void* scratch,
                                cudaStream_t stream) {
    if (n == 0) {
        if (cudaMemsetAsync(total_dev, 0, sizeof(int64_t), stream) != cudaSuccess)
            return check_launch("scan total memset");
        return MG_OK;
    }
    const int blocks = ceil_div(n, kScanTile);
    auto* partials = static_cast<unsigned long long*>(scratch);
    scan_reduce_kernel<<<blocks, kScanThreads, 0, stream>>>(counts, order, n, partials);
    MG_TRY(check_launch("scan_reduce"));
    scan_partials_kernel<<<1, kScanThreads, 0, stream>>>(partials, blocks);
    MG_TRY(check_launch("scan_partials"));
    scan_downsweep_kernel<<<blocks, kScanThreads, 0, stream>>>(counts, order, n, partials,
                                                              out, total_dev);
    return check_launch("scan_downsweep");
}

mg_status launch_tile_ranges(const uint32_t* tile_ids, const uint64_t* keys64, int64_t m,
                             int n_tiles, int32_t* offsets, cudaStream_t stream) {
    if (m == 0) {
        if (cudaMemsetAsync(offsets, 0, sizeof(int32_t) * (n_tiles + 1), stream) !=
            cudaSuccess)
            return check_launch("tile_ranges memset");
        return MG_OK;
    }
    if (keys64 == nullptr && (reinterpret_cast<uintptr_t>(tile_ids) & 15u) == 0u) {
        tile_ranges4_kernel<<<ceil_div((m + 3) / 4, 256), 256, 0, stream>>>(tile_ids, m, n_tiles,
                                                                          offsets);
        return check_launch("tile_ranges");
    }
    tile_ranges_kernel<<<ceil_div(m, 256), 256, 0, stream>>>(tile_ids, keys64, m, n_tiles,
                                                             offsets);
    return check_launch("tile_ranges");
}

}  // namespace mg

// ------------------------------------------------- allocation-free entry point
//
// mg_sort_pairs_u32_noalloc: the same onesweep sort with all of its scratch in
// one static device array, for callers that cannot allocate device memory
// (see include/mg_b200.h). Layout of the array: keys_alt (MAX_N u32) |
// vals_alt (MAX_N u32) | sort scratch for MAX_N 32-bit keys.
namespace mg {
namespace {

constexpr int64_t kNoallocMaxN = MG_SORT_NOALLOC_MAX_N;
constexpr size_t kNoallocPairBytes = sizeof(uint32_t) * (size_t)kNoallocMaxN;
// histograms + tile counters + look-back words for kNoallocMaxN keys, 4 passes
constexpr size_t kNoallocSortBytes =
    ((sizeof(uint32_t) * kRadix * 4 + 255) & ~(size_t)255) + 256 +
    ((sizeof(uint32_t) * (size_t)((kNoallocMaxN + tile_keys<uint32_t>() - 1) /
                                  tile_keys<uint32_t>()) * kRadix * 4 + 255) & ~(size_t)255);
constexpr size_t kNoallocBytes = 2 * kNoallocPairBytes + kNoallocSortBytes;
static_assert(kNoallocBytes == MG_SORT_NOALLOC_SCRATCH_BYTES,
              "MG_SORT_NOALLOC_SCRATCH_BYTES must state the static array's size");

static __device__ __align__(256) unsigned char g_noalloc_sort_scratch[kNoallocBytes];

DeviceSymbolCache g_noalloc_cache;

// Device address of the static array on the current device: looked up with
// that device current, cached per device and context (a device reset, which
// replaces the context, triggers a fresh lookup).
mg_status noalloc_base(unsigned char** out) {
    std::string why;
    void* p = device_symbol_address(&g_noalloc_sort_scratch, &g_noalloc_cache, &why);
    if (p == nullptr) return fail(MG_ERR_CUDA, "sort_pairs_u32_noalloc: " + why);
    *out = static_cast<unsigned char*>(p);
    return MG_OK;
}

}  // namespace
}  // namespace mg

extern "C" mg_status mg_sort_pairs_u32_noalloc(uint32_t* keys, uint32_t* vals, int64_t n,
                                               int32_t bits, mg_stream_t stream) {
    using namespace mg;
    if (n < 0 || n > kNoallocMaxN)
        return fail(MG_ERR_CAPACITY,
                    "sort_pairs_u32_noalloc: " + std::to_string(n) +
                        " pairs exceed the static scratch maximum of " +
                        std::to_string(kNoallocMaxN) +
                        " (MG_SORT_NOALLOC_MAX_N); use mg_sort_pairs_u32 with caller scratch");
    if (bits < 0 || bits > 32)
        return fail(MG_ERR_INVALID_ARGUMENT, "sort_pairs_u32_noalloc: bits must be in 0..32");
    if (n <= 1 || bits == 0) return MG_OK;
    if (keys == nullptr || vals == nullptr)
        return fail(MG_ERR_INVALID_ARGUMENT, "sort_pairs_u32_noalloc: null pointer");
    unsigned char* base = nullptr;
    MG_TRY(noalloc_base(&base));
    uint32_t* keys_alt = reinterpret_cast<uint32_t*>(base);
    uint32_t* vals_alt = reinterpret_cast<uint32_t*>(base + kNoallocPairBytes);
    void* scratch = base + 2 * kNoallocPairBytes;
    cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
    bool in_alt = false;
    // radix_sort_pairs clears the histogram, counter and look-back region it
    // uses before its first kernel, so the array's previous contents are harmless.
    MG_TRY(radix_sort_pairs<uint32_t>(keys, vals, keys_alt, vals_alt, n, bits, scratch,
                                      kNoallocSortBytes, &in_alt, s));
    if (in_alt) {
        if (cudaMemcpyAsync(keys, keys_alt, sizeof(uint32_t) * n, cudaMemcpyDeviceToDevice, s) !=
                cudaSuccess ||
            cudaMemcpyAsync(vals, vals_alt, sizeof(uint32_t) * n, cudaMemcpyDeviceToDevice, s) !=
                cudaSuccess)
            return check_launch("sort_pairs_u32_noalloc copy");
    }
    return MG_OK;
}

// ------------------------------------------------ bounded-wait self-test
//
// mg_sort_lookback_selftest: one onesweep pass launched as the second tile of
// a two-tile sort whose first tile never runs, so the look-back waits on a
// status word that nothing publishes. With a short spin limit the wait runs
// out, the kernel records DEV_ERR_SORT_LOOKBACK_TIMEOUT in the device error
// word and returns; every store stays inside the self-test's own buffers.
namespace mg {
namespace {

constexpr int64_t kSelftestKeys = 2 * (int64_t)tile_keys<uint32_t>();

struct SelftestScratch {
    uint32_t *keys_in, *vals_in, *keys_out, *vals_out, *hist, *tile_counter, *status;
    size_t bytes;
};

SelftestScratch carve_selftest(void* base) {
    SelftestScratch s;
    char* p = static_cast<char*>(base);
    const size_t arr = align256(sizeof(uint32_t) * kSelftestKeys);
    s.keys_in = reinterpret_cast<uint32_t*>(p); p += arr;
    s.vals_in = reinterpret_cast<uint32_t*>(p); p += arr;
    s.keys_out = reinterpret_cast<uint32_t*>(p); p += arr;
    s.vals_out = reinterpret_cast<uint32_t*>(p); p += arr;
    s.hist = reinterpret_cast<uint32_t*>(p); p += align256(sizeof(uint32_t) * kRadix);
    s.tile_counter = reinterpret_cast<uint32_t*>(p); p += 256;
    s.status = reinterpret_cast<uint32_t*>(p); p += align256(sizeof(uint32_t) * 2 * kRadix);
    s.bytes = (size_t)(p - static_cast<char*>(base));
    return s;
}

// Keys with digits 0..127 (never a single digit, so the pass does not take
// its copy-through shortcut), zero digit offsets and look-back words, and the
// tile counter at 1 so the one launched CTA claims tile 1.
__global__ void lookback_selftest_init_kernel(SelftestScratch s) {
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i < kSelftestKeys) {
        s.keys_in[i] = (uint32_t)(i & 0x7f);
        s.vals_in[i] = (uint32_t)i;
        s.keys_out[i] = 0u;
        s.vals_out[i] = 0u;
    }
    if (i < kRadix) s.hist[i] = 0u;
    if (i < 2 * kRadix) s.status[i] = 0u;
    if (i == 0) *s.tile_counter = 1u;
}

}  // namespace
}  // namespace mg

extern "C" size_t mg_sort_lookback_selftest_scratch_bytes(void) {
    return mg::carve_selftest(nullptr).bytes;
}

extern "C" mg_status mg_sort_lookback_selftest(uint32_t spin_limit, void* scratch,
                                               size_t scratch_bytes, mg_stream_t stream) {
    using namespace mg;
    MG_REQUIRE(spin_limit >= 1u && spin_limit <= kLookbackSpinLimit,
               "sort_lookback_selftest: spin_limit must be in 1..2^22");
    MG_REQUIRE(scratch != nullptr && (reinterpret_cast<uintptr_t>(scratch) & 255u) == 0u,
               "sort_lookback_selftest: scratch must be 256-byte aligned");
    const SelftestScratch s = carve_selftest(scratch);
    MG_REQUIRE(scratch_bytes >= s.bytes, "sort_lookback_selftest: scratch too small");
    int32_t* err = device_error_word();
    if (err == nullptr) return fail(MG_ERR_CUDA, "sort_lookback_selftest: no device error word");
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    lookback_selftest_init_kernel<<<ceil_div(kSelftestKeys, 256), 256, 0, st>>>(s);
    MG_TRY(check_launch("lookback_selftest_init"));
    onesweep_pass_kernel<uint32_t><<<1, kSortThreads, 0, st>>>(
        s.keys_in, s.vals_in, s.keys_out, s.vals_out, kSelftestKeys, 0, kRadixBits, s.hist,
        s.tile_counter, s.status, err, spin_limit);
    return check_launch("lookback_selftest_pass");
}
