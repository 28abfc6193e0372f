// C ABI glue: error reporting, the device error word, and the entry points
// that orchestrate several kernels (binning and sorting).
#include <atomic>
#include <mutex>
#include <string>

#include "kernels.cuh"

namespace mg {

namespace {
thread_local std::string g_last_error;
std::atomic<uint64_t> g_launches{0};

__device__ int32_t g_device_error_word;

DeviceSymbolCache g_error_cache;
std::mutex g_symbol_mu;

// The driver's cuCtxGetCurrent / cuCtxGetId, resolved through the runtime (the
// library links no driver stub). Null when the driver lacks them.
using CtxGetCurrentFn = int (*)(void**);
using CtxGetIdFn = int (*)(void*, unsigned long long*);

unsigned long long current_context_id() {
    static CtxGetCurrentFn get_current = [] {
        void* f = nullptr;
        return cudaGetDriverEntryPoint("cuCtxGetCurrent", &f, cudaEnableDefault) == cudaSuccess
                   ? reinterpret_cast<CtxGetCurrentFn>(f)
                   : nullptr;
    }();
    static CtxGetIdFn get_id = [] {
        void* f = nullptr;
        return cudaGetDriverEntryPoint("cuCtxGetId", &f, cudaEnableDefault) == cudaSuccess
                   ? reinterpret_cast<CtxGetIdFn>(f)
                   : nullptr;
    }();
    if (get_current == nullptr || get_id == nullptr) return 0ull;
    void* ctx = nullptr;
    if (get_current(&ctx) != 0 || ctx == nullptr) return 0ull;
    unsigned long long id = 0ull;
    return get_id(ctx, &id) == 0 ? id : 0ull;
}

// Copies the current device's error word (without clearing it) to a device
// int64, on the stream.
__global__ void peek_error_kernel(const int32_t* word, int64_t* out) {
    *out = (int64_t)*(const volatile int32_t*)word;
}

inline size_t align256(size_t x) { return (x + 255) & ~(size_t)255; }

int tile_bits(int n_tiles) {
    int b = 0;
    while ((1 << b) < n_tiles) ++b;
    return b < 1 ? 1 : b;
}

// Stage-A scratch carved into named arrays.
struct PrepareScratch {
    uint32_t* counts;
    uint32_t* dkeys;
    uint32_t* dvals;
    uint32_t* dkeys_alt;
    uint32_t* dvals_alt;
    uint32_t* offsets;
    uint4* recs;  // per Gaussian: the count walk's pass mask and rectangle
    uint32_t* cut_range;  // depth range words (two per view), then the histogram
    size_t range_bytes;   // the range words
    uint32_t* cut_hist;
    int32_t* cutoff;
    size_t cut_zero_bytes;  // range words + histogram, zeroed per call
    void* sort;
    size_t sort_bytes;
    void* scan;
    size_t total;
};

// Rows for n_views * n Gaussians; n_views = 1 is the single-view layout.
PrepareScratch carve_prepare(const void* base, int64_t n, int n_tiles, int n_views = 1) {
    PrepareScratch s;
    char* p = const_cast<char*>(static_cast<const char*>(base));
    n *= n_views;
    n_tiles *= n_views;
    const size_t arr = align256(sizeof(uint32_t) * (size_t)std::max<int64_t>(n, 1));
    s.counts = reinterpret_cast<uint32_t*>(p); p += arr;
    s.dkeys = reinterpret_cast<uint32_t*>(p); p += arr;
    s.dvals = reinterpret_cast<uint32_t*>(p); p += arr;
    s.dkeys_alt = reinterpret_cast<uint32_t*>(p); p += arr;
    s.dvals_alt = reinterpret_cast<uint32_t*>(p); p += arr;
    s.offsets = reinterpret_cast<uint32_t*>(p); p += arr;
    s.recs = reinterpret_cast<uint4*>(p);
    p += align256(sizeof(uint4) * (size_t)std::max<int64_t>(n, 1));
    s.cut_range = reinterpret_cast<uint32_t*>(p);
    const size_t range_words = ((size_t)(2 * n_views) + 63) & ~(size_t)63;
    s.range_bytes = sizeof(uint32_t) * range_words;
    s.cut_hist = s.cut_range + range_words;  // keeps the histogram 256-byte aligned
    s.cut_zero_bytes =
        s.range_bytes + sizeof(uint32_t) * (size_t)std::max(n_tiles, 1) * kSaturationBins;
    p += align256(s.cut_zero_bytes);
    s.cutoff = reinterpret_cast<int32_t*>(p);
    p += align256(sizeof(int32_t) * (size_t)std::max(n_tiles, 1));
    s.sort_bytes = align256(radix_sort_scratch_bytes(n, 32, 4, n_views));
    s.sort = p; p += s.sort_bytes;
    s.scan = p; p += align256(scan_scratch_bytes(n));
    s.total = (size_t)(p - static_cast<const char*>(base));
    return s;
}

// The keep table the prepare stage left over its cut histogram, when it
// built one (the emission ignores it without a cutoff).
const uint64_t* cut_keep(const PrepareScratch& p, int tiles_x) {
    return cut_keep_fits(tiles_x) ? reinterpret_cast<const uint64_t*>(p.cut_hist) : nullptr;
}

struct EmitScratch {
    uint32_t* pair_tiles;
    uint32_t* tiles_alt;
    uint32_t* ids_alt;
    int32_t* batch_offsets;  // batches: tile ranges over all views' tiles
    void* sort;
    size_t sort_bytes;
    size_t total;
};

// m pairs over n_views views of n_tiles tiles each.
EmitScratch carve_emit(void* base, int64_t m, int n_tiles, int n_views = 1) {
    EmitScratch s;
    char* p = static_cast<char*>(base);
    const size_t arr = align256(sizeof(uint32_t) * (size_t)std::max<int64_t>(m, 1));
    s.pair_tiles = reinterpret_cast<uint32_t*>(p); p += arr;
    s.tiles_alt = reinterpret_cast<uint32_t*>(p); p += arr;
    s.ids_alt = reinterpret_cast<uint32_t*>(p); p += arr;
    s.batch_offsets = reinterpret_cast<int32_t*>(p);
    if (n_views > 1) p += align256(sizeof(int32_t) * ((size_t)n_tiles * n_views + 1));
    s.sort_bytes = align256(radix_sort_scratch_bytes(m, tile_bits(n_tiles * n_views), 4));
    s.sort = p; p += s.sort_bytes;
    s.total = (size_t)(p - static_cast<char*>(base));
    return s;
}


}  // namespace

void set_error(const std::string& msg) { g_last_error = msg; }

mg_status check_launch(const char* what) {
    g_launches.fetch_add(1, std::memory_order_relaxed);
    const cudaError_t e = cudaGetLastError();
    if (e == cudaSuccess) return MG_OK;
    set_error(std::string(what) + ": " + cudaGetErrorString(e));
    return MG_ERR_CUDA;
}

void* device_symbol_address(const void* symbol, DeviceSymbolCache* cache, std::string* why) {
    int dev = -1;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= DeviceSymbolCache::kMaxDevices) {
        if (why) *why = "no current CUDA device";
        return nullptr;
    }
    std::lock_guard<std::mutex> lock(g_symbol_mu);
    const unsigned long long id = current_context_id();
    if (cache->addr[dev] != nullptr && id != 0ull && cache->ctx_id[dev] == id)
        return cache->addr[dev];
    void* p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, symbol);
    if (e != cudaSuccess || p == nullptr) {
        if (why) *why = std::string("cudaGetSymbolAddress failed: ") + cudaGetErrorString(e);
        return nullptr;
    }
    // the lookup made the device's context current if it was not yet; an id
    // of 0 (driver without context ids) caches nothing and looks up every time
    cache->ctx_id[dev] = current_context_id();
    cache->addr[dev] = cache->ctx_id[dev] != 0ull ? p : nullptr;
    return p;
}

int32_t* device_error_word() {
    return static_cast<int32_t*>(
        device_symbol_address(&g_device_error_word, &g_error_cache, nullptr));
}

}  // namespace mg

using namespace mg;

extern "C" const char* mg_last_error(void) { return g_last_error.c_str(); }

extern "C" int mg_version(void) { return 1; }

extern "C" uint64_t mg_launch_count(void) { return g_launches.load(std::memory_order_relaxed); }

extern "C" mg_status mg_read_device_error(int32_t* code_out, mg_stream_t stream) {
    MG_REQUIRE(code_out != nullptr, "read_device_error: null output");
    int32_t* w = device_error_word();
    if (w == nullptr) return fail(MG_ERR_CUDA, "read_device_error: no device error word");
    cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
    int32_t host = 0;
    if (cudaMemcpyAsync(&host, w, sizeof(int32_t), cudaMemcpyDeviceToHost, s) != cudaSuccess ||
        cudaMemsetAsync(w, 0, sizeof(int32_t), s) != cudaSuccess ||
        cudaStreamSynchronize(s) != cudaSuccess)
        return check_launch("read_device_error");
    *code_out = host;
    return MG_OK;
}

extern "C" mg_status mg_peek_device_error(int64_t* code_dev, mg_stream_t stream) {
    MG_REQUIRE(code_dev != nullptr, "peek_device_error: null output");
    int32_t* w = device_error_word();
    if (w == nullptr) return fail(MG_ERR_CUDA, "peek_device_error: no device error word");
    peek_error_kernel<<<1, 1, 0, reinterpret_cast<cudaStream_t>(stream)>>>(w, code_dev);
    return check_launch("peek_device_error");
}

extern "C" mg_status mg_preprocess_forward(const float* means, const float* quats,
                                           const float* scales, const float* sh_dc,
                                           const float* sh_rest, mg_sh_layout shl,
                                           const float* opacities, const mg_camera* cam,
                                           int32_t sh_degree, int64_t n, float* uv,
                                           float* conic, float* depth, float* rxy,
                                           int32_t* valid, float* color,
                                           mg_stream_t stream) {
    MG_REQUIRE(cam != nullptr, "preprocess_forward: null camera");
    MG_REQUIRE(sh_degree <= 3, "preprocess_forward: sh_degree must be <= 3");
    MG_REQUIRE(cam->width > 0 && cam->height > 0, "preprocess_forward: empty image");
    if (n == 0) return MG_OK;
    MG_REQUIRE(means && quats && scales && opacities && uv && conic && depth && rxy && valid,
               "preprocess_forward: null pointer");
    MG_REQUIRE((reinterpret_cast<uintptr_t>(quats) & 15u) == 0u,
               "preprocess_forward: quats must be 16-byte aligned");
    if (sh_degree >= 0 && sh_dc != nullptr) {
        const bool fused = shl.stride_dc == 16 && shl.stride_rest == 16 && shl.offset_rest == 1;
        const bool split = shl.stride_dc == 1 && shl.stride_rest == 15 && shl.offset_rest == 0;
        MG_REQUIRE(fused || split, "SH must be either one (N,16,3) tensor or (N,1,3)+(N,15,3)");
        MG_REQUIRE(sh_rest != nullptr && color != nullptr, "preprocess_forward: null SH pointer");
    }
    return launch_preprocess_forward(means, quats, scales, sh_dc, sh_rest, shl, opacities, *cam,
                                     sh_degree, n, uv, conic, depth, rxy, valid, color,
                                     reinterpret_cast<cudaStream_t>(stream));
}

extern "C" mg_status mg_preprocess_forward_views(
    const float* means, const float* quats, const float* scales, const float* sh_dc,
    const float* sh_rest, mg_sh_layout shl, const float* opacities, const mg_camera* cams,
    int32_t n_views, int32_t sh_degree, int64_t n, int64_t view_stride, float* uv, float* conic,
    float* depth, float* rxy, int32_t* valid, float* color, float* visibility,
    const mg_step_prologue* prologue, mg_stream_t stream) {
    MG_REQUIRE(n_views >= 0, "preprocess_forward_views: negative view count");
    MG_REQUIRE(sh_degree <= 3, "preprocess_forward_views: sh_degree must be <= 3");
    if (n == 0 || n_views == 0) return MG_OK;
    MG_REQUIRE(cams != nullptr, "preprocess_forward_views: null cameras");
    MG_REQUIRE(view_stride >= n, "preprocess_forward_views: view_stride below n");
    for (int v = 0; v < n_views; ++v)
        MG_REQUIRE(cams[v].width > 0 && cams[v].height > 0,
                   "preprocess_forward_views: empty image");
    if (prologue != nullptr) {
        const mg_step_prologue& p = *prologue;
        MG_REQUIRE(p.log_scales && p.logit_opac && p.act_scales && p.act_opac,
                   "preprocess_forward_views: prologue needs log_scales, logit_opac and the "
                   "activation outputs");
        MG_REQUIRE(p.filter_3d == nullptr || (p.out_scales && p.out_opac),
                   "preprocess_forward_views: prologue with filter_3d needs out_scales/out_opac");
        for (int k = 0; k < 4; ++k)
            MG_REQUIRE(p.zero[k] == nullptr || p.zero_width[k] > 0,
                       "preprocess_forward_views: prologue zero row width must be positive");
    } else {
        MG_REQUIRE(scales && opacities, "preprocess_forward_views: null scales or opacities");
    }
    MG_REQUIRE(means && quats && uv && conic && depth && rxy && valid,
               "preprocess_forward_views: null pointer");
    MG_REQUIRE((reinterpret_cast<uintptr_t>(quats) & 15u) == 0u,
               "preprocess_forward_views: quats must be 16-byte aligned");
    if (sh_degree >= 0 && sh_dc != nullptr) {
        const bool fused = shl.stride_dc == 16 && shl.stride_rest == 16 && shl.offset_rest == 1;
        const bool split = shl.stride_dc == 1 && shl.stride_rest == 15 && shl.offset_rest == 0;
        MG_REQUIRE(fused || split, "SH must be either one (N,16,3) tensor or (N,1,3)+(N,15,3)");
        MG_REQUIRE(sh_rest != nullptr && color != nullptr,
                   "preprocess_forward_views: null SH pointer");
    }
    return launch_preprocess_forward_views(means, quats, scales, sh_dc, sh_rest, shl, opacities,
                                           cams, n_views, sh_degree, n, view_stride, uv, conic,
                                           depth, rxy, valid, color, visibility, prologue,
                                           reinterpret_cast<cudaStream_t>(stream));
}

extern "C" mg_status mg_sh_colour_views(const float* means, const float* sh_dc,
                                        const float* sh_rest, mg_sh_layout shl,
                                        const float* cam_centers, int32_t n_views,
                                        int32_t sh_degree, int64_t n, int64_t view_stride,
                                        const int32_t* valid, float* color,
                                        mg_stream_t stream) {
    MG_REQUIRE(n_views >= 0 && n_views <= 64, "sh_colour_views: 0..64 views");
    MG_REQUIRE(sh_degree >= 0 && sh_degree <= 3, "sh_colour_views: sh_degree must be 0..3");
    if (n == 0 || n_views == 0) return MG_OK;
    MG_REQUIRE(view_stride >= n, "sh_colour_views: view_stride below n");
    MG_REQUIRE(means && sh_dc && sh_rest && cam_centers && valid && color,
               "sh_colour_views: null pointer");
    const bool fused = shl.stride_dc == 16 && shl.stride_rest == 16 && shl.offset_rest == 1;
    const bool split = shl.stride_dc == 1 && shl.stride_rest == 15 && shl.offset_rest == 0;
    MG_REQUIRE(fused || split, "SH must be either one (N,16,3) tensor or (N,1,3)+(N,15,3)");
    return launch_sh_colour_views(means, sh_dc, sh_rest, shl, cam_centers, n_views, sh_degree, n,
                                  view_stride, valid, color,
                                  reinterpret_cast<cudaStream_t>(stream));
}

extern "C" mg_status mg_bin_count(const float* uv, const float* rxy, const float* conic,
                                  const float* opacity, const int32_t* valid, int64_t n,
                                  int32_t width, int32_t height, int32_t tile, int32_t tiles_x,
                                  int32_t tiles_y, int32_t* counts, mg_stream_t stream) {
    MG_REQUIRE(tile > 0 && tiles_x > 0 && tiles_y > 0, "bin_count: bad tiling");
    return launch_bin_count(uv, rxy, conic, opacity, valid, n, width, height, tile, tiles_x,
                            tiles_y, counts, reinterpret_cast<cudaStream_t>(stream));
}

extern "C" mg_status mg_bin_write(const float* uv, const float* rxy, const float* conic,
                                  const float* opacity, const int32_t* valid,
                                  const float* depth, const int32_t* offsets, int64_t total,
                                  int64_t n, int32_t width, int32_t height, int32_t tile,
                                  int32_t tiles_x, int32_t tiles_y, uint64_t* keys,
                                  int32_t* ids, mg_stream_t stream) {
    MG_REQUIRE(tile > 0 && tiles_x > 0 && tiles_y > 0, "bin_write: bad tiling");
    return launch_bin_write(uv, rxy, conic, opacity, valid, depth, offsets, total, n, width,
                            height, tile, tiles_x, tiles_y, keys, ids,
                            reinterpret_cast<cudaStream_t>(stream));
}

extern "C" size_t mg_sort_scratch_bytes(int64_t n, int32_t bits, int32_t key_bytes) {
    return radix_sort_scratch_bytes(n, bits, key_bytes);
}

template <typename K>
static mg_status sort_pairs_impl(K* keys, uint32_t* vals, K* keys_alt, uint32_t* vals_alt,
                                 int64_t n, int32_t bits, void* scratch, size_t scratch_bytes,
                                 mg_stream_t stream) {
    cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
    bool in_alt = false;
    MG_TRY(radix_sort_pairs<K>(keys, vals, keys_alt, vals_alt, n, bits, scratch, scratch_bytes,
                               &in_alt, s));
    if (in_alt) {
        if (cudaMemcpyAsync(keys, keys_alt, sizeof(K) * n, cudaMemcpyDeviceToDevice, s) !=
                cudaSuccess ||
            cudaMemcpyAsync(vals, vals_alt, sizeof(uint32_t) * n, cudaMemcpyDeviceToDevice, s) !=
                cudaSuccess)
            return check_launch("sort result copy");
    }
    return MG_OK;
}

extern "C" mg_status mg_sort_pairs_u32(uint32_t* keys, uint32_t* vals, uint32_t* keys_alt,
                                       uint32_t* vals_alt, int64_t n, int32_t bits,
                                       void* scratch, size_t scratch_bytes,
                                       mg_stream_t stream) {
    return sort_pairs_impl<uint32_t>(keys, vals, keys_alt, vals_alt, n, bits, scratch,
                                     scratch_bytes, stream);
}

extern "C" mg_status mg_sort_pairs_u64(uint64_t* keys, uint32_t* vals, uint64_t* keys_alt,
                                       uint32_t* vals_alt, int64_t n, int32_t bits,
                                       void* scratch, size_t scratch_bytes,
                                       mg_stream_t stream) {
    return sort_pairs_impl<uint64_t>(keys, vals, keys_alt, vals_alt, n, bits, scratch,
                                     scratch_bytes, stream);
}

extern "C" mg_status mg_tile_ranges(const uint32_t* tile_ids, const uint64_t* keys64, int64_t m,
                                    int32_t n_tiles, int32_t* offsets, mg_stream_t stream) {
    MG_REQUIRE(n_tiles > 0 && offsets != nullptr, "tile_ranges: bad arguments");
    MG_REQUIRE(m == 0 || tile_ids != nullptr || keys64 != nullptr, "tile_ranges: no keys");
    return launch_tile_ranges(tile_ids, keys64, m, n_tiles, offsets,
                              reinterpret_cast<cudaStream_t>(stream));
}

extern "C" size_t mg_bin_prepare_scratch_bytes(int64_t n, int32_t n_tiles) {
    if (n < 0 || n_tiles <= 0) return 0;
    return carve_prepare(nullptr, n, n_tiles).total;
}

extern "C" mg_status mg_bin_prepare(const float* uv, const float* rxy, const float* conic,
                                    const float* opacity, const int32_t* valid,
                                    const float* depth, int64_t n, int32_t width, int32_t height,
                                    int32_t tile, int32_t saturation_cut, int64_t* total_dev,
                                    void* scratch, size_t scratch_bytes, mg_stream_t stream) {
    MG_REQUIRE(tile > 0 && width > 0 && height > 0, "bin_prepare: bad tiling");
    MG_REQUIRE(total_dev != nullptr, "bin_prepare: null total");
    MG_REQUIRE(n < ((int64_t)1 << 30) - 1, "bin_prepare: 2^30 - 1 Gaussians or more (sort limit)");
    const int tiles_x = (width + tile - 1) / tile, tiles_y = (height + tile - 1) / tile;
    const PrepareScratch s = carve_prepare(scratch, n, tiles_x * tiles_y);
    MG_REQUIRE(scratch != nullptr && scratch_bytes >= s.total, "bin_prepare: scratch too small");
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    if (saturation_cut &&
        cudaMemsetAsync(s.cut_range, 0, s.cut_zero_bytes, st) != cudaSuccess)
        return check_launch("bin_prepare cut memset");
    MG_TRY(launch_bin_count_depth(uv, rxy, conic, opacity, valid, depth, n, width, height, tile,
                                  tiles_x, tiles_y, s.counts, s.dkeys, s.dvals, s.recs,
                                  saturation_cut ? s.cut_range : nullptr,
                                  saturation_cut ? s.cut_hist : nullptr,
                                  saturation_cut ? s.cutoff : nullptr, BinViews{}, st));
    bool in_alt = false;
    MG_TRY(radix_sort_pairs<uint32_t>(s.dkeys, s.dvals, s.dkeys_alt, s.dvals_alt, n, 32, s.sort,
                                      s.sort_bytes, &in_alt, st, 1, false));
    if (in_alt &&
        cudaMemcpyAsync(s.dvals, s.dvals_alt, sizeof(uint32_t) * n, cudaMemcpyDeviceToDevice,
                        st) != cudaSuccess)
        return check_launch("bin_prepare copy");
    return exclusive_scan_gather(s.counts, s.dvals, n, s.offsets, total_dev, s.scan, st);
}

extern "C" size_t mg_bin_emit_scratch_bytes(int64_t n, int64_t m, int32_t n_tiles) {
    (void)n;
    return carve_emit(nullptr, m, n_tiles).total;
}

extern "C" mg_status mg_bin_emit(const float* uv, const float* rxy, const float* conic,
                                 const float* opacity, int64_t n, int64_t m, int32_t width,
                                 int32_t height, int32_t tile, int32_t saturation_cut,
                                 const void* prepare_scratch, int32_t* gauss_ids,
                                 int32_t* tile_offsets, void* scratch, size_t scratch_bytes,
                                 mg_stream_t stream) {
    MG_REQUIRE(tile > 0 && width > 0 && height > 0, "bin_emit: bad tiling");
    MG_REQUIRE(m >= 0 && m < ((int64_t)1 << 30) - 1,
               "bin_emit: 2^30 - 1 pairs or more (sort limit)");
    MG_REQUIRE(prepare_scratch != nullptr && tile_offsets != nullptr, "bin_emit: null pointer");
    const int tiles_x = (width + tile - 1) / tile, tiles_y = (height + tile - 1) / tile;
    const int n_tiles = tiles_x * tiles_y;
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    if (m == 0) return launch_tile_ranges(nullptr, nullptr, 0, n_tiles, tile_offsets, st);
    MG_REQUIRE(gauss_ids != nullptr, "bin_emit: null gauss_ids");
    const EmitScratch e = carve_emit(scratch, m, n_tiles);
    MG_REQUIRE(scratch != nullptr && scratch_bytes >= e.total, "bin_emit: scratch too small");
    const PrepareScratch p = carve_prepare(prepare_scratch, n, n_tiles);
    uint32_t* ids = reinterpret_cast<uint32_t*>(gauss_ids);
    MG_TRY(launch_bin_emit(uv, rxy, conic, opacity, p.dvals, p.counts, p.offsets, n, m, width,
                           height, tile, tiles_x, tiles_y, p.recs,
                           saturation_cut ? p.cutoff : nullptr, cut_keep(p, tiles_x),
                           e.pair_tiles, ids, BinViews{},
                           st));
    bool in_alt = false;
    MG_TRY(radix_sort_pairs<uint32_t>(e.pair_tiles, ids, e.tiles_alt, e.ids_alt, m,
                                      tile_bits(n_tiles), e.sort, e.sort_bytes, &in_alt, st));
    const uint32_t* sorted_tiles = in_alt ? e.tiles_alt : e.pair_tiles;
    if (in_alt && cudaMemcpyAsync(ids, e.ids_alt, sizeof(uint32_t) * m,
                                  cudaMemcpyDeviceToDevice, st) != cudaSuccess)
        return check_launch("bin_emit copy");
    return launch_tile_ranges(sorted_tiles, nullptr, m, n_tiles, tile_offsets, st);
}

// ------------------------------------------------------ batches of views
//
// The same two stages for every view of a batch (all of one frame size) at
// once: each stage is one launch over all views, and the batch shares one
// depth sort and one tile sort, whose keys carry the view above the depth
// (tile), so each view's order is the one its own sort gives.

namespace {

mg_status check_views(int64_t n, int32_t n_views, int64_t view_stride,
                      int64_t opacity_view_stride, int32_t width, int32_t height, int32_t tile,
                      const char* what) {
    if (tile <= 0 || width <= 0 || height <= 0)
        return fail(MG_ERR_INVALID_ARGUMENT, std::string(what) + ": bad tiling");
    if (n_views < 1 || n_views > 64)
        return fail(MG_ERR_INVALID_ARGUMENT, std::string(what) + ": 1..64 views");
    if (n < 0 || view_stride < n || opacity_view_stride < 0)
        return fail(MG_ERR_INVALID_ARGUMENT, std::string(what) + ": bad view strides");
    if (n * n_views >= ((int64_t)1 << 30) - 1)  // the radix sort's key count limit
        return fail(MG_ERR_CAPACITY, std::string(what) + ": views x Gaussians reach 2^30 - 1");
    return MG_OK;
}

}  // namespace

extern "C" size_t mg_bin_prepare_views_scratch_bytes(int64_t n, int32_t n_views,
                                                     int32_t n_tiles) {
    if (n < 0 || n_views < 1 || n_tiles <= 0) return 0;
    return carve_prepare(nullptr, n, n_tiles, n_views).total;
}

extern "C" mg_status mg_bin_prepare_views(const float* uv, const float* rxy, const float* conic,
                                          const float* opacity, const int32_t* valid,
                                          const float* depth, int64_t n, int32_t n_views,
                                          int64_t view_stride, int64_t opacity_view_stride,
                                          int32_t width, int32_t height, int32_t tile,
                                          int32_t saturation_cut, int64_t* totals_dev,
                                          void* scratch, size_t scratch_bytes,
                                          mg_stream_t stream) {
    MG_TRY(check_views(n, n_views, view_stride, opacity_view_stride, width, height, tile,
                       "bin_prepare_views"));
    MG_REQUIRE(totals_dev != nullptr, "bin_prepare_views: null totals");
    const int tiles_x = (width + tile - 1) / tile, tiles_y = (height + tile - 1) / tile;
    const PrepareScratch s = carve_prepare(scratch, n, tiles_x * tiles_y, n_views);
    MG_REQUIRE(scratch != nullptr && scratch_bytes >= s.total,
               "bin_prepare_views: scratch too small");
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    if (cudaMemsetAsync(s.cut_range, 0, saturation_cut ? s.cut_zero_bytes : s.range_bytes, st) !=
        cudaSuccess)
        return check_launch("bin_prepare_views memset");
    const int64_t rows = n * n_views;
    if (n > 0) {
        MG_REQUIRE(uv && rxy && conic && opacity && valid && depth,
                   "bin_prepare_views: null pointer");
        BinViews bv;
        bv.n_views = n_views;
        bv.in_stride = view_stride;
        bv.opac_stride = opacity_view_stride;
        bv.batch_keys = 1;
        MG_TRY(launch_bin_count_depth(uv, rxy, conic, opacity, valid, depth, n, width, height,
                                      tile, tiles_x, tiles_y, s.counts, s.dkeys, s.dvals, s.recs,
                                      s.cut_range, saturation_cut ? s.cut_hist : nullptr,
                                      saturation_cut ? s.cutoff : nullptr, bv, st));
        bool in_alt = false;
        MG_TRY(radix_sort_pairs<uint32_t>(s.dkeys, s.dvals, s.dkeys_alt, s.dvals_alt, rows, 32,
                                          s.sort, s.sort_bytes, &in_alt, st, n_views, false));
        if (in_alt && cudaMemcpyAsync(s.dvals, s.dvals_alt, sizeof(uint32_t) * rows,
                                      cudaMemcpyDeviceToDevice, st) != cudaSuccess)
            return check_launch("bin_prepare_views copy");
    }
    MG_TRY(exclusive_scan_gather(s.counts, s.dvals, rows, s.offsets, totals_dev + n_views, s.scan,
                                 st));
    if (n == 0)
        return cudaMemsetAsync(totals_dev, 0, sizeof(int64_t) * (n_views + 2), st) == cudaSuccess
                   ? MG_OK
                   : check_launch("bin_prepare_views totals");
    return launch_view_totals(s.offsets, n, n_views, totals_dev, st);
}

extern "C" size_t mg_bin_emit_views_scratch_bytes(int64_t n, int32_t n_views, int64_t m_total,
                                                  int32_t n_tiles) {
    (void)n;
    if (n_views < 1 || n_tiles <= 0 || m_total < 0) return 0;
    return carve_emit(nullptr, m_total, n_tiles, n_views).total;
}

extern "C" mg_status mg_bin_emit_views(const float* uv, const float* rxy, const float* conic,
                                       const float* opacity, int64_t n, int32_t n_views,
                                       int64_t view_stride, int64_t opacity_view_stride,
                                       int64_t m_total, int32_t width, int32_t height,
                                       int32_t tile, int32_t saturation_cut,
                                       const void* prepare_scratch, int32_t* gauss_ids,
                                       int32_t* tile_offsets, void* scratch,
                                       size_t scratch_bytes, mg_stream_t stream) {
    MG_TRY(check_views(n, n_views, view_stride, opacity_view_stride, width, height, tile,
                       "bin_emit_views"));
    if (m_total < 0 || m_total >= ((int64_t)1 << 30) - 1)  // the tile sort's key count limit
        return fail(MG_ERR_CAPACITY, "bin_emit_views: pair count reaches 2^30 - 1");
    MG_REQUIRE(prepare_scratch != nullptr && tile_offsets != nullptr,
               "bin_emit_views: null pointer");
    const int tiles_x = (width + tile - 1) / tile, tiles_y = (height + tile - 1) / tile;
    const int n_tiles = tiles_x * tiles_y;
    MG_REQUIRE((int64_t)n_tiles * n_views < ((int64_t)1 << 31), "bin_emit_views: too many tiles");
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    if (m_total == 0) {
        if (cudaMemsetAsync(tile_offsets, 0, sizeof(int32_t) * (size_t)n_views * (n_tiles + 1),
                            st) != cudaSuccess)
            return check_launch("bin_emit_views memset");
        return MG_OK;
    }
    MG_REQUIRE(gauss_ids != nullptr && uv && rxy && conic && opacity,
               "bin_emit_views: null pointer");
    const EmitScratch e = carve_emit(scratch, m_total, n_tiles, n_views);
    MG_REQUIRE(scratch != nullptr && scratch_bytes >= e.total, "bin_emit_views: scratch too small");
    const PrepareScratch p = carve_prepare(prepare_scratch, n, n_tiles, n_views);
    BinViews bv;
    bv.n_views = n_views;
    bv.in_stride = view_stride;
    bv.opac_stride = opacity_view_stride;
    uint32_t* ids = reinterpret_cast<uint32_t*>(gauss_ids);
    MG_TRY(launch_bin_emit(uv, rxy, conic, opacity, p.dvals, p.counts, p.offsets, n, m_total,
                           width, height, tile, tiles_x, tiles_y, p.recs,
                           saturation_cut ? p.cutoff : nullptr, cut_keep(p, tiles_x),
                           e.pair_tiles, ids, bv, st));
    bool in_alt = false;
    MG_TRY(radix_sort_pairs<uint32_t>(e.pair_tiles, ids, e.tiles_alt, e.ids_alt, m_total,
                                      tile_bits(n_tiles * n_views), e.sort, e.sort_bytes,
                                      &in_alt, st));
    const uint32_t* sorted_tiles = in_alt ? e.tiles_alt : e.pair_tiles;
    if (in_alt && cudaMemcpyAsync(ids, e.ids_alt, sizeof(uint32_t) * m_total,
                                  cudaMemcpyDeviceToDevice, st) != cudaSuccess)
        return check_launch("bin_emit_views copy");
    if (n_views == 1)
        return launch_tile_ranges(sorted_tiles, nullptr, m_total, n_tiles, tile_offsets, st);
    MG_TRY(launch_tile_ranges(sorted_tiles, nullptr, m_total, n_tiles * n_views,
                              e.batch_offsets, st));
    return launch_view_tile_offsets(e.batch_offsets, n_tiles, n_views, tile_offsets, st);
}
