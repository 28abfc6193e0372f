// Internal launchers shared between the translation units of libmg_b200.so.
#pragma once

#include "common.cuh"

namespace mg {

// preprocess_fwd.cu (built with -fmad=false)
mg_status launch_preprocess_forward(const float* means, const float* quats,
                                    const float* scales, const float* sh_dc,
                                    const float* sh_rest, mg_sh_layout shl,
                                    const float* opacities, const mg_camera& cam,
                                    int sh_degree, int64_t n, float* uv, float* conic,
                                    float* depth, float* rxy, int32_t* valid,
                                    float* color, cudaStream_t stream);
mg_status launch_preprocess_forward_views(const float* means, const float* quats,
                                          const float* scales, const float* sh_dc,
                                          const float* sh_rest, mg_sh_layout shl,
                                          const float* opacities, const mg_camera* cams,
                                          int n_views, int sh_degree, int64_t n,
                                          int64_t view_stride, float* uv, float* conic,
                                          float* depth, float* rxy, int32_t* valid,
                                          float* color, float* vis,
                                          const mg_step_prologue* prologue,
                                          cudaStream_t stream);
// The colour of every view for a projection run without it (n_views <= 64;
// cam_centers: n_views x 3 host floats).
mg_status launch_sh_colour_views(const float* means, const float* sh_dc, const float* sh_rest,
                                mg_sh_layout shl, const float* cam_centers, int n_views,
                                int sh_degree, int64_t n, int64_t view_stride,
                                const int32_t* valid, float* color, cudaStream_t stream);
mg_status launch_bin_count(const float* uv, const float* rxy, const float* conic,
                           const float* opacity, const int32_t* valid, int64_t n,
                           int W, int H, int tile, int tiles_x, int tiles_y,
                           int32_t* counts, cudaStream_t stream);
mg_status launch_bin_write(const float* uv, const float* rxy, const float* conic,
                           const float* opacity, const int32_t* valid,
                           const float* depth, const int32_t* offsets, int64_t total,
                           int64_t n, int W, int H, int tile, int tiles_x,
                           int tiles_y, uint64_t* keys, int32_t* ids,
                           cudaStream_t stream);
// A batch of views binned by one launch per stage (blockIdx.y is the view).
// Inputs are view-major with in_stride rows between views (opacity:
// opac_stride, 0 when the views share it); the per-Gaussian outputs are
// compact, view v's rows at v * n, and view v's cut words at cut_range + 2 v,
// its histogram and cutoffs after those of the views before it. With
// batch_keys set, a depth key is the depth's bit pattern minus that of the
// view's smallest visible depth (rows without a pair: 2^24 - 1), and the
// caller sorts each view's n rows as a segment of its own; otherwise the
// single-view keys.
struct BinViews {
    int n_views = 1;
    int64_t in_stride = 0;
    int64_t opac_stride = 0;
    int batch_keys = 0;
};
// cut_range non-null: the range pass runs (relative depth keys); cut_hist
// non-null: the saturation cut runs as well.
mg_status launch_bin_count_depth(const float* uv, const float* rxy, const float* conic,
                                 const float* opacity, const int32_t* valid,
                                 const float* depth, int64_t n, int W, int H, int tile,
                                 int tiles_x, int tiles_y, uint32_t* counts,
                                 uint32_t* dkeys, uint32_t* dvals, uint4* recs,
                                 uint32_t* cut_range, uint32_t* cut_hist, int32_t* cutoff,
                                 const BinViews& bv, cudaStream_t stream);
// Saturation-cut histogram bins per tile (cut_hist holds n_tiles of them;
// cut_range two zeroed words before the call; see preprocess_fwd.cu).
constexpr int kSaturationBins = 64;
// The saturation cut's keep table: per view, tile row and depth bin, the
// bits of the row's tiles whose cutoff bin is not before that bin, in
// cut_keep_stride(tiles_x) 64-bit words (the last one zero). It is written
// over the cut histogram (consumed by then), which holds it when a row has
// at least 4 tiles; launch_bin_count_depth builds it there in that case.
__host__ __device__ inline int cut_keep_stride(int tiles_x) { return (tiles_x + 63) / 64 + 1; }
inline bool cut_keep_fits(int tiles_x) { return tiles_x >= 4; }
mg_status launch_bin_emit(const float* uv, const float* rxy, const float* conic,
                          const float* opacity, const uint32_t* sorted_gid,
                          const uint32_t* counts, const uint32_t* offsets, int64_t n,
                          int64_t m, int W, int H, int tile, int tiles_x, int tiles_y,
                          const uint4* recs, const int32_t* cutoff, const uint64_t* keep,
                          uint32_t* pair_tiles, uint32_t* pair_ids, const BinViews& bv,
                          cudaStream_t stream);
// Batch bookkeeping: per-view pair totals from the scan of the batch's depth
// order (view v's n sorted slots start at v * n; totals[n_views] holds the
// grand total already), and totals[n_views + 1] = 0 (a reserved word).
mg_status launch_view_totals(const uint32_t* offsets, int64_t n, int n_views,
                             int64_t* totals, cudaStream_t stream);
// Per-view tile offsets starting at 0 from the batch's tile ranges
// (global: n_views * n_tiles + 1 entries; local: n_views * (n_tiles + 1)).
mg_status launch_view_tile_offsets(const int32_t* global, int n_tiles, int n_views,
                                   int32_t* local, cudaStream_t stream);

// sort.cu
// Sorts in place between (keys, vals) and (keys_alt, vals_alt); returns in
// *result_in_alt whether the sorted data ended in the alt buffers.
// With segments > 1 (1..256, dividing n), each run of n / segments keys is
// sorted on its own and stays in place. keys_out false: the sorted values
// only (the last pass writes no keys; the result buffer's keys are stale).
template <typename K>
mg_status radix_sort_pairs(K* keys, uint32_t* vals, K* keys_alt, uint32_t* vals_alt,
                           int64_t n, int bits, void* scratch, size_t scratch_bytes,
                           bool* result_in_alt, cudaStream_t stream, int segments = 1,
                           bool keys_out = true);
size_t radix_sort_scratch_bytes(int64_t n, int bits, int key_bytes, int segments = 1);
// Exclusive scan of counts[order[i]] (order may be null: identity) into
// out[i] (u32); writes the 64-bit total to *total_dev.
size_t scan_scratch_bytes(int64_t n);
mg_status exclusive_scan_gather(const uint32_t* counts, const uint32_t* order,
                                int64_t n, uint32_t* out, int64_t* total_dev,
                                void* scratch, cudaStream_t stream);
mg_status launch_tile_ranges(const uint32_t* tile_ids, const uint64_t* keys64,
                             int64_t m, int n_tiles, int32_t* offsets,
                             cudaStream_t stream);

}  // namespace mg
