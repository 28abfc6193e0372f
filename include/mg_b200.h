/*
 * mg_b200.h -- C ABI of the B200 (sm_100a) Gaussian-splatting training path.
 *
 * Every entry point takes plain device pointers, element counts and a CUDA
 * stream, allocates nothing (the caller owns every output and every scratch
 * buffer, sized with the *_scratch_bytes queries), launches on `stream` and
 * returns an mg_status. No entry point synchronises the device except where
 * its comment says so. Reference citations are `path:line` inside the
 * nandometzger/metal-gauss project.
 *
 * Layouts (all fp32 unless stated, row-major, contiguous unless a stride is
 * passed):
 *   means (N,3), quats (N,4) wxyz unnormalised, scales (N,3) linear,
 *   opacities (N,) in [0,1]; SH rows are 3 floats (one RGB triple). SH is
 *   either one (N,16,3) tensor ("fused") or a DC band (N,1,3) plus bands 1+
 *   (N,15,3) ("split"), described by mg_sh_layout exactly as the reference's
 *   `shl` uniform (metal_gauss/csrc/preprocess.metal:30-51).
 *   Per-Gaussian screen-space gradients use one packed record of
 *   MG_G2D_STRIDE floats per Gaussian (see MG_G2D_*), so the rasteriser's
 *   backward can add a whole record with three 16-byte vector atomics.
 */
#ifndef MG_B200_H
#define MG_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* cudaStream_t without pulling in the CUDA headers. */
typedef struct CUstream_st* mg_stream_t;

typedef enum mg_status {
    MG_OK = 0,
    MG_ERR_INVALID_ARGUMENT = 1, /* bad size, layout, tile or null pointer   */
    MG_ERR_CAPACITY = 2,         /* a count exceeds a buffer or a 32-bit index */
    MG_ERR_CUDA = 3,             /* a CUDA launch or runtime call failed      */
    MG_ERR_DEVICE = 4            /* a kernel set the device error word        */
} mg_status;

/* Human-readable reason for the last non-MG_OK status on this host thread. */
const char* mg_last_error(void);

/* Library version, for the loader's sanity check. */
int mg_version(void);

/* Number of kernels this library has launched in this process (all
 * devices); a benchmark reads it before and after its timed region. */
uint64_t mg_launch_count(void);

/* ------------------------------------------------------------------------ */
/* Camera and layout PODs                                                   */
/* ------------------------------------------------------------------------ */

/* One pinhole view. Passed by pointer to host memory and copied into the
 * kernels' parameter space, so no device->host traffic is needed for it
 * (the reference reads viewmat/cam_center on the host in makeParams,
 * metal_gauss/csrc/rasterize.mm:226-242). */
typedef struct mg_camera {
    float viewmat[16];   /* world -> camera, row-major 4x4 (rows 0..2 used) */
    float fx, fy, cx, cy;
    float cam_center[4]; /* xyz = -R^T t, computed by the caller; w unused  */
    int32_t width, height;
    float near_plane, far_plane;
    float blur;          /* 2D dilation added to the covariance diagonal    */
    float max_radius;    /* radius cull, pixels                             */
} mg_camera;

/* SH row addressing, in units of 3-float rows (preprocess.metal:30-51):
 *   fused (N,16,3): {16, 16, 1};   split (N,1,3)+(N,15,3): {1, 15, 0}. */
typedef struct mg_sh_layout {
    int32_t stride_dc;
    int32_t stride_rest;
    int32_t offset_rest;
    int32_t unused;
} mg_sh_layout;

/* Packed per-Gaussian screen-space gradient record (floats). */
#define MG_G2D_STRIDE 12
#define MG_G2D_UV 0      /* d uv.x, d uv.y                       */
#define MG_G2D_OPACITY 2 /* d opacity                            */
#define MG_G2D_ABSUV 3   /* sum over pixels of |d uv| (absgrad)  */
#define MG_G2D_CONIC 4   /* d conic.x, .y, .z                    */
#define MG_G2D_COLOR 8   /* d color.r, .g, .b                    */

/* ------------------------------------------------------------------------ */
/* Preprocess: projection + EWA conic + SnugBox extent + SH colour          */
/* ------------------------------------------------------------------------ */

/* Replaces preprocess_forward (metal_gauss/csrc/rasterize.mm:244-284,
 * kernel metal_gauss/csrc/preprocess.metal:114-221).
 * sh_degree in 0..3; sh_dc/sh_rest may be NULL (with sh_degree < 0) to skip
 * colour entirely, which is the explicit-colour route of render()
 * (metal_gauss/metal_backend.py:449-462). Outputs: uv (N,2), conic (N,3),
 * depth (N,), rxy (N,2), valid (N,) int32, color (N,3). */
mg_status mg_preprocess_forward(
    const float* means, const float* quats, const float* scales,
    const float* sh_dc, const float* sh_rest, mg_sh_layout shl,
    const float* opacities, const mg_camera* cam, int32_t sh_degree, int64_t n,
    float* uv, float* conic, float* depth, float* rxy, int32_t* valid,
    float* color, mg_stream_t stream);

/* The start of a training step, folded into mg_preprocess_forward_views so
 * it costs no launch of its own (the reference forms the activations with
 * torch elementwise ops, train.py:214-229, and clears gradients through
 * autograd). For every row g < n the projection kernel then
 *   - forms act_scales[g] = exp(log_scales[g]) (N,3) and act_opac[g] =
 *     1 / (1 + exp(-logit_opac[g])) (N,) and writes them;
 *   - with filter_3d (N,) given, applies Mip-Splatting's 3D filter to them as
 *     mg_apply_3d_filter does and writes out_scales / out_opac; the filtered
 *     values are projected, otherwise the activations are;
 *   - sets rows g of each non-NULL zero[k] (row width zero_width[k] floats)
 *     to 0: the gradient rows the step accumulates into;
 *   - WRITES the visibility count (instead of adding to it);
 * and *zero_word (the loss accumulator) is set to 0 once. */
typedef struct mg_step_prologue {
    const float* log_scales;
    const float* logit_opac;
    const float* filter_3d;
    float* act_scales;
    float* act_opac;
    float* out_scales;
    float* out_opac;
    float* zero[4];
    int32_t zero_width[4];
    float* zero_word;
} mg_step_prologue;

/* Training-engine form of mg_preprocess_forward for the views of one batch
 * (same math per view, preprocess.metal:114-221): each Gaussian's
 * parameters and SH rows are read once and projected and coloured for all
 * n_views cameras `cams`. View v's outputs start at row v * view_stride
 * (view_stride >= n) of uv, conic, depth, rxy, valid and color, laid out as
 * in mg_preprocess_forward. With `visibility` given, the number of views in
 * which a Gaussian is valid is ADDED to visibility[g] (float). With
 * `prologue` given (may be NULL), `scales` and `opacities` are ignored and
 * the step prologue above runs first. No reference counterpart: the
 * reference projects one camera per call. */
mg_status mg_preprocess_forward_views(
    const float* means, const float* quats, const float* scales,
    const float* sh_dc, const float* sh_rest, mg_sh_layout shl,
    const float* opacities, const mg_camera* cams, int32_t n_views,
    int32_t sh_degree, int64_t n, int64_t view_stride, float* uv, float* conic,
    float* depth, float* rxy, int32_t* valid, float* color, float* visibility,
    const mg_step_prologue* prologue, mg_stream_t stream);

/* The SH colour half of mg_preprocess_forward_views (preprocess.metal:
 * 203-221), for a projection that ran with sh_dc = NULL and sh_degree = -1:
 * color row v * view_stride + g = the SH colour of Gaussian g seen from
 * camera centre v (+0.5, clamped at 0), or 0 where valid (from that
 * projection) is 0. cam_centers: n_views x 3 host floats, n_views <= 64.
 * The arithmetic is the fused projection's, so the colours are identical.
 * The training engine uses it on several GPUs, so that the next step's
 * projection and binning can run while the SH rows are still being
 * gathered. No reference counterpart. */
mg_status mg_sh_colour_views(const float* means, const float* sh_dc, const float* sh_rest,
                             mg_sh_layout shl, const float* cam_centers, int32_t n_views,
                             int32_t sh_degree, int64_t n, int64_t view_stride,
                             const int32_t* valid, float* color, mg_stream_t stream);

/* Replaces preprocess_backward (rasterize.mm:286-327, kernel
 * preprocess.metal:223-411). The incoming gradients are read through row
 * strides (in floats) so they may point into a packed MG_G2D record
 * (stride MG_G2D_STRIDE) or into plain (N,2)/(N,3) tensors. d_color may be
 * NULL (explicit colours: SH branch skipped, d_sh untouched).
 * Outputs are overwritten: d_means (N,3), d_quats (N,4), d_scales (N,3),
 * d_sh_dc / d_sh_rest in the layout `shl` (may alias, as the fused layout
 * does). */
mg_status mg_preprocess_backward(
    const float* means, const float* quats, const float* scales,
    const float* sh_dc, const float* sh_rest, mg_sh_layout shl,
    const float* d_uv, int64_t d_uv_stride,
    const float* d_conic, int64_t d_conic_stride,
    const float* d_color, int64_t d_color_stride,
    const int32_t* valid, const mg_camera* cam, int32_t sh_degree, int64_t n,
    float* d_means, float* d_quats, float* d_scales,
    float* d_sh_dc, float* d_sh_rest, mg_stream_t stream);

/* Training-engine form of mg_preprocess_backward (same math,
 * preprocess.metal:223-411): reads the rasteriser's packed record grad2d
 * (N, MG_G2D_STRIDE) directly and ADDS one view's gradients into the
 * trainer's parameter storage, with the activation chain of train.py:221-222
 * applied in-kernel:
 *   d_log_scales += d_scales * scales,  d_logit_opac += d_opacity * op (1-op).
 * scales/opacities are the activated values; SH uses the split layout
 * (N,1,3) + (N,15,3). Rows whose colour gradient is zero add nothing to the
 * SH gradients and rows with valid == 0 add nothing to the scale/quaternion
 * gradients, so rows a view never touched cost only their reads. */
mg_status mg_preprocess_backward_accumulate(
    const float* means, const float* quats, const float* scales,
    const float* opacities, const float* sh_dc, const float* sh_rest,
    const float* grad2d, const int32_t* valid, const mg_camera* cam,
    int32_t sh_degree, int64_t n, float* d_means, float* d_quats,
    float* d_log_scales, float* d_logit_opac, float* d_sh_dc,
    float* d_sh_rest, const float* color, float* dpre_out,
    mg_stream_t stream);

/* The projection half of mg_preprocess_backward_accumulate (deferred SH
 * form, preprocess.metal:265-411) for the views of one batch: per Gaussian
 * the parameters are read once and the views' adjoints are summed before
 * they are ADDED to d_means, d_quats, d_log_scales and d_logit_opac
 * (activation chain as in mg_preprocess_backward_accumulate). View v's
 * grad2d records (MG_G2D_STRIDE floats), valid flags and forward colours
 * start at row v * view_stride; dpre_out row v * view_stride + g receives
 * view v's colour gradient gated by colour > 0, the input of
 * mg_sh_backward_views. With filter_3d (N,) given, scales and opacities are
 * the activations BEFORE Mip-Splatting's 3D filter (mipfilter.py:79-93): the
 * forward projected mg_apply_3d_filter's outputs, and the gradients are
 * carried back through the filter (train.py:221-227 with filter_3d constant).
 * grad2d must be 16-byte aligned (records are read as three 16-byte words).
 * No reference counterpart. */
mg_status mg_preprocess_backward_views(
    const float* means, const float* quats, const float* scales,
    const float* opacities, const float* grad2d, const int32_t* valid,
    const float* color, const mg_camera* cams, int32_t n_views, int64_t n,
    int64_t view_stride, const float* filter_3d, float* d_means, float* d_quats,
    float* d_log_scales, float* d_logit_opac, float* dpre_out, mg_stream_t stream);

/* Deferred SH gradient of a batch of views, once per step. With dpre_out
 * given, mg_preprocess_backward_accumulate skips its SH branch and instead
 * writes dpre_out (N,3) = the view's colour gradient where the forward colour
 * `color` is > 0 (the ReLU gate of preprocess.metal:256-262; colour > 0 iff the
 * pre-clamp colour is > 0). This entry point then evaluates the SH adjoint of
 * all n_views views together: d_sh (split layout, OVERWRITTEN) = sum over
 * views of B(dir_v) x dpre_v, and d_means += the view-direction term, reading
 * the coefficients once instead of once per view. cam_centers: n_views x 3
 * host floats; dpre: view v's rows start at row v * view_stride (>= N) of a
 * device array of 3-float rows; n_views <= 64. */
mg_status mg_sh_backward_views(const float* means, const float* sh_dc,
                               const float* sh_rest, int32_t sh_degree,
                               int64_t n, const float* cam_centers,
                               const float* dpre, int32_t n_views,
                               int64_t view_stride,
                               float* d_means, float* d_sh_dc,
                               float* d_sh_rest, mg_stream_t stream);

/* ------------------------------------------------------------------------ */
/* Binning: exact ellipse-vs-tile test, keys, sort, per-tile ranges         */
/* ------------------------------------------------------------------------ */

/* Replaces bin_count (rasterize.mm:485-497; binning.metal:92-104):
 * counts[g] = number of tiles whose rectangle the Gaussian's alpha >= 1/255
 * level set reaches (0 for invalid rows). */
mg_status mg_bin_count(
    const float* uv, const float* rxy, const float* conic,
    const float* opacity, const int32_t* valid, int64_t n,
    int32_t width, int32_t height, int32_t tile, int32_t tiles_x,
    int32_t tiles_y, int32_t* counts, mg_stream_t stream);

/* Replaces bin_write (rasterize.mm:499-516; binning.metal:106-120):
 * keys[offsets[g] + k] = (tile_id << 32) | bits(depth[g]), ids[...] = g,
 * tiles in row-major order per Gaussian. `total` is the key capacity. */
mg_status mg_bin_write(
    const float* uv, const float* rxy, const float* conic,
    const float* opacity, const int32_t* valid, const float* depth,
    const int32_t* offsets, int64_t total, int64_t n,
    int32_t width, int32_t height, int32_t tile, int32_t tiles_x,
    int32_t tiles_y, uint64_t* keys, int32_t* ids, mg_stream_t stream);

/* Stable LSD onesweep radix sort of (key, value) pairs on the low `bits`
 * bits of the key. Replaces torch.argsort(keys) (metal_backend.py:256), which
 * the reference uses because MPS exposes no radix sort. keys_alt/vals_alt are
 * ping-pong buffers of n elements; the sorted result is left in keys/vals.
 * scratch must hold mg_sort_scratch_bytes(n, bits, key_bytes) bytes. The
 * decoupled look-back is bounded; a timeout sets the device error word. */
size_t mg_sort_scratch_bytes(int64_t n, int32_t bits, int32_t key_bytes);
mg_status mg_sort_pairs_u32(uint32_t* keys, uint32_t* vals,
                            uint32_t* keys_alt, uint32_t* vals_alt,
                            int64_t n, int32_t bits, void* scratch,
                            size_t scratch_bytes, mg_stream_t stream);
mg_status mg_sort_pairs_u64(uint64_t* keys, uint32_t* vals,
                            uint64_t* keys_alt, uint32_t* vals_alt,
                            int64_t n, int32_t bits, void* scratch,
                            size_t scratch_bytes, mg_stream_t stream);

/* Allocation-free form of mg_sort_pairs_u32 (this entry point has no
 * counterpart in the reference). For callers that cannot allocate device
 * memory -- a host that owns every byte of the GPU through its own pool and
 * forbids libraries from calling cudaMalloc/cudaFree (those calls synchronise
 * the device and fragment the pool), or a caller whose memory is already
 * fully handed to another allocator such as PyTorch's caching allocator.
 * The caller passes only the pairs to sort; the ping-pong buffers,
 * histograms and look-back words live in one static device array of
 * MG_SORT_NOALLOC_SCRATCH_BYTES inside the library, which every GPU that
 * loads the library holds until the process exits.
 *   - n must be <= MG_SORT_NOALLOC_MAX_N; larger n is rejected with
 *     MG_ERR_CAPACITY and a message, nothing is launched.
 *   - The first call on a device looks up the array's device address for that
 *     device (cudaGetSymbolAddress with that device current); make that first
 *     call before any stream capture. The address is cached per device and
 *     context: after a device reset the next call looks it up again.
 *   - Every call on a device shares the one array, so calls whose work
 *     overlaps on the GPU (different streams, or different host threads)
 *     race and corrupt each other's results: serialise them. The array keeps
 *     the last call's contents; each call clears the parts that must start at
 *     zero itself.
 *   - Calls no cudaMalloc, cudaFree or allocating library routine. */
#define MG_SORT_NOALLOC_MAX_N (1 << 20)
/* 8 MiB of ping-pong buffers + 1 MiB of look-back words + histograms */
#define MG_SORT_NOALLOC_SCRATCH_BYTES 9441536
mg_status mg_sort_pairs_u32_noalloc(uint32_t* keys, uint32_t* vals, int64_t n,
                                    int32_t bits, mg_stream_t stream);

/* Replaces `keys[order] >> 32` + torch.searchsorted (metal_backend.py:
 * 257-260): offsets[t] = first index whose tile id is >= t, offsets[T] = m.
 * `tile_ids` are the sorted tile ids (u32), or NULL with `keys64` set to the
 * sorted 64-bit keys, whose high word is the tile id. */
mg_status mg_tile_ranges(const uint32_t* tile_ids, const uint64_t* keys64,
                         int64_t m, int32_t n_tiles, int32_t* offsets,
                         mg_stream_t stream);

/* The whole binning of one view in the two-stage form, replacing
 * build_tile_lists_metal (metal_backend.py:217-285):
 *   stage A (mg_bin_prepare): per-Gaussian tile counts; stable depth sort of
 *     all Gaussians (invalid ones last); exclusive scan of the counts in
 *     depth order. Writes the pair total to *total_dev (device int64).
 *   stage B (mg_bin_emit): the caller reads the total (the one host sync of
 *     the reference, metal_backend.py:247), then this writes every
 *     (tile, Gaussian) pair in depth order, stably sorts the pairs by tile id
 *     and extracts the per-tile ranges.
 * The result equals a stable sort on (tile_id << 32 | depth_bits) keys
 * emitted in Gaussian order: within a tile, front to back, equal depths by
 * Gaussian index. Scratch sizes come from the two queries.
 *
 * saturation_cut = 1 (both calls, the same value) drops, per tile, the pairs
 * behind the depth at which Gaussians covering the whole tile have provably
 * driven every pixel's transmittance below the rasteriser's 1e-4 stop
 * (a lower bound of their alpha over the tile's pixel centres, summed as
 * optical depth over 64 log-spaced depth bins, with a margin). The lists are
 * then a front-to-back prefix of the full ones: rasterisation results are
 * unchanged, but the lists no longer equal the reference's. 0 gives the
 * reference's lists. n and the pair total must stay below 2^30 - 1 (the
 * radix sort's key count). */
size_t mg_bin_prepare_scratch_bytes(int64_t n, int32_t n_tiles);
mg_status mg_bin_prepare(
    const float* uv, const float* rxy, const float* conic,
    const float* opacity, const int32_t* valid, const float* depth, int64_t n,
    int32_t width, int32_t height, int32_t tile, int32_t saturation_cut,
    int64_t* total_dev, void* scratch, size_t scratch_bytes, mg_stream_t stream);
size_t mg_bin_emit_scratch_bytes(int64_t n, int64_t m, int32_t n_tiles);
mg_status mg_bin_emit(
    const float* uv, const float* rxy, const float* conic,
    const float* opacity, int64_t n, int64_t m,
    int32_t width, int32_t height, int32_t tile, int32_t saturation_cut,
    const void* prepare_scratch, int32_t* gauss_ids, int32_t* tile_offsets,
    void* scratch, size_t scratch_bytes, mg_stream_t stream);

/* The two binning stages for a batch of 1..64 views of one frame size in one
 * call each (no reference counterpart: the reference bins each view inside
 * its own render call, metal_backend.py:239-262). The inputs are view-major
 * (view v's Gaussian g at row v * view_stride + g, opacity at
 * v * opacity_view_stride + g, 0 when the views share it); n * n_views and
 * the batch's pair total must stay below 2^30 - 1 (the radix sort's key
 * count; the per-view calls take more pairs per view).
 *   mg_bin_prepare_views writes n_views + 2 int64 words to totals_dev: each
 *     view's pair total, the batch's total, and a reserved word (0). One
 *     depth sort orders the whole batch, each view's rows on their own
 *     (keys relative to the view's nearest visible depth: any range fits).
 *   mg_bin_emit_views takes the batch total m_total and writes the pairs of
 *     view v to gauss_ids[base_v, base_v + m_v) (base_v: the totals of the
 *     views before v) and its tile offsets, starting at 0 as mg_bin_emit's,
 *     to tile_offsets[v * (n_tiles + 1) ...]. Each view's lists equal the
 *     lists mg_bin_prepare / mg_bin_emit give for that view alone. */
size_t mg_bin_prepare_views_scratch_bytes(int64_t n, int32_t n_views, int32_t n_tiles);
mg_status mg_bin_prepare_views(
    const float* uv, const float* rxy, const float* conic, const float* opacity,
    const int32_t* valid, const float* depth, int64_t n, int32_t n_views,
    int64_t view_stride, int64_t opacity_view_stride, int32_t width, int32_t height,
    int32_t tile, int32_t saturation_cut, int64_t* totals_dev, void* scratch,
    size_t scratch_bytes, mg_stream_t stream);
size_t mg_bin_emit_views_scratch_bytes(int64_t n, int32_t n_views, int64_t m_total,
                                       int32_t n_tiles);
mg_status mg_bin_emit_views(
    const float* uv, const float* rxy, const float* conic, const float* opacity, int64_t n,
    int32_t n_views, int64_t view_stride, int64_t opacity_view_stride, int64_t m_total,
    int32_t width, int32_t height, int32_t tile, int32_t saturation_cut,
    const void* prepare_scratch, int32_t* gauss_ids, int32_t* tile_offsets, void* scratch,
    size_t scratch_bytes, mg_stream_t stream);

/* ------------------------------------------------------------------------ */
/* Rasterisation                                                            */
/* ------------------------------------------------------------------------ */

/* The rasterisers read one 48-byte record per splat (12 floats, 16-byte
 * aligned), packed from the reference's separate uv / conic / opacity /
 * colour arrays by mg_pack_splats. The record layout is private to the
 * library. */
#define MG_SPLAT_FLOATS 12
#define MG_SPLAT_BYTES 48

/* List entries between two forward checkpoints; the backward splits every
 * warp block's walk into segments of this many entries. */
#define MG_RASTER_SEGMENT 256

/* Packs n splats into `splats` (n * MG_SPLAT_BYTES, 16-byte aligned). The
 * reference's rasterize_forward / rasterize_backward (rasterize.mm:79-194)
 * take uv (N,2), conic (N,3), opacity (N,), color (N,3); a caller of this ABI
 * packs them once per view and hands the record array to both passes.
 * grad2d_zero (may be NULL; 16-byte aligned, N x MG_G2D_STRIDE floats) is set
 * to zero in the same pass: the gradient records mg_rasterize_backward of
 * this view accumulates into. */
mg_status mg_pack_splats(const float* uv, const float* conic, const float* opacity,
                         const float* color, int64_t n, void* splats, float* grad2d_zero,
                         mg_stream_t stream);

/* Bytes of rasteriser scratch for one view of width x height with `m`
 * (tile, splat) pairs: work counters, the tile order, per-warp-block walk
 * lengths, the backward's work items and the forward's checkpoints. */
size_t mg_raster_scratch_bytes(int32_t width, int32_t height, int32_t tile, int64_t m);

/* Replaces rasterize_forward (rasterize.mm:79-113; rasterize.metal:61-167).
 * splats from mg_pack_splats, gauss_ids / tile_offsets from binning with m =
 * tile_offsets[n_tiles] pairs, tile in {8, 12, 16, 32}. Outputs rgb (H,W,3),
 * alpha (H,W), final transmittance T (H,W), stop index (H,W) int32.
 * background: NULL, or 3 host floats blended as rgb + max(1-alpha,0)*bg,
 * which is metal_backend.py:539-541 folded into the kernel. tile_work
 * (optional, n_tiles ints) receives each tile's walk length, the largest stop
 * index minus the tile's first index. scratch (mg_raster_scratch_bytes,
 * 16-byte aligned) receives the state the backward of the same view reads
 * when called with segmented = 1; keep it unchanged until then. */
mg_status mg_rasterize_forward(
    const void* splats, const int32_t* gauss_ids, const int32_t* tile_offsets, int64_t m,
    int32_t width, int32_t height, int32_t tile, int32_t tiles_x,
    const float* background, float* out_rgb, float* out_alpha, float* out_T,
    int32_t* out_stop, int32_t* tile_work, void* scratch, size_t scratch_bytes,
    mg_stream_t stream);

/* out_T and out_stop may both be NULL: a forward-only render (the viewer's
 * and render_path's callers, viewer.py:477-485), which writes neither them
 * nor the backward's checkpoints; the scratch is then only workspace. */

/* Mip-Splatting's 2D antialias compensation of opacity, applied before
 * binning as metal_backend.py:506-511 does: out[i] = opacity[i] *
 * sqrt(clamp(det_before / det_after, 0, 1)) with det_before the determinant
 * of the 2D covariance before the `blur` (0.3 px) dilation, recovered from
 * the dilated conic (metal_backend.py:367-393). */
mg_status mg_antialias_opacity(const float* conic, const float* opacity, int64_t n,
                               float blur, float* out, mg_stream_t stream);

/* Adjoint of mg_antialias_opacity (the autograd of metal_backend.py:506-511
 * through antialias_scale, :367-393): from grad_out (N,) = d loss / d out,
 * d_conic (N,3) and d_opacity (N,) are OVERWRITTEN. */
mg_status mg_antialias_opacity_backward(const float* conic, const float* opacity,
                                        const float* grad_out, int64_t n, float blur,
                                        float* d_conic, float* d_opacity, mg_stream_t stream);

/* The training engine's forms for a batch of views (no reference
 * counterpart; the reference applies the compensation per render call):
 * view v's conics, outputs and gradient records at rows v * view_stride,
 * the opacities shared. mg_antialias_opacity_views writes the compensated
 * opacities; mg_antialias_grad2d_views applies the adjoint IN PLACE to
 * gradient records (MG_G2D_*): d opacity against the compensated opacity
 * becomes d opacity against `opacity`, and the compensation's conic term is
 * added to d conic. */
mg_status mg_antialias_opacity_views(const float* conic, const float* opacity, int64_t n,
                                     int32_t n_views, int64_t view_stride, float blur,
                                     float* out, mg_stream_t stream);
mg_status mg_antialias_grad2d_views(const float* conic, const float* opacity, int64_t n,
                                    int32_t n_views, int64_t view_stride, float blur,
                                    float* grad2d, mg_stream_t stream);

/* Replaces rasterize_backward (rasterize.mm:147-194; rasterize.metal:
 * 173-340). grad2d (N, MG_G2D_STRIDE) is ACCUMULATED into (zero it first for
 * a fresh gradient). background as in the forward: the blend's adjoint is
 * applied in-kernel, which needs the forward's alpha (H,W) (grad_alpha may be
 * NULL for zero). want_absgrad adds per-pixel |d uv| into MG_G2D_ABSUV.
 * segmented = 1: `scratch` is the one the forward of this view filled; each
 * warp block's walk is split into MG_RASTER_SEGMENT-entry segments that start
 * from the forward's checkpoints (needs out_rgb and out_alpha of that
 * forward). segmented = 0: scratch is workspace only and every block walks
 * its whole list (out_rgb unused; out_alpha only with a background). */
mg_status mg_rasterize_backward(
    const void* splats, const int32_t* gauss_ids, const int32_t* tile_offsets, int64_t m,
    const float* out_rgb, const float* out_alpha, const float* final_T,
    const int32_t* stop, const float* grad_rgb, const float* grad_alpha,
    int32_t width, int32_t height, int32_t tile, int32_t tiles_x,
    const float* background, int32_t want_absgrad, int64_t n, float* grad2d,
    int32_t segmented, void* scratch, size_t scratch_bytes, mg_stream_t stream);

/* Tile ids ordered by decreasing work: work[t] when `work` is given (e.g.
 * the forward's tile_work), else the list
 * length tile_offsets[t+1] - tile_offsets[t]. Bucketed by powers of two
 * (order inside a bucket is unspecified; results do not depend on it). */
mg_status mg_tile_order(const int32_t* tile_offsets, const int32_t* work,
                        int32_t n_tiles, int32_t* order, mg_stream_t stream);

/* Replaces pack_intersections (rasterize.mm:115-145; rasterize.metal:
 * 358-376): gathers (u, v, opacity), conic and colour by sorted id. */
mg_status mg_pack_intersections(
    const float* uv, const float* conic, const float* opacity,
    const float* color, const int32_t* gauss_ids, int64_t m,
    float* p_xy_opac, float* p_conic, float* p_rgb, mg_stream_t stream);

/* ------------------------------------------------------------------------ */
/* Optimisers                                                               */
/* ------------------------------------------------------------------------ */

/* Replaces adam_step (rasterize.mm:329-360; adam.metal:25-42): one in-place
 * torch.optim.Adam step, eps added after dividing by sqrt(bc2). bc1 and
 * sqrt_bc2 are computed by the caller in double, as torch does. */
mg_status mg_adam_step(float* p, const float* g, float* m, float* v,
                       int64_t n, float lr, float b1, float b2, float eps,
                       float bc1, float sqrt_bc2, mg_stream_t stream);

/* SelectiveAdam row update (metal_gauss/selective_adam.py:116-186): for each
 * row r with visible[r] != 0, k = steps[r] + 1,
 *   m = b1 m + (1-b1) g;  v = b2 v + (1-b2) g^2;
 *   p -= lr * sqrt(1-b2^k) / (1-b1^k) * m / (sqrt(v) + eps),
 * over the row's `row_width` contiguous elements; rows not visible are left
 * untouched. `rows` may exceed the mask length `n_visible` (preallocated
 * capacity rows, selective_adam.py:47-59, are treated as invisible).
 * steps[r] is advanced by mg_selective_adam_advance_steps afterwards. */
mg_status mg_selective_adam_step(float* p, const float* g, float* m, float* v,
                                 const float* steps, const uint8_t* visible,
                                 int64_t n_visible, int64_t rows,
                                 int64_t row_width, float lr, float b1,
                                 float b2, float eps, mg_stream_t stream);
mg_status mg_selective_adam_advance_steps(float* steps, const uint8_t* visible,
                                          int64_t n_visible, int64_t rows,
                                          mg_stream_t stream);

/* Adam over several parameter segments of one flat buffer in ONE launch
 * (the training engine keeps all Gaussian parameters in one allocation).
 * Segment s covers elements [offset, offset + rows * width) of p/g/m/v and
 * uses learning rate lr. With visible_count == NULL this is dense
 * torch.optim.Adam at scalar step `step` (adam.metal:25-42). Otherwise it is
 * SelectiveAdam (selective_adam.py:116-186): only rows r with
 * visible_count[r] > 0 are updated, with the shared per-row step count
 * steps[r] + 1, and steps is advanced for those rows (all `rows` of them)
 * afterwards. A segment may cover only an element range (a data-parallel
 * rank's chunk of the flat buffer; the row of element e is e / width). At
 * most MG_MAX_ADAM_SEGMENTS segments. */
#define MG_MAX_ADAM_SEGMENTS 8
typedef struct mg_adam_segment {
    int64_t offset;      /* first element of the segment's row 0          */
    int32_t width;       /* elements per row                               */
    float lr;
    int64_t elem_begin;  /* update elements [elem_begin, elem_end) of the  */
    int64_t elem_end;    /* segment; elem_end == 0 means all rows * width  */
} mg_adam_segment;
/* row_scratch (selective mode, optional): `rows` floats the entry point uses
 * to form each visible row's bias correction once instead of once per
 * thread; NULL forms it in place. flags: 0, or a step's update split over
 * several calls (e.g. one per parameter group, on different streams):
 *   MG_ADAM_KEEP_STEPS: do not advance `steps` (another call of the same step
 *     does);
 *   MG_ADAM_ROW_FACTORS_READY: row_scratch already holds this step's factors
 *     (formed by an earlier call of the same step); neither form them again
 *     nor read visible_count's values. */
#define MG_ADAM_ROW_FACTORS_READY 1
#define MG_ADAM_KEEP_STEPS 2
mg_status mg_adam_multi(float* p, const float* g, float* m, float* v,
                        int64_t rows, const mg_adam_segment* segments,
                        int32_t n_segments, float b1, float b2, float eps,
                        const float* visible_count, float* steps, int64_t step,
                        float* row_scratch, int32_t flags, mg_stream_t stream);

/* The MCMC regularisers of the reference's training loss (train.py:393-398):
 *   loss += c_opac * mean(sigmoid(logit_opac[:n])) + c_scale * mean(exp(log_scales[:n, 0..2]))
 * where the caller folds the weights (--opac-reg / --scale-reg, 0.01 each) and
 * the ramp aux = max(0, 1 - step / (0.9 steps)) into c_*. ADDS
 * c_opac / n * s (1 - s) to d_logit[i] and c_scale / (3 n) * exp(log_scales)
 * to d_log_scales[i, j], and the loss value to *loss_dev. scratch: 16 bytes. */
mg_status mg_regularizer_grad(const float* logit_opac, const float* log_scales, int64_t n,
                              float c_opac, float c_scale, float* d_logit,
                              float* d_log_scales, float* loss_dev, void* scratch,
                              size_t scratch_bytes, mg_stream_t stream);

/* ------------------------------------------------------------------------ */
/* SSIM (11-tap separable Gaussian, zero padding) and the training loss     */
/* ------------------------------------------------------------------------ */

/* The reference's five SSIM kernels, same layouts (ssim.metal:23-188,
 * bridge rasterize.mm:362-461): x, y are (H,W,3); stacks are (15,H,W) with
 * channels 0-2 x, 3-5 y, 6-8 xx, 9-11 yy, 12-14 xy; w is 11 floats. */
mg_status mg_ssim_stack_blur_h(const float* x, const float* y, const float* w,
                               int32_t height, int32_t width, float* out,
                               mg_stream_t stream);
mg_status mg_ssim_blur15(const float* src, const float* w, int32_t dir,
                         int32_t height, int32_t width, float* dst,
                         mg_stream_t stream);
mg_status mg_ssim_tail_forward(const float* b, int32_t height, int32_t width,
                               float* out, mg_stream_t stream);
mg_status mg_ssim_tail_backward(const float* b, const float* gout,
                                int32_t height, int32_t width, float* gb,
                                mg_stream_t stream);
mg_status mg_ssim_chain_backward(const float* x, const float* y,
                                 const float* d_stack, int32_t height,
                                 int32_t width, float* d_x, mg_stream_t stream);

/* Fused training loss for one view, forward and backward in one pass:
 *   loss = w_l1 * mean|x - y| + w_ssim * (1 - SSIM(x, y))
 * (train.py:389-393 with the defaults w_l1 = 0.8, w_ssim = 0.2), scaled by
 * `scale` (e.g. 1/V for a mean over V views). Writes grad_x (H,W,3) =
 * scale * dloss/dx and ADDS scale*loss into *loss_dev (device float).
 * x, y (H,W,3); w is 11 floats. */
size_t mg_l1_ssim_scratch_bytes(int32_t height, int32_t width);
mg_status mg_l1_ssim_loss(const float* x, const float* y, const float* w,
                          int32_t height, int32_t width, float w_l1,
                          float w_ssim, float scale, float* grad_x,
                          float* loss_dev, void* scratch, size_t scratch_bytes,
                          mg_stream_t stream);

/* mg_l1_ssim_loss with an 8-bit target image y (H,W,3) uint8, read as
 * y / 255 in float32 with IEEE division -- the reference's trainer holds its
 * images as bytes and divides them by 255 (`v.image.to(device).float() /
 * 255.0`, train.py:385) -- so a trainer can keep its targets as the bytes it
 * loaded and copy a quarter of the bytes per step. (torch's CUDA division by
 * a scalar multiplies by the rounded reciprocal instead, which can differ in
 * the last bit.) */
mg_status mg_l1_ssim_loss_u8(const float* x, const uint8_t* y, const float* w,
                             int32_t height, int32_t width, float w_l1, float w_ssim,
                             float scale, float* grad_x, float* loss_dev, void* scratch,
                             size_t scratch_bytes, mg_stream_t stream);

/* ------------------------------------------------------------------------ */
/* Mip-Splatting 3D filter                                                  */
/* ------------------------------------------------------------------------ */

/* Replaces compute_3d_filter (metal_gauss/mipfilter.py:30-76): per Gaussian,
 * the smallest camera depth among the n_views cameras (any number; 64 per
 * kernel launch, the running minimum carried between launches) in whose frame,
 * widened by `margin` on every side, the mean projects in front of
 * `near_plane`; Gaussians no camera sees take the largest such depth of any
 * Gaussian (all take 1 when none is seen); then depth / max focal * sqrt(0.2).
 * Only viewmat, fx, fy, cx, cy, width and height of `cams` are read; they
 * travel in the launches' parameters, so nothing is copied to the device and
 * nothing synchronises. */
size_t mg_compute_3d_filter_scratch_bytes(void);
mg_status mg_compute_3d_filter(const float* means, int64_t n, const mg_camera* cams,
                               int32_t n_views, float near_plane, float margin,
                               float* filter_out, void* scratch, size_t scratch_bytes,
                               mg_stream_t stream);

/* Replaces apply_3d_filter (mipfilter.py:79-93): out_scales =
 * sqrt(scales^2 + f^2), out_opacities = opacities * sqrt(clamp(prod(scales^2)
 * / prod(scales^2 + f^2), 0, 1)); scales (N,3), opacities and filter_3d (N,). */
mg_status mg_apply_3d_filter(const float* scales, const float* opacities,
                             const float* filter_3d, int64_t n, float* out_scales,
                             float* out_opacities, mg_stream_t stream);

/* The adjoint of mg_apply_3d_filter (the autograd of mipfilter.py:79-93 with
 * filter_3d constant): d_scales (N,3) and d_opacities (N,) OVERWRITTEN from
 * the gradients of its two outputs. */
mg_status mg_apply_3d_filter_backward(const float* scales, const float* opacities,
                                      const float* filter_3d, const float* d_out_scales,
                                      const float* d_out_opacities, int64_t n,
                                      float* d_scales, float* d_opacities,
                                      mg_stream_t stream);

/* ------------------------------------------------------------------------ */
/* 3DGS-MCMC densification (metal_gauss/mcmc.py)                            */
/* ------------------------------------------------------------------------ */

/* Rows of `width` floats per Gaussian starting at `ptr` (a parameter, an Adam
 * moment, or a per-row step count with width 1). */
typedef struct {
    float* ptr;
    int32_t width;
} mg_row_segment;

/* Scratch for the MCMC entry points, for `n` rows (the active count for
 * relocation, the capacity for growth). */
size_t mg_mcmc_scratch_bytes(int64_t n);

/* Replaces relocate (mcmc.py:52-104) with reset_adam_state (:107-121) on a
 * Gaussian table: `params` are its parameter segments (<= 32; params[logit_index]
 * the opacity logits, params[log_scales_index] the (N,3) log-scales; every
 * other segment is copied verbatim), `opt_rows` the optimizer rows to zero
 * for every row whose meaning changes. Rows < n_active whose opacity is
 * below dead_thresh are dead; each takes a live row drawn with probability
 * proportional to `weights` (NULL: opacity; non-finite or all-zero weights
 * fall back to opacity), with the multiplicity corrections of the split
 * (o' = 1 - (1 - o)^(1/n), scales times the binomial ratio; n = the draw
 * count of the target, clamped to [1, 51]) applied to copies and targets.
 * `picks` (n_dead rows, NULL: draw them from `seed`) fixes the draws.
 * *moved receives the number of dead rows. Synchronises `stream`. */
mg_status mg_mcmc_relocate(const mg_row_segment* params, int32_t n_params,
                           int32_t logit_index, int32_t log_scales_index,
                           const mg_row_segment* opt_rows, int32_t n_opt_rows,
                           int64_t n_active, float dead_thresh, const float* weights,
                           const int32_t* picks, uint64_t seed, int64_t* moved,
                           void* scratch, size_t scratch_bytes, mg_stream_t stream);

/* Replaces grow (mcmc.py:124-163): rows [n_active, min(target, capacity)) are
 * cloned from rows < n_active drawn with probability proportional to
 * max(weights, 1e-8) (NULL or invalid weights: opacity), with the split's
 * corrections for n = clamp(draws, 1, 51) + 1 applied to clones and targets
 * and their optimizer rows zeroed. *new_active receives the new active
 * count. `picks` as for mg_mcmc_relocate. Synchronises `stream`. */
mg_status mg_mcmc_grow(const mg_row_segment* params, int32_t n_params, int32_t logit_index,
                       int32_t log_scales_index, const mg_row_segment* opt_rows,
                       int32_t n_opt_rows, int64_t n_active, int64_t target, int64_t capacity,
                       const float* weights, const int32_t* picks, uint64_t seed,
                       int64_t* new_active, void* scratch, size_t scratch_bytes,
                       mg_stream_t stream);

/* Replaces add_noise (mcmc.py:166-192): means (N,3) += R(q) (eps * scales)
 * * sigmoid(-100 (opacity - opacity_gate)) * lr_means * weight for the
 * first n rows, eps ~ N(0, 1) from `seed` (or the given (N,3) `eps`),
 * R(q) the rotation of the normalised quaternion (w, x, y, z). */
mg_status mg_mcmc_add_noise(float* means, const float* quats, const float* log_scales,
                            const float* logit_opac, int64_t n, float lr_means, float weight,
                            float opacity_gate, uint64_t seed, const float* eps,
                            mg_stream_t stream);

/* ------------------------------------------------------------------------ */
/* Device error word                                                        */
/* ------------------------------------------------------------------------ */

/* Reads and clears the device error word of the current device (bounded
 * spins that gave up, checked-mode index faults). Synchronises `stream`.
 * *code_out receives 0 when nothing was recorded, else the first code:
 * 1 a sort look-back wait gave up, 2 a tile list reached past the sized pair
 * count. The reference refuses instead of continuing silently
 * (metal_gauss/api.py:18-26); callers raise on a non-zero code. */
mg_status mg_read_device_error(int32_t* code_out, mg_stream_t stream);

/* Copies the device error word of the current device, without clearing it,
 * to the device int64 *code_dev on `stream` (one tiny kernel, no host
 * synchronisation), so a caller can fetch it with a device->host read it
 * already makes. No reference counterpart. */
mg_status mg_peek_device_error(int64_t* code_dev, mg_stream_t stream);

/* Self-test of the sort's bounded wait (no reference counterpart): launches
 * one onesweep pass as the second tile of a two-tile sort whose first tile
 * never publishes its look-back word, with the wait limited to spin_limit
 * rounds (1..2^22; the sort itself uses 2^22). The pass gives up, records code
 * 1 in the device error word and returns; nothing hangs or traps. Read the
 * word with mg_read_device_error afterwards. scratch (256-byte aligned) holds
 * the self-test's own keys and look-back words. */
size_t mg_sort_lookback_selftest_scratch_bytes(void);
mg_status mg_sort_lookback_selftest(uint32_t spin_limit, void* scratch, size_t scratch_bytes,
                                    mg_stream_t stream);

#ifdef __cplusplus
}
#endif

#endif /* MG_B200_H */
