/*
 * fastgs_b200.h - C ABI of the B200 (sm_100a) FastGS differentiable tile
 * rasterizer: libfastgs_b200.so.
 *
 * Conventions
 *   - Every pointer argument is a DEVICE pointer (cudaMalloc / torch CUDA
 *     memory) unless its name ends in _host. Arrays are dense, row-major,
 *     in the reference's layouts (float32 unless stated). Sizes are explicit.
 *   - `stream` is a cudaStream_t (NULL = legacy default stream). All work is
 *     enqueued on it; nothing synchronises unless stated.
 *   - Return value: FGS_OK (0) or an fgs_status code; fgs_last_error() gives a
 *     message for the calling host thread. Invalid arguments are rejected
 *     before anything is launched.
 *   - Outputs are fully written: where the reference leaves an output at its
 *     zero fill (culled Gaussians, unwritten bucket samples), these calls
 *     write zeros, so callers need not clear them. Exceptions (accumulating
 *     gradient outputs) say so.
 *   - Tiles are 16x16 pixels; tile grid = ceil(W/16) x ceil(H/16).
 *
 * Each entry point names the reference interface it replaces
 * (paths relative to the reference project a1091150/fastgs_core).
 */
#ifndef FASTGS_B200_H
#define FASTGS_B200_H

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define FGS_API __attribute__((visibility("default")))
#else
#define FGS_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

enum fgs_status {
  FGS_OK = 0,
  FGS_ERR_INVALID = 1,   /* bad shape / size / argument (reference: std::invalid_argument) */
  FGS_ERR_CUDA = 2,      /* CUDA launch or runtime error */
  FGS_ERR_TIMEOUT = 3,   /* a bounded device-side wait gave up (sort look-back) */
  FGS_ERR_CAPACITY = 4,  /* a size exceeds what the call supports */
};

/* Message for the last failing call on this host thread ("" if none). */
FGS_API const char* fgs_last_error(void);
/* ABI version: 0x000100 = 0.1.0 */
FGS_API int fgs_version(void);

/* ---------------------------------------------------------------------------
 * Preprocess forward.
 * Replaces FastGSPreprocess (fastgs_core/include/fastgs_preprocess.h:13-55,
 * fastgs_core/fastgs_preprocess.cpp:41-168) and the Metal kernel
 * fastgs_preprocess_forward_kernel (fastgs_core/metal/fastgs_preprocess.metal:384-484).
 * focal_x = W / (2 tan_fovx) as fastgs_preprocess.cpp:120-121.
 */
typedef struct fgs_preprocess_params {
  int32_t n;                  /* Gaussians */
  int32_t degree;             /* active SH degree 0..3 */
  int32_t max_sh_coeffs;      /* sh.shape[1] (coefficients excluding DC) */
  float scale_modifier;
  float mult;                 /* FastGS opacity-aware extent multiplier */
  float tan_fovx, tan_fovy;
  int32_t image_width, image_height;
  int32_t use_cov3d_precomp;  /* 1: cov3d_precomp path, 0: scales + quats */
  int32_t use_colors_precomp; /* 1: colors_precomp path, 0: dc + sh */
} fgs_preprocess_params;

FGS_API int fgs_preprocess_forward(const fgs_preprocess_params* p,
                           /* inputs */
                           const float* means3d,        /* [n,3] */
                           const float* dc,             /* [n,3]  (SH path) */
                           const float* sh,             /* [n,max_sh_coeffs,3] */
                           const float* colors_precomp, /* [n,3]  (colour path) */
                           const float* opacities,      /* [n] */
                           const float* scales,         /* [n,3] */
                           const float* quats,          /* [n,4] (w,x,y,z) */
                           const float* cov3d_precomp,  /* [n,6] */
                           const float* viewmatrix,     /* [4,4] */
                           const float* projmatrix,     /* [4,4] */
                           const float* cam_pos,        /* [3] */
                           const float* viewspace_in,   /* [n,4] */
                           /* outputs */
                           int32_t* radii,              /* [n] */
                           float* xys,                  /* [n,2] */
                           float* depths,               /* [n] */
                           float* cov3d,                /* [n,6] */
                           float* rgb,                  /* [n,3] */
                           float* conic_opacity,        /* [n,4] */
                           uint32_t* tiles_touched,     /* [n] */
                           uint8_t* clamped,            /* [n,3] bool */
                           float* viewspace_out,        /* [n,4] */
                           void* stream);

/* ---------------------------------------------------------------------------
 * Inclusive prefix sum of tiles_touched -> point_offsets, and its last
 * element (num_rendered) into *total (device, uint64).
 * Replaces mx::cumsum(tiles_touched) + read_last_u32
 * (fastgs_core/binding/binding.cpp:153-154, :25-31). `scratch` holds
 * fgs_scan_scratch_bytes(n) bytes of device memory.
 */
FGS_API size_t fgs_scan_scratch_bytes(int64_t n);
FGS_API int fgs_inclusive_scan_u32(int64_t n, const uint32_t* in, uint32_t* out, uint64_t* total,
                           void* scratch, void* stream);

/* ---------------------------------------------------------------------------
 * Duplicate with keys: key = (tile_id << 32) | float_bits(depth), value =
 * Gaussian index, written from point_offsets[i-1].
 * Replaces FastGSBinning (fastgs_core/include/fastgs_binning.h:13-34,
 * fastgs_core/fastgs_binning.cpp:28-105) and
 * fastgs_duplicate_with_keys_kernel (fastgs_core/metal/fastgs_binning.metal:182-213).
 */
FGS_API int fgs_duplicate_with_keys(int32_t n, float mult, int32_t tile_bounds_x, int32_t tile_bounds_y,
                            const float* xys, const float* depths,
                            const uint32_t* point_offsets, const float* conic_opacity,
                            const uint32_t* tiles_touched, int64_t num_rendered,
                            uint64_t* keys_unsorted, uint32_t* values_unsorted, void* stream);

/* ---------------------------------------------------------------------------
 * Stable LSD onesweep radix sort of (key, value) pairs on the low `key_bits`
 * bits (32 depth bits + bits of the largest tile id). Inputs are not
 * modified. Replaces mx::argsort + 2x mx::take (fastgs_core/binding/binding.cpp:195-197).
 * `workspace` holds fgs_sort_workspace_bytes(num_rendered, key_bits) bytes.
 * The sort is asynchronous: a bounded look-back wait that gives up cannot
 * fail the call itself. It sets the timeout flag of the workspace instead,
 * which fgs_sort_status reports as FGS_ERR_TIMEOUT, and the output is then
 * not sorted but safe for the consumers: every stored key is all ones (an
 * invalid tile id, so tile prep finds every tile empty) and the values are
 * values_in in input order. Every store stays in bounds.
 */
FGS_API size_t fgs_sort_workspace_bytes(int64_t num_rendered, int32_t key_bits);
FGS_API int fgs_sort_pairs(int64_t num_rendered, int32_t key_bits, const uint64_t* keys_in,
                   const uint32_t* values_in, uint64_t* keys_out, uint32_t* values_out,
                   void* workspace, size_t workspace_bytes, void* stream);

/* As fgs_sort_pairs on key bits [bit_begin, bit_end) only (stable: pairs
 * with equal bits there keep their input order). The workspace is
 * fgs_sort_workspace_bytes(num_rendered, bit_end - bit_begin). */
FGS_API int fgs_sort_pairs_bits(int64_t num_rendered, int32_t bit_begin, int32_t bit_end,
                                const uint64_t* keys_in, const uint32_t* values_in,
                                uint64_t* keys_out, uint32_t* values_out, void* workspace,
                                size_t workspace_bytes, void* stream);

/* Status of the last sort run in `workspace` (fgs_sort_pairs,
 * fgs_sort_pairs_bits, or the depth ordering of fgs_depth_order, whose
 * workspace starts with its sort's): synchronises `stream`, then returns
 * FGS_ERR_TIMEOUT if a look-back wait of that sort gave up, FGS_OK otherwise.
 * workspace == NULL reads the scratch of fgs_sort_pairs_static on the current
 * device. The flag is the int32 at byte offset 0 of the workspace (nonzero =
 * timed out), so a caller that synchronises anyway may instead copy those 4
 * bytes back itself. */
FGS_API int fgs_sort_status(const void* workspace, void* stream);

/* Test hooks of the look-back wait, process-wide: spin_limit polls before a
 * wait gives up (0 restores the default, 2^22), and withhold_first_partition
 * != 0 makes the first partition publish nothing, so that the next one's
 * wait runs out without any fault. Not for production use; not thread-safe. */
FGS_API int fgs_sort_set_test_hooks(int32_t spin_limit, int32_t withhold_first_partition);

/* Depth-first binning, the training path's replacement for sorting the K
 * duplicated (tile | depth) keys on all 32 + ceil(log2 T) bits: the n
 * Gaussians are ordered by depth (stable, so equal depths keep index order),
 * fgs_duplicate_with_keys_ordered emits the keys in that order, and a stable
 * sort of the tile bits [32, 32 + ceil(log2 T)) alone then yields the same
 * sorted keys and values as fgs_sort_pairs on the Gaussian-order keys: within
 * a tile, depth order with ties in index order. No reference counterpart
 * (fastgs_core/binding/binding.cpp:186-197 duplicates, then sorts all bits).
 *
 * fgs_depth_order writes order[n] (Gaussian indices by depth) and
 * tiles_in_order[j] = tiles_touched[order[j]]; the caller scans the latter
 * (fgs_inclusive_scan_u32) for the offsets in order. */
FGS_API size_t fgs_depth_order_workspace_bytes(int32_t n);
FGS_API int fgs_depth_order(int32_t n, const float* depths, const uint32_t* tiles_touched,
                            uint32_t* order, uint32_t* tiles_in_order, void* workspace,
                            size_t workspace_bytes, void* stream);
FGS_API int fgs_duplicate_with_keys_ordered(int32_t n, float mult, int32_t tile_bounds_x,
                                            int32_t tile_bounds_y, const float* xys,
                                            const float* depths, const uint32_t* order,
                                            const uint32_t* offsets_in_order,
                                            const float* conic_opacity,
                                            const uint32_t* tiles_touched, int64_t num_rendered,
                                            uint64_t* keys, uint32_t* values, void* stream);

/* ---------------------------------------------------------------------------
 * fgs_sort_pairs without any allocation. No counterpart in the reference: it
 * exists for callers that cannot allocate device memory when they sort (a
 * host application that gives plug-ins a fixed GPU memory budget and forbids
 * allocation after start-up, or a frame loop that must not call
 * cudaMalloc/cudaFree). The scratch is a fixed area inside the library's
 * device image (about 15 MB, held on every GPU that loads the library until
 * the process exits), so at most FGS_SORT_STATIC_MAX_KEYS keys can be sorted;
 * larger inputs return FGS_ERR_CAPACITY without launching anything. The first
 * call on each device looks the area up (make it before any stream capture).
 * Every call shares that one area: calls that overlap on the GPU (other
 * streams, other host threads) race and must be serialised by the caller.
 * Same arguments and results as fgs_sort_pairs otherwise; fgs_sort_status
 * with a NULL workspace reports the last call's look-back timeout flag.
 */
#define FGS_SORT_STATIC_MAX_KEYS 1048576
FGS_API int fgs_sort_pairs_static(int64_t num_rendered, int32_t key_bits, const uint64_t* keys_in,
                                  const uint32_t* values_in, uint64_t* keys_out,
                                  uint32_t* values_out, void* stream);

/* ---------------------------------------------------------------------------
 * Tile ranges [T,2] (empty tiles [0,0]) and per-tile bucket counts
 * ceil(n_t / 32); plus, new here, the inclusive scan of bucket counts
 * (per_tile_bucket_offset) and its total into *bucket_sum (device uint64).
 * Replaces FastGSTilePrep (fastgs_core/include/fastgs_tile_prep.h:12-28,
 * fastgs_core/fastgs_tile_prep.cpp:26-98; kernels
 * fastgs_core/metal/fastgs_tile_prep.metal:10-53) and the bucket cumsum of
 * fastgs_core/binding/binding.cpp:211-212.
 */
FGS_API int fgs_tile_prep(int64_t num_rendered, int32_t num_tiles, const uint64_t* sorted_keys,
                  uint32_t* ranges, uint32_t* bucket_count, uint32_t* bucket_offsets,
                  uint64_t* bucket_sum, void* stream);

/* Tiles in descending order of splat count (ranges from fgs_tile_prep) into
 * tile_order[num_tiles], for fgs_raster_params.tile_order. No reference
 * counterpart: the reference dispatches tiles in index order
 * (fastgs_core/fastgs_rasterize.cpp:160-168); this changes only which CTA
 * renders which tile. */
FGS_API int fgs_tile_order(int32_t num_tiles, const uint32_t* ranges, uint32_t* tile_order,
                           void* stream);

/* fgs_tile_prep, fgs_tile_order and the invalidation of bucket_to_tile
 * entries [bucket total, bucket_to_tile_len) in two launches, for a caller
 * that sizes the bucket arrays by a bound (the backward pass skips buckets
 * whose tile entry is out of range). */
FGS_API int fgs_tile_prep_ordered(int64_t num_rendered, int32_t num_tiles, const uint64_t* sorted_keys,
                                  uint32_t* ranges, uint32_t* bucket_count, uint32_t* bucket_offsets,
                                  uint64_t* bucket_sum, uint32_t* tile_order, uint32_t* bucket_to_tile,
                                  int64_t bucket_to_tile_len, void* stream);

/* ---------------------------------------------------------------------------
 * Rasterize forward: one CTA per 16x16 tile, front-to-back alpha blending
 * with early termination, per-32-splat bucket samples for the backward pass.
 * Replaces FastGSRasterize (fastgs_core/include/fastgs_rasterize.h:14-51,
 * fastgs_core/fastgs_rasterize.cpp:32-168) and fastgs_render_forward_kernel
 * (fastgs_core/metal/fastgs_rasterize.metal:25-159). sampled_ar is laid out
 * [bucket][channel][256] as the reference writes it. metric_count is
 * overwritten with this render's counts when get_flag != 0 (may be NULL
 * otherwise). max_contrib is the max of n_contrib over in-image pixels.
 */
typedef struct fgs_raster_params {
  int32_t image_width, image_height;
  int32_t num_tiles;
  int64_t bucket_sum;
  int32_t num_gaussians;   /* size of metric_count */
  int32_t get_flag;
  /* Optional [num_tiles] permutation of the tiles: CTA i of the forward pass
   * renders tile tile_order[i] (fgs_tile_order writes the heaviest-first
   * order). NULL renders tile i in CTA i. Results do not depend on it. The
   * backward pass ignores it. */
  const uint32_t* tile_order;
  /* Optional [bucket_sum*256] uint32, bucket-major like sampled_t: bit j of
   * entry (bucket, pixel) is set when splat j of the bucket contributed to
   * the pixel. The forward pass writes it when non-NULL; the backward pass,
   * given the same buffer, takes each pair's contribution from it instead of
   * re-deciding it (the gradients then use the fast exponential). NULL on
   * both sides reproduces the reference's recomputation. */
  uint32_t* contrib_mask;
  /* Nonzero: the forward pass writes the bucket samples (and mask words) of
   * a pixel only while the pixel is live at the bucket's start, and leaves
   * the entries of pixels that terminated earlier unwritten instead of
   * zeroing them; the backward pass, given the same flag, does not read
   * those entries (no splat of such a bucket contributes to the pixel).
   * Zero keeps the reference's fully written layout. Same gradients either
   * way. */
  int32_t sparse_samples;
} fgs_raster_params;

FGS_API int fgs_rasterize_forward(const fgs_raster_params* p, const uint32_t* ranges,
                          const uint32_t* point_list, const uint32_t* bucket_offsets,
                          const float* means2d, const float* colors, const float* conic_opacity,
                          const float* background, const int32_t* metric_map,
                          uint32_t* bucket_to_tile,  /* [bucket_sum] */
                          float* sampled_t,          /* [bucket_sum*256] */
                          float* sampled_ar,         /* [bucket_sum*3*256] */
                          float* final_t,            /* [H*W] */
                          uint32_t* n_contrib,       /* [H*W] */
                          uint32_t* max_contrib,     /* [T] */
                          float* pixel_colors,       /* [3,H*W] */
                          float* out_color,          /* [3,H*W] */
                          int32_t* metric_count,     /* [n] */
                          void* stream);

/* ---------------------------------------------------------------------------
 * Rasterize backward (per-bucket: 32 splats x 256 pixels per warp).
 * Replaces FastGSRasterizeBackward (fastgs_core/fastgs_rasterize_backward.cpp:35-166)
 * and fastgs_render_backward_kernel (fastgs_core/metal/fastgs_rasterize_backward.metal:24-278).
 * Gradients ACCUMULATE into dL_dmeans2d [n,2], dL_dcolors [n,3],
 * dL_dconic_opacity [n,4], dL_dviewspace [n,4]; zero them first for a plain VJP.
 */
FGS_API int fgs_rasterize_backward(const fgs_raster_params* p, const uint32_t* ranges,
                           const uint32_t* point_list, const uint32_t* bucket_offsets,
                           const float* means2d, const float* colors, const float* conic_opacity,
                           const float* background, const float* dL_dout_color,
                           const uint32_t* bucket_to_tile, const float* sampled_t,
                           const float* sampled_ar, const float* final_t,
                           const uint32_t* n_contrib, const uint32_t* max_contrib,
                           const float* pixel_colors, float* dL_dmeans2d, float* dL_dcolors,
                           float* dL_dconic_opacity, float* dL_dviewspace, void* stream);

/* ---------------------------------------------------------------------------
 * Preprocess backward: conic -> cov2D -> (cov3D, means3D), projective
 * Jacobian, SH backward with clamp mask, cov3D -> (scale, quat), identity for
 * viewspace points. Outputs are written (not accumulated); rows of Gaussians
 * with radii <= 0 are zero.
 * Replaces FastGSPreprocessBackward (fastgs_core/fastgs_preprocess_backward.cpp:39-183)
 * and fastgs_preprocess_backward_kernel
 * (fastgs_core/metal/fastgs_preprocess_backward.metal:60-430).
 * focal = 0.5 W / max(tan_fovx, 1e-6) as fastgs_preprocess_backward.cpp:134-137.
 */
FGS_API int fgs_preprocess_backward(const fgs_preprocess_params* p, const float* means3d,
                            const float* scales, const float* quats, const float* viewmatrix,
                            const float* projmatrix, const float* cam_pos, const float* sh,
                            const float* cov3d_precomp, const float* cov3d_fwd,
                            const float* dL_dcov3d,       /* [n,6] may be NULL (= 0) */
                            const float* dL_drgb,         /* [n,3] */
                            const float* dL_dxys,         /* [n,2] */
                            const float* dL_dconic_opacity, /* [n,4] */
                            const float* dL_dviewspace_out, /* [n,4] */
                            const int32_t* radii, const uint8_t* clamped,
                            float* dL_dmeans3d, float* dL_ddc, float* dL_dsh,
                            float* dL_dcolors_precomp, float* dL_dopacities, float* dL_dscales,
                            float* dL_dquats, float* dL_dviewspace_in, void* stream);

/* ===========================================================================
 * Training-step entry points (new here: the reference does this work in
 * Python/MLX inside its training scripts, as cited per function).
 *
 * Flat parameter / gradient layout, 59 floats per Gaussian, N Gaussians:
 *   [0,3N) means3d  [3N,6N) features_dc  [6N,51N) features_rest [N,15,3]
 *   [51N,52N) opacity logits  [52N,55N) log scales  [55N,59N) rotations (raw)
 * Densification statistics `stats`, 4N floats: [0,N) sum |grad_xy|,
 *   [N,2N) sum |grad_abs|, [2N,3N) visible-view count, [3N,4N) max radius.
 */

/* opacity = sigmoid(logit), scale = exp(log_scale), quat = q / (|q| + 1e-8):
 * the getters of scripts/train_scanner_fixed.py:523-535. */
FGS_API int fgs_activate_params(int64_t n, const float* params_flat, float* opacities,
                                float* scales, float* quats, void* stream);

/* Training variants of preprocess forward and backward. They read the flat
 * raw-parameter buffer `params` (59 n floats: means 3, dc 3, sh rest 45,
 * opacity logit 1, log-scale 3, rotation 4, each segment attribute-major) and
 * apply the trainers' activations inside the kernels (opacity =
 * sigmoid(logit), scale = exp(log_scale), rotation = q / (|q| + 1e-8):
 * scripts/train_scanner_fixed.py:523-535), so no activated copy is needed.
 * SH degree 3 layout (15 rest coefficients), scales+quats and dc+sh paths.
 *
 * fgs_preprocess_forward_train: the outputs of fgs_preprocess_forward.
 *
 * fgs_preprocess_backward_train: as fgs_preprocess_backward, chained through
 * the activations, written (accumulate == 0) or added (accumulate != 0) into
 * the flat gradient buffer, and the densification statistics of
 * scripts/train_scanner_fastgs.py:391-405 ([acc | acc_abs | denom |
 * max_radii], 4 n) updated for Gaussians with radii > 0 from dL_dviewspace.
 *
 * fgs_preprocess_backward_adam: the same backward pass of one view followed
 * by the Adam step of fgs_adam_step, in one pass: each Gaussian's gradients
 * are applied to params / exp_avg / exp_avg_sq as soon as they are formed, so
 * no gradient buffer is written or read. group_lr[6] holds the learning rate
 * of each segment in layout order. For a step whose gradient is exactly this
 * one view's (one view, one rank); the result equals
 * fgs_preprocess_backward_train + fgs_adam_step bit for bit.
 *
 * In every Adam entry point a negative group learning rate means that the
 * group does not step: its values and moments are left unchanged (the
 * reference's optimiser cadence, scripts/train_scanner_fastgs.py:160-183). */
FGS_API int fgs_preprocess_forward_train(const fgs_preprocess_params* p, const float* params,
                                         const float* viewmatrix, const float* projmatrix,
                                         const float* cam_pos, const float* viewspace_in,
                                         int32_t* radii, float* xys, float* depths, float* cov3d,
                                         float* rgb, float* conic_opacity, uint32_t* tiles_touched,
                                         uint8_t* clamped, float* viewspace_out, void* stream);
/* The training preprocess forward in two launches, for a caller that wants
 * the colour step later than the geometry (no counterpart in the reference,
 * which evaluates colours inside its one preprocess kernel,
 * fastgs_core/metal/fastgs_preprocess.metal:117-169, 469):
 * fgs_preprocess_forward_train_geometry writes every output of
 * fgs_preprocess_forward_train except rgb and clamped, and reads no SH;
 * fgs_preprocess_colors_train then writes rgb and clamped from `params` and
 * the same tiles_touched, bit for bit as the one-launch call would. The
 * data-parallel trainer uses the split to exchange the SH coefficients of the
 * previous step while the geometry and the binning of this step run. */
FGS_API int fgs_preprocess_forward_train_geometry(const fgs_preprocess_params* p,
                                                  const float* params, const float* viewmatrix,
                                                  const float* projmatrix,
                                                  const float* viewspace_in, int32_t* radii,
                                                  float* xys, float* depths, float* cov3d,
                                                  float* conic_opacity, uint32_t* tiles_touched,
                                                  float* viewspace_out, void* stream);
FGS_API int fgs_preprocess_colors_train(const fgs_preprocess_params* p, const float* params,
                                        const float* cam_pos, const uint32_t* tiles_touched,
                                        float* rgb, uint8_t* clamped, void* stream);
FGS_API int fgs_preprocess_backward_train(const fgs_preprocess_params* p, const float* params,
                                          const float* viewmatrix, const float* projmatrix,
                                          const float* cam_pos, const float* cov3d_fwd,
                                          const float* dL_drgb, const float* dL_dxys,
                                          const float* dL_dconic_opacity,
                                          const float* dL_dviewspace, const int32_t* radii,
                                          const uint8_t* clamped, int32_t accumulate,
                                          float* grad_flat, float* stats, void* stream);
FGS_API int fgs_preprocess_backward_adam(const fgs_preprocess_params* p, const float* viewmatrix,
                                         const float* projmatrix, const float* cam_pos,
                                         const float* cov3d_fwd, const float* dL_drgb,
                                         const float* dL_dxys, const float* dL_dconic_opacity,
                                         const float* dL_dviewspace, const int32_t* radii,
                                         const uint8_t* clamped, float* params, float* exp_avg,
                                         float* exp_avg_sq, const float* group_lr, float beta1,
                                         float beta2, float eps, int32_t step,
                                         int32_t bias_correction, float* stats, void* stream);

/* loss = w_l1 * mean|image - target| + w_ssim * (1 - mean SSIM(image, target))
 * over CHW [3,H,W] float images (SSIM: 11x11 Gaussian window, sigma 1.5, zero
 * padding, C1 = 0.01^2, C2 = 0.03^2), and dL/dimage. loss_out receives
 * {loss, mean L1, mean SSIM} (3 floats, device). `scratch` holds
 * fgs_loss_scratch_bytes(W, H) bytes. The training scripts' loss
 * (scripts/train_scanner_fastgs.py:949-964) with the D-SSIM term added. */
FGS_API size_t fgs_loss_scratch_bytes(int32_t width, int32_t height);
FGS_API int fgs_l1_dssim_loss(int32_t width, int32_t height, const float* image,
                              const float* target, float w_l1, float w_ssim, float* loss_out,
                              float* dL_dimage, void* scratch, void* stream);

/* loss = w_mse * mean (image - target)^2 over CHW [3,H,W] images, and
 * dL/dimage: the reference trainer's loss before --mse-until
 * (scripts/train_scanner_fastgs.py:824, 957-960). loss_out receives {loss,
 * mean squared error, 0}; `scratch` holds fgs_loss_scratch_bytes(W, H) bytes. */
FGS_API int fgs_mse_loss(int32_t width, int32_t height, const float* image, const float* target,
                         float w_mse, float* loss_out, float* dL_dimage, void* scratch, void* stream);

/* Adam over a flat buffer split into num_groups (<= 8) contiguous groups:
 * elements [group_end[k-1], group_end[k]) use group_lr[k] (host arrays).
 * m = b1 m + (1-b1) g; v = b2 v + (1-b2) g^2; p -= lr m' / (sqrt(v') + eps),
 * with m' = m, v' = v unless bias_correction (then / (1 - b^step)): the MLX
 * optim.Adam the reference trainers use (scripts/train_scanner_fastgs.py:76-99).
 * Buffers 16-byte aligned. */
FGS_API int fgs_adam_step(int64_t total, float* params, const float* grads, float* exp_avg,
                          float* exp_avg_sq, int32_t num_groups, const int64_t* group_end,
                          const float* group_lr, float beta1, float beta2, float eps, int32_t step,
                          int32_t bias_correction, void* stream);

/* Data-parallel Adam over NVLink multicast (new here; the reference is single-
 * device). The gradient and parameter buffers are symmetric allocations bound
 * to an NVLink multicast object on every rank (e.g. torch symmetric memory);
 * grads_mc / params_mc are the multicast addresses of this rank's shard,
 * params_local its local copy, exp_avg / exp_avg_sq this rank's moments
 * (shard floats, multiple of 4). The kernel reads the rank-summed gradient with
 * multimem.ld_reduce, applies the Adam rule of fgs_adam_step, and stores the
 * new parameters to every rank with multimem.st. Callers bracket it with a
 * cross-rank barrier before (all gradients written) and after (all stores
 * visible). Group ends are relative to the shard. */
FGS_API int fgs_adam_step_multicast(int64_t shard, const float* params_local, float* params_mc,
                                    const float* grads_mc, float* exp_avg, float* exp_avg_sq,
                                    int32_t num_groups, const int64_t* group_end,
                                    const float* group_lr, float beta1, float beta2, float eps,
                                    int32_t step, int32_t bias_correction, void* stream);

/* Data-parallel Adam over plain peer loads and stores (new here; used at two
 * ranks, where it moves less over NVLink than fgs_adam_step_multicast).
 * params_ranks[r] / grads_ranks[r] (host arrays of `world` pointers) address
 * rank r's copy of this rank's shard in this process (symmetric memory or
 * peer mappings; r == rank is local). The kernel sums the ranks' gradients in
 * rank order, applies the Adam rule of fgs_adam_step to the shard (moments
 * exp_avg / exp_avg_sq are this rank's) and stores the new parameters into
 * every rank's copy. Callers bracket it with a cross-rank barrier before (all
 * gradients written) and after (all stores visible). Group ends are relative
 * to the shard; world <= 8. */
FGS_API int fgs_adam_step_peers(int64_t shard, int32_t world, int32_t rank, float* const* params_ranks,
                                const float* const* grads_ranks, float* exp_avg, float* exp_avg_sq,
                                int32_t num_groups, const int64_t* group_end,
                                const float* group_lr, float beta1, float beta2, float eps,
                                int32_t step, int32_t bias_correction, void* stream);

/* Data-parallel exchange by pushing (new here; the reference is single-
 * device). Rank r owns the flat elements [r shard, (r + 1) shard) of the
 * gradient buffer; grad_ranks[r] (host array of `world` pointers) addresses
 * rank r's whole buffer in this process (symmetric memory or peer mappings).
 * fgs_preprocess_backward_push: fgs_preprocess_backward_train whose gradients
 *   are added (relaxed system-scope float reductions, 16-byte vectors where the
 *   flat index allows) into the owner's buffer, which must hold zeros or
 *   earlier views' sums of this step; the densification statistics update
 *   locally as in fgs_preprocess_backward_train.
 * fgs_adam_step_owner: after a cross-rank barrier, the owner reads its summed
 *   shard `grads` (local), writes zeros back for the next step, applies the
 *   Adam rule of fgs_adam_step to its moments and stores the new parameters
 *   into every rank's copy: params_ranks[r] (this rank's shard in rank r's
 *   buffer), or one multimem.st to params_mc when that multicast address is
 *   given. A second barrier publishes them. Group ends relative to the shard. */
FGS_API int fgs_preprocess_backward_push(const fgs_preprocess_params* p, const float* params,
                                         const float* viewmatrix, const float* projmatrix,
                                         const float* cam_pos, const float* cov3d_fwd,
                                         const float* dL_drgb, const float* dL_dxys,
                                         const float* dL_dconic_opacity,
                                         const float* dL_dviewspace, const int32_t* radii,
                                         const uint8_t* clamped, int32_t world, int64_t shard,
                                         float* const* grad_ranks, float* stats, void* stream);
FGS_API int fgs_adam_step_owner(int64_t shard, int32_t world, int32_t rank,
                                float* const* params_ranks, float* params_mc, float* grads,
                                float* exp_avg, float* exp_avg_sq, int32_t num_groups,
                                const int64_t* group_end, const float* group_lr, float beta1,
                                float beta2, float eps, int32_t step, int32_t bias_correction,
                                void* stream);

/* Adam of a gathered gradient shard (new here): grads[r] (host array of
 * `world` pointers, local memory, e.g. this rank's own gradients and copies of
 * the other ranks' shards brought over by the copy engines) are summed in
 * rank order, as fgs_adam_step_peers sums them, and the Adam rule of
 * fgs_adam_step updates params / exp_avg / exp_avg_sq (shard floats). */
FGS_API int fgs_adam_step_gathered(int64_t shard, int32_t world, const float* const* grads,
                                   float* params, float* exp_avg, float* exp_avg_sq,
                                   int32_t num_groups, const int64_t* group_end,
                                   const float* group_lr, float beta1, float beta2, float eps,
                                   int32_t step, int32_t bias_correction, void* stream);

/* Grid budget of fgs_adam_step_multicast and fgs_adam_step_peers for the
 * launches that follow in this process: at most blocks_per_sm CTAs of 256
 * threads per SM (0 restores their defaults of 4 and 8). Both kernels stride
 * over their shard, so a small budget leaves SMs to kernels running on other
 * streams at the same time, at some cost in the exchange's own speed. Not
 * synchronised between host threads (new here; no counterpart in the
 * reference). */
FGS_API int fgs_set_exchange_grid(int32_t blocks_per_sm);

/* FastGS multi-view score pass (scripts/train_scanner_fastgs.py:262-340):
 * fgs_metric_map: per-pixel mean |pred - target| over channels, min-max
 *   normalised, > loss_thresh -> metric_map [P] int32; *l1_sum (device) gets
 *   sum |pred - target| over all 3P elements. scratch: 4*P + 8 bytes.
 * fgs_score_accumulate: counts_acc += metric_count; score_acc +=
 *   (l1_sum / num_elements) * metric_count.
 * fgs_score_finalize: importance = floor(counts_acc / n_views) (skipped if
 *   importance is NULL), pruning = min-max normalised score_acc. scratch: 8 bytes. */
FGS_API int fgs_metric_map(int64_t num_pixels, const float* pred, const float* target,
                           float loss_thresh, int32_t* metric_map, float* l1_sum, void* scratch,
                           void* stream);
FGS_API int fgs_score_accumulate(int64_t n, const int32_t* metric_count, const float* l1_sum,
                                 int64_t num_elements, float* counts_acc, float* score_acc,
                                 void* stream);
FGS_API int fgs_score_finalize(int64_t n, const float* counts_acc, const float* score_acc,
                               int32_t n_views, float* importance, float* pruning, void* scratch,
                               void* stream);

/* ---------------------------------------------------------------------------
 * FastGS densification on the device (scripts/train_scanner_fastgs.py:470-795).
 * Flat layouts as the training entry points: segment k of width w_k holds
 * rows [0, n) attribute-major at offset (w_0 + ... + w_{k-1}) * n.
 *
 * fgs_gather_rows: dst row j of every segment = src row index[j] (n_in rows
 * in src, n_out in dst; index < 0 writes zeros). Prunes (keep indices),
 * appends copies (0..n-1 then the sources) and appends zero rows (moments).
 *
 * fgs_densify_masks: per Gaussian, bit 0 = clone (importance > threshold,
 * max scale <= dense_extent, |acc / max(denom, 1)| >= grad_thresh), bit 1 =
 * split (importance > threshold, max scale > dense_extent, |acc_abs /
 * max(denom, 1)| >= grad_abs_thresh), bit 2 = importance > threshold.
 * stats = [acc | acc_abs | denom | max_radii].
 *
 * fgs_prune_masks: bit 0 = sigmoid(logit) < min_opacity, bit 1 = max_radii >
 * max_screen (max_screen > 0), bit 2 = max scale > max_world (max_world > 0).
 *
 * fgs_split_fixup: rows [row0, row0 + m) hold copies of their split sources;
 * their means move by R(q) * samples[t] (samples already scaled by the
 * source's scales) and their log-scales become log(exp(s) / (0.8 f)).
 *
 * fgs_opacity_cap: logit(clip(min(sigmoid(l), cap), 1e-6, 1 - 1e-6)) on the
 * opacity segment; the opacity moments (if given) restart at zero. */
FGS_API int fgs_gather_rows(int64_t n_in, int64_t n_out, const int64_t* index, int32_t num_segments,
                            const int32_t* widths, const float* src, float* dst, void* stream);
FGS_API int fgs_densify_masks(int64_t n, const float* params, const float* stats,
                              const float* importance, float grad_thresh, float grad_abs_thresh,
                              float dense_extent, float importance_thresh, uint8_t* mask,
                              void* stream);
FGS_API int fgs_prune_masks(int64_t n, const float* params, const float* max_radii,
                            float min_opacity, float max_screen, float max_world, uint8_t* mask,
                            void* stream);
FGS_API int fgs_split_fixup(int64_t n, int64_t row0, int64_t m, const float* samples,
                            int32_t split_factor, float* params, void* stream);
FGS_API int fgs_opacity_cap(int64_t n, float cap, float* params, float* exp_avg, float* exp_avg_sq,
                            void* stream);

#ifdef __cplusplus
}
#endif
#endif /* FASTGS_B200_H */
