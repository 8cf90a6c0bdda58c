/* gsplat_b200.h — C ABI of libgsplat_b200.so, the B200 (sm_100a) kernels of the
 * 3D Gaussian Splatting training step: cull -> project -> depth sort -> tile
 * binning + tile sort -> compositing forward -> compositing backward ->
 * projection backward -> fused Adam over the pooled buffers -> densify/prune
 * over the fixed-capacity pool.
 *
 * Conventions (every entry point):
 *  - plain device pointers, element counts and strides (in floats); no
 *    framework types.  The library never allocates on these paths, never
 *    frees caller memory and mutates only the buffers documented as outputs.
 *  - ``stream`` is a cudaStream_t passed as void*; every kernel is enqueued on
 *    it asynchronously (NULL = the legacy default stream).  No entry point
 *    synchronises the device.
 *  - the return value is a GS_* status; GS_OK is 0.  gs_last_error() gives a
 *    human-readable message for the calling thread's last failure.
 *  - not reentrant per buffer set; callable from one host thread per device.
 *
 * Replaced reference interface: the pybind11 module ``mlx_gsplat_ext``
 * (src/mlx_extensions.cpp:238-248) — launch_fused_adam_step and
 * clear_buffer_cache — plus the pure-Python rasterizer entry points
 * frustum_culling_mlx / rasterize_gaussians_mlx (mlx_gsplat/rendering.py:41-308),
 * the allocator's split_and_prune (mlx_gsplat/allocator.py:185-292) and the
 * trainer's densify policy (mlx_gsplat/trainer.py:421-519).
 */
#ifndef GSPLAT_B200_H
#define GSPLAT_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ------------------------------------------------------------------ status */
#define GS_OK 0
#define GS_ERR_INVALID 1  /* bad argument (null pointer, size, stride, alignment) */
#define GS_ERR_CUDA 2     /* a CUDA runtime call or kernel launch failed */
#define GS_ERR_CAPACITY 3 /* a caller buffer or the pool is too small */

typedef void* gs_stream_t; /* cudaStream_t */

const char* gs_last_error(void);
int gs_abi_version(void);
/* Number of kernels this library has launched in this process (all threads). */
unsigned long long gs_kernel_launches(void);

/* ------------------------------------------------------------------ types */

/* How the rasterizer turns a Gaussian's colour row into RGB.
 *
 * GS_SH_REFERENCE — mlx_gsplat/rendering.py:229-244: the DC term, plus the
 *   degree-1 term when colors_dim >= 12, whatever the number of stored
 *   coefficients.  Row layout: c[0..2] DC (r, g, b); channel ch's degree-1
 *   coefficients at c[3 + 3ch + (0, 1, 2)], multiplying (y, z, x) of the unit
 *   view direction, all with sign +.
 * GS_SH_FULL — real spherical harmonics up to the degree d that colors_dim
 *   holds (3 (d+1)^2 floats: 3 -> 0, 12 -> 1, 27 -> 2, 48 -> 3; at most 3).
 *   With k = (d+1)^2 - 1, channel ch's coefficients are c[3 + k ch + j],
 *   j < k: the first three are the degree-1 terms of the reference mode
 *   (same order and signs, so both modes agree for d <= 1), then the five
 *   degree-2 and the seven degree-3 basis functions (no reference
 *   counterpart: the reference evaluates degree <= 1 only). */
#define GS_SH_REFERENCE 0
#define GS_SH_FULL 1

/* Read-only Gaussian parameters.  Row ``r`` of a group lives at
 * ``ptr + r * stride``.  Rows are addressed by an "active id" ``i``:
 * ``r = table ? table[i] : i``.  Colours use the same row unless
 * ``colors_by_visible`` is set, in which case colour row = visible position
 * (the reference's rule at mlx_gsplat/rendering.py:143-146). */
typedef struct gs_gaussians {
    const float* means;  int64_t means_stride;  /* [., 3] world positions */
    const float* quats;  int64_t quats_stride;  /* [., 4] (w, x, y, z), unnormalised */
    const float* scales; int64_t scales_stride; /* [., 3] log-scales */
    const float* opac;   int64_t opac_stride;   /* [., 1] opacity logits */
    const float* colors; int64_t colors_stride; /* [., colors_dim] SH coefficients, DC first */
    int32_t colors_dim;                         /* colour floats the rasterizer may read */
    int32_t colors_by_visible;
    const int32_t* table;                       /* optional active-id -> row map */
    int32_t sh_mode;                            /* GS_SH_REFERENCE (0) or GS_SH_FULL */
} gs_gaussians;

/* Gradient outputs, one row per active id (never through ``table``). */
typedef struct gs_gaussian_grads {
    float* means;  int64_t means_stride;
    float* quats;  int64_t quats_stride;
    float* scales; int64_t scales_stride;
    float* opac;   int64_t opac_stride;
    float* colors; int64_t colors_stride;
    int32_t colors_write;     /* colour columns written per row (>= the rasterizer's 3 or 12) */
    int32_t colors_by_visible;
    int32_t accumulate;       /* 1: atomically add into the rows; 0: store */
    float reg;                /* constant added to every written geometry gradient (the trainer's 1e-5 * sum(params)) */
    int32_t reg_color_cols;   /* the first reg_color_cols colour columns also receive ``reg`` */
    int32_t reg_geometry;     /* 0: the geometry columns do not receive ``reg`` (the caller adds it later) */
    int32_t count_col;        /* > 0: every written row also gets 1.0 in this column of the pooled gradient
                                 rows (``quats`` base, ``quats_stride``; pooled row layout only) — the number
                                 of views that saw the row, once rows are summed over GPUs; 0: none */
} gs_gaussian_grads;

/* Pinhole camera.  ``viewmat`` is the row-major world-to-camera matrix
 * (camera point = viewmat @ [x, y, z, 1]); pixel (i, j) of the render grid
 * is centred at (i*sx + sx/2, j*sy + sy/2), sx = width / render_width. */
typedef struct gs_camera {
    float viewmat[16];
    float fx, fy, cx, cy;
    int32_t width, height;
    int32_t render_width, render_height;
} gs_camera;

/* Rasterizer settings.  The dense reference composites every visible
 * Gaussian at every pixel; the tiled kernels bin a Gaussian into a 16x16 tile
 * only when some pixel centre of the tile can see alpha >= alpha_cutoff, and
 * stop a pixel once its transmittance falls below transmittance_min. */
typedef struct gs_raster_settings {
    float alpha_cutoff;      /* e.g. 1e-7 (the default: parity with the dense reference to ~1e-6) */
    float transmittance_min; /* e.g. 1e-6 (parity) */
    int32_t alpha_mask;      /* 1: the compositing kernels multiply each splat's clipped alpha by the
                                multiplier gs_apply_sorted_mask stored in its record; 0 (default): none */
} gs_raster_settings;

/* Per-tile [start, end) ranges into the tile-sorted entry list. */
typedef struct gs_tile_range { int32_t start, end; } gs_tile_range;

/* ------------------------------------------------------------------ Adam */

/* Drop-in for mlx_gsplat_ext.launch_fused_adam_step (src/mlx_extensions.cpp:75-236,
 * bound at :240-244): in place over contiguous pools ``theta/m/v [max_gaussians, dim]``
 * with dense gradients ``g [num_active, dim]`` and ``indices [num_active]``
 * (logical -> physical row).  Semantics of the reference kernel (:102-152):
 * NaN gradients -> 0, weight decay, NaN/Inf moments and step -> 0, float32
 * bias corrections, clamp to [a_min, a_max].  Addresses are device pointers
 * carried as integers, as in the reference. */
int gs_launch_fused_adam_step(uint64_t theta_addr, uint64_t g_addr, uint64_t m_addr, uint64_t v_addr,
                              uint64_t indices_addr, size_t max_gaussians, size_t num_active, int dim,
                              float lr, float beta1, float beta2, float eps, float weight_decay, int step,
                              float a_min, float a_max, gs_stream_t stream);

/* Drop-in for mlx_gsplat_ext.clear_buffer_cache (src/mlx_extensions.cpp:19-36, :245-246).
 * Device pointers need no wrapping on CUDA, so there is no cache; returns GS_OK. */
int gs_clear_buffer_cache(void);

#define GS_ADAM_FUSED 0 /* the Metal kernel's semantics (scrub + clamp, float32 bias corrections) */
#define GS_ADAM_PURE 1  /* mlx_gsplat/optimizer.py:146-175: lr_scale, float64 bias corrections, no scrub/clamp */
#define GS_ADAM_EXACT 0x100 /* OR into gs_fused_adam_slab's mode: IEEE-rounded sqrt and division in the step */

/* One parameter group with explicit row strides (pools whose rows are views
 * into a wider slab).  ``grad_scale`` multiplies g first (1/world_size after
 * a gradient all-reduce).  ``lr``/``beta1``/``beta2`` are the caller's float64
 * values: GS_ADAM_FUSED rounds them to float32 as the Metal kernel's
 * arguments are; GS_ADAM_PURE forms 1 - beta and the bias corrections in
 * float64 first, as the pure-MLX step does with Python floats. */
int gs_fused_adam_group(float* theta, const float* g, float* m, float* v, const int32_t* indices,
                        int64_t num_active, int dim, int64_t pool_stride, int64_t g_stride,
                        double lr, double beta1, double beta2, float eps, float weight_decay, int step,
                        float a_min, float a_max, float lr_scale, float grad_scale, int mode,
                        gs_stream_t stream);

/* All groups of a pooled slab in one float4-vectorised launch.  Pools are
 * ``[max, stride]`` with ``stride % 4 == 0`` and 16-byte-aligned bases;
 * columns [0, ncols) are parameters, the rest padding (left untouched).
 * Per column: clamp bounds ``col_lo/col_hi`` and ``col_lr_scale`` (host arrays
 * of ncols, ncols <= 64).  When ``quat_col >= 0`` (a multiple of 4) the four
 * columns from quat_col are renormalised after the update,
 * q / sqrt(sum q^2 + 1e-8) (mlx_gsplat/trainer.py:380-387).
 * When ``visible_words`` is given (bit r of word r/32 set = row r was seen
 * this step, the bitmask gs_cull leaves in its scratch), a row whose bit is
 * clear does not read g: its gradient is the host row ``unseen_grad_host``
 * (ncols floats), so the caller needs no gradient rows for unseen Gaussians.
 * Rounding: m and v are always rounded exactly as the per-element update
 * (gs_fused_adam_group) rounds them.  The step m / (sqrt(v) / sqrt(bc2) + eps)
 * uses the hardware approximate square root and reciprocal (a few ulp of the
 * step, relative error below 1e-6) unless ``mode`` has GS_ADAM_EXACT, which
 * makes every operation IEEE round-to-nearest (bit-identical to
 * gs_fused_adam_group, at a higher instruction cost).  ``grad_bias_host``
 * (ncols floats, or NULL) is added to every row's gradient before
 * ``grad_scale`` (the regulariser of rows summed over GPUs, added once here
 * instead of by every GPU).
 * Narrow gradient rows: with ``g_cols`` < ncols only columns [0, g_cols) of a
 * gradient row hold gradients; column c >= g_cols takes
 * g[count_col] * count_coef_host[c] (ncols floats) instead — a column whose
 * gradient is only the constant regulariser of each view that saw the row,
 * rebuilt from the row's view count (``count_col`` of gs_gaussian_grads).
 * g_cols = ncols (count_col, count_coef_host unused) reads full rows.
 * ``row_select`` (needs visible_words): GS_ROWS_ALL updates every row;
 * GS_ROWS_SEEN only the rows whose visibility bit is set, GS_ROWS_UNSEEN only
 * the others — two launches with the same ``step``, one per set, give the
 * update of one launch over all rows, and the unseen set needs nothing of
 * the rasterizer's output (it can run as soon as the cull has run). */
#define GS_ROWS_ALL 0
#define GS_ROWS_SEEN 1
#define GS_ROWS_UNSEEN 2
int gs_fused_adam_slab(float* theta, const float* g, float* m, float* v, const int32_t* indices,
                       int64_t num_active, int ncols, int64_t stride, int64_t g_stride,
                       const float* col_lo, const float* col_hi, const float* col_lr_scale, int quat_col,
                       double lr, double beta1, double beta2, float eps, float weight_decay, int step,
                       float grad_scale, int mode, const uint32_t* visible_words, const float* unseen_grad_host,
                       const float* grad_bias_host, int g_cols, int count_col, const float* count_coef_host,
                       int row_select, gs_stream_t stream);

/* ------------------------------------------------------------------ cull */

/* frustum_culling_mlx (mlx_gsplat/rendering.py:41-94): writes the ascending
 * active ids i in [0, n) that pass  z > near, z < far, the 50 px tolerance
 * box around the image and logit >= opacity_threshold (skipped when
 * g->opac is NULL) into ``out_ids`` and their number into ``*out_count``
 * (device int32).  On return the scratch starts (at its first 256-byte
 * boundary) with the visibility bitmask: bit i of 32-bit word i/32 is set when
 * id i passed.  Camera-space z and the projected centre are computed in
 * float32 with every product and sum rounded separately, left to right.
 * Scratch: ``gs_cull_scratch_bytes(n)`` bytes at ``scratch`` (16-byte aligned). */
size_t gs_cull_scratch_bytes(int64_t n);
int gs_cull(const gs_gaussians* g, int64_t n, const gs_camera* cam, float near_plane, float far_plane,
            float opacity_threshold, int32_t* out_ids, int32_t* out_count, void* scratch,
            size_t scratch_bytes, gs_stream_t stream);

/* gs_cull for callers that cannot allocate device memory — it has no
 * counterpart in the reference.  Some hosts of this library cannot provide a
 * scratch buffer: a service binding the C ABI from a managed runtime (Go, JVM,
 * Node) that has no device allocator of its own, or a process whose device
 * memory is all owned by another framework's pool.  This entry point allocates
 * nothing (no cudaMalloc, no cudaFree, no allocating library call): its scratch
 * is a fixed ~1 MiB array built into the library, which every device that
 * loads the library keeps until the process exits.  The caller still passes
 * the inputs and the outputs (out_ids, out_count), exactly as for gs_cull.
 *  - n may be at most 8,388,608 (2^23) active ids; larger n returns
 *    GS_ERR_CAPACITY before any work.
 *  - The first call on each device looks up the array's device address
 *    (cudaGetSymbolAddress) with that device current; make that first call
 *    before any stream capture.  The address is kept with the id of the
 *    context it was taken in: after a cudaDeviceReset the next call (which
 *    then runs in a new context) looks it up again, so that call too should
 *    come before any stream capture.
 *  - All calls share the one array and each call overwrites it: calls that can
 *    overlap on the GPU (other streams, other host threads on the same device)
 *    race; serialise them. */
int gs_cull_noalloc(const gs_gaussians* g, int64_t n, const gs_camera* cam, float near_plane, float far_plane,
                    float opacity_threshold, int32_t* out_ids, int32_t* out_count, gs_stream_t stream);

/* ------------------------------------------------------------------ sort / scan */

/* Stable LSD radix sort of (key, value) uint32 pairs on bits [begin_bit, end_bit).
 * Sorted output lands in keys_out/vals_out.  ``vals_in`` may be NULL (for a
 * non-empty bit range): the values are then the input positions 0..n-1, so
 * vals_out receives the sorting permutation.  Scratch: gs_radix_sort_scratch_bytes(n). */
size_t gs_radix_sort_scratch_bytes(int64_t n);
int gs_radix_sort_pairs(const uint32_t* keys_in, const uint32_t* vals_in, uint32_t* keys_out,
                        uint32_t* vals_out, int64_t n, int begin_bit, int end_bit, void* scratch,
                        size_t scratch_bytes, gs_stream_t stream);

/* Exclusive prefix sum of n uint32 values; out[n] (one extra slot) receives the total. */
size_t gs_scan_scratch_bytes(int64_t n);
int gs_exclusive_scan_u32(const uint32_t* in, uint32_t* out, int64_t n, void* scratch, size_t scratch_bytes,
                          gs_stream_t stream);

/* ------------------------------------------------------------------ rasterizer */

/* Per visible Gaussian v (ids[v] is its active id): camera transform, EWA
 * projection, conic, sigmoid opacity and the SH <= 1 colour of
 * mlx_gsplat/rendering.py:153-244, written as a 48-byte splat record
 * ``splats[v]`` = {u, v, conic_a, conic_b}, {conic_c, conic_d, opacity, r},
 * {g, b, depth, 0}; the sortable depth key ``depth_keys[v]``; and
 * ``tile_counts[v]``, the number of 16x16 tiles binned for it.
 * ``bin_scratch`` (gs_bin_scratch_bytes(num_visible) bytes of device memory,
 * or NULL) carries binning state from here to gs_bin_emit of the same view:
 * the binned tiles of every small tile box as a bitmask, so that emission
 * does not test them again, and the list of splats with very large boxes,
 * which are counted (here) and emitted by whole CTAs instead of one warp. */
size_t gs_bin_scratch_bytes(int64_t num_visible);
int gs_project_forward(const gs_gaussians* g, const int32_t* ids, int64_t num_visible, const gs_camera* cam,
                       const gs_raster_settings* rs, float* splats, uint32_t* depth_keys,
                       uint32_t* tile_counts, void* bin_scratch, gs_stream_t stream);

/* Offsets of each visible Gaussian's binned entries in depth order:
 * offsets[r] = sum of tile_counts[order[q]] for q < r, and offsets[n] = the
 * total number of entries.  Scratch: gs_bin_offsets_scratch_bytes(n). */
size_t gs_bin_offsets_scratch_bytes(int64_t num_visible);
int gs_bin_offsets(const uint32_t* order, const uint32_t* tile_counts, int64_t num_visible, uint32_t* offsets,
                   void* scratch, size_t scratch_bytes, gs_stream_t stream);

/* Writes the tile-binned entries of every visible Gaussian: for depth rank r,
 * v = order[r], entries [offsets[r], offsets[r] + tile_counts[v]) get the tile
 * id in ``tile_keys`` and v in ``entry_vals``.  ``capacity`` bounds the
 * output arrays: a Gaussian whose entries would pass it writes nothing and
 * sets the device flag ``*overflow_flag = 1`` (the caller zeroes it first and
 * reads it back when it did not size the arrays from the scan total).
 * ``bin_scratch`` must be the one gs_project_forward filled for this view
 * (or NULL when that call had none). */
int gs_bin_emit(const float* splats, const uint32_t* order, const uint32_t* offsets, const uint32_t* tile_counts,
                int64_t num_visible, const gs_camera* cam, const gs_raster_settings* rs, uint32_t* tile_keys,
                uint32_t* entry_vals, int64_t capacity, int32_t* overflow_flag, void* bin_scratch,
                gs_stream_t stream);

/* Fills [start, end) per tile from the tile-sorted keys (ranges must hold
 * num_tiles entries; tiles without entries get {0, 0}). */
int gs_tile_ranges(const uint32_t* sorted_tile_keys, int64_t num_entries, int32_t num_tiles,
                   gs_tile_range* ranges, gs_stream_t stream);

/* Dispatch order for the compositing kernels: the num_tiles tile indices
 * ordered by decreasing entry count (bucketed; ties in any order), so the
 * heaviest tiles start first and the launch does not end on a few long tiles.
 * Results do not depend on the order; it only changes when each tile runs. */
int gs_tile_order(const gs_tile_range* ranges, int32_t num_tiles, int32_t* order, gs_stream_t stream);

#define GS_LOSS_NONE 0       /* no loss: the backward takes dL/dcolor, dL/dalpha buffers */
#define GS_LOSS_L1_U8 1      /* mean |C - target| with a uint8 HWC target (scaled by 1/255) */
#define GS_LOSS_L1_F32 2     /* mean |C - target| with a float32 HWC target */
#define GS_LOSS_MEAN 3       /* mean(C) (the reference trainer's loss without a target) */

/* Front-to-back compositing per 16x16 tile with shared-memory staged splats and
 * warp-level early termination: colour [RH, RW, 3] and alpha [RH, RW, 1]
 * (HWC float32), the final transmittance and the number of entries each pixel
 * consumed (for the backward).  With a loss mode, ``loss_partials[tile]``
 * receives that tile's sum of |C - target| (or of C).  Entry values at or
 * beyond ``num_visible`` are never dereferenced (they read splat 0).
 * ``tile_order`` (num_tiles entries from gs_tile_order, or NULL for tile index
 * order) only sets the order in which tiles are dispatched. */
int gs_render_forward(const gs_tile_range* ranges, const int32_t* tile_order, const uint32_t* entry_vals,
                      const float* splats,
                      int64_t num_visible, const gs_camera* cam, const gs_raster_settings* rs, float* out_color, float* out_alpha,
                      float* final_T, int32_t* n_contrib, int loss_mode, const void* target, float* loss_partials,
                      gs_stream_t stream);

/* The rasterizer's optional per-Gaussian alpha mask (mlx_gsplat/rendering.py:289-290:
 * alpha = clip(opacity * g, 0, 0.99) * mask[j]).  As in the reference, mask[j]
 * belongs to the j-th visible Gaussian in depth order (the reference applies it
 * after its depth argsort without permuting it), so ``order`` is the depth
 * sort's permutation (order[j] = visible index of depth rank j, from
 * gs_radix_sort_pairs on the depth keys).  Writes the multiplier (clamped to
 * [0, 1]: binning bounds a splat's reach by its unmasked opacity) into the last
 * float of each splat record and tightens the record's contribution cut to
 * opacity * mask.  Call it after the depth sort and before the compositing
 * kernels, which then need gs_raster_settings.alpha_mask = 1. */
int gs_apply_sorted_mask(float* splats, const int32_t* order, const float* mask, int64_t num_visible,
                         const gs_raster_settings* rs, gs_stream_t stream);

/* Diagnostic (no reference counterpart): the number of (pixel, splat) pairs
 * that take part in the compositing of one view — alpha >= alpha_cutoff
 * while the pixel's transmittance is >= transmittance_min, the pairs both
 * compositing kernels evaluate — added to ``*pairs`` (device uint64).  Runs
 * the forward's arithmetic without writing an image; the arguments mean what
 * they mean for gs_render_forward.  Used to state the compositing kernels'
 * work in pairs per second. */
int gs_render_pair_count(const gs_tile_range* ranges, const int32_t* tile_order, const uint32_t* entry_vals,
                         const float* splats, int64_t num_visible, const gs_camera* cam,
                         const gs_raster_settings* rs, unsigned long long* pairs, gs_stream_t stream);

/* Diagnostic (no reference counterpart): a kernel of ``blocks`` x 256 threads,
 * each running 16 independent fused multiply-add chains for ``iters``
 * iterations — as sm_100 paired (two-lane) instructions when ``paired``, else
 * scalar — writing one float per thread to ``out``.  ``*flops_per_launch``
 * receives the floating-point operations the launch performs.  Timed by the
 * caller, it measures the GPU's fp32 throughput: the denominator of the
 * compositing kernels' compute roofline. */
int gs_fp32_peak_probe(float* out, int64_t out_len, int blocks, int iters, int paired, double* flops_per_launch,
                       gs_stream_t stream);

/* Back-to-front gradient of the compositing: recomputes transmittance from the
 * saved final value and accumulates per visible Gaussian, with warp-reduced
 * atomics, the 12-float record {du, dv, dconic_a, dconic_bc}, {dconic_d,
 * dopacity, dr, dg}, {db, 0, 0, 0} into ``splat_grads`` (zeroed by the caller).
 * dL/dcolor comes from ``dL_dcolor`` [RH,RW,3] (+ ``dL_dalpha`` [RH,RW,1],
 * may be NULL) for GS_LOSS_NONE, or is formed from the loss mode.
 * ``tile_order`` as in gs_render_forward. */
int gs_render_backward(const gs_tile_range* ranges, const int32_t* tile_order, const uint32_t* entry_vals,
                       const float* splats,
                       int64_t num_visible, const gs_camera* cam, const gs_raster_settings* rs, const float* out_color,
                       const float* final_T, const int32_t* n_contrib, int loss_mode, const void* target,
                       const float* dL_dcolor, const float* dL_dalpha, float* splat_grads, gs_stream_t stream);

/* Chains the splat gradients back to the Gaussian parameters (projection,
 * covariance, quaternion normalisation, sigmoid, SH colour and their clip
 * rules) and writes one gradient row per visible Gaussian.  When ``grad2d``
 * is not NULL also adds the densification statistic
 * sqrt(|dL/dmean|^2 + 1e-8) * |z| / fx to grad2d[table[id]] and 1 to
 * count[table[id]] (mlx_gsplat/trainer.py:300-318). */
int gs_project_backward(const gs_gaussians* g, const int32_t* ids, int64_t num_visible, const gs_camera* cam,
                        const float* splat_grads, const gs_gaussian_grads* out, float* grad2d, float* count,
                        gs_stream_t stream);

/* ------------------------------------------------------------------ export */

/* The rows of export_to_ply (mlx_gsplat/trainer.py:570-631) for the active
 * ids 0..num_active-1 of a pooled slab (physical row table[i], ``stride``
 * floats per row, the given column offsets): out[i] = means(3) | 0 0 0 |
 * colour columns | opacity logit clipped to [-5, 2] | log-scales clipped to
 * [-10, -2] | quaternion / (|q| + 1e-8), row-major float32 with
 * ``out_cols`` = 14 + color_cols columns (checked), the PLY vertex layout. */
int gs_export_rows(const float* theta, int64_t stride, const int32_t* table, int64_t num_active, int mean_col,
                   int opac_col, int scale_col, int quat_col, int color_col, int color_cols, float* out,
                   int64_t out_cols, gs_stream_t stream);

/* ------------------------------------------------------------------ loss */

/* The reference trainer's image loss with a target (mlx_gsplat/trainer.py:
 * 164-190, 276-279): l1_weight * mean|C - T| + dssim_weight * (1 - SSIM)/2,
 * SSIM per channel with an 11 x 11 window of ones/121 and zero padding 5,
 * averaged over pixels and channels (the trainer uses 0.8 and 0.2).  ``color``
 * is the rendered HWC float32 image, ``target`` HWC uint8 (scaled by 1/255,
 * ``target_is_u8`` = 1) or float32.  Writes the loss (device float) and, when
 * not NULL, SSIM (device float) and dL/dC (HWC float32, for
 * gs_render_backward with GS_LOSS_NONE).  Scratch:
 * gs_l1_dssim_scratch_bytes(width, height). */
size_t gs_l1_dssim_scratch_bytes(int32_t width, int32_t height);
int gs_l1_dssim_loss(const float* color, const void* target, int target_is_u8, int32_t width, int32_t height,
                     float l1_weight, float dssim_weight, float* loss_out, float* ssim_out, float* dL_dcolor,
                     void* scratch, size_t scratch_bytes, gs_stream_t stream);

/* ------------------------------------------------------------------ target image */

/* bilinear_resize_mlx (mlx_gsplat/rendering.py:6-38), the trainer's resize of
 * each step's target to the render size (mlx_gsplat/trainer.py:231-234):
 * ``src`` HWC [height_in, width_in, channels], uint8 (``src_is_u8`` = 1: each
 * value is first divided by 255 in float32, the trainer's ``image / 255.0``,
 * trainer.py:369) or float32; writes float32 HWC [height_out, width_out,
 * channels] to ``out``.  Sample x of the output reads input column
 * x * ((width_in - 1) / max(1, width_out - 1)) (the scale rounded to float32)
 * between its floor and the next column, likewise in y; every float32
 * operation is the reference's, in its order, so results are bit-identical.
 * Equal sizes give the input unchanged (scaled by 1/255 for uint8). */
int gs_resize_bilinear(const void* src, int src_is_u8, int32_t width_in, int32_t height_in, int32_t channels,
                       float* out, int32_t width_out, int32_t height_out, gs_stream_t stream);

/* ------------------------------------------------------------------ multi-GPU */

/* Barrier across the ``world`` GPUs of a group (no reference counterpart: the
 * reference runs on one device).  ``peer_pads`` is a device array of the
 * group's signal-pad addresses (uint32 [channels x world] in peer-mapped
 * symmetric memory, zeroed before first use); every GPU calls with the same
 * channel and the same epoch sequence (one more per call and channel).
 * Orders all earlier work of every GPU (multimem gradient reductions
 * included) before all later work.  Polling is bounded by ``max_polls``
 * (about 100 ns each): on timeout ``*error_flag`` is set to 1 and the kernel
 * returns. */
int gs_group_barrier(uint32_t* const* peer_pads, int32_t rank, int32_t world, int32_t channel, uint32_t epoch,
                     int32_t* error_flag, int64_t max_polls, gs_stream_t stream);

/* Sum over the group's GPUs of rows [first_row, first_row + num_rows) of a
 * row slab (``stride`` floats per row, a multiple of 4) in symmetric memory,
 * through its NVLink multicast address: every 16 bytes are loaded reduced
 * across all GPUs' copies and stored back to all of them.  Each GPU calls it
 * on a disjoint range between two gs_group_barrier calls (after every GPU
 * wrote its rows; before anyone reads the sums); together the calls leave the
 * same sums in every copy.  ``error_flag`` (device int32, may be NULL): the
 * flag the group barriers set when a wait gives up; when it is non-zero the
 * call reads and writes nothing, so a partial sum is never broadcast. */
int gs_rows_sum_multicast(float* multicast_rows, int64_t first_row, int64_t num_rows, int64_t stride,
                          const int32_t* error_flag, gs_stream_t stream);

/* The slab Adam of one GPU of a views-data-parallel group, fused with the
 * group's gradient sum and parameter broadcast (no reference counterpart: the
 * reference runs on one device).  The GPU updates the rows whose physical slot
 * it owns (slot % world == rank): it reads each such row's gradient summed over
 * every GPU's copy of the gradient rows through their NVLink multicast address
 * ``g_multicast`` (rows by active id, ``g_stride`` floats, narrow rows as in
 * gs_fused_adam_slab), updates theta, m and v in its own memory, and stores the
 * first ``hot_cols`` columns of the new theta row to every GPU through the
 * parameter slab's multicast address ``theta_multicast`` (the columns the
 * rasterizer reads every step; the other columns and the moments stay with the
 * owner until the caller gathers them).  Fused semantics with the approximate
 * step; ``grad_scale`` and ``grad_bias_host`` as in gs_fused_adam_slab.  Call
 * it between two gs_group_barrier calls: after every GPU wrote its gradient
 * rows, before any GPU reads parameters again.  ``error_flag`` (device int32,
 * may be NULL): the flag those barriers set when a wait gives up; when it is
 * non-zero the update is skipped entirely (no partial sums are applied). */
int gs_fused_adam_slab_sharded(float* theta, float* theta_multicast, const float* g_multicast, float* m, float* v,
                               const int32_t* indices, int64_t num_active, int ncols, int64_t stride,
                               int64_t g_stride, const float* col_lo, const float* col_hi, int quat_col, double lr,
                               double beta1, double beta2, float eps, float weight_decay, int step, float grad_scale,
                               const float* grad_bias_host, int g_cols, int count_col, const float* count_coef_host,
                               int rank, int world, int hot_cols, const int32_t* error_flag, gs_stream_t stream);

/* ------------------------------------------------------------------ pool / densify */

/* Row flags of the densify step. */
#define GS_FLAG_PRUNE 1  /* the row is pruned */
#define GS_FLAG_REFINE 2 /* the row is cloned or split into two children */
#define GS_FLAG_SPLIT 4  /* the refinement shrinks the scales by log(1.6) (split, not clone) */

/* Ordered stream compaction: for every r < n with (flags[r] & mask) == value,
 * in ascending r, writes gather ? gather[r] : r to out and the number of rows
 * to *out_count (device int32).  Scratch: gs_cull_scratch_bytes(n).  Used for
 * the pruned slots (allocator.py:200-204), the refined rows and the kept
 * indirection entries (allocator.py:276-277). */
int gs_compact_flags(const uint8_t* flags, int64_t n, uint8_t mask, uint8_t value, const int32_t* gather,
                     int32_t* out, int32_t* out_count, void* scratch, size_t scratch_bytes, gs_stream_t stream);

/* The densify policy per active row (trainer.py:428-477): refine when the
 * average view-space gradient grad2d/max(count,1) > grad_threshold, split when
 * also max(exp(scale)) > small_threshold (else clone); prune on non-finite
 * parameters or | |q| - 1 | > quat_tolerance, and — when prune_geometry —
 * sigmoid(opacity) < dim_threshold or max(exp(scale)) > large_threshold.
 * ``g`` addresses the pooled rows through its table; grad2d/count are
 * indexed by physical slot.  Writes GS_FLAG_* bits to flags[num_active]. */
int gs_densify_masks(const gs_gaussians* g, const float* grad2d, const float* count, int64_t num_active,
                     float grad_threshold, float small_threshold, float large_threshold, float dim_threshold,
                     float quat_tolerance, int prune_geometry, uint8_t* flags, gs_stream_t stream);

/* Child rows of the refined Gaussians (trainer.py:479-507): for child j, whose
 * parent row is theta[parent_slots[j]] and logical row refine_rows[j], writes
 * child1[j] and child2[j] (``stride`` floats each): means + 0.02 * noise
 * (noise_means1 / noise_means2, [n, 3]), scales - log(1.6) when split,
 * opacity logit * 0.95, quaternion / sqrt(|q|^2 + 1e-8) (child 2 after
 * + 0.01 * noise_quats2, [n, 4]), every other column copied. */
int gs_densify_children(const float* theta, int64_t stride, int ncols, const int32_t* parent_slots,
                        const int32_t* refine_rows, const uint8_t* flags, const float* noise_means1,
                        const float* noise_means2, const float* noise_quats2, int64_t num_children, int col_means,
                        int col_scales, int col_quats, int col_opac, float* child1, float* child2,
                        gs_stream_t stream);

/* theta[slots[j]] = vals[j] (row stride vals_stride), or the host row
 * ``reset_row_host`` when vals is NULL; m[slots[j]] and v[slots[j]] zeroed
 * (when given) and grad2d/count[slots[j]] zeroed (when given).  The split,
 * child and prune writes of allocator.py:229-273. */
int gs_pool_write_rows(float* theta, float* m, float* v, int64_t stride, const int32_t* slots, int64_t n,
                       const float* vals, int64_t vals_stride, const float* reset_row_host, float* grad2d,
                       float* count, gs_stream_t stream);

/* out[j] = stack[top - 1 - j] for j < n: the LIFO pops of allocator.py:219. */
int gs_free_pop_reversed(const int32_t* stack, int64_t top, int64_t n, int32_t* out, gs_stream_t stream);

/* Writes ``pattern[0..stride)`` into every row r < n_rows of ``dst`` (row stride ``stride``). */
int gs_fill_rows(float* dst, int64_t n_rows, int64_t stride, const float* pattern_host, gs_stream_t stream);

/* Sets column ``col`` of rows [0, n_rows) to ``value`` (the periodic opacity
 * reset, mlx_gsplat/trainer.py:416-419). */
int gs_fill_column(float* dst, int64_t n_rows, int64_t stride, int col, float value, gs_stream_t stream);

/* Row gather/scatter (no reference counterpart; the sharded multi-GPU Adam
 * packs and unpacks the parameter columns the rasterizer reads): for j < n,
 * dst row (dst_idx ? dst_idx[j] : j) gets the first ``cols`` floats of src row
 * (src_idx ? src_idx[j] : j).  Strides in floats; cols and both strides
 * multiples of 4, bases 16-byte aligned.  Destination rows must be distinct. */
int gs_copy_rows(const float* src, int64_t src_stride, const int32_t* src_idx, float* dst, int64_t dst_stride,
                 const int32_t* dst_idx, int64_t n, int cols, gs_stream_t stream);

/* mask[slots[j]] = value for j < n, skipping slots outside [0, mask_len): the
 * allocator's active-slot mask updates of allocator.py:209-225 (pruned slots
 * cleared, child slots set). */
int gs_mark_slots(int8_t* mask, int64_t mask_len, const int32_t* slots, int64_t n, int value, gs_stream_t stream);

#ifdef __cplusplus
}
#endif
#endif /* GSPLAT_B200_H */
