/*
 * gs_b200.h -- C ABI of the B200 Gaussian-splatting rasterizer.
 *
 * Every entry point takes raw DEVICE pointers, sizes and thresholds by value,
 * and a cudaStream_t (passed as void*; NULL means the legacy default stream).
 * Every launch is asynchronous on that stream. No entry point allocates
 * memory: outputs and scratch are caller-owned (the *_scratch_bytes queries
 * give the scratch sizes). No entry point synchronises the stream except
 * gs_read_total, gs_check_status and gs_sync. Every entry point returns a
 * status code (GS_OK = 0); no C++ exception crosses this boundary.
 *
 * Array layouts are those of the reference's tensors: fp32, C-contiguous,
 * means (N,3), scales (N,3), quaternions (N,4) in (x, y, z, w) order,
 * opacities (N), sh_dc (N,3), sh_rest (N,15,3), world_to_camera (4,4)
 * row-major, intrinsic (3,3) row-major, images (H,W,3).
 *
 * Reference interfaces replaced (ruguangyou/3dgs_from_scratch):
 *   src/cuda/rasterizer.cpp:141-464 -- the pybind11 module `cuda_rasterizer`
 *   src/cuda/kernel.cu:1113-1505    -- the launch_* host functions
 */
#ifndef GS_B200_H
#define GS_B200_H

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define GS_API __attribute__((visibility("default")))
#else
#define GS_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* ---- status codes ---------------------------------------------------- */
#define GS_OK 0
#define GS_ERR_INVALID_ARGUMENT 1   /* bad size, null pointer, misalignment */
#define GS_ERR_CUDA 2               /* a CUDA call failed: see gs_last_cuda_error */
#define GS_ERR_DEVICE_TIMEOUT 3     /* a bounded device-side wait gave up */
#define GS_ERR_CAPACITY 4           /* scratch too small / count beyond 2^30 */
#define GS_ERR_PEER 5               /* another rank reported an error in this step */

/* Tile edge in pixels; the reference hard-codes 16 (src/cuda/wrapper.py:267). */
#define GS_TILE 16

/* Library version (2: gs_blend_forward / gs_blend_backward take the reach
 * buffer and the tile order), last CUDA error code seen, and the number of kernels this
 * library has launched since load (for launch accounting in benchmarks). */
GS_API int gs_version(void);
GS_API int gs_last_cuda_error(void);
GS_API uint64_t gs_launch_count(void);
/* Adds n (may be negative) to the launch count. Launches recorded into a
 * CUDA graph run at each replay, not at capture: a caller that captures
 * takes them off (negative n) and adds them at every replay. */
GS_API void gs_note_launches(int64_t n);

/* Device status word: bounded spin-waits (the sort's decoupled look-back,
 * the scan's look-back) record GS_ERR_DEVICE_TIMEOUT here instead of
 * hanging. gs_check_status synchronises `stream`, returns and clears it.
 * The optimizer kernels (gs_adam_step, gs_dp_adam_step) read it first and
 * skip their update while it is non-zero, so a step whose gradient may be
 * incomplete leaves the parameters and moments unchanged. No counterpart in
 * the reference (which has no device-side waits). */
GS_API int gs_check_status(void *stream);
GS_API int gs_sync(void *stream);

/* The status word copied to dst (one uint32, device memory) on `stream`,
 * not cleared; and the reverse merge: when *src is non-zero (e.g. the
 * maximum of every rank's exported word, reduced over NCCL), the local word
 * becomes GS_ERR_PEER unless it already holds a code. Data-parallel steps
 * that use an NCCL all-reduce merge every rank's status before the
 * optimizer, so that all ranks skip (or apply) the update together. No
 * counterpart in the reference. */
GS_API int gs_status_export(uint32_t *dst, void *stream);
GS_API int gs_status_merge(const uint32_t *src, void *stream);

/* Self-test of the bounded waits: launches one thread that polls the device
 * word *flag_dev (which the caller leaves 0) until the spin limit, then
 * returns the status it recorded -- GS_ERR_DEVICE_TIMEOUT -- with the CUDA
 * context intact. No counterpart in the reference (which has no waits). */
GS_API int gs_selftest_bounded_wait(const uint32_t *flag_dev, void *stream);

/* The same probe without the read-back: it leaves GS_ERR_DEVICE_TIMEOUT in
 * the status word (as a kernel whose wait gave up would), for tests of the
 * kernels gated on it. No counterpart in the reference. */
GS_API int gs_selftest_set_timeout(const uint32_t *flag_dev, void *stream);

/* ---- reference module functions (rasterizer.cpp:141-440) ---------------- */

/* Replaces project_points (rasterizer.cpp:141-191; kernel.cu:411-500).
 * Outputs must be zeroed by the caller, mask (uint8, N) set to 1. */
GS_API int gs_project_points(int n, const float *means, const float *scales, const float *quats,
                      const float *opacities, const float *world_to_camera,
                      const float *intrinsic, float near_plane, float far_plane,
                      float min_opacity, float min_radius, float max_radius, int width,
                      int height, float *points_img, float *depths, float *cov_img,
                      float *conic, float *radii, uint8_t *mask, void *stream);

/* Replaces project_points_backward (rasterizer.cpp:193-232; kernel.cu:502-543).
 * Outputs must be zeroed by the caller (unmasked Gaussians are not written). */
GS_API int gs_project_points_backward(int n, const float *grad_points_img, const float *grad_conic,
                               const float *means, const float *scales, const float *quats,
                               const float *world_to_camera, const float *intrinsic,
                               const float *cov_img, const uint8_t *mask, int width,
                               int height, float *grad_means, float *grad_scales,
                               float *grad_quats, void *stream);

/* Replaces evaluate_spherical_harmonics (rasterizer.cpp:234-257;
 * kernel.cu:545-617). camera_pos is a device float[3]. */
GS_API int gs_evaluate_sh(int n, const float *camera_pos, const float *means, const float *sh_dc,
                   const float *sh_rest, const uint8_t *mask, int sh_sigmoid, float *colors,
                   void *stream);

/* Replaces evaluate_spherical_harmonics_backward (rasterizer.cpp:259-290;
 * kernel.cu:619-782). */
GS_API int gs_evaluate_sh_backward(int n, const float *grad_colors, const float *camera_pos,
                            const float *means, const float *sh_rest, const float *colors,
                            const uint8_t *mask, int sh_sigmoid, float *grad_means,
                            float *grad_dc, float *grad_rest, void *stream);

/* ---- tile intersection: count -> scan -> (host reads total) -> sort -------
 * Together these replace compute_tile_intersection (rasterizer.cpp:292-359;
 * kernel.cu:784-914 and the CUB sort of kernel.cu:1341-1388). The reference
 * reads the total with a blocking .item() (rasterizer.cpp:322); here the
 * caller reads the device total with gs_read_total once per view. */

/* Per-Gaussian tile-rectangle counts (kernel.cu:784-818) into `counts`. */
GS_API int gs_count_tiles(int n, const float *points_img, const float *radii, const uint8_t *mask,
                   int width, int height, int32_t *counts, void *stream);

/* Exclusive scan of n int32 counts into `offsets`, total into *total_dev
 * (device int64). Scratch: gs_scan_scratch_bytes(n). The offsets are int32:
 * once the running total passes INT32_MAX they wrap, *total_dev stays exact,
 * and the kernel records GS_ERR_CAPACITY in the device status word
 * (gs_check_status), so callers with large totals check either. */
GS_API size_t gs_scan_scratch_bytes(int n);
GS_API int gs_exclusive_scan(int n, const int32_t *counts, int32_t *offsets, int64_t *total_dev,
                      void *scratch, size_t scratch_bytes, void *stream);

/* Same exclusive scan as gs_exclusive_scan (int32 offsets that wrap past
 * INT32_MAX with GS_ERR_CAPACITY in the status word, exact int64 total), for
 * callers that pass their input and output buffers but may not allocate
 * device memory (e.g. a host application that owns all GPU memory through its
 * own allocator, or a frame loop that must not call cudaMalloc/cudaFree,
 * which synchronise the device). It allocates nothing: the look-back state
 * lives in a fixed device array inside the library of 8,193 64-bit words
 * (65,544 bytes: 2^24 / 2048 tile words plus one ticket word), so n is
 * limited to 16,777,216 (larger n returns GS_ERR_CAPACITY). The array's
 * address is looked up (cudaGetSymbolAddress) on a host thread's first call
 * in a context, so that first call should come before any stream capture.
 * All calls share the one array: calls whose kernels overlap on the GPU race,
 * so issue them on one stream or otherwise serialise them. This entry point
 * has no counterpart in the reference. */
GS_API int gs_exclusive_scan_noalloc(int n, const int32_t *counts, int32_t *offsets,
                                     int64_t *total_dev, void *stream);

/* Copies the device total (and the device status word) to the host;
 * synchronises `stream`. Returns GS_ERR_DEVICE_TIMEOUT if a bounded wait
 * gave up since the last check. */
GS_API int gs_read_total(const int64_t *total_dev, int64_t *total_host, void *stream);

/* Scratch for gs_tile_layout: n Gaussians, `total` pairs, width x height image. */
GS_API size_t gs_tile_layout_scratch_bytes(int n, int64_t total, int width, int height);

/* Builds the reference's tile layout (kernel.cu:820-914 with the CUB sort of
 * kernel.cu:1341-1388): the per-tile lists of Gaussian ids ordered by
 * (tile, depth bits), ties by Gaussian id, and the per-tile start offsets.
 * Done as two stable onesweep radix sorts -- the n Gaussians by depth bits,
 * then the pairs (emitted in that order) by tile id -- which yields the
 * reference's order exactly. counts are the per-Gaussian tile counts
 * (gs_count_tiles, 0 for culled Gaussians), total their sum. Outputs:
 * keys_sorted (the reference's 64-bit keys; may be NULL), ids_sorted (total),
 * indexing_offset (tiles_x * tiles_y). */
GS_API int gs_tile_layout(int n, const float *points_img, const float *radii, const float *depths,
                   const int32_t *counts, int64_t total, int width, int height,
                   int64_t *keys_sorted, int32_t *ids_sorted, int32_t *indexing_offset,
                   void *scratch, size_t scratch_bytes, void *stream);

/* The tile layout of gs_tile_layout without a host-side pair count, so that
 * a step's layouts queue behind its preprocess with no synchronisation (the
 * reference reads the count with a blocking .item() between the two,
 * rasterizer.cpp:319-322). The pair count is the scan of `counts` on the
 * device, written to *total_dev (int64); every kernel reads it there.
 * ids_sorted holds `capacity` entries and scratch is
 * gs_tile_layout_scratch_bytes(n, capacity, width, height). indexing_offset
 * holds num_tiles + 1 entries: the start offsets and, last, the end of the
 * last tile's list (pass total = -1 to gs_blend_forward / _backward). When
 * the count exceeds `capacity` nothing is emitted (every list is empty),
 * *total_dev still holds the count, and GS_ERR_CAPACITY is recorded in the
 * device status word -- the optimizer kernels then skip the step's update,
 * and the caller grows the buffers and repeats the step. */
GS_API int gs_tile_layout_capped(int n, const float *points_img, const float *radii,
                                 const float *depths, const int32_t *counts, int64_t capacity,
                                 int width, int height, int32_t *ids_sorted,
                                 int32_t *indexing_offset, int64_t *total_dev, void *scratch,
                                 size_t scratch_bytes, void *stream);

/* The same per-tile lists and offsets as gs_tile_layout_capped (same
 * arguments and contract: capacity, the device total, num_tiles + 1
 * offsets, nothing emitted and GS_ERR_CAPACITY recorded beyond the
 * capacity), built by binning instead of sorting all pairs: per-tile
 * counters, their scan, an atomic scatter of every Gaussian's id into its
 * tiles' buckets, and a sort of each bucket on its own by (depth bits, id)
 * -- the order the reference's stable 64-bit sort gives within a tile
 * (kernel.cu:820-914,1341-1388). Scratch: gs_tile_bins_scratch_bytes.
 * tile_order: NULL, or num_tiles ints that receive the blend order of the
 * tiles, as gs_tile_order writes it (computed in the same launch as the
 * offsets, saving gs_tile_order's launch). */
GS_API size_t gs_tile_bins_scratch_bytes(int n, int64_t capacity, int width, int height);
GS_API int gs_tile_bins(int n, const float *points_img, const float *radii, const float *depths,
                        const int32_t *counts, int64_t capacity, int width, int height,
                        int32_t *ids_sorted, int32_t *indexing_offset, int64_t *total_dev,
                        void *scratch, size_t scratch_bytes, int32_t *tile_order,
                        void *stream);

/* Scratch bytes for gs_tile_layout_views (0 on invalid arguments). totals
 * is a HOST array of num_views pair counts. */
GS_API size_t gs_tile_layout_views_scratch_bytes(int n, int num_views, const int64_t *totals,
                                                 int width, int height);

/* The tile layout of num_views views (1..64) of the same n Gaussians in one
 * cooperative launch -- the reference's compute_tile_intersection
 * (rasterizer.cpp:292-359: key emission, the CUB 64-bit sort and the tile
 * ranges of kernel.cu:820-914,1341-1388) for every view of a training step
 * at once, with the same per-tile order as gs_tile_layout (tile, then depth
 * bits, ties by Gaussian id). Inputs are per view at view * n (points_img,
 * radii as float2, depths, counts as written by
 * gs_preprocess_forward_views); totals is a HOST array of the views' pair
 * counts. Outputs: ids_sorted, the views' lists back to back (view v starts
 * at totals[0] + ... + totals[v - 1]); indexing_offset, (num_views, tiles)
 * start offsets local to each view's list. Grid-wide waits are bounded (a
 * timeout is reported through the status word). */
GS_API int gs_tile_layout_views(int n, int num_views, const float *points_img, const float *radii,
                                const float *depths, const int32_t *counts, const int64_t *totals,
                                int width, int height, int32_t *ids_sorted,
                                int32_t *indexing_offset, void *scratch, size_t scratch_bytes,
                                void *stream);

/* Stable LSD radix sort of (uint64 key, int32 value) pairs on key bits
 * [0, end_bit). Replaces radix_sort_double_buffer (kernel.cu:1341-1388).
 * keys/vals are sorted in place; keys_alt/vals_alt are ping-pong buffers of
 * the same size. Scratch: gs_sort_scratch_bytes(n). */
GS_API size_t gs_sort_scratch_bytes(int64_t n);
GS_API int gs_sort_pairs(int64_t n, uint64_t *keys, int32_t *vals, uint64_t *keys_alt,
                  int32_t *vals_alt, int end_bit, void *scratch, size_t scratch_bytes,
                  void *stream);

/* Replaces rasterize (rasterizer.cpp:361-395; kernel.cu:916-987). image
 * must be zeroed by the caller. n is the number of Gaussians (rows of the
 * per-Gaussian arrays); list entries outside [0, n) contribute nothing. work_final_t (float, H*W) and
 * work_pixel_end (int32, H*W) are caller-owned work buffers that receive
 * each pixel's final transmittance and end index. */
GS_API int gs_rasterize(int num_tiles, const int32_t *indexing_offset, int64_t total,
                 const int32_t *ids_sorted, int n, const float *points_img, const float *conic,
                 const float *opacities, const float *colors, int width, int height,
                 float alpha_threshold, float transmittance_threshold,
                 float chi_squared_threshold, float *image, float *work_final_t,
                 int32_t *work_pixel_end, void *stream);

/* Replaces rasterize_backward (rasterizer.cpp:397-440; kernel.cu:989-1111).
 * Gradient outputs must be zeroed by the caller (they are accumulated).
 * Like the reference, it first replays the forward per pixel (into the
 * caller-owned work buffers, H*W each). */
GS_API int gs_rasterize_backward(int num_tiles, const int32_t *indexing_offset, int64_t total,
                          const int32_t *ids_sorted, int n, const float *grad_image,
                          const float *points_img, const float *conic,
                          const float *opacities, const float *colors, int width,
                          int height, float alpha_threshold, float transmittance_threshold,
                          float chi_squared_threshold, float *grad_points_img,
                          float *grad_conic, float *grad_opacities, float *grad_colors,
                          float *work_final_t, int32_t *work_pixel_end, void *stream);

/* ---- fused render path (used by render() in the Python package) ---------
 * gs_preprocess_forward replaces project_points + evaluate_spherical_harmonics
 * + the colour shift/clamp of wrapper.py:264-265 + count_tiles + the total of
 * rasterizer.cpp:319-322 in one pass: projection, EWA covariance, conic,
 * radii, SH colour, per-Gaussian tile counts, and their sum added into
 * *total_dev (int64; zeroed by this call before the kernel). The splat record
 * is float[8] per Gaussian: conic (a, b, c), opacity, colour (r, g, b), 0.
 * Every output element is written (zeros for culled Gaussians). camera_pos is
 * the device float[3] -R^T t (wrapper.py:260). With activate = 1 the
 * parameters are the raw ones of the reference's training loop (log-scales,
 * unnormalised quaternions, opacity logits) and the kernel applies exp,
 * q / max(|q|, 1e-12) and sigmoid itself (scripts/train.py:135-140); the
 * splat record then holds the activated opacity. */
GS_API int gs_preprocess_forward(int n, const float *means, const float *scales, const float *quats,
                          const float *opacities, const float *sh_dc, const float *sh_rest,
                          const float *world_to_camera, const float *intrinsic,
                          const float *camera_pos, float near_plane, float far_plane,
                          float min_opacity, float min_radius, float max_radius, int width,
                          int height, int sh_sigmoid, int activate, float *points_img,
                          float *depths, float *radii, uint8_t *mask, float *splat,
                          int32_t *tile_counts, int64_t *total_dev, void *stream);

/* Blend forward over the splat records; also writes each pixel's final
 * transmittance and end index (one past its last contributing list entry).
 * Every pixel of the image (H,W,3) is written. total is the number of list
 * entries, or -1 when indexing_offset holds num_tiles + 1 entries whose last
 * is the end of the last tile's list (as gs_tile_layout_capped writes it).
 * reach: NULL, or one byte per list entry (as many as ids_sorted holds):
 * the forward stores there, for the entries it visits, which 8x8 pixel
 * blocks of its tile the entry's Gaussian can reach, and gs_blend_backward
 * given the same buffer (layout and splat records unchanged) reads them
 * instead of recomputing them. tile_order: NULL (block b blends tile b) or
 * the num_tiles tile indices in the order to blend them (gs_tile_order). */
GS_API int gs_blend_forward(int num_tiles, const int32_t *indexing_offset, int64_t total,
                     const int32_t *ids_sorted, int n, const float *points_img, const float *splat,
                     int width, int height, float alpha_threshold,
                     float transmittance_threshold, float chi_squared_threshold,
                     float *image, float *final_t, int32_t *pixel_end, uint8_t *reach,
                     const int32_t *tile_order, void *stream);

/* Blend backward: gradient outputs (grad_points_img (N,2), grad_splat (N,8))
 * must be zeroed by the caller (they are accumulated). total as for
 * gs_blend_forward (-1: the end is indexing_offset[num_tiles]). reach: NULL
 * (the masks are recomputed) or the buffer the forward of this view filled.
 * tile_order as for gs_blend_forward. */
GS_API int gs_blend_backward(int num_tiles, const int32_t *indexing_offset, int64_t total,
                      const int32_t *ids_sorted, int n, const float *points_img, const float *splat,
                      const float *grad_image, const float *final_t,
                      const int32_t *pixel_end, int width, int height,
                      float alpha_threshold, float transmittance_threshold,
                      float chi_squared_threshold, float *grad_points_img,
                      float *grad_splat, const uint8_t *reach, const int32_t *tile_order,
                      void *stream);

/* The tiles in the order to blend them, longest lists first (by a length
 * class: exact below 8 entries, then 8 classes per power of two), so that
 * the blend kernels' last wave holds short tiles. num_tiles and total as
 * for gs_blend_forward; order receives num_tiles tile indices. No
 * counterpart in the reference (its blend launches block b on tile b,
 * kernel.cu:1430-1433). */
GS_API int gs_tile_order(int num_tiles, const int32_t *indexing_offset, int64_t total,
                         int32_t *order, void *stream);

/* gs_preprocess_backward_views for the Gaussians first .. first + count - 1
 * of n_total: parameter and gradient pointers are those of all n_total
 * Gaussians (offset here), the per-view upstream arrays hold n_total
 * Gaussians per view. Lets the backward of one range of Gaussians overlap the
 * optimizer step of the previous range. */
GS_API int gs_preprocess_backward_views_range(
    int n_total, int first, int count, int num_views, const float *means, const float *scales,
    const float *quats, const float *opacities, const float *sh_dc, const float *sh_rest,
    const float *world_to_cameras, const float *intrinsics, const float *camera_positions,
    int width, int height, int sh_sigmoid, int activate, int accumulate, const uint8_t *mask,
    const float *grad_points_img, int gp_stride, const float *grad_splat, int gs_stride,
    float *grad_means, float *grad_scales, float *grad_quats, float *grad_opacities,
    float *grad_dc, float *grad_rest, void *stream);

/* Fused preprocess backward: projection, covariance and SH chain for every
 * Gaussian (zeros for culled ones), writing every output element. The
 * upstream gradients are read with element strides (so column views of a
 * packed buffer work): grad_points_img at gp[i*gp_stride + {0,1}], the splat
 * gradient at gs[i*gs_stride + {0..6}] (conic a,b,c, opacity, r, g, b).
 * grad_opacities receives the opacity gradient (may be NULL). With activate = 1
 * the parameters are raw (as for gs_preprocess_forward; opacities required)
 * and the gradients are w.r.t. the raw parameters (exp, normalisation and
 * sigmoid backward applied). With accumulate = 1 the gradients are added into
 * the outputs (the TMA engine's bulk reduce-add in L2) instead of written. */
GS_API int gs_preprocess_backward(int n, const float *means, const float *scales,
                           const float *quats, const float *opacities, const float *sh_dc,
                           const float *sh_rest, const float *world_to_camera,
                           const float *intrinsic, const float *camera_pos, int width,
                           int height, int sh_sigmoid, int activate, int accumulate,
                           const uint8_t *mask, const float *grad_points_img, int gp_stride,
                           const float *grad_splat, int gs_stride, float *grad_means,
                           float *grad_scales, float *grad_quats, float *grad_opacities,
                           float *grad_dc, float *grad_rest, void *stream);

/* gs_preprocess_forward for num_views cameras in one launch: each chunk of
 * parameters is read from HBM once and projected into every view. Camera v:
 * world_to_cameras + 16 v, intrinsics + 9 v, camera_positions + 3 v. Outputs
 * are (num_views, n, ...) arrays (view v's rows at element offset v * n of
 * each; splat (num_views, n, 8)), totals[v] the pair count of view v. No
 * counterpart in the reference, which preprocesses one view per call. */
GS_API int gs_preprocess_forward_views(int n, int num_views, const float *means,
                                       const float *scales, const float *quats,
                                       const float *opacities, const float *sh_dc,
                                       const float *sh_rest, const float *world_to_cameras,
                                       const float *intrinsics, const float *camera_positions,
                                       float near_plane, float far_plane, float min_opacity,
                                       float min_radius, float max_radius, int width, int height,
                                       int sh_sigmoid, int activate, float *points_img,
                                       float *depths, float *radii, uint8_t *mask, float *splat,
                                       int32_t *tile_counts, int64_t *totals, void *stream);

/* gs_preprocess_backward summed over num_views cameras in one launch: the
 * parameters are read once, the gradients written (or added) once. mask is
 * (num_views, n); view v's upstream gradients start at grad_points_img +
 * v * n * gp_stride and grad_splat + v * n * gs_stride. */
GS_API int gs_preprocess_backward_views(int n, int num_views, const float *means,
                                        const float *scales, const float *quats,
                                        const float *opacities, const float *sh_dc,
                                        const float *sh_rest, const float *world_to_cameras,
                                        const float *intrinsics, const float *camera_positions,
                                        int width, int height, int sh_sigmoid, int activate,
                                        int accumulate, const uint8_t *mask,
                                        const float *grad_points_img, int gp_stride,
                                        const float *grad_splat, int gs_stride,
                                        float *grad_means, float *grad_scales,
                                        float *grad_quats, float *grad_opacities, float *grad_dc,
                                        float *grad_rest, void *stream);

/* ---- training step helpers -------------------------------------------------
 * One-launch Adam over a flat fp32 buffer holding consecutive parameter
 * groups (group k = elements [group_ends[k-1], group_ends[k]), host arrays of
 * num_groups <= 8 entries, each end a multiple of 4, the last equal to n).
 * Same update as torch.optim.Adam (no amsgrad, no weight decay) with the
 * per-group learning rates and eps of scripts/train.py:17-44; `step` is the
 * 1-based step count used for bias correction. All four buffers 16-byte
 * aligned. */
GS_API int gs_adam_step(int64_t n, float *params, const float *grads, float *exp_avg,
                        float *exp_avg_sq, int num_groups, const int64_t *group_ends,
                        const float *lrs, const float *eps, float beta1, float beta2,
                        int64_t step, void *stream);

/* gs_adam_step split for replay from a CUDA graph: gs_adam_table fills a
 * host buffer of gs_adam_table_bytes() with the group table of step `step`
 * (the same bias corrections gs_adam_step folds in), the caller copies it to
 * device memory (8-byte aligned) before the launch, and gs_adam_step_table
 * applies the update reading the table there -- so a captured launch applies
 * whatever step the latest upload describes. Same update, bit for bit, and
 * the same status gating as gs_adam_step. */
GS_API size_t gs_adam_table_bytes(void);
GS_API int gs_adam_table(int64_t n, int num_groups, const int64_t *group_ends, const float *lrs,
                         const float *eps, float beta1, float beta2, int64_t step,
                         void *table_host, size_t table_bytes);
GS_API int gs_adam_step_table(int64_t n, float *params, const float *grads, float *exp_avg,
                              float *exp_avg_sq, const void *table_dev, float beta1, float beta2,
                              void *stream);

/* The same Adam update over num_ranges (<= 8) disjoint element ranges of the
 * flat buffers, range r (starts[r], counts[r]: multiples of 4, host arrays)
 * using group r of the device table (gs_adam_table's layout): the slices of
 * the six groups that hold a range of Gaussians, updated as soon as their
 * gradients are complete while the next range's are computed. Same update
 * and status gating as gs_adam_step. */
GS_API int gs_adam_step_ranges(float *params, const float *grads, float *exp_avg,
                               float *exp_avg_sq, int num_ranges, const int64_t *starts,
                               const int64_t *counts, const void *table_dev, float beta1,
                               float beta2, void *stream);

/* The reference's per-view training loss on the raw blended image (H*W*3 =
 * n floats): rendered = clamp(raw, 0, 1) * 255 (wrapper.py:294),
 * l1 = mean(|rendered / 255 - target / 255|) (scripts/train.py:187-191).
 * Adds sum |.| into *loss_sum (device double; divide by n for the mean) and
 * writes d l1 / d raw into grad_raw. target is float [0, 255] or, with
 * target_is_u8 = 1, uint8. */
GS_API int gs_l1_loss_grad(int64_t n, const float *raw_image, const void *target,
                           int target_is_u8, float *grad_raw, double *loss_sum, void *stream);

/* ---- SSIM and the L1 + SSIM training loss ------------------------------
 * No counterpart in the reference's native module: the reference calls the
 * external fused_ssim package (scripts/train.py:193-197, evaluate.py:57-61).
 * SSIM with the 11x11 Gaussian window (sigma 1.5), C1 = 0.01^2,
 * C2 = 0.03^2, zero padding; valid = 1 averages only over the pixels at
 * least 5 from every border (fused_ssim's padding="valid"). */

/* Scratch for gs_ssim_forward / gs_ssim_backward / gs_l1_ssim_loss_grad
 * (planes = 3 for the loss): three fp32 maps of planes * height * width. */
GS_API size_t gs_ssim_scratch_bytes(int planes, int height, int width);

/* SSIM of planar fp32 images (planes = N * C, each height x width): adds the
 * sum of the SSIM map over the counted pixels into *ssim_sum (device double;
 * divide by planes * H * W, or planes * (H - 10) * (W - 10) when valid),
 * and keeps in scratch what gs_ssim_backward needs. */
GS_API int gs_ssim_forward(int planes, int height, int width, const float *img1,
                           const float *img2, int valid, float *scratch, size_t scratch_bytes,
                           double *ssim_sum, void *stream);

/* d mean-SSIM / d img1, times *grad_out (a device float; NULL means 1), from
 * the scratch a gs_ssim_forward on the same images filled. */
GS_API int gs_ssim_backward(int planes, int height, int width, const float *img1,
                            const float *img2, const float *scratch, const float *grad_out,
                            float *grad_img1, void *stream);

/* The reference's training loss on one raw blended (height, width, 3) image
 * (scripts/train.py:183-203): rendered = clamp(raw, 0, 1) * 255 / 255,
 * target / 255, loss = (1 - lambda) * L1 + lambda * (1 - SSIM_valid).
 * Adds sum |rendered - target| into sums[0] and the sum of the valid SSIM map
 * into sums[1] (device doubles), and writes d loss / d raw into grad_raw.
 * height and width must exceed 10. */
GS_API int gs_l1_ssim_loss_grad(int height, int width, const float *raw_image,
                                const void *target, int target_is_u8, float ssim_lambda,
                                float *grad_raw, double *sums, float *scratch,
                                size_t scratch_bytes, void *stream);

/* ---- data-parallel optimizer step over NVLink / NVSwitch -----------------
 * No counterpart in the reference, which trains on one GPU with one view
 * per step (scripts/train.py:160-221); this is the multi-GPU extension of its
 * optimizer step (scripts/train.py:17-44,219-221).
 * One kernel per rank: every rank's flat gradient (n floats) is summed,
 * Adam is applied to this rank's shard [rank * n / world, (rank + 1) * n /
 * world) with this rank's shard of the Adam moments, and the new parameters
 * are written into every rank's flat parameter buffer. grad_ptrs, param_ptrs
 * and flag_ptrs are HOST arrays of `world` device pointers: every rank's
 * gradient buffer, parameter buffer and flag buffer (gs_dp_flag_words(
 * num_blocks) zero-initialised uint32 words), all addressable from this GPU
 * (peer mappings). mc_grad / mc_param are the NVSwitch multicast addresses
 * of the gradient and parameter buffers (then the sum is one
 * multimem.ld_reduce and the write one multimem.st per float4), or both NULL
 * (peer loads and stores). Every rank calls this with the same n, world,
 * num_blocks (<= gs_dp_max_blocks()) and epoch, a value larger (mod 2^31)
 * than at the previous call. n must be a multiple of 4 * world and all
 * buffers 16-byte aligned. grad_shard_out (n / world floats, or NULL)
 * receives this rank's shard of the summed gradient. Waits for other ranks
 * are bounded (4 s); a rank that never arrives makes gs_check_status report
 * GS_ERR_DEVICE_TIMEOUT. Each rank publishes whether its status word holds
 * an error when it arrives; if any does, every rank skips the update (a rank
 * without an error of its own then records GS_ERR_PEER). */
GS_API size_t gs_dp_flag_words(int num_blocks);
GS_API int gs_dp_max_blocks(void);
GS_API int gs_dp_adam_step(int world, int rank, void *const *grad_ptrs, void *const *param_ptrs,
                           void *const *flag_ptrs, void *mc_grad, void *mc_param, int64_t n,
                           float *exp_avg_shard, float *exp_avg_sq_shard, int num_groups,
                           const int64_t *group_ends, const float *lrs, const float *eps,
                           float beta1, float beta2, int64_t step, uint32_t epoch, int num_blocks,
                           float *grad_shard_out, void *stream);

/* ---- adaptive density control on the flat buffers -------------------------
 * The reference's Strategy (src/strategy.py:5-250) on the device. Flat
 * layout: six groups (means, log-scales, raw quaternions, opacity logits,
 * sh_dc, sh_rest: 3, 3, 4, 1, 3, 45 floats per Gaussian) at the element
 * offsets group_offsets[0..5] (HOST array) of one fp32 buffer; Adam moments
 * in the same layout. */

/* strategy.py:48-72 for one view: where both radii are positive,
 * grad_accum[i] += |(g_u * width / 2, g_v * height / 2)|, count[i] += 1.
 * Adds nothing while the device status word holds an error (a failed step,
 * which the caller repeats). */
GS_API int gs_densify_accumulate(int n, const float *grad_points, const float *radii, int width,
                                 int height, float *grad_accum, float *count, void *stream);

/* strategy.py:74-80,118-128: per Gaussian codes[i] = 0 pruned (sigmoid
 * opacity < prune_opacity, or with prune_by_scale max exp(log-scale) >
 * prune_scale), 1 kept, 2 kept and cloned (mean gradient grad_accum /
 * max(count, 1) > grow_grad and max scale < split_scale), 3 split (high
 * gradient, larger); and 0/1 flags (kept: codes 1, 2; cloned: 2; split: 3)
 * whose exclusive scans give the output slots of gs_densify_apply. */
GS_API int gs_densify_plan(int n, const float *params, const int64_t *group_offsets,
                           const float *grad_accum, const float *count, float prune_opacity,
                           int prune_by_scale, float prune_scale, float grow_grad,
                           float split_scale, uint8_t *codes, int32_t *keep_flags,
                           int32_t *clone_flags, int32_t *split_flags, void *stream);

/* strategy.py:83-233: writes the new flat buffer of n_keep + n_clone +
 * 2 n_split Gaussians, ordered [kept and not split][clones][split sample
 * 0][split sample 1], from the codes and the scanned slots (pos_*). Split
 * samples: mean + R(q / |q|) (exp(s) * z), log-scale log(exp(s) / scale_div),
 * the rest repeated; z from noise (2 x n_split x 3 floats, sample-major) or,
 * when noise is NULL, from Philox keyed by (seed, split slot). New Adam
 * moments (when the new_exp_avg* pointers are given): copied for kept
 * Gaussians, zero for clones and split samples. */
GS_API int gs_densify_apply(int n, const uint8_t *codes, const int32_t *pos_keep,
                            const int32_t *pos_clone, const int32_t *pos_split, int64_t n_keep,
                            int64_t n_clone, int64_t n_split, const float *params,
                            const int64_t *group_offsets, float *new_params,
                            const int64_t *new_group_offsets, const float *exp_avg,
                            const float *exp_avg_sq, float *new_exp_avg, float *new_exp_avg_sq,
                            const float *noise, uint64_t seed, float scale_div, void *stream);

/* strategy.py:235-250: opacity_logits = min(opacity_logits, threshold) and
 * the group's Adam moments (if given) zeroed. */
GS_API int gs_reset_opacities(int n, float *opacity_logits, float *exp_avg, float *exp_avg_sq,
                              float threshold, void *stream);

#ifdef __cplusplus
}
#endif

#endif /* GS_B200_H */
