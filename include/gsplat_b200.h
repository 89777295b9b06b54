/*
 * gsplat_b200 — C ABI of the B200-native (sm_100a) Gaussian-splatting
 * rasterizer path of mlx3D.
 *
 * The reference (mlx3D 0.2.0) has no native FFI: its device seam is
 * `mx.fast.metal_kernel(...)` wrapped by `@mx.custom_function` with a `.vjp`
 * (src/mlx3d/splatting/rasterize.py:292-403), and the elementwise MLX graphs of
 * projection.py / sh.py / tiles.py.  Each entry point below replaces one of
 * those seams; the comment above it names the reference code it stands for.
 *
 * Conventions
 *  - Plain device pointers (float32 / int32, C-contiguous) and sizes.  The
 *    library never allocates or frees caller memory; binning scratch is a
 *    caller-provided workspace sized by the *_workspace_*_bytes queries.
 *  - `stream` is a cudaStream_t (NULL = legacy default stream).  All calls are
 *    asynchronous on that stream; nothing synchronises the host.
 *  - Return value: GS_OK or a GS_ERR_* code; gs_last_error() returns a
 *    human-readable message for the last failing call on the calling thread.
 *  - Optional pointers may be NULL where marked.
 */
#ifndef GSPLAT_B200_H
#define GSPLAT_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define GS_OK 0
#define GS_ERR_INVALID_ARG 1
#define GS_ERR_CUDA 2
#define GS_ERR_CAPACITY 3
#define GS_ERR_TIMEOUT 4 /* a bounded device-side wait gave up (see gs_bin_status) */

/* Activation flags for gs_preprocess_forward/backward
 * (src/mlx3d/splatting/model.py:116-122): scales given as log-scales,
 * opacities given as logits. */
#define GS_ACT_EXP_SCALES 1
#define GS_ACT_SIGMOID_OPACITY 2

/* Pinhole camera as the projection sees it (src/mlx3d/cameras/cameras.py:139-173).
 * The reference mixes Python doubles with float32 arrays; each field below is
 * the float32 value the reference's expression ends up using:
 *   fx..cy      = float(camera.fx) ...
 *   neg_fx      = float(-camera.fx)                 (projection.py:83)
 *   clip_x      = float(1.3 * (0.5 * width / fx))   (projection.py:70-72)
 *   znear       = float(camera.znear)               (projection.py:136)
 *   center      = camera_center = -R^T t            (cameras.py:270-273)  */
typedef struct gs_camera {
  float R[9]; /* row-major world->camera rotation */
  float t[3];
  float fx, fy, cx, cy;
  float neg_fx, neg_fy;
  float clip_x, clip_y;
  float znear;
  float center[3];
  int32_t width, height;
} gs_camera;

/* Library version (major*10000 + minor*100 + patch). */
int gs_version(void);

/* Message of the last failing call on this thread ("" if none). */
const char* gs_last_error(void);

/* Number of kernels this library has launched in this process (all
 * devices, all threads); for launch accounting in benchmarks. */
uint64_t gs_kernel_launch_count(void);

/* ---------------------------------------------------------------- projection
 * project_gaussians: EWA projection of (N,3) means, (N,4) wxyz quats and (N,3)
 * linear scales to means2d (N,2), conics (N,3), depths (N), radii (N, float,
 * 0 = culled) and compensation (N).  Replaces src/mlx3d/splatting/projection.py:24-146. */
int gs_project_forward(const gs_camera* cam, const float* means, const float* quats,
                       const float* scales, int64_t n, float blur, int antialias,
                       float* means2d, float* conics, float* depths, float* radii,
                       float* compensation, void* stream);

/* Vector-Jacobian product of gs_project_forward (what MLX autodiff computes
 * through projection.py:56-146).  Any cotangent may be NULL (= zero).  Writes
 * (overwrites) g_means (N,3), g_quats (N,4), g_scales (N,3). */
int gs_project_backward(const gs_camera* cam, const float* means, const float* quats,
                        const float* scales, int64_t n, float blur, int antialias,
                        const float* g_means2d, const float* g_conics, const float* g_depths,
                        const float* g_compensation, float* g_means, float* g_quats,
                        float* g_scales, void* stream);

/* Lens model for the unscented projection (cameras.py:139-173, 290-317):
 * orthographic (fx, fy in pixels per world unit), or pinhole with
 * n_dist = 0 (none), Brown-Conrady dist = (k1, k2, p1, p2, k3) or, with
 * fisheye, OpenCV fisheye dist = (k1, k2, k3, k4). */
typedef struct gs_lens {
  int32_t orthographic;
  int32_t fisheye;
  int32_t n_dist;
  float dist[5];
} gs_lens;

/* project_gaussians_ut (projection.py:149-205): six sigma points
 * mean +- sqrt(3) * (columns of R(q) diag(s)) through the camera model,
 * sample mean and covariance; outputs as gs_project_forward. */
int gs_project_ut_forward(const gs_camera* cam, const gs_lens* lens, const float* means,
                          const float* quats, const float* scales, int64_t n, float blur,
                          int antialias, float* means2d, float* conics, float* depths,
                          float* radii, float* compensation, void* stream);

/* VJP of gs_project_ut_forward (what MLX autodiff computes through
 * projection.py:165-205 and cameras.py:290-317); cotangents may be NULL. */
int gs_project_ut_backward(const gs_camera* cam, const gs_lens* lens, const float* means,
                           const float* quats, const float* scales, int64_t n, float blur,
                           int antialias, const float* g_means2d, const float* g_conics,
                           const float* g_depths, const float* g_compensation, float* g_means,
                           float* g_quats, float* g_scales, void* stream);

/* ------------------------------------------------------------------------ SH
 * eval_sh(degree, sh (N,K,C), dirs (N,3)) -> (N,C), offset by +0.5, unclamped.
 * Replaces src/mlx3d/splatting/sh.py:41-78.  K >= (degree+1)^2. */
int gs_eval_sh_forward(int degree, const float* sh, int64_t n, int k, int channels,
                       const float* dirs, float* out, void* stream);

/* VJP of gs_eval_sh_forward: g_sh (N,K,C) (entries beyond (degree+1)^2 are
 * written as 0) and, if g_dirs != NULL, g_dirs (N,3). */
int gs_eval_sh_backward(int degree, const float* sh, int64_t n, int k, int channels,
                        const float* dirs, const float* g_out, float* g_sh, float* g_dirs,
                        void* stream);

/* ------------------------------------------------------ fused per-Gaussian pass
 * The per-Gaussian half of render_gaussians (src/mlx3d/splatting/render.py:56-80
 * plus tiles.py:54-65) in one kernel: projection, opacity * compensation,
 * view-dependent SH colour max(eval_sh(...), 0) with stop-gradient directions,
 * and the per-Gaussian tile count ("tiles touched").
 *   sh_dc   : (N, 3) rows with stride sh_dc_stride floats   (NULL: no colour)
 *   sh_rest : (N, K-1, 3) rows with stride sh_rest_stride   (NULL if degree 0)
 *   flags   : GS_ACT_* activations applied to scales / opacities first.
 * Outputs: means2d (N,2), conics (N,3), depths, radii, compensation (N),
 * colors (N,3) (ignored if sh_dc == NULL), opacities_out (N), tiles_touched (N). */
int gs_preprocess_forward(const gs_camera* cam, const float* means, const float* quats,
                          const float* scales, const float* opacities, const float* sh_dc,
                          int64_t sh_dc_stride, const float* sh_rest, int64_t sh_rest_stride,
                          int sh_degree, int64_t n, float blur, int antialias, int flags,
                          float* means2d, float* conics, float* depths, float* radii,
                          float* compensation, float* colors, float* opacities_out,
                          int32_t* tiles_touched, void* stream);

/* VJP of gs_preprocess_forward.  Cotangents g_means2d (N,2), g_conics (N,3),
 * g_colors (N,3), g_opacities_out (N) come from gs_rasterize_backward;
 * g_depths / g_compensation (N) may be NULL.  Writes g_means (N,3),
 * g_quats (N,4), g_scales (N,3), g_opacities (N) with respect to the raw
 * inputs (after the activations in `flags`), and the SH gradient rows
 * g_sh_dc / g_sh_rest with the same strides as the inputs. */
int gs_preprocess_backward(const gs_camera* cam, const float* means, const float* quats,
                           const float* scales, const float* opacities, const float* sh_dc,
                           int64_t sh_dc_stride, const float* sh_rest, int64_t sh_rest_stride,
                           int sh_degree, int64_t n, float blur, int antialias, int flags,
                           const float* g_means2d, const float* g_conics,
                           const float* g_colors, const float* g_opacities_out,
                           const float* g_depths, const float* g_compensation,
                           float* g_means, float* g_quats, float* g_scales,
                           float* g_opacities, float* g_sh_dc, float* g_sh_rest,
                           void* stream);

/* View-batched VJP of gs_preprocess_forward: the gradient with respect to the
 * raw inputs summed over n_views views of the same n Gaussians (the sum of
 * n_views gs_preprocess_backward calls, in one pass over the parameters).
 * cams: DEVICE array of n_views gs_camera.  g_screen: per view, rows of 9
 * floats per Gaussian (dL/d means2d 2, conic 3, colour 3, effective opacity
 * 1, as gs_rasterize_backward produces them), view v at g_screen +
 * v * view_stride.  Outputs as gs_preprocess_backward (written, not added).
 * Serves data parallelism over views: a rank that owns a slice of the
 * Gaussians receives every rank's cotangents for that slice (all-to-all)
 * and produces its slice of the summed gradient.  The reference has no
 * multi-device path; its single-view counterpart is MLX autodiff through
 * projection.py / sh.py / render.py:56-80. */
int gs_preprocess_backward_views(const gs_camera* cams, int n_views, const float* means,
                                 const float* quats, const float* scales, const float* opacities,
                                 const float* sh_dc, int64_t sh_dc_stride, const float* sh_rest,
                                 int64_t sh_rest_stride, int sh_degree, int64_t n, float blur, int antialias,
                                 int flags, const float* g_screen, int64_t view_stride, float* g_means,
                                 float* g_quats, float* g_scales, float* g_opacities, float* g_sh_dc,
                                 float* g_sh_rest, void* stream);

/* gs_preprocess_backward_views with the cotangents of each view given as
 * four arrays instead of packed rows: cotangents is a DEVICE array of
 * 4 * n_views pointers, for view v: dL/d means2d (n,2), conic (n,3), colour
 * (n,3) and effective opacity (n) of Gaussian 0 of the slice.  The arrays
 * may live in other GPUs' memory (mapped with gs_peer_open): the kernel
 * reads them with peer loads over NVLink, so a rank reduces its slice of
 * every rank's cotangents without an all-to-all.  No reference
 * counterpart (see gs_preprocess_backward_views). */
int gs_preprocess_backward_views_peer(const gs_camera* cams, int n_views, const float* means,
                                      const float* quats, const float* scales, const float* opacities,
                                      const float* sh_dc, int64_t sh_dc_stride, const float* sh_rest,
                                      int64_t sh_rest_stride, int sh_degree, int64_t n, float blur,
                                      int antialias, int flags, const float* const* cotangents, float* g_means,
                                      float* g_quats, float* g_scales, float* g_opacities, float* g_sh_dc,
                                      float* g_sh_rest, void* stream);

/* Device buffers shared between the processes of one node (CUDA IPC; no
 * reference counterpart: mlx3D is single-device).  gs_peer_alloc allocates
 * `bytes` of device memory on the current device and writes its 64-byte
 * handle; another process maps it with gs_peer_open (its GPU must be able to
 * reach this one: NVLink / NVSwitch peers) and unmaps it with gs_peer_close
 * before the owner calls gs_peer_free. */
#define GS_PEER_HANDLE_BYTES 64
int gs_peer_alloc(size_t bytes, void** dev_ptr, void* handle);
int gs_peer_open(const void* handle, void** dev_ptr);
int gs_peer_close(void* dev_ptr);
int gs_peer_free(void* dev_ptr);

/* ------------------------------------------------------------------- binning
 * bin_gaussians (src/mlx3d/splatting/tiles.py:19-182), split where the
 * reference itself synchronises with the host (tiles.py:68):
 *   1. gs_tile_counts     tiles touched per Gaussian          (tiles.py:49-65)
 *   2. gs_bin_begin       stable depth order of the touching Gaussians and the
 *                         duplicate total D, written to *d_total on the device
 *                                                             (tiles.py:67-68,167-168)
 *   3. (host reads D, sizes the D-dependent buffers)
 *   4. gs_bin_end         duplicates, stable sort by tile, tile ranges
 *                                                             (tiles.py:77-89,169-182)
 * The result equals the reference's key order tile*N + rank(depth): ties in
 * depth keep Gaussian index order.  Empty tiles get the range [0, 0). */
int gs_tile_counts(const float* means2d, const float* radii, int64_t n, int width, int height,
                   int32_t* tiles_touched, void* stream);

size_t gs_bin_workspace_n_bytes(int64_t n);
size_t gs_bin_workspace_d_bytes(int64_t d);

/* D = sum of tiles_touched into *d_total (device), on its own: lets the host
 * read D back while gs_bin_begin's depth sort is still running. */
int gs_bin_total(const int32_t* tiles_touched, int64_t n, int64_t* d_total, void* stream);

int gs_bin_begin(const float* depths, const int32_t* tiles_touched, int64_t n, void* ws_n,
                 size_t ws_n_bytes, int64_t* d_total, void* stream);

int gs_bin_end(const float* means2d, const float* radii, int64_t n, int64_t d, int width,
               int height, void* ws_n, size_t ws_n_bytes, void* ws_d, size_t ws_d_bytes,
               int32_t* sorted_ids, int32_t* tile_ranges, void* stream);

/* Bounded device-side waits: the radix passes and the offsets scan of
 * gs_bin_begin / gs_bin_end (blocks wait for earlier blocks' counts) and the
 * bulk (TMA) staging of gs_preprocess_forward / _backward (threads wait for
 * the copy engine).  A wait that runs out leaves that block's output
 * unwritten and is counted on the device; this reads the total for the
 * current device (synchronous; reset != 0 clears it).  Always 0 unless a
 * GPU stalls for far longer than a kernel takes.  No counterpart in the
 * reference (its sort is mx.argsort; MLX stages nothing). */
int gs_wait_failures(uint64_t* count, int reset);

/* Status of the last gs_bin_begin / gs_bin_end on this workspace_n
 * (synchronises `stream`).  A binning look-back that gives up sets a bit in a
 * status word inside workspace_n: 1 = depth sort, 2 = offsets scan, 4 = tile
 * sort.  Every later binning kernel that depends on the failed stage does
 * nothing, and every tile range stays the empty [0, 0), so a compositor
 * launched on the outputs reads no Gaussian ids.  Returns GS_ERR_TIMEOUT when
 * the word is non-zero (*status_out receives it).  gs_bin_status_offset(n)
 * is the word's byte offset in workspace_n, for callers that copy it
 * asynchronously instead.  Replaces nothing in the reference (mx.argsort,
 * tiles.py:166-173, cannot time out). */
int gs_bin_status(const void* ws_n, size_t ws_n_bytes, int64_t n, uint32_t* status_out, void* stream);
size_t gs_bin_status_offset(int64_t n);

/* Test hook: the number of polls a binning look-back makes before it gives
 * up, on the current device (default 4194304).  0 makes every look-back that
 * has to wait give up at once, which exercises the GS_ERR_TIMEOUT path
 * without stalling anything.  No counterpart in the reference. */
int gs_set_wait_limit(int polls);

/* Hard z-buffer mesh rasterizer over tile-binned triangles
 * (src/mlx3d/renderer/rasterizer.py:29-79 and the call :150-162; the
 * triangles are binned by bin_gaussians on their bounding circles).
 * tri_xy (F, 3, 2) screen-space corners, tri_z (F, 3) camera-space depths,
 * sorted_ids / tile_ranges from the binning; writes pix_to_face (H, W)
 * (nearest triangle with depth > znear, -1 where none) and zbuf (H, W)
 * (its interpolated depth, 0 where none). */
int gs_mesh_rasterize(const float* tri_xy, const float* tri_z, int64_t n_faces, const int32_t* sorted_ids,
                      const int32_t* tile_ranges, int width, int height, float znear, int32_t* pix_to_face,
                      float* zbuf, void* stream);

/* bin_gaussians with the reference's refine_tiles option (`conics` given,
 * tiles.py:91-164): a (Gaussian, tile) duplicate of the square bounding box
 * is kept only if the minimum of the conic form a dx^2 + 2 b dx dy + c dy^2
 * over the tile rectangle is <= 12.  gs_tile_counts_refined replaces
 * gs_tile_counts (kept tiles per Gaussian), gs_bin_end_refined replaces
 * gs_bin_end; gs_bin_begin is shared.  conics (N,3) as gs_project_forward. */
int gs_tile_counts_refined(const float* means2d, const float* radii, const float* conics, int64_t n,
                           int width, int height, int32_t* tiles_touched, void* stream);
int gs_bin_end_refined(const float* means2d, const float* radii, const float* conics, int64_t n,
                       int64_t d, int width, int height, void* ws_n, size_t ws_n_bytes, void* ws_d,
                       size_t ws_d_bytes, int32_t* sorted_ids, int32_t* tile_ranges, void* stream);

/* No-allocation binning.  Has no counterpart in the reference: it exists
 * for callers that cannot allocate device memory (a renderer embedded in an
 * application whose GPU memory belongs to another allocator, a plugin host,
 * a fixed-pool server).  Same results as gs_tile_counts + gs_bin_begin +
 * gs_bin_end, with all scratch space in one file-scope __device__ array of
 * GS_STATIC_BIN_SCRATCH_BYTES (20 MiB) that every GPU loading this library
 * holds until process exit.  Limits: n <= GS_STATIC_BIN_MAX_N,
 * D <= GS_STATIC_BIN_MAX_D; larger sizes return GS_ERR_CAPACITY, as does a
 * sorted_ids capacity below D (*d_out then holds the D needed).  Reads D back
 * to the host (one synchronisation of `stream`).  The first call on a device
 * looks up the array's device address: make it before any stream capture.
 * The address is cached per device for the life of the process; after a
 * cudaDeviceReset the cached address is stale, so do not call this entry
 * point again in that process.  All calls share the array; calls that
 * overlap on the GPU race.  A depth-sort or scan wait that gives up returns
 * GS_ERR_TIMEOUT (found when D is read); a tile-sort wait that gives up
 * leaves every tile range empty and is counted by gs_wait_failures. */
#define GS_STATIC_BIN_MAX_N 131072
#define GS_STATIC_BIN_MAX_D 1048576
#define GS_STATIC_BIN_SCRATCH_BYTES (20u << 20)
int gs_bin_gaussians_static(const float* means2d, const float* radii, const float* depths,
                            int64_t n, int width, int height, int64_t d_capacity,
                            int32_t* sorted_ids, int32_t* tile_ranges, int64_t* d_out,
                            void* stream);

/* --------------------------------------------------------------- compositing
 * Forward tile compositor (gs_rasterize_forward Metal kernel,
 * src/mlx3d/splatting/rasterize.py:28-98, 345-361, and the depth kernel
 * :223-290).  `channels` colour/feature channels per Gaussian (0..64,
 * colors (N,channels)); background (channels) may be NULL (= 0).
 * Outputs (each may be NULL except final_T): image (H,W,channels),
 * final_T (H,W), n_contrib (H,W) int32, depth (H,W) (needs `depths`). */
int gs_rasterize_forward(const float* means2d, const float* conics, const float* colors,
                         int channels, const float* opacities, const float* depths,
                         const int32_t* sorted_ids, const int32_t* tile_ranges,
                         const float* background, int width, int height, int tiles_x,
                         int tiles_y, float* image, float* final_T, int32_t* n_contrib,
                         float* depth, void* stream);

/* Backward tile compositor (gs_rasterize_backward, rasterize.py:100-221,
 * 364-403).  grad_final_T may be NULL.  Zeroes, then accumulates
 * grad_means2d (N,2), grad_conics (N,3), grad_colors (N,channels),
 * grad_opacities (N). */
int gs_rasterize_backward(const float* means2d, const float* conics, const float* colors,
                          int channels, const float* opacities, int64_t n,
                          const int32_t* sorted_ids, const int32_t* tile_ranges,
                          const float* background, int width, int height, int tiles_x,
                          int tiles_y, const float* final_T, const int32_t* n_contrib,
                          const float* grad_image, const float* grad_final_T,
                          float* grad_means2d, float* grad_conics, float* grad_colors,
                          float* grad_opacities, void* stream);

/* ------------------------------------------------------------ training step
 * Photometric loss of GaussianTrainer._render_loss
 * (src/mlx3d/splatting/trainer.py:300-305): loss[0] = (1 - lambda) * L1 +
 * lambda * (1 - SSIM), loss[1] = L1, loss[2] = SSIM, with SSIM as
 * losses/image_metrics.py:29-85 (Gaussian window `window_size` / `sigma`,
 * zero padding, constants (0.01 max_val)^2 and (0.03 max_val)^2, means over
 * H*W*C).  pred / target (H, W, C); `loss` is a device float[3].  The
 * forward leaves per-pixel SSIM partials in the workspace
 * (gs_l1_ssim_workspace_bytes) for gs_l1_ssim_backward, which writes
 * grad_pred = grad_scale * d loss[0] / d pred. */
size_t gs_l1_ssim_workspace_bytes(int height, int width, int channels);
int gs_l1_ssim_forward(const float* pred, const float* target, int height, int width, int channels,
                       float lambda_dssim, float max_val, int window_size, float sigma,
                       void* workspace, size_t workspace_bytes, float* loss, void* stream);
int gs_l1_ssim_backward(const float* pred, const float* target, int height, int width, int channels,
                        float lambda_dssim, float max_val, int window_size, float sigma,
                        const void* workspace, size_t workspace_bytes, float grad_scale,
                        float* grad_pred, void* stream);
/* As gs_l1_ssim_backward with the scale read on the device,
 * grad_sign * grad_scale[0] (an autodiff cotangent, no host read-back), and
 * accumulate != 0 adding to grad_pred instead of overwriting it. */
int gs_l1_ssim_backward_dev(const float* pred, const float* target, int height, int width, int channels,
                            float lambda_dssim, int window_size, float sigma, const void* workspace,
                            size_t workspace_bytes, const float* grad_scale, float grad_sign, int accumulate,
                            float* grad_pred, void* stream);

/* L1 photometric loss mean |pred - target| over n floats (the benchmark
 * loss of the reference's examples/benchmark*.py and the L1 term of
 * trainer.py:300-305): loss[0] on the device, summed in a fixed order
 * (deterministic) through a gs_l1_workspace_bytes scratch buffer;
 * gs_l1_backward writes grad_pred = grad_loss[0] * sign(pred - target) / n. */
size_t gs_l1_workspace_bytes(int64_t n);
int gs_l1_forward(const float* pred, const float* target, int64_t n, void* workspace, size_t workspace_bytes,
                  float* loss, void* stream);
int gs_l1_backward(const float* pred, const float* target, int64_t n, const float* grad_loss, float* grad_pred,
                   void* stream);

/* Per-parameter Adam (mlx.optimizers.Adam as the trainer builds it,
 * trainer.py:128, update order of Adam.apply_single): per group
 *   m = b1 m + (1 - b1) g,  v = b2 v + (1 - b2) g^2,
 *   p -= lr m / (sqrt(v) + eps)                                  (bias_correction = 0)
 *   p -= (lr / (1 - b1^step)) m / (sqrt(v) / sqrt(1 - b2^step) + eps)  (bias_correction = 1)
 * All groups in one launch; `step` is the 1-based update count.  The betas are
 * doubles: b1, b2 and 1 - b1, 1 - b2 are each rounded to float32 from the
 * double value, as MLX does with the Python floats it is given. */
#define GS_ADAM_MAX_GROUPS 8
typedef struct gs_adam_group {
  float* param;
  const float* grad;
  float* m;
  float* v;
  int64_t n;
  float lr;
} gs_adam_group;
int gs_adam_step(const gs_adam_group* groups, int n_groups, double beta1, double beta2, float eps,
                 int bias_correction, int64_t step, void* stream);

#ifdef __cplusplus
}
#endif
#endif /* GSPLAT_B200_H */
