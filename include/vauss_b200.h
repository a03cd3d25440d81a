/*
 * vauss_b200 — C ABI of the B200 (sm_100a) Gaussian-splat training step.
 *
 * Drop-in boundary for the reference trainer's GPU operators (voyager-so/vauss,
 * Brush-derived Rust/CubeCL).  Every entry point names the reference trait
 * method or kernel it replaces (paths relative to the reference project root).
 *
 * Conventions
 *  - All tensor pointers are DEVICE pointers owned by the caller, in the
 *    reference layouts: transforms [N,10] f32 = mean(3), quaternion (w,x,y,z)(4),
 *    log-scale(3); sh_coeffs [N,(d+1)^2,3] f32 or f16; raw_opacities [N] f32;
 *    images [H,W,4] f32 RGBA; ground truth [H,W] u32 packed RGBA8 (r low byte).
 *  - A vs_ctx owns one device, one stream and a grow-only workspace (from the
 *    device's default stream-ordered memory pool, whose release threshold the
 *    ctx raises so that this process keeps freed blocks for reuse).  A
 *    vs_frame owns the per-render intermediates (projected splats, the sorted
 *    intersection list, tile ranges) that the backward of that render reads.
 *  - Calls enqueue work on the ctx stream and return without waiting, except
 *    vs_render_forward, which reads the two projection counts back (the
 *    reference's render-count readback, src/render.rs:590-597) to size the
 *    intersection list exactly.
 *  - Every call returns a vs_status; vs_ctx_last_error() describes the last
 *    failure.  No call aborts the process.
 */
#ifndef VAUSS_B200_H
#define VAUSS_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define VS_API __attribute__((visibility("default")))

typedef enum vs_status {
  VS_OK = 0,
  VS_ERR_INVALID = 1,        /* bad argument (sizes, null pointers, degree) */
  VS_ERR_CAPACITY = 2,       /* a size limit was exceeded (message gives the size) */
  VS_ERR_CUDA = 3,           /* a CUDA runtime call failed */
  VS_ERR_DEVICE_TIMEOUT = 4, /* a bounded device-side wait gave up */
  VS_ERR_UNSUPPORTED = 5
} vs_status;

/* Pinhole view (crates/splat-train-render/src/camera.rs:12-97 + the
 * ProjectUniforms of src/kernels/types.rs:53-82). */
typedef struct vs_camera {
  float viewmat[12]; /* world->camera 3x4, column-major: rotation columns, translation */
  float fx, fy, cx, cy;
  float cam_pos[3];  /* view-direction origin of the SH colour */
  uint32_t img_w, img_h;
} vs_camera;

/* Render options (SplatOps::render arguments, crates/splat-train-render/src/lib.rs:53-115). */
typedef struct vs_render_cfg {
  int32_t mip;           /* SplatRenderMode::Mip: blur 0.1 + opacity compensation; else 0.3 */
  int32_t sh_degree;     /* 0..3 */
  int32_t sh_half;       /* sh_coeffs stored as IEEE binary16 */
  int32_t has_min_scale; /* min_scale [N] is read (Mip-Splatting 3D floor) */
  float log_scale_offset;
  float bg[3];           /* background colour */
} vs_render_cfg;

typedef struct vs_render_counts {
  uint32_t num_visible;
  uint32_t num_tiles;
  uint64_t num_intersections;
} vs_render_counts;

typedef struct vs_ctx vs_ctx;
typedef struct vs_frame vs_frame;

/* ---- context ------------------------------------------------------------ */
VS_API vs_status vs_ctx_create(int device, vs_ctx** out);
VS_API void vs_ctx_destroy(vs_ctx* ctx);
/* Run subsequent work on `cuda_stream` (a cudaStream_t; NULL = legacy default). */
VS_API vs_status vs_ctx_set_stream(vs_ctx* ctx, void* cuda_stream);
VS_API const char* vs_ctx_last_error(const vs_ctx* ctx);
/* Bytes of device workspace the ctx and its frames currently hold. */
VS_API uint64_t vs_ctx_workspace_bytes(const vs_ctx* ctx);
/* Number of kernels this ctx has launched (all entry points together). */
VS_API uint64_t vs_ctx_launch_count(const vs_ctx* ctx);
VS_API const char* vs_version(void);

VS_API vs_status vs_frame_create(vs_ctx* ctx, vs_frame** out);
VS_API void vs_frame_destroy(vs_frame* frame);

/* Frame buffers exposed for inspection and for the backward/optimizer calls. */
typedef enum vs_frame_field {
  VS_FIELD_COMPACT_FROM_GLOBAL = 0, /* u32 [N]   compact id + 1, 0 = culled */
  VS_FIELD_GLOBAL_FROM_COMPACT = 1, /* u32 [V]   */
  VS_FIELD_DEPTHS = 2,              /* f32 [V]   view-space z, compact order */
  VS_FIELD_TILE_COUNTS = 3,         /* u32 [V]   tiles hit, compact order */
  VS_FIELD_PROJECTED = 4,           /* f32 [V,12] [x,y,c00,c01, c11,opac,r,g, b,gid,0,0] */
  VS_FIELD_DEPTH_ORDER = 5,         /* u32 [V]   compact ids sorted by depth */
  VS_FIELD_ISECT_TILE = 6,          /* u32 [I]   tile id of each sorted intersection */
  VS_FIELD_ISECT_COMPACT = 7,       /* u32 [I]   compact id of each sorted intersection */
  VS_FIELD_TILE_RANGES = 8,         /* u32 [T,2] [start,end) after binning */
  VS_FIELD_TILE_USED_END = 9,       /* u32 [T]   one past the last intersection any pixel used */
  VS_FIELD_OPACITIES = 10,          /* f32 [N]   floored sigmoid opacity (0 if culled early) */
  VS_FIELD_MAX_RADIUS = 11          /* f32 [N]   screen radius (fraction of the image) */
} vs_frame_field;
VS_API vs_status vs_frame_buffer(vs_frame* frame, int32_t field, void** dev_ptr, uint64_t* count);
VS_API vs_status vs_frame_counts(const vs_frame* frame, vs_render_counts* out);
/* Copies up to max_bytes of a frame buffer into caller device memory (stream-ordered). */
VS_API vs_status vs_frame_copy(vs_frame* frame, int32_t field, void* dst_device, uint64_t max_bytes);

/* ---- render forward -------------------------------------------------------
 * Replaces SplatOps::render for training passes (crates/splat-train-render/
 * src/render.rs:315-349 -> render_cube :401-979): projection + SH colour
 * (project_forward.rs, project_visible.rs), depth sort, intersection emission,
 * stable tile sort and tile ranges (map_gaussians.rs, splat-train-sort,
 * get_tile_offset.rs), front-to-back compositing (kernels/rasterize.rs with
 * bwd_info).  Writes out_img [H,W,4] and visible [N] (1.0 where a splat
 * contributed to a pixel, else 0.0); counts_out may be NULL, and so may
 * visible when num_splats is 0 (the image is then the background).
 * Images are limited to 65535 tiles per side (VS_ERR_UNSUPPORTED beyond).
 * transforms must start on an 8-byte boundary (VS_ERR_INVALID otherwise);
 * f32 SH coefficients on a 16-byte boundary take the vector-load path. */
VS_API vs_status vs_render_forward(vs_ctx* ctx, vs_frame* frame, const vs_camera* cam, const vs_render_cfg* cfg,
                                   uint32_t num_splats, const float* transforms, const void* sh_coeffs,
                                   const float* raw_opacities, const float* min_scale, float* out_img,
                                   float* visible, vs_render_counts* counts_out);
/* vs_render_forward in three stages (it calls exactly these):
 * project = project_forward_kernel + project_visible_kernel + the count readback,
 * bin = depth sort + emission + tile sort + tile ranges, rasterize = compositing. */
VS_API vs_status vs_render_project(vs_ctx* ctx, vs_frame* frame, const vs_camera* cam, const vs_render_cfg* cfg,
                                   uint32_t num_splats, const float* transforms, const void* sh_coeffs,
                                   const float* raw_opacities, const float* min_scale, vs_render_counts* counts_out);
VS_API vs_status vs_render_bin(vs_ctx* ctx, vs_frame* frame);
VS_API vs_status vs_render_rasterize(vs_ctx* ctx, vs_frame* frame, float* out_img, float* visible);

/* Inference render: render_splats with RasterPass::Forward (crates/splat-train-
 * render/src/gaussian_splats.rs:511-527; kernels/rasterize.rs:380-410 with
 * bwd_info off): the same projection, binning and compositing, written as
 * packed RGBA8 out_rgba8 [H,W] u32 (r in the low byte; each channel
 * clamp(255 c, 0, 255) converted toward zero, alpha = 1 - T), with no
 * visible marks and no backward state (the frame cannot be differentiated). */
VS_API vs_status vs_render_image(vs_ctx* ctx, vs_frame* frame, const vs_camera* cam, const vs_render_cfg* cfg,
                                 uint32_t num_splats, const float* transforms, const void* sh_coeffs,
                                 const float* raw_opacities, const float* min_scale, uint32_t* out_rgba8,
                                 vs_render_counts* counts_out);

/* ---- loss ------------------------------------------------------------------
 * Replaces LossOps::image_loss_forward_train + image_loss_backward_coeffs
 * (crates/splat-train-loss/src/lib.rs:238-469, :821-1028) fused in one pass:
 * per-pixel loss (l1_w*|p-g| + ssim_w*SSIM, 11x11 Gaussian window sigma 1.5,
 * zero padding), weighted per-16x16-tile partial sums partials [3, tiles]
 * (weight 1/(3HW)), the total into *loss_dev (device f32, may be NULL), and
 * d(total)/d(pred) into dl_dpred [H,W,4] (alpha channel 0; may be NULL).
 * The reference training objective is l1_w = 1-w, ssim_w = -w (lib.rs:1227-1257). */
VS_API vs_status vs_loss(vs_ctx* ctx, uint32_t h, uint32_t w, const float* pred, const uint32_t* gt_packed,
                         float l1_w, float ssim_w, float* partials, float* loss_dev, float* dl_dpred);

/* ---- render backward -------------------------------------------------------
 * Replaces SplatBwdOps::rasterize_bwd (src/bwd/render_bwd.rs:27-155 ->
 * rasterize_backwards_planes.rs): per-splat gradients v_combined [V,10] =
 * [xy(2), conic(3), rgb(3), alpha, refine] in compact order (zeroed here). */
VS_API vs_status vs_rasterize_backward(vs_ctx* ctx, vs_frame* frame, const float* out_img, const float* v_output,
                                       float* v_combined);

/* ---- optimizer, reference mode ------------------------------------------- */
typedef struct vs_adam_cfg {
  float beta1, beta2, inv1, inv2, epsilon; /* inv1/inv2 = 1/(1-beta^t) */
  float lr_opac, opac_reg;
  uint32_t round_seed; /* stochastic-rounding stream (the step count) */
} vs_adam_cfg;

/* Replaces ProjectUpdateOps::project_update (src/bwd/project_update.rs:84-224,
 * kernels/project_update.rs:36-178): projection VJP fused with Adam on packed
 * 16/16 moments w_t [N,10], w_o [N] (geo_moments.rs).  lr_scale is a HOST
 * array of 10 per-column learning rates.  Writes color_dir [N+1,6] (row 0
 * zero), v_refine [N], grad_sq [N].  If variance != NULL the SH reduced second
 * moment [N] is also stepped here (crates/splat-train/src/optim.rs:454-469):
 * visible rows v = beta2*v + (1-beta2)*grad_sq, culled rows kept, or
 * v = (1-beta2)*grad_sq on the first step. */
VS_API vs_status vs_project_update(vs_ctx* ctx, vs_frame* frame, const vs_render_cfg* cfg, uint32_t num_splats,
                                   float* transforms, const void* sh_coeffs, float* raw_opacities,
                                   const float* min_scale, const float* v_combined, uint32_t* w_t,
                                   const float* lr_scale, uint32_t* w_o, const vs_adam_cfg* adam, float* color_dir,
                                   float* v_refine, float* grad_sq, float* variance, int32_t first_step);

/* Replaces QuantMomentOps::step_moment on the colour path
 * (crates/splat-train/src/quant_kernels.rs:277-376, step_kernel_w4 :597-714):
 * f16 SH coefficients [N*row_width], int8 first moment in 128-value blocks
 * (codes [blocks*32] u32, scales [blocks] f32), reduced second moment
 * variance [N]; lazy on culled rows (grad_rows == 0).  lr_scale is a HOST
 * array of row_width learning-rate factors. */
VS_API vs_status vs_sh_step(vs_ctx* ctx, uint32_t num_splats, uint32_t row_width, uint16_t* sh_f16,
                            const float* color_dir, const uint32_t* grad_rows, uint32_t* codes, float* scales,
                            const float* variance, const float* lr_scale, float beta, float factor, float inv1,
                            float inv2, float epsilon, float lr, uint32_t round_seed);

/* ---- optimizer, 8-bit m+v mode (the benchmark configuration) --------------
 * The Q8 entry points move parameters and codes in 16-byte pieces: the
 * parameter arrays (transforms, sh_coeffs, raw_opacities) and the code arrays
 * must start on 16-byte boundaries (VS_ERR_INVALID otherwise). */
typedef struct vs_q8_tensor { /* one parameter tensor's moments */
  uint8_t* m_codes;           /* [count] +128-biased signed codes */
  uint8_t* v_codes;           /* [count] sqrt(v) codes */
  float* m_scales;            /* [ceil(count/256)] absmax|m|/127 */
  float* v_scales;            /* [ceil(count/256)] absmax sqrt(v)/255 */
} vs_q8_tensor;

typedef struct vs_q8_cfg {
  float beta1, beta2, inv1, inv2, epsilon;
  float lr_transforms[10]; /* per-column learning rates */
  float lr_sh_dc, lr_sh_rest; /* coefficient 0 and coefficients 1.. */
  float lr_opac, opac_reg;
  uint32_t seed;              /* stochastic rounding stream (the step count) */
  /* housekeeping folded into the step (crates/splat-train/src/housekeep.rs) */
  float noise_scale, noise_limit;
  uint32_t noise_seed;
} vs_q8_cfg;

/* Single-view step: projection VJP from v_combined + Adam with 8-bit m and v
 * (blocks of 256, fp32 absmax scales, stochastic rounding) on transforms,
 * sh_coeffs (f32) and raw_opacities, plus the refine statistics
 * (refine_norm = max, vis_count += visible, max_screen = max) and the
 * low-opacity mean noise: two kernels (the VJP of the visible splats into
 * ctx scratch, then the optimizer).  stats pointers may be NULL.  min_scale
 * is the Mip 3D-filter floor the frame was rendered with (the reference's
 * project_update min_scale/has_min_scale, src/bwd/project_update.rs:84-110):
 * required when the render had one, ignored otherwise. */
VS_API vs_status vs_step_q8(vs_ctx* ctx, vs_frame* frame, const vs_render_cfg* cfg, uint32_t num_splats,
                            float* transforms, float* sh_coeffs, float* raw_opacities, const float* min_scale,
                            const float* v_combined,
                            vs_q8_tensor mom_t, vs_q8_tensor mom_sh, vs_q8_tensor mom_o, const vs_q8_cfg* q8,
                            const float* visible, float* refine_norm, float* vis_count, float* max_screen);

/* Dense projection VJP (the multi-view path, src/bwd/kernels/
 * project_backwards.rs:282-424 + the dense gather of burn_glue.rs:363-395):
 * ACCUMULATES this frame's gradients into grads [N, 10 + 3(d+1)^2 + 1]
 * (transforms | sh | raw opacity) and refine [N]; with vis_accum != NULL also
 * vis_accum += visible (the per-step count of views that saw each splat), and
 * a row whose vis_accum was 0 before the call and whose splat is visible now
 * is overwritten rather than accumulated, so readers that skip rows with
 * vis_accum == 0 need grads cleared only once, not every step. */
VS_API vs_status vs_vjp_dense(vs_ctx* ctx, vs_frame* frame, const vs_render_cfg* cfg, uint32_t num_splats,
                              const float* transforms, const void* sh_coeffs, const float* raw_opacities,
                              const float* min_scale, const float* v_combined, float* grads, float* refine,
                              const float* visible, float* vis_accum);

/* The compact form of vs_vjp_dense for the view-parallel exchange (no
 * reference counterpart): view `slot` (0..31) of this rank's step writes
 * rows [N, VS_COMPACT_ROW] = (transforms gradient 10 | raw-opacity gradient |
 * rasterizer colour gradient 3 | 0 0) of its visible splats, sets bit `slot`
 * of view_mask[g] for them, adds visible to vis_accum and the refine weight to
 * refine, and stores the camera position the VJP used into cam_out[0..2]
 * (cam_out[3] = 0); rows and cam_out are that slot's own arrays.  The SH
 * gradient is the colour gradient times the SH basis of the view direction
 * from cam_out, which the shard owner rebuilds (vs_adam_q8_peer with
 * row_format 1), so 64 bytes per splat and view are written and cross NVLink
 * instead of a dense row.  A splat whose bit was already set (the slot used
 * twice in a step) sets a device error that vs_ctx_check reports as
 * VS_ERR_INVALID; view_mask is cleared by the caller once per step. */
#define VS_COMPACT_ROW 16
VS_API vs_status vs_vjp_compact(vs_ctx* ctx, vs_frame* frame, const vs_render_cfg* cfg, uint32_t num_splats,
                                const float* transforms, const void* sh_coeffs, const float* raw_opacities,
                                const float* min_scale, const float* v_combined, float* rows, float* refine,
                                const float* visible, float* vis_accum, uint32_t* view_mask, uint32_t slot,
                                float* cam_out);

/* Adam (8-bit m+v) from dense gradients grads [N, width] (after the
 * cross-GPU all-reduce).  visible may be NULL (no noise); with opacities NULL
 * the noise gate uses sigmoid(raw_opacities). */
VS_API vs_status vs_adam_q8_dense(vs_ctx* ctx, uint32_t num_splats, int32_t sh_degree, float* transforms,
                                  float* sh_coeffs, float* raw_opacities, const float* grads, vs_q8_tensor mom_t,
                                  vs_q8_tensor mom_sh, vs_q8_tensor mom_o, const vs_q8_cfg* q8,
                                  const float* opacities, const float* visible);

/* ---- view-parallel step over NVLink peer memory -----------------------------
 * No reference counterpart (the reference trains on one device).  One process
 * per GPU; each rank renders its views into dense gradient rows, then every
 * rank updates its shard of the splats from the rows of all ranks read
 * directly over NVLink and stores the new parameters into every replica. */
#define VS_PEER_MAX 8
typedef struct vs_ipc_handle { uint8_t bytes[64]; } vs_ipc_handle;
/* cudaMalloc'd buffer whose IPC handle other ranks can open. */
VS_API vs_status vs_peer_alloc(vs_ctx* ctx, uint64_t bytes, void** dev_ptr, vs_ipc_handle* handle);
VS_API vs_status vs_peer_free(vs_ctx* ctx, void* dev_ptr);
/* Maps another rank's buffer into this process (peer access over NVLink). */
VS_API vs_status vs_peer_open(vs_ctx* ctx, const vs_ipc_handle* handle, void** dev_ptr);
VS_API vs_status vs_peer_close(vs_ctx* ctx, void* dev_ptr);
/* Stream-ordered barrier of `world` ranks: peer_flags[r] is rank r's u32 flag
 * array [world] (zeroed once); epoch must grow by one per call on every rank.
 * A wait that exceeds two seconds sets the ctx's device error, which
 * vs_ctx_check (or the next render's count readback) reports as
 * VS_ERR_DEVICE_TIMEOUT. */
VS_API vs_status vs_peer_barrier(vs_ctx* ctx, uint32_t* const* peer_flags, uint32_t world, uint32_t rank,
                                 uint32_t epoch);
/* Synchronises the ctx stream and reports a pending device-side error. */
VS_API vs_status vs_ctx_check(vs_ctx* ctx);

typedef struct vs_peer_set {
  uint32_t world, rank;
  const float* grads[VS_PEER_MAX];  /* row_format 0: [N, width] dense gradient rows of each rank;
                                       row_format 1: [views][N][VS_COMPACT_ROW] rows of vs_vjp_compact */
  const float* vis[VS_PEER_MAX];    /* [N] views of each rank that saw the splat (rows with 0 are not read) */
  float* transforms[VS_PEER_MAX];   /* the replicas, [N,10] */
  float* sh_coeffs[VS_PEER_MAX];    /* [N,(d+1)^2,3] f32 */
  float* raw_opacities[VS_PEER_MAX];
  uint32_t row_format;              /* 0 dense rows, 1 compact rows (vs_vjp_compact) */
  /* row_format 1: each rank renders `views` views per step; rank r's rows of
   * slot v are grads[r] + v * N * VS_COMPACT_ROW, its camera cams[r] + 4 v,
   * and view_masks[r][g] has bit v set when slot v saw splat g */
  uint32_t views;
  const float* cams[VS_PEER_MAX];
  const uint32_t* view_masks[VS_PEER_MAX];
} vs_peer_set;
/* The 8-bit-moment Adam of vs_adam_q8_dense for splats [splat_begin,
 * splat_end) only (splat_begin a multiple of 256), with the gradient of each
 * splat summed in rank order over the ranks whose vis > 0 and the noise gated
 * on the summed vis; the moments (mom_*) hold that shard only, and the new
 * parameters go to every rank's replica.  With row_format 1 the compact
 * rows of every (rank, view) that saw a splat are summed in that order, the SH
 * gradient rebuilt from each view's colour gradient and camera: bit for bit
 * the sums of one dense row accumulated by vs_vjp_dense over the same views in
 * the same order (with one view per rank, the sums of row_format 0).  All
 * ranks' gradient rows must be complete (vs_peer_barrier) before the call,
 * and no rank may read its replica until every rank's call has finished (a
 * second barrier). */
VS_API vs_status vs_adam_q8_peer(vs_ctx* ctx, uint32_t num_splats, int32_t sh_degree, uint32_t splat_begin,
                                 uint32_t splat_end, const vs_peer_set* peers, vs_q8_tensor mom_t,
                                 vs_q8_tensor mom_sh, vs_q8_tensor mom_o, const vs_q8_cfg* q8);

/* ---- refinement: densify and prune -----------------------------------------
 * The GPU side of SplatTrainer::refine (crates/splat-train/src/train.rs:
 * 1779-2104, refine_splats :2110-2300); the sampling of parents and the
 * budgets are host decisions made from one readback of the table. */
typedef struct vs_refine_cfg {
  float min_opacity;          /* prune below this opacity (1/255) */
  float max_bound;            /* prune scales or |mean - center| beyond this (100 x scene extent) */
  float center[3];            /* scene bounds centre */
  float split_at_screen_size; /* oversized flag threshold (fraction of the image); 0 disables */
} vs_refine_cfg;
/* table [N,8] f32 per splat: prune, non-finite, opacity*visible, oversized,
 * refine_weight*visible, mean xyz (train.rs:1822-1883); visible = vis_weight > 0.
 * sh_width = values per SH row (3 (d+1)^2), sh_half = SH stored as binary16. */
VS_API vs_status vs_refine_table(vs_ctx* ctx, uint32_t num_splats, const float* transforms, const void* sh_coeffs,
                                 uint32_t sh_width, int32_t sh_half, const float* raw_opacities,
                                 const float* refine_weight, const float* vis_weight, const float* max_screen,
                                 const vs_refine_cfg* cfg, float* table);
/* Splits parents[i] into itself and children[i] (device i32 arrays of
 * `count` distinct rows; a child row is a pruned slot or a row appended after
 * the old count, all < num_splats): covariance-aware shrink with split_at_
 * screen_size capping (screen_sizes = per-splat max screen extent, may be NULL
 * when the cap is 0), +- rotated offset, opacity 1 - (1 - o)^(1/sqrt 2) on
 * both, SH row copied to the child (train.rs:2142-2252).  empty_rows get
 * finite invisible filler rows (:2259-2283). */
VS_API vs_status vs_refine_split(vs_ctx* ctx, uint32_t num_splats, float* transforms, void* sh_coeffs,
                                 uint32_t sh_width, int32_t sh_half, float* raw_opacities, uint32_t count,
                                 const int32_t* parents, const int32_t* children, const float* screen_sizes,
                                 float split_at_screen_size, float min_opacity, uint32_t empty_count,
                                 const int32_t* empty_rows);
/* Zeroes both moments of `count` rows (row width `row_width` values) in place
 * (optim.rs:188-215 for the 8-bit moments: zero codes under the unchanged
 * block scales).  Rows appended to a tensor are zero codes too. */
VS_API vs_status vs_q8_reset_rows(vs_ctx* ctx, vs_q8_tensor mom, uint32_t row_width, uint32_t count,
                                  const int32_t* rows);
/* raw = logit(clamp(sigmoid(raw) - amount, 1e-12, 1 - 1e-12)) (train.rs:2285-2296). */
VS_API vs_status vs_opacity_decay(vs_ctx* ctx, uint32_t num_splats, float* raw_opacities, float amount);
/* Mip-Splatting 3D-filter floor per splat, compute_min_scale
 * (crates/splat-train/src/train.rs:353-387): min_scale[i] = sqrt(factor) *
 * min_v |mean_i - centre_v| * inv_focal_v.  view_cams: [V, 4] f32 device rows
 * (centre x, y, z, 1 / max(focal_px, 1e-6)), 16-byte aligned; factor > 0. */
VS_API vs_status vs_min_scale(vs_ctx* ctx, uint32_t num_splats, const float* transforms, const float* view_cams,
                              uint32_t num_views, float factor, float* min_scale);
/* Folds a floor into the raw parameters in place, Splats::bake_min_scale /
 * fold_min_scale (crates/splat-train-render/src/gaussian_splats.rs:165-188,
 * 394-402): log-scales -> log sqrt(s^2 + f^2), opacity scaled by the energy
 * factor and clamped to [1e-6, 1 - 1e-6]. */
VS_API vs_status vs_fold_min_scale(vs_ctx* ctx, uint32_t num_splats, float* transforms, float* raw_opacities,
                                   const float* min_scale);

/* ---- dataset feed: packed RGBA8 ground truth -------------------------------
 * Replaces SceneLoader (crates/splat-train-dataset/src/scene_loader.rs:59-184)
 * and view_to_packed_data (scene.rs:113-161) for decoded 8-bit images.
 * Packing: one u32 per pixel, r in the low byte, a in the high byte; 1, 2, 3
 * or 4 source channels (L, LA, RGB, RGBA); a missing alpha is 255;
 * with alpha and VS_ALPHA_TRANSPARENT the colours are premultiplied in byte
 * space, (c * a + 127) / 255. */
#define VS_ALPHA_MASKED 0
#define VS_ALPHA_TRANSPARENT 1
/* Packs device pixels [height*width*channels] u8 into out [height*width] u32
 * on the ctx stream.  Returns whether the source has alpha in *has_alpha. */
VS_API vs_status vs_pack_view(vs_ctx* ctx, const uint8_t* pixels, uint32_t width, uint32_t height,
                              uint32_t channels, int32_t alpha_mode, uint32_t* out, int32_t* has_alpha);

typedef struct vs_feed vs_feed;
typedef struct vs_feed_cfg {
  uint32_t num_views;
  uint32_t ring_slots;   /* batches staged ahead of the consumer (>= 2; 4 like the reference's channel) */
  uint32_t workers;      /* host threads that copy pixels into pinned memory (0: one per slot) */
  uint32_t hold;         /* batches the consumer uses at once (>= 1) */
  uint64_t cache_bytes;  /* HBM budget for packed views kept resident (max_scene_batch_cache_size) */
  uint64_t seed;
} vs_feed_cfg;
typedef struct vs_scene_batch {
  const uint32_t* img_packed; /* device [height, width]; ready on the ctx stream */
  uint32_t width, height;
  uint32_t view_index;
  int32_t has_alpha;
  int32_t alpha_mode;
  int32_t cached;             /* 1: a resident copy that stays valid until vs_feed_destroy */
  uint64_t h2d_bytes;         /* host-to-device bytes copied for this batch */
} vs_scene_batch;
/* The feed stages views on its own copy stream and worker threads: pinned
 * host slots, device staging slots and the packing kernel, ring_slots batches
 * ahead of the consumer.  Views are visited in epochs, each a fresh seeded
 * shuffle of all views.  A packed view that fits the cache budget (and whose
 * slot is empty) stays resident in HBM, so later visits copy nothing. */
VS_API vs_status vs_feed_create(vs_ctx* ctx, const vs_feed_cfg* cfg, vs_feed** out);
/* Registers view `index` (host pixels, read until vs_feed_destroy: keep them
 * alive and unchanged).  All views are set before the first vs_feed_next. */
VS_API vs_status vs_feed_set_view(vs_feed* feed, uint32_t index, const uint8_t* pixels, uint32_t width,
                                  uint32_t height, uint32_t channels, int32_t alpha_mode);
/* The next batch.  A batch k that is not `cached` stays valid (in stream
 * order on the ctx stream) until the call that hands out batch k + hold. */
VS_API vs_status vs_feed_next(vs_feed* feed, vs_scene_batch* out);
VS_API void vs_feed_destroy(vs_feed* feed);
/* The visiting order (host only, no GPU): `count` view indices from the start
 * of the sequence a feed with this seed and view count follows. */
VS_API vs_status vs_feed_order(uint64_t seed, uint32_t num_views, uint32_t count, uint32_t* out);

/* ---- checkpoint I/O: PLY vertex rows ---------------------------------------
 * Bytes of one PLY vertex row at an SH degree (0 if the degree is not 0..3):
 * 4 * (14 + 3 ((d+1)^2 - 1)). */
VS_API uint64_t vs_ply_row_bytes(int32_t sh_degree);
/* Replaces the row encoding of splat_to_ply (crates/splat-train-serde/src/
 * export.rs:322-425): writes num_splats rows of little-endian f32 to HOST
 * memory host_out (num_splats * vs_ply_row_bytes bytes, pinned or pageable):
 * x y z scale_0..2 opacity rot_0..3 (divided by max(|q|, 1e-12)) f_dc_0..2
 * f_rest_0.. (channel-major).  Blocks until the rows are on the host. */
VS_API vs_status vs_ply_encode(vs_ctx* ctx, uint32_t num_splats, int32_t sh_degree, const float* transforms,
                               const void* sh_coeffs, int32_t sh_half, const float* raw_opacities, void* host_out);
/* Replaces the row decoding of parse_ply (import.rs:386-510): reads
 * num_splats HOST rows of row_bytes and writes transforms [N,10], sh_coeffs
 * [N,C,3] f32 and raw_opacities [N].  offsets / defaults (host, 11 + 3 C
 * entries) describe each output value in the order transforms 0..9,
 * opacity, SH (coefficient-major, channel-minor): the byte offset of its f32
 * in a row (a multiple of 4), or -1 to write the default.  Blocks until done. */
VS_API vs_status vs_ply_decode(vs_ctx* ctx, uint32_t num_splats, const void* host_rows, uint32_t row_bytes,
                               uint32_t sh_coeffs_per_channel, const int32_t* offsets, const float* defaults,
                               float* transforms, float* sh_coeffs, float* raw_opacities);

/* ---- housekeeping (crates/splat-train/src/housekeep.rs:15-39) ------------- */
VS_API vs_status vs_gather_stats(vs_ctx* ctx, uint32_t n, float* refine_norm, float* vis_count, float* max_screen,
                                 const float* refine_weight, const float* visible, const float* radius);
VS_API vs_status vs_noise_means(vs_ctx* ctx, uint32_t n, float* transforms, const float* opacities,
                                const float* visible, float scale, float limit, uint32_t seed);

/* ---- building blocks exposed for tests ------------------------------------ */
/* Stable LSD radix sort of (key, value) u32 pairs on bits [0, key_bits). */
VS_API vs_status vs_radix_sort_pairs(vs_ctx* ctx, uint32_t* keys, uint32_t* values, uint32_t count,
                                     uint32_t key_bits);
/* The same sort with no device allocation inside the call.  It has no
 * counterpart in the reference, whose sort always obtains its temporaries
 * from its backend.  It is for hosts that cannot allocate at the point of the
 * call: ones that keep device memory inside a fixed budget they manage
 * themselves, or that must not let an allocation synchronise or fail
 * mid-stream.  All temporaries live in one statically sized array of the
 * library's device image (about 8.5 MB, held on every device that loads the
 * library until exit); count is limited to VS_SORT_STATIC_MAX_KEYS and larger
 * counts return VS_ERR_CAPACITY.  The first call on a device looks the array
 * up (cudaGetSymbolAddress, which can load the module): make that call before
 * any stream capture on that device.  Nothing in the array has to start at
 * zero.  The array is shared by all calls on a device, so calls that overlap
 * on the GPU (other streams or threads) race; the caller serialises them.
 * The calling thread's current CUDA device is the same on return. */
#define VS_SORT_STATIC_MAX_KEYS (1u << 20)
VS_API vs_status vs_radix_sort_pairs_static(vs_ctx* ctx, uint32_t* keys, uint32_t* values, uint32_t count,
                                            uint32_t key_bits);
/* Inclusive prefix sum of u32 in place; the total (u64) to *total_dev if non-NULL. */
VS_API vs_status vs_scan_inclusive(vs_ctx* ctx, uint32_t* data, uint32_t count, uint64_t* total_dev);
/* Elementwise device math used by the kernels, for tests: which = 0 vs_expf,
 * 1 vs_logf (the functions shared with the CPU oracle), 2 the fma-refined
 * square root and 4 the fma-refined reciprocal, with 3 (IEEE sqrtf) and
 * 5 (IEEE 1 / x) beside them to check that both are correctly rounded. */
VS_API vs_status vs_math_probe(vs_ctx* ctx, int32_t which, const float* x, float* y, uint32_t n);

#ifdef __cplusplus
}
#endif
#endif /* VAUSS_B200_H */
