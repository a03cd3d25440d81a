// C ABI: contexts, frames, workspace, and the render-forward orchestration.
#include <stdarg.h>
#include <stdio.h>

#include "vs_internal.cuh"

vs_status vs_fail(vs_ctx* ctx, vs_status st, const char* fmt, ...) {
  if (ctx) {
    char buf[512];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof(buf), fmt, ap);
    va_end(ap);
    ctx->err = buf;
  }
  return st;
}

vs_status vs_cuda(vs_ctx* ctx, cudaError_t e, const char* what) {
  if (e == cudaSuccess) return VS_OK;
  return vs_fail(ctx, VS_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
}

vs_status vs_ensure(vs_ctx* ctx, DevBuf& b, size_t bytes) {
  if (bytes <= b.bytes && b.ptr) return VS_OK;
  if (b.ptr) {
    // frees are stream-ordered so in-flight work on the old buffer finishes first
    VS_CUDA(ctx, cudaFreeAsync(b.ptr, ctx->stream));
    ctx->workspace -= b.bytes;
    b.ptr = nullptr;
    b.bytes = 0;
  }
  size_t want = bytes < 256 ? 256 : bytes;
  want = want + want / 8;  // headroom so slowly growing sizes do not reallocate every step
  want = (want + 255) & ~(size_t)255;
  cudaError_t e = cudaMallocAsync(&b.ptr, want, ctx->stream);
  if (e != cudaSuccess) {
    b.ptr = nullptr;
    return vs_fail(ctx, e == cudaErrorMemoryAllocation ? VS_ERR_CAPACITY : VS_ERR_CUDA,
                   "workspace allocation of %zu bytes: %s", want, cudaGetErrorString(e));
  }
  b.bytes = want;
  ctx->workspace += want;
  return VS_OK;
}

void vs_release(vs_ctx* ctx, DevBuf& b) {
  if (b.ptr) {
    cudaFreeAsync(b.ptr, ctx->stream);
    ctx->workspace -= b.bytes;
  }
  b.ptr = nullptr;
  b.bytes = 0;
}

vs_status vs_check_device_error(vs_ctx* ctx, const char* stage) {
  VS_CUDA(ctx, cudaMemcpyAsync(ctx->h_pinned + 12, ctx->d_err, 4, cudaMemcpyDeviceToHost, ctx->stream));
  VS_CUDA(ctx, cudaStreamSynchronize(ctx->stream));
  const uint32_t e = ctx->h_pinned[12];
  if (e == 0) return VS_OK;
  VS_CUDA(ctx, cudaMemsetAsync(ctx->d_err, 0, 4, ctx->stream));
  if (e & VS_DERR_WAIT) return vs_fail(ctx, VS_ERR_DEVICE_TIMEOUT, "%s: a bounded device wait gave up", stage);
  if (e & VS_DERR_STATE)
    return vs_fail(ctx, VS_ERR_INVALID, "%s: compact gradient rows were written twice for a splat in one step", stage);
  return vs_fail(ctx, VS_ERR_CAPACITY, "%s: device capacity check failed (0x%x)", stage, e);
}

vs::Uniforms vs_make_uniforms(const vs_camera& c, const vs_render_cfg& cfg) {
  vs::Uniforms u{};
  for (int i = 0; i < 9; ++i) u.rot[i] = c.viewmat[i];
  for (int i = 0; i < 3; ++i) u.trans[i] = c.viewmat[9 + i];
  u.fx = c.fx; u.fy = c.fy; u.cx = c.cx; u.cy = c.cy;
  const float w = (float)c.img_w, h = (float)c.img_h;
  // pinhole Jacobian clamp limits (crates/splat-train-render/src/camera.rs:326-331)
  u.lim_pos_x = (1.15f * w - c.cx) / c.fx;
  u.lim_pos_y = (1.15f * h - c.cy) / c.fy;
  u.lim_neg_x = (-0.15f * w - c.cx) / c.fx;
  u.lim_neg_y = (-0.15f * h - c.cy) / c.fy;
  for (int i = 0; i < 3; ++i) u.cam[i] = c.cam_pos[i];
  u.w = c.img_w; u.h = c.img_h;
  u.tbw = (c.img_w + vs::TILE - 1) / vs::TILE;
  u.tbh = (c.img_h + vs::TILE - 1) / vs::TILE;
  u.log_scale_offset = cfg.log_scale_offset;
  u.mip = cfg.mip; u.has_min_scale = cfg.has_min_scale; u.sh_degree = cfg.sh_degree; u.sh_half = cfg.sh_half;
  for (int i = 0; i < 3; ++i) u.bg[i] = cfg.bg[i];
  return u;
}

namespace {
vs_status set_device(vs_ctx* ctx) { return vs_cuda(ctx, cudaSetDevice(ctx->device), "cudaSetDevice"); }
}  // namespace

extern "C" {

VS_API const char* vs_version(void) { return "vauss_b200 0.1 (sm_100a)"; }

VS_API vs_status vs_ctx_create(int device, vs_ctx** out) {
  if (!out) return VS_ERR_INVALID;
  *out = nullptr;
  vs_ctx* ctx = new vs_ctx();
  ctx->device = device;
  vs_status st = set_device(ctx);
  if (st == VS_OK) {
    // Workspace grows through cudaMallocAsync from the device's default pool.
    // With the pool's default release threshold (0) every synchronisation --
    // one per render, the count readback -- hands freed blocks back to the
    // driver, and a buffer that outgrows its headroom later maps new memory
    // in the middle of a step; keeping freed blocks in this process's pool
    // lets that regrowth reuse them.
    cudaMemPool_t pool = nullptr;
    st = vs_cuda(ctx, cudaDeviceGetDefaultMemPool(&pool, device), "cudaDeviceGetDefaultMemPool");
    uint64_t keep = ~0ull;
    if (st == VS_OK)
      st = vs_cuda(ctx, cudaMemPoolSetAttribute(pool, cudaMemPoolAttrReleaseThreshold, &keep),
                   "cudaMemPoolSetAttribute");
  }
  if (st == VS_OK) st = vs_cuda(ctx, cudaMalloc(&ctx->d_err, 4), "cudaMalloc(err word)");
  if (st == VS_OK) st = vs_cuda(ctx, cudaMemset(ctx->d_err, 0, 4), "cudaMemset(err word)");
  if (st == VS_OK) st = vs_cuda(ctx, cudaMallocHost(&ctx->h_pinned, 64), "cudaMallocHost");
  if (st != VS_OK) {
    if (ctx->d_err) cudaFree(ctx->d_err);
    delete ctx;
    return st;
  }
  *out = ctx;
  return VS_OK;
}

VS_API void vs_ctx_destroy(vs_ctx* ctx) {
  if (!ctx) return;
  cudaSetDevice(ctx->device);
  cudaStreamSynchronize(ctx->stream);
  vs_release(ctx, ctx->sort_keys);
  vs_release(ctx, ctx->sort_vals);
  vs_release(ctx, ctx->sort_hist);
  vs_release(ctx, ctx->scan_sums);
  vs_release(ctx, ctx->misc);
  vs_release(ctx, ctx->io_stage);
  vs_release(ctx, ctx->vjp_rows);
  cudaStreamSynchronize(ctx->stream);
  if (ctx->d_err) cudaFree(ctx->d_err);
  if (ctx->h_pinned) cudaFreeHost(ctx->h_pinned);
  delete ctx;
}

VS_API vs_status vs_ctx_set_stream(vs_ctx* ctx, void* cuda_stream) {
  if (!ctx) return VS_ERR_INVALID;
  ctx->stream = (cudaStream_t)cuda_stream;
  return VS_OK;
}

VS_API const char* vs_ctx_last_error(const vs_ctx* ctx) { return ctx ? ctx->err.c_str() : "null context"; }

VS_API uint64_t vs_ctx_workspace_bytes(const vs_ctx* ctx) { return ctx ? ctx->workspace : 0; }

VS_API uint64_t vs_ctx_launch_count(const vs_ctx* ctx) { return ctx ? ctx->launches : 0; }

VS_API vs_status vs_frame_create(vs_ctx* ctx, vs_frame** out) {
  if (!ctx || !out) return VS_ERR_INVALID;
  vs_frame* f = new vs_frame();
  f->ctx = ctx;
  *out = f;
  return VS_OK;
}

VS_API void vs_frame_destroy(vs_frame* f) {
  if (!f) return;
  vs_ctx* ctx = f->ctx;
  cudaSetDevice(ctx->device);
  DevBuf* bufs[] = {&f->compact_from_global, &f->global_from_compact, &f->depths, &f->tile_counts, &f->tile_masks,
                    &f->projected, &f->depth_order, &f->isect_tile, &f->isect_compact, &f->tile_ranges,
                    &f->tile_used_end, &f->opacities, &f->max_radius, &f->lookback, &f->counters};
  for (DevBuf* b : bufs) vs_release(ctx, *b);
  delete f;
}

VS_API vs_status vs_frame_counts(const vs_frame* f, vs_render_counts* out) {
  if (!f || !out) return VS_ERR_INVALID;
  out->num_visible = f->v;
  out->num_tiles = f->T;
  out->num_intersections = f->I;
  return VS_OK;
}

VS_API vs_status vs_frame_buffer(vs_frame* f, int32_t field, void** dev_ptr, uint64_t* count) {
  if (!f || !dev_ptr || !count) return VS_ERR_INVALID;
  if (!f->rendered) return vs_fail(f->ctx, VS_ERR_INVALID, "frame_buffer: frame has not been rendered");
  switch (field) {
    case VS_FIELD_COMPACT_FROM_GLOBAL: *dev_ptr = f->compact_from_global.ptr; *count = f->n; break;
    case VS_FIELD_GLOBAL_FROM_COMPACT: *dev_ptr = f->global_from_compact.ptr; *count = f->v; break;
    case VS_FIELD_DEPTHS: *dev_ptr = f->depths.ptr; *count = f->v; break;
    case VS_FIELD_TILE_COUNTS: *dev_ptr = f->tile_counts.ptr; *count = f->v; break;
    case VS_FIELD_PROJECTED: *dev_ptr = f->projected.ptr; *count = (uint64_t)f->v * 12; break;
    case VS_FIELD_DEPTH_ORDER: *dev_ptr = f->depth_order.ptr; *count = f->v; break;
    case VS_FIELD_ISECT_TILE: *dev_ptr = f->isect_tile.ptr; *count = f->I; break;
    case VS_FIELD_ISECT_COMPACT: *dev_ptr = f->isect_compact.ptr; *count = f->I; break;
    case VS_FIELD_TILE_RANGES: *dev_ptr = f->tile_ranges.ptr; *count = (uint64_t)f->T * 2; break;
    case VS_FIELD_TILE_USED_END: *dev_ptr = f->tile_used_end.ptr; *count = f->T; break;
    case VS_FIELD_OPACITIES: *dev_ptr = f->opacities.ptr; *count = f->n; break;
    case VS_FIELD_MAX_RADIUS: *dev_ptr = f->max_radius.ptr; *count = f->n; break;
    default: return vs_fail(f->ctx, VS_ERR_INVALID, "frame_buffer: unknown field %d", field);
  }
  return VS_OK;
}

VS_API vs_status vs_frame_copy(vs_frame* f, int32_t field, void* dst_device, uint64_t max_bytes) {
  void* src = nullptr;
  uint64_t count = 0;
  VS_TRY(vs_frame_buffer(f, field, &src, &count));
  const uint64_t bytes = count * 4 < max_bytes ? count * 4 : max_bytes;
  if (bytes == 0) return VS_OK;
  if (!dst_device) return vs_fail(f->ctx, VS_ERR_INVALID, "frame_copy: null destination");
  return vs_cuda(f->ctx, cudaMemcpyAsync(dst_device, src, bytes, cudaMemcpyDeviceToDevice, f->ctx->stream),
                 "frame_copy");
}

VS_API vs_status vs_render_project(vs_ctx* ctx, vs_frame* f, const vs_camera* cam, const vs_render_cfg* cfg,
                                   uint32_t num_splats, const float* transforms, const void* sh_coeffs,
                                   const float* raw_opacities, const float* min_scale, vs_render_counts* counts_out) {
  if (!ctx) return VS_ERR_INVALID;
  if (!f || f->ctx != ctx || !cam || !cfg) return vs_fail(ctx, VS_ERR_INVALID, "render_forward: missing frame/camera/config");
  if (cam->img_w == 0 || cam->img_h == 0) return vs_fail(ctx, VS_ERR_INVALID, "render_forward: zero image size");
  // the emission packs tile coordinates into 16 bits
  if (cam->img_w > 65535u * vs::TILE || cam->img_h > 65535u * vs::TILE)
    return vs_fail(ctx, VS_ERR_UNSUPPORTED, "render_forward: image %ux%u exceeds 65535 tiles per side", cam->img_w,
                   cam->img_h);
  if (cfg->sh_degree < 0 || cfg->sh_degree > 3) return vs_fail(ctx, VS_ERR_UNSUPPORTED, "render_forward: SH degree %d (0..3 supported)", cfg->sh_degree);
  if (num_splats > 0 && (!transforms || !sh_coeffs || !raw_opacities)) return vs_fail(ctx, VS_ERR_INVALID, "render_forward: null splat buffer");
  // projection reads each 40-byte transforms row in 8-byte pieces
  if (reinterpret_cast<uintptr_t>(transforms) & 7u)
    return vs_fail(ctx, VS_ERR_INVALID, "render_forward: transforms must be 8-byte aligned");
  if (cfg->has_min_scale && !min_scale) return vs_fail(ctx, VS_ERR_INVALID, "render_forward: has_min_scale without min_scale");
  if (num_splats > 0xfffffff0u / 10u) return vs_fail(ctx, VS_ERR_CAPACITY, "render_forward: %u splats exceed 32-bit indexing", num_splats);
  VS_TRY(set_device(ctx));
  f->rendered = false;
  f->binned = false;
  f->projected_ok = false;
  f->cfg = *cfg;
  f->u = vs_make_uniforms(*cam, *cfg);
  f->n = num_splats;
  f->T = f->u.tbw * f->u.tbh;
  const size_t n1 = (size_t)num_splats + 1;
  VS_TRY(vs_ensure(ctx, f->compact_from_global, n1 * 4));
  VS_TRY(vs_ensure(ctx, f->global_from_compact, n1 * 4));
  VS_TRY(vs_ensure(ctx, f->depths, n1 * 4));
  VS_TRY(vs_ensure(ctx, f->tile_counts, n1 * 4));
  VS_TRY(vs_ensure(ctx, f->tile_masks, n1 * 8));
  VS_TRY(vs_ensure(ctx, f->projected, n1 * vs::PROJ_F4 * 16));
  VS_TRY(vs_ensure(ctx, f->opacities, n1 * 4));
  VS_TRY(vs_ensure(ctx, f->max_radius, n1 * 4));
  VS_TRY(launch_project(ctx, f, transforms, sh_coeffs, raw_opacities, min_scale));
  // the render-count readback: visible count and intersection total
  VS_CUDA(ctx, cudaMemcpyAsync(ctx->h_pinned, f->counters.ptr, 48, cudaMemcpyDeviceToHost, ctx->stream));
  VS_TRY(vs_check_device_error(ctx, "projection"));  // synchronizes
  f->v = ctx->h_pinned[1];
  uint64_t isect;
  memcpy(&isect, (const char*)ctx->h_pinned + 32, 8);
  f->I = isect;
  f->depth_lo = ~ctx->h_pinned[2];
  f->depth_hi = ctx->h_pinned[3];
  if (f->v > num_splats) return vs_fail(ctx, VS_ERR_CUDA, "render_forward: visible count %u > %u splats", f->v, num_splats);
  if (f->I >= 0xffffffffull)
    return vs_fail(ctx, VS_ERR_CAPACITY, "render_forward: %llu intersections exceed 32-bit indexing",
                   (unsigned long long)f->I);
  f->projected_ok = true;
  if (counts_out) {
    counts_out->num_visible = f->v;
    counts_out->num_tiles = f->T;
    counts_out->num_intersections = f->I;
  }
  return VS_OK;
}

VS_API vs_status vs_render_bin(vs_ctx* ctx, vs_frame* f) {
  if (!ctx) return VS_ERR_INVALID;
  if (!f || !f->projected_ok) return vs_fail(ctx, VS_ERR_INVALID, "render_bin: frame has not been projected");
  VS_TRY(set_device(ctx));
  VS_TRY(launch_bin(ctx, f));
  f->binned = true;
  return VS_OK;
}

VS_API vs_status vs_render_rasterize(vs_ctx* ctx, vs_frame* f, float* out_img, float* visible) {
  if (!ctx) return VS_ERR_INVALID;
  if (!f || !f->binned) return vs_fail(ctx, VS_ERR_INVALID, "render_rasterize: frame has not been binned");
  if (!out_img || (!visible && f->n > 0)) return vs_fail(ctx, VS_ERR_INVALID, "render_rasterize: null output");
  VS_TRY(set_device(ctx));
  VS_TRY(launch_raster_fwd(ctx, f, out_img, visible));
  f->rendered = true;
  return VS_OK;
}

VS_API vs_status vs_render_forward(vs_ctx* ctx, vs_frame* f, const vs_camera* cam, const vs_render_cfg* cfg,
                                   uint32_t num_splats, const float* transforms, const void* sh_coeffs,
                                   const float* raw_opacities, const float* min_scale, float* out_img,
                                   float* visible, vs_render_counts* counts_out) {
  if (!ctx) return VS_ERR_INVALID;
  if (!out_img || (!visible && num_splats > 0)) return vs_fail(ctx, VS_ERR_INVALID, "render_forward: null output");
  VS_TRY(vs_render_project(ctx, f, cam, cfg, num_splats, transforms, sh_coeffs, raw_opacities, min_scale,
                           counts_out));
  VS_TRY(vs_render_bin(ctx, f));
  return vs_render_rasterize(ctx, f, out_img, visible);
}

VS_API vs_status vs_render_image(vs_ctx* ctx, vs_frame* f, const vs_camera* cam, const vs_render_cfg* cfg,
                                 uint32_t num_splats, const float* transforms, const void* sh_coeffs,
                                 const float* raw_opacities, const float* min_scale, uint32_t* out_rgba8,
                                 vs_render_counts* counts_out) {
  if (!ctx) return VS_ERR_INVALID;
  if (!out_rgba8) return vs_fail(ctx, VS_ERR_INVALID, "render_image: null output");
  VS_TRY(vs_render_project(ctx, f, cam, cfg, num_splats, transforms, sh_coeffs, raw_opacities, min_scale,
                           counts_out));
  VS_TRY(vs_render_bin(ctx, f));
  VS_TRY(set_device(ctx));
  VS_TRY(launch_raster_packed(ctx, f, out_rgba8));
  f->rendered = false;  // no backward information was recorded
  return VS_OK;
}

VS_API vs_status vs_loss(vs_ctx* ctx, uint32_t h, uint32_t w, const float* pred, const uint32_t* gt_packed,
                         float l1_w, float ssim_w, float* partials, float* loss_dev, float* dl_dpred) {
  if (!ctx) return VS_ERR_INVALID;
  if (!pred || !gt_packed) return vs_fail(ctx, VS_ERR_INVALID, "loss: null input");
  VS_TRY(set_device(ctx));
  return launch_loss(ctx, h, w, pred, gt_packed, l1_w, ssim_w, partials, loss_dev, dl_dpred);
}

VS_API vs_status vs_rasterize_backward(vs_ctx* ctx, vs_frame* f, const float* out_img, const float* v_output,
                                       float* v_combined) {
  if (!ctx) return VS_ERR_INVALID;
  if (!f || !f->rendered) return vs_fail(ctx, VS_ERR_INVALID, "rasterize_backward: frame has not been rendered");
  if (!out_img || !v_output || (f->v && !v_combined)) return vs_fail(ctx, VS_ERR_INVALID, "rasterize_backward: null buffer");
  VS_TRY(set_device(ctx));
  if (f->v == 0) return VS_OK;
  return launch_raster_bwd(ctx, f, out_img, v_output, v_combined);
}

VS_API vs_status vs_radix_sort_pairs(vs_ctx* ctx, uint32_t* keys, uint32_t* values, uint32_t count,
                                     uint32_t key_bits) {
  if (!ctx) return VS_ERR_INVALID;
  if ((!keys || !values) && count) return vs_fail(ctx, VS_ERR_INVALID, "radix_sort: null buffer");
  if (key_bits > 32) return vs_fail(ctx, VS_ERR_INVALID, "radix_sort: key_bits %u > 32", key_bits);
  VS_TRY(set_device(ctx));
  VS_TRY(vs_ensure(ctx, ctx->sort_keys, (size_t)count * 4 + 4));
  VS_TRY(vs_ensure(ctx, ctx->sort_vals, (size_t)count * 4 + 4));
  bool alt = false;
  VS_TRY(radix_sort_pairs(ctx, keys, values, (uint32_t*)ctx->sort_keys.ptr, (uint32_t*)ctx->sort_vals.ptr, count,
                          key_bits, &alt));
  if (alt) {
    VS_CUDA(ctx, cudaMemcpyAsync(keys, ctx->sort_keys.ptr, (size_t)count * 4, cudaMemcpyDeviceToDevice, ctx->stream));
    VS_CUDA(ctx, cudaMemcpyAsync(values, ctx->sort_vals.ptr, (size_t)count * 4, cudaMemcpyDeviceToDevice, ctx->stream));
  }
  return VS_OK;
}

VS_API vs_status vs_scan_inclusive(vs_ctx* ctx, uint32_t* data, uint32_t count, uint64_t* total_dev) {
  if (!ctx) return VS_ERR_INVALID;
  if (!data && count) return vs_fail(ctx, VS_ERR_INVALID, "scan: null buffer");
  VS_TRY(set_device(ctx));
  return scan_inclusive_u32(ctx, data, count, total_dev);
}

}  // extern "C"

namespace {
__global__ void math_probe_kernel(int which, const float* x, float* y, uint32_t n) {
  const uint32_t i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  const float v = x[i];
  float r;
  switch (which) {
    case 0: r = vs_expf(v); break;
    case 1: r = vs_logf(v); break;
    case 2: r = vs::sqrt_rn(v); break;
    case 3: r = sqrtf(v); break;
    case 4: r = vs::rcp_rn(v); break;
    default: r = 1.0f / v; break;
  }
  y[i] = r;
}
}  // namespace

extern "C" VS_API vs_status vs_math_probe(vs_ctx* ctx, int32_t which, const float* x, float* y, uint32_t n) {
  if (!ctx) return VS_ERR_INVALID;
  if (!x || !y || which < 0 || which > 5) return vs_fail(ctx, VS_ERR_INVALID, "math_probe: bad arguments");
  if (n == 0) return VS_OK;
  math_probe_kernel<<<vs::div_up(n, 256), 256, 0, ctx->stream>>>(which, x, y, n); ++ctx->launches;
  return vs_cuda(ctx, cudaGetLastError(), "math_probe launch");
}
