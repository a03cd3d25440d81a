// Refinement (densify / prune) kernels.
//
// Replaces the GPU side of SplatTrainer::refine (crates/splat-train/src/
// train.rs:1779-2104) and refine_splats (:2110-2300): the per-splat decision
// table that the host reads back once, the split that rewrites each parent
// row and writes its child (into a pruned row or an appended one), the
// invisible filler rows, the optimizer-moment row resets
// (crates/splat-train/src/optim.rs:188-215, quant.rs:97-121) and the
// opacity decay.  The sampling of parents and the budgets are host decisions
// (vauss_b200/refine.py), as in the reference.
#include "vs_internal.cuh"

namespace {

using namespace vs;

constexpr float FRAC_1_SQRT_2 = 0.70710678118654752440f;

__device__ __forceinline__ float sh_value(const void* sh, int half, size_t i) {
  return half ? vs_f16_to_f32(((const uint16_t*)sh)[i]) : ((const float*)sh)[i];
}

// One row per splat: [prune, non-finite, opacity * visible, oversized,
// refine weight * visible, mean x, y, z] (train.rs:1822-1883).
__global__ void refine_table_kernel(uint32_t n, const float* __restrict__ transforms, const void* __restrict__ sh,
                                    uint32_t sh_width, int sh_half, const float* __restrict__ raw_opac,
                                    const float* __restrict__ refine_weight, const float* __restrict__ vis_weight,
                                    const float* __restrict__ max_screen, vs_refine_cfg cfg, float* __restrict__ table) {
  const uint32_t g = blockIdx.x * blockDim.x + threadIdx.x;
  if (g >= n) return;
  const float* t = transforms + (size_t)g * 10;
  bool finite = vs_is_finite(raw_opac[g]);
  for (int k = 0; k < 10; ++k) finite = finite && vs_is_finite(t[k]);
  for (uint32_t k = 0; k < sh_width; ++k) finite = finite && vs_is_finite(sh_value(sh, sh_half, (size_t)g * sh_width + k));
  const float opac = vs_sigmoid(raw_opac[g]);
  const bool alpha_low = opac < cfg.min_opacity;
  bool scale_big = false, out_of_bounds = false;
  for (int k = 0; k < 3; ++k) {
    scale_big = scale_big || vs_expf(t[7 + k]) > cfg.max_bound;
    out_of_bounds = out_of_bounds || fabsf(t[k] - cfg.center[k]) > cfg.max_bound;
  }
  const bool prune = alpha_low || scale_big || out_of_bounds || !finite;
  const float vis = vis_weight[g] > 0.0f ? 1.0f : 0.0f;
  const bool oversized = cfg.split_at_screen_size > 0.0f && max_screen[g] > cfg.split_at_screen_size && vis > 0.0f;
  float* row = table + (size_t)g * 8;
  row[0] = prune ? 1.0f : 0.0f;
  row[1] = finite ? 0.0f : 1.0f;
  row[2] = opac * vis;
  row[3] = oversized ? 1.0f : 0.0f;
  row[4] = refine_weight[g] * vis;
  row[5] = t[0];
  row[6] = t[1];
  row[7] = t[2];
}

// Split of parent p (train.rs:2142-2240): both halves shrink along the axes
// in proportion to their share of the largest squared scale and move apart by
// the rotated offset; the parent keeps its raw rotation, the child takes the
// normalised one; both get the opacity 1 - (1 - o)^(1/sqrt 2).  The child also
// copies the parent's SH row.  Filler rows (no parent left for a pruned slot)
// become finite, invisible splats (:2259-2283).
__global__ void refine_split_kernel(uint32_t count, float* __restrict__ transforms, void* __restrict__ sh,
                                    uint32_t sh_width, int sh_half, float* __restrict__ raw_opac,
                                    const int32_t* __restrict__ parents, const int32_t* __restrict__ children,
                                    const float* __restrict__ screen, float split_at_screen_size, float min_opacity,
                                    uint32_t empty_count, const int32_t* __restrict__ empty_rows) {
  const uint32_t i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i < count) {
    const uint32_t p = (uint32_t)parents[i], c = (uint32_t)children[i];
    float* tp = transforms + (size_t)p * 10;
    float* tc = transforms + (size_t)c * 10;
    float t[10];
    for (int k = 0; k < 10; ++k) t[k] = tp[k];
    const float qw = t[3], qx = t[4], qy = t[5], qz = t[6];
    const float mag = fmaxf(sqrtf(((qw * qw + qx * qx) + qy * qy) + qz * qz), 1.0e-32f);
    const float rw = qw / mag, rx = qx / mag, ry = qy / mag, rz = qz / mag;
    float s[3], ssq[3];
    for (int k = 0; k < 3; ++k) {
      s[k] = vs_expf(t[7 + k]);
      ssq[k] = s[k] * s[k];
    }
    const float max_sq = fmaxf(fmaxf(fmaxf(ssq[0], ssq[1]), ssq[2]), 1.0e-30f);
    float k_max = FRAC_1_SQRT_2;
    if (split_at_screen_size > 0.0f)
      k_max = fminf(split_at_screen_size * (1.0f / fmaxf(screen[p], 1.0e-6f)), FRAC_1_SQRT_2);
    float off[3], new_log[3];
    for (int k = 0; k < 3; ++k) {
      const float kk = -((ssq[k] / max_sq) * (-k_max + 1.0f)) + 1.0f;
      off[k] = sqrtf(fmaxf(-(kk * kk) + 1.0f, 0.0f)) * s[k];
      new_log[k] = t[7 + k] + vs_logf(kk);
    }
    // quaternion_vec_multiply (quat_vec.rs) with the normalised rotation
    const float w2 = rw * rw, x2 = rx * rx, y2 = ry * ry, z2 = rz * rz;
    const float xy = rx * ry, xz = rx * rz, yz = ry * rz, wx = rw * rx, wy = rw * ry, wz = rw * rz;
    const float vx = off[0], vy = off[1], vz = off[2];
    const float sx = (((w2 + x2) - y2) - z2) * vx + ((((xy * vy + xz * vz) + wy * vz) - wz * vy) * 2.0f);
    const float sy = (((w2 - x2) + y2) - z2) * vy + ((((xy * vx + yz * vz) + wz * vx) - wx * vz) * 2.0f);
    const float sz = (((w2 - x2) - y2) + z2) * vz + ((((xz * vx + yz * vy) + wx * vy) - wy * vx) * 2.0f);
    const float opac = vs_sigmoid(raw_opac[p]);
    const float inv = 1.0f - opac;
    const float new_opac = 1.0f - vs_expf(vs_logf(inv) * FRAC_1_SQRT_2);
    const float o = clampf(new_opac, min_opacity, 1.0f - min_opacity);
    const float new_raw = vs_logf(o / (1.0f - o));
    // child first (the parent row is still being read above only from registers)
    tc[0] = t[0] + sx; tc[1] = t[1] + sy; tc[2] = t[2] + sz;
    tc[3] = rw; tc[4] = rx; tc[5] = ry; tc[6] = rz;
    tc[7] = new_log[0]; tc[8] = new_log[1]; tc[9] = new_log[2];
    tp[0] = t[0] - sx; tp[1] = t[1] - sy; tp[2] = t[2] - sz;
    tp[7] = new_log[0]; tp[8] = new_log[1]; tp[9] = new_log[2];
    raw_opac[p] = new_raw;
    raw_opac[c] = new_raw;
    if (sh_half) {
      const uint16_t* src = (const uint16_t*)sh + (size_t)p * sh_width;
      uint16_t* dst = (uint16_t*)sh + (size_t)c * sh_width;
      for (uint32_t k = 0; k < sh_width; ++k) dst[k] = src[k];
    } else {
      const float* src = (const float*)sh + (size_t)p * sh_width;
      float* dst = (float*)sh + (size_t)c * sh_width;
      for (uint32_t k = 0; k < sh_width; ++k) dst[k] = src[k];
    }
  } else if (i - count < empty_count) {
    const uint32_t r = (uint32_t)empty_rows[i - count];
    const float row[10] = {0.0f, 0.0f, 0.0f, 1.0f, 0.0f, 0.0f, 0.0f, -10.0f, -10.0f, -10.0f};
    for (int k = 0; k < 10; ++k) transforms[(size_t)r * 10 + k] = row[k];
    raw_opac[r] = -20.0f;
    for (uint32_t k = 0; k < sh_width; ++k) {
      if (sh_half) ((uint16_t*)sh)[(size_t)r * sh_width + k] = 0;
      else ((float*)sh)[(size_t)r * sh_width + k] = 0.0f;
    }
  }
}

// Zero moment rows in place: code 128 (m = 0) and 0 (v = 0); the block scales
// stay, since zero codes decode to zero under any scale.
__global__ void q8_reset_rows_kernel(uint8_t* __restrict__ m_codes, uint8_t* __restrict__ v_codes, uint32_t width,
                                     uint32_t count, const int32_t* __restrict__ rows) {
  const uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= (uint64_t)count * width) return;
  const uint64_t r = (uint64_t)rows[i / width];
  const uint64_t v = r * width + i % width;
  m_codes[v] = 128u;
  v_codes[v] = 0u;
}

// raw = logit(clamp(sigmoid(raw) - amount, 1e-12, 1 - 1e-12))  (train.rs:2289-2296)
__global__ void opacity_decay_kernel(uint32_t n, float* __restrict__ raw_opac, float amount) {
  const uint32_t g = blockIdx.x * blockDim.x + threadIdx.x;
  if (g >= n) return;
  const float o = clampf(vs_sigmoid(raw_opac[g]) - amount, 1.0e-12f, 1.0f - 1.0e-12f);
  raw_opac[g] = vs_logf(o / (1.0f - o));
}

// Mip-Splatting 3D-filter floor (compute_min_scale, crates/splat-train/src/
// train.rs:353-387): f_i = sqrt(factor) * min over the training views of
// |mean_i - centre_v| / max(focal_v, 1e-6).  `cams` holds per view the centre
// and the reciprocal focal length (the host forms 1 / max(focal, 1e-6) in f32);
// the distance sums the squares in axis order.
__global__ void min_scale_kernel(uint32_t n, const float* __restrict__ transforms, const float4* __restrict__ cams,
                                 uint32_t views, float sqrt_factor, float* __restrict__ out) {
  const uint32_t g = blockIdx.x * blockDim.x + threadIdx.x;
  if (g >= n) return;
  const float mx = transforms[(size_t)g * 10], my = transforms[(size_t)g * 10 + 1], mz = transforms[(size_t)g * 10 + 2];
  float r = __int_as_float(0x7f800000);
  for (uint32_t v = 0; v < views; ++v) {
    const float4 c = cams[v];
    const float dx = mx - c.x, dy = my - c.y, dz = mz - c.z;
    const float dist = sqrtf((dx * dx + dy * dy) + dz * dz);
    r = fminf(r, dist * c.w);
  }
  out[g] = r * sqrt_factor;
}

// Folds the floor into the raw parameters (fold_min_scale, crates/splat-train-
// render/src/gaussian_splats.rs:165-188): log-scales become log sqrt(s^2 + f^2),
// the opacity takes the energy factor exp(sum(log s - new log s)) and is stored
// back as a logit after clamping to [1e-6, 1 - 1e-6].
__global__ void fold_min_scale_kernel(uint32_t n, float* __restrict__ transforms, float* __restrict__ raw_opac,
                                      const float* __restrict__ min_scale) {
  const uint32_t g = blockIdx.x * blockDim.x + threadIdx.x;
  if (g >= n) return;
  float* t = transforms + (size_t)g * 10;
  const float f = min_scale[g], f2 = f * f;
  float diff[3];
  for (int k = 0; k < 3; ++k) {
    const float ls = t[7 + k];
    const float nl = vs_logf(vs_expf(ls * 2.0f) + f2) * 0.5f;
    diff[k] = ls - nl;
    t[7 + k] = nl;
  }
  const float coef = vs_expf((diff[0] + diff[1]) + diff[2]);
  const float o = clampf(vs_sigmoid(raw_opac[g]) * coef, 1.0e-6f, 1.0f - 1.0e-6f);
  raw_opac[g] = vs_logf(o / (1.0f - o));
}

}  // namespace

extern "C" {

VS_API vs_status vs_refine_table(vs_ctx* ctx, uint32_t num_splats, const float* transforms, const void* sh_coeffs,
                                 uint32_t sh_width, int32_t sh_half, const float* raw_opacities,
                                 const float* refine_weight, const float* vis_weight, const float* max_screen,
                                 const vs_refine_cfg* cfg, float* table) {
  if (!ctx) return VS_ERR_INVALID;
  if (!cfg || ((!transforms || !sh_coeffs || !raw_opacities || !refine_weight || !vis_weight || !max_screen ||
                !table) && num_splats))
    return vs_fail(ctx, VS_ERR_INVALID, "refine_table: null argument");
  if (sh_width == 0 || sh_width > 48) return vs_fail(ctx, VS_ERR_INVALID, "refine_table: SH row width %u", sh_width);
  if (num_splats == 0) return VS_OK;
  VS_CUDA(ctx, cudaSetDevice(ctx->device));
  refine_table_kernel<<<div_up(num_splats, 256), 256, 0, ctx->stream>>>(num_splats, transforms, sh_coeffs, sh_width,
                                                                       sh_half, raw_opacities, refine_weight,
                                                                       vis_weight, max_screen, *cfg, table);
  ++ctx->launches;
  return vs_cuda(ctx, cudaGetLastError(), "refine_table launch");
}

VS_API vs_status vs_refine_split(vs_ctx* ctx, uint32_t num_splats, float* transforms, void* sh_coeffs,
                                 uint32_t sh_width, int32_t sh_half, float* raw_opacities, uint32_t count,
                                 const int32_t* parents, const int32_t* children, const float* screen_sizes,
                                 float split_at_screen_size, float min_opacity, uint32_t empty_count,
                                 const int32_t* empty_rows) {
  if (!ctx) return VS_ERR_INVALID;
  if (!transforms || !sh_coeffs || !raw_opacities || (count && (!parents || !children)) ||
      (empty_count && !empty_rows) || (count && split_at_screen_size > 0.0f && !screen_sizes))
    return vs_fail(ctx, VS_ERR_INVALID, "refine_split: null argument");
  if (sh_width == 0 || sh_width > 48) return vs_fail(ctx, VS_ERR_INVALID, "refine_split: SH row width %u", sh_width);
  if ((uint64_t)count + empty_count > num_splats)
    return vs_fail(ctx, VS_ERR_INVALID, "refine_split: %u rows to write in %u splats", count + empty_count, num_splats);
  const uint32_t total = count + empty_count;
  if (total == 0) return VS_OK;
  VS_CUDA(ctx, cudaSetDevice(ctx->device));
  refine_split_kernel<<<div_up(total, 128), 128, 0, ctx->stream>>>(count, transforms, sh_coeffs, sh_width, sh_half,
                                                                   raw_opacities, parents, children, screen_sizes,
                                                                   split_at_screen_size, min_opacity, empty_count,
                                                                   empty_rows);
  ++ctx->launches;
  return vs_cuda(ctx, cudaGetLastError(), "refine_split launch");
}

VS_API vs_status vs_q8_reset_rows(vs_ctx* ctx, vs_q8_tensor mom, uint32_t row_width, uint32_t count,
                                  const int32_t* rows) {
  if (!ctx) return VS_ERR_INVALID;
  if (!mom.m_codes || !mom.v_codes || (count && !rows) || row_width == 0)
    return vs_fail(ctx, VS_ERR_INVALID, "q8_reset_rows: bad arguments");
  const uint64_t total = (uint64_t)count * row_width;
  if (total == 0) return VS_OK;
  VS_CUDA(ctx, cudaSetDevice(ctx->device));
  q8_reset_rows_kernel<<<(uint32_t)((total + 255) / 256), 256, 0, ctx->stream>>>(mom.m_codes, mom.v_codes, row_width,
                                                                                  count, rows);
  ++ctx->launches;
  return vs_cuda(ctx, cudaGetLastError(), "q8_reset_rows launch");
}

VS_API vs_status vs_opacity_decay(vs_ctx* ctx, uint32_t num_splats, float* raw_opacities, float amount) {
  if (!ctx) return VS_ERR_INVALID;
  if (!raw_opacities && num_splats) return vs_fail(ctx, VS_ERR_INVALID, "opacity_decay: null argument");
  if (num_splats == 0) return VS_OK;
  VS_CUDA(ctx, cudaSetDevice(ctx->device));
  opacity_decay_kernel<<<div_up(num_splats, 256), 256, 0, ctx->stream>>>(num_splats, raw_opacities, amount);
  ++ctx->launches;
  return vs_cuda(ctx, cudaGetLastError(), "opacity_decay launch");
}

VS_API vs_status vs_min_scale(vs_ctx* ctx, uint32_t num_splats, const float* transforms, const float* view_cams,
                              uint32_t num_views, float factor, float* min_scale) {
  if (!ctx) return VS_ERR_INVALID;
  if ((num_splats && (!transforms || !min_scale)) || (num_views && !view_cams) || !(factor > 0.0f))
    return vs_fail(ctx, VS_ERR_INVALID, "min_scale: bad arguments");
  if (num_views == 0) return vs_fail(ctx, VS_ERR_INVALID, "min_scale: no training views");
  if (((uintptr_t)view_cams & 15u) != 0) return vs_fail(ctx, VS_ERR_INVALID, "min_scale: view_cams must be 16-byte aligned");
  if (num_splats == 0) return VS_OK;
  VS_CUDA(ctx, cudaSetDevice(ctx->device));
  min_scale_kernel<<<div_up(num_splats, 256), 256, 0, ctx->stream>>>(num_splats, transforms, (const float4*)view_cams,
                                                                     num_views, sqrtf(factor), min_scale);
  ++ctx->launches;
  return vs_cuda(ctx, cudaGetLastError(), "min_scale launch");
}

VS_API vs_status vs_fold_min_scale(vs_ctx* ctx, uint32_t num_splats, float* transforms, float* raw_opacities,
                                   const float* min_scale) {
  if (!ctx) return VS_ERR_INVALID;
  if (num_splats && (!transforms || !raw_opacities || !min_scale))
    return vs_fail(ctx, VS_ERR_INVALID, "fold_min_scale: null argument");
  if (num_splats == 0) return VS_OK;
  VS_CUDA(ctx, cudaSetDevice(ctx->device));
  fold_min_scale_kernel<<<div_up(num_splats, 256), 256, 0, ctx->stream>>>(num_splats, transforms, raw_opacities,
                                                                          min_scale);
  ++ctx->launches;
  return vs_cuda(ctx, cudaGetLastError(), "fold_min_scale launch");
}

}  // extern "C"
