// Optimizer kernels.
//
// Reference mode (drop-in parity with the reference trainer):
//   project_update_kernel -- projection VJP fused with Adam on packed 16/16
//     moments (crates/splat-train-render/src/bwd/kernels/project_update.rs:
//     36-178, geo_moments.rs:26-96), plus the SH reduced-variance update
//     (crates/splat-train/src/optim.rs:454-469);
//   sh_step_kernel -- f16 SH Adam with an 8-bit first moment in 128-value
//     blocks, one warp per block (crates/splat-train/src/quant_kernels.rs:
//     597-714).
// Q8 mode (the benchmark's optimizer: 8-bit m AND v, 256-value blocks):
//   vjp_rows_kernel + q8_kernel<0> -- single view: the projection VJP of
//     each visible splat into a compact row, then Adam on all 59 parameters +
//     refine statistics + mean noise, one CTA per 256 splats;
//   q8_kernel<1>  -- the same Adam from an all-reduced dense gradient;
//   q8_kernel<2>  -- the same Adam for one rank's shard over peer memory,
//     the other ranks' dense rows read and summed from their memory;
//   q8_kernel<3>  -- the same from compact rows (one view per rank): the SH
//     gradient rebuilt per rank from its colour gradient and camera into
//     shared memory;
//   vjp_dense_kernel -- accumulates one view's dense gradient rows, or writes
//     its compact rows.
#include "vjp.cuh"
#include "vs_internal.cuh"

namespace {

using namespace vs;

// ---- packed geometry moments (geo_moments.rs:26-96) ----
constexpr float GEO_U_MAX = 8.0f, GEO_U_CODES = 32767.0f;
constexpr float GEO_U_STEP = GEO_U_MAX / GEO_U_CODES, GEO_U_PER_UNIT = GEO_U_CODES / GEO_U_MAX;
constexpr float GEO_L_MAX = 64.0f, GEO_L_CODES = 65535.0f;
constexpr float GEO_L_STEP = GEO_L_MAX / GEO_L_CODES, GEO_L_PER_UNIT = GEO_L_CODES / GEO_L_MAX;

__device__ __forceinline__ uint32_t pack_geo(float m, float v, float eps, float rl, float ru) {
  const float l = vs_logf(1.0f + sqrtf(fmaxf(v, 0.0f)) / eps) * GEO_L_PER_UNIT;
  const float l_code = floorf(clampf(l + rl, 0.0f, GEO_L_CODES));
  const float scale = eps * vs_expf(l_code * GEO_L_STEP);
  const float uu = fabsf(m) / scale * GEO_U_PER_UNIT;
  const uint32_t u_code = (uint32_t)floorf(clampf(uu + ru, 0.0f, GEO_U_CODES));
  const uint32_t sign = m < 0.0f ? 0x8000u : 0u;
  return ((uint32_t)l_code << 16) | sign | u_code;
}

__device__ __forceinline__ void adam_packed(float* params, uint32_t* words, size_t index, float g, float lr, float b1,
                                            float b2, float inv1, float inv2, float eps, uint32_t seed) {
  const uint32_t word = words[index];
  const float growth = vs_expf((float)(word >> 16) * GEO_L_STEP);
  const float mag = (float)(word & 0x7fffu) * GEO_U_STEP;
  const float un = (word & 0x8000u) ? -mag : mag;
  const float root = eps * (growth - 1.0f);
  const float m1 = un * (eps * growth) * b1 + g * (1.0f - b1);
  const float v1 = root * root * b2 + g * g * (1.0f - b2);
  const float step = (m1 * inv1) / (sqrtf(v1 * inv2) + eps);
  params[index] = params[index] - step * lr;
  const uint32_t hsh = vs_mix_hash((uint32_t)index, seed);
  words[index] = pack_geo(m1, v1, eps, (float)(hsh >> 16) / 65536.0f, (float)(hsh & 0xffffu) / 65536.0f);
}

struct AdamArgs {
  float b1, b2, inv1, inv2, eps, lr_opac, opac_reg;
  uint32_t seed;
  float lr_scale[10];
};

__global__ void __launch_bounds__(256) project_update_kernel(
    Uniforms u, uint32_t n, float* __restrict__ transforms, const void* __restrict__ sh, float* __restrict__ raw_opac,
    const float* __restrict__ min_scale, const uint32_t* __restrict__ compact_from_global,
    const float* __restrict__ v_combined, uint32_t* __restrict__ w_t, uint32_t* __restrict__ w_o, AdamArgs a,
    float* __restrict__ color_dir, float* __restrict__ v_refine, float* __restrict__ grad_sq,
    float* __restrict__ variance, int32_t first_step) {
  const uint32_t g = blockIdx.x * blockDim.x + threadIdx.x;
  if (g >= n) return;
  if (g == 0) {
#pragma unroll
    for (int k = 0; k < 6; ++k) color_dir[k] = 0.0f;
  }
  float gr[10];
#pragma unroll
  for (int k = 0; k < 10; ++k) gr[k] = 0.0f;
  float g_opac = 0.0f, refine = 0.0f, gsq = 0.0f;
  const uint32_t row = compact_from_global[g];
  float* t = transforms + (size_t)g * 10;
  if (row > 0) {
    const float* rg = v_combined + (size_t)(row - 1) * 10;
    float rr[10];
    bool any = false;
#pragma unroll
    for (int k = 0; k < 10; ++k) {
      rr[k] = rg[k];
      any = any || rr[k] != 0.0f;
    }
    float* cd = color_dir + (size_t)row * 6;
    if (any) {
      float tt[10];
#pragma unroll
      for (int k = 0; k < 10; ++k) tt[k] = t[k];
      const VjpOut o = splat_vjp(tt, raw_opac[g], sh, min_scale, g, rr, u);
      cd[0] = rr[5]; cd[1] = rr[6]; cd[2] = rr[7];
      cd[3] = o.dir.x; cd[4] = o.dir.y; cd[5] = o.dir.z;
      gr[0] = o.v_mean.x; gr[1] = o.v_mean.y; gr[2] = o.v_mean.z;
      gr[3] = o.v_q.w; gr[4] = o.v_q.x; gr[5] = o.v_q.y; gr[6] = o.v_q.z;
      gr[7] = o.v_scale.x; gr[8] = o.v_scale.y; gr[9] = o.v_scale.z;
      g_opac = o.v_raw;
      refine = clampf(vs_is_finite(rr[9]) ? rr[9] : 0.0f, 0.0f, 1.0e32f);
      const float c0 = SH_C0 * rr[5], c1 = SH_C0 * rr[6], c2 = SH_C0 * rr[7];
      gsq = (c0 * c0 + c1 * c1 + c2 * c2) / 3.0f;
    } else {
#pragma unroll
      for (int k = 0; k < 6; ++k) cd[k] = 0.0f;
    }
  }
  v_refine[g] = refine;
  grad_sq[g] = gsq;
  if (variance) {
    if (first_step) variance[g] = gsq * (1.0f - a.b2);
    else if (row > 0) variance[g] = variance[g] * a.b2 + gsq * (1.0f - a.b2);
  }
  const float o = 1.0f / (1.0f + vs_expf(-raw_opac[g]));
  g_opac += a.opac_reg * o * (1.0f - o);
  const uint32_t seed_t = a.seed ^ (10u << 24), seed_o = a.seed ^ (1u << 24);
#pragma unroll
  for (int k = 0; k < 10; ++k)
    adam_packed(transforms, w_t, (size_t)g * 10 + k, gr[k], a.lr_scale[k], a.b1, a.b2, a.inv1, a.inv2, a.eps, seed_t);
  adam_packed(raw_opac, w_o, g, g_opac, a.lr_opac, a.b1, a.b2, a.inv1, a.inv2, a.eps, seed_o);
}

__device__ __forceinline__ float sh_basis_one(uint32_t k, float x, float y, float z) {
  float b[16];
  sh_basis_all(x, y, z, b);
  float r = 0.0f;
#pragma unroll
  for (int i = 0; i < 16; ++i) r = (k == (uint32_t)i) ? b[i] : r;
  return r;
}

// Stochastic rounding to f16 storage (quant_kernels.rs:860-890).
__device__ __forceinline__ float stochastic_half(float value, uint32_t index, uint32_t step) {
  const float mag = fabsf(value);
  float result = value;
  if (mag <= 65504.0f) {
    float lower, upper;
    if (mag < 0.00006103515625f) {
      lower = floorf(mag * 16777216.0f) / 16777216.0f;
      upper = lower + 0.000000059604644775390625f;
    } else {
      const uint32_t bits = __float_as_uint(mag) & 0xffffe000u;
      lower = __uint_as_float(bits);
      upper = __uint_as_float(bits + 8192u);
    }
    const uint32_t hsh = vs_mix_hash(index, step);
    const float uni = (float)(hsh >> 8) / 16777216.0f;
    const float prob = (mag - lower) / (upper - lower);
    result = uni < prob ? upper : lower;
    if (value < 0.0f) result = -result;
  }
  return result;
}

struct ShStepArgs {
  float beta, factor, inv1, inv2, eps, lr;
  uint32_t seed;
};

// One warp per 128-value block, one 4-value code word per lane.
__global__ void __launch_bounds__(128) sh_step_kernel(uint32_t count, uint32_t row_width, uint16_t* __restrict__ params,
                                                      const float* __restrict__ color_dir,
                                                      const uint32_t* __restrict__ grad_rows,
                                                      uint32_t* __restrict__ codes, float* __restrict__ scales,
                                                      const float* __restrict__ variance,
                                                      const float* __restrict__ lr_scale, uint32_t nblocks,
                                                      ShStepArgs a) {
  const uint32_t lane = threadIdx.x & 31u;
  const uint32_t block = blockIdx.x * 4 + (threadIdx.x >> 5);
  if (block >= nblocks) return;
  const uint32_t word = block * 32 + lane;
  bool any = false;
#pragma unroll
  for (uint32_t j = 0; j < 4; ++j) {
    const uint32_t i = word * 4 + j;
    if (i < count) any = any || grad_rows[i / row_width] != 0u;
  }
  if (!__any_sync(0xffffffffu, any)) return;
  const uint32_t old = codes[word];
  const float old_scale = scales[block];
  float m[4];
#pragma unroll
  for (uint32_t j = 0; j < 4; ++j) {
    const uint32_t code = (old >> (j * 8)) & 255u;
    m[j] = (word * 4 + j < count) ? ((float)code - 128.0f) * old_scale : 0.0f;
  }
#pragma unroll
  for (uint32_t j = 0; j < 4; ++j) {
    const uint32_t i = word * 4 + j;
    if (i >= count) continue;
    const uint32_t row = i / row_width, col = i % row_width;
    const uint32_t gr = grad_rows[row];
    if (gr == 0u) continue;
    const float* cd = color_dir + (size_t)gr * 6;
    const float basis = sh_basis_one(col / 3, cd[3], cd[4], cd[5]);
    const float gg = basis * cd[col % 3];
    const float moment = m[j] * a.beta + gg * a.factor;
    const float denom = sqrtf(variance[row] * a.inv2) + a.eps;
    const float delta = (moment * a.inv1 / denom) * (lr_scale[col] * a.lr);
    float updated = vs_f16_to_f32(params[i]) - delta;
    updated = stochastic_half(updated, i, a.seed);
    params[i] = vs_f32_to_f16(updated);
    m[j] = moment;
  }
  float local = fmaxf(fmaxf(fabsf(m[0]), fabsf(m[1])), fmaxf(fabsf(m[2]), fabsf(m[3])));
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) local = fmaxf(local, __shfl_xor_sync(0xffffffffu, local, off));
  const float scale = local / 127.0f;
  if (lane == 0) scales[block] = scale;
  uint32_t packed = 0;
#pragma unroll
  for (uint32_t j = 0; j < 4; ++j) {
    uint32_t code = 128u;
    if (scale > 0.0f) code = (uint32_t)(rintf(clampf(m[j] / scale, -127.0f, 127.0f)) + 128.0f);
    packed |= code << (j * 8);
  }
  codes[word] = packed;
}

// Block-wide compaction: the ids of the threads with `flag` set, in thread
// order, into list[0 .. return value).  All threads of the block call it.
template <uint32_t THREADS>
__device__ __forceinline__ uint32_t compact_block(bool flag, uint32_t* list, uint32_t* warp_cnt) {
  const uint32_t tid = threadIdx.x, lane = tid & 31u, warp = tid >> 5;
  const uint32_t bal = __ballot_sync(0xffffffffu, flag);
  if (lane == 0) warp_cnt[warp] = __popc(bal);
  __syncthreads();
  uint32_t off = 0, total = 0;
#pragma unroll
  for (uint32_t w = 0; w < THREADS / 32; ++w) {
    const uint32_t cw = warp_cnt[w];
    off += w < warp ? cw : 0u;
    total += cw;
  }
  if (flag) list[off + __popc(bal & ((1u << lane) - 1u))] = tid;
  __syncthreads();
  return total;
}

// ---- dense VJP ----
// One thread per visible (projected) splat, in compact order; splats that
// projection culled have no rasterizer row and no `visible` mark, so their
// gradient rows, refine sums and view counts stay as they are.  The rows with
// a non-zero rasterizer gradient are compacted per block first, so the VJP
// runs on whole warps.  kCompact writes VS_COMPACT_ROW floats per splat into
// the rows of view slot `slot` (transforms gradient, raw-opacity gradient,
// colour gradient) and marks the splat's bit in view_mask: the view's SH
// gradient is that colour gradient times the SH basis of the view direction,
// which the shard owner rebuilds from the camera position (cam_out).
template <bool kCompact>
__global__ void __launch_bounds__(256) vjp_dense_kernel(Uniforms u, uint32_t v, const float* __restrict__ transforms,
                                                        const void* __restrict__ sh, const float* __restrict__ raw_opac,
                                                        const float* __restrict__ min_scale,
                                                        const uint32_t* __restrict__ global_from_compact,
                                                        const float* __restrict__ v_combined,
                                                        float* __restrict__ grads, float* __restrict__ refine,
                                                        const float* __restrict__ visible,
                                                        float* __restrict__ vis_accum, float* __restrict__ cam_out,
                                                        uint32_t* __restrict__ view_mask, uint32_t slot,
                                                        uint32_t* __restrict__ err) {
  __shared__ uint32_t s_list[256];
  __shared__ uint32_t s_wcnt[8];
  __shared__ uint8_t s_fresh[256];
  const uint32_t c = blockIdx.x * blockDim.x + threadIdx.x;
  const int nc = (u.sh_degree + 1) * (u.sh_degree + 1);
  const int width = kCompact ? VS_COMPACT_ROW : 10 + 3 * nc + 1;
  if (kCompact && c == 0) {
    cam_out[0] = u.cam[0];
    cam_out[1] = u.cam[1];
    cam_out[2] = u.cam[2];
    cam_out[3] = 0.0f;
  }
  bool any = false;
  if (c < v) {
    const uint32_t g = global_from_compact[c];
    // A row not seen before in this step (vis_accum was 0) is overwritten, so
    // readers gated on vis_accum never see an earlier step's values.
    bool fresh = false;
    if (vis_accum) {
      const float seen = vis_accum[g];
      vis_accum[g] = seen + visible[g];
      // a compact row is the slot's own: every visible splat's row is fresh
      fresh = (kCompact || seen == 0.0f) && visible[g] > 0.0f;
    }
    if (kCompact && visible[g] > 0.0f) {
      const uint32_t m = view_mask[g];
      if (m & (1u << slot)) atomicOr(err, VS_DERR_STATE);  // the slot written twice in a step
      view_mask[g] = m | (1u << slot);
    }
    const float* rg = v_combined + (size_t)c * 10;
#pragma unroll
    for (int k = 0; k < 10; ++k) any = any || rg[k] != 0.0f;
    if (!any && fresh)
      for (int k = 0; k < width; ++k) grads[(size_t)g * width + k] = 0.0f;
    s_fresh[threadIdx.x] = fresh ? 1 : 0;
  }
  const uint32_t total = compact_block<256>(any, s_list, s_wcnt);
  if (threadIdx.x >= total) return;
  const uint32_t t = s_list[threadIdx.x];
  const uint32_t cc = blockIdx.x * blockDim.x + t;
  const uint32_t g = global_from_compact[cc];
  const bool fresh = s_fresh[t] != 0;
  const float* rg = v_combined + (size_t)cc * 10;
  float rr[10];
#pragma unroll
  for (int k = 0; k < 10; ++k) rr[k] = rg[k];
  float tt[10];
#pragma unroll
  for (int k = 0; k < 10; ++k) tt[k] = transforms[(size_t)g * 10 + k];
  const VjpOut o = splat_vjp(tt, raw_opac[g], sh, min_scale, g, rr, u);
  float* d = grads + (size_t)g * width;
  const float gv[10] = {o.v_mean.x, o.v_mean.y, o.v_mean.z, o.v_q.w, o.v_q.x, o.v_q.y, o.v_q.z,
                        o.v_scale.x, o.v_scale.y, o.v_scale.z};
  if (kCompact) {
    // the terms a fresh dense row would hold: 0 + x for the accumulated
    // parts, the raw colour gradient for the SH part
    float4* d4 = reinterpret_cast<float4*>(d);
    d4[0] = make_float4(0.0f + gv[0], 0.0f + gv[1], 0.0f + gv[2], 0.0f + gv[3]);
    d4[1] = make_float4(0.0f + gv[4], 0.0f + gv[5], 0.0f + gv[6], 0.0f + gv[7]);
    d4[2] = make_float4(0.0f + gv[8], 0.0f + gv[9], 0.0f + o.v_raw, rr[5]);
    d4[3] = make_float4(rr[6], rr[7], 0.0f, 0.0f);
  } else {
    // 0 + x (not x) on a fresh row keeps the sign of zero of an accumulation
#pragma unroll
    for (int k = 0; k < 10; ++k) d[k] = (fresh ? 0.0f : d[k]) + gv[k];
    float b[16];
    sh_basis_all(o.dir.x, o.dir.y, o.dir.z, b);
    for (int k = 0; k < nc; ++k) {
#pragma unroll
      for (int q = 0; q < 3; ++q) d[10 + k * 3 + q] = (fresh ? 0.0f : d[10 + k * 3 + q]) + rr[5 + q] * b[k];
    }
    d[width - 1] = (fresh ? 0.0f : d[width - 1]) + o.v_raw;
  }
  refine[g] += clampf(vs_is_finite(rr[9]) ? rr[9] : 0.0f, 0.0f, 1.0e32f);
}

// ---- single-view VJP rows (the first half of the fused Q8 step) ----
// One row of VJP_ROW floats per visible splat, in compact (projection) order:
// 0-9 transforms gradient, 10 raw-opacity gradient, 11-13 colour gradient
// (rasterizer rgb), 14-16 view direction, 17 refine weight, 18 = 1 when the
// rasterizer row has a non-zero value, 19 unused.  A row without gradient
// has only its last float4 (refine, flag) written, as zeros; readers take the
// rest only when the flag is set.  Running the VJP here, over the compacted
// rows with a gradient, keeps its dependent gathers and its code out of the
// optimizer kernel.
constexpr uint32_t VJP_ROW = 20;

__global__ void __launch_bounds__(128) vjp_rows_kernel(Uniforms u, uint32_t v, const uint32_t* __restrict__ global_from_compact,
                                                       const float* __restrict__ transforms, const float* __restrict__ sh,
                                                       const float* __restrict__ raw_opac,
                                                       const float* __restrict__ min_scale,
                                                       const float* __restrict__ v_combined, float4* __restrict__ rows) {
  __shared__ uint32_t s_list[128];
  __shared__ uint32_t s_wcnt[4];
  const uint32_t c = blockIdx.x * blockDim.x + threadIdx.x;
  bool active = false;
  if (c < v) {
    const float* rg = v_combined + (size_t)c * 10;
#pragma unroll
    for (int k = 0; k < 10; ++k) active = active || rg[k] != 0.0f;
    // a row without gradient: only its flag (and refine) float4 is read
    if (!active) rows[(size_t)c * (VJP_ROW / 4) + 4] = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
  }
  // the rows with a gradient, compacted so that the VJP runs on whole warps
  const uint32_t total = compact_block<128>(active, s_list, s_wcnt);
  if (threadIdx.x >= total) return;
  const uint32_t cc = blockIdx.x * blockDim.x + s_list[threadIdx.x];
  const float* rg = v_combined + (size_t)cc * 10;
  float rr[10];
#pragma unroll
  for (int k = 0; k < 10; ++k) rr[k] = rg[k];
  const uint32_t g = global_from_compact[cc];
  float tt[10];
#pragma unroll
  for (int k = 0; k < 10; ++k) tt[k] = transforms[(size_t)g * 10 + k];
  // the Mip 3D-filter floor enters the VJP when the frame was rendered with one
  const VjpOut r = splat_vjp(tt, raw_opac[g], sh, min_scale, g, rr, u);
  float o[VJP_ROW];
  o[0] = r.v_mean.x; o[1] = r.v_mean.y; o[2] = r.v_mean.z;
  o[3] = r.v_q.w; o[4] = r.v_q.x; o[5] = r.v_q.y; o[6] = r.v_q.z;
  o[7] = r.v_scale.x; o[8] = r.v_scale.y; o[9] = r.v_scale.z;
  o[10] = r.v_raw;
  o[11] = rr[5]; o[12] = rr[6]; o[13] = rr[7];
  o[14] = r.dir.x; o[15] = r.dir.y; o[16] = r.dir.z;
  o[17] = clampf(vs_is_finite(rr[9]) ? rr[9] : 0.0f, 0.0f, 1.0e32f);
  o[18] = 1.0f;
  o[19] = 0.0f;
  float4* d = rows + (size_t)cc * (VJP_ROW / 4);
#pragma unroll
  for (int k = 0; k < (int)(VJP_ROW / 4); ++k) d[k] = make_float4(o[4 * k], o[4 * k + 1], o[4 * k + 2], o[4 * k + 3]);
}

// ---- Q8 Adam ----
struct Q8T {
  uint8_t* mc;
  uint8_t* vc;
  float* ms;
  float* vs;
};

struct Q8Args {
  float b1, b2, inv1, inv2, eps;
  float sqrt_inv2;  // sqrtf(inv2), so sqrt(v inv2) is evaluated as sqrt(v) * sqrt(inv2)
  float lr_t[10];
  float lr_dc, lr_rest, lr_opac, opac_reg;
  uint32_t seed;
  float noise_scale, noise_limit;
  uint32_t noise_seed;
};

// Sharded update over peer replicas (MODE 2 of q8_kernel); world = 1 and
// zero offsets otherwise.
struct PeerArgs {
  uint32_t world, rank;
  // the ctx's device error word: a barrier before this launch that gave up
  // sets VS_DERR_WAIT there, and the update then touches nothing
  const uint32_t* err;
  uint32_t cta_begin;  // first CTA (256 splats) of the shard
  uint32_t m_off;      // first splat covered by the moment arrays
  // MODE 3 (compact rows): `views` slots per rank, rows of slot v at
  // grads[r] + v * n_all * VS_COMPACT_ROW, cameras cams[r] + 4 v, masks[r][g]
  // bit v when slot v saw splat g
  uint32_t views, n_all;
  const float* cams[VS_PEER_MAX];
  const uint32_t* masks[VS_PEER_MAX];
  const float* grads[VS_PEER_MAX];
  const float* vis[VS_PEER_MAX];
  float* t[VS_PEER_MAX];
  float* sh[VS_PEER_MAX];
  float* o[VS_PEER_MAX];
};

constexpr uint32_t Q8_SPLATS = 256;
constexpr uint32_t Q8_WARPS = 8;
// Stochastic-rounding stream salts per tensor (the reference separates its
// transforms and opacity streams the same way, project_update.rs:163-166).
constexpr uint32_t SALT_T = 10u << 24, SALT_SH = 48u << 24, SALT_O = 1u << 24;

__device__ __forceinline__ float hash_uniform(uint32_t key, uint32_t seed) {
  const uint32_t h = vs_mix_hash(key, seed);
  return (float)((h >> 8) + 1u) / 16777216.0f;
}

// Noise on the mean (crates/splat-train/src/housekeep.rs:134-160).
__device__ __forceinline__ void mean_noise(uint32_t i, float opac, float vis, float scale, float limit, uint32_t seed,
                                           float* nx, float* ny, float* nz) {
  *nx = *ny = *nz = 0.0f;
  const float om = 1.0f - opac;
  const float pw = om > 0.0f ? vs_expf(150.0f * vs_logf(om)) : 0.0f;
  // `vis` is a 0/1 mark, or a per-step count of views that saw the splat
  const float gate = clampf(pw, 0.0f, 1.0f) * fminf(vis, 1.0f);
  if (gate > 0.0f) {
    const float w = gate * scale;
    const uint32_t base = i * 4u;
    const float r1 = sqrtf(-2.0f * vs_logf(hash_uniform(base, seed)));
    const float a1 = 6.2831855f * hash_uniform(base + 1u, seed);
    const float r2 = sqrtf(-2.0f * vs_logf(hash_uniform(base + 2u, seed)));
    const float a2 = 6.2831855f * hash_uniform(base + 3u, seed);
    float s1, c1, s2, c2;
    vs_sincosf(a1, &s1, &c1);
    vs_sincosf(a2, &s2, &c2);
    *nx = clampf(r1 * c1 * w, -limit, limit);
    *ny = clampf(r1 * s1 * w, -limit, limit);
    *nz = clampf(r2 * c2 * w, -limit, limit);
  }
}

// Per-CTA shared state of the Q8 step: per-splat transforms/opacity gradients,
// colour gradient and SH bases (the SH gradient is Y_k(dir) * colour, rebuilt
// per value), mean noise, and the 10 transforms learning rates.
struct Q8Shared {
  const float* gt;     // [256][10]
  const float* go;     // [256]
  const float* vc;     // [256][3]
  const float* bas;    // [256][16]
  const float* noise;  // [256][3]
  const float* lr_t;   // [10]
  const uint32_t* vmask;  // [256] ranks whose rows are read (MODE 2)
  const float* gsh;       // [256][Q8_GSH_STRIDE] summed SH gradients (MODE 3)
};

// Row stride of the MODE 3 SH gradients in shared memory (odd: a warp that
// walks the rows of consecutive splats hits distinct banks).
constexpr uint32_t Q8_GSH_STRIDE = 49;

// One 256-value block of one parameter tensor, by one warp.  `W` is the
// tensor's row width (values per splat), `KIND` 0 = transforms, 1 = SH,
// 2 = opacity.  Lane l owns the four consecutive values jb*256 + 128 h + 4 l
// + e (h < 2, e < 4), so a full block moves with two 16-byte parameter loads
// and two 4-byte loads per code stream per lane; all loads are issued before
// any arithmetic.  A block that runs past the tensor's end (only in the last
// CTA) takes guarded scalar accesses instead.
template <int MODE, uint32_t W, int KIND>
__device__ __forceinline__ void q8_block(uint32_t lane, uint32_t jb, uint32_t vals_here, float* __restrict__ tensor,
                                         const Q8T& q, size_t t_base, uint32_t salt, const Q8Args& a,
                                         const Q8Shared& sm, const float* __restrict__ grow, uint32_t width,
                                         const PeerArgs& pa) {
  float* p = tensor + t_base;
  constexpr bool kPeer = MODE >= 2;
  const size_t mb = kPeer ? t_base - (size_t)pa.m_off * W : t_base;  // offset in the moment arrays
  uint8_t* mcp = q.mc + mb;
  uint8_t* vcp = q.vc + mb;
  const size_t blk = mb / 256u + jb;
  const float ms = q.ms[blk], vsc = q.vs[blk];
  const uint32_t v0 = jb * 256u;
  const bool full = v0 + 256u <= vals_here;
  float pv[8], g[8], lr[8], nz[8];
  uint32_t mw[2], vw[2];
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    const uint32_t li0 = v0 + 128u * h + 4u * lane;
    if (full) {
      const float4 x = *reinterpret_cast<const float4*>(p + li0);
      pv[4 * h] = x.x; pv[4 * h + 1] = x.y; pv[4 * h + 2] = x.z; pv[4 * h + 3] = x.w;
      mw[h] = *reinterpret_cast<const uint32_t*>(mcp + li0);
      vw[h] = *reinterpret_cast<const uint32_t*>(vcp + li0);
    } else {
      mw[h] = 0x80808080u;
      vw[h] = 0u;
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const uint32_t li = li0 + (uint32_t)e;
        const bool ok = li < vals_here;
        pv[4 * h + e] = ok ? p[li] : 0.0f;
        if (ok) {
          mw[h] = (mw[h] & ~(0xffu << (8 * e))) | ((uint32_t)mcp[li] << (8 * e));
          vw[h] |= (uint32_t)vcp[li] << (8 * e);
        }
      }
    }
    // gradient, learning rate and mean noise of the four values
    uint32_t s = li0 / W, col = li0 - s * W;
    uint32_t c3 = col / 3u, r3 = col - 3u * c3;
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const uint32_t li = li0 + (uint32_t)e;
      const bool ok = full || li < vals_here;
      const int k = 4 * h + e;
      nz[k] = 0.0f;
      if (KIND == 0) {
        g[k] = ok ? sm.gt[li] : 0.0f;
        lr[k] = sm.lr_t[col];
        if (col < 3u) nz[k] = ok ? sm.noise[s * 3u + col] : 0.0f;
      } else if (KIND == 1) {
        if (MODE == 1) {
          g[k] = ok ? grow[(size_t)s * width + 10u + col] : 0.0f;
        } else if (MODE == 2) {
          // every rank's load is issued before the sum, which runs in rank order
          const uint32_t vm = ok ? sm.vmask[s] : 0u;
          const size_t off = ((size_t)(t_base / W) + s) * width + 10u + col;
          float tv[VS_PEER_MAX];
#pragma unroll
          for (uint32_t r = 0; r < VS_PEER_MAX; ++r) tv[r] = ((vm >> r) & 1u) ? pa.grads[r][off] : 0.0f;
          float acc = 0.0f;
#pragma unroll
          for (uint32_t r = 0; r < VS_PEER_MAX; ++r)
            if ((vm >> r) & 1u) acc += tv[r];
          g[k] = acc;
        } else if (MODE == 3) {
          g[k] = ok ? sm.gsh[s * Q8_GSH_STRIDE + col] : 0.0f;
        } else {
          g[k] = ok ? sm.vc[s * 3u + r3] * sm.bas[s * 16u + c3] : 0.0f;
        }
        lr[k] = c3 == 0u ? a.lr_dc : a.lr_rest;
      } else {
        g[k] = ok ? sm.go[li] : 0.0f;
        lr[k] = a.lr_opac;
      }
      if (++col == W) {
        col = 0u;
        ++s;
        c3 = 0u;
        r3 = 0u;
      } else if (++r3 == 3u) {
        r3 = 0u;
        ++c3;
      }
    }
  }
  float m1[8], r1[8];
  float am = 0.0f, ar = 0.0f;
#pragma unroll
  for (int k = 0; k < 8; ++k) {
    const uint32_t li = v0 + 128u * (uint32_t)(k >> 2) + 4u * lane + (uint32_t)(k & 3);
    // byte b as a float: 2^23 + b has b in its low mantissa bits (exact)
    const uint32_t mb = (mw[k >> 2] >> (8 * (k & 3))) & 0xffu, vb = (vw[k >> 2] >> (8 * (k & 3))) & 0xffu;
    const float m0 = (__uint_as_float(0x4B000000u | mb) - 8388736.0f) * ms;  // (b - 128) * scale
    const float r0 = (__uint_as_float(0x4B000000u | vb) - 8388608.0f) * vsc;
    const float gg = g[k];
    const float m = fmaf(gg, 1.0f - a.b1, m0 * a.b1);
    const float v = fmaf(gg * gg, 1.0f - a.b2, r0 * r0 * a.b2);
    const float r = sqrt_rn(v);
    const float mh = m * a.inv1;
    const float denom = fmaxf(fmaf(r, a.sqrt_inv2, a.eps), fabsf(mh) * 0.125f);
    // mh / denom as mh times the correctly rounded reciprocal (0 from 2^126 on)
    const float inv_d = denom < 8.5070592e37f ? rcp_rn(denom) : 0.0f;
    float pn = fmaf(-(mh * inv_d), lr[k], pv[k]);
    if (KIND == 0) pn = pn + nz[k];
    pv[k] = pn;
    m1[k] = m;
    r1[k] = r;
    if (full || li < vals_here) {
      am = fmaxf(am, fabsf(m));
      ar = fmaxf(ar, r);
    }
  }
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) {
    am = fmaxf(am, __shfl_xor_sync(0xffffffffu, am, off));
    ar = fmaxf(ar, __shfl_xor_sync(0xffffffffu, ar, off));
  }
  const float nms = am / 127.0f, nvs = ar / 255.0f;
  const float inv_ms = nms > 0.0f ? 1.0f / nms : 0.0f, inv_vs = nvs > 0.0f ? 1.0f / nvs : 0.0f;
  if (lane == 0) {
    q.ms[blk] = nms;
    q.vs[blk] = nvs;
  }
  const uint32_t hbase = (uint32_t)t_base;
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    const uint32_t li0 = v0 + 128u * h + 4u * lane;
    uint32_t mo = 0u, vo = 0u;
    // one hash per pair of values: bytes 0/1 are the m and sqrt(v) uniforms of
    // the even value, bytes 2/3 those of the odd one
    const uint32_t hp[2] = {vs_mix_hash((hbase + li0) >> 1, a.seed ^ salt),
                            vs_mix_hash(((hbase + li0) >> 1) + 1u, a.seed ^ salt)};
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const int k = 4 * h + e;
      const uint32_t hb = hp[e >> 1] >> (16 * (e & 1));
      // (b + 1/2) / 256 for a byte b, exactly: (1 + b 2^-8 + 2^-9) - 1
      const float u1 = __uint_as_float(0x3F804000u | ((hb & 0xffu) << 15)) - 1.0f;
      const float u2 = __uint_as_float(0x3F804000u | (((hb >> 8) & 0xffu) << 15)) - 1.0f;
      // clamp(floor(x), lo, hi) = floor(clamp(x, lo, hi)) for integer bounds
      // (NaN clamps to lo either way); floor of |y| < 2^22 is the low
      // mantissa of y + 1.5 2^23 rounded toward -inf.
      const uint32_t qm = nms > 0.0f
          ? __float_as_uint(__fadd_rd(clampf(fmaf(m1[k], inv_ms, u1), -127.0f, 127.0f), 12582912.0f)) - 0x4B400000u + 128u
          : 128u;
      const uint32_t qr = nvs > 0.0f
          ? __float_as_uint(__fadd_rd(clampf(fmaf(r1[k], inv_vs, u2), 0.0f, 255.0f), 12582912.0f)) - 0x4B400000u
          : 0u;
      mo |= qm << (8 * e);
      vo |= qr << (8 * e);
    }
    // MODE 2 stores the parameters into every replica (peers over NVLink)
    const uint32_t nrep = kPeer ? pa.world : 1u;
    for (uint32_t r = 0; r < nrep; ++r) {
      float* pr = kPeer ? (KIND == 0 ? pa.t[r] : (KIND == 1 ? pa.sh[r] : pa.o[r])) + t_base : p;
      if (full) {
        *reinterpret_cast<float4*>(pr + li0) = make_float4(pv[4 * h], pv[4 * h + 1], pv[4 * h + 2], pv[4 * h + 3]);
      } else {
#pragma unroll
        for (int e = 0; e < 4; ++e)
          if (li0 + (uint32_t)e < vals_here) pr[li0 + e] = pv[4 * h + e];
      }
    }
    if (full) {
      *reinterpret_cast<uint32_t*>(mcp + li0) = mo;
      *reinterpret_cast<uint32_t*>(vcp + li0) = vo;
    } else {
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const uint32_t li = li0 + (uint32_t)e;
        if (li < vals_here) {
          mcp[li] = (uint8_t)(mo >> (8 * e));
          vcp[li] = (uint8_t)(vo >> (8 * e));
        }
      }
    }
  }
}

// MODE 0: single view, VJP rows of vjp_rows_kernel; MODE 1: dense gradient
// rows `grads`; MODE 2: dense rows of every rank summed from peer memory, for
// the shard of CTAs starting at pa.cta_begin, parameters stored to all
// replicas.  `n` is one past the last splat this launch may touch.
template <int MODE>
__global__ void __launch_bounds__(Q8_SPLATS, 4) q8_kernel(
    Uniforms u, uint32_t n, float* __restrict__ transforms, float* __restrict__ sh, float* __restrict__ raw_opac,
    const uint32_t* __restrict__ compact_from_global, const float4* __restrict__ vjp_rows,
    const float* __restrict__ grads, Q8T mt, Q8T msh, Q8T mo, Q8Args a,
    const float* __restrict__ opacities, const float* __restrict__ visible, const float* __restrict__ max_radius,
    float* __restrict__ refine_norm, float* __restrict__ vis_count, float* __restrict__ max_screen, PeerArgs pa) {
  __shared__ float s_gt[Q8_SPLATS * 10];
  __shared__ float s_go[Q8_SPLATS];
  __shared__ float s_vc[MODE == 0 ? Q8_SPLATS * 3 : 1];
  __shared__ float s_bas[MODE == 0 ? Q8_SPLATS * 16 : 1];
  __shared__ float s_noise[Q8_SPLATS * 3];
  __shared__ uint32_t s_vmask[MODE == 2 ? Q8_SPLATS : 1];
  __shared__ float s_lr[10];
  constexpr bool kDense = MODE != 0;
  constexpr bool kPeer = MODE >= 2;
  // MODE 3: the summed SH gradients, [256][Q8_GSH_STRIDE] in dynamic shared memory
  extern __shared__ __align__(16) float s_dyn[];
  float* s_gsh = s_dyn;

  const uint32_t tid = threadIdx.x, lane = tid & 31u, warp = tid >> 5;
  // After a barrier that gave up, the peers' rows may be incomplete and other
  // ranks may still read this replica: no peer load or store, no update.
  if (kPeer && (*(volatile const uint32_t*)pa.err & VS_DERR_WAIT)) return;
  const uint32_t base = ((kPeer ? pa.cta_begin : 0u) + blockIdx.x) * Q8_SPLATS;
  if (tid == 0) {
#pragma unroll
    for (int k = 0; k < 10; ++k) s_lr[k] = a.lr_t[k];
  }
  const int nc = (u.sh_degree + 1) * (u.sh_degree + 1);
  const uint32_t wsh = 3u * (uint32_t)nc;
  const uint32_t width = 10u + wsh + 1u;

  // ---- phase 1: per-splat gradients into shared memory ----
  // MODE 0 reads the splat's VJP row (vjp_rows_kernel) and rebuilds its 16 SH
  // bases from the stored view direction; a splat without a gradient row has
  // zero gradients and bases.
  {
    const uint32_t g = base + tid;
    float gr[10];
#pragma unroll
    for (int k = 0; k < 10; ++k) gr[k] = 0.0f;
    float go = 0.0f;
    float vis_g = 0.0f;  // views that saw the splat (MODE 1 and 2)
    float vc[3] = {0.0f, 0.0f, 0.0f};
    float b[16];
#pragma unroll
    for (int k = 0; k < 16; ++k) b[k] = 0.0f;
    if (g < n) {
      if (MODE == 2) {
        uint32_t vm = 0;
        for (uint32_t r = 0; r < pa.world; ++r) {
          const float vr = pa.vis[r][g];
          if (vr > 0.0f) vm |= 1u << r;
          vis_g += vr;
        }
        for (uint32_t r = 0; r < pa.world; ++r) {
          if (!((vm >> r) & 1u)) continue;
          const float* d = pa.grads[r] + (size_t)g * width;
#pragma unroll
          for (int k = 0; k < 10; ++k) gr[k] += d[k];
          go += d[width - 1];
        }
        s_vmask[tid] = vm;
      } else if (MODE == 3) {
        // compact rows: over every (rank, view slot) that saw the splat, in
        // that order, the transforms and opacity gradients summed and the SH
        // gradient rebuilt from the slot's colour gradient and the view
        // direction and basis computed as splat_vjp computes them (same
        // mean, same camera), each sum from 0 one term per view: the sums of
        // one dense row accumulated over the same views, bit for bit
        float* gs = s_gsh + tid * Q8_GSH_STRIDE;
        for (uint32_t j = 0; j < wsh; ++j) gs[j] = 0.0f;
        uint32_t vm = 0;
        for (uint32_t r = 0; r < pa.world; ++r) {
          const float vr = pa.vis[r][g];
          if (vr > 0.0f) vm |= 1u << r;
          vis_g += vr;
        }
        if (vm) {
          const V3 mean = {transforms[(size_t)g * 10], transforms[(size_t)g * 10 + 1],
                           transforms[(size_t)g * 10 + 2]};
          for (uint32_t r = 0; r < pa.world; ++r) {
            if (!((vm >> r) & 1u)) continue;
            uint32_t slots = pa.masks[r][g];
            if (pa.views < 32) slots &= (1u << pa.views) - 1u;
            while (slots) {
              const uint32_t v = (uint32_t)(__ffs(slots) - 1);
              slots &= slots - 1u;
              const float4* row = reinterpret_cast<const float4*>(
                  pa.grads[r] + ((size_t)v * pa.n_all + g) * VS_COMPACT_ROW);
              const float4 x0 = row[0], x1 = row[1], x2 = row[2], x3 = row[3];
              const float* cp = pa.cams[r] + 4u * v;
              const V3 cam = {cp[0], cp[1], cp[2]};
              gr[0] += x0.x; gr[1] += x0.y; gr[2] += x0.z; gr[3] += x0.w;
              gr[4] += x1.x; gr[5] += x1.y; gr[6] += x1.z; gr[7] += x1.w;
              gr[8] += x2.x; gr[9] += x2.y; go += x2.z;
              const float cv[3] = {x2.w, x3.x, x3.y};
              const V3 uw = v3sub(mean, cam);
              const float ulen = sqrtf(v3dot(uw, uw));
              const V3 dv = v3scale(uw, 1.0f / ulen);
              sh_basis_all(dv.x, dv.y, dv.z, b);
#pragma unroll
              for (int k = 0; k < 16; ++k) {
                if (k < nc) {
#pragma unroll
                  for (int q = 0; q < 3; ++q) gs[k * 3 + q] = gs[k * 3 + q] + cv[q] * b[k];
                }
              }
            }
          }
        }
      } else if (kDense) {
        const float* d = grads + (size_t)g * width;
#pragma unroll
        for (int k = 0; k < 10; ++k) gr[k] = d[k];
        go = d[width - 1];
        if (visible) vis_g = visible[g];
      } else {
        const uint32_t row = compact_from_global[g];
        float refine = 0.0f;
        if (row > 0) {
          const float4* r4 = vjp_rows + (size_t)(row - 1) * (VJP_ROW / 4);
          const float4 x4 = r4[4];  // refine, flag: the only part written for a row without gradient
          if (x4.z != 0.0f) {
            const float4 x0 = r4[0], x1 = r4[1], x2 = r4[2], x3 = r4[3];
            gr[0] = x0.x; gr[1] = x0.y; gr[2] = x0.z; gr[3] = x0.w;
            gr[4] = x1.x; gr[5] = x1.y; gr[6] = x1.z; gr[7] = x1.w;
            gr[8] = x2.x; gr[9] = x2.y; go = x2.z;
            vc[0] = x2.w; vc[1] = x3.x; vc[2] = x3.y;
            sh_basis_all(x3.z, x3.w, x4.x, b);
            refine = x4.y;
          }
        }
        if (refine_norm) refine_norm[g] = fmaxf(refine_norm[g], refine);
        if (vis_count) vis_count[g] += visible[g];
        if (max_screen) max_screen[g] = fmaxf(max_screen[g], max_radius[g]);
      }
    }
#pragma unroll
    for (int k = 0; k < 10; ++k) s_gt[tid * 10 + k] = gr[k];
    s_go[tid] = go;
    if (!kDense) {
      s_vc[tid * 3 + 0] = vc[0];
      s_vc[tid * 3 + 1] = vc[1];
      s_vc[tid * 3 + 2] = vc[2];
#pragma unroll
      for (int k = 0; k < 16; ++k) s_bas[tid * 16 + k] = b[k];
    }
    // opacity regulariser and mean noise, one splat per thread again
    float nx = 0.0f, ny = 0.0f, nz = 0.0f;
    if (g < n) {
      if (a.opac_reg != 0.0f) {
        const float o = 1.0f / (1.0f + vs_expf(-raw_opac[g]));
        s_go[tid] = s_go[tid] + a.opac_reg * o * (1.0f - o);
      }
      if ((visible || kPeer) && a.noise_scale != 0.0f) {
        // without per-view opacities (the multi-view path) the gate uses the
        // unfloored sigmoid opacity, which projection also reports when no
        // min_scale floor is set
        const float op = opacities ? opacities[g] : 1.0f / (1.0f + vs_expf(-raw_opac[g]));
        mean_noise(g, op, kDense ? vis_g : visible[g], a.noise_scale, a.noise_limit, a.noise_seed, &nx, &ny, &nz);
      }
    }
    s_noise[tid * 3 + 0] = nx;
    s_noise[tid * 3 + 1] = ny;
    s_noise[tid * 3 + 2] = nz;
  }
  __syncthreads();

  // ---- phase 2: one warp per 256-value quantization block ----
  const uint32_t splats_here = min(Q8_SPLATS, n - base);
  const uint32_t nb_t = div_up(splats_here * 10u, 256u);
  const uint32_t nb_sh = div_up(splats_here * wsh, 256u);
  const uint32_t total_blocks = nb_t + nb_sh + 1u;
  const Q8Shared sm{s_gt, s_go, s_vc, s_bas, s_noise, s_lr, s_vmask, s_gsh};
  const float* grow = MODE == 1 ? grads + (size_t)base * width : nullptr;
  for (uint32_t job = warp; job < total_blocks; job += Q8_WARPS) {
    if (job < nb_t) {
      q8_block<MODE, 10, 0>(lane, job, splats_here * 10u, transforms, mt, (size_t)base * 10u, SALT_T, a, sm,
                            grow, width, pa);
    } else if (job < nb_t + nb_sh) {
      const uint32_t jb = job - nb_t;
      const size_t tb = (size_t)base * wsh;
      switch (u.sh_degree) {
        case 3: q8_block<MODE, 48, 1>(lane, jb, splats_here * 48u, sh, msh, tb, SALT_SH, a, sm, grow, width, pa); break;
        case 2: q8_block<MODE, 27, 1>(lane, jb, splats_here * 27u, sh, msh, tb, SALT_SH, a, sm, grow, width, pa); break;
        case 1: q8_block<MODE, 12, 1>(lane, jb, splats_here * 12u, sh, msh, tb, SALT_SH, a, sm, grow, width, pa); break;
        default: q8_block<MODE, 3, 1>(lane, jb, splats_here * 3u, sh, msh, tb, SALT_SH, a, sm, grow, width, pa); break;
      }
    } else {
      q8_block<MODE, 1, 2>(lane, 0, splats_here, raw_opac, mo, (size_t)base, SALT_O, a, sm, grow, width, pa);
    }
  }
  // Peer stores complete before the barrier that follows this kernel: the
  // block barrier orders every thread's stores before thread 0's system-scope
  // fence, which releases them all (one fence per CTA instead of one per warp
  // waiting at its exit).
  if (kPeer) {
    __syncthreads();
    if (tid == 0) __threadfence_system();
  }
}

PeerArgs single_rank() {
  PeerArgs pa{};
  pa.world = 1;
  return pa;
}

__global__ void stats_kernel(uint32_t n, float* norm, float* vis, float* screen, const float* weight,
                             const float* visible, const float* radius) {
  const uint32_t i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) {
    norm[i] = fmaxf(norm[i], weight[i]);
    vis[i] += visible[i];
    screen[i] = fmaxf(screen[i], radius[i]);
  }
}

__global__ void noise_kernel(uint32_t n, float* transforms, const float* opacities, const float* visible, float scale,
                             float limit, uint32_t seed) {
  const uint32_t i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  float nx, ny, nz;
  mean_noise(i, opacities[i], visible[i], scale, limit, seed, &nx, &ny, &nz);
  if (nx != 0.0f || ny != 0.0f || nz != 0.0f) {
    float* t = transforms + (size_t)i * 10;
    t[0] += nx;
    t[1] += ny;
    t[2] += nz;
  }
}

Q8T to_q8(const vs_q8_tensor& t) { return {t.m_codes, t.v_codes, t.m_scales, t.v_scales}; }

Q8Args to_args(const vs_q8_cfg& c) {
  Q8Args a;
  a.b1 = c.beta1; a.b2 = c.beta2; a.inv1 = c.inv1; a.inv2 = c.inv2; a.eps = c.epsilon;
  for (int k = 0; k < 10; ++k) a.lr_t[k] = c.lr_transforms[k];
  a.lr_dc = c.lr_sh_dc; a.lr_rest = c.lr_sh_rest; a.lr_opac = c.lr_opac; a.opac_reg = c.opac_reg;
  a.seed = c.seed;
  a.noise_scale = c.noise_scale; a.noise_limit = c.noise_limit; a.noise_seed = c.noise_seed;
  a.sqrt_inv2 = sqrtf(c.inv2);
  return a;
}

bool q8_valid(const vs_q8_tensor& t) { return t.m_codes && t.v_codes && t.m_scales && t.v_scales; }

// The Q8 kernels move parameters and codes in 16-byte pieces (bulk copies and
// vector accesses).
bool a16(const void* p) { return ((uintptr_t)p & 15u) == 0; }
bool q8_aligned(const void* t, const void* sh, const void* o, const vs_q8_tensor& mt, const vs_q8_tensor& msh,
                const vs_q8_tensor& mo) {
  return a16(t) && a16(sh) && a16(o) && a16(mt.m_codes) && a16(mt.v_codes) && a16(msh.m_codes) &&
         a16(msh.v_codes) && a16(mo.m_codes) && a16(mo.v_codes);
}

}  // namespace

// ---------------------------------------------------------------------------
extern "C" {

VS_API vs_status vs_project_update(vs_ctx* ctx, vs_frame* frame, const vs_render_cfg* cfg, uint32_t num_splats,
                                   float* transforms, const void* sh_coeffs, float* raw_opacities,
                                   const float* min_scale, const float* v_combined, uint32_t* w_t,
                                   const float* lr_scale, uint32_t* w_o, const vs_adam_cfg* adam, float* color_dir,
                                   float* v_refine, float* grad_sq, float* variance, int32_t first_step) {
  if (!ctx) return VS_ERR_INVALID;
  if (!frame || !frame->rendered || !cfg || !adam || !lr_scale)
    return vs_fail(ctx, VS_ERR_INVALID, "project_update: missing frame/config");
  if (num_splats != frame->n) return vs_fail(ctx, VS_ERR_INVALID, "project_update: %u splats, frame has %u", num_splats, frame->n);
  if (!transforms || !sh_coeffs || !raw_opacities || !w_t || !w_o || !color_dir || !v_refine || !grad_sq ||
      (frame->v && !v_combined))
    return vs_fail(ctx, VS_ERR_INVALID, "project_update: null buffer");
  if (num_splats == 0) return VS_OK;
  AdamArgs a;
  a.b1 = adam->beta1; a.b2 = adam->beta2; a.inv1 = adam->inv1; a.inv2 = adam->inv2; a.eps = adam->epsilon;
  a.lr_opac = adam->lr_opac; a.opac_reg = adam->opac_reg; a.seed = adam->round_seed;
  for (int k = 0; k < 10; ++k) a.lr_scale[k] = lr_scale[k];
  vs::Uniforms u = frame->u;
  u.sh_half = cfg->sh_half;
  project_update_kernel<<<vs::div_up(num_splats, 256), 256, 0, ctx->stream>>>(
      u, num_splats, transforms, sh_coeffs, raw_opacities, min_scale,
      (const uint32_t*)frame->compact_from_global.ptr, v_combined, w_t, w_o, a, color_dir, v_refine, grad_sq, variance,
      first_step); ++ctx->launches;
  return vs_cuda(ctx, cudaGetLastError(), "project_update launch");
}

VS_API vs_status vs_sh_step(vs_ctx* ctx, uint32_t num_splats, uint32_t row_width, uint16_t* sh_f16,
                            const float* color_dir, const uint32_t* grad_rows, uint32_t* codes, float* scales,
                            const float* variance, const float* lr_scale, float beta, float factor, float inv1,
                            float inv2, float epsilon, float lr, uint32_t round_seed) {
  if (!ctx) return VS_ERR_INVALID;
  if (!sh_f16 || !color_dir || !grad_rows || !codes || !scales || !variance || !lr_scale || row_width == 0 ||
      row_width > 48 || row_width % 3 != 0)
    return vs_fail(ctx, VS_ERR_INVALID, "sh_step: bad arguments");
  const uint64_t count = (uint64_t)num_splats * row_width;
  if (count >= 0xffffffffull) return vs_fail(ctx, VS_ERR_CAPACITY, "sh_step: %llu values exceed u32 indexing", (unsigned long long)count);
  if (count == 0) return VS_OK;
  const uint32_t nblocks = (uint32_t)((count + 127) / 128);
  VS_TRY(vs_ensure(ctx, ctx->misc, 48 * 4));
  VS_CUDA(ctx, cudaMemcpyAsync(ctx->misc.ptr, lr_scale, row_width * 4, cudaMemcpyHostToDevice, ctx->stream));
  ShStepArgs a{beta, factor, inv1, inv2, epsilon, lr, round_seed};
  sh_step_kernel<<<vs::div_up(nblocks, 4), 128, 0, ctx->stream>>>((uint32_t)count, row_width, sh_f16, color_dir,
                                                                  grad_rows, codes, scales, variance,
                                                                  (const float*)ctx->misc.ptr, nblocks, a); ++ctx->launches;
  return vs_cuda(ctx, cudaGetLastError(), "sh_step launch");
}

VS_API vs_status vs_step_q8(vs_ctx* ctx, vs_frame* frame, const vs_render_cfg* cfg, uint32_t num_splats,
                            float* transforms, float* sh_coeffs, float* raw_opacities, const float* min_scale,
                            const float* v_combined,
                            vs_q8_tensor mom_t, vs_q8_tensor mom_sh, vs_q8_tensor mom_o, const vs_q8_cfg* q8,
                            const float* visible, float* refine_norm, float* vis_count, float* max_screen) {
  if (!ctx) return VS_ERR_INVALID;
  if (!frame || !frame->rendered || !cfg || !q8) return vs_fail(ctx, VS_ERR_INVALID, "step_q8: missing frame/config");
  if (num_splats != frame->n) return vs_fail(ctx, VS_ERR_INVALID, "step_q8: %u splats, frame has %u", num_splats, frame->n);
  if (cfg->sh_half) return vs_fail(ctx, VS_ERR_UNSUPPORTED, "step_q8: SH coefficients must be f32");
  if (frame->u.has_min_scale && !min_scale)
    return vs_fail(ctx, VS_ERR_INVALID, "step_q8: the frame was rendered with a min_scale floor; pass it");
  if (!transforms || !sh_coeffs || !raw_opacities || (frame->v && !v_combined) || !q8_valid(mom_t) ||
      !q8_valid(mom_sh) || !q8_valid(mom_o))
    return vs_fail(ctx, VS_ERR_INVALID, "step_q8: null buffer");
  if ((refine_norm || vis_count || max_screen || q8->noise_scale != 0.0f) && !visible)
    return vs_fail(ctx, VS_ERR_INVALID, "step_q8: statistics and noise need `visible`");
  if (!q8_aligned(transforms, sh_coeffs, raw_opacities, mom_t, mom_sh, mom_o))
    return vs_fail(ctx, VS_ERR_INVALID, "step_q8: parameter and code arrays must be 16-byte aligned");
  const uint64_t count_sh = (uint64_t)num_splats * 3 * (cfg->sh_degree + 1) * (cfg->sh_degree + 1);
  if (count_sh >= 0xffffffffull) return vs_fail(ctx, VS_ERR_CAPACITY, "step_q8: %llu SH values exceed u32 indexing", (unsigned long long)count_sh);
  if (num_splats == 0) return VS_OK;
  const Q8Args a = to_args(*q8);
  // the VJP rows live in the ctx's scratch until the optimizer kernel has read them
  VS_TRY(vs_ensure(ctx, ctx->vjp_rows, ((size_t)frame->v + 1) * VJP_ROW * 4));
  if (frame->v > 0) {
    vjp_rows_kernel<<<vs::div_up(frame->v, 128), 128, 0, ctx->stream>>>(
        frame->u, frame->v, (const uint32_t*)frame->global_from_compact.ptr, transforms, sh_coeffs, raw_opacities,
        frame->u.has_min_scale ? min_scale : nullptr, v_combined, (float4*)ctx->vjp_rows.ptr); ++ctx->launches;
  }
  q8_kernel<0><<<vs::div_up(num_splats, Q8_SPLATS), Q8_SPLATS, 0, ctx->stream>>>(
      frame->u, num_splats, transforms, sh_coeffs, raw_opacities, (const uint32_t*)frame->compact_from_global.ptr,
      (const float4*)ctx->vjp_rows.ptr, nullptr, to_q8(mom_t), to_q8(mom_sh), to_q8(mom_o), a,
      (const float*)frame->opacities.ptr, visible, (const float*)frame->max_radius.ptr, refine_norm, vis_count,
      max_screen, single_rank()); ++ctx->launches;
  return vs_cuda(ctx, cudaGetLastError(), "step_q8 launch");
}

VS_API vs_status vs_vjp_dense(vs_ctx* ctx, vs_frame* frame, const vs_render_cfg* cfg, uint32_t num_splats,
                              const float* transforms, const void* sh_coeffs, const float* raw_opacities,
                              const float* min_scale, const float* v_combined, float* grads, float* refine,
                              const float* visible, float* vis_accum) {
  if (!ctx) return VS_ERR_INVALID;
  if (!frame || !frame->rendered || !cfg) return vs_fail(ctx, VS_ERR_INVALID, "vjp_dense: missing frame/config");
  if (num_splats != frame->n) return vs_fail(ctx, VS_ERR_INVALID, "vjp_dense: %u splats, frame has %u", num_splats, frame->n);
  if (!transforms || !sh_coeffs || !raw_opacities || !grads || !refine || (frame->v && !v_combined) ||
      (vis_accum && !visible))
    return vs_fail(ctx, VS_ERR_INVALID, "vjp_dense: null buffer");
  if (num_splats == 0) return VS_OK;
  vs::Uniforms u = frame->u;
  u.sh_half = cfg->sh_half;
  if (frame->v == 0) return VS_OK;
  vjp_dense_kernel<false><<<vs::div_up(frame->v, 256), 256, 0, ctx->stream>>>(
      u, frame->v, transforms, sh_coeffs, raw_opacities, min_scale, (const uint32_t*)frame->global_from_compact.ptr,
      v_combined, grads, refine, visible, vis_accum, nullptr, nullptr, 0u, ctx->d_err); ++ctx->launches;
  return vs_cuda(ctx, cudaGetLastError(), "vjp_dense launch");
}

VS_API vs_status vs_vjp_compact(vs_ctx* ctx, vs_frame* frame, const vs_render_cfg* cfg, uint32_t num_splats,
                                const float* transforms, const void* sh_coeffs, const float* raw_opacities,
                                const float* min_scale, const float* v_combined, float* rows, float* refine,
                                const float* visible, float* vis_accum, uint32_t* view_mask, uint32_t slot,
                                float* cam_out) {
  if (!ctx) return VS_ERR_INVALID;
  if (!frame || !frame->rendered || !cfg) return vs_fail(ctx, VS_ERR_INVALID, "vjp_compact: missing frame/config");
  if (num_splats != frame->n)
    return vs_fail(ctx, VS_ERR_INVALID, "vjp_compact: %u splats, frame has %u", num_splats, frame->n);
  if (!transforms || !sh_coeffs || !raw_opacities || !rows || !refine || !visible || !vis_accum || !cam_out ||
      !view_mask || (frame->v && !v_combined))
    return vs_fail(ctx, VS_ERR_INVALID, "vjp_compact: null buffer");
  if (slot >= 32) return vs_fail(ctx, VS_ERR_INVALID, "vjp_compact: view slot %u (0..31)", slot);
  if ((reinterpret_cast<uintptr_t>(rows) | reinterpret_cast<uintptr_t>(cam_out)) & 15u)
    return vs_fail(ctx, VS_ERR_INVALID, "vjp_compact: rows and cam_out must be 16-byte aligned");
  // with no visible splat no rank reads this rank's rows or camera
  if (num_splats == 0 || frame->v == 0) return VS_OK;
  vs::Uniforms u = frame->u;
  u.sh_half = cfg->sh_half;
  vjp_dense_kernel<true><<<vs::div_up(frame->v, 256), 256, 0, ctx->stream>>>(
      u, frame->v, transforms, sh_coeffs, raw_opacities, min_scale, (const uint32_t*)frame->global_from_compact.ptr,
      v_combined, rows, refine, visible, vis_accum, cam_out, view_mask, slot, ctx->d_err); ++ctx->launches;
  return vs_cuda(ctx, cudaGetLastError(), "vjp_compact launch");
}

VS_API vs_status vs_adam_q8_dense(vs_ctx* ctx, uint32_t num_splats, int32_t sh_degree, float* transforms,
                                  float* sh_coeffs, float* raw_opacities, const float* grads, vs_q8_tensor mom_t,
                                  vs_q8_tensor mom_sh, vs_q8_tensor mom_o, const vs_q8_cfg* q8,
                                  const float* opacities, const float* visible) {
  if (!ctx) return VS_ERR_INVALID;
  if (!q8 || !transforms || !sh_coeffs || !raw_opacities || !grads || !q8_valid(mom_t) || !q8_valid(mom_sh) ||
      !q8_valid(mom_o) || sh_degree < 0 || sh_degree > 3)
    return vs_fail(ctx, VS_ERR_INVALID, "adam_q8_dense: bad arguments");
  if (!q8_aligned(transforms, sh_coeffs, raw_opacities, mom_t, mom_sh, mom_o))
    return vs_fail(ctx, VS_ERR_INVALID, "adam_q8_dense: parameter and code arrays must be 16-byte aligned");
  if (num_splats == 0) return VS_OK;
  vs::Uniforms u{};
  u.sh_degree = sh_degree;
  const Q8Args a = to_args(*q8);
  q8_kernel<1><<<vs::div_up(num_splats, Q8_SPLATS), Q8_SPLATS, 0, ctx->stream>>>(
      u, num_splats, transforms, sh_coeffs, raw_opacities, nullptr, nullptr, grads, to_q8(mom_t),
      to_q8(mom_sh), to_q8(mom_o), a, opacities, visible, nullptr, nullptr, nullptr, nullptr, single_rank());
  ++ctx->launches;
  return vs_cuda(ctx, cudaGetLastError(), "adam_q8_dense launch");
}

VS_API vs_status vs_adam_q8_peer(vs_ctx* ctx, uint32_t num_splats, int32_t sh_degree, uint32_t splat_begin,
                                 uint32_t splat_end, const vs_peer_set* peers, vs_q8_tensor mom_t,
                                 vs_q8_tensor mom_sh, vs_q8_tensor mom_o, const vs_q8_cfg* q8) {
  if (!ctx) return VS_ERR_INVALID;
  if (!q8 || !peers || !q8_valid(mom_t) || !q8_valid(mom_sh) || !q8_valid(mom_o) || sh_degree < 0 || sh_degree > 3)
    return vs_fail(ctx, VS_ERR_INVALID, "adam_q8_peer: bad arguments");
  if (peers->world == 0 || peers->world > VS_PEER_MAX || peers->rank >= peers->world)
    return vs_fail(ctx, VS_ERR_INVALID, "adam_q8_peer: world %u rank %u", peers->world, peers->rank);
  if (splat_begin % Q8_SPLATS != 0 || splat_begin > splat_end || splat_end > num_splats)
    return vs_fail(ctx, VS_ERR_INVALID, "adam_q8_peer: shard [%u, %u) of %u splats", splat_begin, splat_end,
                   num_splats);
  const uint64_t count_sh = (uint64_t)num_splats * 3 * (sh_degree + 1) * (sh_degree + 1);
  if (count_sh >= 0xffffffffull) return vs_fail(ctx, VS_ERR_CAPACITY, "adam_q8_peer: %llu SH values exceed u32 indexing", (unsigned long long)count_sh);
  if (peers->row_format > 1) return vs_fail(ctx, VS_ERR_INVALID, "adam_q8_peer: row format %u", peers->row_format);
  const bool compact = peers->row_format == 1;
  if (compact && (peers->views == 0 || peers->views > 32))
    return vs_fail(ctx, VS_ERR_INVALID, "adam_q8_peer: %u views per rank (1..32)", peers->views);
  PeerArgs pa{};
  pa.world = peers->world;
  pa.rank = peers->rank;
  pa.err = ctx->d_err;
  pa.cta_begin = splat_begin / Q8_SPLATS;
  pa.m_off = splat_begin;
  pa.views = peers->views;
  pa.n_all = num_splats;
  for (uint32_t r = 0; r < peers->world; ++r) {
    if (!peers->grads[r] || !peers->vis[r] || !peers->transforms[r] || !peers->sh_coeffs[r] ||
        !peers->raw_opacities[r] || (compact && !peers->cams[r]))
      return vs_fail(ctx, VS_ERR_INVALID, "adam_q8_peer: null buffer of rank %u", r);
    if (compact && (!peers->view_masks[r] || (reinterpret_cast<uintptr_t>(peers->grads[r]) & 15u)))
      return vs_fail(ctx, VS_ERR_INVALID, "adam_q8_peer: compact rows need view masks and 16-byte alignment");
    pa.cams[r] = compact ? peers->cams[r] : nullptr;
    pa.masks[r] = compact ? peers->view_masks[r] : nullptr;
    if (!q8_aligned(peers->transforms[r], peers->sh_coeffs[r], peers->raw_opacities[r], mom_t, mom_sh, mom_o))
      return vs_fail(ctx, VS_ERR_INVALID, "adam_q8_peer: parameter and code arrays must be 16-byte aligned");
    pa.grads[r] = peers->grads[r];
    pa.vis[r] = peers->vis[r];
    pa.t[r] = peers->transforms[r];
    pa.sh[r] = peers->sh_coeffs[r];
    pa.o[r] = peers->raw_opacities[r];
  }
  if (splat_end == splat_begin) return VS_OK;
  vs::Uniforms u{};
  u.sh_degree = sh_degree;
  const Q8Args a = to_args(*q8);
  const uint32_t me = peers->rank;
  if (compact) {
    // the compact rows are summed, and the SH gradient rebuilt, in shared memory
    constexpr int kGshBytes = (int)(Q8_SPLATS * Q8_GSH_STRIDE * sizeof(float));
    VS_CUDA(ctx, cudaFuncSetAttribute(q8_kernel<3>, cudaFuncAttributeMaxDynamicSharedMemorySize, kGshBytes));
    q8_kernel<3><<<vs::div_up(splat_end - splat_begin, Q8_SPLATS), Q8_SPLATS, kGshBytes, ctx->stream>>>(
        u, splat_end, pa.t[me], pa.sh[me], pa.o[me], nullptr, nullptr, nullptr, to_q8(mom_t), to_q8(mom_sh),
        to_q8(mom_o), a, nullptr, nullptr, nullptr, nullptr, nullptr, nullptr, pa);
  } else {
    q8_kernel<2><<<vs::div_up(splat_end - splat_begin, Q8_SPLATS), Q8_SPLATS, 0, ctx->stream>>>(
        u, splat_end, pa.t[me], pa.sh[me], pa.o[me], nullptr, nullptr, nullptr, to_q8(mom_t), to_q8(mom_sh),
        to_q8(mom_o), a, nullptr, nullptr, nullptr, nullptr, nullptr, nullptr, pa);
  }
  ++ctx->launches;
  return vs_cuda(ctx, cudaGetLastError(), "adam_q8_peer launch");
}

VS_API vs_status vs_gather_stats(vs_ctx* ctx, uint32_t n, float* refine_norm, float* vis_count, float* max_screen,
                                 const float* refine_weight, const float* visible, const float* radius) {
  if (!ctx) return VS_ERR_INVALID;
  if (!refine_norm || !vis_count || !max_screen || !refine_weight || !visible || !radius)
    return vs_fail(ctx, VS_ERR_INVALID, "gather_stats: null buffer");
  if (n == 0) return VS_OK;
  stats_kernel<<<vs::div_up(n, 256), 256, 0, ctx->stream>>>(n, refine_norm, vis_count, max_screen, refine_weight,
                                                            visible, radius); ++ctx->launches;
  return vs_cuda(ctx, cudaGetLastError(), "gather_stats launch");
}

VS_API vs_status vs_noise_means(vs_ctx* ctx, uint32_t n, float* transforms, const float* opacities,
                                const float* visible, float scale, float limit, uint32_t seed) {
  if (!ctx) return VS_ERR_INVALID;
  if (!transforms || !opacities || !visible) return vs_fail(ctx, VS_ERR_INVALID, "noise_means: null buffer");
  if (n == 0) return VS_OK;
  noise_kernel<<<vs::div_up(n, 256), 256, 0, ctx->stream>>>(n, transforms, opacities, visible, scale, limit, seed); ++ctx->launches;
  return vs_cuda(ctx, cudaGetLastError(), "noise_means launch");
}

}  // extern "C"
