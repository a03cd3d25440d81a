// Projection: cull, EWA covariance, conic, tile counting and SH colour for
// every splat, with the visible set compacted in global order.
//
// Replaces the reference's project_forward_kernel + project_visible_kernel
// (crates/splat-train-render/src/kernels/project_forward.rs:26-261,
// kernels/project_visible.rs:97-174).  The reference appends visible splats
// with an atomic counter (nondeterministic order); here each block ranks its
// visible splats and a single-pass decoupled look-back over block aggregates
// gives every visible splat its rank in global order, so the compact ids (and
// everything downstream) are deterministic.
#include <cuda/atomic>

#include "vs_internal.cuh"

namespace {

using namespace vs;

constexpr uint32_t PROJ_BLOCK = 256;
constexpr uint32_t BIG_BOX = 16;  // boxes above this many tiles are walked by the whole warp
constexpr uint32_t SPIN_LIMIT = 1u << 22;

struct ProjOut {
  float xy_x, xy_y;
  S2 conic;
  float opac, pt, depth, radius;
  TileBox box;
  float floor_opac;
  bool floor_reached;
};

// kernels/project_forward.rs:62-194 for one splat.
__device__ bool project_one(const float* __restrict__ t, float raw_opac, const float* min_scale, uint32_t g,
                            const Uniforms& u, ProjOut* o) {
  o->floor_reached = false;
  const V3 mean = {t[0], t[1], t[2]};
  const V3 mean_c = world_to_cam(mean, u);
  if (!(v3finite(mean_c) && mean_c.z <= 1.0e10f)) return false;
  if (mean_c.z < 0.01f) return false;
  const V3 scale = {vs_expf(t[7] + u.log_scale_offset), vs_expf(t[8] + u.log_scale_offset),
                    vs_expf(t[9] + u.log_scale_offset)};
  if (!v3finite(scale)) return false;
  const Q4 qu = {t[3], t[4], t[5], t[6]};
  const float qn = q4dot(qu);
  if (!(qn >= 1.0e-6f && vs_is_finite(qn))) return false;
  if (!vs_is_finite(raw_opac)) return false;
  const Q4 q = q4scale(qu, 1.0f / sqrtf(qn));
  const Floor fl = apply_scale_floor(scale, vs_sigmoid(raw_opac), min_scale, g, u.has_min_scale != 0);
  o->floor_opac = fl.opac;
  o->floor_reached = true;
  const S2 raw = calc_cov2d(fl.scale, q, mean_c, u);
  float comp;
  const S2 cov = compensate_cov2d(raw, u.mip != 0, &comp);
  const float opac = fl.opac * comp;
  if (!s2finite(cov)) return false;
  const float inv_z = 1.0f / mean_c.z;
  const float px = u.fx * mean_c.x * inv_z + u.cx;
  const float py = u.fy * mean_c.y * inv_z + u.cy;
  if (!(opac >= ALPHA_MIN)) return false;
  const float pt = vs_logf(opac * 255.0f);
  const S2 conic = s2inverse(cov);
  float ex, ey;
  bbox_extent(conic, pt, &ex, &ey);
  if (!(ex >= 0.0f && ey >= 0.0f)) return false;
  const float wf = (float)u.w, hf = (float)u.h;
  const bool on_screen = px + ex > 0.0f && px - ex < wf && py + ey > 0.0f && py - ey < hf;
  if (!on_screen) return false;
  o->xy_x = px;
  o->xy_y = py;
  o->conic = conic;
  o->opac = opac;
  o->pt = pt;
  o->depth = mean_c.z;
  o->radius = fmaxf(ex / wf, ey / hf);
  o->box = tile_bbox(px, py, ex, ey, u.tbw, u.tbh);
  return true;
}

// Bit i of the result: box tile i (row-major in the box) is hit.
__device__ uint32_t hit_mask_box(const TileBox& b, float mx, float my, S2 c, float pt) {
  const uint32_t bw = b.x1 - b.x0;
  const uint32_t nb = (b.y1 - b.y0) * bw;
  uint32_t mask = 0;
  for (uint32_t i = 0; i < nb; ++i) {
    const uint32_t tx = i % bw + b.x0, ty = i / bw + b.y0;
    if (tile_hit(tx, ty, mx, my, c, pt)) mask |= 1u << i;
  }
  return mask;
}

// SH colour with the +0.5 offset, NaN scrub and clamp
// (kernels/project_visible.rs:26-61, kernels/sh.rs:51-140), bands <= 3.
__device__ V3 splat_color(const void* sh, bool half, uint32_t g, int deg, V3 mean, const Uniforms& u) {
  const V3 d = v3sub(mean, V3{u.cam[0], u.cam[1], u.cam[2]});
  const V3 v = v3scale(d, 1.0f / sqrtf(v3dot(d, d)));
  const int nc = (deg + 1) * (deg + 1);
  const int cnt = nc * 3;
  const size_t base = (size_t)g * cnt;
  // All coefficients are loaded before any is used: 16-byte loads when the
  // row is f32, a multiple of 16 bytes long (degrees 1 and 3) and the array
  // starts on a 16-byte boundary.
  float cf[48];
  if (!half && (cnt & 3) == 0 && (reinterpret_cast<uintptr_t>(sh) & 15u) == 0) {
    const float4* p4 = reinterpret_cast<const float4*>((const float*)sh + base);
#pragma unroll
    for (int q = 0; q < 12; ++q) {
      const float4 v = 4 * q < cnt ? p4[q] : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
      cf[4 * q] = v.x;
      cf[4 * q + 1] = v.y;
      cf[4 * q + 2] = v.z;
      cf[4 * q + 3] = v.w;
    }
  } else {
#pragma unroll
    for (int k = 0; k < 48; ++k) cf[k] = k < cnt ? sh_load(sh, half, base + k) : 0.0f;
  }
  auto rc = [&](int k) -> V3 { return {cf[k], cf[k + 1], cf[k + 2]}; };
  V3 color = v3scale(rc(0), SH_C0);
  if (deg >= 1) {
    const float f0a = 0.4886025f;
    color = v3add(color, v3scale(rc(3), -f0a * v.y));
    color = v3add(color, v3scale(rc(6), f0a * v.z));
    color = v3add(color, v3scale(rc(9), -f0a * v.x));
    if (deg >= 2) {
      const float z2 = v.z * v.z;
      const float f0b = -1.0925485f * v.z;
      const float f1a = 0.54627424f;
      const float fc1 = v.x * v.x - v.y * v.y;
      const float fs1 = 2.0f * v.x * v.y;
      color = v3add(color, v3scale(rc(12), f1a * fs1));
      color = v3add(color, v3scale(rc(15), f0b * v.y));
      color = v3add(color, v3scale(rc(18), 0.9461747f * z2 - 0.31539157f));
      color = v3add(color, v3scale(rc(21), f0b * v.x));
      color = v3add(color, v3scale(rc(24), f1a * fc1));
      if (deg >= 3) {
        const float f0c = -2.285229f * z2 + 0.4570458f;
        const float f1b = 1.4453057f * v.z;
        const float f2a = -0.5900436f;
        const float fc2 = v.x * fc1 - v.y * fs1;
        const float fs2 = v.x * fs1 + v.y * fc1;
        color = v3add(color, v3scale(rc(27), f2a * fs2));
        color = v3add(color, v3scale(rc(30), f1b * fs1));
        color = v3add(color, v3scale(rc(33), f0c * v.y));
        color = v3add(color, v3scale(rc(36), v.z * (1.8658817f * z2 - 1.119529f)));
        color = v3add(color, v3scale(rc(39), f0c * v.x));
        color = v3add(color, v3scale(rc(42), f1b * fc1));
        color = v3add(color, v3scale(rc(45), f2a * fc2));
      }
    }
  }
  V3 c = {color.x + 0.5f, color.y + 0.5f, color.z + 0.5f};
  c.x = clampf(vs_is_finite(c.x) ? c.x : 0.0f, -100.0f, 100.0f);
  c.y = clampf(vs_is_finite(c.y) ? c.y : 0.0f, -100.0f, 100.0f);
  c.z = clampf(vs_is_finite(c.z) ? c.z : 0.0f, -100.0f, 100.0f);
  return c;
}

// Look-back status word: flag in the high half (1 = block aggregate,
// 2 = inclusive prefix), count in the low half.
__device__ __forceinline__ unsigned long long lb_load(unsigned long long* p) {
  cuda::atomic_ref<unsigned long long, cuda::thread_scope_device> r(*p);
  return r.load(cuda::memory_order_acquire);
}
__device__ __forceinline__ void lb_store(unsigned long long* p, unsigned long long v) {
  cuda::atomic_ref<unsigned long long, cuda::thread_scope_device> r(*p);
  r.store(v, cuda::memory_order_release);
}

__global__ void __launch_bounds__(PROJ_BLOCK, 4) project_kernel(
    Uniforms u, uint32_t n, const float* __restrict__ transforms, const void* __restrict__ sh,
    const float* __restrict__ raw_opac, const float* __restrict__ min_scale, uint32_t* __restrict__ compact_from_global,
    float* __restrict__ opacities, float* __restrict__ max_radius, uint32_t* __restrict__ global_from_compact,
    float* __restrict__ depths, uint32_t* __restrict__ tile_counts, uint2* __restrict__ tile_masks,
    float4* __restrict__ projected,
    unsigned long long* lookback,
    uint32_t* counters /* [0] ticket, [1] visible total, [2] ~min and [3] max of the visible depth bits */,
    unsigned long long* isect_total, uint32_t* err) {
  __shared__ uint32_t s_bid;
  __shared__ uint32_t s_warp_cnt[PROJ_BLOCK / 32];
  __shared__ uint32_t s_block_off;
  __shared__ uint32_t s_total;
  __shared__ unsigned long long s_isect;
  __shared__ uint32_t s_dlo_inv, s_dhi;  // ~min and max of the block's visible depth bits
  const uint32_t tid = threadIdx.x, lane = tid & 31u, warp = tid >> 5;
  if (tid == 0) {
    s_bid = atomicAdd(&counters[0], 1u);  // in-order block ids: look-back only waits on started blocks
    s_isect = 0ull;
    s_dlo_inv = 0u;
    s_dhi = 0u;
  }
  __syncthreads();
  const uint32_t bid = s_bid;
  const uint32_t g = bid * PROJ_BLOCK + tid;

  ProjOut o;
  bool visible = false;
  float t[10];
  if (g < n) {
    const float2* t2 = reinterpret_cast<const float2*>(transforms + (size_t)g * 10);
#pragma unroll
    for (int k = 0; k < 5; ++k) {
      const float2 v = t2[k];
      t[2 * k] = v.x;
      t[2 * k + 1] = v.y;
    }
    visible = project_one(t, raw_opac[g], min_scale, g, u, &o);
    opacities[g] = o.floor_reached ? o.floor_opac : 0.0f;
    max_radius[g] = visible ? o.radius : 0.0f;
  }
  // Block-level ranking of the visible splats; the block's count is published
  // for the look-back at once, and the heavy work below (SH colour, tile
  // counting) runs before this block looks back itself, so by then the blocks
  // before it have usually published theirs.
  const uint32_t ballot = __ballot_sync(0xffffffffu, visible);
  const uint32_t warp_rank = __popc(ballot & ((1u << lane) - 1u));
  if (lane == 0) s_warp_cnt[warp] = __popc(ballot);
  __syncthreads();
  if (tid == 0) {
    uint32_t total = 0;
    for (uint32_t w = 0; w < PROJ_BLOCK / 32; ++w) {
      const uint32_t c = s_warp_cnt[w];
      s_warp_cnt[w] = total;
      total += c;
    }
    s_total = total;
    lb_store(&lookback[bid], ((bid == 0 ? 2ull : 1ull) << 32) | total);
  }
  V3 col = {0.0f, 0.0f, 0.0f};
  if (visible) col = splat_color(sh, u.sh_half != 0, g, u.sh_degree, V3{t[0], t[1], t[2]}, u);
  // Tile counting (kernels/helpers.rs:254-273); large boxes are walked by the
  // whole warp, one splat at a time (project_forward.rs:198-247).
  uint32_t nb = 0;
  if (visible) nb = (o.box.y1 - o.box.y0) * (o.box.x1 - o.box.x0);
  const uint32_t mask = (visible && nb <= BIG_BOX) ? hit_mask_box(o.box, o.xy_x, o.xy_y, o.conic, o.pt) : 0u;
  uint32_t hits = __popc(mask);
  uint32_t pending = __ballot_sync(0xffffffffu, visible && nb > BIG_BOX);
  while (pending) {
    const int leader = __ffs(pending) - 1;
    const float lx = __shfl_sync(0xffffffffu, o.xy_x, leader);
    const float ly = __shfl_sync(0xffffffffu, o.xy_y, leader);
    const S2 lc = {__shfl_sync(0xffffffffu, o.conic.c00, leader), __shfl_sync(0xffffffffu, o.conic.c01, leader),
                   __shfl_sync(0xffffffffu, o.conic.c11, leader)};
    const float lpt = __shfl_sync(0xffffffffu, o.pt, leader);
    const uint32_t lx0 = __shfl_sync(0xffffffffu, o.box.x0, leader);
    const uint32_t ly0 = __shfl_sync(0xffffffffu, o.box.y0, leader);
    const uint32_t lw = __shfl_sync(0xffffffffu, o.box.x1 - o.box.x0, leader);
    const uint32_t ln = __shfl_sync(0xffffffffu, nb, leader);
    uint32_t c = 0;
    for (uint32_t t = lane; t < ln; t += 32) c += tile_hit(t % lw + lx0, t / lw + ly0, lx, ly, lc, lpt) ? 1u : 0u;
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) c += __shfl_xor_sync(0xffffffffu, c, off);
    if ((int)lane == leader) hits = c;
    pending &= pending - 1u;
  }

  unsigned long long hsum = hits;
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) hsum += __shfl_xor_sync(0xffffffffu, hsum, off);
  if (lane == 0 && hsum) atomicAdd(&s_isect, hsum);
  // the depth range of the visible splats sets how many key bits the depth
  // sort needs (depths are positive, so their bits order like the values)
  const uint32_t dbits = visible ? __float_as_uint(o.depth) : 0u;
  const uint32_t whi = __reduce_max_sync(0xffffffffu, dbits);
  const uint32_t wlo_inv = __reduce_max_sync(0xffffffffu, visible ? ~dbits : 0u);
  if (lane == 0 && ballot) {
    atomicMax(&s_dhi, whi);
    atomicMax(&s_dlo_inv, wlo_inv);
  }
  __syncthreads();
  if (warp == 0) {
    const uint32_t total = s_total;
    if (lane == 0 && s_isect) atomicAdd(isect_total, s_isect);
    if (lane == 0 && total) {
      atomicMax(&counters[3], s_dhi);
      atomicMax(&counters[2], s_dlo_inv);
    }
    // Decoupled look-back, a warp at a time: lane l reads the status of block
    // hi - l; the nearest published inclusive prefix ends the walk.  Positions
    // before block 0 read as an inclusive prefix of 0.
    uint32_t exclusive = 0;
    if (bid > 0) {
      int64_t hi = (int64_t)bid - 1;
      uint32_t spins = 0;
      while (true) {
        const int64_t p = hi - (int64_t)lane;
        const unsigned long long s = p >= 0 ? lb_load(&lookback[p]) : (2ull << 32);
        const uint32_t flag = (uint32_t)(s >> 32);
        const uint32_t incl = __ballot_sync(0xffffffffu, flag == 2u);
        const uint32_t pending = __ballot_sync(0xffffffffu, flag == 0u);
        const uint32_t first = incl ? (uint32_t)(__ffs(incl) - 1) : 32u;
        const uint32_t needed = first >= 31u ? 0xffffffffu : ((2u << first) - 1u);
        if (pending & needed) {
          if (++spins > SPIN_LIMIT) {
            if (lane == 0) atomicOr(err, VS_DERR_WAIT);
            break;
          }
          if (spins > 32) __nanosleep(64);
          continue;
        }
        uint32_t part = lane <= first ? (uint32_t)s : 0u;
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) part += __shfl_xor_sync(0xffffffffu, part, off);
        exclusive += part;
        if (first < 32u) break;
        hi -= 32;
      }
      if (lane == 0) lb_store(&lookback[bid], (2ull << 32) | (exclusive + total));
    }
    if (lane == 0) {
      s_block_off = exclusive;
      if (bid == gridDim.x - 1) counters[1] = exclusive + total;
    }
  }
  __syncthreads();
  if (g >= n) return;
  if (!visible) {
    compact_from_global[g] = 0u;
    return;
  }
  const uint32_t c = s_block_off + s_warp_cnt[warp] + warp_rank;
  compact_from_global[g] = c + 1u;
  global_from_compact[c] = g;
  depths[c] = o.depth;
  tile_counts[c] = hits;
  // the emission's input: the hit mask of a small box, or a flag for a large one
  tile_masks[c] = make_uint2(nb <= BIG_BOX ? mask | ((o.box.x1 - o.box.x0) << 16) : 0x80000000u,
                             o.box.x0 | (o.box.y0 << 16));
  float4* row = projected + (size_t)c * PROJ_F4;
  row[0] = make_float4(o.xy_x, o.xy_y, o.conic.c00, o.conic.c01);
  row[1] = make_float4(o.conic.c11, o.opac, col.x, col.y);
  row[2] = make_float4(col.z, __uint_as_float(g), 0.0f, 0.0f);
}

}  // namespace

vs_status launch_project(vs_ctx* ctx, vs_frame* f, const float* transforms, const void* sh, const float* raw_opac,
                         const float* min_scale) {
  const uint32_t n = f->n;
  const uint32_t blocks = n == 0 ? 0 : div_up(n, PROJ_BLOCK);
  VS_TRY(vs_ensure(ctx, f->lookback, (size_t)(blocks + 1) * sizeof(unsigned long long)));
  VS_TRY(vs_ensure(ctx, f->counters, 64));
  VS_CUDA(ctx, cudaMemsetAsync(f->lookback.ptr, 0, (size_t)(blocks + 1) * sizeof(unsigned long long), ctx->stream));
  VS_CUDA(ctx, cudaMemsetAsync(f->counters.ptr, 0, 64, ctx->stream));
  if (blocks == 0) return VS_OK;
  uint32_t* counters = (uint32_t*)f->counters.ptr;
  unsigned long long* isect_total = (unsigned long long*)((char*)f->counters.ptr + 32);
  project_kernel<<<blocks, PROJ_BLOCK, 0, ctx->stream>>>(
      f->u, n, transforms, sh, raw_opac, min_scale, (uint32_t*)f->compact_from_global.ptr, (float*)f->opacities.ptr,
      (float*)f->max_radius.ptr, (uint32_t*)f->global_from_compact.ptr, (float*)f->depths.ptr,
      (uint32_t*)f->tile_counts.ptr, (uint2*)f->tile_masks.ptr, (float4*)f->projected.ptr, (unsigned long long*)f->lookback.ptr, counters,
      isect_total, ctx->d_err); ++ctx->launches;
  return vs_cuda(ctx, cudaGetLastError(), "project_kernel launch");
}
