// Binning: depth sort of the visible splats, intersection emission in depth
// order, stable tile sort and per-tile ranges.
//
// Replaces src/render.rs:689-810 of the reference: DepthSort
// (radix_argsort_with_count on the f32 depth bits), scan_sorted_counts_kernel +
// scan_in_place (kernels/map_gaussians.rs:195-269), map_gaussians_to_intersect
// (:21-174), the tile sort and get_tile_offsets (src/get_tile_offset.rs:11-52).
// The resulting order is (tile, depth, compact id) -- a stable sort on the
// 64-bit key tile << 32 | f32_bits(depth) -- done as a depth sort over the V
// visible splats (over the bits in which their depths differ) followed by a
// stable sort over the tile bits only.
#include "vs_internal.cuh"

namespace {

using namespace vs;

constexpr uint32_t BIN_BLOCK = 256;

// The depth-sort input when every visible depth is equal (no key bits, so no
// radix pass writes the order): ids = 0..v-1, keys the depth bits less the
// smallest.  Otherwise the sort's first pass reads the depths itself.
__global__ void depth_keys_kernel(const float* __restrict__ depths, uint32_t v, uint32_t lo, uint32_t* __restrict__ keys,
                                  uint32_t* __restrict__ ids) {
  const uint32_t i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i < v) {
    keys[i] = __float_as_uint(depths[i]) - lo;
    ids[i] = i;
  }
}

// One thread per depth-sorted splat takes its box's hit mask from projection
// (boxes of up to 16 tiles); the warp then writes the contiguous
// output range of its 32 splats together, lane l taking positions p = p0 + l:
// the owning splat is found by a binary search over the lanes' start offsets
// and the entry is the (p - start)-th hit of its mask, so every store
// instruction covers 32 consecutive entries.  Large boxes are walked by the
// whole warp afterwards (map_gaussians.rs:117-173).  Emission stops at the
// splat's counted budget and pads any shortfall with the sentinel tile id T
// (map_gaussians.rs:76-113); no store goes past the projection's intersection
// total `total`, whatever the offsets hold.
__global__ void __launch_bounds__(BIN_BLOCK) emit_kernel(Uniforms u, uint32_t v, const uint32_t* __restrict__ order,
                                                         const uint32_t* __restrict__ cum,
                                                         const uint2* __restrict__ tile_masks,
                                                         const float4* __restrict__ projected,
                                                         uint32_t* __restrict__ tile_keys,
                                                         uint32_t* __restrict__ compact_vals, uint32_t total) {
  const uint32_t i = blockIdx.x * blockDim.x + threadIdx.x;
  const uint32_t lane = threadIdx.x & 31u;
  const bool active = i < v;
  const uint32_t T = u.tbw * u.tbh;
  uint32_t c = 0, start = 0, budget = 0, nb = 0, bw = 0;
  float px = 0.f, py = 0.f, pt = 0.f;
  S2 conic = {0.f, 0.f, 0.f};
  TileBox b = {0, 0, 0, 0};
  uint2 e = make_uint2(0u, 0u);  // small box: hit mask | width << 16; large: bit 31
  if (active) {
    c = order[i];
    start = i ? cum[i - 1] : 0u;
    budget = cum[i] - start;
    e = tile_masks[c];
  }
  const bool big = active && (e.x & 0x80000000u);
  if (big) {
    const float4 r0 = projected[(size_t)c * PROJ_F4];
    const float4 r1 = projected[(size_t)c * PROJ_F4 + 1];
    px = r0.x; py = r0.y;
    conic = {r0.z, r0.w, r1.x};
    pt = vs_logf(r1.y * 255.0f);
    float ex, ey;
    bbox_extent(conic, pt, &ex, &ey);
    b = tile_bbox(px, py, ex, ey, u.tbw, u.tbh);
    bw = b.x1 - b.x0;
    nb = (b.y1 - b.y0) * bw;
  }
  {
    // [s0, s1): the warp's output range; inactive lanes start at s1
    const uint32_t s1 = __reduce_max_sync(0xffffffffu, active ? start + budget : 0u);
    const uint32_t my_start = active ? start : s1;
    const uint32_t s0 = __shfl_sync(0xffffffffu, my_start, 0);
    const uint32_t info0 = e.x, info1 = e.y;
    for (uint32_t p0 = s0; p0 < s1; p0 += 32) {
      const uint32_t p = p0 + lane;
      uint32_t owner = 0, ostart = s0;
#pragma unroll
      for (uint32_t step = 16; step > 0; step >>= 1) {
        const uint32_t cand = owner + step;
        const uint32_t sc = __shfl_sync(0xffffffffu, my_start, cand);
        if (sc <= p) {
          owner = cand;
          ostart = sc;
        }
      }
      const uint32_t oi0 = __shfl_sync(0xffffffffu, info0, owner);
      const uint32_t oi1 = __shfl_sync(0xffffffffu, info1, owner);
      const uint32_t oc = __shfl_sync(0xffffffffu, c, owner);
      if (p < s1 && p < total && !(oi0 & 0x80000000u)) {
        const uint32_t k = p - ostart, m = oi0 & 0xffffu;
        uint32_t key = T;
        if (k < (uint32_t)__popc(m)) {
          const uint32_t bit = __fns(m, 0u, (int)k + 1), obw = (oi0 >> 16) & 0x1fu;
          key = (bit % obw + (oi1 & 0xffffu)) + (bit / obw + (oi1 >> 16)) * u.tbw;
        }
        tile_keys[p] = key;
        compact_vals[p] = oc;
      }
    }
  }
  uint32_t pending = __ballot_sync(0xffffffffu, big);
  while (pending) {
    const int leader = __ffs(pending) - 1;
    const float lx = __shfl_sync(0xffffffffu, px, leader);
    const float ly = __shfl_sync(0xffffffffu, py, leader);
    const S2 lc = {__shfl_sync(0xffffffffu, conic.c00, leader), __shfl_sync(0xffffffffu, conic.c01, leader),
                   __shfl_sync(0xffffffffu, conic.c11, leader)};
    const float lpt = __shfl_sync(0xffffffffu, pt, leader);
    const uint32_t lx0 = __shfl_sync(0xffffffffu, b.x0, leader);
    const uint32_t ly0 = __shfl_sync(0xffffffffu, b.y0, leader);
    const uint32_t lw = __shfl_sync(0xffffffffu, bw, leader);
    const uint32_t ln = __shfl_sync(0xffffffffu, nb, leader);
    const uint32_t lstart = __shfl_sync(0xffffffffu, start, leader);
    const uint32_t lbudget = __shfl_sync(0xffffffffu, budget, leader);
    const uint32_t lc_id = __shfl_sync(0xffffffffu, c, leader);
    uint32_t emitted = 0;
    for (uint32_t t0 = 0; t0 < ln; t0 += 32) {
      const uint32_t t = t0 + lane;
      const uint32_t tx = t % lw + lx0, ty = t / lw + ly0;
      const bool hit = t < ln && tile_hit(tx, ty, lx, ly, lc, lpt);
      const uint32_t mask = __ballot_sync(0xffffffffu, hit);
      const uint32_t slot = emitted + __popc(mask & ((1u << lane) - 1u));
      if (hit && slot < lbudget && lstart + slot < total) {
        tile_keys[lstart + slot] = tx + ty * u.tbw;
        compact_vals[lstart + slot] = lc_id;
      }
      emitted += __popc(mask);
    }
    for (uint32_t p = min(emitted, lbudget) + lane; p < lbudget && lstart + p < total; p += 32) {
      tile_keys[lstart + p] = T;
      compact_vals[lstart + p] = lc_id;
    }
    pending &= pending - 1u;
  }
}

// [start, end) of every tile present in the sorted list; absent tiles stay
// [0, 0) from the preceding memset.  Sentinel ids (>= T) are skipped.
__global__ void tile_ranges_kernel(const uint32_t* __restrict__ tiles_sorted, uint32_t count, uint32_t T,
                                   uint2* __restrict__ ranges) {
  // four consecutive entries per thread (one 16-byte load) and their two
  // neighbours; ~0u stands for "no entry" before the first and after the last
  const uint32_t q = blockIdx.x * blockDim.x + threadIdx.x;
  const uint32_t i0 = q * 4u;
  if (i0 >= count) return;
  uint32_t t[6];
  t[0] = i0 ? tiles_sorted[i0 - 1] : ~0u;
  if (i0 + 4u <= count) {
    const uint4 v4 = reinterpret_cast<const uint4*>(tiles_sorted)[q];
    t[1] = v4.x, t[2] = v4.y, t[3] = v4.z, t[4] = v4.w;
  } else {
#pragma unroll
    for (uint32_t k = 0; k < 4; ++k) t[1 + k] = i0 + k < count ? tiles_sorted[i0 + k] : ~0u;
  }
  t[5] = i0 + 4u < count ? tiles_sorted[i0 + 4u] : ~0u;
#pragma unroll
  for (uint32_t k = 0; k < 4; ++k) {
    const uint32_t i = i0 + k, cur = t[1 + k];
    if (i >= count || cur >= T) continue;
    if (t[k] != cur) ranges[cur].x = i;
    if (t[k + 2] != cur) ranges[cur].y = i + 1;
  }
}

}  // namespace

vs_status launch_bin(vs_ctx* ctx, vs_frame* f) {
  const uint32_t v = f->v, T = f->T;
  VS_TRY(vs_ensure(ctx, f->tile_ranges, (size_t)T * 8));
  VS_TRY(vs_ensure(ctx, f->tile_used_end, (size_t)T * 4));
  VS_CUDA(ctx, cudaMemsetAsync(f->tile_ranges.ptr, 0, (size_t)T * 8, ctx->stream));
  VS_TRY(vs_ensure(ctx, f->depth_order, (size_t)(v + 1) * 4));
  if (v == 0) {
    f->I = 0;
    return VS_OK;
  }
  // depth sort: keys = depth bits, values = compact ids
  const uint64_t I = f->I;
  const size_t scratch = (size_t)std::max<uint64_t>(v, I) * 4;
  VS_TRY(vs_ensure(ctx, ctx->sort_keys, scratch * 2));
  VS_TRY(vs_ensure(ctx, ctx->sort_vals, scratch * 2));
  uint32_t* k0 = (uint32_t*)ctx->sort_keys.ptr;
  uint32_t* k1 = k0 + scratch / 4;
  uint32_t* v0 = (uint32_t*)ctx->sort_vals.ptr;
  uint32_t* v1 = v0 + scratch / 4;
  const uint32_t blocks_v = div_up(v, BIN_BLOCK);
  if (f->depth_hi < f->depth_lo)
    return vs_fail(ctx, VS_ERR_CUDA, "render_bin: depth range [%08x, %08x] of %u visible splats", f->depth_lo,
                   f->depth_hi, v);
  const uint32_t span = f->depth_hi - f->depth_lo;
  const uint32_t depth_bits = span ? 32u - (uint32_t)__builtin_clz(span) : 0u;
  uint32_t* order = (uint32_t*)f->depth_order.ptr;
  const uint32_t* tile_counts = (const uint32_t*)f->tile_counts.ptr;
  uint32_t* cum;  // the tile counts in depth order, then their inclusive scan: the emission offsets
  if (depth_bits == 0) {
    // every depth equal: the depth order is the compact order
    depth_keys_kernel<<<blocks_v, BIN_BLOCK, 0, ctx->stream>>>((const float*)f->depths.ptr, v, f->depth_lo, k0, order); ++ctx->launches;
    cum = k1;
    VS_TRY(scan_gather_inclusive_u32(ctx, cum, tile_counts, order, v));
  } else {
    // The first pass reads the depth bits less the smallest (the same order in
    // fewer key bits) with the compact ids as values; the last pass writes
    // the ids into depth_order and, beside each, its tile count into v0.  The
    // buffer pairs are chosen so that the last pass writes (k0, depth_order).
    const bool odd = radix_sort_passes(depth_bits) & 1u;
    VS_TRY(radix_sort_from(ctx, (const uint32_t*)f->depths.ptr, nullptr, f->depth_lo, odd ? k0 : k1,
                           odd ? order : v1, odd ? k1 : k0, odd ? v1 : order, v, depth_bits, tile_counts, v0));
    cum = v0;
    VS_TRY(scan_inclusive_u32(ctx, cum, v, nullptr));
  }
  bool alt = false;
  VS_TRY(vs_ensure(ctx, f->isect_tile, (size_t)(I + 1) * 4));
  VS_TRY(vs_ensure(ctx, f->isect_compact, (size_t)(I + 1) * 4));
  if (I == 0) return VS_OK;
  // emit straight into the frame's buffers, sort with the scratch as ping-pong
  uint32_t* tkeys = (uint32_t*)f->isect_tile.ptr;
  uint32_t* tvals = (uint32_t*)f->isect_compact.ptr;
  emit_kernel<<<blocks_v, BIN_BLOCK, 0, ctx->stream>>>(f->u, v, (const uint32_t*)f->depth_order.ptr, cum,
                                                        (const uint2*)f->tile_masks.ptr, (const float4*)f->projected.ptr,
                                                        tkeys, tvals, (uint32_t)I); ++ctx->launches;
  VS_CUDA(ctx, cudaGetLastError());
  const uint32_t tile_bits = 32u - (uint32_t)__builtin_clz(T | 1u);
  uint32_t* sk = (uint32_t*)ctx->sort_keys.ptr;
  uint32_t* sv = (uint32_t*)ctx->sort_vals.ptr;
  VS_TRY(radix_sort_pairs(ctx, tkeys, tvals, sk, sv, (uint32_t)I, tile_bits, &alt));
  if (alt) {
    VS_CUDA(ctx, cudaMemcpyAsync(tkeys, sk, (size_t)I * 4, cudaMemcpyDeviceToDevice, ctx->stream));
    VS_CUDA(ctx, cudaMemcpyAsync(tvals, sv, (size_t)I * 4, cudaMemcpyDeviceToDevice, ctx->stream));
  }
  tile_ranges_kernel<<<div_up(div_up((uint32_t)I, 4u), 256), 256, 0, ctx->stream>>>(tkeys, (uint32_t)I, T,
                                                                        (uint2*)f->tile_ranges.ptr); ++ctx->launches;
  return vs_cuda(ctx, cudaGetLastError(), "bin launch");
}
