// Front-to-back alpha compositing, training variant.
//
// Replaces rasterize_kernel with bwd_info (crates/splat-train-render/src/
// kernels/rasterize.rs:109-420): one 256-thread CTA per 16x16 tile, one pixel
// per thread (Morton order inside the tile, helpers.rs:105-128), splats staged
// 256 at a time in shared memory.  Writes RGBA f32, marks contributing splats
// in `visible`, and records per tile one past the last intersection any pixel
// used (the reference shrinks tile_offsets[t].end in place; here it goes to a
// separate array so the binned ranges stay intact).
//
// Per pixel the arithmetic is: sigma = raster_sigma(...) (two fmas),
// alpha = min(0.999, opac * vs_expf(-sigma)), accept when sigma >= 0 and
// alpha >= 1/255, stop when T (1 - alpha) <= 1e-4 (that splat not applied),
// colour += max(c, 0) * alpha T (fma), final = colour + T bg (fma).
// Splats whose exponent exceeds ln(opac / (1/255 - 5e-4)) + 1e-3 cannot pass
// the alpha test, so their exp is skipped (same decisions, fewer SFU ops).
// Each warp (an 8x4 pixel block) also skips every splat whose exponent
// provably exceeds that cut on the whole block (reach_rect), which only drops
// pixels that would fail the exponent test.
#include "vs_internal.cuh"

namespace {

using namespace vs;

constexpr uint32_t RF_THREADS = 256;

__device__ __forceinline__ uint32_t compact_bits(uint32_t v) {
  uint32_t x = v & 0x55555555u;
  x = (x | (x >> 1)) & 0x33333333u;
  x = (x | (x >> 2)) & 0x0F0F0F0Fu;
  x = (x | (x >> 4)) & 0x00FF00FFu;
  x = (x | (x >> 8)) & 0x0000FFFFu;
  return x;
}

// kPacked: the inference pass (the reference's bwd_info = false) -- packed
// RGBA8 output, no visible marks, no used range ends.
template <bool kPacked>
__global__ void __launch_bounds__(RF_THREADS) raster_fwd_kernel(
    uint32_t w, uint32_t h, uint32_t tbw, float bg_r, float bg_g, float bg_b,
    const uint2* __restrict__ ranges, const uint32_t* __restrict__ isect_compact,
    const float4* __restrict__ projected, float4* __restrict__ out_img, float* __restrict__ visible,
    uint32_t* __restrict__ used_end, uint32_t* __restrict__ out_packed) {
  __shared__ float4 s_a[RF_THREADS];  // x, y, 0.5 c00, c01
  __shared__ float4 s_b[RF_THREADS];  // 0.5 c11, opac, max(r, 0), max(g, 0)
  __shared__ float2 s_c[RF_THREADS];  // max(b, 0), sigma cut
  __shared__ float4 s_rc[RF_THREADS];   // culling constants (reach_cut)
  __shared__ uint32_t s_gid[RF_THREADS];
  __shared__ uint32_t s_hit[RF_THREADS];
  __shared__ uint32_t s_done;
  __shared__ uint32_t s_max_used;

  const uint32_t tile = blockIdx.x;
  const uint32_t tid = threadIdx.x, lane = tid & 31u;
  const uint32_t px = (tile % tbw) * TILE + compact_bits(tid);
  const uint32_t py = (tile / tbw) * TILE + compact_bits(tid >> 1);
  // A warp's 32 Morton-ordered pixels form an 8x4 block.
  const float rx0 = (float)((tile % tbw) * TILE + compact_bits(tid & ~31u)) + 0.5f, rx1 = rx0 + 7.0f;
  const float ry0 = (float)((tile / tbw) * TILE + compact_bits((tid & ~31u) >> 1)) + 0.5f, ry1 = ry0 + 3.0f;
  const bool inside = px < w && py < h;
  const uint2 range = ranges[tile];
  const float fx = (float)px + 0.5f, fy = (float)py + 0.5f;
  if (tid == 0) {
    s_done = 0;
    s_max_used = range.x;
  }
  __syncthreads();
  bool done = !inside;
  if (done) atomicAdd(&s_done, 1u);
  float t_acc = 1.0f, r = 0.0f, g = 0.0f, b = 0.0f;
  uint32_t last = range.x;

  for (uint32_t batch = range.x; batch < range.y; batch += RF_THREADS) {
    __syncthreads();  // previous batch's shared reads are finished; s_done is final
    if (s_done >= RF_THREADS) break;
    const uint32_t cnt = min(RF_THREADS, range.y - batch);
    if (tid < cnt) {
      const uint32_t c = isect_compact[batch + tid];
      const float4 a = projected[(size_t)c * PROJ_F4];
      const float4 bb = projected[(size_t)c * PROJ_F4 + 1];
      const float4 cc = projected[(size_t)c * PROJ_F4 + 2];
      s_a[tid] = make_float4(a.x, a.y, 0.5f * a.z, a.w);
      s_b[tid] = make_float4(0.5f * bb.x, bb.y, fmaxf(bb.z, 0.0f), fmaxf(bb.w, 0.0f));
      const float cut = vs_logf(bb.y / ALPHA_EDGE) + 1.0e-3f;
      s_c[tid] = make_float2(fmaxf(cc.x, 0.0f), cut);
      {
        const ReachCut rc = reach_cut(0.5f * a.z, a.w, 0.5f * bb.x, cut);
        s_rc[tid] = make_float4(rc.kx, rc.ky, rc.tcut, 0.0f);
      }
      s_gid[tid] = __float_as_uint(cc.y);
      s_hit[tid] = 0;
    }
    __syncthreads();
    const bool was_done = done;
    // 32 splats at a time, the warp walks only those that can reach its 8x4
    // block (reach_rect: the skipped ones fail the exponent test everywhere).
    for (uint32_t j0 = 0; j0 < cnt; j0 += 32) {
      if (__all_sync(0xffffffffu, done)) break;
      const uint32_t jl = j0 + lane;
      bool near = false;
      if (jl < cnt) {
        const float4 sa = s_a[jl], rc = s_rc[jl];
        near = reach_rect(sa.x, sa.y, sa.z, sa.w, s_b[jl].x, ReachCut{rc.x, rc.y, rc.z}, rx0, rx1, ry0, ry1);
      }
      uint32_t m = __ballot_sync(0xffffffffu, near);
      while (m) {
        const uint32_t j = j0 + __ffs(m) - 1;
        m &= m - 1u;
        if (done) continue;
        const float4 sa = s_a[j];
        const float4 sb = s_b[j];
        const float2 sc = s_c[j];
        const float sigma = raster_sigma(sa.z, sa.w, sb.x, fx - sa.x, fy - sa.y);
        if (sigma > sc.y) continue;
        // vs_expf_core = vs_expf wherever the result is used: only when
        // 0 <= sigma <= cut < 6 is the splat accepted
        const float alpha = fminf(0.999f, sb.y * vs_expf_core(-sigma));
        if (sigma >= 0.0f && alpha >= ALPHA_MIN) {
          const float next_t = t_acc * (1.0f - alpha);
          if (next_t <= 1.0e-4f) {
            done = true;
          } else {
            if (!kPacked) s_hit[j] = 1u;
            const float vis = alpha * t_acc;
            r = fmaf(sb.z, vis, r);
            g = fmaf(sb.w, vis, g);
            b = fmaf(sc.x, vis, b);
            t_acc = next_t;
            last = batch + j + 1;
          }
        }
      }
    }
    if (!was_done && done) atomicAdd(&s_done, 1u);
    __syncthreads();
    if (!kPacked && tid < cnt && s_hit[tid]) visible[s_gid[tid]] = 1.0f;
  }
  const float fr = fmaf(t_acc, bg_r, r), fg = fmaf(t_acc, bg_g, g), fb = fmaf(t_acc, bg_b, b), fa = 1.0f - t_acc;
  if (kPacked) {
    // rasterize.rs:401-409: clamp(255 c, 0, 255) converted toward zero, r in the low byte
    if (inside) {
      const uint32_t cr = (uint32_t)clampf(fr * 255.0f, 0.0f, 255.0f), cg = (uint32_t)clampf(fg * 255.0f, 0.0f, 255.0f);
      const uint32_t cb = (uint32_t)clampf(fb * 255.0f, 0.0f, 255.0f), ca = (uint32_t)clampf(fa * 255.0f, 0.0f, 255.0f);
      out_packed[(size_t)py * w + px] = cr | (cg << 8) | (cb << 16) | (ca << 24);
    }
    return;
  }
  if (inside) out_img[(size_t)py * w + px] = make_float4(fr, fg, fb, fa);
  atomicMax(&s_max_used, last);
  __syncthreads();
  if (tid == 0) used_end[tile] = s_max_used;
}

}  // namespace

vs_status launch_raster_fwd(vs_ctx* ctx, vs_frame* f, float* out_img, float* visible) {
  if (f->n > 0) VS_CUDA(ctx, cudaMemsetAsync(visible, 0, (size_t)f->n * 4, ctx->stream));
  if (f->T == 0) return VS_OK;
  raster_fwd_kernel<false><<<f->T, RF_THREADS, 0, ctx->stream>>>(
      f->u.w, f->u.h, f->u.tbw, f->u.bg[0], f->u.bg[1], f->u.bg[2], (const uint2*)f->tile_ranges.ptr,
      (const uint32_t*)f->isect_compact.ptr, (const float4*)f->projected.ptr, (float4*)out_img, visible,
      (uint32_t*)f->tile_used_end.ptr, nullptr); ++ctx->launches;
  return vs_cuda(ctx, cudaGetLastError(), "raster_fwd launch");
}

vs_status launch_raster_packed(vs_ctx* ctx, vs_frame* f, uint32_t* out_rgba8) {
  if (f->T == 0) return VS_OK;
  raster_fwd_kernel<true><<<f->T, RF_THREADS, 0, ctx->stream>>>(
      f->u.w, f->u.h, f->u.tbw, f->u.bg[0], f->u.bg[1], f->u.bg[2], (const uint2*)f->tile_ranges.ptr,
      (const uint32_t*)f->isect_compact.ptr, (const float4*)f->projected.ptr, nullptr, nullptr, nullptr, out_rgba8);
  ++ctx->launches;
  return vs_cuda(ctx, cudaGetLastError(), "raster_packed launch");
}
