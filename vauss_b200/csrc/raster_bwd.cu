// Rasterizer backward: per-pixel front-to-back replay with register-resident
// pixel state.
//
// Replaces rasterize_backwards_planes_kernel (crates/splat-train-render/src/
// bwd/kernels/rasterize_backwards_planes.rs:112-682, gaussian branch):
// one 128-thread CTA per tile, each warp an 8x8 quadrant, two pixels per
// thread, splats staged 128 at a time in shared memory (one per thread; larger
// batches halve the barriers and partial-buffer work per splat each time they
// double).  A warp walks only the splats that can reach its quadrant
// (reach_rect).  Per splat, each thread sums its pixels' gradients, a 12-shuffle butterfly
// reduce-scatter leaves one component per lane pair, the four warps' partials
// are added in shared memory, and one atomic add per non-zero (tile, splat,
// component) lands in v_combined [V,10] = [xy(2), conic(3), rgb(3), alpha,
// refine].
//
// The replay evaluates exactly the forward's exponent, alpha and transmittance
// sequence (raster_sigma, vs_expf, the same comparisons), so every
// accept/terminate decision matches the forward pass bit for bit.  The
// gradient sums, whose order already differs from the oracle's (shuffles and
// atomics), fuse each term's last multiply into the accumulation.
#include "vs_internal.cuh"

namespace {

using namespace vs;

constexpr uint32_t RB_THREADS = 128;
constexpr uint32_t RB_WARPS = RB_THREADS / 32;
constexpr uint32_t RB_BATCH = 128;
constexpr uint32_t NG = 10;

__device__ __forceinline__ float sqrt_approx(float x) {
  float y;
  asm("sqrt.approx.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// The hardware reciprocal (about 1 ulp): it only scales gradient terms, whose
// sums already run in another order than the oracle's, never a coverage or
// termination decision.
__device__ __forceinline__ float rcp_approx(float x) {
  float y;
  asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// Butterfly reduce-scatter of the NG = 10 gradient components over a warp in
// 12 shuffles (groups of 5 | 3+2 | 2+1 | 1+1 | pair sum).  Afterwards the even
// lane l holds the warp sum of component reduce10_comp(l) (or nothing, -1).
__device__ __forceinline__ float reduce10(float v[NG], uint32_t lane) {
  {
    const bool hi = lane & 16u;
#pragma unroll
    for (int i = 0; i < 5; ++i) {
      const float keep = hi ? v[i + 5] : v[i];
      const float send = hi ? v[i] : v[i + 5];
      v[i] = keep + __shfl_xor_sync(0xffffffffu, send, 16);
    }
  }
  {
    const bool hi = lane & 8u;
#pragma unroll
    for (int i = 0; i < 3; ++i) {
      const float up = i + 3 < 5 ? v[i + 3] : 0.0f;
      const float keep = hi ? up : v[i];
      const float send = hi ? v[i] : up;
      v[i] = keep + __shfl_xor_sync(0xffffffffu, send, 8);
    }
  }
  {
    const bool hi = lane & 4u;
#pragma unroll
    for (int i = 0; i < 2; ++i) {
      const float up = i + 2 < 3 ? v[i + 2] : 0.0f;
      const float keep = hi ? up : v[i];
      const float send = hi ? v[i] : up;
      v[i] = keep + __shfl_xor_sync(0xffffffffu, send, 4);
    }
  }
  {
    const bool hi = lane & 2u;
    const float keep = hi ? v[1] : v[0];
    const float send = hi ? v[0] : v[1];
    v[0] = keep + __shfl_xor_sync(0xffffffffu, send, 2);
  }
  return v[0] + __shfl_xor_sync(0xffffffffu, v[0], 1);
}

// Component left on lane `lane` by reduce10: 5*b4 + 3*b3 + (2*b2 + b1), valid
// while the offset 2*b2 + b1 is inside its group (3 wide for b3 = 0, else 2).
__host__ __device__ constexpr int reduce10_comp(uint32_t lane) {
  return (2u * ((lane >> 2) & 1u) + ((lane >> 1) & 1u)) >= (((lane >> 3) & 1u) ? 2u : 3u)
             ? -1
             : (int)(5u * ((lane >> 4) & 1u) + 3u * ((lane >> 3) & 1u) + 2u * ((lane >> 2) & 1u) +
                     ((lane >> 1) & 1u));
}

__global__ void __launch_bounds__(RB_THREADS) raster_bwd_kernel(
    uint32_t w, uint32_t h, uint32_t tbw, float bg_r, float bg_g, float bg_b, const uint2* __restrict__ ranges,
    const uint32_t* __restrict__ used_end, const uint32_t* __restrict__ isect_compact,
    const float4* __restrict__ projected, const float4* __restrict__ out_img, const float4* __restrict__ v_out,
    float* __restrict__ v_combined) {
  __shared__ float4 s_a[RB_BATCH];    // x, y, 0.5 c00, c01
  __shared__ float4 s_b[RB_BATCH];    // 0.5 c11, opac, r, g
  __shared__ float2 s_c[RB_BATCH];    // b, sigma cut
  __shared__ float4 s_rc[RB_BATCH];   // culling constants (reach_cut)
  __shared__ uint32_t s_cid[RB_BATCH];
  __shared__ __align__(16) float s_part[RB_WARPS][RB_BATCH][NG];

  const uint32_t tile = blockIdx.x;
  const uint32_t tid = threadIdx.x, lane = tid & 31u, warp = tid >> 5;
  // Warp w owns the 8x8 quadrant (w & 1, w >> 1) of the tile; lane l its
  // pixels (l & 7, l >> 3) and (l & 7, (l >> 3) + 4).
  const uint32_t qx = (tile % tbw) * TILE + (warp & 1u) * 8u, qy = (tile / tbw) * TILE + (warp >> 1) * 8u;
  const uint32_t px = qx + (lane & 7u);
  const float rx0 = (float)qx + 0.5f, rx1 = rx0 + 7.0f, ry0 = (float)qy + 0.5f, ry1 = ry0 + 7.0f;
  const float fx = (float)px + 0.5f;
  const float img_w = (float)w, img_h = (float)h;
  const int comp = reduce10_comp(lane);

  float sr[2], sg[2], sb[2], st[2], vr[2], vg[2], vb[2], vt[2], rs[2], fy[2];
#pragma unroll
  for (int k = 0; k < 2; ++k) {
    const uint32_t py = qy + (lane >> 3) + 4u * k;
    fy[k] = (float)py + 0.5f;
    sr[k] = sg[k] = sb[k] = st[k] = vr[k] = vg[k] = vb[k] = vt[k] = rs[k] = 0.0f;
    if (px < w && py < h) {
      const size_t p = (size_t)py * w + px;
      const float4 o = out_img[p];
      const float4 vo = v_out[p];
      const float t_final = 1.0f - o.w;
      sr[k] = o.x - t_final * bg_r;
      sg[k] = o.y - t_final * bg_g;
      sb[k] = o.z - t_final * bg_b;
      st[k] = 1.0f;
      vr[k] = vo.x;
      vg[k] = vo.y;
      vb[k] = vo.z;
      vt[k] = (vo.w - (bg_r * vo.x + bg_g * vo.y + bg_b * vo.z)) * t_final;
      rs[k] = 1.0f / fmaxf(o.w, 1.0e-5f);
    }
  }

  const uint32_t lo = ranges[tile].x, hi = used_end[tile];
  for (uint32_t batch = lo; batch < hi; batch += RB_BATCH) {
    const uint32_t cnt = min(RB_BATCH, hi - batch);
    {
      float4* z = reinterpret_cast<float4*>(&s_part[0][0][0]);
      for (uint32_t i = tid; i < RB_WARPS * RB_BATCH * NG / 4; i += RB_THREADS) z[i] = make_float4(0.f, 0.f, 0.f, 0.f);
    }
    if (tid < cnt) {
      const uint32_t c = isect_compact[batch + tid];
      const float4 a = projected[(size_t)c * PROJ_F4];
      const float4 bb = projected[(size_t)c * PROJ_F4 + 1];
      const float4 cc = projected[(size_t)c * PROJ_F4 + 2];
      const float cut = vs_logf(bb.y / ALPHA_EDGE) + 1.0e-3f;
      s_a[tid] = make_float4(a.x, a.y, 0.5f * a.z, a.w);
      s_b[tid] = make_float4(0.5f * bb.x, bb.y, bb.z, bb.w);
      s_c[tid] = make_float2(cc.x, cut);
      {
        const ReachCut rc = reach_cut(0.5f * a.z, a.w, 0.5f * bb.x, cut);
        s_rc[tid] = make_float4(rc.kx, rc.ky, rc.tcut, 0.0f);
      }
      s_cid[tid] = c;
    }
    __syncthreads();
    // The warp walks only the splats that can reach its quadrant, testing 32
    // staged splats at a time (a lane each).
    for (uint32_t half = 0; half < RB_BATCH / 32u; ++half) {
      const uint32_t sl = half * 32u + lane;
      bool near = false;
      if (sl < cnt) {
        const float4 sa = s_a[sl], rc = s_rc[sl];
        near = reach_rect(sa.x, sa.y, sa.z, sa.w, s_b[sl].x, ReachCut{rc.x, rc.y, rc.z}, rx0, rx1, ry0, ry1);
      }
      uint32_t m = __ballot_sync(0xffffffffu, near);
      while (m) {
        const uint32_t t = half * 32u + __ffs(m) - 1;
        m &= m - 1u;
        const float4 a = s_a[t];
        const float4 bb = s_b[t];
        const float2 cc = s_c[t];
        const float h00 = a.z, c01 = a.w, h11 = bb.x, opac = bb.y;
        const float c00 = 2.0f * h00, c11 = 2.0f * h11;
        const float cr = fmaxf(bb.z, 0.0f), cg = fmaxf(bb.w, 0.0f), cb = fmaxf(cc.x, 0.0f);
        const float dx = a.x - fx;
        float g[NG];
  #pragma unroll
        for (int i = 0; i < (int)NG; ++i) g[i] = 0.0f;
        bool contributes = false;
  #pragma unroll
        for (int k = 0; k < 2; ++k) {
          const float dy = a.y - fy[k];
          // coverage decisions: the forward's exact arithmetic
          const float sigma = raster_sigma(h00, c01, h11, dx, dy);
          if (!(st[k] > 1.0e-4f && sigma <= cc.y)) continue;
          const float gauss = vs_expf_core(-sigma);  // = vs_expf: used only for 0 <= sigma <= cut < 6
          const float alpha = fminf(0.999f, opac * gauss);
          if (!(sigma >= 0.0f && alpha >= ALPHA_MIN)) continue;
          const float next_t = st[k] * (1.0f - alpha);
          if (next_t <= 1.0e-4f) {
            st[k] = 0.0f;
            continue;
          }
          contributes = true;
          // gradients: the oracle's per-term float steps (the same fmas), each
          // term's last product fused into its accumulation
          const float vis = alpha * st[k];
          if (bb.z >= 0.0f) g[5] = fmaf(vis, vr[k], g[5]);
          if (bb.w >= 0.0f) g[6] = fmaf(vis, vg[k], g[6]);
          if (cc.x >= 0.0f) g[7] = fmaf(vis, vb[k], g[7]);
          const float ra = rcp_approx(1.0f - alpha);  // 1 - alpha in [1e-3, 1]
          const float dot =
              fmaf(fmaf(st[k], cr, -sr[k]), vr[k], fmaf(fmaf(st[k], cg, -sg[k]), vg[k], fmaf(st[k], cb, -sb[k]) * vb[k])) * ra;
          const float v_alpha = fmaf(vt[k], ra, dot);
          const float v_sigma = -alpha * v_alpha;
          const float vxx = v_sigma * fmaf(c00, dx, c01 * dy);
          const float vxy = v_sigma * fmaf(c01, dx, c11 * dy);
          if (opac * gauss <= 0.999f) {
            const float hv = 0.5f * v_sigma;
            g[2] = fmaf(hv * dx, dx, g[2]);
            g[3] = fmaf(v_sigma * dx, dy, g[3]);
            g[4] = fmaf(hv * dy, dy, g[4]);
            g[0] += vxx;
            g[1] += vxy;
            g[8] = fmaf(v_alpha, gauss, g[8]);
            const float ax = vxx * img_w, ay = vxy * img_h;
            // the refine weight is a densification statistic: the hardware
            // square root (a few ulp) is far inside its tolerance
            g[9] = fmaf(sqrt_approx(fmaf(ax, ax, ay * ay)), rs[k], g[9]);
          }
          sr[k] = fmaf(-vis, cr, sr[k]);
          sg[k] = fmaf(-vis, cg, sg[k]);
          sb[k] = fmaf(-vis, cb, sb[k]);
          st[k] = next_t;
        }
        if (__any_sync(0xffffffffu, contributes)) {
          const float sum = reduce10(g, lane);
          if ((lane & 1u) == 0 && comp >= 0) s_part[warp][t][comp] = sum;
        }
      }
    }
    __syncthreads();
    for (uint32_t idx = tid; idx < cnt * NG; idx += RB_THREADS) {
      const uint32_t s = idx / NG, c = idx % NG;
      float sum = 0.0f;
#pragma unroll
      for (uint32_t ww = 0; ww < RB_WARPS; ++ww) sum += s_part[ww][s][c];
      if (sum != 0.0f) atomicAdd(&v_combined[(size_t)s_cid[s] * NG + c], sum);
    }
    __syncthreads();
  }
}

}  // namespace

vs_status launch_raster_bwd(vs_ctx* ctx, vs_frame* f, const float* out_img, const float* v_out, float* v_combined) {
  VS_CUDA(ctx, cudaMemsetAsync(v_combined, 0, (size_t)f->v * NG * 4, ctx->stream));
  if (f->T == 0 || f->I == 0) return VS_OK;
  raster_bwd_kernel<<<f->T, RB_THREADS, 0, ctx->stream>>>(
      f->u.w, f->u.h, f->u.tbw, f->u.bg[0], f->u.bg[1], f->u.bg[2], (const uint2*)f->tile_ranges.ptr,
      (const uint32_t*)f->tile_used_end.ptr, (const uint32_t*)f->isect_compact.ptr, (const float4*)f->projected.ptr,
      (const float4*)out_img, (const float4*)v_out, v_combined); ++ctx->launches;
  return vs_cuda(ctx, cudaGetLastError(), "raster_bwd launch");
}
