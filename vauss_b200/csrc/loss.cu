// Fused L1 + SSIM image loss: forward partial sums and d(loss)/d(pred) in one
// kernel.
//
// The reference runs two launches (crates/splat-train-loss/src/lib.rs:
// image_loss_forward_kernel :238-469 storing nine per-pixel SSIM coefficient
// maps, then image_loss_backward_coeffs_kernel :821-1028 blurring them).  Since
// d(total)/d(partials) is a constant in training, the backward needs nothing
// from the forward but those coefficients, so one CTA per 16x16 tile and
// channel recomputes them over a 5-pixel halo instead of storing 36 B/pixel:
//
//   pred/gt over the tile + 10-pixel halo (zero outside the image)
//   -> horizontal 11-tap blur of (x, x^2, y, y^2, xy)      [36 rows x 26 cols]
//   -> vertical blur, SSIM, per-pixel coefficients * chain  [26 x 26]
//   -> horizontal blur of the three coefficient products    [26 x 16]
//   -> vertical blur at the tile: dL/dpred                  [16 x 16]
//
// Every blur sums in the reference's order (taps d = 1..5 as (left + right) *
// w[5-d], then the centre), so the values equal the two-pass computation bit
// for bit.  The tile's loss sum uses the reference's shared-memory tree
// (lib.rs:108-123).
#include "vs_internal.cuh"

namespace {

using namespace vs;

constexpr int LB = 16;          // tile
constexpr int HALO = 5;
constexpr int R0 = LB + 4 * HALO;  // 36: pred/gt footprint
constexpr int R1 = LB + 2 * HALO;  // 26: coefficient footprint
constexpr int LT = LB * LB;

__constant__ float c_taps[11];

__device__ __forceinline__ float gtap(int i) { return c_taps[i]; }

__global__ void __launch_bounds__(LT) loss_kernel(uint32_t h, uint32_t w, const float* __restrict__ pred,
                                                  const uint32_t* __restrict__ gt, float l1_w, float ssim_w,
                                                  float rgb_weight, float* __restrict__ partials,
                                                  float* __restrict__ dl_dpred) {
  __shared__ float s_x[R0][R0];
  __shared__ float s_y[R0][R0];
  __shared__ float s_h1[5][R0][R1];
  __shared__ float s_cm[3][R1][R1];
  __shared__ float s_h2[3][R1][LB];
  __shared__ float s_red[LT];

  const int c = blockIdx.z;
  const int tid = threadIdx.x;
  const int x0 = blockIdx.x * LB, y0 = blockIdx.y * LB;
  const int W = (int)w, H = (int)h;

  // 1. load pred/gt channel over tile +- 10
  for (int i = tid; i < R0 * R0; i += LT) {
    const int ly = i / R0, lx = i % R0;
    const int gy = y0 - 2 * HALO + ly, gx = x0 - 2 * HALO + lx;
    float xv = 0.0f, yv = 0.0f;
    if (gy >= 0 && gy < H && gx >= 0 && gx < W) {
      const size_t p = (size_t)gy * w + gx;
      xv = pred[p * 4 + c];
      yv = (float)((gt[p] >> (c * 8)) & 0xffu) * (1.0f / 255.0f);
    }
    s_x[ly][lx] = xv;
    s_y[ly][lx] = yv;
  }
  __syncthreads();

  // 2. horizontal blur of the five moments: rows 0..35, columns tile +- 5
  for (int i = tid; i < R0 * R1; i += LT) {
    const int ly = i / R1, lc = i % R1;
    const int lx = lc + HALO;  // column in s_x
    float sx = 0.f, sx2 = 0.f, sy = 0.f, sy2 = 0.f, sxy = 0.f;
#pragma unroll
    for (int d = 1; d < 6; ++d) {
      const float wd = gtap(5 - d);
      const float xl = s_x[ly][lx - d], xr = s_x[ly][lx + d];
      const float yl = s_y[ly][lx - d], yr = s_y[ly][lx + d];
      sx += (xl + xr) * wd;
      sx2 += (xl * xl + xr * xr) * wd;
      sy += (yl + yr) * wd;
      sy2 += (yl * yl + yr * yr) * wd;
      sxy += (xl * yl + xr * yr) * wd;
    }
    const float xc = s_x[ly][lx], yc = s_y[ly][lx], wc = gtap(5);
    sx += xc * wc;
    sx2 += xc * xc * wc;
    sy += yc * wc;
    sy2 += yc * yc * wc;
    sxy += xc * yc * wc;
    s_h1[0][ly][lc] = sx;
    s_h1[1][ly][lc] = sx2;
    s_h1[2][ly][lc] = sy;
    s_h1[3][ly][lc] = sy2;
    s_h1[4][ly][lc] = sxy;
  }
  __syncthreads();

  // 3. vertical blur -> SSIM coefficients (x chain) over tile +- 5; the tile's
  //    own pixels also produce the loss value.
  const float C1 = 0.01f * 0.01f, C2 = 0.03f * 0.03f;
  float my_loss = 0.0f;
  for (int i = tid; i < R1 * R1; i += LT) {
    const int ry = i / R1, rx = i % R1;
    const int gy = y0 - HALO + ry, gx = x0 - HALO + rx;
    const bool in_img = gy >= 0 && gy < H && gx >= 0 && gx < W;
    float c0 = 0.f, c1 = 0.f, c2 = 0.f;
    if (in_img) {
      const int ly = ry + HALO;  // row in s_h1
      float o[5] = {0.f, 0.f, 0.f, 0.f, 0.f};
#pragma unroll
      for (int d = 1; d < 6; ++d) {
        const float wd = gtap(5 - d);
#pragma unroll
        for (int k = 0; k < 5; ++k) o[k] += (s_h1[k][ly - d][rx] + s_h1[k][ly + d][rx]) * wd;
      }
#pragma unroll
      for (int k = 0; k < 5; ++k) o[k] += s_h1[k][ly][rx] * gtap(5);
      const float mu1 = o[0], mu2 = o[2];
      const float mu1_sq = mu1 * mu1, mu2_sq = mu2 * mu2;
      const float s1 = fmaxf(0.0f, o[1] - mu1_sq), s2 = fmaxf(0.0f, o[3] - mu2_sq);
      const float s12 = o[4] - mu1 * mu2;
      const float a = mu1_sq + mu2_sq + C1, b = s1 + s2 + C2;
      const float ct = 2.0f * mu1 * mu2 + C1, dt = 2.0f * s12 + C2;
      const float inv_b = 1.0f / b, inv_ab = 1.0f / (a * b);
      const float cd = ct * dt * inv_ab;
      const bool cl = cd < -1.0f || cd > 1.0f;
      c0 = (cl ? 0.0f : 2.0f * inv_ab * (mu2 * (dt - ct) - mu1 * cd * (b - a))) * rgb_weight;
      c1 = (cl ? 0.0f : -cd * inv_b) * rgb_weight;
      c2 = (cl ? 0.0f : 2.0f * ct * inv_ab) * rgb_weight;
      if (ry >= HALO && ry < HALO + LB && rx >= HALO && rx < HALO + LB) {
        const float raw = (ct * dt) / (a * b);
        const float val = clampf(raw, -1.0f, 1.0f);
        const float p1 = s_x[ry + HALO][rx + HALO], p2 = s_y[ry + HALO][rx + HALO];
        my_loss = l1_w * fabsf(p1 - p2) + ssim_w * val;
        s_red[(ry - HALO) * LB + (rx - HALO)] = my_loss;
      }
    } else if (ry >= HALO && ry < HALO + LB && rx >= HALO && rx < HALO + LB) {
      s_red[(ry - HALO) * LB + (rx - HALO)] = 0.0f;
    }
    s_cm[0][ry][rx] = c0;
    s_cm[1][ry][rx] = c1;
    s_cm[2][ry][rx] = c2;
  }
  __syncthreads();

  // tile loss: tree sum in the reference's order
  for (int stride = LT / 2; stride > 0; stride >>= 1) {
    if (tid < stride) s_red[tid] += s_red[tid + stride];
    __syncthreads();
  }
  if (tid == 0 && partials) {
    const uint32_t tiles = gridDim.x * gridDim.y;
    partials[(size_t)c * tiles + blockIdx.y * gridDim.x + blockIdx.x] = s_red[0] * rgb_weight;
  }
  if (!dl_dpred) return;

  // 4. horizontal blur of the coefficient products: rows tile +- 5, tile columns
  for (int i = tid; i < R1 * LB; i += LT) {
    const int ry = i / LB, tx = i % LB;
    const int rx = tx + HALO;
    float a0 = 0.f, a1 = 0.f, a2 = 0.f;
#pragma unroll
    for (int d = 1; d < 6; ++d) {
      const float wd = gtap(5 - d);
      a0 += (s_cm[0][ry][rx - d] + s_cm[0][ry][rx + d]) * wd;
      a1 += (s_cm[1][ry][rx - d] + s_cm[1][ry][rx + d]) * wd;
      a2 += (s_cm[2][ry][rx - d] + s_cm[2][ry][rx + d]) * wd;
    }
    const float wc = gtap(5);
    a0 += s_cm[0][ry][rx] * wc;
    a1 += s_cm[1][ry][rx] * wc;
    a2 += s_cm[2][ry][rx] * wc;
    s_h2[0][ry][tx] = a0;
    s_h2[1][ry][tx] = a1;
    s_h2[2][ry][tx] = a2;
  }
  __syncthreads();

  // 5. vertical blur at the tile pixels -> dL/dpred
  {
    const int ty = tid / LB, tx = tid % LB;
    const int gy = y0 + ty, gx = x0 + tx;
    if (gy < H && gx < W) {
      const int ry = ty + HALO;
      float s[3] = {0.f, 0.f, 0.f};
#pragma unroll
      for (int d = 1; d < 6; ++d) {
        const float wd = gtap(5 - d);
#pragma unroll
        for (int k = 0; k < 3; ++k) s[k] += (s_h2[k][ry - d][tx] + s_h2[k][ry + d][tx]) * wd;
      }
#pragma unroll
      for (int k = 0; k < 3; ++k) s[k] += s_h2[k][ry][tx] * gtap(5);
      const float p1 = s_x[ty + 2 * HALO][tx + 2 * HALO], g = s_y[ty + 2 * HALO][tx + 2 * HALO];
      const float ssim_grad = s[0] + (2.0f * p1) * s[1] + g * s[2];
      const float diff = p1 - g;
      const float sign = diff > 0.0f ? 1.0f : (diff < 0.0f ? -1.0f : 0.0f);
      const size_t p = (size_t)gy * w + gx;
      dl_dpred[p * 4 + c] = ssim_w * ssim_grad + l1_w * sign * rgb_weight;
      if (c == 0) dl_dpred[p * 4 + 3] = 0.0f;
    }
  }
}

// Deterministic total of the partials (fixed order: per-thread strided sums,
// then a tree).
__global__ void __launch_bounds__(256) loss_total_kernel(const float* __restrict__ partials, uint32_t n,
                                                         float* __restrict__ out) {
  __shared__ float s[256];
  float acc = 0.0f;
  for (uint32_t i = threadIdx.x; i < n; i += 256) acc += partials[i];
  s[threadIdx.x] = acc;
  __syncthreads();
  for (int stride = 128; stride > 0; stride >>= 1) {
    if ((int)threadIdx.x < stride) s[threadIdx.x] += s[threadIdx.x + stride];
    __syncthreads();
  }
  if (threadIdx.x == 0) *out = s[0];
}

}  // namespace

vs_status launch_loss(vs_ctx* ctx, uint32_t h, uint32_t w, const float* pred, const uint32_t* gt, float l1_w,
                      float ssim_w, float* partials, float* loss_dev, float* dl_dpred) {
  if (!ctx->taps_ready) {
    // 11-tap Gaussian window, sigma 1.5, normalised (lib.rs:50-63), computed in
    // double and rounded once.
    float taps[11];
    double t[11], s = 0.0;
    for (int i = 0; i < 11; ++i) {
      const double x = (double)i - 5.0;
      t[i] = exp(-x * x / (2.0 * 1.5 * 1.5));
      s += t[i];
    }
    for (int i = 0; i < 11; ++i) taps[i] = (float)(t[i] / s);
    VS_CUDA(ctx, cudaMemcpyToSymbol(c_taps, taps, sizeof(taps)));
    ctx->taps_ready = true;  // __constant__ memory is per device; one ctx per device
  }
  if (h == 0 || w == 0) return vs_fail(ctx, VS_ERR_INVALID, "loss: empty image");
  const uint32_t tx = div_up(w, 16), ty = div_up(h, 16);
  float* parts = partials;
  if (!parts && loss_dev) {
    VS_TRY(vs_ensure(ctx, ctx->misc, (size_t)3 * tx * ty * 4));
    parts = (float*)ctx->misc.ptr;
  }
  const float rgb_weight = 1.0f / (3.0f * (float)(h * w));
  dim3 grid(tx, ty, 3);
  loss_kernel<<<grid, LT, 0, ctx->stream>>>(h, w, pred, gt, l1_w, ssim_w, rgb_weight, parts, dl_dpred); ++ctx->launches;
  VS_CUDA(ctx, cudaGetLastError());
  if (loss_dev) {
    loss_total_kernel<<<1, 256, 0, ctx->stream>>>(parts, 3 * tx * ty, loss_dev);
    ++ctx->launches;
  }
  return vs_cuda(ctx, cudaGetLastError(), "loss launch");
}
