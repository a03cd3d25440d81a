// Fused L1 + SSIM image loss: forward partial sums and d(loss)/d(pred) in one
// kernel.
//
// The reference runs two launches (crates/splat-train-loss/src/lib.rs:
// image_loss_forward_kernel :238-469 storing nine per-pixel SSIM coefficient
// maps, then image_loss_backward_coeffs_kernel :821-1028 blurring them).  Since
// d(total)/d(partials) is a constant in training, the backward needs nothing
// from the forward but those coefficients, so one CTA per 32x32 block and
// channel recomputes them over a 5-pixel halo instead of storing 36 B/pixel:
//
//   pred/gt over the block + 10-pixel halo (zero outside the image)
//   -> horizontal 11-tap blur of (x, x^2, y, y^2, xy)      [52 rows x 42 cols]
//   -> vertical blur, SSIM, per-pixel coefficients * chain  [42 x 42]
//   -> horizontal blur of the three coefficient products    [42 x 32]
//   -> vertical blur at the block: dL/dpred                 [32 x 32]
//
// Each blur runs as register sliding windows: a thread produces S
// consecutive outputs along the blur direction from one (S + 10)-value
// window (S = 7 over the 42-pixel footprint, 8 over the 32-pixel block, so the
// windows tile both exactly).  Every output still sums in the reference's order (taps d = 1..5 as
// (left + right) * w[5-d], then the centre), so the values equal the two-pass
// computation bit for bit.  The loss partials stay per 16x16 tile, each
// summed with the reference's shared-memory tree (lib.rs:108-123).
#include "vs_internal.cuh"

namespace {

using namespace vs;

constexpr int LB = 32;             // block edge
constexpr int HALO = 5;
constexpr int R0 = LB + 4 * HALO;  // 52: pred/gt footprint
constexpr int R1 = LB + 2 * HALO;  // 42: coefficient footprint
constexpr int NT = 256;
// outputs per thread and window: SEG1 over the 42-pixel coefficient footprint
// (42 = 6 x 7, no overrun), SEG2 over the 32-pixel block
constexpr int SEG1 = 7;
constexpr int SEG2 = 8;
constexpr int WIN1 = SEG1 + 2 * HALO;
constexpr int WIN2 = SEG2 + 2 * HALO;
constexpr int SUB = 16;            // loss partials per 16x16 tile
static_assert(R1 % SEG1 == 0 && LB % SEG2 == 0, "segments tile the footprints");

__constant__ float c_taps[11];

// Shared memory of one CTA (~95 KB, dynamic).  The horizontal moment sums are
// dead once the coefficients exist, so the second horizontal pass reuses them.
struct LossSmem {
  float x[R0][R0];
  float y[R0][R0];
  union {
    float h1[5][R0][R1];
    float h2[3][R1][LB];
  } u;
  float cm[3][R1][R1];
  float red[4][SUB * SUB];
};

__device__ __forceinline__ float gtap(int i) { return c_taps[i]; }

// out[j] = sum over the 11-tap window centred at win[j + 5], in the
// reference's order.
template <int S, int N>
__device__ __forceinline__ void blur_seg(const float (&win)[N], float (&out)[S]) {
  static_assert(N == S + 2 * HALO, "window");
#pragma unroll
  for (int j = 0; j < S; ++j) {
    float acc = 0.0f;
#pragma unroll
    for (int d = 1; d < 6; ++d) acc += (win[j + HALO - d] + win[j + HALO + d]) * gtap(5 - d);
    out[j] = acc + win[j + HALO] * gtap(5);
  }
}

__global__ void __launch_bounds__(NT) loss_kernel(uint32_t h, uint32_t w, const float* __restrict__ pred,
                                                  const uint32_t* __restrict__ gt, float l1_w, float ssim_w,
                                                  float rgb_weight, uint32_t tiles_x, uint32_t tiles_y,
                                                  float* __restrict__ partials, float* __restrict__ dl_dpred) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  LossSmem& sm = *reinterpret_cast<LossSmem*>(smem_raw);
  auto& s_x = sm.x;
  auto& s_y = sm.y;
  auto& s_h1 = sm.u.h1;
  auto& s_h2 = sm.u.h2;
  auto& s_cm = sm.cm;
  auto& s_red = sm.red;

  const int c = blockIdx.z;
  const int tid = threadIdx.x;
  const int x0 = blockIdx.x * LB, y0 = blockIdx.y * LB;
  const int W = (int)w, H = (int)h;

  // 1. pred/gt channel over the block +- 10
  for (int i = tid; i < R0 * R0; i += NT) {
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

  // 2. horizontal blur of the five moments: rows 0..51, columns block +- 5
  constexpr int HSEGS = R1 / SEG1;  // 6
  for (int it = tid; it < R0 * HSEGS; it += NT) {
    const int ly = it / HSEGS, c0 = (it % HSEGS) * SEG1;
    float wx[WIN1], wy[WIN1];
#pragma unroll
    for (int k = 0; k < WIN1; ++k) {
      wx[k] = s_x[ly][c0 + k];
      wy[k] = s_y[ly][c0 + k];
    }
    float m[WIN1], o[SEG1];
    blur_seg(wx, o);
#pragma unroll
    for (int j = 0; j < SEG1; ++j) s_h1[0][ly][c0 + j] = o[j];
#pragma unroll
    for (int k = 0; k < WIN1; ++k) m[k] = wx[k] * wx[k];
    blur_seg(m, o);
#pragma unroll
    for (int j = 0; j < SEG1; ++j) s_h1[1][ly][c0 + j] = o[j];
    blur_seg(wy, o);
#pragma unroll
    for (int j = 0; j < SEG1; ++j) s_h1[2][ly][c0 + j] = o[j];
#pragma unroll
    for (int k = 0; k < WIN1; ++k) m[k] = wy[k] * wy[k];
    blur_seg(m, o);
#pragma unroll
    for (int j = 0; j < SEG1; ++j) s_h1[3][ly][c0 + j] = o[j];
#pragma unroll
    for (int k = 0; k < WIN1; ++k) m[k] = wx[k] * wy[k];
    blur_seg(m, o);
#pragma unroll
    for (int j = 0; j < SEG1; ++j) s_h1[4][ly][c0 + j] = o[j];
  }
  __syncthreads();

  // 3. vertical blur -> SSIM coefficients (x chain) over block +- 5; the
  //    block's own pixels also produce the loss value.
  const float C1 = 0.01f * 0.01f, C2 = 0.03f * 0.03f;
  for (int it = tid; it < R1 * HSEGS; it += NT) {
    const int rx = it % R1, r0 = (it / R1) * SEG1;
    float o[5][SEG1];
#pragma unroll
    for (int k = 0; k < 5; ++k) {
      float win[WIN1];
#pragma unroll
      for (int q = 0; q < WIN1; ++q) win[q] = s_h1[k][r0 + q][rx];
      blur_seg(win, o[k]);
    }
#pragma unroll
    for (int j = 0; j < SEG1; ++j) {
      const int ry = r0 + j;
      const int gy = y0 - HALO + ry, gx = x0 - HALO + rx;
      const bool in_img = gy >= 0 && gy < H && gx >= 0 && gx < W;
      const bool in_blk = ry >= HALO && ry < HALO + LB && rx >= HALO && rx < HALO + LB;
      float c0 = 0.f, c1 = 0.f, c2 = 0.f, loss = 0.0f;
      if (in_img) {
        const float mu1 = o[0][j], mu2 = o[2][j];
        const float mu1_sq = mu1 * mu1, mu2_sq = mu2 * mu2;
        const float s1 = fmaxf(0.0f, o[1][j] - mu1_sq), s2 = fmaxf(0.0f, o[3][j] - mu2_sq);
        const float s12 = o[4][j] - mu1 * mu2;
        const float a = mu1_sq + mu2_sq + C1, b = s1 + s2 + C2;
        const float ct = 2.0f * mu1 * mu2 + C1, dt = 2.0f * s12 + C2;
        // b >= C2 and a b >= C1 C2: both reciprocals are in rcp_rn's exact range
        const float inv_b = rcp_rn(b), inv_ab = rcp_rn(a * b);
        const float cd = ct * dt * inv_ab;
        const bool cl = cd < -1.0f || cd > 1.0f;
        c0 = (cl ? 0.0f : 2.0f * inv_ab * (mu2 * (dt - ct) - mu1 * cd * (b - a))) * rgb_weight;
        c1 = (cl ? 0.0f : -cd * inv_b) * rgb_weight;
        c2 = (cl ? 0.0f : 2.0f * ct * inv_ab) * rgb_weight;
        if (in_blk) {
          const float raw = (ct * dt) / (a * b);
          const float val = clampf(raw, -1.0f, 1.0f);
          const float p1 = s_x[ry + HALO][rx + HALO], p2 = s_y[ry + HALO][rx + HALO];
          loss = l1_w * fabsf(p1 - p2) + ssim_w * val;
        }
      }
      if (in_blk) {
        const int bx = rx - HALO, by = ry - HALO;
        s_red[(by / SUB) * 2 + bx / SUB][(by % SUB) * SUB + bx % SUB] = loss;
      }
      s_cm[0][ry][rx] = c0;
      s_cm[1][ry][rx] = c1;
      s_cm[2][ry][rx] = c2;
    }
  }
  __syncthreads();

  // per-16x16-tile loss: the reference's tree, four tiles side by side
  for (int stride = SUB * SUB / 2; stride > 0; stride >>= 1) {
    for (int i = tid; i < 4 * stride; i += NT) {
      const int q = i / stride, k = i % stride;
      s_red[q][k] += s_red[q][k + stride];
    }
    __syncthreads();
  }
  if (tid < 4 && partials) {
    const uint32_t tx = blockIdx.x * 2 + (tid & 1), ty = blockIdx.y * 2 + (tid >> 1);
    if (tx < tiles_x && ty < tiles_y)
      partials[(size_t)c * tiles_x * tiles_y + ty * tiles_x + tx] = s_red[tid][0] * rgb_weight;
  }
  if (!dl_dpred) return;

  // 4. horizontal blur of the coefficient products: rows block +- 5, block columns
  constexpr int BSEGS = LB / SEG2;  // 4
  for (int it = tid; it < R1 * BSEGS; it += NT) {
    const int ry = it / BSEGS, t0 = (it % BSEGS) * SEG2;
#pragma unroll
    for (int k = 0; k < 3; ++k) {
      float win[WIN2], o[SEG2];
#pragma unroll
      for (int q = 0; q < WIN2; ++q) win[q] = s_cm[k][ry][t0 + q];
      blur_seg(win, o);
#pragma unroll
      for (int j = 0; j < SEG2; ++j) s_h2[k][ry][t0 + j] = o[j];
    }
  }
  __syncthreads();

  // 5. vertical blur at the block pixels -> dL/dpred
  for (int it = tid; it < LB * BSEGS; it += NT) {
    const int tx = it % LB, t0 = (it / LB) * SEG2;
    float s[3][SEG2];
#pragma unroll
    for (int k = 0; k < 3; ++k) {
      float win[WIN2];
#pragma unroll
      for (int q = 0; q < WIN2; ++q) win[q] = s_h2[k][t0 + q][tx];
      blur_seg(win, s[k]);
    }
#pragma unroll
    for (int j = 0; j < SEG2; ++j) {
      const int ty = t0 + j;
      const int gy = y0 + ty, gx = x0 + tx;
      if (gy < H && gx < W) {
        const float p1 = s_x[ty + 2 * HALO][tx + 2 * HALO], g = s_y[ty + 2 * HALO][tx + 2 * HALO];
        const float ssim_grad = s[0][j] + (2.0f * p1) * s[1][j] + g * s[2][j];
        const float diff = p1 - g;
        const float sign = diff > 0.0f ? 1.0f : (diff < 0.0f ? -1.0f : 0.0f);
        const size_t p = (size_t)gy * w + gx;
        dl_dpred[p * 4 + c] = ssim_w * ssim_grad + l1_w * sign * rgb_weight;
        if (c == 0) dl_dpred[p * 4 + 3] = 0.0f;
      }
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
  const uint32_t tx = div_up(w, 16), ty = div_up(h, 16);  // loss partials: per 16x16 tile
  float* parts = partials;
  if (!parts && loss_dev) {
    VS_TRY(vs_ensure(ctx, ctx->misc, (size_t)3 * tx * ty * 4));
    parts = (float*)ctx->misc.ptr;
  }
  const float rgb_weight = 1.0f / (3.0f * (float)(h * w));
  dim3 grid(div_up(w, LB), div_up(h, LB), 3);
  static_assert(sizeof(LossSmem) <= 227 * 1024, "loss shared memory");
  VS_CUDA(ctx, cudaFuncSetAttribute(loss_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sizeof(LossSmem)));
  loss_kernel<<<grid, NT, sizeof(LossSmem), ctx->stream>>>(h, w, pred, gt, l1_w, ssim_w, rgb_weight, tx, ty, parts, dl_dpred);
  ++ctx->launches;
  VS_CUDA(ctx, cudaGetLastError());
  if (loss_dev) {
    loss_total_kernel<<<1, 256, 0, ctx->stream>>>(parts, 3 * tx * ty, loss_dev);
    ++ctx->launches;
  }
  return vs_cuda(ctx, cudaGetLastError(), "loss launch");
}
