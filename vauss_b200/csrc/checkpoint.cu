// Checkpoint I/O: PLY vertex rows encoded and decoded on the GPU.
//
// Export (crates/splat-train-serde/src/export.rs:322-425, write_splat_ply):
// one row of little-endian f32 per splat in the inria property order
//   x y z scale_0..2 opacity rot_0..3 f_dc_0..2 f_rest_0..(3 rest - 1)
// with the quaternion divided by max(|q|, 1e-12) and the SH rest
// coefficients channel-major (all red, then green, then blue).  The rows are
// built by a kernel in chunks; each chunk's device-to-host copy overlaps the
// next chunk's encoding, and a pageable destination is filled from pinned
// staging by several host threads.
//
// Import (import.rs:386-510, parse_ply + interleave_coeffs :181-192): the
// host parses the header and hands the raw rows with a table of byte offsets,
// one per output value (-1 = the property is absent: the default value);
// chunks of rows move to the device through pinned staging and a kernel
// scatters them into the [N,10] / [N,C,3] / [N] layouts.
#include <algorithm>
#include <cstring>
#include <thread>
#include <vector>

#include "vs_internal.cuh"

namespace {

constexpr int kIoThreads = 256;
constexpr size_t kChunkBytes = 64ull << 20;  // rows per chunk: about 64 MB of PLY rows
constexpr uint32_t kMaxDecodeValues = 10 + 1 + 48;

struct DecodeTable {
  int32_t offset[kMaxDecodeValues];  // byte offset in a row, -1 = default
  float fallback[kMaxDecodeValues];
};

// One thread per output word: consecutive threads write consecutive words of
// the row block (coalesced); the reads gather within one splat's parameters.
__global__ void __launch_bounds__(kIoThreads)
    ply_encode_kernel(uint32_t first, uint32_t rows, uint32_t coeffs, const float* __restrict__ transforms,
                      const void* __restrict__ sh, bool sh_half, const float* __restrict__ raw_opac,
                      float* __restrict__ out) {
  const uint32_t rest = coeffs - 1;
  const uint32_t stride = 14 + 3 * rest;
  const uint64_t total = (uint64_t)rows * stride;
  for (uint64_t w = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; w < total;
       w += (uint64_t)gridDim.x * blockDim.x) {
    const uint32_t r = (uint32_t)(w / stride), col = (uint32_t)(w % stride);
    const size_t i = (size_t)first + r;
    const float* t = transforms + i * 10;
    float v;
    if (col < 3) {
      v = t[col];
    } else if (col < 6) {
      v = t[7 + (col - 3)];
    } else if (col == 6) {
      v = raw_opac[i];
    } else if (col < 11) {
      // |q| as ((r0 r0 + r1 r1) + r2 r2) + r3 r3 without contraction, IEEE
      // sqrt and division, max(|q|, 1e-12) with NaN giving 1e-12
      const float n2 = ((t[3] * t[3] + t[4] * t[4]) + t[5] * t[5]) + t[6] * t[6];
      const float rn = fmaxf(sqrtf(n2), 1.0e-12f);
      v = t[3 + (col - 7)] / rn;
    } else if (col < 14) {
      v = vs::sh_load(sh, sh_half, i * coeffs * 3 + (col - 11));
    } else {
      const uint32_t c = col - 14, ch = c / rest, k = 1 + c % rest;
      v = vs::sh_load(sh, sh_half, i * coeffs * 3 + k * 3 + ch);
    }
    out[w] = v;
  }
}

// One thread per output value of a chunk of rows (transforms 10, opacity 1,
// SH C*3 per splat).  Offsets are multiples of 4 (checked by the host call).
__global__ void __launch_bounds__(kIoThreads)
    ply_decode_kernel(uint32_t first, uint32_t rows, uint32_t row_bytes, uint32_t coeffs,
                      const uint8_t* __restrict__ src, DecodeTable table, float* __restrict__ transforms,
                      float* __restrict__ sh, float* __restrict__ raw_opac) {
  const uint32_t per = 11 + coeffs * 3;
  const uint64_t total = (uint64_t)rows * per;
  for (uint64_t w = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; w < total;
       w += (uint64_t)gridDim.x * blockDim.x) {
    const uint32_t r = (uint32_t)(w / per), j = (uint32_t)(w % per);
    const int32_t off = table.offset[j];
    const float v = off >= 0 ? *reinterpret_cast<const float*>(src + (size_t)r * row_bytes + off) : table.fallback[j];
    const size_t i = (size_t)first + r;
    if (j < 10) transforms[i * 10 + j] = v;
    else if (j == 10) raw_opac[i] = v;
    else sh[i * coeffs * 3 + (j - 11)] = v;
  }
}

uint32_t io_blocks(uint64_t work) {
  return (uint32_t)std::max<uint64_t>(1, std::min<uint64_t>((work + kIoThreads - 1) / kIoThreads, 148ull * 16));
}

bool is_pinned(const void* p) {
  cudaPointerAttributes a{};
  if (cudaPointerGetAttributes(&a, p) != cudaSuccess) {
    cudaGetLastError();
    return false;
  }
  return a.type == cudaMemoryTypeHost;
}

// Copies `bytes` with up to 8 host threads.
void parallel_memcpy(void* dst, const void* src, size_t bytes) {
  const size_t per = 8ull << 20;
  const unsigned nt = (unsigned)std::min<size_t>(8, (bytes + per - 1) / per);
  if (nt <= 1) {
    std::memcpy(dst, src, bytes);
    return;
  }
  std::vector<std::thread> ts;
  const size_t part = (bytes + nt - 1) / nt;
  for (unsigned k = 0; k < nt; ++k) {
    const size_t a = k * part, b = std::min(bytes, a + part);
    if (a < b)
      ts.emplace_back([=] { std::memcpy(static_cast<char*>(dst) + a, static_cast<const char*>(src) + a, b - a); });
  }
  for (auto& t : ts) t.join();
}

// Two pinned staging buffers and two events for a chunked transfer.
struct Staging {
  vs_ctx* ctx;
  void* host[2] = {nullptr, nullptr};
  cudaEvent_t done[2] = {nullptr, nullptr};
  explicit Staging(vs_ctx* c) : ctx(c) {}
  vs_status init(size_t bytes) {
    for (int k = 0; k < 2; ++k) {
      VS_CUDA(ctx, cudaHostAlloc(&host[k], bytes, cudaHostAllocDefault));
      VS_CUDA(ctx, cudaEventCreateWithFlags(&done[k], cudaEventDisableTiming));
    }
    return VS_OK;
  }
  ~Staging() {
    for (int k = 0; k < 2; ++k) {
      if (done[k]) cudaEventSynchronize(done[k]), cudaEventDestroy(done[k]);
      if (host[k]) cudaFreeHost(host[k]);
    }
  }
};

}  // namespace

VS_API uint64_t vs_ply_row_bytes(int32_t sh_degree) {
  if (sh_degree < 0 || sh_degree > 3) return 0;
  const uint64_t coeffs = (uint64_t)(sh_degree + 1) * (sh_degree + 1);
  return 4 * (14 + 3 * (coeffs - 1));
}

VS_API vs_status vs_ply_encode(vs_ctx* ctx, uint32_t num_splats, int32_t sh_degree, const float* transforms,
                               const void* sh_coeffs, int32_t sh_half, const float* raw_opacities, void* host_out) {
  if (!ctx) return VS_ERR_INVALID;
  if (sh_degree < 0 || sh_degree > 3) return vs_fail(ctx, VS_ERR_UNSUPPORTED, "ply_encode: SH degree %d", sh_degree);
  if (num_splats == 0) return VS_OK;
  if (!transforms || !sh_coeffs || !raw_opacities || !host_out)
    return vs_fail(ctx, VS_ERR_INVALID, "ply_encode: null argument");
  VS_CUDA(ctx, cudaSetDevice(ctx->device));
  const uint32_t coeffs = (uint32_t)((sh_degree + 1) * (sh_degree + 1));
  const size_t row = vs_ply_row_bytes(sh_degree);
  const uint32_t chunk_rows = (uint32_t)std::max<size_t>(1, std::min<size_t>(kChunkBytes / row, num_splats));
  const size_t chunk_bytes = (size_t)chunk_rows * row;
  VS_TRY(vs_ensure(ctx, ctx->io_stage, 2 * chunk_bytes));
  uint8_t* dev = static_cast<uint8_t*>(ctx->io_stage.ptr);
  const bool direct = is_pinned(host_out);
  Staging st(ctx);
  if (!direct) VS_TRY(st.init(chunk_bytes));
  const uint32_t chunks = (num_splats + chunk_rows - 1) / chunk_rows;
  for (uint32_t c = 0; c <= chunks; ++c) {
    if (c < chunks) {
      const uint32_t first = c * chunk_rows, rows = std::min(chunk_rows, num_splats - first);
      const size_t bytes = (size_t)rows * row;
      uint8_t* d = dev + (size_t)(c & 1) * chunk_bytes;
      // the device half was last read by the copy of chunk c - 2, queued
      // before on this stream
      ply_encode_kernel<<<io_blocks((uint64_t)rows * (row / 4)), kIoThreads, 0, ctx->stream>>>(
          first, rows, coeffs, transforms, sh_coeffs, sh_half != 0, raw_opacities, reinterpret_cast<float*>(d));
      ++ctx->launches;
      VS_CUDA(ctx, cudaGetLastError());
      if (direct) {
        VS_CUDA(ctx, cudaMemcpyAsync(static_cast<uint8_t*>(host_out) + (size_t)first * row, d, bytes,
                                     cudaMemcpyDeviceToHost, ctx->stream));
      } else {
        VS_CUDA(ctx, cudaMemcpyAsync(st.host[c & 1], d, bytes, cudaMemcpyDeviceToHost, ctx->stream));
        VS_CUDA(ctx, cudaEventRecord(st.done[c & 1], ctx->stream));
      }
    }
    if (!direct && c >= 1) {  // chunk c - 1 to its place while chunk c copies
      const uint32_t p = c - 1, first = p * chunk_rows, rows = std::min(chunk_rows, num_splats - first);
      VS_CUDA(ctx, cudaEventSynchronize(st.done[p & 1]));
      parallel_memcpy(static_cast<uint8_t*>(host_out) + (size_t)first * row, st.host[p & 1], (size_t)rows * row);
    }
  }
  VS_CUDA(ctx, cudaStreamSynchronize(ctx->stream));
  return VS_OK;
}

VS_API vs_status vs_ply_decode(vs_ctx* ctx, uint32_t num_splats, const void* host_rows, uint32_t row_bytes,
                               uint32_t sh_coeffs_per_channel, const int32_t* offsets, const float* defaults,
                               float* transforms, float* sh_coeffs, float* raw_opacities) {
  if (!ctx) return VS_ERR_INVALID;
  const uint32_t coeffs = sh_coeffs_per_channel;
  if (coeffs != 1 && coeffs != 4 && coeffs != 9 && coeffs != 16)
    return vs_fail(ctx, VS_ERR_UNSUPPORTED, "ply_decode: %u SH coefficients per channel", coeffs);
  if (num_splats == 0) return VS_OK;
  if (!host_rows || !offsets || !defaults || !transforms || !sh_coeffs || !raw_opacities)
    return vs_fail(ctx, VS_ERR_INVALID, "ply_decode: null argument");
  const uint32_t per = 11 + 3 * coeffs;
  DecodeTable table{};
  if (row_bytes == 0 || row_bytes % 4) return vs_fail(ctx, VS_ERR_INVALID, "ply_decode: row of %u bytes", row_bytes);
  for (uint32_t j = 0; j < per; ++j) {
    const int32_t o = offsets[j];
    if (o >= 0 && (o % 4 || (uint32_t)o + 4 > row_bytes))
      return vs_fail(ctx, VS_ERR_INVALID, "ply_decode: value %u at byte %d of a %u-byte row", j, o, row_bytes);
    table.offset[j] = o;
    table.fallback[j] = defaults[j];
  }
  VS_CUDA(ctx, cudaSetDevice(ctx->device));
  const uint32_t chunk_rows = (uint32_t)std::max<size_t>(1, std::min<size_t>(kChunkBytes / row_bytes, num_splats));
  const size_t chunk_bytes = (size_t)chunk_rows * row_bytes;
  VS_TRY(vs_ensure(ctx, ctx->io_stage, 2 * chunk_bytes));
  uint8_t* dev = static_cast<uint8_t*>(ctx->io_stage.ptr);
  const bool direct = is_pinned(host_rows);
  Staging st(ctx);
  if (!direct) VS_TRY(st.init(chunk_bytes));
  const uint32_t chunks = (num_splats + chunk_rows - 1) / chunk_rows;
  for (uint32_t c = 0; c < chunks; ++c) {
    const uint32_t first = c * chunk_rows, rows = std::min(chunk_rows, num_splats - first);
    const size_t bytes = (size_t)rows * row_bytes;
    const uint8_t* src = static_cast<const uint8_t*>(host_rows) + (size_t)first * row_bytes;
    uint8_t* d = dev + (size_t)(c & 1) * chunk_bytes;
    if (direct) {
      VS_CUDA(ctx, cudaMemcpyAsync(d, src, bytes, cudaMemcpyHostToDevice, ctx->stream));
    } else {
      // staging half c & 1 was last copied from by chunk c - 2
      if (c >= 2) VS_CUDA(ctx, cudaEventSynchronize(st.done[c & 1]));
      parallel_memcpy(st.host[c & 1], src, bytes);
      VS_CUDA(ctx, cudaMemcpyAsync(d, st.host[c & 1], bytes, cudaMemcpyHostToDevice, ctx->stream));
      VS_CUDA(ctx, cudaEventRecord(st.done[c & 1], ctx->stream));
    }
    ply_decode_kernel<<<io_blocks((uint64_t)rows * per), kIoThreads, 0, ctx->stream>>>(
        first, rows, row_bytes, coeffs, d, table, transforms, sh_coeffs, raw_opacities);
    ++ctx->launches;
    VS_CUDA(ctx, cudaGetLastError());
  }
  VS_CUDA(ctx, cudaStreamSynchronize(ctx->stream));
  return VS_OK;
}
