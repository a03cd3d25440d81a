// Host-side internals: context, frames, workspace, launch declarations.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>
#include <string>

#include "../../include/vauss_b200.h"
#include "vs_common.cuh"

// A grow-only device allocation.
struct DevBuf {
  void* ptr = nullptr;
  size_t bytes = 0;
};

struct vs_ctx {
  int device = 0;
  cudaStream_t stream = nullptr;
  std::string err;
  uint32_t* d_err = nullptr;       // device error word (VS_DERR_*)
  uint32_t* h_pinned = nullptr;    // pinned host mirror for small readbacks (16 words)
  uint64_t workspace = 0;          // bytes held by the ctx and its frames
  uint64_t launches = 0;           // kernels launched through this ctx
  bool taps_ready = false;         // SSIM window uploaded to this device's constant memory
  // scratch shared by calls on this ctx (stream-ordered reuse)
  DevBuf sort_keys, sort_vals, sort_hist, scan_sums, misc;
  DevBuf io_stage;  // checkpoint I/O chunks (two halves)
  DevBuf vjp_rows;  // per-visible-splat VJP rows of the single-view Q8 step
};

struct vs_frame {
  vs_ctx* ctx = nullptr;
  vs::Uniforms u{};
  vs_render_cfg cfg{};
  uint32_t n = 0, v = 0, T = 0;
  uint64_t I = 0;
  uint32_t depth_lo = 0, depth_hi = 0;  // bit range of the visible splats' depths (projection readback)
  bool projected_ok = false, binned = false, rendered = false;
  DevBuf compact_from_global, global_from_compact, depths, tile_counts, tile_masks, projected, depth_order;
  DevBuf isect_tile, isect_compact, tile_ranges, tile_used_end, opacities, max_radius;
  DevBuf lookback, counters;  // projection compaction state
};

// Records a message on the ctx and returns `st`.
vs_status vs_fail(vs_ctx* ctx, vs_status st, const char* fmt, ...);
// Checks a CUDA call result.
vs_status vs_cuda(vs_ctx* ctx, cudaError_t e, const char* what);
// Grows `b` to at least `bytes` (contents are not preserved).
vs_status vs_ensure(vs_ctx* ctx, DevBuf& b, size_t bytes);
void vs_release(vs_ctx* ctx, DevBuf& b);
// Reads the device error word, clears it, and maps it to a status.
vs_status vs_check_device_error(vs_ctx* ctx, const char* stage);

#define VS_TRY(expr)                  \
  do {                                \
    vs_status _st = (expr);           \
    if (_st != VS_OK) return _st;     \
  } while (0)
#define VS_CUDA(ctx, expr) VS_TRY(vs_cuda((ctx), (expr), #expr))

vs::Uniforms vs_make_uniforms(const vs_camera& c, const vs_render_cfg& cfg);

// ---- launchers (defined next to their kernels) ----
vs_status launch_project(vs_ctx* ctx, vs_frame* f, const float* transforms, const void* sh, const float* raw_opac,
                         const float* min_scale);
// Stable LSD sort over the low key_bits bits in radix_sort_passes(key_bits)
// passes of at most 9 bits; the result is in keys_alt/vals_alt after an odd
// number of passes (*result_in_alt), else in keys/vals.
uint32_t radix_sort_passes(uint32_t key_bits);
// The same sort with the input read in place: pass 0 reads keys_in[i] -
// key_sub and vals_in[i] (i when vals_in is NULL) and writes (a_keys,
// a_vals), every later pass reads what the previous one wrote and writes the
// other pair, so the result is in (a_*) after an odd number of passes, else
// in (b_*); with gather_out the last pass also writes gather_out[i] =
// gather_src[value i].  Nothing is written when key_bits or count is 0.
vs_status radix_sort_from(vs_ctx* ctx, const uint32_t* keys_in, const uint32_t* vals_in, uint32_t key_sub,
                          uint32_t* a_keys, uint32_t* a_vals, uint32_t* b_keys, uint32_t* b_vals, uint32_t count,
                          uint32_t key_bits, const uint32_t* gather_src, uint32_t* gather_out);
vs_status radix_sort_pairs(vs_ctx* ctx, uint32_t* keys, uint32_t* vals, uint32_t* keys_alt, uint32_t* vals_alt,
                           uint32_t count, uint32_t key_bits, bool* result_in_alt);
vs_status scan_inclusive_u32(vs_ctx* ctx, uint32_t* data, uint32_t count, uint64_t* total_dev);
// out[i] = src[idx[0]] + ... + src[idx[i]]
vs_status scan_gather_inclusive_u32(vs_ctx* ctx, uint32_t* out, const uint32_t* src, const uint32_t* idx,
                                    uint32_t count);
vs_status launch_bin(vs_ctx* ctx, vs_frame* f);
vs_status launch_raster_fwd(vs_ctx* ctx, vs_frame* f, float* out_img, float* visible);
vs_status launch_raster_packed(vs_ctx* ctx, vs_frame* f, uint32_t* out_rgba8);
vs_status launch_raster_bwd(vs_ctx* ctx, vs_frame* f, const float* out_img, const float* v_out, float* v_combined);
vs_status launch_loss(vs_ctx* ctx, uint32_t h, uint32_t w, const float* pred, const uint32_t* gt, float l1_w,
                      float ssim_w, float* partials, float* loss_dev, float* dl_dpred);
