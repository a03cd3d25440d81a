// CPU parity oracle for the Gaussian-splat training step.
//
// TEST INFRASTRUCTURE ONLY.  This file restates, on the host, the
// algorithm of each reference kernel on the training-step path so the CUDA
// kernels in vauss_b200/csrc can be checked against it.  Nothing in the
// product imports, links or calls it; only tests/, __graft_entry__.smoke()
// and bench.py's cpu_baseline leg do.
//
// Reference: voyager-so/vauss (Brush-derived Rust/CubeCL trainer).  Each
// function names the reference file:line it follows; paths are relative to
// the reference project's root.
//
// Arithmetic conventions (shared with the kernels, so integer outputs and the
// front-to-back compositing compare bit-for-bit):
//  * build with -ffp-contract=off; every multiply-add that is fused is written
//    as an explicit fmaf() here and in the kernel;
//  * exp/log/sigmoid come from vauss_b200/csrc/vs_math.h (own Cody-Waite
//    implementations, identical on host and device);
//  * sqrt and division are IEEE correctly rounded on both sides.
// Reductions whose order differs on the GPU (atomics in the rasterizer
// backward) are compared with a tolerance by the tests.

#include <omp.h>
#include <stdint.h>
#include <string.h>
#include <math.h>
#include <algorithm>
#include <vector>
#include <numeric>

#include "../vauss_b200/csrc/vs_math.h"

#define OR_API extern "C" __attribute__((visibility("default")))

namespace {

constexpr uint32_t TILE = 16;
constexpr float ALPHA_MIN = 1.0f / 255.0f;
constexpr float ALPHA_BAND = 1.0e-3f;

struct Camera {
  float vm[12];  // world -> camera 3x4, column-major (rotation columns, then translation)
  float fx, fy, cx, cy;
  float cam[3];
  uint32_t w, h;
};

struct RenderCfg {
  int32_t mip;
  int32_t sh_degree;
  int32_t sh_half;
  int32_t has_min_scale;
  float log_scale_offset;
  float bg[3];
};

struct V3 { float x, y, z; };
struct Q4 { float w, x, y, z; };
struct M3 { float c0x, c0y, c0z, c1x, c1y, c1z, c2x, c2y, c2z; };  // column-major
struct S2 { float c00, c01, c11; };
struct S3 { float c00, c01, c02, c11, c12, c22; };
struct V2 { float x, y; };
struct M23 { V2 c0, c1, c2; };

// ---- math types: crates/splat-train-cube/src/lib.rs ----------------------
inline V3 v3add(V3 a, V3 b) { return {a.x + b.x, a.y + b.y, a.z + b.z}; }
inline V3 v3sub(V3 a, V3 b) { return {a.x - b.x, a.y - b.y, a.z - b.z}; }
inline V3 v3scale(V3 a, float s) { return {a.x * s, a.y * s, a.z * s}; }
// lib.rs:85-89 (lane 3 is zero: the 4-lane sum adds +0 last)
inline float v3dot(V3 a, V3 b) { return ((a.x * b.x + a.y * b.y) + a.z * b.z) + 0.0f; }
inline bool v3finite(V3 a) { return vs_is_finite(a.x) && vs_is_finite(a.y) && vs_is_finite(a.z); }
inline float q4dot(Q4 a) { return ((a.w * a.w + a.x * a.x) + a.y * a.y) + a.z * a.z; }
inline Q4 q4scale(Q4 a, float s) { return {a.w * s, a.x * s, a.y * s, a.z * s}; }

// lib.rs:192-217
inline M3 quat_to_mat3(Q4 q) {
  const float x2 = q.x * q.x, y2 = q.y * q.y, z2 = q.z * q.z;
  const float xy = q.x * q.y, xz = q.x * q.z, yz = q.y * q.z;
  const float wx = q.w * q.x, wy = q.w * q.y, wz = q.w * q.z;
  return {1.0f - 2.0f * (y2 + z2), 2.0f * (xy + wz), 2.0f * (xz - wy),
          2.0f * (xy - wz), 1.0f - 2.0f * (x2 + z2), 2.0f * (yz + wx),
          2.0f * (xz + wy), 2.0f * (yz - wx), 1.0f - 2.0f * (x2 + y2)};
}
inline V3 m3col0(const M3& m) { return {m.c0x, m.c0y, m.c0z}; }
inline V3 m3col1(const M3& m) { return {m.c1x, m.c1y, m.c1z}; }
inline V3 m3col2(const M3& m) { return {m.c2x, m.c2y, m.c2z}; }
inline M3 m3from(V3 a, V3 b, V3 c) { return {a.x, a.y, a.z, b.x, b.y, b.z, c.x, c.y, c.z}; }
// lib.rs:264-269
inline V3 m3mulv(const M3& m, V3 v) {
  return v3add(v3add(v3scale(m3col0(m), v.x), v3scale(m3col1(m), v.y)), v3scale(m3col2(m), v.z));
}
// lib.rs:272-274
inline V3 m3tmulv(const M3& m, V3 v) { return {v3dot(m3col0(m), v), v3dot(m3col1(m), v), v3dot(m3col2(m), v)}; }
inline M3 m3mul(const M3& a, const M3& b) {
  return m3from(m3mulv(a, m3col0(b)), m3mulv(a, m3col1(b)), m3mulv(a, m3col2(b)));
}
inline M3 m3diag(const M3& m, V3 s) {
  return m3from(v3scale(m3col0(m), s.x), v3scale(m3col1(m), s.y), v3scale(m3col2(m), s.z));
}
inline V3 m3row0(const M3& m) { return {m.c0x, m.c1x, m.c2x}; }
inline V3 m3row1(const M3& m) { return {m.c0y, m.c1y, m.c2y}; }
inline V3 m3row2(const M3& m) { return {m.c0z, m.c1z, m.c2z}; }
// lib.rs:307-319
inline S3 m3outer_self(const M3& m) {
  const V3 r0 = m3row0(m), r1 = m3row1(m), r2 = m3row2(m);
  return {v3dot(r0, r0), v3dot(r0, r1), v3dot(r0, r2), v3dot(r1, r1), v3dot(r1, r2), v3dot(r2, r2)};
}
inline V2 v2add(V2 a, V2 b) { return {a.x + b.x, a.y + b.y}; }
inline V2 v2scale(V2 a, float s) { return {a.x * s, a.y * s}; }
inline float v2dot(V2 a, V2 b) { return a.x * b.x + a.y * b.y; }
// lib.rs:343-348
inline V2 m23mulv(const M23& m, V3 v) { return v2add(v2add(v2scale(m.c0, v.x), v2scale(m.c1, v.y)), v2scale(m.c2, v.z)); }
inline M23 m23mul(const M23& m, const M3& n) { return {m23mulv(m, m3col0(n)), m23mulv(m, m3col1(n)), m23mulv(m, m3col2(n))}; }
inline V3 m23row0(const M23& m) { return {m.c0.x, m.c1.x, m.c2.x}; }
inline V3 m23row1(const M23& m) { return {m.c0.y, m.c1.y, m.c2.y}; }
// lib.rs:373-379
inline S2 m23gram(const M23& m) {
  return {m.c0.x * m.c0.x + m.c1.x * m.c1.x + m.c2.x * m.c2.x,
          m.c0.x * m.c0.y + m.c1.x * m.c1.y + m.c2.x * m.c2.y,
          m.c0.y * m.c0.y + m.c1.y * m.c1.y + m.c2.y * m.c2.y};
}
inline V2 s2mulv(S2 s, V2 v) { return v2add(v2scale({s.c00, s.c01}, v.x), v2scale({s.c01, s.c11}, v.y)); }
// lib.rs:359-371
inline S3 m23tcong(const M23& m, S2 s) {
  const V2 sc0 = s2mulv(s, m.c0), sc1 = s2mulv(s, m.c1), sc2 = s2mulv(s, m.c2);
  return {v2dot(m.c0, sc0), v2dot(m.c0, sc1), v2dot(m.c0, sc2), v2dot(m.c1, sc1), v2dot(m.c1, sc2), v2dot(m.c2, sc2)};
}
inline M23 s2mulm23(S2 s, const M23& n) { return {s2mulv(s, n.c0), s2mulv(s, n.c1), s2mulv(s, n.c2)}; }
// lib.rs:432-441
inline S2 s2inverse(S2 s) {
  const float det = s.c00 * s.c11 - s.c01 * s.c01;
  const float inv_det = det > 0.0f ? 1.0f / det : 0.0f;
  return {s.c11 * inv_det, -s.c01 * inv_det, s.c00 * inv_det};
}
inline float s2det(S2 s) { return s.c00 * s.c11 - s.c01 * s.c01; }
inline bool s2finite(S2 s) { return vs_is_finite(s.c00) && vs_is_finite(s.c11) && vs_is_finite(s.c01); }
inline V3 s3row0(S3 s) { return {s.c00, s.c01, s.c02}; }
inline V3 s3row1(S3 s) { return {s.c01, s.c11, s.c12}; }
inline V3 s3row2(S3 s) { return {s.c02, s.c12, s.c22}; }
inline V3 s3mulv(S3 s, V3 v) { return v3add(v3add(v3scale(s3row0(s), v.x), v3scale(s3row1(s), v.y)), v3scale(s3row2(s), v.z)); }
inline S3 s3scale(S3 s, float k) { return {s.c00 * k, s.c01 * k, s.c02 * k, s.c11 * k, s.c12 * k, s.c22 * k}; }
inline M3 s3mulm3(S3 s, const M3& m) { return m3from(s3mulv(s, m3col0(m)), s3mulv(s, m3col1(m)), s3mulv(s, m3col2(m))); }
// lib.rs:511-523 (m * self * m^T)
inline S3 s3cong(S3 s, const M3& m) {
  const V3 sr0 = s3mulv(s, m3row0(m)), sr1 = s3mulv(s, m3row1(m)), sr2 = s3mulv(s, m3row2(m));
  return {v3dot(m3row0(m), sr0), v3dot(m3row0(m), sr1), v3dot(m3row0(m), sr2),
          v3dot(m3row1(m), sr1), v3dot(m3row1(m), sr2), v3dot(m3row2(m), sr2)};
}
// lib.rs:526-538 (m^T * self * m)
inline S3 s3tcong(S3 s, const M3& m) {
  const V3 sc0 = s3mulv(s, m3col0(m)), sc1 = s3mulv(s, m3col1(m)), sc2 = s3mulv(s, m3col2(m));
  return {v3dot(m3col0(m), sc0), v3dot(m3col0(m), sc1), v3dot(m3col0(m), sc2),
          v3dot(m3col1(m), sc1), v3dot(m3col1(m), sc2), v3dot(m3col2(m), sc2)};
}
inline float clampf(float x, float lo, float hi) { return fminf(fmaxf(x, lo), hi); }

// lib.rs:575-579
inline float calc_sigma(float px, float py, S2 c, float xx, float xy) {
  const float dx = px - xx, dy = py - xy;
  return 0.5f * (c.c00 * dx * dx + c.c11 * dy * dy) + c.c01 * dx * dy;
}

// ---- uniforms -----------------------------------------------------------
struct Uniforms {
  M3 rot;
  V3 trans;
  float fx, fy, cx, cy;
  float lim_pos_x, lim_pos_y, lim_neg_x, lim_neg_y;
  V3 cam;
  uint32_t w, h, tbw, tbh;
};

// crates/splat-train-render/src/camera.rs:305-331 (pinhole clamp limits),
// src/render.rs:483-503 (uniform assembly), kernels/types.rs:84-108.
Uniforms make_uniforms(const Camera& c) {
  Uniforms u;
  u.rot = {c.vm[0], c.vm[1], c.vm[2], c.vm[3], c.vm[4], c.vm[5], c.vm[6], c.vm[7], c.vm[8]};
  u.trans = {c.vm[9], c.vm[10], c.vm[11]};
  u.fx = c.fx; u.fy = c.fy; u.cx = c.cx; u.cy = c.cy;
  const float w = (float)c.w, h = (float)c.h;
  u.lim_pos_x = (1.15f * w - c.cx) / c.fx;
  u.lim_pos_y = (1.15f * h - c.cy) / c.fy;
  u.lim_neg_x = (-0.15f * w - c.cx) / c.fx;
  u.lim_neg_y = (-0.15f * h - c.cy) / c.fy;
  u.cam = {c.cam[0], c.cam[1], c.cam[2]};
  u.w = c.w; u.h = c.h;
  u.tbw = (c.w + TILE - 1) / TILE;
  u.tbh = (c.h + TILE - 1) / TILE;
  return u;
}

// kernels/helpers.rs:473-475
inline V3 world_to_cam(V3 m, const Uniforms& u) { return v3add(m3mulv(u.rot, m), u.trans); }

// kernels/camera_model/pinhole.rs:153-177
inline M23 pinhole_jacobian(V3 p, const Uniforms& u) {
  const float inv_z = 1.0f / p.z;
  const float dx = u.fx * inv_z, dy = u.fy * inv_z;
  const float clx = clampf(p.x * inv_z, u.lim_neg_x, u.lim_pos_x);
  const float cly = clampf(p.y * inv_z, u.lim_neg_y, u.lim_pos_y);
  return {{dx, 0.0f}, {0.0f, dy}, {-dx * clx, -dy * cly}};
}

// kernels/camera_model/pinhole.rs:145-151
inline void project_pinhole(V3 p, const Uniforms& u, float* px, float* py) {
  const float inv_z = 1.0f / p.z;
  *px = u.fx * p.x * inv_z + u.cx;
  *py = u.fy * p.y * inv_z + u.cy;
}

// kernels/helpers.rs:195-225
inline S2 calc_cov2d(V3 scale, Q4 quat, V3 mean_c, const Uniforms& u) {
  const M3 ns = m3diag(m3mul(u.rot, quat_to_mat3(quat)), scale);
  const M23 jac = pinhole_jacobian(mean_c, u);
  const M23 v = m23mul(jac, ns);
  S2 raw = m23gram(v);
  const float lim = 1.0e18f;
  const float max_abs = fmaxf(fmaxf(fabsf(raw.c00), fabsf(raw.c11)), fabsf(raw.c01));
  const float sd = max_abs > lim ? lim / max_abs : 1.0f;
  return {raw.c00 * sd, raw.c01 * sd, raw.c11 * sd};
}

// kernels/helpers.rs:230-245
inline S2 compensate_cov2d(S2 c, bool mip, float* comp) {
  const float blur = mip ? 0.1f : 0.3f;
  const S2 b = {c.c00 + blur, c.c01, c.c11 + blur};
  *comp = 1.0f;
  if (mip) {
    const float det_raw = fmaxf(s2det(c), 0.0f);
    const float det_b = s2det(b);
    *comp = sqrtf(det_raw / det_b);
  }
  return b;
}

// kernels/helpers.rs:133-144
inline void bbox_extent(S2 c, float pt, float* ex, float* ey) {
  const float det = c.c00 * c.c11 - c.c01 * c.c01;
  const bool degenerate = det <= 0.0f;
  const float inv_det = degenerate ? 0.0f : 1.0f / det;
  const float x = sqrtf(2.0f * pt * c.c11 * inv_det);
  const float y = sqrtf(2.0f * pt * c.c00 * inv_det);
  *ex = degenerate ? -1.0f : x;
  *ey = degenerate ? -1.0f : y;
}

struct TileBox { uint32_t x0, y0, x1, y1; };
// kernels/helpers.rs:158-190
inline TileBox tile_bbox(float cx, float cy, float ex, float ey, uint32_t bw, uint32_t bh) {
  const float tw = (float)TILE;
  const float x = cx / tw, y = cy / tw, dx = ex / tw, dy = ey / tw;
  const float bwf = (float)bw, bhf = (float)bh;
  return {(uint32_t)clampf(x - dx, 0.0f, bwf), (uint32_t)clampf(y - dy, 0.0f, bhf),
          (uint32_t)clampf(x + dx + 1.0f, 0.0f, bwf), (uint32_t)clampf(y + dy + 1.0f, 0.0f, bhf)};
}

// kernels/helpers.rs:276-314 (StopThePop tile test)
inline bool tile_hit(uint32_t tx, uint32_t ty, float mx, float my, S2 c, float pt) {
  const float min_x = (float)(tx * TILE), min_y = (float)(ty * TILE);
  const float max_x = min_x + (float)TILE, max_y = min_y + (float)TILE;
  const bool x_left = mx < min_x, x_right = mx > max_x;
  const bool in_x = !(x_left || x_right);
  const bool y_above = my < min_y, y_below = my > max_y;
  const bool in_y = !(y_above || y_below);
  if (in_x && in_y) return true;
  const float corner_x = x_left ? min_x : max_x;
  const float corner_y = y_above ? min_y : max_y;
  const float width = max_x - min_x, height = max_y - min_y;
  const float dxf = x_left ? width : -width;
  const float dyf = y_above ? height : -height;
  const float diff_x = mx - corner_x, diff_y = my - corner_y;
  const float tx_raw = (dxf * c.c00 * diff_x + dxf * c.c01 * diff_y) / (dxf * c.c00 * dxf);
  const float ty_raw = (dyf * c.c01 * diff_x + dyf * c.c11 * diff_y) / (dyf * c.c11 * dyf);
  const float txc = in_y ? 0.0f : clampf(tx_raw, 0.0f, 1.0f);
  const float tyc = in_x ? 0.0f : clampf(ty_raw, 0.0f, 1.0f);
  const float px = corner_x + txc * dxf;
  const float py = corner_y + tyc * dyf;
  return calc_sigma(px, py, c, mx, my) <= pt;
}

// kernels/helpers.rs:254-273
inline uint32_t count_tiles(TileBox b, float mx, float my, S2 c, float pt) {
  const uint32_t bw = b.x1 - b.x0;
  const uint32_t n = (b.y1 - b.y0) * bw;
  uint32_t hits = 0;
  for (uint32_t i = 0; i < n; ++i) {
    const uint32_t tx = i % bw + b.x0, ty = i / bw + b.y0;
    if (tile_hit(tx, ty, mx, my, c, pt)) ++hits;
  }
  return hits;
}

struct Floor { V3 scale; float opac, coef; V3 ratio_sq; bool opac_open; };
// kernels/helpers.rs:516-553
inline Floor apply_scale_floor(V3 s, float opac_sig, const float* min_scale, uint32_t g, bool has) {
  Floor f{s, opac_sig, 1.0f, {1.0f, 1.0f, 1.0f}, true};
  if (has) {
    const float fl = min_scale[g], f2 = fl * fl;
    f.scale = {sqrtf(s.x * s.x + f2), sqrtf(s.y * s.y + f2), sqrtf(s.z * s.z + f2)};
    const float rx = s.x / f.scale.x, ry = s.y / f.scale.y, rz = s.z / f.scale.z;
    f.coef = rx * ry * rz;
    f.ratio_sq = {rx * rx, ry * ry, rz * rz};
    const float o = opac_sig * f.coef;
    f.opac_open = o > 1e-6f && o < 1.0f - 1e-6f;
    f.opac = clampf(o, 1e-6f, 1.0f - 1e-6f);
  }
  return f;
}

inline V3 read_scale(const float* t, float off) {
  return {vs_expf(t[7] + off), vs_expf(t[8] + off), vs_expf(t[9] + off)};
}

inline float sh_coeff(const void* sh, bool half, size_t i) {
  return half ? vs_f16_to_f32(((const uint16_t*)sh)[i]) : ((const float*)sh)[i];
}

constexpr float SH_C0 = 0.2820948f;

// kernels/sh.rs:51-140 (sh_coeffs_to_color), bands <= 3
V3 sh_to_color(const void* sh, bool half, size_t base, int deg, V3 v) {
  auto rc = [&](size_t k) -> V3 { return {sh_coeff(sh, half, base + k), sh_coeff(sh, half, base + k + 1), sh_coeff(sh, half, base + k + 2)}; };
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
      const float p4 = f1a * fs1, p5 = f0b * v.y, p6 = 0.9461747f * z2 - 0.31539157f;
      const float p7 = f0b * v.x, p8 = f1a * fc1;
      color = v3add(color, v3scale(rc(12), p4));
      color = v3add(color, v3scale(rc(15), p5));
      color = v3add(color, v3scale(rc(18), p6));
      color = v3add(color, v3scale(rc(21), p7));
      color = v3add(color, v3scale(rc(24), p8));
      if (deg >= 3) {
        const float f0c = -2.285229f * z2 + 0.4570458f;
        const float f1b = 1.4453057f * v.z;
        const float f2a = -0.5900436f;
        const float fc2 = v.x * fc1 - v.y * fs1;
        const float fs2 = v.x * fs1 + v.y * fc1;
        const float p12 = v.z * (1.8658817f * z2 - 1.119529f);
        const float p9 = f2a * fs2, p10 = f1b * fs1, p11 = f0c * v.y;
        const float p13 = f0c * v.x, p14 = f1b * fc1, p15 = f2a * fc2;
        color = v3add(color, v3scale(rc(27), p9));
        color = v3add(color, v3scale(rc(30), p10));
        color = v3add(color, v3scale(rc(33), p11));
        color = v3add(color, v3scale(rc(36), p12));
        color = v3add(color, v3scale(rc(39), p13));
        color = v3add(color, v3scale(rc(42), p14));
        color = v3add(color, v3scale(rc(45), p15));
      }
    }
  }
  return color;
}

// crates/splat-train/src/quant_kernels.rs:789-858 (sh_basis), the same terms
// as kernels/sh.rs:593-671 (sh_coeffs_to_color_vjp).
float sh_basis(uint32_t k, float x, float y, float z) {
  const float z2 = z * z;
  const float fc1 = x * x - y * y;
  const float fs1 = 2.0f * x * y;
  const float fc2 = x * fc1 - y * fs1;
  const float fs2 = x * fs1 + y * fc1;
  const float p6 = 0.9461747f * z2 - 0.31539157f;
  const float p12 = z * (1.8658817f * z2 - 1.119529f);
  const float f0b = -1.0925485f * z;
  const float f0c = -2.285229f * z2 + 0.4570458f;
  const float f1b = 1.4453057f * z;
  const float f2a = -0.5900436f;
  switch (k) {
    case 0: return 0.2820948f;
    case 1: return -0.4886025f * y;
    case 2: return 0.4886025f * z;
    case 3: return -0.4886025f * x;
    case 4: return 0.54627424f * fs1;
    case 5: return f0b * y;
    case 6: return p6;
    case 7: return f0b * x;
    case 8: return 0.54627424f * fc1;
    case 9: return f2a * fs2;
    case 10: return f1b * fs1;
    case 11: return f0c * y;
    case 12: return p12;
    case 13: return f0c * x;
    case 14: return f1b * fc1;
    case 15: return f2a * fc2;
  }
  return 0.0f;
}

// kernels/sh.rs:147-270 (sh_color_viewdir_vjp), bands <= 3
V3 sh_viewdir_vjp(const void* sh, bool half, size_t base, int deg, V3 v, V3 vc) {
  auto sd = [&](size_t k) -> float {
    const V3 c = {sh_coeff(sh, half, base + k), sh_coeff(sh, half, base + k + 1), sh_coeff(sh, half, base + k + 2)};
    return v3dot(c, vc);
  };
  float gx = 0.0f, gy = 0.0f, gz = 0.0f;
  if (deg >= 1) {
    const float f0a = 0.4886025f;
    const float s_n1 = sd(3), s_z0 = sd(6), s_p1 = sd(9);
    gx += -f0a * s_p1;
    gy += -f0a * s_n1;
    gz += f0a * s_z0;
    if (deg >= 2) {
      const float z = v.z, x = v.x, y = v.y;
      const float c2 = -1.0925485f, f1a = 0.54627424f;
      const float s_n2 = sd(12), s_n1b = sd(15), s_z0b = sd(18), s_p1b = sd(21), s_p2 = sd(24);
      gx += 2.0f * f1a * y * s_n2 + c2 * z * s_p1b + 2.0f * f1a * x * s_p2;
      gy += 2.0f * f1a * x * s_n2 + c2 * z * s_n1b - 2.0f * f1a * y * s_p2;
      gz += c2 * y * s_n1b + 2.0f * 0.9461747f * z * s_z0b + c2 * x * s_p1b;
      if (deg >= 3) {
        const float z2 = z * z, x2 = x * x, y2 = y * y;
        const float f2a = -0.5900436f, c1b = 1.4453057f, f1b = c1b * z;
        const float c0c = -2.285229f, f0c = c0c * z2 + 0.4570458f, f0c_dz = 2.0f * c0c * z;
        const float s_n3 = sd(27), s_n2c = sd(30), s_n1c = sd(33), s_z0c = sd(36);
        const float s_p1c = sd(39), s_p2c = sd(42), s_p3 = sd(45);
        const float d12_z = 3.0f * 1.8658817f * z2 - 1.119529f;
        gx += f2a * 6.0f * x * y * s_n3 + 2.0f * f1b * y * s_n2c + f0c * s_p1c + 2.0f * f1b * x * s_p2c +
              f2a * 3.0f * (x2 - y2) * s_p3;
        gy += f2a * 3.0f * (x2 - y2) * s_n3 + 2.0f * f1b * x * s_n2c + f0c * s_n1c + (-2.0f) * f1b * y * s_p2c +
              f2a * (-6.0f) * x * y * s_p3;
        gz += 2.0f * c1b * x * y * s_n2c + f0c_dz * y * s_n1c + d12_z * s_z0c + f0c_dz * x * s_p1c +
              c1b * (x2 - y2) * s_p2c;
      }
    }
  }
  return {gx, gy, gz};
}

// Shared tail of the projection (kernels/project_forward.rs:71-194 and
// kernels/project_visible.rs:114-174): returns false when the splat is culled.
struct ProjOut {
  float xy_x, xy_y;
  S2 conic;
  float opac, power_threshold, depth, radius;
  TileBox box;
  float floor_opac;
  bool floor_reached;  // the floored opacity was written (cull checks up to the raw opacity passed)
};

bool project_one(const float* t, float raw_opac, const float* min_scale, uint32_t g, const Uniforms& u,
                 const RenderCfg& cfg, ProjOut* o) {
  o->floor_reached = false;
  const V3 mean = {t[0], t[1], t[2]};
  const V3 mean_c = world_to_cam(mean, u);
  if (!(v3finite(mean_c) && mean_c.z <= 1.0e10f)) return false;
  if (mean_c.z < 0.01f) return false;
  const V3 scale = read_scale(t, cfg.log_scale_offset);
  if (!v3finite(scale)) return false;
  const Q4 qu = {t[3], t[4], t[5], t[6]};
  const float qn = q4dot(qu);
  if (!(qn >= 1.0e-6f && vs_is_finite(qn))) return false;
  if (!vs_is_finite(raw_opac)) return false;
  const Q4 q = q4scale(qu, 1.0f / sqrtf(qn));
  const Floor fl = apply_scale_floor(scale, vs_sigmoid(raw_opac), min_scale, g, cfg.has_min_scale != 0);
  o->floor_opac = fl.opac;
  o->floor_reached = true;
  const S2 raw = calc_cov2d(fl.scale, q, mean_c, u);
  float comp;
  const S2 cov = compensate_cov2d(raw, cfg.mip != 0, &comp);
  const float opac = fl.opac * comp;
  if (!s2finite(cov)) return false;
  float px, py;
  project_pinhole(mean_c, u, &px, &py);
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
  o->power_threshold = pt;
  o->depth = mean_c.z;
  o->radius = fmaxf(ex / wf, ey / hf);
  o->box = tile_bbox(px, py, ex, ey, u.tbw, u.tbh);
  return true;
}

// kernels/project_visible.rs:26-61 (splat_color): view-dependent colour + 0.5,
// non-finite -> 0, clamped to [-100, 100].
V3 splat_color(const void* sh, bool half, uint32_t g, int deg, V3 mean, const Uniforms& u) {
  const V3 d = v3sub(mean, u.cam);
  const V3 v = v3scale(d, 1.0f / sqrtf(v3dot(d, d)));
  const int nc = (deg + 1) * (deg + 1);
  const V3 raw = sh_to_color(sh, half, (size_t)g * nc * 3, deg, v);
  V3 c = {raw.x + 0.5f, raw.y + 0.5f, raw.z + 0.5f};
  c.x = clampf(vs_is_finite(c.x) ? c.x : 0.0f, -100.0f, 100.0f);
  c.y = clampf(vs_is_finite(c.y) ? c.y : 0.0f, -100.0f, 100.0f);
  c.z = clampf(vs_is_finite(c.z) ? c.z : 0.0f, -100.0f, 100.0f);
  return c;
}

// The rasterizer's per-pixel Gaussian exponent, written with two explicit fmas
// (the kernel uses the same expression): 0.5 c00 dx^2 + c01 dx dy + 0.5 c11 dy^2.
inline float raster_sigma(float h00, float c01, float h11, float dx, float dy) {
  const float t = fmaf(h00, dx, c01 * dy);
  return fmaf(dx, t, (h11 * dy) * dy);
}

// Gaussian taps of the 11x11 SSIM window (sigma 1.5), computed in double and
// rounded once; crates/splat-train-loss/src/lib.rs:50-63.
void gauss_taps(float* w) {
  double t[11], s = 0.0;
  for (int i = 0; i < 11; ++i) {
    const double x = (double)i - 5.0;
    t[i] = exp(-x * x / (2.0 * 1.5 * 1.5));
    s += t[i];
  }
  for (int i = 0; i < 11; ++i) w[i] = (float)(t[i] / s);
}

}  // namespace

// ===========================================================================
// Projection: K1 project_forward + K2 project_visible, with the visible set
// compacted in global order (compact id = rank of the splat among visible
// splats by global index).  Reference: crates/splat-train-render/src/kernels/
// project_forward.rs:26-261, kernels/project_visible.rs:97-174,
// src/render.rs:508-688.
// Outputs:
//  per global splat: compact_from_global (+1, 0 = culled), opacities (the
//  floored sigmoid opacity, 0 when culled early), max_radius, tile_counts;
//  per compact splat: global_from_compact, depths, tile_counts_compact,
//  projected rows [9].
// ===========================================================================
OR_API int or_project(const Camera* cam, const RenderCfg* cfg, uint32_t n, const float* transforms,
                      const void* sh, const float* raw_opac, const float* min_scale,
                      uint32_t* compact_from_global, float* opacities, float* max_radius,
                      uint32_t* tile_counts, uint32_t* global_from_compact, float* depths,
                      uint32_t* tile_counts_compact, float* projected, uint32_t* num_visible,
                      uint64_t* num_isect) {
  const Uniforms u = make_uniforms(*cam);
  std::vector<ProjOut> outs(n);
  std::vector<uint8_t> vis(n, 0);
  std::vector<uint32_t> counts(n, 0);
#pragma omp parallel for schedule(dynamic, 4096)
  for (int64_t gi = 0; gi < (int64_t)n; ++gi) {
    const uint32_t g = (uint32_t)gi;
    ProjOut o;
    const bool v = project_one(transforms + (size_t)g * 10, raw_opac[g], min_scale, g, u, *cfg, &o);
    opacities[g] = o.floor_reached ? o.floor_opac : 0.0f;
    max_radius[g] = v ? o.radius : 0.0f;
    counts[g] = v ? count_tiles(o.box, o.xy_x, o.xy_y, o.conic, o.power_threshold) : 0u;
    tile_counts[g] = counts[g];
    vis[g] = v ? 1 : 0;
    outs[g] = o;
  }
  uint32_t nv = 0;
  uint64_t ni = 0;
  for (uint32_t g = 0; g < n; ++g) {
    if (!vis[g]) {
      compact_from_global[g] = 0;
      continue;
    }
    compact_from_global[g] = nv + 1;
    global_from_compact[nv] = g;
    depths[nv] = outs[g].depth;
    tile_counts_compact[nv] = counts[g];
    ni += counts[g];
    ++nv;
  }
  const int deg = cfg->sh_degree;
  const bool half = cfg->sh_half != 0;
#pragma omp parallel for schedule(static)
  for (int64_t ci = 0; ci < (int64_t)nv; ++ci) {
    const uint32_t g = global_from_compact[ci];
    const ProjOut& o = outs[g];
    const float* t = transforms + (size_t)g * 10;
    const V3 col = splat_color(sh, half, g, deg, {t[0], t[1], t[2]}, u);
    float* p = projected + (size_t)ci * 9;
    p[0] = o.xy_x; p[1] = o.xy_y;
    p[2] = o.conic.c00; p[3] = o.conic.c01; p[4] = o.conic.c11;
    p[5] = o.opac; p[6] = col.x; p[7] = col.y; p[8] = col.z;
  }
  *num_visible = nv;
  *num_isect = ni;
  return 0;
}

// ===========================================================================
// Binning: depth sort (K3), intersection emission in depth order (K4/K5),
// stable tile sort (K6) and tile ranges (K7).
// Reference: src/render.rs:689-810, kernels/map_gaussians.rs:23-174,
// crates/splat-train-sort/src/lib.rs:40-189 (stable LSD radix),
// src/get_tile_offset.rs:11-52.  The order produced is (tile, depth bits,
// compact id), the same as a stable sort on the 64-bit key
// tile << 32 | f32_bits(depth) over compact ids.
// Returns 0, or 2 with *num_isect set when capacity is too small.
// ===========================================================================
OR_API int or_bin(const Camera* cam, uint32_t nv, const float* projected, const float* depths,
                  const uint32_t* tile_counts_compact, uint64_t capacity, uint32_t* depth_order,
                  uint32_t* tile_ids, uint32_t* isect_compact, uint32_t* tile_offsets, uint64_t* num_isect) {
  const Uniforms u = make_uniforms(*cam);
  const uint32_t T = u.tbw * u.tbh;
  std::vector<uint32_t> order(nv);
  std::iota(order.begin(), order.end(), 0u);
  std::stable_sort(order.begin(), order.end(), [&](uint32_t a, uint32_t b) {
    return vs_f2u(depths[a]) < vs_f2u(depths[b]);
  });
  std::vector<uint64_t> offs(nv + 1, 0);
  for (uint32_t i = 0; i < nv; ++i) offs[i + 1] = offs[i] + tile_counts_compact[order[i]];
  const uint64_t total = offs[nv];
  *num_isect = total;
  if (total > capacity) return 2;
  std::vector<uint32_t> tid(total), cid(total);
#pragma omp parallel for schedule(dynamic, 1024)
  for (int64_t si = 0; si < (int64_t)nv; ++si) {
    const uint32_t c = order[si];
    const float* p = projected + (size_t)c * 9;
    const S2 conic = {p[2], p[3], p[4]};
    const float pt = vs_logf(p[5] * 255.0f);
    float ex, ey;
    bbox_extent(conic, pt, &ex, &ey);
    const TileBox b = tile_bbox(p[0], p[1], ex, ey, u.tbw, u.tbh);
    const uint32_t bw = b.x1 - b.x0;
    const uint32_t nb = (b.y1 - b.y0) * bw;
    uint64_t slot = offs[si];
    const uint64_t end = offs[si + 1];
    for (uint32_t i = 0; i < nb && slot < end; ++i) {
      const uint32_t tx = i % bw + b.x0, ty = i / bw + b.y0;
      if (tile_hit(tx, ty, p[0], p[1], conic, pt)) {
        tid[slot] = tx + ty * u.tbw;
        cid[slot] = c;
        ++slot;
      }
    }
    for (; slot < end; ++slot) {  // count drift guard (map_gaussians.rs:105-113)
      tid[slot] = T;
      cid[slot] = c;
    }
  }
  // stable tile sort: counting sort preserves the depth order within a tile
  std::vector<uint64_t> start(T + 2, 0);
  for (uint64_t i = 0; i < total; ++i) start[std::min(tid[i], T) + 1]++;
  for (uint32_t t = 0; t <= T; ++t) start[t + 1] += start[t];
  std::vector<uint64_t> fill(start.begin(), start.end());
  for (uint64_t i = 0; i < total; ++i) {
    const uint32_t t = std::min(tid[i], T);
    const uint64_t at = fill[t]++;
    tile_ids[at] = tid[i];
    isect_compact[at] = cid[i];
  }
  for (uint32_t t = 0; t < T; ++t) {
    const bool empty = start[t] == start[t + 1];
    tile_offsets[2 * t] = empty ? 0u : (uint32_t)start[t];
    tile_offsets[2 * t + 1] = empty ? 0u : (uint32_t)start[t + 1];
  }
  for (uint32_t i = 0; i < nv; ++i) depth_order[i] = order[i];
  return 0;
}

// ===========================================================================
// Rasterize forward, training variant (bwd_info): RGBA f32 output, `visible`
// marks, and the shrink of each tile's range end to one past the last
// intersection any pixel used.  Reference: kernels/rasterize.rs:109-420.
// The Gaussian exponent uses raster_sigma (explicit fmas, as the kernel).
// ===========================================================================
OR_API int or_raster_fwd(const Camera* cam, const float* bg, const float* projected,
                         const uint32_t* global_from_compact, const uint32_t* isect_compact,
                         uint32_t* tile_offsets, float* out_img, float* visible) {
  const Uniforms u = make_uniforms(*cam);
  const uint32_t T = u.tbw * u.tbh;
#pragma omp parallel for schedule(dynamic, 4)
  for (int64_t ti = 0; ti < (int64_t)T; ++ti) {
    const uint32_t tile = (uint32_t)ti;
    const uint32_t tx0 = (tile % u.tbw) * TILE, ty0 = (tile / u.tbw) * TILE;
    const uint32_t lo = tile_offsets[2 * tile], hi = tile_offsets[2 * tile + 1];
    uint32_t max_useful = lo;
    for (uint32_t py = ty0; py < ty0 + TILE; ++py) {
      for (uint32_t px = tx0; px < tx0 + TILE; ++px) {
        if (px >= u.w || py >= u.h) continue;
        const float fx = (float)px + 0.5f, fy = (float)py + 0.5f;
        float t_acc = 1.0f, r = 0.0f, g = 0.0f, b = 0.0f;
        uint32_t last = lo;
        for (uint32_t i = lo; i < hi; ++i) {
          const uint32_t c = isect_compact[i];
          const float* p = projected + (size_t)c * 9;
          const float h00 = 0.5f * p[2], h11 = 0.5f * p[4];
          const float sigma = raster_sigma(h00, p[3], h11, fx - p[0], fy - p[1]);
          const float alpha = fminf(0.999f, p[5] * vs_expf(-sigma));
          if (sigma >= 0.0f && alpha >= ALPHA_MIN) {
            const float next_t = t_acc * (1.0f - alpha);
            if (next_t <= 1.0e-4f) break;
            const uint32_t gid = global_from_compact[c];
#pragma omp atomic write
            visible[gid] = 1.0f;
            const float vis = alpha * t_acc;
            r = fmaf(fmaxf(p[6], 0.0f), vis, r);
            g = fmaf(fmaxf(p[7], 0.0f), vis, g);
            b = fmaf(fmaxf(p[8], 0.0f), vis, b);
            t_acc = next_t;
            last = i + 1;
          }
        }
        max_useful = std::max(max_useful, last);
        float* o = out_img + ((size_t)py * u.w + px) * 4;
        o[0] = fmaf(t_acc, bg[0], r);
        o[1] = fmaf(t_acc, bg[1], g);
        o[2] = fmaf(t_acc, bg[2], b);
        o[3] = 1.0f - t_acc;
      }
    }
    tile_offsets[2 * tile + 1] = max_useful;
  }
  return 0;
}

// ===========================================================================
// Fused L1 + SSIM loss, training forward (partials + per-pixel SSIM
// coefficients) and backward from the coefficients.
// Reference: crates/splat-train-loss/src/lib.rs:238-469 (forward),
// :821-1028 (backward from coefficients), :1227-1257 (l1_dssim weights),
// :1297-1300 (channel weight 1/(3HW)).  Zero padding outside the image; the
// blur sums run in the reference's order.  pred is [H, W, 4]; gt is packed
// RGBA8 [H, W].  partials [3][tiles16] hold weighted per-tile sums in the
// reference's tree order; coeffs [3 ch][3][H*W] hold (dmu1, dsigma1^2,
// dsigma12).
// ===========================================================================
namespace {
inline float gt_chan(const uint32_t* gt, size_t i, uint32_t c) {
  return (float)((gt[i] >> (c * 8)) & 0xffu) * (1.0f / 255.0f);
}
}  // namespace

OR_API int or_loss_fwd(uint32_t h, uint32_t w, const float* pred, const uint32_t* gt, float l1_w, float ssim_w,
                       float* partials, float* coeffs, float* ssim_map) {
  float gw[11];
  gauss_taps(gw);
  const uint32_t tx = (w + 15) / 16, ty = (h + 15) / 16, ntiles = tx * ty;
  const float rgb_weight = 1.0f / (3.0f * (float)(h * w));
  const size_t plane = (size_t)h * w;
  const float C1 = 0.01f * 0.01f, C2 = 0.03f * 0.03f;
  for (uint32_t c = 0; c < 3; ++c) {
    // horizontal pass over every row (zero padded)
    std::vector<float> hs(plane * 5);
#pragma omp parallel for schedule(static)
    for (int64_t yi = 0; yi < (int64_t)h; ++yi) {
      const uint32_t y = (uint32_t)yi;
      for (uint32_t x = 0; x < w; ++x) {
        auto X = [&](int64_t xx) -> float { return (xx < 0 || xx >= (int64_t)w) ? 0.0f : pred[((size_t)y * w + xx) * 4 + c]; };
        auto Y = [&](int64_t xx) -> float { return (xx < 0 || xx >= (int64_t)w) ? 0.0f : gt_chan(gt, (size_t)y * w + xx, c); };
        float sx = 0, sx2 = 0, sy = 0, sy2 = 0, sxy = 0;
        for (int d = 1; d < 6; ++d) {
          const float wd = gw[5 - d];
          const float xl = X((int64_t)x - d), xr = X((int64_t)x + d), yl = Y((int64_t)x - d), yr = Y((int64_t)x + d);
          sx += (xl + xr) * wd;
          sx2 += (xl * xl + xr * xr) * wd;
          sy += (yl + yr) * wd;
          sy2 += (yl * yl + yr * yr) * wd;
          sxy += (xl * yl + xr * yr) * wd;
        }
        const float xc = X(x), yc = Y(x), wc = gw[5];
        sx += xc * wc; sx2 += xc * xc * wc; sy += yc * wc; sy2 += yc * yc * wc; sxy += xc * yc * wc;
        float* o = &hs[((size_t)y * w + x) * 5];
        o[0] = sx; o[1] = sx2; o[2] = sy; o[3] = sy2; o[4] = sxy;
      }
    }
    std::vector<float> loss(plane);
#pragma omp parallel for schedule(static)
    for (int64_t yi = 0; yi < (int64_t)h; ++yi) {
      const uint32_t y = (uint32_t)yi;
      for (uint32_t x = 0; x < w; ++x) {
        auto H = [&](int64_t yy, int k) -> float { return (yy < 0 || yy >= (int64_t)h) ? 0.0f : hs[((size_t)yy * w + x) * 5 + k]; };
        float o[5] = {0, 0, 0, 0, 0};
        for (int d = 1; d < 6; ++d) {
          const float wd = gw[5 - d];
          for (int k = 0; k < 5; ++k) o[k] += (H((int64_t)y - d, k) + H((int64_t)y + d, k)) * wd;
        }
        for (int k = 0; k < 5; ++k) o[k] += H(y, k) * gw[5];
        const float mu1 = o[0], mu2 = o[2];
        const float mu1_sq = mu1 * mu1, mu2_sq = mu2 * mu2;
        const float s1 = fmaxf(0.0f, o[1] - mu1_sq), s2 = fmaxf(0.0f, o[3] - mu2_sq);
        const float s12 = o[4] - mu1 * mu2;
        const float a = mu1_sq + mu2_sq + C1, b = s1 + s2 + C2;
        const float ct = 2.0f * mu1 * mu2 + C1, dt = 2.0f * s12 + C2;
        const float raw = (ct * dt) / (a * b);
        const float val = clampf(raw, -1.0f, 1.0f);
        const float inv_b = 1.0f / b, inv_ab = 1.0f / (a * b);
        const float cd = ct * dt * inv_ab;
        const bool cl = cd < -1.0f || cd > 1.0f;
        const size_t pi = (size_t)y * w + x;
        float* cb = coeffs + (size_t)c * 3 * plane;
        cb[pi] = cl ? 0.0f : 2.0f * inv_ab * (mu2 * (dt - ct) - mu1 * cd * (b - a));
        cb[plane + pi] = cl ? 0.0f : -cd * inv_b;
        cb[2 * plane + pi] = cl ? 0.0f : 2.0f * ct * inv_ab;
        if (ssim_map) ssim_map[pi * 3 + c] = val;
        const float p1 = pred[pi * 4 + c], p2 = gt_chan(gt, pi, c);
        loss[pi] = l1_w * fabsf(p1 - p2) + ssim_w * val;
      }
    }
    // per-tile tree sums (lib.rs:108-123: buf[tid] += buf[tid + stride], stride 128..1)
    for (uint32_t t = 0; t < ntiles; ++t) {
      const uint32_t x0 = (t % tx) * 16, y0 = (t / tx) * 16;
      float buf[256];
      for (uint32_t k = 0; k < 256; ++k) {
        const uint32_t xx = x0 + k % 16, yy = y0 + k / 16;
        buf[k] = (xx < w && yy < h) ? loss[(size_t)yy * w + xx] : 0.0f;
      }
      for (uint32_t stride = 128; stride > 0; stride >>= 1)
        for (uint32_t k = 0; k < stride; ++k) buf[k] += buf[k + stride];
      partials[(size_t)c * ntiles + t] = buf[0] * rgb_weight;
    }
  }
  return 0;
}

OR_API int or_loss_bwd(uint32_t h, uint32_t w, const float* pred, const uint32_t* gt, const float* coeffs,
                       float l1_w, float ssim_w, float* dl_dpred) {
  float gw[11];
  gauss_taps(gw);
  const float rgb_weight = 1.0f / (3.0f * (float)(h * w));
  const size_t plane = (size_t)h * w;
  const float chain = 1.0f * rgb_weight;
  for (uint32_t c = 0; c < 3; ++c) {
    const float* cb = coeffs + (size_t)c * 3 * plane;
    std::vector<float> hs(plane * 3);
#pragma omp parallel for schedule(static)
    for (int64_t yi = 0; yi < (int64_t)h; ++yi) {
      const uint32_t y = (uint32_t)yi;
      for (uint32_t x = 0; x < w; ++x) {
        auto S = [&](int64_t xx, int k) -> float {
          return (xx < 0 || xx >= (int64_t)w) ? 0.0f : cb[k * plane + (size_t)y * w + xx] * chain;
        };
        float a[3] = {0, 0, 0};
        for (int d = 1; d < 6; ++d) {
          const float wd = gw[5 - d];
          for (int k = 0; k < 3; ++k) a[k] += (S((int64_t)x - d, k) + S((int64_t)x + d, k)) * wd;
        }
        for (int k = 0; k < 3; ++k) {
          a[k] += S(x, k) * gw[5];
          hs[((size_t)y * w + x) * 3 + k] = a[k];
        }
      }
    }
#pragma omp parallel for schedule(static)
    for (int64_t yi = 0; yi < (int64_t)h; ++yi) {
      const uint32_t y = (uint32_t)yi;
      for (uint32_t x = 0; x < w; ++x) {
        auto H = [&](int64_t yy, int k) -> float { return (yy < 0 || yy >= (int64_t)h) ? 0.0f : hs[((size_t)yy * w + x) * 3 + k]; };
        float s[3] = {0, 0, 0};
        for (int d = 1; d < 6; ++d) {
          const float wd = gw[5 - d];
          for (int k = 0; k < 3; ++k) s[k] += (H((int64_t)y - d, k) + H((int64_t)y + d, k)) * wd;
        }
        for (int k = 0; k < 3; ++k) s[k] += H(y, k) * gw[5];
        const size_t pi = (size_t)y * w + x;
        const float p1 = pred[pi * 4 + c], g = gt_chan(gt, pi, c);
        const float ssim_grad = s[0] + (2.0f * p1) * s[1] + g * s[2];
        const float diff = p1 - g;
        const float sign = diff > 0.0f ? 1.0f : (diff < 0.0f ? -1.0f : 0.0f);
        dl_dpred[pi * 4 + c] = ssim_w * ssim_grad + l1_w * sign * chain;
      }
    }
  }
  for (size_t pi = 0; pi < plane; ++pi) dl_dpred[pi * 4 + 3] = 0.0f;
  return 0;
}

// ===========================================================================
// Rasterize backward (per-pixel replay, front to back) -> v_combined [V, 10]
// = [xy(2), conic(3), rgb(3), alpha, refine].  Reference:
// src/bwd/kernels/rasterize_backwards_planes.rs:112-682 (gaussian branch,
// :498-602).  Sums are accumulated per splat in double here; the kernel's
// order differs (warp reductions + atomics), so tests use a tolerance.
// ===========================================================================
OR_API int or_raster_bwd(const Camera* cam, const float* bg, uint32_t nv, const float* projected,
                         const uint32_t* isect_compact, const uint32_t* tile_offsets, const float* out_img,
                         const float* v_out, float* v_combined) {
  const Uniforms u = make_uniforms(*cam);
  const uint32_t T = u.tbw * u.tbh;
  std::vector<double> acc((size_t)nv * 10, 0.0);
  const float W = (float)u.w, Hh = (float)u.h;
#pragma omp parallel
  {
    std::vector<double> local((size_t)nv * 10, 0.0);
#pragma omp for schedule(dynamic, 4)
    for (int64_t ti = 0; ti < (int64_t)T; ++ti) {
      const uint32_t tile = (uint32_t)ti;
      const uint32_t tx0 = (tile % u.tbw) * TILE, ty0 = (tile / u.tbw) * TILE;
      const uint32_t lo = tile_offsets[2 * tile], hi = tile_offsets[2 * tile + 1];
      for (uint32_t py = ty0; py < ty0 + TILE; ++py) {
        for (uint32_t px = tx0; px < tx0 + TILE; ++px) {
          if (px >= u.w || py >= u.h) continue;
          const size_t base = ((size_t)py * u.w + px) * 4;
          const float final_a = out_img[base + 3];
          const float t_final = 1.0f - final_a;
          float sr = out_img[base] - t_final * bg[0];
          float sg = out_img[base + 1] - t_final * bg[1];
          float sb = out_img[base + 2] - t_final * bg[2];
          float st = 1.0f;
          const float vr = v_out[base], vg = v_out[base + 1], vb = v_out[base + 2];
          const float vt = (v_out[base + 3] - (bg[0] * vr + bg[1] * vg + bg[2] * vb)) * t_final;
          const float rscale = 1.0f / fmaxf(final_a, 1.0e-5f);
          const float fx = (float)px + 0.5f, fy = (float)py + 0.5f;
          for (uint32_t i = lo; i < hi; ++i) {
            const uint32_t c = isect_compact[i];
            const float* p = projected + (size_t)c * 9;
            const float dx = p[0] - fx, dy = p[1] - fy;
            const float sigma = raster_sigma(0.5f * p[2], p[3], 0.5f * p[4], dx, dy);
            const float gauss = vs_expf(-sigma);
            const float alpha = fminf(0.999f, p[5] * gauss);
            if (!(sigma >= 0.0f && alpha >= ALPHA_MIN)) continue;
            const float next_t = st * (1.0f - alpha);
            if (next_t <= 1.0e-4f) break;
            const float cr = fmaxf(p[6], 0.0f), cg = fmaxf(p[7], 0.0f), cbb = fmaxf(p[8], 0.0f);
            const float vis = alpha * st;
            double* a = &local[(size_t)c * 10];
            if (p[6] >= 0.0f) a[5] += vis * vr;
            if (p[7] >= 0.0f) a[6] += vis * vg;
            if (p[8] >= 0.0f) a[7] += vis * vb;
            // The reference's expressions (rasterize_backwards_planes.rs:560-595)
            // with the multiply-adds fused as written below; the kernel uses the
            // same fmas, so every per-pixel term matches it bit for bit.
            const float ra = 1.0f / (1.0f - alpha);
            const float dot = fmaf(fmaf(st, cr, -sr), vr, fmaf(fmaf(st, cg, -sg), vg, fmaf(st, cbb, -sb) * vb)) * ra;
            const float v_alpha = fmaf(vt, ra, dot);
            const float v_sigma = -alpha * v_alpha;
            const float vxx = v_sigma * fmaf(p[2], dx, p[3] * dy);
            const float vxy = v_sigma * fmaf(p[3], dx, p[4] * dy);
            if (p[5] * gauss <= 0.999f) {
              a[2] += 0.5f * v_sigma * dx * dx;
              a[3] += v_sigma * dx * dy;
              a[4] += 0.5f * v_sigma * dy * dy;
              a[0] += vxx;
              a[1] += vxy;
              a[8] += v_alpha * gauss;
              const float ax = vxx * W, ay = vxy * Hh;
              a[9] += sqrtf(fmaf(ax, ax, ay * ay)) * rscale;
            }
            sr = fmaf(-vis, cr, sr);
            sg = fmaf(-vis, cg, sg);
            sb = fmaf(-vis, cbb, sb);
            st = next_t;
          }
        }
      }
    }
#pragma omp critical
    for (size_t i = 0; i < acc.size(); ++i) acc[i] += local[i];
  }
  for (size_t i = 0; i < acc.size(); ++i) v_combined[i] = (float)acc[i];
  return 0;
}

// ===========================================================================
// Projection VJP for one visible splat.  Reference:
// src/bwd/kernels/project_backwards.rs:20-274 (apply_normalize_vjp,
// quat_to_mat_vjp, inverse2x2_vjp, splat_vjp),
// kernels/camera_model/pinhole.rs:179-245 (calculate_projection_vjp_pinhole).
// Returns the transforms gradient [10] and raw-opacity gradient; writes the
// view direction (the SH gradient is Y_k(dir) * v_color).
// ===========================================================================
namespace {
Q4 normalize_vjp(Q4 q, Q4 g) {
  const float lsq = q4dot(q);
  const float l = sqrtf(lsq);
  const float inv = 1.0f / (l * lsq);
  const float cc0 = -q.w * q.x, cc1 = -q.x * q.y, cc2 = -q.y * q.w;
  const float cs0 = -q.w * q.z, cs1 = -q.x * q.z, cs2 = -q.y * q.z;
  const float qw2 = q.w * q.w, qx2 = q.x * q.x, qy2 = q.y * q.y, qz2 = q.z * q.z;
  return {((lsq - qw2) * g.w + cc0 * g.x + cc2 * g.y + cs0 * g.z) * inv,
          (cc0 * g.w + (lsq - qx2) * g.x + cc1 * g.y + cs1 * g.z) * inv,
          (cc2 * g.w + cc1 * g.x + (lsq - qy2) * g.y + cs2 * g.z) * inv,
          (cs0 * g.w + cs1 * g.x + cs2 * g.y + (lsq - qz2) * g.z) * inv};
}
Q4 quat_to_mat_vjp(Q4 q, const M3& v) {
  const float wg = q.x * (v.c1z - v.c2y) + q.y * (v.c2x - v.c0z) + q.z * (v.c0y - v.c1x);
  const float xg = -2.0f * q.x * (v.c1y + v.c2z) + q.y * (v.c0y + v.c1x) + q.z * (v.c0z + v.c2x) + q.w * (v.c1z - v.c2y);
  const float yg = q.x * (v.c0y + v.c1x) - 2.0f * q.y * (v.c0x + v.c2z) + q.z * (v.c1z + v.c2y) + q.w * (v.c2x - v.c0z);
  const float zg = q.x * (v.c0z + v.c2x) + q.y * (v.c1z + v.c2y) - 2.0f * q.z * (v.c0x + v.c1y) + q.w * (v.c0y - v.c1x);
  return {2.0f * wg, 2.0f * xg, 2.0f * yg, 2.0f * zg};
}
S2 inverse2x2_vjp(S2 m, S2 v) {
  const float t00 = -m.c00 * v.c00 + -m.c01 * v.c01;
  const float t01 = -m.c01 * v.c00 + -m.c11 * v.c01;
  const float t10 = -m.c00 * v.c01 + -m.c01 * v.c11;
  const float t11 = -m.c01 * v.c01 + -m.c11 * v.c11;
  return {t00 * m.c00 + t10 * m.c01, t01 * m.c00 + t11 * m.c01, t01 * m.c01 + t11 * m.c11};
}
V3 projection_vjp_pinhole(const M23& J, V3 mc, S3 cov_c, const Uniforms& u, S2 v_cov2d, V2 v_mean2d) {
  const float fx = u.fx, fy = u.fy;
  const float mx = mc.x, my = mc.y, mz = mc.z;
  const float inv_z = 1.0f / mz;
  const float rx = mx * inv_z, ry = my * inv_z;
  const float cx = clampf(rx, u.lim_neg_x, u.lim_pos_x), cy = clampf(ry, u.lim_neg_y, u.lim_pos_y);
  const bool in_x = rx <= u.lim_pos_x && rx >= u.lim_neg_x;
  const bool in_y = ry <= u.lim_pos_y && ry >= u.lim_neg_y;
  const float iz2 = inv_z * inv_z, iz3 = iz2 * inv_z;
  float vmx = fx * inv_z * v_mean2d.x;
  float vmy = fy * inv_z * v_mean2d.y;
  float vmz = -(fx * mx * v_mean2d.x + fy * my * v_mean2d.y) * iz2;
  const M23 tmp = s2mulm23(v_cov2d, J);
  const float vj00 = 2.0f * v3dot(m23row0(tmp), s3row0(cov_c));
  const float vj11 = 2.0f * v3dot(m23row1(tmp), s3row1(cov_c));
  const float vj20 = 2.0f * v3dot(m23row0(tmp), s3row2(cov_c));
  const float vj21 = 2.0f * v3dot(m23row1(tmp), s3row2(cov_c));
  const float tx = mz * cx, ty = mz * cy;
  if (in_x) vmx += -fx * iz2 * vj20; else vmz += -fx * iz3 * vj20 * tx;
  if (in_y) vmy += -fy * iz2 * vj21; else vmz += -fy * iz3 * vj21 * ty;
  vmz += -fx * iz2 * vj00 - fy * iz2 * vj11 + 2.0f * fx * tx * iz3 * vj20 + 2.0f * fy * ty * iz3 * vj21;
  return {vmx, vmy, vmz};
}

struct VjpOut { V3 v_mean; Q4 v_q; V3 v_scale; float v_raw; V3 dir; };

VjpOut splat_vjp(const float* t, float raw_opac, const void* sh, bool half, int deg, const float* min_scale, uint32_t g,
                 const float* rg, const Uniforms& u, const RenderCfg& cfg) {
  const V3 mean = {t[0], t[1], t[2]};
  const V3 scale_raw = read_scale(t, cfg.log_scale_offset);
  const Q4 qu = {t[3], t[4], t[5], t[6]};
  const float v_mean2d_x = rg[0], v_mean2d_y = rg[1];
  const S2 v_inv = {rg[2], rg[3] * 0.5f, rg[4]};
  const V3 v_color = {rg[5], rg[6], rg[7]};
  const float v_alpha_in = rg[8];
  const Q4 quat = q4scale(qu, 1.0f / sqrtf(q4dot(qu)));
  const float opac_sig = vs_sigmoid(raw_opac);
  const Floor fl = apply_scale_floor(scale_raw, opac_sig, min_scale, g, cfg.has_min_scale != 0);
  const V3 scale = fl.scale;
  const V3 uw = v3sub(mean, u.cam);
  const float ulen = sqrtf(v3dot(uw, uw));
  const V3 v = v3scale(uw, 1.0f / ulen);
  const int nc = (deg + 1) * (deg + 1);
  const V3 v_v_sh = sh_viewdir_vjp(sh, half, (size_t)g * nc * 3, deg, v, v_color);
  const float vdv = v3dot(v, v_v_sh);
  const V3 v_mean_sh = v3scale(v3sub(v_v_sh, v3scale(v, vdv)), 1.0f / ulen);
  const V3 mean_c = world_to_cam(mean, u);
  const M3 r = quat_to_mat3(quat);
  const M3 m = m3diag(r, scale);
  const S2 raw_cov = calc_cov2d(scale, quat, mean_c, u);
  float comp;
  const S2 cov = compensate_cov2d(raw_cov, cfg.mip != 0, &comp);
  const float v_opac_base = fl.opac_open ? comp * v_alpha_in : 0.0f;
  const S2 conic_inv = s2inverse(cov);
  const S2 v_cov2d = inverse2x2_vjp(conic_inv, v_inv);
  const S3 covar = m3outer_self(m);
  const S3 cov_c = s3cong(covar, u.rot);
  const M23 J = pinhole_jacobian(mean_c, u);
  const V3 v_mean_c = projection_vjp_pinhole(J, mean_c, cov_c, u, v_cov2d, {v_mean2d_x, v_mean2d_y});
  const S3 vcc = m23tcong(J, v_cov2d);
  const V3 v_mean = v3add(m3tmulv(u.rot, v_mean_c), v_mean_sh);
  const M3 v_m = s3mulm3(s3scale(s3tcong(vcc, u.rot), 2.0f), m);
  const V3 vlf = {v3dot(m3col0(r), m3col0(v_m)) * scale.x, v3dot(m3col1(r), m3col1(v_m)) * scale.y,
                  v3dot(m3col2(r), m3col2(v_m)) * scale.z};
  const V3 vse = {vlf.x * fl.ratio_sq.x + v_opac_base * fl.opac * (1.0f - fl.ratio_sq.x),
                  vlf.y * fl.ratio_sq.y + v_opac_base * fl.opac * (1.0f - fl.ratio_sq.y),
                  vlf.z * fl.ratio_sq.z + v_opac_base * fl.opac * (1.0f - fl.ratio_sq.z)};
  const Q4 qg = quat_to_mat_vjp(quat, m3diag(v_m, scale));
  const Q4 vq = normalize_vjp(qu, qg);
  const float v_raw = v_opac_base * fl.coef * opac_sig * (1.0f - opac_sig);
  return {v_mean, vq, vse, v_raw, v};
}

// Packed geometry/opacity moments: src/bwd/kernels/geo_moments.rs:26-96.
constexpr float GEO_U_MAX = 8.0f, GEO_U_CODES = 32767.0f;
constexpr float GEO_U_STEP = GEO_U_MAX / GEO_U_CODES, GEO_U_PER_UNIT = GEO_U_CODES / GEO_U_MAX;
constexpr float GEO_L_MAX = 64.0f, GEO_L_CODES = 65535.0f;
constexpr float GEO_L_STEP = GEO_L_MAX / GEO_L_CODES, GEO_L_PER_UNIT = GEO_L_CODES / GEO_L_MAX;

inline float geo_growth(uint32_t w) { return vs_expf((float)(w >> 16) * GEO_L_STEP); }
inline float geo_normalized(uint32_t w) {
  const float mag = (float)(w & 0x7fffu) * GEO_U_STEP;
  return (w & 0x8000u) ? -mag : mag;
}
inline uint32_t pack_geo(float m, float v, float eps, float rl, float ru) {
  const float l = vs_logf(1.0f + sqrtf(fmaxf(v, 0.0f)) / eps) * GEO_L_PER_UNIT;
  const float l_code = floorf(clampf(l + rl, 0.0f, GEO_L_CODES));
  const float scale = eps * vs_expf(l_code * GEO_L_STEP);
  const float uu = fabsf(m) / scale * GEO_U_PER_UNIT;
  const uint32_t u_code = (uint32_t)floorf(clampf(uu + ru, 0.0f, GEO_U_CODES));
  const uint32_t sign = m < 0.0f ? 0x8000u : 0u;
  return ((uint32_t)l_code << 16) | sign | u_code;
}
void adam_packed(float* params, uint32_t* words, size_t index, float g, float lr, float b1, float b2, float inv1,
                 float inv2, float eps, uint32_t seed) {
  const uint32_t word = words[index];
  const float growth = geo_growth(word);
  const float root = eps * (growth - 1.0f);
  const float m1 = geo_normalized(word) * (eps * growth) * b1 + g * (1.0f - b1);
  const float v1 = root * root * b2 + g * g * (1.0f - b2);
  const float step = (m1 * inv1) / (sqrtf(v1 * inv2) + eps);
  params[index] = params[index] - step * lr;
  const uint32_t hsh = vs_mix_hash((uint32_t)index, seed);
  words[index] = pack_geo(m1, v1, eps, (float)(hsh >> 16) / 65536.0f, (float)(hsh & 0xffffu) / 65536.0f);
}
}  // namespace

// ===========================================================================
// Fused projection VJP + packed-moment Adam for transforms and opacity
// (reference mode).  Reference: src/bwd/kernels/project_update.rs:36-178.
// color_dir is [N+1, 6] (row 0 zero); rows past the visible count are not
// written.
// ===========================================================================
OR_API int or_project_update(const Camera* cam, const RenderCfg* cfg, uint32_t n, float* transforms, const void* sh,
                             float* raw_opac, const float* min_scale, const uint32_t* compact_from_global,
                             const float* v_combined, uint32_t* w_t, const float* lr_scale, uint32_t* w_o,
                             float* color_dir, float* v_refine, float* grad_sq, float b1, float b2, float inv1,
                             float inv2, float eps, float lr_opac, float opac_reg, uint32_t round_seed) {
  const Uniforms u = make_uniforms(*cam);
  const bool half = cfg->sh_half != 0;
  for (int k = 0; k < 6; ++k) color_dir[k] = 0.0f;
#pragma omp parallel for schedule(static)
  for (int64_t gi = 0; gi < (int64_t)n; ++gi) {
    const uint32_t g = (uint32_t)gi;
    float gr[10] = {0, 0, 0, 0, 0, 0, 0, 0, 0, 0};
    float g_opac = 0.0f, refine = 0.0f, gsq = 0.0f;
    const uint32_t row = compact_from_global[g];
    if (row > 0) {
      const float* rg = v_combined + (size_t)(row - 1) * 10;
      bool any = false;
      for (int k = 0; k < 10; ++k) any = any || rg[k] != 0.0f;
      float* cd = color_dir + (size_t)row * 6;
      if (any) {
        const VjpOut o = splat_vjp(transforms + (size_t)g * 10, raw_opac[g], sh, half, cfg->sh_degree, min_scale, g, rg,
                                   u, *cfg);
        cd[0] = rg[5]; cd[1] = rg[6]; cd[2] = rg[7];
        cd[3] = o.dir.x; cd[4] = o.dir.y; cd[5] = o.dir.z;
        gr[0] = o.v_mean.x; gr[1] = o.v_mean.y; gr[2] = o.v_mean.z;
        gr[3] = o.v_q.w; gr[4] = o.v_q.x; gr[5] = o.v_q.y; gr[6] = o.v_q.z;
        gr[7] = o.v_scale.x; gr[8] = o.v_scale.y; gr[9] = o.v_scale.z;
        g_opac = o.v_raw;
        const float ri = rg[9];
        refine = clampf(vs_is_finite(ri) ? ri : 0.0f, 0.0f, 1.0e32f);
        const float c0 = SH_C0 * cd[0], c1 = SH_C0 * cd[1], c2 = SH_C0 * cd[2];
        gsq = (c0 * c0 + c1 * c1 + c2 * c2) / 3.0f;
      } else {
        for (int k = 0; k < 6; ++k) cd[k] = 0.0f;
      }
    }
    v_refine[g] = refine;
    grad_sq[g] = gsq;
    const float o = 1.0f / (1.0f + vs_expf(-raw_opac[g]));
    g_opac += opac_reg * o * (1.0f - o);
    const uint32_t seed_t = round_seed ^ (10u << 24), seed_o = round_seed ^ (1u << 24);
    for (int k = 0; k < 10; ++k)
      adam_packed(transforms, w_t, (size_t)g * 10 + k, gr[k], lr_scale[k], b1, b2, inv1, inv2, eps, seed_t);
    adam_packed(raw_opac, w_o, g, g_opac, lr_opac, b1, b2, inv1, inv2, eps, seed_o);
  }
  return 0;
}

// ===========================================================================
// SH Adam step, reference mode: f16 coefficients stepped with stochastic
// rounding, 8-bit block-scaled first moment (block 128, +128-biased codes,
// absmax/127 scale), reduced f32 second moment per splat, lazy on culled rows.
// Reference: crates/splat-train/src/quant_kernels.rs:597-714 (step_kernel_w4),
// :860-890 (stochastic_half); crates/splat-train/src/optim.rs:414-503
// (variance update, coefficients).  `variance` must already hold this step's
// reduced second moment.  Codes are rounded half to even (WGSL round()).
// ===========================================================================
namespace {
float stochastic_half(float value, uint32_t index, uint32_t step) {
  const float mag = fabsf(value);
  float result = value;
  if (mag <= 65504.0f) {
    float lower, upper;
    if (mag < 0.00006103515625f) {
      lower = floorf(mag * 16777216.0f) / 16777216.0f;
      upper = lower + 0.000000059604644775390625f;
    } else {
      const uint32_t bits = vs_f2u(mag) & 0xffffe000u;
      lower = vs_u2f(bits);
      upper = vs_u2f(bits + 8192u);
    }
    const uint32_t hsh = vs_mix_hash(index, step);
    const float uni = (float)(hsh >> 8) / 16777216.0f;
    const float prob = (mag - lower) / (upper - lower);
    result = uni < prob ? upper : lower;
    if (value < 0.0f) result = -result;
  }
  return result;
}
}  // namespace

OR_API int or_sh_step_ref(uint32_t n, uint32_t row_width, uint16_t* params, const float* color_dir,
                          const uint32_t* grad_rows, uint32_t* codes, float* scales, const float* variance,
                          const float* lr_scale, float beta, float factor, float inv1, float inv2, float eps, float lr,
                          uint32_t round_seed) {
  const size_t count = (size_t)n * row_width;
  const size_t blocks = (count + 127) / 128;
#pragma omp parallel for schedule(static)
  for (int64_t bi = 0; bi < (int64_t)blocks; ++bi) {
    const size_t b0 = (size_t)bi * 128;
    bool any = false;
    for (size_t i = b0; i < b0 + 128 && i < count; ++i) any = any || grad_rows[i / row_width] != 0;
    if (!any) continue;
    const float old_scale = scales[bi];
    float m[128];
    for (size_t j = 0; j < 128; ++j) {
      const size_t i = b0 + j;
      const uint32_t code = (codes[i / 4] >> ((i % 4) * 8)) & 255u;
      m[j] = i < count ? ((float)code - 128.0f) * old_scale : 0.0f;
    }
    for (size_t j = 0; j < 128; ++j) {
      const size_t i = b0 + j;
      if (i >= count) continue;
      const size_t row = i / row_width, col = i % row_width;
      const uint32_t gr = grad_rows[row];
      if (gr == 0) continue;
      const float* cd = color_dir + (size_t)gr * 6;
      const float basis = sh_basis((uint32_t)(col / 3), cd[3], cd[4], cd[5]);
      const float gg = basis * cd[col % 3];
      const float moment = m[j] * beta + gg * factor;
      const float denom = sqrtf(variance[row] * inv2) + eps;
      const float delta = (moment * inv1 / denom) * (lr_scale[col] * lr);
      float updated = vs_f16_to_f32(params[i]) - delta;
      updated = stochastic_half(updated, (uint32_t)i, round_seed);
      params[i] = vs_f32_to_f16(updated);
      m[j] = moment;
    }
    float absmax = 0.0f;
    for (size_t j = 0; j < 128; ++j) absmax = fmaxf(absmax, fabsf(m[j]));
    const float scale = absmax / 127.0f;
    scales[bi] = scale;
    for (size_t wv = 0; wv < 32; ++wv) {
      uint32_t packed = 0;
      for (size_t j = 0; j < 4; ++j) {
        uint32_t code = 128;
        if (scale > 0.0f) code = (uint32_t)(rintf(clampf(m[wv * 4 + j] / scale, -127.0f, 127.0f)) + 128.0f);
        packed |= code << (j * 8);
      }
      codes[b0 / 4 + wv] = packed;
    }
  }
  return 0;
}

// ===========================================================================
// Dense projection VJP (multi-view / unfused path): accumulates the
// gradient rows of every visible splat into grads [N, 59] =
// [transforms 10 | sh 48 (coefficient-major, rgb) | raw opacity 1], and the
// refine weight into refine [N].  Reference: src/bwd/kernels/
// project_backwards.rs:282-424 (project_backwards_kernel) with
// kernels/sh.rs:593-671 (sh_coeffs_to_color_vjp), gathered to dense rows as
// src/bwd/burn_glue.rs:363-395 does.  Splats whose raster gradient row is all
// zero contribute nothing (project_backwards.rs:360-382).
// ===========================================================================
OR_API int or_vjp_dense(const Camera* cam, const RenderCfg* cfg, uint32_t n, const float* transforms, const void* sh,
                        const float* raw_opac, const float* min_scale, const uint32_t* compact_from_global,
                        const float* v_combined, float* grads, float* refine) {
  const Uniforms u = make_uniforms(*cam);
  const bool half = cfg->sh_half != 0;
  const int deg = cfg->sh_degree;
  const int nc = (deg + 1) * (deg + 1);
  const int width = 10 + nc * 3 + 1;
#pragma omp parallel for schedule(static)
  for (int64_t gi = 0; gi < (int64_t)n; ++gi) {
    const uint32_t g = (uint32_t)gi;
    const uint32_t row = compact_from_global[g];
    if (row == 0) continue;
    const float* rg = v_combined + (size_t)(row - 1) * 10;
    bool any = false;
    for (int k = 0; k < 10; ++k) any = any || rg[k] != 0.0f;
    if (!any) continue;
    const VjpOut o = splat_vjp(transforms + (size_t)g * 10, raw_opac[g], sh, half, deg, min_scale, g, rg, u, *cfg);
    float* d = grads + (size_t)g * width;
    const float gv[10] = {o.v_mean.x, o.v_mean.y, o.v_mean.z, o.v_q.w, o.v_q.x, o.v_q.y, o.v_q.z,
                          o.v_scale.x, o.v_scale.y, o.v_scale.z};
    for (int k = 0; k < 10; ++k) d[k] += gv[k];
    for (int k = 0; k < nc; ++k) {
      const float bsis = sh_basis((uint32_t)k, o.dir.x, o.dir.y, o.dir.z);
      for (int c = 0; c < 3; ++c) d[10 + k * 3 + c] += rg[5 + c] * bsis;
    }
    d[width - 1] += o.v_raw;
    const float ri = rg[9];
    refine[g] += clampf(vs_is_finite(ri) ? ri : 0.0f, 0.0f, 1.0e32f);
  }
  return 0;
}

// ===========================================================================
// Adam with 8-bit block-quantized first AND second moments (the benchmark
// configurations' "Q8" optimizer; no reference counterpart, defined by this
// project):
//  * blocks of 256 consecutive values of one parameter tensor;
//  * m: signed codes (+128 bias), scale = absmax|m| / 127;
//  * v: sqrt(v) as unsigned codes, scale = absmax sqrt(v) / 255;
//  * both re-encoded with stochastic rounding: h = vs_mix_hash(index / 2,
//    step ^ salt); value index i takes the bytes 2 (i % 2) and 2 (i % 2) + 1
//    of h as b_m, b_v and uniforms u = (b + 1/2) / 256:
//    m code = floor(m/scale + u1), r code = floor(r/scale + u2);
//  * scales enter as reciprocals: code = floor(fma(m, 1/scale, u));
//  * m1 = fma(g, 1 - b1, m0 b1), v1 = fma(g g, 1 - b2, r0 r0 b2),
//    p1 = fma(-(m1 inv1) (1 / d), lr, p0), d = max(fma(sqrt(v1), sqrt(inv2),
//    eps), |m1 inv1| / 8), with 1 / d taken as 0 for d >= 2^126: the normalized
//    update is bounded by 8, the bound the reference's packed geometry codec
//    imposes (src/bwd/kernels/geo_moments.rs:186,192).
// grads [count] (dense); lr per column: lr_col[index % row_width] * lr.
// Optional weight decay of zero gradients is not applied (dense Adam).
// ===========================================================================
OR_API int or_adam_q8(size_t count, uint32_t row_width, float* params, const float* grads, size_t grad_stride,
                      size_t grad_offset, uint8_t* m_codes, uint8_t* v_codes, float* m_scales, float* v_scales,
                      const float* lr_col, float lr, float b1, float b2, float inv1, float inv2, float eps,
                      uint32_t seed) {
  const size_t blocks = (count + 255) / 256;
  const float sqrt_inv2 = sqrtf(inv2);
#pragma omp parallel for schedule(static)
  for (int64_t bi = 0; bi < (int64_t)blocks; ++bi) {
    const size_t b0 = (size_t)bi * 256;
    const size_t nb = std::min<size_t>(256, count - b0);
    float m1[256], r1[256];
    const float ms = m_scales[bi], vsc = v_scales[bi];
    for (size_t j = 0; j < nb; ++j) {
      const size_t i = b0 + j;
      const size_t row = i / row_width, col = i % row_width;
      const float g = grads[row * grad_stride + grad_offset + col];
      const float m0 = ((float)m_codes[i] - 128.0f) * ms;
      const float r0 = (float)v_codes[i] * vsc;
      const float m = fmaf(g, 1.0f - b1, m0 * b1);
      const float v = fmaf(g * g, 1.0f - b2, r0 * r0 * b2);
      const float r = sqrtf(v);
      const float mh = m * inv1;
      const float denom = fmaxf(fmaf(r, sqrt_inv2, eps), fabsf(mh) * 0.125f);
      const float inv_d = denom < 8.5070592e37f ? 1.0f / denom : 0.0f;
      params[i] = fmaf(-(mh * inv_d), lr_col[col] * lr, params[i]);
      m1[j] = m;
      r1[j] = r;
    }
    float am = 0.0f, ar = 0.0f;
    for (size_t j = 0; j < nb; ++j) {
      am = fmaxf(am, fabsf(m1[j]));
      ar = fmaxf(ar, r1[j]);
    }
    const float nms = am / 127.0f, nvs = ar / 255.0f;
    const float inv_ms = nms > 0.0f ? 1.0f / nms : 0.0f, inv_vs = nvs > 0.0f ? 1.0f / nvs : 0.0f;
    m_scales[bi] = nms;
    v_scales[bi] = nvs;
    for (size_t j = 0; j < nb; ++j) {
      const size_t i = b0 + j;
      const uint32_t hb = vs_mix_hash((uint32_t)(i >> 1), seed) >> (16 * (i & 1));
      const float u1 = ((float)(hb & 0xffu) + 0.5f) * (1.0f / 256.0f);
      const float u2 = ((float)((hb >> 8) & 0xffu) + 0.5f) * (1.0f / 256.0f);
      float qm = 0.0f, qr = 0.0f;
      if (nms > 0.0f) qm = clampf(floorf(fmaf(m1[j], inv_ms, u1)), -127.0f, 127.0f);
      if (nvs > 0.0f) qr = clampf(floorf(fmaf(r1[j], inv_vs, u2)), 0.0f, 255.0f);
      m_codes[i] = (uint8_t)((int32_t)qm + 128);
      v_codes[i] = (uint8_t)qr;
    }
  }
  return 0;
}

// ===========================================================================
// Housekeeping.  Reference: crates/splat-train/src/housekeep.rs:107-160.
// noise: N(0,1) (Box-Muller from hashed uniforms) * clamp((1-o)^150, 0, 1) *
// visible * scale, clamped to +-limit, added to the mean columns.  (1-o)^150
// is evaluated as exp(150 ln(1-o)) with the shared functions, sin/cos with
// vs_sincosf.
// ===========================================================================
OR_API int or_gather_stats(uint32_t n, float* norm, float* vis, float* screen, const float* weight,
                           const float* visible, const float* radius) {
  for (uint32_t i = 0; i < n; ++i) {
    norm[i] = fmaxf(norm[i], weight[i]);
    vis[i] += visible[i];
    screen[i] = fmaxf(screen[i], radius[i]);
  }
  return 0;
}

namespace {
inline float hash_uniform(uint32_t key, uint32_t seed) {
  const uint32_t h = vs_mix_hash(key, seed);
  return (float)((h >> 8) + 1u) / 16777216.0f;
}
}  // namespace

OR_API int or_noise_means(uint32_t n, float* transforms, const float* opacities, const float* visible, float scale,
                          float limit, uint32_t seed) {
  for (uint32_t i = 0; i < n; ++i) {
    const float om = 1.0f - opacities[i];
    const float pw = om > 0.0f ? vs_expf(150.0f * vs_logf(om)) : 0.0f;
    const float gate = clampf(pw, 0.0f, 1.0f) * fminf(visible[i], 1.0f);
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
      float* t = transforms + (size_t)i * 10;
      t[0] += clampf(r1 * c1 * w, -limit, limit);
      t[1] += clampf(r1 * s1 * w, -limit, limit);
      t[2] += clampf(r2 * c2 * w, -limit, limit);
    }
  }
  return 0;
}

// Seeded Fisher-Yates shuffle of 0..n-1 driven by splitmix64, the generator of
// the reference's >67M-key sort regression test
// (crates/splat-train-sort/src/lib.rs:358-404).
OR_API void or_splitmix_shuffle(uint32_t* keys, uint64_t n, uint64_t seed) {
  for (uint64_t i = 0; i < n; ++i) keys[i] = (uint32_t)i;
  uint64_t state = seed;
  for (uint64_t i = n - 1; i >= 1; --i) {
    state += 0x9E3779B97F4A7C15ull;
    uint64_t z = state;
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    z ^= z >> 31;
    const uint64_t j = z % (i + 1);
    const uint32_t t = keys[i];
    keys[i] = keys[j];
    keys[j] = t;
  }
}

// Elementary-function probes for the tests.
OR_API void or_expf_batch(const float* x, float* y, size_t n) {
  for (size_t i = 0; i < n; ++i) y[i] = vs_expf(x[i]);
}
OR_API void or_logf_batch(const float* x, float* y, size_t n) {
  for (size_t i = 0; i < n; ++i) y[i] = vs_logf(x[i]);
}
OR_API void or_f16_batch(const float* x, uint16_t* h, float* back, size_t n) {
  for (size_t i = 0; i < n; ++i) {
    h[i] = vs_f32_to_f16(x[i]);
    back[i] = vs_f16_to_f32(h[i]);
  }
}

// ===========================================================================
// Refinement.  Reference: crates/splat-train/src/train.rs:1822-1883 (the
// per-splat decision table), :2142-2252 (refine_splats: the split of each
// parent into itself and a child), :2259-2283 (filler rows), :2285-2296
// (opacity decay), crates/splat-train/src/quat_vec.rs (rotating the offset).
// ===========================================================================
OR_API int or_refine_table(uint32_t n, const float* transforms, const float* sh, uint32_t sh_width,
                           const float* raw_opac, const float* refine_weight, const float* vis_weight,
                           const float* max_screen, float min_opacity, float max_bound, const float* center,
                           float split_at_screen_size, float* table) {
  for (uint32_t g = 0; g < n; ++g) {
    const float* t = transforms + (size_t)g * 10;
    bool finite = vs_is_finite(raw_opac[g]);
    for (int k = 0; k < 10; ++k) finite = finite && vs_is_finite(t[k]);
    for (uint32_t k = 0; k < sh_width; ++k) finite = finite && vs_is_finite(sh[(size_t)g * sh_width + k]);
    const float opac = vs_sigmoid(raw_opac[g]);
    bool big = false, far = false;
    for (int k = 0; k < 3; ++k) {
      if (vs_expf(t[7 + k]) > max_bound) big = true;
      if (fabsf(t[k] - center[k]) > max_bound) far = true;
    }
    const float vis = vis_weight[g] > 0.0f ? 1.0f : 0.0f;
    float* row = table + (size_t)g * 8;
    row[0] = (opac < min_opacity || big || far || !finite) ? 1.0f : 0.0f;
    row[1] = finite ? 0.0f : 1.0f;
    row[2] = opac * vis;
    row[3] = (split_at_screen_size > 0.0f && max_screen[g] > split_at_screen_size && vis > 0.0f) ? 1.0f : 0.0f;
    row[4] = refine_weight[g] * vis;
    row[5] = t[0];
    row[6] = t[1];
    row[7] = t[2];
  }
  return 0;
}

OR_API int or_refine_split(float* transforms, float* sh, uint32_t sh_width, float* raw_opac, uint32_t count,
                           const int32_t* parents, const int32_t* children, const float* screen,
                           float split_at_screen_size, float min_opacity, uint32_t empty_count,
                           const int32_t* empty_rows) {
  const float r2 = 0.70710678118654752440f;  // 1/sqrt(2)
  for (uint32_t i = 0; i < count; ++i) {
    const size_t p = (size_t)parents[i], c = (size_t)children[i];
    float t[10];
    memcpy(t, transforms + p * 10, sizeof(t));
    // cur_rots = raw / max(|raw|, 1e-32)
    const float norm = sqrtf(((t[3] * t[3] + t[4] * t[4]) + t[5] * t[5]) + t[6] * t[6]);
    const float mag = fmaxf(norm, 1.0e-32f);
    const float q[4] = {t[3] / mag, t[4] / mag, t[5] / mag, t[6] / mag};
    // k per axis = 1 - (s_k^2 / max s^2) (1 - k_max)
    float scale[3], sq[3];
    for (int k = 0; k < 3; ++k) {
      scale[k] = vs_expf(t[7 + k]);
      sq[k] = scale[k] * scale[k];
    }
    const float mx = fmaxf(fmaxf(fmaxf(sq[0], sq[1]), sq[2]), 1.0e-30f);
    const float k_max = split_at_screen_size > 0.0f
        ? fminf(split_at_screen_size * (1.0f / fmaxf(screen[p], 1.0e-6f)), r2) : r2;
    float v[3], logs[3];
    for (int k = 0; k < 3; ++k) {
      const float kk = -((sq[k] / mx) * (-k_max + 1.0f)) + 1.0f;
      v[k] = sqrtf(fmaxf(-(kk * kk) + 1.0f, 0.0f)) * scale[k];
      logs[k] = t[7 + k] + vs_logf(kk);
    }
    // offset rotated by q (quat_vec.rs)
    const float w2 = q[0] * q[0], x2 = q[1] * q[1], y2 = q[2] * q[2], z2 = q[3] * q[3];
    const float xy = q[1] * q[2], xz = q[1] * q[3], yz = q[2] * q[3];
    const float wx = q[0] * q[1], wy = q[0] * q[2], wz = q[0] * q[3];
    const float ox = (((w2 + x2) - y2) - z2) * v[0] + ((((xy * v[1] + xz * v[2]) + wy * v[2]) - wz * v[1]) * 2.0f);
    const float oy = (((w2 - x2) + y2) - z2) * v[1] + ((((xy * v[0] + yz * v[2]) + wz * v[0]) - wx * v[2]) * 2.0f);
    const float oz = (((w2 - x2) - y2) + z2) * v[2] + ((((xz * v[0] + yz * v[1]) + wx * v[1]) - wy * v[0]) * 2.0f);
    // both halves: opacity 1 - (1 - o)^(1/sqrt 2), logit of its clamp
    const float o = vs_sigmoid(raw_opac[p]);
    const float po = 1.0f - vs_expf(vs_logf(1.0f - o) * r2);
    const float cl = fminf(fmaxf(po, min_opacity), 1.0f - min_opacity);
    const float raw = vs_logf(cl / (1.0f - cl));
    float* tc = transforms + c * 10;
    float* tp = transforms + p * 10;
    const float child[10] = {t[0] + ox, t[1] + oy, t[2] + oz, q[0], q[1], q[2], q[3], logs[0], logs[1], logs[2]};
    const float parent[10] = {t[0] - ox, t[1] - oy, t[2] - oz, t[3], t[4], t[5], t[6], logs[0], logs[1], logs[2]};
    memcpy(tc, child, sizeof(child));
    memcpy(tp, parent, sizeof(parent));
    raw_opac[p] = raw;
    raw_opac[c] = raw;
    memcpy(sh + c * sh_width, sh + p * sh_width, sh_width * sizeof(float));
  }
  for (uint32_t i = 0; i < empty_count; ++i) {
    const size_t r = (size_t)empty_rows[i];
    const float row[10] = {0.0f, 0.0f, 0.0f, 1.0f, 0.0f, 0.0f, 0.0f, -10.0f, -10.0f, -10.0f};
    memcpy(transforms + r * 10, row, sizeof(row));
    raw_opac[r] = -20.0f;
    for (uint32_t k = 0; k < sh_width; ++k) sh[r * sh_width + k] = 0.0f;
  }
  return 0;
}

OR_API void or_opacity_decay(uint32_t n, float* raw_opac, float amount) {
  for (uint32_t g = 0; g < n; ++g) {
    const float o = fminf(fmaxf(vs_sigmoid(raw_opac[g]) - amount, 1.0e-12f), 1.0f - 1.0e-12f);
    raw_opac[g] = vs_logf(o / (1.0f - o));
  }
}

// Mip-Splatting 3D-filter floor, compute_min_scale (crates/splat-train/src/
// train.rs:353-387); cams rows are (centre x, y, z, 1 / max(focal, 1e-6)).
OR_API void or_min_scale(uint32_t n, const float* transforms, const float* cams, uint32_t views, float factor,
                         float* out) {
  const float sf = sqrtf(factor);
#pragma omp parallel for schedule(static)
  for (int64_t gi = 0; gi < (int64_t)n; ++gi) {
    const float* t = transforms + gi * 10;
    float r = INFINITY;
    for (uint32_t v = 0; v < views; ++v) {
      const float* c = cams + (size_t)v * 4;
      const float dx = t[0] - c[0], dy = t[1] - c[1], dz = t[2] - c[2];
      const float dist = sqrtf((dx * dx + dy * dy) + dz * dz);
      r = fminf(r, dist * c[3]);
    }
    out[gi] = r * sf;
  }
}

// fold_min_scale (crates/splat-train-render/src/gaussian_splats.rs:165-188).
OR_API void or_fold_min_scale(uint32_t n, float* transforms, float* raw_opac, const float* min_scale) {
  for (uint32_t g = 0; g < n; ++g) {
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
    const float o = fminf(fmaxf(vs_sigmoid(raw_opac[g]) * coef, 1.0e-6f), 1.0f - 1.0e-6f);
    raw_opac[g] = vs_logf(o / (1.0f - o));
  }
}

// ---- dataset feed: view_to_packed_data (crates/splat-train-dataset/src/
// scene.rs:113-161) for 8-bit sources.  L / LA widen to RGBA the way
// DynamicImage::into_rgba8 does (l, l, l[, a]); a missing alpha is 255; with
// alpha and the transparent mode each colour byte becomes (c * a + 127) / 255.
OR_API int or_pack_view(const uint8_t* px, uint32_t width, uint32_t height, uint32_t channels, int32_t alpha_mode,
                        uint32_t* out) {
  if (channels < 1 || channels > 4) return 1;
  const bool has_alpha = channels == 2 || channels == 4;
  const bool premultiply = has_alpha && alpha_mode == 1;
  const size_t n = (size_t)width * height;
  for (size_t i = 0; i < n; ++i) {
    const uint8_t* p = px + i * channels;
    uint32_t r, g, b, a = 255;
    if (channels <= 2) {
      r = g = b = p[0];
      if (channels == 2) a = p[1];
    } else {
      r = p[0], g = p[1], b = p[2];
      if (channels == 4) a = p[3];
    }
    if (premultiply) {
      r = (r * a + 127) / 255;
      g = (g * a + 127) / 255;
      b = (b * a + 127) / 255;
    }
    out[i] = r | g << 8 | b << 16 | a << 24;
  }
  return 0;
}

// ---- checkpoint I/O: PLY vertex rows (crates/splat-train-serde/src/
// export.rs:393-417, the encode closure of write_splat_ply).  sh is f32
// [n, coeffs, 3]; each row is x y z scale_0..2 opacity rot_0..3 (divided by
// max(sqrt(((r0 r0 + r1 r1) + r2 r2) + r3 r3), 1e-12)), f_dc_0..2, then the
// rest coefficients channel-major.
OR_API int or_ply_encode(uint32_t n, int32_t degree, const float* transforms, const float* sh, const float* raw_opac,
                         float* out) {
  if (degree < 0 || degree > 3) return 1;
  const uint32_t coeffs = (uint32_t)((degree + 1) * (degree + 1)), rest = coeffs - 1, stride = 14 + 3 * rest;
  for (uint32_t i = 0; i < n; ++i) {
    const float* t = transforms + (size_t)i * 10;
    float* w = out + (size_t)i * stride;
    const float rn = fmaxf(sqrtf(((t[3] * t[3] + t[4] * t[4]) + t[5] * t[5]) + t[6] * t[6]), 1.0e-12f);
    const float head[11] = {t[0], t[1], t[2], t[7], t[8], t[9], raw_opac[i], t[3] / rn, t[4] / rn, t[5] / rn, t[6] / rn};
    for (int k = 0; k < 11; ++k) w[k] = head[k];
    const float* s = sh + (size_t)i * coeffs * 3;
    for (int ch = 0; ch < 3; ++ch) w[11 + ch] = s[ch];
    for (uint32_t ch = 0; ch < 3; ++ch)
      for (uint32_t k = 1; k <= rest; ++k) w[14 + ch * rest + (k - 1)] = s[k * 3 + ch];
  }
  return 0;
}

// Thread count of the OpenMP loops above (a launcher such as torchrun sets
// OMP_NUM_THREADS=1 in every process; the CPU baseline asks for all cores).
OR_API void or_set_num_threads(int n) { omp_set_num_threads(n > 0 ? n : 1); }
OR_API int or_max_threads(void) { return omp_get_max_threads(); }
