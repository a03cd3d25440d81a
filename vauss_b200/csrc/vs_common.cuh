// Shared device-side definitions for the vauss_b200 kernels (sm_100a).
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include "vs_math.h"

namespace vs {

constexpr uint32_t TILE = 16;
constexpr uint32_t TILE_PIX = TILE * TILE;
constexpr float ALPHA_MIN = 1.0f / 255.0f;
// Lower edge of the reference's alpha cutoff band (kernels/helpers.rs:23-24):
// splats whose exponent exceeds ln(a / EDGE) + 1e-3 cannot reach alpha 1/255,
// so the rasterizers skip their exp (rasterize_backwards_planes.rs:512-515).
constexpr float ALPHA_EDGE = 1.0f / 255.0f - 0.5e-3f;
constexpr float SH_C0 = 0.2820948f;
constexpr uint32_t B200_SMS = 148;

// Projection uniforms, built on the host from vs_camera + vs_render_cfg
// (the reference's ProjectUniforms, kernels/types.rs:53-109, with the pinhole
// clamp limits of camera.rs:305-331).
struct Uniforms {
  float rot[9];  // world -> camera rotation, column-major
  float trans[3];
  float fx, fy, cx, cy;
  float lim_pos_x, lim_pos_y, lim_neg_x, lim_neg_y;
  float cam[3];
  uint32_t w, h, tbw, tbh;
  float log_scale_offset;
  int32_t mip, has_min_scale, sh_degree, sh_half;
  float bg[3];
};

// Projected splat row, padded to three float4 for aligned gathers:
// [x, y, c00, c01] [c11, opacity, r, g] [b, global id bits, 0, 0].
constexpr uint32_t PROJ_F4 = 3;

struct V3 { float x, y, z; };
struct Q4 { float w, x, y, z; };
struct M3 { float c0x, c0y, c0z, c1x, c1y, c1z, c2x, c2y, c2z; };
struct S2 { float c00, c01, c11; };
struct S3 { float c00, c01, c02, c11, c12, c22; };
struct V2 { float x, y; };
struct M23 { V2 c0, c1, c2; };

#define VSD __device__ __forceinline__

VSD V3 v3add(V3 a, V3 b) { return {a.x + b.x, a.y + b.y, a.z + b.z}; }
VSD V3 v3sub(V3 a, V3 b) { return {a.x - b.x, a.y - b.y, a.z - b.z}; }
VSD V3 v3scale(V3 a, float s) { return {a.x * s, a.y * s, a.z * s}; }
// 4-lane dot with a zero padding lane (crates/splat-train-cube/src/lib.rs:85-89)
VSD float v3dot(V3 a, V3 b) { return ((a.x * b.x + a.y * b.y) + a.z * b.z) + 0.0f; }
VSD bool v3finite(V3 a) { return vs_is_finite(a.x) && vs_is_finite(a.y) && vs_is_finite(a.z); }
VSD float q4dot(Q4 a) { return ((a.w * a.w + a.x * a.x) + a.y * a.y) + a.z * a.z; }
VSD Q4 q4scale(Q4 a, float s) { return {a.w * s, a.x * s, a.y * s, a.z * s}; }
VSD float clampf(float x, float lo, float hi) { return fminf(fmaxf(x, lo), hi); }

VSD M3 quat_to_mat3(Q4 q) {
  const float x2 = q.x * q.x, y2 = q.y * q.y, z2 = q.z * q.z;
  const float xy = q.x * q.y, xz = q.x * q.z, yz = q.y * q.z;
  const float wx = q.w * q.x, wy = q.w * q.y, wz = q.w * q.z;
  return {1.0f - 2.0f * (y2 + z2), 2.0f * (xy + wz), 2.0f * (xz - wy),
          2.0f * (xy - wz), 1.0f - 2.0f * (x2 + z2), 2.0f * (yz + wx),
          2.0f * (xz + wy), 2.0f * (yz - wx), 1.0f - 2.0f * (x2 + y2)};
}
VSD V3 m3col0(const M3& m) { return {m.c0x, m.c0y, m.c0z}; }
VSD V3 m3col1(const M3& m) { return {m.c1x, m.c1y, m.c1z}; }
VSD V3 m3col2(const M3& m) { return {m.c2x, m.c2y, m.c2z}; }
VSD M3 m3from(V3 a, V3 b, V3 c) { return {a.x, a.y, a.z, b.x, b.y, b.z, c.x, c.y, c.z}; }
VSD V3 m3mulv(const M3& m, V3 v) {
  return v3add(v3add(v3scale(m3col0(m), v.x), v3scale(m3col1(m), v.y)), v3scale(m3col2(m), v.z));
}
VSD V3 m3tmulv(const M3& m, V3 v) { return {v3dot(m3col0(m), v), v3dot(m3col1(m), v), v3dot(m3col2(m), v)}; }
VSD M3 m3mul(const M3& a, const M3& b) {
  return m3from(m3mulv(a, m3col0(b)), m3mulv(a, m3col1(b)), m3mulv(a, m3col2(b)));
}
VSD M3 m3diag(const M3& m, V3 s) {
  return m3from(v3scale(m3col0(m), s.x), v3scale(m3col1(m), s.y), v3scale(m3col2(m), s.z));
}
VSD V3 m3row0(const M3& m) { return {m.c0x, m.c1x, m.c2x}; }
VSD V3 m3row1(const M3& m) { return {m.c0y, m.c1y, m.c2y}; }
VSD V3 m3row2(const M3& m) { return {m.c0z, m.c1z, m.c2z}; }
VSD S3 m3outer_self(const M3& m) {
  const V3 r0 = m3row0(m), r1 = m3row1(m), r2 = m3row2(m);
  return {v3dot(r0, r0), v3dot(r0, r1), v3dot(r0, r2), v3dot(r1, r1), v3dot(r1, r2), v3dot(r2, r2)};
}
VSD V2 v2add(V2 a, V2 b) { return {a.x + b.x, a.y + b.y}; }
VSD V2 v2scale(V2 a, float s) { return {a.x * s, a.y * s}; }
VSD float v2dot(V2 a, V2 b) { return a.x * b.x + a.y * b.y; }
VSD V2 m23mulv(const M23& m, V3 v) { return v2add(v2add(v2scale(m.c0, v.x), v2scale(m.c1, v.y)), v2scale(m.c2, v.z)); }
VSD M23 m23mul(const M23& m, const M3& n) { return {m23mulv(m, m3col0(n)), m23mulv(m, m3col1(n)), m23mulv(m, m3col2(n))}; }
VSD V3 m23row0(const M23& m) { return {m.c0.x, m.c1.x, m.c2.x}; }
VSD V3 m23row1(const M23& m) { return {m.c0.y, m.c1.y, m.c2.y}; }
VSD S2 m23gram(const M23& m) {
  return {m.c0.x * m.c0.x + m.c1.x * m.c1.x + m.c2.x * m.c2.x,
          m.c0.x * m.c0.y + m.c1.x * m.c1.y + m.c2.x * m.c2.y,
          m.c0.y * m.c0.y + m.c1.y * m.c1.y + m.c2.y * m.c2.y};
}
VSD V2 s2mulv(S2 s, V2 v) { return v2add(v2scale({s.c00, s.c01}, v.x), v2scale({s.c01, s.c11}, v.y)); }
VSD S3 m23tcong(const M23& m, S2 s) {
  const V2 sc0 = s2mulv(s, m.c0), sc1 = s2mulv(s, m.c1), sc2 = s2mulv(s, m.c2);
  return {v2dot(m.c0, sc0), v2dot(m.c0, sc1), v2dot(m.c0, sc2), v2dot(m.c1, sc1), v2dot(m.c1, sc2), v2dot(m.c2, sc2)};
}
VSD M23 s2mulm23(S2 s, const M23& n) { return {s2mulv(s, n.c0), s2mulv(s, n.c1), s2mulv(s, n.c2)}; }
VSD S2 s2inverse(S2 s) {
  const float det = s.c00 * s.c11 - s.c01 * s.c01;
  const float inv_det = det > 0.0f ? 1.0f / det : 0.0f;
  return {s.c11 * inv_det, -s.c01 * inv_det, s.c00 * inv_det};
}
VSD float s2det(S2 s) { return s.c00 * s.c11 - s.c01 * s.c01; }
VSD bool s2finite(S2 s) { return vs_is_finite(s.c00) && vs_is_finite(s.c11) && vs_is_finite(s.c01); }
VSD V3 s3row0(S3 s) { return {s.c00, s.c01, s.c02}; }
VSD V3 s3row1(S3 s) { return {s.c01, s.c11, s.c12}; }
VSD V3 s3row2(S3 s) { return {s.c02, s.c12, s.c22}; }
VSD V3 s3mulv(S3 s, V3 v) { return v3add(v3add(v3scale(s3row0(s), v.x), v3scale(s3row1(s), v.y)), v3scale(s3row2(s), v.z)); }
VSD S3 s3scale(S3 s, float k) { return {s.c00 * k, s.c01 * k, s.c02 * k, s.c11 * k, s.c12 * k, s.c22 * k}; }
VSD M3 s3mulm3(S3 s, const M3& m) { return m3from(s3mulv(s, m3col0(m)), s3mulv(s, m3col1(m)), s3mulv(s, m3col2(m))); }
VSD S3 s3cong(S3 s, const M3& m) {
  const V3 sr0 = s3mulv(s, m3row0(m)), sr1 = s3mulv(s, m3row1(m)), sr2 = s3mulv(s, m3row2(m));
  return {v3dot(m3row0(m), sr0), v3dot(m3row0(m), sr1), v3dot(m3row0(m), sr2),
          v3dot(m3row1(m), sr1), v3dot(m3row1(m), sr2), v3dot(m3row2(m), sr2)};
}
VSD S3 s3tcong(S3 s, const M3& m) {
  const V3 sc0 = s3mulv(s, m3col0(m)), sc1 = s3mulv(s, m3col1(m)), sc2 = s3mulv(s, m3col2(m));
  return {v3dot(m3col0(m), sc0), v3dot(m3col0(m), sc1), v3dot(m3col0(m), sc2),
          v3dot(m3col1(m), sc1), v3dot(m3col1(m), sc2), v3dot(m3col2(m), sc2)};
}

VSD M3 view_rot(const Uniforms& u) {
  return {u.rot[0], u.rot[1], u.rot[2], u.rot[3], u.rot[4], u.rot[5], u.rot[6], u.rot[7], u.rot[8]};
}
VSD V3 world_to_cam(V3 m, const Uniforms& u) {
  return v3add(m3mulv(view_rot(u), m), V3{u.trans[0], u.trans[1], u.trans[2]});
}

// Pinhole Jacobian with the 3DGS clamp (kernels/camera_model/pinhole.rs:153-177).
VSD M23 pinhole_jacobian(V3 p, const Uniforms& u) {
  const float inv_z = 1.0f / p.z;
  const float dx = u.fx * inv_z, dy = u.fy * inv_z;
  const float clx = clampf(p.x * inv_z, u.lim_neg_x, u.lim_pos_x);
  const float cly = clampf(p.y * inv_z, u.lim_neg_y, u.lim_pos_y);
  return {{dx, 0.0f}, {0.0f, dy}, {-dx * clx, -dy * cly}};
}

// EWA 2-D covariance (kernels/helpers.rs:195-225).
VSD S2 calc_cov2d(V3 scale, Q4 quat, V3 mean_c, const Uniforms& u) {
  const M3 ns = m3diag(m3mul(view_rot(u), quat_to_mat3(quat)), scale);
  const M23 jac = pinhole_jacobian(mean_c, u);
  const M23 v = m23mul(jac, ns);
  const S2 raw = m23gram(v);
  const float lim = 1.0e18f;
  const float max_abs = fmaxf(fmaxf(fabsf(raw.c00), fabsf(raw.c11)), fabsf(raw.c01));
  const float sd = max_abs > lim ? lim / max_abs : 1.0f;
  return {raw.c00 * sd, raw.c01 * sd, raw.c11 * sd};
}

// Low-pass blur and Mip compensation (kernels/helpers.rs:230-245).
VSD S2 compensate_cov2d(S2 c, bool mip, float* comp) {
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

// Screen half-extent from the conic (kernels/helpers.rs:133-144).
VSD void bbox_extent(S2 c, float pt, float* ex, float* ey) {
  const float det = c.c00 * c.c11 - c.c01 * c.c01;
  const bool degenerate = det <= 0.0f;
  const float inv_det = degenerate ? 0.0f : 1.0f / det;
  const float x = sqrtf(2.0f * pt * c.c11 * inv_det);
  const float y = sqrtf(2.0f * pt * c.c00 * inv_det);
  *ex = degenerate ? -1.0f : x;
  *ey = degenerate ? -1.0f : y;
}

struct TileBox { uint32_t x0, y0, x1, y1; };
// Tile-space bounding box (kernels/helpers.rs:158-190).
VSD TileBox tile_bbox(float cx, float cy, float ex, float ey, uint32_t bw, uint32_t bh) {
  const float tw = (float)TILE;
  const float x = cx / tw, y = cy / tw, dx = ex / tw, dy = ey / tw;
  const float bwf = (float)bw, bhf = (float)bh;
  return {(uint32_t)clampf(x - dx, 0.0f, bwf), (uint32_t)clampf(y - dy, 0.0f, bhf),
          (uint32_t)clampf(x + dx + 1.0f, 0.0f, bwf), (uint32_t)clampf(y + dy + 1.0f, 0.0f, bhf)};
}

VSD float calc_sigma(float px, float py, S2 c, float xx, float xy) {
  const float dx = px - xx, dy = py - xy;
  return 0.5f * (c.c00 * dx * dx + c.c11 * dy * dy) + c.c01 * dx * dy;
}

// Conservative tile-vs-ellipse test (kernels/helpers.rs:276-314, StopThePop).
VSD bool tile_hit(uint32_t tx, uint32_t ty, float mx, float my, S2 c, float pt) {
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

// Rasterizer exponent 0.5 c00 dx^2 + c01 dx dy + 0.5 c11 dy^2 with two fmas
// (sign-symmetric in (dx, dy), so forward and backward agree bit for bit).
VSD float raster_sigma(float h00, float c01, float h11, float dx, float dy) {
  const float t = fmaf(h00, dx, c01 * dy);
  return fmaf(dx, t, (h11 * dy) * dy);
}

// Correctly rounded reciprocal, quotient and square root built from the PTX
// approximations and fma, cheaper than the compiler's general-range sequences
// for 1/x, x/y and sqrtf (which carry range checks and a slow path).
//   rcp_rn(b):  one Newton step on rcp.approx; equal to the IEEE reciprocal
//               for every |b| in [2^-126, 2^126) (checked exhaustively on B200).
//   div_rn(a, b): q = a y, r = fma(-b, q, a), q + r y with y = rcp_rn(b); by
//               Markstein's theorem this is the correctly rounded a / b when
//               |b| is in that range and a, a / b are normal (and it returns
//               0 for a = 0).
//   sqrt_rn(v): s = v rsqrt(v) corrected by one fma, with inputs below 2^-100
//               scaled by 2^64; equal to IEEE sqrtf for every finite v >= 0
//               (checked exhaustively on B200), +inf and NaN included.
// The CPU oracle computes the same values with plain 1 / b, a / b and sqrtf.
VSD float rcp_rn(float b) {
  float y;
  asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(b));
  return fmaf(fmaf(-b, y, 1.0f), y, y);
}
VSD float div_rn(float a, float b) {
  const float y = rcp_rn(b);
  const float q = a * y;
  return fmaf(fmaf(-b, q, a), y, q);
}
VSD float sqrt_rn(float v) {
  const bool tiny = v < 7.888609052210118e-31f;  // 2^-100
  const float vs = tiny ? v * 18446744073709551616.0f : v;  // * 2^64
  float y;
  asm("rsqrt.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(vs));
  float s = vs * y;
  s = fmaf(fmaf(-s, s, vs), 0.5f * y, s);
  s = tiny ? s * 2.3283064365386963e-10f : s;  // * 2^-32
  return (v == 0.0f || v > 3.402823466e38f) ? v : s;  // +-0 and +inf map to themselves
}

// Warp-level culling of splats against a rectangle of pixel centres.
//
// sigma(d) = h00 dx^2 + c01 dx dy + h11 dy^2 (raster_sigma, d = mean - pixel)
// is a convex quadratic, so its minimum over a rectangle is 0 when the mean
// lies inside, else it lies on an edge, where sigma is a 1-D quadratic whose
// unconstrained minimiser is t = -c01 a / (2 h11) (x-edge dx = a) or
// t = -c01 a / (2 h00) (y-edge dy = a), clamped to the edge.  A splat whose
// minimum exceeds 1.02 cut + 1e-3 fails the exponent test (sigma <= cut) at
// every pixel centre of the rectangle: for conics with tr^2 < 1e4 det
// (condition number below ~1e4) the fp32 evaluation of sigma, at a pixel or at
// the edge minimiser, is within 1% of the exact form.  Other conics, NaNs and
// infinities always pass (test cut = +inf or NaN); a negative cut admits no
// pixel, since the exponent must also be >= 0.
struct ReachCut {
  float kx, ky;  // -c01 / (2 h11), -c01 / (2 h00): edge minimisers per unit offset
  float tcut;    // threshold on the rectangle minimum
};

VSD ReachCut reach_cut(float h00, float c01, float h11, float cut) {
  const float c00 = 2.0f * h00, c11 = 2.0f * h11;
  const float det = c00 * c11 - c01 * c01, tr = c00 + c11;
  const bool tame = det > 0.0f && tr > 0.0f && tr * tr < 1.0e4f * det;
  ReachCut r;
  r.kx = tame ? -c01 / c11 : 0.0f;
  r.ky = tame ? -c01 / c00 : 0.0f;
  r.tcut = cut < 0.0f ? -1.0f : (tame ? 1.02f * cut + 1.0e-3f : __int_as_float(0x7f800000));
  return r;
}

VSD float edge_min(float h_a, float c01, float h_t, float a, float k, float lo, float hi) {
  const float t = clampf(k * a, lo, hi);
  return fmaf(a, fmaf(h_a, a, c01 * t), (h_t * t) * t);
}

// True unless every pixel centre in [rx0, rx1] x [ry0, ry1] certainly fails
// sigma <= cut.
VSD bool reach_rect(float mx, float my, float h00, float c01, float h11, ReachCut rc, float rx0, float rx1,
                    float ry0, float ry1) {
  const float dxl = mx - rx1, dxh = mx - rx0, dyl = my - ry1, dyh = my - ry0;
  if (dxl <= 0.0f && dxh >= 0.0f && dyl <= 0.0f && dyh >= 0.0f) return rc.tcut >= 0.0f || rc.tcut != rc.tcut;
  const float m = fminf(fminf(edge_min(h00, c01, h11, dxl, rc.kx, dyl, dyh), edge_min(h00, c01, h11, dxh, rc.kx, dyl, dyh)),
                        fminf(edge_min(h11, c01, h00, dyl, rc.ky, dxl, dxh), edge_min(h11, c01, h00, dyh, rc.ky, dxl, dxh)));
  return !(m > rc.tcut);
}

struct Floor { V3 scale; float opac, coef; V3 ratio_sq; bool opac_open; };
// Mip-Splatting 3D filter floor (kernels/helpers.rs:516-553).
VSD Floor apply_scale_floor(V3 s, float opac_sig, const float* min_scale, uint32_t g, bool has) {
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

VSD float sh_load(const void* sh, bool half, size_t i) {
  return half ? vs_f16_to_f32(((const uint16_t*)sh)[i]) : ((const float*)sh)[i];
}

// Real SH basis Y_k(dir), k < 16 (crates/splat-train/src/quant_kernels.rs:789-858).
VSD void sh_basis_all(float x, float y, float z, float* b) {
  const float z2 = z * z;
  const float fc1 = x * x - y * y;
  const float fs1 = 2.0f * x * y;
  const float fc2 = x * fc1 - y * fs1;
  const float fs2 = x * fs1 + y * fc1;
  const float f0b = -1.0925485f * z;
  const float f0c = -2.285229f * z2 + 0.4570458f;
  const float f1b = 1.4453057f * z;
  const float f2a = -0.5900436f;
  b[0] = 0.2820948f;
  b[1] = -0.4886025f * y;
  b[2] = 0.4886025f * z;
  b[3] = -0.4886025f * x;
  b[4] = 0.54627424f * fs1;
  b[5] = f0b * y;
  b[6] = 0.9461747f * z2 - 0.31539157f;
  b[7] = f0b * x;
  b[8] = 0.54627424f * fc1;
  b[9] = f2a * fs2;
  b[10] = f1b * fs1;
  b[11] = f0c * y;
  b[12] = z * (1.8658817f * z2 - 1.119529f);
  b[13] = f0c * x;
  b[14] = f1b * fc1;
  b[15] = f2a * fc2;
}

__host__ __device__ __forceinline__ uint32_t div_up(uint32_t a, uint32_t b) { return (a + b - 1) / b; }

}  // namespace vs

// Device error word bits (ctx->d_err): set by kernels whose bounded waits
// give up or whose capacity checks fail; read by the host after a stage.
#define VS_DERR_WAIT 1u
#define VS_DERR_CAPACITY 2u
#define VS_DERR_RANGE 4u
#define VS_DERR_STATE 8u  // a call's precondition on device state failed (compact rows seen twice)
