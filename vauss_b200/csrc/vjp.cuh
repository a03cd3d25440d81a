// Projection VJP of one visible splat, shared by the fused optimizer kernels
// and the dense (multi-view) backward.  Follows the reference's splat_vjp
// (crates/splat-train-render/src/bwd/kernels/project_backwards.rs:132-274)
// with apply_normalize_vjp (:20-51), quat_to_mat_vjp (:55-78),
// inverse2x2_vjp (:86-98), calculate_projection_vjp_pinhole
// (kernels/camera_model/pinhole.rs:179-245) and sh_color_viewdir_vjp
// (kernels/sh.rs:147-270).
#pragma once

#include "vs_common.cuh"

namespace vs {

struct VjpOut {
  V3 v_mean;
  Q4 v_q;
  V3 v_scale;
  float v_raw;
  V3 dir;
};

VSD Q4 normalize_vjp(Q4 q, Q4 g) {
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

VSD Q4 quat_to_mat_vjp(Q4 q, const M3& v) {
  const float wg = q.x * (v.c1z - v.c2y) + q.y * (v.c2x - v.c0z) + q.z * (v.c0y - v.c1x);
  const float xg = -2.0f * q.x * (v.c1y + v.c2z) + q.y * (v.c0y + v.c1x) + q.z * (v.c0z + v.c2x) + q.w * (v.c1z - v.c2y);
  const float yg = q.x * (v.c0y + v.c1x) - 2.0f * q.y * (v.c0x + v.c2z) + q.z * (v.c1z + v.c2y) + q.w * (v.c2x - v.c0z);
  const float zg = q.x * (v.c0z + v.c2x) + q.y * (v.c1z + v.c2y) - 2.0f * q.z * (v.c0x + v.c1y) + q.w * (v.c0y - v.c1x);
  return {2.0f * wg, 2.0f * xg, 2.0f * yg, 2.0f * zg};
}

VSD S2 inverse2x2_vjp(S2 m, S2 v) {
  const float t00 = -m.c00 * v.c00 + -m.c01 * v.c01;
  const float t01 = -m.c01 * v.c00 + -m.c11 * v.c01;
  const float t10 = -m.c00 * v.c01 + -m.c01 * v.c11;
  const float t11 = -m.c01 * v.c01 + -m.c11 * v.c11;
  return {t00 * m.c00 + t10 * m.c01, t01 * m.c00 + t11 * m.c01, t01 * m.c01 + t11 * m.c11};
}

VSD V3 projection_vjp_pinhole(const M23& J, V3 mc, S3 cov_c, const Uniforms& u, S2 v_cov2d, V2 v_mean2d) {
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

// SH view-direction VJP for bands <= 3 (kernels/sh.rs:147-270).
VSD V3 sh_viewdir_vjp(const void* sh, bool half, size_t base, int deg, V3 v, V3 vc) {
  // Degree 3 in f32 from a 16-byte aligned array: the 45 coefficients past
  // the DC term are loaded up front as 16-byte vectors (the row is 192 bytes).
  float cf[48];
  const bool vec = !half && deg == 3 && (reinterpret_cast<uintptr_t>(sh) & 15u) == 0;
  if (vec) {
    const float4* p4 = reinterpret_cast<const float4*>((const float*)sh + base);
#pragma unroll
    for (int q = 0; q < 12; ++q) {
      const float4 x = p4[q];
      cf[4 * q] = x.x;
      cf[4 * q + 1] = x.y;
      cf[4 * q + 2] = x.z;
      cf[4 * q + 3] = x.w;
    }
  }
  auto sd = [&](int k) -> float {
    const V3 c = vec ? V3{cf[k], cf[k + 1], cf[k + 2]}
                     : V3{sh_load(sh, half, base + k), sh_load(sh, half, base + k + 1), sh_load(sh, half, base + k + 2)};
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

// rg = the splat's rasterizer gradient row [10]; t = its transforms row.
VSD VjpOut splat_vjp(const float* t, float raw_opac, const void* sh, const float* min_scale, uint32_t g,
                     const float* rg, const Uniforms& u) {
  const bool half = u.sh_half != 0;
  const int deg = u.sh_degree;
  const V3 mean = {t[0], t[1], t[2]};
  const V3 scale_raw = {vs_expf(t[7] + u.log_scale_offset), vs_expf(t[8] + u.log_scale_offset),
                        vs_expf(t[9] + u.log_scale_offset)};
  const Q4 qu = {t[3], t[4], t[5], t[6]};
  const S2 v_inv = {rg[2], rg[3] * 0.5f, rg[4]};
  const V3 v_color = {rg[5], rg[6], rg[7]};
  const Q4 quat = q4scale(qu, 1.0f / sqrtf(q4dot(qu)));
  const float opac_sig = vs_sigmoid(raw_opac);
  const Floor fl = apply_scale_floor(scale_raw, opac_sig, min_scale, g, u.has_min_scale != 0);
  const V3 scale = fl.scale;
  const V3 uw = v3sub(mean, V3{u.cam[0], u.cam[1], u.cam[2]});
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
  const S2 cov = compensate_cov2d(raw_cov, u.mip != 0, &comp);
  const float v_opac_base = fl.opac_open ? comp * rg[8] : 0.0f;
  const S2 conic_inv = s2inverse(cov);
  const S2 v_cov2d = inverse2x2_vjp(conic_inv, v_inv);
  const S3 covar = m3outer_self(m);
  const M3 R = view_rot(u);
  const S3 cov_c = s3cong(covar, R);
  const M23 J = pinhole_jacobian(mean_c, u);
  const V3 v_mean_c = projection_vjp_pinhole(J, mean_c, cov_c, u, v_cov2d, V2{rg[0], rg[1]});
  const S3 vcc = m23tcong(J, v_cov2d);
  const V3 v_mean = v3add(m3tmulv(R, v_mean_c), v_mean_sh);
  const M3 v_m = s3mulm3(s3scale(s3tcong(vcc, R), 2.0f), m);
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

}  // namespace vs
