// Deterministic scalar math shared by the sm_100a kernels and the CPU
// parity oracle.
//
// Every function here is written with IEEE single-precision operations whose
// results are fully specified (+, -, *, /, sqrt, fma, rint, integer and bit
// operations), so the host build (g++ -ffp-contract=off) and the device build
// (nvcc -fmad=false, no fast-math) produce the same bits.  That is what makes
// the integer outputs of the projection (visible set, tile counts, sorted keys,
// tile ranges) and the front-to-back compositing comparable bit-for-bit
// against the oracle.
//
// exp and log are our own, written from the mathematics:
//   exp: Cody-Waite range reduction x = k ln2 + r (two-constant split of ln2),
//        |r| <= ln2/2, then a degree-5 polynomial 1 + r + c2 r^2 + ... in
//        Horner form whose coefficients minimise the largest relative error
//        on that interval (a linear-programming minimax fit; 1.03e-7 before
//        f32 rounding), scaled by 2^k through the exponent bits: within
//        2.2 ulp of e^x (exhaustively checked against double exp; the WGSL
//        exp the reference calls is specified to 3 + 2|x| ulp).  Inputs
//        below -87 flush to +0 (results would be subnormal); inputs >=
//        88.72283 give +inf.
//   log: x = m 2^e with m in [sqrt(1/2), sqrt(2)), s = (m-1)/(m+1),
//        ln m = 2 atanh(s) = 2 (s + s^3/3 + ... + s^11/11)  (|s| <= 0.1716,
//        truncation < 1e-10), ln x = e ln2 + ln m with the same ln2 split.
// Both are accurate to a few ulp (tests compare against libm's double-precision
// results) and, more importantly, identical on host and device.
#pragma once

#include <stdint.h>
#include <math.h>
#include <string.h>

#if defined(__CUDACC__)
#define VS_HD __host__ __device__ __forceinline__
#else
#define VS_HD static inline
#endif

VS_HD uint32_t vs_f2u(float f) {
#if defined(__CUDA_ARCH__)
  return __float_as_uint(f);
#else
  uint32_t u;
  memcpy(&u, &f, 4);
  return u;
#endif
}

VS_HD float vs_u2f(uint32_t u) {
#if defined(__CUDA_ARCH__)
  return __uint_as_float(u);
#else
  float f;
  memcpy(&f, &u, 4);
  return f;
#endif
}

// Bit-level finite test: NaN and +-inf have an all-ones exponent.
VS_HD bool vs_is_finite(float x) { return ((vs_f2u(x) >> 23) & 0xffu) != 0xffu; }

#define VS_LN2_HI 0.693145751953125f        /* ln 2 rounded to 16 significant bits */
#define VS_LN2_LO 1.42860682030941723212e-6f /* ln 2 - VS_LN2_HI */
#define VS_LOG2E 1.44269504088896340736f

// vs_expf without its range checks: equal to vs_expf for x in [-87, 88.72283)
// (outside that range the result is meaningless, so callers use it only
// where their own tests already reject such inputs).
VS_HD float vs_expf_core(float x) {
  // k = rint(x log2e): adding 1.5 * 2^23 rounds |x log2e| < 2^22 to an integer
  // (ties to even, the default rounding mode), whose value then sits in the
  // low mantissa bits, so no float<->int conversion is needed.
  const float shifted = x * VS_LOG2E + 12582912.0f;
  const float k = shifted - 12582912.0f;
  float r = fmaf(k, -VS_LN2_HI, x);
  r = fmaf(k, -VS_LN2_LO, r);
  // e^r ~ 1 + r + c2 r^2 + c3 r^3 + c4 r^4 + c5 r^5 on |r| <= ln2/2, the
  // coefficients minimising the largest relative error over that interval
  // (found by linear programming over a dense grid, exp_minimax.py in this
  // directory; 1.03e-7 before rounding to f32).  With the f32 evaluation the result is within 2.2 ulp of e^x
  // over [-87, 88.72), checked exhaustively against double exp.
  float p = 8.314745500683784e-3f;
  p = fmaf(p, r, 4.189043864607811e-2f);
  p = fmaf(p, r, 1.6667090356349945e-1f);
  p = fmaf(p, r, 4.99992311000824e-1f);
  p = fmaf(p, r, 1.0f);
  p = fmaf(p, r, 1.0f);
  const uint32_t ki = vs_f2u(shifted) - 0x4B400000u;  // k as a two's-complement integer
  return vs_u2f(vs_f2u(p) + (ki << 23));
}

VS_HD float vs_expf(float x) {
  if (!(x < 88.72283f)) return (x != x) ? x : INFINITY;
  if (x < -87.0f) return 0.0f;
  return vs_expf_core(x);
}

VS_HD float vs_logf(float x) {
  if (x != x) return x;
  if (x < 0.0f) return NAN;
  if (x == 0.0f) return -INFINITY;
  if (x == INFINITY) return INFINITY;
  int32_t e = 0;
  uint32_t bits = vs_f2u(x);
  if ((bits >> 23) == 0) {  // subnormal: scale into the normal range
    bits = vs_f2u(x * 8388608.0f);
    e = -23;
  }
  e += (int32_t)((bits >> 23) & 0xffu) - 127;
  float m = vs_u2f((bits & 0x007fffffu) | 0x3f800000u);  // [1, 2)
  if (m > 1.41421356237309504880f) {
    m = m * 0.5f;
    e += 1;
  }
  const float s = (m - 1.0f) / (m + 1.0f);
  const float s2 = s * s;
  float p = 9.09090909090909090909e-2f;  // 1/11
  p = fmaf(p, s2, 1.11111111111111111111e-1f);  // 1/9
  p = fmaf(p, s2, 1.42857142857142857143e-1f);  // 1/7
  p = fmaf(p, s2, 2.0e-1f);                     // 1/5
  p = fmaf(p, s2, 3.33333333333333333333e-1f);  // 1/3
  p = fmaf(p, s2, 1.0f);
  const float lnm = 2.0f * s * p;
  const float ef = (float)e;
  return fmaf(ef, VS_LN2_HI, fmaf(ef, VS_LN2_LO, lnm));
}

VS_HD float vs_sigmoid(float x) { return 1.0f / (1.0f + vs_expf(-x)); }

// Per-element, per-step integer hash (the mixer the reference's stochastic
// rounding uses: crates/splat-train-render/src/bwd/kernels/geo_moments.rs:57-63).
VS_HD uint32_t vs_mix_hash(uint32_t index, uint32_t step) {
  uint32_t h = index ^ (step * 0x9e3779b9u);
  h = (h ^ (h >> 16)) * 0x7feb352du;
  h = (h ^ (h >> 15)) * 0x846ca68bu;
  return h ^ (h >> 16);
}

// IEEE binary16 <-> binary32, round to nearest even (our own bit code).
VS_HD uint16_t vs_f32_to_f16(float f) {
  const uint32_t x = vs_f2u(f);
  const uint32_t sign = (x >> 16) & 0x8000u;
  const uint32_t ax = x & 0x7fffffffu;
  if (ax >= 0x7f800000u) {  // inf or nan
    return (uint16_t)(sign | 0x7c00u | (ax > 0x7f800000u ? 0x200u : 0u));
  }
  if (ax >= 0x477ff000u) return (uint16_t)(sign | 0x7c00u);  // rounds to >= 65520: overflow
  if (ax < 0x38800000u) {  // below the smallest normal half (2^-14)
    if (ax < 0x33000000u) return (uint16_t)sign;  // < 2^-25 rounds to zero
    const uint32_t e = ax >> 23;
    const uint32_t mant = (ax & 0x7fffffu) | 0x800000u;
    const uint32_t shift = 126u - e;  // 14..24 : value = mant * 2^(e-150), half ulp 2^-24
    uint32_t q = mant >> shift;
    const uint32_t rem = mant & ((1u << shift) - 1u);
    const uint32_t half = 1u << (shift - 1u);
    if (rem > half || (rem == half && (q & 1u))) q += 1u;
    return (uint16_t)(sign | q);
  }
  uint32_t h = ((ax >> 13) - (112u << 10));  // rebias exponent 127 -> 15
  const uint32_t rem = ax & 0x1fffu;
  if (rem > 0x1000u || (rem == 0x1000u && (h & 1u))) h += 1u;
  return (uint16_t)(sign | h);
}

VS_HD float vs_f16_to_f32(uint16_t h) {
  const uint32_t sign = ((uint32_t)h & 0x8000u) << 16;
  const uint32_t e = ((uint32_t)h >> 10) & 0x1fu;
  const uint32_t m = (uint32_t)h & 0x3ffu;
  if (e == 0) {
    if (m == 0) return vs_u2f(sign);
    // subnormal half: m * 2^-24 is exact in f32
    const float v = (float)m * 5.9604644775390625e-8f;
    return sign ? -v : v;
  }
  if (e == 31) return vs_u2f(sign | 0x7f800000u | (m << 13));
  return vs_u2f(sign | ((e + 112u) << 23) | (m << 13));
}

// sin/cos of an angle in [0, 2*pi) (Box-Muller angles): quadrant reduction with
// a two-constant pi/2, then Taylor polynomials on |r| <= pi/4.
VS_HD void vs_sincosf(float a, float* s_out, float* c_out) {
  const float q = rintf(a * 0.636619772367581343076f);  // 2/pi
  float r = fmaf(q, -1.5707962513f, a);
  r = fmaf(q, -7.5497894159e-8f, r);
  const float r2 = r * r;
  float s = -2.50521083854417187751e-8f;  // -1/11!
  s = fmaf(s, r2, 2.75573192239858906526e-6f);  // 1/9!
  s = fmaf(s, r2, -1.98412698412698412698e-4f);  // -1/7!
  s = fmaf(s, r2, 8.33333333333333333333e-3f);  // 1/5!
  s = fmaf(s, r2, -1.66666666666666666667e-1f);  // -1/3!
  s = fmaf(s * r2, r, r);
  float c = -2.75573192239858906526e-7f;  // -1/10!
  c = fmaf(c, r2, 2.48015873015873015873e-5f);  // 1/8!
  c = fmaf(c, r2, -1.38888888888888888889e-3f);  // -1/6!
  c = fmaf(c, r2, 4.16666666666666666667e-2f);  // 1/4!
  c = fmaf(c, r2, -0.5f);
  c = fmaf(c, r2, 1.0f);
  const int32_t qi = ((int32_t)q) & 3;
  float so = s, co = c;
  if (qi == 1) { so = c; co = -s; }
  else if (qi == 2) { so = -s; co = -c; }
  else if (qi == 3) { so = -c; co = s; }
  *s_out = so;
  *c_out = co;
}
