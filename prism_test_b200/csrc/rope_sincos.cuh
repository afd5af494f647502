// RoPE angle evaluation for the fused inverse rotation of cached keys.
//
// The reference builds its rotary tables in fp32 (build_cos_sin,
// eval_harness/attention_methods/_method_base.py:353-381):
//     angle = fp32(position) * inv_freq[i]      (one fp32 product, rounded once)
//     cos/sin of that fp32 angle
// and un-rotates with undo_rotary_pos_emb (_method_base.py:336-350):
//     x * cos + rotate_half(x) * (-sin)
// i.e. for i < D/2:  r_i = x_i c_i + x_{i+D/2} s_i,  r_{i+D/2} = x_{i+D/2} c_i - x_i s_i.
//
// To agree with that table the kernels form the identical fp32 product and
// then evaluate sin/cos of it accurately. Angles reach ~4e6 rad, so:
//   * quadrant n = round(x * 2/pi) by the round-to-integer-by-addition method:
//     t = fma(x, 2/pi, 1.5*2^23) holds n in its low mantissa bits (|n| < 2^22),
//     n = t - 1.5*2^23 (no conversion instructions);
//   * Cody & Waite (1980) additive reduction r = x - n*pi/2 with pi/2 split into
//     three fp32 parts applied through FMA. The parts were derived for this
//     file from pi computed by Machin's formula in exact integer arithmetic:
//     P1 = fp32(pi/2), P2 = fp32(pi/2 - P1), P3 = fp32(pi/2 - P1 - P2).
//     x - n*P1 is exact in one FMA for |x| < 2^22, so |r| <= ~pi/4 carries an
//     absolute error of a few 1e-8;
//   * sin/cos of r either by polynomials in t = r^2 (rope_sincos: coefficients
//     fitted for this file by least squares on 4000 Chebyshev nodes, max error
//     7e-9 / 2e-9 on |r| <= 1) or by the hardware approximations __sinf/__cosf
//     on the reduced argument (rope_sincos_fast: absolute error <= 2^-21.4 on
//     [-pi, pi], i.e. ~4e-7, three orders of magnitude inside the 1e-3 score
//     tolerance);
//   * quadrant selection from n mod 4.
// Supported domain: |x| < 2^22 (positions below 4M with inv_freq <= 1).
#pragma once

namespace prism {

struct RopeQuadrant {
  float r;  // reduced argument
  int q;    // quadrant (n mod 4 in the low bits)
};

__device__ __forceinline__ RopeQuadrant rope_reduce(float x) {
  constexpr float kTwoOverPi = 0x1.45f306p-1f;
  constexpr float kMagic = 12582912.0f;  // 1.5 * 2^23
  constexpr float kP1 = 0x1.921fb6p+0f;
  constexpr float kP2 = -0x1.777a5cp-25f;
  constexpr float kP3 = -0x1.ee59dap-50f;
  const float t = fmaf(x, kTwoOverPi, kMagic);
  const float n = t - kMagic;
  float r = fmaf(-n, kP1, x);
  r = fmaf(-n, kP2, r);
  r = fmaf(-n, kP3, r);
  return RopeQuadrant{r, __float_as_int(t)};
}

__device__ __forceinline__ void rope_quadrant_fix(int q, float sr, float cr, float& s_out,
                                                  float& c_out) {
  float ss = (q & 1) ? cr : sr;
  float cc = (q & 1) ? sr : cr;
  ss = (q & 2) ? -ss : ss;
  cc = ((q + 1) & 2) ? -cc : cc;
  s_out = ss;
  c_out = cc;
}

// Polynomial evaluation (fp32, ~1 ulp).
__device__ __forceinline__ void rope_sincos(float x, float& s_out, float& c_out) {
  // sin(r)/r - 1 = t*(S1 + t*(S2 + t*(S3 + t*S4)))
  constexpr float kS1 = -0x1.555556p-3f;
  constexpr float kS2 = 0x1.1110ecp-7f;
  constexpr float kS3 = -0x1.9ffea6p-13f;
  constexpr float kS4 = 0x1.69bbdep-19f;
  // cos(r) - 1 = t*(C1 + t*(C2 + t*(C3 + t*(C4 + t*C5))))
  constexpr float kC1 = -0x1.000000p-1f;
  constexpr float kC2 = 0x1.555554p-5f;
  constexpr float kC3 = -0x1.6c1688p-10f;
  constexpr float kC4 = 0x1.9ffd44p-16f;
  constexpr float kC5 = -0x1.2156dcp-22f;
  const RopeQuadrant rq = rope_reduce(x);
  const float r = rq.r;
  const float t = r * r;
  float ps = fmaf(kS4, t, kS3);
  ps = fmaf(ps, t, kS2);
  ps = fmaf(ps, t, kS1);
  const float sr = fmaf(r * t, ps, r);
  float pc = fmaf(kC5, t, kC4);
  pc = fmaf(pc, t, kC3);
  pc = fmaf(pc, t, kC2);
  pc = fmaf(pc, t, kC1);
  const float cr = fmaf(t, pc, 1.0f);
  rope_quadrant_fix(rq.q, sr, cr, s_out, c_out);
}

// Reduction as above, then the hardware sin/cos approximations on |r| <= ~pi/4.
__device__ __forceinline__ void rope_sincos_fast(float x, float& s_out, float& c_out) {
  const RopeQuadrant rq = rope_reduce(x);
  rope_quadrant_fix(rq.q, __sinf(rq.r), __cosf(rq.r), s_out, c_out);
}

}  // namespace prism
