// Rotary-embedding angle math shared by the RoPE kernels (vl_rope.cu) and
// the decode-step attention (vl_attn.cu).
//
// Reference (VideoLingo-user native/asr/src): build_rope_table
// (engine.cu:892-905) and build_full_rope_table (decoder.cu:950-961) form
// inv_freq(d) = 1/pow(base, 2d/rot) and angle = inv_freq * pos in fp64 and
// round cos/sin to fp32.  Here the fp64 inverse frequencies are built on the
// host and the cos/sin are evaluated on the device per (token, pair).
#pragma once

#include <cmath>

#include "vl_common.cuh"

namespace vl {

constexpr int kMaxHalfRot = 128;

struct InvFreq {
  double v[kMaxHalfRot];
};

inline InvFreq make_inv_freq(double base, int rotary_dim) {
  InvFreq f{};
  for (int d = 0; d < rotary_dim / 2 && d < kMaxHalfRot; ++d)
    f.v[d] = 1.0 / std::pow(base, static_cast<double>(2 * d) / rotary_dim);
  return f;
}

// cos/sin of angle = pos * inv_freq (formed in fp64, as the reference's host
// tables are): the angle is reduced modulo 2*pi in fp64 (Cody-Waite with a
// two-term 2*pi), then evaluated with fp32 sincosf on [-pi, pi].  Against
// rounding fp64 cos/sin to fp32 the difference is below 3e-7 absolute, at a
// fraction of the cost of an fp64 sincos.
__device__ __forceinline__ float2 rope_cos_sin(double angle) {
  constexpr double kTwoPiHi = 6.283185307179586232;        // 2*pi rounded to double
  constexpr double kTwoPiLo = 2.4492935982947064e-16;      // 2*pi - kTwoPiHi
  constexpr double kInvTwoPi = 0.15915494309189533577;
  const double k = rint(angle * kInvTwoPi);
  double r = fma(-k, kTwoPiHi, angle);
  r = fma(-k, kTwoPiLo, r);
  float sn, cs;
  sincosf(static_cast<float>(r), &sn, &cs);
  return make_float2(cs, sn);
}

}  // namespace vl
