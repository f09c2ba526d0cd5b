// Rotary position embedding evaluated in registers.
//
// The reference builds cos / sin tables per token on the host
// (compute_rope_2d, iris_transformer_flux.c:897; _with_t_offset :961;
// compute_rope_text :1055; zi_precompute_rope, iris_transformer_zimage.c:595),
// each entry cosf / sinf of the f32 product pos * freq.  Here every kernel
// that rotates a pair computes the same product from the row's position id
// and the pair's frequency (IrisRopeSpec) and evaluates cos and sin itself.
#pragma once

#include <stdint.h>

#include "iris_kernels.h"

namespace iris {

// cos / sin of a = pos * freq (the reference's f32 product).  a is reduced to
// [-pi, pi] by a = r + k * 2pi with 2pi split into an f32 head and tail
// (Cody-Waite reduction; each fma forms its product k * part exactly), then
// evaluated by the SFU sine / cosine, whose absolute error on [-pi, pi] is
// below 4e-7: the values agree with the reference's tables to within about
// 5e-7, far below the bf16 rounding of the rotated Q / K.
__device__ __forceinline__ void rope_cos_sin(uint32_t pos, float freq, float& c, float& s) {
  const float a = (float)pos * freq;
  const float k = rintf(a * 0.15915494309189535f);   // 1 / (2 pi)
  float r = fmaf(-k, 6.28318548202514648f, a);        // f32(2 pi)
  r = fmaf(-k, -1.7484555314695172e-07f, r);          // 2 pi - f32(2 pi)
  __sincosf(r, &s, &c);
}

// The four position ids of a row, stored as uint16 [4] (one 8-byte load).
struct RopePos {
  uint32_t v[4];
};

__device__ __forceinline__ RopePos rope_load_pos(const uint16_t* pos, int row) {
  const uint2 u = __ldg(reinterpret_cast<const uint2*>(pos) + row);
  RopePos p;
  p.v[0] = u.x & 0xFFFFu;
  p.v[1] = u.x >> 16;
  p.v[2] = u.y & 0xFFFFu;
  p.v[3] = u.y >> 16;
  return p;
}

__device__ __forceinline__ uint32_t rope_axis_pos(const RopePos& p, int axis) {
  return axis == 0 ? p.v[0] : axis == 1 ? p.v[1] : axis == 2 ? p.v[2] : p.v[3];
}

}  // namespace iris
