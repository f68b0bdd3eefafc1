// CROWN ReLU relaxation shared by the fused CROWN kernels: the slope rule
// (verify_zono_bnb.py:503-522) encoded as one float2 per neuron, and its
// decoded form applied to back-substitution coefficients.
#pragma once

#include <cuda_runtime.h>

namespace vcb {

// CROWN slope rule (verify_zono_bnb.py:511-521), sign-encoded:
//   x = dead ? -up_s : up_s,   y = active ? -0.0f : up_t.
// The division only runs where lo < 0 < hi or in the dead corner where
// lo + 1e-8 > 0 (elsewhere up_s is exactly 1 or 0).
__device__ __forceinline__ float2 encode_slope(float lo, float hi) {
  if (lo >= 0.f) return make_float2(1.f, -0.0f);  // active
  const bool dead = hi <= 0.f;
  const float ub_r = fmaxf(fmaxf(hi, 0.f), __fadd_rn(lo, 1e-8f));
  if (ub_r == 0.f) return make_float2(-0.0f, 0.0f);  // dead, up_s = 0
  const float up_s = __fdiv_rn(ub_r, __fsub_rn(ub_r, lo));
  const float up_t = __fmul_rn(-lo, up_s);
  return make_float2(dead ? -up_s : up_s, up_t);
}

struct Slope {
  float pos, neg, icp;  // multiplier for e >= 0, for e < 0, intercept factor
};

// Decoded relaxation of one neuron; alpha (may be NULL) replaces the
// min-area lower slope of unstable neurons (verify_zono_bnb.py:4420-4433).
__device__ __forceinline__ Slope decode_slope(float2 v, const float* alpha) {
  Slope s;
  if (signbit(v.y)) {  // active: identity, no intercept
    s.pos = 1.f; s.neg = 1.f; s.icp = 0.f;
  } else if (signbit(v.x)) {  // dead (lower slope 0)
    s.pos = 0.f; s.neg = -v.x; s.icp = v.y;
  } else {  // unstable
    s.pos = alpha ? __ldg(alpha) : (v.x > 0.5f ? 1.f : 0.f);
    s.neg = v.x; s.icp = v.y;
  }
  return s;
}

// Relaxation of one neuron from its pre-activation bounds as the wide
// layer-wise passes apply it (verify_zono_bnb.py:511-521, 4413-4433): pos
// multiplies e >= 0 (lower slope; alpha on unstable neurons when given), neg
// multiplies e < 0 (upper slope), icp is the intercept factor of min(e, 0).
struct RelaxTc {
  float pos, neg, icp;
  bool unstable;
};

__device__ __forceinline__ RelaxTc relax_tc(float lo, float hi, const float* alpha) {
  RelaxTc r;
  const float lb_r = fminf(lo, 0.f);
  const float ub_r = fmaxf(fmaxf(hi, 0.f), __fadd_rn(lb_r, 1e-8f));
  const float up_s = __fdiv_rn(ub_r, __fsub_rn(ub_r, lb_r));
  const bool active = lo >= 0.f, dead = hi <= 0.f;
  r.unstable = !active && !dead;
  r.neg = up_s;
  r.icp = __fmul_rn(-lb_r, up_s);
  r.pos = active ? 1.f : (dead ? 0.f : (alpha ? *alpha : (up_s > 0.5f ? 1.f : 0.f)));
  return r;
}

}  // namespace vcb
