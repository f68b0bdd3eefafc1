// Batched forward linear bounds (forward LiRPA) of ReLU MLPs over the varying
// input dimensions, with the spec contraction of the multi-subbox input-split
// BaB (forward_lirpa.py:443-680 for fc / relu, verify_graph.py:11522-11560).
//
// Per box, linear lower / upper bounds of every neuron in the K varying input
// coordinates z (x = b + A z): A_lo, A_up (n x K) and b_lo, b_up (n), kept in
// shared memory as n x (K + 1) with b as the last column:
//   * input: A = the columns of the identity at the varying dimensions, b =
//     x_lo on the constant dimensions (0 on the varying ones);
//   * fc: with A_mid = (A_lo + A_up) / 2 and A_half = (A_up - A_lo) / 2,
//     A_lo' = W A_mid - |W| A_half, A_up' = W A_mid + |W| A_half (the bias is
//     added to the b column of W A_mid); box bounds
//     lo = A_lo' x_mid - |A_lo'| x_half + b_lo', hi likewise with A_up';
//   * relu: min-area lower slope (1 if hi / (hi - lo) > 0.5 on unstable
//     neurons), upper slope hi / max(hi - lo, 1e-12) with intercept
//     -slope lo, both applied to the rows;
//   * spec rows w (Q x n_out): spec_A = w+ A_lo + w- A_up, spec_b likewise,
//     lb = spec_A+ x_lo + spec_A- x_hi + spec_b over the varying dimensions.
// One CTA of 128 threads per box; weights read through the read-only cache.
// vcb_mlp_flirpa_fate goes on to the multi-subbox leaf fate (input-domain
// clip, smart-branching scores; vcb_multisub.cuh) on the spec rows while
// they are still in shared memory.
#include <algorithm>

#include "vcb_common.cuh"
#include "vcb_multisub.cuh"

namespace vcb {
namespace {

constexpr int kFT = 128;
constexpr int kFMaxW = 64;   // widest layer
constexpr int kFMaxK = 31;   // varying dimensions

struct FlParams {
  int n_fc, dims[VCB_MAX_FC + 1];
  const float* W;
  const float* b;
  long long w_goff[VCB_MAX_FC];
  int b_goff[VCB_MAX_FC];
  int B, K, Q;
  const float *xl, *xh, *specW;
  const int* var_idx;
  float *spec_A, *spec_b, *lb, *A_lo, *A_up, *b_lo, *b_up;
  // leaf fate (vcb_mlp_flirpa_fate), fate == NULL otherwise
  const float* sub_bias;
  const int* sub;
  int clip_iters;
  int* fate;
  float *oxl, *oxh, *score;
};

__global__ void __launch_bounds__(kFT) flirpa_kernel(const FlParams p) {
  __shared__ float lo_s[kFMaxW * (kFMaxK + 1)], up_s[kFMaxW * (kFMaxK + 1)];
  __shared__ float mid_s[kFMaxW * (kFMaxK + 1)], half_s[kFMaxW * (kFMaxK + 1)];
  __shared__ float xmid[kFMaxK], xhalf[kFMaxK], xlc[kFMaxK], xhc[kFMaxK];
  __shared__ float box_lo[kFMaxW], box_hi[kFMaxW];
  __shared__ float lb_sh[kFMaxW];
  const int box = blockIdx.x;
  const int tid = threadIdx.x;
  const int K = p.K, Kp = K + 1;
  const int n0 = p.dims[0];
  const float* xl = p.xl + (long long)box * n0;
  const float* xh = p.xh + (long long)box * n0;
  for (int k = tid; k < K; k += kFT) {
    const float l = xl[p.var_idx[k]], h = xh[p.var_idx[k]];
    xlc[k] = l;
    xhc[k] = h;
    xmid[k] = __fmul_rn(__fadd_rn(l, h), 0.5f);
    xhalf[k] = __fmul_rn(__fsub_rn(h, l), 0.5f);
  }
  // input bounds: identity columns at the varying dimensions, constants in b
  for (int e = tid; e < n0 * Kp; e += kFT) {
    const int i = e / Kp, c = e - i * Kp;
    float v;
    if (c < K) {
      v = p.var_idx[c] == i ? 1.f : 0.f;
    } else {
      bool varying = false;
      for (int k = 0; k < K; ++k) varying |= p.var_idx[k] == i;
      v = varying ? 0.f : xl[i];
    }
    lo_s[e] = v;
    up_s[e] = v;
  }
  __syncthreads();
  for (int l = 0; l < p.n_fc; ++l) {
    const int nin = p.dims[l], nout = p.dims[l + 1];
    const float* W = p.W + p.w_goff[l];
    const float* bias = p.b + p.b_goff[l];
    for (int e = tid; e < nin * Kp; e += kFT) {
      mid_s[e] = __fmul_rn(__fadd_rn(lo_s[e], up_s[e]), 0.5f);
      half_s[e] = __fmul_rn(__fsub_rn(up_s[e], lo_s[e]), 0.5f);
    }
    __syncthreads();
    for (int e = tid; e < nout * Kp; e += kFT) {
      const int o = e / Kp, c = e - o * Kp;
      float m = 0.f, a = 0.f;
      for (int i = 0; i < nin; ++i) {
        const float w = __ldg(W + (long long)o * nin + i);
        m = fmaf(w, mid_s[i * Kp + c], m);
        a = fmaf(fabsf(w), half_s[i * Kp + c], a);
      }
      if (c == K) m = __fadd_rn(m, __ldg(bias + o));
      lo_s[e] = __fsub_rn(m, a);
      up_s[e] = __fadd_rn(m, a);
    }
    __syncthreads();
    // box bounds of this layer's outputs (the relu's pre-activations)
    for (int o = tid; o < nout; o += kFT) {
      float lm = 0.f, la = 0.f, um = 0.f, ua = 0.f;
      for (int k = 0; k < K; ++k) {
        const float al = lo_s[o * Kp + k], au = up_s[o * Kp + k];
        lm = fmaf(al, xmid[k], lm);
        la = fmaf(fabsf(al), xhalf[k], la);
        um = fmaf(au, xmid[k], um);
        ua = fmaf(fabsf(au), xhalf[k], ua);
      }
      box_lo[o] = __fadd_rn(__fsub_rn(lm, la), lo_s[o * Kp + K]);
      box_hi[o] = __fadd_rn(__fadd_rn(um, ua), up_s[o * Kp + K]);
    }
    __syncthreads();
    if (l < p.n_fc - 1) {
      // relu relaxation applied to the rows
      for (int e = tid; e < nout * Kp; e += kFT) {
        const int o = e / Kp, c = e - o * Kp;
        const float lo = box_lo[o], hi = box_hi[o];
        const bool active = lo >= 0.f, dead = hi <= 0.f;
        const float up_slope = __fdiv_rn(hi, fmaxf(__fsub_rn(hi, lo), 1e-12f));
        const float lbs = active ? 1.f : (dead ? 0.f : (up_slope > 0.5f ? 1.f : 0.f));
        const float ubs = active ? 1.f : (dead ? 0.f : up_slope);
        if (c < K) {
          lo_s[e] = __fmul_rn(lbs, lo_s[e]);
          up_s[e] = __fmul_rn(ubs, up_s[e]);
        } else {
          const float ub_int = (!active && !dead) ? __fmul_rn(-up_slope, lo) : 0.f;
          lo_s[e] = __fadd_rn(__fmul_rn(lbs, lo_s[e]), 0.f);
          up_s[e] = __fadd_rn(__fmul_rn(ubs, up_s[e]), ub_int);
        }
      }
      __syncthreads();
    }
  }
  const int nL = p.dims[p.n_fc];
  if (p.A_lo) {
    for (int e = tid; e < nL * Kp; e += kFT) {
      const int o = e / Kp, c = e - o * Kp;
      const long long go = (long long)box * nL + o;
      if (c < K) {
        p.A_lo[go * K + c] = lo_s[e];
        p.A_up[go * K + c] = up_s[e];
      } else {
        p.b_lo[go] = lo_s[e];
        p.b_up[go] = up_s[e];
      }
    }
  }
  // spec contraction over the output neurons, then concretisation
  for (int e = tid; e < p.Q * Kp; e += kFT) {
    const int q = e / Kp, c = e - q * Kp;
    float sp = 0.f, sn = 0.f;
    for (int o = 0; o < nL; ++o) {
      const float w = __ldg(p.specW + q * nL + o);
      sp = fmaf(fmaxf(w, 0.f), lo_s[o * Kp + c], sp);
      sn = fmaf(fminf(w, 0.f), up_s[o * Kp + c], sn);
    }
    mid_s[e] = __fadd_rn(sp, sn);
  }
  __syncthreads();
  for (int q = tid; q < p.Q; q += kFT) {
    float s = 0.f;
    for (int k = 0; k < K; ++k) {
      const float a = mid_s[q * Kp + k];
      s = __fadd_rn(s, __fadd_rn(__fmul_rn(fmaxf(a, 0.f), xlc[k]),
                                 __fmul_rn(fminf(a, 0.f), xhc[k])));
      if (p.spec_A) p.spec_A[((long long)box * p.Q + q) * K + k] = a;
    }
    const float sb = mid_s[q * Kp + K];
    if (p.spec_b) p.spec_b[(long long)box * p.Q + q] = sb;
    lb_sh[q] = __fadd_rn(s, sb);
    if (p.lb) p.lb[(long long)box * p.Q + q] = lb_sh[q];
  }
  if (p.fate) {
    __syncthreads();
    if (tid == 0)
      ms_leaf_fate(box, p.B, n0, K, p.Q, p.clip_iters, p.xl, p.xh, p.var_idx, mid_s, Kp,
                   mid_s + K, Kp, lb_sh, p.sub_bias + (long long)p.sub[box] * p.Q, p.fate,
                   p.oxl, p.oxh, p.score);
  }
}

int flirpa_setup(const vcb_mlp* net, int32_t B, int32_t K, int32_t Q, const char* who,
                 FlParams& p) {
  if (!net || B < 0 || Q < 0) return fail(VCB_ERR_INVALID, "%s: bad arguments", who);
  const int nfc = net->n_fc;
  if (nfc < 1 || nfc > VCB_MAX_FC) return fail(VCB_ERR_UNSUPPORTED, "%s: n_fc=%d", who, nfc);
  for (int l = 0; l <= nfc; ++l)
    if (net->dims[l] < 1 || net->dims[l] > kFMaxW)
      return fail(VCB_ERR_UNSUPPORTED, "%s: width %d outside [1, %d]", who, net->dims[l],
                  kFMaxW);
  if (K < 1 || K > kFMaxK || K > net->dims[0])
    return fail(VCB_ERR_UNSUPPORTED, "%s: K=%d varying dimensions outside [1, %d]", who, K,
                kFMaxK);
  if (Q > kFMaxW) return fail(VCB_ERR_UNSUPPORTED, "%s: Q=%d > %d", who, Q, kFMaxW);
  if (!net->W || !net->b) return fail(VCB_ERR_INVALID, "%s: NULL weights", who);
  p = FlParams{};
  p.n_fc = nfc;
  long long woff = 0;
  int boff = 0;
  for (int l = 0; l <= nfc; ++l) p.dims[l] = net->dims[l];
  for (int l = 0; l < nfc; ++l) {
    p.w_goff[l] = woff;
    p.b_goff[l] = boff;
    woff += (long long)net->dims[l] * net->dims[l + 1];
    boff += net->dims[l + 1];
  }
  p.W = net->W;
  p.b = net->b;
  p.B = B;
  p.K = K;
  p.Q = Q;
  return VCB_OK;
}

}  // namespace
}  // namespace vcb

extern "C" int vcb_mlp_flirpa(const vcb_mlp* net, int32_t B, int32_t K, const float* xl,
                              const float* xh, const int32_t* var_idx, int32_t Q,
                              const float* spec_W, float* spec_A, float* spec_b, float* lb,
                              float* A_lo, float* A_up, float* b_lo, float* b_up,
                              void* stream) {
  using namespace vcb;
  const char* who = "vcb_mlp_flirpa";
  FlParams p;
  int rc = flirpa_setup(net, B, K, Q, who, p);
  if (rc) return rc;
  if (B == 0) return VCB_OK;
  if (!xl || !xh || !var_idx || !lb || (Q > 0 && !spec_W) ||
      ((A_lo == nullptr) != (A_up == nullptr)) || (A_lo && (!b_lo || !b_up)))
    return fail(VCB_ERR_INVALID, "%s: NULL pointer", who);
  p.xl = xl;
  p.xh = xh;
  p.specW = spec_W;
  p.var_idx = var_idx;
  p.spec_A = spec_A;
  p.spec_b = spec_b;
  p.lb = lb;
  p.A_lo = A_lo;
  p.A_up = A_up;
  p.b_lo = b_lo;
  p.b_up = b_up;
  flirpa_kernel<<<B, kFT, 0, static_cast<cudaStream_t>(stream)>>>(p);
  return check_launch(who);
}

extern "C" int vcb_mlp_flirpa_fate(const vcb_mlp* net, int32_t B, int32_t K, const float* xl,
                                   const float* xh, const int32_t* var_idx, int32_t Q,
                                   const float* spec_W, const float* sub_bias,
                                   const int32_t* sub, int32_t clip_iters, int32_t* fate,
                                   float* out_xl, float* out_xh, float* score, void* stream) {
  using namespace vcb;
  const char* who = "vcb_mlp_flirpa_fate";
  FlParams p;
  int rc = flirpa_setup(net, B, K, Q, who, p);
  if (rc) return rc;
  if (Q < 1 || clip_iters < 0)
    return fail(VCB_ERR_INVALID, "%s: Q=%d clip_iters=%d", who, Q, clip_iters);
  if (!fate || !xl || !xh || !var_idx || !spec_W || !sub_bias || !sub || !out_xl || !out_xh ||
      !score)
    return fail(VCB_ERR_INVALID, "%s: NULL pointer", who);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  cudaError_t e = cudaMemsetAsync(fate + B, 0, sizeof(int32_t), st);
  if (e != cudaSuccess) return cuda_fail(e, who);
  if (B == 0) return VCB_OK;
  p.xl = xl;
  p.xh = xh;
  p.specW = spec_W;
  p.var_idx = var_idx;
  p.sub_bias = sub_bias;
  p.sub = sub;
  p.clip_iters = clip_iters;
  p.fate = fate;
  p.oxl = out_xl;
  p.oxh = out_xh;
  p.score = score;
  flirpa_kernel<<<B, kFT, 0, st>>>(p);
  return check_launch(who);
}
