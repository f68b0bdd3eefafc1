// Fused IBP forward + CROWN back-substitution for ReLU MLPs whose weights fit
// in shared memory (ACAS-Xu-sized networks).
//
// One persistent CTA per SM slot walks tiles of TB subdomains.  Per tile:
//   * IBP forward (verify_zono_bnb.py:1066-1153): per fc layer a register-
//     tiled fp32 GEMM of the (TB x n_in) mid/rad tile against the resident
//     weights, with the ReLU clamp / crossing repair and the CROWN slope rule
//     (verify_zono_bnb.py:503-522) fused into the epilogue.  The slopes stay
//     in shared memory, sign-encoded in two floats per neuron.
//   * CROWN back-substitution (verify_zono_bnb.py:4270-5134): the (TB*Q x n)
//     coefficient tile walks the layers in reverse; each step is a GEMM
//     against the same resident weights (bias stored as an extra weight
//     column, so the bias dot falls out of the GEMM), and the ReLU relaxation
//     plus the intercept partial sums are fused into its epilogue.
//   * Concretisation against the input box, optional A / acc outputs.
// Nothing but the inputs, the outputs and the weights touches HBM.
#include <algorithm>

#include "vcb_common.cuh"

namespace vcb {
namespace {

constexpr int kNT = 128;  // threads per CTA

struct CrownParams {
  int n_fc;
  int dims[VCB_MAX_FC + 1];
  const float* W;
  const float* b;
  long long w_goff[VCB_MAX_FC];
  int b_goff[VCB_MAX_FC];
  int w_soff[VCB_MAX_FC];
  int pw[VCB_MAX_FC];
  int wrows[VCB_MAX_FC];
  long long relu_goff[VCB_MAX_FC];
  int sl_soff, ps;
  int act_soff, pa;
  int ew_soff, pe, ew_rows;
  int acc_soff, bd_soff, part_soff, rt_max;
  int x_soff;
  int spec_soff;
  int smem_floats;
  int B, Q, TB, ntiles;
  const float *xl, *xh, *clo, *chi, *sblo, *sbhi, *alpha, *beta, *specW, *specb;
  float *lb, *A, *accout, *sbolo, *sbohi;
};

__device__ __forceinline__ float4 ld4(const float* p) {
  return *reinterpret_cast<const float4*>(p);
}

// CROWN slope rule (verify_zono_bnb.py:511-521), sign-encoded:
//   a = dead ? -up_s : up_s,   c = active ? -0.0f : up_t.
__device__ __forceinline__ void encode_slope(float lo, float hi, float* a,
                                             float* c) {
  const float lb_r = fminf(lo, 0.f);
  float ub_r = fmaxf(hi, 0.f);
  ub_r = fmaxf(ub_r, __fadd_rn(lb_r, 1e-8f));
  const float up_s = __fdiv_rn(ub_r, __fsub_rn(ub_r, lb_r));
  const float up_t = __fmul_rn(-lb_r, up_s);
  const bool active = lo >= 0.f;
  const bool dead = hi <= 0.f;
  *a = dead ? -up_s : up_s;
  *c = active ? -0.0f : up_t;
}

// ReLU backward step for one coefficient e (verify_zono_bnb.py:4409-4449):
// returns ep*lo_s + en*up_s and adds en*up_t to *part.  Exactly one of ep/en
// is non-zero, so the single product below rounds like the reference's sum.
__device__ __forceinline__ float relu_back(float e, float a, float c,
                                           const float* alpha_ptr,
                                           float* part) {
  if (signbit(c)) return e;  // active: identity, zero intercept
  if (signbit(a)) {          // dead (lo_s = 0)
    if (e < 0.f) {
      *part += __fmul_rn(e, c);
      return __fmul_rn(e, -a);
    }
    return 0.f * e;
  }
  // unstable
  if (e < 0.f) {
    *part += __fmul_rn(e, c);
    return __fmul_rn(e, a);
  }
  const float lo_s = alpha_ptr ? *alpha_ptr : (a > 0.5f ? 1.f : 0.f);
  return __fmul_rn(e, lo_s);
}

__global__ void __launch_bounds__(kNT, 2)
    crown_mlp_kernel(const __grid_constant__ CrownParams p) {
  extern __shared__ __align__(16) float sm[];
  const int tid = threadIdx.x;
  const int nfc = p.n_fc;
  const int n0 = p.dims[0];
  const int nL = p.dims[nfc];
  const int Q = p.Q;
  const int TB = p.TB;

  // ---- resident weights: row o of layer l = [W[o,0..n_in), b[o], 0...]
  for (int l = 0; l < nfc; ++l) {
    const int nin = p.dims[l], nout = p.dims[l + 1], pw = p.pw[l];
    const int total = p.wrows[l] * pw;
    float* dst = sm + p.w_soff[l];
    const float* Wg = p.W + p.w_goff[l];
    const float* bg = p.b + p.b_goff[l];
    for (int idx = tid; idx < total; idx += kNT) {
      const int o = idx / pw;
      const int i = idx - o * pw;
      float v = 0.f;
      if (o < nout) v = (i < nin) ? Wg[(long long)o * nin + i] : (i == nin ? bg[o] : 0.f);
      dst[idx] = v;
    }
  }
  if (tid < 8) sm[p.w_soff[nfc - 1] + p.wrows[nfc - 1] * p.pw[nfc - 1] + tid] = 0.f;
  if (Q > 0) {
    float* ssp = sm + p.spec_soff;
    for (int idx = tid; idx < Q * nL; idx += kNT) ssp[idx] = p.specW[idx];
    for (int idx = tid; idx < Q; idx += kNT) ssp[Q * nL + idx] = p.specb[idx];
  }
  __syncthreads();

  float* sXl = sm + p.x_soff;
  float* sXh = sXl + TB * n0;
  const int n0p = pad4(n0);
  const int RT = TB * Q;

  for (int tile = blockIdx.x; tile < p.ntiles; tile += gridDim.x) {
    const int s0 = tile * TB;
    const int nb = min(TB, p.B - s0);
    const long long gbase = (long long)s0 * n0;
    for (int idx = tid; idx < TB * n0; idx += kNT) {
      const bool v = idx < nb * n0;
      sXl[idx] = v ? p.xl[gbase + idx] : 0.f;
      sXh[idx] = v ? p.xh[gbase + idx] : 0.f;
    }

    if (p.sblo == nullptr) {
      // ------------------------------------------------------ IBP forward
      float* mid = sm + p.act_soff;
      float* rad = mid + TB * p.pa;
      for (int idx = tid; idx < TB * n0p; idx += kNT) {
        const int s = idx / n0p, i = idx - s * n0p;
        float m = 0.f, r = 0.f;
        if (s < nb && i < n0) {
          const float l = p.xl[gbase + s * n0 + i], h = p.xh[gbase + s * n0 + i];
          m = __fmul_rn(__fadd_rn(l, h), 0.5f);
          r = __fmul_rn(__fsub_rn(h, l), 0.5f);
        }
        mid[s * p.pa + i] = m;
        rad[s * p.pa + i] = r;
      }
      __syncthreads();
      for (int l = 0; l < nfc - 1; ++l) {
        const int nin = p.dims[l], nout = p.dims[l + 1], pw = p.pw[l];
        const float* sW = sm + p.w_soff[l];
        const int SG = TB >> 1;
        const int G = (nout + 3) >> 2;
        const bool act = tid < SG * G;
        const int sg = tid % SG, og = tid / SG;
        const int kend = pad4(nin);
        float am[2][4], ar[2][4];
#pragma unroll
        for (int s = 0; s < 2; ++s)
#pragma unroll
          for (int j = 0; j < 4; ++j) am[s][j] = ar[s][j] = 0.f;
        if (act) {
          const float* w0 = sW + og * pw;
          const float* m0 = mid + sg * p.pa;
          const float* m1 = mid + (sg + SG) * p.pa;
          const float* r0 = rad + sg * p.pa;
          const float* r1 = rad + (sg + SG) * p.pa;
          const int gstride = G * pw;
          for (int k = 0; k < kend; k += 4) {
            float4 w[4];
#pragma unroll
            for (int j = 0; j < 4; ++j) w[j] = ld4(w0 + j * gstride + k);
            const float4 M0 = ld4(m0 + k), M1 = ld4(m1 + k);
            const float4 R0 = ld4(r0 + k), R1 = ld4(r1 + k);
#pragma unroll
            for (int j = 0; j < 4; ++j) {
              am[0][j] = fmaf(M0.x, w[j].x, am[0][j]);
              am[0][j] = fmaf(M0.y, w[j].y, am[0][j]);
              am[0][j] = fmaf(M0.z, w[j].z, am[0][j]);
              am[0][j] = fmaf(M0.w, w[j].w, am[0][j]);
              am[1][j] = fmaf(M1.x, w[j].x, am[1][j]);
              am[1][j] = fmaf(M1.y, w[j].y, am[1][j]);
              am[1][j] = fmaf(M1.z, w[j].z, am[1][j]);
              am[1][j] = fmaf(M1.w, w[j].w, am[1][j]);
              const float ax = fabsf(w[j].x), ay = fabsf(w[j].y);
              const float az = fabsf(w[j].z), aw = fabsf(w[j].w);
              ar[0][j] = fmaf(R0.x, ax, ar[0][j]);
              ar[0][j] = fmaf(R0.y, ay, ar[0][j]);
              ar[0][j] = fmaf(R0.z, az, ar[0][j]);
              ar[0][j] = fmaf(R0.w, aw, ar[0][j]);
              ar[1][j] = fmaf(R1.x, ax, ar[1][j]);
              ar[1][j] = fmaf(R1.y, ay, ar[1][j]);
              ar[1][j] = fmaf(R1.z, az, ar[1][j]);
              ar[1][j] = fmaf(R1.w, aw, ar[1][j]);
            }
          }
        }
        __syncthreads();
        if (act) {
          float* slA = sm + p.sl_soff + l * 2 * TB * p.ps;
          float* slC = slA + TB * p.ps;
          const long long goff = p.relu_goff[l];
#pragma unroll
          for (int s = 0; s < 2; ++s) {
            const int row = sg + s * SG;
#pragma unroll
            for (int j = 0; j < 4; ++j) {
              const int o = og + G * j;
              float mo = 0.f, ro = 0.f;
              if (row < nb && o < nout) {
                const float mc = __fadd_rn(am[s][j], sW[o * pw + nin]);
                const float rc = ar[s][j];
                float lo = __fsub_rn(mc, rc);
                float hi = __fadd_rn(mc, rc);
                const long long gi = goff + (long long)(s0 + row) * nout + o;
                if (p.clo) {
                  lo = fmaxf(lo, p.clo[gi]);
                  hi = fminf(hi, p.chi[gi]);
                }
                hi = fmaxf(hi, lo);
                if (p.sbolo) {
                  p.sbolo[gi] = lo;
                  p.sbohi[gi] = hi;
                }
                float a, c;
                encode_slope(lo, hi, &a, &c);
                slA[row * p.ps + o] = a;
                slC[row * p.ps + o] = c;
                const float lc = fmaxf(lo, 0.f), hc = fmaxf(hi, 0.f);
                mo = __fmul_rn(__fadd_rn(lc, hc), 0.5f);
                ro = __fmul_rn(__fsub_rn(hc, lc), 0.5f);
              } else if (o < nout) {
                slA[row * p.ps + o] = 0.f;
                slC[row * p.ps + o] = 0.f;
              }
              mid[row * p.pa + o] = mo;
              rad[row * p.pa + o] = ro;
            }
          }
        }
        __syncthreads();
      }
    } else {
      // --------------------------------- caller-supplied intermediate bounds
      for (int L = 0; L < nfc - 1; ++L) {
        const int n = p.dims[L + 1];
        float* slA = sm + p.sl_soff + L * 2 * TB * p.ps;
        float* slC = slA + TB * p.ps;
        const long long goff = p.relu_goff[L] + (long long)s0 * n;
        for (int idx = tid; idx < TB * n; idx += kNT) {
          const int s = idx / n, c = idx - s * n;
          float a = 0.f, cc = 0.f;
          if (s < nb) encode_slope(p.sblo[goff + idx], p.sbhi[goff + idx], &a, &cc);
          slA[s * p.ps + c] = a;
          slC[s * p.ps + c] = cc;
        }
      }
      __syncthreads();
    }

    if (Q > 0) {
      // --------------------------------------------- CROWN back-substitution
      float* ew = sm + p.ew_soff;
      float* sAcc = sm + p.acc_soff;
      float* sBd = sm + p.bd_soff;
      float* sPart = sm + p.part_soff;
      const float* ssp = sm + p.spec_soff;
      for (int idx = tid; idx < p.ew_rows * p.pe; idx += kNT) {
        const int r = idx / p.pe, o = idx - r * p.pe;
        float v = 0.f;
        if (r < nb * Q && o < nL) v = ssp[(r % Q) * nL + o];
        ew[idx] = v;
      }
      for (int r = tid; r < RT; r += kNT) sAcc[r] = (r < nb * Q) ? ssp[Q * nL + r % Q] : 0.f;
      __syncthreads();
      const int RG = (RT + 3) >> 2;
      for (int l = nfc - 1; l >= 0; --l) {
        const int nin = p.dims[l], nout = p.dims[l + 1], pw = p.pw[l];
        const float* sW = sm + p.w_soff[l];
        const int CG = (nin + 1 + 7) >> 3;
        const bool act = tid < RG * CG;
        const int rg = tid % RG, cg = tid / RG;
        const int kend = pad4(nout);
        float acc[4][8];
#pragma unroll
        for (int j = 0; j < 4; ++j)
#pragma unroll
          for (int c = 0; c < 8; ++c) acc[j][c] = 0.f;
        if (act) {
          const float* e0 = ew + rg * p.pe;
          const int rstride = RG * p.pe;
          const float* wcol = sW + 8 * cg;
          for (int k = 0; k < kend; k += 4) {
            float4 e[4];
#pragma unroll
            for (int j = 0; j < 4; ++j) e[j] = ld4(e0 + j * rstride + k);
#pragma unroll
            for (int kk = 0; kk < 4; ++kk) {
              const float4 wa = ld4(wcol + (k + kk) * pw);
              const float4 wb = ld4(wcol + (k + kk) * pw + 4);
#pragma unroll
              for (int j = 0; j < 4; ++j) {
                const float ev = kk == 0 ? e[j].x : kk == 1 ? e[j].y : kk == 2 ? e[j].z : e[j].w;
                acc[j][0] = fmaf(ev, wa.x, acc[j][0]);
                acc[j][1] = fmaf(ev, wa.y, acc[j][1]);
                acc[j][2] = fmaf(ev, wa.z, acc[j][2]);
                acc[j][3] = fmaf(ev, wa.w, acc[j][3]);
                acc[j][4] = fmaf(ev, wb.x, acc[j][4]);
                acc[j][5] = fmaf(ev, wb.y, acc[j][5]);
                acc[j][6] = fmaf(ev, wb.z, acc[j][6]);
                acc[j][7] = fmaf(ev, wb.w, acc[j][7]);
              }
            }
          }
        }
        __syncthreads();
        if (act) {
          const int L = l - 1;  // relu feeding fc l
          const float* slA = sm + p.sl_soff + (L < 0 ? 0 : L) * 2 * TB * p.ps;
          const float* slC = slA + TB * p.ps;
          const long long goff = L < 0 ? 0 : p.relu_goff[L];
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            const int r = rg + RG * j;
            if (r >= RT) continue;
            const bool rv = r < nb * Q;
            const int s = r / Q;
            float part = 0.f;
#pragma unroll
            for (int c8 = 0; c8 < 8; ++c8) {
              const int c = 8 * cg + c8;
              float v = acc[j][c8];
              if (c < nin) {
                if (!rv) {
                  v = 0.f;
                } else if (L >= 0) {
                  const long long gi = goff + (long long)(s0 + s) * nin + c;
                  v = relu_back(v, slA[s * p.ps + c], slC[s * p.ps + c],
                                p.alpha ? p.alpha + gi : nullptr, &part);
                  if (p.beta) v = __fadd_rn(v, p.beta[gi]);
                }
                ew[r * p.pe + c] = v;
              } else if (c == nin) {
                sBd[r] = rv ? v : 0.f;
                if (c < p.pe) ew[r * p.pe + c] = 0.f;
              } else if (c < p.pe) {
                ew[r * p.pe + c] = 0.f;
              }
            }
            sPart[cg * p.rt_max + r] = part;
          }
        }
        __syncthreads();
        for (int r = tid; r < RT; r += kNT) {
          float a = __fadd_rn(sAcc[r], sBd[r]);
          if (l > 0) {
            float ps = 0.f;
            for (int g = 0; g < CG; ++g) ps = __fadd_rn(ps, sPart[g * p.rt_max + r]);
            a = __fadd_rn(a, ps);
          }
          sAcc[r] = a;
        }
        // the next GEMM reads only ew (written before the barrier above); the
        // next epilogue's writes to sBd/sPart happen after its own barrier.
      }
      __syncthreads();
      // --------------------------------------------------- concretisation
      for (int r = tid; r < nb * Q; r += kNT) {
        const int s = r / Q;
        const float* e = ew + r * p.pe;
        const float* xls = sXl + s * n0;
        const float* xhs = sXh + s * n0;
        float s1 = 0.f, s2 = 0.f;
        for (int i = 0; i < n0; ++i) {
          const float ei = e[i];
          s1 = fmaf(fmaxf(ei, 0.f), xls[i], s1);
          s2 = fmaf(fminf(ei, 0.f), xhs[i], s2);
        }
        const long long go = (long long)s0 * Q + r;
        const float accv = sAcc[r];
        p.lb[go] = __fadd_rn(__fadd_rn(accv, s1), s2);
        if (p.accout) p.accout[go] = accv;
        if (p.A) {
          float* Ar = p.A + go * n0;
          for (int i = 0; i < n0; ++i) Ar[i] = e[i];
        }
      }
    }
    __syncthreads();
  }
}

struct Layout {
  CrownParams p;
  int bytes;
};

// Computes the shared-memory layout for tile size TB; returns false when a
// phase would need more than one work item per thread.
bool make_layout(const vcb_mlp* net, int TB, int Q, Layout* out) {
  CrownParams& p = out->p;
  const int nfc = net->n_fc;
  int off = 0;
  int max_relu = 1, max_in1 = 1, max_w = 1, cg_max = 1, g_max = 1;
  for (int l = 0; l < nfc; ++l) {
    const int nin = net->dims[l], nout = net->dims[l + 1];
    p.pw[l] = pad4odd(nin + 1);
    p.wrows[l] = pad4(nout);
    p.w_soff[l] = off;
    off += p.wrows[l] * p.pw[l];
    max_in1 = std::max(max_in1, nin + 1);
    max_w = std::max(max_w, nin);
    cg_max = std::max(cg_max, (nin + 1 + 7) / 8);
    if (l < nfc - 1) {
      max_relu = std::max(max_relu, nout);
      g_max = std::max(g_max, (nout + 3) / 4);
    }
  }
  max_in1 = std::max(max_in1, net->dims[nfc] + 1);
  off += 8;
  off = pad4(off);
  p.sl_soff = off;
  p.ps = pad4(max_relu);
  off += (nfc - 1) * 2 * TB * p.ps;
  const int SG = TB / 2;
  if (nfc > 1 && SG * g_max > kNT) return false;
  const int RT = TB * Q;
  const int RG = (RT + 3) / 4;
  if (Q > 0 && RG * cg_max > kNT) return false;
  p.pa = pad4odd(std::max(max_w, net->dims[0]));
  p.pe = pad4odd(max_in1);
  p.ew_rows = 4 * RG;
  const int fwd = 2 * TB * p.pa;
  const int bwd = Q > 0 ? p.ew_rows * p.pe : 0;
  p.act_soff = p.ew_soff = off;
  off += pad4(std::max(fwd, bwd));
  p.rt_max = pad4(std::max(RT, 1));
  p.acc_soff = off;
  off += p.rt_max;
  p.bd_soff = off;
  off += p.rt_max;
  p.part_soff = off;
  off += cg_max * p.rt_max;
  p.x_soff = off;
  off += pad4(2 * TB * net->dims[0]);
  p.spec_soff = off;
  off += pad4(Q * net->dims[nfc] + Q);
  p.smem_floats = off;
  out->bytes = off * 4;
  return true;
}

}  // namespace
}  // namespace vcb

extern "C" int vcb_mlp_crown(const vcb_mlp* net, int32_t B, const float* xl,
                             const float* xh, const float* clamp_lo,
                             const float* clamp_hi, const float* sb_in_lo,
                             const float* sb_in_hi, const float* alpha,
                             const float* beta, int32_t Q, const float* spec_W,
                             const float* spec_b, float* lb, float* A,
                             float* acc, float* sb_out_lo, float* sb_out_hi,
                             void* stream) {
  using namespace vcb;
  if (!net) return fail(VCB_ERR_INVALID, "vcb_mlp_crown: net is NULL");
  const int nfc = net->n_fc;
  if (nfc < 1 || nfc > VCB_MAX_FC)
    return fail(VCB_ERR_UNSUPPORTED, "vcb_mlp_crown: n_fc=%d outside [1,%d]", nfc, VCB_MAX_FC);
  for (int l = 0; l <= nfc; ++l)
    if (net->dims[l] <= 0)
      return fail(VCB_ERR_INVALID, "vcb_mlp_crown: dims[%d]=%d", l, net->dims[l]);
  if (B < 0 || Q < 0) return fail(VCB_ERR_INVALID, "vcb_mlp_crown: B=%d Q=%d", B, Q);
  if (!net->W || !net->b || (B > 0 && (!xl || !xh)))
    return fail(VCB_ERR_INVALID, "vcb_mlp_crown: NULL weight or box pointer");
  if ((clamp_lo == nullptr) != (clamp_hi == nullptr) ||
      (sb_in_lo == nullptr) != (sb_in_hi == nullptr) ||
      (sb_out_lo == nullptr) != (sb_out_hi == nullptr))
    return fail(VCB_ERR_INVALID, "vcb_mlp_crown: lo/hi pointers must be given in pairs");
  if (Q > 0 && (!spec_W || !spec_b || !lb))
    return fail(VCB_ERR_INVALID, "vcb_mlp_crown: Q>0 needs spec_W, spec_b and lb");
  if (sb_in_lo && (clamp_lo || sb_out_lo))
    return fail(VCB_ERR_INVALID, "vcb_mlp_crown: sb_in excludes clamps and sb_out");
  if (B == 0) return VCB_OK;

  // Largest even tile that keeps one work item per thread and fits two CTAs
  // per SM; otherwise one CTA per SM.
  Layout lay{};
  bool found = false;
  const int two_cta = (233472 - 2 * 1024) / 2;
  const int one_cta = 232448;
  for (int pass = 0; pass < 2 && !found; ++pass) {
    const int limit = pass == 0 ? two_cta : one_cta;
    for (int TB = 16; TB >= 2; TB -= 2) {
      Layout t{};
      if (make_layout(net, TB, Q, &t) && t.bytes <= limit) {
        lay = t;
        lay.p.TB = TB;
        found = true;
        break;
      }
    }
  }
  if (!found)
    return fail(VCB_ERR_UNSUPPORTED,
                "vcb_mlp_crown: network does not fit the shared-memory-resident kernel");
  CrownParams& p = lay.p;
  p.n_fc = nfc;
  long long woff = 0;
  int boff = 0;
  long long roff = 0;
  for (int l = 0; l <= nfc; ++l) p.dims[l] = net->dims[l];
  for (int l = 0; l < nfc; ++l) {
    p.w_goff[l] = woff;
    p.b_goff[l] = boff;
    woff += (long long)net->dims[l] * net->dims[l + 1];
    boff += net->dims[l + 1];
    if (l < nfc - 1) {
      p.relu_goff[l] = roff;
      roff += (long long)B * net->dims[l + 1];
    }
  }
  p.W = net->W;
  p.b = net->b;
  p.B = B;
  p.Q = Q;
  p.ntiles = (B + p.TB - 1) / p.TB;
  p.xl = xl;
  p.xh = xh;
  p.clo = clamp_lo;
  p.chi = clamp_hi;
  p.sblo = sb_in_lo;
  p.sbhi = sb_in_hi;
  p.alpha = alpha;
  p.beta = beta;
  p.specW = spec_W;
  p.specb = spec_b;
  p.lb = lb;
  p.A = A;
  p.accout = acc;
  p.sbolo = sb_out_lo;
  p.sbohi = sb_out_hi;

  int rc = ensure_smem(reinterpret_cast<const void*>(crown_mlp_kernel), lay.bytes);
  if (rc) return rc;
  int per_sm = 0;
  cudaError_t e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(
      &per_sm, crown_mlp_kernel, kNT, lay.bytes);
  if (e != cudaSuccess) return cuda_fail(e, "vcb_mlp_crown: occupancy");
  if (per_sm < 1) per_sm = 1;
  const int grid = std::min(p.ntiles, sm_count() * per_sm);
  crown_mlp_kernel<<<grid, kNT, lay.bytes, static_cast<cudaStream_t>(stream)>>>(p);
  return check_launch("vcb_mlp_crown: launch");
}
