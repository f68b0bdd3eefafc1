// Layer-wise bound propagation for ReLU MLPs too wide for the
// shared-memory-resident kernels (e.g. 784 -> [256] x 6 -> 10).
//
// Every layer is one launch of a tiled fp32 GEMM (128 x 64 tiles, 256
// threads, 8 x 4 register tiles, double-buffered shared-memory k-slices)
// whose epilogue carries the layer's bound arithmetic:
//   * IBP (verify_zono_bnb.py:1115-1138): mid @ W^T and rad @ |W|^T in one
//     pass, bias, clamps, crossing repair, bounds out, relu'd mid/rad out;
//   * CROWN back-substitution (verify_zono_bnb.py:4379-4453): coef @ [W | b]
//     with the ReLU relaxation (min-area or alpha lower slope) of the
//     preceding layer, the raw coefficients recorded for the alpha adjoint,
//     and per-tile intercept partial sums (reduced later in a fixed order);
//   * alpha adjoint: g @ W^T + b with the derivative of the relaxation, the
//     hand-written counterpart of autograd through the back-substitution
//     (clamp(min=0) and clamp(max=0) both pass gradient at 0).
// Small kernels finish the row sums, concretise against the input box, reduce
// d(sum lb)/d(alpha) over the spec rows of each domain and run Adam + clamp.
// All row-major buffers have leading dimensions that are multiples of 4.
#include <algorithm>
#include <cmath>

#include "vcb_common.cuh"
#include "vcb_gemm.cuh"

namespace vcb {
namespace {


// Relaxation of one neuron from its pre-activation bounds
// (verify_zono_bnb.py:511-521, 4413-4433): multiplier for e >= 0 (lower
// slope; alpha for unstable neurons when given), for e < 0 (upper slope) and
// the intercept factor (applied to min(e, 0)).
struct Relax {
  float pos, neg, icp;
  bool unstable;
};

__device__ __forceinline__ Relax relax_of(float lo, float hi, const float* alpha) {
  Relax r;
  const float lb_r = fminf(lo, 0.f);
  float ub_r = fmaxf(hi, 0.f);
  ub_r = fmaxf(ub_r, __fadd_rn(lb_r, 1e-8f));
  const float up_s = __fdiv_rn(ub_r, __fsub_rn(ub_r, lb_r));
  const float up_t = __fmul_rn(-lb_r, up_s);
  const bool active = lo >= 0.f, dead = hi <= 0.f;
  r.unstable = !active && !dead;
  r.neg = up_s;
  r.icp = up_t;
  if (active) r.pos = 1.f;
  else if (dead) r.pos = 0.f;
  else r.pos = alpha ? *alpha : (up_s > 0.5f ? 1.f : 0.f);
  return r;
}

// ---------------------------------------------------------------------------
// IBP layer: mid/rad (D x n_in, ld lda) -> bounds and relu'd mid/rad out.
// ---------------------------------------------------------------------------
struct IbpArgs {
  int D, nin, nout, lda, ldo;
  const float *mid, *rad, *W, *Wabs, *b, *clo, *chi;  // W, Wabs: nout x nin (ld nin)
  float *sblo, *sbhi, *mid_o, *rad_o;                 // sb: D x nout; mid_o/rad_o: D x ldo
};

// RM rows per thread ((16 RM) x 64 CTA tiles): the host takes the largest
// RM whose grid still gives every SM a tile.
template <int RM>
__global__ void __launch_bounds__(GT) ibp_layer_kernel(const IbpArgs a) {
  extern __shared__ __align__(16) float smem[];
  float acc[RM][4], acc2[RM][4];
  mainloop_rm<true, RM>(a.D, a.nout, a.nin, RowLoad{a.mid, a.lda}, RowLoad{a.W, a.nin},
                        RowLoad{a.rad, a.lda}, RowLoad{a.Wabs, a.nin}, acc, acc2, smem);
  const int ty = threadIdx.x >> 4, tx = threadIdx.x & 15;
  const int m0 = blockIdx.x * (16 * RM) + ty * RM, n0 = blockIdx.y * TN + tx * 4;
#pragma unroll
  for (int i = 0; i < RM; ++i) {
    const int m = m0 + i;
    if (m >= a.D) continue;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int n = n0 + j;
      if (n >= a.nout) continue;
      const float mc = __fadd_rn(acc[i][j], a.b[n]);
      const float rc = acc2[i][j];
      float lo = __fsub_rn(mc, rc), hi = __fadd_rn(mc, rc);
      const long long gi = (long long)m * a.nout + n;
      if (a.clo) {
        lo = fmaxf(lo, a.clo[gi]);
        hi = fminf(hi, a.chi[gi]);
      }
      hi = fmaxf(hi, lo);
      if (a.sblo) {
        a.sblo[gi] = lo;
        a.sbhi[gi] = hi;
      }
      if (a.mid_o) {
        const float lc = fmaxf(lo, 0.f), hc = fmaxf(hi, 0.f);
        a.mid_o[(long long)m * a.ldo + n] = __fmul_rn(__fadd_rn(lc, hc), 0.5f);
        a.rad_o[(long long)m * a.ldo + n] = __fmul_rn(__fsub_rn(hc, lc), 0.5f);
      }
    }
  }
}

// ---------------------------------------------------------------------------
// CROWN backward layer: t = coef (R x nout, ld ldc) @ [W | b] -> coef_o
// (R x nin, ld ldo) after the relaxation of relu layer L (bounds sb of box
// r / Q), raw coefficients to rec (R x nin, ld ldo) when given, the bias dot
// to bd (R), intercept partial sums to part (R x gridDim.y).
// ---------------------------------------------------------------------------
struct BackArgs {
  int R, Q, nin, nout, ldc, ldo;
  const float *coef, *Waug;   // Waug: nout x (nin + 1), ld lda_w
  int ldw;
  const float *sblo, *sbhi, *alpha, *beta;  // (R / Q) x nin, or NULL (no relu)
  float *coef_o, *rec, *bd, *part;
  int alpha_rows;             // alpha is R x nin (one per spec row) instead
};

__global__ void __launch_bounds__(GT) crown_back_kernel(const BackArgs a) {
  extern __shared__ __align__(16) float smem[];
  float acc[8][4], acc2[8][4];
  mainloop<false>(a.R, a.nin + 1, a.nout, RowLoad{a.coef, a.ldc}, ColLoad{a.Waug, a.ldw},
                  RowLoad{nullptr, 0}, ColLoad{nullptr, 0}, acc, acc2, smem);
  const int ty = threadIdx.x >> 4, tx = threadIdx.x & 15;
  const int m0 = blockIdx.x * TM + ty * 8, n0 = blockIdx.y * TN + tx * 4;
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const int m = m0 + i;
    float pt = 0.f;
    if (m < a.R) {
      const int box = m / a.Q;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int n = n0 + j;
        const float v = acc[i][j];
        if (n < a.nin) {
          float o = v;
          if (a.sblo) {
            const long long gi = (long long)box * a.nin + n;
            const long long ai = a.alpha_rows ? (long long)m * a.nin + n : gi;
            const Relax r = relax_of(a.sblo[gi], a.sbhi[gi], a.alpha ? a.alpha + ai : nullptr);
            if (a.rec) a.rec[(long long)m * a.ldo + n] = v;
            if (v < 0.f) {
              pt = fmaf(v, r.icp, pt);
              o = __fmul_rn(v, r.neg);
            } else {
              o = __fmul_rn(v, r.pos);
            }
            if (a.beta) o = __fadd_rn(o, a.beta[gi]);
          }
          a.coef_o[(long long)m * a.ldo + n] = o;
        } else if (n == a.nin) {
          a.bd[m] = v;
        } else if (n < a.ldo) {
          a.coef_o[(long long)m * a.ldo + n] = 0.f;
        }
      }
    }
    // reduce the intercept partials of row m over the 16 column threads
    for (int off = 8; off > 0; off >>= 1) pt += __shfl_xor_sync(0xffffffffu, pt, off, 16);
    if (tx == 0 && m < a.R) a.part[(long long)m * gridDim.y + blockIdx.y] = pt;
  }
}

// acc[r] = (acc[r] + bd[r]) + sum_t part[r][t]  (fixed order)
__global__ void rowsum_kernel(int R, int nparts, int with_part, const float* bd,
                              const float* part, float* acc) {
  for (int r = blockIdx.x * blockDim.x + threadIdx.x; r < R; r += gridDim.x * blockDim.x) {
    float a = __fadd_rn(acc[r], bd[r]);
    if (with_part) {
      float s = 0.f;
      for (int t = 0; t < nparts; ++t) s = __fadd_rn(s, part[(long long)r * nparts + t]);
      a = __fadd_rn(a, s);
    }
    acc[r] = a;
  }
}

// lb[r] = acc[r] + sum_i pos(e)*xl[box] + sum_i neg(e)*xh[box]; optional A
// copy and the adjoint seed g0 = d lb / d e = xl [e >= 0] + xh [e <= 0].
__global__ void concretize_kernel(int R, int Q, int n0, int lde, const float* e,
                                  const float* acc, const float* xl, const float* xh,
                                  float* lb, float* A, float* g0) {
  const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  const int nwarps = (gridDim.x * blockDim.x) >> 5;
  for (int r = warp; r < R; r += nwarps) {
    const int box = r / Q;
    float s1 = 0.f, s2 = 0.f;
    for (int i = lane; i < n0; i += 32) {
      const float ei = e[(long long)r * lde + i];
      const float l = xl[(long long)box * n0 + i], h = xh[(long long)box * n0 + i];
      s1 = fmaf(fmaxf(ei, 0.f), l, s1);
      s2 = fmaf(fminf(ei, 0.f), h, s2);
      if (A) A[(long long)r * n0 + i] = ei;
      if (g0) g0[(long long)r * lde + i] = (ei >= 0.f ? l : 0.f) + (ei <= 0.f ? h : 0.f);
    }
    for (int off = 16; off > 0; off >>= 1) {
      s1 += __shfl_xor_sync(0xffffffffu, s1, off);
      s2 += __shfl_xor_sync(0xffffffffu, s2, off);
    }
    if (lane == 0) lb[r] = __fadd_rn(__fadd_rn(acc[r], s1), s2);
  }
}

// ---------------------------------------------------------------------------
// alpha adjoint layer: ga = g (R x nin, ld ldg) @ W^T + b  (R x nout) is
// d(sum lb)/d(coefficient after relu L's relaxation); with rec (the raw
// coefficient entering that relaxation) it gives
//   dcontrib[r][j] = [unstable] * max(e, 0) * ga            (alpha gradient)
//   dbeta[r][j]    = ga                                      (beta gradient)
//   g_o[r][j] = [e >= 0] pos * ga + [e <= 0] (neg * ga + icp).
// ---------------------------------------------------------------------------
struct AdjArgs {
  int R, Q, nin, nout, ldg, ldo;
  const float *g, *W, *b;       // W: nout x nin (ld nin)
  const float *rec, *sblo, *sbhi, *alpha;  // rec: R x nout (ld ldo); sb/alpha (R/Q) x nout
  float *g_o, *dcontrib;        // R x nout (ld ldo)
  float* dbeta;                 // R x nout (ld ldo): d lb / d beta = ga, or NULL
  int alpha_rows;               // alpha is R x nout (one per spec row) instead
};

__global__ void __launch_bounds__(GT) alpha_adjoint_kernel(const AdjArgs a) {
  extern __shared__ __align__(16) float smem[];
  float acc[8][4], acc2[8][4];
  mainloop<false>(a.R, a.nout, a.nin, RowLoad{a.g, a.ldg}, RowLoad{a.W, a.nin},
                  RowLoad{nullptr, 0}, RowLoad{nullptr, 0}, acc, acc2, smem);
  const int ty = threadIdx.x >> 4, tx = threadIdx.x & 15;
  const int m0 = blockIdx.x * TM + ty * 8, n0 = blockIdx.y * TN + tx * 4;
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const int m = m0 + i;
    if (m >= a.R) continue;
    const int box = m / a.Q;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int n = n0 + j;
      if (n >= a.nout) {
        if (n < a.ldo) a.g_o[(long long)m * a.ldo + n] = 0.f;
        continue;
      }
      const float ga = __fadd_rn(acc[i][j], a.b[n]);
      const long long gi = (long long)box * a.nout + n;
      const float e = a.rec[(long long)m * a.ldo + n];
      const long long ai = a.alpha_rows ? (long long)m * a.nout + n : gi;
      const Relax r = relax_of(a.sblo[gi], a.sbhi[gi], a.alpha ? a.alpha + ai : nullptr);
      a.dcontrib[(long long)m * a.ldo + n] = r.unstable ? __fmul_rn(fmaxf(e, 0.f), ga) : 0.f;
      // beta is added after the relaxation, so its gradient is the adjoint itself
      if (a.dbeta) a.dbeta[(long long)m * a.ldo + n] = ga;
      float go = 0.f;
      if (e >= 0.f) go = __fmul_rn(r.pos, ga);
      if (e <= 0.f) go = __fadd_rn(go, __fadd_rn(__fmul_rn(r.neg, ga), r.icp));
      a.g_o[(long long)m * a.ldo + n] = go;
    }
  }
}

// grad[box][j] = sum_q dcontrib[box*Q + q][j]; then Adam (torch defaults
// betas (0.9, 0.999), eps 1e-8) on the loss -sum(lb), and clamp to [0, 1].
__global__ void alpha_adam_kernel(int D, int Q, int n, int ldc, const float* dcontrib,
                                  float* alpha, float* m1, float* m2, float step_size,
                                  float bc2_sqrt) {
  const long long total = (long long)D * n;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total;
       i += (long long)gridDim.x * blockDim.x) {
    const long long box = i / n;
    const int j = (int)(i - box * n);
    float gsum = 0.f;
    for (int q = 0; q < Q; ++q) gsum = __fadd_rn(gsum, dcontrib[(box * Q + q) * ldc + j]);
    const float g = -gsum;
    // torch's foreach Adam: m.lerp_(g, 0.1); v = v*0.999 + 0.001*g*g;
    // p -= step_size * m / (sqrt(v)/sqrt(bias_correction2) + eps)
    const float mm = __fadd_rn(m1[i], __fmul_rn(0.1f, __fsub_rn(g, m1[i])));
    const float vv = __fadd_rn(__fmul_rn(m2[i], 0.999f), __fmul_rn(__fmul_rn(g, g), 0.001f));
    m1[i] = mm;
    m2[i] = vv;
    const float denom = __fadd_rn(__fdiv_rn(sqrtf(vv), bc2_sqrt), 1e-8f);
    const float p = __fsub_rn(alpha[i], __fmul_rn(step_size, __fdiv_rn(mm, denom)));
    alpha[i] = fminf(fmaxf(p, 0.f), 1.f);
  }
}

int smem_bytes(bool dual) { return gemm_smem_bytes(dual); }

int grid1(long long n) {
  return (int)std::max<long long>(1, std::min<long long>((n + 255) / 256, 8LL * sm_count()));
}

}  // namespace
}  // namespace vcb

using namespace vcb;

extern "C" int vcb_wide_ibp_layer(int32_t D, int32_t nin, int32_t nout, const float* mid,
                                  const float* rad, int32_t lda, const float* W,
                                  const float* Wabs, const float* b, const float* clo,
                                  const float* chi, float* sb_lo, float* sb_hi,
                                  float* mid_o, float* rad_o, int32_t ldo, void* stream) {
  if (D < 0 || nin <= 0 || nout <= 0) return fail(VCB_ERR_INVALID, "vcb_wide_ibp_layer: shape");
  if (D == 0) return VCB_OK;
  if (!mid || !rad || !W || !Wabs || !b || (lda & 3) || (mid_o && (ldo & 3)))
    return fail(VCB_ERR_INVALID, "vcb_wide_ibp_layer: NULL pointer or ld not a multiple of 4");
  IbpArgs a{D, nin, nout, lda, ldo, mid, rad, W, Wabs, b, clo, chi, sb_lo, sb_hi, mid_o, rad_o};
  auto launch = [&](auto kernel, int rm) {
    const int sm = gemm_smem_bytes(true, rm);
    const int rc = ensure_smem(reinterpret_cast<const void*>(kernel), sm);
    if (rc) return rc;
    kernel<<<gemm_grid(D, nout, rm), GT, sm, static_cast<cudaStream_t>(stream)>>>(a);
    return check_launch("vcb_wide_ibp_layer");
  };
  // the largest row tile whose grid still covers every SM (short batches of
  // domains would otherwise leave most SMs idle through the whole K loop)
  auto ctas = [&](int rm) {
    const dim3 g = gemm_grid(D, nout, rm);
    return (long long)g.x * g.y;
  };
  if (ctas(8) >= sm_count()) return launch(ibp_layer_kernel<8>, 8);
  if (ctas(2) >= sm_count()) return launch(ibp_layer_kernel<2>, 2);
  return launch(ibp_layer_kernel<1>, 1);
}

extern "C" int vcb_wide_back_layer(int32_t R, int32_t Q, int32_t nin, int32_t nout,
                                   const float* coef, int32_t ldc, const float* Waug,
                                   int32_t ldw, const float* sb_lo, const float* sb_hi,
                                   const float* alpha, int32_t alpha_rows, const float* beta,
                                   float* coef_o, float* rec, int32_t ldo, float* bd,
                                   float* part, void* stream) {
  if (R < 0 || Q <= 0 || nin <= 0 || nout <= 0)
    return fail(VCB_ERR_INVALID, "vcb_wide_back_layer: shape");
  if (R == 0) return VCB_OK;
  if (!coef || !Waug || !coef_o || !bd || !part || (ldc & 3) || (ldo & 3) || ldw < nin + 1 ||
      ldo < nin + 1)
    return fail(VCB_ERR_INVALID, "vcb_wide_back_layer: NULL pointer or bad leading dimension");
  BackArgs a{R, Q, nin, nout, ldc, ldo, coef, Waug, ldw, sb_lo, sb_hi, alpha, beta,
             coef_o, rec, bd, part, alpha_rows};
  const int sm = smem_bytes(false);
  int rc = ensure_smem(reinterpret_cast<const void*>(crown_back_kernel), sm);
  if (rc) return rc;
  crown_back_kernel<<<gemm_grid(R, nin + 1), GT, sm, static_cast<cudaStream_t>(stream)>>>(a);
  return check_launch("vcb_wide_back_layer");
}

extern "C" int vcb_wide_back_parts(int32_t R, int32_t nin) {
  (void)R;
  return (nin + 1 + TN - 1) / TN;
}

extern "C" int vcb_wide_rowsum(int32_t R, int32_t nparts, int32_t with_part, const float* bd,
                               const float* part, float* acc, void* stream) {
  if (R < 0) return fail(VCB_ERR_INVALID, "vcb_wide_rowsum: R");
  if (R == 0) return VCB_OK;
  rowsum_kernel<<<grid1(R), 256, 0, static_cast<cudaStream_t>(stream)>>>(R, nparts, with_part,
                                                                         bd, part, acc);
  return check_launch("vcb_wide_rowsum");
}

extern "C" int vcb_wide_concretize(int32_t R, int32_t Q, int32_t n0, int32_t lde,
                                   const float* e, const float* acc, const float* xl,
                                   const float* xh, float* lb, float* A, float* g0,
                                   void* stream) {
  if (R < 0 || Q <= 0 || n0 <= 0) return fail(VCB_ERR_INVALID, "vcb_wide_concretize: shape");
  if (R == 0) return VCB_OK;
  concretize_kernel<<<grid1((long long)R * 32), 256, 0, static_cast<cudaStream_t>(stream)>>>(
      R, Q, n0, lde, e, acc, xl, xh, lb, A, g0);
  return check_launch("vcb_wide_concretize");
}

extern "C" int vcb_wide_adjoint_layer(int32_t R, int32_t Q, int32_t nin, int32_t nout,
                                      const float* g, int32_t ldg, const float* W,
                                      const float* b, const float* rec, const float* sb_lo,
                                      const float* sb_hi, const float* alpha,
                                      int32_t alpha_rows, float* g_o, float* dcontrib,
                                      float* dbeta, int32_t ldo, void* stream) {
  if (R < 0 || Q <= 0 || nin <= 0 || nout <= 0)
    return fail(VCB_ERR_INVALID, "vcb_wide_adjoint_layer: shape");
  if (R == 0) return VCB_OK;
  if (!g || !W || !b || !rec || !sb_lo || !sb_hi || !g_o || !dcontrib || (ldg & 3) || (ldo & 3))
    return fail(VCB_ERR_INVALID, "vcb_wide_adjoint_layer: NULL pointer or bad ld");
  AdjArgs a{R, Q, nin, nout, ldg, ldo, g, W, b, rec, sb_lo, sb_hi, alpha, g_o, dcontrib, dbeta,
            alpha_rows};
  const int sm = smem_bytes(false);
  int rc = ensure_smem(reinterpret_cast<const void*>(alpha_adjoint_kernel), sm);
  if (rc) return rc;
  alpha_adjoint_kernel<<<gemm_grid(R, nout), GT, sm, static_cast<cudaStream_t>(stream)>>>(a);
  return check_launch("vcb_wide_adjoint_layer");
}

extern "C" int vcb_wide_alpha_adam(int32_t D, int32_t Q, int32_t n, int32_t ldc,
                                   const float* dcontrib, float* alpha, float* m1, float* m2,
                                   float lr, int32_t step, void* stream) {
  if (D < 0 || Q <= 0 || n <= 0 || step < 1) return fail(VCB_ERR_INVALID, "vcb_wide_alpha_adam");
  if (D == 0) return VCB_OK;
  const double bc1 = 1.0 - std::pow(0.9, step);
  const double bc2 = 1.0 - std::pow(0.999, step);
  alpha_adam_kernel<<<grid1((long long)D * n), 256, 0, static_cast<cudaStream_t>(stream)>>>(
      D, Q, n, ldc, dcontrib, alpha, m1, m2, (float)((double)lr / bc1), (float)std::sqrt(bc2));
  return check_launch("vcb_wide_alpha_adam");
}
