// Tensor-core alpha-CROWN loop for wide ReLU MLPs (the Adam loop of
// verify_milp.py:2762-2807 / verify_zono_bnb.py:5248-5288 over domains x
// spec rows).  Every contraction is a 3xTF32 tcgen05 GEMM (vcb_tc.cu) whose
// epilogue does the layer's bound arithmetic on the accumulator registers
// and writes the next GEMM's operand directly as its TF32 hi / lo split:
//   * back GEMM  C_l = coef @ W_l -> the record C_l, the relaxation of the
//     ReLU below it (+ beta) as the next coef, and per 64-column group the
//     intercept sum plus the next bias dot coef . b_{l-1};
//     the relaxation is read as per-neuron records made once per call
//     (vcb_wtc_relax_init: upper slope + intercept from the bounds, and the
//     lower slope -- alpha, with 1 / 0 fixed on active / dead neurons, whose
//     alpha gradient is zero so Adam leaves them in place);
//   * input GEMM e = coef @ W_0 -> per group sum(e+ xl + e- xh) and the
//     adjoint seed d lb / d e;
//   * adjoint GEMM ga = g @ W_l^T + b_l -> with the record: the per-row alpha
//     gradient [unstable] max(e, 0) ga and the next adjoint.
// Two small kernels close an iteration: vcb_wtc_finish sums each row's
// partials in a fixed order into lb, keeps the best lb and raises the "some
// best lb <= 0" flag; vcb_wtc_adam sums the alpha gradient over each domain's
// spec rows (in order) and takes torch's Adam step on -sum(lb) + clamp.
// Every launch takes an optional device gate and does nothing when *gate ==
// 0, so the host can queue all iterations and the device skip those after
// every best lb turned positive.
#include <algorithm>
#include <cmath>
#include <cstdint>

#include "vcb_common.cuh"
#include "vcb_relu.cuh"
#include "vcb_tc.cuh"

namespace vcb {
namespace {

// Per (domain, neuron) of one ReLU layer: rx = (upper slope, its sign bit set
// when the neuron is stable; intercept factor) and the lower slope pos
// (1 active, 0 dead, the min-area choice on unstable neurons -- the alpha
// init of verify_zono_bnb.py:5170-5173).
__global__ void wtc_relax_init_kernel(long long n, const float* lo, const float* hi, float2* rx,
                                      float* pos, const int* gate) {
  if (gate && *gate == 0) return;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n;
       i += (long long)gridDim.x * blockDim.x) {
    const RelaxTc r = relax_tc(lo[i], hi[i], nullptr);
    rx[i] = make_float2(r.unstable ? r.neg : -r.neg, r.icp);
    pos[i] = r.pos;
  }
}

__global__ void wtc_finish_kernel(int R, const float* acc0, const float* part, int ldpart,
                                  int nparts, float* lb, float* best, int first, int* open,
                                  const int* gate) {
  if (gate && *gate == 0) return;
  for (int m = blockIdx.x * blockDim.x + threadIdx.x; m < R; m += gridDim.x * blockDim.x) {
    float v = acc0[m];
    const float* p = part + (long long)m * ldpart;
#pragma unroll 8
    for (int t = 0; t < nparts; ++t) v = __fadd_rn(v, p[t]);
    lb[m] = v;
    if (best) {
      float b = v;
      if (!first) {
        const float o = best[m];
        b = (isnan(o) || isnan(v)) ? __int_as_float(0x7fc00000) : fmaxf(o, v);  // torch.maximum
      }
      best[m] = b;
      if (open && !(b > 0.f)) *open = 1;
    }
  }
}

// grad[box][j] = sum_q dcontrib[box * Q + q][j]; torch's Adam (betas 0.9 /
// 0.999, eps 1e-8) on the loss -sum(lb), then clamp to [0, 1].
__global__ void wtc_adam_kernel(int D, int Q, int n, int ldd, const float* dcontrib,
                                float* alpha, float* m1, float* m2, float step_size,
                                float bc2_sqrt, const int* gate) {
  if (gate && *gate == 0) return;
  const long long total = (long long)D * n;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total;
       i += (long long)gridDim.x * blockDim.x) {
    const long long box = i / n;
    const int j = (int)(i - box * n);
    float gsum = 0.f;
#pragma unroll 8
    for (int q = 0; q < Q; ++q) gsum = __fadd_rn(gsum, dcontrib[(box * Q + q) * ldd + j]);
    const float g = -gsum;
    const float mm = __fadd_rn(m1[i], __fmul_rn(0.1f, __fsub_rn(g, m1[i])));
    const float vv = __fadd_rn(__fmul_rn(m2[i], 0.999f), __fmul_rn(__fmul_rn(g, g), 0.001f));
    m1[i] = mm;
    m2[i] = vv;
    const float denom = __fadd_rn(__fdiv_rn(sqrtf(vv), bc2_sqrt), 1e-8f);
    const float p = __fsub_rn(alpha[i], __fmul_rn(step_size, __fdiv_rn(mm, denom)));
    alpha[i] = fminf(fmaxf(p, 0.f), 1.f);
  }
}

int grid_for(long long items) {
  const long long b = (items + 255) / 256;
  return (int)std::max<long long>(1, std::min<long long>(b, 16LL * sm_count()));
}

int parts_of(int n) { return (n + 63) / 64; }

}  // namespace
}  // namespace vcb

using namespace vcb;

extern "C" int vcb_wtc_back_gemm(int32_t R, int32_t Q, int32_t N, int32_t K, const float* A_hi,
                                 const float* A_lo, int32_t lda, const float* B_hi,
                                 const float* B_lo, int32_t ldb, float* C, int32_t ldc,
                                 const float* pos, const float* rx, const float* beta,
                                 const float* b_next, float* out_hi,
                                 float* out_lo, int32_t ldo, float* part, int32_t ldpart,
                                 int32_t part0, int32_t* err, const int32_t* gate,
                                 void* stream) {
  if (R < 0 || Q <= 0 || N <= 0 || K <= 0 || (R % Q) || ldc < N || ldo < N || part0 < 0 ||
      part0 + parts_of(N) > ldpart)
    return fail(VCB_ERR_INVALID, "vcb_wtc_back_gemm: R=%d Q=%d N=%d K=%d", R, Q, N, K);
  if (R == 0) return VCB_OK;
  if (!A_hi || !A_lo || !B_hi || !B_lo || !C || !pos || !rx || !out_hi || !out_lo || !part ||
      !err)
    return fail(VCB_ERR_INVALID, "vcb_wtc_back_gemm: NULL pointer");
  TcEpi ep;
  ep.mode = kEpiRelax;
  ep.Q = Q;
  ep.pos = pos;
  ep.rx = reinterpret_cast<const float2*>(rx);
  ep.beta = beta;
  ep.bnext = b_next;
  ep.out_hi = out_hi;
  ep.out_lo = out_lo;
  ep.ldo = ldo;
  ep.part = part;
  ep.ldpart = ldpart;
  ep.part0 = part0;
  return tc_gemm_fused(R, N, K, A_hi, A_lo, lda, B_hi, B_lo, ldb, C, ldc, nullptr, err,
                       static_cast<cudaStream_t>(stream), "vcb_wtc_back_gemm", gate, ep);
}

extern "C" int vcb_wtc_input_gemm(int32_t R, int32_t Q, int32_t N, int32_t K,
                                  const float* A_hi, const float* A_lo, int32_t lda,
                                  const float* B_hi, const float* B_lo, int32_t ldb,
                                  const float* xl, const float* xh, float* g_hi, float* g_lo,
                                  int32_t ldg, float* part, int32_t ldpart, int32_t part0,
                                  int32_t* err, const int32_t* gate, void* stream) {
  if (R < 0 || Q <= 0 || N <= 0 || K <= 0 || (R % Q) || ldg < N || part0 < 0 ||
      part0 + parts_of(N) > ldpart)
    return fail(VCB_ERR_INVALID, "vcb_wtc_input_gemm: R=%d Q=%d N=%d K=%d", R, Q, N, K);
  if (R == 0) return VCB_OK;
  if (!A_hi || !A_lo || !B_hi || !B_lo || !xl || !xh || !g_hi || !g_lo || !part || !err)
    return fail(VCB_ERR_INVALID, "vcb_wtc_input_gemm: NULL pointer");
  TcEpi ep;
  ep.mode = kEpiConcretize;
  ep.Q = Q;
  ep.xl = xl;
  ep.xh = xh;
  ep.out_hi = g_hi;
  ep.out_lo = g_lo;
  ep.ldo = ldg;
  ep.part = part;
  ep.ldpart = ldpart;
  ep.part0 = part0;
  return tc_gemm_fused(R, N, K, A_hi, A_lo, lda, B_hi, B_lo, ldb, nullptr, (N + 3) & ~3,
                       nullptr, err, static_cast<cudaStream_t>(stream), "vcb_wtc_input_gemm",
                       gate, ep);
}

extern "C" int vcb_wtc_adj_gemm(int32_t R, int32_t Q, int32_t N, int32_t K, const float* A_hi,
                                const float* A_lo, int32_t lda, const float* B_hi,
                                const float* B_lo, int32_t ldb, const float* bias,
                                const float* rec, int32_t ldrec, const float* pos,
                                const float* rx, float* dcontrib,
                                int32_t ldd, float* g_hi, float* g_lo, int32_t ldg,
                                int32_t* err, const int32_t* gate, void* stream) {
  if (R < 0 || Q <= 0 || N <= 0 || K <= 0 || (R % Q) || ldrec < N || ldd < N ||
      (g_hi && ldg < N))
    return fail(VCB_ERR_INVALID, "vcb_wtc_adj_gemm: R=%d Q=%d N=%d K=%d", R, Q, N, K);
  if (R == 0) return VCB_OK;
  if (!A_hi || !A_lo || !B_hi || !B_lo || !bias || !rec || !pos || !rx || !dcontrib || !err ||
      ((g_hi == nullptr) != (g_lo == nullptr)))
    return fail(VCB_ERR_INVALID, "vcb_wtc_adj_gemm: NULL pointer");
  TcEpi ep;
  ep.mode = kEpiAdjoint;
  ep.Q = Q;
  ep.pos = pos;
  ep.rx = reinterpret_cast<const float2*>(rx);
  ep.rec = rec;
  ep.ldrec = ldrec;
  ep.dcontrib = dcontrib;
  ep.ldd = ldd;
  ep.out_hi = g_hi;
  ep.out_lo = g_lo;
  ep.ldo = g_hi ? ldg : 4;
  return tc_gemm_fused(R, N, K, A_hi, A_lo, lda, B_hi, B_lo, ldb, nullptr, (N + 3) & ~3, bias,
                       err, static_cast<cudaStream_t>(stream), "vcb_wtc_adj_gemm", gate, ep);
}

extern "C" int vcb_wtc_finish(int32_t R, const float* acc0, const float* part, int32_t ldpart,
                              int32_t nparts, float* lb, float* best, int32_t first,
                              int32_t* open_flag, const int32_t* gate, void* stream) {
  if (R < 0 || nparts < 0 || ldpart < nparts)
    return fail(VCB_ERR_INVALID, "vcb_wtc_finish: R=%d nparts=%d ldpart=%d", R, nparts, ldpart);
  if (R == 0) return VCB_OK;
  if (!acc0 || (nparts > 0 && !part) || !lb)
    return fail(VCB_ERR_INVALID, "vcb_wtc_finish: NULL pointer");
  wtc_finish_kernel<<<grid_for(R), 256, 0, static_cast<cudaStream_t>(stream)>>>(
      R, acc0, part, ldpart, nparts, lb, best, first ? 1 : 0, open_flag, gate);
  return check_launch("vcb_wtc_finish");
}

extern "C" int vcb_wtc_adam(int32_t D, int32_t Q, int32_t n, const float* dcontrib, int32_t ldd,
                            float* alpha, float* m1, float* m2, float lr, int32_t step,
                            const int32_t* gate, void* stream) {
  if (D < 0 || Q <= 0 || n <= 0 || ldd < n || step < 1)
    return fail(VCB_ERR_INVALID, "vcb_wtc_adam: D=%d Q=%d n=%d step=%d", D, Q, n, step);
  if (D == 0) return VCB_OK;
  if (!dcontrib || !alpha || !m1 || !m2)
    return fail(VCB_ERR_INVALID, "vcb_wtc_adam: NULL pointer");
  const double bc1 = 1.0 - std::pow(0.9, step);
  const double bc2 = 1.0 - std::pow(0.999, step);
  wtc_adam_kernel<<<grid_for((long long)D * n), 256, 0, static_cast<cudaStream_t>(stream)>>>(
      D, Q, n, ldd, dcontrib, alpha, m1, m2, (float)((double)lr / bc1), (float)std::sqrt(bc2),
      gate);
  return check_launch("vcb_wtc_adam");
}

extern "C" int vcb_wtc_relax_init(int64_t n, const float* sb_lo, const float* sb_hi, float* rx,
                                  float* pos, const int32_t* gate, void* stream) {
  if (n < 0) return fail(VCB_ERR_INVALID, "vcb_wtc_relax_init: n=%lld", (long long)n);
  if (n == 0) return VCB_OK;
  if (!sb_lo || !sb_hi || !rx || !pos || (reinterpret_cast<uintptr_t>(rx) & 7))
    return fail(VCB_ERR_INVALID, "vcb_wtc_relax_init: NULL or misaligned pointer");
  wtc_relax_init_kernel<<<grid_for(n), 256, 0, static_cast<cudaStream_t>(stream)>>>(
      n, sb_lo, sb_hi, reinterpret_cast<float2*>(rx), pos, gate);
  return check_launch("vcb_wtc_relax_init");
}
