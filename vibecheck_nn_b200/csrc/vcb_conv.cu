// Convolution layers and element-wise ReLU steps for the layer-wise path.
//
// * conv IBP (verify_zono_bnb.py:1106-1113): mid * K + b and rad * |K| as
//   implicit GEMMs (M = boxes x output pixels, N = C_out, K = C_in kh kw; the
//   A operand is an im2col gather of the NCHW input), giving the
//   pre-activation lo/hi.
// * conv back-substitution (verify_zono_bnb.py:4568-4593, the
//   conv_transpose2d of the coefficients): implicit GEMM over input pixels
//   (M = rows x H x W, N = C_in, K = C_out kh kw) whose A operand gathers the
//   output-pixel coefficient that each kernel tap of a stride-s convolution
//   maps onto the input pixel (zero where no output pixel does), so every sum
//   has a fixed order and no atomics are needed.
// * concrete conv forward (the conv branch of _forward_batch_graph,
//   verify_zono_bnb.py:569-575) as the same implicit GEMM with a bias +
//   optional ReLU epilogue, and its vector-Jacobian product (the transposed
//   convolution, masked by the pre-activation of the ReLU feeding the conv).
// * per-row bias dot of a conv layer (the coefficient times the per-channel
//   bias repeated over the spatial positions).
// * IBP ReLU (verify_zono_bnb.py:1123-1138) and CROWN ReLU relaxation
//   (verify_zono_bnb.py:4409-4449) as element-wise kernels with a fixed-order
//   per-row intercept sum.
#include <algorithm>

#include "vcb_common.cuh"
#include "vcb_gemm.cuh"

namespace vcb {
namespace {

struct ConvGeom {
  int C, H, W, Co, Ho, Wo, kh, kw, sh, sw, ph, pw;
};

// im2col gather: row m = (box, output pixel), col k = (c, ki, kj).
struct Im2col {
  const float* x;  // boxes x C x H x W
  ConvGeom g;
  __device__ __forceinline__ float a(int m, int k) const {
    const int hw = g.Ho * g.Wo;
    const int d = m / hw, pix = m - d * hw;
    const int oh = pix / g.Wo, ow = pix - oh * g.Wo;
    const int kk = g.kh * g.kw;
    const int c = k / kk, t = k - c * kk;
    const int ki = t / g.kw, kj = t - ki * g.kw;
    const int ih = oh * g.sh - g.ph + ki, iw = ow * g.sw - g.pw + kj;
    if (ih < 0 || ih >= g.H || iw < 0 || iw >= g.W) return 0.f;
    return __ldg(x + (((long long)d * g.C + c) * g.H + ih) * g.W + iw);
  }
};

// Transposed-convolution gather: row m = (row r, input pixel h, w), col
// k = (co, ki, kj); the output pixel (oh, ow) with oh*sh - ph + ki == h.
struct Col2im {
  const float* e;  // rows x Co x Ho x Wo
  ConvGeom g;
  __device__ __forceinline__ float a(int m, int k) const {
    const int hw = g.H * g.W;
    const int r = m / hw, pix = m - r * hw;
    const int h = pix / g.W, w = pix - h * g.W;
    const int kk = g.kh * g.kw;
    const int co = k / kk, t = k - co * kk;
    const int ki = t / g.kw, kj = t - ki * g.kw;
    const int nh = h + g.ph - ki, nw = w + g.pw - kj;
    if (nh < 0 || nw < 0) return 0.f;
    const int oh = nh / g.sh, ow = nw / g.sw;
    if (oh * g.sh != nh || ow * g.sw != nw || oh >= g.Ho || ow >= g.Wo) return 0.f;
    return __ldg(e + (((long long)r * g.Co + co) * g.Ho + oh) * g.Wo + ow);
  }
};

// B(k, n) = K[co][n][ki][kj] for k = (co, ki, kj): the conv weight read as
// the (C_out kh kw) x C_in operand of the transposed convolution.
struct KernT {
  const float* K;
  ConvGeom g;
  static constexpr bool kFastB = false;
  __device__ __forceinline__ float b(int k, int n) const {
    const int kk = g.kh * g.kw;
    const int co = k / kk, t = k - co * kk;
    return __ldg(K + ((long long)co * g.C + n) * kk + t);
  }
};

struct ConvIbpArgs {
  int D;
  ConvGeom g;
  const float *mid, *rad, *K, *Kabs, *b;
  float *lo, *hi;  // D x Co x Ho x Wo
};

__global__ void __launch_bounds__(GT) conv_ibp_kernel(const ConvIbpArgs a) {
  extern __shared__ __align__(16) float smem[];
  float acc[8][4], acc2[8][4];
  const int KD = a.g.C * a.g.kh * a.g.kw;
  const int M = a.D * a.g.Ho * a.g.Wo;
  mainloop<true>(M, a.g.Co, KD, Im2col{a.mid, a.g}, RowLoad{a.K, KD}, Im2col{a.rad, a.g},
                 RowLoad{a.Kabs, KD}, acc, acc2, smem);
  const int ty = threadIdx.x >> 4, tx = threadIdx.x & 15;
  const int m0 = blockIdx.x * TM + ty * 8, n0 = blockIdx.y * TN + tx * 4;
  const int hw = a.g.Ho * a.g.Wo;
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const int m = m0 + i;
    if (m >= M) continue;
    const int d = m / hw, pix = m - d * hw;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int n = n0 + j;
      if (n >= a.g.Co) continue;
      const float mc = __fadd_rn(acc[i][j], a.b[n]);
      const float rc = acc2[i][j];
      const long long o = ((long long)d * a.g.Co + n) * hw + pix;
      a.lo[o] = __fsub_rn(mc, rc);
      a.hi[o] = __fadd_rn(mc, rc);
    }
  }
}

struct ConvFwdArgs {
  int N;
  ConvGeom g;
  const float *x, *K, *b;
  float *z, *a;  // N x Co x Ho x Wo pre-activation / relu'd output (each optional)
};

__global__ void __launch_bounds__(GT) conv_fwd_kernel(const ConvFwdArgs a) {
  extern __shared__ __align__(16) float smem[];
  float acc[8][4], acc2[8][4];
  const int KD = a.g.C * a.g.kh * a.g.kw;
  const int M = a.N * a.g.Ho * a.g.Wo;
  mainloop<false>(M, a.g.Co, KD, Im2col{a.x, a.g}, RowLoad{a.K, KD}, Im2col{nullptr, a.g},
                  RowLoad{nullptr, KD}, acc, acc2, smem);
  const int ty = threadIdx.x >> 4, tx = threadIdx.x & 15;
  const int m0 = blockIdx.x * TM + ty * 8, n0 = blockIdx.y * TN + tx * 4;
  const int hw = a.g.Ho * a.g.Wo;
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const int m = m0 + i;
    if (m >= M) continue;
    const int d = m / hw, pix = m - d * hw;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int n = n0 + j;
      if (n >= a.g.Co) continue;
      const float v = __fadd_rn(acc[i][j], a.b[n]);
      const long long o = ((long long)d * a.g.Co + n) * hw + pix;
      if (a.z) a.z[o] = v;
      if (a.a) a.a[o] = fmaxf(v, 0.f);
    }
  }
}

struct ConvBackArgs {
  int R;
  ConvGeom g;
  const float *e, *K;
  float* e_in;        // R x C x H x W
  const float* mask;  // R x C x H x W pre-activations: keep e_in where > 0; or NULL
};

__global__ void __launch_bounds__(GT) conv_back_kernel(const ConvBackArgs a) {
  extern __shared__ __align__(16) float smem[];
  float acc[8][4], acc2[8][4];
  const int KD = a.g.Co * a.g.kh * a.g.kw;
  const int M = a.R * a.g.H * a.g.W;
  mainloop<false>(M, a.g.C, KD, Col2im{a.e, a.g}, KernT{a.K, a.g}, Col2im{nullptr, a.g},
                  KernT{nullptr, a.g}, acc, acc2, smem);
  const int ty = threadIdx.x >> 4, tx = threadIdx.x & 15;
  const int m0 = blockIdx.x * TM + ty * 8, n0 = blockIdx.y * TN + tx * 4;
  const int hw = a.g.H * a.g.W;
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const int m = m0 + i;
    if (m >= M) continue;
    const int r = m / hw, pix = m - r * hw;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int n = n0 + j;
      if (n >= a.g.C) continue;
      const long long o = ((long long)r * a.g.C + n) * hw + pix;
      a.e_in[o] = (a.mask && !(a.mask[o] > 0.f)) ? 0.f : acc[i][j];
    }
  }
}

// bd[r] = sum_{c, pix} e[r][c][pix] * b[c]  (one warp per row)
__global__ void conv_bias_dot_kernel(int R, int Co, int hw, const float* e, const float* b,
                                     float* bd) {
  const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  const int nw = (gridDim.x * blockDim.x) >> 5;
  const int n = Co * hw;
  for (int r = warp; r < R; r += nw) {
    float s = 0.f;
    for (int i = lane; i < n; i += 32) s = fmaf(e[(long long)r * n + i], b[i / hw], s);
    for (int off = 16; off > 0; off >>= 1) s += __shfl_xor_sync(0xffffffffu, s, off);
    if (lane == 0) bd[r] = s;
  }
}

// IBP relu: clamp, crossing repair, bounds out, relu'd mid/rad for the next op.
__global__ void ibp_relu_kernel(int D, int n, const float* lo, const float* hi,
                                const float* clo, const float* chi, float* sblo, float* sbhi,
                                float* mid, float* rad, int ldo) {
  const long long total = (long long)D * n;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total;
       i += (long long)gridDim.x * blockDim.x) {
    float l = lo[i], h = hi[i];
    if (clo) {
      l = fmaxf(l, clo[i]);
      h = fminf(h, chi[i]);
    }
    h = fmaxf(h, l);
    sblo[i] = l;
    sbhi[i] = h;
    const long long d = i / n;
    const int j = (int)(i - d * n);
    const float lc = fmaxf(l, 0.f), hc = fmaxf(h, 0.f);
    mid[d * ldo + j] = __fmul_rn(__fadd_rn(lc, hc), 0.5f);
    rad[d * ldo + j] = __fmul_rn(__fsub_rn(hc, lc), 0.5f);
  }
}

// CROWN relu relaxation of coefficient rows (one warp per row):
// e_out = e >= 0 ? e * lower : e * upper (+ beta); part[r] = sum min(e,0) up_t.
__global__ void relu_back_kernel(int R, int Q, int n, int lde, const float* e, int ldo,
                                 float* e_out, const float* sblo, const float* sbhi,
                                 const float* alpha, const float* beta, float* part) {
  const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  const int nw = (gridDim.x * blockDim.x) >> 5;
  for (int r = warp; r < R; r += nw) {
    const long long box = r / Q;
    float s = 0.f;
    for (int j = lane; j < n; j += 32) {
      const long long gi = box * n + j;
      const float lo = sblo[gi], hi = sbhi[gi];
      const float lb_r = fminf(lo, 0.f);
      const float ub_r = fmaxf(fmaxf(hi, 0.f), __fadd_rn(lb_r, 1e-8f));
      const float up_s = __fdiv_rn(ub_r, __fsub_rn(ub_r, lb_r));
      const float up_t = __fmul_rn(-lb_r, up_s);
      float pos;
      if (lo >= 0.f) pos = 1.f;
      else if (hi <= 0.f) pos = 0.f;
      else pos = alpha ? alpha[gi] : (up_s > 0.5f ? 1.f : 0.f);
      const float v = e[(long long)r * lde + j];
      float o;
      if (v < 0.f) {
        s = fmaf(v, up_t, s);
        o = __fmul_rn(v, up_s);
      } else {
        o = __fmul_rn(v, pos);
      }
      if (beta) o = __fadd_rn(o, beta[gi]);
      e_out[(long long)r * ldo + j] = o;
    }
    for (int off = 16; off > 0; off >>= 1) s += __shfl_xor_sync(0xffffffffu, s, off);
    if (lane == 0) part[r] = s;
  }
}

int rows_grid(long long rows) {
  return (int)std::max<long long>(1, std::min<long long>((rows * 32 + 255) / 256, 16LL * sm_count()));
}

ConvGeom geom(const int32_t* s) {
  return ConvGeom{s[0], s[1], s[2], s[3], s[4], s[5], s[6], s[7], s[8], s[9], s[10], s[11]};
}

}  // namespace
}  // namespace vcb

using namespace vcb;

// geometry: {C, H, W, Co, Ho, Wo, kh, kw, sh, sw, ph, pw}
extern "C" int vcb_conv_ibp(int32_t D, const int32_t* geometry, const float* mid,
                            const float* rad, const float* K, const float* Kabs,
                            const float* b, float* lo, float* hi, void* stream) {
  if (D < 0 || !geometry) return fail(VCB_ERR_INVALID, "vcb_conv_ibp: bad arguments");
  if (D == 0) return VCB_OK;
  if (!mid || !rad || !K || !Kabs || !b || !lo || !hi)
    return fail(VCB_ERR_INVALID, "vcb_conv_ibp: NULL pointer");
  ConvIbpArgs a{D, geom(geometry), mid, rad, K, Kabs, b, lo, hi};
  const int sm = gemm_smem_bytes(true);
  int rc = ensure_smem(reinterpret_cast<const void*>(conv_ibp_kernel), sm);
  if (rc) return rc;
  conv_ibp_kernel<<<gemm_grid(D * a.g.Ho * a.g.Wo, a.g.Co), GT, sm,
                    static_cast<cudaStream_t>(stream)>>>(a);
  return check_launch("vcb_conv_ibp");
}

extern "C" int vcb_conv_back(int32_t R, const int32_t* geometry, const float* e,
                             const float* K, float* e_in, void* stream) {
  if (R < 0 || !geometry) return fail(VCB_ERR_INVALID, "vcb_conv_back: bad arguments");
  if (R == 0) return VCB_OK;
  if (!e || !K || !e_in) return fail(VCB_ERR_INVALID, "vcb_conv_back: NULL pointer");
  ConvBackArgs a{R, geom(geometry), e, K, e_in, nullptr};
  const int sm = gemm_smem_bytes(false);
  int rc = ensure_smem(reinterpret_cast<const void*>(conv_back_kernel), sm);
  if (rc) return rc;
  conv_back_kernel<<<gemm_grid(R * a.g.H * a.g.W, a.g.C), GT, sm,
                     static_cast<cudaStream_t>(stream)>>>(a);
  return check_launch("vcb_conv_back");
}

extern "C" int vcb_conv_forward(int32_t N, const int32_t* geometry, const float* x,
                                const float* K, const float* b, float* z, float* a,
                                void* stream) {
  if (N < 0 || !geometry) return fail(VCB_ERR_INVALID, "vcb_conv_forward: bad arguments");
  if (N == 0) return VCB_OK;
  if (!x || !K || !b || (!z && !a)) return fail(VCB_ERR_INVALID, "vcb_conv_forward: NULL pointer");
  ConvFwdArgs args{N, geom(geometry), x, K, b, z, a};
  const int sm = gemm_smem_bytes(false);
  int rc = ensure_smem(reinterpret_cast<const void*>(conv_fwd_kernel), sm);
  if (rc) return rc;
  conv_fwd_kernel<<<gemm_grid(N * args.g.Ho * args.g.Wo, args.g.Co), GT, sm,
                    static_cast<cudaStream_t>(stream)>>>(args);
  return check_launch("vcb_conv_forward");
}

extern "C" int vcb_conv_backward(int32_t N, const int32_t* geometry, const float* g,
                                 const float* K, const float* mask, float* g_in,
                                 void* stream) {
  if (N < 0 || !geometry) return fail(VCB_ERR_INVALID, "vcb_conv_backward: bad arguments");
  if (N == 0) return VCB_OK;
  if (!g || !K || !g_in) return fail(VCB_ERR_INVALID, "vcb_conv_backward: NULL pointer");
  ConvBackArgs a{N, geom(geometry), g, K, g_in, mask};
  const int sm = gemm_smem_bytes(false);
  int rc = ensure_smem(reinterpret_cast<const void*>(conv_back_kernel), sm);
  if (rc) return rc;
  conv_back_kernel<<<gemm_grid(N * a.g.H * a.g.W, a.g.C), GT, sm,
                     static_cast<cudaStream_t>(stream)>>>(a);
  return check_launch("vcb_conv_backward");
}

extern "C" int vcb_conv_bias_dot(int32_t R, int32_t Co, int32_t hw, const float* e,
                                 const float* b, float* bd, void* stream) {
  if (R < 0 || Co <= 0 || hw <= 0) return fail(VCB_ERR_INVALID, "vcb_conv_bias_dot: shape");
  if (R == 0) return VCB_OK;
  conv_bias_dot_kernel<<<rows_grid(R), 256, 0, static_cast<cudaStream_t>(stream)>>>(R, Co, hw,
                                                                                   e, b, bd);
  return check_launch("vcb_conv_bias_dot");
}

extern "C" int vcb_ibp_relu(int32_t D, int32_t n, const float* lo, const float* hi,
                            const float* clo, const float* chi, float* sb_lo, float* sb_hi,
                            float* mid, float* rad, int32_t ldo, void* stream) {
  if (D < 0 || n <= 0 || ldo < n) return fail(VCB_ERR_INVALID, "vcb_ibp_relu: shape");
  if (D == 0) return VCB_OK;
  const long long total = (long long)D * n;
  const int grid = (int)std::max<long long>(1, std::min<long long>((total + 255) / 256, 8LL * sm_count()));
  ibp_relu_kernel<<<grid, 256, 0, static_cast<cudaStream_t>(stream)>>>(D, n, lo, hi, clo, chi,
                                                                      sb_lo, sb_hi, mid, rad, ldo);
  return check_launch("vcb_ibp_relu");
}

extern "C" int vcb_relu_back(int32_t R, int32_t Q, int32_t n, const float* e, int32_t lde,
                             float* e_out, int32_t ldo, const float* sb_lo, const float* sb_hi,
                             const float* alpha, const float* beta, float* part,
                             void* stream) {
  if (R < 0 || Q <= 0 || n <= 0) return fail(VCB_ERR_INVALID, "vcb_relu_back: shape");
  if (R == 0) return VCB_OK;
  if (!e || !e_out || !sb_lo || !sb_hi || !part)
    return fail(VCB_ERR_INVALID, "vcb_relu_back: NULL pointer");
  relu_back_kernel<<<rows_grid(R), 256, 0, static_cast<cudaStream_t>(stream)>>>(
      R, Q, n, lde, e, ldo, e_out, sb_lo, sb_hi, alpha, beta, part);
  return check_launch("vcb_relu_back");
}
