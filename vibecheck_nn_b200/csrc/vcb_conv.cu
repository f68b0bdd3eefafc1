// Convolution layers and element-wise ReLU steps for the layer-wise path.
//
// * conv IBP (verify_zono_bnb.py:1106-1113): mid * K + b and rad * |K| as
//   implicit GEMMs (M = boxes x output pixels, N = C_out, K = C_in kh kw; the
//   A operand is an im2col gather of the NCHW input), giving the
//   pre-activation lo/hi.
// * conv back-substitution (verify_zono_bnb.py:4568-4593, the
//   conv_transpose2d of the coefficients) in two steps: a dense GEMM of the
//   coefficients with the kernel gives every (output pixel, input channel,
//   tap) product (M = rows x Ho x Wo, N = C_in kh kw, K = C_out -- no
//   structural zeros), then a gather sums, for every input pixel, the taps
//   that land on it in a fixed (ki, kj) order: no atomics, deterministic, and
//   both passes read and write contiguously.
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
  static constexpr bool kFastA = true;  // consecutive m = neighbouring output pixels
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

// A(m, k) of the per-tap product: m = (row r, output pixel), k = output
// channel co; e is rows x Co x Ho x Wo, so consecutive m are contiguous.
struct EPix {
  const float* e;
  int Co, hw;
  static constexpr bool kFastA = true;
  __device__ __forceinline__ float a(int m, int k) const {
    const int r = m / hw, pix = m - r * hw;
    return __ldg(e + ((long long)r * Co + k) * hw + pix);
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

// Transposed convolution, step 1: cols^T (C kh kw) x (R Ho Wo) = (e^T K)^T,
// the contribution of every output pixel to every kernel tap of every input
// channel (M = R Ho Wo, N = C kh kw, K = Co).
struct ConvColsArgs {
  int R;
  ConvGeom g;
  const float *e, *K;
  float* cols;  // (C kh kw) x (R Ho Wo)
};

constexpr int kColsPad = TM + 1;  // smem row of the transposed epilogue tile

__global__ void __launch_bounds__(GT) conv_cols_kernel(const ConvColsArgs a) {
  extern __shared__ __align__(16) float smem[];
  float acc[8][4], acc2[8][4];
  const int hw = a.g.Ho * a.g.Wo;
  const int M = a.R * hw;
  const int N = a.g.C * a.g.kh * a.g.kw;
  mainloop<false>(M, N, a.g.Co, EPix{a.e, a.g.Co, hw}, ColLoad{a.K, N}, EPix{nullptr, 0, 1},
                  ColLoad{nullptr, 0}, acc, acc2, smem);
  // transpose the 128 x 64 tile through shared memory so that each column n
  // of cols^T is written as 128 consecutive floats
  const int ty = threadIdx.x >> 4, tx = threadIdx.x & 15;
  const int m0 = blockIdx.x * TM, n0 = blockIdx.y * TN;
#pragma unroll
  for (int i = 0; i < 8; ++i)
#pragma unroll
    for (int j = 0; j < 4; ++j) smem[(tx * 4 + j) * kColsPad + ty * 8 + i] = acc[i][j];
  __syncthreads();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  for (int nn = warp; nn < TN; nn += GT / 32) {
    const int n = n0 + nn;
    if (n >= N) break;
    for (int mm = lane; mm < TM; mm += 32) {
      const int m = m0 + mm;
      if (m < M) a.cols[(long long)n * M + m] = smem[nn * kColsPad + mm];
    }
  }
}

// Step 2: e_in[r][c][h][w] = sum over the taps (ki, kj) whose output pixel
// (oh, ow) = ((h + ph - ki) / sh, (w + pw - kj) / sw) exists, in (ki, kj)
// order; zeroed where mask (the ReLU pre-activation in front, or NULL) <= 0.
// Grid: x over the H W pixels of one (row, channel) plane, y = row C + c.
__global__ void col2im_kernel(int R, ConvGeom g, const float* __restrict__ cols,
                              const float* __restrict__ mask, float* __restrict__ e_in) {
  const int p = blockIdx.x * blockDim.x + threadIdx.x;
  if (p >= g.H * g.W) return;
  const int rc = blockIdx.y;
  const int c = rc % g.C, r = rc / g.C;
  const int h = p / g.W, w = p - h * g.W;
  const long long M = (long long)R * g.Ho * g.Wo;
  const long long rowbase = (long long)r * g.Ho;
  const int kk = g.kh * g.kw;
  float acc = 0.f;
  // the taps that reach (h, w) are ki = (h + ph) mod sh + sh t
  const int hp = h + g.ph, wp = w + g.pw;
  for (int ki = hp % g.sh; ki < g.kh; ki += g.sh) {
    const int nh = hp - ki;
    if (nh < 0) break;
    const int oh = nh / g.sh;
    if (oh >= g.Ho) continue;
    for (int kj = wp % g.sw; kj < g.kw; kj += g.sw) {
      const int nw = wp - kj;
      if (nw < 0) break;
      const int ow = nw / g.sw;
      if (ow >= g.Wo) continue;
      const long long col = (long long)c * kk + ki * g.kw + kj;
      acc += __ldg(cols + col * M + (rowbase + oh) * g.Wo + ow);
    }
  }
  const long long idx = ((long long)rc * g.H + h) * g.W + w;
  e_in[idx] = (mask && !(mask[idx] > 0.f)) ? 0.f : acc;
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

static int conv_transpose(const char* who, int32_t R, const int32_t* geometry, const float* g,
                          const float* K, const float* mask, float* g_in, void* workspace,
                          size_t ws_bytes, void* stream) {
  if (R < 0 || !geometry) return fail(VCB_ERR_INVALID, "%s: bad arguments", who);
  if (R == 0) return VCB_OK;
  if (!g || !K || !g_in) return fail(VCB_ERR_INVALID, "%s: NULL pointer", who);
  ConvColsArgs a{R, geom(geometry), g, K, static_cast<float*>(workspace)};
  const size_t need = (size_t)R * a.g.Ho * a.g.Wo * a.g.C * a.g.kh * a.g.kw * sizeof(float);
  if (!workspace || ws_bytes < need)
    return fail(VCB_ERR_INVALID, "%s: workspace of %zu bytes, need %zu", who, ws_bytes, need);
  if ((long long)R * a.g.C > 65535)
    return fail(VCB_ERR_UNSUPPORTED, "%s: %d rows x %d channels", who, R, a.g.C);
  const int sm = std::max(gemm_smem_bytes(false), TN * kColsPad * 4);
  int rc = ensure_smem(reinterpret_cast<const void*>(conv_cols_kernel), sm);
  if (rc) return rc;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  conv_cols_kernel<<<gemm_grid(R * a.g.Ho * a.g.Wo, a.g.C * a.g.kh * a.g.kw), GT, sm, st>>>(a);
  rc = check_launch(who);
  if (rc) return rc;
  const dim3 grid((a.g.H * a.g.W + 255) / 256, R * a.g.C);
  col2im_kernel<<<grid, 256, 0, st>>>(R, a.g, a.cols, mask, g_in);
  return check_launch(who);
}

extern "C" size_t vcb_conv_back_workspace(int32_t R, const int32_t* geometry) {
  if (R <= 0 || !geometry) return 0;
  const ConvGeom g = geom(geometry);
  return (size_t)R * g.Ho * g.Wo * g.C * g.kh * g.kw * sizeof(float);
}

extern "C" int vcb_conv_back(int32_t R, const int32_t* geometry, const float* e,
                             const float* K, float* e_in, void* workspace, size_t ws_bytes,
                             void* stream) {
  return conv_transpose("vcb_conv_back", R, geometry, e, K, nullptr, e_in, workspace, ws_bytes,
                        stream);
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
                                 void* workspace, size_t ws_bytes, void* stream) {
  return conv_transpose("vcb_conv_backward", N, geometry, g, K, mask, g_in, workspace, ws_bytes,
                        stream);
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
