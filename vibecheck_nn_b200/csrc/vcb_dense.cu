// Concrete (point) evaluation of fc layers for the layer-wise path.
//
// * fc forward (the fc branch of _forward_batch_graph,
//   verify_zono_bnb.py:577-592): z = x W^T + b for N points, with the
//   pre-activation and / or its ReLU written by the epilogue.
// * fc vector-Jacobian product (what autograd computes for PGD's gradient,
//   pgd.py:494 and verify_hybrid_acasxu.py:155): g_in = g W, zeroed where the
//   pre-activation of the ReLU feeding the fc is <= 0 (F.relu's gradient).
#include "vcb_common.cuh"
#include "vcb_gemm.cuh"

namespace vcb {
namespace {

struct FcFwdArgs {
  int N, nin, nout, ldx, ldz, lda;
  const float *x, *W, *b;
  float *z, *a;
};

__global__ void __launch_bounds__(GT) fc_fwd_kernel(const FcFwdArgs a) {
  extern __shared__ __align__(16) float smem[];
  float acc[8][4], acc2[8][4];
  mainloop<false>(a.N, a.nout, a.nin, RowLoad{a.x, a.ldx}, RowLoad{a.W, a.nin},
                  RowLoad{nullptr, 0}, RowLoad{nullptr, 0}, acc, acc2, smem);
  const int ty = threadIdx.x >> 4, tx = threadIdx.x & 15;
  const int m0 = blockIdx.x * TM + ty * 8, n0 = blockIdx.y * TN + tx * 4;
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const int m = m0 + i;
    if (m >= a.N) continue;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int n = n0 + j;
      if (n >= a.nout) continue;
      const float v = __fadd_rn(acc[i][j], a.b[n]);
      if (a.z) a.z[(long long)m * a.ldz + n] = v;
      if (a.a) a.a[(long long)m * a.lda + n] = fmaxf(v, 0.f);
    }
  }
}

struct FcBackArgs {
  int N, nin, nout, ldg, ldm, ldo;
  const float *g, *W, *mask;
  float* g_o;
};

__global__ void __launch_bounds__(GT) fc_back_kernel(const FcBackArgs a) {
  extern __shared__ __align__(16) float smem[];
  float acc[8][4], acc2[8][4];
  mainloop<false>(a.N, a.nin, a.nout, RowLoad{a.g, a.ldg}, ColLoad{a.W, a.nin},
                  RowLoad{nullptr, 0}, ColLoad{nullptr, 0}, acc, acc2, smem);
  const int ty = threadIdx.x >> 4, tx = threadIdx.x & 15;
  const int m0 = blockIdx.x * TM + ty * 8, n0 = blockIdx.y * TN + tx * 4;
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const int m = m0 + i;
    if (m >= a.N) continue;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int n = n0 + j;
      if (n >= a.nin) continue;
      const bool keep = !a.mask || a.mask[(long long)m * a.ldm + n] > 0.f;
      a.g_o[(long long)m * a.ldo + n] = keep ? acc[i][j] : 0.f;
    }
  }
}

}  // namespace
}  // namespace vcb

using namespace vcb;

extern "C" int vcb_fc_forward(int32_t N, int32_t nin, int32_t nout, const float* x,
                              int32_t ldx, const float* W, const float* b, float* z,
                              int32_t ldz, float* a, int32_t lda, void* stream) {
  if (N < 0 || nin <= 0 || nout <= 0 || ldx < nin || (z && ldz < nout) || (a && lda < nout))
    return fail(VCB_ERR_INVALID, "vcb_fc_forward: N=%d nin=%d nout=%d ldx=%d", N, nin, nout,
                ldx);
  if (N == 0) return VCB_OK;
  if (!x || !W || !b || (!z && !a)) return fail(VCB_ERR_INVALID, "vcb_fc_forward: NULL pointer");
  FcFwdArgs args{N, nin, nout, ldx, ldz, lda, x, W, b, z, a};
  const int sm = gemm_smem_bytes(false);
  int rc = ensure_smem(reinterpret_cast<const void*>(fc_fwd_kernel), sm);
  if (rc) return rc;
  fc_fwd_kernel<<<gemm_grid(N, nout), GT, sm, static_cast<cudaStream_t>(stream)>>>(args);
  return check_launch("vcb_fc_forward");
}

extern "C" int vcb_fc_backward(int32_t N, int32_t nin, int32_t nout, const float* g,
                               int32_t ldg, const float* W, const float* mask, int32_t ldm,
                               float* g_o, int32_t ldo, void* stream) {
  if (N < 0 || nin <= 0 || nout <= 0 || ldg < nout || ldo < nin || (mask && ldm < nin))
    return fail(VCB_ERR_INVALID, "vcb_fc_backward: N=%d nin=%d nout=%d", N, nin, nout);
  if (N == 0) return VCB_OK;
  if (!g || !W || !g_o) return fail(VCB_ERR_INVALID, "vcb_fc_backward: NULL pointer");
  FcBackArgs args{N, nin, nout, ldg, ldm, ldo, g, W, mask, g_o};
  const int sm = gemm_smem_bytes(false);
  int rc = ensure_smem(reinterpret_cast<const void*>(fc_back_kernel), sm);
  if (rc) return rc;
  fc_back_kernel<<<gemm_grid(N, nin), GT, sm, static_cast<cudaStream_t>(stream)>>>(args);
  return check_launch("vcb_fc_backward");
}
