// DeepZ zonotope forward for MLPs too wide for the shared-memory kernel
// (the cfg5 shape, 3072 -> [1024] x 8): _forward_zonotope_graph_batched
// (verify_zono_bnb.py:3079-4074) layer by layer.
//
// Layout: the generators of every leaf are stored generator-major -- leaf b
// owns rows [off_b, off_b + Kp_b) of one (rows x n) matrix, row k holding
// generator k's coefficient on every neuron, Kp_b padded to a multiple of 128
// with zero rows -- so one fc layer for the whole batch is ONE GEMM,
// G'^T = G^T W^T, on the tcgen05 3xTF32 kernel (vcb_tc.cu).  Per ReLU:
//   * vcb_zw_relu: lambda = hi / (hi - lo), mu = -hi lo / (2 (hi - lo)) on
//     unstable neurons (lambda 0 / 1 on dead / active ones), c' = lambda c + mu,
//     the unstable count of every leaf and its neurons in index order
//     (verify_zono_bnb.py:3175-3211);
//   * vcb_zw_build: the next GEMM's A operand, TF32-split: the leaf's rows
//     scaled column-wise by lambda, then one new row mu_j e_j per unstable
//     neuron j in index order, then zero padding;
//   * vcb_zw_colsum: per leaf and neuron the fixed-order compensated sum of
//     |G| over the leaf's rows -> lo / hi = c -+ that radius.
// Layer 0 needs no GEMM: its generators are r_i W0[:, i] (one per input
// dimension; zero rows where the radius is 0), built straight from W0^T.
#include <algorithm>

#include "vcb_common.cuh"
#include "vcb_tc.cuh"

namespace vcb {
namespace {

constexpr int ZW_T = 256;

// One CTA per leaf: lambda, mu, c' and the unstable neurons in index order.
__global__ void __launch_bounds__(ZW_T) zw_relu_kernel(int n, const float* __restrict__ c,
                                                       const float* __restrict__ lo,
                                                       const float* __restrict__ hi,
                                                       float* __restrict__ lam,
                                                       float* __restrict__ mu,
                                                       float* __restrict__ c_out,
                                                       int* __restrict__ cnt,
                                                       int* __restrict__ idx_of_rank) {
  __shared__ int warp_sums[ZW_T / 32];
  __shared__ int carry;
  const int b = blockIdx.x, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const long long base = (long long)b * n;
  if (tid == 0) carry = 0;
  __syncthreads();
  for (int j0 = 0; j0 < n; j0 += ZW_T) {
    const int j = j0 + tid;
    int ust = 0;
    if (j < n) {
      const float l = lo[base + j], h = hi[base + j], cc = c[base + j];
      float la, m;
      if (l < 0.f && h > 0.f) {
        const float d = __fsub_rn(h, l);
        la = __fdiv_rn(h, d);
        m = __fdiv_rn(__fmul_rn(-h, l), __fmul_rn(2.f, d));
        ust = 1;
      } else {
        la = (h <= 0.f) ? 0.f : 1.f;
        m = 0.f;
      }
      lam[base + j] = la;
      mu[base + j] = m;
      c_out[base + j] = __fadd_rn(__fmul_rn(la, cc), m);
    }
    // block-wide exclusive scan of the unstable flags
    const unsigned bal = __ballot_sync(0xffffffffu, ust);
    const int before = __popc(bal & ((1u << lane) - 1u));
    if (lane == 0) warp_sums[warp] = __popc(bal);
    __syncthreads();
    int off = carry;
    for (int w = 0; w < warp; ++w) off += warp_sums[w];
    if (ust) idx_of_rank[base + off + before] = j;
    __syncthreads();
    if (tid == 0) {
      int t = 0;
      for (int w = 0; w < ZW_T / 32; ++w) t += warp_sums[w];
      carry += t;
    }
    __syncthreads();
  }
  if (tid == 0) cnt[b] = carry;
}

__device__ __forceinline__ void split_store(float v, float* hi, float* lo, long long i) {
  const uint32_t u = __float_as_uint(v);
  const bool finite = (u & 0x7F800000u) != 0x7F800000u;
  const float h = finite ? __uint_as_float((u + 0x1000u) & 0xFFFFE000u) : v;
  hi[i] = h;
  lo[i] = finite ? __fsub_rn(v, h) : 0.f;
}

// A rows of leaf b (blockIdx.y): [0, k_in) scaled rows, [k_in, k_in + cnt)
// new generators, then zeros up to the next leaf's offset.  Source rows come
// from C (ld ldc) at in_off[b], or -- layer 0 (C == NULL) -- are r_b[k] W0T[k].
__global__ void zw_build_kernel(int n, int ld, const long long* __restrict__ in_off,
                                const int* __restrict__ k_in, const float* __restrict__ C,
                                int ldc, const float* __restrict__ r, int n0,
                                const float* __restrict__ W0T, const float* __restrict__ lam,
                                const float* __restrict__ mu, const int* __restrict__ cnt,
                                const int* __restrict__ idx_of_rank,
                                const long long* __restrict__ out_off, float* __restrict__ Ah,
                                float* __restrict__ Al) {
  const int b = blockIdx.y;
  const long long o0 = out_off[b], rows = out_off[b + 1] - o0;
  const int kin = k_in[b], u = cnt[b];
  const float* lam_b = lam + (long long)b * n;
  const long long total = rows * ld;
  for (long long e = (long long)blockIdx.x * blockDim.x + threadIdx.x; e < total;
       e += (long long)gridDim.x * blockDim.x) {
    const long long row = e / ld;
    const int j = (int)(e - row * ld);
    float v = 0.f;
    if (j < n) {
      if (row < kin) {
        float g;
        if (C) {
          g = C[(in_off[b] + row) * ldc + j];
        } else {
          g = __fmul_rn(W0T[row * (long long)n + j], r[(long long)b * n0 + row]);
        }
        v = __fmul_rn(g, lam_b[j]);
      } else if (row < kin + u) {
        const int jj = idx_of_rank[(long long)b * n + (row - kin)];
        v = (j == jj) ? mu[(long long)b * n + j] : 0.f;
      }
    }
    split_store(v, Ah, Al, (o0 + row) * ld + j);
  }
}

// rad[b][j] = sum over the leaf's k rows of |C[row][j]| in row order with
// Neumaier's compensated summation (the radius sums thousands of terms; the
// compensation keeps it at fp32 rounding of the exact sum); lo = c - rad,
// hi = c + rad.
__global__ void zw_colsum_kernel(int n, const long long* __restrict__ off,
                                 const int* __restrict__ k, const float* __restrict__ C, int ldc,
                                 const float* __restrict__ c, float* __restrict__ lo,
                                 float* __restrict__ hi) {
  const int b = blockIdx.y;
  const int j = blockIdx.x * blockDim.x + threadIdx.x;
  if (j >= n) return;
  const float* p = C + off[b] * ldc + j;
  const int kb = k[b];
  float s = 0.f, comp = 0.f;
  for (int row = 0; row < kb; ++row) {
    const float v = fabsf(p[(long long)row * ldc]);
    const float t = __fadd_rn(s, v);
    comp = __fadd_rn(comp, (s >= v) ? __fadd_rn(__fsub_rn(s, t), v) : __fadd_rn(__fsub_rn(v, t), s));
    s = t;
  }
  s = __fadd_rn(s, comp);
  const long long i = (long long)b * n + j;
  lo[i] = __fsub_rn(c[i], s);
  hi[i] = __fadd_rn(c[i], s);
}

}  // namespace
}  // namespace vcb

using namespace vcb;

extern "C" int vcb_zw_relu(int32_t B, int32_t n, const float* c, const float* lo, const float* hi,
                           float* lam, float* mu, float* c_out, int32_t* cnt,
                           int32_t* idx_of_rank, void* stream) {
  if (B < 0 || n <= 0) return fail(VCB_ERR_INVALID, "vcb_zw_relu: B=%d n=%d", B, n);
  if (B == 0) return VCB_OK;
  if (!c || !lo || !hi || !lam || !mu || !c_out || !cnt || !idx_of_rank)
    return fail(VCB_ERR_INVALID, "vcb_zw_relu: NULL pointer");
  zw_relu_kernel<<<B, ZW_T, 0, static_cast<cudaStream_t>(stream)>>>(n, c, lo, hi, lam, mu, c_out,
                                                                    cnt, idx_of_rank);
  return check_launch("vcb_zw_relu");
}

extern "C" int vcb_zw_build(int32_t B, int32_t n, int32_t ld, const int64_t* in_off,
                            const int32_t* k_in, const float* C, int32_t ldc, const float* r,
                            int32_t n0, const float* W0T, const float* lam, const float* mu,
                            const int32_t* cnt, const int32_t* idx_of_rank,
                            const int64_t* out_off, int64_t rows_hint, float* A_hi, float* A_lo,
                            void* stream) {
  if (B < 0 || n <= 0 || ld < n || ld % 4 || rows_hint < 0)
    return fail(VCB_ERR_INVALID, "vcb_zw_build: B=%d n=%d ld=%d", B, n, ld);
  if (B == 0) return VCB_OK;
  if (!k_in || !lam || !mu || !cnt || !idx_of_rank || !out_off || !A_hi || !A_lo ||
      (C && !in_off) || (!C && (!r || !W0T)))
    return fail(VCB_ERR_INVALID, "vcb_zw_build: NULL pointer");
  const long long per_leaf = (rows_hint / std::max(1, B) + 1) * ld;
  const int bx = (int)std::max<long long>(1, std::min<long long>((per_leaf + 255) / 256, 1024));
  zw_build_kernel<<<dim3(bx, B), 256, 0, static_cast<cudaStream_t>(stream)>>>(
      n, ld, reinterpret_cast<const long long*>(in_off), k_in, C, ldc, r, n0, W0T, lam, mu, cnt,
      idx_of_rank, reinterpret_cast<const long long*>(out_off), A_hi, A_lo);
  return check_launch("vcb_zw_build");
}

extern "C" int vcb_zw_colsum(int32_t B, int32_t n, const int64_t* off, const int32_t* k,
                             const float* C, int32_t ldc, const float* c, float* lo, float* hi,
                             void* stream) {
  if (B < 0 || n <= 0 || ldc < n) return fail(VCB_ERR_INVALID, "vcb_zw_colsum: B=%d n=%d", B, n);
  if (B == 0) return VCB_OK;
  if (!off || !k || !C || !c || !lo || !hi) return fail(VCB_ERR_INVALID, "vcb_zw_colsum: NULL pointer");
  zw_colsum_kernel<<<dim3((n + 255) / 256, B), 256, 0, static_cast<cudaStream_t>(stream)>>>(
      n, reinterpret_cast<const long long*>(off), k, C, ldc, c, lo, hi);
  return check_launch("vcb_zw_colsum");
}
