// Multi-subbox input-split BaB step on the device: leaf fate, input-domain
// clipping, split scores and child emission for one batch of leaves.
//
// Follows the inner loop of _multi_sub_input_split_bab (verify_graph.py):
//   fate    a leaf is safe when any query of its sub-box has a positive
//           margin, forward-LiRPA lower bound + the sub-box's query bias
//                                                            (:11640-11660)
//   clip    two rounds of the closed-form projection of each query's linear
//           bound onto every varying dimension, the minimum over queries
//           (:11121-11177, :11695-11734); a box clipped to empty is safe
//   score   max over queries of max(|A_qk|, 0.1) * width_k / 2 + margin_q
//           on the pre-clip varying widths, -inf on dimensions that do not
//           vary or are at most 1e-12 wide after the clip  (:11780-11802)
//   split   the top K_eff dimensions in CPU torch.topk order, all 2^K_eff
//           combinations of low / high halves per leaf, leaf by leaf; a
//           dimension at most 1e-12 wide is left whole     (:11816-11852)
//
// The fate of a leaf (ms_leaf_fate, vcb_multisub.cuh) runs in one thread
// with the leaf's varying box in registers; vcb_mlp_flirpa_fate calls it at
// the end of the forward-LiRPA kernel, on the spec rows still in shared
// memory, and vcb_multisub_fate on spec rows in global memory.  The emit
// kernel writes the children with one thread per output element after one
// thread per leaf has ranked its dimensions.
#include "vcb_common.cuh"
#include "vcb_multisub.cuh"
#include "vcb_topk.cuh"

namespace vcb {
namespace {

constexpr int kMsMaxDepth = 16;
constexpr int kMsThreads = 128;

struct MsFateParams {
  int B, n, K, Q, iters;
  const float *xl, *xh;  // (B, n)
  const int* var;        // (K) varying dimensions
  const float *A, *sb, *lb;  // (B, Q, K), (B, Q), (B, Q)
  const float* bias;     // (n_sub, Q) query bias of each sub-box
  const int* sub;        // (B) sub-box of each leaf
  int* fate;             // (B + 1): 0 bound-safe, 1 clip-safe, 2 split; [B] = max nz
  float *oxl, *oxh;      // (B, n) clipped boxes
  float* score;          // (B, n)
};

__global__ void __launch_bounds__(kMsThreads) ms_fate_kernel(const MsFateParams p) {
  const int b = blockIdx.x * blockDim.x + threadIdx.x;
  if (b >= p.B) return;
  const long long q0 = (long long)b * p.Q;
  ms_leaf_fate(b, p.B, p.n, p.K, p.Q, p.iters, p.xl, p.xh, p.var, p.A + q0 * p.K, p.K,
               p.sb + q0, 1, p.lb + q0, p.bias + (long long)p.sub[b] * p.Q, p.fate, p.oxl,
               p.oxh, p.score);
}

struct MsEmitParams {
  int U, n, k;
  const int* rows;  // (U) batch row of each splitting leaf
  const float *xl, *xh, *score;  // (B, n)
  const int* sub;   // (B)
  VI* work;         // (U, n)
  int* top;         // (U, k)
  float *kxl, *kxh; // (U 2^k, n)
  int* ksub;        // (U 2^k)
};

__global__ void __launch_bounds__(kMsThreads) ms_rank_kernel(const MsEmitParams p) {
  const int u = blockIdx.x * blockDim.x + threadIdx.x;
  if (u >= p.U) return;
  const int n = p.n;
  const float* s = p.score + (long long)p.rows[u] * n;
  VI* q = p.work + (long long)u * n;
  for (int i = 0; i < n; ++i) q[i] = VI{s[i], i};
  tk_topk(q, n, p.k);
  for (int j = 0; j < p.k; ++j) p.top[(long long)u * p.k + j] = q[j].i;
}

__global__ void __launch_bounds__(kMsThreads) ms_emit_kernel(const MsEmitParams p) {
  const int n = p.n, k = p.k, nch = 1 << k;
  const long long total = (long long)p.U * nch * n;
  for (long long e = blockIdx.x * (long long)blockDim.x + threadIdx.x; e < total;
       e += (long long)gridDim.x * blockDim.x) {
    const int i = (int)(e % n);
    const long long r = e / n;  // child row
    const int c = (int)(r % nch);
    const int u = (int)(r / nch);
    const int b = p.rows[u];
    const float l = p.xl[(long long)b * n + i], h = p.xh[(long long)b * n + i];
    float lo = l, hi = h;
    for (int j = 0; j < k; ++j)
      if (p.top[(long long)u * k + j] == i && __fsub_rn(h, l) > 1e-12f) {
        const float mid = __fmul_rn(__fadd_rn(l, h), 0.5f);
        if ((c >> j) & 1) lo = mid;
        else hi = mid;
      }
    p.kxl[e] = lo;
    p.kxh[e] = hi;
    if (i == 0) p.ksub[r] = p.sub[b];
  }
}

}  // namespace
}  // namespace vcb

extern "C" int vcb_multisub_fate(int32_t B, int32_t n_in, int32_t K, int32_t Q,
                                 const float* xl, const float* xh, const int32_t* var_idx,
                                 const float* spec_A, const float* spec_b, const float* lb,
                                 const float* sub_bias, const int32_t* sub, int32_t clip_iters,
                                 int32_t* fate, float* out_xl, float* out_xh, float* score,
                                 void* stream) {
  using namespace vcb;
  const char* who = "vcb_multisub_fate";
  if (B < 0 || n_in <= 0 || K <= 0 || K > n_in || Q <= 0 || clip_iters < 0)
    return fail(VCB_ERR_INVALID, "%s: B=%d n_in=%d K=%d Q=%d clip_iters=%d", who, B, n_in, K,
                Q, clip_iters);
  if (K > kMsMaxVar || Q > kMsMaxQ)
    return fail(VCB_ERR_UNSUPPORTED, "%s: K=%d (max %d) Q=%d (max %d)", who, K, kMsMaxVar, Q,
                kMsMaxQ);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  cudaError_t e = cudaMemsetAsync(fate + B, 0, sizeof(int32_t), st);
  if (e != cudaSuccess) return cuda_fail(e, who);
  if (B == 0) return VCB_OK;
  MsFateParams p{B, n_in, K, Q, clip_iters, xl, xh, var_idx, spec_A, spec_b, lb, sub_bias, sub,
                 fate, out_xl, out_xh, score};
  ms_fate_kernel<<<(B + kMsThreads - 1) / kMsThreads, kMsThreads, 0, st>>>(p);
  return check_launch(who);
}

extern "C" int64_t vcb_multisub_emit_workspace(int32_t U, int32_t n_in, int32_t k) {
  if (U < 0 || n_in <= 0 || k <= 0) return 0;
  const int64_t a = ((int64_t)U * n_in * (int64_t)sizeof(vcb::VI) + 255) & ~int64_t(255);
  return a + (int64_t)U * k * (int64_t)sizeof(int32_t);
}

extern "C" int vcb_multisub_emit(int32_t U, int32_t n_in, int32_t k, const int32_t* rows,
                                 const float* xl, const float* xh, const float* score,
                                 const int32_t* sub, void* workspace, float* kid_xl,
                                 float* kid_xh, int32_t* kid_sub, void* stream) {
  using namespace vcb;
  const char* who = "vcb_multisub_emit";
  if (U < 0 || n_in <= 0 || k <= 0 || k > n_in)
    return fail(VCB_ERR_INVALID, "%s: U=%d n_in=%d k=%d", who, U, n_in, k);
  if (k > kMsMaxDepth)
    return fail(VCB_ERR_UNSUPPORTED, "%s: k=%d (max %d)", who, k, kMsMaxDepth);
  if (U == 0) return VCB_OK;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  char* w = static_cast<char*>(workspace);
  const int64_t a = ((int64_t)U * n_in * (int64_t)sizeof(VI) + 255) & ~int64_t(255);
  MsEmitParams p{U, n_in, k, rows, xl, xh, score, sub, reinterpret_cast<VI*>(w),
                 reinterpret_cast<int*>(w + a), kid_xl, kid_xh, kid_sub};
  ms_rank_kernel<<<(U + kMsThreads - 1) / kMsThreads, kMsThreads, 0, st>>>(p);
  int rc = check_launch(who);
  if (rc) return rc;
  const long long total = (long long)U * (1 << k) * n_in;
  const long long want = (total + kMsThreads - 1) / kMsThreads;
  const int grid = (int)std::min<long long>(want, (long long)sm_count() * 16);
  ms_emit_kernel<<<grid, kMsThreads, 0, st>>>(p);
  return check_launch(who);
}
