// Fate of one leaf of a multi-subbox BaB batch: safe by its bound, safe by
// input-domain clipping, or to split with its clipped box and smart-branching
// scores (verify_graph.py:11121-11177, :11640-11802).  Shared by the
// forward-LiRPA kernel's fused epilogue and the standalone fate kernel.
//
// Every fp32 operation is rounded as the reference's tensor expression
// rounds it (products, sums, the division); sums over dimensions run in
// dimension order.
#pragma once

#include <cuda_runtime.h>

namespace vcb {
namespace {

constexpr int kMsMaxVar = 32;  // varying dimensions (the forward-LiRPA limit)
constexpr int kMsMaxQ = 64;

// Leaf b of B: box xl/xh (rows of n), the K varying dimensions var; query q's
// coefficients A[q * lda + k], constant sb[q * ldsb], lower bound lb[q] and
// sub-box bias bias[q].  Writes fate[b] (0 / 1 / 2) and, for 2, the clipped
// box and the scores of row b, and raises fate[B] to the leaf's count of
// dimensions wider than 1e-12.
__device__ void ms_leaf_fate(int b, int B, int n, int K, int Q, int iters, const float* xl_all,
                             const float* xh_all, const int* var, const float* A, int lda,
                             const float* sb, int ldsb, const float* lb, const float* bias,
                             int* fate, float* oxl_all, float* oxh_all, float* score_all) {
  const float* xl = xl_all + (long long)b * n;
  const float* xh = xh_all + (long long)b * n;
  bool safe = false;
  for (int q = 0; q < Q; ++q) safe |= __fadd_rn(lb[q], bias[q]) > 0.f;
  if (safe) {
    fate[b] = 0;
    return;
  }
  float cl[kMsMaxVar], ch[kMsMaxVar], w0[kMsMaxVar];
  for (int k = 0; k < K; ++k) {
    cl[k] = xl[var[k]];
    ch[k] = xh[var[k]];
    w0[k] = __fsub_rn(ch[k], cl[k]);
  }
  for (int it = 0; it < iters; ++it) {
    float nl[kMsMaxVar], nh[kMsMaxVar];
    for (int k = 0; k < K; ++k) {
      nl[k] = -INFINITY;
      nh[k] = INFINITY;
    }
    for (int q = 0; q < Q; ++q) {
      const float* a = A + (long long)q * lda;
      // the query's lower bound over the current box
      float lo = 0.f;
      for (int k = 0; k < K; ++k)
        lo = __fadd_rn(lo, __fadd_rn(__fmul_rn(fmaxf(a[k], 0.f), cl[k]),
                                     __fmul_rn(fminf(a[k], 0.f), ch[k])));
      lo = __fadd_rn(lo, __fadd_rn(sb[(long long)q * ldsb], bias[q]));
      for (int k = 0; k < K; ++k) {
        const float ak = a[k];
        const float mid = __fmul_rn(__fadd_rn(ch[k], cl[k]), 0.5f);
        const float rad = __fmul_rn(__fsub_rn(ch[k], cl[k]), 0.5f);
        // lower bound with dimension k left free: its crossing with 0
        const float rest =
            __fsub_rn(lo, __fsub_rn(__fmul_rn(ak, mid), __fmul_rn(fabsf(ak), rad)));
        const float x0 = __fdiv_rn(-rest, fabsf(ak) > 1e-30f ? ak : 1.f);
        if (ak > 0.f) nh[k] = fminf(nh[k], x0);
        if (ak < 0.f) nl[k] = fmaxf(nl[k], x0);
      }
    }
    for (int k = 0; k < K; ++k) {
      ch[k] = fminf(nh[k], ch[k]);
      cl[k] = fmaxf(nl[k], cl[k]);
    }
  }
  bool empty = false;
  for (int k = 0; k < K; ++k) empty |= cl[k] > ch[k];
  if (empty) {
    fate[b] = 1;
    return;
  }
  fate[b] = 2;
  float* oxl = oxl_all + (long long)b * n;
  float* oxh = oxh_all + (long long)b * n;
  float* sc = score_all + (long long)b * n;
  for (int i = 0; i < n; ++i) {
    oxl[i] = xl[i];
    oxh[i] = xh[i];
    sc[i] = -INFINITY;
  }
  for (int k = 0; k < K; ++k) {
    const int d = var[k];
    oxl[d] = cl[k];
    oxh[d] = ch[k];
    float s = -INFINITY;
    for (int q = 0; q < Q; ++q) {
      const float c = fmaxf(fabsf(A[(long long)q * lda + k]), 0.1f);
      const float m = __fadd_rn(lb[q], bias[q]);
      s = fmaxf(s, __fadd_rn(__fmul_rn(__fmul_rn(c, w0[k]), 0.5f), m));
    }
    sc[d] = s;
  }
  int nz = 0;
  for (int i = 0; i < n; ++i) {
    const bool wide = __fsub_rn(oxh[i], oxl[i]) > 1e-12f;
    nz += wide;
    if (!wide) sc[i] = -INFINITY;
  }
  atomicMax(fate + B, nz);
}

}  // namespace
}  // namespace vcb
