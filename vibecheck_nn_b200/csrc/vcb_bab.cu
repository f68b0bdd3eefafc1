// Input-split BaB step on the device: closure, halfspace clipping, branching
// and child emission for one batch of leaves, in one single-CTA launch.
//
// Follows _input_split_batched_inner (verify_graph.py):
//   closure  every disjunct has a query with lb > 0            (:12901-12908)
//   clip     per-(query, dim) projection of {A_q.x + acc_q <= 0} onto the
//            box, per disjunct with a union of the feasible boxes when there
//            are several disjuncts (:12363-12426, :13030-13130)
//   branch   first-max argmax of the width, or of width * sum_q |A_q| (:13236-13295)
//   split    bisection at the midpoint; width <= 1e-12 counts as degenerate;
//            children emitted low block then high block in leaf order
//            (:13353-13382)
// The batch is at most a few thousand leaves with a handful of input
// dimensions, so each thread owns a contiguous run of leaves; a block-wide
// scan of the usable flags gives each child's row.
#include <algorithm>

#include "vcb_common.cuh"

namespace vcb {
namespace {

constexpr int kBT = 1024;
constexpr int kMaxIn = 64;
constexpr int kMaxQ = 64;

struct BabParams {
  int B, n, Q, D, Qs;  // Qs: leading queries that count for the SB score
  int clip, sb;
  const float *xl, *xh, *lb, *A, *acc;
  const int* qd;  // disjunct of each query
  float *lo_xl, *lo_xh, *hi_xl, *hi_xh;
  long long* counters;  // [closed_crown, closed_clip, usable, degenerate]
};

// Clip of box (xl, xh) by the halfspaces of the queries in disjunct d (all
// queries when d < 0) -- verify_graph.py:12388-12426.  Writes the new box and
// returns feasibility.
__device__ bool clip_box(const BabParams& p, int b, int d, const float* xl,
                         const float* xh, float* nxl, float* nxh) {
  const int n = p.n;
  for (int i = 0; i < n; ++i) {
    nxl[i] = -INFINITY;
    nxh[i] = INFINITY;
  }
  bool half_empty = false;
  for (int q = 0; q < p.Q; ++q) {
    if (d >= 0 && p.qd[q] != d) continue;
    const float* Aq = p.A + ((long long)b * p.Q + q) * n;
    const float bq = p.acc[(long long)b * p.Q + q];
    float sp = 0.f, sn = 0.f;
    for (int i = 0; i < n; ++i) {
      const float a = Aq[i];
      sp = __fadd_rn(sp, __fmul_rn(fmaxf(a, 0.f), xl[i]));
      sn = __fadd_rn(sn, __fmul_rn(fminf(a, 0.f), xh[i]));
    }
    const float total_min = __fadd_rn(sp, sn);
    if (__fadd_rn(total_min, bq) > 0.f) half_empty = true;
    for (int i = 0; i < n; ++i) {
      const float a = Aq[i];
      const float contrib = __fadd_rn(__fmul_rn(fmaxf(a, 0.f), xl[i]),
                                      __fmul_rn(fminf(a, 0.f), xh[i]));
      const float l_other = __fsub_rn(total_min, contrib);
      const float a_safe = fabsf(a) > 1e-12f ? a : 1.f;
      const float thr = __fdiv_rn(__fsub_rn(-bq, l_other), a_safe);
      const float cand_h = a > 1e-12f ? thr : xh[i];
      const float cand_l = a < -1e-12f ? thr : xl[i];
      nxh[i] = fminf(nxh[i], cand_h);
      nxl[i] = fmaxf(nxl[i], cand_l);
    }
  }
  bool box_empty = false;
  for (int i = 0; i < n; ++i) {
    nxh[i] = fminf(nxh[i], xh[i]);
    nxl[i] = fmaxf(nxl[i], xl[i]);
    if (nxl[i] > nxh[i]) box_empty = true;
  }
  return !(half_empty || box_empty);
}

// Fate of leaf b: 0 closed by CROWN, 1 closed by clipping, 2 degenerate,
// 3 split.  Fills the box to split and its split dimension.
__device__ int leaf_fate(const BabParams& p, int b, float* bxl, float* bxh, int* ax) {
  const int n = p.n;
  bool closed = true;
  for (int d = 0; d < p.D; ++d) {
    bool any = false;
    for (int q = 0; q < p.Q; ++q)
      if (p.qd[q] == d && p.lb[(long long)b * p.Q + q] > 0.f) any = true;
    closed = closed && any;
  }
  if (closed) return 0;
  float xl[kMaxIn], xh[kMaxIn];
  for (int i = 0; i < n; ++i) {
    xl[i] = p.xl[(long long)b * n + i];
    xh[i] = p.xh[(long long)b * n + i];
  }
  if (p.clip) {
    if (p.D == 1) {
      if (!clip_box(p, b, -1, xl, xh, bxl, bxh)) return 1;
    } else {
      float txl[kMaxIn], txh[kMaxIn];
      bool feas = false;
      for (int i = 0; i < n; ++i) {
        bxl[i] = INFINITY;
        bxh[i] = -INFINITY;
      }
      for (int d = 0; d < p.D; ++d) {
        if (clip_box(p, b, d, xl, xh, txl, txh)) {
          feas = true;
          for (int i = 0; i < n; ++i) {
            bxl[i] = fminf(bxl[i], txl[i]);
            bxh[i] = fmaxf(bxh[i], txh[i]);
          }
        }
      }
      if (!feas) return 1;
    }
  } else {
    for (int i = 0; i < n; ++i) {
      bxl[i] = xl[i];
      bxh[i] = xh[i];
    }
  }
  int best = 0;
  float best_s = -INFINITY;
  for (int i = 0; i < n; ++i) {
    float s = __fsub_rn(bxh[i], bxl[i]);
    if (p.sb) {
      float sens = 0.f;
      for (int q = 0; q < p.Qs; ++q)
        sens = __fadd_rn(sens, fabsf(p.A[((long long)b * p.Q + q) * n + i]));
      s = __fmul_rn(s, sens);
    }
    if (s > best_s || i == 0) {
      best_s = s;
      best = i;
    }
  }
  *ax = best;
  return (__fsub_rn(bxh[best], bxl[best]) > 1e-12f) ? 3 : 2;
}

__global__ void __launch_bounds__(kBT) bab_step_kernel(const BabParams p) {
  __shared__ int warp_sums[kBT / 32];
  __shared__ long long cnt[4];
  const int tid = threadIdx.x;
  if (tid < 4) cnt[tid] = 0;
  const int per = (p.B + kBT - 1) / kBT;
  const int b0 = min(p.B, tid * per), b1 = min(p.B, b0 + per);
  float bxl[kMaxIn], bxh[kMaxIn];
  int local[4] = {0, 0, 0, 0};
  for (int b = b0; b < b1; ++b) {
    int ax;
    const int f = leaf_fate(p, b, bxl, bxh, &ax);
    local[f == 3 ? 2 : (f == 2 ? 3 : f)]++;
  }
  __syncthreads();
  for (int k = 0; k < 4; ++k)
    if (local[k]) atomicAdd(reinterpret_cast<unsigned long long*>(&cnt[k]),
                            (unsigned long long)local[k]);
  // exclusive scan of the usable counts in thread order
  const int lane = tid & 31, warp = tid >> 5;
  int v = local[2];
  for (int off = 1; off < 32; off <<= 1) {
    const int t = __shfl_up_sync(0xffffffffu, v, off);
    if (lane >= off) v += t;
  }
  if (lane == 31) warp_sums[warp] = v;
  __syncthreads();
  if (warp == 0) {
    int w = warp_sums[lane];
    for (int off = 1; off < 32; off <<= 1) {
      const int t = __shfl_up_sync(0xffffffffu, w, off);
      if (lane >= off) w += t;
    }
    warp_sums[lane] = w;
  }
  __syncthreads();
  int pos = v - local[2] + (warp > 0 ? warp_sums[warp - 1] : 0);
  const int n = p.n;
  for (int b = b0; b < b1; ++b) {
    int ax;
    if (leaf_fate(p, b, bxl, bxh, &ax) != 3) continue;
    const float mid = __fmul_rn(__fadd_rn(bxl[ax], bxh[ax]), 0.5f);
    for (int i = 0; i < n; ++i) {
      const long long o = (long long)pos * n + i;
      p.lo_xl[o] = bxl[i];
      p.lo_xh[o] = (i == ax) ? mid : bxh[i];
      p.hi_xl[o] = (i == ax) ? mid : bxl[i];
      p.hi_xh[o] = bxh[i];
    }
    ++pos;
  }
  __syncthreads();
  if (tid < 4) p.counters[tid] = cnt[tid];
}

// ---- wide inputs (n_in > 64, e.g. 3072): one CTA per leaf decides its fate
// with fixed-order block reductions, a single CTA scans the usable flags, and
// one CTA per usable leaf writes its two children.

constexpr int kWT = 256;

struct BabWideParams {
  BabParams p;
  float *bxl, *bxh;  // (B, n) box to split (clipped)
  float *txl, *txh;  // (B, n) one disjunct's clipped box (D > 1)
  int *fate, *ax, *pos;
};

// Fixed-order block sum of one value per thread (tree over the 256 threads).
__device__ float block_sum(float v, float* red) {
  const int tid = threadIdx.x;
  red[tid] = v;
  __syncthreads();
  for (int w = kWT / 2; w > 0; w >>= 1) {
    if (tid < w) red[tid] = __fadd_rn(red[tid], red[tid + w]);
    __syncthreads();
  }
  const float r = red[0];
  __syncthreads();
  return r;
}

// clip_box for the CTA's leaf: every thread owns dims i = tid + k * kWT.
__device__ bool clip_box_block(const BabParams& p, int b, int d, const float* xl,
                               const float* xh, float* nxl, float* nxh, float* red,
                               int* flag) {
  const int n = p.n, tid = threadIdx.x;
  for (int i = tid; i < n; i += kWT) {
    nxl[i] = -INFINITY;
    nxh[i] = INFINITY;
  }
  if (tid == 0) *flag = 0;
  __syncthreads();
  bool half_empty = false;
  for (int q = 0; q < p.Q; ++q) {
    if (d >= 0 && p.qd[q] != d) continue;
    const float* Aq = p.A + ((long long)b * p.Q + q) * n;
    const float bq = p.acc[(long long)b * p.Q + q];
    float sp = 0.f, sn = 0.f;
    for (int i = tid; i < n; i += kWT) {
      const float a = Aq[i];
      sp = __fadd_rn(sp, __fmul_rn(fmaxf(a, 0.f), xl[i]));
      sn = __fadd_rn(sn, __fmul_rn(fminf(a, 0.f), xh[i]));
    }
    sp = block_sum(sp, red);
    sn = block_sum(sn, red);
    const float total_min = __fadd_rn(sp, sn);
    if (__fadd_rn(total_min, bq) > 0.f) half_empty = true;
    for (int i = tid; i < n; i += kWT) {
      const float a = Aq[i];
      const float contrib = __fadd_rn(__fmul_rn(fmaxf(a, 0.f), xl[i]),
                                      __fmul_rn(fminf(a, 0.f), xh[i]));
      const float l_other = __fsub_rn(total_min, contrib);
      const float a_safe = fabsf(a) > 1e-12f ? a : 1.f;
      const float thr = __fdiv_rn(__fsub_rn(-bq, l_other), a_safe);
      const float cand_h = a > 1e-12f ? thr : xh[i];
      const float cand_l = a < -1e-12f ? thr : xl[i];
      nxh[i] = fminf(nxh[i], cand_h);
      nxl[i] = fmaxf(nxl[i], cand_l);
    }
  }
  for (int i = tid; i < n; i += kWT) {
    nxh[i] = fminf(nxh[i], xh[i]);
    nxl[i] = fmaxf(nxl[i], xl[i]);
    if (nxl[i] > nxh[i]) *flag = 1;
  }
  __syncthreads();
  const bool box_empty = *flag != 0;
  __syncthreads();
  return !(half_empty || box_empty);
}

__global__ void __launch_bounds__(kWT) bab_fate_wide_kernel(const BabWideParams w) {
  __shared__ float red[kWT];
  __shared__ int flag, closed_s, best_i[kWT];
  __shared__ float best_v[kWT];
  const BabParams& p = w.p;
  const int b = blockIdx.x, tid = threadIdx.x, n = p.n;
  if (tid == 0) {
    bool closed = true;
    for (int d = 0; d < p.D; ++d) {
      bool any = false;
      for (int q = 0; q < p.Q; ++q)
        if (p.qd[q] == d && p.lb[(long long)b * p.Q + q] > 0.f) any = true;
      closed = closed && any;
    }
    closed_s = closed;
  }
  __syncthreads();
  if (closed_s) {
    if (tid == 0) w.fate[b] = 0;
    return;
  }
  const float* xl = p.xl + (long long)b * n;
  const float* xh = p.xh + (long long)b * n;
  float* bxl = w.bxl + (long long)b * n;
  float* bxh = w.bxh + (long long)b * n;
  if (p.clip) {
    bool feas;
    if (p.D == 1) {
      feas = clip_box_block(p, b, -1, xl, xh, bxl, bxh, red, &flag);
    } else {
      float* txl = w.txl + (long long)b * n;
      float* txh = w.txh + (long long)b * n;
      for (int i = tid; i < n; i += kWT) {
        bxl[i] = INFINITY;
        bxh[i] = -INFINITY;
      }
      feas = false;
      for (int d = 0; d < p.D; ++d) {
        if (clip_box_block(p, b, d, xl, xh, txl, txh, red, &flag)) {
          feas = true;
          for (int i = tid; i < n; i += kWT) {
            bxl[i] = fminf(bxl[i], txl[i]);
            bxh[i] = fmaxf(bxh[i], txh[i]);
          }
        }
      }
    }
    if (!feas) {
      if (tid == 0) w.fate[b] = 1;
      return;
    }
  } else {
    for (int i = tid; i < n; i += kWT) {
      bxl[i] = xl[i];
      bxh[i] = xh[i];
    }
  }
  // first-max argmax of the branching score
  float bv = -INFINITY;
  int bi = n;
  for (int i = tid; i < n; i += kWT) {
    float sc = __fsub_rn(bxh[i], bxl[i]);
    if (p.sb) {
      float sens = 0.f;
      for (int q = 0; q < p.Qs; ++q)
        sens = __fadd_rn(sens, fabsf(p.A[((long long)b * p.Q + q) * n + i]));
      sc = __fmul_rn(sc, sens);
    }
    if (bi == n || sc > bv) {
      bv = sc;
      bi = i;
    }
  }
  best_v[tid] = bv;
  best_i[tid] = bi;
  __syncthreads();
  for (int s = kWT / 2; s > 0; s >>= 1) {
    if (tid < s) {
      const float ov = best_v[tid + s];
      const int oi = best_i[tid + s];
      if (oi < n && (best_i[tid] == n || ov > best_v[tid] ||
                     (ov == best_v[tid] && oi < best_i[tid]))) {
        best_v[tid] = ov;
        best_i[tid] = oi;
      }
    }
    __syncthreads();
  }
  if (tid == 0) {
    const int a = best_i[0];
    w.ax[b] = a;
    w.fate[b] = (__fsub_rn(bxh[a], bxl[a]) > 1e-12f) ? 3 : 2;
  }
}

__global__ void __launch_bounds__(kBT) bab_scan_wide_kernel(int B, const int* __restrict__ fate,
                                                           int* __restrict__ pos,
                                                           long long* __restrict__ counters) {
  __shared__ int warp_sums[kBT / 32];
  __shared__ long long cnt[4];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  if (tid < 4) cnt[tid] = 0;
  __syncthreads();
  const int per = (B + kBT - 1) / kBT;
  const int b0 = min(B, tid * per), b1 = min(B, b0 + per);
  int local[4] = {0, 0, 0, 0};
  for (int b = b0; b < b1; ++b) {
    const int f = fate[b];
    local[f == 3 ? 2 : (f == 2 ? 3 : f)]++;
  }
  for (int k = 0; k < 4; ++k)
    if (local[k]) atomicAdd(reinterpret_cast<unsigned long long*>(&cnt[k]),
                            (unsigned long long)local[k]);
  int v = local[2];
  for (int off = 1; off < 32; off <<= 1) {
    const int t = __shfl_up_sync(0xffffffffu, v, off);
    if (lane >= off) v += t;
  }
  if (lane == 31) warp_sums[warp] = v;
  __syncthreads();
  if (warp == 0) {
    int s = warp_sums[lane];
    for (int off = 1; off < 32; off <<= 1) {
      const int t = __shfl_up_sync(0xffffffffu, s, off);
      if (lane >= off) s += t;
    }
    warp_sums[lane] = s;
  }
  __syncthreads();
  int at = v - local[2] + (warp > 0 ? warp_sums[warp - 1] : 0);
  for (int b = b0; b < b1; ++b) pos[b] = (fate[b] == 3) ? at++ : -1;
  __syncthreads();
  if (tid < 4) counters[tid] = cnt[tid];
}

__global__ void __launch_bounds__(kWT) bab_emit_wide_kernel(const BabWideParams w) {
  const int b = blockIdx.x;
  const int at = w.pos[b];
  if (at < 0) return;
  const int n = w.p.n, ax = w.ax[b];
  const float* bxl = w.bxl + (long long)b * n;
  const float* bxh = w.bxh + (long long)b * n;
  const float mid = __fmul_rn(__fadd_rn(bxl[ax], bxh[ax]), 0.5f);
  for (int i = threadIdx.x; i < n; i += kWT) {
    const long long o = (long long)at * n + i;
    w.p.lo_xl[o] = bxl[i];
    w.p.lo_xh[o] = (i == ax) ? mid : bxh[i];
    w.p.hi_xl[o] = (i == ax) ? mid : bxl[i];
    w.p.hi_xh[o] = bxh[i];
  }
}

}  // namespace
}  // namespace vcb

extern "C" int vcb_bab_step(int32_t B, int32_t n_in, int32_t Q, int32_t D,
                            int32_t q_sens, const int32_t* query_disjunct, const float* xl,
                            const float* xh, const float* lb, const float* A,
                            const float* acc, int32_t clip, int32_t branch_sb,
                            float* lo_xl, float* lo_xh, float* hi_xl, float* hi_xh,
                            int64_t* counters, void* stream) {
  using namespace vcb;
  if (B < 0 || n_in <= 0 || Q <= 0 || D <= 0)
    return fail(VCB_ERR_INVALID, "vcb_bab_step: B=%d n_in=%d Q=%d D=%d", B, n_in, Q, D);
  if (n_in > kMaxIn || Q > kMaxQ)
    return fail(VCB_ERR_UNSUPPORTED, "vcb_bab_step: n_in=%d (max %d), Q=%d (max %d)", n_in,
                kMaxIn, Q, kMaxQ);
  if (!query_disjunct || !counters || (B > 0 && (!xl || !xh || !lb || !lo_xl || !lo_xh ||
                                                 !hi_xl || !hi_xh)))
    return fail(VCB_ERR_INVALID, "vcb_bab_step: NULL pointer");
  if ((clip || branch_sb) && B > 0 && (!A || !acc))
    return fail(VCB_ERR_INVALID, "vcb_bab_step: clipping / SB branching need A and acc");
  if (q_sens <= 0 || q_sens > Q) q_sens = Q;
  BabParams p{B, n_in, Q, D, q_sens, clip ? 1 : 0, branch_sb ? 1 : 0, xl, xh, lb, A, acc,
              query_disjunct, lo_xl, lo_xh, hi_xl, hi_xh,
              reinterpret_cast<long long*>(counters)};
  bab_step_kernel<<<1, kBT, 0, static_cast<cudaStream_t>(stream)>>>(p);
  return check_launch("vcb_bab_step: launch");
}

extern "C" size_t vcb_bab_step_wide_workspace(int32_t B, int32_t n_in) {
  if (B <= 0 || n_in <= 0) return 0;
  return (size_t)B * n_in * 4 * sizeof(float) + (size_t)B * 3 * sizeof(int) + 64;
}

extern "C" int vcb_bab_step_wide(int32_t B, int32_t n_in, int32_t Q, int32_t D, int32_t q_sens,
                                 const int32_t* query_disjunct, const float* xl,
                                 const float* xh, const float* lb, const float* A,
                                 const float* acc, int32_t clip, int32_t branch_sb,
                                 float* lo_xl, float* lo_xh, float* hi_xl, float* hi_xh,
                                 int64_t* counters, void* workspace, size_t workspace_bytes,
                                 void* stream) {
  using namespace vcb;
  if (B < 0 || n_in <= 0 || Q <= 0 || D <= 0)
    return fail(VCB_ERR_INVALID, "vcb_bab_step_wide: B=%d n_in=%d Q=%d D=%d", B, n_in, Q, D);
  if (!query_disjunct || !counters)
    return fail(VCB_ERR_INVALID, "vcb_bab_step_wide: NULL pointer");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (B == 0) {
    if (cudaMemsetAsync(counters, 0, 4 * sizeof(int64_t), st) != cudaSuccess)
      return fail(VCB_ERR_CUDA, "vcb_bab_step_wide: memset");
    return VCB_OK;
  }
  if (!xl || !xh || !lb || !lo_xl || !lo_xh || !hi_xl || !hi_xh)
    return fail(VCB_ERR_INVALID, "vcb_bab_step_wide: NULL pointer");
  if ((clip || branch_sb) && (!A || !acc))
    return fail(VCB_ERR_INVALID, "vcb_bab_step_wide: clipping / SB branching need A and acc");
  if (!workspace || workspace_bytes < vcb_bab_step_wide_workspace(B, n_in))
    return fail(VCB_ERR_INVALID, "vcb_bab_step_wide: workspace too small");
  if (q_sens <= 0 || q_sens > Q) q_sens = Q;
  BabWideParams w{};
  w.p = BabParams{B, n_in, Q, D, q_sens, clip ? 1 : 0, branch_sb ? 1 : 0, xl, xh, lb, A, acc,
                  query_disjunct, lo_xl, lo_xh, hi_xl, hi_xh,
                  reinterpret_cast<long long*>(counters)};
  float* f = static_cast<float*>(workspace);
  const long long bn = (long long)B * n_in;
  w.bxl = f;
  w.bxh = f + bn;
  w.txl = f + 2 * bn;
  w.txh = f + 3 * bn;
  w.fate = reinterpret_cast<int*>(f + 4 * bn);
  w.ax = w.fate + B;
  w.pos = w.ax + B;
  bab_fate_wide_kernel<<<B, kWT, 0, st>>>(w);
  int rc = check_launch("vcb_bab_step_wide: fate");
  if (rc) return rc;
  bab_scan_wide_kernel<<<1, kBT, 0, st>>>(B, w.fate, w.pos, w.p.counters);
  rc = check_launch("vcb_bab_step_wide: scan");
  if (rc) return rc;
  bab_emit_wide_kernel<<<B, kWT, 0, st>>>(w);
  return check_launch("vcb_bab_step_wide: emit");
}
