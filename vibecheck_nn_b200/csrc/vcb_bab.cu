// Input-split BaB step on the device: closure, halfspace clipping, branching
// and child emission for one batch of leaves.
//
// Follows _input_split_batched_inner (verify_graph.py):
//   closure  every disjunct has a query with lb > 0            (:12901-12908)
//   clip     per-(query, dim) projection of {A_q.x + acc_q <= 0} onto the
//            box, per disjunct with a union of the feasible boxes when there
//            are several disjuncts (:12363-12426, :13030-13084), repeated up
//            to clip_iters times while the box shrinks (:13036-13084)
//   branch   first-max argmax of the score: the width, width * sum_q |A_q|
//            (SB), or max_q (max(|A_q|, thr) * width / 2 + lb_q * mw) (SB
//            margin), times a per-dimension boost (:13236-13295)
//   split    K = 1: bisection at the midpoint of the argmax dimension, width
//            <= 1e-12 degenerate, children emitted as a low block then a high
//            block in leaf order (:13353-13382); K > 1: the K best-scoring
//            dimensions, those wider than 1e-12 bisected together, 2^K'
//            children per leaf emitted leaf by leaf in one block, no usable
//            dimension degenerate (:13383-13423)
//
// Iterated clipping runs per leaf until its box stops shrinking.  The
// reference stops every leaf when no leaf of the batch shrinks; a leaf whose
// box did not shrink maps to the same box and the same feasibility in every
// further iteration (the clip is a function of the box and never widens it),
// so the two rules give the same boxes and verdicts.
//
// Two implementations of the same decisions: for n_in <= 64 one CTA whose
// threads each own a contiguous run of leaves (a block-wide scan of the child
// counts gives each child's row); for any n_in one CTA per leaf with
// fixed-order block reductions, a single-CTA scan and one CTA per leaf
// writing its children.
#include <algorithm>

#include "vcb_common.cuh"
#include "vcb_topk.cuh"

namespace vcb {
namespace {

constexpr int kBT = 1024;
constexpr int kMaxIn = 64;
constexpr int kMaxQ = 64;
constexpr int kMaxK = 10;  // split depth: at most 1024 children per leaf

struct BabParams {
  int B, n, Q, D, Qs;  // Qs: leading (unique) queries that count for the SB score
  int clip, clip_iters, sb, margin, K;
  float thr, mw;       // SB margin: coefficient floor and margin weight
  const float* boost;  // (n) SB score multiplier, or NULL
  const float *xl, *xh, *lb, *A, *acc;
  const int* qd;  // disjunct of each query
  float *lo_xl, *lo_xh, *hi_xl, *hi_xh;  // K = 1: low and high child blocks
  float *kid_xl, *kid_xh;                // K > 1: all children, leaf by leaf
  long long* counters;  // [closed_crown, closed_clip, child rows, degenerate]
};

// ---------------------------------------------------------------------------
// shared decisions

__device__ bool leaf_closed(const BabParams& p, int b) {
  bool closed = true;
  for (int d = 0; d < p.D; ++d) {
    bool any = false;
    for (int q = 0; q < p.Q; ++q)
      if (p.qd[q] == d && p.lb[(long long)b * p.Q + q] > 0.f) any = true;
    closed = closed && any;
  }
  return closed;
}

// Branching score of dimension i of leaf b with (clipped) width w
// (verify_graph.py:13244-13290), in the reference's fp32 operation order.
__device__ float branch_score(const BabParams& p, int b, int i, float w) {
  float s;
  if (!p.sb) {
    s = w;
  } else if (p.margin) {
    s = -INFINITY;
    for (int q = 0; q < p.Qs; ++q) {
      const float a = fmaxf(fabsf(p.A[((long long)b * p.Q + q) * p.n + i]), p.thr);
      const float t = __fadd_rn(__fmul_rn(__fmul_rn(a, w), 0.5f),
                                __fmul_rn(p.lb[(long long)b * p.Q + q], p.mw));
      if (q == 0 || t > s) s = t;
    }
  } else {
    float sens = 0.f;
    for (int q = 0; q < p.Qs; ++q)
      sens = __fadd_rn(sens, fabsf(p.A[((long long)b * p.Q + q) * p.n + i]));
    s = __fmul_rn(w, sens);
  }
  if (p.boost) s = __fmul_rn(s, p.boost[i]);
  return s;
}

// K > 1: a dimension is split when its fp32 width, compared in double, is
// above 1e-12 (verify_graph.py:13398); K = 1 compares in fp32 (:13363).
__device__ __forceinline__ bool usable_k(float w) { return (double)w > 1e-12; }

// ---------------------------------------------------------------------------
// n_in <= 64: one CTA, each thread a run of leaves

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

// Clips the box (bxl, bxh) in place, up to clip_iters times while it
// shrinks; false when it is infeasible (the leaf is closed by clipping).
__device__ bool clip_leaf(const BabParams& p, int b, float* bxl, float* bxh) {
  const int n = p.n;
  float nxl[kMaxIn], nxh[kMaxIn];
  for (int it = 0; it < p.clip_iters; ++it) {
    bool feas;
    if (p.D == 1) {
      feas = clip_box(p, b, -1, bxl, bxh, nxl, nxh);
    } else {
      float txl[kMaxIn], txh[kMaxIn];
      feas = false;
      for (int i = 0; i < n; ++i) {
        nxl[i] = INFINITY;
        nxh[i] = -INFINITY;
      }
      for (int d = 0; d < p.D; ++d) {
        if (clip_box(p, b, d, bxl, bxh, txl, txh)) {
          feas = true;
          for (int i = 0; i < n; ++i) {
            nxl[i] = fminf(nxl[i], txl[i]);
            nxh[i] = fmaxf(nxh[i], txh[i]);
          }
        }
      }
    }
    // an infeasible box stays infeasible in later iterations (the clip
    // never widens it), so it closes here
    if (!feas) return false;
    bool shrunk = false;
    for (int i = 0; i < n; ++i) {
      if (nxl[i] > bxl[i] || nxh[i] < bxh[i]) shrunk = true;
      bxl[i] = nxl[i];
      bxh[i] = nxh[i];
    }
    if (!shrunk) break;
  }
  return true;
}

// Fate of leaf b: 0 closed by CROWN, 1 closed by clipping, 2 degenerate,
// 3 split.  Fills the box to split, its split dimensions (in score order)
// and their number.
__device__ int leaf_fate(const BabParams& p, int b, float* bxl, float* bxh, int* dims,
                         int* ndims) {
  const int n = p.n;
  if (leaf_closed(p, b)) return 0;
  for (int i = 0; i < n; ++i) {
    bxl[i] = p.xl[(long long)b * n + i];
    bxh[i] = p.xh[(long long)b * n + i];
  }
  if (p.clip && !clip_leaf(p, b, bxl, bxh)) return 1;
  float sc[kMaxIn];
  for (int i = 0; i < n; ++i) sc[i] = branch_score(p, b, i, __fsub_rn(bxh[i], bxl[i]));
  if (p.K == 1) {
    int best = 0;
    for (int i = 1; i < n; ++i)
      if (sc[i] > sc[best]) best = i;
    dims[0] = best;
    *ndims = 1;
    return (__fsub_rn(bxh[best], bxl[best]) > 1e-12f) ? 3 : 2;
  }
  // the K best scores in torch's CPU topk order (64 K > n here), then the
  // usable ones
  VI q[kMaxIn];
  for (int i = 0; i < n; ++i) q[i] = VI{sc[i], i};
  tk_nth_path(q, n, p.K);
  int nu = 0;
  for (int k = 0; k < p.K; ++k) {
    const int d = q[k].i;
    if (usable_k(__fsub_rn(bxh[d], bxl[d]))) dims[nu++] = d;
  }
  *ndims = nu;
  return nu > 0 ? 3 : 2;
}

__global__ void __launch_bounds__(kBT) bab_step_kernel(const BabParams p) {
  __shared__ int warp_sums[kBT / 32];
  __shared__ long long cnt[4];
  const int tid = threadIdx.x;
  if (tid < 4) cnt[tid] = 0;
  const int per = (p.B + kBT - 1) / kBT;
  const int b0 = min(p.B, tid * per), b1 = min(p.B, b0 + per);
  float bxl[kMaxIn], bxh[kMaxIn];
  int dims[kMaxK], nd;
  long long local[4] = {0, 0, 0, 0};  // closed crown, closed clip, child rows, degenerate
  for (int b = b0; b < b1; ++b) {
    const int f = leaf_fate(p, b, bxl, bxh, dims, &nd);
    if (f == 3) local[2] += p.K == 1 ? 1 : (1 << nd);
    else local[f == 2 ? 3 : f]++;
  }
  __syncthreads();
  for (int k = 0; k < 4; ++k)
    if (local[k]) atomicAdd(reinterpret_cast<unsigned long long*>(&cnt[k]),
                            (unsigned long long)local[k]);
  // exclusive scan of the child-row counts in thread order
  const int lane = tid & 31, warp = tid >> 5;
  int v = (int)local[2];
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
  int pos = v - (int)local[2] + (warp > 0 ? warp_sums[warp - 1] : 0);
  const int n = p.n;
  for (int b = b0; b < b1; ++b) {
    if (leaf_fate(p, b, bxl, bxh, dims, &nd) != 3) continue;
    if (p.K == 1) {
      const int ax = dims[0];
      const float mid = __fmul_rn(__fadd_rn(bxl[ax], bxh[ax]), 0.5f);
      for (int i = 0; i < n; ++i) {
        const long long o = (long long)pos * n + i;
        p.lo_xl[o] = bxl[i];
        p.lo_xh[o] = (i == ax) ? mid : bxh[i];
        p.hi_xl[o] = (i == ax) ? mid : bxl[i];
        p.hi_xh[o] = bxh[i];
      }
      ++pos;
    } else {
      float mids[kMaxK];
      for (int k = 0; k < nd; ++k)
        mids[k] = __fmul_rn(__fadd_rn(bxl[dims[k]], bxh[dims[k]]), 0.5f);
      for (int c = 0; c < (1 << nd); ++c, ++pos) {
        for (int i = 0; i < n; ++i) {
          float lo = bxl[i], hi = bxh[i];
          for (int k = 0; k < nd; ++k)
            if (dims[k] == i) {
              if ((c >> k) & 1) lo = mids[k];  // high half
              else hi = mids[k];               // low half
            }
          p.kid_xl[(long long)pos * n + i] = lo;
          p.kid_xh[(long long)pos * n + i] = hi;
        }
      }
    }
  }
  __syncthreads();
  if (tid < 4) p.counters[tid] = cnt[tid];
}

// ---------------------------------------------------------------------------
// any n_in (e.g. 3072): one CTA per leaf decides its fate with fixed-order
// block reductions, a single CTA scans the child counts, and one CTA per
// leaf writes its children.

constexpr int kWT = 256;

struct BabWideParams {
  BabParams p;
  float *bxl, *bxh;  // (B, n) box to split (clipped)
  float *txl, *txh;  // (B, n) one disjunct's clipped box (D > 1)
  float *uxl, *uxh;  // (B, n) the next iterate of the clip
  int *fate, *nkid, *pos, *dims;  // dims: (B, kMaxK)
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

// Block argmax of score over the dimensions not in `taken` (a shared list of
// ntaken dimensions), ties to the lower index; -1 when none is left.
__device__ int block_argmax(const BabParams& p, int b, const float* bxl, const float* bxh,
                            const int* taken, int ntaken, float* best_v, int* best_i) {
  const int n = p.n, tid = threadIdx.x;
  float bv = -INFINITY;
  int bi = n;
  for (int i = tid; i < n; i += kWT) {
    bool skip = false;
    for (int k = 0; k < ntaken; ++k) skip |= taken[k] == i;
    if (skip) continue;
    const float sc = branch_score(p, b, i, __fsub_rn(bxh[i], bxl[i]));
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
  const int r = best_i[0] < n ? best_i[0] : -1;
  __syncthreads();
  return r;
}

__global__ void __launch_bounds__(kWT) bab_fate_wide_kernel(const BabWideParams w) {
  __shared__ float red[kWT];
  __shared__ int flag, closed_s, shrunk_s, best_i[kWT], taken[kMaxK];
  __shared__ float best_v[kWT];
  __shared__ VI sel[64 * (kMaxK - 1)];  // the top-K selection's pairs
  const BabParams& p = w.p;
  const int b = blockIdx.x, tid = threadIdx.x, n = p.n;
  if (tid == 0) closed_s = leaf_closed(p, b);
  __syncthreads();
  if (closed_s) {
    if (tid == 0) w.fate[b] = 0;
    return;
  }
  float* bxl = w.bxl + (long long)b * n;
  float* bxh = w.bxh + (long long)b * n;
  for (int i = tid; i < n; i += kWT) {
    bxl[i] = p.xl[(long long)b * n + i];
    bxh[i] = p.xh[(long long)b * n + i];
  }
  __syncthreads();
  if (p.clip) {
    // iterate: (bxl, bxh) -> (uxl, uxh), copied back while the box shrinks
    float* uxl = w.uxl + (long long)b * n;
    float* uxh = w.uxh + (long long)b * n;
    for (int it = 0; it < p.clip_iters; ++it) {
      bool feas;
      if (p.D == 1) {
        feas = clip_box_block(p, b, -1, bxl, bxh, uxl, uxh, red, &flag);
      } else {
        float* txl = w.txl + (long long)b * n;
        float* txh = w.txh + (long long)b * n;
        for (int i = tid; i < n; i += kWT) {
          uxl[i] = INFINITY;
          uxh[i] = -INFINITY;
        }
        feas = false;
        for (int d = 0; d < p.D; ++d) {
          if (clip_box_block(p, b, d, bxl, bxh, txl, txh, red, &flag)) {
            feas = true;
            for (int i = tid; i < n; i += kWT) {
              uxl[i] = fminf(uxl[i], txl[i]);
              uxh[i] = fmaxf(uxh[i], txh[i]);
            }
          }
        }
      }
      if (!feas) {
        if (tid == 0) w.fate[b] = 1;
        return;
      }
      if (tid == 0) shrunk_s = 0;
      __syncthreads();
      for (int i = tid; i < n; i += kWT) {
        if (uxl[i] > bxl[i] || uxh[i] < bxh[i]) shrunk_s = 1;
        bxl[i] = uxl[i];
        bxh[i] = uxh[i];
      }
      __syncthreads();
      const bool shrunk = shrunk_s != 0;
      __syncthreads();
      if (!shrunk) break;
    }
  }
  if (p.K == 1) {
    const int a = block_argmax(p, b, bxl, bxh, taken, 0, best_v, best_i);
    if (tid == 0) {
      w.dims[(long long)b * kMaxK] = a;
      const bool ok = __fsub_rn(bxh[a], bxl[a]) > 1e-12f;
      w.fate[b] = ok ? 3 : 2;
      w.nkid[b] = ok ? 1 : 0;
    }
    return;
  }
  // scores to the (free after clipping) txl row, then the top K in torch's
  // CPU topk order by one thread
  float* sc = w.txl + (long long)b * n;
  for (int i = tid; i < n; i += kWT) sc[i] = branch_score(p, b, i, __fsub_rn(bxh[i], bxl[i]));
  __syncthreads();
  if (tid == 0) {
    VI* q = sel;
    const int K = p.K;
    if ((long long)K * 64 <= n) {  // std::partial_sort
      for (int i = 0; i < K; ++i) q[i] = VI{sc[i], i};
      tk_heap_select(q, 0, K, n, [&](int i) { return VI{sc[i], i}; });
      tk_sort_heap(q, 0, K);
    } else {  // n < 64 K <= 64 (kMaxK - 1)
      for (int i = 0; i < n; ++i) q[i] = VI{sc[i], i};
      tk_nth_path(q, n, K);
    }
    int nu = 0;
    for (int k = 0; k < K; ++k) {
      const int d = q[k].i;
      if (usable_k(__fsub_rn(bxh[d], bxl[d]))) w.dims[(long long)b * kMaxK + nu++] = d;
    }
    w.fate[b] = nu > 0 ? 3 : 2;
    w.nkid[b] = nu > 0 ? (1 << nu) : 0;
    w.dims[(long long)b * kMaxK + kMaxK - 1] = nu;  // count of usable dims (K <= kMaxK - 1)
  }
}

__global__ void __launch_bounds__(kBT) bab_scan_wide_kernel(int B, const int* __restrict__ fate,
                                                           const int* __restrict__ nkid,
                                                           int* __restrict__ pos,
                                                           long long* __restrict__ counters) {
  __shared__ int warp_sums[kBT / 32];
  __shared__ long long cnt[4];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  if (tid < 4) cnt[tid] = 0;
  __syncthreads();
  const int per = (B + kBT - 1) / kBT;
  const int b0 = min(B, tid * per), b1 = min(B, b0 + per);
  long long local[4] = {0, 0, 0, 0};
  for (int b = b0; b < b1; ++b) {
    const int f = fate[b];
    if (f == 3) local[2] += nkid[b];
    else local[f == 2 ? 3 : f]++;
  }
  for (int k = 0; k < 4; ++k)
    if (local[k]) atomicAdd(reinterpret_cast<unsigned long long*>(&cnt[k]),
                            (unsigned long long)local[k]);
  int v = (int)local[2];
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
  int at = v - (int)local[2] + (warp > 0 ? warp_sums[warp - 1] : 0);
  for (int b = b0; b < b1; ++b) {
    pos[b] = (fate[b] == 3) ? at : -1;
    if (fate[b] == 3) at += nkid[b];
  }
  __syncthreads();
  if (tid < 4) counters[tid] = cnt[tid];
}

__global__ void __launch_bounds__(kWT) bab_emit_wide_kernel(const BabWideParams w) {
  const int b = blockIdx.x;
  const int at = w.pos[b];
  if (at < 0) return;
  const BabParams& p = w.p;
  const int n = p.n;
  const float* bxl = w.bxl + (long long)b * n;
  const float* bxh = w.bxh + (long long)b * n;
  const int* dims = w.dims + (long long)b * kMaxK;
  if (p.K == 1) {
    const int ax = dims[0];
    const float mid = __fmul_rn(__fadd_rn(bxl[ax], bxh[ax]), 0.5f);
    for (int i = threadIdx.x; i < n; i += kWT) {
      const long long o = (long long)at * n + i;
      p.lo_xl[o] = bxl[i];
      p.lo_xh[o] = (i == ax) ? mid : bxh[i];
      p.hi_xl[o] = (i == ax) ? mid : bxl[i];
      p.hi_xh[o] = bxh[i];
    }
    return;
  }
  const int nd = dims[kMaxK - 1];
  for (int c = 0; c < (1 << nd); ++c) {
    const long long row = (long long)(at + c) * n;
    for (int i = threadIdx.x; i < n; i += kWT) {
      float lo = bxl[i], hi = bxh[i];
      for (int k = 0; k < nd; ++k)
        if (dims[k] == i) {
          const float mid = __fmul_rn(__fadd_rn(bxl[i], bxh[i]), 0.5f);
          if ((c >> k) & 1) lo = mid;  // high half
          else hi = mid;               // low half
        }
      p.kid_xl[row + i] = lo;
      p.kid_xh[row + i] = hi;
    }
  }
}

int check_opts(const vcb_bab_opts* o, int n_in, const char* who) {
  if (!o) return VCB_OK;
  if (o->clip_iters < 1 || o->split_depth < 1 || o->split_depth > kMaxK - 1)
    return fail(VCB_ERR_INVALID, "%s: clip_iters=%d split_depth=%d (1 <= depth <= %d)", who,
                o->clip_iters, o->split_depth, kMaxK - 1);
  if (o->split_depth > n_in)
    return fail(VCB_ERR_INVALID, "%s: split_depth=%d exceeds n_in=%d", who, o->split_depth,
                n_in);
  return VCB_OK;
}

BabParams make_params(int B, int n_in, int Q, int D, int q_sens, const int32_t* qd,
                      const float* xl, const float* xh, const float* lb, const float* A,
                      const float* acc, const vcb_bab_opts& o, float* lo_xl, float* lo_xh,
                      float* hi_xl, float* hi_xh, float* kid_xl, float* kid_xh,
                      int64_t* counters) {
  if (q_sens <= 0 || q_sens > Q) q_sens = Q;
  BabParams p{};
  p.B = B;
  p.n = n_in;
  p.Q = Q;
  p.D = D;
  p.Qs = q_sens;
  p.clip = o.clip ? 1 : 0;
  p.clip_iters = o.clip_iters;
  p.sb = o.branch_sb ? 1 : 0;
  p.margin = o.margin_score ? 1 : 0;
  p.K = o.split_depth;
  p.thr = o.coeff_thresh;
  p.mw = o.margin_weight;
  p.boost = o.boost;
  p.xl = xl;
  p.xh = xh;
  p.lb = lb;
  p.A = A;
  p.acc = acc;
  p.qd = qd;
  p.lo_xl = lo_xl;
  p.lo_xh = lo_xh;
  p.hi_xl = hi_xl;
  p.hi_xh = hi_xh;
  p.kid_xl = kid_xl;
  p.kid_xh = kid_xh;
  p.counters = reinterpret_cast<long long*>(counters);
  return p;
}

vcb_bab_opts default_opts(int32_t clip, int32_t branch_sb) {
  vcb_bab_opts o{};
  o.clip = clip;
  o.clip_iters = 1;
  o.branch_sb = branch_sb;
  o.margin_score = 0;
  o.split_depth = 1;
  o.coeff_thresh = 0.01f;
  o.margin_weight = 1.f;
  o.boost = nullptr;
  return o;
}

}  // namespace
}  // namespace vcb

extern "C" int vcb_bab_step_ex(int32_t B, int32_t n_in, int32_t Q, int32_t D, int32_t q_sens,
                               const int32_t* query_disjunct, const float* xl, const float* xh,
                               const float* lb, const float* A, const float* acc,
                               const vcb_bab_opts* opts, float* lo_xl, float* lo_xh,
                               float* hi_xl, float* hi_xh, float* kid_xl, float* kid_xh,
                               int64_t* counters, void* stream) {
  using namespace vcb;
  const char* who = "vcb_bab_step";
  if (B < 0 || n_in <= 0 || Q <= 0 || D <= 0 || !opts)
    return fail(VCB_ERR_INVALID, "%s: B=%d n_in=%d Q=%d D=%d opts=%p", who, B, n_in, Q, D,
                (const void*)opts);
  int rc = check_opts(opts, n_in, who);
  if (rc) return rc;
  if (n_in > kMaxIn || Q > kMaxQ)
    return fail(VCB_ERR_UNSUPPORTED, "%s: n_in=%d (max %d), Q=%d (max %d)", who, n_in, kMaxIn,
                Q, kMaxQ);
  const vcb_bab_opts& o = *opts;
  if (!query_disjunct || !counters || (B > 0 && (!xl || !xh || !lb)))
    return fail(VCB_ERR_INVALID, "%s: NULL pointer", who);
  if (B > 0 && (o.split_depth == 1 ? (!lo_xl || !lo_xh || !hi_xl || !hi_xh)
                                   : (!kid_xl || !kid_xh)))
    return fail(VCB_ERR_INVALID, "%s: NULL child buffer", who);
  if ((o.clip || o.branch_sb) && B > 0 && (!A || !acc))
    return fail(VCB_ERR_INVALID, "%s: clipping / SB branching need A and acc", who);
  const BabParams p = make_params(B, n_in, Q, D, q_sens, query_disjunct, xl, xh, lb, A, acc, o,
                                  lo_xl, lo_xh, hi_xl, hi_xh, kid_xl, kid_xh, counters);
  bab_step_kernel<<<1, kBT, 0, static_cast<cudaStream_t>(stream)>>>(p);
  return check_launch("vcb_bab_step: launch");
}

extern "C" int vcb_bab_step(int32_t B, int32_t n_in, int32_t Q, int32_t D,
                            int32_t q_sens, const int32_t* query_disjunct, const float* xl,
                            const float* xh, const float* lb, const float* A,
                            const float* acc, int32_t clip, int32_t branch_sb,
                            float* lo_xl, float* lo_xh, float* hi_xl, float* hi_xh,
                            int64_t* counters, void* stream) {
  const vcb_bab_opts o = vcb::default_opts(clip, branch_sb);
  return vcb_bab_step_ex(B, n_in, Q, D, q_sens, query_disjunct, xl, xh, lb, A, acc, &o, lo_xl,
                         lo_xh, hi_xl, hi_xh, nullptr, nullptr, counters, stream);
}

extern "C" size_t vcb_bab_step_wide_workspace(int32_t B, int32_t n_in) {
  if (B <= 0 || n_in <= 0) return 0;
  return (size_t)B * n_in * 6 * sizeof(float) + (size_t)B * (3 + vcb::kMaxK) * sizeof(int) + 64;
}

extern "C" int vcb_bab_step_wide_ex(int32_t B, int32_t n_in, int32_t Q, int32_t D,
                                    int32_t q_sens, const int32_t* query_disjunct,
                                    const float* xl, const float* xh, const float* lb,
                                    const float* A, const float* acc, const vcb_bab_opts* opts,
                                    float* lo_xl, float* lo_xh, float* hi_xl, float* hi_xh,
                                    float* kid_xl, float* kid_xh, int64_t* counters,
                                    void* workspace, size_t workspace_bytes, void* stream) {
  using namespace vcb;
  const char* who = "vcb_bab_step_wide";
  if (B < 0 || n_in <= 0 || Q <= 0 || D <= 0 || !opts)
    return fail(VCB_ERR_INVALID, "%s: B=%d n_in=%d Q=%d D=%d", who, B, n_in, Q, D);
  int rc = check_opts(opts, n_in, who);
  if (rc) return rc;
  const vcb_bab_opts& o = *opts;
  if (!query_disjunct || !counters) return fail(VCB_ERR_INVALID, "%s: NULL pointer", who);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (B == 0) {
    if (cudaMemsetAsync(counters, 0, 4 * sizeof(int64_t), st) != cudaSuccess)
      return fail(VCB_ERR_CUDA, "%s: memset", who);
    return VCB_OK;
  }
  if (!xl || !xh || !lb) return fail(VCB_ERR_INVALID, "%s: NULL pointer", who);
  if (o.split_depth == 1 ? (!lo_xl || !lo_xh || !hi_xl || !hi_xh) : (!kid_xl || !kid_xh))
    return fail(VCB_ERR_INVALID, "%s: NULL child buffer", who);
  if ((o.clip || o.branch_sb) && (!A || !acc))
    return fail(VCB_ERR_INVALID, "%s: clipping / SB branching need A and acc", who);
  if (!workspace || workspace_bytes < vcb_bab_step_wide_workspace(B, n_in))
    return fail(VCB_ERR_INVALID, "%s: workspace too small", who);
  BabWideParams w{};
  w.p = make_params(B, n_in, Q, D, q_sens, query_disjunct, xl, xh, lb, A, acc, o, lo_xl, lo_xh,
                    hi_xl, hi_xh, kid_xl, kid_xh, counters);
  float* f = static_cast<float*>(workspace);
  const long long bn = (long long)B * n_in;
  w.bxl = f;
  w.bxh = f + bn;
  w.txl = f + 2 * bn;
  w.txh = f + 3 * bn;
  w.uxl = f + 4 * bn;
  w.uxh = f + 5 * bn;
  w.fate = reinterpret_cast<int*>(f + 6 * bn);
  w.nkid = w.fate + B;
  w.pos = w.nkid + B;
  w.dims = w.pos + B;
  bab_fate_wide_kernel<<<B, kWT, 0, st>>>(w);
  rc = check_launch("vcb_bab_step_wide: fate");
  if (rc) return rc;
  bab_scan_wide_kernel<<<1, kBT, 0, st>>>(B, w.fate, w.nkid, w.pos, w.p.counters);
  rc = check_launch("vcb_bab_step_wide: scan");
  if (rc) return rc;
  bab_emit_wide_kernel<<<B, kWT, 0, st>>>(w);
  return check_launch("vcb_bab_step_wide: emit");
}

extern "C" int vcb_bab_step_wide(int32_t B, int32_t n_in, int32_t Q, int32_t D, int32_t q_sens,
                                 const int32_t* query_disjunct, const float* xl,
                                 const float* xh, const float* lb, const float* A,
                                 const float* acc, int32_t clip, int32_t branch_sb,
                                 float* lo_xl, float* lo_xh, float* hi_xl, float* hi_xh,
                                 int64_t* counters, void* workspace, size_t workspace_bytes,
                                 void* stream) {
  const vcb_bab_opts o = vcb::default_opts(clip, branch_sb);
  return vcb_bab_step_wide_ex(B, n_in, Q, D, q_sens, query_disjunct, xl, xh, lb, A, acc, &o,
                              lo_xl, lo_xh, hi_xl, hi_xh, nullptr, nullptr, counters, workspace,
                              workspace_bytes, stream);
}
