// Batched PGD counterexample search for ReLU MLPs.
//
// Two kernels share one shared-memory layout (fc weights resident, one tile of
// up to kPS samples per CTA -- kPSBig for the simple attack when the network
// leaves room -- pre-activations kept for the ReLU masks) and the same tile
// forward / backward passes:
//
// * pgd_mlp_kernel -- the sign-gradient PGD of _simple_pgd / _simple_pgd_batched
//   (verify_hybrid_acasxu.py:39-161).  Each sample x (a restart inside its box
//   [lo, hi]) runs n_iter steps of
//     y = f(x);  m_d = max_c (C_c . y + cb_c) over the constraints of disjunct d
//     loss = min_d m_d;  SAT when loss <= 1e-6;
//     x <- clamp(x - lr * sign(dloss/dx) * (hi - lo), lo, hi).
//   max/min route the gradient to the first extremal index (torch autograd).
//   A sample that becomes SAT stops moving; the reported witness is the SAT
//   sample with the smallest (iteration, index) -- the sample the reference's
//   loop, which checks every sample once per iteration and returns the first
//   SAT one, would return.
//
// * pgd_general_kernel -- pgd_attack_general (pgd.py:233-524): optional OSI
//   initialisation (sign ascent on w_r . f(x), :378-402), then per iteration a
//   witness screen (:443-451), the hinge loss sum_c clamp(m_c, min=thr) over the
//   active disjuncts' rows (:469-492, optionally only restart r's disjunct),
//   its gradient, the sign_sgd / adam_sign / adam_clipping step of _PGDOptim
//   (:127-187) and the per-iteration step decay; a final screen after the loop.
//   The plateau give-up (:453-467) depends on the minimum margin over all
//   restarts, so the kernel records that minimum per iteration and the host
//   replays the give-up rule; the wall-time budget is checked in the kernel on
//   the GPU's global timer.
//
// F.relu passes the gradient where the pre-activation is > 0 in both.
#include <algorithm>
#include <climits>

#include "vcb_common.cuh"

namespace vcb {
namespace {

constexpr int kPT = 1024;  // threads per CTA (16 per sample: the iterations are latency-bound)
constexpr int kPS = 64;    // samples per tile
constexpr int kPSBig = 72; // tile of the simple attack when the network leaves room for it
constexpr int kPMaxW = 128;

// Shared-memory layout of the network and one sample tile (offsets in floats).
// The activation rows need no padding beyond n: every loop over inputs stops
// at the layer width.
struct PgdNet {
  int n_fc;
  int dims[VCB_MAX_FC + 1];
  const float* W;
  const float* b;
  long long w_goff[VCB_MAX_FC];
  int b_goff[VCB_MAX_FC];
  int wt_soff[VCB_MAX_FC];  // [W^T; b] ((n_in + 1) rows x pwt floats, zero-padded)
  int pwt[VCB_MAX_FC];
  int pa;                 // activation row stride (odd)
  int pz;                 // pre-activation / gradient row stride (4 x odd)
  int act_soff;           // 2 ping-pong activation buffers, kPS x pa
  int z_soff;             // n_fc pre-activation buffers, kPS x pz
  int g_soff, x_soff, c_soff;
};

struct PgdParams {
  PgdNet net;
  int N, R, n_iter, ncon, D;
  int ntiles;             // tiles of N / ntiles samples, a multiple of the grid
  float lr;
  float* x;               // (N, n_in) in/out
  const float *lo, *hi;   // (N / R, n_in) box of each group of R samples
  const float *C, *cb;    // (ncon, n_out), (ncon,)
  const int* cdis;        // disjunct of each constraint (0..D-1)
  unsigned long long* best;  // min over SAT samples of (iter << 32 | index)
};

struct PgdGenParams {
  PgdNet net;
  int N, R, n_osi, n_iter, ncon, D, n_act, prd, optim, step_rows, plateau;
  int m1_soff, m2_soff, cur_soff, mg_soff;
  float hinge, decay, beta1, beta2, one_m_beta1, one_m_beta2, eps;
  double confirm_thr, hinge_d;
  unsigned long long budget_ns;   // 0: no wall-time budget
  float* x;                       // (N, n_in) in/out
  const float *lo, *hi;           // (N / R, n_in)
  const float* step0;             // (step_rows, n_in); row s % R when step_rows == R
  const float* w_d;               // (R, n_out) OSI projections, or NULL
  const float* inv_bc1;           // (n_iter) float32(1 / float32(1 - beta1^t))
  const float* inv_sbc2;          // (n_iter) float32(1 / float32(sqrt(1 - beta2^t)))
  const float *C, *cb;            // (ncon, n_out), (ncon,)
  const int* cdis;                // disjunct of each row among all D
  const int* cact;                // ordinal of the row's disjunct among the active ones, or -1
  unsigned long long* best;       // min over confirmed witnesses of (screen << 32 | index)
  unsigned int* gmin;             // (n_iter + 2) order-encoded min active margin per screen
  int* t_stop;                    // screen at which the wall-time budget ended the loop
};

__device__ __forceinline__ float sgnf(float v) { return v > 0.f ? 1.f : (v < 0.f ? -1.f : 0.f); }

// Monotone float -> unsigned map, so atomicMin on the code is a float minimum.
__device__ __forceinline__ unsigned int order_code(float f) {
  const unsigned int u = __float_as_uint(f);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

__device__ __forceinline__ float order_decode(unsigned int u) {
  return __uint_as_float((u & 0x80000000u) ? (u & 0x7FFFFFFFu) : ~u);
}

__device__ __forceinline__ unsigned long long global_ns() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// Every fc layer as [W^T; b] in shared memory: row i < n_in holds W[:, i],
// row n_in the bias, columns zero-padded to pwt (a multiple of 4).
__device__ void load_net(const PgdNet& n, float* sm, int tid) {
  for (int l = 0; l < n.n_fc; ++l) {
    const int nin = n.dims[l], nout = n.dims[l + 1], pwt = n.pwt[l];
    float* dt = sm + n.wt_soff[l];
    const float* Wg = n.W + n.w_goff[l];
    const float* bg = n.b + n.b_goff[l];
    for (int i = tid >> 5; i <= nin; i += kPT / 32)
      for (int o = tid & 31; o < pwt; o += 32)
        dt[i * pwt + o] = (o < nout) ? (i < nin ? Wg[(long long)o * nin + i] : bg[o]) : 0.f;
  }
}

// Forward pass of the tile's first ns samples xs (kPS x n0): z_l kept for the
// masks, a_{l+1} = relu(z_l); the network output is z_{n_fc-1}.  A thread
// computes 4 consecutive outputs of one sample: z[o] = sum_i a[i] W[o][i] in
// ascending i, then + b[o].  Rows from ns on are left as they were (the
// passes are bound by shared-memory traffic, which scales with the samples
// processed).
template <int PS>
__device__ void tile_forward(const PgdNet& n, float* sm, const float* xs, int tid, int ns) {
  const int n0 = n.dims[0], pa = n.pa, pz = n.pz;
  float* a_cur = sm + n.act_soff;
  for (int idx = tid; idx < ns * n0; idx += kPT) {
    const int s = idx / n0, i = idx - s * n0;
    a_cur[s * pa + i] = xs[idx];
  }
  __syncthreads();
  for (int l = 0; l < n.n_fc; ++l) {
    const int nin = n.dims[l], nout = n.dims[l + 1], pwt = n.pwt[l];
    const float* sWT = sm + n.wt_soff[l];
    const float* ain = sm + n.act_soff + (l & 1) * PS * pa;
    float* aout = sm + n.act_soff + ((l + 1) & 1) * PS * pa;
    float* z = sm + n.z_soff + l * PS * pz;
    const int nob = pwt >> 2;
    for (int idx = tid; idx < ns * nob; idx += kPT) {
      const int ob = idx / ns, s = idx - ob * ns;
      const int o4 = 4 * ob;
      const float* ar = ain + s * pa;
      float a0 = 0.f, a1 = 0.f, a2 = 0.f, a3 = 0.f;
      for (int i = 0; i < nin; ++i) {
        const float av = ar[i];
        const float4 wv = *reinterpret_cast<const float4*>(sWT + i * pwt + o4);
        a0 = fmaf(av, wv.x, a0);
        a1 = fmaf(av, wv.y, a1);
        a2 = fmaf(av, wv.z, a2);
        a3 = fmaf(av, wv.w, a3);
      }
      const float4 bv = *reinterpret_cast<const float4*>(sWT + nin * pwt + o4);
      const float zz[4] = {__fadd_rn(a0, bv.x), __fadd_rn(a1, bv.y), __fadd_rn(a2, bv.z),
                           __fadd_rn(a3, bv.w)};
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int o = o4 + j;
        if (o < nout) {
          z[s * pz + o] = zz[j];
          aout[s * pa + o] = fmaxf(zz[j], 0.f);
        }
      }
    }
    __syncthreads();
  }
}

// Backward pass of the tile's first ns samples: g (kPS x pz, seeded with
// d loss / d y, zero past n_out) is replaced by d loss / d x in its first n0
// columns.  Sample sl of the tile gets the kPT / ns threads tid = sl + ns k
// (at least kPT / PS of them), each summing whole input columns.
template <int PS>
__device__ void tile_backward(const PgdNet& n, float* sm, int tid, int ns) {
  const int pz = n.pz;
  float* g = sm + n.g_soff;
  const int step = kPT / ns;
  const int sl = tid % ns, i0 = tid / ns;
  const bool active = i0 < step;
  for (int l = n.n_fc - 1; l >= 0; --l) {
    const int nin = n.dims[l], nout = n.dims[l + 1], pwt = n.pwt[l];
    const float* sWT = sm + n.wt_soff[l];
    const float* zprev = (l > 0) ? sm + n.z_soff + (l - 1) * PS * pz : nullptr;
    float vals[(kPMaxW + kPT / PS - 1) / (kPT / PS)];
    const float* grow = g + sl * pz;
    const int kend = pad4(nout);
    int cnt = 0;
    for (int i = active ? i0 : nin; i < nin; i += step) {
      // sum over o in fixed ascending order, 4 at a time (g and W^T rows are
      // zero past n_out)
      const float* wt = sWT + i * pwt;
      float acc = 0.f;
      for (int o = 0; o < kend; o += 4) {
        const float4 gv = *reinterpret_cast<const float4*>(grow + o);
        const float4 wv = *reinterpret_cast<const float4*>(wt + o);
        acc = fmaf(gv.x, wv.x, acc);
        acc = fmaf(gv.y, wv.y, acc);
        acc = fmaf(gv.z, wv.z, acc);
        acc = fmaf(gv.w, wv.w, acc);
      }
      if (zprev && !(zprev[sl * pz + i] > 0.f)) acc = 0.f;
      vals[cnt++] = acc;
    }
    __syncthreads();  // every thread has read g
    cnt = 0;
    for (int i = active ? i0 : pz; i < pz; i += step) g[sl * pz + i] = (i < nin) ? vals[cnt++] : 0.f;
    __syncthreads();
  }
}

template <int PS>
__global__ void __launch_bounds__(kPT, 1) pgd_mlp_kernel(const __grid_constant__ PgdParams p) {
  extern __shared__ __align__(16) float sm[];
  __shared__ int done[PS];
  __shared__ int cstar[PS];
  __shared__ int stop;
  const PgdNet& n = p.net;
  const int tid = threadIdx.x;
  const int nfc = n.n_fc;
  const int n0 = n.dims[0];
  const int nL = n.dims[nfc];
  load_net(n, sm, tid);
  float* Cs = sm + n.c_soff;
  for (int idx = tid; idx < p.ncon * nL; idx += kPT) Cs[idx] = p.C[idx];
  for (int idx = tid; idx < p.ncon; idx += kPT) Cs[p.ncon * nL + idx] = p.cb[idx];
  __syncthreads();
  const int pz = n.pz;
  float* xs = sm + n.x_soff;  // PS x n0 current samples
  float* g = sm + n.g_soff;   // PS x pz gradient rows
  // p.ntiles tiles of N / ntiles samples each (at most PS), a whole number
  // of rounds of the grid: no round with a few tiles while the other CTAs idle
  for (int tile = blockIdx.x; tile < p.ntiles; tile += gridDim.x) {
    const int s0 = (int)((long long)tile * p.N / p.ntiles);
    const int ns = (int)((long long)(tile + 1) * p.N / p.ntiles) - s0;
    for (int idx = tid; idx < PS * n0; idx += kPT) {
      const int s = idx / n0, i = idx - s * n0;
      xs[idx] = s < ns ? p.x[(long long)(s0 + s) * n0 + i] : 0.f;
    }
    for (int s = tid; s < PS; s += kPT) done[s] = s < ns ? 0 : 1;
    __syncthreads();
    for (int it = 0; it < p.n_iter; ++it) {
      // once a SAT sample exists at an earlier iteration nothing here can win
      if (tid == 0) {
        const unsigned long long bk = *reinterpret_cast<volatile unsigned long long*>(p.best);
        stop = (bk >> 32) < (unsigned long long)it;
      }
      __syncthreads();
      if (stop) break;
      tile_forward<PS>(n, sm, xs, tid, ns);
      // ---- margins, SAT check and the output gradient row
      const float* y = sm + n.z_soff + (nfc - 1) * PS * pz;
      for (int s = tid; s < PS; s += kPT) {
        if (done[s]) continue;
        float dmin = 0.f;
        int cbest = 0;
        for (int d = 0; d < p.D; ++d) {
          float dmax = 0.f;
          int carg = -1;
          for (int c = 0; c < p.ncon; ++c) {
            if (p.cdis[c] != d) continue;
            float m = 0.f;
            for (int o = 0; o < nL; ++o) m = fmaf(y[s * pz + o], Cs[c * nL + o], m);
            m = __fadd_rn(m, Cs[p.ncon * nL + c]);
            if (carg < 0 || m > dmax) {
              dmax = m;
              carg = c;
            }
          }
          if (d == 0 || dmax < dmin) {
            dmin = dmax;
            cbest = carg;
          }
        }
        cstar[s] = cbest;
        if (dmin <= 1e-6f) {
          done[s] = 2;
          atomicMin(p.best, ((unsigned long long)it << 32) | (unsigned long long)(s0 + s));
        }
      }
      __syncthreads();
      // ---- backward: g = C[c*], then g <- (g W_l) masked by z_{l-1} > 0
      for (int idx = tid; idx < PS * pz; idx += kPT) {
        const int s = idx / pz, o = idx - s * pz;
        g[idx] = (o < nL && !done[s]) ? Cs[cstar[s] * nL + o] : 0.f;
      }
      __syncthreads();
      tile_backward<PS>(n, sm, tid, ns);
      // ---- sign step and clamp (SAT samples keep the x that was SAT)
      for (int idx = tid; idx < ns * n0; idx += kPT) {
        const int s = idx / n0, i = idx - s * n0;
        if (done[s]) continue;
        const long long bi = (long long)((s0 + s) / p.R) * n0 + i;
        const float lo = p.lo[bi], hi = p.hi[bi];
        const float gv = g[s * pz + i];
        const float step = __fmul_rn(__fmul_rn(p.lr, sgnf(gv)), __fsub_rn(hi, lo));
        const float xn = __fsub_rn(xs[s * n0 + i], step);
        xs[s * n0 + i] = fmaxf(fminf(xn, hi), lo);
      }
      __syncthreads();
    }
    for (int idx = tid; idx < ns * n0; idx += kPT) p.x[(long long)s0 * n0 + idx] = xs[idx];
    __syncthreads();
  }
}

__global__ void __launch_bounds__(kPT, 1)
    pgd_general_kernel(const __grid_constant__ PgdGenParams p) {
  extern __shared__ __align__(16) float sm[];
  __shared__ int stop, final_screen, found, gave_up;
  __shared__ unsigned int tile_min;
  __shared__ double best_min;
  __shared__ int no_improve;
  const PgdNet& n = p.net;
  const int tid = threadIdx.x;
  const int nfc = n.n_fc;
  const int n0 = n.dims[0];
  const int nL = n.dims[nfc];
  const int ncon = p.ncon;
  const unsigned long long t0 = global_ns();
  load_net(n, sm, tid);
  float* Cs = sm + n.c_soff;
  for (int idx = tid; idx < ncon * nL; idx += kPT) Cs[idx] = p.C[idx];
  for (int idx = tid; idx < ncon; idx += kPT) Cs[ncon * nL + idx] = p.cb[idx];
  __syncthreads();
  const int pz = n.pz;
  float* xs = sm + n.x_soff;     // kPS x n0 current iterate
  float* g = sm + n.g_soff;      // kPS x pz gradient rows
  float* m1 = sm + p.m1_soff;    // kPS x n0 Adam first moment
  float* m2 = sm + p.m2_soff;    // kPS x n0 Adam second moment
  float* cur = sm + p.cur_soff;  // kPS x n0 decayed step size
  float* mg = sm + p.mg_soff;    // kPS x ncon margins of the current screen
  const float* y = sm + n.z_soff + (nfc - 1) * kPS * pz;
  const int ntiles = (p.N + kPS - 1) / kPS;
  // with one tile the CTA sees every restart and applies the plateau give-up
  // itself; otherwise the host replays it from gmin
  const bool whole_pool = ntiles == 1;
  for (int tile = blockIdx.x; tile < ntiles; tile += gridDim.x) {
    const int s0 = tile * kPS;
    const int ns = min(kPS, p.N - s0);
    if (tid == 0) {
      best_min = __longlong_as_double(0x7FF0000000000000ll);  // +inf
      no_improve = 0;
    }
    for (int idx = tid; idx < kPS * n0; idx += kPT) {
      const int s = idx / n0, i = idx - s * n0;
      float xv = 0.f, st = 0.f;
      if (s < ns) {
        xv = p.x[(long long)(s0 + s) * n0 + i];
        const int row = p.step_rows == 1 ? 0 : (s0 + s) % p.R;
        st = p.step0[(long long)row * n0 + i];
      }
      xs[idx] = xv;
      cur[idx] = st;
      m1[idx] = 0.f;
      m2[idx] = 0.f;
    }
    __syncthreads();
    // ---- OSI: x <- clamp(x + step0 * sign(d (w_r . f(x)) / dx), lo, hi)
    for (int k = 0; k < p.n_osi; ++k) {
      tile_forward<kPS>(n, sm, xs, tid, ns);
      for (int idx = tid; idx < kPS * pz; idx += kPT) {
        const int s = idx / pz, o = idx - s * pz;
        g[idx] = (o < nL && s < ns) ? p.w_d[(long long)((s0 + s) % p.R) * nL + o] : 0.f;
      }
      __syncthreads();
      tile_backward<kPS>(n, sm, tid, ns);
      for (int idx = tid; idx < ns * n0; idx += kPT) {
        const int s = idx / n0, i = idx - s * n0;
        const long long bi = (long long)((s0 + s) / p.R) * n0 + i;
        const int row = p.step_rows == 1 ? 0 : (s0 + s) % p.R;
        const float st = p.step0[(long long)row * n0 + i];
        const float xn = __fadd_rn(xs[idx], __fmul_rn(st, sgnf(g[s * pz + i])));
        xs[idx] = fminf(fmaxf(xn, p.lo[bi]), p.hi[bi]);
      }
      __syncthreads();
    }
    // ---- screens 1..n_iter with an update after each, then the final screen
    for (int t = 1; t <= p.n_iter + 1; ++t) {
      if (tid == 0) {
        const unsigned long long bk = *reinterpret_cast<volatile unsigned long long*>(p.best);
        stop = (bk >> 32) < (unsigned long long)t;
        final_screen = (t == p.n_iter + 1) ||
                       (p.budget_ns != 0ull && global_ns() - t0 > p.budget_ns);
        found = 0;
        gave_up = 0;
        tile_min = 0xFFFFFFFFu;
      }
      __syncthreads();
      if (stop) break;
      tile_forward<kPS>(n, sm, xs, tid, ns);
      for (int idx = tid; idx < ns * ncon; idx += kPT) {
        const int s = idx / ncon, c = idx - s * ncon;
        float m = 0.f;
        for (int o = 0; o < nL; ++o) m = fmaf(y[s * pz + o], Cs[c * nL + o], m);
        mg[idx] = __fadd_rn(m, Cs[ncon * nL + c]);
      }
      __syncthreads();
      // witness screen: a candidate has an active margin <= 0; it is confirmed
      // when some disjunct has every margin <= the spec's bloat (spec.check)
      for (int s = tid; s < ns; s += kPT) {
        const float* ms = mg + s * ncon;
        float amin = 0.f;
        bool have = false;
        for (int c = 0; c < ncon; ++c)
          if (p.cact[c] >= 0) {
            amin = have ? fminf(amin, ms[c]) : ms[c];
            have = true;
          }
        if (have) atomicMin(&tile_min, order_code(amin));
        if (!(have && amin <= 0.f)) continue;
        bool conf = false;
        for (int d = 0; d < p.D && !conf; ++d) {
          bool any = false;
          float dmax = 0.f;
          for (int c = 0; c < ncon; ++c)
            if (p.cdis[c] == d) {
              dmax = any ? fmaxf(dmax, ms[c]) : ms[c];
              any = true;
            }
          conf = any && (double)dmax <= p.confirm_thr;
        }
        if (conf) {
          found = 1;
          atomicMin(p.best, ((unsigned long long)t << 32) | (unsigned long long)(s0 + s));
        }
      }
      __syncthreads();
      if (tid == 0) {
        if (t <= p.n_iter && tile_min != 0xFFFFFFFFu) atomicMin(p.gmin + t, tile_min);
        if (final_screen && t <= p.n_iter) atomicMin(p.t_stop, t);
        if (whole_pool && !found && !final_screen && tile_min != 0xFFFFFFFFu) {
          // pgd.py:453-467 in double, as the host evaluates it
          const double cur_min = (double)order_decode(tile_min);
          if (cur_min > (double)p.hinge_d) {
            if (cur_min < best_min - 1e-6) {
              best_min = cur_min;
              no_improve = 0;
            } else {
              ++no_improve;
            }
            gave_up = no_improve >= p.plateau;
          } else {
            no_improve = 0;
          }
        }
      }
      __syncthreads();
      if (found || final_screen || gave_up) break;  // block-uniform
      // ---- hinge-loss gradient: sum of the active rows with margin >= thr
      for (int idx = tid; idx < kPS * pz; idx += kPT) {
        const int s = idx / pz, o = idx - s * pz;
        float gv = 0.f;
        if (o < nL && s < ns) {
          const int target = p.prd ? ((s0 + s) % p.R) % p.n_act : -1;
          for (int c = 0; c < ncon; ++c) {
            const int a = p.cact[c];
            if (a < 0 || (target >= 0 && a != target)) continue;
            if (mg[s * ncon + c] >= p.hinge) gv = __fadd_rn(gv, Cs[c * nL + o]);
          }
        }
        g[idx] = gv;
      }
      __syncthreads();
      tile_backward<kPS>(n, sm, tid, ns);
      // ---- optimiser step, clamp, step decay
      const float sc1 = p.inv_bc1[t - 1], sc2 = p.inv_sbc2[t - 1];
      for (int idx = tid; idx < ns * n0; idx += kPT) {
        const int s = idx / n0, i = idx - s * n0;
        const long long bi = (long long)((s0 + s) / p.R) * n0 + i;
        const float gv = g[s * pz + i];
        const float step = cur[idx];
        float delta;
        if (p.optim == 0) {
          delta = __fmul_rn(step, sgnf(gv));
        } else {
          // m.mul_(b1).add_(g, alpha=1-b1); v.mul_(b2).addcmul_(g, g, value=1-b2)
          const float a = fmaf(gv, p.one_m_beta1, __fmul_rn(m1[idx], p.beta1));
          const float v = fmaf(__fmul_rn(gv, gv), p.one_m_beta2, __fmul_rn(m2[idx], p.beta2));
          m1[idx] = a;
          m2[idx] = v;
          const float denom = __fadd_rn(__fmul_rn(__fsqrt_rn(v), sc2), p.eps);
          const float dir = sgnf(__fdiv_rn(a, denom));
          delta = p.optim == 1 ? __fmul_rn(step, dir) : __fmul_rn(__fmul_rn(step, sc1), dir);
        }
        const float xn = __fsub_rn(xs[idx], delta);
        xs[idx] = fminf(fmaxf(xn, p.lo[bi]), p.hi[bi]);
        cur[idx] = __fmul_rn(step, p.decay);
      }
      __syncthreads();
    }
    for (int idx = tid; idx < ns * n0; idx += kPT) p.x[(long long)s0 * n0 + idx] = xs[idx];
    __syncthreads();
  }
}

// ---- layer-wise PGD pieces (networks outside the shared-memory kernels):
// the forward / backward passes run on the layer kernels; these two kernels
// are the per-iteration screen and update of both attacks.

struct ScreenArgs {
  int N, n_out, ldy, ldg, ncon, D, n_act, prd, R, t, simple;
  float hinge;
  double confirm_thr;
  const float *y, *C, *cb;
  const int *cdis, *cact;
  unsigned long long* best;
  unsigned int* gmin;
  float* g;  // (N, n_out) gradient seed of the loss w.r.t. the output
};

// general: hinge-loss seed, witness screen and per-screen minimum margin;
// simple: loss = min_d max_c margin, SAT at <= 1e-6, seed = the routed row.
__global__ void __launch_bounds__(256) pgd_screen_kernel(const ScreenArgs a) {
  __shared__ unsigned int blk_min;
  if (threadIdx.x == 0) blk_min = 0xFFFFFFFFu;
  __syncthreads();
  const int s = blockIdx.x * blockDim.x + threadIdx.x;
  if (s < a.N) {
    const float* ys = a.y + (long long)s * a.ldy;
    float* gs = a.g + (long long)s * a.ldg;
    auto margin = [&](int c) {
      float m = 0.f;
      for (int o = 0; o < a.n_out; ++o) m = fmaf(ys[o], a.C[c * a.n_out + o], m);
      return __fadd_rn(m, a.cb[c]);
    };
    if (a.simple) {
      float dmin = 0.f;
      int cbest = 0;
      for (int d = 0; d < a.D; ++d) {
        float dmax = 0.f;
        int carg = -1;
        for (int c = 0; c < a.ncon; ++c) {
          if (a.cdis[c] != d) continue;
          const float m = margin(c);
          if (carg < 0 || m > dmax) {
            dmax = m;
            carg = c;
          }
        }
        if (d == 0 || dmax < dmin) {
          dmin = dmax;
          cbest = carg;
        }
      }
      if (dmin <= 1e-6f)
        atomicMin(a.best, ((unsigned long long)a.t << 32) | (unsigned long long)s);
      for (int o = 0; o < a.n_out; ++o) gs[o] = a.C[cbest * a.n_out + o];
    } else {
      float amin = 0.f;
      bool have = false;
      for (int c = 0; c < a.ncon; ++c)
        if (a.cact[c] >= 0) {
          const float m = margin(c);
          amin = have ? fminf(amin, m) : m;
          have = true;
        }
      if (have) atomicMin(&blk_min, order_code(amin));
      if (have && amin <= 0.f) {
        bool conf = false;
        for (int d = 0; d < a.D && !conf; ++d) {
          bool any = false;
          float dmax = 0.f;
          for (int c = 0; c < a.ncon; ++c)
            if (a.cdis[c] == d) {
              const float m = margin(c);
              dmax = any ? fmaxf(dmax, m) : m;
              any = true;
            }
          conf = any && (double)dmax <= a.confirm_thr;
        }
        if (conf) atomicMin(a.best, ((unsigned long long)a.t << 32) | (unsigned long long)s);
      }
      const int target = a.prd ? (s % a.R) % a.n_act : -1;
      for (int o = 0; o < a.n_out; ++o) gs[o] = 0.f;
      for (int c = 0; c < a.ncon; ++c) {
        const int ac = a.cact[c];
        if (ac < 0 || (target >= 0 && ac != target)) continue;
        if (!(margin(c) >= a.hinge)) continue;
        for (int o = 0; o < a.n_out; ++o) gs[o] = __fadd_rn(gs[o], a.C[c * a.n_out + o]);
      }
    }
  }
  __syncthreads();
  if (!a.simple && threadIdx.x == 0 && blk_min != 0xFFFFFFFFu) atomicMin(a.gmin, blk_min);
}

struct StepArgs {
  int N, R, n_in, ldg, step_rows, mode, optim, t;  // mode 0 update, 1 OSI ascent, 2 simple
  float decay, lr, beta1, beta2, one_m_beta1, one_m_beta2, eps, sc1, sc2;
  float* x;
  const float *lo, *hi, *g, *step0;
  float *cur, *m1, *m2;
};

__global__ void __launch_bounds__(256) pgd_step_kernel(const StepArgs a) {
  const long long idx = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= (long long)a.N * a.n_in) return;
  const int s = (int)(idx / a.n_in), i = (int)(idx - (long long)s * a.n_in);
  const long long bi = (long long)(s / a.R) * a.n_in + i;
  const float lo = a.lo[bi], hi = a.hi[bi];
  const float gv = a.g[(long long)s * a.ldg + i];
  const float xv = a.x[idx];
  if (a.mode == 2) {  // _simple_pgd: x - lr * sign(g) * width
    const float step = __fmul_rn(__fmul_rn(a.lr, sgnf(gv)), __fsub_rn(hi, lo));
    a.x[idx] = fmaxf(fminf(__fsub_rn(xv, step), hi), lo);
    return;
  }
  const int row = a.step_rows == 1 ? 0 : s % a.R;
  if (a.mode == 1) {  // OSI: x + step0 * sign(g)
    const float st = a.step0[(long long)row * a.n_in + i];
    a.x[idx] = fminf(fmaxf(__fadd_rn(xv, __fmul_rn(st, sgnf(gv))), lo), hi);
    return;
  }
  const float step = a.cur[idx];
  float delta;
  if (a.optim == 0) {
    delta = __fmul_rn(step, sgnf(gv));
  } else {
    const float m = fmaf(gv, a.one_m_beta1, __fmul_rn(a.m1[idx], a.beta1));
    const float v = fmaf(__fmul_rn(gv, gv), a.one_m_beta2, __fmul_rn(a.m2[idx], a.beta2));
    a.m1[idx] = m;
    a.m2[idx] = v;
    const float denom = __fadd_rn(__fmul_rn(__fsqrt_rn(v), a.sc2), a.eps);
    const float dir = sgnf(__fdiv_rn(m, denom));
    delta = a.optim == 1 ? __fmul_rn(step, dir) : __fmul_rn(__fmul_rn(step, a.sc1), dir);
  }
  a.x[idx] = fminf(fmaxf(__fsub_rn(xv, delta), lo), hi);
  a.cur[idx] = __fmul_rn(step, a.decay);
}

// Shared-memory plan of the network and a sample tile; returns the next free
// offset (floats) or -1 when a width is out of range.
int plan_net(const vcb_mlp* net, int ncon, PgdNet& n, const char* who, int ps = kPS) {
  const int nfc = net->n_fc;
  n.n_fc = nfc;
  int off = 0, maxw = 1;
  long long woff = 0;
  int boff = 0;
  for (int l = 0; l <= nfc; ++l) {
    n.dims[l] = net->dims[l];
    if (net->dims[l] <= 0 || net->dims[l] > kPMaxW) {
      fail(VCB_ERR_UNSUPPORTED, "%s: width %d (max %d)", who, net->dims[l], kPMaxW);
      return -1;
    }
    maxw = std::max(maxw, net->dims[l]);
  }
  for (int l = 0; l < nfc; ++l) {
    n.w_goff[l] = woff;
    n.b_goff[l] = boff;
    woff += (long long)net->dims[l] * net->dims[l + 1];
    boff += net->dims[l + 1];
    n.pwt[l] = pad4(net->dims[l + 1]);
    n.wt_soff[l] = off;
    off += pad4((net->dims[l] + 1) * n.pwt[l]);
  }
  n.pa = maxw | 1;         // odd: scalar loads of 32 samples' rows hit 32 banks
  n.pz = pad4odd(maxw);    // 4 x odd: float4 loads of 8 samples' rows hit 32 banks
  n.act_soff = off;
  off += 2 * ps * n.pa;
  n.z_soff = off;
  off += pad4(nfc * ps * n.pz);
  n.g_soff = off;
  off += pad4(ps * n.pz);
  n.x_soff = off;
  off += pad4(ps * net->dims[0]);
  n.c_soff = off;
  off += pad4(ncon * net->dims[nfc] + ncon);
  n.W = net->W;
  n.b = net->b;
  return off;
}

constexpr int kSmemCap = 220 * 1024;

}  // namespace
}  // namespace vcb

extern "C" int vcb_mlp_pgd(const vcb_mlp* net, int32_t N, int32_t R, float* x,
                           const float* lo, const float* hi, int32_t ncon,
                           const float* C, const float* cb, const int32_t* cdis,
                           int32_t D, int32_t n_iter, float lr,
                           unsigned long long* best, void* stream) {
  using namespace vcb;
  if (!net) return fail(VCB_ERR_INVALID, "vcb_mlp_pgd: net is NULL");
  const int nfc = net->n_fc;
  if (nfc < 1 || nfc > VCB_MAX_FC)
    return fail(VCB_ERR_UNSUPPORTED, "vcb_mlp_pgd: n_fc=%d", nfc);
  if (N < 0 || R <= 0 || ncon <= 0 || D <= 0 || n_iter < 0)
    return fail(VCB_ERR_INVALID, "vcb_mlp_pgd: N=%d R=%d ncon=%d D=%d n_iter=%d", N, R,
                ncon, D, n_iter);
  if (N == 0) return VCB_OK;
  if (!x || !lo || !hi || !C || !cb || !cdis || !best || !net->W || !net->b)
    return fail(VCB_ERR_INVALID, "vcb_mlp_pgd: NULL pointer");
  PgdParams p{};
  // tiles of kPSBig samples when the network leaves room for them (10,000
  // restarts of a 50-wide network: one round of 139 tiles), else kPS
  int ps = kPSBig;
  int off = plan_net(net, ncon, p.net, "vcb_mlp_pgd", ps);
  if (off < 0) return VCB_ERR_UNSUPPORTED;
  if (off * 4 > kSmemCap) {
    ps = kPS;
    off = plan_net(net, ncon, p.net, "vcb_mlp_pgd", ps);
  }
  const int bytes = off * 4;
  if (bytes > kSmemCap)
    return fail(VCB_ERR_UNSUPPORTED, "vcb_mlp_pgd: network needs %d bytes of shared memory", bytes);
  p.N = N;
  p.R = R;
  p.n_iter = n_iter;
  p.ncon = ncon;
  p.D = D;
  p.lr = lr;
  p.x = x;
  p.lo = lo;
  p.hi = hi;
  p.C = C;
  p.cb = cb;
  p.cdis = cdis;
  p.best = best;
  auto kern = ps == kPSBig ? pgd_mlp_kernel<kPSBig> : pgd_mlp_kernel<kPS>;
  int rc = ensure_smem(reinterpret_cast<const void*>(kern), bytes);
  if (rc) return rc;
  const int ntiles = (N + ps - 1) / ps;
  const int grid = std::max(1, std::min(ntiles, sm_count()));
  // whole rounds of the grid; each tile N / p.ntiles <= ps samples (and at
  // least one: p.ntiles < 2 ntiles <= N + 1)
  p.ntiles = grid * ((ntiles + grid - 1) / grid);
  kern<<<grid, kPT, bytes, static_cast<cudaStream_t>(stream)>>>(p);
  return check_launch("vcb_mlp_pgd: launch");
}

extern "C" int vcb_mlp_pgd_general(
    const vcb_mlp* net, int32_t N, int32_t R, float* x, const float* lo, const float* hi,
    const float* step0, int32_t step_rows, const float* w_d, int32_t n_osi, int32_t n_iter,
    int32_t optim, float lr_decay, double hinge, int32_t plateau, const float* inv_bc1, const float* inv_sbc2,
    int32_t ncon, const float* C, const float* cb, const int32_t* cdis, const int32_t* cact,
    int32_t D, int32_t n_act, int32_t per_restart_disj, double confirm_thr,
    unsigned long long budget_ns, unsigned long long* best, uint32_t* gmin, int32_t* t_stop,
    void* stream) {
  using namespace vcb;
  if (!net) return fail(VCB_ERR_INVALID, "vcb_mlp_pgd_general: net is NULL");
  const int nfc = net->n_fc;
  if (nfc < 1 || nfc > VCB_MAX_FC)
    return fail(VCB_ERR_UNSUPPORTED, "vcb_mlp_pgd_general: n_fc=%d", nfc);
  if (N < 0 || R <= 0 || ncon <= 0 || D <= 0 || n_act <= 0 || n_iter < 0 || n_osi < 0 ||
      optim < 0 || optim > 2 || (step_rows != 1 && step_rows != R))
    return fail(VCB_ERR_INVALID,
                "vcb_mlp_pgd_general: N=%d R=%d ncon=%d D=%d n_act=%d n_iter=%d n_osi=%d "
                "optim=%d step_rows=%d",
                N, R, ncon, D, n_act, n_iter, n_osi, optim, step_rows);
  if (N == 0) return VCB_OK;
  if (!x || !lo || !hi || !step0 || !C || !cb || !cdis || !cact || !best || !gmin || !t_stop ||
      !net->W || !net->b || (n_osi > 0 && !w_d) || (n_iter > 0 && (!inv_bc1 || !inv_sbc2)))
    return fail(VCB_ERR_INVALID, "vcb_mlp_pgd_general: NULL pointer");
  PgdGenParams p{};
  int off = plan_net(net, ncon, p.net, "vcb_mlp_pgd_general");
  if (off < 0) return VCB_ERR_UNSUPPORTED;
  const int n0 = net->dims[0];
  p.m1_soff = off;
  off += pad4(kPS * n0);
  p.m2_soff = off;
  off += pad4(kPS * n0);
  p.cur_soff = off;
  off += pad4(kPS * n0);
  p.mg_soff = off;
  off += pad4(kPS * ncon);
  const int bytes = off * 4;
  if (bytes > kSmemCap)
    return fail(VCB_ERR_UNSUPPORTED,
                "vcb_mlp_pgd_general: network needs %d bytes of shared memory", bytes);
  p.N = N;
  p.R = R;
  p.n_osi = n_osi;
  p.n_iter = n_iter;
  p.ncon = ncon;
  p.D = D;
  p.n_act = n_act;
  p.prd = per_restart_disj ? 1 : 0;
  p.optim = optim;
  p.step_rows = step_rows;
  p.hinge = static_cast<float>(hinge);
  p.hinge_d = hinge;
  p.plateau = plateau;
  p.decay = lr_decay;
  // the optimiser's Python-float constants, each rounded once to float32
  p.beta1 = static_cast<float>(0.9);
  p.beta2 = static_cast<float>(0.999);
  p.one_m_beta1 = static_cast<float>(1.0 - 0.9);
  p.one_m_beta2 = static_cast<float>(1.0 - 0.999);
  p.eps = 1e-8f;
  p.confirm_thr = confirm_thr;
  p.budget_ns = budget_ns;
  p.x = x;
  p.lo = lo;
  p.hi = hi;
  p.step0 = step0;
  p.w_d = w_d;
  p.inv_bc1 = inv_bc1;
  p.inv_sbc2 = inv_sbc2;
  p.C = C;
  p.cb = cb;
  p.cdis = cdis;
  p.cact = cact;
  p.best = best;
  p.gmin = gmin;
  p.t_stop = t_stop;
  int rc = ensure_smem(reinterpret_cast<const void*>(pgd_general_kernel), bytes);
  if (rc) return rc;
  const int ntiles = (N + kPS - 1) / kPS;
  const int grid = std::max(1, std::min(ntiles, sm_count()));
  pgd_general_kernel<<<grid, kPT, bytes, static_cast<cudaStream_t>(stream)>>>(p);
  return check_launch("vcb_mlp_pgd_general: launch");
}

extern "C" int vcb_pgd_screen(int32_t N, int32_t n_out, const float* y, int32_t ldy,
                              int32_t ncon, const float* C, const float* cb,
                              const int32_t* cdis, const int32_t* cact, int32_t D,
                              int32_t n_act, int32_t per_restart_disj, int32_t R,
                              int32_t simple, float hinge, double confirm_thr, int32_t t,
                              unsigned long long* best, uint32_t* gmin_t, float* g,
                              int32_t ldg, void* stream) {
  using namespace vcb;
  if (N < 0 || n_out <= 0 || ldy < n_out || ldg < n_out || ncon <= 0 || D <= 0 || R <= 0 ||
      t < 0 || (!simple && n_act <= 0))
    return fail(VCB_ERR_INVALID, "vcb_pgd_screen: N=%d n_out=%d ncon=%d D=%d", N, n_out, ncon,
                D);
  if (N == 0) return VCB_OK;
  if (!y || !C || !cb || !cdis || !best || !g || (!simple && (!cact || !gmin_t)))
    return fail(VCB_ERR_INVALID, "vcb_pgd_screen: NULL pointer");
  ScreenArgs a{N, n_out, ldy, ldg, ncon, D, n_act, per_restart_disj ? 1 : 0, R, t,
               simple ? 1 : 0, hinge, confirm_thr, y, C, cb, cdis, cact, best, gmin_t, g};
  pgd_screen_kernel<<<(N + 255) / 256, 256, 0, static_cast<cudaStream_t>(stream)>>>(a);
  return check_launch("vcb_pgd_screen");
}

extern "C" int vcb_pgd_step(int32_t N, int32_t R, int32_t n_in, float* x, const float* lo,
                            const float* hi, const float* g, int32_t ldg, int32_t mode,
                            int32_t optim, int32_t t, const float* step0, int32_t step_rows,
                            float* cur, float* m1, float* m2, float sc1, float sc2,
                            float decay, float lr, void* stream) {
  using namespace vcb;
  if (N < 0 || R <= 0 || n_in <= 0 || ldg < n_in || mode < 0 || mode > 2 || optim < 0 ||
      optim > 2 || (mode != 2 && step_rows != 1 && step_rows != R))
    return fail(VCB_ERR_INVALID, "vcb_pgd_step: N=%d R=%d n_in=%d mode=%d", N, R, n_in, mode);
  if (N == 0) return VCB_OK;
  if (!x || !lo || !hi || !g || (mode == 1 && !step0) ||
      (mode == 0 && (!cur || (optim > 0 && (!m1 || !m2)))))
    return fail(VCB_ERR_INVALID, "vcb_pgd_step: NULL pointer");
  StepArgs a{N, R, n_in, ldg, step_rows, mode, optim, t, decay, lr,
             static_cast<float>(0.9), static_cast<float>(0.999),
             static_cast<float>(1.0 - 0.9), static_cast<float>(1.0 - 0.999), 1e-8f, sc1, sc2,
             x, lo, hi, g, step0, cur, m1, m2};
  const long long n = (long long)N * n_in;
  pgd_step_kernel<<<(unsigned)((n + 255) / 256), 256, 0, static_cast<cudaStream_t>(stream)>>>(a);
  return check_launch("vcb_pgd_step");
}
