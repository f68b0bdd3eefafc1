// Batched sign-gradient PGD for ReLU MLPs (verify_hybrid_acasxu.py:39-161).
//
// Each sample x (a restart inside its box [lo, hi]) runs n_iter steps of
//   y = f(x);  m_d = max_c (C_c . y + cb_c) over the constraints of disjunct d
//   loss = min_d m_d;  SAT when loss <= 1e-6;
//   x <- clamp(x - lr * sign(dloss/dx) * (hi - lo), lo, hi).
// The gradient follows torch autograd on the reference's expression: F.relu
// passes it where the pre-activation is > 0, max/min route it to the first
// extremal index.  A sample that becomes SAT stops moving; the reported
// witness is the SAT sample with the smallest (iteration, index) -- the
// sample the reference's loop, which checks every sample once per iteration
// and returns the first SAT one, would return.
//
// One CTA per tile of kPS samples with the fc weights resident in shared
// memory; the tile's pre-activations (kept for the ReLU masks), activations
// and gradients stay in shared memory for all iterations.
#include <algorithm>

#include "vcb_common.cuh"

namespace vcb {
namespace {

constexpr int kPT = 256;   // threads per CTA
constexpr int kPS = 64;    // samples per tile
constexpr int kPMaxW = 128;

struct PgdParams {
  int n_fc;
  int dims[VCB_MAX_FC + 1];
  const float* W;
  const float* b;
  long long w_goff[VCB_MAX_FC];
  int b_goff[VCB_MAX_FC];
  int w_soff[VCB_MAX_FC];
  int pw[VCB_MAX_FC];
  int wrows[VCB_MAX_FC];
  int pa;                 // activation row stride (multiple of 4)
  int pz;                 // pre-activation / gradient row stride (odd)
  int act_soff;           // 2 ping-pong activation buffers, kPS x pa
  int z_soff;             // n_fc pre-activation buffers, kPS x pz
  int g_soff, x_soff, c_soff;
  int N, R, n_iter, ncon, D;
  float lr;
  float* x;               // (N, n_in) in/out
  const float *lo, *hi;   // (N / R, n_in) box of each group of R samples
  const float *C, *cb;    // (ncon, n_out), (ncon,)
  const int* cdis;        // disjunct of each constraint (0..D-1)
  unsigned long long* best;  // min over SAT samples of (iter << 32 | index)
};

__global__ void __launch_bounds__(kPT, 1) pgd_mlp_kernel(const __grid_constant__ PgdParams p) {
  extern __shared__ __align__(16) float sm[];
  __shared__ int done[kPS];
  __shared__ int cstar[kPS];
  __shared__ int stop;
  const int tid = threadIdx.x;
  const int nfc = p.n_fc;
  const int n0 = p.dims[0];
  const int nL = p.dims[nfc];
  for (int l = 0; l < nfc; ++l) {
    const int nin = p.dims[l], nout = p.dims[l + 1], pw = p.pw[l];
    float* dst = sm + p.w_soff[l];
    const float* Wg = p.W + p.w_goff[l];
    const float* bg = p.b + p.b_goff[l];
    for (int o = tid >> 5; o < p.wrows[l]; o += kPT / 32)
      for (int i = tid & 31; i < pw; i += 32) {
        float v = 0.f;
        if (o < nout) v = (i < nin) ? Wg[(long long)o * nin + i] : (i == nin ? bg[o] : 0.f);
        dst[o * pw + i] = v;
      }
  }
  float* Cs = sm + p.c_soff;
  for (int idx = tid; idx < p.ncon * nL; idx += kPT) Cs[idx] = p.C[idx];
  for (int idx = tid; idx < p.ncon; idx += kPT) Cs[p.ncon * nL + idx] = p.cb[idx];
  __syncthreads();
  const int pa = p.pa, pz = p.pz;
  float* xs = sm + p.x_soff;  // kPS x n0 current samples
  float* g = sm + p.g_soff;   // kPS x pz gradient rows
  const int ntiles = (p.N + kPS - 1) / kPS;
  for (int tile = blockIdx.x; tile < ntiles; tile += gridDim.x) {
    const int s0 = tile * kPS;
    const int ns = min(kPS, p.N - s0);
    for (int idx = tid; idx < kPS * n0; idx += kPT) {
      const int s = idx / n0, i = idx - s * n0;
      xs[idx] = s < ns ? p.x[(long long)(s0 + s) * n0 + i] : 0.f;
    }
    for (int s = tid; s < kPS; s += kPT) done[s] = s < ns ? 0 : 1;
    __syncthreads();
    for (int it = 0; it < p.n_iter; ++it) {
      // once a SAT sample exists at an earlier iteration nothing here can win
      if (tid == 0) {
        const unsigned long long bk = *reinterpret_cast<volatile unsigned long long*>(p.best);
        stop = (bk >> 32) < (unsigned long long)it;
      }
      __syncthreads();
      if (stop) break;
      // ---- forward: z_l stored for the masks, a_{l+1} = relu(z_l)
      float* a_cur = sm + p.act_soff;
      const int n0p = pad4(n0);
      for (int idx = tid; idx < kPS * n0p; idx += kPT) {
        const int s = idx / n0p, i = idx - s * n0p;
        a_cur[s * pa + i] = i < n0 ? xs[s * n0 + i] : 0.f;
      }
      __syncthreads();
      for (int l = 0; l < nfc; ++l) {
        const int nin = p.dims[l], nout = p.dims[l + 1], pw = p.pw[l];
        const float* sW = sm + p.w_soff[l];
        const float* ain = sm + p.act_soff + (l & 1) * kPS * pa;
        float* aout = sm + p.act_soff + ((l + 1) & 1) * kPS * pa;
        float* z = sm + p.z_soff + l * kPS * pz;
        const int kend = pad4(nin);
        const int noutp = pad4(nout);
        for (int idx = tid; idx < kPS * noutp; idx += kPT) {
          const int o = idx / kPS, s = idx - o * kPS;
          if (o >= nout) {
            aout[s * pa + o] = 0.f;
            continue;
          }
          float acc = 0.f;
          const float* ar = ain + s * pa;
          const float* wr = sW + o * pw;
          for (int k = 0; k < kend; k += 4) {
            const float4 av = *reinterpret_cast<const float4*>(ar + k);
            const float4 wv = *reinterpret_cast<const float4*>(wr + k);
            acc = fmaf(av.x, wv.x, acc);
            acc = fmaf(av.y, wv.y, acc);
            acc = fmaf(av.z, wv.z, acc);
            acc = fmaf(av.w, wv.w, acc);
          }
          const float zz = __fadd_rn(acc, wr[nin]);
          z[s * pz + o] = zz;
          aout[s * pa + o] = fmaxf(zz, 0.f);
        }
        __syncthreads();
      }
      // ---- margins, SAT check and the output gradient row
      const float* y = sm + p.z_soff + (nfc - 1) * kPS * pz;
      for (int s = tid; s < kPS; s += kPT) {
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
      for (int idx = tid; idx < kPS * pz; idx += kPT) {
        const int s = idx / pz, o = idx - s * pz;
        g[idx] = (o < nL && !done[s]) ? Cs[cstar[s] * nL + o] : 0.f;
      }
      __syncthreads();
      for (int l = nfc - 1; l >= 0; --l) {
        const int nin = p.dims[l], nout = p.dims[l + 1], pw = p.pw[l];
        const float* sW = sm + p.w_soff[l];
        const float* zprev = (l > 0) ? sm + p.z_soff + (l - 1) * kPS * pz : nullptr;
        constexpr int kStep = kPT / kPS;
        float vals[(kPMaxW + kStep - 1) / kStep];
        const int sl = tid % kPS, i0 = tid / kPS;
        int cnt = 0;
        for (int i = i0; i < nin; i += kStep) {
          float acc = 0.f;
          for (int o = 0; o < nout; ++o) acc = fmaf(g[sl * pz + o], sW[o * pw + i], acc);
          if (zprev && !(zprev[sl * pz + i] > 0.f)) acc = 0.f;
          vals[cnt++] = acc;
        }
        __syncthreads();  // every thread has read g
        cnt = 0;
        for (int i = i0; i < pz; i += kStep) g[sl * pz + i] = (i < nin) ? vals[cnt++] : 0.f;
        __syncthreads();
      }
      // ---- sign step and clamp (SAT samples keep the x that was SAT)
      for (int idx = tid; idx < ns * n0; idx += kPT) {
        const int s = idx / n0, i = idx - s * n0;
        if (done[s]) continue;
        const long long bi = (long long)((s0 + s) / p.R) * n0 + i;
        const float lo = p.lo[bi], hi = p.hi[bi];
        const float gv = g[s * pz + i];
        const float sg = gv > 0.f ? 1.f : (gv < 0.f ? -1.f : 0.f);
        const float step = __fmul_rn(__fmul_rn(p.lr, sg), __fsub_rn(hi, lo));
        const float xn = __fsub_rn(xs[s * n0 + i], step);
        xs[s * n0 + i] = fmaxf(fminf(xn, hi), lo);
      }
      __syncthreads();
    }
    for (int idx = tid; idx < ns * n0; idx += kPT) p.x[(long long)s0 * n0 + idx] = xs[idx];
    __syncthreads();
  }
}

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
  p.n_fc = nfc;
  int off = 0, maxw = 1;
  long long woff = 0;
  int boff = 0;
  for (int l = 0; l <= nfc; ++l) {
    p.dims[l] = net->dims[l];
    if (net->dims[l] <= 0 || net->dims[l] > kPMaxW)
      return fail(VCB_ERR_UNSUPPORTED, "vcb_mlp_pgd: width %d (max %d)", net->dims[l], kPMaxW);
    maxw = std::max(maxw, net->dims[l]);
  }
  for (int l = 0; l < nfc; ++l) {
    p.w_goff[l] = woff;
    p.b_goff[l] = boff;
    woff += (long long)net->dims[l] * net->dims[l + 1];
    boff += net->dims[l + 1];
    p.pw[l] = pad4odd(net->dims[l] + 1);
    p.wrows[l] = pad4(net->dims[l + 1]);
    p.w_soff[l] = off;
    off += p.wrows[l] * p.pw[l];
  }
  off = pad4(off + 8);
  p.pa = pad4odd(maxw);
  p.pz = pad4(maxw) + 1;
  p.act_soff = off;
  off += 2 * kPS * p.pa;
  p.z_soff = off;
  off += pad4(nfc * kPS * p.pz);
  p.g_soff = off;
  off += pad4(kPS * p.pz);
  p.x_soff = off;
  off += pad4(kPS * net->dims[0]);
  p.c_soff = off;
  off += pad4(ncon * net->dims[nfc] + ncon);
  const int bytes = off * 4;
  if (bytes > 220 * 1024)
    return fail(VCB_ERR_UNSUPPORTED, "vcb_mlp_pgd: network needs %d bytes of shared memory", bytes);
  p.W = net->W;
  p.b = net->b;
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
  int rc = ensure_smem(reinterpret_cast<const void*>(pgd_mlp_kernel), bytes);
  if (rc) return rc;
  const int ntiles = (N + kPS - 1) / kPS;
  const int grid = std::max(1, std::min(ntiles, sm_count()));
  pgd_mlp_kernel<<<grid, kPT, bytes, static_cast<cudaStream_t>(stream)>>>(p);
  return check_launch("vcb_mlp_pgd: launch");
}
