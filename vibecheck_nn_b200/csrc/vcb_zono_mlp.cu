// Batched DeepZ zonotope forward for ReLU MLPs whose weights fit in shared
// memory (verify_zono_bnb.py:3079-4074: fc :3140-3173, relu :3175-3211).
//
// One persistent CTA per SM walks the boxes.  Per box the zonotope lives in
// shared memory as a generator-major matrix: row 0 is the centre c, rows
// 1..K the generators (one column per neuron), double-buffered across
// layers.  Per fc layer a register-tiled fp32 GEMM maps every row through the
// resident weights (the centre row also gets the bias); per ReLU the kernel
//   * sums |G| over the generator rows per neuron (fixed-order partial sums),
//   * forms lo/hi, the DeepZ lambda/mu, scales the generators by lambda and
//     appends one generator per unstable neuron (ascending neuron order, the
//     reference's cumsum rank), and
//   * writes the pre-activation bounds sb (and ORs the neuron into the
//     batch-wide "unstable anywhere" mask the CROWN-intermediate pass seeds).
// Generators are kept per box: columns that are zero in this box (an input
// dimension of zero radius, another box's unstable neuron) are never stored.
// They contribute nothing to any bound, so the bounds equal the reference's
// padded layout's.
#include <algorithm>

#include "vcb_common.cuh"

namespace vcb {
namespace {

constexpr int kZT = 512;  // threads per CTA

struct ZonoParams {
  int n_fc;
  int dims[VCB_MAX_FC + 1];
  const float* W;
  const float* b;
  long long w_goff[VCB_MAX_FC];
  int b_goff[VCB_MAX_FC];
  int w_soff[VCB_MAX_FC];
  int pw[VCB_MAX_FC];
  int wrows[VCB_MAX_FC];
  long long relu_goff[VCB_MAX_FC];
  int unst_off[VCB_MAX_FC];  // offset of relu layer L in the union mask
  int kmax;                  // generator rows capacity (excluding centre)
  int pg;                    // row stride of the generator buffers
  int buf_soff[2];
  int red_soff, nred;        // partial |G| sums: nred x pg
  int col_soff;              // per-neuron lambda, mu, flags
  int B, full;               // full: run the last fc layer and emit c/G
  const float *xl, *xh;
  float *sblo, *sbhi;
  int* unstable_any;
  float* c_out;              // (B, n_out) when full
  float* g_out;              // (B, n_out, kmax) when full (compact, zero padded)
  int* k_out;                // (B,) generator count when full
};

__device__ __forceinline__ float4 ld4(const float* p) {
  return *reinterpret_cast<const float4*>(p);
}

__global__ void __launch_bounds__(kZT, 1)
    zono_mlp_kernel(const __grid_constant__ ZonoParams p) {
  extern __shared__ __align__(16) float sm[];
  const int tid = threadIdx.x;
  const int nfc = p.n_fc;
  const int n0 = p.dims[0];
  const int pg = p.pg;

  for (int l = 0; l < nfc; ++l) {
    const int nin = p.dims[l], nout = p.dims[l + 1], pw = p.pw[l];
    float* dst = sm + p.w_soff[l];
    const float* Wg = p.W + p.w_goff[l];
    const float* bg = p.b + p.b_goff[l];
    for (int o = tid >> 5; o < p.wrows[l]; o += kZT / 32) {
      for (int i = tid & 31; i < pw; i += 32) {
        const bool inside = o < nout && i <= nin;
        const float* src = !inside ? p.W : (i < nin ? Wg + (long long)o * nin + i : bg + o);
        const unsigned saddr = static_cast<unsigned>(__cvta_generic_to_shared(dst + o * pw + i));
        asm volatile("cp.async.ca.shared.global [%0], [%1], 4, %2;\n" ::"r"(saddr),
                     "l"(src), "r"(inside ? 4 : 0));
      }
    }
  }
  asm volatile("cp.async.commit_group;\ncp.async.wait_group 0;\n" ::: "memory");
  __syncthreads();

  float* lam_s = sm + p.col_soff;          // per neuron: lambda
  float* mu_s = lam_s + pg;                // per neuron: mu
  int* rank_s = reinterpret_cast<int*>(mu_s + pg);  // new-generator row or -1
  int* nk_s = rank_s + pg;                 // [0]: generator count
  float* red = sm + p.red_soff;

  for (int box = blockIdx.x; box < p.B; box += gridDim.x) {
    float* cur = sm + p.buf_soff[0];
    float* nxt = sm + p.buf_soff[1];
    // ---- input zonotope: centre row + one generator per nonzero radius
    if (tid == 0) {
      int k = 0;
      for (int i = 0; i < n0; ++i) {
        const float lo = p.xl[(long long)box * n0 + i], hi = p.xh[(long long)box * n0 + i];
        if (__fmul_rn(__fsub_rn(hi, lo), 0.5f) != 0.f) ++k;
      }
      nk_s[0] = k;
    }
    for (int idx = tid; idx < pg; idx += kZT) {
      float c = 0.f;
      if (idx < n0) {
        const float lo = p.xl[(long long)box * n0 + idx], hi = p.xh[(long long)box * n0 + idx];
        c = __fmul_rn(__fadd_rn(lo, hi), 0.5f);
      }
      cur[idx] = c;
    }
    __syncthreads();
    int K = nk_s[0];
    for (int idx = tid; idx < K * pg; idx += kZT) cur[pg + idx] = 0.f;
    __syncthreads();
    if (tid == 0) {
      int k = 0;
      for (int i = 0; i < n0; ++i) {
        const float lo = p.xl[(long long)box * n0 + i], hi = p.xh[(long long)box * n0 + i];
        const float r = __fmul_rn(__fsub_rn(hi, lo), 0.5f);
        if (r != 0.f) {
          cur[(1 + k) * pg + i] = r;
          ++k;
        }
      }
    }
    __syncthreads();

    const int last = p.full ? nfc : nfc - 1;
    for (int l = 0; l < last; ++l) {
      const int nin = p.dims[l], nout = p.dims[l + 1], pw = p.pw[l];
      const float* sW = sm + p.w_soff[l];
      // ---- fc: nxt[row][o] = sum_i cur[row][i] W[o][i] (+ b[o] on row 0)
      const int rows = K + 1;
      const int RG = (rows + 3) >> 2;
      const int CG = (nout + 3) >> 2;
      const int kend = pad4(nin);
      for (int it = tid; it < RG * CG; it += kZT) {
        const int cg = it / RG, rg = it - cg * RG;
        float acc[4][4];
#pragma unroll
        for (int j = 0; j < 4; ++j)
#pragma unroll
          for (int c = 0; c < 4; ++c) acc[j][c] = 0.f;
        const float* a0 = cur + rg * pg;  // rows rg + RG*j (conflict-free)
        for (int k = 0; k < kend; k += 4) {
          float4 a[4], w[4];
#pragma unroll
          for (int j = 0; j < 4; ++j) a[j] = ld4(a0 + j * RG * pg + k);
#pragma unroll
          for (int c = 0; c < 4; ++c) w[c] = ld4(sW + (4 * cg + c) * pw + k);
#pragma unroll
          for (int j = 0; j < 4; ++j)
#pragma unroll
            for (int c = 0; c < 4; ++c) {
              acc[j][c] = fmaf(a[j].x, w[c].x, acc[j][c]);
              acc[j][c] = fmaf(a[j].y, w[c].y, acc[j][c]);
              acc[j][c] = fmaf(a[j].z, w[c].z, acc[j][c]);
              acc[j][c] = fmaf(a[j].w, w[c].w, acc[j][c]);
            }
        }
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const int row = rg + RG * j;
          if (row >= rows) continue;
#pragma unroll
          for (int c = 0; c < 4; ++c) {
            const int o = 4 * cg + c;
            float v = acc[j][c];
            if (row == 0 && o < nout) v = __fadd_rn(v, sW[o * pw + nin]);
            nxt[row * pg + o] = (o < nout) ? v : 0.f;
          }
        }
      }
      __syncthreads();
      { float* t = cur; cur = nxt; nxt = t; }
      if (l == nfc - 1) break;  // final fc: no relu
      // ---- relu: |G| row sums per neuron in fixed-order slices
      const int nred = p.nred;
      for (int it = tid; it < nred * nout; it += kZT) {
        const int sidx = it / nout, o = it - sidx * nout;
        float s = 0.f;
        for (int k = 1 + sidx; k <= K; k += nred) s = __fadd_rn(s, fabsf(cur[k * pg + o]));
        red[sidx * pg + o] = s;
      }
      __syncthreads();
      const long long goff = p.relu_goff[l] + (long long)box * nout;
      if (tid < 32) {
        // warp 0: bounds, lambda/mu and the ascending rank of unstable neurons
        int base = 0;
        for (int o0 = 0; o0 < nout; o0 += 32) {
          const int o = o0 + tid;
          bool ust = false;
          if (o < nout) {
            float s = 0.f;
            for (int sidx = 0; sidx < nred; ++sidx) s = __fadd_rn(s, red[sidx * pg + o]);
            const float c = cur[o];
            const float lo = __fsub_rn(c, s), hi = __fadd_rn(c, s);
            ust = (lo < 0.f) && (hi > 0.f);
            const bool dead = hi <= 0.f;
            float lam, mu;
            if (ust) {
              const float d = __fsub_rn(hi, lo);
              lam = __fdiv_rn(hi, d);
              mu = __fdiv_rn(__fmul_rn(-hi, lo), __fmul_rn(2.f, d));
            } else {
              lam = dead ? 0.f : 1.f;
              mu = 0.f;
            }
            lam_s[o] = lam;
            mu_s[o] = mu;
            if (p.sblo) {
              p.sblo[goff + o] = lo;
              p.sbhi[goff + o] = hi;
            }
            if (ust && p.unstable_any) {
              int* f = p.unstable_any + p.unst_off[l] + o;
              if (*reinterpret_cast<volatile int*>(f) == 0) atomicOr(f, 1);
            }
          }
          const unsigned m = __ballot_sync(0xffffffffu, ust);
          if (o < nout) rank_s[o] = ust ? K + base + __popc(m & ((1u << tid) - 1u)) : -1;
          base += __popc(m);
        }
        if (tid == 0) nk_s[0] = K + base;
      }
      __syncthreads();
      const int Knew = nk_s[0];
      // centre and scaled generators into nxt, then the new generators
      for (int idx = tid; idx < (K + 1) * pg; idx += kZT) {
        const int row = idx / pg, o = idx - row * pg;
        float v = cur[idx];
        if (o < nout) v = (row == 0) ? __fadd_rn(__fmul_rn(lam_s[o], v), mu_s[o])
                                     : __fmul_rn(v, lam_s[o]);
        nxt[idx] = v;
      }
      for (int idx = tid; idx < (Knew - K) * pg; idx += kZT) nxt[(K + 1) * pg + idx] = 0.f;
      __syncthreads();
      for (int o = tid; o < nout; o += kZT)
        if (rank_s[o] >= 0) nxt[(rank_s[o] + 1) * pg + o] = mu_s[o];
      __syncthreads();
      { float* t = cur; cur = nxt; nxt = t; }
      K = Knew;
    }
    if (p.full) {
      const int nout = p.dims[nfc];
      for (int o = tid; o < nout; o += kZT) p.c_out[(long long)box * nout + o] = cur[o];
      for (int idx = tid; idx < nout * p.kmax; idx += kZT) {
        const int o = idx / p.kmax, k = idx - o * p.kmax;
        p.g_out[(long long)box * nout * p.kmax + idx] = (k < K) ? cur[(k + 1) * pg + o] : 0.f;
      }
      if (tid == 0) p.k_out[box] = K;
    }
    __syncthreads();
  }
}

}  // namespace
}  // namespace vcb

extern "C" int vcb_mlp_zono(const vcb_mlp* net, int32_t B, const float* xl,
                            const float* xh, float* sb_lo, float* sb_hi,
                            int32_t* unstable_any, float* c_out, float* g_out,
                            int32_t* k_out, void* stream) {
  using namespace vcb;
  if (!net) return fail(VCB_ERR_INVALID, "vcb_mlp_zono: net is NULL");
  const int nfc = net->n_fc;
  if (nfc < 1 || nfc > VCB_MAX_FC)
    return fail(VCB_ERR_UNSUPPORTED, "vcb_mlp_zono: n_fc=%d outside [1,%d]", nfc, VCB_MAX_FC);
  if (B < 0) return fail(VCB_ERR_INVALID, "vcb_mlp_zono: B=%d", B);
  if (B == 0) return VCB_OK;
  if (!net->W || !net->b || !xl || !xh)
    return fail(VCB_ERR_INVALID, "vcb_mlp_zono: NULL weight or box pointer");
  if ((sb_lo == nullptr) != (sb_hi == nullptr))
    return fail(VCB_ERR_INVALID, "vcb_mlp_zono: sb_lo/sb_hi must be given together");
  const bool full = c_out != nullptr;
  if (full && (!g_out || !k_out))
    return fail(VCB_ERR_INVALID, "vcb_mlp_zono: c_out needs g_out and k_out");
  ZonoParams p{};
  p.n_fc = nfc;
  int off = 0, maxn = 1;
  long long woff = 0, roff = 0;
  int boff = 0, uoff = 0, kmax = net->dims[0];
  for (int l = 0; l <= nfc; ++l) {
    if (net->dims[l] <= 0) return fail(VCB_ERR_INVALID, "vcb_mlp_zono: dims[%d]=%d", l, net->dims[l]);
    p.dims[l] = net->dims[l];
    maxn = std::max(maxn, net->dims[l]);
  }
  for (int l = 0; l < nfc; ++l) {
    const int nin = net->dims[l], nout = net->dims[l + 1];
    p.w_goff[l] = woff;
    p.b_goff[l] = boff;
    woff += (long long)nin * nout;
    boff += nout;
    p.pw[l] = pad4odd(nin + 1);
    p.wrows[l] = pad4(nout);
    p.w_soff[l] = off;
    off += p.wrows[l] * p.pw[l];
    if (l < nfc - 1) {
      p.relu_goff[l] = roff;
      roff += (long long)B * nout;
      p.unst_off[l] = uoff;
      uoff += nout;
      kmax += nout;
    }
  }
  if (maxn > 1024) return fail(VCB_ERR_UNSUPPORTED, "vcb_mlp_zono: width %d > 1024", maxn);
  off = pad4(off + 8);
  p.kmax = kmax;
  p.pg = pad4odd(maxn);
  const int rows = pad4(kmax + 1) + 4;
  p.buf_soff[0] = off;
  off += rows * p.pg;
  p.buf_soff[1] = off;
  off += rows * p.pg;
  p.nred = 8;
  p.red_soff = off;
  off += p.nred * p.pg;
  p.col_soff = off;
  off += 4 * p.pg + 4;
  const int bytes = off * 4;
  if (bytes > 232448)
    return fail(VCB_ERR_UNSUPPORTED,
                "vcb_mlp_zono: zonotope of %d generators x %d neurons does not fit shared memory",
                kmax, maxn);
  p.W = net->W;
  p.b = net->b;
  p.B = B;
  p.full = full ? 1 : 0;
  p.xl = xl;
  p.xh = xh;
  p.sblo = sb_lo;
  p.sbhi = sb_hi;
  p.unstable_any = unstable_any;
  p.c_out = c_out;
  p.g_out = g_out;
  p.k_out = k_out;
  int rc = ensure_smem(reinterpret_cast<const void*>(zono_mlp_kernel), bytes);
  if (rc) return rc;
  const int grid = std::max(1, std::min(B, sm_count()));
  zono_mlp_kernel<<<grid, kZT, bytes, static_cast<cudaStream_t>(stream)>>>(p);
  return check_launch("vcb_mlp_zono: launch");
}

extern "C" int vcb_mlp_zono_kmax(const vcb_mlp* net) {
  if (!net || net->n_fc < 1 || net->n_fc > VCB_MAX_FC) return -1;
  int k = net->dims[0];
  for (int l = 1; l < net->n_fc; ++l) k += net->dims[l];
  return k;
}
