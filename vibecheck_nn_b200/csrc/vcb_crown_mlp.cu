// Fused IBP forward + CROWN back-substitution for ReLU MLPs whose weights fit
// in shared memory (ACAS-Xu-sized networks).
//
// One persistent CTA per SM slot (two per SM) walks tiles of TB subdomains.
// All fc weights stay in shared memory (bias stored as an extra weight
// column).  Per tile:
//   * IBP forward (verify_zono_bnb.py:1066-1153): per fc layer a register-
//     tiled fp32 GEMM of the (TB x n_in) mid/rad tile against the weights
//     (ping-pong buffers, one barrier per layer); the ReLU clamp / crossing
//     repair and the CROWN slope rule (verify_zono_bnb.py:503-522) run in its
//     epilogue.  Slopes go to the CTA's slot of the caller's workspace
//     (sign-encoded float2 per neuron, rewritten every tile, so the workspace
//     stays resident in L2).
//   * CROWN back-substitution (verify_zono_bnb.py:4270-5134): the (TB*Q x n)
//     coefficient tile walks the layers in reverse, one GEMM per fc layer
//     whose epilogue applies the ReLU relaxation and sums the intercepts; the
//     bias dot is the GEMM's extra column.  The first step (spec rows times
//     the last layer) is identical for every box and is computed once per CTA.
//   * Concretisation against the input box; optional A / acc outputs.
// Thread tiles are laid out so a warp's weight loads are broadcasts: in the
// forward a warp covers 16 boxes x 2 output groups, in the backward 32 row
// groups x 1 column group.
#include <algorithm>
#include <mutex>

#include "vcb_common.cuh"
#include "vcb_crown_tc.cuh"
#include "vcb_relu.cuh"

namespace vcb {
namespace {

constexpr int kNT = 256;  // threads per CTA

struct CrownParams {
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
  int sl_loff[VCB_MAX_FC];   // float2 offset of relu layer L inside a slot
  long long slot_f2;         // float2 per CTA slot
  int act_soff, pa;          // forward: 2 x (mid | rad), each TB x pa
  int ew_soff, pe, ew_rows;  // backward coefficients (ew_rows x pe, swizzled)
  int acc_soff, bd_soff, part_soff, rt_max;
  int x_soff;
  int v_soff, pv;            // spec x last layer: Q x pv (+ bias column)
  int smem_floats;
  int B, Q, TB, ntiles;
  const float *xl, *xh, *clo, *chi, *sblo, *sbhi, *alpha, *beta, *specW, *specb;
  float *lb, *A, *accout, *sbolo, *sbohi;
  float2* slopes;            // workspace: gridDim.x slots
};

__device__ __forceinline__ float4 ld4(const float* p) {
  return *reinterpret_cast<const float4*>(p);
}

// Logical column k of coefficient row r -> swizzled offset inside the row.
// Rows are pe floats (pe a multiple of 32); the 16-byte chunk index is XORed
// with bits 2..4 of the row so the 4-row register tiles of neighbouring row
// groups hit distinct bank groups.
__device__ __forceinline__ int swz(int r, int k) {
  return ((((k >> 2) ^ ((r >> 2) & 7))) << 2) | (k & 3);
}

__global__ void __launch_bounds__(kNT, 2)
    crown_mlp_kernel(const __grid_constant__ CrownParams p) {
  extern __shared__ __align__(16) float sm[];
  const int tid = threadIdx.x;
  const int nfc = p.n_fc;
  const int n0 = p.dims[0];
  const int nL = p.dims[nfc];
  const int Q = p.Q;
  const int TB = p.TB;
  float2* slot = p.slopes + (long long)blockIdx.x * p.slot_f2;

  // per-thread tile coordinates (fixed for the whole kernel)
  const int SG = TB >> 1;                    // 0 when the forward is skipped
  const int f_og = SG > 0 ? tid / SG : 0;    // forward output group
  const int f_sg = tid - f_og * SG;          // forward box pair (rows sg, sg+SG)
  const int RT = TB * Q;
  const int RG = (RT + 3) >> 2;
  const int b_cg = tid / RG;                 // backward column group
  const int b_rg = tid - b_cg * RG;          // backward row group
  const int r0 = 4 * b_rg;
  int rs[4], rq[4];                          // box and spec row of rows r0..r0+3
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const int r = r0 + j;
    rs[j] = Q > 0 ? min(r / Q, TB - 1) : 0;
    rq[j] = Q > 0 ? min(r - rs[j] * Q, Q - 1) : 0;
  }

  // ---- resident weights: row o of layer l = [W[o,0..n_in), b[o], 0...],
  // copied with cp.async so every element's load is in flight at once.
  for (int l = 0; l < nfc; ++l) {
    const int nin = p.dims[l], nout = p.dims[l + 1], pw = p.pw[l];
    float* dst = sm + p.w_soff[l];
    const float* Wg = p.W + p.w_goff[l];
    const float* bg = p.b + p.b_goff[l];
    for (int o = tid >> 5; o < p.wrows[l]; o += kNT / 32) {
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
  if (tid < 8) sm[p.w_soff[nfc - 1] + p.wrows[nfc - 1] * p.pw[nfc - 1] + tid] = 0.f;
  // ---- spec rows times the last fc layer (identical for every box), from
  // the resident weight rows [W[o, 0..nprev), b[o]]; each thread runs four
  // spec rows' dot products side by side (each one in o order).
  if (Q > 0) {
    __syncthreads();  // the zeroed pad above
    const int nprev = p.dims[nfc - 1];
    const int pwl = p.pw[nfc - 1];
    const float* sWl = sm + p.w_soff[nfc - 1];
    float* V = sm + p.v_soff;
    const int ncol = nprev + 1, nqg = (Q + 3) >> 2;
    for (int item = tid; item < nqg * ncol; item += kNT) {
      const int qg = item / ncol, c = item - qg * ncol;
      const int q0 = 4 * qg;
      float acc4[4] = {0.f, 0.f, 0.f, 0.f};
      for (int o = 0; o < nL; ++o) {
        const float w = sWl[o * pwl + c];
#pragma unroll
        for (int j = 0; j < 4; ++j)
          if (q0 + j < Q) acc4[j] = fmaf(__ldg(p.specW + (q0 + j) * nL + o), w, acc4[j]);
      }
#pragma unroll
      for (int j = 0; j < 4; ++j)
        if (q0 + j < Q) V[(q0 + j) * p.pv + c] = acc4[j];
    }
  }
  __syncthreads();

  float* sXl = sm + p.x_soff;
  float* sXh = sXl + TB * n0;

  for (int tile = blockIdx.x; tile < p.ntiles; tile += gridDim.x) {
    const int s0 = tile * TB;
    const int nb = min(TB, p.B - s0);
    const long long gbase = (long long)s0 * n0;
    for (int idx = tid; idx < TB * n0; idx += kNT) {
      const bool v = idx < nb * n0;
      sXl[idx] = v ? __ldg(p.xl + gbase + idx) : 0.f;
      sXh[idx] = v ? __ldg(p.xh + gbase + idx) : 0.f;
    }
    __syncthreads();

    if (p.sblo == nullptr) {
      // ------------------------------------------------------ IBP forward
      float* act_buf = sm + p.act_soff;
      const int half = 2 * TB * p.pa;  // one (mid | rad) buffer
      {
        const int n0p = pad4(n0);
        for (int s = tid >> 5; s < TB; s += kNT / 32) {
          for (int i = tid & 31; i < n0p; i += 32) {
            float m = 0.f, r = 0.f;
            if (i < n0) {
              const float lo = sXl[s * n0 + i], hi = sXh[s * n0 + i];
              m = __fmul_rn(__fadd_rn(lo, hi), 0.5f);
              r = __fmul_rn(__fsub_rn(hi, lo), 0.5f);
            }
            act_buf[s * p.pa + i] = m;
            act_buf[TB * p.pa + s * p.pa + i] = r;
          }
        }
      }
      __syncthreads();
      for (int l = 0; l < nfc - 1; ++l) {
        const float* mid = act_buf + (l & 1) * half;
        const float* rad = mid + TB * p.pa;
        float* mid_o = act_buf + ((l + 1) & 1) * half;
        float* rad_o = mid_o + TB * p.pa;
        const int nin = p.dims[l], nout = p.dims[l + 1], pw = p.pw[l];
        const float* sW = sm + p.w_soff[l];
        const int G = (nout + 3) >> 2;
        if (f_og < G) {
          float am[2][4], ar[2][4];
#pragma unroll
          for (int s = 0; s < 2; ++s)
#pragma unroll
            for (int j = 0; j < 4; ++j) am[s][j] = ar[s][j] = 0.f;
          const float* w0 = sW + f_og * pw;
          const float* m0 = mid + f_sg * p.pa;
          const float* m1 = mid + (f_sg + SG) * p.pa;
          const float* q0 = rad + f_sg * p.pa;
          const float* q1 = rad + (f_sg + SG) * p.pa;
          const int gstride = G * pw;
          const int kend = pad4(nin);
#pragma unroll 2
          for (int k = 0; k < kend; k += 4) {
            float4 w[4];
#pragma unroll
            for (int j = 0; j < 4; ++j) w[j] = ld4(w0 + j * gstride + k);
            const float4 M0 = ld4(m0 + k), M1 = ld4(m1 + k);
            const float4 R0 = ld4(q0 + k), R1 = ld4(q1 + k);
#pragma unroll
            for (int j = 0; j < 4; ++j) {
              am[0][j] = fmaf(M0.x, w[j].x, am[0][j]);
              am[1][j] = fmaf(M1.x, w[j].x, am[1][j]);
              am[0][j] = fmaf(M0.y, w[j].y, am[0][j]);
              am[1][j] = fmaf(M1.y, w[j].y, am[1][j]);
            }
#pragma unroll
            for (int j = 0; j < 4; ++j) {
              am[0][j] = fmaf(M0.z, w[j].z, am[0][j]);
              am[1][j] = fmaf(M1.z, w[j].z, am[1][j]);
              am[0][j] = fmaf(M0.w, w[j].w, am[0][j]);
              am[1][j] = fmaf(M1.w, w[j].w, am[1][j]);
            }
#pragma unroll
            for (int j = 0; j < 4; ++j) {
              const float ax = fabsf(w[j].x), ay = fabsf(w[j].y);
              ar[0][j] = fmaf(R0.x, ax, ar[0][j]);
              ar[1][j] = fmaf(R1.x, ax, ar[1][j]);
              ar[0][j] = fmaf(R0.y, ay, ar[0][j]);
              ar[1][j] = fmaf(R1.y, ay, ar[1][j]);
            }
#pragma unroll
            for (int j = 0; j < 4; ++j) {
              const float az = fabsf(w[j].z), aw = fabsf(w[j].w);
              ar[0][j] = fmaf(R0.z, az, ar[0][j]);
              ar[1][j] = fmaf(R1.z, az, ar[1][j]);
              ar[0][j] = fmaf(R0.w, aw, ar[0][j]);
              ar[1][j] = fmaf(R1.w, aw, ar[1][j]);
            }
          }
          float2* sl = slot + p.sl_loff[l];
#pragma unroll
          for (int s = 0; s < 2; ++s) {
            const int row = f_sg + s * SG;
#pragma unroll
            for (int j = 0; j < 4; ++j) {
              const int o = f_og + G * j;
              float mo = 0.f, ro = 0.f;
              if (row < nb && o < nout) {
                const float mc = __fadd_rn(am[s][j], sW[o * pw + nin]);
                const float rc = ar[s][j];
                float lo = __fsub_rn(mc, rc);
                float hi = __fadd_rn(mc, rc);
                if (p.clo) {
                  const long long gi = p.relu_goff[l] + (long long)(s0 + row) * nout + o;
                  lo = fmaxf(lo, __ldg(p.clo + gi));
                  hi = fminf(hi, __ldg(p.chi + gi));
                }
                hi = fmaxf(hi, lo);
                if (p.sbolo) {
                  const long long gi = p.relu_goff[l] + (long long)(s0 + row) * nout + o;
                  p.sbolo[gi] = lo;
                  p.sbohi[gi] = hi;
                }
                sl[row * nout + o] = encode_slope(lo, hi);
                const float lc = fmaxf(lo, 0.f), hc = fmaxf(hi, 0.f);
                mo = __fmul_rn(__fadd_rn(lc, hc), 0.5f);
                ro = __fmul_rn(__fsub_rn(hc, lc), 0.5f);
              }
              mid_o[row * p.pa + o] = mo;
              rad_o[row * p.pa + o] = ro;
            }
          }
        }
        __syncthreads();
      }
    } else {
      // --------------------------------- caller-supplied intermediate bounds
      for (int L = 0; L < nfc - 1; ++L) {
        const int n = p.dims[L + 1];
        float2* sl = slot + p.sl_loff[L];
        const long long goff = p.relu_goff[L] + (long long)s0 * n;
        for (int idx = tid; idx < nb * n; idx += kNT)
          sl[idx] = encode_slope(__ldg(p.sblo + goff + idx), __ldg(p.sbhi + goff + idx));
      }
      __syncthreads();
    }

    if (Q > 0) {
      // --------------------------------------------- CROWN back-substitution
      float* ew = sm + p.ew_soff;
      float* sAcc = sm + p.acc_soff;
      float* sBd = sm + p.bd_soff;
      float* sPart = sm + p.part_soff;
      const float* V = sm + p.v_soff;
      const int nvalid = nb * Q;
      for (int r = tid; r < RT; r += kNT) {
        const int q = r - min(r / Q, TB - 1) * Q;
        sAcc[r] = (r < nvalid) ? __ldg(p.specb + q) : 0.f;
      }
      for (int l = nfc - 1; l >= 0; --l) {
        const int nin = p.dims[l], nout = p.dims[l + 1], pw = p.pw[l];
        const float* sW = sm + p.w_soff[l];
        const int CG = (nin + 1 + 7) >> 3;
        const bool act = b_cg < CG;
        const int L = l - 1;  // relu feeding fc l
        // prefetch the slopes of this thread's first box (hidden by the GEMM)
        float2 pre[8];
        const float2* sl = slot + (L >= 0 ? p.sl_loff[L] : 0);
#pragma unroll
        for (int c8 = 0; c8 < 8; ++c8) {
          const int c = 8 * b_cg + c8;
          pre[c8] = (act && L >= 0 && c < nin && rs[0] < nb) ? sl[rs[0] * nin + c]
                                                             : make_float2(0.f, 0.f);
        }
        float acc[4][8];
        if (l == nfc - 1) {
#pragma unroll
          for (int j = 0; j < 4; ++j)
#pragma unroll
            for (int c8 = 0; c8 < 8; ++c8) {
              const int c = 8 * b_cg + c8;
              acc[j][c8] = (act && c <= nin) ? V[rq[j] * p.pv + c] : 0.f;
            }
        } else {
#pragma unroll
          for (int j = 0; j < 4; ++j)
#pragma unroll
            for (int c = 0; c < 8; ++c) acc[j][c] = 0.f;
          if (act) {
            const float* e0 = ew + r0 * p.pe;
            const int xr = b_rg & 7;
            const float* wcol = sW + 8 * b_cg;
            const int kend = pad4(nout);
#pragma unroll 2
            for (int k = 0; k < kend; k += 4) {
              const int kc = (((k >> 2) ^ xr) << 2);
              float4 e[4];
#pragma unroll
              for (int j = 0; j < 4; ++j) e[j] = ld4(e0 + j * p.pe + kc);
#pragma unroll
              for (int kk = 0; kk < 4; ++kk) {
                const float4 wa = ld4(wcol + (k + kk) * pw);
                const float4 wb = ld4(wcol + (k + kk) * pw + 4);
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                  const float ev = kk == 0 ? e[j].x : kk == 1 ? e[j].y : kk == 2 ? e[j].z : e[j].w;
                  acc[j][0] = fmaf(ev, wa.x, acc[j][0]);
                  acc[j][1] = fmaf(ev, wa.y, acc[j][1]);
                  acc[j][2] = fmaf(ev, wa.z, acc[j][2]);
                  acc[j][3] = fmaf(ev, wa.w, acc[j][3]);
                  acc[j][4] = fmaf(ev, wb.x, acc[j][4]);
                  acc[j][5] = fmaf(ev, wb.y, acc[j][5]);
                  acc[j][6] = fmaf(ev, wb.z, acc[j][6]);
                  acc[j][7] = fmaf(ev, wb.w, acc[j][7]);
                }
              }
            }
          }
        }
        __syncthreads();  // every thread has read the coefficient rows
        if (act) {
          const float* alpha = (L >= 0 && p.alpha) ? p.alpha + p.relu_goff[L] + (long long)s0 * nin : nullptr;
          const float* beta = (L >= 0 && p.beta) ? p.beta + p.relu_goff[L] + (long long)s0 * nin : nullptr;
          Slope sv[8];
#pragma unroll
          for (int c8 = 0; c8 < 8; ++c8) {
            const int c = 8 * b_cg + c8;
            if (L < 0) {
              sv[c8].pos = sv[c8].neg = (c < nin) ? 1.f : 0.f;
              sv[c8].icp = 0.f;
            } else {
              sv[c8] = decode_slope(pre[c8], (alpha && c < nin) ? alpha + rs[0] * nin + c : nullptr);
              if (!(c < nin)) sv[c8].pos = sv[c8].neg = sv[c8].icp = 0.f;
            }
          }
          int s_cur = rs[0];
          const int bcg = nin >> 3, bc8 = nin & 7;
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            const int r = r0 + j;
            const bool rv = r < nvalid;
            const int s = rs[j];
            if (L >= 0 && rv && s != s_cur) {  // rows of a second box
              s_cur = s;
#pragma unroll
              for (int c8 = 0; c8 < 8; ++c8) {
                const int c = 8 * b_cg + c8;
                sv[c8] = decode_slope(c < nin ? sl[s * nin + c] : make_float2(0.f, 0.f),
                                      (alpha && c < nin) ? alpha + s * nin + c : nullptr);
                if (!(c < nin)) sv[c8].pos = sv[c8].neg = sv[c8].icp = 0.f;
              }
            }
            float bj = 0.f;
#pragma unroll
            for (int c8 = 0; c8 < 8; ++c8)
              if (c8 == bc8) bj = acc[j][c8];
            const float keep = rv ? 1.f : 0.f;
            float pj = 0.f;
            float out[8];
#pragma unroll
            for (int c8 = 0; c8 < 8; ++c8) {
              const float v = acc[j][c8] * keep;
              const float m = v < 0.f ? sv[c8].neg : sv[c8].pos;
              pj = fmaf(fminf(v, 0.f), sv[c8].icp, pj);
              out[c8] = __fmul_rn(v, m);
            }
            if (beta && rv) {
#pragma unroll
              for (int c8 = 0; c8 < 8; ++c8) {
                const int c = 8 * b_cg + c8;
                if (c < nin) out[c8] = __fadd_rn(out[c8], __ldg(beta + s * nin + c));
              }
            }
            float* row = ew + r * p.pe;
            const int xr = (r >> 2) & 7;
            *reinterpret_cast<float4*>(row + ((((2 * b_cg) ^ xr)) << 2)) =
                make_float4(out[0], out[1], out[2], out[3]);
            *reinterpret_cast<float4*>(row + ((((2 * b_cg + 1) ^ xr)) << 2)) =
                make_float4(out[4], out[5], out[6], out[7]);
            if (r < RT) {
              if (b_cg == bcg) sBd[r] = rv ? bj : 0.f;
              sPart[b_cg * p.rt_max + r] = pj;
            }
          }
        }
        __syncthreads();
        for (int r = tid; r < RT; r += kNT) {
          float a = __fadd_rn(sAcc[r], sBd[r]);
          if (l > 0) {
            float ps = 0.f;
            for (int g = 0; g < CG; ++g) ps = __fadd_rn(ps, sPart[g * p.rt_max + r]);
            a = __fadd_rn(a, ps);
          }
          sAcc[r] = a;
        }
        // the next GEMM reads only ew (complete at the barrier above); the
        // next epilogue rewrites sBd/sPart only after its own barrier.
      }
      __syncthreads();
      // --------------------------------------------------- concretisation
      for (int r = tid; r < nvalid; r += kNT) {
        const int s = r / Q;
        const float* e = ew + r * p.pe;
        const float* xls = sXl + s * n0;
        const float* xhs = sXh + s * n0;
        float s1 = 0.f, s2 = 0.f;
        const long long go = (long long)s0 * Q + r;
        float* Ar = p.A ? p.A + go * n0 : nullptr;
        for (int i = 0; i < n0; ++i) {
          const float ei = e[swz(r, i)];
          s1 = fmaf(fmaxf(ei, 0.f), xls[i], s1);
          s2 = fmaf(fminf(ei, 0.f), xhs[i], s2);
          if (Ar) Ar[i] = ei;
        }
        const float accv = sAcc[r];
        p.lb[go] = __fadd_rn(__fadd_rn(accv, s1), s2);
        if (p.accout) p.accout[go] = accv;
      }
    }
    __syncthreads();
  }
}

struct Layout {
  CrownParams p;
  int bytes;
};

// Shared-memory layout for tile size TB; false when a phase would need more
// than one work item per thread.
bool make_layout(const vcb_mlp* net, int TB, int Q, Layout* out) {
  CrownParams& p = out->p;
  const int nfc = net->n_fc;
  int off = 0;
  int max_w = 1, cg_max = 1, g_max = 1;
  long long slot = 0;
  for (int l = 0; l < nfc; ++l) {
    const int nin = net->dims[l], nout = net->dims[l + 1];
    p.pw[l] = pad4odd(nin + 1);
    p.wrows[l] = pad4(nout);
    p.w_soff[l] = off;
    off += p.wrows[l] * p.pw[l];
    max_w = std::max(max_w, nin);
    cg_max = std::max(cg_max, (nin + 1 + 7) / 8);
    if (l < nfc - 1) {
      g_max = std::max(g_max, (nout + 3) / 4);
      p.sl_loff[l] = (int)slot;
      slot += (long long)TB * nout;
    }
  }
  p.slot_f2 = std::max(slot, 1LL);
  off += 8;
  off = pad4(off);
  const int SG = TB / 2;
  if (nfc > 1 && SG * g_max > kNT) return false;
  if (TB < 1) return false;
  const int RT = TB * Q;
  const int RG = (RT + 3) / 4;
  if (Q > 0 && RG * cg_max > kNT) return false;
  p.pa = pad4odd(std::max(max_w, net->dims[0]));
  p.pe = std::max(32, (8 * cg_max + 31) / 32 * 32);
  p.ew_rows = 4 * RG;
  const int fwd = 4 * TB * p.pa;
  const int bwd = Q > 0 ? p.ew_rows * p.pe : 0;
  p.act_soff = p.ew_soff = off;
  off += pad4(std::max(fwd, bwd));
  p.rt_max = pad4(std::max(RT, 1));
  p.acc_soff = off;
  off += p.rt_max;
  p.bd_soff = off;
  off += p.rt_max;
  p.part_soff = off;
  off += cg_max * p.rt_max;
  p.x_soff = off;
  off += pad4(2 * TB * net->dims[0]);
  p.pv = pad4(net->dims[nfc - 1] + 1);
  p.v_soff = off;
  off += pad4(std::max(Q, 1) * p.pv);
  p.smem_floats = off;
  out->bytes = off * 4;
  return true;
}

struct Plan {
  Layout lay;
  int grid;
  size_t ws_bytes;
};

int plan_crown(const vcb_mlp* net, int B, int Q, bool ibp, Plan* plan) {
  const int nfc = net->n_fc;
  if (nfc < 1 || nfc > VCB_MAX_FC)
    return fail(VCB_ERR_UNSUPPORTED, "vcb_mlp_crown: n_fc=%d outside [1,%d]", nfc, VCB_MAX_FC);
  for (int l = 0; l <= nfc; ++l)
    if (net->dims[l] <= 0)
      return fail(VCB_ERR_INVALID, "vcb_mlp_crown: dims[%d]=%d", l, net->dims[l]);
  if (B < 0 || Q < 0) return fail(VCB_ERR_INVALID, "vcb_mlp_crown: B=%d Q=%d", B, Q);
  // Largest even tile (<= 32) with one work item per thread and two CTAs per
  // SM; otherwise one CTA per SM.
  const int two_cta = (233472 - 2 * 1024) / 2;
  const int one_cta = 232448;
  // Without the IBP forward (caller-supplied bounds) a tile may hold a single
  // box, which many-row specs (the CROWN-intermediate seeds) need.
  const int tb_step = ibp ? 2 : 1;
  // Small batches (a BaB iteration) use the smallest tile (a multiple of
  // tb_step, <= 32) that still covers the batch in one wave of CTAs (two per
  // SM): a tile's time is mostly its chain of dependent layer steps, so a
  // second wave -- even a short one -- would double the launch time.  A
  // box's arithmetic does not depend on the tile size.
  int tb_max = 32;
  const long long slots = 2LL * sm_count();
  if (B > 0 && (long long)B <= 32 * slots) {
    const int t = (int)((B + slots - 1) / slots);
    tb_max = std::max(tb_step, std::min(32, (t + tb_step - 1) / tb_step * tb_step));
  }
  bool found = false;
  for (int pass = 0; pass < 2 && !found; ++pass) {
    const int limit = pass == 0 ? two_cta : one_cta;
    for (int TB = tb_max; TB >= tb_step; TB -= tb_step) {
      Layout t{};
      if (make_layout(net, TB, Q, &t) && t.bytes <= limit) {
        plan->lay = t;
        plan->lay.p.TB = TB;
        found = true;
        break;
      }
    }
  }
  if (!found)
    return fail(VCB_ERR_UNSUPPORTED,
                "vcb_mlp_crown: network does not fit the shared-memory-resident kernel");
  const int TB = plan->lay.p.TB;
  const int ntiles = B > 0 ? (B + TB - 1) / TB : 0;
  const int per_sm = plan->lay.bytes <= two_cta ? 2 : 1;
  plan->grid = std::max(1, std::min(ntiles, sm_count() * per_sm));
  plan->ws_bytes = (size_t)plan->grid * (size_t)plan->lay.p.slot_f2 * sizeof(float2);
  return VCB_OK;
}

}  // namespace
}  // namespace vcb

extern "C" size_t vcb_mlp_crown_workspace(const vcb_mlp* net, int32_t B,
                                          int32_t Q) {
  using namespace vcb;
  if (!net || B <= 0) return 0;
  // Large enough for either mode (the caller-supplied-bounds mode may use a
  // different tile size) and, for networks the tensor-core kernel takes,
  // for that kernel too (its routing threshold may change between calls).
  size_t bytes = 0;
  for (bool ibp : {true, false}) {
    Plan plan;
    if (plan_crown(net, B, Q, ibp, &plan) == VCB_OK) bytes = std::max(bytes, plan.ws_bytes);
  }
  if (crown_tc_eligible(net, Q)) bytes = std::max(bytes, crown_tc_workspace(net, B));
  return bytes;
}

namespace vcb {
namespace {

// Validates the arguments, plans the launch and runs crown_mlp_kernel with
// `slots` as the slope scratch: either `slots_bytes` of caller workspace
// (grid as planned, error if too small) or, when cap_grid is set, a fixed
// buffer whose size caps the number of persistent CTAs.
int launch_crown(const vcb_mlp* net, int32_t B, const float* xl, const float* xh,
                 const float* clamp_lo, const float* clamp_hi, const float* sb_in_lo,
                 const float* sb_in_hi, const float* alpha, const float* beta, int32_t Q,
                 const float* spec_W, const float* spec_b, float* lb, float* A, float* acc,
                 float* sb_out_lo, float* sb_out_hi, void* slots, size_t slots_bytes,
                 bool cap_grid, void* stream, const char* who) {
  if (!net) return fail(VCB_ERR_INVALID, "%s: net is NULL", who);
  if (B < 0 || Q < 0) return fail(VCB_ERR_INVALID, "%s: B=%d Q=%d", who, B, Q);
  if (B == 0) return VCB_OK;  // nothing to bound; output pointers may be NULL
  if (!net->W || !net->b || !xl || !xh)
    return fail(VCB_ERR_INVALID, "%s: NULL weight or box pointer", who);
  if ((clamp_lo == nullptr) != (clamp_hi == nullptr) ||
      (sb_in_lo == nullptr) != (sb_in_hi == nullptr) ||
      (sb_out_lo == nullptr) != (sb_out_hi == nullptr))
    return fail(VCB_ERR_INVALID, "%s: lo/hi pointers must be given in pairs", who);
  if (Q > 0 && (!spec_W || !spec_b || !lb))
    return fail(VCB_ERR_INVALID, "%s: Q>0 needs spec_W, spec_b and lb", who);
  if (sb_in_lo && (clamp_lo || sb_out_lo))
    return fail(VCB_ERR_INVALID, "%s: sb_in excludes clamps and sb_out", who);
  if (!cap_grid && crown_tc_route(net, B, Q))
    return crown_tc_launch(net, B, xl, xh, clamp_lo, clamp_hi, sb_in_lo, sb_in_hi, alpha, beta,
                           Q, spec_W, spec_b, lb, A, acc, sb_out_lo, sb_out_hi, slots,
                           slots_bytes, static_cast<cudaStream_t>(stream), who);
  Plan plan;
  int rc = plan_crown(net, B, Q, /*ibp=*/sb_in_lo == nullptr, &plan);
  if (rc) return rc;
  const size_t slot_bytes = (size_t)plan.lay.p.slot_f2 * sizeof(float2);
  int grid = plan.grid;
  if (cap_grid) {
    const size_t fit = slot_bytes ? slots_bytes / slot_bytes : 0;
    if (fit < 1)
      return fail(VCB_ERR_UNSUPPORTED,
                  "%s: one tile's ReLU slopes need %zu bytes, more than the %zu-byte "
                  "static scratch", who, slot_bytes, slots_bytes);
    grid = (int)std::min<size_t>((size_t)grid, fit);
  } else if (!slots || slots_bytes < plan.ws_bytes) {
    return fail(VCB_ERR_INVALID, "%s: workspace of %zu bytes needed (got %zu)", who,
                plan.ws_bytes, slots_bytes);
  }
  if ((reinterpret_cast<uintptr_t>(slots) & 15) != 0)
    return fail(VCB_ERR_INVALID, "%s: workspace must be 16-byte aligned", who);
  CrownParams& p = plan.lay.p;
  const int nfc = net->n_fc;
  p.n_fc = nfc;
  long long woff = 0;
  int boff = 0;
  long long roff = 0;
  for (int l = 0; l <= nfc; ++l) p.dims[l] = net->dims[l];
  for (int l = 0; l < nfc; ++l) {
    p.w_goff[l] = woff;
    p.b_goff[l] = boff;
    woff += (long long)net->dims[l] * net->dims[l + 1];
    boff += net->dims[l + 1];
    if (l < nfc - 1) {
      p.relu_goff[l] = roff;
      roff += (long long)B * net->dims[l + 1];
    }
  }
  p.W = net->W;
  p.b = net->b;
  p.B = B;
  p.Q = Q;
  p.ntiles = (B + p.TB - 1) / p.TB;
  p.xl = xl;
  p.xh = xh;
  p.clo = clamp_lo;
  p.chi = clamp_hi;
  p.sblo = sb_in_lo;
  p.sbhi = sb_in_hi;
  p.alpha = alpha;
  p.beta = beta;
  p.specW = spec_W;
  p.specb = spec_b;
  p.lb = lb;
  p.A = A;
  p.accout = acc;
  p.sbolo = sb_out_lo;
  p.sbohi = sb_out_hi;
  p.slopes = static_cast<float2*>(slots);
  rc = ensure_smem(reinterpret_cast<const void*>(crown_mlp_kernel), plan.lay.bytes);
  if (rc) return rc;
  crown_mlp_kernel<<<grid, kNT, plan.lay.bytes, static_cast<cudaStream_t>(stream)>>>(p);
  return check_launch(who);
}

}  // namespace
}  // namespace vcb

extern "C" int vcb_mlp_crown(const vcb_mlp* net, int32_t B, const float* xl,
                             const float* xh, const float* clamp_lo,
                             const float* clamp_hi, const float* sb_in_lo,
                             const float* sb_in_hi, const float* alpha,
                             const float* beta, int32_t Q, const float* spec_W,
                             const float* spec_b, float* lb, float* A,
                             float* acc, float* sb_out_lo, float* sb_out_hi,
                             void* workspace, size_t workspace_bytes,
                             void* stream) {
  return vcb::launch_crown(net, B, xl, xh, clamp_lo, clamp_hi, sb_in_lo, sb_in_hi,
                           alpha, beta, Q, spec_W, spec_b, lb, A, acc, sb_out_lo,
                           sb_out_hi, workspace, workspace_bytes, /*cap_grid=*/false,
                           stream, "vcb_mlp_crown");
}

// ---------------------------------------------------------------------------
// Allocation-free variant of vcb_mlp_crown.
//
// Some callers cannot allocate device memory when they bound boxes: a host
// application whose memory pool has already claimed the GPU, or a
// latency-bound loop in which a cudaMalloc (and the device synchronisation it
// can imply) is not allowed.  This entry point takes no workspace: the ReLU
// slope slots live in a file-scope __device__ array of kStaticSlopeBytes that
// every GPU which loads this library holds until the process exits.  The
// array bounds the number of persistent CTAs (one slot each), so a network
// whose single tile needs more than the array is rejected with
// VCB_ERR_UNSUPPORTED.  Every call shares the array: calls that overlap on
// the GPU (different streams, or without ordering between them) race on it.
// Nothing in it needs clearing, because each tile writes its slopes before
// it reads them.
// ---------------------------------------------------------------------------
namespace vcb {
namespace {

constexpr size_t kStaticSlopeBytes = size_t(4) << 20;  // 4 MiB per device
__device__ __align__(256) float2 g_static_slopes[kStaticSlopeBytes / sizeof(float2)];

constexpr int kMaxDevices = 64;
std::mutex g_static_mu;
void* g_static_addr[kMaxDevices] = {};
unsigned long long g_static_ctx[kMaxDevices] = {};  // context the address belongs to

// Unique ID of the current context (cuCtxGetId, reached through the runtime's
// driver entry point so the library needs no link to libcuda); 0 if unknown.
unsigned long long current_context_id() {
  using GetId = int (*)(void*, unsigned long long*);
  static GetId fn = [] {
    void* f = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuCtxGetId", &f, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess)
      f = nullptr;
    return reinterpret_cast<GetId>(f);
  }();
  unsigned long long id = 0;
  if (!fn || fn(nullptr, &id) != 0) return 0;
  return id;
}

// Device address of g_static_slopes on the current device.  The host-side
// symbol is only a stand-in, so the address is looked up with the device
// current and cached per device, together with the ID of the context it was
// looked up in: a device reset (or any other teardown of the primary
// context) reloads the module, and the next call looks the address up again.
int static_slopes_address(void** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_fail(e, "vcb_mlp_crown_noalloc: cudaGetDevice");
  if (dev < 0 || dev >= kMaxDevices)
    return fail(VCB_ERR_UNSUPPORTED, "vcb_mlp_crown_noalloc: device %d", dev);
  std::lock_guard<std::mutex> lk(g_static_mu);
  const unsigned long long ctx = current_context_id();
  if (!g_static_addr[dev] || ctx == 0 || ctx != g_static_ctx[dev]) {
    void* ptr = nullptr;
    e = cudaGetSymbolAddress(&ptr, g_static_slopes);
    if (e != cudaSuccess)
      return cuda_fail(e, "vcb_mlp_crown_noalloc: cudaGetSymbolAddress(g_static_slopes)");
    g_static_addr[dev] = ptr;
    g_static_ctx[dev] = ctx;
  }
  *out = g_static_addr[dev];
  return VCB_OK;
}

}  // namespace
}  // namespace vcb

extern "C" int vcb_mlp_crown_noalloc(const vcb_mlp* net, int32_t B, const float* xl,
                                     const float* xh, const float* clamp_lo,
                                     const float* clamp_hi, const float* sb_in_lo,
                                     const float* sb_in_hi, const float* alpha,
                                     const float* beta, int32_t Q, const float* spec_W,
                                     const float* spec_b, float* lb, float* A,
                                     float* acc, float* sb_out_lo, float* sb_out_hi,
                                     void* stream) {
  using namespace vcb;
  if (B == 0 && net && Q >= 0) return VCB_OK;
  void* slots = nullptr;
  int rc = static_slopes_address(&slots);
  if (rc) return rc;
  return launch_crown(net, B, xl, xh, clamp_lo, clamp_hi, sb_in_lo, sb_in_hi, alpha,
                      beta, Q, spec_W, spec_b, lb, A, acc, sb_out_lo, sb_out_hi, slots,
                      kStaticSlopeBytes, /*cap_grid=*/true, stream,
                      "vcb_mlp_crown_noalloc");
}

extern "C" size_t vcb_mlp_crown_noalloc_capacity(void) { return vcb::kStaticSlopeBytes; }
