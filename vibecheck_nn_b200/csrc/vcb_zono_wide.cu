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
//     |G| over the leaf's rows (per 128-row chunk, then over the chunks)
//     -> lo / hi = c -+ that radius.
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

__device__ __forceinline__ void split1(float v, float& h, float& l) {
  const uint32_t u = __float_as_uint(v);
  const bool finite = (u & 0x7F800000u) != 0x7F800000u;
  h = finite ? __uint_as_float((u + 0x1000u) & 0xFFFFE000u) : v;
  l = finite ? __fsub_rn(v, h) : 0.f;
}

__device__ __forceinline__ void split4(const float (&e)[4], float4& h, float4& l) {
  split1(e[0], h.x, l.x);
  split1(e[1], h.y, l.y);
  split1(e[2], h.z, l.z);
  split1(e[3], h.w, l.w);
}

// A rows of leaf b: [0, k_in) scaled rows, [k_in, k_in + cnt) new
// generators, then zeros up to the next leaf's offset.  Source rows come from
// C (ld ldc) at in_off[b], or -- layer 0 (C == NULL) -- are r_b[k] W0T[k].
// One warp per output row, float4 across the row (ld % 4 == 0); each warp
// walks a contiguous range of rows (the leaf found once, then advanced), and
// a row's loads are all issued before its arithmetic so that a warp keeps up
// to kBuildVec float4 loads per lane in flight.
constexpr int kBuildVec = 8;

__global__ void __launch_bounds__(256) zw_build_kernel(
    int B, int n, int ld, const long long* __restrict__ in_off, const int* __restrict__ k_in,
    const float* __restrict__ C, int ldc, const float* __restrict__ r, int n0,
    const float* __restrict__ W0T, const float* __restrict__ lam, const float* __restrict__ mu,
    const int* __restrict__ cnt, const int* __restrict__ idx_of_rank,
    const long long* __restrict__ out_off, long long total_rows, float* __restrict__ Ah,
    float* __restrict__ Al) {
  const int lane = threadIdx.x & 31;
  const long long warps = (long long)gridDim.x * (blockDim.x >> 5);
  const long long wid = (long long)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const long long per = (total_rows + warps - 1) / warps;
  const long long r0 = wid * per, r1 = min(total_rows, r0 + per);
  if (r0 >= r1) return;
  const int nv = ld >> 2;
  const bool vec = (n & 3) == 0 && (C == nullptr || (ldc & 3) == 0);
  // leaf of the first row: binary search of out_off (B + 1 offsets)
  int b;
  {
    int lo = 0, hi = B;
    while (hi - lo > 1) {
      const int m = (lo + hi) >> 1;
      if (out_off[m] <= r0) lo = m; else hi = m;
    }
    b = lo;
  }
  long long leaf_end = out_off[b + 1];
  for (long long row = r0; row < r1; ++row) {
    while (row >= leaf_end) {
      ++b;
      leaf_end = out_off[b + 1];
    }
    const long long rr = row - out_off[b];
    const int kin = k_in[b], u = cnt[b];
    const float4* lam4 = reinterpret_cast<const float4*>(lam + (long long)b * n);
    float4* dh = reinterpret_cast<float4*>(Ah + row * ld);
    float4* dl = reinterpret_cast<float4*>(Al + row * ld);
    if (rr < kin && vec) {
      const float* src = C ? C + (in_off[b] + rr) * ldc : W0T + rr * (long long)n;
      const float rk = C ? 1.f : r[(long long)b * n0 + rr];
      const float4* src4 = reinterpret_cast<const float4*>(src);
      const int nvn = n >> 2;  // float4 of real columns
      for (int v0 = 0; v0 < nv; v0 += 32 * kBuildVec) {
        float4 g[kBuildVec], lv[kBuildVec];
#pragma unroll
        for (int t = 0; t < kBuildVec; ++t) {
          const int v = v0 + 32 * t + lane;
          g[t] = v < nvn ? src4[v] : make_float4(0.f, 0.f, 0.f, 0.f);
          lv[t] = v < nvn ? lam4[v] : make_float4(0.f, 0.f, 0.f, 0.f);
        }
#pragma unroll
        for (int t = 0; t < kBuildVec; ++t) {
          const int v = v0 + 32 * t + lane;
          if (v >= nv) break;
          float e[4] = {C ? g[t].x : __fmul_rn(g[t].x, rk), C ? g[t].y : __fmul_rn(g[t].y, rk),
                        C ? g[t].z : __fmul_rn(g[t].z, rk), C ? g[t].w : __fmul_rn(g[t].w, rk)};
          e[0] = __fmul_rn(e[0], lv[t].x);
          e[1] = __fmul_rn(e[1], lv[t].y);
          e[2] = __fmul_rn(e[2], lv[t].z);
          e[3] = __fmul_rn(e[3], lv[t].w);
          float4 h, l;
          split4(e, h, l);
          dh[v] = h;
          dl[v] = l;
        }
      }
    } else if (rr < kin) {
      const float* src = C ? C + (in_off[b] + rr) * ldc : W0T + rr * (long long)n;
      const float rk = C ? 1.f : r[(long long)b * n0 + rr];
      for (int v = lane; v < nv; v += 32) {
        float e[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
        for (int t = 0; t < 4; ++t) {
          const int jj = 4 * v + t;
          if (jj < n) {
            const float gg = C ? src[jj] : __fmul_rn(src[jj], rk);
            e[t] = __fmul_rn(gg, lam[(long long)b * n + jj]);
          }
        }
        float4 h, l;
        split4(e, h, l);
        dh[v] = h;
        dl[v] = l;
      }
    } else {
      const int jj = (rr < kin + u) ? idx_of_rank[(long long)b * n + (rr - kin)] : -1;
      const float m = jj >= 0 ? mu[(long long)b * n + jj] : 0.f;
      for (int v = lane; v < nv; v += 32) {
        float e[4];
#pragma unroll
        for (int t = 0; t < 4; ++t) e[t] = (4 * v + t == jj) ? m : 0.f;
        float4 h, l;
        split4(e, h, l);
        dh[v] = h;
        dl[v] = l;
      }
    }
  }
}

// rad[b][j] = sum over the leaf's k rows of |C[row][j]| with Neumaier's
// compensated summation in a fixed order: chunks of kChunk rows (one thread
// per (chunk, column)) give (sum, compensation) partials, then the chunks of
// a leaf are combined in order.  lo = c - rad, hi = c + rad.
constexpr int kChunk = 128;

__device__ __forceinline__ void neumaier(float& s, float& comp, float v) {
  const float t = __fadd_rn(s, v);
  comp = __fadd_rn(comp, (fabsf(s) >= fabsf(v)) ? __fadd_rn(__fsub_rn(s, t), v)
                                                 : __fadd_rn(__fsub_rn(v, t), s));
  s = t;
}

__global__ void __launch_bounds__(256) zw_colsum_part_kernel(
    int n, const long long* __restrict__ off, const int* __restrict__ k,
    const long long* __restrict__ chunk_off, const float* __restrict__ C, int ldc,
    float2* __restrict__ part) {
  const int b = blockIdx.z;
  const int ch = blockIdx.y;  // chunk index inside the leaf
  const int j = blockIdx.x * blockDim.x + threadIdx.x;
  const long long nch = chunk_off[b + 1] - chunk_off[b];
  if (ch >= nch || j >= n) return;
  const int kb = k[b];
  const int r0 = ch * kChunk, r1 = min(kb, r0 + kChunk);
  const float* p = C + (off[b] + r0) * ldc + j;
  float s = 0.f, comp = 0.f;
  int row = r0;
  // eight loads in flight per thread, then the fixed-order compensated sum
  for (; row + 8 <= r1; row += 8) {
    float v[8];
#pragma unroll
    for (int t = 0; t < 8; ++t) v[t] = p[(long long)t * ldc];
#pragma unroll
    for (int t = 0; t < 8; ++t) neumaier(s, comp, fabsf(v[t]));
    p += 8LL * ldc;
  }
  for (; row < r1; ++row) {
    neumaier(s, comp, fabsf(*p));
    p += ldc;
  }
  part[(chunk_off[b] + ch) * n + j] = make_float2(s, comp);
}

__global__ void __launch_bounds__(256) zw_colsum_combine_kernel(
    int n, const long long* __restrict__ chunk_off, const float2* __restrict__ part,
    const float* __restrict__ c, float* __restrict__ lo, float* __restrict__ hi) {
  const int b = blockIdx.y;
  const int j = blockIdx.x * blockDim.x + threadIdx.x;
  if (j >= n) return;
  float s = 0.f, comp = 0.f;
  for (long long ch = chunk_off[b]; ch < chunk_off[b + 1]; ++ch) {
    const float2 v = part[ch * n + j];
    neumaier(s, comp, v.x);
    comp = __fadd_rn(comp, v.y);
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
  if (B == 0 || rows_hint == 0) return VCB_OK;
  if (!k_in || !lam || !mu || !cnt || !idx_of_rank || !out_off || !A_hi || !A_lo ||
      (C && !in_off) || (!C && (!r || !W0T)))
    return fail(VCB_ERR_INVALID, "vcb_zw_build: NULL pointer");
  const long long blocks = std::min<long long>((rows_hint + 7) / 8, 148LL * 64);
  zw_build_kernel<<<(unsigned)blocks, 256, 0, static_cast<cudaStream_t>(stream)>>>(
      B, n, ld, reinterpret_cast<const long long*>(in_off), k_in, C, ldc, r, n0, W0T, lam, mu,
      cnt, idx_of_rank, reinterpret_cast<const long long*>(out_off), rows_hint, A_hi, A_lo);
  return check_launch("vcb_zw_build");
}

extern "C" size_t vcb_zw_colsum_workspace(int64_t total_chunks, int32_t n) {
  if (total_chunks <= 0 || n <= 0) return 0;
  return (size_t)total_chunks * n * sizeof(float2);
}

extern "C" int vcb_zw_colsum(int32_t B, int32_t n, const int64_t* off, const int32_t* k,
                             const int64_t* chunk_off, int32_t max_chunks, const float* C,
                             int32_t ldc, const float* c, float* lo, float* hi, void* workspace,
                             size_t workspace_bytes, void* stream) {
  if (B < 0 || n <= 0 || ldc < n || max_chunks < 0)
    return fail(VCB_ERR_INVALID, "vcb_zw_colsum: B=%d n=%d", B, n);
  if (B == 0) return VCB_OK;
  if (!off || !k || !chunk_off || !C || !c || !lo || !hi || (max_chunks > 0 && !workspace))
    return fail(VCB_ERR_INVALID, "vcb_zw_colsum: NULL pointer");
  if (B > 65535 || max_chunks > 65535)
    return fail(VCB_ERR_UNSUPPORTED, "vcb_zw_colsum: %d leaves, %d chunks", B, max_chunks);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  float2* part = static_cast<float2*>(workspace);
  if (max_chunks > 0) {
    zw_colsum_part_kernel<<<dim3((n + 255) / 256, max_chunks, B), 256, 0, st>>>(
        n, reinterpret_cast<const long long*>(off), k,
        reinterpret_cast<const long long*>(chunk_off), C, ldc, part);
    const int rc = check_launch("vcb_zw_colsum: parts");
    if (rc) return rc;
  }
  zw_colsum_combine_kernel<<<dim3((n + 255) / 256, B), 256, 0, st>>>(
      n, reinterpret_cast<const long long*>(chunk_off), part, c, lo, hi);
  return check_launch("vcb_zw_colsum");
}
