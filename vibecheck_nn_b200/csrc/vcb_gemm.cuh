// Tiled fp32 GEMM mainloop shared by the layer-wise kernels.
//
// C (M x N) = A (M x K) * B (K x N), accumulated per thread as an 8 x 4
// register tile (rows m0 + ty*8 + i, cols n0 + tx*4 + j) of a 128 x 64 CTA
// tile; 256 threads; 16-deep k-slices double-buffered in shared memory.
// Operands come through loader functors:  a(m, k) and b(k, n) return the
// element or 0 outside the matrix, so plain row-major matrices, transposed
// weights and implicit-GEMM convolution gathers share one mainloop.  A
// loader's kFastA / kFastB says which index consecutive threads should walk
// for coalesced loads (m / n when true, k otherwise).  DUAL
// also accumulates A2 * B2 into acc2 (IBP's mid @ W and rad @ |W| together).
#pragma once

#include "vcb_common.cuh"

namespace vcb {

constexpr int TM = 128, TN = 64, TK = 16, GT = 256;

// A (M x K) row-major with leading dimension ld; as B operand (K x N) it is
// read transposed: b(k, n) = p[n * ld + k] (a weight matrix N x K).
struct RowLoad {
  const float* p;
  int ld;
  __device__ __forceinline__ float a(int m, int k) const { return __ldg(p + (long long)m * ld + k); }
  __device__ __forceinline__ float b(int k, int n) const { return __ldg(p + (long long)n * ld + k); }
  static constexpr bool kFastA = false;  // consecutive threads walk k
  static constexpr bool kFastB = true;   // consecutive threads walk k
};

// B (K x N) row-major with leading dimension ld.
struct ColLoad {
  const float* p;
  int ld;
  __device__ __forceinline__ float b(int k, int n) const { return __ldg(p + (long long)k * ld + n); }
  static constexpr bool kFastB = false;  // consecutive threads walk n
};

// RM consecutive staged A values of one k (16-byte loads where RM allows).
template <int RM>
__device__ __forceinline__ void tile_rows(const float* p, float (&v)[RM]) {
  if constexpr (RM % 4 == 0) {
#pragma unroll
    for (int i = 0; i < RM; i += 4) {
      const float4 t = *reinterpret_cast<const float4*>(p + i);
      v[i] = t.x;
      v[i + 1] = t.y;
      v[i + 2] = t.z;
      v[i + 3] = t.w;
    }
  } else if constexpr (RM == 2) {
    const float2 t = *reinterpret_cast<const float2*>(p);
    v[0] = t.x;
    v[1] = t.y;
  } else {
#pragma unroll
    for (int i = 0; i < RM; ++i) v[i] = p[i];
  }
}

// RM rows per thread: the CTA tile is (16 RM) x 64 (RM = 8: the 128 x 64 tile
// above; smaller RM gives more CTAs for short operands).  Each output
// accumulates over k in ascending order whatever RM is.
template <bool DUAL, int RM, class AL, class BL, class AL2, class BL2>
__device__ __forceinline__ void mainloop_rm(int M, int N, int K, const AL& A, const BL& B,
                                            const AL2& A2, const BL2& B2, float (&acc)[RM][4],
                                            float (&acc2)[RM][4], float* smem) {
  constexpr int TMr = 16 * RM;
  const int tid = threadIdx.x;
  const int ty = tid >> 4, tx = tid & 15;
  const int m0 = blockIdx.x * TMr, n0 = blockIdx.y * TN;
  float* As = smem;                      // [2][TK][TM + 4]
  float* Bs = As + 2 * TK * (TMr + 4);    // [2][TK][TN + 4]
  float* As2 = Bs + 2 * TK * (TN + 4);
  float* Bs2 = As2 + (DUAL ? 2 * TK * (TMr + 4) : 0);
#pragma unroll
  for (int i = 0; i < RM; ++i)
#pragma unroll
    for (int j = 0; j < 4; ++j) acc[i][j] = acc2[i][j] = 0.f;
  float ra[RM], rb[4], ra2[RM], rb2[4];
  auto load = [&](int k0) {
#pragma unroll
    for (int u = 0; u < RM; ++u) {
      const int idx = tid + u * GT;  // TMr rows x 16 k
      int mm, kk;
      if (AL::kFastA) { mm = idx % TMr; kk = idx / TMr; } else { mm = idx >> 4; kk = idx & 15; }
      const int gm = m0 + mm, gk = k0 + kk;
      const bool ok = gm < M && gk < K;
      ra[u] = ok ? A.a(gm, gk) : 0.f;
      if (DUAL) ra2[u] = ok ? A2.a(gm, gk) : 0.f;
    }
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const int idx = tid + u * GT;  // 0..1023: 16 k x 64 cols
      int nn, kk;
      if (BL::kFastB) { nn = idx >> 4; kk = idx & 15; } else { kk = idx >> 6; nn = idx & 63; }
      const int gn = n0 + nn, gk = k0 + kk;
      const bool ok = gn < N && gk < K;
      rb[u] = ok ? B.b(gk, gn) : 0.f;
      if (DUAL) rb2[u] = ok ? B2.b(gk, gn) : 0.f;
    }
  };
  auto store = [&](int buf) {
    float* as = As + buf * TK * (TMr + 4);
    float* bs = Bs + buf * TK * (TN + 4);
#pragma unroll
    for (int u = 0; u < RM; ++u) {
      const int idx = tid + u * GT;
      int mm, kk;
      if (AL::kFastA) { mm = idx % TMr; kk = idx / TMr; } else { mm = idx >> 4; kk = idx & 15; }
      as[kk * (TMr + 4) + mm] = ra[u];
      if (DUAL) As2[buf * TK * (TMr + 4) + kk * (TMr + 4) + mm] = ra2[u];
    }
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const int idx = tid + u * GT;
      int nn, kk;
      if (BL::kFastB) { nn = idx >> 4; kk = idx & 15; } else { kk = idx >> 6; nn = idx & 63; }
      bs[kk * (TN + 4) + nn] = rb[u];
      if (DUAL) Bs2[buf * TK * (TN + 4) + kk * (TN + 4) + nn] = rb2[u];
    }
  };
  const int nk = (K + TK - 1) / TK;
  load(0);
  store(0);
  __syncthreads();
  for (int t = 0; t < nk; ++t) {
    const int buf = t & 1;
    if (t + 1 < nk) load((t + 1) * TK);
    const float* as = As + buf * TK * (TMr + 4);
    const float* bs = Bs + buf * TK * (TN + 4);
    const float* as2 = As2 + buf * TK * (TMr + 4);
    const float* bs2 = Bs2 + buf * TK * (TN + 4);
#pragma unroll
    for (int kk = 0; kk < TK; ++kk) {
      float av[RM], cv[RM];
      tile_rows<RM>(as + kk * (TMr + 4) + ty * RM, av);
      const float4 b0 = *reinterpret_cast<const float4*>(bs + kk * (TN + 4) + tx * 4);
      const float bv[4] = {b0.x, b0.y, b0.z, b0.w};
#pragma unroll
      for (int i = 0; i < RM; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[i][j] = fmaf(av[i], bv[j], acc[i][j]);
      if (DUAL) {
        tile_rows<RM>(as2 + kk * (TMr + 4) + ty * RM, cv);
        const float4 d0 = *reinterpret_cast<const float4*>(bs2 + kk * (TN + 4) + tx * 4);
        const float dv[4] = {d0.x, d0.y, d0.z, d0.w};
#pragma unroll
        for (int i = 0; i < RM; ++i)
#pragma unroll
          for (int j = 0; j < 4; ++j) acc2[i][j] = fmaf(cv[i], dv[j], acc2[i][j]);
      }
    }
    if (t + 1 < nk) store(buf ^ 1);
    __syncthreads();
  }
}

template <bool DUAL, class AL, class BL, class AL2, class BL2>
__device__ __forceinline__ void mainloop(int M, int N, int K, const AL& A, const BL& B,
                                         const AL2& A2, const BL2& B2, float (&acc)[8][4],
                                         float (&acc2)[8][4], float* smem) {
  mainloop_rm<DUAL, 8>(M, N, K, A, B, A2, B2, acc, acc2, smem);
}

inline int gemm_smem_bytes(bool dual, int rm = 8) {
  return (2 * TK * (16 * rm + 4) + 2 * TK * (TN + 4)) * (dual ? 2 : 1) * 4;
}

inline dim3 gemm_grid(int M, int N, int rm = 8) {
  return dim3((M + 16 * rm - 1) / (16 * rm), (N + TN - 1) / TN);
}

}  // namespace vcb
