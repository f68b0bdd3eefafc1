// Host-side entry points of the tcgen05 3xTF32 GEMM (vcb_tc.cu) for the
// other translation units.
#pragma once

#include <cuda_runtime.h>

namespace vcb {

// C (M x N, ld ldc) = A B^T (+ bias), A / B given as TF32 hi / lo pairs (see
// vcb_tc.cu); err: device int set on a bounded-wait expiry; gate: optional
// device int, the launch does nothing when it is 0.
int tc_gemm_3xtf32(int M, int N, int K, const float* Ah, const float* Al, int lda,
                   const float* Bh, const float* Bl, int ldb, float* C, int ldc,
                   const float* bias, int* err, cudaStream_t st, const char* who,
                   const int* gate = nullptr);

int tf32_split(long long n, const float* x, float* hi, float* lo, cudaStream_t st);

// Fused epilogues of the 3xTF32 GEMM for the alpha-CROWN layers (row m of C
// belongs to box m / Q; per-box arrays are (R / Q) x N, row-major).  Each
// accumulator thread holds 128 consecutive columns of one row:
//   kEpiStore      C = acc (+ bias);
//   kEpiRelax      C = acc kept as the record; ReLU relaxation (lower slope
//                  pos, rx = (upper slope, negated for stable neurons;
//                  intercept factor)) + beta (or NULL) -> split into out_hi /
//                  out_lo; the group's intercept sum + coef_o . bnext (or
//                  NULL) to part;
//   kEpiAdjoint    ga = acc + bias; with the record rec: dcontrib =
//                  [unstable] max(e, 0) ga, next adjoint split into out_hi /
//                  out_lo (or NULL); C unused;
//   kEpiConcretize e = acc; the group's sum(e+ xl + e- xh) to part and the
//                  adjoint seed xl [e >= 0] + xh [e <= 0] split into out_hi /
//                  out_lo; C unused.
// part: one partial per 64-column group, at part[m * ldpart + part0 + n / 64].
enum TcEpiMode { kEpiStore = 0, kEpiRelax = 1, kEpiAdjoint = 2, kEpiConcretize = 3 };

struct TcEpi {
  int mode = kEpiStore;
  int Q = 1;
  const float* pos = nullptr;   // lower slope per neuron (alpha; 1 active, 0 dead)
  const float2* rx = nullptr;   // (upper slope, sign bit set when stable; intercept factor)
  const float *beta = nullptr, *bnext = nullptr;
  const float *xl = nullptr, *xh = nullptr;
  const float* rec = nullptr;
  int ldrec = 0;
  float *out_hi = nullptr, *out_lo = nullptr;
  int ldo = 0;
  float* dcontrib = nullptr;
  int ldd = 0;
  float* part = nullptr;
  int ldpart = 0, part0 = 0;
};

int tc_gemm_fused(int M, int N, int K, const float* Ah, const float* Al, int lda,
                  const float* Bh, const float* Bl, int ldb, float* C, int ldc,
                  const float* bias, int* err, cudaStream_t st, const char* who,
                  const int* gate, const TcEpi& ep);

}  // namespace vcb
