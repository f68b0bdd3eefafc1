// Host-side entry points of the tcgen05 3xTF32 GEMM (vcb_tc.cu) for the
// other translation units.
#pragma once

#include <cuda_runtime.h>

namespace vcb {

// C (M x N, ld ldc) = A B^T (+ bias), A / B given as TF32 hi / lo pairs (see
// vcb_tc.cu); err: device int set on a bounded-wait expiry.
int tc_gemm_3xtf32(int M, int N, int K, const float* Ah, const float* Al, int lda,
                   const float* Bh, const float* Bl, int ldb, float* C, int ldc,
                   const float* bias, int* err, cudaStream_t st, const char* who);

int tf32_split(long long n, const float* x, float* hi, float* lo, cudaStream_t st);

}  // namespace vcb
