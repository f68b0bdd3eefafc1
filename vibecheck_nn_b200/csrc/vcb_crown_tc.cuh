// Tensor-core variant of the fused IBP + CROWN kernel (vcb_crown_tc.cu):
// routing and launch, used by vcb_mlp_crown.
#pragma once

#include <cuda_runtime.h>

#include <cstddef>

#include "vcb.h"

namespace vcb {

// The network and spec count fit the tensor-core kernel (input and hidden
// widths <= 63, 1 <= n_fc - 1, Q <= 16).
bool crown_tc_eligible(const vcb_mlp* net, int Q);

// vcb_mlp_crown takes the tensor-core kernel for this call: eligible and
// B >= the routing threshold (vcb_mlp_crown_tc_min_batch).
bool crown_tc_route(const vcb_mlp* net, int B, int Q);

// Workspace bytes of the tensor-core kernel (0 when not eligible).
size_t crown_tc_workspace(const vcb_mlp* net, int B);

// Arguments as vcb_mlp_crown, already validated.
int crown_tc_launch(const vcb_mlp* net, int32_t B, const float* xl, const float* xh,
                    const float* clamp_lo, const float* clamp_hi, const float* sb_in_lo,
                    const float* sb_in_hi, const float* alpha, const float* beta, int32_t Q,
                    const float* spec_W, const float* spec_b, float* lb, float* A, float* acc,
                    float* sb_out_lo, float* sb_out_hi, void* ws, size_t ws_bytes,
                    cudaStream_t st, const char* who);

// Reads and clears the device fault word of crown_tc_kernel (set when one of
// its bounded waits expired) after synchronising st; *was_set = 1 if it was.
int crown_tc_fault_take(cudaStream_t st, int* was_set);

}  // namespace vcb
