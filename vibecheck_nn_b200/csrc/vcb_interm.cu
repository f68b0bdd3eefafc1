// CROWN intermediate-bound intersection (verify_zono_bnb.py:4140-4146).
//
// For relu layer L, rows [0, n) of `lb_rows` hold the backward-CROWN lower
// bound of +z_j and rows [n, 2n) that of -z_j for every neuron j of the layer
// (seeded at the layer's feeding op with [+I; -I]).  For the neurons in the
// batch-wide "unstable anywhere" mask, the running (zonotope) bounds are
// intersected in place:
//   lo = max(lo, lb_j),  hi = max(min(hi, -lb_{n+j}), lo).
// Other neurons keep their bounds, exactly as the reference, which seeds
// only the union set.
#include <algorithm>

#include "vcb_common.cuh"

namespace {
__global__ void interm_intersect_kernel(int B, int n, const float* __restrict__ lb_rows,
                                        const int* __restrict__ mask,
                                        float* __restrict__ lo, float* __restrict__ hi) {
  const long long total = (long long)B * n;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total;
       i += (long long)gridDim.x * blockDim.x) {
    const int j = (int)(i % n);
    if (!mask[j]) continue;
    const long long b = i / n;
    const float l_new = fmaxf(lo[i], lb_rows[b * 2 * n + j]);
    const float h_new = fmaxf(fminf(hi[i], -lb_rows[b * 2 * n + n + j]), l_new);
    lo[i] = l_new;
    hi[i] = h_new;
  }
}
}  // namespace

extern "C" int vcb_interm_intersect(int32_t B, int32_t n, const float* lb_rows,
                                    const int32_t* unstable_any, float* lo, float* hi,
                                    void* stream) {
  using namespace vcb;
  if (B < 0 || n <= 0) return fail(VCB_ERR_INVALID, "vcb_interm_intersect: B=%d n=%d", B, n);
  if (B == 0) return VCB_OK;
  if (!lb_rows || !unstable_any || !lo || !hi)
    return fail(VCB_ERR_INVALID, "vcb_interm_intersect: NULL pointer");
  const long long total = (long long)B * n;
  const int block = 256;
  const int grid = (int)std::min<long long>((total + block - 1) / block, 4LL * sm_count() * 8);
  interm_intersect_kernel<<<grid, block, 0, static_cast<cudaStream_t>(stream)>>>(
      B, n, lb_rows, unstable_any, lo, hi);
  return check_launch("vcb_interm_intersect: launch");
}
