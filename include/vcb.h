/*
 * vcb.h -- C ABI of libvcb.so, the sm_100a bound-propagation kernels behind
 * vibecheck's batched input-split branch-and-bound.
 *
 * Every entry point takes plain device pointers, sizes and a cudaStream_t
 * (passed as void*; NULL = legacy default stream), returns an int status
 * (VCB_OK = 0) and never allocates or frees caller memory unless stated.
 * Work is stream-ordered: no entry point synchronises the device unless its
 * comment says so.  vcb_last_error() returns a thread-local message for the
 * last non-zero status.
 *
 * Network descriptor: a ReLU MLP as fc/relu layers.  W holds the fc weight
 * matrices back to back, layer l row-major (dims[l+1] x dims[l]); b holds the
 * biases back to back.  relu layer L sits between fc L and fc L+1, so there
 * are n_fc - 1 relu layers with widths dims[1..n_fc-1].
 *
 * "Packed per-layer" arrays (bounds, clamps, alpha, beta) hold the relu
 * layers back to back, layer L as a contiguous (B x dims[L+1]) block.
 */
#ifndef VCB_H
#define VCB_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define VCB_MAX_FC 16

enum {
  VCB_OK = 0,
  VCB_ERR_INVALID = 1,     /* bad argument: maps to ValueError            */
  VCB_ERR_UNSUPPORTED = 2, /* shape/op outside this kernel: NotImplemented */
  VCB_ERR_CUDA = 3,        /* CUDA runtime error: RuntimeError            */
  VCB_ERR_OOM = 4,         /* device allocation failed: OutOfMemoryError  */
  VCB_ERR_TIMEOUT = 5      /* a bounded device-side wait ran out          */
};

typedef struct vcb_mlp {
  int32_t n_fc;                   /* number of fc layers (relu layers + 1) */
  int32_t dims[VCB_MAX_FC + 1];   /* dims[0] = input width                 */
  const float* W;                 /* device, fc weights back to back       */
  const float* b;                 /* device, fc biases back to back        */
} vcb_mlp;

/* Library version (major*10000 + minor*100 + patch). */
int vcb_version(void);

/* Message for the last non-zero status returned on this thread. */
const char* vcb_last_error(void);

/* Fused IBP forward + CROWN back-substitution for ReLU MLPs whose weights fit
 * in shared memory (the ACAS-Xu-sized path).
 *
 * Replaces, in one launch, vibecheck's
 *   _ibp_forward_graph_batched(xl, xh, gg, device, dtype, relu_clamps)
 *       (src/vibecheck/verify_zono_bnb.py:1066)
 *   _spec_backward_graph_batched(tight, xl, xh, gg, spec_ew, device, dtype,
 *       return_input_linear, alpha_at_layer, relu_split_beta)
 *       (src/vibecheck/verify_zono_bnb.py:4270)
 * and their composition used by the ReLU-split BaB (verify_milp.py:2762).
 *
 *   xl, xh        (B, dims[0]) input boxes.
 *   clamp_lo/hi   packed per-layer relu clamps (-inf/+inf = none), or NULL.
 *   sb_in_lo/hi   packed per-layer pre-activation bounds, or NULL.  When
 *                 given, the IBP forward is skipped and these bounds drive
 *                 the ReLU relaxation (the plain spec-backward call).
 *   alpha         packed per-layer lower slopes for unstable neurons
 *                 (alpha-CROWN), or NULL for the min-area choice.
 *   beta          packed per-layer signed split multipliers, or NULL.
 *   Q, spec_W (Q x dims[n_fc]), spec_b (Q): spec rows; Q = 0 runs IBP only.
 *   lb            (B, Q) output lower bounds, or NULL when Q = 0.
 *   A, acc        optional (B, Q, dims[0]) / (B, Q) input-space linear form
 *                 (spec_q(x) >= A[b,q].x + acc[b,q]), or NULL.
 *   sb_out_lo/hi  optional packed per-layer IBP bounds out (the bounds the
 *                 relaxation used, after clamps and crossing repair).
 *   workspace     device scratch of at least vcb_mlp_crown_workspace(net, B,
 *                 Q) bytes, 16-byte aligned (per-CTA ReLU slope slots).
 *                 Calls that overlap on the GPU must not share it.
 */
int vcb_mlp_crown(const vcb_mlp* net, int32_t B,
                  const float* xl, const float* xh,
                  const float* clamp_lo, const float* clamp_hi,
                  const float* sb_in_lo, const float* sb_in_hi,
                  const float* alpha, const float* beta,
                  int32_t Q, const float* spec_W, const float* spec_b,
                  float* lb, float* A, float* acc,
                  float* sb_out_lo, float* sb_out_hi,
                  void* workspace, size_t workspace_bytes,
                  void* stream);

/* Workspace bytes vcb_mlp_crown needs for (net, B, Q); 0 on bad arguments
 * (vcb_mlp_crown then reports the error). */
size_t vcb_mlp_crown_workspace(const vcb_mlp* net, int32_t B, int32_t Q);

/* Diagnostic: FP32 FFMA throughput probe (no reference counterpart).  Runs
 * `blocks` CTAs of 256 threads, each thread `iters` x 64 dependent-chain FMAs
 * (8 independent chains); FLOPs = blocks * 256 * iters * 128.  `out` must
 * hold blocks*256 floats and is written only in a never-taken branch. */
int vcb_probe_ffma(float* out, int32_t blocks, int32_t iters, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* VCB_H */
