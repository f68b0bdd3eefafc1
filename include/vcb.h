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

/* Deferred device-fault report (no counterpart in the reference, whose
 * PyTorch ops have no bounded device-side waits).  Synchronises `stream`,
 * then returns VCB_ERR_TIMEOUT if the tensor-core CROWN kernel gave up one of
 * its bounded waits on this device since the last call (the boxes it had not
 * finished got NaN bounds), and clears the report; VCB_OK otherwise.
 * Callers check it where they synchronise anyway. */
int vcb_fault_check(void* stream);

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

/* Routing threshold of vcb_mlp_crown (no counterpart in the reference, which
 * has one implementation): networks with input and hidden widths <= 63 and
 * Q <= 16 are bounded by the tensor-core (tcgen05, 3xTF32) kernel when
 * B >= the threshold, else by the fp32 SIMT kernel; results agree to fp32
 * rounding.  Sets the threshold when value >= 0 and returns the previous
 * one (process-wide). */
int32_t vcb_mlp_crown_tc_min_batch(int32_t value);

/* Which kernel vcb_mlp_crown runs for (net, B, Q) under the current
 * threshold: 1 = tensor-core, 0 = SIMT. */
int32_t vcb_mlp_crown_path(const vcb_mlp* net, int32_t B, int32_t Q);

/* Batched forward linear bounds (forward LiRPA, the default bound of the
 * multi-subbox input-split BaB: chunked_batched_forward_linear_bounds,
 * forward_lirpa.py:1391, fc / relu ops :580-687) of B boxes xl/xh (B x
 * dims[0]) over the K varying input dimensions var_idx (int32[K]), then the
 * spec rows spec_W (Q x dims[n_fc]) as in verify_graph.py:11522-11560:
 * spec_A (B x Q x K, may be NULL) = w+ A_lo + w- A_up, spec_b (B x Q, may be
 * NULL) likewise, lb (B x Q) = spec_A+ xl + spec_A- xh + spec_b over the
 * varying dimensions.  A_lo/A_up (B x n_out x K) and b_lo/b_up (B x n_out),
 * the output bounds, are written when non-NULL.  Widths <= 64, 1 <= K <= 31,
 * Q <= 64. */
int vcb_mlp_flirpa(const vcb_mlp* net, int32_t B, int32_t K, const float* xl,
                   const float* xh, const int32_t* var_idx, int32_t Q,
                   const float* spec_W, float* spec_A, float* spec_b, float* lb,
                   float* A_lo, float* A_up, float* b_lo, float* b_up, void* stream);

/* Leaf fate of one multi-subbox BaB batch (verify_graph.py:11640-11802).
 * Leaf b of B (boxes xl/xh, B x n_in; sub-box sub[b]) with the forward-LiRPA
 * outputs of vcb_mlp_flirpa over the K varying dimensions var_idx (spec_A
 * B x Q x K, spec_b and lb B x Q) and the per-sub-box query bias sub_bias
 * (n_sub x Q):
 *   fate[b] = 0  some query has lb + bias > 0 (safe);
 *             1  clip_iters rounds of _clip_input_domain (:11121-11177) over
 *                the varying dimensions leave an empty box (safe);
 *             2  to split: out_xl/out_xh hold the clipped box and score the
 *                smart-branching score of every input dimension (-inf where
 *                the dimension does not vary or is <= 1e-12 wide);
 *   fate[B] = the largest number of dimensions wider than 1e-12 among the
 *             leaves to split (0 when none).
 * Rows with fate 0 / 1 leave out_xl/out_xh/score unwritten.  K <= 32, Q <= 64. */
int vcb_multisub_fate(int32_t B, int32_t n_in, int32_t K, int32_t Q, const float* xl,
                      const float* xh, const int32_t* var_idx, const float* spec_A,
                      const float* spec_b, const float* lb, const float* sub_bias,
                      const int32_t* sub, int32_t clip_iters, int32_t* fate, float* out_xl,
                      float* out_xh, float* score, void* stream);

/* vcb_mlp_flirpa followed by vcb_multisub_fate in one kernel: the spec rows
 * stay in shared memory and only the fates, clipped boxes and scores are
 * written (same arguments and outputs as the two calls, same values). */
int vcb_mlp_flirpa_fate(const vcb_mlp* net, int32_t B, int32_t K, const float* xl,
                        const float* xh, const int32_t* var_idx, int32_t Q,
                        const float* spec_W, const float* sub_bias, const int32_t* sub,
                        int32_t clip_iters, int32_t* fate, float* out_xl, float* out_xh,
                        float* score, void* stream);

/* Children of the U leaves rows[0..U) of a multi-subbox batch
 * (verify_graph.py:11804-11852): each leaf ranks its dimensions by score
 * (B x n_in) in CPU torch.topk order, bisects the first k of them that are
 * wider than 1e-12 and writes its 2^k children (bit j of the child index set
 * = high half of the j-th ranked dimension) to rows u 2^k .. (u+1) 2^k - 1 of
 * kid_xl/kid_xh (U 2^k x n_in), with kid_sub = sub[rows[u]].  workspace holds
 * vcb_multisub_emit_workspace(U, n_in, k) bytes.  k <= 16. */
int64_t vcb_multisub_emit_workspace(int32_t U, int32_t n_in, int32_t k);
int vcb_multisub_emit(int32_t U, int32_t n_in, int32_t k, const int32_t* rows, const float* xl,
                      const float* xh, const float* score, const int32_t* sub, void* workspace,
                      float* kid_xl, float* kid_xh, int32_t* kid_sub, void* stream);

/* Allocation-free variant of vcb_mlp_crown (no counterpart in the
 * reference).  For callers that cannot allocate device memory while they
 * bound boxes -- a host application whose memory pool already owns the GPU,
 * or a latency-bound loop that must not call cudaMalloc -- it takes no
 * workspace: the ReLU-slope scratch is a file-scope __device__ array of
 * vcb_mlp_crown_noalloc_capacity() bytes (4 MiB) that every GPU loading the
 * library holds until exit.  The array caps the number of persistent CTAs;
 * a network whose single tile needs more than the array returns
 * VCB_ERR_UNSUPPORTED.  The first call on a device looks up the array's
 * device address, so make it before any stream capture; the address is
 * cached per device and context, so the first call after a device reset
 * (which reloads the library's module) looks it up again.  All calls share
 * the array: calls that overlap on the GPU race on it.  Arguments and
 * results are those of vcb_mlp_crown. */
int vcb_mlp_crown_noalloc(const vcb_mlp* net, int32_t B,
                          const float* xl, const float* xh,
                          const float* clamp_lo, const float* clamp_hi,
                          const float* sb_in_lo, const float* sb_in_hi,
                          const float* alpha, const float* beta,
                          int32_t Q, const float* spec_W, const float* spec_b,
                          float* lb, float* A, float* acc,
                          float* sb_out_lo, float* sb_out_hi,
                          void* stream);

/* Bytes of the static scratch behind vcb_mlp_crown_noalloc. */
size_t vcb_mlp_crown_noalloc_capacity(void);

/* Batched DeepZ zonotope forward for ReLU MLPs (shared-memory-resident
 * weights).  Replaces _forward_zonotope_graph_batched(xl, xh, gg, device,
 * dtype) (src/vibecheck/verify_zono_bnb.py:3079).
 *
 *   sb_lo/hi      packed per-layer pre-activation bounds out (or NULL).
 *   unstable_any  per relu layer, per neuron int flags (layers back to back,
 *                 dims[1..n_fc-1]); set to 1 where the neuron is unstable in
 *                 some box (the caller zeroes it first), or NULL.
 *   c_out, g_out, k_out  when c_out is non-NULL the last fc layer runs too:
 *                 c_out (B, dims[n_fc]), g_out (B, dims[n_fc], kmax) with the
 *                 box's own generators first and zeros after, k_out (B,) the
 *                 generator count; kmax = vcb_mlp_zono_kmax(net).
 */
int vcb_mlp_zono(const vcb_mlp* net, int32_t B, const float* xl,
                 const float* xh, float* sb_lo, float* sb_hi,
                 int32_t* unstable_any, float* c_out, float* g_out,
                 int32_t* k_out, void* stream);

/* Generator capacity of the zonotope: dims[0] + sum of relu widths. */
int vcb_mlp_zono_kmax(const vcb_mlp* net);

/* CROWN intermediate-bound intersection for one relu layer of width n
 * (src/vibecheck/verify_zono_bnb.py:4140-4146): lb_rows (B, 2n) holds the
 * backward-CROWN lower bounds of [+z_j; -z_j]; where unstable_any[j] is set,
 * lo = max(lo, lb_j) and hi = max(min(hi, -lb_{n+j}), lo), in place on the
 * (B, n) lo/hi arrays. */
int vcb_interm_intersect(int32_t B, int32_t n, const float* lb_rows,
                         const int32_t* unstable_any, float* lo, float* hi,
                         void* stream);

/* One input-split BaB step for a batch of B leaves (single-CTA launch):
 * closure, halfspace clipping, branching and child emission, following
 * _input_split_batched_inner (src/vibecheck/verify_graph.py:12899-13382) and
 * _clip_box_by_halfspaces_batched (verify_graph.py:12363).
 *
 *   query_disjunct (Q) disjunct id of each deduplicated query, 0..D-1.
 *   q_sens         leading queries summed into the SB branching score (the
 *                  unique halfspaces; later rows repeat one for another
 *                  disjunct); <= 0 means all Q.
 *   xl, xh (B, n_in); lb (B, Q); A (B, Q, n_in), acc (B, Q): the CROWN
 *   input-space linear form (needed when clip or branch_sb).
 *   lo_xl/lo_xh, hi_xl/hi_xh (B, n_in): the low-half and high-half children
 *   of the usable leaves, compacted in leaf order.
 *   counters[4]: leaves closed by CROWN, closed by clipping, split (= rows
 *   written to each child block), degenerate (width <= 1e-12, left open).
 */
int vcb_bab_step(int32_t B, int32_t n_in, int32_t Q, int32_t D,
                 int32_t q_sens, const int32_t* query_disjunct, const float* xl,
                 const float* xh, const float* lb, const float* A,
                 const float* acc, int32_t clip, int32_t branch_sb,
                 float* lo_xl, float* lo_xh, float* hi_xl, float* hi_xh,
                 int64_t* counters, void* stream);

/* vcb_bab_step for any input width (n_in > 64 included, e.g. 3072): one CTA
 * per leaf with fixed-order block reductions, then a scan and the child
 * writes -- the same decisions, counters and child order.  workspace: at
 * least vcb_bab_step_wide_workspace(B, n_in) bytes of device memory. */
int vcb_bab_step_wide(int32_t B, int32_t n_in, int32_t Q, int32_t D,
                      int32_t q_sens, const int32_t* query_disjunct,
                      const float* xl, const float* xh, const float* lb,
                      const float* A, const float* acc, int32_t clip,
                      int32_t branch_sb, float* lo_xl, float* lo_xh,
                      float* hi_xl, float* hi_xh, int64_t* counters,
                      void* workspace, size_t workspace_bytes, void* stream);

size_t vcb_bab_step_wide_workspace(int32_t B, int32_t n_in);

/* Branching and clipping settings of the input-split step, the settings keys
 * the reference driver reads in its branching block (verify_graph.py:
 * 13036-13423, settings.py:340-368, 1364). */
typedef struct vcb_bab_opts {
  int32_t clip;          /* input_split_batched_clip_enabled                  */
  int32_t clip_iters;    /* input_split_batched_clip_iters (>= 1)             */
  int32_t branch_sb;     /* SB score (else widest dimension)                  */
  int32_t margin_score;  /* input_split_sb_margin_score                       */
  int32_t split_depth;   /* dimensions split at once this iteration (1..9):   */
                         /* bab_split_depth while the popped batch is below   */
                         /* the batch size, else 1                            */
  float coeff_thresh;    /* input_split_sb_coeff_thresh                       */
  float margin_weight;   /* input_split_sb_margin_weight                      */
  const float* boost;    /* (n_in) device multipliers of the SB score (the    */
                         /* branch boost), or NULL                            */
} vcb_bab_opts;

/* vcb_bab_step / vcb_bab_step_wide with every branching setting, replacing
 * the whole branching block of _input_split_batched_inner (verify_graph.py:
 * 13236-13429): iterated clipping, the SB margin score, the branch boost and
 * K-dimension splits.  For split_depth = 1 the children go to lo_* / hi_*
 * as above; for split_depth = K > 1 each split leaf's K best-scoring
 * dimensions (ties to the lower index) that are wider than 1e-12 are
 * bisected together and its 2^K' children (bit k of the child index set =
 * high half of the k-th dimension) are written leaf by leaf to kid_xl /
 * kid_xh (capacity B * 2^K rows); a leaf with no such dimension counts as
 * degenerate.  counters[2] = child rows written. */
int vcb_bab_step_ex(int32_t B, int32_t n_in, int32_t Q, int32_t D, int32_t q_sens,
                    const int32_t* query_disjunct, const float* xl, const float* xh,
                    const float* lb, const float* A, const float* acc,
                    const vcb_bab_opts* opts, float* lo_xl, float* lo_xh, float* hi_xl,
                    float* hi_xh, float* kid_xl, float* kid_xh, int64_t* counters,
                    void* stream);

int vcb_bab_step_wide_ex(int32_t B, int32_t n_in, int32_t Q, int32_t D, int32_t q_sens,
                         const int32_t* query_disjunct, const float* xl, const float* xh,
                         const float* lb, const float* A, const float* acc,
                         const vcb_bab_opts* opts, float* lo_xl, float* lo_xh,
                         float* hi_xl, float* hi_xh, float* kid_xl, float* kid_xh,
                         int64_t* counters, void* workspace, size_t workspace_bytes,
                         void* stream);

/* Batched sign-gradient PGD for ReLU MLPs (widths <= 128); replaces the loop
 * of _simple_pgd / _simple_pgd_batched (src/vibecheck/verify_hybrid_acasxu.py:
 * 39, 103).
 *
 *   x (N, n_in)    samples, updated in place; sample s belongs to box s / R
 *                  of lo/hi ((N / R), n_in).
 *   C (ncon, n_out), cb (ncon): margin rows; cdis (ncon) disjunct of each
 *                  (0..D-1).  loss = min_d max_{c in d} (C_c . y + cb_c).
 *   best           *best must be initialised to ~0ull; on return it holds
 *                  (iteration << 32 | sample) of the SAT sample (loss <= 1e-6)
 *                  the reference's loop would return first, or stays ~0ull.
 *                  That sample's row of x is the witness.
 */
int vcb_mlp_pgd(const vcb_mlp* net, int32_t N, int32_t R, float* x,
                const float* lo, const float* hi, int32_t ncon,
                const float* C, const float* cb, const int32_t* cdis,
                int32_t D, int32_t n_iter, float lr,
                unsigned long long* best, void* stream);

/* The restart loop of pgd_attack_general (src/vibecheck/pgd.py:233-524) for
 * ReLU MLPs (widths <= 128), OSI initialisation included, in one launch.
 *
 *   x (N, n_in)      restarts' initial draw, updated in place; sample s
 *                    belongs to box s / R of lo/hi ((N / R), n_in) and is
 *                    restart s % R.
 *   step0            (step_rows, n_in) initial step (eps_input * alpha_frac);
 *                    step_rows = 1 (shared) or R (multi-alpha, one per restart).
 *   w_d (R, n_out)   OSI projections; n_osi sign-ascent steps on w_r . f(x)
 *                    with step0 before the loop (n_osi = 0: uniform init).
 *   optim            0 sign_sgd, 1 adam_sign, 2 adam_clipping (_PGDOptim).
 *   lr_decay, hinge  step decay per iteration; hinge-loss clamp threshold
 *                    (margins compare with its float32 value, the plateau
 *                    rule with the double).
 *   plateau          pgd_plateau_iters; applied in the kernel when all R
 *                    restarts fit one tile (R <= 64), else only recorded.
 *   inv_bc1, inv_sbc2 (n_iter): float32 reciprocals of (1 - 0.9^t) and
 *                    sqrt(1 - 0.999^t), t = 1..n_iter, as the GPU's
 *                    scalar-divisor rounds them.
 *   C, cb, cdis      margin rows (margin > 0 = safe), each row's disjunct
 *                    0..D-1; cact the row's ordinal among the attacked
 *                    disjuncts (0..n_act-1) or -1 for a disjunct that is
 *                    only checked (restrict_disj).
 *   per_restart_disj restart r descends only attacked disjunct r % n_act.
 *   confirm_thr      spec.check's unsat_margin_bloat.
 *   budget_ns        wall-time budget of the loop (0 = none).
 *   best             init ~0ull; (screen << 32 | sample) of the first
 *                    confirmed witness (screens 1..n_iter precede the updates,
 *                    n_iter + 1 is the final check); that row of x is it.
 *   gmin (n_iter+2)  init 0xffffffff; per screen the minimum attacked margin
 *                    over all restarts, order-encoded (u >= 2^31: u - 2^31 is
 *                    the bits of a non-negative float; else ~u the bits of a
 *                    negative one) -- the host replays the plateau give-up.
 *   t_stop           init INT32_MAX; the screen at which the budget ran out.
 */
int vcb_mlp_pgd_general(const vcb_mlp* net, int32_t N, int32_t R, float* x,
                        const float* lo, const float* hi, const float* step0,
                        int32_t step_rows, const float* w_d, int32_t n_osi,
                        int32_t n_iter, int32_t optim, float lr_decay,
                        double hinge, int32_t plateau, const float* inv_bc1,
                        const float* inv_sbc2, int32_t ncon, const float* C,
                        const float* cb, const int32_t* cdis,
                        const int32_t* cact, int32_t D, int32_t n_act,
                        int32_t per_restart_disj, double confirm_thr,
                        unsigned long long budget_ns,
                        unsigned long long* best, uint32_t* gmin,
                        int32_t* t_stop, void* stream);

/* Per-iteration pieces of both PGD attacks for networks outside the
 * shared-memory kernels (the forward / backward passes then run on the
 * layer kernels below).
 *
 * vcb_pgd_screen: y (N, n_out, ld ldy) the network outputs of screen t.
 *   simple = 1 (_simple_pgd): loss_s = min_d max_{c in d} margin; SAT at
 *     <= 1e-6 -> atomicMin(best, t << 32 | s); g row = C[routed row].
 *   simple = 0 (pgd_attack_general): candidate = some attacked margin <= 0,
 *     confirmed when a disjunct has every margin <= confirm_thr ->
 *     atomicMin(best, t << 32 | s); *gmin_t = order-encoded minimum attacked
 *     margin (as vcb_mlp_pgd_general's gmin); g row = sum of the attacked rows
 *     with margin >= hinge (restart s % R's disjunct only when
 *     per_restart_disj).
 * vcb_pgd_step: x (N, n_in) in place, box s / R of lo/hi; g (ld ldg) the
 *   input gradient.  mode 0: _PGDOptim step (optim 0/1/2 as above, Adam
 *   state m1/m2 and decayed step cur (N, n_in), sc1 / sc2 this iteration's
 *   reciprocal bias corrections) then cur *= decay; mode 1: OSI ascent
 *   x + step0 * sign(g); mode 2: _simple_pgd's x - lr * sign(g) * (hi - lo).
 *   Every mode clamps x to its box. */
int vcb_pgd_screen(int32_t N, int32_t n_out, const float* y, int32_t ldy,
                   int32_t ncon, const float* C, const float* cb,
                   const int32_t* cdis, const int32_t* cact, int32_t D,
                   int32_t n_act, int32_t per_restart_disj, int32_t R,
                   int32_t simple, float hinge, double confirm_thr, int32_t t,
                   unsigned long long* best, uint32_t* gmin_t, float* g,
                   int32_t ldg, void* stream);

int vcb_pgd_step(int32_t N, int32_t R, int32_t n_in, float* x, const float* lo,
                 const float* hi, const float* g, int32_t ldg, int32_t mode,
                 int32_t optim, int32_t t, const float* step0,
                 int32_t step_rows, float* cur, float* m1, float* m2,
                 float sc1, float sc2, float decay, float lr, void* stream);

/* ---- layer-wise kernels (networks too wide for the shared-memory path,
 * and convolutional networks).  All row-major buffers are float32; "ld"
 * arguments are leading dimensions in elements.  They replace, one layer at a
 * time, the fc / conv / relu branches of _ibp_forward_graph_batched
 * (src/vibecheck/verify_zono_bnb.py:1093-1152) and of
 * _spec_backward_graph_batched (:4379-4593), and the autograd pass of the
 * alpha-CROWN loops (:5248-5288, verify_milp.py:2785-2807). ---- */

/* IBP fc layer: mid/rad (D x nin, ld lda, lda % 4 == 0) times W^T / |W|^T
 * (W: nout x nin) plus b; clamps (D x nout) or NULL; writes the
 * pre-activation bounds sb_lo/hi (D x nout) and, if mid_o is non-NULL, the
 * relu'd mid/rad (D x ldo). */
int vcb_wide_ibp_layer(int32_t D, int32_t nin, int32_t nout, const float* mid,
                       const float* rad, int32_t lda, const float* W,
                       const float* Wabs, const float* b, const float* clo,
                       const float* chi, float* sb_lo, float* sb_hi,
                       float* mid_o, float* rad_o, int32_t ldo, void* stream);

/* CROWN fc step: coef (R x nout, ld ldc) times Waug = [W | b] (nout x
 * (nin+1), ld ldw) -> coef_o (R x nin, ld ldo >= nin+1) and the bias dot bd
 * (R).  With sb_lo/hi ((R/Q) x nin, the bounds of the relu feeding this fc)
 * the relu relaxation (alpha / beta optional, (R/Q) x nin; with alpha_rows
 * alpha is R x nin, one per spec row: the reference's (B, Q, n) form,
 * verify_zono_bnb.py:4423) is applied, the raw coefficients are written to
 * rec (R x ldo) when non-NULL and intercept partial sums to part (R x
 * vcb_wide_back_parts(R, nin)). */
int vcb_wide_back_layer(int32_t R, int32_t Q, int32_t nin, int32_t nout,
                        const float* coef, int32_t ldc, const float* Waug,
                        int32_t ldw, const float* sb_lo, const float* sb_hi,
                        const float* alpha, int32_t alpha_rows, const float* beta,
                        float* coef_o, float* rec, int32_t ldo, float* bd,
                        float* part, void* stream);
int vcb_wide_back_parts(int32_t R, int32_t nin);

/* acc[r] = (acc[r] + bd[r]) + sum_t part[r][t] (if with_part), fixed order. */
int vcb_wide_rowsum(int32_t R, int32_t nparts, int32_t with_part,
                    const float* bd, const float* part, float* acc,
                    void* stream);

/* lb[r] = acc[r] + sum pos(e) xl[r/Q] + sum neg(e) xh[r/Q] over the n0 input
 * coefficients e (R x n0, ld lde); optional A copy (R x n0) and adjoint seed
 * g0 (R x lde) = xl [e >= 0] + xh [e <= 0]. */
int vcb_wide_concretize(int32_t R, int32_t Q, int32_t n0, int32_t lde,
                        const float* e, const float* acc, const float* xl,
                        const float* xh, float* lb, float* A, float* g0,
                        void* stream);

/* alpha adjoint fc step: ga = g (R x nin, ld ldg) W^T + b; with rec (R x
 * nout, ld ldo), the raw coefficients entering relu layer L's relaxation,
 * writes g_o (the adjoint before that relu), dcontrib (per-row alpha
 * gradient, [unstable] max(e,0) ga) and, if non-NULL, dbeta (per-row gradient
 * with respect to the split multiplier beta added after the relaxation: ga). */
int vcb_wide_adjoint_layer(int32_t R, int32_t Q, int32_t nin, int32_t nout,
                           const float* g, int32_t ldg, const float* W,
                           const float* b, const float* rec,
                           const float* sb_lo, const float* sb_hi,
                           const float* alpha, int32_t alpha_rows, float* g_o,
                           float* dcontrib, float* dbeta, int32_t ldo, void* stream);

/* Adam (betas 0.9/0.999, eps 1e-8, as torch.optim.Adam) step `step` on the
 * loss -sum(lb): gradient = -sum over the Q rows of each domain of dcontrib;
 * alpha, m1, m2 (D x n) updated in place; alpha clamped to [0, 1]. */
int vcb_wide_alpha_adam(int32_t D, int32_t Q, int32_t n, int32_t ldc,
                        const float* dcontrib, float* alpha, float* m1,
                        float* m2, float lr, int32_t step, void* stream);

/* Convolution geometry arrays are int32[12] on the host:
 * {C, H, W, C_out, H_out, W_out, kh, kw, stride_h, stride_w, pad_h, pad_w}. */

/* IBP conv layer (NCHW, D boxes): lo/hi = conv(mid, K) + b -/+ conv(rad, |K|). */
int vcb_conv_ibp(int32_t D, const int32_t* geometry, const float* mid,
                 const float* rad, const float* K, const float* Kabs,
                 const float* b, float* lo, float* hi, void* stream);

/* CROWN conv step: e_in (R x C x H x W) = conv_transpose(e (R x C_out x H_out
 * x W_out), K) -- the adjoint of the convolution.  workspace: device scratch
 * of at least vcb_conv_back_workspace(R, geometry) bytes (the per-tap
 * products, R Ho Wo C kh kw floats). */
int vcb_conv_back(int32_t R, const int32_t* geometry, const float* e,
                  const float* K, float* e_in, void* workspace,
                  size_t workspace_bytes, void* stream);

/* Scratch bytes vcb_conv_back / vcb_conv_backward need for R rows. */
size_t vcb_conv_back_workspace(int32_t R, const int32_t* geometry);

/* bd[r] = sum_{c, p} e[r][c][p] b[c] (conv bias dot, e: R x Co x hw). */
int vcb_conv_bias_dot(int32_t R, int32_t Co, int32_t hw, const float* e,
                      const float* b, float* bd, void* stream);

/* IBP relu: clamps (or NULL), crossing repair, sb out, relu'd mid/rad (D x ldo). */
int vcb_ibp_relu(int32_t D, int32_t n, const float* lo, const float* hi,
                 const float* clo, const float* chi, float* sb_lo,
                 float* sb_hi, float* mid, float* rad, int32_t ldo,
                 void* stream);

/* CROWN relu relaxation of coefficient rows e (R x n, ld lde) -> e_out (ld
 * ldo) with the bounds of box r/Q (alpha / beta optional); part[r] = sum of
 * min(e, 0) * up_t. */
int vcb_relu_back(int32_t R, int32_t Q, int32_t n, const float* e,
                  int32_t lde, float* e_out, int32_t ldo, const float* sb_lo,
                  const float* sb_hi, const float* alpha, const float* beta,
                  float* part, void* stream);

/* ---- concrete (point) evaluation: the fc / conv / relu branches of
 * _forward_batch_graph (src/vibecheck/verify_zono_bnb.py:554-770) and their
 * vector-Jacobian products (the autograd backward of PGD's loss,
 * src/vibecheck/pgd.py:494, verify_hybrid_acasxu.py:155). ---- */

/* z = x W^T + b for N points (x: N x nin, ld ldx; W: nout x nin); writes the
 * pre-activation z (ld ldz) and / or relu(z) a (ld lda); either may be NULL,
 * not both. */
int vcb_fc_forward(int32_t N, int32_t nin, int32_t nout, const float* x,
                   int32_t ldx, const float* W, const float* b, float* z,
                   int32_t ldz, float* a, int32_t lda, void* stream);

/* g_o (N x nin, ld ldo) = g (N x nout, ld ldg) W, zeroed where mask (the
 * pre-activation feeding this fc's input ReLU, ld ldm) is <= 0; mask NULL =
 * no ReLU before the fc. */
int vcb_fc_backward(int32_t N, int32_t nin, int32_t nout, const float* g,
                    int32_t ldg, const float* W, const float* mask,
                    int32_t ldm, float* g_o, int32_t ldo, void* stream);

/* Conv forward (NCHW): z = conv(x, K) + b, a = relu(z); either may be NULL. */
int vcb_conv_forward(int32_t N, const int32_t* geometry, const float* x,
                     const float* K, const float* b, float* z, float* a,
                     void* stream);

/* Conv vector-Jacobian product: g_in (N x C x H x W) = conv_transpose(g, K),
 * zeroed where mask (same shape as g_in, or NULL) is <= 0; workspace as for
 * vcb_conv_back. */
int vcb_conv_backward(int32_t N, const int32_t* geometry, const float* g,
                      const float* K, const float* mask, float* g_in,
                      void* workspace, size_t workspace_bytes, void* stream);

/* ---- fp32 GEMM on the tcgen05 tensor cores with error-compensated 3xTF32
 * (the contraction of the wide layers; no single reference counterpart --
 * it replaces the fp32 matmuls / einsums inside the functions above). ---- */

/* hi = x rounded to TF32 (nearest), lo = x - hi, elementwise over n floats. */
int vcb_tf32_split(int64_t n, const float* x, float* hi, float* lo,
                   void* stream);

/* C (M x N, ld ldc) = A B^T (+ bias[n]) with A (M x K, ld lda) and B (N x K,
 * ld ldb) given as split pairs (vcb_tf32_split); every operand 16-byte
 * aligned with ld % 4 == 0.  err: device int32, 0 on entry; set to 1 when a
 * bounded pipeline wait expired (then C is not valid). */
int vcb_tc_gemm(int32_t M, int32_t N, int32_t K, const float* A_hi,
                const float* A_lo, int32_t lda, const float* B_hi,
                const float* B_lo, int32_t ldb, const float* bias, float* C,
                int32_t ldc, int32_t* err, void* stream);

/* vcb_tc_gemm with a device gate: when *gate == 0 (gate non-NULL) the launch
 * returns without touching C, so a host can queue work that the device
 * decides to skip (the alpha-CROWN loop's stop test). */
int vcb_tc_gemm_gated(int32_t M, int32_t N, int32_t K, const float* A_hi,
                      const float* A_lo, int32_t lda, const float* B_hi,
                      const float* B_lo, int32_t ldb, const float* bias, float* C,
                      int32_t ldc, int32_t* err, const int32_t* gate, void* stream);

/* ---- Tensor-core alpha-CROWN loop for wide MLPs (the Adam loop of
 * _ibp_crown_bab, src/vibecheck/verify_milp.py:2762-2807, and
 * _run_alpha_crown_inputsplit_batched, verify_zono_bnb.py:5248-5288).  Each
 * layer is one 3xTF32 GEMM (operands as vcb_tf32_split pairs, 16-byte
 * aligned, ld % 4 == 0) whose epilogue does the layer's bound arithmetic and
 * writes the next GEMM's operand as a TF32 hi / lo pair.  R = D domains x Q
 * spec rows; row r belongs to domain r / Q and per-domain arrays are D x N.
 * Row sums leave as one partial per 64-column group, at part[r * ldpart +
 * part0 + n / 64].  Every call takes an optional device gate and does
 * nothing when *gate == 0; err as for vcb_tc_gemm. ---- */

/* Relaxation records of one ReLU layer from its bounds (n = D x width
 * neurons): rx (n x 2 floats, 8-byte aligned) = (upper slope, negated on
 * stable neurons; intercept factor) and pos = the lower slope (1 active, 0
 * dead, the min-area choice on unstable neurons: the alpha init, which the
 * Adam steps then move on unstable neurons only). */
int vcb_wtc_relax_init(int64_t n, const float* sb_lo, const float* sb_hi, float* rx,
                       float* pos, const int32_t* gate, void* stream);

/* Back-substitution through one layer: C = A B^T (R x N; A = coef (R x K),
 * B = W^T (N x K)) kept as the record; coef_o = relaxation of the ReLU below
 * (pos / rx from vcb_wtc_relax_init, D x N) + beta (or NULL), split into
 * out_hi / out_lo; partials = intercept sum + coef_o . b_next (b_next (N) or
 * NULL). */
int vcb_wtc_back_gemm(int32_t R, int32_t Q, int32_t N, int32_t K, const float* A_hi,
                      const float* A_lo, int32_t lda, const float* B_hi,
                      const float* B_lo, int32_t ldb, float* C, int32_t ldc,
                      const float* pos, const float* rx,
                      const float* beta, const float* b_next, float* out_hi,
                      float* out_lo, int32_t ldo, float* part, int32_t ldpart,
                      int32_t part0, int32_t* err, const int32_t* gate, void* stream);

/* Input layer: e = A B^T (R x N, N = input width) -> partials sum(e+ xl +
 * e- xh) over the domain's box (xl, xh: D x N) and the adjoint seed xl [e >=
 * 0] + xh [e <= 0] split into g_hi / g_lo. */
int vcb_wtc_input_gemm(int32_t R, int32_t Q, int32_t N, int32_t K, const float* A_hi,
                       const float* A_lo, int32_t lda, const float* B_hi,
                       const float* B_lo, int32_t ldb, const float* xl, const float* xh,
                       float* g_hi, float* g_lo, int32_t ldg, float* part,
                       int32_t ldpart, int32_t part0, int32_t* err,
                       const int32_t* gate, void* stream);

/* Adjoint through one layer: ga = A B^T + bias (A = g (R x K), B = W (N x
 * K)); with the record rec (R x N: the C that entered this ReLU's
 * relaxation) and the relaxation pos / rx: dcontrib = [unstable] max(e, 0) ga (R x N, ld ldd) and the
 * next adjoint [e >= 0] pos ga + [e <= 0] (neg ga + icp) split into g_hi /
 * g_lo (or NULL). */
int vcb_wtc_adj_gemm(int32_t R, int32_t Q, int32_t N, int32_t K, const float* A_hi,
                     const float* A_lo, int32_t lda, const float* B_hi, const float* B_lo,
                     int32_t ldb, const float* bias, const float* rec, int32_t ldrec,
                     const float* pos, const float* rx,
                     float* dcontrib, int32_t ldd, float* g_hi, float* g_lo, int32_t ldg,
                     int32_t* err, const int32_t* gate, void* stream);

/* lb[r] = acc0[r] + part[r][0] + ... + part[r][nparts - 1] (in order); best =
 * lb (first) or the NaN-propagating max(best, lb) (best may be NULL);
 * *open_flag = 1 when some best <= 0. */
int vcb_wtc_finish(int32_t R, const float* acc0, const float* part, int32_t ldpart,
                   int32_t nparts, float* lb, float* best, int32_t first,
                   int32_t* open_flag, const int32_t* gate, void* stream);

/* d(sum lb)/d(alpha) = sum over each domain's Q rows of dcontrib (rows in
 * order), then one Adam step (torch defaults; step number `step`, learning
 * rate lr) on -sum(lb) for alpha / m1 / m2 (D x n) and the clamp to [0, 1]. */
int vcb_wtc_adam(int32_t D, int32_t Q, int32_t n, const float* dcontrib, int32_t ldd,
                 float* alpha, float* m1, float* m2, float lr, int32_t step,
                 const int32_t* gate, void* stream);

/* ---- DeepZ zonotope for wide MLPs (_forward_zonotope_graph_batched,
 * src/vibecheck/verify_zono_bnb.py:3079-4074, layer by layer).  Generators
 * are generator-major rows: leaf b owns rows [off[b], off[b+1]) of one
 * (rows x ld) matrix, the first k[b] meaningful, the rest zero; one fc layer
 * of the whole batch is then one vcb_tc_gemm. ---- */

/* ReLU transformer per leaf (B x n): lambda, mu (:3175-3211), c_out = lambda c
 * + mu, cnt[b] = unstable count, idx_of_rank (B x n): leaf b's unstable
 * neurons in index order (first cnt[b] entries). */
int vcb_zw_relu(int32_t B, int32_t n, const float* c, const float* lo,
                const float* hi, float* lam, float* mu, float* c_out,
                int32_t* cnt, int32_t* idx_of_rank, void* stream);

/* Next layer's A operand (TF32 hi / lo, ld ld): leaf b's k_in[b] generator
 * rows scaled column-wise by lambda -- from C (ld ldc) at in_off[b], or, when
 * C is NULL (layer 0), r[b][k] W0T[k] (W0T: n0 x n, the first fc transposed)
 * -- then one row mu_j e_j per unstable neuron, zero rows up to out_off[b+1].
 * rows_hint: out_off[B] (sizes the grid). */
int vcb_zw_build(int32_t B, int32_t n, int32_t ld, const int64_t* in_off,
                 const int32_t* k_in, const float* C, int32_t ldc,
                 const float* r, int32_t n0, const float* W0T,
                 const float* lam, const float* mu, const int32_t* cnt,
                 const int32_t* idx_of_rank, const int64_t* out_off,
                 int64_t rows_hint, float* A_hi, float* A_lo, void* stream);

/* lo / hi (B x n) = c -+ sum over leaf b's first k[b] rows of |C|:
 * compensated sums over 128-row chunks (chunk_off (B+1): prefix of the
 * per-leaf chunk counts ceil(k[b] / 128), max_chunks their maximum), then over
 * a leaf's chunks in order.  workspace: vcb_zw_colsum_workspace(chunk_off[B],
 * n) bytes. */
int vcb_zw_colsum(int32_t B, int32_t n, const int64_t* off, const int32_t* k,
                  const int64_t* chunk_off, int32_t max_chunks, const float* C,
                  int32_t ldc, const float* c, float* lo, float* hi,
                  void* workspace, size_t workspace_bytes, void* stream);

size_t vcb_zw_colsum_workspace(int64_t total_chunks, int32_t n);

/* Diagnostic: FP32 FFMA throughput probe (no reference counterpart).  Runs
 * `blocks` CTAs of 256 threads, each thread `iters` x 64 dependent-chain FMAs
 * (8 independent chains); FLOPs = blocks * 256 * iters * 128.  `out` must
 * hold blocks*256 floats and is written only in a never-taken branch. */
int vcb_probe_ffma(float* out, int32_t blocks, int32_t iters, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* VCB_H */
