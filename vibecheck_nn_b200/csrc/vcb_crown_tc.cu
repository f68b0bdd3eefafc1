// Fused IBP forward + CROWN back-substitution on the 5th-generation tensor
// cores, for ReLU MLPs whose input and hidden widths are at most 63 (the
// ACAS-Xu-sized networks of the batched BaB).  Same contract and results, to
// fp32 rounding, as crown_mlp_kernel; vcb_mlp_crown routes large batches here.
//
// Every contraction is a 128-row tcgen05.mma (kind::tf32) with error-
// compensated 3xTF32 operands: both operands split into TF32 hi and lo parts
// (each rounded to nearest); hi_A hi_B goes to one tensor-memory accumulator
// and the corrections lo_A hi_B + hi_A lo_B to a second, added by the
// epilogue with a round-to-nearest fp32 add.  A tf32 MMA of 128 rows takes
// the same time for every N up to 128 (measured on B200: about 64 cycles), so
// each K step is two MMAs: hi_A against the 128 rows [hi_B; lo_B] (both
// accumulators at once) and lo_A against hi_B.  The tensor cores' fp32
// accumulation truncates inside each K = 8 step, so results carry about twice
// the rounding noise of an fp32 dot product (fp32-class, not bit-parity with
// the SIMT kernel).
//   * IBP forward (verify_zono_bnb.py:1066-1153), one tile = 128 boxes:
//     per fc layer  mid' = mid W^T  and  rad' = rad |W|^T  with the boxes as
//     rows; the epilogue adds the bias, applies the clamps / crossing repair,
//     writes the CROWN slopes (verify_zono_bnb.py:503-522) and forms the
//     next layer's operands.
//   * CROWN back-substitution (verify_zono_bnb.py:4270-5134): one chain of
//     GEMMs per spec row q, rows = the tile's 128 boxes, coefficients
//     ew' = relax(ew) W with the layer bias as an extra column of W^T (its
//     column of the product is the bias dot); two chains run interleaved, so
//     the tensor cores work on one chain while the epilogue relaxes the
//     other.  The first step, spec row times the last layer, is the same for
//     every box and is computed once per CTA.
//   * Concretisation against the input box; optional A / acc outputs.
//
// Operands: the activations / coefficients (A) live in tensor memory, written
// by the epilogue with tcgen05.st as tf32 hi / lo parts, in two slots (slot 0
// = chain 0 / forward mid, slot 1 = chain 1 / forward rad); the weights (B)
// are pre-split, pre-swizzled 64 x 64 images (W, |W| and [W^T; b] per layer,
// built by crown_tc_images into the workspace; per 32-column K block the 64
// hi rows, then the 64 lo rows) streamed through a 4-stage
// shared-memory ring by one bulk copy each.  Tensor memory (512 columns): A
// of slot s at 128 s (hi) and 128 s + 64 (lo), its accumulators at
// 256 + 128 s (hi_A hi_B) and 256 + 128 s + 64 (corrections).
//
// Warps: 0-15 epilogue (warp w reads tensor-memory lanes 32 (w % 4) ..
// 32 (w % 4) + 31, i.e. boxes of the tile, and the 16-column chunk 16 (w /
// 4)), warp 16 loads the weights and issues the MMAs (17 warps leave 96
// registers per thread; the extra warps hide more tensor-memory and L2
// latency than the few spilled registers cost).  The ReLU slopes of a tile go
// to the CTA's workspace slot in neuron-major order ([layer][neuron][box],
// coalesced across a warp) and are read back by the thread that wrote them.
// Every wait is bounded; on expiry the kernel stops, writes NaN to the lower
// bounds (and A / acc / sb outputs) of every box it had not finished -- a NaN
// bound proves nothing -- and sets the workspace error word.
#include <algorithm>
#include <atomic>
#include <type_traits>

#include "vcb_common.cuh"
#include "vcb_crown_tc.cuh"
#include "vcb_relu.cuh"
#include "vcb_tcgen05.cuh"

namespace vcb {
namespace {

using namespace tc5;

// Set by crown_tc_kernel when a bounded wait expired (its unfinished boxes
// got NaN bounds); read and cleared by vcb_fault_check.
__device__ int g_tc_fault;

constexpr int kTB = 128;                   // boxes per tile (MMA rows)
constexpr int kEpi = 16;                   // epilogue warps
constexpr int kCtlWarp = kEpi;             // weight loads + MMA issue
constexpr int kThreads = (kEpi + 1) * 32;  // 544
constexpr int kW = 64;                     // padded operand width
constexpr int kMaxWidth = 63;              // widest hidden / input layer
constexpr int kBlk = kW * 128;             // 8 KB: 64 rows x 32 tf32 (one swizzle column)
constexpr int kKBlk = 2 * kBlk;            // 16 KB: hi rows then lo rows of one K block
constexpr int kImg = 2 * kKBlk;            // a 64 x 64 image, hi + lo
constexpr int kStages = 4;
constexpr int kMaxQ = 16;
constexpr unsigned kSpin = 1u << 24;
constexpr unsigned kSpinSleep = 1u << 20;  // polls of at most ~1 us each
constexpr int kSmem = 1024 + kStages * kImg + (kMaxQ * kW + VCB_MAX_FC * kW + 2 * 2 * 4 * kTB) * 4;
// Half-width of the band around the min-area threshold (lower slope 1 iff
// up_s > 0.5, verify_zono_bnb.py:516) inside which a box's bounds are
// recomputed by crown_tie_kernel.  The tensor cores' IBP bounds differ from
// the fp32 reference's sequential dot products by rounding; on the cfg2
// workload (8 seeds of 65,536 boxes) their upper slopes near 0.5 differ by at
// most 1.1e-6, so a slope further than this from 0.5 takes the reference's
// decision (no box of those seeds changes its decision outside the band;
// about 0.5 % of the boxes are inside it).
constexpr float kTieBand = 4e-6f;

// Row pitch of crown_tie_kernel's network image (floats): covers the bias
// column and a whole number of 16-float blocks, a multiple of 4 with an odd
// number of 16-byte words; rows are padded to a multiple of 8.
__host__ __device__ inline int tie_pitch(int nin) {
  const int need = max(nin + 1, (nin + 15) & ~15);
  return 4 * ((need + 3) / 4 | 1);
}
__host__ __device__ inline int tie_rows(int nout) { return (nout + 7) & ~7; }

// Batches of the input-split BaB (<= 4096 boxes) stay on the SIMT kernel, whose
// rounding the leaf-count parity of the BaB tests is pinned to.
std::atomic<int> g_min_batch{16384};

struct TcParams {
  int n_fc;
  int dims[VCB_MAX_FC + 1];
  const float* W;
  const float* b;
  long long w_goff[VCB_MAX_FC];
  int b_goff[VCB_MAX_FC];
  long long relu_goff[VCB_MAX_FC];
  int sl_off[VCB_MAX_FC];  // float2 offset of relu layer L in a slot
  long long slot_f2;       // float2 per CTA slot
  const uint8_t* img;      // (n_fc - 1) x 3 images of kImg bytes
  int B, Q, ntiles, npass;
  int split_tail;          // the last, partial round's tiles are split by pass (see item_at)
  const float *xl, *xh, *clo, *chi, *sblo, *sbhi, *alpha, *beta, *specW, *specb;
  float *lb, *A, *accout, *sbolo, *sbohi;
  float2* slopes;
  int* err;
  // near-tie re-bound (crown_tie_kernel): on when the kernel computes the IBP
  // bounds itself with the min-area lower slope (no caller bounds, no alpha)
  int tie_on;
  int* tie_flag;          // (B) the box is listed
  int* tie_list;          // boxes with an unstable neuron inside the band, each once
  int* tie_count;
  float* tnet;            // the row images of crown_tie_kernel (see there)
  int tsoff[VCB_MAX_FC];  // fc layer l: tie_rows(dims[l+1]) rows of pitch tpitch[l]
  int tpitch[VCB_MAX_FC];
  int tnet_floats;
};

// Work items of this CTA.  Item i < full is tile i * gridDim.x + blockIdx.x
// with every spec-row pass.  The rem tiles of the last, partial round either
// go whole to CTAs 0 .. rem-1, or (split_tail, 2 rem <= gridDim.x) each to
// two CTAs, b and b + rem, that recompute the forward and take the first and
// second half of the passes: the round then costs a forward and half the
// passes instead of a whole tile while the other CTAs idle.
struct TcItem {
  int tile, pass_lo, pass_hi;
};

__device__ __forceinline__ int items_of(const TcParams& p) {
  const int g = gridDim.x, b = blockIdx.x;
  const int full = p.ntiles / g, rem = p.ntiles - full * g;
  return full + (b < (p.split_tail ? 2 * rem : rem) ? 1 : 0);
}

__device__ __forceinline__ TcItem item_at(const TcParams& p, int i) {
  const int g = gridDim.x, b = blockIdx.x;
  const int full = p.ntiles / g, rem = p.ntiles - full * g;
  if (i < full || !p.split_tail) return TcItem{i * g + b, 0, p.npass};
  const int half = b / rem, hp = (p.npass + 1) / 2;
  return TcItem{full * g + b % rem, half * hp, min(p.npass, (half + 1) * hp)};
}

// Weight images, one thread per (image, row, k); thread 0 also clears the
// error word.  Image 3 l + 0: W_l
// (rows = outputs, K = inputs), + 1: |W_l|, + 2: [W_l^T; b_l] (rows = inputs
// then the bias row, K = outputs).  Each is split into tf32 hi and lo parts,
// laid out per 32-column K block as 128 rows (the 64 hi rows, then the 64 lo
// rows) with the 128-byte swizzle of a K-major tcgen05 operand, so that one
// descriptor covers [hi; lo] as an N = 128 operand and its first 64 rows hi
// alone.
// When the near-tie re-bound is on, the same launch clears the tie flags and
// writes the plain fp32 rows of the network that crown_tie_kernel reads.
__global__ void crown_tc_images(const TcParams p) {
  // crown_tc_kernel may be scheduled now; it waits for this grid's writes
  // (griddepcontrol.wait) before it reads them
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  const int nimg = 3 * (p.n_fc - 1);
  const int idx = blockIdx.x * blockDim.x + threadIdx.x;
  if (idx == 0) {  // the error word and tie count of the launch that follows
    *p.err = 0;
    *p.tie_count = 0;
  }
  if (p.tie_on) {
    if (idx < p.B) p.tie_flag[idx] = 0;
    if (idx < p.tnet_floats) {
      // rows [W_l[o, :], b_l[o], 0 ..], zero rows from dims[l+1] to tie_rows
      int l = 0;
      while (l + 1 < p.n_fc && idx >= p.tsoff[l + 1]) ++l;
      const int nin = p.dims[l], nout = p.dims[l + 1], pitch = p.tpitch[l];
      const int o = (idx - p.tsoff[l]) / pitch, c = (idx - p.tsoff[l]) % pitch;
      float v = 0.f;
      if (o < nout) {
        if (c < nin) v = p.W[p.w_goff[l] + (long long)o * nin + c];
        else if (c == nin) v = p.b[p.b_goff[l] + o];
      }
      p.tnet[idx] = v;
    }
  }
  if (idx >= nimg * kW * kW) return;
  const int im = idx / (kW * kW), n = (idx / kW) % kW, k = idx % kW;
  const int l = im / 3, use = im % 3;
  const int nin = p.dims[l], nout = p.dims[l + 1];
  const float* Wl = p.W + p.w_goff[l];
  float v = 0.f;
  if (use < 2) {
    if (n < nout && k < nin) v = Wl[(long long)n * nin + k];
    if (use == 1) v = fabsf(v);
  } else if (k < nout) {
    if (n < nin) v = Wl[(long long)k * nin + n];
    else if (n == nin) v = p.b[p.b_goff[l] + k];
  }
  uint32_t h, lo;
  tf32_split_rn(v, h, lo);
  const int off = (k >> 5) * kKBlk + (n >> 3) * 1024 + (n & 7) * 128 +
                  ((((k & 31) >> 2) ^ (n & 7)) << 4) + (k & 3) * 4;
  uint8_t* base = const_cast<uint8_t*>(p.img) + (long long)im * kImg;
  *reinterpret_cast<uint32_t*>(base + off) = h;
  *reinterpret_cast<uint32_t*>(base + kBlk + off) = lo;
}

// A B^T over `ksteps` K steps of 8 with 3xTF32: A in tensor memory (hi at
// column a, lo at a + 64), B a weight image in shared memory (16 KB per
// 32-column K block: hi rows, then lo rows); hi_A hi_B into accumulator d,
// hi_A lo_B + lo_A hi_B into d + 64.  Per K step one N = 128 MMA of hi_A
// against [hi_B; lo_B] writes both accumulators, one N = 64 MMA adds lo_A
// hi_B (padding rows of B are zero, so the unused columns stay zero).
__device__ __forceinline__ void gemm_ts(uint32_t d, uint32_t a, uint32_t b, int ksteps) {
  constexpr uint32_t id_both = idesc_tf32(kTB, 2 * kW), id_hi = idesc_tf32(kTB, kW);
  for (int j = 0; j < ksteps; ++j) {
    const uint64_t bd = sw128_desc(b + (uint32_t)((j >> 2) * kKBlk + (j & 3) * 32));
    mma_tf32_ts(d, a + 8 * j, bd, id_both, j > 0 ? 1u : 0u);
    mma_tf32_ts(d + kW, a + kW + 8 * j, bd, id_hi, 1u);
  }
}

// Publish this warp's tensor-memory stores and completed accumulator loads
// to the MMA issuer.
__device__ __forceinline__ void publish(uint64_t* bar) {
  tmem_wait_st();
  fence_before_sync();
  __syncwarp();
  if ((threadIdx.x & 31) == 0) mbar_arrive(bar);
}

__device__ __forceinline__ float2* slot_base(const TcParams& p) {
  return p.slopes + (long long)blockIdx.x * p.slot_f2;
}

// Split NC (4, 8 or 16) finite values and store the hi / lo parts at
// tensor-memory columns taddr and taddr + 64 of this warp's lanes.  The tensor
// cores read only a tf32 operand's top 19 bits (its low 13 bits are ignored:
// measured on B200), so the lo part is stored rounded but unmasked.
template <int NC>
__device__ __forceinline__ void store_operand(uint32_t taddr, const float (&v)[NC]) {
  uint32_t h[NC], l[NC];
#pragma unroll
  for (int j = 0; j < NC; ++j) {
    const uint32_t u = (__float_as_uint(v[j]) + 0x1000u) & 0xFFFFE000u;
    const float r = __fsub_rn(v[j], __uint_as_float(u));
    h[j] = u;
    l[j] = __float_as_uint(r) + 0x1000u;
  }
  if constexpr (NC == 16) {
    tmem_st16(taddr, h);
    tmem_st16(taddr + kW, l);
  } else if constexpr (NC == 8) {
    tmem_st8(taddr, h);
    tmem_st8(taddr + kW, l);
  } else {
    tmem_st4(taddr, h);
    tmem_st4(taddr + kW, l);
  }
}

// Zero hi / lo parts of four columns: the padding of the next MMA's K range
// past a 4-column chunk.
__device__ __forceinline__ void store_zero4(uint32_t taddr) {
  const uint32_t z[4] = {0u, 0u, 0u, 0u};
  tmem_st4(taddr, z);
  tmem_st4(taddr + kW, z);
}

// Sum of the two accumulators (hi_A hi_B and corrections) at tensor-memory
// column taddr and taddr + 64, NC columns.
template <int NC>
__device__ __forceinline__ void load_acc(uint32_t taddr, float (&v)[NC]) {
  uint32_t a[NC], e[NC];
  if constexpr (NC == 16) {
    tmem_ld16(taddr, a);
    tmem_ld16(taddr + kW, e);
  } else if constexpr (NC == 8) {
    tmem_ld8(taddr, a);
    tmem_ld8(taddr + kW, e);
  } else {
    tmem_ld4(taddr, a);
    tmem_ld4(taddr + kW, e);
  }
  tmem_wait_ld(a, e);
#pragma unroll
  for (int j = 0; j < NC; ++j) v[j] = __fadd_rn(__uint_as_float(a[j]), __uint_as_float(e[j]));
}

// encode_slope with CUDA's fast division for up_s = ub / (ub - lb) (within
// 2 ulp): the tensor-core bounds already differ from the fp32 reference by
// rounding, a box whose up_s lies near the 0.5 threshold is listed for the
// exact re-bound, and the upper relaxation moves by ulps of its terms.
// Branch-free: the same records as encode_slope's early returns (active:
// (1, -0); ub_r = 0: up_s = 0, so (-0, 0)) come out of the selects.
__device__ __forceinline__ float2 encode_slope_fast(float lo, float hi) {
  const float ub_r = fmaxf(fmaxf(hi, 0.f), __fadd_rn(lo, 1e-8f));
  const float up_s = __fdividef(ub_r, __fsub_rn(ub_r, lo));
  const float up_t = ub_r == 0.f ? 0.f : __fmul_rn(-lo, up_s);
  const bool active = lo >= 0.f, dead = hi <= 0.f;
  return make_float2(active ? 1.f : (dead ? -up_s : up_s), active ? -0.0f : up_t);
}

using C4 = std::integral_constant<int, 4>;
using C8 = std::integral_constant<int, 8>;
using C16 = std::integral_constant<int, 16>;
using In = std::true_type;    // the chunk lies inside the layer width
using Out = std::false_type;  // it may reach past it (guards on)

// The 16 epilogue warps: warp w owns the tile's boxes 32 (w % 4) + lane
// (tensor-memory lanes) and the 16-column operand chunk 16 (w / 4).  kPlain: no alpha, beta, clamps or sb outputs (the common
// case, without their guards).  Returns false when a wait expired or another
// role failed; then every box of this CTA from the unfinished tile on gets
// NaN outputs.
template <bool kPlain>
__device__ __forceinline__ bool epilogue(const TcParams& p, uint32_t tmem, float2* slot,
                                      const float* sV, const float* sBias,
                                      float* sRow, uint64_t* a_ready, uint64_t* acc_ready,
                                      uint64_t* rows_ready, const volatile int* vfailed) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int qd = warp & 3, gi = warp >> 2;
  const int row = 32 * qd + lane;
  const uint32_t tl = tmem + ((uint32_t)(32 * qd) << 16);
  const int nck = 1;  // chunks of this warp
  auto chunk_c0 = [&](int) { return 16 * gi; };
  const int nfc = p.n_fc, Q = p.Q, n0 = p.dims[0];
  const bool fwd = p.sblo == nullptr;
  unsigned uacc[2] = {0, 0}, urows = 0;
  bool ok = true;
  auto wait_acc = [&](int c) {
    if (!mbar_wait_sleep(&acc_ready[c], uacc[c] & 1, kSpinSleep, vfailed)) return false;
    ++uacc[c];
    fence_after_sync();
    return true;
  };
  const int nitems = items_of(p);
  int it = 0;
  for (; it < nitems; ++it) {
    const TcItem item = item_at(p, it);
    const int tile = item.tile;
    const int box = tile * kTB + row;
    const bool valid = box < p.B;
    const bool full = (tile + 1) * kTB <= p.B;  // every row of the tile is a box
    bool tie = false;
    if (fwd) {
      // ---- layer-0 operands: centre and radius of the box
      for (int k = 0; k < nck; ++k) {
        const int c0 = chunk_c0(k);
        if (c0 >= n0) continue;
        float m[16], r[16];
#pragma unroll
        for (int j = 0; j < 16; ++j) {
          const int i = c0 + j;
          m[j] = r[j] = 0.f;
          if (i < n0 && valid) {
            const float lo = __ldg(p.xl + (long long)box * n0 + i);
            const float hi = __ldg(p.xh + (long long)box * n0 + i);
            m[j] = __fmul_rn(__fadd_rn(lo, hi), 0.5f);
            r[j] = __fmul_rn(__fsub_rn(hi, lo), 0.5f);
          }
        }
        store_operand<16>(tl + c0, m);
        store_operand<16>(tl + 128 + c0, r);
      }
      publish(&a_ready[0]);
      // ---- fc layers 0 .. nfc-2: bounds and slopes of relu layer l
      for (int l = 0; l < nfc - 1; ++l) {
        if (!(ok = wait_acc(0))) break;
        const int nout = p.dims[l + 1];
        const bool last = l == nfc - 2;
        const long long gi0 = p.relu_goff[l] + (long long)box * nout;
        float2* sl = slot + p.sl_off[l] + row;
        bool published = false;
        // one chunk of NC output columns starting at c0 (pad4: zeros in the
        // four columns after it, the rest of the next MMA's K step; IN: every
        // column of the chunk is an output of the layer, no width guards).
        // The next layer's operands are stored and published first; the ReLU
        // slopes, which only the back-substitution reads, follow while the
        // tensor cores run the next layer.
        auto chunk = [&](auto nc, int c0, bool pad4, auto in) {
          constexpr int NC = decltype(nc)::value;
          constexpr bool IN = decltype(in)::value;
          float mc[NC], rc[NC], lo[NC], hi[NC];
          load_acc<NC>(tl + 256 + c0, mc);
          load_acc<NC>(tl + 384 + c0, rc);
          const float* bias = sBias + l * kW + c0;
#pragma unroll
          for (int j = 0; j < NC; ++j) {
            const int o = c0 + j;
            const float mid = __fadd_rn(mc[j], bias[j]);
            lo[j] = __fsub_rn(mid, rc[j]);
            hi[j] = __fadd_rn(mid, rc[j]);
            if (!kPlain && p.clo && valid && (IN || o < nout)) {
              lo[j] = fmaxf(lo[j], __ldg(p.clo + gi0 + o));
              hi[j] = fminf(hi[j], __ldg(p.chi + gi0 + o));
            }
            hi[j] = fmaxf(hi[j], lo[j]);
            const float lc = fmaxf(lo[j], 0.f), hc = fmaxf(hi[j], 0.f);
            mc[j] = (IN || o < nout) ? __fmul_rn(__fadd_rn(lc, hc), 0.5f) : 0.f;
            rc[j] = (IN || o < nout) ? __fmul_rn(__fsub_rn(hc, lc), 0.5f) : 0.f;
          }
          if (!last) {
            store_operand<NC>(tl + c0, mc);
            store_operand<NC>(tl + 128 + c0, rc);
            if (pad4) {
              store_zero4(tl + c0 + NC);
              store_zero4(tl + 128 + c0 + NC);
            }
            publish(&a_ready[0]);
          }
          published = true;
#pragma unroll
          for (int j = 0; j < NC; ++j) {
            const int o = c0 + j;
            if (IN || o < nout) {
              if (!kPlain && p.sbolo && valid) {
                p.sbolo[gi0 + o] = lo[j];
                p.sbohi[gi0 + o] = hi[j];
              }
              const float2 e = encode_slope_fast(lo[j], hi[j]);
              sl[o * kTB] = e;
              // unstable with the upper slope inside the band where rounding
              // can move it across 0.5 (active records have e.x = 1, dead
              // ones e.x <= 0: both are at least 0.5 away)
              tie |= fabsf(__fsub_rn(e.x, 0.5f)) <= kTieBand;
            }
          }
        };
        for (int k = 0; k < nck; ++k) {
          const int c0 = chunk_c0(k);
          if (c0 >= nout) continue;
          if (nout - c0 <= 4) {  // a short tail: 4 columns, then zeros to pad8
            chunk(C4{}, c0, true, Out{});
          } else if (nout - c0 <= 8) {
            chunk(C8{}, c0, false, Out{});
          } else if (nout - c0 >= 16) {
            chunk(C16{}, c0, false, In{});
          } else {
            chunk(C16{}, c0, false, Out{});
          }
        }
        if (!last && !published) publish(&a_ready[0]);
      }
      if (!ok) break;
      // list the box for crown_tie_kernel once (the column warps of a row and
      // the two CTAs of a split tile may all flag it)
      if (tie && valid && p.tie_on && atomicExch(p.tie_flag + box, 1) == 0)
        p.tie_list[atomicAdd(p.tie_count, 1)] = box;
    } else {
      // ---- caller-supplied intermediate bounds: slopes only
      for (int L = 0; L < nfc - 1; ++L) {
        const int n = p.dims[L + 1];
        const long long gi0 = p.relu_goff[L] + (long long)box * n;
        float2* sl = slot + p.sl_off[L] + row;
        for (int k = 0; k < nck; ++k) {
          const int c0 = chunk_c0(k);
          for (int i = c0; i < min(n, c0 + 16); ++i)
            sl[i * kTB] = valid ? encode_slope(__ldg(p.sblo + gi0 + i), __ldg(p.sbhi + gi0 + i))
                                : make_float2(1.f, -0.0f);
        }
      }
    }
    // ---- CROWN back-substitution, spec rows in pairs
    for (int pass = item.pass_lo; ok && pass < item.pass_hi; ++pass) {
      const int nch = min(2, Q - 2 * pass);
      float racc[2] = {0.f, 0.f}, conc[2] = {0.f, 0.f};
      // step l relaxes the product of fc layer l with relu layer l - 1; the
      // first step (l = nfc - 1) takes its product from the spec table
      for (int l = nfc - 1; l >= 0; --l) {
        const int nin = p.dims[l];
        const int L = l - 1;
        const float2* sl = slot + (L >= 0 ? p.sl_off[L] : 0) + row;
        const long long ri = L >= 0 ? p.relu_goff[L] + (long long)box * nin : 0;
        const float* arow = (!kPlain && L >= 0 && p.alpha && valid) ? p.alpha + ri : nullptr;
        const float* brow = (!kPlain && L >= 0 && p.beta && valid) ? p.beta + ri : nullptr;
        for (int c = 0; c < nch; ++c) {
          const int q = 2 * pass + c;
          if (l < nfc - 1 && !(ok = wait_acc(c))) break;
          // one chunk of NC columns starting at c0 (neurons and / or the bias
          // column; IN: neurons only, no width guards)
          auto chunk = [&](auto nc, int c0, auto in) {
            constexpr int NC = decltype(nc)::value;
            constexpr bool IN = decltype(in)::value;
            float v[NC];
            if (l == nfc - 1) {
#pragma unroll
              for (int j = 0; j < NC; ++j) v[j] = sV[q * kW + c0 + j];
            } else {
              load_acc<NC>(tl + 256 + 128 * c + c0, v);
            }
            if (!full && !valid) {
#pragma unroll
              for (int j = 0; j < NC; ++j) v[j] = 0.f;
            }
            const int bc = nin - c0;  // bias column within the chunk
            float bj = 0.f;
            if (!IN && bc < NC) {
#pragma unroll
              for (int j = 0; j < NC; ++j)
                if (j == bc) bj = v[j];
            }
            if (L >= 0) {
              float2 sv[NC];  // slopes, zero beyond the layer width
#pragma unroll
              for (int j = 0; j < NC; ++j)
                sv[j] = (IN || c0 + j < nin) ? sl[(c0 + j) * kTB] : make_float2(0.f, 0.f);
              float pj = 0.f;
#pragma unroll
              for (int j = 0; j < NC; ++j) {
                const float x = v[j];
                if (kPlain) {
                  // slope (0, 0) beyond the layer width gives 0 and no intercept
                  const float pos = sv[j].x > 0.5f ? 1.f : 0.f;
                  const float mlt = x < 0.f ? fabsf(sv[j].x) : pos;
                  v[j] = __fmul_rn(x, mlt);
                  pj = fmaf(fminf(x, 0.f), sv[j].y, pj);
                } else {
                  const int i = c0 + j;
                  v[j] = 0.f;
                  if (IN || i < nin) {
                    const Slope s = decode_slope(sv[j], arow ? arow + i : nullptr);
                    const float mlt = x < 0.f ? s.neg : s.pos;
                    pj = fmaf(fminf(x, 0.f), s.icp, pj);
                    v[j] = __fmul_rn(x, mlt);
                    if (brow) v[j] = __fadd_rn(v[j], __ldg(brow + i));
                  }
                }
              }
              store_operand<NC>(tl + 128 * c + c0, v);
              racc[c] = __fadd_rn(racc[c], __fadd_rn(bj, pj));
            } else {
              // input layer: concretise against the box
              float s1 = 0.f, s2 = 0.f;
              if (valid) {
                for (int i = c0; i < min(nin, c0 + NC); ++i) {
                  float x = 0.f;
#pragma unroll
                  for (int j = 0; j < NC; ++j)
                    if (c0 + j == i) x = v[j];
                  s1 = fmaf(fmaxf(x, 0.f), __ldg(p.xl + (long long)box * n0 + i), s1);
                  s2 = fmaf(fminf(x, 0.f), __ldg(p.xh + (long long)box * n0 + i), s2);
                  if (p.A) p.A[((long long)box * Q + q) * n0 + i] = x;
                }
              }
              racc[c] = __fadd_rn(racc[c], bj);
              conc[c] = __fadd_rn(conc[c], __fadd_rn(s1, s2));
            }
          };
          for (int k = 0; k < nck; ++k) {
            const int c0 = chunk_c0(k);
            if (c0 > nin) continue;  // no neurons and no bias column here
            if (nin + 1 - c0 <= 4) {  // a short tail: 4 columns, then zeros to pad8
              chunk(C4{}, c0, Out{});
              if (L >= 0) store_zero4(tl + 128 * c + c0 + 4);
            } else if (nin + 1 - c0 <= 8) {
              chunk(C8{}, c0, Out{});
            } else if (c0 + 16 <= nin) {
              chunk(C16{}, c0, In{});
            } else {
              chunk(C16{}, c0, Out{});
            }
          }
          if (L >= 0) publish(&a_ready[c]);
        }
        if (!ok) break;
      }
      if (!ok) break;
      // ---- combine the three column warps of every box
      for (int c = 0; c < nch; ++c) {
        sRow[((c * 2 + 0) * 4 + gi) * kTB + row] = racc[c];
        sRow[((c * 2 + 1) * 4 + gi) * kTB + row] = conc[c];
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(rows_ready);
      if (gi == 0) {
        if (!(ok = mbar_wait_sleep(rows_ready, urows & 1, kSpinSleep, vfailed))) break;
        for (int c = 0; c < nch && valid; ++c) {
          const int q = 2 * pass + c;
          const float* ra = sRow + (c * 2 + 0) * 4 * kTB + row;
          const float* co = sRow + (c * 2 + 1) * 4 * kTB + row;
          float a = __ldg(p.specb + q);
          float t = 0.f;
#pragma unroll
          for (int g = 0; g < kEpi / 4; ++g) {
            a = __fadd_rn(a, ra[g * kTB]);
            t = __fadd_rn(t, co[g * kTB]);
          }
          const long long go = (long long)box * Q + q;
          p.lb[go] = __fadd_rn(a, t);
          if (p.accout) p.accout[go] = a;
        }
      }
      ++urows;
    }
    if (!ok) break;
  }
  if (ok) return true;
  // NaN for every box of this CTA from the unfinished tile on
  const float nan = __int_as_float(0x7fffffff);
  for (; it < nitems; ++it) {
    const int box = item_at(p, it).tile * kTB + row;
    if (box >= p.B || gi != 0) continue;
    for (int q = 0; q < Q; ++q) {
      p.lb[(long long)box * Q + q] = nan;
      if (p.accout) p.accout[(long long)box * Q + q] = nan;
      if (p.A)
        for (int i = 0; i < n0; ++i) p.A[((long long)box * Q + q) * n0 + i] = nan;
    }
    if (p.sbolo)
      for (int L = 0; L < nfc - 1; ++L) {
        const int n = p.dims[L + 1];
        for (int i = 0; i < n; ++i) {
          p.sbolo[p.relu_goff[L] + (long long)box * n + i] = nan;
          p.sbohi[p.relu_goff[L] + (long long)box * n + i] = nan;
        }
      }
  }
  return false;
}

template <bool kPlain>
__global__ void __launch_bounds__(kThreads, 1) crown_tc_kernel(const __grid_constant__ TcParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* ring = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  float* sV = reinterpret_cast<float*>(ring + kStages * kImg);  // kMaxQ x kW
  float* sBias = sV + kMaxQ * kW;                               // VCB_MAX_FC x kW
  float* sRow = sBias + VCB_MAX_FC * kW;                        // [chain][kind][chunk][box]
  __shared__ __align__(8) uint64_t w_full[kStages], w_empty[kStages];
  __shared__ __align__(8) uint64_t a_ready[2], acc_ready[2], rows_ready, done;
  __shared__ uint32_t tmem_slot;
  __shared__ int failed;
  volatile int* vfailed = &failed;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nfc = p.n_fc;
  const int Q = p.Q;
  const bool fwd = p.sblo == nullptr;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&w_full[s], 1);
      mbar_init(&w_empty[s], 1);
    }
    for (int c = 0; c < 2; ++c) {
      mbar_init(&a_ready[c], kEpi);
      mbar_init(&acc_ready[c], 1);
    }
    mbar_init(&rows_ready, kEpi);
    mbar_init(&done, 1);
    failed = 0;
    mbar_fence_init();
  }
  for (int idx = threadIdx.x; idx < (nfc - 1) * kW; idx += kThreads) {
    const int l = idx / kW, o = idx % kW;
    sBias[idx] = o < p.dims[l + 1] ? __ldg(p.b + p.b_goff[l] + o) : 0.f;
  }
  {  // spec rows times the last fc layer, bias dot in column dims[nfc - 1]
    const int nprev = p.dims[nfc - 1], nL = p.dims[nfc];
    const float* Wg = p.W + p.w_goff[nfc - 1];
    const float* bg = p.b + p.b_goff[nfc - 1];
    for (int idx = threadIdx.x; idx < Q * kW; idx += kThreads) {
      const int q = idx / kW, c = idx % kW;
      float s = 0.f;
      if (c <= nprev)
        for (int o = 0; o < nL; ++o)
          s = fmaf(__ldg(p.specW + q * nL + o),
                   c < nprev ? __ldg(Wg + (long long)o * nprev + c) : __ldg(bg + o), s);
      sV[idx] = s;
    }
  }
  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_u32(&tmem_slot)),
                 "r"(512));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  fence_before_sync();
  __syncthreads();
  fence_after_sync();
  const uint32_t tmem = tmem_slot;
  // The prologue above reads only the network and the spec; the weight
  // images, the cleared tie flags and error word come from crown_tc_images,
  // launched just before with a programmatic dependency.
  asm volatile("griddepcontrol.wait;" ::: "memory");
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");

  if (warp == kCtlWarp) {
    // ----------------------- control: weight loads and MMA issue (lane 0)
    if (lane == 0) {
      // image sequence of one tile: forward (W_l, |W_l|) for l = 0 .. nfc-2,
      // then per pass [W_l^T; b_l] for l = nfc-2 .. 0
      const unsigned nl = (unsigned)(nfc - 1);
      const unsigned fwdlen = fwd ? 2 * nl : 0;
      const unsigned T = fwdlen + (unsigned)p.npass * nl;
      // image count of this CTA's items (a split item has fewer passes; its
      // images are the first ones of a whole tile's sequence)
      const int nitems = items_of(p);
      unsigned total = 0;
      for (int i = 0; i < nitems; ++i) {
        const TcItem item = item_at(p, i);
        total += fwdlen + (unsigned)(item.pass_hi - item.pass_lo) * nl;
      }
      unsigned issued = 0, used = 0, ua[2] = {0, 0};
      bool ok = true;
      auto image_of = [&](unsigned n) {
        const unsigned t = n % T;
        if (t < fwdlen) return 3 * (t >> 1) + (t & 1);
        return 3 * (nl - 1 - (t - fwdlen) % nl) + 2;
      };
      // keep the ring full; a stage is reloaded once the MMAs reading it completed
      auto refill = [&]() {
        while (issued < total && issued < used + kStages) {
          const int s = issued % kStages;
          if (issued >= kStages &&
              !mbar_wait(&w_empty[s], ((issued / kStages) - 1) & 1, kSpin, vfailed))
            return false;
          mbar_expect_tx(&w_full[s], kImg);
          bulk_load(ring + s * kImg, p.img + (long long)image_of(issued) * kImg, kImg, &w_full[s]);
          ++issued;
        }
        return true;
      };
      auto take = [&](int& s) {
        s = used % kStages;
        if (!mbar_wait(&w_full[s], (used / kStages) & 1, kSpin, vfailed)) return false;
        ++used;
        return true;
      };
      // polled without a suspend hint: this thread issues every MMA, and a
      // late wake-up would delay them all
      auto wait_a = [&](int c) {
        if (!mbar_wait(&a_ready[c], ua[c] & 1, kSpin, vfailed)) return false;
        ++ua[c];
        fence_after_sync();
        return true;
      };
      ok = refill();
      for (int i = 0; ok && i < nitems; ++i) {
        const TcItem item = item_at(p, i);
        if (fwd) {
          for (int l = 0; ok && l < nfc - 1; ++l) {
            int sw, sa;
            if (!(ok = wait_a(0) && take(sw) && take(sa))) break;
            const int ks = (p.dims[l] + 7) >> 3;
            gemm_ts(tmem + 256, tmem, smem_u32(ring + sw * kImg), ks);
            gemm_ts(tmem + 384, tmem + 128, smem_u32(ring + sa * kImg), ks);
            mma_commit(&w_empty[sw]);
            mma_commit(&w_empty[sa]);
            mma_commit(&acc_ready[0]);
            ok = refill();
          }
        }
        for (int pass = item.pass_lo; ok && pass < item.pass_hi; ++pass) {
          for (int l = nfc - 2; ok && l >= 0; --l) {
            int st;
            if (!(ok = take(st))) break;
            const int ks = (p.dims[l + 1] + 7) >> 3;
            for (int c = 0; c < 2 && 2 * pass + c < Q; ++c) {
              if (!(ok = wait_a(c))) break;
              gemm_ts(tmem + 256 + 128 * c, tmem + 128 * c, smem_u32(ring + st * kImg), ks);
              mma_commit(&acc_ready[c]);
            }
            mma_commit(&w_empty[st]);
            if (ok) ok = refill();
          }
        }
      }
      if (!ok) failed = 1;
      // every MMA issued above completes before tensor memory is freed, and
      // every copy issued lands before the CTA exits
      mma_commit(&done);
      if (!mbar_wait(&done, 0, kSpin)) failed = 1;
      for (unsigned k = used; k < issued; ++k)
        if (!mbar_wait(&w_full[k % kStages], (k / kStages) & 1, kSpin)) failed = 1;
    }
  } else {
    // ------------------------------------------------------------ epilogue
    if (!epilogue<kPlain>(p, tmem, slot_base(p), sV, sBias, sRow, a_ready, acc_ready,
                          &rows_ready, vfailed))
      failed = 1;
  }
  fence_before_sync();
  __syncthreads();
  if (warp == 0)
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(512));
  if (threadIdx.x == 0 && failed) {
    atomicExch(p.err, 1);
    atomicExch(&g_tc_fault, 1);
  }
}

// ---------------------------------------------------------------------------
// Near-tie re-bound.  The min-area rule makes the lower slope jump from 0 to
// 1 at up_s = 0.5, so where a box has an unstable neuron with up_s inside
// kTieBand of 0.5 the tensor cores' rounding could pick the other slope than
// the reference and give a different (equally valid) bound.  crown_tc_kernel
// lists those boxes; here each is bounded again with the fp32 SIMT kernel's
// operation order, so that its lb, A and acc equal crown_mlp_kernel's bit
// for bit and its slope decisions are the reference's (the SIMT kernel's
// fp32 IBP bounds are bit-identical to the reference's on these networks).
// Outside the band the two upper slopes do not straddle 0.5: on the cfg2
// workload they differ by at most 1.1e-6 near 0.5.  The IBP bounds written
// by crown_tc_kernel (sb_out) stay.
//
// 64 threads per box, kTieBoxes boxes per CTA.  In the IBP forward thread o
// owns output o: its sequential chains of fused multiply-adds over the layer
// inputs for the centre and the radius.  In the back-substitution thread c
// owns coefficient column c of every spec row (chains over the layer
// outputs, all rows side by side on one weight load); 8-column intercept
// groups and per-row sums follow in crown_mlp_kernel's order.  Operands are
// loaded in blocks ahead of their chains.
//
// The network is read from one row image written by crown_tc_images and
// staged into shared memory by a bulk copy: fc layer l as pad4(dims[l+1])
// rows [W_l[o, :], b_l[o], 0 ..] (zero rows beyond dims[l+1]) of pitch
// tpitch[l], a multiple of 4 with an odd number of 16-byte words, so the
// forward's per-thread 16-byte reads along a row and the back-substitution's
// reads of one row across threads are both conflict-free.  Zero padding adds
// exact zeros, as in crown_mlp_kernel.
constexpr int kTieBoxes = 8;  // boxes per CTA, 64 threads each

struct TieLayout {
  int net_in_smem;  // the network image is staged in shared memory
  int boxes;        // boxes per CTA
  int bar_off;      // mbarrier (8 bytes) at this float offset
  int v_off;        // Q x kW spec-times-last-layer table
  int box_off, box_floats;
  int sl_floats, qp;  // slopes; spec rows padded to 4
  int bytes;
};

__device__ __forceinline__ void tie_bar(int id) {
  asm volatile("bar.sync %0, 64;" ::"r"(id) : "memory");
}

// kNetSmem: the network image is staged in shared memory (else read from
// the workspace); QG: spec rows in groups of 4 (Q <= 4 QG, padded rows zero).
template <bool kNetSmem, int QG>
__global__ void __launch_bounds__(64 * kTieBoxes, 1)
    crown_tie_kernel(const __grid_constant__ TcParams p, const TieLayout t) {
  extern __shared__ __align__(16) float tsm[];
  // launched with a programmatic dependency on crown_tc_kernel: its list and
  // outputs are complete and visible after this wait
  asm volatile("griddepcontrol.wait;" ::: "memory");
  const int count = *p.tie_count;
  const int nb = t.boxes;
  // listed box i goes to CTA i % grid (slot i / grid): the few hundred boxes
  // of a call spread over every SM
  if ((int)blockIdx.x >= count) return;
  const int tid = threadIdx.x, slot = tid >> 6, lt = tid & 63;
  const int nfc = p.n_fc, Q = p.Q, n0 = p.dims[0], QP = t.qp;
  const float* net = kNetSmem ? tsm : p.tnet;
  __shared__ int failed;
  uint64_t* bar = reinterpret_cast<uint64_t*>(tsm + t.bar_off);
  if (kNetSmem && tid == 0) {
    failed = 0;
    mbar_init(bar, 1);
    mbar_fence_init();
    mbar_expect_tx(bar, p.tnet_floats * 4);
    bulk_load(tsm, p.tnet, p.tnet_floats * 4, bar);
  }
  float* V = tsm + t.v_off;
  {  // spec rows times [W_last | b_last], o ascending (crown_mlp_kernel's
     // order), from global memory while the copy lands
    const int nprev = p.dims[nfc - 1], nL = p.dims[nfc];
    const float* Wl = p.W + p.w_goff[nfc - 1];
    const float* bl = p.b + p.b_goff[nfc - 1];
    for (int idx = tid; idx < Q * kW; idx += blockDim.x) {
      const int q = idx / kW, c = idx % kW;
      float acc = 0.f;
      if (c <= nprev)
        for (int o = 0; o < nL; ++o)
          acc = fmaf(__ldg(p.specW + q * nL + o),
                     c < nprev ? __ldg(Wl + (long long)o * nprev + c) : __ldg(bl + o), acc);
      V[idx] = acc;
    }
  }
  if (kNetSmem) {
    if (tid == 0 && !mbar_wait(bar, 0, kSpin)) {
      failed = 1;
      atomicExch(&g_tc_fault, 1);
      mbar_wait(bar, 0, kSpin);  // let the copy land before the CTA exits
    }
    __syncthreads();
    if (failed) return;  // the listed boxes keep crown_tc_kernel's bounds
  }
  __syncthreads();
  // per-box state
  float* bx = tsm + t.box_off + slot * t.box_floats;
  float* sxl = bx;
  float* sxh = sxl + kW;
  float* mid = sxh + kW;      // [2][kW]
  float* rad = mid + 2 * kW;  // [2][kW]
  float2* sl = reinterpret_cast<float2*>(rad + 2 * kW);
  float* ewt = rad + 2 * kW + t.sl_floats;  // [2][kW][QP], column-major: row q of column k at k*QP+q
  float* vneg = ewt + 2 * kW * QP;          // [Q][kW]
  float* vicp = vneg + Q * kW;              // [Q][kW]
  float* part = vicp + Q * kW;              // [Q][8]
  float* racc = part + 8 * Q;               // [QP]
  float* bd = racc + QP;                    // [QP]
  const int bid = 1 + slot;
  for (int round = 0; (round * nb) * (int)gridDim.x + (int)blockIdx.x < count; ++round) {
    const int item = (round * nb + slot) * (int)gridDim.x + (int)blockIdx.x;
    if (item >= count) continue;  // this slot's 64 threads have no box this round
    const int box = p.tie_list[item];
    {
      float lo = 0.f, hi = 0.f;
      if (lt < n0) {
        lo = __ldg(p.xl + (long long)box * n0 + lt);
        hi = __ldg(p.xh + (long long)box * n0 + lt);
      }
      sxl[lt] = lo;
      sxh[lt] = hi;
      mid[lt] = __fmul_rn(__fadd_rn(lo, hi), 0.5f);  // 0 beyond n0
      rad[lt] = __fmul_rn(__fsub_rn(hi, lo), 0.5f);
      if (lt < Q) racc[lt] = __ldg(p.specb + lt);
    }
    tie_bar(bid);
    // ---- IBP forward: thread lt owns output lt
    int soff = 0;
    for (int l = 0; l < nfc - 1; ++l) {
      const int nin = p.dims[l], nout = p.dims[l + 1], pitch = p.tpitch[l];
      const float* m_in = mid + (l & 1) * kW;
      const float* r_in = rad + (l & 1) * kW;
      float* m_out = mid + ((l + 1) & 1) * kW;
      float* r_out = rad + ((l + 1) & 1) * kW;
      if (lt < nout) {
        const float* wr = net + p.tsoff[l] + lt * pitch;
        float am = 0.f, ar = 0.f;
        // whole 16-column blocks: the row's bias column and zero padding
        // meet the zero input padding (exact zeros, as the SIMT kernel's)
        const int kend = (nin + 15) & ~15;
        for (int kb = 0; kb < kend; kb += 16) {
          float4 w[4], m[4], r[4];
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            w[j] = *reinterpret_cast<const float4*>(wr + kb + 4 * j);
            m[j] = *reinterpret_cast<const float4*>(m_in + kb + 4 * j);
            r[j] = *reinterpret_cast<const float4*>(r_in + kb + 4 * j);
          }
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            am = fmaf(m[j].x, w[j].x, am);
            ar = fmaf(r[j].x, fabsf(w[j].x), ar);
            am = fmaf(m[j].y, w[j].y, am);
            ar = fmaf(r[j].y, fabsf(w[j].y), ar);
            am = fmaf(m[j].z, w[j].z, am);
            ar = fmaf(r[j].z, fabsf(w[j].z), ar);
            am = fmaf(m[j].w, w[j].w, am);
            ar = fmaf(r[j].w, fabsf(w[j].w), ar);
          }
        }
        const float mc = __fadd_rn(am, wr[nin]);
        float lo = __fsub_rn(mc, ar);
        float hi = __fadd_rn(mc, ar);
        if (p.clo) {
          const long long gi = p.relu_goff[l] + (long long)box * nout + lt;
          lo = fmaxf(lo, __ldg(p.clo + gi));
          hi = fminf(hi, __ldg(p.chi + gi));
        }
        hi = fmaxf(hi, lo);
        sl[soff + lt] = encode_slope(lo, hi);
        const float lc = fmaxf(lo, 0.f), hc = fmaxf(hi, 0.f);
        m_out[lt] = __fmul_rn(__fadd_rn(lc, hc), 0.5f);
        r_out[lt] = __fmul_rn(__fsub_rn(hc, lc), 0.5f);
      } else {
        m_out[lt] = 0.f;  // the next layer's input padding
        r_out[lt] = 0.f;
      }
      soff += nout;
      tie_bar(bid);
    }
    // ---- back-substitution: thread lt owns column lt of every spec row
    int cur = 0;
    for (int l = nfc - 1; l >= 0; --l) {
      const int nin = p.dims[l], nout = p.dims[l + 1], pitch = p.tpitch[l];
      const float* Wl = net + p.tsoff[l];
      const int L = l - 1;
      const int NC = nin + 1, CG = (NC + 7) >> 3;
      soff -= (L >= 0) ? nin : 0;
      const float* e_in = ewt + cur * kW * QP;
      float* e_out = ewt + (cur ^ 1) * kW * QP;
      const int c = lt;
      if (c <= nin) {
        float a[4 * QG];
#pragma unroll
        for (int q = 0; q < 4 * QG; ++q) a[q] = 0.f;
        if (l == nfc - 1) {
#pragma unroll
          for (int q = 0; q < 4 * QG; ++q)
            if (q < Q) a[q] = V[q * kW + c];
        } else {
          // blocks of 8 rows: the rows past dims[l+1] are zero and meet zero
          // coefficients, so the padded steps add exact zeros
          const int kend = tie_rows(nout);
          for (int kb = 0; kb < kend; kb += 8) {
            float wv[8];
            float4 ev[8][QG];
#pragma unroll
            for (int i = 0; i < 8; ++i) {
              wv[i] = Wl[(kb + i) * pitch + c];
#pragma unroll
              for (int g = 0; g < QG; ++g)
                ev[i][g] = *reinterpret_cast<const float4*>(e_in + (kb + i) * QP + 4 * g);
            }
#pragma unroll
            for (int i = 0; i < 8; ++i) {
#pragma unroll
              for (int g = 0; g < QG; ++g) {
                a[4 * g + 0] = fmaf(ev[i][g].x, wv[i], a[4 * g + 0]);
                a[4 * g + 1] = fmaf(ev[i][g].y, wv[i], a[4 * g + 1]);
                a[4 * g + 2] = fmaf(ev[i][g].z, wv[i], a[4 * g + 2]);
                a[4 * g + 3] = fmaf(ev[i][g].w, wv[i], a[4 * g + 3]);
              }
            }
          }
        }
        Slope sv;
        if (c < nin && L >= 0) {
          sv = decode_slope(sl[soff + c], nullptr);
        } else {
          sv.pos = sv.neg = (c < nin) ? 1.f : 0.f;  // input layer: identity
          sv.icp = 0.f;
        }
        const bool has_beta = L >= 0 && p.beta && c < nin;  // one value per neuron
        const float bv = has_beta ? __ldg(p.beta + p.relu_goff[L] + (long long)box * nin + c) : 0.f;
#pragma unroll
        for (int q = 0; q < 4 * QG; ++q) {
          {
            const float v = a[q];
            const float m = v < 0.f ? sv.neg : sv.pos;
            float o = __fmul_rn(v, m);  // the bias column's entry is a zero product
            if (has_beta) o = __fadd_rn(o, bv);
            e_out[c * QP + q] = q < Q ? o : 0.f;
            if (q < Q) {
              vneg[q * kW + c] = fminf(v, 0.f);
              vicp[q * kW + c] = sv.icp;
              if (c == nin) bd[q] = v;
            }
          }
        }
      } else {
        // columns past the bias: the next layer's padded rows read zeros here
#pragma unroll
        for (int q = 0; q < 4 * QG; ++q) e_out[c * QP + q] = 0.f;
      }
      tie_bar(bid);
      if (l > 0) {  // intercept partial of every 8-column group, in column order
        for (int it = lt; it < Q * CG; it += 64) {
          const int q = it / CG, g = it - q * CG;
          float pj = 0.f;
          for (int cc = 8 * g; cc < min(NC, 8 * g + 8); ++cc)
            pj = fmaf(vneg[q * kW + cc], vicp[q * kW + cc], pj);
          part[q * 8 + g] = pj;
        }
        tie_bar(bid);
      }
      if (lt < Q) {
        float a = __fadd_rn(racc[lt], bd[lt]);
        if (l > 0) {
          float ps = 0.f;
          for (int g = 0; g < CG; ++g) ps = __fadd_rn(ps, part[lt * 8 + g]);
          a = __fadd_rn(a, ps);
        }
        racc[lt] = a;
      }
      cur ^= 1;
      tie_bar(bid);
    }
    // ---- concretisation against the box
    if (lt < Q) {
      const float* e = ewt + cur * kW * QP + lt;
      const long long go = (long long)box * Q + lt;
      float* Ar = p.A ? p.A + go * n0 : nullptr;
      float s1 = 0.f, s2 = 0.f;
      for (int i = 0; i < n0; ++i) {
        const float ei = e[i * QP];
        s1 = fmaf(fmaxf(ei, 0.f), sxl[i], s1);
        s2 = fmaf(fminf(ei, 0.f), sxh[i], s2);
        if (Ar) Ar[i] = ei;
      }
      p.lb[go] = __fadd_rn(__fadd_rn(racc[lt], s1), s2);
      if (p.accout) p.accout[go] = racc[lt];
    }
    tie_bar(bid);
  }
}

TieLayout plan_tie(const TcParams& p) {
  TieLayout t{};
  int relu = 0;
  for (int L = 0; L < p.n_fc - 1; ++L) relu += p.dims[L + 1];
  t.sl_floats = (2 * relu + 3) & ~3;
  t.qp = (std::max(1, p.Q) + 3) & ~3;
  t.box_floats = 6 * kW + t.sl_floats + 2 * kW * t.qp + 2 * p.Q * kW + 8 * p.Q + 2 * t.qp;
  t.box_floats = (t.box_floats + 3) & ~3;
  const int limit = 227 * 1024 / 4;
  const int net = (p.tnet_floats + 3) & ~3;
  t.net_in_smem = net + 4 + kMaxQ * kW + t.box_floats <= limit ? 1 : 0;
  t.bar_off = t.net_in_smem ? net : 0;
  t.v_off = t.bar_off + 4;
  t.box_off = t.v_off + kMaxQ * kW;
  t.boxes = std::max(1, std::min(kTieBoxes, (limit - t.box_off) / t.box_floats));
  t.bytes = (t.box_off + t.boxes * t.box_floats) * 4;
  return t;
}

bool eligible_dims(const vcb_mlp* net) {
  const int nfc = net->n_fc;
  if (nfc < 2 || nfc > VCB_MAX_FC) return false;
  for (int l = 0; l < nfc; ++l)
    if (net->dims[l] < 1 || net->dims[l] > kMaxWidth) return false;
  return net->dims[nfc] >= 1;
}

struct TcPlan {
  int grid;
  long long slot_f2;
  size_t img_bytes, slots_bytes, tnet_off, tnet_bytes, flag_off, list_off, ws_bytes;
  int tnet_floats;
};

inline size_t align256(size_t n) { return (n + 255) & ~static_cast<size_t>(255); }

TcPlan plan_tc(const vcb_mlp* net, int B) {
  TcPlan t;
  const int ntiles = (B + kTB - 1) / kTB;
  t.grid = std::max(1, std::min(ntiles, sm_count()));
  long long slot = 0;
  for (int L = 0; L < net->n_fc - 1; ++L) slot += (long long)net->dims[L + 1] * kTB;
  t.slot_f2 = slot;
  t.img_bytes = (size_t)3 * (net->n_fc - 1) * kImg;
  t.slots_bytes = (size_t)t.grid * slot * sizeof(float2);
  t.tnet_floats = 0;
  for (int l = 0; l < net->n_fc; ++l)
    t.tnet_floats += tie_rows(net->dims[l + 1]) * tie_pitch(net->dims[l]);
  // error word and tie count, the images, the slope slots, the network rows
  // of the tie re-bound, its flags and its list
  t.tnet_off = align256(256 + t.img_bytes + t.slots_bytes);
  t.tnet_bytes = (size_t)t.tnet_floats * sizeof(float);
  t.flag_off = align256(t.tnet_off + t.tnet_bytes);
  t.list_off = align256(t.flag_off + (size_t)B * sizeof(int));
  t.ws_bytes = t.list_off + (size_t)B * sizeof(int);
  return t;
}

}  // namespace

bool crown_tc_eligible(const vcb_mlp* net, int Q) {
  return net && eligible_dims(net) && Q >= 0 && Q <= kMaxQ;
}

bool crown_tc_route(const vcb_mlp* net, int B, int Q) {
  return crown_tc_eligible(net, Q) && B >= g_min_batch.load(std::memory_order_relaxed);
}

size_t crown_tc_workspace(const vcb_mlp* net, int B) {
  if (!net || B <= 0 || !eligible_dims(net)) return 0;
  return plan_tc(net, B).ws_bytes;
}

int crown_tc_launch(const vcb_mlp* net, int32_t B, const float* xl, const float* xh,
                    const float* clamp_lo, const float* clamp_hi, const float* sb_in_lo,
                    const float* sb_in_hi, const float* alpha, const float* beta, int32_t Q,
                    const float* spec_W, const float* spec_b, float* lb, float* A, float* acc,
                    float* sb_out_lo, float* sb_out_hi, void* ws, size_t ws_bytes,
                    cudaStream_t st, const char* who) {
  const TcPlan plan = plan_tc(net, B);
  if (!ws || ws_bytes < plan.ws_bytes)
    return fail(VCB_ERR_INVALID, "%s: workspace of %zu bytes needed (got %zu)", who,
                plan.ws_bytes, ws_bytes);
  if ((reinterpret_cast<uintptr_t>(ws) & 255) != 0)
    return fail(VCB_ERR_INVALID, "%s: workspace must be 256-byte aligned", who);
  TcParams p{};
  const int nfc = net->n_fc;
  p.n_fc = nfc;
  long long woff = 0, roff = 0;
  int boff = 0, soff = 0;
  for (int l = 0; l <= nfc; ++l) p.dims[l] = net->dims[l];
  for (int l = 0; l < nfc; ++l) {
    p.w_goff[l] = woff;
    p.b_goff[l] = boff;
    woff += (long long)net->dims[l] * net->dims[l + 1];
    boff += net->dims[l + 1];
    if (l < nfc - 1) {
      p.relu_goff[l] = roff;
      roff += (long long)B * net->dims[l + 1];
      p.sl_off[l] = soff;
      soff += net->dims[l + 1] * kTB;
    }
  }
  uint8_t* base = static_cast<uint8_t*>(ws);
  p.W = net->W;
  p.b = net->b;
  p.err = reinterpret_cast<int*>(base);
  p.tie_count = reinterpret_cast<int*>(base + 64);
  p.img = base + 256;
  p.slopes = reinterpret_cast<float2*>(base + 256 + plan.img_bytes);
  p.tie_on = (!sb_in_lo && !alpha && Q > 0) ? 1 : 0;
  p.tnet = reinterpret_cast<float*>(base + plan.tnet_off);
  p.tie_flag = reinterpret_cast<int*>(base + plan.flag_off);
  p.tie_list = reinterpret_cast<int*>(base + plan.list_off);
  p.tnet_floats = plan.tnet_floats;
  for (int l = 0, off = 0; l < nfc; ++l) {
    p.tsoff[l] = off;
    p.tpitch[l] = tie_pitch(net->dims[l]);
    off += tie_rows(net->dims[l + 1]) * p.tpitch[l];
  }
  p.slot_f2 = plan.slot_f2;
  p.B = B;
  p.Q = Q;
  p.ntiles = (B + kTB - 1) / kTB;
  p.npass = (Q + 1) / 2;
  {
    const int rem = p.ntiles % plan.grid;
    p.split_tail = (rem > 0 && 2 * rem <= plan.grid && p.npass >= 2) ? 1 : 0;
  }
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
  const int nimg = std::max(3 * (nfc - 1) * kW * kW,
                           p.tie_on ? std::max(B, plan.tnet_floats) : 0);
  crown_tc_images<<<(nimg + 255) / 256, 256, 0, st>>>(p);
  int rc = check_launch(who);
  if (rc) return rc;
  const bool plain = !alpha && !beta && !clamp_lo && !sb_out_lo;
  const void* fn = plain ? reinterpret_cast<const void*>(crown_tc_kernel<true>)
                         : reinterpret_cast<const void*>(crown_tc_kernel<false>);
  rc = ensure_smem(fn, kSmem);
  if (rc) return rc;
  // programmatic dependent launches: each kernel of the chain is scheduled
  // while the previous one drains and waits on the device for its results
  cudaLaunchAttribute pdl[1];
  pdl[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  pdl[0].val.programmaticStreamSerializationAllowed = 1;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(plan.grid);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = kSmem;
  cfg.stream = st;
  cfg.attrs = pdl;
  cfg.numAttrs = 1;
  rc = cuda_fail(plain ? cudaLaunchKernelEx(&cfg, crown_tc_kernel<true>, p)
                       : cudaLaunchKernelEx(&cfg, crown_tc_kernel<false>, p),
                 who);
  if (rc) return rc;
  rc = check_launch(who);
  if (rc || !p.tie_on) return rc;
  // the listed boxes, bounded again with the fp32 kernel's order; a launch
  // whose list is empty returns at once
  const TieLayout tl = plan_tie(p);
  const int qg = tl.qp / 4;
  const void* tie_fn = nullptr;
#define VCB_TIE_FN(S, G) if (tl.net_in_smem == S && qg == G) tie_fn = reinterpret_cast<const void*>(crown_tie_kernel<S, G>);
  VCB_TIE_FN(1, 1) VCB_TIE_FN(1, 2) VCB_TIE_FN(1, 3) VCB_TIE_FN(1, 4)
  VCB_TIE_FN(0, 1) VCB_TIE_FN(0, 2) VCB_TIE_FN(0, 3) VCB_TIE_FN(0, 4)
#undef VCB_TIE_FN
  rc = ensure_smem(tie_fn, tl.bytes);
  if (rc) return rc;
  void* args[] = {const_cast<TcParams*>(&p), const_cast<TieLayout*>(&tl)};
  cfg.gridDim = dim3(sm_count());
  cfg.blockDim = dim3(64 * tl.boxes);
  cfg.dynamicSmemBytes = (size_t)tl.bytes;
  rc = cuda_fail(cudaLaunchKernelExC(&cfg, tie_fn, args), who);
  if (rc) return rc;
  return check_launch(who);
}

int crown_tc_fault_take(cudaStream_t st, int* was_set) {
  int h = 0;
  cudaError_t e = cudaMemcpyFromSymbolAsync(&h, g_tc_fault, sizeof(int), 0,
                                            cudaMemcpyDeviceToHost, st);
  if (e == cudaSuccess) e = cudaStreamSynchronize(st);
  if (e == cudaSuccess && h) {
    const int zero = 0;
    e = cudaMemcpyToSymbolAsync(g_tc_fault, &zero, sizeof(int), 0, cudaMemcpyHostToDevice, st);
    if (e == cudaSuccess) e = cudaStreamSynchronize(st);
  }
  *was_set = h;
  return cuda_fail(e, "vcb_fault_check");
}

}  // namespace vcb

extern "C" int32_t vcb_mlp_crown_path(const vcb_mlp* net, int32_t B, int32_t Q) {
  return vcb::crown_tc_route(net, B, Q) ? 1 : 0;
}

extern "C" int32_t vcb_mlp_crown_tc_min_batch(int32_t value) {
  const int32_t prev = vcb::g_min_batch.load();
  if (value >= 0) vcb::g_min_batch.store(value);
  return prev;
}
