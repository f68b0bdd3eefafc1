// fp32 GEMM on the 5th-generation tensor cores with error-compensated
// 3xTF32 (the contraction behind the wide layers' bound propagation).
//
// C (M x N) = A (M x K) B^T, A and B both K-major (row-major M x K and
// N x K -- activations x weights).  Each operand is pre-split into a TF32
// "hi" part (round to nearest at 10 mantissa bits) and the exact fp32
// remainder "lo" (vcb_tf32_split); the tensor cores form
//   lo_A hi_B + hi_A lo_B + hi_A hi_B
// which is within ~2^-22 of the fp32 product (the dropped lo_A lo_B term).
// The tensor cores' own fp32 accumulation drops low-order bits at every MMA,
// so each 32-wide K chunk accumulates in a fresh TMEM buffer (12 MMAs) and
// the epilogue warps add the chunk partials into fp32 registers with
// round-to-nearest adds: the long sum over K is an ordinary fp32 sum.
//
// Kernel structure (persistent, one CTA per SM walking 128 x 128 output tiles
// with the N tile fastest so the CTAs reading the same A rows run together;
// 6 warps):
//   warp 4 / one thread : TMA producer -- per K chunk, four 128 x 32 fp32
//                         tiles (A hi/lo, B hi/lo) into a 3-stage ring of
//                         shared memory with 128-byte swizzle, each stage
//                         signalled by an mbarrier (complete_tx);
//   warp 5 / one thread : MMA issuer -- tcgen05.mma kind::tf32, M = 128,
//                         N = 128, K = 8, three per K step, chunk kb into TMEM
//                         buffer kb % 4 (4 x 128 columns); tcgen05.commit
//                         frees the smem stage and publishes the buffer;
//   warps 0-3           : accumulators -- warp w owns TMEM lanes 32w..32w+31
//                         (tile rows); per chunk tcgen05.ld of its 128
//                         columns, fp32 adds into registers, then the buffer
//                         is released to the MMA issuer; finally bias + store.
// Every mbarrier wait is bounded: on expiry the kernel records an error
// flag, drains its MMAs through the final commit, frees its TMEM and
// returns, and the host reports VCB_ERR_TIMEOUT.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <algorithm>

#include "vcb_common.cuh"
#include "vcb_tc.cuh"
#include "vcb_tcgen05.cuh"

namespace vcb {
namespace {

constexpr int TC_BM = 128, TC_BK = 32;
constexpr int TMEM_COLS = 512;                   // the whole tensor memory
constexpr int TILE_A_BYTES = TC_BM * TC_BK * 4;  // 16 KB
constexpr unsigned kSpinLimit = 1u << 22;      // pipeline waits (a stage is microseconds)
constexpr unsigned kDoneSpinLimit = 1u << 27;  // the epilogue waits out the whole mainloop

// Tile shapes: BN = 128 (3 smem stages, 4 TMEM chunk buffers) or BN = 256
// (2 stages, 2 buffers; per FLOP half the A bytes from L2 into shared
// memory); 8 accumulator warps either way, warp w holding TMEM lanes
// 32 (w % 4).. and kCols = BN / 2 columns from kCols (w / 4).
template <int BN>
struct TcCfg {
  static constexpr int kStages = BN == 256 ? 2 : 3;
  static constexpr int kNbuf = TMEM_COLS / BN;
  static constexpr int kEpiWarps = 8;
  static constexpr int kCols = BN / 2;
  static constexpr int kThreads = (kEpiWarps + 2) * 32;
  static constexpr int kTileB = BN * TC_BK * 4;
  static constexpr int kStage = 2 * TILE_A_BYTES + 2 * kTileB;
  // stages + the epilogue warps' staging blocks + alignment slack
  static constexpr int kSmem = kStages * kStage + kEpiWarps * 32 * 33 * 4 + 1024;
  // instruction descriptor: D f32, A/B tf32, both K-major, M = 128, N = BN
  static constexpr uint32_t kIdesc = tc5::idesc_tf32(TC_BM, BN);
};

using namespace tc5;

__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, uint64_t* bar,
                                            int x, int y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes "
      "[%0], [%1, {%2, %3}], [%4];" ::"r"(smem_u32(dst)),
      "l"(map), "r"(x), "r"(y), "r"(smem_u32(bar))
      : "memory");
}

struct TcArgs {
  int M, N, K, ldc;
  float* C;
  const float* bias;  // (N) added to every row, or NULL
  int* err;           // set to 1 when a bounded wait expired
  const int* gate;    // when non-NULL and *gate == 0 the launch does nothing
  int vec;            // N % 4 == 0 and every row of every operand 16-byte aligned
  TcEpi ep;
};

// The epilogue stages 32 x 32 blocks (one warp's rows x 32 columns) through
// shared memory so that every global access of a warp covers 128
// contiguous bytes of one row; a pitch of 33 floats keeps both the row-wise
// writes and the column-wise reads free of bank conflicts.
constexpr int kStagePitch = 33;
constexpr int kStageWarpBytes = 32 * kStagePitch * 4;

// Rows of one warp go through the epilogue in batches: all global loads of
// a batch are issued first (read-only path), then the arithmetic and the
// stores, so a warp keeps a batch's worth of loads in flight.
constexpr int kEpiBatch = 8;

// Per-element inputs of one batch row (which of them are read depends on
// the mode).
struct EpiIn {
  float x0, x1, x2, x3;
};

template <int MODE>
__device__ __forceinline__ EpiIn epi_load(const TcArgs& a, int row, int box, int col) {
  const TcEpi& e = a.ep;
  EpiIn in{0.f, 0.f, 0.f, 0.f};
  if (MODE == kEpiStore) return in;
  const int bi = box * a.N + col;  // per-box arrays (the host checks 32-bit offsets)
  if (MODE == kEpiConcretize) {
    in.x0 = __ldg(e.xl + bi);
    in.x1 = __ldg(e.xh + bi);
    return in;
  }
  in.x0 = __ldg(e.pos + bi);
  const float2 rx = __ldg(e.rx + bi);
  in.x1 = rx.x;
  in.x2 = rx.y;
  if (MODE == kEpiRelax) {
    if (e.beta) in.x3 = __ldg(e.beta + bi);
  } else {
    in.x3 = __ldg(e.rec + row * e.ldrec + col);
  }
  return in;
}

// Results of one element: o (the value whose split goes to out_hi /
// out_lo), c (its share of the row's partial sum), d (the alpha-gradient
// row entry).
struct EpiOut {
  float o, c, d;
};

// The arithmetic of one element with value v (see TcEpi); colv: bias[col]
// (store / adjoint) or bnext[col] (relax).
template <int MODE>
__device__ __forceinline__ EpiOut epi_math(const TcArgs& a, float v, const EpiIn& in, float colv) {
  EpiOut r{0.f, 0.f, 0.f};
  if (MODE == kEpiStore) {
    r.o = a.bias ? __fadd_rn(v, colv) : v;
  } else if (MODE == kEpiConcretize) {
    r.c = __fadd_rn(__fmul_rn(fmaxf(v, 0.f), in.x0), __fmul_rn(fminf(v, 0.f), in.x1));
    r.o = (v >= 0.f ? in.x0 : 0.f) + (v <= 0.f ? in.x1 : 0.f);
  } else {
    const float pos = in.x0, neg = fabsf(in.x1), icp = in.x2;
    if (MODE == kEpiRelax) {
      float o;
      if (v < 0.f) {
        r.c = __fmul_rn(v, icp);
        o = __fmul_rn(v, neg);
      } else {
        o = __fmul_rn(v, pos);
      }
      if (a.ep.beta) o = __fadd_rn(o, in.x3);
      if (a.ep.bnext) r.c = fmaf(o, colv, r.c);
      r.o = o;
    } else {  // kEpiAdjoint
      const float ga = __fadd_rn(v, colv);
      const float ek = in.x3;
      r.d = !signbit(in.x1) ? __fmul_rn(fmaxf(ek, 0.f), ga) : 0.f;  // unstable neurons only
      float o = 0.f;
      if (ek >= 0.f) o = __fmul_rn(pos, ga);
      if (ek <= 0.f) o = __fadd_rn(o, __fadd_rn(__fmul_rn(neg, ga), icp));
      r.o = o;
    }
  }
  return r;
}

template <int MODE>
__device__ __forceinline__ void epi_store(const TcArgs& a, int row, int col, float v,
                                          const EpiOut& r) {
  const TcEpi& e = a.ep;
  if (MODE == kEpiStore) {
    a.C[(long long)row * a.ldc + col] = r.o;
    return;
  }
  if (MODE == kEpiRelax) a.C[row * a.ldc + col] = v;  // the record for the adjoint
  if (MODE == kEpiAdjoint) e.dcontrib[row * e.ldd + col] = r.d;
  if (e.out_hi) {
    uint32_t h, l;
    tc5::tf32_split(r.o, h, l);
    const int oi = row * e.ldo + col;
    e.out_hi[oi] = __uint_as_float(h);
    e.out_lo[oi] = __uint_as_float(l);
  }
}

// Epilogue of one warp's 32 rows (rowbase + lane holds acc) x the COLS-column
// group starting at nb; sm: this warp's staging block.  Per batch of rows:
// every load first (staged values, per-box inputs), then the arithmetic,
// then every store, so the rows of a batch overlap.  Row sums leave as one
// partial per 64 columns.
template <int MODE, int COLS>
__device__ __forceinline__ void tc_epilogue(const TcArgs& a, int rowbase, int nb,
                                            const float (&acc)[COLS], float* sm) {
  constexpr bool kSum = MODE == kEpiRelax || MODE == kEpiConcretize;
  const int lane = threadIdx.x & 31;
  const int rows = min(32, a.M - rowbase);
  const int my_box = (rowbase + lane) / a.ep.Q;  // box of row rowbase + lane
  float s = 0.f;  // partial sum of row rowbase + lane over the current 64 columns
#pragma unroll
  for (int c = 0; c < COLS / 32; ++c) {
    if (nb + 32 * c < a.N) {  // warp-uniform
      __syncwarp();
#pragma unroll
      for (int j = 0; j < 32; ++j) sm[lane * kStagePitch + j] = acc[32 * c + j];
      __syncwarp();
      const int col = nb + 32 * c + lane;
      const bool cv = col < a.N;
      float colv = 0.f;
      if (cv) {
        if ((MODE == kEpiStore || MODE == kEpiAdjoint) && a.bias) colv = __ldg(a.bias + col);
        if (MODE == kEpiRelax && a.ep.bnext) colv = __ldg(a.ep.bnext + col);
      }
      for (int r0 = 0; r0 < rows; r0 += kEpiBatch) {
        float v[kEpiBatch];
        EpiIn in[kEpiBatch];
#pragma unroll
        for (int u = 0; u < kEpiBatch; ++u) {
          v[u] = sm[(r0 + u) * kStagePitch + lane];
          const int box = __shfl_sync(0xffffffffu, my_box, r0 + u);
          in[u] = (cv && r0 + u < rows) ? epi_load<MODE>(a, rowbase + r0 + u, box, col)
                                        : EpiIn{0.f, 0.f, 0.f, 0.f};
        }
        EpiOut out[kEpiBatch];
#pragma unroll
        for (int u = 0; u < kEpiBatch; ++u) out[u] = epi_math<MODE>(a, v[u], in[u], colv);
#pragma unroll
        for (int u = 0; u < kEpiBatch; ++u) {
          if (r0 + u < rows) {
            if (cv) epi_store<MODE>(a, rowbase + r0 + u, col, v[u], out[u]);
            if (kSum) sm[(r0 + u) * kStagePitch + lane] = cv ? out[u].c : 0.f;
          }
        }
      }
      if (kSum) {
        __syncwarp();
#pragma unroll
        for (int j = 0; j < 32; ++j) s = __fadd_rn(s, sm[lane * kStagePitch + j]);  // columns of row lane
      }
    }
    if (kSum && (c & 1) == 1) {  // a 64-column group is complete
      const int g0 = nb + 32 * (c - 1);
      if (lane < rows && g0 < a.N)
        a.ep.part[(rowbase + lane) * a.ep.ldpart + a.ep.part0 + g0 / 64] = s;
      s = 0.f;
    }
  }
}

// Vectorised epilogue (TcArgs::vec): each lane takes 4 consecutive columns,
// so a warp instruction covers 4 rows x 32 columns with 16-byte accesses.
// The staging block is 32 rows x 32 floats with the 16-byte chunks of row r
// XOR-swizzled by r % 8 (conflict-free for the row-wise writes and the
// 4-row reads), followed by 32 per-row running sums.
__device__ __forceinline__ float4 ldg4(const float* p) {
  return __ldg(reinterpret_cast<const float4*>(p));
}

__device__ __forceinline__ void stg4(float* p, float4 v) { *reinterpret_cast<float4*>(p) = v; }

__device__ __forceinline__ float f4(const float4& v, int k) {
  return k == 0 ? v.x : (k == 1 ? v.y : (k == 2 ? v.z : v.w));
}

template <int MODE, int COLS>
__device__ __forceinline__ void tc_epilogue_vec(const TcArgs& a, int rowbase, int nb,
                                                const float (&acc)[COLS], float* sm) {
  constexpr bool kSum = MODE == kEpiRelax || MODE == kEpiConcretize;
  constexpr int kRowsPerStep = 4, kSteps = 4;  // 16 rows of loads in flight per batch
  const TcEpi& e = a.ep;
  float* rs = sm + 32 * 32;  // per-row running sums
  const int lane = threadIdx.x & 31;
  const int rows = min(32, a.M - rowbase);
  const int my_box = (rowbase + lane) / e.Q;
  const int sub = lane >> 3, q4 = lane & 7;  // row within a step, 16-byte chunk within the row
  if (kSum) rs[lane] = 0.f;
#pragma unroll
  for (int c = 0; c < COLS / 32; ++c) {
    if (nb + 32 * c < a.N) {  // warp-uniform
      __syncwarp();
#pragma unroll
      for (int j = 0; j < 8; ++j)
        *reinterpret_cast<float4*>(sm + lane * 32 + 4 * (j ^ (lane & 7))) =
            make_float4(acc[32 * c + 4 * j], acc[32 * c + 4 * j + 1], acc[32 * c + 4 * j + 2],
                        acc[32 * c + 4 * j + 3]);
      __syncwarp();
      const int col = nb + 32 * c + 4 * q4;
      const bool cv = col < a.N;
      float4 colv = make_float4(0.f, 0.f, 0.f, 0.f);
      if (cv) {
        if ((MODE == kEpiStore || MODE == kEpiAdjoint) && a.bias) colv = ldg4(a.bias + col);
        if (MODE == kEpiRelax && e.bnext) colv = ldg4(e.bnext + col);
      }
      for (int r0 = 0; r0 < rows; r0 += kRowsPerStep * kSteps) {
        float4 v[kSteps], x0[kSteps], x1[kSteps], x2[kSteps], x3[kSteps];
#pragma unroll
        for (int u = 0; u < kSteps; ++u) {
          const int r = r0 + kRowsPerStep * u + sub;  // <= 31
          v[u] = *reinterpret_cast<const float4*>(sm + r * 32 + 4 * (q4 ^ (r & 7)));
          const int box = __shfl_sync(0xffffffffu, my_box, r);
          const float4 z = make_float4(0.f, 0.f, 0.f, 0.f);
          x0[u] = x1[u] = x2[u] = x3[u] = z;
          if (cv && r < rows && MODE != kEpiStore) {
            const int bi = box * a.N + col;
            if (MODE == kEpiConcretize) {
              x0[u] = ldg4(e.xl + bi);
              x1[u] = ldg4(e.xh + bi);
            } else {
              x0[u] = ldg4(e.pos + bi);
              x1[u] = ldg4(reinterpret_cast<const float*>(e.rx) + 2 * bi);      // cols 0, 1
              x2[u] = ldg4(reinterpret_cast<const float*>(e.rx) + 2 * bi + 4);  // cols 2, 3
              if (MODE == kEpiRelax && e.beta) x3[u] = ldg4(e.beta + bi);
              if (MODE == kEpiAdjoint) x3[u] = ldg4(e.rec + (rowbase + r) * e.ldrec + col);
            }
          }
        }
#pragma unroll
        for (int u = 0; u < kSteps; ++u) {
          const int r = r0 + kRowsPerStep * u + sub;
          const int row = rowbase + r;
          float o[4], cs[4], d[4];
#pragma unroll
          for (int k = 0; k < 4; ++k) {
            EpiIn in{0.f, 0.f, 0.f, 0.f};
            if (MODE == kEpiConcretize) {
              in.x0 = f4(x0[u], k);
              in.x1 = f4(x1[u], k);
            } else if (MODE != kEpiStore) {
              in.x0 = f4(x0[u], k);
              in.x1 = k < 2 ? f4(x1[u], 2 * k) : f4(x2[u], 2 * k - 4);
              in.x2 = k < 2 ? f4(x1[u], 2 * k + 1) : f4(x2[u], 2 * k - 3);
              in.x3 = f4(x3[u], k);
            }
            const EpiOut out = epi_math<MODE>(a, f4(v[u], k), in, f4(colv, k));
            o[k] = out.o;
            cs[k] = out.c;
            d[k] = out.d;
          }
          const bool live = cv && r < rows;
          if (live) {
            if (MODE == kEpiStore) {
              stg4(a.C + (long long)row * a.ldc + col, make_float4(o[0], o[1], o[2], o[3]));
            } else {
              if (MODE == kEpiRelax) stg4(a.C + row * a.ldc + col, v[u]);
              if (MODE == kEpiAdjoint)
                stg4(e.dcontrib + row * e.ldd + col, make_float4(d[0], d[1], d[2], d[3]));
              if (e.out_hi) {
                uint32_t h[4], l[4];
#pragma unroll
                for (int k = 0; k < 4; ++k) tc5::tf32_split(o[k], h[k], l[k]);
                const int oi = row * e.ldo + col;
                stg4(e.out_hi + oi, make_float4(__uint_as_float(h[0]), __uint_as_float(h[1]),
                                                __uint_as_float(h[2]), __uint_as_float(h[3])));
                stg4(e.out_lo + oi, make_float4(__uint_as_float(l[0]), __uint_as_float(l[1]),
                                                __uint_as_float(l[2]), __uint_as_float(l[3])));
              }
            }
          }
          if (kSum) {
            // row r's sum over this chunk: the lane's 4 columns, then its 8 lanes
            float t = live ? __fadd_rn(__fadd_rn(cs[0], cs[1]), __fadd_rn(cs[2], cs[3])) : 0.f;
            t = __fadd_rn(t, __shfl_xor_sync(0xffffffffu, t, 1));
            t = __fadd_rn(t, __shfl_xor_sync(0xffffffffu, t, 2));
            t = __fadd_rn(t, __shfl_xor_sync(0xffffffffu, t, 4));
            if (q4 == 0 && r < rows) rs[r] = __fadd_rn(rs[r], t);
          }
        }
      }
    }
    if (kSum && (c & 1) == 1) {  // a 64-column group is complete
      __syncwarp();
      const int g0 = nb + 32 * (c - 1);
      if (lane < rows && g0 < a.N)
        e.part[(rowbase + lane) * e.ldpart + e.part0 + g0 / 64] = rs[lane];
      __syncwarp();
      rs[lane] = 0.f;
    }
  }
}

template <int BN, int MODE>
__global__ void __launch_bounds__(TcCfg<BN>::kThreads, 1)
    tc_gemm_kernel(const __grid_constant__ CUtensorMap mAh, const __grid_constant__ CUtensorMap mAl,
                   const __grid_constant__ CUtensorMap mBh, const __grid_constant__ CUtensorMap mBl,
                   const TcArgs a) {
  using Cfg = TcCfg<BN>;
  constexpr int TC_BN = BN, TC_STAGES = Cfg::kStages, NBUF = Cfg::kNbuf;
  constexpr int TILE_B_BYTES = Cfg::kTileB, STAGE_BYTES = Cfg::kStage;
  constexpr int EPI = Cfg::kEpiWarps;
  if (a.gate && *a.gate == 0) return;  // uniform: before any barrier or TMEM use
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  __shared__ __align__(8) uint64_t full[TC_STAGES], empty[TC_STAGES];
  __shared__ __align__(8) uint64_t acc_full[NBUF], acc_free[NBUF], done;
  __shared__ uint32_t tmem_slot;
  __shared__ int failed;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // Persistent: the CTA walks tiles blockIdx.x, + gridDim.x, ... with the N
  // tile fastest, so the CTAs that share an A row tile run together (the
  // large A operand streams from HBM once, the other N tiles hit L2); stage,
  // TMEM-buffer and phase counters run on across tiles, so the next tile's
  // loads and MMAs overlap the previous tile's accumulation and stores.
  const int n_tiles = (a.N + TC_BN - 1) / TC_BN;
  const int tiles = ((a.M + TC_BM - 1) / TC_BM) * n_tiles;
  const int nk = (a.K + TC_BK - 1) / TC_BK;
  const volatile int* vfailed = &failed;
  if (threadIdx.x == 0) {
    for (int s = 0; s < TC_STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int q = 0; q < NBUF; ++q) {
      mbar_init(&acc_full[q], 1);
      mbar_init(&acc_free[q], EPI);  // one arrival per accumulator warp
    }
    mbar_init(&done, 1);
    failed = 0;
    mbar_fence_init();
  }
  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_u32(&tmem_slot)),
                 "r"(TMEM_COLS));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  const uint32_t tmem = tmem_slot;

  if (warp == EPI) {
    if (lane == 0) {  // TMA producer
      unsigned g = 0;  // chunks loaded by this CTA
      bool ok = true;
      for (int tile = blockIdx.x; ok && tile < tiles; tile += gridDim.x) {
        const int m0 = (tile / n_tiles) * TC_BM, n0 = (tile % n_tiles) * TC_BN;
        for (int kb = 0; kb < nk; ++kb, ++g) {
          const int s = g % TC_STAGES;
          if (g >= TC_STAGES &&
              !mbar_wait(&empty[s], ((g / TC_STAGES) - 1) & 1, kSpinLimit, vfailed)) {
            ok = false;
            break;
          }
          uint8_t* st = smem + s * STAGE_BYTES;
          mbar_expect_tx(&full[s], STAGE_BYTES);
          tma_load_2d(st, &mAh, &full[s], kb * TC_BK, m0);
          tma_load_2d(st + TILE_A_BYTES, &mAl, &full[s], kb * TC_BK, m0);
          tma_load_2d(st + 2 * TILE_A_BYTES, &mBh, &full[s], kb * TC_BK, n0);
          tma_load_2d(st + 2 * TILE_A_BYTES + TILE_B_BYTES, &mBl, &full[s], kb * TC_BK, n0);
        }
      }
      if (!ok) failed = 1;
      // the copies still in flight land before the CTA exits
      for (unsigned k = g > TC_STAGES ? g - TC_STAGES : 0; k < g; ++k)
        if (!mbar_wait(&full[k % TC_STAGES], (k / TC_STAGES) & 1, kSpinLimit)) failed = 1;
    }
  } else if (warp == EPI + 1) {
    if (lane == 0) {  // MMA issuer
      unsigned g = 0;
      bool ok = true;
      for (int tile = blockIdx.x; ok && tile < tiles; tile += gridDim.x) {
        for (int kb = 0; kb < nk; ++kb, ++g) {
          const int s = g % TC_STAGES;
          const int q = g % NBUF;
          if (!mbar_wait(&full[s], (g / TC_STAGES) & 1, kSpinLimit, vfailed) ||
              (g >= NBUF && !mbar_wait(&acc_free[q], ((g / NBUF) - 1) & 1, kSpinLimit, vfailed))) {
            ok = false;
            break;
          }
          asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
          const uint32_t base = smem_u32(smem + s * STAGE_BYTES);
          const uint32_t ah = base, al = base + TILE_A_BYTES;
          const uint32_t bh = base + 2 * TILE_A_BYTES, bl = bh + TILE_B_BYTES;
          const uint32_t dst = tmem + (uint32_t)(q * TC_BN);
#pragma unroll
          for (int j = 0; j < TC_BK / 8; ++j) {
            const uint32_t off = j * 32;  // 8 tf32 = 32 bytes along K inside the swizzle atom
            mma_tf32_ss(dst, sw128_desc(al + off), sw128_desc(bh + off), Cfg::kIdesc,
                        j > 0 ? 1u : 0u);
            mma_tf32_ss(dst, sw128_desc(ah + off), sw128_desc(bl + off), Cfg::kIdesc, 1u);
            mma_tf32_ss(dst, sw128_desc(ah + off), sw128_desc(bh + off), Cfg::kIdesc, 1u);
          }
          mma_commit(&empty[s]);
          mma_commit(&acc_full[q]);
        }
      }
      if (!ok) failed = 1;
      // every MMA issued above has finished before TMEM can be freed
      mma_commit(&done);
      if (!mbar_wait(&done, 0, kDoneSpinLimit)) failed = 1;
    }
  } else {  // accumulator warps: row m0 + 32 (warp % 4) + lane, columns kCols (warp / 4)..
    constexpr int kCols = Cfg::kCols;
    const int cg = kCols * (warp >> 2);
    const uint32_t lane_addr = tmem + ((uint32_t)((warp & 3) * 32) << 16) + cg;
    unsigned g = 0;
    bool ok = true;
    for (int tile = blockIdx.x; ok && tile < tiles; tile += gridDim.x) {
      const int m0 = (tile / n_tiles) * TC_BM, n0 = (tile % n_tiles) * TC_BN;
      float acc[kCols];
#pragma unroll
      for (int j = 0; j < kCols; ++j) acc[j] = 0.f;
      for (int kb = 0; kb < nk; ++kb, ++g) {
        const int q = g % NBUF;
        if (!mbar_wait(&acc_full[q], (g / NBUF) & 1, kDoneSpinLimit, vfailed)) {
          ok = false;
          break;
        }
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
#pragma unroll
        for (int c0 = 0; c0 < kCols; c0 += 16) {
          uint32_t v[16];
          tmem_ld16(lane_addr + q * TC_BN + c0, v);
          tmem_wait_ld(v);
#pragma unroll
          for (int j = 0; j < 16; ++j) acc[c0 + j] = __fadd_rn(acc[c0 + j], __uint_as_float(v[j]));
        }
        asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
        __syncwarp();
        if (lane == 0) mbar_arrive(&acc_free[q]);
      }
      if (!ok) break;
      if (m0 + (warp & 3) * 32 < a.M) {
        float* sm = reinterpret_cast<float*>(smem + TC_STAGES * STAGE_BYTES +
                                             warp * kStageWarpBytes);
        if (a.vec)
          tc_epilogue_vec<MODE, kCols>(a, m0 + (warp & 3) * 32, n0 + cg, acc, sm);
        else
          tc_epilogue<MODE, kCols>(a, m0 + (warp & 3) * 32, n0 + cg, acc, sm);
      }
    }
    if (!ok) failed = 1;
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  if (warp == 0)
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem),
                 "r"(TMEM_COLS));
  if (threadIdx.x == 0 && failed) atomicExch(a.err, 1);
}

// hi = x rounded to nearest at TF32 precision (10 explicit mantissa bits),
// lo = x - hi (exact in fp32).
__global__ void tf32_split_kernel(long long n, const float* __restrict__ x, float* __restrict__ hi,
                                  float* __restrict__ lo) {
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < n;
       i += (long long)gridDim.x * blockDim.x) {
    uint32_t h, l;
    tf32_split(x[i], h, l);
    hi[i] = __uint_as_float(h);
    lo[i] = __uint_as_float(l);
  }
}

PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  if (!fn) {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  }
  return fn;
}

// Row-major (rows x cols, leading dimension ld) fp32 matrix as box_rows x 32
// tiles with 128-byte swizzle; out-of-range reads fill zeros.
int make_map(CUtensorMap* map, const float* p, int rows, int cols, int ld, int box_rows,
             const char* who) {
  auto fn = encode_fn();
  if (!fn) return fail(VCB_ERR_CUDA, "%s: cuTensorMapEncodeTiled unavailable", who);
  if ((reinterpret_cast<uintptr_t>(p) & 15) || (ld % 4) || ld < cols)
    return fail(VCB_ERR_INVALID, "%s: operand must be 16-byte aligned with ld %% 4 == 0", who);
  cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)ld * 4};
  cuuint32_t box[2] = {TC_BK, (cuuint32_t)box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<float*>(p), dims, strides,
                  box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(VCB_ERR_CUDA, "%s: tensor map encode failed (%d)", who, (int)r);
  return VCB_OK;
}

}  // namespace

namespace {

template <int BN, int EPI>
int launch_tc(int grid, const CUtensorMap& mAh, const CUtensorMap& mAl, const CUtensorMap& mBh,
              const CUtensorMap& mBl, const TcArgs& args, cudaStream_t st) {
  const int rc = ensure_smem(reinterpret_cast<const void*>(tc_gemm_kernel<BN, EPI>),
                             TcCfg<BN>::kSmem);
  if (rc) return rc;
  tc_gemm_kernel<BN, EPI><<<grid, TcCfg<BN>::kThreads, TcCfg<BN>::kSmem, st>>>(mAh, mAl, mBh,
                                                                              mBl, args);
  return VCB_OK;
}

int launch_mode(int grid, const CUtensorMap& mAh, const CUtensorMap& mAl,
                const CUtensorMap& mBh, const CUtensorMap& mBl, const TcArgs& args,
                cudaStream_t st) {
  switch (args.ep.mode) {
    case kEpiRelax: return launch_tc<128, kEpiRelax>(grid, mAh, mAl, mBh, mBl, args, st);
    case kEpiAdjoint: return launch_tc<128, kEpiAdjoint>(grid, mAh, mAl, mBh, mBl, args, st);
    case kEpiConcretize:
      return launch_tc<128, kEpiConcretize>(grid, mAh, mAl, mBh, mBl, args, st);
    default: return launch_tc<128, kEpiStore>(grid, mAh, mAl, mBh, mBl, args, st);
  }
}

}  // namespace

// C = A B^T with 3xTF32 on tcgen05 and the epilogue `ep` (see vcb_tc.cuh);
// err: device int, zero on entry, set on a bounded-wait expiry.
int tc_gemm_fused(int M, int N, int K, const float* Ah, const float* Al, int lda,
                  const float* Bh, const float* Bl, int ldb, float* C, int ldc,
                  const float* bias, int* err, cudaStream_t st, const char* who,
                  const int* gate, const TcEpi& ep) {
  if (M == 0 || N == 0) return VCB_OK;
  // Plain stores of wide outputs take 128 x 256 tiles (half the A traffic
  // per FLOP) when that still gives every SM a tile; the fused epilogues and
  // everything else take 128 x 128 tiles (twice the epilogue warps per
  // output column, and more tiles per CTA to overlap them with the MMAs).
  const long long m_tiles = (M + TC_BM - 1) / TC_BM;
  const int bn = (ep.mode == kEpiStore && N > 128 && m_tiles * ((N + 255) / 256) >= sm_count())
                     ? 256 : 128;
  CUtensorMap mAh, mAl, mBh, mBl;
  int rc = make_map(&mAh, Ah, M, K, lda, TC_BM, who);
  if (!rc) rc = make_map(&mAl, Al, M, K, lda, TC_BM, who);
  if (!rc) rc = make_map(&mBh, Bh, N, K, ldb, bn, who);
  if (!rc) rc = make_map(&mBl, Bl, N, K, ldb, bn, who);
  if (rc) return rc;
  if (ep.mode != kEpiStore) {
    // fused epilogues index with 32-bit offsets
    const long long boxes = M / std::max(ep.Q, 1) + 1;
    const long long lim = 0x7fffffffLL;
    if ((long long)M * std::max(std::max(ldc, ep.ldo), std::max(ep.ldrec, ep.ldd)) >= lim ||
        boxes * N >= lim || (ep.part && (long long)M * ep.ldpart >= lim))
      return fail(VCB_ERR_UNSUPPORTED, "%s: operands beyond 32-bit offsets", who);
  }
  auto al16 = [](const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; };
  const bool vec = N % 4 == 0 && ldc % 4 == 0 && al16(C) && al16(bias) && al16(ep.pos) &&
                   al16(ep.rx) && al16(ep.beta) && al16(ep.bnext) && al16(ep.xl) &&
                   al16(ep.xh) && al16(ep.rec) && al16(ep.out_hi) && al16(ep.out_lo) &&
                   al16(ep.dcontrib) && ep.ldrec % 4 == 0 && ep.ldo % 4 == 0 && ep.ldd % 4 == 0;
  TcArgs args{M, N, K, ldc, C, bias, err, gate, vec ? 1 : 0, ep};
  const long long tiles = m_tiles * ((N + bn - 1) / bn);
  if (tiles > 0x7fffffffLL) return fail(VCB_ERR_UNSUPPORTED, "%s: %lld output tiles", who, tiles);
  const int grid = (int)std::min<long long>(tiles, sm_count());  // persistent: one CTA per SM
  rc = bn == 256 ? launch_tc<256, kEpiStore>(grid, mAh, mAl, mBh, mBl, args, st)  // store only
                 : launch_mode(grid, mAh, mAl, mBh, mBl, args, st);
  if (rc) return rc;
  return check_launch(who);
}

int tc_gemm_3xtf32(int M, int N, int K, const float* Ah, const float* Al, int lda,
                   const float* Bh, const float* Bl, int ldb, float* C, int ldc,
                   const float* bias, int* err, cudaStream_t st, const char* who,
                   const int* gate) {
  return tc_gemm_fused(M, N, K, Ah, Al, lda, Bh, Bl, ldb, C, ldc, bias, err, st, who, gate,
                       TcEpi{});
}

int tf32_split(long long n, const float* x, float* hi, float* lo, cudaStream_t st) {
  if (n <= 0) return VCB_OK;
  const int blocks = (int)std::min<long long>((n + 255) / 256, 148LL * 32);
  tf32_split_kernel<<<blocks, 256, 0, st>>>(n, x, hi, lo);
  return check_launch("vcb_tf32_split");
}

}  // namespace vcb

extern "C" int vcb_tf32_split(int64_t n, const float* x, float* hi, float* lo, void* stream) {
  using namespace vcb;
  if (n < 0 || (n > 0 && (!x || !hi || !lo))) return fail(VCB_ERR_INVALID, "vcb_tf32_split: bad arguments");
  return tf32_split(n, x, hi, lo, static_cast<cudaStream_t>(stream));
}

extern "C" int vcb_tc_gemm_gated(int32_t M, int32_t N, int32_t K, const float* A_hi,
                                 const float* A_lo, int32_t lda, const float* B_hi,
                                 const float* B_lo, int32_t ldb, const float* bias, float* C,
                                 int32_t ldc, int32_t* err, const int32_t* gate, void* stream) {
  using namespace vcb;
  if (M < 0 || N < 0 || K <= 0 || ldc < N)
    return fail(VCB_ERR_INVALID, "vcb_tc_gemm_gated: M=%d N=%d K=%d ldc=%d", M, N, K, ldc);
  if (M == 0 || N == 0) return VCB_OK;
  if (!A_hi || !A_lo || !B_hi || !B_lo || !C || !err)
    return fail(VCB_ERR_INVALID, "vcb_tc_gemm_gated: NULL pointer");
  return tc_gemm_3xtf32(M, N, K, A_hi, A_lo, lda, B_hi, B_lo, ldb, C, ldc, bias, err,
                        static_cast<cudaStream_t>(stream), "vcb_tc_gemm_gated", gate);
}

extern "C" int vcb_tc_gemm(int32_t M, int32_t N, int32_t K, const float* A_hi, const float* A_lo,
                           int32_t lda, const float* B_hi, const float* B_lo, int32_t ldb,
                           const float* bias, float* C, int32_t ldc, int32_t* err,
                           void* stream) {
  using namespace vcb;
  if (M < 0 || N < 0 || K <= 0 || ldc < N)
    return fail(VCB_ERR_INVALID, "vcb_tc_gemm: M=%d N=%d K=%d ldc=%d", M, N, K, ldc);
  if (M == 0 || N == 0) return VCB_OK;
  if (!A_hi || !A_lo || !B_hi || !B_lo || !C || !err)
    return fail(VCB_ERR_INVALID, "vcb_tc_gemm: NULL pointer");
  return tc_gemm_3xtf32(M, N, K, A_hi, A_lo, lda, B_hi, B_lo, ldb, C, ldc, bias, err,
                        static_cast<cudaStream_t>(stream), "vcb_tc_gemm");
}
