// W4A16 GEMV for decode shapes (M <= 8) on large layers, stream-K over the
// SMs, on mma.sync tiles of exactly decoded fp16 operands.
//
// out[M, N] = A[M, K] @ (q[K, N] * s[K/g, N])  -- gemm_int4.int4_gemm
// (gemm_int4.py:75-92) with group scales, q unpacked from Wp[K, N/2] in the
// reference's nibble order (gemm_int4.py:43-50, pack_int4_n at :65-72).
//
// At M <= 8 the layer is a stream over the packed weights (K*N/2 bytes) with
// 2*M*K*N flops, far below one flop per byte. The decode is the four-tile
// form of the tile decode in w4a16_mma.cuh (2 PRMT + 4 LOP3 + 1 mma per 8
// weights and lane) on 16 mma warps: with two warps per scheduler the decode's
// dependency chains left the issue slots ~65 % idle.
//
//  * Units. The weights are cut into units of 64 rows x 1024 columns (64
//    rows of 512 contiguous bytes, 32 KB): wide enough that each DRAM page a
//    unit opens serves half a kilobyte (units one 64-byte column strip wide
//    streamed at about half the HBM rate). A "slice" is a 1024-column strip,
//    KB units tall. Warp w of 16 owns columns [64w, 64w + 64) of every unit
//    (a quarter of one of the unit's four TMA boxes of 64 rows x 128 bytes,
//    128-byte swizzled), its own accumulators: no cross-warp reduction.
//  * Work split (stream-K): units numbered slice-major, CTA c of G (one per
//    SM) takes [U*c/G, U*(c+1)/G). A CTA's range covers parts of a few slices
//    ("segments"). A segment that is a whole slice is stored directly;
//    otherwise the CTA writes its partial to the workspace (slot c + slice,
//    unique per segment) and bumps the slice's arrival counter with an
//    acq_rel atomic; the last arriver sums the slice's partials in CTA order,
//    stores, and re-arms the counter. Fixed summation order: deterministic
//    for a given SM count.
//  * Pipeline. Warp 16 (one thread) is the TMA producer of a ring of as many
//    unit slots as shared memory holds (six, ~220 KB): per unit the
//    activation tile A[0:M, k0:k0+64] and the unit's group-scale row (one
//    mbarrier), then the four weight boxes (one mbarrier each). Warp 17
//    turns each unit's activations into the B fragments the 16 mma warps
//    share (one mbarrier), so their loop is the tile decode alone.
//    Before griddepcontrol.wait it only prefetches weights and scales into
//    L2 (a hint that cannot return stale data), so with programmatic
//    dependent launch the DRAM fetch overlaps the previous kernel's tail;
//    every load into shared memory and every global write comes after the
//    wait. Rows past K and columns past N arrive as zeros (TMA bounds fill).
//  * Arithmetic. The B fragments hold the unit's 64 activation rows in fp16,
//    bf16 rows scaled by 2^S_m per output row m (S from the unit's 64 rows,
//    so the largest magnitude lies in [2^14, 2^15)); the prep warp also
//    stores 2^-S_m and -8 * 2^-24 * sum(a') per row, the tiles' starting
//    value that removes the +8 offsets. Each mma warp runs the tile decode
//    and folds the tiles' fp32 sums with the group scale (the unit lies in
//    one group: groups are multiples of 64) times 2^-S_m. The result is the
//    reference's fp32 dequantize-then-matmul up to summation order.
#include "pk_common.cuh"

#include <cstring>
#include <type_traits>

#include "pk_internal.h"
#include "w4a16_mma.cuh"

namespace pk {
namespace {

using w4mma::Consts;
using w4mma::blk_words;
using w4mma::kKSteps;
using w4mma::kMaxM;
using w4mma::kBoxRowBytes4;  // 128: four warps' 256 columns of one row

constexpr int kWarps = 16;
constexpr int kProducerWarp = kWarps;
constexpr int kPrepWarp = kWarps + 1;
constexpr int kThreads = (kWarps + 2) * 32;
constexpr int kMmaThreads = kWarps * 32;
constexpr int kUnitRows = 64;                         // K rows per unit
constexpr int kWarpCols = 64;                         // columns per warp
constexpr int kSliceCols = kWarps * kWarpCols;        // 1024 columns per slice
constexpr int kBoxes = kWarps / 4;                    // TMA boxes per unit, four warps each
constexpr int kBoxBytes = kUnitRows * kBoxRowBytes4;  // 8192
constexpr int kWBytes = kBoxes * kBoxBytes;           // 32768
constexpr int kSBytes = kSliceCols * 2;               // one group-scale row
constexpr int kSBox = 256;                            // scales per TMA box (box limit 256)

// A ring slot: the unit's weights (four boxes), its group-scale row
// and activations (TMA), then what the prep warp makes of the activations:
// the fp16 B fragments, 2^-S_m and the +8 offsets' starting value per output
// row (8 entries each, whatever M).
template <int M>
struct Cfg {
  static constexpr int kABytes = kUnitRows * 2 * M;  // [m][64] activations
  static constexpr int kActOff = kWBytes + kSBytes;
  static constexpr int kFragOff = kActOff + (kABytes + 15) / 16 * 16;
  static constexpr int kFragBytes = kKSteps * blk_words<M>() * 4;
  static constexpr int kPwOff = kFragOff + kFragBytes;
  static constexpr int kOffOff = kPwOff + 8 * 4;
  static constexpr int kSlotBytes = (kOffOff + 8 * 4 + 1023) / 1024 * 1024;
  // as many ring slots as the shared memory holds
  static constexpr int kStages = (227 * 1024 - 1024 - 512) / kSlotBytes;
  static constexpr int kRingBytes = kStages * kSlotBytes;
  static constexpr int kBarOff = kRingBytes;
  // per slot: activations + scales, B fragments ready, four weight boxes, release
  static constexpr int kBarsPerSlot = 2 + kBoxes + 1;
  static constexpr int kSmemBytes = kBarOff + kBarsPerSlot * kStages * 8 + 16 + 1024;
  static_assert(kStages >= 4, "a ring of at least four units");
  static_assert(kSmemBytes <= 227 * 1024, "shared memory");
};

// CTA owning unit u under the stream-K split [U*c/G, U*(c+1)/G).
__device__ __host__ __forceinline__ int64_t unit_owner(int64_t u, int64_t U, int64_t G) {
  return ((u + 1) * G + U - 1) / U - 1;
}

__device__ __forceinline__ unsigned atomic_add_acq_rel(unsigned* p, unsigned v) {
  unsigned old;
  asm volatile("atom.add.acq_rel.gpu.global.u32 %0, [%1], %2;"
               : "=r"(old)
               : "l"(p), "r"(v)
               : "memory");
  return old;
}

struct GemvParams {
  int N, K, group;
  int group_shift;     // log2(group) when group is a power of two, else -1
  float scalar_scale;
  int out_dtype;
  int64_t ldo;
  int64_t n_offset;    // column of this slice in the output rows
  int world, rank;     // output copies (1: just peer_out[0])
  uint64_t peer_out[kMaxPeers];   // output buffers, peer_out[rank] is this GPU's
  uint64_t peer_flag[kMaxPeers];  // arrival count; this GPU's is followed by its expected count
  unsigned* done;      // CTA completion counter (sharded exchange), zero between calls
  float* partials;
  unsigned* sems;
  int* status;
  uint64_t* stamps;    // optional per-CTA phase times (pk_debug_phase_stamps)
};

// Write column `col` of output row m into every copy of the output.
__device__ __forceinline__ void store_col(const GemvParams& p, int m, int64_t col, float v) {
  const int64_t idx = m * p.ldo + p.n_offset + col;
  for (int r = 0; r < p.world; ++r) {
    if (p.out_dtype == PK_BF16)
      reinterpret_cast<__nv_bfloat16*>(p.peer_out[r])[idx] = __float2bfloat16_rn(v);
    else
      reinterpret_cast<float*>(p.peer_out[r])[idx] = v;
  }
}

// After every CTA's stores: the shared flag barrier of the fused exchange.
__device__ __forceinline__ void sharded_finish(const GemvParams& p, bool stored) {
  peer_exchange_finish(p, stored, p.status, kSiteGemvPeers, gridDim.x);
}

// Index of the scale group holding K row `row` (a shift for power-of-two groups).
__device__ __host__ __forceinline__ int group_of(int row, const GemvParams& p) {
  return p.group_shift >= 0 ? (row >> p.group_shift) : row / p.group;
}

template <int M, typename T, bool kGrouped>
__global__ void __launch_bounds__(kThreads, 1)
    w4a16_gemv_kernel(const __grid_constant__ CUtensorMap tmW,
                      const __grid_constant__ CUtensorMap tmA,
                      const __grid_constant__ CUtensorMap tmS, const GemvParams p,
                      const Consts dc) {
  using C = Cfg<M>;
  constexpr bool kBf16 = std::is_same<T, __nv_bfloat16>::value;
  constexpr int kOut = M * kSliceCols;  // a segment's sums: [m][column]
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  const uint32_t sbase = smem_u32(smem);
  uint64_t* afull = reinterpret_cast<uint64_t*>(smem + C::kBarOff);  // [slot]: activations, scales
  uint64_t* bready = afull + C::kStages;                              // [slot]: B fragments
  uint64_t* wfull = bready + C::kStages;                              // [slot][box]: weights
  uint64_t* empty = wfull + C::kStages * kBoxes;                      // [slot]
  volatile int* last_flag = reinterpret_cast<volatile int*>(empty + C::kStages);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int NS = (p.N + kSliceCols - 1) / kSliceCols;
  const int KB = (p.K + kUnitRows - 1) / kUnitRows;
  const int64_t U = static_cast<int64_t>(NS) * KB;
  const int64_t G = gridDim.x;
  const int64_t cta = blockIdx.x;
  const int64_t u0 = U * cta / G;
  const int64_t u1 = U * (cta + 1) / G;
  const int n_units = static_cast<int>(u1 - u0);
  bool stored = false;  // this thread wrote output (sharded exchange: fence before arriving)
  uint64_t t_entry = 0, t_wait = 0, t_first = 0, t_comp = 0;
  bool was_last = false;
  const bool stamp = p.stamps != nullptr && threadIdx.x == 0;
  if (stamp) t_entry = globaltimer();

  if (threadIdx.x == 0) {
    for (int s = 0; s < C::kStages; ++s) {
      mbar_init(&afull[s], 1);
      mbar_init(&bready[s], 1);
      for (int b = 0; b < kBoxes; ++b) mbar_init(&wfull[s * kBoxes + b], 1);
      mbar_init(&empty[s], kWarps);
    }
    fence_barrier_init();
  }
  __syncthreads();
  // Dependents may start their own prologue (an L2 prefetch of their weights)
  // now; they wait for this grid before touching anything it writes.
  griddep_launch_dependents();

  if (warp == kProducerWarp) {
    if (lane == 0) {
      const uint32_t tx_a = C::kABytes + (kGrouped ? kSBytes : 0);
      tma_prefetch_desc(&tmW);
      tma_prefetch_desc(&tmA);
      if constexpr (kGrouped) tma_prefetch_desc(&tmS);
      const int pre = n_units < C::kStages ? n_units : C::kStages;
      for (int i = 0, s = static_cast<int>(u0 / KB), kb = static_cast<int>(u0 % KB); i < pre;
           ++i) {
        for (int b = 0; b < kBoxes; ++b)
          tma_prefetch_l2_2d(&tmW, s * (kSliceCols / 2) + b * kBoxRowBytes4, kb * kUnitRows);
        if constexpr (kGrouped)
          for (int h = 0; h < kSliceCols / kSBox; ++h)
            tma_prefetch_l2_2d(&tmS, s * kSliceCols + h * kSBox, group_of(kb * kUnitRows, p));
        if (++kb == KB) kb = 0, ++s;
      }
      griddep_wait();
      int issued = 0;
      bool ok = true;
      int slice = static_cast<int>(u0 / KB);
      int kb = static_cast<int>(u0 % KB);
      for (int i = 0, slot = 0, round = 0; i < n_units; ++i) {
        // a suspending wait: a spinning one would take issue slots from the
        // mma warps sharing this warp's scheduler
        if (i >= C::kStages &&
            !mbar_wait_sleep(&empty[slot], (round - 1) & 1, p.status, kSiteGemvProducer)) {
          ok = false;
          break;
        }
        const int k0 = kb * kUnitRows;
        uint8_t* base = smem + slot * C::kSlotBytes;
        mbar_arrive_expect_tx(&afull[slot], tx_a);
        tma_load_2d(base + C::kActOff, &tmA, &afull[slot], k0, 0);
        if constexpr (kGrouped)
          for (int h = 0; h < kSliceCols / kSBox; ++h)
            tma_load_2d(base + kWBytes + h * kSBox * 2, &tmS, &afull[slot],
                        slice * kSliceCols + h * kSBox, group_of(k0, p));
        // the four boxes of a unit are 512 contiguous bytes of each row
        for (int b = 0; b < kBoxes; ++b) {
          mbar_arrive_expect_tx(&wfull[slot * kBoxes + b], kBoxBytes);
          tma_load_2d(base + b * kBoxBytes, &tmW, &wfull[slot * kBoxes + b],
                      slice * (kSliceCols / 2) + b * kBoxRowBytes4, k0);
        }
        issued = i + 1;
        if (++kb == KB) kb = 0, ++slice;
        if (++slot == C::kStages) slot = 0, ++round;
      }
      if (!ok) {
        // let copies already issued land before the CTA's shared memory is released
        const int first = issued > C::kStages ? issued - C::kStages : 0;
        for (int i = first; i < issued; ++i) {
          const int s = i % C::kStages;
          const uint32_t par = (i / C::kStages) & 1;
          mbar_wait(&afull[s], par, nullptr, 0);
          for (int b = 0; b < kBoxes; ++b) mbar_wait(&wfull[s * kBoxes + b], par, nullptr, 0);
        }
      }
    }
    __syncwarp();
  } else if (warp == kPrepWarp) {
    // ---------------- prep warp: activations -> B fragments ----------------
    // Lane l takes rows 2l, 2l + 1 of the unit: bf16 rows scaled by 2^S_m per
    // output row m (S_m from the unit's 64 rows), the offsets' starting value
    // -8 * 2^-24 * sum(a') per row. No global access: no dependency wait.
    bool failed = false;
    for (int i = 0, slot = 0, round = 0; i < n_units;
         ++i, slot = (slot + 1 == C::kStages ? 0 : slot + 1), round += (slot == 0)) {
      const uint32_t base = sbase + slot * C::kSlotBytes;
      if (!failed && !mbar_wait_sleep(&afull[slot], round & 1, p.status, kSiteGemvConsumer))
        failed = true;
      uint32_t raw[M];
#pragma unroll
      for (int m = 0; m < M; ++m) raw[m] = lds_u32(base + C::kActOff + (m * kUnitRows + 2 * lane) * 2);
#pragma unroll
      for (int m = 0; m < M; ++m) {
        const int S =
            kBf16 ? w4mma::scale_exp(__reduce_max_sync(0xffffffffu, w4mma::bf16x2_emax(raw[m])))
                  : 0;
        const uint32_t h2 = w4mma::to_f16x2<T>(raw[m], w4mma::exp2i(S));
        w4mma::sts_u32(base + C::kFragOff + w4mma::bfrag_store_off<M>(lane, m), h2);
        const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&h2));
        float s = f.x + f.y;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
        if (lane == 0) {
          sts_f32(base + C::kPwOff + m * 4, w4mma::exp2i(-S));
          sts_f32(base + C::kOffOff + m * 4, s * -4.76837158203125e-07f);  // -8 * 2^-24
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&bready[slot]);
    }
  } else {
    // ---------------- mma warps ----------------
    griddep_wait();
    if (stamp) t_wait = globaltimer();
    const int g = lane >> 2, t = lane & 3;  // the mma fragments' group and thread-in-group
    float tot[4][4];  // tile j: columns 8g + 2j ([0], [1]) and + 1 ([2], [3]); rows 2t, 2t + 1
#pragma unroll
    for (int j = 0; j < 4; ++j)
#pragma unroll
      for (int e = 0; e < 4; ++e) tot[j][e] = 0.0f;
    const uint32_t bfrag_lane = C::kFragOff + ((g < M ? g : M - 1) * 4 + t) * 8;
    uint32_t roff[4];  // the lane's rows in its box (four warps per box)
    w4mma::lane_rows4(lane, warp & 3, roff);
    const uint32_t box_off = (warp >> 2) * kBoxBytes;
    bool failed = false;
    int slice = static_cast<int>(u0 / KB);
    int kb = static_cast<int>(u0 % KB);
    for (int i = 0, slot = 0, round = 0; i < n_units;
         ++i, slice += (kb + 1 == KB), kb = (kb + 1 == KB ? 0 : kb + 1),
             slot = (slot + 1 == C::kStages ? 0 : slot + 1), round += (slot == 0)) {
      const uint32_t base = sbase + slot * C::kSlotBytes;
      if (!failed && !mbar_wait_sleep(&bready[slot], round & 1, p.status, kSiteGemvConsumer))
        failed = true;
      uint32_t bf[kKSteps][2];
      w4mma::load_bfrags<M>(base + bfrag_lane, bf);
      const uint2 pwv = w4mma::lds_v2(base + C::kPwOff + 8 * t);   // rows 2t, 2t + 1
      const uint2 ofv = w4mma::lds_v2(base + C::kOffOff + 8 * t);
      const float pw0 = __uint_as_float(pwv.x), pw1 = __uint_as_float(pwv.y);
      const float o0 = __uint_as_float(ofv.x), o1 = __uint_as_float(ofv.y);
      const float doff[4] = {o0, o1, 16.0f * o0, 16.0f * o1};
      if (!failed && !mbar_wait_sleep(&wfull[slot * kBoxes + (warp >> 2)], round & 1, p.status,
                                      kSiteGemvConsumer))
        failed = true;
      if (stamp && i == 0) t_first = globaltimer();
      float acc[4][4];
      w4mma::tile_loop4(base + box_off, roff, bf, doff, dc, acc);
      w4mma::fold4<T, kGrouped>(acc, base + kWBytes + (warp * kWarpCols + 8 * g) * 2,
                                p.scalar_scale, pw0, pw1, tot);
      __syncwarp();  // every lane is done with the slot
      if (lane == 0) mbar_arrive(&empty[slot]);

      const bool seg_end = (i + 1 == n_units) || (kb + 1 == KB);
      if (!seg_end) continue;

      // ---- end of a segment: each warp holds its own 128 columns ----
      if (stamp) t_comp = globaltimer();
      const int64_t cfirst = unit_owner(static_cast<int64_t>(slice) * KB, U, G);
      const int64_t clast = unit_owner(static_cast<int64_t>(slice) * KB + KB - 1, U, G);
      const bool whole = cfirst == clast;
      float* mine = p.partials + (cta + slice) * kOut;
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const int n = 2 * t + e;
        if (n < M) {
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            // undo 2^-24 (low nibbles) and 2^-20 (high nibbles)
            const float lo = tot[j][e] * 16777216.0f, hi = tot[j][2 + e] * 1048576.0f;
            const int c = warp * kWarpCols + 8 * g + 2 * j;
            if (whole) {
              const int64_t col = static_cast<int64_t>(slice) * kSliceCols + c;
              if (col < p.N) store_col(p, n, col, lo), stored = true;
              if (col + 1 < p.N) store_col(p, n, col + 1, hi);
            } else {
              __stcg(reinterpret_cast<float2*>(mine + n * kSliceCols + c), make_float2(lo, hi));
            }
          }
        }
      }
#pragma unroll
      for (int j = 0; j < 4; ++j)
#pragma unroll
        for (int e = 0; e < 4; ++e) tot[j][e] = 0.0f;
      if (whole) continue;
      named_bar_sync(1, kMmaThreads);  // every warp's partial is written
      const int x = threadIdx.x;
      if (x == 0) {
        // release: the CTA's partial (ordered before by the barrier) becomes
        // visible with the count; acquire: the last arriver sees every partial
        const unsigned arrived = atomic_add_acq_rel(&p.sems[slice], 1u);
        *last_flag = arrived == static_cast<unsigned>(clast - cfirst) ? 1 : 0;
      }
      named_bar_sync(1, kMmaThreads);
      if (*last_flag) {
        was_last = true;
        // thread x sums outputs x, x + 256, ... of [m][column], in CTA order,
        // with a batch of CTAs' loads in flight before the adds
        constexpr int kPer = kOut / kMmaThreads;
        constexpr int kBatch = 16 / kPer > 0 ? 16 / kPer : 1;
        float sum[kPer];
#pragma unroll
        for (int k = 0; k < kPer; ++k) sum[k] = 0.0f;
        for (int64_t c0 = cfirst; c0 <= clast; c0 += kBatch) {
          float xs[kBatch][kPer];
#pragma unroll
          for (int b = 0; b < kBatch; ++b) {
            if (c0 + b <= clast) {
              const float* src = p.partials + (c0 + b + slice) * kOut;
#pragma unroll
              for (int k = 0; k < kPer; ++k) xs[b][k] = __ldcg(src + x + k * kMmaThreads);
            }
          }
#pragma unroll
          for (int b = 0; b < kBatch; ++b) {
            if (c0 + b <= clast) {
#pragma unroll
              for (int k = 0; k < kPer; ++k) sum[k] += xs[b][k];
            }
          }
        }
#pragma unroll
        for (int k = 0; k < kPer; ++k) {
          const int o = x + k * kMmaThreads;
          const int64_t col = static_cast<int64_t>(slice) * kSliceCols + o % kSliceCols;
          if (col < p.N) {
            store_col(p, o / kSliceCols, col, sum[k]);
            stored = true;
          }
        }
        if (x == 0) p.sems[slice] = 0u;  // re-arm for the next call
      }
      named_bar_sync(1, kMmaThreads);  // last_flag is rewritten by the next segment
    }
  }

  if (stamp) {
    uint32_t smid;
    asm volatile("mov.u32 %0, %%smid;" : "=r"(smid));
    uint64_t* st = p.stamps + static_cast<int64_t>(blockIdx.x) * 8;
    st[0] = t_entry;
    st[1] = t_wait;
    st[2] = t_first;
    st[3] = t_comp;
    st[4] = globaltimer();
    st[5] = smid;
    st[6] = static_cast<uint64_t>(n_units) | (was_last ? (1ull << 32) : 0ull);  // summed a slice
  }
  if (p.world > 1) sharded_finish(p, stored);
  if (stamp) p.stamps[static_cast<int64_t>(blockIdx.x) * 8 + 7] = globaltimer();
}

CUtensorMapDataType tmap_type16(int dt) {
  return dt == PK_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
}

int64_t gemv_units(int64_t N, int64_t K) {
  return ((N + kSliceCols - 1) / kSliceCols) * ((K + kUnitRows - 1) / kUnitRows);
}

// Stream-K grid: one CTA per SM, at most one CTA per unit.
int64_t gemv_grid(int64_t N, int64_t K) {
  const int64_t U = gemv_units(N, K);
  const int64_t cap = static_cast<int64_t>(num_sms());
  return U < cap ? U : cap;
}

}  // namespace

bool gemv_preferred(int64_t M, int64_t N, int64_t K) {
  // Faster than the tcgen05 decode kernel unless a slice's partial sums come
  // from too many CTAs: the fan-in, CTAs per 1024-column slice (~G / NS),
  // costs the slice's last arriver one L2 round trip per batch of partials,
  // and batches shrink as M grows. Measured on B200 (us, stream-K vs decode):
  // M=1: fan-in 11-37 wins (14336x4096 14.3 vs 28.9, 4096x11008 13.3 vs
  // 14.7), 48 and 74 lose (3072^2 8.2 vs 6.4, 2048x8192 11.5 vs 10.5); M=2..4:
  // 14-25 win (6144^2 M=4 12.3 vs 17.2), 37 loses (4096x11008 M=4 21.5 vs
  // 14.6); M=8: 14 wins (11008x4096 22.5 vs 23.3), 19 loses (8192^2 26.2 vs
  // 23.8). Llama-70B up_proj (fan-in 6): M=1 32.4 vs 66, M=8 40.1 vs 84.
  if (M < 1 || M > kMaxM) return false;
  const int64_t NS = (N + kSliceCols - 1) / kSliceCols;
  const int64_t G = gemv_grid(N, K);
  const int64_t fan_in = (G + NS - 1) / NS;
  const int64_t limit = M == 1 ? 40 : (M <= 4 ? 25 : 14);
  return fan_in <= limit;
}

bool gemv_supported(int64_t M, int64_t N, int64_t K, int group, const void* scales, int64_t lda,
                    const void* a, const void* wp) {
  if (M < 1 || M > kMaxM) return false;
  if (N < 128 || N % 32 != 0 || K < kUnitRows) return false;
  if (N > (1ll << 30) || K > (1ll << 30)) return false;
  if ((N + kSliceCols - 1) / kSliceCols >= kMaxCounters) return false;  // the last: sharded calls
  if (lda % 8 != 0 || (reinterpret_cast<uintptr_t>(a) & 15) != 0) return false;
  if ((reinterpret_cast<uintptr_t>(wp) & 15) != 0) return false;
  if (scales != nullptr &&
      (group <= 0 || group % kUnitRows != 0 || (reinterpret_cast<uintptr_t>(scales) & 15) != 0))
    return false;
  return true;
}

size_t gemv_workspace_bytes(int64_t M, int64_t N, int64_t K) {
  const int64_t NS = (N + kSliceCols - 1) / kSliceCols;
  const int64_t KB = (K + kUnitRows - 1) / kUnitRows;
  const int64_t U = NS * KB;
  const int64_t G = gemv_grid(N, K);
  bool split = false;
  for (int64_t j = 0; j < NS && !split; ++j)
    split = unit_owner(j * KB, U, G) != unit_owner(j * KB + KB - 1, U, G);
  if (!split) return 0;
  return kCounterBytes + static_cast<size_t>(G + NS) * M * kSliceCols * sizeof(float);
}

cudaError_t launch_w4a16_gemv(const DecodeArgs& a, cudaStream_t s, const char** why,
                              const OutputShard* shard) {
  if (a.M < 1 || a.M > kMaxM) {
    *why = "GEMV: 1 <= M <= 8";
    return cudaErrorInvalidValue;
  }
  CUtensorMap tmW, tmA, tmS;
  const CUtensorMapDataType dt = tmap_type16(a.a_dtype);
  if (!encode_tmap_2d(&tmW, CU_TENSOR_MAP_DATA_TYPE_UINT8, a.wp, a.N / 2, a.K, a.N / 2,
                      kBoxRowBytes4, kUnitRows, CU_TENSOR_MAP_SWIZZLE_128B, why))
    return cudaErrorInvalidValue;
  if (!encode_tmap_2d(&tmA, dt, a.a, a.K, a.M, a.lda * 2, kUnitRows, static_cast<uint32_t>(a.M),
                      CU_TENSOR_MAP_SWIZZLE_NONE, why))
    return cudaErrorInvalidValue;
  const bool grouped = a.scales != nullptr;
  GemvParams p{};
  p.N = static_cast<int>(a.N);
  p.K = static_cast<int>(a.K);
  p.group = grouped ? a.group : kUnitRows;
  p.group_shift = -1;
  for (int sh = 0; sh < 31; ++sh)
    if ((1 << sh) == p.group) p.group_shift = sh;
  p.scalar_scale = a.scalar_scale;
  p.out_dtype = a.out_dtype;
  p.ldo = a.ldo;
  p.world = 1;
  p.rank = 0;
  p.n_offset = 0;
  p.peer_out[0] = reinterpret_cast<uint64_t>(a.out);
  if (shard != nullptr) {
    if (shard->world < 1 || shard->world > kMaxPeers || shard->done == nullptr) {
      *why = "sharded GEMV: 1 <= world <= 8 and a workspace are required";
      return cudaErrorInvalidValue;
    }
    p.world = shard->world;
    p.rank = shard->rank;
    p.n_offset = shard->n_offset;
    for (int r = 0; r < shard->world; ++r) {
      p.peer_out[r] = shard->peer_out[r];
      p.peer_flag[r] = shard->peer_flag[r];
    }
    p.done = shard->done;
  }
  p.partials = a.partials;
  p.sems = a.sems;
  p.status = a.status;
  p.stamps = phase_stamps(static_cast<size_t>(gemv_grid(a.N, a.K)));
  if (grouped) {
    if (a.group % kUnitRows != 0) {
      *why = "GEMV: the group size must be a multiple of 64";
      return cudaErrorInvalidValue;
    }
    const int64_t groups = (a.K + a.group - 1) / a.group;
    if (!encode_tmap_2d(&tmS, dt, a.scales, a.N, groups, a.N * 2, kSBox, 1,
                        CU_TENSOR_MAP_SWIZZLE_NONE, why))
      return cudaErrorInvalidValue;
  } else {
    std::memcpy(&tmS, &tmW, sizeof(tmS));  // unused
  }
  const int64_t G = gemv_grid(a.N, a.K);
  if (gemv_workspace_bytes(a.M, a.N, a.K) > 0 && (a.partials == nullptr || a.sems == nullptr)) {
    *why = "the split-K GEMV needs a workspace";
    return cudaErrorInvalidValue;
  }
  const Consts dc = w4mma::consts();

  auto launch = [&](auto kernel, int smem_bytes) -> cudaError_t {
    cudaError_t e = set_max_smem(reinterpret_cast<const void*>(kernel), smem_bytes);
    if (e != cudaSuccess) return e;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(static_cast<unsigned>(G), 1, 1);
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = smem_bytes;
    cfg.stream = s;
    cudaLaunchAttribute attr;
    attr.id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr.val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = &attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kernel, tmW, tmA, tmS, p, dc);
  };
  auto by_m = [&](auto mtag) -> cudaError_t {
    constexpr int kM = decltype(mtag)::value;
    constexpr int kBytes = Cfg<kM>::kSmemBytes;
    if (a.a_dtype == PK_BF16)
      return grouped ? launch(w4a16_gemv_kernel<kM, __nv_bfloat16, true>, kBytes)
                     : launch(w4a16_gemv_kernel<kM, __nv_bfloat16, false>, kBytes);
    return grouped ? launch(w4a16_gemv_kernel<kM, __half, true>, kBytes)
                   : launch(w4a16_gemv_kernel<kM, __half, false>, kBytes);
  };
  switch (a.M) {
    case 1: return by_m(std::integral_constant<int, 1>{});
    case 2: return by_m(std::integral_constant<int, 2>{});
    case 3: return by_m(std::integral_constant<int, 3>{});
    case 4: return by_m(std::integral_constant<int, 4>{});
    case 5: return by_m(std::integral_constant<int, 5>{});
    case 6: return by_m(std::integral_constant<int, 6>{});
    case 7: return by_m(std::integral_constant<int, 7>{});
    default: return by_m(std::integral_constant<int, 8>{});
  }
}

}  // namespace pk
