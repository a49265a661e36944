// W4A16 decode GEMV (M = 1..3) for layers that fit one wave of the SMs, on the
// CUDA cores, with the K split reduced inside thread-block clusters.
//
// out[1, N] = A[1, K] @ (q[K, N] * s[K/128, N])  -- gemm_int4.int4_gemm
// (gemm_int4.py:75-92) with group scales, q unpacked from Wp[K, N/2] in the
// reference's nibble order (gemm_int4.py:43-50, pack_int4_n at :65-72).
//
// At 4096 x 4096 the whole layer is 8.4 MB, 1.3 us of HBM time, and the
// launch-to-launch chain of a decode step costs about a microsecond by
// itself; what decides the time per GEMM is how much of each launch's work
// overlaps the launch before it, and how short its own critical path is.
//
//  * Partition. The columns are cut into strips of 128 (64 packed bytes per
//    row); each strip's K rows are split over `split` CTAs (split <= 4),
//    which form one thread-block cluster. CTA r of a strip owns units
//    [U*r/split, U*(r+1)/split) of 512 rows (U = K/512). strips * split <=
//    the SM count, so the grid is one wave of one CTA per SM.
//  * Footprint. ~145 KB of shared memory (a 4-slot ring), so that no SM
//    holds two CTAs of one grid: with room for two, CTAs started early by
//    programmatic dependent launch were packed two to an SM on ~12 SMs, whose
//    doubled arithmetic then set every launch's critical path. Clusters of 4:
//    at one CTA per SM a B200 holds 33 of them at once but only 15 clusters
//    of 8, which left a sixteenth waiting for the first ones to finish.
//  * Loads. Warp 8 (one thread) is the TMA producer of a 4-slot ring: per
//    unit four 128-row weight boxes (each with its own mbarrier, so a warp
//    starts when the box holding its rows lands), the unit's four group-scale
//    rows, and, on a separate barrier, the unit's 512 activations. Before
//    griddepcontrol.wait it prefetches the CTA's weights into L2 (a hint that
//    cannot return stale data); with weight staging on (pk_set_weight_staging)
//    it loads the first units' weights and scales into shared memory there
//    instead, and only the activations wait for the previous kernel.
//  * Arithmetic (the CUDA-core GEMV's exact-product scheme, w4a16_gemv.cu,
//    with fewer instructions per word). Warp w takes rows [64w, 64w + 64) of
//    every unit (within one scale group); lane l the word of columns
//    [8(l % 16), 8(l % 16) + 8) in the rows of parity l / 16: one 32-bit word
//    per row, two rows per warp instruction (128 contiguous bytes).
//    XOR-ing the word with 0x88888888 turns every nibble into q + 8 (0..15); nibbles 0-5 are then masked in place (one AND each) and
//    nibbles 6-7 after one right shift by 8, each read as an fp32 bit pattern
//    worth (q + 8) * 16^p * 2^-149 (p = 0..5: subnormal, or the lowest normal
//    binade, exact). Activations are pre-scaled by 2^S with S = clamp(248 -
//    e_max, 30, 127) over the warp's 64 rows, so every product with a
//    non-negligible activation is a normal fp32 number and exact; one packed
//    fma.rn.f32x2 per two weights accumulates them. Per unit the +8 offset is
//    removed with the sum of the scaled activations, 2^(149 - S - 4p) undone
//    (exact) and the fp32 group scale applied: 1 XOR, 1 shift, 8 AND and 4
//    FMA2 per 8 weights. The two row parities of a column meet by a shuffle.
//    All shared-memory traffic uses explicit ld/st.shared.
//  * M > 1. The nibble decode is shared by the M activation rows: per 8
//    weights the XOR, shift and 8 ANDs are done once and 4 FMA2 per row
//    follow, with S, the +8 offset sum and the group fold per row. Measured
//    at 4096^2 against the tensor-core decode kernel: M = 2 6.58 vs 8.39 us,
//    M = 3 7.79 vs 8.49 us, M = 4 9.23 vs 8.49 us (so M <= 3 here).
//  * Reduction. The 8 warps' column sums meet in shared memory; each other
//    CTA of the cluster then pushes its 128 sums into the leader's (rank 0)
//    shared memory with st.async, which completes bytes on the leader's
//    mbarrier, and exits; the leader waits for them (bounded), sums the
//    strip's columns in CTA order and stores them: deterministic, no global
//    workspace, no atomics, and only one CTA per cluster waits or stores
//    (in the sharded exchange, one system-scope fence per cluster).
//  * Placement. The launch also asks for the spread cluster scheduling
//    policy; on its own that did not keep two CTAs off one SM (the shared-
//    memory footprint does).
#include "pk_common.cuh"

#include <cstring>
#include <mutex>
#include <type_traits>

#include "pk_internal.h"

namespace pk {
namespace {

constexpr int kRows = 512;              // K rows per unit
constexpr int kCols = 128;              // columns per strip
constexpr int kRowBytes = kCols / 2;    // packed bytes per row of a strip (64)
constexpr int kWarps = 8;               // dequant/FMA warps
constexpr int kProducerWarp = kWarps;
constexpr int kThreads = (kWarps + 1) * 32;
constexpr int kRowsPerWarp = kRows / kWarps;  // 64: half a scale group
constexpr int kGroup = 128;
constexpr int kSub = 4;
constexpr int kSubRows = kRows / kSub;            // 128
constexpr int kSubWBytes = kSubRows * kRowBytes;  // 8192
constexpr int kABox = 256;                        // activations per TMA box (box limit 256)
constexpr int kMaxSplit = 4;
constexpr int kStages = 4;
constexpr int kWBytes = kRows * kRowBytes;              // 32768
constexpr int kSBytes = (kRows / kGroup) * kCols * 2;   // 1024: four 16-bit scale rows
constexpr int kMaxM = 3;  // M = 4: the tensor-core decode kernel is faster (8.5 vs 9.2 us)
constexpr int kNumBars = kStages * (kSub + 2) + 1;       // full[kSub], afull, empty per slot; pushed

// Shared-memory layout for M activation rows.
template <int M>
struct Lay {
  static constexpr int kABytes = kRows * 2 * M;          // [box][m][256] activations
  static constexpr int kSlotBytes = kWBytes + kSBytes + kABytes;
  static constexpr int kRingBytes = kStages * kSlotBytes;
  static constexpr int kPairOff = kRingBytes;            // per warp: [64 rows][M] pairs
  static constexpr int kPairBytes = kWarps * kRowsPerWarp * M * 8;
  static constexpr int kInOff = kPairOff + kPairBytes;   // leader: [kMaxSplit][M][kCols] sums
  static constexpr int kInBytes = kMaxSplit * M * kCols * 4;
  static constexpr int kBarOff = kInOff + kInBytes;
  static constexpr int kSmemBytes = kBarOff + kNumBars * 8 + 128;  // + alignment fix-up
  // At the end the ring is free: the cross-warp sums [kWarps][M][kCols] reuse it.
  static constexpr int kRedOff = 0;
  static_assert(kWarps * M * kCols * 4 <= kRingBytes, "reduction buffer fits the ring");
  static_assert(kSmemBytes > 116 * 1024 && kSmemBytes <= 227 * 1024,
                "one CTA per SM: more than half of the SM's shared memory");
  static_assert(kSlotBytes % 128 == 0, "slots stay 128-byte aligned");
};

// The nibble flip as a kernel parameter (a constant-bank operand of the XOR).
struct DecodeConsts {
  uint32_t flip;
};

struct ClusterParams {
  int N, K;
  int split;            // CTAs per strip = cluster size
  int units;            // units per strip (K / 512)
  int early;            // weights and scales loaded before griddepcontrol.wait
  float scalar_scale;   // per-tensor mode (no group scales)
  int out_dtype;
  int64_t ldo;
  void* out;
  OutputShard peers;    // world == 0: unsharded
  int* status;
  uint64_t* stamps;     // optional per-CTA phase times (pk_debug_phase_stamps)
};

__device__ __forceinline__ uint64_t pack2(float lo, float hi) {
  uint64_t r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(lo), "f"(hi));
  return r;
}
__device__ __forceinline__ float2 unpack2(uint64_t v) {
  float2 r;
  asm("mov.b64 {%0, %1}, %2;" : "=f"(r.x), "=f"(r.y) : "l"(v));
  return r;
}
__device__ __forceinline__ uint64_t mul2(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
__device__ __forceinline__ uint64_t fma2(uint64_t a, uint64_t b, uint64_t c) {
  uint64_t d;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
  return d;
}
__device__ __forceinline__ float exp2i(int e) {
  return __uint_as_float(static_cast<uint32_t>(e + 127) << 23);
}

// 16-bit activation at shared address `addr` as fp32.
template <typename T>
__device__ __forceinline__ float lds_act(uint32_t addr) {
  uint16_t h;
  asm volatile("ld.shared.u16 %0, [%1];" : "=h"(h) : "r"(addr));
  if constexpr (std::is_same<T, __nv_bfloat16>::value) {
    return __uint_as_float(static_cast<uint32_t>(h) << 16);
  } else {
    return __half2float(__ushort_as_half(h));
  }
}

// Eight 16-bit scales (one uint4) -> four fp32 pairs.
template <typename T>
__device__ __forceinline__ void scales8(uint4 raw, uint64_t (&s)[4]) {
  const uint32_t w[4] = {raw.x, raw.y, raw.z, raw.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    if constexpr (std::is_same<T, __nv_bfloat16>::value) {
      s[i] = pack2(__uint_as_float(w[i] << 16), __uint_as_float(w[i] & 0xFFFF0000u));
    } else {
      const __half2 h = *reinterpret_cast<const __half2*>(&w[i]);
      const float2 f = __half22float2(h);
      s[i] = pack2(f.x, f.y);
    }
  }
}

__device__ __forceinline__ void cluster_arrive_relaxed() {
  asm volatile("barrier.cluster.arrive.relaxed.aligned;" ::: "memory");
}
__device__ __forceinline__ void cluster_wait_acquire() {
  asm volatile("barrier.cluster.wait.acquire.aligned;" ::: "memory");
}
// 4 bytes into CTA `rank`'s shared memory at the same offset as `local`,
// counted as completed transaction bytes on that CTA's mbarrier at the same
// offset as `bar`.
__device__ __forceinline__ void st_async_f32(uint32_t local, uint32_t bar, uint32_t rank, float v) {
  asm volatile(
      "st.async.shared::cluster.mbarrier::complete_tx::bytes.f32 [%0], %1, [%2];" ::"r"(
          cluster_map(local, rank)),
      "f"(v), "r"(cluster_map(bar, rank))
      : "memory");
}

template <int M, typename T, bool kGrouped>
__global__ void __launch_bounds__(kThreads, 1)
    w4a16_gemv_cluster_kernel(const __grid_constant__ CUtensorMap tmW,
                              const __grid_constant__ CUtensorMap tmA,
                              const __grid_constant__ CUtensorMap tmS,
                              const __grid_constant__ ClusterParams p, const DecodeConsts dc) {
  using L = Lay<M>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 127) &
                                             ~static_cast<uintptr_t>(127));
  const uint32_t sbase = smem_u32(smem);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + L::kBarOff);  // [slot][sub-box]
  uint64_t* afull = full + kStages * kSub;                        // [slot]
  uint64_t* empty = afull + kStages;                              // [slot]
  uint64_t* pushed = empty + kStages;  // leader: the other CTAs' sums have landed

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int strip = blockIdx.x / p.split;
  const int rank = blockIdx.x % p.split;  // the CTA's rank in its cluster
  const int u0 = p.units * rank / p.split;
  const int n_units = p.units * (rank + 1) / p.split - u0;
  uint64_t t_entry = 0, t_wait = 0, t_first = 0, t_comp = 0, t_red = 0;
  const bool stamp = p.stamps != nullptr && threadIdx.x == 0;
  if (stamp) t_entry = globaltimer();

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      for (int j = 0; j < kSub; ++j) mbar_init(&full[s * kSub + j], 1);
      mbar_init(&afull[s], 1);
      mbar_init(&empty[s], kWarps);
    }
    mbar_init(pushed, 1);
    if (rank == 0 && p.split > 1)
      mbar_arrive_expect_tx(pushed, static_cast<uint32_t>((p.split - 1) * M * kCols * 4));
    fence_barrier_init();
  }
  __syncthreads();
  // Every CTA's barriers are initialised before any other CTA of the cluster
  // pushes to them: arrive now, wait before the push.
  if (p.split > 1) cluster_arrive_relaxed();
  // The next launch may start its prologue (weight prefetch) now; it waits
  // for this grid before reading activations or writing anything.
  griddep_launch_dependents();

  bool failed = false;
  uint64_t tot[M][4];
#pragma unroll
  for (int m = 0; m < M; ++m)
#pragma unroll
    for (int q = 0; q < 4; ++q) tot[m][q] = 0ull;
  if (warp == kProducerWarp) {
    if (lane == 0) {
      tma_prefetch_desc(&tmW);
      tma_prefetch_desc(&tmA);
      if constexpr (kGrouped) tma_prefetch_desc(&tmS);
      const uint32_t tx0 = kSubWBytes + (kGrouped ? kSBytes : 0);
      auto issue_w = [&](int i, int slot) {
        const int k0 = (u0 + i) * kRows;
        uint8_t* base = smem + slot * L::kSlotBytes;
        uint64_t* fb = &full[slot * kSub];
        mbar_arrive_expect_tx(&fb[0], tx0);
        tma_load_2d(base, &tmW, &fb[0], strip * kRowBytes, k0);
        if constexpr (kGrouped) tma_load_2d(base + kWBytes, &tmS, &fb[0], strip * kCols, k0 / kGroup);
        for (int j = 1; j < kSub; ++j) {
          mbar_arrive_expect_tx(&fb[j], kSubWBytes);
          tma_load_2d(base + j * kSubWBytes, &tmW, &fb[j], strip * kRowBytes, k0 + j * kSubRows);
        }
      };
      auto issue_a = [&](int i, int slot) {
        mbar_arrive_expect_tx(&afull[slot], L::kABytes);
        for (int h = 0; h < kRows / kABox; ++h)  // box h: [m][256] activations
          tma_load_2d(smem + slot * L::kSlotBytes + kWBytes + kSBytes + h * M * kABox * 2, &tmA,
                      &afull[slot], (u0 + i) * kRows + h * kABox, 0);
      };
      const int pre = n_units < kStages ? n_units : kStages;
      if (p.early) {
        for (int i = 0; i < pre; ++i) issue_w(i, i);
      }
      // the rest of the CTA's weights (all of them without staging) into L2,
      // and the activations of the first units: L2 is coherent, so a line the
      // previous kernel is still writing cannot come back stale
      for (int i = p.early ? pre : 0; i < n_units && i < pre + 4 * kStages; ++i) {
        const int k0 = (u0 + i) * kRows;
        for (int j = 0; j < kSub; ++j) tma_prefetch_l2_2d(&tmW, strip * kRowBytes, k0 + j * kSubRows);
        if constexpr (kGrouped) tma_prefetch_l2_2d(&tmS, strip * kCols, k0 / kGroup);
      }
      for (int i = 0; i < pre; ++i)
        for (int h = 0; h < kRows / kABox; ++h)
          tma_prefetch_l2_2d(&tmA, (u0 + i) * kRows + h * kABox, 0);
      griddep_wait();
      if (!p.early) {
        for (int i = 0; i < pre; ++i) issue_w(i, i);
      }
      for (int i = 0; i < pre; ++i) issue_a(i, i);
      int issued = pre;
      bool ok = true;
      for (int i = pre, slot = pre % kStages, round = pre / kStages; i < n_units; ++i) {
        if (!mbar_wait(&empty[slot], (round - 1) & 1, p.status, kSiteGemvProducer)) {
          ok = false;
          break;
        }
        issue_w(i, slot);
        issue_a(i, slot);
        issued = i + 1;
        if (++slot == kStages) slot = 0, ++round;
      }
      if (!ok) {
        // let copies already issued land before the CTA's shared memory is released
        const int first = issued > kStages ? issued - kStages : 0;
        for (int i = first; i < issued; ++i) {
          for (int j = 0; j < kSub; ++j)
            mbar_wait(&full[(i % kStages) * kSub + j], (i / kStages) & 1, nullptr, 0);
          mbar_wait(&afull[i % kStages], (i / kStages) & 1, nullptr, 0);
        }
      }
    }
    __syncwarp();
  } else {
    // ---------------- dequant / FMA warps ----------------
    griddep_wait();
    if (stamp) t_wait = globaltimer();
    // -8 * 16^p * 2^-149 for the column pairs' positions (0,1), (2,3), (4,5)
    const uint64_t off01 = pack2(__uint_as_float(0x80000008u), __uint_as_float(0x80000080u));
    const uint64_t off23 = pack2(__uint_as_float(0x80000800u), __uint_as_float(0x80008000u));
    const uint64_t off45 = pack2(__uint_as_float(0x80080000u), __uint_as_float(0x80800000u));
    const uint32_t pairs = sbase + L::kPairOff + warp * kRowsPerWarp * M * 8;
    constexpr int kWarpsPerSub = kSubRows / kRowsPerWarp;  // 2
    for (int i = 0, slot = 0, round = 0; i < n_units; ++i) {
      const uint32_t base = sbase + slot * L::kSlotBytes;
      if (!failed && !mbar_wait_sleep(&afull[slot], round & 1, p.status, kSiteGemvConsumer))
        failed = true;
      // Activations ([box of 256 rows][m][256] in the slot): lane l scales rows
      // 64w + l and 64w + 32 + l of every output row m; S_m = clamp(248 -
      // e_max, 30, 127) from the largest exponent among the warp's 64 rows.
      // A lane walks the rows of one parity (lane / 16): the sum of the scaled
      // activations of that parity removes its +8 offsets. Rows 64w + l and
      // 64w + 32 + l have the parity of l, so sum over lanes of equal l % 2.
      uint64_t asum[M], pw01[M], pw23[M], pw45[M];
      {
        const int r0 = warp * kRowsPerWarp;  // the warp's 64 rows lie in one box
        const uint32_t abase =
            base + kWBytes + kSBytes + (r0 / kABox) * M * kABox * 2 + (r0 % kABox) * 2;
#pragma unroll
        for (int m = 0; m < M; ++m) {
          const float av0 = lds_act<T>(abase + (m * kABox + lane) * 2);
          const float av1 = lds_act<T>(abase + (m * kABox + 32 + lane) * 2);
          uint32_t emax = (__float_as_uint(av0) >> 23) & 0xFFu;
          const uint32_t e1 = (__float_as_uint(av1) >> 23) & 0xFFu;
          emax = __reduce_max_sync(0xffffffffu, emax > e1 ? emax : e1);
          int S = 248 - static_cast<int>(emax);
          S = S < 30 ? 30 : (S > 127 ? 127 : S);
          const float as0 = av0 * exp2i(S), as1 = av1 * exp2i(S);
          sts_u64(pairs + (lane * M + m) * 8, pack2(as0, as0));
          sts_u64(pairs + ((32 + lane) * M + m) * 8, pack2(as1, as1));
          float t = as0 + as1;
#pragma unroll
          for (int o = 16; o > 1; o >>= 1) t += __shfl_xor_sync(0xffffffffu, t, o);
          t = __shfl_sync(0xffffffffu, t, lane >> 4);
          asum[m] = pack2(t, t);
          // 2^(149 - S - 4p) for the pairs' positions (0,1), (2,3) and (4,5)
          pw01[m] = pack2(exp2i(149 - S), exp2i(145 - S));
          pw23[m] = pack2(exp2i(141 - S), exp2i(137 - S));
          pw45[m] = pack2(exp2i(133 - S), exp2i(129 - S));
        }
      }
      // sub-box 0 carries the unit's scales; the warp's rows are in sub-box w/2
      if (!failed && !mbar_wait_sleep(&full[slot * kSub], round & 1, p.status, kSiteGemvConsumer))
        failed = true;
      if (warp >= kWarpsPerSub && !failed &&
          !mbar_wait_sleep(&full[slot * kSub + warp / kWarpsPerSub], round & 1, p.status,
                           kSiteGemvConsumer))
        failed = true;
      if (stamp && i == 0) t_first = globaltimer();
      uint64_t sc[4];
      if constexpr (kGrouped) {
        const int srow = (warp * kRowsPerWarp) / kGroup;
        scales8<T>(lds_v4(base + kWBytes + srow * kCols * 2 + (lane & 15) * 16), sc);
      } else {
#pragma unroll
        for (int q = 0; q < 4; ++q) sc[q] = pack2(p.scalar_scale, p.scalar_scale);
      }
      __syncwarp();

      // lane l: word l % 16 (columns 8(l%16) .. +8) of rows 64w + 2i + l / 16
      uint64_t acc[M][4];
#pragma unroll
      for (int m = 0; m < M; ++m)
#pragma unroll
        for (int q = 0; q < 4; ++q) acc[m][q] = 0ull;
      const uint32_t wrow =
          base + (warp * kRowsPerWarp + (lane >> 4)) * kRowBytes + (lane & 15) * 4;
      const uint32_t prow = pairs + (lane >> 4) * M * 8;
      constexpr int kBatch = M == 1 ? 8 : 4;  // rows in flight per lane
#pragma unroll
      for (int b = 0; b < kRowsPerWarp / 2 / kBatch; ++b) {
        uint32_t wv[kBatch];
        uint64_t a2[kBatch][M];
#pragma unroll
        for (int r = 0; r < kBatch; ++r) wv[r] = lds_u32(wrow + (b * kBatch + r) * 2 * kRowBytes);
#pragma unroll
        for (int r = 0; r < kBatch; ++r)
#pragma unroll
          for (int m = 0; m < M; ++m) a2[r][m] = lds_u64(prow + ((b * kBatch + r) * 2 * M + m) * 8);
#pragma unroll
        for (int r = 0; r < kBatch; ++r) {
          const uint32_t w = wv[r] ^ dc.flip;  // every nibble q -> q + 8
          const uint32_t hi = w >> 8;          // nibbles 6, 7 at positions 4, 5
          uint64_t d[4];
          d[0] = pack2(__uint_as_float(w & 0xFu), __uint_as_float(w & 0xF0u));
          d[1] = pack2(__uint_as_float(w & 0xF00u), __uint_as_float(w & 0xF000u));
          d[2] = pack2(__uint_as_float(w & 0xF0000u), __uint_as_float(w & 0xF00000u));
          d[3] = pack2(__uint_as_float(hi & 0xF0000u), __uint_as_float(hi & 0xF00000u));
#pragma unroll
          for (int m = 0; m < M; ++m)
#pragma unroll
            for (int q = 0; q < 4; ++q) acc[m][q] = fma2(d[q], a2[r][m], acc[m][q]);
        }
      }
      // fold the unit: remove the +8 offset, undo 2^S * 16^p, apply the scale
#pragma unroll
      for (int m = 0; m < M; ++m)
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const uint64_t off = q == 0 ? off01 : (q == 1 ? off23 : off45);
          const uint64_t pw = q == 0 ? pw01[m] : (q == 1 ? pw23[m] : pw45[m]);
          const uint64_t c = fma2(off, asum[m], acc[m][q]);
          tot[m][q] = fma2(mul2(c, pw), sc[q], tot[m][q]);
        }
      __syncwarp();  // every lane is done with the slot and the pairs
      if (lane == 0) mbar_arrive(&empty[slot]);
      if (++slot == kStages) slot = 0, ++round;
    }
  }
  if (stamp) t_comp = globaltimer();

  // ---------------- reduction: warps, then the cluster ----------------
  failed = __syncthreads_or(failed) != 0;  // every warp is done with the ring
  if (warp < kWarps) {
    // lanes l and l + 16 hold the two row parities of the same columns
#pragma unroll
    for (int m = 0; m < M; ++m) {
      float2 v[4];
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        v[q] = unpack2(tot[m][q]);
        v[q].x += __shfl_xor_sync(0xffffffffu, v[q].x, 16);
        v[q].y += __shfl_xor_sync(0xffffffffu, v[q].y, 16);
      }
      if (lane < 16) {
        const uint32_t dst = sbase + L::kRedOff + ((warp * M + m) * kCols + lane * 8) * 4;
        sts_v4f(dst, v[0].x, v[0].y, v[1].x, v[1].y);
        sts_v4f(dst + 16, v[2].x, v[2].y, v[3].x, v[3].y);
      }
    }
  }
  __syncthreads();
  // thread t < 128 owns column t of the strip, for every output row m
  float colsum[M];
#pragma unroll
  for (int m = 0; m < M; ++m) {
    colsum[m] = 0.0f;
    if (threadIdx.x < kCols) {
#pragma unroll
      for (int w = 0; w < kWarps; ++w)
        colsum[m] += lds_f32(sbase + L::kRedOff + ((w * M + m) * kCols + threadIdx.x) * 4);
    }
  }
  if (p.split > 1) cluster_wait_acquire();  // the leader's barrier is initialised
  bool stored = false;
  const uint32_t in_base = sbase + L::kInOff;  // [rank][m][kCols]
  if (rank != 0) {
    // push this CTA's column sums into slot `rank` of the leader's buffer
    if (threadIdx.x < kCols) {
#pragma unroll
      for (int m = 0; m < M; ++m)
        st_async_f32(in_base + ((rank * M + m) * kCols + threadIdx.x) * 4, smem_u32(pushed), 0u,
                     colsum[m]);
    }
  } else {
    if (p.split > 1 &&
        !mbar_wait(pushed, 0, p.status, kSiteGemvConsumer))  // the others' sums have landed
      failed = true;
    failed = __syncthreads_or(failed) != 0;
    if (!failed && threadIdx.x < kCols) {
#pragma unroll
      for (int m = 0; m < M; ++m) {
        float v = colsum[m];  // in CTA order: rank 0 first, then ranks 1 .. split-1
        for (int j = 1; j < p.split; ++j)
          v += lds_f32(in_base + ((j * M + m) * kCols + threadIdx.x) * 4);
        emit_out(p.out, p.peers, p.out_dtype,
                 m * p.ldo + static_cast<int64_t>(strip) * kCols + threadIdx.x, v);
      }
      stored = true;
    }
  }
  if (stamp) {
    t_red = globaltimer();
    uint32_t smid;
    asm volatile("mov.u32 %0, %%smid;" : "=r"(smid));
    uint64_t* st = p.stamps + static_cast<int64_t>(blockIdx.x) * 8;
    st[0] = t_entry;
    st[1] = t_wait;
    st[2] = t_first;
    st[3] = t_comp;
    st[4] = t_red;
    st[5] = smid;
    st[6] = static_cast<uint64_t>(n_units);
    st[7] = t_red;  // overwritten with the exchange's end below
  }
  // only the leaders stored: one fence and one arrival per cluster
  if (p.peers.world > 1 && rank == 0)
    peer_exchange_finish(p.peers, stored, p.status, kSiteGemvPeers, gridDim.x / p.split);
  if (stamp) p.stamps[static_cast<int64_t>(blockIdx.x) * 8 + 7] = globaltimer();
}

CUtensorMapDataType tmap_type16(int dt) {
  return dt == PK_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
}

// Whether clusters of `split` CTAs of this kernel can be resident (per
// device and split; 0 unknown, 1 yes, 2 no).
template <typename Kern>
bool cluster_fits(Kern kernel, int split, int smem_bytes, int m) {
  static int cache[64][kMaxM + 1][kMaxSplit + 1] = {};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return false;
  int& c = cache[dev][m][split];
  if (c == 0) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(split, 1, 1);
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = smem_bytes;
    cudaLaunchAttribute attr;
    attr.id = cudaLaunchAttributeClusterDimension;
    attr.val.clusterDim.x = split;
    attr.val.clusterDim.y = 1;
    attr.val.clusterDim.z = 1;
    cfg.attrs = &attr;
    cfg.numAttrs = 1;
    int clusters = 0;
    c = (cudaOccupancyMaxActiveClusters(&clusters, kernel, &cfg) == cudaSuccess && clusters > 0)
            ? 1
            : 2;
    cudaGetLastError();
  }
  return c == 1;
}

int g_weight_staging = 0;        // pk_set_weight_staging
uint64_t* g_phase_stamps = nullptr;  // pk_debug_phase_stamps
size_t g_phase_stamp_bytes = 0;

}  // namespace

void set_weight_staging(int mode) { g_weight_staging = mode != 0 ? 1 : 0; }
int weight_staging() { return g_weight_staging; }
void set_phase_stamps(void* buf, size_t bytes) {
  g_phase_stamps = static_cast<uint64_t*>(buf);
  g_phase_stamp_bytes = buf != nullptr ? bytes : 0;
}
uint64_t* phase_stamps(size_t grid) {
  // two halves of the buffer, alternating launch by launch
  if (g_phase_stamps == nullptr || g_phase_stamp_bytes < grid * 128) return nullptr;
  static int calls = 0;
  return g_phase_stamps + (calls++ & 1) * (g_phase_stamp_bytes / 16);
}

// CTAs per strip: as many as keep strips * split within one CTA per SM, at
// most 4 (clusters of 4 at one CTA per SM: 33 fit a B200 at once, clusters of
// 8 only 15, which left a sixteenth cluster waiting for a second wave) and at
// most one per 512-row unit.
int gemv_cluster_split(int64_t N, int64_t K) {
  const int64_t strips = N / kCols;
  if (strips <= 0) return 0;
  int64_t split = num_sms() / strips;
  if (split > kMaxSplit) split = kMaxSplit;
  if (split > K / kRows) split = K / kRows;
  return static_cast<int>(split);
}

bool gemv_cluster_supported(int64_t M, int64_t N, int64_t K, int group, const void* scales,
                            int64_t lda, const void* a, const void* wp) {
  if (M < 1 || M > kMaxM) return false;
  if (N % kCols != 0 || K % kRows != 0 || N <= 0 || K <= 0) return false;
  if (N > (1ll << 30) || K > (1ll << 30)) return false;
  if (gemv_cluster_split(N, K) < 1) return false;
  if (lda % 8 != 0 || (reinterpret_cast<uintptr_t>(a) & 15) != 0) return false;
  if ((reinterpret_cast<uintptr_t>(wp) & 15) != 0) return false;
  if (scales != nullptr && (group != kGroup || (reinterpret_cast<uintptr_t>(scales) & 15) != 0))
    return false;
  return true;
}

// The cluster form for small layers: its grid keeps at least 3/4 of the SMs
// busy with at least two CTAs per strip, and each CTA has at most 4 units
// (the ring holds them all). Longer K ranges stream better through the
// stream-K GEMV's two CTAs per SM (Llama-70B down_proj: 35 vs 59 us).
bool gemv_cluster_preferred(int64_t M, int64_t N, int64_t K) {
  if (M < 1 || M > kMaxM || N % kCols != 0 || K % kRows != 0) return false;
  const int split = gemv_cluster_split(N, K);
  if (split < 2 || (N / kCols) * split * 4 < 3ll * num_sms()) return false;
  return (K / kRows + split - 1) / split <= kStages;
}

cudaError_t launch_w4a16_gemv_cluster(const DecodeArgs& a, cudaStream_t s, const char** why,
                                      const OutputShard* shard) {
  CUtensorMap tmW, tmA, tmS;
  const CUtensorMapDataType dt = tmap_type16(a.a_dtype);
  if (!encode_tmap_2d(&tmW, CU_TENSOR_MAP_DATA_TYPE_UINT8, a.wp, a.N / 2, a.K, a.N / 2, kRowBytes,
                      kSubRows, CU_TENSOR_MAP_SWIZZLE_NONE, why))
    return cudaErrorInvalidValue;
  if (!encode_tmap_2d(&tmA, dt, a.a, a.K, a.M, a.lda * 2, kABox, static_cast<uint32_t>(a.M),
                      CU_TENSOR_MAP_SWIZZLE_NONE, why))
    return cudaErrorInvalidValue;
  const bool grouped = a.scales != nullptr;
  if (grouped) {
    if (!encode_tmap_2d(&tmS, dt, a.scales, a.N, a.K / kGroup, a.N * 2, kCols, kRows / kGroup,
                        CU_TENSOR_MAP_SWIZZLE_NONE, why))
      return cudaErrorInvalidValue;
  } else {
    std::memcpy(&tmS, &tmW, sizeof(tmS));  // unused
  }
  ClusterParams p{};
  p.N = static_cast<int>(a.N);
  p.K = static_cast<int>(a.K);
  p.split = gemv_cluster_split(a.N, a.K);
  p.units = static_cast<int>(a.K / kRows);
  p.early = g_weight_staging;
  p.scalar_scale = grouped ? 1.0f : a.scalar_scale;
  p.out_dtype = a.out_dtype;
  p.ldo = a.ldo;
  p.out = a.out;
  p.status = a.status;
  const int64_t grid = (a.N / kCols) * p.split;
  p.stamps = phase_stamps(static_cast<size_t>(grid));
  if (shard != nullptr) {
    if (shard->world < 1 || shard->world > kMaxPeers || shard->done == nullptr) {
      *why = "sharded GEMV: 1 <= world <= 8 and a workspace are required";
      return cudaErrorInvalidValue;
    }
    p.peers = *shard;
  }
  const DecodeConsts dc{0x88888888u};

  auto launch = [&](auto kernel, int smem_bytes) -> cudaError_t {
    cudaError_t e = set_max_smem(reinterpret_cast<const void*>(kernel), smem_bytes);
    if (e != cudaSuccess) return e;
    if (p.split > 1 && !cluster_fits(kernel, p.split, smem_bytes, static_cast<int>(a.M))) {
      *why = "clusters of the GEMV's split cannot be resident";
      return cudaErrorInvalidValue;
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(static_cast<unsigned>(grid), 1, 1);
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = smem_bytes;
    cfg.stream = s;
    cudaLaunchAttribute attrs[3];
    attrs[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attrs[0].val.programmaticStreamSerializationAllowed = 1;
    attrs[1].id = cudaLaunchAttributeClusterDimension;
    attrs[1].val.clusterDim.x = static_cast<unsigned>(p.split);
    attrs[1].val.clusterDim.y = 1;
    attrs[1].val.clusterDim.z = 1;
    attrs[2].id = cudaLaunchAttributeClusterSchedulingPolicyPreference;
    attrs[2].val.clusterSchedulingPolicyPreference = cudaClusterSchedulingPolicySpread;
    cfg.attrs = attrs;
    cfg.numAttrs = 3;
    return cudaLaunchKernelEx(&cfg, kernel, tmW, tmA, tmS, p, dc);
  };
  auto by_m = [&](auto mtag) -> cudaError_t {
    constexpr int kM = decltype(mtag)::value;
    constexpr int kBytes = Lay<kM>::kSmemBytes;
    if (a.a_dtype == PK_BF16)
      return grouped ? launch(w4a16_gemv_cluster_kernel<kM, __nv_bfloat16, true>, kBytes)
                     : launch(w4a16_gemv_cluster_kernel<kM, __nv_bfloat16, false>, kBytes);
    return grouped ? launch(w4a16_gemv_cluster_kernel<kM, __half, true>, kBytes)
                   : launch(w4a16_gemv_cluster_kernel<kM, __half, false>, kBytes);
  };
  switch (a.M) {
    case 1: return by_m(std::integral_constant<int, 1>{});
    case 2: return by_m(std::integral_constant<int, 2>{});
    default: return by_m(std::integral_constant<int, 3>{});
  }
}

}  // namespace pk
