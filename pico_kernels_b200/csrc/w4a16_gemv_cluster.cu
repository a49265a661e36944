// W4A16 decode GEMM (M = 1..8) for layers that fit one wave of the SMs: the
// nibbles are decoded in registers into exact fp16 operands of mma.sync
// tiles, and the K split is reduced inside thread-block clusters.
//
// out[M, N] = A[M, K] @ (q[K, N] * s[K/128, N])  -- gemm_int4.int4_gemm
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
//    [U*r/split, U*(r+1)/split) of 512 rows (U = K/512), at most 4 (the
//    ring holds them all). strips * split <= the SM count, so the grid is one
//    wave of one CTA per SM.
//  * Footprint. More than 116 KB of shared memory, so that no SM holds two
//    CTAs of one grid: with room for two, CTAs started early by programmatic
//    dependent launch were packed two to an SM on ~12 SMs, whose doubled
//    work then set every launch's critical path. Clusters of 4: at one CTA
//    per SM a B200 holds 33 of them at once but only 15 clusters of 8.
//  * Loads. Warp 8 (one thread) is the TMA producer: per unit four 128-row
//    weight boxes (64-byte swizzled; each with its own mbarrier, so a warp
//    starts when the box holding its rows lands) and the unit's four group-
//    scale rows. Before griddepcontrol.wait it prefetches the CTA's weights
//    into L2 (a hint that cannot return stale data); with weight staging on
//    (pk_set_weight_staging) it loads them into shared memory there instead.
//    The activations, which the previous kernel may have written, are read
//    by the mma warps themselves after the wait (L2-coherent loads), so the
//    wait-to-first-use chain is one load round trip.
//  * Activations -> B fragments. Each warp converts its rows of every unit
//    into fp16 mma B fragments once (bf16 rows scaled by 2^S_m per output row
//    m, so the largest is in [2^14, 2^15): exact; fp16 rows as they are).
//  * Weights -> A fragments. The tiles are swap-AB: the mma's M dimension is
//    16 output columns, N the (up to 8) output rows, K 16 weight rows. A lane
//    loads 8 bytes (16 columns) of 4 rows per k-step; one PRMT puts byte b of
//    two rows into the two fp16 halves of a word, and one mask-and-flip LOP3
//    leaves (q + 8) * 2^-24 (low nibble) or (q + 8) * 16 * 2^-24 (high nibble)
//    in each half: exact subnormal fp16 values. So every product in the fp32
//    accumulator is exact: 2 PRMT + 4 LOP3 + 1 mma per 8 weights and lane.
//    The +8 offsets enter each unit's tiles as their starting value: one mma
//    of the constant -8 * 2^-24 (or -128 * 2^-24) with the activations.
//  * Fold. Per unit the tiles' sums take the fp32 group scales; at the end
//    2^24 (2^20 for high nibbles) and 2^-S_m are undone exactly.
//  * Reduction. The 8 warps' sums meet in shared memory; each other CTA of
//    the cluster then pushes its sums into the leader's (rank 0) shared
//    memory with st.async, which completes bytes on the leader's mbarrier,
//    and exits; the leader waits for them (bounded), sums the strip's columns
//    in CTA order and stores them: deterministic, no global workspace, no
//    atomics, and only one CTA per cluster waits or stores (in the sharded
//    exchange, one system-scope fence per cluster).
//  * Placement. The launch also asks for the spread cluster scheduling
//    policy; on its own that did not keep two CTAs off one SM (the shared-
//    memory footprint does).
//
// mma.sync rather than tcgen05: the operands are produced in registers and
// consumed there; the decode (6 ALU instructions per 8 weights) sets the
// pace, and the legacy tensor path's rate (measured ~2.3 SM cycles per
// m16n8k16) keeps up with it. A tcgen05 tile would take its A operand from
// shared or tensor memory, a store and a barrier per tile more.
#include "pk_common.cuh"

#include <cstring>
#include <mutex>
#include <type_traits>

#include "pk_internal.h"
#include "w4a16_mma.cuh"

namespace pk {
namespace {

using namespace w4mma;  // units of 512 rows x 128 columns, 8 mma warps, tile decode

constexpr int kProducerWarp = kWarps;
constexpr int kThreads = (kWarps + 1) * 32;
constexpr int kMmaThreads = kWarps * 32;
constexpr int kGroup = 128;
constexpr int kMaxSplit = 4;
constexpr int kStages = 4;                              // units per CTA, all resident
constexpr int kSBytes = (kRows / kGroup) * kCols * 2;   // 1024: four 16-bit scale rows
constexpr int kNumBars = kStages * kSub + 1;            // full[slot][sub-box]; pushed

// Shared-memory layout for M output rows. The ring's weight boxes are
// 64-byte swizzled, so slots are 1024-byte aligned (the pattern's period).
template <int M>
struct Lay {
  static constexpr int kSlotBytes = (kWBytes + kSBytes + 1023) / 1024 * 1024;
  static constexpr int kRingBytes = kStages * kSlotBytes;
  // B fragments per warp: [unit][k-step] blocks (blk_words<M>() words)
  static constexpr int kBlkWords = blk_words<M>();
  static constexpr int kFragOff = kRingBytes;
  static constexpr int kFragWarpBytes = kStages * kKSteps * kBlkWords * 4;
  static constexpr int kFragBytes = kWarps * kFragWarpBytes;
  static constexpr int kInOff = kFragOff + kFragBytes;   // leader: [kMaxSplit][M][kCols] sums
  static constexpr int kInBytes = kMaxSplit * M * kCols * 4;
  static constexpr int kBarOff = kInOff + kInBytes;
  static constexpr int kSmemBytes = kBarOff + kNumBars * 8 + 1024;  // + alignment fix-up
  // At the end the ring is free: the cross-warp sums [kWarps][M][kCols] reuse it.
  static constexpr int kRedOff = 0;
  static_assert(kWarps * M * kCols * 4 <= kRingBytes, "reduction buffer fits the ring");
  static_assert(kSmemBytes > 116 * 1024 && kSmemBytes <= 227 * 1024,
                "one CTA per SM: more than half of the SM's shared memory");
  static_assert(kBlkWords % 32 == 8 || kBlkWords % 32 == 24, "k-step blocks on distinct banks");
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
  const uint16_t* a;    // [M][lda] activations
  int64_t lda;
  OutputShard peers;    // world == 0: unsharded
  int* status;
  uint64_t* stamps;     // optional per-CTA phase times (pk_debug_phase_stamps)
};

// A global load cached in L2 only: after griddepcontrol.wait it sees the
// previous kernel's writes, and no L1 line of this SM can be stale.
__device__ __forceinline__ uint32_t ldg_cg_u32(const void* p) {
  uint32_t v;
  asm volatile("ld.global.cg.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
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
                              const __grid_constant__ CUtensorMap tmS,
                              const __grid_constant__ ClusterParams p, const Consts dc) {
  using L = Lay<M>;
  constexpr bool kBf16 = std::is_same<T, __nv_bfloat16>::value;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  const uint32_t sbase = smem_u32(smem);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + L::kBarOff);  // [unit][sub-box]
  uint64_t* pushed = full + kStages * kSub;  // leader: the other CTAs' sums have landed

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int strip = blockIdx.x / p.split;
  const int rank = blockIdx.x % p.split;  // the CTA's rank in its cluster
  const int u0 = p.units * rank / p.split;
  const int n_units = p.units * (rank + 1) / p.split - u0;  // <= kStages (host-checked)
  uint64_t t_entry = 0, t_wait = 0, t_first = 0, t_comp = 0, t_red = 0;
  const bool stamp = p.stamps != nullptr && threadIdx.x == 0;
  if (stamp) t_entry = globaltimer();

  if (threadIdx.x == 0) {
    for (int j = 0; j < kStages * kSub; ++j) mbar_init(&full[j], 1);
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
  float tot[8][4];  // tile j: columns 16g + 2j ([0], [1]) and + 1 ([2], [3]); rows 2t, 2t + 1
#pragma unroll
  for (int j = 0; j < 8; ++j)
#pragma unroll
    for (int e = 0; e < 4; ++e) tot[j][e] = 0.0f;
  float pw0 = 1.0f, pw1 = 1.0f;  // 2^-S of the lane's tokens 2t, 2t + 1
  if (warp == kProducerWarp) {
    if (lane == 0) {
      tma_prefetch_desc(&tmW);
      if constexpr (kGrouped) tma_prefetch_desc(&tmS);
      auto issue_w = [&](int i) {
        const int k0 = (u0 + i) * kRows;
        uint8_t* base = smem + i * L::kSlotBytes;
        uint64_t* fb = &full[i * kSub];
        mbar_arrive_expect_tx(&fb[0], kSubWBytes + (kGrouped ? kSBytes : 0));
        tma_load_2d(base, &tmW, &fb[0], strip * kRowBytes, k0);
        if constexpr (kGrouped) tma_load_2d(base + kWBytes, &tmS, &fb[0], strip * kCols, k0 / kGroup);
        for (int j = 1; j < kSub; ++j) {
          mbar_arrive_expect_tx(&fb[j], kSubWBytes);
          tma_load_2d(base + j * kSubWBytes, &tmW, &fb[j], strip * kRowBytes, k0 + j * kSubRows);
        }
      };
      if (p.early) {
        for (int i = 0; i < n_units; ++i) issue_w(i);
      } else {
        // into L2 while the previous kernel runs: L2 is coherent, so a line
        // that kernel is still writing cannot come back stale
        for (int i = 0; i < n_units; ++i) {
          const int k0 = (u0 + i) * kRows;
          for (int j = 0; j < kSub; ++j)
            tma_prefetch_l2_2d(&tmW, strip * kRowBytes, k0 + j * kSubRows);
          if constexpr (kGrouped) tma_prefetch_l2_2d(&tmS, strip * kCols, k0 / kGroup);
        }
      }
      griddep_wait();
      if (!p.early) {
        for (int i = 0; i < n_units; ++i) issue_w(i);
      }
    }
    __syncwarp();
  } else {
    // ---------------- mma warps ----------------
    griddep_wait();
    if (stamp) t_wait = globaltimer();
    const LaneMap lm = lane_map(lane);
    const uint32_t frag = sbase + L::kFragOff + warp * L::kFragWarpBytes;
    constexpr uint32_t kUnitFragBytes = kKSteps * L::kBlkWords * 4;
    // Activations of every unit -> fp16 B fragments, with one scale 2^S_m per
    // output row over the warp's rows of all its units (bf16; fp16 as is).
    {
      const int rho = warp * kRowsPerWarp + 2 * lane;
      const uint8_t* a_lane = reinterpret_cast<const uint8_t*>(p.a) +
                              (static_cast<int64_t>(u0) * kRows + rho) * 2;
      uint32_t raw[M][kStages];
#pragma unroll
      for (int m = 0; m < M; ++m)
#pragma unroll
        for (int i = 0; i < kStages; ++i)
          raw[m][i] = i < n_units ? ldg_cg_u32(a_lane + (m * p.lda + i * kRows) * 2) : 0u;
#pragma unroll
      for (int m = 0; m < M; ++m) {
        int S = 0;
        if constexpr (kBf16) {
          uint32_t emax = 0;
#pragma unroll
          for (int i = 0; i < kStages; ++i) emax = max(emax, bf16x2_emax(raw[m][i]));
          S = scale_exp(__reduce_max_sync(0xffffffffu, emax));
        }
        if (m == 2 * lm.t) pw0 = exp2i(-S);
        if (m == 2 * lm.t + 1) pw1 = exp2i(-S);
        const float sc = exp2i(S);
#pragma unroll
        for (int i = 0; i < kStages; ++i)
          if (i < n_units)
            sts_u32(frag + i * kUnitFragBytes + bfrag_store_off<M>(lane, m),
                    to_f16x2<T>(raw[m][i], sc));
      }
    }
    __syncwarp();
    const uint32_t bfrag = frag + ((lm.g < M ? lm.g : M - 1) * 4 + lm.t) * 8;
    for (int i = 0; i < n_units; ++i) {
      const uint32_t base = sbase + i * L::kSlotBytes;
      // sub-box 0 carries the unit's scales; the warp's rows are in sub-box w/2
      if (!failed && !mbar_wait_sleep(&full[i * kSub], 0, p.status, kSiteGemvConsumer))
        failed = true;
      if (warp >= 2 && !failed &&
          !mbar_wait_sleep(&full[i * kSub + warp / 2], 0, p.status, kSiteGemvConsumer))
        failed = true;
      if (stamp && i == 0) t_first = globaltimer();
      unit<M, T, kGrouped, false>(
          lm, base + warp * kRowsPerWarp * kRowBytes, bfrag + i * kUnitFragBytes,
          base + kWBytes + ((warp * kRowsPerWarp) / kGroup) * kCols * 2 + lm.g * 32,
          p.scalar_scale, 1.0f, 1.0f, dc, tot);
    }
  }
  if (stamp) t_comp = globaltimer();

  // ---------------- reduction: warps, then the cluster ----------------
  failed = __syncthreads_or(failed) != 0;  // every warp is done with the ring
  constexpr int kOut = M * kCols;          // sums per CTA: [m][column]
  if (warp < kWarps)
    store_sums<M>(sbase + L::kRedOff + warp * kOut * 4, lane_map(lane), tot, pw0, pw1);
  __syncthreads();
  // thread x < 256 owns sums x, x + 256, ... of the CTA's [m][column]
  constexpr int kPer = (kOut + kMmaThreads - 1) / kMmaThreads;
  float colsum[kPer];
#pragma unroll
  for (int k = 0; k < kPer; ++k) {
    const int o = threadIdx.x + k * kMmaThreads;
    colsum[k] = 0.0f;
    if (threadIdx.x < kMmaThreads && o < kOut) {
#pragma unroll
      for (int w = 0; w < kWarps; ++w) colsum[k] += lds_f32(sbase + L::kRedOff + (w * kOut + o) * 4);
    }
  }
  if (p.split > 1) cluster_wait_acquire();  // the leader's barrier is initialised
  bool stored = false;
  const uint32_t in_base = sbase + L::kInOff;  // [rank][m][column]
  if (rank != 0) {
    // push this CTA's sums into slot `rank` of the leader's buffer
#pragma unroll
    for (int k = 0; k < kPer; ++k) {
      const int o = threadIdx.x + k * kMmaThreads;
      if (threadIdx.x < kMmaThreads && o < kOut)
        st_async_f32(in_base + (rank * kOut + o) * 4, smem_u32(pushed), 0u, colsum[k]);
    }
  } else {
    if (p.split > 1 &&
        !mbar_wait(pushed, 0, p.status, kSiteGemvConsumer))  // the others' sums have landed
      failed = true;
    failed = __syncthreads_or(failed) != 0;
    if (!failed) {
#pragma unroll
      for (int k = 0; k < kPer; ++k) {
        const int o = threadIdx.x + k * kMmaThreads;
        if (threadIdx.x < kMmaThreads && o < kOut) {
          float v = colsum[k];  // in CTA order: rank 0 first, then ranks 1 .. split-1
          for (int j = 1; j < p.split; ++j) v += lds_f32(in_base + (j * kOut + o) * 4);
          emit_out(p.out, p.peers, p.out_dtype,
                   (o / kCols) * p.ldo + static_cast<int64_t>(strip) * kCols + o % kCols, v);
          stored = true;
        }
      }
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
// device, row count and split; 0 unknown, 1 yes, 2 no).
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
  const int split = gemv_cluster_split(N, K);
  if (split < 1 || (K / kRows + split - 1) / split > kStages) return false;  // all units resident
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
  if (!gemv_cluster_supported(a.M, a.N, a.K, a.group, a.scales, a.lda, a.a, a.wp)) {
    *why = "cluster GEMV: unsupported shape or alignment";
    return cudaErrorInvalidValue;
  }
  CUtensorMap tmW, tmS;
  const CUtensorMapDataType dt = tmap_type16(a.a_dtype);
  if (!encode_tmap_2d(&tmW, CU_TENSOR_MAP_DATA_TYPE_UINT8, a.wp, a.N / 2, a.K, a.N / 2, kRowBytes,
                      kSubRows, CU_TENSOR_MAP_SWIZZLE_64B, why))
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
  p.a = static_cast<const uint16_t*>(a.a);
  p.lda = a.lda;
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
  const Consts dc = consts();

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
    return cudaLaunchKernelEx(&cfg, kernel, tmW, tmS, p, dc);
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
    case 3: return by_m(std::integral_constant<int, 3>{});
    case 4: return by_m(std::integral_constant<int, 4>{});
    case 5: return by_m(std::integral_constant<int, 5>{});
    case 6: return by_m(std::integral_constant<int, 6>{});
    case 7: return by_m(std::integral_constant<int, 7>{});
    default: return by_m(std::integral_constant<int, 8>{});
  }
}

}  // namespace pk
