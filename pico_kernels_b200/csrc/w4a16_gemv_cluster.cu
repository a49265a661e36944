// W4A16 decode GEMV (M = 1) for layers that fit one wave of the SMs, on the
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
//  * Partition. The columns are cut into strips of 256 (128 packed bytes per
//    row); each strip's K rows are split over `split` CTAs, which form one
//    thread-block cluster (split <= 8). CTA r of a strip owns units
//    [U*r/split, U*(r+1)/split) of 256 rows (U = K/256). strips * split <=
//    the SM count, so each CTA owns one SM and never waits for a second wave.
//  * Footprint. ~104 KB of shared memory and 288 threads, so that the next
//    launch's CTA (started early by programmatic dependent launch) fits on
//    the same SM and issues its weight traffic while this one computes.
//  * Loads. Warp 8 (one thread) is the TMA producer of a 3-slot ring: per
//    unit four 64-row weight boxes (each with its own mbarrier, so a warp
//    starts when the box holding its rows lands), the unit's two group-scale
//    rows, and, on a separate barrier, the unit's 256 activations. Before
//    griddepcontrol.wait it prefetches the CTA's weights into L2 (a hint that
//    cannot return stale data); with weight staging on (pk_set_weight_staging)
//    it loads the first units' weights and scales into shared memory there
//    instead, and only the activations wait for the previous kernel.
//  * Arithmetic: exactly the CUDA-core GEMV's (w4a16_gemv.cu). Warp w takes
//    rows [32w, 32w + 32) of every unit (one scale group), lane l columns
//    [8l, 8l + 8); one LOP3 per nibble makes the fp32 pattern of
//    (q + 8) * 16^p * 2^-149, activations are pre-scaled by 2^S, one packed
//    fma.rn.f32x2 per two weights accumulates exact products, and per unit
//    the +8 offset is removed, 2^(149 - S - 4p) undone and the fp32 group
//    scale applied. All shared-memory traffic uses explicit ld/st.shared.
//  * Reduction. The 8 warps' column sums meet in shared memory; then, after
//    a cluster barrier, CTA r of the strip reads its share of the columns
//    from all `split` CTAs' shared memory (distributed shared memory) and
//    sums them in CTA order: deterministic, no global workspace, no atomics.
#include "pk_common.cuh"

#include <cstring>
#include <mutex>
#include <type_traits>

#include "pk_internal.h"

namespace pk {
namespace {

constexpr int kRows = 256;              // K rows per unit
constexpr int kCols = 256;              // columns per strip
constexpr int kRowBytes = kCols / 2;    // packed bytes per row of a strip
constexpr int kWarps = 8;               // dequant/FMA warps
constexpr int kProducerWarp = kWarps;
constexpr int kThreads = (kWarps + 1) * 32;
constexpr int kRowsPerWarp = kRows / kWarps;  // 32
constexpr int kGroup = 128;
constexpr int kSub = 4;
constexpr int kSubRows = kRows / kSub;            // 64
constexpr int kSubWBytes = kSubRows * kRowBytes;  // 8192
constexpr int kMaxSplit = 8;
constexpr int kStages = 3;
constexpr int kWBytes = kRows * kRowBytes;              // 32768
constexpr int kSBytes = (kRows / kGroup) * kCols * 2;   // 1024: two 16-bit scale rows
constexpr int kABytes = kRows * 2;                      // 512
constexpr int kSlotBytes = kWBytes + kSBytes + kABytes;  // 34304 = 268 * 128
constexpr int kRingBytes = kStages * kSlotBytes;
constexpr int kPairOff = kRingBytes;                     // per-warp activation pairs
constexpr int kPairBytes = kWarps * kRowsPerWarp * 8;
constexpr int kBarOff = kPairOff + kPairBytes;
constexpr int kNumBars = kStages * (kSub + 2);           // full[kSub], afull, empty per slot
constexpr int kSmemBytes = kBarOff + kNumBars * 8 + 128;  // + 128 for the alignment fix-up
// At the end the ring is free: the cross-warp sums and the CTA's column sums
// (read by the cluster) reuse its first bytes.
constexpr int kRedOff = 0;                               // [kWarps][kCols] floats
constexpr int kSumOff = kWarps * kCols * 4;              // [kCols] floats
static_assert(kSumOff + kCols * 4 <= kRingBytes, "reduction buffers fit the ring");
static_assert(kSmemBytes <= 115712, "two CTAs (this launch and the next) must fit an SM");
static_assert(kSlotBytes % 128 == 0, "slots stay 128-byte aligned");

struct DecodeConsts {
  uint32_t x[4];
};

struct ClusterParams {
  int N, K;
  int split;            // CTAs per strip = cluster size
  int units;            // units per strip (K / 256)
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

__device__ __forceinline__ void cluster_arrive_release() {
  asm volatile("barrier.cluster.arrive.release.aligned;" ::: "memory");
}
__device__ __forceinline__ void cluster_wait_acquire() {
  asm volatile("barrier.cluster.wait.acquire.aligned;" ::: "memory");
}

template <typename T, bool kGrouped>
__global__ void __launch_bounds__(kThreads, 2)
    w4a16_gemv_cluster_kernel(const __grid_constant__ CUtensorMap tmW,
                              const __grid_constant__ CUtensorMap tmA,
                              const __grid_constant__ CUtensorMap tmS,
                              const __grid_constant__ ClusterParams p, const DecodeConsts dc) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 127) &
                                             ~static_cast<uintptr_t>(127));
  const uint32_t sbase = smem_u32(smem);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + kBarOff);  // [slot][sub-box]
  uint64_t* afull = full + kStages * kSub;                        // [slot]
  uint64_t* empty = afull + kStages;                              // [slot]

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
    fence_barrier_init();
  }
  __syncthreads();
  // The next launch may start its prologue (weight prefetch) now; it waits
  // for this grid before reading activations or writing anything.
  griddep_launch_dependents();

  bool failed = false;
  uint64_t tot[4] = {0ull, 0ull, 0ull, 0ull};
  if (warp == kProducerWarp) {
    if (lane == 0) {
      tma_prefetch_desc(&tmW);
      tma_prefetch_desc(&tmA);
      if constexpr (kGrouped) tma_prefetch_desc(&tmS);
      const uint32_t tx0 = kSubWBytes + (kGrouped ? kSBytes : 0);
      auto issue_w = [&](int i, int slot) {
        const int k0 = (u0 + i) * kRows;
        uint8_t* base = smem + slot * kSlotBytes;
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
        mbar_arrive_expect_tx(&afull[slot], kABytes);
        tma_load_2d(smem + slot * kSlotBytes + kWBytes + kSBytes, &tmA, &afull[slot],
                    (u0 + i) * kRows, 0);
      };
      const int pre = n_units < kStages ? n_units : kStages;
      if (p.early) {
        for (int i = 0; i < pre; ++i) issue_w(i, i);
      }
      // the rest of the CTA's weights (all of them without staging) into L2
      for (int i = p.early ? pre : 0; i < n_units && i < pre + 4 * kStages; ++i) {
        const int k0 = (u0 + i) * kRows;
        for (int j = 0; j < kSub; ++j) tma_prefetch_l2_2d(&tmW, strip * kRowBytes, k0 + j * kSubRows);
        if constexpr (kGrouped) tma_prefetch_l2_2d(&tmS, strip * kCols, k0 / kGroup);
      }
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
    // -8 * 16^p * 2^-149 for the column pairs' positions (2,3) and (4,5)
    const uint64_t off23 = pack2(__uint_as_float(0x80000800u), __uint_as_float(0x80008000u));
    const uint64_t off45 = pack2(__uint_as_float(0x80080000u), __uint_as_float(0x80800000u));
    const uint32_t pairs = sbase + kPairOff + warp * kRowsPerWarp * 8;
    constexpr int kWarpsPerSub = kSubRows / kRowsPerWarp;  // 2
    for (int i = 0, slot = 0, round = 0; i < n_units; ++i) {
      const uint32_t base = sbase + slot * kSlotBytes;
      if (!failed && !mbar_wait_sleep(&afull[slot], round & 1, p.status, kSiteGemvConsumer))
        failed = true;
      // Activations: lane l scales row 32w + l; S = clamp(248 - e_max, 30, 127)
      // from the largest exponent among the warp's rows.
      const float av = lds_act<T>(base + kWBytes + kSBytes + (warp * kRowsPerWarp + lane) * 2);
      uint32_t emax = (__float_as_uint(av) >> 23) & 0xFFu;
      emax = __reduce_max_sync(0xffffffffu, emax);
      int S = 248 - static_cast<int>(emax);
      S = S < 30 ? 30 : (S > 127 ? 127 : S);
      const float as = av * exp2i(S);
      sts_u64(pairs + lane * 8, pack2(as, as));
      float t = as;
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) t += __shfl_xor_sync(0xffffffffu, t, o);
      const uint64_t asum = pack2(t, t);
      // 2^(149 - S - 4p) for the pairs' positions (2,3) and (4,5)
      const uint64_t pw23 = pack2(exp2i(141 - S), exp2i(137 - S));
      const uint64_t pw45 = pack2(exp2i(133 - S), exp2i(129 - S));
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
        scales8<T>(lds_v4(base + kWBytes + srow * kCols * 2 + lane * 16), sc);
      } else {
#pragma unroll
        for (int q = 0; q < 4; ++q) sc[q] = pack2(p.scalar_scale, p.scalar_scale);
      }
      __syncwarp();

      uint64_t acc[4] = {0ull, 0ull, 0ull, 0ull};
      const uint32_t wrow = base + warp * kRowsPerWarp * kRowBytes + lane * 4;
#pragma unroll
      for (int b = 0; b < kRowsPerWarp / 8; ++b) {
        uint32_t wv[8];
        uint64_t a2[8];
#pragma unroll
        for (int r = 0; r < 8; ++r) wv[r] = lds_u32(wrow + (b * 8 + r) * kRowBytes);
#pragma unroll
        for (int r = 0; r < 8; ++r) a2[r] = lds_u64(pairs + (b * 8 + r) * 8);
#pragma unroll
        for (int r = 0; r < 8; ++r) {
          const uint32_t w = wv[r];
          const uint32_t lo = w << 8, hi = w >> 8;
          uint64_t d[4];
          d[0] = pack2(__uint_as_float((lo & 0xF00u) ^ dc.x[0]), __uint_as_float((lo & 0xF000u) ^ dc.x[1]));
          d[1] = pack2(__uint_as_float((w & 0xF00u) ^ dc.x[0]), __uint_as_float((w & 0xF000u) ^ dc.x[1]));
          d[2] = pack2(__uint_as_float((w & 0xF0000u) ^ dc.x[2]), __uint_as_float((w & 0xF00000u) ^ dc.x[3]));
          d[3] = pack2(__uint_as_float((hi & 0xF0000u) ^ dc.x[2]), __uint_as_float((hi & 0xF00000u) ^ dc.x[3]));
#pragma unroll
          for (int q = 0; q < 4; ++q) acc[q] = fma2(d[q], a2[r], acc[q]);
        }
      }
      // fold the unit: remove the +8 offset, undo 2^S * 16^p, apply the scale
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const uint64_t c = fma2(q < 2 ? off23 : off45, asum, acc[q]);
        tot[q] = fma2(mul2(c, q < 2 ? pw23 : pw45), sc[q], tot[q]);
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
    const float2 a0 = unpack2(tot[0]), a1 = unpack2(tot[1]);
    const float2 a2 = unpack2(tot[2]), a3 = unpack2(tot[3]);
    const uint32_t dst = sbase + kRedOff + (warp * kCols + lane * 8) * 4;
    sts_v4f(dst, a0.x, a0.y, a1.x, a1.y);
    sts_v4f(dst + 16, a2.x, a2.y, a3.x, a3.y);
  }
  __syncthreads();
  if (threadIdx.x < kCols) {
    float s = 0.0f;
#pragma unroll
    for (int w = 0; w < kWarps; ++w) s += lds_f32(sbase + kRedOff + (w * kCols + threadIdx.x) * 4);
    sts_f32(sbase + kSumOff + threadIdx.x * 4, s);
  }
  cluster_arrive_release();
  cluster_wait_acquire();  // every CTA of the strip has its column sums in place
  bool stored = false;
  if (!failed) {
    // CTA `rank` sums its share of the strip's columns over the cluster, in
    // CTA order
    const int c0 = kCols * rank / p.split, c1 = kCols * (rank + 1) / p.split;
    const int col = c0 + static_cast<int>(threadIdx.x);
    if (col < c1) {
      const uint32_t addr = sbase + kSumOff + col * 4;
      float x[kMaxSplit];
#pragma unroll
      for (int j = 0; j < kMaxSplit; ++j)
        if (j < p.split) x[j] = ld_cluster_f32(cluster_map(addr, static_cast<uint32_t>(j)));
      float v = 0.0f;
#pragma unroll
      for (int j = 0; j < kMaxSplit; ++j)
        if (j < p.split) v += x[j];
      emit_out(p.out, p.peers, p.out_dtype, static_cast<int64_t>(strip) * kCols + col, v);
      stored = true;
    }
  }
  cluster_arrive_release();
  cluster_wait_acquire();  // keep every CTA's shared memory alive until all reads are done
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
    st[7] = 0;
  }
  if (p.peers.world > 1) peer_exchange_finish(p.peers, stored, p.status, kSiteGemvPeers);
}

CUtensorMapDataType tmap_type16(int dt) {
  return dt == PK_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
}

// Whether clusters of `split` CTAs of this kernel can be resident (per
// device and split; 0 unknown, 1 yes, 2 no).
template <typename Kern>
bool cluster_fits(Kern kernel, int split) {
  static int cache[64][kMaxSplit + 1] = {};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return false;
  int& c = cache[dev][split];
  if (c == 0) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(split, 1, 1);
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = kSmemBytes;
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
uint64_t* phase_stamps(size_t need) {
  return g_phase_stamps != nullptr && g_phase_stamp_bytes >= need ? g_phase_stamps : nullptr;
}

// CTAs per strip: as many as keep strips * split within one CTA per SM, at
// most 8 (a portable cluster) and at most one per 256-row unit.
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
  if (M != 1) return false;
  if (N % kCols != 0 || K % kRows != 0 || N <= 0 || K <= 0) return false;
  if (N > (1ll << 30) || K > (1ll << 30)) return false;
  if (gemv_cluster_split(N, K) < 1) return false;
  if (lda % 8 != 0 || (reinterpret_cast<uintptr_t>(a) & 15) != 0) return false;
  if ((reinterpret_cast<uintptr_t>(wp) & 15) != 0) return false;
  if (scales != nullptr && (group != kGroup || (reinterpret_cast<uintptr_t>(scales) & 15) != 0))
    return false;
  return true;
}

// The cluster form wherever its grid keeps at least 3/4 of the SMs busy with
// at least two CTAs per strip (below that the stream-K GEMV balances better).
bool gemv_cluster_preferred(int64_t M, int64_t N, int64_t K) {
  if (M != 1 || N % kCols != 0) return false;
  const int split = gemv_cluster_split(N, K);
  return split >= 2 && (N / kCols) * split * 4 >= 3ll * num_sms();
}

cudaError_t launch_w4a16_gemv_cluster(const DecodeArgs& a, cudaStream_t s, const char** why,
                                      const OutputShard* shard) {
  CUtensorMap tmW, tmA, tmS;
  const CUtensorMapDataType dt = tmap_type16(a.a_dtype);
  if (!encode_tmap_2d(&tmW, CU_TENSOR_MAP_DATA_TYPE_UINT8, a.wp, a.N / 2, a.K, a.N / 2, kRowBytes,
                      kSubRows, CU_TENSOR_MAP_SWIZZLE_NONE, why))
    return cudaErrorInvalidValue;
  if (!encode_tmap_2d(&tmA, dt, a.a, a.K, 1, a.lda * 2, kRows, 1, CU_TENSOR_MAP_SWIZZLE_NONE, why))
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
  p.stamps = phase_stamps(static_cast<size_t>(grid) * 64);
  if (shard != nullptr) {
    if (shard->world < 1 || shard->world > kMaxPeers || shard->done == nullptr) {
      *why = "sharded GEMV: 1 <= world <= 8 and a workspace are required";
      return cudaErrorInvalidValue;
    }
    p.peers = *shard;
  }
  const DecodeConsts dc{{0x800u, 0x8000u, 0x80000u, 0x800000u}};

  auto launch = [&](auto kernel) -> cudaError_t {
    cudaError_t e = set_max_smem(reinterpret_cast<const void*>(kernel), kSmemBytes);
    if (e != cudaSuccess) return e;
    if (p.split > 1 && !cluster_fits(kernel, p.split)) {
      *why = "clusters of the GEMV's split cannot be resident";
      return cudaErrorInvalidValue;
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(static_cast<unsigned>(grid), 1, 1);
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = kSmemBytes;
    cfg.stream = s;
    cudaLaunchAttribute attrs[2];
    attrs[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attrs[0].val.programmaticStreamSerializationAllowed = 1;
    attrs[1].id = cudaLaunchAttributeClusterDimension;
    attrs[1].val.clusterDim.x = static_cast<unsigned>(p.split);
    attrs[1].val.clusterDim.y = 1;
    attrs[1].val.clusterDim.z = 1;
    cfg.attrs = attrs;
    cfg.numAttrs = 2;
    return cudaLaunchKernelEx(&cfg, kernel, tmW, tmA, tmS, p, dc);
  };
  if (a.a_dtype == PK_BF16)
    return grouped ? launch(w4a16_gemv_cluster_kernel<__nv_bfloat16, true>)
                   : launch(w4a16_gemv_cluster_kernel<__nv_bfloat16, false>);
  return grouped ? launch(w4a16_gemv_cluster_kernel<__half, true>)
                 : launch(w4a16_gemv_cluster_kernel<__half, false>);
}

}  // namespace pk
