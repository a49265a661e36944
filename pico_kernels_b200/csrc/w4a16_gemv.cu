// W4A16 GEMV for decode shapes (M <= 2) on sm_100a, on the CUDA cores.
//
// out[M, N] = A[M, K] @ (q[K, N] * s[K/g, N])  -- gemm_int4.int4_gemm
// (gemm_int4.py:75-92) with group scales, q unpacked from Wp[K, N/2] in the
// reference's nibble order (gemm_int4.py:43-50, pack_int4_n at :65-72).
//
// At M <= 2 the layer is a stream over the packed weights (K*N/2 bytes) with
// 2*M*K*N flops: far below one flop per byte, so the tensor cores would only
// add the dequantized-operand round trip through shared memory. This kernel
// streams the weights once and does the arithmetic in fp32 on the CUDA cores.
//
//  * Units. The weights are cut into units of 256 rows x 256 columns (256 x
//    128 packed bytes, 32 KB); a "slice" is a 256-column strip, KB units tall.
//  * Work split (stream-K): units numbered slice-major, CTA c of G (two per
//    SM) takes [U*c/G, U*(c+1)/G). A CTA's range covers parts of a few slices
//    ("segments"). A segment that is a whole slice is stored directly;
//    otherwise the CTA writes its partial to the workspace (slot c + slice,
//    unique per segment) and bumps the slice's arrival counter with an
//    acq_rel atomic; the last arriver sums the slice's partials in CTA order,
//    stores, and re-arms the counter. Fixed summation order: deterministic
//    for a given SM count. (A variant with one 8-CTA cluster per slice and a
//    distributed-shared-memory reduction measured slower even at 4096^2:
//    8.1 vs 7.6 us, half the CTAs per SM.)
//  * Pipeline. Warp 8 (one thread) is the TMA producer: per unit four 2D
//    boxes of 64 weight rows, the unit's group-scale rows and the activation
//    tile A[0:M, k0:k0+256] into a ring of shared-memory slots; each weight
//    box completes its own mbarrier (the first also carries the scales and
//    activations), and a warp waits only for the box holding its rows, so
//    the arithmetic of a CTA's first unit overlaps the rest of its transfer
//    (4096^2 at M = 1 gives one unit per CTA). Before griddepcontrol.wait
//    it only prefetches weights and
//    scales into L2 (a hint that cannot return stale data), so with
//    programmatic dependent launch the DRAM fetch overlaps the previous
//    kernel's tail; every load into shared memory and every global write
//    comes after the wait.
//  * Dequant. Warps 0-7 each take 32 consecutive rows of every unit (inside
//    one scale group); lane l owns columns [8l, 8l+8) of the slice, one
//    32-bit word per row (nibble j = column 8l+j), read with explicit
//    ld.shared. One XOR with 0x88888888 turns every nibble into q + 8;
//    nibbles 0-5 are masked in place (one AND each, bit position 4p, p =
//    0..5) and nibbles 6-7 after a right shift by 8 (positions 4, 5). Read as
//    an fp32 bit pattern below 2^24 that is exactly the number (q + 8) * 16^p
//    * 2^-149 (a subnormal, or the smallest normal binade). The activations are pre-scaled by 2^S, so one
//    packed FMA per two weights accumulates a' * (q + 8) * 16^p * 2^-149 with
//    the product exact and one fp32 rounding, as a plain fp32 dot product
//    would. At the end of each unit the warp removes the +8 offset with the
//    sum of its scaled activations, A' = sum a': acc + (-8 * 16^p * 2^-149) *
//    A', multiplies by 2^(149 - S - 4p) (exact) and then by the fp32 group
//    scale. S is chosen per unit from the largest activation exponent of the
//    warp's rows, S = clamp(248 - e_max, 30, 127), which keeps every scaled
//    activation, product and sum in the normal fp32 range for any activation
//    below 2^98 in magnitude. The result is the reference's fp32
//    dequantize-then-matmul up to summation order (and one extra rounding of
//    the offset term).
#include "pk_common.cuh"

#include <cstring>
#include <type_traits>

#include "pk_internal.h"

namespace pk {
namespace {

constexpr int kRows = 256;              // K rows per unit
constexpr int kCols = 256;              // output columns per slice
constexpr int kRowBytes = kCols / 2;    // packed bytes per row of a slice
constexpr int kWarps = 8;               // dequant/FMA warps
constexpr int kProducerWarp = kWarps;
constexpr int kThreads = (kWarps + 1) * 32;
constexpr int kRowsPerWarp = kRows / kWarps;  // 32: one row per lane for the activations
constexpr int kMaxM = 2;
// A unit's weights arrive as kSub boxes of kSubRows rows, each completing its
// own mbarrier, so the warps owning the first rows start while the rest of
// the unit is still in flight (a CTA often has a single unit).
constexpr int kSub = 4;
constexpr int kSubRows = kRows / kSub;           // 64
constexpr int kSubWBytes = kSubRows * kRowBytes;  // 8192
constexpr int kMaxScaleRows = 4;        // scale rows a unit can touch (group >= 64)
constexpr int kSmemTwoPerSm = 115712;   // per-CTA limit for two resident CTAs (228 KB SM)

template <int M>
struct GemvCfg {
  // M = 1: three slots and ~113 KB; M = 2: two slots. Either way two CTAs
  // of the grid share an SM.
  static constexpr int kStages = M == 1 ? 3 : 2;
  static constexpr int kWBytes = kRows * kRowBytes;          // 32768
  static constexpr int kSBytes = kMaxScaleRows * kCols * 2;  // 2048
  static constexpr int kABytes = kRows * 2 * M;              // 512 * M
  static constexpr int kSlotBytes = ((kWBytes + kSBytes + kABytes + 127) / 128) * 128;
  static constexpr int kRingBytes = kStages * kSlotBytes;
  // Per-warp activation pairs (during a unit) and the cross-warp reduction
  // buffer (at a segment end) share one region: a segment end starts after
  // every warp's last use of its pairs and ends with a barrier.
  static constexpr int kPairBytes = kWarps * kRowsPerWarp * M * 8;
  static constexpr int kRedBytes = kWarps * kCols * 4;  // one output row at a time
  static constexpr int kScratchOff = kRingBytes;
  static constexpr int kScratchBytes = kPairBytes > kRedBytes ? kPairBytes : kRedBytes;
  static constexpr int kBarOff = kScratchOff + kScratchBytes;
  static constexpr int kSmemBytes = kBarOff + (kSub + 1) * kStages * 8 + 16 + 128;
  static constexpr int kCtasPerSm = 2;
  static_assert(kSmemBytes <= kSmemTwoPerSm, "two CTAs must fit an SM");
};

// The nibble flip 0x88888888 (every nibble q -> q + 8), as a kernel parameter
// (a constant-bank operand of the XOR).
struct DecodeConsts {
  uint32_t flip;
};

// fp32 pair helpers (packed f32x2 arithmetic, sm_100)
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

template <typename T>
__device__ __forceinline__ float to_f32(T v);
template <>
__device__ __forceinline__ float to_f32<__nv_bfloat16>(__nv_bfloat16 v) {
  return __bfloat162float(v);
}
template <>
__device__ __forceinline__ float to_f32<__half>(__half v) {
  return __half2float(v);
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

// 2^e for an unbiased exponent in the normal range.
__device__ __forceinline__ float exp2i(int e) { return __uint_as_float(static_cast<uint32_t>(e + 127) << 23); }

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
  int scale_rows;      // group-scale rows per unit in the scale box
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
__device__ __forceinline__ int group_of(int row, const GemvParams& p) {
  return p.group_shift >= 0 ? (row >> p.group_shift) : row / p.group;
}

template <int M, typename T, bool kGrouped>
__global__ void __launch_bounds__(kThreads, GemvCfg<M>::kCtasPerSm)
    w4a16_gemv_kernel(const __grid_constant__ CUtensorMap tmW,
                      const __grid_constant__ CUtensorMap tmA,
                      const __grid_constant__ CUtensorMap tmS, const GemvParams p,
                      const DecodeConsts dc) {
  using C = GemvCfg<M>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 127) &
                                             ~static_cast<uintptr_t>(127));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + C::kBarOff);  // [stage][sub-box]
  uint64_t* empty = full + C::kStages * kSub;
  volatile int* last_flag = reinterpret_cast<volatile int*>(empty + C::kStages);
  float* red = reinterpret_cast<float*>(smem + C::kScratchOff);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int NS = (p.N + kCols - 1) / kCols;
  const int KB = (p.K + kRows - 1) / kRows;
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
      for (int j = 0; j < kSub; ++j) mbar_init(&full[s * kSub + j], 1);
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
      // sub-box 0 also carries the unit's scale rows and activations
      const uint32_t tx0 = kSubWBytes + (kGrouped ? p.scale_rows * kCols * 2 : 0) + C::kABytes;
      tma_prefetch_desc(&tmW);
      tma_prefetch_desc(&tmA);
      if constexpr (kGrouped) tma_prefetch_desc(&tmS);
      const int pre = n_units < 2 * C::kStages ? n_units : 2 * C::kStages;
      for (int i = 0, s = static_cast<int>(u0 / KB), kb = static_cast<int>(u0 % KB); i < pre;
           ++i) {
        for (int j = 0; j < kSub; ++j) tma_prefetch_l2_2d(&tmW, s * kRowBytes, kb * kRows + j * kSubRows);
        if constexpr (kGrouped) tma_prefetch_l2_2d(&tmS, s * kCols, group_of(kb * kRows, p));
        if (++kb == KB) kb = 0, ++s;
      }
      griddep_wait();
      int issued = 0;
      bool ok = true;
      int slice = static_cast<int>(u0 / KB);
      int kb = static_cast<int>(u0 % KB);
      for (int i = 0, slot = 0, round = 0; i < n_units; ++i) {
        if (i >= C::kStages &&
            !mbar_wait(&empty[slot], (round - 1) & 1, p.status, kSiteGemvProducer)) {
          ok = false;
          break;
        }
        const int k0 = kb * kRows;
        uint8_t* base = smem + slot * C::kSlotBytes;
        uint64_t* fb = &full[slot * kSub];
        mbar_arrive_expect_tx(&fb[0], tx0);
        tma_load_2d(base, &tmW, &fb[0], slice * kRowBytes, k0);
        if constexpr (kGrouped)
          tma_load_2d(base + C::kWBytes, &tmS, &fb[0], slice * kCols, group_of(k0, p));
        tma_load_2d(base + C::kWBytes + C::kSBytes, &tmA, &fb[0], k0, 0);
        for (int j = 1; j < kSub; ++j) {
          mbar_arrive_expect_tx(&fb[j], kSubWBytes);
          tma_load_2d(base + j * kSubWBytes, &tmW, &fb[j], slice * kRowBytes, k0 + j * kSubRows);
        }
        issued = i + 1;
        if (++kb == KB) kb = 0, ++slice;
        if (++slot == C::kStages) slot = 0, ++round;
      }
      if (!ok) {
        // let copies already issued land before the CTA's shared memory is released
        const int first = issued > C::kStages ? issued - C::kStages : 0;
        for (int i = first; i < issued; ++i)
          for (int j = 0; j < kSub; ++j)
            mbar_wait(&full[(i % C::kStages) * kSub + j], (i / C::kStages) & 1, nullptr, 0);
      }
    }
    __syncwarp();
  } else {
    // ---------------- dequant / FMA warps ----------------
    griddep_wait();
    if (stamp) t_wait = globaltimer();
    // -8 * 16^p * 2^-149 for the column pairs' positions (2,3) and (4,5): the
    // same bit patterns as the sign flips, negated
    const uint64_t off01 = pack2(__uint_as_float(0x80000008u), __uint_as_float(0x80000080u));
    const uint64_t off23 = pack2(__uint_as_float(0x80000800u), __uint_as_float(0x80008000u));
    const uint64_t off45 = pack2(__uint_as_float(0x80080000u), __uint_as_float(0x80800000u));
    uint64_t acc[M][4], tot[M][4];
#pragma unroll
    for (int m = 0; m < M; ++m)
#pragma unroll
      for (int q = 0; q < 4; ++q) acc[m][q] = tot[m][q] = 0ull;

    uint64_t* pairs = reinterpret_cast<uint64_t*>(smem + C::kScratchOff) + warp * kRowsPerWarp * M;
    bool failed = false;
    int slice = static_cast<int>(u0 / KB);
    int kb = static_cast<int>(u0 % KB);
    for (int i = 0, slot = 0, round = 0; i < n_units;
         ++i, slice += (kb + 1 == KB), kb = (kb + 1 == KB ? 0 : kb + 1),
             slot = (slot + 1 == C::kStages ? 0 : slot + 1), round += (slot == 0)) {
      const int k0 = kb * kRows;
      if (!failed && !mbar_wait_sleep(&full[slot * kSub], round & 1, p.status, kSiteGemvConsumer))
        failed = true;
      if (stamp && i == 0) t_first = globaltimer();
      const uint8_t* base = smem + slot * C::kSlotBytes;

      // Activations: lane l converts row 32*warp + l of every output row m.
      // S = clamp(248 - e_max, 30, 127) from the largest exponent in the warp.
      float av[M];
      uint32_t emax = 0;
      {
        const T* a = reinterpret_cast<const T*>(base + C::kWBytes + C::kSBytes);
#pragma unroll
        for (int m = 0; m < M; ++m) {
          av[m] = to_f32<T>(a[m * kRows + warp * kRowsPerWarp + lane]);
          const uint32_t e = (__float_as_uint(av[m]) >> 23) & 0xFFu;
          emax = e > emax ? e : emax;
        }
      }
      emax = __reduce_max_sync(0xffffffffu, emax);
      int S = 248 - static_cast<int>(emax);
      S = S < 30 ? 30 : (S > 127 ? 127 : S);
      const float two_s = exp2i(S);
      uint64_t asum[M];
#pragma unroll
      for (int m = 0; m < M; ++m) {
        const float as = av[m] * two_s;
        pairs[lane * M + m] = pack2(as, as);
        float t = as;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) t += __shfl_xor_sync(0xffffffffu, t, o);
        asum[m] = pack2(t, t);
      }
      // 2^(149 - S - 4p) for the pairs' positions (2,3) and (4,5)
      const uint64_t pw01 = pack2(exp2i(149 - S), exp2i(145 - S));
      const uint64_t pw23 = pack2(exp2i(141 - S), exp2i(137 - S));
      const uint64_t pw45 = pack2(exp2i(133 - S), exp2i(129 - S));
      uint64_t sc[4];
      if constexpr (kGrouped) {
        const int srow = group_of(k0 + warp * kRowsPerWarp, p) - group_of(k0, p);
        scales8<T>(*reinterpret_cast<const uint4*>(base + C::kWBytes + srow * kCols * 2 + lane * 16),
                   sc);
      } else {
#pragma unroll
        for (int q = 0; q < 4; ++q) sc[q] = pack2(p.scalar_scale, p.scalar_scale);
      }
      __syncwarp();
      // this warp's rows are in sub-box warp * kRowsPerWarp / kSubRows
      constexpr int kWarpsPerSub = kSubRows / kRowsPerWarp;
      if (warp >= kWarpsPerSub && !failed &&
          !mbar_wait_sleep(&full[slot * kSub + warp / kWarpsPerSub], round & 1, p.status,
                           kSiteGemvConsumer))
        failed = true;

      const uint32_t wrow = smem_u32(base) + (warp * kRowsPerWarp * 32 + lane) * 4;
      const uint32_t pairs_s = smem_u32(pairs);
#pragma unroll
      for (int b = 0; b < kRowsPerWarp / 8; ++b) {
        uint32_t wv[8];
#pragma unroll
        for (int r = 0; r < 8; ++r) wv[r] = lds_u32(wrow + (b * 8 + r) * 128);
#pragma unroll
        for (int r = 0; r < 8; ++r) {
          const uint32_t w = wv[r] ^ dc.flip;  // every nibble q -> q + 8
          const uint32_t hi = w >> 8;          // nibbles 6, 7 at positions 4, 5
          uint64_t d[4];
          d[0] = pack2(__uint_as_float(w & 0xFu), __uint_as_float(w & 0xF0u));
          d[1] = pack2(__uint_as_float(w & 0xF00u), __uint_as_float(w & 0xF000u));
          d[2] = pack2(__uint_as_float(w & 0xF0000u), __uint_as_float(w & 0xF00000u));
          d[3] = pack2(__uint_as_float(hi & 0xF0000u), __uint_as_float(hi & 0xF00000u));
#pragma unroll
          for (int m = 0; m < M; ++m) {
            const uint64_t a2 = lds_u64(pairs_s + ((b * 8 + r) * M + m) * 8);
#pragma unroll
            for (int q = 0; q < 4; ++q) acc[m][q] = fma2(d[q], a2, acc[m][q]);
          }
        }
      }
      // fold the unit: remove the +8 offset, undo 2^S * 16^p, apply the scale
#pragma unroll
      for (int m = 0; m < M; ++m)
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const uint64_t off = q == 0 ? off01 : (q == 1 ? off23 : off45);
          const uint64_t pw = q == 0 ? pw01 : (q == 1 ? pw23 : pw45);
          const uint64_t c = fma2(off, asum[m], acc[m][q]);
          tot[m][q] = fma2(mul2(c, pw), sc[q], tot[m][q]);
          acc[m][q] = 0ull;
        }
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[slot]);

      const bool seg_end = (i + 1 == n_units) || (kb + 1 == KB);
      if (!seg_end) continue;

      // ---- end of a segment: reduce over warps, one output row at a time ----
      if (stamp) t_comp = globaltimer();
      named_bar_sync(1, kWarps * 32);  // every warp is done with its pairs
      const int t = threadIdx.x;       // column within the slice
      float v[M];
#pragma unroll
      for (int m = 0; m < M; ++m) {
        float4* dst = reinterpret_cast<float4*>(red + warp * kCols + lane * 8);
        const float2 a0 = unpack2(tot[m][0]), a1 = unpack2(tot[m][1]);
        const float2 a2 = unpack2(tot[m][2]), a3 = unpack2(tot[m][3]);
        dst[0] = make_float4(a0.x, a0.y, a1.x, a1.y);
        dst[1] = make_float4(a2.x, a2.y, a3.x, a3.y);
#pragma unroll
        for (int q = 0; q < 4; ++q) tot[m][q] = 0ull;
        named_bar_sync(1, kWarps * 32);
        float s = 0.0f;
#pragma unroll
        for (int w = 0; w < kWarps; ++w) s += red[w * kCols + t];
        v[m] = s;
        named_bar_sync(1, kWarps * 32);
      }
      const int64_t col = static_cast<int64_t>(slice) * kCols + t;
      auto store = [&](const float* vals) {
        if (col >= p.N) return;
        stored = true;
#pragma unroll
        for (int m = 0; m < M; ++m) store_col(p, m, col, vals[m]);
      };
      const int64_t cfirst = unit_owner(static_cast<int64_t>(slice) * KB, U, G);
      const int64_t clast = unit_owner(static_cast<int64_t>(slice) * KB + KB - 1, U, G);
      if (cfirst == clast) {
        store(v);
        continue;
      }
      float* mine = p.partials + (cta + slice) * (M * kCols);
#pragma unroll
      for (int m = 0; m < M; ++m) __stcg(mine + m * kCols + t, v[m]);
      named_bar_sync(1, kWarps * 32);
      if (t == 0) {
        // release: the CTA's partial (ordered before by the barrier) becomes
        // visible with the count; acquire: the last arriver sees every partial
        const unsigned arrived = atomic_add_acq_rel(&p.sems[slice], 1u);
        *last_flag = arrived == static_cast<unsigned>(clast - cfirst) ? 1 : 0;
      }
      named_bar_sync(1, kWarps * 32);
      if (*last_flag) {
        was_last = true;
        float sum[M];
#pragma unroll
        for (int m = 0; m < M; ++m) sum[m] = 0.0f;
        // A batch of partials' loads in flight before the adds, which stay in
        // CTA order (a loop of load-then-add pays one L2 round trip per CTA).
        constexpr int kBatch = 16 / M;
        for (int64_t c0 = cfirst; c0 <= clast; c0 += kBatch) {
          float x[kBatch][M];
#pragma unroll
          for (int j = 0; j < kBatch; ++j) {
            if (c0 + j <= clast) {
              const float* src = p.partials + (c0 + j + slice) * (M * kCols);
#pragma unroll
              for (int m = 0; m < M; ++m) x[j][m] = __ldcg(src + m * kCols + t);
            }
          }
#pragma unroll
          for (int j = 0; j < kBatch; ++j) {
            if (c0 + j <= clast) {
#pragma unroll
              for (int m = 0; m < M; ++m) sum[m] += x[j][m];
            }
          }
        }
        store(sum);
        if (t == 0) p.sems[slice] = 0u;  // re-arm for the next call
      }
      named_bar_sync(1, kWarps * 32);  // last_flag is rewritten by the next segment
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

// Stream-K grid: two CTAs per SM, at most one CTA per unit.
int64_t gemv_grid(int64_t N, int64_t K) {
  const int64_t U = ((N + kCols - 1) / kCols) * ((K + kRows - 1) / kRows);
  const int64_t cap = 2 * static_cast<int64_t>(num_sms());
  return U < cap ? U : cap;
}

int scale_rows_for(int group) {
  // group-scale rows a 256-row unit can touch
  const int span = (kRows + group - 1) / group + (kRows % group != 0 ? 1 : 0);
  return span < kMaxScaleRows ? span : kMaxScaleRows;
}

}  // namespace

bool gemv_preferred(int64_t M, int64_t N, int64_t K) {
  // Measured on B200 against the tensor-core decode kernel: at M = 1 the GEMV
  // is faster at every size (4096 x 4096: 7.8 vs 8.4 us; Llama-70B up_proj:
  // 35 vs 66 us); at M = 2 only for layers of 16 MB or more (4096 x 4096:
  // 10.1 vs 8.5 us; up_proj: 46 vs 66 us); from M = 3 on the CUDA-core FMAs
  // cost more than the tensor core's wasted columns.
  if (M == 1) return true;
  return M == 2 && K * (N / 2) >= (16ll << 20);
}

bool gemv_supported(int64_t M, int64_t N, int64_t K, int group, const void* scales, int64_t lda,
                    const void* a, const void* wp) {
  if (M < 1 || M > kMaxM) return false;
  if (N < kCols || N % 32 != 0 || K < kRows) return false;
  if (N > (1ll << 30) || K > (1ll << 30)) return false;
  if ((N + kCols - 1) / kCols >= kMaxCounters) return false;  // the last counter: sharded calls
  if (lda % 8 != 0 || (reinterpret_cast<uintptr_t>(a) & 15) != 0) return false;
  if ((reinterpret_cast<uintptr_t>(wp) & 15) != 0) return false;
  if (scales != nullptr &&
      (group <= 0 || group % 64 != 0 || (reinterpret_cast<uintptr_t>(scales) & 15) != 0))
    return false;
  return true;
}

size_t gemv_workspace_bytes(int64_t M, int64_t N, int64_t K) {
  const int64_t NS = (N + kCols - 1) / kCols;
  const int64_t KB = (K + kRows - 1) / kRows;
  const int64_t U = NS * KB;
  const int64_t G = gemv_grid(N, K);
  bool split = false;
  for (int64_t j = 0; j < NS && !split; ++j)
    split = unit_owner(j * KB, U, G) != unit_owner(j * KB + KB - 1, U, G);
  if (!split) return 0;
  return kCounterBytes + static_cast<size_t>(G + NS) * M * kCols * sizeof(float);
}

cudaError_t launch_w4a16_gemv(const DecodeArgs& a, cudaStream_t s, const char** why,
                              const OutputShard* shard) {
  CUtensorMap tmW, tmA, tmS;
  const CUtensorMapDataType dt = tmap_type16(a.a_dtype);
  if (!encode_tmap_2d(&tmW, CU_TENSOR_MAP_DATA_TYPE_UINT8, a.wp, a.N / 2, a.K, a.N / 2, kRowBytes,
                      kSubRows, CU_TENSOR_MAP_SWIZZLE_NONE, why))
    return cudaErrorInvalidValue;
  if (!encode_tmap_2d(&tmA, dt, a.a, a.K, a.M, a.lda * 2, kRows, static_cast<uint32_t>(a.M),
                      CU_TENSOR_MAP_SWIZZLE_NONE, why))
    return cudaErrorInvalidValue;
  const bool grouped = a.scales != nullptr;
  GemvParams p{};
  p.N = static_cast<int>(a.N);
  p.K = static_cast<int>(a.K);
  p.group = grouped ? a.group : kRows;
  p.scale_rows = grouped ? scale_rows_for(a.group) : 1;
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
    const int64_t groups = (a.K + a.group - 1) / a.group;
    if (!encode_tmap_2d(&tmS, dt, a.scales, a.N, groups, a.N * 2, kCols,
                        static_cast<uint32_t>(p.scale_rows), CU_TENSOR_MAP_SWIZZLE_NONE, why))
      return cudaErrorInvalidValue;
  } else {
    std::memcpy(&tmS, &tmW, sizeof(tmS));  // unused
  }
  const int64_t G = gemv_grid(a.N, a.K);
  if (gemv_workspace_bytes(a.M, a.N, a.K) > 0 && (a.partials == nullptr || a.sems == nullptr)) {
    *why = "the split-K GEMV needs a workspace";
    return cudaErrorInvalidValue;
  }
  const DecodeConsts dc{0x88888888u};

  auto launch = [&](auto kernel, int smem_bytes) -> cudaError_t {
    cudaError_t e =
        set_max_smem(reinterpret_cast<const void*>(kernel), smem_bytes);
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
  auto by_m = [&](auto tag, auto grouped_tag) -> cudaError_t {
    using T = decltype(tag);
    constexpr bool kG = decltype(grouped_tag)::value;
    if (a.M == 1) return launch(w4a16_gemv_kernel<1, T, kG>, GemvCfg<1>::kSmemBytes);
    return launch(w4a16_gemv_kernel<2, T, kG>, GemvCfg<2>::kSmemBytes);
  };
  if (a.a_dtype == PK_BF16) {
    return grouped ? by_m(__nv_bfloat16{}, std::true_type{})
                   : by_m(__nv_bfloat16{}, std::false_type{});
  }
  return grouped ? by_m(__half{}, std::true_type{}) : by_m(__half{}, std::false_type{});
}

}  // namespace pk
