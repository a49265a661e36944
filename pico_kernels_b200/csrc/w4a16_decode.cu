// W4A16 GEMM for decode shapes (M <= 32) on sm_100a.
//
// out[M, N] = A[M, K] @ (q[K, N] * s[K/128, N])  -- gemm_int4.int4_gemm
// (gemm_int4.py:75-92) with group scales; q unpacked from Wp[K, N/2] with the
// reference's nibble order (gemm_int4.py:43-50).
//
// Swap-AB: the weight tile is the MMA's M = 128 operand (128 output columns),
// the activations its N = NA operand (M padded to NA = 16 or 32 by TMA zero
// fill), so D[n, m] lives in NA TMEM columns. One CTA owns 128 columns and a contiguous
// range of 128-row K stages (one quantization group each). Warp roles:
//   warps 0-3  epilogue: per group, read the fp32 partial D_g from TMEM and
//              accumulate s[g, n] * D_g in registers (the scale is applied in
//              fp32, after an exact integer MMA); then the split-K reduction
//              and the output store;
//   warp 4     TMA producer: packed weights + activation tile per stage into a
//              ring of shared-memory slots;
//   warp 5     TMEM allocator and MMA issuer (one thread);
//   warps 6-13 dequant: int4 -> exact 16-bit integer codes in registers,
//              written as a 128B-swizzled MN-major operand tile.
// All hand-offs are mbarriers with bounded waits.
//
// Split-K: the `split` CTAs of a column tile either form a thread-block
// cluster and reduce their partials through distributed shared memory, or
// (split > 8) write partials to a global workspace where the last arriver
// reduces them. Both sum partials in split order starting from zero, so the
// result is deterministic and identical between the two modes.
#include "pk_common.cuh"

namespace pk {
namespace {

constexpr int kEpiWarps = 4;
constexpr int kTmaWarp = 4;
constexpr int kMmaWarp = 5;
constexpr int kDeqWarp0 = 6;
constexpr int kDeqWarps = 8;
constexpr int kThreads = (kDeqWarp0 + kDeqWarps) * 32;  // 448

constexpr int kBN = 128;      // output columns per CTA (MMA M)
constexpr int kBK = 128;      // K rows per stage = one quantization group
constexpr int kGroupSlots = 8;                       // TMEM ring of per-group partials
constexpr int kMaxClusterSplit = 8;
constexpr int kWBytes = kBK * (kBN / 2);             // 128 rows x 64 B: 8192
constexpr int kDeqBytes = kBN * 64 * 2;              // 16384 per half stage
constexpr int kDeqLBO = 8192;                        // between the two 64-column atoms
constexpr int kMaxNA = 32;

// Per activation width NA (M padded to the MMA's N): 16 for M <= 16, 32 for
// M <= 32. Shared memory from a 1024-aligned base: a ring of TMA slots (the
// activation tile, then the packed weights), the dequantized half-stage ring,
// barriers. NA = 16 keeps a 6-slot ring (2-6 % faster than 4 slots with 3
// dequant buffers); NA = 32 keeps 4 so that two CTAs still share an SM.
template <int NA>
struct DecCfg {
  static constexpr int kSlots = NA == 16 ? 6 : 4;
  static constexpr int kDeqBufs = 2;
  static constexpr int kTmemCols = kGroupSlots * NA;   // 128 / 256
  static constexpr int kAtileBytes = 2 * NA * 128;     // two 64-column SW128 boxes
  static constexpr int kSlotBytes = kAtileBytes + kWBytes;
  static constexpr int kSlotA = 0;
  static constexpr int kSlotW = kAtileBytes;
  static constexpr int kDeqOff = kSlots * kSlotBytes;
  static constexpr int kBarOff = kDeqOff + kDeqBufs * kDeqBytes;
  static constexpr int kNumBars = 2 * kSlots + 2 * kDeqBufs + 2 * kGroupSlots;
  static constexpr int kSmemBytes = kBarOff + kNumBars * 8 + 16 + 1024;
  static constexpr int kRedOff = kDeqOff;              // split-K partials reuse the dequant ring
  static_assert(NA * kBN * 4 <= kDeqBufs * kDeqBytes, "reduction buffer fits");
  static_assert(kSmemBytes <= 113 * 1024, "two CTAs per SM");
  static_assert(2 * kTmemCols <= 512, "two CTAs' TMEM fits an SM");
};

template <typename T>
struct TypeFmt;
template <>
struct TypeFmt<__nv_bfloat16> {
  static constexpr uint32_t kFmt = 1;
};
template <>
struct TypeFmt<__half> {
  static constexpr uint32_t kFmt = 0;
};

__device__ __forceinline__ float ld_scale(const __nv_bfloat16* p) { return __bfloat162float(*p); }
__device__ __forceinline__ float ld_scale(const __half* p) { return __half2float(*p); }

template <typename T, bool kGrouped, int NA>
__global__ void __launch_bounds__(kThreads, 2)
    w4a16_decode_kernel(const __grid_constant__ CUtensorMap tmA,
                        const __grid_constant__ CUtensorMap tmW, const T* __restrict__ scales,
                        int M, int N, int K, int split, int use_cluster, float scalar_scale,
                        void* __restrict__ out, int out_dtype, int64_t ldo,
                        float* __restrict__ partials, unsigned* __restrict__ sems,
                        int* __restrict__ status, const __grid_constant__ OutputShard peers) {
  using C = DecCfg<NA>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + C::kBarOff);
  uint64_t* slot_empty = full + C::kSlots;
  uint64_t* deq_full = slot_empty + C::kSlots;
  uint64_t* deq_empty = deq_full + C::kDeqBufs;
  uint64_t* tm_full = deq_empty + C::kDeqBufs;
  uint64_t* tm_empty = tm_full + kGroupSlots;
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(tm_empty + kGroupSlots);
  int* s_flag = reinterpret_cast<int*>(tmem_holder + 1);

  const int tid = threadIdx.x;
  const int warp = tid >> 5;
  const int lane = tid & 31;
  const int tile = blockIdx.x;
  const int ks = blockIdx.y;
  const int total_stages = K / kBK;
  const int g_begin = static_cast<int>((static_cast<int64_t>(ks) * total_stages) / split);
  const int g_end = static_cast<int>((static_cast<int64_t>(ks + 1) * total_stages) / split);
  const int S = g_end - g_begin;

  if (warp == kTmaWarp && lane == 0) {
    for (int i = 0; i < C::kSlots; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&slot_empty[i], 1);
    }
    for (int i = 0; i < C::kDeqBufs; ++i) {
      mbar_init(&deq_full[i], kDeqWarps);
      mbar_init(&deq_empty[i], 1);
    }
    for (int i = 0; i < kGroupSlots; ++i) {
      mbar_init(&tm_full[i], 1);
      mbar_init(&tm_empty[i], kEpiWarps);
    }
    fence_barrier_init();
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmW);
  }
  if (warp == kMmaWarp) tmem_alloc(tmem_holder, C::kTmemCols);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_holder;

  // Everything above overlaps the previous grid's tail; global memory is
  // touched only after it has completed.
  griddep_wait();
  griddep_launch_dependents();

  bool fail = false;
  int issued = 0;
  if (warp == kTmaWarp) {
    // ---------------- TMA producer ----------------
    if (lane == 0) {
      for (int s = 0; s < S && !fail; ++s) {
        const int slot = s % C::kSlots;
        if (s >= C::kSlots)
          fail = !mbar_wait(&slot_empty[slot], ((s / C::kSlots) - 1) & 1, status, kSiteDecodeFull);
        if (fail) break;
        uint8_t* base = smem + slot * C::kSlotBytes;
        const int g = g_begin + s;
        mbar_arrive_expect_tx(&full[slot], C::kSlotBytes);
        tma_load_2d(base + C::kSlotW, &tmW, &full[slot], tile * (kBN / 2), g * kBK);
        tma_load_2d(base + C::kSlotA, &tmA, &full[slot], g * kBK, 0);
        tma_load_2d(base + C::kSlotA + NA * 128, &tmA, &full[slot], g * kBK + 64, 0);
        issued = s + 1;
      }
    }
  } else if (warp == kMmaWarp) {
    // ---------------- MMA issuer ----------------
    if (lane == 0) {
      constexpr uint32_t kIdesc = make_idesc(TypeFmt<T>::kFmt, true, false, 128, NA);
      const uint32_t deq_base = smem_u32(smem + C::kDeqOff);
      for (int s = 0; s < S && !fail; ++s) {
        const int slot = s % C::kSlots;
        const int gs = s % kGroupSlots;
        if (kGrouped && s >= kGroupSlots)
          fail = !mbar_wait(&tm_empty[gs], ((s / kGroupSlots) - 1) & 1, status, kSiteDecodeMma);
        for (int h = 0; h < 2 && !fail; ++h) {
          const int u = 2 * s + h;
          const int buf = u % C::kDeqBufs;
          fail = !mbar_wait(&deq_full[buf], (u / C::kDeqBufs) & 1, status, kSiteDecodeMma);
          if (fail) break;
          tc_fence_after();
          const uint32_t a_tile = smem_u32(smem + slot * C::kSlotBytes + C::kSlotA) + h * (NA * 128);
          const uint32_t d_tile = deq_base + buf * kDeqBytes;
          const uint32_t d_tmem = tmem + (kGrouped ? gs * NA : 0);
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            const uint64_t adesc = make_smem_desc(d_tile + j * 2048, kDeqLBO, 1024);
            const uint64_t bdesc = make_smem_desc(a_tile + j * 32, 16, 1024);
            const uint32_t acc = kGrouped ? (h | j) : (s | h | j);
            umma_f16(d_tmem, adesc, bdesc, kIdesc, acc != 0 ? 1u : 0u);
          }
          umma_commit(&deq_empty[buf]);
        }
        if (fail) break;
        umma_commit(&slot_empty[slot]);
        if (kGrouped || s == S - 1) umma_commit(&tm_full[kGrouped ? gs : 0]);
      }
    }
  } else if (warp >= kDeqWarp0) {
    // ---------------- dequant ----------------
    // Lane mapping: 16-byte shared accesses are serviced a quarter-warp (8
    // lanes) at a time, so each quarter must read 8 different bank groups of
    // the 64-byte packed rows and write 8 different bank groups of the
    // swizzled tile. Quarter k of warp w covers rows 8w + 4(k/2) .. +3: lane t
    // takes quad q = t % 4 of row 8w + 4(k/2) + 2((q/2) ^ (k%2)) + t/4.
    const int dt = tid - kDeqWarp0 * 32;
    const int qk = lane >> 3, qt = lane & 7;
    const int wq = qt & 3;   // 16-byte quad of the 64-byte packed row: columns 32wq..32wq+31
    const int r = 8 * (dt >> 5) + 4 * (qk >> 1) + 2 * ((wq >> 1) ^ (qk & 1)) + (qt >> 2);
    const int r8 = r & 7;
    const uint32_t row_off = (r >> 3) * 1024 + r8 * 128;
    for (int s = 0; s < S && !fail; ++s) {
      const int slot = s % C::kSlots;
      fail = !mbar_wait(&full[slot], (s / C::kSlots) & 1, status, kSiteDecodeFull);
      for (int h = 0; h < 2 && !fail; ++h) {
        const int u = 2 * s + h;
        const int buf = u % C::kDeqBufs;
        if (u >= C::kDeqBufs)
          fail = !mbar_wait(&deq_empty[buf], ((u / C::kDeqBufs) - 1) & 1, status, kSiteDecodeMma);
        if (fail) break;
        const uint4 wv = *reinterpret_cast<const uint4*>(smem + slot * C::kSlotBytes + C::kSlotW +
                                                         (64 * h + r) * 64 + wq * 16);
        uint8_t* dq = smem + C::kDeqOff + buf * kDeqBytes + row_off;
        const uint32_t words[4] = {wv.x, wv.y, wv.z, wv.w};
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const int c = 4 * wq + i;  // 8-column chunk 0..15
          uint32_t o[4];
          int4_codes8<T>(words[i], o);
          *reinterpret_cast<uint4*>(dq + (c >> 3) * kDeqLBO + (((c & 7) ^ r8) << 4)) =
              make_uint4(o[0], o[1], o[2], o[3]);
        }
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) mbar_arrive(&deq_full[buf]);
      }
    }
  }

  // ---------------- epilogue: per-group scale in fp32 ----------------
  float acc[NA];
#pragma unroll
  for (int m = 0; m < NA; ++m) acc[m] = 0.0f;
  const int p = tid;  // TMEM lane (epilogue threads only)
  const int nl = (p & ~7) | int4_codes8_column(p & 7);
  const int64_t n = static_cast<int64_t>(tile) * kBN + nl;
  if (warp < kEpiWarps) {
    const uint32_t lane_base = tmem + (static_cast<uint32_t>(warp * 32) << 16);
    if (kGrouped) {
      const T* sp = scales + static_cast<int64_t>(g_begin) * N + n;
      float sc_next = S > 0 ? ld_scale(sp) : 0.0f;
      for (int s = 0; s < S && !fail; ++s) {
        const float sc = sc_next;
        if (s + 1 < S) sc_next = ld_scale(sp + static_cast<int64_t>(s + 1) * N);
        const int gs = s % kGroupSlots;
        fail = !mbar_wait(&tm_full[gs], (s / kGroupSlots) & 1, status, kSiteDecodeFinal);
        if (fail) break;
        tc_fence_after();
        // 16 columns at a time: 32 accumulators plus a 32-column load would
        // not fit the 72 registers two CTAs per SM leave a thread
#pragma unroll
        for (int c = 0; c < NA / 16; ++c) {
          uint32_t raw[16];
          tmem_ld_32x32b_x16(lane_base + gs * NA + c * 16, raw);
          tmem_ld_wait();
#pragma unroll
          for (int m = 0; m < 16; ++m)
            acc[c * 16 + m] = fmaf(sc, __uint_as_float(raw[m]), acc[c * 16 + m]);
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&tm_empty[gs]);
      }
    } else if (S > 0) {
      fail = !mbar_wait(&tm_full[0], 0, status, kSiteDecodeFinal);
      if (!fail) {
        tc_fence_after();
#pragma unroll
        for (int c = 0; c < NA / 16; ++c) {
          uint32_t raw[16];
          tmem_ld_32x32b_x16(lane_base + c * 16, raw);
          tmem_ld_wait();
#pragma unroll
          for (int m = 0; m < 16; ++m) acc[c * 16 + m] = __uint_as_float(raw[m]);
        }
      }
    }
  }

  // ---------------- split-K reduction and output ----------------
  fail = __syncthreads_or(fail) != 0;
  bool stored = false;  // this thread wrote output (sharded exchange: fence before arriving)
  if (use_cluster) {
    float* red = reinterpret_cast<float*>(smem + C::kRedOff);
    if (!fail && warp < kEpiWarps) {
#pragma unroll
      for (int m = 0; m < NA; ++m)
        if (m < M) red[m * kBN + nl] = acc[m];
    }
    cluster_sync();
    if (!fail && warp < kEpiWarps) {
      const int total = M * kBN;
      const int lo = (ks * total) / split, hi = ((ks + 1) * total) / split;
      const uint32_t red_addr = smem_u32(red);
      for (int e = lo + tid; e < hi; e += kEpiWarps * 32) {
        // every CTA's value in flight before the adds (split order kept)
        float x[kMaxClusterSplit];
#pragma unroll
        for (int j = 0; j < kMaxClusterSplit; ++j)
          if (j < split) x[j] = ld_cluster_f32(cluster_map(red_addr + e * 4, static_cast<uint32_t>(j)));
        float sum = 0.0f;
#pragma unroll
        for (int j = 0; j < kMaxClusterSplit; ++j)
          if (j < split) sum += x[j];
        const int m = e / kBN, l = e % kBN;
        emit_out(out, peers, out_dtype, m * ldo + static_cast<int64_t>(tile) * kBN + l,
                 sum * scalar_scale);
        stored = true;
      }
    }
    cluster_sync();  // keep every CTA's shared memory alive until all reads are done
  } else if (split == 1) {
    if (!fail && warp < kEpiWarps) {
#pragma unroll
      for (int m = 0; m < NA; ++m)
        if (m < M) emit_out(out, peers, out_dtype, m * ldo + n, acc[m] * scalar_scale);
      stored = true;
    }
  } else if (!fail && warp < kEpiWarps) {
    float* mine = partials + (static_cast<int64_t>(tile) * split + ks) * M * kBN;
#pragma unroll
    for (int m = 0; m < NA; ++m)
      if (m < M) __stcg(mine + m * kBN + nl, acc[m]);
    __threadfence();
    named_bar_sync(1, kEpiWarps * 32);
    if (tid == 0) *s_flag = (atomicAdd(&sems[tile], 1u) == static_cast<unsigned>(split - 1));
    named_bar_sync(1, kEpiWarps * 32);
    if (*s_flag) {
      __threadfence();
      const float* tp = partials + static_cast<int64_t>(tile) * split * M * kBN;
#pragma unroll
      for (int m = 0; m < NA; ++m) {
        if (m < M) {
          // eight partials' loads in flight before the adds (split order kept)
          float sum = 0.0f;
          for (int j0 = 0; j0 < split; j0 += 8) {
            float x[8];
#pragma unroll
            for (int jj = 0; jj < 8; ++jj) {
              const int j = j0 + jj;
              if (j < split)
                x[jj] = (j == ks) ? acc[m]
                                  : __ldcg(tp + (static_cast<int64_t>(j) * M + m) * kBN + nl);
            }
#pragma unroll
            for (int jj = 0; jj < 8; ++jj)
              if (j0 + jj < split) sum += x[jj];
          }
          emit_out(out, peers, out_dtype, m * ldo + n, sum * scalar_scale);
        }
      }
      stored = true;
      if (tid == 0) sems[tile] = 0u;  // re-arm for the next call
    }
  }

  if (fail && warp == kTmaWarp && lane == 0) {
    // let copies already issued land before the CTA's shared memory is released
    for (int s = 0; s < issued; ++s) mbar_wait(&full[s % C::kSlots], (s / C::kSlots) & 1, nullptr, 0);
  }
  tc_fence_before();
  __syncthreads();
  if (warp == kMmaWarp) tmem_dealloc(tmem, C::kTmemCols);
  if (peers.world > 1) {
    if (use_cluster) {
      // every CTA of the cluster has stored its share of the columns: one
      // system-scope fence and one arrival per cluster (by its rank 0)
      cluster_sync();
      if (cluster_ctarank() == 0)
        peer_exchange_finish(peers, true, status, kSiteDecodePeers, gridDim.x);
    } else {
      peer_exchange_finish(peers, stored, status, kSiteDecodePeers, gridDim.x * gridDim.y);
    }
  }
}

CUtensorMapDataType tmap_type(int dt) {
  return dt == PK_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
}

// Whether a cluster of `split` CTAs of this kernel can be resident (cached per
// device and split; 0 unknown, 1 yes, 2 no).
template <int NA, typename Kern>
bool cluster_fits(Kern kernel, int split) {
  static int cache[64][kMaxClusterSplit + 1] = {};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return false;
  int& c = cache[dev][split];
  if (c == 0) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(1, split, 1);
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = DecCfg<NA>::kSmemBytes;
    cudaLaunchAttribute attr;
    attr.id = cudaLaunchAttributeClusterDimension;
    attr.val.clusterDim.x = 1;
    attr.val.clusterDim.y = split;
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

}  // namespace

bool decode_supported(int64_t M, int64_t N, int64_t K, int group, const void* scales,
                      int64_t lda, const void* a) {
  if (M < 1 || M > kMaxNA) return false;
  if (N % kBN != 0 || K % kBK != 0) return false;
  if (N / kBN > kMaxCounters) return false;
  if (scales != nullptr && group != kBK) return false;
  if (lda % 8 != 0 || (reinterpret_cast<uintptr_t>(a) & 15) != 0) return false;
  if (K > (1ll << 30) || N > (1ll << 30)) return false;
  return true;
}

int decode_pick_split(int64_t M, int64_t N, int64_t K) {
  (void)M;
  const int64_t tiles = N / kBN;
  const int64_t stages = K / kBK;
  const int64_t slots = 2ll * num_sms();  // two CTAs per SM
  int64_t split = slots / (tiles > 0 ? tiles : 1);
  if (split < 1) split = 1;
  if (split > kMaxClusterSplit) split = kMaxClusterSplit;
  if (split > stages) split = stages;
  return static_cast<int>(split);
}

// Workspace of the global-memory reduction: arrival counters + fp32 partials.
// Splits up to 8 normally reduce through distributed shared memory instead
// and use it only when a cluster launch is unavailable.
size_t decode_workspace_bytes(int64_t M, int64_t N, int64_t K, int split) {
  (void)K;
  if (split <= 1) return 0;
  const int64_t tiles = N / kBN;
  return kCounterBytes + static_cast<size_t>(tiles) * split * M * kBN * sizeof(float);
}

namespace {

template <int NA>
cudaError_t launch_decode_na(const DecodeArgs& p, cudaStream_t s, const char** why,
                             const OutputShard& peers) {
  constexpr int kSmemBytes = DecCfg<NA>::kSmemBytes;
  CUtensorMap tmA, tmW;
  const CUtensorMapDataType dt = tmap_type(p.a_dtype);
  if (!encode_tmap_2d(&tmA, dt, p.a, p.K, p.M, p.lda * 2, 64, NA,
                      CU_TENSOR_MAP_SWIZZLE_128B, why))
    return cudaErrorInvalidValue;
  if (!encode_tmap_2d(&tmW, CU_TENSOR_MAP_DATA_TYPE_UINT8, p.wp, p.N / 2, p.K, p.N / 2, kBN / 2,
                      kBK, CU_TENSOR_MAP_SWIZZLE_NONE, why))
    return cudaErrorInvalidValue;
  const bool grouped = p.scales != nullptr;

  auto launch = [&](auto kernel, auto scales_ptr) -> cudaError_t {
    cudaError_t e =
        set_max_smem(reinterpret_cast<const void*>(kernel), kSmemBytes);
    if (e != cudaSuccess) return e;
    int use_cluster = 0;
    if (p.split > 1) {
      if (p.split <= kMaxClusterSplit && !p.force_workspace && cluster_fits<NA>(kernel, p.split)) {
        use_cluster = 1;
      } else if (p.partials == nullptr || p.sems == nullptr) {
        *why = "this split-K launch needs a workspace (cluster reduction unavailable)";
        return cudaErrorInvalidValue;
      }
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(static_cast<unsigned>(p.N / kBN), static_cast<unsigned>(p.split), 1);
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = kSmemBytes;
    cfg.stream = s;
    cudaLaunchAttribute attrs[2];
    int na = 0;
    attrs[na].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attrs[na].val.programmaticStreamSerializationAllowed = 1;
    ++na;
    if (use_cluster) {
      attrs[na].id = cudaLaunchAttributeClusterDimension;
      attrs[na].val.clusterDim.x = 1;
      attrs[na].val.clusterDim.y = p.split;
      attrs[na].val.clusterDim.z = 1;
      ++na;
    }
    cfg.attrs = attrs;
    cfg.numAttrs = na;
    return cudaLaunchKernelEx(&cfg, kernel, tmA, tmW, scales_ptr, static_cast<int>(p.M),
                              static_cast<int>(p.N), static_cast<int>(p.K), p.split, use_cluster,
                              p.scalar_scale, p.out, p.out_dtype, p.ldo, p.partials, p.sems,
                              p.status, peers);
  };
  if (p.a_dtype == PK_BF16) {
    auto sp = static_cast<const __nv_bfloat16*>(p.scales);
    return grouped ? launch(w4a16_decode_kernel<__nv_bfloat16, true, NA>, sp)
                   : launch(w4a16_decode_kernel<__nv_bfloat16, false, NA>, sp);
  }
  auto sp = static_cast<const __half*>(p.scales);
  return grouped ? launch(w4a16_decode_kernel<__half, true, NA>, sp)
                 : launch(w4a16_decode_kernel<__half, false, NA>, sp);
}

}  // namespace

// M <= 16 on 16 activation columns, M <= 32 on 32 (the MMA's N). With a
// shard, the output goes to every rank's buffer and the grid ends with the
// flag barrier of the fused exchange.
cudaError_t launch_w4a16_decode(const DecodeArgs& p, cudaStream_t s, const char** why,
                                const OutputShard* shard) {
  OutputShard peers{};
  if (shard != nullptr) {
    if (shard->world < 1 || shard->world > kMaxPeers || shard->done == nullptr) {
      *why = "sharded decode: 1 <= world <= 8 and a workspace are required";
      return cudaErrorInvalidValue;
    }
    peers = *shard;
  }
  return p.M <= 16 ? launch_decode_na<16>(p, s, why, peers)
                   : launch_decode_na<32>(p, s, why, peers);
}

}  // namespace pk

namespace pk {
int decode_max_cluster_split() { return kMaxClusterSplit; }
}  // namespace pk
