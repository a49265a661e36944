// W4A16 GEMM for 32 < M <= 256 on sm_100a ("skinny" prefill, swap-AB).
//
// out[M, N] = A[M, K] @ (q[K, N] * s[K/g, N])  -- gemm_int4.int4_gemm
// (gemm_int4.py:75-92). Between the decode shapes (M <= 32, the exact-code
// decode kernel) and large M (the tcgen05 prefill kernel with 128-row A
// tiles), the weights dominate: a 128 x 256 prefill tile dequantizes each
// weight tile once per 128-row M tile and keeps one CTA per SM. Here the
// roles swap: the dequantized weight tile is the MMA's M = 128 operand
// (128 output columns), the activations its N = NA operand (NA = 64, 128 or
// 256, M padded by TMA zero fill), so every weight is dequantized exactly
// once, and two CTAs share an SM.
//
// Per CTA: 128 output columns x all of K, in 64-row stages. Warp roles:
//   warps 0-3  epilogue: read D[n, 0..NA) from TMEM once at the end, store
//              out[m, n] (a warp's 32 lanes are 32 consecutive n: coalesced);
//   warp 4     TMA producer: activation tile A[0:NA, k0:k0+64] (128B swizzle),
//              the stage's packed weights and its row of group scales;
//   warp 5     TMEM allocator and MMA issuer (one thread);
//   warps 6-13 dequant: q * s rounded to A's dtype by dequant8 (the prefill
//              path's operand values), written as a 128B-swizzled MN-major
//              tile; per-tensor scales leave the exact codes and multiply in
//              the epilogue.
// One fp32 accumulator of NA TMEM columns for the whole K walk. All hand-offs
// are mbarriers with bounded waits.
#include "pk_common.cuh"

namespace pk {
namespace {

constexpr int kEpiWarps = 4;
constexpr int kTmaWarp = 4;
constexpr int kMmaWarp = 5;
constexpr int kDeqWarp0 = 6;
constexpr int kDeqWarps = 8;
constexpr int kThreads = (kDeqWarp0 + kDeqWarps) * 32;  // 448

constexpr int kBN = 128;                    // output columns per CTA (MMA M)
constexpr int kBK = 64;                     // K rows per stage
constexpr int kWBytes = kBK * (kBN / 2);    // 4096 packed
constexpr int kSBytes = kBN * 2;            // one row of 128 16-bit scales
constexpr int kDeqBytes = kBN * kBK * 2;    // 16384
constexpr int kDeqLBO = kBK * 128;          // 8192: between the two 64-column atoms

template <int NA>
struct SkCfg {
  static constexpr int kAtile = NA * 128;   // NA rows x 64 K: one 128-byte swizzle row each
  static constexpr int kSlotBytes = ((kAtile + kWBytes + kSBytes + 1023) / 1024) * 1024;
  static constexpr int kSlots = NA == 256 ? 2 : (NA == 128 ? 3 : 4);
  static constexpr int kDeqBufs = 2;        // ring of dequantized stages
  static constexpr int kDeqOff = kSlots * kSlotBytes;
  static constexpr int kBarOff = kDeqOff + kDeqBufs * kDeqBytes;
  static constexpr int kNumBars = 2 * kSlots + 2 * kDeqBufs + 1;
  static constexpr int kSmemBytes = kBarOff + kNumBars * 8 + 16 + 1024;
  static constexpr int kTmemCols = NA;
  static_assert(kSmemBytes <= 113 * 1024, "two CTAs per SM");
  static_assert(2 * kTmemCols <= 512, "two CTAs' TMEM fits an SM");
};

template <typename T>
struct SkFmt;
template <>
struct SkFmt<__nv_bfloat16> {
  static constexpr uint32_t kFmt = 1;
};
template <>
struct SkFmt<__half> {
  static constexpr uint32_t kFmt = 0;
};

template <typename T, bool kGrouped, int NA>
__global__ void __launch_bounds__(kThreads, 2)
    w4a16_skinny_kernel(const __grid_constant__ CUtensorMap tmA,
                        const __grid_constant__ CUtensorMap tmW,
                        const __grid_constant__ CUtensorMap tmS, int M, int K, int group,
                        float scalar_scale, void* __restrict__ out, int out_dtype, int64_t ldo,
                        int* __restrict__ status, const __grid_constant__ OutputShard peers) {
  using C = SkCfg<NA>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + C::kBarOff);
  uint64_t* slot_empty = full + C::kSlots;
  uint64_t* deq_full = slot_empty + C::kSlots;
  uint64_t* deq_empty = deq_full + C::kDeqBufs;
  uint64_t* acc_full = deq_empty + C::kDeqBufs;
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(acc_full + 1);

  const int tid = threadIdx.x;
  const int warp = tid >> 5;
  const int lane = tid & 31;
  const int tile = blockIdx.x;
  const int S = K / kBK;

  if (warp == kTmaWarp && lane == 0) {
    for (int i = 0; i < C::kSlots; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&slot_empty[i], 1);
    }
    for (int i = 0; i < C::kDeqBufs; ++i) {
      mbar_init(&deq_full[i], kDeqWarps);
      mbar_init(&deq_empty[i], 1);
    }
    mbar_init(acc_full, 1);
    fence_barrier_init();
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmW);
    if (kGrouped) tma_prefetch_desc(&tmS);
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
      constexpr uint32_t tx = C::kAtile + kWBytes + (kGrouped ? kSBytes : 0);
      for (int s = 0; s < S && !fail; ++s) {
        const int slot = s % C::kSlots;
        if (s >= C::kSlots)
          fail = !mbar_wait(&slot_empty[slot], ((s / C::kSlots) - 1) & 1, status, kSiteSkinnyFull);
        if (fail) break;
        uint8_t* base = smem + slot * C::kSlotBytes;
        const int k0 = s * kBK;
        mbar_arrive_expect_tx(&full[slot], tx);
        tma_load_2d(base, &tmA, &full[slot], k0, 0);
        tma_load_2d(base + C::kAtile, &tmW, &full[slot], tile * (kBN / 2), k0);
        if (kGrouped)
          tma_load_2d(base + C::kAtile + kWBytes, &tmS, &full[slot], tile * kBN, k0 / group);
        issued = s + 1;
      }
    }
  } else if (warp == kMmaWarp) {
    // ---------------- MMA issuer ----------------
    if (lane == 0) {
      constexpr uint32_t kIdesc = make_idesc(SkFmt<T>::kFmt, true, false, 128, NA);
      const uint32_t deq_base = smem_u32(smem + C::kDeqOff);
      for (int s = 0; s < S && !fail; ++s) {
        const int slot = s % C::kSlots;
        const int buf = s % C::kDeqBufs;
        fail = !mbar_wait(&deq_full[buf], (s / C::kDeqBufs) & 1, status, kSiteSkinnyMma);
        if (fail) break;
        tc_fence_after();
        const uint32_t a_tile = smem_u32(smem + slot * C::kSlotBytes);
        const uint32_t d_tile = deq_base + buf * kDeqBytes;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const uint64_t adesc = make_smem_desc(d_tile + j * 2048, kDeqLBO, 1024);
          const uint64_t bdesc = make_smem_desc(a_tile + j * 32, 16, 1024);
          umma_f16(tmem, adesc, bdesc, kIdesc, (s | j) != 0 ? 1u : 0u);
        }
        umma_commit(&deq_empty[buf]);
        umma_commit(&slot_empty[slot]);
      }
      if (!fail) umma_commit(acc_full);
    }
  } else if (warp >= kDeqWarp0) {
    // ---------------- dequant ----------------
    // The decode kernel's conflict-free mapping of 64 packed rows of 64 bytes
    // onto 256 threads: quarter k of warp w covers rows 8w + 4(k/2) .. +3;
    // lane t takes quad q = t % 4 (columns 32q .. 32q + 31) of row
    // 8w + 4(k/2) + 2((q/2) ^ (k%2)) + t/4.
    const int dt = tid - kDeqWarp0 * 32;
    const int qk = lane >> 3, qt = lane & 7;
    const int wq = qt & 3;
    const int r = 8 * (dt >> 5) + 4 * (qk >> 1) + 2 * ((wq >> 1) ^ (qk & 1)) + (qt >> 2);
    const int r8 = r & 7;
    const uint32_t row_off = (r >> 3) * 1024 + r8 * 128;
    for (int s = 0; s < S && !fail; ++s) {
      const int slot = s % C::kSlots;
      const int buf = s % C::kDeqBufs;
      fail = !mbar_wait(&full[slot], (s / C::kSlots) & 1, status, kSiteSkinnyFull);
      if (!fail && s >= C::kDeqBufs)
        fail = !mbar_wait(&deq_empty[buf], ((s / C::kDeqBufs) - 1) & 1, status, kSiteSkinnyMma);
      if (fail) break;
      const uint8_t* base = smem + slot * C::kSlotBytes;
      const uint4 wv = *reinterpret_cast<const uint4*>(base + C::kAtile + r * 64 + wq * 16);
      const uint32_t words[4] = {wv.x, wv.y, wv.z, wv.w};
      uint8_t* dq = smem + C::kDeqOff + buf * kDeqBytes + row_off;
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int c = 4 * wq + i;  // 8-column chunk 0..15
        uint4 sv = make_uint4(0u, 0u, 0u, 0u);
        if (kGrouped)
          sv = *reinterpret_cast<const uint4*>(base + C::kAtile + kWBytes + c * 16);
        uint32_t o[4];
        dequant8<T, kGrouped>(words[i], sv.x, sv.y, sv.z, sv.w, o);
        *reinterpret_cast<uint4*>(dq + (c >> 3) * kDeqLBO + (((c & 7) ^ r8) << 4)) =
            make_uint4(o[0], o[1], o[2], o[3]);
      }
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) mbar_arrive(&deq_full[buf]);
    }
  }

  // ---------------- epilogue: D[n, m] -> out[m, n] ----------------
  bool stored = false;  // this thread wrote output (sharded exchange: fence before arriving)
  if (warp < kEpiWarps && !fail && S > 0) {
    fail = !mbar_wait(acc_full, 0, status, kSiteSkinnyFinal);
    if (!fail) {
      tc_fence_after();
      const uint32_t lane_base = tmem + (static_cast<uint32_t>(warp * 32) << 16);
      const int64_t n = static_cast<int64_t>(tile) * kBN + tid;
      const float sc = kGrouped ? 1.0f : scalar_scale;
#pragma unroll 1
      for (int c = 0; c < NA / 32; ++c) {
        if (c * 32 >= M) break;
        uint32_t raw[32];
        tmem_ld_32x32b_x32(lane_base + c * 32, raw);
        tmem_ld_wait();
#pragma unroll
        for (int i = 0; i < 32; ++i) {
          const int m = c * 32 + i;
          if (m < M) emit_out(out, peers, out_dtype, m * ldo + n, __uint_as_float(raw[i]) * sc);
        }
      }
      stored = true;
    }
  }

  if (fail && warp == kTmaWarp && lane == 0) {
    // let copies already issued land before the CTA's shared memory is released
    const int first = issued > C::kSlots ? issued - C::kSlots : 0;
    for (int s = first; s < issued; ++s)
      mbar_wait(&full[s % C::kSlots], (s / C::kSlots) & 1, nullptr, 0);
  }
  tc_fence_before();
  __syncthreads();
  if (warp == kMmaWarp) tmem_dealloc(tmem, C::kTmemCols);
  if (peers.world > 1)
    peer_exchange_finish(peers, stored, status, kSiteSkinnyPeers, gridDim.x * gridDim.y);
}

CUtensorMapDataType sk_tmap_type(int dt) {
  return dt == PK_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
}

template <int NA>
cudaError_t launch_skinny_na(const DecodeArgs& p, cudaStream_t s, const char** why,
                             const OutputShard& peers) {
  constexpr int kSmem = SkCfg<NA>::kSmemBytes;
  CUtensorMap tmA, tmW, tmS;
  const CUtensorMapDataType dt = sk_tmap_type(p.a_dtype);
  if (!encode_tmap_2d(&tmA, dt, p.a, p.K, p.M, p.lda * 2, 64, NA, CU_TENSOR_MAP_SWIZZLE_128B, why))
    return cudaErrorInvalidValue;
  if (!encode_tmap_2d(&tmW, CU_TENSOR_MAP_DATA_TYPE_UINT8, p.wp, p.N / 2, p.K, p.N / 2, kBN / 2,
                      kBK, CU_TENSOR_MAP_SWIZZLE_NONE, why))
    return cudaErrorInvalidValue;
  const bool grouped = p.scales != nullptr;
  if (grouped) {
    const int64_t G = (p.K + p.group - 1) / p.group;
    if (!encode_tmap_2d(&tmS, dt, p.scales, p.N, G, p.N * 2, kBN, 1, CU_TENSOR_MAP_SWIZZLE_NONE,
                        why))
      return cudaErrorInvalidValue;
  } else {
    tmS = tmW;  // unused
  }
  auto launch = [&](auto kernel) -> cudaError_t {
    cudaError_t e = set_max_smem(reinterpret_cast<const void*>(kernel), kSmem);
    if (e != cudaSuccess) return e;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(static_cast<unsigned>(p.N / kBN), 1, 1);
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = kSmem;
    cfg.stream = s;
    cudaLaunchAttribute attr;
    attr.id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr.val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = &attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kernel, tmA, tmW, tmS, static_cast<int>(p.M),
                              static_cast<int>(p.K), p.group > 0 ? p.group : kBK, p.scalar_scale,
                              p.out, p.out_dtype, p.ldo, p.status, peers);
  };
  if (p.a_dtype == PK_BF16)
    return grouped ? launch(w4a16_skinny_kernel<__nv_bfloat16, true, NA>)
                   : launch(w4a16_skinny_kernel<__nv_bfloat16, false, NA>);
  return grouped ? launch(w4a16_skinny_kernel<__half, true, NA>)
                 : launch(w4a16_skinny_kernel<__half, false, NA>);
}

}  // namespace

bool skinny_supported(int64_t M, int64_t N, int64_t K, int group, const void* scales,
                      int64_t lda, const void* a) {
  if (M <= 32 || M > 256) return false;
  if (N % kBN != 0 || K % kBK != 0) return false;
  if (scales != nullptr && (group % kBK) != 0) return false;
  if (scales != nullptr && (reinterpret_cast<uintptr_t>(scales) & 15) != 0) return false;
  if (lda % 8 != 0 || (reinterpret_cast<uintptr_t>(a) & 15) != 0) return false;
  if (K > (1ll << 30) || N > (1ll << 30)) return false;
  return true;
}

// Whether this kernel beats the fused prefill kernel on an M x N x K call,
// by a model of both built from measured per-stage times on B200 (us per
// 64-row K stage of one CTA; Llama-70B up/down_proj and 4096-wide layers,
// CUDA graphs of back-to-back calls):
//   this kernel, NA = 64 / 128 / 256: 0.46 / 0.55 / 0.88 alone on an SM,
//                                     0.79 / 0.88 / 1.25 with two CTAs per SM;
//   prefill (128 x 256 tiles, one CTA per SM): 0.75 per tile, whatever M <= 128.
// The prefill's wider tiles are cheaper per column once they fill the SMs;
// this kernel wins where the prefill would leave SMs idle or dequantize a
// weight tile once per 128-row M tile (M > 128).
bool skinny_preferred(int64_t M, int64_t N, int64_t K) {
  const int na = M <= 64 ? 0 : (M <= 128 ? 1 : 2);
  const double t1[3] = {0.46, 0.55, 0.88}, t2[3] = {0.79, 0.88, 1.25};
  const int64_t sms = num_sms();
  const double stages = static_cast<double>(K / kBK);
  const int64_t tiles = N / kBN;
  double sk;
  if (tiles <= sms)
    sk = stages * t1[na];
  else
    sk = stages * t2[na] * static_cast<double>((tiles + 2 * sms - 1) / (2 * sms));
  const int64_t pf_tiles = ((M + 127) / 128) * ((N + 255) / 256);
  const double pf = stages * 0.75 * static_cast<double>((pf_tiles + sms - 1) / sms);
  return sk < 0.95 * pf;
}

// With a shard, the output goes to every rank's buffer and the grid ends
// with the flag barrier of the fused exchange.
cudaError_t launch_w4a16_skinny(const DecodeArgs& p, cudaStream_t s, const char** why,
                                const OutputShard* shard) {
  OutputShard peers{};
  if (shard != nullptr) {
    if (shard->world < 1 || shard->world > kMaxPeers || shard->done == nullptr) {
      *why = "sharded skinny GEMM: 1 <= world <= 8 and a workspace are required";
      return cudaErrorInvalidValue;
    }
    peers = *shard;
  }
  if (p.M <= 64) return launch_skinny_na<64>(p, s, why, peers);
  if (p.M <= 128) return launch_skinny_na<128>(p, s, why, peers);
  return launch_skinny_na<256>(p, s, why, peers);
}

}  // namespace pk
