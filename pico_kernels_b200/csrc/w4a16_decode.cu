// W4A16 GEMM for decode shapes (M <= 16) on sm_100a.
//
// out[M, N] = A[M, K] @ (q[K, N] * s[K/128, N])  (gemm_int4.py:75-92 with
// group scales; q unpacked from Wp[K, N/2] as in gemm_int4.py:43-50).
//
// Design (swap-AB): the weight tile is the MMA's M=128 operand (128 output
// columns n), the activations are its N=16 operand (M padded to 16 by TMA
// zero fill), so D[n, m] accumulates in 16 TMEM columns. One CTA owns 128
// columns and a contiguous range of 128-row K stages; stages are TMA-loaded
// into a ring of shared-memory slots (packed weights + activation tile +
// group scales), all issued up front when they fit. 256 threads dequantize
// each 64-row half stage in registers (int4 -> bf16/f16, times the group
// scale) into a 128B-swizzled MN-major tile; thread 0 then issues four
// tcgen05.mma (K=16 each). The K reduction is split over `split` CTAs per
// column tile: each writes its fp32 partial to the workspace, bumps the
// tile's arrival counter, and the last arriver sums all partials in split
// order (deterministic) and writes the output, then re-arms the counter.
#include "pk_common.cuh"

namespace pk {
namespace {

constexpr int kThreads = 256;
constexpr int kBN = 128;     // output columns per CTA (MMA M)
constexpr int kBK = 128;     // K rows per stage (one quantization group)
constexpr int kMmaN = 16;    // padded M (MMA N)
constexpr int kSlots = 4;    // TMA stage ring
constexpr int kDeqBufs = 3;  // dequantized 64-row half-stage ring

// shared memory layout (bytes from a 1024-aligned base)
constexpr int kAtileBytes = 2 * kMmaN * 128;        // two 64-col SW128 boxes: 4096
constexpr int kWBytes = kBK * (kBN / 2);            // 128 rows x 64 B: 8192
constexpr int kScaleBytes = kBN * 2;                // 256
constexpr int kSlotBytes = 13312;                   // A | W | scales, padded to 1 KB
constexpr int kSlotA = 0;
constexpr int kSlotW = kAtileBytes;
constexpr int kSlotS = kAtileBytes + kWBytes;
constexpr int kDeqBytes = kBN * 64 * 2;             // 16384 per half stage
constexpr int kDeqLBO = 8192;                       // between the two 64-column atoms
constexpr int kDeqOff = kSlots * kSlotBytes;
constexpr int kBarOff = kDeqOff + kDeqBufs * kDeqBytes;
constexpr int kSmemBytes = kBarOff + 256 + 1024;    // + barriers + alignment slack

static_assert(kSlotS + kScaleBytes <= kSlotBytes, "slot layout");

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

__device__ __forceinline__ void store_out(void* out, int out_dtype, int64_t idx, float v) {
  if (out_dtype == PK_BF16)
    static_cast<__nv_bfloat16*>(out)[idx] = __float2bfloat16_rn(v);
  else
    static_cast<float*>(out)[idx] = v;
}

template <typename T, bool kGrouped>
__global__ void __launch_bounds__(kThreads, 2)
    w4a16_decode_kernel(const __grid_constant__ CUtensorMap tmA,
                        const __grid_constant__ CUtensorMap tmW,
                        const __grid_constant__ CUtensorMap tmS, int M, int N, int K, int split,
                        float scalar_scale, void* __restrict__ out, int out_dtype, int64_t ldo,
                        float* __restrict__ partials, unsigned* __restrict__ sems,
                        int* __restrict__ status) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + kBarOff);
  uint64_t* mma_done = full + kSlots;
  uint64_t* final_bar = mma_done + kDeqBufs;
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(final_bar + 1);
  __shared__ int s_last;

  const int tid = threadIdx.x;
  const int warp = tid >> 5;
  const int lane = tid & 31;
  const int tile = blockIdx.x;
  const int ks = blockIdx.y;
  const int total_stages = K / kBK;
  const int g_begin = static_cast<int>((static_cast<int64_t>(ks) * total_stages) / split);
  const int g_end = static_cast<int>((static_cast<int64_t>(ks + 1) * total_stages) / split);
  const int S = g_end - g_begin;

  if (tid == 0) {
    for (int i = 0; i < kSlots; ++i) mbar_init(&full[i], 1);
    for (int i = 0; i < kDeqBufs; ++i) mbar_init(&mma_done[i], 1);
    mbar_init(final_bar, 1);
    fence_barrier_init();
  }
  if (warp == 0) tmem_alloc(tmem_holder, 32);
  if (tid == 32) {
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmW);
    if (kGrouped) tma_prefetch_desc(&tmS);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_holder;

  constexpr uint32_t kStageTx = kAtileBytes + kWBytes + (kGrouped ? kScaleBytes : 0);
  auto issue_stage = [&](int s) {
    const int slot = s % kSlots;
    uint8_t* base = smem + slot * kSlotBytes;
    const int g = g_begin + s;
    mbar_arrive_expect_tx(&full[slot], kStageTx);
    tma_load_2d(base + kSlotA, &tmA, &full[slot], g * kBK, 0);
    tma_load_2d(base + kSlotA + kMmaN * 128, &tmA, &full[slot], g * kBK + 64, 0);
    tma_load_2d(base + kSlotW, &tmW, &full[slot], tile * (kBN / 2), g * kBK);
    if (kGrouped) tma_load_2d(base + kSlotS, &tmS, &full[slot], tile * kBN, g);
  };

  int issued = 0;
  if (tid == 0) {
    const int pre = S < kSlots ? S : kSlots;
    for (int s = 0; s < pre; ++s) issue_stage(s);
    issued = pre;
  }

  constexpr uint32_t kIdesc = make_idesc(TypeFmt<T>::kFmt, true, false, 128, kMmaN);
  const uint32_t deq_base = smem_u32(smem + kDeqOff);
  const int w = tid & 15;          // 4-byte word within a 64-byte packed row: columns 8w..8w+7
  const int rsub = tid >> 4;       // 0..15
  const int atom = w >> 3, chunk = w & 7;

  bool fail = false;
  const int halves = 2 * S;
  for (int u = 0; u < halves; ++u) {
    const int s = u >> 1, h = u & 1;
    const int slot = s % kSlots;
    const int buf = u % kDeqBufs;
    uint8_t* base = smem + slot * kSlotBytes;
    if (!fail && h == 0)
      fail = !mbar_wait(&full[slot], (s / kSlots) & 1, status, kSiteDecodeFull);
    if (!fail && u >= kDeqBufs)
      fail = !mbar_wait(&mma_done[buf], ((u / kDeqBufs) - 1) & 1, status, kSiteDecodeMma);
    // the MMAs of half u-3 are done: if that finished a stage, refill its slot
    if (!fail && tid == 0 && u >= kDeqBufs && ((u - kDeqBufs) & 1) && issued < S) {
      issue_stage(issued);
      ++issued;
    }
    if (!fail) {
      uint32_t s01 = 0, s23 = 0, s45 = 0, s67 = 0;
      if (kGrouped) {
        const uint4 sv = *reinterpret_cast<const uint4*>(base + kSlotS + w * 16);
        s01 = sv.x; s23 = sv.y; s45 = sv.z; s67 = sv.w;
      }
      uint8_t* dq = smem + kDeqOff + buf * kDeqBytes;
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int r = rsub + 16 * i;  // row within the half stage, 0..63
        const uint32_t word =
            *reinterpret_cast<const uint32_t*>(base + kSlotW + (64 * h + r) * 64 + w * 4);
        uint32_t o[4];
        dequant8<T, kGrouped>(word, s01, s23, s45, s67, o);
        const int r8 = r & 7;
        const int off = atom * kDeqLBO + (r >> 3) * 1024 + r8 * 128 + ((chunk ^ r8) << 4);
        *reinterpret_cast<uint4*>(dq + off) = make_uint4(o[0], o[1], o[2], o[3]);
      }
      fence_proxy_async_smem();
    }
    fail = __syncthreads_or(fail) != 0;
    if (fail) break;
    if (tid == 0) {
      tc_fence_after();
      const uint32_t a_tile = smem_u32(base + kSlotA) + h * (kMmaN * 128);
      const uint32_t d_tile = deq_base + buf * kDeqBytes;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const uint64_t adesc = make_smem_desc(d_tile + j * 2048, kDeqLBO, 1024);
        const uint64_t bdesc = make_smem_desc(a_tile + j * 32, 16, 1024);
        umma_f16(tmem, adesc, bdesc, kIdesc, (u > 0 || j > 0) ? 1u : 0u);
      }
      umma_commit(&mma_done[buf]);
      if (u == halves - 1) umma_commit(final_bar);
    }
  }

  if (!fail) fail = !mbar_wait(final_bar, 0, status, kSiteDecodeFinal);
  fail = __syncthreads_or(fail) != 0;
  tc_fence_after();

  if (!fail && warp < 4) {
    uint32_t raw[16];
    tmem_ld_32x32b_x16(tmem + (static_cast<uint32_t>(warp * 32) << 16), raw);
    tmem_ld_wait();
    const int nl = warp * 32 + lane;
    const int64_t n = static_cast<int64_t>(tile) * kBN + nl;
    if (split == 1) {
#pragma unroll
      for (int m = 0; m < kMmaN; ++m)
        if (m < M) store_out(out, out_dtype, m * ldo + n, __uint_as_float(raw[m]) * scalar_scale);
    } else {
      float* mine = partials + (static_cast<int64_t>(tile) * split + ks) * M * kBN;
#pragma unroll
      for (int m = 0; m < kMmaN; ++m)
        if (m < M) __stcg(mine + m * kBN + nl, __uint_as_float(raw[m]));
      __threadfence();
      named_bar_sync(1, 128);
      if (tid == 0) s_last = (atomicAdd(&sems[tile], 1u) == static_cast<unsigned>(split - 1));
      named_bar_sync(1, 128);
      if (s_last) {
        __threadfence();
        const float* tile_parts = partials + static_cast<int64_t>(tile) * split * M * kBN;
#pragma unroll
        for (int m = 0; m < kMmaN; ++m) {
          if (m < M) {
            float acc = 0.0f;
            for (int j = 0; j < split; ++j) {
              const float v = (j == ks) ? __uint_as_float(raw[m])
                                        : __ldcg(tile_parts + (static_cast<int64_t>(j) * M + m) * kBN + nl);
              acc += v;
            }
            store_out(out, out_dtype, m * ldo + n, acc * scalar_scale);
          }
        }
        if (tid == 0) sems[tile] = 0u;  // re-arm for the next call
      }
    }
  }

  if (fail && tid == 0) {
    // let copies already issued land before the CTA's shared memory is released
    for (int s = 0; s < issued; ++s) mbar_wait(&full[s % kSlots], (s / kSlots) & 1, nullptr, 0);
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) tmem_dealloc(tmem, 32);
}

CUtensorMapDataType tmap_type(int dt) {
  return dt == PK_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
}

}  // namespace

bool decode_supported(int64_t M, int64_t N, int64_t K, int group, const void* scales,
                      int64_t lda, const void* a) {
  if (M < 1 || M > kMmaN) return false;
  if (N % kBN != 0 || K % kBK != 0) return false;
  if (scales != nullptr && group != kBK) return false;
  if (lda % 8 != 0 || (reinterpret_cast<uintptr_t>(a) & 15) != 0) return false;
  if (K > (1ll << 31) || N > (1ll << 31)) return false;
  return true;
}

int decode_pick_split(int64_t M, int64_t N, int64_t K) {
  (void)M;
  const int64_t tiles = N / kBN;
  const int64_t stages = K / kBK;
  const int64_t slots = 2ll * num_sms();  // two CTAs per SM
  int64_t split = slots / (tiles > 0 ? tiles : 1);
  if (split < 1) split = 1;
  if (split > stages) split = stages;
  if (split > 32) split = 32;
  return static_cast<int>(split);
}

size_t decode_workspace_bytes(int64_t M, int64_t N, int64_t K, int split) {
  (void)K;
  if (split <= 1) return 0;
  const int64_t tiles = N / kBN;
  const size_t sem_bytes = ((tiles * sizeof(unsigned) + 255) / 256) * 256;
  return sem_bytes + static_cast<size_t>(tiles) * split * M * kBN * sizeof(float);
}

cudaError_t launch_w4a16_decode(const DecodeArgs& p, cudaStream_t s, const char** why) {
  CUtensorMap tmA, tmW, tmS;
  const CUtensorMapDataType dt = tmap_type(p.a_dtype);
  if (!encode_tmap_2d(&tmA, dt, p.a, p.K, p.M, p.lda * 2, 64, kMmaN,
                      CU_TENSOR_MAP_SWIZZLE_128B, why))
    return cudaErrorInvalidValue;
  if (!encode_tmap_2d(&tmW, CU_TENSOR_MAP_DATA_TYPE_UINT8, p.wp, p.N / 2, p.K, p.N / 2, kBN / 2,
                      kBK, CU_TENSOR_MAP_SWIZZLE_NONE, why))
    return cudaErrorInvalidValue;
  const bool grouped = p.scales != nullptr;
  if (grouped) {
    if (!encode_tmap_2d(&tmS, dt, p.scales, p.N, p.K / kBK, p.N * 2, kBN, 1,
                        CU_TENSOR_MAP_SWIZZLE_NONE, why))
      return cudaErrorInvalidValue;
  } else {
    tmS = tmW;  // unused
  }
  dim3 grid(static_cast<unsigned>(p.N / kBN), static_cast<unsigned>(p.split));
  auto launch = [&](auto kernel) -> cudaError_t {
    cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         kSmemBytes);
    if (e != cudaSuccess) return e;
    kernel<<<grid, kThreads, kSmemBytes, s>>>(tmA, tmW, tmS, static_cast<int>(p.M),
                                              static_cast<int>(p.N), static_cast<int>(p.K),
                                              p.split, p.scalar_scale, p.out, p.out_dtype, p.ldo,
                                              p.partials, p.sems, p.status);
    return cudaGetLastError();
  };
  if (p.a_dtype == PK_BF16)
    return grouped ? launch(w4a16_decode_kernel<__nv_bfloat16, true>)
                   : launch(w4a16_decode_kernel<__nv_bfloat16, false>);
  return grouped ? launch(w4a16_decode_kernel<__half, true>)
                 : launch(w4a16_decode_kernel<__half, false>);
}

}  // namespace pk
