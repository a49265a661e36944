// Persistent tcgen05 GEMM for sm_100a: C[M, N] = A[M, K] @ B[K, N].
//
// One CTA per SM walks output tiles (grouped raster for L2 reuse). Operands
// are staged by TMA into 128B-swizzled shared-memory tiles: A K-major
// (row-major [M, K]), B MN-major (row-major [K, N], read by the tensor core
// through the descriptor's MN-major mode, so no transpose pass). fp32
// accumulators live in TMEM, double-buffered so the epilogue of one tile
// overlaps the main loop of the next.
//
// Used by three entry points:
//   * fp8 (e4m3 x e4m3, kind::f8f6f4, K = 32 per MMA), epilogue x out_scale
//     -- gemm_fp8.fp8_gemm_kernel (gemm_fp8.py:38-86);
//   * dense fp16/bf16 (kind::f16), optional deterministic split-K --
//     gemm_splitk.gemm_splitk_kernel (gemm_splitk.py:26-64);
//     both on 256 x 256 tiles computed by a CTA pair (gemm_pair_kernel,
//     cta_group::2) when the tiles make more than one wave, else (and for
//     split-K) on one-CTA 128 x 256 tiles;
//   * W4A16 prefill: 128 x 256 tiles; B is produced in shared memory by
//     dequant warps from the packed int4 weights and group scales (q * s
//     rounded to A's dtype) -- gemm_int4.int4_gemm_kernel (gemm_int4.py:21-55).
//     (256 x 128 tiles, two M = 128 MMAs per dequantized B tile, halve the
//     dequant work but re-read B from shared memory twice and measured slower.)
//
// Warp roles: 0 TMA producer, 1 MMA issuer (+ TMEM owner), 2-5 epilogue
// (TMEM lanes 0-127), 6-13 dequant (int4 only).
#include "pk_common.cuh"

namespace pk {
namespace {

constexpr int kTmaWarp = 0, kMmaWarp = 1, kEpiWarp0 = 2, kEpiWarps = 4, kDeqWarp0 = 6;
constexpr int kDeqWarps = 8;
constexpr int kGroupM = 8;

enum Kind { kF16 = 0, kF8 = 1 };

template <int kKind, bool kInt4>
struct Cfg {
  static constexpr int kElem = kKind == kF16 ? 2 : 1;       // bytes per A/B element
  static constexpr int kBK = 128 / kElem;                    // one 128-byte swizzle row of K
  static constexpr int kMmaK = kKind == kF16 ? 16 : 32;
  static constexpr int kKSteps = kBK / kMmaK;                // 4
  // W4A16 tiles: kInt4Wide = 128 x 256 (one MMA per k-step reads each B slice
  // once); otherwise 256 x 128 (two M = 128 MMAs share each dequantized B
  // tile, halving dequant per FLOP but re-reading B from shared memory).
  static constexpr bool kInt4Wide = true;
  static constexpr int kMSub = (kInt4 && !kInt4Wide) ? 2 : 1;  // M = 128 MMAs per k-step
  static constexpr int kBM = 128 * kMSub;                    // CTA tile rows
  static constexpr int kBN = (kInt4 && !kInt4Wide) ? 128 : 256;  // CTA tile columns (= MMA N)
  static constexpr int kATile = kBM * 128;                   // 16 / 32 KB
  static constexpr int kBTile = kBK * kBN * kElem;           // 32 / 16 KB
  static constexpr int kBAtomN = 128 / kElem;                // N per MN-major swizzle atom
  static constexpr int kBBoxes = kBN / kBAtomN;              // TMA boxes per B tile
  static constexpr int kBLBO = kBK * 128;                    // bytes between N atoms
  static constexpr int kBStepBytes = (kMmaK / 8) * 1024;     // B advance per MMA K step
  // int4: packed weights (kBK rows x kBN/2 bytes) + kBN group scales per stage
  static constexpr int kWTile = kInt4 ? kBK * (kBN / 2) : 0;  // 8 / 4 KB
  static constexpr int kSRows = kBN / 64;                     // scale rows of 64 (128 B)
  static constexpr int kSTile = kInt4 ? kBN * 2 : 0;          // 512 / 256 B
  static constexpr int kStages = kInt4 ? 6 : 4;        // int4: 6 x 25 KB (+2-4 % over 4)
  static constexpr int kBBufs = kInt4 ? 2 : 0;                // dequantized B ring
  static constexpr int kStageBytes = kATile + (kInt4 ? kWTile + 1024 : kBTile);
  static constexpr int kStageOff = 0;
  static constexpr int kBBufOff = kStages * kStageBytes;
  static constexpr int kBarOff = kBBufOff + kBBufs * kBTile;
  static constexpr int kSmem = kBarOff + 256 + 1024;
  static constexpr int kThreads = (kInt4 ? kDeqWarp0 + kDeqWarps : kDeqWarp0) * 32;
  static constexpr int kAccCols = kMSub * kBN;                // TMEM columns per accumulator set
  static constexpr uint32_t kIdesc =
      make_idesc(kKind == kF16 ? 1u : 0u, false, true, 128, kBN);  // bf16 / e4m3
  static constexpr uint32_t kIdescF16 = make_idesc(0u, false, true, 128, kBN);
  static_assert(2 * kAccCols <= 512, "two accumulator sets fit TMEM");
  static_assert(kSmem <= 227 * 1024, "shared memory");
};

struct Params {
  int M, N, K;
  int split;             // K splits (dense split-K); 1 otherwise
  int num_m, num_n;      // tiles
  int out_dtype;         // PK_F32 / PK_BF16
  int64_t ldc;
  float out_scale;
  void* out;
  float* partials;       // split-K workspace
  unsigned* sems;
  int group;             // int4 group size
  int grouped;           // int4: 1 = group scales in the dequant, 0 = scalar out_scale
  int a_is_f16;          // 16-bit kinds: A dtype is fp16 (else bf16)
  int* status;
  const float* scale_a;  // fp8 with device scales: out_scale = 1 / (*scale_a * *scale_b)
  const float* scale_b;
  int whole;             // pair kernel: units that are whole tiles; each later tile is two
                         // units of half its columns (the last wave's tail), 16-bit kinds
  OutputShard peers;     // one-CTA kernel without split-K: world > 0 stores every output
                         // into all ranks' buffers and ends with the flag barrier
};

// The epilogue multiplier: the host's out_scale, or, for scales that live on
// the device (written by the previous kernel; read after griddepcontrol.wait),
// 1 / (scale_a * scale_b) formed in double as the reference forms it on the
// host (gemm_fp8.py:106) and rounded once to fp32.
__device__ __forceinline__ float epilogue_scale(const Params& p) {
  if (p.scale_a == nullptr) return p.out_scale;
  return static_cast<float>(1.0 / (static_cast<double>(*p.scale_a) * static_cast<double>(*p.scale_b)));
}

__device__ __forceinline__ void tile_coords(int t, const Params& p, int& tm, int& tn, int& ks) {
  ks = t % p.split;
  t /= p.split;
  const int per_group = kGroupM * p.num_n;
  const int g = t / per_group;
  const int first_m = g * kGroupM;
  const int gm = min(p.num_m - first_m, kGroupM);
  tm = first_m + (t % per_group) % gm;
  tn = (t % per_group) / gm;
}

__device__ __forceinline__ void store8(void* out, int out_dtype, int64_t idx, const float* v,
                                       bool full, int valid) {
  if (out_dtype == PK_BF16) {
    __nv_bfloat16* o = static_cast<__nv_bfloat16*>(out) + idx;
    if (full && (reinterpret_cast<uintptr_t>(o) & 15) == 0) {
      uint4 u;
      __nv_bfloat162 t0 = __floats2bfloat162_rn(v[0], v[1]);
      __nv_bfloat162 t1 = __floats2bfloat162_rn(v[2], v[3]);
      __nv_bfloat162 t2 = __floats2bfloat162_rn(v[4], v[5]);
      __nv_bfloat162 t3 = __floats2bfloat162_rn(v[6], v[7]);
      u.x = *reinterpret_cast<uint32_t*>(&t0);
      u.y = *reinterpret_cast<uint32_t*>(&t1);
      u.z = *reinterpret_cast<uint32_t*>(&t2);
      u.w = *reinterpret_cast<uint32_t*>(&t3);
      *reinterpret_cast<uint4*>(o) = u;
    } else {
      for (int i = 0; i < valid; ++i) o[i] = __float2bfloat16_rn(v[i]);
    }
  } else {
    float* o = static_cast<float*>(out) + idx;
    if (full && (reinterpret_cast<uintptr_t>(o) & 15) == 0) {
      reinterpret_cast<float4*>(o)[0] = make_float4(v[0], v[1], v[2], v[3]);
      reinterpret_cast<float4*>(o)[1] = make_float4(v[4], v[5], v[6], v[7]);
    } else {
      for (int i = 0; i < valid; ++i) o[i] = v[i];
    }
  }
}

// Sum `parts` fp32 partial rows of kBN columns (`stride` floats apart) in part
// order starting from zero, scale, and store the valid columns of output row
// `out_row`. 64 columns at a time, with all 16 loads of a part in flight: a
// loop of one 8-column load per step would pay an L2 round trip per step.
template <int kBN>
__device__ __forceinline__ void sum_parts_row(const float* base, int64_t stride, int parts,
                                              float scale, void* out, int out_dtype,
                                              int64_t out_row, int col0, int N) {
#pragma unroll 1
  for (int c0 = 0; c0 < kBN; c0 += 64) {
    if (col0 + c0 >= N) break;
    float v[64];
#pragma unroll
    for (int i = 0; i < 64; ++i) v[i] = 0.0f;
#pragma unroll 1
    for (int j = 0; j < parts; ++j) {
      const float4* src = reinterpret_cast<const float4*>(base + j * stride + c0);
      float4 x[16];
#pragma unroll
      for (int i = 0; i < 16; ++i) x[i] = __ldcg(src + i);
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        v[4 * i] += x[i].x;
        v[4 * i + 1] += x[i].y;
        v[4 * i + 2] += x[i].z;
        v[4 * i + 3] += x[i].w;
      }
    }
#pragma unroll
    for (int i = 0; i < 64; i += 8) {
      float w[8];
#pragma unroll
      for (int e = 0; e < 8; ++e) w[e] = v[i + e] * scale;
      const int col = col0 + c0 + i;
      if (col < N) store8(out, out_dtype, out_row + col, w, col + 8 <= N, min(8, N - col));
    }
  }
}

template <int kKind, bool kInt4>
__global__ void __launch_bounds__(Cfg<kKind, kInt4>::kThreads, 1)
    gemm_tc_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                   const __grid_constant__ CUtensorMap tmS, const Params p) {
  using C = Cfg<kKind, kInt4>;
  constexpr int BM = C::kBM, BN = C::kBN;
  constexpr int kBBufs = C::kBBufs > 0 ? C::kBBufs : 1;  // divisor for the int4-only paths
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + C::kBarOff);
  uint64_t* empty = full + C::kStages;
  uint64_t* acc_full = empty + C::kStages;
  uint64_t* acc_empty = acc_full + 2;
  uint64_t* bfull = acc_empty + 2;
  uint64_t* bempty = bfull + 2;
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(bempty + 2);
  int* s_flag = reinterpret_cast<int*>(tmem_holder + 1);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int k_tiles_total = (p.K + C::kBK - 1) / C::kBK;
  const int num_units = p.num_m * p.num_n * p.split;
  bool stored = false;  // this thread wrote output (sharded exchange: fence before arriving)

  if (warp == kTmaWarp && lane == 0) {
    for (int i = 0; i < C::kStages; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], kInt4 ? 1 + kDeqWarps : 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&acc_full[i], 1);
      mbar_init(&acc_empty[i], kEpiWarps);
      mbar_init(&bfull[i], kDeqWarps);
      mbar_init(&bempty[i], 1);
    }
    fence_barrier_init();
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
    if (kInt4) tma_prefetch_desc(&tmS);
  }
  if (warp == kMmaWarp) tmem_alloc(tmem_holder, 512);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_holder;
  griddep_wait();

  bool fail = false;
  if (warp == kTmaWarp) {
    // ------------------------------- producer -------------------------------
    if (lane == 0) {
      int it = 0;
      for (int u = blockIdx.x; u < num_units && !fail; u += gridDim.x) {
        int tm, tn, ks;
        tile_coords(u, p, tm, tn, ks);
        const int kt0 = (ks * k_tiles_total) / p.split, kt1 = ((ks + 1) * k_tiles_total) / p.split;
        for (int kt = kt0; kt < kt1 && !fail; ++kt, ++it) {
          const int st = it % C::kStages;
          if (it >= C::kStages)
            fail = !mbar_wait(&empty[st], ((it / C::kStages) - 1) & 1, p.status, kSiteGemmProducer);
          if (fail) break;
          uint8_t* base = smem + C::kStageOff + st * C::kStageBytes;
          const int k0 = kt * C::kBK;
          if (kInt4) {
            mbar_arrive_expect_tx(&full[st], C::kATile + C::kWTile + (p.grouped ? C::kSTile : 0));
            tma_load_2d(base, &tmA, &full[st], k0, tm * BM);
            tma_load_2d(base + C::kATile, &tmB, &full[st], tn * (BN / 2), k0);
            if (p.grouped)
              tma_load_2d(base + C::kATile + C::kWTile, &tmS, &full[st], 0,
                          (k0 / p.group) * (p.N / 64) + tn * C::kSRows);
          } else {
            mbar_arrive_expect_tx(&full[st], C::kATile + C::kBTile);
            tma_load_2d(base, &tmA, &full[st], k0, tm * BM);
#pragma unroll
            for (int b = 0; b < C::kBBoxes; ++b)
              tma_load_2d(base + C::kATile + b * C::kBLBO, &tmB, &full[st],
                          tn * BN + b * C::kBAtomN, k0);
          }
        }
      }
    }
  } else if (warp == kMmaWarp) {
    // ------------------------------ MMA issuer ------------------------------
    if (lane == 0) {
      int it = 0, bit = 0, local = 0;
      for (int u = blockIdx.x; u < num_units && !fail; u += gridDim.x, ++local) {
        int tm, tn, ks;
        tile_coords(u, p, tm, tn, ks);
        const int kt0 = (ks * k_tiles_total) / p.split, kt1 = ((ks + 1) * k_tiles_total) / p.split;
        const int ab = local & 1;
        if (local >= 2)
          fail = !mbar_wait(&acc_empty[ab], ((local >> 1) - 1) & 1, p.status, kSiteGemmMma);
        if (fail) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem + ab * C::kAccCols;
        for (int kt = kt0; kt < kt1 && !fail; ++kt, ++it) {
          const int st = it % C::kStages;
          fail = !mbar_wait(&full[st], (it / C::kStages) & 1, p.status, kSiteGemmMma);
          int bb = 0;
          if (kInt4 && !fail) {
            bb = bit % kBBufs;
            fail = !mbar_wait(&bfull[bb], (bit / kBBufs) & 1, p.status, kSiteGemmMma);
          }
          if (fail) break;
          tc_fence_after();
          const uint32_t a_base = smem_u32(smem + C::kStageOff + st * C::kStageBytes);
          const uint32_t b_base = kInt4 ? smem_u32(smem + C::kBBufOff + bb * C::kBTile)
                                        : a_base + C::kATile;
#pragma unroll
          for (int j = 0; j < C::kKSteps; ++j) {
            const uint64_t bd = make_smem_desc(b_base + j * C::kBStepBytes, C::kBLBO, 1024);
            const uint32_t acc = (kt > kt0 || j > 0) ? 1u : 0u;
#pragma unroll
            for (int h = 0; h < C::kMSub; ++h) {
              const uint64_t ad = make_smem_desc(a_base + h * 16384 + j * 32, 16, 1024);
              const uint32_t d = d_tmem + h * BN;
              if (kKind == kF8)
                umma_f8(d, ad, bd, C::kIdesc, acc);
              else if (p.a_is_f16)
                umma_f16(d, ad, bd, C::kIdescF16, acc);
              else
                umma_f16(d, ad, bd, C::kIdesc, acc);
            }
          }
          umma_commit(&empty[st]);
          if (kInt4) {
            umma_commit(&bempty[bb]);
            ++bit;
          }
        }
        if (fail) break;
        umma_commit(&acc_full[ab]);
      }
    }
  } else if (warp >= kEpiWarp0 && warp < kEpiWarp0 + kEpiWarps) {
    // ------------------------------- epilogue -------------------------------
    const int q = warp & 3;  // TMEM lane quarter this warp may access
    const int row_in_sub = q * 32 + lane;
    const float out_scale = epilogue_scale(p);
    int local = 0;
    for (int u = blockIdx.x; u < num_units && !fail; u += gridDim.x, ++local) {
      int tm, tn, ks;
      tile_coords(u, p, tm, tn, ks);
      const int ab = local & 1;
      fail = !mbar_wait(&acc_full[ab], (local >> 1) & 1, p.status, kSiteGemmEpilogue);
      if (fail) break;
      tc_fence_after();
      const int col0 = tn * BN;
#pragma unroll 1
      for (int h = 0; h < C::kMSub; ++h) {
        const int row_in_tile = h * 128 + row_in_sub;
        const int64_t row = static_cast<int64_t>(tm) * BM + row_in_tile;
        const bool row_ok = row < p.M;
        const uint32_t taddr =
            tmem + (static_cast<uint32_t>(q * 32) << 16) + ab * C::kAccCols + h * BN;
        float* part = nullptr;
        if (p.split > 1)
          part = p.partials +
                 ((static_cast<int64_t>(tm) * p.num_n + tn) * p.split + ks) * (BM * BN) +
                 row_in_tile * BN;
#pragma unroll 1
        for (int c = 0; c < BN / 32; ++c) {
          uint32_t raw[32];
          tmem_ld_32x32b_x32(taddr + c * 32, raw);
          tmem_ld_wait();
          if (p.split > 1) {
#pragma unroll
            for (int i = 0; i < 32; i += 4)
              __stcg(reinterpret_cast<float4*>(part + c * 32 + i),
                     make_float4(__uint_as_float(raw[i]), __uint_as_float(raw[i + 1]),
                                 __uint_as_float(raw[i + 2]), __uint_as_float(raw[i + 3])));
          } else if (row_ok) {
#pragma unroll
            for (int i = 0; i < 32; i += 8) {
              float v[8];
              // int4 B tiles hold each 8-column chunk in the order int4_codes8
              // emits; column e of the chunk sits at position (e%4)*2 + e/4.
#pragma unroll
              for (int e = 0; e < 8; ++e)
                v[e] = __uint_as_float(raw[i + (kInt4 ? ((e & 3) * 2 + (e >> 2)) : e)]) * out_scale;
              const int col = col0 + c * 32 + i;
              if (col < p.N) {
                if (p.peers.world == 0) {
                  store8(p.out, p.out_dtype, row * p.ldc + col, v, col + 8 <= p.N, min(8, p.N - col));
                } else {
                  for (int r = 0; r < p.peers.world; ++r)
                    store8(reinterpret_cast<void*>(p.peers.peer_out[r]), p.out_dtype,
                           row * p.ldc + p.peers.n_offset + col, v, col + 8 <= p.N,
                           min(8, p.N - col));
                  stored = true;
                }
              }
            }
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&acc_empty[ab]);

      if (p.split > 1) {
        // deterministic split-K: the last of the `split` units of this tile sums
        // the partials in split order
        __threadfence();
        named_bar_sync(1, kEpiWarps * 32);
        const int tile_id = tm * p.num_n + tn;
        if (tid == kEpiWarp0 * 32)
          *s_flag = (atomicAdd(&p.sems[tile_id], 1u) == static_cast<unsigned>(p.split - 1));
        named_bar_sync(1, kEpiWarps * 32);
        if (*s_flag) {
          __threadfence();
#pragma unroll 1
          for (int h = 0; h < C::kMSub; ++h) {
            const int row_in_tile = h * 128 + row_in_sub;
            const int64_t row = static_cast<int64_t>(tm) * BM + row_in_tile;
            const float* base = p.partials + static_cast<int64_t>(tile_id) * p.split * (BM * BN) +
                                row_in_tile * BN;
            if (row < p.M)
              sum_parts_row<BN>(base, BM * BN, p.split, out_scale, p.out, p.out_dtype,
                                row * p.ldc, col0, p.N);
          }
          named_bar_sync(1, kEpiWarps * 32);
          if (tid == kEpiWarp0 * 32) p.sems[tile_id] = 0u;  // re-arm
        }
      }
    }
  } else if (kInt4 && warp >= kDeqWarp0) {
    // ------------------------ dequant (W4A16 prefill) ------------------------
    // Stage: packed rows [kBK = 64][kBN/2 bytes] -> B tile [64 k][kBN n],
    // MN-major. A 16-byte shared access is serviced a quarter-warp (8 lanes) at
    // a time, so each quarter reads 8 different bank groups of the packed rows
    // and writes 8 different bank groups of the swizzled tile:
    //  * 128-byte rows (kBN = 256): quarter k of warp w, lane t takes quad t of
    //    rows 4w + ((t/2 + k) & 3) and that row + 32;
    //  * 64-byte rows (kBN = 128): quarter k of warp w, lane t takes quad t % 4
    //    of row 8w + 4(k/2) + 2((q/2) ^ (k%2)) + t/4.
    constexpr int kRowBytes = BN / 2;
    constexpr int kQuads = kRowBytes / 16;             // 16-byte quads per packed row
    constexpr int kRowsPerThread = (C::kBK * kQuads) / (kDeqWarps * 32);  // 2 or 1
    const int dt = tid - kDeqWarp0 * 32;   // 0..255
    const int qk = lane >> 3, qt = lane & 7;
    int wq, rbase;
    if (kQuads == 8) {
      wq = qt;
      rbase = 4 * (dt >> 5) + (((qt >> 1) + qk) & 3);
    } else {
      wq = qt & 3;
      rbase = 8 * (dt >> 5) + 4 * (qk >> 1) + 2 * ((wq >> 1) ^ (qk & 1)) + (qt >> 2);
    }
    int it = 0, bit = 0;
    for (int u = blockIdx.x; u < num_units && !fail; u += gridDim.x) {
      int tm, tn, ks;
      tile_coords(u, p, tm, tn, ks);
      const int kt0 = (ks * k_tiles_total) / p.split, kt1 = ((ks + 1) * k_tiles_total) / p.split;
      for (int kt = kt0; kt < kt1 && !fail; ++kt, ++it, ++bit) {
        const int st = it % C::kStages;
        const int bb = bit % kBBufs;
        fail = !mbar_wait(&full[st], (it / C::kStages) & 1, p.status, kSiteGemmDequant);
        if (!fail && bit >= C::kBBufs)
          fail = !mbar_wait(&bempty[bb], ((bit / kBBufs) - 1) & 1, p.status, kSiteGemmDequant);
        if (fail) break;
        const uint8_t* stage = smem + C::kStageOff + st * C::kStageBytes;
        const uint8_t* sc = stage + C::kATile + C::kWTile;
        // Group scales of this thread's 32 columns, regrouped to the pair order
        // int4_codes8 emits; the scale row arrives 128B-swizzled (chunk c at row
        // c/8, position (c%8) ^ (c/8)), so these reads are conflict-free.
        uint32_t sp[4][4];
        if (p.grouped) {
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            const int c = 4 * wq + i;
            const uint4 s4 =
                *reinterpret_cast<const uint4*>(sc + (c >> 3) * 128 + (((c & 7) ^ (c >> 3)) << 4));
            sp[i][0] = prmt(s4.x, s4.z, 0x5410);
            sp[i][1] = prmt(s4.x, s4.z, 0x7632);
            sp[i][2] = prmt(s4.y, s4.w, 0x5410);
            sp[i][3] = prmt(s4.y, s4.w, 0x7632);
          }
        }
        uint8_t* btile = smem + C::kBBufOff + bb * C::kBTile;
#pragma unroll
        for (int rr = 0; rr < kRowsPerThread; ++rr) {
          const int r = rbase + 32 * rr;
          const int r8 = r & 7;
          const uint4 wv =
              *reinterpret_cast<const uint4*>(stage + C::kATile + r * kRowBytes + wq * 16);
          const uint32_t words[4] = {wv.x, wv.y, wv.z, wv.w};
          uint8_t* bt = btile + (r >> 3) * 1024 + r8 * 128;
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            const int c = 4 * wq + i;  // 8-column chunk
            uint32_t v[4];
            if (p.a_is_f16)
              int4_codes8<__half>(words[i], v);
            else
              int4_codes8<__nv_bfloat16>(words[i], v);
            if (p.grouped) {
              if (p.a_is_f16) {
                __half* tag = nullptr;
                v[0] = mul2(v[0], sp[i][0], tag); v[1] = mul2(v[1], sp[i][1], tag);
                v[2] = mul2(v[2], sp[i][2], tag); v[3] = mul2(v[3], sp[i][3], tag);
              } else {
                __nv_bfloat16* tag = nullptr;
                v[0] = mul2(v[0], sp[i][0], tag); v[1] = mul2(v[1], sp[i][1], tag);
                v[2] = mul2(v[2], sp[i][2], tag); v[3] = mul2(v[3], sp[i][3], tag);
              }
            }
            *reinterpret_cast<uint4*>(bt + (c >> 3) * C::kBLBO + (((c & 7) ^ r8) << 4)) =
                make_uint4(v[0], v[1], v[2], v[3]);
          }
        }
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) {
          mbar_arrive(&bfull[bb]);
          mbar_arrive(&empty[st]);
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == kMmaWarp) tmem_dealloc(tmem, 512);
  if (p.peers.world > 1)
    peer_exchange_finish(p.peers, stored, p.status, kSiteGemmPeers, gridDim.x * gridDim.y);
}

// ---------------------------------------------------------------------------
// Pair tiles (dense fp16/bf16 and fp8, no split): a cluster of two CTAs
// computes a 256 x 256 tile with cta_group::2 MMAs (M = 256, N = 256). CTA r
// stages rows [128 r, 128 r + 128) of the A tile and columns
// [128 r, 128 r + 128) of the B tile; the MMA issued by CTA 0 reads both
// halves and writes rows 128 r .. of D into CTA r's TMEM. Per SM and k-step
// that is 32 KB of operands for the FLOPs a one-CTA 128 x 256 tile needs
// 48 KB for, and the smaller stages allow a deeper ring.
//
// Both CTAs' TMA loads signal CTA 0's `full` barrier (CTA 0 expects the bytes
// of both halves); the MMA completion is multicast to the `empty` and
// `acc_full` barriers of both CTAs; both CTAs' epilogue warps arrive on CTA
// 0's `acc_empty`.
// ---------------------------------------------------------------------------
template <int kKind>
struct PairCfg {
  static constexpr int kElem = kKind == kF16 ? 2 : 1;
  static constexpr int kBK = 128 / kElem;
  static constexpr int kMmaK = kKind == kF16 ? 16 : 32;
  static constexpr int kKSteps = kBK / kMmaK;
  static constexpr int kBM = 256, kBN = 256;            // pair tile
  static constexpr int kHalfM = 128, kHalfN = 128;      // per CTA
  static constexpr int kATile = kHalfM * 128;           // 16 KB
  static constexpr int kBTile = kBK * kHalfN * kElem;   // 16 KB
  static constexpr int kBAtomN = 128 / kElem;
  static constexpr int kBBoxes = kHalfN / kBAtomN;      // 2 (16-bit) / 1 (fp8)
  static constexpr int kBLBO = kBK * 128;
  static constexpr int kBStepBytes = (kMmaK / 8) * 1024;
  static constexpr int kStages = 6;
  static constexpr int kStageBytes = kATile + kBTile;
  static constexpr int kBarOff = kStages * kStageBytes;
  static constexpr int kSmem = kBarOff + 256 + 1024;
  static constexpr int kThreads = kDeqWarp0 * 32;       // TMA, MMA, 4 epilogue warps
  static constexpr int kAccCols = kBN;
  static constexpr uint32_t kIdesc = make_idesc(kKind == kF16 ? 1u : 0u, false, true, 256, kBN);
  static constexpr uint32_t kIdescF16 = make_idesc(0u, false, true, 256, kBN);
  // half-width units (N = 128: 64 columns, one 16-bit swizzle atom, per CTA)
  static constexpr uint32_t kIdescHalf = make_idesc(kKind == kF16 ? 1u : 0u, false, true, 256, kBN / 2);
  static constexpr uint32_t kIdescHalfF16 = make_idesc(0u, false, true, 256, kBN / 2);
  static_assert(2 * kAccCols <= 512, "two accumulator sets fit TMEM");
  static_assert(kSmem <= 227 * 1024, "shared memory");
};

// Pair-schedule unit u: whole tile u, or half `half` (0: columns 0-127, 1:
// 128-255) of tile whole + (u - whole) / 2.
__device__ __forceinline__ void pair_unit(int u, const Params& p, int& tile, int& half) {
  if (u < p.whole) {
    tile = u;
    half = -1;
  } else {
    tile = p.whole + ((u - p.whole) >> 1);
    half = (u - p.whole) & 1;
  }
}

template <int kKind>
__global__ void __launch_bounds__(PairCfg<kKind>::kThreads, 1)
    gemm_pair_kernel(const __grid_constant__ CUtensorMap tmA,
                     const __grid_constant__ CUtensorMap tmB, const Params p) {
  using C = PairCfg<kKind>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + C::kBarOff);
  uint64_t* empty = full + C::kStages;
  uint64_t* acc_full = empty + C::kStages;
  uint64_t* acc_empty = acc_full + 2;
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(acc_empty + 2);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const uint32_t rank = cluster_ctarank();
  const int pair = blockIdx.x >> 1, npairs = gridDim.x >> 1;
  const int k_tiles = (p.K + C::kBK - 1) / C::kBK;
  const int num_units = p.whole + 2 * (p.num_m * p.num_n - p.whole);

  if (warp == kTmaWarp && lane == 0) {
    for (int i = 0; i < C::kStages; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&acc_full[i], 1);
      mbar_init(&acc_empty[i], 2 * kEpiWarps);
    }
    fence_barrier_init();
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
  }
  if (warp == kMmaWarp) tmem_alloc_pair(tmem_holder, 512);
  tc_fence_before();
  cluster_sync();  // both CTAs' barriers exist before either signals the other
  tc_fence_after();
  const uint32_t tmem = *tmem_holder;
  griddep_wait();

  bool fail = false;
  if (warp == kTmaWarp) {
    // ------------------------------- producer -------------------------------
    if (lane == 0) {
      const uint32_t full0 = cluster_map(smem_u32(&full[0]), 0);
      int it = 0;
      for (int u = pair; u < num_units && !fail; u += npairs) {
        int tile, half, tm, tn, ks;
        pair_unit(u, p, tile, half);
        tile_coords(tile, p, tm, tn, ks);
        const int row = tm * C::kBM + static_cast<int>(rank) * C::kHalfM;
        // whole tile: this CTA's 128 columns; half unit: its 64 of the half's 128
        const int col = half < 0 ? tn * C::kBN + static_cast<int>(rank) * C::kHalfN
                                 : tn * C::kBN + half * (C::kBN / 2) + static_cast<int>(rank) * (C::kHalfN / 2);
        const int boxes = half < 0 ? C::kBBoxes : C::kBBoxes / 2;
        const uint32_t tx = 2u * (C::kATile + boxes * (C::kBTile / C::kBBoxes));
        for (int kt = 0; kt < k_tiles && !fail; ++kt, ++it) {
          const int st = it % C::kStages;
          if (it >= C::kStages)
            fail = !mbar_wait(&empty[st], ((it / C::kStages) - 1) & 1, p.status, kSiteGemmProducer);
          if (fail) break;
          uint8_t* base = smem + st * C::kStageBytes;
          const uint32_t bar = full0 + st * 8;
          if (rank == 0) mbar_arrive_expect_tx(&full[st], tx);
          const int k0 = kt * C::kBK;
          tma_load_2d_pair(base, &tmA, bar, k0, row);
          for (int b = 0; b < boxes; ++b)
            tma_load_2d_pair(base + C::kATile + b * C::kBLBO, &tmB, bar, col + b * C::kBAtomN, k0);
        }
      }
    }
  } else if (warp == kMmaWarp) {
    // ----------------------- MMA issuer (CTA 0 only) ------------------------
    if (rank == 0 && lane == 0) {
      int it = 0, local = 0;
      for (int u = pair; u < num_units && !fail; u += npairs, ++local) {
        int tile, half;
        pair_unit(u, p, tile, half);
        const uint32_t idesc = half < 0 ? (p.a_is_f16 ? C::kIdescF16 : C::kIdesc)
                                        : (p.a_is_f16 ? C::kIdescHalfF16 : C::kIdescHalf);
        const int ab = local & 1;
        if (local >= 2)
          fail = !mbar_wait_cluster(&acc_empty[ab], ((local >> 1) - 1) & 1, p.status, kSiteGemmMma);
        if (fail) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem + ab * C::kAccCols;
        for (int kt = 0; kt < k_tiles && !fail; ++kt, ++it) {
          const int st = it % C::kStages;
          fail = !mbar_wait(&full[st], (it / C::kStages) & 1, p.status, kSiteGemmMma);
          if (fail) break;
          tc_fence_after();
          const uint32_t a_base = smem_u32(smem + st * C::kStageBytes);
          const uint32_t b_base = a_base + C::kATile;
#pragma unroll
          for (int s = 0; s < C::kKSteps; ++s) {
            const uint64_t ad = make_smem_desc(a_base + s * 32, 16, 1024);
            const uint64_t bd = make_smem_desc(b_base + s * C::kBStepBytes, C::kBLBO, 1024);
            const uint32_t acc = (kt > 0 || s > 0) ? 1u : 0u;
            if (kKind == kF8)
              umma_f8_pair(d_tmem, ad, bd, idesc, acc);
            else
              umma_f16_pair(d_tmem, ad, bd, idesc, acc);
          }
          umma_commit_pair(&empty[st]);
        }
        if (fail) break;
        umma_commit_pair(&acc_full[ab]);
      }
    }
  } else if (warp >= kEpiWarp0 && warp < kEpiWarp0 + kEpiWarps) {
    // ----------------------- epilogue (both CTAs) ---------------------------
    const int q = warp & 3;  // TMEM lane quarter this warp may access
    const uint32_t acc_empty0 = cluster_map(smem_u32(&acc_empty[0]), 0);
    const float out_scale = epilogue_scale(p);
    int local = 0;
    for (int u = pair; u < num_units && !fail; u += npairs, ++local) {
      int tile, half, tm, tn, ks;
      pair_unit(u, p, tile, half);
      tile_coords(tile, p, tm, tn, ks);
      const int ab = local & 1;
      fail = !mbar_wait(&acc_full[ab], (local >> 1) & 1, p.status, kSiteGemmEpilogue);
      if (fail) break;
      tc_fence_after();
      const int64_t row =
          static_cast<int64_t>(tm) * C::kBM + static_cast<int>(rank) * C::kHalfM + q * 32 + lane;
      const bool row_ok = row < p.M;
      const uint32_t taddr = tmem + (static_cast<uint32_t>(q * 32) << 16) + ab * C::kAccCols;
      const int col0 = tn * C::kBN + (half < 0 ? 0 : half * (C::kBN / 2));
      const int ncols = half < 0 ? C::kBN : C::kBN / 2;
#pragma unroll 1
      for (int c = 0; c < ncols / 32; ++c) {
        uint32_t raw[32];
        tmem_ld_32x32b_x32(taddr + c * 32, raw);
        tmem_ld_wait();
        if (row_ok) {
#pragma unroll
          for (int i = 0; i < 32; i += 8) {
            float v[8];
#pragma unroll
            for (int e = 0; e < 8; ++e) v[e] = __uint_as_float(raw[i + e]) * out_scale;
            const int col = col0 + c * 32 + i;
            if (col < p.N)
              store8(p.out, p.out_dtype, row * p.ldc + col, v, col + 8 <= p.N, min(8, p.N - col));
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_cluster(acc_empty0 + ab * 8);
    }
  }

  tc_fence_before();
  __syncthreads();
  cluster_sync();  // neither CTA leaves while the other may still touch its memory
  tc_fence_after();
  if (warp == kMmaWarp) tmem_dealloc_pair(tmem, 512);
}

CUtensorMapDataType elem_tmap(int dt) {
  switch (dt) {
    case PK_BF16: return CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
    case PK_F16: return CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
    default: return CU_TENSOR_MAP_DATA_TYPE_UINT8;  // e4m3 moves as bytes
  }
}

template <int kKind, bool kInt4>
cudaError_t launch_typed(const GemmArgs& g, cudaStream_t s, const char** why) {
  using C = Cfg<kKind, kInt4>;
  const int elem = C::kElem;
  CUtensorMap tmA, tmB, tmS;
  if (!encode_tmap_2d(&tmA, elem_tmap(g.a_dtype), g.a, g.K, g.M, g.lda * elem, C::kBK, C::kBM,
                      CU_TENSOR_MAP_SWIZZLE_128B, why))
    return cudaErrorInvalidValue;
  if (kInt4) {
    if (!encode_tmap_2d(&tmB, CU_TENSOR_MAP_DATA_TYPE_UINT8, g.b, g.N / 2, g.K, g.N / 2,
                        C::kBN / 2, C::kBK, CU_TENSOR_MAP_SWIZZLE_NONE, why))
      return cudaErrorInvalidValue;
    if (g.scales != nullptr) {
      const int64_t G = (g.K + g.group - 1) / g.group;
      // the scales viewed as rows of 64 (128 bytes), kSRows rows per column tile
      if (!encode_tmap_2d(&tmS, elem_tmap(g.a_dtype), g.scales, 64, G * (g.N / 64), 128, 64,
                          C::kSRows, CU_TENSOR_MAP_SWIZZLE_128B, why))
        return cudaErrorInvalidValue;
    } else {
      tmS = tmB;  // unused
    }
  } else {
    if (!encode_tmap_2d(&tmB, elem_tmap(g.a_dtype), g.b, g.N, g.K, g.ldb * elem, C::kBAtomN,
                        C::kBK, CU_TENSOR_MAP_SWIZZLE_128B, why))
      return cudaErrorInvalidValue;
    tmS = tmB;
  }
  Params p{};
  p.M = static_cast<int>(g.M);
  p.N = static_cast<int>(g.N);
  p.K = static_cast<int>(g.K);
  p.split = g.split;
  p.num_m = static_cast<int>((g.M + C::kBM - 1) / C::kBM);
  p.num_n = static_cast<int>((g.N + C::kBN - 1) / C::kBN);
  p.out_dtype = g.out_dtype;
  p.ldc = g.ldc;
  p.out_scale = g.out_scale;
  p.scale_a = g.scale_a;
  p.scale_b = g.scale_b;
  p.out = g.out;
  p.partials = g.partials;
  p.sems = g.sems;
  p.group = g.group > 0 ? g.group : 1;
  p.grouped = g.scales != nullptr;
  p.a_is_f16 = g.a_dtype == PK_F16;
  p.status = g.status;
  p.peers = g.peers;
  const int units = p.num_m * p.num_n * p.split;
  const int grid = units < num_sms() ? units : num_sms();
  auto kernel = gemm_tc_kernel<kKind, kInt4>;
  cudaError_t e = set_max_smem(reinterpret_cast<const void*>(kernel), C::kSmem);
  if (e != cudaSuccess) return e;
  kernel<<<grid, C::kThreads, C::kSmem, s>>>(tmA, tmB, tmS, p);
  return cudaGetLastError();
}

// Pairs of CTAs that can be resident at once for the pair kernel (one CTA per
// SM): the persistent grid is twice this, capped by the tile count.
template <int kKind>
int pair_slots(cudaStream_t s) {
  static int cached[64] = {};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return num_sms() / 2;
  if (cached[dev] > 0) return cached[dev];
  using C = PairCfg<kKind>;
  cudaLaunchConfig_t cfg = {};
  cudaLaunchAttribute attr;
  attr.id = cudaLaunchAttributeClusterDimension;
  attr.val.clusterDim.x = 2;
  attr.val.clusterDim.y = 1;
  attr.val.clusterDim.z = 1;
  cfg.gridDim = dim3(num_sms(), 1, 1);
  cfg.blockDim = dim3(C::kThreads, 1, 1);
  cfg.dynamicSmemBytes = C::kSmem;
  cfg.stream = s;
  cfg.attrs = &attr;
  cfg.numAttrs = 1;
  int clusters = 0;
  if (cudaOccupancyMaxActiveClusters(&clusters, gemm_pair_kernel<kKind>, &cfg) != cudaSuccess ||
      clusters <= 0) {
    cudaGetLastError();
    clusters = num_sms() / 2;
  }
  cached[dev] = clusters;
  return clusters;
}

template <int kKind>
cudaError_t launch_pair(const GemmArgs& g, cudaStream_t s, const char** why) {
  using C = PairCfg<kKind>;
  CUtensorMap tmA, tmB;
  if (!encode_tmap_2d(&tmA, elem_tmap(g.a_dtype), g.a, g.K, g.M, g.lda * C::kElem, C::kBK,
                      C::kHalfM, CU_TENSOR_MAP_SWIZZLE_128B, why))
    return cudaErrorInvalidValue;
  if (!encode_tmap_2d(&tmB, elem_tmap(g.a_dtype), g.b, g.N, g.K, g.ldb * C::kElem, C::kBAtomN,
                      C::kBK, CU_TENSOR_MAP_SWIZZLE_128B, why))
    return cudaErrorInvalidValue;
  Params p{};
  p.M = static_cast<int>(g.M);
  p.N = static_cast<int>(g.N);
  p.K = static_cast<int>(g.K);
  p.split = 1;
  p.num_m = static_cast<int>((g.M + C::kBM - 1) / C::kBM);
  p.num_n = static_cast<int>((g.N + C::kBN - 1) / C::kBN);
  p.out_dtype = g.out_dtype;
  p.ldc = g.ldc;
  p.out_scale = g.out_scale;
  p.scale_a = g.scale_a;
  p.scale_b = g.scale_b;
  p.out = g.out;
  p.group = 1;
  p.a_is_f16 = g.a_dtype == PK_F16;
  p.status = g.status;
  auto kernel = gemm_pair_kernel<kKind>;
  cudaError_t e = set_max_smem(reinterpret_cast<const void*>(kernel), C::kSmem);
  if (e != cudaSuccess) return e;
  const int tiles = p.num_m * p.num_n;
  const int slots = pair_slots<kKind>(s);
  // A partial last wave of 16-bit tiles runs as half-width units (two per
  // tile, 64 columns per CTA: one swizzle atom) when they still fit one wave,
  // so it takes about half a tile's time. 8-bit B halves would be narrower
  // than a 128-byte swizzle atom: fp8 keeps whole tiles.
  p.whole = tiles;
  const int tail = tiles % slots;
  if (kKind == kF16 && tiles > slots && tail > 0 && 2 * tail <= slots) p.whole = tiles - tail;
  const int units = p.whole + 2 * (tiles - p.whole);
  cudaLaunchConfig_t cfg = {};
  cudaLaunchAttribute attrs[2];
  attrs[0].id = cudaLaunchAttributeClusterDimension;
  attrs[0].val.clusterDim.x = 2;
  attrs[0].val.clusterDim.y = 1;
  attrs[0].val.clusterDim.z = 1;
  attrs[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attrs[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.gridDim = dim3(2 * (units < slots ? units : slots), 1, 1);
  cfg.blockDim = dim3(C::kThreads, 1, 1);
  cfg.dynamicSmemBytes = C::kSmem;
  cfg.stream = s;
  cfg.attrs = attrs;
  cfg.numAttrs = 2;
  return cudaLaunchKernelEx(&cfg, kernel, tmA, tmB, p);
}

// dense split-K tiles (the only configuration that uses the workspace)
using DenseCfg = Cfg<kF16, false>;

}  // namespace

int64_t gemm_tiles(int64_t M, int64_t N) {
  return ((M + DenseCfg::kBM - 1) / DenseCfg::kBM) * ((N + DenseCfg::kBN - 1) / DenseCfg::kBN);
}

size_t gemm_splitk_workspace_bytes(int64_t M, int64_t N, int split) {
  if (split <= 1) return 0;
  const int64_t tiles = gemm_tiles(M, N);
  return kCounterBytes +
         static_cast<size_t>(tiles) * split * DenseCfg::kBM * DenseCfg::kBN * sizeof(float);
}

cudaError_t launch_gemm_tc(const GemmArgs& g, cudaStream_t s, const char** why) {
  if (g.peers.world > 0 && (g.kind != GemmArgs::kW4A16 || g.split > 1)) {
    *why = "the output exchange covers the fused W4A16 prefill without split-K only";
    return cudaErrorInvalidValue;
  }
  // Pair tiles for dense / fp8 products without split-K that have rows for both
  // halves of a pair, unless the pair tiles make at most one wave: then
  // one-CTA tiles keep at least as many SMs busy and start sooner (fp8
  // 2048^3: 14.7 us on one-CTA tiles, 15.7 us on pairs).
  if (g.kind != GemmArgs::kW4A16 && g.split <= 1 && g.M > 128) {
    const bool f8 = g.kind == GemmArgs::kFp8;
    const int64_t tiles = ((g.M + 255) / 256) * ((g.N + 255) / 256);
    if (tiles > (f8 ? pair_slots<kF8>(s) : pair_slots<kF16>(s)))
      return f8 ? launch_pair<kF8>(g, s, why) : launch_pair<kF16>(g, s, why);
  }
  if (g.kind == GemmArgs::kFp8) return launch_typed<kF8, false>(g, s, why);
  if (g.kind == GemmArgs::kW4A16) return launch_typed<kF16, true>(g, s, why);
  return launch_typed<kF16, false>(g, s, why);
}

}  // namespace pk
