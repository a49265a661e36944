// W4A16 decode on mma.sync tiles of exactly decoded fp16 operands, shared by
// the decode GEMVs (w4a16_gemv_cluster.cu, w4a16_gemv.cu).
//
// A unit is 512 K rows x 128 columns of Wp (64 packed bytes per row), loaded
// by TMA with the 64-byte swizzle into a 1024-byte aligned slot. Warp w of 8
// owns rows [64w, 64w + 64): four k-steps of 16 rows.
//
//  * Tiles (swap-AB): an m16n8k16 tile's 16 rows are 16 output columns, its
//    8 columns the (up to 8) output rows, its k the 16 weight rows of a
//    k-step. Lane (g, t) = (lane / 4, lane % 4) reads 8 bytes (columns
//    [16g, 16g + 16)) of rows 2t, 2t + 1, 2t + 8, 2t + 9 of a k-step, which
//    are the tile's k-columns of those numbers. Odd t read each row pair in
//    the other order, so that in every load the four lanes of a group touch
//    rows of both parities and two swizzle phases (the swizzle XORs the
//    16-byte chunk index with (row / 2) % 4): conflict-free.
//  * Decode. One PRMT puts byte b of rows x and x + 1 into halves 0 and 2 of
//    a word; one mask-and-flip LOP3 then leaves (q + 8) * 2^-24 (low nibble,
//    column 2b) or (q + 8) * 16 * 2^-24 (high nibble, column 2b + 1) in each
//    fp16 half: exact subnormal numbers. Tile j = 4h + b of the eight has
//    columns 16g + 2j (tile row g) and 16g + 2j + 1 (tile row g + 8).
//  * Activations. B fragments hold fp16 activations a' = a * 2^S (bf16 rows
//    scaled per output row so that the largest magnitude lies in [2^14,
//    2^15); fp16 rows unscaled). With the weights exact, every product in
//    the fp32 accumulators is exact.
//  * Offsets. Each unit's tiles start from one mma of the constant
//    -8 * 2^-24 (tile rows g) and -128 * 2^-24 (rows g + 8) with the same B
//    fragments: the sum of q * a' remains.
//  * Fold. Per unit the fp32 accumulators take the group scales (and, when
//    S changes from unit to unit, 2^-S); 2^24 and 2^20 are undone at the end.
#pragma once

#include "pk_common.cuh"

#include <type_traits>

namespace pk {
namespace w4mma {

constexpr int kRows = 512;            // K rows per unit
constexpr int kCols = 128;            // columns per unit
constexpr int kRowBytes = kCols / 2;  // 64
constexpr int kWarps = 8;
constexpr int kRowsPerWarp = kRows / kWarps;  // 64
constexpr int kKSteps = kRowsPerWarp / 16;    // 4
constexpr int kSub = 4;                       // TMA boxes per unit
constexpr int kSubRows = kRows / kSub;        // 128
constexpr int kSubWBytes = kSubRows * kRowBytes;
constexpr int kWBytes = kRows * kRowBytes;    // 32768
constexpr int kMaxM = 8;                      // one n8 block of the tile

// 32-bit words of one k-step's B fragments of a warp: lane (g, t) at words
// 2(4g + t), +1 for g < M; padded so that the four k-step blocks of a unit
// start on different banks (8M + pad = 8 or 24 mod 32).
template <int M>
__host__ __device__ constexpr int blk_words() {
  return 8 * M + (M % 2 == 0 ? 8 : 0);
}

// Decode constants as kernel parameters (constant-bank operands of the
// LOP3s, so that the mask and the flip fold into one instruction).
struct Consts {
  uint32_t m_lo;  // low nibbles of both fp16 halves: 0x000F000F
  uint32_t f_lo;  //   their top bits, q -> q + 8: 0x00080008
  uint32_t m_hi;  // high nibbles: 0x00F000F0
  uint32_t f_hi;  //   0x00800080
};
inline Consts consts() { return Consts{0x000F000Fu, 0x00080008u, 0x00F000F0u, 0x00800080u}; }

__device__ __forceinline__ float exp2i(int e) {
  return __uint_as_float(static_cast<uint32_t>(e + 127) << 23);
}

// D += A * B on one m16n8k16 tile: fp16 operands, fp32 accumulators.
__device__ __forceinline__ void mma_16816(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2,
                                          uint32_t a3, uint32_t b0, uint32_t b1) {
  asm("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, "
      "{%8, %9}, {%0, %1, %2, %3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}
__device__ __forceinline__ uint2 lds_v2(uint32_t addr) {
  uint2 v;
  asm volatile("ld.shared.v2.u32 {%0, %1}, [%2];" : "=r"(v.x), "=r"(v.y) : "r"(addr));
  return v;
}
__device__ __forceinline__ void sts_u32(uint32_t addr, uint32_t v) {
  asm volatile("st.shared.u32 [%0], %1;" ::"r"(addr), "r"(v) : "memory");
}

// Per-lane constants of the fragment layout.
struct LaneMap {
  uint32_t sel[4];   // PRMT selectors: byte b of rows x, x + 1 -> halves 0, 2
  uint32_t woff[4];  // byte offsets of the lane's 4 rows in a swizzled k-step
  int g, t;
};
__device__ __forceinline__ LaneMap lane_map(int lane) {
  LaneMap lm;
  lm.g = lane >> 2;
  lm.t = lane & 3;
#pragma unroll
  for (int b = 0; b < 4; ++b)
    lm.sel[b] = (lm.t & 1) ? ((b + 4) | ((b + 4) << 4) | (b << 8) | (b << 12))
                           : (b | (b << 4) | ((b + 4) << 8) | ((b + 4) << 12));
#pragma unroll
  for (int r = 0; r < 4; ++r) {
    const int row = 2 * lm.t + (r >> 1) * 8 + ((r & 1) ^ (lm.t & 1));
    lm.woff[r] =
        row * kRowBytes + ((((lm.g >> 1) ^ ((row >> 1) & 3)) << 4) | ((lm.g & 1) << 3));
  }
  return lm;
}

// Byte offset, within a unit's B-fragment block, of the word that lane l
// writes for output row m: lane l converts rows 2l, 2l + 1 of the warp's 64,
// which are k-step l / 8, B-fragment lane (m, l % 4), register (l / 4) % 2.
template <int M>
__device__ __forceinline__ uint32_t bfrag_store_off(int lane, int m) {
  return ((lane >> 3) * blk_words<M>() + (m * 4 + (lane & 3)) * 2 + ((lane >> 2) & 1)) * 4;
}

// Scale exponent for the largest bf16 exponent field `emax` of a row block:
// S = clamp(141 - e_max, -126, 126) puts the largest magnitude in [2^14, 2^15).
__device__ __forceinline__ int scale_exp(uint32_t emax) {
  int S = 141 - static_cast<int>(emax);
  return S < -126 ? -126 : (S > 126 ? 126 : S);
}
// Largest exponent field of the two bf16 values in `raw`.
__device__ __forceinline__ uint32_t bf16x2_emax(uint32_t raw) {
  const uint32_t e0 = (raw >> 7) & 0xFFu, e1 = (raw >> 23) & 0xFFu;
  return e0 > e1 ? e0 : e1;
}
// Two 16-bit activations (rows 2l, 2l + 1) as an fp16x2 B-fragment word.
template <typename T>
__device__ __forceinline__ uint32_t to_f16x2(uint32_t raw, float sc) {
  if constexpr (std::is_same<T, __nv_bfloat16>::value) {
    const __half2 hv = __floats2half2_rn(__uint_as_float(raw << 16) * sc,
                                         __uint_as_float(raw & 0xFFFF0000u) * sc);
    return *reinterpret_cast<const uint32_t*>(&hv);
  } else {
    return raw;
  }
}

// The B fragments of a unit's four k-steps (bfrag: this lane's entry of
// k-step 0, k-step s at + s * blk_words * 4).
template <int M>
__device__ __forceinline__ void load_bfrags(uint32_t bfrag, uint32_t (&bf)[kKSteps][2]) {
#pragma unroll
  for (int s = 0; s < kKSteps; ++s) {
    const uint2 v = lds_v2(bfrag + s * blk_words<M>() * 4);
    bf[s][0] = v.x;
    bf[s][1] = v.y;
  }
}

// The +8 offsets of a unit through the tensor cores: the constant
// -8 * 2^-24 (tile rows g) and -128 * 2^-24 (rows g + 8) times the
// activations, the starting value of every tile's sum.
__device__ __forceinline__ void offsets_mma(const uint32_t (&bf)[kKSteps][2], float (&doff)[4]) {
  constexpr uint32_t kOffLo = 0x80088008u;  // -8 * 2^-24 in both fp16 halves
  constexpr uint32_t kOffHi = 0x80808080u;  // -128 * 2^-24
#pragma unroll
  for (int e = 0; e < 4; ++e) doff[e] = 0.0f;
#pragma unroll
  for (int s = 0; s < kKSteps; ++s) mma_16816(doff, kOffLo, kOffHi, kOffLo, kOffHi, bf[s][0], bf[s][1]);
}

// The tile loop of one unit of one warp: acc[j] = doff + the tile sums of
// the unit's four k-steps. v holds the first k-step's rows on entry (loaded
// with load_rows); the later k-steps' rows are loaded while a k-step's eight
// A fragments are decoded, and its eight mma's then issue back to back.
__device__ __forceinline__ void load_rows(const LaneMap& lm, uint32_t wbase, int s, uint2 (&v)[4]) {
#pragma unroll
  for (int r = 0; r < 4; ++r) v[r] = lds_v2(wbase + s * 16 * kRowBytes + lm.woff[r]);
}
__device__ __forceinline__ void tile_loop(const LaneMap& lm, uint32_t wbase, uint2 (&v)[4],
                                          const uint32_t (&bf)[kKSteps][2],
                                          const float (&doff)[4], const Consts& dc,
                                          float (&acc)[8][4]) {
#pragma unroll
  for (int j = 0; j < 8; ++j)
#pragma unroll
    for (int e = 0; e < 4; ++e) acc[j][e] = doff[e];
#pragma unroll
  for (int s = 0; s < kKSteps; ++s) {
    uint32_t a[8][4];
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const uint32_t w0 = h ? v[0].y : v[0].x, w1 = h ? v[1].y : v[1].x;
      const uint32_t w2 = h ? v[2].y : v[2].x, w3 = h ? v[3].y : v[3].x;
#pragma unroll
      for (int b = 0; b < 4; ++b) {
        const uint32_t z01 = __byte_perm(w0, w1, lm.sel[b]);
        const uint32_t z23 = __byte_perm(w2, w3, lm.sel[b]);
        a[4 * h + b][0] = (z01 & dc.m_lo) ^ dc.f_lo;
        a[4 * h + b][1] = (z01 & dc.m_hi) ^ dc.f_hi;
        a[4 * h + b][2] = (z23 & dc.m_lo) ^ dc.f_lo;
        a[4 * h + b][3] = (z23 & dc.m_hi) ^ dc.f_hi;
      }
    }
    if (s + 1 < kKSteps) load_rows(lm, wbase, s + 1, v);
#pragma unroll
    for (int j = 0; j < 8; ++j)
      mma_16816(acc[j], a[j][0], a[j][1], a[j][2], a[j][3], bf[s][0], bf[s][1]);
  }
}

// The lane's 32 bytes of group scales (columns 16g .. 16g + 15).
__device__ __forceinline__ void load_scales(uint32_t scale_addr, uint32_t (&sws)[8]) {
  const uint4 s0 = lds_v4(scale_addr), s1 = lds_v4(scale_addr + 16);
  sws[0] = s0.x, sws[1] = s0.y, sws[2] = s0.z, sws[3] = s0.w;
  sws[4] = s1.x, sws[5] = s1.y, sws[6] = s1.z, sws[7] = s1.w;
}

// Fold a unit's tile sums: tot[j][e] += acc[j][e] * scale * (e % 2 ? pw1 :
// pw0) (kPw) or * scale; scale from sws (kGrouped) or scalar_scale.
template <typename T, bool kGrouped, bool kPw>
__device__ __forceinline__ void fold(const float (&acc)[8][4], const uint32_t (&sws)[8],
                                     float scalar_scale, float pw0, float pw1,
                                     float (&tot)[8][4]) {
  constexpr bool kBf16 = std::is_same<T, __nv_bfloat16>::value;
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    float se, so;
    if constexpr (kGrouped) {
      if constexpr (kBf16) {
        se = __uint_as_float(sws[j] << 16);
        so = __uint_as_float(sws[j] & 0xFFFF0000u);
      } else {
        const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&sws[j]));
        se = f.x;
        so = f.y;
      }
    } else {
      se = so = scalar_scale;
    }
    if constexpr (kPw) {
      tot[j][0] = fmaf(acc[j][0], se * pw0, tot[j][0]);
      tot[j][1] = fmaf(acc[j][1], se * pw1, tot[j][1]);
      tot[j][2] = fmaf(acc[j][2], so * pw0, tot[j][2]);
      tot[j][3] = fmaf(acc[j][3], so * pw1, tot[j][3]);
    } else {
      tot[j][0] = fmaf(acc[j][0], se, tot[j][0]);
      tot[j][1] = fmaf(acc[j][1], se, tot[j][1]);
      tot[j][2] = fmaf(acc[j][2], so, tot[j][2]);
      tot[j][3] = fmaf(acc[j][3], so, tot[j][3]);
    }
  }
}

// The tiles of one unit of one warp, started from doff, then folded.
template <int M, typename T, bool kGrouped, bool kPw>
__device__ __forceinline__ void tiles(const LaneMap& lm, uint32_t wbase,
                                      const uint32_t (&bf)[kKSteps][2], uint32_t scale_addr,
                                      float scalar_scale, float pw0, float pw1,
                                      const float (&doff)[4], const Consts& dc,
                                      float (&tot)[8][4]) {
  uint2 v[4];
  load_rows(lm, wbase, 0, v);
  float acc[8][4];
  tile_loop(lm, wbase, v, bf, doff, dc, acc);
  uint32_t sws[8];
  if constexpr (kGrouped) load_scales(scale_addr, sws);
  fold<T, kGrouped, kPw>(acc, sws, scalar_scale, pw0, pw1, tot);
}

// One unit of one warp with its offsets through the tensor cores.
template <int M, typename T, bool kGrouped, bool kPw>
__device__ __forceinline__ void unit(const LaneMap& lm, uint32_t wbase, uint32_t bfrag,
                                     uint32_t scale_addr, float scalar_scale, float pw0,
                                     float pw1, const Consts& dc, float (&tot)[8][4]) {
  uint32_t bf[kKSteps][2];
  load_bfrags<M>(bfrag, bf);
  float doff[4];
  offsets_mma(bf, doff);
  tiles<M, T, kGrouped, kPw>(lm, wbase, bf, scale_addr, scalar_scale, pw0, pw1, doff, dc, tot);
}

// ---------------------------------------------------------------------------
// Four-tile warps (64 columns, 32 packed bytes per row), for kernels with 16
// mma warps. Four warps share a TMA box of 64 rows x 128 bytes, 128-byte
// swizzled (the 16-byte chunk index XOR-ed with row % 8); warp q of a box
// owns bytes [32q, 32q + 32). Lane (g, t) reads the word of columns
// [8g, 8g + 8) of rows 2t, 2t + 1, 2t + 8, 2t + 9 of a k-step, the tile's
// k-columns of those numbers: in every load the four lane groups touch rows
// whose (row / 2) % 4 differ, so their chunks land on different banks
// (conflict-free). Tile j (= byte j of the word) has columns 8g + 2j (tile
// row g) and 8g + 2j + 1 (row g + 8). The B fragments are those of the
// eight-tile form (rows 2l, 2l + 1 per prep lane l).
// ---------------------------------------------------------------------------
constexpr int kRowBytes4 = 32;     // a warp's bytes of one row
constexpr int kBoxRowBytes4 = 128;  // four warps' bytes of one row

// Byte offsets, within a box, of the lane's four rows of k-step 0 (k-step s
// at + s * 16 * 128: 16 rows keep row % 8).
__device__ __forceinline__ void lane_rows4(int lane, int q, uint32_t (&off)[4]) {
  const int g = lane >> 2, t = lane & 3;
#pragma unroll
  for (int r = 0; r < 4; ++r) {
    const int row = 2 * t + (r & 1) + 8 * (r >> 1);
    const int chunk = (2 * q + (g >> 2)) ^ (row & 7);
    off[r] = row * kBoxRowBytes4 + chunk * 16 + (g & 3) * 4;
  }
}

__device__ __forceinline__ void load_rows4(uint32_t box, const uint32_t (&off)[4], int s,
                                           uint32_t (&v)[4]) {
#pragma unroll
  for (int r = 0; r < 4; ++r) v[r] = lds_u32(box + s * 16 * kBoxRowBytes4 + off[r]);
}

// acc[j] = doff + the tile sums of the unit's four k-steps (box: the warp's
// box in the slot, off: lane_rows4).
__device__ __forceinline__ void tile_loop4(uint32_t box, const uint32_t (&off)[4],
                                           const uint32_t (&bf)[kKSteps][2],
                                           const float (&doff)[4], const Consts& dc,
                                           float (&acc)[4][4]) {
#pragma unroll
  for (int j = 0; j < 4; ++j)
#pragma unroll
    for (int e = 0; e < 4; ++e) acc[j][e] = doff[e];
  uint32_t v[4];
  load_rows4(box, off, 0, v);
#pragma unroll
  for (int s = 0; s < kKSteps; ++s) {
    uint32_t a[4][4];
#pragma unroll
    for (int b = 0; b < 4; ++b) {
      const uint32_t sel = b | (b << 4) | ((b + 4) << 8) | ((b + 4) << 12);
      const uint32_t z01 = __byte_perm(v[0], v[1], sel);
      const uint32_t z23 = __byte_perm(v[2], v[3], sel);
      a[b][0] = (z01 & dc.m_lo) ^ dc.f_lo;
      a[b][1] = (z01 & dc.m_hi) ^ dc.f_hi;
      a[b][2] = (z23 & dc.m_lo) ^ dc.f_lo;
      a[b][3] = (z23 & dc.m_hi) ^ dc.f_hi;
    }
    if (s + 1 < kKSteps) load_rows4(box, off, s + 1, v);
#pragma unroll
    for (int j = 0; j < 4; ++j)
      mma_16816(acc[j], a[j][0], a[j][1], a[j][2], a[j][3], bf[s][0], bf[s][1]);
  }
}

// Fold four tiles: tot[j][e] += acc[j][e] * scale * (e % 2 ? pw1 : pw0);
// scale from the lane's 16 bytes of group scales (columns 8g .. 8g + 7).
template <typename T, bool kGrouped>
__device__ __forceinline__ void fold4(const float (&acc)[4][4], uint32_t scale_addr,
                                      float scalar_scale, float pw0, float pw1,
                                      float (&tot)[4][4]) {
  constexpr bool kBf16 = std::is_same<T, __nv_bfloat16>::value;
  uint32_t sws[4] = {0u, 0u, 0u, 0u};
  if constexpr (kGrouped) {
    const uint4 s0 = lds_v4(scale_addr);
    sws[0] = s0.x, sws[1] = s0.y, sws[2] = s0.z, sws[3] = s0.w;
  }
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    float se, so;
    if constexpr (kGrouped) {
      if constexpr (kBf16) {
        se = __uint_as_float(sws[j] << 16);
        so = __uint_as_float(sws[j] & 0xFFFF0000u);
      } else {
        const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&sws[j]));
        se = f.x;
        so = f.y;
      }
    } else {
      se = so = scalar_scale;
    }
    tot[j][0] = fmaf(acc[j][0], se * pw0, tot[j][0]);
    tot[j][1] = fmaf(acc[j][1], se * pw1, tot[j][1]);
    tot[j][2] = fmaf(acc[j][2], so * pw0, tot[j][2]);
    tot[j][3] = fmaf(acc[j][3], so * pw1, tot[j][3]);
  }
}

// The lane's sums as [m][column] partials of its warp: 2^24 (low nibbles)
// and 2^20 (high nibbles) undone, times pw (per output row, when not folded).
template <int M>
__device__ __forceinline__ void store_sums(uint32_t red_warp, const LaneMap& lm,
                                           const float (&tot)[8][4], float pw0, float pw1) {
#pragma unroll
  for (int e = 0; e < 2; ++e) {
    const int n = 2 * lm.t + e;
    const float pw = e ? pw1 : pw0;
    if (n < M) {
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const float lo = tot[j][e] * 16777216.0f * pw, hi = tot[j][2 + e] * 1048576.0f * pw;
        asm volatile("st.shared.v2.f32 [%0], {%1, %2};" ::"r"(
                         red_warp + (n * kCols + 16 * lm.g + 2 * j) * 4),
                     "f"(lo), "f"(hi)
                     : "memory");
      }
    }
  }
}

}  // namespace w4mma
}  // namespace pk
