// int4 quantize / pack / unpack and the fp8 cast: HBM-bound byte work.
//
// Bit-exactness with the reference (torch CPU semantics) rests on:
//   * IEEE fp32 division (this file must not be built with fast-math);
//   * rintf = round half to even, like torch.round;
//   * the stored scale = RNE conversion of the fp32 scale.
#include <cuda_fp8.h>

#include "pk_common.cuh"

namespace pk {
namespace {

template <typename T>
__device__ __forceinline__ float to_f32(T v);
template <>
__device__ __forceinline__ float to_f32<__half>(__half v) { return __half2float(v); }
template <>
__device__ __forceinline__ float to_f32<__nv_bfloat16>(__nv_bfloat16 v) {
  return __bfloat162float(v);
}
template <>
__device__ __forceinline__ float to_f32<float>(float v) { return v; }

template <typename T>
__device__ __forceinline__ T from_f32(float v);
template <>
__device__ __forceinline__ __half from_f32<__half>(float v) { return __float2half_rn(v); }
template <>
__device__ __forceinline__ __nv_bfloat16 from_f32<__nv_bfloat16>(float v) {
  return __float2bfloat16_rn(v);
}
template <>
__device__ __forceinline__ float from_f32<float>(float v) { return v; }

// Round an fp32 value to T and back (the dtype of a torch elementwise result).
template <typename T>
__device__ __forceinline__ float round_through(float v) { return to_f32<T>(from_f32<T>(v)); }

__device__ __forceinline__ int group_code(float w, float s) {
  // quantize.py:59: clamp(round(w / scale), -7, 7)
  float q = rintf(w / s);
  q = fminf(fmaxf(q, -7.0f), 7.0f);
  return static_cast<int>(q);
}

__device__ __forceinline__ float group_scale(float amax) {
  // quantize.py:58: max|w|.clamp_min(1e-12) / qmax, qmax = 7 for 4 bits
  return fmaxf(amax, 1e-12f) / 7.0f;
}

// ---------------------------------------------------------------------------
// Per-group quantize + pack, vectorised path.
// A warp covers 32 columns x one group: lane = 4 column slots (8 columns,
// one 16-byte load each) x 8 row slices; row slice r holds rows r, r+8, ...
// The group absmax is combined across the 8 row slices with xor-shuffles.
// Requirements: 16-bit input, N % 8 == 0, ldw % 8 == 0, 16-byte aligned base,
// group % 8 == 0 and group <= 128.
// ---------------------------------------------------------------------------
constexpr int kQuantWarps = 8;
constexpr int kMaxRowsPerLane = 16;

template <typename Tin, typename Tsc>
__global__ void __launch_bounds__(kQuantWarps * 32)
    quant_int4_group_vec(const Tin* __restrict__ w, int64_t K, int64_t N, int64_t ldw, int group,
                         uint8_t* __restrict__ packed, Tsc* __restrict__ scales) {
  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  const int cs = lane & 3;
  const int rs = lane >> 2;
  const int64_t col0 = (static_cast<int64_t>(blockIdx.x) * kQuantWarps + warp) * 32 + cs * 8;
  const int64_t g = blockIdx.y;
  const int64_t k0 = g * group;
  const int rpl = group >> 3;
  const bool col_ok = col0 < N;

  uint4 v[kMaxRowsPerLane];
#pragma unroll
  for (int i = 0; i < kMaxRowsPerLane; ++i) {
    const int64_t k = k0 + rs + 8 * i;
    if (i < rpl && k < K && col_ok) {
      v[i] = __ldg(reinterpret_cast<const uint4*>(w + k * ldw + col0));
    } else {
      v[i] = make_uint4(0, 0, 0, 0);
    }
  }

  float amax[8];
#pragma unroll
  for (int c = 0; c < 8; ++c) amax[c] = 0.0f;
#pragma unroll
  for (int i = 0; i < kMaxRowsPerLane; ++i) {
    const Tin* e = reinterpret_cast<const Tin*>(&v[i]);
#pragma unroll
    for (int c = 0; c < 8; ++c) amax[c] = fmaxf(amax[c], fabsf(to_f32<Tin>(e[c])));
  }
#pragma unroll
  for (int c = 0; c < 8; ++c) {
    amax[c] = fmaxf(amax[c], __shfl_xor_sync(0xffffffffu, amax[c], 4));
    amax[c] = fmaxf(amax[c], __shfl_xor_sync(0xffffffffu, amax[c], 8));
    amax[c] = fmaxf(amax[c], __shfl_xor_sync(0xffffffffu, amax[c], 16));
  }
  float s[8];
#pragma unroll
  for (int c = 0; c < 8; ++c) s[c] = group_scale(amax[c]);

  if (!col_ok) return;
  const int64_t ldp = N >> 1;
#pragma unroll
  for (int i = 0; i < kMaxRowsPerLane; ++i) {
    const int64_t k = k0 + rs + 8 * i;
    if (i < rpl && k < K) {
      const Tin* e = reinterpret_cast<const Tin*>(&v[i]);
      uint32_t word = 0;
#pragma unroll
      for (int c = 0; c < 8; ++c) {
        const uint32_t nib = static_cast<uint32_t>(group_code(to_f32<Tin>(e[c]), s[c])) & 0xFu;
        word |= nib << (4 * c);
      }
      *reinterpret_cast<uint32_t*>(packed + k * ldp + (col0 >> 1)) = word;
    }
  }
  if (rs == 0) {
#pragma unroll
    for (int c = 0; c < 8; ++c) scales[g * N + col0 + c] = from_f32<Tsc>(s[c]);
  }
}

// Generic path: any dtype, group size, alignment or ragged shape. One thread
// per (column pair, group), two passes over the group's rows.
template <typename Tin, typename Tsc>
__global__ void quant_int4_group_generic(const Tin* __restrict__ w, int64_t K, int64_t N,
                                         int64_t ldw, int group, uint8_t* __restrict__ packed,
                                         Tsc* __restrict__ scales) {
  const int64_t pair = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  const int64_t g = blockIdx.y;
  if (2 * pair >= N) return;
  const int64_t c0 = 2 * pair;
  const int64_t k0 = g * group;
  const int64_t k1 = min(K, k0 + group);
  float a0 = 0.0f, a1 = 0.0f;
  for (int64_t k = k0; k < k1; ++k) {
    a0 = fmaxf(a0, fabsf(to_f32<Tin>(w[k * ldw + c0])));
    a1 = fmaxf(a1, fabsf(to_f32<Tin>(w[k * ldw + c0 + 1])));
  }
  const float s0 = group_scale(a0), s1 = group_scale(a1);
  for (int64_t k = k0; k < k1; ++k) {
    const uint32_t q0 = static_cast<uint32_t>(group_code(to_f32<Tin>(w[k * ldw + c0]), s0)) & 0xF;
    const uint32_t q1 =
        static_cast<uint32_t>(group_code(to_f32<Tin>(w[k * ldw + c0 + 1]), s1)) & 0xF;
    packed[k * (N >> 1) + pair] = static_cast<uint8_t>(q0 | (q1 << 4));
  }
  scales[g * N + c0] = from_f32<Tsc>(s0);
  scales[g * N + c0 + 1] = from_f32<Tsc>(s1);
}

// ---------------------------------------------------------------------------
// absmax: grid-stride max|x| with an integer atomicMax on the fp32 bits
// (valid for non-negative floats).
// ---------------------------------------------------------------------------
template <typename T>
__global__ void absmax_kernel(const T* __restrict__ x, int64_t n, float* __restrict__ out) {
  float m = 0.0f;
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  constexpr int kVec = 16 / sizeof(T);
  const bool vec = (reinterpret_cast<uintptr_t>(x) & 15) == 0;
  if (vec) {
    const int64_t nv = n / kVec;
    for (int64_t j = i; j < nv; j += stride) {
      uint4 u = __ldg(reinterpret_cast<const uint4*>(x) + j);
      const T* e = reinterpret_cast<const T*>(&u);
#pragma unroll
      for (int c = 0; c < kVec; ++c) m = fmaxf(m, fabsf(to_f32<T>(e[c])));
    }
    for (int64_t j = nv * kVec + i; j < n; j += stride) m = fmaxf(m, fabsf(to_f32<T>(x[j])));
  } else {
    for (int64_t j = i; j < n; j += stride) m = fmaxf(m, fabsf(to_f32<T>(x[j])));
  }
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, off));
  __shared__ float red[32];
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = m;
  __syncthreads();
  if (threadIdx.x < 32) {
    m = threadIdx.x < (blockDim.x >> 5) ? red[threadIdx.x] : 0.0f;
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, off));
    if (threadIdx.x == 0) atomicMax(reinterpret_cast<int*>(out), __float_as_int(m));
  }
}

// gemm_int4.py:61: round(w / scale).clamp(-8, 7).to(int8), the quotient held
// in w's dtype.
template <typename T>
__global__ void quant_int4_tensor_kernel(const T* __restrict__ w, int64_t n, float scale,
                                         int8_t* __restrict__ q) {
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
       i += stride) {
    float r = rintf(round_through<T>(to_f32<T>(w[i]) / scale));
    r = fminf(fmaxf(r, -8.0f), 7.0f);
    q[i] = (r == r) ? static_cast<int8_t>(r) : int8_t(0);
  }
}

// gemm_int4.py:65-72, 16 codes -> 8 bytes per thread on the vector path.
__global__ void pack_int4_vec(const int8_t* __restrict__ q, int64_t n16,
                              uint8_t* __restrict__ p) {
  const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= n16) return;
  const uint4 u = __ldg(reinterpret_cast<const uint4*>(q) + i);
  const uint32_t in[4] = {u.x, u.y, u.z, u.w};
  uint32_t out[2] = {0, 0};
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    const uint32_t word = in[j >> 1];
    const int sh = (j & 1) * 16;
    const uint32_t lo = (word >> sh) & 0xF;
    const uint32_t hi = (word >> (sh + 8)) & 0xF;
    out[j >> 2] |= (lo | (hi << 4)) << (8 * (j & 3));
  }
  reinterpret_cast<uint2*>(p)[i] = make_uint2(out[0], out[1]);
}

__global__ void pack_int4_scalar(const int8_t* __restrict__ q, int64_t nbytes,
                                 uint8_t* __restrict__ p) {
  const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= nbytes) return;
  const uint32_t lo = static_cast<uint32_t>(q[2 * i]) & 0xF;
  const uint32_t hi = static_cast<uint32_t>(q[2 * i + 1]) & 0xF;
  p[i] = static_cast<uint8_t>(lo | (hi << 4));
}

__global__ void unpack_int4_kernel(const uint8_t* __restrict__ p, int64_t nbytes,
                                   int8_t* __restrict__ q) {
  const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= nbytes) return;
  const int b = p[i];
  const int lo = b & 0xF, hi = b >> 4;
  q[2 * i] = static_cast<int8_t>(lo >= 8 ? lo - 16 : lo);
  q[2 * i + 1] = static_cast<int8_t>(hi >= 8 ? hi - 16 : hi);
}

// gemm_fp8.py:95: (x * scale) in x's dtype, then RNE to e4m3.
template <typename T>
__global__ void fp8_quantize_kernel(const T* __restrict__ x, int64_t n, float scale,
                                    uint8_t* __restrict__ y) {
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
       i += stride) {
    const float v = round_through<T>(to_f32<T>(x[i]) * scale);
    y[i] = static_cast<uint8_t>(__nv_cvt_float_to_fp8(v, __NV_NOSAT, __NV_E4M3));
  }
}

// gemm_fp8.py:89-95 without the host round trip: scale = E4M3_MAX / amax is
// computed here from the absmax the previous kernel left in device memory
// (fp32 division, correctly rounded: the same float as the reference's
// double quotient rounded to fp32), then (x * scale) in x's dtype, RNE to
// e4m3. Block 0 stores the scale for the GEMM epilogue. An all-zero input
// (where the reference's division raises) gets scale 1. Eight elements per
// thread: one 16-byte load of 16-bit inputs (two of fp32), one 8-byte store.
constexpr float kE4m3Max = 448.0f;

template <typename T>
__global__ void fp8_quantize_dev_kernel(const T* __restrict__ x, int64_t n,
                                        const float* __restrict__ amax, float* __restrict__ scale_out,
                                        uint8_t* __restrict__ y) {
  const float m = *amax;
  const float scale = m > 0.0f ? kE4m3Max / m : 1.0f;
  if (blockIdx.x == 0 && threadIdx.x == 0) *scale_out = scale;
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  const int64_t tid = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  const bool vec = (reinterpret_cast<uintptr_t>(x) & 15) == 0 &&
                   (reinterpret_cast<uintptr_t>(y) & 7) == 0;
  const int64_t n8 = vec ? n / 8 : 0;
  for (int64_t i = tid; i < n8; i += stride) {
    float v[8];
    if constexpr (sizeof(T) == 2) {
      const uint4 u = __ldg(reinterpret_cast<const uint4*>(x) + i);
      const T* e = reinterpret_cast<const T*>(&u);
#pragma unroll
      for (int c = 0; c < 8; ++c) v[c] = to_f32<T>(e[c]);
    } else {
      const float4 a = __ldg(reinterpret_cast<const float4*>(x) + 2 * i);
      const float4 b = __ldg(reinterpret_cast<const float4*>(x) + 2 * i + 1);
      v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w;
      v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
    }
    uint32_t w[2] = {0u, 0u};
#pragma unroll
    for (int c = 0; c < 8; ++c) {
      const uint32_t b8 = __nv_cvt_float_to_fp8(round_through<T>(v[c] * scale), __NV_NOSAT,
                                                __NV_E4M3);
      w[c >> 2] |= b8 << (8 * (c & 3));
    }
    reinterpret_cast<uint2*>(y)[i] = make_uint2(w[0], w[1]);
  }
  for (int64_t i = n8 * 8 + tid; i < n; i += stride) {
    const float v = round_through<T>(to_f32<T>(x[i]) * scale);
    y[i] = static_cast<uint8_t>(__nv_cvt_float_to_fp8(v, __NV_NOSAT, __NV_E4M3));
  }
}

// Dequantize packed int4 weights once into a 16-bit row-major B[K, N] for the
// dense tensor-core GEMM of large-M calls: B[k, n] = q[k, n] * s[k/g, n] rounded
// to T by the same packed instructions the fused W4A16 kernel uses for its MMA
// operand (dequant8), or q exactly when there are no group scales. One thread
// per 8 columns of a row, so a warp's loads (128 B packed, 512 B scales) and its
// 512 B store are each one contiguous access.
template <typename T, bool kGrouped>
__global__ void __launch_bounds__(256)
    dequant_int4_kernel(const uint8_t* __restrict__ wp, const T* __restrict__ scales, int group,
                        int64_t K, int64_t N, T* __restrict__ out) {
  // Blocks stride over rows, threads over a row's 8-column items: no integer
  // division in the loop (a 64-bit one per item made the pass issue-bound).
  const int items = static_cast<int>(N / 8);
  for (int64_t k = blockIdx.x; k < K; k += gridDim.x) {
    const uint32_t* wrow = reinterpret_cast<const uint32_t*>(wp + k * (N / 2));
    const uint4* srow =
        kGrouped ? reinterpret_cast<const uint4*>(scales + (k / group) * N) : nullptr;
    uint4* orow = reinterpret_cast<uint4*>(out + k * N);
    for (int i = threadIdx.x; i < items; i += blockDim.x) {
      const uint32_t w = __ldg(wrow + i);
      uint4 sc = make_uint4(0u, 0u, 0u, 0u);
      if constexpr (kGrouped) sc = __ldg(srow + i);
      uint32_t o[4];
      dequant8<T, kGrouped>(w, sc.x, sc.y, sc.z, sc.w, o);
      orow[i] = make_uint4(o[0], o[1], o[2], o[3]);
    }
  }
}

int grid_for(int64_t n, int threads) {
  const int64_t want = (n + threads - 1) / threads;
  const int64_t cap = static_cast<int64_t>(num_sms()) * 8;
  return static_cast<int>(want < 1 ? 1 : (want > cap ? cap : want));
}

template <typename Tin, typename Tsc>
cudaError_t quant_group_typed(const void* w, int64_t K, int64_t N, int64_t ldw, int group,
                              uint8_t* packed, void* scales, cudaStream_t s) {
  const int64_t G = (K + group - 1) / group;
  const bool vec = sizeof(Tin) == 2 && (N % 8) == 0 && (ldw % 8) == 0 &&
                   (reinterpret_cast<uintptr_t>(w) & 15) == 0 && (group % 8) == 0 &&
                   group <= 8 * kMaxRowsPerLane;
  if constexpr (sizeof(Tin) == 2) {
    if (vec) {
      dim3 grid(static_cast<unsigned>((N + 255) / 256), static_cast<unsigned>(G));
      quant_int4_group_vec<Tin, Tsc><<<grid, kQuantWarps * 32, 0, s>>>(
          static_cast<const Tin*>(w), K, N, ldw, group, packed, static_cast<Tsc*>(scales));
      return cudaGetLastError();
    }
  }
  {
    dim3 grid(static_cast<unsigned>((N / 2 + 127) / 128), static_cast<unsigned>(G));
    quant_int4_group_generic<Tin, Tsc><<<grid, 128, 0, s>>>(
        static_cast<const Tin*>(w), K, N, ldw, group, packed, static_cast<Tsc*>(scales));
  }
  return cudaGetLastError();
}

template <typename Tin>
cudaError_t quant_group_dispatch_scale(const void* w, int64_t K, int64_t N, int64_t ldw,
                                       int group, uint8_t* packed, void* scales, int sdt,
                                       cudaStream_t s) {
  switch (sdt) {
    case PK_F16: return quant_group_typed<Tin, __half>(w, K, N, ldw, group, packed, scales, s);
    case PK_BF16:
      return quant_group_typed<Tin, __nv_bfloat16>(w, K, N, ldw, group, packed, scales, s);
    case PK_F32: return quant_group_typed<Tin, float>(w, K, N, ldw, group, packed, scales, s);
    default: return cudaErrorInvalidValue;
  }
}

// Fake quantization with the reference's group rule, in the input's dtype:
// quantize.quantize_col (quantize.py:42-60) on every column of w[rows, cols]
// (groups of `group` consecutive rows; group <= 0: the whole column), the
// column walk of rtn_layer (quantize.py:63-68) when w is that layer's fp32
// copy. torch evaluates each step of
//   scale = w.abs().max().clamp_min(1e-12) / qmax
//   out   = clamp(round(w / scale), -qmax, qmax) * scale
// in fp32 and rounds the result to the tensor's dtype; each step here does
// the same, so fp16 columns keep the reference's behaviour where its 1e-12
// floor underflows (a zero scale: inf / NaN quotients, NaN out where w = 0).
// The clamp propagates NaN like torch.clamp. One thread per (column, group);
// consecutive threads take consecutive columns (coalesced rows).
template <typename T>
__global__ void fake_quant_groups_kernel(const T* __restrict__ w, int64_t rows, int64_t cols,
                                         int64_t ldw, int64_t group, float qmax,
                                         T* __restrict__ out, int64_t ldo) {
  const int64_t G = (rows + group - 1) / group;
  const int64_t total = G * cols;
  for (int64_t t = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; t < total;
       t += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t c = t % cols, g = t / cols;
    const int64_t r0 = g * group;
    const int64_t r1 = r0 + group < rows ? r0 + group : rows;
    float m = 0.0f;
    for (int64_t r = r0; r < r1; ++r) m = fmaxf(m, fabsf(to_f32<T>(w[r * ldw + c])));
    const float floor_ = round_through<T>(fmaxf(m, 1e-12f));   // .clamp_min(1e-12)
    const float s = round_through<T>(floor_ / qmax);           // / qmax
    for (int64_t r = r0; r < r1; ++r) {
      const float x = round_through<T>(to_f32<T>(w[r * ldw + c]) / s);  // w / scale
      float q = rintf(x);                                                // torch.round
      q = q < -qmax ? -qmax : (q > qmax ? qmax : q);                     // clamp, NaN kept
      out[r * ldo + c] = from_f32<T>(q * s);                             // * scale
    }
  }
}

}  // namespace

cudaError_t launch_quant_int4_group(const void* w, int w_dtype, int64_t K, int64_t N, int64_t ldw,
                                    int group, uint8_t* packed, void* scales, int scale_dtype,
                                    cudaStream_t s) {
  switch (w_dtype) {
    case PK_F16:
      return quant_group_dispatch_scale<__half>(w, K, N, ldw, group, packed, scales, scale_dtype,
                                                s);
    case PK_BF16:
      return quant_group_dispatch_scale<__nv_bfloat16>(w, K, N, ldw, group, packed, scales,
                                                       scale_dtype, s);
    case PK_F32:
      return quant_group_dispatch_scale<float>(w, K, N, ldw, group, packed, scales, scale_dtype,
                                               s);
    default: return cudaErrorInvalidValue;
  }
}

cudaError_t launch_absmax(const void* x, int dtype, int64_t n, float* out, cudaStream_t s) {
  cudaError_t e = cudaMemsetAsync(out, 0, sizeof(float), s);
  if (e != cudaSuccess) return e;
  const int threads = 512;
  const int grid = grid_for(n / 8 + 1, threads);
  switch (dtype) {
    case PK_F16:
      absmax_kernel<__half><<<grid, threads, 0, s>>>(static_cast<const __half*>(x), n, out);
      break;
    case PK_BF16:
      absmax_kernel<__nv_bfloat16>
          <<<grid, threads, 0, s>>>(static_cast<const __nv_bfloat16*>(x), n, out);
      break;
    case PK_F32:
      absmax_kernel<float><<<grid, threads, 0, s>>>(static_cast<const float*>(x), n, out);
      break;
    default: return cudaErrorInvalidValue;
  }
  return cudaGetLastError();
}

cudaError_t launch_quant_int4_tensor(const void* w, int dtype, int64_t n, float scale,
                                     int8_t* codes, cudaStream_t s) {
  const int threads = 256;
  const int grid = grid_for(n, threads);
  switch (dtype) {
    case PK_F16:
      quant_int4_tensor_kernel<__half>
          <<<grid, threads, 0, s>>>(static_cast<const __half*>(w), n, scale, codes);
      break;
    case PK_BF16:
      quant_int4_tensor_kernel<__nv_bfloat16>
          <<<grid, threads, 0, s>>>(static_cast<const __nv_bfloat16*>(w), n, scale, codes);
      break;
    case PK_F32:
      quant_int4_tensor_kernel<float>
          <<<grid, threads, 0, s>>>(static_cast<const float*>(w), n, scale, codes);
      break;
    default: return cudaErrorInvalidValue;
  }
  return cudaGetLastError();
}

cudaError_t launch_pack_int4(const int8_t* q, int64_t K, int64_t N, uint8_t* p, cudaStream_t s) {
  const int64_t n = K * N;
  const bool vec = (n % 16) == 0 && (reinterpret_cast<uintptr_t>(q) & 15) == 0 &&
                   (reinterpret_cast<uintptr_t>(p) & 7) == 0;
  if (vec) {
    const int64_t n16 = n / 16;
    pack_int4_vec<<<static_cast<unsigned>((n16 + 255) / 256), 256, 0, s>>>(q, n16, p);
  } else {
    const int64_t nb = n / 2;
    pack_int4_scalar<<<static_cast<unsigned>((nb + 255) / 256), 256, 0, s>>>(q, nb, p);
  }
  return cudaGetLastError();
}

cudaError_t launch_unpack_int4(const uint8_t* p, int64_t K, int64_t N, int8_t* q,
                               cudaStream_t s) {
  const int64_t nb = K * N / 2;
  unpack_int4_kernel<<<static_cast<unsigned>((nb + 255) / 256), 256, 0, s>>>(p, nb, q);
  return cudaGetLastError();
}

cudaError_t launch_fp8_quantize_device(const void* x, int dtype, int64_t n, float* amax,
                                       float* scale, uint8_t* y, cudaStream_t s) {
  cudaError_t e = launch_absmax(x, dtype, n, amax, s);
  if (e != cudaSuccess) return e;
  const int threads = 256;
  const int grid = grid_for(n / 8 + 1, threads);
  switch (dtype) {
    case PK_F16:
      fp8_quantize_dev_kernel<__half>
          <<<grid, threads, 0, s>>>(static_cast<const __half*>(x), n, amax, scale, y);
      break;
    case PK_BF16:
      fp8_quantize_dev_kernel<__nv_bfloat16>
          <<<grid, threads, 0, s>>>(static_cast<const __nv_bfloat16*>(x), n, amax, scale, y);
      break;
    case PK_F32:
      fp8_quantize_dev_kernel<float>
          <<<grid, threads, 0, s>>>(static_cast<const float*>(x), n, amax, scale, y);
      break;
    default: return cudaErrorInvalidValue;
  }
  return cudaGetLastError();
}

cudaError_t launch_fp8_quantize(const void* x, int dtype, int64_t n, float scale, uint8_t* y,
                                cudaStream_t s) {
  const int threads = 256;
  const int grid = grid_for(n, threads);
  switch (dtype) {
    case PK_F16:
      fp8_quantize_kernel<__half>
          <<<grid, threads, 0, s>>>(static_cast<const __half*>(x), n, scale, y);
      break;
    case PK_BF16:
      fp8_quantize_kernel<__nv_bfloat16>
          <<<grid, threads, 0, s>>>(static_cast<const __nv_bfloat16*>(x), n, scale, y);
      break;
    case PK_F32:
      fp8_quantize_kernel<float><<<grid, threads, 0, s>>>(static_cast<const float*>(x), n, scale, y);
      break;
    default: return cudaErrorInvalidValue;
  }
  return cudaGetLastError();
}

cudaError_t launch_dequant_int4(const uint8_t* wp, const void* scales, int group, int dtype,
                                int64_t K, int64_t N, void* out, cudaStream_t s) {
  if (N % 8 != 0) return cudaErrorInvalidValue;
  const int threads = 256;
  const int64_t cap = static_cast<int64_t>(num_sms()) * 8;
  const int grid = static_cast<int>(K < cap ? K : cap);
  const bool g = scales != nullptr;
  if (dtype == PK_BF16) {
    auto sp = static_cast<const __nv_bfloat16*>(scales);
    auto op = static_cast<__nv_bfloat16*>(out);
    if (g) dequant_int4_kernel<__nv_bfloat16, true><<<grid, threads, 0, s>>>(wp, sp, group, K, N, op);
    else dequant_int4_kernel<__nv_bfloat16, false><<<grid, threads, 0, s>>>(wp, sp, group, K, N, op);
  } else if (dtype == PK_F16) {
    auto sp = static_cast<const __half*>(scales);
    auto op = static_cast<__half*>(out);
    if (g) dequant_int4_kernel<__half, true><<<grid, threads, 0, s>>>(wp, sp, group, K, N, op);
    else dequant_int4_kernel<__half, false><<<grid, threads, 0, s>>>(wp, sp, group, K, N, op);
  } else {
    return cudaErrorInvalidValue;
  }
  return cudaGetLastError();
}

}  // namespace pk

namespace pk {

cudaError_t launch_fake_quant_groups(const void* w, int dtype, int64_t rows, int64_t cols,
                                     int64_t ldw, int64_t group, int bits, void* out, int64_t ldo,
                                     cudaStream_t s) {
  if (group <= 0 || group > rows) group = rows;
  const float qmax = static_cast<float>((1ll << (bits - 1)) - 1);
  const int64_t total = ((rows + group - 1) / group) * cols;
  const int threads = 256;
  int64_t blocks = (total + threads - 1) / threads;
  if (blocks > 65535ll * 16) blocks = 65535ll * 16;
  const dim3 grid(static_cast<unsigned>(blocks));
  switch (dtype) {
    case PK_F32:
      fake_quant_groups_kernel<float><<<grid, threads, 0, s>>>(
          static_cast<const float*>(w), rows, cols, ldw, group, qmax, static_cast<float*>(out), ldo);
      break;
    case PK_F16:
      fake_quant_groups_kernel<__half><<<grid, threads, 0, s>>>(
          static_cast<const __half*>(w), rows, cols, ldw, group, qmax, static_cast<__half*>(out),
          ldo);
      break;
    case PK_BF16:
      fake_quant_groups_kernel<__nv_bfloat16><<<grid, threads, 0, s>>>(
          static_cast<const __nv_bfloat16*>(w), rows, cols, ldw, group, qmax,
          static_cast<__nv_bfloat16*>(out), ldo);
      break;
    default:
      return cudaErrorInvalidValue;
  }
  return cudaGetLastError();
}

}  // namespace pk
