// W4A16 GEMM on CUDA cores for shapes the tensor-core kernels do not take
// (ragged M/N/K, group sizes other than 128, unaligned operands). Dequantizes
// in fp32 (q * s exactly), accumulates in fp32. Correct for any shape with an
// even N; not a performance path.
#include "pk_common.cuh"

namespace pk {
namespace {

template <typename T>
__device__ __forceinline__ float ld_f32(const T* p, int64_t i);
template <>
__device__ __forceinline__ float ld_f32<__half>(const __half* p, int64_t i) {
  return __half2float(p[i]);
}
template <>
__device__ __forceinline__ float ld_f32<__nv_bfloat16>(const __nv_bfloat16* p, int64_t i) {
  return __bfloat162float(p[i]);
}

__device__ __forceinline__ int sext4(int v) { return v >= 8 ? v - 16 : v; }

template <typename T>
__global__ void w4a16_simt_kernel(const T* __restrict__ a, int64_t lda,
                                  const uint8_t* __restrict__ wp, const T* __restrict__ scales,
                                  float scalar_scale, int group, int64_t M, int64_t N, int64_t K,
                                  void* __restrict__ out, int out_dtype, int64_t ldo) {
  const int64_t j = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;  // byte column
  const int64_t m = blockIdx.y;
  if (2 * j >= N || m >= M) return;
  const int64_t ldp = N >> 1;
  float acc0 = 0.0f, acc1 = 0.0f;
  for (int64_t k = 0; k < K; ++k) {
    const int b = wp[k * ldp + j];
    float w0 = static_cast<float>(sext4(b & 0xF));
    float w1 = static_cast<float>(sext4(b >> 4));
    if (scales != nullptr) {
      const int64_t g = k / group;
      w0 *= ld_f32<T>(scales, g * N + 2 * j);
      w1 *= ld_f32<T>(scales, g * N + 2 * j + 1);
    }
    const float av = ld_f32<T>(a, m * lda + k);
    acc0 = fmaf(av, w0, acc0);
    acc1 = fmaf(av, w1, acc1);
  }
  acc0 *= scalar_scale;
  acc1 *= scalar_scale;
  if (out_dtype == PK_BF16) {
    auto* o = static_cast<__nv_bfloat16*>(out);
    o[m * ldo + 2 * j] = __float2bfloat16_rn(acc0);
    o[m * ldo + 2 * j + 1] = __float2bfloat16_rn(acc1);
  } else {
    auto* o = static_cast<float*>(out);
    o[m * ldo + 2 * j] = acc0;
    o[m * ldo + 2 * j + 1] = acc1;
  }
}

}  // namespace

cudaError_t launch_w4a16_simt(const void* a, int a_dtype, int64_t lda, const uint8_t* wp,
                              const void* scales, float scalar_scale, int group, int64_t M,
                              int64_t N, int64_t K, void* out, int out_dtype, int64_t ldo,
                              cudaStream_t s) {
  dim3 grid(static_cast<unsigned>((N / 2 + 127) / 128), static_cast<unsigned>(M));
  if (a_dtype == PK_BF16) {
    w4a16_simt_kernel<__nv_bfloat16><<<grid, 128, 0, s>>>(
        static_cast<const __nv_bfloat16*>(a), lda, wp, static_cast<const __nv_bfloat16*>(scales),
        scalar_scale, group, M, N, K, out, out_dtype, ldo);
  } else {
    w4a16_simt_kernel<__half><<<grid, 128, 0, s>>>(
        static_cast<const __half*>(a), lda, wp, static_cast<const __half*>(scales), scalar_scale,
        group, M, N, K, out, out_dtype, ldo);
  }
  return cudaGetLastError();
}

}  // namespace pk
