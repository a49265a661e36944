// GPTQ producer of packed int4 weights (quantize.py:71-115, act_order=False),
// emitting codes and group scales directly in the W4A16 GEMM's layout.
//
// Working matrix: Wt[K = in, N = out] fp32 (the layer's weight transposed),
// updated in place. The reference walks the input features j in order:
// quantize the column, err = w - q, and subtract outer(err, ratio_j) with
// ratio_j[k] = Hinv[j, k] / Hinv[j, j] from every later feature k
// (quantize.py:99-104). Per group of `group` consecutive features:
//
//   gptq_group_kernel     one thread per output n holds the group's features
//                         in shared memory: group scale from the current
//                         weights (max|w| clamped at 1e-12, / 7), then per
//                         feature: code, error, and the update of the
//                         group's later features, in the reference's order;
//                         codes are written packed (pack_int4_n layout),
//                         scales rounded to the scale dtype, errors kept;
//   gptq_trailing_kernel  every later feature k >= group end receives the
//                         group's updates, applied one feature j at a time in
//                         increasing j.
//
// Each update is a product and a difference rounded separately (no fused
// multiply-add), as torch computes `wq -= torch.outer(err, ratio)`, so given
// the same Hinv the codes and scales equal the sequential restatement bit for
// bit. The work is O(K^2 N) like the reference's loop; it is an offline step.
#include "pk_common.cuh"

namespace pk {
namespace {

constexpr int kGptqMaxGroup = 128;
constexpr int kGptqThreads = 64;     // outputs per block of the group kernel
constexpr int kTrailTN = 32;         // trailing tile: 32 outputs x 64 features
constexpr int kTrailTK = 64;

template <typename S>
__device__ __forceinline__ S to_scale(float v);
template <>
__device__ __forceinline__ float to_scale<float>(float v) { return v; }
template <>
__device__ __forceinline__ __half to_scale<__half>(float v) { return __float2half_rn(v); }
template <>
__device__ __forceinline__ __nv_bfloat16 to_scale<__nv_bfloat16>(float v) {
  return __float2bfloat16_rn(v);
}

// ratio_j[k] = Hinv[j, k] / Hinv[j, j] (quantize.py:102), IEEE division
__device__ __forceinline__ float gptq_ratio(const float* h_inv, int64_t K, int64_t j, int64_t k) {
  return __fdiv_rn(h_inv[j * K + k], h_inv[j * K + j]);
}

template <typename S>
__global__ void __launch_bounds__(kGptqThreads)
    gptq_group_kernel(const float* __restrict__ wt, int64_t K, int64_t N, int64_t j0, int gb,
                      const float* __restrict__ h_inv, float* __restrict__ err,
                      uint8_t* __restrict__ packed, S* __restrict__ scales, int64_t g) {
  extern __shared__ float sm[];
  float* ws = sm;                                  // [gb][kGptqThreads]
  float* rs = sm + gb * kGptqThreads;              // [gb][gb], upper triangle used
  const int tid = threadIdx.x;
  for (int idx = tid; idx < gb * gb; idx += kGptqThreads) {
    const int j = idx / gb, k = idx % gb;
    rs[idx] = k > j ? gptq_ratio(h_inv, K, j0 + j, j0 + k) : 0.0f;
  }
  const int64_t n = static_cast<int64_t>(blockIdx.x) * kGptqThreads + tid;
  const bool valid = n < N;
  float amax = 0.0f;
  for (int k = 0; k < gb; ++k) {
    const float v = valid ? wt[(j0 + k) * N + n] : 0.0f;
    ws[k * kGptqThreads + tid] = v;
    amax = fmaxf(amax, fabsf(v));
  }
  __syncthreads();
  // quantize.py:58 over the group's current weights, fp32 division by 7
  const float s = __fdiv_rn(fmaxf(amax, 1e-12f), 7.0f);
  if (valid) scales[g * N + n] = to_scale<S>(s);
  for (int k = 0; k < gb; ++k) {
    const float v = ws[k * kGptqThreads + tid];
    const float qi = fminf(fmaxf(rintf(__fdiv_rn(v, s)), -7.0f), 7.0f);   // quantize.py:59
    const float e = __fsub_rn(v, __fmul_rn(qi, s));                          // quantize.py:101
    if (valid) err[static_cast<int64_t>(k) * N + n] = e;
    const int code = static_cast<int>(qi);
    const int hi = __shfl_down_sync(0xffffffffu, code, 1);
    if (valid && (n & 1) == 0)
      packed[(j0 + k) * (N / 2) + n / 2] = static_cast<uint8_t>((code & 0xF) | ((hi & 0xF) << 4));
    const float* r = rs + k * gb;
    for (int kk = k + 1; kk < gb; ++kk) {
      float* w = ws + kk * kGptqThreads + tid;
      *w = __fsub_rn(*w, __fmul_rn(e, r[kk]));                               // quantize.py:104
    }
  }
}

__global__ void __launch_bounds__(kTrailTN * 8)
    gptq_trailing_kernel(float* __restrict__ wt, int64_t K, int64_t N, int64_t j0, int gb,
                         const float* __restrict__ h_inv, const float* __restrict__ err) {
  __shared__ float es[kGptqMaxGroup][kTrailTN];
  __shared__ float rs[kGptqMaxGroup][kTrailTK];
  const int tx = threadIdx.x, ty = threadIdx.y;
  const int64_t n0 = static_cast<int64_t>(blockIdx.x) * kTrailTN;
  const int64_t k0 = j0 + gb + static_cast<int64_t>(blockIdx.y) * kTrailTK;
  const int t = ty * kTrailTN + tx;
  for (int idx = t; idx < gb * kTrailTN; idx += kTrailTN * 8) {
    const int j = idx / kTrailTN, c = idx % kTrailTN;
    es[j][c] = n0 + c < N ? err[static_cast<int64_t>(j) * N + n0 + c] : 0.0f;
  }
  for (int idx = t; idx < gb * kTrailTK; idx += kTrailTN * 8) {
    const int j = idx / kTrailTK, r = idx % kTrailTK;
    rs[j][r] = k0 + r < K ? gptq_ratio(h_inv, K, j0 + j, k0 + r) : 0.0f;
  }
  __syncthreads();
  const int64_t n = n0 + tx;
  if (n >= N) return;
  float acc[kTrailTK / 8];
#pragma unroll
  for (int i = 0; i < kTrailTK / 8; ++i) {
    const int64_t k = k0 + ty + 8 * i;
    acc[i] = k < K ? wt[k * N + n] : 0.0f;
  }
  for (int j = 0; j < gb; ++j) {
    const float e = es[j][tx];
#pragma unroll
    for (int i = 0; i < kTrailTK / 8; ++i) acc[i] = __fsub_rn(acc[i], __fmul_rn(e, rs[j][ty + 8 * i]));
  }
#pragma unroll
  for (int i = 0; i < kTrailTK / 8; ++i) {
    const int64_t k = k0 + ty + 8 * i;
    if (k < K) wt[k * N + n] = acc[i];
  }
}

// ---------------------------------------------------------------------------
// The reference's own rule (gptq_layer's quantize_col, quantize.py:100): each
// input feature j is one column of outputs, quantized with scales over groups
// of `out_group` consecutive OUTPUTS (<= 0: the whole column), and replaced by
// its fake-quant values. One CTA walks a block of kRefBlock features in order:
// per feature, the group absmax (shared memory, one warp per group), the
// fp32 scale max.clamp_min(1e-12) / qmax, then per output its code, fake
// value q * s and error (quantize.py:58-59, 101), and the update of the
// block's later features (quantize.py:102-104). The trailing kernel above
// applies the block's updates to the features after it, in feature order.
// ---------------------------------------------------------------------------
constexpr int kRefThreads = 1024;
constexpr int kRefBlock = 32;
constexpr int kRefMaxOut = 16384;

__global__ void __launch_bounds__(kRefThreads)
    gptq_ref_block_kernel(float* __restrict__ wt, int64_t K, int64_t N, int64_t j0, int gb,
                          const float* __restrict__ h_inv, float* __restrict__ err,
                          int64_t out_group, float qmax) {
  extern __shared__ float sm[];
  float* absb = sm;       // [N] |w| of the current feature
  float* sc = sm + N;     // [G] its group scales
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int64_t G = (N + out_group - 1) / out_group;
  for (int k = 0; k < gb; ++k) {
    const int64_t j = j0 + k;
    float* row = wt + j * N;
    for (int64_t n = tid; n < N; n += kRefThreads) absb[n] = fabsf(row[n]);
    __syncthreads();
    for (int64_t g = warp; g < G; g += kRefThreads / 32) {
      const int64_t a = g * out_group, b = a + out_group < N ? a + out_group : N;
      float m = 0.0f;
      for (int64_t n = a + lane; n < b; n += 32) m = fmaxf(m, absb[n]);
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
      if (lane == 0) sc[g] = __fdiv_rn(fmaxf(m, 1e-12f), qmax);   // quantize.py:58
    }
    __syncthreads();
    const float hjj = h_inv[j * K + j];
    for (int64_t n = tid; n < N; n += kRefThreads) {
      const float v = row[n];
      const float s = sc[n / out_group];
      float q = rintf(__fdiv_rn(v, s));                                // quantize.py:59
      q = q < -qmax ? -qmax : (q > qmax ? qmax : q);
      const float fq = __fmul_rn(q, s);
      const float e = __fsub_rn(v, fq);                                // quantize.py:101
      row[n] = fq;                                                     // quantize.py:104
      err[static_cast<int64_t>(k) * N + n] = e;
      for (int kk = k + 1; kk < gb; ++kk) {
        const float r = __fdiv_rn(h_inv[j * K + j0 + kk], hjj);        // quantize.py:102
        float* x = wt + (j0 + kk) * N + n;
        *x = __fsub_rn(*x, __fmul_rn(e, r));                           // quantize.py:103
      }
    }
    __syncthreads();  // absb and sc are rewritten for the next feature
  }
}

template <typename S>
cudaError_t gptq_run(float* wt, const float* h_inv, int64_t K, int64_t N, int group,
                     uint8_t* packed, S* scales, float* err, cudaStream_t s) {
  const size_t smem = (static_cast<size_t>(group) * kGptqThreads +
                       static_cast<size_t>(group) * group) * sizeof(float);
  cudaError_t e = cudaFuncSetAttribute(gptq_group_kernel<S>,
                                       cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       static_cast<int>(smem));
  if (e != cudaSuccess) return e;
  const unsigned gx = static_cast<unsigned>((N + kGptqThreads - 1) / kGptqThreads);
  const unsigned tx = static_cast<unsigned>((N + kTrailTN - 1) / kTrailTN);
  for (int64_t j0 = 0, g = 0; j0 < K; j0 += group, ++g) {
    const int gb = static_cast<int>(K - j0 < group ? K - j0 : group);
    gptq_group_kernel<S><<<gx, kGptqThreads, smem, s>>>(wt, K, N, j0, gb, h_inv, err, packed,
                                                        scales, g);
    const int64_t rest = K - (j0 + gb);
    if (rest > 0) {
      const dim3 grid(tx, static_cast<unsigned>((rest + kTrailTK - 1) / kTrailTK));
      gptq_trailing_kernel<<<grid, dim3(kTrailTN, 8), 0, s>>>(wt, K, N, j0, gb, h_inv, err);
    }
    e = cudaGetLastError();
    if (e != cudaSuccess) return e;
  }
  return cudaSuccess;
}

}  // namespace

int gptq_max_group() { return kGptqMaxGroup; }
int gptq_ref_max_out() { return kRefMaxOut; }

cudaError_t launch_gptq_ref(float* wt, const float* h_inv, int64_t K, int64_t N, int out_group,
                            int bits, float* err, cudaStream_t s) {
  const int64_t og = out_group <= 0 || out_group > N ? N : out_group;
  const int64_t G = (N + og - 1) / og;
  const size_t smem = static_cast<size_t>(N + G) * sizeof(float);
  cudaError_t e = cudaFuncSetAttribute(gptq_ref_block_kernel,
                                       cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       static_cast<int>(smem));
  if (e != cudaSuccess) return e;
  const float qmax = static_cast<float>((1ll << (bits - 1)) - 1);
  const unsigned tx = static_cast<unsigned>((N + kTrailTN - 1) / kTrailTN);
  for (int64_t j0 = 0; j0 < K; j0 += kRefBlock) {
    const int gb = static_cast<int>(K - j0 < kRefBlock ? K - j0 : kRefBlock);
    gptq_ref_block_kernel<<<1, kRefThreads, smem, s>>>(wt, K, N, j0, gb, h_inv, err, og, qmax);
    const int64_t rest = K - (j0 + gb);
    if (rest > 0) {
      const dim3 grid(tx, static_cast<unsigned>((rest + kTrailTK - 1) / kTrailTK));
      gptq_trailing_kernel<<<grid, dim3(kTrailTN, 8), 0, s>>>(wt, K, N, j0, gb, h_inv, err);
    }
    e = cudaGetLastError();
    if (e != cudaSuccess) return e;
  }
  return cudaSuccess;
}

cudaError_t launch_gptq_int4(float* wt, const float* h_inv, int64_t K, int64_t N, int group,
                             uint8_t* packed, void* scales, int scale_dtype, float* err,
                             cudaStream_t s) {
  switch (scale_dtype) {
    case PK_F32:
      return gptq_run<float>(wt, h_inv, K, N, group, packed, static_cast<float*>(scales), err, s);
    case PK_F16:
      return gptq_run<__half>(wt, h_inv, K, N, group, packed, static_cast<__half*>(scales), err, s);
    case PK_BF16:
      return gptq_run<__nv_bfloat16>(wt, h_inv, K, N, group, packed,
                                     static_cast<__nv_bfloat16*>(scales), err, s);
    default: return cudaErrorInvalidValue;
  }
}

}  // namespace pk
