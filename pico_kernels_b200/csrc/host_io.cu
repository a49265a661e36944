// Row copies between page-locked host memory and device buffers, done by a
// kernel instead of the copy engines.
//
// pk_w4a16_gemm_host moves a few KB per call at decode sizes (A [1, 4096]
// bf16 in, y [1, 4096] fp32 out). A cudaMemcpyAsync of that size costs ~9 us
// of stream time on B200 (copy-engine scheduling), more than the GEMM. Page-
// locked host memory is mapped into the device's address space (unified
// addressing; the device pointer comes from cudaHostGetDevicePointer), so a
// small kernel reads or writes it directly over the host link, and chains
// with the GEMM kernels through programmatic dependent launch: it waits for
// the previous kernel before touching memory and lets the next one start
// its prologue early.
#include "pk_common.cuh"

namespace pk {
namespace {

constexpr int kThreads = 256;

// dst rows (pitch dst_pitch bytes) = src rows (pitch src_pitch), row_bytes
// each. `vec`: every address, pitch and row_bytes is a multiple of 16.
__global__ void __launch_bounds__(kThreads)
    copy_rows_kernel(const uint8_t* __restrict__ src, int64_t src_pitch,
                     uint8_t* __restrict__ dst, int64_t dst_pitch, int64_t row_bytes,
                     int64_t rows, int vec) {
  griddep_launch_dependents();
  griddep_wait();
  const int64_t stride = static_cast<int64_t>(gridDim.x) * kThreads;
  const int64_t t0 = static_cast<int64_t>(blockIdx.x) * kThreads + threadIdx.x;
  if (vec) {
    const int64_t per_row = row_bytes / 16;
    const int64_t total = per_row * rows;
    for (int64_t i = t0; i < total; i += stride) {
      const int64_t r = i / per_row, c = i - r * per_row;
      const uint4 v = *reinterpret_cast<const uint4*>(src + r * src_pitch + c * 16);
      *reinterpret_cast<uint4*>(dst + r * dst_pitch + c * 16) = v;
    }
  } else {
    const int64_t total = row_bytes * rows;
    for (int64_t i = t0; i < total; i += stride) {
      const int64_t r = i / row_bytes, c = i - r * row_bytes;
      dst[r * dst_pitch + c] = src[r * src_pitch + c];
    }
  }
}

}  // namespace

cudaError_t launch_copy_rows(const void* src, int64_t src_pitch, void* dst, int64_t dst_pitch,
                             int64_t row_bytes, int64_t rows, cudaStream_t s) {
  if (rows <= 0 || row_bytes <= 0) return cudaSuccess;
  const auto a16 = [](uint64_t v) { return (v & 15u) == 0; };
  const int vec = a16(reinterpret_cast<uintptr_t>(src)) && a16(reinterpret_cast<uintptr_t>(dst)) &&
                  a16(static_cast<uint64_t>(src_pitch)) && a16(static_cast<uint64_t>(dst_pitch)) &&
                  a16(static_cast<uint64_t>(row_bytes));
  const int64_t items = vec ? (row_bytes / 16) * rows : row_bytes * rows;
  int64_t blocks = (items + kThreads - 1) / kThreads;
  const int64_t cap = 4ll * num_sms();
  if (blocks > cap) blocks = cap;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(blocks));
  cfg.blockDim = dim3(kThreads);
  cfg.stream = s;
  cudaLaunchAttribute attr;
  attr.id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr.val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = &attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, copy_rows_kernel, static_cast<const uint8_t*>(src), src_pitch,
                            static_cast<uint8_t*>(dst), dst_pitch, row_bytes, rows, vec);
}

}  // namespace pk
