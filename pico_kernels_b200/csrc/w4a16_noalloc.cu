// pk_w4a16_gemm_noalloc: the decode W4A16 GEMM for callers that may not
// allocate device memory.
//
// Some callers cannot call cudaMalloc: an inference runtime that plans every
// byte of device memory itself and forbids libraries from allocating, or a
// latency-critical decode loop where cudaMalloc's implicit synchronization is
// not acceptable. pk_w4a16_gemm asks them for a split-K workspace; this entry
// point instead reduces the K splits through scratch memory that the library
// owns statically: a file-scope __device__ array that every GPU loading the
// library keeps until the process exits.
//
// Contract:
//   * decode shapes only (what pk_w4a16_gemm runs on its decode path: M <= 32,
//     N % 128 == 0, K % 128 == 0, group 128 or a scalar scale);
//   * the kernel is always the tensor-core decode kernel reducing its K
//     splits through the scratch (never the GEMV that pk_w4a16_gemm picks at
//     M = 1): its result equals pk_w4a16_gemm's with the same explicit split_k
//     bit for bit, and pk_w4a16_gemm's automatic route within the W4A16
//     tolerance;
//   * the reduction scratch a call needs -- tiles * split * M * 128 fp32
//     partials -- must fit kNoAllocPartialBytes (4 MiB) and the tile count
//     kNoAllocMaxTiles. With split_k = 0 the automatic split is lowered until
//     it fits (down to 1, which needs no scratch); an explicit split_k that
//     does not fit fails with PK_ERR_WORKSPACE and launches nothing;
//   * the first call on each device looks up the array's device address
//     (cudaGetSymbolAddress, with that device current); make that first call
//     before any stream capture;
//   * every call on a device shares the one array, which keeps the previous
//     call's contents: each call clears the arrival counters it uses (an
//     asynchronous memset on the caller's stream), and calls whose kernels
//     overlap on the GPU (different streams, no ordering) race on the scratch;
//   * nothing here calls cudaMalloc, cudaFree or an allocating library routine.
#include <mutex>

#include "pk_internal.h"

namespace pk {
namespace {

constexpr size_t kNoAllocPartialBytes = size_t(4) << 20;  // 4 MiB of fp32 partials
constexpr int64_t kNoAllocMaxTiles = 4096;                // 128-column tiles: N <= 524288
constexpr size_t kNoAllocSemBytes = kNoAllocMaxTiles * sizeof(unsigned);

// The scratch: arrival counters first, then the partials.
static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocSemBytes + kNoAllocPartialBytes];

constexpr int kMaxDevices = 64;
void* g_scratch_ptr[kMaxDevices] = {};
std::mutex g_scratch_mu;

// Device address of the scratch array on the current device (looked up once
// per device). Returns nullptr and sets *err on failure.
void* scratch_address(cudaError_t* err) {
  int dev = -1;
  *err = cudaGetDevice(&dev);
  if (*err != cudaSuccess) return nullptr;
  if (dev < 0 || dev >= kMaxDevices) {
    *err = cudaErrorInvalidDevice;
    return nullptr;
  }
  std::lock_guard<std::mutex> lk(g_scratch_mu);
  if (g_scratch_ptr[dev] == nullptr) {
    void* p = nullptr;
    *err = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (*err != cudaSuccess) return nullptr;
    g_scratch_ptr[dev] = p;
  }
  return g_scratch_ptr[dev];
}

}  // namespace
}  // namespace pk

using namespace pk;

extern "C" PK_API int pk_w4a16_gemm_noalloc(const void* a, int a_dtype, int64_t lda,
                                             const uint8_t* wp, const void* scales,
                                             float scalar_scale, int group_size, int64_t M,
                                             int64_t N, int64_t K, void* out, int out_dtype,
                                             int64_t ldo, int split_k, void* stream) {
  auto fail = [](int code, const char* msg) {
    set_error_message(msg);
    return code;
  };
  if (!a || !wp || !out) return fail(PK_ERR_SHAPE, "null pointer");
  if (M <= 0 || N <= 0 || K <= 0 || lda < K || ldo < N)
    return fail(PK_ERR_SHAPE, "invalid shape or leading dimension");
  if (a_dtype != PK_F16 && a_dtype != PK_BF16) return fail(PK_ERR_DTYPE, "A must be f16 or bf16");
  if (out_dtype != PK_F32 && out_dtype != PK_BF16)
    return fail(PK_ERR_DTYPE, "output must be f32 or bf16");
  if (split_k < 0) return fail(PK_ERR_SHAPE, "split_k must be >= 0");
  if (!decode_supported(M, N, K, group_size, scales, lda, a))
    return fail(PK_ERR_UNSUPPORTED,
                "no-alloc entry point covers decode shapes only (M <= 32, N % 128 == 0, "
                "K % 128 == 0, group 128 or scalar scale, 16-byte aligned A)");
  int split = split_k > 0 ? split_k : decode_pick_split(M, N, K);
  if (split > K / 128) split = static_cast<int>(K / 128);
  const int64_t tiles = N / 128;
  const size_t per_split = static_cast<size_t>(tiles) * M * 128 * sizeof(float);
  if (split_k == 0 && split > 1) {
    // The automatic split shrinks to what the scratch holds (down to no split,
    // which needs none); only a split the caller asked for is rejected.
    const int64_t fit = tiles > kNoAllocMaxTiles ? 1 : static_cast<int64_t>(kNoAllocPartialBytes / per_split);
    if (fit < split) split = fit < 1 ? 1 : static_cast<int>(fit);
  }
  const size_t partial_bytes = per_split * split;
  if (split > 1 && (tiles > kNoAllocMaxTiles || partial_bytes > kNoAllocPartialBytes))
    return fail(PK_ERR_WORKSPACE,
                "request exceeds the static split-K scratch (4 MiB of partials, 4096 tiles); "
                "lower split_k or use pk_w4a16_gemm with a workspace");

  cudaStream_t s = static_cast<cudaStream_t>(stream);
  DecodeArgs p{};
  p.a = a;
  p.lda = lda;
  p.wp = wp;
  p.scales = scales;
  p.scalar_scale = scales ? 1.0f : scalar_scale;
  p.M = M;
  p.N = N;
  p.K = K;
  p.out = out;
  p.out_dtype = out_dtype;
  p.ldo = ldo;
  p.a_dtype = a_dtype;
  p.split = split;
  p.status = device_status_ptr();
  if (split > 1) {
    cudaError_t err = cudaSuccess;
    void* scratch = scratch_address(&err);
    if (scratch == nullptr) return fail(PK_ERR_CUDA, cudaGetErrorString(err));
    // arrival counters must start at zero; the array keeps the last call's contents
    err = cudaMemsetAsync(scratch, 0, static_cast<size_t>(tiles) * sizeof(unsigned), s);
    if (err != cudaSuccess) return fail(PK_ERR_CUDA, cudaGetErrorString(err));
    p.sems = static_cast<unsigned*>(scratch);
    p.partials =
        reinterpret_cast<float*>(static_cast<unsigned char*>(scratch) + kNoAllocSemBytes);
    p.force_workspace = true;
  }
  const char* why = "";
  cudaError_t e = launch_w4a16_decode(p, s, &why);
  if (e == cudaErrorInvalidValue && why[0] != '\0') return fail(PK_ERR_ALIGN, why);
  if (e != cudaSuccess) return fail(PK_ERR_CUDA, cudaGetErrorString(e));
  set_error_message("");
  return PK_OK;
}
