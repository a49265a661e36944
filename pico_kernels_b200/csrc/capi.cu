// extern "C" entry points of libpico_b200.so (declared in include/pico_b200.h):
// argument validation, path selection, tensor-map encoding, the device status
// word and the per-thread error message.
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <utility>
#include <vector>

#include "pk_internal.h"

namespace pk {
namespace {

thread_local char g_msg[512] = "";

int fail(int code, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_msg, sizeof(g_msg), fmt, ap);
  va_end(ap);
  return code;
}

int cuda_fail(cudaError_t e, const char* what) {
  return fail(PK_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
}

void ok() { g_msg[0] = '\0'; }

// First error code recorded by a device-side bounded wait, and where; then
// the wait limit in SM cycles as a 64-bit word (0: the built-in default).
__device__ __align__(8) int g_device_status[4];

constexpr int kMaxDevices = 64;
int* g_status_ptr[kMaxDevices] = {};
int g_sms[kMaxDevices] = {};
std::mutex g_mu;

int current_device() {
  int d = 0;
  if (cudaGetDevice(&d) != cudaSuccess || d < 0 || d >= kMaxDevices) return -1;
  return d;
}

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                  const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                  const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                  CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  });
  return fn;
}

cudaStream_t as_stream(void* s) { return static_cast<cudaStream_t>(s); }

bool is16(int dt) { return dt == PK_F16 || dt == PK_BF16; }

}  // namespace

void set_error_message(const char* msg) {
  std::strncpy(g_msg, msg, sizeof(g_msg) - 1);
  g_msg[sizeof(g_msg) - 1] = '\0';
}

int* device_status_ptr() {
  const int d = current_device();
  if (d < 0) return nullptr;
  std::lock_guard<std::mutex> lk(g_mu);
  if (g_status_ptr[d] == nullptr) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_device_status) != cudaSuccess) return nullptr;
    g_status_ptr[d] = static_cast<int*>(p);
  }
  return g_status_ptr[d];
}

int num_sms() {
  const int d = current_device();
  if (d < 0) return 148;
  if (g_sms[d] == 0) {
    int v = 0;
    if (cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, d) != cudaSuccess || v <= 0)
      v = 148;
    g_sms[d] = v;
  }
  return g_sms[d];
}

bool prefill_dequant_once(int64_t M, int64_t N, int64_t K) {
  // Measured at 4096 x 11008 x 4096: fused 518 us vs dense bf16 329 us plus a
  // ~19 us dequantize pass. The fused kernel's extra cost grows with M (one
  // dequantization per 128-row M tile); from M = 1024 the single pass wins.
  return M >= 1024 && N % 32 == 0 && K * N <= (1ll << 34);
}

size_t prefill_workspace_bytes(int64_t N, int64_t K) {
  // 16-bit B[K, N] after the counter region, which stays zero for the
  // split-K kernels sharing the workspace
  return kCounterBytes + static_cast<size_t>(K) * static_cast<size_t>(N) * 2;
}

namespace {

// Encoded maps of recent calls, per host thread: a decode loop calls the same
// layers with the same buffers, and a map depends only on these fields (the
// address, the tensor's shape and stride, the box and the swizzle), so equal
// fields give an equal map and the driver call can be skipped.
struct TmapKey {
  uint64_t base, inner, outer, stride;
  uint32_t dtype, box_inner, box_outer, swizzle;
  bool operator==(const TmapKey& o) const {
    return base == o.base && inner == o.inner && outer == o.outer && stride == o.stride &&
           dtype == o.dtype && box_inner == o.box_inner && box_outer == o.box_outer &&
           swizzle == o.swizzle;
  }
};
constexpr int kTmapCache = 32;
struct TmapCache {
  TmapKey key[kTmapCache];
  CUtensorMap map[kTmapCache];
  int used = 0, next = 0;
};
thread_local TmapCache tmap_cache;

}  // namespace

cudaError_t set_max_smem(const void* kernel, int bytes) {
  // kernel -> (bytes, bit per device already set): the attribute persists in
  // the device's context, so later launches skip the runtime call
  static std::mutex mu;
  static std::vector<std::pair<const void*, std::pair<int, uint64_t>>> done;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) dev = -1;
  const uint64_t bit = (dev >= 0 && dev < 64) ? (1ull << dev) : 0;
  {
    std::lock_guard<std::mutex> lock(mu);
    for (auto& d : done)
      if (d.first == kernel && d.second.first >= bytes && (d.second.second & bit) != 0)
        return cudaSuccess;
  }
  const cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
  if (e != cudaSuccess || bit == 0) return e;
  std::lock_guard<std::mutex> lock(mu);
  for (auto& d : done) {
    if (d.first == kernel) {
      if (d.second.first != bytes) d.second = {bytes, 0};
      d.second.second |= bit;
      return e;
    }
  }
  done.push_back({kernel, {bytes, bit}});
  return e;
}

bool encode_tmap_2d(CUtensorMap* map, CUtensorMapDataType dtype, const void* base,
                    uint64_t inner, uint64_t outer, uint64_t row_stride_bytes, uint32_t box_inner,
                    uint32_t box_outer, CUtensorMapSwizzle swizzle, const char** why) {
  const TmapKey key{reinterpret_cast<uint64_t>(base), inner, outer, row_stride_bytes,
                    static_cast<uint32_t>(dtype), box_inner, box_outer,
                    static_cast<uint32_t>(swizzle)};
  TmapCache& c = tmap_cache;
  for (int i = 0; i < c.used; ++i) {
    if (c.key[i] == key) {
      *map = c.map[i];
      return true;
    }
  }
  EncodeTiledFn fn = encode_fn();
  if (fn == nullptr) {
    *why = "cuTensorMapEncodeTiled unavailable";
    return false;
  }
  const cuuint64_t dims[2] = {inner, outer};
  const cuuint64_t strides[1] = {row_stride_bytes};
  const cuuint32_t box[2] = {box_inner, box_outer};
  const cuuint32_t estr[2] = {1, 1};
  const CUresult r = fn(map, dtype, 2, const_cast<void*>(base), dims, strides, box, estr,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle,
                        CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    *why = "cuTensorMapEncodeTiled rejected the operand (alignment or box)";
    return false;
  }
  const int slot = c.used < kTmapCache ? c.used++ : (c.next++ % kTmapCache);
  c.key[slot] = key;
  c.map[slot] = *map;
  return true;
}

}  // namespace pk

using namespace pk;

extern "C" {

int pk_version(void) { return 100; }

const char* pk_last_error_string(void) { return g_msg; }

int pk_device_status(int* code, int* where, int reset) {
  int* p = device_status_ptr();
  if (p == nullptr) return fail(PK_ERR_CUDA, "device status word unavailable");
  cudaError_t e = cudaDeviceSynchronize();
  if (e != cudaSuccess) return cuda_fail(e, "cudaDeviceSynchronize");
  int h[2] = {0, 0};
  e = cudaMemcpy(h, p, sizeof(h), cudaMemcpyDeviceToHost);
  if (e != cudaSuccess) return cuda_fail(e, "read device status");
  if (code) *code = h[0];
  if (where) *where = h[1];
  if (reset) {
    e = cudaMemset(p, 0, sizeof(h));
    if (e != cudaSuccess) return cuda_fail(e, "reset device status");
  }
  ok();
  return PK_OK;
}

int pk_quant_int4_group(const void* w, int w_dtype, int64_t K, int64_t N, int64_t ldw,
                        int group_size, uint8_t* packed, void* scales, int scale_dtype,
                        void* stream) {
  if (!w || !packed || !scales) return fail(PK_ERR_SHAPE, "null pointer");
  if (K <= 0 || N <= 0 || (N % 2) != 0)
    return fail(PK_ERR_SHAPE, "need K > 0 and an even N > 0 (got K=%lld N=%lld)",
                (long long)K, (long long)N);
  if (ldw < N) return fail(PK_ERR_SHAPE, "ldw %lld < N %lld", (long long)ldw, (long long)N);
  if (group_size <= 0) return fail(PK_ERR_SHAPE, "group_size must be positive");
  if ((K + group_size - 1) / group_size > 65535)
    return fail(PK_ERR_SHAPE, "too many groups along K");
  if (w_dtype != PK_F16 && w_dtype != PK_BF16 && w_dtype != PK_F32)
    return fail(PK_ERR_DTYPE, "weight dtype must be f16, bf16 or f32");
  if (scale_dtype != PK_F16 && scale_dtype != PK_BF16 && scale_dtype != PK_F32)
    return fail(PK_ERR_DTYPE, "scale dtype must be f16, bf16 or f32");
  if ((reinterpret_cast<uintptr_t>(packed) & 3) != 0)
    return fail(PK_ERR_ALIGN, "packed output must be 4-byte aligned");
  cudaError_t e = launch_quant_int4_group(w, w_dtype, K, N, ldw, group_size, packed, scales,
                                          scale_dtype, as_stream(stream));
  if (e != cudaSuccess) return cuda_fail(e, "quant_int4_group launch");
  ok();
  return PK_OK;
}

int pk_absmax(const void* x, int dtype, int64_t n, float* absmax_dev, void* stream) {
  if (!x || !absmax_dev || n <= 0) return fail(PK_ERR_SHAPE, "need a non-empty input");
  if (dtype != PK_F16 && dtype != PK_BF16 && dtype != PK_F32)
    return fail(PK_ERR_DTYPE, "absmax dtype must be f16, bf16 or f32");
  cudaError_t e = launch_absmax(x, dtype, n, absmax_dev, as_stream(stream));
  if (e != cudaSuccess) return cuda_fail(e, "absmax launch");
  ok();
  return PK_OK;
}

int pk_quant_int4_tensor(const void* w, int dtype, int64_t n, float scale, int8_t* codes,
                         void* stream) {
  if (!w || !codes || n <= 0) return fail(PK_ERR_SHAPE, "need a non-empty input");
  if (!is16(dtype) && dtype != PK_F32)
    return fail(PK_ERR_DTYPE, "quantize_int4 input must be f16, bf16 or f32");
  cudaError_t e = launch_quant_int4_tensor(w, dtype, n, scale, codes, as_stream(stream));
  if (e != cudaSuccess) return cuda_fail(e, "quant_int4_tensor launch");
  ok();
  return PK_OK;
}

int pk_pack_int4_n(const int8_t* q, int64_t K, int64_t N, uint8_t* packed, void* stream) {
  if (!q || !packed) return fail(PK_ERR_SHAPE, "null pointer");
  if (K <= 0 || N <= 0 || (N % 2) != 0) return fail(PK_ERR_SHAPE, "N must be even");
  cudaError_t e = launch_pack_int4(q, K, N, packed, as_stream(stream));
  if (e != cudaSuccess) return cuda_fail(e, "pack launch");
  ok();
  return PK_OK;
}

int pk_unpack_int4_n(const uint8_t* packed, int64_t K, int64_t N, int8_t* q, void* stream) {
  if (!q || !packed) return fail(PK_ERR_SHAPE, "null pointer");
  if (K <= 0 || N <= 0 || (N % 2) != 0) return fail(PK_ERR_SHAPE, "N must be even");
  cudaError_t e = launch_unpack_int4(packed, K, N, q, as_stream(stream));
  if (e != cudaSuccess) return cuda_fail(e, "unpack launch");
  ok();
  return PK_OK;
}

size_t pk_w4a16_workspace_size(int64_t M, int64_t N, int64_t K, int split_k) {
  if (M <= 0 || N <= 0 || K <= 0) return 0;
  if (prefill_dequant_once(M, N, K) && K % 64 == 0 && N % 64 == 0)
    return prefill_workspace_bytes(N, K);
  const void* aligned = reinterpret_cast<const void*>(16);
  size_t bytes = 0;
  // the GEMV serves the shapes the decode kernel does not take (other group
  // sizes) whatever its preference: size for both
  if (split_k == 0 && gemv_supported(M, N, K, 128, aligned, 8, aligned, aligned))
    bytes = gemv_workspace_bytes(M, N, K);
  if (decode_supported(M, N, K, 128, nullptr, 8, aligned)) {
    const int split = split_k > 0 ? split_k : decode_pick_split(M, N, K);
    const size_t d = decode_workspace_bytes(M, N, K, split);
    if (d > bytes) bytes = d;
  }
  return bytes;
}

int pk_w4a16_gemm(const void* a, int a_dtype, int64_t lda, const uint8_t* wp, const void* scales,
                  float scalar_scale, int group_size, int64_t M, int64_t N, int64_t K, void* out,
                  int out_dtype, int64_t ldo, int split_k, void* workspace,
                  size_t workspace_bytes, void* stream) {
  if (!a || !wp || !out) return fail(PK_ERR_SHAPE, "null pointer");
  if (M <= 0 || N <= 0 || K <= 0 || (N % 2) != 0)
    return fail(PK_ERR_SHAPE, "need M, K > 0 and an even N > 0 (got M=%lld N=%lld K=%lld)",
                (long long)M, (long long)N, (long long)K);
  if (lda < K || ldo < N) return fail(PK_ERR_SHAPE, "leading dimension too small");
  if (!is16(a_dtype)) return fail(PK_ERR_DTYPE, "A must be f16 or bf16");
  if (out_dtype != PK_F32 && out_dtype != PK_BF16)
    return fail(PK_ERR_DTYPE, "output must be f32 or bf16");
  if (scales != nullptr && group_size <= 0) return fail(PK_ERR_SHAPE, "group_size must be > 0");
  if (split_k < 0) return fail(PK_ERR_SHAPE, "split_k must be >= 0");
  cudaStream_t s = as_stream(stream);

  // M = 1 on layers that fit one wave: the CUDA-core GEMV whose K splits
  // reduce inside thread-block clusters (no workspace).
  if (split_k == 0 && gemv_cluster_preferred(M, N, K) &&
      gemv_cluster_supported(M, N, K, group_size, scales, lda, a, wp)) {
    DecodeArgs p{};
    p.a = a;
    p.lda = lda;
    p.wp = wp;
    p.scales = scales;
    p.group = group_size;
    p.scalar_scale = scales ? 1.0f : scalar_scale;
    p.M = M;
    p.N = N;
    p.K = K;
    p.out = out;
    p.out_dtype = out_dtype;
    p.ldo = ldo;
    p.a_dtype = a_dtype;
    p.split = 1;
    p.status = device_status_ptr();
    const char* why = "";
    cudaError_t e = launch_w4a16_gemv_cluster(p, s, &why);
    if (e == cudaErrorInvalidValue && why[0] != '\0') return fail(PK_ERR_ALIGN, "%s", why);
    if (e != cudaSuccess) return cuda_fail(e, "w4a16 cluster gemv launch");
    ok();
    return PK_OK;
  }

  // Other decode shapes where it is faster, with the automatic split: the
  // stream-K CUDA-core GEMV (a weight stream).
  if (split_k == 0 && gemv_supported(M, N, K, group_size, scales, lda, a, wp) &&
      (gemv_preferred(M, N, K) || !decode_supported(M, N, K, group_size, scales, lda, a))) {
    const size_t need = gemv_workspace_bytes(M, N, K);
    bool have_ws = need == 0;
    if (need > 0 && workspace != nullptr) {
      if (workspace_bytes < need)
        return fail(PK_ERR_WORKSPACE, "the GEMV needs %zu workspace bytes, got %zu", need,
                    workspace_bytes);
      if ((reinterpret_cast<uintptr_t>(workspace) & 255) != 0)
        return fail(PK_ERR_ALIGN, "workspace must be 256-byte aligned");
      have_ws = true;
    }
    if (have_ws) {  // without a workspace the tensor-core decode below reduces in clusters
      DecodeArgs p{};
      p.a = a;
      p.lda = lda;
      p.wp = wp;
      p.scales = scales;
      p.group = group_size;
      p.scalar_scale = scales ? 1.0f : scalar_scale;
      p.M = M;
      p.N = N;
      p.K = K;
      p.out = out;
      p.out_dtype = out_dtype;
      p.ldo = ldo;
      p.a_dtype = a_dtype;
      p.split = 1;
      p.status = device_status_ptr();
      if (need > 0) {
        p.sems = ws_counters(workspace);
        p.partials = ws_partials(workspace);
      }
      const char* why = "";
      cudaError_t e = launch_w4a16_gemv(p, s, &why);
      if (e == cudaErrorInvalidValue && why[0] != '\0') return fail(PK_ERR_ALIGN, "%s", why);
      if (e != cudaSuccess) return cuda_fail(e, "w4a16 gemv launch");
      ok();
      return PK_OK;
    }
  }

  if (decode_supported(M, N, K, group_size, scales, lda, a)) {
    DecodeArgs p{};
    p.a = a;
    p.lda = lda;
    p.wp = wp;
    p.scales = scales;
    p.group = group_size;
    p.scalar_scale = scales ? 1.0f : scalar_scale;
    p.M = M;
    p.N = N;
    p.K = K;
    p.out = out;
    p.out_dtype = out_dtype;
    p.ldo = ldo;
    p.a_dtype = a_dtype;
    int split = split_k > 0 ? split_k : decode_pick_split(M, N, K);
    if (split > K / 128) split = static_cast<int>(K / 128);
    p.split = split;
    p.status = device_status_ptr();
    if (split > 1 && workspace != nullptr) {
      const size_t need = decode_workspace_bytes(M, N, K, split);
      if (workspace_bytes < need)
        return fail(PK_ERR_WORKSPACE, "split-K needs %zu workspace bytes, got %zu", need,
                    workspace_bytes);
      if ((reinterpret_cast<uintptr_t>(workspace) & 255) != 0)
        return fail(PK_ERR_ALIGN, "workspace must be 256-byte aligned");
      p.sems = ws_counters(workspace);
      p.partials = ws_partials(workspace);
    }
    if (split > decode_max_cluster_split() && p.partials == nullptr)
      return fail(PK_ERR_WORKSPACE, "split_k > %d needs %zu workspace bytes",
                  decode_max_cluster_split(), decode_workspace_bytes(M, N, K, split));
    const char* why = "";
    cudaError_t e = launch_w4a16_decode(p, s, &why);
    if (e == cudaErrorInvalidValue && why[0] != '\0') {
      const bool ws = std::strstr(why, "workspace") != nullptr;
      return fail(ws ? PK_ERR_WORKSPACE : PK_ERR_ALIGN, "%s", why);
    }
    if (e != cudaSuccess) return cuda_fail(e, "w4a16 decode launch");
    ok();
    return PK_OK;
  }

  // 32 < M <= 256 where it is faster (skinny_preferred): the swap-AB
  // tensor-core kernel dequantizes every weight once, two CTAs per SM.
  if (split_k == 0 && skinny_supported(M, N, K, group_size, scales, lda, a) &&
      (reinterpret_cast<uintptr_t>(wp) & 15) == 0 && skinny_preferred(M, N, K)) {
    DecodeArgs p{};
    p.a = a;
    p.lda = lda;
    p.wp = wp;
    p.scales = scales;
    p.group = group_size;
    p.scalar_scale = scales ? 1.0f : scalar_scale;
    p.M = M;
    p.N = N;
    p.K = K;
    p.out = out;
    p.out_dtype = out_dtype;
    p.ldo = ldo;
    p.a_dtype = a_dtype;
    p.split = 1;
    p.status = device_status_ptr();
    const char* why = "";
    cudaError_t e = launch_w4a16_skinny(p, s, &why);
    if (e == cudaErrorInvalidValue && why[0] != '\0') return fail(PK_ERR_ALIGN, "%s", why);
    if (e != cudaSuccess) return cuda_fail(e, "w4a16 skinny launch");
    ok();
    return PK_OK;
  }

  // Tensor-core prefill path: 64-row K stages, scales on 64-row boundaries.
  const bool prefill_ok = (K % 64) == 0 && (N % 64) == 0 && (lda % 8) == 0 &&
                          (reinterpret_cast<uintptr_t>(a) & 15) == 0 &&
                          (reinterpret_cast<uintptr_t>(wp) & 15) == 0 &&
                          (scales == nullptr || ((group_size % 64) == 0 &&
                                                 (reinterpret_cast<uintptr_t>(scales) & 15) == 0)) &&
                          M < (1ll << 31) && N < (1ll << 31) && K < (1ll << 31);
  // Large M: dequantize the weights once into the workspace and run the dense
  // tensor-core GEMM (the fused kernel dequantizes every B tile again for each
  // 128-row M tile; at M = 4096 that costs more than the one pass).
  if (prefill_ok && prefill_dequant_once(M, N, K) && workspace != nullptr &&
      workspace_bytes >= prefill_workspace_bytes(N, K) &&
      (reinterpret_cast<uintptr_t>(workspace) & 255) == 0) {
    void* bq = ws_partials(workspace);
    cudaError_t e = launch_dequant_int4(wp, scales, group_size, a_dtype, K, N, bq, s);
    if (e != cudaSuccess) return cuda_fail(e, "w4a16 dequant launch");
    GemmArgs g{};
    g.kind = GemmArgs::kDense16;
    g.a = a;
    g.a_dtype = a_dtype;
    g.lda = lda;
    g.b = bq;
    g.ldb = N;
    g.M = M;
    g.N = N;
    g.K = K;
    g.split = 1;
    g.out = out;
    g.out_dtype = out_dtype;
    g.ldc = ldo;
    g.out_scale = scales ? 1.0f : scalar_scale;
    g.status = device_status_ptr();
    const char* why = "";
    e = launch_gemm_tc(g, s, &why);
    if (e == cudaErrorInvalidValue && why[0] != '\0') return fail(PK_ERR_ALIGN, "%s", why);
    if (e != cudaSuccess) return cuda_fail(e, "w4a16 prefill (dense) launch");
    ok();
    return PK_OK;
  }
  if (prefill_ok) {
    GemmArgs g{};
    g.kind = GemmArgs::kW4A16;
    g.a = a;
    g.a_dtype = a_dtype;
    g.lda = lda;
    g.b = wp;
    g.ldb = N / 2;
    g.scales = scales;
    g.group = group_size;
    g.M = M;
    g.N = N;
    g.K = K;
    g.split = 1;
    g.out = out;
    g.out_dtype = out_dtype;
    g.ldc = ldo;
    g.out_scale = scales ? 1.0f : scalar_scale;
    g.status = device_status_ptr();
    const char* why = "";
    cudaError_t e = launch_gemm_tc(g, s, &why);
    if (e == cudaErrorInvalidValue && why[0] != '\0') return fail(PK_ERR_ALIGN, "%s", why);
    if (e != cudaSuccess) return cuda_fail(e, "w4a16 prefill launch");
    ok();
    return PK_OK;
  }

  cudaError_t e = launch_w4a16_simt(a, a_dtype, lda, wp, scales, scalar_scale, group_size, M, N,
                                    K, out, out_dtype, ldo, s);
  if (e != cudaSuccess) return cuda_fail(e, "w4a16 simt launch");
  ok();
  return PK_OK;
}

int pk_w4a16_gemm_host(const void* a_host, int a_dtype, int64_t lda, const uint8_t* wp,
                       const void* scales, float scalar_scale, int group_size, int64_t M,
                       int64_t N, int64_t K, void* y_host, int out_dtype, void* a_dev,
                       void* y_dev, void* workspace, size_t workspace_bytes, void* stream) {
  if (!a_host || !y_host || !a_dev || !y_dev) return fail(PK_ERR_SHAPE, "null pointer");
  if (M <= 0 || N <= 0 || K <= 0 || lda < K)
    return fail(PK_ERR_SHAPE, "need M, N, K > 0 and lda >= K (got M=%lld N=%lld K=%lld lda=%lld)",
                (long long)M, (long long)N, (long long)K, (long long)lda);
  if (!is16(a_dtype)) return fail(PK_ERR_DTYPE, "A must be f16 or bf16");
  if (out_dtype != PK_F32 && out_dtype != PK_BF16)
    return fail(PK_ERR_DTYPE, "output must be f32 or bf16");
  cudaStream_t s = as_stream(stream);
  // Page-locked buffers are mapped into the device's address space: a small
  // kernel moves the rows (chained with the GEMM by programmatic dependent
  // launch; ~9 us less stream time per copy than the copy engines at decode
  // sizes). Pageable buffers have no device mapping and go through
  // cudaMemcpyAsync.
  void* a_map = nullptr;
  void* y_map = nullptr;
  if (cudaHostGetDevicePointer(&a_map, const_cast<void*>(a_host), 0) != cudaSuccess) {
    cudaGetLastError();
    a_map = nullptr;
  }
  if (cudaHostGetDevicePointer(&y_map, y_host, 0) != cudaSuccess) {
    cudaGetLastError();
    y_map = nullptr;
  }
  // (Reading A through its mapping inside the GEMM instead was measured
  // slower: every CTA of the grid then reads its rows across the host link,
  // 32 times the bytes at M = 1 4096^2 for the cluster GEMV; 13.9 vs 12.8 us
  // per call back to back on one box, although it saves a launch; the copy
  // kernel reads them once.)
  const size_t row = static_cast<size_t>(K) * 2;
  cudaError_t e;
  if (a_map != nullptr)
    e = launch_copy_rows(a_map, lda * 2, a_dev, K * 2, K * 2, M, s);
  else if (lda == K)
    e = cudaMemcpyAsync(a_dev, a_host, row * static_cast<size_t>(M), cudaMemcpyHostToDevice, s);
  else
    e = cudaMemcpy2DAsync(a_dev, row, a_host, static_cast<size_t>(lda) * 2, row,
                          static_cast<size_t>(M), cudaMemcpyHostToDevice, s);
  if (e != cudaSuccess) return cuda_fail(e, "copy of A to the device");
  // Shapes the decode kernel supports run on it or on the GEMV, both of
  // which write their output with plain stores: those go straight to the
  // page-locked output through its device mapping, and the copy out is not
  // needed. Other kernels write y_dev.
  const bool direct_out =
      y_map != nullptr && decode_supported(M, N, K, group_size, scales, K, a_dev);
  const int st = pk_w4a16_gemm(a_dev, a_dtype, K, wp, scales, scalar_scale, group_size, M, N, K,
                               direct_out ? y_map : y_dev, out_dtype, N, 0, workspace,
                               workspace_bytes, stream);
  if (st != PK_OK) return st;
  if (direct_out) {
    ok();
    return PK_OK;
  }
  const int64_t y_bytes = M * N * (out_dtype == PK_F32 ? 4 : 2);
  if (y_map != nullptr)
    e = launch_copy_rows(y_dev, y_bytes, y_map, y_bytes, y_bytes, 1, s);
  else
    e = cudaMemcpyAsync(y_host, y_dev, static_cast<size_t>(y_bytes), cudaMemcpyDeviceToHost, s);
  if (e != cudaSuccess) return cuda_fail(e, "copy of y to the host");
  ok();
  return PK_OK;
}

int pk_fp8_quantize(const void* x, int dtype, int64_t n, float scale, uint8_t* x8,
                    void* stream) {
  if (!x || !x8 || n <= 0) return fail(PK_ERR_SHAPE, "need a non-empty input");
  if (dtype != PK_F16 && dtype != PK_BF16 && dtype != PK_F32)
    return fail(PK_ERR_DTYPE, "fp8 quantize input must be f16, bf16 or f32");
  cudaError_t e = launch_fp8_quantize(x, dtype, n, scale, x8, as_stream(stream));
  if (e != cudaSuccess) return cuda_fail(e, "fp8 quantize launch");
  ok();
  return PK_OK;
}

}  // extern "C"

namespace {

int fp8_gemm_impl(const uint8_t* a8, const uint8_t* b8, int64_t M, int64_t N, int64_t K,
                  float out_scale, const float* a_scale, const float* b_scale, void* out,
                  int out_dtype, void* stream) {
  if (!a8 || !b8 || !out) return fail(PK_ERR_SHAPE, "null pointer");
  if (M <= 0 || N <= 0 || K <= 0) return fail(PK_ERR_SHAPE, "need M, N, K > 0");
  if ((K % 16) != 0 || (N % 16) != 0)
    return fail(PK_ERR_SHAPE, "fp8 GEMM needs K and N multiples of 16 (16-byte TMA rows)");
  if (M >= (1ll << 31) || N >= (1ll << 31) || K >= (1ll << 31))
    return fail(PK_ERR_SHAPE, "dimension too large");
  if (out_dtype != PK_F32 && out_dtype != PK_BF16)
    return fail(PK_ERR_DTYPE, "output must be f32 or bf16");
  if ((reinterpret_cast<uintptr_t>(a8) & 15) || (reinterpret_cast<uintptr_t>(b8) & 15))
    return fail(PK_ERR_ALIGN, "fp8 operands must be 16-byte aligned");
  GemmArgs g{};
  g.kind = GemmArgs::kFp8;
  g.a = a8;
  g.a_dtype = PK_E4M3;
  g.lda = K;
  g.b = b8;
  g.ldb = N;
  g.M = M;
  g.N = N;
  g.K = K;
  g.split = 1;
  g.out = out;
  g.out_dtype = out_dtype;
  g.ldc = N;
  g.out_scale = out_scale;
  g.scale_a = a_scale;
  g.scale_b = b_scale;
  g.status = device_status_ptr();
  const char* why = "";
  cudaError_t e = launch_gemm_tc(g, as_stream(stream), &why);
  if (e == cudaErrorInvalidValue && why[0] != '\0') return fail(PK_ERR_ALIGN, "%s", why);
  if (e != cudaSuccess) return cuda_fail(e, "fp8 GEMM launch");
  ok();
  return PK_OK;
}

// Kernel of the fused exchange for a shape, or -1 when none has one: decided
// from the shape alone (aligned stand-in pointers, lda = K), so that every
// rank of an N-sharded layer reaches the same answer.
enum { kPathGemv = 0, kPathDecode = 1, kPathSkinny = 2, kPathPrefill = 3, kPathCluster = 4 };
// The fused tcgen05 W4A16 prefill: 64-row K stages, scales on 64-row
// boundaries (the shapes pk_w4a16_gemm sends to it without a workspace).
bool prefill_shape_ok(int64_t M, int64_t N, int64_t K, int group, bool grouped) {
  return K % 64 == 0 && N % 64 == 0 && (!grouped || group % 64 == 0) && M < (1ll << 31) &&
         N < (1ll << 31) && K < (1ll << 31);
}
// The prefill kernel's exchange stores every output tile to each peer from
// its epilogue; measured on two GPUs it beats the NCCL all-gather for
// Llama-70B down_proj at M = 256 (4.2 MB of fp32 output per rank: 338 vs
// 350 us) and loses for up_proj (14.7 MB: 197 vs 177 us), so it serves
// outputs of at most 8 MB per rank.
constexpr int64_t kPrefillExchangeMaxBytes = int64_t(8) << 20;
int sharded_path(int64_t M, int64_t N, int64_t K, int group, bool grouped, int out_dtype) {
  const void* aligned = reinterpret_cast<const void*>(256);
  const void* sc = grouped ? aligned : nullptr;
  if (gemv_cluster_preferred(M, N, K) &&
      gemv_cluster_supported(M, N, K, group, sc, K, aligned, aligned))
    return kPathCluster;
  if (gemv_supported(M, N, K, group, sc, K, aligned, aligned) &&
      (gemv_preferred(M, N, K) || !decode_supported(M, N, K, group, sc, K, aligned)))
    return kPathGemv;
  if (decode_supported(M, N, K, group, sc, K, aligned)) return kPathDecode;
  if (skinny_supported(M, N, K, group, sc, K, aligned) && skinny_preferred(M, N, K))
    return kPathSkinny;
  if (prefill_shape_ok(M, N, K, group, grouped) &&
      M * N * (out_dtype == PK_F32 ? 4 : 2) <= kPrefillExchangeMaxBytes)
    return kPathPrefill;
  return -1;
}

}  // namespace

extern "C" {

int pk_fp8_gemm(const uint8_t* a8, const uint8_t* b8, int64_t M, int64_t N, int64_t K,
                float out_scale, void* out, int out_dtype, void* stream) {
  return fp8_gemm_impl(a8, b8, M, N, K, out_scale, nullptr, nullptr, out, out_dtype, stream);
}

int pk_fp8_gemm_scaled(const uint8_t* a8, const uint8_t* b8, int64_t M, int64_t N, int64_t K,
                       const float* a_scale, const float* b_scale, void* out, int out_dtype,
                       void* stream) {
  if (!a_scale || !b_scale) return fail(PK_ERR_SHAPE, "null scale pointer");
  return fp8_gemm_impl(a8, b8, M, N, K, 1.0f, a_scale, b_scale, out, out_dtype, stream);
}

int pk_gptq_int4(float* wt, const float* h_inv, int64_t K, int64_t N, int group_size,
                 uint8_t* packed, void* scales, int scale_dtype, float* err_scratch,
                 void* stream) {
  if (!wt || !h_inv || !packed || !scales || !err_scratch)
    return fail(PK_ERR_SHAPE, "null pointer");
  if (K <= 0 || N <= 0 || (N % 2) != 0) return fail(PK_ERR_SHAPE, "need K > 0 and an even N > 0");
  if (group_size < 1 || group_size > gptq_max_group())
    return fail(PK_ERR_SHAPE, "group_size must be in [1, %d] (got %d)", gptq_max_group(),
                group_size);
  if (scale_dtype != PK_F32 && scale_dtype != PK_F16 && scale_dtype != PK_BF16)
    return fail(PK_ERR_DTYPE, "scales must be f32, f16 or bf16");
  cudaError_t e = launch_gptq_int4(wt, h_inv, K, N, group_size, packed, scales, scale_dtype,
                                   err_scratch, as_stream(stream));
  if (e != cudaSuccess) return cuda_fail(e, "gptq launch");
  ok();
  return PK_OK;
}

int pk_fp8_quantize_device(const void* x, int dtype, int64_t n, uint8_t* x8, float* amax,
                           float* scale, void* stream) {
  if (!x || !x8 || !amax || !scale || n <= 0) return fail(PK_ERR_SHAPE, "need a non-empty input");
  if (amax == scale) return fail(PK_ERR_SHAPE, "amax and scale must be different floats");
  if (dtype != PK_F16 && dtype != PK_BF16 && dtype != PK_F32)
    return fail(PK_ERR_DTYPE, "fp8 quantize input must be f16, bf16 or f32");
  cudaError_t e = launch_fp8_quantize_device(x, dtype, n, amax, scale, x8, as_stream(stream));
  if (e != cudaSuccess) return cuda_fail(e, "fp8 device quantize launch");
  ok();
  return PK_OK;
}

size_t pk_gemm_splitk_workspace_size(int64_t M, int64_t N, int64_t K, int split_k) {
  (void)K;
  if (M <= 0 || N <= 0 || split_k <= 1) return 0;
  return gemm_splitk_workspace_bytes(M, N, split_k);
}

int pk_gemm_splitk(const void* a, const void* b, int dtype, int64_t M, int64_t N, int64_t K,
                   int split_k, float* out, void* workspace, size_t workspace_bytes,
                   void* stream) {
  if (!a || !b || !out) return fail(PK_ERR_SHAPE, "null pointer");
  if (M <= 0 || N <= 0 || K <= 0) return fail(PK_ERR_SHAPE, "need M, N, K > 0");
  if (!is16(dtype)) return fail(PK_ERR_DTYPE, "split-K GEMM inputs must be f16 or bf16");
  if ((K % 8) != 0 || (N % 8) != 0)
    return fail(PK_ERR_SHAPE, "split-K GEMM needs K and N multiples of 8 (16-byte TMA rows)");
  if (M >= (1ll << 31) || N >= (1ll << 31) || K >= (1ll << 31))
    return fail(PK_ERR_SHAPE, "dimension too large");
  if (split_k < 1 || split_k > (K + 63) / 64)
    return fail(PK_ERR_SHAPE, "split_k must be in [1, ceil(K/64)] (got %d)", split_k);
  if ((reinterpret_cast<uintptr_t>(a) & 15) || (reinterpret_cast<uintptr_t>(b) & 15))
    return fail(PK_ERR_ALIGN, "operands must be 16-byte aligned");
  GemmArgs g{};
  g.kind = GemmArgs::kDense16;
  g.a = a;
  g.a_dtype = dtype;
  g.lda = K;
  g.b = b;
  g.ldb = N;
  g.M = M;
  g.N = N;
  g.K = K;
  g.split = split_k;
  g.out = out;
  g.out_dtype = PK_F32;
  g.ldc = N;
  g.out_scale = 1.0f;
  g.status = device_status_ptr();
  if (split_k > 1) {
    const size_t need = gemm_splitk_workspace_bytes(M, N, split_k);
    if (workspace == nullptr || workspace_bytes < need)
      return fail(PK_ERR_WORKSPACE, "split-K needs %zu workspace bytes, got %zu", need,
                  workspace_bytes);
    if ((reinterpret_cast<uintptr_t>(workspace) & 255) != 0)
      return fail(PK_ERR_ALIGN, "workspace must be 256-byte aligned");
    if (gemm_tiles(M, N) > kMaxCounters)
      return fail(PK_ERR_UNSUPPORTED, "split-K over more than %lld output tiles",
                  static_cast<long long>(kMaxCounters));
    g.sems = ws_counters(workspace);
    g.partials = ws_partials(workspace);
  }
  const char* why = "";
  cudaError_t e = launch_gemm_tc(g, as_stream(stream), &why);
  if (e == cudaErrorInvalidValue && why[0] != '\0') return fail(PK_ERR_ALIGN, "%s", why);
  if (e != cudaSuccess) return cuda_fail(e, "split-K GEMM launch");
  ok();
  return PK_OK;
}

int pk_shared_alloc(size_t bytes, void** ptr) {
  if (ptr == nullptr || bytes == 0) return fail(PK_ERR_SHAPE, "need a size and an output pointer");
  *ptr = nullptr;
  cudaError_t e = cudaMalloc(ptr, bytes);
  if (e != cudaSuccess) return cuda_fail(e, "shared buffer allocation");
  e = cudaMemset(*ptr, 0, bytes);
  if (e != cudaSuccess) return cuda_fail(e, "shared buffer clear");
  ok();
  return PK_OK;
}

int pk_shared_free(void* ptr) {
  cudaError_t e = cudaFree(ptr);
  if (e != cudaSuccess) return cuda_fail(e, "shared buffer free");
  ok();
  return PK_OK;
}

int pk_ipc_get_handle(const void* ptr, void* handle64) {
  if (ptr == nullptr || handle64 == nullptr) return fail(PK_ERR_SHAPE, "null pointer");
  cudaIpcMemHandle_t h;
  cudaError_t e = cudaIpcGetMemHandle(&h, const_cast<void*>(ptr));
  if (e != cudaSuccess) return cuda_fail(e, "IPC handle");
  static_assert(sizeof(h) == 64, "CUDA IPC handles are 64 bytes");
  std::memcpy(handle64, &h, sizeof(h));
  ok();
  return PK_OK;
}

int pk_ipc_open(const void* handle64, void** ptr) {
  if (handle64 == nullptr || ptr == nullptr) return fail(PK_ERR_SHAPE, "null pointer");
  cudaIpcMemHandle_t h;
  std::memcpy(&h, handle64, sizeof(h));
  cudaError_t e = cudaIpcOpenMemHandle(ptr, h, cudaIpcMemLazyEnablePeerAccess);
  if (e != cudaSuccess) return cuda_fail(e, "IPC open");
  ok();
  return PK_OK;
}

int pk_ipc_close(void* ptr) {
  cudaError_t e = cudaIpcCloseMemHandle(ptr);
  if (e != cudaSuccess) return cuda_fail(e, "IPC close");
  ok();
  return PK_OK;
}

int pk_w4a16_gemm_sharded(const void* a, int a_dtype, int64_t lda, const uint8_t* wp,
                          const void* scales, float scalar_scale, int group_size, int64_t M,
                          int64_t N, int64_t K, int out_dtype, int64_t ldo, int64_t n_offset,
                          int world, int rank, const uint64_t* peer_out,
                          const uint64_t* peer_flag, void* workspace, size_t workspace_bytes,
                          void* stream) {
  if (!a || !wp || !peer_out || !peer_flag) return fail(PK_ERR_SHAPE, "null pointer");
  if (M <= 0 || N <= 0 || K <= 0 || (N % 2) != 0) return fail(PK_ERR_SHAPE, "bad shape");
  if (world < 1 || world > 8 || rank < 0 || rank >= world)
    return fail(PK_ERR_SHAPE, "need 1 <= world <= 8 and 0 <= rank < world");
  if (n_offset < 0 || ldo < n_offset + N) return fail(PK_ERR_SHAPE, "ldo too small for the slice");
  if (!is16(a_dtype)) return fail(PK_ERR_DTYPE, "A must be f16 or bf16");
  if (out_dtype != PK_F32 && out_dtype != PK_BF16)
    return fail(PK_ERR_DTYPE, "output must be f32 or bf16");
  if (scales != nullptr && group_size <= 0) return fail(PK_ERR_SHAPE, "group_size must be > 0");
  // The same kernel choice as pk_w4a16_gemm's automatic split: the CUDA-core
  // GEMV, the tensor-core decode kernel (M <= 32) or the skinny swap-AB
  // kernel (32 < M <= 256, where it beats the fused prefill kernel). The
  // choice, and with it the PK_ERR_UNSUPPORTED that sends callers to the NCCL
  // all-gather, depends on the shape only, so every rank of a layer takes the
  // same path; a rank whose pointers or leading dimension the chosen kernel
  // cannot read gets PK_ERR_ALIGN, an error, never a silent fallback that its
  // peers would not take.
  const int path = sharded_path(M, N, K, group_size, scales != nullptr, out_dtype);
  if (path < 0)
    return fail(PK_ERR_UNSUPPORTED,
                "the fused exchange covers the GEMV, decode and skinny kernels' shapes only");
  const bool aligned16 = (reinterpret_cast<uintptr_t>(wp) & 15) == 0;
  const bool readable =
      path == kPathCluster  ? gemv_cluster_supported(M, N, K, group_size, scales, lda, a, wp)
      : path == kPathGemv   ? gemv_supported(M, N, K, group_size, scales, lda, a, wp)
      : path == kPathDecode ? decode_supported(M, N, K, group_size, scales, lda, a)
      : path == kPathSkinny ? skinny_supported(M, N, K, group_size, scales, lda, a) && aligned16
                            : lda % 8 == 0 && (reinterpret_cast<uintptr_t>(a) & 15) == 0 &&
                                  aligned16 &&
                                  (scales == nullptr ||
                                   (reinterpret_cast<uintptr_t>(scales) & 15) == 0);
  if (!readable)
    return fail(PK_ERR_ALIGN,
                "sharded W4A16: A, the packed weights and the scales must be 16-byte aligned "
                "with lda a multiple of 8");
  // M = 1 layers that fill one wave run the cluster form, which needs only
  // the completion counter from the workspace
  const bool cluster = path == kPathCluster;
  int split = 1;
  size_t need = kCounterBytes;
  if (path == kPathGemv && !cluster) {
    need = gemv_workspace_bytes(M, N, K);
  } else if (path == kPathDecode) {
    split = decode_pick_split(M, N, K);
    if (split > K / 128) split = static_cast<int>(K / 128);
    need = decode_workspace_bytes(M, N, K, split);
    if (N / 128 >= kMaxCounters - 1)
      return fail(PK_ERR_SHAPE, "too many column tiles for the sharded decode kernel");
  }
  if (need < kCounterBytes) need = kCounterBytes;
  if (workspace == nullptr || workspace_bytes < need)
    return fail(PK_ERR_WORKSPACE, "the sharded GEMM needs %zu workspace bytes, got %zu", need,
                workspace_bytes);
  if ((reinterpret_cast<uintptr_t>(workspace) & 255) != 0)
    return fail(PK_ERR_ALIGN, "workspace must be 256-byte aligned");
  for (int r = 0; r < world; ++r)
    if (peer_out[r] == 0 || peer_flag[r] == 0 || (peer_flag[r] & 7) != 0)
      return fail(PK_ERR_SHAPE, "peer %d: missing output or misaligned flag", r);
  DecodeArgs p{};
  p.a = a;
  p.lda = lda;
  p.wp = wp;
  p.scales = scales;
  p.group = group_size;
  p.scalar_scale = scales ? 1.0f : scalar_scale;
  p.M = M;
  p.N = N;
  p.K = K;
  p.out = reinterpret_cast<void*>(peer_out[rank]);
  p.out_dtype = out_dtype;
  p.ldo = ldo;
  p.a_dtype = a_dtype;
  p.split = split;
  p.status = device_status_ptr();
  p.sems = ws_counters(workspace);
  p.partials = ws_partials(workspace);
  OutputShard sh{};
  sh.n_offset = n_offset;
  sh.world = world;
  sh.rank = rank;
  for (int r = 0; r < world; ++r) {
    sh.peer_out[r] = peer_out[r];
    sh.peer_flag[r] = peer_flag[r];
  }
  sh.done = ws_counters(workspace) + (kMaxCounters - 1);
  const char* why = "";
  if (path == kPathPrefill) {
    GemmArgs g{};
    g.kind = GemmArgs::kW4A16;
    g.a = a;
    g.a_dtype = a_dtype;
    g.lda = lda;
    g.b = wp;
    g.ldb = N / 2;
    g.scales = scales;
    g.group = group_size;
    g.M = M;
    g.N = N;
    g.K = K;
    g.split = 1;
    g.out = reinterpret_cast<void*>(peer_out[rank]);
    g.out_dtype = out_dtype;
    g.ldc = ldo;
    g.out_scale = scales ? 1.0f : scalar_scale;
    g.status = device_status_ptr();
    g.peers = sh;
    cudaError_t e = launch_gemm_tc(g, as_stream(stream), &why);
    if (e == cudaErrorInvalidValue && why[0] != '\0') return fail(PK_ERR_ALIGN, "%s", why);
    if (e != cudaSuccess) return cuda_fail(e, "sharded w4a16 prefill launch");
    ok();
    return PK_OK;
  }
  cudaError_t e = cluster ? launch_w4a16_gemv_cluster(p, as_stream(stream), &why, &sh)
                  : path == kPathGemv     ? launch_w4a16_gemv(p, as_stream(stream), &why, &sh)
                  : path == kPathDecode ? launch_w4a16_decode(p, as_stream(stream), &why, &sh)
                                    : launch_w4a16_skinny(p, as_stream(stream), &why, &sh);
  if (e == cudaErrorInvalidValue && why[0] != '\0') return fail(PK_ERR_ALIGN, "%s", why);
  if (e != cudaSuccess) return cuda_fail(e, "sharded w4a16 gemm launch");
  ok();
  return PK_OK;
}

int pk_fake_quant_groups(const void* w, int dtype, int64_t rows, int64_t cols, int64_t ldw,
                         int64_t group_rows, int bits, void* out, int64_t ldo, void* stream) {
  if (!w || !out) return fail(PK_ERR_SHAPE, "null pointer");
  if (rows <= 0 || cols <= 0 || ldw < cols || ldo < cols)
    return fail(PK_ERR_SHAPE, "need rows, cols > 0 and leading dimensions >= cols");
  if (bits < 2 || bits > 8) return fail(PK_ERR_SHAPE, "bits must be in [2, 8] (got %d)", bits);
  if (dtype != PK_F16 && dtype != PK_BF16 && dtype != PK_F32)
    return fail(PK_ERR_DTYPE, "fake quantization runs on f16, bf16 or f32");
  cudaError_t e = launch_fake_quant_groups(w, dtype, rows, cols, ldw, group_rows, bits, out, ldo,
                                           as_stream(stream));
  if (e != cudaSuccess) return cuda_fail(e, "fake quantization launch");
  ok();
  return PK_OK;
}

int pk_gptq_ref(float* wt, const float* h_inv, int64_t K, int64_t N, int out_group, int bits,
                float* err_scratch, void* stream) {
  if (!wt || !h_inv || !err_scratch) return fail(PK_ERR_SHAPE, "null pointer");
  if (K <= 0 || N <= 0) return fail(PK_ERR_SHAPE, "need K, N > 0");
  if (N > gptq_ref_max_out())
    return fail(PK_ERR_UNSUPPORTED, "the walk holds at most %d outputs per feature (got %lld)",
                gptq_ref_max_out(), (long long)N);
  if (bits < 2 || bits > 8) return fail(PK_ERR_SHAPE, "bits must be in [2, 8] (got %d)", bits);
  cudaError_t e = launch_gptq_ref(wt, h_inv, K, N, out_group, bits, err_scratch, as_stream(stream));
  if (e != cudaSuccess) return cuda_fail(e, "gptq (reference rule) launch");
  ok();
  return PK_OK;
}

int pk_set_wait_limit_ns(int64_t ns) {
  if (ns < 0) return fail(PK_ERR_SHAPE, "the wait limit must be >= 0 ns (0: default)");
  int* p = device_status_ptr();
  if (p == nullptr) return fail(PK_ERR_CUDA, "device status word unavailable");
  int dev = 0, khz = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e == cudaSuccess) e = cudaDeviceGetAttribute(&khz, cudaDevAttrClockRate, dev);
  if (e != cudaSuccess) return cuda_fail(e, "SM clock rate");
  // SM cycles at the highest clock: the limit is at least `ns` at any clock
  long long cycles = ns == 0 ? 0 : ns / 1000000 * khz + (ns % 1000000) * khz / 1000000;
  if (ns > 0 && cycles < 1) cycles = 1;
  e = cudaMemcpy(p + 2, &cycles, sizeof(cycles), cudaMemcpyHostToDevice);
  if (e != cudaSuccess) return cuda_fail(e, "set the wait limit");
  ok();
  return PK_OK;
}

int pk_set_weight_staging(int mode) {
  if (mode != 0 && mode != 1) return fail(PK_ERR_SHAPE, "weight staging mode must be 0 or 1");
  set_weight_staging(mode);
  ok();
  return PK_OK;
}

int pk_debug_phase_stamps(void* dev_buf, size_t bytes) {
  set_phase_stamps(dev_buf, bytes);
  ok();
  return PK_OK;
}

}  // extern "C"
