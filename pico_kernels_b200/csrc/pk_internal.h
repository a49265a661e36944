// Internal declarations shared between the kernel translation units and the
// C-ABI layer (capi.cu). Launchers return cudaError_t; capi.cu validates
// arguments, maps errors to pk_status and records messages.
#pragma once

#include <cstddef>
#include <cstdint>
#include <cuda.h>
#include <cuda_runtime.h>

#include "../../include/pico_b200.h"

namespace pk {

// Device status word: [0] first error code, [1] site that recorded it.
int* device_status_ptr();  // per current device; nullptr on failure

// Message returned by pk_last_error_string() on this host thread.
void set_error_message(const char* msg);

// Sites recorded with PK_ERR_TIMEOUT (which wait gave up).
enum WaitSite : int {
  kSiteDecodeFull = 101,
  kSiteDecodeMma = 102,
  kSiteDecodeFinal = 103,
  kSiteDecodePeers = 104,
  kSiteGemmProducer = 201,
  kSiteGemmMma = 202,
  kSiteGemmEpilogue = 203,
  kSiteGemmDequant = 204,
  kSiteGemmPeers = 205,
  kSiteGemvProducer = 301,
  kSiteGemvConsumer = 302,
  kSiteGemvPeers = 303,
  kSiteSkinnyFull = 401,
  kSiteSkinnyMma = 402,
  kSiteSkinnyFinal = 403,
  kSiteSkinnyPeers = 404,
};

// Host-side tensor map encoding (cuTensorMapEncodeTiled via the runtime's
// driver entry point; nothing links libcuda directly).
bool encode_tmap_2d(CUtensorMap* map, CUtensorMapDataType dtype, const void* base,
                    uint64_t inner, uint64_t outer, uint64_t row_stride_bytes, uint32_t box_inner,
                    uint32_t box_outer, CUtensorMapSwizzle swizzle, const char** why);

int num_sms();  // SM count of the current device (cached)

// cudaFuncSetAttribute(kernel, MaxDynamicSharedMemorySize, bytes) once per
// kernel and device; later calls return without the runtime call.
cudaError_t set_max_smem(const void* kernel, int bytes);

// W4A16 with large M: dequantize the weights once into a 16-bit workspace
// B[K, N] (prefill_workspace_bytes) and run the dense tensor-core GEMM.
bool prefill_dequant_once(int64_t M, int64_t N, int64_t K);
size_t prefill_workspace_bytes(int64_t N, int64_t K);

// Split-K workspaces. Every kernel that reduces through a caller's workspace
// keeps its arrival counters in the first kCounterBytes and its fp32 partials
// after them. Counters are zero between calls (each call re-arms the ones it
// used) and partials are scratch, so one workspace can serve calls of any
// shape and kernel in turn: no call's partials overlay another's counters.
constexpr size_t kCounterBytes = 64 * 1024;
constexpr int64_t kMaxCounters = static_cast<int64_t>(kCounterBytes / sizeof(unsigned));
inline unsigned* ws_counters(void* ws) { return static_cast<unsigned*>(ws); }
inline float* ws_partials(void* ws) {
  return reinterpret_cast<float*>(static_cast<unsigned char*>(ws) + kCounterBytes);
}

// ---- quant_pack.cu --------------------------------------------------------
cudaError_t launch_quant_int4_group(const void* w, int w_dtype, int64_t K, int64_t N, int64_t ldw,
                                    int group, uint8_t* packed, void* scales, int scale_dtype,
                                    cudaStream_t s);
cudaError_t launch_absmax(const void* x, int dtype, int64_t n, float* out, cudaStream_t s);
cudaError_t launch_quant_int4_tensor(const void* w, int dtype, int64_t n, float scale,
                                     int8_t* codes, cudaStream_t s);
cudaError_t launch_pack_int4(const int8_t* q, int64_t K, int64_t N, uint8_t* p, cudaStream_t s);
cudaError_t launch_unpack_int4(const uint8_t* p, int64_t K, int64_t N, int8_t* q,
                               cudaStream_t s);
// reference-rule fake quantization of every column of w[rows, cols], groups of
// `group` rows (<= 0: whole columns), arithmetic rounded to dtype per step
cudaError_t launch_fake_quant_groups(const void* w, int dtype, int64_t rows, int64_t cols,
                                     int64_t ldw, int64_t group, int bits, void* out, int64_t ldo,
                                     cudaStream_t s);
// ---- gptq.cu (GPTQ producer of packed int4 weights) ----------------------
int gptq_max_group();
cudaError_t launch_gptq_int4(float* wt, const float* h_inv, int64_t K, int64_t N, int group,
                             uint8_t* packed, void* scales, int scale_dtype, float* err,
                             cudaStream_t s);
// The reference's own walk (quantize.py:95-104): wt[K = in, N = out] fp32 is
// overwritten with the fake-quant weights, each input feature quantized with
// quantize_col's rule (groups of `out_group` outputs, <= 0: the whole column)
int gptq_ref_max_out();
cudaError_t launch_gptq_ref(float* wt, const float* h_inv, int64_t K, int64_t N, int out_group,
                            int bits, float* err, cudaStream_t s);

// absmax into amax, then the cast with scale = 448 / amax computed on the
// device and stored to `scale` (gemm_fp8.quantize without the host sync)
cudaError_t launch_fp8_quantize_device(const void* x, int dtype, int64_t n, float* amax,
                                       float* scale, uint8_t* y, cudaStream_t s);
cudaError_t launch_fp8_quantize(const void* x, int dtype, int64_t n, float scale, uint8_t* y,
                                cudaStream_t s);
// B[K, N] (dtype) = q * s rounded to dtype, or q when scales == nullptr (N % 8 == 0)
cudaError_t launch_dequant_int4(const uint8_t* wp, const void* scales, int group, int dtype,
                                int64_t K, int64_t N, void* out, cudaStream_t s);

// Output exchange of an N-sharded layer (GEMV, decode and skinny kernels):
// the kernel writes its columns [n_offset, n_offset + N) into every rank's
// buffer, then flags each peer. world == 0 marks an unsharded call (the
// kernels then store to their `out` argument and ignore the rest).
struct OutputShard {
  int64_t n_offset;
  int world, rank;
  uint64_t peer_out[8];
  uint64_t peer_flag[8];  // 8 bytes each: arrival count, then (own only) expected count
  unsigned* done;  // zeroed completion counter (workspace)
};

// ---- host_io.cu (row copies between mapped page-locked host memory and
// device buffers, by a kernel chained with programmatic dependent launch) --
cudaError_t launch_copy_rows(const void* src, int64_t src_pitch, void* dst, int64_t dst_pitch,
                             int64_t row_bytes, int64_t rows, cudaStream_t s);

// ---- w4a16_decode.cu -----------------------------------------------------
struct DecodeArgs {
  const void* a;
  int64_t lda;
  const uint8_t* wp;
  const void* scales;  // nullptr -> scalar_scale
  int group;           // rows per scale group (scales != nullptr)
  float scalar_scale;
  int64_t M, N, K;
  void* out;
  int out_dtype;
  int64_t ldo;
  int split;           // >= 1
  int a_dtype;
  float* partials;     // [n_tiles][split][M][128] when split > 1 (global reduction)
  unsigned* sems;      // [n_tiles] arrival counters, zero between calls
  bool force_workspace;  // reduce through the workspace even when a cluster would fit
  int* status;
};
int decode_max_cluster_split();
bool decode_supported(int64_t M, int64_t N, int64_t K, int group, const void* scales,
                      int64_t lda, const void* a);
int decode_pick_split(int64_t M, int64_t N, int64_t K);
size_t decode_workspace_bytes(int64_t M, int64_t N, int64_t K, int split);

// ---- w4a16_skinny.cu (32 < M <= 256, swap-AB, weights dequantized once) ----
bool skinny_supported(int64_t M, int64_t N, int64_t K, int group, const void* scales,
                      int64_t lda, const void* a);
bool skinny_preferred(int64_t M, int64_t N, int64_t K);
cudaError_t launch_w4a16_skinny(const DecodeArgs& p, cudaStream_t s, const char** why,
                                const OutputShard* shard = nullptr);
cudaError_t launch_w4a16_decode(const DecodeArgs& args, cudaStream_t s, const char** why,
                                const OutputShard* shard = nullptr);

// ---- w4a16_gemv.cu (M <= 2 on the CUDA cores; cluster or stream-K split) -
bool gemv_preferred(int64_t M, int64_t N, int64_t K);  // faster than the decode kernel here
bool gemv_supported(int64_t M, int64_t N, int64_t K, int group, const void* scales, int64_t lda,
                    const void* a, const void* wp);
size_t gemv_workspace_bytes(int64_t M, int64_t N, int64_t K);  // 0: no split-K fixup needed
cudaError_t launch_w4a16_gemv(const DecodeArgs& args, cudaStream_t s, const char** why,
                              const OutputShard* shard = nullptr);

// ---- w4a16_gemv_cluster.cu (M = 1 in one wave, K split reduced in clusters)
bool gemv_cluster_supported(int64_t M, int64_t N, int64_t K, int group, const void* scales,
                            int64_t lda, const void* a, const void* wp);
bool gemv_cluster_preferred(int64_t M, int64_t N, int64_t K);
int gemv_cluster_split(int64_t N, int64_t K);
cudaError_t launch_w4a16_gemv_cluster(const DecodeArgs& args, cudaStream_t s, const char** why,
                                      const OutputShard* shard = nullptr);
// Weight staging (pk_set_weight_staging): 1 = decode GEMVs load weights and
// scales into shared memory before the previous kernel in the stream ends.
void set_weight_staging(int mode);
int weight_staging();
// Phase stamps (pk_debug_phase_stamps): for a launch of `grid` CTAs, the
// half of the buffer this launch writes (halves alternate launch by launch,
// so the last two are kept), or nullptr when unset or too small.
void set_phase_stamps(void* buf, size_t bytes);
uint64_t* phase_stamps(size_t grid);

// ---- gemm_tc.cu (persistent tcgen05 GEMM: fp8, dense split-K, W4A16 prefill)
struct GemmArgs {
  enum Kind { kDense16 = 0, kFp8 = 1, kW4A16 = 2 } kind;
  const void* a;        // [M, K] row-major (ld lda), dtype a_dtype
  int a_dtype;          // PK_F16 / PK_BF16 / PK_E4M3
  int64_t lda;
  const void* b;        // dense/fp8: [K, N] row-major (ld ldb); W4A16: packed uint8 [K, N/2]
  int64_t ldb;
  const void* scales;   // W4A16: [ceil(K/group), N] in a_dtype
  int group;
  int64_t M, N, K;
  int split;            // K splits (dense), else 1
  void* out;
  int out_dtype;        // PK_F32 / PK_BF16
  int64_t ldc;
  float out_scale;
  const float* scale_a;  // fp8: device scales of A and B; when set, the epilogue
  const float* scale_b;  // multiplies by 1 / (scale_a * scale_b) instead of out_scale
  float* partials;      // split-K workspace
  unsigned* sems;
  int* status;
  OutputShard peers;    // W4A16 prefill of an N-sharded layer (world 0: unsharded)
};
int64_t gemm_tiles(int64_t M, int64_t N);
size_t gemm_splitk_workspace_bytes(int64_t M, int64_t N, int split);
cudaError_t launch_gemm_tc(const GemmArgs& g, cudaStream_t s, const char** why);

// ---- w4a16_simt.cu (any shape; CUDA cores) -------------------------------
cudaError_t launch_w4a16_simt(const void* a, int a_dtype, int64_t lda, const uint8_t* wp,
                              const void* scales, float scalar_scale, int group, int64_t M,
                              int64_t N, int64_t K, void* out, int out_dtype, int64_t ldo,
                              cudaStream_t s);

}  // namespace pk
