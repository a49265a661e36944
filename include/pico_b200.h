/*
 * pico_b200.h -- C ABI of the B200 (sm_100a) quantized-matmul path.
 *
 * Drop-in boundary for pico-kernels' quantized-matmul functions. Every entry
 * point takes plain device pointers (pk_w4a16_gemm_host also host pointers),
 * sizes and a cudaStream_t passed as `void*` (NULL = legacy default stream);
 * no framework types cross the boundary. Every entry point is asynchronous on
 * `stream` except where noted, returns a pk_status (0 = success), and on
 * failure leaves a message for pk_last_error_string(). Shapes and layouts
 * follow the reference:
 *   - matrices are row-major with an explicit leading dimension in elements;
 *   - packed int4 weights are uint8 [K, N/2], byte [k, j] holding column 2j
 *     in its low nibble and column 2j+1 in its high nibble (gemm_int4.py:65-72);
 *   - group scales are [ceil(K/group), N], groups running along K.
 *
 * Reference citations are paths within the pico-kernels project.
 */
#ifndef PICO_B200_H_
#define PICO_B200_H_

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define PK_API __attribute__((visibility("default")))
#else
#define PK_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* Status codes. The reference raises AssertionError on bad shapes
 * (gemm_int4.py:78-81, gemm_splitk.py:71); the Python layer maps these codes
 * to ValueError / TypeError / RuntimeError. */
typedef enum {
  PK_OK = 0,
  PK_ERR_SHAPE = 1,        /* a size or leading dimension is invalid        */
  PK_ERR_DTYPE = 2,        /* unsupported dtype combination                 */
  PK_ERR_ALIGN = 3,        /* pointer or stride misaligned for 16-byte TMA  */
  PK_ERR_CUDA = 4,         /* a CUDA runtime/driver call failed             */
  PK_ERR_TIMEOUT = 5,      /* a device-side bounded wait expired            */
  PK_ERR_WORKSPACE = 6,    /* workspace missing or too small                */
  PK_ERR_UNSUPPORTED = 7   /* valid request this build does not implement   */
} pk_status;

/* Element types. */
typedef enum {
  PK_F16 = 0,
  PK_BF16 = 1,
  PK_F32 = 2,
  PK_E4M3 = 3,
  PK_U8 = 4,
  PK_I8 = 5
} pk_dtype;

/* Library version (major*10000 + minor*100 + patch). */
PK_API int pk_version(void);

/* Message of the last failing call on this host thread ("" if none). */
PK_API const char* pk_last_error_string(void);

/* Device status word written by bounded device-side waits. Synchronises the
 * current device. *code = first recorded pk_status (0 if none), *where = the
 * site that recorded it; reset != 0 clears it. */
PK_API int pk_device_status(int* code, int* where, int reset);

/* Limit of every device-side wait of this library on the current device
 * (mbarrier phases, the sharded layers' peer flags), in nanoseconds at the
 * highest SM clock; 0 restores the built-in ~2 s. A wait that runs out
 * records PK_ERR_TIMEOUT and its site in the device status word and the
 * kernel returns without its result (pk_device_status reads it). Synchronous.
 * No counterpart in the reference (Triton kernels have no bounded waits). */
PK_API int pk_set_wait_limit_ns(int64_t ns);

/* ---------------------------------------------------------------------- */
/* int4 quantization and packing                                           */
/* ---------------------------------------------------------------------- */

/* Per-group symmetric int4 quantize + pack of W[K, N] (dtype F16/BF16/F32),
 * groups of `group_size` rows along K (the last group may be ragged).
 *   scale = max|w[group, n]|.clamp_min(1e-12) / 7   (fp32, IEEE division)
 *   q     = clamp(round_half_even(w / scale), -7, 7)
 * Writes packed[K, N/2] (ld N/2) and scales[ceil(K/group), N] rounded to
 * `scale_dtype` (F16/BF16/F32).
 * Replaces quantize.quantize_col applied column-wise (quantize.py:42-68)
 * followed by gemm_int4.pack_int4_n (gemm_int4.py:65-72). */
PK_API int pk_quant_int4_group(const void* w, int w_dtype, int64_t K, int64_t N, int64_t ldw,
                        int group_size, uint8_t* packed, void* scales, int scale_dtype,
                        void* stream);

/* max|x| over n elements (dtype F16/BF16/F32) into *absmax_dev (device fp32).
 * The absmax half of gemm_int4.quantize_int4 (gemm_int4.py:60) and
 * gemm_fp8.quantize (gemm_fp8.py:94). */
PK_API int pk_absmax(const void* x, int dtype, int64_t n, float* absmax_dev, void* stream);

/* Per-tensor int4 codes: q = clamp(round(dtype(w / scale)), -8, 7) as int8,
 * the quotient computed in fp32 and rounded to w's dtype (F16/BF16/F32) before
 * rounding to an integer. Replaces the elementwise half of
 * gemm_int4.quantize_int4 (gemm_int4.py:61). */
PK_API int pk_quant_int4_tensor(const void* w, int dtype, int64_t n, float scale, int8_t* codes,
                         void* stream);

/* Pack int8 codes q[K, N] into uint8 [K, N/2] (gemm_int4.py:65-72). */
PK_API int pk_pack_int4_n(const int8_t* q, int64_t K, int64_t N, uint8_t* packed, void* stream);

/* Unpack uint8 [K, N/2] into sign-extended int8 [K, N]; the inverse used by
 * the reference's round-trip test (tests/test_gemm_int4.py:33-42). */
PK_API int pk_unpack_int4_n(const uint8_t* packed, int64_t K, int64_t N, int8_t* q, void* stream);

/* Fake quantization with the reference's rule, in the input's own dtype:
 * for every column c of w[rows, cols] (dtype F16/BF16/F32, ld ldw) and every
 * group of group_rows consecutive rows (group_rows <= 0: the whole column),
 *   scale = dtype(dtype(max|w|.clamp_min(1e-12)) / qmax),  qmax = 2^(bits-1) - 1
 *   out   = dtype(clamp(round(dtype(w / scale)), -qmax, qmax) * scale)
 * each step computed in fp32 and rounded to the dtype as torch does (so an
 * fp16 group of zeros gets scale 0 and NaN outputs, as in the reference).
 * bits in [2, 8]. out[rows, cols] has the same dtype (ld ldo).
 * Replaces quantize.quantize_col on a column (quantize.py:42-60) and, on a
 * layer's fp32 copy w[out, in], the column walk of quantize.rtn_layer
 * (quantize.py:63-68). */
PK_API int pk_fake_quant_groups(const void* w, int dtype, int64_t rows, int64_t cols, int64_t ldw,
                                int64_t group_rows, int bits, void* out, int64_t ldo,
                                void* stream);

/* ---------------------------------------------------------------------- */
/* W4A16 GEMM                                                              */
/* ---------------------------------------------------------------------- */

/* Bytes of workspace pk_w4a16_gemm needs for this shape with split_k (0 =
 * the library's own choice). Zero when the chosen path needs none. */
PK_API size_t pk_w4a16_workspace_size(int64_t M, int64_t N, int64_t K, int split_k);

/* out[M, N] = A[M, K] @ dequant(Wp) where dequant(Wp)[k, n] =
 *   q[k, n] * scales[k / group_size, n]   if scales != NULL, or
 *   q[k, n] * scalar_scale                 if scales == NULL.
 * A: F16 or BF16 (ld lda). Wp: uint8 [K, N/2] (ld N/2). scales dtype must
 * equal A's dtype. out: F32 or BF16 (ld ldo). split_k: 0 = automatic,
 * 1 = no split, > 1 = split the K reduction over that many CTAs (decode
 * shapes), reduced deterministically in split order through `workspace`
 * (pk_w4a16_workspace_size bytes, zero-filled once before its first use; the
 * kernel leaves it ready for the next call). With split_k = 0 and M <= 8 a
 * decode GEMV on mma.sync tiles of exactly decoded fp16 operands runs
 * instead: on layers that fit one wave of clusters (N % 128 == 0,
 * K % 512 == 0, group 128 or a scalar scale, e.g. 4096 x 4096) its cluster
 * form, which needs no workspace; on other layers (N % 32 == 0, groups a
 * multiple of 64) a stream-K form that reduces through the workspace, and
 * without one the tensor-core decode kernel, which also serves 8 < M <= 32
 * (N and K multiples of 128, group 128 or a scalar scale). For 32 < M <= 256 (N % 128 == 0, K % 64 == 0) a
 * swap-AB tensor-core kernel that dequantizes each weight once runs where a
 * model of measured per-stage times favours it over the tcgen05 prefill
 * kernel, which serves the rest. From
 * M = 1024 the weights are dequantized once into the workspace (16-bit
 * B[K, N] after the counters, pk_w4a16_workspace_size bytes) and the dense
 * tensor-core GEMM runs on it; without that workspace the fused kernel runs.
 * A workspace may serve calls of different shapes and of pk_gemm_splitk in
 * turn (arrival counters sit in its first 64 KB, partials after them), but
 * calls sharing one workspace must not overlap on the GPU.
 * Replaces gemm_int4.int4_gemm (gemm_int4.py:75-92); the reference's
 * per-tensor float scale is scalar_scale, applied in the epilogue instead of
 * a second pass over C (gemm_int4.py:92). */
PK_API int pk_w4a16_gemm(const void* a, int a_dtype, int64_t lda, const uint8_t* wp, const void* scales,
                  float scalar_scale, int group_size, int64_t M, int64_t N, int64_t K, void* out,
                  int out_dtype, int64_t ldo, int split_k, void* workspace,
                  size_t workspace_bytes, void* stream);

/* Decode W4A16 GEMM that allocates nothing and takes no workspace. It has no
 * counterpart in the reference. It exists for callers that cannot call
 * cudaMalloc: a runtime that plans all device memory itself and forbids
 * libraries from allocating, or a latency-critical decode loop that cannot
 * afford cudaMalloc's implicit synchronization. Same arguments as
 * pk_w4a16_gemm minus the workspace, for decode shapes only (M <= 32,
 * N % 128 == 0, K % 128 == 0, group 128 or a scalar scale). It always runs
 * the tensor-core decode kernel with its K splits reduced through memory, so
 * its output equals pk_w4a16_gemm's with the same explicit split_k bit for
 * bit, and pk_w4a16_gemm's automatic route (the GEMV at M = 1) within the
 * W4A16 tolerance. Its split-K
 * partials live in a static 4 MiB device array owned by the library (plus
 * arrival counters for up to 4096 column tiles), held on every GPU that loads
 * the library until exit. With split_k = 0 the automatic split is lowered
 * until tiles * split * M * 512 bytes fit (down to no split); an explicit
 * split_k that does not fit fails with PK_ERR_WORKSPACE before launching. The first call on a
 * device looks up the array's address; make it before any stream capture.
 * All calls on a device share the array: each clears the counters it uses on
 * its stream, and calls that overlap on the GPU race. */
PK_API int pk_w4a16_gemm_noalloc(const void* a, int a_dtype, int64_t lda, const uint8_t* wp,
                                 const void* scales, float scalar_scale, int group_size, int64_t M,
                                 int64_t N, int64_t K, void* out, int out_dtype, int64_t ldo,
                                 int split_k, void* stream);

/* pk_w4a16_gemm for a caller whose activations and outputs live in host
 * memory, in one call: copies A [M, K] from a_host (row stride lda elements)
 * into the device staging buffer a_dev (>= M*K*2 bytes, rows packed to K),
 * runs pk_w4a16_gemm (split_k = 0) into the device staging buffer y_dev
 * (>= M*N elements of out_dtype), then copies y into y_host [M, N]. All
 * steps are enqueued on `stream`; synchronise it before reading y_host. With
 * page-locked host buffers (cudaHostAlloc / torch pin_memory) the copies are
 * done by a small kernel on the buffers' device mapping, and for the decode
 * shapes (those the GEMV or the decode kernel serves) the GEMM writes y_host
 * directly, leaving y_dev untouched; pageable buffers also work, through
 * cudaMemcpyAsync, which then blocks the host. workspace as for pk_w4a16_gemm. This is the host-buffer form of
 * gemm_int4.int4_gemm (gemm_int4.py:75-92) with the caller's tensor moves
 * (`a.cuda()`, `c.cpu()`) folded in. */
PK_API int pk_w4a16_gemm_host(const void* a_host, int a_dtype, int64_t lda, const uint8_t* wp,
                              const void* scales, float scalar_scale, int group_size, int64_t M,
                              int64_t N, int64_t K, void* y_host, int out_dtype, void* a_dev,
                              void* y_dev, void* workspace, size_t workspace_bytes,
                              void* stream);

/* Weight staging of the cluster decode GEMV (M <= 8; process-wide, default 0).
 * mode 0: a GEMV prefetches its weights and scales into L2 before the
 *   kernel ahead of it in the stream has finished (a hint that never returns
 *   stale data), and loads them into shared memory only after it has.
 * mode 1: the GEMV loads its first weights and scales into shared memory
 *   before that kernel has finished; only the activations wait for it. The
 *   caller guarantees that no kernel which lets its dependents start early
 *   (programmatic dependent launch) writes the weights or scales of the
 *   GEMV that follows it. Kernels that do not (every kernel launched without
 *   that trigger, including this library's quantizers) are safe.
 * Applies to calls made after it. No counterpart in the reference (Triton
 * launches have no such overlap). */
PK_API int pk_set_weight_staging(int mode);

/* Profiling aid: while dev_buf is set (NULL turns it off), each CTA of the
 * decode GEMVs (M <= 8) launched afterwards writes 8 uint64 words at
 * dev_buf[slot * bytes / 16 + 8 * cta]: %globaltimer at entry, after
 * griddepcontrol.wait, when its first weights landed, when its arithmetic
 * ended and when its output was stored, then its SM id, its unit count (the
 * stream-K GEMV sets bit 32 in CTAs that summed a slice's partials) and the
 * time it finished, after the sharded exchange's flag barrier if any. `slot` alternates 0, 1 from launch to launch (the
 * two halves of the buffer), so the last two launches of a chain are both
 * kept. Launches whose grid needs more than `bytes` (grid * 128) record
 * nothing. Kernels captured in a CUDA
 * graph keep the setting they were captured with. No counterpart in the
 * reference. */
PK_API int pk_debug_phase_stamps(void* dev_buf, size_t bytes);

/* ---------------------------------------------------------------------- */
/* N-sharded W4A16 layer with the output exchange fused into the GEMV      */
/* ---------------------------------------------------------------------- */

/* Peer memory for the fused exchange. pk_shared_alloc: cudaMalloc'd, zeroed
 * device memory that peers can map; pk_ipc_get_handle writes its 64-byte CUDA
 * IPC handle; pk_ipc_open maps a peer's handle into this process (lazy peer
 * access over NVLink); pk_ipc_close / pk_shared_free release them. No
 * counterpart in the reference (it has no multi-GPU path). */
PK_API int pk_shared_alloc(size_t bytes, void** ptr);
PK_API int pk_shared_free(void* ptr);
PK_API int pk_ipc_get_handle(const void* ptr, void* handle64);
PK_API int pk_ipc_open(const void* handle64, void** ptr);
PK_API int pk_ipc_close(void* ptr);

/* One rank's slice of an N-sharded W4A16 layer, y[M, N_full] = A @ dequant(W),
 * where this rank holds columns [n_offset, n_offset + N) (Wp [K, N/2],
 * scales [K/g, N]). The local kernel (the one pk_w4a16_gemm picks without a
 * workspace and with split_k = 0: the GEMV, the decode kernel, the skinny
 * kernel, or the fused tcgen05 prefill) writes its columns straight into
 * every rank's output buffer peer_out[r] (fp32 or bf16 [M, ldo] with ldo >=
 * N_full, mapped with pk_ipc_open), then its last CTA adds 1 to every peer's
 * arrival count peer_flag[r] (release, system scope) and waits, bounded (the
 * wait limit, pk_set_wait_limit_ns), until its own count reaches the next
 * multiple of world - 1: on return every rank's columns are in
 * peer_out[rank]. Each peer_flag[r] is 8 zero-initialised, 8-byte aligned
 * bytes in rank r's memory (the count, then rank r's own expected count,
 * advanced by the kernel, so CUDA graph replays stay in step). All ranks call
 * it in the same order; a buffer must not be rewritten by the next call
 * before its reader is done (alternate two buffers). Needs a workspace of
 * pk_w4a16_workspace_size bytes (at least 64 KB); world <= 8. The kernel is
 * chosen from the shape alone, so every rank of a layer takes the same path:
 * shapes no kernel with the exchange serves (K or N not a multiple of 64, a
 * group size not a multiple of 64 on the prefill, or a prefill-sized call
 * whose output slice is over 8 MB, where NCCL's all-gather is faster) return
 * PK_ERR_UNSUPPORTED on every rank, and the caller can exchange with NCCL
 * instead; a rank whose A, Wp or scales are not 16-byte aligned (or lda not a
 * multiple of 8) gets PK_ERR_ALIGN, an error rather than a fallback.
 * Replaces the all-gather that gemm_int4.int4_gemm's callers would need on a
 * sharded layer (no counterpart in the reference). */
PK_API int pk_w4a16_gemm_sharded(const void* a, int a_dtype, int64_t lda, const uint8_t* wp,
                                 const void* scales, float scalar_scale, int group_size, int64_t M,
                                 int64_t N, int64_t K, int out_dtype, int64_t ldo, int64_t n_offset,
                                 int world, int rank, const uint64_t* peer_out,
                                 const uint64_t* peer_flag, void* workspace,
                                 size_t workspace_bytes, void* stream);

/* GPTQ producer of packed int4 weights: the loop of quantize.gptq_layer
 * (quantize.py:71-115, act_order=False) run on the GPU, emitting codes and
 * scales in the W4A16 layout instead of fake-quant floats. wt[K, N] fp32
 * (K = input features, N = outputs: the layer's weight transposed) is the
 * working copy and is overwritten; h_inv[K, K] fp32 is the inverse of the
 * damped Hessian (quantize.py:88-93). Scales are per group of group_size
 * (<= 128) consecutive input features and output, taken from the group's
 * error-updated weights when the walk reaches it (max|w| clamped at 1e-12,
 * / 7), stored rounded to scale_dtype as [ceil(K/group), N]; codes
 * clamp(round(w / scale), -7, 7) packed as pk_pack_int4_n into packed[K,
 * N/2]. err_scratch holds group_size * N floats. Updates are applied in the
 * reference's order with separately rounded products and differences. */
PK_API int pk_gptq_int4(float* wt, const float* h_inv, int64_t K, int64_t N, int group_size,
                 uint8_t* packed, void* scales, int scale_dtype, float* err_scratch,
                 void* stream);

/* The GPTQ walk of quantize.gptq_layer itself (quantize.py:95-104) on the
 * GPU, with the reference's quantize_col rule: wt[K, N] fp32 (K = input
 * features, N = outputs: the layer's weight transposed, already permuted by
 * the caller for act_order, quantize.py:97-98) is overwritten with the
 * fake-quant weights. Input feature j in order: scales over groups of
 * out_group consecutive outputs (<= 0: all N; quantize.py:100 with
 * group_size), q = clamp(round(w / scale), -qmax, qmax), err = w - q * scale,
 * and every later feature k receives w[k] -= err * (h_inv[j, k] / h_inv[j, j]),
 * products and differences rounded separately as torch does. h_inv[K, K] is
 * the inverse damped Hessian (quantize.py:88-93). bits in [2, 8]; N <= 16384;
 * err_scratch holds 32 * N floats. */
PK_API int pk_gptq_ref(float* wt, const float* h_inv, int64_t K, int64_t N, int out_group,
                       int bits, float* err_scratch, void* stream);

/* ---------------------------------------------------------------------- */
/* fp8 (e4m3) GEMM                                                         */
/* ---------------------------------------------------------------------- */

/* x8[i] = e4m3(dtype(x[i] * scale)), RNE (F16/BF16/F32 input). The cast half
 * of gemm_fp8.quantize (gemm_fp8.py:95). */
PK_API int pk_fp8_quantize(const void* x, int dtype, int64_t n, float scale, uint8_t* x8, void* stream);

/* out[M, N] = (A8[M, K] @ B8[K, N]) * out_scale with e4m3 inputs, fp32
 * accumulation and a single epilogue multiply; out F32 or BF16.
 * A8 row-major (ld K), B8 row-major (ld N).
 * Replaces gemm_fp8.fp8_gemm_precast (gemm_fp8.py:98-117), where
 * out_scale = 1 / (a_scale * b_scale) (gemm_fp8.py:106). */
PK_API int pk_fp8_gemm(const uint8_t* a8, const uint8_t* b8, int64_t M, int64_t N, int64_t K,
                float out_scale, void* out, int out_dtype, void* stream);

/* gemm_fp8.quantize (gemm_fp8.py:89-95) without the host sync of its .item():
 * amax[0] = max|x| and scale[0] = 448 / amax (1 when x is all zero, where the
 * reference's division raises) are computed and left in DEVICE memory, and
 * x8 = e4m3(dtype(x * scale)) as pk_fp8_quantize would write it with that
 * scale. amax and scale are distinct device floats. Stream-ordered; graph
 * capturable. */
PK_API int pk_fp8_quantize_device(const void* x, int dtype, int64_t n, uint8_t* x8, float* amax,
                           float* scale, void* stream);

/* pk_fp8_gemm with the per-tensor scales read from DEVICE memory (as
 * pk_fp8_quantize_device leaves them): out = (A8 @ B8) / (a_scale[0] *
 * b_scale[0]), the reciprocal formed in double and rounded to fp32 as
 * gemm_fp8.py:106 forms out_scale on the host. */
PK_API int pk_fp8_gemm_scaled(const uint8_t* a8, const uint8_t* b8, int64_t M, int64_t N, int64_t K,
                       const float* a_scale, const float* b_scale, void* out, int out_dtype,
                       void* stream);

/* ---------------------------------------------------------------------- */
/* Dense split-K GEMM                                                      */
/* ---------------------------------------------------------------------- */

/* Bytes of workspace pk_gemm_splitk needs. */
PK_API size_t pk_gemm_splitk_workspace_size(int64_t M, int64_t N, int64_t K, int split_k);

/* out[M, N] fp32 = A[M, K] @ B[K, N] (both F16 or both BF16, row-major) with
 * the K reduction split over split_k slices, partial sums reduced in slice
 * order (deterministic) through `workspace`.
 * Replaces gemm_splitk.triton_gemm_splitk (gemm_splitk.py:67-80), which
 * reduces with fp32 atomics into a zeroed C (gemm_splitk.py:64,72). */
PK_API int pk_gemm_splitk(const void* a, const void* b, int dtype, int64_t M, int64_t N, int64_t K,
                   int split_k, float* out, void* workspace, size_t workspace_bytes, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* PICO_B200_H_ */
