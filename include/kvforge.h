/*
 * kvforge.h -- C ABI of the B200-native KVForge codec (libkvforge_b200.so).
 *
 * This is the drop-in boundary for the reference's codec path. It replaces the
 * stubbed CUDA crate (crates/kvforge-cuda: KernelLauncher in
 * src/kernel_launcher.rs:7-77 and GpuCompressionPipeline in
 * src/gpu_pipeline.rs:10-37) and serves the kvforge-core traits
 * (crates/kvforge-core/src/codec.rs:27-137, src/pipeline.rs:73-80).
 *
 * Conventions
 *  - Plain pointers and sizes only. Tensor pointers are DEVICE pointers unless
 *    a parameter name ends in _host. Streams are cudaStream_t passed as void*
 *    (NULL = legacy default stream).
 *  - Every call returns kvf_status; KVF_OK is 0. The numbering mirrors the
 *    reference KvForgeError variants (crates/kvforge-core/src/error.rs:3-28)
 *    plus two device-side conditions. kvf_last_error() returns the message of
 *    the last failing call on the calling thread.
 *  - Calls are stream-ordered. The only host synchronisations are the ones a
 *    function documents (sizes that must reach the host, and the one-off basis
 *    step, which runs its eigen-solve on the host).
 *  - One kvf_ctx per device. Calls on one context may come from several host
 *    threads at once, each issuing on its own stream; scratch memory is taken
 *    per call from the context's stream-ordered pool, so calls on different
 *    streams share no scratch and never wait for one another. The one
 *    exception is kvf_calibrate_noalloc, whose calls all share one file-scope
 *    device array (see its entry: calls of it that overlap on the GPU race).
 *    The context has one device status word: a device-side error (corrupt
 *    stream, expired wait) is reported by the next call that reads it, which
 *    may be another thread's.
 *  - A compressed layer (kvf_compressed) may be read on any stream:
 *    kvf_decompress_layer and kvf_compressed_attention on a stream other than
 *    the one that built the object first wait (stream-ordered, no host
 *    synchronisation) until the object is complete, and kvf_compressed_free
 *    returns its buffers to the pool only after the last read issued on every
 *    stream before the free. The building stream (the `stream` of
 *    kvf_compress_layer or kvf_compressed_deserialize) must outlive the
 *    object, and the context must outlive every object made with it. The raw
 *    device views of kvf_compressed_tensor_views carry no such ordering:
 *    order their use after the building stream yourself.
 *  - Layout: tensors are [num_heads, seq_len, head_dim] row-major, as in the
 *    reference KVCache (crates/kvforge-core/src/types.rs:5-12).
 */
#ifndef KVFORGE_B200_H
#define KVFORGE_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define KVF_ABI_VERSION 1

typedef enum {
  KVF_OK = 0,
  KVF_ERR_SHAPE_MISMATCH = 1,  /* KvForgeError::ShapeMismatch */
  KVF_ERR_INVALID_CONFIG = 2,  /* KvForgeError::InvalidConfig */
  KVF_ERR_QUANTIZATION = 3,    /* KvForgeError::QuantizationError */
  KVF_ERR_PROJECTION = 4,      /* KvForgeError::ProjectionError */
  KVF_ERR_ENTROPY = 5,         /* KvForgeError::EntropyError */
  KVF_ERR_SERIALIZATION = 6,   /* KvForgeError::SerializationError */
  KVF_ERR_CUDA = 7,            /* KvForgeError::CudaError */
  KVF_ERR_PIPELINE = 8,        /* KvForgeError::PipelineError */
  KVF_ERR_DEVICE_TIMEOUT = 9,  /* a bounded device-side wait gave up */
  KVF_ERR_CORRUPT_STREAM = 10  /* rANS container failed validation on the device */
} kvf_status;

/* DataType (types.rs:106-113) */
typedef enum { KVF_INT4 = 0, KVF_INT8 = 1, KVF_F32 = 2 } kvf_data_type;
/* QuantAxis (types.rs:97-103) */
typedef enum { KVF_PER_CHANNEL = 0, KVF_PER_TOKEN = 1 } kvf_quant_axis;
/* element type of an input tensor; the reference takes f32 only
 * (crates/kvforge-python/src/py_types.rs:21-25); f16 is up-cast exactly. */
typedef enum { KVF_IN_F32 = 0, KVF_IN_F16 = 1 } kvf_in_dtype;
/* CompressionPreset (crates/kvforge-core/src/pipeline.rs:5-15) */
typedef enum {
  KVF_CONSERVATIVE = 0,
  KVF_BALANCED = 1,
  KVF_AGGRESSIVE = 2,
  KVF_ADAPTIVE = 3
} kvf_preset;

/* PipelineConfig (crates/kvforge-core/src/pipeline.rs:17-28) */
typedef struct {
  int32_t preset;
  int32_t key_data_type;
  int32_t value_data_type;
  int32_t enable_projection;
  double projection_variance_threshold;
  int32_t enable_entropy_coding;
  int32_t enable_calibration;
} kvf_pipeline_config;

typedef struct kvf_ctx kvf_ctx;
typedef struct kvf_basis kvf_basis;
typedef struct kvf_compressed kvf_compressed;

/* ---- context ---------------------------------------------------------- */
/* replaces KernelLauncher::new (kernel_launcher.rs:13-17). Free every
 * kvf_compressed built or loaded on a context (kvf_compressed_free) before
 * kvf_destroy(ctx): their buffers come from the context's memory pool and
 * their ordering events from its event cache. */
kvf_status kvf_init(int device, kvf_ctx** out);
kvf_status kvf_destroy(kvf_ctx* ctx);
const char* kvf_last_error(void);
int kvf_abi_version(void);
/* 1: reconstruction uses separate multiply and add in the reference's order
 * (projection.rs:160-166), bit-identical to the CPU oracle.
 * 0 (default): the engine chosen by kvf_set_reconstruct_engine, within
 * relative Frobenius error 1e-5 of the reference loop. */
kvf_status kvf_set_exact_reconstruct(kvf_ctx* ctx, int exact);
/* engine of the non-exact reconstruction (kvf_reconstruct, decompression):
 * CUDA_CORE: one fused multiply-add per term in the reference's order; up to
 *   16 coefficients the basis sits in registers and many small blocks per SM
 *   share the GPU with concurrent work, beyond that a shared-memory kernel
 *   that is bound by its multiply-adds;
 * TENSOR_CORE: for head_dim 128 and up to 64 coefficients, a tcgen05 GEMM
 *   (operands split into two tf32 parts, three products, accumulators in
 *   TMEM) with one block per SM; other shapes fall back to CUDA cores;
 * AUTO (default): CUDA cores up to 16 coefficients, tensor cores above. */
typedef enum { KVF_RECON_AUTO = 0, KVF_RECON_CUDA_CORE = 1, KVF_RECON_TENSOR_CORE = 2 } kvf_recon_engine;
kvf_status kvf_set_reconstruct_engine(kvf_ctx* ctx, int engine);
/* engine of the projection inside quantization (the pipeline's value path,
 * kvf_fused_project_quantize with per-token axis; kvf_project always runs the
 * CUDA-core chain and returns its coefficients):
 * CUDA_CORE / AUTO (default): each coefficient as one fused multiply-add
 *   chain over the channels in the reference's order (up to 32 coefficients
 *   fused with the quantization, beyond that a separate quantization pass);
 * TENSOR_CORE: for f16 input, head_dim 128 and up to 64 coefficients, a
 *   tcgen05 GEMM computes every coefficient with a bounded error, and the
 *   coefficients that decide a code (each row's minimum and maximum, and any
 *   value within that bound of a rounding boundary) are recomputed with the
 *   exact chain, so codes, scales and mins are identical to the CUDA-core
 *   engine's; other shapes use the CUDA-core engine;
 * TENSOR_CORE_APPROX: the same GEMM without the exact recomputation: codes,
 *   scales and mins of the tensor-core coefficients, whose relative error
 *   against the exact chain is near 2^-22 (a code can differ by one level
 *   where a coefficient lies that close to a rounding boundary, and a row's
 *   scale and min in their last bits). */
typedef enum {
  KVF_PROJ_AUTO = 0,
  KVF_PROJ_CUDA_CORE = 1,
  KVF_PROJ_TENSOR_CORE = 2,
  KVF_PROJ_TENSOR_CORE_APPROX = 3
} kvf_proj_engine;
kvf_status kvf_set_projection_engine(kvf_ctx* ctx, int engine);
/* Runs one of the library's bounded device waits against a barrier or status
 * word that nothing completes, with a 2 ms limit: the wait gives up and the
 * next kvf_sync on `stream` reports KVF_ERR_DEVICE_TIMEOUT, after which the
 * context is usable as before. MBARRIER: the wait of the tensor-map copy and
 * tensor-core pipelines; LOOKBACK: the rANS encoder's wait for the offsets of
 * earlier chunks. */
typedef enum { KVF_WAIT_MBARRIER = 0, KVF_WAIT_LOOKBACK = 1 } kvf_wait_kind;
kvf_status kvf_selftest_wait_timeout(kvf_ctx* ctx, int which, void* stream);
/* waits for `stream` and reports any error a device kernel recorded
 * (corrupt rANS container, bounded wait expiry) since the last check */
kvf_status kvf_sync(kvf_ctx* ctx, void* stream);

/* ---- observability (no counterpart in the reference, which has no tracing) --
 * kvf_launch_count: kernels this library has launched in the process.
 * Stage timing: when enabled on a context, each pipeline stage is bracketed by
 * CUDA events on its stream; kvf_profile_read synchronises those events,
 * returns per-stage totals (ms, launches of the stage, algorithmic bytes) for
 * stages 0..KVF_NUM_STAGES-1 and clears them. */
#define KVF_NUM_STAGES 8
enum {
  KVF_STAGE_CALIBRATE = 0,
  KVF_STAGE_PROJECT = 1,
  KVF_STAGE_QUANTIZE = 2,
  KVF_STAGE_ENTROPY_ENCODE = 3,
  KVF_STAGE_ENTROPY_DECODE = 4,
  KVF_STAGE_RECONSTRUCT = 5,
  KVF_STAGE_DEQUANTIZE = 6,
  KVF_STAGE_BASIS = 7
};
uint64_t kvf_launch_count(void);
const char* kvf_stage_name(int32_t stage);
kvf_status kvf_profile_enable(kvf_ctx* ctx, int enable);
kvf_status kvf_profile_read(kvf_ctx* ctx, double* ms, uint64_t* count, double* bytes);

/* PipelineConfig::from_preset (crates/kvforge-core/src/pipeline.rs:30-71) */
kvf_status kvf_pipeline_config_from_preset(int32_t preset, kvf_pipeline_config* out);

/* ---- stage-level entry points (the kvforge-core traits) ----------------- */

/* SensitivityCalibrator::calibrate (codec.rs:27-29; calibration.rs:25-73).
 * keys [H,T,D]; scores out: H floats (device). KVF_ERR_INVALID_CONFIG when
 * T < min_tokens. */
kvf_status kvf_calibrate(kvf_ctx* ctx, const void* keys, int32_t in_dtype, size_t H, size_t T,
                         size_t D, size_t min_tokens, float* scores, void* stream);

/* kvf_calibrate without any device allocation. It has no counterpart in the
 * reference. It is for callers that cannot allocate device memory: a serving
 * engine that reserves all device memory up front and forbids later
 * allocations, or a latency-critical path that cannot afford cudaMalloc's
 * implicit device synchronisation. Results match kvf_calibrate.
 * - Scratch: a file-scope device array of 65536 (head, tile) slots (1 MiB),
 *   loaded with the library and held by every GPU that loads it until the
 *   process exits. A tile is 65536 elements of one head, so the call needs
 *   H * ceil(T * D / 65536) <= 65536 and returns KVF_ERR_INVALID_CONFIG
 *   beyond that, before touching the device.
 * - The first call on a device looks up the array's device address
 *   (cudaGetSymbolAddress, once per device per process); make that first call
 *   before any stream capture begins.
 * - All calls share the one array and each overwrites it: calls that overlap
 *   on the GPU (two streams, or two threads) race and give wrong scores.
 *   Every slot a call reads is written by that call first, so nothing has to
 *   be cleared between calls.
 * It calls no cudaMalloc, cudaFree or allocating library routine. */
kvf_status kvf_calibrate_noalloc(kvf_ctx* ctx, const void* keys, int32_t in_dtype, size_t H, size_t T,
                                 size_t D, size_t min_tokens, float* scores, void* stream);

/* Quantizer::quantize (codec.rs:105-111; quantize.rs:47-163).
 * packed: INT8 -> H*T*D bytes, INT4 -> ceil(H*T*D/2) bytes (low nibble first,
 * pairs over the flat index). scales/mins: H*D (per-channel) or H*T (per-token). */
kvf_status kvf_quantize(kvf_ctx* ctx, const void* data, int32_t in_dtype, size_t H, size_t T,
                        size_t D, int32_t data_type, int32_t axis, uint8_t* packed, float* scales,
                        float* mins, void* stream);

/* Quantizer::dequantize (codec.rs:113-114; quantize.rs:165-231). out f32 [H,T,D]. */
kvf_status kvf_dequantize(kvf_ctx* ctx, const uint8_t* packed, size_t packed_len,
                          const float* scales, const float* mins, int32_t data_type,
                          int32_t axis, size_t H, size_t T, size_t D, float* out, void* stream);

/* Projector::project (codec.rs:50-57; projection.rs:61-140) against a basis.
 * basis_vt [H,R,D] f32 (rows >= ranks[h] are zero), ranks [H] uint64 (device).
 * projected out f32 [H,T,R]; column r of head h is sum_c x[h,t,c]*basis_vt[h,r,c]
 * as one fused multiply-add chain over c = 0..D-1, and +0.0 for r >= ranks[h]. */
kvf_status kvf_project(kvf_ctx* ctx, const void* data, int32_t in_dtype, size_t H, size_t T,
                       size_t D, const float* basis_vt, const uint64_t* ranks, size_t R,
                       float* projected, void* stream);

/* Projector::reconstruct (codec.rs:59-64; projection.rs:142-172). out f32 [H,T,D]. */
kvf_status kvf_reconstruct(kvf_ctx* ctx, const float* projected, size_t H, size_t T, size_t R,
                           size_t D, const float* basis_vt, const uint64_t* ranks, float* out,
                           void* stream);

/* KernelLauncher::fused_project_quantize_int4/int8 (kernel_launcher.rs:19-41):
 * projection then quantization in one call; same outputs as kvf_project
 * followed by kvf_quantize on the projected tensor. */
kvf_status kvf_fused_project_quantize(kvf_ctx* ctx, const void* data, int32_t in_dtype, size_t H,
                                      size_t T, size_t D, const float* basis_vt,
                                      const uint64_t* ranks, size_t R, int32_t data_type,
                                      int32_t axis, uint8_t* packed, float* scales, float* mins,
                                      void* stream);

/* EntropyCodec::encode (codec.rs:131-133; entropy.rs:42-86), container format
 * in the library's documentation. freq out: 256 u32 counts (device) -- the
 * reference's EntropyState.frequencies. out_cap must be at least
 * kvf_rans_max_encoded_len(n). SYNCHRONISES `stream` to return *out_len_host. */
size_t kvf_rans_max_encoded_len(size_t n);
kvf_status kvf_rans_encode(kvf_ctx* ctx, const uint8_t* data, size_t n, uint8_t* out,
                           size_t out_cap, size_t* out_len_host, uint32_t* freq, void* stream);

/* EntropyCodec::decode (codec.rs:135-136; entropy.rs:88-123). freq: 256 u32
 * counts (device). KVF_ERR_ENTROPY when comp_len % 4 != 0 (entropy.rs:94-98).
 * SYNCHRONISES `stream` to report KVF_ERR_CORRUPT_STREAM. */
kvf_status kvf_rans_decode(kvf_ctx* ctx, const uint8_t* comp, size_t comp_len,
                           const uint32_t* freq, size_t original_len, uint8_t* out, void* stream);

/* KernelLauncher::entropy_decode_dequant (kernel_launcher.rs:64-76): rANS
 * decode then dequantize to f32 [H,T,D]. Asynchronous; a corrupt stream is
 * reported by kvf_sync. */
kvf_status kvf_entropy_decode_dequant(kvf_ctx* ctx, const uint8_t* comp, size_t comp_len,
                                      const uint32_t* freq, const float* scales,
                                      const float* mins, int32_t data_type, int32_t axis,
                                      size_t H, size_t T, size_t D, float* out, void* stream);

/* ---- fused dequantize + decode attention (KernelLauncher::
 *      fused_dequant_attention, crates/kvforge-cuda/src/kernel_launcher.rs:43-57;
 *      the kernel is an empty stub in the reference,
 *      crates/kvforge-cuda/kernels/fused_dequant_attention.cu:1-53) --------
 * One query row per head: out[h, :] = softmax(scale * K_h q_h) V_h with K and V
 * the dequantized (and, with a basis, reconstructed) cache, computed on the
 * codes without rebuilding K or V. query [H, D] f32, out [H, D] f32, device.
 * Keys are per-channel codes [H, T, k_cols] with [H, k_cols] scales/mins,
 * values per-token codes [H, T, v_cols] with [H, T] scales/mins (the
 * pipeline's layout); k_data_type / v_data_type INT4 or INT8 (packed as the
 * quantizer packs them). Without a basis the width is head_dim; with one it is
 * the basis's R (basis [H, R, D] and ranks [H], rows from rank on ignored).
 * T = 0 writes zeros. Relative error against an fp64 evaluation of the same
 * formula is at f32 rounding level (the tests bound it by 1e-4). */
kvf_status kvf_fused_dequant_attention(kvf_ctx* ctx, const uint8_t* k_codes, const uint8_t* v_codes,
                                       const float* query, const float* k_scales, const float* k_mins,
                                       const float* v_scales, const float* v_mins, int32_t k_data_type,
                                       int32_t v_data_type, size_t H, size_t T, size_t D, size_t k_cols,
                                       size_t v_cols, const float* k_basis_vt, const uint64_t* k_ranks,
                                       const float* v_basis_vt, const uint64_t* v_ranks, float scale,
                                       float* out, void* stream);
/* the same on a compressed layer (entropy-coded codes are decoded into
 * scratch first); stream-ordered, no host synchronisation */
kvf_status kvf_compressed_attention(kvf_ctx* ctx, const kvf_compressed* c, const float* query, float scale,
                                    float* out, void* stream);

/* ---- projection basis (the calibrated basis) ----------------------------
 * The reference takes a full SVD of each head inside project
 * (projection.rs:81-90). Here the basis step is separate: a Gram matrix
 * X_h^T X_h per head on the device, then an fp64 symmetric eigen-solve on the
 * host; eigenvectors sorted by descending eigenvalue are the right singular
 * vectors, sqrt(eigenvalue) the singular values. Ranks follow select_rank
 * (projection.rs:31-59); R = max rank. SYNCHRONISES `stream`. */
kvf_status kvf_basis_compute(kvf_ctx* ctx, const void* data, int32_t in_dtype, size_t H,
                             size_t T, size_t D, double variance_threshold, size_t max_rank,
                             kvf_basis** out, void* stream);
/* basis from host arrays: basis_vt_host [H,R,D], ranks_host [H] */
kvf_status kvf_basis_from_host(kvf_ctx* ctx, size_t H, size_t R, size_t D,
                               const float* basis_vt_host, const uint64_t* ranks_host,
                               kvf_basis** out);
kvf_status kvf_basis_info(const kvf_basis* b, size_t* H, size_t* R, size_t* D);
/* copies out (host): basis_vt [H,R,D], ranks [H], singular values [H,D]
 * (any pointer may be NULL; singular values are zero for a basis from host) */
kvf_status kvf_basis_download(const kvf_basis* b, float* basis_vt_host, uint64_t* ranks_host,
                              float* sv_host);
const float* kvf_basis_device_vt(const kvf_basis* b);
const uint64_t* kvf_basis_device_ranks(const kvf_basis* b);
kvf_status kvf_basis_free(kvf_basis* b);

/* ---- whole-layer pipeline (CompressionPipeline, core/src/pipeline.rs:73-80;
 *      CpuCompressionPipeline::compress/decompress, cpu/src/pipeline.rs:99-186)
 * keys, values: [H,T,D] device tensors of in_dtype. k_basis / v_basis: the
 * calibrated bases for projection presets; NULL computes them inside the
 * call (a synchronising host eigen-solve, as the reference does an SVD per
 * call). The result lives on the device; sizes that depend on the entropy
 * coder's output are read back on first request. */
kvf_status kvf_compress_layer(kvf_ctx* ctx, const void* keys, const void* values,
                              int32_t in_dtype, size_t H, size_t T, size_t D, size_t layer_idx,
                              const kvf_pipeline_config* cfg, const kvf_basis* k_basis,
                              const kvf_basis* v_basis, kvf_compressed** out, void* stream);
/* keys_out, values_out: f32 [H,T,D] device */
kvf_status kvf_decompress_layer(kvf_ctx* ctx, const kvf_compressed* c, float* keys_out,
                                float* values_out, void* stream);

/* Many layers in one call (the layers of a step: a streaming append, or a
 * rank's shard). Arrays of L device pointers / handles; layer_idx may be NULL
 * (0..L-1). The result out[l] is what kvf_compress_layer gives for layer l,
 * codes, parameters and sizes bit for bit. With keys_out and values_out
 * (arrays of L f32 [H,T,D] device buffers, or both NULL) every layer is also
 * decompressed, as kvf_decompress_layer does (the CUDA-core reconstruction;
 * exact mode honoured). Short chunks -- T <= 128, head_dim <= 128 and a
 * multiple of 4, projection width <= 64, given bases for projection presets,
 * no entropy coding, no calibration -- take one kernel launch for all layers
 * (one CTA per layer, tensor and head); other shapes run the per-layer path
 * for each layer. Stream-ordered; no host synchronisation. No counterpart in
 * the reference, which compresses one KVCache per call (core/src/pipeline.rs:73-80). */
kvf_status kvf_compress_layers(kvf_ctx* ctx, size_t L, const void* const* keys, const void* const* values,
                               int32_t in_dtype, size_t H, size_t T, size_t D, const size_t* layer_idx,
                               const kvf_pipeline_config* cfg, const kvf_basis* const* k_bases,
                               const kvf_basis* const* v_bases, kvf_compressed** out, float* const* keys_out,
                               float* const* values_out, void* stream);

/* Host-buffer variants (pinned or pageable host memory): copy in, run, copy
 * out on `stream`; they synchronise before returning. */
kvf_status kvf_compress_layer_host(kvf_ctx* ctx, const void* keys_host, const void* values_host,
                                   int32_t in_dtype, size_t H, size_t T, size_t D,
                                   size_t layer_idx, const kvf_pipeline_config* cfg,
                                   const kvf_basis* k_basis, const kvf_basis* v_basis,
                                   kvf_compressed** out, void* stream);
kvf_status kvf_decompress_layer_host(kvf_ctx* ctx, const kvf_compressed* c, float* keys_host,
                                     float* values_host, void* stream);

/* CompressedKV accessors (types.rs:36-56). Sizes SYNCHRONISE on first call
 * when entropy coding was enabled. */
kvf_status kvf_compressed_shape(const kvf_compressed* c, size_t* H, size_t* T, size_t* D,
                                size_t* layer_idx);
kvf_status kvf_compressed_size_bytes(kvf_compressed* c, size_t* out);
kvf_status kvf_original_size_bytes(const kvf_compressed* c, size_t* out);
kvf_status kvf_compression_ratio(kvf_compressed* c, double* out);
/* per tensor (0 = keys, 1 = values): rank width R (0 when not projected),
 * quantized byte length before entropy coding, final data length */
kvf_status kvf_compressed_tensor_info(kvf_compressed* c, int32_t which, size_t* R,
                                      size_t* packed_len, size_t* data_len, int32_t* has_entropy);
/* device views of one tensor's buffers (NULL where absent) */
kvf_status kvf_compressed_tensor_views(const kvf_compressed* c, int32_t which,
                                       const uint8_t** data, const float** scales,
                                       const float** mins, const uint32_t** freq,
                                       const float** basis_vt, const uint64_t** ranks);
/* ---- streaming append with basis reuse (an extension: the reference has no
 *      append API and compresses every chunk as its own KVCache, with a fresh
 *      SVD per chunk, crates/kvforge-cpu/src/pipeline.rs:100-163) ----------
 * kvf_compressed_basis: the projection state of one tensor (0 = keys,
 * 1 = values) as a basis handle that shares it, no copy; *out is NULL when
 * that tensor was not projected. Passed to kvf_compress_layer for the later
 * chunks of the same layer, it projects them onto the prefix's basis; each
 * chunk stays a complete CompressedKV in the reference's format.
 * kvf_compressed_basis_bytes: the bytes of projection state
 * (ProjectionState::size_bytes, types.rs:131-135) counted in
 * kvf_compressed_size_bytes. A store that keeps one basis per layer charges a
 * chunk compressed with it size - basis bytes. */
kvf_status kvf_compressed_basis(const kvf_compressed* c, int32_t which, kvf_basis** out);
kvf_status kvf_compressed_basis_bytes(const kvf_compressed* c, size_t* out);

/* calibration scores of the keys (H floats, device), or NULL when calibration
 * was disabled or failed (the reference discards both, pipeline.rs:104-111) */
const float* kvf_compressed_calibration(const kvf_compressed* c);

/* ---- cost model with measured GPU costs (CostModel, crates/kvforge-core/src/cost.rs;
 *      the reference's CpuCostModel is a fixed table, crates/kvforge-cpu/src/cost.rs:9-115)
 * A table row per preset: expected ratio, microseconds per original (f32)
 * byte to compress and to decompress, quality in [0, 1] (1 = lossless). */
typedef struct {
  int32_t preset;
  double compression_ratio;
  double compress_us_per_byte;
  double decompress_us_per_byte;
  double quality;
} kvf_preset_cost;
/* CostEstimate (crates/kvforge-core/src/cost.rs) */
typedef struct {
  int32_t preset;
  double compress_us, transfer_us, decompress_us, total_us, compression_ratio;
} kvf_estimate;
/* BandwidthTier, in declaration order; kvf_bandwidth_bytes_per_us gives
 * BandwidthTier::bytes_per_us (negative for an unknown tier) */
typedef enum {
  KVF_BW_LOCAL = 0,
  KVF_BW_RDMA = 1,
  KVF_BW_ETHERNET_100G = 2,
  KVF_BW_ETHERNET_25G = 3,
  KVF_BW_ETHERNET_10G = 4,
  KVF_BW_WAN = 5
} kvf_bandwidth_tier;
double kvf_bandwidth_bytes_per_us(int32_t tier);
/* Measures Conservative, Balanced and Aggressive on one sample layer (device
 * keys and values [H,T,D] of in_dtype) and writes three rows: per-byte costs
 * from CUDA events over `reps` compress calls and `reps` decompress calls on
 * `stream` (bases calibrated once, outside the timing), the layer's
 * compression ratio, and quality = 1 - the larger relative Frobenius error of
 * keys and values. Allocates its output buffers; SYNCHRONISES. */
kvf_status kvf_cost_measure(kvf_ctx* ctx, const void* keys, const void* values, int32_t in_dtype, size_t H,
                            size_t T, size_t D, int reps, kvf_preset_cost* rows_out, void* stream);
/* CostModel::estimate: the row of `preset` (the first row for a preset the
 * table lacks, as the reference falls back to its first entry); host only */
kvf_status kvf_cost_estimate(const kvf_preset_cost* rows, size_t n, size_t original_bytes, int32_t preset,
                             double bytes_per_us, kvf_estimate* out);
/* CostModel::select_codec: estimates of the rows with quality >= min_quality,
 * by total time, fastest first (ties keep table order); `out` holds n entries,
 * *count gets the number written; host only */
kvf_status kvf_cost_select(const kvf_preset_cost* rows, size_t n, size_t original_bytes, double bytes_per_us,
                           double min_quality, kvf_estimate* out, size_t* count);

/* serialisation to host bytes and back (CompressedKV.to_bytes/from_bytes,
 * crates/kvforge-python/src/py_types.rs:98-110) in the reference's wire
 * format: bincode 1.x of CompressedKV (crates/kvforge-core/src/types.rs:36-148),
 * field for field. quantized_data carries this library's rANS container when
 * entropy coding is on (a reference-written entropy payload deserialises but
 * does not decode: kvf_decompress_layer reports KVF_ERR_CORRUPT_STREAM).
 * Calibration scores are not part of the format. kvf_compressed_serialize
 * with buf == NULL returns the size. */
kvf_status kvf_compressed_serialize(kvf_compressed* c, uint8_t* buf_host, size_t cap,
                                    size_t* len);
kvf_status kvf_compressed_deserialize(kvf_ctx* ctx, const uint8_t* buf_host, size_t len,
                                      kvf_compressed** out, void* stream);
kvf_status kvf_compressed_free(kvf_compressed* c);
/* kvf_compressed_free of cs[0], ..., cs[n-1] in order (NULL entries are
 * skipped): one call for the objects of a kvf_compress_layers step. */
kvf_status kvf_compressed_free_many(kvf_compressed* const* cs, size_t n);

#ifdef __cplusplus
}
#endif
#endif /* KVFORGE_B200_H */
