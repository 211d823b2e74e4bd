// Internal declarations shared by the kernel files and the C-ABI layer.
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cstddef>
#include <cstdint>

#include "../../include/kvforge.h"

namespace kvf {

// ---- rANS container constants (documented in kvf_rans.cu) ----------------
constexpr uint32_t kRansProbBits = 13;
constexpr uint32_t kRansM = 1u << kRansProbBits;
constexpr uint32_t kRansL = 1u << 16;
constexpr uint32_t kRansLanes = 32;
constexpr uint32_t kRansChunk = 8192;                   // symbols per chunk (encoder default)
constexpr uint32_t kRansMaxChunk = kRansLanes * 65535u;  // lane word counts are u16
constexpr uint32_t kRansMagic = 0x3252564Bu;             // "KVR2"
constexpr size_t kRansHeader = 32;
constexpr size_t kRansPayloadHeader = 4 * kRansLanes + 2 * kRansLanes;  // lane states + lane word counts

// dynamic shared memory above this opts in to the larger per-block limit;
// the margin below 48 KB leaves room for a kernel's static shared memory
constexpr size_t kSmemOptIn = 40 * 1024;

// device status bits (ctx->d_status); mapped to kvf_status by the host
constexpr unsigned kDevErrCorrupt = 1u;
constexpr unsigned kDevErrEntropy = 2u;
constexpr unsigned kDevErrTimeout = 4u;

__host__ __device__ inline size_t rans_num_chunks(size_t n, uint32_t chunk) { return (n + chunk - 1) / chunk; }
inline size_t rans_max_len(size_t n, uint32_t chunk) {
  size_t nc = rans_num_chunks(n, chunk);
  return kRansHeader + 4 * (nc + 1) + nc * (kRansPayloadHeader + 2) + 2 * n;
}

inline bool aligned(const void* p, size_t a) { return (reinterpret_cast<uintptr_t>(p) % a) == 0; }

inline float quant_levels(int dt) { return dt == KVF_INT4 ? 15.0f : 255.0f; }
inline size_t packed_len(size_t n, int dt) { return dt == KVF_INT4 ? (n + 1) / 2 : n; }
inline size_t num_params(size_t H, size_t T, size_t D, int axis) {
  return axis == KVF_PER_CHANNEL ? H * D : H * T;
}

// process-wide count of kernels launched by this library (kvf_launch_count)
void note_launches(unsigned n);


#ifdef __CUDACC__
// ---- KIVI arithmetic shared by every kernel that quantizes (quantize.rs) ----
__device__ __forceinline__ float canon0(float v) { return v == 0.0f ? 0.0f : v; }

// NaN-ignoring min/max with -0.0 canonicalised to +0.0: fminf/fmaxf already
// return the other operand for a NaN, and v + 0.0 (IEEE, round to nearest)
// maps -0.0 to +0.0 and leaves every other value unchanged
__device__ __forceinline__ void mm_update(float v, float& mn, float& mx) {
  v = __fadd_rn(v, 0.0f);
  mn = fminf(mn, v);
  mx = fmaxf(mx, v);
}

__device__ __forceinline__ void warp_minmax(float& mn, float& mx) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    mn = fminf(mn, __shfl_xor_sync(0xffffffffu, mn, o));
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
  }
}

__device__ __forceinline__ float make_scale(float mn, float mx, float levels) {
  const float range = __fsub_rn(mx, mn);
  return (range < 1e-10f) ? 1.0f : __fdiv_rn(range, levels);
}

__device__ __forceinline__ uint32_t qcode(float v, float mn, float scale, float levels) {
  const float y = __fdiv_rn(__fsub_rn(v, mn), scale);
  float r = roundf(y);  // half away from zero, as Rust f32::round
  if (isnan(r)) return 0u;  // NaN.clamp() stays NaN; `as u8` maps it to 0
  r = fminf(fmaxf(r, 0.0f), levels);
  return (uint32_t)r;
}

// The same code without a division per element. With inv = RN(1/scale), the
// product y = RN(n * inv) is within 1.5 * 2^-23 * y of RN(n / scale); codes need
// y <= 255.5, so |y - RN(n/scale)| < 2^-14.4. Rounding to an integer can only
// differ when y lies within that distance of a half-integer, and then the
// exact IEEE quotient is computed. NaN and +-inf take the same paths as qcode.
__device__ __forceinline__ uint32_t qcode_fast(float v, float mn, float scale, float inv, float levels) {
  const float n = __fsub_rn(v, mn);
  const float y = __fmul_rn(n, inv);
  const float fl = floorf(y);
  const float fr = __fsub_rn(y, fl);
  float r;
  if (fabsf(__fsub_rn(fr, 0.5f)) < 1.220703125e-4f) {  // within 2^-13 of a half-integer
    r = roundf(__fdiv_rn(n, scale));
  } else {
    // away from the half-integers round-half-away-from-zero is floor + (frac > 1/2);
    // NaN and -inf fall to 0, +inf to levels through the clamp
    r = __fadd_rn(fl, fr > 0.5f ? 1.0f : 0.0f);
  }
  r = fminf(fmaxf(r, 0.0f), levels);  // fmaxf maps NaN to 0 (`as u8` of NaN)
  return (uint32_t)r;
}

// two independent fused multiply-adds in one instruction (fma.rn.f32x2,
// sm_100); each element is rounded once, exactly as __fmaf_rn
__device__ __forceinline__ float2 ffma2(float2 a, float2 b, float2 c) {
  unsigned long long A, B, Cc, Dd;
  asm("mov.b64 %0, {%1, %2};" : "=l"(A) : "f"(a.x), "f"(a.y));
  asm("mov.b64 %0, {%1, %2};" : "=l"(B) : "f"(b.x), "f"(b.y));
  asm("mov.b64 %0, {%1, %2};" : "=l"(Cc) : "f"(c.x), "f"(c.y));
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(Dd) : "l"(A), "l"(B), "l"(Cc));
  float2 d;
  asm("mov.b64 {%0, %1}, %2;" : "=f"(d.x), "=f"(d.y) : "l"(Dd));
  return d;
}

// ---- bounded waits shared by every kernel that waits ----------------------
// device clock in nanoseconds
__device__ __forceinline__ unsigned long long dev_ns() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}
// a wait gives up after this many polls or this much time, whichever is first
constexpr uint32_t kWaitPolls = 1u << 22;
constexpr unsigned long long kWaitNs = 1000000000ull;  // 1 s

// waits until the phase of `parity` of the mbarrier at shared address `bar`
// has completed. false when the wait gave up: the poll or time limit ran
// out, or `abort_flag` (optional, shared memory) was raised by another warp.
__device__ __forceinline__ bool mbar_wait_bounded(uint32_t bar, uint32_t parity, unsigned long long limit_ns,
                                                  const volatile int* abort_flag = nullptr) {
  unsigned long long t0 = 0;
  for (uint32_t i = 0; i < kWaitPolls; ++i) {
    uint32_t done;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
        : "=r"(done)
        : "r"(bar), "r"(parity)
        : "memory");
    if (done) return true;
    if ((i & 255u) == 0u) {  // the clock and the flag are read every 256 polls
      const unsigned long long t = dev_ns();
      if (i == 0) t0 = t;
      else if (t - t0 > limit_ns) return false;
      if (abort_flag && *abort_flag) return false;
    }
  }
  return false;
}

// ---- codes of one row, fetched ahead of their use ---------------------------
// The codes of a row (INT4: nibbles, INT8: bytes, flat index `first` onwards)
// as the aligned 32-bit words that cover them. Loading only fills registers,
// so the loads stay in flight until the codes are taken apart, when the row
// is dequantized; words past the end of the buffer (nbytes) are assembled
// from the bytes that exist, so nothing outside it is read.
template <bool INT4, int K>
constexpr int code_words() {
  return INT4 ? (K - 1) / 8 + 2 : (K - 1) / 4 + 2;
}
template <int NW>
struct CodeWords {
  uint32_t w[NW];
  uint32_t base;  // position of code 0 in the window: nibbles (INT4) or bytes (INT8)
};
template <bool INT4, int NW>
__device__ __forceinline__ void load_code_words(const uint8_t* __restrict__ codes, size_t nbytes, size_t first,
                                                bool ok, CodeWords<NW>& cw) {
  const size_t b0 = INT4 ? (first >> 1) : first;
  const size_t w0 = b0 & ~(size_t)3;
  cw.base = INT4 ? (uint32_t)(first - 2 * w0) : (uint32_t)(first - w0);
#pragma unroll
  for (int j = 0; j < NW; ++j) {
    const size_t a = w0 + 4 * (size_t)j;
    uint32_t v = 0u;
    if (ok) {
      if (a + 4 <= nbytes) {
        v = __ldg(reinterpret_cast<const uint32_t*>(codes + a));
      } else {
#pragma unroll
        for (int b = 0; b < 4; ++b)
          if (a + b < nbytes) v |= (uint32_t)codes[a + b] << (8 * b);
      }
    }
    cw.w[j] = v;
  }
}
// code k of the row (k a compile-time constant after unrolling, so the word
// indices are static); low nibble first within a byte, as the packing
template <bool INT4, int NW>
__device__ __forceinline__ uint32_t code_at(const CodeWords<NW>& cw, int k) {
  const int j = INT4 ? (k >> 3) : (k >> 2);
  const uint32_t p = cw.base + (uint32_t)(INT4 ? (k & 7) : (k & 3));
  const uint64_t v = ((uint64_t)cw.w[j + 1] << 32) | cw.w[j];
  return INT4 ? (uint32_t)(v >> (4 * p)) & 0xFu : (uint32_t)(v >> (8 * p)) & 0xFFu;
}

__device__ __forceinline__ float dq(uint32_t q, float scale, float mn) {
  return __fadd_rn(__fmul_rn((float)q, scale), mn);
}

// order-preserving int image of a (non-NaN, canonical) float, for atomicMin/Max
__device__ __forceinline__ int fkey(float f) {
  const int i = __float_as_int(f);
  return i >= 0 ? i : (i ^ 0x7FFFFFFF);
}
__device__ __forceinline__ float kfloat(int k) { return __int_as_float(k >= 0 ? k : (k ^ 0x7FFFFFFF)); }

#endif  // __CUDACC__

// ---- kernel launchers (return the launch error, if any) -------------------
// quantization (kvf_quant.cu)
// minmax_keys: scratch of 3 * H * D ints for per-channel (unused per-token)
cudaError_t launch_quantize_codes(const void* x, int in_dtype, size_t H, size_t T, size_t D,
                                  int data_type, int axis, uint8_t* codes, float* scales,
                                  float* mins, int* minmax_keys, cudaStream_t st);
// per-token KIVI for even D <= 128 whose D is not a multiple of 4 (or any
// even D): codes written packed (INT4) or as bytes (INT8), optional byte
// histogram; cudaErrorNotSupported when the shape or alignment does not fit
cudaError_t launch_quantize_token_pairs(const void* x, int in_dtype, size_t H, size_t T, size_t D, int data_type,
                                       uint8_t* out, float* scales, float* mins, uint32_t* hist, cudaStream_t st);
cudaError_t launch_pack_int4(const uint8_t* codes, size_t n, uint8_t* packed, uint32_t* hist,
                             cudaStream_t st);
// per-channel quantization in one launch (a thread-block cluster per head,
// partial ranges exchanged through distributed shared memory; the codes pass
// re-reads the tokens from L2): INT8 codes or INT4 bytes packed over the flat
// index into `out`, scales/mins [H, D], optional histogram of the bytes
// written. cudaErrorNotSupported when D / 4 is not a power of two or D > 128.
cudaError_t launch_quantize_channel_cluster(const void* x, int in_dtype, size_t H, size_t T, size_t D, int data_type,
                                            uint8_t* out, float* scales, float* mins, uint32_t* hist,
                                            cudaStream_t st);
// kmin/kmax <- keys of +inf / -inf
cudaError_t launch_minmax_init(int* kmin, int* kmax, size_t np, cudaStream_t st);
// codes (+ INT4 packing, + optional histogram) of projected keys P [H,T,R]
// whose per-(head, r) min/max keys are final; also writes scales/mins [H,R]
cudaError_t launch_quantpack_channel(const float* P, size_t H, size_t T, size_t R, const int* kmin,
                                     const int* kmax, int data_type, float* scales, float* mins,
                                     uint8_t* out, uint32_t* hist, cudaStream_t st);
cudaError_t launch_histogram(const uint8_t* data, size_t n, uint32_t* hist, cudaStream_t st);
cudaError_t launch_dequantize(const uint8_t* packed, const float* scales, const float* mins,
                              int data_type, int axis, size_t H, size_t T, size_t D, float* out,
                              cudaStream_t st);

// projection / calibration / gram (kvf_project.cu)
size_t project_num_tiles(size_t T);
// outputs of the projection kernel; mode 0: P; mode 1: P + per-(head, r)
// min/max keys (kmin/kmax, initialised to +inf/-inf keys); mode 2: per-token
// codes + scales/mins (R <= 32). cpart (optional): key calibration partials,
// project_num_tiles(T) per head.
// mode 2 writes either unpacked codes (`codes`) or, when `packed` is set,
// INT4 bytes packed over the flat index (callers set it only when every
// 128-token tile starts at an even flat index: R or T even); `hist`, when
// set, counts the bytes written (packed bytes, or INT8 codes).
struct ProjectOut {
  int mode = 0;
  float* P = nullptr;
  double* cpart = nullptr;
  int* kmin = nullptr;
  int* kmax = nullptr;
  uint8_t* codes = nullptr;
  uint8_t* packed = nullptr;
  uint32_t* hist = nullptr;
  float* scales = nullptr;
  float* mins = nullptr;
  float levels = 15.0f;
  unsigned* status = nullptr;  // device status word: a bounded wait that expires sets kDevErrTimeout
};
cudaError_t launch_project(const void* x, int in_dtype, size_t H, size_t T, size_t D,
                           const float* basis_vt, const uint64_t* ranks, size_t R, const ProjectOut& o,
                           cudaStream_t st);
size_t calib_partial_tiles(size_t T, size_t D);
cudaError_t launch_calib_partials(const void* x, int in_dtype, size_t H, size_t T, size_t D,
                                  double* calib_part, cudaStream_t st);
// no-allocation calibration: partials for up to kCalibStaticSlots (head, tile)
// pairs in a file-scope device array; its address for `device` (current)
constexpr size_t kCalibStaticSlots = 65536;
cudaError_t calib_static_scratch(int device, double** out);
// the partials are consumed: each head's first slot is overwritten
cudaError_t launch_calib_finalize(double* calib_part, size_t H, size_t tiles, size_t T,
                                  size_t D, float* scores, cudaStream_t st);
// tensor-core projection with the per-token quantization epilogue (mode 2 of
// ProjectOut; kvf_project_tc.cu): f16 input, D == 128, R <= 64;
// cudaErrorNotSupported otherwise (the caller then uses launch_project).
// exact: codes identical to launch_project's; otherwise codes of the
// tensor-core coefficients (relative error near 2^-22 of the exact ones)
cudaError_t launch_project_tc(const void* x, int in_dtype, size_t H, size_t T, size_t D, const float* basis_vt,
                              const uint64_t* ranks, size_t R, bool exact, const ProjectOut& o, cudaStream_t st);
bool project_tc_fits(const void* x, int in_dtype, size_t H, size_t T, size_t D, const float* basis_vt, size_t R);
// cuTensorMapEncodeTiled from the driver (nullptr when unavailable), looked up once
void* tensor_map_encode_fn();
// tensor-core reconstruction (kvf_tc.cu): D == 128, R <= 64; cudaErrorNotSupported
// when the shape or the driver does not allow it (the caller then uses the
// CUDA-core kernels)
cudaError_t launch_reconstruct_tc(const uint8_t* codes, const float* raw, const float* scales, const float* mins,
                                  int data_type, int axis, size_t H, size_t T, size_t R, size_t D,
                                  const float* basis_vt, const uint64_t* ranks, float* out, unsigned* status,
                                  cudaStream_t st);
// packed codes (or raw f32 when data_type == KVF_F32) + params + basis -> f32 [H,T,D];
// exact: the reference's separately rounded order on CUDA cores; otherwise
// engine (kvf_recon_engine) picks the tcgen05 kernel where the shape allows it
cudaError_t launch_dequant_reconstruct(const uint8_t* codes, const float* raw, const float* scales,
                                       const float* mins, int data_type, int axis, size_t H,
                                       size_t T, size_t R, size_t D, const float* basis_vt,
                                       const uint64_t* ranks, int exact, int engine, float* out,
                                       unsigned* status, cudaStream_t st);
size_t gram_num_tiles(size_t T);
cudaError_t launch_gram(const void* x, int in_dtype, size_t H, size_t T, size_t D,
                        float* partial, double* gram, cudaStream_t st);

// rANS (kvf_rans.cu)
// encode and decode build the model from the 256 counts themselves
// container of n symbols into out (capacity rans_max_len), its length into
// out_len; lookback: one zeroed-here word per chunk plus one (the block ticket)
cudaError_t launch_rans_encode(const uint8_t* data, size_t n, uint32_t chunk, const uint32_t* freq,
                               unsigned long long* lookback, uint8_t* out, uint64_t* out_len, unsigned* status,
                               cudaStream_t st);
cudaError_t launch_rans_decode(const uint8_t* comp, size_t comp_len, const uint64_t* comp_len_dev,
                               const uint32_t* freq, size_t n, uint8_t* out, unsigned* status,
                               cudaStream_t st);

// self-tests of the bounded waits (kvf_selftest_wait_timeout): each runs the
// wait the kernels use against a barrier or status word that nothing
// completes, so it gives up after limit_ns and sets kDevErrTimeout
cudaError_t launch_selftest_mbar(unsigned* status, unsigned long long limit_ns, cudaStream_t st);
// lb: two zeroed look-back words
cudaError_t launch_selftest_lookback(unsigned long long* lb, unsigned* status, unsigned long long limit_ns,
                                     cudaStream_t st);

// ---- batched short chunks (kvf_batch.cu) ------------------------------------
// one tensor of one layer: input [H, T, D], optional basis [H, cols, D] and
// ranks [H] (projection), outputs: codes (INT4 packed over the flat index or
// INT8), scales/mins (per channel [H, cols] or per token [H, T]), optional
// byte histogram, optional f32 reconstruction [H, T, D]
struct BatchTensor {
  const void* x = nullptr;
  const float* bvt = nullptr;
  const uint64_t* ranks = nullptr;
  int cols = 0;
  int axis = 0;
  int data_type = 0;
  float levels = 15.0f;
  uint8_t* packed = nullptr;
  float* scales = nullptr;
  float* mins = nullptr;
  uint32_t* hist = nullptr;
  float* out = nullptr;
};
// whether one launch can take layers of this shape (T <= 128, D <= 128,
// D % 4 == 0, cols <= 64 with a basis, a head's INT4 block on a byte)
bool chunk_batch_fits(int in_dtype, size_t H, size_t T, size_t D, size_t cols_max, bool proj);
// descs: 2 * L host descriptors (keys then values of each layer), passed as
// the kernel parameter, up to 128 layers a launch; grid (H, 2, layers).
// exact: the reconstruction rounds each product and sum separately.
cudaError_t launch_chunk_batch(const BatchTensor* descs, size_t L, int in_dtype, size_t H, size_t T, size_t D,
                               size_t cols_max, bool proj, int exact, cudaStream_t st);

// ---- fused dequantize + decode attention (kvf_attn.cu) ----------------------
// keys per channel [H, T, Rk] codes with [H, Rk] params, values per token
// [H, T, Rv] codes with [H, T] params; kvt / vvt [H, R, D] bases or NULL
// (then R = D); part: attention_scratch_floats(H, T, Rv) floats; out [H, D]
size_t attention_tiles(size_t T);
size_t attention_scratch_floats(size_t H, size_t T, size_t Rv);
cudaError_t launch_attention(const uint8_t* kc, int kdt, const uint8_t* vc, int vdt, const float* q,
                             const float* ks, const float* km, const float* vs, const float* vm, const float* kvt,
                             const uint64_t* kranks, const float* vvt, const uint64_t* vranks, size_t H, size_t T,
                             size_t D, size_t Rk, size_t Rv, float scale, float* part, float* out,
                             cudaStream_t st);

}  // namespace kvf
