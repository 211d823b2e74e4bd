// Projection, reconstruction, calibration and Gram kernels (sm_100a).
//
// Projection (crates/kvforge-cpu/src/projection.rs:61-140): the reference
// forms U_k * S_k from an SVD; the same coefficients are X * V_k^T against the
// calibrated basis. Each coefficient is one fused multiply-add chain over
// c = 0..D-1 starting at +0.0 -- the order the CPU oracle uses, so projected
// values (and therefore the quantized codes) are bit-identical to it.
// Coefficients r >= rank_h are written as +0.0 (projection.rs:96).
//
// Reconstruction (projection.rs:142-172): out[h,t,c] = sum_{r<rank_h} p[r] * vt[r,c]
// in r order. EXACT=true rounds the product and the sum separately, as the
// reference does; EXACT=false fuses them (one FMA per term).
//
// Calibration (crates/kvforge-cpu/src/calibration.rs:25-73): fp64 sum and sum
// of squares per head; partials per block are combined in a fixed order, so
// the result is deterministic (it differs from the sequential reference only
// in fp64 rounding order).
#include <algorithm>
#include <cmath>
#include <mutex>

#include "kvf_internal.cuh"

namespace kvf {
namespace {

constexpr int kProjThreads = 128;
constexpr int kRecRows = 128;                    // token rows per reconstruct block
constexpr int kCalibTile = 1 << 16;              // elements per calibration block
constexpr int kGramTile = 512;                   // tokens per Gram block

template <typename TIn>
struct Vec;
template <>
struct Vec<float> {
  static constexpr int N = 4;
  __device__ static void load(const float* p, float* o) {
    const float4 v = __ldg(reinterpret_cast<const float4*>(p));
    o[0] = v.x; o[1] = v.y; o[2] = v.z; o[3] = v.w;
  }
};
template <>
struct Vec<__half> {
  static constexpr int N = 8;
  __device__ static void load(const __half* p, float* o) {
    const uint4 u = __ldg(reinterpret_cast<const uint4*>(p));
    const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&w[k]));
      o[2 * k] = f.x;
      o[2 * k + 1] = f.y;
    }
  }
};

__device__ __forceinline__ float ldf(const float* p, size_t i) { return __ldg(p + i); }
__device__ __forceinline__ float ldf(const __half* p, size_t i) { return __half2float(__ldg(p + i)); }

template <typename T>
__device__ __forceinline__ T warp_sum(T v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// fixed-order block reduction of two doubles; thread 0 gets the result
__device__ __forceinline__ void block_sum2(double& a, double& b) {
  __shared__ double sa[32], sb[32];
  a = warp_sum(a);
  b = warp_sum(b);
  const int w = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) { sa[w] = a; sb[w] = b; }
  __syncthreads();
  if (threadIdx.x == 0) {
    double ta = 0.0, tb = 0.0;
    for (int k = 0; k < (int)(blockDim.x >> 5); ++k) { ta += sa[k]; tb += sb[k]; }
    a = ta;
    b = tb;
  }
}

// ---- projection -------------------------------------------------------------
// grid (ceil(T / 128), H), 128 threads, one token row per thread. The row is
// read in 256-byte segments whose sixteen 16-byte loads are issued together, so
// a whole segment is in flight at once (the kernel is bound by HBM latency
// otherwise). The basis of head h sits transposed in shared memory, vT[c][r],
// so the RG basis values of one c are a broadcast float4 load. Epilogues:
//   MODE 0: write P [H,T,R];
//   MODE 1: write P and fold each column into per-(head, r) min/max with
//           order-preserving integer atomics (keys: per-channel parameters
//           need every token before any code can be formed);
//   MODE 2: quantize the row per token at once -- codes [H,T,R] bytes plus a
//           scale/min per token; P never reaches memory (values; R <= RG).
template <typename TIn>
struct Seg;
template <>
struct Seg<__half> {
  static constexpr int PV = 8;  // elements per 16-byte vector
  __device__ static void unpack(const uint4& u, float* o) {
    const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&w[k]));
      o[2 * k] = f.x;
      o[2 * k + 1] = f.y;
    }
  }
};
template <>
struct Seg<float> {
  static constexpr int PV = 4;
  __device__ static void unpack(const uint4& u, float* o) {
    o[0] = __uint_as_float(u.x);
    o[1] = __uint_as_float(u.y);
    o[2] = __uint_as_float(u.z);
    o[3] = __uint_as_float(u.w);
  }
};

template <typename TIn, int RG, bool VEC, bool CALIB, int MODE>
__global__ void __launch_bounds__(kProjThreads) k_project(const TIn* __restrict__ x, int T, int D,
                                                        const float* __restrict__ bvt,
                                                        const uint64_t* __restrict__ ranks, int R,
                                                        int Rpad, ProjectOut o) {
  extern __shared__ __align__(16) float vT[];  // [D][Rpad]
  const int h = blockIdx.y;
  const uint64_t rk = ranks[h];
  const int rank = (int)(rk < (uint64_t)R ? rk : (uint64_t)R);
  const float* B = bvt + (size_t)h * R * D;
  for (int i = threadIdx.x; i < D * Rpad; i += blockDim.x) {
    const int c = i / Rpad, r = i - c * Rpad;
    vT[i] = (r < rank) ? B[(size_t)r * D + c] : 0.0f;
  }
  __syncthreads();

  const int t = blockIdx.x * kProjThreads + threadIdx.x;
  const bool ok = t < T;
  const size_t g = (size_t)h * T + (ok ? t : 0);
  const TIn* xr = x + g * D;
  double s1 = 0.0, s2 = 0.0;
  for (int rg = 0; rg < R; rg += RG) {
    float acc[RG];
#pragma unroll
    for (int r = 0; r < RG; ++r) acc[r] = 0.0f;
    if (VEC) {
      constexpr int PV = Seg<TIn>::PV;
      for (int c0 = 0; c0 < D; c0 += 16 * PV) {
        const int nv = min(16, (D - c0) / PV);
        uint4 raw[16];
#pragma unroll
        for (int j = 0; j < 16; ++j)
          raw[j] = (ok && j < nv) ? __ldg(reinterpret_cast<const uint4*>(xr + c0) + j) : make_uint4(0u, 0u, 0u, 0u);
#pragma unroll
        for (int j = 0; j < 16; ++j) {
          if (j < nv) {
            float xv[PV];
            Seg<TIn>::unpack(raw[j], xv);
            if (CALIB && rg == 0) {
#pragma unroll
              for (int k = 0; k < PV; ++k) {
                const double v = (double)xv[k];
                s1 += v;
                s2 += v * v;
              }
            }
#pragma unroll
            for (int k = 0; k < PV; ++k) {
              const float4* vr = reinterpret_cast<const float4*>(vT + (size_t)(c0 + j * PV + k) * Rpad + rg);
#pragma unroll
              for (int q = 0; q < RG / 4; ++q) {
                const float4 v = vr[q];
                acc[4 * q + 0] = __fmaf_rn(xv[k], v.x, acc[4 * q + 0]);
                acc[4 * q + 1] = __fmaf_rn(xv[k], v.y, acc[4 * q + 1]);
                acc[4 * q + 2] = __fmaf_rn(xv[k], v.z, acc[4 * q + 2]);
                acc[4 * q + 3] = __fmaf_rn(xv[k], v.w, acc[4 * q + 3]);
              }
            }
          }
        }
      }
    } else {
      for (int c = 0; c < D; ++c) {
        const float xv = ok ? ldf(xr, c) : 0.0f;
        if (CALIB && rg == 0) {
          const double v = (double)xv;
          s1 += v;
          s2 += v * v;
        }
        const float4* vr = reinterpret_cast<const float4*>(vT + (size_t)c * Rpad + rg);
#pragma unroll
        for (int q = 0; q < RG / 4; ++q) {
          const float4 v = vr[q];
          acc[4 * q + 0] = __fmaf_rn(xv, v.x, acc[4 * q + 0]);
          acc[4 * q + 1] = __fmaf_rn(xv, v.y, acc[4 * q + 1]);
          acc[4 * q + 2] = __fmaf_rn(xv, v.z, acc[4 * q + 2]);
          acc[4 * q + 3] = __fmaf_rn(xv, v.w, acc[4 * q + 3]);
        }
      }
    }
    // coefficients r >= rank_h are +0.0 (projection.rs:96)
#pragma unroll
    for (int r = 0; r < RG; ++r)
      if (rg + r >= rank) acc[r] = 0.0f;
    if (MODE == 0 || MODE == 1) {
      float* pr = o.P + g * R;
#pragma unroll
      for (int r = 0; r < RG; ++r) {
        const int rr = rg + r;
        if (rr < R) {  // warp-uniform
          if (ok) pr[rr] = acc[r];
          if (MODE == 1) {
            float mn = INFINITY, mx = -INFINITY;
            if (ok) mm_update(acc[r], mn, mx);
            warp_minmax(mn, mx);
            if ((threadIdx.x & 31) == 0) {
              atomicMin(&o.kmin[(size_t)h * R + rr], fkey(mn));
              atomicMax(&o.kmax[(size_t)h * R + rr], fkey(mx));
            }
          }
        }
      }
    } else {  // MODE 2: per-token quantization of the whole row (R <= RG)
      float mn = INFINITY, mx = -INFINITY;
#pragma unroll
      for (int r = 0; r < RG; ++r)
        if (r < R) mm_update(acc[r], mn, mx);
      const float scale = make_scale(mn, mx, o.levels);
      if (ok) {
        o.scales[g] = scale;
        o.mins[g] = mn;
        uint8_t* cr = o.codes + g * R;
#pragma unroll
        for (int r = 0; r < RG; ++r)
          if (r < R) cr[r] = (uint8_t)qcode(acc[r], mn, scale, o.levels);
      }
    }
  }
  if (CALIB) {
    block_sum2(s1, s2);
    if (threadIdx.x == 0) {
      const size_t slot = (size_t)h * gridDim.x + blockIdx.x;
      o.cpart[2 * slot] = s1;
      o.cpart[2 * slot + 1] = s2;
    }
  }
}

template <typename TIn, int RG, bool VEC, bool CALIB, int MODE>
cudaError_t project_launch(const TIn* x, size_t H, size_t T, size_t D, const float* bvt, const uint64_t* ranks,
                           size_t R, const ProjectOut& o, cudaStream_t st) {
  const int Rpad = (int)(((R + RG - 1) / RG) * RG);
  const size_t smem = (size_t)D * Rpad * sizeof(float);
  const dim3 grid((unsigned)((T + kProjThreads - 1) / kProjThreads), (unsigned)H);
  auto kern = k_project<TIn, RG, VEC, CALIB, MODE>;
  if (smem > kSmemOptIn) {
    const cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
  }
  kern<<<grid, kProjThreads, smem, st>>>(x, (int)T, (int)D, bvt, ranks, (int)R, Rpad, o);
  note_launches(1);
  return cudaGetLastError();
}

template <typename TIn, int RG, bool VEC>
cudaError_t project_mode(const TIn* x, size_t H, size_t T, size_t D, const float* bvt, const uint64_t* ranks,
                         size_t R, const ProjectOut& o, cudaStream_t st) {
  const bool calib = o.cpart != nullptr;
#define KVF_PL(C, M) return project_launch<TIn, RG, VEC, C, M>(x, H, T, D, bvt, ranks, R, o, st)
  if (o.mode == 1) {
    if (calib) KVF_PL(true, 1);
    KVF_PL(false, 1);
  }
  if (o.mode == 2) {
    if (calib) KVF_PL(true, 2);
    KVF_PL(false, 2);
  }
  if (calib) KVF_PL(true, 0);
  KVF_PL(false, 0);
#undef KVF_PL
}

template <typename TIn, bool VEC>
cudaError_t project_vec(const TIn* x, size_t H, size_t T, size_t D, const float* bvt, const uint64_t* ranks,
                        size_t R, const ProjectOut& o, cudaStream_t st) {
  if (R <= 4) return project_mode<TIn, 4, VEC>(x, H, T, D, bvt, ranks, R, o, st);
  if (R <= 8) return project_mode<TIn, 8, VEC>(x, H, T, D, bvt, ranks, R, o, st);
  if (R <= 16) return project_mode<TIn, 16, VEC>(x, H, T, D, bvt, ranks, R, o, st);
  if (o.mode == 2 && R > 32) return cudaErrorInvalidValue;
  return project_mode<TIn, 32, VEC>(x, H, T, D, bvt, ranks, R, o, st);
}

template <typename TIn>
cudaError_t project_typed(const TIn* x, size_t H, size_t T, size_t D, const float* bvt, const uint64_t* ranks,
                          size_t R, const ProjectOut& o, cudaStream_t st) {
  if (D % Seg<TIn>::PV == 0 && aligned(x, 16)) return project_vec<TIn, true>(x, H, T, D, bvt, ranks, R, o, st);
  return project_vec<TIn, false>(x, H, T, D, bvt, ranks, R, o, st);
}

// ---- calibration partials without projection ----------------------------------
template <typename TIn>
__global__ void __launch_bounds__(256) k_calib_partials(const TIn* __restrict__ x, size_t per_head,
                                                        double* __restrict__ cpart) {
  const int h = blockIdx.y;
  const size_t e0 = (size_t)blockIdx.x * kCalibTile;
  const size_t e1 = (e0 + kCalibTile < per_head) ? e0 + kCalibTile : per_head;
  const TIn* xh = x + (size_t)h * per_head;
  double s1 = 0.0, s2 = 0.0;
  for (size_t i = e0 + threadIdx.x; i < e1; i += blockDim.x) {
    const double v = (double)ldf(xh, i);
    s1 += v;
    s2 += v * v;
  }
  block_sum2(s1, s2);
  if (threadIdx.x == 0) {
    const size_t slot = (size_t)h * gridDim.x + blockIdx.x;
    cpart[2 * slot] = s1;
    cpart[2 * slot + 1] = s2;
  }
}

// calibration.rs:56-71: variance per head, clamped at 0, normalised by the max
// (uniform 0.5 when the max is below 1e-12). One block; thread h sums its
// head's partials in block order.
__global__ void k_calib_finalize(const double* __restrict__ cpart, int H, int tiles, double n,
                                 float* __restrict__ scores) {
  extern __shared__ double var[];
  for (int h = threadIdx.x; h < H; h += blockDim.x) {
    double s1 = 0.0, s2 = 0.0;
    for (int k = 0; k < tiles; ++k) {
      s1 += cpart[2 * ((size_t)h * tiles + k)];
      s2 += cpart[2 * ((size_t)h * tiles + k) + 1];
    }
    const double mean = s1 / n;
    const double v = (s2 / n) - (mean * mean);
    var[h] = (isnan(v) || v < 0.0) ? 0.0 : v;  // variance.max(0.0)
  }
  __syncthreads();
  __shared__ double maxv;
  if (threadIdx.x == 0) {
    double m = 0.0;
    for (int h = 0; h < H; ++h) m = var[h] > m ? var[h] : m;
    maxv = m;
  }
  __syncthreads();
  for (int h = threadIdx.x; h < H; h += blockDim.x)
    scores[h] = (maxv < 1e-12) ? 0.5f : (float)(var[h] / maxv);
}

// ---- dequantize + reconstruct ------------------------------------------------
// grid (ceil(T / 128), H), 128 threads. Phase 1: the block dequantizes its
// 128 x R coefficients (q * scale + min, separate roundings) into shared
// memory, transposed dT[r][row]. Phase 2: warp w owns row groups of 8, each
// lane four output columns; per r one float4 of the basis (held in shared
// memory) and two broadcast float4 of coefficients feed 32 multiply-adds.
// Output rows are written with streaming 16-byte stores.
template <int MODE, bool EXACT>  // MODE 0: raw f32 coefficients, 1: INT8 codes, 2: INT4 codes
__global__ void __launch_bounds__(128) k_dequant_reconstruct(
    const uint8_t* __restrict__ codes, const float* __restrict__ raw,
    const float* __restrict__ scales, const float* __restrict__ mins, int axis, int T, int R, int D,
    const float* __restrict__ bvt, const uint64_t* __restrict__ ranks, float* __restrict__ out) {
  extern __shared__ __align__(16) float sm[];
  float* vs = sm;                      // [rank][D]
  float* dT = sm + (size_t)R * D;      // [R][kRecRows]
  const int h = blockIdx.y;
  const uint64_t rk = ranks[h];
  const int rank = (int)(rk < (uint64_t)R ? rk : (uint64_t)R);
  const size_t t0 = (size_t)blockIdx.x * kRecRows;
  const float* B = bvt + (size_t)h * R * D;
  for (int i = threadIdx.x; i < rank * D; i += blockDim.x) vs[i] = __ldg(B + i);
  const size_t flat0 = ((size_t)h * T + t0) * R;
  for (int e = threadIdx.x; e < kRecRows * R; e += blockDim.x) {
    const int row = e / R, r = e - row * R;
    float d = 0.0f;
    if (r < rank && t0 + row < (size_t)T) {
      const size_t fi = flat0 + e;
      if (MODE == 0) {
        d = __ldg(raw + fi);
      } else {
        uint32_t q = codes[MODE == 2 ? (fi >> 1) : fi];
        if (MODE == 2) q = (fi & 1) ? (q >> 4) & 0xF : q & 0xF;
        const size_t p = (axis == KVF_PER_CHANNEL) ? (size_t)h * R + r : (size_t)h * T + t0 + row;
        d = __fadd_rn(__fmul_rn((float)q, __ldg(scales + p)), __ldg(mins + p));
      }
    }
    dT[r * kRecRows + row] = d;
  }
  __syncthreads();
  const int w = threadIdx.x >> 5, lane = threadIdx.x & 31;
  for (int cq = lane; cq < (D >> 2); cq += 32) {
    for (int g8 = w; g8 < kRecRows / 8; g8 += 4) {
      float4 acc[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) acc[i] = make_float4(0.f, 0.f, 0.f, 0.f);
      for (int r = 0; r < rank; ++r) {
        const float4 v = *reinterpret_cast<const float4*>(vs + (size_t)r * D + 4 * cq);
        const float4 d0 = *reinterpret_cast<const float4*>(dT + r * kRecRows + 8 * g8);
        const float4 d1 = *reinterpret_cast<const float4*>(dT + r * kRecRows + 8 * g8 + 4);
        const float dd[8] = {d0.x, d0.y, d0.z, d0.w, d1.x, d1.y, d1.z, d1.w};
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          if (EXACT) {
            acc[i].x = __fadd_rn(acc[i].x, __fmul_rn(dd[i], v.x));
            acc[i].y = __fadd_rn(acc[i].y, __fmul_rn(dd[i], v.y));
            acc[i].z = __fadd_rn(acc[i].z, __fmul_rn(dd[i], v.z));
            acc[i].w = __fadd_rn(acc[i].w, __fmul_rn(dd[i], v.w));
          } else {
            acc[i].x = __fmaf_rn(dd[i], v.x, acc[i].x);
            acc[i].y = __fmaf_rn(dd[i], v.y, acc[i].y);
            acc[i].z = __fmaf_rn(dd[i], v.z, acc[i].z);
            acc[i].w = __fmaf_rn(dd[i], v.w, acc[i].w);
          }
        }
      }
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const size_t t = t0 + 8 * g8 + i;
        if (t < (size_t)T) __stcs(reinterpret_cast<float4*>(out + ((size_t)h * T + t) * D + 4 * cq), acc[i]);
      }
    }
  }
}

// any D: one thread per output element
template <int MODE, bool EXACT>
__global__ void __launch_bounds__(256) k_dequant_reconstruct_scalar(
    const uint8_t* __restrict__ codes, const float* __restrict__ raw,
    const float* __restrict__ scales, const float* __restrict__ mins, int axis, size_t H, size_t T,
    int R, int D, const float* __restrict__ bvt, const uint64_t* __restrict__ ranks,
    float* __restrict__ out) {
  const size_t total = H * T * (size_t)D;
  for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (size_t)gridDim.x * blockDim.x) {
    const size_t g = i / D;
    const int c = (int)(i - g * D);
    const size_t h = g / T;
    const uint64_t rk = ranks[h];
    const int rank = (int)(rk < (uint64_t)R ? rk : (uint64_t)R);
    float acc = 0.0f;
    for (int r = 0; r < rank; ++r) {
      const size_t fi = g * R + r;
      float d;
      if (MODE == 0) {
        d = raw[fi];
      } else {
        uint32_t q = codes[MODE == 2 ? (fi >> 1) : fi];
        if (MODE == 2) q = (fi & 1) ? (q >> 4) & 0xF : q & 0xF;
        const size_t p = (axis == KVF_PER_CHANNEL) ? h * R + r : g;
        d = __fadd_rn(__fmul_rn((float)q, scales[p]), mins[p]);
      }
      const float v = bvt[(h * R + r) * D + c];
      acc = EXACT ? __fadd_rn(acc, __fmul_rn(d, v)) : __fmaf_rn(d, v, acc);
    }
    out[i] = acc;
  }
}

template <int MODE, bool EXACT>
cudaError_t dequant_reconstruct_mode(const uint8_t* codes, const float* raw, const float* scales,
                                     const float* mins, int axis, size_t H, size_t T, size_t R,
                                     size_t D, const float* bvt, const uint64_t* ranks, float* out,
                                     cudaStream_t st) {
  const size_t smem = ((size_t)R * D + (size_t)R * kRecRows) * sizeof(float);
  if (D % 4 == 0 && smem <= 200 * 1024 && aligned(out, 16)) {
    auto kern = k_dequant_reconstruct<MODE, EXACT>;
    if (smem > kSmemOptIn) {
      cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
      if (e != cudaSuccess) return e;
    }
    const dim3 grid((unsigned)((T + kRecRows - 1) / kRecRows), (unsigned)H);
    kern<<<grid, 128, smem, st>>>(codes, raw, scales, mins, axis, (int)T, (int)R, (int)D, bvt, ranks, out);
  } else {
    const size_t total = H * T * D;
    const unsigned grid = (unsigned)std::min<size_t>((total + 255) / 256, 148 * 16);
    k_dequant_reconstruct_scalar<MODE, EXACT><<<grid ? grid : 1, 256, 0, st>>>(
        codes, raw, scales, mins, axis, H, T, (int)R, (int)D, bvt, ranks, out);
  }
  note_launches(1);
  return cudaGetLastError();
}

// ---- Gram matrix X_h^T X_h for the basis step ---------------------------------
// grid (ceil(T / 512), H), 256 threads as a 16 x 16 grid of 8 x 8 output tiles
// (D % 8 == 0, D <= 128); 32 token rows at a time are staged in shared memory
// as f32. Per-block partials are f32 sums of at most 512 products; the reduce
// kernel adds them in fp64 in block order.
template <typename TIn>
__global__ void __launch_bounds__(256) k_gram_tile(const TIn* __restrict__ x, size_t T, int D,
                                                   float* __restrict__ partial) {
  __shared__ __align__(16) float xs[32][128];
  const int h = blockIdx.y;
  const size_t t0 = (size_t)blockIdx.x * kGramTile;
  const size_t t1 = (t0 + kGramTile < T) ? t0 + kGramTile : T;
  const int ti = threadIdx.x >> 4, tj = threadIdx.x & 15;
  const int nt = D >> 3;
  const bool active = ti < nt && tj < nt;
  float acc[8][8];
#pragma unroll
  for (int i = 0; i < 8; ++i)
#pragma unroll
    for (int j = 0; j < 8; ++j) acc[i][j] = 0.0f;
  const TIn* xh = x + (size_t)h * T * D;
  for (size_t tt = t0; tt < t1; tt += 32) {
    for (int e = threadIdx.x; e < 32 * D; e += blockDim.x) {
      const int row = e / D, c = e - row * D;
      xs[row][c] = (tt + row < t1) ? ldf(xh, (tt + row) * D + c) : 0.0f;
    }
    __syncthreads();
    if (active) {
#pragma unroll 4
      for (int k = 0; k < 32; ++k) {
        const float4 a0 = *reinterpret_cast<const float4*>(&xs[k][8 * ti]);
        const float4 a1 = *reinterpret_cast<const float4*>(&xs[k][8 * ti + 4]);
        const float4 b0 = *reinterpret_cast<const float4*>(&xs[k][8 * tj]);
        const float4 b1 = *reinterpret_cast<const float4*>(&xs[k][8 * tj + 4]);
        const float a[8] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w};
        const float b[8] = {b0.x, b0.y, b0.z, b0.w, b1.x, b1.y, b1.z, b1.w};
#pragma unroll
        for (int i = 0; i < 8; ++i)
#pragma unroll
          for (int j = 0; j < 8; ++j) acc[i][j] = __fmaf_rn(a[i], b[j], acc[i][j]);
      }
    }
    __syncthreads();
  }
  if (active) {
    float* out = partial + ((size_t)h * gridDim.x + blockIdx.x) * D * D;
#pragma unroll
    for (int i = 0; i < 8; ++i)
#pragma unroll
      for (int j = 0; j < 8; ++j) out[(size_t)(8 * ti + i) * D + 8 * tj + j] = acc[i][j];
  }
}

// any D (<= 1024): one thread per (i, j), loop over the tile's tokens
template <typename TIn>
__global__ void __launch_bounds__(256) k_gram_tile_scalar(const TIn* __restrict__ x, size_t T, int D,
                                                          float* __restrict__ partial) {
  const int h = blockIdx.y;
  const size_t t0 = (size_t)blockIdx.x * kGramTile;
  const size_t t1 = (t0 + kGramTile < T) ? t0 + kGramTile : T;
  const TIn* xh = x + (size_t)h * T * D;
  float* out = partial + ((size_t)h * gridDim.x + blockIdx.x) * D * D;
  for (int e = threadIdx.x; e < D * D; e += blockDim.x) {
    const int i = e / D, j = e - i * D;
    float acc = 0.0f;
    for (size_t t = t0; t < t1; ++t) acc = __fmaf_rn(ldf(xh, t * D + i), ldf(xh, t * D + j), acc);
    out[e] = acc;
  }
}

__global__ void k_gram_reduce(const float* __restrict__ partial, int tiles, int D,
                              double* __restrict__ gram) {
  const int h = blockIdx.y;
  const size_t DD = (size_t)D * D;
  for (size_t e = (size_t)blockIdx.x * blockDim.x + threadIdx.x; e < DD; e += (size_t)gridDim.x * blockDim.x) {
    double s = 0.0;
    for (int k = 0; k < tiles; ++k) s += (double)partial[((size_t)h * tiles + k) * DD + e];
    gram[(size_t)h * DD + e] = s;
  }
}

}  // namespace

// ---- calibration scratch that needs no allocation ------------------------------
// For callers that cannot allocate device memory (see kvf_calibrate_noalloc in
// include/kvforge.h): the per-block partial sums live in this file-scope array,
// loaded with the library and held by every GPU that loads it until the process
// exits. Host code cannot use the name as a device address; it asks the runtime
// for the address once per device (calib_static_scratch below).
static __device__ __align__(256) double g_calib_static[2 * kCalibStaticSlots];

namespace {
constexpr int kMaxDevices = 64;
std::mutex g_static_mu;
double* g_static_ptr[kMaxDevices] = {};
}  // namespace

cudaError_t calib_static_scratch(int device, double** out) {
  if (device < 0 || device >= kMaxDevices) return cudaErrorInvalidDevice;
  std::lock_guard<std::mutex> lock(g_static_mu);
  if (!g_static_ptr[device]) {
    void* p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, g_calib_static);  // device `device` is current
    if (e != cudaSuccess) return e;
    g_static_ptr[device] = static_cast<double*>(p);
  }
  *out = g_static_ptr[device];
  return cudaSuccess;
}

size_t project_num_tiles(size_t T) { return (T + kProjThreads - 1) / kProjThreads; }

cudaError_t launch_project(const void* x, int in_dtype, size_t H, size_t T, size_t D,
                           const float* basis_vt, const uint64_t* ranks, size_t R, const ProjectOut& o,
                           cudaStream_t st) {
  if (H == 0 || T == 0) return cudaSuccess;
  if (in_dtype == KVF_IN_F16)
    return project_typed(static_cast<const __half*>(x), H, T, D, basis_vt, ranks, R, o, st);
  return project_typed(static_cast<const float*>(x), H, T, D, basis_vt, ranks, R, o, st);
}

size_t calib_partial_tiles(size_t T, size_t D) {
  const size_t per_head = T * D;
  return per_head == 0 ? 1 : (per_head + kCalibTile - 1) / kCalibTile;
}

cudaError_t launch_calib_partials(const void* x, int in_dtype, size_t H, size_t T, size_t D,
                                  double* calib_part, cudaStream_t st) {
  const size_t tiles = calib_partial_tiles(T, D);
  if (H == 0) return cudaSuccess;
  const dim3 grid((unsigned)tiles, (unsigned)H);
  if (in_dtype == KVF_IN_F16)
    k_calib_partials<__half><<<grid, 256, 0, st>>>(static_cast<const __half*>(x), T * D, calib_part);
  else
    k_calib_partials<float><<<grid, 256, 0, st>>>(static_cast<const float*>(x), T * D, calib_part);
  note_launches(1);
  return cudaGetLastError();
}

cudaError_t launch_calib_finalize(const double* calib_part, size_t H, size_t tiles, size_t T,
                                  size_t D, float* scores, cudaStream_t st) {
  if (H == 0) return cudaSuccess;
  const size_t smem = H * sizeof(double);
  if (smem > kSmemOptIn) return cudaErrorInvalidValue;
  k_calib_finalize<<<1, 256, smem, st>>>(calib_part, (int)H, (int)tiles, (double)(T * D), scores);
  note_launches(1);
  return cudaGetLastError();
}

cudaError_t launch_dequant_reconstruct(const uint8_t* codes, const float* raw, const float* scales,
                                       const float* mins, int data_type, int axis, size_t H,
                                       size_t T, size_t R, size_t D, const float* basis_vt,
                                       const uint64_t* ranks, int exact, float* out,
                                       cudaStream_t st) {
  if (H == 0 || T == 0 || D == 0) return cudaSuccess;
  const int mode = raw ? 0 : (data_type == KVF_INT8 ? 1 : 2);
#define KVF_DR(M)                                                                                      \
  return exact ? dequant_reconstruct_mode<M, true>(codes, raw, scales, mins, axis, H, T, R, D, basis_vt, ranks, out, st) \
               : dequant_reconstruct_mode<M, false>(codes, raw, scales, mins, axis, H, T, R, D, basis_vt, ranks, out, st)
  if (mode == 0) { KVF_DR(0); }
  if (mode == 1) { KVF_DR(1); }
  KVF_DR(2);
#undef KVF_DR
}

size_t gram_num_tiles(size_t T) { return T == 0 ? 1 : (T + kGramTile - 1) / kGramTile; }

cudaError_t launch_gram(const void* x, int in_dtype, size_t H, size_t T, size_t D,
                        float* partial, double* gram, cudaStream_t st) {
  const size_t tiles = gram_num_tiles(T);
  if (H == 0) return cudaSuccess;
  const dim3 grid((unsigned)tiles, (unsigned)H);
  const bool fast = (D % 8 == 0) && D <= 128;
  if (in_dtype == KVF_IN_F16) {
    const __half* xp = static_cast<const __half*>(x);
    if (fast) k_gram_tile<__half><<<grid, 256, 0, st>>>(xp, T, (int)D, partial);
    else k_gram_tile_scalar<__half><<<grid, 256, 0, st>>>(xp, T, (int)D, partial);
  } else {
    const float* xp = static_cast<const float*>(x);
    if (fast) k_gram_tile<float><<<grid, 256, 0, st>>>(xp, T, (int)D, partial);
    else k_gram_tile_scalar<float><<<grid, 256, 0, st>>>(xp, T, (int)D, partial);
  }
  const size_t DD = D * D;
  const dim3 rg((unsigned)std::min<size_t>((DD + 255) / 256, 1024), (unsigned)H);
  k_gram_reduce<<<rg, 256, 0, st>>>(partial, (int)tiles, (int)D, gram);
  note_launches(2);
  return cudaGetLastError();
}

}  // namespace kvf
