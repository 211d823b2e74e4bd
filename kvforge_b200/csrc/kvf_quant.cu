// KIVI quantize / dequantize kernels (sm_100a).
//
// Arithmetic follows crates/kvforge-cpu/src/quantize.rs exactly:
//   scale = (max - min) < 1e-10 ? 1 : (max - min) / levels          (quantize.rs:88-89)
//   q     = clamp(round_half_away((v - min) / scale), 0, levels)     (quantize.rs:95, 124)
//   x     = q * scale + min   (separate multiply and add)            (quantize.rs:210, 223)
// with IEEE round-to-nearest intrinsics so nvcc cannot contract or
// approximate any of it. min/max ignore NaN (Rust f32::min/max) and treat
// -0.0 as +0.0 so a parallel reduction gives an order-independent result.
//
// Memory layout: x [H, T, D] row-major; codes are one byte per element
// (flat index), INT4 packing into nibbles is a separate pass.
#include <cooperative_groups.h>

#include <algorithm>
#include <atomic>
#include <cmath>

#include "kvf_internal.cuh"

namespace kvf {
namespace {

constexpr int kSMs = 148;
constexpr int kQpTable = 2048;  // (head, r) parameters kept in shared memory

__device__ __forceinline__ float ldf(const float* p, size_t i) { return __ldg(p + i); }
__device__ __forceinline__ float ldf(const __half* p, size_t i) { return __half2float(__ldg(p + i)); }
__device__ __forceinline__ float4 ld4(const float* p, size_t i) {
  return __ldg(reinterpret_cast<const float4*>(p + i));
}
__device__ __forceinline__ float4 ld4(const __half* p, size_t i) {
  uint2 u = __ldg(reinterpret_cast<const uint2*>(p + i));
  const float2 a = __half22float2(*reinterpret_cast<const __half2*>(&u.x));
  const float2 b = __half22float2(*reinterpret_cast<const __half2*>(&u.y));
  return make_float4(a.x, a.y, b.x, b.y);
}

inline unsigned grid_warps(size_t rows, int warps_per_block) {
  size_t b = (rows + warps_per_block - 1) / warps_per_block;
  const size_t cap = (size_t)kSMs * 32;
  if (b > cap) b = cap;
  return (unsigned)(b ? b : 1);
}

// ---- per-token: one warp per (head, token) row (quantize.rs:102-130) -------
template <typename TIn, int NV>
__global__ void __launch_bounds__(256) k_quant_token_v4(const TIn* __restrict__ x, size_t rows,
                                                        int D, float levels,
                                                        uint8_t* __restrict__ codes,
                                                        float* __restrict__ scales,
                                                        float* __restrict__ mins) {
  const int lane = threadIdx.x & 31;
  const size_t nwarps = ((size_t)gridDim.x * blockDim.x) >> 5;
  const int nq = D >> 2;
  for (size_t g = ((size_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5; g < rows; g += nwarps) {
    const size_t base = g * (size_t)D;
    float4 v[NV];
    float mn = INFINITY, mx = -INFINITY;
#pragma unroll
    for (int k = 0; k < NV; ++k) {
      const int q = lane + 32 * k;
      if (q < nq) {
        v[k] = ld4(x, base + 4 * (size_t)q);
        mm_update(v[k].x, mn, mx);
        mm_update(v[k].y, mn, mx);
        mm_update(v[k].z, mn, mx);
        mm_update(v[k].w, mn, mx);
      }
    }
    warp_minmax(mn, mx);
    const float scale = make_scale(mn, mx, levels);
    const float inv = __frcp_rn(scale);
    if (lane == 0) {
      scales[g] = scale;
      mins[g] = mn;
    }
#pragma unroll
    for (int k = 0; k < NV; ++k) {
      const int q = lane + 32 * k;
      if (q < nq) {
        const uint32_t c = qcode_fast(v[k].x, mn, scale, inv, levels) |
                           (qcode_fast(v[k].y, mn, scale, inv, levels) << 8) |
                           (qcode_fast(v[k].z, mn, scale, inv, levels) << 16) |
                           (qcode_fast(v[k].w, mn, scale, inv, levels) << 24);
        *reinterpret_cast<uint32_t*>(codes + base + 4 * (size_t)q) = c;
      }
    }
  }
}

// D <= 128, D % 4 == 0, 16-byte aligned rows: eight lanes per row and four
// rows per warp, so the per-row work (the range reduction, the scale and its
// reciprocal) is shared by four rows and every lane has four 16-byte loads in
// flight; lane s of a row holds columns 4(s + 8k) .. + 3.
template <typename TIn>
__global__ void __launch_bounds__(256) k_quant_token_r4(const TIn* __restrict__ x, size_t rows, int D,
                                                        float levels, uint8_t* __restrict__ codes,
                                                        float* __restrict__ scales, float* __restrict__ mins) {
  const int lane = threadIdx.x & 31, sub = lane & 7;
  const size_t nwarps = ((size_t)gridDim.x * blockDim.x) >> 5;
  const int nq = D >> 2;
  for (size_t g0 = (((size_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5) * 4; g0 < rows; g0 += nwarps * 4) {
    const size_t g = g0 + (lane >> 3);
    const bool in = g < rows;
    const size_t base = g * (size_t)D;
    float4 v[4];
    float mn = INFINITY, mx = -INFINITY;
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const int q = sub + 8 * k;
      if (in && q < nq) {
        v[k] = ld4(x, base + 4 * (size_t)q);
        mm_update(v[k].x, mn, mx);
        mm_update(v[k].y, mn, mx);
        mm_update(v[k].z, mn, mx);
        mm_update(v[k].w, mn, mx);
      }
    }
#pragma unroll
    for (int o = 4; o > 0; o >>= 1) {
      mn = fminf(mn, __shfl_xor_sync(0xffffffffu, mn, o));
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    }
    if (!in) continue;
    const float scale = make_scale(mn, mx, levels);
    const float inv = __frcp_rn(scale);
    if (sub == 0) {
      scales[g] = scale;
      mins[g] = mn;
    }
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const int q = sub + 8 * k;
      if (q < nq) {
        const uint32_t c = qcode_fast(v[k].x, mn, scale, inv, levels) |
                           (qcode_fast(v[k].y, mn, scale, inv, levels) << 8) |
                           (qcode_fast(v[k].z, mn, scale, inv, levels) << 16) |
                           (qcode_fast(v[k].w, mn, scale, inv, levels) << 24);
        *reinterpret_cast<uint32_t*>(codes + base + 4 * (size_t)q) = c;
      }
    }
  }
}

// Even D <= 128 (projected coefficients whose count is not a multiple of
// four): eight lanes per row, four rows per warp, lane s holds column pairs
// s, s + 8, ... (8-byte loads). INT4: the pair's two codes are one packed
// byte (pairs over the flat index stay inside a row when D is even), written
// directly; INT8: two code bytes. HIST: the bytes written are counted.
template <typename TIn, bool INT4, bool HIST>
__global__ void __launch_bounds__(256) k_quant_token_pairs(const TIn* __restrict__ x, size_t rows, int D,
                                                           float levels, uint8_t* __restrict__ out,
                                                           float* __restrict__ scales, float* __restrict__ mins,
                                                           uint32_t* __restrict__ hist) {
  __shared__ uint32_t sh[HIST ? 256 : 1];
  if (HIST) {
    for (int i = threadIdx.x; i < 256; i += blockDim.x) sh[i] = 0u;
    __syncthreads();
  }
  const int lane = threadIdx.x & 31, sub = lane & 7;
  const size_t nwarps = ((size_t)gridDim.x * blockDim.x) >> 5;
  const int np = D >> 1;  // pairs per row (<= 64)
  for (size_t g0 = (((size_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5) * 4; g0 < rows; g0 += nwarps * 4) {
    const size_t g = g0 + (lane >> 3);
    const bool in = g < rows;
    const size_t base = g * (size_t)D;
    float2 v[8];
    float mn = INFINITY, mx = -INFINITY;
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      const int q = sub + 8 * k;
      if (in && q < np) {
        if constexpr (sizeof(TIn) == 4) {
          v[k] = __ldg(reinterpret_cast<const float2*>(x + base) + q);
        } else {
          v[k] = __half22float2(__ldg(reinterpret_cast<const __half2*>(x + base) + q));
        }
        mm_update(v[k].x, mn, mx);
        mm_update(v[k].y, mn, mx);
      }
    }
#pragma unroll
    for (int o = 4; o > 0; o >>= 1) {
      mn = fminf(mn, __shfl_xor_sync(0xffffffffu, mn, o));
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    }
    if (in) {
      const float scale = make_scale(mn, mx, levels);
      const float inv = __frcp_rn(scale);
      if (sub == 0) {
        scales[g] = scale;
        mins[g] = mn;
      }
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        const int q = sub + 8 * k;
        if (q < np) {
          const uint32_t c0 = qcode_fast(v[k].x, mn, scale, inv, levels);
          const uint32_t c1 = qcode_fast(v[k].y, mn, scale, inv, levels);
          if (INT4) {
            const uint32_t b = (c0 & 0xFu) | ((c1 & 0xFu) << 4);
            out[base / 2 + q] = (uint8_t)b;
            if (HIST) atomicAdd(&sh[b], 1u);
          } else {
            *reinterpret_cast<uint16_t*>(out + base + 2 * (size_t)q) = (uint16_t)(c0 | (c1 << 8));
            if (HIST) {
              atomicAdd(&sh[c0], 1u);
              atomicAdd(&sh[c1], 1u);
            }
          }
        }
      }
    }
  }
  if (HIST) {
    __syncthreads();
    for (int i = threadIdx.x; i < 256; i += blockDim.x)
      if (sh[i]) atomicAdd(&hist[i], sh[i]);
  }
}

template <typename TIn>
__global__ void __launch_bounds__(256) k_quant_token_scalar(const TIn* __restrict__ x, size_t rows,
                                                            int D, float levels,
                                                            uint8_t* __restrict__ codes,
                                                            float* __restrict__ scales,
                                                            float* __restrict__ mins) {
  const int lane = threadIdx.x & 31;
  const size_t nwarps = ((size_t)gridDim.x * blockDim.x) >> 5;
  for (size_t g = ((size_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5; g < rows; g += nwarps) {
    const size_t base = g * (size_t)D;
    float mn = INFINITY, mx = -INFINITY;
    for (int c = lane; c < D; c += 32) mm_update(ldf(x, base + c), mn, mx);
    warp_minmax(mn, mx);
    const float scale = make_scale(mn, mx, levels);
    const float inv = __frcp_rn(scale);
    if (lane == 0) {
      scales[g] = scale;
      mins[g] = mn;
    }
    for (int c = lane; c < D; c += 32) codes[base + c] = (uint8_t)qcode_fast(ldf(x, base + c), mn, scale, inv, levels);
  }
}

// ---- per-channel (quantize.rs:67-101): column min/max over all tokens -------
__global__ void k_minmax_init(int* __restrict__ kmin, int* __restrict__ kmax, size_t np) {
  for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < np; i += (size_t)gridDim.x * blockDim.x) {
    kmin[i] = fkey(INFINITY);
    kmax[i] = fkey(-INFINITY);
  }
}

// grid (token tiles, H); 8 warps stride over the tile's tokens, each lane owns
// a channel of a 32-channel block; partials meet in shared memory, then one
// atomicMin/atomicMax per (head, channel) and block.
template <typename TIn>
__global__ void __launch_bounds__(256) k_colminmax(const TIn* __restrict__ x, size_t T, int D,
                                                   int tpb, int* __restrict__ kmin,
                                                   int* __restrict__ kmax) {
  extern __shared__ float sred[];  // [8][D] minima, then [8][D] maxima
  const int h = blockIdx.y, w = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const size_t t0 = (size_t)blockIdx.x * tpb;
  const size_t t1 = (t0 + tpb < T) ? t0 + tpb : T;
  const TIn* xh = x + (size_t)h * T * D;
  for (int cb = 0; cb < D; cb += 32) {
    const int c = cb + lane;
    float mn = INFINITY, mx = -INFINITY;
    if (c < D)
      for (size_t t = t0 + w; t < t1; t += 8) mm_update(ldf(xh, t * D + c), mn, mx);
    if (c < D) {
      sred[w * D + c] = mn;
      sred[8 * D + w * D + c] = mx;
    }
  }
  __syncthreads();
  for (int c = threadIdx.x; c < D; c += blockDim.x) {
    float mn = sred[c], mx = sred[8 * D + c];
#pragma unroll
    for (int k = 1; k < 8; ++k) {
      mn = fminf(mn, sred[k * D + c]);
      mx = fmaxf(mx, sred[8 * D + k * D + c]);
    }
    atomicMin(&kmin[(size_t)h * D + c], fkey(mn));
    atomicMax(&kmax[(size_t)h * D + c], fkey(mx));
  }
}

// The same per-(head, channel) minima and maxima with four channels per lane
// (D % 4 == 0, D <= 128, rows 4-element aligned): a warp reads whole rows with
// 16-byte (f32) or 8-byte (f16) loads, four rows in flight per lane. Minima and
// maxima do not depend on the order (-0.0 is canonicalised in mm_update), so
// the result equals k_colminmax's.
template <typename TIn>
__global__ void __launch_bounds__(256) k_colminmax_v4(const TIn* __restrict__ x, size_t T, int D,
                                                      int tpb, int* __restrict__ kmin,
                                                      int* __restrict__ kmax) {
  extern __shared__ float sred[];  // [8][D] minima, then [8][D] maxima
  const int h = blockIdx.y, w = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const size_t t0 = (size_t)blockIdx.x * tpb;
  const size_t t1 = (t0 + tpb < T) ? t0 + tpb : T;
  const TIn* xh = x + (size_t)h * T * D;
  const bool on = 4 * lane < D;
  float mn[4], mx[4];
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    mn[k] = INFINITY;
    mx[k] = -INFINITY;
  }
  auto upd = [&](const float4& v) {
    mm_update(v.x, mn[0], mx[0]);
    mm_update(v.y, mn[1], mx[1]);
    mm_update(v.z, mn[2], mx[2]);
    mm_update(v.w, mn[3], mx[3]);
  };
  if (on) {
    const size_t c = 4 * (size_t)lane;
    size_t t = t0 + w;
    for (; t + 24 < t1; t += 32) {
      const float4 a = ld4(xh, t * D + c), b = ld4(xh, (t + 8) * D + c);
      const float4 e = ld4(xh, (t + 16) * D + c), f = ld4(xh, (t + 24) * D + c);
      upd(a);
      upd(b);
      upd(e);
      upd(f);
    }
    for (; t < t1; t += 8) upd(ld4(xh, t * D + c));
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      sred[w * D + 4 * lane + k] = mn[k];
      sred[8 * D + w * D + 4 * lane + k] = mx[k];
    }
  }
  __syncthreads();
  for (int c = threadIdx.x; c < D; c += blockDim.x) {
    float a = sred[c], b = sred[8 * D + c];
#pragma unroll
    for (int k = 1; k < 8; ++k) {
      a = fminf(a, sred[k * D + c]);
      b = fmaxf(b, sred[8 * D + k * D + c]);
    }
    atomicMin(&kmin[(size_t)h * D + c], fkey(a));
    atomicMax(&kmax[(size_t)h * D + c], fkey(b));
  }
}

__global__ void k_params_from_keys(const int* __restrict__ kmin, const int* __restrict__ kmax,
                                   size_t np, float levels, float* __restrict__ scales,
                                   float* __restrict__ mins, float* __restrict__ inv) {
  for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < np; i += (size_t)gridDim.x * blockDim.x) {
    const float mn = kfloat(kmin[i]), mx = kfloat(kmax[i]);
    const float sc = make_scale(mn, mx, levels);
    scales[i] = sc;
    mins[i] = mn;
    inv[i] = __frcp_rn(sc);
  }
}

template <typename TIn, bool V4>
__global__ void __launch_bounds__(256) k_quant_channel(const TIn* __restrict__ x, size_t rows, size_t T,
                                                       int D, float levels,
                                                       const float* __restrict__ scales,
                                                       const float* __restrict__ mins,
                                                       const float* __restrict__ invs,
                                                       uint8_t* __restrict__ codes) {
  const int lane = threadIdx.x & 31;
  const size_t nwarps = ((size_t)gridDim.x * blockDim.x) >> 5;
  for (size_t g = ((size_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5; g < rows; g += nwarps) {
    const size_t base = g * (size_t)D;
    const size_t pb = (g / T) * (size_t)D;
    if (V4) {
      for (int q = lane; q < (D >> 2); q += 32) {
        const float4 v = ld4(x, base + 4 * (size_t)q);
        const float4 s = __ldg(reinterpret_cast<const float4*>(scales + pb) + q);
        const float4 m = __ldg(reinterpret_cast<const float4*>(mins + pb) + q);
        const float4 iv = __ldg(reinterpret_cast<const float4*>(invs + pb) + q);
        const uint32_t c = qcode_fast(v.x, m.x, s.x, iv.x, levels) | (qcode_fast(v.y, m.y, s.y, iv.y, levels) << 8) |
                           (qcode_fast(v.z, m.z, s.z, iv.z, levels) << 16) |
                           (qcode_fast(v.w, m.w, s.w, iv.w, levels) << 24);
        *reinterpret_cast<uint32_t*>(codes + base + 4 * (size_t)q) = c;
      }
    } else {
      for (int c = lane; c < D; c += 32)
        codes[base + c] = (uint8_t)qcode_fast(ldf(x, base + c), __ldg(mins + pb + c), __ldg(scales + pb + c),
                                              __ldg(invs + pb + c), levels);
    }
  }
}

// ---- per-channel in one launch: a thread-block cluster per head -------------
// The per-(head, channel) range needs every token of the head before the
// first code (quantize.rs:67-101). A cluster of C CTAs owns one head: CTA i
// streams tokens [i*S, (i+1)*S) (S = ceil(T / C)) and takes their per-channel
// min/max in registers; the C partial ranges meet through distributed shared
// memory (each CTA reads all C), every CTA forms the same scale and min, then
// reads its tokens again -- from L2, where the first pass just left them --
// and writes their codes. One launch, no atomics, no parameter pass, and a
// small shared-memory footprint, so every cluster is resident at once.
// Thread j handles channels 4(j % (D/4)) .. + 3 of rows j / (D/4),
// j / (D/4) + kQcThreads / (D/4), ... (D / 4 a power of two, D <= 128). INT4 pairs
// (2k, 2k + 1) lie in one row (D even), so a thread packs its four codes into
// two bytes. The optional histogram counts the bytes written.
constexpr int kQcThreads = 512;
constexpr int kQcWarps = kQcThreads / 32;
constexpr int kQcFlight = 8;  // rows in flight per thread in both passes

template <typename TIn, bool INT4>
__global__ void __launch_bounds__(kQcThreads) k_quant_channel_cluster(const TIn* __restrict__ x, int T, int D,
                                                                      int slab, float levels,
                                                                      uint8_t* __restrict__ out,
                                                                      float* __restrict__ scales,
                                                                      float* __restrict__ mins,
                                                                      uint32_t* __restrict__ hist) {
  namespace cg = cooperative_groups;
  cg::cluster_group cluster = cg::this_cluster();
  __shared__ float cmin[128], cmax[128];            // this CTA's partial range per channel
  __shared__ float wred[kQcWarps][2][128];          // per-warp partials; then scale, min, 1/scale
  __shared__ uint32_t shist[256];
  const int h = blockIdx.y, rank = (int)cluster.block_rank();
  const int tid = threadIdx.x;
  const int tpr = D >> 2;                           // threads per row (one float4 / 4 halves each)
  const int rpp = kQcThreads / tpr;                 // rows per pass
  const int rsub = tid / tpr, q = tid - rsub * tpr;
  const int t0 = rank * slab;
  const int nr = max(0, min(slab, T - t0));
  const TIn* xh = x + ((size_t)h * T + (size_t)t0) * D + 4 * q;
  if (hist)
    for (int i = tid; i < 256; i += kQcThreads) shist[i] = 0u;
  float mn[4] = {INFINITY, INFINITY, INFINITY, INFINITY}, mx[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
  {
    int r = rsub;
    for (; r + (kQcFlight - 1) * rpp < nr; r += kQcFlight * rpp) {  // kQcFlight rows in flight per thread
      float4 v[kQcFlight];
#pragma unroll
      for (int u = 0; u < kQcFlight; ++u) v[u] = ld4(xh, (size_t)(r + u * rpp) * D);
#pragma unroll
      for (int u = 0; u < kQcFlight; ++u) {
        mm_update(v[u].x, mn[0], mx[0]);
        mm_update(v[u].y, mn[1], mx[1]);
        mm_update(v[u].z, mn[2], mx[2]);
        mm_update(v[u].w, mn[3], mx[3]);
      }
    }
    for (; r < nr; r += rpp) {
      const float4 v = ld4(xh, (size_t)r * D);
      mm_update(v.x, mn[0], mx[0]);
      mm_update(v.y, mn[1], mx[1]);
      mm_update(v.z, mn[2], mx[2]);
      mm_update(v.w, mn[3], mx[3]);
    }
  }
  // partial ranges: lanes of a warp that share channels (rows of one pass)
  // meet by shuffles, then the warps' partials in shared memory
  const int w = tid >> 5, lane = tid & 31;
  for (int k = 0; k < 4; ++k) {
    for (int o = tpr; o < 32; o <<= 1) {
      mn[k] = fminf(mn[k], __shfl_xor_sync(0xffffffffu, mn[k], o));
      mx[k] = fmaxf(mx[k], __shfl_xor_sync(0xffffffffu, mx[k], o));
    }
  }
  if (lane < tpr) {
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      wred[w][0][4 * lane + k] = mn[k];
      wred[w][1][4 * lane + k] = mx[k];
    }
  }
  __syncthreads();
  for (int c = tid; c < D; c += kQcThreads) {
    float a = INFINITY, b = -INFINITY;
#pragma unroll
    for (int k = 0; k < kQcWarps; ++k) {
      a = fminf(a, wred[k][0][c]);
      b = fmaxf(b, wred[k][1][c]);
    }
    cmin[c] = a;
    cmax[c] = b;
  }
  cluster.sync();  // every CTA's partial range is in its shared memory
  float* gsc = &wred[0][0][0];  // reuse: [D] scales, [D] mins, [D] reciprocals of this head
  float* gmn = gsc + 128;
  float* ginv = gsc + 256;
  for (int c = tid; c < D; c += kQcThreads) {
    float a = INFINITY, b = -INFINITY;
    for (unsigned k = 0; k < cluster.num_blocks(); ++k) {
      const float* rmin = cluster.map_shared_rank(cmin, k);
      const float* rmax = cluster.map_shared_rank(cmax, k);
      a = fminf(a, rmin[c]);
      b = fmaxf(b, rmax[c]);
    }
    const float sc = make_scale(a, b, levels);
    gsc[c] = sc;
    gmn[c] = a;
    ginv[c] = __frcp_rn(sc);
    if (rank == 0) {
      scales[(size_t)h * D + c] = sc;
      mins[(size_t)h * D + c] = a;
    }
  }
  cluster.sync();  // no CTA leaves (or reuses wred) while another still reads its partials
  float s4[4], m4[4], i4[4];
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    s4[k] = gsc[4 * q + k];
    m4[k] = gmn[4 * q + k];
    i4[k] = ginv[4 * q + k];
  }
  auto emit = [&](int r, const float4& f) {
    const float v[4] = {f.x, f.y, f.z, f.w};
    uint32_t c[4];
#pragma unroll
    for (int k = 0; k < 4; ++k) c[k] = qcode_fast(v[k], m4[k], s4[k], i4[k], levels);
    const size_t flat = ((size_t)h * T + (size_t)(t0 + r)) * D + 4 * q;
    if (INT4) {
      const uint32_t b0 = (c[0] & 0xFu) | ((c[1] & 0xFu) << 4), b1 = (c[2] & 0xFu) | ((c[3] & 0xFu) << 4);
      *reinterpret_cast<uint16_t*>(out + flat / 2) = (uint16_t)(b0 | (b1 << 8));
      if (hist) {
        atomicAdd(&shist[b0], 1u);
        atomicAdd(&shist[b1], 1u);
      }
    } else {
      *reinterpret_cast<uint32_t*>(out + flat) = c[0] | (c[1] << 8) | (c[2] << 16) | (c[3] << 24);
      if (hist)
#pragma unroll
        for (int k = 0; k < 4; ++k) atomicAdd(&shist[c[k]], 1u);
    }
  };
  {
    int r = rsub;
    for (; r + (kQcFlight - 1) * rpp < nr; r += kQcFlight * rpp) {
      float4 v[kQcFlight];
#pragma unroll
      for (int u = 0; u < kQcFlight; ++u) v[u] = ld4(xh, (size_t)(r + u * rpp) * D);
#pragma unroll
      for (int u = 0; u < kQcFlight; ++u) emit(r + u * rpp, v[u]);
    }
    for (; r < nr; r += rpp) emit(r, ld4(xh, (size_t)r * D));
  }
  if (hist) {
    __syncthreads();
    for (int i = tid; i < 256; i += kQcThreads)
      if (shist[i]) atomicAdd(&hist[i], shist[i]);
  }
}

template <typename TIn, bool INT4>
cudaError_t launch_qcc(const TIn* x, size_t H, size_t T, size_t D, int C, int slab, float levels, uint8_t* out,
                       float* scales, float* mins, uint32_t* hist, size_t smem, cudaStream_t st) {
  auto kern = k_quant_channel_cluster<TIn, INT4>;
  constexpr int kDevs = 64;
  static std::atomic<int> opted[kDevs];  // shared memory opted in so far, per device
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 0 || dev >= kDevs) return cudaErrorInvalidDevice;
  if ((int)smem > opted[dev].load(std::memory_order_acquire)) {
    if ((e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem)) != cudaSuccess)
      return e;
    opted[dev].store((int)smem, std::memory_order_release);
  }
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3((unsigned)C, (unsigned)H, 1);
  cfg.blockDim = dim3(kQcThreads, 1, 1);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = (unsigned)C;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  e = cudaLaunchKernelEx(&cfg, kern, x, (int)T, (int)D, slab, levels, out, scales, mins, hist);
  if (e == cudaSuccess) note_launches(1);
  return e;
}

// ---- INT4 nibble packing over the flat index (quantize.rs:136-150) ----------
// 32 codes -> 16 packed bytes per thread step; optional 256-bin histogram of
// the packed bytes (entropy.rs:24-31) in per-warp shared sub-histograms.
__device__ __forceinline__ uint32_t pack4(uint32_t w) {
  return (w & 0xFu) | (((w >> 8) & 0xFu) << 4) | (((w >> 16) & 0xFu) << 8) | (((w >> 24) & 0xFu) << 12);
}

__device__ __forceinline__ void hist_word(uint32_t* sh, uint32_t w) {
  atomicAdd(&sh[w & 0xFF], 1u);
  atomicAdd(&sh[(w >> 8) & 0xFF], 1u);
  atomicAdd(&sh[(w >> 16) & 0xFF], 1u);
  atomicAdd(&sh[w >> 24], 1u);
}

template <bool HIST>
__global__ void __launch_bounds__(256) k_pack_int4(const uint8_t* __restrict__ codes, size_t n,
                                                   uint8_t* __restrict__ packed,
                                                   uint32_t* __restrict__ hist, bool vec) {
  __shared__ uint32_t sh[8][256];
  const int w = threadIdx.x >> 5;
  if (HIST) {
    for (int i = threadIdx.x; i < 8 * 256; i += blockDim.x) (&sh[0][0])[i] = 0;
    __syncthreads();
  }
  const size_t n32 = vec ? n / 32 : 0;
  for (size_t j = (size_t)blockIdx.x * blockDim.x + threadIdx.x; j < n32; j += (size_t)gridDim.x * blockDim.x) {
    const uint4 a = __ldg(reinterpret_cast<const uint4*>(codes + 32 * j));
    const uint4 b = __ldg(reinterpret_cast<const uint4*>(codes + 32 * j + 16));
    uint4 o;
    o.x = pack4(a.x) | (pack4(a.y) << 16);
    o.y = pack4(a.z) | (pack4(a.w) << 16);
    o.z = pack4(b.x) | (pack4(b.y) << 16);
    o.w = pack4(b.z) | (pack4(b.w) << 16);
    *reinterpret_cast<uint4*>(packed + 16 * j) = o;
    if (HIST) {
      hist_word(sh[w], o.x);
      hist_word(sh[w], o.y);
      hist_word(sh[w], o.z);
      hist_word(sh[w], o.w);
    }
  }
  {
    const size_t np = (n + 1) / 2;
    for (size_t p = 16 * n32 + (size_t)blockIdx.x * blockDim.x + threadIdx.x; p < np;
         p += (size_t)gridDim.x * blockDim.x) {
      const uint32_t lo = codes[2 * p] & 0xFu;
      const uint32_t hi = (2 * p + 1 < n) ? (codes[2 * p + 1] & 0xFu) : 0u;
      const uint32_t byte = lo | (hi << 4);
      packed[p] = (uint8_t)byte;
      if (HIST) atomicAdd(&sh[w][byte], 1u);
    }
  }
  if (HIST) {
    __syncthreads();
    for (int s = threadIdx.x; s < 256; s += blockDim.x) {
      uint32_t t = 0;
#pragma unroll
      for (int k = 0; k < 8; ++k) t += sh[k][s];
      if (t) atomicAdd(&hist[s], t);
    }
  }
}

__global__ void __launch_bounds__(256) k_histogram(const uint8_t* __restrict__ data, size_t n,
                                                   uint32_t* __restrict__ hist, bool vec) {
  __shared__ uint32_t sh[8][256];
  const int w = threadIdx.x >> 5;
  for (int i = threadIdx.x; i < 8 * 256; i += blockDim.x) (&sh[0][0])[i] = 0;
  __syncthreads();
  const size_t n16 = vec ? n / 16 : 0;
  for (size_t j = (size_t)blockIdx.x * blockDim.x + threadIdx.x; j < n16; j += (size_t)gridDim.x * blockDim.x) {
    const uint4 a = __ldg(reinterpret_cast<const uint4*>(data + 16 * j));
    hist_word(sh[w], a.x);
    hist_word(sh[w], a.y);
    hist_word(sh[w], a.z);
    hist_word(sh[w], a.w);
  }
  for (size_t i = 16 * n16 + (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x)
    atomicAdd(&sh[w][data[i]], 1u);
  __syncthreads();
  for (int s = threadIdx.x; s < 256; s += blockDim.x) {
    uint32_t t = 0;
#pragma unroll
    for (int k = 0; k < 8; ++k) t += sh[k][s];
    if (t) atomicAdd(&hist[s], t);
  }
}

// ---- dequantize without projection (quantize.rs:165-231) --------------------
template <bool INT4, bool V4>
__global__ void __launch_bounds__(256) k_dequant(const uint8_t* __restrict__ packed,
                                                 const float* __restrict__ scales,
                                                 const float* __restrict__ mins, int axis,
                                                 size_t rows, size_t T, int D,
                                                 float* __restrict__ out) {
  const int lane = threadIdx.x & 31;
  const size_t nwarps = ((size_t)gridDim.x * blockDim.x) >> 5;
  for (size_t g = ((size_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5; g < rows; g += nwarps) {
    const size_t base = g * (size_t)D;
    const bool per_channel = (axis == KVF_PER_CHANNEL);
    const size_t pb = per_channel ? (g / T) * (size_t)D : g;
    const float ts = per_channel ? 0.0f : __ldg(scales + g);
    const float tm = per_channel ? 0.0f : __ldg(mins + g);
    if (V4) {
      for (int q = lane; q < (D >> 2); q += 32) {
        const size_t i = base + 4 * (size_t)q;
        uint32_t c0, c1, c2, c3;
        if (INT4) {
          const uint32_t b = *reinterpret_cast<const uint16_t*>(packed + (i >> 1));
          c0 = b & 0xF; c1 = (b >> 4) & 0xF; c2 = (b >> 8) & 0xF; c3 = (b >> 12) & 0xF;
        } else {
          const uint32_t b = *reinterpret_cast<const uint32_t*>(packed + i);
          c0 = b & 0xFF; c1 = (b >> 8) & 0xFF; c2 = (b >> 16) & 0xFF; c3 = b >> 24;
        }
        float4 s, m;
        if (per_channel) {
          s = __ldg(reinterpret_cast<const float4*>(scales + pb) + q);
          m = __ldg(reinterpret_cast<const float4*>(mins + pb) + q);
        } else {
          s = make_float4(ts, ts, ts, ts);
          m = make_float4(tm, tm, tm, tm);
        }
        const float4 o = make_float4(dq(c0, s.x, m.x), dq(c1, s.y, m.y), dq(c2, s.z, m.z), dq(c3, s.w, m.w));
        __stcs(reinterpret_cast<float4*>(out + i), o);
      }
    } else {
      for (int c = lane; c < D; c += 32) {
        const size_t i = base + c;
        const uint32_t b = packed[INT4 ? (i >> 1) : i];
        const uint32_t q = INT4 ? ((i & 1) ? (b >> 4) & 0xF : b & 0xF) : b;
        const float s = per_channel ? __ldg(scales + pb + c) : ts;
        const float m = per_channel ? __ldg(mins + pb + c) : tm;
        out[i] = dq(q, s, m);
      }
    }
  }
}

// D <= 128, D % 4 == 0, vector-aligned buffers: eight lanes per row, four
// rows per warp, the codes of all four loaded before any output is formed;
// lane s of a row writes columns 4(s + 8k) .. + 3. HEAD32: the head index of
// a row by 32-bit division (rows < 2^32).
template <bool INT4, bool HEAD32>
__global__ void __launch_bounds__(256) k_dequant_r4(const uint8_t* __restrict__ packed,
                                                    const float* __restrict__ scales,
                                                    const float* __restrict__ mins, int axis, size_t rows,
                                                    size_t T, int D, float* __restrict__ out) {
  const int lane = threadIdx.x & 31, sub = lane & 7;
  const size_t nwarps = ((size_t)gridDim.x * blockDim.x) >> 5;
  const int nq = D >> 2;
  const bool per_channel = (axis == KVF_PER_CHANNEL);
  for (size_t g0 = (((size_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5) * 4; g0 < rows; g0 += nwarps * 4) {
    const size_t g = g0 + (lane >> 3);
    if (g >= rows) continue;
    const size_t base = g * (size_t)D;
    const size_t hd = HEAD32 ? (size_t)((uint32_t)g / (uint32_t)T) : g / T;
    const size_t pb = hd * (size_t)D;
    const float ts = per_channel ? 0.0f : __ldg(scales + g);
    const float tm = per_channel ? 0.0f : __ldg(mins + g);
    uint32_t b[4];
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const int q = sub + 8 * k;
      b[k] = 0u;
      if (q < nq) {
        const size_t i = base + 4 * (size_t)q;
        b[k] = INT4 ? (uint32_t)*reinterpret_cast<const uint16_t*>(packed + (i >> 1))
                    : *reinterpret_cast<const uint32_t*>(packed + i);
      }
    }
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const int q = sub + 8 * k;
      if (q >= nq) continue;
      uint32_t c0, c1, c2, c3;
      if (INT4) {
        c0 = b[k] & 0xF; c1 = (b[k] >> 4) & 0xF; c2 = (b[k] >> 8) & 0xF; c3 = (b[k] >> 12) & 0xF;
      } else {
        c0 = b[k] & 0xFF; c1 = (b[k] >> 8) & 0xFF; c2 = (b[k] >> 16) & 0xFF; c3 = b[k] >> 24;
      }
      float4 s, m;
      if (per_channel) {
        s = __ldg(reinterpret_cast<const float4*>(scales + pb) + q);
        m = __ldg(reinterpret_cast<const float4*>(mins + pb) + q);
      } else {
        s = make_float4(ts, ts, ts, ts);
        m = make_float4(tm, tm, tm, tm);
      }
      const float4 o = make_float4(dq(c0, s.x, m.x), dq(c1, s.y, m.y), dq(c2, s.z, m.z), dq(c3, s.w, m.w));
      __stcs(reinterpret_cast<float4*>(out + base + 4 * (size_t)q), o);
    }
  }
}

// ---- per-channel codes from projected coefficients ---------------------------
// P [H,T,R] f32 with its per-(head, r) min/max already folded into kmin/kmax
// by the projection kernel. A grid of a few blocks per SM; each thread takes
// groups of eight consecutive codes (two 16-byte loads of P), walks their
// (head, r) parameter index with counters instead of divisions, packs INT4
// nibbles over the flat index and stores the group's bytes with one 4- or
// 8-byte store; packed bytes are counted in per-warp shared histograms that
// are merged once per block. The first np threads also write the (scale,
// min) parameters.
template <bool INT4, bool HIST>
__global__ void __launch_bounds__(256) k_quantpack_channel(const float* __restrict__ P, uint64_t n, uint64_t T,
                                                           uint64_t R, const int* __restrict__ kmin,
                                                           const int* __restrict__ kmax, float levels,
                                                           float* __restrict__ scales, float* __restrict__ mins,
                                                           uint64_t np, uint8_t* __restrict__ out,
                                                           uint32_t* __restrict__ hist, bool vec) {
  __shared__ uint32_t sh[8][256];
  __shared__ float ps[kQpTable], pm[kQpTable], pi[kQpTable];
  const int w = threadIdx.x >> 5;
  if (HIST)
    for (int i = threadIdx.x; i < 8 * 256; i += blockDim.x) (&sh[0][0])[i] = 0;
  const uint64_t tid = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x;
  const uint64_t stride = (uint64_t)gridDim.x * blockDim.x;
  for (uint64_t i = tid; i < np; i += stride) {
    const float mn = kfloat(kmin[i]), mx = kfloat(kmax[i]);
    scales[i] = make_scale(mn, mx, levels);
    mins[i] = mn;
  }
  // (scale, min, 1/scale) per (head, r) in shared memory when they fit
  const bool table = np <= (uint64_t)kQpTable;
  if (table)
    for (uint64_t i = threadIdx.x; i < np; i += blockDim.x) {
      const float mn = kfloat(kmin[i]), mx = kfloat(kmax[i]);
      const float sc = make_scale(mn, mx, levels);
      ps[i] = sc;
      pm[i] = mn;
      pi[i] = __frcp_rn(sc);
    }
  __syncthreads();
  const uint64_t per_head = T * R;
  auto qc = [&](float v, uint64_t p) -> uint32_t {
    if (table) return qcode_fast(v, pm[p], ps[p], pi[p], levels);
    const float mn = kfloat(__ldg(kmin + p)), mx = kfloat(__ldg(kmax + p));
    const float sc = make_scale(mn, mx, levels);
    return qcode_fast(v, mn, sc, __frcp_rn(sc), levels);
  };
  const uint64_t groups = (n + 7) / 8;
  for (uint64_t gi = tid; gi < groups; gi += stride) {
    const uint64_t i0 = 8 * gi;
    float v[8];
    if (vec && i0 + 8 <= n) {
      const float4 a = __ldg(reinterpret_cast<const float4*>(P + i0));
      const float4 b = __ldg(reinterpret_cast<const float4*>(P + i0) + 1);
      v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w;
      v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
    } else {
#pragma unroll
      for (int k = 0; k < 8; ++k) v[k] = (i0 + k < n) ? __ldg(P + i0 + k) : 0.0f;
    }
    uint64_t h = i0 / per_head;
    uint64_t c = i0 - h * per_head;
    uint64_t rr = c % R;
    uint64_t left = per_head - c;  // codes before the next head starts
    uint32_t cd[8];
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      cd[k] = (i0 + k < n) ? qc(v[k], h * R + rr) : 0u;  // no parameter lookups past the end
      if (++rr == R) rr = 0;
      if (--left == 0) {
        ++h;
        left = per_head;
        rr = 0;
      }
    }
    if (INT4) {  // bytes 4 gi .. 4 gi + 3
      const uint64_t nb = (n + 1) / 2, b0 = 4 * gi;
      uint32_t word = 0;
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const uint32_t byte = (cd[2 * k] & 0xFu) | ((i0 + 2 * k + 1 < n) ? (cd[2 * k + 1] & 0xFu) << 4 : 0u);
        word |= byte << (8 * k);
        if (HIST && b0 + k < nb) atomicAdd(&sh[w][byte], 1u);
      }
      if (vec && b0 + 4 <= nb) {
        *reinterpret_cast<uint32_t*>(out + b0) = word;
      } else {
#pragma unroll
        for (int k = 0; k < 4; ++k)
          if (b0 + k < nb) out[b0 + k] = (uint8_t)(word >> (8 * k));
      }
    } else {  // bytes 8 gi .. 8 gi + 7
      if (vec && i0 + 8 <= n) {
        uint2 u;
        u.x = cd[0] | (cd[1] << 8) | (cd[2] << 16) | (cd[3] << 24);
        u.y = cd[4] | (cd[5] << 8) | (cd[6] << 16) | (cd[7] << 24);
        *reinterpret_cast<uint2*>(out + i0) = u;
      } else {
#pragma unroll
        for (int k = 0; k < 8; ++k)
          if (i0 + k < n) out[i0 + k] = (uint8_t)cd[k];
      }
      if (HIST)
#pragma unroll
        for (int k = 0; k < 8; ++k)
          if (i0 + k < n) atomicAdd(&sh[w][cd[k]], 1u);
    }
  }
  if (HIST) {
    __syncthreads();
    for (int s = threadIdx.x; s < 256; s += blockDim.x) {
      uint32_t t = 0;
#pragma unroll
      for (int k = 0; k < 8; ++k) t += sh[k][s];
      if (t) atomicAdd(&hist[s], t);
    }
  }
}

template <typename TIn>
cudaError_t quantize_typed(const TIn* x, size_t H, size_t T, size_t D, int dt, int axis,
                           uint8_t* codes, float* scales, float* mins, int* keys,
                           cudaStream_t st) {
  const float levels = quant_levels(dt);
  const size_t rows = H * T;
  const int Di = (int)D;
  const bool xal = aligned(x, sizeof(TIn) * 4) && aligned(codes, 4);
  if (axis == KVF_PER_TOKEN) {
    if (rows == 0) return cudaSuccess;
    const unsigned grid = grid_warps(rows, 8);
    if (!xal)
      k_quant_token_scalar<TIn><<<grid, 256, 0, st>>>(x, rows, Di, levels, codes, scales, mins);
    else if (D % 4 == 0 && D > 0 && D <= 128)
      k_quant_token_r4<TIn><<<grid_warps((rows + 3) / 4, 8), 256, 0, st>>>(x, rows, Di, levels, codes, scales, mins);
    else if (D % 4 == 0 && D > 0 && D <= 256)
      k_quant_token_v4<TIn, 2><<<grid, 256, 0, st>>>(x, rows, Di, levels, codes, scales, mins);
    else if (D % 4 == 0 && D > 0 && D <= 512)
      k_quant_token_v4<TIn, 4><<<grid, 256, 0, st>>>(x, rows, Di, levels, codes, scales, mins);
    else
      k_quant_token_scalar<TIn><<<grid, 256, 0, st>>>(x, rows, Di, levels, codes, scales, mins);
    note_launches(1);
    return cudaGetLastError();
  }
  // per-channel
  const size_t np = H * D;
  if (np == 0) return cudaSuccess;
  int* kmin = keys;
  int* kmax = keys + np;
  const unsigned ig = (unsigned)std::min<size_t>((np + 255) / 256, 4096);
  k_minmax_init<<<ig, 256, 0, st>>>(kmin, kmax, np);
  if (T > 0) {
    const int tpb = 256;
    const dim3 grid((unsigned)((T + tpb - 1) / tpb), (unsigned)H);
    const size_t smem = 2 * 8 * D * sizeof(float);
    if (smem > kSmemOptIn) {
      cudaError_t e = cudaFuncSetAttribute(k_colminmax<TIn>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
      if (e != cudaSuccess) return e;
    }
    if (D % 4 == 0 && D <= 128 && aligned(x, sizeof(TIn) * 4))
      k_colminmax_v4<TIn><<<grid, 256, smem, st>>>(x, T, Di, tpb, kmin, kmax);
    else
      k_colminmax<TIn><<<grid, 256, smem, st>>>(x, T, Di, tpb, kmin, kmax);
  }
  float* invs = reinterpret_cast<float*>(keys + 2 * np);
  k_params_from_keys<<<ig, 256, 0, st>>>(kmin, kmax, np, levels, scales, mins, invs);
  note_launches(2 + (T > 0 ? 1 : 0) + (rows > 0 ? 1 : 0));
  if (rows > 0) {
    const unsigned grid = grid_warps(rows, 8);
    if (D % 4 == 0 && xal && aligned(scales, 16) && aligned(mins, 16) && aligned(invs, 16))
      k_quant_channel<TIn, true><<<grid, 256, 0, st>>>(x, rows, T, Di, levels, scales, mins, invs, codes);
    else
      k_quant_channel<TIn, false><<<grid, 256, 0, st>>>(x, rows, T, Di, levels, scales, mins, invs, codes);
  }
  return cudaGetLastError();
}

}  // namespace

cudaError_t launch_quantize_codes(const void* x, int in_dtype, size_t H, size_t T, size_t D,
                                  int data_type, int axis, uint8_t* codes, float* scales,
                                  float* mins, int* keys, cudaStream_t st) {
  if (in_dtype == KVF_IN_F16)
    return quantize_typed(static_cast<const __half*>(x), H, T, D, data_type, axis, codes, scales, mins, keys, st);
  return quantize_typed(static_cast<const float*>(x), H, T, D, data_type, axis, codes, scales, mins, keys, st);
}

cudaError_t launch_quantize_token_pairs(const void* x, int in_dtype, size_t H, size_t T, size_t D, int data_type,
                                       uint8_t* out, float* scales, float* mins, uint32_t* hist, cudaStream_t st) {
  const size_t esz = in_dtype == KVF_IN_F16 ? 2 : 4;
  const size_t rows = H * T;
  if (D == 0 || D % 2 || D > 128 || rows == 0 || !aligned(x, 2 * esz) || (data_type == KVF_INT8 && !aligned(out, 2)))
    return cudaErrorNotSupported;
  const unsigned grid = grid_warps((rows + 3) / 4, 8);
  const float levels = quant_levels(data_type);
  const int Di = (int)D;
#define KVF_QTP(TI, I4, HI)                                                                                 \
  k_quant_token_pairs<TI, I4, HI><<<grid, 256, 0, st>>>(static_cast<const TI*>(x), rows, Di, levels, out, scales, \
                                                       mins, hist)
  const bool i4 = data_type == KVF_INT4, hi = hist != nullptr;
  if (in_dtype == KVF_IN_F16) {
    if (i4) { if (hi) KVF_QTP(__half, true, true); else KVF_QTP(__half, true, false); }
    else { if (hi) KVF_QTP(__half, false, true); else KVF_QTP(__half, false, false); }
  } else {
    if (i4) { if (hi) KVF_QTP(float, true, true); else KVF_QTP(float, true, false); }
    else { if (hi) KVF_QTP(float, false, true); else KVF_QTP(float, false, false); }
  }
#undef KVF_QTP
  note_launches(1);
  return cudaGetLastError();
}

cudaError_t launch_quantize_channel_cluster(const void* x, int in_dtype, size_t H, size_t T, size_t D, int data_type,
                                            uint8_t* out, float* scales, float* mins, uint32_t* hist,
                                            cudaStream_t st) {
  const size_t esz = in_dtype == KVF_IN_F16 ? 2 : 4;
  const size_t tpr = D / 4;  // threads per row: a power of two (the shuffle reduction pairs lanes tpr apart)
  if (D == 0 || D > 128 || D % 4 || (tpr & (tpr - 1)) || H == 0 || H > 65535 || T == 0 || T > (1u << 30) ||
      !aligned(x, 4 * esz) || !aligned(out, data_type == KVF_INT4 ? 2 : 4))
    return cudaErrorNotSupported;
  // CTAs per head (a cluster of 1, 2, 4 or 8): enough CTAs for every SM, and
  // at least 32 rows each (non-portable clusters of 16 measured slower: 22.8
  // against 18.6 us on 32 heads x 2048 tokens)
  int C = 1;
  while (C < 8 && H * (size_t)C < 4 * 148 && (T + 2 * C - 1) / (2 * C) >= 32) C *= 2;
  const size_t smem = 0;
  const float levels = quant_levels(data_type);
  auto launch = [&](int c) {
    const int slab = (int)((T + c - 1) / c);
    if (in_dtype == KVF_IN_F16) {
      const __half* xh = static_cast<const __half*>(x);
      return data_type == KVF_INT4
                 ? launch_qcc<__half, true>(xh, H, T, D, c, slab, levels, out, scales, mins, hist, smem, st)
                 : launch_qcc<__half, false>(xh, H, T, D, c, slab, levels, out, scales, mins, hist, smem, st);
    }
    const float* xf = static_cast<const float*>(x);
    return data_type == KVF_INT4
               ? launch_qcc<float, true>(xf, H, T, D, c, slab, levels, out, scales, mins, hist, smem, st)
               : launch_qcc<float, false>(xf, H, T, D, c, slab, levels, out, scales, mins, hist, smem, st);
  };
  return launch(C);
}

cudaError_t launch_minmax_init(int* kmin, int* kmax, size_t np, cudaStream_t st) {
  if (np == 0) return cudaSuccess;
  const unsigned ig = (unsigned)std::min<size_t>((np + 255) / 256, 4096);
  k_minmax_init<<<ig, 256, 0, st>>>(kmin, kmax, np);
  note_launches(1);
  return cudaGetLastError();
}

cudaError_t launch_quantpack_channel(const float* P, size_t H, size_t T, size_t R, const int* kmin,
                                     const int* kmax, int data_type, float* scales, float* mins,
                                     uint8_t* out, uint32_t* hist, cudaStream_t st) {
  const size_t n = H * T * R;
  const size_t np = H * R;
  const size_t nb = std::max(packed_len(n, data_type), np);
  if (nb == 0) return cudaSuccess;
  const size_t groups = (n + 7) / 8;
  const unsigned grid = (unsigned)std::max<size_t>(1, std::min<size_t>((std::max(groups, np) + 255) / 256, (size_t)kSMs * 2));
  const float levels = quant_levels(data_type);
  const bool vec = aligned(P, 16) && aligned(out, 8);
  if (data_type == KVF_INT4) {
    if (hist) k_quantpack_channel<true, true><<<grid, 256, 0, st>>>(P, n, T, R, kmin, kmax, levels, scales, mins, np, out, hist, vec);
    else k_quantpack_channel<true, false><<<grid, 256, 0, st>>>(P, n, T, R, kmin, kmax, levels, scales, mins, np, out, nullptr, vec);
  } else {
    if (hist) k_quantpack_channel<false, true><<<grid, 256, 0, st>>>(P, n, T, R, kmin, kmax, levels, scales, mins, np, out, hist, vec);
    else k_quantpack_channel<false, false><<<grid, 256, 0, st>>>(P, n, T, R, kmin, kmax, levels, scales, mins, np, out, nullptr, vec);
  }
  note_launches(1);
  return cudaGetLastError();
}

cudaError_t launch_pack_int4(const uint8_t* codes, size_t n, uint8_t* packed, uint32_t* hist,
                             cudaStream_t st) {
  if (n == 0) return cudaSuccess;
  size_t work = n / 32;
  unsigned grid = (unsigned)std::min<size_t>((work + 255) / 256, (size_t)kSMs * 8);
  if (grid == 0) grid = 1;
  const bool vec = aligned(codes, 16) && aligned(packed, 16);
  if (!vec) grid = (unsigned)std::min<size_t>((n / 2 + 255) / 256 + 1, (size_t)kSMs * 8);
  if (hist)
    k_pack_int4<true><<<grid, 256, 0, st>>>(codes, n, packed, hist, vec);
  else
    k_pack_int4<false><<<grid, 256, 0, st>>>(codes, n, packed, nullptr, vec);
  note_launches(1);
  return cudaGetLastError();
}

cudaError_t launch_histogram(const uint8_t* data, size_t n, uint32_t* hist, cudaStream_t st) {
  if (n == 0) return cudaSuccess;
  size_t work = n / 16;
  unsigned grid = (unsigned)std::min<size_t>((work + 255) / 256, (size_t)kSMs * 8);
  if (grid == 0) grid = 1;
  const bool vec = aligned(data, 16);
  if (!vec) grid = (unsigned)std::min<size_t>((n + 255) / 256, (size_t)kSMs * 8);
  k_histogram<<<grid, 256, 0, st>>>(data, n, hist, vec);
  note_launches(1);
  return cudaGetLastError();
}

cudaError_t launch_dequantize(const uint8_t* packed, const float* scales, const float* mins,
                              int data_type, int axis, size_t H, size_t T, size_t D, float* out,
                              cudaStream_t st) {
  const size_t rows = H * T;
  if (rows == 0 || D == 0) return cudaSuccess;
  const unsigned grid = grid_warps(rows, 8);
  const bool v4 = (D % 4 == 0) && aligned(out, 16) && aligned(packed, data_type == KVF_INT4 ? 2 : 4) &&
                  (axis != KVF_PER_CHANNEL || (aligned(scales, 16) && aligned(mins, 16)));
  const int Di = (int)D;
  if (v4 && D <= 128) {
    const unsigned g4 = grid_warps((rows + 3) / 4, 8);
    const bool h32 = rows <= 0xffffffffull;
    if (data_type == KVF_INT4) {
      if (h32) k_dequant_r4<true, true><<<g4, 256, 0, st>>>(packed, scales, mins, axis, rows, T, Di, out);
      else k_dequant_r4<true, false><<<g4, 256, 0, st>>>(packed, scales, mins, axis, rows, T, Di, out);
    } else {
      if (h32) k_dequant_r4<false, true><<<g4, 256, 0, st>>>(packed, scales, mins, axis, rows, T, Di, out);
      else k_dequant_r4<false, false><<<g4, 256, 0, st>>>(packed, scales, mins, axis, rows, T, Di, out);
    }
    note_launches(1);
    return cudaGetLastError();
  }
  if (data_type == KVF_INT4) {
    if (v4) k_dequant<true, true><<<grid, 256, 0, st>>>(packed, scales, mins, axis, rows, T, Di, out);
    else k_dequant<true, false><<<grid, 256, 0, st>>>(packed, scales, mins, axis, rows, T, Di, out);
  } else {
    if (v4) k_dequant<false, true><<<grid, 256, 0, st>>>(packed, scales, mins, axis, rows, T, Di, out);
    else k_dequant<false, false><<<grid, 256, 0, st>>>(packed, scales, mins, axis, rows, T, Di, out);
  }
  note_launches(1);
  return cudaGetLastError();
}

}  // namespace kvf
