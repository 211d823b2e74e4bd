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
// the result is deterministic. Inside the key projection each thread first
// sums 64 elements in f32 (the squares of f16 inputs are exact) and adds that
// to its fp64 sums; the scores (a ratio of variances) stay within 1e-6 of the
// sequential fp64 reference, the parity bar for a result the reference
// pipeline discards (pipeline.rs:106-111).
#include <cuda.h>
#include <cudaTypedefs.h>

#include <algorithm>
#include <atomic>
#include <cmath>
#include <mutex>

#include "kvf_internal.cuh"

namespace kvf {
namespace {

constexpr int kRecRows = 128;                    // token rows per reconstruct block
constexpr int kCalibTile = 1 << 16;              // elements per calibration block
constexpr int kGramTile = 512;                   // tokens per Gram block

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
// One persistent kernel. The grid walks (head, 256-token tile) items in
// contiguous ranges per block; warp w owns rows 64w .. 64w + 63 of every tile
// and lane l rows l and l + 32 of those, and computes their R coefficients.
// Each coefficient is a fused multiply-add chain over c = 0..D-1 from +0.0;
// two chains advance per fma.rn.f32x2 (each element rounded once), so values
// are identical to the CPU oracle's fmaf chain. The basis of head h sits
// transposed in shared memory, vT[c][R rounded up to RG], read with broadcast
// 16-byte loads (at compile-time offsets when one pass covers R); each load
// feeds both of a thread's rows. Coefficients are computed RG at a time: one
// pass over a tile up to R = 24, one pass per 32 coefficients up to R = 64.
//
// TMA variant (rows a multiple of 64 bytes, 16-byte aligned input): each warp
// streams its own 64 rows of a tile as column blocks of 64 rows x 64 bytes
// (4 KB), each one 2-D tensor copy (cp.async.bulk.tensor, no multicast) with
// the 64-byte swizzle, issued by lane 0 into the warp's own stages and
// mbarriers, several in flight; the accumulators stay in registers across a
// tile's column blocks, and a later pass streams the tile again (from L2).
// Warps synchronise with each other only when the head
// (and so the shared basis) changes. The swizzle stores 16-byte chunk j of a
// 64-byte row at j ^ (bits 7-8 of the row's address), so the reads of eight
// consecutive rows fall on distinct banks. Small stages keep several CTAs
// resident per SM. Waits are bounded: a wait that expires raises the device
// timeout status.
// Generic variant: scalar loads from global memory.
//
// Epilogues (each thread stores its own rows; consecutive rows are contiguous):
//   MODE 0: P [H,T,R];
//   MODE 1: P and per-(head, r) min/max folded into block-local keys,
//           flushed with one global atomic per (block, head, r);
//   MODE 2: per-token quantization: scale/min per token, codes as bytes or
//           INT4-packed bytes, plus an optional byte histogram.
constexpr int kProjThreads = 128;
constexpr int kProjNR = 2;                           // token rows per thread
constexpr int kProjRows = kProjThreads * kProjNR;    // token rows per tile
constexpr int kColBytes = 64;                        // bytes of each row per streamed column block
constexpr int kProjWarps = kProjThreads / 32;
constexpr int kWarpRows = kProjRows / kProjWarps;    // token rows of a tile streamed by one warp
constexpr int kWarpStage = kWarpRows * kColBytes;    // bytes of one warp's stage

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

__device__ __forceinline__ uint32_t smem_addr(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_addr(bar)), "r"(bytes)
               : "memory");
}
// true once the barrier's phase with the given parity has completed; false
// when the wait gave up (kWaitPolls polls or kWaitNs)
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity) {
  return mbar_wait_bounded(smem_addr(bar), parity, kWaitNs);
}
// 2-D tile copy global -> shared through a tensor map (x: element column, y: row)
__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, int x, int y, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
          smem_addr(dst)),
      "l"(map), "r"(x), "r"(y), "r"(smem_addr(bar))
      : "memory");
}

// shared-memory layout (byte offsets), computed on the host
struct ProjSmem {
  int keys;    // [2 * Rk] int (MODE 1)
  int hist;    // [256] u32 (MODE 2)
  int cstage;  // [kProjRows][R] code bytes (MODE 2, odd R packing)
  int bars;    // [warps][stages] u64 stage barriers (TMA)
  int xbuf;    // [warps][stages][kWarpStage] (TMA), 1024-byte aligned
  int stages;
  int total;
};

// acc[q] holds coefficients (2q, 2q + 1) of one row as a packed f32x2 register
// pair; each basis pair loaded from shared memory feeds both of a thread's rows
template <int RG>
__device__ __forceinline__ void fma_rows(unsigned long long (&acc)[kProjNR][RG / 2], const float (&xv)[kProjNR],
                                         const float* vrow) {
  unsigned long long xx[kProjNR];
#pragma unroll
  for (int rr = 0; rr < kProjNR; ++rr) asm("mov.b64 %0, {%1, %1};" : "=l"(xx[rr]) : "f"(xv[rr]));
  const ulonglong2* vr = reinterpret_cast<const ulonglong2*>(vrow);
#pragma unroll
  for (int q = 0; q < RG / 4; ++q) {
    const ulonglong2 v = vr[q];
#pragma unroll
    for (int rr = 0; rr < kProjNR; ++rr) {
      asm("fma.rn.f32x2 %0, %1, %2, %0;" : "+l"(acc[rr][2 * q]) : "l"(xx[rr]), "l"(v.x));
      asm("fma.rn.f32x2 %0, %1, %2, %0;" : "+l"(acc[rr][2 * q + 1]) : "l"(xx[rr]), "l"(v.y));
    }
  }
}

template <typename TIn, int RG, bool CALIB, int MODE, bool TMA>
__global__ void __launch_bounds__(kProjThreads, (RG <= 12 ? 4 : RG == 32 ? 3 : 2))
    k_project(const __grid_constant__ CUtensorMap xmap, const TIn* __restrict__ x, int H, int T, int D,
              const float* __restrict__ bvt, const uint64_t* __restrict__ ranks, int R, int Rpad, ProjSmem L,
              ProjectOut o) {
  extern __shared__ __align__(1024) uint8_t smraw[];
  float* vT = reinterpret_cast<float*>(smraw);  // [D][Rpad]
  const int Rk = (R + 3) & ~3;
  int* skmin = reinterpret_cast<int*>(smraw + L.keys);
  int* skmax = skmin + Rk;
  uint32_t* shist = reinterpret_cast<uint32_t*>(smraw + L.hist);
  uint8_t* cstage = smraw + L.cstage;
  const int tid = threadIdx.x, w = tid >> 5, lane = tid & 31;
  // this warp's pipeline: its stage barriers and stage buffers
  uint64_t* wbar = reinterpret_cast<uint64_t*>(smraw + L.bars) + w * L.stages;
  uint8_t* wbuf = smraw + L.xbuf + (size_t)w * L.stages * kWarpStage;
  const int tiles = (T + kProjRows - 1) / kProjRows;
  const long long items = (long long)H * tiles;
  const long long i0 = items * blockIdx.x / gridDim.x;
  const long long i1 = items * (blockIdx.x + 1) / gridDim.x;
  const long long nit = i1 - i0;
  constexpr int kColElems = kColBytes / (int)sizeof(TIn);
  const int ncb = TMA ? D / kColElems : 1;  // column blocks per tile
  // several passes (r-groups) only with 32-wide groups (24 < R <= 64); below
  // that one pass, and the basis stride stays a compile-time constant
  constexpr bool kMulti = RG == 32;
  const int nrg = kMulti ? (R + RG - 1) / RG : 1;
  const int vstride = kMulti ? Rpad : RG;  // floats per basis row in shared memory
  const long long units = nit * nrg * ncb;
  const bool hist_on = (MODE == 2) && o.hist != nullptr;
  if (hist_on)
    for (int i = tid; i < 256; i += blockDim.x) shist[i] = 0u;
  if (TMA && lane == 0) {
    for (int s = 0; s < L.stages; ++s) mbar_init(&wbar[s], 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  __syncthreads();

  // unit u = column block (u mod ncb) of r-group pass ((u / ncb) mod nrg) of
  // item (u / (ncb nrg)); this warp's 64 rows of it go to stage u mod stages,
  // copied by lane 0 (a later pass copies the tile again, from L2)
  long long issued = 0;
  auto issue = [&](long long u) {
    if (!TMA || u >= units) return;
    if (lane == 0) {
      const long long it = i0 + u / ((long long)ncb * nrg);
      const int cb = (int)(u % ncb);
      const int h = (int)(it / tiles), tile = (int)(it - (long long)h * tiles);
      const int s = (int)(u % L.stages);
      mbar_expect_tx(&wbar[s], (uint32_t)kWarpStage);
      tma_load_2d(wbuf + (size_t)s * kWarpStage, &xmap, cb * kColElems, h * T + tile * kProjRows + w * kWarpRows,
                  &wbar[s]);
    }
    issued = u + 1;
  };
  auto flush_keys = [&](int hh) {
    if (MODE == 1 && hh >= 0)
      for (int r = tid; r < R; r += blockDim.x) {
        atomicMin(&o.kmin[(size_t)hh * R + r], skmin[r]);
        atomicMax(&o.kmax[(size_t)hh * R + r], skmax[r]);
      }
  };

  for (long long u = 0; u < L.stages - 1; ++u) issue(u);
  int cur_h = -1, rank = 0;
  // A wait that runs out makes the warp dead: it computes and stores nothing
  // more but still reaches every block barrier, so no other warp is left
  // waiting; at the end it waits (bounded) for copies it has in flight.
  bool dead = false;
  long long stuck = -1;
  for (long long li = 0; li < nit; ++li) {
    const long long it = i0 + li;
    const int h = (int)(it / tiles), tile = (int)(it - (long long)h * tiles);
    const size_t g0 = (size_t)h * T + (size_t)tile * kProjRows;
    const int nrows = min(kProjRows, T - tile * kProjRows);
    bool ok[kProjNR];
    size_t g[kProjNR];
    int wrow[kProjNR];  // the row within this warp's 64
#pragma unroll
    for (int rr = 0; rr < kProjNR; ++rr) {
      wrow[rr] = lane + 32 * rr;
      const int row = w * kWarpRows + wrow[rr];
      ok[rr] = row < nrows;
      g[rr] = g0 + (ok[rr] ? row : 0);
    }
    if (h != cur_h) {  // block-uniform: this head's basis
      __syncthreads();  // every warp is done with the previous head's basis and keys
      flush_keys(cur_h);
      const uint64_t rk = ranks[h];
      rank = (int)(rk < (uint64_t)R ? rk : (uint64_t)R);
      const float* B = bvt + (size_t)h * R * D;
      // read row by row (consecutive threads, consecutive channels: coalesced)
      // with 4 loads in flight per thread, and write transposed, vT[c][r]
      const int nv = D * Rpad;
      for (int i0 = tid; i0 < nv; i0 += 4 * (int)blockDim.x) {
        float bv[4];
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          const int i = i0 + u * (int)blockDim.x, r = i / D, c = i - r * D;
          bv[u] = (i < nv && r < rank) ? __ldg(B + (size_t)r * D + c) : 0.0f;
        }
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          const int i = i0 + u * (int)blockDim.x, r = i / D, c = i - r * D;
          if (i < nv) vT[c * Rpad + r] = bv[u];
        }
      }
      if (MODE == 1)
        for (int r = tid; r < R; r += blockDim.x) {
          skmin[r] = fkey(INFINITY);
          skmax[r] = fkey(-INFINITY);
        }
      __syncthreads();
      cur_h = h;
    }
    double s1 = 0.0, s2 = 0.0;
    for (int rg = 0; rg < R; rg += RG) {
      unsigned long long acc2[kProjNR][RG / 2];
#pragma unroll
      for (int rr = 0; rr < kProjNR; ++rr)
#pragma unroll
        for (int r = 0; r < RG / 2; ++r) acc2[rr][r] = 0ull;  // +0.0f in both halves
      for (int cb = 0; cb < ncb; ++cb) {
        const long long u = (li * nrg + rg / RG) * ncb + cb;
        if (TMA) {
          if (!dead) {
            const bool okw = mbar_wait(&wbar[u % L.stages], (uint32_t)((u / L.stages) & 1));
            if (!__all_sync(0xffffffffu, okw)) {
              dead = true;
              stuck = u;
            }
          }
          __syncwarp();  // every lane is done with unit u - 1, whose stage is refilled next
          if (!dead) issue(u + L.stages - 1);
        }
        if (dead) continue;
        if (TMA) {  // vT rows are vstride floats; this pass reads columns rg .. rg + RG - 1
          constexpr int PV = Seg<TIn>::PV;
          const uint8_t* sb[kProjNR];
          int sw[kProjNR];
#pragma unroll
          for (int rr = 0; rr < kProjNR; ++rr) {
            sb[rr] = wbuf + (size_t)(u % L.stages) * kWarpStage + wrow[rr] * kColBytes;
            sw[rr] = (int)(smem_addr(sb[rr]) >> 7) & 3;  // the swizzle XORs address bits 4-5 with bits 7-8
          }
          // calibration sums of this unit's 2 x 32 elements in f32 (squares of
          // f16 inputs are exact in f32), folded into the f64 sums once per
          // unit: one conversion per 64 elements instead of one per element
          float p1 = 0.0f, p2 = 0.0f;
#pragma unroll
          for (int jj = 0; jj < kColBytes / 16; ++jj) {
            float xv[kProjNR][PV];
#pragma unroll
            for (int rr = 0; rr < kProjNR; ++rr)
              Seg<TIn>::unpack(*reinterpret_cast<const uint4*>(sb[rr] + ((jj ^ sw[rr]) << 4)), xv[rr]);
            if (CALIB && rg == 0) {  // calibration sums in the first pass only
#pragma unroll
              for (int rr = 0; rr < kProjNR; ++rr)
#pragma unroll
                for (int k = 0; k < PV; ++k) {
                  const float v = ok[rr] ? xv[rr][k] : 0.0f;
                  p1 = __fadd_rn(p1, v);
                  p2 = __fmaf_rn(v, v, p2);
                }
            }
            const float* vb = vT + (size_t)(cb * kColElems + jj * PV) * vstride + rg;
#pragma unroll
            for (int k = 0; k < PV; ++k) {
              float xk[kProjNR];
#pragma unroll
              for (int rr = 0; rr < kProjNR; ++rr) xk[rr] = xv[rr][k];
              fma_rows<RG>(acc2, xk, vb + k * vstride);
            }
          }
          if (CALIB && rg == 0) {
            s1 += (double)p1;
            s2 += (double)p2;
          }
        } else {
          for (int c = 0; c < D; ++c) {
            float xk[kProjNR];
#pragma unroll
            for (int rr = 0; rr < kProjNR; ++rr) {
              xk[rr] = ok[rr] ? ldf(x + g[rr] * D, c) : 0.0f;
              if (CALIB && rg == 0) {
                const double v = (double)xk[rr];
                s1 += v;
                s2 += v * v;
              }
            }
            fma_rows<RG>(acc2, xk, vT + (size_t)c * Rpad + rg);
          }
        }
      }
      float acc[kProjNR][RG];
#pragma unroll
      for (int rr = 0; rr < kProjNR; ++rr)
#pragma unroll
        for (int r = 0; r < RG / 2; ++r)
          asm("mov.b64 {%0, %1}, %2;" : "=f"(acc[rr][2 * r]), "=f"(acc[rr][2 * r + 1]) : "l"(acc2[rr][r]));
#pragma unroll
      for (int rr = 0; rr < kProjNR; ++rr)
#pragma unroll
        for (int r = 0; r < RG; ++r)
          if (rg + r >= rank) acc[rr][r] = 0.0f;  // projection.rs:96

      if (MODE == 1 && !dead) {  // column min/max of this tile into the block's keys
#pragma unroll
        for (int r = 0; r < RG; ++r) {
          if (rg + r < R) {  // warp-uniform
            float mn = INFINITY, mx = -INFINITY;
#pragma unroll
            for (int rr = 0; rr < kProjNR; ++rr)
              if (ok[rr]) mm_update(acc[rr][r], mn, mx);
            warp_minmax(mn, mx);
            if (lane == 0) {
              atomicMin(&skmin[rg + r], fkey(mn));
              atomicMax(&skmax[rg + r], fkey(mx));
            }
          }
        }
      }
      if ((MODE == 0 || MODE == 1) && !dead) {
#pragma unroll
        for (int rr = 0; rr < kProjNR; ++rr)
          if (ok[rr]) {
            float* pr = o.P + g[rr] * R + rg;
            if (rg + RG <= R && (R & 3) == 0) {
#pragma unroll
              for (int q = 0; q < RG / 4; ++q)
                reinterpret_cast<float4*>(pr)[q] =
                    make_float4(acc[rr][4 * q], acc[rr][4 * q + 1], acc[rr][4 * q + 2], acc[rr][4 * q + 3]);
            } else {
#pragma unroll
              for (int r = 0; r < RG; ++r)
                if (rg + r < R) pr[r] = acc[rr][r];
            }
          }
      } else if (MODE == 2) {  // R <= RG
        const bool direct = o.packed == nullptr || (R & 1) == 0;
        if (!dead) {
#pragma unroll
          for (int rr = 0; rr < kProjNR; ++rr) {
            float mn = INFINITY, mx = -INFINITY;
#pragma unroll
            for (int r = 0; r < RG; ++r)
              if (r < R) mm_update(acc[rr][r], mn, mx);
            const float scale = make_scale(mn, mx, o.levels);
            const float inv = __frcp_rn(scale);
            uint32_t cd[RG];
#pragma unroll
            for (int r = 0; r < RG; ++r) cd[r] = (r < R) ? qcode_fast(acc[rr][r], mn, scale, inv, o.levels) : 0u;
            if (ok[rr]) {
              o.scales[g[rr]] = scale;
              o.mins[g[rr]] = mn;
            }
            if (!direct) {  // odd R: pairs run across rows; pack the tile through shared memory
#pragma unroll
              for (int r = 0; r < RG; ++r)
                if (r < R) cstage[(w * kWarpRows + wrow[rr]) * R + r] = (uint8_t)cd[r];
            } else if (ok[rr] && o.packed) {  // this row's codes start on a byte boundary
              uint8_t* dp = o.packed + (g[rr] * R) / 2;
#pragma unroll
              for (int b = 0; b < RG / 2; ++b)
                if (2 * b < R) {
                  const uint32_t byte = (cd[2 * b] & 0xFu) | ((cd[2 * b + 1] & 0xFu) << 4);
                  dp[b] = (uint8_t)byte;
                  if (hist_on) atomicAdd(&shist[byte], 1u);
                }
            } else if (ok[rr]) {
              uint8_t* dc = o.codes + g[rr] * R;
#pragma unroll
              for (int r = 0; r < RG; ++r)
                if (r < R) {
                  dc[r] = (uint8_t)cd[r];
                  if (hist_on) atomicAdd(&shist[cd[r]], 1u);
                }
            }
          }
        }
        if (!direct) {  // block-uniform
          __syncthreads();
          const int cnt = nrows * R;
          uint8_t* dp = o.packed + (g0 * R) / 2;
          for (int b = tid; b < cnt / 2; b += blockDim.x) {
            const uint32_t byte = (cstage[2 * b] & 0xFu) | ((uint32_t)(cstage[2 * b + 1] & 0xFu) << 4);
            dp[b] = (uint8_t)byte;
            if (hist_on) atomicAdd(&shist[byte], 1u);
          }
          __syncthreads();
        }
      }
    }
    if (CALIB && !dead) {  // this warp's share of the item, one partial slot per warp
      s1 = warp_sum(s1);
      s2 = warp_sum(s2);
      if (lane == 0) {
        const size_t slot = ((size_t)h * tiles + tile) * kProjWarps + w;
        o.cpart[2 * slot] = s1;
        o.cpart[2 * slot + 1] = s2;
      }
    }
  }
  __syncthreads();
  flush_keys(cur_h);
  if (hist_on)
    for (int i = tid; i < 256; i += blockDim.x)
      if (shist[i]) atomicAdd(&o.hist[i], shist[i]);
  if (dead) {
    // copies still in flight land (bounded waits) before the block's shared memory is released
    if (lane == 0 && o.status) atomicOr(o.status, kDevErrTimeout);
    for (long long u = stuck; u < issued; ++u) mbar_wait(&wbar[u % L.stages], (uint32_t)((u / L.stages) & 1));
  }
}

struct LaunchCache {
  int smem = -1;
  int per_sm = 0;
};

PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder() {
  return reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(tensor_map_encode_fn());
}

// [H*T rows, D columns] of TIn, boxes of kProjRows rows x 64 bytes, 64-byte swizzle
template <typename TIn>
bool encode_rows_map(CUtensorMap* map, const TIn* x, size_t rows, size_t D) {
  auto enc = tensor_map_encoder();
  if (!enc) return false;
  const cuuint64_t gdim[2] = {(cuuint64_t)D, (cuuint64_t)rows};
  const cuuint64_t gstride[1] = {(cuuint64_t)(D * sizeof(TIn))};
  const cuuint32_t box[2] = {(cuuint32_t)(kColBytes / sizeof(TIn)), (cuuint32_t)kWarpRows};
  const cuuint32_t estride[2] = {1, 1};
  const CUtensorMapDataType dt =
      sizeof(TIn) == 2 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT32;
  return enc(map, dt, 2, const_cast<TIn*>(x), gdim, gstride, box, estride, CU_TENSOR_MAP_INTERLEAVE_NONE,
             CU_TENSOR_MAP_SWIZZLE_64B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
             CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

template <typename TIn, int RG, bool CALIB, int MODE, bool TMA>
cudaError_t project_launch(const CUtensorMap& map, const TIn* x, size_t H, size_t T, size_t D, const float* bvt,
                           const uint64_t* ranks, size_t R, const ProjectOut& o, cudaStream_t st) {
  auto kern = k_project<TIn, RG, CALIB, MODE, TMA>;
  // per-device launch facts, looked up once per kernel instantiation
  constexpr int kDevs = 64;
  static int max_dyn[kDevs] = {};  // dynamic shared memory this kernel may opt in to (0: not yet known)
  static int opted[kDevs] = {};    // opted in so far
  static int sms[kDevs] = {};
  static LaunchCache cache[kDevs][4];
  static std::mutex mu;  // the caches above are shared by every host thread that launches
  cudaError_t e;
  int dev = 0;
  if ((e = cudaGetDevice(&dev)) != cudaSuccess) return e;
  if (dev < 0 || dev >= kDevs) return cudaErrorInvalidDevice;
  std::unique_lock<std::mutex> lk(mu);
  if (!max_dyn[dev]) {
    int optin = 0;
    cudaFuncAttributes fa{};
    if ((e = cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev)) != cudaSuccess) return e;
    if ((e = cudaFuncGetAttributes(&fa, kern)) != cudaSuccess) return e;
    if ((e = cudaDeviceGetAttribute(&sms[dev], cudaDevAttrMultiProcessorCount, dev)) != cudaSuccess) return e;
    max_dyn[dev] = std::max(1, optin - (int)fa.sharedSizeBytes);
  }
  const int Rpad = (int)(((R + RG - 1) / RG) * RG);
  const int Rk = (int)((R + 3) & ~size_t(3));
  ProjSmem L{};
  int off = (int)(D * Rpad * sizeof(float));
  L.keys = off;
  off += 2 * Rk * 4;
  off = (off + 15) & ~15;
  L.hist = off;
  off += (MODE == 2) ? 256 * 4 : 0;
  L.cstage = off;
  off += (MODE == 2 && o.packed && (R & 1)) ? kProjRows * (int)R : 0;  // odd R packs through shared memory
  off = (off + 15) & ~15;
  L.bars = off;
  off += 8 * kProjWarps * 4;  // up to 4 stage barriers per warp
  off = (off + 1023) & ~1023;  // swizzled stages start on a 1024-byte boundary
  L.xbuf = off;
  // three stages per warp; two for the 32-wide groups (R > 24), whose basis
  // copy is large, so that three CTAs fit on an SM
  L.stages = TMA ? (RG == 32 ? 2 : 3) : 0;
  off += kProjWarps * L.stages * kWarpStage;
  L.total = off;
  if (L.total > max_dyn[dev]) return cudaErrorInvalidValue;
  if (L.total > opted[dev] && L.total > 48 * 1024 - 1024) {
    if ((e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, L.total)) != cudaSuccess)
      return e;
    opted[dev] = L.total;
  }
  int per_sm = 0;
  for (auto& c : cache[dev])
    if (c.smem == L.total) per_sm = c.per_sm;
  if (per_sm == 0) {
    if ((e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, kProjThreads, L.total)) != cudaSuccess)
      return e;
    per_sm = std::max(per_sm, 1);
    for (auto& c : cache[dev])
      if (c.smem < 0) {
        c.smem = L.total;
        c.per_sm = per_sm;
        break;
      }
  }
  const int nsm = sms[dev];
  lk.unlock();
  const size_t items = H * ((T + kProjRows - 1) / kProjRows);
  const size_t grid = std::max<size_t>(1, std::min<size_t>(items, (size_t)per_sm * nsm));
  kern<<<(unsigned)grid, kProjThreads, L.total, st>>>(map, x, (int)H, (int)T, (int)D, bvt, ranks, (int)R, Rpad, L, o);
  note_launches(1);
  return cudaGetLastError();
}

template <typename TIn, int RG, bool TMA>
cudaError_t project_mode(const CUtensorMap& map, const TIn* x, size_t H, size_t T, size_t D, const float* bvt,
                         const uint64_t* ranks, size_t R, const ProjectOut& o, cudaStream_t st) {
  if (o.mode == 1) {
    if (o.cpart) return project_launch<TIn, RG, true, 1, TMA>(map, x, H, T, D, bvt, ranks, R, o, st);
    return project_launch<TIn, RG, false, 1, TMA>(map, x, H, T, D, bvt, ranks, R, o, st);
  }
  if (o.cpart) return cudaErrorInvalidValue;  // calibration is fused into the key path only
  if (o.mode == 2) {
    if (R > (size_t)RG) return cudaErrorInvalidValue;
    return project_launch<TIn, RG, false, 2, TMA>(map, x, H, T, D, bvt, ranks, R, o, st);
  }
  return project_launch<TIn, RG, false, 0, TMA>(map, x, H, T, D, bvt, ranks, R, o, st);
}

template <typename TIn, bool TMA>
cudaError_t project_rg(const CUtensorMap& map, const TIn* x, size_t H, size_t T, size_t D, const float* bvt,
                       const uint64_t* ranks, size_t R, const ProjectOut& o, cudaStream_t st) {
  if (R <= 4) return project_mode<TIn, 4, TMA>(map, x, H, T, D, bvt, ranks, R, o, st);
  if (R <= 8) return project_mode<TIn, 8, TMA>(map, x, H, T, D, bvt, ranks, R, o, st);
  if (R <= 12) return project_mode<TIn, 12, TMA>(map, x, H, T, D, bvt, ranks, R, o, st);
  if (R <= 16) return project_mode<TIn, 16, TMA>(map, x, H, T, D, bvt, ranks, R, o, st);
  if (R <= 24) return project_mode<TIn, 24, TMA>(map, x, H, T, D, bvt, ranks, R, o, st);
  // several r-groups: each pass over a tile computes 32 coefficients; the
  // tensor-copy path streams the tile once per pass (the later passes from L2)
  if (R <= 64) return project_mode<TIn, 32, TMA>(map, x, H, T, D, bvt, ranks, R, o, st);
  return project_mode<TIn, 32, false>(map, x, H, T, D, bvt, ranks, R, o, st);
}

template <typename TIn>
cudaError_t project_typed(const TIn* x, size_t H, size_t T, size_t D, const float* bvt, const uint64_t* ranks,
                          size_t R, const ProjectOut& o, cudaStream_t st) {
  CUtensorMap map{};
  const bool tma = (D * sizeof(TIn)) % kColBytes == 0 && aligned(x, 16) && R <= 64 && H * T < (1ull << 31) &&
                   encode_rows_map(&map, x, H * T, D);
  if (tma) return project_rg<TIn, true>(map, x, H, T, D, bvt, ranks, R, o, st);
  return project_rg<TIn, false>(map, x, H, T, D, bvt, ranks, R, o, st);
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

// The same sums from 16-byte vectors (8 halves or 4 floats), four vectors in
// flight per thread; every element is still converted to fp64 and added on
// its own. Requires a 16-byte aligned x and per_head * sizeof(TIn) a multiple
// of 16 (every head's block and every tile start on a vector).
template <typename TIn>
__global__ void __launch_bounds__(256) k_calib_partials_v(const TIn* __restrict__ x, size_t per_head,
                                                          double* __restrict__ cpart) {
  constexpr int V = 16 / (int)sizeof(TIn);  // elements per vector
  constexpr int kFlight = 4;
  const int h = blockIdx.y;
  const size_t e0 = (size_t)blockIdx.x * kCalibTile;
  const size_t e1 = (e0 + kCalibTile < per_head) ? e0 + kCalibTile : per_head;
  const uint4* xv = reinterpret_cast<const uint4*>(x + (size_t)h * per_head);
  const size_t q0 = e0 / V, q1 = e1 / V;
  double s1 = 0.0, s2 = 0.0;
  auto add = [&](const uint4& u) {
    float f[8];
    if constexpr (sizeof(TIn) == 2) {
      const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const float2 t = __half22float2(*reinterpret_cast<const __half2*>(&w[k]));
        f[2 * k] = t.x;
        f[2 * k + 1] = t.y;
      }
    } else {
      f[0] = __uint_as_float(u.x);
      f[1] = __uint_as_float(u.y);
      f[2] = __uint_as_float(u.z);
      f[3] = __uint_as_float(u.w);
    }
#pragma unroll
    for (int k = 0; k < V; ++k) {
      const double v = (double)f[k];
      s1 += v;
      s2 += v * v;
    }
  };
  size_t q = q0 + threadIdx.x;
  for (; q + (kFlight - 1) * blockDim.x < q1; q += kFlight * blockDim.x) {
    uint4 u[kFlight];
#pragma unroll
    for (int j = 0; j < kFlight; ++j) u[j] = __ldg(xv + q + j * blockDim.x);
#pragma unroll
    for (int j = 0; j < kFlight; ++j) add(u[j]);
  }
  for (; q < q1; q += blockDim.x) add(__ldg(xv + q));
  block_sum2(s1, s2);
  if (threadIdx.x == 0) {
    const size_t slot = (size_t)h * gridDim.x + blockIdx.x;
    cpart[2 * slot] = s1;
    cpart[2 * slot + 1] = s2;
  }
}

// calibration.rs:56-71: variance per head, clamped at 0, normalised by the max
// (uniform 0.5 when the max is below 1e-12). One block; warp w sums the
// partials of heads w, w + 8, ...: lane l adds every 32nd partial in order,
// then a fixed shuffle tree combines the lanes, so the result does not depend
// on scheduling. A head's variance is kept in its own first partial slot
// (only the warp that read the head's partials writes there), so the kernel
// needs no shared memory per head and takes any number of heads.
__global__ void __launch_bounds__(256) k_calib_finalize(double* __restrict__ cpart, int H, int tiles, double n,
                                                        float* __restrict__ scores) {
  __shared__ double wmax[8];
  const int w = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = blockDim.x >> 5;
  for (int h = w; h < H; h += nw) {
    double s1 = 0.0, s2 = 0.0;
    for (int k0 = lane; k0 < tiles; k0 += 32 * 8) {  // eight loads in flight, then the adds in order
      double a[8], b[8];
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const int k = k0 + 32 * j;
        const bool in = k < tiles;
        a[j] = in ? cpart[2 * ((size_t)h * tiles + k)] : 0.0;
        b[j] = in ? cpart[2 * ((size_t)h * tiles + k) + 1] : 0.0;
      }
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        s1 += a[j];
        s2 += b[j];
      }
    }
    s1 = warp_sum(s1);
    s2 = warp_sum(s2);
    if (lane == 0) {
      const double mean = s1 / n;
      const double v = (s2 / n) - (mean * mean);
      cpart[2 * (size_t)h * tiles] = (isnan(v) || v < 0.0) ? 0.0 : v;  // variance.max(0.0)
    }
  }
  __syncthreads();
  double m = 0.0;
  for (int h = threadIdx.x; h < H; h += blockDim.x) {
    const double v = cpart[2 * (size_t)h * tiles];
    m = v > m ? v : m;
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const double u = __shfl_xor_sync(0xffffffffu, m, o);
    m = u > m ? u : m;
  }
  if (lane == 0) wmax[w] = m;
  __syncthreads();
  m = 0.0;
  for (int k = 0; k < nw; ++k) m = wmax[k] > m ? wmax[k] : m;
  for (int h = threadIdx.x; h < H; h += blockDim.x)
    scores[h] = (m < 1e-12) ? 0.5f : (float)(cpart[2 * (size_t)h * tiles] / m);
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

// Register-basis variant (D <= 128, D % 4 == 0, R <= 16): a persistent grid
// walks (head, 128-token tile) items; lane l of every warp keeps columns
// 4l..4l+3 of the head's basis rows in registers for as long as the head
// lasts. Each thread dequantizes one token row of the tile into shared memory
// as duplicated pairs (d, d), so one broadcast 16-byte load supplies the f32x2
// multiplicand of two rows; warp w then computes rows 8g..8g+7 for
// g = w, w + 4, ... with packed fma.rn.f32x2 (EXACT: __fmul_rn then
// __fadd_rn per element). The next
// tile's codes and scales are read into registers before the current tile is
// computed. Terms r >= rank get d = 0 and a zero basis row, which leave every
// sum unchanged (it starts at +0.0), so results equal the per-rank loop.
template <int MODE, bool EXACT, int RG>
__global__ void __launch_bounds__(128, (RG >= 12 ? 3 : 4)) k_reconstruct_reg(const uint8_t* __restrict__ codes,
                                                         size_t ncode_bytes, const float* __restrict__ raw,
                                                         const float* __restrict__ scales,
                                                         const float* __restrict__ mins, int axis, int H, int T,
                                                         int R, int D, const float* __restrict__ bvt,
                                                         const uint64_t* __restrict__ ranks, float* __restrict__ out) {
  __shared__ __align__(16) unsigned long long dT2[2][RG][kRecRows];  // (d, d) per (r, row)
  const int tid = threadIdx.x, w = tid >> 5, lane = tid & 31;
  const int tiles = (T + kRecRows - 1) / kRecRows;
  const long long items = (long long)H * tiles;
  const long long i0 = items * blockIdx.x / gridDim.x;
  const long long i1 = items * (blockIdx.x + 1) / gridDim.x;
  const bool col_ok = 4 * lane < D;

  // this thread's row of item `it`: raw inputs fetched now, dequantized later
  struct RowIn {
    CodeWords<MODE == 0 ? 1 : code_words<MODE == 2, RG>()> cw;  // codes, as loaded
    float raw[MODE == 0 ? RG : 1];
    float sc, mn;
  };
  auto fetch = [&](long long it, RowIn& in) {
    const int h = (int)(it / tiles), tile = (int)(it - (long long)h * tiles);
    const size_t t = (size_t)tile * kRecRows + tid;
    const bool ok = t < (size_t)T;
    const size_t g = (size_t)h * T + (ok ? t : 0);
    if (MODE != 0 && axis != KVF_PER_CHANNEL) {
      in.sc = ok ? __ldg(scales + g) : 0.0f;
      in.mn = ok ? __ldg(mins + g) : 0.0f;
    }
    if (MODE == 0) {
#pragma unroll
      for (int r = 0; r < RG; ++r) in.raw[r] = (ok && r < R) ? __ldg(raw + g * R + r) : 0.0f;
    } else {
      load_code_words<MODE == 2>(codes, ncode_bytes, g * R, ok, in.cw);
    }
  };
  auto stage = [&](long long it, const RowIn& in, int buf, int rank) {
    const int h = (int)(it / tiles), tile = (int)(it - (long long)h * tiles);
    const bool ok = (size_t)tile * kRecRows + tid < (size_t)T;
#pragma unroll
    for (int r = 0; r < RG; ++r) {
      float d = 0.0f;
      if (ok && r < rank) {
        if (MODE == 0) {
          d = in.raw[r];
        } else {
          float sc = in.sc, mn = in.mn;
          if (axis == KVF_PER_CHANNEL) {
            sc = __ldg(scales + (size_t)h * R + r);
            mn = __ldg(mins + (size_t)h * R + r);
          }
          d = __fadd_rn(__fmul_rn((float)code_at<MODE == 2>(in.cw, r), sc), mn);
        }
      }
      unsigned long long dd;
      asm("mov.b64 %0, {%1, %1};" : "=l"(dd) : "f"(d));
      dT2[buf][r][tid] = dd;
    }
  };
  auto rank_of = [&](long long it) {
    const int h = (int)(it / tiles);
    const uint64_t rk = ranks[h];
    return (int)(rk < (uint64_t)R ? rk : (uint64_t)R);
  };

  ulonglong2 vreg[RG];  // basis columns 4l..4l+3 as two packed pairs per row
  int cur_h = -1;
  RowIn nxt;
  if (i0 < i1) {
    fetch(i0, nxt);
    stage(i0, nxt, 0, rank_of(i0));
  }
  __syncthreads();
  for (long long it = i0; it < i1; ++it) {
    const int buf = (int)((it - i0) & 1);
    const int h = (int)(it / tiles), tile = (int)(it - (long long)h * tiles);
    if (it + 1 < i1) fetch(it + 1, nxt);  // loads in flight during this tile's arithmetic
    if (h != cur_h) {
      const int rank = rank_of(it);
      const float* B = bvt + (size_t)h * R * D;
#pragma unroll
      for (int r = 0; r < RG; ++r) {
        float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
        if (r < rank && col_ok) v = __ldg(reinterpret_cast<const float4*>(B + (size_t)r * D + 4 * lane));
        asm("mov.b64 %0, {%1, %2};" : "=l"(vreg[r].x) : "f"(v.x), "f"(v.y));
        asm("mov.b64 %0, {%1, %2};" : "=l"(vreg[r].y) : "f"(v.z), "f"(v.w));
      }
      cur_h = h;
    }
    const size_t t0 = (size_t)tile * kRecRows;
    for (int g8 = w; g8 < kRecRows / 8; g8 += 4) {
      unsigned long long acc[8][2];
#pragma unroll
      for (int i = 0; i < 8; ++i) acc[i][0] = acc[i][1] = 0ull;  // +0.0f
#pragma unroll
      for (int r = 0; r < RG; ++r) {
        const ulonglong2* dp = reinterpret_cast<const ulonglong2*>(&dT2[buf][r][8 * g8]);
#pragma unroll
        for (int p = 0; p < 4; ++p) {
          const ulonglong2 d2 = dp[p];
          const unsigned long long dd[2] = {d2.x, d2.y};
#pragma unroll
          for (int e = 0; e < 2; ++e) {
            const int i = 2 * p + e;
            if (EXACT) {  // separately rounded product and sum, element by element
              float a[4], v[4], d, d2;
              asm("mov.b64 {%0, %1}, %2;" : "=f"(a[0]), "=f"(a[1]) : "l"(acc[i][0]));
              asm("mov.b64 {%0, %1}, %2;" : "=f"(a[2]), "=f"(a[3]) : "l"(acc[i][1]));
              asm("mov.b64 {%0, %1}, %2;" : "=f"(v[0]), "=f"(v[1]) : "l"(vreg[r].x));
              asm("mov.b64 {%0, %1}, %2;" : "=f"(v[2]), "=f"(v[3]) : "l"(vreg[r].y));
              asm("mov.b64 {%0, %1}, %2;" : "=f"(d), "=f"(d2) : "l"(dd[e]));
#pragma unroll
              for (int k = 0; k < 4; ++k) a[k] = __fadd_rn(a[k], __fmul_rn(d, v[k]));
              asm("mov.b64 %0, {%1, %2};" : "=l"(acc[i][0]) : "f"(a[0]), "f"(a[1]));
              asm("mov.b64 %0, {%1, %2};" : "=l"(acc[i][1]) : "f"(a[2]), "f"(a[3]));
            } else {
              asm("fma.rn.f32x2 %0, %1, %2, %0;" : "+l"(acc[i][0]) : "l"(dd[e]), "l"(vreg[r].x));
              asm("fma.rn.f32x2 %0, %1, %2, %0;" : "+l"(acc[i][1]) : "l"(dd[e]), "l"(vreg[r].y));
            }
          }
        }
      }
      if (col_ok) {
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const size_t t = t0 + 8 * g8 + i;
          if (t < (size_t)T) {
            float4 o4;
            asm("mov.b64 {%0, %1}, %2;" : "=f"(o4.x), "=f"(o4.y) : "l"(acc[i][0]));
            asm("mov.b64 {%0, %1}, %2;" : "=f"(o4.z), "=f"(o4.w) : "l"(acc[i][1]));
            __stcs(reinterpret_cast<float4*>(out + ((size_t)h * T + t) * D + 4 * lane), o4);
          }
        }
      }
    }
    if (it + 1 < i1) stage(it + 1, nxt, buf ^ 1, rank_of(it + 1));
    __syncthreads();  // the next tile's coefficients are in place; this buffer is free again
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
  if (D % 4 == 0 && D <= 128 && R <= 16 && aligned(out, 16) && aligned(bvt, 16) && H * T < (1ull << 31) &&
      (MODE == 0 || aligned(codes, 4))) {
    const size_t ncode = MODE == 2 ? (H * T * R + 1) / 2 : H * T * R;  // bytes of the code buffer
    // launch facts per device, shared by every host thread: each value is the
    // same whichever thread computes it, so relaxed atomics suffice
    static std::atomic<int> sms[64];
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
    int nsm = sms[dev].load(std::memory_order_relaxed);
    if (!nsm) {
      if ((e = cudaDeviceGetAttribute(&nsm, cudaDevAttrMultiProcessorCount, dev)) != cudaSuccess) return e;
      sms[dev].store(nsm, std::memory_order_relaxed);
    }
    const size_t items = H * ((T + kRecRows - 1) / kRecRows);
    // persistent grid: as many blocks as fit at once, cached per instantiation and device
#define KVF_RR(RGV)                                                                                           \
  {                                                                                                           \
    auto kern = k_reconstruct_reg<MODE, EXACT, RGV>;                                                          \
    static std::atomic<int> per_sm[64];                                                                       \
    int nb = per_sm[dev].load(std::memory_order_relaxed);                                                     \
    if (!nb) {                                                                                                \
      if ((e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&nb, kern, 128, 0)) != cudaSuccess) return e;    \
      nb = std::max(nb, 1);                                                                                   \
      per_sm[dev].store(nb, std::memory_order_relaxed);                                                       \
    }                                                                                                         \
    const unsigned grid = (unsigned)std::max<size_t>(1, std::min<size_t>(items, (size_t)nsm * nb));           \
    kern<<<grid, 128, 0, st>>>(codes, ncode, raw, scales, mins, axis, (int)H, (int)T, (int)R, (int)D, bvt, ranks, \
                               out);                                                                          \
  }
    if (R <= 4) KVF_RR(4)
    else if (R <= 8) KVF_RR(8)
    else if (R <= 12) KVF_RR(12)
    else KVF_RR(16)
#undef KVF_RR
  } else if (D % 4 == 0 && smem <= 200 * 1024 && aligned(out, 16)) {
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

void* tensor_map_encode_fn() {
  static std::once_flag once;
  static void* fn = nullptr;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q{};
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = p;
  });
  return fn;
}

// calibration partial slots per head of the projection kernel: one per (tile, warp)
size_t project_num_tiles(size_t T) { return ((T + kProjRows - 1) / kProjRows) * kProjWarps; }

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
  const size_t esz = in_dtype == KVF_IN_F16 ? 2 : 4;
  const bool vec = aligned(x, 16) && (T * D * esz) % 16 == 0;  // kCalibTile * esz is a multiple of 16 too
  if (in_dtype == KVF_IN_F16) {
    if (vec) k_calib_partials_v<__half><<<grid, 256, 0, st>>>(static_cast<const __half*>(x), T * D, calib_part);
    else k_calib_partials<__half><<<grid, 256, 0, st>>>(static_cast<const __half*>(x), T * D, calib_part);
  } else {
    if (vec) k_calib_partials_v<float><<<grid, 256, 0, st>>>(static_cast<const float*>(x), T * D, calib_part);
    else k_calib_partials<float><<<grid, 256, 0, st>>>(static_cast<const float*>(x), T * D, calib_part);
  }
  note_launches(1);
  return cudaGetLastError();
}

cudaError_t launch_calib_finalize(double* calib_part, size_t H, size_t tiles, size_t T,
                                  size_t D, float* scores, cudaStream_t st) {
  if (H == 0) return cudaSuccess;
  k_calib_finalize<<<1, 256, 0, st>>>(calib_part, (int)H, (int)tiles, (double)(T * D), scores);
  note_launches(1);
  return cudaGetLastError();
}

cudaError_t launch_dequant_reconstruct(const uint8_t* codes, const float* raw, const float* scales,
                                       const float* mins, int data_type, int axis, size_t H,
                                       size_t T, size_t R, size_t D, const float* basis_vt,
                                       const uint64_t* ranks, int exact, int engine, float* out,
                                       unsigned* status, cudaStream_t st) {
  if (H == 0 || T == 0 || D == 0) return cudaSuccess;
  // tensor cores where chosen and the shape allows them; by default beyond 16
  // coefficients, where the CUDA-core kernel is bound by its multiply-adds
  if (!exact && (engine == KVF_RECON_TENSOR_CORE || (engine == KVF_RECON_AUTO && R > 16))) {
    const cudaError_t e = launch_reconstruct_tc(codes, raw, scales, mins, data_type, axis, H, T, R, D, basis_vt,
                                                ranks, out, status, st);
    if (e != cudaErrorNotSupported) return e;
  }
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

namespace {
// one warp waits on an mbarrier that nothing arrives on
__global__ void k_selftest_mbar(unsigned* status, unsigned long long limit_ns) {
  __shared__ uint64_t bar;
  if (threadIdx.x == 0) {
    mbar_init(&bar, 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  __syncwarp();
  const bool ok = mbar_wait_bounded(smem_addr(&bar), 0, limit_ns);
  if (__any_sync(0xffffffffu, !ok) && threadIdx.x == 0 && status) atomicOr(status, kDevErrTimeout);
}
}  // namespace

cudaError_t launch_selftest_mbar(unsigned* status, unsigned long long limit_ns, cudaStream_t st) {
  k_selftest_mbar<<<1, 32, 0, st>>>(status, limit_ns);
  note_launches(1);
  return cudaGetLastError();
}

}  // namespace kvf
