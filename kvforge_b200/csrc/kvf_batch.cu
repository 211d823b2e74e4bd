// Batched short chunks: compress (and, optionally, decompress) many layers'
// chunks in one launch (sm_100a).
//
// A streaming append compresses a few dozen tokens per layer at a time
// (crates/kvforge-cpu/src/pipeline.rs:100-163 compresses each chunk as its
// own KVCache). Through the per-layer path each chunk costs eight small
// kernels; here one CTA does everything for one (layer, tensor, head):
//   1. the head's chunk rows (T <= 128, D <= 128) and basis rows into shared
//      memory;
//   2. projection: every coefficient as one fmaf chain over c = 0..D-1 from
//      +0.0, +0.0 from the rank on (projection.rs:61-140, the same definition
//      as k_project and the CPU oracle), or the input itself without a basis;
//   3. quantization per token (values) or per channel (keys) with the shared
//      KIVI helpers (quantize.rs:67-130), INT4 packed over the flat index;
//   4. optionally the reconstruction of the decompressed chunk: dequantize
//      (q * scale + min, separately rounded) and sum over r in order with one
//      fused multiply-add per term, or separately rounded in exact mode
//      (projection.rs:142-172).
// Codes, scales and mins are those of the per-layer path bit for bit; the
// reconstruction is the CUDA-core engine's. Heads of one tensor do not
// interact: the padded width R is the basis's, and a head's block of codes
// starts on a byte (the host requires T * R even, or one head).
#include <algorithm>

#include "kvf_internal.cuh"

namespace kvf {
namespace {

constexpr int kBtThreads = 256;
constexpr int kBtMaxT = 128, kBtMaxD = 128, kBtMaxR = 64;
constexpr size_t kBatchSmallCap = 16, kBatchCap = 128;  // layers per launch
constexpr int kBtLoads = 8;    // 16- or 8-byte row loads in flight per thread while staging
constexpr int kBtLoadsB = 32;  // basis element loads in flight per thread

struct BtLayout {  // byte offsets into dynamic shared memory
  int xs, vt, pp, cb, par, hist, vr, total;
  int xstride;  // floats per x row (D + 1: rows on different banks)
  int vstride;  // floats per basis column (64 coefficients + 4: columns c and c + 1 on different banks)
  int tstride;  // floats per row of the transposed dequantized coefficients (T rounded up to 16)
};

__host__ __device__ inline BtLayout bt_layout(int T, int D, int Q, bool proj) {
  BtLayout L{};
  L.xstride = D + 1;
  L.vstride = kBtMaxR + 4;
  L.tstride = (T + 15) & ~15;
  int off = 0;
  L.xs = off;
  const int xfloats = ((T + 3) & ~3) * L.xstride;  // rows up to a multiple of 4 (read, never used)
  off += xfloats * 4;
  off = (off + 15) & ~15;
  L.vt = off;
  off += proj ? D * L.vstride * 4 : 0;
  L.pp = off;
  // coefficients [T][Q + 1], later the dequantized ones transposed [Q][tstride]
  // (without a basis the x rows are used)
  off += proj ? ((T * (Q + 1) > Q * L.tstride ? T * (Q + 1) : Q * L.tstride) * 4 + 15) & ~15 : 0;
  L.cb = off;
  off += ((T * Q + 15) & ~15);
  L.par = off;
  off += 3 * 128 * 4;  // scale, min, 1/scale per row or per channel
  L.hist = off;
  off += 256 * 4;
  // the basis row-major [rank][D] for the reconstruction: in the x rows'
  // place (free after the projection) when they are large enough
  L.vr = L.xs;
  if (proj && xfloats < Q * D) {
    L.vr = off;
    off += Q * D * 4;
  }
  L.total = off;
  return L;
}

__device__ __forceinline__ void fma2(unsigned long long& acc, unsigned long long a, unsigned long long b) {
  asm("fma.rn.f32x2 %0, %1, %2, %0;" : "+l"(acc) : "l"(a), "l"(b));
}
__device__ __forceinline__ unsigned long long dup2(float x) {
  unsigned long long r;
  asm("mov.b64 %0, {%1, %1};" : "=l"(r) : "f"(x));
  return r;
}
__device__ __forceinline__ float2 split2(unsigned long long v) {
  float2 f;
  asm("mov.b64 {%0, %1}, %2;" : "=f"(f.x), "=f"(f.y) : "l"(v));
  return f;
}
// Projection of rows RT * rg .. + RT - 1 onto coefficients 8 cg .. 8 cg + 7.
// A warp takes 8 row groups x 4 coefficient groups, so its row loads hit 8
// different banks and its basis loads 4 different 32-byte spans.
template <int RT>
__device__ __forceinline__ void proj_rows(const float* xs, int xstride, const float* vT, int vstride, int T, int D,
                                          int Q, int rank, int ncg, float* P, int pstride) {
  const int nrg = (T + RT - 1) / RT;
  const int jobs = ((nrg + 7) & ~7) * ncg;
  for (int job = threadIdx.x; job < jobs; job += kBtThreads) {
    const int hi = job >> 3;
    const int cg = hi % ncg, rg = (job & 7) + 8 * (hi / ncg);
    if (rg >= nrg) continue;
    const int t0 = RT * rg;
    unsigned long long acc[RT][4];
#pragma unroll
    for (int i = 0; i < RT; ++i) acc[i][0] = acc[i][1] = acc[i][2] = acc[i][3] = 0ull;
    const float* xr = xs + t0 * xstride;
    const float* vb = vT + 8 * cg;
#pragma unroll 2
    for (int c = 0; c < D; ++c) {
      const ulonglong2 v01 = *reinterpret_cast<const ulonglong2*>(vb + c * vstride);
      const ulonglong2 v23 = *reinterpret_cast<const ulonglong2*>(vb + c * vstride + 4);
#pragma unroll
      for (int i = 0; i < RT; ++i) {
        const unsigned long long xx = dup2(xr[i * xstride + c]);
        fma2(acc[i][0], xx, v01.x);
        fma2(acc[i][1], xx, v01.y);
        fma2(acc[i][2], xx, v23.x);
        fma2(acc[i][3], xx, v23.y);
      }
    }
#pragma unroll
    for (int i = 0; i < RT; ++i) {
      const int t = t0 + i;
      if (t >= T) continue;
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const float2 f = split2(acc[i][q]);
        const int r = 8 * cg + 2 * q;
        if (r < Q) P[t * pstride + r] = (r < rank) ? f.x : 0.0f;  // projection.rs:96
        if (r + 1 < Q) P[t * pstride + r + 1] = (r + 1 < rank) ? f.y : 0.0f;
      }
    }
  }
}

// out rows t0 .. t0 + 7, channels 4cq .. 4cq + 3: sum over r < rank of
// dT[r][t] * vR[r][c] in r order from +0.0, one rounding per term (packed
// fma.rn.f32x2, each element rounded once) or, EXACT, product and sum
// rounded separately
template <bool EXACT>
__device__ __forceinline__ void recon_tile(const float* dT, int ts, const float* vR, int D, int rank, int t0, int cq,
                                           int T, float* out) {
  unsigned long long acc[8][2];
#pragma unroll
  for (int i = 0; i < 8; ++i) acc[i][0] = acc[i][1] = 0ull;
#pragma unroll 2
  for (int r = 0; r < rank; ++r) {
    const ulonglong2 v = *reinterpret_cast<const ulonglong2*>(vR + r * D + 4 * cq);
    const float4 d0 = *reinterpret_cast<const float4*>(dT + r * ts + t0);
    const float4 d1 = *reinterpret_cast<const float4*>(dT + r * ts + t0 + 4);
    const float dd[8] = {d0.x, d0.y, d0.z, d0.w, d1.x, d1.y, d1.z, d1.w};
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      if (EXACT) {
        const float2 a0 = split2(acc[i][0]), a1 = split2(acc[i][1]);
        const float2 v0 = split2(v.x), v1 = split2(v.y);
        const float2 b0 = make_float2(__fadd_rn(a0.x, __fmul_rn(dd[i], v0.x)), __fadd_rn(a0.y, __fmul_rn(dd[i], v0.y)));
        const float2 b1 = make_float2(__fadd_rn(a1.x, __fmul_rn(dd[i], v1.x)), __fadd_rn(a1.y, __fmul_rn(dd[i], v1.y)));
        asm("mov.b64 %0, {%1, %2};" : "=l"(acc[i][0]) : "f"(b0.x), "f"(b0.y));
        asm("mov.b64 %0, {%1, %2};" : "=l"(acc[i][1]) : "f"(b1.x), "f"(b1.y));
      } else {
        const unsigned long long xx = dup2(dd[i]);
        fma2(acc[i][0], xx, v.x);
        fma2(acc[i][1], xx, v.y);
      }
    }
  }
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    if (t0 + i < T) {
      const float2 a = split2(acc[i][0]), b = split2(acc[i][1]);
      __stcs(reinterpret_cast<float4*>(out + (size_t)(t0 + i) * D + 4 * cq), make_float4(a.x, a.y, b.x, b.y));
    }
  }
}

template <typename TIn>
__device__ __forceinline__ float4 ldx4(const TIn* p);
template <>
__device__ __forceinline__ float4 ldx4<float>(const float* p) {
  return __ldg(reinterpret_cast<const float4*>(p));
}
template <>
__device__ __forceinline__ float4 ldx4<__half>(const __half* p) {
  const uint2 u = __ldg(reinterpret_cast<const uint2*>(p));
  const float2 a = __half22float2(*reinterpret_cast<const __half2*>(&u.x));
  const float2 b = __half22float2(*reinterpret_cast<const __half2*>(&u.y));
  return make_float4(a.x, a.y, b.x, b.y);
}

// the descriptors travel as the kernel's parameter (no upload, no staging)
template <int CAP>
struct BatchArgs {
  BatchTensor t[2 * CAP];
};

template <typename TIn, int CAP>
__global__ void __launch_bounds__(kBtThreads) k_chunk_batch(const __grid_constant__ BatchArgs<CAP> args, int H,
                                                            int T, int D, int exact) {
  extern __shared__ __align__(16) uint8_t bsm[];
  const BatchTensor& d = args.t[blockIdx.z * 2 + blockIdx.y];
  const int h = blockIdx.x, tid = threadIdx.x;
  const bool proj = d.bvt != nullptr;
  const int Q = d.cols;  // R with a basis, D without
  const BtLayout L = bt_layout(T, D, Q, proj);
  float* xs = reinterpret_cast<float*>(bsm + L.xs);
  float* vT = reinterpret_cast<float*>(bsm + L.vt);
  float* P = proj ? reinterpret_cast<float*>(bsm + L.pp) : xs;
  const int pstride = proj ? Q + 1 : L.xstride;
  uint8_t* cb = bsm + L.cb;
  float* psc = reinterpret_cast<float*>(bsm + L.par);
  float* pmn = psc + 128;
  float* pinv = pmn + 128;
  uint32_t* shist = reinterpret_cast<uint32_t*>(bsm + L.hist);
  int rank = Q;
  if (proj) {
    const uint64_t rk = d.ranks[h];
    rank = (int)(rk < (uint64_t)Q ? rk : (uint64_t)Q);
  }
  const TIn* x = static_cast<const TIn*>(d.x) + (size_t)h * T * D;
  // 1. rows and basis into shared memory: a thread's first rows and its basis
  // elements are all requested before any of them is stored. Rows: thread =
  // (row tr + k * rpp, 4-column group c4); basis: warp w takes rows w, w + 8,
  // ..., lane l columns l, l + 32, ... (coalesced), stored transposed.
  const int d4 = D >> 2;
  const int rpp = kBtThreads / d4;  // rows per pass
  const int tr = tid / d4, c4 = tid - tr * d4;
  const int w = tid >> 5, lane = tid & 31;
  const float* B = proj ? d.bvt + (size_t)h * Q * D : nullptr;
  auto load_rows = [&](int t0, float4 (&xv)[kBtLoads]) {
#pragma unroll
    for (int k = 0; k < kBtLoads; ++k) {
      const int t = t0 + k * rpp;
      if (tr < rpp && t < T) xv[k] = ldx4<TIn>(x + (size_t)t * D + 4 * c4);
    }
  };
  auto store_rows = [&](int t0, const float4 (&xv)[kBtLoads]) {
#pragma unroll
    for (int k = 0; k < kBtLoads; ++k) {
      const int t = t0 + k * rpp;
      if (tr < rpp && t < T) {
        float* dst = xs + t * L.xstride + 4 * c4;
        dst[0] = xv[k].x;
        dst[1] = xv[k].y;
        dst[2] = xv[k].z;
        dst[3] = xv[k].w;
      }
    }
  };
  {  // every thread: its first rows and all its basis elements
    float4 xv[kBtLoads];
    load_rows(tr, xv);
    if (proj) {
      float bv[kBtLoadsB];
#pragma unroll
      for (int j = 0; j < kBtLoadsB; ++j) {
        const int r = w + 8 * (j >> 2), c = lane + 32 * (j & 3);
        bv[j] = (r < rank && c < D) ? __ldg(B + (size_t)r * D + c) : 0.0f;
      }
      store_rows(tr, xv);
      // vT[c][r]: 64 coefficients per column; rows from the rank on are zero
#pragma unroll
      for (int j = 0; j < kBtLoadsB; ++j) {
        const int r = w + 8 * (j >> 2), c = lane + 32 * (j & 3);
        if (c < D) vT[c * L.vstride + r] = bv[j];
      }
    } else {
      store_rows(tr, xv);
    }
  }
  for (int t0 = tr + kBtLoads * rpp; t0 < T; t0 += kBtLoads * rpp) {  // T > 8 rows per thread
    float4 xv[kBtLoads];
    load_rows(t0, xv);
    store_rows(t0, xv);
  }
  if (d.hist)
    for (int i = tid; i < 256; i += kBtThreads) shist[i] = 0u;
  __syncthreads();

  // 2. projection: thread = RT token rows x 8 coefficients (packed pairs); one
  // pair of 16-byte basis loads feeds all RT rows, and every coefficient is
  // its own chain over c in order (fma.rn.f32x2 rounds each element once, as
  // fmaf). RT = 4 for wide bases, fewer rows per thread (more threads busy)
  // for narrow ones.
  if (proj) {
    const int ncg = (Q + 7) >> 3;
    if (ncg >= 6) proj_rows<4>(xs, L.xstride, vT, L.vstride, T, D, Q, rank, ncg, P, pstride);
    else if (ncg >= 3) proj_rows<2>(xs, L.xstride, vT, L.vstride, T, D, Q, rank, ncg, P, pstride);
    else proj_rows<1>(xs, L.xstride, vT, L.vstride, T, D, Q, rank, ncg, P, pstride);
    __syncthreads();
  }

  // 3. quantization
  const float levels = d.levels;
  if (d.axis == KVF_PER_TOKEN) {
    // eight lanes per row, four rows per warp at a time
    const int sub = lane & 7;
    for (int t = w * 4 + (lane >> 3); t < ((T + 3) & ~3); t += 4 * (kBtThreads / 32)) {
      const bool in = t < T;
      float mn = INFINITY, mx = -INFINITY;
      if (in)
        for (int r = sub; r < Q; r += 8) mm_update(P[t * pstride + r], mn, mx);
#pragma unroll
      for (int o = 4; o > 0; o >>= 1) {
        mn = fminf(mn, __shfl_xor_sync(0xffffffffu, mn, o));
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
      }
      if (in) {
        const float scale = make_scale(mn, mx, levels);
        const float inv = __frcp_rn(scale);
        for (int r = sub; r < Q; r += 8) cb[t * Q + r] = (uint8_t)qcode_fast(P[t * pstride + r], mn, scale, inv, levels);
        if (sub == 0) {
          d.scales[(size_t)h * T + t] = scale;
          d.mins[(size_t)h * T + t] = mn;
          psc[t] = scale;
          pmn[t] = mn;
        }
      }
    }
  } else {
    for (int r = tid; r < Q; r += kBtThreads) {
      float mn = INFINITY, mx = -INFINITY;
#pragma unroll 8
      for (int t = 0; t < T; ++t) mm_update(P[t * pstride + r], mn, mx);
      const float scale = make_scale(mn, mx, levels);
      psc[r] = scale;
      pmn[r] = mn;
      pinv[r] = __frcp_rn(scale);
      d.scales[(size_t)h * Q + r] = scale;
      d.mins[(size_t)h * Q + r] = mn;
    }
    __syncthreads();
    for (int i = tid; i < T * Q; i += kBtThreads) {
      const int t = i / Q, r = i - t * Q;
      cb[i] = (uint8_t)qcode_fast(P[t * pstride + r], pmn[r], psc[r], pinv[r], levels);
    }
  }
  __syncthreads();

  // codes of the head's block, INT4 pairs over the flat index (the block
  // starts on a byte)
  const size_t f0 = (size_t)h * T * Q;
  const int n = T * Q;
  if (d.data_type == KVF_INT4) {
    uint8_t* dp = d.packed + f0 / 2;
    for (int k = tid; k < (n + 1) / 2; k += kBtThreads) {
      const uint32_t lo = cb[2 * k], hi = (2 * k + 1 < n) ? cb[2 * k + 1] : 0u;
      const uint32_t byte = (lo & 0xFu) | ((hi & 0xFu) << 4);
      dp[k] = (uint8_t)byte;
      if (d.hist) atomicAdd(&shist[byte], 1u);
    }
  } else {
    for (int k = tid; k < n; k += kBtThreads) {
      d.packed[f0 + k] = cb[k];
      if (d.hist) atomicAdd(&shist[cb[k]], 1u);
    }
  }

  // 4. the decompressed chunk: dequantized coefficients, then the sum over r
  if (d.out) {
    float* out = d.out + (size_t)h * T * D;
    if (!proj) {
      for (int i = tid; i < T * D; i += kBtThreads) {
        const int t = i / D, c = i - t * D;
        const float sc = (d.axis == KVF_PER_TOKEN) ? psc[t] : psc[c];
        const float mn = (d.axis == KVF_PER_TOKEN) ? pmn[t] : pmn[c];
        __stcs(out + i, dq(cb[i], sc, mn));
      }
    } else {
      // dT[r][t] = q * scale + min (rows from T to tstride zero); vR[r][c]
      // the basis row-major, from its transposed copy
      float* dT = P;
      float* vR = reinterpret_cast<float*>(bsm + L.vr);
      const int ts = L.tstride;
      for (int r = w; r < rank; r += kBtThreads / 32)
        for (int t = lane; t < ts; t += 32) {
          float v = 0.0f;
          if (t < T) {
            const float sc = (d.axis == KVF_PER_TOKEN) ? psc[t] : psc[r];
            const float mn = (d.axis == KVF_PER_TOKEN) ? pmn[t] : pmn[r];
            v = dq(cb[t * Q + r], sc, mn);
          }
          dT[r * ts + t] = v;
        }
      for (int r = w; r < rank; r += kBtThreads / 32)
        for (int c = lane; c < D; c += 32) vR[r * D + c] = vT[c * L.vstride + r];
      __syncthreads();
      // thread = 8 token rows x 4 channels (a warp: 32 channel quads of the
      // same rows): one 16-byte basis load and two broadcast 16-byte loads of
      // coefficients per r, one 16-byte streaming store per row
      const int nrg = (T + 7) >> 3, ncq = D >> 2;
      for (int job = tid; job < nrg * ncq; job += kBtThreads) {
        const int cq = job % ncq, rg = job / ncq;
        if (exact) recon_tile<true>(dT, ts, vR, D, rank, 8 * rg, cq, T, out);
        else recon_tile<false>(dT, ts, vR, D, rank, 8 * rg, cq, T, out);
      }
    }
  }
  if (d.hist) {
    __syncthreads();
    for (int i = tid; i < 256; i += kBtThreads)
      if (shist[i]) atomicAdd(&d.hist[i], shist[i]);
  }
}

}  // namespace

bool chunk_batch_fits(int in_dtype, size_t H, size_t T, size_t D, size_t Q, bool proj) {
  if (in_dtype != KVF_IN_F16 && in_dtype != KVF_IN_F32) return false;
  if (T == 0 || T > (size_t)kBtMaxT || D == 0 || D > (size_t)kBtMaxD || D % 4 || Q == 0 || H == 0 || H > 65535)
    return false;
  if (proj && Q > (size_t)kBtMaxR) return false;
  if (!proj && Q != D) return false;
  if (H > 1 && (T * Q) % 2) return false;  // a head's INT4 block starts on a byte
  return bt_layout((int)T, (int)D, (int)Q, proj).total <= 200 * 1024;
}

namespace {
template <typename TIn, int CAP>
cudaError_t launch_group(const BatchTensor* descs, size_t L, size_t H, size_t T, size_t D, int smem, int exact,
                         cudaStream_t st) {
  BatchArgs<CAP> a;
  for (size_t i = 0; i < 2 * L; ++i) a.t[i] = descs[i];
  auto kern = k_chunk_batch<TIn, CAP>;
  if (smem > (int)kSmemOptIn) {
    const cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e != cudaSuccess) return e;
  }
  kern<<<dim3((unsigned)H, 2, (unsigned)L), kBtThreads, smem, st>>>(a, (int)H, (int)T, (int)D, exact);
  note_launches(1);
  return cudaGetLastError();
}
template <typename TIn>
cudaError_t launch_typed(const BatchTensor* descs, size_t L, size_t H, size_t T, size_t D, int smem, int exact,
                         cudaStream_t st) {
  // up to 16 layers: a 3 KB parameter block; else groups of 128 (24 KB)
  if (L <= kBatchSmallCap) return launch_group<TIn, kBatchSmallCap>(descs, L, H, T, D, smem, exact, st);
  for (size_t l0 = 0; l0 < L; l0 += kBatchCap) {
    const cudaError_t e = launch_group<TIn, kBatchCap>(descs + 2 * l0, std::min(L - l0, kBatchCap), H, T, D, smem,
                                                       exact, st);
    if (e != cudaSuccess) return e;
  }
  return cudaSuccess;
}
}  // namespace

cudaError_t launch_chunk_batch(const BatchTensor* descs, size_t L, int in_dtype, size_t H, size_t T, size_t D,
                               size_t Q, bool proj, int exact, cudaStream_t st) {
  if (L == 0) return cudaSuccess;
  const int smem = bt_layout((int)T, (int)D, (int)Q, proj).total;
  if (in_dtype == KVF_IN_F16) return launch_typed<__half>(descs, L, H, T, D, smem, exact, st);
  return launch_typed<float>(descs, L, H, T, D, smem, exact, st);
}

}  // namespace kvf
