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
constexpr int kBtCh = 16;  // coefficients per thread in the projection (four r-blocks of 16)
constexpr size_t kBatchSmallCap = 16, kBatchCap = 128;  // layers per launch
constexpr int kBtLoads = 8;  // global loads in flight per thread while staging

struct BtLayout {  // byte offsets into dynamic shared memory
  int xs, vt, pp, cb, par, hist, total;
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
  off += T * L.xstride * 4;
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
  L.total = off;
  return L;
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
  // 1. rows and basis into shared memory, eight loads in flight per thread
  const int d4 = D >> 2;
  for (int i0 = tid; i0 < T * d4; i0 += kBtLoads * kBtThreads) {
    float4 v[kBtLoads];
#pragma unroll
    for (int j = 0; j < kBtLoads; ++j) {
      const int i = i0 + j * kBtThreads;
      const int t = i / d4, c4 = i - t * d4;
      if (i < T * d4) v[j] = ldx4<TIn>(x + (size_t)t * D + 4 * c4);
    }
#pragma unroll
    for (int j = 0; j < kBtLoads; ++j) {
      const int i = i0 + j * kBtThreads;
      const int t = i / d4, c4 = i - t * d4;
      if (i < T * d4) {
        float* dst = xs + t * L.xstride + 4 * c4;
        dst[0] = v[j].x;
        dst[1] = v[j].y;
        dst[2] = v[j].z;
        dst[3] = v[j].w;
      }
    }
  }
  if (proj) {  // vT[c][r]: r-blocks of 16 contiguous per column; rows from the rank on are zero
    const float* B = d.bvt + (size_t)h * Q * D;
    const int nrow = rank;  // rank <= Q: rows from the rank on are not read
    for (int i0 = tid; i0 < kBtMaxR * D; i0 += kBtLoads * kBtThreads) {
      float v[kBtLoads];
#pragma unroll
      for (int j = 0; j < kBtLoads; ++j) {
        const int i = i0 + j * kBtThreads;
        v[j] = (i < nrow * D) ? __ldg(B + i) : 0.0f;  // B + r * D + c
      }
#pragma unroll
      for (int j = 0; j < kBtLoads; ++j) {
        const int i = i0 + j * kBtThreads;
        const int r = i / D, c = i - r * D;
        if (i < kBtMaxR * D) vT[c * L.vstride + r] = v[j];
      }
    }
  }
  if (d.hist)
    for (int i = tid; i < 256; i += kBtThreads) shist[i] = 0u;
  __syncthreads();

  // 2. projection: thread = (row t, r-block g); the chains of one thread
  // advance together, each over c in order
  if (proj) {
    const int groups = (Q + kBtCh - 1) / kBtCh;  // 1..4
    for (int job = tid; job < T * groups; job += kBtThreads) {
      const int t = job / groups, g = job - t * groups;
      float acc[kBtCh];
#pragma unroll
      for (int k = 0; k < kBtCh; ++k) acc[k] = 0.0f;
      const float* xr = xs + t * L.xstride;
      const float* vb = vT + g * kBtCh;
#pragma unroll 4
      for (int c = 0; c < D; ++c) {
        const float xv = xr[c];
        const float4* v4 = reinterpret_cast<const float4*>(vb + c * L.vstride);
#pragma unroll
        for (int k4 = 0; k4 < kBtCh / 4; ++k4) {
          const float4 v = v4[k4];
          acc[4 * k4] = __fmaf_rn(xv, v.x, acc[4 * k4]);
          acc[4 * k4 + 1] = __fmaf_rn(xv, v.y, acc[4 * k4 + 1]);
          acc[4 * k4 + 2] = __fmaf_rn(xv, v.z, acc[4 * k4 + 2]);
          acc[4 * k4 + 3] = __fmaf_rn(xv, v.w, acc[4 * k4 + 3]);
        }
      }
#pragma unroll
      for (int k = 0; k < kBtCh; ++k) {
        const int r = g * kBtCh + k;
        if (r < Q) P[t * pstride + r] = (r < rank) ? acc[k] : 0.0f;  // projection.rs:96
      }
    }
    __syncthreads();
  }

  // 3. quantization
  const float levels = d.levels;
  const int w = tid >> 5, lane = tid & 31;
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
      // dT[r][t] = q * scale + min; rows from T to tstride are zero
      float* dT = P;
      const int ts = L.tstride;
      for (int i = tid; i < rank * ts; i += kBtThreads) {
        const int r = i / ts, t = i - r * ts;
        float v = 0.0f;
        if (t < T) {
          const float sc = (d.axis == KVF_PER_TOKEN) ? psc[t] : psc[r];
          const float mn = (d.axis == KVF_PER_TOKEN) ? pmn[t] : pmn[r];
          v = dq(cb[t * Q + r], sc, mn);
        }
        dT[i] = v;
      }
      __syncthreads();
      // thread = (channel c, half of the rows in blocks of 16): one basis
      // column, four broadcast 16-byte loads of coefficients per r
      const int th = (((T + 1) / 2) + 15) & ~15;
      for (int job = tid; job < D * 2; job += kBtThreads) {
        const int c = job >> 1, half = job & 1;
        const int ta = half ? th : 0, tb = half ? T : (th < T ? th : T);
        for (int t0 = ta; t0 < tb; t0 += 16) {
          float acc[16];
#pragma unroll
          for (int k = 0; k < 16; ++k) acc[k] = 0.0f;
#pragma unroll 2
          for (int r = 0; r < rank; ++r) {
            const float v = vT[c * L.vstride + r];
            const float4* p4 = reinterpret_cast<const float4*>(dT + r * ts + t0);
#pragma unroll
            for (int k4 = 0; k4 < 4; ++k4) {
              const float4 p = p4[k4];
              const float pv[4] = {p.x, p.y, p.z, p.w};
#pragma unroll
              for (int j = 0; j < 4; ++j) {
                float& a = acc[4 * k4 + j];
                a = exact ? __fadd_rn(a, __fmul_rn(pv[j], v)) : __fmaf_rn(pv[j], v, a);
              }
            }
          }
#pragma unroll
          for (int k = 0; k < 16; ++k)
            if (t0 + k < tb) __stcs(out + (size_t)(t0 + k) * D + c, acc[k]);
        }
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
