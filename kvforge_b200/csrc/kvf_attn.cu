// Fused dequantization + decode attention on the compressed cache.
//
// The reference declares this step but leaves it empty
// (crates/kvforge-cuda/kernels/fused_dequant_attention.cu:1-53,
// KernelLauncher::fused_dequant_attention, kernel_launcher.rs:43-57): one
// query row per head, K and V dequantized from their INT4/INT8 codes (keys
// per channel, values per token, the pipeline's KIVI layout) and, when
// projected, reconstructed through basis_vt; out[h] = softmax(scale * K_h q_h) V_h.
//
// Neither K nor V is rebuilt here. With a basis, K_h = P_k,h B_k,h (B the
// [R, D] basis rows, zero from rank_h on, projection.rs:160-166), so
//   K_h q_h = P_k,h (B_k,h q_h)   and   p^T V_h = (p^T P_v,h) B_v,h :
// the query is taken into the key basis's R coordinates once, scores are
// R-long dot products over the dequantized coefficients, and the value sum
// is accumulated over R coefficients and taken back to D once per head. A
// head reads its codes and per-token parameters only (Llama-3-8B layer at
// R = 3 / 12, INT4: 1.9 MB instead of 268 MB of f32 K and V).
//
// Kernels: k_attn_tile, one CTA per (128-token tile, head), computes the
// tile's score maximum m, sum l of exp(s - m) and the R-vector
// sum_t exp(s_t - m) P_v[t, :]; k_attn_combine merges the tiles of a head
// (flash-decoding style rescaling by exp(m_i - M)) and applies B_v. Each
// coefficient is dequantized as the reference does it (code * scale, then
// + min, each rounded, quantize.rs:165-231); the sums are f32 in a fixed
// order, so results are deterministic and match an fp64 evaluation of the
// same formula to f32 rounding.
#include <cfloat>

#include "kvf_internal.cuh"

namespace kvf {
namespace {

constexpr int kAttnTile = 128;  // tokens per CTA = threads per CTA
constexpr int kAttnWarps = kAttnTile / 32;

template <bool INT4>
__device__ __forceinline__ float code_at_flat(const uint8_t* __restrict__ c, size_t j) {
  if (INT4) {
    const uint32_t b = __ldg(c + (j >> 1));
    return (float)((b >> ((unsigned)(j & 1) << 2)) & 15u);  // even flat index in the low nibble
  }
  return (float)__ldg(c + j);
}

__device__ __forceinline__ float dequant(float code, float s, float m) { return __fadd_rn(__fmul_rn(code, s), m); }

// block-wide reduction over kAttnTile threads; every thread gets the result
template <bool MAX>
__device__ __forceinline__ float block_reduce(float v, float* red) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float w = __shfl_xor_sync(0xffffffffu, v, o);
    v = MAX ? fmaxf(v, w) : v + w;
  }
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  __syncthreads();  // red may still be read from a previous reduction
  if (lane == 0) red[warp] = v;
  __syncthreads();
  float r = red[0];
#pragma unroll
  for (int i = 1; i < kAttnWarps; ++i) r = MAX ? fmaxf(r, red[i]) : r + red[i];
  return r;
}

// dynamic shared memory: qt[Rk] sk[Rk] mk[Rk] | pp[tile] sv[tile] mv[tile] part[tile]
template <bool KI4, bool VI4>
__global__ void __launch_bounds__(kAttnTile) k_attn_tile(
    const uint8_t* __restrict__ kc, const uint8_t* __restrict__ vc, const float* __restrict__ q,
    const float* __restrict__ ks, const float* __restrict__ km, const float* __restrict__ vs,
    const float* __restrict__ vm, const float* __restrict__ kvt, const uint64_t* __restrict__ kranks, size_t T,
    size_t D, size_t Rk, size_t Rv, float scale, float* __restrict__ part) {
  extern __shared__ float sm[];
  float* qt = sm;
  float* sk = qt + Rk;
  float* mk = sk + Rk;
  float* pp = mk + Rk;
  float* svs = pp + kAttnTile;
  float* mvs = svs + kAttnTile;
  float* acc = mvs + kAttnTile;
  __shared__ float red[kAttnWarps];
  const size_t h = blockIdx.y;
  const size_t tile = blockIdx.x;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;

  // the query in the key basis's coordinates (zero from the head's rank on)
  if (kvt) {
    const size_t rank = kranks[h];
    for (size_t r = warp; r < Rk; r += kAttnWarps) {
      float s = 0.f;
      if (r < rank)
        for (size_t c = lane; c < D; c += 32) s = fmaf(__ldg(kvt + (h * Rk + r) * D + c), __ldg(q + h * D + c), s);
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
      if (lane == 0) qt[r] = s;
    }
  } else {
    for (size_t r = tid; r < Rk; r += kAttnTile) qt[r] = __ldg(q + h * D + r);
  }
  for (size_t r = tid; r < Rk; r += kAttnTile) {
    sk[r] = __ldg(ks + h * Rk + r);
    mk[r] = __ldg(km + h * Rk + r);
  }
  __syncthreads();

  // one token per thread: its score over the dequantized key coefficients
  const size_t t0 = tile * kAttnTile;
  const int n = (int)min((size_t)kAttnTile, T - t0);
  float s = -FLT_MAX;
  if (tid < n) {
    const size_t base = (h * T + t0 + tid) * Rk;
    float dot = 0.f;
    for (size_t r = 0; r < Rk; ++r) dot = fmaf(dequant(code_at_flat<KI4>(kc, base + r), sk[r], mk[r]), qt[r], dot);
    s = dot * scale;
  }
  const float m = block_reduce<true>(s, red);
  const float p = tid < n ? expf(s - m) : 0.f;
  const float l = block_reduce<false>(p, red);
  pp[tid] = p;
  svs[tid] = tid < n ? __ldg(vs + h * T + t0 + tid) : 0.f;
  mvs[tid] = tid < n ? __ldg(vm + h * T + t0 + tid) : 0.f;
  __syncthreads();

  // sum_t p_t P_v[t, r]: for Rv < kAttnTile, G thread groups split the tokens
  // of each column, then the groups are added in order
  float* out = part + (h * gridDim.x + tile) * (2 + Rv);
  if (Rv < (size_t)kAttnTile) {
    const int R = (int)Rv, G = kAttnTile / R;
    const int r = tid % R, g = tid / R;
    float a = 0.f;
    if (g < G)
      for (int i = g; i < n; i += G)
        a = fmaf(pp[i], dequant(code_at_flat<VI4>(vc, (h * T + t0 + i) * Rv + r), svs[i], mvs[i]), a);
    acc[tid] = a;
    __syncthreads();
    if (tid < R) {
      float sum = 0.f;
      for (int gg = 0; gg < G; ++gg) sum += acc[gg * R + tid];
      out[2 + tid] = sum;
    }
  } else {
    for (size_t r = tid; r < Rv; r += kAttnTile) {
      float a = 0.f;
      for (int i = 0; i < n; ++i)
        a = fmaf(pp[i], dequant(code_at_flat<VI4>(vc, (h * T + t0 + i) * Rv + r), svs[i], mvs[i]), a);
      out[2 + r] = a;
    }
  }
  if (tid == 0) {
    out[0] = m;
    out[1] = l;
  }
}

// one CTA per head: merge the tiles, normalise, back to D through B_v
__global__ void __launch_bounds__(kAttnTile) k_attn_combine(const float* __restrict__ part, int ntiles,
                                                            const float* __restrict__ vvt,
                                                            const uint64_t* __restrict__ vranks, size_t D,
                                                            size_t Rv, float* __restrict__ out) {
  extern __shared__ float sm[];
  float* w = sm;             // [ntiles] tile weights exp(m_i - M)
  float* accr = w + ntiles;  // [Rv]
  __shared__ float red[kAttnWarps];
  __shared__ float gsum[kAttnTile];
  const size_t h = blockIdx.x;
  const int tid = threadIdx.x;
  const float* ph = part + h * (size_t)ntiles * (2 + Rv);
  float mx = -FLT_MAX;
  for (int i = tid; i < ntiles; i += kAttnTile) mx = fmaxf(mx, ph[(size_t)i * (2 + Rv)]);
  const float M = block_reduce<true>(mx, red);
  float ls = 0.f;
  for (int i = tid; i < ntiles; i += kAttnTile) {
    const float e = expf(ph[(size_t)i * (2 + Rv)] - M);
    w[i] = e;
    ls = fmaf(ph[(size_t)i * (2 + Rv) + 1], e, ls);
  }
  const float L = block_reduce<false>(ls, red);  // ends with a barrier: w[] is visible
  if (Rv < (size_t)kAttnTile) {
    // G thread groups split the tiles of each coefficient; groups added in order
    const int R = (int)Rv, G = kAttnTile / R;
    const int r = tid % R, g = tid / R;
    float a = 0.f;
    if (g < G)
      for (int i = g; i < ntiles; i += G) a = fmaf(ph[(size_t)i * (2 + Rv) + 2 + r], w[i], a);
    gsum[tid] = a;
    __syncthreads();
    if (tid < R) {
      float sum = 0.f;
      for (int gg = 0; gg < G; ++gg) sum += gsum[gg * R + tid];
      accr[tid] = sum / L;
    }
  } else {
    for (size_t r = tid; r < Rv; r += kAttnTile) {
      float a = 0.f;
      for (int i = 0; i < ntiles; ++i) a = fmaf(ph[(size_t)i * (2 + Rv) + 2 + r], w[i], a);
      accr[r] = a / L;
    }
  }
  __syncthreads();
  if (vvt) {
    const size_t rank = vranks[h];
    for (size_t c = tid; c < D; c += kAttnTile) {
      float o = 0.f;
      for (size_t r = 0; r < rank; ++r) o = fmaf(accr[r], __ldg(vvt + (h * Rv + r) * D + c), o);
      out[h * D + c] = o;
    }
  } else {
    for (size_t c = tid; c < D; c += kAttnTile) out[h * D + c] = accr[c];
  }
}

template <bool KI4, bool VI4>
cudaError_t attn_tile_launch(dim3 grid, size_t smem, cudaStream_t st, const uint8_t* kc, const uint8_t* vc,
                             const float* q, const float* ks, const float* km, const float* vs, const float* vm,
                             const float* kvt, const uint64_t* kranks, size_t T, size_t D, size_t Rk, size_t Rv,
                             float scale, float* part) {
  if (smem > kSmemOptIn) {
    cudaError_t e = cudaFuncSetAttribute(k_attn_tile<KI4, VI4>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         (int)smem);
    if (e != cudaSuccess) return e;
  }
  k_attn_tile<KI4, VI4><<<grid, kAttnTile, smem, st>>>(kc, vc, q, ks, km, vs, vm, kvt, kranks, T, D, Rk, Rv, scale,
                                                       part);
  return cudaGetLastError();
}

}  // namespace

size_t attention_tiles(size_t T) { return (T + kAttnTile - 1) / kAttnTile; }

size_t attention_scratch_floats(size_t H, size_t T, size_t Rv) { return H * attention_tiles(T) * (2 + Rv); }

cudaError_t launch_attention(const uint8_t* kc, int kdt, const uint8_t* vc, int vdt, const float* q,
                             const float* ks, const float* km, const float* vs, const float* vm, const float* kvt,
                             const uint64_t* kranks, const float* vvt, const uint64_t* vranks, size_t H, size_t T,
                             size_t D, size_t Rk, size_t Rv, float scale, float* part, float* out,
                             cudaStream_t st) {
  if (H == 0) return cudaSuccess;
  if (T == 0) return cudaMemsetAsync(out, 0, H * D * sizeof(float), st);
  const size_t ntiles = attention_tiles(T);
  const dim3 grid((unsigned)ntiles, (unsigned)H);
  const size_t smem = (3 * Rk + 4 * kAttnTile) * sizeof(float);
  cudaError_t e;
  if (kdt == KVF_INT4 && vdt == KVF_INT4)
    e = attn_tile_launch<true, true>(grid, smem, st, kc, vc, q, ks, km, vs, vm, kvt, kranks, T, D, Rk, Rv, scale, part);
  else if (kdt == KVF_INT4)
    e = attn_tile_launch<true, false>(grid, smem, st, kc, vc, q, ks, km, vs, vm, kvt, kranks, T, D, Rk, Rv, scale,
                                      part);
  else if (vdt == KVF_INT4)
    e = attn_tile_launch<false, true>(grid, smem, st, kc, vc, q, ks, km, vs, vm, kvt, kranks, T, D, Rk, Rv, scale,
                                      part);
  else
    e = attn_tile_launch<false, false>(grid, smem, st, kc, vc, q, ks, km, vs, vm, kvt, kranks, T, D, Rk, Rv, scale,
                                       part);
  if (e != cudaSuccess) return e;
  const size_t csmem = (ntiles + Rv) * sizeof(float);
  if (csmem > kSmemOptIn) {
    e = cudaFuncSetAttribute(k_attn_combine, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)csmem);
    if (e != cudaSuccess) return e;
  }
  k_attn_combine<<<(unsigned)H, kAttnTile, csmem, st>>>(part, (int)ntiles, vvt, vranks, D, Rv, out);
  e = cudaGetLastError();
  if (e == cudaSuccess) note_launches(2);
  return e;
}

}  // namespace kvf
