// Tensor-core reconstruction (sm_100a): X̂[h] = P̂[h] · V[h] on tcgen05 with the
// accumulator in tensor memory.
//
// The reference reconstructs with a scalar multiply-add loop
// (crates/kvforge-cpu/src/projection.rs:142-172); its result is a tolerance
// check (relative Frobenius error, 1e-4 for fp32), not a bit-exact one, so the
// default reconstruction runs here as a GEMM: M = 128 tokens, N = D = 128
// output channels, K = R coefficients (padded to 8 or 16). Each f32 operand is
// split into two tf32 parts (split_tf32); three kind::tf32 passes
// (hi·hi + hi·lo + lo·hi) leave a relative error near 2^-21 per product. The
// separately rounded CPU order stays available bit for bit on the CUDA-core
// kernel (kvf_set_exact_reconstruct).
//
// One CTA of 128 threads (4 warps) per 128-token tile at a time, persistent
// over (head, tile) items, two CTAs per SM:
//   1. each thread dequantizes its token row (q * scale + min, separately
//      rounded as the reference does) and writes the hi/lo parts into the A
//      operands, K-major core matrices without swizzle; the head's basis was
//      written the same way into the B operands when the head started;
//   2. one thread issues the MMAs and commits them to an mbarrier (bounded
//      wait);
//   3. warp w reads TMEM lanes 32w..32w+31 (its tokens) 32 columns at a time
//      (tcgen05.ld 32x32b.x32) into a 128-byte-swizzled staging tile;
//   4. one thread stores the tile with four 3-D tensor-map stores (box 32
//      channels x 128 tokens x 1 head), so a partial last tile never writes
//      into the next head; the stores drain while the next tile is computed.
// No multicast anywhere; the only wait is the bounded MMA-completion wait.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <algorithm>
#include <mutex>

#include "kvf_internal.cuh"

namespace kvf {
namespace {

constexpr int kTcRows = 128;     // tokens per tile: MMA M, TMEM lanes
constexpr int kTcD = 128;        // output channels: MMA N, TMEM columns
constexpr int kTcThreads = 128;
constexpr uint32_t kTcWaitLimit = 1u << 22;
constexpr int kStageBytes = kTcRows * kTcD * 4;  // 64 KB: 4 column blocks of [128 tokens][128 B]

__device__ __forceinline__ uint32_t sa(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }

// byte offset of element (row, k) of a K-major operand made of 8-row x 16-byte
// core matrices, no swizzle: K chunks of one row group are 128 B apart, row
// groups kchunks * 128 B apart
__device__ __forceinline__ uint32_t kmaj(int row, int k, int kchunks) {
  return (uint32_t)((row >> 3) * (kchunks * 128) + (k >> 2) * 128 + (row & 7) * 16 + (k & 3) * 4);
}

// shared-memory matrix descriptor (tcgen05): start address, leading byte
// offset (between the two K core matrices of one MMA), stride byte offset
// (between 8-row groups), descriptor version 1, no swizzle
__device__ __forceinline__ uint64_t sdesc(uint32_t addr, uint32_t lbo, uint32_t sbo) {
  return (uint64_t)((addr & 0x3FFFFu) >> 4) | ((uint64_t)(lbo >> 4) << 16) | ((uint64_t)(sbo >> 4) << 32) |
         ((uint64_t)1 << 46);
}

// instruction descriptor: D f32, A and B tf32, both K-major, M = 128, N = 128
constexpr uint32_t kIdesc =
    (1u << 4) | (2u << 7) | (2u << 10) | ((uint32_t)(kTcD >> 3) << 17) | ((uint32_t)(kTcRows >> 4) << 24);

__device__ __forceinline__ void mma_tf32(uint32_t tmem_d, uint64_t a, uint64_t b, uint32_t accumulate) {
  const uint32_t z = 0;
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, {%5, %6, %7, %8}, p;\n}\n" ::"r"(tmem_d),
      "l"(a), "l"(b), "r"(kIdesc), "r"(accumulate), "r"(z), "r"(z), "r"(z), "r"(z));
}

__device__ __forceinline__ void mbar_init1(uint64_t* bar) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(sa(bar)) : "memory");
}
__device__ __forceinline__ bool mbar_wait1(uint64_t* bar, uint32_t parity) {
  const uint32_t a = sa(bar);
  for (uint32_t i = 0; i < kTcWaitLimit; ++i) {
    uint32_t done;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
        : "=r"(done)
        : "r"(a), "r"(parity)
        : "memory");
    if (done) return true;
  }
  return false;
}

// x as the sum of two tf32 values: hi = x rounded to 11 significant bits, and
// the remainder x - hi (exact in f32, |.| <= 2^-11 |x|) rounded to 11 bits, so
// hi + lo is within 2^-22 |x| of x. Non-finite x is carried by hi alone.
__device__ __forceinline__ void split_tf32(float x, float& hi, float& lo) {
  uint32_t h, l;
  asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(h) : "f"(x));
  hi = __uint_as_float(h);
  const float r = isfinite(x) ? __fsub_rn(x, hi) : 0.0f;
  asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(l) : "f"(r));
  lo = __uint_as_float(l);
}

// this thread's token row of one item, fetched a tile ahead and dequantized
// when the tile is staged
template <int MODE, int KC>
struct RowIn {
  uint32_t q[MODE == 0 ? 1 : KC];  // codes, one byte each
  float raw[MODE == 0 ? 4 * KC : 1];
  float sc, mn;
};

// MODE 0: raw f32 coefficients, 1: INT8 codes, 2: INT4 codes; KC: K in 4-wide chunks (2 or 4)
template <int MODE, int KC>
__global__ void __launch_bounds__(kTcThreads, 2)
    k_reconstruct_tc(const __grid_constant__ CUtensorMap omap, const uint8_t* __restrict__ codes,
                     const float* __restrict__ raw, const float* __restrict__ scales,
                     const float* __restrict__ mins, int axis, int H, int T, int R,
                     const float* __restrict__ bvt, const uint64_t* __restrict__ ranks,
                     unsigned* __restrict__ status) {
  constexpr int K = 4 * KC;
  constexpr int kOpBytes = kTcRows * K * 4;  // one operand part
  extern __shared__ uint8_t sm_raw[];
  // the 128-byte swizzle of the staging tile is taken from address bits 7-9:
  // the tile starts on a 1024-byte boundary
  uint8_t* sm = sm_raw + ((1024u - (sa(sm_raw) & 1023u)) & 1023u);
  uint8_t* stage = sm;  // [4 column blocks][128 tokens][128 B], swizzled
  uint8_t* a_hi = sm + kStageBytes;
  uint8_t* a_lo = a_hi + kOpBytes;
  uint8_t* b_hi = a_lo + kOpBytes;
  uint8_t* b_lo = b_hi + kOpBytes;
  float* pscale = reinterpret_cast<float*>(b_lo + kOpBytes);  // per-channel parameters of the head [K]
  float* pmin = pscale + K;
  uint64_t* mma_bar = reinterpret_cast<uint64_t*>(pmin + K);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(mma_bar + 1);
  const int tid = threadIdx.x, w = tid >> 5, lane = tid & 31;
  const int tiles = (T + kTcRows - 1) / kTcRows;
  const long long items = (long long)H * tiles;
  const long long i0 = items * blockIdx.x / gridDim.x;
  const long long i1 = items * (blockIdx.x + 1) / gridDim.x;

  auto fetch = [&](long long it, RowIn<MODE, KC>& in) {
    const int h = (int)(it / tiles), tile = (int)(it - (long long)h * tiles);
    const int t = tile * kTcRows + tid;
    const bool ok = t < T;
    const size_t g = (size_t)h * T + (ok ? t : 0);
    in.sc = in.mn = 0.0f;
    if (MODE != 0 && axis != KVF_PER_CHANNEL && ok) {
      in.sc = __ldg(scales + g);
      in.mn = __ldg(mins + g);
    }
#pragma unroll
    for (int k = 0; k < K; ++k) {
      const size_t fi = g * R + k;
      if (MODE == 0) {
        in.raw[k] = (ok && k < R) ? __ldg(raw + fi) : 0.0f;
      } else {
        if ((k & 3) == 0) in.q[k >> 2] = 0u;
        if (ok && k < R) {
          uint32_t q = codes[MODE == 2 ? (fi >> 1) : fi];
          if (MODE == 2) q = (fi & 1) ? (q >> 4) & 0xFu : q & 0xFu;
          in.q[k >> 2] |= q << (8 * (k & 3));
        }
      }
    }
  };

  if (w == 0) {  // 128 TMEM columns: the 128 x 128 f32 accumulator
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(sa(tmem_slot)),
                 "r"(kTcD));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::);
  }
  if (tid == 0) {
    mbar_init1(mma_bar);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  const uint32_t tmem = *tmem_slot;

  int cur_h = -1, rank = 0;
  uint32_t phase = 0;
  bool failed = false;
  RowIn<MODE, KC> cur, nxt;
  if (i0 < i1) fetch(i0, cur);
  for (long long it = i0; it < i1; ++it) {
    const int h = (int)(it / tiles), tile = (int)(it - (long long)h * tiles);
    if (h != cur_h) {  // block-uniform: the head's basis as B operands (rows = output channels)
      const uint64_t rk = ranks[h];
      rank = (int)(rk < (uint64_t)R ? rk : (uint64_t)R);
      const float* B = bvt + (size_t)h * R * kTcD;
      for (int i = tid; i < kTcD * K; i += kTcThreads) {
        const int k = i / kTcD, c = i - k * kTcD;  // consecutive threads read consecutive channels
        const float v = (k < rank) ? __ldg(B + (size_t)k * kTcD + c) : 0.0f;
        float hi, lo;
        split_tf32(v, hi, lo);
        *reinterpret_cast<float*>(b_hi + kmaj(c, k, KC)) = hi;
        *reinterpret_cast<float*>(b_lo + kmaj(c, k, KC)) = lo;
      }
      if (MODE != 0 && axis == KVF_PER_CHANNEL)
        for (int k = tid; k < K; k += kTcThreads) {
          pscale[k] = (k < R) ? __ldg(scales + (size_t)h * R + k) : 0.0f;
          pmin[k] = (k < R) ? __ldg(mins + (size_t)h * R + k) : 0.0f;
        }
      cur_h = h;
      __syncthreads();
    }
    {  // this thread's token row into the A operands; terms k >= rank are zero
      const bool ok = tile * kTcRows + tid < T;
#pragma unroll
      for (int kc = 0; kc < KC; ++kc) {
        float hi4[4], lo4[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int k = 4 * kc + e;
          float d = 0.0f;
          if (ok && k < rank) {
            if (MODE == 0) {
              d = cur.raw[k];
            } else {
              const float q = (float)((cur.q[kc] >> (8 * e)) & 0xFFu);
              const float s = (axis == KVF_PER_CHANNEL) ? pscale[k] : cur.sc;
              const float m = (axis == KVF_PER_CHANNEL) ? pmin[k] : cur.mn;
              d = __fadd_rn(__fmul_rn(q, s), m);  // q * scale + min, separately rounded
            }
          }
          split_tf32(d, hi4[e], lo4[e]);
        }
        *reinterpret_cast<float4*>(a_hi + kmaj(tid, 4 * kc, KC)) = make_float4(hi4[0], hi4[1], hi4[2], hi4[3]);
        *reinterpret_cast<float4*>(a_lo + kmaj(tid, 4 * kc, KC)) = make_float4(lo4[0], lo4[1], lo4[2], lo4[3]);
      }
    }
    // the operands are read by the tensor core through the async proxy
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    __syncthreads();
    if (tid == 0) {
      asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
      const uint32_t sbo = KC * 128;
      const uint8_t* as[3] = {a_hi, a_hi, a_lo};
      const uint8_t* bs[3] = {b_hi, b_lo, b_hi};
      uint32_t acc = 0;
#pragma unroll
      for (int p = 0; p < 3; ++p)
#pragma unroll
        for (int ks = 0; ks < KC / 2; ++ks) {  // one MMA covers K = 8: two 16-byte core-matrix columns
          mma_tf32(tmem, sdesc(sa(as[p]) + ks * 256, 128, sbo), sdesc(sa(bs[p]) + ks * 256, 128, sbo), acc);
          acc = 1;
        }
      asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                       sa(mma_bar))
                   : "memory");
    }
    if (it + 1 < i1) fetch(it + 1, nxt);  // loads in flight during the products and the drain
    const bool ok_wait = mbar_wait1(mma_bar, phase);
    phase ^= 1u;
    if (__syncthreads_or(!ok_wait)) {
      failed = true;
      break;
    }
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    // the previous tile's stores have finished reading the staging tile
    if (tid == 0) asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");
    __syncthreads();
#pragma unroll 1
    for (int cb = 0; cb < kTcD / 32; ++cb) {  // 32 channels per TMEM load
      uint32_t v[32];
      const uint32_t taddr = tmem + ((uint32_t)(32 * w) << 16) + (uint32_t)(32 * cb);
      asm volatile(
          "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, "
          "%14, %15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
          : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]),
            "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15]),
            "=r"(v[16]), "=r"(v[17]), "=r"(v[18]), "=r"(v[19]), "=r"(v[20]), "=r"(v[21]), "=r"(v[22]),
            "=r"(v[23]), "=r"(v[24]), "=r"(v[25]), "=r"(v[26]), "=r"(v[27]), "=r"(v[28]), "=r"(v[29]),
            "=r"(v[30]), "=r"(v[31])
          : "r"(taddr));
      asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
      // token row 32w + lane of column block cb; 16-byte chunk j lands at j ^ (row mod 8)
      const int row = 32 * w + lane;
      uint8_t* rowp = stage + cb * (kTcRows * 128) + row * 128;
#pragma unroll
      for (int j = 0; j < 8; ++j)
        *reinterpret_cast<uint4*>(rowp + ((j ^ (row & 7)) << 4)) =
            make_uint4(v[4 * j], v[4 * j + 1], v[4 * j + 2], v[4 * j + 3]);
    }
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    __syncthreads();
    if (tid == 0) {
#pragma unroll
      for (int cb = 0; cb < kTcD / 32; ++cb)
        asm volatile(
            "cp.async.bulk.tensor.3d.global.shared::cta.bulk_group [%0, {%2, %3, %4}], [%1];" ::"l"(&omap),
            "r"(sa(stage + cb * (kTcRows * 128))), "r"(32 * cb), "r"(tile * kTcRows), "r"(h)
            : "memory");
      asm volatile("cp.async.bulk.commit_group;" ::: "memory");
    }
    cur = nxt;
  }
  if (tid == 0) asm volatile("cp.async.bulk.wait_group 0;" ::: "memory");
  if (failed && tid == 0 && status) atomicOr(status, kDevErrTimeout);
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  if (w == 0) asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTcD));
}

// [H, T, D] f32 output, box 32 channels x 128 tokens x 1 head, 128-byte swizzle
bool encode_out_map(CUtensorMap* map, float* out, size_t H, size_t T) {
  auto enc = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(tensor_map_encode_fn());
  if (!enc) return false;
  const cuuint64_t gdim[3] = {(cuuint64_t)kTcD, (cuuint64_t)T, (cuuint64_t)H};
  const cuuint64_t gstride[2] = {(cuuint64_t)kTcD * 4, (cuuint64_t)T * kTcD * 4};
  const cuuint32_t box[3] = {32, (cuuint32_t)kTcRows, 1};
  const cuuint32_t estride[3] = {1, 1, 1};
  return enc(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, out, gdim, gstride, box, estride, CU_TENSOR_MAP_INTERLEAVE_NONE,
             CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_NONE,
             CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

template <int MODE, int KC>
cudaError_t launch_tc(const CUtensorMap& map, const uint8_t* codes, const float* raw, const float* scales,
                      const float* mins, int axis, size_t H, size_t T, size_t R, const float* bvt,
                      const uint64_t* ranks, unsigned* status, cudaStream_t st) {
  auto kern = k_reconstruct_tc<MODE, KC>;
  const size_t smem = 1024 + kStageBytes + 4 * (size_t)kTcRows * (4 * KC) * 4 + 2 * (4 * KC) * 4 + 64;
  constexpr int kDevs = 64;
  static int sms[kDevs] = {};
  static bool attr[kDevs] = {};
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 0 || dev >= kDevs) return cudaErrorInvalidDevice;
  if (!attr[dev]) {
    if ((e = cudaDeviceGetAttribute(&sms[dev], cudaDevAttrMultiProcessorCount, dev)) != cudaSuccess) return e;
    if ((e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem)) != cudaSuccess)
      return e;
    attr[dev] = true;
  }
  const size_t items = H * ((T + kTcRows - 1) / kTcRows);
  const unsigned grid = (unsigned)std::max<size_t>(1, std::min<size_t>(items, (size_t)sms[dev] * 2));
  kern<<<grid, kTcThreads, smem, st>>>(map, codes, raw, scales, mins, axis, (int)H, (int)T, (int)R, bvt, ranks,
                                       status);
  note_launches(1);
  return cudaGetLastError();
}

}  // namespace

cudaError_t launch_reconstruct_tc(const uint8_t* codes, const float* raw, const float* scales, const float* mins,
                                  int data_type, int axis, size_t H, size_t T, size_t R, size_t D,
                                  const float* basis_vt, const uint64_t* ranks, float* out, unsigned* status,
                                  cudaStream_t st) {
  if (D != (size_t)kTcD || R == 0 || R > 16 || !aligned(out, 16) || H * T == 0 || T >= (1u << 31) ||
      H >= (1u << 31))
    return cudaErrorNotSupported;
  CUtensorMap map{};
  if (!encode_out_map(&map, out, H, T)) return cudaErrorNotSupported;
  const int mode = raw ? 0 : (data_type == KVF_INT8 ? 1 : 2);
#define KVF_TC(M)                                                                                           \
  return (R <= 8) ? launch_tc<M, 2>(map, codes, raw, scales, mins, axis, H, T, R, basis_vt, ranks, status, st) \
                  : launch_tc<M, 4>(map, codes, raw, scales, mins, axis, H, T, R, basis_vt, ranks, status, st)
  if (mode == 0) { KVF_TC(0); }
  if (mode == 1) { KVF_TC(1); }
  KVF_TC(2);
#undef KVF_TC
}

}  // namespace kvf
