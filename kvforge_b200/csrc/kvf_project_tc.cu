// Tensor-core projection with exact codes (sm_100a).
//
// The projected coefficient is defined as in the CUDA-core kernel and the CPU
// oracle: P[h,t,r] = one fmaf chain over c = 0..127 of x[h,t,c] * vt[h,r,c],
// from +0.0 (crates/kvforge-cpu/src/projection.rs:61-140 forms the same
// quantity as U_k S_k). That chain is a fixed sequence of roundings, which a
// tensor-core MMA (unspecified internal order) does not reproduce. This kernel
// still gives the chain's codes, scales and mins bit for bit:
//
//  1. tcgen05 computes an approximation Q of every coefficient. A = the f16
//     token tile as the TMA loaded it (no conversion), B = the basis split into
//     two f16 parts, hi = f16(v) and lo = f16((v - hi) * 2^11), stacked along
//     N; Q = acc_hi + acc_lo * 2^-11. Accumulators live in TMEM.
//  2. Each token row gets a rigorous bound |P - Q| <= Delta_r =
//     ||x||_2 * b_r + 2^-22 |Q| with, per basis row r,
//        b_r = 2^-13 (||hi_r|| + 2^-11 ||lo_r||)   tensor-core accumulation,
//            + ||v_r - (hi_r + 2^-11 lo_r)||        basis split,
//            + 2^-16 ||v_r||                        the chain's own rounding
//     (products of f16 values are exact in f32; 2^-13 is 8x a generous bound
//     of a truncating f32 accumulation, 2^-23 per term of 8 K=16 steps of 16
//     products, and the chain's error is at
//     most 128 u sum |x v| <= 2^-17 ||x|| ||v||, Cauchy-Schwarz).
//  3. Per-token quantization (crates/kvforge-cpu/src/quantize.rs:102-130):
//     the coefficients with the smallest and largest Q are recomputed with
//     the exact chain on CUDA cores (two chains in one pass over the row,
//     which also sums the row's squares for ||x||), and they are the row's
//     exact minimum and maximum unless another coefficient's interval
//     [Q - Delta, Q + Delta] reaches past them. A code is the same for every
//     value in the interval unless it holds a rounding boundary of the code
//     (the code is monotone in the value).
//  4. Rows where either test fails (a near tie for the minimum or maximum, a
//     code near a rounding boundary: a few percent of rows), rows with
//     non-finite inputs, and heads whose basis does not split into finite f16
//     parts are deferred: after its last tile the CTA recomputes every
//     coefficient of those rows exactly (x and basis from global memory) and
//     quantizes them as the oracle does.
// One persistent CTA per SM walks (head, 128-token tile) items with warp roles:
//   warp 0: TMA producer, two 2-D tensor-map loads per tile (64 channels x 128
//           rows each, 128-byte swizzle) into a ring of 5 stages (4 above 16
//           coefficients; no multicast);
//   warp 1: TMEM allocation; converts each new head's basis into a B-operand
//           slot (two slots up to 32 coefficients, one at 64; a slot is reused
//           once every tile of its previous head is done; the f32 rows arrive
//           by bulk copy); lane 0 issues 8 MMAs (K = 16 each) per tile into
//           one of 6 accumulators (4 above 32 coefficients) and commits them
//           to an mbarrier;
//   warps 2-13: three epilogue groups of four warps, taking tiles in turn; a
//           thread owns one token row (its TMEM lane), reads its
//           coefficients, its x row from the stage (norm and exact chains)
//           and writes the quantized row or defers it. The stage is released
//           after the epilogue; the deferred rows are finished by all
//           epilogue threads at the end.
// EXACT = false (KVF_PROJ_TENSOR_CORE_APPROX) skips steps 2-4: the row's
// minimum, maximum and codes come from Q itself, and the stage is released as
// soon as the tile's MMAs complete.
// Every wait is bounded; a wait that runs out raises an abort flag that ends
// every role, and KVF_ERR_DEVICE_TIMEOUT in the status word.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <algorithm>
#include <atomic>

#include "kvf_internal.cuh"

namespace kvf {
namespace {

constexpr int kRows = 128;                       // tokens per tile: MMA M, TMEM lanes
constexpr int kD = 128;                          // head_dim: MMA K
constexpr int kTileBytes = kRows * kD * 2;       // one f16 tile
constexpr int kRegionBytes = kTileBytes / 2;     // 64 channels x 128 rows (one 128-byte swizzle span)
// per coefficient width: epilogue groups of four warps (alternating tiles),
// token-tile stages and TMEM accumulator slots, sized to the shared memory
// and the 512 TMEM columns
template <int RG>
struct PtCfg {
  static constexpr int kGroups = 3;
  static constexpr int kStages = RG <= 16 ? 5 : 4;
  static constexpr int kAcc = RG <= 32 ? 6 : 4;
  static constexpr int kEpiWarps = 4 * kGroups;
  static constexpr int kThreads = 32 * (2 + kEpiWarps);
};
constexpr float kLoScale = 2048.0f;              // lo = f16((v - hi) * 2^11)
constexpr float kLoInv = 1.0f / 2048.0f;
constexpr float kTcRelF = 1.0f / 8192.0f;        // bound of the MMA's accumulation error / sum |products|
constexpr float kChainRelF = 1.0f / 65536.0f;    // bound of the fmaf chain's error / (||x|| ||v||)
constexpr int kBStride = kD + 4;                 // floats per basis row in shared memory (rows 4 banks apart)
constexpr int kDefCap = 2048;                    // deferred rows a CTA keeps for its final pass

// basis slots (B operand + f32 rows + bounds) per head in flight: two up to 32
// coefficients, one at 64, where two would not fit in shared memory
template <int RG>
constexpr int pt_slots() {
  return RG <= 32 ? 2 : 1;
}

struct PtInfo {   // per basis slot
  float bn[64];   // b_r (see above), 0 for r >= rank
  int rank;
  int exact_only;
  int expected;   // epilogue warp arrivals that end the slot's head (4 per tile)
  int pad;
};

struct PtLayout {  // byte offsets from the 1024-aligned base
  int xs, bop, bf, info, bars, dlist, hist, total;
};

__device__ __forceinline__ uint32_t sa(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(sa(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(sa(bar)) : "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(sa(bar)), "r"(bytes) : "memory");
}
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, volatile int* abort_flag) {
  return mbar_wait_bounded(sa(bar), parity, kWaitNs, abort_flag);
}
__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, int x, int y, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
          sa(dst)),
      "l"(map), "r"(x), "r"(y), "r"(sa(bar))
      : "memory");
}

// shared-memory matrix descriptor: K-major, 128-byte swizzle (8 rows x 128 B
// atoms, 1024 B apart), descriptor version 1; the start address may step by
// 32 B inside an atom to select the K = 16 slice
__device__ __forceinline__ uint64_t sdesc_sw128(uint32_t addr) {
  return (uint64_t)((addr & 0x3FFFFu) >> 4) | ((uint64_t)1 << 16) | ((uint64_t)(1024 >> 4) << 32) |
         ((uint64_t)1 << 46) | ((uint64_t)2 << 61);
}
// instruction descriptor: D f32, A and B f16, both K-major, M = 128, N
template <int N>
constexpr uint32_t idesc_f16() {
  return (1u << 4) | ((uint32_t)(N >> 3) << 17) | ((uint32_t)(kRows >> 4) << 24);
}
template <int N>
__device__ __forceinline__ void mma_f16(uint32_t tmem_d, uint64_t a, uint64_t b, uint32_t accumulate) {
  const uint32_t z = 0;
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, {%5, %6, %7, %8}, p;\n}\n" ::"r"(tmem_d),
      "l"(a), "l"(b), "r"(idesc_f16<N>()), "r"(accumulate), "r"(z), "r"(z), "r"(z), "r"(z));
}

__device__ __forceinline__ void tmem_ld8(uint32_t taddr, uint32_t* v) {
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0, %1, %2, %3, %4, %5, %6, %7}, [%8];"
               : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7])
               : "r"(taddr));
}
__device__ __forceinline__ void unpack_h8(const uint4& u, float* o) {
  const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&w[k]));
    o[2 * k] = f.x;
    o[2 * k + 1] = f.y;
  }
}
// 16-byte chunk j (8 channels, 0..15) of the thread's row in a stage
__device__ __forceinline__ uint4 x_chunk(const uint8_t* xrow, int swz, int j) {
  return *reinterpret_cast<const uint4*>(xrow + (j >> 3) * kRegionBytes + (((j & 7) ^ swz) << 4));
}

// One exact coefficient is an fmaf chain over c = 0..127 from +0.0, in the
// oracle's order. Two chains advance together (independent scalar fmaf
// sequences sharing the row's x). exact2_norm: the thread's own row from the
// stage (basis rows in shared memory), plus the row's sum of squares;
// exact2_glb: a row and basis rows in global memory.
__device__ __noinline__ float3 exact2_norm(const uint8_t* x, int sw, const float* va, const float* vb) {
  float pa = 0.0f, pb = 0.0f;
  unsigned long long ss2 = 0ull;
#pragma unroll 2
  for (int j = 0; j < 16; ++j) {
    const uint4 u = x_chunk(x, sw, j);
    const uint32_t wv[4] = {u.x, u.y, u.z, u.w};
    float xv[8];
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&wv[k]));
      unsigned long long F;
      asm("mov.b64 %0, {%1, %2};" : "=l"(F) : "f"(f.x), "f"(f.y));
      asm("fma.rn.f32x2 %0, %1, %1, %0;" : "+l"(ss2) : "l"(F));
      xv[2 * k] = f.x;
      xv[2 * k + 1] = f.y;
    }
    const float4 a0 = *reinterpret_cast<const float4*>(va + 8 * j);
    const float4 a1 = *reinterpret_cast<const float4*>(va + 8 * j + 4);
    const float4 b0 = *reinterpret_cast<const float4*>(vb + 8 * j);
    const float4 b1 = *reinterpret_cast<const float4*>(vb + 8 * j + 4);
    const float av[8] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w};
    const float bv[8] = {b0.x, b0.y, b0.z, b0.w, b1.x, b1.y, b1.z, b1.w};
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      pa = __fmaf_rn(xv[k], av[k], pa);
      pb = __fmaf_rn(xv[k], bv[k], pb);
    }
  }
  float s0, s1;
  asm("mov.b64 {%0, %1}, %2;" : "=f"(s0), "=f"(s1) : "l"(ss2));
  return make_float3(pa, pb, __fadd_ru(s0, s1));
}
__device__ __noinline__ float2 exact2_glb(const __half* __restrict__ x, const float* __restrict__ va,
                                          const float* __restrict__ vb) {
  float pa = 0.0f, pb = 0.0f;
#pragma unroll 4
  for (int j = 0; j < 16; ++j) {
    float xv[8];
    unpack_h8(__ldg(reinterpret_cast<const uint4*>(x) + j), xv);
    const float4 a0 = __ldg(reinterpret_cast<const float4*>(va + 8 * j));
    const float4 a1 = __ldg(reinterpret_cast<const float4*>(va + 8 * j + 4));
    const float4 b0 = __ldg(reinterpret_cast<const float4*>(vb + 8 * j));
    const float4 b1 = __ldg(reinterpret_cast<const float4*>(vb + 8 * j + 4));
    const float av[8] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w};
    const float bv[8] = {b0.x, b0.y, b0.z, b0.w, b1.x, b1.y, b1.z, b1.w};
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      pa = __fmaf_rn(xv[k], av[k], pa);
      pb = __fmaf_rn(xv[k], bv[k], pb);
    }
  }
  return make_float2(pa, pb);
}

// replaces coefficient `r` (a run-time index) of the register array: one
// predicated select per element, written out so that the array stays in
// registers (a compare-and-assign loop compiles to an indexed access)
template <int RG>
__device__ __forceinline__ void set_at(float* P, int r, float v) {
#pragma unroll
  for (int k = 0; k < RG; ++k)
    asm("{\n .reg .pred p;\n setp.eq.s32 p, %1, %2;\n selp.f32 %0, %3, %0, p;\n}" : "+f"(P[k]) : "r"(r), "r"(k), "f"(v));
}

// one quantized row out: scale and min, then the codes (INT4 bytes packed
// within the row, R even; or one byte per code), counted in the histogram
struct RowOut {  // where quantized rows go (the ProjectOut fields the epilogue writes)
  float* scales;
  float* mins;
  uint8_t* packed;
  uint8_t* codes;
  float levels;
};

template <int RG>
__device__ __forceinline__ void write_row(const uint32_t* cd, size_t grow, int R, float scale, float mn,
                                          const RowOut& o, uint32_t* shist, bool hist_on) {
  o.scales[grow] = scale;
  o.mins[grow] = mn;
  if (o.packed) {
    uint8_t* dp = o.packed + (grow * R) / 2;
#pragma unroll
    for (int k = 0; k < RG / 2; ++k)
      if (2 * k < R) {
        const uint32_t byte = (cd[2 * k] & 0xFu) | ((cd[2 * k + 1] & 0xFu) << 4);
        dp[k] = (uint8_t)byte;
        if (hist_on) atomicAdd(&shist[byte], 1u);
      }
  } else {
    uint8_t* dc = o.codes + grow * R;
#pragma unroll
    for (int r = 0; r < RG; ++r)
      if (r < R) {
        dc[r] = (uint8_t)cd[r];
        if (hist_on) atomicAdd(&shist[cd[r]], 1u);
      }
  }
}

// A deferred row: every coefficient by the exact chain (x and basis from
// global memory), then the oracle's per-token quantization.
template <int RG>
__device__ __noinline__ void finish_row(const __half* __restrict__ x, size_t grow, int T, int R,
                                        const float* __restrict__ bvt, const uint64_t* __restrict__ ranks,
                                        float* scales, float* mins, uint8_t* packed, uint8_t* codes, float levels,
                                        uint32_t* shist, bool hist_on) {
  const RowOut o{scales, mins, packed, codes, levels};
  const int h = (int)(grow / (size_t)T);
  const uint64_t rk = ranks[h];
  const int rank = (int)(rk < (uint64_t)R ? rk : (uint64_t)R);
  const __half* xr = x + grow * kD;
  const float* B = bvt + (size_t)h * R * kD;
  float P[RG];
#pragma unroll
  for (int r = 0; r < RG; ++r) P[r] = 0.0f;
  for (int r = 0; r < rank; r += 2) {
    const int r2 = (r + 1 < rank) ? r + 1 : r;
    const float2 e = exact2_glb(xr, B + (size_t)r * kD, B + (size_t)r2 * kD);
    set_at<RG>(P, r, e.x);
    set_at<RG>(P, r2, e.y);
  }
  float mn = INFINITY, mx = -INFINITY;
#pragma unroll
  for (int r = 0; r < RG; ++r)
    if (r < R) mm_update(P[r], mn, mx);
  const float scale = make_scale(mn, mx, o.levels);
  const float inv = __frcp_rn(scale);
  uint32_t cd[RG];
#pragma unroll
  for (int r = 0; r < RG; ++r) cd[r] = (r < R) ? qcode_fast(P[r], mn, scale, inv, o.levels) : 0u;
  write_row<RG>(cd, grow, R, scale, mn, o, shist, hist_on);
}

// head h's R f32 basis rows (512 B each) into a slot's rows of kBStride
// floats, by bulk copies that complete on `bar` (whose expected bytes the
// caller has raised); one thread
__device__ __forceinline__ void copy_basis_rows(float* slot, int h, int R, const float* __restrict__ bvt,
                                                uint64_t* bar) {
  for (int r = 0; r < R; ++r)
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                     sa(slot + r * kBStride)),
                 "l"(bvt + ((size_t)h * R + r) * kD), "r"(kD * 4), "r"(sa(bar))
                 : "memory");
}

// EXACT = false: the approximate engine. Codes come straight from the
// tensor-core coefficients (no exact chains, no deferred rows), and the token
// stage goes back to the TMA producer when its MMAs complete.
template <int RG, bool EXACT>
__global__ void __launch_bounds__(PtCfg<RG>::kThreads, 1)
    k_project_tc(const __grid_constant__ CUtensorMap xmap, const __half* __restrict__ x, int H, int T,
                 const float* __restrict__ bvt, const uint64_t* __restrict__ ranks, int R, PtLayout L, ProjectOut o) {
  constexpr int kStages = PtCfg<RG>::kStages, kAcc = PtCfg<RG>::kAcc, kGroups = PtCfg<RG>::kGroups;
  constexpr int kEpiWarps = PtCfg<RG>::kEpiWarps;
  constexpr int N = 2 * RG;                 // MMA N: RG hi columns, then RG lo columns
  constexpr int kSlotBytes = 2 * N * 128;   // two K regions of N rows x 128 B
  constexpr uint32_t kTmemCols = (kAcc * N <= 32) ? 32 : (kAcc * N <= 64) ? 64 : (kAcc * N <= 128) ? 128
                                 : (kAcc * N <= 256) ? 256 : 512;
  extern __shared__ uint8_t smraw[];
  uint8_t* sm = smraw + ((1024u - (sa(smraw) & 1023u)) & 1023u);
  uint8_t* xs = sm + L.xs;
  constexpr int kSlots = pt_slots<RG>();
  uint8_t* bop = sm + L.bop;
  float* bf = reinterpret_cast<float*>(sm + L.bf);  // [slot][RG][kBStride] f32 basis rows (exact chains)
  PtInfo* info = reinterpret_cast<PtInfo*>(sm + L.info);
  uint64_t* x_full = reinterpret_cast<uint64_t*>(sm + L.bars);
  uint64_t* x_empty = x_full + kStages;
  uint64_t* acc_full = x_empty + kStages;
  uint64_t* acc_empty = acc_full + kAcc;
  uint64_t* bfull = acc_empty + kAcc;       // [2]: the slot's basis is converted
  uint64_t& bcopy = bfull[2];               // the bulk copies of a head's f32 basis rows landed
  int* done = reinterpret_cast<int*>(bfull + 3);  // [2]: epilogue warp arrivals for the slot's head
  volatile int* abort_flag = done + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(done + 4);
  uint32_t* shist = reinterpret_cast<uint32_t*>(sm + L.hist);
  uint32_t* dlist = reinterpret_cast<uint32_t*>(sm + L.dlist);  // deferred rows (global row index)
  int* dcount = done + 3;

  const int tid = threadIdx.x, w = tid >> 5, lane = tid & 31;
  const int tiles = (T + kRows - 1) / kRows;
  const long long items = (long long)H * tiles;
  const long long i0 = items * blockIdx.x / gridDim.x;
  const long long i1 = items * (blockIdx.x + 1) / gridDim.x;
  const int nit = (int)(i1 - i0);
  const int h_first = nit > 0 ? (int)(i0 / tiles) : 0;
  // the range reaches a second head whose basis can be copied at set-up
  const bool two_pre = kSlots > 1 && nit > 0 && (int)((i1 - 1) / tiles) > h_first;
  // token tile n of this block's range into stage n % kStages (one thread)
  auto issue_tile = [&](int n) {
    const int s = n % kStages;
    const long long it = i0 + n;
    const int h = (int)(it / tiles), tile = (int)(it - (long long)h * tiles);
    const int row0 = h * T + tile * kRows;
    uint8_t* dst = xs + (size_t)s * kTileBytes;
    mbar_expect_tx(&x_full[s], (uint32_t)kTileBytes);
    tma_load_2d(dst, &xmap, 0, row0, &x_full[s]);
    tma_load_2d(dst + kRegionBytes, &xmap, 64, row0, &x_full[s]);
  };
  const bool hist_on = o.hist != nullptr;

  if (w == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(sa(tmem_slot)),
                 "r"(kTmemCols));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::);
  }
  if (tid == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&x_full[s], 1);
      mbar_init(&x_empty[s], EXACT ? 4 : 1);
    }
    for (int a = 0; a < kAcc; ++a) {
      mbar_init(&acc_full[a], 1);
      mbar_init(&acc_empty[a], 4);
    }
    mbar_init(&bfull[0], 1);
    mbar_init(&bfull[1], 1);
    mbar_init(&bcopy, 1);
    done[0] = done[1] = 0;
    *abort_flag = 0;
    *dcount = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    // the basis rows of the first head (and of the second, when the tile
    // range reaches it and a second slot exists) are requested before any
    // token tile: behind every SM's first stages (about 24 MB) they would
    // land several microseconds later, and no MMA can start before its basis
    // is converted (requesting the first tiles here too measured slower)
    if (nit > 0) {
      mbar_expect_tx(&bcopy, (uint32_t)((two_pre ? 2 : 1) * R * kD * 4));
      copy_basis_rows(bf, h_first, R, bvt, &bcopy);
      if (two_pre) copy_basis_rows(bf + RG * kBStride, h_first + 1, R, bvt, &bcopy);
    }
  }
  if (hist_on)
    for (int i = tid; i < 256; i += blockDim.x) shist[i] = 0u;
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  const uint32_t tmem = *tmem_slot;
  bool timed_out = false;

  if (w == 0) {
    // ---------------- TMA producer ----------------
    int issued = 0;
    if (lane == 0) {
      for (int n = 0; n < nit; ++n) {
        const int s = n % kStages;
        if (n >= kStages && !mbar_wait(&x_empty[s], (uint32_t)((n / kStages - 1) & 1), abort_flag)) {
          timed_out = true;
          break;
        }
        issue_tile(n);
        issued = n + 1;
      }
      // copies still in flight land before the block's shared memory is released
      if (timed_out || *abort_flag)
        for (int n = std::max(0, issued - kStages); n < issued; ++n)
          mbar_wait_bounded(sa(&x_full[n % kStages]), (uint32_t)((n / kStages) & 1), kWaitNs);
    }
    __syncwarp();
  } else if (w == 1) {
    // ---------------- basis conversion + MMA issue ----------------
    int cur_h = -1, hs = -1, last_acc = -1, nconv = 0;
    for (int n = 0; n < nit && !timed_out; ++n) {
      const long long it = i0 + n;
      const int h = (int)(it / tiles);
      if (h != cur_h) {
        ++hs;
        const int b = hs % kSlots;
        if (hs >= kSlots) {  // every tile of the slot's previous head is done (bounded wait)
          bool ok = true;
          if (lane == 0) {
            const unsigned long long t0 = dev_ns();
            uint32_t polls = 0;
            while (*reinterpret_cast<volatile int*>(&done[b]) < info[b].expected) {
              if (*abort_flag || ++polls > kWaitPolls || dev_ns() - t0 > kWaitNs) {
                ok = false;
                break;
              }
              __nanosleep(64);
            }
          }
          __threadfence_block();
          if (!__shfl_sync(0xffffffffu, (int)ok, 0)) {
            timed_out = true;
            break;
          }
        }
        // head h's basis into slot b. The R f32 rows arrive by bulk copies
        // (512 B each) into the slot's exact-chain copy; then lane l writes
        // channels 4l .. 4l + 3 of every row as f16 parts, hi rows 0..RG-1 and
        // lo rows RG..2RG-1, in two 128-byte swizzled regions (region l / 16,
        // 16-byte chunk (l % 16) / 2); finally (exact engine) 8 lanes per row
        // compute the bound b_r in f32, every rounding upward.
        float* bfs = bf + (size_t)b * RG * kBStride;
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");  // earlier reads of the slot, then the copies
        // the rows of the first head, and of the second with two_pre, were
        // requested at set-up (one barrier phase for both)
        const bool copied = hs == 0 || (hs == 1 && two_pre);
        if (lane == 0 && !copied) {
          mbar_expect_tx(&bcopy, (uint32_t)(R * kD * 4));
          copy_basis_rows(bfs, h, R, bvt, &bcopy);
        }
        const uint64_t rk = ranks[h];
        const int rank = (int)(rk < (uint64_t)R ? rk : (uint64_t)R);
        bool okc = true;
        if (!(hs == 1 && two_pre)) {
          okc = mbar_wait(&bcopy, (uint32_t)(nconv & 1), abort_flag);
          ++nconv;
        }
        if (!__all_sync(0xffffffffu, okc)) {
          timed_out = true;
          break;
        }
        uint8_t* slot = bop + (size_t)b * kSlotBytes;
        uint8_t* reg = slot + (size_t)(lane >> 4) * (N * 128);
        const int chunk = (lane & 15) >> 1, half = (lane & 1) * 8;
        int bad = 0;
#pragma unroll 4
        for (int r = 0; r < RG; ++r) {
          float4 v4 = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
          if (r < rank) v4 = *reinterpret_cast<const float4*>(bfs + r * kBStride + 4 * lane);
          const float vv[4] = {v4.x, v4.y, v4.z, v4.w};
          __half hh[4], ll[4];
#pragma unroll
          for (int k = 0; k < 4; ++k) {
            hh[k] = __float2half_rn(vv[k]);
            ll[k] = __float2half_rn(__fmul_rn(__fsub_rn(vv[k], __half2float(hh[k])), kLoScale));
          }
          *reinterpret_cast<uint2*>(reg + r * 128 + ((chunk ^ (r & 7)) << 4) + half) =
              make_uint2(*reinterpret_cast<const uint32_t*>(&hh[0]), *reinterpret_cast<const uint32_t*>(&hh[2]));
          const int rl = RG + r;
          *reinterpret_cast<uint2*>(reg + rl * 128 + ((chunk ^ (rl & 7)) << 4) + half) =
              make_uint2(*reinterpret_cast<const uint32_t*>(&ll[0]), *reinterpret_cast<const uint32_t*>(&ll[2]));
        }
        // 8 lanes per row (16 columns each), 4 rows at a time: partial sums
        // of squares rounded upward, combined by upward-rounded shuffle adds,
        // so every sum stays an upper bound of the exact one. Only the exact
        // engine's verification reads the bounds.
        for (int r0 = 0; EXACT && r0 < RG; r0 += 4) {
          const int r = r0 + (lane >> 3), c0 = 16 * (lane & 7);
          float sv = 0.0f, sh = 0.0f, sl = 0.0f, se = 0.0f;
          if (r < rank) {
#pragma unroll
            for (int c4 = 0; c4 < 4; ++c4) {
              const float4 v4 = *reinterpret_cast<const float4*>(bfs + r * kBStride + c0 + 4 * c4);
              const float vv[4] = {v4.x, v4.y, v4.z, v4.w};
#pragma unroll
              for (int k = 0; k < 4; ++k) {
                const float hf = __half2float(__float2half_rn(vv[k]));
                const float r1 = __fsub_rn(vv[k], hf);  // exact: hf is vv rounded to 11 bits
                const float lf = __half2float(__float2half_rn(__fmul_rn(r1, kLoScale)));
                const float e = __fsub_rn(r1, __fmul_rn(lf, kLoInv));  // exact for the same reason
                bad |= !(isfinite(vv[k]) && isfinite(hf) && isfinite(lf));
                sv = __fmaf_ru(vv[k], vv[k], sv);
                sh = __fmaf_ru(hf, hf, sh);
                sl = __fmaf_ru(lf, lf, sl);
                se = __fmaf_ru(e, e, se);
              }
            }
          }
#pragma unroll
          for (int o = 4; o > 0; o >>= 1) {
            sv = __fadd_ru(sv, __shfl_xor_sync(0xffffffffu, sv, o));
            sh = __fadd_ru(sh, __shfl_xor_sync(0xffffffffu, sh, o));
            sl = __fadd_ru(sl, __shfl_xor_sync(0xffffffffu, sl, o));
            se = __fadd_ru(se, __shfl_xor_sync(0xffffffffu, se, o));
          }
          // every sum and root rounded up, then 2^-10 more for the sums' rounding
          const float bnd = __fmaf_ru(
              kTcRelF, __fadd_ru(__fsqrt_ru(sh), __fmul_ru(__fsqrt_ru(sl), kLoInv)),
              __fmaf_ru(kChainRelF, __fsqrt_ru(sv), __fsqrt_ru(se)));
          if ((lane & 7) == 0 && r < RG) info[b].bn[r] = (r < rank) ? __fmul_ru(bnd, 1.0f + 1.0f / 1024.0f) : 0.0f;
        }
        bad = __any_sync(0xffffffffu, bad);
        if (lane == 0) {
          const long long hb = (long long)h * tiles;
          const long long lo_it = std::max(i0, hb), hi_it = std::min(i1, hb + tiles);
          info[b].rank = rank;
          info[b].exact_only = bad;
          info[b].expected = 4 * (int)(hi_it - lo_it);
          done[b] = 0;
        }
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");  // the operands are read by the tensor core
        __syncwarp();
        if (lane == 0) mbar_arrive(&bfull[b]);
        cur_h = h;
      }
      if (lane == 0) {
        const int s = n % kStages, a = n % kAcc, b = hs % kSlots;
        bool ok = mbar_wait(&x_full[s], (uint32_t)((n / kStages) & 1), abort_flag);
        if (ok && n >= kAcc) ok = mbar_wait(&acc_empty[a], (uint32_t)((n / kAcc - 1) & 1), abort_flag);
        if (!ok) {
          timed_out = true;
        } else {
          asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
          const uint32_t xa = sa(xs + (size_t)s * kTileBytes);
          const uint32_t ba = sa(bop + (size_t)b * kSlotBytes);
#pragma unroll
          for (int k = 0; k < kD / 16; ++k) {  // K = 16 per MMA: 32 bytes inside a 128-byte swizzle row
            const uint32_t off = (uint32_t)((k & 3) * 32);
            mma_f16<N>(tmem + (uint32_t)(a * N), sdesc_sw128(xa + (k >> 2) * kRegionBytes + off),
                       sdesc_sw128(ba + (k >> 2) * (N * 128) + off), k > 0 ? 1u : 0u);
          }
          asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                           sa(&acc_full[a]))
                       : "memory");
          if (!EXACT)  // the epilogue reads no x: the stage is free once the MMAs have read it
            asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                             sa(&x_empty[s]))
                         : "memory");
          last_acc = n;
        }
      }
      timed_out = __shfl_sync(0xffffffffu, (int)timed_out, 0) != 0;
    }
    if (lane == 0 && last_acc >= 0 && (timed_out || *abort_flag))  // MMAs in flight finish before TMEM is freed
      mbar_wait_bounded(sa(&acc_full[last_acc % kAcc]), (uint32_t)((last_acc / kAcc) & 1), kWaitNs);
    __syncwarp();
  } else {
    // ---------------- epilogue ----------------
    const int q = w & 3;               // TMEM lanes 32q .. 32q + 31 (the warp's place in its warpgroup)
    const int g = (w - 2) >> 2;        // epilogue group
    const int row = 32 * q + lane;     // the thread's token row in a tile
    const int swz = row & 7;
    const float levels = o.levels;
    const RowOut ro{o.scales, o.mins, o.packed, o.codes, o.levels};
    for (int n = g; n < nit; n += kGroups) {
      const long long it = i0 + n;
      const int h = (int)(it / tiles), tile = (int)(it - (long long)h * tiles);
      const int hs = h - h_first, b = hs % kSlots, a = n % kAcc, s = n % kStages;
      const int t = tile * kRows + row;
      const bool ok = t < T;
      const size_t grow = (size_t)h * T + (size_t)(ok ? t : 0);
      bool got = mbar_wait(&bfull[b], (uint32_t)((hs / kSlots) & 1), abort_flag);
      // (the approximate engine reads no x, and its stage may already hold a later tile)
      if (EXACT) got = got && mbar_wait(&x_full[s], (uint32_t)((n / kStages) & 1), abort_flag);
      got = got && mbar_wait(&acc_full[a], (uint32_t)((n / kAcc) & 1), abort_flag);
      if (__any_sync(0xffffffffu, !got)) {  // the warp leaves together (tcgen05.ld is warp-wide)
        timed_out = true;
        break;
      }
      asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
      const uint32_t tacc = tmem + ((uint32_t)(32 * q) << 16) + (uint32_t)(a * N);
      const int rank = info[b].rank;
      // coefficients: Q = hi + lo * 2^-11, columns from the rank on +0.0
      // exactly (projection.rs:96); every loop below is branch-free over RG
      // columns, with the columns from R on masked
      float P[RG];
      {
        constexpr int kC = RG < 32 ? RG : 32;  // columns per TMEM wait
#pragma unroll
        for (int c0 = 0; c0 < RG; c0 += kC) {
          uint32_t hv[kC], lv[kC];
#pragma unroll
          for (int r0 = 0; r0 < kC; r0 += 8) {
            tmem_ld8(tacc + (uint32_t)(c0 + r0), hv + r0);
            tmem_ld8(tacc + (uint32_t)(RG + c0 + r0), lv + r0);
          }
          asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
          for (int k = 0; k < kC; ++k) {
            const float v = __fmaf_rn(__uint_as_float(lv[k]), kLoInv, __uint_as_float(hv[k]));
            P[c0 + k] = (c0 + k < rank) ? v : 0.0f;
          }
        }
      }
      asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
      __syncwarp();
      if (lane == 0) mbar_arrive(&acc_empty[a]);
      if constexpr (!EXACT) {
        float mn = INFINITY, mx = -INFINITY;
#pragma unroll
        for (int r = 0; r < RG; ++r) {
          const float v = __fadd_rn(P[r], 0.0f);  // -0.0 as +0.0, as mm_update
          mn = (r < R) ? fminf(mn, v) : mn;
          mx = (r < R) ? fmaxf(mx, v) : mx;
        }
        const float scale = make_scale(mn, mx, levels);
        const float inv = __frcp_rn(scale);
        uint32_t cd[RG];
#pragma unroll
        for (int r = 0; r < RG; ++r) cd[r] = qcode_fast(P[r], mn, scale, inv, levels);
        if (ok) write_row<RG>(cd, grow, R, scale, mn, ro, shist, hist_on);
        __syncwarp();
        if (lane == 0) atomicAdd(&done[b], 1);
        continue;
      }
      // the smallest and largest approximate coefficients
      int rA = 0, rB = 0;
      float qa = P[0], qb = P[0];
#pragma unroll
      for (int r = 1; r < RG; ++r) {
        const bool lt = r < R && P[r] < qa, gt = r < R && P[r] > qb;
        qa = lt ? P[r] : qa;
        rA = lt ? r : rA;
        qb = gt ? P[r] : qb;
        rB = gt ? r : rB;
      }
      const uint8_t* xrow = xs + (size_t)s * kTileBytes + row * 128;
      const float* B = bf + (size_t)b * RG * kBStride;
      const float3 e = exact2_norm(xrow, swz, B + rA * kBStride, B + rB * kBStride);
      // ||x||_2 rounded up (the sum's relative error is below 2^-17)
      const float xn = __fmul_ru(__fsqrt_ru(e.z), 1.0f + 1.0f / 4096.0f);
      bool defer = info[b].exact_only || !(xn <= 3.0e38f);
      set_at<RG>(P, rA, e.x);
      set_at<RG>(P, rB, e.y);
      // Delta_r of the coefficients still approximate (0 for the exact ones);
      // no other coefficient may lie below the exact minimum or above the
      // exact maximum
      const float* bn = info[b].bn;
      auto delta = [&](int r) {
        const bool exact = r == rA || r == rB || r >= rank;
        return exact ? 0.0f : __fmaf_ru(xn, bn[r], __fmul_ru(fabsf(P[r]), 1.0f / 4194304.0f));
      };
#pragma unroll
      for (int r = 0; r < RG; ++r) {
        const float d = delta(r);
        const bool below = r != rA && __fsub_rd(P[r], d) < e.x;
        const bool above = r != rB && __fadd_ru(P[r], d) > e.y;
        defer = defer || (r < R && (below || above));
      }
      const float mn = __fadd_rn(e.x, 0.0f), mx = __fadd_rn(e.y, 0.0f);  // -0.0 as +0.0, as mm_update
      const float scale = make_scale(mn, mx, levels);
      const float inv = __frcp_rn(scale);
      // codes; one whose value interval reaches within the margin of a
      // rounding boundary (a half-integer of the quotient) defers the row
      const float invm = __fmul_ru(inv, 1.001f);
      uint32_t cd[RG];
#pragma unroll
      for (int r = 0; r < RG; ++r) {
        const float z = __fmul_rn(__fsub_rn(P[r], mn), inv);
        const float tz = __fadd_rn(z, 0.5f);
        const float fl = floorf(tz);
        const float fr = __fsub_rn(tz, fl);
        const float m = __fmaf_ru(delta(r), invm, __fmaf_ru(fabsf(z), 1.0f / 524288.0f, 1.0f / 262144.0f));
        defer = defer || (r < R && (fr < m || fr > 1.0f - m));
        cd[r] = (uint32_t)fminf(fmaxf(fl, 0.0f), levels);
      }
      if (ok) {
        if (!defer) {
          write_row<RG>(cd, grow, R, scale, mn, ro, shist, hist_on);
        } else {
          const int slot = atomicAdd(dcount, 1);
          if (slot < kDefCap) dlist[slot] = (uint32_t)grow;
          else finish_row<RG>(x, grow, T, R, bvt, ranks, ro.scales, ro.mins, ro.packed, ro.codes, ro.levels, shist,
                              hist_on);  // list full: now
        }
      }
      __syncwarp();  // every lane is done with the stage and the slot
      if (lane == 0) {
        __threadfence_block();  // this warp's reads of the slot come before the arrival
        mbar_arrive(&x_empty[s]);
        atomicAdd(&done[b], 1);
      }
    }
    if (timed_out) *abort_flag = 1;
    // the deferred rows, spread over every epilogue thread
    asm volatile("bar.sync 1, %0;" ::"n"(kEpiWarps * 32) : "memory");
    if (!*abort_flag) {
      const int nd = min(*reinterpret_cast<volatile int*>(dcount), kDefCap);
      for (int i = tid - 64; i < nd; i += kEpiWarps * 32)
        finish_row<RG>(x, (size_t)dlist[i], T, R, bvt, ranks, ro.scales, ro.mins, ro.packed, ro.codes, ro.levels,
                       shist, hist_on);
    }
  }
  if (timed_out) {
    *abort_flag = 1;
    if (o.status && lane == 0) atomicOr(o.status, kDevErrTimeout);
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  if (w == 1) asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemCols));
  if (hist_on)
    for (int i = tid; i < 256; i += blockDim.x)
      if (shist[i]) atomicAdd(&o.hist[i], shist[i]);
}

template <int RG>
constexpr PtLayout pt_layout() {
  constexpr int kStages = PtCfg<RG>::kStages, kAcc = PtCfg<RG>::kAcc;
  PtLayout L{};
  int off = 0;
  L.xs = off;
  off += kStages * kTileBytes;
  L.bop = off;
  off += pt_slots<RG>() * (2 * (2 * RG) * 128);
  L.bf = off;
  off += pt_slots<RG>() * RG * kBStride * 4;
  L.info = off;
  off += pt_slots<RG>() * (int)sizeof(PtInfo);
  L.bars = off;
  off += (2 * kStages + 2 * kAcc + 3) * 8 + 4 * 4 + 16;
  L.dlist = off;
  off += kDefCap * 4;
  L.hist = off;
  off += 256 * 4;
  L.total = off + 1024;  // alignment slack for the 1024-byte base
  return L;
}

// [H*T rows, 128 columns] f16, boxes of 64 columns x 128 rows, 128-byte swizzle
bool encode_x_map(CUtensorMap* map, const __half* x, size_t rows) {
  auto enc = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(tensor_map_encode_fn());
  if (!enc) return false;
  const cuuint64_t gdim[2] = {(cuuint64_t)kD, (cuuint64_t)rows};
  const cuuint64_t gstride[1] = {(cuuint64_t)(kD * 2)};
  const cuuint32_t box[2] = {64, (cuuint32_t)kRows};
  const cuuint32_t estride[2] = {1, 1};
  return enc(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<__half*>(x), gdim, gstride, box, estride,
             CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
             CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

template <int RG, bool EXACT>
cudaError_t launch_tc_rg(const CUtensorMap& map, const __half* x, size_t H, size_t T, const float* bvt,
                         const uint64_t* ranks, size_t R, const ProjectOut& o, cudaStream_t st) {
  auto kern = k_project_tc<RG, EXACT>;
  constexpr PtLayout L = pt_layout<RG>();
  // more than half of the SM's shared memory: one CTA per SM, so no other
  // TMEM-allocating kernel of this library shares the SM and the allocation
  // never waits
  static_assert(2 * L.total > 228 * 1024, "one CTA per SM keeps the TMEM allocation non-blocking");
  static_assert(L.total <= 227 * 1024, "shared memory per block");
  constexpr int kDevs = 64;
  static std::atomic<int> sms[kDevs];
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 0 || dev >= kDevs) return cudaErrorInvalidDevice;
  int nsm = sms[dev].load(std::memory_order_acquire);
  if (!nsm) {
    if ((e = cudaDeviceGetAttribute(&nsm, cudaDevAttrMultiProcessorCount, dev)) != cudaSuccess) return e;
    if ((e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, L.total)) != cudaSuccess)
      return e;
    sms[dev].store(nsm, std::memory_order_release);
  }
  const size_t items = H * ((T + kRows - 1) / kRows);
  const unsigned grid = (unsigned)std::max<size_t>(1, std::min<size_t>(items, (size_t)nsm));
  kern<<<grid, PtCfg<RG>::kThreads, L.total, st>>>(map, x, (int)H, (int)T, bvt, ranks, (int)R, L, o);
  note_launches(1);
  return cudaGetLastError();
}

}  // namespace

bool project_tc_fits(const void* x, int in_dtype, size_t H, size_t T, size_t D, const float* basis_vt, size_t R) {
  return in_dtype == KVF_IN_F16 && D == (size_t)kD && R > 0 && R <= 64 && aligned(x, 16) && aligned(basis_vt, 16) &&
         H * T > 0 && H * T < (1ull << 31) && tensor_map_encode_fn() != nullptr;
}

cudaError_t launch_project_tc(const void* x, int in_dtype, size_t H, size_t T, size_t D, const float* basis_vt,
                              const uint64_t* ranks, size_t R, bool exact, const ProjectOut& o, cudaStream_t st) {
  if (o.mode != 2 || !project_tc_fits(x, in_dtype, H, T, D, basis_vt, R) || (o.packed && (R & 1)) || H * T >= (1ull << 32))
    return cudaErrorNotSupported;
  CUtensorMap map{};
  if (!encode_x_map(&map, static_cast<const __half*>(x), H * T)) return cudaErrorNotSupported;
  const __half* xh = static_cast<const __half*>(x);
  if (exact) {
    if (R <= 8) return launch_tc_rg<8, true>(map, xh, H, T, basis_vt, ranks, R, o, st);
    if (R <= 16) return launch_tc_rg<16, true>(map, xh, H, T, basis_vt, ranks, R, o, st);
    if (R <= 32) return launch_tc_rg<32, true>(map, xh, H, T, basis_vt, ranks, R, o, st);
    return launch_tc_rg<64, true>(map, xh, H, T, basis_vt, ranks, R, o, st);
  }
  if (R <= 8) return launch_tc_rg<8, false>(map, xh, H, T, basis_vt, ranks, R, o, st);
  if (R <= 16) return launch_tc_rg<16, false>(map, xh, H, T, basis_vt, ranks, R, o, st);
  if (R <= 32) return launch_tc_rg<32, false>(map, xh, H, T, basis_vt, ranks, R, o, st);
  return launch_tc_rg<64, false>(map, xh, H, T, basis_vt, ranks, R, o, st);
}

}  // namespace kvf
