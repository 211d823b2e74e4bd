// Tensor-core reconstruction (sm_100a): X̂[h] = P̂[h] · V[h] on tcgen05 with the
// accumulators in tensor memory.
//
// The reference reconstructs with a scalar multiply-add loop
// (crates/kvforge-cpu/src/projection.rs:142-172); its result is a tolerance
// check (relative Frobenius error, 1e-4 for fp32), not a bit-exact one, so the
// default reconstruction runs here as a GEMM: M = 128 tokens, N = D = 128
// output channels, K = R coefficients (padded to 8, 16, 32 or 64). Each f32 operand is
// split into two tf32 parts (split_tf32); three kind::tf32 passes
// (hi·hi + hi·lo + lo·hi) leave a relative error near 2^-21 per product. The
// separately rounded CPU order stays available bit for bit on the CUDA-core
// kernel (kvf_set_exact_reconstruct).
//
// The kernel writes 512 B per token and reads 4-64 B, so it is bound by HBM
// writes; its job is to keep tensor-map stores in flight on every SM at all
// times. One persistent CTA per SM walks (head, 128-token tile) items with
// two warp roles that run a tile apart:
//   producer warps 4-7: dequantize one token row per thread (q * scale + min,
//     separately rounded as the reference does; inputs fetched three tiles
//     ahead, one tile for 64 f32 coefficients per row)
//     into the A operands of stage n % 2 (one stage at K = 64; K-major core matrices without
//     swizzle; the head's basis sits the same way in the B operands); one
//     thread issues the MMAs into TMEM accumulator n % 2 and commits them to
//     acc_full[n % 2];
//   epilogue warps 0-3: warp w owns TMEM lanes (tokens) 32w..32w+31; it reads
//     64 columns per wait (two tcgen05.ld 32x32b.x32) into two slots of its
//     private ring of 128-byte-swizzled staging slots and stores each slot with
//     one 3-D tensor-map store (32 channels x 32 tokens x 1 head), so rows past
//     the head's last token are clipped by the copy engine; after its last
//     TMEM read of a tile it frees the accumulator (acc_empty).
// Every mbarrier wait is bounded; a wait that runs out sets an abort flag that
// ends both roles, and kDevErrTimeout in the status word. No multicast.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <algorithm>
#include <atomic>

#include "kvf_internal.cuh"

namespace kvf {
namespace {

constexpr int kTcRows = 128;  // tokens per tile: MMA M, TMEM lanes
constexpr int kTcD = 128;     // output channels: MMA N, TMEM columns per accumulator
constexpr int kEpiWarps = 4;
constexpr int kProdWarps = 4;
constexpr int kTcThreads = 32 * (kEpiWarps + kProdWarps);
constexpr int kProdThreads = 32 * kProdWarps;
constexpr int kRowsPerProd = kTcRows / kProdThreads;  // 1
constexpr int kSlotBytes = 32 * 128;  // one staging slot: 32 tokens x 32 channels
constexpr int kTmemCols = 2 * kTcD;   // two accumulators

// shared-memory plan per K (= 4 KC coefficients): two A-operand stages and
// six staging slots per epilogue warp up to K = 32; one A stage and four slots
// at K = 64, where the operands (4 x 32 KB) leave no room for more
template <int KC>
struct TcPlan {
  static constexpr int kAStages = KC <= 8 ? 2 : 1;
  static constexpr int kSlots = KC <= 8 ? 6 : 4;  // even: filled in pairs
};
// tiles ahead that a producer thread's inputs are fetched: three register
// sets in rotation, or one set for 64 f32 coefficients per row
template <int MODE, int KC>
constexpr int tc_depth() {
  return (MODE == 0 && KC == 16) ? 1 : 3;
}

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

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(sa(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(sa(bar)) : "memory");
}
// waits for the phase of `parity` to complete; false when the wait ran out or
// the other role raised the abort flag
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, volatile int* abort_flag) {
  return mbar_wait_bounded(sa(bar), parity, kWaitNs, abort_flag);
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

// 32 consecutive f32 columns of this warp's 32 TMEM lanes (one per thread)
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t* v) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, "
      "%14, %15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
      : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]),
        "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15]),
        "=r"(v[16]), "=r"(v[17]), "=r"(v[18]), "=r"(v[19]), "=r"(v[20]), "=r"(v[21]), "=r"(v[22]), "=r"(v[23]),
        "=r"(v[24]), "=r"(v[25]), "=r"(v[26]), "=r"(v[27]), "=r"(v[28]), "=r"(v[29]), "=r"(v[30]), "=r"(v[31])
      : "r"(taddr));
}

// named barrier 1 over the producer warps only
__device__ __forceinline__ void producer_sync() {
  asm volatile("bar.sync 1, %0;" ::"n"(kProdThreads) : "memory");
}
// the same barrier, returning whether `p` holds on any producer thread: every
// producer takes the same branch after it
__device__ __forceinline__ bool producer_any(bool p) {
  uint32_t r;
  asm volatile(
      "{\n .reg .pred p, q;\n setp.ne.u32 p, %1, 0;\n bar.red.or.pred q, 1, %2, p;\n selp.u32 %0, 1, 0, q;\n}\n"
      : "=r"(r)
      : "r"((uint32_t)p), "n"(kProdThreads)
      : "memory");
  return r != 0;
}

// one producer thread's token rows of one item, fetched ahead (tc_depth)
template <int MODE, int KC>
struct RowsIn {
  CodeWords<MODE == 0 ? 1 : code_words<MODE == 2, 4 * KC>()> cw[kRowsPerProd];  // codes, as loaded
  float raw[kRowsPerProd][MODE == 0 ? 4 * KC : 1];
  float sc[kRowsPerProd], mn[kRowsPerProd];
};

// MODE 0: raw f32 coefficients, 1: INT8 codes, 2: INT4 codes; KC: K in 4-wide chunks (2, 4, 8 or 16)
template <int MODE, int KC>
__global__ void __launch_bounds__(kTcThreads, 1)
    k_reconstruct_tc(const __grid_constant__ CUtensorMap omap, const uint8_t* __restrict__ codes,
                     size_t ncode_bytes, const float* __restrict__ raw, const float* __restrict__ scales,
                     const float* __restrict__ mins, int axis, int H, int T, int R,
                     const float* __restrict__ bvt, const uint64_t* __restrict__ ranks,
                     unsigned* __restrict__ status) {
  constexpr int K = 4 * KC;
  constexpr int kOpBytes = kTcRows * K * 4;  // one operand part
  constexpr int kAStages = TcPlan<KC>::kAStages;
  constexpr int kSlots = TcPlan<KC>::kSlots;
  extern __shared__ uint8_t sm_raw[];
  // staging slots use the 128-byte swizzle, whose pattern is taken from
  // address bits 7-9: the layout starts on a 1024-byte boundary
  uint8_t* sm = sm_raw + ((1024u - (sa(sm_raw) & 1023u)) & 1023u);
  uint8_t* ring = sm;                                       // [4 warps][kSlots][32 rows][128 B]
  uint8_t* a_ops = ring + kEpiWarps * kSlots * kSlotBytes;  // [kAStages][hi, lo]
  uint8_t* b_hi = a_ops + 2 * kAStages * kOpBytes;
  uint8_t* b_lo = b_hi + kOpBytes;
  float* pscale = reinterpret_cast<float*>(b_lo + kOpBytes);  // per-channel parameters of the head [K]
  float* pmin = pscale + K;
  uint64_t* acc_full = reinterpret_cast<uint64_t*>(pmin + K);  // [2]: the stage's MMAs completed
  uint64_t* acc_empty = acc_full + 2;                          // [2]: the epilogue read the accumulator
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acc_empty + 2);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  const int tid = threadIdx.x, w = tid >> 5, lane = tid & 31;
  const int tiles = (T + kTcRows - 1) / kTcRows;
  const long long items = (long long)H * tiles;
  const long long i0 = items * blockIdx.x / gridDim.x;
  const long long i1 = items * (blockIdx.x + 1) / gridDim.x;

  if (w == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(sa(tmem_slot)),
                 "r"(kTmemCols));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::);
  }
  if (tid == 32) {
    mbar_init(&acc_full[0], 1);
    mbar_init(&acc_full[1], 1);
    mbar_init(&acc_empty[0], kEpiWarps);
    mbar_init(&acc_empty[1], kEpiWarps);
    *abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  const uint32_t tmem = *tmem_slot;
  bool timed_out = false;

  if (w >= kEpiWarps) {
    // ---------------- producer ----------------
    const int pt = tid - 32 * kEpiWarps;
    auto fetch = [&](long long it, RowsIn<MODE, KC>& in) {
      const int h = (int)(it / tiles), tile = (int)(it - (long long)h * tiles);
#pragma unroll
      for (int j = 0; j < kRowsPerProd; ++j) {
        const int t = tile * kTcRows + pt + j * kProdThreads;
        const bool ok = t < T;
        const size_t g = (size_t)h * T + (ok ? t : 0);
        in.sc[j] = in.mn[j] = 0.0f;
        if (MODE != 0 && axis != KVF_PER_CHANNEL && ok) {
          in.sc[j] = __ldg(scales + g);
          in.mn[j] = __ldg(mins + g);
        }
        if (MODE == 0) {
#pragma unroll
          for (int k = 0; k < K; ++k) in.raw[j][k] = (ok && k < R) ? __ldg(raw + g * R + k) : 0.0f;
        } else {
          load_code_words<MODE == 2>(codes, ncode_bytes, g * R, ok, in.cw[j]);
        }
      }
    };
    int cur_h = -1, rank = 0;
    constexpr int kDepth = tc_depth<MODE, KC>();
    // one tile's work; `in` holds its inputs and is refilled with those of the
    // tile kDepth ahead. Returns true when the producers stop (together).
    auto step = [&](long long it, RowsIn<MODE, KC>& in) -> bool {
      const int n = (int)(it - i0), s = n & 1, as_ = n % kAStages;
      const int h = (int)(it / tiles), tile = (int)(it - (long long)h * tiles);
      // a new head's basis may be written once the MMAs of tile n - 1
      // completed; A stage as_ once those of tile n - kAStages did
      if (!timed_out && h != cur_h && n >= 1 && !mbar_wait(&acc_full[(n - 1) & 1], ((n - 1) >> 1) & 1, abort_flag))
        timed_out = true;
      const int m = n - kAStages;
      if (!timed_out && m >= 0 && !mbar_wait(&acc_full[m & 1], (m >> 1) & 1, abort_flag)) timed_out = true;
      if (timed_out) *abort_flag = 1;
      if (producer_any(timed_out || *abort_flag)) return true;
      if (h != cur_h) {
        const uint64_t rk = ranks[h];
        rank = (int)(rk < (uint64_t)R ? rk : (uint64_t)R);
        const float* B = bvt + (size_t)h * R * kTcD;
        constexpr int kPer = kTcD * K / kProdThreads;  // basis elements per producer thread
        float bv[kPer];
#pragma unroll
        for (int u = 0; u < kPer; ++u) {  // all loads first, then the splits
          const int i = pt + u * kProdThreads, k = i / kTcD, c = i - k * kTcD;
          bv[u] = (k < rank) ? __ldg(B + (size_t)k * kTcD + c) : 0.0f;  // consecutive threads, consecutive channels
        }
#pragma unroll
        for (int u = 0; u < kPer; ++u) {
          const int i = pt + u * kProdThreads, k = i / kTcD, c = i - k * kTcD;
          float hi, lo;
          split_tf32(bv[u], hi, lo);
          *reinterpret_cast<float*>(b_hi + kmaj(c, k, KC)) = hi;
          *reinterpret_cast<float*>(b_lo + kmaj(c, k, KC)) = lo;
        }
        if (MODE != 0 && axis == KVF_PER_CHANNEL)
          for (int k = pt; k < K; k += kProdThreads) {
            pscale[k] = (k < R) ? __ldg(scales + (size_t)h * R + k) : 0.0f;
            pmin[k] = (k < R) ? __ldg(mins + (size_t)h * R + k) : 0.0f;
          }
        cur_h = h;
        producer_sync();
      }
      uint8_t* a_hi = a_ops + (2 * as_) * kOpBytes;
      uint8_t* a_lo = a_hi + kOpBytes;
#pragma unroll
      for (int j = 0; j < kRowsPerProd; ++j) {  // terms k >= rank are zero
        const int row = pt + j * kProdThreads;
        const bool ok = tile * kTcRows + row < T;
#pragma unroll
        for (int kc = 0; kc < KC; ++kc) {
          float hi4[4], lo4[4];
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const int k = 4 * kc + e;
            float d = 0.0f;
            if (ok && k < rank) {
              if (MODE == 0) {
                d = in.raw[j][k];
              } else {
                const float q = (float)code_at<MODE == 2>(in.cw[j], k);
                const float sc = (axis == KVF_PER_CHANNEL) ? pscale[k] : in.sc[j];
                const float mn = (axis == KVF_PER_CHANNEL) ? pmin[k] : in.mn[j];
                d = __fadd_rn(__fmul_rn(q, sc), mn);  // q * scale + min, separately rounded
              }
            }
            split_tf32(d, hi4[e], lo4[e]);
          }
          *reinterpret_cast<float4*>(a_hi + kmaj(row, 4 * kc, KC)) = make_float4(hi4[0], hi4[1], hi4[2], hi4[3]);
          *reinterpret_cast<float4*>(a_lo + kmaj(row, 4 * kc, KC)) = make_float4(lo4[0], lo4[1], lo4[2], lo4[3]);
        }
      }
      // the operands are read by the tensor core through the async proxy
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      producer_sync();
      if (pt == 0) {
        // accumulator s is free once the epilogue read tile n - 2 from it
        if (n >= 2 && !mbar_wait(&acc_empty[s], ((n - 2) >> 1) & 1, abort_flag)) {
          timed_out = true;  // the next step's vote ends the producers
          *abort_flag = 1;
        } else {
          asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
          const uint32_t sbo = KC * 128;
          const uint8_t* as[3] = {a_hi, a_hi, a_lo};  // hi·hi + hi·lo + lo·hi
          const uint8_t* bs[3] = {b_hi, b_lo, b_hi};
          uint32_t acc = 0;
#pragma unroll
          for (int p = 0; p < 3; ++p)
#pragma unroll
            for (int ks = 0; ks < KC / 2; ++ks) {  // one MMA covers K = 8: two 16-byte core-matrix columns
              mma_tf32(tmem + (uint32_t)(s * kTcD), sdesc(sa(as[p]) + ks * 256, 128, sbo),
                       sdesc(sa(bs[p]) + ks * 256, 128, sbo), acc);
              acc = 1;
            }
          asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                           sa(&acc_full[s]))
                       : "memory");
        }
      }
      if (it + kDepth < i1) fetch(it + kDepth, in);  // in flight for the next kDepth tiles
      return false;
    };
    if constexpr (kDepth == 3) {
      // three register sets in rotation, so no set is copied while its loads are in flight
      RowsIn<MODE, KC> r0, r1, r2;
      if (i0 < i1) fetch(i0, r0);
      if (i0 + 1 < i1) fetch(i0 + 1, r1);
      if (i0 + 2 < i1) fetch(i0 + 2, r2);
      for (long long it = i0; it < i1; it += 3) {
        if (step(it, r0)) break;
        if (it + 1 < i1 && step(it + 1, r1)) break;
        if (it + 2 < i1 && step(it + 2, r2)) break;
      }
    } else {
      RowsIn<MODE, KC> r0;
      if (i0 < i1) fetch(i0, r0);
      for (long long it = i0; it < i1; ++it)
        if (step(it, r0)) break;
    }
  } else {
    // ---------------- epilogue ----------------
    uint8_t* my_ring = ring + w * (kSlots * kSlotBytes);
    int slot = 0;
    for (long long it = i0; it < i1; ++it) {
      const int n = (int)(it - i0), s = n & 1;
      const int h = (int)(it / tiles), tile = (int)(it - (long long)h * tiles);
      const bool ok = mbar_wait(&acc_full[s], (n >> 1) & 1, abort_flag);
      if (__any_sync(0xffffffffu, !ok)) {  // the warp leaves together (tcgen05.ld is warp-wide)
        timed_out = true;
        *abort_flag = 1;
        break;
      }
      asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
      const int row0 = tile * kTcRows + 32 * w;  // first token of this warp's rows
#pragma unroll 1
      for (int cp = 0; cp < kTcD / 64; ++cp) {  // 64 channels (two TMEM loads, two slots) per wait
        uint32_t v[64];
        const uint32_t taddr = tmem + ((uint32_t)(32 * w) << 16) + (uint32_t)(s * kTcD + 64 * cp);
        tmem_ld32(taddr, v);
        tmem_ld32(taddr + 32, v + 32);
        asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
        if (cp == kTcD / 64 - 1) {  // the accumulator is read: the producer may reuse it
          asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
          __syncwarp();
          if (lane == 0) mbar_arrive(&acc_empty[s]);
        }
        // the store group that used these two slots kSlots / 2 groups ago has read them
        if (lane == 0) asm volatile("cp.async.bulk.wait_group.read %0;" ::"n"(kSlots / 2 - 1) : "memory");
        __syncwarp();
#pragma unroll
        for (int half = 0; half < 2; ++half) {
          uint8_t* rowp = my_ring + (slot + half) * kSlotBytes + lane * 128;
#pragma unroll
          for (int j = 0; j < 8; ++j)  // 16-byte chunk j of row `lane` lands at j ^ (lane mod 8)
            *reinterpret_cast<uint4*>(rowp + ((j ^ (lane & 7)) << 4)) =
                make_uint4(v[32 * half + 4 * j], v[32 * half + 4 * j + 1], v[32 * half + 4 * j + 2],
                           v[32 * half + 4 * j + 3]);
        }
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        __syncwarp();
        if (lane == 0) {
          if (row0 < T)  // rows past T are clipped by the copy; slots wholly past T are skipped
#pragma unroll
            for (int half = 0; half < 2; ++half)
              asm volatile(
                  "cp.async.bulk.tensor.3d.global.shared::cta.bulk_group [%0, {%2, %3, %4}], [%1];" ::"l"(&omap),
                  "r"(sa(my_ring + (slot + half) * kSlotBytes)), "r"(64 * cp + 32 * half), "r"(row0), "r"(h)
                  : "memory");
          asm volatile("cp.async.bulk.commit_group;" ::: "memory");
        }
        slot = (slot + 2 == kSlots) ? 0 : slot + 2;
      }
    }
    if (lane == 0) asm volatile("cp.async.bulk.wait_group 0;" ::: "memory");
  }
  if (timed_out) {
    *abort_flag = 1;
    if (status) atomicOr(status, kDevErrTimeout);
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  if (w == 0) asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemCols));
}

// [H, T, D] f32 output, box 32 channels x 32 tokens x 1 head, 128-byte swizzle
bool encode_out_map(CUtensorMap* map, float* out, size_t H, size_t T) {
  auto enc = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(tensor_map_encode_fn());
  if (!enc) return false;
  const cuuint64_t gdim[3] = {(cuuint64_t)kTcD, (cuuint64_t)T, (cuuint64_t)H};
  const cuuint64_t gstride[2] = {(cuuint64_t)kTcD * 4, (cuuint64_t)T * kTcD * 4};
  const cuuint32_t box[3] = {32, 32, 1};
  const cuuint32_t estride[3] = {1, 1, 1};
  return enc(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, out, gdim, gstride, box, estride, CU_TENSOR_MAP_INTERLEAVE_NONE,
             CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_NONE,
             CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

template <int KC>
constexpr size_t tc_smem() {
  return 1024 + (size_t)kEpiWarps * TcPlan<KC>::kSlots * kSlotBytes +
         (2 * TcPlan<KC>::kAStages + 2) * (size_t)kTcRows * (4 * KC) * 4 + 2 * (4 * KC) * 4 + 64;
}

template <int MODE, int KC>
cudaError_t launch_tc(const CUtensorMap& map, const uint8_t* codes, const float* raw, const float* scales,
                      const float* mins, int axis, size_t H, size_t T, size_t R, const float* bvt,
                      const uint64_t* ranks, unsigned* status, cudaStream_t st) {
  auto kern = k_reconstruct_tc<MODE, KC>;
  constexpr size_t smem = tc_smem<KC>();
  // more than half of the SM's 228 KB of shared memory: at most one CTA of
  // this kernel per SM, so the 256 TMEM columns it allocates are always free
  static_assert(2 * (smem + 1024) > 228 * 1024, "one CTA per SM keeps the TMEM allocation non-blocking");
  // per device: the SM count once the shared-memory opt-in is done (0 before);
  // shared by every host thread, and the same whichever thread sets it
  constexpr int kDevs = 64;
  static std::atomic<int> sms[kDevs];
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 0 || dev >= kDevs) return cudaErrorInvalidDevice;
  int nsm = sms[dev].load(std::memory_order_acquire);
  if (!nsm) {
    if ((e = cudaDeviceGetAttribute(&nsm, cudaDevAttrMultiProcessorCount, dev)) != cudaSuccess) return e;
    if ((e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem)) != cudaSuccess)
      return e;
    sms[dev].store(nsm, std::memory_order_release);
  }
  const size_t items = H * ((T + kTcRows - 1) / kTcRows);
  const unsigned grid = (unsigned)std::max<size_t>(1, std::min<size_t>(items, (size_t)nsm));
  const size_t n = H * T * R;
  const size_t ncode = MODE == 2 ? (n + 1) / 2 : n;  // bytes of the code buffer
  kern<<<grid, kTcThreads, smem, st>>>(map, codes, ncode, raw, scales, mins, axis, (int)H, (int)T, (int)R, bvt,
                                       ranks, status);
  note_launches(1);
  return cudaGetLastError();
}

}  // namespace

cudaError_t launch_reconstruct_tc(const uint8_t* codes, const float* raw, const float* scales, const float* mins,
                                  int data_type, int axis, size_t H, size_t T, size_t R, size_t D,
                                  const float* basis_vt, const uint64_t* ranks, float* out, unsigned* status,
                                  cudaStream_t st) {
  if (D != (size_t)kTcD || R == 0 || R > 64 || !aligned(out, 16) || H * T == 0 || T >= (1u << 31) ||
      H >= (1u << 31) || (codes && !aligned(codes, 4)))
    return cudaErrorNotSupported;
  CUtensorMap map{};
  if (!encode_out_map(&map, out, H, T)) return cudaErrorNotSupported;
  const int mode = raw ? 0 : (data_type == KVF_INT8 ? 1 : 2);
#define KVF_TC(M)                                                                                          \
  {                                                                                                        \
    if (R <= 8) return launch_tc<M, 2>(map, codes, raw, scales, mins, axis, H, T, R, basis_vt, ranks, status, st); \
    if (R <= 16) return launch_tc<M, 4>(map, codes, raw, scales, mins, axis, H, T, R, basis_vt, ranks, status, st); \
    if (R <= 32) return launch_tc<M, 8>(map, codes, raw, scales, mins, axis, H, T, R, basis_vt, ranks, status, st); \
    return launch_tc<M, 16>(map, codes, raw, scales, mins, axis, H, T, R, basis_vt, ranks, status, st);          \
  }
  if (mode == 0) KVF_TC(0)
  if (mode == 1) KVF_TC(1)
  KVF_TC(2)
#undef KVF_TC
}

}  // namespace kvf
