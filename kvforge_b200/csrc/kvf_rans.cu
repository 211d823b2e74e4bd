// Chunked rANS with 32 independent lane streams per chunk (sm_100a).
//
// The reference codes one serial stream with constriction's stack ANS
// (crates/kvforge-cpu/src/entropy.rs:42-123). That stream cannot be split, so
// this library defines its own container, mirrored bit for bit by the CPU
// oracle so that each side decodes the other's output:
//
//   state x in [2^16, 2^32), 16-bit renormalisation words, 13-bit model.
//   header (32 B): u32 magic "KVR2", u32 prob_bits = 13, u32 lanes = 32,
//                  u32 chunk_symbols, u64 original_len, u32 num_chunks,
//                  u32 header_bytes = 32 + 4 * (num_chunks + 1)
//   u32 chunk_offset[num_chunks + 1]: byte offset of each chunk payload from
//                  the container start; the last entry is the total length
//   chunk payload: u32 final_state[32]; u16 lane_words[32];
//                  u16 words[sum(lane_words)]: lane 0's stream, lane 1's, ...,
//                  each in decoding order; one zero u16 when the sum is odd
//
// Symbol i of a chunk belongs to lane i % 32, step i / 32, so a warp reads and
// writes 32 consecutive bytes per step. Each lane is an ordinary rANS coder
// over its own symbols with its own word stream: no lane ever waits for
// another, and a decoding lane knows the address of its next word before it
// needs it, so the only load on a state's dependency chain is the model
// lookup. The price is 64 bytes of word counts per chunk.
//
// Model: counts -> q[s] = max(1, floor(count * 2^13 / N)) for seen symbols,
// 0 for unseen; the deficit goes to the most frequent symbol, an excess is
// removed from the largest entries. Integer only, identical on both sides;
// every encode and decode block builds it from the 256 counts it is given.
//
// Every read of the decoder is bounds-checked against the container; a
// malformed container sets a status bit instead of faulting. The decoder has
// no waits; the encoder's one wait (its look-back for the payload offsets of
// lower-numbered chunks) is bounded and reports a timeout in the status word,
// so no kernel here can hang.
#include <algorithm>
#include <atomic>

#include "kvf_internal.cuh"

namespace kvf {
namespace {

constexpr int kEncWarps = 4;  // encoder: chunks per block (one per scheduler)
constexpr int kDecWarps = 4;       // decoder: chunks per block (one slot table per block, one per scheduler)
constexpr int kDecBlockWarps = 8;  // every warp builds the slot tables; the extra ones then exit
constexpr uint32_t kShift = 32 - kRansProbBits;  // a state >= q << kShift renormalises first

// cp.async helpers: asynchronous global -> shared copies, many in flight per thread
__device__ __forceinline__ void cp_async4(void* smem, const void* gmem) {
  const unsigned s = (unsigned)__cvta_generic_to_shared(smem);
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4;\n" ::"r"(s), "l"(gmem));
}
__device__ __forceinline__ void cp_async16(void* smem, const void* gmem) {
  const unsigned s = (unsigned)__cvta_generic_to_shared(smem);
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;\n" ::"r"(s), "l"(gmem));
}
__device__ __forceinline__ void cp_async_wait_all() {
  asm volatile("cp.async.commit_group;\n" ::);
  asm volatile("cp.async.wait_group 0;\n" ::: "memory");
}

// warp-wide copy of [src, src + bytes) to shared memory at dst, where dst and
// src agree modulo 16 and both are 4-byte aligned: 16-byte copies for the
// aligned body, 4-byte copies for the ends
__device__ __forceinline__ void warp_stage(uint8_t* dst, const uint8_t* src, uint32_t bytes, int lane) {
  const uint32_t head = std::min<uint32_t>((16u - (uint32_t)(reinterpret_cast<uintptr_t>(src) & 15u)) & 15u, bytes);
  const uint32_t body = (bytes - head) & ~15u;
  if ((uint32_t)lane < head / 4) cp_async4(dst + 4 * lane, src + 4 * lane);
  for (uint32_t j = 16 * lane; j < body; j += 16 * 32) cp_async16(dst + head + j, src + head + j);
  const uint32_t tail = head + body;
  for (uint32_t j = tail + 4 * lane; j < bytes; j += 4 * 32) cp_async4(dst + j, src + j);
}

// inclusive prefix sum over the 32 lanes of a warp
__device__ __forceinline__ uint32_t warp_inclusive_scan(uint32_t v, int lane) {
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const uint32_t u = __shfl_up_sync(0xffffffffu, v, o);
    if (lane >= o) v += u;
  }
  return v;
}

// The model (q, cum) built by a whole block from the 256 counts, identical to
// the CPU mirror's: q = max(1, floor(count * 2^13 / N)) for seen symbols; the
// deficit goes to the most frequent symbol (lowest index on ties); an excess
// is removed from the largest entries. Returns false (on every thread) when
// the counts admit no model. Sums and the arg-max use warp shuffles; the
// quotients come from one double reciprocal of N, corrected to the exact
// floor with integer products.
struct ModelSmem {
  unsigned long long wsum[32], wkey[32];
  uint32_t wq[32];
  int bad;
};

__device__ __forceinline__ unsigned long long warp_sum64(unsigned long long v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
__device__ __forceinline__ unsigned long long warp_max64(unsigned long long v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const unsigned long long u = __shfl_xor_sync(0xffffffffu, v, o);
    v = u > v ? u : v;
  }
  return v;
}

__device__ bool build_model(const uint32_t* __restrict__ freq, uint32_t* q, uint32_t* cum, ModelSmem& ms) {
  const int tid = threadIdx.x, nt = blockDim.x, lane = tid & 31, w = tid >> 5, nw = (nt + 31) >> 5;
  unsigned long long n = 0ull, key = 0ull;
  for (int s = tid; s < 256; s += nt) {
    const uint32_t f = freq[s];
    q[s] = f;  // counts for now
    n += f;
    const unsigned long long k = ((unsigned long long)f << 8) | (unsigned long long)(255 - s);
    key = k > key ? k : key;
  }
  n = warp_sum64(n);
  key = warp_max64(key);
  if (lane == 0) {
    ms.wsum[w] = n;
    ms.wkey[w] = key;
  }
  __syncthreads();
  unsigned long long N = 0ull, best = 0ull;
  for (int i = 0; i < nw; ++i) {
    N += ms.wsum[i];
    best = ms.wkey[i] > best ? ms.wkey[i] : best;
  }
  if (N == 0ull) return false;
  const double inv = 1.0 / (double)N;
  uint32_t ssum = 0;
  for (int s = tid; s < 256; s += nt) {
    const uint32_t f = q[s];
    uint32_t qs = 0;
    if (f) {
      // floor(t / N) for t = f * 2^13 < 2^45: the double estimate is off by at most one
      const unsigned long long t = (unsigned long long)f * kRansM;
      unsigned long long v = (unsigned long long)((double)t * inv);
      if (v * N > t) --v;
      else if ((v + 1) * N <= t) ++v;
      qs = (uint32_t)(v < 1ull ? 1ull : v);
    }
    q[s] = qs;
    ssum += qs;
  }
  ssum = (uint32_t)warp_sum64(ssum);
  if (lane == 0) ms.wq[w] = ssum;
  __syncthreads();
  if (tid == 0) {
    unsigned long long S = 0;
    for (int i = 0; i < nw; ++i) S += ms.wq[i];
    const int argmax = 255 - (int)(best & 0xFF);
    ms.bad = 0;
    if (S < kRansM) {
      q[argmax] += (uint32_t)(kRansM - S);
    } else {
      while (S > kRansM) {  // rare: many symbols lifted to 1
        int b = -1;
        for (int k = 0; k < 256; ++k)
          if (q[k] > 1 && (b < 0 || q[k] > q[b])) b = k;
        if (b < 0) { ms.bad = 1; break; }
        unsigned long long d = S - kRansM;
        if (d > q[b] - 1) d = q[b] - 1;
        q[b] -= (uint32_t)d;
        S -= d;
      }
    }
  }
  __syncthreads();
  if (ms.bad) return false;
  if (tid < 32) {  // exclusive prefix over 256 entries: 8 per lane
    uint32_t loc[8], sum = 0;
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      loc[k] = sum;
      sum += q[8 * tid + k];
    }
    const uint32_t base = warp_inclusive_scan(sum, tid) - sum;
#pragma unroll
    for (int k = 0; k < 8; ++k) cum[8 * tid + k] = base + loc[k];
  }
  __syncthreads();
  return true;
}

// Encoder shared memory per warp: the chunk's symbols, then one word region
// per lane. A region holds at least one word per step; its length is an odd
// number of 4-byte words so that lanes writing at equal positions fall in
// different banks.
__host__ __device__ inline uint32_t enc_region_words(uint32_t chunk) {
  uint32_t m = (chunk / kRansLanes + 1) / 2;
  if ((m & 1u) == 0) ++m;
  return 2 * m;
}
__host__ __device__ inline size_t enc_warp_smem(uint32_t chunk) {
  return (size_t)chunk + 2 * (size_t)kRansLanes * enc_region_words(chunk);
}

// Chunk offsets come from a decoupled look-back over one status word per
// chunk (zeroed before the launch): flag in the top two bits (1: the chunk's
// payload size, 2: the inclusive prefix of payload sizes), value below. A warp
// publishes its size, then reads its predecessors' words 32 at a time, adding
// sizes back to the nearest published prefix. A block takes its chunks from
// a ticket counter (one more zeroed word after the status words) when it
// starts, so the predecessors of a chunk belong to the same block or to a
// block that started earlier and is running or done: the wait ends whatever
// order the hardware dispatches blocks in. It is bounded all the same, and a
// warp that gives up reports a device timeout instead of writing.
constexpr unsigned long long kLbSize = 1ull << 62, kLbPrefix = 2ull << 62, kLbValue = (1ull << 62) - 1;
constexpr uint32_t kLbSpinLimit = 1u << 16;

__device__ __forceinline__ unsigned long long ld_acquire(const unsigned long long* p) {
  unsigned long long v;
  asm volatile("ld.acquire.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void st_release(unsigned long long* p, unsigned long long v) {
  asm volatile("st.release.gpu.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}

// bytes of the payloads before chunk c (c > 0); false when the wait gave up
// (kLbSpinLimit polls of one window, or limit_ns in all)
__device__ bool look_back(unsigned long long* lb, uint64_t c, unsigned* status, int lane,
                          unsigned long long& prefix, unsigned long long limit_ns = kWaitNs) {
  prefix = 0ull;
  int64_t top = (int64_t)c - 1;
  uint32_t spins = 0;
  const unsigned long long t0 = dev_ns();
  while (true) {
    const int64_t idx = top - lane;
    const unsigned long long v = idx >= 0 ? ld_acquire(lb + idx) : kLbPrefix;  // before chunk 0: prefix 0
    const unsigned flag = (unsigned)(v >> 62);
    const unsigned pre = __ballot_sync(0xffffffffu, flag == 2u);
    const unsigned empty = __ballot_sync(0xffffffffu, flag == 0u);
    const int pl = pre ? __ffs(pre) - 1 : 31;  // the window ends at the nearest prefix
    const unsigned used = pl == 31 ? 0xffffffffu : ((2u << pl) - 1u);
    if (empty & used) {  // a predecessor has not published yet
      // every lane takes the same branch: the clock and the status word are
      // read per lane, so the decision is a vote
      const bool give_up = ++spins > kLbSpinLimit || dev_ns() - t0 > limit_ns ||
                           (*reinterpret_cast<volatile unsigned*>(status) & kDevErrTimeout);
      if (__any_sync(0xffffffffu, give_up)) return false;
      __nanosleep(64);
      continue;
    }
    prefix += warp_sum64((unsigned)lane <= (unsigned)pl ? (v & kLbValue) : 0ull);
    if (pre) return true;
    top -= 32;
    spins = 0;
  }
}

// One warp per chunk, one lane stream per thread. The chunk's symbols are
// staged in shared memory; each lane encodes its steps from last to first,
// writing renormalisation words backwards into its region. The warp then
// finds its payload's offset by look-back and writes the payload (states,
// counts, lane streams one after another) straight into the container; the
// last chunk writes the container header and length.
__global__ void __launch_bounds__(kEncWarps * 32) k_rans_encode(const uint8_t* __restrict__ data,
                                                               uint64_t n, uint32_t chunk,
                                                               const uint32_t* __restrict__ freq,
                                                               unsigned long long* __restrict__ lb,
                                                               uint8_t* __restrict__ out,
                                                               uint64_t* __restrict__ out_len,
                                                               uint64_t nchunks,
                                                               unsigned* __restrict__ status) {
  extern __shared__ __align__(16) uint8_t sbuf[];
  __shared__ uint32_t q[256], cum[256];
  __shared__ uint4 mdl[256];  // per symbol: {threshold - 1, reciprocal, q, (M - q) | cum << 16}
  __shared__ ModelSmem ms;
  __shared__ unsigned long long ticket;
  const int w = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) ticket = atomicAdd(lb + nchunks, 1ull);  // blocks in the order they started
  __syncthreads();
  const uint64_t c = (uint64_t)ticket * kEncWarps + w;
  const bool live = c < nchunks;
  const uint64_t start = live ? c * chunk : 0;
  const uint32_t nsym = live ? (uint32_t)((n - start < chunk) ? (n - start) : chunk) : 0;
  uint8_t* buf = sbuf + (size_t)w * enc_warp_smem(chunk);
  const uint32_t RS = enc_region_words(chunk);
  uint16_t* words = reinterpret_cast<uint16_t*>(buf + chunk);  // this warp's regions
  uint16_t* region = words + (size_t)lane * RS;
  if (live) {
    const bool vec = (reinterpret_cast<uintptr_t>(data + start) & 15u) == 0;
    const uint32_t n16 = vec ? nsym / 16 : 0;
    for (uint32_t j = lane; j < n16; j += 32) cp_async16(buf + 16 * j, data + start + 16 * j);
    for (uint32_t j = 16 * n16 + lane; j < nsym; j += 32) buf[j] = data[start + j];
  }
  // the model is built while the symbols are in flight
  const bool model_ok = build_model(freq, q, cum, ms);
  for (int i = threadIdx.x; i < 256; i += blockDim.x) {
    // a state renormalises first when x >= q << kShift, i.e. x > thr; q = 2^13
    // (one symbol takes the whole model) never renormalises
    const uint64_t t = ((uint64_t)q[i] << kShift) - 1ull;
    const uint32_t thr = q[i] ? (uint32_t)(t > 0xFFFFFFFFull ? 0xFFFFFFFFull : t) : 0u;
    mdl[i] = make_uint4(thr, q[i] ? 0xFFFFFFFFu / q[i] : 0u, q[i], (kRansM - q[i]) | (cum[i] << 16));
  }
  cp_async_wait_all();
  __syncthreads();
  if (!model_ok) {
    if (threadIdx.x == 0) atomicOr(status, kDevErrEntropy);
    return;
  }
  if (!live) return;

  uint32_t x = kRansL, pos = RS;
  // renormalise (at most one word), then x -> (x / f) * M + x % f + cum,
  // written as floor(xs / f) * (M - f) + xs + cum. The quotient estimate
  // umulhi(xs, floor((2^32 - 1) / f)) is low by at most one; both candidate
  // states are formed and the remainder test picks one, so the state's
  // dependency chain is compare, select, multiply-high, multiply-add, compare,
  // select.
  auto step = [&](const uint4& m) {
    const uint32_t f = m.z, mf = m.w & 0xFFFFu, cm = m.w >> 16;
    const bool need = x > m.x;
    if (need) region[pos - 1] = (uint16_t)(x & 0xFFFFu);
    pos -= need ? 1u : 0u;
    const uint32_t xs = need ? (x >> 16) : x;
    const uint32_t qq = __umulhi(xs, m.y);
    const uint32_t xa = qq * mf + xs + cm;
    x = (xs - qq * f >= f) ? xa + mf : xa;
  };
  const uint32_t steps = (nsym + 31) / 32;
  {  // last (possibly partial) step
    const uint32_t i = (steps - 1) * 32 + lane;
    if (i < nsym) step(mdl[buf[i]]);
  }
  // full steps, from steps - 2 down to 0, four at a time: each of the four
  // model entries in registers is used, then reloaded for the step four
  // further on, so every lookup is issued four steps before the chain needs it
  auto entry = [&](int t) { return mdl[buf[(t > 0 ? t : 0) * 32 + lane]]; };
  int t = (int)steps - 2;
  uint4 m0 = entry(t), m1 = entry(t - 1), m2 = entry(t - 2), m3 = entry(t - 3);
  for (; t >= 3; t -= 4) {
    step(m0);
    m0 = entry(t - 4);
    step(m1);
    m1 = entry(t - 5);
    step(m2);
    m2 = entry(t - 6);
    step(m3);
    m3 = entry(t - 7);
  }
  if (t >= 0) step(m0);
  if (t >= 1) step(m1);
  if (t >= 2) step(m2);

  // payload layout: lane streams one after another, in decoding order; the
  // warp copies one lane's stream at a time with coalesced 2-byte stores
  const uint32_t cnt = RS - pos;
  const uint32_t incl = warp_inclusive_scan(cnt, lane);
  const uint32_t total = __shfl_sync(0xffffffffu, incl, 31);
  const unsigned long long pbytes = kRansPayloadHeader + 2ull * total + 2ull * (total & 1u);
  unsigned long long prefix = 0ull;
  if (c == 0) {
    if (lane == 0) st_release(lb, kLbPrefix | pbytes);
  } else {
    if (lane == 0) st_release(lb + c, kLbSize | pbytes);
    if (!look_back(lb, c, status, lane, prefix)) {
      if (lane == 0) atomicOr(status, kDevErrTimeout);
      return;
    }
    if (lane == 0) st_release(lb + c, kLbPrefix | (prefix + pbytes));
  }
  const uint64_t hdr = kRansHeader + 4ull * (nchunks + 1);
  const uint64_t off = hdr + prefix;
  uint32_t* offs = reinterpret_cast<uint32_t*>(out + kRansHeader);
  uint8_t* pay = out + off;
  reinterpret_cast<uint32_t*>(pay)[lane] = x;
  reinterpret_cast<uint16_t*>(pay + 4 * kRansLanes)[lane] = (uint16_t)cnt;
  uint16_t* dstw = reinterpret_cast<uint16_t*>(pay + kRansPayloadHeader);
  for (int l = 0; l < 32; ++l) {
    const uint32_t cl = __shfl_sync(0xffffffffu, cnt, l);
    const uint32_t el = __shfl_sync(0xffffffffu, incl, l) - cl;
    const uint16_t* src = words + (size_t)l * RS + (RS - cl);
    for (uint32_t j0 = lane; j0 < cl; j0 += 8 * 32) {  // eight loads in flight per lane
      uint16_t v[8];
#pragma unroll
      for (int k = 0; k < 8; ++k) v[k] = (j0 + 32 * k < cl) ? src[j0 + 32 * k] : (uint16_t)0;
#pragma unroll
      for (int k = 0; k < 8; ++k)
        if (j0 + 32 * k < cl) dstw[el + j0 + 32 * k] = v[k];
    }
  }
  if (lane == 0) {
    if (total & 1u) dstw[total] = 0;
    offs[c] = (uint32_t)off;
    if (c == nchunks - 1) {
      const uint64_t len = off + pbytes;
      offs[nchunks] = (uint32_t)len;
      *out_len = len;
      uint32_t* h = reinterpret_cast<uint32_t*>(out);
      h[0] = kRansMagic;
      h[1] = kRansProbBits;
      h[2] = kRansLanes;
      h[3] = chunk;
      h[4] = (uint32_t)(n & 0xFFFFFFFFull);
      h[5] = (uint32_t)(n >> 32);
      h[6] = (uint32_t)nchunks;
      h[7] = (uint32_t)hdr;
    }
  }
}

__device__ __forceinline__ uint32_t rd32(const uint8_t* p) {
  return (uint32_t)p[0] | ((uint32_t)p[1] << 8) | ((uint32_t)p[2] << 16) | ((uint32_t)p[3] << 24);
}

// Decodes one chunk whose payload (pay_bytes at pay, 4-byte aligned, already
// checked to be at least the payload header) sits in shared or global memory.
// Lane l reads its own stream; its next word is loaded one step before it can
// be needed, at an index clamped to the lane's stream, so a corrupt count
// reads nothing outside the payload. Returns true when the chunk is malformed.
template <bool FULL_ONLY>
__device__ __forceinline__ bool decode_chunk(const uint8_t* pay, uint32_t pay_bytes, const uint2* ent,
                                             const uint8_t* sym, uint32_t nsym, uint8_t* __restrict__ o,
                                             int lane) {
  uint32_t x = reinterpret_cast<const uint32_t*>(pay)[lane];
  const uint32_t cnt = reinterpret_cast<const uint16_t*>(pay + 4 * kRansLanes)[lane];
  const uint32_t incl = warp_inclusive_scan(cnt, lane);
  const uint32_t total = __shfl_sync(0xffffffffu, incl, 31);
  if ((uint32_t)kRansPayloadHeader + 2u * total + 2u * (total & 1u) != pay_bytes) return true;
  bool bad = x < kRansL;
  // this lane's stream; a lane without words points at the payload start,
  // whose words it reads but never uses unless the chunk is corrupt
  const uint16_t* wl = cnt ? reinterpret_cast<const uint16_t*>(pay + kRansPayloadHeader) + (incl - cnt)
                           : reinterpret_cast<const uint16_t*>(pay);
  const uint32_t last = cnt ? cnt - 1 : 0;
  uint32_t k = 0;
  uint32_t wn = wl[0];
  const uint32_t full = nsym / 32;
#pragma unroll 4
  for (uint32_t st = 0; st < full; ++st) {
    // chain: mask, one 8-byte lookup, multiply-add, then compare and a byte
    // permute ((x << 16) | word) side by side, select
    const uint32_t slot = x & (kRansM - 1);
    const uint2 e = ent[slot];
    o[32 * st] = sym[slot];
    x = e.x * (x >> kRansProbBits) + e.y;
    const bool need = x < kRansL;
    x = need ? __byte_perm(wn, x, 0x5410) : x;
    k += need ? 1u : 0u;
    wn = wl[min(k, last)];
  }
  if (!FULL_ONLY && full * 32 < nsym) {  // last, partial step
    if (full * 32 + lane < nsym) {
      const uint32_t slot = x & (kRansM - 1);
      const uint2 e = ent[slot];
      o[32 * full] = sym[slot];
      x = e.x * (x >> kRansProbBits) + e.y;
      if (x < kRansL) {
        x = (x << 16) | wn;
        ++k;
      }
    }
  }
  bad = bad || x != kRansL || k != cnt;
  return __any_sync(0xffffffffu, bad);
}

// Decoder shared memory: the slot tables ent[slot] = {q, slot - cum} and
// sym[slot], then one staging buffer per warp holding a chunk payload of the
// default chunk size (with 16 bytes of alignment slack); payloads of larger
// chunks are read from global memory in place.
constexpr uint32_t kDecStageBytes = (uint32_t)kRansPayloadHeader + 2u * kRansChunk + 32u;
constexpr size_t kDecTableBytes = 9 * (size_t)kRansM;  // ent (8 B) + sym (1 B) per slot
constexpr size_t kDecSmem = kDecTableBytes + (size_t)kDecWarps * kDecStageBytes;

__global__ void __launch_bounds__(kDecBlockWarps * 32) k_rans_decode(const uint8_t* __restrict__ comp,
                                                              uint64_t comp_len_host,
                                                              const uint64_t* __restrict__ comp_len_dev,
                                                              const uint32_t* __restrict__ freq,
                                                              uint64_t n, uint8_t* __restrict__ out,
                                                              unsigned* __restrict__ status) {
  extern __shared__ __align__(16) uint8_t dsm[];
  uint2* ent = reinterpret_cast<uint2*>(dsm);  // [2^13]
  uint8_t* sym = dsm + 8 * kRansM;             // [2^13]
  __shared__ uint32_t q[256], cum[256];
  __shared__ ModelSmem ms;
  const int w = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (!build_model(freq, q, cum, ms)) {
    if (threadIdx.x == 0) atomicOr(status, kDevErrEntropy);
    return;
  }
  {  // slot tables: mark the first slot of every coded symbol in sym[], then
     // each warp turns a contiguous span of marks into both tables, a lane
     // taking four consecutive slots per round (one 4-byte mark word in,
     // two 16-byte ent stores and one 4-byte sym store out); the symbol of a
     // slot is the last mark at or before it
    for (uint32_t i = threadIdx.x; i < kRansM / 16; i += blockDim.x)
      reinterpret_cast<uint4*>(sym)[i] = make_uint4(0, 0, 0, 0);
    __syncthreads();
    for (int s = threadIdx.x; s < 256; s += blockDim.x)
      if (q[s]) sym[cum[s]] = (uint8_t)s;
    __syncthreads();
    const uint32_t span = kRansM / (blockDim.x >> 5), lo_k = (uint32_t)w * span;
    int lo = 0, hi = 255;  // symbol of the span's first slot: the last s with cum[s] <= lo_k
    while (lo < hi) {
      const int mid = (lo + hi + 1) >> 1;
      if (cum[mid] <= lo_k) lo = mid; else hi = mid - 1;
    }
    uint32_t carry = (uint32_t)lo;
    const unsigned below = (1u << lane) - 1u;
    for (uint32_t k0 = lo_k; k0 < lo_k + span; k0 += 128) {
      const uint32_t k = k0 + 4 * lane;
      const uint32_t m4 = *reinterpret_cast<const uint32_t*>(sym + k);
      // the last mark among this lane's four slots (marks increase with the slot)
      const uint32_t mlast = (m4 >> 24) ? (m4 >> 24) : (m4 >> 16) & 0xFFu ? (m4 >> 16) & 0xFFu
                           : (m4 >> 8) & 0xFFu ? (m4 >> 8) & 0xFFu : m4 & 0xFFu;
      const unsigned has = __ballot_sync(0xffffffffu, m4 != 0u);
      const unsigned prev = has & below;
      const uint32_t from = __shfl_sync(0xffffffffu, mlast, prev ? 31 - __clz(prev) : 0);
      uint32_t v = prev ? from : carry;
      uint32_t e[4], sw = 0;
#pragma unroll
      for (int b = 0; b < 4; ++b) {
        const uint32_t mb = (m4 >> (8 * b)) & 0xFFu;
        v = mb ? mb : v;
        e[b] = v;
        sw |= v << (8 * b);
      }
      carry = __shfl_sync(0xffffffffu, v, 31);
      uint4* ep = reinterpret_cast<uint4*>(ent + k);
      ep[0] = make_uint4(q[e[0]], k - cum[e[0]], q[e[1]], k + 1 - cum[e[1]]);
      ep[1] = make_uint4(q[e[2]], k + 2 - cum[e[2]], q[e[3]], k + 3 - cum[e[3]]);
      *reinterpret_cast<uint32_t*>(sym + k) = sw;
    }
  }
  __syncthreads();
  if (w >= kDecWarps) return;
  uint8_t* stage = dsm + kDecTableBytes + (size_t)w * kDecStageBytes;
  const uint64_t comp_len = comp_len_dev ? *comp_len_dev : comp_len_host;
  // header checks (every warp reads the same 32 bytes)
  if (comp_len < kRansHeader) { if (threadIdx.x == 0) atomicOr(status, kDevErrCorrupt); return; }
  const uint32_t chunk = rd32(comp + 12);
  const uint64_t nn = (uint64_t)rd32(comp + 16) | ((uint64_t)rd32(comp + 20) << 32);
  const uint64_t nchunks = rd32(comp + 24);
  const uint64_t hdr = kRansHeader + 4ull * (nchunks + 1);
  const bool hdr_ok = rd32(comp) == kRansMagic && rd32(comp + 4) == kRansProbBits &&
                      rd32(comp + 8) == kRansLanes && chunk != 0 && (chunk % 32) == 0 &&
                      chunk <= kRansMaxChunk && nn == n && nchunks == (n + chunk - 1) / chunk &&
                      rd32(comp + 28) == hdr && hdr <= comp_len &&
                      rd32(comp + kRansHeader + 4 * nchunks) == comp_len;
  if (!hdr_ok) { if (threadIdx.x == 0) atomicOr(status, kDevErrCorrupt); return; }
  const uint64_t nwarps = (uint64_t)gridDim.x * kDecWarps;
  for (uint64_t c = (uint64_t)blockIdx.x * kDecWarps + w; c < nchunks; c += nwarps) {
    const uint64_t off = rd32(comp + kRansHeader + 4 * c);
    const uint64_t end = rd32(comp + kRansHeader + 4 * (c + 1));
    if (off < hdr || end > comp_len || end < off + kRansPayloadHeader || ((off | end) & 3u)) {
      if (lane == 0) atomicOr(status, kDevErrCorrupt);
      continue;
    }
    const uint32_t pay_bytes = (uint32_t)(end - off);
    const uint64_t start = c * chunk;
    const uint32_t nsym = (uint32_t)((n - start < chunk) ? (n - start) : chunk);
    uint8_t* o = out + start + lane;
    const uint32_t mis = (uint32_t)(reinterpret_cast<uintptr_t>(comp + off) & 15u);
    bool bad;
    if (mis + pay_bytes <= kDecStageBytes) {
      __syncwarp();  // the previous chunk's reads of the staging buffer are done
      warp_stage(stage + mis, comp + off, pay_bytes, lane);
      cp_async_wait_all();
      __syncwarp();
      bad = (nsym % 32 == 0) ? decode_chunk<true>(stage + mis, pay_bytes, ent, sym, nsym, o, lane)
                             : decode_chunk<false>(stage + mis, pay_bytes, ent, sym, nsym, o, lane);
    } else {
      bad = decode_chunk<false>(comp + off, pay_bytes, ent, sym, nsym, o, lane);
    }
    if (bad && lane == 0) atomicOr(status, kDevErrCorrupt);
  }
}

}  // namespace

namespace {
// dynamic shared memory above the default, opted in once per (kernel, device)
// for the largest size asked so far (the attribute is per device)
constexpr int kOptDevs = 64;
std::atomic<int> enc_opted[kOptDevs], dec_opted[kOptDevs];
template <typename K>
cudaError_t opt_in_smem(K kern, std::atomic<int>* opted, int bytes) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 0 || dev >= kOptDevs) return cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
  if (bytes <= opted[dev].load(std::memory_order_acquire)) return cudaSuccess;
  e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
  if (e == cudaSuccess) {
    int cur = opted[dev].load(std::memory_order_relaxed);
    while (cur < bytes && !opted[dev].compare_exchange_weak(cur, bytes, std::memory_order_acq_rel)) {
    }
  }
  return e;
}
}  // namespace

cudaError_t launch_rans_encode(const uint8_t* data, size_t n, uint32_t chunk, const uint32_t* freq,
                               unsigned long long* lookback, uint8_t* out, uint64_t* out_len, unsigned* status,
                               cudaStream_t st) {
  if (n == 0) return cudaSuccess;
  if (chunk == 0 || chunk % kRansLanes || chunk > kRansMaxChunk) return cudaErrorInvalidValue;
  if (!aligned(out, 4)) return cudaErrorInvalidValue;
  const size_t nc = rans_num_chunks(n, chunk);
  const size_t smem = (size_t)kEncWarps * enc_warp_smem(chunk);
  if (smem > kSmemOptIn) {
    const cudaError_t e = opt_in_smem(k_rans_encode, enc_opted, (int)smem);
    if (e != cudaSuccess) return e;
  }
  cudaError_t e = cudaMemsetAsync(lookback, 0, (nc + 1) * sizeof(unsigned long long), st);  // + the ticket
  if (e != cudaSuccess) return e;
  const unsigned grid = (unsigned)((nc + kEncWarps - 1) / kEncWarps);
  k_rans_encode<<<grid, kEncWarps * 32, smem, st>>>(data, n, chunk, freq, lookback, out, out_len, nc, status);
  note_launches(1);
  return cudaGetLastError();
}

cudaError_t launch_rans_decode(const uint8_t* comp, size_t comp_len, const uint64_t* comp_len_dev,
                               const uint32_t* freq, size_t n, uint8_t* out, unsigned* status,
                               cudaStream_t st) {
  if (n == 0) return cudaSuccess;
  if (!aligned(comp, 4)) return cudaErrorInvalidValue;  // payloads are read as 4-byte words
  // the grid is sized for the encoder's default chunk size; warps loop over
  // chunks, so a container with any chunk size named in its header decodes
  const size_t nc = rans_num_chunks(n, kRansChunk);
  const unsigned grid = (unsigned)((nc + kDecWarps - 1) / kDecWarps);
  const cudaError_t e = opt_in_smem(k_rans_decode, dec_opted, (int)kDecSmem);
  if (e != cudaSuccess) return e;
  k_rans_decode<<<grid, kDecBlockWarps * 32, kDecSmem, st>>>(comp, comp_len, comp_len_dev, freq, n, out, status);
  note_launches(1);
  return cudaGetLastError();
}
namespace {
// chunk 1 looks back at chunk 0, whose status word nothing publishes
__global__ void k_selftest_lookback(unsigned long long* lb, unsigned* status, unsigned long long limit_ns) {
  unsigned long long prefix;
  const bool ok = look_back(lb, 1, status, threadIdx.x & 31, prefix, limit_ns);
  if (!ok && threadIdx.x == 0 && status) atomicOr(status, kDevErrTimeout);
}
}  // namespace

cudaError_t launch_selftest_lookback(unsigned long long* lb, unsigned* status, unsigned long long limit_ns,
                                     cudaStream_t st) {
  cudaError_t e = cudaMemsetAsync(lb, 0, 2 * sizeof(unsigned long long), st);
  if (e != cudaSuccess) return e;
  k_selftest_lookback<<<1, 32, 0, st>>>(lb, status, limit_ns);
  note_launches(1);
  return cudaGetLastError();
}

}  // namespace kvf
