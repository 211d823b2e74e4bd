// Chunked, 32-lane interleaved rANS (sm_100a).
//
// The reference codes one serial stream with constriction's stack ANS
// (crates/kvforge-cpu/src/entropy.rs:42-123). That stream cannot be split, so
// this library defines its own container, mirrored bit for bit by the CPU
// oracle so that each side decodes the other's output:
//
//   state x in [2^16, 2^32), 16-bit renormalisation words, 15-bit model.
//   header (32 B): u32 magic "KVR1", u32 prob_bits = 15, u32 lanes = 32,
//                  u32 chunk_symbols, u64 original_len, u32 num_chunks,
//                  u32 header_bytes = 32 + 4 * (num_chunks + 1)
//   u32 chunk_offset[num_chunks + 1]: byte offset of each chunk payload from
//                  the container start; the last entry is the total length
//   chunk payload: u32 nwords; u32 final_state[32]; u16 words[nwords];
//                  one zero u16 when nwords is odd (4-byte alignment)
//
// One warp codes one chunk; symbol i of a chunk belongs to lane i % 32, step
// i / 32. The encoder runs steps backwards; in each step the active lanes
// renormalise (emitters ordered by descending lane, found with a ballot) and
// then encode. The decoder runs steps forwards and serves consuming lanes in
// ascending order, so it reads the word array front to back.
//
// Model: counts -> q[s] = max(1, floor(count * 2^15 / N)) for seen symbols,
// 0 for unseen; the deficit goes to the most frequent symbol, an excess is
// removed from the largest entries. Integer only, identical on both sides;
// every encode and decode block builds it from the 256 counts it is given.
//
// Every read of the decoder is bounds-checked against the container; a
// malformed container sets a status bit instead of faulting, and there are no
// waits, so no kernel here can hang.
#include <algorithm>

#include "kvf_internal.cuh"

namespace kvf {
namespace {

constexpr int kWarpsPerBlock = 4;  // encoder: chunks per block
constexpr int kDecWarps = 2;       // decoder: chunks per block

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

// exclusive prefix sum of one value per thread over a block of blockDim.x threads
template <typename T>
__device__ __forceinline__ T block_exclusive_scan(T v, T* warp_tot, T* total) {
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5, nw = (blockDim.x + 31) >> 5;
  T incl = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const T u = __shfl_up_sync(0xffffffffu, incl, o);
    if (lane >= o) incl += u;
  }
  if (lane == 31) warp_tot[w] = incl;
  __syncthreads();
  if (w == 0) {
    T t = (lane < nw) ? warp_tot[lane] : T(0);
    T ti = t;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const T u = __shfl_up_sync(0xffffffffu, ti, o);
      if (lane >= o) ti += u;
    }
    if (lane < nw) warp_tot[lane] = ti - t;
    if (lane == nw - 1) *total = ti;
  }
  __syncthreads();
  return warp_tot[w] + incl - v;
}

// The model (q, cum) built by a whole block from the 256 counts, identical to
// the CPU mirror's: q = max(1, floor(count * 2^15 / N)) for
// seen symbols; the deficit goes to the most frequent symbol (lowest index on
// ties); an excess is removed from the largest entries. Returns false (on
// every thread) when the counts admit no model.
struct ModelSmem {
  unsigned long long N, best;
  uint32_t S;
  int bad;
};

__device__ bool build_model(const uint32_t* __restrict__ freq, uint32_t* q, uint32_t* cum, ModelSmem& ms) {
  const int tid = threadIdx.x, nt = blockDim.x;
  if (tid == 0) {
    ms.N = 0ull;
    ms.best = 0ull;
    ms.S = 0u;
    ms.bad = 0;
  }
  __syncthreads();
  unsigned long long n = 0ull, key = 0ull;
  for (int s = tid; s < 256; s += nt) {
    const uint32_t f = freq[s];
    q[s] = f;  // counts for now
    n += f;
    const unsigned long long k = ((unsigned long long)f << 8) | (unsigned long long)(255 - s);
    key = k > key ? k : key;
  }
  atomicAdd(&ms.N, n);
  atomicMax(&ms.best, key);
  __syncthreads();
  const unsigned long long N = ms.N;
  if (N == 0ull) return false;
  uint32_t ssum = 0;
  for (int s = tid; s < 256; s += nt) {
    const uint32_t f = q[s];
    uint32_t qs = 0;
    if (f) {
      const unsigned long long v = ((unsigned long long)f * kRansM) / N;
      qs = (uint32_t)(v < 1ull ? 1ull : v);
    }
    q[s] = qs;
    ssum += qs;
  }
  atomicAdd(&ms.S, ssum);
  __syncthreads();
  if (tid == 0) {
    unsigned long long S = ms.S;
    const int argmax = 255 - (int)(ms.best & 0xFF);
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
    uint32_t incl = sum;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const uint32_t u = __shfl_up_sync(0xffffffffu, incl, o);
      if (tid >= o) incl += u;
    }
    const uint32_t base = incl - sum;
#pragma unroll
    for (int k = 0; k < 8; ++k) cum[8 * tid + k] = base + loc[k];
  }
  __syncthreads();
  return true;
}

// One warp per chunk. The chunk's symbols are staged in shared memory with
// asynchronous copies; the loop is software-pipelined so that the next step's
// symbol and model entries are loaded while the current state is updated.
__global__ void __launch_bounds__(kWarpsPerBlock * 32) k_rans_encode(const uint8_t* __restrict__ data,
                                                                   uint64_t n, uint32_t chunk,
                                                                   const uint32_t* __restrict__ freq,
                                                                   uint8_t* __restrict__ slots,
                                                                   uint64_t nchunks,
                                                                   unsigned* __restrict__ status) {
  extern __shared__ __align__(16) uint8_t sbuf[];  // [warps][chunk]
  __shared__ uint32_t q[256], cum[256], rcp[256];
  __shared__ ModelSmem ms;
  const int w = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint64_t c = (uint64_t)blockIdx.x * kWarpsPerBlock + w;
  const bool live = c < nchunks;
  const uint64_t start = live ? c * chunk : 0;
  const uint32_t nsym = live ? (uint32_t)((n - start < chunk) ? (n - start) : chunk) : 0;
  uint8_t* buf = sbuf + (size_t)w * chunk;
  if (live) {
    const bool vec = (reinterpret_cast<uintptr_t>(data + start) & 15u) == 0;
    const uint32_t n16 = vec ? nsym / 16 : 0;
    for (uint32_t j = lane; j < n16; j += 32) cp_async16(buf + 16 * j, data + start + 16 * j);
    for (uint32_t j = 16 * n16 + lane; j < nsym; j += 32) buf[j] = data[start + j];
  }
  // the model is built while the symbols are in flight
  const bool model_ok = build_model(freq, q, cum, ms);
  for (int i = threadIdx.x; i < 256; i += blockDim.x) rcp[i] = q[i] ? 0xFFFFFFFFu / q[i] : 0u;
  cp_async_wait_all();
  __syncthreads();
  if (!model_ok) {
    if (threadIdx.x == 0) atomicOr(status, kDevErrEntropy);
    return;
  }
  if (!live) return;

  uint8_t* slot = slots + c * rans_slot_bytes(chunk);
  uint16_t* words = reinterpret_cast<uint16_t*>(slot + kRansChunkHeader);
  const uint32_t capw = chunk + 2;
  uint32_t pos = capw;  // words are written backwards, ending at capw
  uint32_t x = kRansL;
  const uint32_t steps = (nsym + 31) / 32;
  const unsigned above_mask = ~((2u << lane) - 1u);  // emitting lanes above this one
  // one encoding step for a lane holding symbol entry (f, cu, rc); `act`
  // false leaves the state alone (only the last step can be partial)
  auto step = [&](bool act, uint32_t f, uint32_t cu, uint32_t rc) {
    const bool need = act && (x >> 17) >= f;  // x >= f * 2^17
    const unsigned mask = __ballot_sync(0xffffffffu, need);
    if (need) words[pos - 1 - __popc(mask & above_mask)] = (uint16_t)(x & 0xFFFFu);
    pos -= __popc(mask);
    const uint32_t xs = need ? (x >> 16) : x;
    uint32_t qq = __umulhi(xs, rc);
    uint32_t r = xs - qq * f;
    const bool fix = r >= f;
    qq += fix ? 1u : 0u;
    r -= fix ? f : 0u;
    x = act ? (qq << kRansProbBits) + r + cu : x;
  };
  // last (possibly partial) step
  {
    const uint32_t i = (steps - 1) * 32 + lane;
    const bool act = i < nsym;
    const uint32_t s = act ? buf[i] : 0u;
    step(act, q[s], cum[s], rcp[s]);
  }
  // full steps, software-pipelined: the next step's model entries load while
  // the current state updates
  if (steps >= 2) {
    uint32_t s = buf[(steps - 2) * 32 + lane];
    uint32_t f = q[s], cu = cum[s], rc = rcp[s];
    for (uint32_t st = steps - 1; st-- > 0;) {
      const uint32_t f0 = f, c0 = cu, r0 = rc;
      if (st > 0) {
        s = buf[(st - 1) * 32 + lane];
        f = q[s];
        cu = cum[s];
        rc = rcp[s];
      }
      step(true, f0, c0, r0);
    }
  }
  uint32_t* hdr = reinterpret_cast<uint32_t*>(slot);
  hdr[1 + lane] = x;
  if (lane == 0) hdr[0] = capw - pos;
}

// header + offsets: one block scans the chunk payload sizes
__global__ void __launch_bounds__(1024) k_rans_offsets(const uint8_t* __restrict__ slots, uint64_t n,
                                                       uint32_t chunk, uint64_t nchunks,
                                                       uint8_t* __restrict__ out,
                                                       uint64_t* __restrict__ out_len) {
  __shared__ unsigned long long wtot[32], total;
  const uint64_t per = (nchunks + blockDim.x - 1) / blockDim.x;
  const uint64_t c0 = threadIdx.x * per;
  const uint64_t c1 = (c0 + per < nchunks) ? c0 + per : nchunks;
  const size_t sb = rans_slot_bytes(chunk);
  unsigned long long local = 0;
  for (uint64_t c = c0; c < c1; ++c) {
    const uint32_t nw = *reinterpret_cast<const uint32_t*>(slots + c * sb);
    local += kRansChunkHeader + 2ull * nw + 2ull * (nw & 1u);
  }
  const unsigned long long excl = block_exclusive_scan<unsigned long long>(local, wtot, &total);
  const uint64_t hdr = kRansHeader + 4ull * (nchunks + 1);
  uint32_t* off = reinterpret_cast<uint32_t*>(out + kRansHeader);
  uint64_t run = hdr + excl;
  for (uint64_t c = c0; c < c1; ++c) {
    off[c] = (uint32_t)run;
    const uint32_t nw = *reinterpret_cast<const uint32_t*>(slots + c * sb);
    run += kRansChunkHeader + 2ull * nw + 2ull * (nw & 1u);
  }
  if (threadIdx.x == 0) {
    const uint64_t len = hdr + total;
    off[nchunks] = (uint32_t)len;
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

// one block per chunk: copy nwords, states and words into place
__global__ void __launch_bounds__(256) k_rans_compact(const uint8_t* __restrict__ slots, uint32_t chunk,
                                                      uint8_t* __restrict__ out) {
  const uint64_t c = blockIdx.x;
  const uint8_t* slot = slots + c * rans_slot_bytes(chunk);
  const uint32_t* off = reinterpret_cast<const uint32_t*>(out + kRansHeader);
  uint8_t* dst = out + off[c];
  const uint32_t* shdr = reinterpret_cast<const uint32_t*>(slot);
  const uint32_t nw = shdr[0];
  uint32_t* dhdr = reinterpret_cast<uint32_t*>(dst);
  for (int i = threadIdx.x; i < 1 + (int)kRansLanes; i += blockDim.x) dhdr[i] = shdr[i];
  const uint16_t* sw = reinterpret_cast<const uint16_t*>(slot + kRansChunkHeader) + (chunk + 2 - nw);
  uint16_t* dw = reinterpret_cast<uint16_t*>(dst + kRansChunkHeader);
  // eight independent loads in flight per thread
  for (uint32_t i0 = threadIdx.x; i0 < nw; i0 += blockDim.x * 8) {
    uint16_t v[8];
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      const uint32_t i = i0 + k * blockDim.x;
      v[k] = (i < nw) ? sw[i] : (uint16_t)0;
    }
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      const uint32_t i = i0 + k * blockDim.x;
      if (i < nw) dw[i] = v[k];
    }
  }
  if ((nw & 1u) && threadIdx.x == 0) dw[nw] = 0;
}

__device__ __forceinline__ uint32_t rd32(const uint8_t* p) {
  return (uint32_t)p[0] | ((uint32_t)p[1] << 8) | ((uint32_t)p[2] << 16) | ((uint32_t)p[3] << 24);
}

// One warp per chunk. Each block builds the model from the 256 counts and
// two per-slot tables in shared memory: ent[slot] = q | (slot - cum) << 16
// (the only lookup on the state's critical path) and sym[slot] (for the
// output byte). The chunk's renormalisation words are staged in shared memory
// with asynchronous 4-byte copies (chunks with more words than the staging
// buffer read them from global memory instead).
constexpr uint32_t kDecStage = 16384;  // words staged per decoding warp (a power of two)

__global__ void __launch_bounds__(kDecWarps * 32) k_rans_decode(const uint8_t* __restrict__ comp,
                                                              uint64_t comp_len_host,
                                                              const uint64_t* __restrict__ comp_len_dev,
                                                              const uint32_t* __restrict__ freq,
                                                              uint64_t n, uint8_t* __restrict__ out,
                                                              unsigned* __restrict__ status) {
  extern __shared__ __align__(16) uint8_t dsm[];
  uint32_t* ent = reinterpret_cast<uint32_t*>(dsm);                     // [2^15]
  uint8_t* sym = dsm + 4 * kRansM;                                      // [2^15]
  uint16_t* wstage = reinterpret_cast<uint16_t*>(dsm + 5 * kRansM);    // [kDecWarps][kDecStage]
  __shared__ uint32_t q[256], cum[256];
  __shared__ ModelSmem ms;
  const int w = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (!build_model(freq, q, cum, ms)) {
    if (threadIdx.x == 0) atomicOr(status, kDevErrEntropy);
    return;
  }
  {  // per-slot tables: each thread fills a contiguous slot range, walking symbols
    const uint32_t per = kRansM / blockDim.x;
    const uint32_t k0 = threadIdx.x * per;
    int lo = 0, hi = 255;
    while (lo < hi) {
      const int mid = (lo + hi + 1) >> 1;
      if (cum[mid] <= k0) lo = mid; else hi = mid - 1;
    }
    int s = lo;
    for (uint32_t k = k0; k < k0 + per; k += 4) {
      uint32_t sw = 0;
      uint4 e4;
      uint32_t* e = &e4.x;
#pragma unroll
      for (int b = 0; b < 4; ++b) {
        const uint32_t kk = k + b;
        while (cum[s] + q[s] <= kk) ++s;
        e[b] = q[s] | ((kk - cum[s]) << 16);
        sw |= (uint32_t)s << (8 * b);
      }
      *reinterpret_cast<uint4*>(ent + k) = e4;
      *reinterpret_cast<uint32_t*>(sym + k) = sw;
    }
  }
  __syncthreads();
  const uint64_t comp_len = comp_len_dev ? *comp_len_dev : comp_len_host;
  // header checks (every warp reads the same 32 bytes)
  if (comp_len < kRansHeader) { if (threadIdx.x == 0) atomicOr(status, kDevErrCorrupt); return; }
  const uint32_t chunk = rd32(comp + 12);
  const uint64_t nn = (uint64_t)rd32(comp + 16) | ((uint64_t)rd32(comp + 20) << 32);
  const uint64_t nchunks = rd32(comp + 24);
  const uint64_t hdr = kRansHeader + 4ull * (nchunks + 1);
  const bool hdr_ok = rd32(comp) == kRansMagic && rd32(comp + 4) == kRansProbBits &&
                      rd32(comp + 8) == kRansLanes && chunk != 0 && (chunk % 32) == 0 && nn == n &&
                      nchunks == (n + chunk - 1) / chunk && rd32(comp + 28) == hdr && hdr <= comp_len &&
                      rd32(comp + kRansHeader + 4 * nchunks) == comp_len;
  if (!hdr_ok) { if (threadIdx.x == 0) atomicOr(status, kDevErrCorrupt); return; }
  uint16_t* stage = wstage + (size_t)w * kDecStage;
  const uint64_t nwarps = (uint64_t)gridDim.x * kDecWarps;
  for (uint64_t c = (uint64_t)blockIdx.x * kDecWarps + w; c < nchunks; c += nwarps) {
    const uint64_t off = rd32(comp + kRansHeader + 4 * c);
    const uint64_t end = rd32(comp + kRansHeader + 4 * (c + 1));
    if (off < hdr || end > comp_len || end < off + kRansChunkHeader || (off & 3u)) {
      if (lane == 0) atomicOr(status, kDevErrCorrupt);
      continue;
    }
    const uint32_t nw = rd32(comp + off);
    if (off + kRansChunkHeader + 2ull * nw + 2ull * (nw & 1u) != end) {
      if (lane == 0) atomicOr(status, kDevErrCorrupt);
      continue;
    }
    uint32_t x = rd32(comp + off + 4 + 4 * lane);
    bool bad = x < kRansL;
    const uint64_t start = c * chunk;
    const uint32_t nsym = (uint32_t)((n - start < chunk) ? (n - start) : chunk);
    const uint32_t full = nsym / 32;  // steps with every lane active
    uint8_t* o = out + start + lane;
    const uint32_t lt = (1u << lane) - 1u;
    uint32_t p = 0;
    if (nw <= kDecStage) {
      // stage pairs of words (the payload is padded to 4 bytes); indices are
      // masked into the staging buffer, so even a corrupt stream reads inside
      // it, and the end-of-chunk checks reject it
      const uint32_t npair = (nw + 1) / 2;
      const uint8_t* src = comp + off + kRansChunkHeader;
      for (uint32_t j = lane; j < npair; j += 32) cp_async4(stage + 2 * j, src + 4 * j);
      cp_async_wait_all();
      __syncwarp();
      for (uint32_t st = 0; st < full; ++st) {
        const uint32_t slot = x & (kRansM - 1);
        const uint32_t e = ent[slot];
        x = (e & 0xFFFFu) * (x >> kRansProbBits) + (e >> 16);
        o[32 * st] = sym[slot];
        const bool need = x < kRansL;
        const unsigned mask = __ballot_sync(0xffffffffu, need);
        const uint32_t w16 = stage[(p + __popc(mask & lt)) & (kDecStage - 1)];
        x = need ? ((x << 16) | w16) : x;
        p += __popc(mask);
      }
      if (full * 32 < nsym) {  // last, partial step
        const bool active = full * 32 + lane < nsym;
        const uint32_t slot = x & (kRansM - 1);
        const uint32_t e = ent[slot];
        if (active) {
          x = (e & 0xFFFFu) * (x >> kRansProbBits) + (e >> 16);
          o[32 * full] = sym[slot];
        }
        const bool need = active && x < kRansL;
        const unsigned mask = __ballot_sync(0xffffffffu, need);
        const uint32_t w16 = stage[(p + __popc(mask & lt)) & (kDecStage - 1)];
        x = need ? ((x << 16) | w16) : x;
        p += __popc(mask);
      }
      bad = bad || p > nw;
    } else {  // words read from global memory, every index checked
      const uint16_t* words = reinterpret_cast<const uint16_t*>(comp + off + kRansChunkHeader);
      const uint32_t steps = (nsym + 31) / 32;
      for (uint32_t st = 0; st < steps; ++st) {
        const bool active = st * 32 + lane < nsym;
        const uint32_t slot = x & (kRansM - 1);
        const uint32_t e = ent[slot];
        if (active) {
          x = (e & 0xFFFFu) * (x >> kRansProbBits) + (e >> 16);
          o[32 * st] = sym[slot];
        }
        const bool need = active && x < kRansL;
        const unsigned mask = __ballot_sync(0xffffffffu, need);
        const uint32_t idx = p + __popc(mask & lt);
        if (need) {
          if (idx < nw) x = (x << 16) | words[idx];
          else { bad = true; x = kRansL; }
        }
        p += __popc(mask);
      }
    }
    bad = bad || x != kRansL || p != nw;
    if (__any_sync(0xffffffffu, bad) && lane == 0) atomicOr(status, kDevErrCorrupt);
    __syncwarp();
  }
}

}  // namespace

cudaError_t launch_rans_encode(const uint8_t* data, size_t n, uint32_t chunk, const uint32_t* freq,
                               uint8_t* slots, unsigned* status, cudaStream_t st) {
  if (n == 0) return cudaSuccess;
  const size_t nc = rans_num_chunks(n, chunk);
  const size_t smem = (size_t)kWarpsPerBlock * chunk;
  if (smem > kSmemOptIn) {
    cudaError_t e = cudaFuncSetAttribute(k_rans_encode, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
  }
  const unsigned grid = (unsigned)((nc + kWarpsPerBlock - 1) / kWarpsPerBlock);
  k_rans_encode<<<grid, kWarpsPerBlock * 32, smem, st>>>(data, n, chunk, freq, slots, nc, status);
  note_launches(1);
  return cudaGetLastError();
}

cudaError_t launch_rans_assemble(const uint8_t* slots, size_t n, uint32_t chunk, uint8_t* out,
                                 uint64_t* out_len, cudaStream_t st) {
  if (n == 0) return cudaSuccess;
  const size_t nc = rans_num_chunks(n, chunk);
  k_rans_offsets<<<1, 1024, 0, st>>>(slots, n, chunk, nc, out, out_len);
  k_rans_compact<<<(unsigned)nc, 256, 0, st>>>(slots, chunk, out);
  note_launches(2);
  return cudaGetLastError();
}

cudaError_t launch_rans_decode(const uint8_t* comp, size_t comp_len, const uint64_t* comp_len_dev,
                               const uint32_t* freq, size_t n, uint8_t* out, unsigned* status,
                               cudaStream_t st) {
  if (n == 0) return cudaSuccess;
  // the grid is sized for the encoder's default chunk size; warps loop over
  // chunks, so a container with any chunk size named in its header decodes
  const size_t nc = rans_num_chunks(n, kRansChunk);
  const unsigned grid = (unsigned)((nc + kDecWarps - 1) / kDecWarps);
  const size_t smem = 5 * (size_t)kRansM + (size_t)kDecWarps * kDecStage * 2;
  const cudaError_t e = cudaFuncSetAttribute(k_rans_decode, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e;
  k_rans_decode<<<grid, kDecWarps * 32, smem, st>>>(comp, comp_len, comp_len_dev, freq, n, out, status);
  note_launches(1);
  return cudaGetLastError();
}
}  // namespace kvf
