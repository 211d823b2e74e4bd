// C-ABI layer of libkvforge_b200: contexts, the whole-layer pipeline, the
// basis step, size accounting and serialisation. Declarations and contracts
// are in include/kvforge.h.
//
// Pipeline (crates/kvforge-cpu/src/pipeline.rs:38-186): keys are quantized
// per channel and values per token; with projection each tensor is first
// projected on its calibrated basis; with entropy coding the packed codes go
// through the chunked rANS coder. Scratch memory comes from the context's
// stream-ordered pool (cudaMallocFromPoolAsync) and is released in stream
// order at the end of each call; result buffers belong to the kvf_compressed
// object.
#include <algorithm>
#include <array>
#include <atomic>
#include <cmath>
#include <cstdio>
#include <cstring>
#include <deque>
#include <exception>
#include <memory>
#include <mutex>
#include <string>
#include <thread>
#include <vector>

#include "kvf_internal.cuh"

using namespace kvf;

namespace kvf {
static std::atomic<uint64_t> g_launches{0};
void note_launches(unsigned n) { g_launches.fetch_add(n, std::memory_order_relaxed); }
}  // namespace kvf

namespace {

thread_local std::string g_err;

kvf_status fail(kvf_status s, const std::string& msg) {
  g_err = msg;
  return s;
}

#define KVF_CUDA(expr)                                                                   \
  do {                                                                                   \
    cudaError_t _e = (expr);                                                             \
    if (_e != cudaSuccess)                                                               \
      return fail(KVF_ERR_CUDA, std::string(#expr) + ": " + cudaGetErrorString(_e));     \
  } while (0)

#define KVF_TRY(expr)                 \
  do {                                \
    kvf_status _s = (expr);           \
    if (_s != KVF_OK) return _s;      \
  } while (0)

inline cudaStream_t S(void* s) { return static_cast<cudaStream_t>(s); }

// makes ctx->device current for the duration of a call and restores the
// caller's device afterwards
struct DeviceGuard {
  int prev = -1;
  bool ok = true;
  explicit DeviceGuard(int dev) {
    if (cudaGetDevice(&prev) != cudaSuccess) prev = -1;
    if (prev != dev) ok = cudaSetDevice(dev) == cudaSuccess;
  }
  ~DeviceGuard() {
    int cur = -1;
    if (prev >= 0 && cudaGetDevice(&cur) == cudaSuccess && cur != prev) cudaSetDevice(prev);
  }
};

// per-call scratch, released in stream order when the call returns
// Requests up to kSmallScratch bytes are carved, 256-byte aligned, from one
// shared block of kScratchBlock bytes, so a call on a small layer makes one
// pool allocation and one free for all its small buffers; larger requests get
// their own allocation.
constexpr size_t kScratchAlign = 256;
constexpr size_t kSmallScratch = 64 * 1024;
constexpr size_t kScratchBlock = 256 * 1024;
inline size_t align_up(size_t n, size_t a) { return (n + a - 1) / a * a; }

struct Scratch {
  cudaStream_t st;
  cudaMemPool_t pool;
  std::vector<void*> ptrs;
  uint8_t* block = nullptr;
  size_t used = 0;
  Scratch(cudaStream_t s, cudaMemPool_t p) : st(s), pool(p) {}
  ~Scratch() {
    for (void* p : ptrs) cudaFreeAsync(p, st);
  }
  void* raw(size_t bytes) {
    void* p = nullptr;
    if (cudaMallocFromPoolAsync(&p, std::max<size_t>(bytes, 1), pool, st) != cudaSuccess) return nullptr;
    ptrs.push_back(p);
    return p;
  }
  template <class T>
  T* get(size_t count) {
    const size_t bytes = std::max<size_t>(count, 1) * sizeof(T);
    if (bytes > kSmallScratch) return static_cast<T*>(raw(bytes));
    const size_t need = align_up(bytes, kScratchAlign);
    if (!block || used + need > kScratchBlock) {
      block = static_cast<uint8_t*>(raw(kScratchBlock));
      used = 0;
      if (!block) return nullptr;
    }
    T* p = reinterpret_cast<T*>(block + used);
    used += need;
    return p;
  }
};

struct BasisData {
  size_t H = 0, R = 0, D = 0;
  float* d_vt = nullptr;        // [H, R, D]
  uint64_t* d_ranks = nullptr;  // [H]
  std::vector<float> vt;
  std::vector<uint64_t> ranks;
  std::vector<float> sv;  // [H, D] singular values (empty for a basis given by the caller)
  int device = 0;
  ~BasisData() {
    if (d_vt || d_ranks) {
      int prev = -1;
      cudaGetDevice(&prev);
      if (prev != device) cudaSetDevice(device);
      if (d_vt) cudaFree(d_vt);
      if (d_ranks) cudaFree(d_ranks);
      if (prev >= 0 && prev != device) cudaSetDevice(prev);
    }
  }
};

// CompressedTensor (crates/kvforge-core/src/types.rs:58-78)
struct TensorC {
  int data_type = KVF_INT8, axis = KVF_PER_CHANNEL;
  bool entropy = false;   // entropy coding enabled (EntropyState present)
  bool has_freq = false;  // container + 256 counts present (non-empty input)
  size_t H = 0, T = 0, D = 0, qcols = 0;
  size_t packed_len = 0, num_params = 0;
  uint8_t* d_data = nullptr;
  size_t data_cap = 0;
  uint64_t* d_len = nullptr;
  bool len_known = false;
  size_t data_len = 0;
  float* d_scales = nullptr;
  float* d_mins = nullptr;
  uint32_t* d_freq = nullptr;
  std::shared_ptr<BasisData> basis;  // projection state, when projected
};

}  // namespace

struct kvf_ctx {
  int device = 0;
  int exact_reconstruct = 0;
  int recon_engine = KVF_RECON_AUTO;
  int proj_engine = KVF_PROJ_AUTO;
  unsigned* d_status = nullptr;
  // the context's own stream-ordered pool: freed blocks stay cached, and a
  // block freed on one stream is reused on another only once its free has
  // completed, so the pool never makes one caller stream wait for another
  cudaMemPool_t pool = nullptr;
  // a layer's value tensor runs on a side stream paired with the caller's
  // stream while its key tensor runs on the caller's stream; fork/join events
  // order the two. One side stream per caller stream, made on first use, so
  // layers issued on different caller streams stay independent.
  struct Side {
    cudaStream_t s = nullptr;
    cudaEvent_t fork = nullptr, join = nullptr;
  };
  // a context may be used from several host threads at once (one caller
  // stream each): the side streams and the profile records are guarded by mu;
  // a deque keeps each Side at a fixed address as more are added
  std::mutex mu;
  std::deque<std::pair<cudaStream_t, Side>> sides;
  cudaError_t side_for(cudaStream_t st, Side** out) {
    std::lock_guard<std::mutex> lock(mu);
    for (auto& kv : sides)
      if (kv.first == st) {
        *out = &kv.second;
        return cudaSuccess;
      }
    Side sd;
    cudaError_t e = cudaStreamCreateWithFlags(&sd.s, cudaStreamNonBlocking);
    if (e == cudaSuccess) e = cudaEventCreateWithFlags(&sd.fork, cudaEventDisableTiming);
    if (e == cudaSuccess) e = cudaEventCreateWithFlags(&sd.join, cudaEventDisableTiming);
    if (e != cudaSuccess) return e;
    sides.emplace_back(st, sd);
    *out = &sides.back().second;
    return cudaSuccess;
  }
  // stage timing (kvf_profile_enable / kvf_profile_read)
  struct Rec {
    int stage;
    cudaEvent_t a, b;
    double bytes;
  };
  int profile = 0;
  std::vector<Rec> recs;
  std::vector<cudaEvent_t> spare;
  // ordering events (no timing) of compressed objects, reused across objects
  std::vector<cudaEvent_t> order_spare;
  cudaError_t order_event(cudaEvent_t* out) {
    {
      std::lock_guard<std::mutex> lock(mu);
      if (!order_spare.empty()) {
        *out = order_spare.back();
        order_spare.pop_back();
        return cudaSuccess;
      }
    }
    return cudaEventCreateWithFlags(out, cudaEventDisableTiming);
  }
  // a waiter that was enqueued before the event goes back keeps the record it saw
  void order_event_release(cudaEvent_t e) {
    std::lock_guard<std::mutex> lock(mu);
    order_spare.push_back(e);
  }
  cudaEvent_t event() {
    std::lock_guard<std::mutex> lock(mu);
    if (!spare.empty()) {
      cudaEvent_t e = spare.back();
      spare.pop_back();
      return e;
    }
    cudaEvent_t e = nullptr;
    cudaEventCreate(&e);
    return e;
  }
};

namespace {
// brackets one pipeline stage with CUDA events when profiling is on
struct StageTimer {
  kvf_ctx* ctx;
  int stage;
  double bytes;
  cudaStream_t st;
  cudaEvent_t a = nullptr;
  StageTimer(kvf_ctx* c, int s, double b, cudaStream_t stream) : ctx(c), stage(s), bytes(b), st(stream) {
    if (ctx && ctx->profile) {
      a = ctx->event();
      cudaEventRecord(a, st);
    }
  }
  ~StageTimer() {
    if (a) {
      cudaEvent_t b = ctx->event();
      cudaEventRecord(b, st);
      std::lock_guard<std::mutex> lock(ctx->mu);
      ctx->recs.push_back({stage, a, b, bytes});
    }
  }
};
}  // namespace

struct kvf_basis {
  std::shared_ptr<BasisData> d;
};

// One device block shared by the objects that one batched call builds; it
// goes back to the pool, on the building stream, when the last of them is
// freed (each free first makes that stream wait for its own readers, so the
// final release follows every reader of every object).
// The objects also share one `ready` event, recorded once for the call.
struct SharedBlock {
  kvf_ctx* ctx = nullptr;
  int device = 0;
  cudaStream_t stream = nullptr;
  void* p = nullptr;
  cudaEvent_t ready = nullptr;
  SharedBlock() = default;
  SharedBlock(const SharedBlock&) = delete;
  SharedBlock& operator=(const SharedBlock&) = delete;
  ~SharedBlock() {
    DeviceGuard g(device);
    if (p) cudaFreeAsync(p, stream);
    if (ready) ctx->order_event_release(ready);
  }
};

struct kvf_compressed {
  kvf_ctx* ctx = nullptr;
  int device = 0;
  cudaStream_t stream = nullptr;
  size_t layer_idx = 0, H = 0, T = 0, D = 0, original_size_bytes = 0;
  TensorC key, value;
  float* d_scores = nullptr;
  std::vector<void*> owned;
  std::shared_ptr<SharedBlock> block;  // buffers inside a block shared with other objects
  // Cross-stream lifetime: `ready` is recorded on `stream` once the object's
  // buffers are complete, and a reader on another stream waits for it first;
  // each reader stream records its own event after its last use, and
  // kvf_compressed_free makes `stream` wait for all of them before the
  // buffers go back to the pool. Readers take a const object, so the use list
  // is mutable and guarded.
  cudaEvent_t ready = nullptr;
  mutable std::mutex use_mu;
  mutable std::vector<std::pair<cudaStream_t, cudaEvent_t>> uses;

  // owned buffers are allocated in the order of the stream that first uses
  // them (a layer's value tensor is built on the context's side stream)
  template <class T>
  T* alloc(size_t count, cudaStream_t on) {
    void* p = nullptr;
    if (cudaMallocFromPoolAsync(&p, std::max<size_t>(count, 1) * sizeof(T), ctx->pool, on) != cudaSuccess)
      return nullptr;
    owned.push_back(p);
    return static_cast<T*>(p);
  }
  template <class T>
  T* alloc(size_t count) {
    return alloc<T>(count, stream);
  }
};

namespace {

kvf_status check_ctx(kvf_ctx* ctx) {
  if (!ctx) return fail(KVF_ERR_INVALID_CONFIG, "null context");
  return KVF_OK;
}

kvf_status check_qcfg(int dt, int axis) {
  if (dt == KVF_F32) return fail(KVF_ERR_QUANTIZATION, "F32 data type does not need quantization");
  if (dt != KVF_INT4 && dt != KVF_INT8) return fail(KVF_ERR_INVALID_CONFIG, "unknown data type");
  if (axis != KVF_PER_CHANNEL && axis != KVF_PER_TOKEN) return fail(KVF_ERR_INVALID_CONFIG, "unknown quantization axis");
  return KVF_OK;
}

kvf_status check_dtype(int in_dtype) {
  if (in_dtype != KVF_IN_F32 && in_dtype != KVF_IN_F16) return fail(KVF_ERR_INVALID_CONFIG, "unknown input dtype");
  return KVF_OK;
}

kvf_status check_shape(size_t H, size_t T, size_t D) {
  if (D > 1024) return fail(KVF_ERR_SHAPE_MISMATCH, "head_dim > 1024 is not supported");
  if (H > 65535) return fail(KVF_ERR_SHAPE_MISMATCH, "num_heads > 65535 is not supported");
  // H * D <= 2^26, so the division keeps the product check free of overflow
  if (H && D && T > (size_t(1) << 40) / (H * D)) return fail(KVF_ERR_SHAPE_MISMATCH, "tensor too large");
  return KVF_OK;
}

// a reader of `c` on stream `st`: waits for the object's buffers to be
// complete when `st` is not the stream that built them
kvf_status reader_enter(const kvf_compressed* c, cudaStream_t st) {
  if (c->ready && st != c->stream) KVF_CUDA(cudaStreamWaitEvent(st, c->ready, 0));
  return KVF_OK;
}
// ... and after its last use: records on `st` what kvf_compressed_free waits for
kvf_status reader_leave(const kvf_compressed* c, cudaStream_t st) {
  if (st == c->stream) return KVF_OK;
  std::lock_guard<std::mutex> lock(c->use_mu);
  cudaEvent_t ev = nullptr;
  for (auto& u : c->uses)
    if (u.first == st) ev = u.second;
  if (!ev) {
    KVF_CUDA(c->ctx->order_event(&ev));
    c->uses.emplace_back(st, ev);
  }
  KVF_CUDA(cudaEventRecord(ev, st));
  return KVF_OK;
}
// marks `c` complete on its own stream (end of compress / deserialize)
kvf_status mark_ready(kvf_compressed* c) {
  if (!c->ready) KVF_CUDA(c->ctx->order_event(&c->ready));
  KVF_CUDA(cudaEventRecord(c->ready, c->stream));
  return KVF_OK;
}

// per-token projection + quantization (ProjectOut mode 2) on the tensor-core
// engine when the context allows it and the shape fits, on CUDA cores
// otherwise (R <= 32 there); both give identical codes, scales and mins
bool token_tc(kvf_ctx* ctx, const void* x, int in_dtype, size_t H, size_t T, size_t D, const float* bvt, size_t R) {
  return (ctx->proj_engine == KVF_PROJ_TENSOR_CORE || ctx->proj_engine == KVF_PROJ_TENSOR_CORE_APPROX) &&
         project_tc_fits(x, in_dtype, H, T, D, bvt, R);
}
cudaError_t project_token(kvf_ctx* ctx, const void* x, int in_dtype, size_t H, size_t T, size_t D,
                          const float* bvt, const uint64_t* ranks, size_t R, const ProjectOut& po, cudaStream_t st) {
  if (token_tc(ctx, x, in_dtype, H, T, D, bvt, R)) {
    const cudaError_t e =
        launch_project_tc(x, in_dtype, H, T, D, bvt, ranks, R, ctx->proj_engine != KVF_PROJ_TENSOR_CORE_APPROX, po, st);
    if (e != cudaErrorNotSupported || R > 32) return e;
  }
  return launch_project(x, in_dtype, H, T, D, bvt, ranks, R, po, st);
}
// INT4 codes are packed inside the projection kernel when each row's codes
// start on a byte (R even); the CUDA-core kernel also packs pairs that run
// across rows when every 256-token tile starts on a byte (T even)
bool token_fuse_pack(bool tc, int dt, size_t R, size_t T) {
  return dt == KVF_INT4 && (R % 2 == 0 || (!tc && T % 2 == 0));
}

// quantize (from f32/f16 input) into `packed`, optional histogram of the packed bytes
kvf_status quantize_into(Scratch& sc, const void* qin, int qdt, size_t H, size_t T, size_t D, int dt,
                         int axis, uint8_t* packed, float* scales, float* mins, uint32_t* hist,
                         cudaStream_t st) {
  const size_t n = H * T * D;
  if (axis == KVF_PER_CHANNEL) {  // one pass over the input where the shape allows it
    const cudaError_t e = launch_quantize_channel_cluster(qin, qdt, H, T, D, dt, packed, scales, mins, hist, st);
    if (e == cudaSuccess) return KVF_OK;
    if (e != cudaErrorNotSupported) return fail(KVF_ERR_CUDA, std::string("per-channel quantize: ") + cudaGetErrorString(e));
  }
  if (axis == KVF_PER_TOKEN && D % 4) {  // even widths that the 16-byte kernel does not take: one pass, packed
    const cudaError_t e = launch_quantize_token_pairs(qin, qdt, H, T, D, dt, packed, scales, mins, hist, st);
    if (e == cudaSuccess) return KVF_OK;
    if (e != cudaErrorNotSupported) return fail(KVF_ERR_CUDA, std::string("per-token quantize: ") + cudaGetErrorString(e));
  }
  int* keys = nullptr;
  if (axis == KVF_PER_CHANNEL) {
    keys = sc.get<int>(3 * H * D);  // min keys, max keys, reciprocal scales
    if (!keys) return fail(KVF_ERR_CUDA, "scratch allocation failed");
  }
  if (dt == KVF_INT8) {
    KVF_CUDA(launch_quantize_codes(qin, qdt, H, T, D, dt, axis, packed, scales, mins, keys, st));
    if (hist) KVF_CUDA(launch_histogram(packed, n, hist, st));
  } else {
    uint8_t* codes = sc.get<uint8_t>(n);
    if (!codes) return fail(KVF_ERR_CUDA, "scratch allocation failed");
    KVF_CUDA(launch_quantize_codes(qin, qdt, H, T, D, dt, axis, codes, scales, mins, keys, st));
    KVF_CUDA(launch_pack_int4(codes, n, packed, hist, st));
  }
  return KVF_OK;
}

// chunk coding (the model is built from `freq` inside the kernel) -> container
// in `out`, its length in d_len
kvf_status rans_encode_into(kvf_ctx* ctx, Scratch& sc, const uint8_t* packed, size_t plen,
                            const uint32_t* freq, uint8_t* out, uint64_t* d_len, cudaStream_t st) {
  const size_t nc = rans_num_chunks(plen, kRansChunk);
  unsigned long long* lookback = sc.get<unsigned long long>(nc + 1);  // status words + block ticket
  if (!lookback) return fail(KVF_ERR_CUDA, "scratch allocation failed");
  KVF_CUDA(launch_rans_encode(packed, plen, kRansChunk, freq, lookback, out, d_len, ctx->d_status, st));
  return KVF_OK;
}

// compress_tensor (crates/kvforge-cpu/src/pipeline.rs:38-72)
//
// With projection the quantizer reads the projection kernel's epilogue:
// keys (per channel) get P plus per-(head, r) min/max from the projection
// kernel, then one quantize + pack + histogram kernel; values (per token) are
// quantized row by row inside the projection kernel, then packed.
kvf_status compress_tensor(kvf_ctx* ctx, kvf_compressed* owner, const void* x, int in_dtype, size_t H,
                           size_t T, size_t D, int dt, int axis, const std::shared_ptr<BasisData>& basis,
                           bool entropy, bool calib, float* d_scores, TensorC* out, cudaStream_t st) {
  KVF_TRY(check_qcfg(dt, axis));
  Scratch sc(st, ctx->pool);
  out->data_type = dt;
  out->axis = axis;
  out->H = H;
  out->T = T;
  out->D = D;
  out->entropy = entropy;
  out->basis = basis;
  if (basis) {
    if (T == 0 || D == 0) return fail(KVF_ERR_PROJECTION, "Cannot project empty tensor");
    if (basis->H != H || basis->D != D)
      return fail(KVF_ERR_SHAPE_MISMATCH, "basis shape does not match the tensor");
  }
  const size_t qcols = basis ? basis->R : D;
  const size_t n = H * T * qcols;
  const size_t plen = packed_len(n, dt);
  const size_t np = num_params(H, T, qcols, axis);
  const size_t in_bytes = H * T * D * (in_dtype == KVF_IN_F16 ? 2 : 4);
  out->qcols = qcols;
  out->packed_len = plen;
  out->num_params = np;
  const bool do_ent = entropy && plen > 0;
  out->has_freq = do_ent;
  // the tensor's own buffers (scales, mins, then the 256 counts, the rANS
  // container and its length, or the packed codes) in one allocation
  const size_t sp = align_up(np * 4, kScratchAlign);
  const size_t data_cap = do_ent ? rans_max_len(plen, kRansChunk) : plen;
  const size_t owned = 2 * sp + (do_ent ? align_up(1024, kScratchAlign) + align_up(data_cap, kScratchAlign) + 8
                                        : std::max<size_t>(plen, 1));
  uint8_t* base = owner->alloc<uint8_t>(owned, st);
  if (!base) return fail(KVF_ERR_CUDA, "allocation failed");
  out->d_scales = reinterpret_cast<float*>(base);
  out->d_mins = reinterpret_cast<float*>(base + sp);
  uint8_t* packed = do_ent ? sc.get<uint8_t>(plen) : base + 2 * sp;
  if (!packed) return fail(KVF_ERR_CUDA, "allocation failed");
  uint32_t* hist = nullptr;
  if (do_ent) {
    out->d_freq = reinterpret_cast<uint32_t*>(base + 2 * sp);
    out->data_cap = data_cap;
    out->d_data = base + 2 * sp + align_up(1024, kScratchAlign);
    out->d_len = reinterpret_cast<uint64_t*>(out->d_data + align_up(data_cap, kScratchAlign));
    KVF_CUDA(cudaMemsetAsync(out->d_freq, 0, 256 * sizeof(uint32_t), st));
    hist = out->d_freq;
  }

  const bool do_calib = calib && d_scores && T >= 64;  // CalibrationConfig::default().min_tokens
  double* cpart = nullptr;
  size_t ctiles = 0;
  if (do_calib) {
    ctiles = basis ? project_num_tiles(T) : calib_partial_tiles(T, D);
    cpart = sc.get<double>(2 * H * ctiles);
    if (!cpart) return fail(KVF_ERR_CUDA, "scratch allocation failed");
  }

  if (basis) {
    ProjectOut po;
  po.status = ctx->d_status;
    po.cpart = cpart;
    po.levels = quant_levels(dt);
    if (axis == KVF_PER_CHANNEL) {
      float* P = sc.get<float>(n);
      int* keys = sc.get<int>(2 * H * qcols);
      if (!P || !keys) return fail(KVF_ERR_CUDA, "scratch allocation failed");
      KVF_CUDA(launch_minmax_init(keys, keys + H * qcols, H * qcols, st));
      po.mode = 1;
      po.P = P;
      po.kmin = keys;
      po.kmax = keys + H * qcols;
      {
        StageTimer tm(ctx, KVF_STAGE_PROJECT, (double)in_bytes + 4.0 * n, st);
        KVF_CUDA(launch_project(x, in_dtype, H, T, D, basis->d_vt, basis->d_ranks, qcols, po, st));
      }
      StageTimer tm(ctx, KVF_STAGE_QUANTIZE, 4.0 * n + (double)plen + 8.0 * np, st);
      KVF_CUDA(launch_quantpack_channel(P, H, T, qcols, po.kmin, po.kmax, dt, out->d_scales, out->d_mins, packed,
                                        hist, st));
    } else if (qcols <= 32 || token_tc(ctx, x, in_dtype, H, T, D, basis->d_vt, qcols)) {
      const bool fuse_pack = token_fuse_pack(token_tc(ctx, x, in_dtype, H, T, D, basis->d_vt, qcols), dt, qcols, T);
      uint8_t* codes = (dt == KVF_INT8) ? packed : (fuse_pack ? nullptr : sc.get<uint8_t>(n));
      if (dt == KVF_INT4 && !fuse_pack && !codes) return fail(KVF_ERR_CUDA, "scratch allocation failed");
      po.mode = 2;
      po.codes = codes;
      po.packed = fuse_pack ? packed : nullptr;
      po.hist = (dt == KVF_INT8 || fuse_pack) ? hist : nullptr;
      po.scales = out->d_scales;
      po.mins = out->d_mins;
      {
        StageTimer tm(ctx, KVF_STAGE_PROJECT, (double)in_bytes + (double)plen + 8.0 * np, st);
        KVF_CUDA(project_token(ctx, x, in_dtype, H, T, D, basis->d_vt, basis->d_ranks, qcols, po, st));
      }
      if (dt == KVF_INT4 && !fuse_pack) {
        StageTimer tm(ctx, KVF_STAGE_QUANTIZE, (double)n + (double)plen, st);
        KVF_CUDA(launch_pack_int4(codes, n, packed, hist, st));
      }
    } else {
      float* P = sc.get<float>(n);
      if (!P) return fail(KVF_ERR_CUDA, "scratch allocation failed");
      po.mode = 0;
      po.P = P;
      {
        StageTimer tm(ctx, KVF_STAGE_PROJECT, (double)in_bytes + 4.0 * n, st);
        KVF_CUDA(launch_project(x, in_dtype, H, T, D, basis->d_vt, basis->d_ranks, qcols, po, st));
      }
      StageTimer tm(ctx, KVF_STAGE_QUANTIZE, 4.0 * n + (double)plen + 8.0 * np, st);
      KVF_TRY(quantize_into(sc, P, KVF_IN_F32, H, T, qcols, dt, axis, packed, out->d_scales, out->d_mins, hist, st));
    }
  } else {
    if (do_calib) {
      StageTimer tm(ctx, KVF_STAGE_CALIBRATE, (double)in_bytes, st);
      KVF_CUDA(launch_calib_partials(x, in_dtype, H, T, D, cpart, st));
    }
    StageTimer tm(ctx, KVF_STAGE_QUANTIZE, (double)in_bytes + (double)plen + 8.0 * np, st);
    KVF_TRY(quantize_into(sc, x, in_dtype, H, T, D, dt, axis, packed, out->d_scales, out->d_mins, hist, st));
  }
  if (cpart) KVF_CUDA(launch_calib_finalize(cpart, H, ctiles, T, D, d_scores, st));

  if (do_ent) {
    StageTimer tm(ctx, KVF_STAGE_ENTROPY_ENCODE, (double)plen, st);
    KVF_TRY(rans_encode_into(ctx, sc, packed, plen, out->d_freq, out->d_data, out->d_len, st));
    out->len_known = false;
  } else {
    out->d_data = packed;
    out->data_cap = plen;
    out->data_len = plen;
    out->len_known = true;
  }
  return KVF_OK;
}

// decompress_tensor (crates/kvforge-cpu/src/pipeline.rs:75-97)
kvf_status decompress_tensor(kvf_ctx* ctx, const TensorC& t, float* out, cudaStream_t st) {
  Scratch sc(st, ctx->pool);
  const uint8_t* codes = t.d_data;
  if (t.has_freq) {
    uint8_t* dec = sc.get<uint8_t>(t.packed_len);
    if (!dec) return fail(KVF_ERR_CUDA, "scratch allocation failed");
    StageTimer tm(ctx, KVF_STAGE_ENTROPY_DECODE, 2.0 * t.packed_len, st);
    KVF_CUDA(launch_rans_decode(t.d_data, t.data_len, t.len_known ? nullptr : t.d_len, t.d_freq, t.packed_len,
                                dec, ctx->d_status, st));
    codes = dec;
  }
  const double out_bytes = (double)t.H * t.T * t.D * 4 + (double)t.packed_len + 8.0 * t.num_params;
  if (t.basis) {
    StageTimer tm(ctx, KVF_STAGE_RECONSTRUCT, out_bytes + (double)t.H * t.basis->R * t.D * 4, st);
    KVF_CUDA(launch_dequant_reconstruct(codes, nullptr, t.d_scales, t.d_mins, t.data_type, t.axis, t.H, t.T,
                                        t.qcols, t.D, t.basis->d_vt, t.basis->d_ranks, ctx->exact_reconstruct,
                                        ctx->recon_engine, out, ctx->d_status, st));
  } else {
    StageTimer tm(ctx, KVF_STAGE_DEQUANTIZE, out_bytes, st);
    KVF_CUDA(launch_dequantize(codes, t.d_scales, t.d_mins, t.data_type, t.axis, t.H, t.T, t.D, out, st));
  }
  return KVF_OK;
}

kvf_status resolve_len(TensorC& t, cudaStream_t st) {
  if (t.len_known) return KVF_OK;
  uint64_t len = 0;
  KVF_CUDA(cudaMemcpyAsync(&len, t.d_len, sizeof(uint64_t), cudaMemcpyDeviceToHost, st));
  KVF_CUDA(cudaStreamSynchronize(st));
  t.data_len = (size_t)len;
  t.len_known = true;
  return KVF_OK;
}

// CompressedTensor::size_bytes (types.rs:66-78 with 91-95, 131-135, 144-148)
size_t tensor_size(const TensorC& t) {
  size_t total = t.data_len + 2 * t.num_params * 4;
  if (t.basis) total += t.H * t.basis->R * t.D * 4 + t.H * 8;
  if (t.entropy) total += (t.has_freq ? 256 * 4 : 0) + 8;
  return total;
}

// ---- fp64 symmetric eigen-solver for the basis step (cyclic Jacobi) ---------
// A (n x n, row-major) is overwritten; eigenvalues land on its diagonal and the
// eigenvectors in the columns of V.
void jacobi_eigen(std::vector<double>& A, size_t n, std::vector<double>& V) {
  V.assign(n * n, 0.0);
  for (size_t i = 0; i < n; ++i) V[i * n + i] = 1.0;
  double fro = 0.0;
  for (double a : A) fro += a * a;
  if (fro == 0.0) return;
  for (int sweep = 0; sweep < 60; ++sweep) {
    double off = 0.0;
    for (size_t p = 0; p < n; ++p)
      for (size_t q = p + 1; q < n; ++q) off += A[p * n + q] * A[p * n + q];
    if (off <= 1e-30 * fro) break;
    for (size_t p = 0; p + 1 < n; ++p) {
      for (size_t q = p + 1; q < n; ++q) {
        const double apq = A[p * n + q];
        if (std::fabs(apq) <= 1e-300) continue;
        const double theta = (A[q * n + q] - A[p * n + p]) / (2.0 * apq);
        const double t = (theta >= 0 ? 1.0 : -1.0) / (std::fabs(theta) + std::sqrt(theta * theta + 1.0));
        const double c = 1.0 / std::sqrt(t * t + 1.0), s = t * c;
        for (size_t k = 0; k < n; ++k) {
          const double akp = A[k * n + p], akq = A[k * n + q];
          A[k * n + p] = c * akp - s * akq;
          A[k * n + q] = s * akp + c * akq;
        }
        for (size_t k = 0; k < n; ++k) {
          const double apk = A[p * n + k], aqk = A[q * n + k];
          A[p * n + k] = c * apk - s * aqk;
          A[q * n + k] = s * apk + c * aqk;
        }
        for (size_t k = 0; k < n; ++k) {
          const double vkp = V[k * n + p], vkq = V[k * n + q];
          V[k * n + p] = c * vkp - s * vkq;
          V[k * n + q] = s * vkp + c * vkq;
        }
      }
    }
  }
}

// select_rank (crates/kvforge-cpu/src/projection.rs:31-59)
size_t select_rank(const float* sv, size_t n, double threshold, size_t max_rank) {
  if (n == 0) return 0;
  double total = 0.0;
  for (size_t i = 0; i < n; ++i) total += (double)sv[i] * (double)sv[i];
  if (total < 1e-12) return 1;
  double cum = 0.0;
  size_t rank = 0;
  for (size_t i = 0; i < n; ++i) {
    cum += (double)sv[i] * (double)sv[i];
    rank += 1;
    if (cum / total >= threshold) break;
  }
  if (max_rank > 0) rank = std::min(rank, max_rank);
  return std::max<size_t>(rank, 1);
}

kvf_status upload_basis(BasisData& b) {
  KVF_CUDA(cudaMalloc(&b.d_vt, std::max<size_t>(b.vt.size(), 1) * sizeof(float)));
  KVF_CUDA(cudaMalloc(&b.d_ranks, std::max<size_t>(b.H, 1) * sizeof(uint64_t)));
  if (!b.vt.empty()) KVF_CUDA(cudaMemcpy(b.d_vt, b.vt.data(), b.vt.size() * sizeof(float), cudaMemcpyHostToDevice));
  if (b.H) KVF_CUDA(cudaMemcpy(b.d_ranks, b.ranks.data(), b.H * sizeof(uint64_t), cudaMemcpyHostToDevice));
  return KVF_OK;
}

kvf_status compute_basis(kvf_ctx* ctx, const void* x, int in_dtype, size_t H, size_t T, size_t D,
                         double threshold, size_t max_rank, std::shared_ptr<BasisData>* out,
                         cudaStream_t st) {
  if (T == 0 || D == 0) return fail(KVF_ERR_PROJECTION, "Cannot project empty tensor");
  auto b = std::make_shared<BasisData>();
  b->device = ctx->device;
  b->H = H;
  b->D = D;
  std::vector<double> G(H * D * D);
  {
    Scratch sc(st, ctx->pool);
    const size_t tiles = gram_num_tiles(T);
    float* partial = sc.get<float>(H * tiles * D * D);
    double* gram = sc.get<double>(H * D * D);
    if (!partial || !gram) return fail(KVF_ERR_CUDA, "scratch allocation failed");
    StageTimer tm(ctx, KVF_STAGE_BASIS, (double)H * T * D * (in_dtype == KVF_IN_F16 ? 2 : 4), st);
    KVF_CUDA(launch_gram(x, in_dtype, H, T, D, partial, gram, st));
    KVF_CUDA(cudaMemcpyAsync(G.data(), gram, G.size() * sizeof(double), cudaMemcpyDeviceToHost, st));
    KVF_CUDA(cudaStreamSynchronize(st));
  }
  b->sv.assign(H * D, 0.0f);
  std::vector<float> full(H * D * D);
  std::atomic<size_t> next{0};
  auto worker = [&]() {
    std::vector<double> A, V;
    std::vector<size_t> idx(D);
    for (size_t h = next++; h < H; h = next++) {
      A.assign(G.begin() + h * D * D, G.begin() + (h + 1) * D * D);
      jacobi_eigen(A, D, V);
      for (size_t i = 0; i < D; ++i) idx[i] = i;
      std::stable_sort(idx.begin(), idx.end(), [&](size_t a, size_t c) { return A[a * D + a] > A[c * D + c]; });
      for (size_t r = 0; r < D; ++r) {
        const size_t k = idx[r];
        const double lam = A[k * D + k];
        b->sv[h * D + r] = (float)std::sqrt(lam > 0.0 ? lam : 0.0);
        size_t big = 0;
        for (size_t c = 1; c < D; ++c)
          if (std::fabs(V[c * D + k]) > std::fabs(V[big * D + k])) big = c;
        const double sgn = V[big * D + k] < 0 ? -1.0 : 1.0;
        for (size_t c = 0; c < D; ++c) full[(h * D + r) * D + c] = (float)(sgn * V[c * D + k]);
      }
    }
  };
  const size_t nth = std::max<size_t>(1, std::min<size_t>(H, std::thread::hardware_concurrency()));
  std::vector<std::thread> pool;
  for (size_t i = 1; i < nth; ++i) pool.emplace_back(worker);
  worker();
  for (auto& th : pool) th.join();
  const size_t k = std::min(T, D);  // the SVD yields min(T, D) singular values
  b->ranks.assign(H, 1);
  size_t R = 0;
  for (size_t h = 0; h < H; ++h) {
    b->ranks[h] = select_rank(&b->sv[h * D], k, threshold, max_rank);
    R = std::max<size_t>(R, b->ranks[h]);
  }
  if (H == 0) R = 1;  // ranks.iter().max().unwrap_or(&1)
  b->R = R;
  b->vt.assign(H * R * D, 0.0f);
  for (size_t h = 0; h < H; ++h)
    for (size_t r = 0; r < b->ranks[h]; ++r)
      std::memcpy(&b->vt[(h * R + r) * D], &full[(h * D + r) * D], D * sizeof(float));
  KVF_TRY(upload_basis(*b));
  *out = b;
  return KVF_OK;
}

// ---- serialisation helpers --------------------------------------------------
struct Writer {
  uint8_t* buf;
  size_t cap, len = 0;
  void put(const void* p, size_t n) {
    if (buf && len + n <= cap) std::memcpy(buf + len, p, n);
    len += n;
  }
  template <class T>
  void v(T x) { put(&x, sizeof(T)); }
};
struct Reader {
  const uint8_t* buf;
  size_t len, pos = 0;
  bool ok = true;
  bool get(void* p, size_t n) {
    if (!ok || pos + n > len) { ok = false; return false; }
    std::memcpy(p, buf + pos, n);
    pos += n;
    return true;
  }
  template <class T>
  T v() { T x{}; get(&x, sizeof(T)); return x; }
};

// The wire format is the reference's: CompressedKV.to_bytes is
// bincode::serialize (crates/kvforge-python/src/py_types.rs:98-110, bincode
// 1.x, Cargo.toml:28) of the structs in crates/kvforge-core/src/types.rs:36-148.
// bincode 1.x with its default options writes little-endian fixed-width
// integers, usize as u64, a Vec as a u64 length then its elements, an Option
// as a u8 tag (0 None, 1 Some) then the value, a unit enum variant as its u32
// declaration index, and struct fields in declaration order:
//   CompressedKV     { layer_idx, original_shape: Shape {num_heads, seq_len, head_dim},
//                      key_data, value_data: CompressedTensor, original_size_bytes }
//   CompressedTensor { quantized_data: Vec<u8>, quant_params: QuantParams,
//                      projection_state: Option<ProjectionState>, entropy_state: Option<EntropyState> }
//   QuantParams      { scales: Vec<f32>, mins: Vec<f32>, data_type: DataType {INT4, INT8, F32},
//                      axis: QuantAxis {PerChannel, PerToken}, shape: Vec<usize> = [H, T, cols] }
//   ProjectionState  { basis_vt: Vec<f32>, ranks: Vec<usize>, num_heads, head_dim,
//                      projected_shape: Vec<usize> = [H, T, R] }
//   EntropyState     { frequencies: Vec<u32> (256, or empty for empty input), original_len }
// quantized_data holds this library's rANS container when entropy coding is on.

kvf_status ser_tensor(TensorC& t, Writer& w, cudaStream_t st) {
  KVF_TRY(resolve_len(t, st));
  std::vector<uint8_t> host;
  auto dl = [&](const void* d, size_t n) -> kvf_status {
    host.resize(n);
    if (n && w.buf) {  // the size pass copies nothing
      KVF_CUDA(cudaMemcpyAsync(host.data(), d, n, cudaMemcpyDeviceToHost, st));
      KVF_CUDA(cudaStreamSynchronize(st));
    }
    w.put(host.data(), n);
    return KVF_OK;
  };
  w.v<uint64_t>(t.data_len);  // quantized_data
  KVF_TRY(dl(t.d_data, t.data_len));
  w.v<uint64_t>(t.num_params);  // quant_params.scales
  KVF_TRY(dl(t.d_scales, t.num_params * 4));
  w.v<uint64_t>(t.num_params);  // quant_params.mins
  KVF_TRY(dl(t.d_mins, t.num_params * 4));
  w.v<uint32_t>((uint32_t)t.data_type);
  w.v<uint32_t>((uint32_t)t.axis);
  w.v<uint64_t>(3);
  w.v<uint64_t>(t.H);
  w.v<uint64_t>(t.T);
  w.v<uint64_t>(t.qcols);
  if (t.basis) {
    w.v<uint8_t>(1);
    w.v<uint64_t>(t.basis->vt.size());
    w.put(t.basis->vt.data(), t.basis->vt.size() * sizeof(float));
    w.v<uint64_t>(t.H);
    w.put(t.basis->ranks.data(), t.H * sizeof(uint64_t));
    w.v<uint64_t>(t.H);
    w.v<uint64_t>(t.D);
    w.v<uint64_t>(3);
    w.v<uint64_t>(t.H);
    w.v<uint64_t>(t.T);
    w.v<uint64_t>(t.qcols);
  } else {
    w.v<uint8_t>(0);
  }
  if (t.entropy) {
    w.v<uint8_t>(1);
    w.v<uint64_t>(t.has_freq ? 256 : 0);
    if (t.has_freq) KVF_TRY(dl(t.d_freq, 256 * 4));
    w.v<uint64_t>(t.packed_len);
  } else {
    w.v<uint8_t>(0);
  }
  return KVF_OK;
}

kvf_status deser_tensor(kvf_compressed* c, TensorC& t, Reader& r, cudaStream_t st) {
  const auto bad = [](const char* what) { return fail(KVF_ERR_SERIALIZATION, what); };
  t.H = c->H; t.T = c->T; t.D = c->D;
  t.data_len = r.v<uint64_t>();
  if (!r.ok || t.data_len > r.len - r.pos) return bad("truncated quantized data");
  const size_t data_pos = r.pos;
  r.pos += t.data_len;
  const uint64_t ns = r.v<uint64_t>();
  if (!r.ok || ns > (r.len - r.pos) / 4) return bad("truncated scales");
  const size_t scales_pos = r.pos;
  r.pos += ns * 4;
  const uint64_t nm = r.v<uint64_t>();
  if (!r.ok || nm != ns || nm > (r.len - r.pos) / 4) return bad("truncated mins");
  const size_t mins_pos = r.pos;
  r.pos += nm * 4;
  const uint32_t dt = r.v<uint32_t>(), ax = r.v<uint32_t>();
  if (!r.ok || dt > 2 || ax > 1) return bad("unknown data type or axis variant");
  t.data_type = (int)dt;
  t.axis = (int)ax;
  KVF_TRY(check_qcfg(t.data_type, t.axis));
  if (r.v<uint64_t>() != 3) return bad("quant_params.shape must have 3 entries");
  const uint64_t qh = r.v<uint64_t>(), qt = r.v<uint64_t>(), qc = r.v<uint64_t>();
  if (!r.ok || qh != t.H || qt != t.T) return bad("quant_params.shape does not match the layer");
  t.qcols = qc;
  const uint8_t ptag = r.v<uint8_t>();
  if (!r.ok || ptag > 1) return bad("bad projection_state tag");
  if (ptag == 1) {
    if (qc == 0 || qc > t.D) return bad("projected width must be in 1..head_dim");
    auto b = std::make_shared<BasisData>();
    b->device = c->device;
    b->H = t.H; b->R = qc; b->D = t.D;
    if (r.v<uint64_t>() != t.H * qc * t.D) return bad("basis_vt length does not match [H, R, D]");
    // sizes come from the wire: check them against the bytes left before
    // allocating anything for them
    if (!r.ok || t.H * qc * t.D > (r.len - r.pos) / 4) return bad("truncated basis_vt");
    b->vt.resize(t.H * qc * t.D);
    if (!r.get(b->vt.data(), b->vt.size() * 4)) return bad("truncated basis_vt");
    if (r.v<uint64_t>() != t.H) return bad("ranks length does not match num_heads");
    if (!r.ok || t.H > (r.len - r.pos) / 8) return bad("truncated ranks");
    b->ranks.resize(t.H);
    if (!r.get(b->ranks.data(), t.H * 8)) return bad("truncated ranks");
    if (r.v<uint64_t>() != t.H || r.v<uint64_t>() != t.D) return bad("projection num_heads / head_dim mismatch");
    if (r.v<uint64_t>() != 3 || r.v<uint64_t>() != t.H || r.v<uint64_t>() != t.T || r.v<uint64_t>() != qc)
      return bad("projected_shape does not match [H, T, R]");
    if (!r.ok) return bad("truncated projection state");
    for (uint64_t rk : b->ranks)
      if (rk > qc) return bad("rank exceeds the projected width");
    KVF_TRY(upload_basis(*b));
    t.basis = b;
  } else if (qc != t.D) {
    return bad("unprojected width must be head_dim");
  }
  const size_t n = t.H * t.T * t.qcols;
  t.packed_len = packed_len(n, t.data_type);
  t.num_params = num_params(t.H, t.T, t.qcols, t.axis);
  if (ns != t.num_params) return bad("parameter count does not match the shape");
  const uint8_t etag = r.v<uint8_t>();
  if (!r.ok || etag > 1) return bad("bad entropy_state tag");
  t.entropy = etag == 1;
  size_t freq_pos = 0;
  if (t.entropy) {
    const uint64_t nf = r.v<uint64_t>();
    if (!r.ok || (nf != 0 && nf != 256) || nf * 4 > r.len - r.pos) return bad("frequencies must have 0 or 256 entries");
    t.has_freq = nf == 256;
    freq_pos = r.pos;
    r.pos += nf * 4;
    if (r.v<uint64_t>() != t.packed_len || !r.ok) return bad("entropy original_len does not match the codes");
  }
  if (!t.has_freq && t.data_len != t.packed_len) return bad("quantized data length does not match the shape");
  if (t.has_freq && t.data_len % 4 != 0) return fail(KVF_ERR_ENTROPY, "Compressed data length not aligned to 4 bytes");
  auto up = [&](void* d, size_t pos, size_t nbytes) -> kvf_status {
    if (nbytes) KVF_CUDA(cudaMemcpyAsync(d, r.buf + pos, nbytes, cudaMemcpyHostToDevice, st));
    return KVF_OK;
  };
  t.d_scales = c->alloc<float>(t.num_params);
  t.d_mins = c->alloc<float>(t.num_params);
  t.data_cap = t.data_len;
  t.d_data = c->alloc<uint8_t>(t.data_len);
  if (!t.d_scales || !t.d_mins || !t.d_data) return fail(KVF_ERR_CUDA, "allocation failed");
  KVF_TRY(up(t.d_data, data_pos, t.data_len));
  KVF_TRY(up(t.d_scales, scales_pos, t.num_params * 4));
  KVF_TRY(up(t.d_mins, mins_pos, t.num_params * 4));
  if (t.has_freq) {
    t.d_freq = c->alloc<uint32_t>(256);
    if (!t.d_freq) return fail(KVF_ERR_CUDA, "allocation failed");
    KVF_TRY(up(t.d_freq, freq_pos, 256 * 4));
  }
  t.len_known = true;
  return KVF_OK;
}

kvf_status read_status(kvf_ctx* ctx, cudaStream_t st) {
  unsigned bits = 0;
  KVF_CUDA(cudaMemcpyAsync(&bits, ctx->d_status, sizeof(unsigned), cudaMemcpyDeviceToHost, st));
  KVF_CUDA(cudaStreamSynchronize(st));
  if (bits) {
    KVF_CUDA(cudaMemsetAsync(ctx->d_status, 0, sizeof(unsigned), st));
    KVF_CUDA(cudaStreamSynchronize(st));
    if (bits & kDevErrCorrupt) return fail(KVF_ERR_CORRUPT_STREAM, "rANS container failed validation");
    if (bits & kDevErrTimeout) return fail(KVF_ERR_DEVICE_TIMEOUT, "a bounded device wait expired");
    return fail(KVF_ERR_ENTROPY, "entropy model could not be built");
  }
  return KVF_OK;
}

}  // namespace

// =============================================================================
extern "C" {

int kvf_abi_version(void) { return KVF_ABI_VERSION; }
const char* kvf_last_error(void) { return g_err.c_str(); }

kvf_status kvf_init(int device, kvf_ctx** out) {
  if (!out) return fail(KVF_ERR_INVALID_CONFIG, "null output pointer");
  int n = 0;
  KVF_CUDA(cudaGetDeviceCount(&n));
  if (device < 0 || device >= n) return fail(KVF_ERR_CUDA, "device ordinal out of range");
  DeviceGuard g(device);
  if (!g.ok) return fail(KVF_ERR_CUDA, "cudaSetDevice failed");
  auto* ctx = new kvf_ctx();
  ctx->device = device;
  cudaMemPoolProps props{};
  props.allocType = cudaMemAllocationTypePinned;
  props.location.type = cudaMemLocationTypeDevice;
  props.location.id = device;
  cudaError_t e = cudaMemPoolCreate(&ctx->pool, &props);
  if (e == cudaSuccess) {
    uint64_t thr = UINT64_MAX;
    int no = 0;
    e = cudaMemPoolSetAttribute(ctx->pool, cudaMemPoolAttrReleaseThreshold, &thr);
    if (e == cudaSuccess) e = cudaMemPoolSetAttribute(ctx->pool, cudaMemPoolReuseAllowInternalDependencies, &no);
  }
  if (e == cudaSuccess) e = cudaMalloc(&ctx->d_status, sizeof(unsigned));
  if (e == cudaSuccess) e = cudaMemset(ctx->d_status, 0, sizeof(unsigned));
  if (e != cudaSuccess) {
    if (ctx->d_status) cudaFree(ctx->d_status);
    if (ctx->pool) cudaMemPoolDestroy(ctx->pool);
    delete ctx;
    return fail(KVF_ERR_CUDA, std::string("context allocation: ") + cudaGetErrorString(e));
  }
  *out = ctx;
  return KVF_OK;
}

kvf_status kvf_destroy(kvf_ctx* ctx) {
  if (!ctx) return KVF_OK;
  DeviceGuard g(ctx->device);
  for (auto& r : ctx->recs) {
    cudaEventDestroy(r.a);
    cudaEventDestroy(r.b);
  }
  for (auto e : ctx->spare) cudaEventDestroy(e);
  for (auto e : ctx->order_spare) cudaEventDestroy(e);
  for (auto& kv : ctx->sides) {
    cudaStreamSynchronize(kv.second.s);
    cudaStreamDestroy(kv.second.s);
    cudaEventDestroy(kv.second.fork);
    cudaEventDestroy(kv.second.join);
  }
  cudaFree(ctx->d_status);
  // outstanding blocks (compressed objects still alive) keep the pool's
  // memory until they are freed
  if (ctx->pool) cudaMemPoolDestroy(ctx->pool);
  delete ctx;
  return KVF_OK;
}

kvf_status kvf_set_exact_reconstruct(kvf_ctx* ctx, int exact) {
  KVF_TRY(check_ctx(ctx));
  ctx->exact_reconstruct = exact ? 1 : 0;
  return KVF_OK;
}

kvf_status kvf_selftest_wait_timeout(kvf_ctx* ctx, int which, void* stream) {
  KVF_TRY(check_ctx(ctx));
  if (which != KVF_WAIT_MBARRIER && which != KVF_WAIT_LOOKBACK)
    return fail(KVF_ERR_INVALID_CONFIG, "unknown wait kind");
  DeviceGuard g(ctx->device);
  cudaStream_t st = S(stream);
  constexpr unsigned long long kLimitNs = 2000000ull;  // 2 ms
  if (which == KVF_WAIT_MBARRIER) {
    KVF_CUDA(launch_selftest_mbar(ctx->d_status, kLimitNs, st));
  } else {
    Scratch sc(st, ctx->pool);
    unsigned long long* lb = sc.get<unsigned long long>(2);
    if (!lb) return fail(KVF_ERR_CUDA, "scratch allocation failed");
    KVF_CUDA(launch_selftest_lookback(lb, ctx->d_status, kLimitNs, st));
  }
  return KVF_OK;
}

kvf_status kvf_set_projection_engine(kvf_ctx* ctx, int engine) {
  KVF_TRY(check_ctx(ctx));
  if (engine < KVF_PROJ_AUTO || engine > KVF_PROJ_TENSOR_CORE_APPROX)
    return fail(KVF_ERR_INVALID_CONFIG, "unknown projection engine");
  ctx->proj_engine = engine;
  return KVF_OK;
}

kvf_status kvf_set_reconstruct_engine(kvf_ctx* ctx, int engine) {
  KVF_TRY(check_ctx(ctx));
  if (engine != KVF_RECON_AUTO && engine != KVF_RECON_CUDA_CORE && engine != KVF_RECON_TENSOR_CORE)
    return fail(KVF_ERR_INVALID_CONFIG, "unknown reconstruction engine");
  ctx->recon_engine = engine;
  return KVF_OK;
}

kvf_status kvf_sync(kvf_ctx* ctx, void* stream) {
  KVF_TRY(check_ctx(ctx));
  DeviceGuard g(ctx->device);
  KVF_CUDA(cudaStreamSynchronize(S(stream)));
  KVF_CUDA(cudaGetLastError());
  return read_status(ctx, S(stream));
}

uint64_t kvf_launch_count(void) { return kvf::g_launches.load(std::memory_order_relaxed); }

const char* kvf_stage_name(int32_t stage) {
  static const char* names[KVF_NUM_STAGES] = {"calibrate", "project", "quantize", "entropy_encode",
                                              "entropy_decode", "reconstruct", "dequantize", "basis"};
  return (stage >= 0 && stage < KVF_NUM_STAGES) ? names[stage] : "unknown";
}

kvf_status kvf_profile_enable(kvf_ctx* ctx, int enable) {
  KVF_TRY(check_ctx(ctx));
  ctx->profile = enable ? 1 : 0;
  return KVF_OK;
}

kvf_status kvf_profile_read(kvf_ctx* ctx, double* ms, uint64_t* count, double* bytes) {
  KVF_TRY(check_ctx(ctx));
  DeviceGuard g(ctx->device);
  for (int i = 0; i < KVF_NUM_STAGES; ++i) {
    if (ms) ms[i] = 0.0;
    if (count) count[i] = 0;
    if (bytes) bytes[i] = 0.0;
  }
  kvf_status st = KVF_OK;
  std::lock_guard<std::mutex> lock(ctx->mu);
  for (auto& r : ctx->recs) {
    float t = 0.0f;
    cudaError_t e = cudaEventSynchronize(r.b);
    if (e == cudaSuccess) e = cudaEventElapsedTime(&t, r.a, r.b);
    if (e != cudaSuccess && st == KVF_OK) st = fail(KVF_ERR_CUDA, cudaGetErrorString(e));
    if (r.stage >= 0 && r.stage < KVF_NUM_STAGES) {
      if (ms) ms[r.stage] += t;
      if (count) count[r.stage] += 1;
      if (bytes) bytes[r.stage] += r.bytes;
    }
    ctx->spare.push_back(r.a);
    ctx->spare.push_back(r.b);
  }
  ctx->recs.clear();
  return st;
}

kvf_status kvf_pipeline_config_from_preset(int32_t preset, kvf_pipeline_config* out) {
  if (!out) return fail(KVF_ERR_INVALID_CONFIG, "null output pointer");
  kvf_pipeline_config c{};
  c.preset = preset;
  switch (preset) {  // crates/kvforge-core/src/pipeline.rs:31-70
    case KVF_CONSERVATIVE:
      c = {preset, KVF_INT8, KVF_INT8, 0, 0.99, 0, 0};
      break;
    case KVF_BALANCED:
      c = {preset, KVF_INT4, KVF_INT4, 1, 0.90, 0, 0};
      break;
    case KVF_AGGRESSIVE:
      c = {preset, KVF_INT4, KVF_INT4, 1, 0.75, 1, 1};
      break;
    case KVF_ADAPTIVE:
      c = {preset, KVF_INT4, KVF_INT4, 1, 0.90, 1, 1};
      break;
    default:
      return fail(KVF_ERR_INVALID_CONFIG, "unknown preset");
  }
  *out = c;
  return KVF_OK;
}

kvf_status kvf_calibrate(kvf_ctx* ctx, const void* keys, int32_t in_dtype, size_t H, size_t T, size_t D,
                         size_t min_tokens, float* scores, void* stream) {
  KVF_TRY(check_ctx(ctx));
  KVF_TRY(check_dtype(in_dtype));
  KVF_TRY(check_shape(H, T, D));
  if (T < min_tokens)
    return fail(KVF_ERR_INVALID_CONFIG, "Need at least " + std::to_string(min_tokens) +
                                            " tokens for calibration, got " + std::to_string(T));
  DeviceGuard g(ctx->device);
  Scratch sc(S(stream), ctx->pool);
  const size_t tiles = calib_partial_tiles(T, D);
  double* cpart = sc.get<double>(2 * H * tiles);
  if (!cpart) return fail(KVF_ERR_CUDA, "scratch allocation failed");
  KVF_CUDA(launch_calib_partials(keys, in_dtype, H, T, D, cpart, S(stream)));
  KVF_CUDA(launch_calib_finalize(cpart, H, tiles, T, D, scores, S(stream)));
  return KVF_OK;
}

// Same computation as kvf_calibrate; the per-block partials go to a
// file-scope device array instead of the stream-ordered pool (contract in
// include/kvforge.h). No cudaMalloc/cudaFree on this path.
kvf_status kvf_calibrate_noalloc(kvf_ctx* ctx, const void* keys, int32_t in_dtype, size_t H, size_t T, size_t D,
                                 size_t min_tokens, float* scores, void* stream) {
  KVF_TRY(check_ctx(ctx));
  KVF_TRY(check_dtype(in_dtype));
  KVF_TRY(check_shape(H, T, D));
  if (T < min_tokens)
    return fail(KVF_ERR_INVALID_CONFIG, "Need at least " + std::to_string(min_tokens) +
                                            " tokens for calibration, got " + std::to_string(T));
  const size_t tiles = calib_partial_tiles(T, D);
  if (H * tiles > kCalibStaticSlots)
    return fail(KVF_ERR_INVALID_CONFIG, "num_heads * ceil(seq_len * head_dim / 65536) = " +
                                            std::to_string(H * tiles) + " exceeds the " +
                                            std::to_string(kCalibStaticSlots) + " static scratch slots");
  DeviceGuard g(ctx->device);
  if (!g.ok) return fail(KVF_ERR_CUDA, "cudaSetDevice failed");
  double* cpart = nullptr;
  KVF_CUDA(calib_static_scratch(ctx->device, &cpart));
  KVF_CUDA(launch_calib_partials(keys, in_dtype, H, T, D, cpart, S(stream)));
  KVF_CUDA(launch_calib_finalize(cpart, H, tiles, T, D, scores, S(stream)));
  return KVF_OK;
}

kvf_status kvf_quantize(kvf_ctx* ctx, const void* data, int32_t in_dtype, size_t H, size_t T, size_t D,
                        int32_t data_type, int32_t axis, uint8_t* packed, float* scales, float* mins,
                        void* stream) {
  KVF_TRY(check_ctx(ctx));
  KVF_TRY(check_dtype(in_dtype));
  KVF_TRY(check_qcfg(data_type, axis));
  KVF_TRY(check_shape(H, T, D));
  DeviceGuard g(ctx->device);
  Scratch sc(S(stream), ctx->pool);
  return quantize_into(sc, data, in_dtype, H, T, D, data_type, axis, packed, scales, mins, nullptr, S(stream));
}

kvf_status kvf_dequantize(kvf_ctx* ctx, const uint8_t* packed, size_t plen, const float* scales,
                          const float* mins, int32_t data_type, int32_t axis, size_t H, size_t T, size_t D,
                          float* out, void* stream) {
  KVF_TRY(check_ctx(ctx));
  if (data_type == KVF_F32) return fail(KVF_ERR_QUANTIZATION, "Cannot dequantize F32 data type");
  KVF_TRY(check_qcfg(data_type, axis));
  KVF_TRY(check_shape(H, T, D));
  const size_t total = H * T * D;
  // quantize.rs:171-197: INT4 unpacks 2 values per byte then truncates
  const size_t got = data_type == KVF_INT4 ? std::min(2 * plen, total) : plen;
  if (got != total)
    return fail(KVF_ERR_QUANTIZATION, "Expected " + std::to_string(total) + " values, got " +
                                          std::to_string(data_type == KVF_INT4 ? 2 * plen : plen));
  DeviceGuard g(ctx->device);
  KVF_CUDA(launch_dequantize(packed, scales, mins, data_type, axis, H, T, D, out, S(stream)));
  return KVF_OK;
}

kvf_status kvf_project(kvf_ctx* ctx, const void* data, int32_t in_dtype, size_t H, size_t T, size_t D,
                       const float* basis_vt, const uint64_t* ranks, size_t R, float* projected,
                       void* stream) {
  KVF_TRY(check_ctx(ctx));
  KVF_TRY(check_dtype(in_dtype));
  KVF_TRY(check_shape(H, T, D));
  if (T == 0 || D == 0) return fail(KVF_ERR_PROJECTION, "Cannot project empty tensor");
  if (R == 0 || R > D) return fail(KVF_ERR_PROJECTION, "projected width must be in 1..head_dim");
  DeviceGuard g(ctx->device);
  ProjectOut po;
  po.status = ctx->d_status;
  po.P = projected;
  KVF_CUDA(launch_project(data, in_dtype, H, T, D, basis_vt, ranks, R, po, S(stream)));
  return KVF_OK;
}

kvf_status kvf_reconstruct(kvf_ctx* ctx, const float* projected, size_t H, size_t T, size_t R, size_t D,
                           const float* basis_vt, const uint64_t* ranks, float* out, void* stream) {
  KVF_TRY(check_ctx(ctx));
  KVF_TRY(check_shape(H, T, D));
  if (R == 0 || R > D) return fail(KVF_ERR_PROJECTION, "projected width must be in 1..head_dim");
  DeviceGuard g(ctx->device);
  KVF_CUDA(launch_dequant_reconstruct(nullptr, projected, nullptr, nullptr, KVF_F32, KVF_PER_TOKEN, H, T, R, D,
                                      basis_vt, ranks, ctx->exact_reconstruct,
                                      ctx->recon_engine, out, ctx->d_status, S(stream)));
  return KVF_OK;
}

kvf_status kvf_fused_project_quantize(kvf_ctx* ctx, const void* data, int32_t in_dtype, size_t H, size_t T,
                                      size_t D, const float* basis_vt, const uint64_t* ranks, size_t R,
                                      int32_t data_type, int32_t axis, uint8_t* packed, float* scales,
                                      float* mins, void* stream) {
  KVF_TRY(check_ctx(ctx));
  KVF_TRY(check_dtype(in_dtype));
  KVF_TRY(check_qcfg(data_type, axis));
  KVF_TRY(check_shape(H, T, D));
  if (T == 0 || D == 0) return fail(KVF_ERR_PROJECTION, "Cannot project empty tensor");
  if (R == 0 || R > D) return fail(KVF_ERR_PROJECTION, "projected width must be in 1..head_dim");
  DeviceGuard g(ctx->device);
  Scratch sc(S(stream), ctx->pool);
  cudaStream_t st = S(stream);
  const size_t n = H * T * R;
  ProjectOut po;
  po.status = ctx->d_status;
  po.levels = quant_levels(data_type);
  if (axis == KVF_PER_CHANNEL) {
    float* P = sc.get<float>(n);
    int* keys = sc.get<int>(2 * H * R);
    if (!P || !keys) return fail(KVF_ERR_CUDA, "scratch allocation failed");
    KVF_CUDA(launch_minmax_init(keys, keys + H * R, H * R, st));
    po.mode = 1;
    po.P = P;
    po.kmin = keys;
    po.kmax = keys + H * R;
    KVF_CUDA(launch_project(data, in_dtype, H, T, D, basis_vt, ranks, R, po, st));
    KVF_CUDA(launch_quantpack_channel(P, H, T, R, po.kmin, po.kmax, data_type, scales, mins, packed, nullptr, st));
    return KVF_OK;
  }
  if (R <= 32 || token_tc(ctx, data, in_dtype, H, T, D, basis_vt, R)) {
    const bool fuse_pack = token_fuse_pack(token_tc(ctx, data, in_dtype, H, T, D, basis_vt, R), data_type, R, T);
    uint8_t* codes = (data_type == KVF_INT8) ? packed : (fuse_pack ? nullptr : sc.get<uint8_t>(n));
    if (data_type == KVF_INT4 && !fuse_pack && !codes) return fail(KVF_ERR_CUDA, "scratch allocation failed");
    po.mode = 2;
    po.codes = codes;
    po.packed = fuse_pack ? packed : nullptr;
    po.scales = scales;
    po.mins = mins;
    KVF_CUDA(project_token(ctx, data, in_dtype, H, T, D, basis_vt, ranks, R, po, st));
    if (data_type == KVF_INT4 && !fuse_pack) KVF_CUDA(launch_pack_int4(codes, n, packed, nullptr, st));
    return KVF_OK;
  }
  float* P = sc.get<float>(n);
  if (!P) return fail(KVF_ERR_CUDA, "scratch allocation failed");
  po.P = P;
  KVF_CUDA(launch_project(data, in_dtype, H, T, D, basis_vt, ranks, R, po, st));
  return quantize_into(sc, P, KVF_IN_F32, H, T, R, data_type, axis, packed, scales, mins, nullptr, st);
}

size_t kvf_rans_max_encoded_len(size_t n) { return rans_max_len(n, kRansChunk); }

kvf_status kvf_rans_encode(kvf_ctx* ctx, const uint8_t* data, size_t n, uint8_t* out, size_t out_cap,
                           size_t* out_len_host, uint32_t* freq, void* stream) {
  KVF_TRY(check_ctx(ctx));
  if (!out_len_host) return fail(KVF_ERR_INVALID_CONFIG, "null length pointer");
  DeviceGuard g(ctx->device);
  cudaStream_t st = S(stream);
  KVF_CUDA(cudaMemsetAsync(freq, 0, 256 * sizeof(uint32_t), st));
  if (n == 0) {
    *out_len_host = 0;
    return KVF_OK;
  }
  if (out_cap < rans_max_len(n, kRansChunk)) return fail(KVF_ERR_ENTROPY, "output capacity too small");
  if (!aligned(out, 4)) return fail(KVF_ERR_INVALID_CONFIG, "output buffer must be 4-byte aligned");
  Scratch sc(st, ctx->pool);
  uint64_t* d_len = sc.get<uint64_t>(1);
  if (!d_len) return fail(KVF_ERR_CUDA, "scratch allocation failed");
  KVF_CUDA(launch_histogram(data, n, freq, st));
  KVF_TRY(rans_encode_into(ctx, sc, data, n, freq, out, d_len, st));
  uint64_t len = 0;
  KVF_CUDA(cudaMemcpyAsync(&len, d_len, sizeof(uint64_t), cudaMemcpyDeviceToHost, st));
  KVF_TRY(read_status(ctx, st));
  *out_len_host = (size_t)len;
  return KVF_OK;
}

kvf_status kvf_rans_decode(kvf_ctx* ctx, const uint8_t* comp, size_t comp_len, const uint32_t* freq,
                           size_t original_len, uint8_t* out, void* stream) {
  KVF_TRY(check_ctx(ctx));
  if (original_len == 0) return KVF_OK;
  if (comp_len % 4 != 0) return fail(KVF_ERR_ENTROPY, "Compressed data length not aligned to 4 bytes");
  if (!aligned(comp, 4)) return fail(KVF_ERR_INVALID_CONFIG, "container must be 4-byte aligned");
  DeviceGuard g(ctx->device);
  cudaStream_t st = S(stream);
  Scratch sc(st, ctx->pool);
  KVF_CUDA(launch_rans_decode(comp, comp_len, nullptr, freq, original_len, out, ctx->d_status, st));
  return read_status(ctx, st);
}

kvf_status kvf_entropy_decode_dequant(kvf_ctx* ctx, const uint8_t* comp, size_t comp_len,
                                      const uint32_t* freq, const float* scales, const float* mins,
                                      int32_t data_type, int32_t axis, size_t H, size_t T, size_t D,
                                      float* out, void* stream) {
  KVF_TRY(check_ctx(ctx));
  KVF_TRY(check_qcfg(data_type, axis));
  KVF_TRY(check_shape(H, T, D));
  if (comp_len % 4 != 0) return fail(KVF_ERR_ENTROPY, "Compressed data length not aligned to 4 bytes");
  if (!aligned(comp, 4)) return fail(KVF_ERR_INVALID_CONFIG, "container must be 4-byte aligned");
  const size_t plen = packed_len(H * T * D, data_type);
  if (plen == 0) return KVF_OK;
  DeviceGuard g(ctx->device);
  cudaStream_t st = S(stream);
  Scratch sc(st, ctx->pool);
  uint8_t* dec = sc.get<uint8_t>(plen);
  if (!dec) return fail(KVF_ERR_CUDA, "scratch allocation failed");
  KVF_CUDA(launch_rans_decode(comp, comp_len, nullptr, freq, plen, dec, ctx->d_status, st));
  KVF_CUDA(launch_dequantize(dec, scales, mins, data_type, axis, H, T, D, out, st));
  return KVF_OK;
}

// ---- fused dequantize + decode attention ------------------------------------
namespace {
kvf_status check_attention(size_t H, size_t T, size_t D, size_t Rk, size_t Rv, int kdt, int vdt, bool kproj,
                           bool vproj) {
  KVF_TRY(check_shape(H, T, D));
  if ((kdt != KVF_INT4 && kdt != KVF_INT8) || (vdt != KVF_INT4 && vdt != KVF_INT8))
    return fail(KVF_ERR_INVALID_CONFIG, "attention takes INT4 or INT8 codes");
  if (D == 0 || Rk == 0 || Rv == 0) return fail(KVF_ERR_SHAPE_MISMATCH, "empty head or coefficient width");
  if ((!kproj && Rk != D) || (!vproj && Rv != D) || Rk > D || Rv > D)
    return fail(KVF_ERR_SHAPE_MISMATCH, "coefficient width must be head_dim without a basis, at most head_dim with one");
  if ((attention_tiles(T) + Rv) * sizeof(float) > 200 * 1024)
    return fail(KVF_ERR_SHAPE_MISMATCH, "sequence too long for one attention call");
  return KVF_OK;
}
}  // namespace

kvf_status kvf_fused_dequant_attention(kvf_ctx* ctx, const uint8_t* k_codes, const uint8_t* v_codes,
                                       const float* query, const float* k_scales, const float* k_mins,
                                       const float* v_scales, const float* v_mins, int32_t k_data_type,
                                       int32_t v_data_type, size_t H, size_t T, size_t D, size_t k_cols,
                                       size_t v_cols, const float* k_basis_vt, const uint64_t* k_ranks,
                                       const float* v_basis_vt, const uint64_t* v_ranks, float scale, float* out,
                                       void* stream) {
  KVF_TRY(check_ctx(ctx));
  if (H && D && (!query || !out)) return fail(KVF_ERR_INVALID_CONFIG, "null pointer");
  if ((k_basis_vt && !k_ranks) || (v_basis_vt && !v_ranks)) return fail(KVF_ERR_INVALID_CONFIG, "basis without ranks");
  if (H == 0) return KVF_OK;
  KVF_TRY(check_attention(H, T, D, k_cols, v_cols, k_data_type, v_data_type, k_basis_vt != nullptr,
                          v_basis_vt != nullptr));
  if (T && (!k_codes || !v_codes || !k_scales || !k_mins || !v_scales || !v_mins))
    return fail(KVF_ERR_INVALID_CONFIG, "null pointer");
  DeviceGuard g(ctx->device);
  cudaStream_t st = S(stream);
  Scratch sc(st, ctx->pool);
  float* part = sc.get<float>(attention_scratch_floats(H, T, v_cols));
  if (!part) return fail(KVF_ERR_CUDA, "scratch allocation failed");
  KVF_CUDA(launch_attention(k_codes, k_data_type, v_codes, v_data_type, query, k_scales, k_mins, v_scales, v_mins,
                            k_basis_vt, k_ranks, v_basis_vt, v_ranks, H, T, D, k_cols, v_cols, scale, part, out, st));
  return KVF_OK;
}

namespace {
kvf_status compressed_attention_body(kvf_ctx* ctx, const kvf_compressed* c, const float* query, float scale,
                                     float* out, cudaStream_t st);
}  // namespace

kvf_status kvf_compressed_attention(kvf_ctx* ctx, const kvf_compressed* c, const float* query, float scale,
                                    float* out, void* stream) {
  KVF_TRY(check_ctx(ctx));
  if (!c) return fail(KVF_ERR_INVALID_CONFIG, "null compressed object");
  const TensorC& k = c->key;
  const TensorC& v = c->value;
  if (k.axis != KVF_PER_CHANNEL || v.axis != KVF_PER_TOKEN)
    return fail(KVF_ERR_INVALID_CONFIG, "attention takes per-channel keys and per-token values");
  if (c->H && c->D && (!query || !out)) return fail(KVF_ERR_INVALID_CONFIG, "null pointer");
  if (c->H == 0) return KVF_OK;
  KVF_TRY(check_attention(c->H, c->T, c->D, k.qcols, v.qcols, k.data_type, v.data_type, k.basis != nullptr,
                          v.basis != nullptr));
  DeviceGuard g(ctx->device);
  cudaStream_t st = S(stream);
  KVF_TRY(reader_enter(c, st));
  const kvf_status s = compressed_attention_body(ctx, c, query, scale, out, st);
  const kvf_status ls = reader_leave(c, st);
  return s != KVF_OK ? s : ls;
}

namespace {
kvf_status compressed_attention_body(kvf_ctx* ctx, const kvf_compressed* c, const float* query, float scale,
                                     float* out, cudaStream_t st) {
  const TensorC& k = c->key;
  const TensorC& v = c->value;
  Scratch sc(st, ctx->pool);
  // entropy-coded tensors are decoded into scratch (allocated on `st` before
  // the fork, freed on `st` after the join): keys on `st`, values on the
  // context's side stream, so the two decodes overlap
  const uint8_t* codes[2] = {k.d_data, v.d_data};
  const TensorC* ts[2] = {&k, &v};
  uint8_t* dec[2] = {nullptr, nullptr};
  for (int i = 0; i < 2; ++i)
    if (ts[i]->has_freq && !(dec[i] = sc.get<uint8_t>(ts[i]->packed_len)))
      return fail(KVF_ERR_CUDA, "scratch allocation failed");
  float* part = sc.get<float>(attention_scratch_floats(c->H, c->T, v.qcols));
  if (!part) return fail(KVF_ERR_CUDA, "scratch allocation failed");
  if (dec[0] || dec[1]) {
    kvf_ctx::Side* sd = nullptr;
    KVF_CUDA(ctx->side_for(st, &sd));
    KVF_CUDA(cudaEventRecord(sd->fork, st));
    KVF_CUDA(cudaStreamWaitEvent(sd->s, sd->fork, 0));
    cudaError_t e = cudaSuccess;
    for (int i = 0; i < 2 && e == cudaSuccess; ++i) {
      const TensorC& t = *ts[i];
      if (!dec[i]) continue;
      e = launch_rans_decode(t.d_data, t.data_len, t.len_known ? nullptr : t.d_len, t.d_freq, t.packed_len, dec[i],
                             ctx->d_status, i == 0 ? st : sd->s);
      codes[i] = dec[i];
    }
    cudaError_t je = cudaEventRecord(sd->join, sd->s);
    if (je == cudaSuccess) je = cudaStreamWaitEvent(st, sd->join, 0);
    KVF_CUDA(e);
    KVF_CUDA(je);
  }
  KVF_CUDA(launch_attention(codes[0], k.data_type, codes[1], v.data_type, query, k.d_scales, k.d_mins, v.d_scales,
                            v.d_mins, k.basis ? k.basis->d_vt : nullptr, k.basis ? k.basis->d_ranks : nullptr,
                            v.basis ? v.basis->d_vt : nullptr, v.basis ? v.basis->d_ranks : nullptr, c->H, c->T,
                            c->D, k.qcols, v.qcols, scale, part, out, st));
  return KVF_OK;
}
}  // namespace

// ---- basis ------------------------------------------------------------------
kvf_status kvf_basis_compute(kvf_ctx* ctx, const void* data, int32_t in_dtype, size_t H, size_t T, size_t D,
                             double variance_threshold, size_t max_rank, kvf_basis** out, void* stream) {
  KVF_TRY(check_ctx(ctx));
  KVF_TRY(check_dtype(in_dtype));
  KVF_TRY(check_shape(H, T, D));
  if (!out) return fail(KVF_ERR_INVALID_CONFIG, "null output pointer");
  DeviceGuard g(ctx->device);
  std::shared_ptr<BasisData> b;
  KVF_TRY(compute_basis(ctx, data, in_dtype, H, T, D, variance_threshold, max_rank, &b, S(stream)));
  *out = new kvf_basis{b};
  return KVF_OK;
}

kvf_status kvf_basis_from_host(kvf_ctx* ctx, size_t H, size_t R, size_t D, const float* basis_vt_host,
                               const uint64_t* ranks_host, kvf_basis** out) {
  KVF_TRY(check_ctx(ctx));
  if (!out || (H && (!basis_vt_host || !ranks_host))) return fail(KVF_ERR_INVALID_CONFIG, "null pointer");
  if (R == 0 || R > D) return fail(KVF_ERR_PROJECTION, "projected width must be in 1..head_dim");
  DeviceGuard g(ctx->device);
  auto b = std::make_shared<BasisData>();
  b->device = ctx->device;
  b->H = H; b->R = R; b->D = D;
  b->vt.assign(basis_vt_host, basis_vt_host + H * R * D);
  b->ranks.assign(ranks_host, ranks_host + H);
  for (uint64_t r : b->ranks)
    if (r > R) return fail(KVF_ERR_PROJECTION, "rank exceeds the projected width");
  KVF_TRY(upload_basis(*b));
  *out = new kvf_basis{b};
  return KVF_OK;
}

kvf_status kvf_basis_info(const kvf_basis* b, size_t* H, size_t* R, size_t* D) {
  if (!b) return fail(KVF_ERR_INVALID_CONFIG, "null basis");
  if (H) *H = b->d->H;
  if (R) *R = b->d->R;
  if (D) *D = b->d->D;
  return KVF_OK;
}

kvf_status kvf_basis_download(const kvf_basis* b, float* vt, uint64_t* ranks, float* sv) {
  if (!b) return fail(KVF_ERR_INVALID_CONFIG, "null basis");
  const BasisData& d = *b->d;
  if (vt) std::memcpy(vt, d.vt.data(), d.vt.size() * sizeof(float));
  if (ranks) std::memcpy(ranks, d.ranks.data(), d.H * sizeof(uint64_t));
  if (sv) {
    if (d.sv.empty()) std::memset(sv, 0, d.H * d.D * sizeof(float));
    else std::memcpy(sv, d.sv.data(), d.sv.size() * sizeof(float));
  }
  return KVF_OK;
}

const float* kvf_basis_device_vt(const kvf_basis* b) { return b ? b->d->d_vt : nullptr; }
const uint64_t* kvf_basis_device_ranks(const kvf_basis* b) { return b ? b->d->d_ranks : nullptr; }

kvf_status kvf_basis_free(kvf_basis* b) {
  delete b;
  return KVF_OK;
}

// ---- whole layer --------------------------------------------------------------
namespace {
// a layer of at most this many elements per tensor runs keys and values on
// one stream (a 64-token chunk of 8 heads is 65536)
constexpr size_t kSmallLayerElems = size_t(1) << 20;
bool small_layer(size_t H, size_t T, size_t D) { return H * T * D <= kSmallLayerElems; }
}  // namespace

kvf_status kvf_compress_layer(kvf_ctx* ctx, const void* keys, const void* values, int32_t in_dtype, size_t H,
                              size_t T, size_t D, size_t layer_idx, const kvf_pipeline_config* cfg,
                              const kvf_basis* k_basis, const kvf_basis* v_basis, kvf_compressed** out,
                              void* stream) {
  KVF_TRY(check_ctx(ctx));
  KVF_TRY(check_dtype(in_dtype));
  KVF_TRY(check_shape(H, T, D));
  if (!cfg || !out) return fail(KVF_ERR_INVALID_CONFIG, "null pointer");
  DeviceGuard g(ctx->device);
  cudaStream_t st = S(stream);
  std::unique_ptr<kvf_compressed> c(new kvf_compressed());
  c->ctx = ctx;
  c->device = ctx->device;
  c->stream = st;
  c->layer_idx = layer_idx;
  c->H = H; c->T = T; c->D = D;
  c->original_size_bytes = 2 * H * T * D * 4;  // KVCache::size_bytes, f32 (types.rs:30-32)
  std::shared_ptr<BasisData> kb, vb;
  if (cfg->enable_projection) {
    if (k_basis) kb = k_basis->d;
    else KVF_TRY(compute_basis(ctx, keys, in_dtype, H, T, D, cfg->projection_variance_threshold, 0, &kb, st));
    if (v_basis) vb = v_basis->d;
    else KVF_TRY(compute_basis(ctx, values, in_dtype, H, T, D, cfg->projection_variance_threshold, 0, &vb, st));
  }
  if (cfg->enable_calibration && T >= 64 && H > 0) {
    c->d_scores = c->alloc<float>(H);
    if (!c->d_scores) return fail(KVF_ERR_CUDA, "allocation failed");
  }
  // keys on the caller's stream, values on its side stream, joined before
  // return; a small layer keeps both on the caller's stream (its kernels are
  // too short to gain from overlapping, and the fork and join cost API calls)
  kvf_ctx::Side* sd = nullptr;
  cudaStream_t vst = st;
  if (!small_layer(H, T, D)) {
    KVF_CUDA(ctx->side_for(st, &sd));
    KVF_CUDA(cudaEventRecord(sd->fork, st));
    KVF_CUDA(cudaStreamWaitEvent(sd->s, sd->fork, 0));
    vst = sd->s;
  }
  kvf_status s = compress_tensor(ctx, c.get(), keys, in_dtype, H, T, D, cfg->key_data_type, KVF_PER_CHANNEL, kb,
                                 cfg->enable_entropy_coding != 0, cfg->enable_calibration != 0, c->d_scores,
                                 &c->key, st);
  if (s == KVF_OK)
    s = compress_tensor(ctx, c.get(), values, in_dtype, H, T, D, cfg->value_data_type, KVF_PER_TOKEN, vb,
                        cfg->enable_entropy_coding != 0, false, nullptr, &c->value, vst);
  cudaError_t je = cudaSuccess;
  if (sd) {
    je = cudaEventRecord(sd->join, sd->s);
    if (je == cudaSuccess) je = cudaStreamWaitEvent(st, sd->join, 0);
  }
  if (s == KVF_OK && je != cudaSuccess) s = fail(KVF_ERR_CUDA, cudaGetErrorString(je));
  if (s == KVF_OK) s = mark_ready(c.get());
  if (s != KVF_OK) {
    std::string msg = g_err;
    kvf_compressed_free(c.release());
    g_err = msg;
    return s;
  }
  *out = c.release();
  return KVF_OK;
}

kvf_status kvf_decompress_layer(kvf_ctx* ctx, const kvf_compressed* c, float* keys_out, float* values_out,
                                void* stream) {
  KVF_TRY(check_ctx(ctx));
  if (!c) return fail(KVF_ERR_INVALID_CONFIG, "null compressed object");
  DeviceGuard g(ctx->device);
  cudaStream_t st = S(stream);
  KVF_TRY(reader_enter(c, st));
  kvf_ctx::Side* sd = nullptr;
  cudaStream_t vst = st;
  if (!small_layer(c->H, c->T, c->D)) {  // as in kvf_compress_layer
    KVF_CUDA(ctx->side_for(st, &sd));
    KVF_CUDA(cudaEventRecord(sd->fork, st));
    KVF_CUDA(cudaStreamWaitEvent(sd->s, sd->fork, 0));
    vst = sd->s;
  }
  kvf_status s = decompress_tensor(ctx, c->key, keys_out, st);
  if (s == KVF_OK) s = decompress_tensor(ctx, c->value, values_out, vst);
  cudaError_t je = cudaSuccess;
  if (sd) {
    je = cudaEventRecord(sd->join, sd->s);
    if (je == cudaSuccess) je = cudaStreamWaitEvent(st, sd->join, 0);
  }
  if (s == KVF_OK && je != cudaSuccess) s = fail(KVF_ERR_CUDA, cudaGetErrorString(je));
  const kvf_status ls = reader_leave(c, st);  // even after a failure: launched kernels may still read
  return s != KVF_OK ? s : ls;
}

namespace {
// the per-layer path for every layer (shapes or configurations the batched
// kernel does not take)
kvf_status compress_layers_each(kvf_ctx* ctx, size_t L, const void* const* keys, const void* const* values,
                                int32_t in_dtype, size_t H, size_t T, size_t D, const size_t* layer_idx,
                                const kvf_pipeline_config* cfg, const kvf_basis* const* k_bases,
                                const kvf_basis* const* v_bases, kvf_compressed** out, float* const* keys_out,
                                float* const* values_out, void* stream) {
  for (size_t l = 0; l < L; ++l) {
    KVF_TRY(kvf_compress_layer(ctx, keys[l], values[l], in_dtype, H, T, D, layer_idx ? layer_idx[l] : l, cfg,
                               k_bases ? k_bases[l] : nullptr, v_bases ? v_bases[l] : nullptr, &out[l], stream));
    if (keys_out && values_out)
      KVF_TRY(kvf_decompress_layer(ctx, out[l], keys_out[l], values_out[l], stream));
  }
  return KVF_OK;
}
}  // namespace

kvf_status kvf_compress_layers(kvf_ctx* ctx, size_t L, const void* const* keys, const void* const* values,
                               int32_t in_dtype, size_t H, size_t T, size_t D, const size_t* layer_idx,
                               const kvf_pipeline_config* cfg, const kvf_basis* const* k_bases,
                               const kvf_basis* const* v_bases, kvf_compressed** out, float* const* keys_out,
                               float* const* values_out, void* stream) {
  KVF_TRY(check_ctx(ctx));
  KVF_TRY(check_dtype(in_dtype));
  KVF_TRY(check_shape(H, T, D));
  if (!cfg || !out || (L && (!keys || !values))) return fail(KVF_ERR_INVALID_CONFIG, "null pointer");
  if ((keys_out == nullptr) != (values_out == nullptr))
    return fail(KVF_ERR_INVALID_CONFIG, "decompression outputs: give both keys_out and values_out, or neither");
  for (size_t l = 0; l < L; ++l) out[l] = nullptr;
  if (L == 0) return KVF_OK;
  KVF_TRY(check_qcfg(cfg->key_data_type, KVF_PER_CHANNEL));
  KVF_TRY(check_qcfg(cfg->value_data_type, KVF_PER_TOKEN));
  DeviceGuard g(ctx->device);
  cudaStream_t st = S(stream);
  const bool proj = cfg->enable_projection != 0;
  // the batched kernel covers projection with given bases, no entropy coding
  // and no calibration (whose result the reference discards, pipeline.rs:104-111)
  bool batch = !cfg->enable_entropy_coding && !(cfg->enable_calibration && T >= 64);
  size_t qmax = D;
  if (batch && proj) {
    if (!k_bases || !v_bases) batch = false;
    qmax = 0;
    for (size_t l = 0; batch && l < L; ++l)
      for (const kvf_basis* b : {k_bases[l], v_bases[l]}) {
        if (!b || b->d->H != H || b->d->D != D) {
          batch = false;
          break;
        }
        qmax = std::max(qmax, b->d->R);
        if (H > 1 && (T * b->d->R) % 2) batch = false;
      }
  }
  if (batch) batch = chunk_batch_fits(in_dtype, H, T, D, qmax, proj);
  // rows are read 16 bytes (f32) or 8 bytes (f16) at a time
  const uintptr_t amask = in_dtype == KVF_IN_F32 ? 15 : 7;
  for (size_t l = 0; batch && l < L; ++l)
    if (!keys[l] || !values[l] || ((reinterpret_cast<uintptr_t>(keys[l]) | reinterpret_cast<uintptr_t>(values[l])) & amask))
      batch = false;
  // decompressed rows are written 16 bytes at a time
  for (size_t l = 0; batch && keys_out && l < L; ++l)
    if (!keys_out[l] || !values_out[l] ||
        ((reinterpret_cast<uintptr_t>(keys_out[l]) | reinterpret_cast<uintptr_t>(values_out[l])) & 15))
      batch = false;
  if (!batch)
    return compress_layers_each(ctx, L, keys, values, in_dtype, H, T, D, layer_idx, cfg, k_bases, v_bases, out,
                                keys_out, values_out, stream);

  std::vector<std::unique_ptr<kvf_compressed>> cs(L);
  std::vector<BatchTensor> desc(2 * L);
  auto release = [&](kvf_status s) {
    std::string msg = g_err;
    for (auto& c : cs)
      if (c) kvf_compressed_free(c.release());
    g_err = msg;
    return s;
  };
  // every layer's parameters and codes in one pool allocation: per tensor
  // scales, mins, codes at offsets off[l][which][0..2]
  std::vector<std::array<std::array<size_t, 3>, 2>> off(L);
  size_t total = 0;
  for (size_t l = 0; l < L; ++l)
    for (int which = 0; which < 2; ++which) {
      const int dt = which ? cfg->value_data_type : cfg->key_data_type;
      const size_t q = proj ? (which ? v_bases[l] : k_bases[l])->d->R : D;
      const size_t sp = align_up(num_params(H, T, q, which ? KVF_PER_TOKEN : KVF_PER_CHANNEL) * 4, kScratchAlign);
      off[l][which] = {total, total + sp, total + 2 * sp};
      total += 2 * sp + align_up(std::max<size_t>(packed_len(H * T * q, dt), 1), kScratchAlign);
    }
  auto block = std::make_shared<SharedBlock>();
  block->ctx = ctx;
  block->device = ctx->device;
  block->stream = st;
  if (cudaMallocFromPoolAsync(&block->p, total, ctx->pool, st) != cudaSuccess) {
    block->p = nullptr;
    return fail(KVF_ERR_CUDA, "allocation failed");
  }
  for (size_t l = 0; l < L; ++l) {
    cs[l].reset(new kvf_compressed());
    kvf_compressed* c = cs[l].get();
    c->ctx = ctx;
    c->device = ctx->device;
    c->stream = st;
    c->block = block;
    c->layer_idx = layer_idx ? layer_idx[l] : l;
    c->H = H; c->T = T; c->D = D;
    c->original_size_bytes = 2 * H * T * D * 4;  // KVCache::size_bytes, f32 (types.rs:30-32)
    for (int which = 0; which < 2; ++which) {
      TensorC& t = which ? c->value : c->key;
      t.data_type = which ? cfg->value_data_type : cfg->key_data_type;
      t.axis = which ? KVF_PER_TOKEN : KVF_PER_CHANNEL;
      t.H = H; t.T = T; t.D = D;
      t.entropy = false;
      t.has_freq = false;
      if (proj) t.basis = (which ? v_bases[l] : k_bases[l])->d;
      t.qcols = proj ? t.basis->R : D;
      t.packed_len = packed_len(H * T * t.qcols, t.data_type);
      t.num_params = num_params(H, T, t.qcols, t.axis);
      uint8_t* base = static_cast<uint8_t*>(block->p);
      t.d_scales = reinterpret_cast<float*>(base + off[l][which][0]);
      t.d_mins = reinterpret_cast<float*>(base + off[l][which][1]);
      t.d_data = base + off[l][which][2];
      t.data_cap = t.data_len = t.packed_len;
      t.len_known = true;
      BatchTensor& bt = desc[2 * l + which];
      bt.x = which ? values[l] : keys[l];
      bt.bvt = proj ? t.basis->d_vt : nullptr;
      bt.ranks = proj ? t.basis->d_ranks : nullptr;
      bt.cols = (int)t.qcols;
      bt.axis = t.axis;
      bt.data_type = t.data_type;
      bt.levels = quant_levels(t.data_type);
      bt.packed = t.d_data;
      bt.scales = t.d_scales;
      bt.mins = t.d_mins;
      bt.out = keys_out ? (which ? values_out[l] : keys_out[l]) : nullptr;
    }
  }
  {
    const cudaError_t e = launch_chunk_batch(desc.data(), L, in_dtype, H, T, D, qmax, proj, ctx->exact_reconstruct, st);
    if (e != cudaSuccess) return release(fail(KVF_ERR_CUDA, std::string("batched chunks: ") + cudaGetErrorString(e)));
  }
  // one ready event for all objects of the call
  {
    cudaError_t e = ctx->order_event(&block->ready);
    if (e == cudaSuccess) e = cudaEventRecord(block->ready, st);
    if (e != cudaSuccess) return release(fail(KVF_ERR_CUDA, std::string("ready event: ") + cudaGetErrorString(e)));
  }
  for (size_t l = 0; l < L; ++l) {
    cs[l]->ready = block->ready;
    out[l] = cs[l].release();
  }
  return KVF_OK;
}

kvf_status kvf_compress_layer_host(kvf_ctx* ctx, const void* keys_host, const void* values_host, int32_t in_dtype,
                                   size_t H, size_t T, size_t D, size_t layer_idx, const kvf_pipeline_config* cfg,
                                   const kvf_basis* k_basis, const kvf_basis* v_basis, kvf_compressed** out,
                                   void* stream) {
  KVF_TRY(check_ctx(ctx));
  KVF_TRY(check_dtype(in_dtype));
  DeviceGuard g(ctx->device);
  cudaStream_t st = S(stream);
  const size_t bytes = H * T * D * (in_dtype == KVF_IN_F16 ? 2 : 4);
  kvf_status s;
  {
    Scratch sc(st, ctx->pool);
    uint8_t* dk = sc.get<uint8_t>(bytes);
    uint8_t* dv = sc.get<uint8_t>(bytes);
    if (!dk || !dv) return fail(KVF_ERR_CUDA, "scratch allocation failed");
    if (bytes) {
      KVF_CUDA(cudaMemcpyAsync(dk, keys_host, bytes, cudaMemcpyHostToDevice, st));
      KVF_CUDA(cudaMemcpyAsync(dv, values_host, bytes, cudaMemcpyHostToDevice, st));
    }
    s = kvf_compress_layer(ctx, dk, dv, in_dtype, H, T, D, layer_idx, cfg, k_basis, v_basis, out, stream);
  }
  if (s != KVF_OK) return s;
  KVF_CUDA(cudaStreamSynchronize(st));
  return KVF_OK;
}

kvf_status kvf_decompress_layer_host(kvf_ctx* ctx, const kvf_compressed* c, float* keys_host, float* values_host,
                                     void* stream) {
  KVF_TRY(check_ctx(ctx));
  if (!c) return fail(KVF_ERR_INVALID_CONFIG, "null compressed object");
  DeviceGuard g(ctx->device);
  cudaStream_t st = S(stream);
  const size_t bytes = c->H * c->T * c->D * 4;
  {
    Scratch sc(st, ctx->pool);
    float* dk = sc.get<float>(c->H * c->T * c->D);
    float* dv = sc.get<float>(c->H * c->T * c->D);
    if (!dk || !dv) return fail(KVF_ERR_CUDA, "scratch allocation failed");
    KVF_TRY(kvf_decompress_layer(ctx, c, dk, dv, stream));
    if (bytes) {
      KVF_CUDA(cudaMemcpyAsync(keys_host, dk, bytes, cudaMemcpyDeviceToHost, st));
      KVF_CUDA(cudaMemcpyAsync(values_host, dv, bytes, cudaMemcpyDeviceToHost, st));
    }
  }
  KVF_CUDA(cudaStreamSynchronize(st));
  return read_status(ctx, st);
}

kvf_status kvf_compressed_shape(const kvf_compressed* c, size_t* H, size_t* T, size_t* D, size_t* layer_idx) {
  if (!c) return fail(KVF_ERR_INVALID_CONFIG, "null compressed object");
  if (H) *H = c->H;
  if (T) *T = c->T;
  if (D) *D = c->D;
  if (layer_idx) *layer_idx = c->layer_idx;
  return KVF_OK;
}

kvf_status kvf_compressed_size_bytes(kvf_compressed* c, size_t* out) {
  if (!c || !out) return fail(KVF_ERR_INVALID_CONFIG, "null pointer");
  DeviceGuard g(c->device);
  KVF_TRY(resolve_len(c->key, c->stream));
  KVF_TRY(resolve_len(c->value, c->stream));
  *out = tensor_size(c->key) + tensor_size(c->value);
  return KVF_OK;
}

// ProjectionState::size_bytes (types.rs:131-135) of both tensors
kvf_status kvf_compressed_basis_bytes(const kvf_compressed* c, size_t* out) {
  if (!c || !out) return fail(KVF_ERR_INVALID_CONFIG, "null pointer");
  size_t total = 0;
  for (const TensorC* t : {&c->key, &c->value})
    if (t->basis) total += t->H * t->basis->R * t->D * 4 + t->H * 8;
  *out = total;
  return KVF_OK;
}

kvf_status kvf_compressed_basis(const kvf_compressed* c, int32_t which, kvf_basis** out) {
  if (!c || !out || (which != 0 && which != 1)) return fail(KVF_ERR_INVALID_CONFIG, "bad arguments");
  const TensorC& t = which == 0 ? c->key : c->value;
  *out = t.basis ? new kvf_basis{t.basis} : nullptr;
  return KVF_OK;
}

kvf_status kvf_original_size_bytes(const kvf_compressed* c, size_t* out) {
  if (!c || !out) return fail(KVF_ERR_INVALID_CONFIG, "null pointer");
  *out = c->original_size_bytes;
  return KVF_OK;
}

kvf_status kvf_compression_ratio(kvf_compressed* c, double* out) {
  size_t comp = 0;
  KVF_TRY(kvf_compressed_size_bytes(c, &comp));
  if (!out) return fail(KVF_ERR_INVALID_CONFIG, "null pointer");
  *out = (double)c->original_size_bytes / (double)comp;  // types.rs:34-36
  return KVF_OK;
}

kvf_status kvf_compressed_tensor_info(kvf_compressed* c, int32_t which, size_t* R, size_t* plen, size_t* dlen,
                                      int32_t* has_entropy) {
  if (!c || (which != 0 && which != 1)) return fail(KVF_ERR_INVALID_CONFIG, "bad arguments");
  TensorC& t = which == 0 ? c->key : c->value;
  DeviceGuard g(c->device);
  KVF_TRY(resolve_len(t, c->stream));
  if (R) *R = t.basis ? t.basis->R : 0;
  if (plen) *plen = t.packed_len;
  if (dlen) *dlen = t.data_len;
  if (has_entropy) *has_entropy = t.entropy ? 1 : 0;
  return KVF_OK;
}

kvf_status kvf_compressed_tensor_views(const kvf_compressed* c, int32_t which, const uint8_t** data,
                                       const float** scales, const float** mins, const uint32_t** freq,
                                       const float** basis_vt, const uint64_t** ranks) {
  if (!c || (which != 0 && which != 1)) return fail(KVF_ERR_INVALID_CONFIG, "bad arguments");
  const TensorC& t = which == 0 ? c->key : c->value;
  if (data) *data = t.d_data;
  if (scales) *scales = t.d_scales;
  if (mins) *mins = t.d_mins;
  if (freq) *freq = t.d_freq;
  if (basis_vt) *basis_vt = t.basis ? t.basis->d_vt : nullptr;
  if (ranks) *ranks = t.basis ? t.basis->d_ranks : nullptr;
  return KVF_OK;
}

const float* kvf_compressed_calibration(const kvf_compressed* c) { return c ? c->d_scores : nullptr; }

namespace {
kvf_status ser_layer(kvf_compressed* c, Writer& w) {
  w.v<uint64_t>(c->layer_idx);
  w.v<uint64_t>(c->H);
  w.v<uint64_t>(c->T);
  w.v<uint64_t>(c->D);
  KVF_TRY(ser_tensor(c->key, w, c->stream));
  KVF_TRY(ser_tensor(c->value, w, c->stream));
  w.v<uint64_t>(c->original_size_bytes);
  return KVF_OK;
}
}  // namespace

kvf_status kvf_compressed_serialize(kvf_compressed* c, uint8_t* buf, size_t cap, size_t* len) {
  if (!c || !len) return fail(KVF_ERR_INVALID_CONFIG, "null pointer");
  DeviceGuard g(c->device);
  Writer w{buf, buf ? cap : 0};
  if (buf) {  // size first, so nothing is copied into a buffer that is too small
    Writer sz{nullptr, 0};
    KVF_TRY(ser_layer(c, sz));
    if (sz.len > cap) {
      *len = sz.len;
      return fail(KVF_ERR_SERIALIZATION, "buffer too small");
    }
  }
  KVF_TRY(ser_layer(c, w));
  *len = w.len;
  if (buf && w.len > cap) return fail(KVF_ERR_SERIALIZATION, "buffer too small");
  return KVF_OK;
}

kvf_status kvf_compressed_deserialize(kvf_ctx* ctx, const uint8_t* buf, size_t len, kvf_compressed** out,
                                      void* stream) {
  KVF_TRY(check_ctx(ctx));
  if (!buf || !out) return fail(KVF_ERR_INVALID_CONFIG, "null pointer");
  DeviceGuard g(ctx->device);
  Reader r{buf, len};
  std::unique_ptr<kvf_compressed> c(new kvf_compressed());
  c->ctx = ctx;
  c->device = ctx->device;
  c->stream = S(stream);
  c->layer_idx = r.v<uint64_t>();
  c->H = r.v<uint64_t>();
  c->T = r.v<uint64_t>();
  c->D = r.v<uint64_t>();
  if (!r.ok) return fail(KVF_ERR_SERIALIZATION, "truncated header");
  if (check_shape(c->H, c->T, c->D) != KVF_OK) return fail(KVF_ERR_SERIALIZATION, "bad shape");
  kvf_status s = KVF_OK;
  try {  // no exception leaves the C ABI: a host allocation that fails is a serialisation error
    s = deser_tensor(c.get(), c->key, r, c->stream);
    if (s == KVF_OK) s = deser_tensor(c.get(), c->value, r, c->stream);
  } catch (const std::exception& ex) {
    s = fail(KVF_ERR_SERIALIZATION, std::string("deserialisation failed: ") + ex.what());
  }
  if (s == KVF_OK) {
    c->original_size_bytes = r.v<uint64_t>();
    if (!r.ok) s = fail(KVF_ERR_SERIALIZATION, "truncated original_size_bytes");
  }
  if (s == KVF_OK && r.pos != r.len) s = fail(KVF_ERR_SERIALIZATION, "trailing bytes");
  if (s == KVF_OK) {
    cudaError_t e = cudaStreamSynchronize(c->stream);
    if (e != cudaSuccess) s = fail(KVF_ERR_CUDA, cudaGetErrorString(e));
  }
  if (s == KVF_OK) s = mark_ready(c.get());
  if (s != KVF_OK) {
    std::string msg = g_err;
    kvf_compressed_free(c.release());
    g_err = msg;
    return s;
  }
  *out = c.release();
  return KVF_OK;
}

kvf_status kvf_compressed_free(kvf_compressed* c) {
  if (!c) return KVF_OK;
  {
    DeviceGuard g(c->device);
    // the buffers go back to the pool on the building stream, after every
    // reader stream's last recorded use
    for (auto& u : c->uses) {
      cudaStreamWaitEvent(c->stream, u.second, 0);
      c->ctx->order_event_release(u.second);
    }
    // an event shared through the block goes back with the block
    if (c->ready && !(c->block && c->ready == c->block->ready)) c->ctx->order_event_release(c->ready);
    for (void* p : c->owned) cudaFreeAsync(p, c->stream);
  }
  delete c;
  return KVF_OK;
}

kvf_status kvf_compressed_free_many(kvf_compressed* const* cs, size_t n) {
  if (!cs && n) return fail(KVF_ERR_INVALID_CONFIG, "null pointer");
  for (size_t i = 0; i < n; ++i) kvf_compressed_free(cs[i]);
  return KVF_OK;
}

// ---- cost model with measured GPU costs --------------------------------------
// CostModel (crates/kvforge-core/src/cost.rs) with rows measured on this GPU;
// the reference's CpuCostModel holds a fixed table (crates/kvforge-cpu/src/cost.rs:26-50)
// and uses the same arithmetic (cost.rs:64-115), restated here.
double kvf_bandwidth_bytes_per_us(int32_t tier) {
  // BandwidthTier::bytes_per_us (crates/kvforge-core/src/cost.rs)
  static const double kBw[] = {25000.0, 12500.0, 10000.0, 2500.0, 1000.0, 100.0};
  return (tier >= 0 && tier < 6) ? kBw[tier] : -1.0;
}

kvf_status kvf_cost_estimate(const kvf_preset_cost* rows, size_t n, size_t original_bytes, int32_t preset,
                             double bytes_per_us, kvf_estimate* out) {
  if (!rows || n == 0 || !out) return fail(KVF_ERR_INVALID_CONFIG, "empty cost table");
  if (!(bytes_per_us > 0.0)) return fail(KVF_ERR_INVALID_CONFIG, "bandwidth must be positive");
  const kvf_preset_cost* e = &rows[0];  // an unknown preset takes the first row, as the reference does
  for (size_t i = 0; i < n; ++i)
    if (rows[i].preset == preset) { e = &rows[i]; break; }
  if (!(e->compression_ratio > 0.0)) return fail(KVF_ERR_INVALID_CONFIG, "compression ratio must be positive");
  const double bytes = (double)original_bytes;
  out->preset = e->preset;
  out->compress_us = bytes * e->compress_us_per_byte;
  out->transfer_us = bytes / e->compression_ratio / bytes_per_us;
  out->decompress_us = bytes * e->decompress_us_per_byte;
  out->total_us = out->compress_us + out->transfer_us + out->decompress_us;
  out->compression_ratio = e->compression_ratio;
  return KVF_OK;
}

kvf_status kvf_cost_select(const kvf_preset_cost* rows, size_t n, size_t original_bytes, double bytes_per_us,
                           double min_quality, kvf_estimate* out, size_t* count) {
  if (!rows || !out || !count) return fail(KVF_ERR_INVALID_CONFIG, "null pointer");
  std::vector<kvf_estimate> est;
  for (size_t i = 0; i < n; ++i) {
    if (!(rows[i].quality >= min_quality)) continue;
    kvf_estimate e;
    KVF_TRY(kvf_cost_estimate(&rows[i], 1, original_bytes, rows[i].preset, bytes_per_us, &e));
    est.push_back(e);
  }
  std::stable_sort(est.begin(), est.end(),
                   [](const kvf_estimate& a, const kvf_estimate& b) { return a.total_us < b.total_us; });
  std::copy(est.begin(), est.end(), out);
  *count = est.size();
  return KVF_OK;
}

kvf_status kvf_cost_measure(kvf_ctx* ctx, const void* keys, const void* values, int32_t in_dtype, size_t H,
                            size_t T, size_t D, int reps, kvf_preset_cost* rows, void* stream) {
  KVF_TRY(check_ctx(ctx));
  KVF_TRY(check_dtype(in_dtype));
  KVF_TRY(check_shape(H, T, D));
  if (!keys || !values || !rows || H * T * D == 0) return fail(KVF_ERR_INVALID_CONFIG, "empty sample");
  if (reps < 1 || reps > 1000) return fail(KVF_ERR_INVALID_CONFIG, "reps must be in 1..1000");
  DeviceGuard g(ctx->device);
  cudaStream_t st = S(stream);
  const size_t n = H * T * D, esz = in_dtype == KVF_IN_F16 ? 2 : 4;
  const double orig = (double)(2 * n * 4);  // KVCache::size_bytes (types.rs:30-32)
  // the sample on the host as f32, for the quality score
  std::vector<float> ref[2];
  const void* src[2] = {keys, values};
  for (int i = 0; i < 2; ++i) {
    std::vector<uint8_t> raw(n * esz);
    KVF_CUDA(cudaMemcpyAsync(raw.data(), src[i], n * esz, cudaMemcpyDeviceToHost, st));
    KVF_CUDA(cudaStreamSynchronize(st));
    ref[i].resize(n);
    if (esz == 2) {
      const __half* hp = reinterpret_cast<const __half*>(raw.data());
      for (size_t j = 0; j < n; ++j) ref[i][j] = __half2float(hp[j]);
    } else {
      std::memcpy(ref[i].data(), raw.data(), n * 4);
    }
  }
  float* dout[2] = {nullptr, nullptr};
  cudaEvent_t ev[4] = {};
  kvf_status s = KVF_OK;
  auto cuda = [&](cudaError_t e) {
    if (e != cudaSuccess && s == KVF_OK) s = fail(KVF_ERR_CUDA, cudaGetErrorString(e));
    return s == KVF_OK;
  };
  for (int i = 0; i < 2; ++i) cuda(cudaMalloc(&dout[i], n * 4));
  for (int i = 0; i < 4; ++i) cuda(cudaEventCreate(&ev[i]));
  const int32_t presets[3] = {KVF_CONSERVATIVE, KVF_BALANCED, KVF_AGGRESSIVE};
  for (int pi = 0; pi < 3 && s == KVF_OK; ++pi) {
    kvf_pipeline_config cfg;
    kvf_pipeline_config_from_preset(presets[pi], &cfg);
    kvf_basis *kb = nullptr, *vb = nullptr;  // calibrated once, outside the timing
    if (cfg.enable_projection) {
      s = kvf_basis_compute(ctx, keys, in_dtype, H, T, D, cfg.projection_variance_threshold, 0, &kb, stream);
      if (s == KVF_OK)
        s = kvf_basis_compute(ctx, values, in_dtype, H, T, D, cfg.projection_variance_threshold, 0, &vb, stream);
    }
    kvf_compressed* c = nullptr;
    double ratio = 0.0;
    if (s == KVF_OK) s = kvf_compress_layer(ctx, keys, values, in_dtype, H, T, D, 0, &cfg, kb, vb, &c, stream);
    if (s == KVF_OK) s = kvf_compression_ratio(c, &ratio);
    if (s == KVF_OK) s = kvf_decompress_layer(ctx, c, dout[0], dout[1], stream);
    if (s == KVF_OK) s = kvf_sync(ctx, stream);
    double err = 0.0;
    for (int i = 0; i < 2 && s == KVF_OK; ++i) {  // relative Frobenius error of each tensor
      std::vector<float> got(n);
      if (!cuda(cudaMemcpyAsync(got.data(), dout[i], n * 4, cudaMemcpyDeviceToHost, st)) ||
          !cuda(cudaStreamSynchronize(st)))
        break;
      double e2 = 0.0, r2 = 0.0;
      for (size_t j = 0; j < n; ++j) {
        const double d = (double)got[j] - (double)ref[i][j];
        e2 += d * d;
        r2 += (double)ref[i][j] * ref[i][j];
      }
      err = std::max(err, r2 > 0.0 ? std::sqrt(e2 / r2) : std::sqrt(e2));
    }
    float ms_c = 0.f, ms_d = 0.f;
    if (s == KVF_OK && cuda(cudaEventRecord(ev[0], st))) {
      for (int r = 0; r < reps && s == KVF_OK; ++r) {
        kvf_compressed* t = nullptr;
        s = kvf_compress_layer(ctx, keys, values, in_dtype, H, T, D, 0, &cfg, kb, vb, &t, stream);
        kvf_compressed_free(t);
      }
      if (cuda(cudaEventRecord(ev[1], st)) && cuda(cudaEventRecord(ev[2], st))) {
        for (int r = 0; r < reps && s == KVF_OK; ++r) s = kvf_decompress_layer(ctx, c, dout[0], dout[1], stream);
        if (cuda(cudaEventRecord(ev[3], st)) && cuda(cudaEventSynchronize(ev[3])))
          if (cuda(cudaEventElapsedTime(&ms_c, ev[0], ev[1]))) cuda(cudaEventElapsedTime(&ms_d, ev[2], ev[3]));
      }
    }
    if (s == KVF_OK) s = kvf_sync(ctx, stream);
    if (s == KVF_OK) {
      rows[pi].preset = presets[pi];
      rows[pi].compression_ratio = ratio;
      rows[pi].compress_us_per_byte = 1e3 * ms_c / reps / orig;
      rows[pi].decompress_us_per_byte = 1e3 * ms_d / reps / orig;
      rows[pi].quality = std::min(1.0, std::max(0.0, 1.0 - err));
    }
    kvf_compressed_free(c);
    kvf_basis_free(kb);
    kvf_basis_free(vb);
  }
  cudaStreamSynchronize(st);
  for (int i = 0; i < 4; ++i)
    if (ev[i]) cudaEventDestroy(ev[i]);
  for (int i = 0; i < 2; ++i)
    if (dout[i]) cudaFree(dout[i]);
  return s;
}

}  // extern "C"
