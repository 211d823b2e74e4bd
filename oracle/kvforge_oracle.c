/*
 * kvforge_oracle.c -- CPU oracle for the KVForge codec path (test infrastructure).
 *
 * Restates, in plain C, the reference Rust CPU crate. Each function cites the
 * reference file:line it follows (paths relative to the reference project).
 * Compiled with -ffp-contract=off so every f32 multiply and add rounds on its
 * own, as Rust does; the one fused multiply-add (the projection dot product)
 * is an explicit fmaf() and defines the order the GPU kernel reproduces.
 *
 * Only tests/, __graft_entry__.smoke() and bench.py's CPU legs use this file.
 */
#include "kvforge_oracle.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

/* -------------------------------------------------------------------------
 * KIVI quantizer -- crates/kvforge-cpu/src/quantize.rs
 * ------------------------------------------------------------------------- */

/* quantize.rs:28-34 */
static float quant_levels(int dt) { return dt == ORC_INT4 ? 15.0f : (dt == ORC_INT8 ? 255.0f : 1.0f); }

/* quantize.rs:37-39 */
uint8_t orc_pack_int4(uint8_t a, uint8_t b) { return (uint8_t)((a & 0x0F) | ((b & 0x0F) << 4)); }

/* quantize.rs:42-44 */
void orc_unpack_int4(uint8_t byte, uint8_t* lo, uint8_t* hi) {
  *lo = byte & 0x0F;
  *hi = (byte >> 4) & 0x0F;
}

size_t orc_packed_len(size_t n, int data_type) { return data_type == ORC_INT4 ? (n + 1) / 2 : n; }

size_t orc_num_params(size_t H, size_t T, size_t D, int axis) {
  return axis == ORC_PER_CHANNEL ? H * D : H * T;
}

/* Rust f32::min / f32::max ignore a NaN operand (quantize.rs:85-86, 115-116).
 * The sign of a zero minimum is left unspecified by Rust; this codec canonicalises
 * -0.0 to +0.0 inside min/max so that the result does not depend on the order
 * of a parallel reduction. */
static inline float canon0(float v) { return v == 0.0f ? 0.0f : v; }
static inline float rmin(float m, float v) {
  if (isnan(v)) return m;
  if (isnan(m)) return v;
  v = canon0(v);
  return v < m ? v : m;
}
static inline float rmax(float m, float v) {
  if (isnan(v)) return m;
  if (isnan(m)) return v;
  v = canon0(v);
  return v > m ? v : m;
}

/* quantize.rs:88-89 (and 117-118) */
static inline float make_scale(float mn, float mx, float levels) {
  float range = mx - mn;
  return (range < 1e-10f) ? 1.0f : range / levels;
}

/* quantize.rs:95 (and 124): ((v - min) / scale).round().clamp(0, levels) as u8.
 * round() is half away from zero (C roundf); clamp keeps NaN and `as u8` maps
 * NaN to 0. */
static inline uint8_t quant_code(float v, float mn, float scale, float levels) {
  float y = (v - mn) / scale;
  float r = roundf(y);
  if (isnan(r)) return 0;
  if (r < 0.0f) r = 0.0f;
  if (r > levels) r = levels;
  return (uint8_t)r;
}

/* quantize.rs:47-163 */
int orc_quantize(const float* data, size_t H, size_t T, size_t D, int data_type, int axis,
                 uint8_t* packed, float* scales, float* mins) {
  if (data_type == ORC_F32) return ORC_ERR_QUANTIZATION; /* quantize.rs:52-56 */
  if (data_type != ORC_INT4 && data_type != ORC_INT8) return ORC_ERR_INVALID_CONFIG;
  const float levels = quant_levels(data_type);
  const size_t n = H * T * D;
  uint8_t* q = (data_type == ORC_INT8) ? packed : (uint8_t*)malloc(n ? n : 1);
  if (!q) return ORC_ERR_PIPELINE;

  if (axis == ORC_PER_CHANNEL) {
    /* quantize.rs:67-101: one (scale, min) per (head, channel), params h*D + c */
    for (size_t h = 0; h < H; ++h) {
      for (size_t c = 0; c < D; ++c) {
        float mn = INFINITY, mx = -INFINITY;
        for (size_t t = 0; t < T; ++t) {
          float v = data[(h * T + t) * D + c];
          mn = rmin(mn, v);
          mx = rmax(mx, v);
        }
        float scale = make_scale(mn, mx, levels);
        scales[h * D + c] = scale;
        mins[h * D + c] = mn;
        for (size_t t = 0; t < T; ++t) {
          size_t i = (h * T + t) * D + c;
          q[i] = quant_code(data[i], mn, scale, levels);
        }
      }
    }
  } else if (axis == ORC_PER_TOKEN) {
    /* quantize.rs:102-130: one (scale, min) per (head, token), params h*T + t */
    for (size_t h = 0; h < H; ++h) {
      for (size_t t = 0; t < T; ++t) {
        const float* row = data + (h * T + t) * D;
        float mn = INFINITY, mx = -INFINITY;
        for (size_t c = 0; c < D; ++c) {
          mn = rmin(mn, row[c]);
          mx = rmax(mx, row[c]);
        }
        float scale = make_scale(mn, mx, levels);
        scales[h * T + t] = scale;
        mins[h * T + t] = mn;
        for (size_t c = 0; c < D; ++c) q[(h * T + t) * D + c] = quant_code(row[c], mn, scale, levels);
      }
    }
  } else {
    if (q != packed) free(q);
    return ORC_ERR_INVALID_CONFIG;
  }

  if (data_type == ORC_INT4) {
    /* quantize.rs:136-150: pairs over the flat index, odd tail in the low nibble */
    size_t i = 0, o = 0;
    while (i + 1 < n) {
      packed[o++] = orc_pack_int4(q[i], q[i + 1]);
      i += 2;
    }
    if (i < n) packed[o++] = orc_pack_int4(q[i], 0);
    free(q);
  }
  return ORC_OK;
}

/* quantize.rs:165-231 */
int orc_dequantize(const uint8_t* packed, size_t packed_len, const float* scales,
                   const float* mins, int data_type, int axis, size_t H, size_t T, size_t D,
                   float* out) {
  const size_t total = H * T * D;
  if (data_type == ORC_F32) return ORC_ERR_QUANTIZATION; /* quantize.rs:184-188 */
  if (data_type == ORC_INT8) {
    if (packed_len != total) return ORC_ERR_QUANTIZATION; /* quantize.rs:191-197 */
  } else if (data_type == ORC_INT4) {
    if (packed_len * 2 < total) return ORC_ERR_QUANTIZATION; /* unpack then truncate, 174-182 */
  } else {
    return ORC_ERR_INVALID_CONFIG;
  }
  for (size_t h = 0; h < H; ++h) {
    for (size_t t = 0; t < T; ++t) {
      for (size_t c = 0; c < D; ++c) {
        size_t i = (h * T + t) * D + c;
        size_t p = (axis == ORC_PER_CHANNEL) ? h * D + c : h * T + t;
        uint8_t qv;
        if (data_type == ORC_INT8) {
          qv = packed[i];
        } else {
          uint8_t lo, hi;
          orc_unpack_int4(packed[i >> 1], &lo, &hi);
          qv = (i & 1) ? hi : lo;
        }
        /* quantize.rs:210 / 223: q * scale + min, two separate roundings */
        float prod = (float)qv * scales[p];
        out[i] = prod + mins[p];
      }
    }
  }
  return ORC_OK;
}

/* -------------------------------------------------------------------------
 * Calibration -- crates/kvforge-cpu/src/calibration.rs:25-73
 * ------------------------------------------------------------------------- */
static inline double dmax_rust(double a, double b) {
  if (isnan(a)) return b;
  if (isnan(b)) return a;
  return a > b ? a : b;
}

int orc_calibrate(const float* keys, size_t H, size_t T, size_t D, size_t min_tokens,
                  float* scores) {
  if (T < min_tokens) return ORC_ERR_INVALID_CONFIG; /* calibration.rs:28-33 */
  const double n = (double)(T * D);
  double* var = (double*)malloc((H ? H : 1) * sizeof(double));
  if (!var) return ORC_ERR_PIPELINE;
  for (size_t h = 0; h < H; ++h) {
    double sum = 0.0, sum_sq = 0.0;
    for (size_t t = 0; t < T; ++t) {
      for (size_t c = 0; c < D; ++c) {
        double v = (double)keys[(h * T + t) * D + c];
        sum += v;
        sum_sq += v * v;
      }
    }
    double mean = sum / n;
    double variance = (sum_sq / n) - (mean * mean);
    var[h] = dmax_rust(variance, 0.0);
  }
  double max_var = 0.0;
  for (size_t h = 0; h < H; ++h) max_var = dmax_rust(max_var, var[h]);
  for (size_t h = 0; h < H; ++h) scores[h] = (max_var < 1e-12) ? 0.5f : (float)(var[h] / max_var);
  free(var);
  return ORC_OK;
}

/* -------------------------------------------------------------------------
 * Projection -- crates/kvforge-cpu/src/projection.rs
 * ------------------------------------------------------------------------- */

/* projection.rs:31-59 */
size_t orc_select_rank(const float* sv, size_t n, double threshold, size_t max_rank) {
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
  if (max_rank > 0 && rank > max_rank) rank = max_rank;
  return rank < 1 ? 1 : rank;
}

/* Cyclic Jacobi eigen-decomposition of a symmetric n x n matrix (fp64).
 * A (row-major) is overwritten; V receives eigenvectors as columns. */
static void jacobi_eigh(double* A, size_t n, double* V) {
  for (size_t i = 0; i < n; ++i)
    for (size_t j = 0; j < n; ++j) V[i * n + j] = (i == j) ? 1.0 : 0.0;
  double total = 0.0;
  for (size_t i = 0; i < n * n; ++i) total += A[i] * A[i];
  if (total == 0.0) return;
  for (int sweep = 0; sweep < 60; ++sweep) {
    double off = 0.0;
    for (size_t p = 0; p < n; ++p)
      for (size_t q = p + 1; q < n; ++q) off += A[p * n + q] * A[p * n + q];
    if (off <= 1e-30 * total) break;
    for (size_t p = 0; p + 1 < n; ++p) {
      for (size_t q = p + 1; q < n; ++q) {
        double apq = A[p * n + q];
        if (fabs(apq) <= 1e-300) continue;
        double app = A[p * n + p], aqq = A[q * n + q];
        double theta = (aqq - app) / (2.0 * apq);
        double t = (theta >= 0 ? 1.0 : -1.0) / (fabs(theta) + sqrt(theta * theta + 1.0));
        double c = 1.0 / sqrt(t * t + 1.0), s = t * c;
        for (size_t k = 0; k < n; ++k) { /* A <- A J */
          double akp = A[k * n + p], akq = A[k * n + q];
          A[k * n + p] = c * akp - s * akq;
          A[k * n + q] = s * akp + c * akq;
        }
        for (size_t k = 0; k < n; ++k) { /* A <- J^T A */
          double apk = A[p * n + k], aqk = A[q * n + k];
          A[p * n + k] = c * apk - s * aqk;
          A[q * n + k] = s * apk + c * aqk;
        }
        for (size_t k = 0; k < n; ++k) { /* V <- V J */
          double vkp = V[k * n + p], vkq = V[k * n + q];
          V[k * n + p] = c * vkp - s * vkq;
          V[k * n + q] = s * vkp + c * vkq;
        }
      }
    }
  }
}

/* Basis for projection.rs:81-90: eigenvectors of X^T X are the right singular
 * vectors of X and sqrt(eigenvalue) its singular values. Rows of basis_full[h]
 * are sorted by descending eigenvalue; each row's largest-magnitude component
 * is made positive. */
int orc_compute_basis(const float* data, size_t H, size_t T, size_t D, float* basis_full,
                      float* sv, int threads) {
  if (T == 0 || D == 0) return ORC_ERR_PROJECTION; /* projection.rs:71-75 */
  int err = 0;
#ifdef _OPENMP
#pragma omp parallel for schedule(dynamic, 1) num_threads(threads > 0 ? threads : 1)
#endif
  for (long hh = 0; hh < (long)H; ++hh) {
    size_t h = (size_t)hh;
    double* G = (double*)calloc(D * D, sizeof(double));
    double* V = (double*)malloc(D * D * sizeof(double));
    size_t* idx = (size_t*)malloc(D * sizeof(size_t));
    if (!G || !V || !idx) { err = 1; free(G); free(V); free(idx); continue; }
    const float* X = data + h * T * D;
    for (size_t t = 0; t < T; ++t) {
      const float* row = X + t * D;
      for (size_t i = 0; i < D; ++i) {
        double xi = (double)row[i];
        double* g = G + i * D;
        for (size_t j = i; j < D; ++j) g[j] += xi * (double)row[j];
      }
    }
    for (size_t i = 0; i < D; ++i)
      for (size_t j = 0; j < i; ++j) G[i * D + j] = G[j * D + i];
    jacobi_eigh(G, D, V);
    for (size_t i = 0; i < D; ++i) idx[i] = i;
    for (size_t i = 1; i < D; ++i) { /* insertion sort, descending eigenvalue, stable */
      size_t k = idx[i];
      double lk = G[k * D + k];
      size_t j = i;
      while (j > 0 && G[idx[j - 1] * D + idx[j - 1]] < lk) { idx[j] = idx[j - 1]; --j; }
      idx[j] = k;
    }
    for (size_t r = 0; r < D; ++r) {
      size_t k = idx[r];
      double lam = G[k * D + k];
      sv[h * D + r] = (float)sqrt(lam > 0.0 ? lam : 0.0);
      size_t big = 0;
      for (size_t c = 1; c < D; ++c)
        if (fabs(V[c * D + k]) > fabs(V[big * D + k])) big = c;
      double sgn = V[big * D + k] < 0 ? -1.0 : 1.0;
      for (size_t c = 0; c < D; ++c) basis_full[(h * D + r) * D + c] = (float)(sgn * V[c * D + k]);
    }
    free(G); free(V); free(idx);
  }
  return err ? ORC_ERR_PIPELINE : ORC_OK;
}

/* projection.rs:77-92 (ranks, max rank) and 118-128 (zero-padded basis) */
size_t orc_select_basis(const float* basis_full, const float* sv, size_t H, size_t T, size_t D,
                        double threshold, size_t max_rank, uint64_t* ranks, float* basis_vt) {
  size_t k = T < D ? T : D; /* nalgebra returns min(T, D) singular values */
  size_t R = 0;
  for (size_t h = 0; h < H; ++h) {
    ranks[h] = orc_select_rank(sv + h * D, k, threshold, max_rank);
    if (ranks[h] > R) R = ranks[h];
  }
  if (H == 0) R = 1; /* ranks.iter().max().unwrap_or(&1) */
  if (basis_vt) {
    for (size_t h = 0; h < H; ++h)
      for (size_t r = 0; r < R; ++r)
        for (size_t c = 0; c < D; ++c)
          basis_vt[(h * R + r) * D + c] = (r < ranks[h]) ? basis_full[(h * D + r) * D + c] : 0.0f;
  }
  return R;
}

/* projection.rs:111-116 computes U_k * S_k; the same quantity is X * V_k^T,
 * computed here as one fmaf chain over c = 0..D-1 starting from +0.0.
 * Columns r >= rank_h stay +0.0 (projection.rs:96). */
int orc_project(const float* data, size_t H, size_t T, size_t D, const float* basis_vt,
                const uint64_t* ranks, size_t R, float* projected, int threads) {
  if (T == 0 || D == 0) return ORC_ERR_PROJECTION;
#ifdef _OPENMP
#pragma omp parallel for schedule(static) num_threads(threads > 0 ? threads : 1)
#endif
  for (long g = 0; g < (long)(H * T); ++g) {
    size_t h = (size_t)g / T;
    const float* x = data + (size_t)g * D;
    float* p = projected + (size_t)g * R;
    for (size_t r = 0; r < R; ++r) {
      float acc = 0.0f;
      if (r < ranks[h]) {
        const float* v = basis_vt + (h * R + r) * D;
        for (size_t c = 0; c < D; ++c) acc = fmaf(x[c], v[c], acc);
      }
      p[r] = acc;
    }
  }
  return ORC_OK;
}

/* projection.rs:142-172: sequential r < rank_h, separate multiply and add */
int orc_reconstruct(const float* projected, size_t H, size_t T, size_t R, size_t D,
                    const float* basis_vt, const uint64_t* ranks, float* out, int threads) {
#ifdef _OPENMP
#pragma omp parallel for schedule(static) num_threads(threads > 0 ? threads : 1)
#endif
  for (long g = 0; g < (long)(H * T); ++g) {
    size_t h = (size_t)g / T;
    const float* p = projected + (size_t)g * R;
    const float* vt = basis_vt + h * R * D;
    float* o = out + (size_t)g * D;
    size_t rank = ranks[h];
    for (size_t c = 0; c < D; ++c) {
      float sum = 0.0f;
      for (size_t r = 0; r < rank; ++r) {
        float prod = p[r] * vt[r * D + c];
        sum = sum + prod;
      }
      o[c] = sum;
    }
  }
  return ORC_OK;
}

/* -------------------------------------------------------------------------
 * Entropy coding. The histogram follows entropy.rs:24-31. The coder is this
 * project's chunked rANS container with 32 independent lane streams per chunk
 * (the reference's single-stream constriction coder, entropy.rs:55-73, cannot
 * be split across threads):
 *
 *   state x in [2^16, 2^32), 16-bit renormalisation words, 13-bit model.
 *   header  (32 B): u32 magic "KVR2", u32 prob_bits=13, u32 lanes=32,
 *                   u32 chunk_symbols, u64 original_len, u32 num_chunks,
 *                   u32 header_bytes (= 32 + 4*(num_chunks+1))
 *   u32 chunk_offset[num_chunks+1]   byte offset of each chunk payload;
 *                                    the last entry is the container length
 *   chunk payload: u32 final_state[32]; u16 lane_words[32];
 *                  u16 words[sum(lane_words)]: lane 0's stream, then lane 1's,
 *                  ..., each in the order the decoder reads it;
 *                  one zero u16 when the word total is odd
 *
 * Chunk c holds symbols [c*chunk, min((c+1)*chunk, n)); symbol i of a chunk
 * belongs to lane i % 32 and step i / 32. Each lane is an ordinary rANS coder
 * over its own symbols: the encoder walks its steps from last to first, emits
 * at most one word per step before encoding, and the decoder walks them first
 * to last, reading that lane's words front to back.
 * ------------------------------------------------------------------------- */
#define RANS_M (1u << ORC_RANS_PROB_BITS)
#define RANS_L (1u << 16)
#define RANS_PAYLOAD_HDR (4u * ORC_RANS_LANES + 2u * ORC_RANS_LANES)

void orc_histogram(const uint8_t* data, size_t n, uint32_t* freq) {
  memset(freq, 0, 256 * sizeof(uint32_t));
  for (size_t i = 0; i < n; ++i) freq[data[i]] += 1;
}

/* Integer-only model: symbols seen q = max(1, floor(count * 2^13 / N)); unseen
 * symbols get no slot. A deficit goes to the most frequent symbol (lowest index
 * on ties); an excess is taken from the largest entries, one symbol at a time. */
int orc_rans_normalize(const uint32_t* freq, uint32_t* q, uint32_t* cum) {
  uint64_t N = 0;
  for (int s = 0; s < 256; ++s) N += freq[s];
  if (N == 0) return ORC_ERR_ENTROPY;
  uint64_t S = 0;
  int argmax = 0;
  for (int s = 0; s < 256; ++s) {
    if (freq[s] == 0) {
      q[s] = 0;
    } else {
      uint64_t v = ((uint64_t)freq[s] * RANS_M) / N;
      q[s] = (uint32_t)(v < 1 ? 1 : v);
    }
    S += q[s];
    if (freq[s] > freq[argmax]) argmax = s;
  }
  if (S < RANS_M) {
    q[argmax] += (uint32_t)(RANS_M - S);
  } else {
    while (S > RANS_M) {
      int best = -1;
      for (int s = 0; s < 256; ++s)
        if (q[s] > 1 && (best < 0 || q[s] > q[best])) best = s;
      if (best < 0) return ORC_ERR_ENTROPY;
      uint64_t d = S - RANS_M;
      if (d > q[best] - 1) d = q[best] - 1;
      q[best] -= (uint32_t)d;
      S -= d;
    }
  }
  uint32_t c = 0;
  for (int s = 0; s < 256; ++s) {
    cum[s] = c;
    c += q[s];
  }
  return ORC_OK;
}

size_t orc_rans_max_encoded_len(size_t n, uint32_t chunk) {
  size_t nc = (n + chunk - 1) / chunk;
  return 32 + 4 * (nc + 1) + nc * (RANS_PAYLOAD_HDR + 2) + 2 * n;
}

static inline void put16(uint8_t* p, uint16_t v) { memcpy(p, &v, 2); }
static inline uint16_t get16(const uint8_t* p) { uint16_t v; memcpy(&v, p, 2); return v; }
static inline void put32(uint8_t* p, uint32_t v) { memcpy(p, &v, 4); }
static inline uint32_t get32(const uint8_t* p) { uint32_t v; memcpy(&v, p, 4); return v; }
static inline uint64_t get64(const uint8_t* p) { uint64_t v; memcpy(&v, p, 8); return v; }

int orc_rans_encode(const uint8_t* data, size_t n, uint32_t chunk, uint8_t* out, size_t out_cap,
                    size_t* out_len, uint32_t* freq) {
  if (chunk == 0 || chunk % ORC_RANS_LANES || chunk > ORC_RANS_MAX_CHUNK) return ORC_ERR_INVALID_CONFIG;
  orc_histogram(data, n, freq);
  if (n == 0) { *out_len = 0; return ORC_OK; }
  uint32_t q[256], cum[256];
  int st = orc_rans_normalize(freq, q, cum);
  if (st) return st;
  size_t nc = (n + chunk - 1) / chunk;
  size_t hdr = 32 + 4 * (nc + 1);
  if (out_cap < hdr) return ORC_ERR_ENTROPY;
  const size_t smax = chunk / ORC_RANS_LANES; /* steps, and so words, per lane at most */
  uint16_t* tmp = (uint16_t*)malloc(sizeof(uint16_t) * ORC_RANS_LANES * smax);
  if (!tmp) return ORC_ERR_PIPELINE;
  size_t pos = hdr;
  for (size_t c = 0; c < nc; ++c) {
    size_t start = c * chunk;
    size_t nsym = (n - start < chunk) ? n - start : chunk;
    size_t steps = (nsym + ORC_RANS_LANES - 1) / ORC_RANS_LANES;
    uint32_t x[ORC_RANS_LANES];
    size_t cnt[ORC_RANS_LANES], total = 0;
    for (unsigned l = 0; l < ORC_RANS_LANES; ++l) {
      uint16_t* region = tmp + (size_t)l * smax; /* filled from its end */
      uint32_t xl = RANS_L;
      size_t k = 0;
      for (size_t st_i = steps; st_i-- > 0;) {
        size_t i = st_i * ORC_RANS_LANES + l;
        if (i >= nsym) continue;
        uint8_t s = data[start + i];
        uint32_t f = q[s];
        uint64_t xmax = ((uint64_t)(RANS_L >> ORC_RANS_PROB_BITS) << 16) * f;
        if ((uint64_t)xl >= xmax) {
          region[smax - 1 - k] = (uint16_t)(xl & 0xFFFFu);
          ++k;
          xl >>= 16;
        }
        xl = ((xl / f) << ORC_RANS_PROB_BITS) + (xl % f) + cum[s];
      }
      x[l] = xl;
      cnt[l] = k;
      total += k;
    }
    size_t bytes = RANS_PAYLOAD_HDR + 2 * total + (total & 1) * 2;
    if (pos + bytes > out_cap) { free(tmp); return ORC_ERR_ENTROPY; }
    put32(out + 32 + 4 * c, (uint32_t)pos);
    uint8_t* w = out + pos + RANS_PAYLOAD_HDR;
    for (unsigned l = 0; l < ORC_RANS_LANES; ++l) {
      put32(out + pos + 4 * l, x[l]);
      put16(out + pos + 4 * ORC_RANS_LANES + 2 * l, (uint16_t)cnt[l]);
      memcpy(w, tmp + (size_t)l * smax + (smax - cnt[l]), 2 * cnt[l]);
      w += 2 * cnt[l];
    }
    if (total & 1) { w[0] = 0; w[1] = 0; }
    pos += bytes;
  }
  free(tmp);
  put32(out + 32 + 4 * nc, (uint32_t)pos);
  put32(out + 0, ORC_RANS_MAGIC);
  put32(out + 4, ORC_RANS_PROB_BITS);
  put32(out + 8, ORC_RANS_LANES);
  put32(out + 12, chunk);
  uint64_t on = n;
  memcpy(out + 16, &on, 8);
  put32(out + 24, (uint32_t)nc);
  put32(out + 28, (uint32_t)hdr);
  *out_len = pos;
  return ORC_OK;
}

int orc_rans_decode(const uint8_t* comp, size_t comp_len, const uint32_t* freq,
                    size_t original_len, uint8_t* out) {
  if (original_len == 0) return ORC_OK;
  if (comp_len % 4 != 0) return ORC_ERR_ENTROPY; /* entropy.rs:94-98 */
  if (comp_len < 32) return ORC_ERR_CORRUPT_STREAM;
  if (get32(comp) != ORC_RANS_MAGIC || get32(comp + 4) != ORC_RANS_PROB_BITS ||
      get32(comp + 8) != ORC_RANS_LANES)
    return ORC_ERR_CORRUPT_STREAM;
  uint32_t chunk = get32(comp + 12);
  uint64_t n = get64(comp + 16);
  uint32_t nc = get32(comp + 24);
  if (chunk == 0 || chunk % ORC_RANS_LANES || chunk > ORC_RANS_MAX_CHUNK || n != original_len)
    return ORC_ERR_CORRUPT_STREAM;
  if ((uint64_t)nc != (n + chunk - 1) / chunk) return ORC_ERR_CORRUPT_STREAM;
  size_t hdr = 32 + 4 * ((size_t)nc + 1);
  if (get32(comp + 28) != hdr || comp_len < hdr) return ORC_ERR_CORRUPT_STREAM;
  if (get32(comp + 32 + 4 * (size_t)nc) != comp_len) return ORC_ERR_CORRUPT_STREAM;
  uint32_t q[256], cum[256];
  if (orc_rans_normalize(freq, q, cum)) return ORC_ERR_ENTROPY;
  uint8_t slot2sym[RANS_M];
  for (int s = 0; s < 256; ++s)
    for (uint32_t k = 0; k < q[s]; ++k) slot2sym[cum[s] + k] = (uint8_t)s;
  for (size_t c = 0; c < nc; ++c) {
    size_t off = get32(comp + 32 + 4 * c), end = get32(comp + 32 + 4 * (c + 1));
    if (off < hdr || end > comp_len || end < off + RANS_PAYLOAD_HDR) return ORC_ERR_CORRUPT_STREAM;
    size_t start = c * (size_t)chunk;
    size_t nsym = (n - start < chunk) ? (size_t)(n - start) : chunk;
    size_t steps = (nsym + ORC_RANS_LANES - 1) / ORC_RANS_LANES;
    size_t base[ORC_RANS_LANES], cnt[ORC_RANS_LANES], total = 0;
    for (unsigned l = 0; l < ORC_RANS_LANES; ++l) {
      cnt[l] = get16(comp + off + 4 * ORC_RANS_LANES + 2 * l);
      base[l] = total;
      total += cnt[l];
    }
    if (off + RANS_PAYLOAD_HDR + 2 * total + (total & 1) * 2 != end) return ORC_ERR_CORRUPT_STREAM;
    const uint8_t* w = comp + off + RANS_PAYLOAD_HDR;
    for (unsigned l = 0; l < ORC_RANS_LANES; ++l) {
      uint32_t xl = get32(comp + off + 4 * l);
      if (xl < RANS_L) return ORC_ERR_CORRUPT_STREAM;
      size_t k = 0;
      for (size_t s_i = 0; s_i < steps; ++s_i) {
        size_t i = s_i * ORC_RANS_LANES + l;
        if (i >= nsym) continue;
        uint32_t slot = xl & (RANS_M - 1);
        uint8_t s = slot2sym[slot];
        xl = q[s] * (xl >> ORC_RANS_PROB_BITS) + slot - cum[s];
        out[start + i] = s;
        if (xl < RANS_L) {
          if (k >= cnt[l]) return ORC_ERR_CORRUPT_STREAM;
          xl = (xl << 16) | get16(w + 2 * (base[l] + k));
          ++k;
        }
      }
      if (xl != RANS_L || k != cnt[l]) return ORC_ERR_CORRUPT_STREAM;
    }
  }
  return ORC_OK;
}

/* Shannon bound of the empirical distribution, in bits (for reporting). */
double orc_entropy_bits(const uint32_t* freq) {
  double N = 0;
  for (int s = 0; s < 256; ++s) N += freq[s];
  double bits = 0;
  for (int s = 0; s < 256; ++s)
    if (freq[s]) bits -= (double)freq[s] * log2((double)freq[s] / N);
  return bits;
}

/* -------------------------------------------------------------------------
 * Per-tensor pipeline -- crates/kvforge-cpu/src/pipeline.rs:38-97
 * ------------------------------------------------------------------------- */
int orc_compress_tensor(const float* x, size_t H, size_t T, size_t D, const orc_tensor_cfg* cfg,
                        orc_tensor_out* out, int threads) {
  memset(out, 0, sizeof(*out));
  const float* qin = x;
  float* proj = NULL;
  size_t qcols = D;
  if (cfg->project) { /* pipeline.rs:48-53 */
    qcols = cfg->R;
    proj = (float*)malloc(((H * T * qcols) > 0 ? H * T * qcols : 1) * sizeof(float));
    if (!proj) return ORC_ERR_PIPELINE;
    int st = orc_project(x, H, T, D, cfg->basis_vt, cfg->ranks, cfg->R, proj, threads);
    if (st) { free(proj); return st; }
    qin = proj;
  }
  size_t n = H * T * qcols;
  size_t plen = orc_packed_len(n, cfg->data_type);
  size_t np = orc_num_params(H, T, qcols, cfg->axis);
  uint8_t* codes = (uint8_t*)malloc(plen ? plen : 1);
  out->scales = (float*)malloc((np ? np : 1) * sizeof(float));
  out->mins = (float*)malloc((np ? np : 1) * sizeof(float));
  out->num_params = np;
  out->qcols = qcols;
  int st = orc_quantize(qin, H, T, qcols, cfg->data_type, cfg->axis, codes, out->scales, out->mins);
  free(proj);
  if (st) { free(codes); orc_tensor_free(out); return st; }
  out->original_len = plen;
  if (cfg->entropy && plen > 0) { /* pipeline.rs:58-64, entropy.rs:42-86 */
    size_t cap = orc_rans_max_encoded_len(plen, ORC_RANS_DEFAULT_CHUNK);
    out->data = (uint8_t*)malloc(cap);
    st = orc_rans_encode(codes, plen, ORC_RANS_DEFAULT_CHUNK, out->data, cap, &out->data_len, out->freq);
    free(codes);
    if (st) { orc_tensor_free(out); return st; }
    out->has_entropy = 1;
  } else {
    out->data = codes;
    out->data_len = plen;
    out->has_entropy = 0;
  }
  return ORC_OK;
}

int orc_decompress_tensor(const orc_tensor_out* in, size_t H, size_t T, size_t D,
                          const orc_tensor_cfg* cfg, float* x_out, int threads) {
  size_t qcols = in->qcols;
  const uint8_t* codes = in->data;
  uint8_t* dec = NULL;
  if (in->has_entropy) { /* pipeline.rs:82-86 */
    dec = (uint8_t*)malloc(in->original_len ? in->original_len : 1);
    int st = orc_rans_decode(in->data, in->data_len, in->freq, in->original_len, dec);
    if (st) { free(dec); return st; }
    codes = dec;
  }
  size_t clen = in->has_entropy ? in->original_len : in->data_len;
  int st;
  if (cfg->project) { /* pipeline.rs:88-96 */
    float* deq = (float*)malloc(((H * T * qcols) > 0 ? H * T * qcols : 1) * sizeof(float));
    st = orc_dequantize(codes, clen, in->scales, in->mins, cfg->data_type, cfg->axis, H, T, qcols, deq);
    if (!st) st = orc_reconstruct(deq, H, T, qcols, D, cfg->basis_vt, cfg->ranks, x_out, threads);
    free(deq);
  } else {
    st = orc_dequantize(codes, clen, in->scales, in->mins, cfg->data_type, cfg->axis, H, T, D, x_out);
  }
  free(dec);
  return st;
}

/* types.rs:66-78, 91-95, 131-135, 144-148 */
size_t orc_tensor_size_bytes(const orc_tensor_out* t, const orc_tensor_cfg* cfg, size_t H,
                             size_t D) {
  size_t total = t->data_len + 2 * t->num_params * 4;
  if (cfg->project) total += H * cfg->R * D * 4 + H * 8;
  if (cfg->entropy) total += (t->original_len > 0 ? 256 * 4 : 0) + 8;
  return total;
}

void orc_tensor_free(orc_tensor_out* t) {
  free(t->data); free(t->scales); free(t->mins);
  t->data = NULL; t->scales = NULL; t->mins = NULL;
}
