/*
 * kvforge_oracle.h -- CPU oracle for the KVForge codec path.
 *
 * TEST INFRASTRUCTURE ONLY. This is a single-threaded (optionally OpenMP)
 * C restatement of the reference Rust CPU crate (crates/kvforge-cpu) plus the
 * CPU mirror of this project's chunked rANS container. It is used by tests/,
 * __graft_entry__.smoke() and bench.py's cpu_baseline / reference arm only, as
 * the checker. The product library (kvforge_b200/) never links or calls it.
 *
 * Parity status:
 *   quantize / dequantize / INT4 pack / calibrate / select_rank / reconstruct:
 *     restated line by line from the reference; pinned against the reference's
 *     own known-answer tests (quantize.rs:246-258, projection.rs:242-253,
 *     entropy.rs:192-199) and its MSE / ratio bounds.
 *   projection basis: the reference takes nalgebra's f32 SVD (projection.rs:84),
 *     which cannot be reproduced here; the basis is the top eigenvectors of the
 *     per-head Gram matrix (same subspace), pinned against an fp64 numpy SVD.
 *   rANS: the reference bitstream comes from constriction 0.4 (entropy.rs:55-73),
 *     absent from the reference tree; this oracle defines the chunked container
 *     and is the CPU side of GPU<->CPU cross-decoding. Parity with the
 *     reference's bitstream is unpinned.
 */
#ifndef KVFORGE_ORACLE_H
#define KVFORGE_ORACLE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* status codes: same numbering as include/kvforge.h */
enum {
  ORC_OK = 0,
  ORC_ERR_SHAPE_MISMATCH = 1,
  ORC_ERR_INVALID_CONFIG = 2,
  ORC_ERR_QUANTIZATION = 3,
  ORC_ERR_PROJECTION = 4,
  ORC_ERR_ENTROPY = 5,
  ORC_ERR_SERIALIZATION = 6,
  ORC_ERR_CUDA = 7,
  ORC_ERR_PIPELINE = 8,
  ORC_ERR_DEVICE_TIMEOUT = 9,
  ORC_ERR_CORRUPT_STREAM = 10
};

enum { ORC_INT4 = 0, ORC_INT8 = 1, ORC_F32 = 2 };            /* DataType, types.rs:106-113 */
enum { ORC_PER_CHANNEL = 0, ORC_PER_TOKEN = 1 };            /* QuantAxis, types.rs:97-103 */

/* rANS container constants (this project's format, mirrored on the GPU) */
#define ORC_RANS_PROB_BITS 13u
#define ORC_RANS_LANES 32u
#define ORC_RANS_DEFAULT_CHUNK 8192u
#define ORC_RANS_MAX_CHUNK (ORC_RANS_LANES * 65535u) /* lane word counts are u16 */
#define ORC_RANS_MAGIC 0x3252564Bu /* "KVR2" */

uint8_t orc_pack_int4(uint8_t a, uint8_t b);
void orc_unpack_int4(uint8_t byte, uint8_t* lo, uint8_t* hi);

size_t orc_packed_len(size_t n, int data_type);
size_t orc_num_params(size_t H, size_t T, size_t D, int axis);

int orc_quantize(const float* data, size_t H, size_t T, size_t D, int data_type, int axis,
                 uint8_t* packed, float* scales, float* mins);
int orc_dequantize(const uint8_t* packed, size_t packed_len, const float* scales,
                   const float* mins, int data_type, int axis, size_t H, size_t T, size_t D,
                   float* out);

int orc_calibrate(const float* keys, size_t H, size_t T, size_t D, size_t min_tokens,
                  float* scores);

size_t orc_select_rank(const float* singular_values, size_t n, double threshold,
                       size_t max_rank /* 0 = None */);

/* basis: gram (fp64) + cyclic Jacobi. basis_vt out [H, D, D] rows sorted by
 * descending eigenvalue; sv out [H, D] (f32 singular values, sqrt of eigenvalues). */
int orc_compute_basis(const float* data, size_t H, size_t T, size_t D, float* basis_full,
                      float* sv, int threads);
/* ranks from sv, then the padded [H, R, D] basis; returns R. */
size_t orc_select_basis(const float* basis_full, const float* sv, size_t H, size_t T, size_t D,
                        double threshold, size_t max_rank, uint64_t* ranks, float* basis_vt);

int orc_project(const float* data, size_t H, size_t T, size_t D, const float* basis_vt,
                const uint64_t* ranks, size_t R, float* projected, int threads);
int orc_reconstruct(const float* projected, size_t H, size_t T, size_t R, size_t D,
                    const float* basis_vt, const uint64_t* ranks, float* out, int threads);

void orc_histogram(const uint8_t* data, size_t n, uint32_t* freq);
int orc_rans_normalize(const uint32_t* freq, uint32_t* qfreq, uint32_t* qcum);
size_t orc_rans_max_encoded_len(size_t n, uint32_t chunk_symbols);
int orc_rans_encode(const uint8_t* data, size_t n, uint32_t chunk_symbols, uint8_t* out,
                    size_t out_cap, size_t* out_len, uint32_t* freq);
int orc_rans_decode(const uint8_t* comp, size_t comp_len, const uint32_t* freq,
                    size_t original_len, uint8_t* out);
double orc_entropy_bits(const uint32_t* freq);

/* ---- per-tensor pipeline (pipeline.rs:38-97) ---- */
typedef struct {
  int data_type;
  int axis;
  int project;         /* projection on/off */
  int entropy;         /* entropy coding on/off */
  size_t R;            /* projected width (1..D) when project */
  const float* basis_vt; /* [H,R,D] */
  const uint64_t* ranks; /* [H] */
} orc_tensor_cfg;

typedef struct {
  uint8_t* data;      size_t data_len;     /* final bytes (container or raw codes) */
  float* scales;      float* mins;         size_t num_params;
  uint32_t freq[256]; int has_entropy;     size_t original_len;
  size_t qcols;       /* D or R */
} orc_tensor_out;

int orc_compress_tensor(const float* x, size_t H, size_t T, size_t D, const orc_tensor_cfg* cfg,
                        orc_tensor_out* out, int threads);
int orc_decompress_tensor(const orc_tensor_out* in, size_t H, size_t T, size_t D,
                          const orc_tensor_cfg* cfg, float* x_out, int threads);
size_t orc_tensor_size_bytes(const orc_tensor_out* t, const orc_tensor_cfg* cfg, size_t H,
                             size_t D);
void orc_tensor_free(orc_tensor_out* t);

#ifdef __cplusplus
}
#endif
#endif
