// h24_internal.cuh -- shared definitions of the libh24 CUDA sources.
#pragma once

#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <stdint.h>

#include <string>

#include "../../include/h24.h"

namespace h24 {

constexpr int kDim = 24;
constexpr int kKissing = 196560;
constexpr int kCount = 196561;

// Screening tiles: the codebook is streamed in tiles of kTileN codewords;
// 196,560 = 1638 x 120, so no tile is padded.  Candidates are tracked per
// chunk of kChunk codewords (two chunks per tile).
constexpr int kTileN = 120;
constexpr int kNumTiles = kKissing / kTileN;                 // 1638
constexpr int kChunk = kTileN / 2;                           // 60
constexpr int kNumChunks = kKissing / kChunk;                // 3276
constexpr int kKPad = 32;                                    // K padded 24 -> 32 (bf16)
constexpr int kRowBytes = kKPad * 2;                         // 64 bytes per operand row
static_assert(kNumTiles * kTileN == kKissing, "tiles cover the codebook exactly");

// fp32 value of LEECH_SCALE = 1/sqrt(8) and of s_lattice = 1/sqrt(2) as torch
// rounds the Python floats (castor.py:49, 68).
constexpr float kLeechScaleF = 0.35355339059327373f;
constexpr float kSLatticeF = 0.7071067811865476f;
// float(kissing_points[0].pow(2).sum()) of castor.py:522.
constexpr double kCSqNorm = 3.999999761581421;

// Per-device tables (all device pointers).
struct Tables {
  int device = -1;
  // bf16 raw coordinates [kKissing][32], core-matrix tiled for the MMA B
  // operand: tile t (kTileN rows) at t*kTileN*64 B; inside it 8-row group g
  // at g*512, 16-byte K chunk c at c*128, row r at r*16.
  const __nv_bfloat16 *cb_tiled = nullptr;
  // raw int8 coordinates [kKissing][24] (kissing point j = codebook row j+1).
  const int8_t *cb_raw = nullptr;
  // Dequant codes [kCount][4] u32 words (16 bytes per codeword, row 0 is the
  // origin): element 8p+e in nibble e of word p, bits 0-1 = position in the
  // codeword's value list, bit 2 of nibbles 0-1 = the list (see h24_capi.cu).
  const uint32_t *cb_nib = nullptr;
  float fingerprint[16];
  // Device counters: [0] atoms sent to the exhaustive scan, [1] candidate
  // chunks rescored, [2] atoms rescored from a bitmap; and the error word set
  // by a timed-out wait.
  int64_t *stats = nullptr;
  int *err = nullptr;
  // Stream-ordered pool for per-call scratch (kept warm between calls).
  cudaMemPool_t pool = nullptr;
};

// Returns the tables of the current device, building them on first use.
// nullptr on failure (message set).
const Tables *tables_for_current_device();
// Tables of the current device only if already built (never allocates).
const Tables *tables_if_ready();

// Error helpers (thread-local message).
const char *last_error_cstr();
void set_error(const std::string &msg);
int fail(int code, const std::string &msg);
int cuda_fail(cudaError_t e, const char *what);

#define H24_CUDA_TRY(expr)                                   \
  do {                                                       \
    cudaError_t _e = (expr);                                 \
    if (_e != cudaSuccess) return ::h24::cuda_fail(_e, #expr); \
  } while (0)

inline bool aligned16(const void *p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// Host-side raw codebook generation (h24_codebook.cpp).  out: [kKissing][24].
bool build_raw_kissing_points(int8_t *out, std::string *err);

// Kernel launchers (stream-ordered; return H24_OK or an error code).
int launch_pack_i32(const int32_t *idx, int64_t n, uint8_t *out, cudaStream_t s);
int launch_pack_i64(const int64_t *idx, int64_t n, uint8_t *out, cudaStream_t s);
int launch_unpack_i32(const uint8_t *p, int64_t groups, int64_t n, int32_t *out, cudaStream_t s);
int launch_unpack_i64(const uint8_t *p, int64_t groups, int64_t n, int64_t *out, cudaStream_t s);
int launch_dequant(const Tables *t, const h24_dequant_layer *layers_dev,
                   const h24_dequant_layer *layers_host, int count, int32_t *bad,
                   cudaStream_t s);
int launch_codebook_f32(const Tables *t, float *out_kissing, cudaStream_t s);
int launch_gather(const Tables *t, const int32_t *idx, int64_t n, int dtype, void *out,
                  cudaStream_t s);
int quantize(const Tables *t, const float *x, int64_t n, int rule, int32_t *out_idx,
             cudaStream_t s);
int quantize_segments(const Tables *t, const float *const *xs, const int64_t *counts, int nseg,
                      int rule, int32_t *out_idx, cudaStream_t s);
int launch_sigma16(const float *w, int64_t rows, int64_t in_f, uint16_t *sigma16,
                   cudaStream_t s);

// Number of kernels this library has launched (all devices, all threads).
void count_launches(int64_t k);

// Instrumentation of the screening kernel.
bool timing_enabled();
void timing_record(cudaEvent_t start, cudaEvent_t stop);

}  // namespace h24
