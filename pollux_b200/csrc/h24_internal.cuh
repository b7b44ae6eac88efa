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

// Structure of the 196,560 kissing points (verified when the tables are
// built): every one is of exactly one type,
//   type 1  (+-4, +-4, 0^22): 276 position pairs x 4 sign pairs;
//   type 2  (+-2^8, 0^16): 759 octads x the 128 sign patterns with an even
//           number of minus signs;
//   type 3  (-3, +-1^23): one of the 4096 Golay codewords c and a position p;
//           coordinate i != p is (-1)^c_i and coordinate p is -3.
// The Golay code is closed under complement, and column c + 2048 holds the
// complement of column c: columns 0-2047 are the zero word (0), the 759
// octads (1-759, in the order of their complements when sorted by bit
// pattern) and one dodecad of each complementary pair (760-2047, the smaller
// bit pattern, ascending); columns 2048-4095 are the all-ones word, the
// weight-16 words (2049-2807, complement of octad o at 2049 + o) and the
// other dodecads.  Every screening row r gives r(~c) = -r(c), so the screen
// multiplies only the first 2048 columns.
constexpr int kGolay = 4096;
constexpr int kGolayHalf = kGolay / 2;        // columns c and c + 2048 are complements
constexpr int kOctads = 759;
constexpr int kW16First = kGolayHalf + 1;     // 2049: first weight-16 Golay column
constexpr int kGolayTileN = 128;              // Golay columns per MMA tile
constexpr int kGolayTiles = kGolay / kGolayTileN;  // 32
constexpr int kTriples = 2024;                // C(24, 3)
constexpr int kTripleRow = 22;                // 21 octads per triple (+1 pad: 176-byte rows)
constexpr int kKPad = 32;                     // K padded 24 -> 32 (bf16)
constexpr int kRowBytes = kKPad * 2;          // 64 bytes per operand row

// fp32 value of LEECH_SCALE = 1/sqrt(8) and of s_lattice = 1/sqrt(2) as torch
// rounds the Python floats (castor.py:49, 68).
constexpr float kLeechScaleF = 0.35355339059327373f;
constexpr float kSLatticeF = 0.7071067811865476f;
// float(kissing_points[0].pow(2).sum()) of castor.py:522.
constexpr double kCSqNorm = 3.999999761581421;

#ifdef __CUDACC__
// fp16 bits of the materialised weight of raw Leech coordinate `raw` (-4..4)
// in a row with fp16 scale `sigma_bits` (pollux.py:485-500):
//   fp16( fp32( fp16(cb16 * sigma16) ) * s_lattice ),  cb16 = fp16(raw * fp32(1/sqrt(8))).
__device__ __forceinline__ uint16_t dequant_value(int raw, uint16_t sigma_bits) {
  const __half cb = __float2half_rn(static_cast<float>(raw) * kLeechScaleF);
  const __half sg = __ushort_as_half(sigma_bits);
  const __half t = __float2half_rn(__half2float(cb) * __half2float(sg));
  const __half w = __float2half_rn(__half2float(t) * kSLatticeF);
  return __half_as_ushort(w);
}
#endif

// Per-device tables (all device pointers).
struct Tables {
  int device = -1;
  // bf16 Golay sign matrix, the B operand of the screening MMAs: column c
  // holds (-1)^c_k for k < 24 and zeros for k = 24..31, in tiles of 128
  // columns in the UMMA canonical K-major layout without swizzle (tile t at
  // t*8192 B; 8-column group g at g*512, 16-byte K chunk q at q*128, column r
  // of the group at r*16).
  const __nv_bfloat16 *golay_tiled = nullptr;
  const uint32_t *golay_mask = nullptr;  // [kGolay] bit i = c_i
  // Kissing-point index (codebook row - 1) of each structured codeword:
  // idx3[c*24 + p] type 3; idx2[o*128 + s] type 2, octad o = complement of
  // Golay column kW16First + o, s = minus signs of its first 7 positions
  // (bit k for the k-th lowest position); idx1[(a*24 + b)*4 + s] type 1,
  // positions a < b, s = (x_a < 0) | (x_b < 0) << 1.
  const int32_t *idx3 = nullptr;
  const int32_t *idx2 = nullptr;
  const int32_t *idx1 = nullptr;
  // The 21 octads through each position triple i < j < k, row C(k,3) +
  // C(j,2) + i of kTripleRow entries (the last unused): .x = the octad's
  // position mask, .y = its five positions outside the triple, 5 bits each
  // (lowest first).
  const uint2 *oct_by_triple = nullptr;
  // raw int8 coordinates [kKissing][24] (kissing point j = codebook row j+1).
  const int8_t *cb_raw = nullptr;
  // Dequant codes [kCount][4] u32 words (16 bytes per codeword, row 0 is the
  // origin): element 8p+e in nibble e of word p, bits 0-1 = position in the
  // codeword's value list, bit 2 of nibbles 0-1 = the list (see h24_capi.cu).
  const uint32_t *cb_nib = nullptr;
  float fingerprint[16];
  // Device counters: [0] atoms sent to the exhaustive scan, [1] exact fp64
  // codeword scores of the rescore, [2] candidate chunks flagged by the
  // screen (32-column units); and the error word set by a timed-out wait.
  int64_t *stats = nullptr;
  int *err = nullptr;
  // Stream-ordered pool for per-call scratch (kept warm between calls).
  cudaMemPool_t pool = nullptr;
  // Non-blocking streams for the host-to-device copies of host-pointer entry
  // points (so that the copy of one batch overlaps the search of the
  // previous) and for their device-to-host result copies (a separate copy
  // engine, so that results return while later batches are copied in).
  cudaStream_t copy_stream = nullptr;
  cudaStream_t d2h_stream = nullptr;
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

// Programmatic dependent launch.  A kernel launched by launch_pdl calls
// pdl_enter() before touching memory: it waits until the previous kernel of
// the stream has completed with its writes visible (griddepcontrol.wait),
// then lets the next kernel launch (griddepcontrol.launch_dependents), so
// that a launch and its ramp overlap the tail of the kernel before it.  In a
// kernel launched without the attribute both instructions do nothing.
__device__ __forceinline__ void pdl_enter() {
  asm volatile("griddepcontrol.wait;" ::: "memory");
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

template <typename K, typename... Args>
cudaError_t launch_pdl(K kernel, dim3 grid, dim3 block, cudaStream_t s, Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = 0;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kernel, args...);
}

// Blocks of `kernel` that one SM holds at once (at least 1).
template <typename K>
int blocks_per_sm(K kernel, int threads, size_t dyn_smem) {
  int per = 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per, kernel, threads, dyn_smem) != cudaSuccess ||
      per < 1)
    per = 1;
  return per;
}

// Grid of at most one resident wave (SMs x `per_sm` blocks), fewer when the
// work needs fewer blocks: a grid-stride kernel then finishes in one wave
// instead of leaving a partial second one.
inline int wave_grid(int64_t want_blocks, int per_sm) {
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const int64_t cap = static_cast<int64_t>(sms) * per_sm;
  return static_cast<int>(want_blocks < 1 ? 1 : (want_blocks < cap ? want_blocks : cap));
}

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
int launch_lut_gemv(const Tables *t, const uint8_t *packed, const uint16_t *sigma16, int64_t rows,
                    int64_t in_f, const float *x, int64_t batch, float *y, int32_t *bad,
                    cudaStream_t s);
int launch_gather(const Tables *t, const int32_t *idx, int64_t n, int dtype, void *out,
                  cudaStream_t s);
int quantize(const Tables *t, const float *x, int64_t n, int rule, int32_t *out_idx,
             cudaStream_t s);
// Atoms of segment i: counts[i] x 24 elements at xs[i], of type `dtype`
// (H24_DTYPE_F32 or H24_DTYPE_BF16), 16-byte aligned.
int quantize_segments(const Tables *t, const void *const *xs, const int64_t *counts, int nseg,
                      int dtype, int rule, int32_t *out_idx, cudaStream_t s);
int project_layers(const Tables *t, const h24_project_layer *layers, int count, cudaStream_t s);
int launch_int8_quantize(const float *w, int64_t rows, int64_t cols, int8_t *q, uint16_t *mu16,
                         cudaStream_t s);
int launch_int8_dequant(const int8_t *q, const uint16_t *mu16, int64_t rows, int64_t cols,
                        uint16_t *out, cudaStream_t s);
// Row scales of `rows` rows of n elements at w (fp32 or bf16), which are rows
// first_row.. of a 16-byte aligned matrix of matrix_rows rows, in the
// reference's arithmetic (h24_rowrms.cu): sigma32 = sqrt(mean(w^2) + 1e-8),
// sigma16 = fp16(clamp_min(sigma32 * sqrt(12), 1e-8)); either may be null.
int launch_row_rms(const void *w, int dtype, int64_t rows, int64_t n, int64_t matrix_rows,
                   int64_t first_row, float *sigma32, uint16_t *sigma16, cudaStream_t s);

// Number of kernels this library has launched (all devices, all threads).
void count_launches(int64_t k);

// Instrumentation of the screening kernel.
bool timing_enabled();
void timing_record(int kernel, cudaEvent_t start, cudaEvent_t stop);

}  // namespace h24
