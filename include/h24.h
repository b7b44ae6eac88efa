/*
 * h24.h -- C ABI of the B200 (sm_100a) H24 codec library (libh24.so).
 *
 * Drop-in device implementation of the hot path of alavicka/pollux:
 * nearest-codeword quantisation onto the 196,561-entry H24 codebook, 18-bit
 * index pack / unpack, and LUT dequantisation to fp16.  Every entry point
 * takes plain device pointers and sizes plus a CUDA stream (cudaStream_t
 * passed as void*; NULL = legacy default stream), launches asynchronously on
 * that stream and returns a status code.  No entry point synchronises the
 * device, except where stated.  Buffers are owned by the caller; the library
 * owns only its per-device codebook tables and stream-ordered scratch.
 *
 * Indices are codebook rows: 0 is the origin, 1..196560 the kissing points.
 */
#ifndef H24_H_
#define H24_H_

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- status codes ------------------------------------------------------ */
#define H24_OK 0
#define H24_ERR_INVALID 1  /* bad argument: size, alignment, null pointer, rule */
#define H24_ERR_CUDA 2     /* a CUDA runtime call failed (message in h24_last_error) */
#define H24_ERR_RANGE 3    /* an input index exceeds 196560 */
#define H24_ERR_TIMEOUT 4  /* a bounded wait inside a kernel ran out */
#define H24_ERR_STATE 5    /* codebook tables could not be built */

/* ---- nearest-codeword rules -------------------------------------------- */
/* Training rule: index 0 iff 2 * max_j(x . kp_j) < 3.999999761581421,
 * else argmax + 1 (castor.py:448-462, 522, 551-557). */
#define H24_RULE_TRAIN 0
/* Pack rule: index 0 iff ||x||_2 < 1e-8, else argmax + 1 (pack.py:169-177). */
#define H24_RULE_PACK 1

/* ---- element types for h24_gather_codewords ---------------------------- */
#define H24_DTYPE_F32 0
#define H24_DTYPE_F16 1
#define H24_DTYPE_BF16 2

/* Message of the last failing call on this thread ("" if none). */
const char *h24_last_error(void);

/* Library version string. */
const char *h24_version(void);

/* Build the codebook tables on the host and upload them to `device`
 * (idempotent; thread-safe).  Replaces the lru-cached table construction of
 * castor._build_codebook_cpu / get_h24_codebook (castor.py:146-199).  Every
 * other call initialises the current device on first use. */
int h24_init(int device);

/* Raw integer coordinates of the 196,560 kissing points, [196560][24] int8 in
 * the reference's row order (codebook row j+1 = raw row j * 1/sqrt(8)),
 * written to HOST memory.  Needs no GPU (castor.py:98-190). */
int h24_codebook_raw(int8_t *out_host);

/* Copy the codebook to device memory as fp32 [196561][24]
 * (get_h24_codebook(device, torch.float32), castor.py:193-199). */
int h24_codebook_f32(float *out, void *stream);

/* codebook_fingerprint(): cb[:4,:4] as 16 floats on the host (castor.py:263-266). */
int h24_fingerprint(float out16[16]);

/* ---- 18-bit pack (castor.pack_indices, castor.py:226-246) ---------------
 * idx: n indices; each is truncated to 32 bits (as .to(torch.int32) does) and
 * then to 18 bits by the byte formulas.  out: ((n+3)/4)*9 bytes; missing tail
 * indices are packed as 0. */
int h24_pack(const int32_t *idx, int64_t n, uint8_t *out, void *stream);
int h24_pack_i64(const int64_t *idx, int64_t n, uint8_t *out, void *stream);

/* ---- 18-bit unpack (castor.unpack_indices, castor.py:249-260) -----------
 * packed: groups*9 bytes.  Writes min(n, 4*groups) indices. */
int h24_unpack(const uint8_t *packed, int64_t groups, int64_t n, int32_t *out, void *stream);
int h24_unpack_i64(const uint8_t *packed, int64_t groups, int64_t n, int64_t *out, void *stream);

/* ---- LUT dequant (PackedH24Linear.materialize, pollux.py:485-500) -------
 * packed: ((rows*in/24+3)/4)*9 bytes, sigma16: rows fp16 bit patterns,
 * out16: rows*in fp16 bit patterns,
 *   out = fp16( fp32( fp16(cb16[idx] * sigma16[row]) ) * 0.70710677f ).
 * in_features must be a positive multiple of 24.  Indices above 196560 are
 * written as the origin and counted into *bad_count (a device int32; may be
 * NULL), which the caller reads to raise the reference's IndexError. */
int h24_dequant(const uint8_t *packed, const uint16_t *sigma16, int64_t rows,
                int64_t in_features, uint16_t *out16, int32_t *bad_count, void *stream);

/* One layer of h24_dequant_batched. */
typedef struct h24_dequant_layer {
  const uint8_t *packed;
  const uint16_t *sigma16;
  uint16_t *out16;
  int64_t rows;
  int64_t in_features;
} h24_dequant_layer;

/* Dequantise `count` layers with one launch per 64 layers (the materialize()
 * loop of PolluxModel.from_packed_checkpoint, pollux.py:748-750).  `layers` is
 * a host array, read before the call returns. */
int h24_dequant_batched(const h24_dequant_layer *layers, int count, int32_t *bad_count,
                        void *stream);

/* ---- per-row RMS scales (castor.row_rms_from_matrix, castor.py:309-313;
 *      the sigma_rows of pack._quantize_h24_layer, pack.py:164) -------------
 * w: rows x in_features, fp32 or bf16 (dtype H24_DTYPE_F32 / H24_DTYPE_BF16;
 * bf16 is widened exactly, as weight.float() does), 16-byte aligned.
 * sigma_out[r] = sqrt(mean(w_r^2) + 1e-8) in fp32, and sigma16_out[r] =
 * fp16(clamp_min(sigma * sqrt(12), 1e-8)) as fp16 bits; either output may be
 * NULL.  The fp32 mean is summed in the order torch's CUDA reduction uses for
 * a contiguous [rows, in_features] tensor, so both are bit-identical to the
 * reference run on a CUDA device (pack.py's default). */
int h24_row_rms(const void *w, int64_t rows, int64_t in_features, int dtype, float *sigma_out,
                uint16_t *sigma16_out, void *stream);

/* ---- H24 projection of pollux_step (pollux.py:874-884), fused ------------
 * For every layer: sigma_r = sqrt(mean(latent_r^2) + 1e-8) (fp32, as
 * h24_row_rms computes it),
 * x = (latent / max(sigma, 1e-8)) / s_lattice, the nearest codeword of each
 * atom of x under the training rule (castor_quantize_leech), and
 * out = (codeword * sigma_r) * s_lattice in fp32 (the p.data.copy_ of the
 * reference).  One search pipeline for all layers, no host synchronisation.
 * sigma (rows fp32) and idx (rows*in/24 int32) are optional outputs. */
typedef struct h24_project_layer {
  const float *latent;
  float *out;
  int64_t rows;
  int64_t in_features;
  float *sigma;
  int32_t *idx;
} h24_project_layer;

int h24_project_layers(const h24_project_layer *layers, int count, void *stream);

/* Matrix-free LUT GEMV (the "future native kernel" of README.md:88, 155-156;
 * generate.py:8-18): y[b][o] = sum_i x[b][i] * W[o][i] for b < batch, where W is
 * the packed layer (rows = out_features) and W[o][i] the fp16 value
 * PackedH24Linear.materialize would produce; W is never materialised.  x: batch
 * x in_features fp32 (16-byte aligned rows), y: batch x rows fp32, fp32
 * products accurate to 2^-14 * sum_i |x[b][i] W[o][i]| (the order differs from
 * a dense matmul's; 3-8 input rows run on the tensor cores with exact bf16
 * products).  Out-of-range packed indices count into *bad_count (if non-null)
 * and read as the origin.  Layers split across several CTAs take a
 * stream-ordered workspace (8 * rows * 4 bytes per slice, at most 8 slices)
 * from the library's device memory pool, freed on the same stream. */
int h24_lut_gemv(const uint8_t *packed, const uint16_t *sigma16, int64_t rows,
                 int64_t in_features, const float *x, int64_t batch, float *y,
                 int32_t *bad_count, void *stream);

/* ---- INT8 token embedding / output head ------------------------------------
 * Per-row INT8 quantisation (pack._quantize_int8, pack.py:124-136):
 * mu = max(max_c |w[r][c]|, 1e-8) in fp32, q = clamp(rint(w / mu * 127),
 * -128, 127), mu16 = fp16(mu).  w: rows x cols fp32 row-major; q: rows x cols
 * int8; mu16: rows fp16 bits.  A NaN in a row makes its mu NaN and every q 0
 * (torch's amax and int8 cast). */
int h24_int8_quantize(const float *w, int64_t rows, int64_t cols, int8_t *q, uint16_t *mu16,
                      void *stream);

/* INT8 reconstruction (PackedInt8Embedding.materialize / PackedInt8Linear.
 * materialize, pollux.py:519-528, 545-554): out16 = fp16(q * fp16(mu16 / 127)),
 * both roundings of the reference kept. */
int h24_int8_dequant(const int8_t *q, const uint16_t *mu16, int64_t rows, int64_t cols,
                     uint16_t *out16, void *stream);

/* ---- nearest codeword (castor._leech_nn_kernel / castor_quantize_leech,
 *      castor.py:386-560; pack._quantize_h24_layer search, pack.py:166-177) --
 * x: n atoms of 24 fp32 values (16-byte aligned), out_idx: n int32 indices.
 * Exact fp64 argmax of x . kp_j (lowest index on ties) under `rule`.  A
 * tcgen05 bf16 screening pass keeps every codeword that can still be the
 * maximum; an fp64 rescore picks the winner. */
int h24_quantize(const float *x, int64_t n, int rule, int32_t *out_idx, void *stream);

/* h24_quantize for atoms of element type `dtype` (H24_DTYPE_F32 or
 * H24_DTYPE_BF16; bf16 coordinates are widened exactly to fp32, as the
 * reference's .float() does before its search, castor.py:516, pack.py:159).
 * x: n atoms of 24 elements, 16-byte aligned. */
int h24_quantize_typed(const void *x, int64_t n, int dtype, int rule, int32_t *out_idx, void *stream);

/* ---- allocation-free nearest codeword (no counterpart in the reference) --
 * Same result as h24_quantize for callers that must not allocate device
 * memory at call time (code under an external memory manager that owns every
 * device allocation, or latency-critical loops).  All per-call scratch lives
 * in one fixed device array of about 10.6 MiB inside the library, so the call
 * makes no cudaMalloc, cudaMallocAsync or cudaFree.  Limits: at most 32768
 * atoms per call (more is H24_ERR_INVALID); the codebook tables must already
 * be resident (call h24_init(device) once at set-up, else H24_ERR_STATE); the
 * first call on a device resolves the array's address (make it before any
 * stream capture); the array is shared by every call on the device and keeps
 * the last call's contents, so calls that overlap on the GPU race. */
int h24_quantize_noalloc(const float *x, int64_t n, int rule, int32_t *out_idx, void *stream);

/* ---- nearest codeword over several inputs in one pipeline ---------------
 * Segment i holds counts[i] atoms of 24 fp32 values at xs[i] (device
 * pointers, 16-byte aligned; `xs` and `counts` are host arrays read before the
 * call returns).  out_idx receives the indices of all segments back to back.
 * One screening launch covers up to 1M atoms of up to 64 segments, so many
 * small matrices fill the GPU like one large one (the per-parameter loop of
 * pollux_step, pollux.py:828-884). */
int h24_quantize_segments(const float *const *xs, const int64_t *counts, int nseg, int rule,
                          int32_t *out_idx, void *stream);

/* ---- fused pack-rule layer quantiser (pack._quantize_h24_layer, pack.py:139-180)
 * w: rows x in_features fp32 row-major (16-byte aligned), rows*in_features a
 * multiple of 24; atoms are consecutive runs of 24 values of the flattened
 * matrix (pack.py:161).  Writes sigma16_out[rows] =
 * fp16(clamp_min(sqrt(mean(w^2)+1e-8) * sqrt(12), 1e-8)) (as h24_row_rms)
 * and the packed indices packed_out[((rows*in/24+3)/4)*9] of the pack rule. */
int h24_quantize_layer(const float *w, int64_t rows, int64_t in_features,
                       uint16_t *sigma16_out, uint8_t *packed_out, void *stream);

/* h24_quantize_layer with the weight and both outputs in host memory (the
 * call shape of pack._quantize_h24_layer on a CPU weight, pack.py:139-180,
 * which returns host tensors).  The rows are processed in chunks: the
 * host-to-device copy of one chunk overlaps the search of the previous one
 * (page-locked host memory gives the overlap; pageable memory works too).
 * Returns once sigma16_out and packed_out are written; H24_ERR_TIMEOUT if a
 * bounded wait of the screening kernel ran out (the outputs are then
 * incomplete). */
int h24_quantize_layer_host(const float *w, int64_t rows, int64_t in_features,
                            uint16_t *sigma16_out, uint8_t *packed_out, void *stream);

/* One layer of h24_quantize_layers. */
typedef struct h24_layer {
  const float *w;
  int64_t rows;
  int64_t in_features;
  uint16_t *sigma16_out;
  uint8_t *packed_out;
} h24_layer;

/* h24_quantize_layer for `count` layers with one shared search pipeline (the
 * H24 branch of pack_checkpoint's loop, pack.py:268-283).  `layers` is a host
 * array read before the call returns. */
int h24_quantize_layers(const h24_layer *layers, int count, void *stream);

/* ---- row ranges, fp32 or bf16 weights ----------------------------------
 * Rows [row_begin, row_end) of one rows x in_features weight matrix: the
 * unit of row sharding across GPUs (each rank quantises its own rows of
 * every matrix; the ranks' outputs concatenate into the single-GPU bytes).
 * `w` points at the WHOLE matrix (elements of the call's dtype); sigma16_out
 * receives row_end - row_begin fp16 scales and packed_out the
 * ((row_end - row_begin) * in_features / 24 + 3) / 4 * 9 packed bytes of
 * those rows.  The range must start on a 4-atom group (row_begin *
 * in_features a multiple of 96) and end on one or at the matrix end.  The
 * row scales are those of the whole matrix, bit for bit (h24_row_rms). */
typedef struct h24_layer_rows {
  const void *w;
  int64_t rows;
  int64_t in_features;
  int64_t row_begin;
  int64_t row_end;
  uint16_t *sigma16_out;
  uint8_t *packed_out;
} h24_layer_rows;

/* Pack-rule quantisation of `count` device-resident row ranges with one shared
 * search pipeline (the H24 branch of pack_checkpoint's loop, pack.py:268-283,
 * on this rank's rows).  dtype: H24_DTYPE_F32 or H24_DTYPE_BF16 (a bf16
 * checkpoint is read as it is and widened exactly, pack.py:159).  `layers` is
 * a host array read before the call returns. */
int h24_quantize_layer_rows(const h24_layer_rows *layers, int count, int dtype, void *stream);

/* Row ranges of weights in HOST memory, outputs in host memory
 * (pack._quantize_h24_layer on CPU weights, pack.py:139-180, which returns
 * host tensors; count > 1 runs the H24 branch of pack_checkpoint's whole loop,
 * pack.py:268-283, as one pipeline).  The rows are copied in chunks whose
 * transfer overlaps the search of the previous chunk, across matrix
 * boundaries (page-locked host weights give the overlap; pageable ones work
 * too), and every sigma16_out / packed_out is written before the call
 * returns.  Returns H24_ERR_TIMEOUT if a bounded wait of the screening kernel
 * ran out (the outputs are then incomplete). */
int h24_quantize_layer_rows_host(const h24_layer_rows *layers, int count, int dtype, void *stream);

/* ---- codeword gather (index_select of castor.py:533, 559) ---------------
 * out[a][0..23] = codebook[idx[a]] converted to `dtype` (H24_DTYPE_*). */
int h24_gather_codewords(const int32_t *idx, int64_t n, int dtype, void *out, void *stream);

/* ---- instrumentation ----------------------------------------------------
 * When enabled, every quantize call records CUDA events on the caller's
 * stream around its prep, tensor-core screening and rescore kernels.
 * h24_timing_read synchronises on the recorded events and returns the summed
 * milliseconds and the number of launches since the last read. */
int h24_timing_enable(int enable);
int h24_timing_read(double *ms, int64_t *launches);

/* Per-kernel form of h24_timing_read: the events recorded around each launch
 * of `kernel` (H24_KERNEL_*) since its last read. */
#define H24_KERNEL_SCREEN 0   /* tcgen05 screening GEMM */
#define H24_KERNEL_RESCORE 1  /* candidate rescore */
#define H24_KERNEL_PREP 2     /* per-atom preparation */
#define H24_KERNEL_COUNT 3
int h24_timing_read_kernel(int kernel, double *ms, int64_t *launches);

/* Counters accumulated by the quantize calls on the current device since the
 * previous read (reading resets them; synchronises `stream`): atoms resolved
 * by the exhaustive fp64 scan, codewords scored exactly in fp64 by the
 * rescore, and the 32-column units behind the screen's flags (a flag of the
 * rows that also stand for the complements counts two). */
int h24_quantize_stats(int64_t *exhaustive_atoms, int64_t *exact_scores, int64_t *flagged_units,
                       void *stream);

/* Number of CUDA kernels this library has launched in this process. */
int64_t h24_launch_count(void);

/* Synchronise `stream` and report a device-side failure of earlier quantize
 * calls on the current device: H24_ERR_TIMEOUT if a bounded wait inside the
 * screening kernel ran out (the word is then cleared), else H24_OK. */
int h24_check(void *stream);


#ifdef __cplusplus
}
#endif

#endif /* H24_H_ */
