/*
 * h24_oracle.c -- CPU restatement of Pollux's H24 hot path.
 *
 * TEST INFRASTRUCTURE ONLY.  This file is the parity checker for the CUDA
 * library in pollux_b200/; it is never part of the product path.  Only the
 * tests, the smoke check and the CPU-baseline leg of the benchmark may load it.
 *
 * What it restates (reference file:line, project alavicka/pollux):
 *   - Golay(24,12) words ........................ castor.py:74-95
 *   - 196,560 kissing points, three types ........ castor.py:98-143
 *   - lexicographic sort + origin prepend ........ castor.py:146-190
 *   - nearest codeword, exact (fp64) argmax of x.kp with the lowest index on
 *     ties and the origin rule of either caller:
 *       training rule  2*max < c_sq_norm ........ castor.py:448-462, 522, 551-557
 *       pack rule      ||x||_2 < 1e-8 ........... pack.py:169-177
 *   - 18-bit pack / unpack (4 indices -> 9 B) .... castor.py:226-260
 *   - LUT dequant with the two fp16 roundings .... pollux.py:485-500
 *
 * The score of codeword j is accumulated in fp64 as
 *     acc = fma((double)x[i], (double)kp[j][i], acc)   for i = 0..23 in order,
 * which is exact up to one fp64 rounding per step because every fp32 x fp32
 * product is exact in fp64.  The CUDA rescore uses the same order, so the two
 * agree bit for bit whenever both consider the winning codeword.
 *
 * Build: see oracle/Makefile (gcc -O3 -pthread -shared).
 */
#include <math.h>
#include <pthread.h>
#include <unistd.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#define H24_DIM 24
#define H24_KISSING 196560
#define H24_COUNT 196561

/* fp32 value of 1/sqrt(8), the Python float LEECH_SCALE rounded to fp32 as
 * torch does when it multiplies a float32 tensor by a Python scalar
 * (castor.py:68, :158). */
static const float kLeechScaleF = 0.35355339059327373f;

/* float(kissing_points[0].pow(2).sum()) at castor.py:522; 4 - 2^-22. */
static const double kCSqNorm = 3.999999761581421;

/* ------------------------------------------------------------------------ */
/* Golay code (castor.py:74-95)                                              */
/* ------------------------------------------------------------------------ */
static const uint32_t kGolayPoly =
    (1u << 11) | (1u << 9) | (1u << 7) | (1u << 6) | (1u << 5) | (1u << 1) | 1u;

static int bit_length(uint32_t v) { int n = 0; while (v) { ++n; v >>= 1; } return n; }

static uint32_t gf2_mod(uint32_t dividend, uint32_t divisor, int deg) {
  uint32_t v = dividend;
  while (bit_length(v) - 1 >= deg) {
    int shift = (bit_length(v) - 1) - deg;
    v ^= divisor << shift;
  }
  return v;
}

static void golay24_words(uint32_t *words /* 4096 */) {
  for (uint32_t msg = 0; msg < 4096; ++msg) {
    uint32_t w23 = (msg << 11) | gf2_mod(msg << 11, kGolayPoly, 11);
    uint32_t parity = (uint32_t)__builtin_popcount(w23) & 1u;
    words[msg] = (parity << 23) | w23;
  }
}

/* ------------------------------------------------------------------------ */
/* Codebook (castor.py:98-190)                                               */
/* ------------------------------------------------------------------------ */
/* np.lexsort over columns 23..0 makes the last key (column 0) primary, so the
 * rows end up in ascending lexicographic order of (col0, col1, ..., col23).
 * Scaling by 1/sqrt(8) is monotonic and keeps the nine raw values distinct,
 * so sorting the raw integers gives the same permutation. */
static int cmp_rows_lex(const void *pa, const void *pb) {
  const int8_t *a = (const int8_t *)pa, *b = (const int8_t *)pb;
  for (int i = 0; i < H24_DIM; ++i) {
    if (a[i] != b[i]) return (a[i] < b[i]) ? -1 : 1;
  }
  return 0;
}

/* Raw integer kissing points (entries in {0,+-1,+-2,+-3,+-4}), sorted as the
 * reference sorts them.  out: [196560][24] int8.  Returns 0 on success. */
int h24o_raw_kissing_points(int8_t *out) {
  uint32_t golay[4096];
  golay24_words(golay);
  size_t n = 0;
  /* Type 1: two coordinates at +-4 (castor.py:108-114). */
  for (int i = 0; i < H24_DIM; ++i)
    for (int j = i + 1; j < H24_DIM; ++j)
      for (int sa = -1; sa <= 1; sa += 2)
        for (int sb = -1; sb <= 1; sb += 2) {
          int8_t *row = out + n * H24_DIM;
          memset(row, 0, H24_DIM);
          row[i] = (int8_t)(4 * sa);
          row[j] = (int8_t)(4 * sb);
          ++n;
        }
  /* Type 2: +-2 on the octads, even number of minus signs (castor.py:118-130). */
  for (int w = 0; w < 4096; ++w) {
    uint32_t word = golay[w];
    if (__builtin_popcount(word) != 8) continue;
    int pos[8], np = 0;
    for (int b = 0; b < 24; ++b) if ((word >> b) & 1u) pos[np++] = b;
    for (int mask = 0; mask < 256; ++mask) {
      int neg = 8 - __builtin_popcount((unsigned)mask);
      if (neg % 2 != 0) continue;
      int8_t *row = out + n * H24_DIM;
      memset(row, 0, H24_DIM);
      for (int k = 0; k < 8; ++k) row[pos[k]] = (int8_t)(((mask >> k) & 1) ? 2 : -2);
      ++n;
    }
  }
  /* Type 3: -1 on the word's support, +1 elsewhere, then -3 at pos
   * (castor.py:134-141). */
  for (int p = 0; p < H24_DIM; ++p)
    for (int w = 0; w < 4096; ++w) {
      int8_t *row = out + n * H24_DIM;
      for (int b = 0; b < 24; ++b) row[b] = ((golay[w] >> b) & 1u) ? -1 : 1;
      row[p] = -3;
      ++n;
    }
  if (n != H24_KISSING) return 1;
  qsort(out, n, H24_DIM, cmp_rows_lex);
  for (size_t r = 1; r < n; ++r)
    if (cmp_rows_lex(out + (r - 1) * H24_DIM, out + r * H24_DIM) == 0) return 2;
  return 0;
}

/* fp32 value the reference stores for raw coordinate v (castor.py:158). */
float h24o_scaled_value(int v) { return (float)v * kLeechScaleF; }

/* Full fp32 codebook [196561][24] with the origin at row 0. */
int h24o_codebook_f32(float *out) {
  int8_t *raw = (int8_t *)malloc((size_t)H24_KISSING * H24_DIM);
  if (!raw) return 3;
  int rc = h24o_raw_kissing_points(raw);
  if (rc == 0) {
    memset(out, 0, H24_DIM * sizeof(float));
    for (size_t k = 0; k < (size_t)H24_KISSING * H24_DIM; ++k)
      out[H24_DIM + k] = h24o_scaled_value(raw[k]);
  }
  free(raw);
  return rc;
}

double h24o_c_sq_norm(void) { return kCSqNorm; }

/* ------------------------------------------------------------------------ */
/* Nearest codeword, exact fp64 (castor.py:386-462, 549-557; pack.py:169-177) */
/* ------------------------------------------------------------------------ */
enum { H24_RULE_TRAIN = 0, H24_RULE_PACK = 1 };

/* kp: [196560][24] fp32 kissing points (codebook rows 1..).
 * x: [n][24] fp32 atoms.  out_idx: [n] int32 codebook indices.
 * out_best (optional): [n] fp64 best score.  nthreads <= 0 uses every core. */
typedef struct {
  const float *kpT, *x;
  int64_t n;
  int rule;
  int32_t *out_idx;
  double *out_best;
  int64_t next; /* next atom block, taken under the lock */
  pthread_mutex_t lock;
} nearest_job;

enum { JB = 1024, AB = 4 };

static void nearest_block(const nearest_job *job, int64_t a0) {
  const float *kpT = job->kpT, *x = job->x;
  int na = (int)((job->n - a0) < AB ? (job->n - a0) : AB);
  double best[AB];
  int32_t arg[AB];
  static __thread double acc[AB][JB];
  for (int a = 0; a < AB; ++a) { best[a] = -INFINITY; arg[a] = 0; }
  for (int64_t j0 = 0; j0 < H24_KISSING; j0 += JB) {
    int nj = (int)((H24_KISSING - j0) < JB ? (H24_KISSING - j0) : JB);
    for (int a = 0; a < na; ++a) {
      for (int jj = 0; jj < nj; ++jj) acc[a][jj] = 0.0;
      for (int i = 0; i < H24_DIM; ++i) {
        const double xi = (double)x[(a0 + a) * H24_DIM + i];
        const float *col = kpT + (size_t)i * H24_KISSING + j0;
        for (int jj = 0; jj < nj; ++jj) acc[a][jj] = fma(xi, (double)col[jj], acc[a][jj]);
      }
      for (int jj = 0; jj < nj; ++jj)
        if (acc[a][jj] > best[a]) { best[a] = acc[a][jj]; arg[a] = (int32_t)(j0 + jj); }
    }
  }
  for (int a = 0; a < na; ++a) {
    const float *xa = x + (a0 + a) * H24_DIM;
    int zero;
    if (job->rule == H24_RULE_PACK) {
      double ss = 0.0;
      for (int i = 0; i < H24_DIM; ++i) ss = fma((double)xa[i], (double)xa[i], ss);
      zero = sqrt(ss) < 1e-8;
    } else {
      zero = (2.0 * best[a]) < kCSqNorm;
    }
    job->out_idx[a0 + a] = zero ? 0 : arg[a] + 1;
    if (job->out_best) job->out_best[a0 + a] = best[a];
  }
}

static void *nearest_worker(void *arg) {
  nearest_job *job = (nearest_job *)arg;
  for (;;) {
    pthread_mutex_lock(&job->lock);
    int64_t a0 = job->next;
    job->next += AB;
    pthread_mutex_unlock(&job->lock);
    if (a0 >= job->n) break;
    nearest_block(job, a0);
  }
  return NULL;
}

void h24o_nearest(const float *kp, const float *x, int64_t n, int rule,
                  int32_t *out_idx, double *out_best, int nthreads) {
  /* Transposed copy so the inner loop runs over codewords. */
  float *kpT = (float *)malloc((size_t)H24_KISSING * H24_DIM * sizeof(float));
  for (int64_t j = 0; j < H24_KISSING; ++j)
    for (int i = 0; i < H24_DIM; ++i) kpT[(size_t)i * H24_KISSING + j] = kp[j * H24_DIM + i];
  if (nthreads <= 0) nthreads = (int)sysconf(_SC_NPROCESSORS_ONLN);
  if (nthreads < 1) nthreads = 1;
  if (nthreads > 256) nthreads = 256;
  nearest_job job = {kpT, x, n, rule, out_idx, out_best, 0, PTHREAD_MUTEX_INITIALIZER};
  pthread_t th[256];
  int started = 0;
  for (int t = 1; t < nthreads; ++t)
    if (pthread_create(&th[started], NULL, nearest_worker, &job) == 0) ++started;
  nearest_worker(&job);
  for (int t = 0; t < started; ++t) pthread_join(th[t], NULL);
  free(kpT);
}

/* Exact fp64 score of atom x against codebook row `index` (0 = origin). */
double h24o_score(const float *kp, const float *x, int32_t index) {
  if (index <= 0) return 0.0;
  const float *c = kp + (size_t)(index - 1) * H24_DIM;
  double acc = 0.0;
  for (int i = 0; i < H24_DIM; ++i) acc = fma((double)x[i], (double)c[i], acc);
  return acc;
}

/* Squared Euclidean distance in fp64 between x and codebook row `index`. */
double h24o_dist2(const float *kp, const float *x, int32_t index) {
  double acc = 0.0;
  for (int i = 0; i < H24_DIM; ++i) {
    double c = index <= 0 ? 0.0 : (double)kp[(size_t)(index - 1) * H24_DIM + i];
    double d = (double)x[i] - c;
    acc += d * d;
  }
  return acc;
}

/* ------------------------------------------------------------------------ */
/* 18-bit pack / unpack (castor.py:226-260)                                  */
/* ------------------------------------------------------------------------ */
/* idx: [n] int32 (already truncated to 32 bits as .to(torch.int32) does).
 * out: [ceil(n/4)*9] bytes.  Missing tail indices are zero. */
void h24o_pack(const int32_t *idx, int64_t n, uint8_t *out) {
  int64_t groups = (n + 3) / 4;
  for (int64_t g = 0; g < groups; ++g) {
    int32_t v[4];
    for (int k = 0; k < 4; ++k) v[k] = (4 * g + k < n) ? idx[4 * g + k] : 0;
    uint8_t *o = out + 9 * g;
    o[0] = (uint8_t)((v[0] >> 10) & 0xFF);
    o[1] = (uint8_t)((v[0] >> 2) & 0xFF);
    o[2] = (uint8_t)(((v[0] & 0x03) << 6) | ((v[1] >> 12) & 0x3F));
    o[3] = (uint8_t)((v[1] >> 4) & 0xFF);
    o[4] = (uint8_t)(((v[1] & 0x0F) << 4) | ((v[2] >> 14) & 0x0F));
    o[5] = (uint8_t)((v[2] >> 6) & 0xFF);
    o[6] = (uint8_t)(((v[2] & 0x3F) << 2) | ((v[3] >> 16) & 0x03));
    o[7] = (uint8_t)((v[3] >> 8) & 0xFF);
    o[8] = (uint8_t)(v[3] & 0xFF);
  }
}

/* packed: [groups*9] bytes -> out: [min(n, 4*groups)] int32. */
void h24o_unpack(const uint8_t *packed, int64_t groups, int64_t n, int32_t *out) {
  int64_t total = 4 * groups;
  if (n > total) n = total;
  for (int64_t g = 0; g < groups; ++g) {
    const uint8_t *c = packed + 9 * g;
    int32_t v[4];
    v[0] = ((int32_t)c[0] << 10) | ((int32_t)c[1] << 2) | ((int32_t)c[2] >> 6);
    v[1] = (((int32_t)c[2] & 0x3F) << 12) | ((int32_t)c[3] << 4) | ((int32_t)c[4] >> 4);
    v[2] = (((int32_t)c[4] & 0x0F) << 14) | ((int32_t)c[5] << 6) | ((int32_t)c[6] >> 2);
    v[3] = (((int32_t)c[6] & 0x03) << 16) | ((int32_t)c[7] << 8) | (int32_t)c[8];
    for (int k = 0; k < 4; ++k)
      if (4 * g + k < n) out[4 * g + k] = v[k];
  }
}

/* ------------------------------------------------------------------------ */
/* LUT dequant (pollux.py:485-500)                                           */
/* ------------------------------------------------------------------------ */
/* w = fp16( fp32(fp16( fp16(cb)*sigma16 )) * fp32(s_lattice) ), element-wise,
 * where fp16(cb) is the fp16 codebook of get_h24_codebook(device, fp16).
 * cb_f32: [196561][24] fp32 codebook, packed: [ceil(atoms/4)*9] bytes,
 * sigma16: [rows] as raw fp16 bits, out16: [rows*in] raw fp16 bits.
 * Returns the number of indices that were out of range (> 196560). */
int64_t h24o_dequant(const float *cb_f32, const uint8_t *packed, const uint16_t *sigma16,
                     int64_t rows, int64_t in_features, uint16_t *out16) {
  const float s_lattice = (float)0.7071067811865476; /* castor.py:49 */
  int64_t atoms = rows * in_features / H24_DIM;
  int64_t apr = in_features / H24_DIM;
  int32_t *idx = (int32_t *)malloc((size_t)(atoms > 0 ? atoms : 1) * sizeof(int32_t));
  h24o_unpack(packed, (atoms + 3) / 4, atoms, idx);
  int64_t bad = 0;
  for (int64_t a = 0; a < atoms; ++a) {
    int64_t row = a / apr;
    _Float16 sg;
    memcpy(&sg, &sigma16[row], 2);
    int32_t k = idx[a];
    if (k < 0 || k > H24_KISSING) { ++bad; k = 0; }
    for (int i = 0; i < H24_DIM; ++i) {
      _Float16 c16 = (_Float16)cb_f32[(size_t)k * H24_DIM + i];
      _Float16 t = (_Float16)((float)c16 * (float)sg);
      _Float16 w = (_Float16)((float)t * s_lattice);
      memcpy(&out16[a * H24_DIM + i], &w, 2);
    }
  }
  free(idx);
  return bad;
}

/* fp16 row scale of the pack rule (pack.py:164), from an fp64 row RMS:
 * fp16(clamp_min(fp32(sigma) * fp32(sqrt(12)), 1e-8)). */
uint16_t h24o_sigma16_from_rms(float rms) {
  const float sqrt12 = (float)3.4641016151377544;
  float s = rms * sqrt12;
  float eps = (float)1e-8;
  if (s < eps) s = eps;
  _Float16 h = (_Float16)s;
  uint16_t bits;
  memcpy(&bits, &h, 2);
  return bits;
}
