// h24_search.cu -- nearest-codeword search over the 196,560 H24 kissing points
// (castor._leech_nn_kernel, castor.py:386-462; castor_quantize_leech,
// castor.py:487-560; the search of pack._quantize_h24_layer, pack.py:166-177).
//
// Result semantics: index = argmax_j fp64(x . kp_j) + 1 with the lowest j on
// ties, where fp64(x . kp_j) accumulates fma(x_i, kp_ji) for i = 0..23 in
// order, kp_ji = fp32(raw_ji * fp32(1/sqrt(8))) as stored by the reference,
// followed by the caller's origin rule (H24_RULE_TRAIN / H24_RULE_PACK).
//
// The search uses the structure of the codebook (h24_internal.cuh) instead of
// scoring all 196,560 codewords.  In raw units (coordinates x 1/sqrt(8)
// removed), with B(c) = sum_i (-1)^c_i x_i for a Golay codeword c:
//   type 3 (c, p):  S = B(c) - x_p (3 + (-1)^c_p)
//                     = sum_{i != p} (-1)^c_i x_i - 3 x_p;
//   type 2 (octad O, signs s):  S = 2 sum_{i in O} s_i x_i
//                     <= 2 T(O),  T(O) = sum_{i in O} |x_i|;
//   type 1 (a, b, signs):  S = 4 (s_a x_a + s_b x_b) <= 4 (|x_a| + |x_b|).
// Per atom four rows go through one GEMM against the Golay sign columns
// ((-1)^c_k, bf16), of which only one column of each complementary pair is
// multiplied (every row r gives r(~c) = -r(c)): "slice" rows x with x_p1 or x_p2 zeroed (p1, p2, p3 =
// the positions of the three smallest coordinates), which give the exact
// type-3 scores of the codewords (c, p1) and (c, p2) up to the constant
// -3 x_p; the plain row, which gives B(c); and the row |x|, whose value at the
// weight-16 column c is 2 T(O) - sum|x| for the octad O = complement of c
// (minus its value at the octad column O).
//
// Pipeline per batch of atoms (one CUDA stream, no host synchronisation):
//   1. prep_kernel      per atom: the four bf16 rows, written straight into
//                       the UMMA shared-memory layout of the screening A
//                       operand, and the per-atom constants (AtomInfo).
//   2. screen_kernel    persistent tcgen05 kernel, one CTA per SM, 64 atoms
//                       (two M=128 tiles of 32 atoms x 4 rows) per work item;
//                       the 2048 representative Golay columns, 16 tiles of
//                       128, are loaded into shared memory once per CTA and
//                       stay there; M128 N128 K32 MMAs into two TMEM
//                       accumulator stages per M-tile, so that the MMAs of one
//                       Golay tile run while the epilogue reads the previous
//                       one.  16 epilogue warps keep, per row and 32-column
//                       sub-chunk, the maximum of |S| (rows 0-2: the columns
//                       and their complements, whose scores are negated, at
//                       once) or, for the |x| row, minus the minimum (the
//                       maximum over the complements); at the end of a work
//                       item they form the atom's best achievable screening
//                       score and flag every sub-chunk that may hold a
//                       codeword within 2E of it (one 64-bit mask per row).
//   3. rescore_kernel   one warp per atom: fp32 scores (from per-atom
//                       partial-sum tables) of the codewords behind the
//                       flagged sub-chunks; a unique best within the fp32 error
//                       bound is the winner, otherwise fp64 scores in the
//                       reference's order for those within the bound, lowest
//                       index on ties; then the origin rule.
//   4. exhaustive_kernel  fp64 scan of all codewords for atoms with more than
//                       kHeavySubs flagged 32-column units (exact ties over
//                       many codewords).
//   5. decode_kernel    kissing-point index of each rescore winner, looked up
//                       in bulk from its candidate code.
//
// Why the flags are sufficient: let S~_j be a screening score with
// |S~_j - sqrt(8) R_j| <= E for every codeword j (R_j the exact score; E from
// the bf16 rounding of x, see prep_kernel).  The atom's `best` is S~ of an
// achievable codeword or a lower bound of the best score among a set of
// codewords computed the same way, so sqrt(8) R_j* >= best - E for the winner
// j*, and S~_j* >= best - 2E = thr.  A chunk is flagged if an upper bound of
// S~ over the codewords it stands for reaches thr:
//   slice rows     the chunk maximum + (-3 x_p);
//   plain row      the chunk maximum + max(4 y3, 2 y3), y3 = -x_p3: every
//                  type-3 codeword (c, p) with p outside {p1, p2} has
//                  y_p <= y3 (y = -x);
//   |x| row        the chunk maximum + sum|hi| = max 2 T~(O) over its octads;
// type-1 codewords are bounded by 4 (|x|_(1) + |x|_(2)) and checked in the
// rescore.  The type-2 contribution to `best` is max_O 2 T~(O) - 4 |x|_(8),
// |x|_(8) the 8th largest |x_i|: flipping the sign of the smallest |x_i| of
// O, which is at most |x|_(8), repairs the parity of any octad.
#include <cstdio>
#include <mutex>

#include "h24_internal.cuh"

namespace h24 {
namespace {

constexpr int kWorkAtoms = 64;                     // atoms per CTA work item
constexpr int kRowsPerAtom = 4;                    // slice p1, slice p2, plain, |x|
constexpr int kMTiles = kWorkAtoms * kRowsPerAtom / 128;  // 2
constexpr int kATileBytes = 128 * kRowBytes;       // 8192
constexpr int kAItemBytes = kMTiles * kATileBytes; // 16384
constexpr int kBTileBytes = kGolayTileN * kRowBytes;  // 8192
constexpr int kSubCols = 32;                       // flagged sub-chunk: a quarter of a Golay tile
constexpr int kScreenTiles = kGolayHalf / kGolayTileN;  // 16 Golay tiles multiplied per work item
constexpr int kOctTiles = (kOctads + 1 + kGolayTileN - 1) / kGolayTileN;  // 6: tiles holding octad columns
constexpr int kOctTailCol = kOctads + 1 - (kOctTiles - 1) * kGolayTileN;  // 120: dodecads from here in tile 5
constexpr int kAccStages = 2;                      // TMEM accumulator stages per M-tile
constexpr int kEpiPerStage = kMTiles * 4;         // 8: epilogue warps reading one accumulator stage
constexpr int kEpiWarps = kEpiPerStage * kAccStages;  // 16: (stage, M-tile, lane quarter)
constexpr int kProducerWarp = kEpiWarps;           // warp 16: TMA producer
constexpr int kIssuerWarp = kEpiWarps + 1;         // warps 17-18: MMA issuer of M-tile 0, 1
constexpr int kScreenThreads = 32 * (kEpiWarps + 1 + kMTiles);  // 608
constexpr uint32_t kTmemCols = kMTiles * kAccStages * kGolayTileN;  // 512
constexpr int kHeavySubs = 384;                    // flagged 32-column units (of 408) beyond which the exhaustive scan runs
constexpr int kMaxSegs = 64;                       // input segments per pipeline batch
constexpr int64_t kBatchAtoms = int64_t(1) << 20;  // atoms per pipeline batch
constexpr unsigned long long kWaitLimitNs = 4000000000ull;  // bounded waits: 4 s (default)
static_assert(kOctTiles == 6 && kOctTailCol == 120, "octad columns 1-759 fill tiles 0-5 up to column 120 of tile 5");
static_assert(kScreenTiles % (2 * kAccStages) == 0, "each stage is used an even number of times per item");

// Row type held by TMEM lane quarter q of M-tile g, and its inverse.  The two
// |x| rows (loaded only for the 6 of the 16 multiplied tiles that hold octad
// columns) sit in lane
// quarters 1 and 2, read by the SM sub-partitions that also run the two MMA
// issuer warps (warp w runs on sub-partition w % 4 and reads quarter w % 4).
__host__ __device__ constexpr int row_of_quarter(int g, int q) {
  return g == 0 ? ((0x2130 >> (4 * q)) & 0xF) : ((q + 1) & 3);
}
__host__ __device__ constexpr int quarter_of_row(int g, int r) {
  return g == 0 ? ((0x1320 >> (4 * r)) & 0xF) : ((r + 3) & 3);
}
static_assert(row_of_quarter(0, quarter_of_row(0, 1)) == 1 && row_of_quarter(0, quarter_of_row(0, 2)) == 2 &&
                  row_of_quarter(0, quarter_of_row(0, 3)) == 3 && row_of_quarter(1, quarter_of_row(1, 0)) == 0 &&
                  row_of_quarter(1, quarter_of_row(1, 3)) == 3 && quarter_of_row(0, 3) == 1 &&
                  quarter_of_row(1, 3) == 2,
              "quarter <-> row type maps are inverse, |x| rows in quarters 1 and 2");

// Sub-chunk of bit b of a row's 64-bit flag mask: bit 32 s + 4 i + j holds
// sub-chunk j (columns 32 j .. 32 j + 31) of Golay tile t = 2 i + s, i.e.
// columns 32 u .. 32 u + 31 for u = 4 t + j (the tiles of accumulator stage s
// fill one 32-bit half of the mask).  For rows 0-2 a bit flags those columns
// together with their complements (columns + 2048); for the |x| row it flags
// only the complements (the weight-16 words).
__host__ __device__ constexpr int sub_of_bit(int b) {
  return 8 * ((b & 31) >> 2) + 4 * (b >> 5) + (b & 3);
}
static_assert(sub_of_bit(0) == 0 && sub_of_bit(3) == 3 && sub_of_bit(32) == 4 && sub_of_bit(4) == 8 &&
                  sub_of_bit(63) == 63,
              "mask bit order");

// Per-atom constants of the search (prep_kernel -> screen and rescore).
struct __align__(16) AtomInfo {
  float off[2];  // -3 x_p1, -3 x_p2: added to the slice rows
  // Bounds of S(c, p) - B(c) = y_p (3 + (-1)^c_p) over the type-3 positions
  // p outside {p1, p2} (y = -x, y3 >= y4 >= every other y_p):
  float u0;      // Golay word without p3: max(4 y3, 2 y4)
  float u1;      // Golay word with p3: max(2 y3, 4 y4, 2 y4)
  float shi;     // sum |hi_i|: added to the |x| row at weight-16 columns
  float t1;      // 4 (|x|_(1) + |x|_(2)): best type-1 score
  float l2s;     // 4 |x|_(3): type-2 parity allowance (>= 4 |x|_(8))
  float two_e;   // 2E, or -1 for an atom with a non-finite coordinate
  float t2lb;    // best type-2 score over the 21 octads through the three largest |x_i|
  uint8_t p[3];  // p1, p2, p3
  int8_t triv;   // index of an atom that needs no search (trivial_index: 0 or 1), else -1
  float thr;     // best - 2E, written by the screen
  float add2;    // the plain row's offset: with x_p3 moved by d in its A row, max(u0 - d, u1 + d)
};
static_assert(sizeof(AtomInfo) == 48, "AtomInfo is three 16-byte loads");

struct __align__(1024) ScreenSmem {
  uint8_t a[2][kAItemBytes];          // A operand of two work items
  uint8_t b[kScreenTiles][kBTileBytes];  // the 16 multiplied Golay tiles, loaded once per CTA
  // Per multiplied Golay tile, pair of 32-column sub-chunks (0-1, 2-3) and
  // epilogue thread slot (M-tile, lane quarter, lane), rounded up to fp16 (so
  // the flags stay conservative): rows 0-2, the maximum of |S| over the
  // sub-chunk, i.e. the larger of its maximum and its complement's; the |x|
  // row, the maximum over the complement sub-chunk (minus the minimum).
  // Each entry is written and read by one thread.
  __half2 cmax[kScreenTiles][2][kWorkAtoms * kRowsPerAtom];
  float rowval[2][kWorkAtoms][kRowsPerAtom][kAccStages];  // row maxima, by work-item parity and stage
  AtomInfo info_st[2][kMTiles][32];   // per-atom constants of the work item, by work-item parity
  uint64_t bar_a_full[2];
  uint64_t bar_a_empty[2];          // one commit per issuer
  uint64_t bar_b_full;              // the Golay tiles have landed
  uint64_t bar_acc_full[kMTiles][kAccStages];
  uint64_t bar_acc_empty[kMTiles][kAccStages];
  uint64_t bar_rows[kMTiles][2];    // the eight warps of an M-tile, by work-item parity
  uint64_t bar_final[kMTiles];      // each issuer's last MMAs
  uint32_t tmem_base;
  int abort_flag;
};
static_assert(sizeof(ScreenSmem) + 1024 <= 227 * 1024, "screen shared memory (plus alignment) fits one CTA");

// ---------------------------------------------------------------------------
// PTX helpers
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint32_t smem_u32(const void *p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void cp_async16(void *dst, const void *src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(dst)), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
__device__ __forceinline__ void cp_async_wait1() { asm volatile("cp.async.wait_group 1;" ::: "memory"); }
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_all;" ::: "memory"); }

__device__ __forceinline__ void mbar_init(uint64_t *bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t *bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
               "r"(bytes)
               : "memory");
}

// Suspend-time hint (ns) of the mbarrier waits: with a hint a waiting thread
// sleeps until the phase completes or the hint expires; 0 = no hint (the
// hardware's own time limit).  Measured on the screen: no hint 0.643 ms per
// launch of 1M atoms, hints of 200 ns and 1 ms 0.674, a test_wait spin 0.692
// (the woken warps start later after a hinted wait).
#ifndef H24_WAIT_HINT_NS
#define H24_WAIT_HINT_NS 0
#endif

// One potentially blocking test of the phase.
__device__ __forceinline__ bool mbar_try_wait(uint64_t *bar, uint32_t parity) {
  uint32_t ok;
#if H24_WAIT_HINT_NS > 0
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity), "r"(static_cast<uint32_t>(H24_WAIT_HINT_NS))
      : "memory");
#else
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
#endif
  return ok != 0;
}

__device__ __forceinline__ unsigned long long global_ns() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
  return t;
}

// Non-blocking test of the phase with the given parity.
__device__ __forceinline__ bool mbar_test(uint64_t *bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Slow path of wait_bar.  Gives up after `limit` ns or when another role of
// the CTA has aborted; on a timeout it raises the CTA abort flag and the
// device error word.
__device__ __noinline__ bool wait_slow(uint64_t *bar, uint32_t parity, volatile int *abort_flag,
                                       int *err, unsigned long long limit) {
  const unsigned long long t0 = global_ns();
  for (;;) {
    if (mbar_try_wait(bar, parity)) return true;
    if (*abort_flag) return false;
    if (global_ns() - t0 > limit) {
      *abort_flag = 1;
      atomicExch(err, H24_ERR_TIMEOUT);
      return false;
    }
  }
}

// Waits for the phase of `bar` with the given parity (inline fast path).
__device__ __forceinline__ bool wait_bar(uint64_t *bar, uint32_t parity, volatile int *abort_flag,
                                         int *err, unsigned long long limit) {
  if (mbar_test(bar, parity)) return true;
  return wait_slow(bar, parity, abort_flag, err, limit);
}

// One arrival on `bar` from lane 0 of a converged warp: a predicated
// instruction rather than a branch around it.
__device__ __forceinline__ void mbar_arrive_lane0(uint64_t *bar, int lane) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.eq.u32 p, %1, 0;\n\t"
      "@p mbarrier.arrive.shared::cta.b64 _, [%0];\n\t}" ::"r"(smem_u32(bar)),
      "r"(lane)
      : "memory");
}

// wait_bar for a whole converged warp, every lane polling (no divergent
// region); the result is the same on all lanes.
__device__ __forceinline__ bool wait_bar_warp(uint64_t *bar, uint32_t parity, volatile int *abort_flag,
                                              int *err, unsigned long long limit) {
  if (__all_sync(0xffffffffu, mbar_test(bar, parity))) return true;
  return __all_sync(0xffffffffu, wait_slow(bar, parity, abort_flag, err, limit));
}

__device__ __forceinline__ void bulk_g2s(void *dst, const void *src, uint32_t bytes, uint64_t *bar,
                                         uint64_t policy) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint "
      "[%0], [%1], %2, [%3], %4;" ::"r"(smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar)), "l"(policy)
      : "memory");
}

__device__ __forceinline__ uint64_t policy_evict_first() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
  return p;
}

__device__ __forceinline__ uint64_t policy_evict_last() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(p));
  return p;
}


__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// Shared-memory matrix descriptor for a K-major operand without swizzle
// (core matrices of 8 rows x 16 bytes): LBO = distance between the two
// K-adjacent core matrices of one MMA (128 B), SBO = distance between 8-row
// groups (512 B), version 1 (sm_100).
__device__ __forceinline__ uint64_t smem_desc(uint32_t addr) {
  return static_cast<uint64_t>((addr >> 4) & 0x3FFFu) | (static_cast<uint64_t>(128 >> 4) << 16) |
         (static_cast<uint64_t>(512 >> 4) << 32) | (uint64_t(1) << 46);
}

// Instruction descriptor: kind::f16, A = B = bf16, D = f32, both K-major,
// M = 128, N = 128.
constexpr uint32_t kIdesc = (1u << 4) | (1u << 7) | (1u << 10) | ((128u >> 3) << 17) |
                            ((128u >> 4) << 24);

// D (TMEM) += A x B, both from shared-memory descriptors; accumulate == 0
// overwrites D.  Executed by a whole converged warp (every lane, warp-uniform
// operands); the lane chosen by elect.sync issues it, the same lane every
// time since the warp is fully active.
__device__ __forceinline__ void mma_bf16_ss(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc,
                                            uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p, e;\n\t"
      "elect.sync _|e, 0xffffffff;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "@e tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(kIdesc), "r"(accumulate)
      : "memory");
}

// Arrival on `bar` once the MMAs issued so far by the elected lane complete
// (whole converged warp, as mma_bf16_ss).
__device__ __forceinline__ void mma_commit(uint64_t *bar) {
  asm volatile(
      "{\n\t.reg .pred e;\n\t"
      "elect.sync _|e, 0xffffffff;\n\t"
      "@e tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];\n\t}" ::"r"(
          smem_u32(bar))
      : "memory");
}

#define H24_R8(b) "=r"(r[b + 0]), "=r"(r[b + 1]), "=r"(r[b + 2]), "=r"(r[b + 3]), \
                  "=r"(r[b + 4]), "=r"(r[b + 5]), "=r"(r[b + 6]), "=r"(r[b + 7])

// 32 lanes x 64 consecutive 32-bit TMEM columns, waited for in the same
// statement.
__device__ __forceinline__ void tmem_ld64_wait(uint32_t taddr, uint32_t *r) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x64.b32 {"
      "%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32,%33,%34,%35,%36,%37,%38,%39,%40,%41,%42,%43,%44,%45,%46,%47,%48,%49,%50,%51,%52,%53,%54,%55,%56,%57,%58,%59,%60,%61,%62,%63}, [%64];\n\t"
      "tcgen05.wait::ld.sync.aligned;"
      : H24_R8(0), H24_R8(8), H24_R8(16), H24_R8(24), H24_R8(32), H24_R8(40), H24_R8(48), H24_R8(56)
      : "r"(taddr)
      : "memory");
}

#undef H24_R8

__device__ __forceinline__ float fmax3(float a, float b, float c) {
  float d;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
  return d;
}

__device__ __forceinline__ float fmin3(float a, float b, float c) {
  float d;
  asm("min.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
  return d;
}

// min(m, the 32 fp32 values held as raw bits): a tree of 3-input min.
__device__ __forceinline__ float min32(float m, const uint32_t *r) {
  float t[11];
#pragma unroll
  for (int k = 0; k < 10; ++k)
    t[k] = fmin3(__uint_as_float(r[3 * k]), __uint_as_float(r[3 * k + 1]),
                 __uint_as_float(r[3 * k + 2]));
  t[10] = fmin3(__uint_as_float(r[30]), __uint_as_float(r[31]), m);
  const float u0 = fmin3(t[0], t[1], t[2]), u1 = fmin3(t[3], t[4], t[5]);
  const float u2 = fmin3(t[6], t[7], t[8]);
  return fmin3(fmin3(u0, u1, u2), t[9], t[10]);
}

// max(m, |the 32 fp32 values held as raw bits|): a tree of 3-input max (the
// absolute values are operand modifiers of the max, not extra instructions).
__device__ __forceinline__ float max32abs(float m, const uint32_t *r) {
  float t[11];
#pragma unroll
  for (int k = 0; k < 10; ++k)
    t[k] = fmax3(fabsf(__uint_as_float(r[3 * k])), fabsf(__uint_as_float(r[3 * k + 1])),
                 fabsf(__uint_as_float(r[3 * k + 2])));
  t[10] = fmax3(fabsf(__uint_as_float(r[30])), fabsf(__uint_as_float(r[31])), m);
  const float u0 = fmax3(t[0], t[1], t[2]), u1 = fmax3(t[3], t[4], t[5]);
  const float u2 = fmax3(t[6], t[7], t[8]);
  return fmax3(fmax3(u0, u1, u2), t[9], t[10]);
}

// ---------------------------------------------------------------------------
// 1. prep
// ---------------------------------------------------------------------------
// Index for atoms that need no search: non-finite input (training rule: the
// origin, as the Triton kernel's never-improving running max snaps; pack rule:
// row 1, torch.max's first NaN), or the pack rule's ||x|| < 1e-8.
// Returns -1 when a search is needed.
__device__ __forceinline__ int trivial_index(const float (&v)[kDim], int rule) {
  bool finite = true;
#pragma unroll
  for (int i = 0; i < kDim; ++i) finite = finite && isfinite(v[i]);
  if (!finite) return rule == H24_RULE_TRAIN ? 0 : 1;
  if (rule == H24_RULE_PACK) {
    double ss = 0.0;
#pragma unroll
    for (int i = 0; i < kDim; ++i) ss = __fma_rn(static_cast<double>(v[i]), static_cast<double>(v[i]), ss);
    if (sqrt(ss) < 1e-8) return 0;
  }
  return -1;
}

// Input atoms of one pipeline batch: segment i holds atoms [start[i],
// start[i+1]) of the batch, stored contiguously at x[i] (24 elements per
// atom, all of the batch's element type: fp32, or bf16 widened exactly to
// fp32 on load, as the reference's weight.float() does, pack.py:159).
struct Segs {
  const void *x[kMaxSegs];
  int64_t start[kMaxSegs + 1];
  int count;
};

template <typename T>
__device__ __forceinline__ const T *atom_ptr(const Segs &sg, int64_t a) {
  int lo = 0, hi = sg.count - 1;
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (sg.start[mid] <= a) lo = mid; else hi = mid - 1;
  }
  return static_cast<const T *>(sg.x[lo]) + (a - sg.start[lo]) * kDim;
}

// 16-byte chunks of one atom of element type T (6 for fp32, 3 for bf16).
template <typename T>
constexpr int atom_chunks() { return static_cast<int>(kDim * sizeof(T) / 16); }

// bf16 bit pattern (low 16 bits of h) widened to fp32: exact.
__device__ __forceinline__ float bf16_bits_to_float(uint32_t h) { return __uint_as_float(h << 16); }

// The 24 coordinates of an atom as fp32, from 16-byte loads; `stream` marks
// data read once (evict-first loads).
template <typename T, bool stream>
__device__ __forceinline__ void load_atom_t(const T *__restrict__ p, float (&v)[kDim]) {
  const uint4 *src = reinterpret_cast<const uint4 *>(p);
#pragma unroll
  for (int q = 0; q < atom_chunks<T>(); ++q) {
    const uint4 u = stream ? __ldcs(src + q) : __ldg(src + q);
    if constexpr (sizeof(T) == 4) {
      v[4 * q + 0] = __uint_as_float(u.x);
      v[4 * q + 1] = __uint_as_float(u.y);
      v[4 * q + 2] = __uint_as_float(u.z);
      v[4 * q + 3] = __uint_as_float(u.w);
    } else {
      const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        v[8 * q + 2 * k] = bf16_bits_to_float(w[k] & 0xFFFFu);
        v[8 * q + 2 * k + 1] = __uint_as_float(w[k] & 0xFFFF0000u);
      }
    }
  }
}

// Byte offset of M-tile lane L, 16-byte K chunk q in an A tile (UMMA
// canonical K-major layout without swizzle: 8-row groups at 512 B, K chunks
// at 128 B, rows at 16 B).
__device__ __forceinline__ uint32_t a_offset(int L, int q) {
  return static_cast<uint32_t>((L >> 3) * 512 + q * 128 + (L & 7) * 16);
}

// Atom a of work item w = a / 64 sits in M-tile g = (a / 32) % 2 at lane
// 32 * quarter_of_row(g, r) + a % 32 for row type r (0 slice p1, 1 slice p2,
// 2 plain, 3 |x|).
template <typename T>
__global__ void __launch_bounds__(256, 4) prep_kernel(const __grid_constant__ Segs sg, int64_t n,
                                                   int64_t n_pad, int rule,
                                                   const uint2 *__restrict__ oct_by_triple,
                                                   uint8_t *__restrict__ a_tiles,
                                                   AtomInfo *__restrict__ info,
                                                   int32_t *__restrict__ ovf_count) {
  // |x_i| of each thread's atom, [position][thread]: a warp's accesses hit 32
  // distinct banks whatever the positions.
  __shared__ float absx[kDim][256];
  pdl_enter();
  const int64_t a = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x;
  // The batch's exhaustive-scan list starts empty (the previous batch on
  // this stream has finished with it; the rescore of this one fills it).
  if (a == 0) *ovf_count = 0;
  if (a >= n_pad) return;
  float v[kDim];
  if (a < n) {
    load_atom_t<T, true>(atom_ptr<T>(sg, a), v);
  } else {
#pragma unroll
    for (int i = 0; i < kDim; ++i) v[i] = 0.f;
  }
  float sum_d = 0.f, sum_d2 = 0.f, sum_x = 0.f, shi = 0.f;
  bool finite = true;
  uint16_t hb[kDim];
  // Three smallest coordinates (lowest position first on ties) and the three
  // largest |x_i|.
  float s0 = INFINITY, s1 = INFINITY, s2 = INFINITY, s3 = INFINITY;
  int q0 = 0, q1 = 1, q2 = 2;
  float top[3];
#pragma unroll
  for (int k = 0; k < 3; ++k) top[k] = 0.f;
  int a0 = 0, a1 = 1, a2 = 2;  // positions of the three largest |x_i|
  uint32_t negm = 0;
#pragma unroll
  for (int i = 0; i < kDim; ++i) {
    const __nv_bfloat16 h = __float2bfloat16_rn(v[i]);
    const float hf = __bfloat162float(h);
    hb[i] = __bfloat16_as_ushort(h);
    const float d = fabsf(v[i] - hf);
    sum_d += d;
    sum_d2 = fmaf(d, d, sum_d2);
    sum_x += fabsf(v[i]);
    shi += fabsf(hf);
    finite = finite && isfinite(v[i]);
    const float x = v[i];
    if (x < s3) {
      if (x < s2) {
        s3 = s2;
        if (x < s1) {
          s2 = s1; q2 = q1;
          if (x < s0) { s1 = s0; q1 = q0; s0 = x; q0 = i; }
          else { s1 = x; q1 = i; }
        } else { s2 = x; q2 = i; }
      } else { s3 = x; }
    }
    negm |= (x < 0.f ? 1u : 0u) << i;
    if (fabsf(x) > top[2]) {
      if (fabsf(x) > top[1]) {
        a2 = a1;
        if (fabsf(x) > top[0]) { a1 = a0; a0 = i; } else { a1 = i; }
      } else { a2 = i; }
    }
    float t = fabsf(x);
#pragma unroll
    for (int k = 0; k < 3; ++k) {
      const float hi_k = fmaxf(top[k], t);
      t = fminf(top[k], t);
      top[k] = hi_k;
    }
  }
  // |sum_i coef_i d_i| <= min(4 sum|d|, sqrt(32) ||d||) for every codeword
  // (|coef| <= 4, sum coef^2 = 32); tensor-core accumulation, the fp32
  // rounding of 3*LEECH_SCALE, the fp32 terms of the screen and rescore and
  // the fp64 rescore add at most 2^-12 * sum|x| (raw units).  The factor
  // 1.001 absorbs the fp32 rounding of these sums.
  const float e_hi = fminf(4.f * sum_d, 5.656854249f * sqrtf(sum_d2));
  const float e = (e_hi + 2.44140625e-4f * sum_x) * 1.001f;
  AtomInfo inf;
  inf.off[0] = -3.f * s0;
  inf.off[1] = -3.f * s1;
  const float y3 = -s2, y4 = -s3;
  inf.u0 = fmaxf(4.f * y3, 2.f * y4);
  inf.u1 = fmaxf(2.f * y3, fmaxf(4.f * y4, 2.f * y4));
  inf.shi = shi;
  inf.t1 = 4.f * (top[0] + top[1]);
  // The parity allowance of the |x|-row bound: 4 min_O |x_i| <= 4 |x|_(8) <=
  // 4 |x|_(3) for every octad O (the larger value only lowers the bound; the
  // prep's type-2 bound over the octads through the three largest |x_i| is
  // the tighter one in practice, and the flags of N(0,1) atoms are the same).
  inf.l2s = 4.f * top[2];
  inf.two_e = finite ? 2.f * e : -1.f;
  // Achievable type-2 score: the best even-parity pattern, 2 T(O) - 4 [odd]
  // min_O |x|, over the 21 octads that contain the three largest |x_i|.
  float t2lb = -INFINITY;
  {
#pragma unroll
    for (int i = 0; i < kDim; ++i) absx[i][threadIdx.x] = fabsf(v[i]);
    // Sort the triple: i < j < k.
    const int i3 = min(a0, min(a1, a2)), k3 = max(a0, max(a1, a2)), j3 = a0 + a1 + a2 - i3 - k3;
    const uint2 *row = oct_by_triple + (k3 * (k3 - 1) * (k3 - 2) / 6 + j3 * (j3 - 1) / 2 + i3) * kTripleRow;
    // The triple's |x| are the three largest: top[0..2].
    const float tri = top[0] + top[1] + top[2];
#pragma unroll 3
    for (int k = 0; k < 21; ++k) {
      const uint2 e = __ldg(row + k);
      float t = tri, mn = top[2];
#pragma unroll
      for (int q = 0; q < 5; ++q) {
        const float ax = absx[(e.y >> (5 * q)) & 31u][threadIdx.x];
        t += ax;
        mn = fminf(mn, ax);
      }
      t2lb = fmaxf(t2lb, 2.f * t - ((__popc(e.x & negm) & 1) ? 4.f * mn : 0.f));
    }
  }
  inf.t2lb = t2lb;
  inf.p[0] = static_cast<uint8_t>(q0);
  inf.p[1] = static_cast<uint8_t>(q1);
  inf.p[2] = static_cast<uint8_t>(q2);
  inf.thr = -INFINITY;
  // The plain row bounds S(c, p) over the positions p outside {p1, p2} by
  // B(c) + u1 for Golay words holding p3 and B(c) + u0 for the others.  Its A
  // row carries x_p3 + d (rounded to bf16), which adds +d to B(c) for words
  // without p3 and -d for words with it (and the opposite for the complement
  // columns, whose scores are negated); then one offset max(u0 - d, u1 + d)
  // bounds both, where max(u0, u1) did before.  d ~ (u0 - u1) / 2.
  uint16_t hb3 = 0;
#pragma unroll
  for (int i = 0; i < kDim; ++i)
    if (i == q2) hb3 = hb[i];
  const float hf3 = __uint_as_float(static_cast<uint32_t>(hb3) << 16);
  const __nv_bfloat16 v3 = __float2bfloat16_rn(hf3 + 0.5f * (inf.u0 - inf.u1));
  const float d3 = __bfloat162float(v3) - hf3;  // exact: both are bf16 values
  inf.add2 = fmaxf(inf.u0 - d3, inf.u1 + d3);
  hb3 = __bfloat16_as_ushort(v3);
  // Atoms that need no search: non-finite, or (pack rule) an exact norm below
  // 1e-8, which needs every |x_i| < 2e-8 first (||x|| >= max |x_i|).
  inf.triv = !finite ? (rule == H24_RULE_TRAIN ? 0 : 1)
                     : (rule == H24_RULE_PACK && top[0] < 2e-8f ? trivial_index(v, rule) : -1);
  info[a] = inf;

  uint8_t *item = a_tiles + (a / kWorkAtoms) * kAItemBytes;
  const int g = static_cast<int>((a >> 5) & (kMTiles - 1)), l = static_cast<int>(a & 31);
#pragma unroll
  for (int r = 0; r < kRowsPerAtom; ++r) {
    uint32_t w[16];
#pragma unroll
    for (int k = 0; k < 12; ++k) {
      uint32_t lo = hb[2 * k], hi = hb[2 * k + 1];
      if (r == 3) { lo &= 0x7FFFu; hi &= 0x7FFFu; }
      if (r < 2) {
        const int p = r == 0 ? q0 : q1;
        if (p == 2 * k) lo = 0;
        if (p == 2 * k + 1) hi = 0;
      }
      if (r == 2) {
        if (q2 == 2 * k) lo = hb3;
        if (q2 == 2 * k + 1) hi = hb3;
      }
      w[k] = lo | (hi << 16);
    }
#pragma unroll
    for (int k = 12; k < 16; ++k) w[k] = 0;
    uint8_t *tile = item + g * kATileBytes;
    const int L = 32 * quarter_of_row(g, r) + l;
#pragma unroll
    for (int q = 0; q < 4; ++q)
      *reinterpret_cast<uint4 *>(tile + a_offset(L, q)) =
          make_uint4(w[4 * q], w[4 * q + 1], w[4 * q + 2], w[4 * q + 3]);
  }
}

// ---------------------------------------------------------------------------
// 2. tcgen05 screening
// ---------------------------------------------------------------------------
struct ScreenArgs {
  const uint8_t *a_tiles;   // [items][kAItemBytes]
  AtomInfo *info;           // [n_pad]; the screen fills in thr
  const uint8_t *golay;     // [kGolayTiles][kBTileBytes]
  uint2 *masks;             // [n][4] flagged 32-column sub-chunks per row type
  int64_t n;
  int64_t items;
  int *err;
  unsigned long long wait_limit_ns;  // limit of every bounded wait
};

__global__ void __launch_bounds__(kScreenThreads, 1) screen_kernel(const ScreenArgs args) {
  extern __shared__ uint8_t smem_raw[];
  ScreenSmem &S = *reinterpret_cast<ScreenSmem *>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  volatile int *abort_flag = &S.abort_flag;

  if (threadIdx.x == 0) {
    for (int i = 0; i < 2; ++i) {
      mbar_init(&S.bar_a_full[i], 1);
      mbar_init(&S.bar_a_empty[i], kMTiles);
      for (int g = 0; g < kMTiles; ++g) mbar_init(&S.bar_rows[g][i], 4 * kAccStages);
    }
    mbar_init(&S.bar_b_full, 1);
    for (int g = 0; g < kMTiles; ++g) {
      for (int s = 0; s < kAccStages; ++s) {
        mbar_init(&S.bar_acc_full[g][s], 1);
        mbar_init(&S.bar_acc_empty[g][s], 4);  // the four lane-quarter warps of M-tile g
      }
      mbar_init(&S.bar_final[g], 1);
    }
    S.abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
  }
  if (warp == kIssuerWarp) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_u32(&S.tmem_base)),
                 "r"(kTmemCols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = S.tmem_base;

  if (warp == kProducerWarp) {
    // ---------------- producer: A of each work item, Golay tiles ----------
    if (lane == 0) {
      const uint64_t keep = policy_evict_last();
      const uint64_t once = policy_evict_first();
      // The Golay tiles are the same for every work item: all 16 are loaded
      // once and stay resident, so the MMAs of the two M-tiles never wait on
      // each other's use of a tile ring.
      mbar_arrive_expect_tx(&S.bar_b_full, kScreenTiles * kBTileBytes);
      for (int t = 0; t < kScreenTiles; ++t)
        bulk_g2s(S.b[t], args.golay + t * kBTileBytes, kBTileBytes, &S.bar_b_full, keep);
      int ab = 0;
      uint32_t aph = 0;
      int last_a[2] = {-1, -1};
      bool ok = true;
      for (int64_t it = blockIdx.x; ok && it < args.items; it += gridDim.x) {
        if (!wait_bar(&S.bar_a_empty[ab], aph ^ 1, abort_flag, args.err, args.wait_limit_ns)) { ok = false; break; }
        mbar_arrive_expect_tx(&S.bar_a_full[ab], kAItemBytes);
        bulk_g2s(S.a[ab], args.a_tiles + it * kAItemBytes, kAItemBytes, &S.bar_a_full[ab], once);
        last_a[ab] = static_cast<int>(aph);
        if (++ab == 2) { ab = 0; aph ^= 1; }
      }
      // Let every copy issued land before the CTA leaves (the Golay tiles
      // too, for a CTA without work items).
      const unsigned long long t0 = global_ns();
      while (!mbar_try_wait(&S.bar_b_full, 0) && global_ns() - t0 < args.wait_limit_ns) {
      }
      if (!ok) {
        for (int i = 0; i < 2; ++i)
          if (last_a[i] >= 0)
            while (!mbar_try_wait(&S.bar_a_full[i], static_cast<uint32_t>(last_a[i])) &&
                   global_ns() - t0 < args.wait_limit_ns) {
            }
      }
    }
  } else if (warp >= kIssuerWarp) {
    // ---------------- MMA issuers, one per M-tile -----------------------------
    // Golay tile t goes into accumulator stage s = t % 2 of M-tile g (TMEM
    // columns 128 (2 g + s)): one M128 N128 K32 product, two K=16 MMAs.  Stage
    // s is used 16 times per work item, so the release awaited before use
    // u = t / 2 has parity (u & 1) ^ 1.
    const int g = warp - kIssuerWarp;
    // The whole warp runs the loop (converged, uniform values); barrier waits
    // are polled by every lane and the MMAs are issued by the elected lane.
    const uint32_t a0 = smem_u32(S.a[0]), b0 = smem_u32(S.b[0]);
    constexpr uint64_t kKStep = 256 >> 4;  // next 16 K: two 16-byte chunks, descriptor units
    int ab = 0;
    uint32_t aph = 0;
    bool ok = blockIdx.x >= args.items ||
              wait_bar_warp(&S.bar_b_full, 0, abort_flag, args.err, args.wait_limit_ns);
    bool issued = false;
    for (int64_t it = blockIdx.x; ok && it < args.items; it += gridDim.x) {
      if (!wait_bar_warp(&S.bar_a_full[ab], aph, abort_flag, args.err, args.wait_limit_ns)) { ok = false; break; }
      tc_fence_after();
      const uint64_t ad = smem_desc(a0 + static_cast<uint32_t>(ab * kAItemBytes + g * kATileBytes));
      for (int t = 0; t < kScreenTiles; ++t) {
        const int s = t & 1;
        if (!wait_bar_warp(&S.bar_acc_empty[g][s], ((t >> 1) & 1) ^ 1, abort_flag, args.err, args.wait_limit_ns)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint64_t bd = smem_desc(b0 + static_cast<uint32_t>(t) * kBTileBytes);
        const uint32_t d = tmem_base + static_cast<uint32_t>((g * kAccStages + s) * kGolayTileN);
        mma_bf16_ss(d, ad, bd, 0);
        mma_bf16_ss(d, ad + kKStep, bd + kKStep, 1);
        mma_commit(&S.bar_acc_full[g][s]);
        issued = true;
      }
      if (!ok) break;
      mma_commit(&S.bar_a_empty[ab]);
      if (++ab == 2) { ab = 0; aph ^= 1; }
    }
    if (issued) {
      // All MMAs of this CTA complete before TMEM is released.
      mma_commit(&S.bar_final[g]);
      const unsigned long long t0 = global_ns();
      while (!mbar_try_wait(&S.bar_final[g], 0) && global_ns() - t0 < args.wait_limit_ns) {
      }
      __syncwarp();
    }
  } else {
    // ---------------- epilogue: one thread per (atom, row type, stage) -------
    // Warp w reads TMEM lane quarter q = w % 4 of M-tile g = (w / 4) % 2 --
    // row type row_of_quarter(g, q) of atoms 32 g .. 32 g + 31 of the work
    // item -- in accumulator stage h = w / 8: the Golay tiles t = h, h + 2,
    // ....  The two warps of a row type thus work a tile apart, one loading
    // from TMEM while the other reduces, and each builds the half of the row's
    // flag mask that its tiles fill (bits of stage h: mask word h).
    const int q = warp & 3;
    const int g = (warp >> 2) % kMTiles;
    const int h = warp / kEpiPerStage;
    const int r = row_of_quarter(g, q);
    const int local = 32 * g + lane;
    const int slot = (g * 4 + q) * 32 + lane;
    const uint32_t t_row = tmem_base + (static_cast<uint32_t>(q * 32) << 16) +
                           static_cast<uint32_t>((g * kAccStages + h) * kGolayTileN);
    bool ok = true;
    int ip = 0;
    uint32_t rph = 0;  // bit i: parity of the next phase of bar_rows[g][i]
    for (int64_t it = blockIdx.x; ok && it < args.items; it += gridDim.x) {
      const int64_t atom = it * kWorkAtoms + local;
      // One warp per M-tile copies its 32 atoms' constants into shared memory
      // now; every warp reads them after the item's barrier, so no register
      // holds them across the tile loop and the copy has the whole item to land.
      const bool stager = q == 0 && h == 0;
      if (stager) {
#pragma unroll
        for (int k = 0; k < 3; ++k)
          cp_async16(reinterpret_cast<uint4 *>(&S.info_st[ip][g][lane]) + k,
                     reinterpret_cast<const uint4 *>(args.info + atom) + k);
        cp_async_commit();
      }
      float rowmax = -INFINITY;
      // Tile t holds columns 128 t .. 128 t + 127; the complements of its two
      // chunks form logical tile t + 16, where every score is negated.  Rows
      // 0-2 keep max |S| per chunk: one flag for a chunk and its complement.
      // The |x| row keeps minus the minimum (its complement chunk's maximum).
#pragma unroll 1
      for (int t = h; t < kScreenTiles; t += kAccStages) {
        if (!wait_bar_warp(&S.bar_acc_full[g][h], (t >> 1) & 1, abort_flag, args.err, args.wait_limit_ns)) {
          ok = false;
          break;
        }
        tc_fence_after();
        float m0 = -INFINITY, m1 = -INFINITY, m2 = -INFINITY, m3 = -INFINITY;
        if (r != 3 || t < kOctTiles) {
          // The tile's two 64-column halves, one TMEM load each.
          uint32_t x[64];
          tmem_ld64_wait(t_row, x);
          if (r == 3) {
            // The |x| row counts only at the weight-16 words, the complements
            // of the octad columns 1-759: minima over those alone.
            if (t == 0) x[0] = 0x7F800000u;  // zero word (its complement: all ones)
            m0 = -min32(INFINITY, x);
            m1 = -min32(INFINITY, x + 32);
          } else {
            m0 = max32abs(0.f, x);
            m1 = max32abs(0.f, x + 32);
          }
          tmem_ld64_wait(t_row + 64u, x);
          // Loaded: hand the stage back to the MMA issuer.
          tc_fence_before();
          __syncwarp();
          mbar_arrive_lane0(&S.bar_acc_empty[g][h], lane);
          if (r == 3) {
            if (t == kOctTiles - 1) {
#pragma unroll
              for (int j2 = kOctTailCol - 64; j2 < 64; ++j2) x[j2] = 0x7F800000u;  // dodecads
            }
            m2 = -min32(INFINITY, x);
            m3 = -min32(INFINITY, x + 32);
          } else {
            m2 = max32abs(0.f, x);
            m3 = max32abs(0.f, x + 32);
          }
        } else {
          tc_fence_before();
          __syncwarp();
          mbar_arrive_lane0(&S.bar_acc_empty[g][h], lane);
        }
        S.cmax[t][0][slot] = __halves2half2(__float2half_ru(m0), __float2half_ru(m1));
        S.cmax[t][1][slot] = __halves2half2(__float2half_ru(m2), __float2half_ru(m3));
        rowmax = fmaxf(rowmax, fmaxf(fmaxf(m0, m1), fmaxf(m2, m3)));
      }
      if (stager) cp_async_wait_all();  // the constants are in shared memory before the barrier
      if (!ok) break;
      // Row maxima of the atom's four rows (both stages), exchanged through
      // shared memory.
      S.rowval[ip][local][r][h] = rowmax;
      __syncwarp();
      mbar_arrive_lane0(&S.bar_rows[g][ip], lane);
      if (!wait_bar_warp(&S.bar_rows[g][ip], (rph >> ip) & 1u, abort_flag, args.err, args.wait_limit_ns)) {
        ok = false;
        break;
      }
      rph ^= 1u << ip;
      const AtomInfo inf = S.info_st[ip][g][lane];
      float rv[kRowsPerAtom];
#pragma unroll
      for (int k = 0; k < kRowsPerAtom; ++k) rv[k] = fmaxf(S.rowval[ip][local][k][0], S.rowval[ip][local][k][1]);
      const float best = fmaxf(fmaxf(fmaxf(rv[0] + inf.off[0], rv[1] + inf.off[1]),
                                     fmaxf(rv[3] + inf.shi - inf.l2s, inf.t1)),
                               inf.t2lb);
      const float thr = best - inf.two_e;
      const float add = r < 2 ? inf.off[r] : (r == 2 ? inf.add2 : inf.shi);
      // A chunk is flagged when (its fp16 maximum) + add >= thr in fp32.  In
      // fp16: maximum >= th with th <= thr - add, lowered by 2^-18 (|thr| +
      // |add|) against the fp32 roundings and rounded down to fp16, so every
      // chunk flagged in fp32 is flagged here (a few more may be).  th stays
      // finite so that chunks without columns (maximum -inf) stay unflagged.
      const float theta = (thr - add) - (fabsf(thr) + fabsf(add)) * 3.814697265625e-6f;
      const __half2 th2 = __half2half2(__float2half_rd(fmaxf(theta, -65504.f)));
      // Mask word h: bit 4 i + j holds sub-chunk j of tile 2 i + h (i = 0..7),
      // whose maxima this warp wrote.
      uint32_t wh = 0;
#pragma unroll
      for (int i = kScreenTiles / 2 - 1; i >= 0; --i) {
        const uint32_t f0 = __hge2_mask(S.cmax[2 * i + h][0][slot], th2);
        const uint32_t f1 = __hge2_mask(S.cmax[2 * i + h][1][slot], th2);
        wh = (wh << 4) | (f0 & 1u) | ((f0 >> 15) & 2u) | ((f1 << 2) & 4u) | ((f1 >> 13) & 8u);
      }
      if (!(inf.two_e >= 0.f)) wh = 0;
      if (atom < args.n) {
        reinterpret_cast<uint32_t *>(args.masks)[(atom * kRowsPerAtom + r) * 2 + h] = wh;
        if (r == 0 && h == 0) args.info[atom].thr = thr;
      }
      ip ^= 1;
    }
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == kIssuerWarp) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem_base),
                 "r"(kTmemCols)
                 : "memory");
  }
}


// ---------------------------------------------------------------------------
// 3. rescore (one warp per atom) and 4. exhaustive fallback
// ---------------------------------------------------------------------------
__device__ __forceinline__ double score64(const float (&x)[kDim], const int8_t *__restrict__ row) {
  const int2 w0 = __ldg(reinterpret_cast<const int2 *>(row));
  const int2 w1 = __ldg(reinterpret_cast<const int2 *>(row + 8));
  const int2 w2 = __ldg(reinterpret_cast<const int2 *>(row + 16));
  const uint32_t words[6] = {static_cast<uint32_t>(w0.x), static_cast<uint32_t>(w0.y),
                             static_cast<uint32_t>(w1.x), static_cast<uint32_t>(w1.y),
                             static_cast<uint32_t>(w2.x), static_cast<uint32_t>(w2.y)};
  double acc = 0.0;
#pragma unroll
  for (int i = 0; i < kDim; ++i) {
    const int raw = static_cast<int8_t>((words[i >> 2] >> (8 * (i & 3))) & 0xFF);
    const float kp = static_cast<float>(raw) * kLeechScaleF;
    acc = __fma_rn(static_cast<double>(x[i]), static_cast<double>(kp), acc);
  }
  return acc;
}

__device__ __forceinline__ void better(double &bs, int &bj, double s, int j) {
  if (s > bs || (s == bs && j < bj)) {
    bs = s;
    bj = j;
  }
}

__device__ __forceinline__ int32_t apply_rule(double best, int bj, int rule) {
  if (rule == H24_RULE_TRAIN && 2.0 * best < kCSqNorm) return 0;
  return bj + 1;
}

struct RescoreArgs {
  const uint4 *masks;        // [2n]: rows 0-1, rows 2-3 (64-bit chunk masks)
  const AtomInfo *info;      // [n], thr included
  const uint32_t *gmask;     // Golay masks
  const int32_t *idx3, *idx2, *idx1;
  const int8_t *cb_raw;
  int32_t *out;
  int32_t *ovf_list;
  int32_t *ovf_count;
  int64_t *stats;            // [0] exhaustive atoms, [1] exact scores, [2] flagged 32-column units
  int64_t n;
  int rule;
};

__device__ __forceinline__ float warp_max(float v) {
  float m;
  asm("redux.sync.max.f32 %0, %1, 0xffffffff;" : "=f"(m) : "f"(v));
  return m;
}

__device__ __forceinline__ float warp_min(float v) {
  float m;
  asm("redux.sync.min.f32 %0, %1, 0xffffffff;" : "=f"(m) : "f"(v));
  return m;
}

__device__ __forceinline__ uint32_t warp_or(uint32_t v) {
  uint32_t m;
  asm("redux.sync.or.b32 %0, %1, 0xffffffff;" : "=r"(m) : "r"(v));
  return m;
}

// What the rescore reads of one atom, staged in shared memory by cp.async one
// atom ahead of its use: eleven 16-byte chunks, chunk k copied by lane k.
struct AtomStage {
  float x[kDim];
  uint4 masks[2];
  AtomInfo info;
};
static_assert(sizeof(AtomStage) == 176 && offsetof(AtomStage, masks) == 96 &&
                  offsetof(AtomStage, info) == 128,
              "AtomStage is eleven 16-byte chunks: coordinates, masks, constants");


constexpr int kRescoreWarps = 8;
constexpr int kRescoreBlocksPerSm = 3;
constexpr int kCandCap = 128;  // fp32 candidates per atom before the fp64 pass

// A listed candidate is held as (type << 24) | its offset in that type's
// index table (idx3: 24 c + p, idx2: 128 o + sign pattern, idx1: 4 (24 a + b)
// + signs); the kissing-point index is looked up only for the candidates
// that reach the fp64 pass.
constexpr uint32_t kCandType3 = 3u << 24, kCandType2 = 2u << 24, kCandType1 = 1u << 24;
constexpr uint32_t kPendingIndex = 0x80000000u;  // output entry holding a candidate code
__device__ __forceinline__ int32_t cand_index(const int32_t *__restrict__ idx3,
                                              const int32_t *__restrict__ idx2,
                                              const int32_t *__restrict__ idx1, uint32_t code) {
  const uint32_t off = code & 0xFFFFFFu;
  const uint32_t type = code >> 24;
  return __ldg((type == 3 ? idx3 : (type == 2 ? idx2 : idx1)) + off);
}

// Running fp64 best of one lane over the candidates beyond the list's
// capacity (exact ties over many codewords), kept in shared memory; it holds
// atom `atom`'s values (it starts afresh on that atom's first overflow).
struct LaneBest {
  double s;
  int j;
  int n;  // fp64 scores taken
  int64_t atom;
};

// fp64 score of a listed candidate beyond the list's capacity: out of line.
__device__ __noinline__ void exact_now(const float (&x)[kDim], const int8_t *__restrict__ cb_raw,
                                       const int32_t *__restrict__ idx3, const int32_t *__restrict__ idx2,
                                       const int32_t *__restrict__ idx1, uint32_t code, LaneBest &lb,
                                       int64_t atom) {
  if (lb.atom != atom) {
    lb.atom = atom;
    lb.s = -INFINITY;
    lb.j = 0x7FFFFFFF;
    lb.n = 0;
  }
  const int32_t j = cand_index(idx3, idx2, idx1, code);
  better(lb.s, lb.j, score64(x, cb_raw + static_cast<int64_t>(j) * kDim), j);
  ++lb.n;
}

// Persistent: each warp takes atoms a = warp, warp + warps, ...; no block
// barrier inside the loop, so a slow atom holds up only its own warp.
//
// Pass 1 recomputes the screening score S' of every codeword behind the
// flagged sub-chunks in fp32 from the exact coordinates (sum_{i in c} x_i is
// four lookups in per-atom tables of the partial sums over each 6-bit group
// of the position mask) and lists those with S' >= thr = best - 2E.  Pass 2 scores
// in fp64, in the reference's order, the listed codewords within 2 e' of the
// largest S', e' = 2^-16 sum|x|, which bounds |S' - sqrt(8) R| with a wide
// margin; the winner and every codeword tied with it are among them.
template <typename In>
__global__ void __launch_bounds__(32 * kRescoreWarps, kRescoreBlocksPerSm)
    rescore_kernel(const __grid_constant__ Segs sg, const RescoreArgs r) {
  __shared__ __align__(16) float tab[kRescoreWarps][4][64];
  __shared__ float cand_s[kRescoreWarps][kCandCap];
  __shared__ uint32_t cand_c[kRescoreWarps][kCandCap];
  __shared__ int cand_n[kRescoreWarps];
  __shared__ AtomStage stage[kRescoreWarps][2];
  __shared__ LaneBest lbest[kRescoreWarps][32];
  extern __shared__ uint32_t gmask_s[];  // [kGolay] Golay masks, staged once per block
  const int lane = threadIdx.x & 31;
  const int w = threadIdx.x >> 5;
  for (int i = threadIdx.x; i < kGolay / 4; i += blockDim.x)
    reinterpret_cast<uint4 *>(gmask_s)[i] = __ldg(reinterpret_cast<const uint4 *>(r.gmask) + i);
  lbest[w][lane].atom = -1;
  __syncthreads();
  float(*T)[64] = tab[w];
  const int64_t nwarps = static_cast<int64_t>(gridDim.x) * kRescoreWarps;
  uint32_t st_exh = 0, st_exact = 0, st_chunks = 0;
  // Lanes 0-10 copy one 16-byte chunk each of atom a's stage (a bf16 atom
  // fills only the first three chunks of the coordinates, as bit patterns,
  // and is widened in place once it has landed).
  constexpr int kXChunks = atom_chunks<In>();
  // The atoms a warp visits only increase, so its segment is found by
  // advancing a cursor rather than by a search per atom.
  int seg = 0;
  // Lanes 6-7 copy chunk lane - 6 of the atom's masks (32 B per atom), lanes
  // 8-10 chunk lane - 8 of its constants (48 B per atom): address base +
  // a * stride.
  const uintptr_t pf_base = lane < 8 ? reinterpret_cast<uintptr_t>(r.masks) + 16 * (lane - 6)
                                     : reinterpret_cast<uintptr_t>(r.info) + 16 * (lane - 8);
  const uintptr_t pf_stride = lane < 8 ? 32 : sizeof(AtomInfo);
  const auto prefetch = [&](int64_t a, int s) {
    if (a < r.n) {
      while (seg + 1 < sg.count && sg.start[seg + 1] <= a) ++seg;
      const uint4 *src =
          lane < 6 ? reinterpret_cast<const uint4 *>(static_cast<const In *>(sg.x[seg]) + (a - sg.start[seg]) * kDim) +
                         lane
                   : reinterpret_cast<const uint4 *>(pf_base + static_cast<uintptr_t>(a) * pf_stride);
      if (lane < 11 && (lane < kXChunks || lane >= 6))
        cp_async16(reinterpret_cast<uint4 *>(&stage[w][s]) + lane, src);
    }
    cp_async_commit();
  };
  int sb = 0;
  prefetch(blockIdx.x * static_cast<int64_t>(kRescoreWarps) + w, 0);
  for (int64_t a = blockIdx.x * static_cast<int64_t>(kRescoreWarps) + w; a < r.n; a += nwarps, sb ^= 1) {
    // The other stage was last read by the previous atom: every lane is done
    // with it before the next atom's copies overwrite it.
    __syncwarp();
    prefetch(a + nwarps, sb ^ 1);
    cp_async_wait1();
    __syncwarp();
    const AtomStage &A = stage[w][sb];
    const float(&v)[kDim] = A.x;  // the atom, read from the stage when needed
    float xl;                     // lane i < 24: x_i; +0 on lanes 24-31
    if constexpr (sizeof(In) == 2) {
      // Widen the 24 bf16 patterns at the start of the coordinates in place.
      float *xs = stage[w][sb].x;
      const uint32_t h = lane < kDim ? reinterpret_cast<const uint16_t *>(xs)[lane] : 0u;
      __syncwarp();
      xl = bf16_bits_to_float(h);
      if (lane < kDim) xs[lane] = xl;
      __syncwarp();
    } else {
      xl = lane < kDim ? A.x[lane] : 0.f;
    }
    const int triv = A.info.triv;
    // Row r's 64-bit sub-chunk mask, read from the stage when its row is
    // processed.  A flag of rows 0-2 stands for 32 columns and their
    // complements: two 32-column units.
    const uint64_t *mrow = reinterpret_cast<const uint64_t *>(A.masks);
    const int nch = 2 * (__popcll(mrow[0]) + __popcll(mrow[1]) + __popcll(mrow[2])) + __popcll(mrow[3]);
    if (triv >= 0) {
      if (lane == 0) r.out[a] = triv;
      continue;
    }
    st_chunks += nch;
    bool heavy = nch > kHeavySubs;
    if (!heavy) {
      const float thr = A.info.thr;
      const AtomInfo inf = A.info;
      __syncwarp();  // the previous atom's table and list reads are done
      if (lane == 0) cand_n[w] = 0;
      LaneBest &lb = lbest[w][lane];
      // Partial-sum tables: T[k][s] = sum of x_{6k+i} over the bits i of s
      // (four tables of 64).  Lanes 8k .. 8k + 7 write table k, lane 8k + m
      // entries 8 m .. 8 m + 7 (two 16-byte stores): bits 3-5 of s are the
      // bits of m, bits 0-2 run over the eight entries.
      {
        const int k = lane >> 3, m = lane & 7;
        const float2 c01 = reinterpret_cast<const float2 *>(A.x)[3 * k];      // x_6k, x_6k+1
        const float2 c23 = reinterpret_cast<const float2 *>(A.x)[3 * k + 1];  // x_6k+2, x_6k+3
        const float2 c45 = reinterpret_cast<const float2 *>(A.x)[3 * k + 2];  // x_6k+4, x_6k+5
        float h3 = 0.f;
        if (m & 1) h3 += c23.y;
        if (m & 2) h3 += c45.x;
        if (m & 4) h3 += c45.y;
        const float s01 = c01.x + c01.y, s02 = c01.x + c23.x, s12 = c01.y + c23.x, s012 = s01 + c23.x;
        float4 *dst = reinterpret_cast<float4 *>(&T[k][8 * m]);
        dst[0] = make_float4(h3, h3 + c01.x, h3 + c01.y, h3 + s01);
        dst[1] = make_float4(h3 + c23.x, h3 + s02, h3 + s12, h3 + s012);
      }
      __syncwarp();
      // Sums over the coordinates, lane i holding x_i.
      const uint32_t negm = __ballot_sync(0xffffffffu, xl < 0.f);
      const auto tsum = [&](uint32_t m) {
        return T[0][m & 63] + T[1][(m >> 6) & 63] + T[2][(m >> 12) & 63] + T[3][m >> 18];
      };
      // Sum of x and of |x|, read from the tables.
      const float sumx = tsum(0xFFFFFFu);
      const float sumabs = sumx - 2.f * tsum(negm);
      const auto push = [&](float sc, uint32_t code) {
        const int k = atomicAdd(&cand_n[w], 1);
        if (k < kCandCap) {
          cand_s[w][k] = sc;
          cand_c[w][k] = code;
        } else {
          exact_now(v, r.cb_raw, r.idx3, r.idx2, r.idx1, code, lb, a);
        }
      };
      const int p1 = inf.p[0], p2 = inf.p[1], p3 = inf.p[2];
      // Type 3 at the slice positions p1, p2.  A flagged sub-chunk of rows
      // 0-2 stands for its columns c < 2048 and their complements c + 2048,
      // whose sums over the coordinates are sum(x) minus theirs: S(c + 2048)
      // = -S(c) for the plain scores.  Lane i takes column 32 u + i.
#pragma unroll 1
      for (int s = 0; s < 2; ++s) {
        uint64_t m = s ? mrow[1] : mrow[0];
        const int p = s ? p2 : p1;
        const float xp = __shfl_sync(0xffffffffu, xl, p);
        while (m) {
          const int c = sub_of_bit(__ffsll(m) - 1) * kSubCols + lane;
          m &= m - 1;
          const uint32_t gm = gmask_s[c];
          const float base = sumx - 2.f * tsum(gm);
          const bool in = (gm >> p & 1u) != 0;
          const float sc = base - xp * (in ? 2.f : 4.f);
          const float scc = -base - xp * (in ? 4.f : 2.f);
          if (sc >= thr || scc >= thr) {
            if (sc >= thr) push(sc, kCandType3 | static_cast<uint32_t>(c * kDim + p));
            if (scc >= thr) push(scc, kCandType3 | static_cast<uint32_t>((c + kGolayHalf) * kDim + p));
          }
        }
      }
      // Type 3 at the other positions, behind flagged sub-chunks of the plain row:
      // each column whose bound reaches thr is broadcast, and lane i < 24
      // scores position i.
      {
        uint64_t m = mrow[2];
        while (m) {
          const int c0 = sub_of_bit(__ffsll(m) - 1) * kSubCols;
          m &= m - 1;
          {
            const int c = c0 + lane;
            const uint32_t gm = gmask_s[c];
            const float bc = sumx - 2.f * tsum(gm);
            const bool in3 = (gm >> p3 & 1u) != 0;
            // Bit j < 32: column c of lane j; bit 32 + j: its complement.
            uint64_t bal = __ballot_sync(0xffffffffu, bc + (in3 ? inf.u1 : inf.u0) >= thr) |
                           static_cast<uint64_t>(__ballot_sync(0xffffffffu, -bc + (in3 ? inf.u0 : inf.u1) >= thr))
                               << 32;
            while (bal) {
              const int bit = __ffsll(bal) - 1;
              bal &= bal - 1;
              const int src = bit & 31;
              const bool comp = bit >= 32;
              const uint32_t gsrc = __shfl_sync(0xffffffffu, gm, src);
              const float bsrc = __shfl_sync(0xffffffffu, bc, src);
              const uint32_t gmc = comp ? ~gsrc & 0xFFFFFFu : gsrc;
              const float bcc = comp ? -bsrc : bsrc;
              const float sc = bcc - xl * ((gmc >> lane & 1u) ? 2.f : 4.f);
              const int col = c0 + src + (comp ? kGolayHalf : 0);
              if (lane < kDim && lane != p1 && lane != p2 && sc >= thr)
                push(sc, kCandType3 | static_cast<uint32_t>(col * kDim + lane));
            }
          }
        }
      }
      // Type 2, behind flagged sub-chunks of the |x| row.  For an octad O with
      // 2 T(O) >= thr, the lanes holding its coordinates give, by warp
      // reductions, the parity of its negative coordinates, its smallest and
      // second smallest |x_i| (m1, m2) and the signs of its best even-parity
      // pattern, of score 2 T(O) - 4 [odd] m1.  Every other pattern of O
      // scores at least 4 (m2 - m1) (odd) or 4 (m1 + m2) (even) less; when
      // that gap is clear of fp64 rounding those patterns can neither win nor
      // tie, and only the best one is listed; else all 128 are scored.
      {
        const float tie_gap = 9.094947e-13f * sumabs;  // 2^-40 sum|x|
        uint64_t m = mrow[3];
        while (m) {
          // Lane i: the complement (a weight-16 word) of column 32 u + i.
          const int c = kGolayHalf + sub_of_bit(__ffsll(m) - 1) * kSubCols + lane;
          m &= m - 1;
          {
            const int o = c - kW16First;
            uint32_t om = 0;
            float t2 = -INFINITY;
            bool oddl = false;  // odd number of negative coordinates in lane's octad
            if (o >= 0 && o < kOctads) {
              const uint32_t gm = gmask_s[c];
              om = ~gm & 0xFFFFFFu;
              t2 = 2.f * (sumabs - (tsum(gm & ~negm) - tsum(gm & negm)));  // 2 T(O)
              oddl = (__popc(om & negm) & 1u) != 0;
            }
            uint32_t bal = __ballot_sync(0xffffffffu, t2 >= thr);
            while (bal) {
              const int src = __ffs(bal) - 1;
              bal &= bal - 1;
              const int oc = c - lane + src - kW16First;  // the octad of lane src's column
              const uint32_t omc = __shfl_sync(0xffffffffu, om, src);
              const float t2c = __shfl_sync(0xffffffffu, t2, src);
              const bool odd = __shfl_sync(0xffffffffu, oddl ? 1 : 0, src) != 0;
              // Lane i < 24 holds x_i; omc has 24 bits, so in_o is false on
              // lanes 24-31.
              const bool in_o = (omc >> lane & 1u) != 0;
              const float ax = in_o ? fabsf(xl) : INFINITY;
              const float m1 = warp_min(ax);
              const float t2x = odd ? t2c - 4.f * m1 : t2c;
              if (t2x < thr) continue;
              // Even parity: the other patterns score at least 4 (m1 + m2) >=
              // 8 m1 less, so the second smallest |x_i| is needed only when
              // 8 m1 does not clear the gap.
              int kmin = 0;
              bool clear = true;
              if (odd || !(8.f * m1 > tie_gap)) {
                kmin = __ffs(__ballot_sync(0xffffffffu, ax == m1)) - 1;  // lowest on ties
                const float m2 = warp_min(lane == kmin ? INFINITY : ax);
                clear = (odd ? 4.f * (m2 - m1) : 4.f * (m1 + m2)) > tie_gap;
              }
              if (clear) {
                // Pattern bit k (k < 7): the coordinate of rank k in O (rank
                // 0 = lowest position) is negative; rank 7 follows from parity.
                const uint32_t rank = __popc(omc & ((1u << lane) - 1u));
                uint32_t pid = warp_or(in_o && xl < 0.f ? 1u << rank : 0u);
                if (odd) pid ^= 1u << __popc(omc & ((1u << kmin) - 1u));
                if (lane == 0) push(t2x, kCandType2 | static_cast<uint32_t>(oc * 128 + (pid & 0x7Fu)));
                continue;
              }
              // Exact ties within O: every sign pattern, across the warp.
              float o8[8];
              uint32_t mo = omc;
#pragma unroll
              for (int k2 = 0; k2 < 8; ++k2) {
                o8[k2] = __shfl_sync(0xffffffffu, xl, (__ffs(mo) - 1) & 31);
                mo &= mo - 1;
              }
#pragma unroll
              for (int t = 0; t < 4; ++t) {
                const int pid = lane + 32 * t;
                float sc = (__popc(pid) & 1) ? -o8[7] : o8[7];
#pragma unroll
                for (int k2 = 0; k2 < 7; ++k2) sc += (pid >> k2 & 1) ? -o8[k2] : o8[k2];
                if (2.f * sc >= thr) push(2.f * sc, kCandType2 | static_cast<uint32_t>(oc * 128 + pid));
              }
            }
          }
        }
      }
      // Type 1: every score is at most t1.
      if (inf.t1 >= thr && lane < kDim) {
        const float xa = A.x[lane];
#pragma unroll 1
        for (int b2 = lane + 1; b2 < kDim; ++b2) {
          const float xb = A.x[b2];
#pragma unroll
          for (int s = 0; s < 4; ++s) {
            const float sc = 4.f * ((s & 1 ? -xa : xa) + (s & 2 ? -xb : xb));
            if (sc >= thr) push(sc, kCandType1 | static_cast<uint32_t>((lane * kDim + b2) * 4 + s));
          }
        }
      }
      __syncwarp();
      const float two_ep = 3.0517578125e-5f * sumabs;  // 2 e'
      if (cand_n[w] == 1) {
        // One listed codeword (the usual case): the unique winner, unless the
        // training rule's origin test is too close to call in fp32 (below).
        const float og = cand_s[w][0] * 0.70710678f - static_cast<float>(kCSqNorm);
        if (r.rule != H24_RULE_TRAIN || fabsf(og) > two_ep) {
          if (lane == 0)
            r.out[a] = (r.rule == H24_RULE_TRAIN && og < 0.f)
                           ? 0
                           : static_cast<int32_t>(kPendingIndex | cand_c[w][0]);
          continue;
        }
      }
      const int nc = min(cand_n[w], kCandCap);
      heavy = cand_n[w] == 0;  // cannot happen while the bound holds
      if (!heavy) {
        float smax = -INFINITY;
        for (int k = lane; k < nc; k += 32) smax = fmaxf(smax, cand_s[w][k]);
        smax = warp_max(smax);
        const float cut = smax - two_ep;
        int nin = 0, jin = 0;
        for (int k = lane; k < nc; k += 32) {
          if (cand_s[w][k] >= cut) {
            ++nin;
            jin = static_cast<int>(cand_c[w][k]);
          }
        }
        // One codeword within 2 e' of the largest S' (and no list overflow):
        // it is the unique winner.  The training rule's origin test
        // 2 R < c_sq_norm, with sqrt(8) R within e' of S', is decided from
        // S' unless S' / sqrt(2) lies within 2 e' of c_sq_norm.
        const uint32_t who = __ballot_sync(0xffffffffu, nin > 0);
        const int src = (__ffs(who) - 1) & 31;
        const int nsrc = __shfl_sync(0xffffffffu, nin, src);
        const int jsrc = __shfl_sync(0xffffffffu, jin, src);
        const float origin_gap = smax * 0.70710678f - static_cast<float>(kCSqNorm);
        const bool quick = __popc(who) == 1 && nsrc == 1 && cand_n[w] <= kCandCap &&
                           (r.rule != H24_RULE_TRAIN || fabsf(origin_gap) > two_ep);
        if (quick) {
          // The winner's kissing-point index is looked up by decode_kernel.
          if (lane == 0)
            r.out[a] = (r.rule == H24_RULE_TRAIN && origin_gap < 0.f)
                           ? 0
                           : static_cast<int32_t>(kPendingIndex | static_cast<uint32_t>(jsrc));
        } else {
          const bool own = lb.atom == a;  // this lane's list overflowed for this atom
          double bs = own ? lb.s : -INFINITY;
          int bj = own ? lb.j : 0x7FFFFFFF, nex = own ? lb.n : 0;
          for (int k = lane; k < nc; k += 32) {
            if (cand_s[w][k] >= cut) {
              const int j = cand_index(r.idx3, r.idx2, r.idx1, cand_c[w][k]);
              better(bs, bj, score64(v, r.cb_raw + static_cast<int64_t>(j) * kDim), j);
              ++nex;
            }
          }
#pragma unroll
          for (int off = 16; off > 0; off >>= 1) {
            const double os = __shfl_xor_sync(0xffffffffu, bs, off);
            const int oj = __shfl_xor_sync(0xffffffffu, bj, off);
            better(bs, bj, os, oj);
            nex += __shfl_xor_sync(0xffffffffu, nex, off);
          }
          st_exact += nex;
          if (lane == 0) r.out[a] = apply_rule(bs, bj, r.rule);
        }
      }
    }
    if (heavy && lane == 0) {
      // Too many candidates (exact ties over many codewords): the exhaustive
      // scan.  Certain origin under the training rule instead when every
      // score is at most 2 ||x|| (Cauchy-Schwarz, ||kp|| = 2) < c_sq_norm / 2.
      double ss = 0.0;
#pragma unroll
      for (int i = 0; i < kDim; ++i)
        ss = __fma_rn(static_cast<double>(v[i]), static_cast<double>(v[i]), ss);
      r.out[a] = 0;
      if (!(r.rule == H24_RULE_TRAIN && 4.0 * sqrt(ss) * (1.0 + 1e-6) < kCSqNorm)) {
        r.ovf_list[atomicAdd(r.ovf_count, 1)] = static_cast<int32_t>(a);
        ++st_exh;
      }
    }
  }
  if (lane == 0) {
    if (st_exh) atomicAdd(reinterpret_cast<unsigned long long *>(&r.stats[0]), static_cast<unsigned long long>(st_exh));
    if (st_exact) atomicAdd(reinterpret_cast<unsigned long long *>(&r.stats[1]), static_cast<unsigned long long>(st_exact));
    if (st_chunks) atomicAdd(reinterpret_cast<unsigned long long *>(&r.stats[2]), static_cast<unsigned long long>(st_chunks));
  }
}

template <typename T>
__global__ void __launch_bounds__(256) exhaustive_kernel(const __grid_constant__ Segs sg, int rule,
                                                         const int32_t *__restrict__ ovf_list,
                                                         const int32_t *__restrict__ ovf_count,
                                                         const int8_t *__restrict__ cb_raw,
                                                         int32_t *__restrict__ out) {
  __shared__ double ws[8];
  __shared__ int wj[8];
  pdl_enter();
  const int count = *ovf_count;
  for (int e = blockIdx.x; e < count; e += gridDim.x) {
    const int64_t a = ovf_list[e];
    float v[kDim];
    load_atom_t<T, false>(atom_ptr<T>(sg, a), v);
    double bs = -INFINITY;
    int bj = 0x7FFFFFFF;
    for (int j = threadIdx.x; j < kKissing; j += blockDim.x)
      better(bs, bj, score64(v, cb_raw + static_cast<int64_t>(j) * kDim), j);
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) {
      const double os = __shfl_xor_sync(0xffffffffu, bs, off);
      const int oj = __shfl_xor_sync(0xffffffffu, bj, off);
      better(bs, bj, os, oj);
    }
    if ((threadIdx.x & 31) == 0) {
      ws[threadIdx.x >> 5] = bs;
      wj[threadIdx.x >> 5] = bj;
    }
    __syncthreads();
    if (threadIdx.x == 0) {
      for (int w = 1; w < 8; ++w) better(bs, bj, ws[w], wj[w]);
      out[a] = apply_rule(bs, bj, rule);
    }
    __syncthreads();
  }
}

// Replaces every pending output entry of the rescore (bit 31 set: the code of
// the winning listed candidate) by its kissing-point index + 1.
__global__ void __launch_bounds__(256) decode_kernel(int32_t *__restrict__ out, int64_t n,
                                                     const int32_t *__restrict__ idx3,
                                                     const int32_t *__restrict__ idx2,
                                                     const int32_t *__restrict__ idx1) {
  pdl_enter();
  for (int64_t a = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; a < n;
       a += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const uint32_t v = static_cast<uint32_t>(out[a]);
    if (v & kPendingIndex) out[a] = cand_index(idx3, idx2, idx1, v & ~kPendingIndex) + 1;
  }
}

std::mutex g_mu;
int g_sms[64] = {};


// Per-atom scratch of one pipeline batch of up to `pad` atoms.
struct Scratch {
  uint8_t *a_tiles;
  AtomInfo *info;
  uint2 *masks;
  int32_t *ovf_list;
  int32_t *ovf_count;
};
constexpr size_t up256(size_t v) { return (v + 255) & ~static_cast<size_t>(255); }
constexpr size_t scratch_bytes(int64_t pad) {
  return up256(static_cast<size_t>(pad) / kWorkAtoms * kAItemBytes) +
         up256(static_cast<size_t>(pad) * sizeof(AtomInfo)) +
         up256(static_cast<size_t>(pad) * kRowsPerAtom * 8) + up256(static_cast<size_t>(pad) * 4) + 256;
}
Scratch carve(uint8_t *base, int64_t pad) {
  Scratch sc;
  size_t o = 0;
  sc.a_tiles = base + o;
  o += up256(static_cast<size_t>(pad) / kWorkAtoms * kAItemBytes);
  sc.info = reinterpret_cast<AtomInfo *>(base + o);
  o += up256(static_cast<size_t>(pad) * sizeof(AtomInfo));
  sc.masks = reinterpret_cast<uint2 *>(base + o);
  o += up256(static_cast<size_t>(pad) * kRowsPerAtom * 8);
  sc.ovf_list = reinterpret_cast<int32_t *>(base + o);
  o += up256(static_cast<size_t>(pad) * 4);
  sc.ovf_count = reinterpret_cast<int32_t *>(base + o);
  return sc;
}

// The five kernels of one batch (prep also empties the exhaustive-scan list).
// Prep, the exhaustive scan and decode use programmatic dependent launch
// (pdl_enter): each waits for its predecessor before touching memory.
template <typename T>
int launch_batch_t(const Tables *t, const Segs &sg, int64_t nbatch, int rule, int32_t *ob,
                   const Scratch &sc, int sms, cudaStream_t s) {
  const int64_t items = (nbatch + kWorkAtoms - 1) / kWorkAtoms;
  const int64_t npad = items * kWorkAtoms;
  // Optional instrumentation: events around the prep, screen and rescore.
  const bool timed = timing_enabled();
  cudaEvent_t ev[6] = {};
  if (timed)
    for (auto &e : ev) cudaEventCreate(&e);
  if (timed) cudaEventRecord(ev[0], s);
  H24_CUDA_TRY(launch_pdl(prep_kernel<T>, dim3(static_cast<unsigned>((npad + 255) / 256)), dim3(256), s, sg,
                          nbatch, npad, rule, t->oct_by_triple, sc.a_tiles, sc.info, sc.ovf_count));
  if (timed) cudaEventRecord(ev[1], s);
  ScreenArgs sa{sc.a_tiles, sc.info, reinterpret_cast<const uint8_t *>(t->golay_tiled), sc.masks,
                nbatch, items, t->err, kWaitLimitNs};
  const int grid = static_cast<int>(items < sms ? items : sms);
  if (timed) cudaEventRecord(ev[2], s);
  screen_kernel<<<grid, kScreenThreads, sizeof(ScreenSmem) + 1024, s>>>(sa);
  if (timed) cudaEventRecord(ev[3], s);
  RescoreArgs ra{reinterpret_cast<const uint4 *>(sc.masks), sc.info, t->golay_mask, t->idx3,
                 t->idx2, t->idx1, t->cb_raw, ob, sc.ovf_list, sc.ovf_count, t->stats, nbatch,
                 rule};
  const int64_t rblocks = (nbatch + kRescoreWarps - 1) / kRescoreWarps;
  const int64_t rcap = static_cast<int64_t>(sms) * kRescoreBlocksPerSm;
  if (timed) cudaEventRecord(ev[4], s);
  rescore_kernel<T><<<static_cast<unsigned>(rblocks < rcap ? rblocks : rcap), 32 * kRescoreWarps,
                      kGolay * sizeof(uint32_t), s>>>(sg, ra);
  if (timed) {
    cudaEventRecord(ev[5], s);
    timing_record(H24_KERNEL_PREP, ev[0], ev[1]);
    timing_record(H24_KERNEL_SCREEN, ev[2], ev[3]);
    timing_record(H24_KERNEL_RESCORE, ev[4], ev[5]);
  }
  H24_CUDA_TRY(launch_pdl(exhaustive_kernel<T>, dim3(2 * sms), dim3(256), s, sg, rule,
                          static_cast<const int32_t *>(sc.ovf_list), static_cast<const int32_t *>(sc.ovf_count),
                          static_cast<const int8_t *>(t->cb_raw), ob));
  const int64_t dblocks = (nbatch + 255) / 256;
  H24_CUDA_TRY(launch_pdl(decode_kernel, dim3(static_cast<unsigned>(dblocks < 8 * sms ? dblocks : 8 * sms)),
                          dim3(256), s, ob, nbatch, t->idx3, t->idx2, t->idx1));
  count_launches(5);
  H24_CUDA_TRY(cudaGetLastError());
  return H24_OK;
}

int launch_batch(const Tables *t, const Segs &sg, int64_t nbatch, int dtype, int rule, int32_t *ob,
                 const Scratch &sc, int sms, cudaStream_t s) {
  return dtype == H24_DTYPE_BF16 ? launch_batch_t<__nv_bfloat16>(t, sg, nbatch, rule, ob, sc, sms, s)
                                 : launch_batch_t<float>(t, sg, nbatch, rule, ob, sc, sms, s);
}

int screen_setup(int dev, int *sms) {
  std::lock_guard<std::mutex> lk(g_mu);
  if (g_sms[dev] == 0) {
    int count = 0;
    H24_CUDA_TRY(cudaDeviceGetAttribute(&count, cudaDevAttrMultiProcessorCount, dev));
    H24_CUDA_TRY(cudaFuncSetAttribute(screen_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                      static_cast<int>(sizeof(ScreenSmem) + 1024)));
    H24_CUDA_TRY(cudaFuncSetAttribute(rescore_kernel<float>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                      static_cast<int>(kGolay * sizeof(uint32_t))));
    H24_CUDA_TRY(cudaFuncSetAttribute(rescore_kernel<__nv_bfloat16>,
                                      cudaFuncAttributeMaxDynamicSharedMemorySize,
                                      static_cast<int>(kGolay * sizeof(uint32_t))));
    // Launch sizes against what each kernel's resources allow.
    const struct { const void *fn; int threads; const char *name; } ks[] = {
        {reinterpret_cast<const void *>(screen_kernel), kScreenThreads, "screen_kernel"},
        {reinterpret_cast<const void *>(rescore_kernel<float>), 32 * kRescoreWarps, "rescore_kernel"},
        {reinterpret_cast<const void *>(rescore_kernel<__nv_bfloat16>), 32 * kRescoreWarps,
         "rescore_kernel(bf16)"},
        {reinterpret_cast<const void *>(prep_kernel<float>), 256, "prep_kernel"},
        {reinterpret_cast<const void *>(prep_kernel<__nv_bfloat16>), 256, "prep_kernel(bf16)"},
        {reinterpret_cast<const void *>(exhaustive_kernel<float>), 256, "exhaustive_kernel"},
        {reinterpret_cast<const void *>(exhaustive_kernel<__nv_bfloat16>), 256, "exhaustive_kernel(bf16)"},
        {reinterpret_cast<const void *>(decode_kernel), 256, "decode_kernel"}};
    for (const auto &k : ks) {
      cudaFuncAttributes at;
      H24_CUDA_TRY(cudaFuncGetAttributes(&at, k.fn));
      if (at.maxThreadsPerBlock < k.threads)
        return fail(H24_ERR_STATE, std::string(k.name) + ": " + std::to_string(at.numRegs) +
                                       " registers allow " + std::to_string(at.maxThreadsPerBlock) +
                                       " threads per block, launch needs " + std::to_string(k.threads));
    }
    g_sms[dev] = count;
  }
  *sms = g_sms[dev];
  return H24_OK;
}

}  // namespace

int quantize_segments(const Tables *t, const void *const *xs, const int64_t *counts, int nseg,
                      int dtype, int rule, int32_t *out_idx, cudaStream_t s) {
  if (dtype != H24_DTYPE_F32 && dtype != H24_DTYPE_BF16)
    return fail(H24_ERR_INVALID, "quantize: atoms must be fp32 or bf16");
  const size_t esize = dtype == H24_DTYPE_BF16 ? 2 : 4;
  int64_t total = 0;
  for (int i = 0; i < nseg; ++i) {
    if (counts[i] < 0) return fail(H24_ERR_INVALID, "quantize: negative segment length");
    if (counts[i] > 0 && (!xs[i] || !aligned16(xs[i])))
      return fail(H24_ERR_INVALID, "quantize: segment pointers must be non-null and 16-byte aligned");
    total += counts[i];
  }
  if (total == 0) return H24_OK;
  int sms = 0;
  int rc = screen_setup(t->device, &sms);
  if (rc != H24_OK) return rc;

  const int64_t batch = total < kBatchAtoms ? total : kBatchAtoms;
  const int64_t pad_max = (batch + kWorkAtoms - 1) / kWorkAtoms * kWorkAtoms;
  uint8_t *scratch = nullptr;
  H24_CUDA_TRY(cudaMallocFromPoolAsync(reinterpret_cast<void **>(&scratch), scratch_bytes(pad_max),
                                       t->pool, s));
  const Scratch sc = carve(scratch, pad_max);
  int seg = 0;
  int64_t seg_off = 0;  // atoms of segment `seg` already consumed
  int64_t done = 0;
  while (done < total && rc == H24_OK) {
    // Collect up to kMaxSegs (pieces of) segments, at most `batch` atoms.
    Segs sg;
    sg.count = 0;
    sg.start[0] = 0;
    int64_t nbatch = 0;
    while (seg < nseg && sg.count < kMaxSegs && nbatch < batch) {
      const int64_t avail = counts[seg] - seg_off;
      if (avail <= 0) { ++seg; seg_off = 0; continue; }
      const int64_t take = avail < batch - nbatch ? avail : batch - nbatch;
      sg.x[sg.count] = static_cast<const uint8_t *>(xs[seg]) + static_cast<size_t>(seg_off) * kDim * esize;
      nbatch += take;
      sg.start[++sg.count] = nbatch;
      seg_off += take;
      if (seg_off == counts[seg]) { ++seg; seg_off = 0; }
    }
    rc = launch_batch(t, sg, nbatch, dtype, rule, out_idx + done, sc, sms, s);
    done += nbatch;
  }
  cudaError_t e = cudaFreeAsync(scratch, s);
  if (rc == H24_OK && e != cudaSuccess) rc = cuda_fail(e, "cudaFreeAsync");
  return rc;
}

int quantize(const Tables *t, const float *x, int64_t n, int rule, int32_t *out_idx,
             cudaStream_t s) {
  const void *xv = x;
  return quantize_segments(t, &xv, &n, 1, H24_DTYPE_F32, rule, out_idx, s);
}

// ===========================================================================
// Allocation-free variant of the nearest-codeword pipeline.
//
// Some callers must not allocate device memory at call time: code running
// under an external memory manager that owns every device allocation (a
// framework's caching allocator or a serving runtime with a fixed memory
// budget), or latency-critical loops where an allocation call would stall or
// fragment memory.  For them h24_quantize_noalloc runs the same kernels with
// all per-call scratch in one file-scope device array of fixed size, so it
// calls no cudaMalloc, cudaMallocAsync, cudaFree or other allocating routine.
//
// Limits and rules:
//   * at most kNoAllocMaxAtoms atoms per call (larger calls are rejected);
//   * the codebook tables must already be resident: call h24_init(device)
//     (or any other h24 entry point) once at set-up, because building them
//     allocates; this entry point returns H24_ERR_STATE otherwise;
//   * the first call on a device resolves the array's device address with
//     cudaGetSymbolAddress (set-up work, no allocation); make that first call
//     before any stream capture;
//   * every call on a device shares the one array and it keeps the previous
//     call's contents: the counter that must start at zero is cleared at
//     the start of each call, everything else is written before it is read.
//     Calls whose executions overlap on the GPU (other streams or host
//     threads without ordering) race on the array.
// ===========================================================================
namespace {

constexpr int64_t kNoAllocMaxAtoms = 32768;
constexpr size_t kNoAllocBytes = scratch_bytes(kNoAllocMaxAtoms);  // 11,141,376 B, about 10.6 MiB
static_assert(kNoAllocMaxAtoms % kWorkAtoms == 0, "whole CTA work items");
static_assert(kNoAllocBytes < (size_t(16) << 20), "modest fixed footprint");

// The scratch array.  In host code this name is a host-side stand-in, not a
// device address: host code must use the address from cudaGetSymbolAddress.
static __device__ __align__(256) uint8_t g_noalloc_scratch[kNoAllocBytes];

std::mutex g_noalloc_mu;
uint8_t *g_noalloc_ptr[64] = {};

// Per-device set-up: resolve the array's device address (once, with the device
// current) and allow the screening kernel its dynamic shared memory.
int noalloc_setup(int dev, uint8_t **out, int *sms) {
  int rc = screen_setup(dev, sms);
  if (rc != H24_OK) return rc;
  std::lock_guard<std::mutex> lk(g_noalloc_mu);
  if (!g_noalloc_ptr[dev]) {
    void *ptr = nullptr;
    cudaError_t e = cudaGetSymbolAddress(&ptr, g_noalloc_scratch);
    if (e != cudaSuccess) return cuda_fail(e, "cudaGetSymbolAddress(noalloc scratch)");
    g_noalloc_ptr[dev] = static_cast<uint8_t *>(ptr);
  }
  *out = g_noalloc_ptr[dev];
  return H24_OK;
}

int quantize_noalloc(const Tables *t, const float *x, int64_t n, int rule, int32_t *out_idx,
                     cudaStream_t s) {
  uint8_t *scratch = nullptr;
  int sms = 0;
  int rc = noalloc_setup(t->device, &scratch, &sms);
  if (rc != H24_OK) return rc;
  Segs sg;
  sg.count = 1;
  sg.x[0] = x;
  sg.start[0] = 0;
  sg.start[1] = n;
  const Scratch sc = carve(scratch, kNoAllocMaxAtoms);
  // The array keeps the previous call's contents; prep clears the overflow
  // counter.
  return launch_batch(t, sg, n, H24_DTYPE_F32, rule, out_idx, sc, sms, s);
}

}  // namespace
}  // namespace h24

extern "C" int h24_quantize_noalloc(const float *x, int64_t n, int rule, int32_t *out_idx,
                                    void *stream) {
  using namespace h24;
  if (n < 0) return fail(H24_ERR_INVALID, "quantize_noalloc: negative atom count");
  if (n > kNoAllocMaxAtoms)
    return fail(H24_ERR_INVALID, "quantize_noalloc: " + std::to_string(n) +
                                     " atoms exceed the allocation-free limit of " +
                                     std::to_string(kNoAllocMaxAtoms) + " atoms per call");
  if (rule != H24_RULE_TRAIN && rule != H24_RULE_PACK)
    return fail(H24_ERR_INVALID, "quantize_noalloc: unknown rule");
  if (n == 0) return H24_OK;
  if (!x || !out_idx) return fail(H24_ERR_INVALID, "quantize_noalloc: null pointer");
  if (!aligned16(x)) return fail(H24_ERR_INVALID, "quantize_noalloc: x must be 16-byte aligned");
  const Tables *t = tables_if_ready();
  if (!t)
    return fail(H24_ERR_STATE,
                "quantize_noalloc: codebook tables are not resident on this device; call "
                "h24_init(device) once at set-up (it allocates them)");
  return quantize_noalloc(t, x, n, rule, out_idx, static_cast<cudaStream_t>(stream));
}
