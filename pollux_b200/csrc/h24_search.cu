// h24_search.cu -- nearest-codeword search over the 196,560 H24 kissing points
// (castor._leech_nn_kernel, castor.py:386-462; castor_quantize_leech,
// castor.py:487-560; the search of pack._quantize_h24_layer, pack.py:166-177).
//
// Result semantics: index = argmax_j fp64(x . kp_j) + 1 with the lowest j on
// ties, where fp64(x . kp_j) accumulates fma(x_i, kp_ji) for i = 0..23 in
// order, kp_ji = fp32(raw_ji * fp32(1/sqrt(8))) as stored by the reference,
// followed by the caller's origin rule (H24_RULE_TRAIN / H24_RULE_PACK).
//
// Pipeline per batch of atoms (one CUDA stream, no host synchronisation):
//   1. prep_kernel      x -> bf16 "hi" rows (24 values + 8 zeros) and a
//                       per-atom bound 2E on |screening score - exact score|.
//   2. screen_kernel    persistent tcgen05 kernel, one CTA per SM.  Each CTA
//                       owns 256 atoms (two M=128 tiles) at a time; their bf16
//                       rows live in tensor memory (A operand), written by the
//                       epilogue warps with tcgen05.st.  The bf16 codebook (raw
//                       integers, exact in bf16, K padded 24 -> 32) streams
//                       through a shared-memory ring by bulk copies, 112
//                       codewords per stage, so the MMAs read only B from shared
//                       memory.  Scores accumulate in TMEM (fp32), double
//                       buffered; 16 epilogue warps read them with tcgen05.ld,
//                       one thread per (atom, 56-codeword chunk parity), and
//                       keep the chunks whose maximum is within 2E of the
//                       running best.
//   3. rescore_kernel   one warp per atom rescans the surviving chunks in fp64
//                       and applies the origin rule.
//   4. exhaustive_kernel  fp64 scan of all codewords for the rare atoms whose
//                       candidate bookkeeping overflowed.
//
// Why the bound is sufficient: with S~ the screening score and R the exact
// score (in raw-integer units), |S~_j - R_j| <= E for every j.  If j* is the
// exact winner and B~ the screening maximum, S~_j* >= R_j* - E >= R_jhat - E
// >= B~ - 2E.  Every chunk whose screening maximum is >= B~ - 2E is kept.
#include <cstdio>
#include <mutex>

#include "h24_internal.cuh"

namespace h24 {
namespace {

constexpr int kBlockAtoms = 256;                    // atoms per CTA work item
constexpr int kStages = 16;                         // codebook ring depth
constexpr int kAccStages = 2;                       // TMEM accumulator stages
constexpr int kBTileBytes = kTileN * kRowBytes;     // 7680
constexpr int kHiBytes = kRowBytes;                 // bf16 row of one atom in global memory
constexpr int kCap = 12;                            // candidate chunks per (atom, half) list
constexpr int kBitmapWords = (kNumChunks + 31) / 32;  // 103 words: one bit per chunk
constexpr int kMaxSegs = 64;                        // input segments per pipeline batch
constexpr int kEpiWarps = 16;                        // 2 M-tiles x 4 lane quarters x 2 halves
constexpr int kLists = 2 * kBlockAtoms;               // one list per (atom, column half)
constexpr int kTileWarps = 8;                        // epilogue warps reading one M-tile
constexpr int kFirstEpiWarp = 3;                      // warp 0 producer, warps 1-2 MMA issuers
constexpr int kScreenThreads = 32 * (kFirstEpiWarp + kEpiWarps);  // 608
constexpr uint32_t kTmemCols = 512;
// TMEM columns: accumulator stage s, M-tile h at s*2*kTileN + h*kTileN; the
// A operand of M-tile h at kAColBase + h*kACols.
constexpr uint32_t kACols = kKPad / 2;                // 16 columns: 32 bf16 per lane
constexpr uint32_t kAColBase = kAccStages * 2 * kTileN;  // 480
static_assert(kAColBase + 2 * kACols == kTmemCols, "accumulators + A operand fill TMEM");
constexpr uint8_t kOverflow = 0xFF;   // exhaustive fp64 scan
constexpr uint8_t kBitmapMode = 0xFE; // candidate chunks in a global bitmap slot
constexpr int64_t kBatchAtoms = int64_t(1) << 22;    // atoms per pipeline batch
constexpr unsigned long long kWaitLimitNs = 4000000000ull;  // bounded waits: 4 s

struct __align__(1024) ScreenSmem {
  uint8_t b[kStages][kBTileBytes];
  float cand_score[kCap][kLists];
  uint16_t cand_chunk[kCap][kLists];
  uint64_t bar_b_full[kStages];
  uint64_t bar_b_empty[kStages];
  uint64_t bar_a_full[2][2];              // [A buffer][M-tile]
  uint64_t bar_acc_full[kAccStages][2];   // [stage][M-tile]
  uint64_t bar_acc_empty[kAccStages][2];
  uint64_t bar_final[2];
  uint32_t tmem_base;
  int abort_flag;
};

// ---------------------------------------------------------------------------
// PTX helpers
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint32_t smem_u32(const void *p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t *bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}

__device__ __forceinline__ void mbar_arrive(uint64_t *bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t *bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
               "r"(bytes)
               : "memory");
}

// Suspend-time hint (ns) of the mbarrier waits: a waiting thread sleeps until
// the phase completes or the hint expires instead of spinning.  0 = no hint.
#ifndef H24_WAIT_HINT_NS
#define H24_WAIT_HINT_NS 1000000
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

// Slow path of wait_bar.  Gives up after kWaitLimitNs or when another role of
// the CTA has aborted; on a timeout it raises the CTA abort flag and the
// device error word.
__device__ __noinline__ bool wait_slow(uint64_t *bar, uint32_t parity, volatile int *abort_flag,
                                       int *err) {
  const unsigned long long t0 = global_ns();
  for (;;) {
    if (mbar_try_wait(bar, parity)) return true;
    if (*abort_flag) return false;
    if (global_ns() - t0 > kWaitLimitNs) {
      *abort_flag = 1;
      atomicExch(err, H24_ERR_TIMEOUT);
      return false;
    }
  }
}

// Waits for the phase of `bar` with the given parity (inline fast path).
__device__ __forceinline__ bool wait_bar(uint64_t *bar, uint32_t parity, volatile int *abort_flag,
                                         int *err) {
  if (mbar_test(bar, parity)) return true;
  return wait_slow(bar, parity, abort_flag, err);
}

__device__ __forceinline__ void bulk_g2s(void *dst, const void *src, uint32_t bytes, uint64_t *bar,
                                         uint64_t policy) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint "
      "[%0], [%1], %2, [%3], %4;" ::"r"(smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar)), "l"(policy)
      : "memory");
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
// M = 128, N = kTileN.
constexpr uint32_t kIdesc = (1u << 4) | (1u << 7) | (1u << 10) |
                            (static_cast<uint32_t>(kTileN >> 3) << 17) | ((128u >> 4) << 24);

// D (TMEM) += A (TMEM) x B (shared memory descriptor); accumulate == 0
// overwrites D.
__device__ __forceinline__ void mma_bf16_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t bdesc,
                                            uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
      "r"(a_tmem), "l"(bdesc), "r"(kIdesc), "r"(accumulate)
      : "memory");
}

// 32 lanes x 16 consecutive 32-bit TMEM columns from registers.
__device__ __forceinline__ void tmem_st16(uint32_t taddr, const uint32_t *v) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], "
      "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};" ::"r"(taddr),
      "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7]),
      "r"(v[8]), "r"(v[9]), "r"(v[10]), "r"(v[11]), "r"(v[12]), "r"(v[13]), "r"(v[14]),
      "r"(v[15])
      : "memory");
}

__device__ __forceinline__ void tmem_wait_st() {
  asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void mma_commit(uint64_t *bar) {
  asm volatile(
      "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
          smem_u32(bar))
      : "memory");
}

#define H24_R8(b) "=r"(r[b + 0]), "=r"(r[b + 1]), "=r"(r[b + 2]), "=r"(r[b + 3]), \
                  "=r"(r[b + 4]), "=r"(r[b + 5]), "=r"(r[b + 6]), "=r"(r[b + 7])

// 32 lanes x 64 consecutive 32-bit TMEM columns.
__device__ __forceinline__ void tmem_ld64(uint32_t taddr, uint32_t *r) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x64.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,"
      "%32,%33,%34,%35,%36,%37,%38,%39,%40,%41,%42,%43,%44,%45,%46,%47,"
      "%48,%49,%50,%51,%52,%53,%54,%55,%56,%57,%58,%59,%60,%61,%62,%63}, [%64];"
      : H24_R8(0), H24_R8(8), H24_R8(16), H24_R8(24), H24_R8(32), H24_R8(40), H24_R8(48),
        H24_R8(56)
      : "r"(taddr));
}
#undef H24_R8

#define H24_T8(b) "+r"(r[b + 0]), "+r"(r[b + 1]), "+r"(r[b + 2]), "+r"(r[b + 3]), \
                  "+r"(r[b + 4]), "+r"(r[b + 5]), "+r"(r[b + 6]), "+r"(r[b + 7])
// Waits for this thread's outstanding tcgen05.ld and ties the loaded registers
// to the wait so that no use of them is scheduled before it.
__device__ __forceinline__ void tmem_wait_ld(uint32_t *r) {
  asm volatile("tcgen05.wait::ld.sync.aligned;"
               : H24_T8(0), H24_T8(8), H24_T8(16), H24_T8(24), H24_T8(32), H24_T8(40),
                 H24_T8(48), H24_T8(56)
               :
               : "memory");
}
#undef H24_T8

__device__ __forceinline__ float fmax3(float a, float b, float c) {
  float d;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
  return d;
}

// Maximum of 60 fp32 values held as raw bits (tree of 3-input max).
__device__ __forceinline__ float max60(const uint32_t *r) {
  float m[20];
#pragma unroll
  for (int k = 0; k < 20; ++k)
    m[k] = fmax3(__uint_as_float(r[3 * k]), __uint_as_float(r[3 * k + 1]),
                 __uint_as_float(r[3 * k + 2]));
  float n[7];
#pragma unroll
  for (int k = 0; k < 6; ++k) n[k] = fmax3(m[3 * k], m[3 * k + 1], m[3 * k + 2]);
  n[6] = fmaxf(m[18], m[19]);
  return fmax3(fmax3(n[0], n[1], n[2]), fmax3(n[3], n[4], n[5]), n[6]);
}

// ---------------------------------------------------------------------------
// 1. prep
// ---------------------------------------------------------------------------
// Input atoms of one pipeline batch: segment i holds atoms [start[i],
// start[i+1]) of the batch, stored contiguously at x[i] (24 fp32 per atom).
struct Segs {
  const float *x[kMaxSegs];
  int64_t start[kMaxSegs + 1];
  int count;
};

__device__ __forceinline__ const float *atom_ptr(const Segs &sg, int64_t a) {
  int lo = 0, hi = sg.count - 1;
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (sg.start[mid] <= a) lo = mid; else hi = mid - 1;
  }
  return sg.x[lo] + (a - sg.start[lo]) * kDim;
}

__global__ void __launch_bounds__(256) prep_kernel(const __grid_constant__ Segs sg, int64_t n,
                                                   int64_t n_pad, uint8_t *__restrict__ a_hi,
                                                   float *__restrict__ two_e) {
  const int64_t a = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x;
  if (a >= n_pad) return;
  float v[kDim];
  if (a < n) {
    const float4 *src = reinterpret_cast<const float4 *>(atom_ptr(sg, a));
#pragma unroll
    for (int q = 0; q < 6; ++q) {
      const float4 f = __ldcs(src + q);
      v[4 * q + 0] = f.x;
      v[4 * q + 1] = f.y;
      v[4 * q + 2] = f.z;
      v[4 * q + 3] = f.w;
    }
  } else {
#pragma unroll
    for (int i = 0; i < kDim; ++i) v[i] = 0.f;
  }
  float sum_d = 0.f, sum_d2 = 0.f, sum_x = 0.f;
  bool finite = true;
  uint32_t hi_bits[12];
#pragma unroll
  for (int i = 0; i < kDim; i += 2) {
    const __nv_bfloat162 h2 = __floats2bfloat162_rn(v[i], v[i + 1]);
    const float h0 = __low2float(h2), h1 = __high2float(h2);
    const float d0 = fabsf(v[i] - h0), d1 = fabsf(v[i + 1] - h1);
    sum_d += d0 + d1;
    sum_d2 = fmaf(d0, d0, fmaf(d1, d1, sum_d2));
    sum_x += fabsf(v[i]) + fabsf(v[i + 1]);
    finite = finite && isfinite(v[i]) && isfinite(v[i + 1]);
    hi_bits[i / 2] = *reinterpret_cast<const uint32_t *>(&h2);
  }
  // |sum_i raw_ji d_i| <= min(4 sum|d|, sqrt(32) ||d||); tensor-core
  // accumulation, the fp32 rounding of 3*LEECH_SCALE and the fp64 rescore add
  // at most 2^-12 * sum|x| (raw units).  The factor 1.001 absorbs the fp32
  // rounding of these sums.
  const float e_hi = fminf(4.f * sum_d, 5.656854249f * sqrtf(sum_d2));
  const float e = (e_hi + 2.44140625e-4f * sum_x) * 1.001f;
  if (a < n) two_e[a] = finite ? 2.f * e : -1.f;
  // Row of 32 bf16 (24 values, 8 zeros): the atom's lane of the A operand.
  uint4 *dst = reinterpret_cast<uint4 *>(a_hi + a * kHiBytes);
#pragma unroll
  for (int c = 0; c < 3; ++c)
    dst[c] = make_uint4(hi_bits[4 * c], hi_bits[4 * c + 1], hi_bits[4 * c + 2], hi_bits[4 * c + 3]);
  dst[3] = make_uint4(0, 0, 0, 0);
}

// ---------------------------------------------------------------------------
// 2. tcgen05 screening
// ---------------------------------------------------------------------------
// Per atom and column half h (chunks 2t+h): cand_n[2a+h] entries (or the
// bitmap / overflow codes), chunk ids cand[(2a+h)*kCap + k] with their
// screening maxima cand_sc[...], and the half's screening maximum best[2a+h].
struct ScreenArgs {
  const uint8_t *a_hi;        // [n_pad][32] bf16 rows
  const float *two_e;
  const uint8_t *cb_tiled;
  uint16_t *cand;     // [n_pad*2][kCap]
  float *cand_sc;     // [n_pad*2][kCap]
  uint8_t *cand_n;    // [n_pad*2]
  float *best;        // [n_pad*2]
  uint32_t *bitmaps;  // [pool_slots][kBitmapWords]
  int32_t *slot_count;
  int32_t pool_slots;
  int64_t n;
  int64_t nblocks;
  int *err;
};

// Per-atom candidate state of one epilogue thread.
struct Cands {
  int cnt = 0;          // list entries in shared memory
  bool ovf = false;     // give up: exhaustive fp64 scan
  int slot = -1;        // bitmap slot once the list has overflowed
  int bm_idx = -1;      // bitmap word being accumulated in bm_word
  uint32_t bm_word = 0;
};

// Bitmap mode: chunks arrive in increasing order, so each 32-chunk word is
// accumulated in a register and stored once.
__device__ __forceinline__ void bitmap_set(const ScreenArgs &args, Cands &c, int chunk) {
  const int w = chunk >> 5;
  if (w != c.bm_idx) {
    if (c.bm_idx >= 0) args.bitmaps[static_cast<int64_t>(c.slot) * kBitmapWords + c.bm_idx] = c.bm_word;
    c.bm_idx = w;
    c.bm_word = 0;
  }
  c.bm_word |= 1u << (chunk & 31);
}

__device__ __forceinline__ void epilogue_insert(ScreenSmem &S, const ScreenArgs &args, int list,
                                                float m, int chunk, float thr, Cands &c) {
  const int local = list;
  if (!(m >= thr)) return;
  if (c.slot >= 0) {
    bitmap_set(args, c, chunk);
    return;
  }
  if (c.cnt == kCap) {
    int k = 0;
    for (int i = 0; i < kCap; ++i) {
      const float sc = S.cand_score[i][local];
      if (sc >= thr) {
        S.cand_score[k][local] = sc;
        S.cand_chunk[k][local] = S.cand_chunk[i][local];
        ++k;
      }
    }
    c.cnt = k;
  }
  if (c.cnt < kCap) {
    S.cand_score[c.cnt][local] = m;
    S.cand_chunk[c.cnt][local] = static_cast<uint16_t>(chunk);
    ++c.cnt;
    return;
  }
  // The list holds kCap chunks within 2E of the running best: exact ties over
  // many chunks.  Move to a bitmap slot (zeroed here by its owner).
  const int slot = atomicAdd(args.slot_count, 1);
  if (slot >= args.pool_slots) {
    c.ovf = true;
    return;
  }
  c.slot = slot;
  uint32_t *bm = args.bitmaps + static_cast<int64_t>(slot) * kBitmapWords;
  for (int w = 0; w < kBitmapWords; ++w) bm[w] = 0u;
  for (int i = 0; i < c.cnt; ++i)
    if (S.cand_score[i][local] >= thr) bitmap_set(args, c, S.cand_chunk[i][local]);
  bitmap_set(args, c, chunk);
}

__global__ void __launch_bounds__(kScreenThreads, 1) screen_kernel(const ScreenArgs args) {
  extern __shared__ uint8_t smem_raw[];
  ScreenSmem &S = *reinterpret_cast<ScreenSmem *>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  volatile int *abort_flag = &S.abort_flag;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&S.bar_b_full[s], 1);
      mbar_init(&S.bar_b_empty[s], 2);       // one commit per MMA issuer
    }
    for (int h = 0; h < 2; ++h) {
      for (int s = 0; s < 2; ++s) mbar_init(&S.bar_a_full[s][h], kTileWarps / 2);
      for (int s = 0; s < kAccStages; ++s) {
        mbar_init(&S.bar_acc_full[s][h], 1);
        mbar_init(&S.bar_acc_empty[s][h], kTileWarps);
      }
      mbar_init(&S.bar_final[h], 1);
    }
    S.abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
  }
  if (warp == 1) {
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

  if (warp == 0) {
    // ---------------- producer: bulk copies of codebook tiles ----------------
    if (lane == 0) {
      const uint64_t keep = policy_evict_last();
      int bs = 0;
      uint32_t bph = 0;
      int last_b[kStages];
      for (int s = 0; s < kStages; ++s) last_b[s] = -1;
      bool ok = true;
      for (int64_t blk = blockIdx.x; ok && blk < args.nblocks; blk += gridDim.x) {
        for (int t = 0; t < kNumTiles; ++t) {
          if (!wait_bar(&S.bar_b_empty[bs], bph ^ 1, abort_flag, args.err)) { ok = false; break; }
          mbar_arrive_expect_tx(&S.bar_b_full[bs], kBTileBytes);
          bulk_g2s(S.b[bs], args.cb_tiled + static_cast<int64_t>(t) * kBTileBytes, kBTileBytes,
                   &S.bar_b_full[bs], keep);
          last_b[bs] = static_cast<int>(bph);
          if (++bs == kStages) { bs = 0; bph ^= 1; }
        }
      }
      if (!ok) {
        // Let every copy already issued land before the CTA leaves.
        for (int s = 0; s < kStages; ++s)
          if (last_b[s] >= 0) {
            const unsigned long long t0 = global_ns();
            while (!mbar_try_wait(&S.bar_b_full[s], static_cast<uint32_t>(last_b[s])) &&
                   global_ns() - t0 < kWaitLimitNs) {
            }
          }
      }
    }
  } else if (warp <= 2) {
    // ---------------- MMA issuers: warp 1 -> M-tile 0, warp 2 -> M-tile 1 ---
    // MMA issue blocks until the tensor core accepts the instruction, so two
    // issuers let one wait on its barriers while the other's MMAs run.
    const int h = warp - 1;
    if (lane == 0) {
      const uint64_t bd0 = smem_desc(smem_u32(S.b[0]));
      constexpr uint64_t kBStep = kBTileBytes >> 4;           // descriptor units
      constexpr uint64_t kKStep = 256 >> 4;                   // next 16 K in shared memory
      constexpr uint32_t kAKStep = 8;                         // next 16 K in TMEM (columns)
      int bs = 0, ab = 0, as = 0;
      uint32_t bph = 0, aph = 0, cph = 0;
      bool ok = true;
      bool issued = false;
      for (int64_t blk = blockIdx.x; ok && blk < args.nblocks; blk += gridDim.x) {
        if (!wait_bar(&S.bar_a_full[ab][h], aph, abort_flag, args.err)) { ok = false; break; }
        tc_fence_after();
        const uint32_t a = tmem_base + kAColBase + static_cast<uint32_t>(h) * kACols;
        for (int t = 0; t < kNumTiles; ++t) {
          if (!wait_bar(&S.bar_b_full[bs], bph, abort_flag, args.err)) { ok = false; break; }
          if (!wait_bar(&S.bar_acc_empty[as][h], cph ^ 1, abort_flag, args.err)) { ok = false; break; }
          tc_fence_after();
          const uint64_t bd = bd0 + static_cast<uint64_t>(bs) * kBStep;
          const uint32_t d = tmem_base + static_cast<uint32_t>(as * 2 * kTileN + h * kTileN);
          mma_bf16_ts(d, a, bd, 0);
          mma_bf16_ts(d, a + kAKStep, bd + kKStep, 1);
          mma_commit(&S.bar_acc_full[as][h]);
          mma_commit(&S.bar_b_empty[bs]);
          issued = true;
          if (++bs == kStages) { bs = 0; bph ^= 1; }
          as ^= 1;
          cph ^= (as == 0);
        }
        if (++ab == 2) { ab = 0; aph ^= 1; }
      }
      if (issued) {
        // All MMAs of this issuer complete before TMEM is released.
        mma_commit(&S.bar_final[h]);
        const unsigned long long t0 = global_ns();
        while (!mbar_try_wait(&S.bar_final[h], 0) && global_ns() - t0 < kWaitLimitNs) {
        }
      }
    }
  } else {
    // ---------------- epilogue: one thread per (atom, column half) --------
    // Warp w may only access TMEM lanes 32*(w%4)..+31.  The 16 warps cover two
    // M=128 tiles x four lane quarters x two column halves of each tile;
    // every half is one 60-codeword candidate chunk (chunk 2t + half).
    const int ew = warp - kFirstEpiWarp;
    const int h = ew >> 3;               // which M=128 tile
    const int q = warp & 3;              // TMEM lane quarter
    const int half = (ew >> 2) & 1;      // column half = chunk parity
    const int local = h * 128 + q * 32 + lane;
    const int list = half * kBlockAtoms + local;
    const uint32_t lane_off = static_cast<uint32_t>(q * 32) << 16;
    // A 64-column load that covers the chunk: half 0 reads columns 0..63
    // (values r[0..59]), half 1 reads 56..119 (values r[4..63]).
    const uint32_t t_lane = tmem_base + lane_off + static_cast<uint32_t>(h * kTileN + half * 56);
    bool ok = true;
    int ab = 0;
    int acc_stage_ = 0;
    uint32_t acc_phase_ = 0;
    for (int64_t blk = blockIdx.x; ok && blk < args.nblocks; blk += gridDim.x) {
      const int64_t atom = blk * kBlockAtoms + local;
      if (half == 0) {
        // Write this atom's bf16 row into the A operand.  It was last read by
        // the MMAs of block blk-1, all complete: this warp has already consumed
        // every accumulator of that block.  The barrier `ab` alternates per
        // block so that its phase parity identifies the block.
        uint32_t v[16];
        const uint4 *src = reinterpret_cast<const uint4 *>(args.a_hi + atom * kHiBytes);
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          const uint4 u = __ldcs(src + k);
          v[4 * k] = u.x;
          v[4 * k + 1] = u.y;
          v[4 * k + 2] = u.z;
          v[4 * k + 3] = u.w;
        }
        tmem_st16(tmem_base + lane_off + kAColBase + static_cast<uint32_t>(h) * kACols, v);
        tmem_wait_st();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&S.bar_a_full[ab][h]);
      }
      ab ^= 1;
      const float te = atom < args.n ? args.two_e[atom] : -1.f;
      const bool track = te >= 0.f;
      float best = -INFINITY;
      float thr = track ? -INFINITY : INFINITY;
      Cands cs;
      // Tiles alternate between the two accumulator stages; a stage's phase
      // parity flips every second tile.  kNumTiles is odd, so the stage and
      // parity sequence continues across blocks.
      for (int t = 0; t < kNumTiles; ++t) {
        // Lane 0 waits on the barrier; the warp then synchronises and fences
        // so that the .sync.aligned TMEM load is ordered after the MMAs.
        bool got = true;
        if (lane == 0) got = wait_bar(&S.bar_acc_full[acc_stage_][h], acc_phase_, abort_flag, args.err);
        if (!__shfl_sync(0xffffffffu, got, 0)) { ok = false; break; }
        tc_fence_after();
        uint32_t r[64];
        tmem_ld64(t_lane + static_cast<uint32_t>(acc_stage_ * 2 * kTileN), r);
        tmem_wait_ld(r);
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&S.bar_acc_empty[acc_stage_][h]);
        acc_stage_ ^= 1;
        acc_phase_ ^= (acc_stage_ == 0);
        float m = -INFINITY;
        if (half == 0) m = max60(r);
        else m = max60(r + 4);
        if (m >= thr) {
          if (m > best) {
            best = m;
            thr = best - te;
          }
          epilogue_insert(S, args, list, m, 2 * t + half, thr, cs);
          if (cs.ovf) thr = INFINITY;
        }
        best = fmaxf(best, m);
      }
      if (!ok) break;
      if (atom < args.n) {
        const int64_t li = atom * 2 + half;
        uint8_t n_out = kOverflow;
        if (track && !cs.ovf) {
          if (cs.slot >= 0) {
            args.bitmaps[static_cast<int64_t>(cs.slot) * kBitmapWords + cs.bm_idx] = cs.bm_word;
            args.cand[li * kCap] = static_cast<uint16_t>(cs.slot & 0xFFFF);
            args.cand[li * kCap + 1] = static_cast<uint16_t>(cs.slot >> 16);
            n_out = kBitmapMode;
          } else {
            int k = 0;
            for (int i = 0; i < cs.cnt; ++i) {
              const float sc = S.cand_score[i][list];
              if (sc >= thr) {
                args.cand[li * kCap + k] = S.cand_chunk[i][list];
                args.cand_sc[li * kCap + k] = sc;
                ++k;
              }
            }
            n_out = static_cast<uint8_t>(k);
          }
        }
        args.cand_n[li] = n_out;
        args.best[li] = best;
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) {
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

__device__ __forceinline__ void load_atom(const float *__restrict__ p, float (&v)[kDim]) {
  const float4 *src = reinterpret_cast<const float4 *>(p);
#pragma unroll
  for (int q = 0; q < 6; ++q) {
    const float4 f = __ldg(src + q);
    v[4 * q] = f.x;
    v[4 * q + 1] = f.y;
    v[4 * q + 2] = f.z;
    v[4 * q + 3] = f.w;
  }
}

// Index for atoms that need no search: non-finite input (training rule: the
// origin, as the Triton kernel's never-improving running max snaps; pack rule:
// row 1, torch.max's first NaN), or the pack rule's ||x|| < 1e-8.
// Returns -1 when a search is needed.
__device__ __forceinline__ int trivial_index(const float (&v)[kDim], int rule) {
  bool finite = true;
  double ss = 0.0;
#pragma unroll
  for (int i = 0; i < kDim; ++i) {
    finite = finite && isfinite(v[i]);
    ss = __fma_rn(static_cast<double>(v[i]), static_cast<double>(v[i]), ss);
  }
  if (!finite) return rule == H24_RULE_TRAIN ? 0 : 1;
  if (rule == H24_RULE_PACK && sqrt(ss) < 1e-8) return 0;
  return -1;
}

__device__ __forceinline__ int32_t apply_rule(double best, int bj, int rule) {
  if (rule == H24_RULE_TRAIN && 2.0 * best < kCSqNorm) return 0;
  return bj + 1;
}

// fp64 rescore of one 60-codeword chunk by a warp (up to two codewords per lane).
__device__ __forceinline__ void rescore_chunk(const float (&v)[kDim], const int8_t *__restrict__ cb_raw,
                                              int c, int lane, double &bs, int &bj) {
#pragma unroll
  for (int half = 0; half < 2; ++half) {
    const int o = half * 32 + lane;
    if (o < kChunk) {
      const int j = c * kChunk + o;
      better(bs, bj, score64(v, cb_raw + static_cast<int64_t>(j) * kDim), j);
    }
  }
}

struct RescoreArgs {
  const uint16_t *cand;
  const float *cand_sc;
  const uint8_t *cand_n;
  const float *best_approx;
  const float *two_e;
  const uint32_t *bitmaps;
  const int8_t *cb_raw;
  int32_t *out;
  int32_t *ovf_list;
  int32_t *ovf_count;
  int64_t *stats;  // [0] exhaustive atoms, [1] rescored chunks, [2] bitmap atoms
  int64_t n;
  int rule;
};

__global__ void __launch_bounds__(256) rescore_kernel(const __grid_constant__ Segs sg,
                                                      const RescoreArgs r) {
  __shared__ int block_ovf, block_chunks, block_bitmap;
  if (threadIdx.x == 0) {
    block_ovf = 0;
    block_chunks = 0;
    block_bitmap = 0;
  }
  __syncthreads();
  const int lane = threadIdx.x & 31;
  const int64_t a = (blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x) >> 5;
  if (a < r.n) {
    float v[kDim];
    load_atom(atom_ptr(sg, a), v);
    const int triv = trivial_index(v, r.rule);
    const int cn0 = r.cand_n[2 * a], cn1 = r.cand_n[2 * a + 1];
    // The screening maximum over both halves sets the candidate threshold.
    const float gbest = fmaxf(r.best_approx[2 * a], r.best_approx[2 * a + 1]);
    const float te = r.two_e[a];
    if (triv >= 0) {
      if (lane == 0) r.out[a] = triv;
    } else if (cn0 == kOverflow || cn1 == kOverflow) {
      // Certain origin under the training rule: even best + E stays below the
      // snap threshold (1e-6 covers the fp32 codebook's rounding).
      const double ub = static_cast<double>(kLeechScaleF) *
                        (static_cast<double>(gbest) + 0.5 * te) * (1.0 + 1e-6);
      if (lane == 0) {
        r.out[a] = 0;
        if (!(r.rule == H24_RULE_TRAIN && 2.0 * ub < kCSqNorm)) {
          r.ovf_list[atomicAdd(r.ovf_count, 1)] = static_cast<int32_t>(a);
          atomicAdd(&block_ovf, 1);
        }
      }
    } else {
      const float thr = gbest - te;
      double bs = -INFINITY;
      int bj = 0x7FFFFFFF;
      int chunks = 0;
      bool used_bitmap = false;
#pragma unroll
      for (int hf = 0; hf < 2; ++hf) {
        const int cn = hf ? cn1 : cn0;
        const int64_t li = 2 * a + hf;
        if (cn == kBitmapMode) {
          used_bitmap = true;
          const int slot = static_cast<int>(r.cand[li * kCap]) |
                           (static_cast<int>(r.cand[li * kCap + 1]) << 16);
          const uint32_t *bm = r.bitmaps + static_cast<int64_t>(slot) * kBitmapWords;
          for (int w = 0; w < kBitmapWords; ++w) {
            uint32_t word = __ldg(bm + w);
            while (word) {
              const int b = __ffs(word) - 1;
              word &= word - 1;
              rescore_chunk(v, r.cb_raw, w * 32 + b, lane, bs, bj);
              ++chunks;
            }
          }
        } else {
          for (int k = 0; k < cn; ++k) {
            if (!(r.cand_sc[li * kCap + k] >= thr)) continue;
            rescore_chunk(v, r.cb_raw, r.cand[li * kCap + k], lane, bs, bj);
            ++chunks;
          }
        }
      }
#pragma unroll
      for (int off = 16; off > 0; off >>= 1) {
        const double os = __shfl_xor_sync(0xffffffffu, bs, off);
        const int oj = __shfl_xor_sync(0xffffffffu, bj, off);
        better(bs, bj, os, oj);
      }
      if (lane == 0) {
        r.out[a] = chunks > 0 ? apply_rule(bs, bj, r.rule) : 0;
        atomicAdd(&block_chunks, chunks);
        if (used_bitmap) atomicAdd(&block_bitmap, 1);
      }
    }
  }
  __syncthreads();
  if (threadIdx.x == 0 && (block_ovf || block_chunks || block_bitmap)) {
    atomicAdd(reinterpret_cast<unsigned long long *>(&r.stats[0]),
              static_cast<unsigned long long>(block_ovf));
    atomicAdd(reinterpret_cast<unsigned long long *>(&r.stats[1]),
              static_cast<unsigned long long>(block_chunks));
    atomicAdd(reinterpret_cast<unsigned long long *>(&r.stats[2]),
              static_cast<unsigned long long>(block_bitmap));
  }
}

__global__ void __launch_bounds__(256) exhaustive_kernel(const __grid_constant__ Segs sg, int rule,
                                                         const int32_t *__restrict__ ovf_list,
                                                         const int32_t *__restrict__ ovf_count,
                                                         const int8_t *__restrict__ cb_raw,
                                                         int32_t *__restrict__ out) {
  __shared__ double ws[8];
  __shared__ int wj[8];
  const int count = *ovf_count;
  for (int e = blockIdx.x; e < count; e += gridDim.x) {
    const int64_t a = ovf_list[e];
    float v[kDim];
    load_atom(atom_ptr(sg, a), v);
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

std::mutex g_mu;
int g_sms[64] = {};

}  // namespace

int quantize_segments(const Tables *t, const float *const *xs, const int64_t *counts, int nseg,
                      int rule, int32_t *out_idx, cudaStream_t s) {
  int64_t total = 0;
  for (int i = 0; i < nseg; ++i) {
    if (counts[i] < 0) return fail(H24_ERR_INVALID, "quantize: negative segment length");
    if (counts[i] > 0 && (!xs[i] || !aligned16(xs[i])))
      return fail(H24_ERR_INVALID, "quantize: segment pointers must be non-null and 16-byte aligned");
    total += counts[i];
  }
  if (total == 0) return H24_OK;
  int sms = 0;
  {
    std::lock_guard<std::mutex> lk(g_mu);
    const int dev = t->device;
    if (g_sms[dev] == 0) {
      int count = 0;
      H24_CUDA_TRY(cudaDeviceGetAttribute(&count, cudaDevAttrMultiProcessorCount, dev));
      H24_CUDA_TRY(cudaFuncSetAttribute(screen_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                        static_cast<int>(sizeof(ScreenSmem) + 1024)));
      g_sms[dev] = count;
    }
    sms = g_sms[dev];
  }

  const int64_t batch = total < kBatchAtoms ? total : kBatchAtoms;
  const int64_t nb_max = (batch + kBlockAtoms - 1) / kBlockAtoms;
  const int64_t pad_max = nb_max * kBlockAtoms;
  const int64_t pool_slots = batch / 4 > 4096 ? batch / 4 : 4096;
  auto up = [](size_t v) { return (v + 255) & ~static_cast<size_t>(255); };
  const size_t off_two_e = up(static_cast<size_t>(pad_max) * kHiBytes);
  const size_t off_cand = off_two_e + up(pad_max * sizeof(float));
  const size_t off_cand_sc = off_cand + up(pad_max * 2 * kCap * sizeof(uint16_t));
  const size_t off_cand_n = off_cand_sc + up(pad_max * 2 * kCap * sizeof(float));
  const size_t off_best = off_cand_n + up(pad_max * 2);
  const size_t off_ovf = off_best + up(pad_max * 2 * sizeof(float));
  const size_t off_bm = off_ovf + up(batch * sizeof(int32_t));
  const size_t off_cnt = off_bm + up(static_cast<size_t>(pool_slots) * kBitmapWords * 4);
  const size_t bytes = off_cnt + 256;
  uint8_t *scratch = nullptr;
  H24_CUDA_TRY(cudaMallocFromPoolAsync(reinterpret_cast<void **>(&scratch), bytes, t->pool, s));
  int rc = H24_OK;
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
      sg.x[sg.count] = xs[seg] + seg_off * kDim;
      nbatch += take;
      sg.start[++sg.count] = nbatch;
      seg_off += take;
      if (seg_off == counts[seg]) { ++seg; seg_off = 0; }
    }
    const int64_t nb = (nbatch + kBlockAtoms - 1) / kBlockAtoms;
    const int64_t npad = nb * kBlockAtoms;
    int32_t *ob = out_idx + done;
    uint8_t *a_hi = scratch;
    float *two_e = reinterpret_cast<float *>(scratch + off_two_e);
    uint16_t *cand = reinterpret_cast<uint16_t *>(scratch + off_cand);
    float *cand_sc = reinterpret_cast<float *>(scratch + off_cand_sc);
    uint8_t *cand_n = scratch + off_cand_n;
    float *best = reinterpret_cast<float *>(scratch + off_best);
    int32_t *ovf_list = reinterpret_cast<int32_t *>(scratch + off_ovf);
    uint32_t *bitmaps = reinterpret_cast<uint32_t *>(scratch + off_bm);
    int32_t *ovf_count = reinterpret_cast<int32_t *>(scratch + off_cnt);
    int32_t *slot_count = ovf_count + 1;
    cudaError_t e = cudaMemsetAsync(ovf_count, 0, 2 * sizeof(int32_t), s);
    if (e != cudaSuccess) { rc = cuda_fail(e, "memset"); break; }
    prep_kernel<<<static_cast<unsigned>((npad + 255) / 256), 256, 0, s>>>(sg, nbatch, npad, a_hi,
                                                                        two_e);
    ScreenArgs sa{a_hi, two_e, reinterpret_cast<const uint8_t *>(t->cb_tiled), cand, cand_sc,
                  cand_n, best, bitmaps, slot_count, static_cast<int32_t>(pool_slots), nbatch, nb,
                  t->err};
    const int grid = static_cast<int>(nb < sms ? nb : sms);
    cudaEvent_t ev0 = nullptr, ev1 = nullptr;
    if (timing_enabled()) {
      cudaEventCreate(&ev0);
      cudaEventCreate(&ev1);
      cudaEventRecord(ev0, s);
    }
    screen_kernel<<<grid, kScreenThreads, sizeof(ScreenSmem) + 1024, s>>>(sa);
    if (ev1) {
      cudaEventRecord(ev1, s);
      timing_record(ev0, ev1);
    }
    RescoreArgs ra{cand, cand_sc, cand_n, best, two_e, bitmaps, t->cb_raw, ob, ovf_list, ovf_count,
                   t->stats, nbatch, rule};
    const int64_t rthreads = nbatch * 32;
    rescore_kernel<<<static_cast<unsigned>((rthreads + 255) / 256), 256, 0, s>>>(sg, ra);
    exhaustive_kernel<<<2 * sms, 256, 0, s>>>(sg, rule, ovf_list, ovf_count, t->cb_raw, ob);
    count_launches(4);
    e = cudaGetLastError();
    if (e != cudaSuccess) rc = cuda_fail(e, "quantize launch");
    done += nbatch;
  }
  cudaError_t e = cudaFreeAsync(scratch, s);
  if (rc == H24_OK && e != cudaSuccess) rc = cuda_fail(e, "cudaFreeAsync");
  return rc;
}

int quantize(const Tables *t, const float *x, int64_t n, int rule, int32_t *out_idx,
             cudaStream_t s) {
  return quantize_segments(t, &x, &n, 1, rule, out_idx, s);
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
//     call's contents: the counters that must start at zero are cleared at
//     the start of each call, everything else is written before it is read.
//     Calls whose executions overlap on the GPU (other streams or host
//     threads without ordering) race on the array.
// ===========================================================================
namespace {

constexpr int64_t kNoAllocMaxAtoms = 32768;
constexpr int64_t kNoAllocPad = kNoAllocMaxAtoms;  // a multiple of kBlockAtoms
constexpr int64_t kNoAllocSlots = kNoAllocMaxAtoms / 4;
constexpr size_t na_up(size_t v) { return (v + 255) & ~static_cast<size_t>(255); }
constexpr size_t kNaTwoE = na_up(kNoAllocPad * kHiBytes);
constexpr size_t kNaCand = kNaTwoE + na_up(kNoAllocPad * sizeof(float));
constexpr size_t kNaCandSc = kNaCand + na_up(kNoAllocPad * 2 * kCap * sizeof(uint16_t));
constexpr size_t kNaCandN = kNaCandSc + na_up(kNoAllocPad * 2 * kCap * sizeof(float));
constexpr size_t kNaBest = kNaCandN + na_up(kNoAllocPad * 2);
constexpr size_t kNaOvf = kNaBest + na_up(kNoAllocPad * 2 * sizeof(float));
constexpr size_t kNaBm = kNaOvf + na_up(kNoAllocMaxAtoms * sizeof(int32_t));
constexpr size_t kNaCnt = kNaBm + na_up(static_cast<size_t>(kNoAllocSlots) * kBitmapWords * 4);
constexpr size_t kNoAllocBytes = kNaCnt + 256;  // about 10.5 MB
static_assert(kNoAllocMaxAtoms % kBlockAtoms == 0, "whole CTA work items");
static_assert(kNoAllocBytes < (size_t(16) << 20), "modest fixed footprint");

// The scratch array.  In host code this name is a host-side stand-in, not a
// device address: host code must use the address from cudaGetSymbolAddress.
static __device__ __align__(256) uint8_t g_noalloc_scratch[kNoAllocBytes];

std::mutex g_noalloc_mu;
uint8_t *g_noalloc_ptr[64] = {};

// Per-device set-up: resolve the array's device address (once, with the device
// current) and allow the screening kernel its dynamic shared memory.
int noalloc_setup(int dev, uint8_t **out) {
  std::lock_guard<std::mutex> lk(g_noalloc_mu);
  if (!g_noalloc_ptr[dev]) {
    void *ptr = nullptr;
    cudaError_t e = cudaGetSymbolAddress(&ptr, g_noalloc_scratch);
    if (e != cudaSuccess) return cuda_fail(e, "cudaGetSymbolAddress(noalloc scratch)");
    e = cudaFuncSetAttribute(screen_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             static_cast<int>(sizeof(ScreenSmem) + 1024));
    if (e != cudaSuccess) return cuda_fail(e, "cudaFuncSetAttribute");
    g_noalloc_ptr[dev] = static_cast<uint8_t *>(ptr);
  }
  *out = g_noalloc_ptr[dev];
  return H24_OK;
}

int quantize_noalloc(const Tables *t, const float *x, int64_t n, int rule, int32_t *out_idx,
                     cudaStream_t s) {
  uint8_t *scratch = nullptr;
  int rc = noalloc_setup(t->device, &scratch);
  if (rc != H24_OK) return rc;
  int sms = 0;
  H24_CUDA_TRY(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, t->device));
  Segs sg;
  sg.count = 1;
  sg.x[0] = x;
  sg.start[0] = 0;
  sg.start[1] = n;
  const int64_t nb = (n + kBlockAtoms - 1) / kBlockAtoms;
  const int64_t npad = nb * kBlockAtoms;
  uint8_t *a_hi = scratch;
  float *two_e = reinterpret_cast<float *>(scratch + kNaTwoE);
  uint16_t *cand = reinterpret_cast<uint16_t *>(scratch + kNaCand);
  float *cand_sc = reinterpret_cast<float *>(scratch + kNaCandSc);
  uint8_t *cand_n = scratch + kNaCandN;
  float *best = reinterpret_cast<float *>(scratch + kNaBest);
  int32_t *ovf_list = reinterpret_cast<int32_t *>(scratch + kNaOvf);
  uint32_t *bitmaps = reinterpret_cast<uint32_t *>(scratch + kNaBm);
  int32_t *ovf_count = reinterpret_cast<int32_t *>(scratch + kNaCnt);
  int32_t *slot_count = ovf_count + 1;
  // The array keeps the previous call's contents: clear the two counters.
  H24_CUDA_TRY(cudaMemsetAsync(ovf_count, 0, 2 * sizeof(int32_t), s));
  prep_kernel<<<static_cast<unsigned>((npad + 255) / 256), 256, 0, s>>>(sg, n, npad, a_hi, two_e);
  ScreenArgs sa{a_hi, two_e, reinterpret_cast<const uint8_t *>(t->cb_tiled), cand, cand_sc,
                cand_n, best, bitmaps, slot_count, static_cast<int32_t>(kNoAllocSlots), n, nb,
                t->err};
  screen_kernel<<<static_cast<int>(nb < sms ? nb : sms), kScreenThreads, sizeof(ScreenSmem) + 1024,
                  s>>>(sa);
  RescoreArgs ra{cand, cand_sc, cand_n, best, two_e, bitmaps, t->cb_raw, out_idx, ovf_list,
                 ovf_count, t->stats, n, rule};
  rescore_kernel<<<static_cast<unsigned>((n * 32 + 255) / 256), 256, 0, s>>>(sg, ra);
  exhaustive_kernel<<<2 * sms, 256, 0, s>>>(sg, rule, ovf_list, ovf_count, t->cb_raw, out_idx);
  count_launches(4);
  H24_CUDA_TRY(cudaGetLastError());
  return H24_OK;
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
