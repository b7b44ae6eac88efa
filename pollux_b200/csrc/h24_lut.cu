// h24_lut.cu -- matrix-free LUT GEMV over packed H24 layers on the
// fifth-generation tensor cores (the README's "future native kernel",
// README.md:88, 155-156): y[b][o] = sum_i x[b][i] * W[o][i] for up to 8 input
// rows per launch, W the fp16 weight PackedH24Linear.materialize produces
// (pollux.py:485-500), never written to HBM.
//
// A CTA owns a tile of 128 weight rows (two threads and one TMEM lane per
// row) and one of `split` (1, 2, 4 or 8) slices of the rows' atoms, chosen so
// that every CTA of the launch is resident at once.  With split > 1 each CTA
// writes its partial sums to a stream-ordered workspace and lut_reduce_kernel
// adds them in slice order, so the result does not depend on scheduling.
//
// The kernel is bound by L2 requests, one 16-byte code-entry gather per
// atom, so everything else is arranged to add few: at the start a CTA turns
// its slice of x into bf16 B tiles in shared memory (coalesced loads), and
// each thread reads its contiguous run of packed bytes in at most three
// aligned 16-byte loads and issues the gathers of up to 6 atoms at once.  Per
// chunk of two atoms (48 k) each thread then expands one atom's 24 weights
// with byte permutes into the two bf16 A pieces in shared memory (K-major core
// matrices, as tcgen05.mma reads them) and one elected thread issues 6 MMAs
// (M = 128, N = 16, K = 16) into a 16-column TMEM accumulator; two stages let
// the expansion of one chunk overlap the MMAs of the previous.
//
// Arithmetic.  W (fp16) = Wh + Wl exactly, Wh = bf16_rn(W) and Wl = W - Wh
// (a multiple of W's fp16 ulp of at most 3 bits, exact in bf16).  x = xh + xl
// + r with xh = bf16_rn(x), xl = bf16_rn(x - xh), |r| <= 2^-17 |x|.  Columns
// 0-7 of B hold xh of input rows 0-7 and columns 8-15 their xl; both A pieces
// multiply B, so D[o][b] + D[o][8+b] = sum_i W_oi (xh + xl)_bi, the bf16
// products exact and summed in fp32 by the tensor core.  bf16 has fp32's
// exponent range, so |y - x W^T| <= 2^-14 sum_i |x_i W_oi| holds for any
// finite x below bf16's largest value (3.39e38).
#include "h24_internal.cuh"

namespace h24 {
namespace {

constexpr int kLutThreads = 256;                         // two threads per row of the tile
constexpr int kTileRows = 128;                           // M of the MMA: weight rows per CTA
constexpr int kMaxB = 8;                                 // input rows per launch
constexpr int kChunkGroups = 6;                          // 8-element k groups per chunk (2 atoms)
constexpr int kAPiece = kChunkGroups * kTileRows * 16;   // 12,288 B: one bf16 piece of the A tile
constexpr int kAStage = 2 * kAPiece;                     // 24,576 B: hi and lo pieces
constexpr int kXTile = kChunkGroups * 16 * 16;           // 1,536 B: the B tile of a chunk (16 columns)
constexpr int kHead = 128;                               // barriers, TMEM address, abort flag
constexpr int kMaxSplit = 8;                             // atom slices per row tile
constexpr int kWindow = 6;                               // atoms per thread gathered together
static_assert(kWindow <= 6, "a window's packed bytes must fit three aligned 16-byte blocks");
static_assert(kLutThreads * 48 <= kAStage, "the byte slots borrow one stage");
constexpr uint32_t kTmemCols = 32;                       // smallest allocation; D uses 16 columns
constexpr unsigned long long kLutWaitNs = 2000000000ull; // bounded waits: 2 s
// Instruction descriptor: kind::f16, A = B = bf16, D = f32, both K-major,
// N = 16 (bits 17-22: N >> 3), M = 128 (bits 24-28: M >> 4).
constexpr uint32_t kLutIdesc = (1u << 4) | (1u << 7) | (1u << 10) | ((16u >> 3) << 17) | ((128u >> 4) << 24);

// Dynamic shared memory: [head | A stage 0 | A stage 1 | B tiles of the
// slice's chunks].
struct LutHead {
  uint64_t mma_done[2];  // one completion per use of a stage
  uint32_t tmem_base;
  int abort;
};
static_assert(sizeof(LutHead) <= kHead, "head");

size_t lut_smem_bytes(int chunks) { return kHead + 2 * static_cast<size_t>(kAStage) + static_cast<size_t>(chunks) * kXTile; }

struct LutArgs {
  const uint8_t *packed;
  const uint16_t *sigma16;
  const float *x;
  float *y;    // split == 1: the result [batch][rows]
  float *ws;   // split > 1: partial sums [split][kMaxB][rows]
  const uint32_t *codes;
  int32_t *bad;
  int *err;
  int64_t rows;
  int64_t in_f;
  int apr;
  int batch;
  int split;
};

__device__ __forceinline__ uint32_t su32(const void *p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// Shared-memory descriptor of a K-major operand without swizzle: `lbo` =
// distance between K-adjacent core matrices (8 rows x 16 bytes), `sbo` =
// distance between 8-row groups, version 1.
__device__ __forceinline__ uint64_t kmajor_desc(uint32_t addr, uint32_t lbo, uint32_t sbo) {
  return static_cast<uint64_t>((addr >> 4) & 0x3FFFu) | (static_cast<uint64_t>((lbo >> 4) & 0x3FFFu) << 16) |
         (static_cast<uint64_t>((sbo >> 4) & 0x3FFFu) << 32) | (uint64_t(1) << 46);
}

// One non-blocking test of the phase.
__device__ __forceinline__ bool bar_done(uint64_t *bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(su32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

__device__ __forceinline__ unsigned long long now_ns() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
  return t;
}

// Waits for the phase of `bar` with the given parity for at most kLutWaitNs;
// on a timeout raises the CTA abort flag and the device error word.
__device__ bool bar_wait(uint64_t *bar, uint32_t parity, volatile int *abort, int *err) {
  if (bar_done(bar, parity)) return true;
  const unsigned long long t0 = now_ns();
  for (;;) {
    if (bar_done(bar, parity)) return true;
    if (*abort) return false;
    if (now_ns() - t0 > kLutWaitNs) {
      *abort = 1;
      atomicExch(err, H24_ERR_TIMEOUT);
      return false;
    }
  }
}

// D (TMEM) += A x B from shared-memory descriptors (accumulate == 0
// overwrites D); a whole converged warp executes it, one elected lane issues.
__device__ __forceinline__ void lut_mma(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p, e;\n\t"
      "elect.sync _|e, 0xffffffff;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "@e tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(kLutIdesc), "r"(accumulate)
      : "memory");
}

__device__ __forceinline__ void lut_commit(uint64_t *bar) {
  asm volatile(
      "{\n\t.reg .pred e;\n\t"
      "elect.sync _|e, 0xffffffff;\n\t"
      "@e tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];\n\t}" ::"r"(su32(bar))
      : "memory");
}

__device__ __forceinline__ void tmem_ld16(uint32_t taddr, float (&d)[16]) {
  uint32_t r[16];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];\n\t"
      "tcgen05.wait::ld.sync.aligned;"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr)
      : "memory");
#pragma unroll
  for (int i = 0; i < 16; ++i) d[i] = __uint_as_float(r[i]);
}

// bf16 bits of bf16_rn(v) and of bf16_rn(v - bf16_rn(v)).
__device__ __forceinline__ void split_bf16(float v, uint32_t &hi, uint32_t &lo) {
  const __nv_bfloat16 h = __float2bfloat16_rn(v);
  hi = __bfloat16_as_ushort(h);
  lo = __bfloat16_as_ushort(__float2bfloat16_rn(v - __bfloat162float(h)));
}

// 8 bf16 weights of one code word (nibble e -> element e) from the value
// list pair (src0, src1): code c selects bytes 2c, 2c+1.
__device__ __forceinline__ uint4 expand8_pair(uint32_t s_lo, uint32_t s_hi, uint32_t src0, uint32_t src1) {
  return make_uint4(__byte_perm(src0, src1, s_lo), __byte_perm(src0, src1, s_lo >> 16),
                    __byte_perm(src0, src1, s_hi), __byte_perm(src0, src1, s_hi >> 16));
}

// The 16 bytes at `p` (16-byte aligned); bytes outside [lo, hi) (the packed
// buffer) are not read and come back as zeros.
__device__ __forceinline__ uint4 load16_within(const uint8_t *p, const uint8_t *lo, const uint8_t *hi) {
  if (p >= lo && p + 16 <= hi) return __ldg(reinterpret_cast<const uint4 *>(p));
  uint32_t w[4] = {0, 0, 0, 0};
#pragma unroll
  for (int k = 0; k < 16; ++k)
    if (p + k >= lo && p + k < hi) w[k >> 2] |= static_cast<uint32_t>(__ldg(p + k)) << (8 * (k & 3));
  return make_uint4(w[0], w[1], w[2], w[3]);
}

__global__ void __launch_bounds__(kLutThreads, 4) lut_tc_kernel(const __grid_constant__ LutArgs a) {
  extern __shared__ __align__(128) uint8_t lut_raw[];
  LutHead &H = *reinterpret_cast<LutHead *>(lut_raw);
  uint8_t *stages = lut_raw + kHead;
  uint8_t *xtiles = stages + 2 * kAStage;
  const int t = threadIdx.x, warp = t >> 5;
  const int row = t & (kTileRows - 1);  // row of the tile (TMEM lane)
  const int h = t >> 7;                 // which half of the slice this thread expands
  const int rank = static_cast<int>(blockIdx.x % a.split);
  const int64_t m0 = static_cast<int64_t>(blockIdx.x / a.split) * kTileRows;
  const int64_t o = m0 + row;
  const bool live = o < a.rows;
  // Atom slice [a_lo, a_lo + n) of the rows; thread half h expands atoms
  // a_lo + h*half + c for c < its count, and chunk c pairs atom a_lo + c with
  // atom a_lo + half + c (the MMA only needs A's and B's k groups to agree).
  const int a_lo = static_cast<int>(static_cast<int64_t>(rank) * a.apr / a.split);
  const int n = static_cast<int>(static_cast<int64_t>(rank + 1) * a.apr / a.split) - a_lo;
  const int half = (n + 1) / 2;
  const int my_first = a_lo + h * half;
  const int my_count = h == 0 ? half : n - half;
  volatile int *abort = &H.abort;

  if (t == 0) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(su32(&H.mma_done[0])));
    asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(su32(&H.mma_done[1])));
    H.abort = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");  // (a cluster of one CTA)
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
  }
  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(su32(&H.tmem_base)),
                 "r"(kTmemCols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  // B tiles of every chunk of the slice.  Entry (b, g, c, p) holds x[b] at
  // atom a_lo + g*half + c, elements 8p..8p+7, as column b (xh) and column
  // 8+b (xl) of k group 3g + p of chunk c's tile (k group j at j*256, column
  // n at (n >> 3)*128 + (n & 7)*16).  Consecutive entries read consecutive 32
  // bytes of one x row.
  for (int e = t; e < kMaxB * 2 * half * 3; e += kLutThreads) {
    const int p = e % 3, c = (e / 3) % half, g = (e / (3 * half)) & 1, b = e / (6 * half);
    const int rel = g * half + c;
    uint32_t vh[4] = {0, 0, 0, 0}, vl[4] = {0, 0, 0, 0};
    if (rel < n && b < a.batch) {
      const float4 *xp =
          reinterpret_cast<const float4 *>(a.x + b * a.in_f + static_cast<int64_t>(a_lo + rel) * kDim + 8 * p);
      const float4 x0 = __ldg(xp), x1 = __ldg(xp + 1);
      const float v[8] = {x0.x, x0.y, x0.z, x0.w, x1.x, x1.y, x1.z, x1.w};
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        uint32_t ha, la, hb, lb;
        split_bf16(v[2 * q], ha, la);
        split_bf16(v[2 * q + 1], hb, lb);
        vh[q] = ha | (hb << 16);
        vl[q] = la | (lb << 16);
      }
    }
    uint8_t *tile = xtiles + static_cast<size_t>(c) * kXTile + (3 * g + p) * 256 + b * 16;
    *reinterpret_cast<uint4 *>(tile) = make_uint4(vh[0], vh[1], vh[2], vh[3]);
    *reinterpret_cast<uint4 *>(tile + 128) = make_uint4(vl[0], vl[1], vl[2], vl[3]);
  }

  // The row's three value lists as bf16 pieces: word k holds two values,
  // (lo, hi) raw coordinates packed as nibbles lo+4 | (hi+4) << 4:
  // words 0-1 {+1,-1,+3,-3}, 2-3 {0,+2,-2,+4}, 4-5 {-2,+4,-4,0}.
  uint32_t Lh[6], Ll[6];
  {
    const uint16_t sg = live ? __ldg(a.sigma16 + o) : static_cast<uint16_t>(0);
    constexpr uint32_t kPairs = 0x82641735u;
#pragma unroll
    for (int k = 0; k < 6; ++k) {
      const uint32_t pair = k < 4 ? (kPairs >> (8 * k)) & 0xFFu : (k == 4 ? 0x82u : 0x40u);
      uint32_t h0, l0, h1, l1;
      split_bf16(__half2float(__ushort_as_half(dequant_value(static_cast<int>(pair & 15u) - 4, sg))), h0, l0);
      split_bf16(__half2float(__ushort_as_half(dequant_value(static_cast<int>(pair >> 4) - 4, sg))), h1, l1);
      Lh[k] = h0 | (h1 << 16);
      Ll[k] = l0 | (l1 << 16);
    }
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  const uint32_t tmem = H.tmem_base;
  const uint8_t *pk_lo = a.packed;
  const uint8_t *pk_hi = a.packed + 9 * ((a.rows * a.apr + 3) >> 2);
  unsigned nbad = 0;
  int i = 0;  // chunks issued so far (stage ring position)

  for (int w0 = 0; w0 < half; w0 += kWindow) {
    // 1. This thread's packed bytes of the window, at most three aligned
    //    16-byte loads into its 48-byte slot, then the code entries of all its
    //    atoms of the window.  The slots borrow stage 1: past the first window
    //    every MMA issued so far must have read it first.
    if (i > 0) bar_wait(&H.mma_done[(i - 1) & 1], static_cast<uint32_t>((i - 1) >> 1) & 1u, abort, a.err);
    const int cnt = live ? max(0, min(kWindow, my_count - w0)) : 0;
    const int64_t A0 = o * a.apr + my_first + w0;
    uint4 *slot = reinterpret_cast<uint4 *>(stages + kAStage) + 3 * t;
    // The span [9*(A0>>2), 9*((A0+cnt-1)>>2) + 9) is at most 27 bytes (cnt <=
    // 6), so with its start rounded down to 16 bytes it lies within three
    // aligned 16-byte blocks.
    const uint8_t *first = a.packed + 9 * (A0 >> 2);
    const uint8_t *base = reinterpret_cast<const uint8_t *>(reinterpret_cast<uintptr_t>(first) & ~uintptr_t(15));
    if (cnt > 0) {
      const uint8_t *end = a.packed + 9 * ((A0 + cnt - 1) >> 2) + 9;
#pragma unroll
      for (int q = 0; q < 3; ++q)
        if (base + 16 * q < end) slot[q] = load16_within(base + 16 * q, pk_lo, pk_hi);
    }
    const uint8_t *sb = reinterpret_cast<const uint8_t *>(slot);
    const int shift0 = static_cast<int>(first - base);
    uint4 cw[kWindow];
#pragma unroll
    for (int k = 0; k < kWindow; ++k) {
      cw[k] = make_uint4(0, 0, 0, 0);
      if (k < cnt) {
        const int64_t A = A0 + k;
        const int off = static_cast<int>(9 * ((A >> 2) - (A0 >> 2)) + 2 * (A & 3)) + shift0;
        const uint32_t v24 =
            (static_cast<uint32_t>(sb[off]) << 16) | (static_cast<uint32_t>(sb[off + 1]) << 8) | sb[off + 2];
        uint32_t idx = (v24 >> (6 - 2 * (A & 3))) & 0x3FFFFu;
        if (idx > static_cast<uint32_t>(kKissing)) {
          ++nbad;
          idx = 0;
        }
        cw[k] = __ldg(reinterpret_cast<const uint4 *>(a.codes) + idx);
      }
    }
    __syncthreads();  // every slot read before chunk writes reuse stage 1

    // 2. The window's chunks: no global loads from here on.
#pragma unroll
    for (int k = 0; k < kWindow; ++k) {
      const int c = w0 + k;
      if (c >= half) break;
      const int bf = i & 1;
      uint8_t *st = stages + bf * kAStage;
      // The MMAs of chunk i-2 read this stage: wait for their commit.
      if (i >= 2) bar_wait(&H.mma_done[bf], static_cast<uint32_t>((i - 2) >> 1) & 1u, abort, a.err);
      // A pieces: row `row`, k group j = 3h + p at j*2048 + row*16 (8-row
      // groups 128 bytes apart, k groups 2048 bytes apart).
      if (live) {
        uint4 *ah = reinterpret_cast<uint4 *>(st + (3 * h) * 2048 + row * 16);
        uint4 *al = reinterpret_cast<uint4 *>(st + kAPiece + (3 * h) * 2048 + row * 16);
        if (k < cnt) {
          constexpr uint32_t kSel = 0x76543210u;
          const uint4 cur = cw[k];
          const uint32_t l = ((cur.x >> 2) & 1u) | ((cur.x >> 5) & 2u);  // the codeword's value list
          const uint32_t h0 = l == 0 ? Lh[0] : (l == 1 ? Lh[2] : Lh[4]);
          const uint32_t h1 = l == 0 ? Lh[1] : (l == 1 ? Lh[3] : Lh[5]);
          const uint32_t q0 = l == 0 ? Ll[0] : (l == 1 ? Ll[2] : Ll[4]);
          const uint32_t q1 = l == 0 ? Ll[1] : (l == 1 ? Ll[3] : Ll[5]);
          const uint32_t words[3] = {cur.x, cur.y, cur.z};
#pragma unroll
          for (int p = 0; p < 3; ++p) {
            const uint32_t s_lo = __byte_perm(kSel, kSel, words[p]);
            const uint32_t s_hi = __byte_perm(kSel, kSel, words[p] >> 16);
            ah[p * 128] = expand8_pair(s_lo, s_hi, h0, h1);
            al[p * 128] = expand8_pair(s_lo, s_hi, q0, q1);
          }
        } else {
#pragma unroll
          for (int p = 0; p < 3; ++p) {
            ah[p * 128] = make_uint4(0, 0, 0, 0);
            al[p * 128] = make_uint4(0, 0, 0, 0);
          }
        }
      }
      // Generic-proxy writes become visible to the tensor core's async proxy.
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      __syncthreads();
      if (warp == 0 && __all_sync(0xffffffffu, *abort == 0)) {
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        const uint32_t abase = su32(st);
        const uint32_t bbase = su32(xtiles + static_cast<size_t>(c) * kXTile);
#pragma unroll
        for (int s = 0; s < 3; ++s) {
          const uint64_t bdesc = kmajor_desc(bbase + s * 512, 256, 128);
          lut_mma(tmem, kmajor_desc(abase + s * 4096, 2048, 128), bdesc, (i > 0 || s > 0) ? 1u : 0u);
          lut_mma(tmem, kmajor_desc(abase + kAPiece + s * 4096, 2048, 128), bdesc, 1u);
        }
        lut_commit(&H.mma_done[bf]);
      }
      ++i;
    }
  }
  // The last chunk's commit covers every MMA of the CTA; warps 0-3 read the
  // accumulator (warp w owns TMEM lanes 32w..32w+31).
  if (h == 0) {
    bar_wait(&H.mma_done[(i - 1) & 1], static_cast<uint32_t>((i - 1) >> 1) & 1u, abort, a.err);
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    float d[16];
    tmem_ld16(tmem + (static_cast<uint32_t>(warp * 32) << 16), d);
    if (live) {
      float *w = a.split == 1 ? a.y + o : a.ws + static_cast<int64_t>(rank) * kMaxB * a.rows + o;
#pragma unroll
      for (int b = 0; b < kMaxB; ++b)
        if (b < a.batch) w[b * a.rows] = d[b] + d[8 + b];
    }
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  if (warp == 0)
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemCols) : "memory");
  const unsigned total_bad = __reduce_add_sync(0xffffffffu, nbad);
  if ((t & 31) == 0 && total_bad && a.bad) atomicAdd(a.bad, static_cast<int32_t>(total_bad));
}

// y[i] = sum over slices s (in order) of ws[s][i], i = b * rows + o.
__global__ void __launch_bounds__(256) lut_reduce_kernel(const float *__restrict__ ws, int split, int64_t n,
                                                         int64_t slice_stride, float *__restrict__ y) {
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    float acc = ws[i];
    for (int q = 1; q < split; ++q) acc += ws[q * slice_stride + i];
    y[i] = acc;
  }
}

// ---------------------------------------------------------------------------
// Batches of 1-2 input rows: half a warp per weight row, fp32 FMAs.  W[o][i]
// is the fp16 value of materialize(), widened to fp32; the 16 lanes of a row
// take atoms a, a+16, a+32, ..., up to kFmaPre of them with their gathers in
// flight together: 18-bit index, one 16-byte code gather, 8 + 8 + 8 weights by
// byte permutes of the row's fp16 value lists, 24 FMAs per input row; then a
// 16-lane tree.  Two rows per warp (64 registers, four blocks per SM) let
// every row of a layer of up to ~9,400 rows be resident at once, so the whole
// layer's gathers are in flight in one wave.  With one or two input rows there are too few products per weight
// for the tensor-core path's staging to pay.
constexpr int kFmaThreads = 256;
constexpr int kFmaWarps = kFmaThreads / 32;
constexpr int kFmaRowsPerWarp = 2;
constexpr int kFmaPre = 5;  // atoms per lane whose gathers are issued together

template <int B>
__global__ void __launch_bounds__(kFmaThreads, 4) lut_fma_kernel(const uint8_t *__restrict__ packed,
                                                                 const uint16_t *__restrict__ sigma16,
                                                                 int64_t rows, int apr,
                                                                 const float *__restrict__ x, int64_t in_f,
                                                                 float *__restrict__ y,
                                                                 const uint32_t *__restrict__ codes,
                                                                 int32_t *__restrict__ bad) {
  pdl_enter();
  const int lane = threadIdx.x & 31;
  const int sl = lane & 15;        // lane within the row's half warp
  const int hb = lane & 16;        // first lane of the half
  const int64_t nrow_slots = static_cast<int64_t>(gridDim.x) * kFmaWarps * kFmaRowsPerWarp;
  constexpr uint32_t kSel = 0x76543210u;
  constexpr uint32_t kPairs = 0x82641735u;  // (lo, hi) raw pairs of words 0-3 of the value lists
  const int k6 = sl < 6 ? sl : 0;
  const uint32_t pair = k6 < 4 ? (kPairs >> (8 * k6)) & 0xFFu : (k6 == 4 ? 0x82u : 0x40u);
  unsigned nbad = 0;
  const int64_t first = (blockIdx.x * static_cast<int64_t>(kFmaWarps) + (threadIdx.x >> 5)) * kFmaRowsPerWarp +
                        (lane >> 4);
  // Every lane runs the same number of iterations (the shuffles below need
  // the whole warp); a half past the last row computes nothing it keeps.
  const int64_t iters = (rows + nrow_slots - 1) / nrow_slots;
  for (int64_t it = 0; it < iters; ++it) {
    const int64_t o = first + it * nrow_slots;
    const bool live = o < rows;
    // The row's fp16 value lists: lane k < 6 of the half builds word k, then
    // every lane of the half gets all six.
    const uint16_t sg = live ? __ldg(sigma16 + o) : static_cast<uint16_t>(0);
    const uint32_t mine = dequant_value(static_cast<int>(pair & 15u) - 4, sg) |
                          (static_cast<uint32_t>(dequant_value(static_cast<int>(pair >> 4) - 4, sg)) << 16);
    uint32_t L[6];
#pragma unroll
    for (int k = 0; k < 6; ++k) L[k] = __shfl_sync(0xffffffffu, mine, hb + k);
    float acc[B];
#pragma unroll
    for (int b = 0; b < B; ++b) acc[b] = 0.f;
    for (int a0 = 0; a0 < apr; a0 += 16 * kFmaPre) {
      uint4 cw[kFmaPre];
#pragma unroll
      for (int j = 0; j < kFmaPre; ++j) {
        const int a = a0 + sl + 16 * j;
        cw[j] = make_uint4(0, 0, 0, 0);
        if (live && a < apr) {
          const int64_t A = o * apr + a;
          const uint8_t *p = packed + 9 * (A >> 2) + 2 * (A & 3);
          const uint32_t v24 =
              (static_cast<uint32_t>(__ldg(p)) << 16) | (static_cast<uint32_t>(__ldg(p + 1)) << 8) | __ldg(p + 2);
          uint32_t idx = (v24 >> (6 - 2 * (A & 3))) & 0x3FFFFu;
          if (idx > static_cast<uint32_t>(kKissing)) {
            ++nbad;
            idx = 0;
          }
          cw[j] = __ldg(reinterpret_cast<const uint4 *>(codes) + idx);
        }
      }
#pragma unroll
      for (int j = 0; j < kFmaPre; ++j) {
        const int a = a0 + sl + 16 * j;
        if (!live || a >= apr) continue;
        const uint32_t words[3] = {cw[j].x, cw[j].y, cw[j].z};
        const uint32_t l = ((cw[j].x >> 2) & 1u) | ((cw[j].x >> 5) & 2u);  // the codeword's value list
        const uint32_t s0 = l == 0 ? L[0] : (l == 1 ? L[2] : L[4]);
        const uint32_t s1 = l == 0 ? L[1] : (l == 1 ? L[3] : L[5]);
#pragma unroll
        for (int part = 0; part < 3; ++part) {
          const uint32_t w = words[part];
          const uint32_t s_lo = __byte_perm(kSel, kSel, w), s_hi = __byte_perm(kSel, kSel, w >> 16);
          const uint32_t hv[4] = {__byte_perm(s0, s1, s_lo), __byte_perm(s0, s1, s_lo >> 16),
                                  __byte_perm(s0, s1, s_hi), __byte_perm(s0, s1, s_hi >> 16)};
          float wf[8];
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const float2 f = __half22float2(*reinterpret_cast<const __half2 *>(&hv[e]));
            wf[2 * e] = f.x;
            wf[2 * e + 1] = f.y;
          }
          const int64_t col = static_cast<int64_t>(a) * kDim + 8 * part;
#pragma unroll
          for (int b = 0; b < B; ++b) {
            const float4 x0 = __ldg(reinterpret_cast<const float4 *>(x + b * in_f + col));
            const float4 x1 = __ldg(reinterpret_cast<const float4 *>(x + b * in_f + col + 4));
            acc[b] = fmaf(x0.x, wf[0], acc[b]);
            acc[b] = fmaf(x0.y, wf[1], acc[b]);
            acc[b] = fmaf(x0.z, wf[2], acc[b]);
            acc[b] = fmaf(x0.w, wf[3], acc[b]);
            acc[b] = fmaf(x1.x, wf[4], acc[b]);
            acc[b] = fmaf(x1.y, wf[5], acc[b]);
            acc[b] = fmaf(x1.z, wf[6], acc[b]);
            acc[b] = fmaf(x1.w, wf[7], acc[b]);
          }
        }
      }
    }
#pragma unroll
    for (int b = 0; b < B; ++b) {
#pragma unroll
      for (int off = 8; off > 0; off >>= 1) acc[b] += __shfl_xor_sync(0xffffffffu, acc[b], off);
      if (sl == 0 && live) y[b * rows + o] = acc[b];
    }
  }
  const unsigned total_bad = __reduce_add_sync(0xffffffffu, nbad);
  if (lane == 0 && total_bad && bad) atomicAdd(bad, static_cast<int32_t>(total_bad));
}

// CTAs of lut_tc_kernel with `smem` bytes of dynamic shared memory that one
// SM holds, from shared memory, registers and threads (the occupancy API
// answers 1 for this kernel); more CTAs than fit would only queue.
int lut_ctas_per_sm(int dev, size_t smem) {
  int smem_sm = 0, reserved = 0;
  cudaDeviceGetAttribute(&smem_sm, cudaDevAttrMaxSharedMemoryPerMultiprocessor, dev);
  cudaDeviceGetAttribute(&reserved, cudaDevAttrReservedSharedMemoryPerBlock, dev);
  cudaFuncAttributes fa;
  if (cudaFuncGetAttributes(&fa, lut_tc_kernel) != cudaSuccess) return 1;
  const int by_smem = smem_sm / static_cast<int>(smem + reserved);
  const int by_regs = 65536 / (((fa.numRegs * 32 + 255) / 256) * 256 * (kLutThreads / 32));
  int per = by_smem < by_regs ? by_smem : by_regs;
  per = per < 2048 / kLutThreads ? per : 2048 / kLutThreads;
  return per > 0 ? per : 1;
}

}  // namespace

int launch_lut_gemv(const Tables *t, const uint8_t *packed, const uint16_t *sigma16, int64_t rows,
                    int64_t in_f, const float *x, int64_t batch, float *y, int32_t *bad,
                    cudaStream_t s) {
  if (rows < 0 || in_f <= 0 || in_f % kDim != 0 || batch < 0)
    return fail(H24_ERR_INVALID, "lut_gemv: in_features must be a positive multiple of 24");
  if (rows == 0 || batch == 0) return H24_OK;
  if (!packed || !sigma16 || !x || !y) return fail(H24_ERR_INVALID, "lut_gemv: null pointer");
  if (!aligned16(x)) return fail(H24_ERR_INVALID, "lut_gemv: x must be 16-byte aligned");
  if (in_f / kDim > (int64_t(1) << 30)) return fail(H24_ERR_INVALID, "lut_gemv: in_features too large");
  int dev = 0, sms = 148;
  H24_CUDA_TRY(cudaGetDevice(&dev));
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const int apr = static_cast<int>(in_f / kDim);
  const int64_t mtiles = (rows + kTileRows - 1) / kTileRows;
  // Split each tile's atoms over `split` CTAs (at most 8, each with at least
  // one atom): the largest split whose CTAs are all resident at once.  The
  // B tiles of a slice's chunks live in shared memory, so fewer fit per SM
  // when the slices are long.
  int split = 1;
  size_t smem = lut_smem_bytes((apr + 1) / 2);
  for (int cand = kMaxSplit; cand >= 1; cand >>= 1) {
    if (cand > apr) continue;
    const int chunks = ((apr + cand - 1) / cand + 1) / 2;  // chunks of the longest slice
    const size_t need = lut_smem_bytes(chunks);
    if (need > 227 * 1024) continue;
    const int64_t resident = static_cast<int64_t>(sms) * lut_ctas_per_sm(dev, need);
    if (mtiles * cand <= resident || cand == 1) {
      split = cand;
      smem = need;
      break;
    }
  }
  if (smem > 227 * 1024) return fail(H24_ERR_INVALID, "lut_gemv: in_features too large for the LUT GEMV");
  H24_CUDA_TRY(cudaFuncSetAttribute(lut_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem)));
  H24_CUDA_TRY(cudaFuncSetAttribute(lut_tc_kernel, cudaFuncAttributePreferredSharedMemoryCarveout,
                                    cudaSharedmemCarveoutMaxShared));
  float *ws = nullptr;
  if (split > 1)
    H24_CUDA_TRY(cudaMallocFromPoolAsync(reinterpret_cast<void **>(&ws),
                                         static_cast<size_t>(split) * kMaxB * rows * sizeof(float), t->pool, s));
  int rc = H24_OK;
  for (int64_t b0 = 0; b0 < batch && rc == H24_OK; b0 += kMaxB) {
    const int nb = static_cast<int>(batch - b0 < kMaxB ? batch - b0 : kMaxB);
    if (nb <= 2) {
      const int64_t per_block = static_cast<int64_t>(kFmaWarps) * kFmaRowsPerWarp;
      const int grid = wave_grid((rows + per_block - 1) / per_block,
                                 nb == 1 ? blocks_per_sm(lut_fma_kernel<1>, kFmaThreads, 0)
                                         : blocks_per_sm(lut_fma_kernel<2>, kFmaThreads, 0));
      // Programmatic dependent launch (pdl_enter): consecutive layers' GEMVs
      // launch while the previous one finishes.
      const cudaError_t e =
          nb == 1 ? launch_pdl(lut_fma_kernel<1>, dim3(grid), dim3(kFmaThreads), s, packed, sigma16, rows, apr,
                               x + b0 * in_f, in_f, y + b0 * rows, t->cb_nib, bad)
                  : launch_pdl(lut_fma_kernel<2>, dim3(grid), dim3(kFmaThreads), s, packed, sigma16, rows, apr,
                               x + b0 * in_f, in_f, y + b0 * rows, t->cb_nib, bad);
      count_launches(1);
      if (e != cudaSuccess) rc = cuda_fail(e, "lut_gemv launch");
      continue;
    }
    LutArgs args;
    args.packed = packed;
    args.sigma16 = sigma16;
    args.x = x + b0 * in_f;
    args.y = y + b0 * rows;
    args.ws = ws;
    args.codes = t->cb_nib;
    args.bad = bad;
    args.err = t->err;
    args.rows = rows;
    args.in_f = in_f;
    args.apr = apr;
    args.batch = static_cast<int>(batch - b0 < kMaxB ? batch - b0 : kMaxB);
    args.split = split;
    lut_tc_kernel<<<static_cast<unsigned>(mtiles * split), kLutThreads, smem, s>>>(args);
    cudaError_t e = cudaGetLastError();
    count_launches(1);
    if (e == cudaSuccess && split > 1) {
      const int64_t n = static_cast<int64_t>(args.batch) * rows;
      lut_reduce_kernel<<<wave_grid((n + 255) / 256, 8), 256, 0, s>>>(ws, split, n,
                                                                       static_cast<int64_t>(kMaxB) * rows, args.y);
      e = cudaGetLastError();
      count_launches(1);
    }
    if (e != cudaSuccess) rc = cuda_fail(e, "lut_gemv launch");
  }
  if (ws) {
    const cudaError_t e = cudaFreeAsync(ws, s);
    if (rc == H24_OK && e != cudaSuccess) rc = cuda_fail(e, "cudaFreeAsync");
  }
  return rc;
}

}  // namespace h24
