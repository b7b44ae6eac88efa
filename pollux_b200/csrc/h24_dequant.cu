// h24_dequant.cu -- LUT dequantisation of packed H24 layers (pollux.py:485-500)
// and the codeword gather of castor_quantize_leech's output (castor.py:533).
// The matrix-free LUT GEMV over the same code table is in h24_lut.cu.
//
// Dequant: every weight element of row r takes one of nine fp16 values,
//   F(v, r) = fp16( fp32( fp16(cb16[v] * sigma16[r]) ) * 0.70710677f ),
// where v is the raw Leech coordinate (-4..4) of the element's codeword and
// cb16[v] = fp16(v * fp32(1/sqrt(8))).  Both roundings of the reference are
// reproduced, so the result is bit-identical given the same indices and
// scales.
//
// The 48-byte fp16 output of an atom (1.5 sectors) and its one code-entry
// gather (one sector) pass each SM's L1-to-crossbar interface, which moves a
// sector per cycle and bounds the kernel (80 % busy).  A codeword holds
// at most four distinct coordinates, fixed by its type, so the codebook is
// stored as 2-bit positions in a per-type value list (16 bytes per codeword,
// one 32-byte sector, 3.1 MB, L2-resident) and two output values come from
// one byte permute (prmt) of the row's values for that list: per atom one
// 16-byte gather of its code entry (staged in shared memory), per 8 elements
// six prmt and one 16-byte store.  Each warp owns an equal contiguous range
// of atoms (one resident wave, no block barriers) and walks it in sub-tiles
// of up to 128 atoms, loading the next sub-tile's packed bytes while it
// expands the current one; output unit u (8 elements) of a sub-tile goes to
// lane u mod 32, so every store instruction writes 512 contiguous bytes (four
// whole 128-byte lines when the output is 128-byte aligned).  The per-row
// value lists live in an 8-row shared-memory ring.
#include <cstddef>

#include "h24_internal.cuh"

namespace h24 {
namespace {

constexpr int kThreads = 256;
constexpr int kWarpsPerBlock = kThreads / 32;
constexpr int kSub = 128;        // atoms per sub-tile
constexpr int kSlots = 8;        // rows in the per-warp value-list ring
constexpr int kMaxBatch = 64;    // keeps the kernel parameter block under 4 KB

struct DequantBatch {
  h24_dequant_layer layer[kMaxBatch];
  int64_t atom_start[kMaxBatch + 1];  // atoms before each layer
  int count;
};

// Per-warp shared memory: the sub-tile's packed bytes, the code words and
// value-list offsets of its atoms and the value lists of up to 8 rows.
constexpr int kPackedChunks = 20;  // 16-byte chunks: <= 297 bytes from a 16-byte-aligned start
struct WarpSmem {
  alignas(16) uint32_t lists[kSlots][8];  // [slot][2*list .. 2*list+1] = a prmt source pair
  alignas(16) uint8_t packed[16 * kPackedChunks];
  uint32_t code[3 * kSub];                // code words of atom a at 3a .. 3a+2
  uint8_t lofs[kSub];                     // list_offset() of atom a
};
static_assert(offsetof(WarpSmem, lists) % 8 == 0 && offsetof(WarpSmem, packed) % 16 == 0 &&
                  sizeof(WarpSmem) % 16 == 0,
              "value lists are read as 8-byte pairs, packed bytes stored as 16-byte chunks");

// Value lists of rows r_lo..r_hi (at most kSlots) into their ring slots, the
// code orders of h24_capi.cu's table:
//   list 0 {+1,-1,+3,-3}, list 1 {0,+2,-2,+4}, list 2 {-2,+4,-4,0},
// stored as six words of two fp16 values (one prmt source pair per list).
// Lane 8j+k computes word k of row r_lo+j, so 4 rows take one pass.
__device__ __forceinline__ void build_lists(uint32_t (*lists)[8], const uint16_t *sigma16,
                                            int64_t r_lo, int64_t r_hi, int lane) {
  const int k = lane & 7;
  // (lo, hi) raw coordinates of word k, packed as nibbles lo+4 | (hi+4) << 4.
  constexpr uint32_t kPairs = 0x82641735u;  // words 0-3: (1,-1) (3,-3) (0,2) (-2,4)
  const uint32_t pair = k < 4 ? (kPairs >> (8 * k)) & 0xFFu : (k == 4 ? 0x82u : 0x40u);  // (-2,4) (-4,0)
  for (int64_t r = r_lo + (lane >> 3); r <= r_hi; r += 4) {
    if (k < 6) {
      const uint16_t sg = __ldg(sigma16 + r);
      const uint32_t lo = dequant_value(static_cast<int>(pair & 15u) - 4, sg);
      const uint32_t hi = dequant_value(static_cast<int>(pair >> 4) - 4, sg);
      lists[r & (kSlots - 1)][k] = lo | (hi << 16);
    }
  }
}

// Byte offset in a warp's value-list ring of the prmt source pair that the
// code words of a codeword use: its row's ring slot and its list (bit 2 of
// nibbles 0 and 1 of every word of its entry).
__device__ __forceinline__ uint32_t list_offset(uint32_t slot, uint32_t w) {
  return 32u * slot + 8u * (((w >> 2) & 1u) | ((w >> 5) & 2u));
}

// 8 fp16 outputs from one code word (nibble e -> element e) and the row's
// value list for the word's codeword type.
__device__ __forceinline__ uint4 expand8(uint32_t w, uint2 src) {
  // Code c -> the prmt selector pair (2c, 2c+1) of fp16 value c; the list bit
  // (bit 2) only selects the identical upper copy of the table.
  constexpr uint32_t kSel = 0x76543210u;
  const uint32_t s_lo = __byte_perm(kSel, kSel, w);
  const uint32_t s_hi = __byte_perm(kSel, kSel, w >> 16);
  uint4 o;
  o.x = __byte_perm(src.x, src.y, s_lo);
  o.y = __byte_perm(src.x, src.y, s_lo >> 16);
  o.z = __byte_perm(src.x, src.y, s_hi);
  o.w = __byte_perm(src.x, src.y, s_hi >> 16);
  return o;
}

// Where a sub-tile's packed bytes lie: `chunks` 16-byte chunks from the
// aligned address `base`, the first byte of group la0/4 at offset `shift`.
// Every chunk read holds at least one byte of the stream, so it lies in
// mapped memory even where the stream is an unaligned view.
struct PackedSpan {
  const uint4 *base;
  int shift, chunks;
};

__device__ __forceinline__ PackedSpan packed_span(const uint8_t *packed, int64_t la0, int na) {
  const int nbytes = 9 * ((static_cast<int>(la0 & 3) + na - 1) / 4 + 1);
  const uint8_t *src = packed + 9 * (la0 >> 2);
  const uintptr_t a = reinterpret_cast<uintptr_t>(src) & ~static_cast<uintptr_t>(15);
  PackedSpan p;
  p.base = reinterpret_cast<const uint4 *>(a);
  p.shift = static_cast<int>(reinterpret_cast<uintptr_t>(src) - a);
  p.chunks = (p.shift + nbytes + 15) / 16;
  return p;
}

// x / d for the in-row positions x < d + kSub of a sub-tile, by one
// multiply-high: with m = ceil(2^32 / d) and e = m d - 2^32 < d,
// floor(x m / 2^32) = floor(x / d) whenever x e < 2^32, which holds for
// d <= 65,000 ((d + 127)(d - 1) < 2^32); longer rows divide.
struct RowDiv {
  uint64_t m;
  uint32_t d;
  __device__ __forceinline__ explicit RowDiv(uint32_t d_) : m(((1ull << 32) + d_ - 1) / d_), d(d_) {}
  __device__ __forceinline__ uint32_t operator()(uint32_t x) const {
    return d <= 65000u ? static_cast<uint32_t>((x * m) >> 32) : x / d;
  }
};

// Atoms of the sub-tile that starts at global atom g inside layer li: at most
// kSub, within the layer and the warp's range, and over at most 8 rows (so the
// value lists fit the ring); a row-limited length is a multiple of 8 atoms so
// that the output stays 128-byte aligned.
__device__ __forceinline__ int sub_atoms(const DequantBatch &b, int li, int64_t g, int64_t g_end,
                                         int32_t apr) {
  int64_t lim = b.atom_start[li + 1] - g;
  if (g_end - g < lim) lim = g_end - g;
  int64_t rows7 = 7 * static_cast<int64_t>(apr);
  if (rows7 >= 8) rows7 &= ~static_cast<int64_t>(7);
  if (rows7 < lim) lim = rows7;
  return static_cast<int>(lim < kSub ? lim : kSub);
}

__global__ void __launch_bounds__(kThreads, 4) dequant_kernel(const __grid_constant__ DequantBatch b,
                                                           const uint4 *__restrict__ codes,
                                                           int32_t *__restrict__ bad) {
  __shared__ WarpSmem smem[kWarpsPerBlock];
  pdl_enter();
  const int lane = threadIdx.x & 31;
  WarpSmem &W = smem[threadIdx.x >> 5];
  const int64_t total = b.atom_start[b.count];
  const int64_t nwarps = static_cast<int64_t>(gridDim.x) * kWarpsPerBlock;
  const int64_t wid = blockIdx.x * static_cast<int64_t>(kWarpsPerBlock) + (threadIdx.x >> 5);
  // Warp ranges are multiples of 32 atoms (1536 output bytes), so sub-tiles
  // start 128-byte aligned in every layer whose atom count is a multiple of 8.
  const int64_t per = ((total + nwarps - 1) / nwarps + 31) & ~static_cast<int64_t>(31);
  const int64_t g_begin = wid * per < total ? wid * per : total;
  const int64_t g_end = g_begin + per < total ? g_begin + per : total;
  if (g_begin >= g_end) return;

  int li = 0;
  while (b.atom_start[li + 1] <= g_begin) ++li;
  int32_t apr = static_cast<int32_t>(b.layer[li].in_features / kDim);
  int64_t row = (g_begin - b.atom_start[li]) / apr;  // row of the sub-tile's first atom
  int32_t off = static_cast<int32_t>(g_begin - b.atom_start[li] - row * apr);  // its position in the row
  int64_t built_hi = row - 1;
  RowDiv rdiv(static_cast<uint32_t>(apr));
  int na = sub_atoms(b, li, g_begin, g_end, apr);
  PackedSpan span = packed_span(b.layer[li].packed, g_begin - b.atom_start[li], na);
  uint4 pk = make_uint4(0, 0, 0, 0);
  if (lane < span.chunks) pk = __ldcs(span.base + lane);
  unsigned nbad = 0;

  for (int64_t g = g_begin; g < g_end;) {
    const h24_dequant_layer &L = b.layer[li];
    const int64_t la0 = g - b.atom_start[li];
    const int64_t r1 = row + rdiv(static_cast<uint32_t>(off + na - 1));
    // 1. This sub-tile's packed bytes (loaded during the previous sub-tile).
    if (lane < kPackedChunks) reinterpret_cast<uint4 *>(W.packed)[lane] = pk;
    // 2. Value lists of rows not yet in the ring.
    if (r1 > built_hi) {
      build_lists(W.lists, L.sigma16, built_hi + 1 > row ? built_hi + 1 : row, r1, lane);
      built_hi = r1;
    }
    __syncwarp();
    // 3. 18-bit index, code words and value-list offset of each atom: one
    //    16-byte gather (one 32-byte sector) per atom.
    const int q0 = static_cast<int>(la0 & 3);
#pragma unroll
    for (int k = 0; k < kSub / 32; ++k) {
      const int a = lane + 32 * k;
      if (a < na) {
        const int sa = q0 + a, q = sa & 3;
        const uint8_t *p = W.packed + span.shift + 9 * (sa >> 2) + 2 * q;
        const uint32_t v24 = (static_cast<uint32_t>(p[0]) << 16) | (static_cast<uint32_t>(p[1]) << 8) | p[2];
        uint32_t idx = (v24 >> (6 - 2 * q)) & 0x3FFFFu;
        if (idx > static_cast<uint32_t>(kKissing)) {
          ++nbad;
          idx = 0;
        }
        const uint4 c = __ldg(codes + idx);
        W.code[3 * a] = c.x;
        W.code[3 * a + 1] = c.y;
        W.code[3 * a + 2] = c.z;
        const uint32_t rl = rdiv(static_cast<uint32_t>(off + a));
        W.lofs[a] = static_cast<uint8_t>(list_offset(static_cast<uint32_t>((row + rl) & (kSlots - 1)), c.x));
      }
    }
    uint4 *dst = reinterpret_cast<uint4 *>(L.out16 + la0 * kDim);
    const int units = 3 * na;
    // Advance to the next sub-tile and start loading its packed bytes.
    g += na;
    off += na;
    if (off >= apr) {
      const int32_t dr = static_cast<int32_t>(rdiv(static_cast<uint32_t>(off)));
      row += dr;
      off -= dr * apr;
    }
    if (g < g_end) {
      if (b.atom_start[li + 1] <= g) {  // entering a layer (its first atom)
        while (b.atom_start[li + 1] <= g) ++li;
        apr = static_cast<int32_t>(b.layer[li].in_features / kDim);
        rdiv = RowDiv(static_cast<uint32_t>(apr));
        row = 0;
        off = 0;
        built_hi = -1;
      }
      na = sub_atoms(b, li, g, g_end, apr);
      span = packed_span(b.layer[li].packed, g - b.atom_start[li], na);
      if (lane < span.chunks) pk = __ldcs(span.base + lane);
    }
    __syncwarp();
    // 4. Output unit u (8 elements, 16 bytes) of the sub-tile goes to lane
    //    u mod 32: every store instruction writes 512 contiguous bytes.
#pragma unroll
    for (int m = 0; m < 3 * kSub / 32; ++m) {
      const int u = 32 * m + lane;
      if (u < units)
        __stcs(dst + u, expand8(W.code[u], *reinterpret_cast<const uint2 *>(
                                               reinterpret_cast<const uint8_t *>(W.lists) + W.lofs[u / 3])));
    }
    __syncwarp();
  }
  const unsigned total_bad = __reduce_add_sync(0xffffffffu, nbad);
  if (lane == 0 && total_bad && bad) atomicAdd(bad, static_cast<int32_t>(total_bad));
}

template <typename T>
__device__ __forceinline__ T convert_value(float v);
template <>
__device__ __forceinline__ float convert_value<float>(float v) { return v; }
template <>
__device__ __forceinline__ __half convert_value<__half>(float v) { return __float2half_rn(v); }
template <>
__device__ __forceinline__ __nv_bfloat16 convert_value<__nv_bfloat16>(float v) {
  return __float2bfloat16_rn(v);
}

template <typename T>
__global__ void gather_kernel(const int32_t *__restrict__ idx, int64_t n,
                              const int8_t *__restrict__ cb_raw, T *__restrict__ out) {
  const int64_t total = n * 3;  // 8 elements per work item
  for (int64_t w = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; w < total;
       w += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t a = w / 3;
    const int part = static_cast<int>(w - 3 * a);
    const int32_t k = idx[a];
    T vals[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      const int raw = (k >= 1 && k <= kKissing)
                          ? cb_raw[static_cast<int64_t>(k - 1) * kDim + part * 8 + e]
                          : 0;
      vals[e] = convert_value<T>(static_cast<float>(raw) * kLeechScaleF);
    }
#pragma unroll
    for (int e = 0; e < 8; ++e) out[a * kDim + part * 8 + e] = vals[e];
  }
}

__global__ void codebook_f32_kernel(const int8_t *__restrict__ cb_raw, float *__restrict__ out) {
  const int64_t total = static_cast<int64_t>(kKissing) * kDim;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x)
    out[i] = static_cast<float>(cb_raw[i]) * kLeechScaleF;
}

int sm_count() {
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  return sms;
}

// Blocks of dequant_kernel resident per SM (same on every device of a run).
int resident_blocks() {
  static const int n = [] {
    int v = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&v, dequant_kernel, kThreads, 0) != cudaSuccess ||
        v < 1)
      v = 4;
    return v;
  }();
  return n;
}

}  // namespace

int launch_dequant(const Tables *t, const h24_dequant_layer * /*layers_dev*/,
                   const h24_dequant_layer *layers, int count, int32_t *bad, cudaStream_t s) {
  for (int base = 0; base < count; base += kMaxBatch) {
    DequantBatch b;
    b.count = 0;
    b.atom_start[0] = 0;
    for (int i = base; i < count && b.count < kMaxBatch; ++i) {
      const h24_dequant_layer &L = layers[i];
      if (L.rows < 0 || L.in_features <= 0 || L.in_features % kDim != 0)
        return fail(H24_ERR_INVALID, "dequant: in_features must be a positive multiple of 24");
      if (L.rows == 0) continue;
      if (!L.packed || !L.sigma16 || !L.out16)
        return fail(H24_ERR_INVALID, "dequant: null pointer");
      if (!aligned16(L.out16))
        return fail(H24_ERR_INVALID, "dequant: out16 must be 16-byte aligned");
      b.layer[b.count] = L;
      b.atom_start[b.count + 1] = b.atom_start[b.count] + L.rows * (L.in_features / kDim);
      ++b.count;
    }
    if (b.count == 0) continue;
    // One resident wave; every warp gets at least one full sub-tile.
    const int64_t atoms = b.atom_start[b.count];
    const int64_t want = (atoms + kSub * kWarpsPerBlock - 1) / (kSub * kWarpsPerBlock);
    const int64_t cap = static_cast<int64_t>(sm_count()) * resident_blocks();
    const int grid = static_cast<int>(want < cap ? want : cap);
    // Programmatic dependent launch (pdl_enter): the launch overlaps the
    // tail of the kernel before it.
    H24_CUDA_TRY(launch_pdl(dequant_kernel, dim3(grid), dim3(kThreads), s, b,
                            reinterpret_cast<const uint4 *>(t->cb_nib), bad));
    count_launches(1);
  }
  return H24_OK;
}

int launch_codebook_f32(const Tables *t, float *out_kissing, cudaStream_t s) {
  codebook_f32_kernel<<<sm_count() * 4, 256, 0, s>>>(t->cb_raw, out_kissing);
  H24_CUDA_TRY(cudaGetLastError());
  count_launches(1);
  return H24_OK;
}

int launch_gather(const Tables *t, const int32_t *idx, int64_t n, int dtype, void *out,
                  cudaStream_t s) {
  if (n <= 0) return H24_OK;
  const int64_t items = n * 3;
  const int threads = 256;
  const int64_t want = (items + threads - 1) / threads;
  const int64_t cap = static_cast<int64_t>(sm_count()) * 16;
  const int grid = static_cast<int>(want < cap ? want : cap);
  switch (dtype) {
    case H24_DTYPE_F32:
      gather_kernel<float><<<grid, threads, 0, s>>>(idx, n, t->cb_raw, static_cast<float *>(out));
      break;
    case H24_DTYPE_F16:
      gather_kernel<__half><<<grid, threads, 0, s>>>(idx, n, t->cb_raw, static_cast<__half *>(out));
      break;
    case H24_DTYPE_BF16:
      gather_kernel<__nv_bfloat16>
          <<<grid, threads, 0, s>>>(idx, n, t->cb_raw, static_cast<__nv_bfloat16 *>(out));
      break;
    default:
      return fail(H24_ERR_INVALID, "gather: unknown dtype");
  }
  H24_CUDA_TRY(cudaGetLastError());
  count_launches(1);
  return H24_OK;
}

}  // namespace h24
