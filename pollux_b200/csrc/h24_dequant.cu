// h24_dequant.cu -- LUT dequantisation of packed H24 layers (pollux.py:485-500)
// and the codeword gather of castor_quantize_leech's output (castor.py:533).
//
// Dequant: every weight element of row r takes one of nine fp16 values,
//   F(v, r) = fp16( fp32( fp16(cb16[v] * sigma16[r]) ) * 0.70710677f ),
// where v is the raw Leech coordinate (-4..4) of the element's codeword and
// cb16[v] = fp16(v * fp32(1/sqrt(8))).  Both roundings of the reference are
// reproduced, so the result is bit-identical given the same indices and
// scales.  The codebook is read as 4-bit codes (12 bytes per codeword, 2.4 MB,
// L2-resident); the per-row values live in a shared-memory LUT built once per
// tile.  The kernel is bound by the 48-byte fp16 output per atom: each warp
// writes its 32 atoms (1536 bytes) as three fully coalesced 512-byte stores.
#include "h24_internal.cuh"

namespace h24 {
namespace {

constexpr int kThreads = 256;
constexpr int kTileAtoms = kThreads;  // one atom per thread and tile
constexpr int kMaxBatch = 64;  // keeps the kernel parameter block under 4 KB

struct DequantBatch {
  h24_dequant_layer layer[kMaxBatch];
  int64_t tile_start[kMaxBatch + 1];
  int count;
};

__device__ __forceinline__ uint16_t dequant_value(int raw, uint16_t sigma_bits) {
  const __half cb = __float2half_rn(static_cast<float>(raw) * kLeechScaleF);
  const __half sg = __ushort_as_half(sigma_bits);
  const __half t = __float2half_rn(__half2float(cb) * __half2float(sg));
  const __half w = __float2half_rn(__half2float(t) * kSLatticeF);
  return __half_as_ushort(w);
}

__global__ void __launch_bounds__(kThreads) dequant_kernel(const __grid_constant__ DequantBatch b,
                                                           const uint32_t *__restrict__ cb_nib,
                                                           int32_t *__restrict__ bad) {
  __shared__ uint16_t lut[kTileAtoms][16];
  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  const int64_t total = b.tile_start[b.count];
  for (int64_t tile = blockIdx.x; tile < total; tile += gridDim.x) {
    int li = 0;
    while (li + 1 < b.count && b.tile_start[li + 1] <= tile) ++li;
    const h24_dequant_layer L = b.layer[li];
    const int64_t apr = L.in_features / kDim;
    const int64_t atoms = L.rows * apr;
    const int64_t a0 = (tile - b.tile_start[li]) * kTileAtoms;
    const int64_t a_last = (a0 + kTileAtoms < atoms ? a0 + kTileAtoms : atoms) - 1;
    const int64_t r_first = a0 / apr;
    const int nrows = static_cast<int>(a_last / apr - r_first + 1);

    // Per-row LUT: lut[row - r_first][raw + 4].
    for (int e = threadIdx.x; e < nrows * 9; e += kThreads) {
      const int rl = e / 9, code = e - rl * 9;
      lut[rl][code] = dequant_value(code - 4, L.sigma16[r_first + rl]);
    }
    __syncthreads();

    // Each lane decodes the index of its own atom.
    const int64_t wa0 = a0 + warp * 32;
    const int64_t atom = wa0 + lane;
    uint32_t info = 0;
    bool bad_idx = false;
    if (atom < atoms) {
      const int64_t g = atom >> 2;
      const int k = static_cast<int>(atom & 3);
      const uint8_t *p = L.packed + 9 * g + 2 * k;
      const uint32_t v24 = (static_cast<uint32_t>(__ldg(p)) << 16) |
                           (static_cast<uint32_t>(__ldg(p + 1)) << 8) | __ldg(p + 2);
      uint32_t idx = (v24 >> (6 - 2 * k)) & 0x3FFFFu;
      if (idx > static_cast<uint32_t>(kKissing)) {
        bad_idx = true;
        idx = 0;
      }
      const uint32_t rl = static_cast<uint32_t>(atom / apr - r_first);
      info = idx | (rl << 18);
    }
    const unsigned nbad = __popc(__ballot_sync(0xffffffffu, bad_idx));
    if (lane == 0 && nbad && bad) atomicAdd(bad, static_cast<int32_t>(nbad));

    // 32 atoms x 48 bytes = 96 uint4 per warp; lane writes uint4 lane+32j.
#pragma unroll
    for (int j = 0; j < 3; ++j) {
      const int v = lane + 32 * j;
      const int src = v / 3;
      const int part = v - 3 * src;
      const uint32_t inf = __shfl_sync(0xffffffffu, info, src);
      if (wa0 + src < atoms) {
        const uint32_t idx = inf & 0x3FFFFu;
        const uint16_t *row = lut[inf >> 18];
        const uint32_t word = __ldg(cb_nib + 3 * idx + part);
        uint32_t o[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const uint32_t lo = row[(word >> (8 * e)) & 0xF];
          const uint32_t hi = row[(word >> (8 * e + 4)) & 0xF];
          o[e] = lo | (hi << 16);
        }
        uint4 *dst = reinterpret_cast<uint4 *>(L.out16 + (wa0 + src) * kDim + part * 8);
        __stcs(dst, make_uint4(o[0], o[1], o[2], o[3]));
      }
    }
    __syncthreads();
  }
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

}  // namespace

int launch_dequant(const Tables *t, const h24_dequant_layer * /*layers_dev*/,
                   const h24_dequant_layer *layers, int count, int32_t *bad, cudaStream_t s) {
  for (int base = 0; base < count; base += kMaxBatch) {
    DequantBatch b;
    b.count = 0;
    b.tile_start[0] = 0;
    for (int i = base; i < count && b.count < kMaxBatch; ++i) {
      const h24_dequant_layer &L = layers[i];
      if (L.rows < 0 || L.in_features <= 0 || L.in_features % kDim != 0)
        return fail(H24_ERR_INVALID, "dequant: in_features must be a positive multiple of 24");
      if (L.rows == 0) continue;
      if (!L.packed || !L.sigma16 || !L.out16)
        return fail(H24_ERR_INVALID, "dequant: null pointer");
      if (!aligned16(L.out16))
        return fail(H24_ERR_INVALID, "dequant: out16 must be 16-byte aligned");
      const int64_t atoms = L.rows * (L.in_features / kDim);
      b.layer[b.count] = L;
      b.tile_start[b.count + 1] = b.tile_start[b.count] + (atoms + kTileAtoms - 1) / kTileAtoms;
      ++b.count;
    }
    if (b.count == 0) continue;
    const int64_t tiles = b.tile_start[b.count];
    const int64_t cap = static_cast<int64_t>(sm_count()) * 8;
    const int grid = static_cast<int>(tiles < cap ? tiles : cap);
    dequant_kernel<<<grid, kThreads, 0, s>>>(b, t->cb_nib, bad);
    H24_CUDA_TRY(cudaGetLastError());
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
