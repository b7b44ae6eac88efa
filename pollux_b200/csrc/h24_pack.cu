// h24_pack.cu -- 18-bit index pack / unpack (castor.py:226-260).
//
// Format: indices are taken four at a time (i0,i1,i2,i3); the 9 output bytes
// are the big-endian 72-bit integer i0<<54 | i1<<36 | i2<<18 | i3, each index
// first truncated to 32 bits and then masked to 18 bits by the byte formulas.
//
// Both kernels move a tile of 1024 groups (4096 indices, 9216 packed bytes)
// per block iteration.  The packed side of a tile is staged in shared memory
// so that global traffic on both sides is 16-byte vectors: the packed stream
// has no 16-byte structure of its own (9-byte groups), the index stream does.
// HBM-bound: 4 + 2.25 bytes per index (int32 side).
#include "h24_internal.cuh"

namespace h24 {
namespace {

constexpr int kThreads = 256;
constexpr int kGroupsPerThread = 4;
constexpr int kTileGroups = kThreads * kGroupsPerThread;  // 1024
constexpr int kTileBytes = kTileGroups * 9;               // 9216 = 576 x 16

__device__ __forceinline__ void pack_group(int32_t i0, int32_t i1, int32_t i2, int32_t i3,
                                           uint8_t *o) {
  o[0] = static_cast<uint8_t>((i0 >> 10) & 0xFF);
  o[1] = static_cast<uint8_t>((i0 >> 2) & 0xFF);
  o[2] = static_cast<uint8_t>(((i0 & 0x03) << 6) | ((i1 >> 12) & 0x3F));
  o[3] = static_cast<uint8_t>((i1 >> 4) & 0xFF);
  o[4] = static_cast<uint8_t>(((i1 & 0x0F) << 4) | ((i2 >> 14) & 0x0F));
  o[5] = static_cast<uint8_t>((i2 >> 6) & 0xFF);
  o[6] = static_cast<uint8_t>(((i2 & 0x3F) << 2) | ((i3 >> 16) & 0x03));
  o[7] = static_cast<uint8_t>((i3 >> 8) & 0xFF);
  o[8] = static_cast<uint8_t>(i3 & 0xFF);
}

__device__ __forceinline__ int4 unpack_group(const uint8_t *c) {
  int32_t b[9];
#pragma unroll
  for (int k = 0; k < 9; ++k) b[k] = c[k];
  int4 v;
  v.x = (b[0] << 10) | (b[1] << 2) | (b[2] >> 6);
  v.y = ((b[2] & 0x3F) << 12) | (b[3] << 4) | (b[4] >> 4);
  v.z = ((b[4] & 0x0F) << 14) | (b[5] << 6) | (b[6] >> 2);
  v.w = ((b[6] & 0x03) << 16) | (b[7] << 8) | b[8];
  return v;
}

template <typename T>
__device__ __forceinline__ int4 load_group(const T *idx, int64_t g, int64_t n, bool vec_ok);

template <>
__device__ __forceinline__ int4 load_group<int32_t>(const int32_t *idx, int64_t g, int64_t n,
                                                    bool vec_ok) {
  const int64_t i = 4 * g;
  if (vec_ok && i + 3 < n) return __ldcs(reinterpret_cast<const int4 *>(idx + i));
  int4 v;
  v.x = (i + 0 < n) ? idx[i + 0] : 0;
  v.y = (i + 1 < n) ? idx[i + 1] : 0;
  v.z = (i + 2 < n) ? idx[i + 2] : 0;
  v.w = (i + 3 < n) ? idx[i + 3] : 0;
  return v;
}

template <>
__device__ __forceinline__ int4 load_group<int64_t>(const int64_t *idx, int64_t g, int64_t n,
                                                    bool vec_ok) {
  const int64_t i = 4 * g;
  int4 v;
  if (vec_ok && i + 3 < n) {
    const longlong2 a = __ldcs(reinterpret_cast<const longlong2 *>(idx + i));
    const longlong2 b = __ldcs(reinterpret_cast<const longlong2 *>(idx + i + 2));
    v.x = static_cast<int32_t>(a.x);
    v.y = static_cast<int32_t>(a.y);
    v.z = static_cast<int32_t>(b.x);
    v.w = static_cast<int32_t>(b.y);
    return v;
  }
  v.x = (i + 0 < n) ? static_cast<int32_t>(idx[i + 0]) : 0;
  v.y = (i + 1 < n) ? static_cast<int32_t>(idx[i + 1]) : 0;
  v.z = (i + 2 < n) ? static_cast<int32_t>(idx[i + 2]) : 0;
  v.w = (i + 3 < n) ? static_cast<int32_t>(idx[i + 3]) : 0;
  return v;
}

template <typename T>
__global__ void __launch_bounds__(kThreads) pack_kernel(const T *__restrict__ idx, int64_t n,
                                                        uint8_t *__restrict__ out, bool vec_in,
                                                        bool vec_out) {
  __shared__ __align__(16) uint8_t tile[kTileBytes];
  const int64_t groups = (n + 3) / 4;
  const int64_t tiles = (groups + kTileGroups - 1) / kTileGroups;
  for (int64_t t = blockIdx.x; t < tiles; t += gridDim.x) {
    const int64_t g0 = t * kTileGroups;
#pragma unroll
    for (int k = 0; k < kGroupsPerThread; ++k) {
      const int gl = threadIdx.x + k * kThreads;
      const int64_t g = g0 + gl;
      if (g < groups) {
        const int4 v = load_group<T>(idx, g, n, vec_in);
        pack_group(v.x, v.y, v.z, v.w, tile + 9 * gl);
      }
    }
    __syncthreads();
    const int64_t bytes_left = 9 * (groups - g0);
    const int tile_bytes = bytes_left < kTileBytes ? static_cast<int>(bytes_left) : kTileBytes;
    uint8_t *dst = out + 9 * g0;
    if (vec_out) {
      const int nvec = tile_bytes / 16;
      for (int v = threadIdx.x; v < nvec; v += kThreads)
        __stcs(reinterpret_cast<int4 *>(dst) + v, reinterpret_cast<const int4 *>(tile)[v]);
      for (int b = nvec * 16 + threadIdx.x; b < tile_bytes; b += kThreads) dst[b] = tile[b];
    } else {
      for (int b = threadIdx.x; b < tile_bytes; b += kThreads) dst[b] = tile[b];
    }
    __syncthreads();
  }
}

template <typename T>
__device__ __forceinline__ void store_group(T *out, int64_t g, int64_t n, int4 v, bool vec_ok);

template <>
__device__ __forceinline__ void store_group<int32_t>(int32_t *out, int64_t g, int64_t n, int4 v,
                                                     bool vec_ok) {
  const int64_t i = 4 * g;
  if (vec_ok && i + 3 < n) {
    __stcs(reinterpret_cast<int4 *>(out + i), v);
    return;
  }
  if (i + 0 < n) out[i + 0] = v.x;
  if (i + 1 < n) out[i + 1] = v.y;
  if (i + 2 < n) out[i + 2] = v.z;
  if (i + 3 < n) out[i + 3] = v.w;
}

template <>
__device__ __forceinline__ void store_group<int64_t>(int64_t *out, int64_t g, int64_t n, int4 v,
                                                     bool vec_ok) {
  const int64_t i = 4 * g;
  if (vec_ok && i + 3 < n) {
    __stcs(reinterpret_cast<longlong2 *>(out + i), make_longlong2(v.x, v.y));
    __stcs(reinterpret_cast<longlong2 *>(out + i + 2), make_longlong2(v.z, v.w));
    return;
  }
  if (i + 0 < n) out[i + 0] = v.x;
  if (i + 1 < n) out[i + 1] = v.y;
  if (i + 2 < n) out[i + 2] = v.z;
  if (i + 3 < n) out[i + 3] = v.w;
}

template <typename T>
__global__ void __launch_bounds__(kThreads) unpack_kernel(const uint8_t *__restrict__ packed,
                                                          int64_t groups, int64_t n,
                                                          T *__restrict__ out, bool vec_in,
                                                          bool vec_out) {
  __shared__ __align__(16) uint8_t tile[kTileBytes];
  const int64_t used_groups = (n + 3) / 4 < groups ? (n + 3) / 4 : groups;
  const int64_t tiles = (used_groups + kTileGroups - 1) / kTileGroups;
  for (int64_t t = blockIdx.x; t < tiles; t += gridDim.x) {
    const int64_t g0 = t * kTileGroups;
    const int64_t bytes_left = 9 * (used_groups - g0);
    const int tile_bytes = bytes_left < kTileBytes ? static_cast<int>(bytes_left) : kTileBytes;
    const uint8_t *src = packed + 9 * g0;
    if (vec_in) {
      const int nvec = tile_bytes / 16;
      for (int v = threadIdx.x; v < nvec; v += kThreads)
        reinterpret_cast<int4 *>(tile)[v] = __ldcs(reinterpret_cast<const int4 *>(src) + v);
      for (int b = nvec * 16 + threadIdx.x; b < tile_bytes; b += kThreads) tile[b] = src[b];
    } else {
      for (int b = threadIdx.x; b < tile_bytes; b += kThreads) tile[b] = src[b];
    }
    __syncthreads();
#pragma unroll
    for (int k = 0; k < kGroupsPerThread; ++k) {
      const int gl = threadIdx.x + k * kThreads;
      const int64_t g = g0 + gl;
      if (g < used_groups) store_group<T>(out, g, n, unpack_group(tile + 9 * gl), vec_out);
    }
    __syncthreads();
  }
}

int grid_for(int64_t tiles) {
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const int64_t cap = static_cast<int64_t>(sms) * 8;
  return static_cast<int>(tiles < cap ? (tiles > 0 ? tiles : 1) : cap);
}

}  // namespace

int launch_pack_i32(const int32_t *idx, int64_t n, uint8_t *out, cudaStream_t s) {
  if (n <= 0) return H24_OK;
  const int64_t tiles = ((n + 3) / 4 + kTileGroups - 1) / kTileGroups;
  pack_kernel<int32_t><<<grid_for(tiles), kThreads, 0, s>>>(idx, n, out, aligned16(idx),
                                                            aligned16(out));
  H24_CUDA_TRY(cudaGetLastError());
  count_launches(1);
  return H24_OK;
}

int launch_pack_i64(const int64_t *idx, int64_t n, uint8_t *out, cudaStream_t s) {
  if (n <= 0) return H24_OK;
  const int64_t tiles = ((n + 3) / 4 + kTileGroups - 1) / kTileGroups;
  pack_kernel<int64_t><<<grid_for(tiles), kThreads, 0, s>>>(idx, n, out, aligned16(idx),
                                                            aligned16(out));
  H24_CUDA_TRY(cudaGetLastError());
  count_launches(1);
  return H24_OK;
}

int launch_unpack_i32(const uint8_t *p, int64_t groups, int64_t n, int32_t *out, cudaStream_t s) {
  if (n <= 0 || groups <= 0) return H24_OK;
  const int64_t used = (n + 3) / 4 < groups ? (n + 3) / 4 : groups;
  const int64_t tiles = (used + kTileGroups - 1) / kTileGroups;
  unpack_kernel<int32_t><<<grid_for(tiles), kThreads, 0, s>>>(p, groups, n, out, aligned16(p),
                                                              aligned16(out));
  H24_CUDA_TRY(cudaGetLastError());
  count_launches(1);
  return H24_OK;
}

int launch_unpack_i64(const uint8_t *p, int64_t groups, int64_t n, int64_t *out, cudaStream_t s) {
  if (n <= 0 || groups <= 0) return H24_OK;
  const int64_t used = (n + 3) / 4 < groups ? (n + 3) / 4 : groups;
  const int64_t tiles = (used + kTileGroups - 1) / kTileGroups;
  unpack_kernel<int64_t><<<grid_for(tiles), kThreads, 0, s>>>(p, groups, n, out, aligned16(p),
                                                              aligned16(out));
  H24_CUDA_TRY(cudaGetLastError());
  count_launches(1);
  return H24_OK;
}

}  // namespace h24
