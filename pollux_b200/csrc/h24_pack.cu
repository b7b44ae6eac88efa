// h24_pack.cu -- 18-bit index pack / unpack (castor.py:226-260).
//
// Format: indices are taken four at a time (i0,i1,i2,i3); the 9 output bytes
// are the big-endian 72-bit integer i0<<54 | i1<<36 | i2<<18 | i3, each index
// first truncated to 32 bits and then masked to 18 bits by the byte formulas.
//
// Both kernels are launched with programmatic stream serialization: a kernel
// lets the next one in the stream launch as soon as it starts, and waits
// (griddepcontrol.wait) for the previous one to complete before reading its
// input, so the launch and ramp of one call overlap the tail of the previous
// kernel.  Without such a launch the two instructions do nothing.
//
// Both kernels run independent warps (no block-wide barriers), each moving
// 128 groups (512 indices, 1152 packed bytes) per iteration through its own
// shared-memory slice, so that global traffic on both sides is fully
// coalesced 16-byte vectors: the packed stream has no 16-byte structure of its
// own (9-byte groups), the index stream does.  In shared memory a lane owns 4
// consecutive groups: 16 indices on one side, 9 aligned 32-bit words on the
// other.  HBM-bound: 4 + 2.25 bytes per index (int32 side).
#include "h24_internal.cuh"

namespace h24 {
namespace {

constexpr int kThreads = 256;
constexpr int kWarps = kThreads / 32;
constexpr int kWarpGroups = 128;                  // groups per warp iteration
constexpr int kWarpIndices = 4 * kWarpGroups;     // 512
constexpr int kWarpBytes = 9 * kWarpGroups;       // 1152 = 72 x 16

// 16-byte slot of index vector c (group c, c in [0,128)) in a warp's slice.
// Lanes write c = lane + 32j and read c = 4*lane + i; the XOR makes both
// patterns conflict-free for 128-bit accesses (8 distinct slots mod 8 in
// every quarter warp).
__device__ __forceinline__ int swz(int c) { return c ^ ((c >> 3) & 7); }


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

// The 9 bytes of groups 4*lane .. 4*lane+3 as nine little-endian words.
__device__ __forceinline__ void pack_quad(const int4 *v, uint32_t *w) {
  uint8_t o[36];
#pragma unroll
  for (int i = 0; i < 4; ++i) pack_group(v[i].x, v[i].y, v[i].z, v[i].w, o + 9 * i);
#pragma unroll
  for (int k = 0; k < 9; ++k)
    w[k] = static_cast<uint32_t>(o[4 * k]) | (static_cast<uint32_t>(o[4 * k + 1]) << 8) |
           (static_cast<uint32_t>(o[4 * k + 2]) << 16) | (static_cast<uint32_t>(o[4 * k + 3]) << 24);
}

template <typename T>
__device__ __forceinline__ int4 load_vec(const T *p);
template <>
__device__ __forceinline__ int4 load_vec<int32_t>(const int32_t *p) {
  return __ldcs(reinterpret_cast<const int4 *>(p));
}
template <>
__device__ __forceinline__ int4 load_vec<int64_t>(const int64_t *p) {
  const longlong2 a = __ldcs(reinterpret_cast<const longlong2 *>(p));
  const longlong2 b = __ldcs(reinterpret_cast<const longlong2 *>(p + 2));
  return make_int4(static_cast<int32_t>(a.x), static_cast<int32_t>(a.y), static_cast<int32_t>(b.x),
                   static_cast<int32_t>(b.y));
}

// `fast` = both pointers 16-byte aligned: whole warp tiles take the vector
// path, the remaining groups (or all of them) one thread per group.
template <typename T>
__global__ void __launch_bounds__(kThreads) pack_kernel(const T *__restrict__ idx, int64_t n,
                                                        uint8_t *__restrict__ out, bool fast) {
  __shared__ int4 slice[kWarps][kWarpGroups];  // 2 KB per warp
  pdl_enter();
  const int lane = threadIdx.x & 31;
  int4 *S = slice[threadIdx.x >> 5];
  const int64_t groups = (n + 3) / 4;
  const int64_t full = fast ? n / kWarpIndices : 0;
  const int64_t nwarps = static_cast<int64_t>(gridDim.x) * kWarps;
  for (int64_t wt = blockIdx.x * static_cast<int64_t>(kWarps) + (threadIdx.x >> 5); wt < full;
       wt += nwarps) {
    const T *src = idx + wt * kWarpIndices;
    int4 v[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) v[j] = load_vec<T>(src + 4 * (lane + 32 * j));
#pragma unroll
    for (int j = 0; j < 4; ++j) S[swz(lane + 32 * j)] = v[j];
    __syncwarp();
#pragma unroll
    for (int i = 0; i < 4; ++i) v[i] = S[swz(4 * lane + i)];
    uint32_t w[9];
    pack_quad(v, w);
    __syncwarp();
    uint32_t *W = reinterpret_cast<uint32_t *>(S);
#pragma unroll
    for (int k = 0; k < 9; ++k) W[9 * lane + k] = w[k];  // stride 9 words: conflict-free
    __syncwarp();
    int4 *dst = reinterpret_cast<int4 *>(out + wt * kWarpBytes);
#pragma unroll
    for (int m = 0; m < 3; ++m) {
      const int c = lane + 32 * m;
      if (c < kWarpBytes / 16) __stcs(dst + c, S[c]);
    }
    __syncwarp();
  }
  for (int64_t g = full * kWarpGroups + blockIdx.x * static_cast<int64_t>(kThreads) + threadIdx.x;
       g < groups; g += static_cast<int64_t>(gridDim.x) * kThreads) {
    const int4 v = load_group<T>(idx, g, n, false);
    uint8_t o[9];
    pack_group(v.x, v.y, v.z, v.w, o);
#pragma unroll
    for (int k = 0; k < 9; ++k) out[9 * g + k] = o[k];
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
__device__ __forceinline__ void store_vec(T *p, int4 v);
template <>
__device__ __forceinline__ void store_vec<int32_t>(int32_t *p, int4 v) {
  __stcs(reinterpret_cast<int4 *>(p), v);
}
template <>
__device__ __forceinline__ void store_vec<int64_t>(int64_t *p, int4 v) {
  __stcs(reinterpret_cast<longlong2 *>(p), make_longlong2(v.x, v.y));
  __stcs(reinterpret_cast<longlong2 *>(p + 2), make_longlong2(v.z, v.w));
}

template <typename T>
__global__ void __launch_bounds__(kThreads) unpack_kernel(const uint8_t *__restrict__ packed,
                                                          int64_t groups, int64_t n,
                                                          T *__restrict__ out, bool fast) {
  __shared__ int4 slice[kWarps][kWarpGroups];
  pdl_enter();
  const int lane = threadIdx.x & 31;
  int4 *S = slice[threadIdx.x >> 5];
  const int64_t used_groups = (n + 3) / 4 < groups ? (n + 3) / 4 : groups;
  int64_t full = 0;
  if (fast) {
    const int64_t by_n = n / kWarpIndices, by_groups = groups / kWarpGroups;
    full = by_n < by_groups ? by_n : by_groups;
  }
  const int64_t nwarps = static_cast<int64_t>(gridDim.x) * kWarps;
  for (int64_t wt = blockIdx.x * static_cast<int64_t>(kWarps) + (threadIdx.x >> 5); wt < full;
       wt += nwarps) {
    const int4 *src = reinterpret_cast<const int4 *>(packed + wt * kWarpBytes);
    int4 p[3];
#pragma unroll
    for (int m = 0; m < 3; ++m) {
      const int c = lane + 32 * m;
      if (c < kWarpBytes / 16) p[m] = __ldcs(src + c);
    }
#pragma unroll
    for (int m = 0; m < 3; ++m) {
      const int c = lane + 32 * m;
      if (c < kWarpBytes / 16) S[c] = p[m];
    }
    __syncwarp();
    const uint32_t *W = reinterpret_cast<const uint32_t *>(S);
    uint8_t b[36];
#pragma unroll
    for (int k = 0; k < 9; ++k) {
      const uint32_t w = W[9 * lane + k];
#pragma unroll
      for (int e = 0; e < 4; ++e) b[4 * k + e] = static_cast<uint8_t>(w >> (8 * e));
    }
    int4 v[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) v[i] = unpack_group(b + 9 * i);
    __syncwarp();
#pragma unroll
    for (int i = 0; i < 4; ++i) S[swz(4 * lane + i)] = v[i];
    __syncwarp();
    T *dst = out + wt * kWarpIndices;
#pragma unroll
    for (int j = 0; j < 4; ++j) store_vec<T>(dst + 4 * (lane + 32 * j), S[swz(lane + 32 * j)]);
    __syncwarp();
  }
  for (int64_t g = full * kWarpGroups + blockIdx.x * static_cast<int64_t>(kThreads) + threadIdx.x;
       g < used_groups; g += static_cast<int64_t>(gridDim.x) * kThreads)
    store_group<T>(out, g, n, unpack_group(packed + 9 * g), false);
}

// Enough warps for the vector tiles (or for one thread per remaining group),
// capped at one resident wave of `kernel`.
template <typename K>
int grid_for(K kernel, int64_t tiles, int64_t rest_groups) {
  int64_t want = (tiles + kWarps - 1) / kWarps;
  const int64_t rest = (rest_groups + kThreads - 1) / kThreads;
  if (rest > want) want = rest;
  return wave_grid(want, blocks_per_sm(kernel, kThreads, 0));
}

template <typename T>
int launch_pack(const T *idx, int64_t n, uint8_t *out, cudaStream_t s) {
  if (n <= 0) return H24_OK;
  const bool fast = aligned16(idx) && aligned16(out);
  const int64_t tiles = fast ? n / kWarpIndices : 0;
  const int64_t rest = (n + 3) / 4 - tiles * kWarpGroups;
  H24_CUDA_TRY(launch_pdl(pack_kernel<T>, dim3(grid_for(pack_kernel<T>, tiles, rest)), dim3(kThreads), s, idx,
                          n, out, fast));
  count_launches(1);
  return H24_OK;
}

template <typename T>
int launch_unpack(const uint8_t *p, int64_t groups, int64_t n, T *out, cudaStream_t s) {
  if (n <= 0 || groups <= 0) return H24_OK;
  const bool fast = aligned16(p) && aligned16(out);
  const int64_t used = (n + 3) / 4 < groups ? (n + 3) / 4 : groups;
  int64_t tiles = 0;
  if (fast) tiles = n / kWarpIndices < groups / kWarpGroups ? n / kWarpIndices : groups / kWarpGroups;
  H24_CUDA_TRY(launch_pdl(unpack_kernel<T>, dim3(grid_for(unpack_kernel<T>, tiles, used - tiles * kWarpGroups)),
                          dim3(kThreads), s, p, groups, n, out, fast));
  count_launches(1);
  return H24_OK;
}

}  // namespace

int launch_pack_i32(const int32_t *idx, int64_t n, uint8_t *out, cudaStream_t s) {
  return launch_pack<int32_t>(idx, n, out, s);
}

int launch_pack_i64(const int64_t *idx, int64_t n, uint8_t *out, cudaStream_t s) {
  return launch_pack<int64_t>(idx, n, out, s);
}

int launch_unpack_i32(const uint8_t *p, int64_t groups, int64_t n, int32_t *out, cudaStream_t s) {
  return launch_unpack<int32_t>(p, groups, n, out, s);
}

int launch_unpack_i64(const uint8_t *p, int64_t groups, int64_t n, int64_t *out, cudaStream_t s) {
  return launch_unpack<int64_t>(p, groups, n, out, s);
}

}  // namespace h24
