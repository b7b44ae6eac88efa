// h24_int8.cu -- per-row INT8 quantisation of the token embedding and output
// head (pack._quantize_int8, pack.py:124-136) and its reconstruction
// (PackedInt8Embedding / PackedInt8Linear.materialize, pollux.py:510-563).
//
//   mu_r  = max(max_c |w_rc|, fp32(1e-8))              fp32, exact (NaN if any w is)
//   q_rc  = clamp(rint(fp32(fp32(w_rc / mu_r) * 127)), -128, 127)   int8
//   mu16  = fp16_rn(mu_r)
//   w16   = fp16_rn(fp32(q_rc) * fp32(fp16_rn(fp32(mu16) / 127)))
//
// Division and products are IEEE round-to-nearest as in the reference's fp32
// and fp16 tensor arithmetic (rint = round half to even, torch.round).  Both
// kernels are HBM-bound: 4 B read + 1 B written per element to quantise,
// 1 B read + 2 B written to reconstruct.  Rows of up to 4,096 elements are
// streamed through shared memory: each warp owns a row at a time and has the
// next one in flight (cp.async, two buffers per warp), so HBM reads continue
// while the current row is reduced and quantised; other rows take two passes,
// the second hitting L1/L2.
#include "h24_internal.cuh"

namespace h24 {
namespace {

constexpr int kThreads = 256;
constexpr float kEps = 1e-8f;
constexpr int kStreamThreads = 128;  // 4 warps per block in the streaming kernel
constexpr int kStreamMaxCols = 4096;   // rows that fit the two shared-memory buffers of a warp

// NaN (a NaN or infinite w, or a NaN row scale) becomes 0, as torch's
// int8 cast of the clamped NaN does.
__device__ __forceinline__ int8_t quant_one(float w, float mu) {
  const float t = __fmul_rn(__fdiv_rn(w, mu), 127.0f);
  if (isnan(t)) return 0;
  const float r = fminf(fmaxf(rintf(t), -128.0f), 127.0f);
  return static_cast<int8_t>(static_cast<int>(r));
}

// quant_one without a division for almost every element.  t = fp32(w * s)
// with s = fp32(127 / mu) differs from the reference's fp32(fp32(w / mu) *
// 127) by at most 4 * 2^-24 * |127 w / mu| <= 3.1e-5 (|w| <= mu: mu is the
// row's max), so when t lies farther than 1e-4 from every half-integer both
// round to the same integer; otherwise (rarely) the reference's two roundings
// are evaluated as they are.
__device__ __forceinline__ int8_t quant_fast(float w, float mu, float s) {
  const float t = __fmul_rn(w, s);
  const float f = t - rintf(t);
  if (!(fabsf(fabsf(f) - 0.5f) > 1e-4f)) return quant_one(w, mu);  // near a tie, or NaN
  const float r = fminf(fmaxf(rintf(t), -128.0f), 127.0f);
  return static_cast<int8_t>(static_cast<int>(r));
}

// amax propagates NaN: max.NaN returns NaN when either input is NaN.
__device__ __forceinline__ float max_nan(float a, float b) {
  float r;
  asm("max.NaN.f32 %0, %1, %2;" : "=f"(r) : "f"(a), "f"(b));
  return r;
}

// max_nan(m, |f.x|, |f.y|, |f.z|, |f.w|)
__device__ __forceinline__ float absmax4(float m, float4 f) {
  return max_nan(max_nan(m, fabsf(f.x)), max_nan(max_nan(fabsf(f.y), fabsf(f.z)), fabsf(f.w)));
}

__device__ __forceinline__ float row_mu(float m) { return m != m ? m : fmaxf(m, kEps); }  // clamp_min keeps NaN

__device__ __forceinline__ uint16_t mu_bits(float mu) {
  return mu != mu ? static_cast<uint16_t>(0x7E00) : __half_as_ushort(__float2half_rn(mu));
}

// Four quant_fast results as packed int8 (element 0 in the low byte).  One
// test covers the four elements: when any lies within 1e-4 of a half-integer
// (or is NaN) all four take quant_one.  No clamp: |t| <= 127 (1 + 2^-22)
// < 127.5, so rint(t) already lies in [-127, 127].
__device__ __forceinline__ uint32_t quant4(float4 f, float mu, float sc) {
  const float t0 = __fmul_rn(f.x, sc), t1 = __fmul_rn(f.y, sc);
  const float t2 = __fmul_rn(f.z, sc), t3 = __fmul_rn(f.w, sc);
  const float r0 = rintf(t0), r1 = rintf(t1), r2 = rintf(t2), r3 = rintf(t3);
  const bool far = (fabsf(fabsf(t0 - r0) - 0.5f) > 1e-4f) & (fabsf(fabsf(t1 - r1) - 0.5f) > 1e-4f) &
                   (fabsf(fabsf(t2 - r2) - 0.5f) > 1e-4f) & (fabsf(fabsf(t3 - r3) - 0.5f) > 1e-4f);
  int i0, i1, i2, i3;
  if (far) {
    i0 = __float2int_rz(r0);
    i1 = __float2int_rz(r1);
    i2 = __float2int_rz(r2);
    i3 = __float2int_rz(r3);
  } else {
    i0 = quant_one(f.x, mu);
    i1 = quant_one(f.y, mu);
    i2 = quant_one(f.z, mu);
    i3 = quant_one(f.w, mu);
  }
  return __byte_perm(__byte_perm(i0, i1, 0x0040), __byte_perm(i2, i3, 0x0040), 0x5410);
}

__device__ __forceinline__ void cp_async16(void *dst, const void *src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(static_cast<uint32_t>(__cvta_generic_to_shared(dst))),
               "l"(src)
               : "memory");
}

// One warp per row (grid-stride over rows) for rows 16-byte aligned with
// cols % 4 == 0 and cols <= kStreamMaxCols.  The warp's two shared-memory
// buffers alternate: row i+1 is copied in while row i is reduced and
// quantised.  Lane l copies and later reads the float4s l, l+32, ... of a
// row, so each lane waits only for its own copies (cp.async.wait_group).
__global__ void __launch_bounds__(kStreamThreads) int8_quant_stream_kernel(const float *__restrict__ w,
                                                                           int64_t rows, int64_t cols,
                                                                           int8_t *__restrict__ q,
                                                                           uint16_t *__restrict__ mu16) {
  extern __shared__ __align__(16) float4 int8_rows[];
  const int lane = threadIdx.x & 31;
  const int nv = static_cast<int>(cols / 4);
  float4 *buf = int8_rows + static_cast<size_t>(threadIdx.x >> 5) * 2 * nv;
  const int64_t nwarps = static_cast<int64_t>(gridDim.x) * (kStreamThreads / 32);
  int64_t r = blockIdx.x * static_cast<int64_t>(kStreamThreads / 32) + (threadIdx.x >> 5);
  auto issue = [&](int64_t row, float4 *dst) {
    if (row < rows) {
      const float4 *src = reinterpret_cast<const float4 *>(w + row * cols);
      for (int c = lane; c < nv; c += 32) cp_async16(dst + c, src + c);
    }
    asm volatile("cp.async.commit_group;" ::: "memory");  // one group per row, empty past the end
  };
  issue(r, buf);
  for (int i = 0; r < rows; ++i, r += nwarps) {
    const float4 *cur = buf + (i & 1) * nv;
    issue(r + nwarps, buf + ((i + 1) & 1) * nv);
    asm volatile("cp.async.wait_group 1;" ::: "memory");  // this lane's copies of row r landed
    // Four independent float4 per step in both passes (the trip count is a
    // runtime value, so the loops are unrolled by hand for latency overlap).
    float mm[4] = {0.f, 0.f, 0.f, 0.f};
    int c = lane;
    for (; c + 96 < nv; c += 128) {
#pragma unroll
      for (int k = 0; k < 4; ++k) mm[k] = absmax4(mm[k], cur[c + 32 * k]);
    }
    for (; c < nv; c += 32) mm[0] = absmax4(mm[0], cur[c]);
    float m = max_nan(max_nan(mm[0], mm[1]), max_nan(mm[2], mm[3]));
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) m = max_nan(m, __shfl_xor_sync(0xffffffffu, m, off));
    const float mu = row_mu(m);
    const float sc = __fdiv_rn(127.0f, mu);
    int *q4 = reinterpret_cast<int *>(q + r * cols);
    c = lane;
    for (; c + 96 < nv; c += 128) {
      float4 f[4];
#pragma unroll
      for (int k = 0; k < 4; ++k) f[k] = cur[c + 32 * k];
#pragma unroll
      for (int k = 0; k < 4; ++k) __stcs(q4 + c + 32 * k, static_cast<int>(quant4(f[k], mu, sc)));
    }
    for (; c < nv; c += 32) __stcs(q4 + c, static_cast<int>(quant4(cur[c], mu, sc)));
    if (lane == 0) mu16[r] = mu_bits(mu);
    __syncwarp();
  }
  asm volatile("cp.async.wait_group 0;" ::: "memory");
}

// One warp per row (grid-stride over rows), two passes over the row.
__global__ void __launch_bounds__(kThreads) int8_quant_kernel(const float *__restrict__ w, int64_t rows,
                                                              int64_t cols, int8_t *__restrict__ q,
                                                              uint16_t *__restrict__ mu16, bool vec) {
  const int lane = threadIdx.x & 31;
  const int64_t nwarps = static_cast<int64_t>(gridDim.x) * (kThreads / 32);
  for (int64_t r = blockIdx.x * static_cast<int64_t>(kThreads / 32) + (threadIdx.x >> 5); r < rows;
       r += nwarps) {
    const float *row = w + r * cols;
    int8_t *qrow = q + r * cols;
    float m = 0.f;
    if (vec) {
      const float4 *row4 = reinterpret_cast<const float4 *>(row);
      for (int64_t c = lane; c < cols / 4; c += 32) m = absmax4(m, __ldg(row4 + c));
    } else {
      for (int64_t c = lane; c < cols; c += 32) m = max_nan(m, fabsf(__ldg(row + c)));
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) m = max_nan(m, __shfl_xor_sync(0xffffffffu, m, off));
    const float mu = row_mu(m);
    const float sc = __fdiv_rn(127.0f, mu);
    if (vec) {
      const float4 *row4 = reinterpret_cast<const float4 *>(row);
      int *q4 = reinterpret_cast<int *>(qrow);
      for (int64_t c = lane; c < cols / 4; c += 32) q4[c] = static_cast<int>(quant4(__ldg(row4 + c), mu, sc));
    } else {
      for (int64_t c = lane; c < cols; c += 32) qrow[c] = quant_fast(__ldg(row + c), mu, sc);
    }
    if (lane == 0) mu16[r] = mu_bits(mu);
  }
}

// fp32(fp16_rn(fp32(mu16) / 127)): the reconstruction scale of row r.
__device__ __forceinline__ float row_scale(const uint16_t *mu16, int64_t r) {
  return __half2float(__float2half_rn(__fdiv_rn(__half2float(__ushort_as_half(__ldg(mu16 + r))), 127.0f)));
}

// Two fp16 outputs (low half = first) from the two low bytes of `word`.
__device__ __forceinline__ uint32_t deq2(uint32_t word, float s) {
  const float a = static_cast<float>(static_cast<int8_t>(word & 0xFF));
  const float b = static_cast<float>(static_cast<int8_t>((word >> 8) & 0xFF));
  return static_cast<uint32_t>(__half_as_ushort(__float2half_rn(__fmul_rn(a, s)))) |
         (static_cast<uint32_t>(__half_as_ushort(__float2half_rn(__fmul_rn(b, s)))) << 16);
}

// vec (cols % 16 == 0, 16-byte aligned): one warp per row, the row scale
// computed once, 16 elements per lane and step; else one element per thread.
__global__ void __launch_bounds__(kThreads) int8_dequant_kernel(const int8_t *__restrict__ q,
                                                                const uint16_t *__restrict__ mu16,
                                                                int64_t rows, int64_t cols,
                                                                uint16_t *__restrict__ out, bool vec) {
  pdl_enter();
  if (vec) {
    const int lane = threadIdx.x & 31;
    const int64_t nwarps = static_cast<int64_t>(gridDim.x) * (kThreads / 32);
    const int per_row = static_cast<int>(cols / 16);
    for (int64_t r = blockIdx.x * static_cast<int64_t>(kThreads / 32) + (threadIdx.x >> 5); r < rows;
         r += nwarps) {
      const float s = row_scale(mu16, r);
      const int4 *src = reinterpret_cast<const int4 *>(q + r * cols);
      uint4 *dst = reinterpret_cast<uint4 *>(out + r * cols);
      for (int c0 = 0; c0 < per_row; c0 += 64) {
        int4 v[2];
#pragma unroll
        for (int k = 0; k < 2; ++k) {
          const int c = c0 + lane + 32 * k;
          v[k] = c < per_row ? __ldcs(src + c) : make_int4(0, 0, 0, 0);
        }
#pragma unroll
        for (int k = 0; k < 2; ++k) {
          const int c = c0 + lane + 32 * k;
          if (c < per_row) {
            const uint32_t w0 = static_cast<uint32_t>(v[k].x), w1 = static_cast<uint32_t>(v[k].y);
            const uint32_t w2 = static_cast<uint32_t>(v[k].z), w3 = static_cast<uint32_t>(v[k].w);
            __stcs(dst + 2 * c, make_uint4(deq2(w0, s), deq2(w0 >> 16, s), deq2(w1, s), deq2(w1 >> 16, s)));
            __stcs(dst + 2 * c + 1, make_uint4(deq2(w2, s), deq2(w2 >> 16, s), deq2(w3, s), deq2(w3 >> 16, s)));
          }
        }
      }
    }
  } else {
    const int64_t stride = static_cast<int64_t>(gridDim.x) * kThreads;
    const int64_t total = rows * cols;
    for (int64_t i = blockIdx.x * static_cast<int64_t>(kThreads) + threadIdx.x; i < total; i += stride) {
      const int64_t r = i / cols;
      out[i] = __half_as_ushort(__float2half_rn(__fmul_rn(static_cast<float>(__ldg(q + i)), row_scale(mu16, r))));
    }
  }
}

// One resident wave of `kernel`, or fewer blocks when `work` items (of
// `per_block` per block) need fewer.
template <typename K>
int grid_for(K kernel, int64_t work, int per_block) {
  return wave_grid((work + per_block - 1) / per_block, blocks_per_sm(kernel, kThreads, 0));
}

}  // namespace

int launch_int8_quantize(const float *w, int64_t rows, int64_t cols, int8_t *q, uint16_t *mu16,
                         cudaStream_t s) {
  if (rows == 0 || cols == 0) return H24_OK;
  const bool vec = cols % 4 == 0 && aligned16(w) && (reinterpret_cast<uintptr_t>(q) & 3) == 0;
  if (vec && cols <= kStreamMaxCols) {
    const size_t smem = static_cast<size_t>(kStreamThreads / 32) * 2 * cols * sizeof(float);
    H24_CUDA_TRY(cudaFuncSetAttribute(int8_quant_stream_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                      static_cast<int>(smem)));
    H24_CUDA_TRY(cudaFuncSetAttribute(int8_quant_stream_kernel, cudaFuncAttributePreferredSharedMemoryCarveout,
                                      cudaSharedmemCarveoutMaxShared));
    const int grid = wave_grid((rows + kStreamThreads / 32 - 1) / (kStreamThreads / 32),
                               blocks_per_sm(int8_quant_stream_kernel, kStreamThreads, smem));
    int8_quant_stream_kernel<<<grid, kStreamThreads, smem, s>>>(w, rows, cols, q, mu16);
  } else
    int8_quant_kernel<<<grid_for(int8_quant_kernel, rows, kThreads / 32), kThreads, 0, s>>>(
        w, rows, cols, q, mu16, vec);
  H24_CUDA_TRY(cudaGetLastError());
  count_launches(1);
  return H24_OK;
}

int launch_int8_dequant(const int8_t *q, const uint16_t *mu16, int64_t rows, int64_t cols,
                        uint16_t *out, cudaStream_t s) {
  if (rows == 0 || cols == 0) return H24_OK;
  const bool vec = cols % 16 == 0 && aligned16(q) && aligned16(out);
  const int grid = vec ? grid_for(int8_dequant_kernel, rows, kThreads / 32)
                       : grid_for(int8_dequant_kernel, rows * cols, kThreads);
  // Programmatic dependent launch (pdl_enter): the launch overlaps the tail
  // of the kernel before it.
  H24_CUDA_TRY(launch_pdl(int8_dequant_kernel, dim3(grid), dim3(kThreads), s, q, mu16, rows, cols, out, vec));
  count_launches(1);
  return H24_OK;
}

}  // namespace h24
