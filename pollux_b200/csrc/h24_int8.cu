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
// 1 B read + 2 B written to reconstruct.  Rows of up to 2,048 elements are
// quantised from registers (one read of the row); longer rows take a second
// pass that hits L1/L2.
#include "h24_internal.cuh"

namespace h24 {
namespace {

constexpr int kThreads = 256;
constexpr float kEps = 1e-8f;
constexpr int kRegVec = 16;  // float4 per lane held in registers: rows of up to 2048 elements

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

// amax propagates NaN.
__device__ __forceinline__ float max_nan(float a, float b) { return (a != a || b != b) ? NAN : fmaxf(a, b); }

__device__ __forceinline__ float row_mu(float m) { return m != m ? m : fmaxf(m, kEps); }  // clamp_min keeps NaN

__device__ __forceinline__ uint16_t mu_bits(float mu) {
  return mu != mu ? static_cast<uint16_t>(0x7E00) : __half_as_ushort(__float2half_rn(mu));
}

__device__ __forceinline__ uint32_t quant4(float4 f, float mu, float sc) {
  const uint32_t b0 = static_cast<uint8_t>(quant_fast(f.x, mu, sc));
  const uint32_t b1 = static_cast<uint8_t>(quant_fast(f.y, mu, sc));
  const uint32_t b2 = static_cast<uint8_t>(quant_fast(f.z, mu, sc));
  const uint32_t b3 = static_cast<uint8_t>(quant_fast(f.w, mu, sc));
  return b0 | (b1 << 8) | (b2 << 16) | (b3 << 24);
}

// One warp per row (grid-stride over rows), the row held in registers:
// rows 16-byte aligned with cols % 4 == 0 and cols <= 2048.
__global__ void __launch_bounds__(kThreads) int8_quant_reg_kernel(const float *__restrict__ w, int64_t rows,
                                                                  int64_t cols, int8_t *__restrict__ q,
                                                                  uint16_t *__restrict__ mu16) {
  const int lane = threadIdx.x & 31;
  const int64_t nwarps = static_cast<int64_t>(gridDim.x) * (kThreads / 32);
  const int nv = static_cast<int>(cols / 4);
  for (int64_t r = blockIdx.x * static_cast<int64_t>(kThreads / 32) + (threadIdx.x >> 5); r < rows;
       r += nwarps) {
    const float4 *row4 = reinterpret_cast<const float4 *>(w + r * cols);
    float4 f[kRegVec];
#pragma unroll
    for (int k = 0; k < kRegVec; ++k) {
      const int c = lane + 32 * k;
      f[k] = c < nv ? __ldcs(row4 + c) : make_float4(0.f, 0.f, 0.f, 0.f);
    }
    float m = 0.f;
#pragma unroll
    for (int k = 0; k < kRegVec; ++k)
      m = max_nan(m, max_nan(max_nan(fabsf(f[k].x), fabsf(f[k].y)), max_nan(fabsf(f[k].z), fabsf(f[k].w))));
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) m = max_nan(m, __shfl_xor_sync(0xffffffffu, m, off));
    const float mu = row_mu(m);
    const float sc = __fdiv_rn(127.0f, mu);
    int *q4 = reinterpret_cast<int *>(q + r * cols);
#pragma unroll
    for (int k = 0; k < kRegVec; ++k) {
      const int c = lane + 32 * k;
      if (c < nv) __stcs(q4 + c, static_cast<int>(quant4(f[k], mu, sc)));
    }
    if (lane == 0) mu16[r] = mu_bits(mu);
  }
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
      for (int64_t c = lane; c < cols / 4; c += 32) {
        const float4 f = __ldg(row4 + c);
        m = max_nan(m, max_nan(max_nan(fabsf(f.x), fabsf(f.y)), max_nan(fabsf(f.z), fabsf(f.w))));
      }
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
  if (vec && cols <= 4 * 32 * kRegVec)
    int8_quant_reg_kernel<<<grid_for(int8_quant_reg_kernel, rows, kThreads / 32), kThreads, 0, s>>>(
        w, rows, cols, q, mu16);
  else
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
  int8_dequant_kernel<<<grid, kThreads, 0, s>>>(q, mu16, rows, cols, out, vec);
  H24_CUDA_TRY(cudaGetLastError());
  count_launches(1);
  return H24_OK;
}

}  // namespace h24
