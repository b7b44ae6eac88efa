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
// kernels are HBM-bound: 4 B read + 1 B written per element to quantise (the
// second pass over a row hits L1/L2), 1 B read + 2 B written to reconstruct.
#include "h24_internal.cuh"

namespace h24 {
namespace {

constexpr int kThreads = 256;
constexpr float kEps = 1e-8f;

// NaN (a NaN or infinite w, or a NaN row scale) becomes 0, as torch's
// int8 cast of the clamped NaN does.
__device__ __forceinline__ int8_t quant_one(float w, float mu) {
  const float t = __fmul_rn(__fdiv_rn(w, mu), 127.0f);
  if (isnan(t)) return 0;
  const float r = fminf(fmaxf(rintf(t), -128.0f), 127.0f);
  return static_cast<int8_t>(static_cast<int>(r));
}

// amax propagates NaN.
__device__ __forceinline__ float max_nan(float a, float b) { return (a != a || b != b) ? NAN : fmaxf(a, b); }

// One warp per row (grid-stride over rows).
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
    const float mu = m != m ? m : fmaxf(m, kEps);  // clamp_min keeps NaN
    if (vec) {
      const float4 *row4 = reinterpret_cast<const float4 *>(row);
      char4 *q4 = reinterpret_cast<char4 *>(qrow);
      for (int64_t c = lane; c < cols / 4; c += 32) {
        const float4 f = __ldg(row4 + c);
        q4[c] = make_char4(quant_one(f.x, mu), quant_one(f.y, mu), quant_one(f.z, mu),
                           quant_one(f.w, mu));
      }
    } else {
      for (int64_t c = lane; c < cols; c += 32) qrow[c] = quant_one(__ldg(row + c), mu);
    }
    if (lane == 0) mu16[r] = mu != mu ? static_cast<uint16_t>(0x7E00) : __half_as_ushort(__float2half_rn(mu));
  }
}

// 16 elements per thread when rows are 16-element aligned, else one.
__global__ void __launch_bounds__(kThreads) int8_dequant_kernel(const int8_t *__restrict__ q,
                                                                const uint16_t *__restrict__ mu16,
                                                                int64_t rows, int64_t cols,
                                                                uint16_t *__restrict__ out, bool vec) {
  const int64_t stride = static_cast<int64_t>(gridDim.x) * kThreads;
  const int64_t tid = blockIdx.x * static_cast<int64_t>(kThreads) + threadIdx.x;
  if (vec) {
    const int64_t per_row = cols / 16;
    const int64_t total = rows * per_row;
    for (int64_t i = tid; i < total; i += stride) {
      const int64_t r = i / per_row;
      const float s = __half2float(__float2half_rn(
          __fdiv_rn(__half2float(__ushort_as_half(__ldg(mu16 + r))), 127.0f)));
      const int4 v = __ldcs(reinterpret_cast<const int4 *>(q) + i);
      const uint32_t wv[4] = {static_cast<uint32_t>(v.x), static_cast<uint32_t>(v.y),
                              static_cast<uint32_t>(v.z), static_cast<uint32_t>(v.w)};
      uint32_t o[8];
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        const uint32_t word = wv[k >> 1] >> (16 * (k & 1));
        const float a = static_cast<float>(static_cast<int8_t>(word & 0xFF));
        const float b = static_cast<float>(static_cast<int8_t>((word >> 8) & 0xFF));
        o[k] = static_cast<uint32_t>(__half_as_ushort(__float2half_rn(__fmul_rn(a, s)))) |
               (static_cast<uint32_t>(__half_as_ushort(__float2half_rn(__fmul_rn(b, s)))) << 16);
      }
      uint4 *dst = reinterpret_cast<uint4 *>(out) + 2 * i;
      __stcs(dst, make_uint4(o[0], o[1], o[2], o[3]));
      __stcs(dst + 1, make_uint4(o[4], o[5], o[6], o[7]));
    }
  } else {
    const int64_t total = rows * cols;
    for (int64_t i = tid; i < total; i += stride) {
      const int64_t r = i / cols;
      const float s = __half2float(__float2half_rn(
          __fdiv_rn(__half2float(__ushort_as_half(__ldg(mu16 + r))), 127.0f)));
      out[i] = __half_as_ushort(__float2half_rn(__fmul_rn(static_cast<float>(__ldg(q + i)), s)));
    }
  }
}

int grid_for(int64_t work, int per_block) {
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const int64_t want = (work + per_block - 1) / per_block;
  const int64_t cap = static_cast<int64_t>(sms) * 8;
  return static_cast<int>(want < cap ? (want > 0 ? want : 1) : cap);
}

}  // namespace

int launch_int8_quantize(const float *w, int64_t rows, int64_t cols, int8_t *q, uint16_t *mu16,
                         cudaStream_t s) {
  if (rows == 0 || cols == 0) return H24_OK;
  const bool vec = cols % 4 == 0 && aligned16(w) && (reinterpret_cast<uintptr_t>(q) & 3) == 0;
  int8_quant_kernel<<<grid_for(rows, kThreads / 32), kThreads, 0, s>>>(w, rows, cols, q, mu16, vec);
  H24_CUDA_TRY(cudaGetLastError());
  count_launches(1);
  return H24_OK;
}

int launch_int8_dequant(const int8_t *q, const uint16_t *mu16, int64_t rows, int64_t cols,
                        uint16_t *out, cudaStream_t s) {
  if (rows == 0 || cols == 0) return H24_OK;
  const bool vec = cols % 16 == 0 && aligned16(q) && aligned16(out);
  const int64_t work = vec ? rows * (cols / 16) : rows * cols;
  int8_dequant_kernel<<<grid_for(work, kThreads), kThreads, 0, s>>>(q, mu16, rows, cols, out, vec);
  H24_CUDA_TRY(cudaGetLastError());
  count_launches(1);
  return H24_OK;
}

}  // namespace h24
