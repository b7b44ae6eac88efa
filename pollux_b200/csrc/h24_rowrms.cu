// h24_rowrms.cu -- per-row RMS scales of the reference, bit for bit:
//   training rule  sigma   = sqrt(mean(w^2, -1) + 1e-8)           (row_rms_from_matrix,
//                                                                  castor.py:309-313)
//   pack rule      sigma16 = fp16(clamp_min(sigma * sqrt(12), 1e-8)) (pack.py:164)
// with w = weight.float() (bf16 weights widen exactly) and the squares w*w
// rounded to fp32.
//
// The reference runs these on CUDA tensors (pack.py's --device defaults to
// cuda; pollux_step runs on the training device), so the fp32 mean is the one
// torch's CUDA reduction produces.  Its summation order is fixed by the
// launch plan torch chooses for a contiguous [rows, n] tensor reduced over
// its last dimension (PyTorch 2.11, ATen/native/cuda/Reduce.cuh:
// setReduceConfig, input_vectorized_thread_reduce_impl, thread_reduce_impl,
// block_x_reduce, block_y_reduce; MeanOps in ATen/native/SharedReduceOps.h),
// restated here:
//   * rows of at least 128 elements are read as 4-element vectors; lane x of a
//     block row keeps four accumulators, one per vector element, over the
//     vectors x, x + step, x + 2 step, ...; a row whose start is not 16-byte
//     aligned first hands its head elements to lanes shift..3, and the ragged
//     tail goes to lanes 0..; the accumulators combine as ((a0 + a1) + a2) + a3;
//   * shorter rows are read element by element with four accumulators over
//     the indices x + k step (k = 0..3, then the next four);
//   * block width bw and height bh: dim0 = n (n / 4 when vectorised),
//     d0 = last_pow2(dim0) capped at 512, d1 = last_pow2(rows) capped at 512,
//     bw = min(d0, 32), bh = min(d1, 512 / bw), bw = min(d0, 512 / bh);
//   * if ceil(n / bw) >= min(16 bh, 256) the bh warps of a block share one row
//     (step bw * bh, then a shared-memory tree over y), otherwise each block
//     row y reduces its own row (step bw);
//   * lanes combine through shared memory down to 32 (offsets bw/2 .. 32), then
//     by shuffles with offsets 16, 8, 4, 2, 1 (or from bw/2 when bw < 32);
//   * mean = sum * factor with factor = fp32(rows) / fp32(rows * n).
// Rows longer than about 131,000 elements make torch split a row across
// blocks as well; this kernel keeps one block per row there, so such rows may
// differ from torch's mean in the last bit.
#include "h24_internal.cuh"

namespace h24 {
namespace {

struct MeanPlan {
  int vec;       // 4-element vector loads
  int bw, bh;    // block shape
  int split;     // the bh rows of threads share one matrix row
  float factor;  // MeanOps factor
};

int64_t last_pow2(int64_t v) {
  int64_t p = 1;
  while (p * 2 <= v) p *= 2;
  return p;
}

MeanPlan mean_plan(int64_t rows, int64_t n) {
  MeanPlan p;
  p.vec = n >= 128 ? 1 : 0;
  const int64_t dim0 = p.vec ? n / 4 : n;
  const int d0 = static_cast<int>(dim0 < 512 ? last_pow2(dim0) : 512);
  const int d1 = static_cast<int>(rows < 512 ? last_pow2(rows) : 512);
  int bw = d0 < 32 ? d0 : 32;
  const int bh = d1 < 512 / bw ? d1 : 512 / bw;
  bw = d0 < 512 / bh ? d0 : 512 / bh;
  p.bw = bw;
  p.bh = bh;
  const int64_t vpt = (n + bw - 1) / bw;
  const int thresh = 16 * bh < 256 ? 16 * bh : 256;
  p.split = vpt >= thresh ? 1 : 0;
  p.factor = static_cast<float>(rows) / static_cast<float>(rows * n);
  return p;
}

template <typename T>
__device__ __forceinline__ float sq_at(const T *__restrict__ p, int64_t i) {
  float v;
  if constexpr (sizeof(T) == 4) {
    v = __ldg(reinterpret_cast<const float *>(p) + i);
  } else {
    v = __uint_as_float(static_cast<uint32_t>(__ldg(reinterpret_cast<const unsigned short *>(p) + i)) << 16);
  }
  return __fmul_rn(v, v);
}

// Squares of the 4-element vector at element offset e (e a multiple of 4 from
// a 16-byte aligned fp32 address, i.e. 8-byte aligned for bf16).
template <typename T>
__device__ __forceinline__ float4 sq_vec4(const T *__restrict__ p, int64_t e) {
  float4 f;
  if constexpr (sizeof(T) == 4) {
    f = __ldg(reinterpret_cast<const float4 *>(p + e));
  } else {
    const uint2 u = __ldg(reinterpret_cast<const uint2 *>(p + e));
    f = make_float4(__uint_as_float(u.x << 16), __uint_as_float(u.x & 0xFFFF0000u),
                    __uint_as_float(u.y << 16), __uint_as_float(u.y & 0xFFFF0000u));
  }
  return make_float4(__fmul_rn(f.x, f.x), __fmul_rn(f.y, f.y), __fmul_rn(f.z, f.z), __fmul_rn(f.w, f.w));
}

// Rows [0, rows) at w are rows first_row.. of a matrix whose row count fixed
// the plan p (a row shard reduces exactly as in the whole matrix).
template <typename T>
__global__ void __launch_bounds__(512) row_rms_kernel(const T *__restrict__ w, int64_t rows, int64_t n,
                                                      int64_t first_row, const MeanPlan p,
                                                      float *__restrict__ sigma32,
                                                      uint16_t *__restrict__ sigma16) {
  __shared__ float red[512];
  pdl_enter();
  const int x = threadIdx.x, y = threadIdx.y;
  const int64_t row = p.split ? static_cast<int64_t>(blockIdx.x) : static_cast<int64_t>(blockIdx.x) * p.bh + y;
  const bool tail_owner = !p.split || y == 0;
  float v = 0.f;
  if (row < rows) {
    const T *data = w + row * n;
    const int64_t step = p.split ? static_cast<int64_t>(p.bw) * p.bh : p.bw;
    const int64_t idx0 = p.split ? x + static_cast<int64_t>(y) * p.bw : x;
    if (p.vec) {
      // Element misalignment of the row start (the matrix itself is 16-byte
      // aligned): the first 4 - shift elements are the head.
      int64_t end = n, base = 0;
      float a0 = 0.f;
      const int shift = static_cast<int>(((first_row + row) * n) & 3);
      if (shift > 0) {
        if (x >= shift && x < 4 && tail_owner) a0 = sq_at(data, x - shift);
        base = 4 - shift;
        end = n - base;
      }
      float a1 = 0.f, a2 = 0.f, a3 = 0.f;
      // Four vectors in flight per lane, added in the same order as one at a
      // time.
      int64_t i = idx0;
      for (; (i + 3 * step) * 4 + 3 < end; i += 4 * step) {
        float4 q[4];
#pragma unroll
        for (int k = 0; k < 4; ++k) q[k] = sq_vec4(data, base + (i + k * step) * 4);
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          a0 = __fadd_rn(a0, q[k].x);
          a1 = __fadd_rn(a1, q[k].y);
          a2 = __fadd_rn(a2, q[k].z);
          a3 = __fadd_rn(a3, q[k].w);
        }
      }
      for (; i * 4 + 3 < end; i += step) {
        const float4 q = sq_vec4(data, base + i * 4);
        a0 = __fadd_rn(a0, q.x);
        a1 = __fadd_rn(a1, q.y);
        a2 = __fadd_rn(a2, q.z);
        a3 = __fadd_rn(a3, q.w);
      }
      const int64_t tail = end - end % 4;
      if (tail_owner && tail + x < end) a0 = __fadd_rn(a0, sq_at(data, base + tail + x));
      v = __fadd_rn(__fadd_rn(__fadd_rn(a0, a1), a2), a3);
    } else {
      float acc[4] = {0.f, 0.f, 0.f, 0.f};
      int64_t i = idx0;
      for (; i + 3 * step < n; i += 4 * step) {
        float q[4];
#pragma unroll
        for (int k = 0; k < 4; ++k) q[k] = sq_at(data, i + k * step);
#pragma unroll
        for (int k = 0; k < 4; ++k) acc[k] = __fadd_rn(acc[k], q[k]);
      }
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        if (i >= n) break;
        acc[k] = __fadd_rn(acc[k], sq_at(data, i));
        i += step;
      }
      v = __fadd_rn(__fadd_rn(__fadd_rn(acc[0], acc[1]), acc[2]), acc[3]);
    }
  }
  // Lanes of a block row: shared-memory tree down to 32, then shuffles.
  int dim_x = p.bw;
  if (dim_x > 32) {
    const int base = x + y * p.bw;
    red[base] = v;
    for (int off = dim_x / 2; off >= 32; off >>= 1) {
      __syncthreads();
      if (x < off && x + off < p.bw) {
        v = __fadd_rn(v, red[base + off]);
        red[base] = v;
      }
    }
    dim_x = 32;
  }
  __syncthreads();
  // A block of fewer than 32 threads is a partial warp: shuffle among its lanes.
  const int nthreads = p.bw * p.bh;
  const unsigned mask = nthreads >= 32 ? 0xffffffffu : (1u << nthreads) - 1u;
  for (int off = dim_x >> 1; off > 0; off >>= 1) v = __fadd_rn(v, __shfl_down_sync(mask, v, off));
  if (p.split) {
    __syncthreads();
    const int base = x + y * p.bw;
    red[base] = v;
    for (int off = p.bh / 2; off > 0; off >>= 1) {
      __syncthreads();
      if (y < off && y + off < p.bh) {
        v = __fadd_rn(v, red[base + off * p.bw]);
        red[base] = v;
      }
    }
  }
  if (x == 0 && (!p.split || y == 0) && row < rows) {
    const float mean = __fmul_rn(v, p.factor);
    const float sg = __fsqrt_rn(__fadd_rn(mean, 1e-8f));
    if (sigma32) sigma32[row] = sg;
    if (sigma16) {
      // clamp_min keeps a NaN (torch's clamp propagates it).
      float s = __fmul_rn(sg, 3.4641016151377544f);
      s = isnan(s) ? s : fmaxf(s, 1e-8f);
      sigma16[row] = __half_as_ushort(__float2half_rn(s));
    }
  }
}

}  // namespace

int launch_row_rms(const void *w, int dtype, int64_t rows, int64_t n, int64_t matrix_rows,
                   int64_t first_row, float *sigma32, uint16_t *sigma16, cudaStream_t s) {
  if (rows <= 0) return H24_OK;
  if (n <= 0) return fail(H24_ERR_INVALID, "row_rms: in_features must be positive");
  if (first_row < 0 || first_row + rows > matrix_rows)
    return fail(H24_ERR_INVALID, "row_rms: rows outside the matrix");
  // The matrix starts 16-byte aligned: rows first_row.. start where they would.
  const size_t esize = dtype == H24_DTYPE_BF16 ? 2 : 4;
  if ((reinterpret_cast<uintptr_t>(w) - static_cast<uintptr_t>(first_row * n) * esize) & 15u)
    return fail(H24_ERR_INVALID, "row_rms: the matrix must be 16-byte aligned");
  const MeanPlan p = mean_plan(matrix_rows, n);
  const int64_t blocks = p.split ? rows : (rows + p.bh - 1) / p.bh;
  const dim3 block(p.bw, p.bh);
  // Launched with programmatic stream serialization (pdl_enter): the row
  // scales of consecutive matrices launch while the previous ones finish.
  const dim3 grid(static_cast<unsigned>(blocks));
  if (dtype == H24_DTYPE_BF16)
    H24_CUDA_TRY(launch_pdl(row_rms_kernel<__nv_bfloat16>, grid, block, s, static_cast<const __nv_bfloat16 *>(w),
                            rows, n, first_row, p, sigma32, sigma16));
  else if (dtype == H24_DTYPE_F32)
    H24_CUDA_TRY(launch_pdl(row_rms_kernel<float>, grid, block, s, static_cast<const float *>(w), rows, n,
                            first_row, p, sigma32, sigma16));
  else
    return fail(H24_ERR_INVALID, "row_rms: weights must be fp32 or bf16");
  count_launches(1);
  return H24_OK;
}

}  // namespace h24
