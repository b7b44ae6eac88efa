// h24_project.cu -- the H24 projection of pollux_step (pollux.py:874-884),
// fused and batched over parameters:
//   sigma_r  = sqrt(mean_c(w_rc^2) + 1e-8)                    fp32 per row
//   x        = (w / max(sigma_r, 1e-8)) / fp32(s_lattice)     fp32, two IEEE divisions
//   idx      = nearest codeword of every 24-atom of x, training rule (h24_search.cu)
//   p_rc     = fp32( fp32(cb32[idx][c % 24] * sigma_r) * fp32(s_lattice) )
// (normalize_matrix_by_row_rms, castor.py:316-333; castor_quantize_leech,
// castor.py:487-560; scale_matrix_by_row_rms, castor.py:336-339).  sigma is
// computed by the row-scale kernel of h24_rowrms.cu, in the summation order of
// torch's CUDA mean, so it is bit-identical to row_rms_from_matrix on a CUDA
// latent.
#include "h24_internal.cuh"

namespace h24 {
namespace {

constexpr int kThreads = 256;
constexpr int kWarps = kThreads / 32;
constexpr int kMaxBatch = 48;  // keeps the kernel parameter block under 4 KB

struct ProjBatch {
  h24_project_layer layer[kMaxBatch];
  int64_t row_start[kMaxBatch + 1];   // rows before each layer
  int64_t atom_start[kMaxBatch + 1];  // atoms before each layer
  int count;
};

__device__ __forceinline__ int find_layer(const ProjBatch &b, int64_t v, const int64_t *start) {
  int lo = 0, hi = b.count - 1;
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (start[mid] <= v) lo = mid; else hi = mid - 1;
  }
  return lo;
}

// One warp per row of every layer: the row's atoms of x into the shared
// scratch, from the row's sigma (already computed).
__global__ void __launch_bounds__(kThreads) project_prep_kernel(const __grid_constant__ ProjBatch b,
                                                                const float *__restrict__ sigma,
                                                                float *__restrict__ xs) {
  const int lane = threadIdx.x & 31;
  const int64_t total = b.row_start[b.count];
  const int64_t nwarps = static_cast<int64_t>(gridDim.x) * kWarps;
  for (int64_t gr = blockIdx.x * static_cast<int64_t>(kWarps) + (threadIdx.x >> 5); gr < total;
       gr += nwarps) {
    const int li = find_layer(b, gr, b.row_start);
    const h24_project_layer &L = b.layer[li];
    const int64_t r = gr - b.row_start[li];
    const float *row = L.latent + r * L.in_features;
    const float sg = sigma[gr];
    const float sgc = fmaxf(sg, 1e-8f);
    if (lane == 0 && L.sigma) L.sigma[r] = sg;
    float *xrow = xs + (b.atom_start[li] + r * (L.in_features / kDim)) * kDim;
    for (int64_t c = lane; c < L.in_features; c += 32)
      xrow[c] = __fdiv_rn(__fdiv_rn(__ldg(row + c), sgc), kSLatticeF);
  }
}

// p = (cb32[idx] * sigma) * s_lattice: one thread per (atom, 8-value part).
__global__ void __launch_bounds__(kThreads) project_store_kernel(const __grid_constant__ ProjBatch b,
                                                                 const float *__restrict__ sigma,
                                                                 const int32_t *__restrict__ idx,
                                                                 const int8_t *__restrict__ cb_raw) {
  const int64_t total = b.atom_start[b.count] * 3;
  for (int64_t t = blockIdx.x * static_cast<int64_t>(kThreads) + threadIdx.x; t < total;
       t += static_cast<int64_t>(gridDim.x) * kThreads) {
    const int64_t ga = t / 3;
    const int part = static_cast<int>(t - 3 * ga);
    const int li = find_layer(b, ga, b.atom_start);
    const h24_project_layer &L = b.layer[li];
    const int64_t la = ga - b.atom_start[li];
    const int64_t apr = L.in_features / kDim;
    const int64_t r = la / apr;
    const float sg = __ldg(sigma + b.row_start[li] + r);
    const int32_t k = __ldg(idx + ga);
    float o[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      const int raw = k > 0 ? cb_raw[static_cast<int64_t>(k - 1) * kDim + 8 * part + e] : 0;
      const float cb = static_cast<float>(raw) * kLeechScaleF;
      o[e] = __fmul_rn(__fmul_rn(cb, sg), kSLatticeF);
    }
    float *dst = L.out + la * kDim + 8 * part;
#pragma unroll
    for (int e = 0; e < 8; ++e) dst[e] = o[e];
    if (part == 0 && L.idx) L.idx[la] = k;
  }
}

// One resident wave of `kernel`, or fewer blocks when the work needs fewer.
template <typename K>
int grid_for(K kernel, int64_t work, int per_block) {
  return wave_grid((work + per_block - 1) / per_block, blocks_per_sm(kernel, kThreads, 0));
}

}  // namespace

int project_layers(const Tables *t, const h24_project_layer *layers, int count, cudaStream_t s) {
  for (int base = 0; base < count; base += kMaxBatch) {
    ProjBatch b;
    b.count = 0;
    b.row_start[0] = 0;
    b.atom_start[0] = 0;
    for (int i = base; i < count && b.count < kMaxBatch; ++i) {
      const h24_project_layer &L = layers[i];
      if (L.rows < 0 || L.in_features <= 0 || L.in_features % kDim != 0)
        return fail(H24_ERR_INVALID, "project: in_features must be a positive multiple of 24");
      if (L.rows == 0) continue;
      if (!L.latent || !L.out) return fail(H24_ERR_INVALID, "project: null pointer");
      b.layer[b.count] = L;
      b.row_start[b.count + 1] = b.row_start[b.count] + L.rows;
      b.atom_start[b.count + 1] = b.atom_start[b.count] + L.rows * (L.in_features / kDim);
      ++b.count;
    }
    if (b.count == 0) continue;
    const int64_t rows = b.row_start[b.count], atoms = b.atom_start[b.count];
    auto up = [](size_t v) { return (v + 255) & ~static_cast<size_t>(255); };
    const size_t off_x = up(static_cast<size_t>(rows) * 4);
    const size_t off_idx = off_x + up(static_cast<size_t>(atoms) * kDim * 4);
    uint8_t *scratch = nullptr;
    H24_CUDA_TRY(cudaMallocFromPoolAsync(reinterpret_cast<void **>(&scratch),
                                         off_idx + up(static_cast<size_t>(atoms) * 4), t->pool, s));
    float *sigma = reinterpret_cast<float *>(scratch);
    float *xs = reinterpret_cast<float *>(scratch + off_x);
    int32_t *idx = reinterpret_cast<int32_t *>(scratch + off_idx);
    int rc = H24_OK;
    for (int i = 0; i < b.count && rc == H24_OK; ++i) {
      if (!aligned16(b.layer[i].latent)) rc = fail(H24_ERR_INVALID, "project: latent must be 16-byte aligned");
      else rc = launch_row_rms(b.layer[i].latent, H24_DTYPE_F32, b.layer[i].rows, b.layer[i].in_features,
                               b.layer[i].rows, 0, sigma + b.row_start[i], nullptr, s);
    }
    cudaError_t le = cudaSuccess;
    if (rc == H24_OK) {
      project_prep_kernel<<<grid_for(project_prep_kernel, rows, kWarps), kThreads, 0, s>>>(b, sigma, xs);
      le = cudaGetLastError();
      if (le != cudaSuccess) rc = cuda_fail(le, "project_prep launch");
    }
    if (rc == H24_OK) {
      count_launches(1);
      rc = quantize(t, xs, atoms, H24_RULE_TRAIN, idx, s);
    }
    if (rc == H24_OK) {
      project_store_kernel<<<grid_for(project_store_kernel, atoms * 3, kThreads), kThreads, 0, s>>>(b, sigma, idx, t->cb_raw);
      le = cudaGetLastError();
      if (le != cudaSuccess) rc = cuda_fail(le, "project_store launch");
      else count_launches(1);
    }
    const cudaError_t e = cudaFreeAsync(scratch, s);
    if (rc != H24_OK) return rc;
    H24_CUDA_TRY(e);
  }
  return H24_OK;
}

}  // namespace h24
