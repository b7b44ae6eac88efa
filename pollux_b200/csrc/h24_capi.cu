// h24_capi.cu -- extern "C" entry points of libh24 (declared in include/h24.h),
// per-device codebook tables, error reporting and instrumentation, plus the
// pack-rule row-scale kernel.
#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <cstdlib>
#include <cstring>
#include <atomic>
#include <mutex>
#include <unordered_map>
#include <string>
#include <utility>
#include <vector>

#include "h24_internal.cuh"

namespace h24 {

// ---------------------------------------------------------------------------
// errors
// ---------------------------------------------------------------------------
namespace {
thread_local std::string t_last_error;
}

const char *last_error_cstr() { return t_last_error.c_str(); }

void set_error(const std::string &msg) { t_last_error = msg; }

int fail(int code, const std::string &msg) {
  t_last_error = msg;
  return code;
}

int cuda_fail(cudaError_t e, const char *what) {
  t_last_error = std::string(what) + ": " + cudaGetErrorString(e);
  return H24_ERR_CUDA;
}

// ---------------------------------------------------------------------------
// codebook tables
// ---------------------------------------------------------------------------
namespace {

constexpr int kMaxDevices = 64;
std::mutex g_tables_mu;
Tables g_tables[kMaxDevices];
bool g_tables_ok[kMaxDevices] = {};

struct HostTables {
  std::vector<int8_t> raw;         // [kKissing][24]
  std::vector<uint16_t> golay;     // [kGolay][32] bf16 bits, tiled (Tables::golay_tiled)
  std::vector<uint32_t> golay_mask;  // [kGolay]
  std::vector<int32_t> idx3, idx2, idx1;
  std::vector<uint32_t> oct_by_triple;  // [kTriples][kTripleRow][2]
  std::vector<uint32_t> nib;       // [kCount][4] dequant codes
  float fingerprint[16];
  bool ok = false;
  std::string err;
};

uint16_t bf16_bits_of_int(int v) {
  // Small integers are exact in bf16: the top half of their fp32 pattern.
  const float f = static_cast<float>(v);
  uint32_t u;
  std::memcpy(&u, &f, 4);
  return static_cast<uint16_t>(u >> 16);
}

// Decomposes the kissing points into the three types (see h24_internal.cuh)
// and fills the Golay operand and the index maps.  Fails, with a message,
// if the codebook does not have that structure.
bool build_structure(HostTables &H) {
  // Type 3: the sign word w (bit i = coordinate i negative) and the position
  // p of the -3.  The Golay codeword is w or w ^ (1 << p); it is the one of
  // the two that occurs for all 24 positions.
  std::unordered_map<uint32_t, int> seen;
  std::vector<std::pair<uint32_t, int>> t3;  // (w, p) per type-3 point, with j
  std::vector<int> t3j;
  for (int j = 0; j < kKissing; ++j) {
    const int8_t *r = &H.raw[static_cast<size_t>(j) * kDim];
    int p = -1, maxabs = 0;
    uint32_t w = 0;
    for (int i = 0; i < kDim; ++i) {
      maxabs = std::max(maxabs, std::abs(int(r[i])));
      if (r[i] < 0) w |= 1u << i;
      if (r[i] == -3) p = i;
    }
    if (maxabs == 3) {
      if (p < 0) { H.err = "type-3 point without a -3"; return false; }
      t3.emplace_back(w, p);
      t3j.push_back(j);
      ++seen[w];
      ++seen[w ^ (1u << p)];
    }
  }
  std::vector<uint32_t> golay;
  for (const auto &kv : seen)
    if (kv.second == kDim) golay.push_back(kv.first);
  if (golay.size() != static_cast<size_t>(kGolay) || t3.size() != static_cast<size_t>(kGolay) * kDim) {
    H.err = "type-3 points do not form Golay codeword x position pairs";
    return false;
  }
  std::sort(golay.begin(), golay.end(), [](uint32_t a, uint32_t b) {
    const int wa = __builtin_popcount(a), wb = __builtin_popcount(b);
    return wa != wb ? wa < wb : a < b;
  });
  // Complement-paired column order (see h24_internal.cuh): the first half
  // from the zero word, the octads (as complements of the sorted weight-16
  // words) and the smaller dodecad of each pair; column c + 2048 = ~column c.
  {
    std::vector<uint32_t> w16, dodec;
    for (const uint32_t w : golay) {
      const int wt = __builtin_popcount(w);
      if (wt == 16) w16.push_back(w);
      if (wt == 12 && w < (~w & 0xFFFFFFu)) dodec.push_back(w);
    }
    if (w16.size() != static_cast<size_t>(kOctads) || dodec.size() != static_cast<size_t>(kGolayHalf - 1 - kOctads)) {
      H.err = "unexpected Golay weight distribution";
      return false;
    }
    std::vector<uint32_t> order;
    order.push_back(0);
    for (const uint32_t w : w16) order.push_back(~w & 0xFFFFFFu);
    for (const uint32_t w : dodec) order.push_back(w);
    for (int c = 0; c < kGolayHalf; ++c) order.push_back(~order[c] & 0xFFFFFFu);
    golay.swap(order);
  }
  std::unordered_map<uint32_t, int> col;
  for (int c = 0; c < kGolay; ++c) col[golay[c]] = c;
  if (col.size() != static_cast<size_t>(kGolay) || __builtin_popcount(golay[kW16First]) != 16 ||
      __builtin_popcount(golay[kGolayHalf]) != 24 || __builtin_popcount(golay[kW16First + kOctads - 1]) != 16 ||
      __builtin_popcount(golay[kW16First + kOctads]) != 12 || __builtin_popcount(golay[kOctads]) != 8) {
    H.err = "unexpected Golay weight distribution";
    return false;
  }
  H.golay_mask = golay;
  H.idx3.assign(static_cast<size_t>(kGolay) * kDim, -1);
  for (size_t k = 0; k < t3.size(); ++k) {
    const uint32_t w = t3[k].first;
    const int p = t3[k].second;
    auto it = col.find(w);
    if (it == col.end()) it = col.find(w ^ (1u << p));
    if (it == col.end()) { H.err = "type-3 point outside the Golay code"; return false; }
    H.idx3[static_cast<size_t>(it->second) * kDim + p] = t3j[k];
  }
  // Types 1 and 2.
  H.idx2.assign(static_cast<size_t>(kOctads) * 128, -1);
  H.idx1.assign(static_cast<size_t>(kDim) * kDim * 4, -1);
  for (int j = 0; j < kKissing; ++j) {
    const int8_t *r = &H.raw[static_cast<size_t>(j) * kDim];
    int maxabs = 0;
    uint32_t nz = 0;
    for (int i = 0; i < kDim; ++i) {
      maxabs = std::max(maxabs, std::abs(int(r[i])));
      if (r[i] != 0) nz |= 1u << i;
    }
    if (maxabs == 2) {
      const auto it = col.find(~nz & 0xFFFFFFu);
      const int o = it == col.end() ? -1 : it->second - kW16First;
      if (o < 0 || o >= kOctads || __builtin_popcount(nz) != 8) { H.err = "type-2 support is not an octad"; return false; }
      int s = 0, k = 0, minus = 0;
      for (int i = 0; i < kDim; ++i)
        if (nz >> i & 1) {
          if (r[i] < 0) { ++minus; if (k < 7) s |= 1 << k; }
          ++k;
        }
      if (minus & 1) { H.err = "type-2 point with an odd number of minus signs"; return false; }
      H.idx2[static_cast<size_t>(o) * 128 + s] = j;
    } else if (maxabs == 4) {
      int a = -1, b = -1;
      for (int i = 0; i < kDim; ++i)
        if (r[i] != 0) (a < 0 ? a : b) = i;
      if (b < 0 || __builtin_popcount(nz) != 2) { H.err = "type-1 point without two nonzeros"; return false; }
      const int s = (r[a] < 0) | ((r[b] < 0) << 1);
      H.idx1[(static_cast<size_t>(a) * kDim + b) * 4 + s] = j;
    }
  }
  for (const int32_t v : H.idx3) if (v < 0) { H.err = "missing type-3 point"; return false; }
  for (const int32_t v : H.idx2) if (v < 0) { H.err = "missing type-2 point"; return false; }
  int t1 = 0;
  for (const int32_t v : H.idx1) t1 += v >= 0;
  if (t1 != 276 * 4) { H.err = "missing type-1 point"; return false; }
  // The 21 octads through each position triple (Steiner system S(5,8,24)).
  H.oct_by_triple.assign(static_cast<size_t>(kTriples) * kTripleRow * 2, 0);
  {
    std::vector<int> fill(kTriples, 0);
    const auto c3 = [](int k) { return k * (k - 1) * (k - 2) / 6; };
    const auto c2 = [](int j) { return j * (j - 1) / 2; };
    for (int o = 0; o < kOctads; ++o) {
      const uint32_t om = ~golay[kW16First + o] & 0xFFFFFFu;
      for (int k = 2; k < kDim; ++k)
        for (int j = 1; j < k; ++j)
          for (int i = 0; i < j; ++i)
            if ((om >> i & 1) && (om >> j & 1) && (om >> k & 1)) {
              const int t = c3(k) + c2(j) + i;
              if (fill[t] >= 21) { H.err = "more than 21 octads through a triple"; return false; }
              uint32_t rest = 0;
              int nr = 0;
              for (int q = 0; q < kDim; ++q)
                if ((om >> q & 1) && q != i && q != j && q != k) rest |= static_cast<uint32_t>(q) << (5 * nr++);
              const size_t e = (static_cast<size_t>(t) * kTripleRow + fill[t]++) * 2;
              H.oct_by_triple[e] = om;
              H.oct_by_triple[e + 1] = rest;
            }
    }
    for (int t = 0; t < kTriples; ++t)
      if (fill[t] != 21) { H.err = "a position triple is not in 21 octads"; return false; }
  }
  // B operand: column c = (-1)^c_k, canonical tiled layout.
  H.golay.assign(static_cast<size_t>(kGolay) * kKPad, 0);
  for (int c = 0; c < kGolay; ++c) {
    const int t = c / kGolayTileN, cc = c % kGolayTileN, g = cc / 8, rr = cc % 8;
    for (int k = 0; k < kDim; ++k) {
      const size_t byte = static_cast<size_t>(t) * kGolayTileN * kRowBytes + g * 512 + (k / 8) * 128 +
                          rr * 16 + (k % 8) * 2;
      H.golay[byte / 2] = bf16_bits_of_int((golay[c] >> k & 1) ? -1 : 1);
    }
  }
  return true;
}

const HostTables &host_tables() {
  static HostTables H;
  static std::once_flag once;
  std::call_once(once, [] {
    H.raw.resize(static_cast<size_t>(kKissing) * kDim);
    if (!build_raw_kissing_points(H.raw.data(), &H.err)) return;
    if (!build_structure(H)) return;
    // Dequant codes, 16 bytes per codeword (word k = elements 8k..8k+7, one
    // nibble each; word 3 is zero).  A codeword takes at most four distinct
    // values, fixed by its type: {+1,-1,+3,-3} (one 3, 23 ones), {0,+2,-2}
    // (eight twos; also the origin) or {0,+4,-4} (two fours).  Nibble bits
    // 0-1 index the type's value list (dequant_value_lists in h24_dequant.cu
    // holds the same orders), bit 2 of nibbles 0 and 1 of every word holds
    // the list selector (0, 1, 2), bit 3 stays zero.
    H.nib.assign(static_cast<size_t>(kCount) * 4, 0);
    for (int row = 0; row < kCount && H.err.empty(); ++row) {
      const int8_t *cw = row == 0 ? nullptr : &H.raw[static_cast<size_t>(row - 1) * kDim];
      int maxabs = 0;
      for (int k = 0; k < kDim; ++k) maxabs = std::max(maxabs, cw ? std::abs(int(cw[k])) : 0);
      const int list = maxabs == 4 ? 2 : (maxabs == 3 ? 0 : 1);
      for (int k = 0; k < kDim; ++k) {
        const int raw = cw ? cw[k] : 0;
        int code = -1;
        if (list == 0) code = raw == 1 ? 0 : raw == -1 ? 1 : raw == 3 ? 2 : raw == -3 ? 3 : -1;
        if (list == 1) code = raw == 0 ? 0 : raw == 2 ? 1 : raw == -2 ? 2 : -1;
        if (list == 2) code = raw == 0 ? 3 : raw == 4 ? 1 : raw == -4 ? 2 : -1;
        if (code < 0) {
          H.err = "codeword " + std::to_string(row) + " mixes value types";
          break;
        }
        const int e = k % 8;
        uint32_t nib = static_cast<uint32_t>(code);
        if (e == 0) nib |= static_cast<uint32_t>(list & 1) << 2;
        if (e == 1) nib |= static_cast<uint32_t>(list >> 1) << 2;
        H.nib[static_cast<size_t>(row) * 4 + k / 8] |= nib << (4 * e);
      }
    }
    if (!H.err.empty()) return;
    for (int r = 0; r < 4; ++r)
      for (int c = 0; c < 4; ++c)
        H.fingerprint[r * 4 + c] =
            r == 0 ? 0.f
                   : static_cast<float>(H.raw[static_cast<size_t>(r - 1) * kDim + c]) * kLeechScaleF;
    H.ok = true;
  });
  return H;
}

int build_device_tables(int dev, Tables *T) {
  const HostTables &H = host_tables();
  if (!H.ok) return fail(H24_ERR_STATE, "codebook construction failed: " + H.err);
  void *p = nullptr;
  const auto upload = [&p](const void *src, size_t bytes) -> int {
    H24_CUDA_TRY(cudaMalloc(&p, bytes));
    H24_CUDA_TRY(cudaMemcpy(p, src, bytes, cudaMemcpyHostToDevice));
    return H24_OK;
  };
  int rc = upload(H.golay.data(), H.golay.size() * sizeof(uint16_t));
  if (rc != H24_OK) return rc;
  T->golay_tiled = static_cast<const __nv_bfloat16 *>(p);
  if ((rc = upload(H.golay_mask.data(), H.golay_mask.size() * 4)) != H24_OK) return rc;
  T->golay_mask = static_cast<const uint32_t *>(p);
  if ((rc = upload(H.idx3.data(), H.idx3.size() * 4)) != H24_OK) return rc;
  T->idx3 = static_cast<const int32_t *>(p);
  if ((rc = upload(H.idx2.data(), H.idx2.size() * 4)) != H24_OK) return rc;
  T->idx2 = static_cast<const int32_t *>(p);
  if ((rc = upload(H.idx1.data(), H.idx1.size() * 4)) != H24_OK) return rc;
  T->idx1 = static_cast<const int32_t *>(p);
  if ((rc = upload(H.oct_by_triple.data(), H.oct_by_triple.size() * 4)) != H24_OK) return rc;
  T->oct_by_triple = static_cast<const uint2 *>(p);
  H24_CUDA_TRY(cudaMalloc(&p, H.raw.size()));
  H24_CUDA_TRY(cudaMemcpy(p, H.raw.data(), H.raw.size(), cudaMemcpyHostToDevice));
  T->cb_raw = static_cast<const int8_t *>(p);
  H24_CUDA_TRY(cudaMalloc(&p, H.nib.size() * sizeof(uint32_t)));
  H24_CUDA_TRY(
      cudaMemcpy(p, H.nib.data(), H.nib.size() * sizeof(uint32_t), cudaMemcpyHostToDevice));
  T->cb_nib = static_cast<const uint32_t *>(p);
  H24_CUDA_TRY(cudaMalloc(&p, 3 * sizeof(int64_t) + 16));
  H24_CUDA_TRY(cudaMemset(p, 0, 3 * sizeof(int64_t) + 16));
  T->stats = static_cast<int64_t *>(p);
  T->err = reinterpret_cast<int *>(static_cast<char *>(p) + 3 * sizeof(int64_t));
  cudaMemPoolProps props = {};
  props.allocType = cudaMemAllocationTypePinned;
  props.handleTypes = cudaMemHandleTypeNone;
  props.location.type = cudaMemLocationTypeDevice;
  props.location.id = dev;
  H24_CUDA_TRY(cudaMemPoolCreate(&T->pool, &props));
  uint64_t keep = ~uint64_t(0);
  H24_CUDA_TRY(cudaMemPoolSetAttribute(T->pool, cudaMemPoolAttrReleaseThreshold, &keep));
  H24_CUDA_TRY(cudaStreamCreateWithFlags(&T->copy_stream, cudaStreamNonBlocking));
  H24_CUDA_TRY(cudaStreamCreateWithFlags(&T->d2h_stream, cudaStreamNonBlocking));
  std::memcpy(T->fingerprint, H.fingerprint, sizeof(T->fingerprint));
  T->device = dev;
  return H24_OK;
}

}  // namespace

const Tables *tables_for_current_device() {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) {
    cuda_fail(e, "cudaGetDevice");
    return nullptr;
  }
  if (dev < 0 || dev >= kMaxDevices) {
    set_error("device ordinal out of range");
    return nullptr;
  }
  std::lock_guard<std::mutex> lk(g_tables_mu);
  if (!g_tables_ok[dev]) {
    if (build_device_tables(dev, &g_tables[dev]) != H24_OK) return nullptr;
    g_tables_ok[dev] = true;
  }
  return &g_tables[dev];
}

// Tables of the current device if they are already built, else nullptr; never
// allocates (used by the allocation-free entry point).
const Tables *tables_if_ready() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return nullptr;
  std::lock_guard<std::mutex> lk(g_tables_mu);
  return g_tables_ok[dev] ? &g_tables[dev] : nullptr;
}

// ---------------------------------------------------------------------------
// instrumentation
// ---------------------------------------------------------------------------
namespace {
std::mutex g_timing_mu;
bool g_timing = false;
// Recorded (start, stop) event pairs per instrumented kernel (H24_KERNEL_*).
std::vector<std::pair<cudaEvent_t, cudaEvent_t>> g_events[H24_KERNEL_COUNT];
}  // namespace

namespace {
std::atomic<int64_t> g_launches{0};
}

void count_launches(int64_t k) { g_launches.fetch_add(k, std::memory_order_relaxed); }

bool timing_enabled() {
  std::lock_guard<std::mutex> lk(g_timing_mu);
  return g_timing;
}

void timing_record(int kernel, cudaEvent_t start, cudaEvent_t stop) {
  std::lock_guard<std::mutex> lk(g_timing_mu);
  g_events[kernel].emplace_back(start, stop);
}

}  // namespace h24

// ===========================================================================
// extern "C" API
// ===========================================================================
using namespace h24;

#define H24_TABLES_OR_FAIL(T)                       \
  const Tables *T = tables_for_current_device();    \
  if (!T) return H24_ERR_STATE

static cudaStream_t as_stream(void *s) { return static_cast<cudaStream_t>(s); }

// Reads the device error word of T's device after the work on `s` (which it
// synchronises) and clears it: H24_ERR_TIMEOUT if a bounded wait inside the
// screening kernel or the LUT GEMV ran out, else H24_OK.
static int take_device_error(const Tables *T, cudaStream_t s) {
  int err = 0;
  H24_CUDA_TRY(cudaMemcpyAsync(&err, T->err, sizeof(int), cudaMemcpyDeviceToHost, s));
  H24_CUDA_TRY(cudaStreamSynchronize(s));
  if (err != 0) {
    H24_CUDA_TRY(cudaMemsetAsync(T->err, 0, sizeof(int), s));
    H24_CUDA_TRY(cudaStreamSynchronize(s));
    return fail(H24_ERR_TIMEOUT, "a bounded wait in a tensor-core kernel ran out");
  }
  return H24_OK;
}

extern "C" {

const char *h24_last_error(void) { return last_error_cstr(); }

const char *h24_version(void) { return "h24-b200 0.1 (sm_100a, tcgen05)"; }

int h24_init(int device) {
  int prev = 0;
  H24_CUDA_TRY(cudaGetDevice(&prev));
  H24_CUDA_TRY(cudaSetDevice(device));
  const Tables *t = tables_for_current_device();
  cudaSetDevice(prev);
  return t ? H24_OK : H24_ERR_STATE;
}

int h24_codebook_raw(int8_t *out_host) {
  if (!out_host) return fail(H24_ERR_INVALID, "codebook_raw: null pointer");
  const HostTables &H = host_tables();
  if (!H.ok) return fail(H24_ERR_STATE, "codebook construction failed: " + H.err);
  std::memcpy(out_host, H.raw.data(), H.raw.size());
  return H24_OK;
}

int h24_codebook_f32(float *out, void *stream) {
  H24_TABLES_OR_FAIL(T);
  if (!out) return fail(H24_ERR_INVALID, "codebook_f32: null pointer");
  // Row 0 is the origin; rows 1.. are the kissing points.
  H24_CUDA_TRY(cudaMemsetAsync(out, 0, kDim * sizeof(float), as_stream(stream)));
  count_launches(0);
  return launch_codebook_f32(T, out + kDim, as_stream(stream));
}

int h24_fingerprint(float out16[16]) {
  H24_TABLES_OR_FAIL(T);
  if (!out16) return fail(H24_ERR_INVALID, "fingerprint: null pointer");
  std::memcpy(out16, T->fingerprint, 16 * sizeof(float));
  return H24_OK;
}

int h24_pack(const int32_t *idx, int64_t n, uint8_t *out, void *stream) {
  if (n < 0) return fail(H24_ERR_INVALID, "pack: negative length");
  if (n > 0 && (!idx || !out)) return fail(H24_ERR_INVALID, "pack: null pointer");
  return launch_pack_i32(idx, n, out, as_stream(stream));
}

int h24_pack_i64(const int64_t *idx, int64_t n, uint8_t *out, void *stream) {
  if (n < 0) return fail(H24_ERR_INVALID, "pack: negative length");
  if (n > 0 && (!idx || !out)) return fail(H24_ERR_INVALID, "pack: null pointer");
  return launch_pack_i64(idx, n, out, as_stream(stream));
}

int h24_unpack(const uint8_t *packed, int64_t groups, int64_t n, int32_t *out, void *stream) {
  if (n < 0 || groups < 0) return fail(H24_ERR_INVALID, "unpack: negative size");
  if (n > 0 && groups > 0 && (!packed || !out)) return fail(H24_ERR_INVALID, "unpack: null pointer");
  return launch_unpack_i32(packed, groups, n, out, as_stream(stream));
}

int h24_unpack_i64(const uint8_t *packed, int64_t groups, int64_t n, int64_t *out, void *stream) {
  if (n < 0 || groups < 0) return fail(H24_ERR_INVALID, "unpack: negative size");
  if (n > 0 && groups > 0 && (!packed || !out)) return fail(H24_ERR_INVALID, "unpack: null pointer");
  return launch_unpack_i64(packed, groups, n, out, as_stream(stream));
}

int h24_dequant(const uint8_t *packed, const uint16_t *sigma16, int64_t rows, int64_t in_features,
                uint16_t *out16, int32_t *bad_count, void *stream) {
  H24_TABLES_OR_FAIL(T);
  h24_dequant_layer L{packed, sigma16, out16, rows, in_features};
  return launch_dequant(T, nullptr, &L, 1, bad_count, as_stream(stream));
}

int h24_dequant_batched(const h24_dequant_layer *layers, int count, int32_t *bad_count,
                        void *stream) {
  H24_TABLES_OR_FAIL(T);
  if (count < 0 || (count > 0 && !layers)) return fail(H24_ERR_INVALID, "dequant_batched: bad layer list");
  return launch_dequant(T, nullptr, layers, count, bad_count, as_stream(stream));
}

int h24_project_layers(const h24_project_layer *layers, int count, void *stream) {
  H24_TABLES_OR_FAIL(T);
  if (count < 0 || (count > 0 && !layers)) return fail(H24_ERR_INVALID, "project_layers: bad layer list");
  for (int i = 0; i < count; ++i)
    if (layers[i].rows > 0 && layers[i].latent && !aligned16(layers[i].latent))
      return fail(H24_ERR_INVALID, "project_layers: latent must be 16-byte aligned");
  return project_layers(T, layers, count, as_stream(stream));
}

int h24_lut_gemv(const uint8_t *packed, const uint16_t *sigma16, int64_t rows,
                 int64_t in_features, const float *x, int64_t batch, float *y,
                 int32_t *bad_count, void *stream) {
  H24_TABLES_OR_FAIL(T);
  return launch_lut_gemv(T, packed, sigma16, rows, in_features, x, batch, y, bad_count,
                         as_stream(stream));
}

int h24_int8_quantize(const float *w, int64_t rows, int64_t cols, int8_t *q, uint16_t *mu16,
                      void *stream) {
  if (rows < 0 || cols < 0) return fail(H24_ERR_INVALID, "int8_quantize: negative size");
  if (rows > 0 && cols > 0 && (!w || !q || !mu16)) return fail(H24_ERR_INVALID, "int8_quantize: null pointer");
  return launch_int8_quantize(w, rows, cols, q, mu16, as_stream(stream));
}

int h24_int8_dequant(const int8_t *q, const uint16_t *mu16, int64_t rows, int64_t cols,
                     uint16_t *out16, void *stream) {
  if (rows < 0 || cols < 0) return fail(H24_ERR_INVALID, "int8_dequant: negative size");
  if (rows > 0 && cols > 0 && (!q || !mu16 || !out16)) return fail(H24_ERR_INVALID, "int8_dequant: null pointer");
  return launch_int8_dequant(q, mu16, rows, cols, out16, as_stream(stream));
}

int h24_quantize(const float *x, int64_t n, int rule, int32_t *out_idx, void *stream) {
  H24_TABLES_OR_FAIL(T);
  if (n < 0) return fail(H24_ERR_INVALID, "quantize: negative atom count");
  if (rule != H24_RULE_TRAIN && rule != H24_RULE_PACK)
    return fail(H24_ERR_INVALID, "quantize: unknown rule");
  if (n == 0) return H24_OK;
  if (!x || !out_idx) return fail(H24_ERR_INVALID, "quantize: null pointer");
  if (!aligned16(x)) return fail(H24_ERR_INVALID, "quantize: x must be 16-byte aligned");
  return quantize(T, x, n, rule, out_idx, as_stream(stream));
}

int h24_quantize_typed(const void *x, int64_t n, int dtype, int rule, int32_t *out_idx, void *stream) {
  H24_TABLES_OR_FAIL(T);
  if (n < 0) return fail(H24_ERR_INVALID, "quantize: negative atom count");
  if (rule != H24_RULE_TRAIN && rule != H24_RULE_PACK)
    return fail(H24_ERR_INVALID, "quantize: unknown rule");
  if (n == 0) return H24_OK;
  if (!x || !out_idx) return fail(H24_ERR_INVALID, "quantize: null pointer");
  if (!aligned16(x)) return fail(H24_ERR_INVALID, "quantize: x must be 16-byte aligned");
  return quantize_segments(T, &x, &n, 1, dtype, rule, out_idx, as_stream(stream));
}

int h24_row_rms(const void *w, int64_t rows, int64_t in_features, int dtype, float *sigma_out,
                uint16_t *sigma16_out, void *stream) {
  if (rows < 0) return fail(H24_ERR_INVALID, "row_rms: negative row count");
  if (rows > 0 && (!w || (!sigma_out && !sigma16_out))) return fail(H24_ERR_INVALID, "row_rms: null pointer");
  return launch_row_rms(w, dtype, rows, in_features, rows, 0, sigma_out, sigma16_out, as_stream(stream));
}

int h24_quantize_segments(const float *const *xs, const int64_t *counts, int nseg, int rule,
                          int32_t *out_idx, void *stream) {
  H24_TABLES_OR_FAIL(T);
  if (nseg < 0 || (nseg > 0 && (!xs || !counts)))
    return fail(H24_ERR_INVALID, "quantize_segments: bad segment list");
  if (rule != H24_RULE_TRAIN && rule != H24_RULE_PACK)
    return fail(H24_ERR_INVALID, "quantize_segments: unknown rule");
  int64_t total = 0;
  for (int i = 0; i < nseg; ++i) total += counts[i] > 0 ? counts[i] : 0;
  if (total > 0 && !out_idx) return fail(H24_ERR_INVALID, "quantize_segments: null output");
  std::vector<const void *> xv(xs, xs + nseg);
  return quantize_segments(T, xv.data(), counts, nseg, H24_DTYPE_F32, rule, out_idx, as_stream(stream));
}

// A validated row range of one layer: rows [r0, r1) of a rows x in matrix,
// whose atoms start on a 4-index group and end on one (or at the matrix end).
struct RowRange {
  const uint8_t *w;  // the whole matrix
  int64_t rows, in, r0, r1;
  uint16_t *sigma16;
  uint8_t *packed;
  int64_t atoms() const { return (r1 - r0) * in / kDim; }
};

static int validate_rows(const h24_layer_rows &L, size_t esize, bool host, RowRange *out) {
  if (L.rows < 0 || L.in_features <= 0 || (L.rows * L.in_features) % kDim != 0)
    return fail(H24_ERR_INVALID, "quantize_layer: rows*in_features must be a multiple of 24");
  if (L.row_begin < 0 || L.row_end < L.row_begin || L.row_end > L.rows)
    return fail(H24_ERR_INVALID, "quantize_layer: row range outside the matrix");
  const int64_t a0 = L.row_begin * L.in_features, a1 = L.row_end * L.in_features;
  if (a0 % (4 * kDim) != 0 || (L.row_end != L.rows && a1 % (4 * kDim) != 0))
    return fail(H24_ERR_INVALID,
                "quantize_layer: a row range must start and end on a whole 9-byte group of 4 atoms");
  if (L.row_end > L.row_begin) {
    if (!L.w || !L.sigma16_out || !L.packed_out) return fail(H24_ERR_INVALID, "quantize_layer: null pointer");
    if (!host && !aligned16(L.w)) return fail(H24_ERR_INVALID, "quantize_layer: w must be 16-byte aligned");
  }
  *out = RowRange{static_cast<const uint8_t *>(L.w), L.rows, L.in_features, L.row_begin, L.row_end,
                  L.sigma16_out, L.packed_out};
  (void)esize;
  return H24_OK;
}

// Pack-rule quantisation of device-resident row ranges: row scales, one
// shared search pipeline over all ranges, then the 18-bit pack of each.
static int quantize_ranges(const Tables *T, const std::vector<RowRange> &R, int dtype, cudaStream_t s) {
  const size_t esize = dtype == H24_DTYPE_BF16 ? 2 : 4;
  std::vector<const void *> xs;
  std::vector<int64_t> counts;
  int64_t total = 0;
  for (const RowRange &r : R) {
    xs.push_back(r.w + static_cast<size_t>(r.r0 * r.in) * esize);
    counts.push_back(r.atoms());
    total += r.atoms();
  }
  if (total == 0) return H24_OK;
  for (const RowRange &r : R) {
    int rc = launch_row_rms(r.w + static_cast<size_t>(r.r0 * r.in) * esize, dtype, r.r1 - r.r0, r.in, r.rows,
                            r.r0, nullptr, r.sigma16, s);
    if (rc != H24_OK) return rc;
  }
  int32_t *idx = nullptr;
  H24_CUDA_TRY(cudaMallocFromPoolAsync(reinterpret_cast<void **>(&idx),
                                       static_cast<size_t>(total) * sizeof(int32_t), T->pool, s));
  int rc = quantize_segments(T, xs.data(), counts.data(), static_cast<int>(xs.size()), dtype,
                             H24_RULE_PACK, idx, s);
  int64_t off = 0;
  for (size_t i = 0; i < R.size() && rc == H24_OK; ++i) {
    rc = launch_pack_i32(idx + off, counts[i], R[i].packed, s);
    off += counts[i];
  }
  cudaError_t e = cudaFreeAsync(idx, s);
  if (rc == H24_OK && e != cudaSuccess) rc = cuda_fail(e, "cudaFreeAsync");
  return rc;
}

int h24_quantize_layer_rows(const h24_layer_rows *layers, int count, int dtype, void *stream) {
  H24_TABLES_OR_FAIL(T);
  if (count < 0 || (count > 0 && !layers)) return fail(H24_ERR_INVALID, "quantize_layers: bad list");
  if (dtype != H24_DTYPE_F32 && dtype != H24_DTYPE_BF16)
    return fail(H24_ERR_INVALID, "quantize_layers: weights must be fp32 or bf16");
  const size_t esize = dtype == H24_DTYPE_BF16 ? 2 : 4;
  std::vector<RowRange> R(count);
  for (int i = 0; i < count; ++i) {
    int rc = validate_rows(layers[i], esize, false, &R[i]);
    if (rc != H24_OK) return rc;
  }
  // Segments of the pipeline must be 16-byte aligned: a range starting inside
  // the matrix starts at a multiple of 96 elements, so it is if w is.
  return quantize_ranges(T, R, dtype, as_stream(stream));
}

int h24_quantize_layers(const h24_layer *layers, int count, void *stream) {
  if (count < 0 || (count > 0 && !layers)) return fail(H24_ERR_INVALID, "quantize_layers: bad list");
  std::vector<h24_layer_rows> L(count);
  for (int i = 0; i < count; ++i)
    L[i] = h24_layer_rows{layers[i].w, layers[i].rows, layers[i].in_features, 0, layers[i].rows,
                          layers[i].sigma16_out, layers[i].packed_out};
  return h24_quantize_layer_rows(L.data(), count, H24_DTYPE_F32, stream);
}

int h24_quantize_layer(const float *w, int64_t rows, int64_t in_features, uint16_t *sigma16_out,
                       uint8_t *packed_out, void *stream) {
  h24_layer L{w, rows, in_features, sigma16_out, packed_out};
  return h24_quantize_layers(&L, 1, stream);
}

// Host-memory form over many row ranges, one pipeline for all of them.  The
// ranges are cut into pieces of whole rows that start on 4-atom groups and
// gathered, across range boundaries, into batches of up to 2^20 atoms; batch
// k is copied host-to-device (one copy per piece) into one of kHostSlots
// device slots on the copy stream while the caller's stream quantises batch
// k-1 (row scales of each piece with its whole matrix's plan, one search over
// all the batch's pieces, 18-bit pack into each range's device output), so
// the transfer hides behind the search.  The bytes and scales of a batch's
// pieces go back to the host on a third stream as soon as the batch is
// packed; the call returns once they are all written.
static constexpr int kHostSlots = 3;
static constexpr int64_t kHostBatchAtoms = int64_t(1) << 20;  // atoms per batch (one search call)
static constexpr int64_t kHostFirstBatch = int64_t(1) << 17;   // the first batch; each next one doubles
static constexpr int kHostPieces = 64;                         // row ranges per batch

int h24_quantize_layer_rows_host(const h24_layer_rows *layers, int count, int dtype, void *stream) {
  H24_TABLES_OR_FAIL(T);
  if (count < 0 || (count > 0 && !layers)) return fail(H24_ERR_INVALID, "quantize_layer_host: bad list");
  if (dtype != H24_DTYPE_F32 && dtype != H24_DTYPE_BF16)
    return fail(H24_ERR_INVALID, "quantize_layer_host: weights must be fp32 or bf16");
  const size_t esize = dtype == H24_DTYPE_BF16 ? 2 : 4;
  std::vector<RowRange> R(count);
  for (int i = 0; i < count; ++i) {
    int rc = validate_rows(layers[i], esize, true, &R[i]);
    if (rc != H24_OK) return rc;
  }
  auto up = [](size_t v) { return (v + 255) & ~static_cast<size_t>(255); };
  // Batches of up to kHostBatchAtoms atoms, each made of pieces: row ranges
  // of one matrix that start on a whole 4-atom group (rows [c0, c1) of range
  // li, at byte offset `off` of the batch's slot), at most kHostPieces per
  // batch.  A batch is one search over all its pieces, so the device works on
  // batches as large as the device-resident path's whatever the matrix sizes.
  // The first batch holds kHostFirstBatch atoms and each next one twice as
  // many up to that size: the search starts after a short copy, and even a
  // single matrix's copy overlaps its search.
  struct Piece { int li; int64_t c0, c1; size_t off; };
  struct Batch { size_t first, count; int64_t atoms; size_t bytes; };
  std::vector<Piece> pieces;
  std::vector<Batch> batches;
  std::vector<size_t> out_pk(count), out_sig(count);
  size_t out_bytes = 0;
  {
    Batch cur{0, 0, 0, 0};
    int64_t cap = kHostFirstBatch;
    for (int i = 0; i < count; ++i) {
      const RowRange &r = R[i];
      out_pk[i] = out_bytes;
      out_bytes += up(static_cast<size_t>((r.atoms() + 3) / 4) * 9);
      out_sig[i] = out_bytes;
      out_bytes += up(static_cast<size_t>(r.r1 - r.r0) * 2);
      if (r.r1 == r.r0) continue;
      int64_t g = r.in, h = 96;
      while (h) { const int64_t t2 = g % h; g = h; h = t2; }
      const int64_t rg = 96 / g;  // rows per whole number of 4-atom groups
      for (int64_t c0 = r.r0; c0 < r.r1;) {
        int64_t fit = (cap - cur.atoms) * kDim / r.in / rg * rg;
        if (cur.count == 0 && fit < rg) fit = rg;  // a row group wider than a batch goes alone
        if (fit <= 0 || cur.count == static_cast<size_t>(kHostPieces)) {
          batches.push_back(cur);
          cur = Batch{pieces.size(), 0, 0, 0};
          cap = cap * 2 < kHostBatchAtoms ? cap * 2 : kHostBatchAtoms;
          continue;
        }
        const int64_t c1 = c0 + fit < r.r1 ? c0 + fit : r.r1;
        pieces.push_back({i, c0, c1, cur.bytes});
        cur.atoms += (c1 - c0) * r.in / kDim;
        cur.bytes += up(static_cast<size_t>((c1 - c0) * r.in) * esize);
        ++cur.count;
        c0 = c1;
      }
    }
    if (cur.count) batches.push_back(cur);
  }
  if (batches.empty()) return H24_OK;
  size_t slot_bytes = 0;
  int64_t batch_atoms = 0;
  for (const Batch &b : batches) {
    slot_bytes = std::max(slot_bytes, b.bytes);
    batch_atoms = std::max(batch_atoms, b.atoms);
  }
  cudaStream_t s = as_stream(stream);
  const size_t idx_bytes = up(static_cast<size_t>(batch_atoms) * 4);
  const size_t off_slots = up(out_bytes);
  const size_t off_idx = off_slots + kHostSlots * slot_bytes;
  uint8_t *buf = nullptr;
  H24_CUDA_TRY(cudaMallocFromPoolAsync(reinterpret_cast<void **>(&buf), off_idx + kHostSlots * idx_bytes,
                                       T->pool, s));
  std::vector<cudaEvent_t> evs;
  int rc = H24_OK;
  auto event = [&](cudaEvent_t *e) -> int {
    cudaError_t ce = cudaEventCreateWithFlags(e, cudaEventDisableTiming);
    if (ce != cudaSuccess) return cuda_fail(ce, "cudaEventCreate");
    evs.push_back(*e);
    return H24_OK;
  };
  cudaEvent_t ready = nullptr, copied[kHostSlots] = {}, freed[kHostSlots] = {};
  rc = event(&ready);
  // The outputs of batch k are copied out after its pack (event done[k]).
  std::vector<cudaEvent_t> done(batches.size(), nullptr);
  for (size_t k = 0; k < batches.size() && rc == H24_OK; ++k) rc = event(&done[k]);
  for (int k = 0; k < kHostSlots && rc == H24_OK; ++k) {
    rc = event(&copied[k]);
    if (rc == H24_OK) rc = event(&freed[k]);
  }
  // The copy stream starts after the buffer exists on the caller's stream.
  if (rc == H24_OK) {
    cudaError_t ce = cudaEventRecord(ready, s);
    if (ce == cudaSuccess) ce = cudaStreamWaitEvent(T->copy_stream, ready, 0);
    if (ce != cudaSuccess) rc = cuda_fail(ce, "copy stream order");
  }
  std::vector<const void *> xs;
  std::vector<int64_t> na;
  for (size_t k = 0; k < batches.size() && rc == H24_OK; ++k) {
    const Batch &b = batches[k];
    const int sl = static_cast<int>(k % kHostSlots);
    uint8_t *slot = buf + off_slots + sl * slot_bytes;
    int32_t *idx = reinterpret_cast<int32_t *>(buf + off_idx + sl * idx_bytes);
    // Copy into the slot once the batch that used it before is quantised.
    cudaError_t ce = cudaSuccess;
    if (k >= static_cast<size_t>(kHostSlots)) ce = cudaStreamWaitEvent(T->copy_stream, freed[sl], 0);
    for (size_t q = b.first; q < b.first + b.count && ce == cudaSuccess; ++q) {
      const Piece &pc = pieces[q];
      const RowRange &r = R[pc.li];
      ce = cudaMemcpyAsync(slot + pc.off, r.w + static_cast<size_t>(pc.c0 * r.in) * esize,
                           static_cast<size_t>((pc.c1 - pc.c0) * r.in) * esize, cudaMemcpyHostToDevice,
                           T->copy_stream);
    }
    if (ce == cudaSuccess) ce = cudaEventRecord(copied[sl], T->copy_stream);
    if (ce == cudaSuccess) ce = cudaStreamWaitEvent(s, copied[sl], 0);
    if (ce != cudaSuccess) { rc = cuda_fail(ce, "batch copy"); break; }
    xs.clear();
    na.clear();
    for (size_t q = b.first; q < b.first + b.count && rc == H24_OK; ++q) {
      const Piece &pc = pieces[q];
      const RowRange &r = R[pc.li];
      uint16_t *sig = reinterpret_cast<uint16_t *>(buf + out_sig[pc.li]) + (pc.c0 - r.r0);
      rc = launch_row_rms(slot + pc.off, dtype, pc.c1 - pc.c0, r.in, r.rows, pc.c0, nullptr, sig, s);
      xs.push_back(slot + pc.off);
      na.push_back((pc.c1 - pc.c0) * r.in / kDim);
    }
    if (rc == H24_OK)
      rc = quantize_segments(T, xs.data(), na.data(), static_cast<int>(xs.size()), dtype, H24_RULE_PACK, idx, s);
    int64_t a0 = 0;
    for (size_t q = b.first; q < b.first + b.count && rc == H24_OK; ++q) {
      const Piece &pc = pieces[q];
      const RowRange &r = R[pc.li];
      const int64_t n = (pc.c1 - pc.c0) * r.in / kDim;
      uint8_t *pk = buf + out_pk[pc.li] + static_cast<size_t>((pc.c0 - r.r0) * r.in / kDim / 4) * 9;
      rc = launch_pack_i32(idx + a0, n, pk, s);
      a0 += n;
    }
    if (rc == H24_OK) {
      ce = cudaEventRecord(freed[sl], s);
      if (ce == cudaSuccess) ce = cudaEventRecord(done[k], s);
      if (ce != cudaSuccess) rc = cuda_fail(ce, "slot release");
    }
    // The batch's pieces of every range's bytes and scales back to the host.
    // A piece starts on a whole 4-atom group, so its bytes are whole 9-byte
    // groups; the last piece of a range ends with the range's last group.
    if (rc == H24_OK) ce = cudaStreamWaitEvent(T->d2h_stream, done[k], 0);
    for (size_t q = b.first; q < b.first + b.count && rc == H24_OK && ce == cudaSuccess; ++q) {
      const Piece &pc = pieces[q];
      const RowRange &r = R[pc.li];
      const size_t p0 = static_cast<size_t>((pc.c0 - r.r0) * r.in / kDim / 4) * 9;
      const size_t p1 = pc.c1 == r.r1 ? static_cast<size_t>((r.atoms() + 3) / 4) * 9
                                      : static_cast<size_t>((pc.c1 - r.r0) * r.in / kDim / 4) * 9;
      ce = cudaMemcpyAsync(r.sigma16 + (pc.c0 - r.r0), buf + out_sig[pc.li] + (pc.c0 - r.r0) * 2,
                           static_cast<size_t>(pc.c1 - pc.c0) * 2, cudaMemcpyDeviceToHost, T->d2h_stream);
      if (ce == cudaSuccess)
        ce = cudaMemcpyAsync(r.packed + p0, buf + out_pk[pc.li] + p0, p1 - p0, cudaMemcpyDeviceToHost,
                             T->d2h_stream);
    }
    if (rc == H24_OK && ce != cudaSuccess) rc = cuda_fail(ce, "output copy");
  }
  // Every copy-stream and result-stream operation is ordered before the free
  // (also after an error part way through the batches).
  for (cudaStream_t cs : {T->copy_stream, T->d2h_stream}) {
    cudaEvent_t drained = nullptr;
    if (cudaEventCreateWithFlags(&drained, cudaEventDisableTiming) == cudaSuccess) {
      evs.push_back(drained);
      if (cudaEventRecord(drained, cs) == cudaSuccess) cudaStreamWaitEvent(s, drained, 0);
    }
  }
  const cudaError_t fe = cudaFreeAsync(buf, s);
  const cudaError_t se = cudaStreamSynchronize(s);
  for (cudaEvent_t e : evs) cudaEventDestroy(e);
  if (rc != H24_OK) return rc;
  if (fe != cudaSuccess) return cuda_fail(fe, "cudaFreeAsync");
  if (se != cudaSuccess) return cuda_fail(se, "cudaStreamSynchronize");
  // The call has synchronised: report (and clear) a timed-out wait of the
  // screening kernel instead of returning incomplete indices.
  return take_device_error(T, s);
}

int h24_quantize_layer_host(const float *w, int64_t rows, int64_t in_features, uint16_t *sigma16_out,
                            uint8_t *packed_out, void *stream) {
  h24_layer_rows L{w, rows, in_features, 0, rows, sigma16_out, packed_out};
  return h24_quantize_layer_rows_host(&L, 1, H24_DTYPE_F32, stream);
}

int h24_gather_codewords(const int32_t *idx, int64_t n, int dtype, void *out, void *stream) {
  H24_TABLES_OR_FAIL(T);
  if (n < 0) return fail(H24_ERR_INVALID, "gather: negative length");
  if (n > 0 && (!idx || !out)) return fail(H24_ERR_INVALID, "gather: null pointer");
  return launch_gather(T, idx, n, dtype, out, as_stream(stream));
}

int h24_timing_enable(int enable) {
  std::lock_guard<std::mutex> lk(g_timing_mu);
  g_timing = enable != 0;
  return H24_OK;
}

int h24_timing_read_kernel(int kernel, double *ms, int64_t *launches) {
  if (kernel < 0 || kernel >= H24_KERNEL_COUNT) return fail(H24_ERR_INVALID, "timing: unknown kernel");
  std::vector<std::pair<cudaEvent_t, cudaEvent_t>> ev;
  {
    std::lock_guard<std::mutex> lk(g_timing_mu);
    ev.swap(g_events[kernel]);
  }
  double total = 0.0;
  int rc = H24_OK;
  for (auto &p : ev) {
    cudaError_t e = cudaEventSynchronize(p.second);
    float t = 0.f;
    if (e == cudaSuccess) e = cudaEventElapsedTime(&t, p.first, p.second);
    if (e != cudaSuccess && rc == H24_OK) rc = cuda_fail(e, "timing");
    total += t;
    cudaEventDestroy(p.first);
    cudaEventDestroy(p.second);
  }
  if (ms) *ms = total;
  if (launches) *launches = static_cast<int64_t>(ev.size());
  return rc;
}

int h24_timing_read(double *ms, int64_t *launches) {
  return h24_timing_read_kernel(H24_KERNEL_SCREEN, ms, launches);
}

int h24_quantize_stats(int64_t *exhaustive_atoms, int64_t *exact_scores, int64_t *flagged_units,
                       void *stream) {
  H24_TABLES_OR_FAIL(T);
  int64_t h[3] = {0, 0, 0};
  cudaStream_t s = as_stream(stream);
  H24_CUDA_TRY(cudaMemcpyAsync(h, T->stats, sizeof(h), cudaMemcpyDeviceToHost, s));
  H24_CUDA_TRY(cudaStreamSynchronize(s));
  H24_CUDA_TRY(cudaMemsetAsync(T->stats, 0, sizeof(h), s));
  if (exhaustive_atoms) *exhaustive_atoms = h[0];
  if (exact_scores) *exact_scores = h[1];
  if (flagged_units) *flagged_units = h[2];
  return H24_OK;
}

int64_t h24_launch_count(void) { return g_launches.load(std::memory_order_relaxed); }

int h24_check(void *stream) {
  H24_TABLES_OR_FAIL(T);
  return take_device_error(T, as_stream(stream));
}

}  // extern "C"
