// h24_codebook.cpp -- host construction of the H24 codebook's raw coordinates.
//
// The table must equal the reference's byte for byte, so the steps follow
// castor.py:74-190: the (24,12) Golay words from the generator polynomial,
// the three kinds of kissing points, and a lexicographic sort with column 0 as
// the primary key (np.lexsort over columns 23..0).  Raw coordinates are kept
// as small integers; the fp32 values are raw * fp32(1/sqrt(8)).
#include <algorithm>
#include <array>
#include <cstdint>
#include <cstring>
#include <string>
#include <vector>

#include "h24_internal.cuh"

namespace h24 {
namespace {

using Row = std::array<int8_t, kDim>;

// Golay(23,12) systematic encoding: message bits above an 11-bit remainder of
// msg * x^11 modulo the generator, extended by an overall parity bit 23
// (castor.py:74-95).
uint32_t golay24(uint32_t msg) {
  const uint32_t poly = (1u << 11) | (1u << 9) | (1u << 7) | (1u << 6) | (1u << 5) | (1u << 1) | 1u;
  uint32_t rem = msg << 11;
  for (int bit = 22; bit >= 11; --bit)
    if (rem & (1u << bit)) rem ^= poly << (bit - 11);
  uint32_t w23 = (msg << 11) | rem;
  uint32_t parity = static_cast<uint32_t>(__builtin_popcount(w23) & 1);
  return (parity << 23) | w23;
}

}  // namespace

bool build_raw_kissing_points(int8_t *out, std::string *err) {
  std::vector<uint32_t> words(4096);
  for (uint32_t m = 0; m < 4096; ++m) words[m] = golay24(m);

  std::vector<Row> rows;
  rows.reserve(kKissing);
  // Two coordinates at +-4 (castor.py:108-114).
  for (int i = 0; i < kDim; ++i)
    for (int j = i + 1; j < kDim; ++j)
      for (int a : {-4, 4})
        for (int b : {-4, 4}) {
          Row r{};
          r[i] = static_cast<int8_t>(a);
          r[j] = static_cast<int8_t>(b);
          rows.push_back(r);
        }
  // +-2 on each octad (weight-8 word), even number of minus signs (castor.py:118-130).
  for (uint32_t w : words) {
    if (__builtin_popcount(w) != 8) continue;
    int pos[8], np = 0;
    for (int b = 0; b < kDim; ++b)
      if (w & (1u << b)) pos[np++] = b;
    for (int signs = 0; signs < 256; ++signs) {
      if ((8 - __builtin_popcount(static_cast<unsigned>(signs))) & 1) continue;
      Row r{};
      for (int k = 0; k < 8; ++k) r[pos[k]] = static_cast<int8_t>((signs >> k) & 1 ? 2 : -2);
      rows.push_back(r);
    }
  }
  // -1 on a word's support, +1 elsewhere, and -3 at one position (castor.py:134-141).
  for (int p = 0; p < kDim; ++p)
    for (uint32_t w : words) {
      Row r;
      for (int b = 0; b < kDim; ++b) r[b] = (w >> b) & 1u ? -1 : 1;
      r[p] = -3;
      rows.push_back(r);
    }

  if (static_cast<int>(rows.size()) != kKissing) {
    if (err) *err = "kissing point count " + std::to_string(rows.size()) + " != 196560";
    return false;
  }
  for (const Row &r : rows) {
    int n2 = 0;
    for (int8_t v : r) n2 += v * v;
    if (n2 != 32) {
      if (err) *err = "kissing point with squared raw norm != 32";
      return false;
    }
  }
  std::sort(rows.begin(), rows.end());  // lexicographic, column 0 primary
  for (size_t k = 1; k < rows.size(); ++k)
    if (rows[k] == rows[k - 1]) {
      if (err) *err = "duplicate kissing point";
      return false;
    }
  for (size_t k = 0; k < rows.size(); ++k) std::memcpy(out + k * kDim, rows[k].data(), kDim);
  return true;
}

}  // namespace h24
