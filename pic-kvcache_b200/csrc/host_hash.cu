// Host-side fingerprints for the scheduler's token-range lookup (no GPU work).
//
// The fingerprint of a window is the 64-bit polynomial hash of
// cacheblend_vllm/hashing.py:18-22: h = sum_i (t_i + 1) B^(W-1-i) mod 2^64,
// B = 1,000,003.  The reference evaluates it at every offset with an
// N x W sliding matmul (hashing.py:42-53); here one rolling pass in wrapping
// uint64 arithmetic gives the same values in O(N):
//   h_{i+1} = h_i B - (t_i + 1) B^W + (t_{i+W} + 1)   (mod 2^64).
#include <stdint.h>

#include <algorithm>

#include "cb_common.cuh"

namespace {
constexpr uint64_t kBase = 1000003ull;
}

extern "C" int cb_window_hashes(const int64_t* tokens, int64_t n, int64_t window, uint64_t* out) {
  cb::clear_error();
  CB_REQUIRE(window > 0, "window must be positive");
  CB_REQUIRE(n >= 0, "negative token count");
  if (n < window) return CB_OK;
  CB_REQUIRE(tokens != nullptr && out != nullptr, "null pointer argument");
  uint64_t pw = 1;  // B^W
  uint64_t h = 0;
  for (int64_t i = 0; i < window; ++i) {
    h = h * kBase + static_cast<uint64_t>(tokens[i]) + 1u;
    pw *= kBase;
  }
  out[0] = h;
  for (int64_t i = 0; i + window < n; ++i) {
    h = h * kBase - (static_cast<uint64_t>(tokens[i]) + 1u) * pw +
        static_cast<uint64_t>(tokens[i + window]) + 1u;
    out[i + 1] = h;
  }
  return CB_OK;
}

// Offsets whose window hash is one of `known` (ascending, distinct), in
// ascending order; writes at most `max_out` and returns the count in *count.
extern "C" int cb_hash_candidates(const uint64_t* hashes, int64_t n, const uint64_t* known,
                                  int64_t num_known, int64_t* out, int64_t max_out,
                                  int64_t* count) {
  cb::clear_error();
  CB_REQUIRE(n >= 0 && num_known >= 0 && max_out >= 0, "negative size");
  CB_REQUIRE(count != nullptr, "null output");
  *count = 0;
  if (n == 0 || num_known == 0) return CB_OK;
  CB_REQUIRE(hashes != nullptr && known != nullptr && (out != nullptr || max_out == 0),
             "null pointer argument");
  // a 2^16-bit filter on the low hash bits rejects almost every offset without a
  // search (fingerprints are uniform in their low bits)
  static thread_local uint64_t filter[1024];
  std::fill(filter, filter + 1024, 0ull);
  for (int64_t k = 0; k < num_known; ++k) filter[(known[k] >> 6) & 1023u] |= 1ull << (known[k] & 63u);
  int64_t found = 0;
  for (int64_t i = 0; i < n; ++i) {
    const uint64_t h = hashes[i];
    if (!((filter[(h >> 6) & 1023u] >> (h & 63u)) & 1u)) continue;
    if (std::binary_search(known, known + num_known, h)) {
      if (found < max_out) out[found] = i;
      ++found;
    }
  }
  *count = found;
  return CB_OK;
}
