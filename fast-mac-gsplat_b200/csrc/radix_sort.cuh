// Stable LSD radix sort of (uint64 key, uint32 value) pairs, onesweep style:
// one kernel builds the histograms of every digit pass at once, then each
// 8-bit digit pass ranks a partition of 1024-4096 keys (fewer keys per
// partition for short inputs) in shared memory, resolves its global per-digit
// offsets with decoupled look-back, and scatters.
#pragma once

#include <stddef.h>
#include <stdint.h>

#include <cuda_runtime.h>

#include "gsb_host.cuh"

namespace gsb {

constexpr int kSortThreads = 256;
constexpr int kSortWarps = kSortThreads / 32;
constexpr int kRadix = 256;
constexpr int kRadixBits = 8;
constexpr int64_t kSortMaxN = (int64_t(1) << 30) - 1;  // 30-bit look-back payload
constexpr int kSortMaxPasses = 8;                     // 64-bit keys

inline int sort_passes(int begin_bit, int end_bit) {
  return end_bit > begin_bit ? (end_bit - begin_bit + kRadixBits - 1) / kRadixBits : 0;
}

// Carves the sort's scratch: temp key/value buffers, histograms, partition
// counters and per-pass look-back tiles. Returns the status of the launches
// when running (base != nullptr); measuring mode launches nothing.
// scratch_zeroed: the caller has already cleared the sort's zero-initialised
// scratch (radix_sort_zero_region) in an earlier kernel, saving a memset launch.
// digit_hist: when given, the kernel that wrote the keys has already counted
// their digits there (pass p's 256 counts at digit_hist + 256 p, digits of
// bits begin_bit + 8p ...), so the histogram launch is skipped.
cudaError_t radix_sort_pairs(Carver& ws, const uint64_t* keys_in, const uint32_t* vals_in,
                             uint64_t* keys_out, uint32_t* vals_out, int64_t n, int begin_bit,
                             int end_bit, uint32_t* status, cudaStream_t stream, bool scratch_zeroed,
                             const uint32_t* digit_hist = nullptr);
// Key ranges instead of sorted keys (32-bit keys, at least one pass): the
// last pass does not write keys_out; for each key value k < n it leaves in
// first[k] (zeroed beforehand, by the caller) the count of output positions
// from k's first position to the end (n_pairs - position), 0 when k does not
// occur, and the same in block[k / kRangesBlock] for the first key of each
// block of kRangesBlock key values.
constexpr int kRangesBlock = 256;
struct SortRanges {
  int32_t* first = nullptr;
  int32_t* block = nullptr;
  int64_t n = 0;
};

// 32-bit keys (end_bit <= 32): 8 bytes per pair moved per pass instead of 12.
cudaError_t radix_sort_pairs(Carver& ws, const uint32_t* keys_in, const uint32_t* vals_in,
                             uint32_t* keys_out, uint32_t* vals_out, int64_t n, int begin_bit,
                             int end_bit, uint32_t* status, cudaStream_t stream, bool scratch_zeroed,
                             const uint32_t* digit_hist = nullptr, SortRanges ranges = SortRanges{});

// The words a radix_sort_pairs call carved from `ws` (at its current offset)
// needs cleared before it runs (histograms, partition counters, look-back).
struct ZeroRegion {
  uint32_t* ptr = nullptr;
  size_t words = 0;
};
ZeroRegion radix_sort_zero_region(Carver ws, int64_t n, int begin_bit, int end_bit, bool keys32);

}  // namespace gsb
