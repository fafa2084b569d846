// Onesweep LSD radix sort for (uint64 key, uint32 value) pairs on sm_100a.
//
// Replaces the per-tile threadgroup bitonic sort of the reference
// (variants/v8_project3d/csrc/metal/gsplat_v8_project3d_kernels.metal:594-617, capped at
// GSP_FAST_CAP entries per tile) with one global, stable, uncapped sort.
#include <mutex>

#include "gsb_common.cuh"
#include "gsb_host.cuh"
#include "radix_sort.cuh"

namespace gsb {
namespace {

constexpr uint32_t kFlagAgg = 0x40000000u;  // partition aggregate published
constexpr uint32_t kFlagInc = 0x80000000u;  // inclusive prefix published
constexpr uint32_t kValueMask = 0x3fffffffu;
constexpr int kMaxPasses = kSortMaxPasses;
constexpr int kLookWin = 8;  // predecessors read per look-back step

// Histograms of every digit pass in one read of the keys. A thread takes
// kHistItems consecutive keys per round and counts runs of equal digits before
// touching the shared histogram, so clustered keys (a tile sort's high digit is
// constant over long stretches) cost one shared atomic per run instead of one
// per key on a few hot counters.
constexpr int kHistItems = 16;
template <typename K>
__global__ void __launch_bounds__(kSortThreads)
    rs_histogram(const K* __restrict__ keys, int64_t n, int begin_bit, int passes,
                 int last_bits, uint32_t* __restrict__ hist) {
  pdl_wait();
  pdl_trigger();
  __shared__ uint32_t s_hist[kMaxPasses][kRadix];
  for (int i = threadIdx.x; i < passes * kRadix; i += kSortThreads) s_hist[i / kRadix][i % kRadix] = 0;
  __syncthreads();
  const int64_t stride = (int64_t)gridDim.x * kSortThreads * kHistItems;
  // 16-byte loads need a 16-byte aligned key array (a caller's pointer to the
  // exported sort may not be); otherwise the keys are read one by one.
  const bool vec = (reinterpret_cast<uintptr_t>(keys) & 15u) == 0u;
  for (int64_t i0 = ((int64_t)blockIdx.x * kSortThreads + threadIdx.x) * kHistItems; i0 < n; i0 += stride) {
    K k[kHistItems];
    const int cnt = (int)min((int64_t)kHistItems, n - i0);
    if (cnt == kHistItems && vec) {
      constexpr int kPer = 16 / sizeof(K);
#pragma unroll
      for (int v = 0; v < kHistItems / kPer; ++v) {
        const uint4 q = reinterpret_cast<const uint4*>(keys + i0)[v];
        const K* qk = reinterpret_cast<const K*>(&q);
#pragma unroll
        for (int u = 0; u < kPer; ++u) k[v * kPer + u] = qk[u];
      }
    } else {
#pragma unroll
      for (int u = 0; u < kHistItems; ++u) k[u] = u < cnt ? keys[i0 + u] : K(0);
    }
    for (int p = 0; p < passes; ++p) {
      const int bits = (p == passes - 1) ? last_bits : kRadixBits;
      const int sh = begin_bit + p * kRadixBits;
      const uint32_t dm = (1u << bits) - 1u;
      uint32_t run_d = (uint32_t)(k[0] >> sh) & dm, run_n = 1;
#pragma unroll
      for (int u = 1; u < kHistItems; ++u) {
        if (u < cnt) {
          const uint32_t d = (uint32_t)(k[u] >> sh) & dm;
          if (d == run_d) {
            ++run_n;
          } else {
            atomicAdd(&s_hist[p][run_d], run_n);
            run_d = d;
            run_n = 1;
          }
        }
      }
      atomicAdd(&s_hist[p][run_d], run_n);
    }
  }
  __syncthreads();
  for (int i = threadIdx.x; i < passes * kRadix; i += kSortThreads) {
    const uint32_t v = s_hist[i / kRadix][i % kRadix];
    if (v) atomicAdd(&hist[i], v);
  }
}

// Shared memory of one pass: the partition's keys and values staged in digit
// order (so the global scatter is coalesced), and the digit bookkeeping.
template <typename K, int ITEMS>
struct OnesweepSmem {
  K keys[kSortThreads * ITEMS];
  uint32_t vals[kSortThreads * ITEMS];
  uint32_t vstage[kSortThreads * ITEMS];  // the partition's values in input order (cp.async)
  uint32_t warp_hist[kSortWarps][kRadix];  // per-warp digit counts, then exclusive over warps
  uint32_t local_base[kRadix];             // exclusive scan of the partition's digit counts
  uint32_t global_base[kRadix];            // digit base + look-back exclusive prefix
  uint32_t scan[kSortWarps];
  uint32_t part;
  long long fence_sink;
};

// Ranks one warp's ITEMS x 32 keys by digit, stably in (item, lane) order,
// counting into the warp's digit histogram. The lanes holding the same digit
// come from one ballot per digit bit (cheaper than match.any): NB ballots on
// bits 0 .. NB-1 (a digit has no set bit above its pass's width), and with
// kSentinel one more on bit kRadixBits, set only in the invalid lanes' digit
// kRadix (past the end of the keys).
template <int NB, bool kSentinel, typename K, int ITEMS>
__device__ __forceinline__ void rank_items(const K (&k)[ITEMS], uint32_t (&rank)[ITEMS], int64_t seg, int64_t n,
                                           int shift, uint32_t dmask, int lane, uint32_t lt_mask,
                                           uint32_t* __restrict__ warp_hist) {
#pragma unroll
  for (int i = 0; i < ITEMS; ++i) {
    const int64_t idx = seg + i * 32 + lane;
    const bool valid = !kSentinel || idx < n;
    const uint32_t d = valid ? ((uint32_t)(k[i] >> shift) & dmask) : kRadix;
    uint32_t peers = 0xffffffffu;
#pragma unroll
    for (int b = 0; b < NB + (kSentinel ? 1 : 0); ++b) {
      const int bit = b < NB ? b : kRadixBits;
      const bool on = (d >> bit) & 1u;
      const uint32_t bal = __ballot_sync(kFullMask, on);
      peers &= on ? bal : ~bal;
    }
    uint32_t cnt_before = 0;
    if (valid) cnt_before = warp_hist[d];
    __syncwarp();
    rank[i] = cnt_before + __popc(peers & lt_mask);
    const int leader = 31 - __clz(peers);
    if (valid && lane == leader) warp_hist[d] = cnt_before + __popc(peers);
    __syncwarp();
  }
}

// One digit pass. Keys are held warp-striped: warp w owns the contiguous
// segment [tile + w*32*ITEMS, +32*ITEMS) and lane l holds its items i*32+l, so
// (item, lane) order is input order and the lane-order ranking is stable. Each
// CTA also turns the pass's global digit histogram into exclusive digit bases
// itself (a 256-entry scan), so no separate launch precedes the pass. The
// ranked keys are first placed in digit order in shared memory (while the
// look-back resolves), then written out by consecutive threads, so each
// digit's run leaves the CTA as contiguous stores.
// kRanges (the last pass of a sort whose caller asked for key ranges): the
// sorted keys are not written; instead the first output position of each key
// value a partition holds is recorded as atomicMax(first[key], n - pos), so
// first[] (zeroed beforehand) ends up holding n - (the key's first position),
// 0 for a key value that does not occur; block[] gets the same per block of
// kRangesBlock key values.
// kPrefix (the first pass of a long sort, see rs_part_counts): partition
// blockIdx.x reads its per-digit exclusive prefix over the partitions before it
// from prefix[] instead of resolving it by look-back.
template <typename K, int ITEMS, bool kRanges = false, bool kPrefix = false>
__global__ void __launch_bounds__(kSortThreads, (ITEMS >= 16 ? 3 : 0))
    rs_onesweep(const K* __restrict__ keys_in, const uint32_t* __restrict__ vals_in,
                K* __restrict__ keys_out, uint32_t* __restrict__ vals_out, int64_t n,
                int shift, int bits, const uint32_t* __restrict__ hist,
                uint32_t* __restrict__ lookback, uint32_t* __restrict__ part_counter,
                uint32_t* __restrict__ status, int32_t* __restrict__ first, int32_t* __restrict__ block,
                int64_t first_n, const uint32_t* __restrict__ prefix) {
  pdl_wait();
  pdl_trigger();
  constexpr int kTile = kSortThreads * ITEMS;
  extern __shared__ __align__(16) unsigned char s_raw[];
  OnesweepSmem<K, ITEMS>& sm = *reinterpret_cast<OnesweepSmem<K, ITEMS>*>(s_raw);

  const int tid = threadIdx.x;
  const int lane = tid & 31, warp = tid >> 5;
  if (tid == 0) sm.part = kPrefix ? blockIdx.x : atomicAdd(part_counter, 1u);
  for (int i = tid; i < kSortWarps * kRadix; i += kSortThreads) (&sm.warp_hist[0][0])[i] = 0u;
  __syncthreads();
  const uint32_t part = sm.part;
  const uint32_t dmask = (1u << bits) - 1u;
  const int64_t tile0 = (int64_t)part * kTile;
  const int64_t seg = tile0 + (int64_t)warp * (32 * ITEMS);
  K k[ITEMS];
  uint32_t rank[ITEMS];
  const uint32_t lt_mask = (1u << lane) - 1u;
  {
    const int valid = (int)min((int64_t)kTile, n - tile0);
    for (int e = tid; e < valid; e += kSortThreads) cp_async4(&sm.vstage[e], vals_in + tile0 + e);
    cp_async_commit();
  }
#pragma unroll
  for (int i = 0; i < ITEMS; ++i) {
    const int64_t idx = seg + i * 32 + lane;
    k[i] = idx < n ? keys_in[idx] : K(0);
  }
  // Exclusive digit bases of this pass (the histogram load overlaps the key loads).
  uint32_t digit_base;
  {
    const uint32_t h = hist[tid];
    uint32_t x = h;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const uint32_t y = __shfl_up_sync(kFullMask, x, o);
      if (lane >= o) x += y;
    }
    if (lane == 31) sm.scan[warp] = x;
    __syncthreads();
    uint32_t wsum = 0;
#pragma unroll
    for (int w = 0; w < kSortWarps; ++w) wsum += (w < warp) ? sm.scan[w] : 0u;
    digit_base = wsum + x - h;
  }
  // Scheduling fence: a read of %clock64 here (consumed by a shared store so it
  // stays) keeps ptxas from moving the key loads and the digit-base work into
  // the ranking loop. Measured on B200: a 60M-pair two-pass sort 1.99 -> 1.34 ms.
  {
    long long c;
    asm volatile("mov.u64 %0, %%clock64;" : "=l"(c));
    if (tid == 0) sm.fence_sink = c;
  }

  // A full partition ballots exactly the pass's digit bits (a last pass of
  // fewer bits takes fewer ballots); the last, partial one also sets its
  // invalid lanes apart by the sentinel bit.
  if (tile0 + kTile <= n) {
    switch (bits) {
      case 7: rank_items<7, false>(k, rank, seg, n, shift, dmask, lane, lt_mask, sm.warp_hist[warp]); break;
      case 6: rank_items<6, false>(k, rank, seg, n, shift, dmask, lane, lt_mask, sm.warp_hist[warp]); break;
      case 5: rank_items<5, false>(k, rank, seg, n, shift, dmask, lane, lt_mask, sm.warp_hist[warp]); break;
      case 4: rank_items<4, false>(k, rank, seg, n, shift, dmask, lane, lt_mask, sm.warp_hist[warp]); break;
      default: rank_items<kRadixBits, false>(k, rank, seg, n, shift, dmask, lane, lt_mask, sm.warp_hist[warp]); break;
    }
  } else {
    rank_items<kRadixBits, true>(k, rank, seg, n, shift, dmask, lane, lt_mask, sm.warp_hist[warp]);
  }
  __syncthreads();

  // Digit t: exclusive scan over warps, partition total, its local base (a
  // block scan over digits), then publish the aggregate for the look-back.
  const int t = tid;
  uint32_t sum = 0;
#pragma unroll
  for (int w = 0; w < kSortWarps; ++w) {
    const uint32_t c = sm.warp_hist[w][t];
    sm.warp_hist[w][t] = sum;
    sum += c;
  }
  uint32_t* my = lookback + (size_t)part * kRadix + t;
  if (!kPrefix) st_volatile_u32(my, (part == 0 ? kFlagInc : kFlagAgg) | sum);
  {
    uint32_t x = sum;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const uint32_t y = __shfl_up_sync(kFullMask, x, o);
      if (lane >= o) x += y;
    }
    __syncthreads();  // sm.scan is reused
    if (lane == 31) sm.scan[warp] = x;
    __syncthreads();
    uint32_t wsum = 0;
#pragma unroll
    for (int w = 0; w < kSortWarps; ++w) wsum += (w < warp) ? sm.scan[w] : 0u;
    sm.local_base[t] = wsum + x - sum;
  }
  cp_async_wait<0>();
  __syncthreads();
  // Stage the partition in digit order.
#pragma unroll
  for (int i = 0; i < ITEMS; ++i) {
    const int64_t idx = seg + i * 32 + lane;
    if (idx < n) {
      const uint32_t d = (uint32_t)(k[i] >> shift) & dmask;
      const uint32_t lp = sm.local_base[d] + sm.warp_hist[warp][d] + rank[i];
      sm.keys[lp] = k[i];
      sm.vals[lp] = sm.vstage[warp * 32 * ITEMS + i * 32 + lane];
    }
  }
  // Decoupled look-back for digit t.
  uint32_t exclusive = 0;
  if (kPrefix) {
    exclusive = prefix[(size_t)part * kRadix + t];
  } else if (part != 0) {
    // Windowed look-back: read kLookWin predecessors at once, consume them
    // nearest-first until an inclusive prefix is found (one L2 round trip per
    // window instead of one per predecessor).
    int64_t j = (int64_t)part - 1;
    int spins = 0;
    bool failed = false, done = false;
    while (!done && !failed) {
      uint32_t w[kLookWin];
#pragma unroll
      for (int q = 0; q < kLookWin; ++q)
        w[q] = (j - q >= 0) ? ld_volatile_u32(lookback + (size_t)(j - q) * kRadix + t) : kFlagInc;
#pragma unroll
      for (int q = 0; q < kLookWin; ++q) {
        if (done || failed) break;
        uint32_t x = w[q];
        while (!(x & (kFlagAgg | kFlagInc))) {
          if (++spins > kSpinLimit || ((spins & 1023) == 0 && ld_volatile_u32(&status[GSB_STATUS_ERROR]))) {
            failed = true;
            break;
          }
          __nanosleep(32);
          x = ld_volatile_u32(lookback + (size_t)(j - q) * kRadix + t);
        }
        if (failed) break;
        exclusive += x & kValueMask;
        if (x & kFlagInc) done = true;
      }
      j -= kLookWin;
    }
    if (failed) raise_error(status, GSB_DEVERR_LOOKBACK_TIMEOUT, kSiteSortLookback);
    st_volatile_u32(my, kFlagInc | ((exclusive + sum) & kValueMask));
  }
  sm.global_base[t] = digit_base + exclusive;
  __syncthreads();

  // Coalesced scatter: staged entry e goes to global_base[d] + (e - local_base[d]).
  const int valid_n = (int)min((int64_t)kTile, n - tile0);
#pragma unroll
  for (int i = 0; i < ITEMS; ++i) {
    const int e = i * kSortThreads + tid;
    if (e < valid_n) {
      const K key = sm.keys[e];
      const uint32_t d = (uint32_t)(key >> shift) & dmask;
      const uint32_t pos = sm.global_base[d] + ((uint32_t)e - sm.local_base[d]);
      if (kRanges) {
        // Staged keys of one digit keep the previous passes' order, so equal
        // keys are adjacent and the first of a run starts the key here.
        const K prev = e == 0 ? key : sm.keys[e - 1];
        if ((e == 0 || prev != key) && (int64_t)key < first_n) {
          const int32_t v = (int32_t)(n - (int64_t)pos);
          atomicMax(&first[(size_t)key], v);
          if (e == 0 || prev / kRangesBlock != key / kRangesBlock) atomicMax(&block[(size_t)key / kRangesBlock], v);
        }
      } else {
        keys_out[pos] = key;
      }
      vals_out[pos] = sm.vals[e];
    }
  }
}

// Reduce-then-scan for the first pass of a long sort (n >= kPrefixMinN, two
// or more passes), in place of that pass's decoupled look-back, whose walk
// back to an inclusive prefix (about 40 partitions) bound the pass. One CTA
// per onesweep partition counts its keys' digits for every pass
// (rs_part_counts, which also replaces the histogram launch); 256-partition
// groups are summed (rs_group_sums); one CTA scans the group sums of the first
// pass over the groups and writes every pass's digit totals (rs_group_scan);
// then each group's partitions get their exclusive prefixes, in place of
// their first-pass counts (rs_part_prefix). Later passes keep the look-back:
// their partitions hold the previous pass's output, which exists only after it.
constexpr int64_t kPrefixMinN = int64_t(1) << 22;
constexpr int kPrefixGroup = 256;   // partitions per group
constexpr int kPrefixThreads = 1024;  // 4 threads per digit in the scan kernels
constexpr int kPrefixSlices = kPrefixThreads / kRadix;

// counts[(p * parts + part) * kRadix + d]: keys of partition `part` (the
// onesweep partition of ITEMS x 256 keys) with digit d in pass p.
template <typename K, int ITEMS>
__global__ void __launch_bounds__(kSortThreads)
    rs_part_counts(const K* __restrict__ keys, int64_t n, int begin_bit, int passes, int last_bits,
                   uint32_t* __restrict__ counts, int64_t parts) {
  pdl_wait();
  pdl_trigger();
  __shared__ uint32_t s_cnt[kMaxPasses][kRadix];
  for (int i = threadIdx.x; i < passes * kRadix; i += kSortThreads) s_cnt[i / kRadix][i % kRadix] = 0;
  __syncthreads();
  const int64_t part = blockIdx.x;
  const int64_t i0 = part * (int64_t)(kSortThreads * ITEMS) + (int64_t)threadIdx.x * ITEMS;
  const int cnt = (int)max((int64_t)0, min((int64_t)ITEMS, n - i0));
  if (cnt > 0) {
    K k[ITEMS];
    // ITEMS * sizeof(K) is a multiple of 16, so a 16-byte aligned array gives aligned chunks.
    const bool vec = (reinterpret_cast<uintptr_t>(keys) & 15u) == 0u;
    if (cnt == ITEMS && vec) {
      constexpr int kPer = 16 / sizeof(K);
#pragma unroll
      for (int v = 0; v < ITEMS / kPer; ++v) {
        const uint4 q = reinterpret_cast<const uint4*>(keys + i0)[v];
        const K* qk = reinterpret_cast<const K*>(&q);
#pragma unroll
        for (int u = 0; u < kPer; ++u) k[v * kPer + u] = qk[u];
      }
    } else {
#pragma unroll
      for (int u = 0; u < ITEMS; ++u) k[u] = u < cnt ? keys[i0 + u] : K(0);
    }
    for (int p = 0; p < passes; ++p) {
      const int bits = (p == passes - 1) ? last_bits : kRadixBits;
      const int sh = begin_bit + p * kRadixBits;
      const uint32_t dm = (1u << bits) - 1u;
      uint32_t run_d = (uint32_t)(k[0] >> sh) & dm, run_n = 1;
#pragma unroll
      for (int u = 1; u < ITEMS; ++u) {
        if (u < cnt) {
          const uint32_t d = (uint32_t)(k[u] >> sh) & dm;
          if (d == run_d) {
            ++run_n;
          } else {
            atomicAdd(&s_cnt[p][run_d], run_n);
            run_d = d;
            run_n = 1;
          }
        }
      }
      atomicAdd(&s_cnt[p][run_d], run_n);
    }
  }
  __syncthreads();
  for (int i = threadIdx.x; i < passes * kRadix; i += kSortThreads) {
    const int p = i / kRadix, d = i % kRadix;
    counts[((size_t)p * parts + part) * kRadix + d] = s_cnt[p][d];
  }
}

// gsum[(p * groups + g) * kRadix + d]: the counts of group g's partitions.
__global__ void __launch_bounds__(kPrefixThreads)
    rs_group_sums(const uint32_t* __restrict__ counts, int64_t parts, uint32_t* __restrict__ gsum, int groups) {
  pdl_wait();
  pdl_trigger();
  __shared__ uint32_t s_part[kPrefixSlices][kRadix];
  const int g = blockIdx.x, p = blockIdx.y;
  const int d = threadIdx.x % kRadix, q = threadIdx.x / kRadix;
  const int64_t r0 = (int64_t)g * kPrefixGroup, r1 = min(parts, r0 + kPrefixGroup);
  uint32_t s = 0;
#pragma unroll 8
  for (int64_t r = r0 + q; r < r1; r += kPrefixSlices) s += counts[((size_t)p * parts + r) * kRadix + d];
  s_part[q][d] = s;
  __syncthreads();
  if (q == 0) {
    uint32_t t = 0;
#pragma unroll
    for (int i = 0; i < kPrefixSlices; ++i) t += s_part[i][d];
    gsum[((size_t)p * groups + g) * kRadix + d] = t;
  }
}

// One CTA: the first pass's group sums become exclusive prefixes over the
// groups (in place), and hist[p * kRadix + d] receives every pass's totals.
__global__ void __launch_bounds__(kPrefixThreads)
    rs_group_scan(uint32_t* __restrict__ gsum, int groups, int passes, uint32_t* __restrict__ hist) {
  pdl_wait();
  pdl_trigger();
  __shared__ uint32_t s_part[kPrefixSlices][kRadix];
  const int d = threadIdx.x % kRadix, q = threadIdx.x / kRadix;
  const int per = (groups + kPrefixSlices - 1) / kPrefixSlices;
  const int g0 = min(groups, q * per), g1 = min(groups, g0 + per);
  for (int p = 0; p < passes; ++p) {
    uint32_t* row = gsum + (size_t)p * groups * kRadix;
    uint32_t s = 0;
#pragma unroll 8
    for (int g = g0; g < g1; ++g) s += row[(size_t)g * kRadix + d];
    s_part[q][d] = s;
    __syncthreads();
    uint32_t before = 0, total = 0;
#pragma unroll
    for (int i = 0; i < kPrefixSlices; ++i) {
      before += i < q ? s_part[i][d] : 0u;
      total += s_part[i][d];
    }
    if (p == 0) {
      for (int g = g0; g < g1; ++g) {
        const uint32_t v = row[(size_t)g * kRadix + d];
        row[(size_t)g * kRadix + d] = before;
        before += v;
      }
    }
    if (q == 0) hist[p * kRadix + d] = total;
    __syncthreads();  // s_part is reused
  }
}

// One CTA per group: the first pass's partition counts of group g become the
// partitions' exclusive prefixes (group prefix + the group's partitions before).
__global__ void __launch_bounds__(kPrefixThreads)
    rs_part_prefix(uint32_t* __restrict__ counts, int64_t parts, const uint32_t* __restrict__ gprefix) {
  pdl_wait();
  pdl_trigger();
  __shared__ uint32_t s_part[kPrefixSlices][kRadix];
  const int g = blockIdx.x;
  const int d = threadIdx.x % kRadix, q = threadIdx.x / kRadix;
  const int64_t r0 = (int64_t)g * kPrefixGroup, r1 = min(parts, r0 + kPrefixGroup);
  const int64_t per = (r1 - r0 + kPrefixSlices - 1) / kPrefixSlices;
  const int64_t a = min(r1, r0 + q * per), b = min(r1, a + per);
  uint32_t s = 0;
#pragma unroll 8
  for (int64_t r = a; r < b; ++r) s += counts[(size_t)r * kRadix + d];
  s_part[q][d] = s;
  __syncthreads();
  uint32_t off = gprefix[(size_t)g * kRadix + d];
#pragma unroll
  for (int i = 0; i < kPrefixSlices; ++i) off += i < q ? s_part[i][d] : 0u;
  for (int64_t r = a; r < b; ++r) {
    const uint32_t v = counts[(size_t)r * kRadix + d];
    counts[(size_t)r * kRadix + d] = off;
    off += v;
  }
}

template <typename K>
__global__ void rs_copy(const K* __restrict__ ki, const uint32_t* __restrict__ vi, K* __restrict__ ko,
                        uint32_t* __restrict__ vo, int64_t n) {
  pdl_wait();
  pdl_trigger();
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride) {
    ko[i] = ki[i];
    vo[i] = vi[i];
  }
}

int grid_for(int64_t n, int threads, int max_blocks) {
  int64_t b = (n + threads - 1) / threads;
  if (b < 1) b = 1;
  if (b > max_blocks) b = max_blocks;
  return (int)b;
}

}  // namespace

// Opts the 8- and 16-item passes into more than 48 KB of dynamic shared
// memory (once per device and key type).
template <typename K>
static cudaError_t onesweep_smem_optin() {
  static bool done[64] = {false};
  static std::mutex mu;  // host threads may sort concurrently
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  std::lock_guard<std::mutex> lock(mu);
  if (done[dev & 63]) return cudaSuccess;
  e = cudaFuncSetAttribute(rs_onesweep<K, 16>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           (int)sizeof(OnesweepSmem<K, 16>));
  if (e == cudaSuccess)
    e = cudaFuncSetAttribute(rs_onesweep<K, 8>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             (int)sizeof(OnesweepSmem<K, 8>));
  if (e == cudaSuccess)
    e = cudaFuncSetAttribute(rs_onesweep<K, 16, false, true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             (int)sizeof(OnesweepSmem<K, 16>));
  if (e == cudaSuccess)
    e = cudaFuncSetAttribute(rs_onesweep<K, 8, false, true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             (int)sizeof(OnesweepSmem<K, 8>));
  if constexpr (sizeof(K) == 4) {
    if (e == cudaSuccess)
      e = cudaFuncSetAttribute(rs_onesweep<K, 16, true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                               (int)sizeof(OnesweepSmem<K, 16>));
    if (e == cudaSuccess)
      e = cudaFuncSetAttribute(rs_onesweep<K, 8, true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                               (int)sizeof(OnesweepSmem<K, 8>));
  }
  if (e == cudaSuccess) done[dev & 63] = true;
  return e;
}

static int sort_items(int64_t n) {
  // Enough partitions to put about two CTAs on every SM: a pass over few keys
  // is latency-bound, and a smaller partition shortens each CTA's serial work.
  if (n >= (int64_t)kSortThreads * 16 * 296) return 16;
  if (n >= (int64_t)kSortThreads * 8 * 296) return 8;
  return 4;
}

template <typename K, bool kRanges, bool kPrefix = false>
static auto onesweep_kernel(int items) {
  return items == 16 ? rs_onesweep<K, 16, kRanges, kPrefix>
                     : items == 8 ? rs_onesweep<K, 8, kRanges, kPrefix> : rs_onesweep<K, 4, kRanges, kPrefix>;
}

template <typename K>
static cudaError_t radix_sort_pairs_t(Carver& ws, const K* keys_in, const uint32_t* vals_in, K* keys_out,
                                      uint32_t* vals_out, int64_t n, int begin_bit, int end_bit, uint32_t* status,
                                      cudaStream_t stream, bool scratch_zeroed, const uint32_t* digit_hist,
                                      SortRanges ranges) {
  const int passes = sort_passes(begin_bit, end_bit);
  const int items = sort_items(n);
  const int64_t tile = (int64_t)kSortThreads * items;
  const int64_t parts = (n + tile - 1) / tile;
  // Scratch layout (identical in measuring and running mode). Histograms,
  // partition counters and look-back words are contiguous: one memset clears them.
  K* k_tmp = ws.take<K>(passes > 1 ? (size_t)n : 0);
  uint32_t* v_tmp = ws.take<uint32_t>(passes > 1 ? (size_t)n : 0);
  const size_t zero_words = (size_t)kMaxPasses * kRadix + kMaxPasses + (size_t)passes * (size_t)parts * kRadix;
  uint32_t* zeroed = ws.take<uint32_t>(zero_words);
  uint32_t* hist = digit_hist ? const_cast<uint32_t*>(digit_hist) : zeroed;
  uint32_t* counters = zeroed + (size_t)kMaxPasses * kRadix;
  uint32_t* lookback = counters + kMaxPasses;
  // Reduce-then-scan for the first pass (rs_part_counts): per-partition counts
  // of every pass, then group sums. Fully written, never cleared.
  const bool prefix_mode = n >= kPrefixMinN && passes >= 2;
  const int groups = (int)((parts + kPrefixGroup - 1) / kPrefixGroup);
  uint32_t* pcounts = ws.take<uint32_t>(prefix_mode ? (size_t)passes * (size_t)parts * kRadix : 0);
  uint32_t* gsum = ws.take<uint32_t>(prefix_mode ? (size_t)passes * (size_t)groups * kRadix : 0);
  if (prefix_mode) hist = zeroed;  // rs_group_scan writes the totals of every pass there
  if (ws.base == nullptr) return cudaSuccess;
  if (n <= 0) return cudaSuccess;
  if (passes == 0) {
    launch_pdl(rs_copy<K>, grid_for(n, 256, 148 * 8), 256, 0, stream, keys_in, vals_in, keys_out, vals_out, n);
    note_launches(1);
    return cudaGetLastError();
  }
  const int last_bits = (end_bit - begin_bit) - (passes - 1) * kRadixBits;
  cudaError_t e = onesweep_smem_optin<K>();
  if (e != cudaSuccess) return e;
  if (!scratch_zeroed) {
    e = cudaMemsetAsync(zeroed, 0, sizeof(uint32_t) * zero_words, stream);
    if (e != cudaSuccess) return e;
  }
  if (prefix_mode) {
    auto counts_kernel = items == 16 ? rs_part_counts<K, 16> : items == 8 ? rs_part_counts<K, 8> : rs_part_counts<K, 4>;
    launch_pdl(counts_kernel, (unsigned)parts, kSortThreads, 0, stream, keys_in, n, begin_bit, passes, last_bits,
               pcounts, parts);
    launch_pdl(rs_group_sums, dim3((unsigned)groups, (unsigned)passes), kPrefixThreads, 0, stream,
               (const uint32_t*)pcounts, parts, gsum, groups);
    launch_pdl(rs_group_scan, 1, kPrefixThreads, 0, stream, gsum, groups, passes, hist);
    launch_pdl(rs_part_prefix, (unsigned)groups, kPrefixThreads, 0, stream, pcounts, parts, (const uint32_t*)gsum);
    note_launches(4);
  } else if (!digit_hist) {
    launch_pdl(rs_histogram<K>, grid_for((n + kHistItems - 1) / kHistItems, kSortThreads, 148 * 4), kSortThreads, 0,
               stream, keys_in, n, begin_bit, passes, last_bits, hist);
    note_launches(1);
  }
  // Ping-pong so the last pass writes keys_out: pass p writes out when
  // (passes-1-p) is even, else tmp.
  const K* ki = keys_in;
  const uint32_t* vi = vals_in;
  for (int p = 0; p < passes; ++p) {
    const bool to_out = ((passes - 1 - p) % 2) == 0;
    K* ko = to_out ? keys_out : k_tmp;
    uint32_t* vo = to_out ? vals_out : v_tmp;
    const int bits = (p == passes - 1) ? last_bits : kRadixBits;
    auto kernel = onesweep_kernel<K, false>(items);
    if (prefix_mode && p == 0) kernel = onesweep_kernel<K, false, true>(items);
    if constexpr (sizeof(K) == 4)
      if (ranges.first && p == passes - 1) kernel = onesweep_kernel<K, true>(items);
    const size_t smem = items == 16 ? sizeof(OnesweepSmem<K, 16>)
                                    : items == 8 ? sizeof(OnesweepSmem<K, 8>) : sizeof(OnesweepSmem<K, 4>);
    launch_pdl(kernel, (unsigned)parts, kSortThreads, smem, stream, 
        ki, vi, ko, vo, n, begin_bit + p * kRadixBits, bits, hist + p * kRadix,
        lookback + (size_t)p * (size_t)parts * kRadix, counters + p, status, ranges.first, ranges.block, ranges.n,
        (const uint32_t*)pcounts);
    note_launches(1);
    ki = ko;
    vi = vo;
  }
  return cudaGetLastError();
}

cudaError_t radix_sort_pairs(Carver& ws, const uint64_t* keys_in, const uint32_t* vals_in, uint64_t* keys_out,
                             uint32_t* vals_out, int64_t n, int begin_bit, int end_bit, uint32_t* status,
                             cudaStream_t stream, bool scratch_zeroed, const uint32_t* digit_hist) {
  return radix_sort_pairs_t(ws, keys_in, vals_in, keys_out, vals_out, n, begin_bit, end_bit, status, stream,
                            scratch_zeroed, digit_hist, SortRanges{});
}

cudaError_t radix_sort_pairs(Carver& ws, const uint32_t* keys_in, const uint32_t* vals_in, uint32_t* keys_out,
                             uint32_t* vals_out, int64_t n, int begin_bit, int end_bit, uint32_t* status,
                             cudaStream_t stream, bool scratch_zeroed, const uint32_t* digit_hist,
                             SortRanges ranges) {
  return radix_sort_pairs_t(ws, keys_in, vals_in, keys_out, vals_out, n, begin_bit, end_bit, status, stream,
                            scratch_zeroed, digit_hist, ranges);
}

template <typename K>
static ZeroRegion radix_sort_zero_region_t(Carver ws, int64_t n, int begin_bit, int end_bit) {
  const int passes = sort_passes(begin_bit, end_bit);
  const int64_t tile = (int64_t)kSortThreads * sort_items(n);
  const int64_t parts = (n + tile - 1) / tile;
  ws.take<K>(passes > 1 ? (size_t)n : 0);
  ws.take<uint32_t>(passes > 1 ? (size_t)n : 0);
  const size_t zero_words = (size_t)kMaxPasses * kRadix + kMaxPasses + (size_t)passes * (size_t)parts * kRadix;
  ZeroRegion z;
  z.words = zero_words;
  z.ptr = ws.take<uint32_t>(zero_words);
  return z;
}

ZeroRegion radix_sort_zero_region(Carver ws, int64_t n, int begin_bit, int end_bit, bool keys32) {
  return keys32 ? radix_sort_zero_region_t<uint32_t>(ws, n, begin_bit, end_bit)
                : radix_sort_zero_region_t<uint64_t>(ws, n, begin_bit, end_bit);
}

}  // namespace gsb

extern "C" size_t gsb_radix_sort_pairs_workspace_size(int64_t n, int begin_bit, int end_bit) {
  gsb::Carver c(nullptr);
  gsb::radix_sort_pairs(c, (const uint64_t*)nullptr, nullptr, nullptr, nullptr, n, begin_bit, end_bit, nullptr, 0,
                        false);
  return c.off + 256;
}

extern "C" int gsb_radix_sort_pairs(const uint64_t* keys_in, const uint32_t* vals_in,
                                    uint64_t* keys_out, uint32_t* vals_out, int64_t n,
                                    int begin_bit, int end_bit, uint32_t* status, void* workspace,
                                    size_t workspace_bytes, void* stream) {
  if (n < 0 || begin_bit < 0 || end_bit > 64 || end_bit < begin_bit) return GSB_ERR_INVALID_ARGUMENT;
  if (n > gsb::kSortMaxN) return GSB_ERR_CAPACITY;
  if (n > 0 && (!keys_in || !vals_in || !keys_out || !vals_out || !status)) return GSB_ERR_INVALID_ARGUMENT;
  if (keys_in == keys_out && n > 0) return GSB_ERR_INVALID_ARGUMENT;
  if (workspace_bytes < gsb_radix_sort_pairs_workspace_size(n, begin_bit, end_bit)) return GSB_ERR_WORKSPACE;
  if (n > 0 && workspace == nullptr) return GSB_ERR_WORKSPACE;
  gsb::Carver c(workspace);
  const cudaError_t e = gsb::radix_sort_pairs(c, keys_in, vals_in, keys_out, vals_out, n, begin_bit, end_bit,
                                              status, static_cast<cudaStream_t>(stream), false);
  return e == cudaSuccess ? GSB_OK : GSB_ERR_CUDA;
}

// ---------------------------------------------------------------------------
// Allocation-free sort (gsb_radix_sort_pairs_noalloc): the same sort with its
// scratch (temporary keys and values, digit histograms, partition counters and
// look-back words) in a fixed device array of this library instead of a
// caller-provided workspace. It serves callers that cannot allocate device
// memory at all, such as a host application that budgets every byte of GPU
// memory itself and hands a plugin only the buffers of each call.
//
// The array is a file-scope __device__ variable: every GPU that loads this
// library holds kNoallocScratchBytes of it until the process exits. Its name is
// only a host-side stand-in in host code, so the host looks its device address
// up once per device (cudaGetSymbolAddress, with that device current) and
// passes that address to the kernels.
// ---------------------------------------------------------------------------
namespace gsb {
namespace {

constexpr int64_t kNoallocMaxPairs = GSB_SORT_NOALLOC_MAX_PAIRS;
// Scratch of the largest allowed sort (2^18 pairs, 64 key bits: 8 passes of
// 1,024-key partitions) is 2 MiB of keys, 1 MiB of values and 2.1 MB of
// histograms and look-back words; the set-up checks that it fits.
constexpr size_t kNoallocScratchBytes = GSB_SORT_NOALLOC_SCRATCH_BYTES;
constexpr int kNoallocMaxDevices = 64;

__device__ __align__(256) unsigned char g_sort_scratch[kNoallocScratchBytes];

// Device address of g_sort_scratch on the current device, looked up on the
// first call for that device (under a lock: host threads may sort at once).
int noalloc_scratch(void** out) {
  static void* addr[kNoallocMaxDevices] = {};
  static std::mutex mu;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return GSB_ERR_CUDA;
  if (dev < 0 || dev >= kNoallocMaxDevices) return GSB_ERR_UNSUPPORTED;
  std::lock_guard<std::mutex> lock(mu);
  if (addr[dev] == nullptr) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_sort_scratch) != cudaSuccess || p == nullptr) return GSB_ERR_CUDA;
    addr[dev] = p;
  }
  *out = addr[dev];
  return GSB_OK;
}

}  // namespace
}  // namespace gsb

extern "C" int gsb_radix_sort_pairs_noalloc(const uint64_t* keys_in, const uint32_t* vals_in, uint64_t* keys_out,
                                            uint32_t* vals_out, int64_t n, int begin_bit, int end_bit,
                                            uint32_t* status, void* stream) {
  if (n < 0 || begin_bit < 0 || end_bit > 64 || end_bit < begin_bit) return GSB_ERR_INVALID_ARGUMENT;
  if (n > gsb::kNoallocMaxPairs) return GSB_ERR_CAPACITY;
  if (n > 0 && (!keys_in || !vals_in || !keys_out || !vals_out || !status)) return GSB_ERR_INVALID_ARGUMENT;
  if (keys_in == keys_out && n > 0) return GSB_ERR_INVALID_ARGUMENT;
  if (gsb_radix_sort_pairs_workspace_size(n, begin_bit, end_bit) > gsb::kNoallocScratchBytes)
    return GSB_ERR_CAPACITY;
  if (n == 0) return GSB_OK;
  void* scratch = nullptr;
  const int rc = gsb::noalloc_scratch(&scratch);
  if (rc != GSB_OK) return rc;
  // scratch_zeroed = false: the sort clears its histograms, counters and
  // look-back words (left over from the previous call) with a memset first.
  gsb::Carver c(scratch);
  const cudaError_t e = gsb::radix_sort_pairs(c, keys_in, vals_in, keys_out, vals_out, n, begin_bit, end_bit,
                                              status, static_cast<cudaStream_t>(stream), false);
  return e == cudaSuccess ? GSB_OK : GSB_ERR_CUDA;
}
