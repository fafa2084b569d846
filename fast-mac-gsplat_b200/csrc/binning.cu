// Tile binning on sm_100a: depth sort, exact tile-overlap counts, decoupled
// look-back scan, deterministic pair emission, stable tile sort, tile ranges.
//
// Reference behaviour (nbardy/fast-mac-gsplat):
//   depth sort + gathers   variants/v8_project3d/torch_gsplat_bridge_v8_project3d/rasterize.py:708-717
//   count_tiles            variants/v8_project3d/csrc/metal/gsplat_v8_project3d_kernels.metal:697-741
//   cumsum + .item()       variants/v8_project3d/csrc/metal/gsplat_metal.mm:358-364
//   emit_binned_ids        …/gsplat_v8_project3d_kernels.metal:743-780 (atomic cursors)
//   bitonic_sort_ids       …/gsplat_v8_project3d_kernels.metal:594-617
// The B200 design replaces the per-tile atomic cursors + per-tile bitonic sort
// with deterministic scan offsets in depth-rank order followed by a stable
// radix sort on the tile bits, so every output is bit-reproducible.
#include <algorithm>

#include "gsb_common.cuh"
#include "gsb_host.cuh"
#include "radix_sort.cuh"

namespace gsb {
namespace {

constexpr int kScanThreads = 256;
constexpr int kScanItems = 2;
constexpr int kScanTile = kScanThreads * kScanItems;
constexpr unsigned long long kScanAgg = 1ull << 62;
constexpr unsigned long long kScanInc = 2ull << 62;
constexpr unsigned long long kScanMask = (1ull << 62) - 1ull;
constexpr int kLookWin = 8;  // predecessors read per look-back step

// One splat's candidate tiles (its snugbox in tiles, row-major) and the
// constants of the exact ellipse-rectangle test. The two divisions of
// ellipse_rect do not depend on the tile and are taken once here; the test
// then evaluates the same correctly rounded operation sequence per tile.
struct SplatTiles {
  float mx, my, a, b, c, tau, kc, ka, b2;  // b2 = 2b (exact: a power-of-two product)
  float rw;  // 1 / w, correctly rounded (cand_row)
  int tx0, ty0, w, n;  // candidates [tx0, tx0 + w) x [ty0, ty0 + n / w); n = 0: none
};

// quad_form with its constant factor 2b taken once per splat: the same
// correctly rounded operation sequence, so the same value bit for bit.
__device__ __forceinline__ float quad_form_b2(float a, float b2, float c, float dx, float dy) {
  const float t0 = __fmul_rn(__fmul_rn(a, dx), dx);
  const float t1 = __fmul_rn(__fmul_rn(b2, dx), dy);
  const float t2 = __fmul_rn(__fmul_rn(c, dy), dy);
  return __fadd_rn(__fadd_rn(t0, t1), t2);
}

__device__ __forceinline__ SplatTiles splat_tiles(float mx, float my, float a, float b, float c, float op,
                                                  const Meta& m) {
  SplatTiles s;
  s.mx = mx, s.my = my, s.a = a, s.b = b, s.c = c, s.b2 = __fmul_rn(2.0f, b);
  s.tau = 0.0f, s.kc = 0.0f, s.ka = 0.0f;
  s.rw = 1.0f;
  s.tx0 = 0, s.ty0 = 0, s.w = 1, s.n = 0;
  float tau;
  if (!support_tau(op, m.alpha_thr, m.eps, &tau)) return s;
  const PixBox bb = snugbox(mx, my, a, b, c, tau, m.W, m.H, m.eps);
  if (bb.x0 > bb.x1 || bb.y0 > bb.y1) return s;
  s.tau = tau;
  s.tx0 = bb.x0 / kTile;
  s.ty0 = bb.y0 / kTile;
  s.w = bb.x1 / kTile - s.tx0 + 1;
  s.n = s.w * (bb.y1 / kTile - s.ty0 + 1);
  s.rw = __frcp_rn((float)s.w);
  if (c > 1e-8f) s.kc = -__fdiv_rn(b, c);
  if (a > 1e-8f) s.ka = -__fdiv_rn(b, a);
  return s;
}

// ellipse_rect of tile (tx, ty) with the hoisted constants (same decisions).
__device__ __forceinline__ bool tile_hit(const SplatTiles& s, int tx, int ty, const Meta& m) {
  const float rx0 = tile_rx0(tx), rx1 = tile_rx1(tx, m.W);
  const float ry0 = tile_rx0(ty), ry1 = tile_rx1(ty, m.H);
  if (s.mx >= rx0 && s.mx <= rx1 && s.my >= ry0 && s.my <= ry1) return true;
  const float dx0 = __fsub_rn(rx0, s.mx);
  const float dx1 = __fsub_rn(rx1, s.mx);
  const float dy0 = __fsub_rn(ry0, s.my);
  const float dy1 = __fsub_rn(ry1, s.my);
  float qmin = __int_as_float(0x7f800000);
  qmin = fminf(qmin, quad_form_b2(s.a, s.b2, s.c, dx0, dy0));
  qmin = fminf(qmin, quad_form_b2(s.a, s.b2, s.c, dx0, dy1));
  qmin = fminf(qmin, quad_form_b2(s.a, s.b2, s.c, dx1, dy0));
  qmin = fminf(qmin, quad_form_b2(s.a, s.b2, s.c, dx1, dy1));
  if (s.c > 1e-8f) {
    float dy = fminf(fmaxf(__fmul_rn(s.kc, dx0), dy0), dy1);
    qmin = fminf(qmin, quad_form_b2(s.a, s.b2, s.c, dx0, dy));
    dy = fminf(fmaxf(__fmul_rn(s.kc, dx1), dy0), dy1);
    qmin = fminf(qmin, quad_form_b2(s.a, s.b2, s.c, dx1, dy));
  }
  if (s.a > 1e-8f) {
    float dx = fminf(fmaxf(__fmul_rn(s.ka, dy0), dx0), dx1);
    qmin = fminf(qmin, quad_form_b2(s.a, s.b2, s.c, dx, dy0));
    dx = fminf(fmaxf(__fmul_rn(s.ka, dy1), dx0), dx1);
    qmin = fminf(qmin, quad_form_b2(s.a, s.b2, s.c, dx, dy1));
  }
  return qmin <= s.tau;
}

// Row of candidate `local` (0 <= local < n) of a splat whose box is w tiles
// wide; rw = 1 / w (the estimate is corrected to the exact quotient).
__device__ __forceinline__ int cand_row(int local, int w, float rw) {
  int r = (int)(((float)local + 0.5f) * rw);
  while (r > 0 && r * w > local) --r;
  while ((r + 1) * w <= local) ++r;
  return r;
}
__device__ __forceinline__ int cand_row(int local, int w) { return cand_row(local, w, __frcp_rn((float)w)); }

// Hit tiles of a splat row by row (k_prepare). Within one row of tiles (a
// horizontal strip of pixel centres [ry0, ry1]) the support ellipse q <= T is
// convex, so the row's tiles that meet it are the ones whose column range
// [rx0, rx1] meets the ellipse's x-extent inside the strip: one run of tiles.
// For T_in = tau (1 - 2^-7) and T_out = tau (1 + 2^-7) that gives, per row,
// the tiles that surely hit and the only ones that can; the tiles between the
// two runs (one or two at each end of a row) go to the exact tile_hit. So the
// hit sets stay exactly the reference's while the work is per row, not per
// candidate tile.
//
// Why it is sound. Let q(p) = d^T A d (d = p - mean, A = [[a, b], [b, c]]).
// For a positive definite A with a, c > 1e-8 the points tile_hit evaluates
// (the mean when it lies in the rectangle, the 4 corners, and the minimum of q
// on each edge at the clamped stationary point) include a minimiser of q over
// the rectangle, so its float minimum differs from the exact minimum only by
// rounding. Each evaluated q is a sum of three products of correctly rounded
// factors, within about 9 eps (a dx^2 + 2|b dx dy| + c dy^2) <= 18 eps k q of
// its exact value, with k = (a + c) / lambda_min <= (a + c)^2 / det. The float
// rectangle corners (rx - mx rounded) move the evaluated points by at most
// eps (|d| + 32) px, which changes q by a relative 3 eps (R_major + 32) /
// R_minor at the threshold (R = sqrt(tau / lambda)). span_geom admits a splat
// only when k <= 2^12 and lambda_max <= a + c <= 2^8 tau (R_minor >= 1/16 px),
// which bounds both effects by 4.5e-3 of tau, below the 2^-7 (7.8e-3) between
// tau and T_in, T_out. A tile that meets the ellipse at T_in therefore has a
// float minimum below tau (a hit); one that misses it at T_out has every
// evaluated q above tau (a miss). The extents are computed in float relative
// to the mean (strip_extent bounds their effect on q at 1e-4 tau, far inside
// the margin), and the tile columns are found by comparisons with the float
// rectangle edges.
constexpr double kSpanMargin = 0x1p-7;
// Splats with fewer candidate tiles take the exact test for each: for them the
// row walk's setup costs more than the tests it saves.
constexpr int kSpanMinCands = 32;

struct SpanGeom {
  float det, ia, bc;          // ia = 1 / a, bc = b / c (the mean and b: the splat's floats)
  float E[2], XR[2], aT[2];  // per threshold (0: T_in, 1: T_out): y and x half extents, a T
};

// The constants of the row walk, or false when the splat is outside the
// conditions above (it then takes the exact test for every candidate). The
// admission test is done in double; the constants are rounded to float.
__device__ __forceinline__ bool span_geom(const SplatTiles& s, SpanGeom& g) {
  if (s.n < kSpanMinCands) return false;
  const float a = s.a, b = s.b, c = s.c;
  if (!(a > 1e-8f) || !(c > 1e-8f) || !(a < 1e30f) || !(c < 1e30f) || !(fabsf(b) < 1e30f)) return false;
  if (!(fabsf(s.mx) < 0x1p22f) || !(fabsf(s.my) < 0x1p22f)) return false;
  const double da = a, db = b, dc = c;
  const double det = da * dc - db * db;  // products exact in double
  const double tr = da + dc;
  if (!(det > 0.0) || !(tr * tr <= 4096.0 * det) || !(tr <= 256.0 * (double)s.tau)) return false;
  g.det = (float)det, g.ia = (float)(1.0 / da), g.bc = (float)(db / dc);
#pragma unroll
  for (int k = 0; k < 2; ++k) {
    const double T = (double)s.tau * (k ? 1.0 + kSpanMargin : 1.0 - kSpanMargin);
    g.E[k] = (float)sqrt(da * T / det);
    g.XR[k] = (float)sqrt(dc * T / det);
    g.aT[k] = (float)(da * T);
  }
  return true;
}

// x-extent [xl, xr] (relative to the mean) of the ellipse q <= T_k within the
// strip e in [e0, e1] (relative to the mean); false when they do not meet.
// The right boundary x(e) = (-b e + sqrt(a T - det e^2)) / a is concave with its
// maximum XR at e = -(b / c) XR, the left one convex with its minimum -XR at
// e = (b / c) XR; off those points the extreme is at an end of the strip.
// In float: an error dD in D = a T - det e^2 (at most about 2^-22 a T here)
// moves the boundary where dq/dx = 2 sqrt(D), so q changes by at most 2 dD / a
// (2^-21 T); the -b e / a term, the square root and the division add relative
// errors of a few 2^-24 in x, which change q by at most 2^-18 T (|b| <= 32
// sqrt(det) under the k <= 2^12 admission); the strip ends and the column
// edges are taken relative to the mean (fl(r - m), off by 2^-24 |r - m|), which
// changes q by at most 2^-23 (R + 16) / R_minor < 4e-5 T. All stay far inside
// the 2^-7 margin.
__device__ __forceinline__ bool strip_extent(const SpanGeom& g, float b, int k, float e0, float e1, float& xl,
                                             float& xr) {
  const float lo = fmaxf(e0, -g.E[k]), hi = fminf(e1, g.E[k]);
  if (!(lo <= hi)) return false;
  const float es = g.bc * g.XR[k];
  const float sl = sqrtf(fmaxf(fmaf(-g.det * lo, lo, g.aT[k]), 0.0f));
  const float sh = sqrtf(fmaxf(fmaf(-g.det * hi, hi, g.aT[k]), 0.0f));
  const float cl = -b * lo, ch = -b * hi;
  xr = (-es >= lo && -es <= hi) ? g.XR[k] : fmaxf(cl + sl, ch + sh) * g.ia;
  xl = (es >= lo && es <= hi) ? -g.XR[k] : fminf(cl - sl, ch - sh) * g.ia;
  return true;
}

// Column rectangle edges as tile_rx0 / tile_rx1 compute them (the same float
// values), with (float)t formed as (2^23 + t) - 2^23, exact for 0 <= t < 2^23,
// instead of a conversion instruction.
__device__ __forceinline__ float col_float(int t) { return __int_as_float(0x4B000000 | t) - 8388608.0f; }
__device__ __forceinline__ float col_rx0(int t) { return fmaf(16.0f, col_float(t), 0.5f); }
__device__ __forceinline__ float col_rx1(int t, float rmax) { return fminf(rmax, fmaf(16.0f, col_float(t), 15.5f)); }

// First column t in [t0, t1] whose rectangle reaches right of x (rx1 - mx >= x,
// relative to the mean mx), or t1 + 1; last column in [t0, t1] reaching left of
// x (rx0 - mx <= x), or t0 - 1. rmax = tile_rx1's image clip, (W - 1) + 0.5.
// The estimate is corrected by the comparisons themselves, which are monotone
// in t.
__device__ __forceinline__ int first_col_reaching(float x, float mx, int t0, int t1, float rmax) {
  int t = min(max(__float2int_ru((mx + x - 15.5f) * 0.0625f), t0), t1 + 1);
  while (t > t0 && col_rx1(t - 1, rmax) - mx >= x) --t;
  while (t <= t1 && col_rx1(t, rmax) - mx < x) ++t;
  return t;
}
__device__ __forceinline__ int last_col_reaching(float x, float mx, int t0, int t1) {
  int t = min(max(__float2int_rd((mx + x - 0.5f) * 0.0625f), t0 - 1), t1);
  while (t < t1 && col_rx0(t + 1) - mx <= x) ++t;
  while (t >= t0 && col_rx0(t) - mx > x) --t;
  return t;
}

constexpr int kMaskCands = 64;  // splats with at most this many candidate tiles keep a hit mask
// Larger splats keep their hit bits in the region after the per-splat slots of
// tile_masks: kBigMaskWords words per splat on average are reserved, handed out
// in splat-sized pieces by an atomic cursor (status word GSB_STATUS_MASK_WORDS).
// A splat that finds the region full keeps no bits and is tested again by k_emit.
constexpr uint32_t kBigMaskWords = 8;
constexpr unsigned long long kNoBigMask = ~0ull;

// Per-warp shared state of warp_tiles and warp_count_tiles.
struct WarpTilesSmem {
  SplatTiles t[32];
  int incl[32];                  // inclusive scan of the candidate counts
  int hits[32];                  // running hit count per owner
  unsigned long long mask[32];   // hit mask per owner with <= kMaskCands candidates (warp_count_tiles)
  int big[32];                   // word offset of a larger owner's hit bits, or -1
};

// Hit bits of splats with more than kMaskCands candidates (k_prepare writes,
// k_emit reads): words[big + (local >> 5)] bit (local & 31) marks candidate local.
struct BigBits {
  uint32_t* words = nullptr;  // nullptr: none
  uint32_t capacity = 0;      // words in the region
  uint32_t* cursor = nullptr; // words handed out so far (k_prepare)
};

// Owner of concatenated candidate k (0 <= k < the warp's total): the first
// lane whose inclusive candidate count exceeds k.
__device__ __forceinline__ int find_owner(const int* incl, int k) {
  int lo = 0, hi = 31;
#pragma unroll
  for (int step = 0; step < 5; ++step) {
    const int mid = (lo + hi) >> 1;
    if (incl[mid] > k) hi = mid;
    else lo = mid + 1;
  }
  return lo;
}

// Visits every candidate tile of the warp's 32 splats (lane j owns splat j),
// spread evenly over the lanes: round r tests candidates 32r .. 32r+31 of the
// warp's concatenated row-major candidate lists, so a warp costs its total
// candidate count / 32 rounds however unevenly the splats are sized. Hits are
// numbered per owner in row-major tile order (the reference's loop order):
// visit(owner, tx, ty, slot) runs for each hit with slot = its index in the
// owner's list. On return sm.hits[j] is splat j's hit count.
template <typename Visit>
__device__ __forceinline__ void warp_tiles(const SplatTiles& mine, const Meta& m, WarpTilesSmem& sm, Visit&& visit) {
  const int lane = threadIdx.x & 31;
  long long incl = mine.n;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const long long y = __shfl_up_sync(kFullMask, incl, o);
    if (lane >= o) incl += y;
  }
  const long long total = __shfl_sync(kFullMask, incl, 31);
  sm.hits[lane] = 0;
  sm.t[lane] = mine;
  if (total > 0x7fffffffll) {
    // Beyond int range for the warp: each lane walks its own candidates.
    int cnt = 0;
    for (int local = 0; local < mine.n; ++local) {
      const int row = cand_row(local, mine.w, mine.rw);
      const int tx = mine.tx0 + (local - row * mine.w), ty = mine.ty0 + row;
      if (tile_hit(mine, tx, ty, m)) visit(lane, tx, ty, cnt++);
    }
    sm.hits[lane] = cnt;
    __syncwarp();
    return;
  }
  sm.incl[lane] = (int)incl;
  __syncwarp();
  for (int base = 0; base < (int)total; base += 32) {
    const int k = base + lane;
    int owner = -1, tx = 0, ty = 0;
    bool hit = false;
    if (k < (int)total) {
      owner = find_owner(sm.incl, k);
      const SplatTiles& s = sm.t[owner];
      const int local = k - (owner ? sm.incl[owner - 1] : 0);
      const int row = cand_row(local, s.w, s.rw);
      tx = s.tx0 + (local - row * s.w);
      ty = s.ty0 + row;
      hit = tile_hit(s, tx, ty, m);
    }
    // Owners are non-decreasing across lanes: segments of equal owner.
    const int prev = __shfl_up_sync(kFullMask, owner, 1);
    const unsigned starts = __ballot_sync(kFullMask, lane == 0 || owner != prev);
    const unsigned hits = __ballot_sync(kFullMask, hit);
    const unsigned le = (lane == 31) ? 0xffffffffu : ((2u << lane) - 1u);
    const int seg0 = 31 - __clz(starts & le);
    const unsigned above = starts & ~le;
    const unsigned seg = (above ? ((1u << (__ffs(above) - 1)) - 1u) : 0xffffffffu) & ~((1u << seg0) - 1u);
    const int before = __popc(hits & seg & ((1u << lane) - 1u));
    const int base_slot = owner >= 0 ? sm.hits[owner] : 0;
    __syncwarp();
    if (lane == seg0 && owner >= 0) sm.hits[owner] = base_slot + __popc(hits & seg);
    if (hit) visit(owner, tx, ty, base_slot + before);
    __syncwarp();
  }
}

// k_prepare's per-warp shared state: warp_tiles' arrays, the row-walk
// constants of the lanes' splats, and the queue of tiles left to the exact test.
struct CountSmem {
  WarpTilesSmem t;
  SpanGeom g[32];
  int qlocal[64];
  unsigned char qowner[64];
};

// Hit counts (sm.hits), hit masks (sm.mask, splats with <= kMaskCands
// candidates) and hit-bit words (`big`) of the warp's 32 splats, for k_prepare.
// Splats that meet span_geom's conditions are walked row by row (rounds of 32
// rows of the warp's splats, one row per lane): the sure run of each row is
// counted and its bits are ORed in at once, and the unsure tiles at the ends of
// the runs are queued and run through tile_hit 32 at a time. The others take
// tile_hit for every candidate: a larger one with hit-bit words is walked by
// the whole warp on its own, 32 candidates per round in row-major order (the
// round's ballot is its hit word, written whole), the rest share rounds of 32
// candidates as in warp_tiles.
__device__ __forceinline__ void warp_count_tiles(const SplatTiles& mine, const Meta& m, CountSmem& cs, BigBits big) {
  WarpTilesSmem& sm = cs.t;
  const int lane = threadIdx.x & 31;
  const unsigned lt = (1u << lane) - 1u;
  SpanGeom geom;
  const bool span = span_geom(mine, geom);
  // One cursor atomic per warp: the lanes' word counts are summed, and each
  // lane takes its piece of the warp's range (if the range fits, else none).
  int b = -1;
  if (big.words) {
    const uint32_t words = mine.n > kMaskCands ? ((uint32_t)mine.n + 31u) >> 5 : 0u;
    uint32_t excl = words;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const uint32_t y = __shfl_up_sync(kFullMask, excl, o);
      if (lane >= o) excl += y;
    }
    const uint32_t warp_words = __shfl_sync(kFullMask, excl, 31);
    excl -= words;
    uint32_t at = 0u;
    if (lane == 0 && warp_words) at = atomicAdd(big.cursor, warp_words);
    at = __shfl_sync(kFullMask, at, 0);
    if (words && at <= big.capacity && warp_words <= big.capacity - at) b = (int)(at + excl);
  }
  sm.big[lane] = b;
  sm.t[lane] = mine;
  sm.mask[lane] = 0ull;
  sm.hits[lane] = 0;
  if (span) cs.g[lane] = geom;
  __syncwarp();

  // 1. Exact walk of the larger splats outside the row walk that got words.
  unsigned walk = __ballot_sync(kFullMask, b >= 0 && !span);
  while (walk) {
    const int j = __ffs(walk) - 1;
    walk &= walk - 1;
    const SplatTiles& s = sm.t[j];
    const int bj = sm.big[j];
    int hits = 0;
    for (int base = 0; base < s.n; base += 32) {
      const int local = base + lane;
      bool hit = false;
      if (local < s.n) {
        const int row = cand_row(local, s.w, s.rw);
        hit = tile_hit(s, s.tx0 + (local - row * s.w), s.ty0 + row, m);
      }
      const unsigned bal = __ballot_sync(kFullMask, hit);
      hits += __popc(bal);
      if (lane == 0) big.words[bj + (base >> 5)] = bal;
    }
    if (lane == 0) sm.hits[j] = hits;
  }
  // 2. The words of the row-walked splats are cleared (their runs are ORed in).
  unsigned clear = __ballot_sync(kFullMask, b >= 0 && span);
  while (clear) {
    const int j = __ffs(clear) - 1;
    clear &= clear - 1;
    uint32_t* const w = big.words + sm.big[j];
    for (int i = lane; i < (sm.t[j].n + 31) >> 5; i += 32) w[i] = 0u;
  }
  __syncwarp();

  // 3. Exact shared rounds for the other splats outside the row walk.
  {
    const int n = (!span && b < 0) ? mine.n : 0;
    long long incl = n;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const long long y = __shfl_up_sync(kFullMask, incl, o);
      if (lane >= o) incl += y;
    }
    const long long total = __shfl_sync(kFullMask, incl, 31);
    if (total > 0x7fffffffll) {
      // Beyond int range for the warp: each lane tests its own candidates.
      int cnt = 0;
      unsigned long long mask = 0ull;
      for (int local = 0; local < n; ++local) {
        const int row = cand_row(local, mine.w, mine.rw);
        if (tile_hit(mine, mine.tx0 + (local - row * mine.w), mine.ty0 + row, m)) {
          if (n <= kMaskCands) mask |= 1ull << local;
          ++cnt;
        }
      }
      if (n > 0) sm.hits[lane] = cnt, sm.mask[lane] = mask;
    } else if (total > 0) {
      sm.incl[lane] = (int)incl;
      __syncwarp();
      for (int base = 0; base < (int)total; base += 32) {
        const int k = base + lane;
        int owner = -1, local = 0;
        bool hit = false;
        if (k < (int)total) {
          owner = find_owner(sm.incl, k);
          const SplatTiles& s = sm.t[owner];
          local = k - (owner ? sm.incl[owner - 1] : 0);
          const int row = cand_row(local, s.w, s.rw);
          hit = tile_hit(s, s.tx0 + (local - row * s.w), s.ty0 + row, m);
        }
        // Owners are non-decreasing across lanes: the first lane of each
        // segment of equal owner adds the segment's hits.
        const int prev = __shfl_up_sync(kFullMask, owner, 1);
        const unsigned starts = __ballot_sync(kFullMask, lane == 0 || owner != prev);
        const unsigned hits = __ballot_sync(kFullMask, hit);
        const unsigned le = (lane == 31) ? 0xffffffffu : ((2u << lane) - 1u);
        const int seg0 = 31 - __clz(starts & le);
        const unsigned above = starts & ~le;
        const unsigned seg = (above ? ((1u << (__ffs(above) - 1)) - 1u) : 0xffffffffu) & ~((1u << seg0) - 1u);
        if (lane == seg0 && owner >= 0) {
          sm.hits[owner] += __popc(hits & seg);
          // The segment's lanes hold consecutive candidates local, local+1, ...
          if (sm.t[owner].n <= kMaskCands) sm.mask[owner] |= (unsigned long long)((hits & seg) >> seg0) << local;
        }
        __syncwarp();
      }
    }
    __syncwarp();
  }

  // 4. Row walk of the splats that meet span_geom's conditions.
  const int rows = span ? mine.n / mine.w : 0;
  int incl = rows;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int y = __shfl_up_sync(kFullMask, incl, o);
    if (lane >= o) incl += y;
  }
  const int total = __shfl_sync(kFullMask, incl, 31);
  if (total == 0) return;
  sm.incl[lane] = incl;
  __syncwarp();
  int qn = 0;
  // The exact test of up to 32 queued tiles.
  auto flush = [&]() {
    __syncwarp();
    const int take = min(qn, 32);
    if (lane < take) {
      const int local = cs.qlocal[lane], owner = cs.qowner[lane];
      const SplatTiles& s = sm.t[owner];
      const int row = cand_row(local, s.w, s.rw);
      if (tile_hit(s, s.tx0 + (local - row * s.w), s.ty0 + row, m)) {
        atomicAdd(&sm.hits[owner], 1);
        if (s.n <= kMaskCands) atomicOr(&sm.mask[owner], 1ull << local);
        else if (sm.big[owner] >= 0) atomicOr(big.words + sm.big[owner] + (local >> 5), 1u << (local & 31));
      }
    }
    const int rest = qn - take;
    int mv = 0, mo = 0;
    if (lane < rest) mv = cs.qlocal[32 + lane], mo = cs.qowner[32 + lane];
    __syncwarp();
    if (lane < rest) cs.qlocal[lane] = mv, cs.qowner[lane] = (unsigned char)mo;
    __syncwarp();
    qn = rest;
  };
  for (int base = 0; base < total; base += 32) {
    const int k = base + lane;
    int owner = 0, row0 = 0, t0 = 0;
    int pl = 0, ph = -1, hl = 0, hh = -1;  // possible and sure column runs
    if (k < total) {
      owner = find_owner(sm.incl, k);
      const SplatTiles& s = sm.t[owner];
      const SpanGeom& g = cs.g[owner];
      const int r = k - (owner ? sm.incl[owner - 1] : 0);
      const int ty = s.ty0 + r;
      const float e0 = tile_rx0(ty) - s.my, e1 = tile_rx1(ty, m.H) - s.my;
      const float rmax = (float)(m.W - 1) + 0.5f;
      t0 = s.tx0;
      row0 = r * s.w;
      const int t1 = s.tx0 + s.w - 1;
      float xl, xr;
      if (strip_extent(g, s.b, 1, e0, e1, xl, xr)) {
        pl = first_col_reaching(xl, s.mx, t0, t1, rmax);
        ph = last_col_reaching(xr, s.mx, t0, t1);
        if (pl <= ph && strip_extent(g, s.b, 0, e0, e1, xl, xr)) {
          hl = first_col_reaching(xl, s.mx, t0, t1, rmax);
          hh = last_col_reaching(xr, s.mx, t0, t1);
        }
      }
      if (hl <= hh) {
        atomicAdd(&sm.hits[owner], hh - hl + 1);
        const int l0 = row0 + (hl - t0), l1 = row0 + (hh - t0);
        if (s.n <= kMaskCands) {
          atomicOr(&sm.mask[owner], (~0ull >> (63 - (l1 - l0))) << l0);
        } else if (sm.big[owner] >= 0) {
          uint32_t* const wd = big.words + sm.big[owner];
          for (int wi = l0 >> 5; wi <= (l1 >> 5); ++wi) {
            const int lo = max(l0 - 32 * wi, 0), hi = min(l1 - 32 * wi, 31);
            atomicOr(&wd[wi], (0xffffffffu >> (31 - (hi - lo))) << lo);
          }
        }
      }
    }
    // The unsure columns: [pl, ph] minus the sure run [hl, hh].
    int a0 = pl, a1 = ph, b0 = 0, b1 = -1;
    if (hl <= hh) a1 = hl - 1, b0 = hh + 1, b1 = ph;
    const int na = max(a1 - a0 + 1, 0), u = na + max(b1 - b0 + 1, 0);
    for (int i = 0; __any_sync(kFullMask, i < u); ++i) {
      const bool has = i < u;
      const unsigned bal = __ballot_sync(kFullMask, has);
      if (has) {
        const int col = i < na ? a0 + i : b0 + (i - na);
        const int at = qn + __popc(bal & lt);
        cs.qlocal[at] = row0 + (col - t0);
        cs.qowner[at] = (unsigned char)owner;
      }
      qn += __popc(bal);
      if (qn >= 32) flush();
    }
  }
  while (qn > 0) flush();
  __syncwarp();
}

// The depth sort's digit histogram (radix_sort_pairs' digit_hist) is counted
// by k_prepare, which writes the depth keys, instead of a histogram launch
// over them: counts in shared memory per CTA, added to the global counts once
// per CTA; the global counts are cleared by k_clear_words in the launch before.
// (The tile keys are not counted in k_emit: their low digits differ from pair
// to pair, one shared atomic each, which made the c4 emit phase 52 us slower
// than the separate histogram pass.)
constexpr int kDepthHistPasses = kSortMaxPasses;  // 64-bit depth keys

__global__ void k_clear_words(uint32_t* __restrict__ a, int na, uint32_t* __restrict__ b, int nb) {
  pdl_wait();
  pdl_trigger();
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i < na) a[i] = 0u;
  if (i < nb) b[i] = 0u;
}

__device__ __forceinline__ void flush_hist(const uint32_t* s, uint32_t* g, int words) {
  for (int i = threadIdx.x; i < words; i += blockDim.x) {
    const uint32_t v = s[i];
    if (v) atomicAdd(&g[i], v);
  }
}

// Scratch that later kernels of the same phase need cleared, zeroed by the
// phase's first kernel instead of separate memset launches.
struct ZeroList {
  uint32_t* ptr[3];
  size_t words[3];
};

__device__ __forceinline__ void zero_words(const ZeroList& z) {
  const size_t stride = (size_t)gridDim.x * blockDim.x;
  const size_t t0 = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
#pragma unroll
  for (int r = 0; r < 3; ++r)
    for (size_t i = t0; i < z.words[r]; i += stride) z.ptr[r][i] = 0u;
}

// Per splat in input order: depth-sort key (view in the high word) and the
// exact number of tiles its support ellipse touches; the pair total is added
// into status words 4-5 (64-bit) for the host's early read.
template <typename K>
__global__ void __launch_bounds__(256)
    k_prepare(Meta m, const float2* __restrict__ means2d, const float* __restrict__ conics,
              const float* __restrict__ opacities, const float* __restrict__ depths,
              K* __restrict__ sort_keys, uint32_t* __restrict__ sort_vals,
              uint32_t* __restrict__ counts, unsigned long long* __restrict__ masks, uint32_t* __restrict__ status,
              ZeroList zero, BigBits big, uint32_t* __restrict__ depth_hist, int depth_passes) {
  pdl_wait();
  pdl_trigger();
  __shared__ CountSmem s_count[8];
  __shared__ uint32_t s_hist[(sizeof(K) == 4 ? 4 : kDepthHistPasses) * kRadix];  // the depth keys' digit counts
  for (int i = threadIdx.x; i < depth_passes * kRadix; i += blockDim.x) s_hist[i] = 0u;
  __syncthreads();
  zero_words(zero);  // the depth sort's and the scan's scratch
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  const bool valid = i < m.BG;
  SplatTiles t = splat_tiles(0.f, 0.f, 0.f, 0.f, 0.f, 0.f, m);
  if (valid) {
    const int b = fast_div(i, m.div_G);
    // One view: the 32-bit depth key alone; several: the view in the high word.
    const K key = (K)(((uint64_t)(uint32_t)b << 32) | depth_key(depths[i]));
    sort_keys[i] = key;
    sort_vals[i] = (uint32_t)i;
    for (int p = 0; p < depth_passes; ++p) atomicAdd(&s_hist[p * kRadix + ((uint32_t)(key >> (8 * p)) & 255u)], 1u);
    const float2 mu = means2d[i];
    t = splat_tiles(mu.x, mu.y, conics[3 * i + 0], conics[3 * i + 1], conics[3 * i + 2], opacities[i], m);
  }
  // Splats with at most kMaskCands candidates also record which ones hit, so
  // k_emit writes their pairs without testing the tiles again.
  warp_count_tiles(t, m, s_count[warp], big);
  const WarpTilesSmem& sm = s_count[warp].t;
  const uint32_t n = valid ? (uint32_t)sm.hits[lane] : 0u;
  if (valid) {
    counts[i] = n;
    // The slot: the hit mask, or for a larger splat the word offset of its
    // hit bits (kNoBigMask when it has none).
    masks[i] = t.n <= kMaskCands ? sm.mask[lane]
                                 : (sm.big[lane] >= 0 ? (unsigned long long)sm.big[lane] : kNoBigMask);
  }
  unsigned long long wsum = n;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) wsum += __shfl_xor_sync(kFullMask, wsum, o);
  if (lane == 0 && wsum) atomicAdd(reinterpret_cast<unsigned long long*>(status + GSB_STATUS_PAIR_TOTAL64), wsum);
  __syncthreads();
  flush_hist(s_hist, depth_hist, depth_passes * kRadix);
}

// Reduce-then-scan for the pair offsets of many splats (kScanPrefixMinSplats
// up to kScanPrefixMaxParts partitions), in place of k_gather_scan's look-back:
// each partition's count total in rank order (k_scan_part_sums), then one CTA
// turns the totals into exclusive prefixes (k_scan_part_prefix), both in the
// look-back array, which that mode does not otherwise use.
constexpr int kScanPrefixMinSplats = 1 << 16;  // c1/c3 (65,536): prepare -5 us
constexpr int kScanPrefixMaxParts = 1 << 16;
constexpr int kScanPrefixThreads = 1024;

__global__ void __launch_bounds__(kScanThreads)
    k_scan_part_sums(int BG, const uint32_t* __restrict__ sorted_vals, const uint32_t* __restrict__ counts,
                     unsigned long long* __restrict__ psum) {
  pdl_wait();
  pdl_trigger();
  __shared__ unsigned long long s_warp[kScanThreads / 32];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int64_t r0 = (int64_t)blockIdx.x * kScanTile + (int64_t)tid * kScanItems;
  unsigned long long t = 0;
#pragma unroll
  for (int i = 0; i < kScanItems; ++i)
    if (r0 + i < BG) t += counts[sorted_vals[r0 + i]];
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) t += __shfl_down_sync(kFullMask, t, o);
  if (lane == 0) s_warp[warp] = t;
  __syncthreads();
  if (tid == 0) {
    unsigned long long b = 0;
#pragma unroll
    for (int w = 0; w < kScanThreads / 32; ++w) b += s_warp[w];
    psum[blockIdx.x] = b;
  }
}

// One CTA, in place: psum[p] becomes the sum of psum[q] for q < p.
__global__ void __launch_bounds__(kScanPrefixThreads) k_scan_part_prefix(unsigned long long* __restrict__ psum, int parts) {
  pdl_wait();
  pdl_trigger();
  __shared__ unsigned long long s_warp[kScanPrefixThreads / 32];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int chunk = (parts + kScanPrefixThreads - 1) / kScanPrefixThreads;
  const int lo = min(parts, tid * chunk), hi = min(parts, lo + chunk);
  unsigned long long t = 0;
  for (int p = lo; p < hi; ++p) t += psum[p];
  unsigned long long x = t;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const unsigned long long y = __shfl_up_sync(kFullMask, x, o);
    if (lane >= o) x += y;
  }
  if (lane == 31) s_warp[warp] = x;
  __syncthreads();
  unsigned long long run = x - t;
  for (int w = 0; w < warp; ++w) run += s_warp[w];
  for (int p = lo; p < hi; ++p) {
    const unsigned long long v = psum[p];
    psum[p] = run;
    run += v;
  }
}

// Gathers splats into depth-rank order (packed 48-byte records), and turns the
// per-splat tile counts into exclusive pair offsets with a single-pass chained
// scan (dynamic partition ids + decoupled look-back), or, with kPrefix, with
// the partition prefixes k_scan_part_prefix left in `lookback`.
template <typename K, bool kPrefix = false>
__global__ void __launch_bounds__(kScanThreads, 2)
    k_gather_scan(Meta m, const K* __restrict__ sorted_keys,
                  const uint32_t* __restrict__ sorted_vals, const float2* __restrict__ means2d,
                  const float* __restrict__ conics, const float* __restrict__ colors,
                  const float* __restrict__ opacities, const uint32_t* __restrict__ counts,
                  const unsigned long long* __restrict__ masks_in, unsigned long long* __restrict__ masks_out,
                  float4* __restrict__ rec, int32_t* __restrict__ perm,
                  int32_t* __restrict__ pair_offsets, unsigned long long* __restrict__ lookback,
                  uint32_t* __restrict__ part_counter, uint32_t* __restrict__ status) {
  pdl_wait();
  pdl_trigger();
  __shared__ uint32_t s_part;
  __shared__ unsigned long long s_warp[kScanThreads / 32];
  __shared__ unsigned long long s_exclusive;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  if (tid == 0) s_part = kPrefix ? blockIdx.x : atomicAdd(part_counter, 1u);
  __syncthreads();
  const int64_t part = s_part;
  const int64_t r0 = part * kScanTile + (int64_t)tid * kScanItems;

  // Loads first (all independent: the ranks' source indices, then every
  // gathered field), so a thread has all its memory requests in flight at once.
  uint32_t orig[kScanItems];
#pragma unroll
  for (int i = 0; i < kScanItems; ++i) orig[i] = (r0 + i < m.BG) ? sorted_vals[r0 + i] : 0u;
  uint32_t c[kScanItems], dk[kScanItems];
  float2 mu[kScanItems];
  float ca[kScanItems], cb[kScanItems], cc[kScanItems], op[kScanItems], cr[kScanItems], cg[kScanItems],
      cbl[kScanItems];
#pragma unroll
  for (int i = 0; i < kScanItems; ++i) {
    const bool ok = r0 + i < m.BG;
    const uint32_t o = orig[i];
    c[i] = ok ? counts[o] : 0u;
    dk[i] = ok ? (uint32_t)sorted_keys[r0 + i] : 0u;
    mu[i] = ok ? means2d[o] : make_float2(0.f, 0.f);
    ca[i] = ok ? conics[3 * o + 0] : 0.f;
    cb[i] = ok ? conics[3 * o + 1] : 0.f;
    cc[i] = ok ? conics[3 * o + 2] : 0.f;
    op[i] = ok ? opacities[o] : 0.f;
    cr[i] = ok ? colors[3 * o + 0] : 0.f;
    cg[i] = ok ? colors[3 * o + 1] : 0.f;
    cbl[i] = ok ? colors[3 * o + 2] : 0.f;
  }
  asm volatile("" ::: "memory");  // all gathers in flight before the first use
  unsigned long long tsum = 0;
#pragma unroll
  for (int i = 0; i < kScanItems; ++i) tsum += c[i];
  // Block-wide exclusive scan of the thread sums.
  unsigned long long x = tsum;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const unsigned long long y = __shfl_up_sync(kFullMask, x, o);
    if (lane >= o) x += y;
  }
  if (lane == 31) s_warp[warp] = x;
  __syncthreads();
  unsigned long long warp_off = 0, block_total = 0;
#pragma unroll
  for (int w = 0; w < kScanThreads / 32; ++w) {
    const unsigned long long v = s_warp[w];
    if (w < warp) warp_off += v;
    block_total += v;
  }
  const unsigned long long thread_excl = warp_off + x - tsum;

  if (tid == 0) {
    unsigned long long excl = 0;
    if (kPrefix) {
      excl = lookback[part];
    } else if (part == 0) {
      st_volatile_u64(&lookback[0], kScanInc | block_total);
    } else {
      st_volatile_u64(&lookback[part], kScanAgg | block_total);
      // Windowed look-back (kLookWin predecessors per L2 round trip).
      int64_t j = part - 1;
      int spins = 0;
      bool failed = false, done = false;
      while (!done && !failed) {
        unsigned long long w[kLookWin];
#pragma unroll
        for (int q = 0; q < kLookWin; ++q) w[q] = (j - q >= 0) ? ld_volatile_u64(&lookback[j - q]) : kScanInc;
#pragma unroll
        for (int q = 0; q < kLookWin; ++q) {
          if (done || failed) break;
          unsigned long long x = w[q];
          while (!(x & (kScanAgg | kScanInc))) {
            if (++spins > kSpinLimit || ((spins & 1023) == 0 && ld_volatile_u32(&status[GSB_STATUS_ERROR]))) {
              failed = true;
              break;
            }
            __nanosleep(32);
            x = ld_volatile_u64(&lookback[j - q]);
          }
          if (failed) break;
          excl += x & kScanMask;
          if (x & kScanInc) done = true;
        }
        j -= kLookWin;
      }
      if (failed) raise_error(status, GSB_DEVERR_LOOKBACK_TIMEOUT, kSiteScanLookback);
      st_volatile_u64(&lookback[part], kScanInc | ((excl + block_total) & kScanMask));
    }
    s_exclusive = excl;
  }
  // The gathered records are written while thread 0 waits on its predecessors.
#pragma unroll
  for (int i = 0; i < kScanItems; ++i) {
    const int64_t r = r0 + i;
    if (r < m.BG) {
      const int b = fast_div((int)r, m.div_G);
      rec[3 * r + 0] = make_float4(mu[i].x, mu[i].y, ca[i], cb[i]);
      rec[3 * r + 1] = make_float4(cc[i], op[i], cr[i], cg[i]);
      rec[3 * r + 2] = make_float4(cbl[i], __uint_as_float(dk[i]), vis_log_threshold(op[i], m.alpha_thr, m.max_alpha),
                                   sat_log_threshold(op[i], m.max_alpha));
      perm[r] = (int32_t)(orig[i] - (uint32_t)b * (uint32_t)m.G);
      if (masks_out) masks_out[r] = masks_in[orig[i]];
    }
  }
  __syncthreads();
  unsigned long long run = s_exclusive + thread_excl;
#pragma unroll
  for (int i = 0; i < kScanItems; ++i) {
    const int64_t r = r0 + i;
    if (r < m.BG) {
      pair_offsets[r] = (int32_t)run;
      run += c[i];
      if (r == (int64_t)m.BG - 1) {
        if (run > 0x7fffffffull) {
          raise_error(status, GSB_DEVERR_PAIR_OVERFLOW, kSiteScanTotal);
          pair_offsets[m.BG] = 0;
          status[GSB_STATUS_TOTAL_PAIRS] = 0;
        } else {
          pair_offsets[m.BG] = (int32_t)run;
          status[GSB_STATUS_TOTAL_PAIRS] = (uint32_t)run;
        }
      }
    }
  }
}

// Re-runs the tile test per splat in depth-rank order (warp-cooperatively, as
// k_prepare) and writes its pairs at its scan slot, in row-major tile order:
// key = global tile index (32 bits), value = rank index. The stable sort on
// the tile key then leaves each tile's list in rank (= depth) order.
// Per-warp shared state of warp_emit_bits (the owners' constants) and of k_emit.
struct BitsEmitSmem {
  int incl[32];  // inclusive scan of the owners' half-word counts
  int done[32];  // pairs written per owner so far
  int bo[32], w[32], tx0[32], ty0[32], start[32], cnt[32];
  float rw[32];
  uint32_t mlo[32], mhi[32];  // an owner's 64-bit hit mask (bo == kMaskWords) as two words
  uint32_t tbase[32];
};
// One round's staged pairs (in slot order) and, per half-word of the round,
// its owner, first staged pair and that pair's slot.
constexpr int kEmitStage = 512;  // 32 half-words x 16 candidates
struct EmitStage {
  uint32_t key[kEmitStage];
  unsigned char lane[kEmitStage];
  int owner[32], q0[32], slot0[32];
};
struct EmitSmem {
  BitsEmitSmem bits;
  union {  // the bit writer, then warp_tiles for the splats without bits
    EmitStage stage;
    WarpTilesSmem tiles;
  } u;
};

// Writes the pairs of the warp's splats that kept hit bits: bo >= 0 for a
// larger splat's words in the hit-bit region, bo == kMaskWords for a small
// splat whose 64-bit hit mask (`mask`) stands for its words. The 32 splats of
// a warp own one contiguous range of pair slots, so all their pairs leave as
// consecutive stores. The bits are taken as half-words of 16 candidates, 32 per
// round (round r covers half-words 32r .. 32r+31 of the warp's concatenated
// lists). Lane L expands half-word L: it walks the set bits in order, steps the
// tile row and column from the previous bit, and stages each pair's key at its
// place among the round's pairs (the popcount prefix over the lanes). The warp
// then writes the staged pairs with consecutive lanes on consecutive slots.
// Each splat's pairs keep row-major candidate order. Returns the number of
// pairs of this lane's splat (sm.start, sm.cnt and sm.tbase are set by the
// caller).
constexpr int kMaskWords = -2;
__device__ __forceinline__ int warp_emit_bits(int bo, unsigned long long mask, const SplatTiles& t, int r0,
                                              const uint32_t* __restrict__ words, const Meta& m,
                                              uint32_t* __restrict__ keys, uint32_t* __restrict__ vals,
                                              BitsEmitSmem& sm, EmitStage& st) {
  const int lane = threadIdx.x & 31;
  const int nh = (bo >= 0 || bo == kMaskWords) ? (t.n + 15) >> 4 : 0;
  int incl = nh;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int y = __shfl_up_sync(kFullMask, incl, o);
    if (lane >= o) incl += y;
  }
  const int total = __shfl_sync(kFullMask, incl, 31);
  if (total == 0) return 0;
  sm.incl[lane] = incl;
  sm.done[lane] = 0;
  sm.bo[lane] = bo;
  sm.w[lane] = t.w;
  sm.rw[lane] = t.rw;
  sm.tx0[lane] = t.tx0;
  sm.ty0[lane] = t.ty0;
  sm.mlo[lane] = (uint32_t)mask;
  sm.mhi[lane] = (uint32_t)(mask >> 32);
  __syncwarp();
  for (int base = 0; base < total; base += 32) {
    const int k = base + lane;
    int owner = 32, hw = 0;  // 32: no half-word (past the end)
    uint32_t bits = 0u;
    if (k < total) {
      owner = find_owner(sm.incl, k);
      hw = k - (owner ? sm.incl[owner - 1] : 0);
      const int ob = sm.bo[owner];
      const uint32_t word = ob >= 0 ? words[ob + (hw >> 1)] : ((hw >> 1) == 0 ? sm.mlo[owner] : sm.mhi[owner]);
      bits = (hw & 1) ? (word >> 16) : (word & 0xffffu);
    }
    const int pc = __popc(bits);
    int pre = pc;  // inclusive prefix of the popcounts over the warp
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int y = __shfl_up_sync(kFullMask, pre, o);
      if (lane >= o) pre += y;
    }
    const int prev = __shfl_up_sync(kFullMask, owner, 1);
    const int next = __shfl_down_sync(kFullMask, owner, 1);
    const unsigned heads = __ballot_sync(kFullMask, lane == 0 || owner != prev);
    const unsigned le = (lane == 31) ? 0xffffffffu : ((2u << lane) - 1u);
    const int seg0 = 31 - __clz(heads & le);
    const int before_seg = __shfl_sync(kFullMask, pre, seg0 > 0 ? seg0 - 1 : 0);
    const int seg_base = seg0 > 0 ? before_seg : 0;  // popcounts of earlier segments in this round
    const int done = owner < 32 ? sm.done[owner] : 0;
    const int q0 = pre - pc;
    st.owner[lane] = owner;
    st.q0[lane] = q0;
    st.slot0[lane] = done + (q0 - seg_base);
    __syncwarp();
    if (owner < 32 && (lane == 31 || next != owner)) sm.done[owner] = done + (pre - seg_base);
    if (bits) {
      const int w = sm.w[owner];
      const int local0 = hw * 16;
      const int row = cand_row(local0, w, sm.rw[owner]);
      int col = local0 - row * w, at = 0, q = q0;
      uint32_t key = sm.tbase[owner] + (uint32_t)((sm.ty0[owner] + row) * m.tiles_x + sm.tx0[owner]);
      while (bits) {
        const int b = __ffs(bits) - 1;
        bits &= bits - 1;
        col += b - at;
        at = b;
        while (col >= w) {
          col -= w;
          key += (uint32_t)m.tiles_x;
        }
        st.key[q] = key + (uint32_t)col;
        st.lane[q] = (unsigned char)lane;
        ++q;
      }
    }
    __syncwarp();
    const int round_pairs = __shfl_sync(kFullMask, pre, 31);
    for (int q = lane; q < round_pairs; q += 32) {
      const int l = st.lane[q];
      const int o = st.owner[l];
      const int slot = st.slot0[l] + (q - st.q0[l]);
      if (slot < sm.cnt[o]) {
        const int64_t idx = (int64_t)sm.start[o] + slot;
        keys[idx] = st.key[q];
        vals[idx] = (uint32_t)(r0 + o);
      }
    }
    __syncwarp();
  }
  return sm.done[lane];
}

__global__ void __launch_bounds__(256)
    k_emit(Meta m, const float4* __restrict__ rec, const int32_t* __restrict__ pair_offsets,
           const unsigned long long* __restrict__ masks, uint32_t* __restrict__ keys, uint32_t* __restrict__ vals,
           uint32_t* __restrict__ status, ZeroList zero, BigBits big) {
  pdl_wait();
  pdl_trigger();
  __shared__ EmitSmem s_emit[8];
  zero_words(zero);  // the tile sort's scratch
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int r = blockIdx.x * blockDim.x + threadIdx.x;
  const bool valid = r < m.BG;
  SplatTiles t = splat_tiles(0.f, 0.f, 0.f, 0.f, 0.f, 0.f, m);
  int start = 0, cnt = 0;
  uint32_t tbase = 0;
  if (valid) {
    start = pair_offsets[r];
    cnt = pair_offsets[r + 1] - start;
    const float4 p0 = rec[3 * r + 0];
    const float4 p1 = rec[3 * r + 1];
    tbase = (uint32_t)fast_div(r, m.div_G) * (uint32_t)m.tiles_per_image;
    if (cnt > 0) t = splat_tiles(p0.x, p0.y, p0.z, p0.w, p1.x, p1.y, m);
  }
  // A splat with a recorded hit mask writes its pairs straight from it (the
  // set bits in row-major candidate order); a larger one with hit bits reads
  // them from the region; the others are tested again.
  int own_hits = -1;
  int bo = -1;  // where this splat's hit bits are: region offset, kMaskWords, or none (-1)
  unsigned long long mask = 0ull;
  if (masks && big.words && t.n > kMaskCands) {
    const unsigned long long v = masks[r];
    if (v != kNoBigMask) bo = (int)v;
  }
  if (masks && t.n > 0 && t.n <= kMaskCands) {
    mask = masks[r];
    own_hits = __popcll(mask);
    bo = kMaskWords;
  }
  EmitSmem& es = s_emit[warp];
  es.bits.start[lane] = start;
  es.bits.cnt[lane] = cnt;
  es.bits.tbase[lane] = tbase;
  const int r0 = r - lane;
  // Splats with hit bits (a mask or region words): their pairs straight from
  // the bits, written by the whole warp.
  if (masks) {
    const int bit_hits = warp_emit_bits(bo, mask, t, r0, big.words, m, keys, vals, es.bits, es.u.stage);
    if (bo >= 0) own_hits = bit_hits;
    if (bo != -1) t.n = 0;
  }
  __syncwarp();  // the stage is reused by warp_tiles
  WarpTilesSmem& sm = es.u.tiles;
  warp_tiles(
      t, m, sm,
      [&](int owner, int tx, int ty, int slot) {
        if (slot < es.bits.cnt[owner]) {
          const int64_t idx = (int64_t)es.bits.start[owner] + slot;
          keys[idx] = es.bits.tbase[owner] + (uint32_t)(ty * m.tiles_x + tx);
          vals[idx] = (uint32_t)(r0 + owner);
        }
      });
  const int hits = own_hits >= 0 ? own_hits : sm.hits[lane];
  if (valid && hits != cnt) raise_error(status, GSB_DEVERR_PAIR_OVERFLOW, kSiteEmit);
}

// tile_offsets[t] = index of the first sorted pair of tile t (= exclusive
// prefix of per-tile counts); every entry is written by exactly one thread.
// A thread takes 4 consecutive sorted pairs (one 16-byte load of keys).
// keys64 (optional) receives (tile << 32) | depth_key of each sorted pair.
__global__ void __launch_bounds__(256)
    k_ranges(const uint32_t* __restrict__ keys, const uint32_t* __restrict__ vals, const float4* __restrict__ rec,
             int64_t n_pairs, int total_tiles, int32_t* __restrict__ tile_offsets, uint64_t* __restrict__ keys64) {
  pdl_wait();
  pdl_trigger();
  const int64_t i0 = 4 * ((int64_t)blockIdx.x * blockDim.x + threadIdx.x);
  if (i0 >= n_pairs) return;
  uint32_t k[4];
  if (i0 + 4 <= n_pairs) {
    const uint4 q = *reinterpret_cast<const uint4*>(keys + i0);  // keys is 256-byte aligned
    k[0] = q.x, k[1] = q.y, k[2] = q.z, k[3] = q.w;
  } else {
#pragma unroll
    for (int u = 0; u < 4; ++u) k[u] = (i0 + u < n_pairs) ? keys[i0 + u] : 0u;
  }
  int64_t prev = (i0 == 0) ? -1 : (int64_t)keys[i0 - 1];
#pragma unroll
  for (int u = 0; u < 4; ++u) {
    const int64_t i = i0 + u;
    if (i < n_pairs) {
      const int64_t t = k[u];
      for (int64_t s = prev + 1; s <= t; ++s) tile_offsets[s] = (int32_t)i;
      if (i == n_pairs - 1)
        for (int64_t s = t + 1; s <= total_tiles; ++s) tile_offsets[s] = (int32_t)n_pairs;
      if (keys64) keys64[i] = ((uint64_t)t << 32) | __float_as_uint(rec[3 * (size_t)vals[i] + 2].y);
      prev = t;
    }
  }
}

// Tile offsets from the last sort pass's key ranges (SortRanges), in place:
// off[t] (t < tiles) holds n - (tile t's first pair position), 0 for an empty
// tile, and block[k] the same for the first pair of 256-tile block k. An empty
// tile starts where the next non-empty tile does (or at n), so off[t] is the
// minimum start over tiles s >= t, and off[tiles] = n. One CTA per block: the
// start after its block comes from the block entries to its right (the
// largest n - position there), the rest from a block-wide suffix minimum.
__global__ void __launch_bounds__(kRangesBlock)
    k_ranges_fix(int32_t* __restrict__ off, const int32_t* __restrict__ block, int tiles, int32_t n) {
  pdl_wait();
  pdl_trigger();
  __shared__ int32_t s_red[kRangesBlock / 32];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int blocks = (tiles + kRangesBlock - 1) / kRangesBlock;
  // The first pair after this block: the largest block entry to the right.
  int32_t far = 0;
  for (int k = blockIdx.x + 1 + tid; k < blocks; k += kRangesBlock) far = max(far, block[k]);
  far = __reduce_max_sync(kFullMask, far);
  if (lane == 0) s_red[warp] = far;
  __syncthreads();
  int32_t right_v = 0;
#pragma unroll
  for (int w = 0; w < kRangesBlock / 32; ++w) right_v = max(right_v, s_red[w]);
  const int32_t right = right_v > 0 ? n - right_v : n;
  __syncthreads();  // s_red is reused
  const int t = blockIdx.x * kRangesBlock + tid;
  int32_t x = n;
  if (t < tiles) {
    const int32_t v = off[t];
    x = v > 0 ? n - v : n;
  }
  // Inclusive suffix minimum within the warp, then over the warps to the right.
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int32_t y = __shfl_down_sync(kFullMask, x, o);
    if (lane + o < 32) x = min(x, y);
  }
  if (lane == 0) s_red[warp] = x;
  __syncthreads();
  for (int w = warp + 1; w < kRangesBlock / 32; ++w) x = min(x, s_red[w]);
  if (t < tiles) off[t] = min(x, right);
  if (t == tiles - 1) off[tiles] = n;
}

__global__ void k_fill_i32(int32_t* __restrict__ p, int64_t n, int32_t v) {
  pdl_wait();
  pdl_trigger();
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) p[i] = v;
}

__global__ void __launch_bounds__(256)
    k_tile_max(const int32_t* __restrict__ tile_offsets, int total_tiles, uint32_t* __restrict__ status) {
  pdl_wait();
  pdl_trigger();
  const int t = blockIdx.x * blockDim.x + threadIdx.x;
  uint32_t c = 0;
  if (t < total_tiles) c = (uint32_t)(tile_offsets[t + 1] - tile_offsets[t]);
  c = __reduce_max_sync(kFullMask, c);
  if ((threadIdx.x & 31) == 0 && c) atomicMax(&status[GSB_STATUS_MAX_TILE_COUNT], c);
}

// Workspace carve of gsb_bin_prepare (shared by size query and run).
struct PrepareWs {
  uint64_t* keys_in;  // 64-bit keys (B > 1), or 32-bit keys in the same space (B == 1)
  uint32_t* vals_in;
  uint64_t* keys_sorted;
  uint32_t* vals_sorted;
  uint32_t* counts;
  unsigned long long* masks;  // hit masks of splats with <= kMaskCands candidates, input order
  unsigned long long* lookback;
  uint32_t* counter;
  uint32_t* depth_hist;  // digit counts of the depth keys (k_prepare -> depth sort)
};

void carve_prepare(Carver& c, const Meta& m, PrepareWs* w) {
  const size_t n = (size_t)m.BG;
  w->keys_in = c.take<uint64_t>(n);
  w->vals_in = c.take<uint32_t>(n);
  w->keys_sorted = c.take<uint64_t>(n);
  w->vals_sorted = c.take<uint32_t>(n);
  w->counts = c.take<uint32_t>(n);
  w->masks = c.take<unsigned long long>(n);
  w->lookback = c.take<unsigned long long>((n + kScanTile - 1) / kScanTile + 1);
  w->counter = c.take<uint32_t>(1);
  w->depth_hist = c.take<uint32_t>((size_t)kDepthHistPasses * kRadix);
}

int depth_sort_end_bit(const Meta& m) { return 32 + (m.B > 1 ? bits_for(m.B - 1) : 0); }
bool depth_keys32(const Meta& m) { return m.B == 1; }
int depth_passes(const Meta& m) { return sort_passes(0, depth_keys32(m) ? 32 : depth_sort_end_bit(m)); }

}  // namespace
}  // namespace gsb

using namespace gsb;

extern "C" size_t gsb_bin_prepare_workspace_size(const gsb_raster_meta* meta) {
  Meta m;
  if (make_meta(meta, &m) != GSB_OK) return 0;
  Carver c(nullptr);
  PrepareWs w;
  carve_prepare(c, m, &w);
  radix_sort_pairs(c, (const uint64_t*)nullptr, nullptr, nullptr, nullptr, m.BG, 0, depth_sort_end_bit(m), nullptr,
                   0, false);
  return c.off + 256;
}

namespace {
// Words of the hit-bit region that follows the B*G slots of tile_masks.
uint32_t big_mask_capacity(const Meta& m) {
  return (uint32_t)std::min<uint64_t>((uint64_t)m.BG * kBigMaskWords, 0x7fffffffull);
}
BigBits big_bits_of(const Meta& m, uint64_t* tile_masks, uint32_t* status) {
  BigBits b;
  if (tile_masks && m.BG > 0) {
    b.words = reinterpret_cast<uint32_t*>(tile_masks + m.BG);
    b.capacity = big_mask_capacity(m);
    b.cursor = status + GSB_STATUS_MASK_WORDS;
  }
  return b;
}
}  // namespace

extern "C" size_t gsb_bin_tile_masks_size(const gsb_raster_meta* meta) {
  Meta m;
  if (make_meta(meta, &m) != GSB_OK) return 0;
  return (size_t)m.BG * sizeof(uint64_t) + (size_t)big_mask_capacity(m) * sizeof(uint32_t);
}

extern "C" int gsb_bin_count(const gsb_raster_meta* meta, const float* means2d, const float* conics,
                             const float* opacities, const float* depths, uint64_t* tile_masks, uint32_t* status,
                             void* workspace, size_t workspace_bytes, void* stream_) {
  Meta m;
  int rc = make_meta(meta, &m);
  if (rc != GSB_OK) return rc;
  if (!status) return GSB_ERR_INVALID_ARGUMENT;
  if (m.BG > 0 && (!means2d || !conics || !opacities || !depths)) return GSB_ERR_INVALID_ARGUMENT;
  if (m.BG >= kSortMaxN) return GSB_ERR_CAPACITY;
  if (workspace_bytes < gsb_bin_prepare_workspace_size(meta) || (m.BG > 0 && !workspace))
    return GSB_ERR_WORKSPACE;
  cudaStream_t stream = static_cast<cudaStream_t>(stream_);
  if (m.BG == 0) return cuda_status(cudaMemsetAsync(status, 0, sizeof(uint32_t) * GSB_STATUS_WORDS, stream));
  Carver c(workspace);
  PrepareWs w;
  carve_prepare(c, m, &w);
  // The status block and the depth keys' digit counts start at zero.
  const int dpasses = depth_passes(m);
  launch_pdl(k_clear_words, grid1d(std::max(GSB_STATUS_WORDS, dpasses * kRadix), 256), 256, 0, stream, status,
             GSB_STATUS_WORDS, w.depth_hist, dpasses * kRadix);
  note_launches(1);
  const int parts = (m.BG + kScanTile - 1) / kScanTile;
  const ZeroRegion sz = radix_sort_zero_region(c, m.BG, 0, depth_keys32(m) ? 32 : depth_sort_end_bit(m),
                                               depth_keys32(m));
  ZeroList zero;
  zero.ptr[0] = reinterpret_cast<uint32_t*>(w.lookback);
  zero.words[0] = 2 * (size_t)(parts + 1);
  zero.ptr[1] = w.counter;
  zero.words[1] = 1;
  zero.ptr[2] = sz.ptr;
  zero.words[2] = sz.words;
  if (depth_keys32(m))
    launch_pdl(k_prepare<uint32_t>, grid1d(m.BG, 256), 256, 0, stream, m, reinterpret_cast<const float2*>(means2d),
               conics, opacities, depths, reinterpret_cast<uint32_t*>(w.keys_in), w.vals_in, w.counts, w.masks,
               status, zero, big_bits_of(m, tile_masks, status), w.depth_hist, dpasses);
  else
    launch_pdl(k_prepare<uint64_t>, grid1d(m.BG, 256), 256, 0, stream, m, reinterpret_cast<const float2*>(means2d),
               conics, opacities, depths, w.keys_in, w.vals_in, w.counts, w.masks, status, zero,
               big_bits_of(m, tile_masks, status), w.depth_hist, dpasses);
  note_launches(1);
  return cuda_status(cudaGetLastError());
}

namespace {
// k_scan_part_sums + k_scan_part_prefix into the look-back array (its words
// were cleared by k_prepare; both kernels overwrite what they use).
void launch_scan_prefix(const Meta& m, const PrepareWs& w, int parts, cudaStream_t stream) {
  launch_pdl(k_scan_part_sums, parts, kScanThreads, 0, stream, m.BG, (const uint32_t*)w.vals_sorted,
             (const uint32_t*)w.counts, w.lookback);
  launch_pdl(k_scan_part_prefix, 1, kScanPrefixThreads, 0, stream, w.lookback, parts);
  note_launches(2);
}
}  // namespace

extern "C" int gsb_bin_sort_scan(const gsb_raster_meta* meta, const float* means2d, const float* conics,
                                 const float* colors, const float* opacities, const float* depths, int32_t* perm,
                                 float* rec, int32_t* pair_offsets, uint64_t* tile_masks, uint32_t* status,
                                 void* workspace, size_t workspace_bytes, void* stream_) {
  Meta m;
  int rc = make_meta(meta, &m);
  if (rc != GSB_OK) return rc;
  if (!status || !pair_offsets) return GSB_ERR_INVALID_ARGUMENT;
  if (m.BG > 0 && (!means2d || !conics || !colors || !opacities || !depths || !perm || !rec))
    return GSB_ERR_INVALID_ARGUMENT;
  if (m.BG >= kSortMaxN) return GSB_ERR_CAPACITY;
  if (workspace_bytes < gsb_bin_prepare_workspace_size(meta) || (m.BG > 0 && !workspace))
    return GSB_ERR_WORKSPACE;
  cudaStream_t stream = static_cast<cudaStream_t>(stream_);
  if (m.BG == 0) return cuda_status(cudaMemsetAsync(pair_offsets, 0, sizeof(int32_t), stream));
  Carver c(workspace);
  PrepareWs w;
  carve_prepare(c, m, &w);
  // k_prepare (gsb_bin_count) cleared the scan's look-back words and counter
  // and the depth sort's scratch.
  const int parts = (m.BG + kScanTile - 1) / kScanTile;
  // Many splats: the pair-offset prefixes come from a reduce-then-scan
  // (k_scan_part_sums, k_scan_part_prefix) instead of the scan's look-back.
  const bool scan_prefix = m.BG >= kScanPrefixMinSplats && parts <= kScanPrefixMaxParts;
  cudaError_t e;
  if (depth_keys32(m)) {
    uint32_t* k32_in = reinterpret_cast<uint32_t*>(w.keys_in);
    uint32_t* k32_sorted = reinterpret_cast<uint32_t*>(w.keys_sorted);
    // 32-bit keys in the 64-bit key buffers; the sort's scratch (carved after
    // them) is smaller than the 64-bit sort's that the workspace is sized for.
    e = radix_sort_pairs(c, k32_in, w.vals_in, k32_sorted, w.vals_sorted, m.BG, 0, 32, status, stream, true,
                         w.depth_hist);
    if (e != cudaSuccess) return GSB_ERR_CUDA;
    if (scan_prefix) launch_scan_prefix(m, w, parts, stream);
    launch_pdl(scan_prefix ? k_gather_scan<uint32_t, true> : k_gather_scan<uint32_t>, parts, kScanThreads, 0, stream,
        m, k32_sorted, w.vals_sorted, reinterpret_cast<const float2*>(means2d), conics, colors, opacities, w.counts,
        w.masks, reinterpret_cast<unsigned long long*>(tile_masks), reinterpret_cast<float4*>(rec), perm,
        pair_offsets, w.lookback, w.counter, status);
  } else {
    e = radix_sort_pairs(c, w.keys_in, w.vals_in, w.keys_sorted, w.vals_sorted, m.BG, 0, depth_sort_end_bit(m),
                         status, stream, true, w.depth_hist);
    if (e != cudaSuccess) return GSB_ERR_CUDA;
    if (scan_prefix) launch_scan_prefix(m, w, parts, stream);
    launch_pdl(scan_prefix ? k_gather_scan<uint64_t, true> : k_gather_scan<uint64_t>, parts, kScanThreads, 0, stream,
        m, w.keys_sorted, w.vals_sorted, reinterpret_cast<const float2*>(means2d), conics, colors, opacities,
        w.counts, w.masks, reinterpret_cast<unsigned long long*>(tile_masks), reinterpret_cast<float4*>(rec), perm,
        pair_offsets, w.lookback, w.counter, status);
  }
  note_launches(1);
  return cuda_status(cudaGetLastError());
}

extern "C" int gsb_bin_prepare(const gsb_raster_meta* meta, const float* means2d, const float* conics,
                               const float* colors, const float* opacities, const float* depths, int32_t* perm,
                               float* rec, int32_t* pair_offsets, uint32_t* status, void* workspace,
                               size_t workspace_bytes, void* stream) {
  int rc = gsb_bin_count(meta, means2d, conics, opacities, depths, /*tile_masks=*/nullptr, status, workspace,
                         workspace_bytes, stream);
  if (rc != GSB_OK) return rc;
  return gsb_bin_sort_scan(meta, means2d, conics, colors, opacities, depths, perm, rec, pair_offsets,
                           /*tile_masks=*/nullptr, status, workspace, workspace_bytes, stream);
}

namespace {
struct EmitWs {
  uint32_t* keys;         // emitted tile keys, rank order
  uint32_t* vals;
  uint32_t* keys_sorted;  // tile keys after the sort
  int32_t* block_first;   // per 256-tile block: n - its first pair position (SortRanges.block)
};
void carve_emit(Carver& c, const Meta& m, int64_t P, EmitWs* w) {
  w->keys = c.take<uint32_t>((size_t)P);
  w->vals = c.take<uint32_t>((size_t)P);
  w->keys_sorted = c.take<uint32_t>((size_t)P);
  w->block_first = c.take<int32_t>(((size_t)m.total_tiles + kRangesBlock - 1) / kRangesBlock);
}
int tile_end_bit(const Meta& m) { return m.total_tiles > 1 ? bits_for(m.total_tiles - 1) : 0; }
}  // namespace

extern "C" size_t gsb_bin_emit_workspace_size(const gsb_raster_meta* meta, int64_t total_pairs) {
  Meta m;
  if (make_meta(meta, &m) != GSB_OK || total_pairs < 0) return 0;
  Carver c(nullptr);
  EmitWs w;
  carve_emit(c, m, total_pairs, &w);
  radix_sort_pairs(c, (const uint32_t*)nullptr, nullptr, nullptr, nullptr, total_pairs, 0, tile_end_bit(m), nullptr,
                   0, false);
  return c.off + 256;
}

namespace {
// gsb_bin_emit (fold_request false) and gsb_bin_emit_ranges (true, keys NULL).
int bin_emit(const gsb_raster_meta* meta, const float* rec, const int32_t* pair_offsets, const uint64_t* tile_masks,
             int64_t total_pairs, uint64_t* keys, int32_t* binned_ids, int32_t* tile_offsets, uint32_t* status,
             void* workspace, size_t workspace_bytes, void* stream_, bool fold_request) {
  Meta m;
  int rc = make_meta(meta, &m);
  if (rc != GSB_OK) return rc;
  if (total_pairs < 0 || !tile_offsets || !status) return GSB_ERR_INVALID_ARGUMENT;
  if (total_pairs >= kSortMaxN) return GSB_ERR_CAPACITY;
  if (total_pairs > 0 && (!rec || !pair_offsets || !binned_ids)) return GSB_ERR_INVALID_ARGUMENT;
  if (workspace_bytes < gsb_bin_emit_workspace_size(meta, total_pairs) || (total_pairs > 0 && !workspace))
    return GSB_ERR_WORKSPACE;
  cudaStream_t stream = static_cast<cudaStream_t>(stream_);
  const int64_t T1 = (int64_t)m.total_tiles + 1;
  if (total_pairs == 0) {
    launch_pdl(k_fill_i32, grid1d(T1, 256), 256, 0, stream, tile_offsets, T1, 0);
    note_launches(1);
    return cuda_status(cudaGetLastError());
  }
  Carver c(workspace);
  EmitWs w;
  carve_emit(c, m, total_pairs, &w);
  const ZeroRegion sz = radix_sort_zero_region(c, total_pairs, 0, tile_end_bit(m), true);
  // Folded ranges: the last tile-sort pass records each tile's first position
  // and k_ranges_fix turns them into offsets, so the sorted tile keys are
  // neither written nor read back (one tile: no pass, k_ranges instead).
  const bool fold_ranges = fold_request && sort_passes(0, tile_end_bit(m)) > 0;
  ZeroList zero;
  zero.ptr[0] = sz.ptr;
  zero.words[0] = sz.words;
  zero.ptr[1] = fold_ranges ? reinterpret_cast<uint32_t*>(tile_offsets) : nullptr;
  zero.words[1] = fold_ranges ? (size_t)T1 : 0;
  const size_t nblocks = ((size_t)m.total_tiles + kRangesBlock - 1) / kRangesBlock;
  zero.ptr[2] = fold_ranges ? reinterpret_cast<uint32_t*>(w.block_first) : nullptr;
  zero.words[2] = fold_ranges ? nblocks : 0;
  launch_pdl(k_emit, grid1d(m.BG, 256), 256, 0, stream, m, reinterpret_cast<const float4*>(rec), pair_offsets,
             reinterpret_cast<const unsigned long long*>(tile_masks), w.keys, w.vals, status, zero,
             big_bits_of(m, const_cast<uint64_t*>(tile_masks), status));
  note_launches(1);
  SortRanges ranges;
  if (fold_ranges) {
    ranges.first = tile_offsets;
    ranges.block = w.block_first;
    ranges.n = m.total_tiles;
  }
  cudaError_t e = radix_sort_pairs(c, w.keys, w.vals, w.keys_sorted, reinterpret_cast<uint32_t*>(binned_ids),
                                   total_pairs, 0, tile_end_bit(m), status, stream, /*scratch_zeroed=*/true,
                                   nullptr, ranges);
  if (e != cudaSuccess) return GSB_ERR_CUDA;
  if (fold_ranges) {
    launch_pdl(k_ranges_fix, (unsigned)nblocks, kRangesBlock, 0, stream, tile_offsets, (const int32_t*)w.block_first,
               m.total_tiles, (int32_t)total_pairs);
    note_launches(1);
    return cuda_status(cudaGetLastError());
  }
  launch_pdl(k_ranges, grid1d((total_pairs + 3) / 4, 256), 256, 0, stream, w.keys_sorted, reinterpret_cast<const uint32_t*>(binned_ids),
                                                         reinterpret_cast<const float4*>(rec), total_pairs,
                                                         m.total_tiles, tile_offsets, keys);
  note_launches(1);
  return cuda_status(cudaGetLastError());
}
}  // namespace

extern "C" int gsb_bin_emit(const gsb_raster_meta* meta, const float* rec, const int32_t* pair_offsets,
                            const uint64_t* tile_masks, int64_t total_pairs, uint64_t* keys, int32_t* binned_ids,
                            int32_t* tile_offsets, uint32_t* status, void* workspace,
                            size_t workspace_bytes, void* stream_) {
  return bin_emit(meta, rec, pair_offsets, tile_masks, total_pairs, keys, binned_ids, tile_offsets, status,
                  workspace, workspace_bytes, stream_, false);
}

extern "C" int gsb_bin_emit_ranges(const gsb_raster_meta* meta, const float* rec, const int32_t* pair_offsets,
                                   const uint64_t* tile_masks, int64_t total_pairs, int32_t* binned_ids,
                                   int32_t* tile_offsets, uint32_t* status, void* workspace,
                                   size_t workspace_bytes, void* stream_) {
  return bin_emit(meta, rec, pair_offsets, tile_masks, total_pairs, nullptr, binned_ids, tile_offsets, status,
                  workspace, workspace_bytes, stream_, true);
}

extern "C" int gsb_tile_stats(const gsb_raster_meta* meta, const int32_t* tile_offsets, uint32_t* status,
                              void* stream_) {
  Meta m;
  int rc = make_meta(meta, &m);
  if (rc != GSB_OK) return rc;
  if (!tile_offsets || !status) return GSB_ERR_INVALID_ARGUMENT;
  cudaStream_t stream = static_cast<cudaStream_t>(stream_);
  cudaError_t e = cudaMemsetAsync(&status[GSB_STATUS_MAX_TILE_COUNT], 0, sizeof(uint32_t), stream);
  if (e != cudaSuccess) return GSB_ERR_CUDA;
  launch_pdl(k_tile_max, grid1d(m.total_tiles, 256), 256, 0, stream, tile_offsets, m.total_tiles, status);
  note_launches(1);
  return cuda_status(cudaGetLastError());
}
