// Front-to-back compositing (forward) and its reverse-order VJP (backward) on
// 16x16 tiles.
//
// Reference math: variants/v8_project3d/csrc/metal/gsplat_v8_project3d_kernels.metal
//   eval_alpha 574-592, tile_fast_forward_state 853-929, tile_fast_backward_saved 931-1063.
// Forward contract (docs/v8_critical_theory_notes.md:60-80): a pixel consumes its
// tile list in depth order while T > T_thr; a splat is visible when power <= 0
// and alpha = min(max_alpha, op*exp(power)) >= alpha_thr; C += T*alpha*c;
// T *= 1-alpha; the pixel stops once T <= T_thr. The visibility and saturation
// gates are decided on `power` against per-splat log thresholds stored in the
// record (vis_log_threshold / sat_log_threshold), with `power` evaluated by a
// fixed sequence of correctly rounded ops (power_at), so the CPU oracle makes
// the same decisions bit for bit.
//
// The forward saves per pixel the final transmittance and last_idx = the number
// of list entries the pixel consumed (the saturation index + 1, or the tile's
// count when it never saturates: the reference's per-pixel stop), so the
// backward starts from the exact per-pixel state without recompositing.
//
// Work split. Most tiles carry short lists (c3: 6 pairs on average), where a
// CTA per tile is dominated by barriers and per-splat overheads. Tiles with at
// most kShortMax pairs are processed by ONE WARP each (8 pixels per lane, the
// column terms of the exponent shared by the lane's 8 rows, backward gradients
// summed over the lane's pixels before a single warp reduction). Longer lists
// go to a CTA per tile (128 threads, two packed pixels each), which finds its
// tiles itself by scanning tile_offsets. The warp kernels are persistent; the
// CTA kernels run a slice of tiles per resident CTA, or one CTA per tile in
// dense scenes (long_tile_grid).
//
// The training forward also copies each short tile's records, in list order,
// into pair_rec [P,12] (a by-product of its gather). The backward warp kernel
// then prefetches a tile's per-pixel state, and for tiles of at most kBwdHalf
// records also its records and ids, with cp.async one tile ahead, so its
// per-tile load latency overlaps the previous tile's arithmetic.
#include <mutex>

#include "gsb_common.cuh"
#include "gsb_host.cuh"

namespace gsb {
namespace {

constexpr int kShortMax = 96;   // pairs per tile handled by one warp (forward)
// The backward warp kernel takes the same tiles (it reads the records the
// forward warp kernel copied to pair_rec). Its record buffer holds
// kBwdShortMax records as two halves: tiles of at most kBwdHalf records are
// prefetched one tile ahead into alternate halves; a longer one uses both.
constexpr int kBwdShortMax = 96;
constexpr int kBwdHalf = kBwdShortMax / 2;
static_assert(kBwdShortMax <= kShortMax, "the backward warp kernel reads pair_rec of forward warp-kernel tiles");
constexpr int kWarpBatch = 32;  // records staged per warp round (forward)
constexpr int kLanePx = 8;      // pixels per lane in the warp kernels: rows py0 + 2i
constexpr int kWarps = 8;       // warps per CTA (forward warp kernel, CTA kernels)
constexpr int kBwdWarps = 4;    // warps per CTA (backward warp kernel)
constexpr int kBatch = 256;     // records staged per CTA round (long kernels)
constexpr int kCtaThreads = 128;  // threads per long tile in the CTA kernels (2 pixels each)
constexpr int kDenseSplatsPerTile = 4;  // B*G / tiles from which the CTA kernels get one CTA per tile
constexpr int kGradComps = 9;

struct TileCoord {
  int b, tx, ty;
};

__device__ __forceinline__ TileCoord tile_coord(const Meta& m, int tile) {
  TileCoord c;
  c.b = fast_div(tile, m.div_tiles_per_image);
  const int local = tile - c.b * m.tiles_per_image;
  c.ty = fast_div(local, m.div_tiles_x);
  c.tx = local - c.ty * m.tiles_x;
  return c;
}

__device__ __forceinline__ int load_gi(const int32_t* __restrict__ ids, int k, int BG, uint32_t* status,
                                       uint32_t site) {
  int gi = __ldg(&ids[k]);
  if ((unsigned)gi >= (unsigned)BG) {
    raise_error(status, GSB_DEVERR_BOUNDS, site);
    gi = -1;
  }
  return gi;
}

// A record that is never visible (used for out-of-range ids).
__device__ __forceinline__ void invisible_rec(float4* r) {
  const float inf = __int_as_float(0x7f800000);
  r[0] = make_float4(0.f, 0.f, 0.f, 0.f);
  r[1] = make_float4(0.f, 0.f, 0.f, 0.f);
  r[2] = make_float4(0.f, 0.f, inf, inf);
}

__device__ __forceinline__ void load_rec(const float4* __restrict__ rec, int gi, float4* dst) {
  if (gi >= 0) {
    dst[0] = __ldg(&rec[3 * gi + 0]);
    dst[1] = __ldg(&rec[3 * gi + 1]);
    dst[2] = __ldg(&rec[3 * gi + 2]);
  } else {
    invisible_rec(dst);
  }
}

// Warp-wide sum of v[0..15]; on return lane L holds the total of v[L >> 1]
// (recursive halving: 16 shuffles instead of 5 per value).
__device__ __forceinline__ float warp_reduce_scatter16(float (&v)[16], int lane) {
#pragma unroll
  for (int half = 8, bit = 16; half >= 1; half >>= 1, bit >>= 1) {
    const bool up = lane & bit;
#pragma unroll
    for (int i = 0; i < half; ++i) {
      const float send = up ? v[i] : v[i + half];
      const float keep = up ? v[i + half] : v[i];
      v[i] = keep + __shfl_xor_sync(kFullMask, send, bit);
    }
  }
  return v[0] + __shfl_xor_sync(kFullMask, v[0], 1);
}

// Dynamic tile assignment of the backward warp kernel: a warp takes its next
// tile from a counter in the status block (lane 0's atomic, broadcast), so a
// warp that met longer lists takes fewer tiles and the kernel's tail shrinks.
// It pays when a warp sees many tiles (c3: 28); with a few per warp (1080p
// frames: 3.5) the claims made three tiles ahead fix most of the assignment
// anyway, and the static grid stride measured faster, so the host chooses
// (kMinTilesPerWarpForClaims). The counter is 0 when the warp kernel starts:
// gsb_bin_count clears the status block, and the long-tile CTA kernel that
// follows every backward warp kernel resets it once the warp kernel has
// completed (it starts with griddepcontrol.wait).
constexpr int kMinTilesPerWarpForClaims = 8;
__device__ __forceinline__ int claim_tiles(uint32_t* counter, int count, int lane) {
  int t = 0;
  if (lane == 0) t = (int)atomicAdd(counter, (unsigned)count);
  return __shfl_sync(kFullMask, t, 0);
}

// ---------------------------------------------------------------------------
// Forward
// ---------------------------------------------------------------------------
// A lane's 8 pixels are 4 packed pairs: pair q holds rows py0 + 4q and
// py0 + 4q + 2 of the lane's column. The loop over a tile's records is free of
// per-pixel branches: an invisible or finished pixel gets alpha = 0, which
// leaves its colour and transmittance bit-for-bit unchanged (w = T*0 = 0,
// T*(1-0) = T), so the 8 pixels' chains interleave. The results equal those of
// a per-pixel `if (visible)` loop exactly, for finite colours; kGuard (a batch
// holding a non-finite colour) adds w*c only where the splat is visible.
template <bool kGuard, bool kSat>
__device__ __forceinline__ void fwd_warp_batch(const Meta& m, const float4 (*recs)[3], int cnt, int base, float fx,
                                               const F2 (&fy)[kLanePx / 2], F2 (&T)[kLanePx / 2],
                                               F2 (&cr)[kLanePx / 2], F2 (&cg)[kLanePx / 2], F2 (&cb)[kLanePx / 2],
                                               int (&last)[kLanePx]) {
  const F2 one = f2(1.0f), log2e = f2(kLog2e);
#pragma unroll 1
  for (int j = 0; j < cnt; ++j) {
    const float4 p0 = recs[j][0];
    const float4 p1 = recs[j][1];
    const float4 p2 = recs[j][2];
    const PowerCol pc = power_col(p0.z, p0.w, p1.x, __fsub_rn(fx, p0.x));
    const F2 ta = f2(pc.ta), tb = f2(pc.tb), ch = f2(pc.ch), mu_y = f2(p0.y);
    const F2 col_r = f2(p1.z), col_g = f2(p1.w), col_b = f2(p2.x), op = f2(p1.y);
    const int consumed = base + j + 1;
#pragma unroll
    for (int q = 0; q < kLanePx / 2; ++q) {
      const F2 power = power_at2(ta, tb, ch, sub2(fy[q], mu_y));
      float pl, ph, tl, th, xl, xh;
      split(power, pl, ph);
      split(T[q], tl, th);
      split(mul2(power, log2e), xl, xh);
      float vl_, vh_;  // op * exp(power), capped at max_alpha where a record may saturate
      if (kSat) {
        vl_ = fminf(m.max_alpha, p1.y * ex2_approx(xl));
        vh_ = fminf(m.max_alpha, p1.y * ex2_approx(xh));
      } else {
        split(mul2(op, f2(ex2_approx(xl), ex2_approx(xh))), vl_, vh_);
      }
      float al, ah;
      int vis_l = 1, vis_h = 1;
      if (kGuard) {
        al = vis_select_fwd_v(tl, m.T_thr, pl, p2.z, vl_, consumed, last[2 * q], vis_l);
        ah = vis_select_fwd_v(th, m.T_thr, ph, p2.z, vh_, consumed, last[2 * q + 1], vis_h);
      } else {
        al = vis_select_fwd(tl, m.T_thr, pl, p2.z, vl_, consumed, last[2 * q]);
        ah = vis_select_fwd(th, m.T_thr, ph, p2.z, vh_, consumed, last[2 * q + 1]);
      }
      const F2 alpha = f2(al, ah);
      const F2 w = mul2(T[q], alpha);
      if (kGuard) {
        cr[q] = select2(vis_l, vis_h, fma2(w, col_r, cr[q]), cr[q]);
        cg[q] = select2(vis_l, vis_h, fma2(w, col_g, cg[q]), cg[q]);
        cb[q] = select2(vis_l, vis_h, fma2(w, col_b, cb[q]), cb[q]);
      } else {
        cr[q] = fma2(w, col_r, cr[q]);
        cg[q] = fma2(w, col_g, cg[q]);
        cb[q] = fma2(w, col_b, cb[q]);
      }
      T[q] = mul2(T[q], sub2(one, alpha));
    }
  }
}

template <bool kSave>
__global__ void __launch_bounds__(kWarps * 32, 2)
    k_render_fwd_warp(Meta m, const float4* __restrict__ rec, const int32_t* __restrict__ toff,
                      const int32_t* __restrict__ ids, float* __restrict__ out, float* __restrict__ final_T,
                      int32_t* __restrict__ last_idx, float4* __restrict__ pair_rec,
                      uint32_t* __restrict__ status) {
  pdl_wait();
  pdl_trigger();
  __shared__ float4 s_rec[kWarps][kWarpBatch][3];
  __shared__ __align__(16) float s_out[kWarps][kTilePixels * 3];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  float4(*my)[3] = s_rec[warp];
  float* srgb = s_out[warp];
  const int stride = gridDim.x * kWarps;
  for (int tile = blockIdx.x * kWarps + warp; tile < m.total_tiles; tile += stride) {
    const int start = __ldg(&toff[tile]);
    const int n = __ldg(&toff[tile + 1]) - start;
    if (n > kShortMax) continue;  // k_render_fwd_cta finds and renders the long tiles
    const TileCoord tc = tile_coord(m, tile);
    const int px = tc.tx * kTile + (lane & 15);
    const int py0 = tc.ty * kTile + (lane >> 4);
    const float fx = (float)px + 0.5f;
    const float fy0 = (float)py0 + 0.5f;  // row i is at fy0 + 2i (exact)
    // T > T_thr marks a live pixel; pixels outside the image start dead (T = 0).
    // last[i] = entries the pixel consumed (the reference's per-pixel stop): the
    // index + 1 of the last entry it met while still live.
    F2 fy[kLanePx / 2], T[kLanePx / 2], cr[kLanePx / 2], cg[kLanePx / 2], cb[kLanePx / 2];
    int last[kLanePx];
#pragma unroll
    for (int q = 0; q < kLanePx / 2; ++q) {
      fy[q] = f2(fy0 + (float)(4 * q), fy0 + (float)(4 * q + 2));
      const bool in_lo = px < m.W && py0 + 4 * q < m.H;
      const bool in_hi = px < m.W && py0 + 4 * q + 2 < m.H;
      T[q] = f2(in_lo ? 1.0f : 0.0f, in_hi ? 1.0f : 0.0f);
      cr[q] = cg[q] = cb[q] = f2(0.0f);
      last[2 * q] = last[2 * q + 1] = 0;
    }
    for (int base = 0; base < n; base += kWarpBatch) {
      bool live = false;
#pragma unroll
      for (int q = 0; q < kLanePx / 2; ++q) {
        float tl, th;
        split(T[q], tl, th);
        live |= (tl > m.T_thr) | (th > m.T_thr);
      }
      if (!__any_sync(kFullMask, live)) break;
      const int cnt = min(kWarpBatch, n - base);
      __syncwarp();
      bool bad_color = false, sat = false;
      if (lane < cnt) {
        float4 r[3];
        load_rec(rec, load_gi(ids, start + base + lane, m.BG, status, kSiteRender), r);
        my[lane][0] = r[0];
        my[lane][1] = r[1];
        my[lane][2] = r[2];
        bad_color = !finite_rgb(r[1].z, r[1].w, r[2].x);
        sat = may_saturate(r[1].y, m.max_alpha);
        if (kSave) {
          float4* dst = pair_rec + 3 * (size_t)(start + base + lane);
          dst[0] = r[0];
          dst[1] = r[1];
          dst[2] = r[2];
        }
      }
      const bool guard = __any_sync(kFullMask, bad_color), any_sat = __any_sync(kFullMask, sat);
      __syncwarp();
      if (!live) continue;
      if (guard)
        fwd_warp_batch<true, true>(m, my, cnt, base, fx, fy, T, cr, cg, cb, last);
      else if (any_sat)
        fwd_warp_batch<false, true>(m, my, cnt, base, fx, fy, T, cr, cg, cb, last);
      else
        fwd_warp_batch<false, false>(m, my, cnt, base, fx, fy, T, cr, cg, cb, last);
    }
    const bool full = (tc.tx * kTile + kTile <= m.W) && (tc.ty * kTile + kTile <= m.H) && ((m.W & 3) == 0);
    if (full) {
      const size_t pix0 = ((size_t)tc.b * m.H + py0) * m.W + px;
#pragma unroll
      for (int q = 0; q < kLanePx / 2; ++q) {
        float tv[2], rv[2], gv[2], bv[2];
        split(T[q], tv[0], tv[1]);
        split(cr[q], rv[0], rv[1]);
        split(cg[q], gv[0], gv[1]);
        split(cb[q], bv[0], bv[1]);
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          const int idx = ((lane >> 4) + 4 * q + 2 * h) * kTile + (lane & 15);
          srgb[3 * idx + 0] = fmaf(tv[h], m.bg_r, rv[h]);
          srgb[3 * idx + 1] = fmaf(tv[h], m.bg_g, gv[h]);
          srgb[3 * idx + 2] = fmaf(tv[h], m.bg_b, bv[h]);
          if (kSave) {
            const size_t pix = pix0 + (size_t)(4 * q + 2 * h) * (size_t)m.W;
            final_T[pix] = tv[h];
            last_idx[pix] = last[2 * q + h];
          }
        }
      }
      __syncwarp();
      const size_t row0 = ((size_t)tc.b * m.H + tc.ty * kTile) * m.W + tc.tx * kTile;
#pragma unroll
      for (int i = 0; i < 6; ++i) {  // 16 rows x 12 float4 = 192 = 6 per lane
        const int qq = lane + 32 * i, r = qq / 12, k = qq - r * 12;
        const float4 v = *reinterpret_cast<const float4*>(&srgb[r * 48 + 4 * k]);
        *reinterpret_cast<float4*>(out + 3 * (row0 + (size_t)r * m.W) + 4 * k) = v;
      }
      __syncwarp();
    } else if (px < m.W) {
      const size_t pix0 = ((size_t)tc.b * m.H + py0) * m.W + px;
#pragma unroll
      for (int q = 0; q < kLanePx / 2; ++q) {
        float tv[2], rv[2], gv[2], bv[2];
        split(T[q], tv[0], tv[1]);
        split(cr[q], rv[0], rv[1]);
        split(cg[q], gv[0], gv[1]);
        split(cb[q], bv[0], bv[1]);
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          const int py = py0 + 4 * q + 2 * h;
          if (py < m.H) {
            const size_t pix = pix0 + (size_t)(4 * q + 2 * h) * (size_t)m.W;
            out[3 * pix + 0] = fmaf(tv[h], m.bg_r, rv[h]);
            out[3 * pix + 1] = fmaf(tv[h], m.bg_g, gv[h]);
            out[3 * pix + 2] = fmaf(tv[h], m.bg_b, bv[h]);
            if (kSave) {
              final_T[pix] = tv[h];
              last_idx[pix] = last[2 * q + h];
            }
          }
        }
      }
    }
  }
}

// The CTA kernels find their long tiles themselves (no list, counter or
// memset between the warp and CTA kernels): in chunk k, thread i of CTA b
// checks tile b + (blockDim.x * k + i) * gridDim.x (blockDim.x = kCtaThreads),
// so the long tiles of a clustered
// scene spread over all CTAs. The tiles found are compacted into s_long (one
// ballot per warp); a tile is long when short_max < pairs <= long_max. Returns
// how many. All threads call it; it ends with a barrier.
__device__ __forceinline__ int collect_long_tiles(const Meta& m, const int32_t* __restrict__ toff, int short_max,
                                                  int long_max, long long chunk, int* s_long, int* s_warp) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const long long t = (long long)blockIdx.x + (chunk * blockDim.x + threadIdx.x) * (long long)gridDim.x;
  bool is_long = false;
  if (t < m.total_tiles) {
    const int n = __ldg(&toff[t + 1]) - __ldg(&toff[t]);
    is_long = n > short_max && n <= long_max;
  }
  const unsigned bal = __ballot_sync(kFullMask, is_long);
  if (lane == 0) s_warp[warp] = __popc(bal);
  __syncthreads();
  int off = 0, total = 0;
  for (int w = 0; w < (int)(blockDim.x >> 5); ++w) {
    off += w < warp ? s_warp[w] : 0;
    total += s_warp[w];
  }
  if (is_long) s_long[off + __popc(bal & ((1u << lane) - 1u))] = (int)t;
  __syncthreads();
  return total;
}
// True while chunk k of this CTA's strided slice starts inside the tile range.
__device__ __forceinline__ bool long_chunk_live(const Meta& m, long long chunk) {
  return (long long)blockIdx.x + chunk * blockDim.x * (long long)gridDim.x < m.total_tiles;
}

// One staged batch of the CTA kernel over a thread's 2 packed pixels (kGuard:
// as fwd_warp_batch). A warp leaves the batch once its 64 pixels are finished.
template <bool kGuard, bool kSat>
__device__ __forceinline__ void fwd_cta_batch(const Meta& m, const float4 (*recs)[3], int cnt, int base, float fx,
                                              F2 fy, F2& T, F2& cr, F2& cg, F2& cb, int& last_l, int& last_h) {
  const F2 one = f2(1.0f), log2e = f2(kLog2e);
#pragma unroll 1
  for (int j = 0; j < cnt; ++j) {
    const float4 p0 = recs[j][0];
    const float4 p1 = recs[j][1];
    const float4 p2 = recs[j][2];
    const PowerCol pc = power_col(p0.z, p0.w, p1.x, __fsub_rn(fx, p0.x));
    const F2 power = power_at2(f2(pc.ta), f2(pc.tb), f2(pc.ch), sub2(fy, f2(p0.y)));
    const int consumed = base + j + 1;
    float pl, ph, xl, xh, tl, th;
    split(T, tl, th);
    if (!__any_sync(kFullMask, (tl > m.T_thr) | (th > m.T_thr))) break;
    split(power, pl, ph);
    split(mul2(power, log2e), xl, xh);
    float vl_, vh_;  // op * exp(power), capped at max_alpha where a record may saturate
    if (kSat) {
      vl_ = fminf(m.max_alpha, p1.y * ex2_approx(xl));
      vh_ = fminf(m.max_alpha, p1.y * ex2_approx(xh));
    } else {
      split(mul2(f2(p1.y), f2(ex2_approx(xl), ex2_approx(xh))), vl_, vh_);
    }
    float al, ah;
    int vis_l = 1, vis_h = 1;
    if (kGuard) {
      al = vis_select_fwd_v(tl, m.T_thr, pl, p2.z, vl_, consumed, last_l, vis_l);
      ah = vis_select_fwd_v(th, m.T_thr, ph, p2.z, vh_, consumed, last_h, vis_h);
    } else {
      al = vis_select_fwd(tl, m.T_thr, pl, p2.z, vl_, consumed, last_l);
      ah = vis_select_fwd(th, m.T_thr, ph, p2.z, vh_, consumed, last_h);
    }
    const F2 alpha = f2(al, ah);
    const F2 w = mul2(T, alpha);
    if (kGuard) {
      cr = select2(vis_l, vis_h, fma2(w, f2(p1.z), cr), cr);
      cg = select2(vis_l, vis_h, fma2(w, f2(p1.w), cg), cg);
      cb = select2(vis_l, vis_h, fma2(w, f2(p2.x), cb), cb);
    } else {
      cr = fma2(w, f2(p1.z), cr);
      cg = fma2(w, f2(p1.w), cg);
      cb = fma2(w, f2(p2.x), cb);
    }
    T = mul2(T, sub2(one, alpha));
  }
}

// CTA of kCtaThreads per long tile. A thread owns 2 pixels of one column (rows
// r and r + 8), packed as one f32x2 pair, and runs the warp kernel's
// branch-free record body on them, so the per-record work is amortised over 2
// pixels and done with packed instructions. Records are staged kBatch at a time
// in shared memory; the CTA stops early once no pixel is live.
template <bool kSave>
__global__ void __launch_bounds__(kCtaThreads, 8)
    k_render_fwd_cta(Meta m, const float4* __restrict__ rec, const int32_t* __restrict__ toff,
                     const int32_t* __restrict__ ids, float* __restrict__ out, float* __restrict__ final_T,
                     int32_t* __restrict__ last_idx, uint32_t* __restrict__ status) {
  pdl_wait();
  pdl_trigger();
  __shared__ float4 s_rec[kBatch][3];
  __shared__ int s_long[kCtaThreads], s_warp[kCtaThreads / 32];
  const int t = threadIdx.x;
  const F2 one = f2(1.0f), log2e = f2(kLog2e);
  for (long long chunk = 0; long_chunk_live(m, chunk); ++chunk) {
    const int n_long = collect_long_tiles(m, toff, kShortMax, 0x7fffffff, chunk, s_long, s_warp);
    for (int k = 0; k < n_long; ++k) {
      const int tile = s_long[k];
      const TileCoord tc = tile_coord(m, tile);
      const int px = tc.tx * kTile + (t & 15);
      const int py0 = tc.ty * kTile + (t >> 4);  // rows py0 and py0 + 8
      const float fx = (float)px + 0.5f;
      const F2 fy = f2((float)py0 + 0.5f, (float)py0 + 8.5f);
      const bool in_lo = px < m.W && py0 < m.H, in_hi = px < m.W && py0 + 8 < m.H;
      F2 T = f2(in_lo ? 1.0f : 0.0f, in_hi ? 1.0f : 0.0f), cr = f2(0.0f), cg = f2(0.0f), cb = f2(0.0f);
      int last_l = 0, last_h = 0;
      const int start = __ldg(&toff[tile]);
      const int n = __ldg(&toff[tile + 1]) - start;
      for (int base = 0; base < n; base += kBatch) {
        float tl, th;
        split(T, tl, th);
        const bool live = (tl > m.T_thr) | (th > m.T_thr);
        if (__syncthreads_count(live) == 0) break;
        const int cnt = min(kBatch, n - base);
        bool bad_color = false, sat = false;
        for (int i = t; i < cnt; i += kCtaThreads) {
          load_rec(rec, load_gi(ids, start + base + i, m.BG, status, kSiteRender), s_rec[i]);
          bad_color |= !finite_rgb(s_rec[i][1].z, s_rec[i][1].w, s_rec[i][2].x);
          sat |= may_saturate(s_rec[i][1].y, m.max_alpha);
        }
        const bool guard = __syncthreads_or(bad_color);
        if (guard)
          fwd_cta_batch<true, true>(m, s_rec, cnt, base, fx, fy, T, cr, cg, cb, last_l, last_h);
        else if (__syncthreads_or(sat))
          fwd_cta_batch<false, true>(m, s_rec, cnt, base, fx, fy, T, cr, cg, cb, last_l, last_h);
        else
          fwd_cta_batch<false, false>(m, s_rec, cnt, base, fx, fy, T, cr, cg, cb, last_l, last_h);
        __syncthreads();  // s_rec is refilled by the next batch
      }
      float tv[2], rv[2], gv[2], bv[2];
      split(T, tv[0], tv[1]);
      split(cr, rv[0], rv[1]);
      split(cg, gv[0], gv[1]);
      split(cb, bv[0], bv[1]);
      const int lastv[2] = {last_l, last_h};
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const int py = py0 + 8 * h;
        if (px < m.W && py < m.H) {
          const size_t pix = ((size_t)tc.b * m.H + py) * m.W + px;
          out[3 * pix + 0] = fmaf(tv[h], m.bg_r, rv[h]);
          out[3 * pix + 1] = fmaf(tv[h], m.bg_g, gv[h]);
          out[3 * pix + 2] = fmaf(tv[h], m.bg_b, bv[h]);
          if (kSave) {
            final_T[pix] = tv[h];
            last_idx[pix] = lastv[h];
          }
        }
      }
    }
  }
}

// ---------------------------------------------------------------------------
// Backward
// ---------------------------------------------------------------------------

// Per-pixel VJP of one visible splat (…metal:1017-1034), advancing the reverse
// recurrence (T_cur, gT). The splat's geometric gradients of all pixels that
// share dx (one lane's column) are accumulated as moments of g_power:
// S[0] = sum gp, S[1] = sum gp dy, S[2] = sum gp dy^2, expanded once per
// splat by vjp_expand (g_mean = gp (a dx + b dy, b dx + c dy), g_conic =
// gp (-dx^2/2, -dx dy, -dy^2/2)). S[3] = d opacity, S[4..6] = d color.
// For a visible splat op >= alpha_thr > eps, so raw / max(op, eps) = exp(power).
__device__ __forceinline__ void pixel_vjp(const Meta& m, float dy, float power, const float4& p1,
                                          const float4& p2, float gr, float gg, float gb, float& T_cur, float& gT,
                                          float* S) {
  const float e = __expf(power);
  const float raw = p1.y * e;
  const float alpha = fminf(m.max_alpha, raw);
  const float T_prev = __fdividef(T_cur, fmaxf(1.0f - alpha, m.eps));
  const float dot_gc = gr * p1.z + gg * p1.w + gb * p2.x;
  const float g_alpha = T_prev * (dot_gc - gT);
  const float wc = T_prev * alpha;
  const float g_raw = (power < p2.w) ? g_alpha : 0.0f;  // raw < max_alpha
  const float gp = g_raw * raw;
  S[0] += gp;
  const float gpdy = gp * dy;
  S[1] += gpdy;
  S[2] = fmaf(gpdy, dy, S[2]);
  S[3] = fmaf(g_raw, e, S[3]);
  S[4] = fmaf(gr, wc, S[4]);
  S[5] = fmaf(gg, wc, S[5]);
  S[6] = fmaf(gb, wc, S[6]);
  gT = alpha * dot_gc + (1.0f - alpha) * gT;
  T_cur = T_prev;
}

// pixel_vjp for two pixels of one column at once (packed pair arithmetic),
// free of branches: a pixel that does not see the splat (vis false) gets
// alpha = 0 and zero gradient terms, which leaves its (T_cur, gT) unchanged
// (T_cur * rcp(1 - 0) = T_cur; gT + 0 * d = gT) and adds nothing to S.
// gT advances as gT + alpha (dot_gc - gT), the same value as
// alpha dot_gc + (1 - alpha) gT up to rounding. S[t] holds per-half partial sums.
// Only gT can carry a non-finite colour into a pixel that does not see the
// splat (the other terms are selected or multiplied by finite zeros); kGuard
// selects it.
// kClampOm: clamp 1 - alpha at eps (only needed when max_alpha > 1 - eps;
// otherwise 1 - alpha >= 1 - max_alpha >= eps already).
template <bool kClampOm, bool kGuard, bool kCheckLast, bool kFirst, bool kSat = true>
__device__ __forceinline__ void pixel_vjp2(const Meta& m, int j, int last_l, int last_h, F2 dy, float pl, float ph,
                                           F2 op, float vis_thr, float sat_thr, F2 col_r, F2 col_g, F2 col_b,
                                           F2 gr, F2 gg, F2 gb, F2& T_cur, F2& gT, F2 (&S)[7]) {
  float xl, xh;
  split(mul2(f2(pl, ph), f2(kLog2e)), xl, xh);
  const F2 e = f2(ex2_approx(xl), ex2_approx(xh));
  float rl, rh;
  split(mul2(op, e), rl, rh);
  unsigned pass_l, pass_h;
  int vis_l = 1, vis_h = 1;
  const float al = vis_select_bwd<kCheckLast, kGuard, kSat>(j, last_l, pl, vis_thr, sat_thr,
                                                            kSat ? fminf(m.max_alpha, rl) : rl, pass_l, vis_l);
  const float ah = vis_select_bwd<kCheckLast, kGuard, kSat>(j, last_h, ph, vis_thr, sat_thr,
                                                            kSat ? fminf(m.max_alpha, rh) : rh, pass_h, vis_h);
  const F2 alpha = f2(al, ah);
  float oml, omh;
  split(sub2(f2(1.0f), alpha), oml, omh);
  if (kClampOm) {
    oml = fmaxf(oml, m.eps);
    omh = fmaxf(omh, m.eps);
  }
  const F2 T_prev = mul2(T_cur, f2(rcp_approx(oml), rcp_approx(omh)));
  const F2 dot_gc = fma2(gb, col_b, fma2(gg, col_g, mul2(gr, col_r)));
  const F2 d = sub2(dot_gc, gT);
  const F2 g_alpha = mul2(T_prev, d);
  const F2 wc = mul2(T_prev, alpha);
  // raw < max_alpha (power below the saturation log-threshold) passes g_alpha
  // to raw: d op = g_alpha e, d power = g_alpha raw = (g_alpha e) op. The gate
  // is an AND of the float bits with the pass mask.
  float gel, geh;
  split(mul2(g_alpha, e), gel, geh);
  const F2 ge = f2(__uint_as_float(__float_as_uint(gel) & pass_l), __uint_as_float(__float_as_uint(geh) & pass_h));
  const F2 gp = mul2(ge, op);
  const F2 gpdy = mul2(gp, dy);
  if (kFirst) {  // the lane's first pixel pair of this record starts the sums
    S[0] = gp;
    S[1] = gpdy;
    S[2] = mul2(gpdy, dy);
    S[3] = ge;
    S[4] = mul2(gr, wc);
    S[5] = mul2(gg, wc);
    S[6] = mul2(gb, wc);
  } else {
    S[0] = add2(S[0], gp);
    S[1] = add2(S[1], gpdy);
    S[2] = fma2(gpdy, dy, S[2]);
    S[3] = add2(S[3], ge);
    S[4] = fma2(gr, wc, S[4]);
    S[5] = fma2(gg, wc, S[5]);
    S[6] = fma2(gb, wc, S[6]);
  }
  // kGuard (a non-finite colour among the staged records): d is NaN for every
  // pixel, so gT moves only where the splat is visible.
  gT = kGuard ? select2(vis_l, vis_h, fma2(alpha, d, gT), gT) : fma2(alpha, d, gT);
  T_cur = T_prev;
}

// Expands one lane's moments S into the 9 gradient components (grad record order).
__device__ __forceinline__ void vjp_expand(const float* S, float dx, float a, float b, float c, float (&v)[16]) {
  v[0] = a * dx * S[0] + b * S[1];
  v[1] = b * dx * S[0] + c * S[1];
  v[2] = -0.5f * dx * dx * S[0];
  v[3] = -dx * S[1];
  v[4] = -0.5f * S[2];
  v[5] = S[3];
  v[6] = S[4];
  v[7] = S[5];
  v[8] = S[6];
#pragma unroll
  for (int q = 9; q < 16; ++q) v[q] = 0.0f;
}

// One warp's shared memory in the backward warp kernel: the per-pixel state of
// its next tile (single buffer: it is copied to registers when the tile
// starts, after which the next tile's prefetch may overwrite it), the records
// and ids of the current and next tile (double buffer), and the rows of the
// chunked gradient reduction.
struct BwdState {
  float grad[kTilePixels * 3];  // row-major 16x16 pixels x rgb
  float T[kTilePixels];
  int last[kTilePixels];
};
struct BwdRecs {
  float4 rec[kBwdShortMax][3];  // rows [0, kBwdHalf) and [kBwdHalf, kBwdShortMax): the two halves
  int ids[kBwdShortMax];
};
constexpr int kRedChunk = 3;    // records whose gradients are reduced together
constexpr int kRedStride = 36;  // padded row (32 lanes + 4): conflict-free 16-byte row reads
struct BwdWarpSmem {
  BwdState st;
  BwdRecs rb;
  float red[kRedChunk * kGradComps][kRedStride];
  int red_gi[kRedChunk];
};

// Where the backward adds its per-splat gradients. The sink type is a template
// argument of the backward kernels, so each mode compiles without the other's
// branches.
//
// RecSink: the packed records grad_rec [B*G*12] in depth-rank order (the
// un-sort is a separate launch); the staged target index is the rank itself.
struct RecSink {
  float* rec;
  __device__ __forceinline__ int index(const Meta&, int r) const { return r; }
  // Adds gradient component comp (0-8, grad-record order) of target idx.
  __device__ __forceinline__ void add(int idx, int comp, float v) const {
    atomicAdd(rec + (size_t)idx * GSB_REC_FLOATS + comp, v);
  }
  // All 9 components of one target (the CTA kernel's per-thread totals).
  __device__ __forceinline__ void add9(int idx, const float (&a)[kGradComps]) const {
    float4* g4 = reinterpret_cast<float4*>(rec + (size_t)idx * GSB_REC_FLOATS);
    atomicAdd(g4 + 0, make_float4(a[0], a[1], a[2], a[3]));
    atomicAdd(g4 + 1, make_float4(a[4], a[5], a[6], a[7]));
    atomicAdd(rec + (size_t)idx * GSB_REC_FLOATS + 8, a[8]);
  }
};

// InputSink: straight into the input-order outputs (the un-sort folded into
// the atomics): splat rank r goes to o = (r / G) G + perm[r], components 0-1
// to means2d [o*2], 2-4 to conics [o*3], 5 to opacities [o], 6-8 to colors
// [o*3]; a null output is skipped. The targets are zeroed beforehand.
struct InputSink {
  const int32_t* perm;
  float* means2d;
  float* conics;
  float* colors;
  float* opacities;
  // -1 stays -1 (an id out of range).
  __device__ __forceinline__ int index(const Meta& m, int r) const {
    return r < 0 ? r : fast_div(r, m.div_G) * m.G + __ldg(&perm[r]);
  }
  __device__ __forceinline__ void add(int idx, int comp, float v) const {
    float* dst;
    if (comp < 2) dst = means2d ? means2d + 2 * (size_t)idx + comp : nullptr;
    else if (comp < 5) dst = conics ? conics + 3 * (size_t)idx + (comp - 2) : nullptr;
    else if (comp == 5) dst = opacities ? opacities + idx : nullptr;
    else dst = colors ? colors + 3 * (size_t)idx + (comp - 6) : nullptr;
    if (dst) atomicAdd(dst, v);
  }
  __device__ __forceinline__ void add9(int idx, const float (&a)[kGradComps]) const {
#pragma unroll
    for (int q = 0; q < kGradComps; ++q)
      if (a[q] != 0.0f) add(idx, q, a[q]);
  }
};

struct TileOff {
  int start, n;
};

__device__ __forceinline__ TileOff load_off(const int32_t* __restrict__ toff, int tile, int total_tiles) {
  TileOff o{0, 0};
  if (tile < total_tiles) {
    o.start = __ldg(&toff[tile]);
    o.n = __ldg(&toff[tile + 1]) - o.start;
  }
  return o;
}

// Issues (does not wait for) the cp.async copies of one short tile's per-pixel
// state.
__device__ __forceinline__ void prefetch_bwd_state(const Meta& m, int tile, TileOff off, BwdState* st, int lane,
                                                   const float* __restrict__ grad,
                                                   const float* __restrict__ final_T,
                                                   const int32_t* __restrict__ last_idx) {
  if (tile >= m.total_tiles || off.n == 0 || off.n > kBwdShortMax) return;
  const TileCoord tc = tile_coord(m, tile);
  const int x0 = tc.tx * kTile, y0 = tc.ty * kTile;
  const bool full = (x0 + kTile <= m.W) && (y0 + kTile <= m.H) && ((m.W & 3) == 0);
  if (full) {
    // 16-byte chunks, one loop per array so no lane diverges: per row 12 of
    // grad, 4 of T, 4 of last_idx.
    const size_t pix0 = ((size_t)tc.b * m.H + y0) * m.W + x0;
#pragma unroll
    for (int i = 0; i < 6; ++i) {  // 16 rows x 12 chunks = 192 = 6 per lane
      const int q = lane + 32 * i, r = q / 12, k = q - r * 12;
      cp_async16(&st->grad[r * 48 + 4 * k], grad + 3 * (pix0 + (size_t)r * m.W) + 4 * k);
    }
#pragma unroll
    for (int i = 0; i < 2; ++i) {  // 16 rows x 4 chunks = 64 = 2 per lane, for T and for last_idx
      const int q = lane + 32 * i, r = q >> 2, k = q & 3;
      cp_async16(&st->T[r * 16 + 4 * k], final_T + pix0 + (size_t)r * m.W + 4 * k);
      cp_async16(&st->last[r * 16 + 4 * k], last_idx + pix0 + (size_t)r * m.W + 4 * k);
    }
  } else {
    for (int p = lane; p < kTilePixels; p += 32) {
      const int r = p >> 4, c = p & 15;
      if (x0 + c < m.W && y0 + r < m.H) {
        const size_t pix = ((size_t)tc.b * m.H + y0 + r) * m.W + x0 + c;
        cp_async4(&st->grad[3 * p + 0], grad + 3 * pix + 0);
        cp_async4(&st->grad[3 * p + 1], grad + 3 * pix + 1);
        cp_async4(&st->grad[3 * p + 2], grad + 3 * pix + 2);
        cp_async4(&st->T[p], final_T + pix);
        cp_async4(&st->last[p], last_idx + pix);
      } else {
        st->grad[3 * p + 0] = st->grad[3 * p + 1] = st->grad[3 * p + 2] = 0.0f;
        st->T[p] = 1.0f;
        st->last[p] = 0;
      }
    }
  }
}

// Issues the cp.async copies of one short tile's records and ids into rows
// [row0, row0 + n) of the record buffer.
__device__ __forceinline__ void prefetch_bwd_recs(TileOff off, BwdRecs* rb, int row0, int lane,
                                                  const float4* __restrict__ pair_rec,
                                                  const int32_t* __restrict__ ids) {
  if (off.n == 0 || off.n > kBwdShortMax) return;
  for (int q = lane; q < 3 * off.n; q += 32)
    cp_async16(&rb->rec[row0][0] + q, pair_rec + 3 * (size_t)off.start + q);
  for (int q = lane; q < off.n; q += 32) cp_async4(&rb->ids[row0 + q], ids + off.start + q);
}

// Sums the staged gradient rows of `count` records (row = record slot x
// component, one value per lane) and adds each nonzero total to the sink: lane
// L takes row L, reads it with 16-byte loads and sums it as packed pairs.
template <class Sink>
__device__ __forceinline__ void flush_red(BwdWarpSmem& W, int count, int lane, const Sink& sink) {
  __syncwarp();
  if (lane < count * kGradComps) {
    const float4* row = reinterpret_cast<const float4*>(&W.red[lane][0]);
    F2 acc0 = f2(0.0f), acc1 = f2(0.0f);
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const float4 v = row[i];
      acc0 = add2(acc0, f2(v.x, v.y));
      acc1 = add2(acc1, f2(v.z, v.w));
    }
    float a0, a1, a2, a3;
    split(acc0, a0, a1);
    split(acc1, a2, a3);
    const float total = (a0 + a1) + (a2 + a3);
    const int slot = lane / kGradComps, comp = lane - slot * kGradComps;
    const int gi = W.red_gi[slot];
    if (gi >= 0 && total != 0.0f) sink.add(gi, comp, total);
  }
  __syncwarp();
}

// One record (row row0 + j of the warp's record buffer) of the reverse walk for
// a lane's 8 pixels, with the per-record gradient reduction staged every
// kRedChunk records. kGuard: a record's colour is not finite (pixel_vjp2).
// kCheckLast: some pixel of the warp stops before this record (j >= the
// warp's smallest last_idx), so each pixel tests j < last.
template <bool kClampOm, bool kGuard, bool kCheckLast, bool kSat, class Sink>
__device__ __forceinline__ void bwd_warp_record(const Meta& m, BwdWarpSmem& W, int row0, int j, int lane, float fx,
                                                const F2 (&fy)[kLanePx / 2], const F2 (&gr)[kLanePx / 2],
                                                const F2 (&gg)[kLanePx / 2], const F2 (&gb)[kLanePx / 2],
                                                F2 (&Tc)[kLanePx / 2], F2 (&gT)[kLanePx / 2],
                                                const int (&last)[kLanePx], int& slot, uint32_t* __restrict__ status,
                                                const Sink& sink) {
  const BwdRecs& R = W.rb;
  const float4 p0 = R.rec[row0 + j][0];
  const float4 p1 = R.rec[row0 + j][1];
  const float4 p2 = R.rec[row0 + j][2];
  const float dx = __fsub_rn(fx, p0.x);
  const PowerCol pc = power_col(p0.z, p0.w, p1.x, dx);
  const F2 ta = f2(pc.ta), tb = f2(pc.tb), ch = f2(pc.ch), mu_y = f2(p0.y);
  const F2 col_r = f2(p1.z), col_g = f2(p1.w), col_b = f2(p2.x), op = f2(p1.y);
  F2 S[7];
#pragma unroll
  for (int q = 0; q < kLanePx / 2; ++q) {
    const F2 dy = sub2(fy[q], mu_y);
    const F2 power = power_at2(ta, tb, ch, dy);
    float pl, ph;
    split(power, pl, ph);
    if (q == 0)
      pixel_vjp2<kClampOm, kGuard, kCheckLast, true, kSat>(m, j, last[0], last[1], dy, pl, ph, op, p2.z, p2.w, col_r,
                                                     col_g, col_b, gr[0], gg[0], gb[0], Tc[0], gT[0], S);
    else
      pixel_vjp2<kClampOm, kGuard, kCheckLast, false, kSat>(m, j, last[2 * q], last[2 * q + 1], dy, pl, ph, op, p2.z,
                                                      p2.w, col_r, col_g, col_b, gr[q], gg[q], gb[q], Tc[q], gT[q],
                                                      S);
  }
  float Sv[7];
#pragma unroll
  for (int t = 0; t < 7; ++t) {
    float lo, hi;
    split(S[t], lo, hi);
    Sv[t] = lo + hi;
  }
  float v[16];
  vjp_expand(Sv, dx, p0.z, p0.w, p1.x, v);
  // Stage this splat's 9 lane values; every kRedChunk splats the warp
  // sums the staged rows (one row per lane) and adds them to the sink.
#pragma unroll
  for (int t = 0; t < kGradComps; ++t) W.red[slot * kGradComps + t][lane] = v[t];
  if (lane == 0) {
    int gi = R.ids[row0 + j];
    if ((unsigned)gi >= (unsigned)m.BG) {
      raise_error(status, GSB_DEVERR_BOUNDS, kSiteRenderBwd);
      gi = -1;
    }
    W.red_gi[slot] = sink.index(m, gi);
  }
  if (++slot == kRedChunk) {
    flush_red(W, slot, lane, sink);
    slot = 0;
  }
}

// The reverse walk over one short tile's records (rows row0 .. row0 +
// tile_last of the warp's record buffer). Records at or past lmin (the warp's
// smallest last_idx) test each pixel's stop; the ones before it are reached by
// every pixel and skip that test.
template <bool kClampOm, bool kGuard, bool kSat, class Sink>
__device__ __forceinline__ void bwd_warp_records(const Meta& m, BwdWarpSmem& W, int row0, int tile_last, int lmin,
                                                 int lane, float fx, const F2 (&fy)[kLanePx / 2],
                                                 const F2 (&gr)[kLanePx / 2], const F2 (&gg)[kLanePx / 2],
                                                 const F2 (&gb)[kLanePx / 2], F2 (&Tc)[kLanePx / 2],
                                                 F2 (&gT)[kLanePx / 2], const int (&last)[kLanePx],
                                                 uint32_t* __restrict__ status, const Sink& sink) {
  int slot = 0;
  int j = tile_last - 1;
#pragma unroll 1
  for (; j >= lmin; --j)
    bwd_warp_record<kClampOm, kGuard, true, kSat>(m, W, row0, j, lane, fx, fy, gr, gg, gb, Tc, gT, last, slot, status,
                                            sink);
#pragma unroll 1
  for (; j >= 0; --j)
    bwd_warp_record<kClampOm, kGuard, false, kSat>(m, W, row0, j, lane, fx, fy, gr, gg, gb, Tc, gT, last, slot, status,
                                             sink);
  if (slot > 0) flush_red(W, slot, lane, sink);
}

template <bool kClampOm, class Sink>
__global__ void __launch_bounds__(kBwdWarps * 32, 4)
    k_render_bwd_warp(Meta m, const float4* __restrict__ pair_rec, const int32_t* __restrict__ toff,
                      const int32_t* __restrict__ ids, const float* __restrict__ final_T,
                      const int32_t* __restrict__ last_idx, const float* __restrict__ grad,
                      Sink sink, uint32_t* __restrict__ status, int claims) {
  pdl_wait();
  pdl_trigger();
  extern __shared__ float4 s_dyn[];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  BwdWarpSmem& W = reinterpret_cast<BwdWarpSmem*>(s_dyn)[warp];
  // Tiles are claimed one at a time, three ahead of use: the current tile, the
  // next one (state and records prefetched), the one after (offsets loaded),
  // and a claim in flight for the tile after that.
  // Without claims (claims == 0) the k-th tile of a warp is the grid stride's.
  uint32_t* const claim = status + GSB_STATUS_TILE_CLAIM;
  const int stride = gridDim.x * kBwdWarps;
  int next_static = blockIdx.x * kBwdWarps + warp;
  auto take = [&]() {
    if (claims) return claim_tiles(claim, 1, lane);
    const int t = next_static;
    next_static += stride;
    return t;
  };
  int tile = take();
  int nxt_tile = take();
  int nn_tile = take();
  TileOff cur = load_off(toff, tile, m.total_tiles);
  TileOff nxt = load_off(toff, nxt_tile, m.total_tiles);
  if (tile < m.total_tiles) prefetch_bwd_state(m, tile, cur, &W.st, lane, grad, final_T, last_idx);
  prefetch_bwd_recs(cur, &W.rb, 0, lane, pair_rec, ids);
  cp_async_commit();
  int row0 = 0;          // first record row of the current tile
  bool pending = false;  // the current tile's records are not copied yet
  while (tile < m.total_tiles) {
    int pend = next_static;  // the tile after nn: a claim in flight until the end of this tile
    if (claims) pend = lane == 0 ? (int)atomicAdd(claim, 1u) : 0;
    else next_static += stride;
    const TileOff nn = load_off(toff, nn_tile, m.total_tiles);
    cp_async_wait<0>();
    __syncwarp();
    if (pending) {  // after or before a tile of more than kBwdHalf records: copy now, into rows from 0
      prefetch_bwd_recs(cur, &W.rb, 0, lane, pair_rec, ids);
      cp_async_commit();
      cp_async_wait<0>();
      __syncwarp();
    }
    const BwdRecs& R = W.rb;
    const int n = cur.n;
    const bool work = n > 0 && n <= kBwdShortMax;
    const TileCoord tc = tile_coord(m, tile);
    const int px = tc.tx * kTile + (lane & 15);
    const int py0 = tc.ty * kTile + (lane >> 4);
    const float fx = (float)px + 0.5f;
    const float fy0 = (float)py0 + 0.5f;
    // Pair q holds rows py0 + 4q and py0 + 4q + 2 (see the forward kernel).
    F2 fy[kLanePx / 2], gr[kLanePx / 2], gg[kLanePx / 2], gb[kLanePx / 2], Tc[kLanePx / 2], gT[kLanePx / 2];
    int last[kLanePx];
    int lmax = 0, lmin = n;
    if (work) {
#pragma unroll
      for (int q = 0; q < kLanePx / 2; ++q) {
        fy[q] = f2(fy0 + (float)(4 * q), fy0 + (float)(4 * q + 2));
        const int pl = ((lane >> 4) + 4 * q) * kTile + (lane & 15);
        const int ph = pl + 2 * kTile;
        gr[q] = f2(W.st.grad[3 * pl + 0], W.st.grad[3 * ph + 0]);
        gg[q] = f2(W.st.grad[3 * pl + 1], W.st.grad[3 * ph + 1]);
        gb[q] = f2(W.st.grad[3 * pl + 2], W.st.grad[3 * ph + 2]);
        Tc[q] = f2(W.st.T[pl], W.st.T[ph]);
        gT[q] = fma2(gb[q], f2(m.bg_b), fma2(gg[q], f2(m.bg_g), mul2(gr[q], f2(m.bg_r))));
        last[2 * q] = min(W.st.last[pl], n);
        last[2 * q + 1] = min(W.st.last[ph], n);
        lmax = max(lmax, max(last[2 * q], last[2 * q + 1]));
        lmin = min(lmin, min(last[2 * q], last[2 * q + 1]));
      }
    }
    __syncwarp();  // W.st is read: the next tile's prefetch may overwrite it
    // The next tile's records go into the other half now when both tiles fit
    // a half; otherwise they are copied when that tile starts.
    const bool recs_now = cur.n <= kBwdHalf && nxt.n <= kBwdHalf;
    const int next_row0 = recs_now ? kBwdHalf - row0 : 0;
    if (nxt_tile < m.total_tiles) prefetch_bwd_state(m, nxt_tile, nxt, &W.st, lane, grad, final_T, last_idx);
    if (recs_now) prefetch_bwd_recs(nxt, &W.rb, next_row0, lane, pair_rec, ids);
    cp_async_commit();
    if (work) {  // tiles above kBwdShortMax: k_render_bwd_cta finds them
      const int tile_last = __reduce_max_sync(kFullMask, lmax);
      const int warp_lmin = __reduce_min_sync(kFullMask, lmin);
      // A non-finite colour among the records this tile walks takes the guarded
      // body; a record that may saturate takes the body with the saturation test.
      bool bad_color = false, sat = false;
      for (int q = lane; q < tile_last; q += 32) {
        bad_color |= !finite_rgb(W.rb.rec[row0 + q][1].z, W.rb.rec[row0 + q][1].w, W.rb.rec[row0 + q][2].x);
        sat |= may_saturate(W.rb.rec[row0 + q][1].y, m.max_alpha);
      }
      const bool guard = __any_sync(kFullMask, bad_color), any_sat = __any_sync(kFullMask, sat);
      if (guard)
        bwd_warp_records<kClampOm, true, true>(m, W, row0, tile_last, warp_lmin, lane, fx, fy, gr, gg, gb, Tc, gT,
                                               last, status, sink);
      else if (any_sat)
        bwd_warp_records<kClampOm, false, true>(m, W, row0, tile_last, warp_lmin, lane, fx, fy, gr, gg, gb, Tc, gT,
                                                last, status, sink);
      else
        bwd_warp_records<kClampOm, false, false>(m, W, row0, tile_last, warp_lmin, lane, fx, fy, gr, gg, gb, Tc,
                                                 gT, last, status, sink);
    }
    tile = nxt_tile;
    nxt_tile = nn_tile;
    nn_tile = claims ? __shfl_sync(kFullMask, pend, 0) : pend;
    cur = nxt;
    nxt = nn;
    row0 = next_row0;
    pending = !recs_now;
  }
  cp_async_wait<0>();
}

// Sums the staged rows of `count` records of one warp (row = record slot x
// component, one value per lane) into the CTA's per-record accumulators.
__device__ __forceinline__ void flush_red_cta(float (*red)[kRedStride], const int* red_j, int count, int lane,
                                              float (*acc)[kGradComps]) {
  __syncwarp();
  if (lane < count * kGradComps) {
    const float4* row = reinterpret_cast<const float4*>(&red[lane][0]);
    F2 a0 = f2(0.0f), a1 = f2(0.0f);
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const float4 v = row[i];
      a0 = add2(a0, f2(v.x, v.y));
      a1 = add2(a1, f2(v.z, v.w));
    }
    float x0, x1, x2, x3;
    split(a0, x0, x1);
    split(a1, x2, x3);
    const float total = (x0 + x1) + (x2 + x3);
    const int slot = lane / kGradComps, comp = lane - slot * kGradComps;
    if (total != 0.0f) atomicAdd(&acc[red_j[slot]][comp], total);
  }
  __syncwarp();
}

// CTA of kCtaThreads per long tile, 2 pixels per thread as in the forward CTA
// kernel, with the warp kernel's packed per-pixel VJP (pixel_vjp2). Per record a
// thread sums its pair's moments, expands them once, and the warp reduces the
// 9 gradient components of its 64 pixels (one reduce-scatter) into shared
// accumulators; each batch of records ends with one vector atomic per record.
template <bool kClampOm, class Sink>
__global__ void __launch_bounds__(kCtaThreads)
    k_render_bwd_cta(Meta m, const float4* __restrict__ rec, const int32_t* __restrict__ toff,
                     const int32_t* __restrict__ ids, const float* __restrict__ final_T,
                     const int32_t* __restrict__ last_idx, const float* __restrict__ grad,
                     Sink sink, uint32_t* __restrict__ status) {
  pdl_wait();
  pdl_trigger();
  __shared__ float4 s_rec[kBatch][3];
  __shared__ int s_gi[kBatch];
  __shared__ float s_acc[kBatch][kGradComps];
  __shared__ __align__(16) float s_red[kCtaThreads / 32][kRedChunk * kGradComps][kRedStride];
  __shared__ int s_red_j[kCtaThreads / 32][kRedChunk];
  __shared__ int s_max[kCtaThreads / 32];
  __shared__ int s_long[kCtaThreads], s_warp[kCtaThreads / 32];
  const int t = threadIdx.x, lane = t & 31, warp = t >> 5;
  if (blockIdx.x == 0 && t == 0) status[GSB_STATUS_TILE_CLAIM] = 0u;  // the warp kernel has completed
  for (long long chunk = 0; long_chunk_live(m, chunk); ++chunk) {
    const int n_long = collect_long_tiles(m, toff, kBwdShortMax, 0x7fffffff, chunk, s_long, s_warp);
    for (int k = 0; k < n_long; ++k) {
      const int tile = s_long[k];
      const TileCoord tc = tile_coord(m, tile);
      const int px = tc.tx * kTile + (t & 15);
      const int py0 = tc.ty * kTile + (t >> 4);  // rows py0 and py0 + 8
      const float fx = (float)px + 0.5f;
      const F2 fy = f2((float)py0 + 0.5f, (float)py0 + 8.5f);
      const int start = toff[tile];
      const int n = toff[tile + 1] - start;
      float g[2][3] = {{0.f, 0.f, 0.f}, {0.f, 0.f, 0.f}}, Tv[2] = {1.0f, 1.0f};
      int lastv[2] = {0, 0};
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const int py = py0 + 8 * h;
        if (px < m.W && py < m.H) {
          const size_t pix = ((size_t)tc.b * m.H + py) * m.W + px;
          g[h][0] = grad[3 * pix + 0];
          g[h][1] = grad[3 * pix + 1];
          g[h][2] = grad[3 * pix + 2];
          Tv[h] = final_T[pix];
          lastv[h] = min(last_idx[pix], n);
        }
      }
      const F2 gr = f2(g[0][0], g[1][0]), gg = f2(g[0][1], g[1][1]), gb = f2(g[0][2], g[1][2]);
      F2 Tc = f2(Tv[0], Tv[1]);
      F2 gT = fma2(gb, f2(m.bg_b), fma2(gg, f2(m.bg_g), mul2(gr, f2(m.bg_r))));
      const int wmax = __reduce_max_sync(kFullMask, max(lastv[0], lastv[1]));
      if (lane == 0) s_max[warp] = wmax;
      __syncthreads();
      int tile_last = 0;
#pragma unroll
      for (int w = 0; w < kCtaThreads / 32; ++w) tile_last = max(tile_last, s_max[w]);
      for (int bend = tile_last; bend > 0; bend -= kBatch) {
        const int bstart = max(0, bend - kBatch);
        const int cnt = bend - bstart;
        bool bad_color = false, sat = false;
        for (int i = t; i < cnt; i += kCtaThreads) {
          const int gi = load_gi(ids, start + bstart + i, m.BG, status, kSiteRenderBwd);
          s_gi[i] = sink.index(m, gi);
          load_rec(rec, gi, s_rec[i]);
          bad_color |= !finite_rgb(s_rec[i][1].z, s_rec[i][1].w, s_rec[i][2].x);
          sat |= may_saturate(s_rec[i][1].y, m.max_alpha);
        }
        for (int i = t; i < cnt * kGradComps; i += kCtaThreads) (&s_acc[0][0])[i] = 0.0f;
        // A non-finite colour in the batch: the guarded per-pixel VJP; a record
        // that may saturate: the saturation test (both CTA-uniform).
        const bool guard = __syncthreads_or(bad_color);
        const bool any_sat = __syncthreads_or(sat);
        int slot = 0;
#pragma unroll 1
        for (int jj = cnt - 1; jj >= 0; --jj) {
          const int j = bstart + jj;
          const float4 p0 = s_rec[jj][0];
          const float4 p1 = s_rec[jj][1];
          const float4 p2 = s_rec[jj][2];
          const float dx = __fsub_rn(fx, p0.x);
          const PowerCol pc = power_col(p0.z, p0.w, p1.x, dx);
          const F2 dy = sub2(fy, f2(p0.y));
          const F2 power = power_at2(f2(pc.ta), f2(pc.tb), f2(pc.ch), dy);
          float pl, ph;
          split(power, pl, ph);
          // Skip (warp-uniform) a record no pixel of this warp sees before its stop:
          // its alpha is 0 there, so it changes no state and adds no gradient.
          const bool vis = ((j < lastv[0]) & (pl <= 0.0f) & (pl >= p2.z)) | ((j < lastv[1]) & (ph <= 0.0f) & (ph >= p2.z));
          if (!__any_sync(kFullMask, vis)) continue;
          F2 S[7];
          if (guard)
            pixel_vjp2<kClampOm, true, true, true>(m, j, lastv[0], lastv[1], dy, pl, ph, f2(p1.y), p2.z, p2.w,
                                                   f2(p1.z), f2(p1.w), f2(p2.x), gr, gg, gb, Tc, gT, S);
          else if (any_sat)
            pixel_vjp2<kClampOm, false, true, true>(m, j, lastv[0], lastv[1], dy, pl, ph, f2(p1.y), p2.z, p2.w,
                                                    f2(p1.z), f2(p1.w), f2(p2.x), gr, gg, gb, Tc, gT, S);
          else
            pixel_vjp2<kClampOm, false, true, true, false>(m, j, lastv[0], lastv[1], dy, pl, ph, f2(p1.y), p2.z,
                                                           p2.w, f2(p1.z), f2(p1.w), f2(p2.x), gr, gg, gb, Tc, gT, S);
          float Sv[7];
#pragma unroll
          for (int q = 0; q < 7; ++q) {
            float lo, hi;
            split(S[q], lo, hi);
            Sv[q] = lo + hi;
          }
          float v[16];
          vjp_expand(Sv, dx, p0.z, p0.w, p1.x, v);
          // Stage the lane values of this record; every kRedChunk records the
          // warp sums the staged rows (one row per lane) into s_acc.
#pragma unroll
          for (int q = 0; q < kGradComps; ++q) s_red[warp][slot * kGradComps + q][lane] = v[q];
          if (lane == 0) s_red_j[warp][slot] = jj;
          if (++slot == kRedChunk) {
            flush_red_cta(s_red[warp], s_red_j[warp], slot, lane, s_acc);
            slot = 0;
          }
        }
        if (slot > 0) flush_red_cta(s_red[warp], s_red_j[warp], slot, lane, s_acc);
        __syncthreads();
        for (int i = t; i < cnt; i += kCtaThreads) {
          const int gi = s_gi[i];
          float acc[kGradComps];
          bool nz = false;
#pragma unroll
          for (int q = 0; q < kGradComps; ++q) {
            acc[q] = s_acc[i][q];
            nz |= (acc[q] != 0.0f);
          }
          if (nz && gi >= 0) {
            sink.add9(gi, acc);
          }
        }
        __syncthreads();  // s_rec / s_acc are refilled by the next batch
      }
    }
  }
}

// grad_rec (depth-rank order, packed) -> user layout in input order, one
// thread per rank scattering its values (for small splat counts, where one
// launch is all the time there is).
__global__ void __launch_bounds__(256)
    k_unsort(Meta m, const int32_t* __restrict__ perm, const float4* __restrict__ grad_rec,
             float* __restrict__ g_means2d, float* __restrict__ g_conics, float* __restrict__ g_colors,
             float* __restrict__ g_opac) {
  pdl_wait();
  pdl_trigger();
  const int r = blockIdx.x * blockDim.x + threadIdx.x;
  if (r >= m.BG) return;
  const int b = fast_div(r, m.div_G);
  const int o = b * m.G + perm[r];
  const float4 q0 = grad_rec[3 * r + 0];
  const float4 q1 = grad_rec[3 * r + 1];
  const float4 q2 = grad_rec[3 * r + 2];
  if (g_means2d) {
    g_means2d[2 * o + 0] = q0.x;
    g_means2d[2 * o + 1] = q0.y;
  }
  if (g_conics) {
    g_conics[3 * o + 0] = q0.z;
    g_conics[3 * o + 1] = q0.w;
    g_conics[3 * o + 2] = q1.x;
  }
  if (g_opac) g_opac[o] = q1.y;
  if (g_colors) {
    g_colors[3 * o + 0] = q1.z;
    g_colors[3 * o + 1] = q1.w;
    g_colors[3 * o + 2] = q2.x;
  }
}

// The same as a gather, for large splat counts: scattering each rank's 9 values to a random input position cost one
// partly written 32-byte sector per value. First the inverse permutation is
// written, one 4-byte slot per splat, into the first requested output tensor
// (its element o * inv_stride); then the thread of input position o reads its
// rank there, loads that rank's packed gradients and writes all of o's outputs
// with consecutive stores, its own inverse slot included (no other thread
// reads that slot).
__global__ void __launch_bounds__(256)
    k_unsort_invert(Meta m, const int32_t* __restrict__ perm, int32_t* __restrict__ inv, int inv_stride) {
  pdl_wait();
  pdl_trigger();
  const int r = blockIdx.x * blockDim.x + threadIdx.x;
  if (r >= m.BG) return;
  const int b = fast_div(r, m.div_G);
  inv[(size_t)(b * m.G + perm[r]) * inv_stride] = r;
}

__global__ void __launch_bounds__(256)
    k_unsort_gather(Meta m, const int32_t* inv, int inv_stride, const float4* __restrict__ grad_rec,
                    float* g_means2d, float* g_conics, float* g_colors, float* g_opac) {  // inv aliases an output
  pdl_wait();
  pdl_trigger();
  const int o = blockIdx.x * blockDim.x + threadIdx.x;
  if (o >= m.BG) return;
  const int r = inv[(size_t)o * inv_stride];
  if ((unsigned)r >= (unsigned)m.BG) return;  // perm is a permutation: every slot was written
  const float4 q0 = grad_rec[3 * r + 0];
  const float4 q1 = grad_rec[3 * r + 1];
  const float4 q2 = grad_rec[3 * r + 2];
  if (g_means2d) {
    g_means2d[2 * o + 0] = q0.x;
    g_means2d[2 * o + 1] = q0.y;
  }
  if (g_conics) {
    g_conics[3 * o + 0] = q0.z;
    g_conics[3 * o + 1] = q0.w;
    g_conics[3 * o + 2] = q1.x;
  }
  if (g_opac) g_opac[o] = q1.y;
  if (g_colors) {
    g_colors[3 * o + 0] = q1.z;
    g_colors[3 * o + 1] = q1.w;
    g_colors[3 * o + 2] = q2.x;
  }
}

// From this many splats the un-sort runs as invert + gather (c4's 2^20:
// 93 -> 38 us); below it one scatter launch is as fast (65,536: 10.8 us).
constexpr int kGatherUnsortMin = 1 << 18;

constexpr size_t kBwdWarpSmem = sizeof(BwdWarpSmem) * kBwdWarps;

// Persistent grid sizes (CTAs resident per SM x SMs), cached per device.
struct GridCache {
  int sms = 0;
  int fwd_warp[2] = {0, 0}, fwd_cta[2] = {0, 0}, bwd_warp = 0, bwd_cta = 0;
};

const GridCache& grids() {
  static GridCache cache[64];
  static std::mutex mu;  // host threads may launch concurrently: fill each entry once, under the lock
  int dev = 0;
  cudaGetDevice(&dev);
  std::lock_guard<std::mutex> lock(mu);
  GridCache& g = cache[dev & 63];
  if (g.sms == 0) {
    int sms = 148;
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    for (const void* fn : {(const void*)k_render_bwd_warp<true, RecSink>, (const void*)k_render_bwd_warp<false, RecSink>,
                           (const void*)k_render_bwd_warp<true, InputSink>,
                           (const void*)k_render_bwd_warp<false, InputSink>})
      cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kBwdWarpSmem);
    auto occ = [&](const void* fn, int threads, size_t smem) {
      int b = 1;
      if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&b, fn, threads, smem) != cudaSuccess || b < 1) b = 1;
      return b * sms;
    };
    g.fwd_warp[0] = occ((const void*)k_render_fwd_warp<false>, kWarps * 32, 0);
    g.fwd_warp[1] = occ((const void*)k_render_fwd_warp<true>, kWarps * 32, 0);
    g.fwd_cta[0] = occ((const void*)k_render_fwd_cta<false>, kCtaThreads, 0);
    g.fwd_cta[1] = occ((const void*)k_render_fwd_cta<true>, kCtaThreads, 0);
    // One grid for both sinks: the smaller residency of the two.
    g.bwd_warp = min(occ((const void*)k_render_bwd_warp<false, RecSink>, kBwdWarps * 32, kBwdWarpSmem),
                     occ((const void*)k_render_bwd_warp<false, InputSink>, kBwdWarps * 32, kBwdWarpSmem));
    g.bwd_cta = min(occ((const void*)k_render_bwd_cta<false, RecSink>, kCtaThreads, 0),
                    occ((const void*)k_render_bwd_cta<false, InputSink>, kCtaThreads, 0));
    g.sms = sms;
  }
  return g;
}

}  // namespace
}  // namespace gsb

using namespace gsb;

// The compositing kernels need no scratch (the CTA kernels find their long
// tiles themselves); the workspace arguments stay in the ABI, unused.
extern "C" size_t gsb_render_workspace_size(const gsb_raster_meta* meta) {
  Meta m;
  (void)make_meta(meta, &m);
  return 0;
}

namespace gsb {
namespace {

// Grid of the long-tile CTA kernels. Each CTA scans a strided slice of the
// tiles and renders the long ones it finds, one after another. Where long tiles
// are common (many splats per tile: clustered or dense scenes), one CTA per
// tile instead gives every long tile its own CTA, and the hardware block
// scheduler hands them to SMs as slots free up, which balances tiles of very
// different lengths; the extra CTAs exit after two loads. With about one
// splat per tile (c2, c3) a slice per resident CTA keeps the scan cheap.
int long_tile_grid(const Meta& m, int resident) {
  if ((int64_t)m.BG >= kDenseSplatsPerTile * (int64_t)m.total_tiles) return max(1, m.total_tiles);
  return max(1, min(resident, m.total_tiles));
}

// The forward's two launches: warp per short tile, then CTA per long tile.
int launch_forward(const Meta& m, const float* rec, const int32_t* tile_offsets, const int32_t* binned_ids,
                   float* out_rgb, float* final_T, int32_t* last_idx, float* pair_rec, uint32_t* status,
                   cudaStream_t stream) {
  const GridCache& g = grids();
  const float4* r4 = reinterpret_cast<const float4*>(rec);
  float4* pr4 = reinterpret_cast<float4*>(pair_rec);
  const int warp_grid = max(1, min(g.fwd_warp[final_T ? 1 : 0], (m.total_tiles + kWarps - 1) / kWarps));
  const int cta_grid = long_tile_grid(m, g.fwd_cta[final_T ? 1 : 0]);
  cudaError_t e;
  if (final_T) {
    e = launch_pdl(k_render_fwd_warp<true>, warp_grid, kWarps * 32, 0, stream, m, r4, tile_offsets, binned_ids,
                   out_rgb, final_T, last_idx, pr4, status);
    if (e == cudaSuccess)
      e = launch_pdl(k_render_fwd_cta<true>, cta_grid, kCtaThreads, 0, stream, m, r4, tile_offsets, binned_ids,
                     out_rgb, final_T, last_idx, status);
  } else {
    e = launch_pdl(k_render_fwd_warp<false>, warp_grid, kWarps * 32, 0, stream, m, r4, tile_offsets, binned_ids,
                   out_rgb, nullptr, nullptr, nullptr, status);
    if (e == cudaSuccess)
      e = launch_pdl(k_render_fwd_cta<false>, cta_grid, kCtaThreads, 0, stream, m, r4, tile_offsets, binned_ids,
                     out_rgb, nullptr, nullptr, status);
  }
  note_launches(2);
  return cuda_status(e);
}

}  // namespace
}  // namespace gsb

extern "C" int gsb_render_forward(const gsb_raster_meta* meta, const float* rec, const int32_t* tile_offsets,
                                  const int32_t* binned_ids, float* out_rgb, float* final_T, int32_t* last_idx,
                                  float* pair_rec, uint32_t* status, void* workspace, size_t workspace_bytes,
                                  void* stream_) {
  Meta m;
  int rc = make_meta(meta, &m);
  if (rc != GSB_OK) return rc;
  if (!tile_offsets || !out_rgb || !status) return GSB_ERR_INVALID_ARGUMENT;
  if ((final_T == nullptr) != (last_idx == nullptr) || (final_T == nullptr) != (pair_rec == nullptr))
    return GSB_ERR_INVALID_ARGUMENT;
  if (m.BG > 0 && !rec) return GSB_ERR_INVALID_ARGUMENT;
  (void)workspace;
  (void)workspace_bytes;
  return launch_forward(m, rec, tile_offsets, binned_ids, out_rgb, final_T, last_idx, pair_rec, status,
                        static_cast<cudaStream_t>(stream_));
}

namespace gsb {
namespace {
// Launches both backward kernels into `sink` (zeroed by the caller).
template <class Sink>
int render_backward_launch(const Meta& m, const float* rec, const int32_t* tile_offsets, const int32_t* binned_ids,
                           const float* final_T, const int32_t* last_idx, const float* pair_rec,
                           const float* grad_rgb, const Sink& sink, uint32_t* status, cudaStream_t stream) {
  const GridCache& g = grids();
  const float4* r4 = reinterpret_cast<const float4*>(rec);
  const int warp_grid = max(1, min(g.bwd_warp, (m.total_tiles + kBwdWarps - 1) / kBwdWarps));
  const int cta_grid = long_tile_grid(m, g.bwd_cta);
  const int claims = m.total_tiles >= kMinTilesPerWarpForClaims * warp_grid * kBwdWarps ? 1 : 0;
  // 1 - alpha needs the eps clamp only when max_alpha > 1 - eps.
  const bool clamp_om = !(1.0f - m.max_alpha >= m.eps);
  auto bwd_warp = clamp_om ? k_render_bwd_warp<true, Sink> : k_render_bwd_warp<false, Sink>;
  auto bwd_cta = clamp_om ? k_render_bwd_cta<true, Sink> : k_render_bwd_cta<false, Sink>;
  cudaError_t e = launch_pdl(bwd_warp, warp_grid, kBwdWarps * 32, kBwdWarpSmem, stream, m,
                             reinterpret_cast<const float4*>(pair_rec), tile_offsets, binned_ids, final_T, last_idx,
                             grad_rgb, sink, status, claims);
  if (e == cudaSuccess)
    e = launch_pdl(bwd_cta, cta_grid, kCtaThreads, 0, stream, m, r4, tile_offsets, binned_ids, final_T,
                   last_idx, grad_rgb, sink, status);
  note_launches(2);
  return cuda_status(e);
}
}  // namespace
}  // namespace gsb

extern "C" int gsb_render_backward(const gsb_raster_meta* meta, const float* rec, const int32_t* tile_offsets,
                                   const int32_t* binned_ids, const float* final_T, const int32_t* last_idx,
                                   const float* pair_rec, const float* grad_rgb, float* grad_rec, uint32_t* status,
                                   void* workspace, size_t workspace_bytes, void* stream_) {
  Meta m;
  int rc = make_meta(meta, &m);
  if (rc != GSB_OK) return rc;
  if (!tile_offsets || !final_T || !last_idx || !grad_rgb || !status) return GSB_ERR_INVALID_ARGUMENT;
  if (m.BG > 0 && (!rec || !grad_rec || !pair_rec)) return GSB_ERR_INVALID_ARGUMENT;
  // pair_rec is staged with 16-byte asynchronous copies.
  if (reinterpret_cast<uintptr_t>(pair_rec) & 15u) return GSB_ERR_INVALID_ARGUMENT;
  (void)workspace;
  (void)workspace_bytes;
  cudaStream_t stream = static_cast<cudaStream_t>(stream_);
  if (m.BG > 0) {
    cudaError_t e = cudaMemsetAsync(grad_rec, 0, sizeof(float) * GSB_REC_FLOATS * (size_t)m.BG, stream);
    if (e != cudaSuccess) return GSB_ERR_CUDA;
  }
  const RecSink sink{grad_rec};
  return render_backward_launch(m, rec, tile_offsets, binned_ids, final_T, last_idx, pair_rec, grad_rgb, sink,
                                status, stream);
}

extern "C" int gsb_render_backward_inputs(const gsb_raster_meta* meta, const float* rec, const int32_t* tile_offsets,
                                          const int32_t* binned_ids, const float* final_T, const int32_t* last_idx,
                                          const float* pair_rec, const float* grad_rgb, const int32_t* perm,
                                          float* g_means2d, float* g_conics, float* g_colors, float* g_opacities,
                                          uint32_t* status, void* stream_) {
  Meta m;
  int rc = make_meta(meta, &m);
  if (rc != GSB_OK) return rc;
  if (!tile_offsets || !final_T || !last_idx || !grad_rgb || !status) return GSB_ERR_INVALID_ARGUMENT;
  if (m.BG > 0 && (!rec || !pair_rec || !perm)) return GSB_ERR_INVALID_ARGUMENT;
  if (reinterpret_cast<uintptr_t>(pair_rec) & 15u) return GSB_ERR_INVALID_ARGUMENT;
  const InputSink sink{perm, g_means2d, g_conics, g_colors, g_opacities};
  return render_backward_launch(m, rec, tile_offsets, binned_ids, final_T, last_idx, pair_rec, grad_rgb, sink,
                                status, static_cast<cudaStream_t>(stream_));
}

extern "C" int gsb_unsort_grads(const gsb_raster_meta* meta, const int32_t* perm, const float* grad_rec,
                                float* g_means2d, float* g_conics, float* g_colors, float* g_opacities,
                                void* stream_) {
  Meta m;
  int rc = make_meta(meta, &m);
  if (rc != GSB_OK) return rc;
  if (m.BG == 0) return GSB_OK;
  if (!perm || !grad_rec) return GSB_ERR_INVALID_ARGUMENT;
  // The inverse permutation's slots: the first requested output (opacities
  // have one float per splat, the others two or three).
  int32_t* inv = nullptr;
  int stride = 0;
  if (g_opacities) inv = reinterpret_cast<int32_t*>(g_opacities), stride = 1;
  else if (g_means2d) inv = reinterpret_cast<int32_t*>(g_means2d), stride = 2;
  else if (g_conics) inv = reinterpret_cast<int32_t*>(g_conics), stride = 3;
  else if (g_colors) inv = reinterpret_cast<int32_t*>(g_colors), stride = 3;
  if (!inv) return GSB_OK;  // no gradient requested
  cudaStream_t stream = static_cast<cudaStream_t>(stream_);
  if (m.BG < kGatherUnsortMin) {
    const cudaError_t e1 = launch_pdl(k_unsort, grid1d(m.BG, 256), 256, 0, stream, m, perm,
                                      reinterpret_cast<const float4*>(grad_rec), g_means2d, g_conics, g_colors,
                                      g_opacities);
    note_launches(1);
    return cuda_status(e1);
  }
  cudaError_t e = launch_pdl(k_unsort_invert, grid1d(m.BG, 256), 256, 0, stream, m, perm, inv, stride);
  if (e == cudaSuccess)
    e = launch_pdl(k_unsort_gather, grid1d(m.BG, 256), 256, 0, stream, m, static_cast<const int32_t*>(inv), stride,
                   reinterpret_cast<const float4*>(grad_rec), g_means2d, g_conics, g_colors, g_opacities);
  note_launches(2);
  return cuda_status(e);
}
