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
// record (see vis_log_threshold), with `power` evaluated in the reference's
// operation order by round-to-nearest ops, so the CPU oracle makes the same
// decisions bit for bit.
//
// The forward saves per pixel the final transmittance and last_idx = 1 + index
// (within the tile list) of the last visible splat, so the backward starts from
// the exact per-pixel state without recompositing.
//
// Work split. Most tiles carry short lists (c3: 6 pairs on average), where a
// CTA per tile is dominated by barriers and per-splat overheads. Tiles with at
// most kShortMax pairs are processed by ONE WARP each (8 pixels per lane, the
// column's dx terms shared by the lane's 8 rows, backward gradients summed over
// the lane's pixels before a single warp reduction). Longer lists are appended
// to a device list and processed by a CTA per tile (one pixel per thread), so a
// hot tile is spread over 8 warps. Both kernels are persistent grids.
#include "gsb_common.cuh"
#include "gsb_host.cuh"

namespace gsb {
namespace {

constexpr int kShortMax = 64;   // pairs per tile handled by one warp
constexpr int kWarpBatch = 32;  // records staged per warp round
constexpr int kLanePx = 8;      // pixels per lane in the warp kernels: rows py0 + 2i
constexpr int kWarps = 8;       // warps per CTA
constexpr int kBatch = 256;     // records staged per CTA round (long kernels)
constexpr int kGradComps = 9;

struct TileCoord {
  int b, tx, ty;
};

__device__ __forceinline__ TileCoord tile_coord(const Meta& m, int tile) {
  TileCoord c;
  c.b = tile / m.tiles_per_image;
  const int local = tile - c.b * m.tiles_per_image;
  c.ty = local / m.tiles_x;
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

__device__ __forceinline__ void load_rec(const float4* __restrict__ rec, int gi, float4* dst) {
  if (gi >= 0) {
    dst[0] = __ldg(&rec[3 * gi + 0]);
    dst[1] = __ldg(&rec[3 * gi + 1]);
    dst[2] = __ldg(&rec[3 * gi + 2]);
  } else {  // bad index: a record that is never visible
    const float inf = __int_as_float(0x7f800000);
    dst[0] = make_float4(0.f, 0.f, 0.f, 0.f);
    dst[1] = make_float4(0.f, 0.f, 0.f, 0.f);
    dst[2] = make_float4(0.f, 0.f, inf, inf);
  }
}

// Warp-wide sum of v[0..15]; on return lane L holds the total of v[L >> 1] in
// v[0] (recursive halving: 16 shuffles instead of 5 per value).
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

// ---------------------------------------------------------------------------
// Forward
// ---------------------------------------------------------------------------
template <bool kSave>
__global__ void __launch_bounds__(kWarps * 32, 3)
    k_render_fwd_warp(Meta m, const float4* __restrict__ rec, const int32_t* __restrict__ toff,
                      const int32_t* __restrict__ ids, float* __restrict__ out, float* __restrict__ final_T,
                      int32_t* __restrict__ last_idx, int32_t* __restrict__ long_tiles,
                      uint32_t* __restrict__ long_count, uint32_t* __restrict__ status) {
  __shared__ float4 s_rec[kWarps][kWarpBatch][3];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  float4(*my)[3] = s_rec[warp];
  const int stride = gridDim.x * kWarps;
  for (int tile = blockIdx.x * kWarps + warp; tile < m.total_tiles; tile += stride) {
    const int start = __ldg(&toff[tile]);
    const int n = __ldg(&toff[tile + 1]) - start;
    if (n > kShortMax) {
      if (lane == 0) long_tiles[atomicAdd(long_count, 1u)] = tile;
      continue;
    }
    const TileCoord tc = tile_coord(m, tile);
    const int px = tc.tx * kTile + (lane & 15);
    const int py0 = tc.ty * kTile + (lane >> 4);
    const float fx = (float)px + 0.5f;
    const float fy0 = (float)py0 + 0.5f;  // row i is at fy0 + 2i (exact)
    float T[kLanePx], cr[kLanePx], cg[kLanePx], cb[kLanePx];
    uint32_t last4[2] = {0u, 0u};  // last_idx of pixel i in byte i&3 of last4[i>>2] (n <= kShortMax < 256)
    uint32_t alive = 0;
#pragma unroll
    for (int i = 0; i < kLanePx; ++i) {
      T[i] = 1.0f;
      cr[i] = cg[i] = cb[i] = 0.0f;
      if (px < m.W && py0 + 2 * i < m.H && 1.0f > m.T_thr) alive |= 1u << i;
    }
    for (int base = 0; base < n; base += kWarpBatch) {
      if (!__any_sync(kFullMask, alive)) break;
      const int cnt = min(kWarpBatch, n - base);
      __syncwarp();
      if (lane < cnt) load_rec(rec, load_gi(ids, start + base + lane, m.BG, status, kSiteRender), my[lane]);
      __syncwarp();
      if (alive) {
        for (int j = 0; j < cnt; ++j) {
          const float4 p0 = my[j][0];
          const float4 p1 = my[j][1];
          const float4 p2 = my[j][2];
          const float dx = __fsub_rn(fx, p0.x);
          const float ta = __fmul_rn(__fmul_rn(p0.z, dx), dx);
          const float tb = __fmul_rn(__fmul_rn(2.0f, p0.w), dx);
#pragma unroll
          for (int i = 0; i < kLanePx; ++i) {
            const float power = power_rn(ta, tb, p1.x, __fsub_rn(fy0 + (float)(2 * i), p0.y));
            if (((alive >> i) & 1u) && power <= 0.0f && power >= p2.z) {
              const float alpha = fminf(m.max_alpha, p1.y * __expf(power));
              const float w = T[i] * alpha;
              cr[i] = fmaf(w, p1.z, cr[i]);
              cg[i] = fmaf(w, p1.w, cg[i]);
              cb[i] = fmaf(w, p2.x, cb[i]);
              T[i] *= 1.0f - alpha;
              last4[i >> 2] = (last4[i >> 2] & ~(0xffu << (8 * (i & 3)))) | ((uint32_t)(base + j + 1) << (8 * (i & 3)));
              if (T[i] <= m.T_thr) alive &= ~(1u << i);
            }
          }
        }
      }
    }
    if (px < m.W) {
#pragma unroll
      for (int i = 0; i < kLanePx; ++i) {
        const int py = py0 + 2 * i;
        if (py < m.H) {
          const size_t pix = ((size_t)tc.b * m.H + py) * m.W + px;
          out[3 * pix + 0] = fmaf(T[i], m.bg_r, cr[i]);
          out[3 * pix + 1] = fmaf(T[i], m.bg_g, cg[i]);
          out[3 * pix + 2] = fmaf(T[i], m.bg_b, cb[i]);
          if (kSave) {
            final_T[pix] = T[i];
            last_idx[pix] = (int32_t)((last4[i >> 2] >> (8 * (i & 3))) & 0xffu);
          }
        }
      }
    }
  }
}

// CTA per long tile, one pixel per thread, 256-record shared-memory batches.
template <bool kSave>
__global__ void __launch_bounds__(kTilePixels)
    k_render_fwd_cta(Meta m, const float4* __restrict__ rec, const int32_t* __restrict__ toff,
                     const int32_t* __restrict__ ids, float* __restrict__ out, float* __restrict__ final_T,
                     int32_t* __restrict__ last_idx, const int32_t* __restrict__ long_tiles,
                     const uint32_t* __restrict__ long_count, uint32_t* __restrict__ status) {
  __shared__ float4 s_rec[kBatch][3];
  const uint32_t n_long = *long_count;
  for (uint32_t k = blockIdx.x; k < n_long; k += gridDim.x) {
    const int tile = long_tiles[k];
    const TileCoord tc = tile_coord(m, tile);
    const int px = tc.tx * kTile + (threadIdx.x & 15);
    const int py = tc.ty * kTile + (threadIdx.x >> 4);
    const bool valid = px < m.W && py < m.H;
    const int start = toff[tile];
    const int n = toff[tile + 1] - start;
    const float fx = (float)px + 0.5f, fy = (float)py + 0.5f;
    float T = 1.0f, cr = 0.0f, cg = 0.0f, cb = 0.0f;
    int last = 0;
    bool alive = valid && (T > m.T_thr);
    for (int base = 0; base < n; base += kBatch) {
      if (__syncthreads_count(alive) == 0) break;
      const int cnt = min(kBatch, n - base);
      if ((int)threadIdx.x < cnt)
        load_rec(rec, load_gi(ids, start + base + threadIdx.x, m.BG, status, kSiteRender), s_rec[threadIdx.x]);
      __syncthreads();
      if (alive) {
        for (int j = 0; j < cnt; ++j) {
          const float4 p0 = s_rec[j][0];
          const float4 p1 = s_rec[j][1];
          const float dx = __fsub_rn(fx, p0.x);
          const float power = power_rn(__fmul_rn(__fmul_rn(p0.z, dx), dx), __fmul_rn(__fmul_rn(2.0f, p0.w), dx),
                                       p1.x, __fsub_rn(fy, p0.y));
          const float4 p2 = s_rec[j][2];
          if (!(power <= 0.0f && power >= p2.z)) continue;
          const float alpha = fminf(m.max_alpha, p1.y * __expf(power));
          const float w = T * alpha;
          cr = fmaf(w, p1.z, cr);
          cg = fmaf(w, p1.w, cg);
          cb = fmaf(w, p2.x, cb);
          T *= 1.0f - alpha;
          last = base + j + 1;
          if (T <= m.T_thr) {
            alive = false;
            break;
          }
        }
      }
    }
    if (valid) {
      const size_t pix = ((size_t)tc.b * m.H + py) * m.W + px;
      out[3 * pix + 0] = fmaf(T, m.bg_r, cr);
      out[3 * pix + 1] = fmaf(T, m.bg_g, cg);
      out[3 * pix + 2] = fmaf(T, m.bg_b, cb);
      if (kSave) {
        final_T[pix] = T;
        last_idx[pix] = last;
      }
    }
    __syncthreads();  // s_rec reuse by the next tile
  }
}

// ---------------------------------------------------------------------------
// Backward
// ---------------------------------------------------------------------------

// Per-pixel VJP of one visible splat (…metal:1017-1034). Adds the pixel's 9
// partials to v and advances the reverse recurrence (T_cur, gT).
__device__ __forceinline__ void pixel_vjp(const Meta& m, float dx, float dy, float power, const float4& p0,
                                          const float4& p1, const float4& p2, float gr, float gg, float gb,
                                          float& T_cur, float& gT, float* v) {
  const float e = __expf(power);
  const float raw = p1.y * e;
  const float alpha = fminf(m.max_alpha, raw);
  const float T_prev = __fdividef(T_cur, fmaxf(1.0f - alpha, m.eps));
  const float dot_gc = gr * p1.z + gg * p1.w + gb * p2.x;
  const float g_alpha = T_prev * (dot_gc - gT);
  const float wc = T_prev * alpha;
  const float g_raw = (power < p2.w) ? g_alpha : 0.0f;  // raw < max_alpha
  const float g_power = g_raw * raw;
  const float a = p0.z, b = p0.w, c = p1.x;
  v[0] += g_power * (a * dx + b * dy);
  v[1] += g_power * (b * dx + c * dy);
  v[2] += g_power * (-0.5f) * dx * dx;
  v[3] += g_power * (-1.0f) * dx * dy;
  v[4] += g_power * (-0.5f) * dy * dy;
  v[5] += g_raw * __fdividef(raw, fmaxf(p1.y, m.eps));
  v[6] += gr * wc;
  v[7] += gg * wc;
  v[8] += gb * wc;
  gT = alpha * dot_gc + (1.0f - alpha) * gT;
  T_cur = T_prev;
}

__global__ void __launch_bounds__(kWarps * 32, 2)
    k_render_bwd_warp(Meta m, const float4* __restrict__ rec, const int32_t* __restrict__ toff,
                      const int32_t* __restrict__ ids, const float* __restrict__ final_T,
                      const int32_t* __restrict__ last_idx, const float* __restrict__ grad,
                      float* __restrict__ grad_rec, int32_t* __restrict__ long_tiles,
                      uint32_t* __restrict__ long_count, uint32_t* __restrict__ status) {
  __shared__ float4 s_rec[kWarps][kWarpBatch][3];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  float4(*my)[3] = s_rec[warp];
  const int stride = gridDim.x * kWarps;
  for (int tile = blockIdx.x * kWarps + warp; tile < m.total_tiles; tile += stride) {
    const int start = __ldg(&toff[tile]);
    const int n = __ldg(&toff[tile + 1]) - start;
    if (n > kShortMax) {
      if (lane == 0) long_tiles[atomicAdd(long_count, 1u)] = tile;
      continue;
    }
    if (n == 0) continue;
    const TileCoord tc = tile_coord(m, tile);
    const int px = tc.tx * kTile + (lane & 15);
    const int py0 = tc.ty * kTile + (lane >> 4);
    const float fx = (float)px + 0.5f;
    const float fy0 = (float)py0 + 0.5f;
    float gr[kLanePx], gg[kLanePx], gb[kLanePx], Tc[kLanePx], gT[kLanePx];
    int last[kLanePx];
    int lmax = 0;
#pragma unroll
    for (int i = 0; i < kLanePx; ++i) {
      const int py = py0 + 2 * i;
      gr[i] = gg[i] = gb[i] = 0.0f;
      Tc[i] = 1.0f;
      last[i] = 0;
      if (px < m.W && py < m.H) {
        const size_t pix = ((size_t)tc.b * m.H + py) * m.W + px;
        gr[i] = grad[3 * pix + 0];
        gg[i] = grad[3 * pix + 1];
        gb[i] = grad[3 * pix + 2];
        Tc[i] = final_T[pix];
        last[i] = min(last_idx[pix], n);
      }
      gT[i] = gr[i] * m.bg_r + gg[i] * m.bg_g + gb[i] * m.bg_b;
      lmax = max(lmax, last[i]);
    }
    const int tile_last = __reduce_max_sync(kFullMask, lmax);
    for (int bend = tile_last; bend > 0; bend -= kWarpBatch) {
      const int bstart = max(0, bend - kWarpBatch);
      const int cnt = bend - bstart;
      __syncwarp();
      int my_gi = -1;
      if (lane < cnt) {
        my_gi = load_gi(ids, start + bstart + lane, m.BG, status, kSiteRenderBwd);
        load_rec(rec, my_gi, my[lane]);
      }
      __syncwarp();
      for (int jj = cnt - 1; jj >= 0; --jj) {
        const int j = bstart + jj;
        const float4 p0 = my[jj][0];
        const float4 p1 = my[jj][1];
        const float4 p2 = my[jj][2];
        const float dx = __fsub_rn(fx, p0.x);
        const float ta = __fmul_rn(__fmul_rn(p0.z, dx), dx);
        const float tb = __fmul_rn(__fmul_rn(2.0f, p0.w), dx);
        float v[16];
#pragma unroll
        for (int q = 0; q < 16; ++q) v[q] = 0.0f;
        bool any = false;
#pragma unroll
        for (int i = 0; i < kLanePx; ++i) {
          if (j < last[i]) {
            const float dy = __fsub_rn(fy0 + (float)(2 * i), p0.y);
            const float power = power_rn(ta, tb, p1.x, dy);
            if (power <= 0.0f && power >= p2.z) {
              pixel_vjp(m, dx, dy, power, p0, p1, p2, gr[i], gg[i], gb[i], Tc[i], gT[i], v);
              any = true;
            }
          }
        }
        if (__any_sync(kFullMask, any)) {
          const float total = warp_reduce_scatter16(v, lane);
          const int gi = __shfl_sync(kFullMask, my_gi, jj);
          const int comp = lane >> 1;
          if (!(lane & 1) && comp < kGradComps && gi >= 0)
            atomicAdd(grad_rec + (size_t)gi * GSB_REC_FLOATS + comp, total);
        }
      }
    }
  }
}

__global__ void __launch_bounds__(kTilePixels)
    k_render_bwd_cta(Meta m, const float4* __restrict__ rec, const int32_t* __restrict__ toff,
                     const int32_t* __restrict__ ids, const float* __restrict__ final_T,
                     const int32_t* __restrict__ last_idx, const float* __restrict__ grad,
                     float* __restrict__ grad_rec, const int32_t* __restrict__ long_tiles,
                     const uint32_t* __restrict__ long_count, uint32_t* __restrict__ status) {
  __shared__ float4 s_rec[kBatch][3];
  __shared__ int s_gi[kBatch];
  __shared__ float s_acc[kBatch][kGradComps];
  __shared__ int s_max[kWarps];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const uint32_t n_long = *long_count;
  for (uint32_t k = blockIdx.x; k < n_long; k += gridDim.x) {
    const int tile = long_tiles[k];
    const TileCoord tc = tile_coord(m, tile);
    const int px = tc.tx * kTile + (threadIdx.x & 15);
    const int py = tc.ty * kTile + (threadIdx.x >> 4);
    const bool valid = px < m.W && py < m.H;
    const int start = toff[tile];
    const int n = toff[tile + 1] - start;
    float gr = 0.f, gg = 0.f, gb = 0.f, T_cur = 1.0f;
    int last = 0;
    if (valid) {
      const size_t pix = ((size_t)tc.b * m.H + py) * m.W + px;
      gr = grad[3 * pix + 0];
      gg = grad[3 * pix + 1];
      gb = grad[3 * pix + 2];
      T_cur = final_T[pix];
      last = min(last_idx[pix], n);
    }
    float gT = gr * m.bg_r + gg * m.bg_g + gb * m.bg_b;
    const float fx = (float)px + 0.5f, fy = (float)py + 0.5f;
    const int wmax = __reduce_max_sync(kFullMask, last);
    if (lane == 0) s_max[warp] = wmax;
    __syncthreads();
    int tile_last = 0;
#pragma unroll
    for (int w = 0; w < kWarps; ++w) tile_last = max(tile_last, s_max[w]);

    for (int bend = tile_last; bend > 0; bend -= kBatch) {
      const int bstart = max(0, bend - kBatch);
      const int cnt = bend - bstart;
      if ((int)threadIdx.x < cnt) {
        const int gi = load_gi(ids, start + bstart + threadIdx.x, m.BG, status, kSiteRenderBwd);
        s_gi[threadIdx.x] = gi;
        load_rec(rec, gi, s_rec[threadIdx.x]);
      }
      for (int i = threadIdx.x; i < cnt * kGradComps; i += kTilePixels) (&s_acc[0][0])[i] = 0.0f;
      __syncthreads();
      for (int jj = cnt - 1; jj >= 0; --jj) {
        const int j = bstart + jj;
        float v[16];
#pragma unroll
        for (int q = 0; q < 16; ++q) v[q] = 0.0f;
        bool any = false;
        if (j < last) {
          const float4 p0 = s_rec[jj][0];
          const float4 p1 = s_rec[jj][1];
          const float dx = __fsub_rn(fx, p0.x);
          const float dy = __fsub_rn(fy, p0.y);
          const float power = power_rn(__fmul_rn(__fmul_rn(p0.z, dx), dx), __fmul_rn(__fmul_rn(2.0f, p0.w), dx),
                                       p1.x, dy);
          const float4 p2 = s_rec[jj][2];
          if (power <= 0.0f && power >= p2.z) {
            pixel_vjp(m, dx, dy, power, p0, p1, p2, gr, gg, gb, T_cur, gT, v);
            any = true;
          }
        }
        if (__any_sync(kFullMask, any)) {
          const float total = warp_reduce_scatter16(v, lane);
          const int comp = lane >> 1;
          if (!(lane & 1) && comp < kGradComps) atomicAdd(&s_acc[jj][comp], total);
        }
      }
      __syncthreads();
      if ((int)threadIdx.x < cnt) {
        const int s = threadIdx.x;
        const int gi = s_gi[s];
        float acc[kGradComps];
        bool nz = false;
#pragma unroll
        for (int q = 0; q < kGradComps; ++q) {
          acc[q] = s_acc[s][q];
          nz |= (acc[q] != 0.0f);
        }
        if (nz && gi >= 0) {
          float4* g4 = reinterpret_cast<float4*>(grad_rec + (size_t)gi * GSB_REC_FLOATS);
          atomicAdd(g4 + 0, make_float4(acc[0], acc[1], acc[2], acc[3]));
          atomicAdd(g4 + 1, make_float4(acc[4], acc[5], acc[6], acc[7]));
          atomicAdd(grad_rec + (size_t)gi * GSB_REC_FLOATS + 8, acc[8]);
        }
      }
      __syncthreads();
    }
  }
}

// grad_rec (depth-rank order, packed) -> user layout in input order.
__global__ void __launch_bounds__(256)
    k_unsort(Meta m, const int32_t* __restrict__ perm, const float4* __restrict__ grad_rec,
             float* __restrict__ g_means2d, float* __restrict__ g_conics, float* __restrict__ g_colors,
             float* __restrict__ g_opac) {
  const int r = blockIdx.x * blockDim.x + threadIdx.x;
  if (r >= m.BG) return;
  const int b = r / m.G;
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

// Persistent grid sizes (CTAs resident per SM x SMs), cached per device.
struct GridCache {
  int sms = 0;
  int fwd_warp[2] = {0, 0}, fwd_cta[2] = {0, 0}, bwd_warp = 0, bwd_cta = 0;
};

const GridCache& grids() {
  static GridCache cache[64];
  int dev = 0;
  cudaGetDevice(&dev);
  GridCache& g = cache[dev & 63];
  if (g.sms == 0) {
    int sms = 148;
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    auto occ = [&](const void* fn, int threads) {
      int b = 1;
      if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&b, fn, threads, 0) != cudaSuccess || b < 1) b = 1;
      return b * sms;
    };
    g.fwd_warp[0] = occ((const void*)k_render_fwd_warp<false>, kWarps * 32);
    g.fwd_warp[1] = occ((const void*)k_render_fwd_warp<true>, kWarps * 32);
    g.fwd_cta[0] = occ((const void*)k_render_fwd_cta<false>, kTilePixels);
    g.fwd_cta[1] = occ((const void*)k_render_fwd_cta<true>, kTilePixels);
    g.bwd_warp = occ((const void*)k_render_bwd_warp, kWarps * 32);
    g.bwd_cta = occ((const void*)k_render_bwd_cta, kTilePixels);
    g.sms = sms;
  }
  return g;
}

struct RenderWs {
  uint32_t* long_count;
  int32_t* long_tiles;
};

void carve_render(Carver& c, const Meta& m, RenderWs* w) {
  w->long_count = c.take<uint32_t>(1);
  w->long_tiles = c.take<int32_t>((size_t)m.total_tiles);
}

}  // namespace
}  // namespace gsb

using namespace gsb;

extern "C" size_t gsb_render_workspace_size(const gsb_raster_meta* meta) {
  Meta m;
  if (make_meta(meta, &m) != GSB_OK) return 0;
  Carver c(nullptr);
  RenderWs w;
  carve_render(c, m, &w);
  return c.off + 256;
}

extern "C" int gsb_render_forward(const gsb_raster_meta* meta, const float* rec, const int32_t* tile_offsets,
                                  const int32_t* binned_ids, float* out_rgb, float* final_T, int32_t* last_idx,
                                  uint32_t* status, void* workspace, size_t workspace_bytes, void* stream_) {
  Meta m;
  int rc = make_meta(meta, &m);
  if (rc != GSB_OK) return rc;
  if (!tile_offsets || !out_rgb || !status) return GSB_ERR_INVALID_ARGUMENT;
  if ((final_T == nullptr) != (last_idx == nullptr)) return GSB_ERR_INVALID_ARGUMENT;
  if (m.BG > 0 && !rec) return GSB_ERR_INVALID_ARGUMENT;
  if (!workspace || workspace_bytes < gsb_render_workspace_size(meta)) return GSB_ERR_WORKSPACE;
  cudaStream_t stream = static_cast<cudaStream_t>(stream_);
  Carver c(workspace);
  RenderWs w;
  carve_render(c, m, &w);
  if (cudaMemsetAsync(w.long_count, 0, sizeof(uint32_t), stream) != cudaSuccess) return GSB_ERR_CUDA;
  const GridCache& g = grids();
  const float4* r4 = reinterpret_cast<const float4*>(rec);
  const int warp_grid = max(1, min(g.fwd_warp[final_T ? 1 : 0], (m.total_tiles + kWarps - 1) / kWarps));
  const int cta_grid = max(1, min(g.fwd_cta[final_T ? 1 : 0], m.total_tiles));
  if (final_T) {
    k_render_fwd_warp<true><<<warp_grid, kWarps * 32, 0, stream>>>(m, r4, tile_offsets, binned_ids, out_rgb,
                                                                   final_T, last_idx, w.long_tiles, w.long_count,
                                                                   status);
    k_render_fwd_cta<true><<<cta_grid, kTilePixels, 0, stream>>>(m, r4, tile_offsets, binned_ids, out_rgb, final_T,
                                                                 last_idx, w.long_tiles, w.long_count, status);
  } else {
    k_render_fwd_warp<false><<<warp_grid, kWarps * 32, 0, stream>>>(m, r4, tile_offsets, binned_ids, out_rgb,
                                                                    nullptr, nullptr, w.long_tiles, w.long_count,
                                                                    status);
    k_render_fwd_cta<false><<<cta_grid, kTilePixels, 0, stream>>>(m, r4, tile_offsets, binned_ids, out_rgb, nullptr,
                                                                  nullptr, w.long_tiles, w.long_count, status);
  }
  note_launches(2);
  return cuda_status(cudaGetLastError());
}

extern "C" int gsb_render_backward(const gsb_raster_meta* meta, const float* rec, const int32_t* tile_offsets,
                                   const int32_t* binned_ids, const float* final_T, const int32_t* last_idx,
                                   const float* grad_rgb, float* grad_rec, uint32_t* status, void* workspace,
                                   size_t workspace_bytes, void* stream_) {
  Meta m;
  int rc = make_meta(meta, &m);
  if (rc != GSB_OK) return rc;
  if (!tile_offsets || !final_T || !last_idx || !grad_rgb || !status) return GSB_ERR_INVALID_ARGUMENT;
  if (m.BG > 0 && (!rec || !grad_rec)) return GSB_ERR_INVALID_ARGUMENT;
  if (!workspace || workspace_bytes < gsb_render_workspace_size(meta)) return GSB_ERR_WORKSPACE;
  cudaStream_t stream = static_cast<cudaStream_t>(stream_);
  if (m.BG > 0) {
    cudaError_t e = cudaMemsetAsync(grad_rec, 0, sizeof(float) * GSB_REC_FLOATS * (size_t)m.BG, stream);
    if (e != cudaSuccess) return GSB_ERR_CUDA;
  }
  Carver c(workspace);
  RenderWs w;
  carve_render(c, m, &w);
  if (cudaMemsetAsync(w.long_count, 0, sizeof(uint32_t), stream) != cudaSuccess) return GSB_ERR_CUDA;
  const GridCache& g = grids();
  const float4* r4 = reinterpret_cast<const float4*>(rec);
  const int warp_grid = max(1, min(g.bwd_warp, (m.total_tiles + kWarps - 1) / kWarps));
  const int cta_grid = max(1, min(g.bwd_cta, m.total_tiles));
  k_render_bwd_warp<<<warp_grid, kWarps * 32, 0, stream>>>(m, r4, tile_offsets, binned_ids, final_T, last_idx,
                                                           grad_rgb, grad_rec, w.long_tiles, w.long_count, status);
  k_render_bwd_cta<<<cta_grid, kTilePixels, 0, stream>>>(m, r4, tile_offsets, binned_ids, final_T, last_idx,
                                                         grad_rgb, grad_rec, w.long_tiles, w.long_count, status);
  note_launches(2);
  return cuda_status(cudaGetLastError());
}

extern "C" int gsb_unsort_grads(const gsb_raster_meta* meta, const int32_t* perm, const float* grad_rec,
                                float* g_means2d, float* g_conics, float* g_colors, float* g_opacities,
                                void* stream_) {
  Meta m;
  int rc = make_meta(meta, &m);
  if (rc != GSB_OK) return rc;
  if (m.BG == 0) return GSB_OK;
  if (!perm || !grad_rec) return GSB_ERR_INVALID_ARGUMENT;
  cudaStream_t stream = static_cast<cudaStream_t>(stream_);
  k_unsort<<<grid1d(m.BG, 256), 256, 0, stream>>>(m, perm, reinterpret_cast<const float4*>(grad_rec), g_means2d,
                                                  g_conics, g_colors, g_opacities);
  note_launches(1);
  return cuda_status(cudaGetLastError());
}
