// Front-to-back compositing (forward) and its reverse-order VJP (backward) on
// 16x16 tiles, one CTA per tile and one thread per pixel.
//
// Reference math: variants/v8_project3d/csrc/metal/gsplat_v8_project3d_kernels.metal
//   eval_alpha 574-592, tile_fast_forward_state 853-929, tile_fast_backward_saved 931-1063.
// Forward contract (docs/v8_critical_theory_notes.md:60-80): a pixel consumes its
// tile list in depth order while T > T_thr; a splat is visible when power <= 0
// and alpha = min(max_alpha, op*exp(power)) >= alpha_thr; C += T*alpha*c;
// T *= 1-alpha; the pixel stops once T <= T_thr.
// Instead of the reference's per-tile stop count the forward saves per pixel
// the final transmittance and last_idx = 1 + index (within the tile list) of the
// last visible splat, so the backward starts from the exact per-pixel state
// without recompositing.
#include "gsb_common.cuh"
#include "gsb_host.cuh"

namespace gsb {
namespace {

constexpr int kBatch = 256;  // splats staged in shared memory per round

struct TilePixel {
  int tile, b, px, py, pix;
  bool valid;
};

__device__ __forceinline__ TilePixel tile_pixel(const Meta& m) {
  TilePixel t;
  t.tile = blockIdx.x;
  t.b = t.tile / m.tiles_per_image;
  const int local = t.tile - t.b * m.tiles_per_image;
  const int ty = local / m.tiles_x;
  const int tx = local - ty * m.tiles_x;
  t.px = tx * kTile + (threadIdx.x & (kTile - 1));
  t.py = ty * kTile + (threadIdx.x >> 4);
  t.valid = t.px < m.W && t.py < m.H;
  t.pix = t.valid ? (t.b * m.H + t.py) * m.W + t.px : 0;
  return t;
}

// Stages splat records rec[ids[lo..lo+cnt)] into shared memory (one record per
// thread, 3 x 16-byte loads, L2-resident after first touch).
__device__ __forceinline__ void stage_batch(const float4* __restrict__ rec, const int32_t* __restrict__ ids,
                                            int lo, int cnt, int BG, float4* s0, float4* s1, float4* s2,
                                            int* s_gi, uint32_t* status, uint32_t site) {
  const int t = threadIdx.x;
  if (t < cnt) {
    int gi = ids[lo + t];
    if ((unsigned)gi >= (unsigned)BG) {
      raise_error(status, GSB_DEVERR_BOUNDS, site);
      gi = -1;
    }
    if (gi >= 0) {
      s0[t] = __ldg(&rec[3 * gi + 0]);
      s1[t] = __ldg(&rec[3 * gi + 1]);
      s2[t] = __ldg(&rec[3 * gi + 2]);
    } else {
      s0[t] = make_float4(0.f, 0.f, 0.f, 0.f);
      s1[t] = make_float4(0.f, 0.f, 0.f, 0.f);  // opacity 0: never visible
      s2[t] = make_float4(0.f, 0.f, 0.f, 0.f);
    }
    if (s_gi) s_gi[t] = gi;
  }
}

template <bool kSaveState>
__global__ void __launch_bounds__(kTilePixels)
    k_render_fwd(Meta m, const float4* __restrict__ rec, const int32_t* __restrict__ tile_offsets,
                 const int32_t* __restrict__ ids, float* __restrict__ out_rgb,
                 float* __restrict__ final_T, int32_t* __restrict__ last_idx,
                 uint32_t* __restrict__ status) {
  __shared__ float4 s0[kBatch], s1[kBatch], s2[kBatch];
  const TilePixel tp = tile_pixel(m);
  const int start = tile_offsets[tp.tile];
  const int n = tile_offsets[tp.tile + 1] - start;
  const float fx = (float)tp.px + 0.5f, fy = (float)tp.py + 0.5f;
  float T = 1.0f, cr = 0.0f, cg = 0.0f, cb = 0.0f;
  int last = 0;
  bool alive = tp.valid && (T > m.T_thr);

  for (int base = 0; base < n; base += kBatch) {
    if (__syncthreads_count(alive) == 0) break;  // whole tile saturated
    const int cnt = min(kBatch, n - base);
    stage_batch(rec, ids, start + base, cnt, m.BG, s0, s1, s2, nullptr, status, kSiteRender);
    __syncthreads();
    if (alive) {
      for (int j = 0; j < cnt; ++j) {
        const float4 p0 = s0[j];
        const float4 p1 = s1[j];
        const float dx = fx - p0.x, dy = fy - p0.y;
        const float power = -0.5f * (p0.z * dx * dx + 2.0f * p0.w * dx * dy + p1.x * dy * dy);
        if (power > 0.0f) continue;
        const float alpha = fminf(m.max_alpha, p1.y * expf(power));
        if (!(alpha >= m.alpha_thr)) continue;
        const float4 p2 = s2[j];
        const float w = T * alpha;
        cr += w * p1.z;
        cg += w * p1.w;
        cb += w * p2.x;
        T *= (1.0f - alpha);
        last = base + j + 1;
        if (T <= m.T_thr) {
          alive = false;
          break;
        }
      }
    }
  }
  if (tp.valid) {
    out_rgb[3 * (size_t)tp.pix + 0] = cr + T * m.bg_r;
    out_rgb[3 * (size_t)tp.pix + 1] = cg + T * m.bg_g;
    out_rgb[3 * (size_t)tp.pix + 2] = cb + T * m.bg_b;
    if (kSaveState) {
      final_T[tp.pix] = T;
      last_idx[tp.pix] = last;
    }
  }
}

constexpr int kGradComps = 9;

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(kFullMask, v, o);
  return v;
}

__global__ void __launch_bounds__(kTilePixels)
    k_render_bwd(Meta m, const float4* __restrict__ rec, const int32_t* __restrict__ tile_offsets,
                 const int32_t* __restrict__ ids, const float* __restrict__ final_T,
                 const int32_t* __restrict__ last_idx, const float* __restrict__ grad_rgb,
                 float* __restrict__ grad_rec, uint32_t* __restrict__ status) {
  __shared__ float4 s0[kBatch], s1[kBatch], s2[kBatch];
  __shared__ int s_gi[kBatch];
  __shared__ float s_acc[kBatch][kGradComps];
  __shared__ int s_max[kTilePixels / 32];

  const TilePixel tp = tile_pixel(m);
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int start = tile_offsets[tp.tile];
  const int n = tile_offsets[tp.tile + 1] - start;

  float gr = 0.f, gg = 0.f, gb = 0.f, T_cur = 1.0f;
  int last = 0;
  if (tp.valid) {
    gr = grad_rgb[3 * (size_t)tp.pix + 0];
    gg = grad_rgb[3 * (size_t)tp.pix + 1];
    gb = grad_rgb[3 * (size_t)tp.pix + 2];
    T_cur = final_T[tp.pix];
    last = min(last_idx[tp.pix], n);
  }
  float gT = gr * m.bg_r + gg * m.bg_g + gb * m.bg_b;
  const float fx = (float)tp.px + 0.5f, fy = (float)tp.py + 0.5f;

  int wmax = __reduce_max_sync(kFullMask, last);
  if (lane == 0) s_max[warp] = wmax;
  __syncthreads();
  int tile_last = 0;
#pragma unroll
  for (int w = 0; w < kTilePixels / 32; ++w) tile_last = max(tile_last, s_max[w]);

  for (int bend = tile_last; bend > 0; bend -= kBatch) {
    const int bstart = max(0, bend - kBatch);
    const int cnt = bend - bstart;
    stage_batch(rec, ids, start + bstart, cnt, m.BG, s0, s1, s2, s_gi, status, kSiteRenderBwd);
    for (int i = threadIdx.x; i < cnt * kGradComps; i += kTilePixels) (&s_acc[0][0])[i] = 0.0f;
    __syncthreads();

    for (int jj = cnt - 1; jj >= 0; --jj) {
      const int j = bstart + jj;
      float v[kGradComps];
#pragma unroll
      for (int q = 0; q < kGradComps; ++q) v[q] = 0.0f;
      bool contrib = false;
      if (j < last) {
        const float4 p0 = s0[jj];
        const float4 p1 = s1[jj];
        const float dx = fx - p0.x, dy = fy - p0.y;
        const float a = p0.z, bq = p0.w, c = p1.x, op = p1.y;
        const float power = -0.5f * (a * dx * dx + 2.0f * bq * dx * dy + c * dy * dy);
        if (power <= 0.0f) {
          const float raw = op * expf(power);
          const float alpha = fminf(m.max_alpha, raw);
          if (alpha >= m.alpha_thr) {
            const float4 p2 = s2[jj];
            const float T_prev = T_cur / fmaxf(1.0f - alpha, m.eps);
            const float dot_gc = gr * p1.z + gg * p1.w + gb * p2.x;
            const float g_alpha = T_prev * (dot_gc - gT);
            const float wc = T_prev * alpha;
            const float g_raw = (raw < m.max_alpha) ? g_alpha : 0.0f;
            const float g_power = g_raw * raw;
            v[0] = g_power * (a * dx + bq * dy);   // d mean_x = -d dx
            v[1] = g_power * (bq * dx + c * dy);   // d mean_y
            v[2] = g_power * (-0.5f) * dx * dx;    // d a
            v[3] = g_power * (-1.0f) * dx * dy;    // d b
            v[4] = g_power * (-0.5f) * dy * dy;    // d c
            v[5] = g_raw * (raw / fmaxf(op, m.eps));  // d opacity
            v[6] = gr * wc;
            v[7] = gg * wc;
            v[8] = gb * wc;
            gT = alpha * dot_gc + (1.0f - alpha) * gT;
            T_cur = T_prev;
            contrib = true;
          }
        }
      }
      if (__any_sync(kFullMask, contrib)) {
#pragma unroll
        for (int q = 0; q < kGradComps; ++q) v[q] = warp_sum(v[q]);
        if (lane == 0) {
#pragma unroll
          for (int q = 0; q < kGradComps; ++q) atomicAdd(&s_acc[jj][q], v[q]);
        }
      }
    }
    __syncthreads();
    // One vector atomic pair + one scalar atomic per (splat, tile).
    if (threadIdx.x < cnt) {
      const int s = threadIdx.x;
      const int gi = s_gi[s];
      float acc[kGradComps];
      bool any = false;
#pragma unroll
      for (int q = 0; q < kGradComps; ++q) {
        acc[q] = s_acc[s][q];
        any |= (acc[q] != 0.0f);
      }
      if (any && gi >= 0) {
        float4* g4 = reinterpret_cast<float4*>(grad_rec + (size_t)gi * GSB_REC_FLOATS);
        atomicAdd(g4 + 0, make_float4(acc[0], acc[1], acc[2], acc[3]));
        atomicAdd(g4 + 1, make_float4(acc[4], acc[5], acc[6], acc[7]));
        atomicAdd(grad_rec + (size_t)gi * GSB_REC_FLOATS + 8, acc[8]);
      }
    }
    __syncthreads();
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

}  // namespace
}  // namespace gsb

using namespace gsb;

extern "C" int gsb_render_forward(const gsb_raster_meta* meta, const float* rec, const int32_t* tile_offsets,
                                  const int32_t* binned_ids, float* out_rgb, float* final_T,
                                  int32_t* last_idx, uint32_t* status, void* stream_) {
  Meta m;
  int rc = make_meta(meta, &m);
  if (rc != GSB_OK) return rc;
  if (!tile_offsets || !out_rgb || !status) return GSB_ERR_INVALID_ARGUMENT;
  if ((final_T == nullptr) != (last_idx == nullptr)) return GSB_ERR_INVALID_ARGUMENT;
  if (m.BG > 0 && !rec) return GSB_ERR_INVALID_ARGUMENT;
  cudaStream_t stream = static_cast<cudaStream_t>(stream_);
  const float4* r4 = reinterpret_cast<const float4*>(rec);
  if (final_T) {
    k_render_fwd<true><<<m.total_tiles, kTilePixels, 0, stream>>>(m, r4, tile_offsets, binned_ids, out_rgb,
                                                                  final_T, last_idx, status);
  } else {
    k_render_fwd<false><<<m.total_tiles, kTilePixels, 0, stream>>>(m, r4, tile_offsets, binned_ids, out_rgb,
                                                                   nullptr, nullptr, status);
  }
  note_launches(1);
  return cuda_status(cudaGetLastError());
}

extern "C" int gsb_render_backward(const gsb_raster_meta* meta, const float* rec, const int32_t* tile_offsets,
                                   const int32_t* binned_ids, const float* final_T, const int32_t* last_idx,
                                   const float* grad_rgb, float* grad_rec, uint32_t* status, void* stream_) {
  Meta m;
  int rc = make_meta(meta, &m);
  if (rc != GSB_OK) return rc;
  if (!tile_offsets || !final_T || !last_idx || !grad_rgb || !status) return GSB_ERR_INVALID_ARGUMENT;
  if (m.BG > 0 && (!rec || !grad_rec)) return GSB_ERR_INVALID_ARGUMENT;
  cudaStream_t stream = static_cast<cudaStream_t>(stream_);
  if (m.BG > 0) {
    cudaError_t e = cudaMemsetAsync(grad_rec, 0, sizeof(float) * GSB_REC_FLOATS * (size_t)m.BG, stream);
    if (e != cudaSuccess) return GSB_ERR_CUDA;
  }
  k_render_bwd<<<m.total_tiles, kTilePixels, 0, stream>>>(m, reinterpret_cast<const float4*>(rec), tile_offsets,
                                                          binned_ids, final_T, last_idx, grad_rgb, grad_rec,
                                                          status);
  note_launches(1);
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
