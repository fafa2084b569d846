/*
 * gsplat_oracle.c — CPU oracle for the B200 rasterizer. TEST INFRASTRUCTURE ONLY:
 * used by tests/, __graft_entry__.smoke() and bench.py's cpu_baseline / --impl
 * reference legs as the checker and the timed CPU baseline. Never linked into,
 * or called by, the product path.
 *
 * A plain-C restatement of the reference rasterizer (nbardy/fast-mac-gsplat), which
 * only exists as Metal compute kernels (no CPU build is possible):
 *   binning      variants/v8_project3d/csrc/metal/gsplat_v8_project3d_kernels.metal:526-572, 697-780
 *   ordering     stable depth argsort (variants/v8_project3d/torch_gsplat_bridge_v8_project3d/rasterize.py:708)
 *                then ascending rank per tile (…kernels.metal:594-617)
 *   forward      tile_fast_forward_state (…kernels.metal:853-929)
 *   backward     tile_fast_backward_saved (…kernels.metal:931-1063), which recomputes T_final
 *   projection   project_pinhole_forward / _backward (…kernels.metal:66-174, 217-501)
 * Compiled with -ffp-contract=off and no fast-math: every float operation of the
 * binning path is one IEEE round-to-nearest op, evaluated left to right as the
 * Metal source reads. tau's log is evaluated in double by det_log below and
 * rounded once to float (the Metal source calls fp32 log; its bits are
 * device-specific, so the restatement fixes a reproducible, more accurate choice).
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#ifdef _OPENMP
#include <omp.h>
#endif

#define TILE 16
#define REC 12

typedef struct orc_meta {
  int32_t height, width, tile_size, batch_size, gaussians_per_batch;
  float alpha_threshold, transmittance_threshold, background[3], eps, max_alpha;
} orc_meta;

typedef struct {
  int H, W, tiles_x, tiles_y, tpi, B, G, BG, total_tiles;
} dims_t;

static dims_t dims_of(const orc_meta* m) {
  dims_t d;
  d.H = m->height;
  d.W = m->width;
  d.tiles_x = (m->width + TILE - 1) / TILE;
  d.tiles_y = (m->height + TILE - 1) / TILE;
  d.tpi = d.tiles_x * d.tiles_y;
  d.B = m->batch_size;
  d.G = m->gaussians_per_batch;
  d.BG = d.B * d.G;
  d.total_tiles = d.tpi * d.B;
  return d;
}

static uint32_t f2u(float f) { uint32_t u; memcpy(&u, &f, 4); return u; }
static float u2f(uint32_t u) { float f; memcpy(&f, &u, 4); return f; }

/* Order-preserving depth key; -0 -> +0 and every NaN -> +qNaN (torch sorts NaN last). */
uint32_t orc_depth_key(float d) {
  uint32_t u = f2u(d);
  if ((u & 0x7fffffffu) == 0u) u = 0u;
  if ((u & 0x7fffffffu) > 0x7f800000u) u = 0x7fc00000u;
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

/* ln(x) for positive normal x from IEEE + - * / only (atanh series after
 * reduction to m in [sqrt(1/2), sqrt(2))). */
double orc_det_log(double x) {
  int64_t bits;
  memcpy(&bits, &x, 8);
  int e = (int)((bits >> 52) & 0x7ff) - 1023;
  int64_t mb = (bits & 0x000fffffffffffffLL) | 0x3ff0000000000000LL;
  double m;
  memcpy(&m, &mb, 8);
  if (m > 1.4142135623730951) {
    m = m * 0.5;
    e += 1;
  }
  const double s = (m - 1.0) / (m + 1.0);
  const double s2 = s * s;
  double p = 0.037037037037037035;
  p = p * s2 + 0.04;
  p = p * s2 + 0.043478260869565216;
  p = p * s2 + 0.047619047619047616;
  p = p * s2 + 0.05263157894736842;
  p = p * s2 + 0.058823529411764705;
  p = p * s2 + 0.06666666666666667;
  p = p * s2 + 0.07692307692307693;
  p = p * s2 + 0.09090909090909091;
  p = p * s2 + 0.1111111111111111;
  p = p * s2 + 0.14285714285714285;
  p = p * s2 + 0.2;
  p = p * s2 + 0.3333333333333333;
  p = p * s2 + 1.0;
  const double lm = (2.0 * s) * p;
  return (double)e * 0.6931471805599453 + lm;
}

/* alpha_support_params (…kernels.metal:530-535). */
static int support_tau(float op, float thr, float eps, float* tau) {
  if (!(op > thr)) return 0;
  const float ratio = fmaxf(thr / fmaxf(op, eps), eps);
  const float t = (float)(-2.0 * orc_det_log((double)ratio));
  *tau = t;
  return isfinite(t) && t > 0.0f;
}

/* Visibility of a splat at a pixel, decided on `power` instead of on the
 * rounded product op*exp(power): alpha = min(max_alpha, op*e^power) >= thr
 * <=> power >= ln(thr/op) (when max_alpha >= thr). The threshold is computed
 * once per splat with det_log and rounded to float, so the decision is the
 * same bit-for-bit wherever it is evaluated. +inf: never visible; -inf: always
 * (op = +inf). */
float orc_vis_log_threshold(float op, float thr, float max_alpha) {
  if (!(op >= thr) || !(max_alpha >= thr)) return INFINITY;
  const double ratio = (double)thr / (double)op;
  if (!(ratio > 0.0)) return -INFINITY;
  return (float)orc_det_log(ratio);
}

/* Saturation gate of the backward (raw < max_alpha) decided as power <
 * ln(max_alpha/op); +inf when op <= 0 (never saturates). */
float orc_sat_log_threshold(float op, float max_alpha) {
  if (!(op > 0.0f)) return INFINITY;
  const double ratio = (double)max_alpha / (double)op;
  if (!(ratio > 0.0)) return -INFINITY;
  return (float)orc_det_log(ratio);
}

/* Gaussian exponent at pixel offset (dx, dy): -0.5 (a dx^2 + 2 b dx dy + c dy^2)
 * (…kernels.metal:587), evaluated as fma(-c/2 dy, dy, fma(-b dx, dy, (-a/2 dx) dx)).
 * Every step is one correctly rounded IEEE op (fmaf is a single rounding), so the
 * value is reproducible bit for bit by any IEEE evaluator of the same sequence. */
float orc_power(float a, float b, float c, float dx, float dy) {
  const float ta = ((-0.5f * a) * dx) * dx;
  const float tb = (-b) * dx;
  const float cd = (-0.5f * c) * dy;
  return fmaf(cd, dy, fmaf(tb, dy, ta));
}

static int clamp_f2i(float x) {
  x = fminf(fmaxf(x, -1073741824.0f), 1073741824.0f);
  return (int)x;
}
static int imax(int a, int b) { return a > b ? a : b; }
static int imin(int a, int b) { return a < b ? a : b; }

static float quad_form(float a, float b, float c, float dx, float dy) {
  return a * dx * dx + 2.0f * b * dx * dy + c * dy * dy;
}

/* ellipse_intersects_rect (…kernels.metal:548-572). */
static int ellipse_rect(float mx, float my, float a, float b, float c, float tau, float rx0, float ry0,
                        float rx1, float ry1) {
  const float dx0 = rx0 - mx, dx1 = rx1 - mx, dy0 = ry0 - my, dy1 = ry1 - my;
  if (mx >= rx0 && mx <= rx1 && my >= ry0 && my <= ry1) return 1;
  float qmin = INFINITY;
  qmin = fminf(qmin, quad_form(a, b, c, dx0, dy0));
  qmin = fminf(qmin, quad_form(a, b, c, dx0, dy1));
  qmin = fminf(qmin, quad_form(a, b, c, dx1, dy0));
  qmin = fminf(qmin, quad_form(a, b, c, dx1, dy1));
  if (c > 1e-8f) {
    float dy = fminf(fmaxf(-(b / c) * dx0, dy0), dy1);
    qmin = fminf(qmin, quad_form(a, b, c, dx0, dy));
    dy = fminf(fmaxf(-(b / c) * dx1, dy0), dy1);
    qmin = fminf(qmin, quad_form(a, b, c, dx1, dy));
  }
  if (a > 1e-8f) {
    float dx = fminf(fmaxf(-(b / a) * dy0, dx0), dx1);
    qmin = fminf(qmin, quad_form(a, b, c, dx, dy0));
    dx = fminf(fmaxf(-(b / a) * dy1, dx0), dx1);
    qmin = fminf(qmin, quad_form(a, b, c, dx, dy1));
  }
  return qmin <= tau;
}

/* count_tiles / emit_binned_ids loop (…kernels.metal:707-741, 752-779). Writes
 * up to `cap` local tile ids (ty*tiles_x+tx) into out (if non-NULL); returns the count. */
static int splat_tiles(const dims_t* d, const orc_meta* m, float mx, float my, float a, float b, float c,
                       float op, int32_t* out, int cap) {
  float tau;
  if (!support_tau(op, m->alpha_threshold, m->eps, &tau)) return 0;
  const float det = fmaxf(a * c - b * b, m->eps);
  const float hx = sqrtf(fmaxf(tau * c / det, 0.0f));
  const float hy = sqrtf(fmaxf(tau * a / det, 0.0f));
  const int x0 = imax(0, clamp_f2i(floorf(mx - hx - 0.5f)));
  const int x1 = imin(d->W - 1, clamp_f2i(ceilf(mx + hx - 0.5f)));
  const int y0 = imax(0, clamp_f2i(floorf(my - hy - 0.5f)));
  const int y1 = imin(d->H - 1, clamp_f2i(ceilf(my + hy - 0.5f)));
  if (x0 > x1 || y0 > y1) return 0;
  int n = 0;
  for (int ty = y0 / TILE; ty <= y1 / TILE; ++ty) {
    const float ry0 = (float)(ty * TILE) + 0.5f;
    const float ry1 = fminf((float)(d->H - 1) + 0.5f, (float)((ty + 1) * TILE - 1) + 0.5f);
    for (int tx = x0 / TILE; tx <= x1 / TILE; ++tx) {
      const float rx0 = (float)(tx * TILE) + 0.5f;
      const float rx1 = fminf((float)(d->W - 1) + 0.5f, (float)((tx + 1) * TILE - 1) + 0.5f);
      if (ellipse_rect(mx, my, a, b, c, tau, rx0, ry0, rx1, ry1)) {
        if (out && n < cap) out[n] = ty * d->tiles_x + tx;
        ++n;
      }
    }
  }
  return n;
}

typedef struct {
  uint32_t key;
  int32_t idx;
} kv32_t;

static int cmp_kv32(const void* x, const void* y) {
  const kv32_t* a = (const kv32_t*)x;
  const kv32_t* b = (const kv32_t*)y;
  if (a->key != b->key) return a->key < b->key ? -1 : 1;
  return a->idx < b->idx ? -1 : (a->idx > b->idx);
}

/* Phase 1: stable per-view depth argsort, gather into records, per-splat tile
 * counts in rank order, exclusive scan. Returns the total pair count. */
int64_t orc_bin_prepare(const orc_meta* m, const float* means2d, const float* conics, const float* colors,
                        const float* opacities, const float* depths, int32_t* perm, float* rec,
                        int32_t* pair_offsets) {
  const dims_t d = dims_of(m);
  kv32_t* kv = (kv32_t*)malloc(sizeof(kv32_t) * (size_t)(d.G > 0 ? d.G : 1));
  int32_t* cnt = (int32_t*)malloc(sizeof(int32_t) * (size_t)(d.BG > 0 ? d.BG : 1));
  for (int b = 0; b < d.B; ++b) {
    for (int g = 0; g < d.G; ++g) {
      kv[g].key = orc_depth_key(depths[b * d.G + g]);
      kv[g].idx = g;
    }
    qsort(kv, (size_t)d.G, sizeof(kv32_t), cmp_kv32);
    for (int r = 0; r < d.G; ++r) {
      const int o = b * d.G + kv[r].idx;
      const int64_t gi = (int64_t)b * d.G + r;
      perm[gi] = kv[r].idx;
      float* R = rec + gi * REC;
      R[0] = means2d[2 * o + 0];
      R[1] = means2d[2 * o + 1];
      R[2] = conics[3 * o + 0];
      R[3] = conics[3 * o + 1];
      R[4] = conics[3 * o + 2];
      R[5] = opacities[o];
      R[6] = colors[3 * o + 0];
      R[7] = colors[3 * o + 1];
      R[8] = colors[3 * o + 2];
      R[9] = u2f(kv[r].key);
      R[10] = orc_vis_log_threshold(opacities[o], m->alpha_threshold, m->max_alpha);
      R[11] = orc_sat_log_threshold(opacities[o], m->max_alpha);
    }
  }
#pragma omp parallel for schedule(dynamic, 256)
  for (int i = 0; i < d.BG; ++i) {
    const float* R = rec + (int64_t)i * REC;
    cnt[i] = splat_tiles(&d, m, R[0], R[1], R[2], R[3], R[4], R[5], NULL, 0);
  }
  int64_t run = 0;
  for (int i = 0; i < d.BG; ++i) {
    pair_offsets[i] = (int32_t)run;
    run += cnt[i];
  }
  pair_offsets[d.BG] = (int32_t)run;
  free(kv);
  free(cnt);
  return run;
}

typedef struct {
  uint64_t key;
  int32_t val;
} kv64_t;

static int cmp_kv64(const void* x, const void* y) {
  const kv64_t* a = (const kv64_t*)x;
  const kv64_t* b = (const kv64_t*)y;
  if (a->key != b->key) return a->key < b->key ? -1 : 1;
  return a->val < b->val ? -1 : (a->val > b->val);
}

/* Phase 2: emit (global_tile<<32 | depth_key, rank) pairs, sort them by
 * (key, rank), and build tile offsets (exclusive prefix of per-tile counts). */
void orc_bin_emit(const orc_meta* m, const float* rec, const int32_t* pair_offsets, int64_t P, uint64_t* keys,
                  int32_t* binned_ids, int32_t* tile_offsets) {
  const dims_t d = dims_of(m);
  kv64_t* kv = (kv64_t*)malloc(sizeof(kv64_t) * (size_t)(P > 0 ? P : 1));
  int64_t* per_tile = (int64_t*)calloc((size_t)d.total_tiles + 1, sizeof(int64_t));
#pragma omp parallel
  {
    int32_t* tiles = (int32_t*)malloc(sizeof(int32_t) * (size_t)d.tpi);
#pragma omp for schedule(dynamic, 256)
    for (int r = 0; r < d.BG; ++r) {
      const float* R = rec + (int64_t)r * REC;
      const int n = splat_tiles(&d, m, R[0], R[1], R[2], R[3], R[4], R[5], tiles, d.tpi);
      const int b = r / d.G;
      const uint32_t dk = f2u(R[9]);
      const int64_t start = pair_offsets[r];
      for (int k = 0; k < n && start + k < pair_offsets[r + 1]; ++k) {
        const uint64_t tile = (uint64_t)b * (uint64_t)d.tpi + (uint64_t)tiles[k];
        kv[start + k].key = (tile << 32) | dk;
        kv[start + k].val = r;
      }
    }
    free(tiles);
  }
  qsort(kv, (size_t)P, sizeof(kv64_t), cmp_kv64);
  for (int64_t i = 0; i < P; ++i) {
    keys[i] = kv[i].key;
    binned_ids[i] = kv[i].val;
    per_tile[kv[i].key >> 32] += 1;
  }
  int64_t run = 0;
  for (int t = 0; t < d.total_tiles; ++t) {
    tile_offsets[t] = (int32_t)run;
    run += per_tile[t];
  }
  tile_offsets[d.total_tiles] = (int32_t)run;
  free(kv);
  free(per_tile);
}

/* Forward compositing per pixel, in the reference's order and gates. Also
 * reports the saved state: final T and last_idx = the number of list entries
 * the pixel consumed (the reference's per-pixel stop: saturation index + 1, or
 * the tile count when the pixel never saturates). */
void orc_render_forward(const orc_meta* m, const float* rec, const int32_t* tile_offsets, const int32_t* ids,
                        float* out_rgb, float* final_T, int32_t* last_idx) {
  const dims_t d = dims_of(m);
#pragma omp parallel for schedule(dynamic, 4)
  for (int tile = 0; tile < d.total_tiles; ++tile) {
    const int b = tile / d.tpi, local = tile % d.tpi;
    const int ty = local / d.tiles_x, tx = local % d.tiles_x;
    const int start = tile_offsets[tile], n = tile_offsets[tile + 1] - start;
    for (int py = ty * TILE; py < imin(ty * TILE + TILE, d.H); ++py) {
      for (int px = tx * TILE; px < imin(tx * TILE + TILE, d.W); ++px) {
        const float fx = (float)px + 0.5f, fy = (float)py + 0.5f;
        float T = 1.0f, cr = 0.0f, cg = 0.0f, cb = 0.0f;
        int last = 0; /* entries consumed: n, or the saturation index + 1 */
        if (T > m->transmittance_threshold) {
          last = n;
          for (int j = 0; j < n; ++j) {
            const float* R = rec + (int64_t)ids[start + j] * REC;
            const float dx = fx - R[0], dy = fy - R[1];
            const float power = orc_power(R[2], R[3], R[4], dx, dy);
            if (!(power <= 0.0f && power >= R[10])) continue; /* eval_alpha gate, see orc_vis_log_threshold */
            const float alpha = fminf(m->max_alpha, R[5] * expf(power));
            const float w = T * alpha;
            cr += w * R[6];
            cg += w * R[7];
            cb += w * R[8];
            T *= (1.0f - alpha);
            if (T <= m->transmittance_threshold) {
              last = j + 1;
              break;
            }
          }
        }
        const int64_t pix = ((int64_t)b * d.H + py) * d.W + px;
        out_rgb[3 * pix + 0] = cr + T * m->background[0];
        out_rgb[3 * pix + 1] = cg + T * m->background[1];
        out_rgb[3 * pix + 2] = cb + T * m->background[2];
        if (final_T) final_T[pix] = T;
        if (last_idx) last_idx[pix] = last;
      }
    }
  }
}

/* Backward per pixel as tile_fast_backward_saved: recompute T_final and the
 * stop index by a forward pass, then walk the list in reverse. Accumulates in
 * double into grad_rec [BG*12] (same packed layout as the device). */
void orc_render_backward(const orc_meta* m, const float* rec, const int32_t* tile_offsets, const int32_t* ids,
                         const float* grad_rgb, float* grad_rec) {
  const dims_t d = dims_of(m);
  double* acc = (double*)calloc((size_t)(d.BG > 0 ? d.BG : 1) * 9, sizeof(double));
#pragma omp parallel
  {
    double* loc = (double*)calloc((size_t)(d.BG > 0 ? d.BG : 1) * 9, sizeof(double));
#pragma omp for schedule(dynamic, 4)
    for (int tile = 0; tile < d.total_tiles; ++tile) {
      const int b = tile / d.tpi, local = tile % d.tpi;
      const int ty = local / d.tiles_x, tx = local % d.tiles_x;
      const int start = tile_offsets[tile], n = tile_offsets[tile + 1] - start;
      if (n == 0) continue;
      for (int py = ty * TILE; py < imin(ty * TILE + TILE, d.H); ++py) {
        for (int px = tx * TILE; px < imin(tx * TILE + TILE, d.W); ++px) {
          const float fx = (float)px + 0.5f, fy = (float)py + 0.5f;
          const int64_t pix = ((int64_t)b * d.H + py) * d.W + px;
          const float gr = grad_rgb[3 * pix + 0], gg = grad_rgb[3 * pix + 1], gb = grad_rgb[3 * pix + 2];
          float T_final = 1.0f;
          int end_i = n;
          if (T_final > m->transmittance_threshold) {
            for (int j = 0; j < n; ++j) {
              const float* R = rec + (int64_t)ids[start + j] * REC;
              const float dx = fx - R[0], dy = fy - R[1];
              const float power = orc_power(R[2], R[3], R[4], dx, dy);
              if (!(power <= 0.0f && power >= R[10])) continue;
              const float alpha = fminf(m->max_alpha, R[5] * expf(power));
              T_final *= (1.0f - alpha);
              if (T_final <= m->transmittance_threshold) {
                end_i = j + 1;
                break;
              }
            }
          } else {
            end_i = 0;
          }
          float T_cur = T_final;
          float gT = gr * m->background[0] + gg * m->background[1] + gb * m->background[2];
          for (int j = end_i - 1; j >= 0; --j) {
            const int gi = ids[start + j];
            const float* R = rec + (int64_t)gi * REC;
            const float dx = fx - R[0], dy = fy - R[1];
            const float a = R[2], bq = R[3], c = R[4], op = R[5];
            const float power = orc_power(a, bq, c, dx, dy);
            if (!(power <= 0.0f && power >= R[10])) continue;
            const float raw = op * expf(power);
            const float alpha = fminf(m->max_alpha, raw);
            const float T_prev = T_cur / fmaxf(1.0f - alpha, m->eps);
            const float dot_gc = gr * R[6] + gg * R[7] + gb * R[8];
            const float g_alpha = T_prev * (dot_gc - gT);
            const float wc = T_prev * alpha;
            const float g_raw = (power < R[11]) ? g_alpha : 0.0f; /* raw < max_alpha */
            const float g_power = g_raw * raw;
            double* A = loc + (int64_t)gi * 9;
            A[0] += g_power * (a * dx + bq * dy);
            A[1] += g_power * (bq * dx + c * dy);
            A[2] += g_power * (-0.5f) * dx * dx;
            A[3] += g_power * (-1.0f) * dx * dy;
            A[4] += g_power * (-0.5f) * dy * dy;
            A[5] += g_raw * (raw / fmaxf(op, m->eps));
            A[6] += gr * wc;
            A[7] += gg * wc;
            A[8] += gb * wc;
            gT = alpha * dot_gc + (1.0f - alpha) * gT;
            T_cur = T_prev;
          }
        }
      }
    }
#pragma omp critical
    {
      for (int64_t i = 0; i < (int64_t)d.BG * 9; ++i) acc[i] += loc[i];
    }
    free(loc);
  }
  for (int64_t i = 0; i < d.BG; ++i) {
    for (int q = 0; q < 9; ++q) grad_rec[i * REC + q] = (float)acc[i * 9 + q];
    grad_rec[i * REC + 9] = grad_rec[i * REC + 10] = grad_rec[i * REC + 11] = 0.0f;
  }
  free(acc);
}

/* ---- pinhole projection (…kernels.metal:66-174, 217-501) ----------------- */
typedef struct {
  float r00, r01, r02, r10, r11, r12, r20, r21, r22;
} rot_t;

static rot_t quat_rot(float qr, float qi, float qj, float qk) {
  rot_t g;
  g.r00 = 1.0f - 2.0f * (qj * qj + qk * qk);
  g.r01 = 2.0f * (qi * qj - qr * qk);
  g.r02 = 2.0f * (qi * qk + qr * qj);
  g.r10 = 2.0f * (qi * qj + qr * qk);
  g.r11 = 1.0f - 2.0f * (qi * qi + qk * qk);
  g.r12 = 2.0f * (qj * qk - qr * qi);
  g.r20 = 2.0f * (qi * qk - qr * qj);
  g.r21 = 2.0f * (qj * qk + qr * qi);
  g.r22 = 1.0f - 2.0f * (qi * qi + qj * qj);
  return g;
}

static float symb(const float u[3], const float C[6], const float v[3]) {
  /* C = c00 c01 c02 c11 c12 c22 */
  return u[0] * (C[0] * v[0] + C[1] * v[1] + C[2] * v[2]) + u[1] * (C[1] * v[0] + C[3] * v[1] + C[4] * v[2]) +
         u[2] * (C[2] * v[0] + C[4] * v[1] + C[5] * v[2]);
}

void orc_project_forward(int B, int G, const float* means3d, const float* scales, const float* quats,
                         const float* opacities, const float* c2w, const float* cam, float near_plane,
                         float* out_means2d, float* out_conics, float* out_opac, float* out_depth) {
#pragma omp parallel for schedule(static)
  for (int64_t i = 0; i < (int64_t)B * G; ++i) {
    const int b = (int)(i / G);
    const float* M = c2w + 16 * b;
    const float* K = cam + 4 * b;
    const float sx2 = scales[3 * i] * scales[3 * i], sy2 = scales[3 * i + 1] * scales[3 * i + 1],
                sz2 = scales[3 * i + 2] * scales[3 * i + 2];
    const rot_t g = quat_rot(quats[4 * i], quats[4 * i + 1], quats[4 * i + 2], quats[4 * i + 3]);
    const float C[6] = {
        g.r00 * g.r00 * sx2 + g.r01 * g.r01 * sy2 + g.r02 * g.r02 * sz2,
        g.r00 * g.r10 * sx2 + g.r01 * g.r11 * sy2 + g.r02 * g.r12 * sz2,
        g.r00 * g.r20 * sx2 + g.r01 * g.r21 * sy2 + g.r02 * g.r22 * sz2,
        g.r10 * g.r10 * sx2 + g.r11 * g.r11 * sy2 + g.r12 * g.r12 * sz2,
        g.r10 * g.r20 * sx2 + g.r11 * g.r21 * sy2 + g.r12 * g.r22 * sz2,
        g.r20 * g.r20 * sx2 + g.r21 * g.r21 * sy2 + g.r22 * g.r22 * sz2,
    };
    const float dx = means3d[3 * i] - M[3], dy = means3d[3 * i + 1] - M[7], dz = means3d[3 * i + 2] - M[11];
    const float x = dx * M[0] + dy * M[4] + dz * M[8];
    const float y = dx * M[1] + dy * M[5] + dz * M[9];
    const float z = dx * M[2] + dy * M[6] + dz * M[10];
    const float c0[3] = {M[0], M[4], M[8]}, c1[3] = {M[1], M[5], M[9]}, c2[3] = {M[2], M[6], M[10]};
    const float cc00 = symb(c0, C, c0), cc01 = symb(c0, C, c1), cc02 = symb(c0, C, c2);
    const float cc11 = symb(c1, C, c1), cc12 = symb(c1, C, c2), cc22 = symb(c2, C, c2);
    const int front = z > near_plane;
    const float zs = front ? fmaxf(z, near_plane) : 1.0f;
    const float xp = front ? x : 0.0f, yp = front ? y : 0.0f;
    const float j00 = K[0] / zs, j02 = -(K[0] * xp) / (zs * zs), j11 = K[1] / zs, j12 = -(K[1] * yp) / (zs * zs);
    const float cov00 = j00 * j00 * cc00 + 2.0f * j00 * j02 * cc02 + j02 * j02 * cc22 + 0.3f;
    const float cov01 = j00 * j11 * cc01 + j00 * j12 * cc02 + j02 * j11 * cc12 + j02 * j12 * cc22;
    const float cov11 = j11 * j11 * cc11 + 2.0f * j11 * j12 * cc12 + j12 * j12 * cc22 + 0.3f;
    const float det = fmaxf(cov00 * cov11 - cov01 * cov01, 1e-6f);
    out_means2d[2 * i] = (K[0] * xp) / zs + K[2];
    out_means2d[2 * i + 1] = (K[1] * yp) / zs + K[3];
    out_conics[3 * i] = cov11 / det;
    out_conics[3 * i + 1] = -cov01 / det;
    out_conics[3 * i + 2] = cov00 / det;
    out_opac[i] = front ? opacities[i] : 0.0f;
    out_depth[i] = z;
  }
}
