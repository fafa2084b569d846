// Shared device-side definitions for the sm_100a rasterizer kernels.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include "gsplat_b200.h"

namespace gsb {

constexpr int kTile = 16;          // tile edge in pixels (reference GSP_TILE_SIZE)
constexpr int kTilePixels = 256;   // one thread per pixel of a tile
constexpr uint32_t kFullMask = 0xffffffffu;

// Error-site identifiers written to status[GSB_STATUS_ERROR_SITE].
enum ErrorSite : uint32_t {
  kSiteSortLookback = 1,
  kSiteScanLookback = 2,
  kSiteEmit = 3,
  kSiteRender = 4,
  kSiteRenderBwd = 5,
  kSiteScanTotal = 6,
};

// Raster configuration passed to kernels by value (no device meta tensors, no
// host re-parse of meta tensors per op as in csrc/shared/common.h:28-37).
struct Meta {
  int H, W;
  int tiles_x, tiles_y, tiles_per_image;
  int B, G, BG, total_tiles;
  float alpha_thr, T_thr, bg_r, bg_g, bg_b, eps, max_alpha;
};

__device__ __forceinline__ void raise_error(uint32_t* status, uint32_t flag, uint32_t site) {
  if (status != nullptr) {
    atomicOr(&status[GSB_STATUS_ERROR], flag);
    atomicCAS(&status[GSB_STATUS_ERROR_SITE], 0u, site);
  }
}

__device__ __forceinline__ uint32_t ld_volatile_u32(const uint32_t* p) {
  return *reinterpret_cast<const volatile uint32_t*>(p);
}
__device__ __forceinline__ void st_volatile_u32(uint32_t* p, uint32_t v) {
  *reinterpret_cast<volatile uint32_t*>(p) = v;
}
__device__ __forceinline__ unsigned long long ld_volatile_u64(const unsigned long long* p) {
  return *reinterpret_cast<const volatile unsigned long long*>(p);
}
__device__ __forceinline__ void st_volatile_u64(unsigned long long* p, unsigned long long v) {
  *reinterpret_cast<volatile unsigned long long*>(p) = v;
}

// Bounded spin budget for decoupled look-back waits. A predecessor partition
// always holds a smaller dynamically assigned index, so it is resident and
// finishes without waiting on us; the bound only guards against faults.
constexpr int kSpinLimit = 1 << 22;

// ---------------------------------------------------------------------------
// Order-preserving depth key. Maps a float to a uint32 whose unsigned order is
// the float order torch.argsort uses: -0.0 and +0.0 compare equal (both map to
// the +0.0 key, so the stable sort keeps input order) and every NaN maps to the
// canonical +qNaN key, above +inf (torch sorts NaN last).
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint32_t depth_key(float d) {
  uint32_t u = __float_as_uint(d);
  if ((u & 0x7fffffffu) == 0u) u = 0u;
  if ((u & 0x7fffffffu) > 0x7f800000u) u = 0x7fc00000u;
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

// ---------------------------------------------------------------------------
// Bit-exact binning math. Every float/double operation is an explicit
// round-to-nearest intrinsic, so no FMA contraction or reassociation happens
// and the CPU oracle (compiled with -ffp-contract=off) evaluates the very same
// IEEE operation sequence. Follows
//   variants/v8_project3d/csrc/metal/gsplat_v8_project3d_kernels.metal:526-572.
// ---------------------------------------------------------------------------

// Natural log in double precision from IEEE + - * / only: x = m * 2^e with
// m in [sqrt(1/2), sqrt(2)), ln m = 2 atanh(s), s = (m-1)/(m+1), summed as the
// odd series 2 s sum_k s^(2k)/(2k+1) (|s| <= 0.1716, 13 terms reach double
// rounding). Requires a positive normal x.
__device__ __forceinline__ double det_log(double x) {
  long long bits = __double_as_longlong(x);
  int e = (int)((bits >> 52) & 0x7ff) - 1023;
  double m = __longlong_as_double((bits & 0x000fffffffffffffLL) | 0x3ff0000000000000LL);
  if (m > 1.4142135623730951) {
    m = __dmul_rn(m, 0.5);
    e += 1;
  }
  const double s = __ddiv_rn(__dsub_rn(m, 1.0), __dadd_rn(m, 1.0));
  const double s2 = __dmul_rn(s, s);
  double p = 0.037037037037037035;  // 1/27
  p = __dadd_rn(__dmul_rn(p, s2), 0.04);
  p = __dadd_rn(__dmul_rn(p, s2), 0.043478260869565216);
  p = __dadd_rn(__dmul_rn(p, s2), 0.047619047619047616);
  p = __dadd_rn(__dmul_rn(p, s2), 0.05263157894736842);
  p = __dadd_rn(__dmul_rn(p, s2), 0.058823529411764705);
  p = __dadd_rn(__dmul_rn(p, s2), 0.06666666666666667);
  p = __dadd_rn(__dmul_rn(p, s2), 0.07692307692307693);
  p = __dadd_rn(__dmul_rn(p, s2), 0.09090909090909091);
  p = __dadd_rn(__dmul_rn(p, s2), 0.1111111111111111);
  p = __dadd_rn(__dmul_rn(p, s2), 0.14285714285714285);
  p = __dadd_rn(__dmul_rn(p, s2), 0.2);
  p = __dadd_rn(__dmul_rn(p, s2), 0.3333333333333333);
  p = __dadd_rn(__dmul_rn(p, s2), 1.0);
  const double lm = __dmul_rn(__dmul_rn(2.0, s), p);
  return __dadd_rn(__dmul_rn((double)e, 0.6931471805599453), lm);
}

// alpha_support_params (…metal:530-535): tau = -2 ln(max(thr / max(op, eps), eps)).
// The log is evaluated in double by det_log and rounded once to float.
__device__ __forceinline__ bool support_tau(float opacity, float thr, float eps, float* tau) {
  if (!(opacity > thr)) return false;
  const float ratio = fmaxf(__fdiv_rn(thr, fmaxf(opacity, eps)), eps);
  const float t = __double2float_rn(__dmul_rn(-2.0, det_log((double)ratio)));
  *tau = t;
  return isfinite(t) && (t > 0.0f);
}

// Visibility and saturation thresholds of a splat, in `power` units. A splat is
// visible at a pixel iff power <= 0 && power >= vis (the reference gate
// min(max_alpha, op*exp(power)) >= alpha_thr, …metal:586-591, restated as
// power >= ln(alpha_thr/op)); its alpha saturates iff power >= sat (the
// backward gate raw < max_alpha, …metal:1022, is power < ln(max_alpha/op)).
// Both logs go through det_log, so every evaluator makes identical decisions.
__device__ __forceinline__ float vis_log_threshold(float op, float thr, float max_alpha) {
  if (!(op >= thr) || !(max_alpha >= thr)) return __int_as_float(0x7f800000);
  const double ratio = __ddiv_rn((double)thr, (double)op);
  if (!(ratio > 0.0)) return __int_as_float(0xff800000);
  return __double2float_rn(det_log(ratio));
}
__device__ __forceinline__ float sat_log_threshold(float op, float max_alpha) {
  if (!(op > 0.0f)) return __int_as_float(0x7f800000);
  const double ratio = __ddiv_rn((double)max_alpha, (double)op);
  if (!(ratio > 0.0)) return __int_as_float(0xff800000);
  return __double2float_rn(det_log(ratio));
}

// Gaussian exponent -0.5 (a dx^2 + 2 b dx dy + c dy^2) (…metal:587), evaluated as
// fma(ch dy, dy, fma(tb, dy, ta)) with ta = ((-a/2) dx) dx, tb = (-b) dx,
// ch = -c/2. Each step is one correctly rounded IEEE operation, matching the CPU
// oracle bit for bit. ta and tb are shared by every pixel of a column.
struct PowerCol {
  float ta, tb, ch;
};
__device__ __forceinline__ PowerCol power_col(float a, float b, float c, float dx) {
  PowerCol p;
  p.ta = __fmul_rn(__fmul_rn(__fmul_rn(-0.5f, a), dx), dx);
  p.tb = __fmul_rn(-b, dx);
  p.ch = __fmul_rn(-0.5f, c);
  return p;
}
__device__ __forceinline__ float power_at(const PowerCol& p, float dy) {
  return __fmaf_rn(__fmul_rn(p.ch, dy), dy, __fmaf_rn(p.tb, dy, p.ta));
}

// cp.async (LDGSTS) helpers: asynchronous global -> shared copies, tracked per
// thread in commit groups.
__device__ __forceinline__ void cp_async4(void* smem, const void* gmem) {
  const unsigned s = (unsigned)__cvta_generic_to_shared(smem);
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4;\n" ::"r"(s), "l"(gmem) : "memory");
}
__device__ __forceinline__ void cp_async16(void* smem, const void* gmem) {
  const unsigned s = (unsigned)__cvta_generic_to_shared(smem);
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;\n" ::"r"(s), "l"(gmem) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;\n" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;\n" ::"n"(N) : "memory");
}

// float -> int after clamping into int range (the clamp keeps NaN/huge means
// deterministic; every in-range value converts exactly as int(x) would).
__device__ __forceinline__ int clamp_f2i(float x) {
  x = fminf(fmaxf(x, -1073741824.0f), 1073741824.0f);
  return (int)x;
}

struct PixBox {
  int x0, y0, x1, y1;
};

// snugbox (…metal:537-546).
__device__ __forceinline__ PixBox snugbox(float mx, float my, float a, float b, float c, float tau,
                                          int W, int H, float eps) {
  const float det = fmaxf(__fsub_rn(__fmul_rn(a, c), __fmul_rn(b, b)), eps);
  const float hx = __fsqrt_rn(fmaxf(__fdiv_rn(__fmul_rn(tau, c), det), 0.0f));
  const float hy = __fsqrt_rn(fmaxf(__fdiv_rn(__fmul_rn(tau, a), det), 0.0f));
  PixBox r;
  r.x0 = max(0, clamp_f2i(floorf(__fsub_rn(__fsub_rn(mx, hx), 0.5f))));
  r.x1 = min(W - 1, clamp_f2i(ceilf(__fsub_rn(__fadd_rn(mx, hx), 0.5f))));
  r.y0 = max(0, clamp_f2i(floorf(__fsub_rn(__fsub_rn(my, hy), 0.5f))));
  r.y1 = min(H - 1, clamp_f2i(ceilf(__fsub_rn(__fadd_rn(my, hy), 0.5f))));
  return r;
}

// q(dx,dy) = a dx dx + 2 b dx dy + c dy dy, evaluated left to right.
__device__ __forceinline__ float quad_form(float a, float b, float c, float dx, float dy) {
  const float t0 = __fmul_rn(__fmul_rn(a, dx), dx);
  const float t1 = __fmul_rn(__fmul_rn(__fmul_rn(2.0f, b), dx), dy);
  const float t2 = __fmul_rn(__fmul_rn(c, dy), dy);
  return __fadd_rn(__fadd_rn(t0, t1), t2);
}

// ellipse_intersects_rect (…metal:548-572): min of the quadratic form over the
// pixel-centre rectangle (corners + interior edge minima) against tau.
__device__ __forceinline__ bool ellipse_rect(float mx, float my, float a, float b, float c,
                                             float tau, float rx0, float ry0, float rx1,
                                             float ry1) {
  if (mx >= rx0 && mx <= rx1 && my >= ry0 && my <= ry1) return true;
  const float dx0 = __fsub_rn(rx0, mx);
  const float dx1 = __fsub_rn(rx1, mx);
  const float dy0 = __fsub_rn(ry0, my);
  const float dy1 = __fsub_rn(ry1, my);
  float qmin = __int_as_float(0x7f800000);
  qmin = fminf(qmin, quad_form(a, b, c, dx0, dy0));
  qmin = fminf(qmin, quad_form(a, b, c, dx0, dy1));
  qmin = fminf(qmin, quad_form(a, b, c, dx1, dy0));
  qmin = fminf(qmin, quad_form(a, b, c, dx1, dy1));
  if (c > 1e-8f) {
    const float k = -__fdiv_rn(b, c);
    float dy = fminf(fmaxf(__fmul_rn(k, dx0), dy0), dy1);
    qmin = fminf(qmin, quad_form(a, b, c, dx0, dy));
    dy = fminf(fmaxf(__fmul_rn(k, dx1), dy0), dy1);
    qmin = fminf(qmin, quad_form(a, b, c, dx1, dy));
  }
  if (a > 1e-8f) {
    const float k = -__fdiv_rn(b, a);
    float dx = fminf(fmaxf(__fmul_rn(k, dy0), dx0), dx1);
    qmin = fminf(qmin, quad_form(a, b, c, dx, dy0));
    dx = fminf(fmaxf(__fmul_rn(k, dy1), dx0), dx1);
    qmin = fminf(qmin, quad_form(a, b, c, dx, dy1));
  }
  return qmin <= tau;
}

// Pixel-centre rectangle of tile (tx, ty), clipped to the image (…metal:729-733).
__device__ __forceinline__ float tile_rx0(int tx) { return (float)(tx * kTile) + 0.5f; }
__device__ __forceinline__ float tile_rx1(int tx, int W) {
  return fminf((float)(W - 1) + 0.5f, (float)((tx + 1) * kTile - 1) + 0.5f);
}

// Calls fn(tx, ty) for every tile whose rectangle the splat's support ellipse
// touches, in row-major tile order (the count_tiles/emit_binned_ids loop).
template <typename Fn>
__device__ __forceinline__ void for_each_tile(float mx, float my, float a, float b, float c,
                                              float opacity, const Meta& m, Fn&& fn) {
  float tau;
  if (!support_tau(opacity, m.alpha_thr, m.eps, &tau)) return;
  const PixBox bb = snugbox(mx, my, a, b, c, tau, m.W, m.H, m.eps);
  if (bb.x0 > bb.x1 || bb.y0 > bb.y1) return;
  const int tx0 = bb.x0 / kTile, tx1 = bb.x1 / kTile;
  const int ty0 = bb.y0 / kTile, ty1 = bb.y1 / kTile;
  for (int ty = ty0; ty <= ty1; ++ty) {
    const float ry0 = tile_rx0(ty);
    const float ry1 = tile_rx1(ty, m.H);
    for (int tx = tx0; tx <= tx1; ++tx) {
      if (ellipse_rect(mx, my, a, b, c, tau, tile_rx0(tx), ry0, tile_rx1(tx, m.W), ry1)) fn(tx, ty);
    }
  }
}

}  // namespace gsb
