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
  kSitePeerStart = 7,
  kSitePeerEnd = 8,
};

// Raster configuration passed to kernels by value (no device meta tensors, no
// host re-parse of meta tensors per op as in csrc/shared/common.h:28-37).
// Division of a non-negative int32 n by a run-time invariant d >= 1 without a
// divide instruction: q = (umulhi(n, mul) + n) >> shift, with shift =
// ceil(log2 d) and mul = floor(2^32 (2^shift - d) / d) + 1 (Granlund and
// Montgomery, "Division by invariant integers using multiplication", 1994,
// round-up method; for n < 2^31 the sum stays below 2^32). Set on the host.
struct FastDiv {
  uint32_t mul, shift;
};
__device__ __forceinline__ int fast_div(int n, FastDiv f) {
  return (int)((__umulhi((uint32_t)n, f.mul) + (uint32_t)n) >> f.shift);
}

struct Meta {
  int H, W;
  int tiles_x, tiles_y, tiles_per_image;
  int B, G, BG, total_tiles;
  float alpha_thr, T_thr, bg_r, bg_g, bg_b, eps, max_alpha;
  FastDiv div_tiles_x, div_tiles_per_image, div_G;  // div_G: G, or 1 when G = 0
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

// Packed fp32 pairs for the sm_100 f32x2 instructions: one instruction applies
// the same correctly rounded IEEE operation to both halves (no flush to zero,
// like the scalar __fadd_rn/__fmul_rn/__fmaf_rn), so a packed result equals
// the two scalar results bit for bit while taking one issue slot.
// Programmatic dependent launch (sm_90+). Every kernel of this library is
// launched with programmatic stream serialization (launch_pdl) and begins with
// pdl_wait(): it blocks, in hardware and without spinning, until the preceding
// grid of the stream has completed and its writes are visible, so the kernel
// reads and writes nothing before that. pdl_trigger() then lets the next
// kernel of the stream be scheduled once every CTA of this grid has started,
// which hides the launch latency between the dependent kernels of a step.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

struct F2 {
  unsigned long long v;
};
__device__ __forceinline__ F2 f2(float lo, float hi) {
  F2 r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r.v) : "f"(lo), "f"(hi));
  return r;
}
__device__ __forceinline__ F2 f2(float x) { return f2(x, x); }
__device__ __forceinline__ void split(F2 a, float& lo, float& hi) {
  asm("mov.b64 {%0, %1}, %2;" : "=f"(lo), "=f"(hi) : "l"(a.v));
}
__device__ __forceinline__ F2 add2(F2 a, F2 b) {
  F2 r;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(r.v) : "l"(a.v), "l"(b.v));
  return r;
}
__device__ __forceinline__ F2 sub2(F2 a, F2 b) {
  F2 r;
  asm("sub.rn.f32x2 %0, %1, %2;" : "=l"(r.v) : "l"(a.v), "l"(b.v));
  return r;
}
__device__ __forceinline__ F2 mul2(F2 a, F2 b) {
  F2 r;
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(r.v) : "l"(a.v), "l"(b.v));
  return r;
}
__device__ __forceinline__ F2 fma2(F2 a, F2 b, F2 c) {
  F2 r;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(r.v) : "l"(a.v), "l"(b.v), "l"(c.v));
  return r;
}
// power_at for two rows of one column (same PowerCol, dy = (lo, hi)).
__device__ __forceinline__ F2 power_at2(F2 ta, F2 tb, F2 ch, F2 dy) {
  return fma2(mul2(ch, dy), dy, fma2(tb, dy, ta));
}

// exp(x) = 2^(x log2 e) on the PTX ex2.approx.ftz.f32 instruction (relative
// error about 2^-22 for the arguments met here: x in [ln(alpha_thr/op), 0] for
// a visible splat, so no subnormal results), and 1/x on rcp.approx.ftz.f32.
// Written as bare PTX so the compositing loops stay free of branches.
constexpr float kLog2e = 1.4426950408889634f;
__device__ __forceinline__ float ex2_approx(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}
__device__ __forceinline__ float rcp_approx(float x) {
  float y;
  asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// Branch-free visibility select for the compositing loops, written as one PTX
// block so the compiler cannot turn it into a branch around the exponential
// (the value is computed unconditionally by the caller):
//   live = T > t_thr;  vis = live && power <= 0 && power >= vis_thr
//   returns vis ? value : 0, and sets last = live ? consumed : last.
__device__ __forceinline__ float vis_select_fwd(float T, float t_thr, float power, float vis_thr, float value,
                                                int consumed, int& last) {
  float r;
  asm("{\n\t.reg .pred pl, pv;\n\t"
      "setp.gt.f32 pl, %2, %3;\n\t"
      "setp.le.and.f32 pv, %4, 0f00000000, pl;\n\t"
      "setp.ge.and.f32 pv, %4, %5, pv;\n\t"
      "selp.f32 %0, %6, 0f00000000, pv;\n\t"
      "selp.b32 %1, %7, %1, pl;\n\t}"
      : "=f"(r), "+r"(last)
      : "f"(T), "f"(t_thr), "f"(power), "f"(vis_thr), "f"(value), "r"(consumed));
  return r;
}
// vis_select_fwd that also reports vis (0/1), for the guarded loops below.
__device__ __forceinline__ float vis_select_fwd_v(float T, float t_thr, float power, float vis_thr, float value,
                                                  int consumed, int& last, int& vis) {
  float r;
  asm("{\n\t.reg .pred pl, pv;\n\t"
      "setp.gt.f32 pl, %3, %4;\n\t"
      "setp.le.and.f32 pv, %5, 0f00000000, pl;\n\t"
      "setp.ge.and.f32 pv, %5, %6, pv;\n\t"
      "selp.f32 %0, %7, 0f00000000, pv;\n\t"
      "selp.b32 %1, %8, %1, pl;\n\t"
      "selp.b32 %2, 1, 0, pv;\n\t}"
      : "=f"(r), "+r"(last), "=r"(vis)
      : "f"(T), "f"(t_thr), "f"(power), "f"(vis_thr), "f"(value), "r"(consumed));
  return r;
}

// Non-finite colours. The branch-free loops give a pixel that does not see a
// splat alpha = 0 and still evaluate w*c (forward) and alpha*(<g,c> - gT)
// (backward); with a NaN or infinite colour those products are NaN although
// w or alpha is 0, and the NaN would spread to every pixel of the tile. The
// reference skips such pixels (a per-pixel branch), so a pixel that does not
// see the splat keeps its state. The loops therefore check the colours of each
// staged batch of records (a warp- or CTA-uniform decision) and run a guarded
// form of the body, which selects the updated value only where the splat is
// visible, when one of them is not finite. Finite colours take the unguarded
// body; for them both forms give the same values.
__device__ __forceinline__ bool finite_rgb(float r, float g, float b) {
  return (fabsf(r) <= 3.402823466e38f) & (fabsf(g) <= 3.402823466e38f) & (fabsf(b) <= 3.402823466e38f);
}
// Saturation. alpha = min(max_alpha, op * exp(power)), and the backward passes
// the gradient to op * exp(power) only below max_alpha. A visible splat has
// power <= 0, where ex2.approx returns at most 1 + 2^-22, so a splat with
// op < max_alpha (1 - 2^-20) never reaches max_alpha: for a batch of records
// that all satisfy this (a warp- or CTA-uniform check, like the colour check),
// the loops drop the min and the saturation test (kSat false) with the same
// results bit for bit.
constexpr float kNoSatMargin = 1.0f - 0x1p-20f;
__device__ __forceinline__ bool may_saturate(float op, float max_alpha) { return !(op < max_alpha * kNoSatMargin); }

// Per half: vis ? v : keep.
__device__ __forceinline__ F2 select2(int vis_lo, int vis_hi, F2 v, F2 keep) {
  float vl, vh, kl, kh;
  split(v, vl, vh);
  split(keep, kl, kh);
  return f2(vis_lo ? vl : kl, vis_hi ? vh : kh);
}

// Backward form: vis = j < last && power <= 0 && power >= vis_thr (kCheckLast
// false drops the j < last term, for records every pixel of the warp reaches);
// returns vis ? value : 0, and pass_mask = all ones when vis && power < sat_thr
// else 0 (the caller ANDs it into the bits of a float, a select that also
// clears a NaN). kWantVis also reports vis as 0/1 (the guarded loops).
// kSat false: no record of the batch can saturate (opacity below max_alpha by
// a margin, see kNoSatMargin), so sat_thr > 0 >= power and pass_mask = vis.
template <bool kCheckLast, bool kWantVis, bool kSat = true>
__device__ __forceinline__ float vis_select_bwd(int j, int last, float power, float vis_thr, float sat_thr,
                                                float value, unsigned& pass_mask, int& vis) {
  float r;
  if (!kSat) {
    if (kCheckLast && kWantVis) {
      asm("{\n\t.reg .pred pv;\n\t"
          "setp.lt.s32 pv, %3, %4;\n\t"
          "setp.le.and.f32 pv, %5, 0f00000000, pv;\n\t"
          "setp.ge.and.f32 pv, %5, %6, pv;\n\t"
          "selp.f32 %0, %7, 0f00000000, pv;\n\t"
          "selp.b32 %1, -1, 0, pv;\n\t"
          "selp.b32 %2, 1, 0, pv;\n\t}"
          : "=f"(r), "=r"(pass_mask), "=r"(vis)
          : "r"(j), "r"(last), "f"(power), "f"(vis_thr), "f"(value));
    } else if (kCheckLast) {
      asm("{\n\t.reg .pred pv;\n\t"
          "setp.lt.s32 pv, %2, %3;\n\t"
          "setp.le.and.f32 pv, %4, 0f00000000, pv;\n\t"
          "setp.ge.and.f32 pv, %4, %5, pv;\n\t"
          "selp.f32 %0, %6, 0f00000000, pv;\n\t"
          "selp.b32 %1, -1, 0, pv;\n\t}"
          : "=f"(r), "=r"(pass_mask)
          : "r"(j), "r"(last), "f"(power), "f"(vis_thr), "f"(value));
    } else if (kWantVis) {
      asm("{\n\t.reg .pred pv;\n\t"
          "setp.le.f32 pv, %3, 0f00000000;\n\t"
          "setp.ge.and.f32 pv, %3, %4, pv;\n\t"
          "selp.f32 %0, %5, 0f00000000, pv;\n\t"
          "selp.b32 %1, -1, 0, pv;\n\t"
          "selp.b32 %2, 1, 0, pv;\n\t}"
          : "=f"(r), "=r"(pass_mask), "=r"(vis)
          : "f"(power), "f"(vis_thr), "f"(value));
    } else {
      asm("{\n\t.reg .pred pv;\n\t"
          "setp.le.f32 pv, %2, 0f00000000;\n\t"
          "setp.ge.and.f32 pv, %2, %3, pv;\n\t"
          "selp.f32 %0, %4, 0f00000000, pv;\n\t"
          "selp.b32 %1, -1, 0, pv;\n\t}"
          : "=f"(r), "=r"(pass_mask)
          : "f"(power), "f"(vis_thr), "f"(value));
    }
    (void)sat_thr;
    return r;
  }
  if (kCheckLast && kWantVis) {
    asm("{\n\t.reg .pred pv, ps;\n\t"
        "setp.lt.s32 pv, %3, %4;\n\t"
        "setp.le.and.f32 pv, %5, 0f00000000, pv;\n\t"
        "setp.ge.and.f32 pv, %5, %6, pv;\n\t"
        "setp.lt.and.f32 ps, %5, %7, pv;\n\t"
        "selp.f32 %0, %8, 0f00000000, pv;\n\t"
        "selp.b32 %1, -1, 0, ps;\n\t"
        "selp.b32 %2, 1, 0, pv;\n\t}"
        : "=f"(r), "=r"(pass_mask), "=r"(vis)
        : "r"(j), "r"(last), "f"(power), "f"(vis_thr), "f"(sat_thr), "f"(value));
  } else if (kCheckLast) {
    asm("{\n\t.reg .pred pv, ps;\n\t"
        "setp.lt.s32 pv, %2, %3;\n\t"
        "setp.le.and.f32 pv, %4, 0f00000000, pv;\n\t"
        "setp.ge.and.f32 pv, %4, %5, pv;\n\t"
        "setp.lt.and.f32 ps, %4, %6, pv;\n\t"
        "selp.f32 %0, %7, 0f00000000, pv;\n\t"
        "selp.b32 %1, -1, 0, ps;\n\t}"
        : "=f"(r), "=r"(pass_mask)
        : "r"(j), "r"(last), "f"(power), "f"(vis_thr), "f"(sat_thr), "f"(value));
  } else if (kWantVis) {
    asm("{\n\t.reg .pred pv, ps;\n\t"
        "setp.le.f32 pv, %3, 0f00000000;\n\t"
        "setp.ge.and.f32 pv, %3, %4, pv;\n\t"
        "setp.lt.and.f32 ps, %3, %5, pv;\n\t"
        "selp.f32 %0, %6, 0f00000000, pv;\n\t"
        "selp.b32 %1, -1, 0, ps;\n\t"
        "selp.b32 %2, 1, 0, pv;\n\t}"
        : "=f"(r), "=r"(pass_mask), "=r"(vis)
        : "f"(power), "f"(vis_thr), "f"(sat_thr), "f"(value));
  } else {
    asm("{\n\t.reg .pred pv, ps;\n\t"
        "setp.le.f32 pv, %2, 0f00000000;\n\t"
        "setp.ge.and.f32 pv, %2, %3, pv;\n\t"
        "setp.lt.and.f32 ps, %2, %4, pv;\n\t"
        "selp.f32 %0, %5, 0f00000000, pv;\n\t"
        "selp.b32 %1, -1, 0, ps;\n\t}"
        : "=f"(r), "=r"(pass_mask)
        : "f"(power), "f"(vis_thr), "f"(sat_thr), "f"(value));
  }
  return r;
}

}  // namespace gsb
