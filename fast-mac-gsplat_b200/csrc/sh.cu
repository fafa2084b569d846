// View-dependent colour from real spherical harmonics (degree 0-3) and its VJP.
//
// Not part of the reference, whose colours are raw RGB inputs
// (variants/v8_project3d/torch_gsplat_bridge_v8_project3d/rasterize.py:958-1003):
// this is the first widening step after the rasterizer path. It turns per-
// Gaussian SH coefficients into the [B,G,3] colours rasterize_pinhole_gaussians
// takes, for every camera, so a 3D training step carries the full per-Gaussian
// parameter set (48 SH floats + 11 geometry floats).
//
// colour_c = max(0, 0.5 + sum_k coeff[k][c] Y_k(d)), d = normalize(mean - camera
// centre), with the real SH basis Y_k in the common (y, z, x) ordering and
// normalisation constants sqrt((2l+1)/(4 pi) (l-|m|)!/(l+|m|)!) (times sqrt 2
// for m != 0). The clamp passes no gradient where it is active.
#include <algorithm>

#include "gsb_common.cuh"
#include "gsb_host.cuh"

namespace gsb {
namespace {

constexpr int kShMaxK = 16;

// Real SH basis up to degree 3 at unit direction (x, y, z); fills Y[0..K).
__device__ __forceinline__ void sh_basis(int K, float x, float y, float z, float (&Y)[kShMaxK]) {
  const float c0 = 0.28209479177387814f;
  const float c1 = 0.4886025119029199f;
  Y[0] = c0;
  if (K <= 1) return;
  Y[1] = -c1 * y;
  Y[2] = c1 * z;
  Y[3] = -c1 * x;
  if (K <= 4) return;
  const float xx = x * x, yy = y * y, zz = z * z, xy = x * y, yz = y * z, xz = x * z;
  Y[4] = 1.0925484305920792f * xy;
  Y[5] = -1.0925484305920792f * yz;
  Y[6] = 0.31539156525252005f * (2.0f * zz - xx - yy);
  Y[7] = -1.0925484305920792f * xz;
  Y[8] = 0.5462742152960396f * (xx - yy);
  if (K <= 9) return;
  Y[9] = -0.5900435899266435f * y * (3.0f * xx - yy);
  Y[10] = 2.890611442640554f * xy * z;
  Y[11] = -0.4570457994644658f * y * (4.0f * zz - xx - yy);
  Y[12] = 0.3731763325901154f * z * (2.0f * zz - 3.0f * xx - 3.0f * yy);
  Y[13] = -0.4570457994644658f * x * (4.0f * zz - xx - yy);
  Y[14] = 1.445305721320277f * z * (xx - yy);
  Y[15] = -0.5900435899266435f * x * (xx - 3.0f * yy);
}

// d Y_k / d(x, y, z) for k < K (treating x, y, z as independent).
__device__ __forceinline__ void sh_basis_grad(int K, float x, float y, float z, float (&dx)[kShMaxK],
                                              float (&dy)[kShMaxK], float (&dz)[kShMaxK]) {
  const float c1 = 0.4886025119029199f;
#pragma unroll
  for (int k = 0; k < kShMaxK; ++k) dx[k] = dy[k] = dz[k] = 0.0f;
  if (K <= 1) return;
  dy[1] = -c1;
  dz[2] = c1;
  dx[3] = -c1;
  if (K <= 4) return;
  const float a = 1.0925484305920792f, b = 0.31539156525252005f, c = 0.5462742152960396f;
  dx[4] = a * y;          dy[4] = a * x;
  dy[5] = -a * z;         dz[5] = -a * y;
  dx[6] = -2.0f * b * x;  dy[6] = -2.0f * b * y;  dz[6] = 4.0f * b * z;
  dx[7] = -a * z;         dz[7] = -a * x;
  dx[8] = 2.0f * c * x;   dy[8] = -2.0f * c * y;
  if (K <= 9) return;
  const float xx = x * x, yy = y * y, zz = z * z;
  const float e9 = -0.5900435899266435f, e10 = 2.890611442640554f, e11 = -0.4570457994644658f,
              e12 = 0.3731763325901154f, e14 = 1.445305721320277f;
  dx[9] = e9 * 6.0f * x * y;                 dy[9] = e9 * (3.0f * xx - 3.0f * yy);
  dx[10] = e10 * y * z;                      dy[10] = e10 * x * z;                  dz[10] = e10 * x * y;
  dx[11] = e11 * (-2.0f * x * y);            dy[11] = e11 * (4.0f * zz - xx - 3.0f * yy);
  dz[11] = e11 * 8.0f * y * z;
  dx[12] = e12 * (-6.0f * x * z);            dy[12] = e12 * (-6.0f * y * z);
  dz[12] = e12 * (6.0f * zz - 3.0f * xx - 3.0f * yy);
  dx[13] = e11 * (4.0f * zz - 3.0f * xx - yy);  dy[13] = e11 * (-2.0f * x * y);    dz[13] = e11 * 8.0f * x * z;
  dx[14] = e14 * 2.0f * x * z;               dy[14] = -e14 * 2.0f * y * z;          dz[14] = e14 * (xx - yy);
  dx[15] = e9 * (3.0f * xx - 3.0f * yy);     dy[15] = e9 * (-6.0f * x * y);
}

struct Dir {
  float x, y, z, inv;  // unit direction and 1/|mean - centre|
};

__device__ __forceinline__ Dir view_dir(const float* __restrict__ means3d, const float* __restrict__ c2w, int g,
                                        int b) {
  const float* cw = c2w + 16 * b;
  const float dx = means3d[3 * g + 0] - __ldg(cw + 3);
  const float dy = means3d[3 * g + 1] - __ldg(cw + 7);
  const float dz = means3d[3 * g + 2] - __ldg(cw + 11);
  Dir d;
  d.inv = rsqrtf(fmaxf(dx * dx + dy * dy + dz * dz, 1e-24f));
  d.x = dx * d.inv;
  d.y = dy * d.inv;
  d.z = dz * d.inv;
  return d;
}

// One thread per (view, Gaussian): colours [B, G, 3].
__global__ void __launch_bounds__(256)
    k_sh_fwd(int B, int G, FastDiv gdiv, int K, const float* __restrict__ coeffs, const float* __restrict__ means3d,
             const float* __restrict__ c2w, float* __restrict__ colors) {
  pdl_wait();
  pdl_trigger();
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= (int64_t)B * G) return;
  const int b = fast_div((int)i, gdiv), g = (int)(i - (int64_t)b * G);  // i < 2^31 (checked on the host)
  const Dir d = view_dir(means3d, c2w, g, b);
  float Y[kShMaxK];
  sh_basis(K, d.x, d.y, d.z, Y);
  const float* cf = coeffs + (size_t)g * K * 3;
  float r = 0.5f, gg = 0.5f, bb = 0.5f;
#pragma unroll
  for (int k = 0; k < kShMaxK; ++k) {
    if (k < K) {
      r = fmaf(cf[3 * k + 0], Y[k], r);
      gg = fmaf(cf[3 * k + 1], Y[k], gg);
      bb = fmaf(cf[3 * k + 2], Y[k], bb);
    }
  }
  colors[3 * i + 0] = fmaxf(r, 0.0f);
  colors[3 * i + 1] = fmaxf(gg, 0.0f);
  colors[3 * i + 2] = fmaxf(bb, 0.0f);
}

// One thread per Gaussian, looping over the views (the coefficients are shared,
// so their gradient needs no atomics). Camera-centre gradients: per-CTA
// shared-memory sums, one atomic per view and axis per CTA (B <= kShSmemViews),
// else one per thread.
constexpr int kShSmemViews = 64;

__global__ void __launch_bounds__(256)
    k_sh_bwd(int B, int G, int K, const float* __restrict__ coeffs, const float* __restrict__ means3d,
             const float* __restrict__ c2w, const float* __restrict__ colors, const float* __restrict__ g_colors,
             float* __restrict__ g_coeffs, float* __restrict__ g_means3d, float* __restrict__ g_c2w) {
  pdl_wait();
  pdl_trigger();
  __shared__ float s_center[kShSmemViews][3];
  const bool smem_views = B <= kShSmemViews;
  if (g_c2w && smem_views)
    for (int t = threadIdx.x; t < B * 3; t += blockDim.x) (&s_center[0][0])[t] = 0.0f;
  __syncthreads();
  const int g = blockIdx.x * blockDim.x + threadIdx.x;
  if (g < G) {
    const float* cf = coeffs + (size_t)g * K * 3;
    float gc[kShMaxK][3];
#pragma unroll
    for (int k = 0; k < kShMaxK; ++k) gc[k][0] = gc[k][1] = gc[k][2] = 0.0f;
    float gm[3] = {0.0f, 0.0f, 0.0f};
    for (int b = 0; b < B; ++b) {
      const int64_t i = (int64_t)b * G + g;
      // The clamp at zero passes no gradient (colours[i] is the clamped output).
      const float u0 = colors[3 * i + 0] > 0.0f ? g_colors[3 * i + 0] : 0.0f;
      const float u1 = colors[3 * i + 1] > 0.0f ? g_colors[3 * i + 1] : 0.0f;
      const float u2 = colors[3 * i + 2] > 0.0f ? g_colors[3 * i + 2] : 0.0f;
      if (u0 == 0.0f && u1 == 0.0f && u2 == 0.0f) continue;
      const Dir d = view_dir(means3d, c2w, g, b);
      float Y[kShMaxK], dYx[kShMaxK], dYy[kShMaxK], dYz[kShMaxK];
      sh_basis(K, d.x, d.y, d.z, Y);
      sh_basis_grad(K, d.x, d.y, d.z, dYx, dYy, dYz);
      float gx = 0.0f, gy = 0.0f, gz = 0.0f;  // d loss / d unit direction
#pragma unroll
      for (int k = 0; k < kShMaxK; ++k) {
        if (k < K) {
          gc[k][0] = fmaf(u0, Y[k], gc[k][0]);
          gc[k][1] = fmaf(u1, Y[k], gc[k][1]);
          gc[k][2] = fmaf(u2, Y[k], gc[k][2]);
          const float w = u0 * cf[3 * k + 0] + u1 * cf[3 * k + 1] + u2 * cf[3 * k + 2];
          gx = fmaf(w, dYx[k], gx);
          gy = fmaf(w, dYy[k], gy);
          gz = fmaf(w, dYz[k], gz);
        }
      }
      // d/d(mean) of normalize(mean - centre): (g - (g.n) n) / |mean - centre|.
      const float gn = gx * d.x + gy * d.y + gz * d.z;
      const float mx = (gx - gn * d.x) * d.inv, my = (gy - gn * d.y) * d.inv, mz = (gz - gn * d.z) * d.inv;
      gm[0] += mx;
      gm[1] += my;
      gm[2] += mz;
      if (g_c2w) {  // the centre enters with the opposite sign
        if (smem_views) {
          atomicAdd(&s_center[b][0], -mx);
          atomicAdd(&s_center[b][1], -my);
          atomicAdd(&s_center[b][2], -mz);
        } else {
          atomicAdd(&g_c2w[16 * b + 3], -mx);
          atomicAdd(&g_c2w[16 * b + 7], -my);
          atomicAdd(&g_c2w[16 * b + 11], -mz);
        }
      }
    }
    float* gco = g_coeffs + (size_t)g * K * 3;
#pragma unroll
    for (int k = 0; k < kShMaxK; ++k) {
      if (k < K) {
        gco[3 * k + 0] = gc[k][0];
        gco[3 * k + 1] = gc[k][1];
        gco[3 * k + 2] = gc[k][2];
      }
    }
    if (g_means3d) {
      g_means3d[3 * g + 0] = gm[0];
      g_means3d[3 * g + 1] = gm[1];
      g_means3d[3 * g + 2] = gm[2];
    }
  }
  if (g_c2w && smem_views) {
    __syncthreads();
    for (int t = threadIdx.x; t < B * 3; t += blockDim.x) {
      const float v = (&s_center[0][0])[t];
      if (v != 0.0f) atomicAdd(&g_c2w[16 * (t / 3) + 4 * (t % 3) + 3], v);
    }
  }
}

int sh_k(int degree) { return (degree + 1) * (degree + 1); }

}  // namespace
}  // namespace gsb

using namespace gsb;

extern "C" int gsb_sh_forward(int32_t batch_size, int32_t gaussians, int32_t degree, const float* sh_coeffs,
                              const float* means3d, const float* camera_to_world, float* colors, void* stream) {
  if (batch_size <= 0 || gaussians < 0 || degree < 0 || degree > 3) return GSB_ERR_INVALID_ARGUMENT;
  const int64_t n = (int64_t)batch_size * gaussians;
  if (n == 0) return GSB_OK;
  if (!sh_coeffs || !means3d || !camera_to_world || !colors) return GSB_ERR_INVALID_ARGUMENT;
  if (n >= (int64_t(1) << 31)) return GSB_ERR_CAPACITY;
  launch_pdl(k_sh_fwd, grid1d(n, 256), 256, 0, static_cast<cudaStream_t>(stream), batch_size, gaussians,
             make_fast_div((uint32_t)gaussians), sh_k(degree),
                                                                          sh_coeffs, means3d, camera_to_world,
                                                                          colors);
  note_launches(1);
  return cuda_status(cudaGetLastError());
}

extern "C" int gsb_sh_backward(int32_t batch_size, int32_t gaussians, int32_t degree, const float* sh_coeffs,
                               const float* means3d, const float* camera_to_world, const float* colors,
                               const float* grad_colors, float* g_sh_coeffs, float* g_means3d,
                               float* g_camera_to_world, void* stream) {
  if (batch_size <= 0 || gaussians < 0 || degree < 0 || degree > 3) return GSB_ERR_INVALID_ARGUMENT;
  if (gaussians == 0) return GSB_OK;
  if (!sh_coeffs || !means3d || !camera_to_world || !colors || !grad_colors || !g_sh_coeffs)
    return GSB_ERR_INVALID_ARGUMENT;
  if ((int64_t)batch_size * gaussians >= (int64_t(1) << 31)) return GSB_ERR_CAPACITY;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (g_camera_to_world &&
      cudaMemsetAsync(g_camera_to_world, 0, sizeof(float) * 16 * (size_t)batch_size, s) != cudaSuccess)
    return GSB_ERR_CUDA;
  launch_pdl(k_sh_bwd, grid1d(gaussians, 256), 256, 0, s, batch_size, gaussians, sh_k(degree), sh_coeffs, means3d,
                                                  camera_to_world, colors, grad_colors, g_sh_coeffs, g_means3d,
                                                  g_camera_to_world);
  note_launches(1);
  return cuda_status(cudaGetLastError());
}
