// Pinhole EWA projection of 3D Gaussians and its VJP, one thread per Gaussian.
//
// Reference: variants/v8_project3d/csrc/metal/gsplat_v8_project3d_kernels.metal
//   project_pinhole_forward 66-174, project_pinhole_backward 217-501;
//   torch restatement variants/v8_project3d/torch_gsplat_bridge_v8_project3d/rasterize.py:288-358.
// Conventions kept from the reference: scales are linear (squared here), quats
// are (r,i,j,k) and not normalised, camera_to_world is row-major [4,4] with the
// camera axes in its columns (x_cam = R^T (m - t)), +z is forward, EWA adds 0.3
// to the 2D covariance diagonal and clamps the determinant at 1e-6, splats with
// z <= near_plane get opacity 0.
#include <algorithm>

#include "gsb_common.cuh"
#include "gsb_host.cuh"

namespace gsb {
namespace {

struct Rot {
  float r00, r01, r02, r10, r11, r12, r20, r21, r22;
};

__device__ __forceinline__ Rot quat_to_rot(float qr, float qi, float qj, float qk) {
  Rot g;
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

struct Sym3 {
  float c00, c01, c02, c11, c12, c22;
};

// u^T C v for symmetric C.
__device__ __forceinline__ float sym_bilinear(const float3& u, const Sym3& C, const float3& v) {
  return u.x * (C.c00 * v.x + C.c01 * v.y + C.c02 * v.z) + u.y * (C.c01 * v.x + C.c11 * v.y + C.c12 * v.z) +
         u.z * (C.c02 * v.x + C.c12 * v.y + C.c22 * v.z);
}

struct Cam {
  float r00, r01, r02, tx, r10, r11, r12, ty, r20, r21, r22, tz;
  float fx, fy, cx, cy;
};

__device__ __forceinline__ Cam load_cam(const float* __restrict__ c2w, const float* __restrict__ cp, int b) {
  const float4* m4 = reinterpret_cast<const float4*>(c2w + 16 * b);
  const float4 row0 = __ldg(m4 + 0), row1 = __ldg(m4 + 1), row2 = __ldg(m4 + 2);
  const float4 k = __ldg(reinterpret_cast<const float4*>(cp) + b);
  Cam c;
  c.r00 = row0.x; c.r01 = row0.y; c.r02 = row0.z; c.tx = row0.w;
  c.r10 = row1.x; c.r11 = row1.y; c.r12 = row1.z; c.ty = row1.w;
  c.r20 = row2.x; c.r21 = row2.y; c.r22 = row2.z; c.tz = row2.w;
  c.fx = k.x; c.fy = k.y; c.cx = k.z; c.cy = k.w;
  return c;
}

// Everything the forward computes, reused by the backward.
struct Proj {
  Rot R;
  Sym3 C;        // world covariance R diag(s^2) R^T
  float sx2, sy2, sz2;
  float dx, dy, dz, x, y, z;
  float3 col0, col1, col2;
  Sym3 Cc;       // camera covariance
  bool front;
  float z_safe, x_p, y_p;
  float j00, j02, j11, j12;
  float cov00, cov01, cov11, det_raw, det;
};

__device__ __forceinline__ Proj project_one(const float3 mu, const float3 s, const float4 q, const Cam& k,
                                            float near_plane) {
  Proj p;
  p.sx2 = s.x * s.x;
  p.sy2 = s.y * s.y;
  p.sz2 = s.z * s.z;
  p.R = quat_to_rot(q.x, q.y, q.z, q.w);
  const Rot& g = p.R;
  p.C.c00 = g.r00 * g.r00 * p.sx2 + g.r01 * g.r01 * p.sy2 + g.r02 * g.r02 * p.sz2;
  p.C.c01 = g.r00 * g.r10 * p.sx2 + g.r01 * g.r11 * p.sy2 + g.r02 * g.r12 * p.sz2;
  p.C.c02 = g.r00 * g.r20 * p.sx2 + g.r01 * g.r21 * p.sy2 + g.r02 * g.r22 * p.sz2;
  p.C.c11 = g.r10 * g.r10 * p.sx2 + g.r11 * g.r11 * p.sy2 + g.r12 * g.r12 * p.sz2;
  p.C.c12 = g.r10 * g.r20 * p.sx2 + g.r11 * g.r21 * p.sy2 + g.r12 * g.r22 * p.sz2;
  p.C.c22 = g.r20 * g.r20 * p.sx2 + g.r21 * g.r21 * p.sy2 + g.r22 * g.r22 * p.sz2;
  p.dx = mu.x - k.tx;
  p.dy = mu.y - k.ty;
  p.dz = mu.z - k.tz;
  p.x = p.dx * k.r00 + p.dy * k.r10 + p.dz * k.r20;
  p.y = p.dx * k.r01 + p.dy * k.r11 + p.dz * k.r21;
  p.z = p.dx * k.r02 + p.dy * k.r12 + p.dz * k.r22;
  p.col0 = make_float3(k.r00, k.r10, k.r20);
  p.col1 = make_float3(k.r01, k.r11, k.r21);
  p.col2 = make_float3(k.r02, k.r12, k.r22);
  p.Cc.c00 = sym_bilinear(p.col0, p.C, p.col0);
  p.Cc.c01 = sym_bilinear(p.col0, p.C, p.col1);
  p.Cc.c02 = sym_bilinear(p.col0, p.C, p.col2);
  p.Cc.c11 = sym_bilinear(p.col1, p.C, p.col1);
  p.Cc.c12 = sym_bilinear(p.col1, p.C, p.col2);
  p.Cc.c22 = sym_bilinear(p.col2, p.C, p.col2);
  p.front = p.z > near_plane;
  p.z_safe = p.front ? fmaxf(p.z, near_plane) : 1.0f;
  p.x_p = p.front ? p.x : 0.0f;
  p.y_p = p.front ? p.y : 0.0f;
  p.j00 = k.fx / p.z_safe;
  p.j02 = -(k.fx * p.x_p) / (p.z_safe * p.z_safe);
  p.j11 = k.fy / p.z_safe;
  p.j12 = -(k.fy * p.y_p) / (p.z_safe * p.z_safe);
  const Sym3& cc = p.Cc;
  p.cov00 = p.j00 * p.j00 * cc.c00 + 2.0f * p.j00 * p.j02 * cc.c02 + p.j02 * p.j02 * cc.c22 + 0.3f;
  p.cov01 = p.j00 * p.j11 * cc.c01 + p.j00 * p.j12 * cc.c02 + p.j02 * p.j11 * cc.c12 + p.j02 * p.j12 * cc.c22;
  p.cov11 = p.j11 * p.j11 * cc.c11 + 2.0f * p.j11 * p.j12 * cc.c12 + p.j12 * p.j12 * cc.c22 + 0.3f;
  p.det_raw = p.cov00 * p.cov11 - p.cov01 * p.cov01;
  p.det = fmaxf(p.det_raw, 1e-6f);
  return p;
}

__global__ void __launch_bounds__(256)
    k_project_fwd(int B, int G, FastDiv gdiv, const float* __restrict__ means3d, const float* __restrict__ scales,
                  const float4* __restrict__ quats, const float* __restrict__ opacities,
                  const float* __restrict__ c2w, const float* __restrict__ cam, float near_plane,
                  float2* __restrict__ out_means2d, float* __restrict__ out_conics,
                  float* __restrict__ out_opac, float* __restrict__ out_depth) {
  pdl_wait();
  pdl_trigger();
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= (int64_t)B * G) return;
  const int b = fast_div((int)i, gdiv);  // i < 2^31 (checked on the host)
  const Cam k = load_cam(c2w, cam, b);
  const float3 mu = make_float3(means3d[3 * i + 0], means3d[3 * i + 1], means3d[3 * i + 2]);
  const float3 s = make_float3(scales[3 * i + 0], scales[3 * i + 1], scales[3 * i + 2]);
  const Proj p = project_one(mu, s, quats[i], k, near_plane);
  out_means2d[i] = make_float2((k.fx * p.x_p) / p.z_safe + k.cx, (k.fy * p.y_p) / p.z_safe + k.cy);
  out_conics[3 * i + 0] = p.cov11 / p.det;
  out_conics[3 * i + 1] = -p.cov01 / p.det;
  out_conics[3 * i + 2] = p.cov00 / p.det;
  out_opac[i] = p.front ? opacities[i] : 0.0f;
  out_depth[i] = p.z;
}

// d(u^T C v): accumulates into gC and returns (gu, gv) contributions.
__device__ __forceinline__ void sym_bilinear_bwd(float g, const float3& u, const Sym3& C, const float3& v, Sym3& gC,
                                                 float3& gu, float3& gv) {
  gC.c00 += g * u.x * v.x;
  gC.c01 += g * (u.x * v.y + u.y * v.x);
  gC.c02 += g * (u.x * v.z + u.z * v.x);
  gC.c11 += g * u.y * v.y;
  gC.c12 += g * (u.y * v.z + u.z * v.y);
  gC.c22 += g * u.z * v.z;
  const float3 cv = make_float3(C.c00 * v.x + C.c01 * v.y + C.c02 * v.z, C.c01 * v.x + C.c11 * v.y + C.c12 * v.z,
                                C.c02 * v.x + C.c12 * v.y + C.c22 * v.z);
  const float3 cu = make_float3(C.c00 * u.x + C.c01 * u.y + C.c02 * u.z, C.c01 * u.x + C.c11 * u.y + C.c12 * u.z,
                                C.c02 * u.x + C.c12 * u.y + C.c22 * u.z);
  gu = make_float3(g * cv.x, g * cv.y, g * cv.z);
  gv = make_float3(g * cu.x, g * cu.y, g * cu.z);
}

__device__ __forceinline__ float3 add3(float3 a, float3 b) { return make_float3(a.x + b.x, a.y + b.y, a.z + b.z); }

// VJP of one Gaussian: writes its per-Gaussian gradients and returns its view;
// cg receives its 16 camera-gradient terms (zeros when !active).
__device__ __forceinline__ int project_bwd_one(
    FastDiv gdiv, int64_t n, int64_t i, bool active, const float2* __restrict__ g_m2d, const float* __restrict__ g_con,
    const float* __restrict__ g_opac_in, const float* __restrict__ g_depth, const float* __restrict__ means3d,
    const float* __restrict__ scales, const float4* __restrict__ quats, const float* __restrict__ c2w,
    const float* __restrict__ cam, float near_plane, float* __restrict__ g_means3d, float* __restrict__ g_scales,
    float4* __restrict__ g_quats, float* __restrict__ g_opac, float (&cg)[16]) {
  const int64_t ii = active ? i : n - 1;  // inactive lanes recompute a valid item, contribute zeros
  const int b = fast_div((int)ii, gdiv);  // ii < 2^31 (checked on the host)
  const Cam k = load_cam(c2w, cam, b);
  const float3 mu = make_float3(means3d[3 * ii + 0], means3d[3 * ii + 1], means3d[3 * ii + 2]);
  const float3 s = make_float3(scales[3 * ii + 0], scales[3 * ii + 1], scales[3 * ii + 2]);
  const float4 q = quats[ii];
  const Proj p = project_one(mu, s, q, k, near_plane);
  const Rot& gr = p.R;
  const Sym3& cc = p.Cc;

  const float inv_z = 1.0f / p.z_safe;
  const float inv_z2 = inv_z * inv_z;
  const float inv_z3 = inv_z2 * inv_z;
  // The reference backward recomputes J with multiplications by 1/z (…metal:315-321).
  const float j00 = k.fx * inv_z, j02 = -(k.fx * p.x_p) * inv_z2;
  const float j11 = k.fy * inv_z, j12 = -(k.fy * p.y_p) * inv_z2;

  const float2 gm = (active && g_m2d) ? g_m2d[ii] : make_float2(0.f, 0.f);
  const float ga = (active && g_con) ? g_con[3 * ii + 0] : 0.f;
  const float gb = (active && g_con) ? g_con[3 * ii + 1] : 0.f;
  const float gc = (active && g_con) ? g_con[3 * ii + 2] : 0.f;

  const float det = p.det;
  float g_cov00 = gc / det;
  float g_cov01 = -gb / det;
  float g_cov11 = ga / det;
  const float g_det = -(ga * p.cov11 - gb * p.cov01 + gc * p.cov00) / (det * det);
  if (p.det_raw > 1e-6f) {
    g_cov00 += g_det * p.cov11;
    g_cov11 += g_det * p.cov00;
    g_cov01 += g_det * (-2.0f * p.cov01);
  }

  Sym3 gcc;
  gcc.c00 = g_cov00 * j00 * j00;
  gcc.c02 = g_cov00 * (2.0f * j00 * j02);
  gcc.c22 = g_cov00 * j02 * j02;
  float g_j00 = g_cov00 * (2.0f * j00 * cc.c00 + 2.0f * j02 * cc.c02);
  float g_j02 = g_cov00 * (2.0f * j00 * cc.c02 + 2.0f * j02 * cc.c22);
  gcc.c01 = g_cov01 * j00 * j11;
  gcc.c02 += g_cov01 * j00 * j12;
  gcc.c12 = g_cov01 * j02 * j11;
  gcc.c22 += g_cov01 * j02 * j12;
  g_j00 += g_cov01 * (j11 * cc.c01 + j12 * cc.c02);
  g_j02 += g_cov01 * (j11 * cc.c12 + j12 * cc.c22);
  float g_j11 = g_cov01 * (j00 * cc.c01 + j02 * cc.c12);
  float g_j12 = g_cov01 * (j00 * cc.c02 + j02 * cc.c22);
  gcc.c11 = g_cov11 * j11 * j11;
  gcc.c12 += g_cov11 * (2.0f * j11 * j12);
  gcc.c22 += g_cov11 * j12 * j12;
  g_j11 += g_cov11 * (2.0f * j11 * cc.c11 + 2.0f * j12 * cc.c12);
  g_j12 += g_cov11 * (2.0f * j11 * cc.c12 + 2.0f * j12 * cc.c22);

  float g_x = 0.f, g_y = 0.f;
  float g_z = (active && g_depth) ? g_depth[ii] : 0.f;
  float g_fx = 0.f, g_fy = 0.f;
  const float g_cx = gm.x, g_cy = gm.y;
  const float x = p.x, y = p.y;
  if (p.front) {
    g_fx += gm.x * x * inv_z;
    g_x += gm.x * k.fx * inv_z;
    g_z += gm.x * (-(k.fx * x) * inv_z2);
    g_fy += gm.y * y * inv_z;
    g_y += gm.y * k.fy * inv_z;
    g_z += gm.y * (-(k.fy * y) * inv_z2);
    g_fx += g_j00 * inv_z;
    g_z += g_j00 * (-k.fx * inv_z2);
    g_fx += g_j02 * (-x * inv_z2);
    g_x += g_j02 * (-k.fx * inv_z2);
    g_z += g_j02 * (2.0f * k.fx * x * inv_z3);
    g_fy += g_j11 * inv_z;
    g_z += g_j11 * (-k.fy * inv_z2);
    g_fy += g_j12 * (-y * inv_z2);
    g_y += g_j12 * (-k.fy * inv_z2);
    g_z += g_j12 * (2.0f * k.fy * y * inv_z3);
  } else {
    g_fx += g_j00;
    g_fy += g_j11;
  }

  Sym3 gC = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
  float3 g_col0 = make_float3(0.f, 0.f, 0.f), g_col1 = g_col0, g_col2 = g_col0, gu, gv;
  sym_bilinear_bwd(gcc.c00, p.col0, p.C, p.col0, gC, gu, gv);
  g_col0 = add3(g_col0, add3(gu, gv));
  sym_bilinear_bwd(gcc.c01, p.col0, p.C, p.col1, gC, gu, gv);
  g_col0 = add3(g_col0, gu);
  g_col1 = add3(g_col1, gv);
  sym_bilinear_bwd(gcc.c02, p.col0, p.C, p.col2, gC, gu, gv);
  g_col0 = add3(g_col0, gu);
  g_col2 = add3(g_col2, gv);
  sym_bilinear_bwd(gcc.c11, p.col1, p.C, p.col1, gC, gu, gv);
  g_col1 = add3(g_col1, add3(gu, gv));
  sym_bilinear_bwd(gcc.c12, p.col1, p.C, p.col2, gC, gu, gv);
  g_col1 = add3(g_col1, gu);
  g_col2 = add3(g_col2, gv);
  sym_bilinear_bwd(gcc.c22, p.col2, p.C, p.col2, gC, gu, gv);
  g_col2 = add3(g_col2, add3(gu, gv));

  const float g_dx = g_x * k.r00 + g_y * k.r01 + g_z * k.r02;
  const float g_dy = g_x * k.r10 + g_y * k.r11 + g_z * k.r12;
  const float g_dz = g_x * k.r20 + g_y * k.r21 + g_z * k.r22;
  g_col0 = add3(g_col0, make_float3(g_x * p.dx, g_x * p.dy, g_x * p.dz));
  g_col1 = add3(g_col1, make_float3(g_y * p.dx, g_y * p.dy, g_y * p.dz));
  g_col2 = add3(g_col2, make_float3(g_z * p.dx, g_z * p.dy, g_z * p.dz));

  const float g_sx2 = gC.c00 * gr.r00 * gr.r00 + gC.c01 * gr.r00 * gr.r10 + gC.c02 * gr.r00 * gr.r20 +
                      gC.c11 * gr.r10 * gr.r10 + gC.c12 * gr.r10 * gr.r20 + gC.c22 * gr.r20 * gr.r20;
  const float g_sy2 = gC.c00 * gr.r01 * gr.r01 + gC.c01 * gr.r01 * gr.r11 + gC.c02 * gr.r01 * gr.r21 +
                      gC.c11 * gr.r11 * gr.r11 + gC.c12 * gr.r11 * gr.r21 + gC.c22 * gr.r21 * gr.r21;
  const float g_sz2 = gC.c00 * gr.r02 * gr.r02 + gC.c01 * gr.r02 * gr.r12 + gC.c02 * gr.r02 * gr.r22 +
                      gC.c11 * gr.r12 * gr.r12 + gC.c12 * gr.r12 * gr.r22 + gC.c22 * gr.r22 * gr.r22;
  const float sx2 = p.sx2, sy2 = p.sy2, sz2 = p.sz2;
  const float g00 = sx2 * (2.0f * gC.c00 * gr.r00 + gC.c01 * gr.r10 + gC.c02 * gr.r20);
  const float g10 = sx2 * (gC.c01 * gr.r00 + 2.0f * gC.c11 * gr.r10 + gC.c12 * gr.r20);
  const float g20 = sx2 * (gC.c02 * gr.r00 + gC.c12 * gr.r10 + 2.0f * gC.c22 * gr.r20);
  const float g01 = sy2 * (2.0f * gC.c00 * gr.r01 + gC.c01 * gr.r11 + gC.c02 * gr.r21);
  const float g11 = sy2 * (gC.c01 * gr.r01 + 2.0f * gC.c11 * gr.r11 + gC.c12 * gr.r21);
  const float g21 = sy2 * (gC.c02 * gr.r01 + gC.c12 * gr.r11 + 2.0f * gC.c22 * gr.r21);
  const float g02 = sz2 * (2.0f * gC.c00 * gr.r02 + gC.c01 * gr.r12 + gC.c02 * gr.r22);
  const float g12 = sz2 * (gC.c01 * gr.r02 + 2.0f * gC.c11 * gr.r12 + gC.c12 * gr.r22);
  const float g22 = sz2 * (gC.c02 * gr.r02 + gC.c12 * gr.r12 + 2.0f * gC.c22 * gr.r22);

  const float qr = q.x, qi = q.y, qj = q.z, qk = q.w;
  float g_qr = 0.f, g_qi = 0.f, g_qj = 0.f, g_qk = 0.f;
  g_qj += -4.0f * qj * g00; g_qk += -4.0f * qk * g00;
  g_qi += 2.0f * qj * g01; g_qj += 2.0f * qi * g01; g_qr += -2.0f * qk * g01; g_qk += -2.0f * qr * g01;
  g_qi += 2.0f * qk * g02; g_qk += 2.0f * qi * g02; g_qr += 2.0f * qj * g02; g_qj += 2.0f * qr * g02;
  g_qi += 2.0f * qj * g10; g_qj += 2.0f * qi * g10; g_qr += 2.0f * qk * g10; g_qk += 2.0f * qr * g10;
  g_qi += -4.0f * qi * g11; g_qk += -4.0f * qk * g11;
  g_qj += 2.0f * qk * g12; g_qk += 2.0f * qj * g12; g_qr += -2.0f * qi * g12; g_qi += -2.0f * qr * g12;
  g_qi += 2.0f * qk * g20; g_qk += 2.0f * qi * g20; g_qr += -2.0f * qj * g20; g_qj += -2.0f * qr * g20;
  g_qj += 2.0f * qk * g21; g_qk += 2.0f * qj * g21; g_qr += 2.0f * qi * g21; g_qi += 2.0f * qr * g21;
  g_qi += -4.0f * qi * g22; g_qj += -4.0f * qj * g22;

  if (active) {
    g_means3d[3 * i + 0] = g_dx;
    g_means3d[3 * i + 1] = g_dy;
    g_means3d[3 * i + 2] = g_dz;
    g_scales[3 * i + 0] = 2.0f * s.x * g_sx2;
    g_scales[3 * i + 1] = 2.0f * s.y * g_sy2;
    g_scales[3 * i + 2] = 2.0f * s.z * g_sz2;
    g_quats[i] = make_float4(g_qr, g_qi, g_qj, g_qk);
    g_opac[i] = p.front ? ((g_opac_in) ? g_opac_in[i] : 0.f) : 0.f;
  }

  cg[0] = g_col0.x; cg[1] = g_col1.x; cg[2] = g_col2.x; cg[3] = -g_dx;
  cg[4] = g_col0.y; cg[5] = g_col1.y; cg[6] = g_col2.y; cg[7] = -g_dy;
  cg[8] = g_col0.z; cg[9] = g_col1.z; cg[10] = g_col2.z; cg[11] = -g_dz;
  cg[12] = g_fx; cg[13] = g_fy; cg[14] = g_cx; cg[15] = g_cy;
  if (!active) {
#pragma unroll
    for (int t = 0; t < 16; ++t) cg[t] = 0.f;
  }
  return b;
}

__device__ __forceinline__ void cam_grad_atomics(float* g_c2w, float* g_cam, int b, const float (&v)[16]) {
#pragma unroll
  for (int t = 0; t < 12; ++t) atomicAdd(&g_c2w[16 * b + t], v[t]);
#pragma unroll
  for (int t = 0; t < 4; ++t) atomicAdd(&g_cam[4 * b + t], v[12 + t]);
}

// Persistent grid (a few CTAs per SM), one Gaussian per thread per iteration.
// The 16 per-view camera-gradient sums are accumulated per thread, then
// reduced across the CTA in shared memory: one atomic per value per CTA
// instead of per warp (all of a view's atomics hit one cache line, so their
// number sets the cost: 16 per warp at c4 serialised to ~0.46 ms).
__global__ void __launch_bounds__(256)
    k_project_bwd(int B, int G, FastDiv gdiv, const float2* __restrict__ g_m2d, const float* __restrict__ g_con,
                  const float* __restrict__ g_opac_in, const float* __restrict__ g_depth,
                  const float* __restrict__ means3d, const float* __restrict__ scales,
                  const float4* __restrict__ quats, const float* __restrict__ c2w, const float* __restrict__ cam,
                  float near_plane, float* __restrict__ g_means3d, float* __restrict__ g_scales,
                  float4* __restrict__ g_quats, float* __restrict__ g_opac, float* __restrict__ g_c2w,
                  float* __restrict__ g_cam) {
  pdl_wait();
  pdl_trigger();
  __shared__ float s_red[8][16];
  __shared__ int s_view;
  const int64_t n = (int64_t)B * G;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  float acc[16];
#pragma unroll
  for (int t = 0; t < 16; ++t) acc[t] = 0.f;
  int cur = -1;  // view of acc
  for (int64_t base = (int64_t)blockIdx.x * blockDim.x; base < n; base += (int64_t)gridDim.x * blockDim.x) {
    const int64_t i = base + threadIdx.x;
    const bool active = i < n;
    float cg[16];
    const int b = project_bwd_one(gdiv, n, i, active, g_m2d, g_con, g_opac_in, g_depth, means3d, scales, quats, c2w,
                                  cam, near_plane, g_means3d, g_scales, g_quats, g_opac, cg);
    if (active) {
      if (b != cur) {  // a thread crosses into the next view: flush the previous one
        if (cur >= 0) cam_grad_atomics(g_c2w, g_cam, cur, acc);
#pragma unroll
        for (int t = 0; t < 16; ++t) acc[t] = 0.f;
        cur = b;
      }
#pragma unroll
      for (int t = 0; t < 16; ++t) acc[t] += cg[t];
    }
  }
  if (threadIdx.x == 0) s_view = -1;
  __syncthreads();
  if (cur >= 0) atomicMax(&s_view, cur);
  __syncthreads();
  const int ref = s_view;
  if (__syncthreads_and(cur < 0 || cur == ref)) {
    if (ref < 0) return;  // the CTA had no Gaussian
#pragma unroll
    for (int t = 0; t < 16; ++t) {
      float v = acc[t];
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(kFullMask, v, o);
      if (lane == 0) s_red[warp][t] = v;
    }
    __syncthreads();
    if (threadIdx.x < 16) {
      float v = 0.f;
#pragma unroll
      for (int w = 0; w < 8; ++w) v += s_red[w][threadIdx.x];
      if (threadIdx.x < 12) atomicAdd(&g_c2w[16 * ref + threadIdx.x], v);
      else atomicAdd(&g_cam[4 * ref + threadIdx.x - 12], v);
    }
  } else if (cur >= 0) {
    cam_grad_atomics(g_c2w, g_cam, cur, acc);
  }
}

}  // namespace
}  // namespace gsb

using namespace gsb;

extern "C" int gsb_project_forward(int32_t batch_size, int32_t gaussians_per_batch, const float* means3d,
                                   const float* scales, const float* quats, const float* opacities,
                                   const float* camera_to_world, const float* camera_params, float near_plane,
                                   float* out_means2d, float* out_conics, float* out_opacities, float* out_depths,
                                   void* stream_) {
  if (batch_size <= 0 || gaussians_per_batch < 0) return GSB_ERR_INVALID_ARGUMENT;
  const int64_t n = (int64_t)batch_size * gaussians_per_batch;
  if (n == 0) return GSB_OK;
  if (n >= (int64_t(1) << 31)) return GSB_ERR_INVALID_ARGUMENT;
  if (!means3d || !scales || !quats || !opacities || !camera_to_world || !camera_params || !out_means2d ||
      !out_conics || !out_opacities || !out_depths)
    return GSB_ERR_INVALID_ARGUMENT;
  cudaStream_t stream = static_cast<cudaStream_t>(stream_);
  launch_pdl(k_project_fwd, grid1d(n, 256), 256, 0, stream, batch_size, gaussians_per_batch,
             make_fast_div((uint32_t)gaussians_per_batch), means3d, scales,
                                                    reinterpret_cast<const float4*>(quats), opacities,
                                                    camera_to_world, camera_params, near_plane,
                                                    reinterpret_cast<float2*>(out_means2d), out_conics,
                                                    out_opacities, out_depths);
  note_launches(1);
  return cuda_status(cudaGetLastError());
}

extern "C" int gsb_project_backward(int32_t batch_size, int32_t gaussians_per_batch, const float* grad_means2d,
                                    const float* grad_conics, const float* grad_opacities, const float* grad_depths,
                                    const float* means3d, const float* scales, const float* quats,
                                    const float* opacities, const float* camera_to_world,
                                    const float* camera_params, float near_plane, float* g_means3d,
                                    float* g_scales, float* g_quats, float* g_opacities, float* g_camera_to_world,
                                    float* g_camera_params, void* stream_) {
  (void)opacities;
  if (batch_size <= 0 || gaussians_per_batch < 0) return GSB_ERR_INVALID_ARGUMENT;
  const int64_t n = (int64_t)batch_size * gaussians_per_batch;
  if (n >= (int64_t(1) << 31)) return GSB_ERR_INVALID_ARGUMENT;
  if (!g_camera_to_world || !g_camera_params) return GSB_ERR_INVALID_ARGUMENT;
  cudaStream_t stream = static_cast<cudaStream_t>(stream_);
  cudaError_t e = cudaMemsetAsync(g_camera_to_world, 0, sizeof(float) * 16 * batch_size, stream);
  if (e != cudaSuccess) return GSB_ERR_CUDA;
  e = cudaMemsetAsync(g_camera_params, 0, sizeof(float) * 4 * batch_size, stream);
  if (e != cudaSuccess) return GSB_ERR_CUDA;
  if (n == 0) return GSB_OK;
  if (!means3d || !scales || !quats || !camera_to_world || !camera_params || !g_means3d || !g_scales ||
      !g_quats || !g_opacities)
    return GSB_ERR_INVALID_ARGUMENT;
  int sms = 148, dev = 0;
  if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const int64_t want = (n + 255) / 256;
  const int grid = (int)std::max<int64_t>(1, std::min<int64_t>(want, 2 * (int64_t)sms));
  launch_pdl(k_project_bwd, grid, 256, 0, stream, 
      batch_size, gaussians_per_batch, make_fast_div((uint32_t)gaussians_per_batch),
      reinterpret_cast<const float2*>(grad_means2d), grad_conics, grad_opacities,
      grad_depths, means3d, scales, reinterpret_cast<const float4*>(quats), camera_to_world, camera_params,
      near_plane, g_means3d, g_scales, reinterpret_cast<float4*>(g_quats), g_opacities, g_camera_to_world,
      g_camera_params);
  note_launches(1);
  return cuda_status(cudaGetLastError());
}
