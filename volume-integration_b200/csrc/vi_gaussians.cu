// Gaussian-attribute front end (extension): per-Gaussian preprocess, its
// backward, and tile binning of the projected Gaussians.
//
// The reference's primitives are cubes of one fixed world size: its preprocess
// projects a centre and a bounding radius only (cuda_integrator/forward.cu:82-87,
// :100-102), and its spherical-harmonics constants are unused
// (cuda_integrator/auxiliary.h:30-48).  This file adds the standard front end of
// Gaussian splatting (EWA splatting: Zwicker et al. 2001; 3D Gaussian splatting:
// Kerbl et al. 2023) as a separate entry point with its own oracle.  Per
// Gaussian i:
//
//   t      = view * p (transformPoint4x3);    culled when t.z <= near_plane
//   means2D = ndc2pix(proj * p / w)            as the cube preprocess
//   Sigma  = R(q) diag(m s)^2 R(q)^T          q normalised, m = scale_modifier
//   cov2D  = J W Sigma W^T J^T + 0.3 I         W = view rotation, J = d(pixel)/d(t)
//            at t with t.x/t.z, t.y/t.z clamped to +-1.3 tan(fov)
//   conic  = cov2D^-1 (upper triangle);        culled when det(cov2D) == 0
//   radius = ceil(3 sqrt(largest eigenvalue)), lambda = mid +- sqrt(max(0.1, mid^2 - det))
//   tiles  = area of getRect(means2D, radius); culled when 0
//   rgb    = max(0, sum_k sh_k Y_k(dir) + 0.5), dir = normalise(p - cam_pos),
//            real spherical harmonics up to degree 3
//
// Every forward operation is rounded explicitly (no contraction), so the CPU
// restatement reproduces radii, tile counts and all float outputs bit for bit.
// The backward is the exact derivative of this forward (including the clamps of
// J and of the colour, and the quaternion normalisation); culled Gaussians get
// zero gradients.
//
// Binning reuses the renderer's machinery: a stable depth sort of the visible
// Gaussians, the overlap scan in that order, emission of (tile, Gaussian) per
// tile of the rectangle, a stable sort by tile id and the tile ranges; the
// result equals a stable sort of the 64-bit keys tile << 32 | depth bits.
#include <cuda_runtime.h>

#include <cstdint>
#include <cstdio>

#include "../../include/volume_integration_b200.h"
#include "vi_common.cuh"
#include "vi_internal.h"

namespace vi {
namespace {

constexpr int kGaussThreads = 128;
constexpr int kMaxShCoeffs = 16;

// Real spherical-harmonics normalisation constants, degrees 0..3 (the common
// graphics sign convention: Y_1 = -C1 y, Y_2 = C1 z, Y_3 = -C1 x).
__constant__ float kC0 = 0.28209479177387814f;
__constant__ float kC1 = 0.4886025119029199f;
__constant__ float kC2[5] = {1.0925484305920792f, -1.0925484305920792f, 0.31539156525252005f, -1.0925484305920792f,
                             0.5462742152960396f};
__constant__ float kC3[7] = {-0.5900435899266435f, 2.890611442640554f, -0.4570457994644658f, 0.3731763325901154f,
                             -0.4570457994644658f, 1.445305721320277f, -0.5900435899266435f};

__device__ __forceinline__ float fdiv(float a, float b) { return __fdiv_rn(a, b); }
__device__ __forceinline__ float fsqrt(float a) { return __fsqrt_rn(a); }

// The 16 basis values at unit direction (x, y, z), as the products the forward
// forms them (each basis value, then times its coefficient).
__device__ __forceinline__ void sh_basis(float x, float y, float z, int deg, float* Y) {
  Y[0] = kC0;
  if (deg < 1) return;
  Y[1] = fmul(-kC1, y);
  Y[2] = fmul(kC1, z);
  Y[3] = fmul(-kC1, x);
  if (deg < 2) return;
  const float xx = fmul(x, x), yy = fmul(y, y), zz = fmul(z, z);
  const float xy = fmul(x, y), yz = fmul(y, z), xz = fmul(x, z);
  Y[4] = fmul(kC2[0], xy);
  Y[5] = fmul(kC2[1], yz);
  Y[6] = fmul(kC2[2], fsub(fsub(fmul(2.0f, zz), xx), yy));
  Y[7] = fmul(kC2[3], xz);
  Y[8] = fmul(kC2[4], fsub(xx, yy));
  if (deg < 3) return;
  Y[9] = fmul(fmul(kC3[0], y), fsub(fmul(3.0f, xx), yy));
  Y[10] = fmul(fmul(kC3[1], xy), z);
  Y[11] = fmul(fmul(kC3[2], y), fsub(fsub(fmul(4.0f, zz), xx), yy));
  Y[12] = fmul(fmul(kC3[3], z), fsub(fsub(fmul(2.0f, zz), fmul(3.0f, xx)), fmul(3.0f, yy)));
  Y[13] = fmul(fmul(kC3[4], x), fsub(fsub(fmul(4.0f, zz), xx), yy));
  Y[14] = fmul(fmul(kC3[5], z), fsub(xx, yy));
  Y[15] = fmul(fmul(kC3[6], x), fsub(xx, fmul(3.0f, yy)));
}

// Gradients of the basis values with respect to (x, y, z) (plain arithmetic).
__device__ __forceinline__ void sh_basis_grad(float x, float y, float z, int deg, float3* dY) {
  dY[0] = make_float3(0.f, 0.f, 0.f);
  if (deg < 1) return;
  dY[1] = make_float3(0.f, -kC1, 0.f);
  dY[2] = make_float3(0.f, 0.f, kC1);
  dY[3] = make_float3(-kC1, 0.f, 0.f);
  if (deg < 2) return;
  dY[4] = make_float3(kC2[0] * y, kC2[0] * x, 0.f);
  dY[5] = make_float3(0.f, kC2[1] * z, kC2[1] * y);
  dY[6] = make_float3(-2.f * kC2[2] * x, -2.f * kC2[2] * y, 4.f * kC2[2] * z);
  dY[7] = make_float3(kC2[3] * z, 0.f, kC2[3] * x);
  dY[8] = make_float3(2.f * kC2[4] * x, -2.f * kC2[4] * y, 0.f);
  if (deg < 3) return;
  const float xx = x * x, yy = y * y, zz = z * z;
  dY[9] = make_float3(6.f * kC3[0] * x * y, kC3[0] * (3.f * xx - 3.f * yy), 0.f);
  dY[10] = make_float3(kC3[1] * y * z, kC3[1] * x * z, kC3[1] * x * y);
  dY[11] = make_float3(-2.f * kC3[2] * x * y, kC3[2] * (4.f * zz - xx - 3.f * yy), 8.f * kC3[2] * y * z);
  dY[12] = make_float3(-6.f * kC3[3] * x * z, -6.f * kC3[3] * y * z, kC3[3] * (6.f * zz - 3.f * xx - 3.f * yy));
  dY[13] = make_float3(kC3[4] * (4.f * zz - 3.f * xx - yy), -2.f * kC3[4] * x * y, 8.f * kC3[4] * x * z);
  dY[14] = make_float3(2.f * kC3[5] * x * z, -2.f * kC3[5] * y * z, kC3[5] * (xx - yy));
  dY[15] = make_float3(kC3[6] * (3.f * xx - 3.f * yy), -6.f * kC3[6] * x * y, 0.f);
}

struct GaussCam {
  const float* view;
  const float* proj;
  float cx, cy, cz;  // camera position
  int W, H;
  unsigned gx, gy;
  float fx, fy, limx, limy, near_plane, mod;
  int deg, M;
};

// Rotation matrix of the normalised quaternion (r, x, y, z), rows R[0..2].
struct Rot {
  float r, x, y, z, n;  // normalised components and the input norm
  float R[3][3];
};
__device__ __forceinline__ Rot rotation(float4 q) {
  Rot o;
  o.n = fsqrt(fadd(fadd(fadd(fmul(q.x, q.x), fmul(q.y, q.y)), fmul(q.z, q.z)), fmul(q.w, q.w)));
  o.r = fdiv(q.x, o.n);
  o.x = fdiv(q.y, o.n);
  o.y = fdiv(q.z, o.n);
  o.z = fdiv(q.w, o.n);
  const float r = o.r, x = o.x, y = o.y, z = o.z;
  o.R[0][0] = fsub(1.0f, fmul(2.0f, fadd(fmul(y, y), fmul(z, z))));
  o.R[0][1] = fmul(2.0f, fsub(fmul(x, y), fmul(r, z)));
  o.R[0][2] = fmul(2.0f, fadd(fmul(x, z), fmul(r, y)));
  o.R[1][0] = fmul(2.0f, fadd(fmul(x, y), fmul(r, z)));
  o.R[1][1] = fsub(1.0f, fmul(2.0f, fadd(fmul(x, x), fmul(z, z))));
  o.R[1][2] = fmul(2.0f, fsub(fmul(y, z), fmul(r, x)));
  o.R[2][0] = fmul(2.0f, fsub(fmul(x, z), fmul(r, y)));
  o.R[2][1] = fmul(2.0f, fadd(fmul(y, z), fmul(r, x)));
  o.R[2][2] = fsub(1.0f, fmul(2.0f, fadd(fmul(x, x), fmul(y, y))));
  return o;
}

// Everything of the forward that the backward needs again.
struct GaussFwd {
  float3 t;        // view-space position
  float3 h;        // proj * p: x, y, w
  float pw;        // 1 / (w + 1e-7)
  Rot rot;
  float s[3];      // modified scales
  float M[3][3];   // R diag(s)
  float S[6];      // Sigma: xx, xy, xz, yy, yz, zz
  float txc, tyc;  // clamped t.x, t.y
  bool clx, cly;   // the clamps were active
  float J00, J02, J11, J12;
  float u0[3], u1[3];  // rows of J W
  float a, b, c, det;
};

__device__ __forceinline__ float sym(const float* S, int i, int j) {
  const int k = i <= j ? (i == 0 ? j : (i == 1 ? 2 + j : 5)) : (j == 0 ? i : (j == 1 ? 2 + i : 5));
  return S[k];
}

// Forward geometry up to the 2D covariance; false when culled at the near plane.
__device__ __forceinline__ bool gauss_geometry(const GaussCam& cm, float3 p, float3 sc, float4 q, GaussFwd& f) {
  f.t = t43(p, cm.view);
  if (f.t.z <= cm.near_plane) return false;
  f.h = t44_xyw(p, cm.proj);
  f.pw = fdiv(1.0f, fadd(f.h.z, 0.0000001f));
  f.rot = rotation(q);
  f.s[0] = fmul(cm.mod, sc.x);
  f.s[1] = fmul(cm.mod, sc.y);
  f.s[2] = fmul(cm.mod, sc.z);
#pragma unroll
  for (int j = 0; j < 3; j++)
#pragma unroll
    for (int k = 0; k < 3; k++) f.M[j][k] = fmul(f.rot.R[j][k], f.s[k]);
  const int ia[6] = {0, 0, 0, 1, 1, 2}, ib[6] = {0, 1, 2, 1, 2, 2};
#pragma unroll
  for (int e = 0; e < 6; e++) {
    const int a = ia[e], b = ib[e];
    f.S[e] = fadd(fadd(fmul(f.M[a][0], f.M[b][0]), fmul(f.M[a][1], f.M[b][1])), fmul(f.M[a][2], f.M[b][2]));
  }
  const float tz = f.t.z;
  const float txtz = fdiv(f.t.x, tz), tytz = fdiv(f.t.y, tz);
  f.clx = txtz < -cm.limx || txtz > cm.limx;
  f.cly = tytz < -cm.limy || tytz > cm.limy;
  f.txc = fmul(fminf(cm.limx, fmaxf(-cm.limx, txtz)), tz);
  f.tyc = fmul(fminf(cm.limy, fmaxf(-cm.limy, tytz)), tz);
  const float tz2 = fmul(tz, tz);
  f.J00 = fdiv(cm.fx, tz);
  f.J02 = -fdiv(fmul(cm.fx, f.txc), tz2);
  f.J11 = fdiv(cm.fy, tz);
  f.J12 = -fdiv(fmul(cm.fy, f.tyc), tz2);
  // W rows: (m0, m4, m8), (m1, m5, m9), (m2, m6, m10)
  const float* m = cm.view;
#pragma unroll
  for (int k = 0; k < 3; k++) {
    f.u0[k] = fadd(fmul(f.J00, m[4 * k]), fmul(f.J02, m[4 * k + 2]));
    f.u1[k] = fadd(fmul(f.J11, m[4 * k + 1]), fmul(f.J12, m[4 * k + 2]));
  }
  float v[3], w[3];
#pragma unroll
  for (int i = 0; i < 3; i++) {
    v[i] = fadd(fadd(fmul(sym(f.S, i, 0), f.u0[0]), fmul(sym(f.S, i, 1), f.u0[1])), fmul(sym(f.S, i, 2), f.u0[2]));
    w[i] = fadd(fadd(fmul(sym(f.S, i, 0), f.u1[0]), fmul(sym(f.S, i, 1), f.u1[1])), fmul(sym(f.S, i, 2), f.u1[2]));
  }
  f.a = fadd(fadd(fadd(fmul(f.u0[0], v[0]), fmul(f.u0[1], v[1])), fmul(f.u0[2], v[2])), 0.3f);
  f.b = fadd(fadd(fmul(f.u1[0], v[0]), fmul(f.u1[1], v[1])), fmul(f.u1[2], v[2]));
  f.c = fadd(fadd(fadd(fmul(f.u1[0], w[0]), fmul(f.u1[1], w[1])), fmul(f.u1[2], w[2])), 0.3f);
  f.det = fsub(fmul(f.a, f.c), fmul(f.b, f.b));
  return true;
}

// Shared-memory row stride (floats) of one Gaussian's `per` SH floats: odd, so
// the threads of a warp, each reading its own row element by element, hit
// distinct banks (a stride of 48 would put 16 threads on each bank).
__host__ __device__ inline int sh_stride(int per) { return per | 1; }

// Stages the block's n rows of `per` floats (contiguous at src) into padded
// shared rows with coalesced global loads (16-byte when the rows allow it).
__device__ __forceinline__ void stage_in(float* dst, const float* __restrict__ src, int n, int per, int stride) {
  const int count = n * per;
  if ((((uintptr_t)src) & 15u) == 0 && per % 4 == 0) {
    const float4* g4 = reinterpret_cast<const float4*>(src);
    for (int i = threadIdx.x; i < (count >> 2); i += blockDim.x) {
      const float4 v = __ldg(g4 + i);
      const int e = 4 * i, row = e / per;
      float* d = dst + row * stride + (e - row * per);
      d[0] = v.x; d[1] = v.y; d[2] = v.z; d[3] = v.w;
    }
  } else {
    for (int i = threadIdx.x; i < count; i += blockDim.x) dst[(i / per) * stride + i % per] = __ldg(src + i);
  }
}
__device__ __forceinline__ void stage_out(float* __restrict__ dst, const float* src, int n, int per, int stride) {
  const int count = n * per;
  if ((((uintptr_t)dst) & 15u) == 0 && per % 4 == 0) {
    float4* g4 = reinterpret_cast<float4*>(dst);
    for (int i = threadIdx.x; i < (count >> 2); i += blockDim.x) {
      const int e = 4 * i, row = e / per;
      const float* s = src + row * stride + (e - row * per);
      g4[i] = make_float4(s[0], s[1], s[2], s[3]);
    }
  } else {
    for (int i = threadIdx.x; i < count; i += blockDim.x) dst[i] = src[(i / per) * stride + i % per];
  }
}

// One thread per Gaussian; the block's SH coefficients (the bulk of the input)
// come through shared memory with coalesced 16-byte loads.
__global__ void __launch_bounds__(kGaussThreads) gauss_preprocess_kernel(
    int P, GaussCam cm, const float* __restrict__ means3D, const float* __restrict__ scales,
    const float* __restrict__ rotations, const float* __restrict__ opacities, const float* __restrict__ shs,
    int* __restrict__ radii, float* __restrict__ means2D, float* __restrict__ depths, float* __restrict__ cov3D,
    float* __restrict__ conic_opacity, float* __restrict__ rgb, uint8_t* __restrict__ clamped,
    uint32_t* __restrict__ tiles_touched) {
  extern __shared__ float4 sh_smem4[];
  float* sh_s = reinterpret_cast<float*>(sh_smem4);
  const int i0 = blockIdx.x * kGaussThreads;
  const int n = min(kGaussThreads, P - i0);
  const int per = cm.M * 3, stride = sh_stride(per);
  stage_in(sh_s, shs + (size_t)i0 * per, n, per, stride);
  __syncthreads();
  const int i = i0 + (int)threadIdx.x;
  if (i >= P) return;

  radii[i] = 0;
  tiles_touched[i] = 0;
  means2D[2 * i] = 0.0f;
  means2D[2 * i + 1] = 0.0f;
  depths[i] = 0.0f;
  reinterpret_cast<float4*>(conic_opacity)[i] = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
  for (int k = 0; k < 6; k++) cov3D[6 * i + k] = 0.0f;
#pragma unroll
  for (int k = 0; k < 3; k++) {
    rgb[3 * i + k] = 0.0f;
    clamped[3 * i + k] = 0;
  }
  const float3 p = make_float3(means3D[3 * i], means3D[3 * i + 1], means3D[3 * i + 2]);
  const float3 sc = make_float3(scales[3 * i], scales[3 * i + 1], scales[3 * i + 2]);
  const float4 q = reinterpret_cast<const float4*>(rotations)[i];
  GaussFwd f;
  if (!gauss_geometry(cm, p, sc, q, f)) return;
  if (f.det == 0.0f) return;
  const float idet = fdiv(1.0f, f.det);
  const float mid = fmul(0.5f, fadd(f.a, f.c));
  const float disc = fsqrt(fmaxf(0.1f, fsub(fmul(mid, mid), f.det)));
  const float l1 = fadd(mid, disc), l2 = fsub(mid, disc);
  const int r = (int)ceilf(fmul(3.0f, fsqrt(fmaxf(l1, l2))));
  const float2 m2 = make_float2(ndc2pix(fmul(f.h.x, f.pw), cm.W), ndc2pix(fmul(f.h.y, f.pw), cm.H));
  uint2 mn, mx;
  get_rect(m2, r, cm.gx, cm.gy, mn, mx);
  const uint32_t area = (mx.x - mn.x) * (mx.y - mn.y);
  if (area == 0) return;

  // colour from the spherical harmonics
  const float dx = fsub(p.x, cm.cx), dy = fsub(p.y, cm.cy), dz = fsub(p.z, cm.cz);
  const float len = fsqrt(fadd(fadd(fmul(dx, dx), fmul(dy, dy)), fmul(dz, dz)));
  const float x = fdiv(dx, len), y = fdiv(dy, len), z = fdiv(dz, len);
  float Y[kMaxShCoeffs];
  sh_basis(x, y, z, cm.deg, Y);
  const int nb = (cm.deg + 1) * (cm.deg + 1);
  const float* sh = sh_s + threadIdx.x * stride;
  float col[3] = {0.f, 0.f, 0.f};
#pragma unroll
  for (int k = 0; k < kMaxShCoeffs; k++) {
    if (k < nb) {
#pragma unroll
      for (int ch = 0; ch < 3; ch++) col[ch] = fadd(col[ch], fmul(Y[k], sh[3 * k + ch]));
    }
  }
#pragma unroll
  for (int ch = 0; ch < 3; ch++) {
    const float v = fadd(col[ch], 0.5f);
    clamped[3 * i + ch] = v < 0.0f ? 1 : 0;
    rgb[3 * i + ch] = fmaxf(v, 0.0f);
  }
  radii[i] = r;
  tiles_touched[i] = area;
  means2D[2 * i] = m2.x;
  means2D[2 * i + 1] = m2.y;
  depths[i] = f.t.z;
  reinterpret_cast<float4*>(conic_opacity)[i] =
      make_float4(fmul(f.c, idet), fmul(-f.b, idet), fmul(f.a, idet), opacities[i]);
#pragma unroll
  for (int k = 0; k < 6; k++) cov3D[6 * i + k] = f.S[k];
}

// Exact derivative of gauss_preprocess_kernel's outputs means2D, depths, cov3D,
// conic (x, y, z of conic_opacity) and rgb with respect to means3D, scales,
// rotations and shs.  The SH gradients leave through shared memory with
// coalesced 16-byte stores.
__global__ void __launch_bounds__(kGaussThreads, 5) gauss_backward_kernel(
    int P, GaussCam cm, const float* __restrict__ means3D, const float* __restrict__ scales,
    const float* __restrict__ rotations, const float* __restrict__ shs, const int* __restrict__ radii,
    const uint8_t* __restrict__ clamped, const float* __restrict__ dL_dmeans2D, const float* __restrict__ dL_ddepths,
    const float* __restrict__ dL_dcov3D, const float* __restrict__ dL_dconic, const float* __restrict__ dL_drgb,
    float* __restrict__ dL_dmeans3D, float* __restrict__ dL_dscales, float* __restrict__ dL_drotations,
    float* __restrict__ dL_dshs) {
  extern __shared__ float4 sh_smem4[];
  float* sh_s = reinterpret_cast<float*>(sh_smem4);
  const int i0 = blockIdx.x * kGaussThreads;
  const int n = min(kGaussThreads, P - i0);
  const int per = cm.M * 3, stride = sh_stride(per);
  stage_in(sh_s, shs + (size_t)i0 * per, n, per, stride);
  __syncthreads();
  const int i = i0 + (int)threadIdx.x;
  float* dsh = sh_s + threadIdx.x * stride;  // this Gaussian's coefficients, then their gradients
  bool live = i < P && radii[i] > 0;
  float3 dp = make_float3(0.f, 0.f, 0.f);
  float dsc[3] = {0.f, 0.f, 0.f}, dq[4] = {0.f, 0.f, 0.f, 0.f};
  if (live) {
    const float3 p = make_float3(means3D[3 * i], means3D[3 * i + 1], means3D[3 * i + 2]);
    const float3 sc = make_float3(scales[3 * i], scales[3 * i + 1], scales[3 * i + 2]);
    const float4 q = reinterpret_cast<const float4*>(rotations)[i];
    GaussFwd f;
    live = gauss_geometry(cm, p, sc, q, f);
    if (live) {
      // ---- colour -> SH coefficients and direction
      const float dxv = p.x - cm.cx, dyv = p.y - cm.cy, dzv = p.z - cm.cz;
      const float len = fsqrt(fadd(fadd(fmul(dxv, dxv), fmul(dyv, dyv)), fmul(dzv, dzv)));
      const float x = fdiv(dxv, len), y = fdiv(dyv, len), z = fdiv(dzv, len);
      float Y[kMaxShCoeffs];
      float3 dY[kMaxShCoeffs];
      sh_basis(x, y, z, cm.deg, Y);
      sh_basis_grad(x, y, z, cm.deg, dY);
      const int nb = (cm.deg + 1) * (cm.deg + 1);
      float g[3];
#pragma unroll
      for (int ch = 0; ch < 3; ch++) g[ch] = clamped[3 * i + ch] ? 0.0f : dL_drgb[3 * i + ch];
      float3 ddir = make_float3(0.f, 0.f, 0.f);
#pragma unroll
      for (int k = 0; k < kMaxShCoeffs; k++) {
        if (k < nb) {
          float sdot = 0.0f;
#pragma unroll
          for (int ch = 0; ch < 3; ch++) {
            sdot += dsh[3 * k + ch] * g[ch];
            dsh[3 * k + ch] = Y[k] * g[ch];
          }
          ddir.x += dY[k].x * sdot;
          ddir.y += dY[k].y * sdot;
          ddir.z += dY[k].z * sdot;
        }
      }
      for (int k = nb; k < cm.M; k++) dsh[3 * k] = dsh[3 * k + 1] = dsh[3 * k + 2] = 0.0f;
      const float dd = x * ddir.x + y * ddir.y + z * ddir.z;
      dp.x += (ddir.x - x * dd) / len;
      dp.y += (ddir.y - y * dd) / len;
      dp.z += (ddir.z - z * dd) / len;

      // ---- conic -> (a, b, c); A = c/det, B = -b/det, C = a/det, det = ac - b^2
      const float a = f.a, b = f.b, c = f.c, det = f.det;
      const float gA = dL_dconic[4 * i], gB = dL_dconic[4 * i + 1], gC = dL_dconic[4 * i + 2];
      const float id2 = 1.0f / (det * det);
      float da = (-c * c * gA + b * c * gB - b * b * gC) * id2;
      float db = (2.f * b * c * gA - (a * c + b * b) * gB + 2.f * a * b * gC) * id2;
      float dc = (-b * b * gA + a * b * gB - a * a * gC) * id2;
      if (det == 0.0f) da = db = dc = 0.0f;  // culled in the forward (radii == 0 already)

      // ---- (a, b, c) -> Sigma and the rows u0, u1 of J W
      // a = u0 S u0^T, b = u1 S u0^T, c = u1 S u1^T; G[i][j] = dL/dSigma_ij (entries independent)
      float G[3][3];
#pragma unroll
      for (int r = 0; r < 3; r++)
#pragma unroll
        for (int s = 0; s < 3; s++) G[r][s] = da * f.u0[r] * f.u0[s] + db * f.u1[r] * f.u0[s] + dc * f.u1[r] * f.u1[s];
      // the stored cov3D entries feed Sigma directly: one entry of G each
      {
        const int ia[6] = {0, 0, 0, 1, 1, 2}, ib[6] = {0, 1, 2, 1, 2, 2};
#pragma unroll
        for (int e = 0; e < 6; e++) G[ia[e]][ib[e]] += dL_dcov3D[6 * i + e];
      }
      float Su0[3], Su1[3];
#pragma unroll
      for (int r = 0; r < 3; r++) {
        Su0[r] = sym(f.S, r, 0) * f.u0[0] + sym(f.S, r, 1) * f.u0[1] + sym(f.S, r, 2) * f.u0[2];
        Su1[r] = sym(f.S, r, 0) * f.u1[0] + sym(f.S, r, 1) * f.u1[1] + sym(f.S, r, 2) * f.u1[2];
      }
      float du0[3], du1[3];
#pragma unroll
      for (int k = 0; k < 3; k++) {
        du0[k] = 2.f * da * Su0[k] + db * Su1[k];
        du1[k] = db * Su0[k] + 2.f * dc * Su1[k];
      }
      // ---- u = J W -> J
      const float* m = cm.view;
      float dJ00 = 0.f, dJ02 = 0.f, dJ11 = 0.f, dJ12 = 0.f;
#pragma unroll
      for (int k = 0; k < 3; k++) {
        dJ00 += du0[k] * m[4 * k];
        dJ02 += du0[k] * m[4 * k + 2];
        dJ11 += du1[k] * m[4 * k + 1];
        dJ12 += du1[k] * m[4 * k + 2];
      }
      // ---- J -> t (with the clamps of t.x / t.z and t.y / t.z)
      const float tz = f.t.z, itz = 1.0f / tz, itz2 = itz * itz, itz3 = itz2 * itz;
      float3 dt = make_float3(0.f, 0.f, 0.f);
      dt.z += -dJ00 * cm.fx * itz2 + dJ02 * 2.f * cm.fx * f.txc * itz3 - dJ11 * cm.fy * itz2 +
              dJ12 * 2.f * cm.fy * f.tyc * itz3;
      const float dtxc = -dJ02 * cm.fx * itz2, dtyc = -dJ12 * cm.fy * itz2;
      const float txtz = fdiv(f.t.x, tz), tytz = fdiv(f.t.y, tz);
      if (f.clx) dt.z += dtxc * (txtz < 0.f ? -cm.limx : cm.limx);
      else dt.x += dtxc;  // txc = (t.x / t.z) t.z
      if (f.cly) dt.z += dtyc * (tytz < 0.f ? -cm.limy : cm.limy);
      else dt.y += dtyc;
      dt.z += dL_ddepths ? dL_ddepths[i] : 0.0f;
      // t = view * p
      dp.x += m[0] * dt.x + m[1] * dt.y + m[2] * dt.z;
      dp.y += m[4] * dt.x + m[5] * dt.y + m[6] * dt.z;
      dp.z += m[8] * dt.x + m[9] * dt.y + m[10] * dt.z;

      // ---- means2D -> p through the projection
      const float gx = dL_dmeans2D[2 * i] * 0.5f * (float)cm.W, gy = dL_dmeans2D[2 * i + 1] * 0.5f * (float)cm.H;
      const float dhx = gx * f.pw, dhy = gy * f.pw, dhw = -(gx * f.h.x + gy * f.h.y) * f.pw * f.pw;
      const float* pr = cm.proj;
      dp.x += pr[0] * dhx + pr[1] * dhy + pr[3] * dhw;
      dp.y += pr[4] * dhx + pr[5] * dhy + pr[7] * dhw;
      dp.z += pr[8] * dhx + pr[9] * dhy + pr[11] * dhw;

      // ---- Sigma = M M^T, M = R diag(s): dL/dM = (G + G^T) M
      float dR[3][3];
#pragma unroll
      for (int j = 0; j < 3; j++)
#pragma unroll
        for (int k = 0; k < 3; k++) {
          const float dM = (G[j][0] + G[0][j]) * f.M[0][k] + (G[j][1] + G[1][j]) * f.M[1][k] +
                           (G[j][2] + G[2][j]) * f.M[2][k];
          dR[j][k] = dM * f.s[k];
          dsc[k] += dM * f.rot.R[j][k];
        }
#pragma unroll
      for (int k = 0; k < 3; k++) dsc[k] *= cm.mod;
      // R(q^) -> q^ -> q
      const float r = f.rot.r, x4 = f.rot.x, y4 = f.rot.y, z4 = f.rot.z;
      float gr = 0.f, gxq = 0.f, gyq = 0.f, gzq = 0.f;
      gyq += -4.f * y4 * dR[0][0]; gzq += -4.f * z4 * dR[0][0];
      gxq += 2.f * y4 * dR[0][1]; gyq += 2.f * x4 * dR[0][1]; gr += -2.f * z4 * dR[0][1]; gzq += -2.f * r * dR[0][1];
      gxq += 2.f * z4 * dR[0][2]; gzq += 2.f * x4 * dR[0][2]; gr += 2.f * y4 * dR[0][2]; gyq += 2.f * r * dR[0][2];
      gxq += 2.f * y4 * dR[1][0]; gyq += 2.f * x4 * dR[1][0]; gr += 2.f * z4 * dR[1][0]; gzq += 2.f * r * dR[1][0];
      gxq += -4.f * x4 * dR[1][1]; gzq += -4.f * z4 * dR[1][1];
      gyq += 2.f * z4 * dR[1][2]; gzq += 2.f * y4 * dR[1][2]; gr += -2.f * x4 * dR[1][2]; gxq += -2.f * r * dR[1][2];
      gxq += 2.f * z4 * dR[2][0]; gzq += 2.f * x4 * dR[2][0]; gr += -2.f * y4 * dR[2][0]; gyq += -2.f * r * dR[2][0];
      gyq += 2.f * z4 * dR[2][1]; gzq += 2.f * y4 * dR[2][1]; gr += 2.f * x4 * dR[2][1]; gxq += 2.f * r * dR[2][1];
      gxq += -4.f * x4 * dR[2][2]; gyq += -4.f * y4 * dR[2][2];
      const float qd = r * gr + x4 * gxq + y4 * gyq + z4 * gzq, in = 1.0f / f.rot.n;
      dq[0] = (gr - r * qd) * in;
      dq[1] = (gxq - x4 * qd) * in;
      dq[2] = (gyq - y4 * qd) * in;
      dq[3] = (gzq - z4 * qd) * in;
    }
  }
  if (!live && i < P)
    for (int k = 0; k < per; k++) dsh[k] = 0.0f;
  if (i < P) {
    dL_dmeans3D[3 * i] = dp.x;
    dL_dmeans3D[3 * i + 1] = dp.y;
    dL_dmeans3D[3 * i + 2] = dp.z;
#pragma unroll
    for (int k = 0; k < 3; k++) dL_dscales[3 * i + k] = dsc[k];
    reinterpret_cast<float4*>(dL_drotations)[i] = make_float4(dq[0], dq[1], dq[2], dq[3]);
  }
  __syncthreads();
  stage_out(dL_dshs + (size_t)i0 * per, sh_s, n, per, stride);
}

__global__ void __launch_bounds__(256) gauss_depth_keys_kernel(int P, const float* __restrict__ depths,
                                                               const uint32_t* __restrict__ tiles_touched,
                                                               uint32_t* __restrict__ keys, uint32_t* __restrict__ idx) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= P) return;
  keys[i] = tiles_touched[i] ? __float_as_uint(depths[i]) : 0xffffffffu;
  idx[i] = (uint32_t)i;
}

int gfail(int code, const char* fmt, long long a = 0, long long b = 0) {
  char buf[256];
  snprintf(buf, sizeof buf, fmt, a, b);
  return set_error(code, buf);
}

int make_cam(GaussCam& cm, int P, int deg, int M, float mod, const float* view, const float* proj, const float* cam,
             int W, int H, float tanx, float tany, float near_plane) {
  if (P < 0 || W <= 0 || H <= 0) return gfail(VI_ERR_INVALID_ARGUMENT, "gaussians: bad sizes P=%lld, W*H=%lld", P, (long long)W * H);
  if (deg < 0 || deg > 3) return gfail(VI_ERR_UNSUPPORTED, "gaussians: sh_degree=%lld (0..3 supported)", deg);
  if (M < (deg + 1) * (deg + 1) || M > kMaxShCoeffs)
    return gfail(VI_ERR_INVALID_ARGUMENT, "gaussians: %lld SH coefficients per Gaussian for degree %lld", M, deg);
  if (!(tanx > 0.f) || !(tany > 0.f)) return gfail(VI_ERR_INVALID_ARGUMENT, "gaussians: tan_fov must be positive");
  if (P > 0 && (!view || !proj || !cam)) return gfail(VI_ERR_INVALID_ARGUMENT, "gaussians: a camera pointer is NULL");
  cm.view = view;
  cm.proj = proj;
  cm.W = W;
  cm.H = H;
  cm.gx = (unsigned)(W + VI_TILE - 1) / VI_TILE;
  cm.gy = (unsigned)(H + VI_TILE - 1) / VI_TILE;
  cm.fx = cm.fy = cm.limx = cm.limy = 0.0f;  // set by host_camera
  cm.cx = cm.cy = cm.cz = 0.0f;
  cm.mod = mod;
  cm.deg = deg;
  cm.M = M;
  cm.near_plane = near_plane;
  return VI_OK;
}

}  // namespace
}  // namespace vi

using namespace vi;

namespace {

// Host-side camera constants: the focal lengths and clamp limits are rounded
// once, in float, exactly as the CPU restatement forms them.
void host_camera(GaussCam& cm, const float* cam_pos_host, float tanx, float tany) {
  const volatile float two_tx = 2.0f * tanx, two_ty = 2.0f * tany;
  cm.fx = (float)cm.W / two_tx;
  cm.fy = (float)cm.H / two_ty;
  cm.limx = 1.3f * tanx;
  cm.limy = 1.3f * tany;
  cm.cx = cam_pos_host[0];
  cm.cy = cam_pos_host[1];
  cm.cz = cam_pos_host[2];
}

}  // namespace

extern "C" int vi_preprocess_gaussians(int P, int sh_degree, int sh_coeffs, const float* means3D, const float* scales,
                                       const float* rotations, const float* opacities, const float* shs,
                                       float scale_modifier, const float* viewmatrix, const float* projmatrix,
                                       const float* cam_pos_host, int image_width, int image_height, float tan_fovx,
                                       float tan_fovy, float near_plane, int* radii, float* means2D, float* depths,
                                       float* cov3D, float* conic_opacity, float* rgb, uint8_t* clamped,
                                       uint32_t* tiles_touched, void* stream) {
  GaussCam cm;
  int rc = make_cam(cm, P, sh_degree, sh_coeffs, scale_modifier, viewmatrix, projmatrix, cam_pos_host, image_width,
                    image_height, tan_fovx, tan_fovy, near_plane);
  if (rc) return rc;
  if (P == 0) return VI_OK;
  if (!means3D || !scales || !rotations || !opacities || !shs || !radii || !means2D || !depths || !cov3D ||
      !conic_opacity || !rgb || !clamped || !tiles_touched)
    return gfail(VI_ERR_INVALID_ARGUMENT, "vi_preprocess_gaussians: a required pointer is NULL");
  if (((uintptr_t)rotations & 15u) || ((uintptr_t)conic_opacity & 15u))
    return gfail(VI_ERR_INVALID_ARGUMENT, "vi_preprocess_gaussians: rotations and conic_opacity must be 16-byte aligned");
  host_camera(cm, cam_pos_host, tan_fovx, tan_fovy);
  const size_t smem = sizeof(float) * (size_t)kGaussThreads * sh_stride(sh_coeffs * 3);
  cudaFuncSetAttribute(gauss_preprocess_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  gauss_preprocess_kernel<<<(P + kGaussThreads - 1) / kGaussThreads, kGaussThreads, smem, (cudaStream_t)stream>>>(
      P, cm, means3D, scales, rotations, opacities, shs, radii, means2D, depths, cov3D, conic_opacity, rgb, clamped,
      tiles_touched);
  note_launches(1);
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return set_error(VI_ERR_CUDA, cudaGetErrorString(e));
  return VI_OK;
}

extern "C" int vi_preprocess_gaussians_backward(
    int P, int sh_degree, int sh_coeffs, const float* means3D, const float* scales, const float* rotations,
    const float* shs, float scale_modifier, const float* viewmatrix, const float* projmatrix, const float* cam_pos_host,
    int image_width, int image_height, float tan_fovx, float tan_fovy, float near_plane, const int* radii,
    const uint8_t* clamped, const float* dL_dmeans2D, const float* dL_ddepths, const float* dL_dcov3D,
    const float* dL_dconic_opacity, const float* dL_drgb, float* dL_dmeans3D, float* dL_dscales,
    float* dL_drotations, float* dL_dshs, void* stream) {
  GaussCam cm;
  int rc = make_cam(cm, P, sh_degree, sh_coeffs, scale_modifier, viewmatrix, projmatrix, cam_pos_host, image_width,
                    image_height, tan_fovx, tan_fovy, near_plane);
  if (rc) return rc;
  if (P == 0) return VI_OK;
  if (!means3D || !scales || !rotations || !shs || !radii || !clamped || !dL_dmeans2D || !dL_dcov3D ||
      !dL_dconic_opacity || !dL_drgb || !dL_dmeans3D || !dL_dscales || !dL_drotations || !dL_dshs)
    return gfail(VI_ERR_INVALID_ARGUMENT, "vi_preprocess_gaussians_backward: a required pointer is NULL");
  if (((uintptr_t)rotations & 15u) || ((uintptr_t)dL_drotations & 15u))
    return gfail(VI_ERR_INVALID_ARGUMENT, "vi_preprocess_gaussians_backward: rotations must be 16-byte aligned");
  host_camera(cm, cam_pos_host, tan_fovx, tan_fovy);
  const size_t smem = sizeof(float) * (size_t)kGaussThreads * sh_stride(sh_coeffs * 3);
  cudaFuncSetAttribute(gauss_backward_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  gauss_backward_kernel<<<(P + kGaussThreads - 1) / kGaussThreads, kGaussThreads, smem, (cudaStream_t)stream>>>(
      P, cm, means3D, scales, rotations, shs, radii, clamped, dL_dmeans2D, dL_ddepths, dL_dcov3D, dL_dconic_opacity,
      dL_drgb, dL_dmeans3D, dL_dscales, dL_drotations, dL_dshs);
  note_launches(1);
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return set_error(VI_ERR_CUDA, cudaGetErrorString(e));
  return VI_OK;
}

namespace {

// Scratch of vi_bin_gaussians: the depth sort and scan over P, then the tile
// sort over R (the renderer's BinState), carved from one caller buffer.
struct GaussBin {
  GeomState g;
  BinState b;
  size_t bytes;
};

GaussBin gauss_bin_layout(char* base, size_t P, uint64_t R, int tb) {
  GaussBin o{};
  uintptr_t cur = 0;
  auto take = [&](size_t bytes) {
    cur = align_up(cur);
    char* p = reinterpret_cast<char*>(reinterpret_cast<uintptr_t>(base) + cur);
    cur += bytes;
    return p;
  };
  o.g.status = (uint32_t*)take(64 * sizeof(uint32_t));
  o.g.dkeys = (uint32_t*)take(P * 4);
  o.g.didx = (uint32_t*)take(P * 4);
  o.g.dkeys_alt = (uint32_t*)take(P * 4);
  o.g.didx_alt = (uint32_t*)take(P * 4);
  o.g.offsets = (uint32_t*)take(P * 4);
  o.g.block_sums = (uint32_t*)take(((P + kScanBlock - 1) / kScanBlock + 1) * 4);
  char* st = take(sort_temp_bytes(P, 4, 0, 32));
  sort_temp_carve(st, P, 4, 0, 32, o.g.sort);
  cur = align_up(cur);
  BinState sizing = bin_layout(nullptr, R, tb);
  char* bb = take(sizing.bytes);
  o.b = bin_layout(bb, R, tb);
  o.bytes = align_up(cur) + 256;
  return o;
}

}  // namespace

extern "C" uint64_t vi_bin_gaussians_scratch_bytes(int P, uint64_t num_rendered, int image_width, int image_height) {
  if (P < 0 || image_width <= 0 || image_height <= 0) return 0;
  const size_t tiles = (size_t)((image_width + VI_TILE - 1) / VI_TILE) * ((image_height + VI_TILE - 1) / VI_TILE);
  return gauss_bin_layout(nullptr, (size_t)P, num_rendered, tile_bits(tiles)).bytes;
}

extern "C" int vi_bin_gaussians(int P, int image_width, int image_height, const int* radii, const float* means2D,
                                const float* depths, const uint32_t* tiles_touched, uint64_t num_rendered,
                                void* scratch, uint64_t scratch_bytes, uint32_t* point_list, uint32_t* tile_ids,
                                uint32_t* ranges, void* stream) {
  if (P < 0 || image_width <= 0 || image_height <= 0)
    return gfail(VI_ERR_INVALID_ARGUMENT, "vi_bin_gaussians: bad sizes P=%lld, W*H=%lld", P,
                 (long long)image_width * image_height);
  cudaStream_t s = (cudaStream_t)stream;
  const unsigned gx = (unsigned)(image_width + VI_TILE - 1) / VI_TILE, gy = (unsigned)(image_height + VI_TILE - 1) / VI_TILE;
  const size_t tiles = (size_t)gx * gy;
  if (!ranges) return gfail(VI_ERR_INVALID_ARGUMENT, "vi_bin_gaussians: ranges is NULL");
  if (num_rendered >= (1ull << 30))
    return gfail(VI_ERR_TOO_MANY_OVERLAPS, "vi_bin_gaussians: %lld overlaps exceed 2^30", (long long)num_rendered);
  const int tb = tile_bits(tiles);
  const GaussBin need = gauss_bin_layout(nullptr, (size_t)P, num_rendered, tb);
  if (!scratch || scratch_bytes < need.bytes)
    return gfail(VI_ERR_INVALID_ARGUMENT, "vi_bin_gaussians: scratch of %lld bytes, %lld needed", (long long)scratch_bytes,
                 (long long)need.bytes);
  if (((uintptr_t)scratch) & 255u) return gfail(VI_ERR_INVALID_ARGUMENT, "vi_bin_gaussians: scratch must be 256-byte aligned");
  if (P > 0 && (!radii || !means2D || !depths || !tiles_touched))
    return gfail(VI_ERR_INVALID_ARGUMENT, "vi_bin_gaussians: a required input pointer is NULL");
  if (num_rendered > 0 && !point_list) return gfail(VI_ERR_INVALID_ARGUMENT, "vi_bin_gaussians: point_list is NULL");
  GaussBin gb = gauss_bin_layout((char*)scratch, (size_t)P, num_rendered, tb);
  Scene sc{};
  sc.P = P;
  sc.W = image_width;
  sc.H = image_height;
  sc.gx = gx;
  sc.gy = gy;
  gb.g.radii = const_cast<int*>(radii);
  gb.g.means2D = const_cast<float*>(means2D);
  gb.g.tiles_touched = const_cast<uint32_t*>(tiles_touched);
  cudaMemsetAsync(gb.g.status, 0, 64 * sizeof(uint32_t), s);
  uint64_t total = 0;
  const uint32_t* sorted_idx = gb.g.didx;
  if (P > 0) {
    gauss_depth_keys_kernel<<<(P + 255) / 256, 256, 0, s>>>(P, depths, tiles_touched, gb.g.dkeys, gb.g.didx);
    note_launches(1);
    const bool alt = onesweep_sort_u32(gb.g.dkeys, gb.g.didx, gb.g.dkeys_alt, gb.g.didx_alt, (uint64_t)P, 0, 32,
                                       gb.g.sort, gb.g.status, s);
    sorted_idx = alt ? gb.g.didx_alt : gb.g.didx;
    launch_offsets_scan(sc, gb.g, sorted_idx, s);
    uint32_t st[4] = {0, 0, 0, 0};
    cudaError_t e = begin_status_read(gb.g.status, s);
    if (e == cudaSuccess) e = finish_status_read(st);
    if (e != cudaSuccess) return set_error(VI_ERR_CUDA, cudaGetErrorString(e));
    if (st[0]) return gfail(VI_ERR_DEVICE, "vi_bin_gaussians: device status 0x%llx", st[0]);
    total = (uint64_t)st[2] | ((uint64_t)st[3] << 32);
  }
  if (total != num_rendered)
    return gfail(VI_ERR_INVALID_ARGUMENT, "vi_bin_gaussians: num_rendered=%lld but the tiles touched sum to %lld",
                 (long long)num_rendered, (long long)total);
  const uint32_t* sorted_tiles = gb.b.tkeys;
  const uint32_t* plist = gb.b.tvals;
  if (total > 0) {
    launch_duplicate(sc, gb.g, sorted_idx, gb.b, s);
    const bool alt = onesweep_sort_u32(gb.b.tkeys, gb.b.tvals, gb.b.tkeys_alt, gb.b.tvals_alt, total, 0, tb,
                                       gb.b.sort, gb.g.status, s);
    plist = alt ? gb.b.tvals_alt : gb.b.tvals;
    sorted_tiles = alt ? gb.b.tkeys_alt : gb.b.tkeys;
    cudaMemcpyAsync(point_list, plist, total * sizeof(uint32_t), cudaMemcpyDeviceToDevice, s);
    if (tile_ids) cudaMemcpyAsync(tile_ids, sorted_tiles, total * sizeof(uint32_t), cudaMemcpyDeviceToDevice, s);
  }
  launch_ranges(total, sorted_tiles, ranges, tiles, s);
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return set_error(VI_ERR_CUDA, cudaGetErrorString(e));
  return VI_OK;
}
