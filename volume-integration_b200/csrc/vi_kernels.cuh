// Device pieces shared by the feature, render and backward kernels.
#pragma once
#include "vi_common.cuh"
#include "vi_internal.h"

namespace vi {

// Stencil coefficients (forward.cu:297-323): genus 2 -> 5 taps, otherwise 3 taps.
struct Stencil {
  int S;
  float c[5];
};
__host__ __device__ inline Stencil make_stencil(int genus) {
  Stencil s;
  if (genus == 2) {
    s.S = 5;
    s.c[0] = 1.0f / 12.0f; s.c[1] = -2.0f / 3.0f; s.c[2] = 0.0f; s.c[3] = 2.0f / 3.0f; s.c[4] = -1.0f / 12.0f;
  } else {
    s.S = 3;
    s.c[0] = -0.5f; s.c[1] = 0.0f; s.c[2] = 0.5f; s.c[3] = 0.0f; s.c[4] = 0.0f;
  }
  return s;
}

// |d/dx| + |d/dy| + |d/dz| of an occupancy given as a bit per grid point
// (bit g set = grid point g occupied).  With conf>0 bits this is the forward's
// stencil (forward.cu:557-611); with "screen point in this pixel" bits it is the
// backward's (backward.cu:654-689).  Requires V <= 32.
__device__ __forceinline__ float occ_mag(uint32_t occ, int g, int G, const Stencil& st) {
  int z = g / (G * G), rem = g % (G * G), y = rem / G, x = rem % G, off = (st.S - 1) / 2;
  float gx = 0.0f, gy = 0.0f, gz = 0.0f;
  for (int s = 0; s < st.S; s++) {
    int r = s - off, n;
    n = x + r;
    if (n >= 0 && n < G && ((occ >> (z * G * G + y * G + n)) & 1u)) gx = fadd(gx, st.c[s]);
    n = y + r;
    if (n >= 0 && n < G && ((occ >> (z * G * G + n * G + x)) & 1u)) gy = fadd(gy, st.c[s]);
    n = z + r;
    if (n >= 0 && n < G && ((occ >> (n * G * G + y * G + x)) & 1u)) gz = fadd(gz, st.c[s]);
  }
  return fadd(fadd(fabsf(gx), fabsf(gy)), fabsf(gz));
}

// F contiguous table floats of one (entry, level).
template <int F>
struct FVec {
  float v[F];
};
template <int F>
__device__ __forceinline__ FVec<F> load_feat(const float* __restrict__ p) {
  FVec<F> r;
  if constexpr (F == 2) {
    float2 a = __ldg(reinterpret_cast<const float2*>(p));
    r.v[0] = a.x; r.v[1] = a.y;
  } else if constexpr (F == 4) {
    float4 a = __ldg(reinterpret_cast<const float4*>(p));
    r.v[0] = a.x; r.v[1] = a.y; r.v[2] = a.z; r.v[3] = a.w;
  } else if constexpr (F == 8) {
    float4 a = __ldg(reinterpret_cast<const float4*>(p));
    float4 b = __ldg(reinterpret_cast<const float4*>(p) + 1);
    r.v[0] = a.x; r.v[1] = a.y; r.v[2] = a.z; r.v[3] = a.w;
    r.v[4] = b.x; r.v[5] = b.y; r.v[6] = b.z; r.v[7] = b.w;
  } else {
#pragma unroll
    for (int f = 0; f < F; f++) r.v[f] = __ldg(p + f);
  }
  return r;
}

// Trilinear hashgrid features of one point, level by level (hashgrid.h:207-299).
// For each level, fn(l, acc) receives the F interpolated features.  Corners
// are visited dx, dy, dz as the reference does; corners whose trilinear weight
// is exactly zero are skipped (their product with a finite table value is
// zero, so the sum is unchanged), which is most corners of points clamped to
// the faces of the hashgrid box.
template <int F, typename Fn>
__device__ __forceinline__ void for_each_level(const Scene& sc, float3 pos, Fn&& fn) {
  const uint32_t p0 = (uint32_t)__ldg(sc.primes), p1 = (uint32_t)__ldg(sc.primes + 1),
                 p2 = (uint32_t)__ldg(sc.primes + 2);
  const float3 nrm = hash_norm(pos);
#pragma unroll 2
  for (int l = 0; l < sc.L; l++) {
    const int res = __ldg(sc.res + l);
    const bool hsh = __ldg(sc.do_hash + l) != 0;
    int3 b;
    float3 t;
    level_setup_n(nrm, res, b, t);
    float acc[F];
#pragma unroll
    for (int f = 0; f < F; f++) acc[f] = 0.0f;
    const float* lvl = sc.table + (size_t)l * F;
#pragma unroll
    for (int dx = 0; dx < 2; dx++) {
      const float wx = dx == 0 ? 1.0f - t.x : t.x;
#pragma unroll
      for (int dy = 0; dy < 2; dy++) {
        const float wy = dy == 0 ? 1.0f - t.y : t.y;
#pragma unroll
        for (int dz = 0; dz < 2; dz++) {
          const float wz = dz == 0 ? 1.0f - t.z : t.z;
          const float w = wx * wy * wz;
          if (w != 0.0f) {
            const int e = corner_entry(b.x + dx, b.y + dy, b.z + dz, res, hsh, p0, p1, p2, sc.T, sc.Tmask);
            if (e >= 0) {
              const FVec<F> v = load_feat<F>(lvl + (size_t)e * sc.L * F);
#pragma unroll
              for (int f = 0; f < F; f++) acc[f] += v.v[f] * w;
            }
          }
        }
      }
    }
    fn(l, acc, b, t, res, hsh);
  }
}

}  // namespace vi
