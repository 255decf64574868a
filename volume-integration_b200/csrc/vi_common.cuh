// Shared device helpers for the volume-integration renderer (sm_100a).
//
// Every floating-point helper whose result feeds a discrete decision (tile
// rectangles, pixel membership of a grid point, sort keys) is written with
// explicitly rounded intrinsics so nvcc cannot contract a*b+c into an FMA: the
// results are then bit-identical to the reference's written operation order
// (cuda_integrator/auxiliary.h:50-86, hashgrid.h:225-242 of the reference).
#pragma once
#include <climits>
#include <cstdint>
#include <cuda_runtime.h>

#define VI_TILE 16
#define VI_TILE_PIX 256

namespace vi {

// Status bits latched in the device status word (never a trap).
enum : uint32_t {
  VI_ERR_LOOKBACK_TIMEOUT = 1u << 0,  // a sort look-back gave up after its spin limit
  VI_ERR_RECORD_OVERFLOW = 1u << 1,   // more per-primitive records than grid points (cannot happen)
  VI_ERR_STAGE_TIMEOUT = 1u << 2,     // a render tile's bulk-copy wait gave up (it fell back to global reads)
};

struct Mat {
  float m[16];
};

__device__ __forceinline__ float fmul(float a, float b) { return __fmul_rn(a, b); }
__device__ __forceinline__ float fadd(float a, float b) { return __fadd_rn(a, b); }
__device__ __forceinline__ float fsub(float a, float b) { return __fsub_rn(a, b); }

// transformPoint4x3 (auxiliary.h:67-75): ((m0*x + m4*y) + m8*z) + m12, no contraction.
__device__ __forceinline__ float3 t43(float3 p, const float* __restrict__ m) {
  float3 r;
  r.x = fadd(fadd(fadd(fmul(m[0], p.x), fmul(m[4], p.y)), fmul(m[8], p.z)), m[12]);
  r.y = fadd(fadd(fadd(fmul(m[1], p.x), fmul(m[5], p.y)), fmul(m[9], p.z)), m[13]);
  r.z = fadd(fadd(fadd(fmul(m[2], p.x), fmul(m[6], p.y)), fmul(m[10], p.z)), m[14]);
  return r;
}

// transformPoint4x4 (auxiliary.h:77-86): only x, y and w are ever used.
__device__ __forceinline__ float3 t44_xyw(float3 p, const float* __restrict__ m) {
  float3 r;
  r.x = fadd(fadd(fadd(fmul(m[0], p.x), fmul(m[4], p.y)), fmul(m[8], p.z)), m[12]);
  r.y = fadd(fadd(fadd(fmul(m[1], p.x), fmul(m[5], p.y)), fmul(m[9], p.z)), m[13]);
  r.z = fadd(fadd(fadd(fmul(m[3], p.x), fmul(m[7], p.y)), fmul(m[11], p.z)), m[15]);
  return r;
}

// ndc2Pix (auxiliary.h:50-53) is evaluated in double by the reference.
__device__ __forceinline__ float ndc2pix(float v, int S) {
  return (float)(__dmul_rn(__dadd_rn(__dmul_rn(__dadd_rn((double)v, 1.0), (double)S), -1.0), 0.5));
}

// Screen position of a world point.  fwd: 1/(w+1e-7) (forward.cu:432);
// backward recompute: 1/w (backward.cu:325).
__device__ __forceinline__ float2 project(float3 p, const float* __restrict__ proj, int W, int H, bool fwd) {
  float3 h = t44_xyw(p, proj);
  float pw = fwd ? __fdiv_rn(1.0f, fadd(h.z, 0.0000001f)) : __fdiv_rn(1.0f, h.z);
  return make_float2(ndc2pix(fmul(h.x, pw), W), ndc2pix(fmul(h.y, pw), H));
}

// The pixel a screen point falls in, as used by `px <= s.x < px+1` tests
// (forward.cu:493-494): floor, with non-finite values mapped to a value that
// never equals a pixel coordinate.
__device__ __forceinline__ int pix_coord(float s) {
  float f = floorf(s);
  if (!(f >= -1.0e9f && f <= 1.0e9f)) return INT_MIN;
  return (int)f;
}

// Grid point position from precomputed (float(coord) - gof) offsets (forward.cu:421-428).
__device__ __forceinline__ float3 grid_pos_rel(float3 c, float3 rel, float step) {
  return make_float3(fadd(c.x, fmul(rel.x, step)), fadd(c.y, fmul(rel.y, step)), fadd(c.z, fmul(rel.z, step)));
}

// Grid point position (forward.cu:416-428).
__device__ __forceinline__ float3 grid_pos(float3 c, int g, int G, float step, float gof) {
  int z = g / (G * G), rem = g % (G * G), y = rem / G, x = rem % G;
  float3 p;
  p.x = fadd(c.x, fmul(fsub((float)x, gof), step));
  p.y = fadd(c.y, fmul(fsub((float)y, gof), step));
  p.z = fadd(c.z, fmul(fsub((float)z, gof), step));
  return p;
}

// Position normalised to the hashgrid box and clamped to [0, 1]: (p - lo) / ext
// per axis, where the reference's box is fixed at lo = -1.3, ext = 2.6
// (hashgrid.h:225-235).  It does not depend on the level, so callers compute it
// once per point.
__device__ __forceinline__ float3 hash_norm(float3 pos, const float* lo, const float* ext) {
  return make_float3(fmaxf(0.0f, fminf(1.0f, __fdiv_rn(fsub(pos.x, lo[0]), ext[0]))),
                     fmaxf(0.0f, fminf(1.0f, __fdiv_rn(fsub(pos.y, lo[1]), ext[1]))),
                     fmaxf(0.0f, fminf(1.0f, __fdiv_rn(fsub(pos.z, lo[2]), ext[2]))));
}

// floor of x for 0 <= x < 2^23 on the FMA and integer pipes: adding 2^23 with
// round-down leaves 2^23 + floor(x) exactly, so the integer floor is its bit
// pattern minus that of 2^23 and the float floor is exact as well.  Equal to
// floorf(x) and (int)floorf(x) on that range.
__device__ __forceinline__ void floor_small(float x, int& i, float& f) {
  const float y = __fadd_rd(x, 8388608.0f);
  i = __float_as_int(y) - 0x4b000000;
  f = fsub(y, 8388608.0f);
}

// Hashgrid level set-up (hashgrid.h:237-242): integer base corner and fractions.
// n is in [0, 1] and res < 2^23, so every product is in [0, 2^23).
__device__ __forceinline__ void level_setup_nf(float3 n, float rf, int3& b, float3& t) {
  float px = fmul(n.x, rf), py = fmul(n.y, rf), pz = fmul(n.z, rf);
  float fx, fy, fz;
  floor_small(px, b.x, fx);
  floor_small(py, b.y, fy);
  floor_small(pz, b.z, fz);
  t = make_float3(fsub(px, fx), fsub(py, fy), fsub(pz, fz));
}

__device__ __forceinline__ void level_setup(float3 pos, const float* lo, const float* ext, int res, int3& b, float3& t) {
  float3 n = hash_norm(pos, lo, ext);
  float rf = (float)res;
  float px = fmul(n.x, rf), py = fmul(n.y, rf), pz = fmul(n.z, rf);
  float fx = floorf(px), fy = floorf(py), fz = floorf(pz);
  b = make_int3((int)fx, (int)fy, (int)fz);
  t = make_float3(fsub(px, fx), fsub(py, fy), fsub(pz, fz));
}

// Table entry of one corner or -1 (hashgrid.h:258-275).  Tmask != 0 when T is a
// power of two (the modulo is then a mask, which is the same value).
__device__ __forceinline__ int corner_entry(int cx, int cy, int cz, int res, bool use_hash, uint32_t p0,
                                            uint32_t p1, uint32_t p2, uint32_t T, uint32_t Tmask) {
  if (use_hash) {
    uint32_t h = ((uint32_t)cx * p0) ^ ((uint32_t)cy * p1) ^ ((uint32_t)cz * p2);
    return (int)(Tmask ? (h & Tmask) : (h % T));
  }
  if (cx < 0 || cx >= res || cy < 0 || cy >= res || cz < 0 || cz >= res) return -1;
  uint32_t e = (uint32_t)cz * (uint32_t)res * (uint32_t)res + (uint32_t)cy * (uint32_t)res + (uint32_t)cx;
  return e >= T ? -1 : (int)e;
}

__device__ __forceinline__ float sigmoidf_(float x) { return 1.0f / (1.0f + expf(-x)); }

// getRect (auxiliary.h:55-65), with the float conversions of the reference.  The
// division by the tile size 16 is written as a multiplication by 0.0625: both
// round the same exact value x * 2^-4, so the result is identical.
__device__ __forceinline__ void get_rect(float2 p, int r, unsigned gx, unsigned gy, uint2& mn, uint2& mx) {
  float rf = (float)r;
  int a;
  a = max(0, (int)(fmul(fsub(p.x, rf), 0.0625f)));
  mn.x = min(gx, (unsigned)a);
  a = max(0, (int)(fmul(fsub(p.y, rf), 0.0625f)));
  mn.y = min(gy, (unsigned)a);
  a = max(0, (int)(fmul(fsub(fadd(fadd(p.x, rf), (float)VI_TILE), 1.0f), 0.0625f)));
  mx.x = min(gx, (unsigned)a);
  a = max(0, (int)(fmul(fsub(fadd(fadd(p.y, rf), (float)VI_TILE), 1.0f), 0.0625f)));
  mx.y = min(gy, (unsigned)a);
}


}  // namespace vi
