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

// Coordinates of grid point g (flat index z*G^2 + y*G + x) and its offset from the
// cube centre in grid steps, formed once per thread.
struct GridPt {
  int g, x, y, z;
  float3 rel;
};
__device__ __forceinline__ GridPt grid_point(int g, int G, float gof) {
  GridPt p;
  p.g = g;
  p.z = g / (G * G);
  const int rem = g % (G * G);
  p.y = rem / G;
  p.x = rem % G;
  p.rel = make_float3(fsub((float)p.x, gof), fsub((float)p.y, gof), fsub((float)p.z, gof));
  return p;
}

// |d/dx| + |d/dy| + |d/dz| of an occupancy given as a bit per grid point
// (bit g set = grid point g occupied).  With conf>0 bits this is the forward's
// stencil (forward.cu:557-611); with "screen point in this pixel" bits it is the
// backward's (backward.cu:654-689).  Requires V <= 32.
__device__ __forceinline__ float occ_mag(uint32_t occ, const GridPt& p, int G, const Stencil& st) {
  const int g = p.g, x = p.x, y = p.y, z = p.z;
  if (st.S == 3) {
    // Taps (-1/2, 0, 1/2): each axis term is +-1/2 exactly when one of the two
    // in-range neighbours is occupied, so the float sum is 0.5 * count (0..1.5).
    const int GG = G * G;
    const uint32_t xm = x > 0 ? (occ >> (g - 1)) & 1u : 0u, xp = x + 1 < G ? (occ >> (g + 1)) & 1u : 0u;
    const uint32_t ym = y > 0 ? (occ >> (g - G)) & 1u : 0u, yp = y + 1 < G ? (occ >> (g + G)) & 1u : 0u;
    const uint32_t zm = z > 0 ? (occ >> (g - GG)) & 1u : 0u, zp = z + 1 < G ? (occ >> (g + GG)) & 1u : 0u;
    const uint32_t n = (xm ^ xp) + (ym ^ yp) + (zm ^ zp);
    return (n & 1u ? 0.5f : 0.0f) + (n & 2u ? 1.0f : 0.0f);
  }
  const int off = (st.S - 1) / 2;
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
__device__ __forceinline__ float occ_mag(uint32_t occ, int g, int G, const Stencil& st) {
  return occ_mag(occ, grid_point(g, G, 0.0f), G, st);
}

// occ_mag for grids of more than 32 points (G = 4, 5): the occupancy is a bit
// array of 32-bit words (bit g of word g / 32).  Same taps, same order of
// additions as the reference loop (forward.cu:557-611, backward.cu:654-689).
__device__ __forceinline__ bool occ_bit(const uint32_t* occ, int i) { return (occ[i >> 5] >> (i & 31)) & 1u; }
__device__ __forceinline__ float occ_mag_w(const uint32_t* occ, const GridPt& p, int G, const Stencil& st) {
  const int x = p.x, y = p.y, z = p.z;
  const int off = (st.S - 1) / 2;
  float gx = 0.0f, gy = 0.0f, gz = 0.0f;
  for (int s = 0; s < st.S; s++) {
    int r = s - off, n;
    n = x + r;
    if (n >= 0 && n < G && occ_bit(occ, z * G * G + y * G + n)) gx = fadd(gx, st.c[s]);
    n = y + r;
    if (n >= 0 && n < G && occ_bit(occ, z * G * G + n * G + x)) gy = fadd(gy, st.c[s]);
    n = z + r;
    if (n >= 0 && n < G && occ_bit(occ, n * G * G + y * G + x)) gz = fadd(gz, st.c[s]);
  }
  return fadd(fadd(fabsf(gx), fabsf(gy)), fabsf(gz));
}

// Grids of more than 32 points are handled by block-per-primitive kernels
// (one thread per grid point, kWideThreads >= 125 = 5^3).
constexpr int kWideThreads = 128;
constexpr int kWideWords = kWideThreads / 32;

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

// The eight corners of one point at one hashgrid level (hashgrid.h:237-287).
// Corner k has offsets dx = k >> 2, dy = (k >> 1) & 1, dz = k & 1, so ascending k
// is the reference's dx, dy, dz nesting order.  Per-axis weights and index terms
// are formed once; `mask` has bit k set for every corner whose weight is not
// trivially zero (an axis with fraction 0 keeps only its lower corner) and whose
// table index is valid.  A skipped corner would add table * 0, which leaves a
// sum of finite values unchanged.
struct LevelCorners {
  float wx0, wx1, wy0, wy1, wz0, wz1;
  uint32_t ix0, ix1, iy0, iy1, iz0, iz1;
  uint32_t mask;
  bool hsh;
};

__device__ __forceinline__ LevelCorners level_corners(float3 nrm, int res, float resf, bool hsh, uint32_t p0,
                                                      uint32_t p1, uint32_t p2, uint32_t T) {
  LevelCorners c;
  int3 b;
  float3 t;
  level_setup_nf(nrm, resf, b, t);
  c.hsh = hsh;
  c.wx0 = 1.0f - t.x; c.wx1 = t.x;
  c.wy0 = 1.0f - t.y; c.wy1 = t.y;
  c.wz0 = 1.0f - t.z; c.wz1 = t.z;
  uint32_t mx = t.x != 0.0f ? 3u : 1u, my = t.y != 0.0f ? 3u : 1u, mz = t.z != 0.0f ? 3u : 1u;
  if (hsh) {
    c.ix0 = (uint32_t)b.x * p0; c.ix1 = c.ix0 + p0;
    c.iy0 = (uint32_t)b.y * p1; c.iy1 = c.iy0 + p1;
    c.iz0 = (uint32_t)b.z * p2; c.iz1 = c.iz0 + p2;
  } else {
    // dense grid: index z*res^2 + y*res + x (uint32, as the reference), in range only
    const uint32_t r = (uint32_t)res;
    c.ix0 = (uint32_t)b.x; c.ix1 = (uint32_t)(b.x + 1);
    c.iy0 = (uint32_t)b.y * r; c.iy1 = (uint32_t)(b.y + 1) * r;
    c.iz0 = (uint32_t)b.z * r * r; c.iz1 = (uint32_t)(b.z + 1) * r * r;
    mx &= (b.x >= 0 && b.x < res ? 1u : 0u) | (b.x + 1 >= 0 && b.x + 1 < res ? 2u : 0u);
    my &= (b.y >= 0 && b.y < res ? 1u : 0u) | (b.y + 1 >= 0 && b.y + 1 < res ? 2u : 0u);
    mz &= (b.z >= 0 && b.z < res ? 1u : 0u) | (b.z + 1 >= 0 && b.z + 1 < res ? 2u : 0u);
  }
  uint32_t m = ((mx & 1u) ? 0x0fu : 0u) | ((mx & 2u) ? 0xf0u : 0u);
  m &= ((my & 1u) ? 0x33u : 0u) | ((my & 2u) ? 0xccu : 0u);
  m &= ((mz & 1u) ? 0x55u : 0u) | ((mz & 2u) ? 0xaau : 0u);
  // Dense index bound: the corner sums grow with each offset, so when the
  // highest corner in the mask is below T (and res^3 cannot wrap) all are.
  const bool small = res < 1625;
  const uint32_t top = ((m & 0xf0u) ? c.ix1 : c.ix0) + ((m & 0xccu) ? c.iy1 : c.iy0) + ((m & 0xaau) ? c.iz1 : c.iz0);
  if (!hsh && !(small && top < T)) {
    uint32_t mm = m;
    while (mm) {
      const int k = __ffs(mm) - 1;
      mm &= mm - 1;
      if (((k & 4) ? c.ix1 : c.ix0) + ((k & 2) ? c.iy1 : c.iy0) + ((k & 1) ? c.iz1 : c.iz0) >= T) m &= ~(1u << k);
    }
  }
  c.mask = m;
  return c;
}

// Trilinear hashgrid features of one (position, level) query (hashgrid.h:244-287),
// accumulated into acc[F].  Each lane may hold a different position and level:
// the eight corners are unrolled, so the corner choice is resolved at compile
// time and only the per-lane mask test remains.  Corners are visited in
// ascending k with weight (wx * wy) * wz, as in the reference.
template <int F, bool POW2>
__device__ __forceinline__ void gather_level(const LevelCorners& c, const float* __restrict__ lvl, uint32_t stride,
                                             uint32_t T, uint32_t Tmask, float* acc) {
  const uint32_t hxy[4] = {c.hsh ? c.ix0 ^ c.iy0 : c.ix0 + c.iy0, c.hsh ? c.ix0 ^ c.iy1 : c.ix0 + c.iy1,
                           c.hsh ? c.ix1 ^ c.iy0 : c.ix1 + c.iy0, c.hsh ? c.ix1 ^ c.iy1 : c.ix1 + c.iy1};
  const float wxy[4] = {c.wx0 * c.wy0, c.wx0 * c.wy1, c.wx1 * c.wy0, c.wx1 * c.wy1};
#pragma unroll
  for (int k = 0; k < 8; k++) {
    if ((c.mask >> k) & 1u) {
      const uint32_t z = (k & 1) ? c.iz1 : c.iz0;
      uint32_t e;
      if (c.hsh) {
        const uint32_t h = hxy[k >> 1] ^ z;
        e = POW2 ? (h & Tmask) : (h % T);
      } else {
        e = hxy[k >> 1] + z;
      }
      const float w = wxy[k >> 1] * ((k & 1) ? c.wz1 : c.wz0);
      const FVec<F> v = load_feat<F>(lvl + (size_t)e * stride);
#pragma unroll
      for (int f = 0; f < F; f++) acc[f] += v.v[f] * w;
    }
  }
}

// The eight corners of the hashgrid box (normalised position in {0, 1}^3;
// corner c has x = c >> 2, y = (c >> 1) & 1, z = c & 1).  A primitive whose grid
// points all clamp to one corner reads fixed table entries with weight 1, so a
// block computes these eight feature vectors once.
__device__ __forceinline__ bool box_corner(float4 n) {
  return (n.x == 0.0f || n.x == 1.0f) && (n.y == 0.0f || n.y == 1.0f) && (n.z == 0.0f || n.z == 1.0f);
}
__device__ __forceinline__ int box_corner_index(float4 n) {
  return (n.x == 1.0f ? 4 : 0) | (n.y == 1.0f ? 2 : 0) | (n.z == 1.0f ? 1 : 0);
}
__device__ __forceinline__ float3 box_corner_pos(int c) {
  return make_float3((float)((c >> 2) & 1), (float)((c >> 1) & 1), (float)(c & 1));
}
// cphi[c * DP + l * F + f] for the 8 corners; the whole block, ends with a barrier.
// STRIDES: address the table through sc.tab_l / sc.tab_e (the feature stage's
// level-major copy); otherwise it is the caller's entry-major table.  POW2: 1 if
// the table size is a power of two (sc.Tmask != 0), 0 if not, -1 to test it here.
template <int F, bool STRIDES = false, int POW2 = -1>
__device__ void box_corner_features(const Scene& sc, const int* res_s, const float* resf_s, const int* hash_s,
                                    uint32_t p0, uint32_t p1, uint32_t p2, int DP, float* cphi) {
  const int L = sc.L;
  for (int t = threadIdx.x; t < 8 * L; t += blockDim.x) {
    const int c = t / L, l = t - (t / L) * L;
    const LevelCorners lc = level_corners(box_corner_pos(c), res_s[l], resf_s[l], hash_s[l] != 0, p0, p1, p2, sc.T);
    float acc[F];
#pragma unroll
    for (int f = 0; f < F; f++) acc[f] = 0.0f;
    const float* lvl = sc.table + (size_t)l * (STRIDES ? sc.tab_l : (size_t)F);
    const uint32_t stride = STRIDES ? sc.tab_e : (uint32_t)(L * F);
    if (POW2 == 1 || (POW2 < 0 && sc.Tmask))
      gather_level<F, true>(lc, lvl, stride, sc.T, sc.Tmask, acc);
    else
      gather_level<F, false>(lc, lvl, stride, sc.T, sc.Tmask, acc);
#pragma unroll
    for (int f = 0; f < F; f++) cphi[c * DP + l * F + f] = acc[f];
  }
  __syncthreads();
}

// Lanes of a warp grouped by bit-identical normalised hashgrid position: every
// member of a class reads the same table entries with the same weights, so the
// class's features are gathered once.  Points clamped to a face of the fixed
// hashgrid box share positions, which is why a primitive often has one or three
// classes rather than one per grid point.  Must be called by the whole warp.
struct PosClasses {
  uint32_t leaders;  // lowest member lane of every class
  uint32_t peers;    // members of this lane's class (member lanes only)
  int U;             // number of classes
  int cls;           // this lane's class index, 0..U-1 (member lanes only)
};
__device__ __forceinline__ PosClasses pos_classes(float3 nrm, bool member) {
  const uint32_t full = 0xffffffffu, lane = threadIdx.x & 31u;
  const uint32_t mm = __ballot_sync(full, member);
  const uint32_t peers = __match_any_sync(full, __float_as_uint(nrm.x)) & __match_any_sync(full, __float_as_uint(nrm.y)) &
                         __match_any_sync(full, __float_as_uint(nrm.z)) & mm;
  PosClasses pc;
  pc.peers = peers;
  pc.leaders = __ballot_sync(full, member && (peers & ((1u << lane) - 1u)) == 0u);
  pc.U = __popc(pc.leaders);
  pc.cls = member ? __popc(pc.leaders & ((1u << (__ffs(peers) - 1)) - 1u)) : 0;
  return pc;
}

// W phi per position class: mlp[u * OMAX + o] = sum_i W[o][i] phi_u[i] for
// u < U, with W rows and phi rows DP floats apart (16-byte aligned, D used).
// When there are few (class, output) items, two or four lanes split one sum
// and combine with shuffles.  Must be called by the whole warp.
template <int OMAX>
__device__ __forceinline__ void class_linear(const float* W_s, const float* phi_s, int DP, int D, int U, float* mlp_s) {
  const int lane = (int)(threadIdx.x & 31u);
  const int items = U * OMAX;
  const int sh = items <= 8 ? 2 : (items <= 16 ? 1 : 0);  // log2 lanes per item
  const int P = 1 << sh, n4 = D >> 2, per = (n4 + P - 1) >> sh;
  for (int base = 0; base < (items << sh); base += 32) {
    const int t = base + lane, item = t >> sh, part = t & (P - 1);
    const int u = item / OMAX, o = item % OMAX;
    float acc = 0.0f;
    if (u < U) {
      const float4* wr = reinterpret_cast<const float4*>(W_s + o * DP);
      const float4* pr = reinterpret_cast<const float4*>(phi_s + u * DP);
      const int i1 = min(n4, (part + 1) * per);
      for (int i4 = part * per; i4 < i1; i4++) {
        const float4 a = wr[i4], b = pr[i4];
        acc = __fmaf_rn(a.x, b.x, acc);
        acc = __fmaf_rn(a.y, b.y, acc);
        acc = __fmaf_rn(a.z, b.z, acc);
        acc = __fmaf_rn(a.w, b.w, acc);
      }
      if (part == P - 1)
        for (int i = D & ~3; i < D; i++) acc = __fmaf_rn(W_s[o * DP + i], phi_s[u * DP + i], acc);
    }
    if (sh >= 1) acc += __shfl_xor_sync(0xffffffffu, acc, 1);
    if (sh >= 2) acc += __shfl_xor_sync(0xffffffffu, acc, 2);
    if (u < U && part == 0) mlp_s[u * OMAX + o] = acc;
  }
}

// Walks the items (class u, level l) of a warp level by level: the lanes form
// segments of U lanes (lane = segment * U + u), segment j holds level l0 + j,
// and one step covers per = 32 / U levels.  Lanes of one segment query the same
// level, so grid points that share table entries share load requests; with
// U > 16 a step is a single level.
struct LevelWalk {
  int per, seg, u, L;
  __device__ __forceinline__ LevelWalk(int U, int levels) : L(levels) {
    const int lane = (int)(threadIdx.x & 31u);
    per = 32 / U;
    seg = lane / U;
    u = lane - seg * U;
  }
  __device__ __forceinline__ int level(int l0) const { return l0 + seg; }
  __device__ __forceinline__ bool valid(int l0) const { return seg < per && l0 + seg < L; }
};

}  // namespace vi

// ---- bulk copies global -> shared completed on an mbarrier (sm_90+ PTX) ----
// Plain cp.async.bulk (no cluster multicast); both addresses 16-byte aligned and
// the size a multiple of 16, which every caller guarantees.
namespace vi {
__device__ __forceinline__ uint32_t smem_addr(const void* p) {
  return (uint32_t)__cvta_generic_to_shared(p);
}
__device__ __forceinline__ void mbar_init(uint64_t* mbar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(mbar)), "r"(count) : "memory");
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* mbar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_addr(mbar)), "r"(bytes)
               : "memory");
}
// Orders this thread's earlier generic-proxy accesses of shared memory before
// later async-proxy (bulk copy) writes to it.
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}
__device__ __forceinline__ void bulk_copy_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* mbar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                   smem_addr(dst)),
               "l"(src), "r"(bytes), "r"(smem_addr(mbar))
               : "memory");
}
// Waits for the phase of the given parity to complete, at most `limit` polls
// (each try_wait suspends for a bounded time).  Returns false on timeout.
__device__ __forceinline__ bool mbar_wait(uint64_t* mbar, uint32_t parity, int limit) {
  for (int i = 0; i < limit; i++) {
    uint32_t ok;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}"
        : "=r"(ok)
        : "r"(smem_addr(mbar)), "r"(parity)
        : "memory");
    if (ok) return true;
  }
  return false;
}
}  // namespace vi
