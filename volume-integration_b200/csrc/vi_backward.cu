// Backward pass (reference cuda_integrator/backward.cu:51-792, hashgrid.h:9-96).
//
// The reference walks every tile entry in reverse, recomputes stage 1 for it and
// lets the pixels that list it as their next contributor accumulate gradients
// with global atomics.  The same quantities are computed here in two kernels:
//
//  1. backward_pixel: one thread per pixel walks its own contributors in
//     reverse (the pixel's state dL/dout and accum_after evolve exactly as in
//     backward.cu:771-778) and writes dL/d(pre-activation) of each contributing
//     (primitive, pixel) record.  Blend and density come from the forward record
//     (identical to the reference's recompute when the forward and backward
//     projections put every grid point in the same pixel; the records of the
//     other primitives are recomputed with the backward projection first, by
//     recompute_records_kernel, from a list the feature stage keeps).
//  2. backward_prim: one warp per primitive, lane = grid point, gathers its
//     contributing records and produces (hashgrid work once per distinct
//     normalised position of the primitive's grid points)
//       dconf[q,g]  = sum_p (dIn_p . phi_g) * g'_{p,g}                (backward.cu:697-710)
//       dtable      += (sum_p dIn_p * g'_{p,g} * conf_g) * corner weight (hashgrid.h:43-95)
//       dW          += dpre_p (x) in_p                                  (backward.cu:621-641)
//     where g' is the stencil magnitude of "neighbour's screen point lies in
//     pixel p" (backward.cu:644-689).  The table scatter is linear in dIn, so
//     each position class scatters once per level and corner instead of once
//     per pixel and grid point; its features come from the feature stage's
//     cache.  dW is reduced per CTA before global atomics; db = sum_p dpre_p is
//     summed by the per-pixel pass, which writes every dpre_p once.
//  3. backward_corner: the primitives whose grid points all clamp to one corner
//     of the reference's fixed hashgrid box, which step 2 then skips: the same
//     quantities with the box corner's features, without position classes.
//
// With the exact-gradient flag steps 1 and 2 compute the derivative of the
// forward instead (backward_pixel_exact_kernel, backward_prim_kernel<.., true,
// ..>), and step 2 takes every primitive.
#include <cuda_runtime.h>

#include <cstdint>

#include "vi_kernels.cuh"

namespace vi {
namespace {

// Generic (runtime F) hashgrid features, used only on the rare recompute path.
__device__ void gather_generic(const Scene& sc, float3 pos, float* phi) {
  const uint32_t p0 = (uint32_t)sc.primes[0], p1 = (uint32_t)sc.primes[1], p2 = (uint32_t)sc.primes[2];
  for (int l = 0; l < sc.L; l++) {
    const int res = sc.res[l];
    const bool hsh = sc.do_hash[l] != 0;
    int3 b;
    float3 t;
    level_setup(pos, sc.hlo, sc.hext, res, b, t);
    for (int f = 0; f < sc.F; f++) phi[l * sc.F + f] = 0.0f;
    for (int dx = 0; dx < 2; dx++) {
      float wx = dx == 0 ? 1.0f - t.x : t.x;
      for (int dy = 0; dy < 2; dy++) {
        float wy = dy == 0 ? 1.0f - t.y : t.y;
        for (int dz = 0; dz < 2; dz++) {
          float wz = dz == 0 ? 1.0f - t.z : t.z;
          float w = wx * wy * wz;
          int e = corner_entry(b.x + dx, b.y + dy, b.z + dz, res, hsh, p0, p1, p2, sc.T, sc.Tmask);
          if (e >= 0) {
            const float* src = sc.table + ((size_t)e * sc.L + l) * sc.F;
            for (int f = 0; f < sc.F; f++) phi[l * sc.F + f] += src[f] * w;
          }
        }
      }
    }
  }
}

// Activated properties of primitive q seen from pixel (px, py) with the backward
// projection 1/w (backward.cu:404-569).
template <int OMAX>
__device__ __noinline__ void recompute_props(const Scene& sc, uint32_t q, int px, int py, float* props) {
  const int V = sc.V, G = sc.G, D = sc.D, O = sc.O;
  const Stencil st = make_stencil(sc.genus);
  const float* conf = sc.conf + (size_t)q * V;
  uint32_t posm[kWideWords] = {0u, 0u, 0u, 0u};
  for (int g = 0; g < V; g++)
    if (conf[g] > 0.0f) posm[g >> 5] |= 1u << (g & 31);
  const float3 c = make_float3(sc.means[3 * q], sc.means[3 * q + 1], sc.means[3 * q + 2]);
  float acc[OMAX];
  for (int o = 0; o < OMAX; o++) acc[o] = 0.0f;
  float phi[64];
  for (int g = 0; g < V; g++) {
    if (!(conf[g] > 0.0f)) continue;
    const float3 pos = grid_pos(c, g, G, sc.step, sc.gof);
    const float2 sb = project(pos, sc.proj, sc.W, sc.H, false);
    if (pix_coord(sb.x) != px || pix_coord(sb.y) != py) continue;
    const float mag = occ_mag_w(posm, grid_point(g, G, 0.0f), G, st);
    if (!(mag > 1e-7f)) continue;
    gather_generic(sc, pos, phi);
    const float wgt = fmul(conf[g], mag);
    for (int o = 0; o < O; o++) {
      float s = 0.0f;
      for (int i = 0; i < D; i++) s += sc.Wl[o * D + i] * phi[i];
      acc[o] = fadd(acc[o], fmul(s, wgt));
    }
  }
  for (int o = 0; o < OMAX; o++) {
    const float pre = fadd(acc[o], sc.bl[o < O ? o : 0]);
    props[o] = o < O - 1 ? sigmoidf_(pre) : (o == O - 1 ? expf(pre) : 0.0f);
  }
}

// dL/db = the sum of dL/dpre over every contributing record (backward.cu:
// 621-641); each record is written by exactly one pixel, so the per-pixel pass
// sums it: per thread, then per warp by shuffles and per block in shared
// memory, then one atomic per output and block.  Called by every thread of a
// 256-thread block.
template <int OMAX>
__device__ __forceinline__ void block_add_db(const float* dbl, int O, float* __restrict__ db) {
  __shared__ float part[8][OMAX];
  const int w = threadIdx.x >> 5, lane = threadIdx.x & 31;
#pragma unroll
  for (int o = 0; o < OMAX; o++) {
    float x = dbl[o];
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) x += __shfl_xor_sync(0xffffffffu, x, off);
    if (lane == 0) part[w][o] = x;
  }
  __syncthreads();
  if ((int)threadIdx.x < O) {
    float x = 0.0f;
#pragma unroll
    for (int ww = 0; ww < 8; ww++) x += part[ww][threadIdx.x];
    if (x != 0.0f) atomicAdd(&db[threadIdx.x], x);
  }
}

template <int OMAX>
__global__ void __launch_bounds__(256) backward_pixel_kernel(Scene sc, GeomState g, ImgState im,
                                                            const float* __restrict__ dL_dcolor,
                                                            const float* __restrict__ dL_dfeat,
                                                            float* __restrict__ db) {
  const size_t N = (size_t)sc.W * sc.H;
  const size_t pix = blockIdx.x * (size_t)blockDim.x + threadIdx.x;
  float dbl[OMAX];
#pragma unroll
  for (int o = 0; o < OMAX; o++) dbl[o] = 0.0f;
  const int K = sc.K;
  const int nc = pix < N ? min(im.n_contrib[pix], K) : 0;
  if (nc > 0) {
  const int O = sc.O, B = O - 1, Fout = sc.Fout;
  float dOut[OMAX - 1], after[OMAX - 1];
#pragma unroll
  for (int d = 0; d < OMAX - 1; d++) {
    dOut[d] = 0.0f;
    after[d] = 0.0f;
  }
  dOut[0] = dL_dcolor[pix];
  dOut[1] = dL_dcolor[N + pix];
  dOut[2] = dL_dcolor[2 * N + pix];
  after[0] = sc.bg[0];
  after[1] = sc.bg[1];
  after[2] = sc.bg[2];
#pragma unroll
  for (int f = 0; f < OMAX - 4; f++)
    if (f < Fout) dOut[3 + f] = dL_dfeat ? dL_dfeat[f * N + pix] : 0.0f;
  // Contributors are visited in reverse; the record slot, delta t and
  // properties of the next one are loaded while the current one is processed.
  const uint32_t* crec = im.contrib_rec + pix * K;
  const float* cdt = im.delta_t + pix * K;
  uint32_t r_next = crec[nc - 1];
  float dt_next = cdt[nc - 1];
  float4 pn[OMAX / 4];
  {
    const float4* src = reinterpret_cast<const float4*>(g.rec_props + (size_t)(r_next & ~kBwdDiffers) * OMAX);
#pragma unroll
    for (int o4 = 0; o4 < OMAX / 4; o4++) pn[o4] = src[o4];
  }
  for (int k = nc - 1; k >= 0; k--) {
    const uint32_t r = r_next, rec = r & ~kBwdDiffers;
    const float dt = dt_next;
    float props[OMAX];
#pragma unroll
    for (int o4 = 0; o4 < OMAX / 4; o4++) {
      props[4 * o4] = pn[o4].x; props[4 * o4 + 1] = pn[o4].y; props[4 * o4 + 2] = pn[o4].z; props[4 * o4 + 3] = pn[o4].w;
    }
    if (k > 0) {
      r_next = crec[k - 1];
      dt_next = cdt[k - 1];
      const float4* src = reinterpret_cast<const float4*>(g.rec_props + (size_t)(r_next & ~kBwdDiffers) * OMAX);
#pragma unroll
      for (int o4 = 0; o4 < OMAX / 4; o4++) pn[o4] = src[o4];
    }
    float dens = 0.0f;
#pragma unroll
    for (int o = 0; o < OMAX; o++)
      if (o == B) dens = props[o];
    float dalpha = 0.0f, dpre[OMAX];
#pragma unroll
    for (int d = 0; d < OMAX - 1; d++) {
      if (d < B) {
        const float y = props[d];
        const float dbl = dOut[d] * y;
        dalpha += dbl * (y - after[d]);
        dpre[d] = dbl * y * (1.0f - y);
      }
    }
#pragma unroll
    for (int o = 0; o < OMAX; o++) {
      if (o == B) dpre[o] = dalpha * dens * dt * dens;
      else if (o > B) dpre[o] = 0.0f;
    }
    float4* dst = reinterpret_cast<float4*>(g.rec_dpre + (size_t)rec * OMAX);
#pragma unroll
    for (int o4 = 0; o4 < OMAX / 4; o4++) dst[o4] = make_float4(dpre[4 * o4], dpre[4 * o4 + 1], dpre[4 * o4 + 2], dpre[4 * o4 + 3]);
    g.rec_pix[rec] = (uint32_t)pix + 1u;
#pragma unroll
    for (int o = 0; o < OMAX; o++) dbl[o] += dpre[o];
#pragma unroll
    for (int d = 0; d < OMAX - 1; d++) {
      if (d < B) {
        const float y = props[d];
        dOut[d] *= y;
        after[d] = y + after[d] * (1.0f - y);
      }
    }
  }
  }
  block_add_db<OMAX>(dbl, sc.O, db);
}

// Exact-gradient mode, per pixel: the derivative of the forward's compositing
// (forward.cu:649-785 as this build computes it) with respect to each
// contribution's activated properties and delta t.  With T_i the
// transmittance before contribution i and a_i its alpha, the colour is
// C = sum_i T_i a_i c_i + T_n bg (clamped to [0, 1]) and
//   dC/dc_i = T_i a_i,   dC/da_i = T_i (c_i - A_i),
// where A_i, the colour behind contribution i, follows A <- a c + (1 - a) A
// from A = bg back to front; features likewise from 0, visibility 1 - T_n with
// dT_n/da_i = -T_i prod_{j>i} (1 - a_j).  A first front-to-back pass recovers
// the unclamped colour for the clamp.  dL/d(delta t) moves the depths of the
// composited primitive and of the one whose arrival composited it; depth is
// the view-space z of the centre, so dL/dmeans3D gains dL/ddepth * (m2, m6, m10).
template <int OMAX>
__global__ void __launch_bounds__(256) backward_pixel_exact_kernel(Scene sc, GeomState g, ImgState im,
                                                                  const uint32_t* __restrict__ point_list,
                                                                  const float* __restrict__ dL_dcolor,
                                                                  const float* __restrict__ dL_dfeat,
                                                                  const float* __restrict__ dL_dvis,
                                                                  float* __restrict__ dmeans,
                                                                  float* __restrict__ db) {
  const size_t N = (size_t)sc.W * sc.H;
  const size_t pix = blockIdx.x * (size_t)blockDim.x + threadIdx.x;
  float dbl[OMAX];
#pragma unroll
  for (int o = 0; o < OMAX; o++) dbl[o] = 0.0f;
  const int K = sc.K;
  const int nc = pix < N ? min(im.n_contrib[pix], K) : 0;
  if (nc > 0) {
  const int O = sc.O, B = O - 1, Fout = sc.Fout, V = sc.V;
  const uint32_t* crec = im.contrib_rec + pix * K;
  const float* cdt = im.delta_t + pix * K;
  const float* ctr = im.trans + pix * K;
  const uint32_t* ctg = im.trig + pix * K;
  auto load_props = [&](uint32_t rec, float* props) {
    const float4* src = reinterpret_cast<const float4*>(g.rec_props + (size_t)rec * OMAX);
#pragma unroll
    for (int o4 = 0; o4 < OMAX / 4; o4++) {
      const float4 v = src[o4];
      props[4 * o4] = v.x; props[4 * o4 + 1] = v.y; props[4 * o4 + 2] = v.z; props[4 * o4 + 3] = v.w;
    }
  };
  auto alpha_of = [&](float sigma, float dt, float& e) {
    e = expf(-sigma * dt);
    return fminf(fmaxf(1.0f - e, 0.0f), 1.0f);
  };
  // Pass 1: the unclamped colour (the final clamp's derivative is 0 outside (0, 1)).
  float C[3] = {0.0f, 0.0f, 0.0f};
  for (int k = 0; k < nc; k++) {
    float props[OMAX], e;
    load_props(crec[k] & ~kBwdDiffers, props);
    float sig = 0.0f;
#pragma unroll
    for (int o = 0; o < OMAX; o++)
      if (o == B) sig = props[o];
    const float a = alpha_of(sig, cdt[k], e), w = ctr[k] * a;
#pragma unroll
    for (int c = 0; c < 3; c++) C[c] += w * props[c];
  }
  const float Tn = im.final_T[pix];
  float gC[3], A[OMAX - 1];
#pragma unroll
  for (int c = 0; c < 3; c++) {
    const float x = C[c] + Tn * sc.bg[c];
    gC[c] = (x > 0.0f && x < 1.0f) ? dL_dcolor[c * N + pix] : 0.0f;
    A[c] = sc.bg[c];
  }
  float gF[OMAX - 4];
#pragma unroll
  for (int f = 0; f < OMAX - 4; f++) {
    gF[f] = (f < Fout && dL_dfeat) ? dL_dfeat[f * N + pix] : 0.0f;
    A[3 + f] = 0.0f;
  }
  const float gV = dL_dvis ? dL_dvis[pix] : 0.0f;
  float Vp = 1.0f;  // prod_{j>i} (1 - a_j)
  const float vz0 = sc.view[2], vz1 = sc.view[6], vz2 = sc.view[10];
  // Pass 2, back to front.
  for (int k = nc - 1; k >= 0; k--) {
    const uint32_t rec = crec[k] & ~kBwdDiffers;
    float props[OMAX], e;
    load_props(rec, props);
    float sig = 0.0f;
#pragma unroll
    for (int o = 0; o < OMAX; o++)
      if (o == B) sig = props[o];
    const float dt = cdt[k], T = ctr[k];
    const float a = alpha_of(sig, dt, e), Ta = T * a;
    float dLda = gV * T * Vp, dpre[OMAX];
#pragma unroll
    for (int d = 0; d < OMAX - 1; d++) {
      if (d < B) {
        const float y = props[d], g = d < 3 ? gC[d] : gF[d - 3];
        dLda += g * T * (y - A[d]);
        dpre[d] = g * Ta * y * (1.0f - y);  // sigmoid
      }
    }
    // a = 1 - exp(-sigma dt): da/dsigma = dt e, da/ddt = sigma e; sigma = exp(pre)
    const bool inside = a > 0.0f && a < 1.0f;
    const float dLds = inside ? dLda * dt * e : 0.0f;
    const float dLddt = inside ? dLda * sig * e : 0.0f;
#pragma unroll
    for (int o = 0; o < OMAX; o++) {
      if (o == B) dpre[o] = dLds * sig;
      else if (o > B) dpre[o] = 0.0f;
    }
    float4* dst = reinterpret_cast<float4*>(g.rec_dpre + (size_t)rec * OMAX);
#pragma unroll
    for (int o4 = 0; o4 < OMAX / 4; o4++) dst[o4] = make_float4(dpre[4 * o4], dpre[4 * o4 + 1], dpre[4 * o4 + 2], dpre[4 * o4 + 3]);
    g.rec_pix[rec] = (uint32_t)pix + 1u;
#pragma unroll
    for (int o = 0; o < OMAX; o++) dbl[o] += dpre[o];
    // delta t = depth(trigger) - depth(this primitive), or max_distance - depth
    if (dLddt != 0.0f) {
      const uint32_t q = rec / V;
      atomicAdd(dmeans + 3 * q, -dLddt * vz0);
      atomicAdd(dmeans + 3 * q + 1, -dLddt * vz1);
      atomicAdd(dmeans + 3 * q + 2, -dLddt * vz2);
      const uint32_t tg = ctg[k];
      if (tg != 0xffffffffu) {
        const uint32_t qt = point_list[tg];
        atomicAdd(dmeans + 3 * qt, dLddt * vz0);
        atomicAdd(dmeans + 3 * qt + 1, dLddt * vz1);
        atomicAdd(dmeans + 3 * qt + 2, dLddt * vz2);
      }
    }
#pragma unroll
    for (int d = 0; d < OMAX - 1; d++)
      if (d < B) A[d] = a * props[d] + (1.0f - a) * A[d];
    Vp *= 1.0f - a;
  }
  }
  block_add_db<OMAX>(dbl, sc.O, db);
}

template <int F>
__device__ __forceinline__ void atomic_vec(float* p, const float* x) {
  if constexpr (F == 2) {
    atomicAdd(reinterpret_cast<float2*>(p), make_float2(x[0], x[1]));
  } else if constexpr (F == 4) {
    atomicAdd(reinterpret_cast<float4*>(p), make_float4(x[0], x[1], x[2], x[3]));
  } else if constexpr (F == 8) {
    atomicAdd(reinterpret_cast<float4*>(p), make_float4(x[0], x[1], x[2], x[3]));
    atomicAdd(reinterpret_cast<float4*>(p) + 1, make_float4(x[4], x[5], x[6], x[7]));
  } else {
#pragma unroll
    for (int f = 0; f < F; f++) atomicAdd(p + f, x[f]);
  }
}

constexpr int kBwdWarps = 4;

__host__ __device__ inline int pad4(int x) { return (x + 3) & ~3; }
__host__ __device__ inline int bwd_dp(int D) { return pad4(D) + 4; }
// Shared memory of backward_prim_kernel.  Head: W [OMAX][DP] (rows of the
// linear layer), level resolution / hash flag [L], box-corner features [8][DP]
// and coefficients [8][OMAX].  Per warp: phi [32][DP] (features of each position class), two lane
// rows [32][OMAX] (conf * vA and E of each grid point; the first later holds W
// phi of each class), two class rows [32][OMAX] (their sums per class; the first
// stages the records' dL/dpre before that), class positions [32] float4, class
// member masks [32] and the warp's dW partial sums [OMAX][D] (lane j owns
// columns j, j + 32).
__host__ __device__ inline int bwd_head_floats(int D, int L, int OMAX) {
  return OMAX * bwd_dp(D) + 3 * pad4(L) + 8 * bwd_dp(D) + 8 * OMAX;
}
__host__ __device__ inline int bwd_warp_floats(int D, int OMAX) {
  return 32 * bwd_dp(D) + 4 * 32 * OMAX + 4 * 32 + 32 + OMAX * D;
}

// Gathers the features of one (position, level) query into acc[F] and, when doA,
// scatters A[f] * (corner weight) into the table gradient at each corner
// (hashgrid.h:43-95): the same corners, weights and order as gather_level.
template <int F, bool POW2>
__device__ __forceinline__ void gather_scatter_level(const LevelCorners& c, const float* __restrict__ lvl,
                                                     float* __restrict__ dst, uint32_t stride, uint32_t T,
                                                     uint32_t Tmask, bool doA, const float* A, float* acc) {
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
      if (doA) {
        float x[F];
#pragma unroll
        for (int f = 0; f < F; f++) x[f] = A[f] * w;
        atomic_vec<F>(dst + (size_t)e * stride, x);
      }
    }
  }
}

// gather_scatter_level plus the derivative of the interpolation with respect to
// the cell fractions: dt3[a] += sum_f A[f] * sum_k table_k,f * dw_k/dt_a, where
// w_k = wx wy wz and each factor is 1 - t or t (exact-gradient mode).
template <int F, bool POW2>
__device__ __forceinline__ void gather_scatter_grad_level(const LevelCorners& c, const float* __restrict__ lvl,
                                                          float* __restrict__ dst, uint32_t stride, uint32_t T,
                                                          uint32_t Tmask, bool doA, const float* A, float* acc,
                                                          float* dt3) {
  const uint32_t hxy[4] = {c.hsh ? c.ix0 ^ c.iy0 : c.ix0 + c.iy0, c.hsh ? c.ix0 ^ c.iy1 : c.ix0 + c.iy1,
                           c.hsh ? c.ix1 ^ c.iy0 : c.ix1 + c.iy0, c.hsh ? c.ix1 ^ c.iy1 : c.ix1 + c.iy1};
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
      const float wx = (k & 4) ? c.wx1 : c.wx0, wy = (k & 2) ? c.wy1 : c.wy0, wz = (k & 1) ? c.wz1 : c.wz0;
      const float w = wx * wy * wz;
      const FVec<F> v = load_feat<F>(lvl + (size_t)e * stride);
      float av = 0.0f;
#pragma unroll
      for (int f = 0; f < F; f++) {
        acc[f] += v.v[f] * w;
        av += A[f] * v.v[f];
      }
      dt3[0] += av * ((k & 4) ? 1.0f : -1.0f) * wy * wz;
      dt3[1] += av * ((k & 2) ? 1.0f : -1.0f) * wx * wz;
      dt3[2] += av * ((k & 1) ? 1.0f : -1.0f) * wx * wy;
      if (doA) {
        float x[F];
#pragma unroll
        for (int f = 0; f < F; f++) x[f] = A[f] * w;
        atomic_vec<F>(dst + (size_t)e * stride, x);
      }
    }
  }
}

// The scatter half of gather_scatter_level: A[f] * (corner weight) into the
// table gradient at each corner of one (position, level) query.
template <int F, bool POW2>
__device__ __forceinline__ void scatter_level(const LevelCorners& c, float* __restrict__ dst, uint32_t stride,
                                              uint32_t T, uint32_t Tmask, const float* A) {
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
      float x[F];
#pragma unroll
      for (int f = 0; f < F; f++) x[f] = A[f] * w;
      atomic_vec<F>(dst + (size_t)e * stride, x);
    }
  }
}

// Sum over the warp of v[idx] for this lane's idx = lane >> (5 - log2 NV):
// recursive halving (each lane keeps half of its values and adds its partner's
// copy of that half), then butterflies over the remaining lane bits.  NV - 1 +
// (5 - log2 NV) shuffles in all; the whole warp calls it.
template <int NV>
__device__ __forceinline__ float warp_reduce_scatter(float* v, uint32_t lane) {
  constexpr int LOG = NV == 8 ? 3 : NV == 16 ? 4 : 5;
  static_assert(NV == 8 || NV == 16 || NV == 32, "8, 16 or 32 values");
#pragma unroll
  for (int s = 0; s < 5; s++) {
    const int b = 16 >> s;
    if (s < LOG) {
      const int h = NV >> (s + 1);
      const bool up = (lane & (uint32_t)b) != 0u;
#pragma unroll
      for (int i = 0; i < h; i++) {
        const float send = up ? v[i] : v[i + h];
        const float keep = up ? v[i + h] : v[i];
        v[i] = keep + __shfl_xor_sync(0xffffffffu, send, b);
      }
    } else {
      v[0] += __shfl_xor_sync(0xffffffffu, v[0], b);
    }
  }
  return v[0];
}

// scatter_level for a warp whose lanes query one level: when every lane that
// scatters (`on`) lies in the same hashgrid cell, the eight corners' terms
// A[f] * (corner weight) are summed over the warp first and each (corner,
// feature) takes one atomic instead of one per lane (a primitive's grid points
// lie in one cell at the coarse levels whenever the box is not much larger than
// the scene).  Otherwise every lane scatters its own corners.  The whole warp
// calls it; the atomics add the same terms, only their grouping differs.
template <int F, bool POW2>
__device__ __forceinline__ void scatter_level_warp(bool on, const LevelCorners& c, float* __restrict__ dst,
                                                   uint32_t stride, uint32_t T, uint32_t Tmask, const float* A,
                                                   uint32_t lane) {
  const uint32_t onm = __ballot_sync(0xffffffffu, on);
  if (onm == 0u) return;
  const int lead = __ffs(onm) - 1;
  const uint32_t x0 = __shfl_sync(0xffffffffu, c.ix0, lead), y0 = __shfl_sync(0xffffffffu, c.iy0, lead),
                 z0 = __shfl_sync(0xffffffffu, c.iz0, lead);
  const bool same = !on || (c.ix0 == x0 && c.iy0 == y0 && c.iz0 == z0);
  if constexpr (F == 1 || F == 2 || F == 4) {
    if (__all_sync(0xffffffffu, same)) {
      constexpr int NV = 8 * F;
      float v[NV];
      const float wxy[4] = {c.wx0 * c.wy0, c.wx0 * c.wy1, c.wx1 * c.wy0, c.wx1 * c.wy1};
#pragma unroll
      for (int k = 0; k < 8; k++) {
        const bool use = on && ((c.mask >> k) & 1u);
        const float w = wxy[k >> 1] * ((k & 1) ? c.wz1 : c.wz0);
#pragma unroll
        for (int f = 0; f < F; f++) v[k * F + f] = use ? A[f] * w : 0.0f;
      }
      const float sum = warp_reduce_scatter<NV>(v, lane);
      const uint32_t um = __reduce_or_sync(0xffffffffu, on ? c.mask : 0u);
      // the shared cell's corner indices (the lead lane's)
      const uint32_t x1 = __shfl_sync(0xffffffffu, c.ix1, lead), y1 = __shfl_sync(0xffffffffu, c.iy1, lead),
                     z1 = __shfl_sync(0xffffffffu, c.iz1, lead);
      const bool hsh = __shfl_sync(0xffffffffu, c.hsh ? 1 : 0, lead) != 0;
      constexpr int SH = NV == 8 ? 2 : NV == 16 ? 1 : 0;  // lanes holding one sum: lane % 2^SH == 0
      if ((lane & ((1u << SH) - 1u)) == 0u) {
        const int idx = (int)(lane >> SH), k = idx / F, f = idx - k * F;
        if ((um >> k) & 1u) {
          const uint32_t x = (k & 4) ? x1 : x0, y = (k & 2) ? y1 : y0, z = (k & 1) ? z1 : z0;
          uint32_t e;
          if (hsh) {
            const uint32_t h = x ^ y ^ z;
            e = POW2 ? (h & Tmask) : (h % T);
          } else {
            e = x + y + z;
          }
          atomicAdd(dst + (size_t)e * stride + f, sum);
        }
      }
      return;
    }
  }
  if (on) scatter_level<F, POW2>(c, dst, stride, T, Tmask, A);
}

// The table-gradient scatter of a primitive with more than 16 position
// classes, all cached: one class per lane, every lane on the same level, so
// each level's scatter is summed over the warp when the classes share a cell
// (scatter_level_warp).
template <int F, int OMAX>
__device__ __forceinline__ void scatter_classes_warp(const float* W_s, const float* S_s, const uint32_t* mem_s,
                                                  const float4* npos_s, const int* res_s, const float* resf_s,
                                                  const int* hash_s, uint32_t p0, uint32_t p1, uint32_t p2,
                                                  uint32_t T, uint32_t Tmask, int L, int DP, int U, uint32_t amask,
                                                  float* __restrict__ dtable, uint32_t stride, uint32_t lane) {
  const bool cl = (int)lane < U;
  const bool on = cl && (mem_s[cl ? lane : 0] & amask) != 0u;
  const float4 n4 = npos_s[cl ? lane : 0];
  const float3 nn = make_float3(n4.x, n4.y, n4.z);
  float S[OMAX];
#pragma unroll
  for (int o = 0; o < OMAX; o++) S[o] = on ? S_s[lane * OMAX + o] : 0.0f;
  for (int l = 0; l < L; l++) {
    const LevelCorners lc = level_corners(nn, res_s[l], resf_s[l], hash_s[l] != 0, p0, p1, p2, T);
    float A[F];
#pragma unroll
    for (int f = 0; f < F; f++) {
      float sum = 0.0f;
#pragma unroll
      for (int o = 0; o < OMAX; o++) sum += W_s[o * DP + l * F + f] * S[o];
      A[f] = sum;
    }
    float* dst = dtable + (size_t)l * F;
    if (Tmask)
      scatter_level_warp<F, true>(on, lc, dst, stride, T, Tmask, A, lane);
    else
      scatter_level_warp<F, false>(on, lc, dst, stride, T, Tmask, A, lane);
  }
}

// One warp per primitive, lane g = grid point g.  With dIn_p = W^T dpre_p
// (backward.cu:608-619), every per-pair sum collapses onto O-wide vectors:
//   v_g  = sum_p g'_{p,g} dpre_p                 -> dconf_g = v_g . (W phi_g)
//   vA_g = sum_p [|g' conf_g| > 1e-9] g' dpre_p  -> table coefficient W^T (conf_g vA_g)
//   E_g  = w_g dpre_{p(g)}                       -> dW += E_g (x) phi_g
// Grid points at the same normalised hashgrid position share phi and table
// corners, so conf*vA and E are summed per position class; the hashgrid gather
// (for phi) and scatter (for the table gradient) then run once per (class,
// level), spread over the warp's lanes.
// SKIPC: primitives whose grid points all clamp to one box corner are left to
// backward_corner_kernel (launched after this one).
// WARP: primitives with more than 16 position classes, all cached, sum each
// level's table-gradient scatter over the warp (scatter_classes_warp).  It is a
// separate instance, taken when the caller sets the hashgrid box: inside the
// scene's own bounds every grid point is a class and the points of one
// primitive share cells at most levels, while with the reference's fixed box
// few primitives have that many classes, and this kernel's loop measured 20%
// slower with the extra path in it (its instruction fetch stalls grew eightfold).
// EXACT: the exact-gradient mode (see backward_pixel_exact_kernel): grid points
// join records by the forward projection, dconf = mag (W phi) . dpre for the
// grid points that form the record, the table coefficient of a class is
// W^T (sum of E), and dL/dmeans3D gains the hashgrid's spatial derivative.
template <int F, int OMAX, bool EXACT, bool WARP, bool SKIPC>
__global__ void __launch_bounds__(kBwdWarps * 32, 5) backward_prim_kernel(Scene sc, GeomState g, float* __restrict__ dmeans,
                                                                      float* __restrict__ dconf,
                                                                      float* __restrict__ dtable, float* __restrict__ dW) {
  extern __shared__ float4 smem4[];
  float* smem = reinterpret_cast<float*>(smem4);
  const int L = sc.L, D = L * F, DP = bwd_dp(D), O = sc.O, V = sc.V, G = sc.G;
  float* W_s = smem;                                      // [OMAX][DP]
  float* resf_s = W_s + OMAX * DP;                        // [L]
  int* res_s = reinterpret_cast<int*>(resf_s + pad4(L));  // [L]
  int* hash_s = res_s + pad4(L);                          // [L]
  float* cphi_s = reinterpret_cast<float*>(hash_s + pad4(L));  // [8][DP] box-corner features
  float* cS_s = cphi_s + 8 * DP;  // [8][OMAX] the block's table-gradient coefficients at the box corners
  const int w = threadIdx.x >> 5;
  const uint32_t lane = threadIdx.x & 31;
  float* phi_s = smem + bwd_head_floats(D, L, OMAX) + w * bwd_warp_floats(D, OMAX);  // [32][DP]
  float* cv_s = phi_s + 32 * DP;      // [32][OMAX] lane conf*vA, then class W phi
  float* el_s = cv_s + 32 * OMAX;     // [32][OMAX] lane E
  float* S_s = el_s + 32 * OMAX;      // [32][OMAX] class sum of conf*vA
  float* Es_s = S_s + 32 * OMAX;      // [32][OMAX] class sum of E
  float4* npos_s = reinterpret_cast<float4*>(Es_s + 32 * OMAX);  // [32]
  uint32_t* mem_s = reinterpret_cast<uint32_t*>(npos_s + 32);     // [32]
  float* dWw = reinterpret_cast<float*>(mem_s + 32);              // [OMAX][D]

  for (int i = threadIdx.x; i < OMAX * DP; i += blockDim.x) {
    const int o = i / DP, d = i % DP;
    W_s[i] = o < O && d < D ? sc.Wl[o * D + d] : 0.0f;
  }
  for (int i = (int)(threadIdx.x & 31); i < OMAX * D; i += 32) dWw[i] = 0.0f;
  for (int i = threadIdx.x; i < L; i += blockDim.x) {
    res_s[i] = sc.res[i];
    resf_s[i] = (float)sc.res[i];
    hash_s[i] = sc.do_hash[i];
  }
  for (int i = threadIdx.x; i < 8 * OMAX; i += blockDim.x) cS_s[i] = 0.0f;
  __syncthreads();

  const Stencil st = make_stencil(sc.genus);
  const GridPt gpt = grid_point((int)lane < V ? (int)lane : 0, G, sc.gof);
  const uint32_t p0 = (uint32_t)__ldg(sc.primes), p1 = (uint32_t)__ldg(sc.primes + 1),
                 p2 = (uint32_t)__ldg(sc.primes + 2);
  if (!EXACT) box_corner_features<F>(sc, res_s, resf_s, hash_s, p0, p1, p2, DP, cphi_s);
  const uint32_t lt_mask = (1u << lane) - 1u;
  const uint32_t stride = (uint32_t)D;
  // dW column `lane` (the first 32 columns) accumulates in registers; columns
  // 32.. (D > 32) in the warp's shared dWw.
  float dwr[OMAX];
#pragma unroll
  for (int o = 0; o < OMAX; o++) dwr[o] = 0.0f;

  // Primitives are handed out in batches of kGrab per warp from a counter
  // (status[5]): warps that draw cheap primitives take more, so no warp idles at
  // the final reduction while the counter sees one atomic per batch.  The
  // batch's record counts (one load) pick the primitives with records, and the
  // inputs of the next one are loaded while the current one is processed.
  constexpr int kGrab = 8;
  const bool act = (int)lane < V;
  uint32_t rp_next = 0u;
  float conf_next = 0.0f;
  float3 c_next = make_float3(0.0f, 0.0f, 0.0f);
  int q_next = -1;
  for (;;) {
    int q0 = 0;
    if (lane == 0) q0 = (int)atomicAdd(g.status + 5, (unsigned)kGrab);
    q0 = __shfl_sync(0xffffffffu, q0, 0);
    if (q0 >= sc.P) break;
    const uint32_t cnt = (int)lane < kGrab && q0 + (int)lane < sc.P ? g.rec_cnt[q0 + lane] : 0u;
    uint32_t batch = __ballot_sync(0xffffffffu, (cnt & ~kBwdDiffers) != 0u);
    if (SKIPC) {  // box-corner primitives are backward_corner_kernel's
      const uint32_t cbx = (int)lane < kGrab && q0 + (int)lane < sc.P ? g.cls_base[q0 + lane] : kNoCache;
      batch &= ~__ballot_sync(0xffffffffu, cbx != kNoCache && (cbx & kCornerCache) != 0u);
    }
    while (batch) {
    const int q = q0 + __ffs(batch) - 1;
    batch &= batch - 1;
    const size_t s0 = (size_t)q * V;
    uint32_t rp;  // pixel + 1 of each grid point's contributing record, else 0
    float conf;
    float3 c;
    if (q_next == q) {
      rp = rp_next;
      conf = conf_next;
      c = c_next;
    } else {
      rp = act ? g.rec_pix[s0 + lane] : 0u;
      conf = act ? sc.conf[s0 + lane] : 0.0f;
      c = make_float3(sc.means[3 * q], sc.means[3 * q + 1], sc.means[3 * q + 2]);
    }
    if (batch) {
      q_next = q0 + __ffs(batch) - 1;
      const size_t s1 = (size_t)q_next * V;
      rp_next = act ? g.rec_pix[s1 + lane] : 0u;
      conf_next = act ? sc.conf[s1 + lane] : 0.0f;
      c_next = make_float3(sc.means[3 * q_next], sc.means[3 * q_next + 1], sc.means[3 * q_next + 2]);
    }
    const uint32_t cm = __ballot_sync(0xffffffffu, rp != 0u);
    if (cm == 0) continue;

    const float3 pos = grid_pos_rel(c, gpt.rel, sc.step);
    // the reference's backward recomputes screen positions with 1/w
    // (backward.cu:325); the exact mode follows the forward's 1/(w + 1e-7)
    const float2 sb = project(pos, sc.proj, sc.W, sc.H, EXACT);
    const int bx = pix_coord(sb.x), by = pix_coord(sb.y);
    const int bpix = (act && bx >= 0 && bx < sc.W && by >= 0 && by < sc.H) ? by * sc.W + bx : -1;
    const uint32_t posm = __ballot_sync(0xffffffffu, act && conf > 0.0f);
    const float mag = act ? occ_mag(posm, gpt, G, st) : 0.0f;
    const float wE = (act && conf > 0.0f && mag > 1e-7f) ? fmul(conf, mag) : 0.0f;

    // dL/dpre of every contributing record, loaded in parallel (lane j: record j)
    // and staged in S_s, which is free until the class sums.
    if ((cm >> lane) & 1u) {
      const float4* src = reinterpret_cast<const float4*>(g.rec_dpre + (s0 + lane) * OMAX);
      float4* dstr = reinterpret_cast<float4*>(S_s + lane * OMAX);
#pragma unroll
      for (int o4 = 0; o4 < OMAX / 4; o4++) dstr[o4] = src[o4];
    }
    __syncwarp();

    float v[OMAX], vA[OMAX];
#pragma unroll
    for (int o = 0; o < OMAX; o++) v[o] = vA[o] = 0.0f;
    bool hasE = false, hasV = false, hasA = false;
    // g'_{p,g} dL/dpre_p summed over the contributing records p.
    auto add_record = [&](int j, float gp) {
      hasV = true;
      const bool doA = fabsf(fmul(gp, conf)) > 1e-9f;
      hasA |= doA;
      const float4* src = reinterpret_cast<const float4*>(S_s + j * OMAX);
#pragma unroll
      for (int o4 = 0; o4 < OMAX / 4; o4++) {
        const float4 d = src[o4];
        const float x0 = gp * d.x, x1 = gp * d.y, x2 = gp * d.z, x3 = gp * d.w;
        v[4 * o4] += x0; v[4 * o4 + 1] += x1; v[4 * o4 + 2] += x2; v[4 * o4 + 3] += x3;
        if (doA) {
          vA[4 * o4] += x0; vA[4 * o4 + 1] += x1; vA[4 * o4 + 2] += x2; vA[4 * o4 + 3] += x3;
        }
      }
    };
    if (EXACT) {
      // Only the grid points that form a record carry gradient (E rows).
      int myrec = -1;
      uint32_t m = cm;
      while (m) {
        const int j = __ffs(m) - 1;
        m &= m - 1;
        const int ppix = (int)__shfl_sync(0xffffffffu, rp, j) - 1;
        if (bpix == ppix) myrec = j;
      }
      if (myrec >= 0 && wE != 0.0f) {
        hasE = true;
#pragma unroll
        for (int o = 0; o < OMAX; o++) el_s[lane * OMAX + o] = fmul(wE, S_s[myrec * OMAX + o]);
      }
    } else if (st.S == 3) {
      // 3-tap stencil: an axis adds 1/2 to record p exactly when one of the two
      // neighbours along it lies in p's pixel (backward.cu:654-689), so a grid
      // point only meets the records of its neighbours' pixels.  myrec = the
      // record of this grid point's own pixel, or -1.
      int myrec = -1;
      uint32_t m = cm;
      while (m) {
        const int j = __ffs(m) - 1;
        m &= m - 1;
        const int ppix = (int)__shfl_sync(0xffffffffu, rp, j) - 1;
        if (bpix == ppix) myrec = j;
      }
      if (myrec >= 0 && wE != 0.0f) {
        hasE = true;
#pragma unroll
        for (int o = 0; o < OMAX; o++) el_s[lane * OMAX + o] = fmul(wE, S_s[myrec * OMAX + o]);
      }
      const int GG = G * G, gi = (int)lane;
      int c[6];
      c[0] = __shfl_sync(0xffffffffu, myrec, (gi + 31) & 31);
      c[1] = __shfl_sync(0xffffffffu, myrec, (gi + 1) & 31);
      c[2] = __shfl_sync(0xffffffffu, myrec, (gi + 32 - G) & 31);
      c[3] = __shfl_sync(0xffffffffu, myrec, (gi + G) & 31);
      c[4] = __shfl_sync(0xffffffffu, myrec, (gi + 32 - GG) & 31);
      c[5] = __shfl_sync(0xffffffffu, myrec, (gi + GG) & 31);
      if (!act || gpt.x == 0) c[0] = -1;
      if (!act || gpt.x + 1 >= G) c[1] = -1;
      if (!act || gpt.y == 0) c[2] = -1;
      if (!act || gpt.y + 1 >= G) c[3] = -1;
      if (!act || gpt.z == 0) c[4] = -1;
      if (!act || gpt.z + 1 >= G) c[5] = -1;
#pragma unroll
      for (int a = 0; a < 3; a++)
        if (c[2 * a] == c[2 * a + 1]) c[2 * a] = c[2 * a + 1] = -1;
#pragma unroll
      for (int i = 0; i < 6; i++) {
        if (c[i] >= 0) {
          int cnt = 1;
#pragma unroll
          for (int k = i + 1; k < 6; k++)
            if (c[k] == c[i]) {
              cnt++;
              c[k] = -1;
            }
          add_record(c[i], 0.5f * (float)cnt);
        }
      }
    } else {
      uint32_t m = cm;
      while (m) {
        const int j = __ffs(m) - 1;
        m &= m - 1;
        const int ppix = (int)__shfl_sync(0xffffffffu, rp, j) - 1;  // pixel of this contribution
        const uint32_t inm = __ballot_sync(0xffffffffu, bpix == ppix);
        if (((inm >> lane) & 1u) && wE != 0.0f) {
          hasE = true;
#pragma unroll
          for (int o = 0; o < OMAX; o++) el_s[lane * OMAX + o] = fmul(wE, S_s[j * OMAX + o]);
        }
        const float gp = act ? occ_mag(inm, gpt, G, st) : 0.0f;
        if (gp > 1e-7f) add_record(j, gp);
      }
    }
    const bool gather = hasE || hasV;
    __syncwarp();  // S_s reads done before the class sums overwrite it
    if (!__any_sync(0xffffffffu, gather)) continue;

    // Lane rows, then position classes of the gathering lanes.
    if (!hasE) {
#pragma unroll
      for (int o = 0; o < OMAX; o++) el_s[lane * OMAX + o] = 0.0f;
    }
#pragma unroll
    for (int o = 0; o < OMAX; o++) cv_s[lane * OMAX + o] = hasA ? conf * vA[o] : 0.0f;
    // With the forward's class features (phi_cache) the classes are those of
    // all grid points, as in the feature stage; otherwise those of the
    // gathering lanes only.
    const uint32_t cb = EXACT ? kNoCache : g.cls_base[q];  // the exact mode gathers (spatial derivative)
    const bool cached = cb != kNoCache;
    const bool member = cached ? act : gather;
    const float3 nrm = hash_norm(pos, sc.hlo, sc.hext);
    const PosClasses pc = pos_classes(nrm, member);
    const uint32_t amask = __ballot_sync(0xffffffffu, hasA);
    const uint32_t emask = __ballot_sync(0xffffffffu, hasE);
    if (member && (pc.peers & lt_mask) == 0u) {
      npos_s[pc.cls] = make_float4(nrm.x, nrm.y, nrm.z, 0.0f);
      mem_s[pc.cls] = pc.peers;
    }
    __syncwarp();
    // Class sums of conf*vA and E.  Rows of lanes outside every class are zero.
    if (pc.U == 1) {
      // One class: lanes cover (vector, output[, half]) and sum rows directly.
      static_assert(OMAX == 8 || OMAX == 16, "OMAX is 8 or 16");
      if constexpr (OMAX == 8) {
        const int half = (int)lane & 1, o = ((int)lane >> 1) & 7, vec = (int)lane >> 4;
        const float* rows = vec ? el_s : cv_s;
        float x = 0.0f;
#pragma unroll
        for (int r = 0; r < 16; r++) x += rows[(2 * r + half) * OMAX + o];
        x += __shfl_xor_sync(0xffffffffu, x, 1);
        if (half == 0) (vec ? Es_s : S_s)[o] = x;
      } else {
        const int o = (int)lane & 15, vec = (int)lane >> 4;
        const float* rows = vec ? el_s : cv_s;
        float x = 0.0f;
#pragma unroll 8
        for (int r = 0; r < 32; r++) x += rows[r * OMAX + o];
        (vec ? Es_s : S_s)[o] = x;
      }
    } else {
      // (class, output) items; members in lane order.
      for (int base = 0; base < pc.U * OMAX; base += 32) {
        const int item = base + (int)lane, u = item / OMAX, o = item % OMAX;
        if (u < pc.U) {
          float sa = 0.0f, se = 0.0f;
          uint32_t mm = mem_s[u];
          while (mm) {
            const int src = __ffs(mm) - 1;
            mm &= mm - 1;
            sa += cv_s[src * OMAX + o];
            se += el_s[src * OMAX + o];
          }
          S_s[u * OMAX + o] = sa;
          Es_s[u * OMAX + o] = se;
        }
      }
    }
    __syncwarp();

    const bool corner = cached && (cb & kCornerCache) != 0u;
    if (corner) {
      // every grid point clamps to box corner cc: features from the block's
      // corner vectors, table coefficient summed per block (one class, S_s[0])
      const int cc = (int)(cb & 7u);
      for (int i = (int)lane; i < D; i += 32) phi_s[i] = cphi_s[cc * DP + i];
      if (amask && (int)lane < OMAX) atomicAdd(&cS_s[cc * OMAX + lane], S_s[lane]);
    } else if (cached) {
      const float* src = g.phi_cache + (size_t)cb * D;
      for (int i = (int)lane; i < pc.U * D; i += 32) phi_s[(i / D) * DP + i % D] = src[i];
    }
    // One pass over (class, level) items, level by level: scatter the table
    // gradient, and gather phi unless the forward cached it.  Lanes of one
    // level that hit the same table entry share one request.
    const LevelWalk it(pc.U, L);
    float dpos[3] = {0.0f, 0.0f, 0.0f};
    const bool warp_scatter = WARP && !EXACT && cached && !corner && pc.U > 16;
    if (warp_scatter)
      scatter_classes_warp<F, OMAX>(W_s, S_s, mem_s, npos_s, res_s, resf_s, hash_s, p0, p1, p2, sc.T, sc.Tmask, L,
                                    DP, pc.U, amask, dtable, stride, lane);
    for (int l0 = (corner || warp_scatter) ? L : 0; l0 < L; l0 += it.per) {
      if (!it.valid(l0)) continue;
      const int l = it.level(l0), u = it.u;
      const bool doA = (mem_s[u] & (EXACT ? emask : amask)) != 0u;
      if (cached && !doA) continue;
      const float4 n4 = npos_s[u];
      const LevelCorners lc = level_corners(make_float3(n4.x, n4.y, n4.z), res_s[l], resf_s[l], hash_s[l] != 0,
                                            p0, p1, p2, sc.T);
      float A[F], acc[F];
#pragma unroll
      for (int f = 0; f < F; f++) {
        acc[f] = 0.0f;
        // table coefficient of this level: sum_o W[o][l*F+f] S_u[o]
        float sum = 0.0f;
        if (doA) {
#pragma unroll
          for (int o = 0; o < OMAX; o++) sum += W_s[o * DP + l * F + f] * (EXACT ? Es_s : S_s)[u * OMAX + o];
        }
        A[f] = sum;
      }
      const float* lvl = sc.table + (size_t)l * F;
      float* dst = dtable + (size_t)l * F;
      if (cached) {
        if (sc.Tmask)
          scatter_level<F, true>(lc, dst, stride, sc.T, sc.Tmask, A);
        else
          scatter_level<F, false>(lc, dst, stride, sc.T, sc.Tmask, A);
        continue;
      }
      if (EXACT) {
        float dt3[3] = {0.0f, 0.0f, 0.0f};  // sum_f A_f dphi_f / dt per axis
        if (sc.Tmask)
          gather_scatter_grad_level<F, true>(lc, lvl, dst, stride, sc.T, sc.Tmask, doA, A, acc, dt3);
        else
          gather_scatter_grad_level<F, false>(lc, lvl, dst, stride, sc.T, sc.Tmask, doA, A, acc, dt3);
        // t = frac(n * res), n = clamp((p - lo) / ext): dt/dp = res / ext where not clamped
        const float r = resf_s[l];
        if (n4.x > 0.0f && n4.x < 1.0f) dpos[0] += dt3[0] * __fdiv_rn(r, sc.hext[0]);
        if (n4.y > 0.0f && n4.y < 1.0f) dpos[1] += dt3[1] * __fdiv_rn(r, sc.hext[1]);
        if (n4.z > 0.0f && n4.z < 1.0f) dpos[2] += dt3[2] * __fdiv_rn(r, sc.hext[2]);
      } else if (sc.Tmask) {
        gather_scatter_level<F, true>(lc, lvl, dst, stride, sc.T, sc.Tmask, doA, A, acc);
      } else {
        gather_scatter_level<F, false>(lc, lvl, dst, stride, sc.T, sc.Tmask, doA, A, acc);
      }
#pragma unroll
      for (int f = 0; f < F; f++) phi_s[u * DP + l * F + f] = acc[f];
    }
    if (EXACT) {
      // grid point positions are the centre plus fixed offsets: dL/dmeans3D += sum
#pragma unroll
      for (int a = 0; a < 3; a++)
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) dpos[a] += __shfl_xor_sync(0xffffffffu, dpos[a], off);
      if (lane == 0 && (dpos[0] != 0.0f || dpos[1] != 0.0f || dpos[2] != 0.0f)) {
        dmeans[3 * q] += dpos[0];  // one warp per primitive; the per-pixel kernel's atomics finished
        dmeans[3 * q + 1] += dpos[1];
        dmeans[3 * q + 2] += dpos[2];
      }
    }
    __syncwarp();
    // W phi per class (into cv_s, free now).
    float* mlp_s = cv_s;
    class_linear<OMAX>(W_s, phi_s, DP, D, pc.U, mlp_s);
    __syncwarp();
    if (act) {
      float dX = 0.0f;
      if (EXACT) {
        // d pre / d conf_g = mag_g (W phi_g) on the record of g's pixel; E_g = conf_g mag_g dpre
        if (hasE) {
          const float* mr = mlp_s + pc.cls * OMAX;
          const float* er = el_s + lane * OMAX;
          float s = 0.0f;
#pragma unroll
          for (int o = 0; o < OMAX; o++) s += mr[o] * er[o];
          dX = __fdiv_rn(s, conf);
        }
      } else if (gather) {
        const float* mr = mlp_s + pc.cls * OMAX;
#pragma unroll
        for (int o = 0; o < OMAX / 2; o++) dX += v[2 * o] * mr[2 * o] + v[2 * o + 1] * mr[2 * o + 1];
      }
      dconf[s0 + lane] = dX;
    }
    // dW += (class sum of E) (x) phi_class; lane jj owns columns jj, jj + 32.
    if (emask) {
      for (int u = 0; u < pc.U; u++) {
        if ((mem_s[u] & emask) == 0u) continue;
        const float4* er = reinterpret_cast<const float4*>(Es_s + u * OMAX);
        if ((int)lane < D) {
          const float x = phi_s[u * DP + lane];
#pragma unroll
          for (int o4 = 0; o4 < OMAX / 4; o4++) {
            const float4 e4 = er[o4];
            dwr[4 * o4] += e4.x * x;
            dwr[4 * o4 + 1] += e4.y * x;
            dwr[4 * o4 + 2] += e4.z * x;
            dwr[4 * o4 + 3] += e4.w * x;
          }
        }
        for (int jj = (int)lane + 32; jj < D; jj += 32) {
          const float x = phi_s[u * DP + jj];
#pragma unroll
          for (int o = 0; o < OMAX; o++) dWw[o * D + jj] += Es_s[u * OMAX + o] * x;
        }
      }
    }
    __syncwarp();
    }
  }

  // CTA reduction of dW and db, then one global atomic per element.
  if ((int)lane < D) {
#pragma unroll
    for (int o = 0; o < OMAX; o++) dWw[o * D + lane] = dwr[o];
  }
  __syncwarp();
  __syncthreads();
  // Table gradient of the box-corner primitives: one scatter per (corner, level).
  for (int t = threadIdx.x; t < 8 * L; t += blockDim.x) {
    const int c = t / L, l = t - (t / L) * L;
    bool any = false;
    for (int o = 0; o < OMAX; o++) any |= cS_s[c * OMAX + o] != 0.0f;
    if (!any) continue;
    float A[F];
#pragma unroll
    for (int f = 0; f < F; f++) {
      float sum = 0.0f;
#pragma unroll
      for (int o = 0; o < OMAX; o++) sum += W_s[o * DP + l * F + f] * cS_s[c * OMAX + o];
      A[f] = sum;
    }
    const LevelCorners lc = level_corners(box_corner_pos(c), res_s[l], resf_s[l], hash_s[l] != 0, p0, p1, p2, sc.T);
    if (sc.Tmask)
      scatter_level<F, true>(lc, dtable + (size_t)l * F, stride, sc.T, sc.Tmask, A);
    else
      scatter_level<F, false>(lc, dtable + (size_t)l * F, stride, sc.T, sc.Tmask, A);
  }
  const float* warp0 = smem + bwd_head_floats(D, L, OMAX) + (bwd_warp_floats(D, OMAX) - OMAX * D);
  for (int i = threadIdx.x; i < O * D; i += blockDim.x) {
    float x = 0.0f;
    for (int ww = 0; ww < kBwdWarps; ww++) x += warp0[(size_t)ww * bwd_warp_floats(D, OMAX) + i];
    if (x != 0.0f) atomicAdd(&dW[i], x);
  }
}

// Per-primitive backward of the box-corner primitives (every grid point clamps
// to one corner cc of the hashgrid box, so every grid point has the features
// phi_cc of that corner): the reference's formula with the 3-tap stencil, as
// backward_prim_kernel computes it for such a primitive, without position
// classes, gathers or a per-primitive linear layer.  One warp per primitive,
// lane g = grid point g.  Per primitive: v_g, vA_g and E_g over the records
// (the 3-tap search of backward_prim_kernel), dconf_g = v_g . (W phi_cc) from
// the block's eight corner vectors W phi_c, and the warp's sums of conf_g vA_g
// and E_g, added per corner into the block's shared rows with one
// reduce-scatter.  At the end of the block: the table gradient at each corner's
// entries (W^T of the summed conf vA, one scatter per corner and level) and
// dW += sum over corners of (summed E) (x) phi_c.
constexpr int kCornerWarps = 8;
__host__ __device__ inline int corner_head_floats(int D, int L, int OMAX) {
  return OMAX * bwd_dp(D) + 3 * pad4(L) + 8 * bwd_dp(D) + 3 * 8 * OMAX;
}
template <int F, int OMAX>
__global__ void __launch_bounds__(kCornerWarps * 32, OMAX == 8 ? 4 : 2) backward_corner_kernel(Scene sc, GeomState g,
                                                                             float* __restrict__ dconf,
                                                                             float* __restrict__ dtable,
                                                                             float* __restrict__ dW) {
  extern __shared__ float4 smem4[];
  float* smem = reinterpret_cast<float*>(smem4);
  const int L = sc.L, D = L * F, DP = bwd_dp(D), O = sc.O, V = sc.V, G = sc.G;
  float* W_s = smem;                                      // [OMAX][DP]
  float* resf_s = W_s + OMAX * DP;                        // [L]
  int* res_s = reinterpret_cast<int*>(resf_s + pad4(L));  // [L]
  int* hash_s = res_s + pad4(L);                          // [L]
  float* cphi_s = reinterpret_cast<float*>(hash_s + pad4(L));  // [8][DP] box-corner features
  float* cmlp_s = cphi_s + 8 * DP;  // [8][OMAX] W phi_c
  float* cS_s = cmlp_s + 8 * OMAX;  // [8][OMAX] sums of conf * vA per corner
  float* cE_s = cS_s + 8 * OMAX;    // [8][OMAX] sums of E per corner
  const int w = threadIdx.x >> 5;
  const uint32_t lane = threadIdx.x & 31;
  float* S_s = smem + corner_head_floats(D, L, OMAX) + w * 32 * OMAX;  // [32][OMAX] the records' dL/dpre

  for (int i = threadIdx.x; i < OMAX * DP; i += blockDim.x) {
    const int o = i / DP, d = i % DP;
    W_s[i] = o < O && d < D ? sc.Wl[o * D + d] : 0.0f;
  }
  for (int i = threadIdx.x; i < L; i += blockDim.x) {
    res_s[i] = sc.res[i];
    resf_s[i] = (float)sc.res[i];
    hash_s[i] = sc.do_hash[i];
  }
  for (int i = threadIdx.x; i < 16 * OMAX; i += blockDim.x) cS_s[i] = 0.0f;  // cS_s and cE_s
  __syncthreads();
  const uint32_t p0 = (uint32_t)__ldg(sc.primes), p1 = (uint32_t)__ldg(sc.primes + 1),
                 p2 = (uint32_t)__ldg(sc.primes + 2);
  box_corner_features<F>(sc, res_s, resf_s, hash_s, p0, p1, p2, DP, cphi_s);
  for (int t = threadIdx.x; t < 8 * OMAX; t += blockDim.x) {
    const int c = t / OMAX, o = t % OMAX;
    float acc = 0.0f;
    for (int i = 0; i < D; i++) acc = __fmaf_rn(W_s[o * DP + i], cphi_s[c * DP + i], acc);
    cmlp_s[t] = acc;
  }
  __syncthreads();

  const Stencil st = make_stencil(sc.genus);
  const GridPt gpt = grid_point((int)lane < V ? (int)lane : 0, G, sc.gof);
  const bool act = (int)lane < V;
  constexpr int kGrab = 8;
  // the next primitive's record pixels, confidences and centre are loaded while
  // the current one is processed
  int q_next = -1;
  uint32_t rp_next = 0u;
  float conf_next = 0.0f;
  float3 c_next = make_float3(0.0f, 0.0f, 0.0f);
  for (;;) {
    int q0 = 0;
    if (lane == 0) q0 = (int)atomicAdd(g.status + 8, (unsigned)kGrab);
    q0 = __shfl_sync(0xffffffffu, q0, 0);
    if (q0 >= sc.P) break;
    const bool in = (int)lane < kGrab && q0 + (int)lane < sc.P;
    const uint32_t cnt = in ? g.rec_cnt[q0 + lane] : 0u;
    const uint32_t cbx = in ? g.cls_base[q0 + lane] : kNoCache;
    uint32_t batch = __ballot_sync(0xffffffffu, (cnt & ~kBwdDiffers) != 0u && cbx != kNoCache &&
                                                    (cbx & kCornerCache) != 0u);
    while (batch) {
      const int qi = __ffs(batch) - 1;
      batch &= batch - 1;
      const int q = q0 + qi;
      const int cc = (int)(__shfl_sync(0xffffffffu, cbx, qi) & 7u);
      const size_t s0 = (size_t)q * V;
      uint32_t rp;  // pixel + 1 of each grid point's record, else 0
      float conf;
      float3 c;
      if (q_next == q) {
        rp = rp_next;
        conf = conf_next;
        c = c_next;
      } else {
        rp = act ? g.rec_pix[s0 + lane] : 0u;
        conf = act ? sc.conf[s0 + lane] : 0.0f;
        c = make_float3(sc.means[3 * q], sc.means[3 * q + 1], sc.means[3 * q + 2]);
      }
      if (batch) {
        q_next = q0 + __ffs(batch) - 1;
        const size_t s1 = (size_t)q_next * V;
        rp_next = act ? g.rec_pix[s1 + lane] : 0u;
        conf_next = act ? sc.conf[s1 + lane] : 0.0f;
        c_next = make_float3(sc.means[3 * q_next], sc.means[3 * q_next + 1], sc.means[3 * q_next + 2]);
      }
      const uint32_t cm = __ballot_sync(0xffffffffu, rp != 0u);
      if (cm == 0) continue;
      const float3 pos = grid_pos_rel(c, gpt.rel, sc.step);
      const float2 sb = project(pos, sc.proj, sc.W, sc.H, false);  // backward.cu:325
      const int bx = pix_coord(sb.x), by = pix_coord(sb.y);
      const int bpix = (act && bx >= 0 && bx < sc.W && by >= 0 && by < sc.H) ? by * sc.W + bx : -1;
      const uint32_t posm = __ballot_sync(0xffffffffu, act && conf > 0.0f);
      const float mag = act ? occ_mag(posm, gpt, G, st) : 0.0f;
      const float wE = (act && conf > 0.0f && mag > 1e-7f) ? fmul(conf, mag) : 0.0f;
      if ((cm >> lane) & 1u) {
        const float4* src = reinterpret_cast<const float4*>(g.rec_dpre + (s0 + lane) * OMAX);
        float4* dstr = reinterpret_cast<float4*>(S_s + lane * OMAX);
#pragma unroll
        for (int o4 = 0; o4 < OMAX / 4; o4++) dstr[o4] = src[o4];
      }
      __syncwarp();
      float v[OMAX], vA[OMAX], el[OMAX];
#pragma unroll
      for (int o = 0; o < OMAX; o++) v[o] = vA[o] = el[o] = 0.0f;
      bool hasV = false, hasA = false;
      // the record of this grid point's own pixel, and E from it
      int myrec = -1;
      uint32_t m = cm;
      while (m) {
        const int j = __ffs(m) - 1;
        m &= m - 1;
        if (bpix == (int)__shfl_sync(0xffffffffu, rp, j) - 1) myrec = j;
      }
      const bool hasE = myrec >= 0 && wE != 0.0f;
      if (hasE) {
#pragma unroll
        for (int o = 0; o < OMAX; o++) el[o] = fmul(wE, S_s[myrec * OMAX + o]);
      }
      // 3-tap stencil: an axis adds 1/2 to record p exactly when one of the two
      // neighbours along it lies in p's pixel (backward.cu:654-689)
      const int GG = G * G, gi = (int)lane;
      int nb[6];
      nb[0] = __shfl_sync(0xffffffffu, myrec, (gi + 31) & 31);
      nb[1] = __shfl_sync(0xffffffffu, myrec, (gi + 1) & 31);
      nb[2] = __shfl_sync(0xffffffffu, myrec, (gi + 32 - G) & 31);
      nb[3] = __shfl_sync(0xffffffffu, myrec, (gi + G) & 31);
      nb[4] = __shfl_sync(0xffffffffu, myrec, (gi + 32 - GG) & 31);
      nb[5] = __shfl_sync(0xffffffffu, myrec, (gi + GG) & 31);
      if (!act || gpt.x == 0) nb[0] = -1;
      if (!act || gpt.x + 1 >= G) nb[1] = -1;
      if (!act || gpt.y == 0) nb[2] = -1;
      if (!act || gpt.y + 1 >= G) nb[3] = -1;
      if (!act || gpt.z == 0) nb[4] = -1;
      if (!act || gpt.z + 1 >= G) nb[5] = -1;
#pragma unroll
      for (int a = 0; a < 3; a++)
        if (nb[2 * a] == nb[2 * a + 1]) nb[2 * a] = nb[2 * a + 1] = -1;
#pragma unroll
      for (int i = 0; i < 6; i++) {
        if (nb[i] >= 0) {
          int k = 1;
#pragma unroll
          for (int kk = i + 1; kk < 6; kk++)
            if (nb[kk] == nb[i]) {
              k++;
              nb[kk] = -1;
            }
          const float gp = 0.5f * (float)k;
          hasV = true;
          const bool doA = fabsf(fmul(gp, conf)) > 1e-9f;
          hasA |= doA;
          const float4* src = reinterpret_cast<const float4*>(S_s + nb[i] * OMAX);
#pragma unroll
          for (int o4 = 0; o4 < OMAX / 4; o4++) {
            const float4 d = src[o4];
            const float x0 = gp * d.x, x1 = gp * d.y, x2 = gp * d.z, x3 = gp * d.w;
            v[4 * o4] += x0; v[4 * o4 + 1] += x1; v[4 * o4 + 2] += x2; v[4 * o4 + 3] += x3;
            if (doA) {
              vA[4 * o4] += x0; vA[4 * o4 + 1] += x1; vA[4 * o4 + 2] += x2; vA[4 * o4 + 3] += x3;
            }
          }
        }
      }
      __syncwarp();  // S_s reads done before the next primitive stages its records
      const bool gather = hasE || hasV;
      if (!__any_sync(0xffffffffu, gather)) continue;
      if (act) {
        float dX = 0.0f;
        if (gather) {
          const float* mr = cmlp_s + cc * OMAX;
#pragma unroll
          for (int o = 0; o < OMAX / 2; o++) dX += v[2 * o] * mr[2 * o] + v[2 * o + 1] * mr[2 * o + 1];
        }
        dconf[s0 + lane] = dX;
      }
      // sums over the warp of conf * vA and of E, added to corner cc's rows
      constexpr int NV = 2 * OMAX;
      float sv[NV];
#pragma unroll
      for (int o = 0; o < OMAX; o++) {
        sv[o] = hasA ? conf * vA[o] : 0.0f;
        sv[OMAX + o] = el[o];
      }
      const float tot = warp_reduce_scatter<NV>(sv, lane);
      constexpr int SH = NV == 16 ? 1 : 0;  // lanes holding one sum: lane % 2^SH == 0
      if ((lane & ((1u << SH) - 1u)) == 0u && tot != 0.0f) {
        const int idx = (int)(lane >> SH);
        atomicAdd(idx < OMAX ? &cS_s[cc * OMAX + idx] : &cE_s[cc * OMAX + idx - OMAX], tot);
      }
    }
  }
  __syncthreads();
  // Table gradient at the box corners: one scatter per (corner, level).
  const uint32_t stride = (uint32_t)D;
  for (int t = threadIdx.x; t < 8 * L; t += blockDim.x) {
    const int c = t / L, l = t - (t / L) * L;
    bool any = false;
    for (int o = 0; o < OMAX; o++) any |= cS_s[c * OMAX + o] != 0.0f;
    if (!any) continue;
    float A[F];
#pragma unroll
    for (int f = 0; f < F; f++) {
      float sum = 0.0f;
#pragma unroll
      for (int o = 0; o < OMAX; o++) sum += W_s[o * DP + l * F + f] * cS_s[c * OMAX + o];
      A[f] = sum;
    }
    const LevelCorners lc = level_corners(box_corner_pos(c), res_s[l], resf_s[l], hash_s[l] != 0, p0, p1, p2, sc.T);
    if (sc.Tmask)
      scatter_level<F, true>(lc, dtable + (size_t)l * F, stride, sc.T, sc.Tmask, A);
    else
      scatter_level<F, false>(lc, dtable + (size_t)l * F, stride, sc.T, sc.Tmask, A);
  }
  // dW += sum_c (E sum of corner c) (x) phi_c
  for (int i = threadIdx.x; i < O * D; i += blockDim.x) {
    const int o = i / D, d = i - (i / D) * D;
    float x = 0.0f;
#pragma unroll
    for (int c = 0; c < 8; c++) x += cE_s[c * OMAX + o] * cphi_s[c * DP + d];
    if (x != 0.0f) atomicAdd(&dW[i], x);
  }
}

// Per-primitive backward for grids of more than 32 points (G = 4, 5; the
// reference allows up to 5, backward.cu:26-33): one block of kWideThreads per
// primitive, thread g = grid point g, following the reference's formula
// (backward.cu:404-765) record by record.  For every contributing record p, the
// grid points whose backward screen position lies in p's pixel are the
// occupancy of g'_{p,.}; each grid point accumulates
//   v_g = sum_p g'_{p,g} dpre_p, vA_g (the terms with |g' conf_g| > 1e-9) and
//   E_g = w_g dpre_{p(g)} for the record of its own pixel,
// then gathers its features phi_g, scatters W^T (conf_g vA_g) into the table
// gradient at its corners, writes dconf_g = v_g . (W phi_g), and the block sums
// dW += E_g (x) phi_g (one global atomic per element at the end).
template <int F, int OMAX, bool POW2>
__global__ void __launch_bounds__(kWideThreads) backward_prim_wide_kernel(Scene sc, GeomState g,
                                                                         float* __restrict__ dconf,
                                                                         float* __restrict__ dtable,
                                                                         float* __restrict__ dW) {
  extern __shared__ float4 smem4[];
  float* smem = reinterpret_cast<float*>(smem4);
  const int L = sc.L, D = L * F, DP = bwd_dp(D), O = sc.O, V = sc.V, G = sc.G;
  float* W_s = smem;                                           // [OMAX][DP]
  float* resf_s = W_s + OMAX * DP;                             // [L]
  int* res_s = reinterpret_cast<int*>(resf_s + pad4(L));       // [L]
  int* hash_s = res_s + pad4(L);                               // [L]
  float* dpre_s = reinterpret_cast<float*>(hash_s + pad4(L));  // [kWideThreads][OMAX] dL/dpre of record j
  float* el_s = dpre_s + kWideThreads * OMAX;                  // [kWideThreads][OMAX] E of grid point g
  float* phi_s = el_s + kWideThreads * OMAX;                   // [kWideThreads][DP] phi of grid point g
  float* dw_s = phi_s + kWideThreads * DP;                     // [OMAX][D] the block's dW
  uint32_t* rp_s = reinterpret_cast<uint32_t*>(dw_s + OMAX * D);  // [kWideThreads] pixel + 1 of record j
  uint32_t* ef_s = rp_s + kWideThreads;                        // [kWideThreads] grid point g has E
  uint32_t* occ_s = ef_s + kWideThreads;                       // [kWideWords] conf > 0
  uint32_t* inm_s = occ_s + kWideWords;                        // [kWideWords] in the pixel of one record
  int* misc_s = reinterpret_cast<int*>(inm_s + kWideWords);    // [4] claimed primitive
  const int t = threadIdx.x, lane = t & 31, w = t >> 5;
  for (int i = t; i < OMAX * DP; i += blockDim.x) {
    const int o = i / DP, d = i % DP;
    W_s[i] = o < O && d < D ? sc.Wl[o * D + d] : 0.0f;
  }
  for (int i = t; i < L; i += blockDim.x) {
    res_s[i] = sc.res[i];
    resf_s[i] = (float)sc.res[i];
    hash_s[i] = sc.do_hash[i];
  }
  for (int i = t; i < OMAX * D; i += blockDim.x) dw_s[i] = 0.0f;
  const Stencil st = make_stencil(sc.genus);
  const bool act = t < V;
  const GridPt gp = grid_point(act ? t : 0, G, sc.gof);
  const uint32_t p0 = (uint32_t)__ldg(sc.primes), p1 = (uint32_t)__ldg(sc.primes + 1),
                 p2 = (uint32_t)__ldg(sc.primes + 2);
  for (;;) {
    __syncthreads();  // the previous primitive's shared reads are done
    if (t == 0) misc_s[0] = (int)atomicAdd(g.status + 5, 1u);
    __syncthreads();
    const int q = misc_s[0];
    if (q >= sc.P) break;
    if ((g.rec_cnt[q] & ~kBwdDiffers) == 0u) continue;
    const size_t s0 = (size_t)q * V;
    const uint32_t rp = act ? g.rec_pix[s0 + t] : 0u;  // record slot t
    rp_s[t] = rp;
    if (rp) {
      const float4* src = reinterpret_cast<const float4*>(g.rec_dpre + (s0 + t) * OMAX);
      float4* dst = reinterpret_cast<float4*>(dpre_s + t * OMAX);
#pragma unroll
      for (int o4 = 0; o4 < OMAX / 4; o4++) dst[o4] = src[o4];
    }
    const float conf = act ? sc.conf[s0 + t] : 0.0f;
    const float3 c = make_float3(sc.means[3 * q], sc.means[3 * q + 1], sc.means[3 * q + 2]);
    const float3 pos = grid_pos_rel(c, gp.rel, sc.step);
    const float2 sb = project(pos, sc.proj, sc.W, sc.H, false);  // backward.cu:325
    const int bx = pix_coord(sb.x), by = pix_coord(sb.y);
    const int bpix = (act && bx >= 0 && bx < sc.W && by >= 0 && by < sc.H) ? by * sc.W + bx : -1;
    const uint32_t occw = __ballot_sync(0xffffffffu, act && conf > 0.0f);
    if (lane == 0) occ_s[w] = occw;
    if (!__syncthreads_or(rp != 0u)) continue;  // also publishes rp_s, dpre_s, occ_s
    const float mag = act ? occ_mag_w(occ_s, gp, G, st) : 0.0f;
    const float wE = (act && conf > 0.0f && mag > 1e-7f) ? fmul(conf, mag) : 0.0f;
    float v[OMAX], vA[OMAX], e[OMAX];
#pragma unroll
    for (int o = 0; o < OMAX; o++) v[o] = vA[o] = e[o] = 0.0f;
    bool hasE = false, hasV = false, hasA = false;
    for (int j = 0; j < V; j++) {
      const uint32_t rj = rp_s[j];
      if (rj == 0u) continue;  // block-uniform
      const int ppix = (int)rj - 1;
      const uint32_t inw = __ballot_sync(0xffffffffu, bpix == ppix);
      __syncthreads();  // the previous record's inm_s reads are done
      if (lane == 0) inm_s[w] = inw;
      __syncthreads();
      if (bpix == ppix && wE != 0.0f) {
        hasE = true;
#pragma unroll
        for (int o = 0; o < OMAX; o++) e[o] = fmul(wE, dpre_s[j * OMAX + o]);
      }
      const float gpv = act ? occ_mag_w(inm_s, gp, G, st) : 0.0f;
      if (gpv > 1e-7f) {
        hasV = true;
        const bool doA = fabsf(fmul(gpv, conf)) > 1e-9f;
        hasA |= doA;
#pragma unroll
        for (int o = 0; o < OMAX; o++) {
          const float x = gpv * dpre_s[j * OMAX + o];
          v[o] += x;
          if (doA) vA[o] += x;
        }
      }
    }
    if (hasE || hasV) {
      // features of this grid point and the table-gradient scatter, level by level
      const float3 n = hash_norm(pos, sc.hlo, sc.hext);
      float cv[OMAX];
#pragma unroll
      for (int o = 0; o < OMAX; o++) cv[o] = hasA ? conf * vA[o] : 0.0f;
#pragma unroll 1
      for (int l = 0; l < L; l++) {
        const LevelCorners lc = level_corners(n, res_s[l], resf_s[l], hash_s[l] != 0, p0, p1, p2, sc.T);
        float A[F], acc[F];
#pragma unroll
        for (int f = 0; f < F; f++) {
          acc[f] = 0.0f;
          float sum = 0.0f;
          if (hasA) {
#pragma unroll
            for (int o = 0; o < OMAX; o++) sum += W_s[o * DP + l * F + f] * cv[o];
          }
          A[f] = sum;
        }
        gather_scatter_level<F, POW2>(lc, sc.table + (size_t)l * F, dtable + (size_t)l * F, (uint32_t)D, sc.T,
                                      sc.Tmask, hasA, A, acc);
#pragma unroll
        for (int f = 0; f < F; f++) phi_s[t * DP + l * F + f] = acc[f];
      }
      float dX = 0.0f;
#pragma unroll
      for (int o = 0; o < OMAX; o++) {
        float m = 0.0f;
        for (int i = 0; i < D; i++) m = __fmaf_rn(W_s[o * DP + i], phi_s[t * DP + i], m);
        dX += v[o] * m;
      }
      dconf[s0 + t] = dX;
    }
    ef_s[t] = hasE ? 1u : 0u;
#pragma unroll
    for (int o = 0; o < OMAX; o++) el_s[t * OMAX + o] = e[o];
    __syncthreads();
    // dW += sum_g E_g (x) phi_g: each (output, input) element is owned by one thread
    for (int it = t; it < O * D; it += kWideThreads) {
      const int o = it / D, i = it - (it / D) * D;
      float sum = 0.0f;
      for (int u = 0; u < V; u++)
        if (ef_s[u]) sum += el_s[u * OMAX + o] * phi_s[u * DP + i];
      dw_s[o * D + i] += sum;
    }
  }
  for (int it = t; it < O * D; it += kWideThreads)
    if (dw_s[it] != 0.0f) atomicAdd(&dW[it], dw_s[it]);
}

template <int F, int OMAX>
void launch_prim_wide(const Scene& sc, GeomState& g, float* dconf, float* dtable, float* dW, cudaStream_t s) {
  const int D = sc.L * F;
  const size_t smem = sizeof(float) * (OMAX * bwd_dp(D) + 3 * pad4(sc.L) + 2 * kWideThreads * OMAX +
                                       kWideThreads * bwd_dp(D) + OMAX * D + 2 * kWideThreads + 2 * kWideWords + 4);
  auto k = sc.Tmask ? backward_prim_wide_kernel<F, OMAX, true> : backward_prim_wide_kernel<F, OMAX, false>;
  cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  cudaMemsetAsync(g.status + 5, 0, sizeof(uint32_t), s);
  int blocks = resident_blocks(reinterpret_cast<const void*>(k), kWideThreads, smem);
  blocks = blocks < sc.P ? blocks : sc.P;
  if (blocks < 1) blocks = 1;
  k<<<blocks, kWideThreads, smem, s>>>(sc, g, dconf, dtable, dW);
  note_launches(1);
}

template <int F, int OMAX>
void launch_prim_t(const Scene& sc, GeomState& g, float* dmeans, float* dconf, float* dtable, float* dW,
                   cudaStream_t s) {
  if (sc.V > 32) {  // G = 4, 5 (reference mode only; the API rejects the exact mode there)
    launch_prim_wide<F, OMAX>(sc, g, dconf, dtable, dW, s);
    return;
  }
  const int D = sc.L * F;
  size_t smem = sizeof(float) * (bwd_head_floats(D, sc.L, OMAX) + kBwdWarps * bwd_warp_floats(D, OMAX));
  // Box-corner primitives go to backward_corner_kernel (reference formula,
  // 3-tap stencil, the reference's fixed box: where they are common).
  const bool split = !sc.exact && !sc.own_box && make_stencil(sc.genus).S == 3;
  auto k = sc.exact     ? backward_prim_kernel<F, OMAX, true, false, false>
           : sc.own_box ? backward_prim_kernel<F, OMAX, false, true, false>
           : split      ? backward_prim_kernel<F, OMAX, false, false, true>
                        : backward_prim_kernel<F, OMAX, false, false, false>;
  cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  cudaMemsetAsync(g.status + 5, 0, sizeof(uint32_t), s);
  // A resident grid: warps draw primitives from the counter until it runs out.
  int blocks = (sc.P + kBwdWarps - 1) / kBwdWarps;
  const int resident = resident_blocks(reinterpret_cast<const void*>(k), kBwdWarps * 32, smem);
  blocks = blocks < resident ? blocks : resident;
  if (blocks < 1) blocks = 1;
  // the table gradient stays in L2 while primitives scatter into it
  cudaLaunchAttribute attr[1];
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(blocks);
  cfg.blockDim = dim3(kBwdWarps * 32);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cfg.attrs = attr;
  cfg.numAttrs = l2_persist_attr(dtable, (size_t)sc.T * sc.L * F * sizeof(float), attr);
  cudaLaunchKernelEx(&cfg, k, sc, g, dmeans, dconf, dtable, dW);
  note_launches(1);
  if (split) {
    const size_t csmem = sizeof(float) * (corner_head_floats(D, sc.L, OMAX) + kCornerWarps * 32 * OMAX);
    auto kc = backward_corner_kernel<F, OMAX>;
    cudaFuncSetAttribute(kc, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)csmem);
    cudaMemsetAsync(g.status + 8, 0, sizeof(uint32_t), s);
    int cblocks = (sc.P + kCornerWarps - 1) / kCornerWarps;
    const int cres = resident_blocks(reinterpret_cast<const void*>(kc), kCornerWarps * 32, csmem);
    cblocks = cblocks < cres ? cblocks : cres;
    if (cblocks < 1) cblocks = 1;
    kc<<<cblocks, kCornerWarps * 32, csmem, s>>>(sc, g, dconf, dtable, dW);
    note_launches(1);
  }
}

// Properties of the records of primitives whose backward projection puts a
// grid point in another pixel than the forward's (kBwdDiffers, listed by the
// feature stage), re-derived as the reference's backward does
// (backward.cu:404-569) and written over the forward's rec_props, which the
// render has consumed.  One thread per (listed primitive, record slot); the
// per-pixel pass then reads rec_props alone.
template <int OMAX>
__global__ void __launch_bounds__(128) recompute_records_kernel(Scene sc, GeomState g) {
  const uint32_t n_list = g.status[7];
  const uint32_t V = (uint32_t)sc.V;
  for (uint64_t t = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; t < (uint64_t)n_list * V;
       t += (uint64_t)gridDim.x * blockDim.x) {
    const uint32_t q = g.differs_list[t / V], j = (uint32_t)(t % V);
    if (j >= (g.rec_cnt[q] & ~kBwdDiffers)) continue;
    const size_t slot = (size_t)q * V + j;
    const uint32_t key = g.rec_key[slot], tile = key >> 8;
    const int px = (int)((tile % sc.gx) * VI_TILE + (key & 15u)), py = (int)((tile / sc.gx) * VI_TILE + ((key >> 4) & 15u));
    float props[OMAX];
    recompute_props<OMAX>(sc, q, px, py, props);
#pragma unroll
    for (int o = 0; o < OMAX; o++) g.rec_props[slot * OMAX + o] = props[o];
  }
}

}  // namespace

void launch_backward(const Scene& sc, GeomState& g, const ImgState& im, const uint32_t* point_list,
                     const float* dL_dcolor, const float* dL_dfeat, const float* dL_dvis, float* dmeans, float* dconf,
                     float* dtable, float* dW, float* db, cudaStream_t s) {
  const size_t N = (size_t)sc.W * sc.H;
  cudaMemsetAsync(g.rec_pix, 0, (size_t)sc.P * sc.V * sizeof(uint32_t), s);
  const bool o16 = sc.O > 8;
  stage_begin(kStBwdPixel, s);
  if (!sc.exact && sc.P > 0) {  // the exact mode differentiates the forward's properties
    if (o16)
      recompute_records_kernel<16><<<148 * 4, 128, 0, s>>>(sc, g);
    else
      recompute_records_kernel<8><<<148 * 4, 128, 0, s>>>(sc, g);
    note_launches(1);
  }
  if (N > 0) {
    note_launches(1);
    const unsigned blocks = (unsigned)((N + 255) / 256);
    if (sc.exact) {
      if (o16)
        backward_pixel_exact_kernel<16><<<blocks, 256, 0, s>>>(sc, g, im, point_list, dL_dcolor, dL_dfeat, dL_dvis, dmeans, db);
      else
        backward_pixel_exact_kernel<8><<<blocks, 256, 0, s>>>(sc, g, im, point_list, dL_dcolor, dL_dfeat, dL_dvis, dmeans, db);
    } else if (o16) {
      backward_pixel_kernel<16><<<blocks, 256, 0, s>>>(sc, g, im, dL_dcolor, dL_dfeat, db);
    } else {
      backward_pixel_kernel<8><<<blocks, 256, 0, s>>>(sc, g, im, dL_dcolor, dL_dfeat, db);
    }
  }
  stage_end(kStBwdPixel, s);
  stage_begin(kStBwdPrim, s);
  switch (sc.F) {
    case 1: o16 ? launch_prim_t<1, 16>(sc, g, dmeans, dconf, dtable, dW, s) : launch_prim_t<1, 8>(sc, g, dmeans, dconf, dtable, dW, s); break;
    case 2: o16 ? launch_prim_t<2, 16>(sc, g, dmeans, dconf, dtable, dW, s) : launch_prim_t<2, 8>(sc, g, dmeans, dconf, dtable, dW, s); break;
    case 4: o16 ? launch_prim_t<4, 16>(sc, g, dmeans, dconf, dtable, dW, s) : launch_prim_t<4, 8>(sc, g, dmeans, dconf, dtable, dW, s); break;
    case 8: o16 ? launch_prim_t<8, 16>(sc, g, dmeans, dconf, dtable, dW, s) : launch_prim_t<8, 8>(sc, g, dmeans, dconf, dtable, dW, s); break;
    default: break;
  }
  stage_end(kStBwdPrim, s);
}

}  // namespace vi
