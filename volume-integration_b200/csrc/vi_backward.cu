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
//     projections put every grid point in the same pixel; otherwise the
//     record is recomputed with the backward projection).
//  2. backward_prim: one warp per primitive, lane = grid point, gathers its
//     contributing records and produces
//       dconf[q,g]  = sum_p (dIn_p . phi_g) * g'_{p,g}                (backward.cu:697-710)
//       dtable      += (sum_p dIn_p * g'_{p,g} * conf_g) * corner weight (hashgrid.h:43-95)
//       dW, db      += dpre_p (x) in_p, dpre_p                          (backward.cu:621-641)
//     where g' is the stencil magnitude of "neighbour's screen point lies in
//     pixel p" (backward.cu:644-689).  The table scatter is linear in dIn, so
//     each grid point scatters once per level and corner instead of once per
//     pixel, and lanes hitting the same entry are reduced inside the warp before
//     one vector atomic.  dW/db are reduced per CTA before global atomics.
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
    level_setup(pos, res, b, t);
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
  float conf[32];
  uint32_t posm = 0;
  for (int g = 0; g < V; g++) {
    conf[g] = sc.conf[(size_t)q * V + g];
    if (conf[g] > 0.0f) posm |= 1u << g;
  }
  const float3 c = make_float3(sc.means[3 * q], sc.means[3 * q + 1], sc.means[3 * q + 2]);
  float acc[OMAX];
  for (int o = 0; o < OMAX; o++) acc[o] = 0.0f;
  float phi[64];
  for (int g = 0; g < V; g++) {
    if (!(conf[g] > 0.0f)) continue;
    const float3 pos = grid_pos(c, g, G, sc.step, sc.gof);
    const float2 sb = project(pos, sc.proj, sc.W, sc.H, false);
    if (pix_coord(sb.x) != px || pix_coord(sb.y) != py) continue;
    const float mag = occ_mag(posm, g, G, st);
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

template <int OMAX>
__global__ void __launch_bounds__(256) backward_pixel_kernel(Scene sc, GeomState g, ImgState im,
                                                            const float* __restrict__ dL_dcolor,
                                                            const float* __restrict__ dL_dfeat) {
  const size_t N = (size_t)sc.W * sc.H;
  const size_t pix = blockIdx.x * (size_t)blockDim.x + threadIdx.x;
  if (pix >= N) return;
  const int K = sc.K;
  int nc = min(im.n_contrib[pix], K);
  if (nc <= 0) return;
  const int O = sc.O, B = O - 1, Fout = sc.Fout, V = sc.V;
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
  const int px = (int)(pix % sc.W), py = (int)(pix / sc.W);
  for (int k = nc - 1; k >= 0; k--) {
    const uint32_t rec = im.contrib_rec[pix * K + k];
    const float dt = im.delta_t[pix * K + k];
    const uint32_t q = rec / V;
    float props[OMAX];
    if (g.rec_cnt[q] & kBwdDiffers) {
      recompute_props<OMAX>(sc, q, px, py, props);
    } else {
      const float4* src = reinterpret_cast<const float4*>(g.rec_props + (size_t)rec * OMAX);
#pragma unroll
      for (int o4 = 0; o4 < OMAX / 4; o4++) {
        float4 v = src[o4];
        props[4 * o4] = v.x; props[4 * o4 + 1] = v.y; props[4 * o4 + 2] = v.z; props[4 * o4 + 3] = v.w;
      }
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
    for (int d = 0; d < OMAX - 1; d++) {
      if (d < B) {
        const float y = props[d];
        dOut[d] *= y;
        after[d] = y + after[d] * (1.0f - y);
      }
    }
  }
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

constexpr int kBwdWarps = 8;

// Floats of shared memory each warp of backward_prim_kernel owns: phi rows, E
// rows and its dW partial sums.
__host__ __device__ inline int bwd_warp_floats(int D, int OMAX) { return 32 * (D + 1) + 32 * OMAX + OMAX * D; }

// One warp per primitive, lane g = grid point g.  With dIn_p = W^T dpre_p
// (backward.cu:608-619), every per-pair sum collapses onto O-wide vectors:
//   v_g  = sum_p g'_{p,g} dpre_p                 -> dconf_g = v_g . (W phi_g)
//   vA_g = sum_p [|g' conf_g| > 1e-9] g' dpre_p  -> table coefficient conf_g W^T vA_g
//   E_g  = w_g dpre_{p(g)}                       -> dW += E_g (x) phi_g
// so each contributing pixel costs O multiply-adds per lane, and the hashgrid
// gather (for phi_g) and scatter (for the table gradient) share one level loop.
template <int F, int OMAX>
__global__ void __launch_bounds__(kBwdWarps * 32, 3) backward_prim_kernel(Scene sc, GeomState g, float* __restrict__ dconf,
                                                                      float* __restrict__ dtable, float* __restrict__ dW,
                                                                      float* __restrict__ db) {
  extern __shared__ float smem[];
  const int L = sc.L, D = L * F, O = sc.O, V = sc.V, G = sc.G;
  const int DS = D + 1;
  float* W_s = smem;              // [D][OMAX]: W transposed
  float* dW_s = W_s + D * OMAX;   // [OMAX][D]
  float* db_s = dW_s + OMAX * D;  // [OMAX]
  float* resf_s = db_s + OMAX;    // [L] level resolutions as float
  const int w = threadIdx.x >> 5;
  const uint32_t lane = threadIdx.x & 31;
  float* phi_s = resf_s + L + w * bwd_warp_floats(D, OMAX);  // [32][DS]
  float* E_s = phi_s + 32 * DS;                                        // [32][OMAX]
  float* dWw = E_s + 32 * OMAX;  // [OMAX][D] this warp's dW partial sums; lane j owns columns j, j+32
  for (int i = (int)lane; i < OMAX * D; i += 32) dWw[i] = 0.0f;

  for (int i = threadIdx.x; i < D * OMAX; i += blockDim.x) {
    const int d = i / OMAX, o = i % OMAX;
    W_s[i] = o < O ? sc.Wl[o * D + d] : 0.0f;
    dW_s[i] = 0.0f;
  }
  for (int i = threadIdx.x; i < OMAX; i += blockDim.x) db_s[i] = 0.0f;
  for (int i = threadIdx.x; i < L; i += blockDim.x) resf_s[i] = (float)sc.res[i];
  __syncthreads();

  const Stencil st = make_stencil(sc.genus);
  const GridPt gpt = grid_point((int)lane < V ? (int)lane : 0, G, sc.gof);
  const uint32_t p0 = (uint32_t)__ldg(sc.primes), p1 = (uint32_t)__ldg(sc.primes + 1),
                 p2 = (uint32_t)__ldg(sc.primes + 2);
  float dbacc = 0.0f;

  // Primitives are handed out in batches of kGrab per warp from a counter
  // (status[5]): warps that draw cheap primitives take more, so no warp idles at
  // the final reduction while the counter sees one atomic per batch.
  constexpr int kGrab = 8;
  for (int q0 = 0, qi = kGrab;;) {
    if (qi == kGrab) {
      if (lane == 0) q0 = (int)atomicAdd(g.status + 5, (unsigned)kGrab);
      q0 = __shfl_sync(0xffffffffu, q0, 0);
      qi = 0;
    }
    const int q = q0 + qi++;
    if (q >= sc.P) break;
    const uint32_t n = g.rec_cnt[q] & ~kBwdDiffers;
    if (n == 0) continue;
    const size_t s0 = (size_t)q * V;
    const uint32_t rp = lane < n ? g.rec_pix[s0 + lane] : 0u;
    const uint32_t cm = __ballot_sync(0xffffffffu, rp != 0u);
    if (cm == 0) continue;

    const bool act = (int)lane < V;
    const float conf = act ? sc.conf[s0 + lane] : 0.0f;
    const float3 c = make_float3(sc.means[3 * q], sc.means[3 * q + 1], sc.means[3 * q + 2]);
    const float3 pos = grid_pos_rel(c, gpt.rel, sc.step);
    const float2 sb = project(pos, sc.proj, sc.W, sc.H, false);
    const int bx = pix_coord(sb.x), by = pix_coord(sb.y);
    const int bpix = (act && bx >= 0 && bx < sc.W && by >= 0 && by < sc.H) ? by * sc.W + bx : -1;
    const uint32_t posm = __ballot_sync(0xffffffffu, act && conf > 0.0f);
    const float mag = act ? occ_mag(posm, gpt, G, st) : 0.0f;
    const float wE = (act && conf > 0.0f && mag > 1e-7f) ? fmul(conf, mag) : 0.0f;

    float v[OMAX], vA[OMAX];
#pragma unroll
    for (int o = 0; o < OMAX; o++) v[o] = vA[o] = 0.0f;
    bool hasE = false, hasV = false, hasA = false;
    uint32_t m = cm;
    while (m) {
      const int j = __ffs(m) - 1;
      m &= m - 1;
      const size_t slot = s0 + j;
      const int ppix = (int)__shfl_sync(0xffffffffu, rp, j) - 1;  // pixel of this contribution
      float dpre[OMAX];
      const float4* src = reinterpret_cast<const float4*>(g.rec_dpre + slot * OMAX);
#pragma unroll
      for (int o4 = 0; o4 < OMAX / 4; o4++) {
        const float4 x = src[o4];
        dpre[4 * o4] = x.x; dpre[4 * o4 + 1] = x.y; dpre[4 * o4 + 2] = x.z; dpre[4 * o4 + 3] = x.w;
      }
      if ((int)lane < O) dbacc += g.rec_dpre[slot * OMAX + lane];
      const uint32_t inm = __ballot_sync(0xffffffffu, bpix == ppix);
      if (((inm >> lane) & 1u) && wE != 0.0f) {
        hasE = true;
#pragma unroll
        for (int o = 0; o < OMAX; o++) E_s[lane * OMAX + o] = fmul(wE, dpre[o]);
      }
      const float gp = act ? occ_mag(inm, gpt, G, st) : 0.0f;
      if (gp > 1e-7f) {
        hasV = true;
        const bool doA = fabsf(fmul(gp, conf)) > 1e-9f;
        hasA |= doA;
#pragma unroll
        for (int o = 0; o < OMAX; o++) {
          const float x = gp * dpre[o];
          v[o] += x;
          if (doA) vA[o] += x;
        }
      }
    }
    if (!__any_sync(0xffffffffu, hasE || hasV)) continue;

    // One pass over the levels: gather phi_g (for dconf and dW), scatter the table gradient.
    float2 mlp2[OMAX / 2];
#pragma unroll
    for (int o = 0; o < OMAX / 2; o++) mlp2[o] = make_float2(0.0f, 0.0f);
    float* phi_row = phi_s + lane * DS;
    const bool gather = hasE || hasV;
    const float3 nrm = hash_norm(pos);
    const uint32_t amask = __ballot_sync(0xffffffffu, hasA);
    const int afirst = amask ? __ffs(amask) - 1 : 0;
#pragma unroll 1
    for (int l = 0; l < L; l++) {
      const LevelCorners lc =
          level_corners(nrm, __ldg(sc.res + l), resf_s[l], __ldg(sc.do_hash + l) != 0, p0, p1, p2, sc.T);
      const uint32_t cmask = (gather || hasA) ? lc.mask : 0u;
      float acc[F], a[F];
#pragma unroll
      for (int f = 0; f < F; f++) {
        acc[f] = 0.0f;
        // table coefficient of this level: conf_g * sum_o W[o][l*F+f] vA[o]
        float2 sum = make_float2(0.0f, 0.0f);
        const float2* wr = reinterpret_cast<const float2*>(W_s + (l * F + f) * OMAX);
#pragma unroll
        for (int o = 0; o < OMAX / 2; o++) sum = __ffma2_rn(wr[o], make_float2(vA[2 * o], vA[2 * o + 1]), sum);
        a[f] = conf * (sum.x + sum.y);
      }
      // Every lane with a table gradient on the same cell set (points clamped to
      // the hashgrid box): sum per corner across the warp, one atomic per corner.
      bool uni = false;
      if (amask) {
        const uint32_t m0 = __shfl_sync(0xffffffffu, cmask, afirst);
        const uint32_t i0 = __shfl_sync(0xffffffffu, lc.ix0, afirst);
        const uint32_t j0 = __shfl_sync(0xffffffffu, lc.iy0, afirst);
        const uint32_t k0 = __shfl_sync(0xffffffffu, lc.iz0, afirst);
        uni = __all_sync(0xffffffffu, !hasA || (cmask == m0 && lc.ix0 == i0 && lc.iy0 == j0 && lc.iz0 == k0)) &&
              __popc(amask) > 1;
      }
      const float* lvl = sc.table + (size_t)l * F;
      float* dst = dtable + (size_t)l * F;
      uint32_t um = __reduce_or_sync(0xffffffffu, cmask);
      while (um) {
        const int k = __ffs(um) - 1;
        um &= um - 1;
        const bool on = (cmask >> k) & 1u;
        const uint32_t e = on ? corner_index(lc, k, sc.T, sc.Tmask) : 0u;
        const float cw = on ? corner_weight(lc, k) : 0.0f;
        if (gather && on) {
          const FVec<F> x = load_feat<F>(lvl + (size_t)e * L * F);
#pragma unroll
          for (int f = 0; f < F; f++) acc[f] += x.v[f] * cw;
        }
        if (uni) {
          if ((__shfl_sync(0xffffffffu, cmask, afirst) >> k) & 1u) {
            float x[F];
#pragma unroll
            for (int f = 0; f < F; f++) {
              float y = hasA ? a[f] * cw : 0.0f;
#pragma unroll
              for (int off = 16; off > 0; off >>= 1) y += __shfl_xor_sync(0xffffffffu, y, off);
              x[f] = y;
            }
            if ((int)lane == afirst) atomic_vec<F>(dst + (size_t)e * L * F, x);
          }
        } else if (hasA && on) {
          float x[F];
#pragma unroll
          for (int f = 0; f < F; f++) x[f] = a[f] * cw;
          atomic_vec<F>(dst + (size_t)e * L * F, x);
        }
      }
#pragma unroll
      for (int f = 0; f < F; f++) {
        const float x = acc[f];
        const float2* wr = reinterpret_cast<const float2*>(W_s + (l * F + f) * OMAX);
#pragma unroll
        for (int o = 0; o < OMAX / 2; o++) mlp2[o] = __ffma2_rn(wr[o], make_float2(x, x), mlp2[o]);
        if (hasE) phi_row[l * F + f] = x;
      }
    }
    if (act) {
      float dX = 0.0f;
#pragma unroll
      for (int o = 0; o < OMAX / 2; o++) dX += v[2 * o] * mlp2[o].x + v[2 * o + 1] * mlp2[o].y;
      dconf[s0 + lane] = dX;
    }
    // dW += E_g (x) phi_g over the lanes with an E contribution.
    const uint32_t em = __ballot_sync(0xffffffffu, hasE);
    __syncwarp();
    for (int jj = (int)lane; jj < D; jj += 32) {
      float acc[OMAX];
#pragma unroll
      for (int o = 0; o < OMAX; o++) acc[o] = dWw[o * D + jj];
      uint32_t mm = em;
      while (mm) {
        const int gg = __ffs(mm) - 1;
        mm &= mm - 1;
        const float x = phi_s[gg * DS + jj];
#pragma unroll
        for (int o = 0; o < OMAX; o++) acc[o] += E_s[gg * OMAX + o] * x;
      }
#pragma unroll
      for (int o = 0; o < OMAX; o++) dWw[o * D + jj] = acc[o];
    }
    __syncwarp();
  }

  // CTA reduction of dW and db, then one global atomic per element.
  __syncwarp();
  for (int i = (int)lane; i < O * D; i += 32)
    if (dWw[i] != 0.0f) atomicAdd(&dW_s[i], dWw[i]);
  if ((int)lane < O && dbacc != 0.0f) atomicAdd(&db_s[lane], dbacc);
  __syncthreads();
  for (int i = threadIdx.x; i < O * D; i += blockDim.x)
    if (dW_s[i] != 0.0f) atomicAdd(&dW[i], dW_s[i]);
  for (int i = threadIdx.x; i < O; i += blockDim.x)
    if (db_s[i] != 0.0f) atomicAdd(&db[i], db_s[i]);
}

template <int F, int OMAX>
void launch_prim_t(const Scene& sc, GeomState& g, float* dconf, float* dtable, float* dW, float* db, cudaStream_t s) {
  const int D = sc.L * F;
  size_t smem = sizeof(float) * (2 * OMAX * D + OMAX + sc.L + kBwdWarps * bwd_warp_floats(D, OMAX));
  auto k = backward_prim_kernel<F, OMAX>;
  cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  cudaMemsetAsync(g.status + 5, 0, sizeof(uint32_t), s);
  int blocks = (sc.P + kBwdWarps - 1) / kBwdWarps;
  blocks = blocks < 148 * 8 ? blocks : 148 * 8;
  if (blocks < 1) blocks = 1;
  k<<<blocks, kBwdWarps * 32, smem, s>>>(sc, g, dconf, dtable, dW, db);
  note_launches(1);
}

}  // namespace

void launch_backward(const Scene& sc, GeomState& g, const ImgState& im, const float* dL_dcolor, const float* dL_dfeat,
                     float* dconf, float* dtable, float* dW, float* db, cudaStream_t s) {
  const size_t N = (size_t)sc.W * sc.H;
  cudaMemsetAsync(g.rec_pix, 0, (size_t)sc.P * sc.V * sizeof(uint32_t), s);
  const bool o16 = sc.O > 8;
  stage_begin(kStBwdPixel, s);
  if (N > 0) {
    note_launches(1);
    const unsigned blocks = (unsigned)((N + 255) / 256);
    if (o16)
      backward_pixel_kernel<16><<<blocks, 256, 0, s>>>(sc, g, im, dL_dcolor, dL_dfeat);
    else
      backward_pixel_kernel<8><<<blocks, 256, 0, s>>>(sc, g, im, dL_dcolor, dL_dfeat);
  }
  stage_end(kStBwdPixel, s);
  stage_begin(kStBwdPrim, s);
  switch (sc.F) {
    case 1: o16 ? launch_prim_t<1, 16>(sc, g, dconf, dtable, dW, db, s) : launch_prim_t<1, 8>(sc, g, dconf, dtable, dW, db, s); break;
    case 2: o16 ? launch_prim_t<2, 16>(sc, g, dconf, dtable, dW, db, s) : launch_prim_t<2, 8>(sc, g, dconf, dtable, dW, db, s); break;
    case 4: o16 ? launch_prim_t<4, 16>(sc, g, dconf, dtable, dW, db, s) : launch_prim_t<4, 8>(sc, g, dconf, dtable, dW, db, s); break;
    case 8: o16 ? launch_prim_t<8, 16>(sc, g, dconf, dtable, dW, db, s) : launch_prim_t<8, 8>(sc, g, dconf, dtable, dW, db, s); break;
    default: break;
  }
  stage_end(kStBwdPrim, s);
}

}  // namespace vi
