// Feature stage: stage 1 of the reference render kernel (forward.cu:401-463),
// run once per visible primitive instead of once per (tile, primitive), fused
// with the per-pixel accumulation of stage 2 (forward.cu:481-643), which for a
// given (primitive, pixel) depends only on the primitive.
//
// One warp per primitive, lane g = grid point g (V = G^3 <= 32).  Per lane:
// confidence, forward and backward screen positions and the conf>0 stencil
// magnitude.  The hashgrid features and the linear layer are then computed once
// per distinct normalised position rather than once per grid point: lanes are
// grouped by position, the (position, level) pairs are spread over the warp's
// lanes level by level, and the linear layer runs over (position, output) pairs.  Lanes that
// land in the same pixel are summed in grid-point order by the lowest such lane,
// exactly the order of the reference's loop, and every pixel whose occupancy sum
// passes the reference's 1e-7 test becomes one record:
//   key   = tile * 256 + pixel-in-tile (only tiles inside the primitive's rect)
//   props = sigmoid(acc + b) for colour and features, exp(acc + b) for density.
// Records of a primitive are stored grouped by tile, ascending, in slots
// [q*V, q*V + count).
#include <cuda_runtime.h>

#include <cstdint>

#include "vi_kernels.cuh"

namespace vi {
namespace {

constexpr int kFeatWarps = 8;

__host__ __device__ inline int pad4(int x) { return (x + 3) & ~3; }
// Shared memory: W [OMAX][DP] (rows of the linear layer, DP = pad4(D) + 4 to
// spread rows over banks), bias, per-level resolution / hash flag, then per warp
// phi [32][DP] (features of each position class), mlp [32][OMAX] (W phi of each
// class), class positions [32] float4, and per-lane magnitude, weight and class.
__host__ __device__ inline int feat_dp(int D) { return pad4(D) + 4; }
__host__ __device__ inline int feat_head_floats(int D, int L, int OMAX) {
  return OMAX * feat_dp(D) + OMAX + 3 * pad4(L) + 8 * feat_dp(D) + 8 * OMAX;
}
__host__ __device__ inline int feat_warp_floats(int D, int OMAX) { return 32 * feat_dp(D) + 32 * OMAX + 4 * 32 + 3 * 32; }

// POW2: the table size T is a power of two (hash modulo by mask).
template <int F, int OMAX, bool POW2>
__global__ void __launch_bounds__(kFeatWarps * 32, 3) features_kernel(Scene sc, GeomState g) {
  extern __shared__ float4 smem4[];
  float* smem = reinterpret_cast<float*>(smem4);
  const int L = sc.L, D = L * F, DP = feat_dp(D), O = sc.O, V = sc.V, G = sc.G;
  float* W_s = smem;                                       // [OMAX][DP]
  float* b_s = W_s + OMAX * DP;                            // [OMAX]
  float* resf_s = b_s + OMAX;                              // [L] level resolutions as float
  int* res_s = reinterpret_cast<int*>(resf_s + pad4(L));   // [L]
  int* hash_s = res_s + pad4(L);                           // [L]
  float* cphi_s = reinterpret_cast<float*>(hash_s + pad4(L));  // [8][DP] box-corner features
  float* cmlp_s = cphi_s + 8 * DP;                             // [8][OMAX] W phi of the box corners
  const int w = threadIdx.x >> 5, lane = threadIdx.x & 31;
  float* phi_s = smem + feat_head_floats(D, L, OMAX) + w * feat_warp_floats(D, OMAX);  // [32][DP]
  float* mlp_s = phi_s + 32 * DP;                                                    // [32][OMAX]
  float4* npos_s = reinterpret_cast<float4*>(mlp_s + 32 * OMAX);                     // [32]
  float* mag_s = reinterpret_cast<float*>(npos_s + 32);                              // [32]
  float* wgt_s = mag_s + 32;                                                         // [32]
  int* cls_s = reinterpret_cast<int*>(wgt_s + 32);                                   // [32]
  for (int i = threadIdx.x; i < L; i += blockDim.x) {
    res_s[i] = sc.res[i];
    resf_s[i] = (float)sc.res[i];
    hash_s[i] = sc.do_hash[i];
  }
  for (int i = threadIdx.x; i < OMAX * DP; i += blockDim.x) {
    const int o = i / DP, d = i % DP;
    W_s[i] = o < O && d < D ? sc.Wl[o * D + d] : 0.0f;
  }
  for (int i = threadIdx.x; i < OMAX; i += blockDim.x) b_s[i] = i < O ? sc.bl[i] : 0.0f;
  __syncthreads();
  {
    const uint32_t c0 = (uint32_t)__ldg(sc.primes), c1 = (uint32_t)__ldg(sc.primes + 1), c2 = (uint32_t)__ldg(sc.primes + 2);
    box_corner_features<F, true, POW2 ? 1 : 0>(sc, res_s, resf_s, hash_s, c0, c1, c2, DP, cphi_s);
    for (int t = threadIdx.x; t < 8 * OMAX; t += blockDim.x) {
      const int c = t / OMAX, o = t % OMAX;
      float acc = 0.0f;
      for (int i = 0; i < D; i++) acc = __fmaf_rn(W_s[o * DP + i], cphi_s[c * DP + i], acc);
      cmlp_s[t] = acc;
    }
    __syncthreads();
  }

  const Stencil st = make_stencil(sc.genus);
  const GridPt gp = grid_point(lane < V ? lane : 0, G, sc.gof);
  const uint32_t lt_mask = (1u << lane) - 1;
  const uint32_t p0 = (uint32_t)__ldg(sc.primes), p1 = (uint32_t)__ldg(sc.primes + 1),
                 p2 = (uint32_t)__ldg(sc.primes + 2);
  const uint32_t stride = sc.tab_e;
  const int OP = OMAX;
  // Warps claim chunks of 32 consecutive primitives from a counter (status[4]):
  // the cost of a primitive varies widely, so a fixed share per warp would
  // leave most warps idle at the end.  One radii load per chunk picks its
  // visible primitives.
  for (;;) {
    int ch = 0;
    if (lane == 0) ch = (int)atomicAdd(g.status + 4, 1u);
    const int qb = __shfl_sync(0xffffffffu, ch, 0) * 32;
    if (qb >= sc.P) break;
    const int ql = qb + lane;
    const int rl = ql < sc.P ? g.radii[ql] : 0;
    if (ql < sc.P && rl <= 0) {
      g.rec_cnt[ql] = 0;
      g.cls_base[ql] = kNoCache;
    }
    uint32_t vis = __ballot_sync(0xffffffffu, rl > 0);
    while (vis) {
    const int qi = __ffs(vis) - 1;
    vis &= vis - 1;
    const int q = qb + qi;
    const int r = __shfl_sync(0xffffffffu, rl, qi);
    const float3 c = make_float3(sc.means[3 * q], sc.means[3 * q + 1], sc.means[3 * q + 2]);
    const float2 m2 = make_float2(g.means2D[2 * q], g.means2D[2 * q + 1]);
    // getRect with the same float arithmetic as preprocess (auxiliary.h:55-65).
    const float rf = (float)r;
    const unsigned x0 = min(sc.gx, (unsigned)max(0, (int)fmul(fsub(m2.x, rf), 0.0625f)));
    const unsigned y0 = min(sc.gy, (unsigned)max(0, (int)fmul(fsub(m2.y, rf), 0.0625f)));
    const unsigned x1 = min(sc.gx, (unsigned)max(0, (int)fmul(fsub(fadd(fadd(m2.x, rf), 16.0f), 1.0f), 0.0625f)));
    const unsigned y1 = min(sc.gy, (unsigned)max(0, (int)fmul(fsub(fadd(fadd(m2.y, rf), 16.0f), 1.0f), 0.0625f)));

    const bool act = lane < V;
    const float conf = act ? sc.conf[(size_t)q * V + lane] : 0.0f;
    const float3 pos = grid_pos_rel(c, gp.rel, sc.step);
    const float2 sf = project(pos, sc.proj, sc.W, sc.H, true);
    const float2 sb = project(pos, sc.proj, sc.W, sc.H, false);
    const int fx = pix_coord(sf.x), fy = pix_coord(sf.y);
    const bool differs = __any_sync(0xffffffffu, act && (fx != pix_coord(sb.x) || fy != pix_coord(sb.y)));
    const uint32_t posm = __ballot_sync(0xffffffffu, act && conf > 0.0f);
    const float mag = act ? occ_mag(posm, gp, G, st) : 0.0f;
    const bool inside = fx >= 0 && fx < sc.W && fy >= 0 && fy < sc.H;
    const unsigned tx = (unsigned)fx >> 4, ty = (unsigned)fy >> 4;
    const bool vpt = act && conf > 0.0f && inside && tx >= x0 && tx < x1 && ty >= y0 && ty < y1;
    const bool need = vpt && mag > 1e-7f;

    uint32_t cbase = kNoCache;
    if (__any_sync(0xffffffffu, need)) {
      // Features of each distinct position of all grid points (the backward
      // reads them from phi_cache): items (class u, level l) over the lanes.
      const PosClasses pc = pos_classes(hash_norm(pos, sc.hlo, sc.hext), act);
      if (act && (pc.peers & lt_mask) == 0) {
        const float3 n = hash_norm(pos, sc.hlo, sc.hext);
        npos_s[pc.cls] = make_float4(n.x, n.y, n.z, 0.0f);
      }
      __syncwarp();
      const float4 n0 = npos_s[0];
      if (pc.U == 1 && box_corner(n0)) {
        // every grid point clamps to one corner of the hashgrid box
        const int cc = box_corner_index(n0);
        if (lane < OMAX) mlp_s[lane] = cmlp_s[cc * OMAX + lane];
        cbase = kCornerCache | (uint32_t)cc;
      } else {
        // Two steps of the level walk at a time, so that each lane has the
        // loads of two (class, level) items in flight.
        const LevelWalk it(pc.U, L);
        for (int l0 = 0; l0 < L; l0 += 2 * it.per) {
          const bool v0 = it.valid(l0), v1 = it.valid(l0 + it.per);
          const float4 n4 = npos_s[it.u];
          const float3 nn = make_float3(n4.x, n4.y, n4.z);
          const int la = it.level(l0), lb = it.level(l0 + it.per);
          float acc0[F], acc1[F];
#pragma unroll
          for (int f = 0; f < F; f++) acc0[f] = acc1[f] = 0.0f;
          if (v0) {
            const LevelCorners lc = level_corners(nn, res_s[la], resf_s[la], hash_s[la] != 0, p0, p1, p2, sc.T);
            gather_level<F, POW2>(lc, sc.table + (size_t)la * sc.tab_l, stride, sc.T, sc.Tmask, acc0);
          }
          if (v1) {
            const LevelCorners lc = level_corners(nn, res_s[lb], resf_s[lb], hash_s[lb] != 0, p0, p1, p2, sc.T);
            gather_level<F, POW2>(lc, sc.table + (size_t)lb * sc.tab_l, stride, sc.T, sc.Tmask, acc1);
          }
          if (v0) {
#pragma unroll
            for (int f = 0; f < F; f++) phi_s[it.u * DP + la * F + f] = acc0[f];
          }
          if (v1) {
#pragma unroll
            for (int f = 0; f < F; f++) phi_s[it.u * DP + lb * F + f] = acc1[f];
          }
        }
        __syncwarp();
        // Keep the classes' features for the backward in phi_cache: slots
        // [q*V, q*V + U) when the cache holds V slots per primitive, else U
        // consecutive slots from a counter (status[6]) while they fit.
        if ((uint64_t)g.phi_cap >= (uint64_t)sc.P * (uint64_t)V) {
          cbase = (uint32_t)q * (uint32_t)V;
        } else {
          if (lane == 0) {
            const uint32_t b = atomicAdd(g.status + 6, (uint32_t)pc.U);
            cbase = (uint64_t)b + (uint64_t)pc.U <= (uint64_t)g.phi_cap ? b : kNoCache;
          }
          cbase = __shfl_sync(0xffffffffu, cbase, 0);
        }
        if (cbase != kNoCache) {
          float* dst = g.phi_cache + (size_t)cbase * D;
          for (int i = lane; i < pc.U * D; i += 32) dst[i] = phi_s[(i / D) * DP + i % D];
        }
        // Linear layer per class: mlp[u][o] = sum_i W[o][i] phi_u[i].
        class_linear<OMAX>(W_s, phi_s, DP, D, pc.U, mlp_s);
      }
      if (need) {
        cls_s[lane] = pc.cls;
        wgt_s[lane] = fmul(conf, mag);
      }
    }
    mag_s[lane] = mag;
    __syncwarp();

    const uint32_t key = vpt ? (uint32_t)fy * (uint32_t)sc.W + (uint32_t)fx : 0xffffffffu - lane;
    const uint32_t peers = __match_any_sync(0xffffffffu, key);
    bool is_rec = false;
    float props[OMAX];
    if (vpt && (peers & lt_mask) == 0) {
      float ogs = 0.0f, acc[OMAX];
#pragma unroll
      for (int o = 0; o < OMAX; o++) acc[o] = 0.0f;
      uint32_t m = peers;
      while (m) {
        const int src = __ffs(m) - 1;
        m &= m - 1;
        const float mg = mag_s[src];
        ogs = fadd(ogs, mg);
        if (mg > 1e-7f) {  // a lane with features: conf > 0 and in this pixel
          const float wg = wgt_s[src];
          const float4* mr = reinterpret_cast<const float4*>(mlp_s + cls_s[src] * OMAX);
#pragma unroll
          for (int o4 = 0; o4 < OMAX / 4; o4++) {
            const float4 x = mr[o4];
            acc[4 * o4] = fadd(acc[4 * o4], fmul(x.x, wg));
            acc[4 * o4 + 1] = fadd(acc[4 * o4 + 1], fmul(x.y, wg));
            acc[4 * o4 + 2] = fadd(acc[4 * o4 + 2], fmul(x.z, wg));
            acc[4 * o4 + 3] = fadd(acc[4 * o4 + 3], fmul(x.w, wg));
          }
        }
      }
      if (!(ogs < 1e-7f)) {
        is_rec = true;
#pragma unroll
        for (int o = 0; o < OMAX; o++) {
          const float pre = fadd(acc[o], b_s[o]);
          props[o] = o < O - 1 ? sigmoidf_(pre) : (o == O - 1 ? expf(pre) : 0.0f);
        }
      }
    }
    // Records are grouped by tile, ascending, and in lane order inside a tile
    // (the render finds a tile's records by key; their order inside it is free).
    const uint32_t recmask = __ballot_sync(0xffffffffu, is_rec);
    const uint32_t tkey = ty * sc.gx + tx;
    const uint32_t rkey = (tkey << 8) | (((unsigned)fy & 15u) << 4) | ((unsigned)fx & 15u);
    uint32_t rank = 0, rem = recmask;
    while (rem) {
      const uint32_t t = __shfl_sync(0xffffffffu, tkey, __ffs(rem) - 1);
      const uint32_t grp = __ballot_sync(0xffffffffu, is_rec && tkey == t);
      rem &= ~grp;
      if (t < tkey) rank += __popc(grp);
      else if (t == tkey) rank += __popc(grp & lt_mask);
    }
    if (is_rec) {
      const size_t slot = (size_t)q * V + rank;
      g.rec_key[slot] = rkey;
      float4* dst = reinterpret_cast<float4*>(g.rec_props + slot * OP);
#pragma unroll
      for (int o4 = 0; o4 < OMAX / 4; o4++)
        dst[o4] = make_float4(props[4 * o4], props[4 * o4 + 1], props[4 * o4 + 2], props[4 * o4 + 3]);
    }
    if (lane == 0) {
      g.rec_cnt[q] = (uint32_t)__popc(recmask) | (differs ? kBwdDiffers : 0u);
      g.cls_base[q] = cbase;
      // the backward re-derives these records' properties with its own projection
      if (differs && recmask) g.differs_list[atomicAdd(g.status + 7, 1u)] = (uint32_t)q;
    }
    __syncwarp();
    }
  }
}

// Grids of G = 4 or 5 (V = 64 or 125 grid points, up to the reference's
// MAX_GRID_SIZE of 5, forward.cu:204-205): one block of kWideThreads threads per
// primitive, thread t = grid point t, with the cross-point steps (occupancy
// stencil, per-pixel sums in grid-point order, record ranking) through shared
// memory.  Every grid point that contributes gathers its own features (no
// position classes and no feature cache: the backward gathers again).  The
// records are the same as the warp kernel's: one per pixel whose occupancy
// sum passes 1e-7, grouped by tile, ascending.
template <int F, int OMAX, bool POW2>
__global__ void __launch_bounds__(kWideThreads) features_wide_kernel(Scene sc, GeomState g) {
  extern __shared__ float4 smem4[];
  float* smem = reinterpret_cast<float*>(smem4);
  const int L = sc.L, D = L * F, DP = feat_dp(D), O = sc.O, V = sc.V, G = sc.G;
  float* W_s = smem;                                       // [OMAX][DP]
  float* b_s = W_s + OMAX * DP;                            // [OMAX]
  float* resf_s = b_s + OMAX;                              // [L]
  int* res_s = reinterpret_cast<int*>(resf_s + pad4(L));   // [L]
  int* hash_s = res_s + pad4(L);                           // [L]
  float* mlp_s = reinterpret_cast<float*>(hash_s + pad4(L));  // [kWideThreads][OMAX] W phi per grid point
  float* mag_s = mlp_s + kWideThreads * OMAX;                 // [kWideThreads]
  float* wgt_s = mag_s + kWideThreads;                        // [kWideThreads] conf * mag
  uint32_t* key_s = reinterpret_cast<uint32_t*>(wgt_s + kWideThreads);  // [kWideThreads] pixel or ~0
  uint32_t* rtile_s = key_s + kWideThreads;                   // [kWideThreads] tile of a record or ~0
  uint32_t* occ_s = rtile_s + kWideThreads;                   // [kWideWords] conf > 0 bits
  int* misc_s = reinterpret_cast<int*>(occ_s + kWideWords);   // [4] claimed primitive
  const int t = threadIdx.x, lane = t & 31, w = t >> 5;
  for (int i = t; i < L; i += blockDim.x) {
    res_s[i] = sc.res[i];
    resf_s[i] = (float)sc.res[i];
    hash_s[i] = sc.do_hash[i];
  }
  for (int i = t; i < OMAX * DP; i += blockDim.x) {
    const int o = i / DP, d = i % DP;
    W_s[i] = o < O && d < D ? sc.Wl[o * D + d] : 0.0f;
  }
  for (int i = t; i < OMAX; i += blockDim.x) b_s[i] = i < O ? sc.bl[i] : 0.0f;
  const Stencil st = make_stencil(sc.genus);
  const bool act = t < V;
  const GridPt gp = grid_point(act ? t : 0, G, sc.gof);
  const uint32_t p0 = (uint32_t)__ldg(sc.primes), p1 = (uint32_t)__ldg(sc.primes + 1),
                 p2 = (uint32_t)__ldg(sc.primes + 2);
  for (;;) {
    __syncthreads();  // the previous primitive's shared reads are done
    if (t == 0) misc_s[0] = (int)atomicAdd(g.status + 4, 1u);
    __syncthreads();
    const int q = misc_s[0];
    if (q >= sc.P) break;
    const int r = g.radii[q];
    if (r <= 0) {
      if (t == 0) {
        g.rec_cnt[q] = 0;
        g.cls_base[q] = kNoCache;
      }
      continue;
    }
    const float3 c = make_float3(sc.means[3 * q], sc.means[3 * q + 1], sc.means[3 * q + 2]);
    const float2 m2 = make_float2(g.means2D[2 * q], g.means2D[2 * q + 1]);
    const float rf = (float)r;
    const unsigned x0 = min(sc.gx, (unsigned)max(0, (int)fmul(fsub(m2.x, rf), 0.0625f)));
    const unsigned y0 = min(sc.gy, (unsigned)max(0, (int)fmul(fsub(m2.y, rf), 0.0625f)));
    const unsigned x1 = min(sc.gx, (unsigned)max(0, (int)fmul(fsub(fadd(fadd(m2.x, rf), 16.0f), 1.0f), 0.0625f)));
    const unsigned y1 = min(sc.gy, (unsigned)max(0, (int)fmul(fsub(fadd(fadd(m2.y, rf), 16.0f), 1.0f), 0.0625f)));
    const float conf = act ? sc.conf[(size_t)q * V + t] : 0.0f;
    const float3 pos = grid_pos_rel(c, gp.rel, sc.step);
    const float2 sf = project(pos, sc.proj, sc.W, sc.H, true);
    const float2 sb = project(pos, sc.proj, sc.W, sc.H, false);
    const int fx = pix_coord(sf.x), fy = pix_coord(sf.y);
    const uint32_t occw = __ballot_sync(0xffffffffu, act && conf > 0.0f);
    if (lane == 0) occ_s[w] = occw;
    const bool differs =
        __syncthreads_or(act && (fx != pix_coord(sb.x) || fy != pix_coord(sb.y))) != 0;  // also publishes occ_s
    const float mag = act ? occ_mag_w(occ_s, gp, G, st) : 0.0f;
    const bool inside = fx >= 0 && fx < sc.W && fy >= 0 && fy < sc.H;
    const unsigned tx = (unsigned)fx >> 4, ty = (unsigned)fy >> 4;
    const bool vpt = act && conf > 0.0f && inside && tx >= x0 && tx < x1 && ty >= y0 && ty < y1;
    const bool need = vpt && mag > 1e-7f;
    if (need) {
      // hashgrid features of this grid point (hashgrid.h:244-287), then W phi
      const float3 n = hash_norm(pos, sc.hlo, sc.hext);
      float phi[64];
#pragma unroll 1
      for (int l = 0; l < L; l++) {
        float acc[F];
#pragma unroll
        for (int f = 0; f < F; f++) acc[f] = 0.0f;
        const LevelCorners lc = level_corners(n, res_s[l], resf_s[l], hash_s[l] != 0, p0, p1, p2, sc.T);
        gather_level<F, POW2>(lc, sc.table + (size_t)l * sc.tab_l, sc.tab_e, sc.T, sc.Tmask, acc);
#pragma unroll
        for (int f = 0; f < F; f++) phi[l * F + f] = acc[f];
      }
      for (int o = 0; o < OMAX; o++) {
        float a = 0.0f;
        for (int i = 0; i < D; i++) a = __fmaf_rn(W_s[o * DP + i], phi[i], a);
        mlp_s[t * OMAX + o] = a;
      }
    }
    mag_s[t] = mag;
    wgt_s[t] = need ? fmul(conf, mag) : 0.0f;
    key_s[t] = vpt ? (uint32_t)fy * (uint32_t)sc.W + (uint32_t)fx : 0xffffffffu;
    __syncthreads();
    // The lowest grid point of each pixel sums that pixel's grid points in
    // grid-point order (forward.cu:481-627) and decides whether it is a record.
    bool is_rec = false;
    float props[OMAX];
    const uint32_t key = key_s[t];
    if (vpt) {
      bool lowest = true;
      for (int u = 0; u < t && lowest; u++) lowest = key_s[u] != key;
      if (lowest) {
        float ogs = 0.0f, acc[OMAX];
#pragma unroll
        for (int o = 0; o < OMAX; o++) acc[o] = 0.0f;
        for (int u = t; u < V; u++) {
          if (key_s[u] != key) continue;
          const float mg = mag_s[u];
          ogs = fadd(ogs, mg);
          if (mg > 1e-7f) {
            const float wg = wgt_s[u];
#pragma unroll
            for (int o = 0; o < OMAX; o++) acc[o] = fadd(acc[o], fmul(mlp_s[u * OMAX + o], wg));
          }
        }
        if (!(ogs < 1e-7f)) {
          is_rec = true;
#pragma unroll
          for (int o = 0; o < OMAX; o++) {
            const float pre = fadd(acc[o], b_s[o]);
            props[o] = o < O - 1 ? sigmoidf_(pre) : (o == O - 1 ? expf(pre) : 0.0f);
          }
        }
      }
    }
    const uint32_t tkey = ty * sc.gx + tx;
    rtile_s[t] = is_rec ? tkey : 0xffffffffu;
    const int nrec = __syncthreads_count(is_rec);
    if (is_rec) {
      // grouped by tile, ascending; grid-point order inside a tile
      uint32_t rank = 0;
      for (int u = 0; u < V; u++) {
        const uint32_t tu = rtile_s[u];
        rank += (tu < tkey || (tu == tkey && u < t)) ? 1u : 0u;
      }
      const size_t slot = (size_t)q * V + rank;
      g.rec_key[slot] = (tkey << 8) | (((unsigned)fy & 15u) << 4) | ((unsigned)fx & 15u);
      float4* dst = reinterpret_cast<float4*>(g.rec_props + slot * OMAX);
#pragma unroll
      for (int o4 = 0; o4 < OMAX / 4; o4++)
        dst[o4] = make_float4(props[4 * o4], props[4 * o4 + 1], props[4 * o4 + 2], props[4 * o4 + 3]);
    }
    if (t == 0) {
      g.rec_cnt[q] = (uint32_t)nrec | (differs ? kBwdDiffers : 0u);
      g.cls_base[q] = kNoCache;
      if (differs && nrec) g.differs_list[atomicAdd(g.status + 7, 1u)] = (uint32_t)q;
    }
  }
}

template <int F, int OMAX, bool POW2>
void launch_features_wide(const Scene& sc, GeomState& g, cudaStream_t s) {
  const int D = sc.L * F;
  const size_t smem = sizeof(float) * (OMAX * feat_dp(D) + OMAX + 3 * pad4(sc.L) + kWideThreads * OMAX +
                                       4 * kWideThreads + kWideWords + 4);
  auto k = features_wide_kernel<F, OMAX, POW2>;
  cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  int blocks = resident_blocks(reinterpret_cast<const void*>(k), kWideThreads, smem);
  blocks = blocks < sc.P ? blocks : sc.P;
  if (blocks < 1) blocks = 1;
  k<<<blocks, kWideThreads, smem, s>>>(sc, g);
  note_launches(1);
}

template <int F, int OMAX, bool POW2>
void launch_features_p(const Scene& sc, GeomState& g, cudaStream_t s) {
  if (sc.V > 32) {
    launch_features_wide<F, OMAX, POW2>(sc, g, s);
    return;
  }
  const int D = sc.L * F;
  size_t smem = sizeof(float) * (feat_head_floats(D, sc.L, OMAX) + kFeatWarps * feat_warp_floats(D, OMAX));
  auto k = features_kernel<F, OMAX, POW2>;
  cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  // A resident grid: warps claim chunks until the counter runs out.
  int blocks = ((sc.P + 31) / 32 + kFeatWarps - 1) / kFeatWarps;
  const int resident = resident_blocks(reinterpret_cast<const void*>(k), kFeatWarps * 32, smem);
  blocks = blocks < resident ? blocks : resident;
  if (blocks < 1) blocks = 1;
  // the table stays in L2 while primitives gather from it
  cudaLaunchAttribute attr[1];
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(blocks);
  cfg.blockDim = dim3(kFeatWarps * 32);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cfg.attrs = attr;
  cfg.numAttrs = l2_persist_attr(sc.table, (size_t)sc.T * sc.L * F * sizeof(float), attr);
  cudaLaunchKernelEx(&cfg, k, sc, g);
  note_launches(1);
}

template <int F, int OMAX>
void launch_features_t(const Scene& sc, GeomState& g, cudaStream_t s) {
  if (sc.Tmask)
    launch_features_p<F, OMAX, true>(sc, g, s);
  else
    launch_features_p<F, OMAX, false>(sc, g, s);
}

}  // namespace

void launch_features(const Scene& sc, GeomState& g, cudaStream_t s) {
  if (sc.P == 0) return;
  const bool o16 = sc.O > 8;
  switch (sc.F) {
    case 1: o16 ? launch_features_t<1, 16>(sc, g, s) : launch_features_t<1, 8>(sc, g, s); break;
    case 2: o16 ? launch_features_t<2, 16>(sc, g, s) : launch_features_t<2, 8>(sc, g, s); break;
    case 4: o16 ? launch_features_t<4, 16>(sc, g, s) : launch_features_t<4, 8>(sc, g, s); break;
    case 8: o16 ? launch_features_t<8, 16>(sc, g, s) : launch_features_t<8, 8>(sc, g, s); break;
    default: break;  // rejected by the API before launch
  }
}

}  // namespace vi
