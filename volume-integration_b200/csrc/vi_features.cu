// Feature stage: stage 1 of the reference render kernel (forward.cu:401-463),
// run once per visible primitive instead of once per (tile, primitive), fused
// with the per-pixel accumulation of stage 2 (forward.cu:481-643), which for a
// given (primitive, pixel) depends only on the primitive.
//
// One warp per primitive, lane g = grid point g (V = G^3 <= 32).  Per lane:
// confidence, forward and backward screen positions, the conf>0 stencil
// magnitude, hashgrid features (L levels x 8 corners) and the linear layer.
// Lanes that land in the same pixel are then summed in grid-point order by the
// lowest such lane, exactly the order of the reference's loop, and every pixel
// whose occupancy sum passes the reference's 1e-7 test becomes one record:
//   key   = tile * 256 + pixel-in-tile (only tiles inside the primitive's rect)
//   props = sigmoid(acc + b) for colour and features, exp(acc + b) for density.
// Records of a primitive are stored sorted by key in slots [q*V, q*V + count).
#include <cuda_runtime.h>

#include <cstdint>

#include "vi_kernels.cuh"

namespace vi {
namespace {

constexpr int kFeatWarps = 8;

template <int F, int OMAX>
__global__ void __launch_bounds__(kFeatWarps * 32, 4) features_kernel(Scene sc, GeomState g) {
  extern __shared__ float smem[];
  const int D = sc.L * F, O = sc.O, V = sc.V, G = sc.G;
  float* W_s = smem;                       // [D][OMAX] (transposed for broadcast reads)
  float* b_s = W_s + D * OMAX;             // [OMAX]
  float* resf_s = b_s + OMAX;              // [L] level resolutions as float
  const int w = threadIdx.x >> 5, lane = threadIdx.x & 31;
  float* c_s = resf_s + sc.L + w * (32 * OMAX + 32);  // [32][OMAX]
  float* mag_s = c_s + 32 * OMAX;                      // [32]
  for (int i = threadIdx.x; i < sc.L; i += blockDim.x) resf_s[i] = (float)sc.res[i];

  for (int i = threadIdx.x; i < D * OMAX; i += blockDim.x) {
    int d = i / OMAX, o = i % OMAX;
    W_s[i] = o < O ? sc.Wl[o * D + d] : 0.0f;
  }
  for (int i = threadIdx.x; i < OMAX; i += blockDim.x) b_s[i] = i < O ? sc.bl[i] : 0.0f;
  __syncthreads();

  const Stencil st = make_stencil(sc.genus);
  const GridPt gp = grid_point(lane < V ? lane : 0, G, sc.gof);
  const uint32_t lt_mask = (1u << lane) - 1;
  const int OP = OMAX;
  const int nwarps = gridDim.x * kFeatWarps;
  for (int q = blockIdx.x * kFeatWarps + w; q < sc.P; q += nwarps) {
    const int r = g.radii[q];
    if (r <= 0) {
      if (lane == 0) g.rec_cnt[q] = 0;
      continue;
    }
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

    float cvec[OMAX];
#pragma unroll
    for (int o = 0; o < OMAX; o++) cvec[o] = 0.0f;
    if (__any_sync(0xffffffffu, need)) {
      // Linear layer accumulated level by level: mlp[o] = sum_i W[o][i] phi[i], i ascending.
      float2 mlp[OMAX / 2];  // output pairs, two fused multiply-adds per instruction
#pragma unroll
      for (int o = 0; o < OMAX / 2; o++) mlp[o] = make_float2(0.0f, 0.0f);
      for_each_level<F>(sc, resf_s, pos, need, [&](int l, const float* phi) {
        if (!need) return;
#pragma unroll
        for (int f = 0; f < F; f++) {
          const float2 x = make_float2(phi[f], phi[f]);
          const float4* wr = reinterpret_cast<const float4*>(W_s + (l * F + f) * OMAX);
#pragma unroll
          for (int o4 = 0; o4 < OMAX / 4; o4++) {
            const float4 ww = wr[o4];
            mlp[2 * o4] = __ffma2_rn(make_float2(ww.x, ww.y), x, mlp[2 * o4]);
            mlp[2 * o4 + 1] = __ffma2_rn(make_float2(ww.z, ww.w), x, mlp[2 * o4 + 1]);
          }
        }
      });
      if (need) {
        const float wgt = fmul(conf, mag);
#pragma unroll
        for (int o = 0; o < OMAX / 2; o++) {
          cvec[2 * o] = fmul(mlp[o].x, wgt);
          cvec[2 * o + 1] = fmul(mlp[o].y, wgt);
        }
      }
    }
#pragma unroll
    for (int o = 0; o < OMAX; o++) c_s[lane * OMAX + o] = cvec[o];
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
        if (mg > 1e-7f) {
#pragma unroll
          for (int o = 0; o < OMAX; o++) acc[o] = fadd(acc[o], c_s[src * OMAX + o]);
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
    const uint32_t recmask = __ballot_sync(0xffffffffu, is_rec);
    const uint32_t rkey = ((ty * sc.gx + tx) << 8) | (((unsigned)fy & 15u) << 4) | ((unsigned)fx & 15u);
    uint32_t rank = 0;
#pragma unroll 4
    for (int l = 0; l < 32; l++) {
      const uint32_t k = __shfl_sync(0xffffffffu, rkey, l);
      if (((recmask >> l) & 1u) && k < rkey) rank++;
    }
    if (is_rec) {
      const size_t slot = (size_t)q * V + rank;
      g.rec_key[slot] = rkey;
      float4* dst = reinterpret_cast<float4*>(g.rec_props + slot * OP);
#pragma unroll
      for (int o4 = 0; o4 < OMAX / 4; o4++)
        dst[o4] = make_float4(props[4 * o4], props[4 * o4 + 1], props[4 * o4 + 2], props[4 * o4 + 3]);
    }
    if (lane == 0) g.rec_cnt[q] = (uint32_t)__popc(recmask) | (differs ? kBwdDiffers : 0u);
    __syncwarp();
  }
}

template <int F, int OMAX>
void launch_features_t(const Scene& sc, GeomState& g, cudaStream_t s) {
  const int D = sc.L * F;
  size_t smem = sizeof(float) * (D * OMAX + OMAX + sc.L + kFeatWarps * (32 * OMAX + 32));
  auto k = features_kernel<F, OMAX>;
  cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  int blocks = (sc.P + kFeatWarps - 1) / kFeatWarps;
  blocks = blocks < 148 * 8 ? blocks : 148 * 8;
  if (blocks < 1) blocks = 1;
  k<<<blocks, kFeatWarps * 32, smem, s>>>(sc, g);
  note_launches(1);
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
