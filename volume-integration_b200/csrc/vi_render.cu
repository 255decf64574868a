// Per-tile compositing: the per-pixel part of the reference render kernel
// (forward.cu:467-785) over the records written by the feature stage.
//
// One CTA per 16x16 tile, one thread per pixel.  The tile's sorted list is
// walked in batches of 64 entries.  For each batch the CTA locates every
// entry's records inside this tile (they are contiguous: records are sorted by
// tile) and marks, per pixel, a 64-bit mask of the entries that have a record
// for it.  Each pixel then visits its set bits in list order and runs the
// reference's pending-primitive compositing, so a pixel touches only the
// primitives that actually cover it.  A __syncthreads_count at the top of each
// batch ends the tile once every pixel is done (forward.cu:369-372).
#include <cuda_runtime.h>

#include <cstdint>
#include <cstdlib>

#include "vi_kernels.cuh"

namespace vi {
namespace {

constexpr int kBatch = 64;
// Entries whose record keys a warp loads at once during a batch's set-up: all
// of its kBatch / 8 entries (loading them in two or four rounds, with fewer
// registers, measured slower).
constexpr int kKeyGroup = kBatch / (VI_TILE_PIX / 32);

// Rows of the shared staging buffer of STAGE (record properties of one batch).
template <int OMAX>
__host__ __device__ constexpr int stage_rows() { return OMAX == 8 ? 384 : 160; }
// Polls of a batch's staging mbarrier before the tile gives up on staging.
constexpr int kStageWaitLimit = 1 << 20;

// WIDE: primitives of more than 32 grid points (G = 4, 5), whose records a
// warp reads 32 slots at a time.
// STAGE: each batch's in-tile record properties are brought into shared memory
// by plain bulk copies (cp.async.bulk, one per entry: its records in this tile
// are contiguous and 32- or 64-byte rows), completed on an mbarrier, so the
// pixels' compositing reads shared memory instead of dependent global loads.
// A pixel's pending record can outlive its batch's buffer, so its properties
// move into a per-thread shared row when it becomes pending.  A batch whose
// records exceed the buffer reads global memory, and a wait that gives up
// after kStageWaitLimit polls latches VI_ERR_STAGE_TIMEOUT and ends staging
// for the tile.
template <int OMAX, bool WIDE, bool STAGE>
__global__ void __launch_bounds__(VI_TILE_PIX, 4) render_kernel(Scene sc, const uint32_t* __restrict__ point_list,
                                                            const uint32_t* __restrict__ ranges,
                                                            const float* __restrict__ depths,
                                                            const uint32_t* __restrict__ rec_cnt,
                                                            const uint32_t* __restrict__ rec_key,
                                                            const float* __restrict__ rec_props,
                                                            float* __restrict__ out_color, float* __restrict__ out_feat,
                                                            float* __restrict__ vis, float* __restrict__ final_T,
                                                            int32_t* __restrict__ n_contrib,
                                                            int32_t* __restrict__ contrib_idx,
                                                            float* __restrict__ delta_t,
                                                            uint32_t* __restrict__ contrib_rec,
                                                            float* __restrict__ trans, uint32_t* __restrict__ trig,
                                                            uint32_t* __restrict__ status, int stage_wait_limit,
                                                            bool stage_withhold) {
  __shared__ unsigned long long mask[VI_TILE_PIX];
  __shared__ uint8_t slot[VI_TILE_PIX * kBatch];
  __shared__ uint32_t ent_rec[kBatch];
  __shared__ uint32_t ent_flag[kBatch];  // kBwdDiffers of the entry's primitive
  __shared__ float ent_depth[kBatch];
  constexpr int kRows = STAGE ? stage_rows<OMAX>() : 1;
  __shared__ uint32_t ent_cnt[STAGE ? kBatch : 1];  // records of the entry in this tile
  __shared__ uint32_t ent_off[STAGE ? kBatch : 1];  // their first row in stage
  __shared__ alignas(128) float stage[kRows * OMAX];
  __shared__ alignas(16) float pend_s[STAGE ? VI_TILE_PIX * OMAX : 4];
  __shared__ alignas(8) uint64_t mbar;
  __shared__ int stage_use;  // this batch reads stage
  __shared__ int stage_live;  // staging still enabled for this tile

  const int tid = threadIdx.x;
  const unsigned tile = blockIdx.x;
  const unsigned bx = tile % sc.gx, by = tile / sc.gx;
  const unsigned px = bx * VI_TILE + (tid & 15), py = by * VI_TILE + (tid >> 4);
  const bool inside = px < (unsigned)sc.W && py < (unsigned)sc.H;
  const size_t pix = (size_t)py * sc.W + px;
  const int O = sc.O, K = sc.K, Fout = sc.Fout, V = sc.V;

  float T = 1.0f, C0 = 0.0f, C1 = 0.0f, C2 = 0.0f;
  float Fe[OMAX - 4];
#pragma unroll
  for (int f = 0; f < OMAX - 4; f++) Fe[f] = 0.0f;
  int cnt = 0;
  bool done = !inside, has_p = false;
  uint32_t pend_rec = 0, pend_gidx = 0, pend_flag = 0;
  float pend_depth = sc.near_plane, T_pend = 0.0f;

  const uint32_t r0 = ranges[2 * tile], r1 = ranges[2 * tile + 1];
  const uint32_t klo = tile << 8;
  uint32_t phase = 0;
  if constexpr (STAGE) {
    if (tid == 0) {
      mbar_init(&mbar, 1);
      stage_live = 1;
    }
    __syncthreads();
  }

  // trigger: list index of the entry whose arrival composites the pending one,
  // ~0 for the final composite against max_distance (kept for the exact backward)
  auto composite = [&](float dt, uint32_t trigger) {
    const float* pp = STAGE ? pend_s + tid * OMAX : rec_props + (size_t)pend_rec * OMAX;
    float alpha = 1.0f - expf(-pp[O - 1] * dt);
    alpha = fminf(fmaxf(alpha, 0.0f), 1.0f);
    const float wgt = T_pend * alpha;
    C0 += wgt * pp[0];
    C1 += wgt * pp[1];
    C2 += wgt * pp[2];
#pragma unroll
    for (int f = 0; f < OMAX - 4; f++)
      if (f < Fout) Fe[f] += wgt * pp[3 + f];
    T = T_pend * (1.0f - alpha);
    const size_t w = pix * K + cnt;
    contrib_idx[w] = (int32_t)pend_gidx;
    delta_t[w] = dt;
    contrib_rec[w] = pend_rec | pend_flag;  // the backward's recompute flag rides in bit 31
    if (trans) {
      trans[w] = T_pend;
      trig[w] = trigger;
    }
    cnt++;
  };

  for (uint32_t base = r0; base < r1; base += kBatch) {
    if (__syncthreads_count(!done) == 0) break;
    const int nb = (int)min((uint32_t)kBatch, r1 - base);
    mask[tid] = 0ull;
    __syncthreads();
    // Warp w takes entries w, w+8, ...: lane i fetches entry w+8i's primitive,
    // record count and depth; then every lane loads one record key of each of
    // those primitives at once (lane = record slot, V <= 27), and one ballot per
    // entry finds the records in this tile (contiguous: records are grouped by
    // tile).  Two rounds of loads per batch, where a search per entry chains
    // several.  Grids of more than 32 points take one entry at a time.
    {
      const int w = tid >> 5, lane = tid & 31;
      constexpr int kPer = kBatch / (VI_TILE_PIX / 32);  // entries per warp
      const int el = w + (VI_TILE_PIX / 32) * lane;
      uint32_t q_l = 0u, rc_l = 0u;
      float d_l = 0.0f;
      if (lane < kPer && el < nb) {
        q_l = point_list[base + el];
        rc_l = rec_cnt[q_l];
        d_l = depths[q_l];
      }
      if constexpr (WIDE) {
        // Entry by entry, the primitive's record keys 32 slots at a time; the
        // records of this tile are contiguous from slot lo.
        for (int i = 0; i < kPer; i++) {
          const int e = w + (VI_TILE_PIX / 32) * i;
          if (e >= nb) break;  // warp-uniform
          const uint32_t q = __shfl_sync(0xffffffffu, q_l, i);
          const uint32_t rc = __shfl_sync(0xffffffffu, rc_l, i);
          const float d = __shfl_sync(0xffffffffu, d_l, i);
          const uint32_t n = rc & ~kBwdDiffers;
          int lo = -1;
          for (uint32_t s0 = 0; s0 < n; s0 += 32) {
            const uint32_t sl = s0 + (uint32_t)lane;
            const uint32_t key = sl < n ? rec_key[(size_t)q * V + sl] : 0xffffffffu;
            const uint32_t in = __ballot_sync(0xffffffffu, (key & ~255u) == klo);
            if (!in) continue;
            if (lo < 0) lo = (int)(s0 + (uint32_t)__ffs(in) - 1u);
            if ((in >> lane) & 1u) {
              const uint32_t lp = key & 255u;
              slot[lp * kBatch + e] = (uint8_t)(sl - (uint32_t)lo);
              atomicOr(&mask[lp], 1ull << e);
            }
          }
          if (lane == 0) {
            ent_rec[e] = (uint32_t)((size_t)q * V + (lo < 0 ? 0u : (uint32_t)lo));
            ent_flag[e] = rc & kBwdDiffers;
            ent_depth[e] = d;
          }
          if constexpr (STAGE) {
            if (lane == 0) ent_cnt[e] = 0u;  // wide grids do not stage
          }
        }
      } else {
#pragma unroll
      for (int i0 = 0; i0 < kPer; i0 += kKeyGroup) {
      uint32_t key[kKeyGroup];
#pragma unroll
      for (int j = 0; j < kKeyGroup; j++) {
        const int i = i0 + j, e = w + (VI_TILE_PIX / 32) * i;
        const uint32_t q = __shfl_sync(0xffffffffu, q_l, i);
        const uint32_t n = __shfl_sync(0xffffffffu, rc_l, i) & ~kBwdDiffers;
        key[j] = (e < nb && (uint32_t)lane < n) ? rec_key[(size_t)q * V + lane] : 0xffffffffu;
      }
#pragma unroll
      for (int j = 0; j < kKeyGroup; j++) {
        const int i = i0 + j, e = w + (VI_TILE_PIX / 32) * i;
        if (e >= nb) break;  // warp-uniform
        const uint32_t in = __ballot_sync(0xffffffffu, (key[j] & ~255u) == klo);
        const uint32_t q = __shfl_sync(0xffffffffu, q_l, i);
        const uint32_t rc = __shfl_sync(0xffffffffu, rc_l, i);
        const float d = __shfl_sync(0xffffffffu, d_l, i);
        const uint32_t lo = in ? (uint32_t)__ffs(in) - 1u : 0u;
        if (lane == 0) {
          ent_rec[e] = (uint32_t)((size_t)q * V + lo);
          ent_flag[e] = rc & kBwdDiffers;
          ent_depth[e] = d;
          if constexpr (STAGE) ent_cnt[e] = (uint32_t)__popc(in);
        }
        if ((in >> lane) & 1u) {
          const uint32_t lp = key[j] & 255u;
          slot[lp * kBatch + e] = (uint8_t)(lane - lo);
          atomicOr(&mask[lp], 1ull << e);
        }
      }
      }
      }
    }
    __syncthreads();
    bool use_stage = false;
    if constexpr (STAGE) {
      if (tid < 32) {
        // first staging row of every entry: exclusive scan of the record
        // counts, two entries per lane
        const int e0 = 2 * tid, e1 = 2 * tid + 1;
        const uint32_t c0 = e0 < nb ? ent_cnt[e0] : 0u, c1 = e1 < nb ? ent_cnt[e1] : 0u;
        uint32_t incl = c0 + c1;
#pragma unroll
        for (int off = 1; off < 32; off <<= 1) {
          const uint32_t x = __shfl_up_sync(0xffffffffu, incl, off);
          if (tid >= off) incl += x;
        }
        const uint32_t excl = incl - c0 - c1;
        if (e0 < nb) ent_off[e0] = excl;
        if (e1 < nb) ent_off[e1] = excl + c0;
        const uint32_t total = __shfl_sync(0xffffffffu, incl, 31);
        if (tid == 0) {
          const int use = stage_live && total > 0u && total <= (uint32_t)kRows;
          stage_use = use;
          if (use && !stage_withhold) mbar_arrive_expect_tx(&mbar, total * OMAX * (uint32_t)sizeof(float));
        }
      }
      __syncthreads();
      if (stage_use) {
        if (!stage_withhold && tid < nb && ent_cnt[tid] > 0u) {
          fence_proxy_async_smem();
          bulk_copy_g2s(stage + ent_off[tid] * OMAX, rec_props + (size_t)ent_rec[tid] * OMAX,
                        ent_cnt[tid] * OMAX * (uint32_t)sizeof(float), &mbar);
        }
        use_stage = mbar_wait(&mbar, phase, stage_wait_limit);
        phase ^= 1u;
        if (!use_stage) {
          stage_live = 0;  // read global memory from here on
          atomicOr(status, VI_ERR_STAGE_TIMEOUT);
        }
      }
    }
    if (!done) {
      unsigned long long m = mask[tid];
      while (m) {
        const int e = __ffsll(m) - 1;
        m &= m - 1;
        const uint32_t sl = slot[tid * kBatch + e];
        const uint32_t rec = ent_rec[e] + sl;
        const float depth = ent_depth[e];
        if (has_p) {
          const float dt = fmaxf(0.0f, depth - pend_depth);
          if (dt > 1e-5f && cnt < K) composite(dt, base + e);
        }
        if (T >= 1e-4f && cnt < K) {
          if constexpr (STAGE) {
            const float4* src = use_stage ? reinterpret_cast<const float4*>(stage + (ent_off[e] + sl) * OMAX)
                                          : reinterpret_cast<const float4*>(rec_props + (size_t)rec * OMAX);
            float4* dst = reinterpret_cast<float4*>(pend_s + tid * OMAX);
#pragma unroll
            for (int o4 = 0; o4 < OMAX / 4; o4++) dst[o4] = src[o4];
          }
          pend_rec = rec;
          pend_flag = ent_flag[e];
          pend_depth = depth;
          pend_gidx = base + e;
          has_p = true;
          T_pend = T;
        } else {
          has_p = false;
          done = true;
        }
        if (T < 1e-4f || cnt >= K) done = true;
        if (done) break;
      }
    }
  }
  if constexpr (STAGE) {
    // a wait that gave up may leave its copies in flight: give them a bounded
    // time to land before the block's shared memory is released
    if (tid == 0 && !stage_live) mbar_wait(&mbar, phase ^ 1u, stage_wait_limit);
  }
  if (!inside) return;
  if (has_p && T >= 1e-4f && cnt < K) {
    const float dt = fmaxf(0.0f, sc.max_distance - pend_depth);
    if (dt > 1e-5f) composite(dt, 0xffffffffu);
  }
  const size_t N = (size_t)sc.W * sc.H;
  out_color[pix] = fminf(fmaxf(C0 + T * sc.bg[0], 0.0f), 1.0f);
  out_color[N + pix] = fminf(fmaxf(C1 + T * sc.bg[1], 0.0f), 1.0f);
  out_color[2 * N + pix] = fminf(fmaxf(C2 + T * sc.bg[2], 0.0f), 1.0f);
#pragma unroll
  for (int f = 0; f < OMAX - 4; f++)
    if (f < Fout) out_feat[f * N + pix] = Fe[f];
  vis[pix] = 1.0f - T;
  final_T[pix] = T;
  n_contrib[pix] = cnt;
}

}  // namespace

void launch_render(const Scene& sc, const GeomState& g, const uint32_t* point_list, ImgState& im, float* out_color,
                   float* out_feat, float* vis, cudaStream_t s) {
  const unsigned tiles = sc.gx * sc.gy;
  if (tiles == 0) return;
  note_launches(1);
  // Bulk-copy staging of the records for grids of at most 32 points: opt-in
  // (VI_RENDER_TMA=1).  At equal occupancy (4 blocks per SM) the unstaged form
  // measured faster: 0.480 against 0.489 ms on the headline scene, 21.6
  // against 25.5 ms on the 4K stress scene, where batches often hold more
  // records than the stage buffer.
  // Testing hook for the bounded wait (VI_RENDER_TMA_TEST_TIMEOUT=1, which
  // also turns staging on): the batches' barrier arrival and copies are
  // withheld, so nothing completes the phase every pixel waits on (and nothing
  // is in flight); each tile gives up after 256 polls, latches
  // VI_ERR_STAGE_TIMEOUT and reads global memory, with the same results.
  const char* t = std::getenv("VI_RENDER_TMA_TEST_TIMEOUT");
  const bool test_timeout = t && t[0] == '1';
  const char* e = std::getenv("VI_RENDER_TMA");
  const bool stage = ((e && e[0] == '1') || test_timeout) && sc.V <= 32;
  const int wait_limit = test_timeout ? 256 : kStageWaitLimit;
  auto k = sc.O > 8 ? (sc.V > 32 ? render_kernel<16, true, false>
                                 : (stage ? render_kernel<16, false, true> : render_kernel<16, false, false>))
                    : (sc.V > 32 ? render_kernel<8, true, false>
                                 : (stage ? render_kernel<8, false, true> : render_kernel<8, false, false>));
  k<<<tiles, VI_TILE_PIX, 0, s>>>(sc, point_list, im.ranges, g.depths, g.rec_cnt, g.rec_key, g.rec_props, out_color,
                                  out_feat, vis, im.final_T, im.n_contrib, im.contrib_idx, im.delta_t, im.contrib_rec,
                                  im.trans, im.trig, g.status, wait_limit, test_timeout);
}

}  // namespace vi
