// Per-primitive preprocess and tile binning for sm_100a.
//
//   preprocess        reference cuda_integrator/forward.cu:27-110
//   offsets scan      reference cuda_integrator/integrator_impl.cu:306
//   duplicate         reference cuda_integrator/integrator_impl.cu:106-147
//   tile ranges       reference cuda_integrator/integrator_impl.cu:152-178
//   mark_visible      reference cuda_integrator/integrator_impl.cu:66-78
//
// Binning order.  The reference sorts (tile << 32 | depth bits) with a stable
// radix sort, whose ties keep primitive-index order.  Here the visible
// primitives are first sorted by depth bits (stable, so ties keep index order),
// the overlaps are emitted in that depth order, and a stable sort by tile id
// follows.  Both produce the order (tile, depth bits, primitive index): the
// same point list with far fewer passes over the R overlaps.
#include <cuda_runtime.h>

#include <cstdint>

#include "vi_common.cuh"
#include "vi_internal.h"

namespace vi {
namespace {

__global__ void __launch_bounds__(256) preprocess_kernel(Scene sc, GeomState g) {
  int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= sc.P) return;
  g.radii[i] = 0;
  g.tiles_touched[i] = 0;
  g.dkeys[i] = 0xffffffffu;
  g.didx[i] = (uint32_t)i;
  float3 p = make_float3(sc.means[3 * i], sc.means[3 * i + 1], sc.means[3 * i + 2]);
  float3 pv = t43(p, sc.view);
  if (pv.z <= 0.2f) return;  // in_frustum (auxiliary.h:165)
  float3 h = t44_xyw(p, sc.proj);
  float pw = __fdiv_rn(1.0f, fadd(h.z, 0.0000001f));
  float px = fmul(h.x, pw), py = fmul(h.y, pw);
  float world_radius = fmul(sc.scale, 0.86602540378f);
  float view_depth = (float)__dadd_rn((double)fabsf(pv.z), 1e-6);
  float srx = __fdiv_rn(fmul(world_radius, sc.focal_x), view_depth);
  float sry = __fdiv_rn(fmul(world_radius, sc.focal_y), view_depth);
  int r = (int)ceilf(fmaxf(srx, sry));
  float2 img = make_float2(ndc2pix(px, sc.W), ndc2pix(py, sc.H));
  uint2 mn, mx;
  get_rect(img, r, sc.gx, sc.gy, mn, mx);
  if ((mx.x - mn.x) * (mx.y - mn.y) == 0) return;
  if (r <= 0) return;  // see the oracle's header: a zero radius is culled
  g.depths[i] = pv.z;
  g.radii[i] = r;
  g.means2D[2 * i] = img.x;
  g.means2D[2 * i + 1] = img.y;
  g.tiles_touched[i] = (mx.y - mn.y) * (mx.x - mn.x);
  g.dkeys[i] = __float_as_uint(pv.z);
}

// ---- exclusive scan of tiles_touched in depth order (three small kernels) ----
__device__ __forceinline__ uint32_t block_excl_scan(uint32_t v, uint32_t* wsum, uint32_t& total) {
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5, nw = blockDim.x >> 5;
  uint32_t x = v;
#pragma unroll
  for (int off = 1; off < 32; off <<= 1) {
    uint32_t y = __shfl_up_sync(0xffffffffu, x, off);
    if (lane >= off) x += y;
  }
  if (lane == 31) wsum[w] = x;
  __syncthreads();
  if (w == 0) {
    uint32_t s = lane < nw ? wsum[lane] : 0;
#pragma unroll
    for (int off = 1; off < 32; off <<= 1) {
      uint32_t y = __shfl_up_sync(0xffffffffu, s, off);
      if (lane >= off) s += y;
    }
    if (lane < nw) wsum[lane] = s;
  }
  __syncthreads();
  total = wsum[nw - 1];
  uint32_t r = x - v + (w > 0 ? wsum[w - 1] : 0);
  __syncthreads();
  return r;
}

// kScanBlock items per block, 256 threads x 8 items.
__global__ void __launch_bounds__(256) scan_reduce_kernel(int P, const uint32_t* __restrict__ idx,
                                                          const uint32_t* __restrict__ tt, uint32_t* block_sums) {
  __shared__ uint32_t wsum[8];
  uint32_t s = 0;
  int base = blockIdx.x * kScanBlock + threadIdx.x * 8;
#pragma unroll
  for (int k = 0; k < 8; k++) {
    int r = base + k;
    if (r < P) s += tt[idx[r]];
  }
  uint32_t total;
  block_excl_scan(s, wsum, total);
  if (threadIdx.x == 0) block_sums[blockIdx.x] = total;
}

// One block: exclusive scan of the block sums; writes the grand total (u64) to status[2..3].
__global__ void __launch_bounds__(1024) scan_blocks_kernel(int nblocks, uint32_t* block_sums, uint32_t* status) {
  __shared__ uint32_t wsum[32];
  __shared__ unsigned long long carry;
  if (threadIdx.x == 0) carry = 0;
  __syncthreads();
  for (int base = 0; base < nblocks; base += 1024) {
    int i = base + threadIdx.x;
    uint32_t v = i < nblocks ? block_sums[i] : 0;
    uint32_t total;
    uint32_t e = block_excl_scan(v, wsum, total);
    unsigned long long c = carry;
    if (i < nblocks) block_sums[i] = (uint32_t)(c + e);
    __syncthreads();
    if (threadIdx.x == 0) carry = c + total;
    __syncthreads();
  }
  if (threadIdx.x == 0) *(unsigned long long*)(status + 2) = carry;
}

__global__ void __launch_bounds__(256) scan_down_kernel(int P, const uint32_t* __restrict__ idx,
                                                        const uint32_t* __restrict__ tt,
                                                        const uint32_t* __restrict__ block_sums,
                                                        uint32_t* __restrict__ offsets) {
  __shared__ uint32_t wsum[8];
  uint32_t v[8], s = 0;
  int base = blockIdx.x * kScanBlock + threadIdx.x * 8;
#pragma unroll
  for (int k = 0; k < 8; k++) {
    int r = base + k;
    v[k] = r < P ? tt[idx[r]] : 0;
    s += v[k];
  }
  uint32_t total;
  uint32_t e = block_excl_scan(s, wsum, total) + block_sums[blockIdx.x];
#pragma unroll
  for (int k = 0; k < 8; k++) {
    int r = base + k;
    if (r < P) offsets[r] = e;
    e += v[k];
  }
}

// Emits (tile id, primitive) for every tile of a primitive's rectangle, row-major,
// primitives taken in depth order (integrator_impl.cu:134-145 emission order).
__global__ void __launch_bounds__(256) duplicate_kernel(Scene sc, const int* __restrict__ radii,
                                                        const float* __restrict__ means2D,
                                                        const uint32_t* __restrict__ tt,
                                                        const uint32_t* __restrict__ sorted_idx,
                                                        const uint32_t* __restrict__ offsets, uint32_t* __restrict__ keys,
                                                        uint32_t* __restrict__ vals) {
  int r = blockIdx.x * blockDim.x + threadIdx.x;
  if (r >= sc.P) return;
  uint32_t q = sorted_idx[r];
  if (tt[q] == 0) return;
  uint32_t off = offsets[r];
  uint2 mn, mx;
  get_rect(make_float2(means2D[2 * q], means2D[2 * q + 1]), radii[q], sc.gx, sc.gy, mn, mx);
  for (unsigned y = mn.y; y < mx.y; y++)
    for (unsigned x = mn.x; x < mx.x; x++) {
      keys[off] = y * sc.gx + x;
      vals[off] = q;
      off++;
    }
}

__global__ void __launch_bounds__(256) ranges_kernel(uint64_t R, const uint32_t* __restrict__ tiles,
                                                     uint32_t* __restrict__ ranges) {
  uint64_t i = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x;
  if (i >= R) return;
  uint32_t cur = tiles[i];
  if (i == 0) ranges[2 * cur] = 0;
  else {
    uint32_t prev = tiles[i - 1];
    if (cur != prev) {
      ranges[2 * prev + 1] = (uint32_t)i;
      ranges[2 * cur] = (uint32_t)i;
    }
  }
  if (i == R - 1) ranges[2 * cur + 1] = (uint32_t)R;
}

// Copies status words 0..3 (the status bits and the overlap count) into mapped
// pinned host memory.  A kernel rather than a device-to-host copy, so that the
// host's read of the count does not queue behind large device-to-host copies a
// caller runs on other streams in the same copy engine.
__global__ void publish_status_kernel(const uint32_t* __restrict__ status, volatile uint32_t* host_dst) {
  if (threadIdx.x < 4) host_dst[threadIdx.x] = status[threadIdx.x];
  __threadfence_system();
}

__global__ void __launch_bounds__(256) mark_visible_kernel(int P, const float* __restrict__ means,
                                                           const float* __restrict__ view, bool* __restrict__ present) {
  int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= P) return;
  float3 p = make_float3(means[3 * i], means[3 * i + 1], means[3 * i + 2]);
  present[i] = !(t43(p, view).z <= 0.2f);
}

}  // namespace

void launch_preprocess(const Scene& sc, GeomState& g, cudaStream_t s) {
  if (sc.P == 0) return;
  preprocess_kernel<<<(sc.P + 255) / 256, 256, 0, s>>>(sc, g);
  note_launches(1);
}

void launch_offsets_scan(const Scene& sc, GeomState& g, const uint32_t* sorted_idx, cudaStream_t s) {
  int nb = (sc.P + kScanBlock - 1) / kScanBlock;
  scan_reduce_kernel<<<nb, 256, 0, s>>>(sc.P, sorted_idx, g.tiles_touched, g.block_sums);
  scan_blocks_kernel<<<1, 1024, 0, s>>>(nb, g.block_sums, g.status);
  scan_down_kernel<<<nb, 256, 0, s>>>(sc.P, sorted_idx, g.tiles_touched, g.block_sums, g.offsets);
  note_launches(3);
}

void launch_duplicate(const Scene& sc, const GeomState& g, const uint32_t* sorted_idx, BinState& b, cudaStream_t s) {
  duplicate_kernel<<<(sc.P + 255) / 256, 256, 0, s>>>(sc, g.radii, g.means2D, g.tiles_touched, sorted_idx, g.offsets,
                                                      b.tkeys, b.tvals);
  note_launches(1);
}

void launch_ranges(uint64_t R, const uint32_t* sorted_tiles, uint32_t* ranges, size_t tiles, cudaStream_t s) {
  cudaMemsetAsync(ranges, 0, tiles * 2 * sizeof(uint32_t), s);
  if (R == 0) return;
  ranges_kernel<<<(unsigned)((R + 255) / 256), 256, 0, s>>>(R, sorted_tiles, ranges);
  note_launches(1);
}

void launch_publish_status(const uint32_t* status, uint32_t* host_mapped, cudaStream_t s) {
  publish_status_kernel<<<1, 32, 0, s>>>(status, host_mapped);
  note_launches(1);
}

void launch_mark_visible(int P, const float* means, const float* view, bool* present, cudaStream_t s) {
  if (P == 0) return;
  mark_visible_kernel<<<(P + 255) / 256, 256, 0, s>>>(P, means, view, present);
  note_launches(1);
}


}  // namespace vi
