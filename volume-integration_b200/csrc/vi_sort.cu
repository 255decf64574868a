// Stable LSD radix sort of (key, u32 value) pairs for sm_100a, one kernel per
// 8-bit digit pass in the "onesweep" style: every CTA ranks one tile of keys,
// publishes its digit counts, resolves its global digit offsets by decoupled
// look-back over the preceding tiles, and scatters through shared memory.
//
// It replaces cub::DeviceRadixSort::SortPairs in the reference binning step
// (cuda_integrator/integrator_impl.cu:341-349).  Stability gives the same
// permutation as CUB on the same bit range.
//
// Look-back waits are bounded: after a spin limit (kSpinLimit polls in
// production) a CTA latches VI_ERR_LOOKBACK_TIMEOUT in the status word, stops
// waiting and writes only in-bounds positions, so a lost predecessor can never
// hang the GPU.
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdint>

#include "vi_common.cuh"
#include "vi_internal.h"

namespace vi {
namespace {

constexpr uint32_t kFlagAgg = 1u << 30;
constexpr uint32_t kFlagInc = 2u << 30;
constexpr uint32_t kCountMask = (1u << 30) - 1;
constexpr int kSpinLimit = 1 << 20;

template <typename K>
struct SortCfg;
template <>
struct SortCfg<uint32_t> {
  static constexpr int kItems = 16;
};
template <>
struct SortCfg<uint64_t> {
  static constexpr int kItems = 12;
};

__device__ __forceinline__ uint32_t ld_volatile(const uint32_t* p) { return *(const volatile uint32_t*)p; }
__device__ __forceinline__ void st_volatile(uint32_t* p, uint32_t v) { *(volatile uint32_t*)p = v; }

template <typename K>
__device__ __forceinline__ uint32_t digit_of(K k, int shift, uint32_t mask) {
  return (uint32_t)(k >> shift) & mask;
}

__global__ void fill_u32_kernel(uint32_t* p, uint32_t v, int n) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) p[i] = v;
}
void fill_u32_async(uint32_t* p, uint32_t v, int n, cudaStream_t s) {
  fill_u32_kernel<<<1, 32, 0, s>>>(p, v, n);
  note_launches(1);
}

// Digit histograms of every pass in one read of the keys.
template <typename K>
__global__ void __launch_bounds__(256) hist_kernel(const K* __restrict__ keys, uint64_t n, int begin_bit,
                                                   int end_bit, int passes, uint32_t* __restrict__ hist) {
  __shared__ uint32_t sh[8 * kRadix];
  for (int i = threadIdx.x; i < passes * kRadix; i += blockDim.x) sh[i] = 0;
  __syncthreads();
  for (uint64_t i = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; i < n; i += (uint64_t)gridDim.x * blockDim.x) {
    K k = keys[i];
    for (int p = 0; p < passes; p++) {
      int shift = begin_bit + 8 * p;
      int bits = min(8, end_bit - shift);
      atomicAdd(&sh[p * kRadix + digit_of(k, shift, (1u << bits) - 1)], 1u);
    }
  }
  __syncthreads();
  for (int i = threadIdx.x; i < passes * kRadix; i += blockDim.x)
    if (sh[i]) atomicAdd(&hist[i], sh[i]);
}

// Exclusive scan of each pass's 256 digit counts (one block per pass).
__global__ void __launch_bounds__(kRadix) hist_scan_kernel(uint32_t* hist) {
  __shared__ uint32_t sh[kRadix];
  uint32_t* h = hist + blockIdx.x * kRadix;
  int t = threadIdx.x;
  uint32_t v = h[t];
  sh[t] = v;
  __syncthreads();
  for (int off = 1; off < kRadix; off <<= 1) {
    uint32_t x = t >= off ? sh[t - off] : 0;
    __syncthreads();
    sh[t] += x;
    __syncthreads();
  }
  h[t] = sh[t] - v;
}

template <typename K>
struct alignas(16) PassSmem {
  static constexpr int kTile = kSortThreads * SortCfg<K>::kItems;
  K keys[kTile];
  uint32_t vals[kTile];
  uint32_t warp_hist[kSortThreads / 32][kRadix];
  uint32_t block_start[kRadix];
  uint32_t digit_out[kRadix];
  uint32_t tile_id;
};

template <typename K>
__global__ void __launch_bounds__(kSortThreads) onesweep_pass_kernel(
    const K* __restrict__ keys_in, const uint32_t* __restrict__ vals_in, K* __restrict__ keys_out,
    uint32_t* __restrict__ vals_out, uint64_t n, int shift, uint32_t mask, const uint32_t* __restrict__ digit_base,
    uint32_t* __restrict__ lookback, uint32_t* __restrict__ tile_counter, uint32_t* __restrict__ status,
    int spin_limit) {
  constexpr int kItems = SortCfg<K>::kItems;
  constexpr int kTile = kSortThreads * kItems;
  constexpr int kWarps = kSortThreads / 32;
  __shared__ PassSmem<K> sm;
  const int tid = threadIdx.x, w = tid >> 5, lane = tid & 31;

  if (tid == 0) sm.tile_id = atomicAdd(tile_counter, 1u);
  for (int i = tid; i < kWarps * kRadix; i += kSortThreads) (&sm.warp_hist[0][0])[i] = 0;
  __syncthreads();
  const uint32_t tile = sm.tile_id;
  const uint64_t base = (uint64_t)tile * kTile;
  const uint32_t tile_n = (uint32_t)min((uint64_t)kTile, n - base);

  // Warp-striped load: item i of lane l of warp w sits at w*32*kItems + i*32 + l,
  // so (warp, item, lane) order is the input order.
  K key[kItems];
  uint32_t val[kItems];
  uint32_t rank[kItems];
#pragma unroll
  for (int i = 0; i < kItems; i++) {
    uint32_t loc = (uint32_t)w * 32 * kItems + i * 32 + lane;
    bool ok = loc < tile_n;
    key[i] = ok ? keys_in[base + loc] : (K)0;
    val[i] = ok ? vals_in[base + loc] : 0u;
  }
  const uint32_t lt_mask = (1u << lane) - 1;
#pragma unroll
  for (int i = 0; i < kItems; i++) {
    uint32_t loc = (uint32_t)w * 32 * kItems + i * 32 + lane;
    bool ok = loc < tile_n;
    uint32_t d = ok ? digit_of(key[i], shift, mask) : (uint32_t)(kRadix + lane);
    uint32_t peers = __match_any_sync(0xffffffffu, d);
    uint32_t before = __popc(peers & lt_mask);
    uint32_t b = ok ? sm.warp_hist[w][d] : 0u;
    __syncwarp();
    if (ok && before == 0) sm.warp_hist[w][d] = b + __popc(peers);
    __syncwarp();
    rank[i] = b + before;
  }
  __syncthreads();

  // Thread d owns digit d: warp-exclusive prefix and the tile's digit count.
  const uint32_t d = tid;
  uint32_t cnt = 0;
#pragma unroll
  for (int ww = 0; ww < kWarps; ww++) {
    uint32_t c = sm.warp_hist[ww][d];
    sm.warp_hist[ww][d] = cnt;
    cnt += c;
  }
  uint32_t* my = lookback + (uint64_t)tile * kRadix + d;
  __threadfence();
  st_volatile(my, (tile == 0 ? kFlagInc : kFlagAgg) | cnt);

  // Block-exclusive scan over digits (block_start) for the shared-memory reorder.
  {
    uint32_t v = cnt;
#pragma unroll
    for (int off = 1; off < 32; off <<= 1) {
      uint32_t x = __shfl_up_sync(0xffffffffu, v, off);
      if (lane >= off) v += x;
    }
    __shared__ uint32_t wsum[kWarps];
    if (lane == 31) wsum[w] = v;
    __syncthreads();
    uint32_t wo = 0;
    for (int ww = 0; ww < w; ww++) wo += wsum[ww];
    sm.block_start[d] = wo + v - cnt;
  }

  // Decoupled look-back over preceding tiles.
  uint32_t excl = 0;
  if (tile > 0) {
    int64_t pred = (int64_t)tile - 1;
    int spins = 0;
    bool timed_out = false;
    while (pred >= 0) {
      uint32_t v = ld_volatile(lookback + (uint64_t)pred * kRadix + d);
      if ((v & ~kCountMask) == 0) {
        if (++spins > spin_limit) {
          timed_out = true;
          break;
        }
        __nanosleep(32);
        continue;
      }
      excl += v & kCountMask;
      if ((v & ~kCountMask) == kFlagInc) break;
      pred--;
    }
    if (timed_out) atomicOr(status, VI_ERR_LOOKBACK_TIMEOUT);
    __threadfence();
    st_volatile(my, kFlagInc | ((excl + cnt) & kCountMask));
  }
  sm.digit_out[d] = digit_base[d] + excl;
  __syncthreads();

  // Reorder the tile in shared memory by digit (stable), then write runs out.
#pragma unroll
  for (int i = 0; i < kItems; i++) {
    uint32_t loc = (uint32_t)w * 32 * kItems + i * 32 + lane;
    if (loc < tile_n) {
      uint32_t dd = digit_of(key[i], shift, mask);
      uint32_t slot = sm.block_start[dd] + sm.warp_hist[w][dd] + rank[i];
      sm.keys[slot] = key[i];
      sm.vals[slot] = val[i];
    }
  }
  __syncthreads();
  for (uint32_t sidx = tid; sidx < tile_n; sidx += kSortThreads) {
    K k = sm.keys[sidx];
    uint32_t dd = digit_of(k, shift, mask);
    uint64_t out = (uint64_t)sm.digit_out[dd] + (sidx - sm.block_start[dd]);
    if (out < n) {
      keys_out[out] = k;
      vals_out[out] = sm.vals[sidx];
    }
  }
}

// withhold_first_tile (testing only): the tile counters start at 1 and one CTA
// fewer is launched, so tile 0 never publishes and tile 1's look-back runs into
// its spin limit.  Every launched CTA still gets a tile id below t.tiles.
template <typename K>
bool sort_impl(K* keys, uint32_t* vals, K* alt_keys, uint32_t* alt_vals, uint64_t n, int begin_bit, int end_bit,
               const SortTemp& t, uint32_t* status, cudaStream_t s, int spin_limit = kSpinLimit,
               bool withhold_first_tile = false) {
  if (n <= 1 || end_bit <= begin_bit) return false;
  if (withhold_first_tile && t.tiles < 2) return false;
  constexpr int kTile = kSortThreads * SortCfg<K>::kItems;
  const int passes = t.passes;
  cudaMemsetAsync(t.hist, 0, sizeof(uint32_t) * kRadix * passes, s);
  if (withhold_first_tile)
    fill_u32_async(t.counters, 1u, passes, s);
  else
    cudaMemsetAsync(t.counters, 0, sizeof(uint32_t) * passes, s);
  cudaMemsetAsync(t.lookback, 0, sizeof(uint32_t) * kRadix * (size_t)t.tiles * passes, s);
  int hblocks = (int)std::min<uint64_t>((n + 255) / 256, 148 * 8);
  hist_kernel<K><<<hblocks, 256, 0, s>>>(keys, n, begin_bit, end_bit, passes, t.hist);
  note_launches(2 + passes);
  hist_scan_kernel<<<passes, kRadix, 0, s>>>(t.hist);
  K* kin = keys;
  uint32_t* vin = vals;
  K* kout = alt_keys;
  uint32_t* vout = alt_vals;
  for (int p = 0; p < passes; p++) {
    int shift = begin_bit + 8 * p;
    int bits = min(8, end_bit - shift);
    onesweep_pass_kernel<K><<<t.tiles - (withhold_first_tile ? 1u : 0u), kSortThreads, 0, s>>>(
        kin, vin, kout, vout, n, shift, (1u << bits) - 1, t.hist + p * kRadix,
        t.lookback + (size_t)p * t.tiles * kRadix, t.counters + p, status, spin_limit);
    K* tk = kin;
    kin = kout;
    kout = tk;
    uint32_t* tv = vin;
    vin = vout;
    vout = tv;
  }
  (void)kTile;
  return (passes & 1) != 0;
}

}  // namespace

size_t sort_temp_bytes(uint64_t n, int key_bytes, int begin_bit, int end_bit) {
  int passes = end_bit > begin_bit ? (end_bit - begin_bit + 7) / 8 : 0;
  uint64_t tile = (uint64_t)kSortThreads * (key_bytes == 8 ? SortCfg<uint64_t>::kItems : SortCfg<uint32_t>::kItems);
  uint64_t tiles = (n + tile - 1) / tile;
  return align_up(sizeof(uint32_t) * kRadix * passes) + align_up(sizeof(uint32_t) * kRadix * tiles * passes) +
         align_up(sizeof(uint32_t) * (passes > 0 ? passes : 1));
}

void sort_temp_carve(char* base, uint64_t n, int key_bytes, int begin_bit, int end_bit, SortTemp& t) {
  t.passes = end_bit > begin_bit ? (end_bit - begin_bit + 7) / 8 : 0;
  uint64_t tile = (uint64_t)kSortThreads * (key_bytes == 8 ? SortCfg<uint64_t>::kItems : SortCfg<uint32_t>::kItems);
  t.tiles = (uint32_t)((n + tile - 1) / tile);
  t.hist = (uint32_t*)base;
  base += align_up(sizeof(uint32_t) * kRadix * t.passes);
  t.lookback = (uint32_t*)base;
  base += align_up(sizeof(uint32_t) * kRadix * (size_t)t.tiles * t.passes);
  t.counters = (uint32_t*)base;
}

bool onesweep_sort_u32(uint32_t* keys, uint32_t* vals, uint32_t* alt_keys, uint32_t* alt_vals, uint64_t n,
                       int begin_bit, int end_bit, const SortTemp& t, uint32_t* status, cudaStream_t s) {
  return sort_impl<uint32_t>(keys, vals, alt_keys, alt_vals, n, begin_bit, end_bit, t, status, s);
}

bool onesweep_sort_u64(uint64_t* keys, uint32_t* vals, uint64_t* alt_keys, uint32_t* alt_vals, uint64_t n,
                       int begin_bit, int end_bit, const SortTemp& t, uint32_t* status, cudaStream_t s) {
  return sort_impl<uint64_t>(keys, vals, alt_keys, alt_vals, n, begin_bit, end_bit, t, status, s);
}

bool onesweep_sort_u64_withheld(uint64_t* keys, uint32_t* vals, uint64_t* alt_keys, uint32_t* alt_vals, uint64_t n,
                                int begin_bit, int end_bit, const SortTemp& t, uint32_t* status, int spin_limit,
                                cudaStream_t s) {
  return sort_impl<uint64_t>(keys, vals, alt_keys, alt_vals, n, begin_bit, end_bit, t, status, s, spin_limit, true);
}

}  // namespace vi
