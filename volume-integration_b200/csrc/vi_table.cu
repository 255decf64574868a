// A level-major copy of the hashgrid feature table for the feature stage.
//
// The reference stores the table entry-major, [T][L][F] (hashgrid.h:253-287):
// entry e's features of every level share one row of L*F floats.  A query
// reads one entry per corner at one level, so each 8-byte (F = 2) read claims
// its own 32-byte sector.  Level-major, [L][T][F], the two corners of a query
// that differ along x (hash prime 1, or the dense index's unit stride) are
// neighbouring entries and usually share a sector, and so do the neighbouring
// grid points of one primitive at the fine levels.  The forward copies the
// caller's table into this layout once per call (T*L*F floats read and
// written) and the feature stage gathers from the copy.  Values, weights and
// summation order are unchanged, so the features are bit-identical; only the
// addresses move.  The backward keeps the caller's layout: its table-gradient
// atomics into a level-major scratch measured slower (neighbouring entries in
// one sector collide at the L2), and its kernel with run-time table strides
// was 13% slower even in the caller's layout.
#include <cstdlib>
#include <cstring>

#include "vi_internal.h"

namespace vi {
namespace {

constexpr int kEntriesPerBlock = 32;

// dst[l][e][f] = src[e][l][f] for kEntriesPerBlock entries per block, staged
// in shared memory: rows of L*F floats in, L runs of 32*F floats out.
__global__ void __launch_bounds__(256) table_to_level_major_kernel(const float* __restrict__ src,
                                                                     float* __restrict__ dst, uint32_t T, int L,
                                                                     int F) {
  extern __shared__ float tile[];  // [kEntriesPerBlock][L*F]
  const int D = L * F;
  const uint64_t e0 = (uint64_t)blockIdx.x * kEntriesPerBlock;
  const int ne = T - e0 < (uint64_t)kEntriesPerBlock ? (int)(T - e0) : kEntriesPerBlock;
  const float* s = src + e0 * D;
  for (int i = threadIdx.x; i < ne * D; i += blockDim.x) tile[i] = s[i];
  __syncthreads();
  const int run = ne * F;
  for (int i = threadIdx.x; i < L * run; i += blockDim.x) {
    const int l = i / run, j = i - l * run, e = j / F, f = j - e * F;
    dst[((uint64_t)l * T + e0) * F + j] = tile[e * D + l * F + f];
  }
}

}  // namespace

bool table_level_major() {
  const char* e = std::getenv("VI_TABLE_LAYOUT");
  return !(e && std::strcmp(e, "entry") == 0);
}

void launch_table_to_level_major(const float* src, float* dst, uint32_t T, int L, int F, cudaStream_t s) {
  if (T == 0) return;
  const unsigned blocks = (unsigned)((T + kEntriesPerBlock - 1) / kEntriesPerBlock);
  table_to_level_major_kernel<<<blocks, 256, sizeof(float) * kEntriesPerBlock * L * F, s>>>(src, dst, T, L, F);
  note_launches(1);
}

}  // namespace vi
