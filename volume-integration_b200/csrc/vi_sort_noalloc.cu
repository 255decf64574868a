// vi_sort_pairs_noalloc: the stable radix sort of vi_sort_pairs for callers that
// must not allocate device memory.  Some hosts own every byte of device memory
// themselves -- an engine or plugin host with a fixed memory budget, a serving
// process whose allocator is sized up front -- and some cannot afford the
// implicit device-wide synchronisation that cudaMalloc/cudaFree may perform in
// the middle of a frame.  They pass keys and values in and out; the sort's own
// scratch (digit histograms, look-back words, tile counters, status word) lives
// in a fixed device array inside this library.
#include <cuda_runtime.h>

#include <cstdint>
#include <cstring>
#include <mutex>

#include "../../include/volume_integration_b200.h"
#include "vi_common.cuh"
#include "vi_internal.h"

namespace vi {
namespace {

// Scratch for at most VI_SORT_NOALLOC_MAX_KEYS keys over any bit range: 256 bytes
// of status word, then the sort's histograms, look-back words and counters.
// Every GPU that loads the library keeps this array until the process exits.
constexpr size_t kScratchBytes = VI_SORT_NOALLOC_SCRATCH_BYTES;
static __device__ __align__(256) unsigned char g_sort_scratch[kScratchBytes];

std::mutex g_mu;
void* g_scratch_addr[64] = {};  // device address of g_sort_scratch per device

}  // namespace

int set_error(int code, const char* msg);

}  // namespace vi

using namespace vi;

extern "C" int vi_sort_pairs_noalloc(uint64_t* keys_in, uint32_t* vals_in, uint64_t* keys_out, uint32_t* vals_out,
                                     uint64_t n, int begin_bit, int end_bit, void* stream) {
  cudaStream_t s = (cudaStream_t)stream;
  if (n > VI_SORT_NOALLOC_MAX_KEYS)
    return set_error(VI_ERR_INVALID_ARGUMENT, "vi_sort_pairs_noalloc: n exceeds VI_SORT_NOALLOC_MAX_KEYS (2^20)");
  if (begin_bit < 0 || end_bit > 64 || begin_bit > end_bit)
    return set_error(VI_ERR_INVALID_ARGUMENT, "vi_sort_pairs_noalloc: bit range outside [0, 64]");
  if (n == 0) return VI_OK;
  if (256 + sort_temp_bytes(n, 8, begin_bit, end_bit) > kScratchBytes)
    return set_error(VI_ERR_INVALID_ARGUMENT, "vi_sort_pairs_noalloc: scratch too small for this size");
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess || dev < 0 || dev >= 64) return set_error(VI_ERR_CUDA, "vi_sort_pairs_noalloc: no device");
  char* base;
  {
    // The array's name is only a host-side stand-in: the kernels need its device
    // address, resolved once per device while that device is current.
    std::lock_guard<std::mutex> lk(g_mu);
    if (!g_scratch_addr[dev]) {
      void* p = nullptr;
      e = cudaGetSymbolAddress(&p, g_sort_scratch);
      if (e != cudaSuccess) return set_error(VI_ERR_CUDA, "vi_sort_pairs_noalloc: cudaGetSymbolAddress failed");
      g_scratch_addr[dev] = p;
    }
    base = (char*)g_scratch_addr[dev];
  }
  uint32_t* status = (uint32_t*)base;
  SortTemp st;
  sort_temp_carve(base + 256, n, 8, begin_bit, end_bit, st);
  // The array keeps the previous call's contents: the status word is cleared
  // here, the histograms, counters and look-back words inside the sort.
  cudaMemsetAsync(status, 0, sizeof(uint32_t), s);
  const bool alt = onesweep_sort_u64(keys_in, vals_in, keys_out, vals_out, n, begin_bit, end_bit, st, status, s);
  if (!alt) {
    cudaMemcpyAsync(keys_out, keys_in, n * 8, cudaMemcpyDeviceToDevice, s);
    cudaMemcpyAsync(vals_out, vals_in, n * 4, cudaMemcpyDeviceToDevice, s);
  }
  e = cudaGetLastError();
  if (e != cudaSuccess) return set_error(VI_ERR_CUDA, cudaGetErrorString(e));
  // A look-back wait that gave up leaves positions of keys_out unwritten: wait
  // for the sort and report it rather than return unsorted output as VI_OK.
  return read_sort_status(status, nullptr, s, "vi_sort_pairs_noalloc");
}
