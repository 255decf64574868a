// Test infrastructure: a C entry layer over the reference extension's own CUDA
// sources (compiled in place by oracle/ref/Makefile), used to pin the CPU
// oracle against the reference itself.  Nothing in the product loads this.
//
// ref_binning_*   runs the reference's preprocess, CUB scan, duplicateWithKeys,
//                 CUB radix sort and identifyTileRanges in the order of
//                 cuda_integrator/integrator_impl.cu:277-365, stopping before
//                 the render kernel.  These kernels have no CTA barriers of
//                 their own, so any input is safe to run.
// ref_forward_*   calls the reference's whole Integrator::forward
// ref_backward_*  and Integrator::backward.  The reference render kernel skips
//                 a CTA barrier for pixels that no grid point covers
//                 (forward.cu:629-631 vs :715), so callers only pass scenes in
//                 which, by construction and CPU check, every active pixel is
//                 covered by every primitive it visits; every thread then takes
//                 the same barriers.  The *_bf libraries link the barrier-fixed
//                 render kernel (barrier_fix.py) instead, which takes every
//                 barrier on any scene.
// ref_time_*      timing of the reference's kernels (bottom of this file).
#include <cuda_runtime.h>

#include <cstdint>
#include <cstdio>
#include <functional>

#include "forward.h"
#include "integrator_impl.h"

uint32_t getHigherMsb(uint32_t n);  // integrator_impl.cu:47
__global__ void duplicateWithKeys(int P, const float2* points_xy, const float* depths, const uint32_t* offsets,
                                  uint64_t* gaussian_keys_unsorted, uint32_t* gaussian_values_unsorted, int* radii,
                                  dim3 grid);                                         // integrator_impl.cu:106
__global__ void identifyTileRanges(int L, uint64_t* point_list_keys, uint2* ranges);  // integrator_impl.cu:152

namespace {

int err(const char* where) {
  cudaError_t e = cudaDeviceSynchronize();
  if (e == cudaSuccess) e = cudaGetLastError();
  if (e != cudaSuccess) {
    fprintf(stderr, "ref_harness %s: %s\n", where, cudaGetErrorString(e));
    return 1;
  }
  return 0;
}

struct Binning {
  int P = 0, tiles = 0;
  long long R = 0;
  int* radii = nullptr;
  float2* means2D = nullptr;
  float* depths = nullptr;
  uint32_t *tt = nullptr, *offsets = nullptr, *vu = nullptr, *vs = nullptr;
  uint64_t *ku = nullptr, *ks = nullptr;
  uint2* ranges = nullptr;
  void *scan_tmp = nullptr, *sort_tmp = nullptr;
  void release() {
    void* ps[] = {radii, means2D, depths, tt, offsets, vu, vs, ku, ks, ranges, scan_tmp, sort_tmp};
    for (void* p : ps)
      if (p) cudaFree(p);
    *this = Binning();
  }
} g_bin;

char* g_buf[3] = {nullptr, nullptr, nullptr};
size_t g_cap[3] = {0, 0, 0};
int g_P = 0, g_W = 0, g_H = 0, g_K = 0, g_R = 0;

std::function<char*(size_t)> buffer(int i) {
  return [i](size_t n) -> char* {
    if (n == 0) return g_buf[i];  // backward: reuse (integrate_primitives.cu:56-60)
    if (g_cap[i] < n) {
      if (g_buf[i]) cudaFree(g_buf[i]);
      cudaMalloc((void**)&g_buf[i], n);
      g_cap[i] = n;
    }
    return g_buf[i];
  };
}

}  // namespace

extern "C" int ref_binning_run(int P, const float* means, float scale, const float* view, const float* proj, int W,
                               int H, float tan_fovx, float tan_fovy, long long* R_out) {
  g_bin.release();
  Binning& b = g_bin;
  b.P = P;
  const dim3 grid((W + 15) / 16, (H + 15) / 16, 1);
  b.tiles = grid.x * grid.y;
  cudaMalloc((void**)&b.radii, sizeof(int) * P);
  cudaMalloc((void**)&b.means2D, sizeof(float2) * P);
  cudaMalloc((void**)&b.depths, sizeof(float) * P);
  cudaMalloc((void**)&b.tt, sizeof(uint32_t) * P);
  cudaMalloc((void**)&b.offsets, sizeof(uint32_t) * P);
  const float focal_y = (float)H / (2.0f * tan_fovy);  // integrator_impl.cu:273-274
  const float focal_x = (float)W / (2.0f * tan_fovx);
  FORWARD::preprocess(P, means, scale, view, proj, W, H, tan_fovx, tan_fovy, focal_x, focal_y, b.radii, b.means2D,
                      b.depths, grid, b.tt, false);
  size_t scan_bytes = 0;
  cub::DeviceScan::InclusiveSum(nullptr, scan_bytes, b.tt, b.offsets, P);
  cudaMalloc(&b.scan_tmp, scan_bytes);
  cub::DeviceScan::InclusiveSum(b.scan_tmp, scan_bytes, b.tt, b.offsets, P);
  int R = 0;
  cudaMemcpy(&R, b.offsets + P - 1, sizeof(int), cudaMemcpyDeviceToHost);
  b.R = R;
  size_t n = R > 0 ? (size_t)R : 1;
  cudaMalloc((void**)&b.ku, 8 * n);
  cudaMalloc((void**)&b.ks, 8 * n);
  cudaMalloc((void**)&b.vu, 4 * n);
  cudaMalloc((void**)&b.vs, 4 * n);
  cudaMemset(b.ku, 0xff, 8 * n);  // slots the reference never writes stay deterministic
  cudaMemset(b.vu, 0xff, 4 * n);
  duplicateWithKeys<<<(P + 255) / 256, 256>>>(P, b.means2D, b.depths, b.offsets, b.ku, b.vu, b.radii, grid);
  const int bit = (int)getHigherMsb(grid.x * grid.y);
  size_t sort_bytes = 0;
  cub::DeviceRadixSort::SortPairs(nullptr, sort_bytes, b.ku, b.ks, b.vu, b.vs, R, 0, 32 + bit);
  cudaMalloc(&b.sort_tmp, sort_bytes > 0 ? sort_bytes : 1);
  cub::DeviceRadixSort::SortPairs(b.sort_tmp, sort_bytes, b.ku, b.ks, b.vu, b.vs, R, 0, 32 + bit);
  cudaMalloc((void**)&b.ranges, sizeof(uint2) * b.tiles);
  cudaMemset(b.ranges, 0, sizeof(uint2) * b.tiles);
  if (R > 0) identifyTileRanges<<<(R + 255) / 256, 256>>>(R, b.ks, b.ranges);
  *R_out = R;
  return err("binning");
}

extern "C" int ref_binning_fetch(int* radii, float* means2D, float* depths, uint32_t* tiles_touched, uint64_t* keys,
                                 uint32_t* point_list, uint32_t* ranges) {
  Binning& b = g_bin;
  cudaMemcpy(radii, b.radii, sizeof(int) * b.P, cudaMemcpyDeviceToHost);
  cudaMemcpy(means2D, b.means2D, sizeof(float2) * b.P, cudaMemcpyDeviceToHost);
  cudaMemcpy(depths, b.depths, sizeof(float) * b.P, cudaMemcpyDeviceToHost);
  cudaMemcpy(tiles_touched, b.tt, sizeof(uint32_t) * b.P, cudaMemcpyDeviceToHost);
  if (b.R > 0) {
    cudaMemcpy(keys, b.ks, 8 * b.R, cudaMemcpyDeviceToHost);
    cudaMemcpy(point_list, b.vs, 4 * b.R, cudaMemcpyDeviceToHost);
  }
  cudaMemcpy(ranges, b.ranges, sizeof(uint2) * b.tiles, cudaMemcpyDeviceToHost);
  int rc = err("binning fetch");
  g_bin.release();
  return rc;
}

extern "C" int ref_mark_visible(int P, float* means, float* view, float* proj, bool* present) {
  CudaIntegrator::Integrator it;
  it.markVisible(P, means, view, proj, present);
  return err("mark_visible");
}

extern "C" int ref_forward_run(int P, int W, int H, const float* means, float scale, const float* view,
                               const float* proj, const float* cam_pos, float near_plane, float max_distance,
                               float tan_fovx, float tan_fovy, const float* conf, const float* table, const int* res,
                               const int* do_hash, const int* primes, int T, const float* Wl, const float* bl,
                               int genus, int G, int K, float occ, const float* bg, float* out_color, float* out_feat,
                               float* vis, unsigned F, unsigned Fout, unsigned I, unsigned L, int* R_out) {
  CudaIntegrator::Integrator it;
  int R = it.forward(buffer(0), buffer(1), buffer(2), P, W, H, means, scale, view, proj, cam_pos, near_plane,
                     max_distance, tan_fovx, tan_fovy, conf, table, res, do_hash, primes, T, Wl, bl, genus, G, K, occ,
                     bg, out_color, out_feat, vis, F, Fout, I, L, 3, nullptr, false);
  g_P = P;
  g_W = W;
  g_H = H;
  g_K = K;
  g_R = R;
  *R_out = R;
  return err("forward");
}

extern "C" int ref_forward_fetch(float* final_T, int* n_contrib, int* contrib_idx, float* delta_t, uint32_t* ranges,
                                 uint64_t* keys, uint32_t* point_list, int* radii) {
  const size_t N = (size_t)g_W * g_H, tiles = (size_t)((g_W + 15) / 16) * ((g_H + 15) / 16);
  char* ip = g_buf[2];
  CudaIntegrator::ImageState im = CudaIntegrator::ImageState::fromChunk(ip, N, g_K);
  cudaMemcpy(final_T, im.final_transmittance, 4 * N, cudaMemcpyDeviceToHost);
  cudaMemcpy(n_contrib, im.num_contrib_per_pixel, 4 * N, cudaMemcpyDeviceToHost);
  cudaMemcpy(contrib_idx, im.pixel_contributing_indices, 4 * N * g_K, cudaMemcpyDeviceToHost);
  cudaMemcpy(delta_t, im.delta_t, 4 * N * g_K, cudaMemcpyDeviceToHost);
  cudaMemcpy(ranges, im.ranges, 8 * tiles, cudaMemcpyDeviceToHost);
  char* gp = g_buf[0];
  CudaIntegrator::GeometryState gs = CudaIntegrator::GeometryState::fromChunk(gp, g_P);
  cudaMemcpy(radii, gs.internal_radii, 4 * g_P, cudaMemcpyDeviceToHost);
  if (g_R > 0) {
    char* bp = g_buf[1];
    CudaIntegrator::BinningState bs = CudaIntegrator::BinningState::fromChunk(bp, g_R);
    cudaMemcpy(keys, bs.point_list_keys, 8 * (size_t)g_R, cudaMemcpyDeviceToHost);
    cudaMemcpy(point_list, bs.point_list, 4 * (size_t)g_R, cudaMemcpyDeviceToHost);
  }
  return err("forward fetch");
}

extern "C" int ref_backward_run(const float* dL_dcolor, const float* dL_dfeat, const float* means, float scale,
                                const float* view, const float* proj, const float* cam_pos, float near_plane,
                                float max_distance, float tan_fovx, float tan_fovy, const float* conf,
                                const float* table, const int* res, const int* do_hash, const int* primes, int T,
                                const float* Wl, const float* bl, int genus, int G, int K, float occ, const float* bg,
                                unsigned F, unsigned Fout, unsigned L, uint32_t table_size, float* dmeans, float* dconf,
                                float* dtable, float* dW, float* db) {
  CudaIntegrator::Integrator it;
  if (g_R > 0)
    it.backward(buffer(0), buffer(1), buffer(2), g_P, g_R, g_W, g_H, means, scale, view, proj, cam_pos, near_plane,
                max_distance, tan_fovx, tan_fovy, conf, table, res, do_hash, primes, T, Wl, bl, genus, G, K, occ, bg, F,
                Fout, L, 3, table_size, dL_dcolor, dL_dfeat, dmeans, dconf, dtable, dW, db, 0, false);
  return err("backward");
}

// ---------------------------------------------------------------------------
// Timing of the reference's kernels on a B200 (test infrastructure: the
// baseline the B200 renderer is measured against).  Buffers are allocated
// before the timed region; times are CUDA events on the legacy stream the
// reference launches on, averaged over `reps` repetitions.
//
// ref_time_binning: preprocess, CUB inclusive scan (+ the 4-byte read of R the
// reference makes, integrator_impl.cu:311), duplicateWithKeys, CUB radix sort
// over bits [0, 32 + getHigherMsb(tiles)) and identifyTileRanges, in the order
// of integrator_impl.cu:277-365.  ms[0..4] = those five stages, ms[5] = the sort
// alone again on already-duplicated keys (CUB keys/s), R_out = overlaps.
// ---------------------------------------------------------------------------
extern "C" int ref_time_binning(int P, const float* means, float scale, const float* view, const float* proj, int W,
                                int H, float tan_fovx, float tan_fovy, int reps, double* ms, long long* R_out) {
  Binning b;
  b.P = P;
  const dim3 grid((W + 15) / 16, (H + 15) / 16, 1);
  b.tiles = grid.x * grid.y;
  cudaMalloc((void**)&b.radii, sizeof(int) * P);
  cudaMalloc((void**)&b.means2D, sizeof(float2) * P);
  cudaMalloc((void**)&b.depths, sizeof(float) * P);
  cudaMalloc((void**)&b.tt, sizeof(uint32_t) * P);
  cudaMalloc((void**)&b.offsets, sizeof(uint32_t) * P);
  const float focal_y = (float)H / (2.0f * tan_fovy);
  const float focal_x = (float)W / (2.0f * tan_fovx);
  size_t scan_bytes = 0;
  cub::DeviceScan::InclusiveSum(nullptr, scan_bytes, b.tt, b.offsets, P);
  cudaMalloc(&b.scan_tmp, scan_bytes);
  // one untimed pass to size the R-dependent buffers
  FORWARD::preprocess(P, means, scale, view, proj, W, H, tan_fovx, tan_fovy, focal_x, focal_y, b.radii, b.means2D,
                      b.depths, grid, b.tt, false);
  cub::DeviceScan::InclusiveSum(b.scan_tmp, scan_bytes, b.tt, b.offsets, P);
  int R = 0;
  cudaMemcpy(&R, b.offsets + P - 1, sizeof(int), cudaMemcpyDeviceToHost);
  b.R = R;
  const size_t n = R > 0 ? (size_t)R : 1;
  cudaMalloc((void**)&b.ku, 8 * n);
  cudaMalloc((void**)&b.ks, 8 * n);
  cudaMalloc((void**)&b.vu, 4 * n);
  cudaMalloc((void**)&b.vs, 4 * n);
  const int bit = (int)getHigherMsb(grid.x * grid.y);
  size_t sort_bytes = 0;
  cub::DeviceRadixSort::SortPairs(nullptr, sort_bytes, b.ku, b.ks, b.vu, b.vs, R, 0, 32 + bit);
  cudaMalloc(&b.sort_tmp, sort_bytes > 0 ? sort_bytes : 1);
  cudaMalloc((void**)&b.ranges, sizeof(uint2) * b.tiles);
  if (err("binning set-up")) {
    b.release();
    return 1;
  }
  cudaEvent_t ev[7];
  for (auto& e : ev) cudaEventCreate(&e);
  double acc[6] = {0, 0, 0, 0, 0, 0};
  for (int r = 0; r < reps + 1; r++) {  // repetition 0 warms up
    cudaEventRecord(ev[0]);
    FORWARD::preprocess(P, means, scale, view, proj, W, H, tan_fovx, tan_fovy, focal_x, focal_y, b.radii,
                        b.means2D, b.depths, grid, b.tt, false);
    cudaEventRecord(ev[1]);
    cub::DeviceScan::InclusiveSum(b.scan_tmp, scan_bytes, b.tt, b.offsets, P);
    int Rr = 0;
    cudaMemcpy(&Rr, b.offsets + P - 1, sizeof(int), cudaMemcpyDeviceToHost);
    cudaEventRecord(ev[2]);
    duplicateWithKeys<<<(P + 255) / 256, 256>>>(P, b.means2D, b.depths, b.offsets, b.ku, b.vu, b.radii, grid);
    cudaEventRecord(ev[3]);
    cub::DeviceRadixSort::SortPairs(b.sort_tmp, sort_bytes, b.ku, b.ks, b.vu, b.vs, R, 0, 32 + bit);
    cudaEventRecord(ev[4]);
    cudaMemset(b.ranges, 0, sizeof(uint2) * b.tiles);
    if (R > 0) identifyTileRanges<<<(R + 255) / 256, 256>>>(R, b.ks, b.ranges);
    cudaEventRecord(ev[5]);
    cub::DeviceRadixSort::SortPairs(b.sort_tmp, sort_bytes, b.ku, b.ks, b.vu, b.vs, R, 0, 32 + bit);
    cudaEventRecord(ev[6]);
    cudaEventSynchronize(ev[6]);
    if (r == 0) continue;
    for (int i = 0; i < 5; i++) {
      float t = 0.0f;
      cudaEventElapsedTime(&t, ev[i], ev[i + 1]);
      acc[i] += t;
    }
    float t = 0.0f;
    cudaEventElapsedTime(&t, ev[5], ev[6]);
    acc[5] += t;
  }
  for (int i = 0; i < 6; i++) ms[i] = acc[i] / (reps > 0 ? reps : 1);
  *R_out = R;
  for (auto& e : ev) cudaEventDestroy(e);
  const int rc = err("binning timing");
  b.release();
  return rc;
}

// Time of the last ref_forward_run / ref_backward_run call (CUDA events around
// the whole Integrator call; the reference synchronises the device inside).
namespace {
float g_last_ms = 0.0f;
}
extern "C" double ref_last_call_ms(void) { return g_last_ms; }

extern "C" int ref_timed_forward(int P, int W, int H, const float* means, float scale, const float* view,
                                 const float* proj, const float* cam_pos, float near_plane, float max_distance,
                                 float tan_fovx, float tan_fovy, const float* conf, const float* table, const int* res,
                                 const int* do_hash, const int* primes, int T, const float* Wl, const float* bl,
                                 int genus, int G, int K, float occ, const float* bg, float* out_color, float* out_feat,
                                 float* vis, unsigned F, unsigned Fout, unsigned I, unsigned L, int* R_out) {
  cudaEvent_t a, b;
  cudaEventCreate(&a);
  cudaEventCreate(&b);
  cudaEventRecord(a);
  const int rc = ref_forward_run(P, W, H, means, scale, view, proj, cam_pos, near_plane, max_distance, tan_fovx,
                                 tan_fovy, conf, table, res, do_hash, primes, T, Wl, bl, genus, G, K, occ, bg,
                                 out_color, out_feat, vis, F, Fout, I, L, R_out);
  cudaEventRecord(b);
  cudaEventSynchronize(b);
  cudaEventElapsedTime(&g_last_ms, a, b);
  cudaEventDestroy(a);
  cudaEventDestroy(b);
  return rc;
}

extern "C" int ref_timed_backward(const float* dL_dcolor, const float* dL_dfeat, const float* means, float scale,
                                  const float* view, const float* proj, const float* cam_pos, float near_plane,
                                  float max_distance, float tan_fovx, float tan_fovy, const float* conf,
                                  const float* table, const int* res, const int* do_hash, const int* primes, int T,
                                  const float* Wl, const float* bl, int genus, int G, int K, float occ,
                                  const float* bg, unsigned F, unsigned Fout, unsigned L, uint32_t table_size,
                                  float* dmeans, float* dconf, float* dtable, float* dW, float* db) {
  cudaEvent_t a, b;
  cudaEventCreate(&a);
  cudaEventCreate(&b);
  cudaEventRecord(a);
  const int rc = ref_backward_run(dL_dcolor, dL_dfeat, means, scale, view, proj, cam_pos, near_plane, max_distance,
                                  tan_fovx, tan_fovy, conf, table, res, do_hash, primes, T, Wl, bl, genus, G, K, occ,
                                  bg, F, Fout, L, table_size, dmeans, dconf, dtable, dW, db);
  cudaEventRecord(b);
  cudaEventSynchronize(b);
  cudaEventElapsedTime(&g_last_ms, a, b);
  cudaEventDestroy(a);
  cudaEventDestroy(b);
  return rc;
}
