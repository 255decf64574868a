// C ABI of the renderer: argument checks, state-buffer layouts and the stage
// order of one forward / backward call (reference
// cuda_integrator/integrator_impl.cu:196-469 and :474-756).
#include <cuda_runtime.h>

#include <algorithm>
#include <atomic>
#include <cstdarg>
#include <mutex>
#include <vector>
#include <cstdint>
#include <cstdio>
#include <cmath>
#include <cstdlib>
#include <cstring>

#include "../../include/volume_integration_b200.h"
#include "vi_common.cuh"
#include "vi_internal.h"

namespace vi {
namespace {

thread_local char g_err[512];

int fail(int code, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_err, sizeof g_err, fmt, ap);
  va_end(ap);
  return code;
}

int cuda_fail(cudaError_t e, const char* where) {
  return fail(VI_ERR_CUDA, "%s: %s", where, cudaGetErrorString(e));
}

// Layout helper: carves consecutive 256-byte aligned arrays out of a base
// address (or out of address 0 to measure the total size).
struct Carver {
  uintptr_t base, cur;
  explicit Carver(char* b) : base((uintptr_t)b), cur(0) {}
  template <typename T>
  T* take(size_t count) {
    cur = align_up(cur);
    T* p = (T*)(base + cur);
    cur += sizeof(T) * count;
    return p;
  }
  size_t size() const { return align_up(cur) + 256; }
};

int props_stride(int O) { return O > 8 ? 16 : 8; }

// Mapped pinned host words the forward reads the overlap count from (this
// thread's; the device address is the same under unified addressing).
thread_local uint64_t* g_pinned = nullptr;
thread_local uint32_t* g_pinned_dev = nullptr;
thread_local cudaEvent_t g_events[64] = {};

cudaEvent_t event_for_device() {
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64) dev = 0;
  if (!g_events[dev]) cudaEventCreateWithFlags(&g_events[dev], cudaEventDisableTiming);
  return g_events[dev];
}

std::atomic<unsigned long long> g_launch_count{0};

// Stage timing: events recorded on the launching stream, resolved on read.
struct StagePair {
  int stage;
  cudaEvent_t a, b;
};
std::mutex g_prof_mu;
bool g_prof_on = false;
std::vector<StagePair> g_prof_pending;
std::vector<cudaEvent_t> g_prof_free;
double g_prof_ms[kStCount] = {};
unsigned long long g_prof_calls[kStCount] = {};
thread_local cudaEvent_t g_open[kStCount] = {};

cudaEvent_t prof_event() {
  if (!g_prof_free.empty()) {
    cudaEvent_t e = g_prof_free.back();
    g_prof_free.pop_back();
    return e;
  }
  cudaEvent_t e;
  cudaEventCreate(&e);
  return e;
}

}  // namespace

void note_launches(int n) { g_launch_count.fetch_add((unsigned long long)n, std::memory_order_relaxed); }

namespace {
std::mutex g_l2_mu;
bool g_l2_limit_set[64] = {};
}  // namespace

int l2_persist_attr(const void* base, size_t bytes, cudaLaunchAttribute* attr) {
  // Opt-in: on the headline scene the window sped the feature stage up by 3.5%
  // (10% inside the scene's own bounds), but the table's persisting lines stay
  // in L2 after it and the render and the per-pixel backward, which live on
  // L2, slowed down by more than that (frame 4.33 -> 5.84 ms).
  const char* e = std::getenv("VI_L2_WINDOW");
  if (!(e && e[0] == '1') || !base || !bytes) return 0;
  int dev = 0, max_win = 0, max_persist = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 0;
  cudaDeviceGetAttribute(&max_win, cudaDevAttrMaxAccessPolicyWindowSize, dev);
  cudaDeviceGetAttribute(&max_persist, cudaDevAttrMaxPersistingL2CacheSize, dev);
  if (max_win <= 0 || max_persist <= 0) return 0;
  {
    std::lock_guard<std::mutex> lk(g_l2_mu);
    if (!g_l2_limit_set[dev]) {
      if (cudaDeviceSetLimit(cudaLimitPersistingL2CacheSize, (size_t)max_persist) != cudaSuccess) {
        cudaGetLastError();
        return 0;
      }
      g_l2_limit_set[dev] = true;
    }
  }
  attr->id = cudaLaunchAttributeAccessPolicyWindow;
  attr->val.accessPolicyWindow.base_ptr = const_cast<void*>(base);
  attr->val.accessPolicyWindow.num_bytes = std::min(bytes, (size_t)max_win);
  attr->val.accessPolicyWindow.hitRatio =
      (float)std::min(1.0, (double)max_persist / (double)attr->val.accessPolicyWindow.num_bytes);
  attr->val.accessPolicyWindow.hitProp = cudaAccessPropertyPersisting;
  attr->val.accessPolicyWindow.missProp = cudaAccessPropertyStreaming;
  return 1;
}

int resident_blocks(const void* kernel, int threads, size_t smem) {
  int dev = 0, sms = 0, per = 0;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per, kernel, threads, smem);
  return (sms > 0 ? sms : 1) * (per > 0 ? per : 1);
}

void stage_begin(Stage st, cudaStream_t s) {
  if (!g_prof_on) return;
  std::lock_guard<std::mutex> lk(g_prof_mu);
  g_open[st] = prof_event();
  cudaEventRecord(g_open[st], s);
}

void stage_end(Stage st, cudaStream_t s) {
  if (!g_prof_on || !g_open[st]) return;
  std::lock_guard<std::mutex> lk(g_prof_mu);
  cudaEvent_t e = prof_event();
  cudaEventRecord(e, s);
  g_prof_pending.push_back({(int)st, g_open[st], e});
  g_open[st] = nullptr;
}

size_t phi_cache_max_bytes() {
  const char* e = std::getenv("VI_PHI_CACHE_BYTES");
  if (!e || !*e) return kPhiCacheMaxBytes;
  char* end = nullptr;
  const unsigned long long v = std::strtoull(e, &end, 10);
  return (end && *end == '\0') ? (size_t)v : kPhiCacheMaxBytes;
}

GeomState geom_layout(char* base, size_t P, int V, int O, int D, size_t table_floats) {
  GeomState g;
  Carver c(base);
  const int OP = props_stride(O);
  g.status = c.take<uint32_t>(64);
  g.depths = c.take<float>(P);
  g.radii = c.take<int>(P);
  g.means2D = c.take<float>(2 * P);
  g.tiles_touched = c.take<uint32_t>(P);
  g.dkeys = c.take<uint32_t>(P);
  g.didx = c.take<uint32_t>(P);
  g.dkeys_alt = c.take<uint32_t>(P);
  g.didx_alt = c.take<uint32_t>(P);
  g.offsets = c.take<uint32_t>(P);
  g.block_sums = c.take<uint32_t>((P + kScanBlock - 1) / kScanBlock + 1);
  g.rec_cnt = c.take<uint32_t>(P);
  g.rec_key = c.take<uint32_t>(P * V);
  g.rec_props = c.take<float>(P * V * OP);
  g.rec_pix = c.take<uint32_t>(P * V);
  g.rec_dpre = c.take<float>(P * V * OP);
  char* st = c.take<char>(sort_temp_bytes(P, 4, 0, 32));
  sort_temp_carve(st, P, 4, 0, 32, g.sort);
  g.differs_list = c.take<uint32_t>(P);
  // Last, so the offsets above do not depend on D.
  g.cls_base = c.take<uint32_t>(P);
  const size_t want = V <= 32 ? P * (size_t)V : 0;  // grids of G = 4, 5 gather again in the backward
  size_t cap = D > 0 ? std::min(want, phi_cache_max_bytes() / (sizeof(float) * (size_t)D)) : 0;
  cap = std::min(cap, (size_t)kCornerCache - 1);  // the top bit of cls_base marks box-corner primitives
  g.phi_cap = (uint32_t)cap;
  g.phi_cache = c.take<float>(cap * (size_t)D);
  // After everything the backward reads: only the forward uses it.
  g.table_lm = table_floats ? c.take<float>(table_floats) : nullptr;
  g.bytes = c.size();
  return g;
}

BinState bin_layout(char* base, uint64_t R, int tb) {
  BinState b;
  Carver c(base);
  b.tkeys = c.take<uint32_t>(R);
  b.tvals = c.take<uint32_t>(R);
  b.tkeys_alt = c.take<uint32_t>(R);
  b.tvals_alt = c.take<uint32_t>(R);
  char* st = c.take<char>(sort_temp_bytes(R, 4, 0, tb));
  sort_temp_carve(st, R, 4, 0, tb, b.sort);
  b.bytes = c.size();
  return b;
}

ImgState img_layout(char* base, size_t N, int K, size_t tiles, bool exact) {
  ImgState m;
  Carver c(base);
  m.ranges = c.take<uint32_t>(2 * tiles);
  m.final_T = c.take<float>(N);
  m.n_contrib = c.take<int32_t>(N);
  m.contrib_idx = c.take<int32_t>(N * (size_t)K);
  m.delta_t = c.take<float>(N * (size_t)K);
  m.contrib_rec = c.take<uint32_t>(N * (size_t)K);
  m.trans = exact ? c.take<float>(N * (size_t)K) : nullptr;
  m.trig = exact ? c.take<uint32_t>(N * (size_t)K) : nullptr;
  m.bytes = c.size();
  return m;
}

namespace {

// Checks shared by forward and backward; fills the per-call constants.
int make_scene(Scene& sc, int P, const float* means3D, const float* conf, float scale, const float* view,
               const float* proj, float tanfovx, float tanfovy, int H, int W, float near_plane, float max_distance,
               const float* table, const int* res, const int* do_hash, const int* primes, int T, const float* Wl,
               const float* bl, int genus, int G, int K, const float* bg, unsigned F, unsigned Fout, unsigned L,
               unsigned channels, const float* hash_bounds) {
  if (channels != 3)
    return fail(VI_ERR_UNSUPPORTED, "num_output_channels=%u: only 3 colour channels are implemented (as the "
                                    "reference, forward.cu:838)", channels);
  if (P < 0 || H < 0 || W < 0 || K < 0) return fail(VI_ERR_INVALID_ARGUMENT, "negative size (P=%d H=%d W=%d K=%d)", P, H, W, K);
  if (G < 1 || G > 5)
    return fail(VI_ERR_UNSUPPORTED, "grid_size=%d: supported sizes are 1..5 (the reference's MAX_GRID_SIZE, "
                                    "forward.cu:204-205)", G);
  if (!(F == 1 || F == 2 || F == 4 || F == 8))
    return fail(VI_ERR_UNSUPPORTED, "input_feature_dim=%u: supported values are 1, 2, 4, 8", F);
  if (L < 1 || L * F > 64) return fail(VI_ERR_UNSUPPORTED, "hashgrid_levels*input_feature_dim=%u must be in [1, 64]", L * F);
  if (Fout > 12) return fail(VI_ERR_UNSUPPORTED, "output_feature_dim=%u: at most 12 is supported", Fout);
  if (T <= 0) return fail(VI_ERR_INVALID_ARGUMENT, "feature_offset=%d must be positive", T);
  if ((size_t)W * H >= (1ull << 31)) return fail(VI_ERR_UNSUPPORTED, "image of %d x %d pixels is too large", W, H);
  if (P > 0 && (!means3D || !conf || !view || !proj || !table || !res || !do_hash || !primes || !Wl || !bl || !bg))
    return fail(VI_ERR_INVALID_ARGUMENT, "a required input pointer is NULL");
  sc.P = P; sc.W = W; sc.H = H; sc.G = G; sc.V = G * G * G;
  sc.L = (int)L; sc.F = (int)F; sc.D = (int)(L * F); sc.Fout = (int)Fout; sc.O = (int)Fout + 4;
  sc.K = K; sc.genus = genus;
  sc.T = (uint32_t)T;
  sc.tab_l = F;  // the caller's entry-major layout until a level-major copy replaces it
  sc.tab_e = L * F;
  sc.Tmask = ((uint32_t)T & ((uint32_t)T - 1)) == 0 ? (uint32_t)T - 1 : 0u;
  sc.scale = scale;
  sc.step = G > 1 ? scale / (float)(G - 1) : scale;  // forward.cu:395
  sc.gof = (float)(G - 1) / 2.0f;                    // forward.cu:396
  sc.near_plane = near_plane; sc.max_distance = max_distance;
  sc.focal_y = (float)H / (2.0f * tanfovy);  // integrator_impl.cu:273-274
  sc.focal_x = (float)W / (2.0f * tanfovx);
  sc.means = means3D; sc.conf = conf; sc.view = view; sc.proj = proj; sc.table = table;
  sc.res = res; sc.do_hash = do_hash; sc.primes = primes; sc.Wl = Wl; sc.bl = bl; sc.bg = bg;
  sc.gx = (unsigned)(W + VI_TILE - 1) / VI_TILE;
  sc.gy = (unsigned)(H + VI_TILE - 1) / VI_TILE;
  sc.exact = false;
  sc.own_box = hash_bounds != nullptr;
  for (int a = 0; a < 3; a++) {
    if (!hash_bounds) {
      sc.hlo[a] = -1.3f;  // hashgrid.h:225-226
      sc.hext[a] = 2.6f;
      continue;
    }
    const float lo = hash_bounds[a], hi = hash_bounds[3 + a];
    if (!(std::isfinite(lo) && std::isfinite(hi) && hi > lo) || !std::isfinite(hi - lo))
      return fail(VI_ERR_INVALID_ARGUMENT, "hash_bounds axis %d: need finite lo < hi, got [%g, %g]", a, lo, hi);
    sc.hlo[a] = lo;
    sc.hext[a] = hi - lo;
  }
  return VI_OK;
}

int check(cudaStream_t s, int debug, const char* where, const uint32_t* status) {
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, where);
  if (debug) {
    e = cudaStreamSynchronize(s);
    if (e != cudaSuccess) return cuda_fail(e, where);
    if (status) {
      uint32_t st = 0;
      cudaMemcpy(&st, status, 4, cudaMemcpyDeviceToHost);
      if (st) return fail(VI_ERR_DEVICE, "%s: device status 0x%x", where, st);
    }
  }
  return VI_OK;
}

}  // namespace

cudaError_t begin_status_read(const uint32_t* status, cudaStream_t s) {
  if (!g_pinned) {
    cudaError_t e = cudaHostAlloc((void**)&g_pinned, 64, cudaHostAllocPortable | cudaHostAllocMapped);
    if (e != cudaSuccess) return e;
    e = cudaHostGetDevicePointer((void**)&g_pinned_dev, g_pinned, 0);
    if (e != cudaSuccess) {
      cudaFreeHost(g_pinned);
      g_pinned = nullptr;
      return e;
    }
  }
  launch_publish_status(status, g_pinned_dev, s);
  return cudaEventRecord(event_for_device(), s);
}

cudaError_t finish_status_read(uint32_t words[4]) {
  const cudaError_t e = cudaEventSynchronize(event_for_device());
  if (e != cudaSuccess) return e;
  const volatile uint32_t* pinned = reinterpret_cast<const volatile uint32_t*>(g_pinned);
  for (int i = 0; i < 4; i++) words[i] = pinned[i];
  return cudaSuccess;
}

// Records a message for vi_last_error() and returns code (for other translation units).
int set_error(int code, const char* msg) { return fail(code, "%s", msg); }

static_assert(VI_ERR_LOOKBACK_TIMEOUT == VI_DEVICE_LOOKBACK_TIMEOUT, "status bits of the public header");
static_assert(VI_ERR_RECORD_OVERFLOW == VI_DEVICE_RECORD_OVERFLOW, "status bits of the public header");
static_assert(VI_ERR_STAGE_TIMEOUT == VI_DEVICE_STAGE_TIMEOUT, "status bits of the public header");

int read_sort_status(const uint32_t* status, uint32_t* out, cudaStream_t s, const char* where) {
  uint32_t st = 0;  // host stack memory: no allocation on this path
  cudaError_t e = cudaMemcpyAsync(&st, status, sizeof st, cudaMemcpyDeviceToHost, s);
  if (e == cudaSuccess) e = cudaStreamSynchronize(s);
  if (e != cudaSuccess) return cuda_fail(e, where);
  if (out) *out = st;
  if (st)
    return fail(VI_ERR_DEVICE, "%s: device status 0x%x%s", where, st,
                (st & VI_ERR_LOOKBACK_TIMEOUT) ? " (a look-back wait gave up; the output is unspecified)" : "");
  return VI_OK;
}

int tile_bits(size_t tiles) {
  // getHigherMsb (integrator_impl.cu:47-62)
  uint32_t n = (uint32_t)tiles, msb = sizeof(n) * 4, step = msb;
  while (step > 1) {
    step /= 2;
    if (n >> msb) msb += step; else msb -= step;
  }
  if (n >> msb) msb++;
  return (int)msb;
}


}  // namespace vi

using namespace vi;

extern "C" const char* vi_last_error(void) { return g_err; }

extern "C" int vi_sort_end_bit(uint32_t num_tiles) { return 32 + tile_bits(num_tiles); }

namespace {
int forward_impl(
    vi_resize_fn geom_buffer, void* geom_user, vi_resize_fn binning_buffer, void* binning_user,
    vi_resize_fn img_buffer, void* img_user, float* out_color, float* out_features, float* visibility_info,
    int* num_rendered, int P, const float* means3D, const float* primitive_confidences, float primitive_scale,
    const float* viewmatrix, const float* projmatrix, const float* cam_pos, float tan_fovx, float tan_fovy,
    int image_height, int image_width, float near_plane, float max_distance, const float* feature_table,
    uint64_t feature_table_numel, const int* resolution, const int* do_hash, const int* primes, int feature_offset,
    const float* linear_weights, uint64_t linear_weights_numel, const float* linear_bias,
    uint64_t linear_bias_numel, int stencil_genus, int grid_size, int max_primitives_per_ray,
    float occupancy_threshold, const float* bg_color, unsigned input_feature_dim, unsigned output_feature_dim,
    unsigned intermediate_feature_dim, unsigned hashgrid_levels, unsigned num_output_channels, int debug,
    void* stream, const float* hash_bounds, unsigned flags) {
  (void)cam_pos;
  (void)occupancy_threshold;  // has no effect in the reference either (forward.cu:118-140 is never called)
  cudaStream_t s = (cudaStream_t)stream;
  if (!num_rendered || !geom_buffer || !binning_buffer || !img_buffer)
    return fail(VI_ERR_INVALID_ARGUMENT, "num_rendered and the three buffer callbacks are required");
  *num_rendered = 0;
  Scene sc;
  int rc = make_scene(sc, P, means3D, primitive_confidences, primitive_scale, viewmatrix, projmatrix, tan_fovx,
                      tan_fovy, image_height, image_width, near_plane, max_distance, feature_table, resolution,
                      do_hash, primes, feature_offset, linear_weights, linear_bias, stencil_genus, grid_size,
                      max_primitives_per_ray, bg_color, input_feature_dim, output_feature_dim, hashgrid_levels,
                      num_output_channels, hash_bounds);
  if (rc) return rc;
  if (flags & ~VI_FLAG_EXACT_GRADIENTS) return fail(VI_ERR_INVALID_ARGUMENT, "unknown flags 0x%x", flags);
  sc.exact = (flags & VI_FLAG_EXACT_GRADIENTS) != 0;
  if (sc.exact && sc.V > 32)
    return fail(VI_ERR_UNSUPPORTED, "exact_gradients needs grid_size <= 3 (got %d)", grid_size);
  if (intermediate_feature_dim != hashgrid_levels * input_feature_dim)
    return fail(VI_ERR_INVALID_ARGUMENT,
                "intermediate_feature_dim=%u must equal hashgrid_levels*input_feature_dim=%u (the reference reads "
                "uninitialised weights otherwise, forward.cu:326-331 vs :457)",
                intermediate_feature_dim, hashgrid_levels * input_feature_dim);
  if (feature_table_numel < (uint64_t)sc.T * sc.L * sc.F)
    return fail(VI_ERR_INVALID_ARGUMENT, "feature_table has %llu elements, needs feature_offset*L*F=%llu",
                (unsigned long long)feature_table_numel, (unsigned long long)sc.T * sc.L * sc.F);
  if (((uintptr_t)feature_table) % (size_t)(sc.F >= 4 ? 16 : sc.F * 4) != 0)
    return fail(VI_ERR_INVALID_ARGUMENT, "feature_table must be aligned to %d bytes (vector loads of one entry)",
                sc.F >= 4 ? 16 : sc.F * 4);
  if (linear_weights_numel < (uint64_t)sc.O * sc.D || linear_bias_numel < (uint64_t)sc.O)
    return fail(VI_ERR_INVALID_ARGUMENT, "linear layer needs %d weights and %d biases, got %llu and %llu",
                sc.O * sc.D, sc.O, (unsigned long long)linear_weights_numel, (unsigned long long)linear_bias_numel);
  const size_t N = (size_t)sc.W * sc.H;
  if (P == 0 || N == 0) {
    // integrate_primitives.cu:153-190: zero images, empty state.
    if (N) {
      cudaMemsetAsync(out_color, 0, 3 * N * sizeof(float), s);
      if (sc.Fout) cudaMemsetAsync(out_features, 0, sc.Fout * N * sizeof(float), s);
      cudaMemsetAsync(visibility_info, 0, N * sizeof(float), s);
    }
    return check(s, debug, "empty forward", nullptr);
  }
  const size_t tiles = (size_t)sc.gx * sc.gy;

  const size_t tfl = table_level_major() ? (size_t)sc.T * sc.L * sc.F : 0;
  GeomState g = geom_layout(nullptr, P, sc.V, sc.O, sc.D, tfl);
  char* gb = geom_buffer(geom_user, g.bytes);
  if (!gb) return fail(VI_ERR_ALLOC, "geometry buffer of %zu bytes", g.bytes);
  if ((uintptr_t)gb & 255) return fail(VI_ERR_INVALID_ARGUMENT, "state buffers must be 256-byte aligned");
  g = geom_layout(gb, P, sc.V, sc.O, sc.D, tfl);
  ImgState im = img_layout(nullptr, N, sc.K, tiles, sc.exact);
  char* ib = img_buffer(img_user, im.bytes);
  if (!ib) return fail(VI_ERR_ALLOC, "image buffer of %zu bytes", im.bytes);
  if ((uintptr_t)ib & 255) return fail(VI_ERR_INVALID_ARGUMENT, "state buffers must be 256-byte aligned");
  im = img_layout(ib, N, sc.K, tiles, sc.exact);

  cudaMemsetAsync(g.status, 0, 64 * sizeof(uint32_t), s);
  stage_begin(kStPreprocess, s);
  launch_preprocess(sc, g, s);
  stage_end(kStPreprocess, s);
  if ((rc = check(s, debug, "preprocess", g.status))) return rc;
  stage_begin(kStDepthSort, s);
  const bool depth_alt =
      onesweep_sort_u32(g.dkeys, g.didx, g.dkeys_alt, g.didx_alt, (uint64_t)P, 0, 32, g.sort, g.status, s);
  stage_end(kStDepthSort, s);
  const uint32_t* sorted_idx = depth_alt ? g.didx_alt : g.didx;
  if ((rc = check(s, debug, "depth sort", g.status))) return rc;
  stage_begin(kStOffsets, s);
  launch_offsets_scan(sc, g, sorted_idx, s);
  stage_end(kStOffsets, s);
  cudaError_t e = begin_status_read(g.status, s);
  if (e != cudaSuccess) return cuda_fail(e, "overlap count readback");
  // The feature stage depends only on preprocess: queue it before blocking on
  // the overlap count so the GPU works while the host waits.
  stage_begin(kStFeatures, s);
  if (g.table_lm) {
    launch_table_to_level_major(sc.table, g.table_lm, sc.T, sc.L, sc.F, s);
    sc.table = g.table_lm;
    sc.tab_l = (size_t)sc.T * sc.F;
    sc.tab_e = (uint32_t)sc.F;
  }
  launch_features(sc, g, s);
  stage_end(kStFeatures, s);
  if ((rc = check(s, debug, "features", g.status))) return rc;
  uint32_t words[4];
  e = finish_status_read(words);
  if (e != cudaSuccess) return cuda_fail(e, "overlap count readback");
  const uint32_t st0 = words[0];
  const uint64_t R = (uint64_t)words[2] | ((uint64_t)words[3] << 32);
  if (st0) return fail(VI_ERR_DEVICE, "device status 0x%x after binning", st0);
  if (R >= (1ull << 30)) return fail(VI_ERR_TOO_MANY_OVERLAPS, "%llu overlaps exceed 2^30", (unsigned long long)R);

  const int tb = tile_bits(tiles);
  BinState b = bin_layout(nullptr, R, tb);
  char* bb = binning_buffer(binning_user, b.bytes);
  if (!bb) return fail(VI_ERR_ALLOC, "binning buffer of %zu bytes", b.bytes);
  if ((uintptr_t)bb & 255) return fail(VI_ERR_INVALID_ARGUMENT, "state buffers must be 256-byte aligned");
  b = bin_layout(bb, R, tb);
  const uint32_t* point_list = b.tvals;
  const uint32_t* sorted_tiles = b.tkeys;
  stage_begin(kStBinning, s);
  if (R > 0) {
    launch_duplicate(sc, g, sorted_idx, b, s);
    if ((rc = check(s, debug, "duplicate", g.status))) return rc;
    const bool alt = onesweep_sort_u32(b.tkeys, b.tvals, b.tkeys_alt, b.tvals_alt, R, 0, tb, b.sort, g.status, s);
    point_list = alt ? b.tvals_alt : b.tvals;
    sorted_tiles = alt ? b.tkeys_alt : b.tkeys;
    if ((rc = check(s, debug, "tile sort", g.status))) return rc;
  }
  launch_ranges(R, sorted_tiles, im.ranges, tiles, s);
  stage_end(kStBinning, s);
  stage_begin(kStRender, s);
  launch_render(sc, g, point_list, im, out_color, out_features, visibility_info, s);
  stage_end(kStRender, s);
  if ((rc = check(s, debug, "render", g.status))) return rc;
  *num_rendered = (int)R;
  return VI_OK;
}

int backward_impl(
    float* dL_dmeans3D, float* dL_dconfidences, float* dL_dfeature_table, float* dL_dlinear_weights,
    float* dL_dlinear_bias, const float* dL_dout_color, const float* dL_dout_features, char* geom_buffer,
    char* binning_buffer, char* img_buffer, const float* means3D, const float* primitive_confidences,
    float primitive_scale, const float* viewmatrix, const float* projmatrix, const float* cam_pos, float tan_fovx,
    float tan_fovy, int image_height, int image_width, float near_plane, float max_distance,
    const float* feature_table, const int* resolution, const int* do_hash, const int* primes, int feature_offset,
    const float* linear_weights, const float* linear_bias, int stencil_genus, int grid_size,
    int max_primitives_per_ray, float occupancy_threshold, const float* bg_color, unsigned input_feature_dim,
    unsigned output_feature_dim, unsigned hashgrid_levels, unsigned num_output_channels,
    uint64_t feature_table_size, int P, int num_rendered, int debug, void* stream, const float* hash_bounds,
    unsigned flags, const float* dL_dvisibility) {
  (void)cam_pos;
  (void)occupancy_threshold;
  cudaStream_t s = (cudaStream_t)stream;
  Scene sc;
  int rc = make_scene(sc, P, means3D, primitive_confidences, primitive_scale, viewmatrix, projmatrix, tan_fovx,
                      tan_fovy, image_height, image_width, near_plane, max_distance, feature_table, resolution,
                      do_hash, primes, feature_offset, linear_weights, linear_bias, stencil_genus, grid_size,
                      max_primitives_per_ray, bg_color, input_feature_dim, output_feature_dim, hashgrid_levels,
                      num_output_channels, hash_bounds);
  if (rc) return rc;
  if (flags & ~VI_FLAG_EXACT_GRADIENTS) return fail(VI_ERR_INVALID_ARGUMENT, "unknown flags 0x%x", flags);
  sc.exact = (flags & VI_FLAG_EXACT_GRADIENTS) != 0;
  if (sc.exact && sc.V > 32)
    return fail(VI_ERR_UNSUPPORTED, "exact_gradients needs grid_size <= 3 (got %d)", grid_size);
  if (feature_table_size < (uint64_t)sc.T * sc.L * sc.F)
    return fail(VI_ERR_INVALID_ARGUMENT, "feature_table_size=%llu < feature_offset*L*F", (unsigned long long)feature_table_size);
  // Zeroed outputs (integrator_impl.cu:573-577).
  if (P > 0) {
    cudaMemsetAsync(dL_dmeans3D, 0, (size_t)P * 3 * sizeof(float), s);
    cudaMemsetAsync(dL_dconfidences, 0, (size_t)P * sc.V * sizeof(float), s);
  }
  cudaMemsetAsync(dL_dfeature_table, 0, feature_table_size * sizeof(float), s);
  cudaMemsetAsync(dL_dlinear_weights, 0, (size_t)sc.O * sc.D * sizeof(float), s);
  cudaMemsetAsync(dL_dlinear_bias, 0, (size_t)sc.O * sizeof(float), s);
  const size_t N = (size_t)sc.W * sc.H;
  if (num_rendered <= 0 || P == 0 || N == 0) return check(s, debug, "empty backward", nullptr);
  if (!geom_buffer || !img_buffer) return fail(VI_ERR_INVALID_ARGUMENT, "forward state buffers are required");
  if (((uintptr_t)geom_buffer & 255) || ((uintptr_t)img_buffer & 255))
    return fail(VI_ERR_INVALID_ARGUMENT, "state buffers must be 256-byte aligned");
  if (((uintptr_t)feature_table) % (size_t)(sc.F >= 4 ? 16 : sc.F * 4) != 0 ||
      ((uintptr_t)dL_dfeature_table) % (size_t)(sc.F >= 4 ? 16 : sc.F * 4) != 0)
    return fail(VI_ERR_INVALID_ARGUMENT, "feature_table and its gradient must be aligned to one entry's vector");
  GeomState g = geom_layout(geom_buffer, P, sc.V, sc.O, sc.D, 0);  // the caller's table: no level-major copy
  ImgState im = img_layout(img_buffer, N, sc.K, (size_t)sc.gx * sc.gy, sc.exact);
  const uint32_t* point_list = nullptr;
  if (sc.exact) {
    // the list index of a composite's trigger resolves to a primitive through the point list
    if (!binning_buffer) return fail(VI_ERR_INVALID_ARGUMENT, "the exact-gradient backward needs the binning buffer");
    const int tb = tile_bits((size_t)sc.gx * sc.gy);
    BinState b = bin_layout(binning_buffer, (uint64_t)num_rendered, tb);
    // The tile sort runs ceil(bits/8) passes; an odd count leaves the result in the alternate arrays.
    const bool alt = num_rendered > 1 && (((tb + 7) / 8) & 1);
    point_list = alt ? b.tvals_alt : b.tvals;
  }
  launch_backward(sc, g, im, point_list, dL_dout_color, sc.Fout ? dL_dout_features : nullptr, dL_dvisibility,
                  dL_dmeans3D, dL_dconfidences, dL_dfeature_table, dL_dlinear_weights, dL_dlinear_bias, s);
  return check(s, debug, "backward", g.status);
}

}  // namespace

extern "C" int vi_integrate_primitives(
    vi_resize_fn geom_buffer, void* geom_user, vi_resize_fn binning_buffer, void* binning_user,
    vi_resize_fn img_buffer, void* img_user, float* out_color, float* out_features, float* visibility_info,
    int* num_rendered, int P, const float* means3D, const float* primitive_confidences, float primitive_scale,
    const float* viewmatrix, const float* projmatrix, const float* cam_pos, float tan_fovx, float tan_fovy,
    int image_height, int image_width, float near_plane, float max_distance, const float* feature_table,
    uint64_t feature_table_numel, const int* resolution, const int* do_hash, const int* primes, int feature_offset,
    const float* linear_weights, uint64_t linear_weights_numel, const float* linear_bias,
    uint64_t linear_bias_numel, int stencil_genus, int grid_size, int max_primitives_per_ray,
    float occupancy_threshold, const float* bg_color, unsigned input_feature_dim, unsigned output_feature_dim,
    unsigned intermediate_feature_dim, unsigned hashgrid_levels, unsigned num_output_channels, int debug,
    void* stream) {
  return forward_impl(geom_buffer, geom_user, binning_buffer, binning_user, img_buffer, img_user, out_color, out_features,
                      visibility_info, num_rendered, P, means3D, primitive_confidences, primitive_scale, viewmatrix,
                      projmatrix, cam_pos, tan_fovx, tan_fovy, image_height, image_width, near_plane, max_distance,
                      feature_table, feature_table_numel, resolution, do_hash, primes, feature_offset, linear_weights,
                      linear_weights_numel, linear_bias, linear_bias_numel, stencil_genus, grid_size,
                      max_primitives_per_ray, occupancy_threshold, bg_color, input_feature_dim, output_feature_dim,
                      intermediate_feature_dim, hashgrid_levels, num_output_channels, debug, stream, nullptr, 0u);
}

extern "C" int vi_integrate_primitives_ex(
    vi_resize_fn geom_buffer, void* geom_user, vi_resize_fn binning_buffer, void* binning_user,
    vi_resize_fn img_buffer, void* img_user, float* out_color, float* out_features, float* visibility_info,
    int* num_rendered, int P, const float* means3D, const float* primitive_confidences, float primitive_scale,
    const float* viewmatrix, const float* projmatrix, const float* cam_pos, float tan_fovx, float tan_fovy,
    int image_height, int image_width, float near_plane, float max_distance, const float* feature_table,
    uint64_t feature_table_numel, const int* resolution, const int* do_hash, const int* primes, int feature_offset,
    const float* linear_weights, uint64_t linear_weights_numel, const float* linear_bias,
    uint64_t linear_bias_numel, int stencil_genus, int grid_size, int max_primitives_per_ray,
    float occupancy_threshold, const float* bg_color, unsigned input_feature_dim, unsigned output_feature_dim,
    unsigned intermediate_feature_dim, unsigned hashgrid_levels, unsigned num_output_channels, int debug,
    void* stream, const float* hash_bounds, unsigned flags) {
  return forward_impl(geom_buffer, geom_user, binning_buffer, binning_user, img_buffer, img_user, out_color, out_features,
                      visibility_info, num_rendered, P, means3D, primitive_confidences, primitive_scale, viewmatrix,
                      projmatrix, cam_pos, tan_fovx, tan_fovy, image_height, image_width, near_plane, max_distance,
                      feature_table, feature_table_numel, resolution, do_hash, primes, feature_offset, linear_weights,
                      linear_weights_numel, linear_bias, linear_bias_numel, stencil_genus, grid_size,
                      max_primitives_per_ray, occupancy_threshold, bg_color, input_feature_dim, output_feature_dim,
                      intermediate_feature_dim, hashgrid_levels, num_output_channels, debug, stream, hash_bounds,
                      flags);
}

extern "C" int vi_integrate_primitives_backward(
    float* dL_dmeans3D, float* dL_dconfidences, float* dL_dfeature_table, float* dL_dlinear_weights,
    float* dL_dlinear_bias, const float* dL_dout_color, const float* dL_dout_features, char* geom_buffer,
    char* binning_buffer, char* img_buffer, const float* means3D, const float* primitive_confidences,
    float primitive_scale, const float* viewmatrix, const float* projmatrix, const float* cam_pos, float tan_fovx,
    float tan_fovy, int image_height, int image_width, float near_plane, float max_distance,
    const float* feature_table, const int* resolution, const int* do_hash, const int* primes, int feature_offset,
    const float* linear_weights, const float* linear_bias, int stencil_genus, int grid_size,
    int max_primitives_per_ray, float occupancy_threshold, const float* bg_color, unsigned input_feature_dim,
    unsigned output_feature_dim, unsigned hashgrid_levels, unsigned num_output_channels,
    uint64_t feature_table_size, int P, int num_rendered, int debug, void* stream) {
  return backward_impl(dL_dmeans3D, dL_dconfidences, dL_dfeature_table, dL_dlinear_weights, dL_dlinear_bias,
                       dL_dout_color, dL_dout_features, geom_buffer, binning_buffer, img_buffer, means3D,
                       primitive_confidences, primitive_scale, viewmatrix, projmatrix, cam_pos, tan_fovx, tan_fovy,
                       image_height, image_width, near_plane, max_distance, feature_table, resolution, do_hash,
                       primes, feature_offset, linear_weights, linear_bias, stencil_genus, grid_size,
                       max_primitives_per_ray, occupancy_threshold, bg_color, input_feature_dim, output_feature_dim,
                       hashgrid_levels, num_output_channels, feature_table_size, P, num_rendered, debug, stream, nullptr,
                       0u, nullptr);
}

extern "C" int vi_integrate_primitives_backward_ex(
    float* dL_dmeans3D, float* dL_dconfidences, float* dL_dfeature_table, float* dL_dlinear_weights,
    float* dL_dlinear_bias, const float* dL_dout_color, const float* dL_dout_features, char* geom_buffer,
    char* binning_buffer, char* img_buffer, const float* means3D, const float* primitive_confidences,
    float primitive_scale, const float* viewmatrix, const float* projmatrix, const float* cam_pos, float tan_fovx,
    float tan_fovy, int image_height, int image_width, float near_plane, float max_distance,
    const float* feature_table, const int* resolution, const int* do_hash, const int* primes, int feature_offset,
    const float* linear_weights, const float* linear_bias, int stencil_genus, int grid_size,
    int max_primitives_per_ray, float occupancy_threshold, const float* bg_color, unsigned input_feature_dim,
    unsigned output_feature_dim, unsigned hashgrid_levels, unsigned num_output_channels,
    uint64_t feature_table_size, int P, int num_rendered, int debug, void* stream, const float* hash_bounds,
    unsigned flags, const float* dL_dvisibility) {
  return backward_impl(dL_dmeans3D, dL_dconfidences, dL_dfeature_table, dL_dlinear_weights, dL_dlinear_bias,
                       dL_dout_color, dL_dout_features, geom_buffer, binning_buffer, img_buffer, means3D,
                       primitive_confidences, primitive_scale, viewmatrix, projmatrix, cam_pos, tan_fovx, tan_fovy,
                       image_height, image_width, near_plane, max_distance, feature_table, resolution, do_hash,
                       primes, feature_offset, linear_weights, linear_bias, stencil_genus, grid_size,
                       max_primitives_per_ray, occupancy_threshold, bg_color, input_feature_dim, output_feature_dim,
                       hashgrid_levels, num_output_channels, feature_table_size, P, num_rendered, debug, stream, hash_bounds,
                       flags, dL_dvisibility);
}

extern "C" int vi_mark_visible(int P, const float* means3D, const float* viewmatrix, const float* projmatrix,
                               uint8_t* present, void* stream) {
  (void)projmatrix;
  if (P < 0) return fail(VI_ERR_INVALID_ARGUMENT, "P=%d", P);
  launch_mark_visible(P, means3D, viewmatrix, (bool*)present, (cudaStream_t)stream);
  return check((cudaStream_t)stream, 0, "mark_visible", nullptr);
}

extern "C" size_t vi_sort_pairs_temp_bytes(uint64_t n, int begin_bit, int end_bit) {
  return sort_temp_bytes(n, 8, begin_bit, end_bit) + 512;
}

// Shared body of vi_sort_pairs and its withheld-tile testing hook.
static int sort_pairs_impl(uint64_t* keys_in, uint32_t* vals_in, uint64_t* keys_out, uint32_t* vals_out, uint64_t n,
                           int begin_bit, int end_bit, void* temp, size_t temp_bytes, int spin_limit, bool withheld,
                           uint32_t* device_status, cudaStream_t s) {
  if (device_status) *device_status = 0;
  if (n >= (1ull << 30)) return fail(VI_ERR_INVALID_ARGUMENT, "n=%llu must be < 2^30", (unsigned long long)n);
  if (begin_bit < 0 || end_bit > 64 || begin_bit > end_bit) return fail(VI_ERR_INVALID_ARGUMENT, "bit range [%d,%d)", begin_bit, end_bit);
  if (temp_bytes < vi_sort_pairs_temp_bytes(n, begin_bit, end_bit)) return fail(VI_ERR_INVALID_ARGUMENT, "temp too small");
  if (n == 0) return VI_OK;
  char* t = (char*)(((uintptr_t)temp + 255) / 256 * 256);
  uint32_t* status = (uint32_t*)t;  // first 256 bytes
  SortTemp st;
  sort_temp_carve(t + 256, n, 8, begin_bit, end_bit, st);
  if (withheld && st.tiles < 2)
    return fail(VI_ERR_INVALID_ARGUMENT, "withheld-tile sort needs at least two tiles (n=%llu)", (unsigned long long)n);
  cudaMemsetAsync(status, 0, 4, s);
  const bool alt = withheld ? onesweep_sort_u64_withheld(keys_in, vals_in, keys_out, vals_out, n, begin_bit, end_bit, st,
                                                         status, spin_limit, s)
                            : onesweep_sort_u64(keys_in, vals_in, keys_out, vals_out, n, begin_bit, end_bit, st, status, s);
  if (!alt) {
    cudaMemcpyAsync(keys_out, keys_in, n * 8, cudaMemcpyDeviceToDevice, s);
    cudaMemcpyAsync(vals_out, vals_in, n * 4, cudaMemcpyDeviceToDevice, s);
  }
  int rc = check(s, 0, "sort_pairs", nullptr);
  if (rc) return rc;
  return read_sort_status(status, device_status, s, "sort_pairs");
}

extern "C" int vi_sort_pairs(uint64_t* keys_in, uint32_t* vals_in, uint64_t* keys_out, uint32_t* vals_out, uint64_t n,
                             int begin_bit, int end_bit, void* temp, size_t temp_bytes, void* stream) {
  return sort_pairs_impl(keys_in, vals_in, keys_out, vals_out, n, begin_bit, end_bit, temp, temp_bytes, 1 << 20, false,
                         nullptr, (cudaStream_t)stream);
}

extern "C" int vi_sort_pairs_withheld_tile(uint64_t* keys_in, uint32_t* vals_in, uint64_t* keys_out, uint32_t* vals_out,
                                           uint64_t n, int begin_bit, int end_bit, void* temp, size_t temp_bytes,
                                           int spin_limit, uint32_t* device_status, void* stream) {
  if (spin_limit < 1 || spin_limit > (1 << 20)) return fail(VI_ERR_INVALID_ARGUMENT, "spin_limit=%d outside [1, 2^20]", spin_limit);
  return sort_pairs_impl(keys_in, vals_in, keys_out, vals_out, n, begin_bit, end_bit, temp, temp_bytes, spin_limit, true,
                         device_status, (cudaStream_t)stream);
}

extern "C" int vi_get_state_layout(int P, int64_t num_rendered, int image_height, int image_width,
                                   int max_primitives_per_ray, int grid_size, unsigned output_feature_dim,
                                   vi_state_layout* out) {
  if (!out || P < 0 || num_rendered < 0 || grid_size < 1) return fail(VI_ERR_INVALID_ARGUMENT, "bad layout query");
  const int V = grid_size * grid_size * grid_size, O = (int)output_feature_dim + 4;
  const size_t N = (size_t)image_width * image_height;
  const size_t tiles = (size_t)((image_width + 15) / 16) * ((image_height + 15) / 16);
  GeomState g = geom_layout(nullptr, P, V, O, 0, 0);
  const int tb = tile_bits(tiles);
  BinState b = bin_layout(nullptr, (uint64_t)num_rendered, tb);
  ImgState m = img_layout(nullptr, N, max_primitives_per_ray, tiles, false);
  out->geom_bytes = g.bytes;
  out->binning_bytes = b.bytes;
  out->img_bytes = m.bytes;
  out->status = (size_t)g.status;
  out->depths = (size_t)g.depths;
  out->radii = (size_t)g.radii;
  out->means2D = (size_t)g.means2D;
  out->tiles_touched = (size_t)g.tiles_touched;
  out->rec_cnt = (size_t)g.rec_cnt;
  out->rec_key = (size_t)g.rec_key;
  out->rec_props = (size_t)g.rec_props;
  out->props_stride = props_stride(O);
  // The tile sort runs ceil(bits/8) passes; an odd count leaves the result in the alternate arrays.
  const bool alt = num_rendered > 1 && (((tb + 7) / 8) & 1);
  out->sorted_tiles = (size_t)(alt ? b.tkeys_alt : b.tkeys);
  out->point_list = (size_t)(alt ? b.tvals_alt : b.tvals);
  out->ranges = (size_t)m.ranges;
  out->final_T = (size_t)m.final_T;
  out->n_contrib = (size_t)m.n_contrib;
  out->contrib_idx = (size_t)m.contrib_idx;
  out->delta_t = (size_t)m.delta_t;
  out->contrib_rec = (size_t)m.contrib_rec;
  return VI_OK;
}

extern "C" int vi_read_device_status(const char* geom_buffer, uint32_t* status, void* stream) {
  GeomState g = geom_layout((char*)geom_buffer, 0, 1, 4, 0, 0);
  cudaError_t e = cudaMemcpyAsync(status, g.status, 4, cudaMemcpyDeviceToHost, (cudaStream_t)stream);
  if (e == cudaSuccess) e = cudaStreamSynchronize((cudaStream_t)stream);
  return e == cudaSuccess ? VI_OK : cuda_fail(e, "read status");
}

extern "C" uint64_t vi_kernel_launches(void) { return g_launch_count.load(); }

extern "C" int vi_profile_enable(int on) {
  std::lock_guard<std::mutex> lk(g_prof_mu);
  g_prof_on = on != 0;
  return VI_OK;
}

extern "C" int vi_profile_read(double* ms, uint64_t* calls, int n, int reset) {
  std::lock_guard<std::mutex> lk(g_prof_mu);
  for (auto& p : g_prof_pending) {
    cudaError_t e = cudaEventSynchronize(p.b);
    if (e != cudaSuccess) return cuda_fail(e, "profile read");
    float t = 0.0f;
    cudaEventElapsedTime(&t, p.a, p.b);
    g_prof_ms[p.stage] += t;
    g_prof_calls[p.stage] += 1;
    g_prof_free.push_back(p.a);
    g_prof_free.push_back(p.b);
  }
  g_prof_pending.clear();
  for (int i = 0; i < n && i < kStCount; i++) {
    if (ms) ms[i] = g_prof_ms[i];
    if (calls) calls[i] = g_prof_calls[i];
  }
  if (reset)
    for (int i = 0; i < kStCount; i++) {
      g_prof_ms[i] = 0.0;
      g_prof_calls[i] = 0;
    }
  return VI_OK;
}
