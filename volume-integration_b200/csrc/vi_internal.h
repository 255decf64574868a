// Internal (non-exported) declarations shared by the renderer's translation units:
// the private layouts of the three state buffers and the kernel launchers.
#pragma once
#include <cstddef>
#include <cstdint>
#include <cuda_runtime.h>

namespace vi {

constexpr int kSortThreads = 256;
constexpr int kRadix = 256;

inline size_t align_up(size_t x, size_t a = 256) { return (x + a - 1) / a * a; }

// Number of kernels this library has launched (all threads), for launch accounting.
void note_launches(int n);

// Records a message for vi_last_error() and returns code.
int set_error(int code, const char* msg);

// Waits for `s`, copies the 4-byte sort status word to the host (stack memory,
// no allocation) and returns VI_ERR_DEVICE with a message when a bit is set;
// *out (may be null) receives the word.
int read_sort_status(const uint32_t* status, uint32_t* out, cudaStream_t s, const char* where);

// Bits of a tile id for `tiles` tiles (the reference's getHigherMsb).
int tile_bits(size_t tiles);

// Reads status words 0..3 back to the host without a device-to-host copy (a
// tiny copy would queue behind a caller's large read-backs in the copy engine):
// begin_status_read queues a one-warp kernel on `s` that writes them into this
// thread's mapped pinned buffer, finish_status_read waits for it and returns
// them.  One read in flight per host thread.
cudaError_t begin_status_read(const uint32_t* status, cudaStream_t s);
cudaError_t finish_status_read(uint32_t words[4]);

// Fills *attr with an access-policy window that keeps [base, base + bytes) in
// L2 (persisting hits, streaming misses) for one kernel launch and returns 1,
// or returns 0 when it is unavailable or not switched on (VI_L2_WINDOW=1).  The
// first call on a device sets this process's persisting-L2 carve-out to the
// device's maximum (a limit of the context, not a setting of the GPU).
int l2_persist_attr(const void* base, size_t bytes, cudaLaunchAttribute* attr);

// Blocks of `threads` threads and `smem` dynamic shared bytes that the current
// device holds resident at once (SM count x blocks per SM), for persistent
// grids that loop over their work.
int resident_blocks(const void* kernel, int threads, size_t smem);

// Optional per-stage CUDA-event timing on the launching stream.
enum Stage { kStPreprocess, kStDepthSort, kStOffsets, kStFeatures, kStBinning, kStRender, kStBwdPixel, kStBwdPrim,
             kStCount };
void stage_begin(Stage st, cudaStream_t s);
void stage_end(Stage st, cudaStream_t s);

// Scratch of one onesweep sort (see vi_sort.cu).
struct SortTemp {
  uint32_t* hist = nullptr;      // passes x 256 digit counts, then exclusive starts
  uint32_t* lookback = nullptr;  // passes x tiles x 256 status words
  uint32_t* counters = nullptr;  // passes tile counters
  int passes = 0;
  uint32_t tiles = 0;
};
size_t sort_temp_bytes(uint64_t n, int key_bytes, int begin_bit, int end_bit);
void sort_temp_carve(char* base, uint64_t n, int key_bytes, int begin_bit, int end_bit, SortTemp& t);

// Stable LSD radix sort of (key, value) pairs over bits [begin_bit, end_bit).
// keys/vals hold the input; alt_* are same-sized scratch.  Returns true when the
// sorted result ended up in alt_*, false when it is in keys/vals.
bool onesweep_sort_u32(uint32_t* keys, uint32_t* vals, uint32_t* alt_keys, uint32_t* alt_vals, uint64_t n,
                       int begin_bit, int end_bit, const SortTemp& t, uint32_t* status, cudaStream_t s);
bool onesweep_sort_u64(uint64_t* keys, uint32_t* vals, uint64_t* alt_keys, uint32_t* alt_vals, uint64_t n,
                       int begin_bit, int end_bit, const SortTemp& t, uint32_t* status, cudaStream_t s);
// The same sort with tile 0 of every pass withheld and look-back waits limited
// to spin_limit polls (testing the bounded wait; needs t.tiles >= 2).
bool onesweep_sort_u64_withheld(uint64_t* keys, uint32_t* vals, uint64_t* alt_keys, uint32_t* alt_vals, uint64_t n,
                                int begin_bit, int end_bit, const SortTemp& t, uint32_t* status, int spin_limit,
                                cudaStream_t s);

// ---------------------------------------------------------------------------
// Geometry state: everything sized by the primitive count P.
// ---------------------------------------------------------------------------
struct GeomState {
  uint32_t* status;          // [0] status bits, [2..3] num_rendered as u64, [4] feature-stage chunk counter, [5] backward work counter, [6] phi_cache slots used, [7] entries of differs_list
  float* depths;             // [P] view-space z of the centre
  int* radii;                // [P]
  float* means2D;            // [2P]
  uint32_t* tiles_touched;   // [P]
  uint32_t* dkeys;           // [P] depth sort keys (float bits, invisible = ~0)
  uint32_t* didx;            // [P] primitive index, sorted along with dkeys
  uint32_t* dkeys_alt;       // [P]
  uint32_t* didx_alt;        // [P]
  uint32_t* offsets;         // [P] exclusive overlap offsets in depth order
  uint32_t* block_sums;      // [scan blocks]
  uint32_t* rec_cnt;         // [P] record count | kBwdDiffers
  uint32_t* rec_key;         // [P*V] tile*256 + pixel-in-tile, grouped by tile (ascending) per primitive
  float* rec_props;          // [P*V*O] activated colour, features, density per record
  uint32_t* rec_pix;         // [P*V] pixel + 1 of a contributing record, 0 otherwise (backward)
  float* rec_dpre;           // [P*V*O] dL/d(pre-activation) per contributing record
  SortTemp sort;
  uint32_t* differs_list;    // [P] primitives with records whose backward projection differs (kBwdDiffers)
  uint32_t* cls_base;        // [P] first slot of the primitive's position classes in phi_cache, or kNoCache
  float* phi_cache;          // [phi_cap][D] hashgrid features of each position class (feature stage)
  uint32_t phi_cap;          // slots in phi_cache
  float* table_lm;           // [L][T][F] the feature stage's level-major copy of the table (forward only; else null)
  size_t bytes;
};
constexpr uint32_t kNoCache = 0xffffffffu;
// cls_base of a primitive whose grid points all clamp to box corner c: kCornerCache | c
// (its features are one of the eight box-corner vectors every block computes).
constexpr uint32_t kCornerCache = 0x80000000u;
// Upper bound of phi_cache: every position class of every primitive when that
// fits, else this many bytes (primitives that find no room gather in the
// backward).  The environment variable VI_PHI_CACHE_BYTES overrides it (0 turns
// the cache off); it is read at every call, and the backward does not need the
// value the forward used, since phi_cache is the last array the backward reads.
constexpr size_t kPhiCacheMaxBytes = 8ull << 30;
size_t phi_cache_max_bytes();
constexpr uint32_t kBwdDiffers = 0x80000000u;
constexpr int kScanBlock = 2048;
// table_floats: T*L*F when the feature stage reads a level-major copy of the
// table (the forward), else 0.  The copy is the layout's last array, so the
// backward, which does not read it, lays the buffer out with 0.
GeomState geom_layout(char* base, size_t P, int V, int O, int D, size_t table_floats);

// Whether the feature stage reads a level-major copy [L][T][F] of the caller's
// entry-major table [T][L][F] (VI_TABLE_LAYOUT=entry turns it off; read at every
// forward).  The backward reads the caller's table and scatters into the
// caller's gradient.
bool table_level_major();
void launch_table_to_level_major(const float* src, float* dst, uint32_t T, int L, int F, cudaStream_t s);

// Binning state: everything sized by the overlap count R.
struct BinState {
  uint32_t* tkeys;      // [R] tile ids
  uint32_t* tvals;      // [R] primitive ids
  uint32_t* tkeys_alt;  // [R]
  uint32_t* tvals_alt;  // [R]
  SortTemp sort;
  size_t bytes;
};
BinState bin_layout(char* base, uint64_t R, int tile_bits);

// Image state: everything sized by the pixel count N.
struct ImgState {
  uint32_t* ranges;       // [2*tiles]
  float* final_T;         // [N]
  int32_t* n_contrib;     // [N]
  int32_t* contrib_idx;   // [N*K] index into the sorted overlap list
  float* delta_t;         // [N*K]
  uint32_t* contrib_rec;  // [N*K] record slot of the contribution | kBwdDiffers of its primitive
  // Exact-gradient mode only (null otherwise):
  float* trans;           // [N*K] transmittance before the contribution
  uint32_t* trig;         // [N*K] list index of the entry whose arrival composited it, ~0 = max_distance
  size_t bytes;
};
ImgState img_layout(char* base, size_t N, int K, size_t tiles, bool exact);

// ---------------------------------------------------------------------------
// Per-call constants.
// ---------------------------------------------------------------------------
struct Scene {
  int P, W, H, G, V, D, O, L, F, Fout, K, genus;
  uint32_t T, Tmask;
  float scale, step, gof, near_plane, max_distance, focal_x, focal_y;
  const float* means;
  const float* conf;
  const float* view;
  const float* proj;
  const float* table;
  const int* res;
  const int* do_hash;
  const int* primes;
  const float* Wl;
  const float* bl;
  const float* bg;
  uint64_t table_numel;
  unsigned gx, gy;
  float hlo[3], hext[3];  // hashgrid box: lower corner and extent per axis (reference: -1.3, 2.6)
  bool exact;             // exact-gradient mode (VI_FLAG_EXACT_GRADIENTS)
  bool own_box;           // the caller set the hashgrid box (hash_bounds), else the reference's fixed box
  // Addressing of `table`: the features of (entry e, level l) start at
  // l * tab_l + e * tab_e floats.  The caller's entry-major layout (read by the
  // backward): tab_l = F, tab_e = L*F; the feature stage's level-major copy:
  // tab_l = T*F, tab_e = F.
  size_t tab_l;
  uint32_t tab_e;
};

void launch_preprocess(const Scene& sc, GeomState& g, cudaStream_t s);
void launch_offsets_scan(const Scene& sc, GeomState& g, const uint32_t* sorted_idx, cudaStream_t s);
void launch_duplicate(const Scene& sc, const GeomState& g, const uint32_t* sorted_idx, BinState& b,
                      cudaStream_t s);
void launch_ranges(uint64_t R, const uint32_t* sorted_tiles, uint32_t* ranges, size_t tiles, cudaStream_t s);
void launch_mark_visible(int P, const float* means, const float* view, bool* present, cudaStream_t s);
// Status words 0..3 into mapped pinned host memory (host_mapped: its device address).
void launch_publish_status(const uint32_t* status, uint32_t* host_mapped, cudaStream_t s);
void launch_features(const Scene& sc, GeomState& g, cudaStream_t s);
void launch_render(const Scene& sc, const GeomState& g, const uint32_t* point_list, ImgState& im,
                   float* out_color, float* out_feat, float* vis, cudaStream_t s);
void launch_backward(const Scene& sc, GeomState& g, const ImgState& im, const uint32_t* point_list,
                     const float* dL_dcolor, const float* dL_dfeat, const float* dL_dvis, float* dmeans, float* dconf,
                     float* dtable, float* dW, float* db, cudaStream_t s);

}  // namespace vi
