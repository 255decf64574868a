/*
 * C ABI of the B200 volume-integration renderer (libvi_b200.so).
 *
 * Plain pointers and sizes only; every pointer argument is CUDA device memory
 * unless stated otherwise, and every call is asynchronous on `stream` (a
 * cudaStream_t; NULL = legacy default stream) except where noted.  Each entry
 * point returns a vi_status code; vi_last_error() gives a message for the
 * calling thread's last failure.
 *
 * The entry points replace the reference extension's pybind functions
 * (reference: ext.cpp:18-20, integrate_primitives.h:42-139) one for one, with
 * the same argument order and meaning; a torch binding with the reference's
 * exact Python signature sits on top of them (volume_integration._C).
 */
#ifndef VOLUME_INTEGRATION_B200_H
#define VOLUME_INTEGRATION_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef enum vi_status {
  VI_OK = 0,
  VI_ERR_INVALID_ARGUMENT = 1, /* a size or pointer is inconsistent */
  VI_ERR_UNSUPPORTED = 2,      /* a configuration outside what the kernels implement */
  VI_ERR_ALLOC = 3,            /* a state-buffer callback returned NULL */
  VI_ERR_CUDA = 4,             /* a CUDA runtime call failed */
  VI_ERR_TOO_MANY_OVERLAPS = 5,/* more than 2^30 tile/primitive overlaps */
  VI_ERR_DEVICE = 6            /* a kernel latched an error in the state's status word */
} vi_status;

/*
 * Bits of the device status word that kernels latch instead of trapping (a
 * bounded wait that gives up, an impossible count).  A call that reads a set bit
 * returns VI_ERR_DEVICE, and vi_last_error() names the bits.  Who reads it:
 *   - vi_integrate_primitives(_ex): always after preprocess, depth sort and the
 *     overlap scan (with the overlap count); after every later stage (tile sort,
 *     render) only when debug is set, or afterwards through vi_read_device_status;
 *   - vi_integrate_primitives_backward(_ex): only when debug is set;
 *   - vi_sort_pairs, vi_sort_pairs_noalloc: always (they wait for the sort).
 * After VI_DEVICE_LOOKBACK_TIMEOUT the sorted output of that call is unspecified.
 */
#define VI_DEVICE_LOOKBACK_TIMEOUT 0x1u /* a sort's look-back gave up after its spin limit */
#define VI_DEVICE_RECORD_OVERFLOW 0x2u  /* more records than grid points for a primitive */
#define VI_DEVICE_STAGE_TIMEOUT 0x4u    /* a render tile's bulk-copy wait gave up; it read global memory instead */

/* Grows the caller's byte buffer to at least nbytes and returns its device
 * address (reference: resizeFunctional, integrate_primitives.cu:54-68). */
typedef char* (*vi_resize_fn)(void* user, size_t nbytes);

/* Message for the calling thread's last non-VI_OK return. */
const char* vi_last_error(void);

/*
 * Forward pass.  Replaces IntegratePrimitivesCUDA
 * (reference: integrate_primitives.h:42-82, integrate_primitives.cu:74-287) and
 * Integrator::forward (cuda_integrator/integrator_impl.cu:196-469).
 *
 * Outputs (caller-allocated, overwritten): out_color [3,H,W], out_features
 * [output_feature_dim,H,W], visibility_info [H,W] (float32, CHW), and
 * *num_rendered (host int).  The three state buffers are obtained through the
 * callbacks and must be passed unchanged to the backward.  Inputs follow the
 * reference's positional order; resolution/do_hash hold hashgrid_levels
 * entries, primes 3, viewmatrix/projmatrix 16 column-major floats, bg_color 3.
 * Blocks the host once, to read the overlap count.  That count reaches the
 * host through 64 bytes of mapped pinned host memory (allocated on the calling
 * thread's first forward and kept), written by a one-warp kernel, so the wait
 * does not queue behind device-to-host copies the caller runs on other
 * streams.
 */
int vi_integrate_primitives(
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
    void* stream);

/*
 * Backward pass.  Replaces IntegratePrimitivesBackwardCUDA
 * (reference: integrate_primitives.h:86-133, integrate_primitives.cu:294-432) and
 * Integrator::backward (cuda_integrator/integrator_impl.cu:474-756).
 *
 * Gradient outputs (caller-allocated, overwritten): dL_dmeans3D [P,3] (zeros,
 * as in the reference), dL_dconfidences [P,G^3], dL_dfeature_table
 * [feature_table_size], dL_dlinear_weights [O*D], dL_dlinear_bias [O] with
 * D = hashgrid_levels*input_feature_dim, O = 3 + output_feature_dim + 1.
 * geom/binning/img are the device addresses of the forward's state buffers.
 */
int vi_integrate_primitives_backward(
    float* dL_dmeans3D, float* dL_dconfidences, float* dL_dfeature_table, float* dL_dlinear_weights,
    float* dL_dlinear_bias, const float* dL_dout_color, const float* dL_dout_features, char* geom_buffer,
    char* binning_buffer, char* img_buffer, const float* means3D, const float* primitive_confidences,
    float primitive_scale, const float* viewmatrix, const float* projmatrix, const float* cam_pos, float tan_fovx,
    float tan_fovy, int image_height, int image_width, float near_plane, float max_distance,
    const float* feature_table, const int* resolution, const int* do_hash, const int* primes, int feature_offset,
    const float* linear_weights, const float* linear_bias, int stencil_genus, int grid_size,
    int max_primitives_per_ray, float occupancy_threshold, const float* bg_color, unsigned input_feature_dim,
    unsigned output_feature_dim, unsigned hashgrid_levels, unsigned num_output_channels,
    uint64_t feature_table_size, int P, int num_rendered, int debug, void* stream);

/*
 * The two calls above with two extensions, neither with a counterpart in the
 * reference:
 *
 * hash_bounds: a hashgrid box other than the reference's fixed [-1.3, 1.3]^3
 *   (reference: hashgrid.h:23-24, :125-126, :225-226).  Scenes larger than that
 *   box clamp most positions to its faces; this lets them use their own
 *   bounds.  Host pointer to 6 floats {lo_x, lo_y, lo_z, hi_x, hi_y, hi_z}
 *   with lo < hi per axis, or NULL for the reference's box.  Positions
 *   normalise as clamp((p - lo) / (hi - lo), 0, 1).
 * flags: VI_FLAG_EXACT_GRADIENTS makes the backward the derivative of the
 *   forward (the reference's backward is not: no transmittance factor, another
 *   occupancy, no delta-t terms), including dL/dmeans3D through the depths and
 *   the hashgrid's spatial derivative, and dL/dvisibility
 *   (dL_dvisibility, [H*W] or NULL).  The forward then keeps two more arrays
 *   per contribution in the image buffer.
 *
 * The backward must get the bounds and flags the forward got.
 */
#define VI_FLAG_EXACT_GRADIENTS 1u
int vi_integrate_primitives_ex(
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
    void* stream, const float* hash_bounds, unsigned flags);
int vi_integrate_primitives_backward_ex(
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
    unsigned flags, const float* dL_dvisibility);

/* Frustum test per primitive (view-space z > 0.2).  Replaces markVisible
 * (reference: integrate_primitives.h:136-139, integrate_primitives.cu:436-462). */
int vi_mark_visible(int P, const float* means3D, const float* viewmatrix, const float* projmatrix, uint8_t* present,
                    void* stream);

/*
 * Stable radix sort of (uint64 key, uint32 value) pairs over key bits
 * [begin_bit, end_bit): the sort the reference binning step takes from
 * cub::DeviceRadixSort::SortPairs (reference:
 * cuda_integrator/integrator_impl.cu:341-349).  temp must hold
 * vi_sort_pairs_temp_bytes(n, begin_bit, end_bit) bytes; keys_in/vals_in are
 * used as scratch and are clobbered.  n < 2^30.  The kernels run on `stream`;
 * the call then blocks the host until they finish, to read the sort's status
 * word (its first 4 bytes sit 0-255 bytes into temp, at the first 256-byte
 * boundary) and returns VI_ERR_DEVICE if a look-back wait gave up
 * (VI_DEVICE_LOOKBACK_TIMEOUT).
 */
size_t vi_sort_pairs_temp_bytes(uint64_t n, int begin_bit, int end_bit);
int vi_sort_pairs(uint64_t* keys_in, uint32_t* vals_in, uint64_t* keys_out, uint32_t* vals_out, uint64_t n,
                  int begin_bit, int end_bit, void* temp, size_t temp_bytes, void* stream);

/*
 * vi_sort_pairs for callers that must not allocate device memory (hosts that own
 * every byte of device memory, or that cannot take the implicit device-wide
 * synchronisation of cudaMalloc/cudaFree mid-frame).  No counterpart in the
 * reference.  Same contract as vi_sort_pairs except that the sort's scratch lives
 * in a fixed device array of VI_SORT_NOALLOC_SCRATCH_BYTES inside libvi_b200.so
 * (held by every GPU that loads the library until the process exits), so no temp
 * buffer is passed:
 *   - n <= VI_SORT_NOALLOC_MAX_KEYS; larger n returns VI_ERR_INVALID_ARGUMENT;
 *   - keys_in/vals_in are clobbered; the sorted pairs land in keys_out/vals_out;
 *   - the first call on a device looks up the array's device address (make that
 *     first call before any stream capture) and keeps it for the process: do not
 *     call it on a device after cudaDeviceReset() there;
 *   - every call uses the same array: calls that overlap on the GPU (other
 *     streams, other threads) race and must be serialised by the caller;
 *   - like vi_sort_pairs it blocks the host until the sort ends and returns
 *     VI_ERR_DEVICE after a look-back timeout (VI_DEVICE_LOOKBACK_TIMEOUT); the
 *     status word is read with a 4-byte device-to-host copy into host stack
 *     memory.
 * Calls no cudaMalloc, cudaFree or allocating library routine.
 */
#define VI_SORT_NOALLOC_MAX_KEYS (1u << 20)
#define VI_SORT_NOALLOC_SCRATCH_BYTES (3u << 20)
int vi_sort_pairs_noalloc(uint64_t* keys_in, uint32_t* vals_in, uint64_t* keys_out, uint32_t* vals_out, uint64_t n,
                          int begin_bit, int end_bit, void* stream);

/*
 * Testing hook for the sort's bounded look-back wait; no counterpart in the
 * reference.  vi_sort_pairs with tile 0 of every digit pass withheld: one CTA
 * fewer runs and the tile counter starts at 1, so tile 1 waits for a predecessor
 * that never publishes and gives up after spin_limit polls (1 <= spin_limit <=
 * 2^20; vi_sort_pairs uses 2^20).  Every launched CTA still works on a tile that
 * exists and writes only inside keys_out/vals_out.  n must span at least two
 * tiles of 3072 keys.  Returns VI_ERR_DEVICE with *device_status (host) holding
 * VI_DEVICE_LOOKBACK_TIMEOUT; the outputs are then unspecified.
 */
int vi_sort_pairs_withheld_tile(uint64_t* keys_in, uint32_t* vals_in, uint64_t* keys_out, uint32_t* vals_out,
                                uint64_t n, int begin_bit, int end_bit, void* temp, size_t temp_bytes,
                                int spin_limit, uint32_t* device_status, void* stream);

/* Number of key bits the reference sorts on: 32 + getHigherMsb(tiles)
 * (reference: cuda_integrator/integrator_impl.cu:47-62, :341). */
int vi_sort_end_bit(uint32_t num_tiles);

/*
 * Byte offsets of the integer state inside the forward's buffers, so callers
 * (and parity tests) can read radii, the sorted point list, tile ranges and the
 * per-pixel contributor lists in the reference's formats
 * (reference: cuda_integrator/integrator_impl.h:35-146).
 */
typedef struct vi_state_layout {
  size_t geom_bytes, binning_bytes, img_bytes;
  /* geometry buffer */
  size_t status, depths, radii, means2D, tiles_touched, rec_cnt, rec_key, rec_props;
  int props_stride;
  /* binning buffer: sorted tile ids and primitive ids (the point list) */
  size_t sorted_tiles, point_list;
  /* image buffer */
  size_t ranges, final_T, n_contrib, contrib_idx, delta_t, contrib_rec;
} vi_state_layout;
int vi_get_state_layout(int P, int64_t num_rendered, int image_height, int image_width, int max_primitives_per_ray,
                        int grid_size, unsigned output_feature_dim, vi_state_layout* out);

/*
 * ---- Gaussian-attribute front end (extension) ----
 * No counterpart in the reference: its primitives are cubes of one fixed world
 * size, projected by centre and bounding radius only
 * (cuda_integrator/forward.cu:82-87, :100-102; the spherical-harmonics
 * constants of cuda_integrator/auxiliary.h:30-48 are unused).  These entry
 * points are the standard per-Gaussian front end of splatting: projection, 3D
 * and 2D covariance (EWA, with the 0.3 pixel low-pass), conic, radius and tiles
 * touched, and colour from real spherical harmonics of degree 0..3.
 *
 * Layouts (row-major, float32 unless noted): means3D, scales [P][3];
 * rotations [P][4] quaternions (r, x, y, z), 16-byte aligned; opacities [P];
 * shs [P][sh_coeffs][3] with (sh_degree+1)^2 <= sh_coeffs <= 16; viewmatrix and
 * projmatrix as the renderer's (device pointers); cam_pos_host is a HOST
 * pointer to 3 floats.  Outputs: radii [P] int32 (0 = culled), means2D [P][2],
 * depths [P] (view-space z), cov3D [P][6] (xx, xy, xz, yy, yz, zz),
 * conic_opacity [P][4] (inverse 2D covariance a, b, c and the opacity; 16-byte
 * aligned), rgb [P][3], clamped [P][3] uint8 (colour clamped at 0), and
 * tiles_touched [P] uint32.  Culled Gaussians (t.z <= near_plane, singular 2D
 * covariance or an empty tile rectangle) have every output zero.
 */
int vi_preprocess_gaussians(int P, int sh_degree, int sh_coeffs, const float* means3D, const float* scales,
                            const float* rotations, const float* opacities, const float* shs, float scale_modifier,
                            const float* viewmatrix, const float* projmatrix, const float* cam_pos_host,
                            int image_width, int image_height, float tan_fovx, float tan_fovy, float near_plane,
                            int* radii, float* means2D, float* depths, float* cov3D, float* conic_opacity, float* rgb,
                            uint8_t* clamped, uint32_t* tiles_touched, void* stream);

/*
 * Exact derivative of vi_preprocess_gaussians.  Incoming gradients: means2D
 * [P][2], depths [P] (may be NULL), cov3D [P][6], conic_opacity [P][4] (the
 * fourth component, the opacity's, is not used: it passes through to
 * opacities unchanged), rgb [P][3].  Writes dL/dmeans3D [P][3], dL/dscales
 * [P][3], dL/drotations [P][4] (16-byte aligned) and dL/dshs [P][sh_coeffs][3];
 * culled Gaussians (radii == 0) get zeros.
 */
int vi_preprocess_gaussians_backward(int P, int sh_degree, int sh_coeffs, const float* means3D, const float* scales,
                                     const float* rotations, const float* shs, float scale_modifier,
                                     const float* viewmatrix, const float* projmatrix, const float* cam_pos_host,
                                     int image_width, int image_height, float tan_fovx, float tan_fovy,
                                     float near_plane, const int* radii, const uint8_t* clamped,
                                     const float* dL_dmeans2D, const float* dL_ddepths, const float* dL_dcov3D,
                                     const float* dL_dconic_opacity, const float* dL_drgb, float* dL_dmeans3D,
                                     float* dL_dscales, float* dL_drotations, float* dL_dshs, void* stream);

/*
 * Tile binning of projected Gaussians: the point list sorted by (tile, depth,
 * index) and per-tile [start, end) ranges, the same result as the reference
 * renderer's duplicateWithKeys + 64-bit radix sort + identifyTileRanges
 * (cuda_integrator/integrator_impl.cu:106-178) applied to these Gaussians.
 * num_rendered must equal the sum of tiles_touched (checked after the scan,
 * which blocks the host; a mismatch is an error).  scratch is 256-byte
 * aligned device memory of vi_bin_gaussians_scratch_bytes(); point_list and
 * tile_ids (optional) hold num_rendered entries, ranges 2 * tiles.
 */
uint64_t vi_bin_gaussians_scratch_bytes(int P, uint64_t num_rendered, int image_width, int image_height);
int vi_bin_gaussians(int P, int image_width, int image_height, const int* radii, const float* means2D,
                     const float* depths, const uint32_t* tiles_touched, uint64_t num_rendered, void* scratch,
                     uint64_t scratch_bytes, uint32_t* point_list, uint32_t* tile_ids, uint32_t* ranges,
                     void* stream);

/* Reads the status word a forward latched in its geometry buffer (blocks). */
int vi_read_device_status(const char* geom_buffer, uint32_t* status, void* stream);

/* Kernels launched by this library so far (all threads, all devices). */
uint64_t vi_kernel_launches(void);

/*
 * Per-stage timing with CUDA events on the launching stream (off by default).
 * Stages, in order: 0 preprocess, 1 depth sort, 2 overlap offsets, 3 feature
 * stage, 4 binning (duplicate + tile sort + ranges), 5 render, 6 backward
 * per-pixel, 7 backward per-primitive.  vi_profile_read waits for the recorded
 * events and returns the summed milliseconds and call counts per stage.
 */
int vi_profile_enable(int on);
int vi_profile_read(double* ms, uint64_t* calls, int n, int reset);

#ifdef __cplusplus
}
#endif
#endif /* VOLUME_INTEGRATION_B200_H */
