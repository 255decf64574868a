// torch binding `volume_integration._C`: the reference's three functions with
// their exact positional signatures (reference ext.cpp:16-20,
// integrate_primitives.h:42-139), forwarded to the C ABI of libvi_b200.so.
// Tensors become device pointers; state buffers are uint8 tensors grown by a
// resize callback, as the reference's resizeFunctional does
// (integrate_primitives.cu:54-68).  Errors raise RuntimeError.
#include <c10/cuda/CUDAGuard.h>
#include <c10/cuda/CUDAStream.h>
#include <torch/extension.h>

#include <tuple>
#include <vector>

#include "volume_integration_b200.h"

namespace {

using torch::Tensor;

char* resize_cb(void* user, size_t n) {
  auto* t = static_cast<Tensor*>(user);
  t->resize_({(int64_t)n});
  return reinterpret_cast<char*>(t->data_ptr());
}

Tensor cuda_f32(const Tensor& t, const char* name) {
  TORCH_CHECK(t.is_cuda(), name, " must be a CUDA tensor");
  return t.to(torch::kFloat32).contiguous();
}
// The kernels load one table entry's features as one vector: realign views with an odd offset.
Tensor aligned_table(const Tensor& t) {
  Tensor c = cuda_f32(t, "feature_table");
  if (reinterpret_cast<uintptr_t>(c.data_ptr()) % 16 != 0) c = c.clone();
  return c;
}
Tensor cuda_i32(const Tensor& t, const char* name) {
  TORCH_CHECK(t.is_cuda(), name, " must be a CUDA tensor");
  return t.to(torch::kInt32).contiguous();
}
void ok(int rc) { TORCH_CHECK(rc == VI_OK, "volume_integration: ", vi_last_error(), " (status ", rc, ")"); }

// Hashgrid box {lo_x, lo_y, lo_z, hi_x, hi_y, hi_z}; empty = the reference's fixed box.
const float* bounds_ptr(const std::vector<double>& hb, float* buf) {
  if (hb.empty()) return nullptr;
  TORCH_CHECK(hb.size() == 6, "hash_bounds needs 6 values (lo xyz, hi xyz), got ", hb.size());
  for (int i = 0; i < 6; i++) buf[i] = (float)hb[i];
  return buf;
}

std::tuple<int, Tensor, Tensor, Tensor, Tensor, Tensor, Tensor> integrate_primitives_ex(
    const Tensor& means3D, const Tensor& primitive_confidences, const double primitive_scale,
    const Tensor& viewmatrix, const Tensor& projmatrix, const Tensor& cam_pos, const double tan_fovx,
    const double tan_fovy, const int64_t image_height, const int64_t image_width, const double near_plane,
    const double max_distance, const Tensor& feature_table, const Tensor& resolution, const Tensor& do_hash,
    const Tensor& primes, const int64_t feature_offset, const Tensor& linear_weights, const Tensor& linear_bias,
    const int64_t stencil_genus, const int64_t grid_size, const int64_t max_primitives_per_ray,
    const double occupancy_threshold, const Tensor& bg_color, const int64_t input_feature_dim,
    const int64_t output_feature_dim, const int64_t intermediate_feature_dim, const int64_t hashgrid_levels,
    const int64_t num_output_channels, const bool debug, const std::vector<double>& hash_bounds, const int64_t flags) {
  TORCH_CHECK(means3D.dim() == 2 && means3D.size(1) == 3, "means3D must have shape (P, 3)");
  float hb[6];
  const at::cuda::CUDAGuard guard(means3D.device());
  const int P = (int)means3D.size(0), H = (int)image_height, W = (int)image_width;
  Tensor m = cuda_f32(means3D, "means3D"), c = cuda_f32(primitive_confidences, "primitive_confidences");
  Tensor vm = cuda_f32(viewmatrix, "viewmatrix"), pm = cuda_f32(projmatrix, "projmatrix");
  Tensor cp = cuda_f32(cam_pos, "cam_pos"), ft = aligned_table(feature_table);
  Tensor rs = cuda_i32(resolution, "resolution"), dh = cuda_i32(do_hash, "do_hash"), pr = cuda_i32(primes, "primes");
  Tensor lw = cuda_f32(linear_weights, "linear_weights"), lb = cuda_f32(linear_bias, "linear_bias");
  Tensor bg = cuda_f32(bg_color, "bg_color");
  TORCH_CHECK(vm.numel() >= 16 && pm.numel() >= 16, "viewmatrix/projmatrix need 16 elements");
  TORCH_CHECK(rs.numel() >= hashgrid_levels && dh.numel() >= hashgrid_levels, "resolution/do_hash need L entries");
  TORCH_CHECK(pr.numel() >= 3 && bg.numel() >= 3, "primes and bg_color need 3 entries");
  TORCH_CHECK(c.numel() == (int64_t)P * grid_size * grid_size * grid_size, "primitive_confidences must be (P, G^3)");
  auto fo = m.options();
  Tensor out_color = torch::empty({(int64_t)num_output_channels, H, W}, fo);
  Tensor out_features = torch::empty({output_feature_dim, H, W}, fo);
  Tensor visibility = torch::empty({H, W}, fo);
  auto bo = fo.dtype(torch::kUInt8);
  Tensor geom = torch::empty({0}, bo), binning = torch::empty({0}, bo), img = torch::empty({0}, bo);
  int num_rendered = 0;
  ok(vi_integrate_primitives_ex(
      resize_cb, &geom, resize_cb, &binning, resize_cb, &img, out_color.data_ptr<float>(),
      out_features.data_ptr<float>(), visibility.data_ptr<float>(), &num_rendered, P, m.data_ptr<float>(),
      c.data_ptr<float>(), (float)primitive_scale, vm.data_ptr<float>(), pm.data_ptr<float>(), cp.data_ptr<float>(),
      (float)tan_fovx, (float)tan_fovy, H, W, (float)near_plane, (float)max_distance, ft.data_ptr<float>(),
      (uint64_t)ft.numel(), rs.data_ptr<int>(), dh.data_ptr<int>(), pr.data_ptr<int>(), (int)feature_offset,
      lw.data_ptr<float>(), (uint64_t)lw.numel(), lb.data_ptr<float>(), (uint64_t)lb.numel(), (int)stencil_genus,
      (int)grid_size, (int)max_primitives_per_ray, (float)occupancy_threshold, bg.data_ptr<float>(),
      (unsigned)input_feature_dim, (unsigned)output_feature_dim, (unsigned)intermediate_feature_dim,
      (unsigned)hashgrid_levels, (unsigned)num_output_channels, debug ? 1 : 0,
      at::cuda::getCurrentCUDAStream().stream(), bounds_ptr(hash_bounds, hb), (unsigned)flags));
  return {num_rendered, out_color, out_features, visibility, geom, binning, img};
}

// The reference's 30-argument signature (integrate_primitives.h:42-62).
std::tuple<int, Tensor, Tensor, Tensor, Tensor, Tensor, Tensor> integrate_primitives(
    const Tensor& means3D, const Tensor& primitive_confidences, const double primitive_scale,
    const Tensor& viewmatrix, const Tensor& projmatrix, const Tensor& cam_pos, const double tan_fovx,
    const double tan_fovy, const int64_t image_height, const int64_t image_width, const double near_plane,
    const double max_distance, const Tensor& feature_table, const Tensor& resolution, const Tensor& do_hash,
    const Tensor& primes, const int64_t feature_offset, const Tensor& linear_weights, const Tensor& linear_bias,
    const int64_t stencil_genus, const int64_t grid_size, const int64_t max_primitives_per_ray,
    const double occupancy_threshold, const Tensor& bg_color, const int64_t input_feature_dim,
    const int64_t output_feature_dim, const int64_t intermediate_feature_dim, const int64_t hashgrid_levels,
    const int64_t num_output_channels, const bool debug) {
  return integrate_primitives_ex(means3D, primitive_confidences, primitive_scale, viewmatrix, projmatrix, cam_pos,
                                 tan_fovx, tan_fovy, image_height, image_width, near_plane, max_distance,
                                 feature_table, resolution, do_hash, primes, feature_offset, linear_weights,
                                 linear_bias, stencil_genus, grid_size, max_primitives_per_ray, occupancy_threshold,
                                 bg_color, input_feature_dim, output_feature_dim, intermediate_feature_dim,
                                 hashgrid_levels, num_output_channels, debug, {}, 0);
}

std::tuple<Tensor, Tensor, Tensor, Tensor, Tensor> integrate_primitives_backward_ex(
    const Tensor& dL_dout_color, const Tensor& dL_dout_features, const Tensor& geomBuffer,
    const Tensor& binningBuffer, const Tensor& imgBuffer, const Tensor& means3D, const Tensor& primitive_confidences,
    const double primitive_scale, const Tensor& viewmatrix, const Tensor& projmatrix, const Tensor& cam_pos,
    const double tan_fovx, const double tan_fovy, const int64_t image_height, const int64_t image_width,
    const double near_plane, const double max_distance, const Tensor& feature_table, const Tensor& resolution,
    const Tensor& do_hash, const Tensor& primes, const int64_t feature_offset, const Tensor& linear_weights,
    const Tensor& linear_bias, const int64_t stencil_genus, const int64_t grid_size,
    const int64_t max_primitives_per_ray, const double occupancy_threshold, const Tensor& bg_color,
    const int64_t input_feature_dim, const int64_t output_feature_dim, const int64_t hashgrid_levels,
    const int64_t num_output_channels, const int64_t feature_table_size, const int64_t P, const int64_t num_rendered,
    const bool debug, const std::vector<double>& hash_bounds, const int64_t flags, const Tensor& dL_dvisibility) {
  const at::cuda::CUDAGuard guard(means3D.device());
  float hb[6];
  Tensor gv = dL_dvisibility.numel() ? cuda_f32(dL_dvisibility, "dL_dvisibility") : dL_dvisibility;
  TORCH_CHECK(!gv.numel() || gv.numel() == image_height * image_width, "dL_dvisibility must be (H, W)");
  Tensor m = cuda_f32(means3D, "means3D"), c = cuda_f32(primitive_confidences, "primitive_confidences");
  Tensor vm = cuda_f32(viewmatrix, "viewmatrix"), pm = cuda_f32(projmatrix, "projmatrix");
  Tensor cp = cuda_f32(cam_pos, "cam_pos"), ft = aligned_table(feature_table);
  Tensor rs = cuda_i32(resolution, "resolution"), dh = cuda_i32(do_hash, "do_hash"), pr = cuda_i32(primes, "primes");
  Tensor lw = cuda_f32(linear_weights, "linear_weights"), lb = cuda_f32(linear_bias, "linear_bias");
  Tensor bg = cuda_f32(bg_color, "bg_color");
  Tensor gc = cuda_f32(dL_dout_color, "dL_dout_color");
  Tensor gf = dL_dout_features.numel() ? cuda_f32(dL_dout_features, "dL_dout_features") : dL_dout_features;
  TORCH_CHECK(gc.numel() == 3 * image_height * image_width, "dL_dout_color must be (3, H, W)");
  TORCH_CHECK(gf.numel() == output_feature_dim * image_height * image_width, "dL_dout_features must be (F_out, H, W)");
  const int64_t D = hashgrid_levels * input_feature_dim, O = num_output_channels + output_feature_dim + 1;
  TORCH_CHECK(lw.numel() >= O * D && lb.numel() >= O, "linear layer needs ", O * D, " weights and ", O, " biases");
  TORCH_CHECK(c.numel() == P * grid_size * grid_size * grid_size, "primitive_confidences must be (P, G^3)");
  Tensor dmeans = torch::empty_like(m), dconf = torch::empty_like(c), dtable = torch::empty_like(ft);
  Tensor dW = torch::empty_like(lw), db = torch::empty_like(lb);
  ok(vi_integrate_primitives_backward_ex(
      dmeans.data_ptr<float>(), dconf.data_ptr<float>(), dtable.data_ptr<float>(), dW.data_ptr<float>(),
      db.data_ptr<float>(), gc.data_ptr<float>(), gf.numel() ? gf.data_ptr<float>() : nullptr,
      geomBuffer.numel() ? reinterpret_cast<char*>(geomBuffer.data_ptr()) : nullptr,
      binningBuffer.numel() ? reinterpret_cast<char*>(binningBuffer.data_ptr()) : nullptr,
      imgBuffer.numel() ? reinterpret_cast<char*>(imgBuffer.data_ptr()) : nullptr, m.data_ptr<float>(),
      c.data_ptr<float>(), (float)primitive_scale, vm.data_ptr<float>(), pm.data_ptr<float>(), cp.data_ptr<float>(),
      (float)tan_fovx, (float)tan_fovy, (int)image_height, (int)image_width, (float)near_plane, (float)max_distance,
      ft.data_ptr<float>(), rs.data_ptr<int>(), dh.data_ptr<int>(), pr.data_ptr<int>(), (int)feature_offset,
      lw.data_ptr<float>(), lb.data_ptr<float>(), (int)stencil_genus, (int)grid_size, (int)max_primitives_per_ray,
      (float)occupancy_threshold, bg.data_ptr<float>(), (unsigned)input_feature_dim, (unsigned)output_feature_dim,
      (unsigned)hashgrid_levels, (unsigned)num_output_channels, (uint64_t)feature_table_size, (int)P,
      (int)num_rendered, debug ? 1 : 0, at::cuda::getCurrentCUDAStream().stream(), bounds_ptr(hash_bounds, hb),
      (unsigned)flags, gv.numel() ? gv.data_ptr<float>() : nullptr));
  return {dmeans, dconf, dtable, dW, db};
}

// The reference's 37-argument signature (integrate_primitives.h:66-113).
std::tuple<Tensor, Tensor, Tensor, Tensor, Tensor> integrate_primitives_backward(
    const Tensor& dL_dout_color, const Tensor& dL_dout_features, const Tensor& geomBuffer,
    const Tensor& binningBuffer, const Tensor& imgBuffer, const Tensor& means3D, const Tensor& primitive_confidences,
    const double primitive_scale, const Tensor& viewmatrix, const Tensor& projmatrix, const Tensor& cam_pos,
    const double tan_fovx, const double tan_fovy, const int64_t image_height, const int64_t image_width,
    const double near_plane, const double max_distance, const Tensor& feature_table, const Tensor& resolution,
    const Tensor& do_hash, const Tensor& primes, const int64_t feature_offset, const Tensor& linear_weights,
    const Tensor& linear_bias, const int64_t stencil_genus, const int64_t grid_size,
    const int64_t max_primitives_per_ray, const double occupancy_threshold, const Tensor& bg_color,
    const int64_t input_feature_dim, const int64_t output_feature_dim, const int64_t hashgrid_levels,
    const int64_t num_output_channels, const int64_t feature_table_size, const int64_t P, const int64_t num_rendered,
    const bool debug) {
  return integrate_primitives_backward_ex(
      dL_dout_color, dL_dout_features, geomBuffer, binningBuffer, imgBuffer, means3D, primitive_confidences,
      primitive_scale, viewmatrix, projmatrix, cam_pos, tan_fovx, tan_fovy, image_height, image_width, near_plane,
      max_distance, feature_table, resolution, do_hash, primes, feature_offset, linear_weights, linear_bias,
      stencil_genus, grid_size, max_primitives_per_ray, occupancy_threshold, bg_color, input_feature_dim,
      output_feature_dim, hashgrid_levels, num_output_channels, feature_table_size, P, num_rendered, debug, {}, 0,
      Tensor());
}

Tensor mark_visible(Tensor& means3D, Tensor& viewmatrix, Tensor& projmatrix) {
  const at::cuda::CUDAGuard guard(means3D.device());
  Tensor m = cuda_f32(means3D, "means3D"), vm = cuda_f32(viewmatrix, "viewmatrix");
  Tensor pm = cuda_f32(projmatrix, "projmatrix");
  Tensor present = torch::empty({m.size(0)}, m.options().dtype(torch::kBool));
  ok(vi_mark_visible((int)m.size(0), m.data_ptr<float>(), vm.data_ptr<float>(), pm.data_ptr<float>(),
                     reinterpret_cast<uint8_t*>(present.data_ptr()), at::cuda::getCurrentCUDAStream().stream()));
  return present;
}

// Views of the integer state inside the forward's buffers, in the reference's
// formats (integrator_impl.h:35-146); used by parity tests and debugging.
py::dict state_views(const Tensor& geom, const Tensor& binning, const Tensor& img, int64_t P, int64_t R, int64_t H,
                     int64_t W, int64_t K, int64_t G, int64_t Fout) {
  vi_state_layout L;
  ok(vi_get_state_layout((int)P, R, (int)H, (int)W, (int)K, (int)G, (unsigned)Fout, &L));
  auto view = [](const Tensor& buf, size_t off, int64_t n, torch::ScalarType t) {
    int64_t sz = n * (int64_t)c10::elementSize(t);
    return buf.narrow(0, (int64_t)off, sz).view(t);
  };
  const int64_t N = H * W, tiles = ((W + 15) / 16) * ((H + 15) / 16), V = G * G * G;
  py::dict d;
  if (geom.numel()) {
    d["depths"] = view(geom, L.depths, P, torch::kFloat32);
    d["radii"] = view(geom, L.radii, P, torch::kInt32);
    d["means2D"] = view(geom, L.means2D, 2 * P, torch::kFloat32).view({P, 2});
    d["tiles_touched"] = view(geom, L.tiles_touched, P, torch::kInt32);
    d["rec_cnt"] = view(geom, L.rec_cnt, P, torch::kInt32);
    d["rec_key"] = view(geom, L.rec_key, P * V, torch::kInt32);
    d["rec_props"] = view(geom, L.rec_props, P * V * L.props_stride, torch::kFloat32);
    d["status"] = view(geom, L.status, 4, torch::kInt32);
  }
  if (binning.numel() && R > 0) {
    d["sorted_tiles"] = view(binning, L.sorted_tiles, R, torch::kInt32);
    d["point_list"] = view(binning, L.point_list, R, torch::kInt32);
  }
  if (img.numel()) {
    d["ranges"] = view(img, L.ranges, 2 * tiles, torch::kInt32).view({tiles, 2});
    d["final_T"] = view(img, L.final_T, N, torch::kFloat32);
    d["n_contrib"] = view(img, L.n_contrib, N, torch::kInt32);
    d["contrib_idx"] = view(img, L.contrib_idx, N * K, torch::kInt32);
    d["delta_t"] = view(img, L.delta_t, N * K, torch::kFloat32);
    d["contrib_rec"] = view(img, L.contrib_rec, N * K, torch::kInt32);
  }
  return d;
}

// Stable sort of int64 keys (read as uint64) with int32 values over [begin_bit, end_bit).
std::tuple<Tensor, Tensor> sort_pairs(const Tensor& keys, const Tensor& vals, int64_t begin_bit, int64_t end_bit) {
  TORCH_CHECK(keys.is_cuda() && keys.scalar_type() == torch::kInt64, "keys must be CUDA int64");
  TORCH_CHECK(vals.is_cuda() && vals.scalar_type() == torch::kInt32 && vals.numel() == keys.numel(),
              "vals must be CUDA int32 of the same length");
  const at::cuda::CUDAGuard guard(keys.device());
  Tensor kin = keys.contiguous().clone(), vin = vals.contiguous().clone();
  Tensor kout = torch::empty_like(kin), vout = torch::empty_like(vin);
  size_t tb = vi_sort_pairs_temp_bytes((uint64_t)kin.numel(), (int)begin_bit, (int)end_bit);
  Tensor temp = torch::empty({(int64_t)tb}, kin.options().dtype(torch::kUInt8));
  ok(vi_sort_pairs(reinterpret_cast<uint64_t*>(kin.data_ptr()), reinterpret_cast<uint32_t*>(vin.data_ptr()),
                   reinterpret_cast<uint64_t*>(kout.data_ptr()), reinterpret_cast<uint32_t*>(vout.data_ptr()),
                   (uint64_t)kin.numel(), (int)begin_bit, (int)end_bit, temp.data_ptr(), tb,
                   at::cuda::getCurrentCUDAStream().stream()));
  return {kout, vout};
}

}  // namespace

// ---- Gaussian-attribute front end (extension; no counterpart in the reference) ----

Tensor aligned16(const Tensor& t) {
  Tensor c = cuda_f32(t, "tensor");
  if (reinterpret_cast<uintptr_t>(c.data_ptr()) % 16 != 0) c = c.clone();
  return c;
}

// The camera position by value (a device tensor costs a blocking copy).
std::vector<float> host3(const Tensor& t) {
  Tensor h = t.detach().to(torch::kCPU, torch::kFloat32).contiguous().view({-1});
  TORCH_CHECK(h.numel() == 3, "campos must hold 3 values");
  return {h[0].item<float>(), h[1].item<float>(), h[2].item<float>()};
}

// (radii, means2D, depths, cov3D, conic_opacity, rgb, clamped, tiles_touched)
std::tuple<Tensor, Tensor, Tensor, Tensor, Tensor, Tensor, Tensor, Tensor> preprocess_gaussians(
    const Tensor& means3D, const Tensor& scales, const Tensor& rotations, const Tensor& opacities, const Tensor& shs,
    int64_t sh_degree, double scale_modifier, const Tensor& viewmatrix, const Tensor& projmatrix, const Tensor& campos,
    int64_t image_width, int64_t image_height, double tan_fovx, double tan_fovy, double near_plane) {
  const at::cuda::OptionalCUDAGuard guard(means3D.device());
  Tensor m = cuda_f32(means3D, "means3D"), sc = cuda_f32(scales, "scales"), q = aligned16(rotations);
  Tensor op = cuda_f32(opacities, "opacities"), sh = cuda_f32(shs, "shs");
  Tensor vm = cuda_f32(viewmatrix, "viewmatrix"), pm = cuda_f32(projmatrix, "projmatrix");
  const int64_t P = m.size(0);
  TORCH_CHECK(m.dim() == 2 && m.size(1) == 3 && sc.sizes() == m.sizes(), "means3D and scales must be [P, 3]");
  TORCH_CHECK(q.dim() == 2 && q.size(0) == P && q.size(1) == 4, "rotations must be [P, 4]");
  TORCH_CHECK(op.numel() == P, "opacities must hold P values");
  TORCH_CHECK(sh.dim() == 3 && sh.size(0) == P && sh.size(2) == 3, "shs must be [P, M, 3]");
  const std::vector<float> cp = host3(campos);
  auto f32 = m.options();
  Tensor radii = torch::empty({P}, f32.dtype(torch::kInt32));
  Tensor means2D = torch::empty({P, 2}, f32), depths = torch::empty({P}, f32), cov3D = torch::empty({P, 6}, f32);
  Tensor conic = torch::empty({P, 4}, f32), rgb = torch::empty({P, 3}, f32);
  Tensor clamped = torch::empty({P, 3}, f32.dtype(torch::kUInt8));
  Tensor tiles = torch::empty({P}, f32.dtype(torch::kInt32));
  ok(vi_preprocess_gaussians((int)P, (int)sh_degree, (int)sh.size(1), m.data_ptr<float>(), sc.data_ptr<float>(),
                             q.data_ptr<float>(), op.data_ptr<float>(), sh.data_ptr<float>(), (float)scale_modifier,
                             vm.data_ptr<float>(), pm.data_ptr<float>(), cp.data(), (int)image_width,
                             (int)image_height, (float)tan_fovx, (float)tan_fovy, (float)near_plane,
                             radii.data_ptr<int>(), means2D.data_ptr<float>(), depths.data_ptr<float>(),
                             cov3D.data_ptr<float>(), conic.data_ptr<float>(), rgb.data_ptr<float>(),
                             reinterpret_cast<uint8_t*>(clamped.data_ptr()),
                             reinterpret_cast<uint32_t*>(tiles.data_ptr()), at::cuda::getCurrentCUDAStream().stream()));
  return {radii, means2D, depths, cov3D, conic, rgb, clamped, tiles};
}

// (dL/dmeans3D, dL/dscales, dL/drotations, dL/dshs)
std::tuple<Tensor, Tensor, Tensor, Tensor> preprocess_gaussians_backward(
    const Tensor& means3D, const Tensor& scales, const Tensor& rotations, const Tensor& shs, int64_t sh_degree,
    double scale_modifier, const Tensor& viewmatrix, const Tensor& projmatrix, const Tensor& campos,
    int64_t image_width, int64_t image_height, double tan_fovx, double tan_fovy, double near_plane,
    const Tensor& radii, const Tensor& clamped, const Tensor& dL_dmeans2D, const Tensor& dL_ddepths,
    const Tensor& dL_dcov3D, const Tensor& dL_dconic_opacity, const Tensor& dL_drgb) {
  const at::cuda::OptionalCUDAGuard guard(means3D.device());
  Tensor m = cuda_f32(means3D, "means3D"), sc = cuda_f32(scales, "scales"), q = aligned16(rotations);
  Tensor sh = cuda_f32(shs, "shs");
  Tensor vm = cuda_f32(viewmatrix, "viewmatrix"), pm = cuda_f32(projmatrix, "projmatrix");
  Tensor rd = cuda_i32(radii, "radii");
  TORCH_CHECK(clamped.is_cuda() && clamped.scalar_type() == torch::kUInt8, "clamped must be a CUDA uint8 tensor");
  Tensor cl = clamped.contiguous();
  const int64_t P = m.size(0);
  Tensor g2 = cuda_f32(dL_dmeans2D, "dL_dmeans2D"), gd = cuda_f32(dL_ddepths, "dL_ddepths");
  Tensor gcov = cuda_f32(dL_dcov3D, "dL_dcov3D"), gco = cuda_f32(dL_dconic_opacity, "dL_dconic_opacity");
  Tensor grgb = cuda_f32(dL_drgb, "dL_drgb");
  TORCH_CHECK(g2.numel() == 2 * P && gd.numel() == P && gcov.numel() == 6 * P && gco.numel() == 4 * P &&
                  grgb.numel() == 3 * P && rd.numel() == P && cl.numel() == 3 * P,
              "gradient shapes do not match P");
  const std::vector<float> cp = host3(campos);
  Tensor dm = torch::empty({P, 3}, m.options()), ds = torch::empty({P, 3}, m.options());
  Tensor dq = torch::empty({P, 4}, m.options()), dsh = torch::empty_like(sh);
  ok(vi_preprocess_gaussians_backward(
      (int)P, (int)sh_degree, (int)sh.size(1), m.data_ptr<float>(), sc.data_ptr<float>(), q.data_ptr<float>(),
      sh.data_ptr<float>(), (float)scale_modifier, vm.data_ptr<float>(), pm.data_ptr<float>(), cp.data(),
      (int)image_width, (int)image_height, (float)tan_fovx, (float)tan_fovy, (float)near_plane, rd.data_ptr<int>(),
      reinterpret_cast<const uint8_t*>(cl.data_ptr()), g2.data_ptr<float>(), gd.data_ptr<float>(),
      gcov.data_ptr<float>(), gco.data_ptr<float>(), grgb.data_ptr<float>(), dm.data_ptr<float>(),
      ds.data_ptr<float>(), dq.data_ptr<float>(), dsh.data_ptr<float>(), at::cuda::getCurrentCUDAStream().stream()));
  return {dm, ds, dq, dsh};
}

// (point_list [R] int32, tile ids [R] int32, ranges [tiles, 2] int32)
std::tuple<Tensor, Tensor, Tensor> bin_gaussians(const Tensor& radii, const Tensor& means2D, const Tensor& depths,
                                                 const Tensor& tiles_touched, int64_t image_width,
                                                 int64_t image_height) {
  const at::cuda::OptionalCUDAGuard guard(radii.device());
  Tensor rd = cuda_i32(radii, "radii"), m2 = cuda_f32(means2D, "means2D"), dp = cuda_f32(depths, "depths");
  Tensor tt = cuda_i32(tiles_touched, "tiles_touched");
  const int64_t P = rd.numel();
  TORCH_CHECK(m2.numel() == 2 * P && dp.numel() == P && tt.numel() == P, "binning inputs must describe P Gaussians");
  const int64_t R = P ? tt.sum(torch::kInt64).item<int64_t>() : 0;  // buffer sizing; the scan re-checks it
  const int64_t tiles = ((image_width + 15) / 16) * ((image_height + 15) / 16);
  auto i32 = rd.options();
  Tensor point_list = torch::empty({R}, i32), tile_ids = torch::empty({R}, i32);
  Tensor ranges = torch::empty({tiles, 2}, i32);
  const uint64_t nbytes = vi_bin_gaussians_scratch_bytes((int)P, (uint64_t)R, (int)image_width, (int)image_height);
  TORCH_CHECK(nbytes > 0, "volume_integration: bad binning sizes");
  Tensor scratch = torch::empty({(int64_t)nbytes + 256}, rd.options().dtype(torch::kUInt8));
  char* base = reinterpret_cast<char*>(scratch.data_ptr());
  char* al = reinterpret_cast<char*>((reinterpret_cast<uintptr_t>(base) + 255) & ~uintptr_t(255));
  ok(vi_bin_gaussians((int)P, (int)image_width, (int)image_height, rd.data_ptr<int>(), m2.data_ptr<float>(),
                      dp.data_ptr<float>(), reinterpret_cast<const uint32_t*>(tt.data_ptr()), (uint64_t)R, al, nbytes,
                      R ? reinterpret_cast<uint32_t*>(point_list.data_ptr()) : nullptr,
                      R ? reinterpret_cast<uint32_t*>(tile_ids.data_ptr()) : nullptr,
                      reinterpret_cast<uint32_t*>(ranges.data_ptr()), at::cuda::getCurrentCUDAStream().stream()));
  return {point_list, tile_ids, ranges};
}

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.def("integrate_primitives", &integrate_primitives, "Integrate Primitives CUDA forward");
  m.def("integrate_primitives_backward", &integrate_primitives_backward, "Integrate Primitives CUDA backward");
  m.def("integrate_primitives_ex", &integrate_primitives_ex,
        "integrate_primitives plus a hashgrid box (6 floats, or [] for the reference's box) and flags "
        "(1 = exact gradients)");
  m.def("integrate_primitives_backward_ex", &integrate_primitives_backward_ex,
        "integrate_primitives_backward plus the hashgrid box, flags and dL/dvisibility (empty = none)");
  m.attr("FLAG_EXACT_GRADIENTS") = (int64_t)VI_FLAG_EXACT_GRADIENTS;
  m.def("mark_visible", &mark_visible, "Mark Visible Primitives CUDA");
  m.def("preprocess_gaussians", &preprocess_gaussians, "Gaussian-attribute preprocess (extension)");
  m.def("preprocess_gaussians_backward", &preprocess_gaussians_backward,
        "Exact derivative of the Gaussian-attribute preprocess (extension)");
  m.def("bin_gaussians", &bin_gaussians, "Tile binning of projected Gaussians (extension)");
  m.def("state_views", &state_views, "Integer state of a forward call in the reference's formats");
  m.def("sort_pairs", &sort_pairs, "Stable radix sort of (uint64 key, uint32 value) pairs");
  m.def("sort_end_bit", [](int64_t tiles) { return vi_sort_end_bit((uint32_t)tiles); });
  m.def("kernel_launches", []() { return (uint64_t)vi_kernel_launches(); });
  m.def("profile_enable", [](bool on) { ok(vi_profile_enable(on ? 1 : 0)); });
  m.def("profile_read", [](bool reset) {
    double ms[8];
    uint64_t calls[8];
    ok(vi_profile_read(ms, calls, 8, reset ? 1 : 0));
    static const char* names[8] = {"preprocess", "depth_sort", "offsets", "features",
                                   "binning", "render", "bwd_pixel", "bwd_prim"};
    py::dict d;
    for (int i = 0; i < 8; i++) d[names[i]] = py::make_tuple(ms[i], calls[i]);
    return d;
  });
}
