// Test infrastructure: a Python module around the reference rasterizer's own
// kernels (cuda_rasterizer/rasterizer_impl_v2.cu, minimally patched by
// oracle/ref/build_ref.py into oracle/_ref/). It re-exports the reference's
// render_sar / render_sar_with_settings / render_sar_backward bindings and
// adds `intermediates`, which runs the reference's preprocess_kernel,
// compute_ranges_kernel, build_tile_gaussian_list_kernel and
// build_shadow_tile_list_kernel on one view and returns their outputs, so that
// the tests can compare tile lists bit for bit. Only tests/ and bench.py's
// reference leg load it.
#include <torch/extension.h>
#include <pybind11/pybind11.h>

// The reference source defines PYBIND11_MODULE(cuda_rasterizer_sar, m) {...};
// turn that block into a registration function of this module instead.
#pragma push_macro("PYBIND11_MODULE")
#undef PYBIND11_MODULE
#define PYBIND11_MODULE(name, variable) static void sarr_ref_register_##name(::pybind11::module_& variable)
#include "rasterizer_impl_v2_patched.cu"
#undef PYBIND11_MODULE
#pragma pop_macro("PYBIND11_MODULE")

namespace {

// The host view setup the reference performs before its kernels
// (CUDASARRenderer::render, :1100-1120), restated.
struct RefView {
  float rx, ry, rz, alpha, beta, Rc, theta, phi;
};

RefView ref_view(float radar_z, float track, float inc, float az) {
  RefView v;
  const float deg = 0.017453292519943295f;
  const float track_rad = track * deg, inc_rad = inc * deg, az_rad = az * deg;
  float sb = sinf(inc_rad) * cosf(az_rad);
  sb = fmaxf(fminf(sb, 1.0f), -1.0f);
  const float beta = asinf(sb);
  const float tb = tanf(beta);
  v.rx = radar_z * tb * sinf(track_rad);
  v.ry = -radar_z * tb * cosf(track_rad);
  v.rz = radar_z;
  v.Rc = radar_z / cosf(beta);
  v.alpha = track_rad;
  v.beta = beta;
  v.theta = beta;
  v.phi = track_rad < 0.0f ? track_rad + 2.0f * PI : track_rad;
  return v;
}

std::vector<torch::Tensor> intermediates(torch::Tensor means, torch::Tensor cov6, torch::Tensor sigma,
                                         torch::Tensor sh, float radar_z, float track, float inc,
                                         float az, float rho_r, float rho_a, int Nr, int Na) {
  TORCH_CHECK(means.is_cuda() && means.is_contiguous(), "means must be contiguous CUDA");
  TORCH_CHECK(cov6.is_contiguous() && sigma.is_contiguous() && sh.is_contiguous(), "contiguous inputs");
  TORCH_CHECK(sh.dim() == 2 && sh.size(1) == SH_COEFFS_SIZE, "sh must be [N,16]");
  const int n = (int)means.size(0);
  const auto fo = means.options();
  const auto io = fo.dtype(torch::kInt32);
  const int tiles_x = (Na + BLOCK_X - 1) / BLOCK_X, tiles_y = (Nr + BLOCK_Y - 1) / BLOCK_Y;
  const int T = tiles_x * tiles_y;
  auto f = torch::zeros({13, n}, fo);
  auto valid = torch::zeros({n}, fo.dtype(torch::kBool));
  auto ranges = torch::zeros({4, n}, io);
  auto cnt = torch::zeros({T}, io);
  auto lst = torch::full({T, MAX_GAUSSIANS_PER_TILE}, -1, io);
  auto scnt = torch::zeros({T}, io);
  auto slst = torch::full({T, MAX_GAUSSIANS_PER_TILE}, -1, io);
  const RefView v = ref_view(radar_z, track, inc, az);
  float h_basis[SH_COEFFS_SIZE];
  compute_sh_basis_host(v.theta, v.phi, h_basis);
  auto basis = torch::from_blob(h_basis, {SH_COEFFS_SIZE}, torch::kFloat32).to(means.device());
  if (n == 0 || T == 0) return {f, valid, ranges, cnt, lst, scnt, slst, basis};
  float* F = f.data_ptr<float>();
  const size_t N = (size_t)n;
  bool* V = valid.data_ptr<bool>();
  int* R = ranges.data_ptr<int>();
  const int blocks = (n + 255) / 256;
  preprocess_kernel<<<blocks, 256>>>(
      means.data_ptr<float>(), cov6.data_ptr<float>(), sigma.data_ptr<float>(), sh.data_ptr<float>(),
      basis.data_ptr<float>(), v.rx, v.ry, v.rz, v.alpha, v.beta, v.Rc, rho_r, rho_a, Nr, Na, F,
      F + N, F + 2 * N, F + 3 * N, F + 4 * N, F + 5 * N, F + 6 * N, F + 7 * N, F + 8 * N, F + 9 * N,
      F + 10 * N, F + 11 * N, F + 12 * N, V, n);
  compute_ranges_kernel<<<blocks, 256>>>(F, F + N, F + 2 * N, F + 3 * N, F + 4 * N, V, Nr, Na, R,
                                         R + N, R + 2 * N, R + 3 * N, n);
  build_tile_gaussian_list_kernel<<<dim3(tiles_x, tiles_y), dim3(1, 1)>>>(
      F, F + N, R, R + N, R + 2 * N, R + 3 * N, F + 11 * N, V, tiles_x, tiles_y, Nr, Na,
      cnt.data_ptr<int>(), lst.data_ptr<int>(), n);
  build_shadow_tile_list_kernel<<<dim3(tiles_x, tiles_y), dim3(1, 1)>>>(
      F + 5 * N, F + 6 * N, F + 7 * N, F + 8 * N, F + 9 * N, F + 11 * N, V, tiles_x, tiles_y, Nr, Na,
      scnt.data_ptr<int>(), slst.data_ptr<int>(), n);
  const cudaError_t e = cudaGetLastError();
  TORCH_CHECK(e == cudaSuccess, "reference kernels failed: ", cudaGetErrorString(e));
  return {f, valid, ranges, cnt, lst, scnt, slst, basis};
}

}  // namespace

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  sarr_ref_register_cuda_rasterizer_sar(m);
  m.def("intermediates", &intermediates,
        "reference preprocess / ranges / tile lists / shadow lists of one view");
}
