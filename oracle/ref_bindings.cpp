// Python binding of the reference's own quantiser and norm host launchers, so
// the unmodified reference kernels can run on a B200 as a GPU oracle.
// TEST INFRASTRUCTURE ONLY (see oracle/__init__.py).
//
// The functions declared here are defined in the reference sources that
// oracle/build_ref.py compiles from where they lie:
//   csrc/kernels/fp8_quantize.cu    (compute_fp8_scale :194, quantise_to_e4m3 :222,
//                                    quantise_to_e5m2 :241, dequantise_e4m3 :260,
//                                    dequantise_e5m2 :277)
//   csrc/kernels/layernorm_fused.cu (layernorm_fused_impl :266, rmsnorm_fused :312)
// The declarations must match those definitions; everything else is ours.
#include <torch/extension.h>

#include <utility>
#include <vector>

float compute_fp8_scale(const torch::Tensor& input, float fp8_max_val);
std::pair<torch::Tensor, float> quantise_to_e4m3(const torch::Tensor& fp16);
std::pair<torch::Tensor, float> quantise_to_e5m2(const torch::Tensor& fp16);
torch::Tensor dequantise_e4m3(const torch::Tensor& fp8, float scale, const std::vector<int64_t>& shape);
torch::Tensor dequantise_e5m2(const torch::Tensor& fp8, float scale, const std::vector<int64_t>& shape);
std::vector<torch::Tensor> layernorm_fused_impl(const torch::Tensor& x, const c10::optional<torch::Tensor>& residual,
                                                const torch::Tensor& gamma, const torch::Tensor& beta, float epsilon,
                                                bool want_sum);
torch::Tensor rmsnorm_fused(const torch::Tensor& x, const torch::Tensor& residual, const torch::Tensor& gamma,
                            float epsilon);

namespace {

void require(const torch::Tensor& t, const char* name, int64_t multiple_of) {
  TORCH_CHECK(t.is_cuda() && t.is_contiguous(), name, " must be a contiguous CUDA tensor");
  // The reference kernels read 8 elements per thread without a tail check.
  TORCH_CHECK(t.numel() % multiple_of == 0, name, " element count must be a multiple of ", multiple_of);
}

}  // namespace

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.def("compute_fp8_scale", [](const torch::Tensor& x, float mx) {
    require(x, "x", 1);
    return compute_fp8_scale(x, mx);
  });
  m.def("quantise_e4m3", [](const torch::Tensor& x) {
    require(x, "x", 8);
    return quantise_to_e4m3(x);
  });
  m.def("quantise_e5m2", [](const torch::Tensor& x) {
    require(x, "x", 8);
    return quantise_to_e5m2(x);
  });
  m.def("dequantise_e4m3", [](const torch::Tensor& q, float s, const std::vector<int64_t>& shape) {
    require(q, "q", 8);
    return dequantise_e4m3(q, s, shape);
  });
  m.def("dequantise_e5m2", [](const torch::Tensor& q, float s, const std::vector<int64_t>& shape) {
    require(q, "q", 8);
    return dequantise_e5m2(q, s, shape);
  });
  m.def("layernorm_fused_residual",
        [](const torch::Tensor& x, const c10::optional<torch::Tensor>& res, const torch::Tensor& g,
           const torch::Tensor& b, float eps) {
          require(x, "x", 8);
          TORCH_CHECK(x.size(-1) % 8 == 0, "last dim must be a multiple of 8");
          auto r = layernorm_fused_impl(x, res, g, b, eps, true);
          return std::make_tuple(r[0], r[1]);
        });
  m.def("rmsnorm_fused", [](const torch::Tensor& x, const torch::Tensor& res, const torch::Tensor& g, float eps) {
    require(x, "x", 8);
    TORCH_CHECK(x.size(-1) % 8 == 0, "last dim must be a multiple of 8");
    return rmsnorm_fused(x, res, g, eps);
  });
}
