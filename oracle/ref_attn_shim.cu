// Checker build of the REFERENCE's own sm80+ INT8 attention (diffucore 0.2.4,
// src/diffucore/kernels/int8_attn_sm80.cu), compiled from its source where it lies by
// oracle/build_ref.py into oracle/_ref/. TEST INFRASTRUCTURE ONLY: the tests use it to pin the
// CPU oracle (K codes, K column sums) and to compare outputs; nothing in the product loads it.
//
// The reference file is included unchanged; this shim only adds a torch op `dcref::k_prep` that
// runs the reference's three prep kernels (kv_stats_kernel, k_sum_kernel, k_quant_kernel) the way
// its host `fwd` does (int8_attn_sm80.cu:468-485) and returns their outputs, which `fwd` keeps
// internal.
#include "int8_attn_sm80.cu"

namespace {

std::vector<torch::Tensor> k_prep(torch::Tensor k) {
  check_input(k, "k");
  const at::cuda::CUDAGuard guard(k.device());
  auto stream = at::cuda::getCurrentCUDAStream();
  const int B = k.size(0), Lk = k.size(1), H = k.size(2);
  const int Lk_pad = (Lk + BC - 1) / BC * BC;
  auto i8 = k.options().dtype(torch::kInt8);
  auto f32 = k.options().dtype(torch::kFloat32);
  auto ki = torch::zeros({B, H, Lk_pad, D}, i8);
  auto ks = torch::empty({B, H, Lk_pad / BC}, f32);
  const int nwin = (Lk + FLUSH_EVERY * BC - 1) / (FLUSH_EVERY * BC);
  auto kpart = torch::empty({B, H, nwin, D}, f32);
  auto ksum = torch::empty({B, H, D}, f32);
  auto vb = torch::zeros({B, H}, f32);
  kv_stats_kernel<<<dim3(nwin, H, B), 256, 0, stream>>>(
      (const half*)k.data_ptr(), (const half*)k.data_ptr(), kpart.data_ptr<float>(), vb.data_ptr<float>(), Lk, H,
      k.stride(0), k.stride(1), k.stride(2), k.stride(0), k.stride(1), k.stride(2));
  k_sum_kernel<<<B * H, D, 0, stream>>>(kpart.data_ptr<float>(), ksum.data_ptr<float>(), nwin);
  k_quant_kernel<<<dim3(Lk_pad / BC, H, B), NT, 0, stream>>>(
      (const half*)k.data_ptr(), ksum.data_ptr<float>(), ki.data_ptr<int8_t>(), ks.data_ptr<float>(), Lk, H, Lk_pad,
      k.stride(0), k.stride(1), k.stride(2));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  return {ki, ks, ksum};
}

}  // namespace

TORCH_LIBRARY(dcref, m) { m.def("k_prep(Tensor k) -> Tensor[]", &k_prep); }
