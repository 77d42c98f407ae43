// PyTorch extension `flashgmm_b200._C`: the reference's op module (`flash_gmm_native`,
// flash_gmm/csrc/binding.cpp:94-108) as compiled pybind11 bindings over this library's C
// ABI (include/flashgmm_b200.h).  Same op names, argument names, defaults and return lists
// as the reference: flash_em_fused(X, mu, var, log_pi, BN=64, BK=8),
// standard_e_step(X, mu, var, log_pi), flash_e_step(X, mu, var, log_pi, BK=4),
// standard_m_step(X, gamma).
//
// Differences, all deliberate: CUDA tensors only (the reference dispatches CPU tensors to
// OpenMP, binding.cpp:68-75; here there is no CPU path and a CPU tensor is an error);
// every argument's dtype, shape, device and contiguity is checked (the reference checks
// only X's dtype and rank, binding.cpp:38-39, 66); launches go on the current stream and
// failures raise with the library's message.  BN / BK are accepted and ignored: tile
// shapes are fixed by the kernels (the reference's CUDA launcher also ignores BK,
// flash_gmm_cuda.cu:430-447).  Scratch comes from torch's caching allocator.
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>

#include "../../include/flashgmm_b200.h"

namespace {

void check_f32_cuda(const torch::Tensor &t, const char *name, int dim, const torch::Device *dev) {
  TORCH_CHECK(t.scalar_type() == torch::kFloat32, name, " must be float32");
  TORCH_CHECK(t.dim() == dim, name, " must be ", dim, "D");
  TORCH_CHECK(t.is_cuda(), name, " must be a CUDA tensor (flashgmm_b200 has no CPU path)");
  if (dev) TORCH_CHECK(t.device() == *dev, name, " is on ", t.device(), ", expected ", *dev);
}

void check_rc(int rc, const char *op) {
  TORCH_CHECK(rc == FGMM_OK, op, ": flashgmm_b200 error ", rc, ": ", fgmm_last_error());
}

struct Params {
  torch::Tensor X, mu, var, lp;
  int64_t N;
  int d, K;
};

Params params(const torch::Tensor &X, const torch::Tensor &mu, const torch::Tensor &var,
              const torch::Tensor &log_pi) {
  check_f32_cuda(X, "X", 2, nullptr);
  const torch::Device dev = X.device();
  check_f32_cuda(mu, "mu", 2, &dev);
  check_f32_cuda(var, "var", 2, &dev);
  check_f32_cuda(log_pi, "log_pi", 1, &dev);
  const int64_t N = X.size(0), d = X.size(1), K = mu.size(0);
  TORCH_CHECK(mu.size(1) == d && var.size(0) == K && var.size(1) == d && log_pi.size(0) == K,
              "shape mismatch: X", X.sizes(), " mu", mu.sizes(), " var", var.sizes(), " log_pi",
              log_pi.sizes());
  return {X.contiguous(), mu.contiguous(), var.contiguous(), log_pi.contiguous(), N, (int)d, (int)K};
}

torch::Tensor scratch(size_t bytes, const torch::Device &dev) {
  return torch::empty({(int64_t)std::max<size_t>(bytes, 256)},
                      torch::TensorOptions().dtype(torch::kUInt8).device(dev));
}

std::vector<torch::Tensor> flash_em_fused(torch::Tensor X, torch::Tensor mu, torch::Tensor var,
                                          torch::Tensor log_pi, int64_t /*BN*/, int64_t /*BK*/) {
  Params p = params(X, mu, var, log_pi);
  const c10::cuda::CUDAGuard guard(p.X.device());
  const size_t nb = fgmm_em_fused_workspace_bytes(p.N, p.d, p.K);
  TORCH_CHECK(nb > 0, "flash_em_fused: unsupported shape N=", p.N, " K=", p.K, " d=", p.d);
  auto ws = scratch(nb, p.X.device());
  auto opt = p.X.options();
  auto new_mu = torch::empty({p.K, p.d}, opt), new_var = torch::empty({p.K, p.d}, opt);
  auto new_lp = torch::empty({p.K}, opt), ln = torch::empty({p.N}, opt);
  check_rc(fgmm_em_fused(p.X.data_ptr<float>(), p.N, p.d, p.mu.data_ptr<float>(),
                         p.var.data_ptr<float>(), p.lp.data_ptr<float>(), p.K,
                         new_mu.data_ptr<float>(), new_var.data_ptr<float>(),
                         new_lp.data_ptr<float>(), ln.data_ptr<float>(), ws.data_ptr(), ws.numel(),
                         at::cuda::getCurrentCUDAStream().stream()),
           "flash_em_fused");
  return {new_mu, new_var, new_lp, ln};
}

std::vector<torch::Tensor> standard_e_step(torch::Tensor X, torch::Tensor mu, torch::Tensor var,
                                           torch::Tensor log_pi) {
  Params p = params(X, mu, var, log_pi);
  const c10::cuda::CUDAGuard guard(p.X.device());
  const size_t nb = fgmm_e_step_workspace_bytes(p.N, p.d, p.K);
  TORCH_CHECK(nb > 0, "standard_e_step: unsupported shape N=", p.N, " K=", p.K, " d=", p.d);
  auto ws = scratch(nb, p.X.device());
  auto gamma = torch::empty({p.N, (int64_t)p.K}, p.X.options());
  auto ln = torch::empty({p.N}, p.X.options());
  check_rc(fgmm_e_step(p.X.data_ptr<float>(), p.N, p.d, p.mu.data_ptr<float>(),
                       p.var.data_ptr<float>(), p.lp.data_ptr<float>(), p.K,
                       gamma.data_ptr<float>(), ln.data_ptr<float>(), ws.data_ptr(), ws.numel(),
                       at::cuda::getCurrentCUDAStream().stream()),
           "standard_e_step");
  return {gamma, ln};
}

std::vector<torch::Tensor> flash_e_step(torch::Tensor X, torch::Tensor mu, torch::Tensor var,
                                        torch::Tensor log_pi, int64_t /*BK*/) {
  // the same responsibilities and log-normalizers as standard_e_step (the reference runs
  // this op on the CPU only, flash_gmm_cpu.cpp:108-168)
  return standard_e_step(X, mu, var, log_pi);
}

std::vector<torch::Tensor> standard_m_step(torch::Tensor X, torch::Tensor gamma) {
  check_f32_cuda(X, "X", 2, nullptr);
  const torch::Device dev = X.device();
  check_f32_cuda(gamma, "gamma", 2, &dev);
  TORCH_CHECK(gamma.size(0) == X.size(0), "shape mismatch: X", X.sizes(), " gamma", gamma.sizes());
  auto Xc = X.contiguous(), gc = gamma.contiguous();
  const int64_t N = X.size(0);
  const int d = (int)X.size(1), K = (int)gamma.size(1);
  const c10::cuda::CUDAGuard guard(dev);
  const size_t nb = fgmm_m_step_workspace_bytes(N, d, K);
  TORCH_CHECK(nb > 0, "standard_m_step: unsupported shape N=", N, " K=", K, " d=", d);
  auto ws = scratch(nb, dev);
  auto opt = X.options();
  auto mu = torch::empty({K, d}, opt), var = torch::empty({K, d}, opt), lp = torch::empty({K}, opt);
  check_rc(fgmm_m_step(Xc.data_ptr<float>(), N, d, gc.data_ptr<float>(), K, mu.data_ptr<float>(),
                       var.data_ptr<float>(), lp.data_ptr<float>(), ws.data_ptr(), ws.numel(),
                       at::cuda::getCurrentCUDAStream().stream()),
           "standard_m_step");
  return {mu, var, lp};
}

}  // namespace

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.doc() = "flashgmm_b200 CUDA ops with the reference's op-module interface";
  m.def("flash_em_fused", &flash_em_fused, "One fused EM iteration (CUDA)", py::arg("X"),
        py::arg("mu"), py::arg("var"), py::arg("log_pi"), py::arg("BN") = 64, py::arg("BK") = 8);
  m.def("standard_e_step", &standard_e_step, "E-step with materialised responsibilities (CUDA)",
        py::arg("X"), py::arg("mu"), py::arg("var"), py::arg("log_pi"));
  m.def("flash_e_step", &flash_e_step, "E-step, same outputs as standard_e_step (CUDA)",
        py::arg("X"), py::arg("mu"), py::arg("var"), py::arg("log_pi"), py::arg("BK") = 4);
  m.def("standard_m_step", &standard_m_step, "M-step from responsibilities (CUDA)", py::arg("X"),
        py::arg("gamma"));
}
