// sion:: LibTorch wrappers and the Python module `sion_b200._sion`.
//
// Same validation, output allocation, stream pickup and error conversion as the
// reference wrappers (src/sion/gemm/sgemm/sgemm.cpp:5-32,
// src/sion/gemm/hgemm/hgemm.cpp:4-83, src/sion/gemm/gemm.cpp:10-31,
// src/sion/flash_attention/flash_attn.cpp:7-66), calling the felix:: API with
// the reference's kernel names. Differences, all additive:
//   * C is zero-filled when beta != 0 (the reference reads uninitialised
//     torch::empty memory there, sgemm.cpp:19,27);
//   * flash_attention accepts any seqlen (the reference requires seqlen % 64);
//   * flash_attention_lse also returns the fp32 log-sum-exp; both take an
//     optional causal mask;
//   * the Python functions take named arguments (python/binding.cpp:6-11 has none).
#include <sion/sion.hpp>

#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <felix/felix.hpp>
#include <torch/extension.h>

namespace sion {

namespace {
torch::Tensor make_output(int64_t M, int64_t N, const torch::TensorOptions& opt, float beta) {
  return beta != 0.f ? torch::zeros({M, N}, opt) : torch::empty({M, N}, opt);
}
}  // namespace

torch::Tensor sgemm(const torch::Tensor& A, const torch::Tensor& B, float alpha, float beta) {
  TORCH_CHECK(A.is_cuda(), "A must be CUDA tensor");
  TORCH_CHECK(B.is_cuda(), "B must be CUDA tensor");
  TORCH_CHECK(A.dtype() == torch::kFloat32, "A must be float32");
  TORCH_CHECK(B.dtype() == torch::kFloat32, "B must be float32");
  TORCH_CHECK(A.dim() == 2 && B.dim() == 2, "A and B must be 2D");
  const c10::cuda::CUDAGuard guard(A.device());
  auto Ac = A.contiguous();
  auto Bc = B.contiguous();
  const int64_t M = Ac.size(0), K = Ac.size(1), N = Bc.size(1);
  TORCH_CHECK(Bc.size(0) == K, "B.size(0) must match A.size(1)");
  auto C = make_output(M, N, Ac.options(), beta);
  cudaStream_t stream = at::cuda::getCurrentCUDAStream();
  auto status = felix::ampere_sgemm_launch(uint32_t(M), uint32_t(N), uint32_t(K), alpha,
                                           Ac.data_ptr<float>(), Bc.data_ptr<float>(), beta,
                                           C.data_ptr<float>(), stream);
  TORCH_CHECK(status.ok(), "SGEMM launch failed: ", status.str());
  return C;
}

namespace {
torch::Tensor hgemm_impl(const torch::Tensor& A, const torch::Tensor& B, float alpha, float beta,
                         bool nt) {
  TORCH_CHECK(A.is_cuda(), "A must be CUDA tensor");
  TORCH_CHECK(B.is_cuda(), "B must be CUDA tensor");
  TORCH_CHECK(A.dtype() == torch::kFloat16, "A must be float16");
  TORCH_CHECK(B.dtype() == torch::kFloat16, "B must be float16");
  TORCH_CHECK(A.dim() == 2, "A must be 2D");
  TORCH_CHECK(B.dim() == 2, "B must be 2D");
  TORCH_CHECK(A.is_contiguous(), "A must be contiguous");
  TORCH_CHECK(B.is_contiguous(), "B must be contiguous");
  const c10::cuda::CUDAGuard guard(A.device());
  const int64_t M = A.size(0), K = A.size(1);
  const int64_t N = nt ? B.size(0) : B.size(1);
  if (nt) {
    TORCH_CHECK(B.size(1) == K, "B.size(1) must match A.size(1) for NT GEMM");
  } else {
    TORCH_CHECK(B.size(0) == K, "B.size(0) must match A.size(1)");
  }
  auto C = make_output(M, N, A.options(), beta);
  cudaStream_t stream = at::cuda::getCurrentCUDAStream();
  auto status = felix::ampere_hgemm_launch(
      uint32_t(M), uint32_t(N), uint32_t(K), alpha,
      reinterpret_cast<const half*>(A.data_ptr<at::Half>()),
      reinterpret_cast<const half*>(B.data_ptr<at::Half>()), beta,
      reinterpret_cast<half*>(C.data_ptr<at::Half>()), stream,
      nt ? "cute_hgemm_128x128_nt" : "cute_hgemm_128x128_nn");
  TORCH_CHECK(status.ok(), nt ? "HGEMM NT launch failed: " : "HGEMM launch failed: ",
              status.str());
  return C;
}
}  // namespace

torch::Tensor hgemm(const torch::Tensor& A, const torch::Tensor& B, float alpha, float beta) {
  return hgemm_impl(A, B, alpha, beta, false);
}

torch::Tensor hgemm_nt(const torch::Tensor& A, const torch::Tensor& B, float alpha, float beta) {
  return hgemm_impl(A, B, alpha, beta, true);
}

torch::Tensor gemm(const torch::Tensor& A, const torch::Tensor& B, float alpha, float beta) {
  TORCH_CHECK(A.is_cuda(), "A must be CUDA tensor");
  TORCH_CHECK(B.is_cuda(), "B must be CUDA tensor");
  TORCH_CHECK(A.dtype() == B.dtype(), "A and B must have the same dtype");
  switch (A.scalar_type()) {
    case torch::kFloat32: return sgemm(A, B, alpha, beta);
    case torch::kFloat16: return hgemm(A, B, alpha, beta);
    default: TORCH_CHECK(false, "Unsupported dtype for gemm: ", A.dtype());
  }
}

namespace {
void check_attn_inputs(const torch::Tensor& Q, const torch::Tensor& K, const torch::Tensor& V) {
  TORCH_CHECK(Q.is_cuda() && K.is_cuda() && V.is_cuda(), "All tensors must be CUDA tensors");
  TORCH_CHECK(Q.dtype() == torch::kHalf && K.dtype() == torch::kHalf && V.dtype() == torch::kHalf,
              "All tensors must be half");
  TORCH_CHECK(Q.dim() == 4 && K.dim() == 4 && V.dim() == 4, "All tensors must be 4D");
  TORCH_CHECK(Q.sizes() == K.sizes() && Q.sizes() == V.sizes(),
              "query, key and value must have the same shape [B, H, S, D]");
}

std::tuple<torch::Tensor, torch::Tensor> attn_impl(const torch::Tensor& query,
                                                   const torch::Tensor& key,
                                                   const torch::Tensor& value, bool want_lse,
                                                   bool causal) {
  check_attn_inputs(query, key, value);
  const c10::cuda::CUDAGuard guard(query.device());
  auto Q = query.contiguous(), K = key.contiguous(), V = value.contiguous();
  const int64_t B = Q.size(0), H = Q.size(1), S = Q.size(2), D = Q.size(3);
  auto O = torch::empty({B, H, S, D}, Q.options());
  torch::Tensor L;
  if (want_lse) L = torch::empty({B, H, S}, Q.options().dtype(torch::kFloat32));
  half* q = reinterpret_cast<half*>(Q.data_ptr<at::Half>());
  half* k = reinterpret_cast<half*>(K.data_ptr<at::Half>());
  half* v = reinterpret_cast<half*>(V.data_ptr<at::Half>());
  half* o = reinterpret_cast<half*>(O.data_ptr<at::Half>());
  float* l = want_lse ? L.data_ptr<float>() : nullptr;
  cudaStream_t stream = at::cuda::getCurrentCUDAStream();
  felix::FelixStatus status;
  switch (D) {
    case 64:
      status = (want_lse || causal)
                   ? felix::flash_attn_fwd_lse_launch<64, 64>(q, k, v, o, l, uint32_t(H),
                                                              uint32_t(B), uint32_t(S), stream,
                                                              causal)
                        : felix::ampere_flash_attn_launch<64, 64>(q, k, v, o, uint32_t(H),
                                                                  uint32_t(B), uint32_t(S), stream);
      break;
    case 128:
      status = (want_lse || causal)
                   ? felix::flash_attn_fwd_lse_launch<128, 64>(q, k, v, o, l, uint32_t(H),
                                                               uint32_t(B), uint32_t(S), stream,
                                                               causal)
                   : felix::ampere_flash_attn_launch<128, 64>(q, k, v, o, uint32_t(H),
                                                              uint32_t(B), uint32_t(S), stream);
      break;
    default: TORCH_CHECK(false, "flash_attention: unsupported head dimension ", D);
  }
  TORCH_CHECK(status.ok(), "flash_attention: kernel launch failed: ", status.str());
  return {O, L};
}
}  // namespace

torch::Tensor flash_attention(const torch::Tensor& query, const torch::Tensor& key,
                              const torch::Tensor& value) {
  return std::get<0>(attn_impl(query, key, value, false, false));
}

torch::Tensor flash_attention(const torch::Tensor& query, const torch::Tensor& key,
                              const torch::Tensor& value, bool causal) {
  return std::get<0>(attn_impl(query, key, value, false, causal));
}

std::tuple<torch::Tensor, torch::Tensor> flash_attention_lse(const torch::Tensor& query,
                                                             const torch::Tensor& key,
                                                             const torch::Tensor& value,
                                                             bool causal) {
  return attn_impl(query, key, value, true, causal);
}

std::tuple<torch::Tensor, torch::Tensor, torch::Tensor> flash_attention_backward(
    const torch::Tensor& query, const torch::Tensor& key, const torch::Tensor& value,
    const torch::Tensor& out, const torch::Tensor& lse, const torch::Tensor& grad_out,
    bool causal) {
  check_attn_inputs(query, key, value);
  TORCH_CHECK(out.sizes() == query.sizes() && grad_out.sizes() == query.sizes(),
              "out and grad_out must have the shape of query");
  TORCH_CHECK(out.dtype() == torch::kHalf && grad_out.dtype() == torch::kHalf,
              "out and grad_out must be half");
  TORCH_CHECK(out.is_cuda() && grad_out.is_cuda() && lse.is_cuda(), "All tensors must be CUDA tensors");
  const int64_t B = query.size(0), H = query.size(1), S = query.size(2), D = query.size(3);
  TORCH_CHECK(lse.dtype() == torch::kFloat32 && lse.dim() == 3 && lse.size(0) == B &&
                  lse.size(1) == H && lse.size(2) == S,
              "lse must be float32 [B, H, S]");
  const c10::cuda::CUDAGuard guard(query.device());
  auto Q = query.contiguous(), K = key.contiguous(), V = value.contiguous();
  auto O = out.contiguous(), G = grad_out.contiguous(), L = lse.contiguous();
  auto dQ = torch::empty_like(Q), dK = torch::empty_like(Q), dV = torch::empty_like(Q);
  auto hp = [](const torch::Tensor& t) { return reinterpret_cast<half*>(t.data_ptr<at::Half>()); };
  cudaStream_t stream = at::cuda::getCurrentCUDAStream();
  felix::FelixStatus status;
  switch (D) {
    case 64:
      status = felix::flash_attn_bwd_launch<64>(hp(Q), hp(K), hp(V), hp(O), hp(G),
                                                L.data_ptr<float>(), hp(dQ), hp(dK), hp(dV),
                                                uint32_t(H), uint32_t(B), uint32_t(S), stream,
                                                causal);
      break;
    case 128:
      status = felix::flash_attn_bwd_launch<128>(hp(Q), hp(K), hp(V), hp(O), hp(G),
                                                 L.data_ptr<float>(), hp(dQ), hp(dK), hp(dV),
                                                 uint32_t(H), uint32_t(B), uint32_t(S), stream,
                                                 causal);
      break;
    default: TORCH_CHECK(false, "flash_attention_backward: unsupported head dimension ", D);
  }
  TORCH_CHECK(status.ok(), "flash_attention_backward: kernel launch failed: ", status.str());
  return {dQ, dK, dV};
}

}  // namespace sion

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  namespace py = pybind11;
  m.doc() = "Sion operators on sm_100a (tcgen05 HGEMM / flash attention, FFMA SGEMM)";
  m.def("sgemm", &sion::sgemm, "fp32 GEMM: alpha * A @ B + beta * C", py::arg("A"), py::arg("B"),
        py::arg("alpha") = 1.0f, py::arg("beta") = 0.0f);
  m.def("hgemm", &sion::hgemm, "fp16 GEMM, B stored K x N", py::arg("A"), py::arg("B"),
        py::arg("alpha") = 1.0f, py::arg("beta") = 0.0f);
  m.def("hgemm_nt", &sion::hgemm_nt, "fp16 GEMM, B stored N x K", py::arg("A"), py::arg("B"),
        py::arg("alpha") = 1.0f, py::arg("beta") = 0.0f);
  m.def("gemm", &sion::gemm, "GEMM dispatching on dtype (fp32 -> sgemm, fp16 -> hgemm)",
        py::arg("A"), py::arg("B"), py::arg("alpha") = 1.0f, py::arg("beta") = 0.0f);
  m.def("flash_attention",
        py::overload_cast<const torch::Tensor&, const torch::Tensor&, const torch::Tensor&, bool>(
            &sion::flash_attention),
        "flash attention forward (causal=True: query i sees keys 0..i)", py::arg("query"),
        py::arg("key"), py::arg("value"), py::arg("causal") = false);
  m.def("flash_attention_lse", &sion::flash_attention_lse,
        "flash attention forward returning (O, fp32 LSE)", py::arg("query"), py::arg("key"),
        py::arg("value"), py::arg("causal") = false);
  m.def("flash_attention_backward", &sion::flash_attention_backward,
        "flash attention backward returning (dQ, dK, dV)", py::arg("query"), py::arg("key"),
        py::arg("value"), py::arg("out"), py::arg("lse"), py::arg("grad_out"),
        py::arg("causal") = false);
}
