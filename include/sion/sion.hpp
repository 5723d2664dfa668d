// sion:: LibTorch wrappers over the felix operators. Same signatures as the
// reference (include/sion/sion.hpp:4-14); flash_attention_lse is new.
#pragma once
#include <torch/torch.h>
#include <tuple>

namespace sion {

torch::Tensor flash_attention(const torch::Tensor& query, const torch::Tensor& key,
                              const torch::Tensor& value);
torch::Tensor sgemm(const torch::Tensor& A, const torch::Tensor& B, float alpha, float beta);
torch::Tensor hgemm(const torch::Tensor& A, const torch::Tensor& B, float alpha, float beta);
torch::Tensor hgemm_nt(const torch::Tensor& A, const torch::Tensor& B, float alpha, float beta);
torch::Tensor gemm(const torch::Tensor& A, const torch::Tensor& B, float alpha, float beta);

// new: causal-mask variant (query i attends to keys 0..i)
torch::Tensor flash_attention(const torch::Tensor& query, const torch::Tensor& key,
                              const torch::Tensor& value, bool causal);
// new: (O, LSE) with LSE fp32 [B, H, S]
std::tuple<torch::Tensor, torch::Tensor> flash_attention_lse(const torch::Tensor& query,
                                                             const torch::Tensor& key,
                                                             const torch::Tensor& value,
                                                             bool causal = false);
// new: gradients (dQ, dK, dV) of flash_attention given its inputs, the forward
// output O and LSE (from flash_attention_lse) and the output gradient dO
std::tuple<torch::Tensor, torch::Tensor, torch::Tensor> flash_attention_backward(
    const torch::Tensor& query, const torch::Tensor& key, const torch::Tensor& value,
    const torch::Tensor& out, const torch::Tensor& lse, const torch::Tensor& grad_out,
    bool causal = false);

}  // namespace sion
