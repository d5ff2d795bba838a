// Test-only operator registration for the reference's own CUDA code.
//
// oracle/build_ref.py compiles the reference's GEMM, permute and unpermute
// sources (csrc/int8_hybrid_grouped_gemm.cu, csrc/int8_grouped_gemm.cu,
// csrc/moe_permute_unpermute_op.cu,
// csrc/permute_unpermute_kernels/moe_permute_unpermute_kernel.cu) where they
// lie in the reference tree, together with this file, into
// oracle/_ref/libi8moe_ref.so.  The reference registers its ops from
// csrc/torch_bindings.cpp under the namespace "int8_hybrid_moe", the same
// namespace this repository's product library uses, so that file is not
// compiled; this one registers the host entry points the parity tests need
// under "int8_hybrid_moe_ref" instead.  The prototypes below are the
// reference's host functions (csrc/torch_bindings.cpp:14-60), declared again
// because the reference declares them only in that file.
//
// Not part of the product: only tests/ load the resulting library, as the
// checker of libi8moe.so.
#include <torch/library.h>
#include <torch/types.h>

#include <optional>
#include <string>

void cutlass_int8_grouped_mm_host(torch::Tensor, torch::Tensor, torch::Tensor, double, double,
                                  torch::Tensor, torch::Tensor);
void cutlass_int8_blockwise_hybrid_grouped_host(torch::Tensor, torch::Tensor, torch::Tensor,
                                                torch::Tensor, torch::Tensor, torch::Tensor,
                                                torch::Tensor, torch::Tensor, torch::Tensor,
                                                int64_t, int64_t, std::optional<torch::Tensor>);
void cutlass_int8_blockwise_hybrid_grouped_bias_host(
    torch::Tensor, torch::Tensor, torch::Tensor, torch::Tensor, torch::Tensor, torch::Tensor,
    torch::Tensor, torch::Tensor, torch::Tensor, torch::Tensor, int64_t, int64_t,
    std::optional<torch::Tensor>);
void cutlass_int8_blockwise_hybrid_grouped_small_host(
    torch::Tensor, torch::Tensor, torch::Tensor, torch::Tensor, torch::Tensor, torch::Tensor,
    torch::Tensor, torch::Tensor, torch::Tensor, int64_t, int64_t,
    std::optional<torch::Tensor>);
void cutlass_int8_blockwise_hybrid_grouped_small_bias_host(
    torch::Tensor, torch::Tensor, torch::Tensor, torch::Tensor, torch::Tensor, torch::Tensor,
    torch::Tensor, torch::Tensor, torch::Tensor, torch::Tensor, int64_t, int64_t,
    std::optional<torch::Tensor>);
void moe_permute(const torch::Tensor& input, const torch::Tensor& topk_ids,
                 const torch::Tensor& token_expert_indices,
                 const std::optional<torch::Tensor>& expert_map, int64_t n_expert,
                 int64_t n_local_expert, int64_t topk, torch::Tensor& permuted_input,
                 torch::Tensor& expert_first_token_offset, torch::Tensor& inv_permuted_idx,
                 torch::Tensor& permuted_idx);
void moe_permute_metadata(const torch::Tensor& topk_ids,
                          const torch::Tensor& token_expert_indices,
                          const std::optional<torch::Tensor>& expert_map, int64_t n_expert,
                          int64_t n_local_expert, int64_t topk,
                          torch::Tensor& expert_first_token_offset,
                          torch::Tensor& inv_permuted_idx, torch::Tensor& permuted_idx);
void moe_unpermute(const torch::Tensor& permuted_hidden_states,
                   const torch::Tensor& topk_weights, const torch::Tensor& inv_permuted_idx,
                   const std::optional<torch::Tensor>& expert_first_token_offset,
                   int64_t topk, torch::Tensor& hidden_states);

TORCH_LIBRARY(int8_hybrid_moe_ref, m) {
  m.def("grouped_mm(Tensor a, Tensor b, Tensor(a!) out, float a_scale, float b_scale, "
        "Tensor expert_offsets, Tensor problem_sizes) -> ()");
  m.impl("grouped_mm", torch::kCUDA, &cutlass_int8_grouped_mm_host);
  const char* hy =
      "(Tensor a_q, Tensor a_qscale, Tensor a_fscale, Tensor b_q, Tensor b_qscale, "
      "Tensor b_fscale, Tensor expert_offsets, Tensor problem_sizes, Tensor(a!) out, "
      "int quant_block_size, int super_group_size, Tensor? scale_offsets=None) -> ()";
  const char* hyb =
      "(Tensor a_q, Tensor a_qscale, Tensor a_fscale, Tensor b_q, Tensor b_qscale, "
      "Tensor b_fscale, Tensor expert_offsets, Tensor problem_sizes, Tensor(a!) out, "
      "Tensor bias, int quant_block_size, int super_group_size, "
      "Tensor? scale_offsets=None) -> ()";
  m.def((std::string("hybrid") + hy).c_str());
  m.impl("hybrid", torch::kCUDA, &cutlass_int8_blockwise_hybrid_grouped_host);
  m.def((std::string("hybrid_bias") + hyb).c_str());
  m.impl("hybrid_bias", torch::kCUDA, &cutlass_int8_blockwise_hybrid_grouped_bias_host);
  m.def((std::string("hybrid_small") + hy).c_str());
  m.impl("hybrid_small", torch::kCUDA, &cutlass_int8_blockwise_hybrid_grouped_small_host);
  m.def((std::string("hybrid_small_bias") + hyb).c_str());
  m.impl("hybrid_small_bias", torch::kCUDA,
         &cutlass_int8_blockwise_hybrid_grouped_small_bias_host);
  m.def("permute(Tensor input, Tensor topk_ids, Tensor token_expert_indices, "
        "Tensor? expert_map, int n_expert, int n_local_expert, int topk, "
        "Tensor! permuted_input, Tensor! expert_first_token_offset, "
        "Tensor! inv_permuted_idx, Tensor! permuted_idx) -> ()");
  m.impl("permute", torch::kCUDA, &moe_permute);
  m.def("permute_metadata(Tensor topk_ids, Tensor token_expert_indices, Tensor? expert_map, "
        "int n_expert, int n_local_expert, int topk, Tensor! expert_first_token_offset, "
        "Tensor! inv_permuted_idx, Tensor! permuted_idx) -> ()");
  m.impl("permute_metadata", torch::kCUDA, &moe_permute_metadata);
  m.def("unpermute(Tensor permuted_hidden_states, Tensor topk_weights, "
        "Tensor inv_permuted_idx, Tensor? expert_first_token_offset, int topk, "
        "Tensor! hidden_states) -> ()");
  m.impl("unpermute", torch::kCUDA, &moe_unpermute);
}
