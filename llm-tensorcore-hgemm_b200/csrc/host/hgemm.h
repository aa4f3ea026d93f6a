// Torch-facing host layer of llm_hgemm._C: the reference's input/output
// contract and name dispatch (reference csrc/hgemm.h:9-34), calling the
// sm_100a kernels only through the C ABI in hgemm_sm100.h.
#pragma once

#include <cstdint>
#include <map>
#include <optional>
#include <string>
#include <tuple>

#include <torch/extension.h>

struct HgemmProblem {
    int64_t m;
    int64_t n;
    int64_t k;
    int device;
};

// Reference csrc/contract.cpp:3-22 (same checks, same messages).
HgemmProblem validate_hgemm_inputs(const torch::Tensor& a, const torch::Tensor& b);

// Reference csrc/dispatch.cpp:37-44. `epilogue` extends the reference's
// "none"-only argument: "bias", "residual", "bias+residual", "silu_mul",
// "bias+silu_mul" (the operand tensors are passed as bias / residual).
torch::Tensor hgemm(const torch::Tensor& a, const torch::Tensor& b,
                    const std::string& implementation, const std::string& epilogue,
                    const std::optional<torch::Tensor>& bias, const std::optional<torch::Tensor>& residual);

// Reference csrc/dispatch.cpp:47-96.
void hgemm_out(const torch::Tensor& a, const torch::Tensor& b, torch::Tensor out,
               const std::string& implementation, const std::string& epilogue,
               const std::optional<torch::Tensor>& bias, const std::optional<torch::Tensor>& residual);

// FP32-output variant for tensor-parallel K-split partials (no reference
// counterpart: the reference is single-GPU).
void hgemm_out_f32(const torch::Tensor& a, const torch::Tensor& b, torch::Tensor out,
                   const std::string& implementation);

// Reference csrc/dispatch.cpp:99-101 (always false: no CUTLASS here).
bool has_cutlass();

// Reference csrc/dispatch.cpp:104-128.
std::map<std::string, int64_t> backend_info(const std::string& implementation, int64_t m = 0, int64_t n = 0,
                                            int64_t k = 0);

// Names of the kernel configurations, in C-ABI id order ("auto" first).
std::vector<std::string> implementations();

// (configuration name, K splits) that `implementation` resolves to for a, b.
std::tuple<std::string, int64_t> resolve(const torch::Tensor& a, const torch::Tensor& b,
                                         const std::string& implementation);
