// Output contract, implementation-name resolution and launch on the current
// stream (reference csrc/dispatch.cpp:18-128). Every launch goes through the
// C ABI (hgemm_sm100_run); a non-zero status becomes a RuntimeError.
#include <c10/cuda/CUDAGuard.h>
#include <c10/cuda/CUDAStream.h>

#include "hgemm.h"
#include "hgemm_sm100.h"

namespace {

void validate_output(const torch::Tensor& out, const HgemmProblem& problem, const torch::Tensor& a,
                     torch::ScalarType dtype, const char* dtype_name) {
    TORCH_CHECK(out.is_cuda(), "out must be a CUDA tensor");
    TORCH_CHECK(out.device() == a.device(), "out must be on the same CUDA device as a and b");
    TORCH_CHECK(out.scalar_type() == dtype, "out must have dtype ", dtype_name);
    TORCH_CHECK(out.dim() == 2, "out must be two-dimensional");
    TORCH_CHECK(out.size(0) == problem.m && out.size(1) == problem.n, "out must have shape [",
                problem.m, ", ", problem.n, "]");
    TORCH_CHECK(out.is_contiguous(), "out must be contiguous row-major");
}

int32_t config_id(const std::string& implementation) {
    const int32_t id = hgemm_sm100_config_from_name(implementation.c_str());
    TORCH_CHECK(id >= 0, "unknown implementation: ", implementation);
    return id;
}

HgemmSm100Args make_args(const torch::Tensor& a, const torch::Tensor& b, const torch::Tensor& out,
                         const HgemmProblem& p, int32_t cfg, int32_t flags) {
    HgemmSm100Args args{};
    args.a = a.data_ptr();
    args.b = b.data_ptr();
    args.c = out.defined() ? out.data_ptr() : nullptr;
    args.m = p.m;
    args.n = p.n;
    args.k = p.k;
    args.lda = p.k;
    args.ldb = p.n;
    args.ldc = p.n;
    args.config = cfg;
    args.split_k = 0;
    args.flags = flags;
    args.status = nullptr;
    args.timeout_ns = 0;
    args.workspace = nullptr;
    args.workspace_bytes = 0;
    return args;
}

void run(const torch::Tensor& a, const torch::Tensor& b, torch::Tensor& out, const HgemmProblem& p,
         int32_t cfg, int32_t flags) {
    const c10::cuda::CUDAGuard device_guard(a.device());
    const cudaStream_t stream = c10::cuda::getCurrentCUDAStream(p.device).stream();
    HgemmSm100Args args = make_args(a, b, out, p, cfg, flags);
    // Operands TMA cannot describe (offset views; pitches not a multiple of 8
    // halves) are staged in a workspace from the caching allocator. It is
    // allocated on the current stream, so its reuse is stream-ordered after
    // the kernels that read it.
    torch::Tensor workspace;
    const size_t ws = hgemm_sm100_workspace_size(&args);
    if (ws > 0) {
        workspace = torch::empty({static_cast<int64_t>(ws)},
                                 torch::TensorOptions().dtype(torch::kUInt8).device(a.device()));
        args.workspace = workspace.data_ptr();
        args.workspace_bytes = ws;
    }
    const int rc = hgemm_sm100_run(&args, stream);
    TORCH_CHECK(rc == HGEMM_SM100_OK, "hgemm_sm100_run failed: ", hgemm_sm100_status_string(rc));
}

}  // namespace

torch::Tensor hgemm(const torch::Tensor& a, const torch::Tensor& b, const std::string& implementation,
                    const std::string& epilogue) {
    const auto problem = validate_hgemm_inputs(a, b);
    auto out = torch::empty({problem.m, problem.n}, a.options());
    hgemm_out(a, b, out, implementation, epilogue);
    return out;
}

void hgemm_out(const torch::Tensor& a, const torch::Tensor& b, torch::Tensor out,
               const std::string& implementation, const std::string& epilogue) {
    const auto problem = validate_hgemm_inputs(a, b);
    validate_output(out, problem, a, torch::kFloat16, "torch.float16");
    TORCH_CHECK(epilogue == "none", "HGEMM supports only epilogue='none'");
    const int32_t cfg = config_id(implementation);
    run(a, b, out, problem, cfg, 0);
}

void hgemm_out_f32(const torch::Tensor& a, const torch::Tensor& b, torch::Tensor out,
                   const std::string& implementation) {
    const auto problem = validate_hgemm_inputs(a, b);
    validate_output(out, problem, a, torch::kFloat32, "torch.float32");
    const int32_t cfg = config_id(implementation);
    run(a, b, out, problem, cfg, HGEMM_SM100_FLAG_OUT_F32);
}

bool has_cutlass() { return false; }

std::map<std::string, int64_t> backend_info(const std::string& implementation) {
    const int32_t cfg = config_id(implementation);
    return {{"algorithm_id", -1},
            {"workspace_bytes", static_cast<int64_t>(hgemm_sm100_workspace_bytes(cfg, 0, 0, 0))}};
}

std::vector<std::string> implementations() {
    std::vector<std::string> names;
    for (int32_t i = 0; i < hgemm_sm100_num_configs(); ++i) names.emplace_back(hgemm_sm100_config_name(i));
    return names;
}

std::tuple<std::string, int64_t> resolve(const torch::Tensor& a, const torch::Tensor& b,
                                         const std::string& implementation) {
    const auto problem = validate_hgemm_inputs(a, b);
    const int32_t cfg = config_id(implementation);
    const c10::cuda::CUDAGuard device_guard(a.device());
    torch::Tensor none;
    HgemmSm100Args args = make_args(a, b, none, problem, cfg, 0);
    args.c = a.data_ptr();  // only checked for non-null; nothing is launched
    // As hgemm_out would: a staging workspace whenever one is needed (its
    // address is not used by resolution).
    args.workspace_bytes = hgemm_sm100_workspace_size(&args);
    if (args.workspace_bytes > 0) args.workspace = reinterpret_cast<void*>(uintptr_t{256});
    int32_t resolved = 0, split = 0;
    const int rc = hgemm_sm100_resolve(&args, &resolved, &split);
    TORCH_CHECK(rc == HGEMM_SM100_OK, "hgemm_sm100_resolve failed: ", hgemm_sm100_status_string(rc));
    return {hgemm_sm100_config_name(resolved), split};
}
