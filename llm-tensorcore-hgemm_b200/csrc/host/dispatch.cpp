// Output contract, implementation-name resolution and launch on the current
// stream (reference csrc/dispatch.cpp:18-128). Every launch goes through the
// C ABI (hgemm_sm100_run); a non-zero status becomes a RuntimeError.
#include <c10/cuda/CUDAGuard.h>
#include <c10/cuda/CUDAStream.h>

#include "hgemm.h"
#include "hgemm_sm100.h"

namespace {

void validate_output(const torch::Tensor& out, const HgemmProblem& problem, const torch::Tensor& a,
                     torch::ScalarType dtype, const char* dtype_name, int64_t out_cols) {
    TORCH_CHECK(out.is_cuda(), "out must be a CUDA tensor");
    TORCH_CHECK(out.device() == a.device(), "out must be on the same CUDA device as a and b");
    TORCH_CHECK(out.scalar_type() == dtype, "out must have dtype ", dtype_name);
    TORCH_CHECK(out.dim() == 2, "out must be two-dimensional");
    TORCH_CHECK(out.size(0) == problem.m && out.size(1) == out_cols, "out must have shape [",
                problem.m, ", ", out_cols, "]");
    TORCH_CHECK(out.is_contiguous(), "out must be contiguous row-major");
}

// Fused epilogue: the name's terms joined by '+' (each at most once), and the
// operand tensors they need.
struct Epilogue {
    int32_t bits = 0;
    torch::Tensor bias, residual;
};

Epilogue parse_epilogue(const std::string& name, const HgemmProblem& p, const torch::Tensor& a,
                        const std::optional<torch::Tensor>& bias, const std::optional<torch::Tensor>& residual) {
    Epilogue e;
    if (name != "none") {
        size_t start = 0;
        while (true) {
            const size_t end = name.find('+', start);
            const std::string term = name.substr(start, end == std::string::npos ? std::string::npos : end - start);
            const int32_t bit = term == "bias"       ? HGEMM_SM100_EPI_BIAS
                                : term == "residual" ? HGEMM_SM100_EPI_RESIDUAL
                                : term == "silu_mul" ? HGEMM_SM100_EPI_SILU_MUL
                                                     : 0;
            TORCH_CHECK(bit != 0 && !(e.bits & bit), "unsupported HGEMM epilogue '", name,
                        "' (none, bias, residual, bias+residual, silu_mul, bias+silu_mul)");
            e.bits |= bit;
            if (end == std::string::npos) break;
            start = end + 1;
        }
        TORCH_CHECK(!((e.bits & HGEMM_SM100_EPI_RESIDUAL) && (e.bits & HGEMM_SM100_EPI_SILU_MUL)),
                    "unsupported HGEMM epilogue '", name, "': residual does not combine with silu_mul");
    }
    const bool want_bias = e.bits & HGEMM_SM100_EPI_BIAS, want_res = e.bits & HGEMM_SM100_EPI_RESIDUAL;
    TORCH_CHECK(want_bias == bias.has_value(), want_bias ? "epilogue '" + name + "' needs a bias tensor"
                                                         : "bias given but epilogue '" + name + "' has no bias term");
    TORCH_CHECK(want_res == residual.has_value(),
                want_res ? "epilogue '" + name + "' needs a residual tensor"
                         : "residual given but epilogue '" + name + "' has no residual term");
    if (want_bias) {
        const torch::Tensor& t = *bias;
        TORCH_CHECK(t.is_cuda() && t.device() == a.device(), "bias must be on the same CUDA device as a and b");
        TORCH_CHECK(t.scalar_type() == torch::kFloat16, "bias must have dtype torch.float16");
        TORCH_CHECK(t.dim() == 1 && t.size(0) == p.n && t.is_contiguous(), "bias must be a contiguous [", p.n,
                    "] tensor");
        e.bias = t;
    }
    if (want_res) {
        const torch::Tensor& t = *residual;
        TORCH_CHECK(t.is_cuda() && t.device() == a.device(), "residual must be on the same CUDA device as a and b");
        TORCH_CHECK(t.scalar_type() == torch::kFloat16, "residual must have dtype torch.float16");
        TORCH_CHECK(t.dim() == 2 && t.size(0) == p.m && t.size(1) == p.n && t.stride(1) == 1 &&
                        t.stride(0) >= p.n,
                    "residual must be a [", p.m, ", ", p.n, "] tensor with unit column stride");
        e.residual = t;
    }
    if (e.bits & HGEMM_SM100_EPI_SILU_MUL)
        TORCH_CHECK(p.n % 2 == 0, "epilogue silu_mul needs an even N (gate/up column pairs), got N=", p.n);
    return e;
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
         int32_t cfg, int32_t flags, const Epilogue& epi = Epilogue{}) {
    const c10::cuda::CUDAGuard device_guard(a.device());
    const cudaStream_t stream = c10::cuda::getCurrentCUDAStream(p.device).stream();
    HgemmSm100Args args = make_args(a, b, out, p, cfg, flags);
    args.epilogue = epi.bits;
    if (epi.bits & HGEMM_SM100_EPI_SILU_MUL) args.ldc = p.n / 2;
    if (epi.bias.defined()) args.bias = epi.bias.data_ptr();
    if (epi.residual.defined()) {
        args.residual = epi.residual.data_ptr();
        args.ldr = epi.residual.stride(0);
    }
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
                    const std::string& epilogue, const std::optional<torch::Tensor>& bias,
                    const std::optional<torch::Tensor>& residual) {
    const auto problem = validate_hgemm_inputs(a, b);
    const bool silu = epilogue.find("silu_mul") != std::string::npos;
    auto out = torch::empty({problem.m, silu && problem.n % 2 == 0 ? problem.n / 2 : problem.n}, a.options());
    hgemm_out(a, b, out, implementation, epilogue, bias, residual);
    return out;
}

void hgemm_out(const torch::Tensor& a, const torch::Tensor& b, torch::Tensor out,
               const std::string& implementation, const std::string& epilogue,
               const std::optional<torch::Tensor>& bias, const std::optional<torch::Tensor>& residual) {
    const auto problem = validate_hgemm_inputs(a, b);
    const Epilogue epi = parse_epilogue(epilogue, problem, a, bias, residual);
    validate_output(out, problem, a, torch::kFloat16, "torch.float16",
                    (epi.bits & HGEMM_SM100_EPI_SILU_MUL) ? problem.n / 2 : problem.n);
    const int32_t cfg = config_id(implementation);
    run(a, b, out, problem, cfg, 0, epi);
}

void hgemm_out_f32(const torch::Tensor& a, const torch::Tensor& b, torch::Tensor out,
                   const std::string& implementation) {
    const auto problem = validate_hgemm_inputs(a, b);
    validate_output(out, problem, a, torch::kFloat32, "torch.float32", problem.n);
    const int32_t cfg = config_id(implementation);
    run(a, b, out, problem, cfg, HGEMM_SM100_FLAG_OUT_F32);
}

bool has_cutlass() { return false; }

std::map<std::string, int64_t> backend_info(const std::string& implementation, int64_t m, int64_t n, int64_t k) {
    const int32_t cfg = config_id(implementation);
    // Without a shape (the reference's form) there is no workspace to
    // report; with one, the bytes an aligned problem of that shape takes on
    // the current device (stream-K partial slots, split-K exchange slots).
    const bool shaped = m > 0 && n > 0 && k > 0;
    const int64_t ws = shaped ? static_cast<int64_t>(hgemm_sm100_workspace_bytes(cfg, m, n, k)) : 0;
    return {{"algorithm_id", -1}, {"workspace_bytes", ws}};
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
