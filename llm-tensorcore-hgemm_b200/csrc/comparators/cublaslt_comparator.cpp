// Benchmark-only comparator: cuBLASLt FP16 GEMM with FP32 compute on the
// current stream. It is what the reference's `auto` meant
// (csrc/references/cublaslt_ref.cu:181-206: first heuristic result cached per
// shape, 32 MiB workspace, per thread and device). Here it is never reachable
// from llm_hgemm.hgemm: bench.py calls it to report the ratio to cuBLASLt.
#include <c10/cuda/CUDAGuard.h>
#include <c10/cuda/CUDAStream.h>
#include <cublasLt.h>
#include <torch/extension.h>

#include <map>
#include <tuple>

namespace {

constexpr size_t kWorkspaceBytes = 32u << 20;

#define LT_CHECK(expr)                                                                    \
    do {                                                                                  \
        cublasStatus_t _s = (expr);                                                       \
        TORCH_CHECK(_s == CUBLAS_STATUS_SUCCESS, "cuBLASLt call failed (", #expr, "): ", \
                    static_cast<int>(_s));                                                \
    } while (0)

struct Plan {
    cublasLtMatmulDesc_t op = nullptr;
    cublasLtMatrixLayout_t la = nullptr, lb = nullptr, lc = nullptr;
    cublasLtMatmulAlgo_t algo{};
};

struct Context {
    cublasLtHandle_t handle = nullptr;
    torch::Tensor workspace;
    std::map<std::tuple<int64_t, int64_t, int64_t>, Plan> plans;
};

Context& context(int device) {
    thread_local std::map<int, Context> contexts;
    Context& ctx = contexts[device];
    if (ctx.handle == nullptr) {
        LT_CHECK(cublasLtCreate(&ctx.handle));
        ctx.workspace = torch::empty({static_cast<int64_t>(kWorkspaceBytes)},
                                     torch::TensorOptions().dtype(torch::kUInt8).device(torch::kCUDA, device));
    }
    return ctx;
}

// Row-major C[M,N] = A[M,K] B[K,N] is column-major C^T[N,M] = B^T[N,K] A^T[K,M]:
// cuBLASLt's "A" is our B (N x K, ld N), its "B" is our A (K x M, ld K).
Plan& plan(Context& ctx, int64_t m, int64_t n, int64_t k) {
    auto key = std::make_tuple(m, n, k);
    auto it = ctx.plans.find(key);
    if (it != ctx.plans.end()) return it->second;
    Plan p;
    LT_CHECK(cublasLtMatmulDescCreate(&p.op, CUBLAS_COMPUTE_32F, CUDA_R_32F));
    LT_CHECK(cublasLtMatrixLayoutCreate(&p.la, CUDA_R_16F, n, k, n));
    LT_CHECK(cublasLtMatrixLayoutCreate(&p.lb, CUDA_R_16F, k, m, k));
    LT_CHECK(cublasLtMatrixLayoutCreate(&p.lc, CUDA_R_16F, n, m, n));
    cublasLtMatmulPreference_t pref;
    LT_CHECK(cublasLtMatmulPreferenceCreate(&pref));
    size_t ws = kWorkspaceBytes;
    LT_CHECK(cublasLtMatmulPreferenceSetAttribute(pref, CUBLASLT_MATMUL_PREF_MAX_WORKSPACE_BYTES, &ws,
                                                  sizeof(ws)));
    cublasLtMatmulHeuristicResult_t result{};
    int found = 0;
    LT_CHECK(cublasLtMatmulAlgoGetHeuristic(ctx.handle, p.op, p.la, p.lb, p.lc, p.lc, pref, 1, &result,
                                            &found));
    cublasLtMatmulPreferenceDestroy(pref);
    TORCH_CHECK(found > 0, "cuBLASLt found no algorithm for ", m, "x", n, "x", k);
    p.algo = result.algo;
    return ctx.plans.emplace(key, p).first->second;
}

void cublaslt_out(const torch::Tensor& a, const torch::Tensor& b, torch::Tensor out) {
    TORCH_CHECK(a.is_cuda() && b.is_cuda() && out.is_cuda(), "CUDA tensors required");
    TORCH_CHECK(a.scalar_type() == torch::kFloat16 && b.scalar_type() == torch::kFloat16 &&
                    out.scalar_type() == torch::kFloat16,
                "float16 tensors required");
    TORCH_CHECK(a.is_contiguous() && b.is_contiguous() && out.is_contiguous(), "contiguous tensors required");
    TORCH_CHECK(a.dim() == 2 && b.dim() == 2 && a.size(1) == b.size(0), "shape mismatch");
    const int64_t m = a.size(0), k = a.size(1), n = b.size(1);
    TORCH_CHECK(out.size(0) == m && out.size(1) == n, "out shape mismatch");
    const c10::cuda::CUDAGuard guard(a.device());
    Context& ctx = context(a.get_device());
    Plan& p = plan(ctx, m, n, k);
    const float alpha = 1.f, beta = 0.f;
    const cudaStream_t stream = c10::cuda::getCurrentCUDAStream(a.get_device()).stream();
    LT_CHECK(cublasLtMatmul(ctx.handle, p.op, &alpha, b.data_ptr(), p.la, a.data_ptr(), p.lb, &beta,
                            out.data_ptr(), p.lc, out.data_ptr(), p.lc, &p.algo,
                            ctx.workspace.data_ptr(), kWorkspaceBytes, stream));
}

}  // namespace

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
    m.doc() = "benchmark-only cuBLASLt comparator";
    m.def("cublaslt_out", &cublaslt_out, py::arg("a"), py::arg("b"), py::arg("out"));
}
