// libgemm3_b200_cublaslt.so: the same NVFP4 GEMM through cuBLASLt on this GPU, as the vendor
// baseline and a second implementation to compare outputs with. Not used by the gemm3_b200 API;
// declared in include/nvfp4_cublaslt.h.
//
// C[M,N] (row-major) = alpha * dequant(A)[M,K] . dequant(B)[N,K]^T. cuBLASLt is column-major, so
// the call computes C^T = B . A^T: its "A" operand is our B (K x N column-major = [N, K/2]
// row-major bytes, transposed), its "B" operand our A (K x M column-major, not transposed), and
// its D is C^T as N x M column-major = C as [M, N] row-major. The scale tensors keep the 128x4
// swizzled layout, which is the layout cuBLASLt's VEC16_UE4M3 block scaling reads.
#include <cublasLt.h>
#include <cuda_runtime.h>

#include <cstdint>
#include <map>
#include <mutex>
#include <tuple>

#include "../../include/nvfp4_cublaslt.h"

namespace {

struct Plan {
  cublasLtMatmulDesc_t op = nullptr;
  cublasLtMatrixLayout_t la = nullptr, lb = nullptr, lc = nullptr;
  cublasLtMatmulAlgo_t algo{};
  size_t workspace = 0;
};

std::mutex g_mu;
cublasLtHandle_t g_handle[64] = {};
std::map<std::tuple<int, int64_t, int64_t, int64_t, int, int64_t>, Plan> g_plans;
thread_local int g_last_cublas = 0;

// Recorded as 100 * (source line of the failing call) + cublasStatus_t.
int fail(cublasStatus_t s, int line) {
  g_last_cublas = 100 * line + static_cast<int>(s);
  return NVFP4_CUBLASLT_ERR_CUBLAS;
}

#define G3_LT(expr)                                             \
  do {                                                          \
    cublasStatus_t s_ = (expr);                                 \
    if (s_ != CUBLAS_STATUS_SUCCESS) return fail(s_, __LINE__); \
  } while (0)

int make_plan(cublasLtHandle_t h, int64_t m, int64_t n, int64_t k, int out_dtype, int64_t ws_bytes, const void* sfa,
              const void* sfb, Plan* p) {
  G3_LT(cublasLtMatmulDescCreate(&p->op, CUBLAS_COMPUTE_32F, CUDA_R_32F));
  const cublasOperation_t ta = CUBLAS_OP_T, tb = CUBLAS_OP_N;
  G3_LT(cublasLtMatmulDescSetAttribute(p->op, CUBLASLT_MATMUL_DESC_TRANSA, &ta, sizeof(ta)));
  G3_LT(cublasLtMatmulDescSetAttribute(p->op, CUBLASLT_MATMUL_DESC_TRANSB, &tb, sizeof(tb)));
  const cublasLtMatmulMatrixScale_t mode = CUBLASLT_MATMUL_MATRIX_SCALE_VEC16_UE4M3;
  G3_LT(cublasLtMatmulDescSetAttribute(p->op, CUBLASLT_MATMUL_DESC_A_SCALE_MODE, &mode, sizeof(mode)));
  G3_LT(cublasLtMatmulDescSetAttribute(p->op, CUBLASLT_MATMUL_DESC_B_SCALE_MODE, &mode, sizeof(mode)));
  G3_LT(cublasLtMatmulDescSetAttribute(p->op, CUBLASLT_MATMUL_DESC_A_SCALE_POINTER, &sfb, sizeof(sfb)));
  G3_LT(cublasLtMatmulDescSetAttribute(p->op, CUBLASLT_MATMUL_DESC_B_SCALE_POINTER, &sfa, sizeof(sfa)));
  const cudaDataType_t ct = out_dtype == NVFP4_CUBLASLT_BF16 ? CUDA_R_16BF : CUDA_R_16F;
  G3_LT(cublasLtMatrixLayoutCreate(&p->la, CUDA_R_4F_E2M1, k, n, k));
  G3_LT(cublasLtMatrixLayoutCreate(&p->lb, CUDA_R_4F_E2M1, k, m, k));
  G3_LT(cublasLtMatrixLayoutCreate(&p->lc, ct, n, m, n));
  cublasLtMatmulPreference_t pref = nullptr;
  G3_LT(cublasLtMatmulPreferenceCreate(&pref));
  const uint64_t ws = static_cast<uint64_t>(ws_bytes);
  cublasStatus_t s =
      cublasLtMatmulPreferenceSetAttribute(pref, CUBLASLT_MATMUL_PREF_MAX_WORKSPACE_BYTES, &ws, sizeof(ws));
  cublasLtMatmulHeuristicResult_t res{};
  int found = 0;
  if (s == CUBLAS_STATUS_SUCCESS)
    s = cublasLtMatmulAlgoGetHeuristic(h, p->op, p->la, p->lb, p->lc, p->lc, pref, 1, &res, &found);
  cublasLtMatmulPreferenceDestroy(pref);
  if (s != CUBLAS_STATUS_SUCCESS) return fail(s, __LINE__);
  if (found < 1) return NVFP4_CUBLASLT_ERR_NO_ALGO;
  p->algo = res.algo;
  p->workspace = res.workspaceSize;
  return NVFP4_CUBLASLT_OK;
}

}  // namespace

extern "C" {

int nvfp4_cublaslt_gemm(const void* a, const void* b, const void* sfa, const void* sfb, void* c, float alpha,
                        int64_t m, int64_t n, int64_t k, int32_t out_dtype, void* workspace, int64_t workspace_bytes,
                        void* stream) {
  if (!a || !b || !sfa || !sfb || !c || m < 1 || n < 1 || k < 64 || n % 64 || k % 64 || workspace_bytes < 0)
    return NVFP4_CUBLASLT_ERR_INVALID_VALUE;
  if (out_dtype != NVFP4_CUBLASLT_F16 && out_dtype != NVFP4_CUBLASLT_BF16) return NVFP4_CUBLASLT_ERR_INVALID_VALUE;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return NVFP4_CUBLASLT_ERR_CUDA;
  Plan plan;
  cublasLtHandle_t h = nullptr;
  {
    std::lock_guard<std::mutex> lock(g_mu);
    if (g_handle[dev] == nullptr) G3_LT(cublasLtCreate(&g_handle[dev]));
    h = g_handle[dev];
    const auto key = std::make_tuple(dev, m, n, k, static_cast<int>(out_dtype), workspace_bytes);
    auto it = g_plans.find(key);
    if (it == g_plans.end()) {
      Plan fresh;
      const int rc = make_plan(h, m, n, k, out_dtype, workspace_bytes, sfa, sfb, &fresh);
      if (rc != NVFP4_CUBLASLT_OK) return rc;
      it = g_plans.emplace(key, fresh).first;
    }
    plan = it->second;
  }
  // Scale pointers are set per call (the plan is shared by calls with other buffers); the
  // attribute writes touch only the host-side descriptor, under the lock.
  std::lock_guard<std::mutex> lock(g_mu);
  G3_LT(cublasLtMatmulDescSetAttribute(plan.op, CUBLASLT_MATMUL_DESC_A_SCALE_POINTER, &sfb, sizeof(sfb)));
  G3_LT(cublasLtMatmulDescSetAttribute(plan.op, CUBLASLT_MATMUL_DESC_B_SCALE_POINTER, &sfa, sizeof(sfa)));
  const float beta = 0.0f;
  G3_LT(cublasLtMatmul(h, plan.op, &alpha, b, plan.la, a, plan.lb, &beta, c, plan.lc, c, plan.lc, &plan.algo,
                       workspace, static_cast<size_t>(workspace_bytes), static_cast<cudaStream_t>(stream)));
  return NVFP4_CUBLASLT_OK;
}

int32_t nvfp4_cublaslt_last_status(void) { return g_last_cublas; }

}  // extern "C"
