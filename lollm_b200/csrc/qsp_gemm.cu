// qsp_gemm entry point: argument checks and the choice of kernel for the dtype.
// bf16 → tcgen05 tensor-core kernel (qsp_gemm_tc.cu); fp32 → CUDA-core kernel
// (qsp_gemm_simt.cu), which keeps the fp32 parity configurations within 1e-4.
#include "qsp_common.cuh"

namespace qsp {
int gemm_simt(const void* a, int64_t lda, const void* w, int64_t ldw, void* c, int64_t ldc,
              int64_t m, int64_t n, int64_t k, int dtype, int flags, cudaStream_t st);
int gemm_tc(const void* a, int64_t lda, const void* w, int64_t ldw, void* c, int64_t ldc, int64_t m,
            int64_t n, int64_t k, int flags, void* workspace, size_t ws_bytes, cudaStream_t st);
size_t gemm_tc_workspace(int64_t m, int64_t n, int64_t k);
}  // namespace qsp

using namespace qsp;

extern "C" size_t qsp_gemm_workspace_bytes(int64_t m, int64_t n, int64_t k, int dtype) {
  if (dtype != QSP_BF16 || m <= 0 || n <= 0 || k <= 0) return 0;
  return gemm_tc_workspace(m, n, k);
}

extern "C" int qsp_gemm(const void* a, int64_t lda, const void* w, int64_t ldw, void* c,
                        int64_t ldc, int64_t m, int64_t n, int64_t k, int dtype, int flags,
                        void* workspace, size_t workspace_bytes, void* stream) {
  QSP_REQUIRE(a && w && c, "qsp_gemm: null pointer");
  QSP_REQUIRE(m >= 0 && n > 0 && k > 0, "qsp_gemm: bad shape m=%lld n=%lld k=%lld", (long long)m,
              (long long)n, (long long)k);
  QSP_REQUIRE(lda >= k && ldw >= k && ldc >= n, "qsp_gemm: leading dimension too small");
  QSP_REQUIRE(m < (1ll << 31) && n < (1ll << 31), "qsp_gemm: shape too large");
  if (m == 0) return QSP_OK;
  cudaStream_t st = as_stream(stream);
  if (dtype == QSP_BF16) {
    const int rc = gemm_tc(a, lda, w, ldw, c, ldc, m, n, k, flags, workspace, workspace_bytes, st);
    if (rc != QSP_ERR_UNSUPPORTED) return rc;
  }
  return gemm_simt(a, lda, w, ldw, c, ldc, m, n, k, dtype, flags, st);
}
