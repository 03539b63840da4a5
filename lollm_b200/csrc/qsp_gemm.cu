// qsp_gemm entry point: argument checks and the choice of kernel for the shape and dtype.
#include "qsp_common.cuh"

namespace qsp {
int gemm_simt(const void* a, int64_t lda, const void* w, int64_t ldw, void* c, int64_t ldc,
              int64_t m, int64_t n, int64_t k, int dtype, int flags, cudaStream_t st);
}  // namespace qsp

using namespace qsp;

extern "C" int qsp_gemm(const void* a, int64_t lda, const void* w, int64_t ldw, void* c,
                        int64_t ldc, int64_t m, int64_t n, int64_t k, int dtype, int flags,
                        void* stream) {
  QSP_REQUIRE(a && w && c, "qsp_gemm: null pointer");
  QSP_REQUIRE(m >= 0 && n > 0 && k > 0, "qsp_gemm: bad shape m=%lld n=%lld k=%lld", (long long)m,
              (long long)n, (long long)k);
  QSP_REQUIRE(lda >= k && ldw >= k && ldc >= n, "qsp_gemm: leading dimension too small");
  if (m == 0) return QSP_OK;
  return gemm_simt(a, lda, w, ldw, c, ldc, m, n, k, dtype, flags, as_stream(stream));
}
