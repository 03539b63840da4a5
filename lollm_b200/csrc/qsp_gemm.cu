// GEMM entry points: argument checks and the choice of kernel for the dtype.
// bf16 → tcgen05 tensor-core kernel (qsp_gemm_tc.cu); fp32 → CUDA-core kernel
// (qsp_gemm_simt.cu), which keeps the fp32 parity configurations within 1e-4.
// bf16 plain products with 128 < m ≤ 256 rows (the verify step) first try the cluster split-K
// kernel (qsp_gemm_cl.cu: partials reduced through distributed shared memory). Otherwise the
// persistent kernel runs, and the fused
// variants apply the op that follows a projection in the decoder layer (residual add + next
// RMSNorm, or SwiGLU) inside its split-K merge when it splits, and with the standalone kernels
// otherwise: same results either way.
#include <stdlib.h>

#include <algorithm>

#include "qsp_common.cuh"

namespace qsp {
int gemm_simt(const void* a, int64_t lda, const void* w, int64_t ldw, void* c, int64_t ldc,
              int64_t m, int64_t n, int64_t k, int dtype, int flags, cudaStream_t st);
struct GemmEpi {
  int kind;
  const __nv_bfloat16* norm_w;
  __nv_bfloat16* y;
  int64_t ldy;
  float eps;
};
int gemm_tc(const void* a, int64_t lda, const void* w, int64_t ldw, void* c, int64_t ldc, int64_t m,
            int64_t n, int64_t k, int flags, void* workspace, size_t ws_bytes, cudaStream_t st,
            const GemmEpi* epi, int* split_out);
size_t gemm_tc_workspace(int64_t m, int64_t n, int64_t k);
int gemm_cl(const void* a, int64_t lda, const void* w, int64_t ldw, void* c, int64_t ldc, int64_t m, int64_t n,
            int64_t k, int mode, cudaStream_t st);
int gemm_pair(const void* a, int64_t lda, const void* w, int64_t ldw, void* c, int64_t ldc, int64_t m, int64_t n,
              int64_t k, int mode, const void* norm_w, void* y, int64_t ldy, float eps, void* workspace,
              size_t ws_bytes, cudaStream_t st);
size_t gemm_pair_workspace(int64_t m, int64_t n, int64_t k);
int gemm_pair_persistent(const void* a, int64_t lda, const void* w, int64_t ldw, void* c, int64_t ldc, int64_t m,
                         int64_t n, int64_t k, cudaStream_t st);

// Plain verify-row products whose tiles take several rounds (the vocabulary projection) take
// the persistent CTA-pair kernel unless QSP_GEMM_PAIRP=0 (comparisons).
static bool pairp_on() {
  static int v = -1;
  if (v < 0) {
    const char* e = getenv("QSP_GEMM_PAIRP");
    v = e != nullptr ? atoi(e) : 1;
  }
  return v != 0;
}

// Which products take the CTA-pair kernel (bit 0: plain, bit 1: SwiGLU, bit 2: residual +
// RMSNorm). By default plain products at least PAIR_WIDE_N columns wide and the SwiGLU
// projections do. Measured on B200 at 256 rows, with two k-blocks per TMA box:
//   GDN input projection (12352 × 2048): 13.7 µs, against 24.0 on the cluster kernel;
//   attention q|k|v (9216 × 2048): 13.5 µs, against 15.7 on the cluster kernel;
//   MLP gate|up + SwiGLU (12288 × 2048): 19.2 µs, against 23.1 on the split-K kernel + merge.
// The residual + RMSNorm tails stay on the split-K kernel (2048 columns give the pairs too few
// tiles: 21.9 against 12.6 µs, 28.8 against 14.3 µs). QSP_GEMM_PAIR=<bits> applies the pair
// kernel to exactly the products of those kinds instead, for comparisons.
constexpr int64_t PAIR_WIDE_N = 8192;
static int pair_modes() {
  static int v = -2;
  if (v == -2) {
    const char* e = getenv("QSP_GEMM_PAIR");
    v = e != nullptr ? atoi(e) : -1;
  }
  return v;
}
static bool pair_for(int bit, int64_t n) {
  const int v = pair_modes();
  return v < 0 ? ((bit == 1 && n >= PAIR_WIDE_N) || bit == 2) : (v & bit) != 0;
}

}  // namespace qsp

using namespace qsp;

extern "C" size_t qsp_gemm_workspace_bytes(int64_t m, int64_t n, int64_t k, int dtype) {
  if (dtype != QSP_BF16 || m <= 0 || n <= 0 || k <= 0) return 0;
  return std::max(gemm_tc_workspace(m, n, k), gemm_pair_workspace(m, n, k));
}

static int check_gemm_args(const void* a, const void* w, const void* c, int64_t m, int64_t n, int64_t k,
                           int64_t lda, int64_t ldw, int64_t ldc) {
  QSP_REQUIRE(a && w && c, "qsp_gemm: null pointer");
  QSP_REQUIRE(m >= 0 && n > 0 && k > 0, "qsp_gemm: bad shape m=%lld n=%lld k=%lld", (long long)m,
              (long long)n, (long long)k);
  QSP_REQUIRE(lda >= k && ldw >= k && ldc >= n, "qsp_gemm: leading dimension too small");
  QSP_REQUIRE(m < (1ll << 31) && n < (1ll << 31), "qsp_gemm: shape too large");
  return QSP_OK;
}

// product into c; *fused = 1 if a split-K merge already applied `epi`
static int gemm_any(const void* a, int64_t lda, const void* w, int64_t ldw, void* c, int64_t ldc, int64_t m,
                    int64_t n, int64_t k, int dtype, int flags, void* ws, size_t ws_bytes, cudaStream_t st,
                    const GemmEpi* epi, int* fused) {
  *fused = 0;
  if (dtype == QSP_BF16) {
    // verify-sized rows, plain product: one cluster per output tile, split-K partials reduced
    // on chip. (Measured on B200: faster than the persistent kernel + merge for the wide
    // projections — qkv 16.3 vs 20.6 µs, in_proj 23.9 vs 24.6 µs — and slower for the
    // residual and SwiGLU tails, which therefore keep the persistent kernel.)
    // verify-sized rows: one CTA pair per tile of weight rows, whole K, epilogue in place
    if (flags == 0 && epi == nullptr && pairp_on()) {
      const int rp = gemm_pair_persistent(a, lda, w, ldw, c, ldc, m, n, k, st);
      if (rp != QSP_ERR_UNSUPPORTED) return rp;
    }
    if (flags == 0 && epi == nullptr && pair_for(1, n)) {
      const int rp = gemm_pair(a, lda, w, ldw, c, ldc, m, n, k, 0, nullptr, nullptr, 0, 0.f, ws, ws_bytes, st);
      if (rp != QSP_ERR_UNSUPPORTED) return rp;
    }
    if (epi != nullptr && epi->kind == 2 && flags == 0 && pair_for(2, n)) {
      const int rp = gemm_pair(a, lda, w, ldw, epi->y, epi->ldy, m, n / 2, k, 1, nullptr, nullptr, 0, 0.f, ws,
                               ws_bytes, st);
      if (rp != QSP_ERR_UNSUPPORTED) {
        *fused = rp == QSP_OK;
        return rp;
      }
    }
    if (epi != nullptr && epi->kind == 1 && flags == QSP_GEMM_ACCUMULATE && pair_for(4, n)) {
      const int rp = gemm_pair(a, lda, w, ldw, c, ldc, m, n, k, 2, epi->norm_w, epi->y, epi->ldy, epi->eps, ws,
                               ws_bytes, st);
      if (rp != QSP_ERR_UNSUPPORTED) {
        *fused = rp == QSP_OK;
        return rp;
      }
    }
    if (flags == 0 && epi == nullptr) {
      const int rcl = gemm_cl(a, lda, w, ldw, c, ldc, m, n, k, 0, st);
      if (rcl != QSP_ERR_UNSUPPORTED) return rcl;
    }
    const int rc = gemm_tc(a, lda, w, ldw, c, ldc, m, n, k, flags, ws, ws_bytes, st, epi, fused);
    if (rc != QSP_ERR_UNSUPPORTED) return rc;
    *fused = 0;
  }
  return gemm_simt(a, lda, w, ldw, c, ldc, m, n, k, dtype, flags, st);
}

extern "C" int qsp_gemm(const void* a, int64_t lda, const void* w, int64_t ldw, void* c,
                        int64_t ldc, int64_t m, int64_t n, int64_t k, int dtype, int flags,
                        void* workspace, size_t workspace_bytes, void* stream) {
  int rc = check_gemm_args(a, w, c, m, n, k, lda, ldw, ldc);
  if (rc) return rc;
  if (m == 0) return QSP_OK;
  int fused = 0;
  return gemm_any(a, lda, w, ldw, c, ldc, m, n, k, dtype, flags, workspace, workspace_bytes, as_stream(stream),
                  nullptr, &fused);
}

extern "C" int qsp_gemm_residual_rmsnorm(const void* a, int64_t lda, const void* w, int64_t ldw, void* x,
                                         int64_t ldx, const void* norm_w, void* y, int64_t ldy, int64_t m,
                                         int64_t n, int64_t k, float eps, int dtype, void* workspace,
                                         size_t workspace_bytes, void* stream) {
  int rc = check_gemm_args(a, w, x, m, n, k, lda, ldw, ldx);
  if (rc) return rc;
  QSP_REQUIRE(norm_w && y && ldy >= n, "qsp_gemm_residual_rmsnorm: bad norm weight / output");
  if (m == 0) return QSP_OK;
  GemmEpi epi{1, static_cast<const __nv_bfloat16*>(norm_w), static_cast<__nv_bfloat16*>(y), ldy, eps};
  int fused = 0;
  rc = gemm_any(a, lda, w, ldw, x, ldx, m, n, k, dtype, QSP_GEMM_ACCUMULATE, workspace, workspace_bytes,
                as_stream(stream), &epi, &fused);
  if (rc || fused) return rc;
  return qsp_rmsnorm(x, ldx, norm_w, y, ldy, m, n, eps, dtype, stream);
}

extern "C" int qsp_gemm_swiglu(const void* a, int64_t lda, const void* w_gu, int64_t ldw, void* act,
                               int64_t ld_act, void* gu_tmp, int64_t ld_gu, int64_t m, int64_t inter, int64_t k,
                               int dtype, void* workspace, size_t workspace_bytes, void* stream) {
  int rc = check_gemm_args(a, w_gu, gu_tmp, m, 2 * inter, k, lda, ldw, ld_gu);
  if (rc) return rc;
  QSP_REQUIRE(act && ld_act >= inter, "qsp_gemm_swiglu: bad activation output");
  if (m == 0) return QSP_OK;
  GemmEpi epi{2, nullptr, static_cast<__nv_bfloat16*>(act), ld_act, 0.f};
  int fused = 0;
  rc = gemm_any(a, lda, w_gu, ldw, gu_tmp, ld_gu, m, 2 * inter, k, dtype, 0, workspace, workspace_bytes,
                as_stream(stream), &epi, &fused);
  if (rc || fused) return rc;
  return qsp_swiglu(gu_tmp, ld_gu, act, ld_act, m, inter, dtype, stream);
}
