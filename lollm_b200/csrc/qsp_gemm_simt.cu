// CUDA-core GEMM c[m,n] = a[m,k]·w[n,k]ᵀ, fp32 accumulation. Used for the fp32 parity
// configurations (tensor cores have no fp32 mode that keeps 1e-4 relative accuracy).
#include "qsp_common.cuh"

namespace qsp {

constexpr int SG_BM = 64, SG_BN = 64, SG_BK = 16;

template <typename T>
__global__ void __launch_bounds__(256) gemm_simt_kernel(const T* __restrict__ a, int64_t lda,
                                                        const T* __restrict__ w, int64_t ldw,
                                                        T* __restrict__ c, int64_t ldc, int m,
                                                        int n, int k, int accumulate) {
  __shared__ float As[SG_BK][SG_BM + 4];
  __shared__ float Ws[SG_BK][SG_BN + 4];
  const int tid = threadIdx.x;
  const int tx = tid % 16, ty = tid / 16;           // 16 x 16 threads, 4 x 4 outputs each
  const int m0 = blockIdx.y * SG_BM, n0 = blockIdx.x * SG_BN;
  float acc[4][4] = {};
  for (int k0 = 0; k0 < k; k0 += SG_BK) {
    // 64 x 16 tiles: 1024 elements each, 4 per thread
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int e = tid + i * 256;
      const int r = e / SG_BK, kk = e % SG_BK;
      const int gm = m0 + r, gn = n0 + r, gk = k0 + kk;
      As[kk][r] = (gm < m && gk < k) ? dt<T>::to_f(a[(int64_t)gm * lda + gk]) : 0.0f;
      Ws[kk][r] = (gn < n && gk < k) ? dt<T>::to_f(w[(int64_t)gn * ldw + gk]) : 0.0f;
    }
    __syncthreads();
#pragma unroll
    for (int kk = 0; kk < SG_BK; ++kk) {
      float av[4], wv[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) av[i] = As[kk][ty * 4 + i];
#pragma unroll
      for (int j = 0; j < 4; ++j) wv[j] = Ws[kk][tx * 4 + j];
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[i][j] = fmaf(av[i], wv[j], acc[i][j]);
    }
    __syncthreads();
  }
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int gm = m0 + ty * 4 + i;
    if (gm >= m) continue;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int gn = n0 + tx * 4 + j;
      if (gn >= n) continue;
      T* p = c + (int64_t)gm * ldc + gn;
      float v = dt<T>::round(acc[i][j]);
      if (accumulate) v = v + dt<T>::to_f(*p);
      *p = dt<T>::from_f(v);
    }
  }
}

int gemm_simt(const void* a, int64_t lda, const void* w, int64_t ldw, void* c, int64_t ldc,
              int64_t m, int64_t n, int64_t k, int dtype, int flags, cudaStream_t st) {
  dim3 grid((unsigned)((n + SG_BN - 1) / SG_BN), (unsigned)((m + SG_BM - 1) / SG_BM));
  QSP_REQUIRE(grid.y <= 65535, "qsp_gemm: m too large for the CUDA-core path");
  QSP_DISPATCH_DTYPE(dtype, T, {
    gemm_simt_kernel<T><<<grid, 256, 0, st>>>((const T*)a, lda, (const T*)w, ldw, (T*)c, ldc,
                                              (int)m, (int)n, (int)k,
                                              (flags & QSP_GEMM_ACCUMULATE) ? 1 : 0);
  });
  return check_launch("qsp_gemm(simt)");
}

}  // namespace qsp
