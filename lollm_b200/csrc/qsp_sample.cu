// Token selection over the vocabulary: row argmax, greedy exact-match verification, the
// lossless p/q speculative sampler and inverse-CDF categorical draws. Per-row work is one CTA
// per row (a vocabulary row is ≤ 1.2 MB, read once or twice from HBM).
#include "qsp_common.cuh"

namespace qsp {

constexpr int SEL_THREADS = 512;

struct ArgBest {
  float v;
  long long i;
};
__device__ __forceinline__ ArgBest arg_better(ArgBest a, ArgBest b) {
  // larger value wins; ties → smaller index (torch.argmax returns the first maximum)
  if (b.v > a.v || (b.v == a.v && b.i < a.i)) return b;
  return a;
}
__device__ __forceinline__ ArgBest warp_argbest(ArgBest best) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    ArgBest other{__shfl_xor_sync(0xffffffffu, best.v, o), __shfl_xor_sync(0xffffffffu, best.i, o)};
    best = arg_better(best, other);
  }
  return best;
}

// Block argmax of one row (blockDim = SEL_THREADS). A 16-byte-aligned row is read with
// 16-byte loads, four in flight per thread; the tail (and unaligned rows) element by element.
template <typename T>
__device__ long long row_argmax(const T* __restrict__ row, int64_t vocab) {
  __shared__ float sv[32];
  __shared__ long long si[32];
  ArgBest best{-INFINITY, LLONG_MAX};
  constexpr int EPV = 16 / (int)sizeof(T);
  int64_t done = 0;
  if ((reinterpret_cast<uintptr_t>(row) & 15) == 0) {
    const int64_t nvec = vocab / EPV;
    const uint4* rv = reinterpret_cast<const uint4*>(row);
    const int64_t bd = blockDim.x;
    for (int64_t v0 = threadIdx.x; v0 < nvec; v0 += 4 * bd) {
      uint4 x[4];
#pragma unroll
      for (int u = 0; u < 4; ++u)
        if (v0 + u * bd < nvec) x[u] = __ldg(rv + v0 + u * bd);
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        if (v0 + u * bd >= nvec) break;
        float f[EPV];
        const uint32_t w[4] = {x[u].x, x[u].y, x[u].z, x[u].w};
        if constexpr (sizeof(T) == 4) {
#pragma unroll
          for (int e = 0; e < 4; ++e) f[e] = __uint_as_float(w[e]);
        } else {
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            f[2 * e] = __uint_as_float(w[e] << 16);
            f[2 * e + 1] = __uint_as_float(w[e] & 0xffff0000u);
          }
        }
        const long long j0 = (v0 + u * bd) * EPV;
#pragma unroll
        for (int e = 0; e < EPV; ++e) best = arg_better(best, ArgBest{f[e], j0 + e});
      }
    }
    done = nvec * EPV;
  }
  for (int64_t j = done + threadIdx.x; j < vocab; j += blockDim.x)
    best = arg_better(best, ArgBest{dt<T>::to_f(row[j]), (long long)j});
  best = warp_argbest(best);
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
  if (lane == 0) { sv[warp] = best.v; si[warp] = best.i; }
  __syncthreads();
  if (warp == 0) {
    best = lane < nw ? ArgBest{sv[lane], si[lane]} : ArgBest{-INFINITY, LLONG_MAX};
    best = warp_argbest(best);
    if (lane == 0) si[0] = best.i == LLONG_MAX ? 0 : best.i;
  }
  __syncthreads();
  return si[0];
}

template <typename T>
__global__ void __launch_bounds__(SEL_THREADS) argmax_kernel(const T* __restrict__ logits, int64_t ld,
                                                             int64_t vocab, int64_t* out,
                                                             int64_t out_stride) {
  const long long i = row_argmax<T>(logits + (int64_t)blockIdx.x * ld, vocab);
  if (threadIdx.x == 0) out[(int64_t)blockIdx.x * out_stride] = i;
}

__global__ void greedy_accept_kernel(int B, int T, const int64_t* __restrict__ amax,
                                     const int64_t* __restrict__ drafts, int64_t dld,
                                     int32_t* accept_n, int64_t* next_tok) {
  const int b = blockIdx.x * blockDim.x + threadIdx.x;
  if (b >= B) return;
  const int k = T - 1;
  int a = 0;
  while (a < k && drafts[(int64_t)b * dld + a] == amax[(int64_t)b * T + a]) ++a;
  accept_n[b] = a;
  next_tok[b] = amax[(int64_t)b * T + a];
}

// Row statistics of softmax(l/τ): stats = {max l, Σ exp((l − max)/τ)}.
template <typename T>
__global__ void __launch_bounds__(SEL_THREADS) softmax_stats_kernel(const T* __restrict__ logits,
                                                                    int64_t ld, int64_t vocab,
                                                                    float inv_temp,
                                                                    float* __restrict__ stats) {
  __shared__ float red[32];
  const T* row = logits + (int64_t)blockIdx.x * ld;
  float m = -INFINITY;
  for (int64_t j = threadIdx.x; j < vocab; j += blockDim.x) m = fmaxf(m, dt<T>::to_f(row[j]));
  m = warp_max(m);
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
  if (lane == 0) red[warp] = m;
  __syncthreads();
  m = warp_max(lane < nw ? red[lane] : -INFINITY);
  float z = 0.f;
  for (int64_t j = threadIdx.x; j < vocab; j += blockDim.x) z += expf((dt<T>::to_f(row[j]) - m) * inv_temp);
  z = block_sum(z, red);
  if (threadIdx.x == 0) {
    stats[2 * blockIdx.x] = m;
    stats[2 * blockIdx.x + 1] = z;
  }
}

template <typename T>
__device__ __forceinline__ float prob_at(const T* row, int64_t x, const float* st, float inv_temp) {
  return expf((dt<T>::to_f(row[x]) - st[0]) * inv_temp) / st[1];
}

// Inverse CDF over non-negative weights w(x), x in [0, vocab): the smallest x whose inclusive
// prefix sum exceeds u·Σw. Each thread owns one contiguous slice; slice sums (fp64) get an
// exclusive scan in shared memory and the owning thread walks its slice. Deterministic for a
// fixed block size. `part` is shared memory of blockDim+1 doubles.
template <typename WF>
__device__ long long block_inverse_cdf(WF weight, int64_t vocab, float u, double* part,
                                       long long* res) {
  const int tid = threadIdx.x, nt = blockDim.x;
  const int64_t per = (vocab + nt - 1) / nt;
  const int64_t lo = min((int64_t)tid * per, vocab), hi = min(lo + per, vocab);
  double s = 0.0;
  long long last_pos = -1;
  for (int64_t x = lo; x < hi; ++x) {
    const float w = weight(x);
    s += (double)w;
    if (w > 0.f) last_pos = x;
  }
  part[tid] = s;
  if (tid == 0) res[0] = -1;
  res[1] = -1;
  __syncthreads();
  if (tid == 0) {
    double run = 0.0;
    for (int i = 0; i < nt; ++i) {
      const double v = part[i];
      part[i] = run;
      run += v;
    }
    part[nt] = run;
  }
  __syncthreads();
  const double target = (double)u * part[nt];
  if (s > 0.0 && part[tid] <= target && target < part[tid] + s) {
    double run = part[tid];
    long long pick = last_pos;
    for (int64_t x = lo; x < hi; ++x) {
      const float w = weight(x);
      run += (double)w;
      if (w > 0.f && run > target) { pick = x; break; }
    }
    res[0] = pick;
  }
  __syncthreads();
  if (res[0] < 0) {  // u·Σw at or past the total (rounding): the last positive-weight index
    if (last_pos >= 0) atomicMax(&res[1], last_pos);
    __syncthreads();
    if (tid == 0) res[0] = res[1] < 0 ? 0 : res[1];
    __syncthreads();
  }
  return res[0];
}

// Per sequence: speculative accept chain, then the residual / bonus draw.
template <typename T>
__global__ void __launch_bounds__(SEL_THREADS) spec_sample_kernel(
    const T* __restrict__ tl, int64_t ld_t, const T* __restrict__ dl, int64_t ld_d, int k,
    int64_t vocab, float inv_temp, const int64_t* __restrict__ drafts, int64_t dld,
    const float* __restrict__ u_acc,
    const float* __restrict__ u_res, const float* __restrict__ tstats, const float* __restrict__ dstats,
    int32_t* accept_n, int64_t* next_tok) {
  __shared__ double part[SEL_THREADS + 1];
  __shared__ long long res[2];
  const int b = blockIdx.x;
  int a = 0;
  for (; a < k; ++a) {
    const int64_t d = drafts[(int64_t)b * dld + a];
    const float p = prob_at(tl + ((int64_t)b * (k + 1) + a) * ld_t, d, tstats + 2 * ((int64_t)b * (k + 1) + a), inv_temp);
    const float q = prob_at(dl + ((int64_t)b * k + a) * ld_d, d, dstats + 2 * ((int64_t)b * k + a), inv_temp);
    if (!(u_acc[(int64_t)b * k + a] * q < p)) break;
  }
  const T* prow = tl + ((int64_t)b * (k + 1) + a) * ld_t;
  const float* pst = tstats + 2 * ((int64_t)b * (k + 1) + a);
  long long pick;
  if (a < k) {
    const T* qrow = dl + ((int64_t)b * k + a) * ld_d;
    const float* qst = dstats + 2 * ((int64_t)b * k + a);
    auto resid = [&](int64_t x) -> float {
      return fmaxf(0.f, prob_at(prow, x, pst, inv_temp) - prob_at(qrow, x, qst, inv_temp));
    };
    pick = block_inverse_cdf(resid, vocab, u_res[b], part, res);
    // p == q everywhere leaves no residual mass: fall back to p
    if (part[SEL_THREADS] <= 0.0) {
      __syncthreads();
      auto pw = [&](int64_t x) -> float { return prob_at(prow, x, pst, inv_temp); };
      pick = block_inverse_cdf(pw, vocab, u_res[b], part, res);
    }
  } else {
    auto pw = [&](int64_t x) -> float { return prob_at(prow, x, pst, inv_temp); };
    pick = block_inverse_cdf(pw, vocab, u_res[b], part, res);
  }
  if (threadIdx.x == 0) {
    accept_n[b] = a;
    next_tok[b] = pick;
  }
}

template <typename T>
__global__ void __launch_bounds__(SEL_THREADS) sample_rows_kernel(const T* __restrict__ logits, int64_t ld,
                                                                  int64_t vocab, float inv_temp,
                                                                  const float* __restrict__ u,
                                                                  const float* __restrict__ stats,
                                                                  int64_t* out, int64_t out_stride) {
  __shared__ double part[SEL_THREADS + 1];
  __shared__ long long res[2];
  const int64_t r = blockIdx.x;
  const T* row = logits + r * ld;
  const float* st = stats + 2 * r;
  auto pw = [&](int64_t x) -> float { return prob_at(row, x, st, inv_temp); };
  const long long pick = block_inverse_cdf(pw, vocab, u[r], part, res);
  if (threadIdx.x == 0) out[r * out_stride] = pick;
}

}  // namespace qsp

using namespace qsp;

extern "C" {

size_t qsp_select_workspace_bytes(int64_t rows, int64_t vocab) {
  (void)vocab;
  return (size_t)rows * 2 * sizeof(float) + (size_t)rows * sizeof(int64_t) + 64;
}

int qsp_argmax_rows(const void* logits, int64_t ld, int64_t rows, int64_t vocab, int64_t* out,
                    int64_t out_stride, int dtype, void* stream) {
  QSP_REQUIRE(logits && out && out_stride >= 1, "qsp_argmax_rows: null pointer / bad stride");
  QSP_REQUIRE(rows >= 0 && rows < (1ll << 31) && vocab > 0 && ld >= vocab, "qsp_argmax_rows: bad shape");
  if (rows == 0) return QSP_OK;
  QSP_DISPATCH_DTYPE(dtype, T, {
    argmax_kernel<T><<<(unsigned)rows, SEL_THREADS, 0, as_stream(stream)>>>((const T*)logits, ld, vocab, out,
                                                                            out_stride);
  });
  return check_launch("qsp_argmax_rows");
}

int qsp_greedy_verify(const void* logits, int64_t ld, int32_t batch, int32_t tokens, int64_t vocab,
                      const int64_t* drafts, int64_t drafts_ld, int32_t* accept_n,
                      int64_t* next_tok, int64_t* argmax_out, float* workspace, int dtype,
                      void* stream) {
  QSP_REQUIRE(logits && accept_n && next_tok, "qsp_greedy_verify: null pointer");
  QSP_REQUIRE(batch > 0 && tokens >= 1 && vocab > 0 && ld >= vocab, "qsp_greedy_verify: bad shape");
  QSP_REQUIRE(tokens == 1 || drafts != nullptr, "qsp_greedy_verify: drafts required when tokens > 1");
  int64_t* amax = argmax_out;
  if (amax == nullptr) {
    QSP_REQUIRE(workspace != nullptr && aligned(workspace, 8), "qsp_greedy_verify: need argmax_out or a workspace");
    amax = reinterpret_cast<int64_t*>(workspace);
  }
  const int64_t rows = (int64_t)batch * tokens;
  cudaStream_t st = as_stream(stream);
  QSP_DISPATCH_DTYPE(dtype, T, {
    argmax_kernel<T><<<(unsigned)rows, SEL_THREADS, 0, st>>>((const T*)logits, ld, vocab, amax, 1);
  });
  int rc = check_launch("qsp_greedy_verify(argmax)");
  if (rc) return rc;
  greedy_accept_kernel<<<(batch + 127) / 128, 128, 0, st>>>(batch, tokens, amax, drafts, drafts_ld,
                                                            accept_n, next_tok);
  return check_launch("qsp_greedy_verify(accept)");
}

int qsp_spec_sample(const void* target_logits, int64_t ld_t, const void* draft_logits, int64_t ld_d,
                    int32_t batch, int32_t k, int64_t vocab, float temperature, const int64_t* drafts,
                    int64_t drafts_ld, const float* u_accept, const float* u_resample,
                    int32_t* accept_n, int64_t* next_tok, float* workspace, int dtype,
                    void* stream) {
  QSP_REQUIRE(target_logits && accept_n && next_tok && u_resample && workspace, "qsp_spec_sample: null pointer");
  QSP_REQUIRE(batch > 0 && k >= 0 && vocab > 0 && ld_t >= vocab, "qsp_spec_sample: bad shape");
  QSP_REQUIRE(k == 0 || (draft_logits && drafts && u_accept && ld_d >= vocab), "qsp_spec_sample: drafts missing");
  QSP_REQUIRE(temperature > 0.f, "qsp_spec_sample: temperature must be > 0 (use qsp_greedy_verify)");
  const float inv_t = 1.0f / temperature;
  const int64_t trows = (int64_t)batch * (k + 1), drows = (int64_t)batch * k;
  float* tstats = workspace;
  float* dstats = workspace + 2 * trows;
  cudaStream_t st = as_stream(stream);
  QSP_DISPATCH_DTYPE(dtype, T, {
    softmax_stats_kernel<T><<<(unsigned)trows, SEL_THREADS, 0, st>>>((const T*)target_logits, ld_t, vocab, inv_t, tstats);
    if (drows > 0)
      softmax_stats_kernel<T><<<(unsigned)drows, SEL_THREADS, 0, st>>>((const T*)draft_logits, ld_d, vocab, inv_t, dstats);
    int rc = check_launch("qsp_spec_sample(stats)");
    if (rc) return rc;
    spec_sample_kernel<T><<<batch, SEL_THREADS, 0, st>>>((const T*)target_logits, ld_t, (const T*)draft_logits,
                                                         ld_d, k, vocab, inv_t, drafts, drafts_ld, u_accept,
                                                         u_resample,
                                                         tstats, dstats, accept_n, next_tok);
  });
  return check_launch("qsp_spec_sample");
}

int qsp_sample_rows(const void* logits, int64_t ld, int64_t rows, int64_t vocab, float temperature,
                    const float* u, int64_t* out, int64_t out_stride, float* workspace, int dtype,
                    void* stream) {
  QSP_REQUIRE(logits && out, "qsp_sample_rows: null pointer");
  QSP_REQUIRE(rows >= 0 && rows < (1ll << 31) && vocab > 0 && ld >= vocab, "qsp_sample_rows: bad shape");
  if (rows == 0) return QSP_OK;
  if (temperature <= 0.f) return qsp_argmax_rows(logits, ld, rows, vocab, out, out_stride, dtype, stream);
  QSP_REQUIRE(u && workspace, "qsp_sample_rows: uniforms and workspace required");
  const float inv_t = 1.0f / temperature;
  cudaStream_t st = as_stream(stream);
  QSP_DISPATCH_DTYPE(dtype, T, {
    softmax_stats_kernel<T><<<(unsigned)rows, SEL_THREADS, 0, st>>>((const T*)logits, ld, vocab, inv_t, workspace);
    sample_rows_kernel<T><<<(unsigned)rows, SEL_THREADS, 0, st>>>((const T*)logits, ld, vocab, inv_t, u, workspace,
                                                                  out, out_stride);
  });
  return check_launch("qsp_sample_rows");
}

}  // extern "C"
