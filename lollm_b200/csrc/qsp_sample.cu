// Token selection over the vocabulary: row argmax, greedy exact-match verification, the
// lossless p/q speculative sampler and inverse-CDF categorical draws. Per-row work is one CTA
// per row (a vocabulary row is ≤ 1.2 MB, read once or twice from HBM), except the argmax of
// few rows, which splits each row over a thread-block cluster.
#include "qsp_common.cuh"

#include <cooperative_groups.h>

namespace qsp {

constexpr int SEL_THREADS = 512;

struct ArgBest {
  float v;
  long long i;
};
// Set when an argmax met a NaN logit (read through qsp_device_status).
__device__ int g_sample_error = 0;

__device__ __forceinline__ ArgBest arg_better(ArgBest a, ArgBest b) {
  // larger value wins; ties → smaller index (torch.argmax returns the first maximum). A NaN
  // ranks above every number, as in torch.argmax, so a row holding NaNs selects its first NaN.
  const bool an = a.v != a.v, bn = b.v != b.v;
  if (an || bn) return (bn && (!an || b.i < a.i)) ? b : a;
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

// NaN-propagating running maxima (PTX max.NaN): they only tell whether a NaN was seen.
__device__ __forceinline__ float fmax_nan(float a, float b) {
  float d;
  asm("max.NaN.f32 %0, %1, %2;" : "=f"(d) : "f"(a), "f"(b));
  return d;
}
__device__ __forceinline__ uint32_t bmax_nan2(uint32_t a, uint32_t b) {
  uint32_t d;
  asm("max.NaN.bf16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
  return d;
}

// Block argmax of one row (blockDim = SEL_THREADS): the best (value, index), index LLONG_MAX
// when no element compares (an all-NaN row). A 16-byte-aligned row is read with 16-byte
// loads, four in flight per thread; the tail (and unaligned rows) element by element. Each
// thread visits its elements in increasing index order, so a strict `>` keeps its first
// maximum; threads combine with ties going to the smaller index. A NaN-propagating max runs
// alongside; when the row holds a NaN (rare) the row is scanned again for its first NaN,
// which is the result (torch.argmax ranks NaN above every number). vocab < 2^31.
template <typename T>
__device__ ArgBest row_argbest(const T* __restrict__ row, int64_t vocab) {
  __shared__ float sv[32];
  __shared__ long long si[32];
  float bv = -INFINITY;
  int bi = INT_MAX;
  float nanmax = -INFINITY;
  uint32_t nan2 = 0xff80ff80u;   // two bf16 -inf
  constexpr int EPV = 16 / (int)sizeof(T);
  int64_t done = 0;
  if ((reinterpret_cast<uintptr_t>(row) & 15) == 0) {
    const int nvec = (int)(vocab / EPV);
    const uint4* rv = reinterpret_cast<const uint4*>(row);
    const int bd = blockDim.x;
    for (int v0 = threadIdx.x; v0 < nvec; v0 += 4 * bd) {
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
          for (int e = 0; e < 4; ++e) {
            f[e] = __uint_as_float(w[e]);
            nanmax = fmax_nan(nanmax, f[e]);
          }
        } else {
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            f[2 * e] = __uint_as_float(w[e] << 16);
            f[2 * e + 1] = __uint_as_float(w[e] & 0xffff0000u);
            nan2 = bmax_nan2(nan2, w[e]);
          }
        }
        const int j0 = (v0 + u * bd) * EPV;
#pragma unroll
        for (int e = 0; e < EPV; ++e)
          if (f[e] > bv) { bv = f[e]; bi = j0 + e; }
      }
    }
    done = (int64_t)nvec * EPV;
  }
  for (int64_t j = done + threadIdx.x; j < vocab; j += blockDim.x) {
    const float f = dt<T>::to_f(row[j]);
    nanmax = fmax_nan(nanmax, f);
    if (f > bv) { bv = f; bi = (int)j; }
  }
  const bool has_nan = nanmax != nanmax || __uint_as_float(nan2 << 16) != __uint_as_float(nan2 << 16) ||
                       __uint_as_float(nan2 & 0xffff0000u) != __uint_as_float(nan2 & 0xffff0000u);
  ArgBest best{bv, bi == INT_MAX ? LLONG_MAX : (long long)bi};
  if (__syncthreads_or(has_nan)) {   // rare: the first NaN of the row
    long long first = LLONG_MAX;
    for (int64_t j = threadIdx.x; j < vocab; j += blockDim.x) {
      const float f = dt<T>::to_f(row[j]);
      if (f != f) { first = j; break; }
    }
    best = ArgBest{__int_as_float(0x7fffffff), first};   // NaN, or (NaN, LLONG_MAX): no NaN here
  }
  best = warp_argbest(best);
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
  if (lane == 0) { sv[warp] = best.v; si[warp] = best.i; }
  __syncthreads();
  if (warp == 0) {
    best = lane < nw ? ArgBest{sv[lane], si[lane]} : ArgBest{-INFINITY, LLONG_MAX};
    best = warp_argbest(best);
    if (lane == 0) { sv[0] = best.v; si[0] = best.i; }
  }
  __syncthreads();
  const ArgBest r{sv[0], si[0]};
  __syncthreads();   // sv/si are reused by the next call
  return r;
}
template <typename T>
__device__ long long row_argmax(const T* __restrict__ row, int64_t vocab) {
  const ArgBest b = row_argbest<T>(row, vocab);
  if (b.v != b.v && threadIdx.x == 0) atomicExch(&g_sample_error, QSP_DEV_NAN_LOGITS);
  return b.i == LLONG_MAX ? 0 : b.i;
}

template <typename T>
__global__ void __launch_bounds__(SEL_THREADS) argmax_kernel(const T* __restrict__ logits, int64_t ld,
                                                             int64_t vocab, int64_t* out,
                                                             int64_t out_stride) {
  const long long i = row_argmax<T>(logits + (int64_t)blockIdx.x * ld, vocab);
  if (threadIdx.x == 0) out[(int64_t)blockIdx.x * out_stride] = i;
}

// Argmax with S CTAs per row (one thread-block cluster per row): CTA r scans the r-th of S
// 16-byte-aligned chunks and rank 0 combines the S results through distributed shared memory.
// Ties go to the smaller index, as in the one-CTA kernel.
template <typename T, int S>
__global__ void __cluster_dims__(S, 1, 1) __launch_bounds__(SEL_THREADS)
argmax_split_kernel(const T* __restrict__ logits, int64_t ld, int64_t vocab, int64_t* out, int64_t out_stride) {
  namespace cg = cooperative_groups;
  __shared__ float cv;
  __shared__ long long ci;
  cg::cluster_group cl = cg::this_cluster();
  const int rank = (int)cl.block_rank();
  const int64_t row = blockIdx.x / S;
  constexpr int EPV = 16 / (int)sizeof(T);
  const int64_t chunk = ((vocab + S - 1) / S + EPV - 1) / EPV * EPV;
  const int64_t lo = min(vocab, (int64_t)rank * chunk), hi = min(vocab, lo + chunk);
  ArgBest b{-INFINITY, LLONG_MAX};
  if (hi > lo) {
    b = row_argbest<T>(logits + row * ld + lo, hi - lo);
    if (b.i != LLONG_MAX) b.i += lo;
  }
  if (threadIdx.x == 0) {
    cv = b.v;
    ci = b.i;
  }
  cl.sync();
  if (rank == 0 && threadIdx.x == 0) {
    ArgBest best{cv, ci};
    for (int r = 1; r < S; ++r) best = arg_better(best, ArgBest{*cl.map_shared_rank(&cv, r), *cl.map_shared_rank(&ci, r)});
    if (best.v != best.v) atomicExch(&g_sample_error, QSP_DEV_NAN_LOGITS);
    out[row * out_stride] = best.i == LLONG_MAX ? 0 : best.i;
  }
  cl.sync();   // every CTA keeps its shared memory until rank 0 has read it
}

// rows × S CTAs: S (1, 2, 4 or 8) doubles while the grid is under two CTAs per SM and each
// chunk keeps at least 4096 elements.
template <typename T>
static int launch_argmax(const T* logits, int64_t ld, int64_t rows, int64_t vocab, int64_t* out, int64_t out_stride,
                         cudaStream_t st) {
  static int sms = 0;
  if (sms == 0) {
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    if (sms <= 0) sms = 148;
  }
  int S = 1;
  while (S < 8 && rows * S < 2 * sms && vocab / (2 * S) >= 4096) S *= 2;
  const unsigned g = (unsigned)(rows * S);
  switch (S) {
    case 1: argmax_kernel<T><<<g, SEL_THREADS, 0, st>>>(logits, ld, vocab, out, out_stride); break;
    case 2: argmax_split_kernel<T, 2><<<g, SEL_THREADS, 0, st>>>(logits, ld, vocab, out, out_stride); break;
    case 4: argmax_split_kernel<T, 4><<<g, SEL_THREADS, 0, st>>>(logits, ld, vocab, out, out_stride); break;
    default: argmax_split_kernel<T, 8><<<g, SEL_THREADS, 0, st>>>(logits, ld, vocab, out, out_stride); break;
  }
  return check_launch("qsp_argmax_rows");
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
    if (z != z) atomicExch(&g_sample_error, QSP_DEV_NAN_LOGITS);   // a NaN logit poisons Z
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


// ------------------------------------------------------------------ filtered sampling
// The token filters of sample_next (src/generate.py:17-37), row by row: repetition penalty
// over a context, temperature, top-k, top-p. filter_rows_kernel materialises the row's
// penalised, scaled logits w (fp32, rounded to the model dtype after every op the reference
// does in that dtype) and a threshold `thr`: the kept tokens are exactly {j : w[j] ≥ thr}.
// Thresholds come from exact radix selects over the order-preserving 32-bit keys of w: top-k
// is the k-th largest value (ties with it survive, like torch.topk + `<`), top-p is the value
// of the first token, in descending order, at which the cumulative softmax mass exceeds
// top_p (masses as 2^-40 fixed point, so the select is exact and order-independent; tokens
// tied with that value are all kept, where the reference keeps them in sort order).
struct FilterRow {
  float m, z, thr, pad;   // max kept w, Σ_kept e^{w−m}, threshold
};

__device__ __forceinline__ uint32_t fkey(float f) {
  const uint32_t u = __float_as_uint(f);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}
__device__ __forceinline__ float fkey_inv(uint32_t k) {
  return __uint_as_float((k & 0x80000000u) ? (k & 0x7fffffffu) : ~k);
}

constexpr double FIX_SCALE = 1099511627776.0;   // 2^40

template <typename T>
__global__ void __launch_bounds__(SEL_THREADS) filter_rows_kernel(
    const T* __restrict__ logits, int64_t ld, int rows_per_seq, int64_t vocab, qsp_sample_params sp,
    float* __restrict__ wrows, FilterRow* __restrict__ stats, int64_t* __restrict__ amax) {
  __shared__ unsigned long long hist[256];
  __shared__ float red[32];
  __shared__ uint32_t sel_sh;
  __shared__ unsigned long long above_sh, tot_sh;
  const int64_t r = blockIdx.x;
  const int b = (int)(r / rows_per_seq), t = (int)(r % rows_per_seq);
  const T* row = logits + r * ld;
  float* w = wrows + r * vocab;
  const bool greedy = !(sp.temperature > 0.f);
  const int tid = threadIdx.x;
  // 1. w = logits (/ temperature, in the logits dtype), then the penalty on the context
  for (int64_t j = tid; j < vocab; j += blockDim.x) {
    const float x = dt<T>::to_f(row[j]);
    w[j] = greedy ? x : dt<T>::round(x / sp.temperature);
  }
  __syncthreads();
  if (sp.repetition_penalty != 1.f) {
    // context lengths are clamped to the rows they index
    const int nh = sp.hist ? (int)min((int64_t)max(sp.hist_n[b], 0), sp.hist_ld) : 0;
    const int ns = sp.step_ids ? (int)min((int64_t)(sp.step_base + t), sp.step_ld) : 0;
    for (int i = tid; i < nh + ns; i += blockDim.x) {
      const int64_t id = i < nh ? sp.hist[(int64_t)b * sp.hist_ld + i] : sp.step_ids[(int64_t)b * sp.step_ld + (i - nh)];
      if (id < 0 || id >= vocab) continue;
      const float x = dt<T>::to_f(row[id]);
      const float y = dt<T>::round(x > 0.f ? x / sp.repetition_penalty : x * sp.repetition_penalty);
      w[id] = greedy ? y : dt<T>::round(y / sp.temperature);   // duplicates write the same value
    }
  }
  __syncthreads();
  if (greedy) {
    if (amax) {
      const long long i = row_argmax<float>(w, vocab);
      if (tid == 0) amax[r] = i;
    }
    return;
  }
  // 2. top-k: the k-th largest w (radix select over 8-bit digits, most significant first)
  float thr = -INFINITY;
  if (sp.top_k > 0 && sp.top_k < vocab) {
    uint32_t prefix = 0, mask = 0;
    long long kk = sp.top_k;
    for (int shift = 24; shift >= 0; shift -= 8) {
      for (int i = tid; i < 256; i += blockDim.x) hist[i] = 0;
      __syncthreads();
      for (int64_t j = tid; j < vocab; j += blockDim.x) {
        const uint32_t key = fkey(w[j]);
        if ((key & mask) == prefix) atomicAdd(&hist[(key >> shift) & 255u], 1ull);
      }
      __syncthreads();
      if (tid == 0) {
        unsigned long long c = 0;
        uint32_t sel = 0;
        for (int d = 255; d >= 0; --d) {
          if (c + hist[d] >= (unsigned long long)kk) { sel = (uint32_t)d; break; }
          c += hist[d];
        }
        kk -= (long long)c;
        sel_sh = sel;
        above_sh = (unsigned long long)kk;
      }
      __syncthreads();
      prefix |= sel_sh << shift;
      mask |= 255u << shift;
      kk = (long long)above_sh;
      __syncthreads();
    }
    thr = fkey_inv(prefix);
  }
  // 3. max over the kept tokens
  float m = -INFINITY;
  for (int64_t j = tid; j < vocab; j += blockDim.x)
    if (w[j] >= thr) m = fmaxf(m, w[j]);
  m = warp_max(m);
  {
    const int lane = tid & 31, warp = tid >> 5, nw = blockDim.x >> 5;
    if (lane == 0) red[warp] = m;
    __syncthreads();
    m = warp_max(lane < nw ? red[lane] : -INFINITY);
    __syncthreads();
  }
  // 4. top-p: descend the key digits by fixed-point softmax mass
  if (sp.top_p > 0.f && sp.top_p < 1.f && m > -INFINITY) {
    if (tid == 0) tot_sh = 0;
    __syncthreads();
    unsigned long long q = 0;
    for (int64_t j = tid; j < vocab; j += blockDim.x)
      if (w[j] >= thr) q += (unsigned long long)((double)expf(w[j] - m) * FIX_SCALE);
    atomicAdd(&tot_sh, q);
    __syncthreads();
    const unsigned long long tgt = (unsigned long long)((double)sp.top_p * (double)tot_sh);
    if (tgt < tot_sh) {
      uint32_t prefix = 0, mask = 0;
      unsigned long long above = 0;
      for (int shift = 24; shift >= 0; shift -= 8) {
        for (int i = tid; i < 256; i += blockDim.x) hist[i] = 0;
        __syncthreads();
        for (int64_t j = tid; j < vocab; j += blockDim.x) {
          const float x = w[j];
          if (!(x >= thr)) continue;
          const uint32_t key = fkey(x);
          if ((key & mask) == prefix)
            atomicAdd(&hist[(key >> shift) & 255u], (unsigned long long)((double)expf(x - m) * FIX_SCALE));
        }
        __syncthreads();
        if (tid == 0) {
          unsigned long long c = above;
          uint32_t sel = 0;
          for (int d = 255; d >= 0; --d) {
            if (c + hist[d] > tgt) { sel = (uint32_t)d; break; }
            c += hist[d];
          }
          sel_sh = sel;
          above_sh = c;
        }
        __syncthreads();
        prefix |= sel_sh << shift;
        mask |= 255u << shift;
        above = above_sh;
        __syncthreads();
      }
      thr = fmaxf(thr, fkey_inv(prefix));
    }
  }
  // 5. normaliser over the kept tokens
  float z = 0.f;
  for (int64_t j = tid; j < vocab; j += blockDim.x)
    if (w[j] >= thr) z += expf(w[j] - m);
  z = block_sum(z, red);
  if (tid == 0) {
    stats[r] = FilterRow{m, z, thr, 0.f};
    if (z != z) atomicExch(&g_sample_error, QSP_DEV_NAN_LOGITS);
  }
}

__device__ __forceinline__ float filtered_p(const float* w, const FilterRow& s, int64_t x) {
  const float v = w[x];
  return v >= s.thr ? expf(v - s.m) / s.z : 0.f;
}

__global__ void __launch_bounds__(SEL_THREADS) sample_filtered_kernel(const float* __restrict__ wrows, int64_t vocab,
                                                                      const FilterRow* __restrict__ stats,
                                                                      const float* __restrict__ u, int64_t* out,
                                                                      int64_t out_stride) {
  __shared__ double part[SEL_THREADS + 1];
  __shared__ long long res[2];
  const int64_t r = blockIdx.x;
  const float* w = wrows + r * vocab;
  const FilterRow s = stats[r];
  auto pw = [&](int64_t x) -> float { return filtered_p(w, s, x); };
  const long long pick = block_inverse_cdf(pw, vocab, u[r], part, res);
  if (threadIdx.x == 0) out[r * out_stride] = pick;
}

__global__ void amax_copy_kernel(const int64_t* __restrict__ amax, int64_t rows, int64_t* out, int64_t out_stride) {
  const int64_t r = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (r < rows) out[r * out_stride] = amax[r];
}

// Per sequence: speculative accept chain over the filtered p (target) and q (draft) rows,
// then the residual / bonus draw.
__global__ void __launch_bounds__(SEL_THREADS) spec_filtered_kernel(
    const float* __restrict__ tw, const float* __restrict__ dw, int k, int64_t vocab,
    const FilterRow* __restrict__ ts, const FilterRow* __restrict__ ds, const int64_t* __restrict__ drafts,
    int64_t dld, const float* __restrict__ u_acc, const float* __restrict__ u_res, int32_t* accept_n,
    int64_t* next_tok) {
  __shared__ double part[SEL_THREADS + 1];
  __shared__ long long res[2];
  const int b = blockIdx.x;
  int a = 0;
  for (; a < k; ++a) {
    const int64_t d = drafts[(int64_t)b * dld + a];
    const int64_t tr = (int64_t)b * (k + 1) + a, dr = (int64_t)b * k + a;
    const float p = (d >= 0 && d < vocab) ? filtered_p(tw + tr * vocab, ts[tr], d) : 0.f;
    const float q = (d >= 0 && d < vocab) ? filtered_p(dw + dr * vocab, ds[dr], d) : 0.f;
    if (!(u_acc[(int64_t)b * k + a] * q < p)) break;
  }
  const int64_t tr = (int64_t)b * (k + 1) + a;
  const float* pw_row = tw + tr * vocab;
  const FilterRow pst = ts[tr];
  long long pick;
  if (a < k) {
    const int64_t dr = (int64_t)b * k + a;
    const float* qw_row = dw + dr * vocab;
    const FilterRow qst = ds[dr];
    auto resid = [&](int64_t x) -> float { return fmaxf(0.f, filtered_p(pw_row, pst, x) - filtered_p(qw_row, qst, x)); };
    pick = block_inverse_cdf(resid, vocab, u_res[b], part, res);
    if (part[SEL_THREADS] <= 0.0) {   // p == q everywhere leaves no residual mass: draw from p
      __syncthreads();
      auto pw = [&](int64_t x) -> float { return filtered_p(pw_row, pst, x); };
      pick = block_inverse_cdf(pw, vocab, u_res[b], part, res);
    }
  } else {
    auto pw = [&](int64_t x) -> float { return filtered_p(pw_row, pst, x); };
    pick = block_inverse_cdf(pw, vocab, u_res[b], part, res);
  }
  if (threadIdx.x == 0) {
    accept_n[b] = a;
    next_tok[b] = pick;
  }
}

int sample_device_error(int reset) {
  int v = 0;
  if (cudaMemcpyFromSymbol(&v, g_sample_error, sizeof(int)) != cudaSuccess) return 0;
  if (reset && v != 0) {
    const int zero = 0;
    cudaMemcpyToSymbol(g_sample_error, &zero, sizeof(int));
  }
  return v;
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
  QSP_REQUIRE(rows >= 0 && rows < (1ll << 31) && vocab > 0 && vocab < (1ll << 31) && ld >= vocab, "qsp_argmax_rows: bad shape");
  if (rows == 0) return QSP_OK;
  QSP_DISPATCH_DTYPE(dtype, T, { return launch_argmax<T>((const T*)logits, ld, rows, vocab, out, out_stride, as_stream(stream)); });
}

int qsp_greedy_verify(const void* logits, int64_t ld, int32_t batch, int32_t tokens, int64_t vocab,
                      const int64_t* drafts, int64_t drafts_ld, int32_t* accept_n,
                      int64_t* next_tok, int64_t* argmax_out, float* workspace, int dtype,
                      void* stream) {
  QSP_REQUIRE(logits && accept_n && next_tok, "qsp_greedy_verify: null pointer");
  QSP_REQUIRE(batch > 0 && tokens >= 1 && vocab > 0 && vocab < (1ll << 31) && ld >= vocab, "qsp_greedy_verify: bad shape");
  QSP_REQUIRE(tokens == 1 || drafts != nullptr, "qsp_greedy_verify: drafts required when tokens > 1");
  int64_t* amax = argmax_out;
  if (amax == nullptr) {
    QSP_REQUIRE(workspace != nullptr && aligned(workspace, 8), "qsp_greedy_verify: need argmax_out or a workspace");
    amax = reinterpret_cast<int64_t*>(workspace);
  }
  const int64_t rows = (int64_t)batch * tokens;
  cudaStream_t st = as_stream(stream);
  int rc = QSP_OK;
  QSP_DISPATCH_DTYPE(dtype, T, { rc = launch_argmax<T>((const T*)logits, ld, rows, vocab, amax, 1, st); });
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
  QSP_REQUIRE(batch > 0 && k >= 0 && vocab > 0 && vocab < (1ll << 31) && ld_t >= vocab, "qsp_spec_sample: bad shape");
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
  QSP_REQUIRE(rows >= 0 && rows < (1ll << 31) && vocab > 0 && vocab < (1ll << 31) && ld >= vocab, "qsp_sample_rows: bad shape");
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

static size_t filter_layout(int64_t rows, int64_t vocab, size_t* stats_off, size_t* amax_off) {
  size_t off = (size_t)rows * vocab * sizeof(float);
  off = (off + 255) / 256 * 256;
  *stats_off = off;
  off += (size_t)rows * sizeof(FilterRow);
  off = (off + 255) / 256 * 256;
  *amax_off = off;
  off += (size_t)rows * sizeof(int64_t);
  return off;
}

extern "C" size_t qsp_filter_workspace_bytes(int64_t rows, int64_t vocab) {
  if (rows <= 0 || vocab <= 0) return 0;
  size_t a, b;
  return filter_layout(rows, vocab, &a, &b);
}

static int check_params(const qsp_sample_params* sp, const char* who) {
  QSP_REQUIRE(sp != nullptr, "%s: null params", who);
  QSP_REQUIRE(sp->repetition_penalty > 0.f, "%s: repetition_penalty must be > 0", who);
  QSP_REQUIRE(sp->hist == nullptr || (sp->hist_n != nullptr && sp->hist_ld >= 0), "%s: hist needs hist_n", who);
  QSP_REQUIRE(sp->step_ids == nullptr || (sp->step_ld >= 0 && sp->step_base >= 0), "%s: bad step ids", who);
  return QSP_OK;
}

template <typename T>
static int launch_filter(const void* logits, int64_t ld, int64_t rows, int32_t rows_per_seq, int64_t vocab,
                         const qsp_sample_params& sp, float* w, FilterRow* st, int64_t* amax, cudaStream_t s) {
  filter_rows_kernel<T><<<(unsigned)rows, SEL_THREADS, 0, s>>>((const T*)logits, ld, rows_per_seq, vocab, sp, w, st,
                                                                amax);
  return check_launch("qsp filter_rows");
}

extern "C" {

int qsp_sample_filtered(const void* logits, int64_t ld, int64_t rows, int32_t rows_per_seq, int64_t vocab,
                        const qsp_sample_params* params, const float* u, int64_t* out, int64_t out_stride,
                        void* workspace, size_t workspace_bytes, int dtype, void* stream) {
  int rc = check_params(params, "qsp_sample_filtered");
  if (rc) return rc;
  QSP_REQUIRE(logits && out && out_stride >= 1 && rows_per_seq >= 1, "qsp_sample_filtered: null pointer / bad stride");
  QSP_REQUIRE(rows >= 0 && rows < (1ll << 31) && vocab > 0 && vocab < (1ll << 31) && ld >= vocab, "qsp_sample_filtered: bad shape");
  if (rows == 0) return QSP_OK;
  const bool greedy = !(params->temperature > 0.f);
  QSP_REQUIRE(greedy || u != nullptr, "qsp_sample_filtered: uniforms required");
  size_t so, ao;
  const size_t need = filter_layout(rows, vocab, &so, &ao);
  QSP_REQUIRE(workspace && aligned(workspace, 256) && workspace_bytes >= need,
              "qsp_sample_filtered: workspace of %zu bytes (256-byte aligned) required", need);
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  float* w = reinterpret_cast<float*>(ws);
  FilterRow* st = reinterpret_cast<FilterRow*>(ws + so);
  int64_t* amax = reinterpret_cast<int64_t*>(ws + ao);
  cudaStream_t s = as_stream(stream);
  QSP_DISPATCH_DTYPE(dtype, T, { rc = launch_filter<T>(logits, ld, rows, rows_per_seq, vocab, *params, w, st, amax, s); });
  if (rc) return rc;
  if (greedy) {
    amax_copy_kernel<<<(unsigned)((rows + 127) / 128), 128, 0, s>>>(amax, rows, out, out_stride);
    return check_launch("qsp_sample_filtered(argmax)");
  }
  sample_filtered_kernel<<<(unsigned)rows, SEL_THREADS, 0, s>>>(w, vocab, st, u, out, out_stride);
  return check_launch("qsp_sample_filtered");
}

int qsp_spec_sample_filtered(const void* target_logits, int64_t ld_t, const void* draft_logits, int64_t ld_d,
                             int32_t batch, int32_t k, int64_t vocab, const qsp_sample_params* params,
                             const int64_t* drafts, int64_t drafts_ld, const float* u_accept,
                             const float* u_resample, int32_t* accept_n, int64_t* next_tok, void* workspace,
                             size_t workspace_bytes, int dtype, void* stream) {
  int rc = check_params(params, "qsp_spec_sample_filtered");
  if (rc) return rc;
  QSP_REQUIRE(target_logits && accept_n && next_tok, "qsp_spec_sample_filtered: null pointer");
  QSP_REQUIRE(batch > 0 && k >= 0 && vocab > 0 && vocab < (1ll << 31) && ld_t >= vocab, "qsp_spec_sample_filtered: bad shape");
  QSP_REQUIRE(k == 0 || drafts != nullptr, "qsp_spec_sample_filtered: drafts missing");
  const bool greedy = !(params->temperature > 0.f);
  QSP_REQUIRE(greedy || (u_resample && (k == 0 || (draft_logits && u_accept && ld_d >= vocab))),
              "qsp_spec_sample_filtered: draft logits and uniforms required");
  const int64_t trows = (int64_t)batch * (k + 1), drows = greedy ? 0 : (int64_t)batch * k;
  size_t so, ao;
  const size_t need = filter_layout(trows + drows, vocab, &so, &ao);
  QSP_REQUIRE(workspace && aligned(workspace, 256) && workspace_bytes >= need,
              "qsp_spec_sample_filtered: workspace of %zu bytes (256-byte aligned) required", need);
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  float* w = reinterpret_cast<float*>(ws);
  FilterRow* st = reinterpret_cast<FilterRow*>(ws + so);
  int64_t* amax = reinterpret_cast<int64_t*>(ws + ao);
  cudaStream_t s = as_stream(stream);
  QSP_DISPATCH_DTYPE(dtype, T, {
    rc = launch_filter<T>(target_logits, ld_t, trows, k + 1, vocab, *params, w, st, amax, s);
    if (!rc && drows > 0)
      rc = launch_filter<T>(draft_logits, ld_d, drows, k, vocab, *params, w + trows * vocab, st + trows, nullptr, s);
  });
  if (rc) return rc;
  if (greedy) {
    greedy_accept_kernel<<<(batch + 127) / 128, 128, 0, s>>>(batch, k + 1, amax, drafts, drafts_ld, accept_n, next_tok);
    return check_launch("qsp_spec_sample_filtered(greedy accept)");
  }
  spec_filtered_kernel<<<batch, SEL_THREADS, 0, s>>>(w, w + trows * vocab, k, vocab, st, st + trows, drafts, drafts_ld,
                                                     u_accept, u_resample, accept_n, next_tok);
  return check_launch("qsp_spec_sample_filtered");
}

}  // extern "C"
