// Error plumbing, embedding, norms, SwiGLU, MTP single-token attention and the per-sequence
// cache bookkeeping kernels.
#include "qsp_common.cuh"

#include <string.h>

namespace qsp {

static thread_local char g_err[1024] = "";

int set_error(int code, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_err, sizeof(g_err), fmt, ap);
  va_end(ap);
  return code;
}

int check_launch(const char* what) {
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return set_error(QSP_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
  return QSP_OK;
}

// ------------------------------------------------------------------ embedding
template <typename T>
__global__ void embed_kernel(const int64_t* __restrict__ ids, int64_t ids_stride, const T* __restrict__ table,
                             int64_t vocab, int64_t dim, T* __restrict__ out, int64_t ld_out,
                             int32_t* bad) {
  const int64_t r = blockIdx.x;
  const int64_t id = ids[r * ids_stride];
  T* o = out + r * ld_out;
  if (id < 0 || id >= vocab) {
    for (int64_t j = threadIdx.x; j < dim; j += blockDim.x) o[j] = dt<T>::from_f(0.0f);
    if (bad != nullptr && threadIdx.x == 0) *bad = 1;
    return;
  }
  const T* src = table + id * dim;
  for (int64_t j = threadIdx.x; j < dim; j += blockDim.x) o[j] = src[j];
}

// ------------------------------------------------------------------ RMSNorm (1 + w)
// One CTA per row; statistics in fp32 exactly as the reference: x̂ = x·rsqrt(mean(x²)+eps),
// y = round(x̂·(1 + w)).
template <typename T, bool ADD>
__global__ void rmsnorm_kernel(T* __restrict__ x, int64_t ld_x, const T* __restrict__ h,
                               const T* __restrict__ w, T* __restrict__ y, int64_t ld_y,
                               int64_t dim, float eps) {
  pdl_trigger();
  pdl_wait();
  extern __shared__ float srow[];
  __shared__ float red[32];
  const int64_t r = blockIdx.x;
  T* xr = x + r * ld_x;
  float ss = 0.0f;
#pragma unroll 8   // the row's loads in flight together (a 2048-wide row is 8 per thread)
  for (int64_t j = threadIdx.x; j < dim; j += blockDim.x) {
    float v = dt<T>::to_f(xr[j]);
    if (ADD) {
      v = dt<T>::round(v + dt<T>::to_f(h[r * dim + j]));
      xr[j] = dt<T>::from_f(v);
    }
    srow[j] = v;
    ss = fmaf(v, v, ss);
  }
  const float tot = block_sum(ss, red);
  const float inv = rsqrtf(tot / (float)dim + eps);
  T* yr = y + r * ld_y;
#pragma unroll 8
  for (int64_t j = threadIdx.x; j < dim; j += blockDim.x) {
    const float v = srow[j] * inv;
    yr[j] = dt<T>::from_f(v * (dt<T>::to_f(w[j]) + 1.0f));
  }
}

// ------------------------------------------------------------------ SwiGLU
template <typename T>
__global__ void swiglu_kernel(const T* __restrict__ gu, int64_t ld_gu, T* __restrict__ y,
                              int64_t ld_y, int64_t inter) {
  pdl_trigger();
  pdl_wait();
  const int64_t r = blockIdx.y;
  for (int64_t j = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; j < inter;
       j += (int64_t)gridDim.x * blockDim.x) {
    const float g = dt<T>::to_f(gu[r * ld_gu + j]);
    const float u = dt<T>::to_f(gu[r * ld_gu + inter + j]);
    // reference: F.silu(gate) (rounded to dtype) * up (rounded)
    const float s = dt<T>::round(siluf_(g));
    y[r * ld_y + j] = dt<T>::from_f(s * u);
  }
}

// ------------------------------------------------------------------ MTP single-token attention
// out[r, h*hd + d] = round(v[r, (h / n_rep)*hd + d]) * round(sigmoid(gate[r, h*2hd + hd + d]))
template <typename T>
__global__ void mtp_attn_kernel(const T* __restrict__ qg, int64_t ld_qg, int64_t ghs,
                                const T* __restrict__ v, int64_t ld_v, T* __restrict__ out,
                                int64_t ld_out, int n_heads, int n_rep, int hd) {
  const int64_t r = blockIdx.y;
  const int total = n_heads * hd;
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < total; i += gridDim.x * blockDim.x) {
    const int h = i / hd, d = i % hd;
    const float gate = dt<T>::to_f(qg[r * ld_qg + (int64_t)h * ghs + d]);
    const float vv = dt<T>::to_f(v[r * ld_v + (int64_t)(h / n_rep) * hd + d]);
    out[r * ld_out + i] = dt<T>::from_f(vv * dt<T>::round(sigmoidf_(gate)));
  }
}

// ------------------------------------------------------------------ cache bookkeeping
template <typename T>
__global__ void select_rows_kernel(const T* __restrict__ src, int64_t ld_src, int T_,
                                   const int32_t* __restrict__ index, T* __restrict__ dst,
                                   int64_t ld_dst, int64_t dim) {
  const int b = blockIdx.x;
  int i = index[b];
  i = i < 0 ? 0 : (i >= T_ ? T_ - 1 : i);
  const T* s = src + ((int64_t)b * T_ + i) * ld_src;
  for (int64_t j = threadIdx.x; j < dim; j += blockDim.x) dst[(int64_t)b * ld_dst + j] = s[j];
}

__global__ void finalize_kernel(int B, int T, int spec, int32_t* lens, int32_t* replay,
                                int32_t* conv_off, int32_t* parity) {
  const int b = blockIdx.x * blockDim.x + threadIdx.x;
  if (b < B) {
    lens[b] += T;
    replay[b] = spec ? T : 0;
    conv_off[b] = spec ? T : 0;
  }
  if (b == 0) parity[0] ^= 1;
}

// Set when qsp_cache_accept met an accepted count outside [0, T-1] (read through
// qsp_device_status); the count is clamped into range so the cache stays consistent.
__device__ int g_core_error = 0;

__global__ void accept_kernel(int B, int T, const int32_t* acc, int32_t* lens, int32_t* replay,
                              int32_t* conv_off) {
  const int b = blockIdx.x * blockDim.x + threadIdx.x;
  if (b >= B) return;
  int keep = acc[b] + 1;
  if (keep < 1 || keep > T) atomicExch(&g_core_error, QSP_DEV_BAD_ACCEPT);
  keep = keep < 1 ? 1 : (keep > T ? T : keep);
  lens[b] -= (T - keep);
  replay[b] = keep;
  conv_off[b] = keep;
}

__global__ void commit_tokens_kernel(int B, int T, int64_t* ids, const int32_t* acc,
                                     const int64_t* next_tok, int64_t* out, int64_t cap,
                                     int32_t* n_out) {
  const int b = blockIdx.x * blockDim.x + threadIdx.x;
  if (b >= B) return;
  int keep = acc[b] + 1;
  keep = keep < 1 ? 1 : (keep > T ? T : keep);
  int64_t n = n_out[b];
  for (int j = 0; j < keep; ++j) {
    if (n + j < cap) out[(int64_t)b * cap + n + j] = ids[(int64_t)b * T + j];
  }
  n_out[b] = (int32_t)(n + keep);
  ids[(int64_t)b * T] = next_tok[b];
}

int core_device_error(int reset) {
  int v = 0;
  if (cudaMemcpyFromSymbol(&v, g_core_error, sizeof(int)) != cudaSuccess) return 0;
  if (reset && v != 0) {
    const int zero = 0;
    cudaMemcpyToSymbol(g_core_error, &zero, sizeof(int));
  }
  return v;
}

}  // namespace qsp

using namespace qsp;

extern "C" {

const char* qsp_last_error(void) { return g_err; }
int qsp_abi_version(void) { return QSP_ABI_VERSION; }

int qsp_embed(const int64_t* ids, int64_t ids_stride, int64_t rows, const void* table,
              int64_t vocab, int64_t dim, void* out, int64_t ld_out, int32_t* bad_ids, int dtype,
              void* stream) {
  QSP_REQUIRE(ids && table && out, "qsp_embed: null pointer");
  QSP_REQUIRE(rows >= 0 && vocab > 0 && dim > 0 && ld_out >= dim, "qsp_embed: bad shape");
  if (rows == 0) return QSP_OK;
  QSP_REQUIRE(rows < (1ll << 31) && ids_stride >= 1, "qsp_embed: bad rows/ids_stride");
  QSP_DISPATCH_DTYPE(dtype, T, {
    embed_kernel<T><<<(unsigned)rows, 256, 0, as_stream(stream)>>>(
        ids, ids_stride, (const T*)table, vocab, dim, (T*)out, ld_out, bad_ids);
  });
  return check_launch("qsp_embed");
}

int qsp_rmsnorm(const void* x, int64_t ld_x, const void* w, void* y, int64_t ld_y, int64_t rows,
                int64_t dim, float eps, int dtype, void* stream) {
  QSP_REQUIRE(x && w && y, "qsp_rmsnorm: null pointer");
  QSP_REQUIRE(rows >= 0 && dim > 0 && dim <= 12288 && ld_x >= dim && ld_y >= dim,
              "qsp_rmsnorm: bad shape");
  if (rows == 0) return QSP_OK;
  QSP_DISPATCH_DTYPE(dtype, T, {
    return launch_pdl("qsp_rmsnorm", rmsnorm_kernel<T, false>, dim3((unsigned)rows), dim3(256),
                      dim * sizeof(float), as_stream(stream), (T*)x, ld_x, (const T*)nullptr, (const T*)w, (T*)y,
                      ld_y, dim, eps);
  });
  return QSP_OK;
}

int qsp_add_rmsnorm(void* x, const void* h, const void* w, void* y, int64_t rows, int64_t dim,
                    float eps, int dtype, void* stream) {
  QSP_REQUIRE(x && h && w && y, "qsp_add_rmsnorm: null pointer");
  QSP_REQUIRE(rows >= 0 && dim > 0 && dim <= 12288, "qsp_add_rmsnorm: bad shape");
  if (rows == 0) return QSP_OK;
  QSP_DISPATCH_DTYPE(dtype, T, {
    return launch_pdl("qsp_add_rmsnorm", rmsnorm_kernel<T, true>, dim3((unsigned)rows), dim3(256),
                      dim * sizeof(float), as_stream(stream), (T*)x, dim, (const T*)h, (const T*)w, (T*)y, dim,
                      dim, eps);
  });
  return QSP_OK;
}

int qsp_swiglu(const void* gu, int64_t ld_gu, void* y, int64_t ld_y, int64_t rows, int64_t inter,
               int dtype, void* stream) {
  QSP_REQUIRE(gu && y, "qsp_swiglu: null pointer");
  QSP_REQUIRE(rows >= 0 && inter > 0 && ld_gu >= 2 * inter && ld_y >= inter && rows < 65536,
              "qsp_swiglu: bad shape");
  if (rows == 0) return QSP_OK;
  const unsigned gx = (unsigned)((inter + 255) / 256 < 64 ? (inter + 255) / 256 : 64);
  QSP_DISPATCH_DTYPE(dtype, T, {
    return launch_pdl("qsp_swiglu", swiglu_kernel<T>, dim3(gx, (unsigned)rows), dim3(256), 0, as_stream(stream),
                      (const T*)gu, ld_gu, (T*)y, ld_y, inter);
  });
  return QSP_OK;
}

int qsp_mtp_single_token_attn(const void* qg, int64_t ld_qg, int64_t gate_head_stride,
                              const void* v, int64_t ld_v, void* out, int64_t ld_out,
                              int64_t rows, int32_t n_heads, int32_t n_kv_heads,
                              int32_t head_dim, int dtype, void* stream) {
  QSP_REQUIRE(qg && v && out, "qsp_mtp_single_token_attn: null pointer");
  QSP_REQUIRE(gate_head_stride >= head_dim, "qsp_mtp_single_token_attn: bad gate_head_stride");
  QSP_REQUIRE(rows >= 0 && rows < 65536 && n_heads > 0 && n_kv_heads > 0 &&
                  n_heads % n_kv_heads == 0 && head_dim > 0,
              "qsp_mtp_single_token_attn: bad shape");
  QSP_REQUIRE(ld_qg >= (int64_t)(n_heads - 1) * gate_head_stride + head_dim && ld_v >= (int64_t)n_kv_heads * head_dim &&
                  ld_out >= (int64_t)n_heads * head_dim,
              "qsp_mtp_single_token_attn: bad leading dimension");
  if (rows == 0) return QSP_OK;
  const int total = n_heads * head_dim;
  const unsigned gx = (unsigned)((total + 255) / 256);
  QSP_DISPATCH_DTYPE(dtype, T, {
    mtp_attn_kernel<T><<<dim3(gx, (unsigned)rows), 256, 0, as_stream(stream)>>>(
        (const T*)qg, ld_qg, gate_head_stride, (const T*)v, ld_v, (T*)out, ld_out, n_heads,
        n_heads / n_kv_heads, head_dim);
  });
  return check_launch("qsp_mtp_single_token_attn");
}

int qsp_select_rows(const void* src, int64_t ld_src, int32_t batch, int32_t tokens,
                    const int32_t* index, void* dst, int64_t ld_dst, int64_t dim, int dtype,
                    void* stream) {
  QSP_REQUIRE(src && index && dst, "qsp_select_rows: null pointer");
  QSP_REQUIRE(batch > 0 && tokens > 0 && dim > 0 && ld_src >= dim && ld_dst >= dim,
              "qsp_select_rows: bad shape");
  QSP_DISPATCH_DTYPE(dtype, T, {
    select_rows_kernel<T><<<batch, 256, 0, as_stream(stream)>>>((const T*)src, ld_src, tokens, index,
                                                                (T*)dst, ld_dst, dim);
  });
  return check_launch("qsp_select_rows");
}

int qsp_cache_finalize(int32_t batch, int32_t tokens, int32_t speculative, int32_t* seq_lens,
                       int32_t* replay_n, int32_t* conv_off, int32_t* parity, void* stream) {
  QSP_REQUIRE(seq_lens && replay_n && conv_off && parity, "qsp_cache_finalize: null pointer");
  QSP_REQUIRE(batch > 0 && tokens >= 0, "qsp_cache_finalize: bad shape");
  finalize_kernel<<<(batch + 127) / 128, 128, 0, as_stream(stream)>>>(
      batch, tokens, speculative, seq_lens, replay_n, conv_off, parity);
  return check_launch("qsp_cache_finalize");
}

int qsp_cache_accept(int32_t batch, int32_t tokens, const int32_t* accept_n, int32_t* seq_lens,
                     int32_t* replay_n, int32_t* conv_off, void* stream) {
  QSP_REQUIRE(accept_n && seq_lens && replay_n && conv_off, "qsp_cache_accept: null pointer");
  QSP_REQUIRE(batch > 0 && tokens > 0, "qsp_cache_accept: bad shape");
  accept_kernel<<<(batch + 127) / 128, 128, 0, as_stream(stream)>>>(batch, tokens, accept_n,
                                                                    seq_lens, replay_n, conv_off);
  return check_launch("qsp_cache_accept");
}

int qsp_commit_tokens(int32_t batch, int32_t tokens, int64_t* ids, const int32_t* accept_n,
                      const int64_t* next_tok, int64_t* out, int64_t out_cap, int32_t* n_out,
                      void* stream) {
  QSP_REQUIRE(ids && accept_n && next_tok && out && n_out, "qsp_commit_tokens: null pointer");
  QSP_REQUIRE(batch > 0 && tokens > 0 && out_cap > 0, "qsp_commit_tokens: bad shape");
  commit_tokens_kernel<<<(batch + 127) / 128, 128, 0, as_stream(stream)>>>(
      batch, tokens, ids, accept_n, next_tok, out, out_cap, n_out);
  return check_launch("qsp_commit_tokens");
}

}  // extern "C"
