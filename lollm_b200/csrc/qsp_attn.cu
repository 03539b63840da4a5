// Gated full attention over the paged KV cache: prep (QK-norm, partial RoPE, KV append),
// split-KV attention of the T new queries, and the merge of the splits with the σ(gate)
// output gate.
#include "qsp_common.cuh"

#include <algorithm>
#include <atomic>

namespace qsp {

int launch_attn_mma(const qsp_attn_layer& L, cudaStream_t st);
int launch_attn_tma(const qsp_attn_layer& L, cudaStream_t st);
int launch_attn_ws(const qsp_attn_layer& L, cudaStream_t st);
int attn_ws_chunk(const qsp_attn_layer& L);

// ------------------------------------------------------------------ prep
// One CTA per token row m = b*T + t; warps loop over the q and k heads (one head per warp
// when the heads fit in 32 warps).
template <typename T>
__global__ void attn_prep_kernel(const qsp_attn_layer L) {
  pdl_trigger();
  pdl_wait();
  extern __shared__ float sx[];  // [warps][hd]
  const int m = blockIdx.x;
  const int b = m / L.tokens, t = m % L.tokens;
  const int hd = L.head_dim, rd = L.rotary_dim, half = rd / 2;
  const int nh = L.n_heads, nkv = L.n_kv_heads;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
  const T* row = static_cast<const T*>(L.qkv) + (int64_t)m * L.ld_qkv;
  const int pos = L.seq_lens[b] + t;
  const int lp = pos / L.page_size, slot = pos % L.page_size;
  int page = -1;
  if (pos >= 0 && pos < L.rope_rows && lp < L.max_pages) page = L.page_table[(int64_t)b * L.max_pages + lp];
  const bool ok = page >= 0 && page < L.num_pages;
  if (!ok) {
    if (threadIdx.x == 0 && L.bad_index != nullptr) *L.bad_index = 1;
  }
  const T* cosr = static_cast<const T*>(L.rope_cos) + (int64_t)(ok ? pos : 0) * rd;
  const T* sinr = static_cast<const T*>(L.rope_sin) + (int64_t)(ok ? pos : 0) * rd;
  float* xs = sx + warp * hd;
  for (int hh = warp; hh < nh + nkv; hh += nw) {
    const bool isq = hh < nh;
    const T* src = isq ? row + (int64_t)hh * 2 * hd : row + (int64_t)nh * 2 * hd + (int64_t)(hh - nh) * hd;
    const T* w = static_cast<const T*>(isq ? L.q_norm_w : L.k_norm_w);
    float ss = 0.f;
    for (int d = lane; d < hd; d += 32) {
      const float v = dt<T>::to_f(src[d]);
      xs[d] = v;
      ss = fmaf(v, v, ss);
    }
    ss = warp_sum(ss);
    const float inv = rsqrtf(ss / (float)hd + L.eps);
    for (int d = lane; d < hd; d += 32) xs[d] = dt<T>::round(xs[d] * inv * (dt<T>::to_f(w[d]) + 1.0f));
    __syncwarp();
    T* dst;
    if (isq) dst = static_cast<T*>(L.q_buf) + ((int64_t)m * nh + hh) * hd;
    else dst = ok ? static_cast<T*>(L.k_pages) + (((int64_t)page * nkv + (hh - nh)) * L.page_size + slot) * hd : nullptr;
    if (dst != nullptr) {
      for (int d = lane; d < hd; d += 32) {
        float v = xs[d];
        if (d < rd) {
          const float c = dt<T>::to_f(cosr[d]), s = dt<T>::to_f(sinr[d]);
          const float r = d < half ? -xs[d + half] : xs[d - half];
          v = dt<T>::round(dt<T>::round(v * c) + dt<T>::round(r * s));
        }
        dst[d] = dt<T>::from_f(v);
      }
    }
    __syncwarp();
  }
  if (ok) {
    const T* vsrc = row + (int64_t)nh * 2 * hd + (int64_t)nkv * hd;
    for (int e = threadIdx.x; e < nkv * hd; e += blockDim.x) {
      const int g = e / hd, d = e % hd;
      static_cast<T*>(L.v_pages)[(((int64_t)page * nkv + g) * L.page_size + slot) * hd + d] = vsrc[e];
    }
  }
}

// ------------------------------------------------------------------ split-KV attention (CUDA cores)
// CTA (split s, kv head g, sequence b × row group). Rows r of the group map to
// (t = r / n_rep, q head g*n_rep + r % n_rep). Keys are staged 32 at a time; lane j scores key j.
constexpr int AT_KT = 32;

template <typename T, int HD, int RPW>
__global__ void __launch_bounds__(128) attn_simt_kernel(const qsp_attn_layer L, int chunk,
                                                        int n_row_groups) {
  pdl_trigger();
  pdl_wait();
  constexpr int DPL = HD / 32;
  extern __shared__ float smem[];
  const int s = blockIdx.x, g = blockIdx.y;
  const int b = blockIdx.z / n_row_groups, rgp = blockIdx.z % n_row_groups;
  const int nrep = L.n_heads / L.n_kv_heads;
  const int rows_total = nrep * L.tokens;
  const int row0 = rgp * 4 * RPW;
  const int nrows = min(4 * RPW, rows_total - row0);
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int base_len = L.seq_lens[b];
  const int kv_len = base_len + L.tokens;
  const int k_begin = s * chunk;
  const int k_end = min(kv_len, k_begin + chunk);
  // smem: Q [4*RPW][HD] fp32, K [32][HD+1] fp32, V [32][HD] fp32
  float* Qs = smem;
  float* Ks = Qs + 4 * RPW * HD;
  float* Vs = Ks + AT_KT * (HD + 1);

  const T* qb = static_cast<const T*>(L.q_buf);
  for (int e = threadIdx.x; e < nrows * HD; e += blockDim.x) {
    const int r = e / HD, d = e % HD;
    const int rr = row0 + r, t = rr / nrep, hq = g * nrep + rr % nrep;
    Qs[r * HD + d] = dt<T>::to_f(qb[(((int64_t)b * L.tokens + t) * L.n_heads + hq) * HD + d]);
  }
  float acc[RPW][DPL];
  float mrow[RPW], lrow[RPW];
#pragma unroll
  for (int i = 0; i < RPW; ++i) {
    mrow[i] = -INFINITY;
    lrow[i] = 0.f;
#pragma unroll
    for (int j = 0; j < DPL; ++j) acc[i][j] = 0.f;
  }
  const T* kp = static_cast<const T*>(L.k_pages);
  const T* vp = static_cast<const T*>(L.v_pages);
  for (int k0 = k_begin; k0 < k_end; k0 += AT_KT) {
    __syncthreads();
    for (int e = threadIdx.x; e < AT_KT * HD; e += blockDim.x) {
      const int j = e / HD, d = e % HD;
      const int pos = k0 + j;
      float kv = 0.f, vv = 0.f;
      if (pos < k_end && pos / L.page_size < L.max_pages) {
        const int page = L.page_table[(int64_t)b * L.max_pages + pos / L.page_size];
        if (page >= 0 && page < L.num_pages) {
          const int64_t off = (((int64_t)page * L.n_kv_heads + g) * L.page_size + pos % L.page_size) * HD + d;
          kv = dt<T>::to_f(kp[off]);
          vv = dt<T>::to_f(vp[off]);
        }
      }
      Ks[j * (HD + 1) + d] = kv;
      Vs[j * HD + d] = vv;
    }
    __syncthreads();
    const int kpos = k0 + lane;
#pragma unroll
    for (int i = 0; i < RPW; ++i) {
      const int r = warp + 4 * i;
      if (r >= nrows) break;
      const int rr = row0 + r;
      const int qpos = base_len + rr / nrep;
      float sc = 0.f;
      const float* q = Qs + r * HD;
      const float* kr = Ks + lane * (HD + 1);
#pragma unroll 8
      for (int d = 0; d < HD; ++d) sc = fmaf(q[d], kr[d], sc);
      sc *= L.scale;
      const bool vis = kpos < k_end && kpos <= qpos;
      sc = vis ? sc : -INFINITY;
      const float mt = warp_max(sc);
      const float mnew = fmaxf(mrow[i], mt);
      if (mnew == -INFINITY) continue;  // nothing visible yet for this row
      const float alpha = expf(mrow[i] - mnew);
      const float p = vis ? expf(sc - mnew) : 0.f;
      lrow[i] = lrow[i] * alpha + warp_sum(p);
      mrow[i] = mnew;
#pragma unroll
      for (int j = 0; j < DPL; ++j) acc[i][j] *= alpha;
      for (int jj = 0; jj < AT_KT; ++jj) {
        const float pj = __shfl_sync(0xffffffffu, p, jj);
        if (pj != 0.f) {
#pragma unroll
          for (int j = 0; j < DPL; ++j) acc[i][j] = fmaf(pj, Vs[jj * HD + lane + 32 * j], acc[i][j]);
        }
      }
    }
  }
  // write partials: o (unnormalised), m, l
#pragma unroll
  for (int i = 0; i < RPW; ++i) {
    const int r = warp + 4 * i;
    if (r >= nrows) break;
    const int rr = row0 + r, t = rr / nrep, hq = g * nrep + rr % nrep;
    const int64_t idx = (((int64_t)b * L.n_heads + hq) * L.tokens + t) * L.num_splits + s;
    float* po = L.partial + idx * (HD + 2);
#pragma unroll
    for (int j = 0; j < DPL; ++j) po[lane + 32 * j] = acc[i][j];
    if (lane == 0) {
      po[HD] = mrow[i];
      po[HD + 1] = lrow[i];
    }
  }
}

// ------------------------------------------------------------------ merge splits + gate
// One warp per (token row m, q head): the np partials (o unnormalised, m natural-log max,
// l) of the row are merged with weights e^{m_p − M}, then σ(gate) is applied.
template <typename T, int HD>
// np_all partials per row in the workspace; with split_len > 0 (the tensor-core kernel:
// fixed-length key splits, two partials each) only the 2·ceil(kv_len / split_len) partials of
// the row's sequence exist and only those are read.
__global__ void __launch_bounds__(256, 2) attn_combine_kernel(const qsp_attn_layer L, int np_all, int split_len) {
  pdl_trigger();
  pdl_wait();
  const int lane = threadIdx.x & 31;
  const int pair = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (pair >= L.batch * L.tokens * L.n_heads) return;
  const int m = pair / L.n_heads, hq = pair % L.n_heads;
  const int b = m / L.tokens, t = m % L.tokens;
  constexpr int hd = HD;
  const float* base = L.partial + ((((int64_t)b * L.n_heads + hq) * L.tokens + t) * np_all) * (hd + 2);
  int np = np_all;
  if (split_len > 0) {
    const int kv_len = max(L.seq_lens[b] + L.tokens, 1);
    np = min(np_all, 2 * ((kv_len + split_len - 1) / split_len));
  }
  float M = -INFINITY;
  for (int p = lane; p < np; p += 32) M = fmaxf(M, base[(int64_t)p * (hd + 2) + hd]);
  M = warp_max(M);
  float den = 0.f;
  for (int p = lane; p < np; p += 32) {
    const float mp = base[(int64_t)p * (hd + 2) + hd];
    if (mp != -INFINITY) den = fmaf(expf(mp - M), base[(int64_t)p * (hd + 2) + hd + 1], den);
  }
  den = warp_sum(den);
  const T* row = static_cast<const T*>(L.qkv) + (int64_t)m * L.ld_qkv;
  T* o = static_cast<T*>(L.out) + (int64_t)m * L.ld_out + (int64_t)hq * hd;
  // lane (2·lane + 64·i, +1) of every partial: the weights e^{m_p − M} are computed once per
  // partial (lane p of each 32-partial group) and broadcast; four partials' columns are
  // loaded together, so the merge waits on memory once per four partials (the sum keeps the
  // partial order)
  constexpr int MAXI = (HD + 63) / 64;
  float2 n[MAXI];
#pragma unroll
  for (int i = 0; i < MAXI; ++i) n[i] = make_float2(0.f, 0.f);
  if (M != -INFINITY) {
    for (int p0 = 0; p0 < np; p0 += 32) {
      const int pl = p0 + lane;
      const float mpl = pl < np ? base[(int64_t)pl * (hd + 2) + hd] : -INFINITY;
      const float wl = mpl != -INFINITY ? expf(mpl - M) : 0.f;
      const int cnt = min(32, np - p0);
      for (int j0 = 0; j0 < cnt; j0 += 4) {
        float2 v[4][MAXI];
        float w[4];
        bool use[4];
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          const int j = j0 + u;   // < 32; lanes j ≥ cnt hold an empty partial (m = −∞)
          const float mp = __shfl_sync(0xffffffffu, mpl, j);
          w[u] = __shfl_sync(0xffffffffu, wl, j);
          use[u] = j < cnt && mp != -INFINITY;
          const float* q = base + (int64_t)(p0 + j) * (hd + 2);
#pragma unroll
          for (int i = 0; i < MAXI; ++i)
            v[u][i] = (use[u] && 2 * lane + 64 * i < hd) ? *reinterpret_cast<const float2*>(q + 2 * lane + 64 * i)
                                                        : make_float2(0.f, 0.f);
        }
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          if (!use[u]) continue;
#pragma unroll
          for (int i = 0; i < MAXI; ++i) {
            if (2 * lane + 64 * i < hd) {
              n[i].x = fmaf(w[u], v[u][i].x, n[i].x);
              n[i].y = fmaf(w[u], v[u][i].y, n[i].y);
            }
          }
        }
      }
    }
  }
#pragma unroll
  for (int i = 0; i < MAXI; ++i) {
    const int d0 = 2 * lane + 64 * i;
    if (d0 >= hd) continue;
#pragma unroll
    for (int k = 0; k < 2; ++k) {
      const int d = d0 + k;
      const float attn = dt<T>::round(den > 0.f ? (k ? n[i].y : n[i].x) / den : 0.f);
      const float gate = dt<T>::to_f(row[(int64_t)hq * 2 * hd + hd + d]);
      o[d] = dt<T>::from_f(attn * dt<T>::round(sigmoidf_(gate)));
    }
  }
}

static int attn_chunk(const qsp_attn_layer& L) {
  const int cap = L.max_pages * L.page_size;
  int chunk = (cap + L.num_splits - 1) / L.num_splits;
  chunk = ((chunk + AT_KT - 1) / AT_KT) * AT_KT;
  return chunk;
}

template <typename T>
static int launch_combine(const qsp_attn_layer& L, int np, cudaStream_t st, int split_len = 0) {
  const int pairs = L.batch * L.tokens * L.n_heads;
  const dim3 grid((pairs + 7) / 8);
  switch (L.head_dim) {   // validated: 32, 64, 128 or 256
    case 32: return launch_pdl("qsp_attn_verify(combine)", attn_combine_kernel<T, 32>, grid, dim3(256), 0, st, L, np, split_len);
    case 64: return launch_pdl("qsp_attn_verify(combine)", attn_combine_kernel<T, 64>, grid, dim3(256), 0, st, L, np, split_len);
    case 128: return launch_pdl("qsp_attn_verify(combine)", attn_combine_kernel<T, 128>, grid, dim3(256), 0, st, L, np, split_len);
    default: return launch_pdl("qsp_attn_verify(combine)", attn_combine_kernel<T, 256>, grid, dim3(256), 0, st, L, np, split_len);
  }
}

template <typename T, int HD, int RPW>
static int launch_attn_simt(const qsp_attn_layer& L, cudaStream_t st) {
  const int rows_total = (L.n_heads / L.n_kv_heads) * L.tokens;
  const int n_rg = (rows_total + 4 * RPW - 1) / (4 * RPW);
  const size_t smem = (size_t)(4 * RPW * HD + AT_KT * (HD + 1) + AT_KT * HD) * sizeof(float);
  auto kern = attn_simt_kernel<T, HD, RPW>;
  cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  dim3 grid(L.num_splits, L.n_kv_heads, L.batch * n_rg);
  int rc = launch_pdl("qsp_attn_verify(simt)", kern, grid, dim3(128), smem, st, L, attn_chunk(L), n_rg);
  if (rc) return rc;
  return launch_combine<T>(L, L.num_splits, st);
}

// Scratch for qsp_attn_verify_static. Some callers cannot allocate at the moment they
// launch: an allocator hook that is itself running inside an allocation, a host that has
// handed all free device memory to its own pool, or code that must not touch the caching
// allocator while another thread captures a graph. For them the split-KV partials live in
// this fixed region, one per device (a __device__ variable exists once per device context).
__device__ __align__(256) float g_attn_static_scratch[QSP_ATTN_STATIC_SCRATCH_BYTES / sizeof(float)];

constexpr int ATTN_STATIC_MAX_DEVICES = 64;
static std::atomic<float*> g_attn_static_addr[ATTN_STATIC_MAX_DEVICES];

// Device address of this device's region (looked up once per device, on that device).
static int attn_static_scratch(float** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return set_error(QSP_ERR_CUDA, "qsp_attn_verify_static: cudaGetDevice: %s", cudaGetErrorString(e));
  if (dev < 0 || dev >= ATTN_STATIC_MAX_DEVICES)
    return set_error(QSP_ERR_UNSUPPORTED, "qsp_attn_verify_static: device %d beyond %d", dev, ATTN_STATIC_MAX_DEVICES);
  float* p = g_attn_static_addr[dev].load(std::memory_order_acquire);
  if (p == nullptr) {
    void* a = nullptr;
    e = cudaGetSymbolAddress(&a, g_attn_static_scratch);
    if (e != cudaSuccess || a == nullptr)
      return set_error(QSP_ERR_CUDA, "qsp_attn_verify_static: cudaGetSymbolAddress: %s", cudaGetErrorString(e));
    p = static_cast<float*>(a);
    g_attn_static_addr[dev].store(p, std::memory_order_release);
  }
  *out = p;
  return QSP_OK;
}

}  // namespace qsp

using namespace qsp;

static int validate_attn(const qsp_attn_layer* p, bool need_ws) {
  QSP_REQUIRE(p != nullptr, "qsp_attn: null layer");
  const qsp_attn_layer& L = *p;
  QSP_REQUIRE(L.qkv && L.q_norm_w && L.k_norm_w && L.rope_cos && L.rope_sin && L.k_pages &&
                  L.v_pages && L.page_table && L.seq_lens && L.q_buf,
              "qsp_attn: null pointer");
  QSP_REQUIRE(L.batch > 0 && L.tokens > 0 && L.batch * L.tokens < (1 << 30), "qsp_attn: bad batch/tokens");
  QSP_REQUIRE(L.n_heads > 0 && L.n_kv_heads > 0 && L.n_heads % L.n_kv_heads == 0,
              "qsp_attn: n_heads must be a multiple of n_kv_heads");
  QSP_REQUIRE(L.head_dim == 32 || L.head_dim == 64 || L.head_dim == 128 || L.head_dim == 256,
              "qsp_attn: head_dim %d not built", L.head_dim);
  QSP_REQUIRE(L.rotary_dim >= 0 && L.rotary_dim <= L.head_dim && L.rotary_dim % 2 == 0,
              "qsp_attn: bad rotary_dim");
  QSP_REQUIRE(L.page_size > 0 && L.max_pages > 0 && L.num_pages > 0, "qsp_attn: bad paging");
  QSP_REQUIRE(L.ld_qkv >= 2ll * L.n_heads * L.head_dim + 2ll * L.n_kv_heads * L.head_dim,
              "qsp_attn: ld_qkv too small");
  if (need_ws) {
    QSP_REQUIRE(L.out && L.partial && L.num_splits > 0 && L.ld_out >= (int64_t)L.n_heads * L.head_dim,
                "qsp_attn_verify: missing output/workspace");
  }
  return QSP_OK;
}

extern "C" {

int qsp_attn_prep(const qsp_attn_layer* layer, void* stream) {
  int rc = validate_attn(layer, false);
  if (rc) return rc;
  const qsp_attn_layer& L = *layer;
  // a warp per q/k head (up to 32): each head's load → norm → RoPE → store chain runs once
  // per row instead of once per head a warp would otherwise loop over
  const int warps = std::min(L.n_heads + L.n_kv_heads, 32);
  const size_t smem = (size_t)warps * L.head_dim * sizeof(float);
  QSP_DISPATCH_DTYPE(L.dtype, T, {
    return launch_pdl("qsp_attn_prep", attn_prep_kernel<T>, dim3(L.batch * L.tokens), dim3(32 * warps), smem,
                      as_stream(stream), L);
  });
  return QSP_OK;
}

int qsp_attn_verify(const qsp_attn_layer* layer, void* stream) {
  int rc = validate_attn(layer, true);
  if (rc) return rc;
  const qsp_attn_layer& L = *layer;
  cudaStream_t st = as_stream(stream);
  if (L.dtype == QSP_BF16) {
    // tensor-core path (head_dim 64/128/256); other shapes use the CUDA-core kernel below
    int rc2 = launch_attn_ws(L, st);
    if (rc2 == QSP_OK) return launch_combine<__nv_bfloat16>(L, 2 * L.num_splits, st, attn_ws_chunk(L));
    if (rc2 == QSP_ERR_UNSUPPORTED) rc2 = launch_attn_mma(L, st);
    if (rc2 == QSP_OK) return launch_combine<__nv_bfloat16>(L, L.num_splits, st);
    if (rc2 != QSP_ERR_UNSUPPORTED) return rc2;
  }
  QSP_DISPATCH_DTYPE(L.dtype, T, {
    switch (L.head_dim) {
      case 32: return launch_attn_simt<T, 32, 16>(L, st);
      case 64: return launch_attn_simt<T, 64, 16>(L, st);
      case 128: return launch_attn_simt<T, 128, 8>(L, st);
      default: return launch_attn_simt<T, 256, 8>(L, st);
    }
  });
}

size_t qsp_attn_workspace_bytes(int32_t batch, int32_t tokens, int32_t n_heads, int32_t head_dim,
                                int32_t num_splits) {
  // two partials per split (the tensor-core path writes one per key half)
  return (size_t)batch * tokens * n_heads * num_splits * 2 * (head_dim + 2) * sizeof(float);
}

int qsp_attn_verify_static(const qsp_attn_layer* layer, void* stream) {
  QSP_REQUIRE(layer != nullptr, "qsp_attn_verify_static: null layer");
  qsp_attn_layer L = *layer;
  QSP_REQUIRE(L.batch > 0 && L.tokens > 0 && L.n_heads > 0 && L.head_dim > 0 && L.num_splits > 0,
              "qsp_attn_verify_static: batch, tokens, heads, head_dim and num_splits must be positive");
  // the size product in overflow-checked steps: a wrapped product must not pass the limit
  size_t need = 2 * sizeof(float) * ((size_t)L.head_dim + 2);
  bool wrapped = false;
  for (const int32_t f : {L.batch, L.tokens, L.n_heads, L.num_splits})
    wrapped = wrapped || __builtin_mul_overflow(need, (size_t)f, &need);
  QSP_REQUIRE(!wrapped && need <= QSP_ATTN_STATIC_SCRATCH_BYTES,
              "qsp_attn_verify_static: this shape needs %zu bytes of split-KV scratch; the static region "
              "holds %zu (use qsp_attn_verify with a caller workspace, or fewer splits)",
              need, (size_t)QSP_ATTN_STATIC_SCRATCH_BYTES);
  float* scratch = nullptr;
  const int rc = attn_static_scratch(&scratch);
  if (rc) return rc;
  L.partial = scratch;
  return qsp_attn_verify(&L, stream);
}

}  // extern "C"
