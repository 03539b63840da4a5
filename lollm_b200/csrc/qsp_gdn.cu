// Gated DeltaNet verify/commit kernel: one CTA per (value head, sequence).
//
// The fp32 recurrent state of the head (dk x dv, 64 KB at 128x128) lives in registers for
// the whole call: thread (warp w, lane l) owns columns 4*cg..4*cg+3 with cg = 8w + (l&7) and
// rows rg, rg+4, rg+8, ... with rg = l>>3, so every reduction over rows (Sᵀk, Sᵀq) is an
// in-thread sum plus two xor-shuffles, and a float4 load of one row by the 8 lanes of a row
// group is a fully used 128-byte line. HBM traffic is one state read plus (when the state
// changes) one write per call — the algorithmic minimum of the recurrence.
//
// Rollback by index: see the qsp_gdn_layer comment in include/qsp.h.
#include "qsp_common.cuh"

namespace qsp {

constexpr int GDN_TB = 4;  // tokens per prologue block

template <typename T, int DK, int DV>
struct __align__(16) GdnSmem {
  float q[GDN_TB][DK];
  float k[GDN_TB][DK];
  float v[GDN_TB][DV];
  float z[GDN_TB][DV];
  float o[GDN_TB][DV];
  float g[GDN_TB];
  float beta[GDN_TB];
  float red[32];
};

// One state update S ← S·e^g; δ = (v − Sᵀk)·β; S ← S + k δᵀ. Explicit _rn intrinsics keep
// the arithmetic identical wherever it is inlined (the replay of kept tokens must reproduce
// the original forward bit for bit).
template <int RPT>
__device__ __forceinline__ void gdn_update(float4 (&S)[RPT], const float* __restrict__ kvec,
                                           const float* __restrict__ vvec, float g, float beta,
                                           int rg, int cg) {
  const float d = expf(g);
  float4 kv = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
  for (int i = 0; i < RPT; ++i) {
    const float kr = kvec[4 * i + rg];
    S[i].x = __fmul_rn(S[i].x, d);
    S[i].y = __fmul_rn(S[i].y, d);
    S[i].z = __fmul_rn(S[i].z, d);
    S[i].w = __fmul_rn(S[i].w, d);
    kv.x = __fmaf_rn(S[i].x, kr, kv.x);
    kv.y = __fmaf_rn(S[i].y, kr, kv.y);
    kv.z = __fmaf_rn(S[i].z, kr, kv.z);
    kv.w = __fmaf_rn(S[i].w, kr, kv.w);
  }
#pragma unroll
  for (int o = 8; o <= 16; o <<= 1) {
    kv.x = __fadd_rn(kv.x, __shfl_xor_sync(0xffffffffu, kv.x, o));
    kv.y = __fadd_rn(kv.y, __shfl_xor_sync(0xffffffffu, kv.y, o));
    kv.z = __fadd_rn(kv.z, __shfl_xor_sync(0xffffffffu, kv.z, o));
    kv.w = __fadd_rn(kv.w, __shfl_xor_sync(0xffffffffu, kv.w, o));
  }
  const float4 vv = *reinterpret_cast<const float4*>(vvec + 4 * cg);
  float4 dl;
  dl.x = __fmul_rn(__fsub_rn(vv.x, kv.x), beta);
  dl.y = __fmul_rn(__fsub_rn(vv.y, kv.y), beta);
  dl.z = __fmul_rn(__fsub_rn(vv.z, kv.z), beta);
  dl.w = __fmul_rn(__fsub_rn(vv.w, kv.w), beta);
#pragma unroll
  for (int i = 0; i < RPT; ++i) {
    const float kr = kvec[4 * i + rg];
    S[i].x = __fmaf_rn(kr, dl.x, S[i].x);
    S[i].y = __fmaf_rn(kr, dl.y, S[i].y);
    S[i].z = __fmaf_rn(kr, dl.z, S[i].z);
    S[i].w = __fmaf_rn(kr, dl.w, S[i].w);
  }
}

template <int RPT>
__device__ __forceinline__ float4 gdn_readout(const float4 (&S)[RPT], const float* __restrict__ qvec,
                                              int rg) {
  float4 o = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
  for (int i = 0; i < RPT; ++i) {
    const float qr = qvec[4 * i + rg];
    o.x = __fmaf_rn(S[i].x, qr, o.x);
    o.y = __fmaf_rn(S[i].y, qr, o.y);
    o.z = __fmaf_rn(S[i].z, qr, o.z);
    o.w = __fmaf_rn(S[i].w, qr, o.w);
  }
#pragma unroll
  for (int s = 8; s <= 16; s <<= 1) {
    o.x = __fadd_rn(o.x, __shfl_xor_sync(0xffffffffu, o.x, s));
    o.y = __fadd_rn(o.y, __shfl_xor_sync(0xffffffffu, o.y, s));
    o.z = __fadd_rn(o.z, __shfl_xor_sync(0xffffffffu, o.z, s));
    o.w = __fadd_rn(o.w, __shfl_xor_sync(0xffffffffu, o.w, s));
  }
  return o;
}

// l2norm in the reference's arithmetic: x·rsqrt(Σx² + 1e-6) evaluated in the model dtype
// (each op rounded for bf16; plain fp32 otherwise). `x` is DK floats in shared memory,
// normalised in place by one warp.
template <typename T, int DK>
__device__ __forceinline__ void warp_l2norm(float* x, float post_scale, int lane) {
  float ss = 0.f;
  for (int i = lane; i < DK; i += 32) ss += dt<T>::round(x[i] * x[i]);
  ss = warp_sum(ss);
  const float s = dt<T>::round(dt<T>::round(ss) + 1e-6f);
  const float r = dt<T>::round(rsqrtf(s));
  for (int i = lane; i < DK; i += 32) x[i] = dt<T>::round(x[i] * r) * post_scale;
}

template <typename T, int DK, int DV>
__global__ void __launch_bounds__(DV, (DV >= 128 ? 3 : 4))
gdn_verify_kernel(const qsp_gdn_layer L) {
  constexpr int RPT = DK / 4;
  constexpr int NT = DV;
  __shared__ GdnSmem<T, DK, DV> sm;

  const int h = blockIdx.x, b = blockIdx.y;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int cg = warp * 8 + (lane & 7), rg = lane >> 3;
  const int T_ = L.tokens, K = L.conv_kernel, Ts = L.max_spec_tokens;
  const int Hv = L.n_v_heads, Hk = L.n_k_heads, vpk = Hv / Hk, kh = h / vpk;
  const int key_dim = Hk * DK, conv_dim = 2 * key_dim + Hv * DV, value_dim = Hv * DV;
  const bool spec = L.speculative != 0;
  const T* proj = static_cast<const T*>(L.proj);
  const T* cw = static_cast<const T*>(L.conv_w);
  T* hist = static_cast<T*>(L.conv_hist);
  T* out = static_cast<T*>(L.out);
  const int par = L.parity[0];
  // device-side counters are clamped to the buffers they index (they are produced by
  // qsp_cache_finalize / qsp_cache_accept and never exceed max_spec_tokens)
  const int R = min(max(L.replay_n[b], 0), Ts);
  const int coff = min(max(L.conv_off[b], 0), Ts);
  const int hist_rows = K - 1 + Ts;
  const T* hist_in = hist + ((int64_t)par * L.batch + b) * hist_rows * conv_dim;
  T* hist_out = hist + ((int64_t)(par ^ 1) * L.batch + b) * hist_rows * conv_dim;
  const int pstride = DK + DV + 2;
  float* pend = L.pending + (((int64_t)b * Hv + h) * Ts) * pstride;
  float* state = L.state + ((int64_t)b * Hv + h) * DK * DV;

  // 1. the state of this head into registers (issued first; latency overlaps the replay load)
  float4 S[RPT];
#pragma unroll
  for (int i = 0; i < RPT; ++i)
    S[i] = *reinterpret_cast<const float4*>(state + (int64_t)(4 * i + rg) * DV + 4 * cg);

  // 2. replay the kept tokens of the previous speculative call
  for (int j0 = 0; j0 < R; j0 += GDN_TB) {
    const int nj = min(GDN_TB, R - j0);
    __syncthreads();
    for (int e = tid; e < nj * pstride; e += NT) {
      const int j = e / pstride, c = e % pstride;
      const float val = pend[(int64_t)(j0 + j) * pstride + c];
      if (c < DK) sm.k[j][c] = val;
      else if (c < DK + DV) sm.v[j][c - DK] = val;
      else if (c == DK + DV) sm.g[j] = val;
      else sm.beta[j] = val;
    }
    __syncthreads();
    for (int j = 0; j < nj; ++j) gdn_update<RPT>(S, sm.k[j], sm.v[j], sm.g[j], sm.beta[j], rg, cg);
  }
  if (R > 0 && spec) {
#pragma unroll
    for (int i = 0; i < RPT; ++i)
      *reinterpret_cast<float4*>(state + (int64_t)(4 * i + rg) * DV + 4 * cg) = S[i];
  }

  // conv input x(c, i) over the combined sequence [window (K-1 rows) | raw tokens]
  auto xin = [&](int c, int i) -> float {
    if (i < K - 1) return dt<T>::to_f(hist_in[(int64_t)(coff + i) * conv_dim + c]);
    return dt<T>::to_f(proj[(int64_t)(b * T_ + (i - (K - 1))) * L.ld_proj + c]);
  };
  // channels this CTA owns for the conv history: its v channels, and the q/k channels of its
  // k head when it is the first v head of the group
  const bool own_qk = (h % vpk) == 0;
  const int n_own = DV + (own_qk ? 2 * DK : 0);
  auto own_channel = [&](int e) -> int {
    if (e < DV) return 2 * key_dim + h * DV + e;
    e -= DV;
    if (e < DK) return kh * DK + e;
    return key_dim + kh * DK + (e - DK);
  };
  if (spec) {
    for (int e = tid; e < n_own * (K - 1 + T_); e += NT) {
      const int i = e / n_own, c = own_channel(e % n_own);
      hist_out[(int64_t)i * conv_dim + c] = dt<T>::from_f(xin(c, i));
    }
  } else {
    for (int e = tid; e < n_own * (K - 1); e += NT) {
      const int i = e / n_own, c = own_channel(e % n_own);
      hist_out[(int64_t)i * conv_dim + c] = dt<T>::from_f(xin(c, T_ + i));
    }
  }

  const float qscale = (float)(1.0 / sqrt((double)DK));  // dk^-0.5 rounded once to fp32
  const float A = -expf(dt<T>::to_f(static_cast<const T*>(L.a_log)[h]));
  const float dtb = dt<T>::to_f(static_cast<const T*>(L.dt_bias)[h]);
  const T* normw = static_cast<const T*>(L.norm_w);

  for (int t0 = 0; t0 < T_; t0 += GDN_TB) {
    const int nt = min(GDN_TB, T_ - t0);
    __syncthreads();
    // 3. prologue: conv + SiLU for q, k, v channels; z, β, g
    for (int e = tid; e < nt * (2 * DK + 2 * DV); e += NT) {
      const int t = e / (2 * DK + 2 * DV);
      int c = e % (2 * DK + 2 * DV);
      const int tok = t0 + t;
      const T* prow = proj + (int64_t)(b * T_ + tok) * L.ld_proj;
      if (c < 2 * DK + DV) {
        int ch;
        float* dst;
        if (c < DK) { ch = kh * DK + c; dst = &sm.q[t][c]; }
        else if (c < 2 * DK) { ch = key_dim + kh * DK + (c - DK); dst = &sm.k[t][c - DK]; }
        else { ch = 2 * key_dim + h * DV + (c - 2 * DK); dst = &sm.v[t][c - 2 * DK]; }
        float acc = 0.f;
        for (int j = 0; j < K; ++j) acc = fmaf(dt<T>::to_f(cw[(int64_t)ch * K + j]), xin(ch, tok + j), acc);
        *dst = dt<T>::round(siluf_(dt<T>::round(acc)));
      } else {
        c -= 2 * DK + DV;
        sm.z[t][c] = dt<T>::to_f(prow[conv_dim + h * DV + c]);
      }
    }
    if (tid < nt) {
      const T* prow = proj + (int64_t)(b * T_ + t0 + tid) * L.ld_proj;
      const float bb = dt<T>::to_f(prow[conv_dim + value_dim + h]);
      const float aa = dt<T>::to_f(prow[conv_dim + value_dim + Hv + h]);
      sm.beta[tid] = dt<T>::round(sigmoidf_(bb));
      sm.g[tid] = A * softplusf_(aa + dtb);
    }
    __syncthreads();
    // l2norm of q (with the dk^-0.5 scale applied after, in fp32) and k: one warp per vector
    for (int vidx = warp; vidx < 2 * nt; vidx += NT / 32) {
      const int t = vidx >> 1;
      if (vidx & 1) warp_l2norm<T, DK>(sm.k[t], 1.0f, lane);
      else warp_l2norm<T, DK>(sm.q[t], qscale, lane);
    }
    __syncthreads();
    // 4. recurrence + readout; pending (k, v, g, β) for the next call's replay
    for (int t = 0; t < nt; ++t) {
      gdn_update<RPT>(S, sm.k[t], sm.v[t], sm.g[t], sm.beta[t], rg, cg);
      const float4 o = gdn_readout<RPT>(S, sm.q[t], rg);
      if (rg == 0) *reinterpret_cast<float4*>(&sm.o[t][4 * cg]) = o;
    }
    if (spec) {
      for (int e = tid; e < nt * pstride; e += NT) {
        const int t = e / pstride, c = e % pstride;
        float val;
        if (c < DK) val = sm.k[t][c];
        else if (c < DK + DV) val = sm.v[t][c - DK];
        else if (c == DK + DV) val = sm.g[t];
        else val = sm.beta[t];
        pend[(int64_t)(t0 + t) * pstride + c] = val;
      }
    }
    __syncthreads();
    // 5. RMSNormGated over dv per token: w·round(x̂) · silu(z), x = round(core)
    for (int t = warp; t < nt; t += NT / 32) {
      float ss = 0.f;
      for (int c = lane; c < DV; c += 32) {
        const float x = dt<T>::round(sm.o[t][c]);
        ss = fmaf(x, x, ss);
      }
      ss = warp_sum(ss);
      const float inv = rsqrtf(ss / (float)DV + L.eps);
      T* orow = out + (int64_t)(b * T_ + t0 + t) * L.ld_out + h * DV;
      for (int c = lane; c < DV; c += 32) {
        const float xh = dt<T>::round(dt<T>::round(sm.o[t][c]) * inv);
        const float wx = dt<T>::round(dt<T>::to_f(normw[c]) * xh);
        orow[c] = dt<T>::from_f(wx * siluf_(sm.z[t][c]));
      }
    }
  }

  if (!spec) {
#pragma unroll
    for (int i = 0; i < RPT; ++i)
      *reinterpret_cast<float4*>(state + (int64_t)(4 * i + rg) * DV + 4 * cg) = S[i];
  }
}

template <typename T>
static int launch_gdn(const qsp_gdn_layer& L, cudaStream_t st) {
  dim3 grid(L.n_v_heads, L.batch);
#define QSP_GDN_CASE(DKV)                                                    \
  if (L.head_k == DKV && L.head_v == DKV) {                                  \
    gdn_verify_kernel<T, DKV, DKV><<<grid, DKV, 0, st>>>(L);                 \
    return check_launch("qsp_gdn_verify");                                   \
  }
  QSP_GDN_CASE(32)
  QSP_GDN_CASE(64)
  QSP_GDN_CASE(128)
#undef QSP_GDN_CASE
  return set_error(QSP_ERR_UNSUPPORTED, "qsp_gdn_verify: head dims %d/%d not built", L.head_k,
                   L.head_v);
}

}  // namespace qsp

using namespace qsp;

extern "C" int qsp_gdn_verify(const qsp_gdn_layer* layer, void* stream) {
  QSP_REQUIRE(layer != nullptr, "qsp_gdn_verify: null layer");
  const qsp_gdn_layer& L = *layer;
  QSP_REQUIRE(L.proj && L.conv_w && L.a_log && L.dt_bias && L.norm_w && L.state && L.conv_hist &&
                  L.pending && L.replay_n && L.conv_off && L.parity && L.out,
              "qsp_gdn_verify: null pointer");
  QSP_REQUIRE(L.batch > 0 && L.batch <= 65535 && L.tokens >= 0, "qsp_gdn_verify: bad batch/tokens");
  QSP_REQUIRE(L.n_k_heads > 0 && L.n_v_heads > 0 && L.n_v_heads % L.n_k_heads == 0,
              "qsp_gdn_verify: v heads must be a multiple of k heads");
  QSP_REQUIRE(L.conv_kernel >= 2 && L.conv_kernel <= 8, "qsp_gdn_verify: conv kernel %d", L.conv_kernel);
  QSP_REQUIRE(L.max_spec_tokens >= 1, "qsp_gdn_verify: max_spec_tokens must be >= 1");
  QSP_REQUIRE(!L.speculative || (L.tokens >= 1 && L.tokens <= L.max_spec_tokens),
              "qsp_gdn_verify: speculative call with %d tokens > max_spec_tokens %d", L.tokens,
              L.max_spec_tokens);
  const int64_t conv_dim = 2ll * L.n_k_heads * L.head_k + (int64_t)L.n_v_heads * L.head_v;
  QSP_REQUIRE(L.ld_proj >= conv_dim + (int64_t)L.n_v_heads * L.head_v + 2 * L.n_v_heads,
              "qsp_gdn_verify: ld_proj too small");
  QSP_REQUIRE(L.ld_out >= (int64_t)L.n_v_heads * L.head_v, "qsp_gdn_verify: ld_out too small");
  QSP_REQUIRE(aligned(L.state, 16) && aligned(L.pending, 16), "qsp_gdn_verify: state/pending must be 16-byte aligned");
  QSP_DISPATCH_DTYPE(L.dtype, T, { return launch_gdn<T>(L, as_stream(stream)); });
}
