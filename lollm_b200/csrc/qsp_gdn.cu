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

#include <algorithm>

namespace qsp {

constexpr int GDN_TB = 8;    // tokens per block (a whole verify step)
constexpr int GDN_KMAX = 4;  // largest conv kernel


// Packed fp32x2 helpers (sm_100): each lane rounds exactly like the scalar instruction.
__device__ __forceinline__ uint64_t pk2(float a, float b) {
  uint64_t r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(a), "f"(b));
  return r;
}
__device__ __forceinline__ float2 upk2(uint64_t r) {
  float2 v;
  asm("mov.b64 {%0, %1}, %2;" : "=f"(v.x), "=f"(v.y) : "l"(r));
  return v;
}
__device__ __forceinline__ uint64_t ffma2(uint64_t a, uint64_t b, uint64_t c) {
  uint64_t d;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
  return d;
}
__device__ __forceinline__ uint64_t fmul2(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
__device__ __forceinline__ float2 shfl_add2(float2 v, int o) {
  v.x = __fadd_rn(v.x, __shfl_xor_sync(0xffffffffu, v.x, o));
  v.y = __fadd_rn(v.y, __shfl_xor_sync(0xffffffffu, v.y, o));
  return v;
}

// One state update S ← S·e^g; δ = (v − Sᵀk)·β; S ← S + k δᵀ, on packed column pairs. The
// thread's state is S2[2i] = columns (4cg, 4cg+1), S2[2i+1] = (4cg+2, 4cg+3) of row 4i+rg.
// kd holds k duplicated as (k, k) pairs. Every operation is an explicitly rounded IEEE op, so
// the arithmetic is identical wherever this is inlined (the replay of kept tokens reproduces
// the original forward bit for bit).
template <int RPT>
__device__ __forceinline__ void gdn_update(uint64_t (&S2)[2 * RPT], const float2* __restrict__ kd,
                                           const float* __restrict__ vvec, float g, float beta, int rg, int cg) {
  const float d = expf(g);
  const uint64_t dd = pk2(d, d);
  uint64_t a0 = 0, a1 = 0, b0 = 0, b1 = 0;   // (0.f, 0.f); even rows → a, odd rows → b
#pragma unroll
  for (int i = 0; i < RPT; ++i) {
    const float2 kr = kd[4 * i + rg];
    const uint64_t kk = *reinterpret_cast<const uint64_t*>(&kr);
    S2[2 * i] = fmul2(S2[2 * i], dd);
    S2[2 * i + 1] = fmul2(S2[2 * i + 1], dd);
    if (i & 1) {
      b0 = ffma2(S2[2 * i], kk, b0);
      b1 = ffma2(S2[2 * i + 1], kk, b1);
    } else {
      a0 = ffma2(S2[2 * i], kk, a0);
      a1 = ffma2(S2[2 * i + 1], kk, a1);
    }
  }
  float2 kv0 = upk2(a0), kv1 = upk2(a1);
  {
    const float2 o0 = upk2(b0), o1 = upk2(b1);
    kv0 = make_float2(__fadd_rn(kv0.x, o0.x), __fadd_rn(kv0.y, o0.y));
    kv1 = make_float2(__fadd_rn(kv1.x, o1.x), __fadd_rn(kv1.y, o1.y));
  }
  kv0 = shfl_add2(kv0, 8);
  kv1 = shfl_add2(kv1, 8);
  kv0 = shfl_add2(kv0, 16);
  kv1 = shfl_add2(kv1, 16);
  const float4 vv = *reinterpret_cast<const float4*>(vvec + 4 * cg);
  const uint64_t dl0 = pk2(__fmul_rn(__fsub_rn(vv.x, kv0.x), beta), __fmul_rn(__fsub_rn(vv.y, kv0.y), beta));
  const uint64_t dl1 = pk2(__fmul_rn(__fsub_rn(vv.z, kv1.x), beta), __fmul_rn(__fsub_rn(vv.w, kv1.y), beta));
#pragma unroll
  for (int i = 0; i < RPT; ++i) {
    const float2 kr = kd[4 * i + rg];
    const uint64_t kk = *reinterpret_cast<const uint64_t*>(&kr);
    S2[2 * i] = ffma2(kk, dl0, S2[2 * i]);
    S2[2 * i + 1] = ffma2(kk, dl1, S2[2 * i + 1]);
  }
}

// o = Sᵀq for the thread's 4 columns (q duplicated as (q, q) pairs in qd).
template <int RPT>
__device__ __forceinline__ float4 gdn_readout(const uint64_t (&S2)[2 * RPT], const float2* __restrict__ qd, int rg) {
  uint64_t a0 = 0, a1 = 0, b0 = 0, b1 = 0;
#pragma unroll
  for (int i = 0; i < RPT; ++i) {
    const float2 qr = qd[4 * i + rg];
    const uint64_t qq = *reinterpret_cast<const uint64_t*>(&qr);
    if (i & 1) {
      b0 = ffma2(S2[2 * i], qq, b0);
      b1 = ffma2(S2[2 * i + 1], qq, b1);
    } else {
      a0 = ffma2(S2[2 * i], qq, a0);
      a1 = ffma2(S2[2 * i + 1], qq, a1);
    }
  }
  float2 o0 = upk2(a0), o1 = upk2(a1);
  {
    const float2 e0 = upk2(b0), e1 = upk2(b1);
    o0 = make_float2(__fadd_rn(o0.x, e0.x), __fadd_rn(o0.y, e0.y));
    o1 = make_float2(__fadd_rn(o1.x, e1.x), __fadd_rn(o1.y, e1.y));
  }
  o0 = shfl_add2(o0, 8);
  o1 = shfl_add2(o1, 8);
  o0 = shfl_add2(o0, 16);
  o1 = shfl_add2(o1, 16);
  return make_float4(o0.x, o0.y, o1.x, o1.y);
}

// l2norm in the reference's arithmetic: x·rsqrt(Σx² + 1e-6) evaluated in the model dtype
// (each op rounded for bf16; plain fp32 otherwise). `x` is DK floats in shared memory,
// normalised in place by one warp.
template <typename T, int DK>
__device__ __forceinline__ void warp_l2norm(float2* x, float post_scale, int lane) {
  float ss = 0.f;
  for (int i = lane; i < DK; i += 32) ss += dt<T>::round(x[i].x * x[i].x);
  ss = warp_sum(ss);
  const float s = dt<T>::round(dt<T>::round(ss) + 1e-6f);
  const float r = dt<T>::round(rsqrtf(s));
  for (int i = lane; i < DK; i += 32) {
    const float y = dt<T>::round(x[i].x * r) * post_scale;
    x[i] = make_float2(y, y);
  }
}

// 16-byte vector of T converted to floats
template <typename T>
__device__ __forceinline__ void load16_as_float(const T* src, float* dst) {
  const uint4 u = *reinterpret_cast<const uint4*>(src);
  if constexpr (sizeof(T) == 4) {
    dst[0] = __uint_as_float(u.x); dst[1] = __uint_as_float(u.y);
    dst[2] = __uint_as_float(u.z); dst[3] = __uint_as_float(u.w);
  } else {
    const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      dst[2 * i] = __uint_as_float(w[i] << 16);
      dst[2 * i + 1] = __uint_as_float(w[i] & 0xffff0000u);
    }
  }
}

template <typename T, int DK, int DV>
struct __align__(128) GdnSmem {
  static constexpr int NCH = 2 * DK + DV;   // q, k, v conv channels of one value head
  static constexpr int PS = DK + DV + 4;    // pending row: k | v | g | beta | pad
  float sst[DK * DV];                       // next head's state (TMA bulk prefetch target)
  T xr[GDN_KMAX - 1 + GDN_TB][NCH];         // raw conv inputs: window rows, then tokens
  T zr[GDN_TB][DV];                         // raw output gate z
  T cwr[NCH][GDN_KMAX];                     // conv weights of this head's channels
  float pr[GDN_TB][PS];                     // pending rows to replay
  float2 q[GDN_TB][DK];                     // q, k duplicated as (x, x) pairs (packed FMA operands)
  float2 k[GDN_TB][DK];
  float v[GDN_TB][DV];
  float o[GDN_TB][DV];
  float g[GDN_TB];
  float beta[GDN_TB];
  float ab[GDN_TB][2];                      // a, b of this head
  uint64_t bar;                             // state prefetch barrier
};

__device__ int g_gdn_error = 0;

__device__ __forceinline__ uint32_t gsm(const void* p) { return static_cast<uint32_t>(__cvta_generic_to_shared(p)); }

__device__ __forceinline__ void gcp16(void* dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(gsm(dst)), "l"(src) : "memory");
}

__device__ __forceinline__ bool gdn_wait(uint64_t* bar, uint32_t parity) {
  for (uint32_t i = 0; i < (1u << 24); ++i) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\tselp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok) : "r"(gsm(bar)), "r"(parity) : "memory");
    if (ok) return true;
    if (i > 256) __nanosleep(64);
  }
  atomicExch(&g_gdn_error, 201);
  return false;
}

// Prefetch one head's fp32 state (contiguous DK*DV floats) into shared memory with a single
// bulk copy that completes on `bar`.
__device__ __forceinline__ void gdn_prefetch_state(float* dst, const float* src, uint64_t* bar, uint32_t bytes) {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(gsm(bar)), "r"(bytes) : "memory");
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(gsm(dst)),
               "l"(src), "r"(bytes), "r"(gsm(bar))
               : "memory");
}

// Persistent: CTA c handles (sequence, value head) units c, c+G, c+2G, ... . While a unit is
// computed from registers, the next unit's state streams into shared memory, so the HBM
// traffic of the recurrence (one state read and one write per head) overlaps the math. A
// unit's small inputs (conv window, token rows, z, weights, pending rows) are staged with
// cp.async (all in flight at once, raw in shared memory).
template <typename T, int DK, int DV>
__global__ void __launch_bounds__(DV, 2)
gdn_verify_kernel(const qsp_gdn_layer L) {
  using SMT = GdnSmem<T, DK, DV>;
  constexpr int RPT = DK / 4;
  constexpr int NT = DV;
  constexpr int NCH = SMT::NCH;
  constexpr int PS = SMT::PS;
  constexpr int EPV = 16 / (int)sizeof(T);   // elements per 16-byte vector
  extern __shared__ __align__(128) uint8_t gdn_smem_raw[];
  SMT& sm = *reinterpret_cast<SMT*>(gdn_smem_raw);

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int cg = warp * 8 + (lane & 7), rg = lane >> 3;
  const int T_ = L.tokens, K = L.conv_kernel, Ts = L.max_spec_tokens;
  const int Hv = L.n_v_heads, Hk = L.n_k_heads, vpk = Hv / Hk;
  const int key_dim = Hk * DK, conv_dim = 2 * key_dim + Hv * DV, value_dim = Hv * DV;
  const bool spec = L.speculative != 0;
  const T* proj = static_cast<const T*>(L.proj);
  const T* cw = static_cast<const T*>(L.conv_w);
  T* hist = static_cast<T*>(L.conv_hist);
  T* out = static_cast<T*>(L.out);
  const int par = L.parity[0];
  const int hist_rows = K - 1 + Ts;
  const int units = L.batch * Hv;
  const float qscale = (float)(1.0 / sqrt((double)DK));  // dk^-0.5 rounded once to fp32
  const T* normw = static_cast<const T*>(L.norm_w);
  constexpr uint32_t SBYTES = DK * DV * 4;

  if (tid == 0) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(gsm(&sm.bar)) : "memory");
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  __syncthreads();
  if (tid == 0 && blockIdx.x < units)
    gdn_prefetch_state(sm.sst, L.state + (int64_t)blockIdx.x * DK * DV, &sm.bar, SBYTES);

  uint32_t it = 0;
  for (int u = blockIdx.x; u < units; u += gridDim.x, ++it) {
    const int b = u / Hv, h = u % Hv, kh = h / vpk;
    // device-side counters are clamped to the buffers they index (they are produced by
    // qsp_cache_finalize / qsp_cache_accept and never exceed max_spec_tokens)
    const int R = min(max(L.replay_n[b], 0), Ts);
    const int coff = min(max(L.conv_off[b], 0), Ts);
    const T* hist_in = hist + ((int64_t)par * L.batch + b) * hist_rows * conv_dim;
    T* hist_out = hist + ((int64_t)(par ^ 1) * L.batch + b) * hist_rows * conv_dim;
    float* pend = L.pending + (((int64_t)b * Hv + h) * Ts) * PS;
    float* state = L.state + ((int64_t)b * Hv + h) * DK * DV;
    // global channel of local conv channel c (q | k | v segments of this head)
    const int seg0 = kh * DK, seg1 = key_dim + kh * DK - DK, seg2 = 2 * key_dim + h * DV - 2 * DK;
    auto gch = [&](int c) -> int { return c + (c < DK ? seg0 : (c < 2 * DK ? seg1 : seg2)); };

    // 1. stage this unit's inputs (cp.async: every copy in flight at once)
    for (int e = tid; e < R * (PS / 4); e += NT) gcp16(&sm.pr[0][0] + e * 4, pend + e * 4);
    for (int e = tid; e < NCH * GDN_KMAX * (int)sizeof(T) / 16 && K == GDN_KMAX; e += NT) {
      const int c = (e * 16 / (int)sizeof(T)) / GDN_KMAX;   // first channel of this 16-byte chunk
      const int within = (e * 16 / (int)sizeof(T)) % GDN_KMAX;
      gcp16(&sm.cwr[c][within], cw + (int64_t)gch(c) * GDN_KMAX + within);
    }
    if (K != GDN_KMAX) {   // narrower conv kernels: element loads
      for (int e = tid; e < NCH * K; e += NT) sm.cwr[e / K][e % K] = cw[(int64_t)gch(e / K) * K + e % K];
    }
    auto stage_tokens = [&](int t0, int nt) {
      for (int t = 0; t < nt; ++t) {
        const T* prow = proj + (int64_t)(b * T_ + t0 + t) * L.ld_proj;
        for (int c = tid * EPV; c < NCH; c += NT * EPV) gcp16(&sm.xr[K - 1 + t][c], prow + gch(c));
        for (int c = tid * EPV; c < DV; c += NT * EPV) gcp16(&sm.zr[t][c], prow + conv_dim + h * DV + c);
      }
      if (tid < 2 * nt) {
        const int t = tid >> 1, w = tid & 1;   // w = 0: b, 1: a
        sm.ab[t][w] = dt<T>::to_f(proj[(int64_t)(b * T_ + t0 + t) * L.ld_proj + conv_dim + value_dim + w * Hv + h]);
      }
    };
    for (int i = 0; i < K - 1; ++i)
      for (int c = tid * EPV; c < NCH; c += NT * EPV) gcp16(&sm.xr[i][c], hist_in + (int64_t)(coff + i) * conv_dim + gch(c));
    stage_tokens(0, min(GDN_TB, T_));
    asm volatile("cp.async.commit_group;" ::: "memory");

    // 2. this unit's state: prefetched into shared memory → registers
    gdn_wait(&sm.bar, it & 1u);
    uint64_t S[2 * RPT];
#pragma unroll
    for (int i = 0; i < RPT; ++i) {
      const float4 v4 = *reinterpret_cast<const float4*>(&sm.sst[(4 * i + rg) * DV + 4 * cg]);
      S[2 * i] = pk2(v4.x, v4.y);
      S[2 * i + 1] = pk2(v4.z, v4.w);
    }
    asm volatile("cp.async.wait_all;" ::: "memory");
    __syncthreads();   // inputs staged; every thread holds its state slice
    for (int e = tid; e < R * DK; e += NT) {   // replay keys, duplicated into pairs
      const float kv = sm.pr[e / DK][e % DK];
      sm.k[e / DK][e % DK] = make_float2(kv, kv);
    }
    __syncthreads();
    // 3. prefetch the next unit's state while this one computes
    if (tid == 0 && u + (int)gridDim.x < units)
      gdn_prefetch_state(sm.sst, L.state + (int64_t)(u + gridDim.x) * DK * DV, &sm.bar, SBYTES);

    // 4. replay the kept tokens of the previous speculative call
    auto store_state = [&]() {
#pragma unroll
      for (int i = 0; i < RPT; ++i) {
        const float2 lo = upk2(S[2 * i]), hi = upk2(S[2 * i + 1]);
        *reinterpret_cast<float4*>(state + (int64_t)(4 * i + rg) * DV + 4 * cg) = make_float4(lo.x, lo.y, hi.x, hi.y);
      }
    };
    for (int j = 0; j < R; ++j) gdn_update<RPT>(S, sm.k[j], &sm.pr[j][DK], sm.pr[j][DK + DV], sm.pr[j][DK + DV + 1], rg, cg);
    if (R > 0 && spec) store_state();

    // conv-history ownership: every head writes its v channels; the first v head of a k-head
    // group also writes that group's q and k channels
    const int c_first = ((h % vpk) == 0) ? 0 : 2 * DK;
    auto write_hist_rows = [&](int src_row0, int n_rows) {
      for (int i = 0; i < n_rows; ++i)
        for (int c = c_first + tid * EPV; c < NCH; c += NT * EPV)
          *reinterpret_cast<uint4*>(hist_out + (int64_t)i * conv_dim + gch(c)) =
              *reinterpret_cast<const uint4*>(&sm.xr[src_row0 + i][c]);
    };
    if (T_ == 0) write_hist_rows(0, K - 1);

    const float A = -expf(dt<T>::to_f(static_cast<const T*>(L.a_log)[h]));
    const float dtb = dt<T>::to_f(static_cast<const T*>(L.dt_bias)[h]);

    for (int t0 = 0; t0 < T_; t0 += GDN_TB) {
      const int nt = min(GDN_TB, T_ - t0);
      __syncthreads();   // the replay is done with the k pairs
      // 5. conv + SiLU (fp32 accumulate, rounded like F.conv1d then F.silu), gates
      for (int c = tid; c < NCH; c += NT) {
        float w[GDN_KMAX];
#pragma unroll
        for (int j = 0; j < GDN_KMAX; ++j) w[j] = j < K ? dt<T>::to_f(sm.cwr[c][j]) : 0.f;
        for (int t = 0; t < nt; ++t) {
          float acc = 0.f;
          for (int j = 0; j < K; ++j) acc = fmaf(w[j], dt<T>::to_f(sm.xr[t + j][c]), acc);
          const float a = dt<T>::round(siluf_(dt<T>::round(acc)));
          if (c < DK) sm.q[t][c] = make_float2(a, a);
          else if (c < 2 * DK) sm.k[t][c - DK] = make_float2(a, a);
          else sm.v[t][c - 2 * DK] = a;
        }
      }
      if (tid < nt) {
        sm.beta[tid] = dt<T>::round(sigmoidf_(sm.ab[tid][0]));
        sm.g[tid] = A * softplusf_(sm.ab[tid][1] + dtb);
      }
      if (spec && t0 == 0) write_hist_rows(0, K - 1 + nt);
      __syncthreads();
      for (int vidx = warp; vidx < 2 * nt; vidx += NT / 32) {
        const int t = vidx >> 1;
        if (vidx & 1) warp_l2norm<T, DK>(sm.k[t], 1.0f, lane);
        else warp_l2norm<T, DK>(sm.q[t], qscale, lane);
      }
      __syncthreads();
      // 6. recurrence + readout; pending (k, v, g, β) for the next call's replay
      for (int t = 0; t < nt; ++t) {
        gdn_update<RPT>(S, sm.k[t], sm.v[t], sm.g[t], sm.beta[t], rg, cg);
        const float4 o = gdn_readout<RPT>(S, sm.q[t], rg);
        if (rg == 0) *reinterpret_cast<float4*>(&sm.o[t][4 * cg]) = o;
      }
      if (spec) {
        for (int t = 0; t < nt; ++t) {
          float* prow = pend + (int64_t)(t0 + t) * PS;
          for (int c4 = tid * 4; c4 < PS; c4 += NT * 4) {
            float4 v4;
            if (c4 < DK) v4 = make_float4(sm.k[t][c4].x, sm.k[t][c4 + 1].x, sm.k[t][c4 + 2].x, sm.k[t][c4 + 3].x);
            else if (c4 < DK + DV) v4 = *reinterpret_cast<const float4*>(&sm.v[t][c4 - DK]);
            else v4 = make_float4(sm.g[t], sm.beta[t], 0.f, 0.f);
            *reinterpret_cast<float4*>(prow + c4) = v4;
          }
        }
      }
      __syncthreads();
      // 7. RMSNormGated over dv per token: w·round(x̂) · silu(z), x = round(core)
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
          orow[c] = dt<T>::from_f(wx * siluf_(dt<T>::to_f(sm.zr[t][c])));
        }
      }
      const bool last = t0 + nt >= T_;
      if (last) {
        if (!spec) write_hist_rows(nt, K - 1);   // the window after the last token
      } else {
        // slide the window (last K-1 combined rows to the front) and stage the next block;
        // source and destination rows may overlap: read everything, barrier, then write
        constexpr int SLIDE = ((GDN_KMAX - 1) * NCH + NT - 1) / NT;
        T keep[SLIDE];
        __syncthreads();
#pragma unroll
        for (int q4 = 0; q4 < SLIDE; ++q4) {
          const int e = tid + q4 * NT;
          keep[q4] = e < (K - 1) * NCH ? sm.xr[nt + e / NCH][e % NCH] : T{};
        }
        __syncthreads();
#pragma unroll
        for (int q4 = 0; q4 < SLIDE; ++q4) {
          const int e = tid + q4 * NT;
          if (e < (K - 1) * NCH) sm.xr[e / NCH][e % NCH] = keep[q4];
        }
        stage_tokens(t0 + nt, min(GDN_TB, T_ - t0 - nt));
        asm volatile("cp.async.commit_group;" ::: "memory");
        asm volatile("cp.async.wait_all;" ::: "memory");
        __syncthreads();
      }
    }

    if (!spec) store_state();
    __syncthreads();   // the next unit's staging overwrites the inputs
  }
}

static int sm_count_gdn() {
  static int n = 0;
  if (n == 0) {
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    if (n <= 0) n = 148;
  }
  return n;
}

template <typename T, int DK, int DV>
static int launch_gdn_dims(const qsp_gdn_layer& L, cudaStream_t st) {
  auto kern = gdn_verify_kernel<T, DK, DV>;
  const size_t smem = sizeof(GdnSmem<T, DK, DV>);
  static bool set = false;
  if (!set) {
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess)
      return set_error(QSP_ERR_CUDA, "qsp_gdn_verify: cannot reserve %zu bytes of shared memory", smem);
    set = true;
  }
  const int units = L.batch * L.n_v_heads;
  const int grid = std::min(units, 2 * sm_count_gdn());
  kern<<<grid, DV, smem, st>>>(L);
  return check_launch("qsp_gdn_verify");
}

template <typename T>
static int launch_gdn(const qsp_gdn_layer& L, cudaStream_t st) {
  if (L.head_k == 32 && L.head_v == 32) return launch_gdn_dims<T, 32, 32>(L, st);
  if (L.head_k == 64 && L.head_v == 64) return launch_gdn_dims<T, 64, 64>(L, st);
  if (L.head_k == 128 && L.head_v == 128) return launch_gdn_dims<T, 128, 128>(L, st);
  return set_error(QSP_ERR_UNSUPPORTED, "qsp_gdn_verify: head dims %d/%d not built", L.head_k, L.head_v);
}

int gdn_device_error(int reset) {
  int v = 0;
  cudaMemcpyFromSymbol(&v, g_gdn_error, sizeof(int));
  if (reset && v) {
    const int z = 0;
    cudaMemcpyToSymbol(g_gdn_error, &z, sizeof(int));
  }
  return v;
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
  QSP_REQUIRE(L.conv_kernel >= 2 && L.conv_kernel <= GDN_KMAX, "qsp_gdn_verify: conv kernel %d (max %d)",
              L.conv_kernel, GDN_KMAX);
  QSP_REQUIRE(L.max_spec_tokens >= 1 && L.max_spec_tokens <= GDN_TB,
              "qsp_gdn_verify: max_spec_tokens must be in [1, %d]", GDN_TB);
  QSP_REQUIRE(!L.speculative || (L.tokens >= 1 && L.tokens <= L.max_spec_tokens),
              "qsp_gdn_verify: speculative call with %d tokens > max_spec_tokens %d", L.tokens,
              L.max_spec_tokens);
  const int64_t conv_dim = 2ll * L.n_k_heads * L.head_k + (int64_t)L.n_v_heads * L.head_v;
  QSP_REQUIRE(L.ld_proj >= conv_dim + (int64_t)L.n_v_heads * L.head_v + 2 * L.n_v_heads,
              "qsp_gdn_verify: ld_proj too small");
  QSP_REQUIRE(L.ld_out >= (int64_t)L.n_v_heads * L.head_v, "qsp_gdn_verify: ld_out too small");
  QSP_REQUIRE(aligned(L.state, 16) && aligned(L.pending, 16) && aligned(L.proj, 16) && aligned(L.conv_hist, 16),
              "qsp_gdn_verify: state/pending/proj/conv_hist must be 16-byte aligned");
  const int esz = L.dtype == QSP_F32 ? 4 : 2;
  QSP_REQUIRE((L.ld_proj * esz) % 16 == 0, "qsp_gdn_verify: ld_proj must be a multiple of 16 bytes");
  QSP_DISPATCH_DTYPE(L.dtype, T, { return launch_gdn<T>(L, as_stream(stream)); });
}
