// Gated DeltaNet verify/commit: the token mixer core of one GDN layer.
//
// Calls of at most max_spec_tokens tokens (every speculative verify, flushes, short commits)
// run two kernels:
//   gdn_prep_kernel   one CTA per (sequence, key head): causal conv + SiLU over the head's
//                     q, k and v channels, l2norm of q and k, the gates g and β, and the Gram
//                     products k_s·k_t, k_s·q_t of the call's tokens. Results go to a per-layer
//                     token ring (`pending`, two parity slots) that the NEXT call also reads
//                     to replay kept tokens, and the raw inputs to the conv-history ring.
//   gdn_chunk_kernel  persistent, one (sequence, value head) at a time: the fp32 state, one
//                     column per thread, is updated over all the call's tokens at once in
//                     chunked (WY) form — one pass computes Sᵀk_s and Sᵀq_t for every token,
//                     a per-column triangular recursion gives the δ's, and one rank-n pass
//                     writes the new state. The columns of S evolve independently under the
//                     delta rule, so nothing is reduced across threads except the gated
//                     RMSNorm of the output.
// Longer commit calls (prefill) replay the kept tokens with gdn_chunk_kernel, then run
// gdn_prefill_kernel, which applies the tokens in blocks of 8 with the same chunked update,
// computing each block's conv, gates, l2norm and Gram products itself.
//
// HBM traffic is one state read plus (when the state changes) one write per head and call —
// the algorithmic minimum of the recurrence. Rollback by index: see include/qsp.h.
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

// 16-byte vector of T converted to floats
// two adjacent elements (4- or 8-byte aligned) as floats, and the reverse
__device__ __forceinline__ float2 gdn_ld2f(const float* p) { return *reinterpret_cast<const float2*>(p); }
__device__ __forceinline__ float2 gdn_ld2f(const __nv_bfloat16* p) {
  return __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(p));
}
__device__ __forceinline__ void gdn_st2(float* p, float a, float b) { *reinterpret_cast<float2*>(p) = make_float2(a, b); }
__device__ __forceinline__ void gdn_st2(__nv_bfloat16* p, float a, float b) {
  *reinterpret_cast<__nv_bfloat162*>(p) = __halves2bfloat162(__float2bfloat16_rn(a), __float2bfloat16_rn(b));
}

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
// bulk copy that completes on `bar`. The state is read once per call (the layers' states do not
// fit L2): it is loaded with an L2 evict-first policy.
__device__ __forceinline__ void gdn_prefetch_state(float* dst, const float* src, uint64_t* bar, uint32_t bytes) {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(gsm(bar)), "r"(bytes) : "memory");
  uint64_t pol;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(pol));
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], %4;" ::"r"(gsm(dst)),
               "l"(src), "r"(bytes), "r"(gsm(bar)), "l"(pol)
               : "memory");
}

// ------------------------------------------------------------------ token ring
// Per layer, `pending` holds two arrays of per-(parity, sequence, value head, slot) records;
// slot t describes token t of the call that wrote that parity:
//   A: k̂ [dk] | v [dv] (model dtype) | Gkk [8] (k_s·k_t, s < t) | (d, β, 0, 0)   fp32 tail
//   B: q̂ [dk] | z [dv] (model dtype) | Gkq [8] (k_s·(dk^-1/2 q_t), s <= t)         fp32 tail
// with d = e^g, g = −exp(A_log)·softplus(a + dt_bias), q̂ before the dk^-1/2 scale. k̂, q̂ and
// the Gram products belong to the key head and are repeated in each of its value heads'
// records, so one unit's rows are contiguous: a speculative call writes the slots of
// parity^1, and the next call replays kept tokens from the A records of parity.
template <typename T, int DK, int DV>
struct __align__(16) GdnRecA {
  T k[DK];
  T v[DV];
  float gkk[GDN_TB];
  float4 db;
};
template <typename T, int DK, int DV>
struct __align__(16) GdnRecB {
  T q[DK];
  T z[DV];
  float gkq[GDN_TB];
};

struct GdnRing {
  int64_t recA, recB;   // bytes per record
  int64_t offB;         // byte offset of array B
};

inline GdnRing gdn_ring(int batch, int Hv, int Ts, int DK, int DV, int esz) {
  GdnRing r;
  r.recA = (int64_t)(DK + DV) * esz + GDN_TB * 4 + 16;
  r.recB = (int64_t)(DK + DV) * esz + GDN_TB * 4;
  r.offB = 2ll * batch * Hv * Ts * r.recA;
  return r;
}

// ------------------------------------------------------------------ prep
// One CTA per (sequence b, key head kh): the q and k channels of kh and the v channels of its
// VPK value heads (a compile-time group shape, so every index below is shifts and adds).
// Every input (conv window, token rows, conv weights) is staged into shared memory with
// cp.async first, so the CTA waits for global memory once; results are assembled in shared
// memory and written to the records with 16-byte stores. Arithmetic per element is the
// reference's: conv accumulated in fp32 and rounded like F.conv1d, SiLU rounded, l2norm
// x·rsqrt(Σx² + 1e-6) with each op rounded to the model dtype.
// Dynamic shared memory: xr [K-1+T][nchg] T | cwr [nchg][K] T | qk [T][2·dk] fp32 |
// yst [T][2·dk + VPK·dv] T (normalised q, k and the v outputs of each token, record order).
inline size_t gdn_prep_smem(int nchg, int K, int T, int DK, int esz) {
  const int Tm = T > 0 ? T : 1;
  size_t a = (size_t)(K - 1 + T) * nchg * esz;
  a = (a + 15) / 16 * 16;
  size_t b = (size_t)nchg * K * esz;
  b = (b + 15) / 16 * 16;
  return a + b + (size_t)Tm * 2 * DK * 4 + (size_t)Tm * nchg * esz;
}

// KT / TT > 0 fix the conv kernel width and the call's token count at compile time (the
// verify step's 4 and 4), so every loop over taps and tokens unrolls without run-time bounds;
// 0 reads them from the layer.
template <typename T, int DK, int DV, int VPK, int KT = 0, int TT = 0>
__global__ void __launch_bounds__(256, 8) gdn_prep_kernel(const qsp_gdn_layer L, const GdnRing RG) {
  pdl_trigger();
  pdl_wait();
  using RA = GdnRecA<T, DK, DV>;
  using RB = GdnRecB<T, DK, DV>;
  extern __shared__ __align__(16) uint8_t gdn_prep_raw[];
  constexpr int ESZ = (int)sizeof(T), EPV = 16 / ESZ;
  constexpr int NCHG = 2 * DK + VPK * DV;   // q | k | v of the group
  constexpr int CPR = NCHG / EPV;            // 16-byte chunks per row
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  constexpr int NW = 256 / 32;
  const int Hk = L.n_k_heads, Hv = L.n_v_heads;
  const int b = blockIdx.x / Hk, kh = blockIdx.x % Hk;
  const int T_ = TT > 0 ? TT : L.tokens, K = KT > 0 ? KT : L.conv_kernel, Ts = L.max_spec_tokens;
  const int key_dim = Hk * DK, conv_dim = 2 * key_dim + Hv * DV, value_dim = Hv * DV;
  const int nrows = K - 1 + T_;
  const bool spec = L.speculative != 0;
  T* xr = reinterpret_cast<T*>(gdn_prep_raw);
  T* cwr = reinterpret_cast<T*>(gdn_prep_raw + ((size_t)nrows * NCHG * ESZ + 15) / 16 * 16);
  float* qk = reinterpret_cast<float*>(reinterpret_cast<uint8_t*>(cwr) + ((size_t)NCHG * K * ESZ + 15) / 16 * 16);
  T* yst = reinterpret_cast<T*>(qk + (size_t)(T_ > 0 ? T_ : 1) * 2 * DK);
  const T* __restrict__ proj = static_cast<const T*>(L.proj);
  const T* __restrict__ cw = static_cast<const T*>(L.conv_w);
  T* hist = static_cast<T*>(L.conv_hist);
  const int par = L.parity[0];
  const int coff = min(max(L.conv_off[b], 0), Ts);
  const int hist_rows = K - 1 + Ts;
  const T* hin = hist + ((int64_t)par * L.batch + b) * hist_rows * conv_dim;
  T* hout = hist + ((int64_t)(par ^ 1) * L.batch + b) * hist_rows * conv_dim;
  uint8_t* ring = static_cast<uint8_t*>(L.pending);
  // record (value head kh·VPK + g, slot t) written by this call: slot index (g·Ts + t) from
  // the group's first record
  const int64_t rec0 = (((int64_t)(par ^ 1) * L.batch + b) * Hv + (int64_t)kh * VPK) * Ts;
  uint8_t* baseA = ring + rec0 * RG.recA;
  uint8_t* baseB = ring + RG.offB + rec0 * RG.recB;
  auto recA = [&](int g, int t) { return reinterpret_cast<RA*>(baseA + (int64_t)(g * Ts + t) * RG.recA); };
  auto recB = [&](int g, int t) { return reinterpret_cast<RB*>(baseB + (int64_t)(g * Ts + t) * RG.recB); };
  // global channel of local channel c (q of kh | k of kh | v of the group's heads)
  auto gch = [&](int c) -> int {
    return c < DK ? kh * DK + c : (c < 2 * DK ? key_dim + kh * DK + (c - DK) : 2 * key_dim + kh * VPK * DV + (c - 2 * DK));
  };

  // 1. stage: window rows, token rows, conv weights (16-byte chunks, all in flight)
  for (int e = tid; e < nrows * CPR; e += 256) {
    const int i = e / CPR, c = (e % CPR) * EPV;
    const T* src = i < K - 1 ? hin + (int64_t)(coff + i) * conv_dim + gch(c)
                             : proj + (int64_t)(b * T_ + i - (K - 1)) * L.ld_proj + gch(c);
    gcp16(xr + i * NCHG + c, src);
  }
  for (int e = tid; e < NCHG * K / EPV; e += 256) {
    const int c = e * EPV / K;   // first channel of the chunk; a chunk never crosses a segment
    gcp16(cwr + e * EPV, cw + (int64_t)gch(c) * K + (e * EPV - c * K));
  }
  asm volatile("cp.async.commit_group;" ::: "memory");
  // gates of the group's value heads (scalar loads, in flight with the copies)
  if (tid < VPK * T_) {
    const int t = tid / VPK, g = tid % VPK, hh = kh * VPK + g;
    const T* prow = proj + (int64_t)(b * T_ + t) * L.ld_proj + conv_dim + value_dim;
    const float bb = dt<T>::to_f(prow[hh]), aa = dt<T>::to_f(prow[Hv + hh]);
    const float A = -expf(dt<T>::to_f(static_cast<const T*>(L.a_log)[hh]));
    const float dtb = dt<T>::to_f(static_cast<const T*>(L.dt_bias)[hh]);
    // the per-token decay d = e^g and β = σ(b)
    recA(g, t)->db = make_float4(expf(A * softplusf_(aa + dtb)), dt<T>::round(sigmoidf_(bb)), 0.f, 0.f);
  }
  // output gate z of the group's heads: copied into the B records (16-byte chunks)
  constexpr int ZC = DV / EPV;
  for (int e = tid; e < T_ * VPK * ZC; e += 256) {
    const int t = e / (VPK * ZC), r = e % (VPK * ZC);
    const int g = r / ZC, c = (r % ZC) * EPV;
    *reinterpret_cast<uint4*>(recB(g, t)->z + c) =
        *reinterpret_cast<const uint4*>(proj + (int64_t)(b * T_ + t) * L.ld_proj + conv_dim + (kh * VPK + g) * DV + c);
  }
  asm volatile("cp.async.wait_all;" ::: "memory");
  __syncthreads();

  // 2. conv-history ring: spec keeps window + tokens (the next call starts at row keep),
  //    commit keeps the window after the last token
  {
    const int r0 = spec ? 0 : T_, nr = spec ? nrows : K - 1;
    for (int e = tid; e < nr * CPR; e += 256) {
      const int i = e / CPR, c = (e % CPR) * EPV;
      *reinterpret_cast<uint4*>(hout + (int64_t)i * conv_dim + gch(c)) =
          *reinterpret_cast<const uint4*>(xr + (r0 + i) * NCHG + c);
    }
  }
  // 3. conv + SiLU: a thread takes a pair of adjacent channels for every token (taps read
  //    once, paired loads and stores); per output the taps accumulate in order jj = 0..K-1
  for (int cp = tid; cp < NCHG / 2; cp += 256) {
    const int c = 2 * cp;
    float w0[GDN_KMAX], w1[GDN_KMAX];
#pragma unroll
    for (int jj = 0; jj < GDN_KMAX; ++jj) {
      w0[jj] = jj < K ? dt<T>::to_f(cwr[c * K + jj]) : 0.f;
      w1[jj] = jj < K ? dt<T>::to_f(cwr[(c + 1) * K + jj]) : 0.f;
    }
    for (int t = 0; t < T_; ++t) {
      float a0 = 0.f, a1 = 0.f;
#pragma unroll
      for (int jj = 0; jj < GDN_KMAX; ++jj) {
        if (jj < K) {
          const float2 xv = gdn_ld2f(xr + (t + jj) * NCHG + c);   // the channel pair in one load
          a0 = fmaf(w0[jj], xv.x, a0);
          a1 = fmaf(w1[jj], xv.y, a1);
        }
      }
      const float s0 = dt<T>::round(siluf_(dt<T>::round(a0)));
      const float s1 = dt<T>::round(siluf_(dt<T>::round(a1)));
      if (c < 2 * DK) {
        *reinterpret_cast<float2*>(qk + t * 2 * DK + c) = make_float2(s0, s1);
      } else {
        gdn_st2(yst + t * NCHG + c, s0, s1);
      }
    }
  }
  __syncthreads();
  // 4. l2norm of q and k, one warp per vector; the model-dtype results go to yst (record
  //    order q | k), the fp32 ones stay in qk for the Gram products (q scaled by dk^-0.5)
  const float qscale = (float)(1.0 / sqrt((double)DK));   // dk^-0.5 rounded once to fp32
  for (int vi = warp; vi < 2 * T_; vi += NW) {
    const int t = vi >> 1;
    const bool isk = vi & 1;
    float* xv = qk + t * 2 * DK + (isk ? DK : 0);
    T* yv = yst + t * NCHG + (isk ? DK : 0);
    float ss = 0.f;
#pragma unroll
    for (int i = lane; i < DK; i += 32) ss += dt<T>::round(xv[i] * xv[i]);
    ss = warp_sum(ss);
    const float sq = dt<T>::round(dt<T>::round(ss) + 1e-6f);
    const float r = dt<T>::round(rsqrtf(sq));
#pragma unroll
    for (int i = lane; i < DK; i += 32) {
      const float y = dt<T>::round(xv[i] * r);
      yv[i] = dt<T>::from_f(y);
      xv[i] = isk ? y : y * qscale;
    }
  }
  __syncthreads();
  // 5. records: k̂ and v into the A records, q̂ into the B records (16-byte chunks; k̂ and q̂
  //    belong to the key head and are repeated in each of its value heads' records)
  {
    constexpr int QC = DK / EPV, VC = DV / EPV, PER = 2 * QC + VC;   // chunks per (head, token)
    for (int e = tid; e < T_ * VPK * PER; e += 256) {
      const int t = e / (VPK * PER), r = e % (VPK * PER);
      const int g = r / PER, j = r % PER;
      const T* src;
      T* dst;
      if (j < QC) { src = yst + t * NCHG + j * EPV; dst = recB(g, t)->q + j * EPV; }
      else if (j < 2 * QC) { src = yst + t * NCHG + DK + (j - QC) * EPV; dst = recA(g, t)->k + (j - QC) * EPV; }
      else { src = yst + t * NCHG + 2 * DK + g * DV + (j - 2 * QC) * EPV; dst = recA(g, t)->v + (j - 2 * QC) * EPV; }
      *reinterpret_cast<uint4*>(dst) = *reinterpret_cast<const uint4*>(src);
    }
  }
  // 6. Gram products of the call's tokens (fixed summation order: they are replayed later)
  const int nkk = T_ * (T_ - 1) / 2, nkq = T_ * (T_ + 1) / 2;
  for (int e = warp; e < nkk + nkq; e += NW) {
    int s, t;
    const bool isq = e >= nkk;
    if (!isq) {   // pairs s < t, t = 1..T-1
      int rem = e;
      t = 1;
      while (rem >= t) { rem -= t; ++t; }
      s = rem;
    } else {      // pairs s <= t, t = 0..T-1
      int rem = e - nkk;
      t = 0;
      while (rem >= t + 1) { rem -= t + 1; ++t; }
      s = rem;
    }
    const float* ks = qk + s * 2 * DK + DK;
    const float* o = qk + t * 2 * DK + (isq ? 0 : DK);
    float acc = 0.f;
#pragma unroll
    for (int i = lane; i < DK; i += 32) acc = fmaf(ks[i], o[i], acc);
    acc = warp_sum(acc);
    if (lane < VPK) {
      if (isq) recB(lane, t)->gkq[s] = acc;
      else recA(lane, t)->gkk[s] = acc;
    }
  }
}

// ------------------------------------------------------------------ chunked update
// Column j of the state evolves on its own: with d_s = e^{g_s}, Γ(r, s) = d_{r+1}···d_s and
// P_s = (S_0ᵀk_s)_j, Q_t = (S_0ᵀq_t)_j over the call's tokens s, t:
//   δ_s = β_s·(v_s − Γ(−1, s)·P_s − Σ_{r<s} Γ(r, s)(k_r·k_s)·δ_r)
//   o_t = Γ(−1, t)·Q_t + Σ_{r<=t} Γ(r, t)(k_r·q_t)·δ_r
//   S_n = Γ(−1, n−1)·S_0 + Σ_s Γ(s, n−1)·k_s δ_sᵀ
// which is the reference's token-by-token recurrence (S ← S·d; δ = (v − Sᵀk)β; S += kδᵀ;
// o = Sᵀq) reassociated. Every quantity is computed by one fixed formula from the tokens up
// to it, so the replay of kept tokens reproduces a fresh forward over them bit for bit.
//
// Thread (warp w, lane l) holds rows [dk/4·rg, dk/4·(rg+1)) of columns 4cg..4cg+3, rg = l>>3,
// cg = 8w + (l&7), as packed pairs of adjacent rows. A pass over the state reads each vector
// with 16-byte loads shared by the 8 lanes of a row block; the 4 row blocks are combined by a
// butterfly after which lane l owns column 4cg + rg for the per-column recursion.
// TB: token slots per call processed by the update kernel (4 when max_spec_tokens ≤ 4, the
// verify step's k + 1, else GDN_TB); the records keep GDN_TB Gram slots either way.
template <typename T, int DK, int DV, int TB>
struct __align__(16) GdnChunkIn {     // one unit's token records (filled by bulk copies)
  GdnRecA<T, DK, DV> rep[TB];         // the previous call's tokens (replay)
  GdnRecA<T, DK, DV> na[TB];          // this call's tokens
  GdnRecB<T, DK, DV> nb[TB];
};

template <typename T, int DK, int DV, int TB>
struct __align__(128) GdnChunkSmem {
  float sst[DK * DV];                 // state of the next unit (TMA bulk prefetch target)
  float vec[3 * TB][DK];          // fp32 slots: replay k 0..7, new k 8..15, scaled new q 16..23
  GdnChunkIn<T, DK, DV, TB> in[2];        // double-buffered token records
  float tabA[2][TB][TB];      // Γ(r, s)·k_r·k_s   (replay, new)
  float tabB[TB][TB];         // Γ(r, t)·k_r·q_t   (new)
  float gam[2][TB];               // Γ(−1, s)
  float tail[2][TB];              // Γ(s, n−1)
  float red[(DV + 31) / 32][TB];
  uint64_t bar;                       // state prefetch
  uint64_t ibar[2];                   // token records
};

// Column sums over this thread's rows of S·x_v for 4 consecutive vector slots, reduced over
// the 4 row blocks by a butterfly: on return own[v] = (Sᵀx_v) at column 4cg + rg.
template <int DK, int NV = 4>
__device__ __forceinline__ void gdn_dots4(const uint64_t (&S)[4][DK / 8], const float* __restrict__ vec0, int rg,
                                          float* own) {
  constexpr int RB = DK / 4;
  uint64_t acc[NV][4];
#pragma unroll
  for (int v = 0; v < NV; ++v)
#pragma unroll
    for (int c = 0; c < 4; ++c) acc[v][c] = 0;
#pragma unroll
  for (int m = 0; m < RB / 4; ++m) {
#pragma unroll
    for (int v = 0; v < NV; ++v) {
      const ulonglong2 kk = *reinterpret_cast<const ulonglong2*>(vec0 + v * DK + RB * rg + 4 * m);
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        acc[v][c] = ffma2(S[c][2 * m], kk.x, acc[v][c]);
        acc[v][c] = ffma2(S[c][2 * m + 1], kk.y, acc[v][c]);
      }
    }
  }
  const bool hi = rg & 2, lo = rg & 1;
#pragma unroll
  for (int v = 0; v < NV; ++v) {
    float p[4];
#pragma unroll
    for (int c = 0; c < 4; ++c) {
      const float2 x = upk2(acc[v][c]);
      p[c] = __fadd_rn(x.x, x.y);
    }
    // rows blocks {0,2} ↔ {1,3} halves of the column group, then pairs
    const float s0 = hi ? p[0] : p[2], s1 = hi ? p[1] : p[3];
    float k0 = hi ? p[2] : p[0], k1 = hi ? p[3] : p[1];
    k0 = __fadd_rn(k0, __shfl_xor_sync(0xffffffffu, s0, 16));
    k1 = __fadd_rn(k1, __shfl_xor_sync(0xffffffffu, s1, 16));
    const float snd = lo ? k0 : k1, keep = lo ? k1 : k0;
    own[v] = __fadd_rn(keep, __shfl_xor_sync(0xffffffffu, snd, 8));
  }
}

// S ← γ·S + Σ_{s<n} c_s·x_s (terms in order of s); c_s of column 4cg+c comes from lane
// (c, cg), which owns that column's recursion.
template <int DK, int TB>
__device__ __forceinline__ void gdn_rank(uint64_t (&S)[4][DK / 8], const float* __restrict__ vec0, float gamma,
                                         const float (&cown)[TB], int n, int rg, int lane) {
  constexpr int RB = DK / 4;
  const uint64_t gg = pk2(gamma, gamma);
#pragma unroll
  for (int c = 0; c < 4; ++c)
#pragma unroll
    for (int p = 0; p < RB / 2; ++p) S[c][p] = fmul2(S[c][p], gg);
#pragma unroll 1
  for (int s = 0; s < n; ++s) {
    float cs = cown[0];
#pragma unroll
    for (int i = 1; i < TB; ++i) cs = s == i ? cown[i] : cs;
    uint64_t cc[4];
#pragma unroll
    for (int c = 0; c < 4; ++c) {
      const float x = __shfl_sync(0xffffffffu, cs, (c << 3) | (lane & 7));
      cc[c] = pk2(x, x);
    }
    const float* x = vec0 + s * DK + RB * rg;
#pragma unroll
    for (int m = 0; m < RB / 4; ++m) {
      const ulonglong2 kk = *reinterpret_cast<const ulonglong2*>(x + 4 * m);
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        S[c][2 * m] = ffma2(kk.x, cc[c], S[c][2 * m]);
        S[c][2 * m + 1] = ffma2(kk.y, cc[c], S[c][2 * m + 1]);
      }
    }
  }
}

// δ_s of this lane's column over n tokens (P = Sᵀk_s of the column, v_s from the records)
template <typename T, int DK, int DV, int TB>
__device__ __forceinline__ void gdn_deltas(const float (&P)[TB], const GdnRecA<T, DK, DV>* rec, int col,
                                           const float (*A)[TB], const float* gam, int n, float (&dl)[TB]) {
#pragma unroll
  for (int s = 0; s < TB; ++s) {
    dl[s] = 0.f;
    if (s < n) {
      float acc = __fmul_rn(gam[s], P[s]);
#pragma unroll
      for (int r = 0; r < s; ++r) acc = __fmaf_rn(A[r][s], dl[r], acc);
      dl[s] = __fmul_rn(__fsub_rn(dt<T>::to_f(rec[s].v[col]), acc), rec[s].db.y);
    }
  }
}

__device__ __forceinline__ void gdn_bulk(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(gsm(dst)),
               "l"(src), "r"(bytes), "r"(gsm(bar))
               : "memory");
}

// Warp 0 stages unit u's records into `in` with three bulk copies completing on `bar`: the A
// records of all Ts replay slots (parity par; the unit uses the first replay_n of them) and
// this call's N A and B records (parity par^1).
template <typename T, int DK, int DV, int TB>
__device__ __forceinline__ void gdn_stage(GdnChunkIn<T, DK, DV, TB>& in, uint64_t* bar, const qsp_gdn_layer& L,
                                          const GdnRing& RG, int u, int N, int par, int lane) {
  const int Ts = L.max_spec_tokens;
  const uint8_t* ring = static_cast<const uint8_t*>(L.pending);
  const int64_t a_par = ((int64_t)par * L.batch * L.n_v_heads + u) * Ts;        // record index of slot 0
  const int64_t a_new = ((int64_t)(par ^ 1) * L.batch * L.n_v_heads + u) * Ts;
  if (lane == 0) {
    const uint32_t total = (uint32_t)(Ts * RG.recA + N * (RG.recA + RG.recB));
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(gsm(bar)), "r"(total) : "memory");
  }
  __syncwarp();
  if (lane == 0) gdn_bulk(in.rep, ring + a_par * RG.recA, (uint32_t)(Ts * RG.recA), bar);
  if (lane == 1 && N > 0) gdn_bulk(in.na, ring + a_new * RG.recA, (uint32_t)(N * RG.recA), bar);
  if (lane == 2 && N > 0) gdn_bulk(in.nb, ring + RG.offB + a_new * RG.recB, (uint32_t)(N * RG.recB), bar);
}

// Persistent: CTA c handles (sequence, value head) units c, c+G, ... . While a unit computes,
// the next unit's state and token records stream into shared memory.
template <typename T, int DK, int DV, int TB>
__global__ void __launch_bounds__(DV, 2)
gdn_chunk_kernel(const qsp_gdn_layer L, const GdnRing RG, const int n_new) {
  pdl_trigger();
  pdl_wait();
  using SM = GdnChunkSmem<T, DK, DV, TB>;
  extern __shared__ __align__(128) uint8_t gdn_chunk_raw[];
  SM& sm = *reinterpret_cast<SM*>(gdn_chunk_raw);
  constexpr int RB = DK / 4;          // rows per thread
  constexpr int ESZ = (int)sizeof(T);
  constexpr int EPV = 16 / ESZ;
  constexpr int CK = DK / EPV;        // 16-byte chunks per k/q row
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int rg = lane >> 3, cg = warp * 8 + (lane & 7);
  const int col = 4 * cg + rg;        // the column this lane owns after a butterfly
  const int Hv = L.n_v_heads;
  const int Ts = L.max_spec_tokens;
  const bool spec = L.speculative != 0;
  const int par = L.parity[0];
  const int units = L.batch * Hv;
  const int N = n_new;
  const float qscale = (float)(1.0 / sqrt((double)DK));
  T* out = static_cast<T*>(L.out);
  const float wn = dt<T>::to_f(static_cast<const T*>(L.norm_w)[col]);
  constexpr uint32_t SBYTES = DK * DV * 4;
  const int G = gridDim.x;

  if (tid == 0) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(gsm(&sm.bar)) : "memory");
    asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(gsm(&sm.ibar[0])) : "memory");
    asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(gsm(&sm.ibar[1])) : "memory");
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  __syncthreads();
  if ((int)blockIdx.x < units) {
    if (tid == 0) gdn_prefetch_state(sm.sst, L.state + (int64_t)blockIdx.x * DK * DV, &sm.bar, SBYTES);
    if (warp == 0) gdn_stage<T, DK, DV, TB>(sm.in[0], &sm.ibar[0], L, RG, blockIdx.x, N, par, lane);
  }
  int r_next = (int)blockIdx.x < units ? L.replay_n[blockIdx.x / Hv] : 0;

  uint32_t it = 0;
  for (int u = blockIdx.x; u < units; u += G, ++it) {
    const int b = u / Hv, h = u % Hv;
    // device-side counters are clamped to the buffers they index (they are produced by
    // qsp_cache_finalize / qsp_cache_accept and never exceed max_spec_tokens)
    const int R = min(max(r_next, 0), Ts);
    const int buf = it & 1;
    GdnChunkIn<T, DK, DV, TB>& in = sm.in[buf];
    // 1. the next unit's records go into the other buffer (free since the last unit ended)
    if (u + G < units) {
      if (warp == 0) gdn_stage<T, DK, DV, TB>(sm.in[buf ^ 1], &sm.ibar[buf ^ 1], L, RG, u + G, N, par, lane);
      r_next = L.replay_n[(u + G) / Hv];
    }
    float* state = L.state + (int64_t)u * DK * DV;

    // 2. this unit's state: prefetched into shared memory → registers
    gdn_wait(&sm.bar, it & 1u);
    uint64_t S[4][RB / 2];
#pragma unroll
    for (int p = 0; p < RB / 2; ++p) {
      const float4 r0 = *reinterpret_cast<const float4*>(&sm.sst[(RB * rg + 2 * p) * DV + 4 * cg]);
      const float4 r1 = *reinterpret_cast<const float4*>(&sm.sst[(RB * rg + 2 * p + 1) * DV + 4 * cg]);
      S[0][p] = pk2(r0.x, r1.x);
      S[1][p] = pk2(r0.y, r1.y);
      S[2][p] = pk2(r0.z, r1.z);
      S[3][p] = pk2(r0.w, r1.w);
    }
    gdn_wait(&sm.ibar[buf], (it >> 1) & 1u);
    __syncthreads();   // sst consumed by every thread
    if (tid == 0 && u + G < units)
      gdn_prefetch_state(sm.sst, L.state + (int64_t)(u + G) * DK * DV, &sm.bar, SBYTES);

    // 3. fp32 vector slots and the coefficient tables
    for (int e = tid; e < 3 * TB * CK; e += DV) {
      const int v = e / CK, c = e % CK;   // vector slot, 16-byte chunk of it
      const T* src;
      float sc = 1.f;
      if (v < TB) {
        if (v >= R) continue;
        src = in.rep[v].k;
      } else if (v < 2 * TB) {
        if (v - TB >= N) continue;
        src = in.na[v - TB].k;
      } else {
        if (v - 2 * TB >= N) continue;
        src = in.nb[v - 2 * TB].q;
        sc = qscale;
      }
      float x[EPV];
      load16_as_float<T>(src + c * EPV, x);
#pragma unroll
      for (int i = 0; i < EPV; ++i) sm.vec[v][c * EPV + i] = x[i] * sc;
    }
    for (int e = tid; e < 2 * (TB + 1) * TB; e += DV) {
      const int ch = e / ((TB + 1) * TB);           // 0 replay, 1 new
      const int r = (e / TB) % (TB + 1) - 1, s = e % TB;
      const int n = ch ? N : R;
      const GdnRecA<T, DK, DV>* ra = ch ? in.na : in.rep;
      if (s >= n || r > s) continue;
      float ratio = 1.f;                                      // Γ(r, s) = d_{r+1}···d_s
      for (int i = r + 1; i <= s; ++i) ratio = __fmul_rn(ratio, ra[i].db.x);
      if (r < 0) sm.gam[ch][s] = ratio;
      if (r >= 0 && r < s) sm.tabA[ch][r][s] = __fmul_rn(ratio, ra[s].gkk[r]);
      if (ch == 1 && r >= 0) sm.tabB[r][s] = __fmul_rn(ratio, in.nb[s].gkq[r]);
      if (r >= 0 && s == n - 1) sm.tail[ch][r] = ratio;
    }
    __syncthreads();

    // the new state is not read again in this step: stored with an L2 evict-first policy so
    // its 64 KB per head do not displace the step's re-read data
    auto store_state = [&]() {
      uint64_t pol;
      asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(pol));
#pragma unroll
      for (int p = 0; p < RB / 2; ++p) {
        const float2 a = upk2(S[0][p]), bq = upk2(S[1][p]), c2 = upk2(S[2][p]), d2 = upk2(S[3][p]);
        float* d0 = state + (int64_t)(RB * rg + 2 * p) * DV + 4 * cg;
        float* d1 = d0 + DV;
        asm volatile("st.global.L2::cache_hint.v4.f32 [%0], {%1, %2, %3, %4}, %5;" ::"l"(d0), "f"(a.x), "f"(bq.x),
                     "f"(c2.x), "f"(d2.x), "l"(pol) : "memory");
        asm volatile("st.global.L2::cache_hint.v4.f32 [%0], {%1, %2, %3, %4}, %5;" ::"l"(d1), "f"(a.y), "f"(bq.y),
                     "f"(c2.y), "f"(d2.y), "l"(pol) : "memory");
      }
    };
    // 4. phase 0 replays the kept tokens of the previous speculative call; phase 1 applies this
    //    call's tokens. One copy of the pass code serves both (and keeps the replay's
    //    arithmetic identical to a fresh forward over the same tokens).
    float o[TB];
#pragma unroll 1
    for (int ph = 0; ph < 2; ++ph) {
      const int n = ph ? N : R;
      if (n == 0) continue;
      const int kslot = ph ? TB : 0;
      const int ngk = (n + 3) >> 2, ng = ph ? 2 * ngk : ngk;
      float Pk[TB], Pq[TB], dl[TB];
#pragma unroll
      for (int i = 0; i < TB; ++i) Pk[i] = Pq[i] = 0.f;
#pragma unroll 1
      for (int g = 0; g < ng; ++g) {   // pass 1: Sᵀk_s, then (phase 1) Sᵀq_t, four slots at a time
        const bool isq = g >= ngk;
        const int g4 = isq ? g - ngk : g;
        float t4[4] = {0.f, 0.f, 0.f, 0.f};
        // the last group of a call with n % 4 in {1, 2} only needs that many slots
        const int left = n - 4 * g4;
        const float* vg = sm.vec[(isq ? 2 * TB : kslot) + 4 * g4];
        if (left == 1) gdn_dots4<DK, 1>(S, vg, rg, t4);
        else if (left == 2) gdn_dots4<DK, 2>(S, vg, rg, t4);
        else gdn_dots4<DK>(S, vg, rg, t4);
#pragma unroll
        for (int i = 0; i < 4; ++i) {
#pragma unroll
          for (int jj = 0; jj < TB / 4; ++jj) {
            if (g4 == jj) {
              if (isq) Pq[4 * jj + i] = t4[i];
              else Pk[4 * jj + i] = t4[i];
            }
          }
        }
      }
      gdn_deltas<T, DK, DV, TB>(Pk, ph ? in.na : in.rep, col, sm.tabA[ph], sm.gam[ph], n, dl);
      if (ph) {
#pragma unroll
        for (int t = 0; t < TB; ++t) {
          o[t] = 0.f;
          if (t < N) {
            float acc = __fmul_rn(sm.gam[1][t], Pq[t]);
#pragma unroll
            for (int r = 0; r <= t; ++r) acc = __fmaf_rn(sm.tabB[r][t], dl[r], acc);
            o[t] = acc;
          }
        }
      }
      // the state after these tokens: needed by phase 1 after a replay, and stored when it is
      // committed (the replay always; this call's tokens only when not speculative)
      if (ph == 0 || !spec) {
        float c[TB];
#pragma unroll
        for (int s = 0; s < TB; ++s) c[s] = s < n ? __fmul_rn(sm.tail[ph][s], dl[s]) : 0.f;
        gdn_rank<DK>(S, sm.vec[kslot], sm.gam[ph][n - 1], c, n, rg, lane);
        if (ph == 1 || spec || N == 0) store_state();
      }
    }
    if (N > 0) {
      // 6. RMSNormGated over the dv columns of each token: w·round(x̂)·silu(z), x = round(core)
      // the per-token sums of squares, their butterflies interleaved (same order per token as
      // warp_sum)
      float ssq[TB];
#pragma unroll
      for (int t = 0; t < TB; ++t) {
        const float x = dt<T>::round(o[t]);
        ssq[t] = x * x;
      }
#pragma unroll
      for (int sh = 16; sh > 0; sh >>= 1)
#pragma unroll
        for (int t = 0; t < TB; ++t) ssq[t] += __shfl_xor_sync(0xffffffffu, ssq[t], sh);
      if (lane == 0) {
#pragma unroll
        for (int t = 0; t < TB; ++t)
          if (t < N) sm.red[warp][t] = ssq[t];
      }
      __syncthreads();
#pragma unroll
      for (int t = 0; t < TB; ++t) {
        if (t < N) {
          float ss = 0.f;
          for (int w = 0; w < (DV + 31) / 32; ++w) ss += sm.red[w][t];
          const float inv = rsqrtf(ss / (float)DV + L.eps);
          const float xh = dt<T>::round(dt<T>::round(o[t]) * inv);
          const float wx = dt<T>::round(wn * xh);
          out[(int64_t)(b * N + t) * L.ld_out + h * DV + col] = dt<T>::from_f(wx * siluf_(dt<T>::to_f(in.nb[t].z[col])));
        }
      }
    }
    __syncthreads();   // the next unit's staging overwrites this unit's buffers
  }
}

// ------------------------------------------------------------------ chunked prefill
// A commit of T > max_spec_tokens tokens (prompt prefill), in blocks of GDN_TB tokens: each
// block does the conv + SiLU, gates, l2norm and Gram products of the prep kernel for this unit
// in shared memory, then the chunk kernel's block update — one pass over the state for Sᵀk_s
// and Sᵀq_t, the per-column triangular recursion for δ_s and o_t, one rank-n update — instead
// of a state pass per token. Arithmetic per quantity is the prep and chunk kernels' (the same
// roundings; the block form is the reference's chunked delta rule, blocks.py:59-113, with
// 8-token chunks). Any kept tokens of a previous speculative call were replayed into the
// state before this launch. Persistent: CTA c handles (sequence, value head) units c, c+G, ...;
// the next unit's state streams into shared memory while the current one computes.
template <typename T, int DK, int DV>
struct __align__(128) GdnPrefillSmem {
  static constexpr int NCH = 2 * DK + DV;   // q, k, v conv channels of one value head
  float sst[DK * DV];                       // next unit's state (bulk prefetch target)
  float vec[2 * GDN_TB][DK];                // k̂ slots 0..7, dk^-1/2·q̂ slots 8..15 (fp32)
  float vv[GDN_TB][DV];                     // v (model-dtype values)
  T xr[GDN_KMAX - 1 + GDN_TB][NCH];         // raw conv inputs: window rows, then tokens
  T zr[GDN_TB][DV];                         // raw output gate z
  T cwr[NCH][GDN_KMAX];                     // conv weights of this head's channels
  float ab[GDN_TB][2];                      // b, a of this head
  float beta[GDN_TB], dcy[GDN_TB];          // β_s, d_s = e^{g_s}
  float tabA[GDN_TB][GDN_TB];               // Γ(r, s)·k_r·k_s
  float tabB[GDN_TB][GDN_TB];               // Γ(r, t)·k_r·q_t
  float gam[GDN_TB], tail[GDN_TB];          // Γ(−1, s), Γ(s, n−1)
  float red[(DV + 31) / 32][GDN_TB];
  uint64_t bar;
};

template <typename T, int DK, int DV>
__global__ void __launch_bounds__(DV, 2)
gdn_prefill_kernel(const qsp_gdn_layer L) {
  pdl_trigger();
  pdl_wait();
  using SMT = GdnPrefillSmem<T, DK, DV>;
  constexpr int NCH = SMT::NCH;
  constexpr int RB = DK / 4;            // rows per thread
  constexpr int NT = DV;
  constexpr int EPV = 16 / (int)sizeof(T);
  extern __shared__ __align__(128) uint8_t gdn_pf_raw[];
  SMT& sm = *reinterpret_cast<SMT*>(gdn_pf_raw);
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int rg = lane >> 3, cg = warp * 8 + (lane & 7);
  const int col = 4 * cg + rg;          // the column this lane owns after a butterfly
  const int T_ = L.tokens, K = L.conv_kernel, Ts = L.max_spec_tokens;
  const int Hv = L.n_v_heads, Hk = L.n_k_heads, vpk = Hv / Hk;
  const int key_dim = Hk * DK, conv_dim = 2 * key_dim + Hv * DV, value_dim = Hv * DV;
  const T* proj = static_cast<const T*>(L.proj);
  const T* cw = static_cast<const T*>(L.conv_w);
  T* hist = static_cast<T*>(L.conv_hist);
  T* out = static_cast<T*>(L.out);
  const int par = L.parity[0];
  const int hist_rows = K - 1 + Ts;
  const int units = L.batch * Hv;
  const float qscale = (float)(1.0 / sqrt((double)DK));   // dk^-0.5 rounded once to fp32
  const float wn = dt<T>::to_f(static_cast<const T*>(L.norm_w)[col]);
  constexpr uint32_t SBYTES = DK * DV * 4;

  if (tid == 0) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(gsm(&sm.bar)) : "memory");
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  __syncthreads();
  if (tid == 0 && (int)blockIdx.x < units)
    gdn_prefetch_state(sm.sst, L.state + (int64_t)blockIdx.x * DK * DV, &sm.bar, SBYTES);

  uint32_t it = 0;
  for (int u = blockIdx.x; u < units; u += gridDim.x, ++it) {
    const int b = u / Hv, h = u % Hv, kh = h / vpk;
    const int coff = min(max(L.conv_off[b], 0), Ts);
    const T* hist_in = hist + ((int64_t)par * L.batch + b) * hist_rows * conv_dim;
    T* hist_out = hist + ((int64_t)(par ^ 1) * L.batch + b) * hist_rows * conv_dim;
    float* state = L.state + ((int64_t)b * Hv + h) * DK * DV;
    const int seg0 = kh * DK, seg1 = key_dim + kh * DK - DK, seg2 = 2 * key_dim + h * DV - 2 * DK;
    auto gch = [&](int c) -> int { return c + (c < DK ? seg0 : (c < 2 * DK ? seg1 : seg2)); };

    // 1. stage this unit's conv weights, window and first token block (cp.async)
    for (int e = tid; e < NCH * GDN_KMAX / EPV && K == GDN_KMAX; e += NT) {
      const int c = e * EPV / GDN_KMAX, within = e * EPV % GDN_KMAX;
      gcp16(&sm.cwr[c][within], cw + (int64_t)gch(c) * GDN_KMAX + within);
    }
    if (K != GDN_KMAX) {
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

    // 2. this unit's state: shared memory → registers (thread (rg, cg) holds rows
    //    RB·rg .. RB·rg+RB-1 of columns 4cg..4cg+3 as packed row pairs), then the next
    //    unit's prefetch
    gdn_wait(&sm.bar, it & 1u);
    uint64_t S[4][RB / 2];
#pragma unroll
    for (int p = 0; p < RB / 2; ++p) {
      const float4 r0 = *reinterpret_cast<const float4*>(&sm.sst[(RB * rg + 2 * p) * DV + 4 * cg]);
      const float4 r1 = *reinterpret_cast<const float4*>(&sm.sst[(RB * rg + 2 * p + 1) * DV + 4 * cg]);
      S[0][p] = pk2(r0.x, r1.x);
      S[1][p] = pk2(r0.y, r1.y);
      S[2][p] = pk2(r0.z, r1.z);
      S[3][p] = pk2(r0.w, r1.w);
    }
    asm volatile("cp.async.wait_all;" ::: "memory");
    __syncthreads();   // sst consumed; inputs staged
    if (tid == 0 && u + (int)gridDim.x < units)
      gdn_prefetch_state(sm.sst, L.state + (int64_t)(u + gridDim.x) * DK * DV, &sm.bar, SBYTES);

    const float A = -expf(dt<T>::to_f(static_cast<const T*>(L.a_log)[h]));
    const float dtb = dt<T>::to_f(static_cast<const T*>(L.dt_bias)[h]);
    const int c_first = ((h % vpk) == 0) ? 0 : 2 * DK;   // conv-history ownership (seq kernel)

    for (int t0 = 0; t0 < T_; t0 += GDN_TB) {
      const int n = min(GDN_TB, T_ - t0);
      // 3. conv + SiLU (the prep kernel's arithmetic), gates
      for (int c = tid; c < NCH; c += NT) {
        float w[GDN_KMAX];
#pragma unroll
        for (int j = 0; j < GDN_KMAX; ++j) w[j] = j < K ? dt<T>::to_f(sm.cwr[c][j]) : 0.f;
        for (int t = 0; t < n; ++t) {
          float acc = 0.f;
#pragma unroll
          for (int j = 0; j < GDN_KMAX; ++j)
            if (j < K) acc = fmaf(w[j], dt<T>::to_f(sm.xr[t + j][c]), acc);
          const float a = dt<T>::round(siluf_(dt<T>::round(acc)));
          if (c < DK) sm.vec[GDN_TB + t][c] = a;
          else if (c < 2 * DK) sm.vec[t][c - DK] = a;
          else sm.vv[t][c - 2 * DK] = a;
        }
      }
      if (tid < n) {
        sm.beta[tid] = dt<T>::round(sigmoidf_(sm.ab[tid][0]));
        sm.dcy[tid] = expf(A * softplusf_(sm.ab[tid][1] + dtb));
      }
      __syncthreads();
      // 4. l2norm of q and k (warp per vector; x·round(rsqrt(round(Σ round(x²)) + 1e-6)))
      for (int vi = warp; vi < 2 * n; vi += NT / 32) {
        const int t = vi >> 1;
        const bool isk = vi & 1;
        float* xv = sm.vec[isk ? t : GDN_TB + t];
        float ss = 0.f;
#pragma unroll
        for (int i = lane; i < DK; i += 32) ss += dt<T>::round(xv[i] * xv[i]);
        ss = warp_sum(ss);
        const float sq = dt<T>::round(dt<T>::round(ss) + 1e-6f);
        const float r = dt<T>::round(rsqrtf(sq));
#pragma unroll
        for (int i = lane; i < DK; i += 32) {
          const float y = dt<T>::round(xv[i] * r);
          xv[i] = isk ? y : y * qscale;
        }
      }
      __syncthreads();
      // 5. Gram products in the prep kernel's order, straight into the coefficient tables
      //    (Γ(r, s) = d_{r+1}···d_s), and Γ(−1, s), Γ(s, n−1)
      const int nkk = n * (n - 1) / 2, nkq = n * (n + 1) / 2;
      for (int e = warp; e < nkk + nkq; e += NT / 32) {
        int s, t;
        const bool isq = e >= nkk;
        if (!isq) {   // pairs s < t
          int rem = e;
          t = 1;
          while (rem >= t) { rem -= t; ++t; }
          s = rem;
        } else {      // pairs s <= t
          int rem = e - nkk;
          t = 0;
          while (rem >= t + 1) { rem -= t + 1; ++t; }
          s = rem;
        }
        const float* ks = sm.vec[s];
        const float* o = sm.vec[isq ? GDN_TB + t : t];
        float acc = 0.f;
#pragma unroll
        for (int i = lane; i < DK; i += 32) acc = fmaf(ks[i], o[i], acc);
        acc = warp_sum(acc);
        if (lane == 0) {
          float ratio = 1.f;
          for (int i = s + 1; i <= t; ++i) ratio = __fmul_rn(ratio, sm.dcy[i]);
          if (isq) sm.tabB[s][t] = __fmul_rn(ratio, acc);
          else sm.tabA[s][t] = __fmul_rn(ratio, acc);
        }
      }
      if (tid < n) {
        float ratio = 1.f;
        for (int i = 0; i <= tid; ++i) ratio = __fmul_rn(ratio, sm.dcy[i]);
        sm.gam[tid] = ratio;
        float tl = 1.f;
        for (int i = tid + 1; i <= n - 1; ++i) tl = __fmul_rn(tl, sm.dcy[i]);
        sm.tail[tid] = tl;
      }
      __syncthreads();
      // 6. Sᵀk_s and Sᵀq_t (four slots per pass), δ_s and o_t of this lane's column
      float Pk[GDN_TB], Pq[GDN_TB], dl[GDN_TB], o[GDN_TB];
#pragma unroll
      for (int i = 0; i < GDN_TB; ++i) Pk[i] = Pq[i] = 0.f;
      const int ng = (n + 3) >> 2;
#pragma unroll 1
      for (int g = 0; g < 2 * ng; ++g) {
        const bool isq = g >= ng;
        const int g4 = isq ? g - ng : g;
        float t4[4] = {0.f, 0.f, 0.f, 0.f};
        const int left = n - 4 * g4;
        const float* vg = sm.vec[(isq ? GDN_TB : 0) + 4 * g4];
        if (left == 1) gdn_dots4<DK, 1>(S, vg, rg, t4);
        else if (left == 2) gdn_dots4<DK, 2>(S, vg, rg, t4);
        else gdn_dots4<DK>(S, vg, rg, t4);
#pragma unroll
        for (int i = 0; i < 4; ++i) {
#pragma unroll
          for (int jj = 0; jj < GDN_TB / 4; ++jj) {
            if (g4 == jj) {
              if (isq) Pq[4 * jj + i] = t4[i];
              else Pk[4 * jj + i] = t4[i];
            }
          }
        }
      }
#pragma unroll
      for (int s = 0; s < GDN_TB; ++s) {
        dl[s] = 0.f;
        if (s < n) {
          float acc = __fmul_rn(sm.gam[s], Pk[s]);
#pragma unroll
          for (int r = 0; r < s; ++r) acc = __fmaf_rn(sm.tabA[r][s], dl[r], acc);
          dl[s] = __fmul_rn(__fsub_rn(sm.vv[s][col], acc), sm.beta[s]);
        }
      }
#pragma unroll
      for (int t = 0; t < GDN_TB; ++t) {
        o[t] = 0.f;
        if (t < n) {
          float acc = __fmul_rn(sm.gam[t], Pq[t]);
#pragma unroll
          for (int r = 0; r <= t; ++r) acc = __fmaf_rn(sm.tabB[r][t], dl[r], acc);
          o[t] = acc;
        }
      }
      // 7. S ← Γ(−1, n−1)·S + Σ_s Γ(s, n−1)·k_s δ_sᵀ
      {
        float c[GDN_TB];
#pragma unroll
        for (int s2 = 0; s2 < GDN_TB; ++s2) c[s2] = s2 < n ? __fmul_rn(sm.tail[s2], dl[s2]) : 0.f;
        gdn_rank<DK>(S, sm.vec[0], sm.gam[n - 1], c, n, rg, lane);
      }
      // 8. RMSNormGated over the dv columns of each token (the chunk kernel's step 6)
      float ssq[GDN_TB];
#pragma unroll
      for (int t = 0; t < GDN_TB; ++t) {
        const float x = dt<T>::round(o[t]);
        ssq[t] = x * x;
      }
#pragma unroll
      for (int sh = 16; sh > 0; sh >>= 1)
#pragma unroll
        for (int t = 0; t < GDN_TB; ++t) ssq[t] += __shfl_xor_sync(0xffffffffu, ssq[t], sh);
      if (lane == 0) {
#pragma unroll
        for (int t = 0; t < GDN_TB; ++t)
          if (t < n) sm.red[warp][t] = ssq[t];
      }
      __syncthreads();
#pragma unroll
      for (int t = 0; t < GDN_TB; ++t) {
        if (t < n) {
          float ss = 0.f;
          for (int w2 = 0; w2 < (DV + 31) / 32; ++w2) ss += sm.red[w2][t];
          const float inv = rsqrtf(ss / (float)DV + L.eps);
          const float xh = dt<T>::round(dt<T>::round(o[t]) * inv);
          const float wx = dt<T>::round(wn * xh);
          out[(int64_t)(b * T_ + t0 + t) * L.ld_out + h * DV + col] = dt<T>::from_f(wx * siluf_(dt<T>::to_f(sm.zr[t][col])));
        }
      }
      // 9. the conv window: after the last block, written to the other parity; otherwise
      //    slid (its last K-1 combined rows to the front) and the next block staged
      const bool last = t0 + n >= T_;
      if (last) {
        for (int i = 0; i < K - 1; ++i)
          for (int cc = c_first + tid * EPV; cc < NCH; cc += NT * EPV)
            *reinterpret_cast<uint4*>(hist_out + (int64_t)i * conv_dim + gch(cc)) =
                *reinterpret_cast<const uint4*>(&sm.xr[n + i][cc]);
      } else {
        constexpr int SLIDE = ((GDN_KMAX - 1) * NCH + NT - 1) / NT;
        T keep[SLIDE];
        __syncthreads();   // every thread is done with this block's rows
#pragma unroll
        for (int q4 = 0; q4 < SLIDE; ++q4) {
          const int e = tid + q4 * NT;
          keep[q4] = e < (K - 1) * NCH ? sm.xr[n + e / NCH][e % NCH] : T{};
        }
        __syncthreads();
#pragma unroll
        for (int q4 = 0; q4 < SLIDE; ++q4) {
          const int e = tid + q4 * NT;
          if (e < (K - 1) * NCH) sm.xr[e / NCH][e % NCH] = keep[q4];
        }
        stage_tokens(t0 + n, min(GDN_TB, T_ - t0 - n));
        asm volatile("cp.async.commit_group;" ::: "memory");
        asm volatile("cp.async.wait_all;" ::: "memory");
      }
      __syncthreads();   // the next block (or unit) overwrites the vector slots and tables
    }
    // 10. the committed state
#pragma unroll
    for (int p = 0; p < RB / 2; ++p) {
      const float2 a = upk2(S[0][p]), bq = upk2(S[1][p]), c2 = upk2(S[2][p]), d2 = upk2(S[3][p]);
      float* d0 = state + (int64_t)(RB * rg + 2 * p) * DV + 4 * cg;
      *reinterpret_cast<float4*>(d0) = make_float4(a.x, bq.x, c2.x, d2.x);
      *reinterpret_cast<float4*>(d0 + DV) = make_float4(a.y, bq.y, c2.y, d2.y);
    }
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

template <typename K>
static int reserve_smem(K kern, size_t smem, bool& done) {
  if (!done) {
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess)
      return set_error(QSP_ERR_CUDA, "qsp_gdn_verify: cannot reserve %zu bytes of shared memory", smem);
    done = true;
  }
  return QSP_OK;
}

template <typename T, int DK, int DV>
static int launch_gdn_dims(const qsp_gdn_layer& L, cudaStream_t st) {
  const GdnRing RG = gdn_ring(L.batch, L.n_v_heads, L.max_spec_tokens, DK, DV, (int)sizeof(T));
  const int units = L.batch * L.n_v_heads;
  const int grid = std::min(units, 2 * sm_count_gdn());
  // the update kernel sizes its per-call token loops by max_spec_tokens (4 in the verify step)
  const bool tb4 = L.max_spec_tokens <= 4;
  auto chunk = tb4 ? gdn_chunk_kernel<T, DK, DV, 4> : gdn_chunk_kernel<T, DK, DV, GDN_TB>;
  const size_t csmem = tb4 ? sizeof(GdnChunkSmem<T, DK, DV, 4>) : sizeof(GdnChunkSmem<T, DK, DV, GDN_TB>);
  static bool chunk_set[2] = {false, false};
  int rc = reserve_smem(chunk, csmem, chunk_set[tb4]);
  if (rc) return rc;
  if (L.tokens <= L.max_spec_tokens) {
    const int nchg = 2 * DK + (L.n_v_heads / L.n_k_heads) * DV;
    const size_t psmem = gdn_prep_smem(nchg, L.conv_kernel, L.tokens, DK, (int)sizeof(T));
    const int vpk = L.n_v_heads / L.n_k_heads;
    if (vpk != 1 && vpk != 2 && vpk != 4)
      return set_error(QSP_ERR_UNSUPPORTED, "qsp_gdn_verify: %d value heads per key head not built (1, 2 or 4)", vpk);
    // the verify step's shape (conv width 4, 4 tokens) runs a specialised instance
    const bool fixed = L.conv_kernel == 4 && L.tokens == 4;
    auto prep = fixed ? (vpk == 1 ? gdn_prep_kernel<T, DK, DV, 1, 4, 4>
                                  : (vpk == 2 ? gdn_prep_kernel<T, DK, DV, 2, 4, 4> : gdn_prep_kernel<T, DK, DV, 4, 4, 4>))
                      : (vpk == 1 ? gdn_prep_kernel<T, DK, DV, 1>
                                  : (vpk == 2 ? gdn_prep_kernel<T, DK, DV, 2> : gdn_prep_kernel<T, DK, DV, 4>));
    static size_t prep_set[2][5] = {{0, 0, 0, 0, 0}, {0, 0, 0, 0, 0}};
    if (psmem > prep_set[fixed][vpk]) {
      if (cudaFuncSetAttribute(prep, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)psmem) != cudaSuccess)
        return set_error(QSP_ERR_CUDA, "qsp_gdn_verify: cannot reserve %zu bytes of shared memory", psmem);
      prep_set[fixed][vpk] = psmem;
    }
    rc = launch_pdl("qsp_gdn_verify(prep)", prep, dim3(L.batch * L.n_k_heads), dim3(256), psmem, st, L, RG);
    if (rc) return rc;
    return launch_pdl("qsp_gdn_verify(chunk)", chunk, dim3(grid), dim3(DV), csmem, st, L, RG, (int)L.tokens);
  }
  // long commit call: replay kept tokens into the state, then the tokens in 8-token blocks
  rc = launch_pdl("qsp_gdn_verify(replay)", chunk, dim3(grid), dim3(DV), csmem, st, L, RG, 0);
  if (rc) return rc;
  auto pf = gdn_prefill_kernel<T, DK, DV>;
  const size_t pfsmem = sizeof(GdnPrefillSmem<T, DK, DV>);
  static bool pf_set = false;
  rc = reserve_smem(pf, pfsmem, pf_set);
  if (rc) return rc;
  return launch_pdl("qsp_gdn_verify(prefill)", pf, dim3(grid), dim3(DV), pfsmem, st, L);
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
  QSP_REQUIRE(aligned(L.state, 16) && aligned(L.pending, 16) && aligned(L.proj, 16) && aligned(L.conv_hist, 16) &&
                  aligned(L.conv_w, 16),
              "qsp_gdn_verify: state/pending/proj/conv_hist/conv_w must be 16-byte aligned");
  const int esz = L.dtype == QSP_F32 ? 4 : 2;
  QSP_REQUIRE((L.ld_proj * esz) % 16 == 0, "qsp_gdn_verify: ld_proj must be a multiple of 16 bytes");
  QSP_DISPATCH_DTYPE(L.dtype, T, { return launch_gdn<T>(L, as_stream(stream)); });
}

extern "C" size_t qsp_gdn_pending_bytes(int32_t batch, int32_t n_k_heads, int32_t n_v_heads, int32_t head_k,
                                        int32_t head_v, int32_t max_spec_tokens, int32_t dtype) {
  if (batch <= 0 || n_k_heads <= 0 || n_v_heads <= 0 || head_k <= 0 || head_v <= 0 || max_spec_tokens <= 0)
    return 0;
  const int esz = dtype == QSP_F32 ? 4 : 2;
  const GdnRing RG = gdn_ring(batch, n_v_heads, max_spec_tokens, head_k, head_v, esz);
  return (size_t)2 * batch * n_v_heads * max_spec_tokens * (RG.recA + RG.recB);
}
