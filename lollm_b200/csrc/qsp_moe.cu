// Sparse MoE FFN of the qwen3_5_moe family (src/qwen3_5_moe/blocks.py:347-421) for the
// verify step: router + top-k + routed SwiGLU experts + shared expert, then the residual add
// and the next RMSNorm.
//
// Launches (one stream, in order):
//   1. router GEMM      R = xn · [router | shared gate | pad | shared gate_proj | shared up]ᵀ
//   2. moe_route        per token: fp32 softmax over the expert logits, top-k (largest value,
//                       then lowest index), optional renormalisation, weights rounded to the
//                       model dtype, selected experts sorted ascending; a rank inside each
//                       expert's token list (atomic counter); shared-expert SwiGLU + gate
//   3. moe_gather       exclusive scan of the per-expert counts → offsets; every (token, slot)
//                       pair gets its row in expert-sorted order and its input row copied there
//   4. expert gate|up   grouped GEMM over the sorted rows, SwiGLU in the epilogue
//   5. expert down      grouped GEMM, product · routing weight in the epilogue (per pair)
//   6. shared down      plain GEMM
//   7. moe_combine      per token: Σ over its experts in ascending expert order, rounding to
//                       the model dtype after every add (index_add_ into a model-dtype buffer),
//                       + σ(shared gate)·shared, residual add, next RMSNorm
// bf16 runs steps 4-5 on tcgen05 tensor cores: a persistent CTA per SM walks work units
// (expert, 128 output rows), streaming the expert's weight rows through a TMA ring once per
// 64 routed tokens, with the expert's sorted token rows as the MMA N dimension. fp32 (parity
// configurations) runs them on CUDA cores. The position of a pair inside its expert's list
// depends on atomic order, but every output column of a GEMM is computed independently of
// the others, so results do not depend on it.
#include "qsp_common.cuh"
#include "qsp_tc.cuh"

namespace qsp {

__device__ int g_moe_dev_error = 0;

int moe_device_error(int reset) {
  int v = 0;
  if (cudaMemcpyFromSymbol(&v, g_moe_dev_error, sizeof(int)) != cudaSuccess) return 0;
  if (reset && v) {
    const int zero = 0;
    cudaMemcpyToSymbol(g_moe_dev_error, &zero, sizeof(int));
  }
  return v;
}

constexpr int MOE_MAX_EXPERTS = 1024;
constexpr int MOE_MAX_TOPK = 16;
constexpr int MOE_MAX_HIDDEN = 8192;

static int64_t round_up(int64_t v, int64_t a) { return (v + a - 1) / a * a; }

int64_t moe_router_rows(int64_t E, int64_t Is) { return round_up(E + (Is > 0 ? 1 : 0), 8); }

// ------------------------------------------------------------------ workspace layout
struct MoeWs {
  size_t r, act_s, sig, idx, wts, rank, pos_of, counts, offsets, tok_of, w_of, e_of, xs, as, yw, s, gemm, total;
  int64_t n_route, n_in, pairs;
};

static MoeWs moe_layout(int64_t m, int64_t H, int64_t E, int64_t k, int64_t I, int64_t Is, int dtype) {
  const size_t es = dtype == QSP_BF16 ? 2 : 4;
  MoeWs w{};
  size_t off = 0;
  auto take = [&](size_t b) {
    const size_t o = off;
    off += (b + 255) & ~size_t(255);
    return o;
  };
  w.n_route = moe_router_rows(E, Is);
  w.n_in = w.n_route + 2 * Is;
  w.pairs = m * k;
  const size_t P = (size_t)w.pairs;
  w.r = take((size_t)m * w.n_in * es);
  w.act_s = take((size_t)m * (Is > 0 ? Is : 1) * es);
  w.sig = take((size_t)m * 4);
  w.idx = take(P * 4);
  w.wts = take(P * 4);
  w.rank = take(P * 4);
  w.pos_of = take(P * 4);
  w.counts = take((size_t)E * 4);
  w.offsets = take((size_t)(E + 1) * 4);
  w.tok_of = take(P * 4);
  w.w_of = take(P * 4);
  w.e_of = take(P * 4);
  w.xs = take(P * H * es);
  w.as = take(P * I * es);
  w.yw = take(P * H * es);
  w.s = take((size_t)m * H * es);
  const size_t g1 = qsp_gemm_workspace_bytes(m, w.n_in, H, dtype);
  const size_t g2 = Is > 0 ? qsp_gemm_workspace_bytes(m, H, Is, dtype) : 0;
  w.gemm = take(std::max(std::max(g1, g2), (size_t)256));
  w.total = off;
  return w;
}

// ------------------------------------------------------------------ 2. route
// One warp per token. Shared memory: this warp's copy of the expert logits.
template <typename T>
__global__ void __launch_bounds__(256) moe_route_kernel(const T* __restrict__ R, int64_t ld_r, int m, int E,
                                                        int k, int norm, int Is, int n_route,
                                                        int* __restrict__ idx, float* __restrict__ wts,
                                                        int* __restrict__ rank, int* __restrict__ counts,
                                                        T* __restrict__ act_s, float* __restrict__ sig) {
  pdl_trigger();
  pdl_wait();
  extern __shared__ float route_smem[];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int t = blockIdx.x * 8 + warp;
  if (t >= m) return;
  float* lg = route_smem + (size_t)warp * E;
  __shared__ int sel_e[8][MOE_MAX_TOPK];
  __shared__ float sel_p[8][MOE_MAX_TOPK];
  const T* row = R + (int64_t)t * ld_r;
  float mx = -INFINITY;
  for (int j = lane; j < E; j += 32) {
    const float v = dt<T>::to_f(row[j]);
    lg[j] = v;
    mx = fmaxf(mx, v);
  }
  mx = warp_max(mx);
  float z = 0.f;
  for (int j = lane; j < E; j += 32) z += expf(lg[j] - mx);
  z = warp_sum(z);
  __syncwarp();
  // top-k by repeated warp argmax; ties go to the lower expert index
  float psum = 0.f;
  for (int r = 0; r < k; ++r) {
    float bv = -INFINITY;
    int bi = 0x7fffffff;
    for (int j = lane; j < E; j += 32) {
      const float v = lg[j];
      if (v > bv || (v == bv && j < bi)) { bv = v; bi = j; }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
      const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
      if (ov > bv || (ov == bv && oi < bi)) { bv = ov; bi = oi; }
    }
    const float p = expf(bv - mx) / z;   // softmax(logits, fp32)[bi]
    psum += p;
    if (lane == 0) {
      sel_e[warp][r] = bi;
      sel_p[warp][r] = p;
      lg[bi] = -INFINITY;
    }
    __syncwarp();
  }
  if (lane == 0) {
    // ascending expert order: the order the reference's expert loop adds the outputs in
    for (int a = 1; a < k; ++a) {
      const int e = sel_e[warp][a];
      const float p = sel_p[warp][a];
      int b = a - 1;
      while (b >= 0 && sel_e[warp][b] > e) {
        sel_e[warp][b + 1] = sel_e[warp][b];
        sel_p[warp][b + 1] = sel_p[warp][b];
        --b;
      }
      sel_e[warp][b + 1] = e;
      sel_p[warp][b + 1] = p;
    }
  }
  __syncwarp();
  if (lane < k) {
    const int e = sel_e[warp][lane];
    float w = sel_p[warp][lane];
    if (norm) w = w / psum;
    const int64_t pi = (int64_t)t * k + lane;
    idx[pi] = e;
    wts[pi] = dt<T>::round(w);
    rank[pi] = atomicAdd(&counts[e], 1);
  }
  if (Is > 0) {
    if (lane == 0) sig[t] = dt<T>::round(sigmoidf_(dt<T>::to_f(row[E])));
    T* a = act_s + (int64_t)t * Is;
    for (int j = lane; j < Is; j += 32) {
      const float g = dt<T>::to_f(row[n_route + j]);
      const float u = dt<T>::to_f(row[n_route + Is + j]);
      a[j] = dt<T>::from_f(dt<T>::round(siluf_(g)) * u);
    }
  }
}

// ------------------------------------------------------------------ 3. gather
// Every block scans the counts (E ≤ 1024) into shared offsets; block 0 also publishes them.
// One warp per (token, slot) pair copies the token's input row to the pair's sorted row.
template <typename T>
__global__ void __launch_bounds__(256) moe_gather_kernel(const T* __restrict__ xn, int64_t ld_xn, int m, int H,
                                                         int E, int k, const int* __restrict__ idx,
                                                         const float* __restrict__ wts,
                                                         const int* __restrict__ rank,
                                                         const int* __restrict__ counts, int* __restrict__ offsets,
                                                         int* __restrict__ pos_of, int* __restrict__ tok_of,
                                                         float* __restrict__ w_of, int* __restrict__ e_of,
                                                         T* __restrict__ xs, int32_t* __restrict__ counts_out) {
  pdl_trigger();
  pdl_wait();
  __shared__ int offs[MOE_MAX_EXPERTS + 1];
  __shared__ int wsum[8];
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  // thread tid owns experts 4·tid .. 4·tid+3
  int c[4], loc = 0;
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    const int e = tid * 4 + q;
    c[q] = e < E ? counts[e] : 0;
    loc += c[q];
  }
  int incl = loc;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int v = __shfl_up_sync(0xffffffffu, incl, o);
    if (lane >= o) incl += v;
  }
  if (lane == 31) wsum[warp] = incl;
  __syncthreads();
  int base = 0;
  for (int w = 0; w < warp; ++w) base += wsum[w];
  int run = base + incl - loc;
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    const int e = tid * 4 + q;
    if (e < E) offs[e] = run;
    run += c[q];
  }
  if (tid == 255) offs[E] = run;   // total (E ≤ 1024 = 4·256)
  __syncthreads();
  if (blockIdx.x == 0) {
    for (int e = tid; e <= E; e += 256) offsets[e] = offs[e];
    if (counts_out)
      for (int e = tid; e < E; e += 256) counts_out[e] = counts[e];
  }
  const int64_t p = (int64_t)blockIdx.x * 8 + warp;
  if (p >= (int64_t)m * k) return;
  const int t = (int)(p / k);
  const int e = idx[p];
  const int pos = offs[e] + rank[p];
  if (lane == 0) {
    pos_of[p] = pos;
    tok_of[pos] = t;
    w_of[pos] = wts[p];
    e_of[pos] = e;
  }
  const T* src = xn + (int64_t)t * ld_xn;
  T* dst = xs + (int64_t)pos * H;
  constexpr int V = 16 / sizeof(T);
  if ((H % V) == 0 && (((uintptr_t)src) & 15) == 0) {
    const int4* s4 = reinterpret_cast<const int4*>(src);
    int4* d4 = reinterpret_cast<int4*>(dst);
    for (int j = lane; j < H / V; j += 32) d4[j] = s4[j];
  } else {
    for (int j = lane; j < H; j += 32) dst[j] = src[j];
  }
}

// ------------------------------------------------------------------ 4/5 on CUDA cores
// One warp per output element (fixed lane-strided order + butterfly sum): the fp32 path.
template <typename T>
__global__ void __launch_bounds__(256) moe_gate_up_simt_kernel(const T* __restrict__ xs, int H,
                                                               const T* __restrict__ gu, int I,
                                                               const int* __restrict__ e_of, int P,
                                                               T* __restrict__ as) {
  pdl_trigger();
  pdl_wait();
  const int pos = blockIdx.x;
  const int j = blockIdx.y * 8 + (threadIdx.x >> 5), lane = threadIdx.x & 31;
  if (pos >= P || j >= I) return;
  const int e = e_of[pos];
  const T* x = xs + (int64_t)pos * H;
  const T* wg = gu + ((int64_t)e * 2 * I + j) * H;
  const T* wu = wg + (int64_t)I * H;
  float g = 0.f, u = 0.f;
  for (int h = lane; h < H; h += 32) {
    const float xv = dt<T>::to_f(x[h]);
    g = fmaf(xv, dt<T>::to_f(wg[h]), g);
    u = fmaf(xv, dt<T>::to_f(wu[h]), u);
  }
  g = warp_sum(g);
  u = warp_sum(u);
  if (lane == 0)
    as[(int64_t)pos * I + j] = dt<T>::from_f(dt<T>::round(siluf_(dt<T>::round(g))) * dt<T>::round(u));
}

template <typename T>
__global__ void __launch_bounds__(256) moe_down_simt_kernel(const T* __restrict__ as, int I,
                                                            const T* __restrict__ dn, int H,
                                                            const int* __restrict__ e_of,
                                                            const float* __restrict__ w_of, int P,
                                                            T* __restrict__ yw) {
  pdl_trigger();
  pdl_wait();
  const int pos = blockIdx.x;
  const int n = blockIdx.y * 8 + (threadIdx.x >> 5), lane = threadIdx.x & 31;
  if (pos >= P || n >= H) return;
  const int e = e_of[pos];
  const T* a = as + (int64_t)pos * I;
  const T* w = dn + ((int64_t)e * H + n) * I;
  float d = 0.f;
  for (int j = lane; j < I; j += 32) d = fmaf(dt<T>::to_f(a[j]), dt<T>::to_f(w[j]), d);
  d = warp_sum(d);
  if (lane == 0) yw[(int64_t)pos * H + n] = dt<T>::from_f(dt<T>::round(d) * w_of[pos]);
}

// ------------------------------------------------------------------ 4/5 on tensor cores
// Work unit = (expert e, a block of weight rows). For each tile of ≤ 64 of the expert's
// sorted token rows, the unit streams the expert's weight rows over K through the ring; the
// MMA is D[128 weight rows × N tokens] += W[128 × 16] · Xᵀ[16 × N] with N = the tile's rows
// rounded up to 16, one accumulator per 128-row weight tile (NA of them per stage).
// SWI (gate|up): the two tiles are gate rows and the matching up rows, SwiGLU in the
// epilogue. Otherwise (down): NA consecutive 128-row tiles of output rows, each product times
// the pair's routing weight in the epilogue.
template <int NA>
struct MoeTcCfg {
  static constexpr int TN = 64;                   // token rows per tile
  static constexpr int A_BYTES = 128 * 64 * 2;    // 128 weight rows x 64 K (bf16)
  static constexpr int B_BYTES = TN * 64 * 2;
  static constexpr int STAGE = NA * A_BYTES + B_BYTES;
  static constexpr int STAGES = (200 * 1024) / STAGE;
  static constexpr int ACC_COLS = TN;
  static constexpr int BUF_COLS = NA * ACC_COLS;  // one tile's accumulators
  static constexpr uint32_t TMEM_COLS = 256;      // two tiles in flight (epilogue overlaps MMA)
  static constexpr size_t SMEM = (size_t)STAGES * STAGE + 1024 + 256;
};

struct MoeTcArgs {
  const int* offsets;      // [E+1] expert row ranges in sorted order
  int E, RB, n_kb;         // experts, 128-row output blocks per expert, 64-wide K blocks
  int rows_per_expert;     // weight rows per expert in the 2-D view (2I or H)
  int out_w;               // output width (I for gate|up, H for down)
  __nv_bfloat16* out;      // [P, out_w]: As (gate|up) or Yw (down)
  const float* w_of;       // [P] routing weight per sorted row (down)
};

template <int NA, bool SWI>
__global__ void __launch_bounds__(192, 1)
moe_tc_kernel(const __grid_constant__ CUtensorMap tm_w, const __grid_constant__ CUtensorMap tm_x, const MoeTcArgs A) {
  pdl_trigger();
  pdl_wait();
  using C = MoeTcCfg<NA>;
  using namespace tc;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + C::STAGES * C::STAGE);
  uint64_t* empty = full + C::STAGES;
  uint64_t* acc_full = empty + C::STAGES;   // [2]
  uint64_t* acc_empty = acc_full + 2;       // [2]
  uint32_t* tslot = reinterpret_cast<uint32_t*>(acc_empty + 2);
  volatile int* abort = reinterpret_cast<volatile int*>(tslot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int units = A.E * A.RB;
  if (threadIdx.x == 0) {
    for (int s = 0; s < C::STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&acc_full[b], 1);
      mbar_init(&acc_empty[b], 128);
    }
    *abort = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 1) tmem_alloc(tslot, C::TMEM_COLS);
  fence_before();
  __syncthreads();
  fence_after();
  const uint32_t tmem = *tslot;

  if (warp == 0) {
    // producer: the whole warp runs the loop, one elected lane issues (qsp_tc.cuh)
    if (lane == 0) {
      asm volatile("prefetch.tensormap [%0];" ::"l"(&tm_w) : "memory");
      asm volatile("prefetch.tensormap [%0];" ::"l"(&tm_x) : "memory");
    }
    __syncwarp();
    uint32_t it = 0;
    bool ok = true;
    for (int u = blockIdx.x; u < units && ok; u += gridDim.x) {
      const int e = u / A.RB, rb = u % A.RB;
      const int off = __ldg(&A.offsets[e]), n_e = __ldg(&A.offsets[e + 1]) - off;
      const int row0 = e * A.rows_per_expert + rb * (SWI ? 128 : 128 * NA);
      for (int t0 = 0; t0 < n_e && ok; t0 += C::TN) {
        // one TMA box per operand and stage (an SM's TMA moves a bounded number of boxes per
        // µs): both weight tiles as one box (SWI: a 3-D box over [gate, up] halves; otherwise
        // NA·128 consecutive rows), the expert's token rows as one TN-row box (rows past the
        // expert's belong to the next expert or read as zeros past the last row; the MMA's N
        // covers only the expert's own)
        const uint32_t bytes = NA * C::A_BYTES + C::B_BYTES;
        for (int kb = 0; kb < A.n_kb; ++kb, ++it) {
          const int s = it % C::STAGES;
          const uint32_t ph = (it / C::STAGES) & 1u;
          if (it >= (uint32_t)C::STAGES && !mbar_wait_warp(&empty[s], ph ^ 1u, 201, &g_moe_dev_error, abort)) {
            ok = false;
            break;
          }
          uint8_t* st = smem + s * C::STAGE;
          mbar_expect_tx_warp(&full[s], bytes);
          if (SWI) {
            asm volatile(
                "{\n\t.reg .pred e;\n\t.reg .b64 pol;\n\telect.sync _|e, 0xffffffff;\n\t"
                "createpolicy.fractional.L2::evict_first.b64 pol, 1.0;\n\t"
                "@e cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1, "
                "{%3, %4, %5}], [%2], pol;\n\t}" ::"r"(smem_u32(st)),
                "l"(&tm_w), "r"(smem_u32(&full[s])), "r"(kb * 64), "r"(row0), "r"(0)
                : "memory");
          } else {
            tma_load_2d_evict_first_warp(st, &tm_w, &full[s], kb * 64, row0);
          }
          tma_load_2d_warp(st + NA * C::A_BYTES, &tm_x, &full[s], kb * 64, off + t0);
        }
      }
    }
  } else if (warp == 1) {
    // MMA issuer: the whole warp runs the loop, one elected lane issues
    uint32_t it = 0, ti = 0;
    bool ok = true;
    for (int u = blockIdx.x; u < units; u += gridDim.x) {
      const int e = u / A.RB;
      const int off = __ldg(&A.offsets[e]), n_e = __ldg(&A.offsets[e + 1]) - off;
      for (int t0 = 0; t0 < n_e; t0 += C::TN, ++ti) {
        const int nt = min(C::TN, n_e - t0);
        const uint32_t idesc = idesc_bf16(128, max(16, (nt + 15) & ~15));
        const uint32_t buf = ti & 1u, use = ti >> 1;
        if (ok && use >= 1 && !mbar_wait_warp(&acc_empty[buf], (use - 1) & 1u, 204, &g_moe_dev_error, abort)) ok = false;
        fence_after();
        const uint32_t d = tmem + buf * C::BUF_COLS;
        for (int kb = 0; kb < A.n_kb; ++kb, ++it) {
          const int s = it % C::STAGES;
          const uint32_t ph = (it / C::STAGES) & 1u;
          if (ok && !mbar_wait_warp(&full[s], ph, 202, &g_moe_dev_error, abort)) ok = false;
          fence_after();
          if (ok) {
            const uint32_t a0 = smem_u32(smem + s * C::STAGE);
            const uint32_t b0 = a0 + NA * C::A_BYTES;
#pragma unroll
            for (int q = 0; q < NA; ++q)
              umma4_bf16_warp(d + q * C::ACC_COLS, sdesc_sw128(a0 + q * C::A_BYTES), sdesc_sw128(b0), idesc,
                              kb > 0 ? 1u : 0u);
          }
          umma_commit_warp(&empty[s]);
        }
        umma_commit_warp(&acc_full[buf]);
      }
    }
  } else {
    // epilogue: warp w reads TMEM lanes 32·(w%4)..+31 = output rows rb·128 + 32·(w%4) + lane
    const int quad = warp & 3;
    uint32_t ti = 0;
    for (int u = blockIdx.x; u < units; u += gridDim.x) {
      const int e = u / A.RB, rb = u % A.RB;
      const int off = __ldg(&A.offsets[e]), n_e = __ldg(&A.offsets[e + 1]) - off;
      const int orow = rb * (SWI ? 128 : 128 * NA) + quad * 32 + lane;
      for (int t0 = 0; t0 < n_e; t0 += C::TN, ++ti) {
        const int nt = min(C::TN, n_e - t0);
        const uint32_t buf = ti & 1u, use = ti >> 1;
        const bool ok = mbar_wait(&acc_full[buf], use & 1u, 203, &g_moe_dev_error, abort);
        fence_after();
        const uint32_t tb = tmem + buf * C::BUF_COLS + ((uint32_t)(quad * 32) << 16);
        for (int c0 = 0; c0 < nt; c0 += 32) {
          float v[32];
          tmem_ld32(tb + c0, v);
          if (SWI) {
            float w[32];
            tmem_ld32(tb + C::ACC_COLS + c0, w);
            if (ok && orow < A.out_w) {
#pragma unroll
              for (int j = 0; j < 32; ++j) {
                if (c0 + j < nt) {
                  const int pos = off + t0 + c0 + j;
                  const float g = dt<__nv_bfloat16>::round(v[j]);
                  const float s = dt<__nv_bfloat16>::round(siluf_(g));
                  A.out[(int64_t)pos * A.out_w + orow] = __float2bfloat16_rn(s * dt<__nv_bfloat16>::round(w[j]));
                }
              }
            }
          } else {
            // down projection: accumulator q holds output rows orow + 128·q
#pragma unroll
            for (int q = 0; q < NA; ++q) {
              if (q > 0) tmem_ld32(tb + q * C::ACC_COLS + c0, v);
              const int oq = orow + q * 128;
              if (ok && oq < A.out_w) {
#pragma unroll
                for (int j = 0; j < 32; ++j) {
                  if (c0 + j < nt) {
                    const int pos = off + t0 + c0 + j;
                    const float r = dt<__nv_bfloat16>::round(v[j]);
                    A.out[(int64_t)pos * A.out_w + oq] = __float2bfloat16_rn(r * __ldg(&A.w_of[pos]));
                  }
                }
              }
            }
          }
        }
        fence_before();
        mbar_arrive(&acc_empty[buf]);
      }
    }
  }
  fence_before();
  __syncthreads();
  if (warp == 1) {
    fence_after();
    tmem_dealloc(tmem, C::TMEM_COLS);
  }
}

// The stacked [E·2I, H] gate|up weight viewed as [2 halves (gate, up; I rows apart)][E·2I − I
// rows][H]: a box of 64 columns × 128 rows × both halves brings a unit's 128 gate rows and the
// matching 128 up rows in one request, laid out as the two 128-row tiles one after the other
// (the same rows two 2-D boxes at row0 and row0 + I would bring; rows of the first half past
// E·2I − I read as zeros, so no address leaves the weight).
static bool make_map_gate_up(CUtensorMap* m, const void* base, int64_t E, int64_t I, int64_t H) {
  tc::EncodeTiled enc = tc::get_encode();
  if (!enc) return false;
  cuuint64_t dims[3] = {(cuuint64_t)H, (cuuint64_t)(E * 2 * I - I), 2};
  cuuint64_t strides[2] = {(cuuint64_t)(H * 2), (cuuint64_t)(I * H * 2)};
  cuuint32_t box[3] = {64u, 128u, 2u};
  cuuint32_t es[3] = {1, 1, 1};
  return enc(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(base), dims, strides, box, es,
             CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
             CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

template <int NA, bool SWI>
static int launch_moe_tc(const CUtensorMap& mw, const CUtensorMap& mx, const MoeTcArgs& a, cudaStream_t st) {
  using C = MoeTcCfg<NA>;
  auto kern = moe_tc_kernel<NA, SWI>;
  static bool attr_set = false;
  if (!attr_set) {
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)C::SMEM) != cudaSuccess)
      return set_error(QSP_ERR_CUDA, "qsp_moe_ffn: cannot reserve %zu bytes of shared memory", C::SMEM);
    attr_set = true;
  }
  const int units = a.E * a.RB;
  const int grid = std::min(units, tc::sm_count());
  return launch_pdl("qsp_moe_ffn(tcgen05 experts)", kern, dim3(grid), dim3(192), C::SMEM, st, mw, mx, a);
}

// ------------------------------------------------------------------ 7. combine
// One CTA per token: y = Σ_slots Yw (ascending expert order, model-dtype rounding per add)
// + round(σ·shared); x := round(x + y); optional y_out = RMSNorm(x)·(1+w).
constexpr int CB_MAXV = MOE_MAX_HIDDEN / 1024;
template <typename T>
__global__ void __launch_bounds__(256) moe_combine_kernel(const T* __restrict__ yw, int H, int k,
                                                          const int* __restrict__ pos_of,
                                                          const T* __restrict__ s, const float* __restrict__ sig,
                                                          T* __restrict__ x, int64_t ldx,
                                                          const T* __restrict__ norm_w, T* __restrict__ y,
                                                          int64_t ldy, float eps) {
  pdl_trigger();
  pdl_wait();
  __shared__ float red[32];
  __shared__ int pos[MOE_MAX_TOPK];
  const int t = blockIdx.x;
  if (threadIdx.x < k) pos[threadIdx.x] = pos_of[(int64_t)t * k + threadIdx.x];
  __syncthreads();
  const float g = s ? sig[t] : 0.f;
  float r[CB_MAXV][4];
  float ss = 0.f;
#pragma unroll
  for (int v = 0; v < CB_MAXV; ++v) {
    const int col = (threadIdx.x + v * 256) * 4;
    if (col < H) {
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        if (col + q >= H) break;
        float acc = 0.f;
        for (int j = 0; j < k; ++j) acc = dt<T>::round(acc + dt<T>::to_f(yw[(int64_t)pos[j] * H + col + q]));
        if (s) acc = dt<T>::round(acc + dt<T>::round(g * dt<T>::to_f(s[(int64_t)t * H + col + q])));
        T* xp = x + (int64_t)t * ldx + col + q;
        const float xv = dt<T>::round(dt<T>::to_f(*xp) + acc);
        *xp = dt<T>::from_f(xv);
        r[v][q] = xv;
        ss = fmaf(xv, xv, ss);
      }
    }
  }
  if (!norm_w) return;
  const float tot = block_sum(ss, red);
  const float inv = rsqrtf(tot / (float)H + eps);
#pragma unroll
  for (int v = 0; v < CB_MAXV; ++v) {
    const int col = (threadIdx.x + v * 256) * 4;
    if (col < H) {
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        if (col + q >= H) break;
        y[(int64_t)t * ldy + col + q] = dt<T>::from_f(r[v][q] * inv * (dt<T>::to_f(norm_w[col + q]) + 1.0f));
      }
    }
  }
}

}  // namespace qsp

using namespace qsp;

extern "C" int64_t qsp_moe_router_rows(int32_t n_experts, int32_t shared_inter) {
  if (n_experts <= 0 || shared_inter < 0) return 0;
  return moe_router_rows(n_experts, shared_inter);
}

extern "C" size_t qsp_moe_workspace_bytes(int32_t tokens, int32_t hidden, int32_t n_experts, int32_t top_k,
                                          int32_t inter, int32_t shared_inter, int32_t dtype) {
  if (tokens < 0 || hidden <= 0 || n_experts <= 0 || top_k <= 0 || inter <= 0 || shared_inter < 0) return 0;
  if (dtype != QSP_F32 && dtype != QSP_BF16) return 0;
  return moe_layout(tokens, hidden, n_experts, top_k, inter, shared_inter, dtype).total;
}

extern "C" int qsp_moe_ffn(const qsp_moe_layer* L, void* stream) {
  QSP_REQUIRE(L != nullptr, "qsp_moe_ffn: null layer");
  const int64_t m = L->tokens, H = L->hidden, E = L->n_experts, k = L->top_k, I = L->inter, Is = L->shared_inter;
  QSP_REQUIRE(m >= 0 && H > 0 && I > 0 && Is >= 0, "qsp_moe_ffn: bad sizes");
  QSP_REQUIRE(E >= 1 && E <= MOE_MAX_EXPERTS, "qsp_moe_ffn: n_experts %lld outside [1, %d]", (long long)E,
              MOE_MAX_EXPERTS);
  QSP_REQUIRE(k >= 1 && k <= E && k <= MOE_MAX_TOPK, "qsp_moe_ffn: top_k %lld outside [1, min(E, %d)]",
              (long long)k, MOE_MAX_TOPK);
  QSP_REQUIRE(H <= MOE_MAX_HIDDEN, "qsp_moe_ffn: hidden %lld > %d", (long long)H, MOE_MAX_HIDDEN);
  QSP_REQUIRE(L->dtype == QSP_F32 || L->dtype == QSP_BF16, "qsp_moe_ffn: unsupported dtype %d", (int)L->dtype);
  QSP_REQUIRE(L->xn && L->w_in && L->gate_up && L->down && L->x, "qsp_moe_ffn: null pointer");
  QSP_REQUIRE(Is == 0 || L->shared_down, "qsp_moe_ffn: shared_down is NULL with shared_inter > 0");
  QSP_REQUIRE(!L->norm_w || (L->y && L->ld_y >= H), "qsp_moe_ffn: bad norm output");
  QSP_REQUIRE(L->ld_xn >= H && L->ld_x >= H, "qsp_moe_ffn: leading dimension too small");
  QSP_REQUIRE(m * k < (1ll << 31), "qsp_moe_ffn: too many (token, expert) pairs");
  if (m == 0) return QSP_OK;
  const MoeWs W = moe_layout(m, H, E, k, I, Is, L->dtype);
  QSP_REQUIRE(L->workspace && L->workspace_bytes >= W.total && aligned(L->workspace, 256),
              "qsp_moe_ffn: workspace needs %zu bytes (256-byte aligned), got %zu", W.total, L->workspace_bytes);
  cudaStream_t st = as_stream(stream);
  uint8_t* ws = static_cast<uint8_t*>(L->workspace);
  auto at = [&](size_t o) { return static_cast<void*>(ws + o); };
  int* counts = static_cast<int*>(at(W.counts));
  if (cudaMemsetAsync(counts, 0, (size_t)E * 4, st) != cudaSuccess)
    return set_error(QSP_ERR_CUDA, "qsp_moe_ffn: memset failed");
  const size_t es = L->dtype == QSP_BF16 ? 2 : 4;
  // 1. one GEMM for everything that reads xn: router logits, shared gate, shared gate|up
  int rc = qsp_gemm(L->xn, L->ld_xn, L->w_in, H, at(W.r), W.n_in, m, W.n_in, H, L->dtype, 0, at(W.gemm),
                    W.total - W.gemm, stream);
  if (rc) return rc;
  const int P = (int)W.pairs;
  QSP_DISPATCH_DTYPE(L->dtype, T, {
    // 2. route
    const size_t rsmem = (size_t)8 * E * sizeof(float);
    rc = launch_pdl("qsp_moe_ffn(route)", moe_route_kernel<T>, dim3((unsigned)((m + 7) / 8)), dim3(256), rsmem, st,
                    (const T*)at(W.r), (int64_t)W.n_in, (int)m, (int)E, (int)k, L->norm_topk_prob ? 1 : 0, (int)Is,
                    (int)W.n_route, (int*)at(W.idx), (float*)at(W.wts), (int*)at(W.rank), counts, (T*)at(W.act_s),
                    (float*)at(W.sig));
    if (rc) return rc;
    // 3. gather
    rc = launch_pdl("qsp_moe_ffn(gather)", moe_gather_kernel<T>, dim3((unsigned)((P + 7) / 8)), dim3(256), 0, st,
                    (const T*)L->xn, (int64_t)L->ld_xn, (int)m, (int)H, (int)E, (int)k, (const int*)at(W.idx),
                    (const float*)at(W.wts), (const int*)at(W.rank), (const int*)counts, (int*)at(W.offsets),
                    (int*)at(W.pos_of), (int*)at(W.tok_of), (float*)at(W.w_of), (int*)at(W.e_of), (T*)at(W.xs),
                    L->expert_counts);
    if (rc) return rc;
    // 4-5. routed experts
    // tensor-core path when every operand can go through TMA (16-byte rows and bases)
    CUtensorMap m_gu, m_xs, m_dn, m_as;
    const bool tc_ok = L->dtype == QSP_BF16 && (H % 8) == 0 && (I % 8) == 0 && aligned(L->gate_up, 16) &&
                       aligned(L->down, 16) && make_map_gate_up(&m_gu, L->gate_up, E, I, H) &&
                       tc::make_map_bf16(&m_xs, at(W.xs), P, H, H, MoeTcCfg<2>::TN) &&
                       tc::make_map_bf16(&m_dn, L->down, E * H, I, I, 256) &&
                       tc::make_map_bf16(&m_as, at(W.as), P, I, I, MoeTcCfg<2>::TN);
    if (tc_ok) {
      MoeTcArgs a{};
      a.offsets = (const int*)at(W.offsets);
      a.E = (int)E;
      a.RB = (int)((I + 127) / 128);
      a.n_kb = (int)((H + 63) / 64);
      a.rows_per_expert = (int)(2 * I);
      a.out_w = (int)I;
      a.out = (__nv_bfloat16*)at(W.as);
      rc = launch_moe_tc<2, true>(m_gu, m_xs, a, st);
      if (rc) return rc;
      a.RB = (int)((H + 255) / 256);   // 256 output rows (two accumulators) per unit
      a.n_kb = (int)((I + 63) / 64);
      a.rows_per_expert = (int)H;
      a.out_w = (int)H;
      a.out = (__nv_bfloat16*)at(W.yw);
      a.w_of = (const float*)at(W.w_of);
      rc = launch_moe_tc<2, false>(m_dn, m_as, a, st);
      if (rc) return rc;
    } else {
      rc = launch_pdl("qsp_moe_ffn(gate|up simt)", moe_gate_up_simt_kernel<T>, dim3((unsigned)P, (unsigned)((I + 7) / 8)),
                      dim3(256), 0, st, (const T*)at(W.xs), (int)H, (const T*)L->gate_up, (int)I,
                      (const int*)at(W.e_of), P, (T*)at(W.as));
      if (rc) return rc;
      rc = launch_pdl("qsp_moe_ffn(down simt)", moe_down_simt_kernel<T>, dim3((unsigned)P, (unsigned)((H + 7) / 8)),
                      dim3(256), 0, st, (const T*)at(W.as), (int)I, (const T*)L->down, (int)H, (const int*)at(W.e_of),
                      (const float*)at(W.w_of), P, (T*)at(W.yw));
      if (rc) return rc;
    }
    // 6. shared expert down projection
    if (Is > 0) {
      rc = qsp_gemm(at(W.act_s), Is, L->shared_down, Is, at(W.s), H, m, H, Is, L->dtype, 0, at(W.gemm),
                    W.total - W.gemm, stream);
      if (rc) return rc;
    }
    // 7. combine + residual + next norm
    rc = launch_pdl("qsp_moe_ffn(combine)", moe_combine_kernel<T>, dim3((unsigned)m), dim3(256), 0, st,
                    (const T*)at(W.yw), (int)H, (int)k, (const int*)at(W.pos_of),
                    Is > 0 ? (const T*)at(W.s) : (const T*)nullptr, (const float*)at(W.sig), (T*)L->x,
                    (int64_t)L->ld_x, (const T*)L->norm_w, (T*)L->y, (int64_t)L->ld_y, L->eps);
  });
  (void)es;
  return rc;
}
