// bf16 split-KV verify attention on tensor cores (warp-level mma.sync m16n8k16).
//
// CTA = (key split s, kv head g, sequence b × row group). A row group is 32 query rows
// (t, q head) = n_rep heads × tokens sharing this kv head, so K/V are read from HBM once per
// (sequence, kv head, split) for all of them (GQA without materialising the expansion).
// Keys stream through a 2-stage cp.async ring of 64-key tiles in padded shared memory (row
// pitch hd+8 elements: ldmatrix without bank conflicts). Warp w computes rows 16·(w&1)..+15
// against keys 32·(w>>1)..+31 of every tile: S = QKᵀ in fp32, online softmax in registers
// (exp2 with the scale folded in), P·V with P taken straight from the S accumulators. The two
// key-half warps of a row tile merge through shared memory at the end and write one
// unnormalised partial (o, m, l) per row; attn_combine_kernel merges the splits and applies
// the output gate.
#include "qsp_common.cuh"

#include <cuda.h>

#include <algorithm>
#include <mutex>

namespace qsp {

constexpr int AM_KT = 64;        // keys per tile
constexpr int AM_ROWS = 32;      // query rows per CTA
constexpr int AM_THREADS = 128;

__device__ __forceinline__ uint32_t su32(const void* p) { return static_cast<uint32_t>(__cvta_generic_to_shared(p)); }

__device__ __forceinline__ void cp16(void* dst, const void* src, bool valid) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(su32(dst)), "l"(src), "r"(valid ? 16 : 0)
               : "memory");
}
__device__ __forceinline__ void cp_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

__device__ __forceinline__ void ldsm_x4(uint32_t (&r)[4], const void* p) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(su32(p)));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t (&r)[4], const void* p) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(su32(p)));
}
__device__ __forceinline__ void mma16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
__device__ __forceinline__ uint32_t pack_bf16(float lo, float hi) {
  __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&v);
}

template <int HD>
struct AmSmem {
  static constexpr int PITCH = HD + 8;  // elements
  static constexpr int TILE = AM_KT * PITCH;
  static constexpr size_t BYTES = (size_t)(AM_ROWS * PITCH + 4 * TILE) * 2;
};

template <int HD>
__global__ void __launch_bounds__(AM_THREADS, 1)
attn_mma_kernel(const qsp_attn_layer L, int n_row_groups) {
  pdl_trigger();
  pdl_wait();
  using SM = AmSmem<HD>;
  constexpr int P = SM::PITCH;
  constexpr int NKS = HD / 16;   // k-steps over head_dim
  constexpr int NNT = HD / 8;    // n-tiles of O
  extern __shared__ __align__(16) __nv_bfloat16 sm[];
  __nv_bfloat16* sQ = sm;
  __nv_bfloat16* sK[2] = {sm + AM_ROWS * P, sm + AM_ROWS * P + SM::TILE};
  __nv_bfloat16* sV[2] = {sm + AM_ROWS * P + 2 * SM::TILE, sm + AM_ROWS * P + 3 * SM::TILE};

  const int s = blockIdx.x, g = blockIdx.y;
  const int b = blockIdx.z / n_row_groups, rgp = blockIdx.z % n_row_groups;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int nrep = L.n_heads / L.n_kv_heads;
  const int rows_total = nrep * L.tokens;
  const int row0 = rgp * AM_ROWS;
  const int nrows = min(AM_ROWS, rows_total - row0);
  const int base_len = L.seq_lens[b];
  const int kv_len = base_len + L.tokens;
  // this split's key range, even across splits and aligned to whole tiles
  int chunk = (kv_len + L.num_splits - 1) / L.num_splits;
  chunk = ((chunk + AM_KT - 1) / AM_KT) * AM_KT;
  const int k_begin = s * chunk;
  const int k_end = min(kv_len, k_begin + chunk);
  const int64_t idx0 = ((int64_t)b * L.n_heads) * L.tokens;

  if (k_begin >= k_end) {  // empty split: an all-masked partial
    for (int r = tid; r < nrows; r += AM_THREADS) {
      const int rr = row0 + r, t = rr / nrep, hq = g * nrep + rr % nrep;
      float* po = L.partial + ((idx0 + (int64_t)hq * L.tokens + t) * L.num_splits + s) * (HD + 2);
      po[HD] = -INFINITY;
      po[HD + 1] = 0.f;
    }
    return;
  }

  const __nv_bfloat16* kp = static_cast<const __nv_bfloat16*>(L.k_pages);
  const __nv_bfloat16* vp = static_cast<const __nv_bfloat16*>(L.v_pages);
  const __nv_bfloat16* qb = static_cast<const __nv_bfloat16*>(L.q_buf);

  // Q rows of this group (rows beyond nrows zero-filled)
  for (int e = tid; e < AM_ROWS * (HD / 8); e += AM_THREADS) {
    const int r = e / (HD / 8), c = e % (HD / 8);
    const int rr = row0 + r;
    const bool ok = r < nrows;
    const int t = ok ? rr / nrep : 0, hq = ok ? g * nrep + rr % nrep : 0;
    const __nv_bfloat16* src = qb + (((int64_t)b * L.tokens + t) * L.n_heads + hq) * HD + c * 8;
    cp16(sQ + r * P + c * 8, ok ? src : qb, ok);
  }
  auto load_tile = [&](int k0, int st) {
    for (int e = tid; e < AM_KT * (HD / 8); e += AM_THREADS) {
      const int j = e / (HD / 8), c = e % (HD / 8);
      const int pos = k0 + j;
      bool ok = pos < k_end;
      int64_t off = 0;
      if (ok) {
        const int lp = pos / L.page_size;
        const int page = lp < L.max_pages ? L.page_table[(int64_t)b * L.max_pages + lp] : -1;
        ok = page >= 0 && page < L.num_pages;
        if (ok) off = (((int64_t)page * L.n_kv_heads + g) * L.page_size + pos % L.page_size) * HD + c * 8;
      }
      cp16(sK[st] + j * P + c * 8, ok ? kp + off : kp, ok);
      cp16(sV[st] + j * P + c * 8, ok ? vp + off : vp, ok);
    }
  };

  const int n_tiles = (k_end - k_begin + AM_KT - 1) / AM_KT;
  load_tile(k_begin, 0);
  cp_commit();

  const int mt = warp & 1, kh = warp >> 1;       // row tile, key half
  const int gq = lane >> 2, tq = lane & 3;
  const float sl2 = L.scale * 1.4426950408889634f;  // scale in log2 units
  // rows of this thread: mt*16 + gq and +8 → absolute query positions
  int qpos[2];
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    const int r = mt * 16 + gq + 8 * h;
    qpos[h] = (r < nrows) ? base_len + (row0 + r) / nrep : -1;
  }
  float o[NNT][4];
#pragma unroll
  for (int i = 0; i < NNT; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;
  float mrow[2] = {-INFINITY, -INFINITY}, lrow[2] = {0.f, 0.f};

  for (int it = 0; it < n_tiles; ++it) {
    const int st = it & 1;
    if (it + 1 < n_tiles) {
      load_tile(k_begin + (it + 1) * AM_KT, st ^ 1);
      cp_commit();
      cp_wait<1>();
    } else {
      cp_wait<0>();
    }
    __syncthreads();
    const int k0 = k_begin + it * AM_KT;
    // S = Q Kᵀ for 16 rows x 32 keys
    float sacc[4][4];
#pragma unroll
    for (int i = 0; i < 4; ++i) sacc[i][0] = sacc[i][1] = sacc[i][2] = sacc[i][3] = 0.f;
#pragma unroll
    for (int ks = 0; ks < NKS; ++ks) {
      uint32_t a[4];
      ldsm_x4(a, sQ + (mt * 16 + (lane & 7) + 8 * ((lane >> 3) & 1)) * P + ks * 16 + 8 * (lane >> 4));
#pragma unroll
      for (int np = 0; np < 2; ++np) {
        uint32_t bb[4];
        const int key = kh * 32 + np * 16 + (lane & 7) + 8 * (lane >> 4);
        ldsm_x4(bb, sK[st] + key * P + ks * 16 + 8 * ((lane >> 3) & 1));
        mma16816(sacc[2 * np], a, bb[0], bb[1]);
        mma16816(sacc[2 * np + 1], a, bb[2], bb[3]);
      }
    }
    // mask (causal over the new tokens, and the split end), scale, online softmax
    float tmax[2] = {-INFINITY, -INFINITY};
#pragma unroll
    for (int nt = 0; nt < 4; ++nt) {
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int h = e >> 1;
        const int key = k0 + kh * 32 + nt * 8 + 2 * tq + (e & 1);
        const bool vis = key < k_end && key <= qpos[h];
        const float v = vis ? sacc[nt][e] * sl2 : -INFINITY;
        sacc[nt][e] = v;
        tmax[h] = fmaxf(tmax[h], v);
      }
    }
    float alpha[2];
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      tmax[h] = fmaxf(tmax[h], __shfl_xor_sync(0xffffffffu, tmax[h], 1));
      tmax[h] = fmaxf(tmax[h], __shfl_xor_sync(0xffffffffu, tmax[h], 2));
      const float mnew = fmaxf(mrow[h], tmax[h]);
      alpha[h] = (mnew == -INFINITY) ? 1.f : exp2f(mrow[h] - mnew);
      mrow[h] = mnew;
    }
    float psum[2] = {0.f, 0.f};
#pragma unroll
    for (int nt = 0; nt < 4; ++nt) {
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int h = e >> 1;
        const float p = (mrow[h] == -INFINITY) ? 0.f : exp2f(sacc[nt][e] - mrow[h]);
        sacc[nt][e] = p;
        psum[h] += p;
      }
    }
#pragma unroll
    for (int h = 0; h < 2; ++h) lrow[h] = lrow[h] * alpha[h] + psum[h];
#pragma unroll
    for (int i = 0; i < NNT; ++i) {
      o[i][0] *= alpha[0];
      o[i][1] *= alpha[0];
      o[i][2] *= alpha[1];
      o[i][3] *= alpha[1];
    }
    // O += P V over this warp's 32 keys (two k-steps of 16)
#pragma unroll
    for (int kk = 0; kk < 2; ++kk) {
      uint32_t pa[4];
      pa[0] = pack_bf16(sacc[2 * kk][0], sacc[2 * kk][1]);
      pa[1] = pack_bf16(sacc[2 * kk][2], sacc[2 * kk][3]);
      pa[2] = pack_bf16(sacc[2 * kk + 1][0], sacc[2 * kk + 1][1]);
      pa[3] = pack_bf16(sacc[2 * kk + 1][2], sacc[2 * kk + 1][3]);
      const int keyr = kh * 32 + kk * 16 + (lane & 7) + 8 * ((lane >> 3) & 1);
#pragma unroll
      for (int dp = 0; dp < NNT / 2; ++dp) {
        uint32_t vb[4];
        ldsm_x4_t(vb, sV[st] + keyr * P + dp * 16 + 8 * (lane >> 4));
        mma16816(o[2 * dp], pa, vb[0], vb[1]);
        mma16816(o[2 * dp + 1], pa, vb[2], vb[3]);
      }
    }
    __syncthreads();  // the stage is refilled next iteration
  }

  // row sums over the 4 threads of a row
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    lrow[h] += __shfl_xor_sync(0xffffffffu, lrow[h], 1);
    lrow[h] += __shfl_xor_sync(0xffffffffu, lrow[h], 2);
  }
  // merge the two key halves of each row tile through shared memory (reusing the K/V ring)
  float* xo = reinterpret_cast<float*>(sK[0]);            // [2 row tiles][16][HD]
  float* xm = xo + 2 * 16 * HD;                           // [2][16] m, then l
  if (kh == 1) {
#pragma unroll
    for (int i = 0; i < NNT; ++i) {
      const int d = i * 8 + 2 * tq;
      float* r0 = xo + ((mt * 16) + gq) * HD + d;
      float* r1 = xo + ((mt * 16) + gq + 8) * HD + d;
      r0[0] = o[i][0]; r0[1] = o[i][1];
      r1[0] = o[i][2]; r1[1] = o[i][3];
    }
    if (tq == 0) {
      xm[mt * 16 + gq] = mrow[0];
      xm[mt * 16 + gq + 8] = mrow[1];
      xm[32 + mt * 16 + gq] = lrow[0];
      xm[32 + mt * 16 + gq + 8] = lrow[1];
    }
  }
  __syncthreads();
  if (kh == 0) {
    float f0[2], f1[2], mm[2], ll[2];
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const int r = mt * 16 + gq + 8 * h;
      const float m2 = xm[r], l2 = xm[32 + r];
      const float M = fmaxf(mrow[h], m2);
      f0[h] = (mrow[h] == -INFINITY) ? 0.f : exp2f(mrow[h] - M);
      f1[h] = (m2 == -INFINITY) ? 0.f : exp2f(m2 - M);
      mm[h] = M;
      ll[h] = lrow[h] * f0[h] + l2 * f1[h];
    }
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const int r = mt * 16 + gq + 8 * h;
      if (r >= nrows) continue;
      const int rr = row0 + r, t = rr / nrep, hq = g * nrep + rr % nrep;
      float* po = L.partial + ((idx0 + (int64_t)hq * L.tokens + t) * L.num_splits + s) * (HD + 2);
      const float* x = xo + r * HD;
#pragma unroll
      for (int i = 0; i < NNT; ++i) {
        const int d = i * 8 + 2 * tq;
        po[d] = o[i][2 * h] * f0[h] + x[d] * f1[h];
        po[d + 1] = o[i][2 * h + 1] * f0[h] + x[d + 1] * f1[h];
      }
      if (tq == 0) {
        po[HD] = mm[h] * 0.6931471805599453f;  // log2 units → natural log (attn_combine_kernel)
        po[HD + 1] = ll[h];
      }
    }
  }
}

int launch_attn_mma(const qsp_attn_layer& L, cudaStream_t st);

int launch_attn_mma(const qsp_attn_layer& L, cudaStream_t st) {
  const int rows_total = (L.n_heads / L.n_kv_heads) * L.tokens;
  const int n_rg = (rows_total + AM_ROWS - 1) / AM_ROWS;
  dim3 grid(L.num_splits, L.n_kv_heads, L.batch * n_rg);
#define QSP_AM_CASE(HDV)                                                                     \
  case HDV: {                                                                                \
    auto kern = attn_mma_kernel<HDV>;                                                        \
    const size_t smem = AmSmem<HDV>::BYTES;                                                  \
    static bool set = false;                                                                 \
    if (!set) {                                                                              \
      if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) \
          != cudaSuccess)                                                                    \
        return set_error(QSP_ERR_CUDA, "qsp_attn_verify: cannot reserve shared memory");     \
      set = true;                                                                            \
    }                                                                                        \
    return launch_pdl("qsp_attn_verify(mma)", kern, grid, dim3(AM_THREADS), smem, st, L, n_rg); \
  }
  switch (L.head_dim) {
    QSP_AM_CASE(64)
    QSP_AM_CASE(128)
    QSP_AM_CASE(256)
    default:
      return QSP_ERR_UNSUPPORTED;
  }
#undef QSP_AM_CASE
}


// ------------------------------------------------------------------ TMA-fed variant
// Same math and work split as attn_mma_kernel, fed differently: key tiles of 32 rows arrive by
// TMA (one 2-D box per 64 head dims of K and of V, 128-byte swizzled) into a 4-stage ring, so
// three tiles are in flight while one is computed and no thread spends time on page-table
// lookups or per-row copies. Q fragments stay in registers for the whole key range; the
// running row maximum is only raised when a tile exceeds it by more than 2^8 (scores are
// exponentiated against the stale maximum otherwise, exactly, since l uses the same one), so
// the O accumulators are rarely rescaled. Requires bf16, page_size a multiple of 32.
constexpr int AT2_KT = 32;     // keys per tile
constexpr int AT2_NST = 4;     // ring stages
constexpr float AT2_SLACK = 8.f;   // log2 units the running max may lag

__device__ int g_attn_error = 0;

template <int HD>
struct At2Smem {
  static constexpr int NB = HD / 64;               // 128-byte boxes per key row
  static constexpr int BOX = AT2_KT * 128;         // bytes per box
  static constexpr int KV = NB * BOX;              // bytes of K (or V) per tile
  static constexpr int STAGE = 2 * KV;
  static constexpr int QP = HD + 8;                // padded Q row (elements)
  static constexpr size_t RING = (size_t)AT2_NST * STAGE;
  static constexpr size_t QBYTES = (size_t)AM_ROWS * QP * 2;
  static constexpr size_t BYTES = 1024 + RING + QBYTES + 128;
};

// Key/value tiles are read once per call: an L2 evict-first policy keeps them from displacing
// the split partials that the merge kernel reads next.
__device__ __forceinline__ void at2_tma(void* dst, const CUtensorMap* map, uint64_t* bar, int x, int y) {
  uint64_t pol;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(pol));
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1, {%3, %4}], [%2], %5;" ::"r"(
          su32(dst)),
      "l"(map), "r"(su32(bar)), "r"(x), "r"(y), "l"(pol)
      : "memory");
}

// The whole head-dim width of a 32-key tile as ONE 3-D box over the view
// [hd/64 column blocks][rows][64 elements] (strides hd·2 B and 128 B): it lands column block
// after column block, each 32 rows × 128 B swizzled — the layout of hd/64 separate 2-D boxes —
// in one TMA request instead of hd/64 (an SM's TMA moves a bounded number of boxes per µs).
__device__ __forceinline__ void at3_tma(void* dst, const CUtensorMap* map, uint64_t* bar, int y) {
  uint64_t pol;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(pol));
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1, {%3, %4, %5}], "
      "[%2], %6;" ::"r"(su32(dst)),
      "l"(map), "r"(su32(bar)), "r"(0), "r"(y), "r"(0), "l"(pol)
      : "memory");
}

__device__ __forceinline__ void at2_wait(uint64_t* bar, uint32_t parity) {
  for (uint32_t i = 0; i < (1u << 24); ++i) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\tselp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok) : "r"(su32(bar)), "r"(parity) : "memory");
    if (ok) return;
    if (i > 256) __nanosleep(64);
  }
  atomicExch(&g_attn_error, 301);
}

// byte offset of (row r, 16-byte chunk c) inside a 128-byte-swizzled box
__device__ __forceinline__ int at2_swz(int r, int c) { return r * 128 + ((c ^ (r & 7)) << 4); }

template <int HD>
__global__ void __launch_bounds__(AM_THREADS, 1)
attn_tma_kernel(const __grid_constant__ CUtensorMap tmK, const __grid_constant__ CUtensorMap tmV,
                const qsp_attn_layer L, int n_row_groups) {
  pdl_trigger();
  pdl_wait();
  using SM = At2Smem<HD>;
  constexpr int QP = SM::QP;
  constexpr int NKS = HD / 16;
  constexpr int NNT = HD / 8;
  extern __shared__ __align__(16) uint8_t at2_raw[];
  uint8_t* ring = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(at2_raw) + 1023) & ~uintptr_t(1023));
  __nv_bfloat16* sQ = reinterpret_cast<__nv_bfloat16*>(ring + SM::RING);
  uint64_t* full = reinterpret_cast<uint64_t*>(ring + SM::RING + SM::QBYTES);
  int* valid = reinterpret_cast<int*>(full + AT2_NST);

  const int s = blockIdx.x, g = blockIdx.y;
  const int b = blockIdx.z / n_row_groups, rgp = blockIdx.z % n_row_groups;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int nrep = L.n_heads / L.n_kv_heads;
  const int rows_total = nrep * L.tokens;
  const int row0 = rgp * AM_ROWS;
  const int nrows = min(AM_ROWS, rows_total - row0);
  const int base_len = L.seq_lens[b];
  const int kv_len = base_len + L.tokens;
  int chunk = (kv_len + L.num_splits - 1) / L.num_splits;
  chunk = ((chunk + AT2_KT - 1) / AT2_KT) * AT2_KT;
  const int k_begin = s * chunk;
  const int k_end = min(kv_len, k_begin + chunk);
  const int64_t idx0 = ((int64_t)b * L.n_heads) * L.tokens;

  if (k_begin >= k_end) {  // empty split: an all-masked partial
    for (int r = tid; r < nrows; r += AM_THREADS) {
      const int rr = row0 + r, t = rr / nrep, hq = g * nrep + rr % nrep;
      float* po = L.partial + ((idx0 + (int64_t)hq * L.tokens + t) * L.num_splits + s) * (HD + 2);
      po[HD] = -INFINITY;
      po[HD + 1] = 0.f;
    }
    return;
  }
  const int n_tiles = (k_end - k_begin + AT2_KT - 1) / AT2_KT;

  if (tid == 0) {
    for (int i = 0; i < AT2_NST; ++i)
      asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(su32(&full[i])) : "memory");
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  // Q rows of this group (rows beyond nrows zero-filled)
  const __nv_bfloat16* qb = static_cast<const __nv_bfloat16*>(L.q_buf);
  for (int e = tid; e < AM_ROWS * (HD / 8); e += AM_THREADS) {
    const int r = e / (HD / 8), c = e % (HD / 8);
    const int rr = row0 + r;
    const bool ok = r < nrows;
    const int t = ok ? rr / nrep : 0, hq = ok ? g * nrep + rr % nrep : 0;
    const __nv_bfloat16* src = qb + (((int64_t)b * L.tokens + t) * L.n_heads + hq) * HD + c * 8;
    cp16(sQ + r * QP + c * 8, ok ? src : qb, ok);
  }
  cp_commit();
  __syncthreads();   // barriers initialised

  // tile j of this split → ring stage j % NST (one thread issues every copy)
  auto issue = [&](int j) {
    const int st = j % AT2_NST;
    const int key0 = k_begin + j * AT2_KT;
    const int lp = key0 / L.page_size;
    const int page = lp < L.max_pages ? L.page_table[(int64_t)b * L.max_pages + lp] : -1;
    const bool ok = page >= 0 && page < L.num_pages;
    const int row = ok ? (page * L.n_kv_heads + g) * L.page_size + key0 % L.page_size : 0;
    valid[st] = ok;
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(su32(&full[st])), "r"(SM::STAGE)
                 : "memory");
    uint8_t* kd = ring + st * SM::STAGE;
#pragma unroll
    for (int nb = 0; nb < SM::NB; ++nb) {
      at2_tma(kd + nb * SM::BOX, &tmK, &full[st], nb * 64, row);
      at2_tma(kd + SM::KV + nb * SM::BOX, &tmV, &full[st], nb * 64, row);
    }
  };
  if (tid == 0)
    for (int j = 0; j < AT2_NST - 1 && j < n_tiles; ++j) issue(j);

  const int mt = warp & 1, kh = warp >> 1;       // row tile, key half (16 keys of a tile)
  const int gq = lane >> 2, tq = lane & 3;
  const float sl2 = L.scale * 1.4426950408889634f;  // scale in log2 units
  int qpos[2];
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    const int r = mt * 16 + gq + 8 * h;
    qpos[h] = (r < nrows) ? base_len + (row0 + r) / nrep : -1;
  }
  cp_wait<0>();
  __syncthreads();   // Q staged
  uint32_t qa[NKS][4];
#pragma unroll
  for (int ks = 0; ks < NKS; ++ks)
    ldsm_x4(qa[ks], sQ + (mt * 16 + (lane & 7) + 8 * ((lane >> 3) & 1)) * QP + ks * 16 + 8 * (lane >> 4));

  float o[NNT][4];
#pragma unroll
  for (int i = 0; i < NNT; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;
  float mrow[2] = {-INFINITY, -INFINITY}, lrow[2] = {0.f, 0.f};
  // this lane's ldmatrix rows inside a tile
  const int kr = kh * 16 + (lane & 7) + 8 * (lane >> 4);          // K (QKᵀ, non-transposed)
  const int kc = (lane >> 3) & 1;
  const int vr = kh * 16 + (lane & 7) + 8 * ((lane >> 3) & 1);    // V (PV, transposed)
  const int vc = lane >> 4;

  for (int it = 0; it < n_tiles; ++it) {
    const int st = it % AT2_NST;
    if (tid == 0 && it + AT2_NST - 1 < n_tiles) issue(it + AT2_NST - 1);   // its stage was freed last iteration
    at2_wait(&full[st], (uint32_t)(it / AT2_NST) & 1u);
    const bool tile_ok = valid[st] != 0;
    const uint8_t* kt = ring + st * SM::STAGE;
    const uint8_t* vt = kt + SM::KV;
    const int k0 = k_begin + it * AT2_KT;
    // S = Q Kᵀ for 16 rows x 16 keys; even and odd k-steps accumulate separately
    float sa[2][4], sb[2][4];
#pragma unroll
    for (int i = 0; i < 2; ++i) sa[i][0] = sa[i][1] = sa[i][2] = sa[i][3] = sb[i][0] = sb[i][1] = sb[i][2] = sb[i][3] = 0.f;
#pragma unroll
    for (int ks = 0; ks < NKS; ++ks) {
      uint32_t bb[4];
      const int d0 = ks * 16 + 8 * kc;
      ldsm_x4(bb, kt + (d0 >> 6) * SM::BOX + at2_swz(kr, (d0 & 63) >> 3));
      if (ks & 1) {
        mma16816(sb[0], qa[ks], bb[0], bb[1]);
        mma16816(sb[1], qa[ks], bb[2], bb[3]);
      } else {
        mma16816(sa[0], qa[ks], bb[0], bb[1]);
        mma16816(sa[1], qa[ks], bb[2], bb[3]);
      }
    }
    // mask (causal over the new tokens, split end, unmapped pages), scale
    float tmax[2] = {-INFINITY, -INFINITY};
#pragma unroll
    for (int nt = 0; nt < 2; ++nt) {
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int h = e >> 1;
        const int key = k0 + kh * 16 + nt * 8 + 2 * tq + (e & 1);
        const bool vis = tile_ok && key < k_end && key <= qpos[h];
        const float v = vis ? (sa[nt][e] + sb[nt][e]) * sl2 : -INFINITY;
        sa[nt][e] = v;
        tmax[h] = fmaxf(tmax[h], v);
      }
    }
    bool need[2];
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      tmax[h] = fmaxf(tmax[h], __shfl_xor_sync(0xffffffffu, tmax[h], 1));
      tmax[h] = fmaxf(tmax[h], __shfl_xor_sync(0xffffffffu, tmax[h], 2));
      need[h] = tmax[h] > mrow[h] + AT2_SLACK;
    }
    if (__any_sync(0xffffffffu, need[0] || need[1])) {
      float alpha[2];
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        alpha[h] = 1.f;
        if (need[h]) {
          alpha[h] = (mrow[h] == -INFINITY) ? 0.f : exp2f(mrow[h] - tmax[h]);
          mrow[h] = tmax[h];
          lrow[h] *= alpha[h];
        }
      }
#pragma unroll
      for (int i = 0; i < NNT; ++i) {
        o[i][0] *= alpha[0];
        o[i][1] *= alpha[0];
        o[i][2] *= alpha[1];
        o[i][3] *= alpha[1];
      }
    }
    float psum[2] = {0.f, 0.f};
#pragma unroll
    for (int nt = 0; nt < 2; ++nt) {
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int h = e >> 1;
        const float p = (mrow[h] == -INFINITY) ? 0.f : exp2f(sa[nt][e] - mrow[h]);
        sa[nt][e] = p;
        psum[h] += p;
      }
    }
    lrow[0] += psum[0];
    lrow[1] += psum[1];
    // O += P V over this warp's 16 keys (one k-step)
    uint32_t pa[4];
    pa[0] = pack_bf16(sa[0][0], sa[0][1]);
    pa[1] = pack_bf16(sa[0][2], sa[0][3]);
    pa[2] = pack_bf16(sa[1][0], sa[1][1]);
    pa[3] = pack_bf16(sa[1][2], sa[1][3]);
#pragma unroll
    for (int dp = 0; dp < NNT / 2; ++dp) {
      uint32_t vb[4];
      const int d0 = dp * 16 + 8 * vc;
      ldsm_x4_t(vb, vt + (d0 >> 6) * SM::BOX + at2_swz(vr, (d0 & 63) >> 3));
      mma16816(o[2 * dp], pa, vb[0], vb[1]);
      mma16816(o[2 * dp + 1], pa, vb[2], vb[3]);
    }
    __syncthreads();  // every warp is done with this stage; it is refilled next iteration
  }

  // row sums over the 4 threads of a row
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    lrow[h] += __shfl_xor_sync(0xffffffffu, lrow[h], 1);
    lrow[h] += __shfl_xor_sync(0xffffffffu, lrow[h], 2);
  }
  // merge the two key halves of each row tile through shared memory (the idle ring)
  float* xo = reinterpret_cast<float*>(ring);             // [2 row tiles][16][HD]
  float* xm = xo + 2 * 16 * HD;                           // [2][16] m, then l
  if (kh == 1) {
#pragma unroll
    for (int i = 0; i < NNT; ++i) {
      const int d = i * 8 + 2 * tq;
      float* r0 = xo + ((mt * 16) + gq) * HD + d;
      float* r1 = xo + ((mt * 16) + gq + 8) * HD + d;
      r0[0] = o[i][0]; r0[1] = o[i][1];
      r1[0] = o[i][2]; r1[1] = o[i][3];
    }
    if (tq == 0) {
      xm[mt * 16 + gq] = mrow[0];
      xm[mt * 16 + gq + 8] = mrow[1];
      xm[32 + mt * 16 + gq] = lrow[0];
      xm[32 + mt * 16 + gq + 8] = lrow[1];
    }
  }
  __syncthreads();
  if (kh == 0) {
    float f0[2], f1[2], mm[2], ll[2];
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const int r = mt * 16 + gq + 8 * h;
      const float m2 = xm[r], l2 = xm[32 + r];
      const float M = fmaxf(mrow[h], m2);
      f0[h] = (mrow[h] == -INFINITY) ? 0.f : exp2f(mrow[h] - M);
      f1[h] = (m2 == -INFINITY) ? 0.f : exp2f(m2 - M);
      mm[h] = M;
      ll[h] = lrow[h] * f0[h] + l2 * f1[h];
    }
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const int r = mt * 16 + gq + 8 * h;
      if (r >= nrows) continue;
      const int rr = row0 + r, t = rr / nrep, hq = g * nrep + rr % nrep;
      float* po = L.partial + ((idx0 + (int64_t)hq * L.tokens + t) * L.num_splits + s) * (HD + 2);
      const float* x = xo + r * HD;
#pragma unroll
      for (int i = 0; i < NNT; ++i) {
        const int d = i * 8 + 2 * tq;
        po[d] = o[i][2 * h] * f0[h] + x[d] * f1[h];
        po[d + 1] = o[i][2 * h + 1] * f0[h] + x[d + 1] * f1[h];
      }
      if (tq == 0) {
        po[HD] = mm[h] * 0.6931471805599453f;  // log2 units → natural log (attn_combine_kernel)
        po[HD + 1] = ll[h];
      }
    }
  }
}

using At2Encode = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                               const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                               CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static At2Encode at2_encode() {
  static At2Encode fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<At2Encode>(p);
  });
  return fn;
}

// Paged K or V of one layer as a 2-D bf16 tensor [num_pages·n_kv·page_size rows, hd], box of
// 32 rows x 64 head dims, 128-byte swizzle.
// [rows, hd] bf16 viewed as [hd/64][rows][64] for at3_tma: box = 64 × AT2_KT rows × hd/64.
static bool at3_map(CUtensorMap* m, const void* base, int64_t rows, int hd) {
  At2Encode enc = at2_encode();
  if (!enc || hd % 64 != 0) return false;
  cuuint64_t dims[3] = {64, (cuuint64_t)rows, (cuuint64_t)(hd / 64)};
  cuuint64_t strides[2] = {(cuuint64_t)hd * 2, 128};
  cuuint32_t box[3] = {64, (cuuint32_t)AT2_KT, (cuuint32_t)(hd / 64)};
  cuuint32_t es[3] = {1, 1, 1};
  return enc(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(base), dims, strides, box, es,
             CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
             CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

static bool at2_map(CUtensorMap* m, const void* base, int64_t rows, int hd) {
  At2Encode enc = at2_encode();
  if (!enc) return false;
  cuuint64_t dims[2] = {(cuuint64_t)hd, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)hd * 2};
  cuuint32_t box[2] = {64, (cuuint32_t)AT2_KT};
  cuuint32_t es[2] = {1, 1};
  return enc(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box, es,
             CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
             CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

int launch_attn_tma(const qsp_attn_layer& L, cudaStream_t st);

// QSP_ERR_UNSUPPORTED when the shape is not one this path handles (the caller falls back).
int launch_attn_tma(const qsp_attn_layer& L, cudaStream_t st) {
  if (L.head_dim != 64 && L.head_dim != 128 && L.head_dim != 256) return QSP_ERR_UNSUPPORTED;
  if (L.page_size % AT2_KT != 0) return QSP_ERR_UNSUPPORTED;
  const int64_t rows = (int64_t)L.num_pages * L.n_kv_heads * L.page_size;
  if (rows >= (1ll << 31) || !aligned(L.k_pages, 16) || !aligned(L.v_pages, 16)) return QSP_ERR_UNSUPPORTED;
  CUtensorMap mk, mv;
  if (!at2_map(&mk, L.k_pages, rows, L.head_dim) || !at2_map(&mv, L.v_pages, rows, L.head_dim))
    return QSP_ERR_UNSUPPORTED;
  const int rows_total = (L.n_heads / L.n_kv_heads) * L.tokens;
  const int n_rg = (rows_total + AM_ROWS - 1) / AM_ROWS;
  dim3 grid(L.num_splits, L.n_kv_heads, L.batch * n_rg);
#define QSP_AT2_CASE(HDV)                                                                    \
  case HDV: {                                                                                \
    auto kern = attn_tma_kernel<HDV>;                                                        \
    const size_t smem = At2Smem<HDV>::BYTES;                                                 \
    static bool set = false;                                                                 \
    if (!set) {                                                                              \
      if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) \
          != cudaSuccess)                                                                    \
        return set_error(QSP_ERR_CUDA, "qsp_attn_verify: cannot reserve shared memory");     \
      set = true;                                                                            \
    }                                                                                        \
    return launch_pdl("qsp_attn_verify(tma)", kern, grid, dim3(AM_THREADS), smem, st, mk, mv, L, n_rg); \
  }
  switch (L.head_dim) {
    QSP_AT2_CASE(64)
    QSP_AT2_CASE(128)
    QSP_AT2_CASE(256)
    default:
      return QSP_ERR_UNSUPPORTED;
  }
#undef QSP_AT2_CASE
}


// ------------------------------------------------------------------ persistent, warp-specialised
// Warp 4 produces: for every work item (split s, kv head g, sequence b x row group) of this CTA
// it brings the item's Q rows (bulk copies) and its key tiles (TMA, as above) into a 4-stage
// ring, running ahead across item boundaries. Warps 0-3 consume as in attn_tma_kernel, and
// each key-half warp writes its own partial (o, m, l), so a split yields two partials that
// the merge kernel combines with the rest. Empty/full barriers per stage; no CTA-wide sync.
// Ring depth measured on B200 (µs per call at the step's lengths / over configs[2]): 2 stages
// 86.6 / 610.7, 3 stages 76.5 / 534.3, 4 stages 73.1 / 507.2, 5 stages 76.2 / 529.6,
// 6 stages 76.2 / 553.6.
constexpr int AT3_NST = 4;
constexpr int AT3_THREADS = 160;

template <int HD>
struct At3Smem {
  static constexpr int NB = HD / 64;
  static constexpr int BOX = AT2_KT * 128;
  static constexpr int KV = NB * BOX;
  static constexpr int STAGE = 2 * KV;
  static constexpr int QB = AM_ROWS * HD * 2;      // unpadded Q rows of one item
  static constexpr size_t RING = (size_t)AT3_NST * STAGE;
  static constexpr size_t BYTES = 1024 + RING + 2 * (size_t)QB + 256;
};

__host__ __device__ __forceinline__ int at3_chunk(const qsp_attn_layer& L) {
  const int cap = L.max_pages * L.page_size;
  const int chunk = (cap + L.num_splits - 1) / L.num_splits;
  return ((chunk + AT2_KT - 1) / AT2_KT) * AT2_KT;
}

struct At3Item {
  int s, g, b, row0, nrows, k_begin, k_end, base_len;
};

__device__ __forceinline__ At3Item at3_item(const qsp_attn_layer& L, int item, int n_rg) {
  At3Item w;
  w.s = item % L.num_splits;
  int rest = item / L.num_splits;
  w.g = rest % L.n_kv_heads;
  rest /= L.n_kv_heads;
  w.b = rest / n_rg;
  const int rgp = rest % n_rg;
  const int nrep = L.n_heads / L.n_kv_heads;
  w.row0 = rgp * AM_ROWS;
  w.nrows = min(AM_ROWS, nrep * L.tokens - w.row0);
  w.base_len = L.seq_lens[w.b];
  const int kv_len = w.base_len + L.tokens;
  // splits of a fixed length (the cache capacity over num_splits, whole 32-key tiles): a
  // sequence uses ceil(kv_len / chunk) of them and the rest of its items are empty, so short
  // sequences of a ragged batch write few partials; the last split takes any keys past the
  // capacity (they have no pages and stay masked)
  const int chunk = at3_chunk(L);
  w.k_begin = w.s * chunk;
  w.k_end = (w.s == L.num_splits - 1) ? kv_len : min(kv_len, w.k_begin + chunk);
  return w;
}

__device__ __forceinline__ void at3_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(su32(bar)) : "memory");
}

template <int HD>
__global__ void __launch_bounds__(AT3_THREADS, 1)
attn_ws_kernel(const __grid_constant__ CUtensorMap tmK, const __grid_constant__ CUtensorMap tmV,
               const qsp_attn_layer L, int n_rg, int n_items) {
  pdl_trigger();
  pdl_wait();
  using SM = At3Smem<HD>;
  constexpr int NKS = HD / 16;
  constexpr int NNT = HD / 8;
  extern __shared__ __align__(16) uint8_t at3_raw[];
  uint8_t* ring = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(at3_raw) + 1023) & ~uintptr_t(1023));
  __nv_bfloat16* sQ = reinterpret_cast<__nv_bfloat16*>(ring + SM::RING);   // [2][32][HD]
  uint64_t* full = reinterpret_cast<uint64_t*>(ring + SM::RING + 2 * SM::QB);
  uint64_t* empty = full + AT3_NST;
  uint64_t* qfull = empty + AT3_NST;
  uint64_t* qempty = qfull + 2;
  int* valid = reinterpret_cast<int*>(qempty + 2);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int nrep = L.n_heads / L.n_kv_heads;
  if (tid == 0) {
    for (int i = 0; i < AT3_NST; ++i) {
      asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(su32(&full[i])) : "memory");
      asm volatile("mbarrier.init.shared::cta.b64 [%0], 4;" ::"r"(su32(&empty[i])) : "memory");
    }
    for (int i = 0; i < 2; ++i) {
      asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(su32(&qfull[i])) : "memory");
      asm volatile("mbarrier.init.shared::cta.b64 [%0], 4;" ::"r"(su32(&qempty[i])) : "memory");
    }
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  __syncthreads();

  if (warp == 4) {
    // ---------------- producer (one lane)
    if (lane != 0) return;
    const __nv_bfloat16* qbuf = static_cast<const __nv_bfloat16*>(L.q_buf);
    uint32_t tc = 0, qc = 0;
    for (int item = blockIdx.x; item < n_items; item += gridDim.x) {
      const At3Item w = at3_item(L, item, n_rg);
      if (w.k_begin >= w.k_end) continue;
      const int qb = qc & 1;
      at2_wait(&qempty[qb], ((qc >> 1) & 1u) ^ 1u);
      asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(su32(&qfull[qb])),
                   "r"((uint32_t)(w.nrows * HD * 2))
                   : "memory");
      __nv_bfloat16* qd = sQ + qb * AM_ROWS * HD;
      for (int r = 0; r < w.nrows;) {   // one bulk copy per token: its run of q heads
        const int rr = w.row0 + r, t = rr / nrep, h0 = rr % nrep;
        const int cnt = min(nrep - h0, w.nrows - r);
        const __nv_bfloat16* src = qbuf + (((int64_t)w.b * L.tokens + t) * L.n_heads + w.g * nrep + h0) * HD;
        asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                         su32(qd + r * HD)),
                     "l"(src), "r"((uint32_t)(cnt * HD * 2)), "r"(su32(&qfull[qb]))
                     : "memory");
        r += cnt;
      }
      ++qc;
      const int n_tiles = (w.k_end - w.k_begin + AT2_KT - 1) / AT2_KT;
      for (int j = 0; j < n_tiles; ++j, ++tc) {
        const int st = tc % AT3_NST;
        at2_wait(&empty[st], ((tc / AT3_NST) & 1u) ^ 1u);
        const int key0 = w.k_begin + j * AT2_KT;
        const int lp = key0 / L.page_size;
        const int page = lp < L.max_pages ? L.page_table[(int64_t)w.b * L.max_pages + lp] : -1;
        const bool ok = page >= 0 && page < L.num_pages;
        const int row = ok ? (page * L.n_kv_heads + w.g) * L.page_size + key0 % L.page_size : 0;
        valid[st] = ok;
        asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(su32(&full[st])), "r"(SM::STAGE)
                     : "memory");
        uint8_t* kd = ring + st * SM::STAGE;
        at3_tma(kd, &tmK, &full[st], row);
        at3_tma(kd + SM::KV, &tmV, &full[st], row);
      }
    }
    return;
  }

  // ---------------- consumers: warps 0-3
  const int mt = warp & 1, kh = warp >> 1;
  const int gq = lane >> 2, tq = lane & 3;
  const float sl2 = L.scale * 1.4426950408889634f;
  const int kr = kh * 16 + (lane & 7) + 8 * (lane >> 4);
  const int kc = (lane >> 3) & 1;
  const int vr = kh * 16 + (lane & 7) + 8 * ((lane >> 3) & 1);
  const int vc = lane >> 4;
  const int NP = 2 * L.num_splits;   // partials per row: two key halves per split
  uint32_t tc = 0, qc = 0;
  for (int item = blockIdx.x; item < n_items; item += gridDim.x) {
    const At3Item w = at3_item(L, item, n_rg);
    const int64_t idx0 = ((int64_t)w.b * L.n_heads) * L.tokens;
    if (w.k_begin >= w.k_end) continue;   // past the sequence's keys: the merge reads no partial of it
    int qpos[2];
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const int r = mt * 16 + gq + 8 * h;
      qpos[h] = (r < w.nrows) ? w.base_len + (w.row0 + r) / nrep : -1;
    }
    const int qb = qc & 1;
    at2_wait(&qfull[qb], (qc >> 1) & 1u);
    uint32_t qa[NKS][4];
    const __nv_bfloat16* qs = sQ + qb * AM_ROWS * HD;
#pragma unroll
    for (int ks = 0; ks < NKS; ++ks)
      ldsm_x4(qa[ks], qs + (mt * 16 + (lane & 7) + 8 * ((lane >> 3) & 1)) * HD + ks * 16 + 8 * (lane >> 4));
    __syncwarp();
    if (lane == 0) at3_arrive(&qempty[qb]);
    ++qc;

    float o[NNT][4];
#pragma unroll
    for (int i = 0; i < NNT; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;
    float mrow[2] = {-INFINITY, -INFINITY}, lrow[2] = {0.f, 0.f};
    const int n_tiles = (w.k_end - w.k_begin + AT2_KT - 1) / AT2_KT;
    for (int it = 0; it < n_tiles; ++it, ++tc) {
      const int st = tc % AT3_NST;
      at2_wait(&full[st], (tc / AT3_NST) & 1u);
      const bool tile_ok = valid[st] != 0;
      const uint8_t* kt = ring + st * SM::STAGE;
      const uint8_t* vt = kt + SM::KV;
      const int k0 = w.k_begin + it * AT2_KT;
      float sa[2][4], sb[2][4];
#pragma unroll
      for (int i = 0; i < 2; ++i) sa[i][0] = sa[i][1] = sa[i][2] = sa[i][3] = sb[i][0] = sb[i][1] = sb[i][2] = sb[i][3] = 0.f;
#pragma unroll
      for (int ks = 0; ks < NKS; ++ks) {
        uint32_t bb[4];
        const int d0 = ks * 16 + 8 * kc;
        ldsm_x4(bb, kt + (d0 >> 6) * SM::BOX + at2_swz(kr, (d0 & 63) >> 3));
        if (ks & 1) {
          mma16816(sb[0], qa[ks], bb[0], bb[1]);
          mma16816(sb[1], qa[ks], bb[2], bb[3]);
        } else {
          mma16816(sa[0], qa[ks], bb[0], bb[1]);
          mma16816(sa[1], qa[ks], bb[2], bb[3]);
        }
      }
      float tmax[2] = {-INFINITY, -INFINITY};
#pragma unroll
      for (int nt = 0; nt < 2; ++nt) {
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int h = e >> 1;
          const int key = k0 + kh * 16 + nt * 8 + 2 * tq + (e & 1);
          const bool vis = tile_ok && key < w.k_end && key <= qpos[h];
          const float v = vis ? (sa[nt][e] + sb[nt][e]) * sl2 : -INFINITY;
          sa[nt][e] = v;
          tmax[h] = fmaxf(tmax[h], v);
        }
      }
      bool need[2];
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        tmax[h] = fmaxf(tmax[h], __shfl_xor_sync(0xffffffffu, tmax[h], 1));
        tmax[h] = fmaxf(tmax[h], __shfl_xor_sync(0xffffffffu, tmax[h], 2));
        need[h] = tmax[h] > mrow[h] + AT2_SLACK;
      }
      if (__any_sync(0xffffffffu, need[0] || need[1])) {
        float alpha[2];
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          alpha[h] = 1.f;
          if (need[h]) {
            alpha[h] = (mrow[h] == -INFINITY) ? 0.f : exp2f(mrow[h] - tmax[h]);
            mrow[h] = tmax[h];
            lrow[h] *= alpha[h];
          }
        }
#pragma unroll
        for (int i = 0; i < NNT; ++i) {
          o[i][0] *= alpha[0];
          o[i][1] *= alpha[0];
          o[i][2] *= alpha[1];
          o[i][3] *= alpha[1];
        }
      }
      float psum[2] = {0.f, 0.f};
#pragma unroll
      for (int nt = 0; nt < 2; ++nt) {
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int h = e >> 1;
          const float p = (mrow[h] == -INFINITY) ? 0.f : exp2f(sa[nt][e] - mrow[h]);
          sa[nt][e] = p;
          psum[h] += p;
        }
      }
      lrow[0] += psum[0];
      lrow[1] += psum[1];
      uint32_t pa[4];
      pa[0] = pack_bf16(sa[0][0], sa[0][1]);
      pa[1] = pack_bf16(sa[0][2], sa[0][3]);
      pa[2] = pack_bf16(sa[1][0], sa[1][1]);
      pa[3] = pack_bf16(sa[1][2], sa[1][3]);
#pragma unroll
      for (int dp = 0; dp < NNT / 2; ++dp) {
        uint32_t vb[4];
        const int d0 = dp * 16 + 8 * vc;
        ldsm_x4_t(vb, vt + (d0 >> 6) * SM::BOX + at2_swz(vr, (d0 & 63) >> 3));
        mma16816(o[2 * dp], pa, vb[0], vb[1]);
        mma16816(o[2 * dp + 1], pa, vb[2], vb[3]);
      }
      __syncwarp();
      if (lane == 0) at3_arrive(&empty[st]);
    }
    // this warp's partial: rows of its row tile over its key half
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      lrow[h] += __shfl_xor_sync(0xffffffffu, lrow[h], 1);
      lrow[h] += __shfl_xor_sync(0xffffffffu, lrow[h], 2);
    }
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const int r = mt * 16 + gq + 8 * h;
      if (r >= w.nrows) continue;
      const int rr = w.row0 + r, t = rr / nrep, hq = w.g * nrep + rr % nrep;
      float* po = L.partial + ((idx0 + (int64_t)hq * L.tokens + t) * NP + 2 * w.s + kh) * (HD + 2);
#pragma unroll
      for (int i = 0; i < NNT; ++i) {
        const int d = i * 8 + 2 * tq;
        *reinterpret_cast<float2*>(po + d) = make_float2(o[i][2 * h], o[i][2 * h + 1]);
      }
      if (tq == 0) {
        po[HD] = mrow[h] == -INFINITY ? -INFINITY : mrow[h] * 0.6931471805599453f;
        po[HD + 1] = lrow[h];
      }
    }
  }
}

int launch_attn_ws(const qsp_attn_layer& L, cudaStream_t st);

int attn_ws_chunk(const qsp_attn_layer& L) { return at3_chunk(L); }

int launch_attn_ws(const qsp_attn_layer& L, cudaStream_t st) {
  if (L.head_dim != 64 && L.head_dim != 128 && L.head_dim != 256) return QSP_ERR_UNSUPPORTED;
  if (L.page_size % AT2_KT != 0) return QSP_ERR_UNSUPPORTED;
  const int64_t rows = (int64_t)L.num_pages * L.n_kv_heads * L.page_size;
  if (rows >= (1ll << 31) || !aligned(L.k_pages, 16) || !aligned(L.v_pages, 16) || !aligned(L.q_buf, 16))
    return QSP_ERR_UNSUPPORTED;
  CUtensorMap mk, mv;
  if (!at3_map(&mk, L.k_pages, rows, L.head_dim) || !at3_map(&mv, L.v_pages, rows, L.head_dim))
    return QSP_ERR_UNSUPPORTED;
  const int rows_total = (L.n_heads / L.n_kv_heads) * L.tokens;
  const int n_rg = (rows_total + AM_ROWS - 1) / AM_ROWS;
  const int64_t n_items64 = (int64_t)L.num_splits * L.n_kv_heads * L.batch * n_rg;
  if (n_items64 >= (1ll << 31)) return QSP_ERR_UNSUPPORTED;
  const int n_items = (int)n_items64;
  static int sms = 0;
  if (sms == 0) {
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    if (sms <= 0) sms = 148;
  }
  const int grid = std::min(n_items, sms);
#define QSP_AT3_CASE(HDV)                                                                    \
  case HDV: {                                                                                \
    auto kern = attn_ws_kernel<HDV>;                                                         \
    const size_t smem = At3Smem<HDV>::BYTES;                                                 \
    static bool set = false;                                                                 \
    if (!set) {                                                                              \
      if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) \
          != cudaSuccess)                                                                    \
        return set_error(QSP_ERR_CUDA, "qsp_attn_verify: cannot reserve shared memory");     \
      set = true;                                                                            \
    }                                                                                        \
    return launch_pdl("qsp_attn_verify(ws)", kern, grid, dim3(AT3_THREADS), smem, st, mk, mv, L, n_rg, n_items); \
  }
  switch (L.head_dim) {
    QSP_AT3_CASE(64)
    QSP_AT3_CASE(128)
    QSP_AT3_CASE(256)
    default:
      return QSP_ERR_UNSUPPORTED;
  }
#undef QSP_AT3_CASE
}

int attn_device_error(int reset) {
  int v = 0;
  cudaMemcpyFromSymbol(&v, g_attn_error, sizeof(int));
  if (reset && v) {
    const int z = 0;
    cudaMemcpyToSymbol(g_attn_error, &z, sizeof(int));
  }
  return v;
}

}  // namespace qsp
