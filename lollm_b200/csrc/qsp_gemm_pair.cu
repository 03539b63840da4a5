// Pair GEMM for the verify step's projections (128 < m ≤ 256 token rows):
// c[m, n] = a[m, k] · w[n, k]ᵀ, bf16 in, fp32 accumulate.
//
// A CTA pair (a cluster of two CTAs, tcgen05 cta_group::2) owns one tile of N weight rows x
// all 256 token rows over the whole K range. CTA r stages token rows [128r, 128r + 128) of the
// activations and weight rows [N/2·r, N/2·r + N/2) of the tile; the pair's rank 0 issues
// 256 x N x 16 MMAs that read both CTAs' halves, and each CTA's TMEM accumulates its 128 token
// rows x N columns. N (a multiple of 16, at most 256) is chosen so that the tiles fill the SMs
// in one wave, so there are no split-K partials and no merge pass: every weight byte is
// brought into shared memory once, the activations are re-read from L2 once per tile.
// Epilogues (each epilogue thread owns one token row of its CTA's accumulator):
//   STORE    c = round(acc)
//   SWIGLU   the tile is N/2 gate rows + the matching N/2 up rows of a [gate; up] weight;
//            act = round(round(silu(round(g))) · round(u))
//   RESNORM  x = round(x + round(acc)) in place, plus the tile's Σ x² per token row into a
//            small buffer; pair_rmsnorm_kernel then writes y = round(x·rsqrt(Σ/n + eps)·(1 + w))
// Waits are bounded (an expired wait records a code in g_gemm_pair_error and the CTA exits);
// before exiting, each CTA waits until every MMA-completion arrival aimed at its barriers has
// landed, and the pair meets at a cluster barrier, so no CTA leaves while its partner can still
// signal it or read its shared memory.
#include <algorithm>

#include "qsp_common.cuh"
#include "qsp_tc.cuh"

namespace qsp {

__device__ int g_gemm_pair_error = 0;

int gemm_pair_device_error(int reset) {
  int v = 0;
  if (cudaMemcpyFromSymbol(&v, g_gemm_pair_error, sizeof(int)) != cudaSuccess) return 0;
  if (reset && v) {
    const int zero = 0;
    cudaMemcpyToSymbol(g_gemm_pair_error, &zero, sizeof(int));
  }
  return v;
}

enum { PAIR_STORE = 0, PAIR_SWIGLU = 1, PAIR_RESNORM = 2 };
constexpr int PAIR_X_BYTES = 128 * 64 * 2;             // 128 token rows x 64 K (bf16)
constexpr int PAIR_SMEM_MAX = 232448;                   // 227 KB opt-in per CTA
constexpr int PAIR_AUX = 1024 + 512;                    // alignment slack + barriers
constexpr int PAIR_MAX_STAGES = 16;

// 3-D TMA load (k-blocks kb, kb+1 of rows [y, y + box rows) over the view [k-blocks][rows][64])
// into this CTA's shared memory, completing on the pair leader's barrier; weights evict-first.
__device__ __forceinline__ void tma_load_3d_pair_warp(void* dst, const CUtensorMap* map, uint32_t bar_cluster, int y,
                                                      int kb, bool evict_first) {
  if (evict_first) {
    asm volatile(
        "{\n\t.reg .pred e;\n\t.reg .b64 pol;\n\telect.sync _|e, 0xffffffff;\n\t"
        "createpolicy.fractional.L2::evict_first.b64 pol, 1.0;\n\t"
        "@e cp.async.bulk.tensor.3d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint "
        "[%0], [%1, {%3, %4, %5}], [%2], pol;\n\t}" ::"r"(tc::smem_u32(dst)),
        "l"(map), "r"(bar_cluster), "r"(0), "r"(y), "r"(kb)
        : "memory");
  } else {
    asm volatile(
        "{\n\t.reg .pred e;\n\telect.sync _|e, 0xffffffff;\n\t"
        "@e cp.async.bulk.tensor.3d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, "
        "%4, %5}], [%2];\n\t}" ::"r"(tc::smem_u32(dst)),
        "l"(map), "r"(bar_cluster), "r"(0), "r"(y), "r"(kb)
        : "memory");
  }
}

// bf16 row-major [rows, cols] viewed as [cols/64 k-blocks][rows][64 elements] (cols a multiple
// of 64): a box of kps k-blocks × box_rows rows lands k-block after k-block in shared memory,
// each as 128B-swizzled K-major rows.
static bool make_map3_bf16(CUtensorMap* m, const void* base, int64_t rows, int64_t cols, int64_t ld, int box_rows,
                           int kps) {
  tc::EncodeTiled enc = tc::get_encode();
  if (!enc || cols % 64 != 0) return false;
  cuuint64_t dims[3] = {64, (cuuint64_t)rows, (cuuint64_t)(cols / 64)};
  cuuint64_t strides[2] = {(cuuint64_t)(ld * 2), 128};
  cuuint32_t box[3] = {64, (cuuint32_t)box_rows, (cuuint32_t)kps};
  cuuint32_t es[3] = {1, 1, 1};
  return enc(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(base), dims, strides, box, es,
             CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
             CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

struct PairArgs {
  __nv_bfloat16* c;   // STORE: product; SWIGLU: activation; RESNORM: residual stream x
  int64_t ldc;
  float* sumsq;       // RESNORM: [tiles][m] Σ x² of each tile's columns
  int m, n;           // token rows; output columns (STORE/RESNORM: n; SWIGLU: inter)
  int N;              // weight rows per tile (MMA N)
  int n_kb, stages, w_bytes, tmem_cols;
  int up_off;         // SWIGLU: first up row of the [gate; up] weight (= inter)
};

template <int MODE, int KP>
__global__ void __launch_bounds__(192, 1)
gemm_pair_kernel(const __grid_constant__ CUtensorMap tm_w, const __grid_constant__ CUtensorMap tm_x,
                 const __grid_constant__ CUtensorMap tm_c, const PairArgs A) {
  using namespace tc;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int S = A.stages;
  // a stage holds KP k-blocks: [k-block][128 token rows][128 B], then [k-block][N/2 rows][128 B]
  // (KP = 2: each operand one 3-D TMA box)
  const uint32_t x_bytes = KP * PAIR_X_BYTES;
  const uint32_t stage_bytes = x_bytes + KP * A.w_bytes;
  const int steps = A.n_kb / KP;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + (size_t)S * stage_bytes);   // used in rank 0
  uint64_t* empty = full + S;
  uint64_t* acc_full = empty + S;
  uint32_t* tslot = reinterpret_cast<uint32_t*>(acc_full + 1);
  volatile int* abort = reinterpret_cast<volatile int*>(tslot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();
  const int tile = blockIdx.x >> 1;
  const int half = A.N >> 1;
  const int wrow = MODE == PAIR_SWIGLU ? (rank == 0 ? tile * half : A.up_off + tile * half)
                                       : tile * A.N + (int)rank * half;
  const int trow = (int)rank * 128;
  pdl_trigger();

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(acc_full, 1);
    *abort = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 1) tmem_alloc_pair(tslot, (uint32_t)A.tmem_cols);
  fence_before();
  cluster_sync_all();   // both CTAs' barriers are initialised before any cross-CTA arrival
  fence_after();
  const uint32_t tmem = *tslot;

  if (warp == 0) {
    // producer: the whole warp runs the loop, one elected lane issues (see qsp_tc.cuh)
    if (lane == 0) {
      asm volatile("prefetch.tensormap [%0];" ::"l"(&tm_w) : "memory");
      asm volatile("prefetch.tensormap [%0];" ::"l"(&tm_x) : "memory");
    }
    __syncwarp();
    // both CTAs' bytes of a stage complete on rank 0's full barrier, which rank 0 arms for both
    auto load_w = [&](uint8_t* st, uint32_t fb, int i) {
      if (KP == 1) tma_load_2d_pair_evict_first_warp(st + x_bytes, &tm_w, fb, i * 64, wrow);
      else tma_load_3d_pair_warp(st + x_bytes, &tm_w, fb, wrow, i * KP, true);
    };
    auto load_x = [&](uint8_t* st, uint32_t fb, int i) {
      if (KP == 1) tma_load_2d_pair_warp(st, &tm_x, fb, i * 64, trow);
      else tma_load_3d_pair_warp(st, &tm_x, fb, trow, i * KP, false);
    };
    const int npre = min(steps, S);
    for (int i = 0; i < npre; ++i) {
      const uint32_t fb = cluster_addr(smem_u32(&full[i]), 0);
      if (rank == 0) mbar_expect_tx_warp(&full[i], 2 * stage_bytes);
      load_w(smem + i * stage_bytes, fb, i);
    }
    pdl_wait();   // activations are the previous kernel's output
    for (int i = 0; i < npre; ++i) load_x(smem + i * stage_bytes, cluster_addr(smem_u32(&full[i]), 0), i);
    bool ok = true;
    for (int i = npre; i < steps; ++i) {
      const int s = i % S;
      const uint32_t ph = (i / S) & 1u;
      ok = mbar_wait_warp(&empty[s], ph ^ 1u, 601, &g_gemm_pair_error, abort);
      if (!ok) break;
      const uint32_t fb = cluster_addr(smem_u32(&full[s]), 0);
      uint8_t* st = smem + s * stage_bytes;
      if (rank == 0) mbar_expect_tx_warp(&full[s], 2 * stage_bytes);
      load_w(st, fb, i);
      load_x(st, fb, i);
    }
    // the last release of every stage (an MMA-completion arrival from rank 0) has landed
    for (int s = 0; ok && s < npre; ++s) {
      const int last = (steps - 1 - s) / S;
      ok = mbar_wait_warp(&empty[s], (uint32_t)last & 1u, 602, &g_gemm_pair_error, abort);
    }
  } else if (warp == 1) {
    pdl_wait();
    if (rank == 0) {   // MMA issuer: the whole warp, one elected lane issues
      const uint32_t idesc = idesc_bf16(256, A.N);
      bool ok = true;
      for (int i = 0; i < steps; ++i) {
        const int s = i % S;
        const uint32_t ph = (i / S) & 1u;
        if (ok) ok = mbar_wait_warp(&full[s], ph, 603, &g_gemm_pair_error, abort);
        fence_after();
        if (ok) {
          const uint32_t xa = smem_u32(smem + s * stage_bytes);
#pragma unroll
          for (int kk = 0; kk < KP; ++kk)
            umma4_bf16_pair_warp(tmem, sdesc_sw128(xa + kk * PAIR_X_BYTES), sdesc_sw128(xa + x_bytes + kk * A.w_bytes),
                                 idesc, (i > 0 || kk > 0) ? 1u : 0u);
        }
        umma_commit_pair_warp(&empty[s]);
      }
      umma_commit_pair_warp(acc_full);
    }
  } else {
    // ------------------------------------------------------------------ epilogue
    pdl_wait();
    const int quad = warp & 3;
    const bool ok = mbar_wait(acc_full, 0, 604, &g_gemm_pair_error, abort);
    fence_after();
    const int t = trow + quad * 32 + lane;
    const bool live = ok && t < A.m;
    const uint32_t tbase = tmem + ((uint32_t)(quad * 32) << 16);
    // STORE / SWIGLU: each warp stages its 32 token rows x (N or N/2) bf16 outputs densely in
    // the idle ring and writes them with one TMA store (rows >= m and columns >= n are clipped)
    __nv_bfloat16* stg = reinterpret_cast<__nv_bfloat16*>(smem) + (size_t)quad * 32 * A.N;
    if (MODE == PAIR_SWIGLU) {
      for (int c0 = 0; c0 < half; c0 += 8) {
        float g[8], u[8];
        tmem_ld8(tbase + c0, g);
        tmem_ld8(tbase + half + c0, u);
        uint4 ov;
        __nv_bfloat16* oh = reinterpret_cast<__nv_bfloat16*>(&ov);
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          const float sg = dt<__nv_bfloat16>::round(siluf_(dt<__nv_bfloat16>::round(g[e])));
          oh[e] = __float2bfloat16_rn(sg * dt<__nv_bfloat16>::round(u[e]));
        }
        *reinterpret_cast<uint4*>(stg + lane * half + c0) = ov;
      }
      fence_proxy_async_smem();
      __syncwarp();
      if (ok && lane == 0) {
        tma_store_2d(&tm_c, stg, tile * half, trow + quad * 32);
        tma_store_commit_wait();
      }
      __syncwarp();
    } else {
      // STORE: c = round(acc). RESNORM: x = round(x + round(acc)) (x read by each thread from
      // its own token row), plus the tile's Σ x² of the row into sumsq[tile][row]
      const int n0 = tile * A.N;
      const __nv_bfloat16* xrow = A.c + (int64_t)t * A.ldc;
      float ss = 0.f;
      for (int c0 = 0; c0 < A.N; c0 += 16) {
        float v[16];
        tmem_ld16(tbase + c0, v);
        uint4 ov[2];
        __nv_bfloat16* oh = reinterpret_cast<__nv_bfloat16*>(ov);
        if (MODE == PAIR_RESNORM) {
          const int col = n0 + c0;
          uint4 xv[2] = {make_uint4(0, 0, 0, 0), make_uint4(0, 0, 0, 0)};
          if (live && col < A.n) {   // n is a multiple of 16: whole chunks only
            xv[0] = *reinterpret_cast<const uint4*>(xrow + col);
            xv[1] = *reinterpret_cast<const uint4*>(xrow + col + 8);
          }
          const __nv_bfloat16* xh = reinterpret_cast<const __nv_bfloat16*>(xv);
#pragma unroll
          for (int e = 0; e < 16; ++e) {
            const float r = dt<__nv_bfloat16>::round(dt<__nv_bfloat16>::round(v[e]) + __bfloat162float(xh[e]));
            oh[e] = __float2bfloat16_rn(r);
            ss = fmaf(r, r, ss);
          }
        } else {
#pragma unroll
          for (int e = 0; e < 16; ++e) oh[e] = __float2bfloat16_rn(v[e]);
        }
        uint4* dst = reinterpret_cast<uint4*>(stg + lane * A.N + c0);
        dst[0] = ov[0];
        dst[1] = ov[1];
      }
      fence_proxy_async_smem();
      __syncwarp();
      if (ok && lane == 0) {
        tma_store_2d(&tm_c, stg, n0, trow + quad * 32);
        tma_store_commit_wait();
      }
      __syncwarp();
      // columns past n hold zeros (x and the weights read as zeros there), so ss is exact
      if (MODE == PAIR_RESNORM && live) A.sumsq[(int64_t)tile * A.m + t] = ss;
    }
  }
  fence_before();
  __syncthreads();
  cluster_sync_all();   // the partner is done with this CTA's shared memory and TMEM
  if (warp == 1) {
    fence_after();
    tmem_dealloc_pair(tmem, (uint32_t)A.tmem_cols);
  }
}

// y[r, :] = round(x[r, :]·rsqrt(Σ_tiles sumsq[tile][r] / n + eps)·(1 + w)), one CTA per row;
// the per-tile sums are added in tile order.
__global__ void __launch_bounds__(256) pair_rmsnorm_kernel(const __nv_bfloat16* __restrict__ x, int64_t ldx,
                                                           const float* __restrict__ sumsq, int tiles, int m,
                                                           const __nv_bfloat16* __restrict__ w,
                                                           __nv_bfloat16* __restrict__ y, int64_t ldy, int n,
                                                           float eps) {
  pdl_trigger();
  pdl_wait();
  const int row = blockIdx.x;
  float ss = 0.f;
  for (int tl = 0; tl < tiles; ++tl) ss += sumsq[(int64_t)tl * m + row];
  const float inv = rsqrtf(ss / (float)n + eps);
  const __nv_bfloat16* xr = x + (int64_t)row * ldx;
  __nv_bfloat16* yr = y + (int64_t)row * ldy;
  for (int col = threadIdx.x * 8; col < n; col += blockDim.x * 8) {
    const uint4 xv = *reinterpret_cast<const uint4*>(xr + col);
    const uint4 wv = *reinterpret_cast<const uint4*>(w + col);
    const __nv_bfloat16* xh = reinterpret_cast<const __nv_bfloat16*>(&xv);
    const __nv_bfloat16* wh = reinterpret_cast<const __nv_bfloat16*>(&wv);
    uint4 ov;
    __nv_bfloat16* oh = reinterpret_cast<__nv_bfloat16*>(&ov);
#pragma unroll
    for (int e = 0; e < 8; ++e) oh[e] = __float2bfloat16_rn(__bfloat162float(xh[e]) * inv * (__bfloat162float(wh[e]) + 1.0f));
    *reinterpret_cast<uint4*>(yr + col) = ov;
  }
}

// ------------------------------------------------------------------ host side
struct PairPlan {
  int N, tiles, stages, w_bytes, tmem_cols, n_kb, kp;
};

static int ceil_div(int64_t a, int64_t b) { return (int)((a + b - 1) / b); }

// Pairs that can be resident at once (one CTA per SM at this shared-memory size); at most
// half the SMs.
static int resident_pairs() {
  static int n = 0;
  if (n != 0) return n;
  auto kern = gemm_pair_kernel<PAIR_STORE, 1>;   // every mode has the same resources
  n = tc::sm_count() / 2;
  if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, PAIR_SMEM_MAX) != cudaSuccess) {
    (void)cudaGetLastError();
    return n;
  }
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(2 * n);
  cfg.blockDim = dim3(192);
  cfg.dynamicSmemBytes = PAIR_SMEM_MAX;
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeClusterDimension;
  at[0].val.clusterDim.x = 2;
  at[0].val.clusterDim.y = 1;
  at[0].val.clusterDim.z = 1;
  cfg.attrs = at;
  cfg.numAttrs = 1;
  int c = 0;
  if (cudaOccupancyMaxActiveClusters(&c, kern, &cfg) != cudaSuccess) {
    (void)cudaGetLastError();
    c = 0;
  }
  if (c > 0 && c < n) n = c;
  return n;
}

// Tile width: the smallest multiple of 16 (SWIGLU: of 8 per half) that covers the output in
// at most one pair per two SMs.
static bool pair_plan(int64_t m, int64_t n_out, int64_t k, int mode, PairPlan* p) {
  if (m <= 128 || m > 256) return false;
  const int pairs = resident_pairs();
  int N, tiles;
  if (mode == PAIR_SWIGLU) {
    const int half = 8 * ceil_div(ceil_div(n_out, pairs), 8);
    if (half > 128) return false;
    N = 2 * half;
    tiles = ceil_div(n_out, half);
  } else {
    N = 16 * ceil_div(ceil_div(n_out, pairs), 16);
    if (N > 256) return false;
    if (N < 32) N = 32;
    tiles = ceil_div(n_out, N);
  }
  p->N = N;
  p->tiles = tiles;
  p->w_bytes = (N / 2) * 128;
  // two k-blocks per stage (one 3-D box per operand) when K allows and three stages still fit
  p->n_kb = ceil_div(k, 64);
  p->kp = (k % 128 == 0 && (PAIR_SMEM_MAX - PAIR_AUX) / (2 * (PAIR_X_BYTES + p->w_bytes)) >= 3) ? 2 : 1;
  const int stage = p->kp * (PAIR_X_BYTES + p->w_bytes);
  p->stages = std::min(PAIR_MAX_STAGES, (PAIR_SMEM_MAX - PAIR_AUX) / stage);
  int cols = 32;
  while (cols < N) cols *= 2;
  p->tmem_cols = cols;
  return true;
}

size_t gemm_pair_workspace(int64_t m, int64_t n, int64_t k) {
  PairPlan p{};
  if (!pair_plan(m, n, k, PAIR_RESNORM, &p)) return 0;
  return (size_t)p.tiles * (size_t)m * sizeof(float);
}

template <int MODE, int KP>
static int launch_pair(const CUtensorMap& mw, const CUtensorMap& mx, const CUtensorMap& mc, const PairPlan& p,
                       const PairArgs& args,
                       cudaStream_t st) {
  auto kern = gemm_pair_kernel<MODE, KP>;
  const size_t smem = (size_t)p.stages * KP * (PAIR_X_BYTES + p.w_bytes) + PAIR_AUX;
  static bool attr_set = false;
  if (!attr_set) {
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, PAIR_SMEM_MAX) != cudaSuccess)
      return set_error(QSP_ERR_CUDA, "qsp_gemm(pair): cannot reserve %d bytes of shared memory", PAIR_SMEM_MAX);
    attr_set = true;
  }
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(2 * p.tiles);
  cfg.blockDim = dim3(192);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute at[2];
  at[0].id = cudaLaunchAttributeClusterDimension;
  at[0].val.clusterDim.x = 2;
  at[0].val.clusterDim.y = 1;
  at[0].val.clusterDim.z = 1;
  at[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  at[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = at;
  cfg.numAttrs = 2;
  const cudaError_t e = cudaLaunchKernelEx(&cfg, kern, mw, mx, mc, args);
  if (e != cudaSuccess) {
    (void)cudaGetLastError();
    return set_error(QSP_ERR_CUDA, "qsp_gemm(pair): %s", cudaGetErrorString(e));
  }
  return check_launch("qsp_gemm(pair)");
}

// mode PAIR_STORE: c = a·wᵀ over n columns. PAIR_SWIGLU: c is the activation [m, inter] of a
// [gate; up] weight with 2·n rows (n = inter). PAIR_RESNORM: c is the residual stream x
// (+= the product), then y = RMSNorm(x)·(1 + norm_w); needs `workspace` for the row sums.
// Returns QSP_ERR_UNSUPPORTED when the shape or alignment does not fit this kernel.
int gemm_pair(const void* a, int64_t lda, const void* w, int64_t ldw, void* c, int64_t ldc, int64_t m, int64_t n,
              int64_t k, int mode, const void* norm_w, void* y, int64_t ldy, float eps, void* workspace,
              size_t ws_bytes, cudaStream_t st) {
  if (!aligned(a, 16) || !aligned(w, 16) || !aligned(c, 16) || (lda * 2) % 16 != 0 || (ldw * 2) % 16 != 0 ||
      (ldc * 2) % 16 != 0 || k % 8 != 0 || n % 8 != 0)
    return QSP_ERR_UNSUPPORTED;
  PairPlan p{};
  if (!pair_plan(m, n, k, mode, &p)) return QSP_ERR_UNSUPPORTED;
  if (mode == PAIR_RESNORM) {
    if (n % 16 != 0 || !aligned(y, 16) || !aligned(norm_w, 16) || (ldy * 2) % 16 != 0 || workspace == nullptr ||
        !aligned(workspace, 16) || ws_bytes < (size_t)p.tiles * (size_t)m * sizeof(float))
      return QSP_ERR_UNSUPPORTED;
  }
  const int64_t w_rows = mode == PAIR_SWIGLU ? 2 * n : n;
  CUtensorMap mw, mx, mc;
  const bool maps = p.kp == 2 ? make_map3_bf16(&mw, w, w_rows, k, ldw, p.N / 2, 2) && make_map3_bf16(&mx, a, m, k, lda, 128, 2)
                              : tc::make_map_bf16(&mw, w, w_rows, k, ldw, p.N / 2) && tc::make_map_bf16(&mx, a, m, k, lda, 128);
  if (!maps || !tc::make_store_map_bf16(&mc, c, m, n, ldc, 32, mode == PAIR_SWIGLU ? p.N / 2 : p.N))
    return QSP_ERR_UNSUPPORTED;
  PairArgs args{};
  args.c = static_cast<__nv_bfloat16*>(c);
  args.ldc = ldc;
  args.sumsq = static_cast<float*>(workspace);
  args.m = (int)m;
  args.n = (int)n;
  args.N = p.N;
  args.n_kb = p.n_kb;
  args.stages = p.stages;
  args.w_bytes = p.w_bytes;
  args.tmem_cols = p.tmem_cols;
  args.up_off = (int)n;
  int rc;
  if (p.kp == 2) {
    if (mode == PAIR_SWIGLU) rc = launch_pair<PAIR_SWIGLU, 2>(mw, mx, mc, p, args, st);
    else if (mode == PAIR_RESNORM) rc = launch_pair<PAIR_RESNORM, 2>(mw, mx, mc, p, args, st);
    else rc = launch_pair<PAIR_STORE, 2>(mw, mx, mc, p, args, st);
  } else {
    if (mode == PAIR_SWIGLU) rc = launch_pair<PAIR_SWIGLU, 1>(mw, mx, mc, p, args, st);
    else if (mode == PAIR_RESNORM) rc = launch_pair<PAIR_RESNORM, 1>(mw, mx, mc, p, args, st);
    else rc = launch_pair<PAIR_STORE, 1>(mw, mx, mc, p, args, st);
  }
  if (rc || mode != PAIR_RESNORM) return rc;
  return launch_pdl("qsp_gemm(pair rmsnorm)", pair_rmsnorm_kernel, dim3((unsigned)m), dim3(256), 0, st,
                    static_cast<const __nv_bfloat16*>(c), ldc, static_cast<const float*>(workspace), p.tiles, (int)m,
                    static_cast<const __nv_bfloat16*>(norm_w), static_cast<__nv_bfloat16*>(y), ldy, (int)n, eps);
}


// ------------------------------------------------------------------ persistent pair (STORE)
// For plain products whose tiles take several rounds of the pairs (the vocabulary projection
// over the verify rows): pair p computes tiles p, p + P, p + 2P, ... of N weight rows × all
// 256 token rows, whole K each. Both CTAs stream their halves through one continuous ring
// across tiles; rank 0 issues the MMAs into one of two TMEM accumulator buffers (N ≤ 256
// columns each), so a tile's epilogue overlaps the next tile's MMAs. Each epilogue thread owns
// one token row of its CTA's accumulator and writes its bf16 outputs with 16-byte stores, then
// its warp releases the buffer on rank 0's barrier (8 arrivals: 4 warps in each CTA).
// Per SM and k-block the ring takes 16 KB of activations and N/2·128 B of weights, against
// 32 KB + 16 KB for a 128-row unit of the persistent single-CTA kernel. A ring stage holds
// two k-blocks, each operand loaded as one 3-D TMA box: an SM's TMA moves a bounded number of
// boxes per microsecond, and 16 KB boxes would cap its ingest near 55 GB/s.
struct PairPArgs {
  __nv_bfloat16* c;
  int64_t ldc;
  int m, n;           // token rows, output columns
  int N;              // weight rows per tile (MMA N, a multiple of 16, ≤ 256)
  int tiles, n_kb, stages, w_bytes;   // n_kb: k-blocks (even); w_bytes: weights of one k-block
};
constexpr int PAIRP_KPS = 2;         // k-blocks per ring stage

__global__ void __launch_bounds__(192, 1)
gemm_pairp_kernel(const __grid_constant__ CUtensorMap tm_w, const __grid_constant__ CUtensorMap tm_x,
                  const PairPArgs A) {
  using namespace tc;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int S = A.stages;
  constexpr int KP = PAIRP_KPS;
  const uint32_t x_bytes = KP * PAIR_X_BYTES;               // [k-block][128 token rows][128 B]
  const uint32_t stage_bytes = x_bytes + KP * A.w_bytes;    // then [k-block][N/2 rows][128 B]
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + (size_t)S * stage_bytes);   // used in rank 0
  uint64_t* empty = full + S;
  uint64_t* acc_full = empty + S;    // [2], both CTAs (MMA commits are multicast)
  uint64_t* acc_empty = acc_full + 2;  // [2], rank 0 (arrivals from both CTAs' epilogue warps)
  uint32_t* tslot = reinterpret_cast<uint32_t*>(acc_empty + 2);
  volatile int* abort = reinterpret_cast<volatile int*>(tslot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();
  const int pair = blockIdx.x >> 1, P = gridDim.x >> 1;
  const int half = A.N >> 1;
  const int trow = (int)rank * 128;
  const int my_tiles = pair < A.tiles ? (A.tiles - 1 - pair) / P + 1 : 0;
  const int steps = A.n_kb / KP;          // ring stages per tile
  const int total = my_tiles * steps;     // ring iterations of this CTA
  pdl_trigger();

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&acc_full[b], 1);
      mbar_init(&acc_empty[b], 8);
    }
    *abort = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 1) tmem_alloc_pair(tslot, 512u);
  fence_before();
  cluster_sync_all();   // both CTAs' barriers are initialised before any cross-CTA arrival
  fence_after();
  const uint32_t tmem = *tslot;

  if (warp == 0) {
    // producer: the whole warp runs the loop, one elected lane issues; both CTAs' bytes of a
    // stage complete on rank 0's full barrier, which rank 0 arms for both
    if (lane == 0) {
      asm volatile("prefetch.tensormap [%0];" ::"l"(&tm_w) : "memory");
      asm volatile("prefetch.tensormap [%0];" ::"l"(&tm_x) : "memory");
    }
    __syncwarp();
    const int npre = min(total, S);
    for (int i = 0; i < npre; ++i) {   // weights of the first ring pass before the dependency wait
      const int tile = pair + (i / steps) * P, kb = (i % steps) * KP;
      if (rank == 0) mbar_expect_tx_warp(&full[i], 2 * stage_bytes);
      tma_load_3d_pair_warp(smem + i * stage_bytes + x_bytes, &tm_w, cluster_addr(smem_u32(&full[i]), 0),
                            tile * A.N + (int)rank * half, kb, true);
    }
    pdl_wait();   // activations are the previous kernel's output
    for (int i = 0; i < npre; ++i)
      tma_load_3d_pair_warp(smem + i * stage_bytes, &tm_x, cluster_addr(smem_u32(&full[i]), 0), trow,
                            (i % steps) * KP, false);
    bool ok = true;
    for (int i = npre; i < total; ++i) {
      const int s = i % S;
      const uint32_t ph = (i / S) & 1u;
      ok = mbar_wait_warp(&empty[s], ph ^ 1u, 611, &g_gemm_pair_error, abort);
      if (!ok) break;
      const int tile = pair + (i / steps) * P, kb = (i % steps) * KP;
      const uint32_t fb = cluster_addr(smem_u32(&full[s]), 0);
      uint8_t* st = smem + s * stage_bytes;
      if (rank == 0) mbar_expect_tx_warp(&full[s], 2 * stage_bytes);
      tma_load_3d_pair_warp(st + x_bytes, &tm_w, fb, tile * A.N + (int)rank * half, kb, true);
      tma_load_3d_pair_warp(st, &tm_x, fb, trow, kb, false);
    }
    // the last release of every stage (an MMA-completion arrival from rank 0) has landed
    for (int s = 0; ok && s < npre; ++s) {
      const int last = (total - 1 - s) / S;
      ok = mbar_wait_warp(&empty[s], (uint32_t)last & 1u, 612, &g_gemm_pair_error, abort);
    }
  } else if (warp == 1) {
    pdl_wait();
    if (rank == 0) {   // MMA issuer: the whole warp, one elected lane issues
      const uint32_t idesc = idesc_bf16(256, A.N);
      bool ok = true;
      int i = 0;
      for (int ti = 0; ti < my_tiles; ++ti) {
        const uint32_t b = ti & 1, use = ti >> 1;
        if (ok && use >= 1) ok = mbar_wait_warp(&acc_empty[b], (use - 1) & 1u, 613, &g_gemm_pair_error, abort);
        fence_after();
        for (int j = 0; j < steps; ++j, ++i) {
          const int s = i % S;
          const uint32_t ph = (i / S) & 1u;
          if (ok) ok = mbar_wait_warp(&full[s], ph, 614, &g_gemm_pair_error, abort);
          fence_after();
          if (ok) {
            const uint32_t xa = smem_u32(smem + s * stage_bytes);
#pragma unroll
            for (int kk = 0; kk < KP; ++kk)
              umma4_bf16_pair_warp(tmem + b * 256, sdesc_sw128(xa + kk * PAIR_X_BYTES),
                                   sdesc_sw128(xa + x_bytes + kk * A.w_bytes), idesc, (j > 0 || kk > 0) ? 1u : 0u);
          }
          umma_commit_pair_warp(&empty[s]);
        }
        umma_commit_pair_warp(&acc_full[b]);
      }
    }
  } else {
    // ------------------------------------------------------------------ epilogue
    pdl_wait();
    const int quad = warp & 3;
    const int t = trow + quad * 32 + lane;
    const uint32_t release = cluster_addr(smem_u32(&acc_empty[0]), 0);
    for (int ti = 0; ti < my_tiles; ++ti) {
      const uint32_t b = ti & 1;
      const bool ok = mbar_wait(&acc_full[b], (ti >> 1) & 1u, 615, &g_gemm_pair_error, abort);
      fence_after();
      const int n0 = (pair + ti * P) * A.N;
      const uint32_t tbase = tmem + b * 256 + ((uint32_t)(quad * 32) << 16);
      __nv_bfloat16* crow = A.c + (int64_t)t * A.ldc;
      for (int c0 = 0; c0 < A.N; c0 += 16) {
        float v[16];
        tmem_ld16(tbase + c0, v);
        if (!ok || t >= A.m) continue;
        const int col = n0 + c0;
        if (col + 16 <= A.n) {
          uint4 ov[2];
          __nv_bfloat16* oh = reinterpret_cast<__nv_bfloat16*>(ov);
#pragma unroll
          for (int e = 0; e < 16; ++e) oh[e] = __float2bfloat16_rn(v[e]);
          reinterpret_cast<uint4*>(crow + col)[0] = ov[0];
          reinterpret_cast<uint4*>(crow + col)[1] = ov[1];
        } else {
#pragma unroll
          for (int e = 0; e < 16; ++e)
            if (col + e < A.n) crow[col + e] = __float2bfloat16_rn(v[e]);
        }
      }
      fence_before();
      __syncwarp();
      if (lane == 0)
        asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(release + b * 8u)
                     : "memory");
    }
  }
  fence_before();
  __syncthreads();
  cluster_sync_all();   // the partner's arrivals have landed; it is done with this CTA's memory
  if (warp == 1) {
    fence_after();
    tmem_dealloc_pair(tmem, 512u);
  }
}

// Tile width of the persistent pair kernel: the multiple of 16 in [128, 256] that minimises
// the per-CTA ingest (rounds of tiles × the bytes of one k-block: 16 KB of activations + N/2
// weight rows), ties to the wider tile. Returns false when one round covers the output (the
// one-shot kernel's case) or the shape does not fit.
static bool pairp_plan(int64_t m, int64_t n, int64_t k, int pairs, int* N_out, int* tiles_out) {
  if (m <= 128 || m > 256 || pairs <= 0 || n <= 256 * (int64_t)pairs) return false;
  double best = 1e300;
  for (int N = 256; N >= 128; N -= 16) {
    const int64_t tiles = (n + N - 1) / N;
    const int64_t rounds = (tiles + pairs - 1) / pairs;
    const double cost = (double)rounds * (PAIR_X_BYTES + (N / 2) * 128);
    if (cost < best) {
      best = cost;
      *N_out = N;
      *tiles_out = (int)tiles;
    }
  }
  (void)k;
  return true;
}

// c[m, n] = a · wᵀ through the persistent pair kernel; QSP_ERR_UNSUPPORTED when the shape or
// alignment does not fit (the caller then takes another kernel).
int gemm_pair_persistent(const void* a, int64_t lda, const void* w, int64_t ldw, void* c, int64_t ldc, int64_t m,
                         int64_t n, int64_t k, cudaStream_t st) {
  if (!aligned(a, 16) || !aligned(w, 16) || !aligned(c, 16) || (lda * 2) % 16 != 0 || (ldw * 2) % 16 != 0 ||
      (ldc * 2) % 16 != 0 || k % 8 != 0)
    return QSP_ERR_UNSUPPORTED;
  const int pairs = resident_pairs();
  int N = 0, tiles = 0;
  if (k % (64 * PAIRP_KPS) != 0 || !pairp_plan(m, n, k, pairs, &N, &tiles)) return QSP_ERR_UNSUPPORTED;
  PairPArgs args{};
  args.c = static_cast<__nv_bfloat16*>(c);
  args.ldc = ldc;
  args.m = (int)m;
  args.n = (int)n;
  args.N = N;
  args.tiles = tiles;
  args.n_kb = ceil_div(k, 64);
  args.w_bytes = (N / 2) * 128;
  const int stage = PAIRP_KPS * (PAIR_X_BYTES + args.w_bytes);
  args.stages = std::min(PAIR_MAX_STAGES, (PAIR_SMEM_MAX - PAIR_AUX) / stage);
  if (args.stages < 2) return QSP_ERR_UNSUPPORTED;
  CUtensorMap mw, mx;
  if (!make_map3_bf16(&mw, w, n, k, ldw, N / 2, PAIRP_KPS) || !make_map3_bf16(&mx, a, m, k, lda, 128, PAIRP_KPS))
    return QSP_ERR_UNSUPPORTED;
  auto kern = gemm_pairp_kernel;
  const size_t smem = (size_t)args.stages * stage + PAIR_AUX;
  static bool attr_set = false;
  if (!attr_set) {
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, PAIR_SMEM_MAX) != cudaSuccess)
      return set_error(QSP_ERR_CUDA, "qsp_gemm(pair, persistent): cannot reserve %d bytes of shared memory",
                       PAIR_SMEM_MAX);
    attr_set = true;
  }
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(2 * std::min(pairs, tiles));
  cfg.blockDim = dim3(192);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute at[2];
  at[0].id = cudaLaunchAttributeClusterDimension;
  at[0].val.clusterDim.x = 2;
  at[0].val.clusterDim.y = 1;
  at[0].val.clusterDim.z = 1;
  at[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  at[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = at;
  cfg.numAttrs = 2;
  const cudaError_t e = cudaLaunchKernelEx(&cfg, kern, mw, mx, args);
  if (e != cudaSuccess) {
    (void)cudaGetLastError();
    return set_error(QSP_ERR_CUDA, "qsp_gemm(pair, persistent): %s", cudaGetErrorString(e));
  }
  return check_launch("qsp_gemm(pair, persistent)");
}

}  // namespace qsp
