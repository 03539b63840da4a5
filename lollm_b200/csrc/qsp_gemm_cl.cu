// Cluster split-K GEMM for the verify step's projections (M = batch·(k+1) ≤ 256 token rows):
// c[m, n] = a[m, k] · w[n, k]ᵀ with fp32 accumulation, bf16 in and out.
//
// One output tile (NACC·128 weight rows × all 256 token rows) is computed by a thread-block
// cluster of S CTAs, CTA rank r taking k-blocks [r·kps, (r+1)·kps). Each CTA streams its
// weight and activation tiles through a TMA ring into tcgen05.mma (accumulators in TMEM), as
// the persistent GEMM does. Instead of writing fp32 partials to global memory and merging
// them in a second kernel, the S CTAs exchange them through distributed shared memory: the
// token rows are cut into S owner slices (32-row granularity); every CTA sends each slice it
// does not own to the owner's shared memory, and the owner sums the S partials in split order
// (rank 0 first: the same order the global merge used, so results do not depend on timing)
// and applies the epilogue:
//   STORE   c = round(Σ)
//   ADD     c = round(c + round(Σ))          (residual add into the stream)
//   SWIGLU  act[:, j] = round(round(silu(round(Σ_gate))) · round(Σ_up)) with the tile's
//           accumulator 0 on gate rows [128t, 128t+128) and accumulator 1 on the matching up
//           rows [inter + 128t, ...) of a [gate; up] weight
// The exchange lands in the ring buffers, which are idle once every CTA of the cluster has
// finished its main loop. Cluster-wide waits use mbarriers with remote arrivals and bounded
// polling (an expired wait records an error code and lets the CTA finish); the only unbounded
// wait is the hardware cluster barrier at the start, which every CTA reaches immediately.
#include "qsp_common.cuh"
#include "qsp_tc.cuh"

namespace qsp {

__device__ int g_gemm_cl_error = 0;

int gemm_cl_device_error(int reset) {
  int v = 0;
  if (cudaMemcpyFromSymbol(&v, g_gemm_cl_error, sizeof(int)) != cudaSuccess) return 0;
  if (reset && v) {
    const int zero = 0;
    cudaMemcpyToSymbol(g_gemm_cl_error, &zero, sizeof(int));
  }
  return v;
}

enum { CL_STORE = 0, CL_ADD = 1, CL_SWIGLU = 2 };
constexpr int CL_MT = 256;        // token rows per tile (the MMA N dimension)
constexpr int CL_MAX_S = 8;

template <int NACC>
struct ClCfg {
  static constexpr int W_BYTES = NACC * 128 * 64 * 2;    // NACC boxes of 128 weight rows x 64 K
  static constexpr int X_BYTES = CL_MT * 64 * 2;         // 256 token rows x 64 K
  static constexpr int STAGE = W_BYTES + X_BYTES;
  static constexpr int STAGES = (196 * 1024) / STAGE;    // 4 (NACC 1) or 3 (NACC 2)
  static constexpr uint32_t TMEM_COLS = NACC * CL_MT;
  static constexpr size_t RING = (size_t)STAGES * STAGE;
  // the largest exchange buffer a plan may use ((S-1) slices of ≤ MAX_SLICE rows)
  static constexpr size_t MAX_XCHG = 224 * 1024;
  static constexpr size_t BUF = RING > MAX_XCHG ? RING : MAX_XCHG;
  static constexpr size_t SMEM = BUF + 1024 + 256;
};

struct ClArgs {
  __nv_bfloat16* c;
  int64_t ldc;
  int m, n_rows;      // token rows; valid weight rows (STORE/ADD: n; SWIGLU: inter)
  int n_kb, kps, S, mode;
  int box1;           // weight-row offset of accumulator 1's box (128, or inter for SWIGLU)
};

// Owner slices of the 256 token rows in 32-row chunks, as even as possible: slice r starts at
// chunk r·(8/S) + min(r, 8 % S).
__host__ __device__ __forceinline__ int slice_begin(int r, int S) {
  constexpr int chunks = CL_MT / 32;
  return 32 * (r * (chunks / S) + (r < chunks % S ? r : chunks % S));
}

__device__ __forceinline__ uint32_t cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
__device__ __forceinline__ uint32_t map_rank(uint32_t saddr, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(saddr), "r"(rank));
  return r;
}
__device__ __forceinline__ void st_cluster_f32(uint32_t addr, float v) {
  asm volatile("st.shared::cluster.f32 [%0], %1;" ::"r"(addr), "f"(v) : "memory");
}
__device__ __forceinline__ void arrive_remote(uint32_t cluster_addr) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr) : "memory");
}
__device__ __forceinline__ bool try_wait_cluster(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(tc::smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}
__device__ __forceinline__ bool wait_cluster(uint64_t* bar, int code) {
  for (uint32_t i = 0; i < tc::WAIT_LIMIT; ++i) {
    if (try_wait_cluster(bar, 0)) return true;
    if (i > 256) __nanosleep(64);
  }
  atomicExch(&g_gemm_cl_error, code);
  return false;
}

template <int NACC, int MODE>
__global__ void __launch_bounds__(192, 1)
gemm_cl_kernel(const __grid_constant__ CUtensorMap tm_w, const __grid_constant__ CUtensorMap tm_x, const ClArgs A) {
  using C = ClCfg<NACC>;
  using namespace tc;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + C::BUF);
  uint64_t* empty = full + C::STAGES;
  uint64_t* acc_full = empty + C::STAGES;
  uint64_t* cl_ready = acc_full + 1;   // every CTA of the cluster finished its main loop
  uint64_t* cl_done = cl_ready + 1;    // every CTA finished writing its partials to the owners
  uint32_t* tslot = reinterpret_cast<uint32_t*>(cl_done + 1);
  volatile int* abort = reinterpret_cast<volatile int*>(tslot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int S = A.S;
  const uint32_t me = cluster_rank();
  const int tile = blockIdx.x / S;
  const int kb0 = (int)me * A.kps, nk = min(A.n_kb, kb0 + A.kps) - kb0;
  pdl_trigger();

  if (threadIdx.x == 0) {
    for (int s = 0; s < C::STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(acc_full, 1);
    mbar_init(cl_ready, S);
    mbar_init(cl_done, S);
    *abort = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 1) tmem_alloc(tslot, C::TMEM_COLS);
  fence_before();
  // every CTA's barriers are initialised before any remote arrival
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
  fence_after();
  const uint32_t tmem = *tslot;
  const int row0 = tile * (NACC == 2 && MODE != CL_SWIGLU ? 256 : 128);

  if (warp == 0) {
    // producer: the whole warp runs the loop, one elected lane issues (qsp_tc.cuh)
    if (lane == 0) {
      asm volatile("prefetch.tensormap [%0];" ::"l"(&tm_w) : "memory");
      asm volatile("prefetch.tensormap [%0];" ::"l"(&tm_x) : "memory");
    }
    __syncwarp();
    // weights of the first ring pass before the dependency wait, activations after it
    // NACC = 2 outside SWIGLU: the two accumulators' 256 weight rows are contiguous and come as
    // one 256-row box (fewer, larger TMA requests); SWIGLU's gate and up rows are two boxes
    constexpr bool ONE_BOX = NACC == 1 || MODE != CL_SWIGLU;
    const int npre = min(nk, C::STAGES);
    for (int i = 0; i < npre; ++i) {
      uint8_t* st = smem + i * C::STAGE;
      mbar_expect_tx_warp(&full[i], C::STAGE);
      tma_load_2d_evict_first_warp(st, &tm_w, &full[i], (kb0 + i) * 64, row0);
      if (!ONE_BOX) tma_load_2d_evict_first_warp(st + 128 * 128, &tm_w, &full[i], (kb0 + i) * 64, row0 + A.box1);
    }
    pdl_wait();
    for (int i = 0; i < npre; ++i) tma_load_2d_warp(smem + i * C::STAGE + C::W_BYTES, &tm_x, &full[i], (kb0 + i) * 64, 0);
    for (int i = npre; i < nk; ++i) {
      const int s = i % C::STAGES;
      const uint32_t ph = (i / C::STAGES) & 1u;
      if (!mbar_wait_warp(&empty[s], ph ^ 1u, 301, &g_gemm_cl_error, abort)) break;
      uint8_t* st = smem + s * C::STAGE;
      mbar_expect_tx_warp(&full[s], C::STAGE);
      tma_load_2d_evict_first_warp(st, &tm_w, &full[s], (kb0 + i) * 64, row0);
      if (!ONE_BOX) tma_load_2d_evict_first_warp(st + 128 * 128, &tm_w, &full[s], (kb0 + i) * 64, row0 + A.box1);
      tma_load_2d_warp(st + C::W_BYTES, &tm_x, &full[s], (kb0 + i) * 64, 0);
    }
  } else if (warp == 1) {
    pdl_wait();
    // MMA issuer: the whole warp runs the loop, one elected lane issues
    constexpr uint32_t idesc = idesc_bf16(128, CL_MT);
    bool ok = true;
    for (int i = 0; i < nk; ++i) {
      const int s = i % C::STAGES;
      const uint32_t ph = (i / C::STAGES) & 1u;
      if (ok && !mbar_wait_warp(&full[s], ph, 302, &g_gemm_cl_error, abort)) ok = false;
      fence_after();
      if (ok) {
        const uint32_t a0 = smem_u32(smem + s * C::STAGE);
        const uint32_t b0 = a0 + C::W_BYTES;
#pragma unroll
        for (int q = 0; q < NACC; ++q)
          umma4_bf16_warp(tmem + q * CL_MT, sdesc_sw128(a0 + q * 128 * 128), sdesc_sw128(b0), idesc, i > 0 ? 1u : 0u);
      }
      umma_commit_warp(&empty[s]);
    }
    umma_commit_warp(acc_full);
  } else {
    // ---------------------------------------------------------------- exchange + epilogue
    pdl_wait();
    const int quad = warp & 3;
    const int et = threadIdx.x - 64;               // 0..127
    const bool ok = mbar_wait(acc_full, 0, 303, &g_gemm_cl_error, abort);
    fence_after();
    // phase A: this CTA's ring is idle; tell every CTA of the cluster
    if (et == 0)
      for (int r = 0; r < S; ++r) arrive_remote(map_rank(smem_u32(cl_ready), (uint32_t)r));
    const bool ready = wait_cluster(cl_ready, 304);
    const uint32_t lrow = quad * 32 + lane;        // TMEM lane = weight row within an accumulator
    // exchange buffer of the owner: slots for the S-1 other ranks, each [slice rows][NACC][128] fp32
    const int slot_rows = slice_begin(1, S) - slice_begin(0, S);   // slice 0 is the largest
    const uint32_t slot_bytes = (uint32_t)slot_rows * NACC * 128 * 4;
    const uint32_t buf = smem_u32(smem);
    for (int o = 0; o < S; ++o) {
      if (o == (int)me) continue;
      const int t0 = slice_begin(o, S), t1 = slice_begin(o + 1, S);
      const uint32_t slot = (uint32_t)((int)me < o ? me : me - 1);
      const uint32_t rbase = map_rank(buf + slot * slot_bytes, (uint32_t)o);
      for (int c0 = t0; c0 < t1; c0 += 32) {
#pragma unroll
        for (int q = 0; q < NACC; ++q) {
          float v[32];
          tmem_ld32(tmem + q * CL_MT + c0 + ((uint32_t)(quad * 32) << 16), v);
          if (ok && ready) {
#pragma unroll
            for (int j = 0; j < 32; ++j)
              st_cluster_f32(rbase + (((uint32_t)(c0 - t0 + j) * NACC + q) * 128 + lrow) * 4, v[j]);
          }
        }
      }
    }
    // phase B: partials delivered (named barrier over the 128 epilogue threads, then release)
    asm volatile("bar.sync 1, 128;" ::: "memory");
    if (et == 0) {
      asm volatile("fence.acq_rel.cluster;" ::: "memory");
      for (int r = 0; r < S; ++r) arrive_remote(map_rank(smem_u32(cl_done), (uint32_t)r));
    }
    const bool done = wait_cluster(cl_done, 305);
    // reduce this CTA's slice in split order, stage 32 token rows of bf16 results in shared
    // memory, then write them out as whole rows with 16-byte stores (the residual add of ADD
    // is applied in that pass)
    const int t0 = slice_begin(me, S), t1 = slice_begin(me + 1, S);
    const int out_cols = MODE == CL_SWIGLU ? 128 : NACC * 128;
    const int col0 = MODE == CL_SWIGLU ? tile * 128 : row0;
    const float* xb = reinterpret_cast<const float*>(smem);
    __nv_bfloat16* stg = reinterpret_cast<__nv_bfloat16*>(smem + (size_t)(S - 1) * slot_bytes);
    const bool live = ok && ready && done;
    for (int c0 = t0; c0 < t1; c0 += 32) {
      // Σ over the S splits in rank order; the split loop stays rolled and its body (one
      // add per value) small, so the loop runs from the instruction cache
      float v[NACC][32], acc[NACC][32];
#pragma unroll
      for (int q = 0; q < NACC; ++q) {
        tmem_ld32(tmem + q * CL_MT + c0 + ((uint32_t)(quad * 32) << 16), v[q]);
#pragma unroll
        for (int j = 0; j < 32; ++j) acc[q][j] = 0.f;
      }
#pragma unroll 1
      for (int r = 0; r < S; ++r) {
        if (r == (int)me) {
#pragma unroll
          for (int q = 0; q < NACC; ++q)
#pragma unroll
            for (int j = 0; j < 32; ++j) acc[q][j] += v[q][j];
        } else {
          const int slot = r < (int)me ? r : r - 1;
          const float* src = xb + (size_t)slot * (slot_bytes / 4) + (size_t)(c0 - t0) * NACC * 128 + lrow;
#pragma unroll
          for (int j = 0; j < 32; ++j)
#pragma unroll
            for (int q = 0; q < NACC; ++q) acc[q][j] += src[(j * NACC + q) * 128];
        }
      }
      if (MODE == CL_SWIGLU) {
#pragma unroll
        for (int j = 0; j < 32; ++j) {
          const float g = dt<__nv_bfloat16>::round(siluf_(dt<__nv_bfloat16>::round(acc[0][j])));
          stg[j * out_cols + lrow] = __float2bfloat16_rn(g * dt<__nv_bfloat16>::round(acc[NACC - 1][j]));
        }
      } else {
#pragma unroll
        for (int q = 0; q < NACC; ++q)
#pragma unroll
          for (int j = 0; j < 32; ++j) stg[j * out_cols + q * 128 + lrow] = __float2bfloat16_rn(acc[q][j]);
      }
      asm volatile("bar.sync 1, 128;" ::: "memory");
      const int vpr = out_cols / 8;   // 16-byte vectors per staged row
      for (int idx = et; idx < 32 * vpr; idx += 128) {
        const int j = idx / vpr, cv = idx - j * vpr;
        const int tok = c0 + j, col = col0 + cv * 8;
        if (!live || tok >= A.m || col >= A.n_rows) continue;
        const uint4 sv = *reinterpret_cast<const uint4*>(stg + j * out_cols + cv * 8);
        __nv_bfloat16* dst = A.c + (int64_t)tok * A.ldc + col;
        if (col + 8 <= A.n_rows) {
          if (MODE == CL_ADD) {
            const uint4 xv = *reinterpret_cast<const uint4*>(dst);
            const __nv_bfloat16* sh = reinterpret_cast<const __nv_bfloat16*>(&sv);
            const __nv_bfloat16* xh = reinterpret_cast<const __nv_bfloat16*>(&xv);
            uint4 ov;
            __nv_bfloat16* oh = reinterpret_cast<__nv_bfloat16*>(&ov);
#pragma unroll
            for (int e = 0; e < 8; ++e) oh[e] = __float2bfloat16_rn(__bfloat162float(sh[e]) + __bfloat162float(xh[e]));
            *reinterpret_cast<uint4*>(dst) = ov;
          } else {
            *reinterpret_cast<uint4*>(dst) = sv;
          }
        } else {
          const __nv_bfloat16* sh = reinterpret_cast<const __nv_bfloat16*>(&sv);
          for (int e = 0; e < 8 && col + e < A.n_rows; ++e) {
            float r = __bfloat162float(sh[e]);
            if (MODE == CL_ADD) r += __bfloat162float(dst[e]);
            dst[e] = __float2bfloat16_rn(r);
          }
        }
      }
      asm volatile("bar.sync 1, 128;" ::: "memory");
    }
  }
  fence_before();
  __syncthreads();
  if (warp == 1) {
    fence_after();
    tc::tmem_dealloc(tmem, C::TMEM_COLS);
  }
}

// ------------------------------------------------------------------ host side
struct ClPlan {
  int nacc, S, tiles, kps, n_kb;
};

template <int NACC>
static int max_clusters(int S) {
  static int cache[CL_MAX_S + 1] = {0};
  if (cache[S] != 0) return cache[S];
  using C = ClCfg<NACC>;
  auto kern = gemm_cl_kernel<NACC, CL_STORE>;   // every mode has the same resources
  if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)C::SMEM) != cudaSuccess) {
    (void)cudaGetLastError();
    return cache[S] = -1;
  }
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(S * 64);
  cfg.blockDim = dim3(192);
  cfg.dynamicSmemBytes = C::SMEM;
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeClusterDimension;
  at[0].val.clusterDim.x = S;
  at[0].val.clusterDim.y = 1;
  at[0].val.clusterDim.z = 1;
  cfg.attrs = at;
  cfg.numAttrs = 1;
  int n = 0;
  if (cudaOccupancyMaxActiveClusters(&n, kern, &cfg) != cudaSuccess) {
    (void)cudaGetLastError();
    n = -1;
  }
  return cache[S] = (n > 0 ? n : -1);
}

static int clusters_for(int nacc, int S) { return nacc == 2 ? max_clusters<2>(S) : max_clusters<1>(S); }


// Picks (accumulators, cluster size) for one tile per cluster, all clusters co-resident.
// Estimated µs: ~3 of fixed cost, the CTA's ring ingest at ~80 GB/s, and the exchange
// ((S-1)/S of the tile's fp32 partials) at ~100 GB/s. Returns false when nothing fits.
static bool cl_plan(int64_t m, int64_t rows, int64_t k, int mode, ClPlan* out) {
  if (m <= 128 || m > CL_MT) return false;
  const int n_kb = (int)((k + 63) / 64);
  double best = 1e30;
  bool found = false;
  for (int nacc = 1; nacc <= 2; ++nacc) {
    if (mode == CL_SWIGLU && nacc != 2) continue;
    const int tiles = (int)((rows + (mode == CL_SWIGLU ? 128 : 128 * nacc) - 1) / (mode == CL_SWIGLU ? 128 : 128 * nacc));
    for (int S = 1; S <= CL_MAX_S; ++S) {
      const int kps = (n_kb + S - 1) / S;
      if ((n_kb + kps - 1) / kps != S) continue;   // every rank gets k-blocks
      const int slice_max = slice_begin(1, S) - slice_begin(0, S);
      const size_t out_cols = mode == CL_SWIGLU ? 128 : (size_t)nacc * 128;
      const size_t need = (size_t)(S - 1) * slice_max * nacc * 128 * 4 + 32 * out_cols * 2;   // exchange + staging
      if (need > (nacc == 2 ? ClCfg<2>::BUF : ClCfg<1>::BUF)) continue;
      if (tiles * S > tc::sm_count()) continue;
      const int mc = clusters_for(nacc, S);
      if (mc <= 0 || tiles > mc) continue;
      const double t = 3.0 + (double)kps * (nacc * 128 + CL_MT) * 128 / 80e3 +
                       (S > 1 ? (double)(S - 1) / S * nacc * 128 * CL_MT * 4 / 100e3 : 0.0);
      if (t < best) {
        best = t;
        found = true;
        out->nacc = nacc;
        out->S = S;
        out->tiles = tiles;
        out->kps = kps;
        out->n_kb = n_kb;
      }
    }
  }
  return found;
}

template <int NACC, int MODE>
static int launch_cl(const void* a, int64_t lda, const void* w, int64_t ldw, int64_t w_rows, int64_t k, const ClPlan& p,
                     ClArgs args, cudaStream_t st) {
  using C = ClCfg<NACC>;
  CUtensorMap mw, mx;
  const int w_box = (NACC == 2 && MODE != CL_SWIGLU) ? 256 : 128;
  if (!tc::make_map_bf16(&mw, w, w_rows, k, ldw, w_box) || !tc::make_map_bf16(&mx, a, args.m, k, lda, CL_MT))
    return QSP_ERR_UNSUPPORTED;
  auto kern = gemm_cl_kernel<NACC, MODE>;
  static bool attr_set = false;
  if (!attr_set) {
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)C::SMEM) != cudaSuccess)
      return set_error(QSP_ERR_CUDA, "qsp_gemm(cluster): cannot reserve %zu bytes of shared memory", C::SMEM);
    attr_set = true;
  }
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(p.tiles * p.S);
  cfg.blockDim = dim3(192);
  cfg.dynamicSmemBytes = C::SMEM;
  cfg.stream = st;
  cudaLaunchAttribute at[2];
  at[0].id = cudaLaunchAttributeClusterDimension;
  at[0].val.clusterDim.x = p.S;
  at[0].val.clusterDim.y = 1;
  at[0].val.clusterDim.z = 1;
  at[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  at[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = at;
  cfg.numAttrs = 2;
  const cudaError_t e = cudaLaunchKernelEx(&cfg, kern, mw, mx, args);
  if (e != cudaSuccess) {
    (void)cudaGetLastError();
    return set_error(QSP_ERR_CUDA, "qsp_gemm(cluster): %s", cudaGetErrorString(e));
  }
  return check_launch("qsp_gemm(cluster)");
}

// Cluster split-K path for 128 < m ≤ 256 token rows. mode: CL_STORE / CL_ADD over `n` output
// columns, or CL_SWIGLU over `n = inter` activation columns of a [gate; up] weight with
// 2·inter rows. Returns QSP_ERR_UNSUPPORTED when no plan applies (the caller then uses the
// persistent split-K kernel).
int gemm_cl(const void* a, int64_t lda, const void* w, int64_t ldw, void* c, int64_t ldc, int64_t m, int64_t n,
            int64_t k, int mode, cudaStream_t st) {
  if (!aligned(a, 16) || !aligned(w, 16) || !aligned(c, 16) || (lda * 2) % 16 != 0 || (ldw * 2) % 16 != 0 ||
      (ldc * 2) % 16 != 0 || k % 8 != 0)
    return QSP_ERR_UNSUPPORTED;
  ClPlan p{};
  if (!cl_plan(m, n, k, mode, &p)) return QSP_ERR_UNSUPPORTED;
  ClArgs args{};
  args.c = static_cast<__nv_bfloat16*>(c);
  args.ldc = ldc;
  args.m = (int)m;
  args.n_rows = (int)n;
  args.n_kb = p.n_kb;
  args.kps = p.kps;
  args.S = p.S;
  args.mode = mode;
  args.box1 = mode == CL_SWIGLU ? (int)n : 128;
  const int64_t w_rows = mode == CL_SWIGLU ? 2 * n : n;
  if (mode == CL_SWIGLU) return launch_cl<2, CL_SWIGLU>(a, lda, w, ldw, w_rows, k, p, args, st);
  if (mode == CL_ADD)
    return p.nacc == 2 ? launch_cl<2, CL_ADD>(a, lda, w, ldw, w_rows, k, p, args, st)
                       : launch_cl<1, CL_ADD>(a, lda, w, ldw, w_rows, k, p, args, st);
  return p.nacc == 2 ? launch_cl<2, CL_STORE>(a, lda, w, ldw, w_rows, k, p, args, st)
                     : launch_cl<1, CL_STORE>(a, lda, w, ldw, w_rows, k, p, args, st);
}

}  // namespace qsp
